// store_kvcache: slot-mapped scatter of new K/V rows into the paged pools.
//
// Replaces the reference's per-sequence Python write loops
// (femtovllm/models/qwen/qwen3.py:240-264 decode, 322-366 prefill), which issue
// 2 copy launches per sequence (decode) or per block run (prefill) per layer.
// Here one launch moves every (token, kv head) row of K and V: each row is
// head_dim contiguous elements on both sides (the pool is head-major inside a
// page, [blocks][Hkv][16][D]), so a row is a run of 16-byte vectors that a
// group of lanes copies with one coalesced load and one coalesced store each.
// HBM-bound: 2 * T * Hkv * D * sizeof(T) bytes read and written, plus 8 T
// bytes of slot_mapping.
//
// Two kernels: store_kvcache_bulk_kernel (16-byte-aligned rows, the usual
// case) moves whole rows with the TMA engine's bulk copies, global -> shared ->
// global, and store_kvcache_kernel (any alignment) moves them as vectors
// through registers.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fvb {

// VEC_BYTES = 16 on the aligned path, sizeof(elem) otherwise.
//
// Work split: a token has R = 2 * n_kv_heads rows (K rows, then V rows) of
// L = row_bytes / VEC_BYTES lanes.  Thread tid of a block owns lane tid % L of
// row slot tid / L for the whole launch: with R * L <= threads a block pass
// covers threads / (R * L) whole tokens, otherwise one token with each thread
// taking rows slot, slot + threads / L, ...  Tokens advance by a block-uniform
// stride, two per step so two loads are in flight; no division in the loop
// (a power-of-two page size splits the slot with a shift; 2.9 % faster than a
// 64-bit division per row at 65k tokens).
template <int VEC_BYTES>
__global__ void __launch_bounds__(256) store_kvcache_kernel(const uint8_t* __restrict__ k,
                                                            const uint8_t* __restrict__ v,
                                                            int64_t token_stride_b, int64_t head_stride_b,
                                                            uint8_t* __restrict__ k_pool,
                                                            uint8_t* __restrict__ v_pool, int64_t num_slots,
                                                            const int64_t* __restrict__ slot_mapping,
                                                            int64_t num_tokens, int n_kv_heads, int row_bytes,
                                                            int block_size, int block_shift,
                                                            int* __restrict__ err) {
  using Vec = typename std::conditional<
      VEC_BYTES == 16, uint4,
      typename std::conditional<VEC_BYTES == 8, uint2,
                                typename std::conditional<VEC_BYTES == 4, uint32_t, uint16_t>::type>::type>::type;
  const int L = row_bytes / VEC_BYTES;            // vectors per row
  const int Lb = min(L, int(blockDim.x));          // lanes per row slot (rows wider than a block loop)
  const int R = 2 * n_kv_heads;                    // rows per token
  const int slots_pb = int(blockDim.x) / Lb;       // row slots per block
  const int tid = int(threadIdx.x);
  const int lane = tid % Lb, slot_id = tid / Lb;
  if (slot_id >= slots_pb) return;  // the block's last partial row group (L does not divide blockDim.x)
  const bool packed = R <= slots_pb;
  const int tpb = packed ? slots_pb / R : 1;  // tokens per block pass
  if (packed && slot_id >= tpb * R) return;  // spare row slots
  const int tok_off = packed ? slot_id / R : 0;
  const int row0 = packed ? slot_id % R : slot_id;
  const int row_step = packed ? R : slots_pb;
  const int64_t tstride = int64_t(gridDim.x) * tpb;
  auto src_of = [&](int64_t t, int row, int ln) -> const Vec* {
    const int h = row < n_kv_heads ? row : row - n_kv_heads;
    return reinterpret_cast<const Vec*>((row < n_kv_heads ? k : v) + t * token_stride_b + h * head_stride_b +
                                        int64_t(ln) * VEC_BYTES);
  };
  auto dst_of = [&](int64_t slot, int row, int ln) -> Vec* {
    const int h = row < n_kv_heads ? row : row - n_kv_heads;
    const int64_t blk = block_shift >= 0 ? (slot >> block_shift) : slot / block_size;
    const int off = int(slot - blk * block_size);
    return reinterpret_cast<Vec*>((row < n_kv_heads ? k_pool : v_pool) +
                                  ((blk * n_kv_heads + h) * block_size + off) * int64_t(row_bytes) +
                                  int64_t(ln) * VEC_BYTES);
  };
  for (int64_t t = int64_t(blockIdx.x) * tpb + tok_off; t < num_tokens; t += 2 * tstride) {
    const int64_t t2 = t + tstride;
    const bool has2 = t2 < num_tokens;
    int64_t s1 = __ldg(slot_mapping + t);
    int64_t s2 = has2 ? __ldg(slot_mapping + t2) : -1;
    if (s1 >= num_slots) {
      if (row0 == 0 && lane == 0) record_error(err, FVB_ERR_BAD_SLOT, int(t));
      s1 = -1;
    }
    if (s2 >= num_slots) {
      if (row0 == 0 && lane == 0) record_error(err, FVB_ERR_BAD_SLOT, int(t2));
      s2 = -1;
    }
    for (int row = row0; row < R; row += row_step) {
      for (int ln = lane; ln < L; ln += Lb) {
        const Vec a = *src_of(t, row, ln);
        Vec b{};
        if (has2) b = *src_of(t2, row, ln);
        if (s1 >= 0) *dst_of(s1, row, ln) = a;  // -1: padding token, skipped
        if (s2 >= 0) *dst_of(s2, row, ln) = b;
      }
    }
  }
}

// Bulk-copy path.  A CTA takes chunks of `tok` tokens (grid-stride): thread 0
// loads each token's K rows and V rows (n_kv_heads rows each, one bulk copy per
// token and tensor when a token's heads are contiguous, one per row otherwise)
// into one of two shared-memory stages, completing on that stage's mbarrier;
// then every thread stores rows of the chunk (K rows, then V rows, per token)
// to their pool slots with one bulk store each (cp.async.bulk global <- shared,
// one bulk group per thread and chunk).  The next chunk's loads go to the other
// stage as soon as this thread's stores of the chunk before it have been read
// out of shared memory, so a chunk's loads overlap the previous chunk's stores.
// Measured at 65,536 tokens of (8 heads x 128 dims, bf16) with random slots:
// 5.79 TB/s against 4.94 TB/s for the vector kernel (chunks of 4 tokens, 64
// threads, 4 CTAs per SM; 2, 8 and 16 tokens or 3, 5, 6 and 8 CTAs per SM were
// slower).
constexpr int kBulkThreads = 64;
constexpr int kBulkCtasPerSm = 4;
constexpr int kBulkStageBytes = 16 * 1024;  // tokens per chunk = this / (bytes of a token's rows), at most 4
constexpr int64_t kBulkMinTokens = 4096;

__device__ __forceinline__ void bulk_s2g(void* dst_gmem, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem), "r"(src_smem),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk stores have all finished reading shared memory.
__device__ __forceinline__ void bulk_wait_reads() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's bulk stores have all completed.
__device__ __forceinline__ void bulk_wait_done() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kBulkThreads) store_kvcache_bulk_kernel(
    const uint8_t* __restrict__ k, const uint8_t* __restrict__ v, int64_t token_stride_b, int64_t head_stride_b,
    uint8_t* __restrict__ k_pool, uint8_t* __restrict__ v_pool, int64_t num_slots,
    const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int n_kv_heads, int row_bytes, int tok,
    int block_size, int block_shift, int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int R = 2 * n_kv_heads;  // rows per token
  const int tok_bytes = R * row_bytes;
  const int stage_bytes = tok * tok_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 2 * stage_bytes);
  const int tid = threadIdx.x;
  const bool heads_contiguous = head_stride_b == row_bytes;
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t nchunks = (num_tokens + tok - 1) / tok;
  auto load_chunk = [&](int64_t c, int st) {  // thread 0
    const int64_t t0 = c * tok;
    const int nt = num_tokens - t0 < tok ? int(num_tokens - t0) : tok;
    mbar_arrive_expect_tx(&bar[st], uint32_t(nt) * uint32_t(tok_bytes));
    uint8_t* dst = sm + st * stage_bytes;
    for (int i = 0; i < nt; ++i) {
      const uint8_t* ks = k + (t0 + i) * token_stride_b;
      const uint8_t* vs = v + (t0 + i) * token_stride_b;
      uint8_t* d = dst + i * tok_bytes;
      if (heads_contiguous) {
        bulk_g2s(d, ks, uint32_t(n_kv_heads * row_bytes), &bar[st]);
        bulk_g2s(d + n_kv_heads * row_bytes, vs, uint32_t(n_kv_heads * row_bytes), &bar[st]);
      } else {
        for (int h = 0; h < n_kv_heads; ++h) {
          bulk_g2s(d + h * row_bytes, ks + h * head_stride_b, uint32_t(row_bytes), &bar[st]);
          bulk_g2s(d + (n_kv_heads + h) * row_bytes, vs + h * head_stride_b, uint32_t(row_bytes), &bar[st]);
        }
      }
    }
  };
  int it = 0;
  if (tid == 0 && int64_t(blockIdx.x) < nchunks) load_chunk(blockIdx.x, 0);
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
    const int st = it & 1;
    bulk_wait_reads();  // the other stage's stores (previous chunk) are out of shared memory
    __syncthreads();
    if (tid == 0 && c + gridDim.x < nchunks) load_chunk(c + gridDim.x, st ^ 1);
    const bool landed = mbar_wait(&bar[st], uint32_t(it >> 1) & 1u, err, 0x500);
    if (!__syncthreads_and(landed)) break;
    const int64_t t0 = c * tok;
    for (int row = tid; row < tok * R; row += kBulkThreads) {
      const int i = row / R, r = row - i * R;
      const int64_t t = t0 + i;
      if (t >= num_tokens) continue;
      const int64_t slot = __ldg(slot_mapping + t);
      if (slot >= num_slots) {
        if (r == 0) record_error(err, FVB_ERR_BAD_SLOT, int(t));
        continue;
      }
      if (slot < 0) continue;  // padding token
      const int h = r < n_kv_heads ? r : r - n_kv_heads;
      const int64_t blk = block_shift >= 0 ? (slot >> block_shift) : slot / block_size;
      const int off = int(slot - blk * block_size);
      uint8_t* dst = (r < n_kv_heads ? k_pool : v_pool) +
                     ((blk * n_kv_heads + h) * block_size + off) * int64_t(row_bytes);
      bulk_s2g(dst, smem_u32(sm + st * stage_bytes + row * row_bytes), uint32_t(row_bytes));
    }
    bulk_commit_group();
  }
  bulk_wait_done();  // no copy of this CTA is in flight when it exits
}

cudaError_t launch_store_kvcache(const void* k, const void* v, int64_t token_stride, int64_t head_stride,
                                 void* k_pool, void* v_pool, int64_t num_blocks, const int64_t* slot_mapping,
                                 int64_t num_tokens, int n_kv_heads, int head_dim, int block_size, int esize,
                                 int* err, cudaStream_t stream) {
  if (num_tokens == 0) return cudaSuccess;
  const int row_bytes = head_dim * esize;
  const int64_t ts_b = token_stride * esize, hs_b = head_stride * esize;
  auto aligned = [](const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  int vec_bytes = esize;
  for (int cand : {16, 8, 4}) {
    if (cand >= esize && row_bytes % cand == 0 && ts_b % cand == 0 && hs_b % cand == 0 && aligned(k, cand) &&
        aligned(v, cand) && aligned(k_pool, cand) && aligned(v_pool, cand)) {
      vec_bytes = cand;
      break;
    }
  }
  // grid: enough blocks for every token once (two per step), capped at 8 resident CTAs per SM
  const int lanes = std::min(row_bytes / vec_bytes, 256), slots_pb = 256 / lanes, rows = 2 * n_kv_heads;
  const int64_t tpb = rows <= slots_pb ? slots_pb / rows : 1;
  int64_t blocks = (num_tokens + 2 * tpb - 1) / (2 * tpb);
  const int64_t cap = int64_t(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const int threads = 256;
  const int64_t num_slots = num_blocks * block_size;
  int block_shift = -1;  // page size a power of two: slot / block_size as a shift
  for (int b = 0; b < 31; ++b)
    if ((1 << b) == block_size) block_shift = b;
  auto* kb = static_cast<const uint8_t*>(k);
  auto* vb = static_cast<const uint8_t*>(v);
  auto* kp = static_cast<uint8_t*>(k_pool);
  auto* vp = static_cast<uint8_t*>(v_pool);
  const int tok_bytes = 2 * n_kv_heads * row_bytes;
  // Small writes (a decode step's one token per sequence) keep the one-round-trip vector kernel:
  // at 256 tokens it took 4.5 us against 5.4 us for the staged bulk copies.
  if (vec_bytes == 16 && tok_bytes <= kBulkStageBytes && num_tokens >= kBulkMinTokens) {
    // Bulk copies need 16-byte-aligned addresses and sizes: every row start and length here is.
    // tok * tok_bytes <= 16 KB, so the two stages stay under the 48 KB default dynamic shared memory.
    const int tok = std::min(4, kBulkStageBytes / tok_bytes);
    const int smem = 2 * tok * tok_bytes + 16;
    const int64_t nchunks = (num_tokens + tok - 1) / tok;
    const int64_t grid = std::min<int64_t>(nchunks, int64_t(device_sm_count()) * kBulkCtasPerSm);
    store_kvcache_bulk_kernel<<<unsigned(grid), kBulkThreads, smem, stream>>>(
        kb, vb, ts_b, hs_b, kp, vp, num_slots, slot_mapping, num_tokens, n_kv_heads, row_bytes, tok, block_size,
        block_shift, err);
    return cudaGetLastError();
  }
  switch (vec_bytes) {
    case 16:
      store_kvcache_kernel<16><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                         slot_mapping, num_tokens, n_kv_heads,
                                                                         row_bytes, block_size, block_shift, err);
      break;
    case 8:
      store_kvcache_kernel<8><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, block_shift, err);
      break;
    case 4:
      store_kvcache_kernel<4><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, block_shift, err);
      break;
    default:
      store_kvcache_kernel<2><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, block_shift, err);
      break;
  }
  return cudaGetLastError();
}

// slot_mapping[t] = table[s][pos_t / P] * P + pos_t % P for every new token t
// of sequence s, -1 when the table entry is -1 or pos_t lies outside the row.
// The index arithmetic of the reference's write loops (qwen3.py:250-264
// decode, 335-361 prefill), computed on the device.  cu_seqlens == nullptr
// means one token per sequence (decode: token t belongs to sequence t).
__global__ void __launch_bounds__(256) build_slot_mapping_kernel(const int32_t* __restrict__ positions,
                                                                 int64_t num_tokens,
                                                                 const int32_t* __restrict__ cu_seqlens, int num_seqs,
                                                                 const int32_t* __restrict__ block_tables,
                                                                 int max_blocks_per_seq, int block_size,
                                                                 int64_t* __restrict__ slot_mapping, int* err) {
  const int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (t >= num_tokens) return;
  int s;
  if (cu_seqlens == nullptr) {
    s = int(t);
  } else {
    int lo = 0, hi = num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(cu_seqlens + mid) <= t) lo = mid; else hi = mid - 1;
    }
    s = lo;
  }
  const int pos = __ldg(positions + t);
  const int page = pos >= 0 ? pos / block_size : -1;
  int64_t slot = -1;
  if (page < 0 || page >= max_blocks_per_seq || s >= num_seqs) {
    record_error(err, FVB_ERR_INVALID_ARGUMENT, int(t));
  } else {
    const int blk = __ldg(block_tables + int64_t(s) * max_blocks_per_seq + page);
    if (blk >= 0) slot = int64_t(blk) * block_size + pos % block_size;
  }
  slot_mapping[t] = slot;
}

cudaError_t launch_build_slot_mapping(const int32_t* positions, int64_t num_tokens, const int32_t* cu_seqlens,
                                      int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                                      int block_size, int64_t* slot_mapping, int* err, cudaStream_t stream) {
  if (num_tokens == 0) return cudaSuccess;
  const int64_t blocks = (num_tokens + 255) / 256;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  build_slot_mapping_kernel<<<unsigned(blocks), 256, 0, stream>>>(positions, num_tokens, cu_seqlens, num_seqs,
                                                                  block_tables, max_blocks_per_seq, block_size,
                                                                  slot_mapping, err);
  return cudaGetLastError();
}

}  // namespace fvb
