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
#include "common.cuh"
#include "kernels.h"

namespace fvb {

// VEC_BYTES = 16 on the aligned path, sizeof(elem) otherwise.
template <int VEC_BYTES>
__global__ void __launch_bounds__(256) store_kvcache_kernel(const uint8_t* __restrict__ k,
                                                            const uint8_t* __restrict__ v,
                                                            int64_t token_stride_b, int64_t head_stride_b,
                                                            uint8_t* __restrict__ k_pool,
                                                            uint8_t* __restrict__ v_pool, int64_t num_slots,
                                                            const int64_t* __restrict__ slot_mapping,
                                                            int64_t num_tokens, int n_kv_heads, int row_bytes,
                                                            int block_size, int* __restrict__ err) {
  using Vec = typename std::conditional<
      VEC_BYTES == 16, uint4,
      typename std::conditional<VEC_BYTES == 8, uint2,
                                typename std::conditional<VEC_BYTES == 4, uint32_t, uint16_t>::type>::type>::type;
  const int vecs_per_row = row_bytes / VEC_BYTES;
  // Work item = (token, kv head, K-or-V, vector); K and V of a row are
  // adjacent items so one warp streams both.
  const int64_t items_per_token = int64_t(n_kv_heads) * 2 * vecs_per_row;
  const int64_t total = num_tokens * items_per_token;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / items_per_token;
    int rem = int(i - t * items_per_token);
    const int h = rem / (2 * vecs_per_row);
    rem -= h * 2 * vecs_per_row;
    const int which = rem / vecs_per_row;  // 0 = K, 1 = V
    const int vec = rem - which * vecs_per_row;
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {
      record_error(err, FVB_ERR_BAD_SLOT, int(t));
      continue;
    }
    const int64_t blk = slot / block_size;
    const int off = int(slot - blk * block_size);
    const uint8_t* src = (which ? v : k) + t * token_stride_b + h * head_stride_b + int64_t(vec) * VEC_BYTES;
    uint8_t* dst = (which ? v_pool : k_pool) + ((blk * n_kv_heads + h) * block_size + off) * int64_t(row_bytes) +
                   int64_t(vec) * VEC_BYTES;
    *reinterpret_cast<Vec*>(dst) = *reinterpret_cast<const Vec*>(src);
  }
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
  const int64_t items = num_tokens * n_kv_heads * 2 * (row_bytes / vec_bytes);
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  int64_t blocks = (items + threads - 1) / threads;
  const int64_t cap = int64_t(sms) * 8;  // grid-stride beyond 8 resident CTAs per SM
  if (blocks > cap) blocks = cap;
  const int64_t num_slots = num_blocks * block_size;
  auto* kb = static_cast<const uint8_t*>(k);
  auto* vb = static_cast<const uint8_t*>(v);
  auto* kp = static_cast<uint8_t*>(k_pool);
  auto* vp = static_cast<uint8_t*>(v_pool);
  switch (vec_bytes) {
    case 16:
      store_kvcache_kernel<16><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                         slot_mapping, num_tokens, n_kv_heads,
                                                                         row_bytes, block_size, err);
      break;
    case 8:
      store_kvcache_kernel<8><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, err);
      break;
    case 4:
      store_kvcache_kernel<4><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, err);
      break;
    default:
      store_kvcache_kernel<2><<<unsigned(blocks), threads, 0, stream>>>(kb, vb, ts_b, hs_b, kp, vp, num_slots,
                                                                        slot_mapping, num_tokens, n_kv_heads,
                                                                        row_bytes, block_size, err);
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
