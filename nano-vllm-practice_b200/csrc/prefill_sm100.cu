// Varlen chunked-prefill causal attention over paged, prefix-cached KV on the
// 5th-generation tensor cores (tcgen05 + TMEM), bf16 / f16.
//
// Replaces the reference's default prefill, the Triton kernel
// femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:6-162 (one
// 16-key page per iteration, K/V re-read per query head), and the SIMT
// PagedAttentionGemmKernel (csrc/paged_attention/paged_attention_gemm.cu:24-302).
// Semantics (the reference's): key j is visible to query i of sequence s iff
// j < kv_lens[s] and j <= positions[i]; softmax in fp32; output cast to T.
//
// Work item = (query tile, kv head).  A tile is 128 rows: 128 / n_rep
// consecutive query tokens of one sequence x the n_rep query heads of the kv
// head's GQA group, so every K/V tile fetched serves the whole group.  KV is
// consumed in 128-key tiles (8 pages).
//
//   warp 0      TMA producer: the Q tile once, then for every KV tile the 8
//               pages of K and of V, page by page through the block table
//               (2-D tensor maps over the pools viewed as [blocks*Hkv*16, D],
//               128-byte swizzle), into a ring of kStages K and V slots.
//   warp 1      owns TMEM (512 columns: S double buffer 2x128, O D columns)
//               and issues the MMAs from one thread:
//                 S[j%2] = Q K_j^T   (M=128, N=128, K=D; both K-major in smem)
//                 O     += P_j V_j   (M=128, N=D,  K=128; P K-major, V MN-major)
//               S_{j+1} is issued before PV_j so the tensor pipe computes the
//               next scores while the softmax works on the current ones.
//   warps 2-5   softmax / epilogue, one thread per tile row (TMEM lane
//               quarter = warp % 4): read S_j from TMEM, mask, online softmax
//               in fp32 (log2 domain), rescale O in TMEM when the running max
//               grows, write P_j (bf16/f16) into a 128-byte-swizzled smem
//               tile for the PV MMA, and finally O / l -> global.
//
// Every mbarrier wait is bounded; a timeout records FVB_ERR_DEVICE_TIMEOUT and
// the CTA tears down (TMEM is always freed).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fvb {
namespace {

constexpr int kTileM = 128;                      // rows: query tokens x GQA heads
constexpr int kTileN = 128;                      // keys per KV tile
constexpr int kThreads = 192;                    // 6 warps
constexpr int kSoftmaxThreads = 128;
constexpr int kHalfBytes = 128 * 128;            // 128 rows x one 128-byte swizzle span
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int kHalves = D / 64;         // 128-byte spans per row of Q / K / V
  static constexpr int kStages = D == 128 ? 2 : 3;
  static constexpr int kQBytes = kHalves * kHalfBytes;
  static constexpr int kKVBytes = kHalves * kHalfBytes;  // 128 keys of K (or V)
  static constexpr int kPBytes = 2 * kHalfBytes;         // 128 rows x 128 keys
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKVBytes;
  static constexpr int kOffP = kOffV + kStages * kKVBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_empty[2], p_full, o_done
  static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 1 + 1;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColO = 256;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Every lane waits; the warp proceeds only if all lanes saw the phase (keeps
// the .sync.aligned tcgen05 instructions that follow warp-uniform).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  const bool ok = mbar_wait(bar, parity, err, site);
  return __all_sync(0xffffffffu, ok);
}

// Exclusive scan of ceil(q_len / tile_tokens) over the sequences -> cu_tiles[0..num_seqs].
__global__ void __launch_bounds__(1024) prefill_plan_kernel(const int32_t* __restrict__ cu_seqlens, int num_seqs,
                                                            int tile_tokens, int32_t* __restrict__ cu_tiles) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (threadIdx.x == 0) {
    carry = 0;
    cu_tiles[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < num_seqs; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int v = 0;
    if (s < num_seqs) {
      const int ql = __ldg(cu_seqlens + s + 1) - __ldg(cu_seqlens + s);
      v = ql > 0 ? (ql + tile_tokens - 1) / tile_tokens : 0;
    }
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = lane < nwarps ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? warp_tot[warp - 1] : 0) + carry;
    if (s < num_seqs) cu_tiles[s + 1] = incl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
}

template <typename T, int D, int NREP>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, T* __restrict__ out, int64_t q_len_flatten, int num_seqs,
    int n_kv_heads, int64_t num_blocks, const int32_t* __restrict__ cu_seqlens, const int32_t* __restrict__ cu_tiles,
    const int32_t* __restrict__ block_tables, int max_blocks_per_seq, const int32_t* __restrict__ kv_lens,
    const int32_t* __restrict__ positions, int* __restrict__ err) {
  using C = Cfg<D>;
  constexpr int TOK = kTileM / NREP;  // query tokens per tile
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::kStages;
  uint64_t* v_full = k_empty + C::kStages;
  uint64_t* v_empty = v_full + C::kStages;
  uint64_t* s_full = v_empty + C::kStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);

  // ---- work item ----
  const int tile_id = blockIdx.x, kvh = blockIdx.y;
  if (tile_id >= __ldg(cu_tiles + num_seqs)) return;
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_tiles + mid) <= tile_id) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int tile = tile_id - __ldg(cu_tiles + s);
  const int q_end = __ldg(cu_seqlens + s + 1);
  const int t0 = __ldg(cu_seqlens + s) + tile * TOK;
  const int t_last = min(t0 + TOK, q_end) - 1;
  int kv_len = __ldg(kv_lens + s);
  if (kv_len > max_blocks_per_seq * kPageSize) {
    if (threadIdx.x == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
    kv_len = max_blocks_per_seq * kPageSize;
  }
  const int pos_last = min(__ldg(positions + t_last), kv_len - 1);
  const int n_tiles = pos_last >= 0 ? pos_last / kTileN + 1 : 0;
  const int need_pages = pos_last / kPageSize + 1;  // pages holding keys 0 .. pos_last
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (n_tiles == 0) {  // empty context (never produced by the engine): zeros, not garbage
    for (int e = threadIdx.x; e < kTileM * D; e += kThreads) {
      const int r = e / D, tok = t0 + r % TOK;
      if (tok < q_end) out[(int64_t(kvh * NREP + r / TOK) * q_len_flatten + tok) * D + e % D] = Elem<T>::from_f(0.f);
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftmaxThreads);
    }
    mbar_init(p_full, kSoftmaxThreads);
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sm_q = smem_u32(smem + C::kOffQ);
  const uint32_t sm_k = smem_u32(smem + C::kOffK);
  const uint32_t sm_v = smem_u32(smem + C::kOffV);
  const uint32_t sm_p = smem_u32(smem + C::kOffP);

  if (warp == 0) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
      for (int g = 0; g < NREP; ++g) {
        const int row = int((int64_t(kvh) * NREP + g) * q_len_flatten + t0);
#pragma unroll
        for (int h = 0; h < C::kHalves; ++h) {
          tma_load_2d(smem + C::kOffQ + h * kHalfBytes + g * TOK * 128, &qmap, h * 64, row, q_full);
        }
      }
      const int32_t* table = block_tables + int64_t(s) * max_blocks_per_seq;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % C::kStages, use = j / C::kStages;
        const int p0 = j * (kTileN / kPageSize);
        const int np = min(kTileN / kPageSize, need_pages - p0);
        const uint32_t bytes = uint32_t(np) * kPageSize * D * 2;
        int rows[kTileN / kPageSize];
        for (int pi = 0; pi < np; ++pi) {
          int blk = __ldg(table + p0 + pi);
          if (blk < 0 || blk >= num_blocks) {
            record_error(err, FVB_ERR_BAD_PAGE, s);
            blk = 0;
          }
          rows[pi] = (blk * n_kv_heads + kvh) * kPageSize;
        }
        if (use > 0 && !mbar_wait(&k_empty[st], (use - 1) & 1, err, 0x300)) break;
        mbar_arrive_expect_tx(&k_full[st], bytes);
        for (int pi = 0; pi < np; ++pi) {
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
            tma_load_2d(smem + C::kOffK + st * C::kKVBytes + h * kHalfBytes + pi * kPageSize * 128, &kmap, h * 64,
                        rows[pi], &k_full[st]);
          }
        }
        if (use > 0 && !mbar_wait(&v_empty[st], (use - 1) & 1, err, 0x301)) break;
        mbar_arrive_expect_tx(&v_full[st], bytes);
        for (int pi = 0; pi < np; ++pi) {
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
            tma_load_2d(smem + C::kOffV + st * C::kKVBytes + h * kHalfBytes + pi * kPageSize * 128, &vmap, h * 64,
                        rows[pi], &v_full[st]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ============================
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(kBF16, kTileM, kTileN, false);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBF16, kTileM, D, true);
      bool ok = mbar_wait(q_full, 0, err, 0x310);
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j < n_tiles) {
          const int st = j % C::kStages, sb = j & 1;
          ok = mbar_wait(&k_full[st], (j / C::kStages) & 1, err, 0x311);
          if (ok && j >= 2) ok = mbar_wait(&s_empty[sb], ((j >> 1) - 1) & 1, err, 0x312);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kst = sm_k + st * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
            umma_f16_ss(tmem + C::kColS + sb * kTileN, umma_sdesc_sw128(sm_q + off, 16, 1024),
                        umma_sdesc_sw128(kst + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[sb]);
          umma_commit(&k_empty[st]);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj % C::kStages;
          ok = mbar_wait(p_full, jj & 1, err, 0x313);
          if (ok) ok = mbar_wait(&v_full[st], (jj / C::kStages) & 1, err, 0x314);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vst = sm_v + st * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            umma_f16_ss(tmem + C::kColO, umma_sdesc_sw128(sm_p + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024),
                        umma_sdesc_sw128(vst + kk * 16 * 128, kHalfBytes, 1024), idesc_o,
                        (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(o_done);
          umma_commit(&v_empty[st]);
        }
      }
    }
  } else {
    // ============================ softmax / epilogue ============================
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // tile row == TMEM lane
    const int g = r / TOK, tok = t0 + r % TOK;
    const bool row_valid = tok <= t_last;
    const int head = kvh * NREP + g;
    int pos = row_valid ? __ldg(positions + tok) : pos_last;
    pos = max(min(pos, kv_len - 1), 0);
    const float scale = kLog2e * rsqrtf(float(D));
    const uint32_t t_row = tmem + (uint32_t(q4 * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      ok = warp_wait(&s_full[sb], (j >> 1) & 1, err, 0x320);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_ld_32cols(t_row + C::kColS + sb * kTileN + c4 * 32, sr[c4]);
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);

      const int kbase = j * kTileN;
      const bool masked = kbase + kTileN - 1 > pos;
      float mt = -INFINITY;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float x = __uint_as_float(sr[c4][c]);
          if (masked && kbase + c4 * 32 + c > pos) x = -INFINITY;
          sr[c4][c] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      }
      const float m_new = fmaxf(m, mt);  // finite: key 0 is visible to every row in tile 0
      const float ms = m_new * scale;
      const float corr = fast_exp2((m - m_new) * scale);
      float rs = 0.f;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p = fast_exp2(fmaf(__uint_as_float(sr[c4][c]), scale, -ms));
          rs += p;
          sr[c4][c] = __float_as_uint(p);
        }
      }
      l = l * corr + rs;
      if (j > 0) {
        // PV_{j-1} must be done before O is rescaled and the P tile overwritten.
        ok = warp_wait(o_done, (j - 1) & 1, err, 0x321);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, m_new > m)) {
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            uint32_t o[32];
            tmem_ld_32cols(t_row + C::kColO + cc * 32, o);
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
            tmem_st_32cols(t_row + C::kColO + cc * 32, o);
          }
          tmem_wait_st();
        }
      }
      m = m_new;
      // P row (K-major, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r % 8))
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        const uint32_t* src = &sr[cc >> 2][(cc & 3) * 8];
        uint4 v;
        v.x = pack2<T>(__uint_as_float(src[0]), __uint_as_float(src[1]));
        v.y = pack2<T>(__uint_as_float(src[2]), __uint_as_float(src[3]));
        v.z = pack2<T>(__uint_as_float(src[4]), __uint_as_float(src[5]));
        v.w = pack2<T>(__uint_as_float(src[6]), __uint_as_float(src[7]));
        sts_v4(sm_p + (cc >> 3) * kHalfBytes + r * 128 + (((cc & 7) ^ (r & 7)) << 4), v);
      }
      if (j == n_tiles - 1 && kbase + kTileN - 1 > pos_last) {
        // Keys past pos_last are masked for every row (P = 0), but their V rows are
        // unloaded or uninitialised pool slots: zero them so 0 * NaN cannot occur.
        const int st = j % C::kStages;
        ok = warp_wait(&v_full[st], (j / C::kStages) & 1, err, 0x322);
        if (!ok) break;
        if (kbase + r > pos_last) {
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
#pragma unroll
            for (int c = 0; c < 8; ++c) sts_v4(sm_v + st * C::kKVBytes + h * kHalfBytes + r * 128 + c * 16,
                                               make_uint4(0, 0, 0, 0));
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = warp_wait(o_done, (n_tiles - 1) & 1, err, 0x323);
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      T* orow = out + (int64_t(head) * q_len_flatten + tok) * D;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        tmem_ld_32cols(t_row + C::kColO + cc * 32, o);
        if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack2<T>(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
            v.y = pack2<T>(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
            v.z = pack2<T>(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
            v.w = pack2<T>(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
            dst[q] = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <typename T, int D, int NREP>
cudaError_t launch_tc(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                      int n_kv_heads, int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens,
                      const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                      const int32_t* positions, const PrefillPlan& plan, void* workspace, int* err,
                      cudaStream_t stream) {
  using C = Cfg<D>;
  constexpr int TOK = kTileM / NREP;
  const CUtensorMapDataType tdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap qmap, kmap, vmap;
  const uint64_t pool_rows = uint64_t(num_blocks) * n_kv_heads * kPageSize;
  cudaError_t ce = make_tma_2d(&qmap, q, tdt, D, uint64_t(n_kv_heads) * NREP * q_len_flatten, D * 2, 64, TOK, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&kmap, k_pool, tdt, D, pool_rows, D * 2, 64, kPageSize, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&vmap, v_pool, tdt, D, pool_rows, D * 2, 64, kPageSize, true);
  if (ce != cudaSuccess) return ce;
  int32_t* cu_tiles = static_cast<int32_t*>(workspace);
  prefill_plan_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, num_seqs, TOK, cu_tiles);
  ce = cudaGetLastError();
  if (ce != cudaSuccess) return ce;
  auto kern = prefill_tc_kernel<T, D, NREP>;
  ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (ce != cudaSuccess) return ce;
  dim3 grid(unsigned(plan.max_tiles), unsigned(n_kv_heads));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(qmap, kmap, vmap, static_cast<T*>(out), q_len_flatten, num_seqs,
                                                  n_kv_heads, num_blocks, cu_seqlens, cu_tiles, block_tables,
                                                  max_blocks_per_seq, kv_lens, positions, err);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t dispatch_tc(int nrep, const void* q, void* out, const void* k_pool, const void* v_pool,
                        int64_t num_blocks, int n_kv_heads, int num_seqs, int64_t q_len_flatten,
                        const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                        const int32_t* kv_lens, const int32_t* positions, const PrefillPlan& plan, void* ws, int* err,
                        cudaStream_t stream) {
#define FVB_TC_ARGS q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens, block_tables, \
                    max_blocks_per_seq, kv_lens, positions, plan, ws, err, stream
  switch (nrep) {
    case 1:
      return launch_tc<T, D, 1>(FVB_TC_ARGS);
    case 2:
      return launch_tc<T, D, 2>(FVB_TC_ARGS);
    case 4:
      return launch_tc<T, D, 4>(FVB_TC_ARGS);
    case 8:
      return launch_tc<T, D, 8>(FVB_TC_ARGS);
    default:
      return cudaErrorInvalidValue;
  }
#undef FVB_TC_ARGS
}

}  // namespace

PrefillPlan plan_prefill(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int64_t q_len_flatten,
                         int max_q_len, int dtype) {
  (void)head_dim;
  (void)max_q_len;
  PrefillPlan p{};
  if (dtype == FVB_DTYPE_F32 || n_kv_heads <= 0 || n_heads % n_kv_heads) {
    p.tile_tokens = 0;
    p.max_tiles = 0;
    p.ws_bytes = 0;
    return p;
  }
  p.tile_tokens = kTileM / (n_heads / n_kv_heads);
  // Each sequence wastes at most one partial tile.
  p.max_tiles = (q_len_flatten + p.tile_tokens - 1) / p.tile_tokens + num_seqs;
  p.ws_bytes = ((size_t(num_seqs) + 1) * 4 + 255) & ~size_t(255);
  return p;
}

cudaError_t launch_prefill(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                           int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                           const int32_t* cu_seqlens, int max_q_len, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* kv_lens, const int32_t* positions, int dtype,
                           const PrefillPlan& plan, void* workspace, int* err, cudaStream_t stream) {
  (void)max_q_len;
  if (num_seqs == 0 || q_len_flatten == 0) return cudaSuccess;
  const int nrep = n_heads / n_kv_heads;
#define FVB_DISPATCH_ARGS nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens, \
                          block_tables, max_blocks_per_seq, kv_lens, positions, plan, workspace, err, stream
  if (dtype == FVB_DTYPE_BF16) {
    return head_dim == 128 ? dispatch_tc<__nv_bfloat16, 128>(FVB_DISPATCH_ARGS)
                           : dispatch_tc<__nv_bfloat16, 64>(FVB_DISPATCH_ARGS);
  }
  return head_dim == 128 ? dispatch_tc<__half, 128>(FVB_DISPATCH_ARGS) : dispatch_tc<__half, 64>(FVB_DISPATCH_ARGS);
#undef FVB_DISPATCH_ARGS
}

}  // namespace fvb
