// Varlen chunked-prefill causal attention over paged, prefix-cached KV on the
// 5th-generation tensor cores (tcgen05 + TMEM), bf16 / f16.
//
// Replaces the reference's default prefill, the Triton kernel
// femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:6-162 (one
// 16-key page per iteration, K/V re-read per query head), and the SIMT
// PagedAttentionGemmKernel (csrc/paged_attention/paged_attention_gemm.cu:24-302).
// Semantics (the reference's): key j is visible to query i of sequence s iff
// j < kv_lens[s] and j <= positions[i]; softmax in fp32; output cast to T.
// Decode mode (cu_seqlens == positions == nullptr): token s is sequence s's one
// query at position kv_lens[s] - 1; the decode entry points use it for GQA >= 5,
// where the n_rep heads of a group (padded to 8 or 16 tile heads) fill a 128-row
// tile well enough that the tensor cores beat the SIMT split-KV decode.  Its
// items are single query tiles, so the two softmax warpgroups share the one tile
// and take alternate KV tiles ("interleaved KV", merged in the epilogue).
// Prefill batches with GQA groups of 1-4 give their single-token sequences no tile
// here: launch_prefill hands them to the split-KV decode kernel (decode.cu), which
// runs on the SMs this kernel's last wave frees.
//
// Query tile = 128 rows: 128 / n_rep consecutive query tokens of one sequence
// x the n_rep query heads of one kv head's GQA group, so every K/V byte
// fetched serves the whole group.  Work item = (two consecutive query tiles
// of one sequence, kv head); KV is consumed in 128-key tiles (8 pages).
//
//   warpgroup 0  warp 0: TMA producer - both Q tiles once, then the 8 K and
//                8 V pages of every KV tile through the block table (2-D
//                tensor maps over the pools viewed as [blocks*Hkv*16, D],
//                128-byte swizzle) into a ring of K and V stages.
//                warp 1: owns TMEM and issues every MMA from one thread:
//                  S_i  = Q_i K_j^T   (SS: Q_i and K_j in smem)
//                  O_i += P_i V_j     (TS: P_i in TMEM over S_i, V_j in smem)
//                in the order S_0, S_1, PV_0, S_0', PV_1, S_1', ... so one
//                tile's MMAs run while the other tile's softmax runs.
//   warpgroups 1, 2  softmax of query tile 0 / 1, one thread per row (TMEM
//                lane): S_i from TMEM, causal/prefix mask, online softmax in
//                the log2 domain with lazy rescaling (O_i and l are rescaled
//                only when the row max grows by more than 2^8), P_i packed to
//                16-bit into S_i's TMEM columns, and finally O_i / l -> out.
//
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,256+D),
// O_1 [384,384+D).  MMAs of one thread execute in issue order, so S_i of the
// next KV tile (issued after PV_i) never overwrites P_i before PV_i read it,
// and the commit that signals S_i also covers the preceding PV_i (the softmax
// may then rescale O_i).  Every mbarrier wait is bounded; a timeout records
// FVB_ERR_DEVICE_TIMEOUT and the CTA still frees its TMEM.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fvb {
namespace {

constexpr int kTileM = 128;            // rows per query tile: query tokens x GQA heads
constexpr int kTileN = 128;            // keys per KV tile
constexpr int kThreads = 384;          // 3 warpgroups
constexpr int kWgThreads = 128;
constexpr int kHalfBytes = 128 * 128;  // 128 rows x one 128-byte swizzle span
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;   // lazy-rescale threshold (P <= 2^8)
constexpr int kSortMaxSeqs = 2048;

template <int D>
struct Cfg {
  static constexpr int kHalves = D / 64;  // 128-byte spans per row of Q / K / V
  // K and V rings are separate: K is needed one MMA slot earlier than V, so
  // it gets the deeper ring when shared memory is short (D = 128).
  static constexpr int kKStages = D == 128 ? 3 : 4;
  static constexpr int kVStages = D == 128 ? 2 : 4;
  static constexpr int kQTileBytes = kHalves * kHalfBytes;
  static constexpr int kKVBytes = kHalves * kHalfBytes;  // 128 keys of K (or V)
  static constexpr int kOffQ = 0;                        // two query tiles
  static constexpr int kOffK = 2 * kQTileBytes;
  static constexpr int kOffV = kOffK + kKStages * kKVBytes;
  static constexpr int kOffBar = kOffV + kVStages * kKVBytes;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], o_done[2]
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * (kVStages + 1) + 6;  // + decode mode's extra V stage
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};
__device__ __forceinline__ uint32_t col_s(int i) { return uint32_t(i) * 128u; }
__device__ __forceinline__ uint32_t col_o(int i) { return 256u + uint32_t(i) * 128u; }

// max(a, b, c) in one instruction (3-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

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

// Work plan of one launch (one CTA):
//  order[p]    = p-th sequence by descending kv_len (identity beyond kSortMaxSeqs
//                sequences), so the longest-context work is dispatched first;
//  cu_items[p] = exclusive scan of ceil(ceil(q_len / tile_tokens) / tiles_per_item)
//                (work items of that many query tiles) over that order; sequences of
//                one query token get none when skip_single is set (the split-KV decode
//                kernel serves them).
__global__ void __launch_bounds__(1024) prefill_plan_kernel(const int32_t* __restrict__ cu_seqlens,
                                                            const int32_t* __restrict__ kv_lens, int num_seqs,
                                                            int tile_tokens, int tiles_per_item,
                                                            int32_t* __restrict__ order,
                                                            int32_t* __restrict__ cu_items, int skip_single) {
  __shared__ int kv_sh[kSortMaxSeqs];
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const bool sort = num_seqs <= kSortMaxSeqs;
  if (sort) {
    for (int t = threadIdx.x; t < num_seqs; t += blockDim.x) kv_sh[t] = __ldg(kv_lens + t);
  }
  if (threadIdx.x == 0) {
    carry = 0;
    cu_items[0] = 0;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < num_seqs; s += blockDim.x) {
    int rank = s;
    if (sort) {
      const int ks = kv_sh[s];
      rank = 0;
      for (int t = 0; t < num_seqs; ++t) {
        const int kt = kv_sh[t];
        rank += (kt > ks) || (kt == ks && t < s);
      }
    }
    order[rank] = s;
  }
  __syncthreads();
  for (int base = 0; base < num_seqs; base += blockDim.x) {
    const int p = base + threadIdx.x;
    int v = 0;
    if (p < num_seqs) {
      const int s = order[p];
      // decode mode (cu_seqlens == nullptr): one query token per sequence
      const int ql = cu_seqlens ? __ldg(cu_seqlens + s + 1) - __ldg(cu_seqlens + s) : 1;
      const int tiles = ql > 0 && !(skip_single && ql == 1) ? (ql + tile_tokens - 1) / tile_tokens : 0;
      v = (tiles + tiles_per_item - 1) / tiles_per_item;
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
    if (p < num_seqs) cu_items[p + 1] = incl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
}

template <typename T, int D, int NREP, bool kIlv>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, T* __restrict__ out, int64_t q_len_flatten, int num_seqs,
    int n_kv_heads, int64_t num_blocks, const int32_t* __restrict__ cu_seqlens, const int32_t* __restrict__ order,
    const int32_t* __restrict__ cu_items, const int32_t* __restrict__ block_tables, int max_blocks_per_seq,
    const int32_t* __restrict__ kv_lens, int kv_cap, const int32_t* __restrict__ positions, const QOLayout lay,
    int group, int chunks, int tiles_per_split, int max_splits, float* __restrict__ ws_o,
    float* __restrict__ ws_lse, int* __restrict__ err) {
  using C = Cfg<D>;
  constexpr int TOK = kTileM / NREP;  // query tokens per tile
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  launch_dependents();  // decode mode: the split combine may start once every CTA is resident
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::kKStages;
  // Decode mode (kIlv) never loads query tile 1, so its shared-memory slot is one more V stage
  // (GQA 8 / 16 decode 1.5-3.8 % faster than with the two-stage ring).
  constexpr int kVS = kIlv ? C::kVStages + 1 : C::kVStages;
  auto v_off = [](int st) -> int {
    return (kIlv && st == C::kVStages) ? C::kOffQ + C::kQTileBytes : C::kOffV + st * C::kKVBytes;
  };
  uint64_t* v_full = k_empty + C::kKStages;
  uint64_t* v_empty = v_full + kVS;
  uint64_t* s_full = v_empty + kVS;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_done = p_full + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);

  // ---- work item: (query-tile pair, kv head); the heaviest items have the lowest ids ----
  // CTA = (work item, kv head, chunk): a GQA group of `group` query heads is served in
  // chunks of NREP heads (the tile's head slots); slots past the group load a real
  // head's q and are never written.
  // With split-KV (decode mode, tiles_per_split > 0) each such CTA is further one of
  // max_splits ranges of 128-key tiles.
  const int nsp = tiles_per_split > 0 ? max_splits : 1;
  const int split = int(blockIdx.x) % nsp, cta = int(blockIdx.x) / nsp;
  const int units = n_kv_heads * chunks;
  const int item = cta / units, unit = cta % units;
  const int kvh = unit / chunks, chunk = unit % chunks;
  const int head0 = kvh * group + chunk * NREP;     // query head of tile slot g = head0 + g
  const int nvh = min(NREP, group - chunk * NREP);  // slots that are real heads
  if (item >= __ldg(cu_items + num_seqs)) return;
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_items + mid) <= item) lo = mid; else hi = mid - 1;
  }
  const int s = __ldg(order + lo);
  // decode mode (cu_seqlens == nullptr): token s of sequence s, at position kv_len - 1
  const int q_begin = cu_seqlens ? __ldg(cu_seqlens + s) : s;
  const int q_end = cu_seqlens ? __ldg(cu_seqlens + s + 1) : s + 1;
  const int ntq = (q_end - q_begin + TOK - 1) / TOK;
  const int pair = (ntq + 1) / 2 - 1 - (item - __ldg(cu_items + lo));  // last (longest-context) pair first
  const bool has1 = 2 * pair + 1 < ntq;
  // kv_cap <= the block-table row; in decode mode also <= max_kv_len and the split plan's
  // reach, so a longer kv_len is reported and clamped, never read past or dropped unseen.
  int kv_len = __ldg(kv_lens + s);
  if (kv_len > kv_cap) {
    if (threadIdx.x == 0 && split == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
    kv_len = kv_cap;
  }
  int t0[2], t_last[2], p_last[2], nkv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    t0[i] = q_begin + (2 * pair + i) * TOK;
    t_last[i] = min(t0[i] + TOK, q_end) - 1;
    const bool live = i == 0 || has1;
    const int p_tok = positions ? __ldg(positions + t_last[i]) : kv_len - 1;
    p_last[i] = (live && kv_len > 0) ? max(min(p_tok, kv_len - 1), 0) : -1;
    nkv[i] = p_last[i] >= 0 ? p_last[i] / kTileN + 1 : 0;
  }
  int n_kv = max(nkv[0], nkv[1]);
  const int pos_max = max(p_last[0], p_last[1]);  // last key visible to any row of the item
  const int need_pages = pos_max / kPageSize + 1;  // pages holding every visible key
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (n_kv == 0) {  // empty context (never produced by the engine): zeros, not garbage
    for (int e = threadIdx.x; split == 0 && e < 2 * kTileM * D; e += kThreads) {
      const int i = e / (kTileM * D), r = (e / D) % kTileM, tok = t0[i] + r % TOK;
      if ((i == 0 || has1) && tok <= t_last[i] && r / TOK < nvh)
        out[int64_t(tok) * lay.o_ts + int64_t(head0 + r / TOK) * lay.o_hs + e % D] = Elem<T>::from_f(0.f);
    }
    return;
  }
  // KV tiles of this CTA: [j0, j0 + n_kv) in global tile numbers; the loops below
  // count j from 0 (ring slots, barrier phases, the softmax's first tile) and add
  // j0 for page and key offsets.
  int j0 = 0;
  bool partial_out = false;  // more than one split: write a normalised partial + log2-sum-exp
  if (tiles_per_split > 0) {
    const int ns = (n_kv + tiles_per_split - 1) / tiles_per_split;
    if (split >= ns) return;  // this split lies past the sequence (uniform per CTA)
    j0 = split * tiles_per_split;
    partial_out = ns > 1;
#pragma unroll
    for (int i = 0; i < 2; ++i) nkv[i] = max(0, min(nkv[i], j0 + tiles_per_split) - j0);
    n_kv = max(nkv[0], nkv[1]);
  }
  // Interleaved KV (kIlv, the decode-mode instantiations): an item with one query
  // tile and two or more KV tiles gives both softmax groups query tile 0, group 0
  // the even and group 1 the odd KV tiles (local numbering), and merges their
  // (max, sum, O) in the epilogue.  The tile's S -> softmax -> PV chain then
  // alternates with a second independent chain, as a tile pair's two chains do.
  // (Measured 9 % faster on GQA-8 decode; prefill launches, whose single-tile items
  // are few and off the critical path, keep the plain mode: 1 % slower there.)
  const bool ilv = kIlv && !has1 && n_kv >= 2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kWgThreads);
      mbar_init(&o_done[i], 1);
    }
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
  const int wg = threadIdx.x / kWgThreads;

  if (wg == 0) {
    if ((warp == 0 || warp == 2) && lane == 0) {
      // ======================= TMA producers: warp 0 = Q + K, warp 2 = V =======================
      const bool is_k = warp == 0;
      prefetch_tensormap(is_k ? &kmap : &vmap);
      if (is_k) {
        prefetch_tensormap(&qmap);
        mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * C::kQTileBytes);
        for (int i = 0; i < (has1 ? 2 : 1); ++i) {
#pragma unroll
          for (int g = 0; g < NREP; ++g) {
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h) {
              // box = TOK tokens x 64 dims of head head0 + g (rows past the end read as zeros)
              tma_load_3d(smem + C::kOffQ + i * C::kQTileBytes + h * kHalfBytes + g * TOK * 128, &qmap, h * 64, t0[i],
                          head0 + min(g, nvh - 1), q_full);
            }
          }
        }
      }
      const int nst_ring = is_k ? C::kKStages : kVS;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* ring = smem + (is_k ? C::kOffK : C::kOffV);
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      const int32_t* table = block_tables + int64_t(s) * max_blocks_per_seq;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % nst_ring, use = j / nst_ring;
        const int p0 = (j0 + j) * (kTileN / kPageSize);
        const int np = min(kTileN / kPageSize, need_pages - p0);
        int rows[kTileN / kPageSize];
        for (int pi = 0; pi < np; ++pi) {
          int blk = __ldg(table + p0 + pi);
          if (blk < 0 || blk >= num_blocks) {
            record_error(err, FVB_ERR_BAD_PAGE, s);
            blk = 0;
          }
          rows[pi] = (blk * n_kv_heads + kvh) * kPageSize;
        }
        if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1, err, is_k ? 0x300 : 0x301)) break;
        mbar_arrive_expect_tx(&full[st], uint32_t(np) * kPageSize * D * 2);
        for (int pi = 0; pi < np; ++pi) {
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
            uint8_t* stage = is_k ? ring + st * C::kKVBytes : smem + v_off(st);
            tma_load_2d(stage + h * kHalfBytes + pi * kPageSize * 128, map, h * 64, rows[pi], &full[st]);
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ============================ MMA issuer ============================
      constexpr uint32_t idesc_s = umma_idesc_f16(kBF16, kTileM, kTileN, false);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBF16, kTileM, D, true);
      const uint32_t sm_q = smem_u32(smem + C::kOffQ);
      const uint32_t sm_k = smem_u32(smem + C::kOffK);
      const uint32_t sm_v = smem_u32(smem + C::kOffV);
      // Descriptors are built once; an operand at byte offset `off` from a base is
      // base descriptor + off / 16 (shared-memory addresses stay below 256 KB, so
      // the 14-bit start-address field never carries).
      const uint64_t dq = umma_sdesc_sw128(sm_q, 16, 1024);
      const uint64_t dk = umma_sdesc_sw128(sm_k, 16, 1024);
      const uint64_t dv = umma_sdesc_sw128(sm_v, kHalfBytes, 1024);
      // S_i = Q_qi K^T (K in ring stage st) into S_i's TMEM columns
      auto issue_s = [&](int i, int qi, int st) {
        const uint64_t qd = dq + uint64_t((qi * C::kQTileBytes) >> 4);
        const uint64_t kd = dk + uint64_t((st * C::kKVBytes) >> 4);
        const uint32_t d_tmem = tmem + col_s(i);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = uint64_t(((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4);
          umma_f16_ss(d_tmem, qd + off, kd + off, idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int i, int st, bool acc) {
        const uint64_t vd = dv + uint64_t((v_off(st) - C::kOffV) >> 4);
        const uint32_t d_tmem = tmem + col_o(i), a_tmem = tmem + col_s(i);
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {
          umma_f16_ts(d_tmem, a_tmem + kk * 8, vd + uint64_t((kk * 16 * 128) >> 4), idesc_o,
                      (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, err, 0x310) && mbar_wait(&k_full[0], 0, err, 0x311);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0, 0);
        umma_commit(&s_full[0]);
        if (has1) {
          issue_s(1, 1, 0);
          umma_commit(&s_full[1]);
        }
        umma_commit(&k_empty[0]);
      }
      if (ilv) {
        // KV tile j belongs to group j & 1: S_{j&1} = Q_0 K_j^T, then O_{j&1} += P V_j;
        // the S on K_{j+2} follows the PV of K_j (it overwrites the P that PV reads).
        if (ok) ok = mbar_wait(&k_full[1], 0, err, 0x317);  // stage 1, first use
        if (ok) {
          tc_fence_after();
          issue_s(1, 0, 1);
          umma_commit(&s_full[1]);
          umma_commit(&k_empty[1]);
        }
        for (int j = 0; ok && j < n_kv; ++j) {
          const int i = j & 1, st = j % kVS;
          ok = mbar_wait(&p_full[i], (j >> 1) & 1, err, 0x312 + 3 * i) &&
               mbar_wait(&v_full[st], (j / kVS) & 1, err, 0x313 + 3 * i);
          if (!ok) break;
          tc_fence_after();
          issue_pv(i, st, j > 1);
          umma_commit(&v_empty[st]);
          if (j + 2 >= n_kv) {
            umma_commit(&o_done[i]);
            continue;
          }
          const int kst = (j + 2) % C::kKStages;
          ok = mbar_wait(&k_full[kst], ((j + 2) / C::kKStages) & 1, err, 0x314);
          if (!ok) break;
          tc_fence_after();
          issue_s(i, 0, kst);
          umma_commit(&s_full[i]);
          umma_commit(&k_empty[kst]);
        }
      }
      for (int j = 0; ok && !ilv && j < n_kv; ++j) {
        const int st = j % kVS, nst = (j + 1) % C::kKStages;
        const uint32_t vph = (j / kVS) & 1, nkph = ((j + 1) / C::kKStages) & 1;
        bool k_next = false;
        if (j < nkv[0]) {
          ok = mbar_wait(&p_full[0], j & 1, err, 0x312) && mbar_wait(&v_full[st], vph, err, 0x313);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, st, j > 0);
          if (j == nkv[0] - 1) umma_commit(&o_done[0]);
          if (j + 1 < nkv[0]) {
            ok = mbar_wait(&k_full[nst], nkph, err, 0x314);
            if (!ok) break;
            k_next = true;
            tc_fence_after();
            issue_s(0, 0, nst);
            umma_commit(&s_full[0]);
          }
          if (!has1) {
            umma_commit(&v_empty[st]);
            if (j + 1 < nkv[0]) umma_commit(&k_empty[nst]);
          }
        }
        if (has1 && j < nkv[1]) {
          ok = mbar_wait(&p_full[1], j & 1, err, 0x315) && mbar_wait(&v_full[st], vph, err, 0x316);
          if (!ok) break;
          tc_fence_after();
          issue_pv(1, st, j > 0);
          if (j == nkv[1] - 1) umma_commit(&o_done[1]);
          umma_commit(&v_empty[st]);
          if (j + 1 < nkv[1]) {
            if (!k_next) {
              ok = mbar_wait(&k_full[nst], nkph, err, 0x317);
              if (!ok) break;
              tc_fence_after();
            }
            issue_s(1, 1, nst);
            umma_commit(&s_full[1]);
            umma_commit(&k_empty[nst]);
          }
        }
      }
    }
  } else if (wg == 1 || has1 || ilv) {
    // ============================ softmax / epilogue of query tile i ============================
    // (interleaved KV: group i of query tile 0's rows, over KV tiles i, i + 2, ...)
    const int i = wg - 1;
    const int qi = ilv ? 0 : i;  // query tile of this group's rows
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // tile row == TMEM lane
    const int g = r / TOK, tok = t0[qi] + r % TOK;
    const bool row_valid = tok <= t_last[qi] && g < nvh;
    const int head = head0 + g;
    int pos = (row_valid && positions) ? __ldg(positions + tok) : p_last[qi];
    pos = max(min(pos, kv_len - 1), 0);
    const float scale = kLog2e * rsqrtf(float(D));
    const float2 scale2 = make_float2(scale, scale);
    const uint32_t t_row = tmem + (uint32_t(q4 * 32) << 16);
    float m_ref = -INFINITY;  // raw-score reference max of P and l
    float l = 0.f;
    bool ok = true;
    const int my_tiles = ilv ? (n_kv + 1 - i) / 2 : nkv[i];
    for (int jj = 0; jj < my_tiles; ++jj) {
      const int j = ilv ? 2 * jj + i : jj;  // local KV tile
      ok = warp_wait(&s_full[i], jj & 1, err, 0x320 + i);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld_128cols(t_row + col_s(i), sr);
      const int kbase = (j0 + j) * kTileN;
      if (kbase + kTileN - 1 > pos) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (kbase + c > pos) sr[c] = __float_as_uint(-INFINITY);
        }
      }
      float mx[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = __uint_as_float(sr[a]);
#pragma unroll
      for (int c = 8; c < 120; c += 16) {
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = fmax3(mx[a], __uint_as_float(sr[c + a]), __uint_as_float(sr[c + 8 + a]));
      }
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = fmaxf(mx[a], __uint_as_float(sr[120 + a]));
      const float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      // Lazy rescale: keep the reference max unless this tile's max exceeds it by
      // more than 2^8; rows that grow rescale l now and O (in TMEM) after P is out.
      float corr = 1.f;
      bool rescale = false;
      if (jj == 0) {
        // finite for tile 0 (key 0 is visible to every row); with interleaved KV a
        // row may see no key of group 1's first tile: -inf until a later tile
        m_ref = mt;
      } else {
        const bool grow = (mt - m_ref) * scale > kRescaleLog2;
        rescale = __any_sync(0xffffffffu, grow);
        if (grow) {
          corr = fast_exp2((m_ref - mt) * scale);
          l *= corr;
          m_ref = mt;
        }
      }
      // P = 2^((s - m_ref) * scale) <= 2^8, packed to 16 bits into S_i's first 64 columns
      // (P = 0 while the row has seen no key).
      const float ms = (kIlv && m_ref == -INFINITY) ? 0.f : m_ref * scale;
      const float2 nms2 = make_float2(-ms, -ms);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float2 x =
            __ffma2_rn(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), scale2, nms2);
        const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        acc[(c >> 1) & 3] = __fadd2_rn(acc[(c >> 1) & 3], p);
        pk[c >> 1] = pack2<T>(p.x, p.y);
      }
      const float2 a01 = __fadd2_rn(acc[0], acc[1]), a23 = __fadd2_rn(acc[2], acc[3]);
      const float2 a = __fadd2_rn(a01, a23);
      l += a.x + a.y;
      tmem_st_64cols(t_row + col_s(i), pk);
      if (rescale) {
        // O_i holds P V over earlier tiles relative to the old m_ref (PV_{j-1} is
        // complete: S_i of this tile was issued after it).
        const float2 corr2 = make_float2(corr, corr);
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          tmem_ld_32cols(t_row + col_o(i) + cc * 32, o);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float2 v = __fmul2_rn(make_float2(__uint_as_float(o[c]), __uint_as_float(o[c + 1])), corr2);
            o[c] = __float_as_uint(v.x);
            o[c + 1] = __float_as_uint(v.y);
          }
          tmem_st_32cols(t_row + col_o(i) + cc * 32, o);
        }
      }
      tmem_wait_st();
      if (j == n_kv - 1 && kbase + kTileN - 1 > pos_max) {
        // Keys past the last visible one (pos_max) in the final KV tile are either
        // not loaded (stale shared memory) or uninitialised pool slots: P is 0
        // there, but 0 * NaN is not, so zero those V rows before the PV reads them.
        const int st = j % kVS;
        ok = warp_wait(&v_full[st], (j / kVS) & 1, err, 0x324 + i);
        if (!ok) break;
        if (kbase + r > pos_max) {
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
              sts_v4(smem_u32(smem + v_off(st) + h * kHalfBytes + r * 128 + c * 16), make_uint4(0, 0, 0, 0));
          }
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      mbar_arrive(&p_full[i]);
    }
    if (ok) ok = warp_wait(&o_done[i], 0, err, 0x326 + i);
    // out = O_i / l, or with interleaved KV the merge of both groups' rows:
    // M = max(m_0, m_1), L = sum l_g 2^(m_g - M), out = sum O_g 2^(m_g - M) / L.
    // The groups swap (max, sum) through shared memory and each finishes half of the
    // columns from both O's.
    const float m_log2 = m_ref * scale;  // -inf for a row that saw no key
    float f_own, f_oth = 0.f, lse;
    int cc_begin = 0, cc_end = D / 32;
    if (ilv) {
      // K ring stage 0: every QK^T has completed once this group's o_done has (the last one
      // is issued before either group's last PV), and no K copy is pending.
      float* xm = reinterpret_cast<float*>(smem + C::kOffK);
      float* xl = xm + 2 * kTileM;
      xm[i * kTileM + r] = m_log2;
      xl[i * kTileM + r] = l;
      ok = named_barrier_and(1, 2 * kWgThreads, ok);
      if (ok) ok = warp_wait(&o_done[1 - i], 0, err, 0x326 + (1 - i));
      const float m_oth = xm[(1 - i) * kTileM + r], l_oth = xl[(1 - i) * kTileM + r];
      const float M = fmaxf(m_log2, m_oth);  // finite: group 0's first tile holds key 0
      const float w_own = fast_exp2(m_log2 - M), w_oth = fast_exp2(m_oth - M);
      const float L = fmaf(l, w_own, l_oth * w_oth);
      f_own = w_own / L;
      f_oth = w_oth / L;
      lse = M + __log2f(L);
      cc_begin = i * (D / 64);
      cc_end = cc_begin + D / 64;
    } else {
      f_own = 1.f / l;
      lse = m_log2 + __log2f(l);
    }
    if (ok) {
      tc_fence_after();
      T* orow = out + int64_t(tok) * lay.o_ts + int64_t(head) * lay.o_hs;
      // split partial of (sequence tok, head): O / l in fp32 and log2(sum exp) in log2 units,
      // the layout decode_combine_kernel merges ([seq][head][split][D], [seq][head][split])
      const int64_t pidx = (int64_t(tok) * (n_kv_heads * group) + head) * max_splits + split;
      if (partial_out && row_valid && (!ilv || i == 0)) ws_lse[pidx] = lse;
#pragma unroll 1
      for (int cc = cc_begin; cc < cc_end; ++cc) {
        uint32_t o[32];
        float v[32];
        tmem_ld_32cols(t_row + col_o(i) + cc * 32, o);
        if (ilv) {
          uint32_t o2[32];
          tmem_ld_32cols(t_row + col_o(1 - i) + cc * 32, o2);
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = fmaf(__uint_as_float(o[c]), f_own, __uint_as_float(o2[c]) * f_oth);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(o[c]) * f_own;
        }
        if (partial_out) {
          if (row_valid) {
            float4* dst = reinterpret_cast<float4*>(ws_o + pidx * D + cc * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[q * 4 + 0], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
          }
        } else if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<T>(v[q * 8 + 0], v[q * 8 + 1]);
            w.y = pack2<T>(v[q * 8 + 2], v[q * 8 + 3]);
            w.z = pack2<T>(v[q * 8 + 4], v[q * 8 + 5]);
            w.w = pack2<T>(v[q * 8 + 6], v[q * 8 + 7]);
            dst[q] = w;
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

template <typename T, int D, int NREP, bool kIlv>
cudaError_t launch_tc(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                      int n_kv_heads, int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens,
                      const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens, int kv_cap,
                      const int32_t* positions, const PrefillPlan& plan, const QOLayout& lay, int group,
                      int tiles_per_split, int max_splits, float* ws_o, float* ws_lse, void* workspace, int* err,
                      cudaStream_t stream) {
  using C = Cfg<D>;
  constexpr int TOK = kTileM / NREP;
  const int chunks = (group + NREP - 1) / NREP;
  const CUtensorMapDataType tdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap qmap, kmap, vmap;
  const uint64_t pool_rows = uint64_t(num_blocks) * n_kv_heads * kPageSize;
  // q as (D, tokens, heads) with the caller's strides: any (T, H, D)-indexable layout.
  const uint64_t qdims[3] = {uint64_t(D), uint64_t(q_len_flatten), uint64_t(n_kv_heads) * group};
  const uint64_t qstrides[2] = {uint64_t(lay.q_ts) * 2, uint64_t(lay.q_hs) * 2};
  const uint32_t qbox[3] = {64, uint32_t(TOK), 1};
  cudaError_t ce = make_tma_3d(&qmap, q, tdt, qdims, qstrides, qbox, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&kmap, k_pool, tdt, D, pool_rows, D * 2, 64, kPageSize, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&vmap, v_pool, tdt, D, pool_rows, D * 2, 64, kPageSize, true);
  if (ce != cudaSuccess) return ce;
  int32_t* order = static_cast<int32_t*>(workspace);
  int32_t* cu_items = order + ((num_seqs + 63) & ~63);
  ce = launch_prefill_plan(cu_seqlens, kv_lens, num_seqs, TOK, 2, order, cu_items, stream,
                           cu_seqlens != nullptr && plan.single_rows_apart ? 1 : 0);
  if (ce != cudaSuccess) return ce;
  auto kern = prefill_tc_kernel<T, D, NREP, kIlv>;
  ce = set_smem_once<prefill_tc_kernel<T, D, NREP, kIlv>>(C::kSmemBytes);
  if (ce != cudaSuccess) return ce;
  const int64_t ctas = plan.max_tiles * n_kv_heads * chunks * (tiles_per_split > 0 ? max_splits : 1);
  if (ctas > 0x7fffffff) return cudaErrorInvalidValue;
  kern<<<unsigned(ctas), kThreads, C::kSmemBytes, stream>>>(qmap, kmap, vmap, static_cast<T*>(out), q_len_flatten,
                                                            num_seqs, n_kv_heads, num_blocks, cu_seqlens, order,
                                                            cu_items, block_tables, max_blocks_per_seq, kv_lens,
                                                            kv_cap, positions, lay, group, chunks, tiles_per_split,
                                                            max_splits, ws_o, ws_lse, err);
  return cudaGetLastError();
}

template <typename T, int D, bool kIlv>
cudaError_t dispatch_tc(int nrep, const void* q, void* out, const void* k_pool, const void* v_pool,
                        int64_t num_blocks, int n_kv_heads, int num_seqs, int64_t q_len_flatten,
                        const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                        const int32_t* kv_lens, int kv_cap, const int32_t* positions, const PrefillPlan& plan,
                        const QOLayout& lay, int tiles_per_split, int max_splits, float* ws_o, float* ws_lse, void* ws,
                        int* err, cudaStream_t stream) {
#define FVB_TC_ARGS q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens, block_tables, \
                    max_blocks_per_seq, kv_lens, kv_cap, positions, plan, lay, nrep, tiles_per_split, max_splits,  \
                    ws_o, ws_lse, ws, err, stream
  if constexpr (kIlv) {
    // decode mode serves groups of 5 and more: tiles of 8 or 16 heads
    return tc_tile_heads(nrep) == 8 ? launch_tc<T, D, 8, true>(FVB_TC_ARGS) : launch_tc<T, D, 16, true>(FVB_TC_ARGS);
  } else {
    switch (tc_tile_heads(nrep)) {
      case 1:
        return launch_tc<T, D, 1, false>(FVB_TC_ARGS);
      case 2:
        return launch_tc<T, D, 2, false>(FVB_TC_ARGS);
      case 4:
        return launch_tc<T, D, 4, false>(FVB_TC_ARGS);
      case 8:
        return launch_tc<T, D, 8, false>(FVB_TC_ARGS);
      default:
        return launch_tc<T, D, 16, false>(FVB_TC_ARGS);
    }
  }
#undef FVB_TC_ARGS
}

}  // namespace

cudaError_t launch_prefill_plan(const int32_t* cu_seqlens, const int32_t* kv_lens, int num_seqs, int tile_tokens,
                                int tiles_per_item, int32_t* order, int32_t* cu_items, cudaStream_t stream,
                                int skip_single) {
  prefill_plan_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, kv_lens, num_seqs, tile_tokens, tiles_per_item, order,
                                              cu_items, skip_single);
  return cudaGetLastError();
}

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
  p.tile_tokens = kTileM / tc_tile_heads(n_heads / n_kv_heads);
  // Work items are query-tile pairs; each sequence wastes at most one partial pair.
  p.max_tiles = (q_len_flatten + 2 * p.tile_tokens - 1) / (2 * p.tile_tokens) + num_seqs;
  // order[num_seqs] (padded to 64 entries) + cu_items[num_seqs + 1]
  p.ws_bytes = ((size_t((num_seqs + 63) & ~63) + num_seqs + 1) * 4 + 255) & ~size_t(255);
  // Sequences of one query token (decode rows of a mixed batch) fill 1 / tile_tokens of a
  // query tile here; with GQA groups of up to 4 they go to the split-KV decode kernel
  // instead, whose partials (at most kSingleRowMaxSplits splits per row) follow the plan
  // when they fit in 64 MB (and the sequences in the decode grid's third dimension).
  const int group = n_heads / n_kv_heads;
  const size_t rows = size_t(num_seqs) * n_heads * kSingleRowMaxSplits;
  const size_t single_bytes = ((rows * head_dim * 4 + 255) & ~size_t(255)) + rows * 4;
  p.single_rows_apart = group <= 4 && single_bytes <= (size_t(64) << 20) && num_seqs <= 65535;
  p.off_single = p.ws_bytes;
  if (p.single_rows_apart) p.ws_bytes += single_bytes;
  return p;
}

cudaError_t launch_prefill(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                           int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                           const int32_t* cu_seqlens, int max_q_len, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* kv_lens, const int32_t* positions, int dtype,
                           const PrefillPlan& plan, const QOLayout& lay, void* workspace, int* err,
                           cudaStream_t stream) {
  (void)max_q_len;
  if (num_seqs == 0 || q_len_flatten == 0) return cudaSuccess;
  const int nrep = n_heads / n_kv_heads;
  const int kv_cap = int(std::min<int64_t>(int64_t(max_blocks_per_seq) * kPageSize, 0x7fffffff));
#define FVB_DISPATCH_ARGS nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens, \
                          block_tables, max_blocks_per_seq, kv_lens, kv_cap, positions, plan, lay, 0, 1, nullptr,  \
                          nullptr, workspace, err, stream
  cudaError_t ce;
  if (dtype == FVB_DTYPE_BF16) {
    ce = head_dim == 128 ? dispatch_tc<__nv_bfloat16, 128, false>(FVB_DISPATCH_ARGS)
                         : dispatch_tc<__nv_bfloat16, 64, false>(FVB_DISPATCH_ARGS);
  } else {
    ce = head_dim == 128 ? dispatch_tc<__half, 128, false>(FVB_DISPATCH_ARGS)
                         : dispatch_tc<__half, 64, false>(FVB_DISPATCH_ARGS);
  }
#undef FVB_DISPATCH_ARGS
  if (ce != cudaSuccess || !plan.single_rows_apart) return ce;
  // The split-KV decode kernel takes the single-token sequences (prefill_plan_kernel gave
  // them no tile), launched as a programmatic dependent of the tensor-core kernel so its
  // CTAs fill the SMs that kernel's last wave leaves idle.  Its plan is sized for the
  // block table's capacity, with splits lengthened until there are at most
  // kSingleRowMaxSplits.
  DecodePlan dp = plan_decode(num_seqs, n_heads, n_kv_heads, head_dim, kv_cap, device_sm_count());
  const int max_pages = std::max(1, (kv_cap + kPageSize - 1) / kPageSize);
  while (dp.max_splits > kSingleRowMaxSplits) {
    dp.pages_per_split *= 2;
    dp.max_splits = (max_pages + dp.pages_per_split - 1) / dp.pages_per_split;
  }
  return launch_decode(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs, block_tables,
                       max_blocks_per_seq, kv_lens, kv_cap, dtype, dp, lay,
                       static_cast<uint8_t*>(workspace) + plan.off_single, err, stream, cu_seqlens, positions);
}

TcDecodePlan plan_tc_decode(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int max_kv_len, int num_sms) {
  TcDecodePlan p{};
  p.base = plan_prefill(num_seqs, n_heads, n_kv_heads, head_dim, num_seqs, 1, FVB_DTYPE_BF16);
  p.tiles_per_split = 0;
  p.max_splits = 1;
  p.ws_bytes = p.base.ws_bytes;
  if (num_seqs <= 0 || n_kv_heads <= 0) return p;
  const int group = n_heads / n_kv_heads, tile = tc_tile_heads(group);
  const int64_t ctas = int64_t(num_seqs) * n_kv_heads * ((group + tile - 1) / tile);
  const int kv_tiles = std::max(1, (max_kv_len + kTileN - 1) / kTileN);
  // One resident CTA per SM (TMEM and shared memory): split the KV range until there
  // are about two waves, keeping at least 4 tiles (512 keys) per split.
  const int64_t target = int64_t(num_sms) * 2;
  if (ctas >= target || kv_tiles < 8) return p;
  int splits = int(std::min<int64_t>((target + ctas - 1) / ctas, kv_tiles / 4));
  if (splits <= 1) return p;
  const int tps = (kv_tiles + splits - 1) / splits;
  splits = (kv_tiles + tps - 1) / tps;
  if (splits <= 1) return p;
  p.tiles_per_split = tps;
  p.max_splits = splits;
  const size_t rows = size_t(num_seqs) * n_heads * splits;
  p.off_o = p.base.ws_bytes;
  p.off_lse = p.off_o + ((rows * head_dim * 4 + 255) & ~size_t(255));
  p.ws_bytes = p.off_lse + rows * 4;
  return p;
}

cudaError_t launch_tc_decode(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                             int n_heads, int n_kv_heads, int head_dim, int num_seqs, const int32_t* block_tables,
                             int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, int dtype,
                             const TcDecodePlan& plan, const QOLayout& lay, void* workspace, int* err,
                             cudaStream_t stream) {
  if (num_seqs == 0) return cudaSuccess;
  const int nrep = n_heads / n_kv_heads;
  // The longest context any sequence may attend over: max_kv_len, the block-table row and,
  // with split-KV, the splits the plan launches (the combine sizes its shared memory and
  // reads its partial rows by the same bound).
  int64_t cap = std::min<int64_t>(max_kv_len, int64_t(max_blocks_per_seq) * kPageSize);
  if (plan.tiles_per_split > 0) cap = std::min<int64_t>(cap, int64_t(plan.max_splits) * plan.tiles_per_split * kTileN);
  const int kv_cap = int(cap);
  float* ws_o = nullptr;
  float* ws_lse = nullptr;
  if (plan.tiles_per_split > 0) {
    ws_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.off_o);
    ws_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.off_lse);
  }
  // decode mode: no cu_seqlens / positions (token s = sequence s at position kv_len - 1)
#define FVB_TCD_ARGS nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, int64_t(num_seqs), nullptr, \
                     block_tables, max_blocks_per_seq, kv_lens, kv_cap, nullptr, plan.base, lay,                  \
                     plan.tiles_per_split, plan.max_splits, ws_o, ws_lse, workspace, err, stream
  cudaError_t ce;
  if (dtype == FVB_DTYPE_BF16) {
    ce = head_dim == 128 ? dispatch_tc<__nv_bfloat16, 128, true>(FVB_TCD_ARGS)
                         : dispatch_tc<__nv_bfloat16, 64, true>(FVB_TCD_ARGS);
  } else {
    ce = head_dim == 128 ? dispatch_tc<__half, 128, true>(FVB_TCD_ARGS) : dispatch_tc<__half, 64, true>(FVB_TCD_ARGS);
  }
#undef FVB_TCD_ARGS
  if (ce != cudaSuccess || plan.tiles_per_split == 0) return ce;
  return launch_decode_combine(ws_o, ws_lse, out, kv_lens, kv_cap, num_seqs, n_heads,
                               head_dim, plan.tiles_per_split * (kTileN / kPageSize), plan.max_splits, dtype, lay,
                               stream);
}

}  // namespace fvb
