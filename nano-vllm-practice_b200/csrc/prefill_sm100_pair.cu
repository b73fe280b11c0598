// Varlen chunked-prefill causal attention on CTA pairs (tcgen05 cta_group::2),
// bf16 / f16, head_dim 128.
//
// Replaces the same reference prefill as prefill_sm100.cu (the Triton kernel
// femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:6-162 and the SIMT
// PagedAttentionGemmKernel, csrc/paged_attention/paged_attention_gemm.cu:24-302)
// with the same semantics: key j is visible to query i of sequence s iff
// j < kv_lens[s] and j <= positions[i]; softmax in fp32; output cast to T.
//
// A cluster of two CTAs (two SMs) works on four consecutive 128-row query tiles
// of one sequence and one kv head's GQA group (tile rows = 128 / n_rep tokens x
// n_rep heads, as in prefill_sm100.cu).  The pair computes two M = 256 tiles:
//   pair tile A = (CTA 0: query tile 4i,     CTA 1: query tile 4i + 1)
//   pair tile B = (CTA 0: query tile 4i + 2, CTA 1: query tile 4i + 3)
// Every MMA is a cta_group::2 MMA issued by one thread of CTA 0: A operands (Q,
// P) come 128 rows from each CTA's shared memory, B operands are split by
// columns, so each CTA fetches only half of every K tile (keys 64r..64r+63 of
// the 128) and half of every V tile (head dims 64r..64r+63).  That halves each
// SM's K/V bytes and shared-memory stages, which leaves room for P in shared
// memory: PV reads P from shared memory (an SS MMA) instead of TMEM, so
//   * the MMA can issue S(j+1) as soon as the softmax has loaded S(j) from TMEM
//     (S and P no longer share TMEM columns), and the softmax of one KV tile
//     overlaps the next tile's QK^T instead of waiting for it;
//   * the softmax never writes TMEM on the P path (TMEM stores slowed the MMA
//     bursts they overlapped).
//
//   warp 0 lane 0   TMA producer of Q (both pair tiles, once) and of this CTA's
//                   K halves into a 3-stage ring
//   warp 1          TMEM owner (cta_group::2 allocation of 512 columns); in CTA 0
//                   lane 0 issues every MMA of the pair
//   warp 2 lane 0   TMA producer of this CTA's V halves into a 3-stage ring
//   warp 3 lane 0   relay: waits for this CTA's Q / K / V stages to land and
//                   arrives on CTA 0's stage barriers, so the MMA issuer knows
//                   both halves are present
//   warpgroups 1, 2 softmax of pair tile A / B for this CTA's 128 rows, one
//                   thread per row (TMEM lane): S from TMEM, mask, online softmax
//                   in the log2 domain with lazy rescaling, P (16-bit) into shared
//                   memory in the 128-byte-swizzled K-major layout the MMA reads,
//                   and finally O / l -> out.
//
// TMEM (each CTA, its 128 rows): S_A [0,128), S_B [128,256), O_A [256,384),
// O_B [384,512).  Barrier protocol per pair tile p and KV tile j:
//   s_full[p]  (each CTA)  MMA commit: S_p(j) is in TMEM
//   s_free[p]  (CTA 0, 8)  each softmax warp of both CTAs: S_p(j) loaded
//   p_full[p]  (CTA 0, 8)  each softmax warp of both CTAs: P_p(j) stored (and O rescaled)
//   p_free[p]  (each CTA)  MMA commit: PV_p(j) done, P buffer free, O_p current
// Every wait is bounded (2 s of %globaltimer, FVB_ERR_DEVICE_TIMEOUT); every
// thread of both CTAs reaches the final cluster barrier on every path, after
// which both CTAs free the pair's TMEM.  No load uses multicast.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace fvb {
namespace {

constexpr int kD = 128;                  // head dim served by this kernel
constexpr int kRows = 128;               // rows of a query tile in one CTA
constexpr int kKeys = 128;               // keys per KV tile
constexpr int kThreads = 384;
constexpr int kWg = 128;
constexpr int kStages = 3;               // K and V ring depth
constexpr int kQTile = kRows * kD * 2;   // 32 KB: 2 spans of [128 rows][128 B]
constexpr int kQSpan = kRows * 128;      // 16 KB
constexpr int kKHalf = 64 * kD * 2;      // 16 KB: 64 keys x 128 dims, 2 spans of [64 rows][128 B]
constexpr int kKSpan = 64 * 128;         // 8 KB
constexpr int kVHalf = kKeys * 64 * 2;   // 16 KB: 128 keys x 64 dims, 1 span of [128 rows][128 B]
constexpr int kPTile = kRows * kKeys * 2;  // 32 KB: 2 spans of [128 rows][128 B]
constexpr int kPSpan = kRows * 128;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQTile;
constexpr int kOffV = kOffK + kStages * kKHalf;
constexpr int kOffP = kOffV + kStages * kVHalf;
constexpr int kOffBar = kOffP + 2 * kPTile;
// ql_full, q_full, kl_full[S], k_full[S], k_empty[S], vl_full[S], v_full[S], v_empty[S],
// s_full[2], s_free[2], p_full[2], p_free[2], mma_done
constexpr int kNumBars = 2 + 6 * kStages + 9;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint16_t kBothCtas = 0x3;

__device__ __forceinline__ uint32_t col_s(int p) { return uint32_t(p) * 128u; }
__device__ __forceinline__ uint32_t col_o(int p) { return 256u + uint32_t(p) * 128u; }

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

// Every lane waits; the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  const bool ok = mbar_wait(bar, parity, err, site);
  return __all_sync(0xffffffffu, ok);
}

template <typename T, int NREP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) prefill_pair_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, T* __restrict__ out, int num_seqs, int n_kv_heads, int64_t num_blocks,
    const int32_t* __restrict__ cu_seqlens, const int32_t* __restrict__ order, const int32_t* __restrict__ cu_items,
    const int32_t* __restrict__ block_tables, int max_blocks_per_seq, const int32_t* __restrict__ kv_lens,
    int kv_cap, const int32_t* __restrict__ positions, const QOLayout lay, int group, int chunks,
    int* __restrict__ err) {
  constexpr int TOK = kRows / NREP;  // query tokens per tile
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* ql_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* kl_full = bars + 2;
  uint64_t* k_full = kl_full + kStages;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* vl_full = k_empty + kStages;
  uint64_t* v_full = vl_full + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;  // [2]
  uint64_t* s_free = s_full + 2;         // [2]
  uint64_t* p_full = s_free + 2;         // [2]
  uint64_t* p_free = p_full + 2;         // [2]
  uint64_t* mma_done = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item of the pair: up to four query tiles of one (sequence, kv head, head chunk) ----
  const int cid = int(blockIdx.x) >> 1;
  const int units = n_kv_heads * chunks;
  const int item = cid / units, unit = cid % units;
  const int kvh = unit / chunks, chunk = unit % chunks;
  const int head0 = kvh * group + chunk * NREP;
  const int nvh = min(NREP, group - chunk * NREP);
  if (item >= __ldg(cu_items + num_seqs)) return;  // uniform over the pair
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_items + mid) <= item) lo = mid; else hi = mid - 1;
  }
  const int s = __ldg(order + lo);
  const int q_begin = __ldg(cu_seqlens + s), q_end = __ldg(cu_seqlens + s + 1);
  const int ntq = (q_end - q_begin + TOK - 1) / TOK;
  const int it = (ntq + 3) / 4 - 1 - (item - __ldg(cu_items + lo));  // last (longest-context) item first
  const bool has_b = 4 * it + 2 < ntq;
  const int npairs = has_b ? 2 : 1;
  int kv_len = __ldg(kv_lens + s);
  if (kv_len > kv_cap) {
    if (threadIdx.x == 0 && rank == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
    kv_len = kv_cap;
  }
  // Last visible key of each of the four tiles (-1: tile past the sequence), and per pair tile
  // the number of 128-key tiles its two halves need (the same in both CTAs).
  int p_last4[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int tile = 4 * it + t;
    int pl = -1;
    if (tile < ntq && kv_len > 0) {
      const int tl = min(q_begin + (tile + 1) * TOK, q_end) - 1;
      pl = max(min(__ldg(positions + tl), kv_len - 1), 0);
    }
    p_last4[t] = pl;
  }
  int nkv[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int pm = max(p_last4[2 * p], p_last4[2 * p + 1]);
    nkv[p] = (p < npairs && pm >= 0) ? pm / kKeys + 1 : 0;
  }
  const int n_kv = max(nkv[0], nkv[1]);
  const int pos_max = max(max(p_last4[0], p_last4[1]), max(p_last4[2], p_last4[3]));
  const int need_pages = pos_max / kPageSize + 1;

  if (n_kv == 0) {  // empty context (never produced by the engine): zeros for this CTA's rows
    for (int e = threadIdx.x; e < 2 * kRows * kD; e += kThreads) {
      const int p = e / (kRows * kD), r = (e / kD) % kRows;
      const int tile = 4 * it + 2 * p + int(rank), tok = q_begin + tile * TOK + r % TOK;
      if (tile < ntq && tok < q_end && r / TOK < nvh)
        out[int64_t(tok) * lay.o_ts + int64_t(head0 + r / TOK) * lay.o_hs + e % kD] = Elem<T>::from_f(0.f);
    }
    return;  // uniform over the pair
  }

  if (threadIdx.x == 0) {
    mbar_init(ql_full, 1);
    mbar_init(q_full, 2);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kl_full[i], 1);
      mbar_init(&k_full[i], 2);
      mbar_init(&k_empty[i], 1);
      mbar_init(&vl_full[i], 1);
      mbar_init(&v_full[i], 2);
      mbar_init(&v_empty[i], 1);
    }
    for (int p = 0; p < 2; ++p) {
      mbar_init(&s_full[p], 1);
      mbar_init(&s_free[p], 8);
      mbar_init(&p_full[p], 8);
      mbar_init(&p_free[p], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int wg = threadIdx.x / kWg;
  const int32_t* table = block_tables + int64_t(s) * max_blocks_per_seq;

  if (wg == 0) {
    if (warp == 0 && lane == 0) {
      // ============ Q (this CTA's rows of both pair tiles) and K halves (keys 64r..64r+63) ============
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      int issued = 0;  // K tiles whose copies were started
      mbar_arrive_expect_tx(ql_full, uint32_t(npairs) * kQTile);
      for (int p = 0; p < npairs; ++p) {
        const int t0 = q_begin + (4 * it + 2 * p + int(rank)) * TOK;  // may lie past the sequence: rows unused
#pragma unroll
        for (int g = 0; g < NREP; ++g) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_3d(smem + kOffQ + p * kQTile + h * kQSpan + g * TOK * 128, &qmap, h * 64, t0,
                        head0 + min(g, nvh - 1), ql_full);
        }
      }
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % kStages, use = j / kStages;
        const int p0 = j * (kKeys / kPageSize) + 4 * int(rank);
        const int np = max(0, min(4, need_pages - p0));
        int rows[4];
        for (int pi = 0; pi < np; ++pi) {
          int blk = __ldg(table + p0 + pi);
          if (blk < 0 || blk >= num_blocks) {
            record_error(err, FVB_ERR_BAD_PAGE, s);
            blk = 0;
          }
          rows[pi] = (blk * n_kv_heads + kvh) * kPageSize;
        }
        if (use > 0 && !mbar_wait(&k_empty[st], (use - 1) & 1, err, 0x400)) break;
        mbar_arrive_expect_tx(&kl_full[st], uint32_t(np) * kPageSize * kD * 2);
        for (int pi = 0; pi < np; ++pi) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(smem + kOffK + st * kKHalf + h * kKSpan + pi * kPageSize * 128, &kmap, h * 64, rows[pi],
                        &kl_full[st]);
        }
        issued = j + 1;
      }
      // Before this CTA may exit, every copy it started has landed (bounded waits).
      mbar_wait(ql_full, 0, err, 0x405);
      for (int jj = max(0, issued - kStages); jj < issued; ++jj)
        mbar_wait(&kl_full[jj % kStages], (jj / kStages) & 1, err, 0x406);
    } else if (warp == 2 && lane == 0) {
      // ============ V halves (head dims 64r..64r+63 of every key) ============
      prefetch_tensormap(&vmap);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % kStages, use = j / kStages;
        const int p0 = j * (kKeys / kPageSize);
        const int np = max(0, min(kKeys / kPageSize, need_pages - p0));
        int rows[kKeys / kPageSize];
        for (int pi = 0; pi < np; ++pi) {
          int blk = __ldg(table + p0 + pi);
          if (blk < 0 || blk >= num_blocks) {
            record_error(err, FVB_ERR_BAD_PAGE, s);
            blk = 0;
          }
          rows[pi] = (blk * n_kv_heads + kvh) * kPageSize;
        }
        if (use > 0 && !mbar_wait(&v_empty[st], (use - 1) & 1, err, 0x401)) break;
        mbar_arrive_expect_tx(&vl_full[st], uint32_t(np) * kPageSize * 128);
        for (int pi = 0; pi < np; ++pi)
          tma_load_2d(smem + kOffV + st * kVHalf + pi * kPageSize * 128, &vmap, int(rank) * 64, rows[pi],
                      &vl_full[st]);
        issued = j + 1;
      }
      for (int jj = max(0, issued - kStages); jj < issued; ++jj)
        mbar_wait(&vl_full[jj % kStages], (jj / kStages) & 1, err, 0x407);
    } else if (warp == 3 && lane == 0) {
      // ============ relay: this CTA's stages landed -> CTA 0's stage barriers ============
      // In the order the MMA issuer consumes them: Q, K0, K1, V0, K2, V1, ..., V(n-1).
      bool ok = mbar_wait(ql_full, 0, err, 0x402);
      if (ok) mbar_arrive_cluster(cluster_smem_addr(q_full, 0));
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {
          const int st = j % kStages;
          ok = mbar_wait(&kl_full[st], (j / kStages) & 1, err, 0x403);
          if (!ok) break;
          mbar_arrive_cluster(cluster_smem_addr(&k_full[st], 0));
        }
        if (j > 0) {
          const int jv = j - 1, st = jv % kStages;
          ok = mbar_wait(&vl_full[st], (jv / kStages) & 1, err, 0x404);
          if (!ok) break;
          mbar_arrive_cluster(cluster_smem_addr(&v_full[st], 0));
        }
      }
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ============================ MMA issuer of the pair ============================
      constexpr uint32_t idesc_s = umma_idesc_f16(kBF16, 2 * kRows, kKeys, false);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBF16, 2 * kRows, kD, true);
      // Descriptors are built once; an operand at byte offset `off` from a base is base
      // descriptor + off / 16 (shared-memory addresses stay below 256 KB).
      const uint64_t dq = umma_sdesc_sw128(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t dk = umma_sdesc_sw128(smem_u32(smem + kOffK), 16, 1024);
      const uint64_t dp = umma_sdesc_sw128(smem_u32(smem + kOffP), 16, 1024);
      const uint64_t dv = umma_sdesc_sw128(smem_u32(smem + kOffV), kVHalf, 1024);
      auto issue_s = [&](int p, int st) {
        const uint64_t qd = dq + uint64_t((p * kQTile) >> 4);
        const uint64_t kd = dk + uint64_t((st * kKHalf) >> 4);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t qo = uint64_t(((kk >> 2) * kQSpan + (kk & 3) * 32) >> 4);
          const uint64_t ko = uint64_t(((kk >> 2) * kKSpan + (kk & 3) * 32) >> 4);
          umma_f16_ss_pair(tmem + col_s(p), qd + qo, kd + ko, idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int p, int st, bool acc) {
        const uint64_t pd = dp + uint64_t((p * kPTile) >> 4);
        const uint64_t vd = dv + uint64_t((st * kVHalf) >> 4);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t po = uint64_t(((kk >> 2) * kPSpan + (kk & 3) * 32) >> 4);
          umma_f16_ss_pair(tmem + col_o(p), pd + po, vd + uint64_t((kk * 16 * 128) >> 4), idesc_o,
                           (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait_cluster(q_full, 0, err, 0x410) && mbar_wait_cluster(&k_full[0], 0, err, 0x411);
      if (ok) {
        tc_fence_after();
        for (int p = 0; p < npairs; ++p) {
          if (nkv[p] > 0) {
            issue_s(p, 0);
            umma_commit_pair(&s_full[p], kBothCtas);
          }
        }
        umma_commit_pair(&k_empty[0], kBothCtas);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int jn = j + 1;
        if (jn < n_kv) {
          // QK^T of the next KV tile as soon as each softmax has read this tile's S
          const int st = jn % kStages;
          ok = mbar_wait_cluster(&k_full[st], (jn / kStages) & 1, err, 0x412);
          for (int p = 0; ok && p < npairs; ++p) {
            if (jn < nkv[p]) {
              ok = mbar_wait_cluster(&s_free[p], j & 1, err, 0x413 + p);
              if (!ok) break;
              tc_fence_after();
              issue_s(p, st);
              umma_commit_pair(&s_full[p], kBothCtas);
            }
          }
          if (!ok) break;
          umma_commit_pair(&k_empty[st], kBothCtas);
        }
        const int sv = j % kStages;
        ok = mbar_wait_cluster(&v_full[sv], (j / kStages) & 1, err, 0x415);
        for (int p = 0; ok && p < npairs; ++p) {
          if (j < nkv[p]) {
            ok = mbar_wait_cluster(&p_full[p], j & 1, err, 0x416 + p);
            if (!ok) break;
            tc_fence_after();
            issue_pv(p, sv, j > 0);
            umma_commit_pair(&p_free[p], kBothCtas);
          }
        }
        if (!ok) break;
        umma_commit_pair(&v_empty[sv], kBothCtas);
      }
      // Every MMA of the pair has completed before either CTA frees TMEM or exits.
      umma_commit_pair(mma_done, 0x1);
      mbar_wait(mma_done, 0, err, 0x418);
    }
  } else if (wg - 1 < npairs) {
    // ============================ softmax / epilogue of pair tile p, this CTA's rows ============================
    const int p = wg - 1;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // tile row == TMEM lane
    const int tile = 4 * it + 2 * p + int(rank);
    const int g = r / TOK, tok = q_begin + tile * TOK + r % TOK;
    const bool row_valid = tile < ntq && tok < q_end && g < nvh;
    const int head = head0 + g;
    const int p_pair = max(p_last4[2 * p], p_last4[2 * p + 1]);
    int pos = row_valid ? __ldg(positions + tok) : p_pair;
    pos = max(min(pos, kv_len - 1), 0);
    const float scale = kLog2e * rsqrtf(float(kD));
    const float2 scale2 = make_float2(scale, scale);
    const uint32_t t_row = tmem + (uint32_t(q4 * 32) << 16);
    const uint32_t s_free_leader = cluster_smem_addr(&s_free[p], 0);
    const uint32_t p_full_leader = cluster_smem_addr(&p_full[p], 0);
    const uint32_t p_row = smem_u32(smem + kOffP + p * kPTile) + uint32_t(r) * 128u;
    const int nk = nkv[p];
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      ok = warp_wait(&s_full[p], j & 1, err, 0x420 + p);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld_128cols(t_row + col_s(p), sr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(s_free_leader);  // S_p may be overwritten by the next QK^T
      const int kbase = j * kKeys;
      if (kbase + kKeys - 1 > pos) {
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
      // Lazy rescale: keep the reference max unless this tile's max exceeds it by more than 2^8.
      float corr = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_ref = mt;  // finite: key 0 is visible to every row
      } else {
        const bool grow = (mt - m_ref) * scale > kRescaleLog2;
        rescale = __any_sync(0xffffffffu, grow);
        if (grow) {
          corr = fast_exp2((m_ref - mt) * scale);
          l *= corr;
          m_ref = mt;
        }
      }
      const float ms = m_ref * scale;
      const float2 nms2 = make_float2(-ms, -ms);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), scale2, nms2);
        const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        acc[(c >> 1) & 3] = __fadd2_rn(acc[(c >> 1) & 3], e);
        pk[c >> 1] = pack2<T>(e.x, e.y);
      }
      const float2 a01 = __fadd2_rn(acc[0], acc[1]), a23 = __fadd2_rn(acc[2], acc[3]);
      const float2 a = __fadd2_rn(a01, a23);
      l += a.x + a.y;
      // PV_p(j-1) has finished: the P buffer is free and O_p holds every earlier tile.
      if (j > 0) {
        ok = warp_wait(&p_free[p], (j - 1) & 1, err, 0x422 + p);
        if (!ok) break;
        tc_fence_after();
      }
      // P row r: 128 keys = two 128-byte spans, 16-byte chunk c of a span at chunk (c ^ (r & 7)).
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t span = uint32_t(c >> 3) * kPSpan;
        const uint32_t chunk = uint32_t((c & 7) ^ (r & 7)) * 16u;
        sts_v4(p_row + span + chunk, make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
      }
      if (rescale) {
        const float2 corr2 = make_float2(corr, corr);
#pragma unroll 1
        for (int cc = 0; cc < kD / 32; ++cc) {
          uint32_t o[32];
          tmem_ld_32cols(t_row + col_o(p) + cc * 32, o);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float2 v = __fmul2_rn(make_float2(__uint_as_float(o[c]), __uint_as_float(o[c + 1])), corr2);
            o[c] = __float_as_uint(v.x);
            o[c + 1] = __float_as_uint(v.y);
          }
          tmem_st_32cols(t_row + col_o(p) + cc * 32, o);
        }
        tmem_wait_st();
      }
      if (j == n_kv - 1 && kbase + kKeys - 1 > pos_max) {
        // Keys past the last visible one in the final KV tile are either not loaded (stale
        // shared memory) or uninitialised pool slots: P is 0 there, but 0 * NaN is not, so
        // zero those rows of this CTA's V half before the PV reads them.
        const int st = j % kStages;
        ok = warp_wait(&vl_full[st], (j / kStages) & 1, err, 0x424 + p);
        if (!ok) break;
        if (kbase + r > pos_max) {
#pragma unroll
          for (int c = 0; c < 8; ++c)
            sts_v4(smem_u32(smem + kOffV + st * kVHalf + r * 128 + c * 16), make_uint4(0, 0, 0, 0));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(p_full_leader);
    }
    if (ok && nk > 0) ok = warp_wait(&p_free[p], (nk - 1) & 1, err, 0x426 + p);
    if (ok && nk > 0) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      T* orow = out + int64_t(tok) * lay.o_ts + int64_t(head) * lay.o_hs;
#pragma unroll 1
      for (int cc = 0; cc < kD / 32; ++cc) {
        uint32_t o[32];
        tmem_ld_32cols(t_row + col_o(p) + cc * 32, o);
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

  // Every thread of both CTAs: no MMA of the pair is in flight and no arrival is
  // pending once both CTAs are here; then both free the pair's TMEM.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

template <typename T, int NREP>
cudaError_t launch_pair_t(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                          int n_kv_heads, int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens,
                          const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens, int kv_cap,
                          const int32_t* positions, int64_t max_items, const QOLayout& lay, int group,
                          void* workspace, int* err, cudaStream_t stream) {
  constexpr int TOK = kRows / NREP;
  const int chunks = (group + NREP - 1) / NREP;
  const CUtensorMapDataType tdt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap qmap, kmap, vmap;
  const uint64_t pool_rows = uint64_t(num_blocks) * n_kv_heads * kPageSize;
  const uint64_t qdims[3] = {uint64_t(kD), uint64_t(q_len_flatten), uint64_t(n_kv_heads) * group};
  const uint64_t qstrides[2] = {uint64_t(lay.q_ts) * 2, uint64_t(lay.q_hs) * 2};
  const uint32_t qbox[3] = {64, uint32_t(TOK), 1};
  cudaError_t ce = make_tma_3d(&qmap, q, tdt, qdims, qstrides, qbox, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&kmap, k_pool, tdt, kD, pool_rows, kD * 2, 64, kPageSize, true);
  if (ce == cudaSuccess) ce = make_tma_2d(&vmap, v_pool, tdt, kD, pool_rows, kD * 2, 64, kPageSize, true);
  if (ce != cudaSuccess) return ce;
  int32_t* order = static_cast<int32_t*>(workspace);
  int32_t* cu_items = order + ((num_seqs + 63) & ~63);
  ce = launch_prefill_plan(cu_seqlens, kv_lens, num_seqs, TOK, 4, order, cu_items, stream);
  if (ce != cudaSuccess) return ce;
  ce = set_smem_once<prefill_pair_kernel<T, NREP>>(kSmemBytes);
  if (ce != cudaSuccess) return ce;
  const int64_t ctas = 2 * max_items * n_kv_heads * chunks;
  if (ctas > 0x7fffffff) return cudaErrorInvalidValue;
  prefill_pair_kernel<T, NREP><<<unsigned(ctas), kThreads, kSmemBytes, stream>>>(
      qmap, kmap, vmap, static_cast<T*>(out), num_seqs, n_kv_heads, num_blocks, cu_seqlens, order, cu_items,
      block_tables, max_blocks_per_seq, kv_lens, kv_cap, positions, lay, group, chunks, err);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_pair(int nrep, const void* q, void* out, const void* k_pool, const void* v_pool,
                          int64_t num_blocks, int n_kv_heads, int num_seqs, int64_t q_len_flatten,
                          const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                          const int32_t* kv_lens, int kv_cap, const int32_t* positions, int64_t max_items,
                          const QOLayout& lay, void* ws, int* err, cudaStream_t stream) {
#define FVB_PAIR_ARGS q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens, \
                      block_tables, max_blocks_per_seq, kv_lens, kv_cap, positions, max_items, lay, nrep, ws, err, stream
  switch (tc_tile_heads(nrep)) {
    case 1:
      return launch_pair_t<T, 1>(FVB_PAIR_ARGS);
    case 2:
      return launch_pair_t<T, 2>(FVB_PAIR_ARGS);
    case 4:
      return launch_pair_t<T, 4>(FVB_PAIR_ARGS);
    case 8:
      return launch_pair_t<T, 8>(FVB_PAIR_ARGS);
    default:
      return launch_pair_t<T, 16>(FVB_PAIR_ARGS);
  }
#undef FVB_PAIR_ARGS
}

}  // namespace

int64_t prefill_pair_max_items(int num_seqs, int n_heads, int n_kv_heads, int64_t q_len_flatten) {
  const int tok = kRows / tc_tile_heads(n_heads / n_kv_heads);
  // Items are groups of four query tiles; each sequence wastes at most one partial item.
  return (q_len_flatten + 4 * int64_t(tok) - 1) / (4 * int64_t(tok)) + num_seqs;
}

cudaError_t launch_prefill_pair(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                int n_heads, int n_kv_heads, int num_seqs, int64_t q_len_flatten,
                                const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                                const int32_t* kv_lens, const int32_t* positions, int dtype, const QOLayout& lay,
                                void* workspace, int* err, cudaStream_t stream) {
  if (num_seqs == 0 || q_len_flatten == 0) return cudaSuccess;
  const int nrep = n_heads / n_kv_heads;
  const int kv_cap = int(std::min<int64_t>(int64_t(max_blocks_per_seq) * kPageSize, 0x7fffffff));
  const int64_t max_items = prefill_pair_max_items(num_seqs, n_heads, n_kv_heads, q_len_flatten);
  if (dtype == FVB_DTYPE_BF16)
    return dispatch_pair<__nv_bfloat16>(nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten,
                                        cu_seqlens, block_tables, max_blocks_per_seq, kv_lens, kv_cap, positions,
                                        max_items, lay, workspace, err, stream);
  return dispatch_pair<__half>(nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, q_len_flatten,
                               cu_seqlens, block_tables, max_blocks_per_seq, kv_lens, kv_cap, positions, max_items,
                               lay, workspace, err, stream);
}

}  // namespace fvb
