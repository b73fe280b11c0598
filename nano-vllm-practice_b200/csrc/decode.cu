// Decode paged attention over block tables with GQA: split-KV ("flash
// decoding") on SIMT cores, HBM-bound.
//
// Replaces PagedAttentionGemvKernel (csrc/paged_attention/paged_attention_gemv.cu:16-221
// of the reference), which runs one CTA per (sequence, query head), re-reads
// every K/V page once per query head of a GQA group with 2-byte strided loads,
// and keeps all scores in shared memory (so kv_len <= 8192).
//
// Here one CTA serves one (KV split, kv head, sequence) and all n_rep query
// heads of the group, so each K/V byte leaves HBM once:
//
//   warp 0      producer: lane 0 walks the split's pages through the block
//               table and streams them into a 4-slot shared-memory ring, K
//               pages by 2-D TMA with 128-byte swizzle, V pages by 1-D bulk
//               copy; completion is signalled on per-slot mbarriers.
//   warps 1..4  consumers: warp w owns ring slot w (stages w, w+4, ...).  A
//               stage is 32 tokens (2 pages); lane t computes the full q.k dot
//               products of token t for all n_rep heads (q broadcast from
//               shared memory, K chunks read through the swizzle so the 32
//               lanes hit distinct banks), the warp keeps an online softmax in
//               the log2 domain, then lane l accumulates p * V for head dims
//               [l*D/32, (l+1)*D/32) over the stage's tokens.
//
// Arithmetic: with 16-bit K/V the q.k products use sm_100's mixed-precision
// FMA (fma.rn.f32.bf16 / .f16), which takes the 16-bit halves as loaded, and
// p * V runs on packed fp32x2 FMAs; both give exactly the fp32 FMA results of
// the unpacked form, in fewer issue slots (the kernel is HBM-bound only once
// the issue rate stays below the memory rate, which at 4 query heads per kv
// head it did not before).
//
// At the end the four warps' (max, sum, acc) are merged in shared memory; a
// sequence with a single split writes its output directly, otherwise the
// normalised partial and its log-sum-exp go to the workspace and
// decode_combine_kernel, launched as a programmatic dependent, merges the splits.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

constexpr int kStageTokens = 32;  // one token per lane
constexpr int kStagePages = kStageTokens / kPageSize;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = 32 * (1 + kConsumerWarps);
constexpr float kLog2e = 1.4426950408889634f;

template <typename T, int D, int NREP>
struct DecodeTraits {
  static constexpr int kEsize = sizeof(T);
  static constexpr int kRowBytes = D * kEsize;     // one token of one kv head: 128, 256 or 512 B
  static constexpr int kHalves = kRowBytes / 128;  // 128-byte TMA boxes per row
  static constexpr int kBoxCols = 128 / kEsize;
  static constexpr int kPageBytes = kPageSize * kRowBytes;
  static constexpr int kStageBytes = kStageTokens * kRowBytes;  // K (or V) bytes of one stage
  static constexpr int kChunks = kRowBytes / 16;                // 16-byte chunks per K row
  static constexpr int kVec = 16 / kEsize;                      // elements per chunk
  static constexpr int kDPL = D / 32;                           // V dims per lane
  static constexpr int kSlots = kConsumerWarps;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kSlots * kStageBytes;
  static constexpr int kOffQ = 2 * kSlots * kStageBytes;      // T [NREP][D], as given (scaled after the dot)
  static constexpr int kOffP = kOffQ + NREP * D * kEsize;     // float [warp][token][NREP]
  static constexpr int kOffBar = kOffP + kConsumerWarps * kStageTokens * NREP * 4;
  static constexpr int kSmemBytes = kOffBar + 2 * kSlots * 8 + 1024;  // + 1024-B alignment slack
  // Warp-merge scratch (float acc[warp][NREP][D], m[warp][NREP], l[warp][NREP]) aliases the ring.
  static_assert(kConsumerWarps * NREP * (D + 2) * 4 <= 2 * kSlots * kStageBytes, "merge scratch");
  static_assert(kRowBytes % 128 == 0, "row must be whole 128-byte swizzle spans");
};

template <typename T, int DPL>
__device__ __forceinline__ void load_dims(uint32_t addr, float* f) {
  constexpr int kBytes = DPL * sizeof(T);
  if constexpr (kBytes == 16) {
    unpack16<T>(lds_v4(addr), f);
  } else if constexpr (kBytes == 8) {
    uint32_t a, b;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
    if constexpr (sizeof(T) == 4) {
      f[0] = __uint_as_float(a);
      f[1] = __uint_as_float(b);
    } else {
      uint4 v = make_uint4(a, b, 0, 0);
      float tmp[8];
      unpack16<T>(v, tmp);
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = tmp[i];
    }
  } else {
    static_assert(kBytes == 4, "dims per lane");
    uint32_t a;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a) : "r"(addr));
    uint4 v = make_uint4(a, 0, 0, 0);
    float tmp[8];
    unpack16<T>(v, tmp);
    f[0] = tmp[0];
    f[1] = tmp[1];
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int D, int NREP>
__global__ void __launch_bounds__(kDecodeThreads) decode_split_kernel(
    const __grid_constant__ CUtensorMap kmap, const T* __restrict__ q, T* __restrict__ out,
    const uint8_t* __restrict__ v_pool, int64_t num_blocks, int n_kv_heads, int num_seqs,
    const int32_t* __restrict__ block_tables, int max_blocks_per_seq, const int32_t* __restrict__ kv_lens,
    int kv_cap, int pages_per_split, int max_splits, float* __restrict__ ws_o, float* __restrict__ ws_lse,
    const QOLayout lay, int group, int chunks, const int32_t* __restrict__ q_index,
    const int32_t* __restrict__ q_pos, int* __restrict__ err) {
  using Tr = DecodeTraits<T, D, NREP>;
  launch_dependents();  // the combine may take free SM slots once every split CTA is resident
  if (blockIdx.x == gridDim.x - 1 && blockIdx.y == gridDim.y - 1 && blockIdx.z == gridDim.z - 1) {
    // Launched as a programmatic dependent of the tensor-core prefill kernel (single-token
    // rows of a prefill batch, which read nothing that kernel writes): the other CTAs run
    // on the SMs its tail frees, and this one holds the grid open until that kernel has
    // completed, so whatever waits for this grid (the combine, the next launch on the
    // stream) also sees the prefill rows.  A no-op in an ordinary launch.
    grid_dependency_wait();
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  T* qs = reinterpret_cast<T*>(smem + Tr::kOffQ);
  float* ps = reinterpret_cast<float*>(smem + Tr::kOffP);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Tr::kOffBar);
  uint64_t* empty = full + Tr::kSlots;

  // blockIdx.y = (kv head, chunk): a GQA group of `group` query heads is served in
  // chunks of NREP heads; heads of the last chunk past the group are computed on a
  // copy of a real head's q and never written.
  const int split = blockIdx.x, kvh = blockIdx.y / chunks, chunk = blockIdx.y % chunks, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_heads = n_kv_heads * group;
  const int head0 = kvh * group + chunk * NREP;       // query head of row r = head0 + r
  const int nvh = min(NREP, group - chunk * NREP);    // rows that are real heads
  int tok = b;  // q / out row of sequence b
  if (q_index != nullptr) {
    // Single-token sequences of a prefill batch (q_index = its cu_seqlens): sequence b's
    // query is row q_index[b] at position q_pos[row], which sees keys 0 .. position (the
    // tensor-core prefill kernel's mask, position clamped to [0, kv_len - 1]); the other
    // sequences belong to that kernel.
    tok = __ldg(q_index + b);
    if (__ldg(q_index + b + 1) - tok != 1) return;
  }
  int kv_len = max(__ldg(kv_lens + b), 0);
  if (kv_len > kv_cap) {
    // Longer than max_kv_len or than the block table row: never read past either.
    if (split == 0 && threadIdx.x == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, b);
    kv_len = kv_cap;
  }
  if (q_index != nullptr && kv_len > 0) kv_len = min(kv_len, max(__ldg(q_pos + tok), 0) + 1);
  const int npages = (kv_len + kPageSize - 1) / kPageSize;
  const int nsplits = (npages + pages_per_split - 1) / pages_per_split;
  const int page_begin = split * pages_per_split;

  if (npages == 0) {
    // Empty context: the reference never produces one; emit zeros, not garbage.
    if (split == 0) {
      for (int e = threadIdx.x; e < nvh * D; e += blockDim.x) {
        const int r = e / D, d = e % D;
        out[int64_t(tok) * lay.o_ts + int64_t(head0 + r) * lay.o_hs + d] = Elem<T>::from_f(0.f);
      }
    }
    return;
  }
  if (page_begin >= npages) return;  // this split lies past the sequence (uniform per CTA)
  const int page_end = min(npages, page_begin + pages_per_split);
  const int n_iter = (page_end - page_begin + kStagePages - 1) / kStagePages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Tr::kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
  // q for the NREP heads of this group, in its own type: 16-byte reads then cover
  // 8 (16-bit) dims; the log2-domain scale is applied to the finished dot product.
  for (int e = threadIdx.x; e < NREP * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    qs[e] = q[int64_t(tok) * lay.q_ts + int64_t(head0 + min(r, nvh - 1)) * lay.q_hs + d];
  }
  const float qk_scale = kLog2e * rsqrtf(float(D));
  __syncthreads();

  const int32_t* table = block_tables + int64_t(b) * max_blocks_per_seq;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      for (int it = 0; it < n_iter; ++it) {
        const int slot = it % Tr::kSlots;
        const int use = it / Tr::kSlots;
        if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1, err, 0x100 + slot)) return;
        const int p0 = page_begin + it * kStagePages;
        const int np = min(kStagePages, page_end - p0);
        mbar_arrive_expect_tx(&full[slot], uint32_t(np) * 2u * Tr::kPageBytes);
        uint8_t* kdst = smem + Tr::kOffK + slot * Tr::kStageBytes;
        uint8_t* vdst = smem + Tr::kOffV + slot * Tr::kStageBytes;
        for (int j = 0; j < np; ++j) {
          int blk = __ldg(table + p0 + j);
          if (blk < 0 || blk >= num_blocks) {
            record_error(err, FVB_ERR_BAD_PAGE, b);
            blk = 0;  // keep the copy in bounds; the error word reports the bad table
          }
          const int row = (blk * n_kv_heads + kvh) * kPageSize;
#pragma unroll
          for (int hf = 0; hf < Tr::kHalves; ++hf) {
            tma_load_2d(kdst + j * Tr::kPageBytes + hf * 2048, &kmap, hf * Tr::kBoxCols, row, &full[slot]);
          }
          bulk_g2s(vdst + j * Tr::kPageBytes, v_pool + int64_t(row) * Tr::kRowBytes, Tr::kPageBytes, &full[slot]);
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  float m[NREP], l[NREP], acc[NREP][Tr::kDPL];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < Tr::kDPL; ++i) acc[r][i] = 0.f;
  }
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t qs_addr = smem_u32(qs);
  float* pw = ps + cw * kStageTokens * NREP;
  // Lane-constant part of this lane's K row address inside a slot.
  const int kr = lane & 15;
  const uint32_t k_lane_off = (lane >> 4) * Tr::kPageBytes + kr * 128;
  bool ok = true;

  for (int it = cw; it < n_iter; it += kConsumerWarps) {
    const int slot = it % Tr::kSlots;
    if (!mbar_wait(&full[slot], (it / Tr::kSlots) & 1, err, 0x200 + slot)) {
      ok = false;
      break;
    }
    const int tok0 = (page_begin + it * kStagePages) * kPageSize;
    const int nvalid = min(kStageTokens, kv_len - tok0);
    const uint32_t kslot = smem_base + Tr::kOffK + slot * Tr::kStageBytes;
    const uint32_t vslot = smem_base + Tr::kOffV + slot * Tr::kStageBytes;

    // s[r] = q_r . k_lane  (log2 units).  Four independent fp32 partial sums per
    // head (two packed fp32x2 accumulators) keep the FMA dependency chains short.
    float2 sp[NREP][2];
#pragma unroll
    for (int r = 0; r < NREP; ++r) sp[r][0] = sp[r][1] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < Tr::kChunks; ++c) {
      const uint32_t kaddr = kslot + k_lane_off + (c >> 3) * 2048 + ((((c & 7) ^ (kr & 7))) << 4);
      if constexpr (Tr::kEsize == 2) {
        // 16-bit q and k feed mixed-precision FMAs as they are (no unpacking);
        // element e accumulates into sp[r][(e / 2) & 1].x / .y, as the fp32 branch.
        const uint4 k4 = lds_v4(kaddr);
        const uint32_t kw[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int r = 0; r < NREP; ++r) {
          const uint4 q4 = lds_v4(qs_addr + (r * D + c * Tr::kVec) * Tr::kEsize);  // broadcast
          const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) fma_pair16<T>(qw[i], kw[i], sp[r][i & 1]);
        }
      } else {
        float kf[Tr::kVec];
        unpack16<T>(lds_v4(kaddr), kf);
#pragma unroll
        for (int r = 0; r < NREP; ++r) {
          float qf[Tr::kVec];  // one broadcast 16-byte read per head and chunk
          unpack16<T>(lds_v4(qs_addr + (r * D + c * Tr::kVec) * Tr::kEsize), qf);
#pragma unroll
          for (int e = 0; e < Tr::kVec; e += 4) {
            sp[r][0] = __ffma2_rn(make_float2(qf[e + 0], qf[e + 1]), make_float2(kf[e + 0], kf[e + 1]), sp[r][0]);
            sp[r][1] = __ffma2_rn(make_float2(qf[e + 2], qf[e + 3]), make_float2(kf[e + 2], kf[e + 3]), sp[r][1]);
          }
        }
      }
    }
    float s[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) s[r] = ((sp[r][0].x + sp[r][1].x) + (sp[r][0].y + sp[r][1].y)) * qk_scale;
    const bool valid = lane < nvalid;
    float pv_[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float sr = valid ? s[r] : -INFINITY;
      const float mn = fmaxf(m[r], warp_max(sr));  // finite: token 0 of a stage is always valid
      const float corr = fast_exp2(m[r] - mn);
      const float p = fast_exp2(sr - mn);
      m[r] = mn;
      l[r] = l[r] * corr + p;
#pragma unroll
      for (int i = 0; i < Tr::kDPL; ++i) acc[r][i] *= corr;
      pv_[r] = p;
    }
    // this lane's NREP probabilities in one store (the [token][NREP] layout the PV loop reads)
    if constexpr (NREP % 4 == 0) {
#pragma unroll
      for (int r = 0; r < NREP; r += 4)
        *reinterpret_cast<float4*>(pw + lane * NREP + r) = make_float4(pv_[r], pv_[r + 1], pv_[r + 2], pv_[r + 3]);
    } else if constexpr (NREP == 2) {
      *reinterpret_cast<float2*>(pw + lane * NREP) = make_float2(pv_[0], pv_[1]);
    } else {
#pragma unroll
      for (int r = 0; r < NREP; ++r) pw[lane * NREP + r] = pv_[r];
    }
    __syncwarp();
    // acc[r][:] += sum_t p[t][r] * V[t][lane dims]
    const uint32_t v_lane = vslot + lane * Tr::kDPL * Tr::kEsize;
#pragma unroll 4
    for (int t = 0; t < nvalid; ++t) {
      float vf[Tr::kDPL];
      load_dims<T, Tr::kDPL>(v_lane + t * Tr::kRowBytes, vf);
      float pr[NREP];
      if constexpr (NREP % 4 == 0) {
#pragma unroll
        for (int r = 0; r < NREP; r += 4) {
          const float4 pv = *reinterpret_cast<const float4*>(pw + t * NREP + r);
          pr[r] = pv.x;
          pr[r + 1] = pv.y;
          pr[r + 2] = pv.z;
          pr[r + 3] = pv.w;
        }
      } else {
#pragma unroll
        for (int r = 0; r < NREP; ++r) pr[r] = pw[t * NREP + r];
      }
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        if constexpr (Tr::kDPL % 2 == 0) {
          // packed fp32x2 FMAs over dimension pairs: the same per-element FMA, half the issues
#pragma unroll
          for (int i = 0; i < Tr::kDPL; i += 2) {
            const float2 a = __ffma2_rn(make_float2(pr[r], pr[r]), make_float2(vf[i], vf[i + 1]),
                                        make_float2(acc[r][i], acc[r][i + 1]));
            acc[r][i] = a.x;
            acc[r][i + 1] = a.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < Tr::kDPL; ++i) acc[r][i] = fmaf(pr[r], vf[i], acc[r][i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // ---------------- merge the four warps ----------------
  named_barrier(1, 32 * kConsumerWarps);  // every consumer is done with the ring
  float* wacc = reinterpret_cast<float*>(smem);                 // [warp][NREP][D]
  float* wm = wacc + kConsumerWarps * NREP * D;                 // [warp][NREP]
  float* wl = wm + kConsumerWarps * NREP;                       // [warp][NREP]
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    const float lsum = warp_sum(l[r]);
    if (lane == 0) {
      wm[cw * NREP + r] = ok ? m[r] : -INFINITY;
      wl[cw * NREP + r] = ok ? lsum : 0.f;
    }
#pragma unroll
    for (int i = 0; i < Tr::kDPL; ++i) wacc[(cw * NREP + r) * D + lane * Tr::kDPL + i] = ok ? acc[r][i] : 0.f;
  }
  named_barrier(1, 32 * kConsumerWarps);
  const int tid = threadIdx.x - 32;
  for (int e = tid; e < NREP * D; e += 32 * kConsumerWarps) {
    const int r = e / D, d = e % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, wm[w * NREP + r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = fast_exp2(wm[w * NREP + r] - mx);
      L += wl[w * NREP + r] * f;
      O += wacc[(w * NREP + r) * D + d] * f;
    }
    if (r >= nvh) continue;
    const int head = head0 + r;
    if (nsplits == 1) {
      out[int64_t(tok) * lay.o_ts + int64_t(head) * lay.o_hs + d] = Elem<T>::from_f(O / L);
    } else {
      const int64_t idx = (int64_t(b) * n_heads + head) * max_splits + split;
      ws_o[idx * D + d] = O / L;
      if (d == 0) ws_lse[idx] = mx + __log2f(L);
    }
  }
}

// Merge the split partials of every (sequence, head) that has more than one
// split.  One CTA of kCmbThreads per (sequence, head).  A partial row (D fp32) is
// read by D / 4 threads with 16-byte loads, so the CTA covers kGroups rows per pass;
// thread (g, c) walks rows g, g + kGroups, ... with kCmbUnroll rows in flight and
// keeps an online log2-sum-exp merge of them (running max m, sum l and the
// weighted column sums), and the kGroups row groups are merged in shared memory.
// The many independent 16-byte loads per CTA keep the partials streaming; one
// load per thread and split (a CTA per head with a thread per dim) left the merge
// latency-bound at long contexts, where a sequence has ~100 splits.
//
// Launched as a programmatic dependent of the split kernel (which triggers at its
// start): its CTAs take free SM slots during the split kernel's last wave and
// wait in grid_dependency_wait until the partials are complete.
constexpr int kCmbThreads = 256;
constexpr int kCmbUnroll = 4;

template <typename T>
__device__ __forceinline__ void store4(T* p, const float4& v) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    __align__(8) T h[4] = {Elem<T>::from_f(v.x), Elem<T>::from_f(v.y), Elem<T>::from_f(v.z), Elem<T>::from_f(v.w)};
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(h);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kCmbThreads) decode_combine_kernel(const float* __restrict__ ws_o,
                                                                     const float* __restrict__ ws_lse,
                                                                     T* __restrict__ out,
                                                                     const int32_t* __restrict__ kv_lens, int kv_cap,
                                                                     int num_seqs, int n_heads, int pages_per_split,
                                                                     int max_splits, const QOLayout lay,
                                                                     const int32_t* __restrict__ q_index,
                                                                     const int32_t* __restrict__ q_pos) {
  constexpr int kLanes = D / 4;                  // threads per partial row
  constexpr int kGroups = kCmbThreads / kLanes;  // rows per pass: 8 (D 128) or 16 (D 64)
  __shared__ float4 g_acc[kGroups][kLanes];
  __shared__ float g_m[kGroups], g_l[kGroups];
  const int b = blockIdx.x / n_heads, head = blockIdx.x % n_heads;
  // kv_lens was written before the split kernel started (read before the wait).
  int kv_len = min(max(__ldg(kv_lens + b), 0), kv_cap);
  int tok = b;
  bool merge = true;
  if (q_index != nullptr) {  // as in the split kernel: single-token sequences of a prefill batch
    tok = __ldg(q_index + b);
    merge = __ldg(q_index + b + 1) - tok == 1;
    if (merge && kv_len > 0) kv_len = min(kv_len, max(__ldg(q_pos + tok), 0) + 1);
  }
  const int npages = (kv_len + kPageSize - 1) / kPageSize;
  const int nsplits = (npages + pages_per_split - 1) / pages_per_split;
  // Every CTA waits for the split grid, also those with nothing to merge: the combine grid
  // then completes after the split kernel, so work queued behind it on the stream sees the
  // rows the split kernel wrote directly.
  grid_dependency_wait();
  if (!merge || nsplits <= 1) return;  // written directly by the split kernel (or not a row of ours)
  const int g = threadIdx.x / kLanes, c = threadIdx.x % kLanes;
  const int64_t base = (int64_t(b) * n_heads + head) * max_splits;
  const float4* src = reinterpret_cast<const float4*>(ws_o + base * D) + c;
  float m = -INFINITY, l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = g; s0 < nsplits; s0 += kCmbUnroll * kGroups) {
    float4 o[kCmbUnroll];
    float ls[kCmbUnroll];
#pragma unroll
    for (int u = 0; u < kCmbUnroll; ++u) {
      const int s = s0 + u * kGroups;
      const bool in = s < nsplits;
      // L2-coherent loads (.cg): the rows were written by the previous grid.
      o[u] = in ? __ldcg(src + int64_t(s) * kLanes) : make_float4(0.f, 0.f, 0.f, 0.f);
      ls[u] = in ? __ldcg(ws_lse + base + s) : -INFINITY;
    }
    float mn = m;
#pragma unroll
    for (int u = 0; u < kCmbUnroll; ++u) mn = fmaxf(mn, ls[u]);  // finite: row s0 exists
    const float corr = fast_exp2(m - mn);                        // 0 on the first pass
    l *= corr;
    acc.x *= corr;
    acc.y *= corr;
    acc.z *= corr;
    acc.w *= corr;
#pragma unroll
    for (int u = 0; u < kCmbUnroll; ++u) {
      const float w = fast_exp2(ls[u] - mn);  // 0 for rows past nsplits
      l += w;
      acc.x = fmaf(w, o[u].x, acc.x);
      acc.y = fmaf(w, o[u].y, acc.y);
      acc.z = fmaf(w, o[u].z, acc.z);
      acc.w = fmaf(w, o[u].w, acc.w);
    }
    m = mn;
  }
  g_acc[g][c] = acc;  // groups without rows leave m = -inf, l = 0, acc = 0
  if (c == 0) {
    g_m[g] = m;
    g_l[g] = l;
  }
  __syncthreads();
  if (g != 0) return;
  float M = g_m[0];  // finite: group 0 holds split 0
#pragma unroll
  for (int k = 1; k < kGroups; ++k) M = fmaxf(M, g_m[k]);
  float L = 0.f;
  float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < kGroups; ++k) {
    const float w = fast_exp2(g_m[k] - M);
    const float4 a = g_acc[k][c];
    L = fmaf(g_l[k], w, L);
    O.x = fmaf(a.x, w, O.x);
    O.y = fmaf(a.y, w, O.y);
    O.z = fmaf(a.z, w, O.z);
    O.w = fmaf(a.w, w, O.w);
  }
  store4(out + int64_t(tok) * lay.o_ts + int64_t(head) * lay.o_hs + 4 * c,
         make_float4(O.x / L, O.y / L, O.z / L, O.w / L));
}

template <typename T, int D>
cudaError_t launch_combine_t(const float* ws_o, const float* ws_lse, void* out, const int32_t* kv_lens, int kv_cap,
                             int num_seqs, int n_heads, int pages_per_split, int max_splits, const QOLayout& lay,
                             cudaStream_t stream, const int32_t* q_index = nullptr, const int32_t* q_pos = nullptr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(num_seqs) * unsigned(n_heads));
  cfg.blockDim = dim3(kCmbThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_combine_kernel<T, D>, ws_o, ws_lse, static_cast<T*>(out), kv_lens, kv_cap,
                            num_seqs, n_heads, pages_per_split, max_splits, lay, q_index, q_pos);
}

template <typename T, int D, int NREP>
cudaError_t launch_decode_t(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                            int n_kv_heads, int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                            const int32_t* kv_lens, int max_kv_len, const DecodePlan& plan, const QOLayout& lay,
                            int group, void* workspace, int* err, cudaStream_t stream, const int32_t* q_index,
                            const int32_t* q_pos) {
  using Tr = DecodeTraits<T, D, NREP>;
  const bool after_prefill = q_index != nullptr;  // programmatic dependent of the prefill kernel
  const int kv_cap = int(std::min<int64_t>(std::min<int64_t>(max_kv_len, int64_t(max_blocks_per_seq) * kPageSize),
                                           int64_t(plan.max_splits) * plan.pages_per_split * kPageSize));
  CUtensorMap kmap;
  const CUtensorMapDataType tdt = sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cudaError_t ce = make_tma_2d(&kmap, k_pool, tdt, D, uint64_t(num_blocks) * n_kv_heads * kPageSize,
                                Tr::kRowBytes, Tr::kBoxCols, kPageSize, true);
  if (ce != cudaSuccess) return ce;
  auto kern = decode_split_kernel<T, D, NREP>;
  ce = set_smem_once<decode_split_kernel<T, D, NREP>>(Tr::kSmemBytes);
  if (ce != cudaSuccess) return ce;
  float* ws_o = nullptr;
  float* ws_lse = nullptr;
  if (plan.max_splits > 1) {
    ws_o = static_cast<float*>(workspace);
    const size_t o_bytes = size_t(num_seqs) * n_kv_heads * group * plan.max_splits * D * 4;
    ws_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((o_bytes + 255) & ~size_t(255)));
  }
  const int chunks = (group + NREP - 1) / NREP;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.max_splits, n_kv_heads * chunks, num_seqs);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = Tr::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_prefill ? 1 : 0;
  ce = cudaLaunchKernelEx(&cfg, kern, kmap, static_cast<const T*>(q), static_cast<T*>(out),
                          static_cast<const uint8_t*>(v_pool), num_blocks, n_kv_heads, num_seqs, block_tables,
                          max_blocks_per_seq, kv_lens, kv_cap, plan.pages_per_split, plan.max_splits, ws_o, ws_lse,
                          lay, group, chunks, q_index, q_pos, err);
  if (ce == cudaSuccess) ce = cudaGetLastError();
  if (ce != cudaSuccess || plan.max_splits <= 1) return ce;
  return launch_combine_t<T, D>(ws_o, ws_lse, out, kv_lens, kv_cap, num_seqs, n_kv_heads * group,
                                plan.pages_per_split, plan.max_splits, lay, stream, q_index, q_pos);
}

template <typename T, int D>
cudaError_t dispatch_nrep(int nrep, const void* q, void* out, const void* k_pool, const void* v_pool,
                          int64_t num_blocks, int n_kv_heads, int num_seqs, const int32_t* block_tables,
                          int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, const DecodePlan& plan,
                          const QOLayout& lay, void* ws, int* err, cudaStream_t stream, const int32_t* q_index,
                          const int32_t* q_pos) {
#define FVB_DT_ARGS q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, block_tables, max_blocks_per_seq, \
                    kv_lens, max_kv_len, plan, lay, nrep, ws, err, stream, q_index, q_pos
  switch (decode_tile_heads(nrep)) {
    case 1:
      return launch_decode_t<T, D, 1>(FVB_DT_ARGS);
    case 2:
      return launch_decode_t<T, D, 2>(FVB_DT_ARGS);
    case 4:
      return launch_decode_t<T, D, 4>(FVB_DT_ARGS);
    default:
      return launch_decode_t<T, D, 8>(FVB_DT_ARGS);
  }
#undef FVB_DT_ARGS
}

}  // namespace

DecodePlan plan_decode(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int max_kv_len, int num_sms) {
  DecodePlan p{};
  const int max_pages = std::max(1, (max_kv_len + kPageSize - 1) / kPageSize);
  const int group = n_kv_heads > 0 ? n_heads / n_kv_heads : 1;
  const int tile = decode_tile_heads(group);
  const int64_t units = int64_t(num_seqs) * n_kv_heads * ((group + tile - 1) / tile);
  // Splits of up to 256 pages (4096 tokens): each CTA start costs a pipeline fill
  // and drain, which at 1024-token splits held 32k-131k-token contexts 5-8 %
  // below the longer splits.  The longest sequence keeps at least 4 splits down to
  // 64 pages (contexts of 512-4096 tokens keep 1024-token splits, whose shorter
  // tail measured 0.6 % faster there), and splits halve (down to 4 pages) until
  // there are enough CTAs for ~4 waves of 3 resident CTAs per SM.
  const int64_t target = int64_t(num_sms) * 3 * 4;
  int pps = 256;
  while (pps > 64 && max_pages < 4 * pps) pps /= 2;
  while (pps > 4 && units * ((max_pages + pps - 1) / pps) < target) pps /= 2;
  p.pages_per_split = pps;
  p.max_splits = (max_pages + pps - 1) / pps;
  if (p.max_splits > 1) {
    const size_t o_bytes = size_t(num_seqs) * n_heads * p.max_splits * head_dim * 4;
    const size_t lse_bytes = size_t(num_seqs) * n_heads * p.max_splits * 4;
    p.ws_bytes = ((o_bytes + 255) & ~size_t(255)) + lse_bytes;
  } else {
    p.ws_bytes = 0;
  }
  return p;
}

cudaError_t launch_decode(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                          int n_heads, int n_kv_heads, int head_dim, int num_seqs, const int32_t* block_tables,
                          int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, int dtype,
                          const DecodePlan& plan, const QOLayout& lay, void* workspace, int* err,
                          cudaStream_t stream, const int32_t* q_index, const int32_t* q_pos) {
  if (num_seqs == 0) return cudaSuccess;
  const int nrep = n_heads / n_kv_heads;
#define FVB_DECODE_ARGS nrep, q, out, k_pool, v_pool, num_blocks, n_kv_heads, num_seqs, block_tables, \
                        max_blocks_per_seq, kv_lens, max_kv_len, plan, lay, workspace, err, stream, q_index, q_pos
  if (dtype == FVB_DTYPE_BF16) {
    return head_dim == 128 ? dispatch_nrep<__nv_bfloat16, 128>(FVB_DECODE_ARGS)
                           : dispatch_nrep<__nv_bfloat16, 64>(FVB_DECODE_ARGS);
  } else if (dtype == FVB_DTYPE_F16) {
    return head_dim == 128 ? dispatch_nrep<__half, 128>(FVB_DECODE_ARGS) : dispatch_nrep<__half, 64>(FVB_DECODE_ARGS);
  } else {
    return head_dim == 128 ? dispatch_nrep<float, 128>(FVB_DECODE_ARGS) : dispatch_nrep<float, 64>(FVB_DECODE_ARGS);
  }
#undef FVB_DECODE_ARGS
}


cudaError_t launch_decode_combine(const float* ws_o, const float* ws_lse, void* out, const int32_t* kv_lens,
                                  int kv_cap, int num_seqs, int n_heads, int head_dim, int pages_per_split,
                                  int max_splits, int dtype, const QOLayout& lay, cudaStream_t stream) {
  if (num_seqs == 0 || max_splits <= 1) return cudaSuccess;
#define FVB_CMB_ARGS ws_o, ws_lse, out, kv_lens, kv_cap, num_seqs, n_heads, pages_per_split, max_splits, lay, stream
  if (dtype == FVB_DTYPE_BF16) {
    return head_dim == 128 ? launch_combine_t<__nv_bfloat16, 128>(FVB_CMB_ARGS)
                           : launch_combine_t<__nv_bfloat16, 64>(FVB_CMB_ARGS);
  } else if (dtype == FVB_DTYPE_F16) {
    return head_dim == 128 ? launch_combine_t<__half, 128>(FVB_CMB_ARGS) : launch_combine_t<__half, 64>(FVB_CMB_ARGS);
  }
  return head_dim == 128 ? launch_combine_t<float, 128>(FVB_CMB_ARGS) : launch_combine_t<float, 64>(FVB_CMB_ARGS);
#undef FVB_CMB_ARGS
}

}  // namespace fvb
