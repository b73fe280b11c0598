// Next-token sampling over a batch of logit rows in one launch: presence
// penalty, greedy argmax and temperature sampling.
//
// The reference's Sampler.forward (femtovllm/engine/sampler.py:15-114) builds
// Python lists of the sampling parameters, a padded token table and a
// (B, vocab) count matrix (scatter_add), then splits the batch into greedy
// and sampled rows with index gathers, argmax, division, softmax and
// multinomial: about a dozen launches, several full passes over the logits
// and host round trips.  Here every row is read once from HBM:
//
//   apply = any |presence_penalties[r]| > 1e-5 over the batch  (sampler.py:31-35)
//   x[i]  = apply && token i occurs in the row's token table ? l[i] - p : l[i]    (sampler.py:56-76, fp32)
//   greedy row (temperature < 1e-5, sampler.py:41-46): first index of max x     (torch.argmax, :88-95)
//   sampled row: x / T (rounded to the logits' type when !apply, as the reference's
//     in-place division of bf16/fp16 logits does, :97-104), one draw from
//     softmax(x / T) (:106-109) by inverse CDF in vocabulary order with one
//     Philox4x32-10 uniform per row.
//
// Grid: one CTA per (row, chunk of the vocabulary); each of its 8 warps reduces
// a contiguous sub-chunk to a partial, (max, first index) for greedy rows or
// (max, sum of 2^(x2 - max)) in the log2 domain for sampled rows.  The last CTA
// of a row (an atomic ticket) merges the partials, draws the uniform, finds the
// sub-chunk holding it and rescans only that sub-chunk (at most 4096 logits,
// from L2) for the exact token.  The last row to finish advances the RNG
// offset, so a CUDA-graph replay draws fresh numbers.  Tickets are reset by
// the kernel that used them.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMinChunk = 2048;   // multiple of 32 * kWarps, so every sub-chunk is 16-byte aligned
constexpr int kMaxChunk = 32768;  // presence bitmap of one chunk: kMaxChunk / 32 words of shared memory
constexpr float kGreedyBelow = 1e-5f;
constexpr float kPenaltyAbove = 1e-5f;
constexpr float kLog2e = 1.4426950408889634f;

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC 2011): ten rounds of two 32x32->64 multiplies, key bumped by
// the Weyl constants between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = c.x * 0xD2511F53u, hi0 = __umulhi(c.x, 0xD2511F53u);
    const uint32_t lo1 = c.z * 0xCD9E8D57u, hi1 = __umulhi(c.z, 0xCD9E8D57u);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

struct SampleArgs {
  const void* logits;
  int64_t row_stride;  // elements
  int64_t vocab;
  int num_rows;
  const float* temps;
  const float* pens;
  const int64_t* table;
  int64_t table_stride, table_len;
  unsigned long long* rng;  // {seed, offset}
  int64_t* out;
  float2* partials;   // [row][split][warp]
  unsigned* tickets;  // [num_rows] per-row tickets, then the grid ticket
  int chunk, nsplit;
  bool vec_ok;
};

// How a row is treated (uniform over a CTA).
enum { kModeGreedy = 0, kModeSampleF32 = 1, kModeSampleRounded = 2 };
struct RowMode {
  int mode;
  bool pen_on;
  float pen, t, inv_t, c;  // c = log2(e) / T
};

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}

// 2^x on the SFU without the volatile qualifier, so the compiler may schedule it freely.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// l minus the row's penalty when bit e of `bits` (token present) is set.
template <bool PEN>
__device__ __forceinline__ float penalize(float l, uint32_t bits, int e, float pen) {
  if (!PEN) return l;
  int m;  // bit e sign-extended: all ones when the token is present
  asm("bfe.s32 %0, %1, %2, 1;" : "=r"(m) : "r"(bits), "r"(e));
  return l - __int_as_float(m & __float_as_int(pen));
}

template <typename T>
__device__ __forceinline__ float rounded_quotient(float x, const RowMode& md);

// Weight 2^(exponent - m) of one penalized logit of a sampled row (the rescan's form).
template <typename T>
__device__ __forceinline__ float weight(float x, const RowMode& md, float m) {
  return md.mode == kModeSampleF32 ? ex2(fmaf(x, md.c, -m)) : ex2(fmaf(rounded_quotient<T>(x, md), kLog2e, -m));
}

// Loads the group of 16 / sizeof(T) logits starting at `i` (a multiple of the group size
// from the row start) into floats; entries at or past `hi` are -inf and not counted.
template <typename T>
__device__ __forceinline__ int load_group(const T* row, int64_t i, int64_t hi, bool vec_ok, float* v) {
  constexpr int VE = 16 / sizeof(T);
  if (vec_ok && i + VE <= hi) {
    unpack16<T>(ldg_nc_v4(row + i), v);
    return VE;
  }
  const int n = int(hi - i < VE ? hi - i : VE);
#pragma unroll
  for (int e = 0; e < VE; ++e) v[e] = e < n ? Elem<T>::to_f(row[i + e]) : -INFINITY;
  return n;
}

// cp.async.bulk.prefetch.L2: the copy engine pulls [p, p + bytes) into L2 (16-byte aligned, size
// a multiple of 16); a hint, nothing waits on it.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t presence_bits(const uint32_t* bitmap, int64_t off, int ve) {
  return (bitmap[off >> 5] >> (off & 31)) & ((1u << ve) - 1u);
}

template <int N>
__device__ __forceinline__ float tree_max(const float* x) {
  if constexpr (N == 1) {
    return x[0];
  } else {
    return fmaxf(tree_max<N / 2>(x), tree_max<N - N / 2>(x + N / 2));
  }
}

// The reference's in-place x / T of a sampled row on the rounded path, stored in the logits'
// dtype.  x * (1/T) plus one residual correction (fma(-q, T, x) is exact) gives the rounded
// quotient in all but rare double-rounding cases; the residual is NaN only for infinite x,
// where q is already right.
template <typename T>
__device__ __forceinline__ float rounded_quotient(float x, const RowMode& md) {
  const float q = x * md.inv_t;
  const float r = fmaf(-q, md.t, x);
  const float q1 = fmaf(r, md.inv_t, q);
  return round_to<T>(r == r ? q1 : q);
}

// Folds NV groups of logits (group u starts at index i + u * step; entries past the range are
// -inf) into a lane's partial: greedy (max, first index); sampled (m, s) meaning s * 2^m in the
// log2 domain, s kept in four independent sums.  Sampled rows rescale lazily: the reference m
// moves only when a group's maximum passes it by more than 8, so weights stay below 2^8.
template <typename T, int MODE, bool PEN, int NV>
__device__ __forceinline__ void consume(float* x, const uint32_t* bits, int64_t i, int step, const RowMode& md,
                                        float& pa, float* acc, int& pi) {
  constexpr int VE = 16 / sizeof(T), N = NV * VE;
#pragma unroll
  for (int j = 0; j < N; ++j) x[j] = penalize<PEN>(x[j], bits[j / VE], j % VE, md.pen);
  if (MODE == kModeSampleRounded) {
#pragma unroll
    for (int j = 0; j < N; ++j) x[j] = rounded_quotient<T>(x[j], md);
  }
  const float g = tree_max<N>(x);
  if (MODE == kModeGreedy) {
    if (g > pa) {  // strictly: an earlier (smaller) index keeps a tie; -inf never wins
      int k = N - 1;
#pragma unroll
      for (int j = N - 1; j >= 0; --j)
        if (x[j] == g) k = j;
      pa = g;
      pi = int(i + int64_t(k / VE) * step + k % VE);
    }
    return;
  }
  const float scale = MODE == kModeSampleF32 ? md.c : kLog2e;
  const float gy = g * scale;
  if (gy > pa + 8.f) {
    const float f = ex2(pa - gy);  // 0 while pa is -inf
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] *= f;
    pa = gy;
  }
  if (pa == -INFINITY) return;
#pragma unroll
  for (int j = 0; j < N; ++j) acc[j & 3] += ex2(fmaf(x[j], scale, -pa));
}

// One warp's sub-chunk [lo, hi) of a row: U 16-byte loads in flight per lane while the
// whole unrolled step is in range, then one group at a time with bounds.
template <typename T, int MODE, bool PEN>
__device__ __forceinline__ void pass1(const T* lrow, int64_t lo, int64_t hi, int64_t c0, bool vec_ok,
                                      const uint32_t* bitmap, const RowMode& md, float& pa, float& pb, int& pi) {
  constexpr int VE = 16 / sizeof(T), U = 4, STEP = 32 * VE;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t i = lo + (threadIdx.x & 31) * VE;
  if (vec_ok) {
    for (; i + (U - 1) * STEP + VE <= hi; i += U * STEP) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = ldg_nc_v4(lrow + i + u * STEP);
      float x[U * VE];
      uint32_t bits[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        unpack16<T>(raw[u], x + u * VE);
        bits[u] = PEN ? presence_bits(bitmap, i + u * STEP - c0, VE) : 0u;
      }
      consume<T, MODE, PEN, U>(x, bits, i, STEP, md, pa, acc, pi);
    }
  }
  for (; i < hi; i += STEP) {
    float x[VE];
    uint32_t bits[1];
    load_group<T>(lrow, i, hi, vec_ok, x);
    bits[0] = PEN ? presence_bits(bitmap, i - c0, VE) : 0u;
    consume<T, MODE, PEN, 1>(x, bits, i, STEP, md, pa, acc, pi);
  }
  pb = (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// Marks in `bitmap` the tokens of row `row`'s table that fall in [lo, lo + len): the table
// row is read with 16-byte loads (two ids each), eight ids in flight per thread.
__device__ __forceinline__ void mark(uint32_t* bitmap, int64_t id, int64_t lo, int64_t len) {
  const uint64_t d = uint64_t(id - lo);  // ids below lo wrap past len
  if (d < uint64_t(len)) atomicOr(&bitmap[d >> 5], 1u << (d & 31));
}

__device__ void build_bitmap(const SampleArgs& a, int row, int64_t lo, int64_t len, uint32_t* bitmap) {
  const int words = int((len + 31) >> 5);
  for (int w = threadIdx.x; w < words; w += kThreads) bitmap[w] = 0u;
  __syncthreads();
  const int64_t* trow = a.table + int64_t(row) * a.table_stride;
  const int head = (reinterpret_cast<uintptr_t>(trow) & 15) != 0 ? 1 : 0;  // rows are 8-byte aligned
  const int64_t n = a.table_len - head, pairs = n >> 1;
  if (threadIdx.x == 0) {
    if (head) mark(bitmap, __ldg(trow), lo, len);
    if (n & 1) mark(bitmap, __ldg(trow + a.table_len - 1), lo, len);
  }
  const longlong2* tv = reinterpret_cast<const longlong2*>(trow + head);
  constexpr int R = 4;  // pairs in flight per thread
  for (int64_t p0 = threadIdx.x; p0 < pairs; p0 += R * kThreads) {
    longlong2 v[R];
#pragma unroll
    for (int k = 0; k < R; ++k)
      v[k] = p0 + k * kThreads < pairs ? __ldg(tv + p0 + k * kThreads) : make_longlong2(-1, -1);
#pragma unroll
    for (int k = 0; k < R; ++k) {
      mark(bitmap, v[k].x, lo, len);
      mark(bitmap, v[k].y, lo, len);
    }
  }
  __syncthreads();
}

// Greedy partial merge: larger value wins, the smaller index on ties (torch.argmax
// returns the first maximal index); index INT_MAX marks "nothing seen".
__device__ __forceinline__ void merge_max(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// Sampled partial merge in the log2 domain: (m, s) stands for s * 2^m.
__device__ __forceinline__ void merge_lse(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  if (m2 > m) {
    s = s * fast_exp2(m - m2) + s2;
    m = m2;
  } else {
    s += s2 * fast_exp2(m2 - m);
  }
}

// Exclusive block scan of one double per thread; returns the exclusive prefix, *total the sum.
__device__ double block_exclusive_scan(double x, double* warp_sums, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  double excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = 0.0;
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  double before = 0.0, all = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const double ws = warp_sums[w];
    if (w < warp) before += ws;
    all += ws;
  }
  __syncthreads();
  *total = all;
  return before + excl;
}

// The thread that owns the target of an inverse-CDF search: the last thread with
// weight whose run starts at or before it (unique whatever the rounding); -1 if none.
__device__ int block_claimer(bool has_weight, double before, double target, int* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int c = has_weight && before <= target ? int(threadIdx.x) : -1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c = max(c, __shfl_xor_sync(0xffffffffu, c, o));
  if (lane == 0) red_i[warp] = c;
  __syncthreads();
  c = red_i[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) c = max(c, red_i[w]);
  __syncthreads();
  return c;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 4) sample_kernel(SampleArgs a) {
  constexpr int VE = 16 / sizeof(T);
  __shared__ uint32_t bitmap[kMaxChunk / 32];
  __shared__ double warp_sums[kWarps];
  __shared__ float red_f[kWarps];
  __shared__ int red_i[kWarps];
  __shared__ int s_flag;
  __shared__ double s_target;
  __shared__ unsigned long long s_rng[2];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = int(blockIdx.x / unsigned(a.nsplit));
  const int split = int(blockIdx.x - unsigned(row) * unsigned(a.nsplit));
  const T* lrow = static_cast<const T*>(a.logits) + int64_t(row) * a.row_stride;
  const int64_t c0 = int64_t(split) * a.chunk;
  const int64_t c1 = c0 + a.chunk < a.vocab ? c0 + a.chunk : a.vocab;
  const int sub = a.chunk / kWarps;
  const int64_t lo = c0 + int64_t(warp) * sub;
  const int64_t hi = lo + sub < c1 ? lo + sub : c1;
  // Start the HBM stream first: each warp asks the copy engine to bring its sub-chunk into L2
  // while the CTA reads its parameters and builds the presence bitmap.
  if (a.vec_ok && lane == 0 && hi > lo) {
    const uint32_t bytes = uint32_t((hi - lo) * int64_t(sizeof(T))) & ~15u;
    if (bytes) bulk_prefetch_l2(lrow + lo, bytes);
  }

  // Batch-wide penalty switch, as the reference decides it from all rows' parameters.
  int anyp = 0;
  if (a.pens != nullptr)
    for (int r = threadIdx.x; r < a.num_rows; r += kThreads) anyp |= fabsf(__ldg(a.pens + r)) > kPenaltyAbove;
  anyp = __syncthreads_or(anyp);

  RowMode md;
  const float t = __ldg(a.temps + row);
  const bool greedy = t < kGreedyBelow;
  md.pen = anyp ? __ldg(a.pens + row) : 0.f;
  md.pen_on = anyp && md.pen != 0.f && a.table_len > 0;
  md.mode = greedy ? kModeGreedy
                   : (!anyp && Elem<T>::kDtype != FVB_DTYPE_F32 ? kModeSampleRounded : kModeSampleF32);
  md.t = greedy ? 1.f : t;
  md.inv_t = greedy ? 1.f : 1.f / t;
  md.c = md.inv_t * kLog2e;

  if (md.pen_on) build_bitmap(a, row, c0, c1 - c0, bitmap);

  // ---- pass 1: this warp's sub-chunk to one partial ----
  float pa = -INFINITY, pb = 0.f;  // greedy: (value, index bits); sampled: (m, s)
  int pi = INT_MAX;
  switch (md.mode * 2 + int(md.pen_on)) {
    case 0: pass1<T, kModeGreedy, false>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
    case 1: pass1<T, kModeGreedy, true>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
    case 2: pass1<T, kModeSampleF32, false>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
    case 3: pass1<T, kModeSampleF32, true>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
    case 4: pass1<T, kModeSampleRounded, false>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
    default: pass1<T, kModeSampleRounded, true>(lrow, lo, hi, c0, a.vec_ok, bitmap, md, pa, pb, pi); break;
  }
  // Warp reduction (lanes hold increasing, interleaved indices: ties go to the smaller index).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a2 = __shfl_xor_sync(0xffffffffu, pa, o);
    const float b2 = __shfl_xor_sync(0xffffffffu, pb, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, pi, o);
    if (greedy) merge_max(pa, pi, a2, i2);
    else merge_lse(pa, pb, a2, b2);
  }
  float2* rp = a.partials + (int64_t(row) * a.nsplit) * kWarps;
  if (lane == 0) {
    rp[split * kWarps + warp] = make_float2(pa, greedy ? __int_as_float(pi) : pb);
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_flag = atomicAdd(a.tickets + row, 1u) == unsigned(a.nsplit - 1);
  }
  __syncthreads();
  if (!s_flag) return;

  // ---- the last CTA of the row: merge, draw, rescan ----
  __threadfence();
  if (threadIdx.x == 0) {
    s_rng[0] = __ldcg(a.rng);
    s_rng[1] = __ldcg(a.rng + 1);
  }
  const int np = a.nsplit * kWarps;
  if (greedy) {
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int k = threadIdx.x; k < np; k += kThreads) {
      const float2 p = __ldcg(rp + k);
      merge_max(bv, bi, p.x, __float_as_int(p.y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      merge_max(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
      red_f[warp] = bv;
      red_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kWarps; ++w) merge_max(bv, bi, red_f[w], red_i[w]);
      a.out[row] = bi == INT_MAX ? 0 : bi;
    }
  } else {
    // Global max of the partials.
    float gm = -INFINITY;
    for (int k = threadIdx.x; k < np; k += kThreads) gm = fmaxf(gm, __ldcg(rp + k).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    if (lane == 0) red_f[warp] = gm;
    __syncthreads();
    gm = red_f[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) gm = fmaxf(gm, red_f[w]);
    // Each thread owns a contiguous run of partials; their weights s * 2^(m - gm) in fp64.
    const int pp = (np + kThreads - 1) / kThreads;
    const int k0 = threadIdx.x * pp, k1 = min(k0 + pp, np);
    double wsum = 0.0;
    for (int k = k0; k < k1; ++k) {
      const float2 p = __ldcg(rp + k);
      if (p.x != -INFINITY) wsum += double(p.y) * double(fast_exp2(p.x - gm));
    }
    double total;
    const double before = block_exclusive_scan(wsum, warp_sums, &total);
    const uint4 r = philox4x32_10(make_uint4(unsigned(row), 0u, unsigned(s_rng[1]), unsigned(s_rng[1] >> 32)),
                                  unsigned(s_rng[0]), unsigned(s_rng[0] >> 32));
    const double u = double((uint64_t(r.x) << 21) | (r.y >> 11)) * 0x1p-53;  // [0, 1)
    const double target = u * total;
    // The partial whose interval [before_k, before_k + w_k) holds the target.
    const int owner = block_claimer(gm != -INFINITY && wsum > 0.0, before, target, red_i);
    if (threadIdx.x == owner) {
      double acc = before;
      int kk = -1;
      double rest = INFINITY;  // past the run's last weight (rounding): its last token
      for (int k = k0; k < k1; ++k) {
        const float2 p = __ldcg(rp + k);
        if (p.x == -INFINITY || p.y <= 0.f) continue;
        const double w = double(p.y) * double(fast_exp2(p.x - gm));
        if (w <= 0.0) continue;
        kk = k;
        if (target < acc + w) {
          rest = target - acc;
          break;
        }
        acc += w;
      }
      s_flag = kk;
      s_target = rest;
    }
    __syncthreads();
    const int ks = owner < 0 ? -1 : s_flag;
    if (ks < 0) {  // every logit is -inf: nothing to draw from
      if (threadIdx.x == 0) a.out[row] = 0;
    } else {
      // Rescan sub-chunk ks in vocabulary order: each thread a contiguous run of groups.
      const int64_t rlo = int64_t(ks / kWarps) * a.chunk + int64_t(ks % kWarps) * sub;
      const int64_t rhi = min(rlo + sub, min(int64_t(ks / kWarps) * a.chunk + a.chunk, a.vocab));
      if (md.pen_on) build_bitmap(a, row, rlo, rhi - rlo, bitmap);
      const int64_t len = rhi - rlo;
      const int64_t per = ((len + int64_t(kThreads) * VE - 1) / (int64_t(kThreads) * VE)) * VE;
      const int64_t t0 = rlo + threadIdx.x * per, t1 = min(t0 + per, rhi);
      double local = 0.0;
      for (int64_t i = t0; i < t1; i += VE) {
        float v[VE];
        const int n = load_group<T>(lrow, i, t1, a.vec_ok, v);
        const uint32_t bits = md.pen_on ? presence_bits(bitmap, i - rlo, VE) : 0u;
#pragma unroll
        for (int e = 0; e < VE; ++e)
          if (e < n) local += double(weight<T>(md.pen_on ? penalize<true>(v[e], bits, e, md.pen) : v[e], md, gm));
      }
      double rtotal;
      const double rbefore = block_exclusive_scan(local, warp_sums, &rtotal);
      const double tt = s_target;
      const int rowner = block_claimer(local > 0.0, rbefore, tt, red_i);
      if (threadIdx.x == rowner) {
        double acc = rbefore;
        int pick = -1;
        for (int64_t i = t0; i < t1 && !(pick >= 0 && tt < acc); i += VE) {
          float v[VE];
          const int n = load_group<T>(lrow, i, t1, a.vec_ok, v);
          const uint32_t bits = md.pen_on ? presence_bits(bitmap, i - rlo, VE) : 0u;
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            if (e >= n || (pick >= 0 && tt < acc)) continue;
            const float ev = weight<T>(md.pen_on ? penalize<true>(v[e], bits, e, md.pen) : v[e], md, gm);
            if (ev > 0.f) {
              acc += double(ev);
              pick = int(i + e);  // the first token whose cumulative weight passes tt, else the last
            }
          }
        }
        a.out[row] = pick;
      } else if (rowner < 0 && threadIdx.x == 0) {
        a.out[row] = rlo;  // unreachable while the partial had weight; keeps the output defined
      }
    }
  }
  if (threadIdx.x == 0) {
    a.tickets[row] = 0u;
    __threadfence();
    if (atomicAdd(a.tickets + a.num_rows, 1u) == unsigned(a.num_rows - 1)) {
      a.rng[1] = s_rng[1] + 1ull;
      a.tickets[a.num_rows] = 0u;
    }
  }
}

struct SamplePlan {
  int chunk, nsplit;
};

// Vocabulary chunks per row: about four CTAs per SM over the batch, at most 24 per row (each
// chunk re-reads the row's token table), at least what the shared-memory bitmap allows.
// Measured on B200 (151,936-token rows): 256 rows best at 5 chunks, 64 at 9-10, 8 at 20-40.
SamplePlan plan_sample(int num_rows, int64_t vocab, int num_sms) {
  const int64_t nmin = (vocab + kMaxChunk - 1) / kMaxChunk, nmax = (vocab + kMinChunk - 1) / kMinChunk;
  int64_t n = (int64_t(num_sms) * 4 + num_rows - 1) / num_rows;
  n = std::min<int64_t>(std::min<int64_t>(n, 24), nmax);
  n = std::max(n, nmin);
  const int64_t chunk = std::max<int64_t>(((vocab + n - 1) / n + 255) / 256 * 256, kMinChunk);
  return SamplePlan{int(chunk), int((vocab + chunk - 1) / chunk)};
}

size_t tickets_bytes(int num_rows) { return (size_t(num_rows + 1) * sizeof(unsigned) + 255) / 256 * 256; }

}  // namespace

size_t sample_workspace_size(int num_rows, int64_t vocab) {
  const int64_t max_splits = (vocab + kMinChunk - 1) / kMinChunk;
  return tickets_bytes(num_rows) + size_t(num_rows) * size_t(max_splits) * kWarps * sizeof(float2);
}

cudaError_t launch_sample(const void* logits, int64_t row_stride, int num_rows, int64_t vocab, int dtype,
                          const float* temps, const float* pens, const int64_t* table, int64_t table_stride,
                          int64_t table_len, unsigned long long* rng, int64_t* out, void* workspace,
                          cudaStream_t stream) {
  const SamplePlan plan = plan_sample(num_rows, vocab, device_sm_count());
  SampleArgs a;
  a.logits = logits;
  a.row_stride = row_stride;
  a.vocab = vocab;
  a.num_rows = num_rows;
  a.temps = temps;
  a.pens = pens;
  a.table = table;
  a.table_stride = table_stride;
  a.table_len = table_len;
  a.rng = rng;
  a.out = out;
  a.tickets = static_cast<unsigned*>(workspace);
  a.partials = reinterpret_cast<float2*>(static_cast<char*>(workspace) + tickets_bytes(num_rows));
  a.chunk = plan.chunk;
  a.nsplit = plan.nsplit;
  const int es = dtype == FVB_DTYPE_F32 ? 4 : 2;
  a.vec_ok = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (row_stride * es) % 16 == 0;
  const unsigned grid = unsigned(int64_t(num_rows) * plan.nsplit);
  switch (dtype) {
    case FVB_DTYPE_F32: sample_kernel<float><<<grid, kThreads, 0, stream>>>(a); break;
    case FVB_DTYPE_BF16: sample_kernel<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(a); break;
    default: sample_kernel<__half><<<grid, kThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace fvb
