// Next-token sampling over a batch of logit rows in one pass over the logits:
// presence penalty, greedy argmax and temperature sampling.
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
// Two launches.  sample_partials_kernel streams the logits once: one wave of CTAs, each owning
// an equal span of the batch (one or more row parts); each of a CTA's 8 warps folds a
// contiguous run of a part into one partial per 2048 columns, (max, first index) for greedy
// rows or (m, s) with s = sum 2^(x2 - m) in the log2 domain for sampled rows.  No CTA-wide
// barrier on that path (only around the presence bitmap of penalised rows, whose words the
// warps also store for the finish kernel).  sample_finish_kernel, one CTA per row and launched
// as a programmatic dependent of the first, merges the row's partials, draws the Philox uniform,
// finds the 2048-column run holding it and rescans only that run for the exact token.  The
// partials kernel's first thread copies the RNG key and offset into the workspace for the finish
// kernel and advances the offset, so a CUDA-graph replay draws fresh numbers.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMinPart = 2048;     // columns of the smallest CTA span
constexpr int kMaxPart = 131072;   // presence bitmap of one part: kMaxPart / 32 words of shared memory
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
  float2* partials;   // [row][part slot < maxparts][warp][sub-run < maxsub]
  uint32_t* presence; // [row][vocab / 32]: presence bitmaps of penalised rows, for the finish kernel
  unsigned* ctl;      // {unused (zero), batch-wide penalty flag, -, -, this launch's Philox key and offset}
  int64_t vp, per;    // row length rounded up to 256; columns per CTA
  int maxparts, maxsub;  // part slots per row; partials per warp run
  int64_t pwords;        // presence words per row: ceil(vocab / 32)
  bool vec_ok;
};

// How a row is treated (uniform over a CTA).
enum { kModeGreedy = 0, kModeSampleF32 = 1, kModeSampleRounded = 2 };
struct RowMode {
  int mode;
  bool pen_on;
  float pen, t, inv_t, c;  // c = log2(e) / T
  float kpen;              // 2^(-pen * c) - 1: weight change of a penalised token (sampled rows)
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

// Columns per partial: each warp reports one partial per 2048 columns of its run, so the finish
// kernel rescans at most 2048 logits (one 16-byte vector a thread) to place the draw.
constexpr int kSubCols = 2048;

// A lane's running state over one sub-run.  Greedy: max and the first column holding it.  Sampled:
// (m, s) meaning s * 2^m in the log2 domain, s in four independent sums plus `accp`, the part of s
// from penalised tokens.
struct Lane {
  float pa, accp;
  float acc[4];
  int pbase;
};

__device__ __forceinline__ void lane_reset(Lane& st) {
  st.pa = -INFINITY;
  st.accp = 0.f;
  st.acc[0] = st.acc[1] = st.acc[2] = st.acc[3] = 0.f;
  st.pbase = -1;
}

// Folds one 16-byte vector (columns i..i+VE-1; entries past the range are -inf) into a lane.  The
// row's treatment (MODE, PEN) is a template parameter: each warp run calls the loop built for its
// row, so the per-vector code carries no mode tests.  Greedy rows penalise every element.  Sampled
// rows on the fp32 path weigh the raw logits and sum the weights of penalised tokens apart:
// 2^((l - p) c - m) = 2^(l c - m) * 2^(-p c), so the penalty becomes one factor per partial.
// Sampled rows rescale lazily: m moves only when a vector's maximum passes it by more than 8
// (weights stay below 2^8; a negative penalty lifts penalised weights by 2^(|p| c) on top).
template <typename T, int MODE, bool PEN>
__device__ __forceinline__ void consume(float* x, uint32_t bits, int i, const RowMode& md, Lane& st) {
  constexpr int VE = 16 / sizeof(T);
  if constexpr (MODE == kModeGreedy) {
    if constexpr (PEN) {
#pragma unroll
      for (int e = 0; e < VE; ++e) x[e] = penalize<true>(x[e], bits, e, md.pen);
    }
    const float g = tree_max<VE>(x);
    if (g > st.pa) {  // strictly: an earlier vector keeps a tie; -inf never wins
      int k = i + VE - 1;
#pragma unroll
      for (int e = VE - 2; e >= 0; --e)
        if (x[e] == g) k = i + e;
      st.pa = g;
      st.pbase = k;  // the first column holding the new maximum
    }
  } else {
    float scale = md.c;
    if constexpr (MODE == kModeSampleRounded) {
#pragma unroll
      for (int e = 0; e < VE; ++e) x[e] = rounded_quotient<T>(x[e], md);
      scale = kLog2e;
    }
    const float gy = tree_max<VE>(x) * scale;  // scale > 0: the max commutes with it
    if (gy > st.pa + 8.f) {
      const float f = ex2(st.pa - gy);  // 0 while pa is -inf
#pragma unroll
      for (int q = 0; q < 4; ++q) st.acc[q] *= f;
      st.accp *= f;
      st.pa = gy;
    }
    if (st.pa == -INFINITY) return;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const float w = ex2(fmaf(x[e], scale, -st.pa));
      st.acc[e & 3] += w;
      if constexpr (PEN) {
        if (bits & (1u << e)) st.accp += w;
      }
    }
  }
}

// Reduces the warp's lanes to one partial and writes it (lane 0): greedy (value, first index);
// sampled (m, s) with the penalty factor applied.
template <int MODE, bool PEN>
__device__ __forceinline__ void emit(const Lane& st, const RowMode& md, float2* dst) {
  constexpr bool greedy = MODE == kModeGreedy;
  float pa = st.pa, pb = 0.f;
  int pi = INT_MAX;
  if constexpr (greedy) {
    pi = st.pbase >= 0 ? st.pbase : INT_MAX;
  } else {
    pb = (st.acc[0] + st.acc[1]) + (st.acc[2] + st.acc[3]);
    if constexpr (PEN) pb = fmaxf(0.f, fmaf(md.kpen, st.accp, pb));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a2 = __shfl_xor_sync(0xffffffffu, pa, o);
    if constexpr (greedy) {
      merge_max(pa, pi, a2, __shfl_xor_sync(0xffffffffu, pi, o));
    } else {
      merge_lse(pa, pb, a2, __shfl_xor_sync(0xffffffffu, pb, o));
    }
  }
  if ((threadIdx.x & 31) == 0) *dst = make_float2(pa, greedy ? __int_as_float(pi) : pb);
}

// One warp's run [lo, hi) of a row, one partial per kSubCols columns (maxsub partials written,
// empty ones neutral).  Warp-uniform loop with U 16-byte loads in flight per lane; a countdown
// marks the partial boundaries.  Column indices are 32-bit (vocab < 2^31).  When the row is not
// 16-byte aligned (vec_ok false) every load goes through the bounded scalar path.
template <typename T, int MODE, bool PEN>
__device__ __forceinline__ void pass1(const T* lrow, int lo, int hi, int c0, bool vec_ok, const uint32_t* bitmap,
                                      const RowMode& md, float2* dst, int maxsub) {
  constexpr int VE = 16 / sizeof(T), U = 4, STEP = 32 * VE, IT = U * STEP;
  static_assert(kSubCols % IT == 0, "sub-runs are whole iterations");
  const int lane = threadIdx.x & 31;
  Lane st;
  lane_reset(st);
  int sub = 0, emitted = lo;  // partials written; columns covered by them end at `emitted`
  int ib = lo;                // warp-uniform column of the current iteration
  if (vec_ok) {
    int left = kSubCols;
    for (; ib + IT <= hi; ib += IT) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = ldg_nc_v4(lrow + ib + u * STEP + lane * VE);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = ib + u * STEP + lane * VE;
        float x[VE];
        unpack16<T>(raw[u], x);
        const uint32_t bits = PEN ? presence_bits(bitmap, i - c0, VE) : 0u;
        consume<T, MODE, PEN>(x, bits, i, md, st);
      }
      left -= IT;
      if (left == 0) {
        emit<MODE, PEN>(st, md, dst + sub);
        ++sub;
        emitted = ib + IT;
        left = kSubCols;
        lane_reset(st);
      }
    }
  }
  // The rest, one vector per lane at a time with bounds.
  for (; ib < hi; ib += STEP) {
    if (ib > emitted && (ib - lo) % kSubCols == 0 && sub < maxsub) {
      emit<MODE, PEN>(st, md, dst + sub);
      ++sub;
      emitted = ib;
      lane_reset(st);
    }
    const int i = ib + lane * VE;
    float x[VE];
    if (i < hi) {
      load_group<T>(lrow, i, hi, vec_ok, x);
    } else {
#pragma unroll
      for (int e = 0; e < VE; ++e) x[e] = -INFINITY;
    }
    const uint32_t bits = PEN && i < hi ? presence_bits(bitmap, i - c0, VE) : 0u;
    consume<T, MODE, PEN>(x, bits, i, md, st);
  }
  if (hi > emitted && sub < maxsub) {  // the last, partial sub-run
    emit<MODE, PEN>(st, md, dst + sub);
    ++sub;
  }
  if (lane == 0)
    for (; sub < maxsub; ++sub)
      dst[sub] = MODE == kModeGreedy ? make_float2(-INFINITY, __int_as_float(INT_MAX)) : make_float2(-INFINITY, 0.f);
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

// ---------------------------------------------------------------------------
// Launch geometry.  The batch is laid out as rows of vp = vocab rounded up to 256 entries (the
// padding is never read) and CTA c owns the span [c * per, (c + 1) * per) of that layout: one
// or more row parts of equal total length, so the CTAs of the single wave finish together.  A
// row's parts are numbered by slot (vocabulary order); each part's 8 warps take equal runs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t first_cta(int64_t r, const SampleArgs& a) { return r * a.vp / a.per; }
__device__ __forceinline__ int parts_of_row(int64_t r, const SampleArgs& a) {
  return int((r * a.vp + a.vp - 1) / a.per - first_cta(r, a) + 1);
}
// Columns [lo, hi) of part `slot` of row r, hi capped at the vocabulary (empty for padding).
__device__ __forceinline__ void part_cols(const SampleArgs& a, int64_t r, int slot, int64_t& lo, int64_t& hi) {
  const int64_t c = first_cta(r, a) + slot, rs = r * a.vp;
  lo = max(c * a.per, rs) - rs;
  hi = max(lo, min(min((c + 1) * a.per, rs + a.vp) - rs, a.vocab));
}
// Warp w's run of a part: multiples of 32 columns, so 16-byte vectors stay aligned.
__device__ __forceinline__ void warp_cols(int64_t lo, int64_t hi, int w, int64_t& wlo, int64_t& whi) {
  const int64_t sub = (hi - lo + 32 * kWarps - 1) / (32 * kWarps) * 32;
  wlo = min(lo + w * sub, hi);
  whi = min(wlo + sub, hi);
}

template <typename T>
__device__ __forceinline__ RowMode row_mode(const SampleArgs& a, float t, float pen, int anyp) {
  RowMode md;
  const bool greedy = t < kGreedyBelow;
  md.pen = anyp ? pen : 0.f;
  md.pen_on = anyp && md.pen != 0.f && a.table_len > 0;
  md.mode = greedy ? kModeGreedy
                   : (!anyp && Elem<T>::kDtype != FVB_DTYPE_F32 ? kModeSampleRounded : kModeSampleF32);
  md.t = greedy ? 1.f : t;
  md.inv_t = greedy ? 1.f : 1.f / t;
  md.c = md.inv_t * kLog2e;
  md.kpen = md.pen_on && !greedy ? ex2(-md.pen * md.c) - 1.f : 0.f;
  return md;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 4) sample_partials_kernel(SampleArgs a) {
  __shared__ uint32_t bitmap[kMaxPart / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t total = int64_t(a.num_rows) * a.vp;
  const int64_t f0 = int64_t(blockIdx.x) * a.per, f1 = min(f0 + a.per, total);
  // Batch-wide penalty switch, as the reference decides it from all rows' parameters, and the
  // parameters of this CTA's rows (at most kThreads of them cached) in the same round trip.
  __shared__ float s_temp[kThreads], s_pen[kThreads];
  const int64_t row0 = f0 / a.vp;
  const int nrows = f1 > f0 ? int((f1 - 1) / a.vp - row0 + 1) : 0;
  if (threadIdx.x < nrows) {
    s_temp[threadIdx.x] = __ldg(a.temps + row0 + threadIdx.x);
    s_pen[threadIdx.x] = a.pens != nullptr ? __ldg(a.pens + row0 + threadIdx.x) : 0.f;
  }
  int anyp = 0;
  if (a.pens != nullptr)
    for (int r = threadIdx.x; r < a.num_rows; r += kThreads) anyp |= fabsf(__ldg(a.pens + r)) > kPenaltyAbove;
  anyp = __syncthreads_or(anyp);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    a.ctl[1] = unsigned(anyp);
    // This launch's Philox key and counter offset, handed to the finish kernel, and the offset
    // advanced for the next launch (the finish kernel reads only the copy).
    const unsigned long long seed = __ldcg(a.rng), off = __ldcg(a.rng + 1);
    *reinterpret_cast<ulonglong2*>(a.ctl + 4) = make_ulonglong2(seed, off);
    a.rng[1] = off + 1ull;
  }
  for (int64_t f = f0; f < f1;) {
    const int64_t row = f / a.vp, fe = min(f1, (row + 1) * a.vp);
    const int64_t lo = f - row * a.vp, hi = max(lo, min(fe - row * a.vp, a.vocab));
    const int slot = int(blockIdx.x - first_cta(row, a));
    const int rr = int(row - row0);
    const RowMode md = rr < kThreads ? row_mode<T>(a, s_temp[rr], s_pen[rr], anyp)
                                     : row_mode<T>(a, __ldg(a.temps + row), a.pens ? __ldg(a.pens + row) : 0.f, anyp);
    if (md.pen_on) {
      __syncthreads();  // every warp is done with the previous part's bitmap
      build_bitmap(a, int(row), lo, hi - lo, bitmap);
    }
    const T* lrow = static_cast<const T*>(a.logits) + row * a.row_stride;
    int64_t wlo, whi;
    warp_cols(lo, hi, warp, wlo, whi);
    float2* dst = a.partials + ((row * a.maxparts + slot) * kWarps + warp) * a.maxsub;
    const int wl = int(wlo), wh = int(whi), c0 = int(lo);
    switch (md.mode * 2 + int(md.pen_on)) {  // pen_on implies the fp32 path for sampled rows
      case 0: pass1<T, kModeGreedy, false>(lrow, wl, wh, c0, a.vec_ok, bitmap, md, dst, a.maxsub); break;
      case 1: pass1<T, kModeGreedy, true>(lrow, wl, wh, c0, a.vec_ok, bitmap, md, dst, a.maxsub); break;
      case 2: pass1<T, kModeSampleF32, false>(lrow, wl, wh, c0, a.vec_ok, bitmap, md, dst, a.maxsub); break;
      case 3: pass1<T, kModeSampleF32, true>(lrow, wl, wh, c0, a.vec_ok, bitmap, md, dst, a.maxsub); break;
      default: pass1<T, kModeSampleRounded, false>(lrow, wl, wh, c0, a.vec_ok, bitmap, md, dst, a.maxsub); break;
    }
    if (md.pen_on) {  // this warp's run of the bitmap, for the finish kernel's rescan
      uint32_t* dst = a.presence + row * a.pwords;
      for (int64_t w = wlo / 32 + lane; w < (whi + 31) / 32; w += 32) dst[w] = bitmap[w - lo / 32];
    }
    f = fe;
  }
}

struct Shared {
  double warp_sums[kWarps];
  float red_f[kWarps];
  int red_i[kWarps];
  int flag;
  double target;
};

// One CTA per row: merge the row's partials; greedy rows take the maximum, sampled rows draw.
template <typename T>
__global__ void __launch_bounds__(kThreads) sample_finish_kernel(SampleArgs a) {
  constexpr int VE = 16 / sizeof(T);
  __shared__ uint32_t bitmap[kSubCols / 32];
  __shared__ Shared sm;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = blockIdx.x;
  const T* lrow = static_cast<const T*>(a.logits) + int64_t(row) * a.row_stride;
  const float t_row = __ldg(a.temps + row), p_row = a.pens != nullptr ? __ldg(a.pens + row) : 0.f;
  // Launched as a programmatic dependent of sample_partials_kernel: everything above overlaps its
  // tail; after the wait its partials, flag, key copy and presence words are complete and visible.
  const float2* rp = a.partials + int64_t(row) * a.maxparts * kWarps * a.maxsub;
  const int np = parts_of_row(row, a) * kWarps * a.maxsub;
  constexpr int kRun = 4;
  const int pp = (np + kThreads - 1) / kThreads;
  const int k0 = min(int(threadIdx.x) * pp, np), k1 = min(k0 + pp, np);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The flag, the key and (sampled rows) the first partials in one round trip.
  const unsigned anyp_u = __ldcg(a.ctl + 1);
  const ulonglong2 key = __ldcg(reinterpret_cast<const ulonglong2*>(a.ctl + 4));
  float2 run[kRun];
  if (t_row >= kGreedyBelow) {
#pragma unroll
    for (int j = 0; j < kRun; ++j) run[j] = k0 + j < k1 ? __ldcg(rp + k0 + j) : make_float2(-INFINITY, 0.f);
  }
  const RowMode md = row_mode<T>(a, t_row, p_row, int(anyp_u));
  if (md.mode == kModeGreedy) {
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
      sm.red_f[warp] = bv;
      sm.red_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kWarps; ++w) merge_max(bv, bi, sm.red_f[w], sm.red_i[w]);
      a.out[row] = bi == INT_MAX ? 0 : bi;
    }
  } else {
    // Each thread a contiguous run of partials (the first kRun loaded above).
    float gm = -INFINITY;
#pragma unroll
    for (int j = 0; j < kRun; ++j) gm = fmaxf(gm, run[j].x);
    for (int k = k0 + kRun; k < k1; ++k) gm = fmaxf(gm, __ldcg(rp + k).x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    if (lane == 0) sm.red_f[warp] = gm;
    __syncthreads();
    gm = sm.red_f[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) gm = fmaxf(gm, sm.red_f[w]);
    auto pweight = [&](float2 p) {
      return p.x == -INFINITY || p.y <= 0.f ? 0.0 : double(p.y) * double(ex2(p.x - gm));
    };
    double wsum = 0.0;
#pragma unroll
    for (int j = 0; j < kRun; ++j) wsum += pweight(run[j]);
    for (int k = k0 + kRun; k < k1; ++k) wsum += pweight(__ldcg(rp + k));
    double total;
    const double before = block_exclusive_scan(wsum, sm.warp_sums, &total);
    const uint4 r = philox4x32_10(make_uint4(unsigned(row), 0u, unsigned(key.y), unsigned(key.y >> 32)),
                                  unsigned(key.x), unsigned(key.x >> 32));
    const double u = double((uint64_t(r.x) << 21) | (r.y >> 11)) * 0x1p-53;  // [0, 1)
    const double target = u * total;
    // The partial whose interval [before_k, before_k + w_k) holds the target.
    const int owner = block_claimer(gm != -INFINITY && wsum > 0.0, before, target, sm.red_i);
    if (threadIdx.x == owner) {
      double acc = before;
      int kk = -1;
      double rest = INFINITY;  // past the run's last weight (rounding): its last token
      bool done = false;
      auto step = [&](int k, float2 pk) {
        const double w = pweight(pk);
        if (done || w <= 0.0) return;
        kk = k;
        if (target < acc + w) {
          rest = target - acc;
          done = true;
        } else {
          acc += w;
        }
      };
#pragma unroll
      for (int j = 0; j < kRun; ++j)
        if (k0 + j < k1) step(k0 + j, run[j]);
      for (int k = k0 + kRun; k < k1 && !done; ++k) step(k, __ldcg(rp + k));
      sm.flag = kk;
      sm.target = rest;
    }
    __syncthreads();
    const int ks = owner < 0 ? -1 : sm.flag;
    if (ks < 0) {  // every logit is -inf: nothing to draw from
      if (threadIdx.x == 0) a.out[row] = 0;
    } else {
      // Rescan run ks in vocabulary order: each thread a contiguous stretch of kPer columns whose
      // weights stay in registers; the logits and the presence words are fetched in one round trip.
      constexpr int kPer = kSubCols / kThreads;
      static_assert(kPer == 8 && kPer % VE == 0, "a stretch is whole 16-byte groups within one word");
      int64_t plo, phi, wlo, whi;
      part_cols(a, row, ks / (kWarps * a.maxsub), plo, phi);
      warp_cols(plo, phi, (ks / a.maxsub) % kWarps, wlo, whi);
      const int64_t rlo = min(wlo + int64_t(ks % a.maxsub) * kSubCols, whi), rhi = min(rlo + kSubCols, whi);
      const int64_t t0 = min(rlo + int64_t(threadIdx.x) * kPer, rhi), t1 = min(t0 + kPer, rhi);
      float v[kPer];
#pragma unroll
      for (int g = 0; g < kPer / VE; ++g) load_group<T>(lrow, t0 + g * VE, t1, a.vec_ok, v + g * VE);
      if (md.pen_on) {  // the run's presence bits, as the partials kernel stored them
        for (int64_t w = rlo / 32 + threadIdx.x; w < (rhi + 31) / 32; w += kThreads)
          bitmap[w - rlo / 32] = __ldcg(a.presence + int64_t(row) * a.pwords + w);
        __syncthreads();
      }
      const uint32_t bits = md.pen_on && t0 < t1 ? presence_bits(bitmap, t0 - rlo, kPer) : 0u;
      float w[kPer];
      double local = 0.0;
#pragma unroll
      for (int e = 0; e < kPer; ++e) {
        w[e] = t0 + e < t1 ? weight<T>(md.pen_on ? penalize<true>(v[e], bits, e, md.pen) : v[e], md, gm) : 0.f;
        local += double(w[e]);
      }
      double rtotal;
      const double rbefore = block_exclusive_scan(local, sm.warp_sums, &rtotal);
      const double tt = sm.target;
      const int rowner = block_claimer(local > 0.0, rbefore, tt, sm.red_i);
      if (rowner < 0) {
        if (threadIdx.x == 0) a.out[row] = rlo;  // unreachable while the partial had weight
      } else if (threadIdx.x == rowner) {
        // The first column whose cumulative weight passes tt; rounding past the stretch's own
        // total leaves the last column with weight.
        double acc = rbefore;
        int64_t pick = t0;
        bool done = false;
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          if (done || w[e] <= 0.f) continue;
          acc += double(w[e]);
          pick = t0 + e;
          done = tt < acc;
        }
        a.out[row] = pick;
      }
    }
  }
}

// One wave of resident CTAs (4 per SM) over the whole batch, each span at least 2048 columns and
// twice the token-table length (every part re-reads its row's table), at most kMaxPart columns.
struct SamplePlan {
  int64_t vp, per;
  unsigned grid;
};

SamplePlan plan_sample(int num_rows, int64_t vocab, int64_t table_len, int num_sms) {
  const int64_t vp = (vocab + 255) / 256 * 256, total = int64_t(num_rows) * vp;
  int64_t per = (total + int64_t(num_sms) * 4 - 1) / (int64_t(num_sms) * 4);
  per = std::max<int64_t>(per, std::max<int64_t>(kMinPart, 2 * table_len));
  per = std::min<int64_t>((per + 255) / 256 * 256, kMaxPart);
  return SamplePlan{vp, per, unsigned((total + per - 1) / per)};
}

int max_parts(int64_t vocab) { return int(((vocab + 255) / 256 * 256 + kMinPart - 1) / kMinPart + 2); }
// Sub-run partials per warp run: runs are at most ceil(per / 256) * 32 columns.
int max_sub(int64_t per) { return int(((per + 255) / 256 * 32 + kSubCols - 1) / kSubCols); }
constexpr int kMaxSub = (kMaxPart / 256 * 32 + kSubCols - 1) / kSubCols;  // for per = kMaxPart

constexpr size_t kCtlBytes = 256;  // {grid ticket, penalty flag}, padded
size_t partials_bytes(int num_rows, int64_t vocab) {
  return (size_t(num_rows) * size_t(max_parts(vocab)) * kWarps * kMaxSub * sizeof(float2) + 255) / 256 * 256;
}

// The partials kernel, then the finish kernel as its programmatic dependent (its launch and row
// parameters overlap the partials kernel's tail; griddepcontrol.wait orders the rest).
template <typename T>
cudaError_t launch_pair(const SampleArgs& a, unsigned grid, int num_rows, cudaStream_t stream) {
  sample_partials_kernel<T><<<grid, kThreads, 0, stream>>>(a);
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return ce;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(num_rows));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sample_finish_kernel<T>, a);
}

}  // namespace

size_t sample_workspace_size(int num_rows, int64_t vocab) {
  return kCtlBytes + partials_bytes(num_rows, vocab) + size_t(num_rows) * size_t((vocab + 31) / 32) * 4;
}

cudaError_t launch_sample(const void* logits, int64_t row_stride, int num_rows, int64_t vocab, int dtype,
                          const float* temps, const float* pens, const int64_t* table, int64_t table_stride,
                          int64_t table_len, unsigned long long* rng, int64_t* out, void* workspace,
                          cudaStream_t stream) {
  const SamplePlan plan = plan_sample(num_rows, vocab, table_len, device_sm_count());
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
  a.ctl = static_cast<unsigned*>(workspace);
  a.partials = reinterpret_cast<float2*>(static_cast<char*>(workspace) + kCtlBytes);
  a.presence = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + kCtlBytes + partials_bytes(num_rows, vocab));
  a.pwords = (vocab + 31) / 32;
  a.vp = plan.vp;
  a.per = plan.per;
  a.maxparts = max_parts(vocab);
  a.maxsub = max_sub(plan.per);
  const int es = dtype == FVB_DTYPE_F32 ? 4 : 2;
  a.vec_ok = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (row_stride * es) % 16 == 0;
  switch (dtype) {
    case FVB_DTYPE_F32: return launch_pair<float>(a, plan.grid, num_rows, stream);
    case FVB_DTYPE_BF16: return launch_pair<__nv_bfloat16>(a, plan.grid, num_rows, stream);
    default: return launch_pair<__half>(a, plan.grid, num_rows, stream);
  }
}

}  // namespace fvb
