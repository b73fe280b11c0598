// Fused q/k RMSNorm + rotary embedding + KV-cache write, one pass over the
// projection outputs.
//
// Replaces, per attention layer, the reference's
//   q = q_norm(q); k = k_norm(k)                         (qwen3.py:234-235, nn.RMSNorm over d_head)
//   q = rotary_embd(q, positions); k = rotary_embd(k, positions)   (qwen3.py:237-238, :53-138)
//   the Python KV-write loops                            (qwen3.py:240-264 decode, 322-366 prefill)
//   q.transpose(0, 1) + .contiguous() at the op boundary (qwen3.py:270, femtovllm/ops/__init__.py:41-42)
// which read and write Q and K three times and launch one copy per sequence
// (decode) or per block run (prefill).  Here every (token, head) row is read
// once and written once:
//   q_out[h][t][:] = rope(rmsnorm(q[t][h][:]) * q_w)                  (head-major, as the
//                                                                       attention entry points take it)
//   k_pool[slot / P][h][slot % P][:] = rope(rmsnorm(k[t][h][:]) * k_w)
//   v_pool[slot / P][h][slot % P][:] = v[t][h][:]                      (bit-exact copy)
// with rmsnorm(x) = x / sqrt(mean(x^2) + eps) and
// rope(y)[d] = y[d] cos[pos][d] + (d < D/2 ? -y[d + D/2] : y[d - D/2]) sin[pos][d]
// (the reference's cos * x + sin * cat(-y2, y1), qwen3.py:103-138), cos / sin
// being the caller's tables of shape [rope_rows][D] (the rotary module's
// buffers).  Arithmetic is fp32 from the loaded values to the single rounding
// of the result.
//
// Layout: a row is D contiguous elements = D * sizeof(T) / 16 lanes.  Lane
// `sub` holds 8 bytes of the lower half of the row (dims sub*E/2 ...) and the
// matching 8 bytes of the upper half (dims D/2 + sub*E/2 ...), so each rotary
// pair (d, d + D/2) sits in one thread and needs no shuffle; only the row's
// sum of squares is reduced over the lanes by xor shuffles.  (One 16-byte
// vector per lane with the partner a shuffle away measured ~10 % slower.)
// Row loads and stores stay coalesced: the lanes of a row cover each half's
// bytes contiguously.  HBM-bound:
// (Hq + 2 Hkv) D sizeof(T) bytes read and written per token, plus 12 bytes
// of position / slot and the cos / sin rows (L2-resident).  The arithmetic is
// in packed fp32x2 (FFMA2 / FMUL2) to keep the issue rate below the memory rate.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* in);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* in) {
  return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]), __float_as_uint(in[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* in) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* in) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// Rotary pairs in one thread: 8 bytes from the lower half of a row and the matching 8 bytes of the
// upper half, as one uint4 (.x .y lower, .z .w upper).
template <typename T, int D>
__device__ __forceinline__ uint4 ldg_pair(const T* row, int sub) {
  constexpr int H = 8 / int(sizeof(T));
  const uint2 lo = __ldg(reinterpret_cast<const uint2*>(row + sub * H));
  const uint2 hi = __ldg(reinterpret_cast<const uint2*>(row + D / 2 + sub * H));
  return make_uint4(lo.x, lo.y, hi.x, hi.y);
}
template <typename T, int D>
__device__ __forceinline__ void st_pair(T* row, int sub, const uint4& v) {
  constexpr int H = 8 / int(sizeof(T));
  *reinterpret_cast<uint2*>(row + sub * H) = make_uint2(v.x, v.y);
  *reinterpret_cast<uint2*>(row + D / 2 + sub * H) = make_uint2(v.z, v.w);
}

constexpr int kThreads = 192;         // q / k rows
constexpr int kVThreads = 32;         // one warp copying the value rows with bulk copies
constexpr int kAllThreads = kThreads + kVThreads;
constexpr int kCtasPerSm = 4;
constexpr int kVStages = 4;           // value-row stages of the copy warp
constexpr int kVStageMax = 8 * 1024;  // value bytes of one block pass (else the q / k threads copy them)

__device__ __forceinline__ void bulk_s2g_v(void* dst_gmem, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem), "r"(src_smem),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_v() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_reads_v() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_done_v() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Work split.  A block is kThreads q / k threads plus one copy warp.  A row is
// one head of one token; the q / k threads form S = kThreads / L row slots.
// The copy warp moves the value rows (a bit-exact copy) with bulk copies:
// global -> shared (one copy per token when its heads are contiguous) ->
// each row's pool slot, kVStages block passes deep, so those bytes are in
// flight without registers while the q / k threads take only the q and k
// rows: units = Hq + Hkv heads per token (Hq + 2 Hkv when a pass's value rows
// exceed kVStageMax and the q / k threads copy them too).  A block takes
// S / units whole tokens per pass when units <= S (slot j -> token j / units,
// head j % units), otherwise one token per pass with slot j taking heads
// j, j + S, j + 2S, ...  Each thread's heads are fixed for the whole launch,
// so the norm weights are loaded once, position / slot / cos / sin once per
// token, and only the rows themselves per head.  Measured on 65k tokens of
// Hq 16 / Hkv 8 (bf16, D 128): 4.54 TB/s with 256 threads copying every row
// (3 CTAs per SM, 80 registers), 5.01 TB/s with 192 q / k threads + the copy
// warp at 4 CTAs per SM; 3 or 5 CTAs per SM, 128 or 256 q / k threads and 8
// value stages were slower.
// I is the type of every element offset: int when all of the launch's tensors are
// smaller than 2^31 elements (3.3 % faster on 65k tokens of 32 heads), int64_t otherwise.
template <typename T, int D, typename I, bool VT>
__global__ void __launch_bounds__(kAllThreads, kCtasPerSm) qk_norm_rope_store_kernel(
    const T* __restrict__ q, I q_ts, I q_hs, const T* __restrict__ k, I k_ts, I k_hs,
    const T* __restrict__ v, I v_ts, I v_hs, const T* __restrict__ q_w, const T* __restrict__ k_w,
    float eps, const T* __restrict__ cos_t, const T* __restrict__ sin_t, int rope_rows,
    const int32_t* __restrict__ positions, const int64_t* __restrict__ slot_mapping, int num_tokens,
    int n_heads, int n_kv_heads, T* __restrict__ q_out, T* __restrict__ k_pool, T* __restrict__ v_pool,
    int64_t num_slots, int block_size, int block_shift, int* __restrict__ err) {
  constexpr int E = 16 / int(sizeof(T));  // elements per lane
  constexpr int L = D / E;                // lanes per row
  constexpr int HALF = L / 2;             // first xor distance of the row reduction
  constexpr int S = kThreads / L;         // row slots per block
  static_assert(L >= 2 && L <= 32 && 32 % L == 0, "row must tile a warp");
  static_assert(E % 2 == 0, "pairs of elements");
  // VT: value rows go through the copy warp (bulk copies, global -> shared -> pool rows); the
  // q / k threads then take only the Hq + Hkv q and k rows of a token.
  const int units = n_heads + (VT ? 1 : 2) * n_kv_heads;
  const int lane = threadIdx.x & 31;
  const bool packed = units <= S;
  const int tpb = packed ? S / units : 1;  // tokens per block pass
  const int tstride = gridDim.x * tpb;
  if (threadIdx.x >= kThreads) {
    // ======================== value rows: global -> shared -> pool, bulk copies ========================
    if constexpr (VT) {
      extern __shared__ __align__(128) uint8_t vsm[];
      constexpr int ROW = D * int(sizeof(T));
      const int pass_bytes = tpb * n_kv_heads * ROW;
      uint64_t* vbar = reinterpret_cast<uint64_t*>(vsm + kVStages * pass_bytes);
      if (lane == 0) {
        for (int i = 0; i < kVStages; ++i) mbar_init(&vbar[i], 1);
        fence_mbar_init();
      }
      __syncwarp();
      const bool heads_contiguous = v_hs == I(D);
      auto load_pass = [&](int p) {  // lane 0
        const int tb = blockIdx.x * tpb + p * tstride;
        const int nt = min(tpb, num_tokens - tb);
        const int st = p % kVStages;
        mbar_arrive_expect_tx(&vbar[st], uint32_t(nt * n_kv_heads * ROW));
        uint8_t* dst = vsm + st * pass_bytes;
        for (int i = 0; i < nt; ++i) {
          const T* src = v + I(tb + i) * v_ts;
          if (heads_contiguous) {
            bulk_g2s(dst + i * n_kv_heads * ROW, src, uint32_t(n_kv_heads * ROW), &vbar[st]);
          } else {
            for (int h = 0; h < n_kv_heads; ++h)
              bulk_g2s(dst + (i * n_kv_heads + h) * ROW, src + I(h) * v_hs, uint32_t(ROW), &vbar[st]);
          }
        }
      };
      const int npass = blockIdx.x * tpb < num_tokens ? (num_tokens - blockIdx.x * tpb + tstride - 1) / tstride : 0;
      if (lane == 0) {
        for (int p = 0; p < kVStages - 1 && p < npass; ++p) load_pass(p);
      }
      for (int p = 0; p < npass; ++p) {
        // the stage the next load reuses held pass p - 1: every lane's stores of it have read it
        bulk_wait_reads_v();
        __syncwarp();
        if (lane == 0 && p + kVStages - 1 < npass) load_pass(p + kVStages - 1);
        const int st = p % kVStages;
        if (!__all_sync(0xffffffffu, mbar_wait(&vbar[st], uint32_t(p / kVStages) & 1u, err, 0x340))) {
          // give the loads still in flight (passes p + 1 .. p + kVStages - 1) a bounded wait before exiting
          for (int q2 = p + 1; q2 < npass && q2 < p + kVStages; ++q2)
            mbar_wait(&vbar[q2 % kVStages], uint32_t(q2 / kVStages) & 1u, err, 0x341);
          break;
        }
        const int tb = blockIdx.x * tpb + p * tstride;
        const int nt = min(tpb, num_tokens - tb);
        for (int rr = lane; rr < nt * n_kv_heads; rr += 32) {
          const int i = rr / n_kv_heads, h = rr - i * n_kv_heads;
          const int64_t slot = __ldg(slot_mapping + tb + i);
          if (slot < 0 || slot >= num_slots) continue;  // padding, or reported by the q / k threads
          const int64_t blk = block_shift >= 0 ? (slot >> block_shift) : slot / block_size;
          const int off = int(slot - blk * block_size);
          bulk_s2g_v(v_pool + ((I(blk) * n_kv_heads + h) * block_size + off) * I(D),
                     smem_u32(vsm + st * pass_bytes + rr * ROW), uint32_t(ROW));
        }
        bulk_commit_v();
      }
      bulk_wait_done_v();  // no copy of this warp is in flight when it exits
    }
    return;
  }
  const int sub = threadIdx.x % L;
  const int j = threadIdx.x / L;
  if (packed && j >= tpb * units) return;  // spare slot (its whole row group leaves together)
  const int tok_off = packed ? j / units : 0;
  const int u0 = packed ? j % units : j;
  const int ustep = packed ? units : S;  // next head of this slot (one past the end when packed)
  const uint32_t gmask = L == 32 ? 0xffffffffu : (((1u << L) - 1u) << (lane & ~(L - 1)));
  const float inv_d = 1.f / float(D);
  const uint4 wq = ldg_pair<T, D>(q_w, sub), wk = ldg_pair<T, D>(k_w, sub);  // unpacked where used

  // Norm + rope of one q or k row piece held as raw (lower / upper half pairs, row-group
  // uniform).  The weights and the token's cos / sin stay packed until here: fewer live
  // registers let the row loads of both heads issue early (measured ~5 % faster).
  auto norm_rope = [&](const uint4& raw, const uint4& wv, const uint4& cr, const uint4& sr) -> uint4 {
    float c[E], sn[E];
    unpack16<T>(cr, c);
    unpack16<T>(sr, sn);
    float x[E], w[E];
    unpack16<T>(raw, x);
    unpack16<T>(wv, w);
    float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 x2 = make_float2(x[e], x[e + 1]);
      ss2 = __ffma2_rn(x2, x2, ss2);
    }
    float ss = ss2.x + ss2.y;
#pragma unroll
    for (int o = HALF; o >= 1; o >>= 1) ss += __shfl_xor_sync(gmask, ss, o);
    const float inv = rsqrtf(ss * inv_d + eps);
    const float2 inv2 = make_float2(inv, inv);
    float y[E];
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 yy = __fmul2_rn(__fmul2_rn(make_float2(x[e], x[e + 1]), inv2), make_float2(w[e], w[e + 1]));
      y[e] = yy.x;
      y[e + 1] = yy.y;
    }
    // y[e] (e < E/2) is dim d of the lower half and y[e + E/2] dim d + D/2: the partner is local.
    float r[E];
#pragma unroll
    for (int e = 0; e < E / 2; e += 2) {
      const float2 ylo = make_float2(y[e], y[e + 1]), yhi = make_float2(y[e + E / 2], y[e + E / 2 + 1]);
      const float2 lo = __ffma2_rn(ylo, make_float2(c[e], c[e + 1]), __fmul2_rn(yhi, make_float2(-sn[e], -sn[e + 1])));
      const float2 hi = __ffma2_rn(yhi, make_float2(c[e + E / 2], c[e + E / 2 + 1]),
                                   __fmul2_rn(ylo, make_float2(sn[e + E / 2], sn[e + E / 2 + 1])));
      r[e] = lo.x;
      r[e + 1] = lo.y;
      r[e + E / 2] = hi.x;
      r[e + E / 2 + 1] = hi.y;
    }
    return pack16<T>(r);
  };

  auto load_row = [&](int t, int uu) -> uint4 {
    if (uu < n_heads) return ldg_pair<T, D>(q + (I(t) * q_ts + I(uu) * q_hs), sub);
    if (uu < n_heads + n_kv_heads) return ldg_pair<T, D>(k + (I(t) * k_ts + I(uu - n_heads) * k_hs), sub);
    return ldg16(v + (I(t) * v_ts + I(uu - n_heads - n_kv_heads) * v_hs + I(sub * E)));
  };
  int t = blockIdx.x * tpb + tok_off;
  // position and slot of the next token are fetched one token ahead
  int pos_n = t < num_tokens ? __ldg(positions + t) : 0;
  int64_t slot_n = t < num_tokens ? __ldg(slot_mapping + t) : -1;
  for (; t < num_tokens; t += tstride) {
    const int pos = pos_n;
    int64_t slot = slot_n;
    // Rows first (independent of the position), then the position-dependent tables.
    const bool has_b = u0 + ustep < units;
    const uint4 ra = load_row(t, u0);
    const uint4 rb = has_b ? load_row(t, u0 + ustep) : make_uint4(0, 0, 0, 0);
    if (t + tstride < num_tokens) {
      pos_n = __ldg(positions + t + tstride);
      slot_n = __ldg(slot_mapping + t + tstride);
    }
    const bool rope_ok = pos >= 0 && pos < rope_rows;
    uint4 c = make_uint4(0, 0, 0, 0), sn = make_uint4(0, 0, 0, 0);
    if (rope_ok) {
      c = ldg_pair<T, D>(cos_t + I(pos) * D, sub);
      sn = ldg_pair<T, D>(sin_t + I(pos) * D, sub);
    }
    if (slot >= num_slots) {
      if (sub == 0) record_error(err, FVB_ERR_BAD_SLOT, t);
      slot = -1;
    }
    if (!rope_ok && u0 == 0 && sub == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, t);
    const I blk = slot < 0 ? 0 : block_shift >= 0 ? I(slot >> block_shift) : I(slot / block_size);
    const int off = slot >= 0 ? int(slot - int64_t(blk) * block_size) : 0;
    auto finish = [&](int uu, const uint4& raw) {
      if (uu < n_heads) {
        if (rope_ok) st_pair<T, D>(q_out + (I(uu) * num_tokens + t) * D, sub, norm_rope(raw, wq, c, sn));
      } else if (uu < n_heads + n_kv_heads) {
        if (rope_ok && slot >= 0)
          st_pair<T, D>(k_pool + ((blk * n_kv_heads + (uu - n_heads)) * block_size + off) * I(D), sub,
                        norm_rope(raw, wk, c, sn));
      } else if (slot >= 0) {  // value row: bit-exact copy
        *reinterpret_cast<uint4*>(v_pool + (((blk * n_kv_heads + (uu - n_heads - n_kv_heads)) * block_size + off) * I(D) +
                                            I(sub * E))) = raw;
      }
    };
    finish(u0, ra);
    if (has_b) finish(u0 + ustep, rb);
    // Heads beyond two per slot (more than 2 S heads per token), two at a time.
    for (int u = u0 + 2 * ustep; u < units; u += 2 * ustep) {
      const int ub = u + ustep;
      const uint4 xa = load_row(t, u);
      const uint4 xb = ub < units ? load_row(t, ub) : make_uint4(0, 0, 0, 0);
      finish(u, xa);
      if (ub < units) finish(ub, xb);
    }
  }
}

// Rotary pairs of a row staged in shared memory (the split of ldg_pair).
template <typename T, int D>
__device__ __forceinline__ uint4 lds_pair(uint32_t row, int sub) {
  uint32_t a, b, c, d;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(row + sub * 8));
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(c), "=r"(d) : "r"(row + D * int(sizeof(T)) / 2 + sub * 8));
  return make_uint4(a, b, c, d);
}

// Warp-specialised kernel (the default path): small blocks of kWsQkThreads q / k threads plus
// one copy warp, kWsCtasPerSm of them per SM.  The copy warp streams every row of a block
// pass (the q, k and v rows of its tokens) into a kWsStages-deep shared-memory ring with
// bulk copies (one per tensor and token when its heads are contiguous); the q / k threads
// wait on the pass's full barrier, compute from shared memory and release the stage (one
// arrival per warp); the copy warp stores the value rows from the stage to their pool
// slots.  No register holds a row in flight and no block-wide barrier orders the passes,
// so each SM keeps 8 x 3 passes of rows (192 KB at 32 heads x 256 bytes) streaming.
// Measured on 65k tokens of Hq 16 / Hkv 8 (bf16, D 128), same-box A/B: 6.06-6.11 TB/s
// against 4.93-5.02 for qk_norm_rope_store_kernel with its copy warp (blocks of 192
// q / k threads, 4 per SM); blocks of 128 q / k threads at 6 per SM 5.69-5.87, of 32 at 12
// per SM 5.72-5.89, of 192 at 4 per SM 5.37-5.41.
constexpr int kWsQkThreads = 64;
constexpr int kWsThreads = kWsQkThreads + 32;
constexpr int kWsCtasPerSm = 8;
constexpr int kWsStages = 3;
constexpr int kWsSmemMax = 200 * 1024;  // larger passes (over ~66 KB of rows) take the other kernel

template <typename T, int D, typename I>
__global__ void __launch_bounds__(kWsThreads, kWsCtasPerSm) qk_norm_rope_ws_kernel(
    const T* __restrict__ q, I q_ts, I q_hs, const T* __restrict__ k, I k_ts, I k_hs,
    const T* __restrict__ v, I v_ts, I v_hs, const T* __restrict__ q_w, const T* __restrict__ k_w,
    float eps, const T* __restrict__ cos_t, const T* __restrict__ sin_t, int rope_rows,
    const int32_t* __restrict__ positions, const int64_t* __restrict__ slot_mapping, int num_tokens,
    int n_heads, int n_kv_heads, T* __restrict__ q_out, T* __restrict__ k_pool, T* __restrict__ v_pool,
    int64_t num_slots, int block_size, int block_shift, int* __restrict__ err) {
  constexpr int E = 16 / int(sizeof(T));
  constexpr int L = D / E;
  constexpr int HALF = L / 2;
  constexpr int S = kWsQkThreads / L;
  constexpr int ROW = D * int(sizeof(T));
  extern __shared__ __align__(128) uint8_t wsm[];
  const int units_qk = n_heads + n_kv_heads;
  const int units = units_qk + n_kv_heads;  // rows of a token in a stage: q, k, v
  const int lane = threadIdx.x & 31;
  const bool packed = units_qk <= S;
  const int tpb = packed ? S / units_qk : 1;
  const int tstride = gridDim.x * tpb;
  const int pass_bytes = tpb * units * ROW;
  uint64_t* full = reinterpret_cast<uint64_t*>(wsm + kWsStages * pass_bytes);
  uint64_t* empty = full + kWsStages;
  const int t_first = blockIdx.x * tpb;
  const int npass = t_first < num_tokens ? (num_tokens - t_first + tstride - 1) / tstride : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWsStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWsQkThreads / 32 + 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (threadIdx.x >= kWsQkThreads) {
    // ============================== copy warp ==============================
    auto load_pass = [&](int p) {  // lane 0
      const int tb = t_first + p * tstride;
      const int nt = min(tpb, num_tokens - tb);
      const int st = p % kWsStages;
      mbar_arrive_expect_tx(&full[st], uint32_t(nt * units * ROW));
      uint8_t* dst = wsm + st * pass_bytes;
      for (int i = 0; i < nt; ++i) {
        const I t = I(tb + i);
        uint8_t* d = dst + i * units * ROW;
        if (q_hs == I(D)) {
          bulk_g2s(d, q + t * q_ts, uint32_t(n_heads * ROW), &full[st]);
        } else {
          for (int h = 0; h < n_heads; ++h) bulk_g2s(d + h * ROW, q + t * q_ts + I(h) * q_hs, uint32_t(ROW), &full[st]);
        }
        d += n_heads * ROW;
        if (k_hs == I(D)) {
          bulk_g2s(d, k + t * k_ts, uint32_t(n_kv_heads * ROW), &full[st]);
        } else {
          for (int h = 0; h < n_kv_heads; ++h)
            bulk_g2s(d + h * ROW, k + t * k_ts + I(h) * k_hs, uint32_t(ROW), &full[st]);
        }
        d += n_kv_heads * ROW;
        if (v_hs == I(D)) {
          bulk_g2s(d, v + t * v_ts, uint32_t(n_kv_heads * ROW), &full[st]);
        } else {
          for (int h = 0; h < n_kv_heads; ++h)
            bulk_g2s(d + h * ROW, v + t * v_ts + I(h) * v_hs, uint32_t(ROW), &full[st]);
        }
      }
    };
    if (lane == 0) {
      for (int p = 0; p < kWsStages - 1 && p < npass; ++p) load_pass(p);
    }
    bool ok = true;
    for (int p = 0; p < npass; ++p) {
      if (p > 0) {
        // this warp's value stores of pass p - 1 have read the stage; release it
        bulk_wait_reads_v();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[(p - 1) % kWsStages]);
      }
      const int pn = p + kWsStages - 1;
      if (lane == 0 && pn < npass) {
        // the stage of pass pn last held pass p - 1: every warp has released it
        if (pn >= kWsStages) ok = mbar_wait(&empty[pn % kWsStages], uint32_t(pn / kWsStages - 1) & 1u, err, 0x342);
        if (ok) load_pass(pn);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const int st = p % kWsStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[st], uint32_t(p / kWsStages) & 1u, err, 0x343))) break;
      const int tb = t_first + p * tstride;
      const int nt = min(tpb, num_tokens - tb);
      for (int rr = lane; rr < nt * n_kv_heads; rr += 32) {
        const int i = rr / n_kv_heads, h = rr - i * n_kv_heads;
        const int64_t slot = __ldg(slot_mapping + tb + i);
        if (slot < 0 || slot >= num_slots) continue;  // padding, or reported by the q / k threads
        const int64_t blk = block_shift >= 0 ? (slot >> block_shift) : slot / block_size;
        const int off = int(slot - blk * block_size);
        bulk_s2g_v(v_pool + ((I(blk) * n_kv_heads + h) * block_size + off) * I(D),
                   smem_u32(wsm + st * pass_bytes + (i * units + units_qk + h) * ROW), uint32_t(ROW));
      }
      bulk_commit_v();
    }
    bulk_wait_done_v();
    return;
  }

  // ============================== q / k threads ==============================
  const int sub = threadIdx.x % L;
  const int j = threadIdx.x / L;
  const bool active = !packed || j < tpb * units_qk;  // spare slots still release the stages
  const int tok_off = packed ? j / units_qk : 0;
  const int u0 = packed ? j % units_qk : j;
  const int ustep = packed ? units_qk : S;
  const uint32_t gmask = L == 32 ? 0xffffffffu : (((1u << L) - 1u) << (lane & ~(L - 1)));
  const float inv_d = 1.f / float(D);
  const uint4 wq = ldg_pair<T, D>(q_w, sub), wk = ldg_pair<T, D>(k_w, sub);
  auto norm_rope = [&](const uint4& raw, const uint4& wv, const uint4& cr, const uint4& sr) -> uint4 {
    float c[E], sn[E];
    unpack16<T>(cr, c);
    unpack16<T>(sr, sn);
    float x[E], w[E];
    unpack16<T>(raw, x);
    unpack16<T>(wv, w);
    float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 x2 = make_float2(x[e], x[e + 1]);
      ss2 = __ffma2_rn(x2, x2, ss2);
    }
    float ss = ss2.x + ss2.y;
#pragma unroll
    for (int o = HALF; o >= 1; o >>= 1) ss += __shfl_xor_sync(gmask, ss, o);
    const float inv = rsqrtf(ss * inv_d + eps);
    const float2 inv2 = make_float2(inv, inv);
    float y[E];
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 yy = __fmul2_rn(__fmul2_rn(make_float2(x[e], x[e + 1]), inv2), make_float2(w[e], w[e + 1]));
      y[e] = yy.x;
      y[e + 1] = yy.y;
    }
    float r[E];
#pragma unroll
    for (int e = 0; e < E / 2; e += 2) {
      const float2 ylo = make_float2(y[e], y[e + 1]), yhi = make_float2(y[e + E / 2], y[e + E / 2 + 1]);
      const float2 lo = __ffma2_rn(ylo, make_float2(c[e], c[e + 1]), __fmul2_rn(yhi, make_float2(-sn[e], -sn[e + 1])));
      const float2 hi = __ffma2_rn(yhi, make_float2(c[e + E / 2], c[e + E / 2 + 1]),
                                   __fmul2_rn(ylo, make_float2(sn[e + E / 2], sn[e + E / 2 + 1])));
      r[e] = lo.x;
      r[e + 1] = lo.y;
      r[e + E / 2] = hi.x;
      r[e + E / 2 + 1] = hi.y;
    }
    return pack16<T>(r);
  };
  const uint32_t sbase = smem_u32(wsm);
  int t = t_first + tok_off;
  int pos_n = t < num_tokens ? __ldg(positions + t) : 0;
  int64_t slot_n = t < num_tokens ? __ldg(slot_mapping + t) : -1;
  for (int p = 0; p < npass; ++p, t += tstride) {
    const int st = p % kWsStages;
    const bool work = active && t < num_tokens;
    const int pos = pos_n;
    int64_t slot = slot_n;
    if (t + tstride < num_tokens) {
      pos_n = __ldg(positions + t + tstride);
      slot_n = __ldg(slot_mapping + t + tstride);
    }
    const bool rope_ok = pos >= 0 && pos < rope_rows;
    uint4 c = make_uint4(0, 0, 0, 0), sn = make_uint4(0, 0, 0, 0);
    if (work && rope_ok) {
      c = ldg_pair<T, D>(cos_t + I(pos) * D, sub);
      sn = ldg_pair<T, D>(sin_t + I(pos) * D, sub);
    }
    if (!__all_sync(0xffffffffu, mbar_wait(&full[st], uint32_t(p / kWsStages) & 1u, err, 0x344))) break;
    if (work) {
      if (slot >= num_slots) {
        if (sub == 0) record_error(err, FVB_ERR_BAD_SLOT, t);
        slot = -1;
      }
      if (!rope_ok && u0 == 0 && sub == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, t);
      const I blk = slot < 0 ? 0 : block_shift >= 0 ? I(slot >> block_shift) : I(slot / block_size);
      const int off = slot >= 0 ? int(slot - int64_t(blk) * block_size) : 0;
      const uint32_t tok_row = sbase + uint32_t(st * pass_bytes + tok_off * units * ROW);
      for (int uu = u0; uu < units_qk; uu += ustep) {
        const uint4 raw = lds_pair<T, D>(tok_row + uu * ROW, sub);
        if (uu < n_heads) {
          if (rope_ok) st_pair<T, D>(q_out + (I(uu) * num_tokens + t) * D, sub, norm_rope(raw, wq, c, sn));
        } else if (rope_ok && slot >= 0) {
          st_pair<T, D>(k_pool + ((blk * n_kv_heads + (uu - n_heads)) * block_size + off) * I(D), sub,
                        norm_rope(raw, wk, c, sn));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
}

template <typename T, int D>
cudaError_t launch_typed(const void* q, int64_t q_ts, int64_t q_hs, const void* k, int64_t k_ts, int64_t k_hs,
                         const void* v, int64_t v_ts, int64_t v_hs, const void* q_w, const void* k_w, float eps,
                         const void* cos_t, const void* sin_t, int rope_rows, const int32_t* positions,
                         const int64_t* slot_mapping, int64_t num_tokens, int n_heads, int n_kv_heads, void* q_out,
                         void* k_pool, void* v_pool, int64_t num_blocks, int block_size, int* err,
                         cudaStream_t stream) {
  constexpr int L = D / (16 / int(sizeof(T)));
  constexpr int S = kThreads / L;
  constexpr int ROW = D * int(sizeof(T));
  const int units_vt = n_heads + n_kv_heads;
  const int64_t tpb_vt = units_vt <= S ? S / units_vt : 1;
  const bool vt = tpb_vt * n_kv_heads * ROW <= kVStageMax;
  const int units = vt ? units_vt : n_heads + 2 * n_kv_heads;
  const int64_t tpb = units <= S ? S / units : 1;
  const size_t vsmem = vt ? size_t(kVStages) * tpb * n_kv_heads * ROW + kVStages * 8 : 0;
  int64_t blocks = (num_tokens + tpb - 1) / tpb;
  const int64_t cap = int64_t(device_sm_count()) * kCtasPerSm * 8;  // 8 waves, then token-stride
  if (blocks > cap) blocks = cap;
  int block_shift = -1;  // page size a power of two: slot / block_size as a shift
  for (int b = 0; b < 31; ++b)
    if ((1 << b) == block_size) block_shift = b;
  // Largest element offset any thread forms, in each tensor.
  auto span = [&](int64_t ts, int64_t hs, int heads) { return (num_tokens - 1) * ts + int64_t(heads - 1) * hs + D; };
  const int64_t widest = std::max({span(q_ts, q_hs, n_heads), span(k_ts, k_hs, n_kv_heads), span(v_ts, v_hs, n_kv_heads),
                                   int64_t(n_heads) * num_tokens * D, num_blocks * n_kv_heads * block_size * D,
                                   int64_t(rope_rows) * D});
#define FVB_QKN_LAUNCH(I, VTF)                                                                                         \
  qk_norm_rope_store_kernel<T, D, I, VTF><<<unsigned(blocks), kAllThreads, vsmem, stream>>>(                          \
      static_cast<const T*>(q), I(q_ts), I(q_hs), static_cast<const T*>(k), I(k_ts), I(k_hs),                         \
      static_cast<const T*>(v), I(v_ts), I(v_hs), static_cast<const T*>(q_w), static_cast<const T*>(k_w), eps,       \
      static_cast<const T*>(cos_t), static_cast<const T*>(sin_t), rope_rows, positions, slot_mapping,                \
      int(num_tokens), n_heads, n_kv_heads, static_cast<T*>(q_out), static_cast<T*>(k_pool), static_cast<T*>(v_pool), \
      num_blocks * block_size, block_size, block_shift, err)
  const bool narrow = widest < (int64_t(1) << 31);
  constexpr int kWsS = kWsQkThreads / L;
  const int64_t ws_tpb = units_vt <= kWsS ? kWsS / units_vt : 1;
  const int64_t ws_pass = ws_tpb * (n_heads + 2 * n_kv_heads) * ROW;
  const size_t wsmem = size_t(kWsStages) * ws_pass + 2 * kWsStages * 8;
  if (wsmem <= size_t(kWsSmemMax)) {
    int64_t wblocks = (num_tokens + ws_tpb - 1) / ws_tpb;
    const int64_t wcap = int64_t(device_sm_count()) * kWsCtasPerSm * 8;  // 8 waves, then token-stride
    if (wblocks > wcap) wblocks = wcap;
#define FVB_QKN_WS(I)                                                                                                  \
  do {                                                                                                                 \
    cudaError_t ce = set_smem_once<qk_norm_rope_ws_kernel<T, D, I>>(kWsSmemMax);                                     \
    if (ce != cudaSuccess) return ce;                                                                                  \
    qk_norm_rope_ws_kernel<T, D, I><<<unsigned(wblocks), kWsThreads, wsmem, stream>>>(                               \
        static_cast<const T*>(q), I(q_ts), I(q_hs), static_cast<const T*>(k), I(k_ts), I(k_hs),                       \
        static_cast<const T*>(v), I(v_ts), I(v_hs), static_cast<const T*>(q_w), static_cast<const T*>(k_w), eps,     \
        static_cast<const T*>(cos_t), static_cast<const T*>(sin_t), rope_rows, positions, slot_mapping,              \
        int(num_tokens), n_heads, n_kv_heads, static_cast<T*>(q_out), static_cast<T*>(k_pool),                       \
        static_cast<T*>(v_pool), num_blocks * block_size, block_size, block_shift, err);                             \
  } while (0)
    if (narrow) FVB_QKN_WS(int); else FVB_QKN_WS(int64_t);
#undef FVB_QKN_WS
    return cudaGetLastError();
  }
  if (vt) {
    if (narrow) FVB_QKN_LAUNCH(int, true); else FVB_QKN_LAUNCH(int64_t, true);
  } else {
    if (narrow) FVB_QKN_LAUNCH(int, false); else FVB_QKN_LAUNCH(int64_t, false);
  }
#undef FVB_QKN_LAUNCH
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dim(int head_dim, const void* q, int64_t q_ts, int64_t q_hs, const void* k, int64_t k_ts,
                       int64_t k_hs, const void* v, int64_t v_ts, int64_t v_hs, const void* q_w, const void* k_w,
                       float eps, const void* cos_t, const void* sin_t, int rope_rows, const int32_t* positions,
                       const int64_t* slot_mapping, int64_t num_tokens, int n_heads, int n_kv_heads, void* q_out,
                       void* k_pool, void* v_pool, int64_t num_blocks, int block_size, int* err,
                       cudaStream_t stream) {
#define FVB_QKN_ARGS q, q_ts, q_hs, k, k_ts, k_hs, v, v_ts, v_hs, q_w, k_w, eps, cos_t, sin_t, rope_rows, positions, \
                     slot_mapping, num_tokens, n_heads, n_kv_heads, q_out, k_pool, v_pool, num_blocks, block_size,  \
                     err, stream
  if (head_dim == 128) return launch_typed<T, 128>(FVB_QKN_ARGS);
  if (head_dim == 64) return launch_typed<T, 64>(FVB_QKN_ARGS);
#undef FVB_QKN_ARGS
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_qk_norm_rope_store(const void* q, int64_t q_ts, int64_t q_hs, const void* k, int64_t k_ts,
                                      int64_t k_hs, const void* v, int64_t v_ts, int64_t v_hs, const void* q_w,
                                      const void* k_w, float eps, const void* cos_t, const void* sin_t, int rope_rows,
                                      const int32_t* positions, const int64_t* slot_mapping, int64_t num_tokens,
                                      int n_heads, int n_kv_heads, int head_dim, void* q_out, void* k_pool,
                                      void* v_pool, int64_t num_blocks, int block_size, int dtype, int* err,
                                      cudaStream_t stream) {
  if (num_tokens == 0) return cudaSuccess;
#define FVB_QKN_ARGS head_dim, q, q_ts, q_hs, k, k_ts, k_hs, v, v_ts, v_hs, q_w, k_w, eps, cos_t, sin_t, rope_rows, \
                     positions, slot_mapping, num_tokens, n_heads, n_kv_heads, q_out, k_pool, v_pool, num_blocks,   \
                     block_size, err, stream
  switch (dtype) {
    case FVB_DTYPE_F32:
      return launch_dim<float>(FVB_QKN_ARGS);
    case FVB_DTYPE_BF16:
      return launch_dim<__nv_bfloat16>(FVB_QKN_ARGS);
    case FVB_DTYPE_F16:
      return launch_dim<__half>(FVB_QKN_ARGS);
    default:
      return cudaErrorInvalidValue;
  }
#undef FVB_QKN_ARGS
}

}  // namespace fvb
