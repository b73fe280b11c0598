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
// Layout: a row is D contiguous elements = D * sizeof(T) / 16 lanes, each
// holding one 16-byte vector.  The row's sum of squares is reduced over
// those lanes by xor shuffles, and the rotary partner half (d +- D/2) lives
// in the lane half a row away, one more xor shuffle.  HBM-bound:
// (Hq + 2 Hkv) D sizeof(T) bytes read and written per token, plus 12 bytes
// of position / slot and the cos / sin rows (L2-resident).
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

constexpr int kThreads = 256;

// Row r of the launch = (token r / units, unit r % units); unit u < Hq is a
// query head, u < Hq + Hkv a key head, the rest value heads.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) qk_norm_rope_store_kernel(
    const T* __restrict__ q, int64_t q_ts, int64_t q_hs, const T* __restrict__ k, int64_t k_ts, int64_t k_hs,
    const T* __restrict__ v, int64_t v_ts, int64_t v_hs, const T* __restrict__ q_w, const T* __restrict__ k_w,
    float eps, const T* __restrict__ cos_t, const T* __restrict__ sin_t, int rope_rows,
    const int32_t* __restrict__ positions, const int64_t* __restrict__ slot_mapping, int64_t num_tokens,
    int n_heads, int n_kv_heads, T* __restrict__ q_out, T* __restrict__ k_pool, T* __restrict__ v_pool,
    int64_t num_slots, int block_size, int* __restrict__ err) {
  constexpr int E = 16 / int(sizeof(T));  // elements per lane
  constexpr int L = D / E;                // lanes per row
  constexpr int HALF = L / 2;             // lane distance of the rotary partner
  static_assert(L >= 2 && L <= 32 && 32 % L == 0, "row must tile a warp");
  constexpr int kRowsPerBlock = kThreads / L;
  const int units = n_heads + 2 * n_kv_heads;
  const int64_t rows = num_tokens * units;
  const int sub = threadIdx.x % L;
  const bool first_half = sub < HALF;
  const float inv_d = 1.f / float(D);
  // The loop bound is block-uniform, so every lane of a warp reaches the shuffles.
  for (int64_t base = int64_t(blockIdx.x) * kRowsPerBlock; base < rows;
       base += int64_t(gridDim.x) * kRowsPerBlock) {
    const int64_t row = base + threadIdx.x / L;
    const bool live = row < rows;
    const int64_t t = live ? row / units : 0;
    const int u = live ? int(row - t * units) : 0;
    const int kind = u < n_heads ? 0 : (u < n_heads + n_kv_heads ? 1 : 2);  // q / k / v
    const int h = kind == 0 ? u : (kind == 1 ? u - n_heads : u - n_heads - n_kv_heads);
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (live) {
      const T* src = kind == 0 ? q + t * q_ts + h * q_hs : (kind == 1 ? k + t * k_ts + h * k_hs : v + t * v_ts + h * v_hs);
      raw = ldg16(src + sub * E);
    }
    int64_t slot = -1;
    if (live && kind != 0) {
      slot = __ldg(slot_mapping + t);
      if (slot >= num_slots) {
        record_error(err, FVB_ERR_BAD_SLOT, int(t));
        slot = -1;
      }
    }
    int pos = 0;
    bool rope_ok = false;
    if (live && kind != 2) {
      pos = __ldg(positions + t);
      rope_ok = pos >= 0 && pos < rope_rows;
      if (!rope_ok) record_error(err, FVB_ERR_INVALID_ARGUMENT, int(t));
    }
    // RMSNorm (all lanes take part in the shuffles, value rows included).
    float x[E];
    unpack16<T>(raw, x);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
    for (int o = HALF; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * inv_d + eps);
    float w[E], c[E], s[E];
    if (kind != 2 && rope_ok) {
      unpack16<T>(ldg16((kind == 0 ? q_w : k_w) + sub * E), w);
      unpack16<T>(ldg16(cos_t + int64_t(pos) * D + sub * E), c);
      unpack16<T>(ldg16(sin_t + int64_t(pos) * D + sub * E), s);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) w[e] = c[e] = s[e] = 0.f;
    }
    float y[E];
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = x[e] * inv * w[e];
    float r[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float yp = __shfl_xor_sync(0xffffffffu, y[e], HALF);
      r[e] = fmaf(y[e], c[e], (first_half ? -yp : yp) * s[e]);
    }
    if (!live) continue;
    if (kind == 0) {
      if (rope_ok) {
        *reinterpret_cast<uint4*>(q_out + (int64_t(h) * num_tokens + t) * D + sub * E) = pack16<T>(r);
      }
    } else if (slot >= 0 && (kind == 2 || rope_ok)) {
      const int64_t blk = slot / block_size;
      const int off = int(slot - blk * block_size);
      T* dst = (kind == 1 ? k_pool : v_pool) + ((blk * n_kv_heads + h) * block_size + off) * D + sub * E;
      *reinterpret_cast<uint4*>(dst) = kind == 1 ? pack16<T>(r) : raw;
    }
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
  const int64_t rows = num_tokens * (n_heads + 2 * n_kv_heads);
  int64_t blocks = (rows + kThreads / L - 1) / (kThreads / L);
  const int64_t cap = int64_t(device_sm_count()) * 8;  // 8 resident CTAs per SM, then grid-stride
  if (blocks > cap) blocks = cap;
  qk_norm_rope_store_kernel<T, D><<<unsigned(blocks), kThreads, 0, stream>>>(
      static_cast<const T*>(q), q_ts, q_hs, static_cast<const T*>(k), k_ts, k_hs, static_cast<const T*>(v), v_ts,
      v_hs, static_cast<const T*>(q_w), static_cast<const T*>(k_w), eps, static_cast<const T*>(cos_t),
      static_cast<const T*>(sin_t), rope_rows, positions, slot_mapping, num_tokens, n_heads, n_kv_heads,
      static_cast<T*>(q_out), static_cast<T*>(k_pool), static_cast<T*>(v_pool), num_blocks * block_size, block_size,
      err);
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
