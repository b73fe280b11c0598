// Varlen chunked-prefill attention on SIMT cores, for fp32 operands.
//
// fp32 attention must match an fp32 reference within 1e-4, which the
// tensor cores' TF32 inputs cannot; the bf16/f16 path runs on tcgen05
// (prefill_sm100.cu).  Same semantics as the reference prefill
// (femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:80-160): key j
// is visible to query i iff j < kv_len[s] and j <= positions[i]; online
// softmax in fp32.
//
// One warp per (query token, head).  Keys are taken 32 at a time: lane l
// computes the full q.k dot of key j0+l (q broadcast from shared memory),
// the warp updates its running max/sum, then lane l accumulates p * V for
// head dims [l*D/32, (l+1)*D/32).
#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kWarpsPerCta = 4;

__device__ __forceinline__ float warp_max_s(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_s(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(32 * kWarpsPerCta) prefill_simt_kernel(
    const T* __restrict__ q, T* __restrict__ out, const T* __restrict__ k_pool, const T* __restrict__ v_pool,
    int64_t num_blocks, int n_heads, int n_kv_heads, int num_seqs, int64_t q_len_flatten,
    const int32_t* __restrict__ cu_seqlens, const int32_t* __restrict__ block_tables, int max_blocks_per_seq,
    const int32_t* __restrict__ kv_lens, const int32_t* __restrict__ positions, const QOLayout lay,
    int* __restrict__ err) {
  constexpr int kDPL = D / 32;
  __shared__ float qsh[kWarpsPerCta][D];
  __shared__ float psh[kWarpsPerCta][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kWarpsPerCta + warp;  // (head, token) pair, token fastest
  if (row >= int64_t(n_heads) * q_len_flatten) return;
  const int head = int(row / q_len_flatten);
  const int64_t tok = row - int64_t(head) * q_len_flatten;
  // Sequence owning this token: last s with cu_seqlens[s] <= tok.
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_seqlens + mid) <= tok) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int kvh = head / (n_heads / n_kv_heads);
  int kv_len = __ldg(kv_lens + s);
  if (kv_len > max_blocks_per_seq * kPageSize) {
    if (lane == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
    kv_len = max_blocks_per_seq * kPageSize;
  }
  const int pos = __ldg(positions + tok);
  const int n_keys = min(kv_len, pos + 1);
  const float scale = kLog2e * rsqrtf(float(D));
  const T* qrow = q + tok * lay.q_ts + int64_t(head) * lay.q_hs;
  for (int d = lane; d < D; d += 32) qsh[warp][d] = Elem<T>::to_f(qrow[d]) * scale;
  __syncwarp();
  const int32_t* table = block_tables + int64_t(s) * max_blocks_per_seq;
  float m = -INFINITY, l = 0.f, acc[kDPL];
#pragma unroll
  for (int i = 0; i < kDPL; ++i) acc[i] = 0.f;
  for (int j0 = 0; j0 < n_keys; j0 += 32) {
    const int j = j0 + lane;
    float sc = -INFINITY;
    if (j < n_keys) {
      int blk = __ldg(table + j / kPageSize);
      if (blk < 0 || blk >= num_blocks) {
        record_error(err, FVB_ERR_BAD_PAGE, s);
        blk = 0;
      }
      const T* kr = k_pool + ((int64_t(blk) * n_kv_heads + kvh) * kPageSize + (j % kPageSize)) * D;
      float dot = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) dot = fmaf(qsh[warp][d], Elem<T>::to_f(kr[d]), dot);
      sc = dot;
    }
    const float mn = fmaxf(m, warp_max_s(sc));
    const float corr = fast_exp2(m - mn);
    const float p = fast_exp2(sc - mn);
    m = mn;
    l = l * corr + warp_sum_s(p);
#pragma unroll
    for (int i = 0; i < kDPL; ++i) acc[i] *= corr;
    psh[warp][lane] = p;
    __syncwarp();
    const int nk = min(32, n_keys - j0);
    for (int t = 0; t < nk; ++t) {
      const int jj = j0 + t;
      int blk = __ldg(table + jj / kPageSize);
      if (blk < 0 || blk >= num_blocks) blk = 0;
      const T* vr = v_pool + ((int64_t(blk) * n_kv_heads + kvh) * kPageSize + (jj % kPageSize)) * D;
      const float pt = psh[warp][t];
#pragma unroll
      for (int i = 0; i < kDPL; ++i) acc[i] = fmaf(pt, Elem<T>::to_f(vr[lane * kDPL + i]), acc[i]);
    }
    __syncwarp();
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  T* orow = out + tok * lay.o_ts + int64_t(head) * lay.o_hs;
  for (int i = 0; i < kDPL; ++i) orow[lane * kDPL + i] = Elem<T>::from_f(acc[i] * inv);
}

template <typename T>
cudaError_t launch_simt_t(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                          int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                          const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                          const int32_t* kv_lens, const int32_t* positions, const QOLayout& lay, int* err,
                          cudaStream_t stream) {
  const int64_t rows = int64_t(n_heads) * q_len_flatten;
  const int64_t blocks = (rows + kWarpsPerCta - 1) / kWarpsPerCta;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  auto args = [&](auto kern) {
    kern<<<unsigned(blocks), 32 * kWarpsPerCta, 0, stream>>>(
        static_cast<const T*>(q), static_cast<T*>(out), static_cast<const T*>(k_pool),
        static_cast<const T*>(v_pool), num_blocks, n_heads, n_kv_heads, num_seqs, q_len_flatten, cu_seqlens,
        block_tables, max_blocks_per_seq, kv_lens, positions, lay, err);
  };
  if (head_dim == 128) args(prefill_simt_kernel<T, 128>);
  else args(prefill_simt_kernel<T, 64>);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_simt(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                                const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                                const int32_t* kv_lens, const int32_t* positions, int dtype, const QOLayout& lay,
                                int* err, cudaStream_t stream) {
  if (q_len_flatten == 0 || num_seqs == 0) return cudaSuccess;
  switch (dtype) {
    case FVB_DTYPE_BF16:
      return launch_simt_t<__nv_bfloat16>(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim,
                                          num_seqs, q_len_flatten, cu_seqlens, block_tables, max_blocks_per_seq,
                                          kv_lens, positions, lay, err, stream);
    case FVB_DTYPE_F16:
      return launch_simt_t<__half>(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs,
                                   q_len_flatten, cu_seqlens, block_tables, max_blocks_per_seq, kv_lens,
                                   positions, lay, err, stream);
    default:
      return launch_simt_t<float>(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs,
                                  q_len_flatten, cu_seqlens, block_tables, max_blocks_per_seq, kv_lens, positions,
                                  lay, err, stream);
  }
}

}  // namespace fvb
