// Varlen attention metadata built on the device from per-sequence scalars.
//
// Replaces the host loops of the reference's ModelRunner
// (femtovllm/engine/model_runner.py:186-205 prefill route, :280-290 decode
// route, pad_block_tables :46-72), which build Python lists per step and copy
// them to the device.  For sequence s with p_s = num_computed[s] cached
// tokens and n_s = num_new[s] new ones:
//   cu_seqlens[s + 1] = sum_{r <= s} n_r          (cu_seqlens[0] = 0)
//   kv_lens[s]        = p_s + n_s
//   positions[t]      = p_s + (t - cu_seqlens[s])  for the new tokens t of s
//   block_tables[s][i] = flat_blocks[cu_blocks[s] + i]  (i < blocks of s), else -1
//   slot_mapping[t]   = block_tables[s][pos / 16] * 16 + pos % 16, or -1
// The decode route is the special case n_s = 1.  Two launches: a one-CTA scan
// (sequences), then one grid-stride fill over table entries and tokens.
#include "common.cuh"
#include "kernels.h"

namespace fvb {
namespace {

__global__ void __launch_bounds__(1024) varlen_scan_kernel(const int32_t* __restrict__ num_computed,
                                                           const int32_t* __restrict__ num_new, int num_seqs,
                                                           int64_t num_tokens, int32_t* __restrict__ cu_seqlens,
                                                           int32_t* __restrict__ kv_lens, int* __restrict__ err) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (threadIdx.x == 0) {
    carry = 0;
    cu_seqlens[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < num_seqs; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int n = 0;
    if (s < num_seqs) {
      n = __ldg(num_new + s);
      const int p = __ldg(num_computed + s);
      if (n < 0 || p < 0) {
        record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
        n = max(n, 0);
      }
      kv_lens[s] = max(p, 0) + n;
    }
    int x = n;
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
    if (s < num_seqs) cu_seqlens[s + 1] = incl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0 && int64_t(carry) != num_tokens) record_error(err, FVB_ERR_INVALID_ARGUMENT, -1);
}

__global__ void __launch_bounds__(256) varlen_fill_kernel(
    const int32_t* __restrict__ num_computed, const int32_t* __restrict__ cu_seqlens, int num_seqs,
    const int32_t* __restrict__ flat_blocks, int64_t num_flat_blocks, const int32_t* __restrict__ cu_blocks,
    int max_blocks_per_seq, int64_t num_tokens, int block_size, int32_t* __restrict__ positions,
    int32_t* __restrict__ block_tables, int64_t* __restrict__ slot_mapping, int* __restrict__ err) {
  const int64_t entries = int64_t(num_seqs) * max_blocks_per_seq;
  const int64_t total = entries + num_tokens;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    if (i < entries) {
      const int s = int(i / max_blocks_per_seq), e = int(i - int64_t(s) * max_blocks_per_seq);
      const int b0 = __ldg(cu_blocks + s);
      int nb = __ldg(cu_blocks + s + 1) - b0;
      if (nb < 0 || nb > max_blocks_per_seq || b0 < 0 || int64_t(b0) + nb > num_flat_blocks) {
        if (e == 0) record_error(err, FVB_ERR_INVALID_ARGUMENT, s);
        nb = 0;  // a malformed row reads nothing
      }
      block_tables[i] = e < nb ? __ldg(flat_blocks + b0 + e) : -1;
      continue;
    }
    const int64_t t = i - entries;
    int lo = 0, hi = num_seqs - 1;  // last sequence whose first token is <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(cu_seqlens + mid) <= t) lo = mid; else hi = mid - 1;
    }
    const int s = lo;
    const int pos = max(__ldg(num_computed + s), 0) + int(t - __ldg(cu_seqlens + s));
    positions[t] = pos;
    if (slot_mapping != nullptr) {
      const int b0 = __ldg(cu_blocks + s);
      int nb = __ldg(cu_blocks + s + 1) - b0;
      if (nb < 0 || nb > max_blocks_per_seq || b0 < 0 || int64_t(b0) + nb > num_flat_blocks) nb = 0;
      const int page = pos / block_size;
      int64_t slot = -1;
      if (page < nb) {
        const int blk = __ldg(flat_blocks + b0 + page);
        if (blk >= 0) slot = int64_t(blk) * block_size + pos % block_size;
      }
      slot_mapping[t] = slot;
    }
  }
}

}  // namespace

cudaError_t launch_build_varlen_metadata(const int32_t* num_computed, const int32_t* num_new, int num_seqs,
                                         const int32_t* flat_blocks, int64_t num_flat_blocks,
                                         const int32_t* cu_blocks, int max_blocks_per_seq, int64_t num_tokens,
                                         int32_t* positions,
                                         int32_t* cu_seqlens, int32_t* kv_lens, int32_t* block_tables,
                                         int64_t* slot_mapping, int* err, cudaStream_t stream) {
  varlen_scan_kernel<<<1, 1024, 0, stream>>>(num_computed, num_new, num_seqs, num_tokens, cu_seqlens, kv_lens, err);
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return ce;
  const int64_t total = int64_t(num_seqs) * max_blocks_per_seq + num_tokens;
  if (total == 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = int64_t(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  varlen_fill_kernel<<<unsigned(blocks), 256, 0, stream>>>(num_computed, cu_seqlens, num_seqs, flat_blocks,
                                                           num_flat_blocks, cu_blocks, max_blocks_per_seq, num_tokens,
                                                           kPageSize, positions, block_tables, slot_mapping, err);
  return cudaGetLastError();
}

}  // namespace fvb
