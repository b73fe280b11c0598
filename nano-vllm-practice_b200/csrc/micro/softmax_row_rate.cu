// Measurement program (not part of the library): cycles one warp per SM sub-partition
// spends on the prefill softmax of one 128-column score row, and the SFU issue rate of
// exp2, on a B200.
//
// The prefill kernel's softmax gives each thread one query row of a 128-key tile:
// 3-input max over the row, (s - m) * scale on packed fp32 FMAs, 128 exp2, a packed
// fp32 row sum and a pack of P to bf16x2.  Variants here replace the exp2 source:
//   * ex2.approx.ftz.f32 (what the kernel uses);
//   * no exp at all (the rest of the row's work);
//   * ex2.approx.f16x2 (two values per instruction, P converted to bf16 after);
//   * the first 2K columns on the FMA pipe: x = n + f with n = round(x) by adding
//     1.5 * 2^23, 2^f by a degree-3 polynomial on [-0.5, 0.5], and n added into the
//     exponent bits.  The coefficients are a least-squares fit of the relative error
//     refined by Lawson iterations (max relative error 7.5e-5), made for this program.
//
// Build and run (one GPU, about two seconds):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o softmax_row_rate softmax_row_rate.cu
//   ./softmax_row_rate
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>

namespace {

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t ex2h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t cvt_h2(float hi, float lo) {
  uint32_t y;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(y) : "f"(hi), "f"(lo));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA pipe.  x is clamped to -126 so that n + 127 >= 1 keeps
// the exponent field from wrapping (the result there is ~1e-38, not 0).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 shift = make_float2(12582912.f, 12582912.f);
  const float2 t = __fadd2_rn(x, shift);
  const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(f, make_float2(0.055171433836221695f, 0.055171433836221695f),
                        make_float2(0.24261081218719482f, 0.24261081218719482f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

enum Variant { kMufu = 0, kNoExp = 1, kHalf2 = 2, kFma = 3 };

template <int V, int K>
__global__ void __launch_bounds__(128, 1) row_kernel(const float* in, uint32_t* out, long long* cyc, int iters) {
  float sr[128];
  for (int c = 0; c < 128; ++c) sr[c] = in[(threadIdx.x * 128 + c) & 4095];
  const float2 scale2 = make_float2(0.127f, 0.127f);
  uint32_t chk = 0;
  float l = 0.f, bias = 0.f;
  __syncwarp();
  const long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    float mx[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) mx[a] = sr[a] + bias;
#pragma unroll
    for (int c = 8; c < 120; c += 16)
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = fmax3(mx[a], sr[c + a], sr[c + 8 + a]);
#pragma unroll
    for (int a = 0; a < 8; ++a) mx[a] = fmaxf(mx[a], sr[120 + a]);
    const float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
    const float2 nms2 = make_float2(-mt * 0.127f, -mt * 0.127f);
    float2 acc[4] = {};
    uint32_t pk[64];
#pragma unroll
    for (int c = 0; c < 128; c += 2) {
      const float2 x = __ffma2_rn(make_float2(sr[c], sr[c + 1]), scale2, nms2);
      float2 p;
      if (V == kMufu || (V == kFma && c >= 2 * K)) {
        p = make_float2(ex2f(x.x), ex2f(x.y));
      } else if (V == kFma) {
        p = exp2_fma2(x);
      } else if (V == kHalf2) {
        const uint32_t h = ex2h2(cvt_h2(x.y, x.x));
        p = __half22float2(*reinterpret_cast<const __half2*>(&h));
      } else {
        p = x;
      }
      pk[c >> 1] = pack_bf(p.x, p.y);
      acc[(c >> 1) & 3] = __fadd2_rn(acc[(c >> 1) & 3], p);
    }
    const float2 a = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
    l += a.x + a.y;
#pragma unroll
    for (int c = 0; c < 64; ++c) chk ^= pk[c];
    bias = l * 1e-30f;  // carries a dependence into the next iteration
  }
  const long long t1 = clock64();
  out[blockIdx.x * 128 + threadIdx.x] = chk ^ __float_as_uint(l);
  if (threadIdx.x == 0) cyc[blockIdx.x] = t1 - t0;
}

// Issue rate: 16 independent exp2 chains per thread, one warp per sub-partition.
template <bool HALF2>
__global__ void __launch_bounds__(128, 1) rate_kernel(const float* in, uint32_t* out, long long* cyc, int iters) {
  float x[16];
  uint32_t h[16];
  for (int c = 0; c < 16; ++c) {
    x[c] = -in[(threadIdx.x + c) & 4095] * 1e-3f;
    h[c] = __float_as_uint(x[c]) & 0xBBFFBBFFu;
  }
  __syncwarp();
  const long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      if (HALF2)
        h[c] = ex2h2(h[c]) ^ 0x3c003c00u;
      else
        x[c] = ex2f(x[c]) - 1.0f;
    }
  }
  const long long t1 = clock64();
  uint32_t chk = 0;
  for (int c = 0; c < 16; ++c) chk ^= __float_as_uint(x[c]) ^ h[c];
  out[blockIdx.x * 128 + threadIdx.x] = chk;
  if (threadIdx.x == 0) cyc[blockIdx.x] = t1 - t0;
}

}  // namespace

int main() {
  constexpr int kBlocks = 148, kIters = 2000;
  float* in = nullptr;
  uint32_t* out = nullptr;
  long long* cyc = nullptr;
  if (cudaMalloc(&in, 4096 * sizeof(float)) != cudaSuccess || cudaMalloc(&out, kBlocks * 128 * 4) != cudaSuccess ||
      cudaMalloc(&cyc, kBlocks * sizeof(long long)) != cudaSuccess) {
    std::printf("allocation failed\n");
    return 1;
  }
  static float h_in[4096];
  for (int i = 0; i < 4096; ++i) h_in[i] = float((i * 2654435761u) % 1000) / 100.f - 5.f;
  cudaMemcpy(in, h_in, sizeof(h_in), cudaMemcpyHostToDevice);
  long long h_cyc[kBlocks];
  auto report = [&](const char* name, double per) {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      std::printf("error: %s\n", cudaGetErrorString(e));
      std::exit(1);
    }
    cudaMemcpy(h_cyc, cyc, sizeof(h_cyc), cudaMemcpyDeviceToHost);
    double s = 0;
    for (int b = 0; b < kBlocks; ++b) s += double(h_cyc[b]);
    std::printf("%-34s %8.2f cycles\n", name, s / kBlocks / kIters / per);
  };
  rate_kernel<false><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("ex2.approx.ftz.f32 per warp instr", 16);
  rate_kernel<true><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("ex2.approx.f16x2 per warp instr", 16);
  row_kernel<kMufu, 0><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 128 ex2.f32 (kernel)", 1);
  row_kernel<kNoExp, 0><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: no exp", 1);
  row_kernel<kHalf2, 0><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 64 ex2.f16x2", 1);
  row_kernel<kFma, 8><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 16 of 128 on the FMA pipe", 1);
  row_kernel<kFma, 16><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 32 of 128 on the FMA pipe", 1);
  row_kernel<kFma, 32><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 64 of 128 on the FMA pipe", 1);
  row_kernel<kFma, 64><<<kBlocks, 128>>>(in, out, cyc, kIters);
  report("row: 128 of 128 on the FMA pipe", 1);
  cudaFree(in);
  cudaFree(out);
  cudaFree(cyc);
  return 0;
}
