// Shared device helpers for the sm_100a attention hot path.
//
// Everything here is a thin wrapper over one documented PTX instruction
// (PTX ISA 8.7: mbarrier, cp.async.bulk, cp.async.bulk.tensor, tcgen05.*,
// fence.proxy.async, ex2.approx).  Every wait on an mbarrier is bounded: it
// gives up after kWaitTimeoutNs of %globaltimer, records an error code in the
// library's device error word and returns false, so a logic error can never
// spin a GPU forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "femtovllm_b200.h"

namespace fvb {

// Page size of the KV pools (kKVLenPerPage, csrc/utils/constants.cuh:75 of the reference).
constexpr int kPageSize = 16;
// A bounded mbarrier wait gives up after this many nanoseconds.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

// Device error word, int[2] = {code, info}: the first error recorded since
// the last host read (capi.cu owns it; kernels get its address as an
// argument).  Kernels only ever CAS 0 -> code, so the first cause wins.
__device__ __forceinline__ void record_error(int* err, int code, int info) {
  if (atomicCAS(err, 0, code) == 0) atomicExch(err + 1, info);
}

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int kDtype = FVB_DTYPE_F32;
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kDtype = FVB_DTYPE_BF16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elem<__half> {
  static constexpr int kDtype = FVB_DTYPE_F16;
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

// Unpack a 16-byte vector of T into floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* out);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float* out) {
  out[0] = __uint_as_float(v.x);
  out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z);
  out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& v, float* out) {
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits.
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// acc.x += lo(q) * lo(k) and acc.y += hi(q) * hi(k) for two packed 16-bit pairs, by
// the mixed-precision FMA of sm_100 (fma.rn.f32.bf16 / .f16): the 16-bit operands are
// taken as they are, the product is exact and rounded once, so the result equals an
// fp32 FMA on the converted values without the conversion instructions.
template <typename T>
__device__ __forceinline__ void fma_pair16(uint32_t q, uint32_t k, float2& acc);
template <>
__device__ __forceinline__ void fma_pair16<__nv_bfloat16>(uint32_t q, uint32_t k, float2& acc) {
  asm("{\n\t.reg .b16 ql, qh, kl, kh;\n\t"
      "mov.b32 {ql, qh}, %2;\n\tmov.b32 {kl, kh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, ql, kl, %0;\n\tfma.rn.f32.bf16 %1, qh, kh, %1;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(q), "r"(k));
}
template <>
__device__ __forceinline__ void fma_pair16<__half>(uint32_t q, uint32_t k, float2& acc) {
  asm("{\n\t.reg .b16 ql, qh, kl, kh;\n\t"
      "mov.b32 {ql, qh}, %2;\n\tmov.b32 {kl, kh}, %3;\n\t"
      "fma.rn.f32.f16 %0, ql, kl, %0;\n\tfma.rn.f32.f16 %1, qh, kh, %1;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(q), "r"(k));
}
template <>
__device__ __forceinline__ void fma_pair16<float>(uint32_t, uint32_t, float2&) {}

// 2^x on the SFU (ex2.approx.ftz.f32); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make mbarrier.init visible to the async proxy (TMA / tcgen05 arrivals).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records FVB_ERR_DEVICE_TIMEOUT with `site`) if it has not after
// kWaitTimeoutNs.  Callers treat false as "abandon the work item".
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, FVB_ERR_DEVICE_TIMEOUT, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk copies (TMA engine), global -> shared, completion on an mbarrier.
// No multicast form is used anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst_smem, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst_smem)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst_smem, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst_smem)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch.  launch_dependents lets a kernel launched after
// this one with cudaLaunchAttributeProgrammaticStreamSerialization start once every
// CTA of this grid has executed it (or exited); that kernel's grid_dependency_wait
// returns when this grid has completed and its memory writes are visible.  Both are
// no-ops for kernels launched without the attribute.
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over nthreads threads that also returns the AND of pred over them.
__device__ __forceinline__ bool named_barrier_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Read-only 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(addr));
  return r;
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace fvb
