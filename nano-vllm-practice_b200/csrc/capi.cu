// extern "C" entry points of libfemtovllm_b200.so (declared in
// include/femtovllm_b200.h).  Host-side validation of every scalar argument,
// the 16-byte alignment rules of the TMA / vector paths, workspace sizing,
// and mapping of CUDA errors to fvb_status.  Nothing here allocates.  Every compute entry point
// opens an NVTX range named after itself, so Nsight Systems timelines and `ncu --nvtx` filters
// see the library's calls (NVTX is a no-op unless a tool is attached).
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace fvb {

// {first error code, its info} since the last fvb_read_device_error on this device.
__device__ int g_device_error[2] = {0, 0};

namespace {

// NVTX range for the lifetime of one entry-point call.
struct TraceRange {
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

constexpr int kMaxDevices = 64;
std::atomic<int*> g_err_ptr[kMaxDevices] = {};

// Device address of g_device_error on the current device, resolved once per device.
// Threads racing on the first call all resolve the same address; the atomic keeps the
// cache itself race-free.
int* device_error_ptr(cudaError_t* e) {
  int dev = 0;
  *e = cudaGetDevice(&dev);
  if (*e != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    *e = cudaErrorInvalidDevice;
    return nullptr;
  }
  int* cached = g_err_ptr[dev].load(std::memory_order_acquire);
  if (!cached) {
    void* p = nullptr;
    *e = cudaGetSymbolAddress(&p, g_device_error);
    if (*e != cudaSuccess) return nullptr;
    cached = static_cast<int*>(p);
    g_err_ptr[dev].store(cached, std::memory_order_release);
  }
  return cached;
}

thread_local int t_last_cuda_error = 0;

int esize_of(int dtype) {
  switch (dtype) {
    case FVB_DTYPE_F32:
      return 4;
    case FVB_DTYPE_BF16:
    case FVB_DTYPE_F16:
      return 2;
    default:
      return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return FVB_OK;
  t_last_cuda_error = int(e);
  return FVB_ERR_CUDA;
}

// Any whole GQA group (kv_head = q_head / (n_heads / n_kv_heads), as the reference).
bool gqa_ok(int n_heads, int n_kv_heads) {
  return n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0;
}

// Common checks of the attention entry points.
int check_attention(const void* q, const void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                    int n_heads, int n_kv_heads, int head_dim, int block_size, int num_seqs,
                    const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens, int dtype) {
  if (esize_of(dtype) == 0) return FVB_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return FVB_ERR_UNSUPPORTED;
  if (block_size != kPageSize) return FVB_ERR_UNSUPPORTED;
  if (!gqa_ok(n_heads, n_kv_heads)) return FVB_ERR_UNSUPPORTED;
  if (num_seqs < 0 || num_blocks < 1 || max_blocks_per_seq < 0) return FVB_ERR_INVALID_ARGUMENT;
  if (num_seqs > 0 && (!q || !out || !k_pool || !v_pool || !block_tables || !kv_lens))
    return FVB_ERR_INVALID_ARGUMENT;
  if (num_blocks * n_kv_heads * kPageSize > int64_t(0x7fffffff)) return FVB_ERR_UNSUPPORTED;  // TMA row coordinate
  if (!aligned16(q) || !aligned16(out) || !aligned16(k_pool) || !aligned16(v_pool)) return FVB_ERR_MISALIGNED;
  return FVB_OK;
}

// Decode route: 16-bit GQA >= 5 runs on the tcgen05 attention kernel (measured 1.68x
// the SIMT split-KV kernel at GQA 8, config-2 lengths; groups of 5-7 pad to 8 heads on
// either path); smaller groups and fp32 keep the split-KV kernel, HBM-bound for them.
bool decode_on_tensor_cores(int n_heads, int n_kv_heads, int dtype) {
  return dtype != FVB_DTYPE_F32 && n_kv_heads > 0 && n_heads / n_kv_heads >= 5;
}

// q / out strides (elements): non-negative, and every row start 16-byte aligned
// (the tensor-core prefill loads q rows with TMA and stores out rows as 16-byte vectors).
int check_layout(const QOLayout& lay, int dtype) {
  const int64_t es = esize_of(dtype);
  const int64_t st[4] = {lay.q_ts, lay.q_hs, lay.o_ts, lay.o_hs};
  for (int64_t x : st) {
    if (x < 0) return FVB_ERR_INVALID_ARGUMENT;
    if ((x * es) % 16 != 0) return FVB_ERR_MISALIGNED;
  }
  return FVB_OK;
}

}  // namespace

int device_sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

namespace {
cudaError_t tensor_map_encoder(EncodeTiledFn* out) {
  static std::atomic<EncodeTiledFn> encode{nullptr};  // resolved once; concurrent first calls agree
  EncodeTiledFn fnp = encode.load(std::memory_order_acquire);
  if (!fnp) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qres;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &qres);
    if (e != cudaSuccess) return e;
    if (qres != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    fnp = reinterpret_cast<EncodeTiledFn>(fn);
    encode.store(fnp, std::memory_order_release);
  }
  *out = fnp;
  return cudaSuccess;
}
}  // namespace

cudaError_t make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                        uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn encode = nullptr;
  cudaError_t e = tensor_map_encoder(&encode);
  if (e != cudaSuccess) return e;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tma_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims3[3],
                        const uint64_t stride_bytes[2], const uint32_t box3[3], bool swizzle128) {
  EncodeTiledFn encode = nullptr;
  cudaError_t e = tensor_map_encoder(&encode);
  if (e != cudaSuccess) return e;
  const cuuint64_t dims[3] = {dims3[0], dims3[1], dims3[2]};
  const cuuint64_t strides[2] = {stride_bytes[0], stride_bytes[1]};
  const cuuint32_t box[3] = {box3[0], box3[1], box3[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {
// One thread waits, through the same bounded mbar_wait every kernel uses, on a
// barrier that no thread ever arrives on: the wait must give up after its limit,
// record FVB_ERR_DEVICE_TIMEOUT with `site` and let the kernel end normally.
__global__ void bounded_wait_probe_kernel(int* err, int site) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, err, site);
}
}  // namespace

}  // namespace fvb

using namespace fvb;

extern "C" {

const char* fvb_status_string(int status) {
  switch (status) {
    case FVB_OK:
      return "FVB_OK";
    case FVB_ERR_INVALID_ARGUMENT:
      return "FVB_ERR_INVALID_ARGUMENT";
    case FVB_ERR_UNSUPPORTED:
      return "FVB_ERR_UNSUPPORTED";
    case FVB_ERR_MISALIGNED:
      return "FVB_ERR_MISALIGNED";
    case FVB_ERR_WORKSPACE_TOO_SMALL:
      return "FVB_ERR_WORKSPACE_TOO_SMALL";
    case FVB_ERR_CUDA:
      return "FVB_ERR_CUDA";
    case FVB_ERR_DEVICE_TIMEOUT:
      return "FVB_ERR_DEVICE_TIMEOUT";
    case FVB_ERR_BAD_PAGE:
      return "FVB_ERR_BAD_PAGE";
    case FVB_ERR_BAD_SLOT:
      return "FVB_ERR_BAD_SLOT";
    case FVB_ERR_NO_DEVICE_SUPPORT:
      return "FVB_ERR_NO_DEVICE_SUPPORT";
    default:
      return "FVB_ERR_UNKNOWN";
  }
}

int fvb_last_cuda_error(void) { return t_last_cuda_error; }

int fvb_kv_len_per_page(void) { return kPageSize; }
int fvb_dim_head(void) { return 128; }
int fvb_max_kv_len(void) { return 1 << 30; }

int fvb_read_device_error(int* code, int* info, void* stream) {
  if (!code || !info) return FVB_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = cuda_status(cudaStreamSynchronize(s));
  if (st) return st;
  int word[2] = {0, 0};
  st = cuda_status(cudaMemcpyFromSymbol(word, g_device_error, sizeof(word)));
  if (st) return st;
  *code = word[0];
  *info = word[1];
  const int zero[2] = {0, 0};
  return cuda_status(cudaMemcpyToSymbol(g_device_error, zero, sizeof(zero)));
}

int fvb_check_bounded_wait(int site, void* stream) {
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err, site);
  return cuda_status(cudaGetLastError());
}

int fvb_store_kvcache(const void* k, const void* v, int64_t token_stride, int64_t head_stride, void* k_pool,
                      void* v_pool, int64_t num_blocks, const int64_t* slot_mapping, int64_t num_tokens,
                      int n_kv_heads, int head_dim, int block_size, int dtype, void* stream) {
  TraceRange trace("fvb_store_kvcache");
  const int es = esize_of(dtype);
  if (es == 0) return FVB_ERR_UNSUPPORTED;
  if (num_tokens < 0 || n_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks < 0 ||
      token_stride < 0 || head_stride < 0)
    return FVB_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return FVB_OK;
  if (!k || !v || !k_pool || !v_pool || !slot_mapping) return FVB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(slot_mapping) & 7) != 0) return FVB_ERR_MISALIGNED;
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  return cuda_status(launch_store_kvcache(k, v, token_stride, head_stride, k_pool, v_pool, num_blocks, slot_mapping,
                                          num_tokens, n_kv_heads, head_dim, block_size, es, err,
                                          static_cast<cudaStream_t>(stream)));
}

int fvb_build_varlen_metadata(const int32_t* num_computed, const int32_t* num_new, int num_seqs,
                              const int32_t* flat_blocks, int64_t num_flat_blocks, const int32_t* cu_blocks,
                              int max_blocks_per_seq, int64_t num_tokens, int32_t* positions, int32_t* cu_seqlens,
                              int32_t* kv_lens, int32_t* block_tables, int64_t* slot_mapping, void* stream) {
  TraceRange trace("fvb_build_varlen_metadata");
  if (num_seqs <= 0 || num_tokens < 0 || max_blocks_per_seq < 0 || num_flat_blocks < 0 ||
      num_tokens >= (int64_t(1) << 31))
    return FVB_ERR_INVALID_ARGUMENT;
  if (!num_computed || !num_new || !cu_blocks || !cu_seqlens || !kv_lens) return FVB_ERR_INVALID_ARGUMENT;
  if (num_tokens > 0 && !positions) return FVB_ERR_INVALID_ARGUMENT;
  if (max_blocks_per_seq > 0 && !block_tables) return FVB_ERR_INVALID_ARGUMENT;
  if (num_flat_blocks > 0 && !flat_blocks) return FVB_ERR_INVALID_ARGUMENT;
  if (slot_mapping && (reinterpret_cast<uintptr_t>(slot_mapping) & 7) != 0) return FVB_ERR_MISALIGNED;
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  return cuda_status(launch_build_varlen_metadata(num_computed, num_new, num_seqs, flat_blocks, num_flat_blocks,
                                                  cu_blocks, max_blocks_per_seq, num_tokens, positions, cu_seqlens,
                                                  kv_lens, block_tables, slot_mapping, err,
                                                  static_cast<cudaStream_t>(stream)));
}

int fvb_qk_norm_rope_store(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
                           int64_t k_token_stride, int64_t k_head_stride, const void* v, int64_t v_token_stride,
                           int64_t v_head_stride, const void* q_norm_weight, const void* k_norm_weight, float eps,
                           const void* rope_cos, const void* rope_sin, int rope_rows, const int32_t* positions,
                           const int64_t* slot_mapping, int64_t num_tokens, int n_heads, int n_kv_heads,
                           int head_dim, void* q_out, void* k_pool, void* v_pool, int64_t num_blocks, int block_size,
                           int dtype, void* stream) {
  TraceRange trace("fvb_qk_norm_rope_store");
  const int es = esize_of(dtype);
  if (es == 0) return FVB_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return FVB_ERR_UNSUPPORTED;
  if (num_tokens < 0 || n_heads <= 0 || n_kv_heads <= 0 || rope_rows <= 0 || block_size <= 0 || num_blocks < 0 ||
      q_token_stride < 0 || q_head_stride < 0 || k_token_stride < 0 || k_head_stride < 0 || v_token_stride < 0 ||
      v_head_stride < 0 || !(eps >= 0.f) || eps > 1.f)
    return FVB_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return FVB_OK;
  if (num_tokens * (n_heads + 2 * int64_t(n_kv_heads)) >= (int64_t(1) << 31)) return FVB_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !q_norm_weight || !k_norm_weight || !rope_cos || !rope_sin || !positions || !slot_mapping ||
      !q_out || !k_pool || !v_pool)
    return FVB_ERR_INVALID_ARGUMENT;
  // One 16-byte vector per lane: every row start must be 16-byte aligned.
  const void* vec_ptrs[] = {q, k, v, q_norm_weight, k_norm_weight, rope_cos, rope_sin, q_out, k_pool, v_pool};
  for (const void* p : vec_ptrs) {
    if (!aligned16(p)) return FVB_ERR_MISALIGNED;
  }
  const int64_t strides[] = {q_token_stride, q_head_stride, k_token_stride, k_head_stride, v_token_stride,
                             v_head_stride};
  for (int64_t st : strides) {
    if ((st * es) % 16 != 0) return FVB_ERR_MISALIGNED;
  }
  if ((reinterpret_cast<uintptr_t>(slot_mapping) & 7) != 0 || (reinterpret_cast<uintptr_t>(positions) & 3) != 0)
    return FVB_ERR_MISALIGNED;
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  return cuda_status(launch_qk_norm_rope_store(
      q, q_token_stride, q_head_stride, k, k_token_stride, k_head_stride, v, v_token_stride, v_head_stride,
      q_norm_weight, k_norm_weight, eps, rope_cos, rope_sin, rope_rows, positions, slot_mapping, num_tokens, n_heads,
      n_kv_heads, head_dim, q_out, k_pool, v_pool, num_blocks, block_size, dtype, err,
      static_cast<cudaStream_t>(stream)));
}

size_t fvb_sample_workspace_size(int num_rows, int64_t vocab) {
  if (num_rows <= 0 || vocab <= 0) return 0;
  return sample_workspace_size(num_rows, vocab);
}

int fvb_sample_tokens(const void* logits, int64_t row_stride, int num_rows, int64_t vocab, int dtype,
                      const float* temperatures, const float* presence_penalties, const int64_t* token_table,
                      int64_t table_stride, int64_t table_len, uint64_t* rng_state, int64_t* token_ids,
                      void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("fvb_sample_tokens");
  const int es = esize_of(dtype);
  if (es == 0) return FVB_ERR_UNSUPPORTED;
  if (num_rows < 0 || vocab <= 0 || vocab >= (int64_t(1) << 31) || row_stride < vocab || table_len < 0 ||
      (table_len > 0 && (token_table == nullptr || table_stride < table_len)))
    return FVB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return FVB_OK;
  if (int64_t(num_rows) * ((vocab + 2047) / 2048) >= (int64_t(1) << 31)) return FVB_ERR_INVALID_ARGUMENT;
  if (!logits || !temperatures || !rng_state || !token_ids || !workspace) return FVB_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < sample_workspace_size(num_rows, vocab)) return FVB_ERR_WORKSPACE_TOO_SMALL;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0 || !aligned16(workspace) ||
      (reinterpret_cast<uintptr_t>(rng_state) & 7) != 0 || (reinterpret_cast<uintptr_t>(token_ids) & 7) != 0 ||
      (reinterpret_cast<uintptr_t>(temperatures) & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(presence_penalties) & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(token_table) & 7) != 0)
    return FVB_ERR_MISALIGNED;
  return cuda_status(launch_sample(logits, row_stride, num_rows, vocab, dtype, temperatures, presence_penalties,
                                   token_table, table_stride, table_len,
                                   reinterpret_cast<unsigned long long*>(rng_state), token_ids, workspace,
                                   static_cast<cudaStream_t>(stream)));
}

int fvb_build_slot_mapping(const int32_t* positions, int64_t num_tokens, const int32_t* cu_seqlens, int num_seqs,
                           const int32_t* block_tables, int max_blocks_per_seq, int block_size,
                           int64_t* slot_mapping, void* stream) {
  TraceRange trace("fvb_build_slot_mapping");
  if (num_tokens < 0 || num_seqs < 0 || max_blocks_per_seq < 0 || block_size <= 0) return FVB_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return FVB_OK;
  if (!positions || !block_tables || !slot_mapping || num_seqs == 0) return FVB_ERR_INVALID_ARGUMENT;
  if (!cu_seqlens && num_tokens > num_seqs) return FVB_ERR_INVALID_ARGUMENT;
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  return cuda_status(launch_build_slot_mapping(positions, num_tokens, cu_seqlens, num_seqs, block_tables,
                                               max_blocks_per_seq, block_size, slot_mapping, err,
                                               static_cast<cudaStream_t>(stream)));
}

size_t fvb_paged_attention_decode_workspace_size(int num_seqs, int n_heads, int n_kv_heads, int head_dim,
                                                 int max_kv_len) {
  if (num_seqs <= 0 || !gqa_ok(n_heads, n_kv_heads)) return 0;
  const size_t split_ws = plan_decode(num_seqs, n_heads, n_kv_heads, head_dim, max_kv_len, device_sm_count()).ws_bytes;
  if (!decode_on_tensor_cores(n_heads, n_kv_heads, FVB_DTYPE_BF16)) return split_ws;
  // 16-bit GQA >= 5 decodes on the tensor-core path (whose plan does not depend on the
  // dtype); fp32 keeps the split-KV plan.  The size covers both.
  const size_t tc_ws = plan_tc_decode(num_seqs, n_heads, n_kv_heads, head_dim, max_kv_len, device_sm_count()).ws_bytes;
  return split_ws > tc_ws ? split_ws : tc_ws;
}

int fvb_paged_attention_decode(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                               int n_heads, int n_kv_heads, int head_dim, int block_size, int num_seqs,
                               const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                               int max_kv_len, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  const QOLayout lay = head_major_layout(num_seqs, head_dim);
  return fvb_paged_attention_decode_strided(q, lay.q_ts, lay.q_hs, out, lay.o_ts, lay.o_hs, k_pool, v_pool,
                                            num_blocks, n_heads, n_kv_heads, head_dim, block_size, num_seqs,
                                            block_tables, max_blocks_per_seq, kv_lens, max_kv_len, dtype, workspace,
                                            workspace_bytes, stream);
}

int fvb_paged_attention_decode_strided(const void* q, int64_t q_token_stride, int64_t q_head_stride, void* out,
                                       int64_t out_token_stride, int64_t out_head_stride, const void* k_pool,
                                       const void* v_pool, int64_t num_blocks, int n_heads, int n_kv_heads,
                                       int head_dim, int block_size, int num_seqs, const int32_t* block_tables,
                                       int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, int dtype,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("fvb_paged_attention_decode_strided");
  int st = check_attention(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, block_size, num_seqs,
                           block_tables, max_blocks_per_seq, kv_lens, dtype);
  if (st) return st;
  const QOLayout lay{q_token_stride, q_head_stride, out_token_stride, out_head_stride};
  st = check_layout(lay, dtype);
  if (st) return st;
  if (num_seqs == 0) return FVB_OK;
  if (max_kv_len < 0 || int64_t(max_kv_len) > int64_t(max_blocks_per_seq) * kPageSize) return FVB_ERR_INVALID_ARGUMENT;
  if (decode_on_tensor_cores(n_heads, n_kv_heads, dtype)) {
    // One 128-row tile per (sequence, kv head) holds the group's n_rep heads: the
    // tcgen05 attention kernel in decode mode (no cu_seqlens / positions).
    const TcDecodePlan tp = plan_tc_decode(num_seqs, n_heads, n_kv_heads, head_dim, max_kv_len, device_sm_count());
    if (!workspace || workspace_bytes < tp.ws_bytes) return FVB_ERR_WORKSPACE_TOO_SMALL;
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return FVB_ERR_MISALIGNED;
    cudaError_t e;
    int* err = device_error_ptr(&e);
    if (!err) return cuda_status(e);
    return cuda_status(launch_tc_decode(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs,
                                        block_tables, max_blocks_per_seq, kv_lens, max_kv_len, dtype, tp, lay,
                                        workspace, err, static_cast<cudaStream_t>(stream)));
  }
  const DecodePlan plan = plan_decode(num_seqs, n_heads, n_kv_heads, head_dim, max_kv_len, device_sm_count());
  if (plan.ws_bytes > 0 && (!workspace || workspace_bytes < plan.ws_bytes)) return FVB_ERR_WORKSPACE_TOO_SMALL;
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255)) return FVB_ERR_MISALIGNED;
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  return cuda_status(launch_decode(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs,
                                   block_tables, max_blocks_per_seq, kv_lens, max_kv_len, dtype, plan, lay, workspace,
                                   err, static_cast<cudaStream_t>(stream)));
}

size_t fvb_paged_attention_prefill_workspace_size(int num_seqs, int n_heads, int n_kv_heads, int head_dim,
                                                  int64_t q_len_flatten, int max_q_len) {
  if (num_seqs <= 0 || !gqa_ok(n_heads, n_kv_heads)) return 0;
  // The tile plan (one int32 per sequence + 1) is the same for bf16 and f16;
  // the fp32 path needs none but accepts it.
  return plan_prefill(num_seqs, n_heads, n_kv_heads, head_dim, q_len_flatten, max_q_len, FVB_DTYPE_BF16).ws_bytes;
}

int fvb_paged_attention_prefill(const void* q, void* out, const void* k_pool, const void* v_pool,
                                int64_t num_blocks, int n_heads, int n_kv_heads, int head_dim, int block_size,
                                int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens, int max_q_len,
                                const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                                const int32_t* positions, int dtype, void* workspace, size_t workspace_bytes,
                                void* stream) {
  const QOLayout lay = head_major_layout(q_len_flatten, head_dim);
  return fvb_paged_attention_prefill_strided(q, lay.q_ts, lay.q_hs, out, lay.o_ts, lay.o_hs, k_pool, v_pool,
                                             num_blocks, n_heads, n_kv_heads, head_dim, block_size, num_seqs,
                                             q_len_flatten, cu_seqlens, max_q_len, block_tables, max_blocks_per_seq,
                                             kv_lens, positions, dtype, workspace, workspace_bytes, stream);
}

int fvb_paged_attention_prefill_strided(const void* q, int64_t q_token_stride, int64_t q_head_stride, void* out,
                                        int64_t out_token_stride, int64_t out_head_stride, const void* k_pool,
                                        const void* v_pool, int64_t num_blocks, int n_heads, int n_kv_heads,
                                        int head_dim, int block_size, int num_seqs, int64_t q_len_flatten,
                                        const int32_t* cu_seqlens, int max_q_len, const int32_t* block_tables,
                                        int max_blocks_per_seq, const int32_t* kv_lens, const int32_t* positions,
                                        int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  TraceRange trace("fvb_paged_attention_prefill_strided");
  int st = check_attention(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, block_size, num_seqs,
                           block_tables, max_blocks_per_seq, kv_lens, dtype);
  if (st) return st;
  const QOLayout lay{q_token_stride, q_head_stride, out_token_stride, out_head_stride};
  st = check_layout(lay, dtype);
  if (st) return st;
  if (q_len_flatten < 0 || max_q_len < 0) return FVB_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || q_len_flatten == 0) return FVB_OK;
  if (!cu_seqlens || !positions) return FVB_ERR_INVALID_ARGUMENT;
  if (q_len_flatten > int64_t(0x7fffffff)) return FVB_ERR_UNSUPPORTED;  // TMA token coordinate of q
  cudaError_t e;
  int* err = device_error_ptr(&e);
  if (!err) return cuda_status(e);
  if (dtype == FVB_DTYPE_F32) {
    return cuda_status(launch_prefill_simt(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim,
                                           num_seqs, q_len_flatten, cu_seqlens, block_tables, max_blocks_per_seq,
                                           kv_lens, positions, dtype, lay, err, static_cast<cudaStream_t>(stream)));
  }
  const PrefillPlan plan = plan_prefill(num_seqs, n_heads, n_kv_heads, head_dim, q_len_flatten, max_q_len, dtype);
  if (!workspace || workspace_bytes < plan.ws_bytes) return FVB_ERR_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return FVB_ERR_MISALIGNED;
  return cuda_status(launch_prefill(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, num_seqs,
                                    q_len_flatten, cu_seqlens, max_q_len, block_tables, max_blocks_per_seq, kv_lens,
                                    positions, dtype, plan, lay, workspace, err, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
