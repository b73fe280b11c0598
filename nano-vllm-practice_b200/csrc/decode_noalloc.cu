// Decode paged attention for callers that cannot allocate device memory.
//
// The split-KV decode (decode.cu) keeps one fp32 partial output row and one
// log-sum-exp per (sequence, head, split) in a caller-provided workspace.
// Some callers cannot provide one at call time: an engine that reserves
// nearly all of HBM for its KV block pool at start-up and forbids further
// device allocations, or a host runtime whose device memory is owned by a
// different allocator and which may not call cudaMalloc / cudaFree on the
// decode path (cudaFree synchronizes the whole device).
//
// fvb_paged_attention_decode_noalloc takes the same arguments as
// fvb_paged_attention_decode minus the workspace, and uses instead the fixed
// array g_decode_scratch below (FVB_DECODE_NOALLOC_SCRATCH_BYTES = 32 MiB),
// which a GPU holds from the first call on it until the process exits.
//
// * Set-up: the first call on a device resolves the array's device address
//   with cudaGetSymbolAddress (with that device current) and caches it per
//   device ordinal.  Under CUDA's default lazy module loading this lookup is
//   also what loads the array onto the device, so make that first call before
//   any stream capture and before the engine reserves the rest of HBM for its
//   KV pool; a call with num_seqs = 0 does only this.  The cached address
//   belongs to the device's primary context (the one the runtime API uses).
// * Limit: a launch whose split plan needs more than 32 MiB of partials is
//   rejected with FVB_ERR_WORKSPACE_TOO_SMALL before anything runs (e.g. 8
//   sequences x 32 heads at 128k tokens still fit; 64 such sequences do not).
// * Sharing: every call on a device uses the same array and leaves the last
//   call's partials in it.  Nothing in it has to start at zero (each launch
//   writes every partial it later reads), but two calls whose kernels overlap
//   on the GPU (e.g. on two streams) race on it.
// * No cudaMalloc, cudaFree or allocating library routine is called.
#include <atomic>

#include "common.cuh"  // femtovllm_b200.h: the declaration and FVB_DECODE_NOALLOC_SCRATCH_BYTES

namespace fvb {
namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[FVB_DECODE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxScratchDevices = 64;
std::atomic<void*> g_scratch_addr[kMaxScratchDevices];

// Device address of g_decode_scratch on the current device; resolved once per device.
int scratch_for_current_device(void** addr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FVB_ERR_CUDA;
  if (dev < 0 || dev >= kMaxScratchDevices) return FVB_ERR_UNSUPPORTED;
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return FVB_ERR_CUDA;
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *addr = p;
  return FVB_OK;
}

}  // namespace
}  // namespace fvb

extern "C" int fvb_paged_attention_decode_noalloc(const void* q, void* out, const void* k_pool, const void* v_pool,
                                                  int64_t num_blocks, int n_heads, int n_kv_heads, int head_dim,
                                                  int block_size, int num_seqs, const int32_t* block_tables,
                                                  int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len,
                                                  int dtype, void* stream) {
  void* scratch = nullptr;
  const int st = fvb::scratch_for_current_device(&scratch);
  if (st != FVB_OK) return st;
  // Same validation, plan and kernels as the workspace entry point; the plan's
  // partials must fit the fixed array or the call is rejected unrun.
  return fvb_paged_attention_decode(q, out, k_pool, v_pool, num_blocks, n_heads, n_kv_heads, head_dim, block_size,
                                    num_seqs, block_tables, max_blocks_per_seq, kv_lens, max_kv_len, dtype, scratch,
                                    FVB_DECODE_NOALLOC_SCRATCH_BYTES, stream);
}
