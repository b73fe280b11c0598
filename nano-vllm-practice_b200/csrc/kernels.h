// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

namespace fvb {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize, bytes) for kernel Kern once per
// device (bytes is fixed per kernel), keeping the driver call off every launch.
template <auto Kern>
cudaError_t set_smem_once(int bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return ce;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  ce = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (ce == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return ce;
}

// Host-side encoder for 2-D tiled TMA descriptors (cuTensorMapEncodeTiled,
// resolved through the runtime's driver entry point so nothing links libcuda).
// rows x cols elements, row pitch `row_bytes`, box {box_cols, box_rows},
// 128-byte swizzle when swizzle128 is set.
cudaError_t make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols,
                        uint64_t rows, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// The same encoder for a 3-D box: dims {d0, d1, d2} elements, byte strides of
// dims 1 and 2 (multiples of 16, in any order), box {b0, b1, b2}.
cudaError_t make_tma_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims[3],
                        const uint64_t stride_bytes[2], const uint32_t box[3], bool swizzle128);

// Where q and out live: element (token t, head h, d) at t * ts + h * hs + d.
// Head-major (n_heads, T, D), the reference op layout, is {D, T * D}; the
// projection / o_proj layout (T, n_heads, D) is {n_heads * D, D}.
struct QOLayout {
  int64_t q_ts, q_hs, o_ts, o_hs;
};
inline QOLayout head_major_layout(int64_t tokens, int head_dim) {
  return QOLayout{head_dim, tokens * head_dim, head_dim, tokens * head_dim};
}

cudaError_t launch_store_kvcache(const void* k, const void* v, int64_t token_stride, int64_t head_stride,
                                 void* k_pool, void* v_pool, int64_t num_blocks, const int64_t* slot_mapping,
                                 int64_t num_tokens, int n_kv_heads, int head_dim, int block_size, int esize,
                                 int* err, cudaStream_t stream);

cudaError_t launch_build_slot_mapping(const int32_t* positions, int64_t num_tokens, const int32_t* cu_seqlens,
                                      int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                                      int block_size, int64_t* slot_mapping, int* err, cudaStream_t stream);

// Split-KV plan of one decode launch.  Deterministic in its inputs and the
// device's SM count, so the workspace size can be asked for ahead of the call.
// Query heads one decode CTA serves: the GQA group size rounded up to 1, 2, 4 or 8.
// Larger groups are served in chunks of 8 heads (K/V read once per chunk).
inline int decode_tile_heads(int group) { return group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8; }
// Query heads of one 128-row tensor-core tile (128 / heads tokens each): the GQA group
// rounded up to a power of two, at most 16 (8 tokens, one 1024-byte swizzle atom per head).
inline int tc_tile_heads(int group) { return group <= 8 ? decode_tile_heads(group) : 16; }

struct DecodePlan {
  int pages_per_split;  // multiple of the 2-page stage
  int max_splits;       // ceil(ceil(max_kv_len / 16) / pages_per_split)
  size_t ws_bytes;      // partial outputs + log-sum-exps
};
DecodePlan plan_decode(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int max_kv_len, int num_sms);

cudaError_t launch_decode(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                          int n_heads, int n_kv_heads, int head_dim, int num_seqs, const int32_t* block_tables,
                          int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, int dtype,
                          const DecodePlan& plan, const QOLayout& lay, void* workspace, int* err,
                          cudaStream_t stream, const int32_t* q_index = nullptr, const int32_t* q_pos = nullptr);
// With q_index (a prefill batch's cu_seqlens) and q_pos (its positions), launch_decode
// serves only the sequences with exactly one query token, row q_index[s] at position
// q_pos[row], and leaves every other sequence's rows untouched.  That launch is a
// programmatic dependent of the kernel before it on the stream (the tensor-core prefill
// kernel, which writes only the other rows) and completes after it.

// Splits of the decode plan that serves a prefill batch's single-token sequences: the
// prefill workspace reserves partials for this many splits per (sequence, head).
constexpr int kSingleRowMaxSplits = 16;

struct PrefillPlan {
  int tile_tokens;      // query tokens per tile (128 / GQA group on the tensor-core path)
  int64_t max_tiles;    // upper bound on query tiles over all sequences
  bool single_rows_apart;  // single-token sequences go to the split-KV decode kernel
  size_t off_single;       // their split partials in the workspace
  size_t ws_bytes;
};
PrefillPlan plan_prefill(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int64_t q_len_flatten,
                         int max_q_len, int dtype);

cudaError_t launch_prefill(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                           int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                           const int32_t* cu_seqlens, int max_q_len, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* kv_lens, const int32_t* positions, int dtype,
                           const PrefillPlan& plan, const QOLayout& lay, void* workspace, int* err,
                           cudaStream_t stream);

// One-CTA work plan of the tensor-core prefill kernels (prefill_sm100.cu): sequences by
// descending kv_len, and the scan of work items of `tiles_per_item` query tiles each
// (none for single-token sequences when skip_single is set).
cudaError_t launch_prefill_plan(const int32_t* cu_seqlens, const int32_t* kv_lens, int num_seqs, int tile_tokens,
                                int tiles_per_item, int32_t* order, int32_t* cu_items, cudaStream_t stream,
                                int skip_single = 0);

// Decode on the tensor-core attention kernel (decode mode: token s of sequence s at
// position kv_len - 1), with split-KV when there are too few (sequence, kv head) CTAs.
struct TcDecodePlan {
  PrefillPlan base;     // one work item per sequence
  int tiles_per_split;  // 128-key tiles per split; 0 = no split
  int max_splits;
  size_t off_o, off_lse;  // fp32 partials [seq][head][split][D] and log2-sum-exps in the workspace
  size_t ws_bytes;
};
TcDecodePlan plan_tc_decode(int num_seqs, int n_heads, int n_kv_heads, int head_dim, int max_kv_len, int num_sms);
cudaError_t launch_tc_decode(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                             int n_heads, int n_kv_heads, int head_dim, int num_seqs, const int32_t* block_tables,
                             int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len, int dtype,
                             const TcDecodePlan& plan, const QOLayout& lay, void* workspace, int* err,
                             cudaStream_t stream);
// Merge split partials (decode.cu): sequences with more than one split of
// pages_per_split pages; the others were written directly.
cudaError_t launch_decode_combine(const float* ws_o, const float* ws_lse, void* out, const int32_t* kv_lens,
                                  int kv_cap, int num_seqs, int n_heads, int head_dim, int pages_per_split,
                                  int max_splits, int dtype, const QOLayout& lay, cudaStream_t stream);

cudaError_t launch_prefill_simt(const void* q, void* out, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                int n_heads, int n_kv_heads, int head_dim, int num_seqs, int64_t q_len_flatten,
                                const int32_t* cu_seqlens, const int32_t* block_tables, int max_blocks_per_seq,
                                const int32_t* kv_lens, const int32_t* positions, int dtype, const QOLayout& lay,
                                int* err, cudaStream_t stream);

// Fused q/k RMSNorm + rotary embedding + K/V pool write (qk_norm_rope.cu).
// Strides are in elements; q_out is [n_heads][num_tokens][head_dim].
cudaError_t launch_qk_norm_rope_store(const void* q, int64_t q_ts, int64_t q_hs, const void* k, int64_t k_ts,
                                      int64_t k_hs, const void* v, int64_t v_ts, int64_t v_hs, const void* q_w,
                                      const void* k_w, float eps, const void* cos_t, const void* sin_t, int rope_rows,
                                      const int32_t* positions, const int64_t* slot_mapping, int64_t num_tokens,
                                      int n_heads, int n_kv_heads, int head_dim, void* q_out, void* k_pool,
                                      void* v_pool, int64_t num_blocks, int block_size, int dtype, int* err,
                                      cudaStream_t stream);

// Varlen metadata from per-sequence counts (metadata.cu); slot_mapping may be null.
cudaError_t launch_build_varlen_metadata(const int32_t* num_computed, const int32_t* num_new, int num_seqs,
                                         const int32_t* flat_blocks, int64_t num_flat_blocks, const int32_t* cu_blocks,
                                         int max_blocks_per_seq, int64_t num_tokens, int32_t* positions,
                                         int32_t* cu_seqlens, int32_t* kv_lens, int32_t* block_tables,
                                         int64_t* slot_mapping, int* err, cudaStream_t stream);

// Next-token sampling (sampler.cu): presence penalty, greedy argmax, temperature
// sampling (two launches); the workspace counter is zero before the first launch and left zero.
size_t sample_workspace_size(int num_rows, int64_t vocab);
cudaError_t launch_sample(const void* logits, int64_t row_stride, int num_rows, int64_t vocab, int dtype,
                          const float* temps, const float* pens, const int64_t* table, int64_t table_stride,
                          int64_t table_len, unsigned long long* rng, int64_t* out, void* workspace,
                          cudaStream_t stream);

int device_sm_count();

}  // namespace fvb
