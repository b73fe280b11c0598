/*
 * femtovllm_b200.h - C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in replacement for the native entry points of fishAndShrimp/
 * nano-vllm-practice ("FemtoVLLM") on its attention path.  All functions take
 * plain device pointers, sizes and a CUDA stream (as void*), never allocate,
 * and return an fvb_status.  Tensor layouts are the reference's:
 *
 *   K/V pool    [num_blocks][n_kv_heads][block_size = 16][head_dim], contiguous
 *               (femtovllm/engine/core_engine.py:140-162)
 *   q, out      [n_heads][q_len_flatten][head_dim], contiguous ("head-major",
 *               femtovllm/ops/__init__.py:82-156)
 *   block table int32 [num_seqs][max_blocks_per_seq], -1 padded
 *               (femtovllm/engine/model_runner.py:46-72)
 *   kv_lens, positions, cu_seqlens: int32
 *
 * dtype codes: FVB_DTYPE_F32, FVB_DTYPE_BF16, FVB_DTYPE_F16.
 * head_dim: 64 or 128.  n_heads / n_kv_heads (GQA group): any whole group, 1 to 16 and
 * beyond (tiles hold 1, 2, 4, 8 or 16 heads; groups of 3, 5, 6, 7 pad to the next tile).
 */
#ifndef FEMTOVLLM_B200_H_
#define FEMTOVLLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FVB_API __attribute__((visibility("default")))
#else
#define FVB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FVB_DTYPE_F32 = 0,
  FVB_DTYPE_BF16 = 1,
  FVB_DTYPE_F16 = 2,
};

typedef enum fvb_status {
  FVB_OK = 0,
  FVB_ERR_INVALID_ARGUMENT = 1,   /* null pointer, negative size, inconsistent shapes */
  FVB_ERR_UNSUPPORTED = 2,        /* dtype / head_dim / GQA group / block_size not built */
  FVB_ERR_MISALIGNED = 3,         /* a pointer or stride breaks the 16-byte rule */
  FVB_ERR_WORKSPACE_TOO_SMALL = 4,
  FVB_ERR_CUDA = 5,               /* a CUDA runtime call failed (see fvb_last_cuda_error) */
  FVB_ERR_DEVICE_TIMEOUT = 6,     /* a bounded device-side wait gave up */
  FVB_ERR_BAD_PAGE = 7,           /* block-table entry < 0 or >= num_blocks inside kv_len */
  FVB_ERR_BAD_SLOT = 8,           /* slot_mapping entry >= num_blocks * block_size */
  FVB_ERR_NO_DEVICE_SUPPORT = 9,  /* the current device is not sm_100 */
} fvb_status;

/* Human-readable name of a status code (static storage). */
FVB_API const char* fvb_status_string(int status);

/* Last CUDA runtime error code seen by an entry point on this thread (0 if none). */
FVB_API int fvb_last_cuda_error(void);

/* Compile-time contract constants, exported like femtovllm._C's attributes
 * (csrc/bindings.cpp:62-66: kKVLenPerPage, kDimHead, kMaxKVLenNonSplit).
 * fvb_max_kv_len() replaces kMaxKVLenNonSplit = 8192
 * (csrc/utils/constants.cuh:39): decode here is split-KV, so the only limit is
 * the int32 indexing of the block table. */
FVB_API int fvb_kv_len_per_page(void);
FVB_API int fvb_dim_head(void);
FVB_API int fvb_max_kv_len(void);

/* Read and clear the device error word that kernels set when they meet a bad
 * page or slot, or give up a bounded wait.  Synchronizes `stream`.
 * *code = 0 when nothing was recorded; *info is the first failing index/site. */
FVB_API int fvb_read_device_error(int* code, int* info, void* stream);

/*
 * Diagnostic: launches one thread that waits, through the bounded mbarrier wait all kernels here use,
 * on a barrier nothing completes.  The wait gives up after its limit (2 s), records
 * FVB_ERR_DEVICE_TIMEOUT with info = site in the device error word (fvb_read_device_error) and the
 * kernel ends normally, so the context stays usable.  Shows how a stalled pipeline is reported instead
 * of hanging the GPU.  No counterpart in the reference.
 */
FVB_API int fvb_check_bounded_wait(int site, void* stream);

/*
 * store_kvcache: pool[slot / 16][h][slot % 16][:] = new[t][h][:] for K and V.
 *
 * Replaces the Python KV-write loops of QwenSelfAttention
 * (femtovllm/models/qwen/qwen3.py:240-264 decode, 322-366 prefill,
 * 450-490 PyTorch path), which have no native counterpart in the reference.
 * slot_mapping[t] = block_table[s][pos_t / 16] * 16 + pos_t % 16, int64;
 * -1 skips the token.  k / v: [num_tokens][n_kv_heads][head_dim] with
 * element strides (token_stride, head_stride, 1).  Bit-exact copy.  The pool
 * may use any page size block_size > 0 (16 above stands for it); the
 * attention entry points read pools of 16-token pages only.
 */
FVB_API int fvb_store_kvcache(const void* k, const void* v, int64_t token_stride, int64_t head_stride,
                      void* k_pool, void* v_pool, int64_t num_blocks, const int64_t* slot_mapping,
                      int64_t num_tokens, int n_kv_heads, int head_dim, int block_size, int dtype,
                      void* stream);

/*
 * Next-token sampling over num_rows logit rows (two kernel launches, one pass over the logits): the
 * reference's Sampler.forward (femtovllm/engine/sampler.py:15-114), which the model runner calls on lm_head's output
 * (femtovllm/engine/model_runner.py:150-157).  Row b: logits[b * row_stride + i], i < vocab.
 *   apply = any |presence_penalties[r]| > 1e-5 over all rows (sampler.py:31-35);
 *   x[i] = logits[b][i] - presence_penalties[b] if apply and token i occurs in
 *          token_table[b][0 .. table_len) (entries outside [0, vocab) are padding, the reference
 *          pads with vocab), else logits[b][i]                          (sampler.py:56-76)
 *   temperatures[b] < 1e-5: token_ids[b] = first index of the maximum of x  (torch.argmax, :88-95)
 *   otherwise: token_ids[b] drawn from softmax(x / temperatures[b])         (:97-109), by inverse CDF
 *          over vocabulary order with the uniform of Philox4x32-10(key = rng_state[0],
 *          counter = {b, 0, rng_state[1]}); x / T is rounded to the logits' dtype when !apply, as the
 *          reference's in-place division of 16-bit logits does.
 * presence_penalties may be NULL (no penalty); token_table int64 [num_rows][table_stride].
 * rng_state: device uint64[2] {seed, offset}; each launch adds 1 to offset, on the device.
 * workspace: fvb_sample_workspace_size(num_rows, vocab) bytes, 16-byte aligned; its first 4 bytes
 * (reserved) must be zero before the first launch (e.g. cudaMemsetAsync once) and every launch leaves them
 * zero.
 * Replaces the reference's Python lists, count matrix and per-group launches; no counterpart in its
 * native module.
 */
FVB_API size_t fvb_sample_workspace_size(int num_rows, int64_t vocab);
FVB_API int fvb_sample_tokens(const void* logits, int64_t row_stride, int num_rows, int64_t vocab, int dtype,
                              const float* temperatures, const float* presence_penalties,
                              const int64_t* token_table, int64_t table_stride, int64_t table_len,
                              uint64_t* rng_state, int64_t* token_ids, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * slot_mapping[t] = block_tables[s][positions[t] / 16] * 16 + positions[t] % 16 for every
 * token t of sequence s (cu_seqlens[s] <= t < cu_seqlens[s+1]); -1 where the table entry
 * is -1 (the token is then skipped by fvb_store_kvcache).  cu_seqlens may be NULL for one
 * token per sequence (decode).  The index arithmetic of the reference's KV-write loops
 * (femtovllm/models/qwen/qwen3.py:250-264 decode, 335-361 prefill) on the device; the
 * reference builds no slot mapping of its own (its metadata is assembled on the host in
 * femtovllm/engine/model_runner.py:159-339).
 */
FVB_API int fvb_build_slot_mapping(const int32_t* positions, int64_t num_tokens, const int32_t* cu_seqlens,
                                   int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                                   int block_size, int64_t* slot_mapping, void* stream);

/*
 * Varlen attention metadata from per-sequence counts, on the device.  For sequence s with
 * num_computed[s] cached and num_new[s] new tokens (decode: num_new[s] = 1):
 *   cu_seqlens[s + 1] = num_new[0] + ... + num_new[s], cu_seqlens[0] = 0          (num_seqs + 1 entries)
 *   kv_lens[s] = num_computed[s] + num_new[s]                                      (num_seqs entries)
 *   positions[t] = num_computed[s] + t - cu_seqlens[s] for each new token t of s   (num_tokens entries)
 *   block_tables[s][i] = flat_blocks[cu_blocks[s] + i] for i < cu_blocks[s+1] - cu_blocks[s], else -1
 *                                                                   (num_seqs x max_blocks_per_seq, int32)
 *   slot_mapping[t] (optional, may be NULL) as fvb_build_slot_mapping.
 * The host loops of ModelRunner._route_prefill / _route_decode
 * (femtovllm/engine/model_runner.py:186-205, 280-290) and pad_block_tables (:46-72), which build these as
 * Python lists each step.  num_tokens (the sum of num_new) and max_blocks_per_seq (the widest row) are the
 * caller's, as the scheduler knows them; a mismatch or a malformed cu_blocks row is recorded in the device
 * error word (FVB_ERR_INVALID_ARGUMENT) and never read out of bounds.  Two launches, no host synchronization.
 */
FVB_API int fvb_build_varlen_metadata(const int32_t* num_computed, const int32_t* num_new, int num_seqs,
                                      const int32_t* flat_blocks, int64_t num_flat_blocks,
                                      const int32_t* cu_blocks, int max_blocks_per_seq, int64_t num_tokens,
                                      int32_t* positions, int32_t* cu_seqlens, int32_t* kv_lens,
                                      int32_t* block_tables, int64_t* slot_mapping, void* stream);

/*
 * Fused q/k RMSNorm + rotary embedding + KV-cache write, one pass over the projection outputs:
 *   q_out[h][t][:]                      = rope(rmsnorm(q[t][h][:]) * q_norm_weight)
 *   k_pool[slot / 16][h][slot % 16][:]  = rope(rmsnorm(k[t][h][:]) * k_norm_weight)
 *   v_pool[slot / 16][h][slot % 16][:]  = v[t][h][:]   (bit-exact)
 * rmsnorm(x) = x / sqrt(mean(x^2) + eps) over head_dim (nn.RMSNorm, femtovllm/models/qwen/qwen3.py:181-183);
 * rope(y)[d] = y[d] * cos[p][d] + (d < D/2 ? -y[d + D/2] : y[d - D/2]) * sin[p][d] with p = positions[t]
 * (QwenRotaryEmbedding.forward, qwen3.py:53-138; rope_cos / rope_sin are its [rope_rows][head_dim]
 * buffers, in `dtype`).  Replaces qwen3.py:234-238 plus the KV-write loops (qwen3.py:240-264, 322-366)
 * and the q transpose + contiguous copy before the attention op (qwen3.py:270, 372;
 * femtovllm/ops/__init__.py:41-42): q_out is [n_heads][num_tokens][head_dim], the layout
 * fvb_paged_attention_decode / _prefill take.  q / k / v are [num_tokens][heads][head_dim] with element
 * strides (token_stride, head_stride, 1), e.g. views into one fused qkv projection output; every row
 * start and every pointer must be 16-byte aligned.  slot_mapping as for fvb_store_kvcache (-1 skips the
 * K/V write of a token; q_out is written regardless).  head_dim 64 or 128.  A position outside
 * [0, rope_rows) records FVB_ERR_INVALID_ARGUMENT in the device error word and leaves that row unwritten.
 */
FVB_API int fvb_qk_norm_rope_store(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
                                   int64_t k_token_stride, int64_t k_head_stride, const void* v,
                                   int64_t v_token_stride, int64_t v_head_stride, const void* q_norm_weight,
                                   const void* k_norm_weight, float eps, const void* rope_cos, const void* rope_sin,
                                   int rope_rows, const int32_t* positions, const int64_t* slot_mapping,
                                   int64_t num_tokens, int n_heads, int n_kv_heads, int head_dim, void* q_out,
                                   void* k_pool, void* v_pool, int64_t num_blocks, int block_size, int dtype,
                                   void* stream);

/*
 * Decode paged attention (one query token per sequence), split-KV.
 *
 * Replaces PagedAttentionGemvCuda (csrc/paged_attention/paged_attention_gemv.cu:223-308,
 * bound at csrc/bindings.cpp:52-59; Python wrapper femtovllm/ops/__init__.py:82-107).
 * q, out: [n_heads][num_seqs][head_dim]; out[h][b] = softmax(q k^T / sqrt(D)) v over
 * keys 0 .. kv_lens[b]-1 of kv head h / (n_heads / n_kv_heads).
 * max_kv_len must be >= every kv_lens[b] (the reference passes it from the host).
 * workspace: device buffer of at least fvb_paged_attention_decode_workspace_size() bytes.
 */
FVB_API size_t fvb_paged_attention_decode_workspace_size(int num_seqs, int n_heads, int n_kv_heads, int head_dim,
                                                 int max_kv_len);
FVB_API int fvb_paged_attention_decode(const void* q, void* out, const void* k_pool, const void* v_pool,
                               int64_t num_blocks, int n_heads, int n_kv_heads, int head_dim, int block_size,
                               int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                               const int32_t* kv_lens, int max_kv_len, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * fvb_paged_attention_decode / _prefill with q and out at any (token, head) strides, in elements:
 * element (t, h, d) of q is q[t * q_token_stride + h * q_head_stride + d], likewise for out.  The reference
 * op layout (n_heads, T, D) is strides (D, T * D); the projection / o_proj layout (T, n_heads, D) is
 * (n_heads * D, D).  With the latter, the copies the reference makes around the op (q.transpose(0, 1) +
 * .contiguous(), femtovllm/ops/__init__.py:41-42; attn.transpose(0, 1).contiguous() before o_proj,
 * femtovllm/models/qwen/qwen3.py:278, 385) are not needed.  Every stride times the element size must be a
 * multiple of 16 bytes.  Workspace sizes as for the unstrided entry points.
 */
FVB_API int fvb_paged_attention_decode_strided(const void* q, int64_t q_token_stride, int64_t q_head_stride,
                                               void* out, int64_t out_token_stride, int64_t out_head_stride,
                                               const void* k_pool, const void* v_pool, int64_t num_blocks,
                                               int n_heads, int n_kv_heads, int head_dim, int block_size,
                                               int num_seqs, const int32_t* block_tables, int max_blocks_per_seq,
                                               const int32_t* kv_lens, int max_kv_len, int dtype, void* workspace,
                                               size_t workspace_bytes, void* stream);
FVB_API int fvb_paged_attention_prefill_strided(const void* q, int64_t q_token_stride, int64_t q_head_stride,
                                                void* out, int64_t out_token_stride, int64_t out_head_stride,
                                                const void* k_pool, const void* v_pool, int64_t num_blocks,
                                                int n_heads, int n_kv_heads, int head_dim, int block_size,
                                                int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens,
                                                int max_q_len, const int32_t* block_tables, int max_blocks_per_seq,
                                                const int32_t* kv_lens, const int32_t* positions, int dtype,
                                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode paged attention without a caller-provided workspace.  No counterpart
 * in the reference.  For callers that cannot allocate device memory when they
 * call: an engine that has reserved nearly all HBM for its KV block pool, or a
 * host runtime that may not call cudaMalloc / cudaFree on the decode path
 * (cudaFree synchronizes the device).  Same arguments and result as
 * fvb_paged_attention_decode minus the workspace: the split partials live in a
 * fixed FVB_DECODE_NOALLOC_SCRATCH_BYTES (32 MiB) array inside the library,
 * which a GPU holds from the first call on it until the process exits.  A
 * launch whose partials need more is rejected unrun with
 * FVB_ERR_WORKSPACE_TOO_SMALL.  The first call on a device looks up the array's
 * device address (with CUDA's default lazy module loading, that is also when
 * the 32 MiB are taken on the device), so make that call before any stream
 * capture and before the KV pool reserves the rest of HBM: a warm-up call with
 * num_seqs = 0 does it and runs nothing.  The address is cached per device
 * ordinal, so it is valid in the runtime's primary context of that device (the
 * context the CUDA runtime and PyTorch use); a caller that switches to its own
 * driver-API contexts must not use this entry point.  All calls on a device
 * share the array (nothing in it needs to start at zero), so calls whose
 * kernels overlap on the GPU race.  Allocates nothing.
 */
#define FVB_DECODE_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
FVB_API int fvb_paged_attention_decode_noalloc(const void* q, void* out, const void* k_pool, const void* v_pool,
                                               int64_t num_blocks, int n_heads, int n_kv_heads, int head_dim,
                                               int block_size, int num_seqs, const int32_t* block_tables,
                                               int max_blocks_per_seq, const int32_t* kv_lens, int max_kv_len,
                                               int dtype, void* stream);

/*
 * Varlen chunked-prefill causal attention over paged, prefix-cached KV.
 *
 * Replaces PagedAttentionGemmCuda (csrc/paged_attention/paged_attention_gemm.cu:304-394,
 * bound at csrc/bindings.cpp:41-50) and the default Triton prefill
 * paged_attention_gemm_triton (femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:165-235);
 * Python wrapper femtovllm/ops/__init__.py:110-156.
 * q, out: [n_heads][q_len_flatten][head_dim]; sequence s owns query tokens
 * cu_seqlens[s] .. cu_seqlens[s+1]-1; query i sees key j iff j < kv_lens[s] and
 * j <= positions[i].  Sequences with one new token (decode rows) may be mixed in
 * the same launch (the reference's unified CUSTOM_GEMM route, qwen3.py:575-581).
 * bf16 / f16 run on tcgen05 tensor cores; f32 runs on a SIMT fp32 kernel.
 */
FVB_API size_t fvb_paged_attention_prefill_workspace_size(int num_seqs, int n_heads, int n_kv_heads, int head_dim,
                                                  int64_t q_len_flatten, int max_q_len);
FVB_API int fvb_paged_attention_prefill(const void* q, void* out, const void* k_pool, const void* v_pool,
                                int64_t num_blocks, int n_heads, int n_kv_heads, int head_dim, int block_size,
                                int num_seqs, int64_t q_len_flatten, const int32_t* cu_seqlens, int max_q_len,
                                const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                                const int32_t* positions, int dtype, void* workspace, size_t workspace_bytes,
                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FEMTOVLLM_B200_H_ */
