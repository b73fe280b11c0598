// femtovllm_b200._C: the PyTorch face of libfemtovllm_b200.so.
//
// Mirrors the reference's native module femtovllm._C (csrc/bindings.cpp:41-66):
// the same entry-point names and argument order (PagedAttentionGemvCuda,
// PagedAttentionGemmCuda) and the same attributes (kMaxKVLenNonSplit,
// kKVLenPerPage, kDimHead), plus StoreKVCacheCuda for the slot-mapped KV write
// the reference does in Python, QKNormRopeStoreCuda for the fused q/k norm +
// rotary embedding + KV write and SampleTokensCuda for the sampler.  Each
// function validates like the reference's TORCH_CHECKs (csrc/paged_attention/paged_attention_gemv.cu:231-274,
// paged_attention_gemm.cu:314-358), allocates the output (and the split-KV
// workspace) with the caching allocator, and calls the C ABI on the current
// CUDA stream.  The same functions are also registered as torch.ops.femtovllm_b200.*.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime_api.h>
#include <torch/extension.h>

#include "femtovllm_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat:
      return FVB_DTYPE_F32;
    case at::kBFloat16:
      return FVB_DTYPE_BF16;
    case at::kHalf:
      return FVB_DTYPE_F16;
    default:
      TORCH_CHECK(false, "femtovllm_b200: unsupported dtype ", t, " (float32, bfloat16, float16)");
  }
  return -1;
}

void check_status(int st, const char* what) {
  if (st == FVB_OK) return;
  if (st == FVB_ERR_CUDA) {
    const int ce = fvb_last_cuda_error();
    TORCH_CHECK(false, what, " failed: ", fvb_status_string(st), " (", cudaGetErrorString(cudaError_t(ce)), ")");
  }
  TORCH_CHECK(false, what, " failed: ", fvb_status_string(st));
}

// out of shape (n_heads, T, D): head-major memory, or a transposed view of a
// (T, n_heads, D) buffer when token_major (then out.transpose(0, 1) is contiguous).
at::Tensor new_out(const at::Tensor& q, bool token_major) {
  if (!token_major) return torch::empty({q.size(0), q.size(1), q.size(2)}, q.options());
  return torch::empty({q.size(1), q.size(0), q.size(2)}, q.options()).transpose(0, 1);
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

void check_pools(const at::Tensor& q, const at::Tensor& k_pool, const at::Tensor& v_pool) {
  TORCH_CHECK(q.is_cuda() && k_pool.is_cuda() && v_pool.is_cuda(), "q, k_pool and v_pool must be CUDA tensors");
  TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1, "d_head must be the contiguous dimension of q");
  TORCH_CHECK(k_pool.is_contiguous() && v_pool.is_contiguous(), "k_pool and v_pool must be contiguous");
  TORCH_CHECK(q.dim() == 3, "q must be (n_heads, q_len_flatten, d_head)");
  TORCH_CHECK(k_pool.dim() == 4 && v_pool.dim() == 4, "pools must be (num_blocks, n_kv_heads, block_size, d_head)");
  TORCH_CHECK(q.size(-1) == k_pool.size(-1) && q.size(-1) == v_pool.size(-1), "d_head mismatch");
  for (int i = 0; i < 4; ++i) TORCH_CHECK(k_pool.size(i) == v_pool.size(i), "k_pool / v_pool shape mismatch");
  TORCH_CHECK(q.scalar_type() == k_pool.scalar_type() && q.scalar_type() == v_pool.scalar_type(),
              "q, k_pool and v_pool must share a dtype");
  TORCH_CHECK(q.get_device() == k_pool.get_device() && q.get_device() == v_pool.get_device(),
              "q and the pools must be on one device");
}

}  // namespace

torch::Tensor PagedAttentionGemvCuda(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                                     torch::Tensor kv_page_tables, torch::Tensor kv_lens, int64_t max_kv_len,
                                     bool out_token_major) {
  check_pools(q, k_pool, v_pool);
  TORCH_CHECK(kv_page_tables.scalar_type() == torch::kInt32 && kv_lens.scalar_type() == torch::kInt32,
              "kv_page_tables and kv_lens must be int32");
  TORCH_CHECK(kv_page_tables.is_cuda() && kv_lens.is_cuda(), "kv_page_tables and kv_lens must be CUDA tensors");
  TORCH_CHECK(kv_page_tables.dim() == 2 && kv_page_tables.is_contiguous(), "kv_page_tables must be (B, max_blocks)");
  TORCH_CHECK(kv_lens.is_contiguous(), "kv_lens must be contiguous");
  const int n_heads = int(q.size(0));
  const int num_seqs = int(q.size(1));
  const int head_dim = int(q.size(2));
  TORCH_CHECK(kv_page_tables.size(0) == num_seqs && kv_lens.numel() == num_seqs,
              "one block table row and one kv_len per sequence");
  c10::cuda::CUDAGuard guard(q.device());
  auto out = new_out(q, out_token_major);
  const size_t ws_bytes = fvb_paged_attention_decode_workspace_size(num_seqs, n_heads, int(k_pool.size(1)), head_dim,
                                                                    int(max_kv_len));
  torch::Tensor ws;
  if (ws_bytes > 0) ws = torch::empty({int64_t(ws_bytes)}, q.options().dtype(torch::kUInt8));
  check_status(fvb_paged_attention_decode_strided(q.data_ptr(), q.stride(1), q.stride(0), out.data_ptr(),
                                                  out.stride(1), out.stride(0), k_pool.data_ptr(), v_pool.data_ptr(),
                                                  k_pool.size(0), n_heads, int(k_pool.size(1)), head_dim,
                                          int(k_pool.size(2)), num_seqs, kv_page_tables.data_ptr<int32_t>(),
                                          int(kv_page_tables.size(1)), kv_lens.data_ptr<int32_t>(), int(max_kv_len),
                                          dtype_code(q.scalar_type()), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                                          stream_of(q)),
               "PagedAttentionGemvCuda");
  return out;
}

torch::Tensor PagedAttentionGemmCuda(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                                     torch::Tensor cu_seqlens, int64_t max_q_len, torch::Tensor kv_page_tables,
                                     torch::Tensor kv_lens, torch::Tensor positions, bool out_token_major) {
  check_pools(q, k_pool, v_pool);
  for (const auto* t : {&cu_seqlens, &kv_page_tables, &kv_lens, &positions}) {
    TORCH_CHECK(t->scalar_type() == torch::kInt32, "metadata tensors must be int32");
    TORCH_CHECK(t->is_cuda() && t->is_contiguous(), "metadata tensors must be contiguous CUDA tensors");
  }
  const int num_seqs = int(cu_seqlens.numel()) - 1;
  TORCH_CHECK(num_seqs >= 0, "cu_seqlens must have num_seqs + 1 entries");
  TORCH_CHECK(kv_page_tables.dim() == 2 && kv_page_tables.size(0) == num_seqs, "kv_page_tables must be (B, max_blocks)");
  TORCH_CHECK(kv_lens.numel() == num_seqs, "one kv_len per sequence");
  const int n_heads = int(q.size(0));
  const int64_t q_len_flatten = q.size(1);
  const int head_dim = int(q.size(2));
  TORCH_CHECK(positions.numel() == q_len_flatten, "one position per query token");
  c10::cuda::CUDAGuard guard(q.device());
  auto out = new_out(q, out_token_major);
  const size_t ws_bytes = fvb_paged_attention_prefill_workspace_size(num_seqs, n_heads, int(k_pool.size(1)), head_dim,
                                                                     q_len_flatten, int(max_q_len));
  torch::Tensor ws;
  if (ws_bytes > 0) ws = torch::empty({int64_t(ws_bytes)}, q.options().dtype(torch::kUInt8));
  check_status(fvb_paged_attention_prefill_strided(q.data_ptr(), q.stride(1), q.stride(0), out.data_ptr(),
                                                   out.stride(1), out.stride(0), k_pool.data_ptr(),
                                                   v_pool.data_ptr(), k_pool.size(0), n_heads, int(k_pool.size(1)),
                                                   head_dim,
                                           int(k_pool.size(2)), num_seqs, q_len_flatten,
                                           cu_seqlens.data_ptr<int32_t>(), int(max_q_len),
                                           kv_page_tables.data_ptr<int32_t>(), int(kv_page_tables.size(1)),
                                           kv_lens.data_ptr<int32_t>(), positions.data_ptr<int32_t>(),
                                           dtype_code(q.scalar_type()), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                                           stream_of(q)),
               "PagedAttentionGemmCuda");
  return out;
}

void StoreKVCacheCuda(torch::Tensor k, torch::Tensor v, torch::Tensor k_pool, torch::Tensor v_pool,
                      torch::Tensor slot_mapping) {
  TORCH_CHECK(k.is_cuda() && v.is_cuda() && k_pool.is_cuda() && v_pool.is_cuda() && slot_mapping.is_cuda(),
              "all arguments must be CUDA tensors");
  TORCH_CHECK(k.dim() == 3 && v.dim() == 3, "k and v must be (num_tokens, n_kv_heads, d_head)");
  TORCH_CHECK(k.sizes() == v.sizes() && k.strides() == v.strides(), "k and v must have one shape and stride");
  TORCH_CHECK(k.stride(2) == 1, "d_head must be the contiguous dimension of k and v");
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.sizes() == v_pool.sizes(), "pools must be (num_blocks, Hkv, 16, d_head)");
  TORCH_CHECK(k_pool.is_contiguous() && v_pool.is_contiguous(), "pools must be contiguous");
  TORCH_CHECK(k_pool.size(1) == k.size(1) && k_pool.size(3) == k.size(2), "pool and k head shapes differ");
  TORCH_CHECK(k.scalar_type() == k_pool.scalar_type() && v.scalar_type() == v_pool.scalar_type() &&
                  k.scalar_type() == v.scalar_type(),
              "k, v and the pools must share a dtype");
  TORCH_CHECK(slot_mapping.scalar_type() == torch::kInt64 && slot_mapping.is_contiguous() &&
                  slot_mapping.numel() == k.size(0),
              "slot_mapping must be a contiguous int64 tensor with one entry per token");
  c10::cuda::CUDAGuard guard(k.device());
  check_status(fvb_store_kvcache(k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k_pool.data_ptr(),
                                 v_pool.data_ptr(), k_pool.size(0), slot_mapping.data_ptr<int64_t>(), k.size(0),
                                 int(k.size(1)), int(k.size(2)), int(k_pool.size(2)), dtype_code(k.scalar_type()),
                                 stream_of(k)),
               "StoreKVCacheCuda");
}

// positions, cu_seqlens, kv_lens, -1-padded block tables and slot mapping from
// per-sequence counts and a flat block list (cu_blocks: exclusive scan of the row lengths).
std::vector<torch::Tensor> BuildVarlenMetadataCuda(torch::Tensor num_computed, torch::Tensor num_new,
                                                   torch::Tensor flat_blocks, torch::Tensor cu_blocks,
                                                   int64_t max_blocks_per_seq, int64_t num_tokens) {
  for (const auto* t : {&num_computed, &num_new, &flat_blocks, &cu_blocks}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(),
                "num_computed, num_new, flat_blocks and cu_blocks must be contiguous int32 CUDA tensors");
  }
  const int64_t B = num_computed.numel();
  TORCH_CHECK(B > 0 && num_new.numel() == B && cu_blocks.numel() == B + 1, "one count per sequence, B + 1 cu_blocks");
  c10::cuda::CUDAGuard guard(num_computed.device());
  auto opt = num_computed.options();
  auto positions = torch::empty({num_tokens}, opt);
  auto cu_seqlens = torch::empty({B + 1}, opt);
  auto kv_lens = torch::empty({B}, opt);
  auto tables = torch::empty({B, max_blocks_per_seq}, opt);
  auto slots = torch::empty({num_tokens}, opt.dtype(torch::kInt64));
  check_status(fvb_build_varlen_metadata(num_computed.data_ptr<int32_t>(), num_new.data_ptr<int32_t>(), int(B),
                                         flat_blocks.numel() ? flat_blocks.data_ptr<int32_t>() : nullptr,
                                         flat_blocks.numel(), cu_blocks.data_ptr<int32_t>(), int(max_blocks_per_seq),
                                         num_tokens, num_tokens ? positions.data_ptr<int32_t>() : nullptr,
                                         cu_seqlens.data_ptr<int32_t>(), kv_lens.data_ptr<int32_t>(),
                                         max_blocks_per_seq ? tables.data_ptr<int32_t>() : nullptr,
                                         num_tokens ? slots.data_ptr<int64_t>() : nullptr, stream_of(num_computed)),
               "BuildVarlenMetadataCuda");
  return {positions, cu_seqlens, kv_lens, tables, slots};
}

// Fused q/k RMSNorm + rotary embedding + KV write; returns q in the head-major
// (n_heads, num_tokens, d_head) layout the attention ops take.
torch::Tensor QKNormRopeStoreCuda(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor q_norm_weight,
                                  torch::Tensor k_norm_weight, double eps, torch::Tensor rope_cos,
                                  torch::Tensor rope_sin, torch::Tensor positions, torch::Tensor k_pool,
                                  torch::Tensor v_pool, torch::Tensor slot_mapping) {
  const std::vector<at::Tensor> all = {q, k, v, q_norm_weight, k_norm_weight, rope_cos, rope_sin, positions,
                                       k_pool, v_pool, slot_mapping};
  for (const auto& t : all) TORCH_CHECK(t.is_cuda() && t.get_device() == q.get_device(), "all arguments must be CUDA tensors on one device");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q, k, v must be (num_tokens, heads, d_head)");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1, "d_head must be the contiguous dimension of q, k, v");
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(2) == k.size(2), "q / k / v shapes differ");
  const int64_t D = q.size(2);
  TORCH_CHECK(q_norm_weight.dim() == 1 && k_norm_weight.dim() == 1 && q_norm_weight.numel() == D &&
                  k_norm_weight.numel() == D && q_norm_weight.is_contiguous() && k_norm_weight.is_contiguous(),
              "norm weights must be contiguous (d_head,) tensors");
  TORCH_CHECK(rope_cos.dim() == 2 && rope_cos.sizes() == rope_sin.sizes() && rope_cos.size(1) == D &&
                  rope_cos.is_contiguous() && rope_sin.is_contiguous(),
              "rope_cos / rope_sin must be contiguous (rows, d_head) tensors");
  TORCH_CHECK(positions.scalar_type() == torch::kInt32 && positions.is_contiguous() && positions.numel() == q.size(0),
              "positions must be a contiguous int32 tensor with one entry per token");
  TORCH_CHECK(slot_mapping.scalar_type() == torch::kInt64 && slot_mapping.is_contiguous() &&
                  slot_mapping.numel() == q.size(0),
              "slot_mapping must be a contiguous int64 tensor with one entry per token");
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.sizes() == v_pool.sizes() && k_pool.is_contiguous() && v_pool.is_contiguous(),
              "pools must be contiguous (num_blocks, n_kv_heads, block_size, d_head)");
  TORCH_CHECK(k_pool.size(1) == k.size(1) && k_pool.size(3) == D, "pool and k head shapes differ");
  const auto dt = q.scalar_type();
  for (const auto& t : {k, v, q_norm_weight, k_norm_weight, rope_cos, rope_sin, k_pool, v_pool})
    TORCH_CHECK(t.scalar_type() == dt, "q, k, v, the norm weights, the rope tables and the pools must share a dtype");
  c10::cuda::CUDAGuard guard(q.device());
  auto q_out = torch::empty({q.size(1), q.size(0), D}, q.options());
  check_status(fvb_qk_norm_rope_store(q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
                                      v.data_ptr(), v.stride(0), v.stride(1), q_norm_weight.data_ptr(),
                                      k_norm_weight.data_ptr(), float(eps), rope_cos.data_ptr(), rope_sin.data_ptr(),
                                      int(rope_cos.size(0)), positions.data_ptr<int32_t>(),
                                      slot_mapping.data_ptr<int64_t>(), q.size(0), int(q.size(1)), int(k.size(1)),
                                      int(D), q_out.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.size(0),
                                      int(k_pool.size(2)), dtype_code(dt), stream_of(q)),
               "QKNormRopeStoreCuda");
  return q_out;
}

torch::Tensor BuildSlotMappingCuda(torch::Tensor positions, std::optional<torch::Tensor> cu_seqlens,
                                  torch::Tensor block_tables) {
  TORCH_CHECK(positions.is_cuda() && block_tables.is_cuda(), "positions and block_tables must be CUDA tensors");
  TORCH_CHECK(positions.scalar_type() == torch::kInt32 && block_tables.scalar_type() == torch::kInt32,
              "positions and block_tables must be int32");
  TORCH_CHECK(positions.is_contiguous() && block_tables.is_contiguous() && block_tables.dim() == 2,
              "positions must be contiguous, block_tables (num_seqs, max_blocks) contiguous");
  int num_seqs = int(block_tables.size(0));
  const int32_t* cu = nullptr;
  if (cu_seqlens.has_value()) {
    TORCH_CHECK(cu_seqlens->is_cuda() && cu_seqlens->scalar_type() == torch::kInt32 && cu_seqlens->is_contiguous(),
                "cu_seqlens must be a contiguous int32 CUDA tensor");
    TORCH_CHECK(cu_seqlens->numel() == num_seqs + 1, "cu_seqlens must have num_seqs + 1 entries");
    cu = cu_seqlens->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard guard(positions.device());
  auto slots = torch::empty({positions.numel()}, positions.options().dtype(torch::kInt64));
  check_status(fvb_build_slot_mapping(positions.data_ptr<int32_t>(), positions.numel(), cu, num_seqs,
                                      block_tables.data_ptr<int32_t>(), int(block_tables.size(1)), 16,
                                      slots.data_ptr<int64_t>(), stream_of(positions)),
               "BuildSlotMappingCuda");
  return slots;
}

// Next-token ids (int64, (B,)) from logits (B, vocab): the reference's Sampler.forward
// (femtovllm/engine/sampler.py:15-114) with device tensors in place of its Python lists.
// rng_state: int64 (2,) {seed, offset} on the device, advanced by one per call.  workspace:
// optional uint8 buffer of fvb_sample_workspace_size bytes, zero before its first use
// (kept zero by every call); a fresh zeroed one is allocated when absent.
torch::Tensor SampleTokensCuda(torch::Tensor logits, torch::Tensor temperatures,
                               c10::optional<torch::Tensor> presence_penalties,
                               c10::optional<torch::Tensor> token_table, torch::Tensor rng_state,
                               c10::optional<torch::Tensor> workspace) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1,
              "logits must be a (B, vocab) CUDA tensor with contiguous rows");
  const int64_t B = logits.size(0), V = logits.size(1);
  TORCH_CHECK(temperatures.is_cuda() && temperatures.scalar_type() == torch::kFloat32 &&
                  temperatures.is_contiguous() && temperatures.numel() == B,
              "temperatures must be a contiguous float32 CUDA tensor of B entries");
  const float* pens = nullptr;
  if (presence_penalties.has_value()) {
    TORCH_CHECK(presence_penalties->is_cuda() && presence_penalties->scalar_type() == torch::kFloat32 &&
                    presence_penalties->is_contiguous() && presence_penalties->numel() == B,
                "presence_penalties must be a contiguous float32 CUDA tensor of B entries");
    pens = presence_penalties->data_ptr<float>();
  }
  const int64_t* table = nullptr;
  int64_t table_stride = 0, table_len = 0;
  if (token_table.has_value() && token_table->numel() > 0) {
    TORCH_CHECK(token_table->is_cuda() && token_table->scalar_type() == torch::kInt64 && token_table->dim() == 2 &&
                    token_table->size(0) == B && token_table->stride(1) == 1,
                "token_table must be an int64 (B, table_len) CUDA tensor with contiguous rows");
    table = token_table->data_ptr<int64_t>();
    table_stride = token_table->stride(0);
    table_len = token_table->size(1);
  }
  TORCH_CHECK(rng_state.is_cuda() && rng_state.scalar_type() == torch::kInt64 && rng_state.numel() == 2 &&
                  rng_state.is_contiguous(),
              "rng_state must be a contiguous int64 CUDA tensor {seed, offset}");
  c10::cuda::CUDAGuard guard(logits.device());
  const size_t ws_bytes = fvb_sample_workspace_size(int(B), V);
  torch::Tensor ws;
  if (workspace.has_value()) {
    ws = *workspace;
    TORCH_CHECK(ws.is_cuda() && ws.is_contiguous() && size_t(ws.nbytes()) >= ws_bytes,
                "workspace must be a contiguous CUDA buffer of at least ", ws_bytes, " bytes");
  } else {
    ws = torch::zeros({int64_t(ws_bytes > 0 ? ws_bytes : 1)}, logits.options().dtype(torch::kUInt8));
  }
  auto out = torch::empty({B}, logits.options().dtype(torch::kInt64));
  check_status(fvb_sample_tokens(logits.data_ptr(), logits.stride(0), int(B), V, dtype_code(logits.scalar_type()),
                                 temperatures.data_ptr<float>(), pens, table, table_stride, table_len,
                                 reinterpret_cast<uint64_t*>(rng_state.data_ptr<int64_t>()), out.data_ptr<int64_t>(),
                                 ws.data_ptr(), size_t(ws.nbytes()), stream_of(logits)),
               "SampleTokensCuda");
  return out;
}

int64_t SampleWorkspaceSize(int64_t num_rows, int64_t vocab) {
  return int64_t(fvb_sample_workspace_size(int(num_rows), vocab));
}

std::tuple<int64_t, int64_t> ReadDeviceError() {
  int code = 0, info = 0;
  check_status(fvb_read_device_error(&code, &info,
                                     static_cast<void*>(at::cuda::getCurrentCUDAStream().stream())),
               "ReadDeviceError");
  return {code, info};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.attr("kMaxKVLenNonSplit") = fvb_max_kv_len();
  m.attr("kKVLenPerPage") = fvb_kv_len_per_page();
  m.attr("kDimHead") = fvb_dim_head();
  m.def("PagedAttentionGemvCuda", &PagedAttentionGemvCuda, "decode paged attention (split-KV, sm_100a)",
        py::arg("q"), py::arg("k_pool"), py::arg("v_pool"), py::arg("kv_page_tables"), py::arg("kv_lens"),
        py::arg("max_kv_len"), py::arg("out_token_major") = false);
  m.def("PagedAttentionGemmCuda", &PagedAttentionGemmCuda, "varlen chunked-prefill paged attention (sm_100a)",
        py::arg("q"), py::arg("k_pool"), py::arg("v_pool"), py::arg("cu_seqlens"), py::arg("max_q_len"),
        py::arg("kv_page_tables"), py::arg("kv_lens"), py::arg("positions"), py::arg("out_token_major") = false);
  m.def("StoreKVCacheCuda", &StoreKVCacheCuda, "slot-mapped KV-cache write");
  m.def("BuildSlotMappingCuda", &BuildSlotMappingCuda, "slot of every new token from positions and block tables",
        py::arg("positions"), py::arg("cu_seqlens") = py::none(), py::arg("block_tables"));
  m.def("BuildVarlenMetadataCuda", &BuildVarlenMetadataCuda,
        "positions, cu_seqlens, kv_lens, padded block tables and slot mapping from per-sequence counts");
  m.def("QKNormRopeStoreCuda", &QKNormRopeStoreCuda,
        "fused q/k RMSNorm + rotary embedding + KV-cache write; returns q as (n_heads, num_tokens, d_head)");
  m.def("SampleTokensCuda", &SampleTokensCuda,
        "next-token ids: presence penalty, greedy argmax / temperature sampling (one pass over the logits)", py::arg("logits"),
        py::arg("temperatures"), py::arg("presence_penalties") = py::none(), py::arg("token_table") = py::none(),
        py::arg("rng_state"), py::arg("workspace") = py::none());
  m.def("SampleWorkspaceSize", &SampleWorkspaceSize, "workspace bytes of SampleTokensCuda");
  m.def("ReadDeviceError", &ReadDeviceError, "read and clear the device error word (synchronizes)");
}

TORCH_LIBRARY(femtovllm_b200, m) {
  m.def(
      "paged_attention_decode(Tensor q, Tensor k_pool, Tensor v_pool, Tensor block_tables, Tensor kv_lens, "
      "int max_kv_len, bool out_token_major=False) -> Tensor");
  m.def(
      "paged_attention_prefill(Tensor q, Tensor k_pool, Tensor v_pool, Tensor cu_seqlens, int max_q_len, "
      "Tensor block_tables, Tensor kv_lens, Tensor positions, bool out_token_major=False) -> Tensor");
  m.def("store_kvcache(Tensor k, Tensor v, Tensor(a!) k_pool, Tensor(b!) v_pool, Tensor slot_mapping) -> ()");
  m.def("build_slot_mapping(Tensor positions, Tensor? cu_seqlens, Tensor block_tables) -> Tensor");
  m.def(
      "qk_norm_rope_store(Tensor q, Tensor k, Tensor v, Tensor q_norm_weight, Tensor k_norm_weight, float eps, "
      "Tensor rope_cos, Tensor rope_sin, Tensor positions, Tensor(a!) k_pool, Tensor(b!) v_pool, "
      "Tensor slot_mapping) -> Tensor");
  m.def(
      "build_varlen_metadata(Tensor num_computed, Tensor num_new, Tensor flat_blocks, Tensor cu_blocks, "
      "int max_blocks_per_seq, int num_tokens) -> Tensor[]");
  m.def(
      "sample_tokens(Tensor logits, Tensor temperatures, Tensor? presence_penalties, Tensor? token_table, "
      "Tensor(a!) rng_state, Tensor(b!)? workspace) -> Tensor");
}

TORCH_LIBRARY_IMPL(femtovllm_b200, CUDA, m) {
  m.impl("paged_attention_decode", &PagedAttentionGemvCuda);
  m.impl("paged_attention_prefill", &PagedAttentionGemmCuda);
  m.impl("store_kvcache", &StoreKVCacheCuda);
  m.impl("build_slot_mapping", &BuildSlotMappingCuda);
  m.impl("qk_norm_rope_store", &QKNormRopeStoreCuda);
  m.impl("build_varlen_metadata", &BuildVarlenMetadataCuda);
  m.impl("sample_tokens", &SampleTokensCuda);
}
