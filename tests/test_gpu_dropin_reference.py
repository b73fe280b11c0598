"""Drop-in test through the reference's own attention module.

The reference package (installed under ``baseline/_ref``) is imported with this
repository's extension in place of its ``femtovllm._C`` (``oracle/reference_module.py``).
Its ``QwenSelfAttention.forward_varlen_custom_gemv`` / ``forward_varlen_custom_gemm``
(``femtovllm/models/qwen/qwen3.py:200-387``) then write the KV pools with their own
loops and call ``femtovllm.ops.paged_attention_gemv`` / ``_gemm``, which reach
``PagedAttentionGemvCuda`` / ``PagedAttentionGemmCuda`` of this repository unchanged.
Their outputs are compared with the reference's ``forward_varlen_pytorch``
(``qwen3.py:389-544``) run in fp32 on the same values, and the pools they wrote with
the pools the PyTorch path wrote, bit for bit.  The reference's default prefill (its
Triton kernel) is checked against the same fp32 result, so the tolerance is shown to
hold for the reference's own GPU path too.

Skipped when the reference is not installed on the box.
"""

import numpy as np
import pytest
import torch

from femtovllm_b200 import workloads
from oracle import reference_module

pytestmark = pytest.mark.gpu

if not reference_module.available():
    pytest.skip("the reference is not installed under baseline/_ref on this box", allow_module_level=True)

TOL = {torch.float32: (1e-4, 1e-4), torch.bfloat16: (2e-2, 2e-3)}


def _pytorch_fp32(attn, b, md):
    """forward_varlen_pytorch in fp32 (math SDPA, no TF32) on the batch's values; (out, k_pool, v_pool)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    x = reference_module.packed_input(b.q.float(), b.k_new.float(), b.v_new.float())
    kp, vp = b.k_pool.float().clone(), b.v_pool.float().clone()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad(), sdpa_kernel(SDPBackend.MATH):
            out, _ = attn.forward_varlen_pytorch(x, kp, vp, md)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    return out, kp, vp


def _custom(attn, b, md, route, impl_gemm=None):
    femtovllm, _, _, Impl = reference_module.import_reference()
    x = reference_module.packed_input(b.q, b.k_new, b.v_new)
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    saved = femtovllm._DEV.impl_custom_gemm, femtovllm._DEV.impl_custom_gemv
    femtovllm._DEV.impl_custom_gemm = impl_gemm or Impl.CUDA
    femtovllm._DEV.impl_custom_gemv = Impl.CUDA
    try:
        with torch.no_grad():
            fwd = attn.forward_varlen_custom_gemv if route == "gemv" else attn.forward_varlen_custom_gemm
            out, _ = fwd(x, kp, vp, md)
    finally:
        femtovllm._DEV.impl_custom_gemm, femtovllm._DEV.impl_custom_gemv = saved
    torch.cuda.synchronize()
    return out, kp, vp


def _close(got, ref, dtype, what):
    g = got.float()
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    err = (g - ref).abs()
    max_tol, mean_tol = TOL[dtype]
    assert err.max().item() <= max_tol, f"{what}: max abs {err.max().item():.3g}"
    assert err.mean().item() <= mean_tol, f"{what}: mean abs {err.mean().item():.3g}"


def _batch(name):
    if name == "config1_decode_fp32":
        return workloads.config1(), "gemv"
    if name == "decode_bf16_gqa2":
        return workloads.config2(num_seqs=24), "gemv"
    if name == "decode_bf16_gqa8":
        return workloads.custom([5000, 700, 3000, 33], [1, 1, 1, 1], 32, 4, 128, torch.bfloat16, seed=12,
                                qkv_scale=0.3), "gemv"
    if name == "chunked_prefill_bf16":
        return workloads.config3(num_seqs=6), "gemm"
    if name == "mixed_config4_bf16":
        return workloads.config4(), "gemm"
    raise KeyError(name)


CASES = ["config1_decode_fp32", "decode_bf16_gqa2", "decode_bf16_gqa8", "chunked_prefill_bf16", "mixed_config4_bf16"]


@pytest.mark.parametrize("name", CASES)
def test_reference_module_runs_on_this_extension(name, cuda_device):
    b, route = _batch(name)
    b.materialize(cuda_device)
    attn = reference_module.attention_module(b.n_heads, b.n_kv_heads, b.head_dim).to(cuda_device)
    md = reference_module.metadata(b.kv_lens, b.q_lens, b.block_tables, cuda_device)
    ref, kp_ref, vp_ref = _pytorch_fp32(attn, b, md)
    out, kp, vp = _custom(attn, b, md, route)
    _close(out, ref, b.dtype, f"{name} via femtovllm.ops -> this _C")
    # the custom route's own write loop and the PyTorch path's write put the same rows in the pools
    assert torch.equal(kp, kp_ref.to(b.dtype)) and torch.equal(vp, vp_ref.to(b.dtype))


@pytest.mark.parametrize("name", ["chunked_prefill_bf16", "mixed_config4_bf16"])
def test_reference_triton_prefill_meets_the_same_tolerance(name, cuda_device):
    """The reference's default prefill (its Triton kernel, femtovllm/ops/triton/paged_attention/
    paged_attention_gemm.py) against the same fp32 result: the harness and tolerance are sound."""
    pytest.importorskip("triton")
    _, _, _, Impl = reference_module.import_reference()
    b, _ = _batch(name)
    b.materialize(cuda_device)
    attn = reference_module.attention_module(b.n_heads, b.n_kv_heads, b.head_dim).to(cuda_device)
    md = reference_module.metadata(b.kv_lens, b.q_lens, b.block_tables, cuda_device)
    ref, _, _ = _pytorch_fp32(attn, b, md)
    out_triton, _, _ = _custom(attn, b, md, "gemm", impl_gemm=Impl.TRITON)
    _close(out_triton, ref, b.dtype, f"{name} reference Triton")
    out, _, _ = _custom(attn, b, md, "gemm")
    diff = (out.float() - out_triton.float()).abs()
    assert diff.max().item() <= 2 * TOL[b.dtype][0], diff.max().item()
    assert np.isfinite(diff.mean().item())
