"""q / out at (token, head) strides: the strided entry points and the ops' out_token_major.

The reference copies q into head-major order before the op
(femtovllm/ops/__init__.py:41-42) and copies the output back to token-major
order before o_proj (femtovllm/models/qwen/qwen3.py:278, 385).  The kernels
read q and write out through strides instead; the result must be bit-identical
to the head-major call (same arithmetic, other addresses).
"""

import ctypes

import pytest
import torch

import cabi
from femtovllm_b200 import capi, ops, workloads

pytestmark = pytest.mark.gpu


def _thd_views(b):
    """q as the projection emits it: a (T, Hq, D) buffer, seen as (Hq, T, D)."""
    q_thd = b.q.transpose(0, 1).contiguous()
    return q_thd, q_thd.transpose(0, 1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_prefill_token_major_equals_head_major(dtype, cuda_device):
    b = workloads.custom([300, 17, 1, 900], [300, 1, 1, 77], 16, 8, 128, dtype, seed=21).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    ref = ops.paged_attention_gemm(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], int(b.q_lens.max()), 32, None, None,
                                   md["block_tables"], md["kv_lens"], md["positions"])
    _, q_view = _thd_views(b)
    out = ops.paged_attention_gemm(q_view, b.k_pool, b.v_pool, md["cu_seqlens"], int(b.q_lens.max()), 32, None, None,
                                   md["block_tables"], md["kv_lens"], md["positions"], out_token_major=True)
    assert out.shape == ref.shape and out.transpose(0, 1).is_contiguous()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("nrep", [2, 4])
def test_decode_token_major_equals_head_major(nrep, cuda_device):
    b = workloads.custom([40, 4000, 1, 1024], [1, 1, 1, 1], 8 * nrep, 8, 128, torch.bfloat16, seed=nrep).materialize(
        cuda_device)
    md = b.device_metadata(cuda_device)
    ref = ops.paged_attention_gemv(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    _, q_view = _thd_views(b)
    out = ops.paged_attention_gemv(q_view, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len,
                                   out_token_major=True)
    assert out.transpose(0, 1).is_contiguous() and torch.equal(out, ref)
    o = torch.ops.femtovllm_b200.paged_attention_decode(q_view, b.k_pool, b.v_pool, md["block_tables"],
                                                        md["kv_lens"], b.max_kv_len, True)
    assert torch.equal(o, ref)


def test_c_abi_strided_entry_points(cuda_device):
    b = workloads.custom([100, 33], [100, 1], 16, 8, 128, torch.bfloat16, seed=3).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    T, H, D = b.num_tokens, 16, 128
    ref = cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], int(b.q_lens.max()), md["block_tables"],
                       md["kv_lens"], md["positions"])
    q_thd = b.q.transpose(0, 1).contiguous()
    out_thd = torch.empty(T, H, D, dtype=b.dtype, device=cuda_device)
    lib = cabi.lib()
    wsb = lib.fvb_paged_attention_prefill_workspace_size(b.num_seqs, H, 8, D, T, int(b.q_lens.max()))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=cuda_device)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(q_ts, o_ts):
        return lib.fvb_paged_attention_prefill_strided(
            q_thd.data_ptr(), q_ts, D, out_thd.data_ptr(), o_ts, D, b.k_pool.data_ptr(), b.v_pool.data_ptr(),
            b.num_blocks, H, 8, D, 16, b.num_seqs, T, md["cu_seqlens"].data_ptr(), int(b.q_lens.max()),
            md["block_tables"].data_ptr(), md["block_tables"].shape[1], md["kv_lens"].data_ptr(),
            md["positions"].data_ptr(), capi.dtype_code(b.dtype), ws.data_ptr(), wsb, s)

    capi.check(call(H * D, H * D), "prefill_strided")
    assert torch.equal(out_thd.transpose(0, 1), ref)
    assert call(H * D + 4, H * D) == 3  # FVB_ERR_MISALIGNED: rows 8 bytes off a 16-byte boundary
    assert call(-1, H * D) == 1  # FVB_ERR_INVALID_ARGUMENT
