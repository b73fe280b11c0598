"""fvb_paged_attention_decode_noalloc: decode without a caller-provided workspace.

Callers that cannot allocate device memory at call time (an engine that has
reserved nearly all HBM for its KV block pool, or a host runtime that may not
call cudaMalloc / cudaFree on the decode path) use this entry point; it keeps
the split-KV partials in a fixed 32 MiB array inside the library instead.
These tests call it through the C ABI and compare it with the workspace entry
point on the same inputs, twice in a row (the second call reuses the array the
first one left behind).  This file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

import cabi
from femtovllm_b200 import capi, workloads

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 * 1024 * 1024
FVB_ERR_WORKSPACE_TOO_SMALL = 4


def _noalloc_fn():
    lib = cabi.lib()
    fn = lib.fvb_paged_attention_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] + [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_int,
                                                                                   ctypes.c_void_p, ctypes.c_int,
                                                                                   ctypes.c_int, ctypes.c_void_p]
    return fn


def decode_noalloc(q, k_pool, v_pool, tables, kv_lens, max_kv_len):
    hq, b, d = q.shape
    out = torch.empty_like(q)
    st = _noalloc_fn()(
        q.data_ptr(), out.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0], hq, k_pool.shape[1], d,
        k_pool.shape[2], b, tables.data_ptr(), tables.shape[1], kv_lens.data_ptr(), int(max_kv_len),
        capi.dtype_code(q.dtype), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    return st, out


# config 2 / config 1: the SIMT split-KV route; the GQA-8 case of few long sequences: the
# tcgen05 route with split-KV, whose tile plan and partials both live in the scratch array.
CASES = {
    "config2_bf16_gqa2": lambda: workloads.config2(),
    "config1_fp32_gqa4": lambda: workloads.config1(),
    "gqa8_bf16_tensor_core_split": lambda: workloads.custom([8192, 7000, 8100, 6001], [1, 1, 1, 1], 32, 4, 128,
                                                            torch.bfloat16, seed=8),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_matches_workspace_entry_point_on_two_calls(case, cuda_device):
    b = CASES[case]().materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    ws_bytes = cabi.lib().fvb_paged_attention_decode_workspace_size(b.num_seqs, b.n_heads, b.n_kv_heads, b.head_dim,
                                                                    b.max_kv_len)
    assert ws_bytes <= SCRATCH_BYTES
    ref = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    for _ in range(2):
        st, out = decode_noalloc(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
        assert st == 0, capi.STATUS_NAMES.get(st, st)
        torch.cuda.synchronize()
        # the same plan and kernels run on the same inputs: the outputs are bit-identical
        assert torch.isfinite(out.float()).all()
        assert torch.equal(out, ref)
    assert cabi.read_device_error() == (0, 0)


def test_noalloc_warm_up_call_with_no_sequences(cuda_device):
    """num_seqs = 0 resolves the array's address (loading it on the device) and runs nothing."""
    z = torch.zeros(1, dtype=torch.bfloat16, device=cuda_device)
    t = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    st = _noalloc_fn()(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, 8, 2, 128, 16, 0, t.data_ptr(), 1,
                       t.data_ptr(), 0, capi.dtype_code(torch.bfloat16),
                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0


def test_noalloc_rejects_a_plan_larger_than_its_scratch(cuda_device):
    # 64 sequences x 32 heads at 131072 tokens need ~135 MB of split partials.
    hq, hkv, d, n = 32, 8, 128, 64
    max_kv = 131072
    q = torch.zeros(hq, n, d, dtype=torch.bfloat16, device=cuda_device)
    pool = torch.zeros(1, hkv, 16, d, dtype=torch.bfloat16, device=cuda_device)
    tables = torch.zeros(n, max_kv // 16, dtype=torch.int32, device=cuda_device)
    lens = torch.full((n,), max_kv, dtype=torch.int32, device=cuda_device)
    need = cabi.lib().fvb_paged_attention_decode_workspace_size(n, hq, hkv, d, max_kv)
    assert need > SCRATCH_BYTES
    st, _ = decode_noalloc(q, pool, pool, tables, lens, max_kv)
    assert st == FVB_ERR_WORKSPACE_TOO_SMALL
    assert np.isscalar(st)
