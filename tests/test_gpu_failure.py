"""A stalled pipeline is reported, not hung (GPU).

Every kernel here waits on mbarriers (TMA completions, MMA commits, softmax hand-offs)
with a bounded wait: after ~2 s it records FVB_ERR_DEVICE_TIMEOUT in the device error
word and the kernel ends.  fvb_check_bounded_wait runs that wait on a barrier nothing
completes; the host must read the timeout with its site, and the context must still run
real work correctly afterwards.  No fault, trap or endless loop is involved.
"""

import time

import numpy as np
import pytest
import torch

import cabi
import oracle
from femtovllm_b200 import capi, workloads

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_a_timeout_and_the_context_survives(cuda_device):
    lib = cabi.lib()
    cabi.read_device_error()
    t0 = time.monotonic()
    capi.check(lib.fvb_check_bounded_wait(0x1234, None), "fvb_check_bounded_wait")
    code, info = cabi.read_device_error()  # synchronizes
    waited = time.monotonic() - t0
    assert (code, info) == (6, 0x1234)  # FVB_ERR_DEVICE_TIMEOUT at the given site
    assert 1.0 < waited < 30.0
    # the same context runs a decode call correctly afterwards
    b = workloads.custom([100, 2000, 17], [1, 1, 1], 8, 2, 128, torch.bfloat16, seed=1).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    assert cabi.read_device_error() == (0, 0)
    ref = oracle.decode_attention(b.q.float().cpu().numpy(), b.k_pool.float().cpu().numpy(),
                                  b.v_pool.float().cpu().numpy(), b.block_tables, b.kv_lens)
    assert np.abs(out.float().cpu().numpy() - ref).max() < 2e-2
