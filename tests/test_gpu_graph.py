"""A decode step captured in a CUDA graph and replayed (GPU).

Small-batch decode is launch-bound, so an engine captures its step once and
replays it (the reference's engine runs it eagerly, step by step:
femtovllm/engine/model_runner.py:97-114).  The step here is the whole
attention path of one layer: slot mapping from positions and block tables,
the fused q/k norm + rotary embedding + KV write, and split-KV decode
attention.  Each replay after new inputs were copied into the captured
tensors must equal an eager run of the same step on the same inputs, bit for
bit (the kernels are deterministic: no atomics, fixed split plan), including
the pool rows the step writes.
"""

import numpy as np
import pytest
import torch

import oracle
from femtovllm_b200 import ops, workloads

pytestmark = pytest.mark.gpu


def _step_inputs(B, dev, seed, max_ctx):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, max_ctx - 8, size=B)
    # room in every table for 8 more tokens than the first step needs
    b = workloads.custom(ctx + 8, np.ones(B, np.int32), 16, 8, 128, torch.bfloat16, seed=seed).materialize(dev)
    T, Hq, Hkv, D = B, 16, 8, 128
    x = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).to(torch.bfloat16)
    cos, sin = oracle.rope_tables(max_ctx + 16, D)
    st = {
        "x": x,
        "q": x[:, : Hq * D].view(T, Hq, D),
        "k": x[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D),
        "v": x[:, (Hq + Hkv) * D :].view(T, Hkv, D),
        "q_w": (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16),
        "k_w": (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16),
        "cos": torch.from_numpy(cos).to(dev, torch.bfloat16),
        "sin": torch.from_numpy(sin).to(dev, torch.bfloat16),
        "positions": torch.from_numpy(ctx.astype(np.int32)).to(dev),  # the new token sits at position ctx
        "kv_lens": torch.from_numpy((ctx + 1).astype(np.int32)).to(dev),
        "block_tables": torch.from_numpy(b.block_tables).to(dev),
        "k_pool": b.k_pool,
        "v_pool": b.v_pool,
    }
    return st


def _step(st, max_kv_len):
    slots = ops.build_slot_mapping(st["positions"], st["block_tables"])
    q_hm = ops.qk_norm_rope_store(st["q"], st["k"], st["v"], st["q_w"], st["k_w"], 1e-6, st["cos"], st["sin"],
                                  st["positions"], st["k_pool"], st["v_pool"], slots)
    return ops.paged_attention_gemv(q_hm, st["k_pool"], st["v_pool"], st["block_tables"], st["kv_lens"], max_kv_len)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_decode_step_replays_in_a_cuda_graph(B, cuda_device):
    max_ctx = 4096
    st = _step_inputs(B, cuda_device, seed=100 + B, max_ctx=max_ctx)
    # One bound for every replay, the table capacity; the kernels read the real kv_lens on the device.
    max_kv_len = st["block_tables"].shape[1] * 16
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            _step(st, max_kv_len)  # warm-up: per-device setup happens outside the capture
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _step(st, max_kv_len)
    for it in range(4):
        # next decode step: new projections, every sequence one token longer
        st["x"].copy_(torch.randn_like(st["x"], dtype=torch.float32).to(torch.bfloat16))
        st["positions"].add_(1)
        st["kv_lens"].add_(1)
        kp0, vp0 = st["k_pool"].clone(), st["v_pool"].clone()
        g.replay()
        torch.cuda.synchronize()
        got, kp_g, vp_g = out.clone(), st["k_pool"].clone(), st["v_pool"].clone()
        st["k_pool"].copy_(kp0)
        st["v_pool"].copy_(vp0)
        ref = _step(st, max_kv_len)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), it
        assert torch.equal(kp_g, st["k_pool"]) and torch.equal(vp_g, st["v_pool"]), it
    del g


@pytest.mark.parametrize("n_heads", [32, 64])
def test_mixed_prefill_replays_in_a_cuda_graph(n_heads, cuda_device):
    # A unified batch of decode rows and prefill chunks: at GQA 4 the single-token rows run on the
    # split-KV decode kernel launched as a programmatic dependent of the tensor-core kernel, which a
    # capture turns into a programmatic edge; at GQA 8 they stay in the tensor-core kernel.
    q_lens = np.array([1, 64, 1, 1, 200, 1, 33])
    kv = np.array([700, 64, 3000, 17, 1500, 9000, 100])
    b = workloads.custom(kv, q_lens, n_heads, 8, 128, torch.bfloat16, seed=n_heads).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    q = b.q.clone()

    def attend():
        return ops.paged_attention_gemm(q, b.k_pool, b.v_pool, md["cu_seqlens"], b.max_q_len, 32, None, None,
                                        md["block_tables"], md["kv_lens"], md["positions"])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            attend()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = attend()
    for it in range(3):
        q.copy_((torch.randn_like(q, dtype=torch.float32) * (1 + it)).to(q.dtype))
        g.replay()
        torch.cuda.synchronize()
        got = out.clone()
        ref = attend()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), it
    del g
