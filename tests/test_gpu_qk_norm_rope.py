"""GPU parity of the fused q/k RMSNorm + rotary embedding + KV write (fvb_qk_norm_rope_store).

Checked through the C ABI against the CPU oracle (pinned to the reference's own
q_norm / k_norm / QwenRotaryEmbedding / write loop by tests/golden/norm_rope_*.npz),
and at full size against a plain PyTorch fp32 restatement on the GPU.
Tolerances: |got - ref| <= tol * max(1, |ref|) with tol = 1e-4 (fp32) or 2e-2
(bf16 / f16), and mean-abs <= 1e-5 / 2e-3.  The scale matters here: unlike
attention outputs, normalised-and-weighted rows reach |y| ~ 8, where one bf16
half-ulp alone is 0.03.  V rows and every pool row the op must not touch are
compared bit for bit.
"""

import numpy as np
import pytest
import torch

import cabi
import oracle
from conftest import NORM_ROPE_CASES, load_norm_rope
from femtovllm_b200 import ops, workloads

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-5), torch.bfloat16: (2e-2, 2e-3), torch.float16: (2e-2, 2e-3)}


def _check_close(got, ref, dtype):
    mx, mean = TOL[dtype]
    ref = np.asarray(ref, np.float64)
    err = np.abs(np.asarray(got, np.float64) - ref)
    worst = (err / np.maximum(1.0, np.abs(ref))).max()
    assert worst <= mx and err.mean() <= mean, (worst, err.mean())


def _packed_views(q_thd, k, v):
    """q (T, Hq, D), k / v (T, Hkv, D) as strided views of one (T, (Hq + 2 Hkv) D) buffer."""
    T, hq, d = q_thd.shape
    hkv = k.shape[1]
    x = torch.cat([q_thd.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], dim=1)
    return (x[:, : hq * d].view(T, hq, d), x[:, hq * d : (hq + hkv) * d].view(T, hkv, d),
            x[:, (hq + hkv) * d :].view(T, hkv, d))


def _oracle(q, k, v, q_w, k_w, eps, cos, sin, positions, k_pool, v_pool, slots):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    kp, vp = f(k_pool), f(v_pool)
    q_out = oracle.qk_norm_rope_store(f(q), f(k), f(v), f(q_w), f(k_w), eps, f(cos), f(sin),
                                      positions.cpu().numpy(), kp, vp, slots.cpu().numpy())
    return q_out, kp, vp


def _compare_pools(kp_gpu, vp_gpu, kp_ref, vp_ref, kp_before, slots, dtype):
    s = slots.cpu().numpy()
    live = s[s >= 0]
    written = np.zeros(kp_ref.shape[:3], bool)
    written[live // 16, :, live % 16] = True
    kg, vg = kp_gpu.float().cpu().numpy(), vp_gpu.float().cpu().numpy()
    assert np.array_equal(vg.view(np.uint32), vp_ref.view(np.uint32))  # V: bit-exact copy, rest untouched
    kb = kp_before.float().cpu().numpy()
    assert np.array_equal(kg[~written].view(np.uint32), kb[~written].view(np.uint32))
    _check_close(kg[written], kp_ref[written], dtype)


def _rope(rows, d, dtype, device):
    cos, sin = oracle.rope_tables(rows, d)
    return torch.from_numpy(cos).to(device, dtype), torch.from_numpy(sin).to(device, dtype)


def _weights(d, dtype, device, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple((1.0 + 0.25 * torch.randn(d, generator=g)).to(dtype).to(device) for _ in range(2))


@pytest.mark.parametrize("name", NORM_ROPE_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_golden_norm_rope_store(name, dtype, cuda_device):
    d = load_norm_rope(name)
    dev = cuda_device
    T, hq, hkv, D = len(d["positions"]), d["n_heads"], d["n_kv_heads"], d["head_dim"]
    cos, sin = oracle.rope_tables(d["rope_rows"], D)
    cos[d["positions"]] = d["cos_rows"]
    sin[d["positions"]] = d["sin_rows"]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)  # noqa: E731
    q, k, v = _packed_views(t(d["q"]), t(d["k_new"]), t(d["v_new"]))
    q_w, k_w, cos_t, sin_t = t(d["q_norm_weight"]), t(d["k_norm_weight"]), t(cos), t(sin)
    kp, vp = t(d["k_pool"]), t(d["v_pool"])
    kp_before = kp.clone()
    pos = torch.from_numpy(d["positions"]).to(dev)
    slots = torch.from_numpy(oracle.build_slot_mapping(d["positions"], d["seq_of_token"], d["block_tables"])).to(dev)
    q_ref, kp_ref, vp_ref = _oracle(q, k, v, q_w, k_w, d["eps"], cos_t, sin_t, pos, kp, vp, slots)
    cabi.read_device_error()
    q_out = cabi.qk_norm_rope_store(q, k, v, q_w, k_w, d["eps"], cos_t, sin_t, pos, kp, vp, slots)
    assert cabi.read_device_error() == (0, 0)
    if dtype == torch.float32:  # straight against the reference's own fp32 outputs
        _check_close(q_out.cpu().numpy(), d["q_ref"], dtype)
        idx = d["k_written_idx"]
        _check_close(kp.cpu().numpy()[idx[:, 0], idx[:, 1], idx[:, 2]], d["k_written_rows"], dtype)
    _check_close(q_out.float().cpu().numpy(), q_ref, dtype)
    _compare_pools(kp, vp, kp_ref, vp_ref, kp_before, slots, dtype)


# (128, 8, 128): a block pass of 144 rows; in fp32 its three staged passes (216 KB) exceed the
# warp-specialised kernel's shared-memory limit, so that case runs the other kernel.
SHAPES = [(16, 8, 128), (32, 8, 128), (8, 8, 64), (8, 1, 64), (4, 2, 128), (128, 8, 128)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"hq{s[0]}_hkv{s[1]}_d{s[2]}")
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_sweep_against_oracle(shape, dtype, cuda_device):
    hq, hkv, D = shape
    b = workloads.custom([300, 17, 1, 2048, 64], [300, 1, 1, 37, 64], hq, hkv, D, dtype, seed=hq + D).materialize(
        cuda_device)
    md = b.device_metadata(cuda_device)
    q, k, v = _packed_views(b.q.transpose(0, 1), b.k_new, b.v_new)
    q_w, k_w = _weights(D, dtype, cuda_device, seed=D)
    cos, sin = _rope(4096, D, dtype, cuda_device)
    slots = md["slot_mapping"].clone()
    slots[5] = -1  # padding token: q still produced, k / v not written
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    q_ref, kp_ref, vp_ref = _oracle(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp, vp, slots)
    cabi.read_device_error()
    q_out = cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp, vp, slots)
    assert cabi.read_device_error() == (0, 0)
    _check_close(q_out.float().cpu().numpy(), q_ref, dtype)
    _compare_pools(kp, vp, kp_ref, vp_ref, b.k_pool, slots, dtype)


def test_torch_op_matches_c_abi(cuda_device):
    b = workloads.custom([100, 33], [100, 1], 16, 8, 128, torch.bfloat16, seed=9).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    q, k, v = _packed_views(b.q.transpose(0, 1), b.k_new, b.v_new)
    q_w, k_w = _weights(128, torch.bfloat16, cuda_device, seed=1)
    cos, sin = _rope(1024, 128, torch.bfloat16, cuda_device)
    kp1, vp1 = b.k_pool.clone(), b.v_pool.clone()
    kp2, vp2 = b.k_pool.clone(), b.v_pool.clone()
    a = cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp1, vp1, md["slot_mapping"])
    o = ops.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp2, vp2, md["slot_mapping"])
    t = torch.ops.femtovllm_b200.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp2, vp2,
                                                    md["slot_mapping"])
    assert o.shape == (16, b.num_tokens, 128)
    assert torch.equal(a, o) and torch.equal(a, t)
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)


def test_feeds_prefill_attention(cuda_device):
    """The head-major q it returns and the pools it writes are what the prefill kernel reads:
    fused stage + tcgen05 prefill against oracle stage + oracle prefill."""
    dtype = torch.bfloat16
    b = workloads.custom([200, 77, 1000], [200, 13, 130], 16, 8, 128, dtype, seed=5).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    q, k, v = _packed_views(b.q.transpose(0, 1), b.k_new, b.v_new)
    q_w, k_w = _weights(128, dtype, cuda_device, seed=2)
    cos, sin = _rope(2048, 128, dtype, cuda_device)
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    q_ref, kp_ref, vp_ref = _oracle(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp, vp, md["slot_mapping"])
    q_out = ops.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp, vp, md["slot_mapping"])
    out = cabi.prefill(q_out, kp, vp, md["cu_seqlens"], int(b.q_lens.max()), md["block_tables"], md["kv_lens"],
                       md["positions"])
    # The oracle attends over bf16-rounded q / k (as the kernel does) in fp64.
    q_b = torch.from_numpy(q_ref).to(dtype).float().numpy()
    kp_b = torch.from_numpy(kp_ref).to(dtype).float().numpy()
    ref = oracle.prefill_attention(q_b, kp_b, vp_ref, b.cu_seqlens, b.block_tables, b.kv_lens, b.positions)
    _check_close(out.float().cpu().numpy(), ref, dtype)


def test_full_size_config3_tokens_against_torch_fp32(cuda_device):
    """Config-3 token count (Hq 16, Hkv 8, D 128, ~70k new tokens) against a PyTorch fp32
    restatement on the GPU; V rows must land bit-exact in their slots."""
    dtype = torch.bfloat16
    b = workloads.config3().materialize(cuda_device, k_pool_fill=False)
    b.k_pool.zero_()
    b.v_pool.zero_()
    md = b.device_metadata(cuda_device)
    T = b.num_tokens
    q, k, v = _packed_views(b.q.transpose(0, 1), b.k_new, b.v_new)
    del b.q
    q_w, k_w = _weights(128, dtype, cuda_device, seed=3)
    rows = int(b.kv_lens.max())
    cos, sin = _rope(rows, 128, dtype, cuda_device)
    q_out = ops.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], b.k_pool, b.v_pool,
                                   md["slot_mapping"])
    torch.cuda.synchronize()
    pos = md["positions"].long()

    def ref(x, w):
        x = x.float()
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        c, s = cos.float()[pos][:, None], sin.float()[pos][:, None]
        return y * c + torch.cat([-y[..., 64:], y[..., :64]], -1) * s

    for h0 in range(0, 16, 4):  # in head chunks to bound the fp32 temporaries
        r = ref(q[:, h0 : h0 + 4], q_w).transpose(0, 1)
        err = (q_out[h0 : h0 + 4].float() - r).abs()
        assert (err / r.abs().clamp(min=1.0)).max().item() <= 2e-2 and err.mean().item() <= 2e-3
    slots = md["slot_mapping"]
    blk, off = slots // 16, slots % 16
    kr = ref(k, k_w)
    kg = b.k_pool[blk, :, off].float()
    err = (kg - kr).abs()
    assert (err / kr.abs().clamp(min=1.0)).max().item() <= 2e-2 and err.mean().item() <= 2e-3
    assert torch.equal(b.v_pool[blk, :, off], v)
    assert T == slots.numel()


def test_bad_slot_and_position_are_reported(cuda_device):
    dtype = torch.bfloat16
    b = workloads.custom([40, 20], [40, 20], 8, 2, 128, dtype, seed=4).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    q, k, v = _packed_views(b.q.transpose(0, 1), b.k_new, b.v_new)
    q_w, k_w = _weights(128, dtype, cuda_device, seed=4)
    cos, sin = _rope(64, 128, dtype, cuda_device)
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    slots = md["slot_mapping"].clone()
    slots[7] = b.num_blocks * 16  # one past the pool
    cabi.read_device_error()
    cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, md["positions"], kp, vp, slots)
    code, info = cabi.read_device_error()
    assert (code, info) == (8, 7)  # FVB_ERR_BAD_SLOT at token 7
    pos = md["positions"].clone()
    pos[3] = 64  # == rope_rows: outside the tables
    cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, pos, kp, vp, md["slot_mapping"])
    code, info = cabi.read_device_error()
    assert (code, info) == (1, 3)  # FVB_ERR_INVALID_ARGUMENT at token 3


def test_host_side_rejections(cuda_device):
    dtype = torch.bfloat16
    T, hq, hkv = 8, 4, 2
    x = torch.zeros(T, (hq + 2 * hkv) * 96 + 8, dtype=dtype, device=cuda_device)
    pos = torch.zeros(T, dtype=torch.int32, device=cuda_device)
    slots = torch.full((T,), -1, dtype=torch.int64, device=cuda_device)
    cos = torch.zeros(16, 128, dtype=dtype, device=cuda_device)
    w = torch.ones(128, dtype=dtype, device=cuda_device)
    pool = torch.zeros(2, hkv, 16, 128, dtype=dtype, device=cuda_device)
    q_out = torch.empty(hq, T, 128, dtype=dtype, device=cuda_device)
    # head_dim 96 is not a supported size
    q96 = x[:, : hq * 96].view(T, hq, 96)
    k96 = x[:, hq * 96 : (hq + hkv) * 96].view(T, hkv, 96)
    st = cabi.qk_norm_rope_store_status(q96, k96, k96, w, w, 1e-6, cos, cos, pos, pool, pool, slots, q_out)
    assert st == 2  # FVB_ERR_UNSUPPORTED
    # rows 4 elements (8 bytes) off a 16-byte boundary
    y = torch.zeros(T, (hq + 2 * hkv) * 128 + 4, dtype=dtype, device=cuda_device)
    qm = y[:, 4 : 4 + hq * 128].view(T, hq, 128)
    km = y[:, 4 + hq * 128 : 4 + (hq + hkv) * 128].view(T, hkv, 128)
    st = cabi.qk_norm_rope_store_status(qm, km, km, w, w, 1e-6, cos, cos, pos, pool, pool, slots, q_out)
    assert st == 3  # FVB_ERR_MISALIGNED
    with pytest.raises(ValueError):
        ops.qk_norm_rope_store(qm.cpu(), km, km, w, w, 1e-6, cos, cos, pos, pool, pool, slots)


@pytest.mark.parametrize("page", [8, 12, 32])
def test_other_page_sizes_write_the_same_rows(page, cuda_device):
    """Any page size: each slot's K / V row equals the one written with 16-token pages (powers of
    two split the slot by a shift, others by a division), and q_out does not depend on it."""
    T, hq, hkv, d = 200, 8, 4, 128
    g = torch.Generator().manual_seed(100 + page)
    x = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).to(cuda_device)
    q = x[:, : hq * d].view(T, hq, d)
    k = x[:, hq * d : (hq + hkv) * d].view(T, hkv, d)
    v = x[:, (hq + hkv) * d :].view(T, hkv, d)
    q_w = (1 + 0.25 * torch.randn(d, generator=g)).to(torch.bfloat16).to(cuda_device)
    k_w = (1 + 0.25 * torch.randn(d, generator=g)).to(torch.bfloat16).to(cuda_device)
    rows = 512
    inv = 1e-6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d)
    theta = torch.arange(rows, dtype=torch.float32)[:, None] * inv[None]
    theta = torch.cat([theta, theta], -1)
    cos = theta.cos().to(torch.bfloat16).to(cuda_device)
    sin = theta.sin().to(torch.bfloat16).to(cuda_device)
    positions = torch.randint(0, rows, (T,), generator=g, dtype=torch.int32).to(cuda_device)
    cap = 2 * T
    slots = torch.randperm(cap, generator=g)[:T].to(torch.int64)

    def run(p):
        nb = (cap + p - 1) // p
        kp = torch.zeros(nb, hkv, p, d, dtype=torch.bfloat16, device=cuda_device)
        vp = torch.zeros_like(kp)
        q_out = cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, positions, kp, vp, slots.to(cuda_device))
        return q_out.cpu(), kp.cpu()[slots // p, :, slots % p], vp.cpu()[slots // p, :, slots % p]

    for a, b in zip(run(16), run(page)):
        assert torch.equal(a, b)
    assert torch.equal(run(page)[2], v.cpu())



def test_pools_past_2_31_elements_write_the_same_rows(cuda_device):
    """Pools of more than 2^31 elements take the 64-bit-offset kernel: its q_out and the rows it writes near
    the top of such a pool equal what the 32-bit-offset kernel writes into a small pool."""
    T, hq, hkv, d = 96, 8, 8, 128
    g = torch.Generator().manual_seed(77)
    x = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).to(cuda_device)
    q = x[:, : hq * d].view(T, hq, d)
    k = x[:, hq * d : (hq + hkv) * d].view(T, hkv, d)
    v = x[:, (hq + hkv) * d :].view(T, hkv, d)
    q_w, k_w = _weights(d, torch.bfloat16, cuda_device, seed=77)
    cos, sin = _rope(256, d, torch.bfloat16, cuda_device)
    positions = torch.randint(0, 256, (T,), generator=g, dtype=torch.int32).to(cuda_device)
    small_blocks = 16
    rel = torch.randperm(small_blocks * 16, generator=g)[:T].to(torch.int64)
    big_blocks = (1 << 31) // (hkv * 16 * d) + 64  # 2^31 elements per pool and a little more: 4.3 GB each
    base = (big_blocks - small_blocks) * 16  # the same rows, at the top of the big pool

    def run(nb, offset):
        kp = torch.zeros(nb, hkv, 16, d, dtype=torch.bfloat16, device=cuda_device)
        vp = torch.zeros_like(kp)
        slots = (rel + offset).to(cuda_device)
        cabi.read_device_error()
        q_out = cabi.qk_norm_rope_store(q, k, v, q_w, k_w, 1e-6, cos, sin, positions, kp, vp, slots)
        assert cabi.read_device_error() == (0, 0)
        sl = slots.cpu()
        rows = (kp[sl // 16, :, sl % 16].cpu(), vp[sl // 16, :, sl % 16].cpu())
        del kp, vp
        torch.cuda.empty_cache()
        return (q_out.cpu(),) + rows

    small = run(small_blocks, 0)
    big = run(big_blocks, base)
    for a, b in zip(small, big):
        assert torch.equal(a, b)
    assert torch.equal(big[2], v.cpu())
