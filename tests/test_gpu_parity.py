"""GPU parity of the C ABI against the oracle and the reference's golden outputs.

Tolerances (vs an fp32-or-wider reference): KV writes and slot indexing
bit-exact; fp32 attention max-abs <= 1e-4; bf16 / f16 attention max-abs <= 2e-2
and mean-abs <= 2e-3.
"""

import numpy as np
import pytest
import torch

import cabi
import oracle
import torch_ref
from conftest import GOLDEN_CASES, golden_after, load_golden
from femtovllm_b200 import workloads

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-4), torch.bfloat16: (2e-2, 2e-3), torch.float16: (2e-2, 2e-3)}


def assert_close(out: torch.Tensor, ref: np.ndarray, dtype, what=""):
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref)
    max_tol, mean_tol = TOL[dtype]
    assert err.max() <= max_tol, f"{what}: max abs {err.max():.3g} > {max_tol}"
    assert err.mean() <= mean_tol, f"{what}: mean abs {err.mean():.3g} > {mean_tol}"


def _dev(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


# ---------------------------------------------------------------------------
# golden fixtures (made by running the reference itself)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_golden_store_then_attend(name, dtype, cuda_device):
    d = load_golden(name)
    dev = cuda_device
    kp, vp = _dev(d["k_pool"], dev, dtype), _dev(d["v_pool"], dev, dtype)
    slots = _dev(oracle.build_slot_mapping(d["positions"], d["seq_of_token"], d["block_tables"]), dev)
    cabi.store_kvcache(_dev(d["k_new"], dev, dtype), _dev(d["v_new"], dev, dtype), kp, vp, slots)
    torch.cuda.synchronize()
    # bit-exact against the rows the reference's write loop produced
    assert torch.equal(kp.cpu(), torch.from_numpy(golden_after(d, "k")).to(dtype))
    assert torch.equal(vp.cpu(), torch.from_numpy(golden_after(d, "v")).to(dtype))
    q = _dev(d["q"], dev, dtype)
    tables = _dev(d["block_tables"], dev)
    kv_lens = _dev(d["kv_lens"], dev)
    if d["is_decode"]:
        out = cabi.decode(q, kp, vp, tables, kv_lens, int(d["kv_lens"].max()))
        assert_close(out, d["out_ref"], dtype, f"{name} decode")
    out = cabi.prefill(q, kp, vp, _dev(d["cu_seqlens"], dev), int(d["q_lens"].max()), tables, kv_lens,
                       _dev(d["positions"], dev))
    assert_close(out, d["out_ref"], dtype, f"{name} prefill")
    assert cabi.read_device_error() == (0, 0)


# ---------------------------------------------------------------------------
# seeded sweeps against the oracle
# ---------------------------------------------------------------------------

DECODE_LENS = [1, 2, 15, 16, 17, 31, 32, 33, 64, 100, 257, 1000, 2049, 5000]


# Group sizes of the Qwen3 family (2, 4, 5 for 14B, 8, 16 for 235B) plus odd ones.
GQA_SIZES = [1, 2, 3, 4, 5, 6, 8, 16]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("n_rep", GQA_SIZES)
def test_decode_sweep(dtype, head_dim, n_rep, cuda_device):
    hkv = 2
    rng = np.random.default_rng(head_dim * 10 + n_rep)
    lens = rng.permutation(DECODE_LENS)
    b = workloads.custom(lens, np.ones(len(lens)), hkv * n_rep, hkv, head_dim, dtype, seed=n_rep).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    ref = oracle.decode_attention(b.q.float().cpu().numpy(), b.k_pool.float().cpu().numpy(),
                                  b.v_pool.float().cpu().numpy(), b.block_tables, b.kv_lens)
    assert_close(out, ref, dtype, f"decode {dtype} D{head_dim} rep{n_rep}")


def test_decode_without_splits_writes_directly(cuda_device):
    # Many (seq, kv head) units and short contexts: the plan uses one split per sequence.
    lens = np.random.default_rng(0).integers(1, 900, size=300)
    b = workloads.custom(lens, np.ones(300), 16, 8, 128, torch.bfloat16, seed=5).materialize(cuda_device)
    assert cabi.lib().fvb_paged_attention_decode_workspace_size(300, 16, 8, 128, b.max_kv_len) == 0
    md = b.device_metadata(cuda_device)
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    sub = [0, 1, 2, int(np.argmax(lens)), int(np.argmin(lens))]
    ref = oracle.decode_attention(b.q[:, sub].float().cpu().numpy(), b.k_pool.float().cpu().numpy(),
                                  b.v_pool.float().cpu().numpy(), b.block_tables[sub], b.kv_lens[sub])
    assert_close(out[:, sub], ref, torch.bfloat16, "no-split decode")


PREFILL_CASES = [
    # (q_lens, prefixes)
    ([1, 1, 1], [0, 15, 300]),
    ([5, 16, 17, 31], [0, 0, 3, 16]),
    ([128, 64, 200], [0, 77, 1000]),
    ([300, 1, 129], [5000, 40, 0]),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("n_rep", GQA_SIZES)
@pytest.mark.parametrize("case", range(len(PREFILL_CASES)))
def test_prefill_sweep(dtype, head_dim, n_rep, case, cuda_device):
    q_lens, pre = map(np.asarray, PREFILL_CASES[case])
    hkv = 2
    b = workloads.custom(q_lens + pre, q_lens, hkv * n_rep, hkv, head_dim, dtype, seed=case).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], b.max_q_len, md["block_tables"], md["kv_lens"],
                       md["positions"])
    ref = oracle.prefill_attention(b.q.float().cpu().numpy(), b.k_pool.float().cpu().numpy(),
                                   b.v_pool.float().cpu().numpy(), b.cu_seqlens, b.block_tables, b.kv_lens,
                                   b.positions, acc_dtype=np.float32)
    assert_close(out, ref, dtype, f"prefill case{case} {dtype} D{head_dim} rep{n_rep}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("n_rep", [1, 2, 4, 8])
def test_prefill_single_token_rows_at_earlier_positions(dtype, head_dim, n_rep, cuda_device):
    # One-token sequences of a mixed batch whose query sits before the last cached key
    # (a recomputed token) see keys 0 .. position only, whichever kernel serves them
    # (groups of 1-4 send them to the split-KV decode kernel, 8 keeps them in tiles).
    q_lens = np.array([1, 40, 1, 1, 1, 130, 1])
    kv = np.array([300, 100, 50, 5000, 17, 130, 70000])
    hkv = 2
    b = workloads.custom(kv, q_lens, hkv * n_rep, hkv, head_dim, dtype, seed=n_rep).materialize(cuda_device)
    pos = b.positions.copy()
    cu = b.cu_seqlens
    for s, p in [(0, 123), (2, 0), (3, 2047), (4, 16), (6, 65535)]:
        assert q_lens[s] == 1
        pos[cu[s]] = p
    md = b.device_metadata(cuda_device)
    cabi.read_device_error()
    out = cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], b.max_q_len, md["block_tables"], md["kv_lens"],
                       torch.from_numpy(pos).to(cuda_device))
    ref = oracle.prefill_attention(b.q.float().cpu().numpy(), b.k_pool.float().cpu().numpy(),
                                   b.v_pool.float().cpu().numpy(), cu, b.block_tables, b.kv_lens, pos,
                                   acc_dtype=np.float32)
    assert_close(out, ref, dtype, f"single-token rows {dtype} D{head_dim} rep{n_rep}")
    assert cabi.read_device_error() == (0, 0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_store_kvcache_sweep_bit_exact(dtype, cuda_device):
    b = workloads.custom([40, 1, 17, 300], [40, 1, 9, 100], 8, 4, 128, dtype, seed=3).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    # strided views, as the projection outputs are: (T, Hkv * D) viewed as (T, Hkv, D)
    packed = torch.cat([b.k_new.reshape(b.num_tokens, -1), b.v_new.reshape(b.num_tokens, -1)], dim=1)
    k = packed[:, : 4 * 128].view(b.num_tokens, 4, 128)
    v = packed[:, 4 * 128 :].view(b.num_tokens, 4, 128)
    slots = md["slot_mapping"].clone()
    slots[3] = -1  # a padding token is skipped
    cabi.store_kvcache(k, v, kp, vp, slots)
    kref = b.k_pool.cpu().clone()
    vref = b.v_pool.cpu().clone()
    s = slots.cpu().numpy()
    live = s >= 0
    kref[s[live] // 16, :, s[live] % 16] = b.k_new.cpu()[live]
    vref[s[live] // 16, :, s[live] % 16] = b.v_new.cpu()[live]
    assert torch.equal(kp.cpu(), kref) and torch.equal(vp.cpu(), vref)


@pytest.mark.parametrize("T", [77, 5000])
@pytest.mark.parametrize("layout", ["contiguous", "head_major_view", "unaligned"])
def test_store_kvcache_layouts_bit_exact(layout, T, cuda_device):
    """The write path for each input layout and size: 5000 tokens of 16-byte-aligned rows take the bulk
    copies (one per token and tensor when a token's heads are adjacent, one per row otherwise); 77 tokens
    and rows off a 16-byte boundary take the vector kernel.  Every case writes the pools the reference
    loop writes, bit for bit."""
    hkv, d = 4, 128
    g = torch.Generator().manual_seed(31)
    kh = torch.randn(hkv, T, d, generator=g).to(torch.bfloat16)
    vh = torch.randn(hkv, T, d, generator=g).to(torch.bfloat16)
    if layout == "contiguous":
        k, v = kh.transpose(0, 1).contiguous().to(cuda_device), vh.transpose(0, 1).contiguous().to(cuda_device)
    elif layout == "head_major_view":  # (T, Hkv, D) view of head-major storage: head stride T * D
        k, v = kh.to(cuda_device).transpose(0, 1), vh.to(cuda_device).transpose(0, 1)
    else:  # one element past a 16-byte boundary
        flat = torch.empty(2 * T * hkv * d + 2, dtype=torch.bfloat16, device=cuda_device)
        k = flat[1 : 1 + T * hkv * d].view(T, hkv, d)
        v = flat[1 + T * hkv * d : 1 + 2 * T * hkv * d].view(T, hkv, d)
        k.copy_(kh.transpose(0, 1))
        v.copy_(vh.transpose(0, 1))
    nb = (2 * T + 15) // 16
    slots = torch.randperm(nb * 16, generator=g)[:T].to(torch.int64)
    slots[3] = -1
    slots[T - 1] = -1  # a padding token in the last chunk too
    bad = T - 7
    slots[bad] = nb * 16  # one past the pool: reported, skipped, the rest still written
    kref = torch.zeros(nb, hkv, 16, d, dtype=torch.bfloat16)
    vref = torch.zeros_like(kref)
    kp, vp = kref.to(cuda_device), vref.to(cuda_device)
    cabi.read_device_error()
    cabi.store_kvcache(k, v, kp, vp, slots.to(cuda_device))
    s = slots.numpy()
    live = (s >= 0) & (s < nb * 16)
    kref[s[live] // 16, :, s[live] % 16] = kh.transpose(0, 1)[live]
    vref[s[live] // 16, :, s[live] % 16] = vh.transpose(0, 1)[live]
    assert torch.equal(kp.cpu(), kref) and torch.equal(vp.cpu(), vref)
    assert cabi.read_device_error() == (8, bad)  # FVB_ERR_BAD_SLOT at that token


@pytest.mark.parametrize("page", [8, 12, 32])
def test_store_kvcache_other_page_sizes_bit_exact(page, cuda_device):
    """The write accepts any page size: powers of two split the slot by a shift, others by a division."""
    T, hkv, d = 300, 4, 128
    g = torch.Generator().manual_seed(page)
    k = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    v = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    nb = (2 * T + page - 1) // page
    slots = torch.randperm(nb * page, generator=g)[:T].to(torch.int64)
    slots[5] = -1
    kref = torch.zeros(nb, hkv, page, d, dtype=torch.bfloat16)
    vref = torch.zeros_like(kref)
    kp, vp = kref.to(cuda_device), vref.to(cuda_device)
    cabi.store_kvcache(k.to(cuda_device), v.to(cuda_device), kp, vp, slots.to(cuda_device))
    s = slots.numpy()
    live = s >= 0
    kref[s[live] // page, :, s[live] % page] = k[live]
    vref[s[live] // page, :, s[live] % page] = v[live]
    assert torch.equal(kp.cpu(), kref) and torch.equal(vp.cpu(), vref)


# ---------------------------------------------------------------------------
# full-size configurations (sampled oracle checks + size-independent properties)
# ---------------------------------------------------------------------------


def _sample(b, n=6, seed=0):
    rng = np.random.default_rng(seed)
    pick = {int(np.argmin(b.kv_lens)), int(np.argmax(b.kv_lens))}
    while len(pick) < min(n, b.num_seqs):
        pick.add(int(rng.integers(b.num_seqs)))
    return sorted(pick)


def _check_every_row(out, b, md, what, seqs, decode):
    """Every output row against the fp32 device restatement (tests/torch_ref.py), which is
    itself pinned to the numpy oracle on `seqs` first."""
    ref = torch_ref.paged_attention_fp32(b.q, b.k_pool, b.v_pool, None if decode else md["cu_seqlens"],
                                         md["block_tables"], md["kv_lens"], None if decode else md["positions"])
    sub = workloads.subset_for_oracle(b, seqs)
    if decode:
        pin = oracle.decode_attention(sub["q"], sub["k_pool"], sub["v_pool"], sub["block_tables"], sub["kv_lens"])
    else:
        pin = oracle.prefill_attention(sub["q"], sub["k_pool"], sub["v_pool"], sub["cu_seqlens"],
                                       sub["block_tables"], sub["kv_lens"], sub["positions"])
    tok = torch.from_numpy(sub["tokens"]).to(out.device)
    pin_err = np.abs(ref[:, tok].cpu().numpy() - pin).max()
    assert pin_err <= 1e-5, f"{what}: device restatement differs from the oracle by {pin_err:.3g}"
    assert_close(out[:, tok], pin, b.dtype, f"{what} (oracle sample)")
    got = out.float()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs()
    max_tol, mean_tol = TOL[b.dtype]
    worst = int(err.amax(dim=(0, 2)).argmax())
    assert err.max().item() <= max_tol, f"{what}: max abs {err.max().item():.3g} (token {worst}) > {max_tol}"
    assert err.mean().item() <= mean_tol, f"{what}: mean abs {err.mean().item():.3g} > {mean_tol}"
    return ref


def test_config2_decode_full_size(cuda_device):
    b = workloads.config2().materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    cabi.store_kvcache(b.k_new, b.v_new, b.k_pool, b.v_pool, md["slot_mapping"])
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    out2 = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    assert torch.equal(out, out2), "decode is not deterministic"
    _check_every_row(out, b, md, "config2", _sample(b), decode=True)
    # the new token is visible: its slot now holds k_new
    seqs = _sample(b)
    s = b.slot_mapping[seqs[0]]
    assert torch.equal(b.k_pool[s // 16, :, s % 16], b.k_new[seqs[0]])
    assert cabi.read_device_error() == (0, 0)


@pytest.mark.parametrize("world,rank", [(1, 0), (4, 3), (8, 0), (8, 7)])
def test_config5_long_decode_shard_every_row(world, rank, cuda_device):
    """The rank's LPT shard of config 5 exactly as `bench.py` runs it (own pool, own tables)."""
    b = workloads.config5(rank=rank, world=world).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    _check_every_row(out, b, md, f"config5 rank {rank} of {world}", [int(np.argmax(b.kv_lens))], decode=True)
    assert cabi.read_device_error() == (0, 0)


@pytest.mark.parametrize("n_heads,n_seqs", [(64, 16), (128, 4)])
def test_tensor_core_decode_split_every_row(n_heads, n_seqs, cuda_device):
    """GQA 8 / 16 decode on the tcgen05 route with split-KV (few long sequences)."""
    lens = np.random.default_rng(n_heads).integers(32768, 131073, size=n_seqs)
    b = workloads.custom(lens, np.ones(n_seqs), n_heads, 8, 128, torch.bfloat16, seed=n_heads,
                         pool_factor=1.05).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)
    _check_every_row(out, b, md, f"tc decode GQA {n_heads // 8}", [int(np.argmin(b.kv_lens))], decode=True)
    assert cabi.read_device_error() == (0, 0)


def test_config3_prefill_full_size(cuda_device):
    b = workloads.config3().materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], b.max_q_len, md["block_tables"], md["kv_lens"],
                       md["positions"])
    _check_every_row(out, b, md, "config3", [int(np.argmin(b.kv_lens)), 7], decode=False)
    assert cabi.read_device_error() == (0, 0)


def test_config4_mixed_full_size(cuda_device):
    b = workloads.config4().materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    out = cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], b.max_q_len, md["block_tables"], md["kv_lens"],
                       md["positions"])
    dec = [int(i) for i in np.nonzero(b.q_lens == 1)[0][:3]]
    pre = [int(np.nonzero(b.q_lens > 1)[0][0])]
    _check_every_row(out, b, md, "config4", dec + pre, decode=False)
    # decode rows through the decode kernel agree with the unified launch
    dmask = b.q_lens == 1
    tok = torch.from_numpy(b.cu_seqlens[:-1][dmask].astype(np.int64)).to(cuda_device)
    tabs = md["block_tables"][torch.from_numpy(np.nonzero(dmask)[0]).to(cuda_device)].contiguous()
    lens = md["kv_lens"][torch.from_numpy(np.nonzero(dmask)[0]).to(cuda_device)].contiguous()
    dout = cabi.decode(b.q[:, tok].contiguous(), b.k_pool, b.v_pool, tabs, lens, int(b.kv_lens[dmask].max()))
    diff = (dout.float() - out[:, tok].float()).abs()
    assert diff.max().item() <= 2e-2 and diff.mean().item() <= 2e-3, (diff.max().item(), diff.mean().item())
    assert cabi.read_device_error() == (0, 0)


# ---------------------------------------------------------------------------
# bad metadata is reported, never read out of bounds
# ---------------------------------------------------------------------------


def test_bad_page_and_slot_are_reported(cuda_device):
    b = workloads.custom([40, 20], [1, 1], 4, 2, 64, torch.bfloat16, seed=1).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    cabi.read_device_error()
    tables = md["block_tables"].clone()
    tables[0, 1] = -1  # a hole inside kv_len
    cabi.decode(b.q, b.k_pool, b.v_pool, tables, md["kv_lens"], b.max_kv_len)
    assert cabi.read_device_error()[0] == 7  # FVB_ERR_BAD_PAGE
    tables[0, 1] = b.num_blocks + 5  # past the pool
    cabi.prefill(b.q, b.k_pool, b.v_pool, md["cu_seqlens"], 1, tables, md["kv_lens"], md["positions"])
    assert cabi.read_device_error()[0] == 7
    slots = md["slot_mapping"].clone()
    slots[1] = b.num_blocks * 16  # one past the last slot
    kp = b.k_pool.clone()
    cabi.store_kvcache(b.k_new, b.v_new, kp, b.v_pool.clone(), slots)
    assert cabi.read_device_error() == (8, 1)  # FVB_ERR_BAD_SLOT at token 1
    s0 = int(slots[0])
    assert torch.equal(kp[s0 // 16, :, s0 % 16], b.k_new[0])  # the good token is still written


def test_kv_len_beyond_max_kv_len_is_clamped_and_reported(cuda_device):
    b = workloads.custom([40, 20], [1, 1], 4, 2, 64, torch.bfloat16, seed=2).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    cabi.read_device_error()
    cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], 32)  # max_kv_len < kv_lens[0]
    assert cabi.read_device_error()[0] == 1


@pytest.mark.parametrize("lens,max_kv", [([3000, 200, 5000], 4000), ([300, 900, 40], 512)])
def test_tensor_core_decode_clamps_kv_len_to_max_kv_len(lens, max_kv, cuda_device):
    """GQA 8 (tcgen05 route, split-KV for these few sequences): a kv_len above max_kv_len is
    reported and attends over the first max_kv_len keys, like the SIMT route."""
    b = workloads.custom(lens, np.ones(len(lens)), 64, 8, 128, torch.bfloat16, seed=4).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    cabi.read_device_error()
    out = cabi.decode(b.q, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], max_kv)
    code, info = cabi.read_device_error()
    assert code == 1 and b.kv_lens[info] > max_kv
    clamped = torch.clamp(md["kv_lens"], max=max_kv)
    ref = torch_ref.paged_attention_fp32(b.q, b.k_pool, b.v_pool, None, md["block_tables"], clamped)
    assert torch.isfinite(out.float()).all()
    err = (out.float() - ref).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (err.max().item(), err.mean().item())


# ---------------------------------------------------------------------------
# the PyTorch-registered boundary (femtovllm_b200.ops / torch.ops) = the C ABI
# ---------------------------------------------------------------------------


def test_torch_ops_match_c_abi(cuda_device):
    from femtovllm_b200 import ops

    b = workloads.custom([70, 33, 200], [1, 1, 1], 8, 2, 128, torch.bfloat16, seed=9).materialize(cuda_device)
    md = b.device_metadata(cuda_device)
    kp1, vp1 = b.k_pool.clone(), b.v_pool.clone()
    ops.store_kvcache(b.k_new, b.v_new, kp1, vp1, md["slot_mapping"])
    kp2, vp2 = b.k_pool.clone(), b.v_pool.clone()
    torch.ops.femtovllm_b200.store_kvcache(b.k_new, b.v_new, kp2, vp2, md["slot_mapping"])
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    a = ops.paged_attention_gemv(b.q, kp1, vp1, md["block_tables"], md["kv_lens"], b.max_kv_len)
    c = cabi.decode(b.q, kp1, vp1, md["block_tables"], md["kv_lens"], b.max_kv_len)
    assert torch.equal(a, c)
    # transposed (non-contiguous) q is made contiguous, as the reference wrapper does
    qt = b.q.transpose(0, 1).contiguous().transpose(0, 1)
    assert torch.equal(ops.paged_attention_gemv(qt, kp1, vp1, md["block_tables"], md["kv_lens"], b.max_kv_len), a)
    g = ops.paged_attention_gemm(b.q, kp1, vp1, md["cu_seqlens"], 1, 32, None, None, md["block_tables"],
                                 md["kv_lens"], md["positions"])
    assert (g.float() - a.float()).abs().max().item() <= 2e-2
    with pytest.raises(RuntimeError):
        ops.paged_attention_gemv(b.q.to(torch.float64), kp1, vp1, md["block_tables"], md["kv_lens"], b.max_kv_len)


# ---------------------------------------------------------------------------
# on-device slot mapping (the reference write loops' index arithmetic)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("make", [workloads.config3, workloads.config4, workloads.config1])
def test_build_slot_mapping_matches_oracle(make, cuda_device):
    from femtovllm_b200 import ops

    b = make()
    md = b.device_metadata(cuda_device)
    slots = ops.build_slot_mapping(md["positions"], md["block_tables"], md["cu_seqlens"])
    ref = oracle.build_slot_mapping(b.positions, b.seq_of_token, b.block_tables)
    assert np.array_equal(slots.cpu().numpy(), ref)
    if b.is_decode:  # one token per sequence: cu_seqlens may be omitted
        assert torch.equal(ops.build_slot_mapping(md["positions"], md["block_tables"]), slots)


def test_build_slot_mapping_edges(cuda_device):
    from femtovllm_b200 import ops

    tables = torch.tensor([[3, -1, 7], [5, 2, -1]], dtype=torch.int32, device=cuda_device)
    pos = torch.tensor([0, 15, 16, 33, 0, 17, 40], dtype=torch.int32, device=cuda_device)
    cu = torch.tensor([0, 4, 7], dtype=torch.int32, device=cuda_device)
    cabi.read_device_error()
    slots = ops.build_slot_mapping(pos, tables, cu).cpu().tolist()
    # seq 0: 3*16+0, 3*16+15, page 1 is -1 -> -1, 7*16+1 ; seq 1: 5*16+0, 2*16+1, page 2 is -1 -> -1
    assert slots == [48, 63, -1, 113, 80, 33, -1]
    assert cabi.read_device_error() == (0, 0)
    ops.build_slot_mapping(torch.tensor([48], dtype=torch.int32, device=cuda_device), tables[:1])  # page 3 > row
    assert cabi.read_device_error()[0] == 1
