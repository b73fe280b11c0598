"""fvb_sample_tokens on the GPU against the oracle (itself pinned to the reference's Sampler).

Greedy rows must match exactly.  A sampled row must pick a token whose CDF interval, as the oracle
computes it in fp64 and widened by 3e-6 for the kernel's fp32 / ex2.approx sums, holds the row's
Philox uniform.  The distribution itself is checked against the reference's own draws.
"""

import numpy as np
import pytest
import torch

import cabi
from conftest import chi2_critical, load_sampler_cases
from oracle import sampler as S

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _dev():
    return torch.device("cuda", 0)


def _rng(seed, offset=0):
    return torch.tensor([seed, offset], dtype=torch.int64, device=_dev())


def _table(rows, vocab, rng, max_len):
    """Ragged token histories padded with vocab (the reference's pad id), plus some junk ids."""
    table = np.full((rows, max_len), vocab, np.int64)
    for b in range(rows):
        n = int(rng.integers(0, max_len + 1))
        table[b, :n] = rng.integers(0, vocab, n)
    if max_len >= 2:
        table[0, -2:] = [-5, vocab + 3]  # outside [0, vocab): ignored
    return table


def _run(logits_f32, dtype, temps, pens, table, seed, offset, view_pad=0):
    """Kernel ids for logits given as fp32 values representable in `dtype`."""
    B, V = logits_f32.shape
    full = torch.zeros(B, V + view_pad, dtype=DT[dtype], device=_dev())
    full[:, :V] = torch.from_numpy(logits_f32).to(_dev(), DT[dtype])
    lg = full[:, :V]
    t = torch.from_numpy(np.asarray(temps, np.float32)).to(_dev())
    p = None if pens is None else torch.from_numpy(np.asarray(pens, np.float32)).to(_dev())
    tb = None if table is None else torch.from_numpy(table).to(_dev())
    state = _rng(seed, offset)
    ids = cabi.sample_tokens(lg, t, p, tb, state)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), state.cpu().numpy()


def _representable(x, dtype):
    return torch.from_numpy(x).to(DT[dtype]).float().numpy()


def _check_against_oracle(logits, dtype, temps, pens, table, seed, offset, ids, tol=3e-6):
    """Greedy rows: the oracle's argmax exactly.  Sampled rows: the kernel's token must carry weight
    and its CDF interval, widened by `tol` for the kernel's fp32 sums, must hold the row's uniform;
    most rows must also match the oracle's token exactly."""
    want, _ = S.sample(logits, dtype, temps, pens, table, seed=seed, offset=offset)
    p = S.probabilities(logits, dtype, temps, pens, table)
    u = S.uniforms(len(ids), seed, offset)
    greedy = np.asarray(temps, np.float32) < 1e-5
    np.testing.assert_array_equal(ids[greedy], want[greedy])
    for b in np.nonzero(~greedy)[0]:
        k = int(ids[b])
        assert p[b, k] > 0, (b, k)
        cdf = np.cumsum(p[b])
        cdf /= cdf[-1]
        lo = cdf[k - 1] if k > 0 else 0.0
        assert lo - tol <= u[b] <= cdf[k] + tol, (b, k, int(want[b]), lo, cdf[k], u[b])
    assert (ids == want).mean() >= 0.5


def test_greedy_golden_cases():
    for name, c in load_sampler_cases().items():
        greedy = c["temps"] < 1e-5
        if not greedy.any():
            continue
        ids, _ = _run(c["logits"], c["dtype"], c["temps"], c["pens"], c["table"], seed=1, offset=0)
        np.testing.assert_array_equal(ids[greedy], c["counts"].argmax(axis=1)[greedy], err_msg=name)


@pytest.mark.parametrize("dtype", ["bf16", "f32", "f16"])
@pytest.mark.parametrize("vocab", [151936, 50001, 12, 6149])
@pytest.mark.parametrize("penalty", [False, True])
def test_rows_match_oracle(dtype, vocab, penalty):
    rng = np.random.default_rng(vocab * 7 + len(dtype) + penalty)
    B = 12
    logits = _representable((rng.standard_normal((B, vocab)) * 2.5).astype(np.float32), dtype)
    if vocab > 1000:  # equal maxima across chunks: the first index wins
        logits[1, vocab - 3] = logits[1, 5] = logits[1].max() + 1
    temps = np.array([0.0, 0.0, 0.6, 1.0, 1.0, 1.4, 0.3, 2.0, 0.9, 0.0, 1.0, 1e-6], np.float32)
    pens = table = None
    if penalty:
        pens = np.array([1.0, 0.5, 2.0, 0.0, -0.4, 1.0, 1.0, 0.7, 1.0, 3.0, 0.0, 1.0], np.float32)
        table = _table(B, vocab, rng, 64)
        table[9, 0] = int(np.argmax(logits[9]))  # the penalty moves this greedy row's argmax
    ids, state = _run(logits, dtype, temps, pens, table, seed=1234 + vocab, offset=3)
    assert state[1] == 4
    _check_against_oracle(logits, dtype, temps, pens, table, 1234 + vocab, 3, ids)


def test_unaligned_rows_take_the_scalar_path():
    """Row stride V + 1 (bf16): rows are not 16-byte aligned; same answers as the oracle."""
    rng = np.random.default_rng(3)
    B, V = 6, 40000
    logits = _representable((rng.standard_normal((B, V)) * 3).astype(np.float32), "bf16")
    temps = np.array([0.0, 1.0, 0.8, 0.0, 1.2, 1.0], np.float32)
    pens = np.array([1.0, 0.0, 1.0, 0.0, 0.5, 1.0], np.float32)
    table = _table(B, V, rng, 100)
    ids, _ = _run(logits, "bf16", temps, pens, table, seed=9, offset=0, view_pad=1)
    _check_against_oracle(logits, "bf16", temps, pens, table, 9, 0, ids)


def test_degenerate_rows():
    """All -inf (greedy and sampled: token 0, like torch.argmax), one finite logit, near-uniform T."""
    V = 5000
    logits = np.zeros((5, V), np.float32)
    logits[0] = -np.inf
    logits[1] = -np.inf
    logits[2] = -np.inf
    logits[2, 4321] = 3.0
    logits[3, 17] = 1.0
    logits[4] = np.linspace(-1, 1, V, dtype=np.float32)
    temps = np.array([0.0, 1.0, 1.0, 1e-6, 1e4], np.float32)
    ids, _ = _run(logits, "f32", temps, None, None, seed=2, offset=0)
    assert ids[0] == 0 and ids[1] == 0 and ids[2] == 4321 and ids[3] == 17
    _check_against_oracle(logits, "f32", temps, None, None, 2, 0, ids)  # row 4's uniform is row 4's


def test_distribution_matches_reference_draws():
    """Each golden row repeated 5000 times in one launch (one Philox counter per row): the kernel's
    counts fit the oracle probabilities, which the reference's own draws fit (CPU test)."""
    R = 5000
    for name, c in load_sampler_cases().items():
        sampled = np.nonzero(c["temps"] >= 1e-5)[0]
        if len(sampled) == 0:
            continue
        B, V = c["logits"].shape
        rows = np.repeat(np.arange(B), R)
        ids, _ = _run(c["logits"][rows], c["dtype"], c["temps"][rows], c["pens"][rows], c["table"][rows],
                      seed=77, offset=0)
        p = S.probabilities(c["logits"], c["dtype"], c["temps"], c["pens"], c["table"])
        for b in range(B):
            got = np.bincount(ids[rows == b], minlength=V)
            if c["temps"][b] < 1e-5:
                assert got[c["counts"][b].argmax()] == R, (name, b)
                continue
            e = p[b] * R
            m = e > 0
            assert got[~m].sum() == 0, (name, b)
            chi = float((((got - e) ** 2)[m] / e[m]).sum())
            assert chi < chi2_critical(int(m.sum()) - 1), (name, b, chi)
            # and the two samples (kernel, reference) are homogeneous; tokens seen fewer than 20
            # times in both together are pooled into one bin
            obs = np.stack([got, c["counts"][b]])
            big = obs.sum(0) >= 20
            obs = np.concatenate([obs[:, big], obs[:, ~big].sum(1, keepdims=True)], axis=1)
            obs = obs[:, obs.sum(0) > 0]
            exp = obs.sum(1, keepdims=True) * obs.sum(0, keepdims=True) / obs.sum()
            chi_h = float(((obs - exp) ** 2 / exp).sum())
            assert chi_h < chi2_critical(obs.shape[1] - 1), (name, b, chi_h)


def test_rng_state_repeats_and_advances():
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal((16, 32000)) * 2).astype(np.float32)
    temps = np.ones(16, np.float32)
    a, sa = _run(logits, "f32", temps, None, None, seed=42, offset=10)
    b, sb = _run(logits, "f32", temps, None, None, seed=42, offset=10)
    c, _ = _run(logits, "f32", temps, None, None, seed=42, offset=11)
    np.testing.assert_array_equal(a, b)
    assert sa[1] == 11 and sb[1] == 11 and sa[0] == 42
    assert (a != c).any()
    _check_against_oracle(logits, "f32", temps, None, None, 42, 11, c)


def test_workspace_counters_left_zero_and_reusable():
    rng = np.random.default_rng(8)
    B, V = 64, 151936
    logits = torch.from_numpy((rng.standard_normal((B, V)) * 2).astype(np.float32)).to(_dev(), torch.bfloat16)
    temps = torch.full((B,), 0.8, device=_dev())
    ws = torch.zeros(cabi.lib().fvb_sample_workspace_size(B, V), dtype=torch.uint8, device=_dev())
    state = _rng(3)
    first = cabi.sample_tokens(logits, temps, None, None, state, ws)
    reserved = ws[:4].view(torch.int32)  # the workspace's reserved first word
    torch.cuda.synchronize()
    assert int(reserved.item()) == 0
    assert state.cpu().tolist() == [3, 1]  # one launch advanced the offset by one
    state2 = _rng(3)
    again = cabi.sample_tokens(logits, temps, None, None, state2, ws)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_graph_replay_draws_fresh_numbers():
    """sample_tokens captured in a CUDA graph: every replay advances the device offset."""
    from femtovllm_b200 import ops

    rng = np.random.default_rng(12)
    B, V = 32, 151936
    host = _representable((rng.standard_normal((B, V)) * 2).astype(np.float32), "bf16")
    logits = torch.from_numpy(host).to(_dev(), torch.bfloat16)
    temps_np = np.where(np.arange(B) % 4 == 0, 0.0, 1.0).astype(np.float32)
    temps = torch.from_numpy(temps_np).to(_dev())
    state = ops.new_rng_state(99, _dev())
    ws = ops.sample_workspace(B, V, _dev())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = ops.sample_tokens(logits, temps, None, None, state, ws)  # warm-up, offset 0
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    _check_against_oracle(host, "bf16", temps_np, None, None, 99, 0, out.cpu().numpy())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ops.sample_tokens(logits, temps, None, None, state, ws)
    for off in (1, 2, 3):
        g.replay()
        torch.cuda.synchronize()
        _check_against_oracle(host, "bf16", temps_np, None, None, 99, off, out.cpu().numpy())
    assert int(state[1]) == 4
    del g


def test_sampler_module_is_a_dropin():
    """femtovllm_b200.sampler.Sampler takes the reference's (logits, scheduled) and returns a list."""
    from types import SimpleNamespace

    from femtovllm_b200.sampler import Sampler

    c = load_sampler_cases()["greedy_pen_f32"]
    seqs = [(SimpleNamespace(token_ids=[int(t) for t in row if t < c["logits"].shape[1]],
                             sampling_params=SimpleNamespace(temperature=float(tp), presence_penalty=float(pp))), 1)
            for row, tp, pp in zip(c["table"], c["temps"], c["pens"])]
    ids = Sampler(seed=1)(torch.from_numpy(c["logits"]).to(_dev()), seqs)
    assert isinstance(ids, list) and all(isinstance(i, int) for i in ids)
    assert ids == [int(i) for i in c["counts"].argmax(axis=1)]
