"""The CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py)."""

import numpy as np
import pytest

import oracle
from conftest import GOLDEN_CASES, chi2_critical, golden_after, load_golden, load_sampler_cases


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_slot_scatter_matches_reference_write(name):
    d = load_golden(name)
    slots = oracle.build_slot_mapping(d["positions"], d["seq_of_token"], d["block_tables"])
    kp, vp = d["k_pool"].copy(), d["v_pool"].copy()
    oracle.store_kvcache(d["k_new"], d["v_new"], kp, vp, slots)
    assert np.array_equal(kp.view(np.uint32), golden_after(d, "k").view(np.uint32))
    assert np.array_equal(vp.view(np.uint32), golden_after(d, "v").view(np.uint32))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_literal_write_loops_match_reference(name):
    d = load_golden(name)
    kp, vp = d["k_pool"].copy(), d["v_pool"].copy()
    tables = [[int(x) for x in row if x >= 0] for row in d["block_tables"]]
    if d["is_decode"]:
        oracle.store_kvcache_decode_loop(d["k_new"], d["v_new"], kp, vp, d["positions"], tables)
    else:
        oracle.store_kvcache_prefill_loop(d["k_new"], d["v_new"], kp, vp, d["positions"], d["cu_seqlens"], tables)
    assert np.array_equal(kp, golden_after(d, "k"))
    assert np.array_equal(vp, golden_after(d, "v"))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_attention_matches_reference(name):
    d = load_golden(name)
    kp, vp = golden_after(d, "k"), golden_after(d, "v")
    if d["is_decode"]:
        out = oracle.decode_attention(d["q"], kp, vp, d["block_tables"], d["kv_lens"])
    else:
        out = oracle.prefill_attention(d["q"], kp, vp, d["cu_seqlens"], d["block_tables"], d["kv_lens"], d["positions"])
    # The reference ran fp32 SDPA; the oracle accumulates in fp64.
    err = np.abs(out - d["out_ref"]).max()
    assert err < 2e-5, err


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_torch_restatement_matches_reference(name):
    """tests/torch_ref.py (the full-row checker of the GPU tests) on the reference's own outputs."""
    import torch

    import torch_ref

    d = load_golden(name)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    kp, vp = t(golden_after(d, "k")), t(golden_after(d, "v"))
    out = torch_ref.paged_attention_fp32(t(d["q"]), kp, vp, t(d["cu_seqlens"]), t(d["block_tables"]),
                                         t(d["kv_lens"]), t(d["positions"]), q_chunk=5)
    assert np.abs(out.numpy() - d["out_ref"]).max() < 2e-5
    if d["is_decode"]:
        dec = torch_ref.paged_attention_fp32(t(d["q"]), kp, vp, None, t(d["block_tables"]), t(d["kv_lens"]))
        assert np.abs(dec.numpy() - d["out_ref"]).max() < 2e-5


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_decode_and_prefill_forms_agree(name):
    d = load_golden(name)
    if not d["is_decode"]:
        pytest.skip("prefill case")
    kp, vp = golden_after(d, "k"), golden_after(d, "v")
    a = oracle.decode_attention(d["q"], kp, vp, d["block_tables"], d["kv_lens"])
    b = oracle.prefill_attention(d["q"], kp, vp, d["cu_seqlens"], d["block_tables"], d["kv_lens"], d["positions"])
    assert np.allclose(a, b, atol=1e-12)


def test_oracle_catches_a_planted_mask_error():
    """A wrong mask (j < pos instead of j <= pos) in a copy of the oracle must fail the check."""
    d = load_golden("toy_prefill")
    kp, vp = golden_after(d, "k"), golden_after(d, "v")
    hq, _, dd = d["q"].shape
    s = 0
    q0, q1 = d["cu_seqlens"][s], d["cu_seqlens"][s + 1]
    ks = oracle.gather_seq_kv(kp, d["block_tables"][s], d["kv_lens"][s])
    vs = oracle.gather_seq_kv(vp, d["block_tables"][s], d["kv_lens"][s])
    pos = d["positions"][q0:q1]
    bad_visible = np.arange(d["kv_lens"][s])[None, :] < pos[:, None]
    n_rep = hq // kp.shape[1]
    bad = oracle.paged_attention._attend(d["q"][:n_rep, q0:q1], ks[0], vs[0], bad_visible, np.float64)
    assert np.abs(bad - d["out_ref"][:n_rep, q0:q1]).max() > 1e-3


# ---------------------------------------------------------------------------
# q/k RMSNorm + rotary embedding + KV write (norm_rope_* fixtures)
# ---------------------------------------------------------------------------

from conftest import NORM_ROPE_CASES, load_norm_rope  # noqa: E402


@pytest.mark.parametrize("name", NORM_ROPE_CASES)
def test_rope_tables_match_reference_buffers(name):
    d = load_norm_rope(name)
    cos, sin = oracle.rope_tables(d["rope_rows"], d["head_dim"])
    # Same float32 formula, but torch's pow rounds a few inv_freq entries one
    # ulp away from numpy's; theta = pos * inv_freq carries that ulp times pos
    # (up to ~1e-4 at position 3000).
    assert np.abs(cos[d["positions"]] - d["cos_rows"]).max() < 2e-4
    assert np.abs(sin[d["positions"]] - d["sin_rows"]).max() < 2e-4


@pytest.mark.parametrize("name", NORM_ROPE_CASES)
def test_norm_rope_store_matches_reference(name):
    d = load_norm_rope(name)
    cos, sin = oracle.rope_tables(d["rope_rows"], d["head_dim"])
    cos[d["positions"]] = d["cos_rows"]  # the reference module's own buffer rows
    sin[d["positions"]] = d["sin_rows"]
    slots = oracle.build_slot_mapping(d["positions"], d["seq_of_token"], d["block_tables"])
    kp, vp = d["k_pool"].copy(), d["v_pool"].copy()
    q_out = oracle.qk_norm_rope_store(d["q"], d["k_new"], d["v_new"], d["q_norm_weight"], d["k_norm_weight"],
                                      d["eps"], cos, sin, d["positions"], kp, vp, slots)
    # The reference ran fp32 (a handful of roundings per element); the oracle is fp64.
    assert np.abs(q_out - d["q_ref"]).max() < 2e-6
    changed = np.argwhere((kp != d["k_pool"]).any(-1))
    assert np.array_equal(changed, d["k_written_idx"])
    assert np.abs(kp[tuple(changed.T)] - d["k_written_rows"]).max() < 2e-6
    vidx = d["v_written_idx"]
    assert np.array_equal(vp[vidx[:, 0], vidx[:, 1], vidx[:, 2]].view(np.uint32),
                          d["v_written_rows"].view(np.uint32))
    untouched = np.ones(vp.shape[:3], bool)
    untouched[vidx[:, 0], vidx[:, 1], vidx[:, 2]] = False
    assert np.array_equal(vp[untouched], d["v_pool"][untouched])


def test_norm_rope_oracle_catches_a_planted_rotation_error():
    """Rotating with cat(y2, -y1) (the wrong sign convention) in a copy of the oracle must fail."""
    d = load_norm_rope(NORM_ROPE_CASES[0])
    x = oracle.rms_norm(d["q"], d["q_norm_weight"], d["eps"])
    half = x.shape[-1] // 2
    c = d["cos_rows"][:, None, :].astype(np.float64)
    s = d["sin_rows"][:, None, :].astype(np.float64)
    bad = c * x + s * np.concatenate([x[..., half:], -x[..., :half]], axis=-1)
    assert np.abs(bad.transpose(1, 0, 2) - d["q_ref"]).max() > 1e-2


# ---------------------------------------------------------------------------
# per-step metadata (metadata_routes.npz, from the reference's ModelRunner routes)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("route", ["prefill", "decode"])
def test_varlen_metadata_matches_reference_routes(route):
    from conftest import GOLDEN

    z = np.load(GOLDEN / "metadata_routes.npz")
    flat, cu_b = z[f"{route}_flat_blocks"], z[f"{route}_cu_blocks"]
    tables = [flat[cu_b[i] : cu_b[i + 1]].tolist() for i in range(len(cu_b) - 1)]
    md = oracle.varlen_metadata(z[f"{route}_num_computed"], z[f"{route}_num_new"], tables)
    assert np.array_equal(md["positions"], z[f"{route}_positions"])
    assert np.array_equal(md["kv_lens"], z[f"{route}_kv_lens"])
    assert np.array_equal(md["block_tables"], z[f"{route}_block_tables"])
    assert md["max_q_len"] == int(z[f"{route}_max_q_len"]) and md["max_kv_len"] == int(z[f"{route}_max_kv_len"])
    if f"{route}_cu_seqlens" in z.files:
        assert np.array_equal(md["cu_seqlens"], z[f"{route}_cu_seqlens"])


# ---------------------------------------------------------------------------
# Sampler (femtovllm/engine/sampler.py)
# ---------------------------------------------------------------------------
def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors of its authors' Random123 distribution."""
    from oracle.sampler import philox4x32_10

    kat = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in kat:
        got = philox4x32_10(np.array([ctr], np.uint64), key)[0]
        assert tuple(int(x) for x in got) == want


def test_sampler_greedy_matches_reference():
    """Greedy rows: the reference's ids (ties, penalties that move the argmax, negative and tiny penalties)."""
    from oracle import sampler as S

    cases = load_sampler_cases()
    for name, c in cases.items():
        greedy = c["temps"] < 1e-5
        if not greedy.any():
            continue
        ref_ids = c["counts"].argmax(axis=1)
        assert (c["counts"][greedy].max(axis=1) == c["counts"][greedy].sum(axis=1)).all(), name
        ids, _ = S.sample(c["logits"], c["dtype"], c["temps"], c["pens"], c["table"])
        np.testing.assert_array_equal(ids[greedy], ref_ids[greedy], err_msg=name)


def test_sampler_distribution_matches_reference_draws():
    """Sampled rows: the reference's multinomial counts fit the oracle's probabilities (chi-square,
    alpha 1e-4), with and without the batch-wide penalty that keeps bf16 logits in fp32."""
    from oracle import sampler as S

    for name, c in load_sampler_cases().items():
        p = S.probabilities(c["logits"], c["dtype"], c["temps"], c["pens"], c["table"])
        for b in np.nonzero(c["temps"] >= 1e-5)[0]:
            n = c["counts"][b].sum()
            e = p[b] * n
            m = e > 0
            assert c["counts"][b][~m].sum() == 0, (name, b)
            chi = float((((c["counts"][b] - e) ** 2)[m] / e[m]).sum())
            assert chi < chi2_critical(int(m.sum()) - 1), (name, b, chi)


def test_sampler_oracle_catches_a_planted_temperature_error():
    """The distribution test has power: dividing by T twice fails it."""
    from oracle import sampler as S

    c = load_sampler_cases()["dist_bf16"]
    bad_t = c["temps"] * c["temps"]
    p = S.probabilities(c["logits"], c["dtype"], bad_t, c["pens"], c["table"])
    b = 0
    e = p[b] * c["counts"][b].sum()
    chi = float((((c["counts"][b] - e) ** 2) / e).sum())
    assert chi > chi2_critical(len(e) - 1)
