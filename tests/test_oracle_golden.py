"""The CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py)."""

import numpy as np
import pytest

import oracle
from conftest import GOLDEN_CASES, golden_after, load_golden


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
