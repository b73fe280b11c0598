"""CPU-side checks: the C ABI loads and validates, the host mirror imports, workloads and sharding."""

import ctypes
import os
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from femtovllm_b200 import capi, workloads


@pytest.fixture(scope="module")
def lib():
    return capi.load()


def test_library_exports_every_header_symbol(lib):
    names = capi.header_symbols()
    assert len(names) >= 11
    for n in names:
        assert hasattr(lib, n), n


def test_constants(lib):
    assert lib.fvb_kv_len_per_page() == 16
    assert lib.fvb_dim_head() == 128
    assert lib.fvb_max_kv_len() >= 131072  # split-KV lifts the reference's 8192 cap
    assert lib.fvb_status_string(0) == b"FVB_OK"
    assert lib.fvb_status_string(7) == b"FVB_ERR_BAD_PAGE"


def _decode_args(**over):
    a = dict(q=16, out=16, k=16, v=16, nb=10, hq=8, hkv=2, d=128, bs=16, b=2, tables=16, maxblk=4, lens=16,
             maxkv=50, dtype=1, ws=0, wsb=0, stream=None)
    a.update(over)
    return (a["q"], a["out"], a["k"], a["v"], a["nb"], a["hq"], a["hkv"], a["d"], a["bs"], a["b"], a["tables"],
            a["maxblk"], a["lens"], a["maxkv"], a["dtype"], a["ws"], a["wsb"], a["stream"])


@pytest.mark.parametrize(
    "over,status",
    [
        (dict(d=96), 2),  # head_dim
        (dict(hq=7, hkv=2), 2),  # heads not a whole number of GQA groups
        (dict(bs=32), 2),  # block size
        (dict(dtype=7), 2),
        (dict(q=8), 3),  # 16-byte rule
        (dict(nb=0), 1),
        (dict(b=-1), 1),
        (dict(maxkv=65), 1),  # longer than the block-table row
    ],
)
def test_decode_rejects_bad_arguments_without_touching_the_device(lib, over, status):
    assert lib.fvb_paged_attention_decode(*_decode_args(**over)) == status


def test_store_rejects_bad_arguments(lib):
    # dtype, negative sizes, misaligned slot mapping
    assert lib.fvb_store_kvcache(16, 16, 256, 128, 16, 16, 10, 16, 4, 2, 128, 16, 9, None) == 2
    assert lib.fvb_store_kvcache(16, 16, 256, 128, 16, 16, 10, 16, -1, 2, 128, 16, 1, None) == 1
    assert lib.fvb_store_kvcache(16, 16, 256, 128, 16, 16, 10, 12, 4, 2, 128, 16, 1, None) == 3
    assert lib.fvb_store_kvcache(0, 0, 0, 0, 0, 0, 0, 0, 0, 2, 128, 16, 1, None) == 0  # empty: no-op
    # any positive page size is a valid write target; zero is not
    assert lib.fvb_store_kvcache(16, 16, 256, 128, 16, 16, 10, 16, 4, 2, 128, 0, 1, None) == 1


def test_prefill_rejects_bad_arguments(lib):
    args = [16, 16, 16, 16, 10, 8, 2, 128, 16, 2, 20, 16, 10, 16, 4, 16, 16, 1, 0, 0, None]
    bad = list(args)
    bad[7] = 80
    assert lib.fvb_paged_attention_prefill(*bad) == 2
    bad = list(args)
    bad[11] = 0  # cu_seqlens null
    assert lib.fvb_paged_attention_prefill(*bad) == 1
    bad = list(args)
    bad[8] = 32  # attention reads 16-token pages only
    assert lib.fvb_paged_attention_prefill(*bad) == 2


def _sample_args(**over):
    """fvb_sample_tokens arguments with fake (never dereferenced) 256-byte aligned pointers."""
    a = dict(logits=256, row_stride=1024, num_rows=4, vocab=1000, dtype=1, temps=256, pens=256, table=256,
             table_stride=8, table_len=8, rng=256, out=256, ws=256, ws_bytes=1 << 20, stream=None)
    a.update(over)
    return [a[k] for k in ("logits", "row_stride", "num_rows", "vocab", "dtype", "temps", "pens", "table",
                           "table_stride", "table_len", "rng", "out", "ws", "ws_bytes", "stream")]


@pytest.mark.parametrize(
    "over,status",
    [
        (dict(dtype=9), 2),                      # unsupported dtype
        (dict(vocab=0), 1),                      # empty vocabulary
        (dict(row_stride=999), 1),               # rows overlap
        (dict(table=0), 1),                      # table_len > 0 without a table
        (dict(table_stride=4), 1),               # table rows overlap
        (dict(out=0), 1),                        # no output
        (dict(ws_bytes=16), 4),                  # workspace too small
        (dict(ws=264), 3),                       # workspace not 16-byte aligned
        (dict(rng=260), 3),                      # rng state not 8-byte aligned
        (dict(num_rows=0), 0),                   # empty batch: no-op
    ],
)
def test_sample_rejects_bad_arguments_without_touching_the_device(lib, over, status):
    assert lib.fvb_sample_tokens(*_sample_args(**over)) == status


def test_sample_workspace_size(lib):
    assert lib.fvb_sample_workspace_size(0, 1000) == 0
    small = lib.fvb_sample_workspace_size(4, 1000)
    assert small > 0 and lib.fvb_sample_workspace_size(256, 151936) > 64 * small


def test_decode_workspace_plan(lib):
    # Plenty of (seq, kv head) units and short contexts: no split, no workspace.
    assert lib.fvb_paged_attention_decode_workspace_size(1024, 16, 8, 128, 512) == 0
    # Long contexts split; the workspace holds a partial row + a log-sum-exp per (seq, head, split).
    # (131,072 tokens over 8 sequences: 4096-token splits, 32 per sequence)
    ws = lib.fvb_paged_attention_decode_workspace_size(8, 32, 8, 128, 131072)
    assert ws >= 8 * 32 * (131072 // 4096) * 129 * 4
    # config-2 lengths keep 1024-token splits
    assert lib.fvb_paged_attention_decode_workspace_size(16, 16, 8, 128, 4096) >= 16 * 16 * 4 * 129 * 4
    assert lib.fvb_paged_attention_decode_workspace_size(0, 32, 8, 128, 131072) == 0


def test_prefill_workspace_reserves_single_token_partials(lib):
    # The tile plan: order[num_seqs] padded to 64 entries + cu_items[num_seqs + 1], int32, 256-byte rounded.
    plan = lambda n: ((-(-n // 64) * 64 + n + 1) * 4 + 255) // 256 * 256  # noqa: E731
    # GQA 1-4: the single-token sequences' split partials follow (16 splits per (sequence, head)).
    rows = 32 * 32 * 16
    single = (rows * 128 * 4 + 255) // 256 * 256 + rows * 4
    assert lib.fvb_paged_attention_prefill_workspace_size(32, 32, 8, 128, 4120, 512) == plan(32) + single
    # GQA 8 keeps its decode rows in tensor-core tiles: the plan alone.
    assert lib.fvb_paged_attention_prefill_workspace_size(32, 64, 8, 128, 4120, 512) == plan(32)
    # Past 64 MB of partials the single-token sequences stay on the tensor-core kernel as well.
    assert lib.fvb_paged_attention_prefill_workspace_size(4096, 32, 8, 128, 4096, 1) == plan(4096)


def test_torch_extension_mirrors_reference_module():
    from femtovllm_b200 import _C, ops

    for name in ("PagedAttentionGemvCuda", "PagedAttentionGemmCuda", "StoreKVCacheCuda"):
        assert callable(getattr(_C, name))
    assert (ops.KV_LEN_PER_PAGE, ops.DIM_HEAD) == (16, 128)
    assert ops.MAX_KV_LEN_NON_SPLIT >= 131072
    assert hasattr(torch.ops.femtovllm_b200, "paged_attention_decode")
    assert hasattr(torch.ops.femtovllm_b200, "paged_attention_prefill")
    assert hasattr(torch.ops.femtovllm_b200, "store_kvcache")


def test_ops_reject_cpu_tensors_like_the_reference():
    from femtovllm_b200 import ops

    q = torch.zeros(8, 2, 128)
    pool = torch.zeros(4, 2, 16, 128)
    with pytest.raises(ValueError):
        ops.paged_attention_gemv(q, pool, pool, torch.zeros(2, 1, dtype=torch.int32), torch.ones(2, dtype=torch.int32), 1)
    with pytest.raises(ValueError):
        ops.store_kvcache(torch.zeros(2, 2, 128), torch.zeros(2, 2, 128), pool, pool, torch.zeros(2, dtype=torch.int64))


REFERENCE = Path(os.environ.get("FEMTOVLLM_REFERENCE", Path(__file__).resolve().parents[2] / "reference"))


@pytest.mark.skipif(not (REFERENCE / "femtovllm" / "ops" / "__init__.py").exists(), reason="reference tree absent")
def test_reference_ops_module_binds_this_extension_as_its_C(monkeypatch):
    """Drop-in: the reference's femtovllm.ops imports with femtovllm._C = femtovllm_b200._C."""
    import subprocess
    import sys

    code = f"""
import sys
sys.path.insert(0, {str(REFERENCE)!r})
from femtovllm_b200 import _C
sys.modules['femtovllm._C'] = _C
import femtovllm.ops as fops
assert fops._cuda_backend is _C
assert fops.KV_LEN_PER_PAGE == 16 and fops.DIM_HEAD == 128
assert fops.MAX_KV_LEN_NON_SPLIT >= 131072
print('ok')
"""
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(Path(__file__).resolve().parents[1] / "nano-vllm-practice_b200")])
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert res.returncode == 0 and "ok" in res.stdout, res.stderr[-2000:]


# ---------------------------------------------------------------------------
# workloads and sharding
# ---------------------------------------------------------------------------


def test_config_shapes():
    c1 = workloads.config1()
    assert (c1.n_heads, c1.n_kv_heads, c1.head_dim, c1.num_blocks, c1.dtype) == (8, 2, 64, 128, torch.float32)
    assert c1.kv_lens.min() >= 2 and c1.kv_lens.max() <= 257
    c2 = workloads.config2()
    assert c2.num_seqs == 256 and c2.kv_lens.min() >= 512 and c2.kv_lens.max() <= 4096
    assert c2.num_blocks == int(np.ceil(1.2 * ((c2.kv_lens + 15) // 16).sum()))
    c3 = workloads.config3()
    assert c3.num_seqs == 64 and c3.q_lens.min() >= 128 and c3.q_lens.max() <= 2048
    assert (c3.kv_lens - c3.q_lens).max() <= 8192
    c4 = workloads.config4()
    assert (c4.q_lens == 1).sum() == 24 and (c4.q_lens == 512).sum() == 8
    assert (c4.block_tables[:, :256] == c4.block_tables[0, :256]).all()


@pytest.mark.parametrize("cfg", [workloads.config1, workloads.config2, workloads.config3, workloads.config4])
def test_tables_cover_kv_and_slots_match_oracle(cfg):
    b = cfg()
    npages = (b.kv_lens + 15) // 16
    for s in range(b.num_seqs):
        row = b.block_tables[s]
        assert (row[: npages[s]] >= 0).all() and (row[npages[s] :] == -1).all()
        assert row[: npages[s]].max() < b.num_blocks
    slots = oracle.build_slot_mapping(b.positions, b.seq_of_token, b.block_tables)
    assert np.array_equal(slots, b.slot_mapping)
    assert len(np.unique(slots)) == len(slots)  # every new token gets its own slot


def test_private_blocks_are_disjoint():
    b = workloads.config4()
    private = np.concatenate([r[256:][r[256:] >= 0] for r in b.block_tables])
    assert len(np.unique(private)) == len(private)
    assert not set(private) & set(b.block_tables[0, :256])


def test_lpt_sharding_balances_and_partitions():
    lengths = workloads.config5_lengths()
    for world in (1, 2, 4, 8):
        parts = workloads.shard_lpt(lengths, world)
        allidx = np.sort(np.concatenate(parts))
        assert np.array_equal(allidx, np.arange(len(lengths)))
        loads = [lengths[p].sum() for p in parts]
        assert max(loads) <= min(loads) + lengths.max()


def test_algorithmic_work_formulas():
    b = workloads.custom([20, 5], [4, 1], 4, 2, 64, torch.bfloat16)
    # pairs: seq0: 4 queries with prefix 16 -> 4*16 + 4*5/2 = 74; seq1: 1 query, prefix 4 -> 4 + 1 = 5
    assert b.attn_flops() == 4 * 64 * 4 * 79
    assert b.kv_bytes() == 2 * 25 * 2 * 64 * 2
