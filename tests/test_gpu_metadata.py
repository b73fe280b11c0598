"""GPU parity of build_varlen_metadata (positions, cu_seqlens, kv_lens, padded block tables, slots).

Integer work: every output must equal the oracle (pinned to the reference's own
ModelRunner routes by tests/golden/metadata_routes.npz) exactly.
"""

import ctypes

import numpy as np
import pytest
import torch

import cabi
import oracle
from conftest import GOLDEN
from femtovllm_b200 import ops

pytestmark = pytest.mark.gpu


def _check(num_computed, num_new, tables, dev):
    flat = np.asarray([b for t in tables for b in t], np.int32)
    cu_b = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int32)
    width = max(len(t) for t in tables)
    T = int(np.sum(num_new))
    d = lambda a: torch.from_numpy(np.asarray(a, np.int32)).to(dev)  # noqa: E731
    cabi.read_device_error()
    got = ops.build_varlen_metadata(d(num_computed), d(num_new), d(flat), d(cu_b), width, T)
    assert cabi.read_device_error() == (0, 0)
    ref = oracle.varlen_metadata(num_computed, num_new, tables)
    for k in ("positions", "cu_seqlens", "kv_lens", "block_tables", "slot_mapping"):
        assert np.array_equal(got[k].cpu().numpy(), ref[k]), k


@pytest.mark.parametrize("route", ["prefill", "decode"])
def test_golden_routes(route, cuda_device):
    z = np.load(GOLDEN / "metadata_routes.npz")
    flat, cu_b = z[f"{route}_flat_blocks"], z[f"{route}_cu_blocks"]
    tables = [flat[cu_b[i] : cu_b[i + 1]].tolist() for i in range(len(cu_b) - 1)]
    _check(z[f"{route}_num_computed"], z[f"{route}_num_new"], tables, cuda_device)


@pytest.mark.parametrize("B", [1, 256, 3000])
def test_random_batches(B, cuda_device):
    rng = np.random.default_rng(B)
    num_computed = rng.integers(0, 5000, size=B)
    num_new = np.where(rng.random(B) < 0.7, 1, rng.integers(1, 700, size=B))
    free = list(rng.permutation(int(((num_computed + num_new) // 16 + 2).sum()) + 16))
    tables = []
    for p, n in zip(num_computed, num_new):
        need = (int(p + n) + 15) // 16
        row = [int(free.pop()) for _ in range(need + int(rng.integers(0, 2)))]
        if rng.random() < 0.1 and len(row) > 1:
            row[-1] = -1  # a -1 entry past the sequence's pages
        tables.append(row)
    _check(num_computed, num_new, tables, cuda_device)


def test_feeds_store_and_prefill(cuda_device):
    """The slots it builds are the ones build_slot_mapping builds from its own positions / tables."""
    rng = np.random.default_rng(7)
    num_computed, num_new = rng.integers(0, 300, size=9), rng.integers(1, 90, size=9)
    free = list(rng.permutation(1000))
    tables = [[int(free.pop()) for _ in range((int(p + n) + 15) // 16)] for p, n in zip(num_computed, num_new)]
    d = lambda a: torch.from_numpy(np.asarray(a, np.int32)).to(cuda_device)  # noqa: E731
    flat = [b for t in tables for b in t]
    cu_b = np.concatenate([[0], np.cumsum([len(t) for t in tables])])
    md = ops.build_varlen_metadata(d(num_computed), d(num_new), d(flat), d(cu_b), max(map(len, tables)),
                                   int(num_new.sum()))
    slots = ops.build_slot_mapping(md["positions"], md["block_tables"], md["cu_seqlens"])
    assert torch.equal(slots, md["slot_mapping"])


def test_mismatches_are_reported(cuda_device):
    d = lambda a: torch.from_numpy(np.asarray(a, np.int32)).to(cuda_device)  # noqa: E731
    cabi.read_device_error()
    # num_tokens one short of sum(num_new)
    ops.build_varlen_metadata(d([0, 5]), d([3, 4]), d([1, 2]), d([0, 1, 2]), 1, 6)
    assert cabi.read_device_error()[0] == 1  # FVB_ERR_INVALID_ARGUMENT
    # a row longer than max_blocks_per_seq is not read
    md = ops.build_varlen_metadata(d([0, 0]), d([3, 4]), d([1, 2, 3]), d([0, 2, 3]), 1, 7)
    code, info = cabi.read_device_error()
    assert (code, info) == (1, 0)
    assert md["block_tables"].cpu().tolist() == [[-1], [3]]
    lib = cabi.lib()
    st = lib.fvb_build_varlen_metadata(None, None, 0, None, 0, None, 0, 0, None, None, None, None, None,
                                       ctypes.c_void_p(0))
    assert st == 1
