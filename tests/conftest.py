import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "nano-vllm-practice_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def load_golden(name: str) -> dict:
    """Decode one fixture written by tests/golden/make_golden.py (float32 arrays)."""
    z = np.load(GOLDEN / f"{name}.npz")
    d = {k: z[k] for k in z.files}
    for k in ("q", "k_new", "v_new", "k_pool", "v_pool"):
        d[k] = _bits_to_f32(d.pop(f"{k}_bits"))
    for k in ("k", "v"):
        d[f"{k}_written_rows"] = _bits_to_f32(d.pop(f"{k}_written_bits"))
    for k in ("n_heads", "n_kv_heads", "head_dim", "num_blocks"):
        d[k] = int(d[k])
    q_lens = d["q_lens"]
    d["seq_of_token"] = np.repeat(np.arange(len(q_lens)), q_lens)
    d["is_decode"] = bool((q_lens == 1).all())
    return d


def golden_after(d: dict, which: str) -> np.ndarray:
    """The pool the reference produced: pool before, with the rows it wrote."""
    pool = d[f"{which}_pool"].copy()
    idx = d[f"{which}_written_idx"]
    pool[idx[:, 0], idx[:, 1], idx[:, 2]] = d[f"{which}_written_rows"]
    return pool


GOLDEN_CASES = sorted(
    p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("norm_rope_", "metadata_", "sampler"))
)
NORM_ROPE_CASES = sorted(p.stem for p in GOLDEN.glob("norm_rope_*.npz"))


def load_norm_rope(name: str) -> dict:
    """Decode one norm_rope_* fixture (q/k RMSNorm + rotary embedding + KV write stage)."""
    z = np.load(GOLDEN / f"{name}.npz")
    d = {k: z[k] for k in z.files}
    for k in ("q", "k_new", "v_new", "k_pool", "v_pool", "q_norm_weight", "k_norm_weight"):
        d[k] = _bits_to_f32(d.pop(f"{k}_bits"))
    d["v_written_rows"] = _bits_to_f32(d.pop("v_written_bits"))
    d["k_written_rows"] = d.pop("k_written")
    for k in ("n_heads", "n_kv_heads", "head_dim", "num_blocks", "rope_rows"):
        d[k] = int(d[k])
    d["eps"] = float(d["eps"])
    q_lens = d["q_lens"]
    d["seq_of_token"] = np.repeat(np.arange(len(q_lens)), q_lens)
    return d


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def load_sampler_cases() -> dict:
    """tests/golden/sampler.npz as {case: {dtype, logits, temps, pens, table, counts}}."""
    z = np.load(GOLDEN / "sampler.npz")
    out = {}
    for name in (str(n) for n in z["names"]):
        out[name] = {k: z[f"{name}_{k}"] for k in ("logits", "temps", "pens", "table", "counts")}
        out[name]["dtype"] = str(z[f"{name}_dtype"])
    return out


def chi2_critical(dof: int, alpha: float = 1e-4) -> float:
    from scipy.stats import chi2

    return float(chi2.ppf(1.0 - alpha, dof))
