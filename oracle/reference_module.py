"""The reference's own attention module, imported from its installed copy (test infrastructure).

Checker and CPU-baseline code only: the GPU drop-in test (``tests/test_gpu_dropin_reference.py``)
and ``bench.py``'s CPU legs use it; the product package never imports it.

The reference package (fishAndShrimp/nano-vllm-practice, "FemtoVLLM") is installed with
``pip install --no-index --no-build-isolation --target baseline/_ref <reference tree>``
into ``baseline/_ref`` (git-ignored; it travels to the GPU box with the working tree).
``femtovllm/ops/__init__.py:6-26`` binds ``femtovllm._C`` at import time, so this module
puts this repository's extension (``femtovllm_b200._C``, same entry names, argument order
and attributes) into ``sys.modules["femtovllm._C"]`` first: the reference then runs its
own Python code (``QwenSelfAttention``, ``femtovllm.ops``, the Triton prefill) with this
repository's kernels behind ``PagedAttentionGemvCuda`` / ``PagedAttentionGemmCuda``,
which is the drop-in the boundary promises.  The reference's own compiled ``_C`` is never
loaded.

``attention_module`` builds a ``QwenSelfAttention`` (``femtovllm/models/qwen/qwen3.py:141``)
whose projections slice a packed input ``x = [q | k | v]`` and whose q/k norms, rotary
embedding and o_proj are identities, so that its forwards compute exactly the attention
of given q / k / v (the same construction ``tests/golden/make_golden.py`` uses).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]
REF_DIR = REPO / "baseline" / "_ref"
PAGE = 16

_ref = None


def available() -> bool:
    return (REF_DIR / "femtovllm" / "__init__.py").exists()


def import_reference():
    """(femtovllm, QwenSelfAttention, VarlenAttnMetadata, ImplCustomKernel) from baseline/_ref."""
    global _ref
    if _ref is not None:
        return _ref
    if not available():
        raise ImportError(f"the reference is not installed under {REF_DIR}")
    pkg_root = str(REPO / "nano-vllm-practice_b200")
    if pkg_root not in sys.path:
        sys.path.insert(0, pkg_root)
    from femtovllm_b200 import _C as this_extension

    loaded = sys.modules.get("femtovllm")
    if loaded is not None and not str(getattr(loaded, "__file__", "")).startswith(str(REF_DIR)):
        raise ImportError(f"another femtovllm is already imported: {loaded.__file__}")
    sys.modules["femtovllm._C"] = this_extension
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import femtovllm
    import femtovllm.ops
    from femtovllm.models.qwen.qwen3 import QwenSelfAttention
    from femtovllm.protocol import ImplCustomKernel, VarlenAttnMetadata

    assert femtovllm.ops._cuda_backend is this_extension
    _ref = (femtovllm, QwenSelfAttention, VarlenAttnMetadata, ImplCustomKernel)
    return _ref


class _Slice(torch.nn.Module):
    def __init__(self, a, b):
        super().__init__()
        self.a, self.b = a, b

    def forward(self, x):
        return x[:, self.a : self.b]


class _NoRope(torch.nn.Module):
    def forward(self, x, positions=None):
        return x


def attention_module(n_heads: int, n_kv_heads: int, head_dim: int):
    """A QwenSelfAttention computing plain attention of the q / k / v packed in its input."""
    import types

    _, QwenSelfAttention, _, _ = import_reference()
    cfg = types.SimpleNamespace(head_dim=head_dim, rms_norm_eps=1e-6)
    d_model = head_dim * (n_heads + 2 * n_kv_heads)
    attn = QwenSelfAttention(d_model, n_heads, n_kv_heads, max_seqlen=4, dropout_p=0.0, config=cfg)
    hq, hk = n_heads * head_dim, n_kv_heads * head_dim
    attn.w_q = _Slice(0, hq)
    attn.w_k = _Slice(hq, hq + hk)
    attn.w_v = _Slice(hq + hk, hq + 2 * hk)
    attn.q_norm = torch.nn.Identity()
    attn.k_norm = torch.nn.Identity()
    attn.rotary_embd = _NoRope()
    attn.o_proj = torch.nn.Identity()
    return attn.eval()


def packed_input(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor) -> torch.Tensor:
    """x = [q | k | v] per token from q (Hq, T, D) and k_new / v_new (T, Hkv, D)."""
    hq, t, d = q.shape
    return torch.cat([q.transpose(0, 1).reshape(t, hq * d), k_new.reshape(t, -1), v_new.reshape(t, -1)], dim=1)


def metadata(kv_lens, q_lens, block_tables, device, q_tile: int = 32):
    """The reference's VarlenAttnMetadata (femtovllm/protocol.py:58-81) for one batch, built the way
    ModelRunner._route_prefill / _route_decode build it (model_runner.py:159-339)."""
    _, _, VarlenAttnMetadata, _ = import_reference()
    kv_lens = np.asarray(kv_lens, np.int64)
    q_lens = np.asarray(q_lens, np.int64)
    raw_cu = [0] + np.cumsum(q_lens).astype(int).tolist()
    raw_pos = []
    for kl, ql in zip(kv_lens, q_lens):
        raw_pos.extend(range(int(kl) - int(ql), int(kl)))
    npages = (kv_lens + PAGE - 1) // PAGE
    raw_tables = [[int(x) for x in row[:n]] for row, n in zip(np.asarray(block_tables), npages)]
    width = max(len(t) for t in raw_tables)
    padded = [t + [-1] * (width - len(t)) for t in raw_tables]
    cu_tiles, tile_seq = [0], []
    for s, ql in enumerate(q_lens):
        n = (int(ql) + q_tile - 1) // q_tile
        cu_tiles.append(cu_tiles[-1] + n)
        tile_seq += [s] * n
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=device)  # noqa: E731
    return VarlenAttnMetadata(
        positions=i32(raw_pos), raw_positions=raw_pos, cu_seqlens=i32(raw_cu), raw_cu_seqlens=raw_cu,
        max_q_len=int(q_lens.max()), Q_TILE_SIZE=q_tile, raw_cu_q_tiles=cu_tiles, cu_q_tiles=i32(cu_tiles),
        raw_q_tile_to_seq_idx=tile_seq, q_tile_to_seq_idx=i32(tile_seq), k_cache_pools=None, v_cache_pools=None,
        kv_lens=i32(kv_lens.tolist()), max_kv_len=int(kv_lens.max()), block_tables=i32(padded),
        raw_block_tables=raw_tables, is_decoding=bool((q_lens == 1).all()),
    )
