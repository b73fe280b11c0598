"""numpy restatement of the stage between the q/k/v projections and the
attention op (test infrastructure).

In ``QwenSelfAttention.forward_varlen_custom_gemv`` / ``_gemm``
(``femtovllm/models/qwen/qwen3.py:228-264``, ``:308-366``) the reference
runs, per layer:

* ``q = q_norm(q); k = k_norm(k)`` -- ``nn.RMSNorm(d_head, eps)``
  (``qwen3.py:181-183``): ``x / sqrt(mean(x^2) + eps) * weight`` over ``d_head``;
* ``q = rotary_embd(q, positions); k = rotary_embd(k, positions)`` --
  ``QwenRotaryEmbedding`` (``qwen3.py:17-138``), varlen route:
  ``cos[pos] * x + sin[pos] * cat(-x2, x1)`` with ``x1, x2`` the two halves of
  ``d_head`` and ``cos``/``sin`` the module's ``(max_seqlen, d_head)`` buffers
  (``qwen3.py:36-49``, base ``1e6``);
* the KV-write loop (k after norm + rope, v as projected);
* ``q.transpose(0, 1)`` into the attention op (head-major).

Pinned against ``tests/golden/norm_rope_*.npz``, which record what the
reference's own modules produce (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np

from oracle.paged_attention import store_kvcache


def rope_tables(max_seqlen: int, d_head: int, base: float = 1000000.0):
    """``(cos, sin)``, each ``(max_seqlen, d_head)`` float32, as ``QwenRotaryEmbedding.__init__``
    builds its buffers (``qwen3.py:30-49``): ``inv_freq[i] = (1/base) ** (2 i / d_head)``,
    ``theta = pos * inv_freq`` duplicated over both halves."""
    if d_head % 2:
        raise ValueError(f"d_head must be even, now {d_head=}")
    i = np.arange(d_head // 2, dtype=np.float32)
    inv_freq = np.float32(1.0 / base) ** (np.float32(2) * i / np.float32(d_head))
    theta = np.arange(max_seqlen, dtype=np.float32)[:, None] * inv_freq[None, :].astype(np.float32)
    theta = np.concatenate([theta, theta], axis=-1)
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


def rms_norm(x, weight, eps):
    """``nn.RMSNorm`` over the last axis (``qwen3.py:181-183``), in float64."""
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(weight, np.float64)


def apply_rope(x, cos, sin, positions):
    """``QwenRotaryEmbedding.forward`` varlen route (``qwen3.py:103-138``): ``x`` is
    ``(T, H, D)``, ``positions`` ``(T,)`` absolute indices into the tables."""
    x = np.asarray(x, np.float64)
    c = np.asarray(cos, np.float64)[positions][:, None, :]
    s = np.asarray(sin, np.float64)[positions][:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return c * x + s * rot


def qk_norm_rope_store(q, k, v, q_norm_weight, k_norm_weight, eps, cos, sin, positions, k_pool, v_pool,
                       slot_mapping):
    """The whole stage.  ``q`` ``(T, Hq, D)``, ``k``/``v`` ``(T, Hkv, D)``.  Writes k (normed,
    rotated, cast to the pool dtype) and v into the pools at ``slot_mapping`` (``-1`` skips)
    and returns q normed and rotated, head-major ``(Hq, T, D)`` float64."""
    positions = np.asarray(positions, np.int64)
    qn = apply_rope(rms_norm(q, q_norm_weight, eps), cos, sin, positions)
    kn = apply_rope(rms_norm(k, k_norm_weight, eps), cos, sin, positions)
    store_kvcache(kn.astype(k_pool.dtype), np.asarray(v).astype(v_pool.dtype), k_pool, v_pool, slot_mapping)
    return np.ascontiguousarray(qn.transpose(1, 0, 2))
