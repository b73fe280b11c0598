"""fp32 restatement of the reference's varlen paged attention, run with torch on the device.

Test infrastructure only.  It restates the attention part of
``QwenSelfAttention.forward_varlen_pytorch`` (femtovllm/models/qwen/qwen3.py:430-542):
gather each sequence's pages from the pool (partial last page, ``qwen3.py:450-497``),
replicate every kv head over its ``n_rep`` query heads (``qwen3.py:504-523``; done here
by grouping the query heads instead of copying K/V), and a softmax over keys
``j < kv_len`` with ``j <= positions[i]`` (``qwen3.py:188-198, 527-535``), all in fp32.

It exists so that the full-size configurations can be checked on every output row in
seconds; ``tests/test_gpu_parity.py`` pins it against the numpy oracle (``oracle/``)
on sampled sequences before trusting it on the rest.
"""

from __future__ import annotations

import contextlib

import torch

PAGE = 16


@contextlib.contextmanager
def exact_fp32_matmul():
    """fp32 matmuls without TF32 inputs (restored on exit)."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def _gather(pool: torch.Tensor, table_row: torch.Tensor, kv_len: int) -> torch.Tensor:
    """(Hkv, kv_len, D) fp32 view of one sequence's keys (or values)."""
    npg = (kv_len + PAGE - 1) // PAGE
    pages = table_row[:npg].long()
    x = pool.index_select(0, pages).float()  # (npg, Hkv, 16, D)
    hkv, d = x.shape[1], x.shape[3]
    return x.permute(1, 0, 2, 3).reshape(hkv, npg * PAGE, d)[:, :kv_len]


@torch.no_grad()
def paged_attention_fp32(q, k_pool, v_pool, cu_seqlens, block_tables, kv_lens, positions=None,
                         q_chunk: int = 256) -> torch.Tensor:
    """out (Hq, T, D) fp32 for q (Hq, T, D) over paged K/V.

    ``cu_seqlens`` / ``positions`` None = decode: token s is sequence s's query at
    position ``kv_lens[s] - 1``.
    """
    hq, t, d = q.shape
    hkv = k_pool.shape[1]
    n_rep = hq // hkv
    dev = q.device
    lens = [int(x) for x in kv_lens.tolist()]
    b = len(lens)
    cu = list(range(b + 1)) if cu_seqlens is None else [int(x) for x in cu_seqlens.tolist()]
    if positions is None:
        positions = (kv_lens.to(dev).long() - 1)
    out = torch.empty(hq, t, d, dtype=torch.float32, device=dev)
    scale = d ** -0.5
    with exact_fp32_matmul():
        for s in range(b):
            q0, q1, L = cu[s], cu[s + 1], lens[s]
            if q1 == q0:
                continue
            k = _gather(k_pool, block_tables[s], L)  # (Hkv, L, D)
            v = _gather(v_pool, block_tables[s], L)
            keys = torch.arange(L, device=dev)
            for a in range(q0, q1, q_chunk):
                e = min(a + q_chunk, q1)
                c = e - a
                qg = q[:, a:e].float().reshape(hkv, n_rep * c, d)  # heads of a group are consecutive
                sc = torch.bmm(qg, k.transpose(1, 2)).mul_(scale).view(hkv, n_rep, c, L)
                vis = keys[None, :] <= positions[a:e].to(dev).long()[:, None]  # (c, L)
                sc.masked_fill_(~vis, float("-inf"))
                p = torch.softmax(sc, dim=-1).view(hkv, n_rep * c, L)
                out[:, a:e] = torch.bmm(p, v).view(hq, c, d)
    return out
