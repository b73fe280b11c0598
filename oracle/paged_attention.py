"""numpy restatement of the reference attention hot path (test infrastructure).

Every function cites the reference lines it restates (paths are relative to
the fishAndShrimp/nano-vllm-practice tree).  Layouts are the reference's:

* K/V pools: ``(num_blocks, n_kv_heads, block_size=16, d_head)``
  (``femtovllm/engine/core_engine.py:140-162``),
* q / out at the op boundary: head-major ``(n_heads, q_len_flatten, d_head)``
  (``femtovllm/ops/__init__.py:82-156``),
* block tables: int32 ``(B, max_blocks)`` padded with -1
  (``femtovllm/engine/model_runner.py:46-72``),
* new k / v: ``(T, n_kv_heads, d_head)`` as the projections emit them
  (``femtovllm/models/qwen/qwen3.py:231-232``).

Attention math (shared by every reference path): scale ``1/sqrt(D)``; GQA
``kv_head = q_head // n_rep`` (consecutive replication,
``qwen3.py:504-523``); key ``j`` is visible to query ``i`` iff
``j < kv_len[s]`` and ``j <= positions[i]`` (the right-bottom mask of
``qwen3.py:188-198`` stated on absolute positions, as the Triton kernel does at
``femtovllm/ops/triton/paged_attention/paged_attention_gemm.py:110-120``);
softmax in fp32 (or wider); output cast to the input dtype by the caller.
"""

from __future__ import annotations

import numpy as np

BLOCK_SIZE = 16  # kKVLenPerPage, csrc/utils/constants.cuh:75


# ---------------------------------------------------------------------------
# KV-cache write
# ---------------------------------------------------------------------------


def store_kvcache_decode_loop(k, v, k_pool, v_pool, raw_positions, raw_block_tables):
    """Decode KV write, restating ``qwen3.py:240-264`` literally.

    For each sequence b: ``blk = table[pos // P]``, ``off = pos % P`` and
    ``pool[blk, :, off] = new[b]`` (one token per sequence).  Mutates the pools.
    """
    block_size = k_pool.shape[2]
    for b in range(len(raw_block_tables)):
        pos = int(raw_positions[b])
        blk = raw_block_tables[b][pos // block_size]
        off = pos % block_size
        k_pool[blk, :, off] = k[b]
        v_pool[blk, :, off] = v[b]


def store_kvcache_prefill_loop(k, v, k_pool, v_pool, raw_positions, raw_cu_seqlens, raw_block_tables):
    """Prefill KV write, restating the block-run loop of ``qwen3.py:322-366``.

    Starts at table entry ``positions[q_begin] // P`` and writes runs of
    ``min(P - off, remaining)`` tokens per block until the sequence's new
    tokens are exhausted or a ``-1`` table entry is met.  Mutates the pools.
    """
    block_size = k_pool.shape[2]
    for b in range(len(raw_block_tables)):
        q_begin, q_end = int(raw_cu_seqlens[b]), int(raw_cu_seqlens[b + 1])
        table = raw_block_tables[b]
        off = int(raw_positions[q_begin])
        skip = off // block_size
        off %= block_size
        q_curr = q_begin
        for blk in table[skip:]:
            if blk < 0 or q_curr >= q_end:
                break
            n = min(block_size - off, q_end - q_curr)
            k_pool[blk, :, off : off + n] = np.swapaxes(k[q_curr : q_curr + n], 0, 1)
            v_pool[blk, :, off : off + n] = np.swapaxes(v[q_curr : q_curr + n], 0, 1)
            off += n
            q_curr += n
            off -= block_size


def build_slot_mapping(positions, seq_of_token, block_tables, block_size=BLOCK_SIZE):
    """Slot of every new token, from the same block-walk arithmetic.

    ``slot = table[s][pos // P] * P + pos % P`` is where ``qwen3.py:250-264``
    (decode) and ``qwen3.py:335-361`` (prefill) put token ``pos`` of sequence
    ``s``; a ``-1`` table entry gives slot ``-1`` (skip).  The reference has no
    ``slot_mapping`` tensor of its own; this is its index math, vectorised.
    """
    positions = np.asarray(positions, dtype=np.int64)
    seq_of_token = np.asarray(seq_of_token, dtype=np.int64)
    tables = np.asarray(block_tables, dtype=np.int64)
    blk = tables[seq_of_token, positions // block_size]
    slot = blk * block_size + positions % block_size
    slot[blk < 0] = -1
    return slot


def store_kvcache(k, v, k_pool, v_pool, slot_mapping):
    """Scatter ``k[t]``, ``v[t]`` (``(Hkv, D)`` each) to their slots; ``-1`` skips.

    Same destination as the reference loops above for the slots that
    ``build_slot_mapping`` produces.  Mutates the pools; bytes are copied
    unchanged (the check on this is bit-exact).
    """
    slot_mapping = np.asarray(slot_mapping, dtype=np.int64)
    block_size = k_pool.shape[2]
    live = np.nonzero(slot_mapping >= 0)[0]
    blk = slot_mapping[live] // block_size
    off = slot_mapping[live] % block_size
    k_pool[blk, :, off] = k[live]
    v_pool[blk, :, off] = v[live]


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------


def gather_seq_kv(pool, table, kv_len):
    """Pages of one sequence, concatenated: ``(Hkv, kv_len, D)``.

    Restates the page gather of ``qwen3.py:450-497`` (whole blocks, then the
    partial last block) and of the reference tests'
    ``torch.cat([pool[x] for x in table], -2)[:, :kv_len]``
    (``femtovllm/ops/triton/paged_attention/test_paged_attention_gemm.py:148-160``).
    """
    n_pages = (int(kv_len) + pool.shape[2] - 1) // pool.shape[2]
    pages = [int(x) for x in table[:n_pages]]
    if any(p < 0 for p in pages):
        raise ValueError("block table has a -1 entry inside kv_len")
    kv = np.concatenate([pool[p] for p in pages], axis=1)
    return kv[:, : int(kv_len)]


def _attend(q, k, v, visible, acc_dtype):
    """softmax(q k^T / sqrt(D), masked) v for one kv head group.

    q: (n_rep, T, D); k, v: (L, D); visible: (T, L) bool.
    """
    d = q.shape[-1]
    qf = q.astype(acc_dtype)
    s = np.matmul(qf, k.astype(acc_dtype).T) * acc_dtype(1.0 / np.sqrt(d))
    s = np.where(visible[None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.matmul(p, v.astype(acc_dtype))


def decode_attention(q, k_pool, v_pool, block_tables, kv_lens, acc_dtype=np.float64):
    """Decode paged attention: one query token per sequence.

    q: ``(Hq, B, D)``; returns ``(Hq, B, D)`` in ``acc_dtype``.  Restates the
    reference methodology of ``csrc/paged_attention/test_paged_attention_gemv.py:58-89``
    (SDPA over the gathered pages, ``enable_gqa``) with the GQA mapping of
    ``qwen3.py:504-523``; the query sees keys ``0 .. kv_len-1``
    (``model_runner.py:283-291``: ``kv_len = pos + 1``).
    """
    hq, batch, d = q.shape
    hkv = k_pool.shape[1]
    n_rep = hq // hkv
    out = np.empty((hq, batch, d), dtype=acc_dtype)
    for b in range(batch):
        kv_len = int(kv_lens[b])
        ks = gather_seq_kv(k_pool, block_tables[b], kv_len)
        vs = gather_seq_kv(v_pool, block_tables[b], kv_len)
        visible = np.ones((1, kv_len), dtype=bool)
        for g in range(hkv):
            qs = q[g * n_rep : (g + 1) * n_rep, b : b + 1]
            out[g * n_rep : (g + 1) * n_rep, b : b + 1] = _attend(qs, ks[g], vs[g], visible, acc_dtype)
    return out


def prefill_attention(q, k_pool, v_pool, cu_seqlens, block_tables, kv_lens, positions, acc_dtype=np.float64):
    """Varlen chunked-prefill causal attention over paged KV.

    q: ``(Hq, T, D)`` with sequence s owning tokens
    ``cu_seqlens[s] .. cu_seqlens[s+1]-1``; returns ``(Hq, T, D)``.
    Restates ``qwen3.py:430-542`` (per-sequence gather, consecutive GQA
    replication, SDPA with the right-bottom mask) with the mask stated on
    absolute positions as the kernels do (``paged_attention_gemm.py:110-120``;
    ``csrc/paged_attention/paged_attention_gemm.cu:181-184``).  Decode rows are
    just sequences with one new token, so this also covers the unified
    mixed-batch launch (``qwen3.py:575-581``).
    """
    hq, _, d = q.shape
    hkv = k_pool.shape[1]
    n_rep = hq // hkv
    out = np.zeros(q.shape, dtype=acc_dtype)
    for s in range(len(cu_seqlens) - 1):
        q0, q1 = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        if q1 == q0:
            continue
        kv_len = int(kv_lens[s])
        ks = gather_seq_kv(k_pool, block_tables[s], kv_len)
        vs = gather_seq_kv(v_pool, block_tables[s], kv_len)
        pos = np.asarray(positions[q0:q1], dtype=np.int64)
        visible = np.arange(kv_len)[None, :] <= pos[:, None]
        for g in range(hkv):
            qs = q[g * n_rep : (g + 1) * n_rep, q0:q1]
            out[g * n_rep : (g + 1) * n_rep, q0:q1] = _attend(qs, ks[g], vs[g], visible, acc_dtype)
    return out
