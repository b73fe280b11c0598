"""Seeded synthetic inputs with the shapes of the five benchmark configurations.

No dataset is involved: every configuration is a synthetic paged-KV batch.
Lengths and block tables are drawn on the host with numpy (seeded);
Q / K / V contents are drawn on the target device with a seeded torch
generator, so full-size pools never cross PCIe.

Conventions (the reference engine's, ``femtovllm/engine/model_runner.py:159-339``):

* a decode sequence's new token sits at ``position = kv_len - 1``; a prefill
  chunk of ``c`` tokens covers ``positions = kv_len - c .. kv_len - 1``;
* ``block_tables`` are int32, ``-1`` padded, with physical blocks drawn
  without replacement from a shuffled pool (non-contiguous);
* ``slot_mapping[t] = table[s][pos // 16] * 16 + pos % 16`` for every new token.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch

PAGE = 16


@dataclasses.dataclass
class PagedBatch:
    name: str
    n_heads: int
    n_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    num_blocks: int
    kv_lens: np.ndarray  # int32 [B]
    q_lens: np.ndarray  # int32 [B]  (1 for decode sequences)
    block_tables: np.ndarray  # int32 [B, max_blocks], -1 padded
    seed: int
    qkv_scale: float = 1.0
    shared_prefix_blocks: int = 0
    # device tensors (filled by materialize)
    q: Optional[torch.Tensor] = None  # (Hq, T, D)
    k_new: Optional[torch.Tensor] = None  # (T, Hkv, D)
    v_new: Optional[torch.Tensor] = None
    k_pool: Optional[torch.Tensor] = None  # (num_blocks, Hkv, 16, D)
    v_pool: Optional[torch.Tensor] = None

    # ---- derived host metadata ----
    @property
    def num_seqs(self) -> int:
        return len(self.kv_lens)

    @property
    def cu_seqlens(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.q_lens)]).astype(np.int32)

    @property
    def num_tokens(self) -> int:
        return int(self.q_lens.sum())

    @property
    def positions(self) -> np.ndarray:
        return np.concatenate(
            [np.arange(kl - ql, kl, dtype=np.int32) for kl, ql in zip(self.kv_lens, self.q_lens)]
        ).astype(np.int32)

    @property
    def seq_of_token(self) -> np.ndarray:
        return np.repeat(np.arange(self.num_seqs), self.q_lens).astype(np.int64)

    @property
    def slot_mapping(self) -> np.ndarray:
        pos = self.positions.astype(np.int64)
        blk = self.block_tables[self.seq_of_token, pos // PAGE].astype(np.int64)
        return blk * PAGE + pos % PAGE

    @property
    def max_kv_len(self) -> int:
        return int(self.kv_lens.max())

    @property
    def max_q_len(self) -> int:
        return int(self.q_lens.max())

    @property
    def is_decode(self) -> bool:
        return bool((self.q_lens == 1).all())

    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes one attention launch must read (each kv head once)."""
        es = torch.finfo(self.dtype).bits // 8
        return int(2 * self.kv_lens.astype(np.int64).sum() * self.n_kv_heads * self.head_dim * es)

    def unique_kv_bytes(self) -> int:
        """K+V bytes of the distinct pages the launch attends over (a page shared by several
        requests' tables, as a common prefix, counted once)."""
        es = torch.finfo(self.dtype).bits // 8
        npages = (self.kv_lens.astype(np.int64) + PAGE - 1) // PAGE
        pages = np.concatenate([self.block_tables[s, : int(n)] for s, n in enumerate(npages)])
        return int(2 * np.unique(pages).size * PAGE * self.n_kv_heads * self.head_dim * es)

    def decode_bytes(self) -> int:
        """Algorithmic HBM bytes of one decode launch: K+V, q, out, block tables, kv_lens."""
        es = torch.finfo(self.dtype).bits // 8
        qo = 2 * self.num_seqs * self.n_heads * self.head_dim * es
        tables = 4 * int(((self.kv_lens + PAGE - 1) // PAGE).sum()) + 4 * self.num_seqs
        return self.kv_bytes() + qo + tables

    def store_bytes(self) -> int:
        """Algorithmic bytes of one store_kvcache launch: rows read + written, plus slots."""
        es = torch.finfo(self.dtype).bits // 8
        return 2 * 2 * self.num_tokens * self.n_kv_heads * self.head_dim * es + 8 * self.num_tokens

    def attn_flops(self) -> float:
        """Algorithmic FLOPs over visible (query, key) pairs: 4 * D * Hq * pairs."""
        pairs = 0
        for kl, ql in zip(self.kv_lens.astype(np.int64), self.q_lens.astype(np.int64)):
            p = kl - ql
            pairs += ql * p + ql * (ql + 1) // 2
        return 4.0 * self.head_dim * self.n_heads * pairs

    # ---- device data ----
    def materialize(self, device, k_pool_fill: bool = True) -> "PagedBatch":
        """Draw q, the new k/v rows and both pools on `device` (seeded)."""
        g = torch.Generator(device=device)
        g.manual_seed(self.seed)
        T, Hq, Hkv, D = self.num_tokens, self.n_heads, self.n_kv_heads, self.head_dim
        s = self.qkv_scale

        def rnd(shape):
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32 if self.dtype == torch.float32 else self.dtype)
            if s != 1.0:
                t.mul_(s)
            return t.to(self.dtype)

        self.q = rnd((Hq, T, D))
        self.k_new = rnd((T, Hkv, D))
        self.v_new = rnd((T, Hkv, D))
        shape = (self.num_blocks, Hkv, PAGE, D)
        if k_pool_fill:
            self.k_pool = rnd(shape)
            self.v_pool = rnd(shape)
        else:
            self.k_pool = torch.empty(shape, device=device, dtype=self.dtype)
            self.v_pool = torch.empty(shape, device=device, dtype=self.dtype)
        return self

    def device_metadata(self, device) -> dict:
        return {
            "block_tables": torch.from_numpy(self.block_tables).to(device),
            "kv_lens": torch.from_numpy(self.kv_lens).to(device),
            "cu_seqlens": torch.from_numpy(self.cu_seqlens).to(device),
            "positions": torch.from_numpy(self.positions).to(device),
            "slot_mapping": torch.from_numpy(self.slot_mapping).to(device),
        }


def _tables(rng, kv_lens, num_blocks, shared_prefix=None):
    """Disjoint random block tables (plus an optional shared head), -1 padded."""
    nblk = (kv_lens + PAGE - 1) // PAGE
    perm = rng.permutation(num_blocks).astype(np.int32)
    head = np.zeros(0, dtype=np.int32) if shared_prefix is None else shared_prefix
    rows, at = [], 0
    for n in nblk:
        own = int(n) - len(head)
        rows.append(np.concatenate([head, perm[at : at + own]]))
        at += own
    if at > num_blocks:
        raise ValueError("pool too small")
    width = int(nblk.max())
    out = np.full((len(kv_lens), width), -1, dtype=np.int32)
    for i, r in enumerate(rows):
        out[i, : len(r)] = r
    return out


def _pool_blocks(kv_lens, factor=1.2, extra=0):
    return int(np.ceil(factor * ((kv_lens + PAGE - 1) // PAGE).sum())) + extra


def config1(seed: int = 1) -> PagedBatch:
    """CPU-runnable decode, fp32: B=4, Hq=8, Hkv=2, D=64, context U[1,256], pool 128.

    The context of L tokens is cached; the new token is written at position L
    (slot from the table), so attention runs over kv_len = L + 1.
    """
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 257, size=4)
    kv_lens = (ctx + 1).astype(np.int32)
    tables = _tables(rng, kv_lens, 128)
    return PagedBatch("config1_decode_fp32", 8, 2, 64, torch.float32, 128, kv_lens, np.ones(4, np.int32), tables, seed)


def config2(seed: int = 2, num_seqs: int = 256) -> PagedBatch:
    """Decode, bf16: B=256, Hq=16, Hkv=8, D=128, kv_len U[512,4096], pool 1.2x."""
    rng = np.random.default_rng(seed)
    kv_lens = rng.integers(512, 4097, size=num_seqs).astype(np.int32)
    nb = _pool_blocks(kv_lens)
    tables = _tables(rng, kv_lens, nb)
    return PagedBatch(
        "config2_decode_bf16", 16, 8, 128, torch.bfloat16, nb, kv_lens, np.ones(num_seqs, np.int32), tables, seed,
        qkv_scale=1.0 / np.sqrt(128.0),
    )


def config3(seed: int = 3, num_seqs: int = 64) -> PagedBatch:
    """Varlen chunked prefill, bf16, causal: 64 seqs, Hq=16, Hkv=8, D=128,
    chunk U[128,2048], cached prefix U[0,8192]."""
    rng = np.random.default_rng(seed)
    c = rng.integers(128, 2049, size=num_seqs)
    p = rng.integers(0, 8193, size=num_seqs)
    kv_lens = (p + c).astype(np.int32)
    nb = _pool_blocks(kv_lens)
    tables = _tables(rng, kv_lens, nb)
    return PagedBatch("config3_prefill_bf16", 16, 8, 128, torch.bfloat16, nb, kv_lens, c.astype(np.int32), tables, seed)


def config4(seed: int = 4) -> PagedBatch:
    """Unified mixed batch with prefix sharing, bf16: 32 requests sharing one
    4096-token prefix (256 shared blocks), private suffix U[64,1024] (cached);
    24 decode (1 new token) and 8 prefill (512-token chunks) in one launch;
    Hq=32, Hkv=8, D=128."""
    rng = np.random.default_rng(seed)
    n = 32
    suffix = rng.integers(64, 1025, size=n)
    is_prefill = np.zeros(n, dtype=bool)
    is_prefill[rng.permutation(n)[:8]] = True
    q_lens = np.where(is_prefill, 512, 1).astype(np.int32)
    kv_lens = (4096 + suffix + q_lens).astype(np.int32)
    private = ((kv_lens - 4096 + PAGE - 1) // PAGE).sum()
    nb = 256 + int(np.ceil(1.2 * private))
    perm = rng.permutation(nb).astype(np.int32)
    shared = perm[:256]
    rest_rng = np.random.default_rng(seed + 1000)
    tables = np.full((n, int(((kv_lens + PAGE - 1) // PAGE).max())), -1, dtype=np.int32)
    at = 256
    for i in range(n):
        own = int((kv_lens[i] + PAGE - 1) // PAGE) - 256
        tables[i, :256] = shared
        tables[i, 256 : 256 + own] = perm[at : at + own]
        at += own
    del rest_rng
    return PagedBatch(
        "config4_mixed_bf16", 32, 8, 128, torch.bfloat16, nb, kv_lens, q_lens, tables, seed, shared_prefix_blocks=256
    )


def config5_lengths(seed: int = 5, total: int = 64) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(32768, 131073, size=total).astype(np.int32)


def shard_lpt(lengths: np.ndarray, world: int) -> list[np.ndarray]:
    """Longest-processing-time partition of sequences over ranks (indices per rank)."""
    order = np.argsort(-lengths, kind="stable")
    load = np.zeros(world, dtype=np.int64)
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = int(np.argmin(load))
        parts[r].append(int(i))
        load[r] += int(lengths[i])
    return [np.array(sorted(p), dtype=np.int64) for p in parts]


def config5(seed: int = 5, rank: int = 0, world: int = 1, total: int = 64) -> PagedBatch:
    """Long-context decode sharded by request: total B=64, Hq=32, Hkv=8, D=128,
    kv_len U[32768,131072]; this rank's LPT shard with its own pool (1.2x)."""
    lengths = config5_lengths(seed, total)
    mine = shard_lpt(lengths, world)[rank]
    kv_lens = lengths[mine]
    rng = np.random.default_rng(seed * 1000 + rank)
    nb = _pool_blocks(kv_lens)
    tables = _tables(rng, kv_lens, nb)
    return PagedBatch(
        f"config5_long_decode_bf16_r{rank}of{world}", 32, 8, 128, torch.bfloat16, nb, kv_lens,
        np.ones(len(kv_lens), np.int32), tables, seed * 1000 + rank,
    )


def custom(
    kv_lens, q_lens, n_heads, n_kv_heads, head_dim, dtype, seed=0, pool_factor=1.5, extra_blocks=3, qkv_scale=1.0
) -> PagedBatch:
    """Arbitrary small batch for parity tests (random non-contiguous tables)."""
    rng = np.random.default_rng(seed)
    kv_lens = np.asarray(kv_lens, dtype=np.int32)
    q_lens = np.asarray(q_lens, dtype=np.int32)
    nb = _pool_blocks(kv_lens, pool_factor, extra_blocks)
    tables = _tables(rng, kv_lens, nb)
    return PagedBatch("custom", n_heads, n_kv_heads, head_dim, dtype, nb, kv_lens, q_lens, tables, seed,
                      qkv_scale=qkv_scale)


def subset_for_oracle(batch: PagedBatch, seqs) -> dict:
    """numpy copy (float32) of the pages and queries of `seqs`, renumbered.

    Lets the CPU oracle check a sample of a full-size GPU batch without
    copying the whole pool back.
    """
    seqs = [int(s) for s in seqs]
    cu = batch.cu_seqlens
    tok = np.concatenate([np.arange(cu[s], cu[s + 1]) for s in seqs])
    npages = [(int(batch.kv_lens[s]) + PAGE - 1) // PAGE for s in seqs]
    blocks = np.concatenate([batch.block_tables[s, :n] for s, n in zip(seqs, npages)]).astype(np.int64)
    uniq, inv = np.unique(blocks, return_inverse=True)
    idx = torch.from_numpy(uniq).to(batch.k_pool.device)
    kp = batch.k_pool.index_select(0, idx).float().cpu().numpy()
    vp = batch.v_pool.index_select(0, idx).float().cpu().numpy()
    tables = np.full((len(seqs), max(npages)), -1, dtype=np.int32)
    at = 0
    for i, n in enumerate(npages):
        tables[i, :n] = inv[at : at + n]
        at += n
    q = batch.q.index_select(1, torch.from_numpy(tok).to(batch.q.device)).float().cpu().numpy()
    q_lens = batch.q_lens[seqs]
    return {
        "q": q,
        "k_pool": kp,
        "v_pool": vp,
        "block_tables": tables,
        "kv_lens": batch.kv_lens[seqs].copy(),
        "cu_seqlens": np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32),
        "positions": batch.positions[tok],
        "tokens": tok,
    }
