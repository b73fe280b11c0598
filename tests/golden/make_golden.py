"""Generate the golden fixtures in this directory from the reference itself.

Usage (needs the fishAndShrimp/nano-vllm-practice source tree, CPU only):

    python tests/golden/make_golden.py --reference <path to the reference tree>

The reference package imports on CPU once ``femtovllm._C`` is a stub module
carrying its three constants (kMaxKVLenNonSplit, kKVLenPerPage, kDimHead;
``csrc/bindings.cpp:62-66``), since ``femtovllm/ops/__init__.py:6-26`` is its
only hard dependency on the native module.  For every case this script
builds a ``QwenSelfAttention`` (``femtovllm/models/qwen/qwen3.py:141``) whose
projections slice a packed input ``x = [q | k | v]``, whose q/k norms, RoPE
and o_proj are identities, and runs:

* ``forward_varlen_pytorch`` (``qwen3.py:389-544``): the reference KV write
  plus per-sequence page gather, GQA replication and SDPA with the
  right-bottom mask -> ``out`` and the pools after the write;
* the KV-write loop of ``forward_varlen_custom_gemv`` (decode,
  ``qwen3.py:240-264``) or ``forward_varlen_custom_gemm`` (prefill,
  ``qwen3.py:322-366``), with the attention op replaced by a stub -> the pools
  after that loop.

The ``norm_rope_*`` fixtures instead keep the reference's q_norm / k_norm
(``nn.RMSNorm``, ``qwen3.py:181-183``, with seeded weights) and its
``QwenRotaryEmbedding`` (``qwen3.py:17-138``), and record the q that
``forward_varlen_custom_gemm`` / ``_gemv`` hand to the attention op plus the
pool rows their write loops produce: the stage that ``qk_norm_rope_store``
fuses.

``metadata_routes.npz`` records the VarlenAttnMetadata that the reference's own
``ModelRunner._route_prefill`` / ``_route_decode`` (``model_runner.py:159-339``)
build from scheduled sequences, for ``build_varlen_metadata``.

``sampler.npz`` records the reference's ``Sampler`` (``femtovllm/engine/sampler.py``)
run on stand-in sequences: the ids of greedy rows and the token counts of many draws
of sampled rows, for ``sample_tokens``.

All inputs are bf16-representable (stored as bf16 bits) so one fixture serves
both the fp32 and the bf16 checks; the reference runs in fp32.  Each fixture
stores the pools before the write and only the rows the reference changed.
"""

from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
PAGE = 16


def _import_reference(ref: Path):
    stub = types.ModuleType("femtovllm._C")
    stub.kMaxKVLenNonSplit = 8192
    stub.kKVLenPerPage = 16
    stub.kDimHead = 128
    sys.modules["femtovllm._C"] = stub
    sys.path.insert(0, str(ref))
    import femtovllm  # noqa: F401
    import femtovllm.ops
    from femtovllm.models.qwen.qwen3 import QwenSelfAttention
    from femtovllm.protocol import VarlenAttnMetadata

    return femtovllm, QwenSelfAttention, VarlenAttnMetadata


class _Slice(torch.nn.Module):
    def __init__(self, a, b):
        super().__init__()
        self.a, self.b = a, b

    def forward(self, x):
        return x[:, self.a : self.b]


class _NoRope(torch.nn.Module):
    def forward(self, x, positions=None):
        return x


def _bf16_vals(gen, shape, scale=1.0):
    return (torch.randn(shape, generator=gen) * scale).to(torch.bfloat16).to(torch.float32)


def _make_case(name, kv_lens, q_lens, Hq, Hkv, D, num_blocks, tables, seed, scale=1.0):
    kv_lens = np.asarray(kv_lens, np.int32)
    q_lens = np.asarray(q_lens, np.int32)
    gen = torch.Generator().manual_seed(seed)
    T = int(q_lens.sum())
    return {
        "name": name,
        "Hq": Hq,
        "Hkv": Hkv,
        "D": D,
        "kv_lens": kv_lens,
        "q_lens": q_lens,
        "tables": tables,
        "num_blocks": num_blocks,
        "q": _bf16_vals(gen, (Hq, T, D), scale),
        "k_new": _bf16_vals(gen, (T, Hkv, D), scale),
        "v_new": _bf16_vals(gen, (T, Hkv, D), scale),
        "k_pool": _bf16_vals(gen, (num_blocks, Hkv, PAGE, D), scale),
        "v_pool": _bf16_vals(gen, (num_blocks, Hkv, PAGE, D), scale),
    }


def _random_tables(rng, kv_lens, num_blocks, shared=None):
    perm = list(rng.permutation(num_blocks))
    head = [] if shared is None else list(shared)
    perm = [b for b in perm if b not in set(head)]
    rows = []
    for kl in kv_lens:
        n = (int(kl) + PAGE - 1) // PAGE - len(head)
        rows.append(head + [int(x) for x in perm[:n]])
        perm = perm[n:]
    return rows


def cases():
    out = []
    # 1. BASELINE config 1 shape: decode, B=4, Hq=8, Hkv=2, D=64, context U[1,256] + 1 new token, pool 128.
    rng = np.random.default_rng(1)
    ctx = rng.integers(1, 257, size=4)
    kv = ctx + 1
    tables = _random_tables(rng, kv, 128)
    out.append(_make_case("cfg1_decode", kv, [1] * 4, 8, 2, 64, 128, tables, 11))
    # 2. Reference GEMV test structure (csrc/paged_attention/test_paged_attention_gemv.py:22-50) at page 16:
    #    tables [[0,4,5,6],[1,8,9]], kv_lens [59,44], Hq 8 / Hkv 4, D 128.
    out.append(_make_case("toy_decode", [59, 44], [1, 1], 8, 4, 128, 10, [[0, 4, 5, 6], [1, 8, 9]], 12))
    # 3. Reference Triton prefill test structure (ops/triton/paged_attention/test_paged_attention_gemm.py:18-102):
    #    cu_seqlens [0,8,24], kv_lens [59,44], same tables.
    out.append(_make_case("toy_prefill", [59, 44], [8, 16], 8, 4, 128, 10, [[0, 4, 5, 6], [1, 8, 9]], 13))
    # 4. Chunked prefill over cached prefixes, page-boundary edges, GQA 2.
    rng = np.random.default_rng(4)
    c = np.array([1, 17, 33, 64, 100])
    p = np.array([0, 15, 16, 47, 200])
    tables = _random_tables(rng, p + c, 40)
    out.append(_make_case("chunked_prefix_gqa2", p + c, c, 4, 2, 128, 40, tables, 14))
    # 5. Mixed decode + prefill sharing a 32-token (2-block) prefix, GQA 4.
    rng = np.random.default_rng(5)
    q_lens = np.array([1, 20, 1, 1, 37, 1])
    suffix = np.array([5, 0, 16, 31, 3, 60])
    kv = 32 + suffix + q_lens
    tables = _random_tables(rng, kv, 24, shared=[7, 3])
    out.append(_make_case("mixed_shared_prefix_gqa4", kv, q_lens, 8, 2, 128, 24, tables, 15))
    # 6. GQA 8, D 64, ragged chunks incl. a 1-token prefill row.
    rng = np.random.default_rng(6)
    c = np.array([5, 40, 1])
    p = np.array([10, 0, 70])
    tables = _random_tables(rng, p + c, 12)
    out.append(_make_case("gqa8_d64", p + c, c, 8, 1, 64, 12, tables, 16))
    # 7. MHA (GQA 1), D 64, decode with kv_len 1 and exact page multiples.
    rng = np.random.default_rng(7)
    kv = np.array([1, 16, 32, 17])
    tables = _random_tables(rng, kv, 8)
    out.append(_make_case("mha_d64_decode_edges", kv, [1] * 4, 4, 4, 64, 8, tables, 17))
    return out


def _varlen_metadata(kv_lens, q_lens, tables, VarlenAttnMetadata):
    """The reference's VarlenAttnMetadata (femtovllm/protocol.py:58-81) for one batch."""
    raw_cu = [0] + np.cumsum(q_lens).tolist()
    raw_pos = []
    for kl, ql in zip(kv_lens, q_lens):
        raw_pos.extend(range(int(kl) - int(ql), int(kl)))
    raw_tables = [list(map(int, t)) for t in tables]
    width = max(len(t) for t in raw_tables)
    padded = [t + [-1] * (width - len(t)) for t in raw_tables]
    is_decoding = bool((q_lens == 1).all())
    Q_TILE = 32
    cu_tiles, tile_seq = [0], []
    for s, ql in enumerate(q_lens):
        n = (int(ql) + Q_TILE - 1) // Q_TILE
        cu_tiles.append(cu_tiles[-1] + n)
        tile_seq += [s] * n
    md = VarlenAttnMetadata(
        positions=torch.tensor(raw_pos, dtype=torch.int32),
        raw_positions=raw_pos,
        cu_seqlens=torch.tensor(raw_cu, dtype=torch.int32),
        raw_cu_seqlens=raw_cu,
        max_q_len=int(q_lens.max()),
        Q_TILE_SIZE=Q_TILE,
        raw_cu_q_tiles=cu_tiles,
        cu_q_tiles=torch.tensor(cu_tiles, dtype=torch.int32),
        raw_q_tile_to_seq_idx=tile_seq,
        q_tile_to_seq_idx=torch.tensor(tile_seq, dtype=torch.int32),
        k_cache_pools=None,
        v_cache_pools=None,
        kv_lens=torch.tensor(kv_lens, dtype=torch.int32),
        max_kv_len=int(kv_lens.max()),
        block_tables=torch.tensor(padded, dtype=torch.int32),
        raw_block_tables=raw_tables,
        is_decoding=is_decoding,
    )
    return md, padded, raw_cu, raw_pos, is_decoding


def run_reference(case, femtovllm, QwenSelfAttention, VarlenAttnMetadata):
    Hq, Hkv, D = case["Hq"], case["Hkv"], case["D"]
    kv_lens, q_lens = case["kv_lens"], case["q_lens"]
    T = int(q_lens.sum())
    md, padded, raw_cu, raw_pos, is_decoding = _varlen_metadata(kv_lens, q_lens, case["tables"], VarlenAttnMetadata)

    cfg = types.SimpleNamespace(head_dim=D, rms_norm_eps=1e-6)
    d_model = D * (Hq + 2 * Hkv)
    attn = QwenSelfAttention(d_model, Hq, Hkv, max_seqlen=4, dropout_p=0.0, config=cfg)
    attn.w_q = _Slice(0, Hq * D)
    attn.w_k = _Slice(Hq * D, (Hq + Hkv) * D)
    attn.w_v = _Slice((Hq + Hkv) * D, (Hq + 2 * Hkv) * D)
    attn.q_norm = torch.nn.Identity()
    attn.k_norm = torch.nn.Identity()
    attn.rotary_embd = _NoRope()
    attn.o_proj = torch.nn.Identity()
    attn.eval()

    q_tok = case["q"].transpose(0, 1).reshape(T, Hq * D)
    x = torch.cat([q_tok, case["k_new"].reshape(T, Hkv * D), case["v_new"].reshape(T, Hkv * D)], dim=1)
    kp, vp = case["k_pool"].clone(), case["v_pool"].clone()
    with torch.no_grad():
        o, _ = attn.forward_varlen_pytorch(x, kp, vp, md)
    out = o.reshape(T, Hq, D).transpose(0, 1).contiguous()

    # The custom-kernel routes' own KV-write loops, with the attention op stubbed out.
    kp2, vp2 = case["k_pool"].clone(), case["v_pool"].clone()
    stub = lambda q, **kw: torch.zeros_like(q)  # noqa: E731
    saved = (femtovllm.ops.paged_attention_gemv, femtovllm.ops.paged_attention_gemm)
    femtovllm.ops.paged_attention_gemv = stub
    femtovllm.ops.paged_attention_gemm = stub
    try:
        with torch.no_grad():
            if is_decoding:
                attn.forward_varlen_custom_gemv(x, kp2, vp2, md)
            else:
                attn.forward_varlen_custom_gemm(x, kp2, vp2, md)
    finally:
        femtovllm.ops.paged_attention_gemv, femtovllm.ops.paged_attention_gemm = saved
    return out, (kp, vp), (kp2, vp2), padded, raw_cu, raw_pos


def norm_rope_cases():
    """Cases for the q/k RMSNorm + rotary embedding + KV write stage (qwen3.py:228-264, 322-366)."""
    out = []
    # Attention is stubbed here, so only the pages that receive new tokens need
    # real blocks: the cached-prefix pages of every table row point at block 0.
    def tables_for(kv, q, num_blocks, seed):
        rng = np.random.default_rng(seed)
        free = [int(b) for b in rng.permutation(np.arange(1, num_blocks))]
        rows = []
        for kl, ql in zip(kv, q):
            first, last = (int(kl) - int(ql)) // PAGE, (int(kl) - 1) // PAGE
            rows.append([0] * first + [free.pop() for _ in range(first, last + 1)])
        return rows

    # Prefill chunks over cached prefixes, GQA 4, D 128, positions up to ~3000.
    c = np.array([5, 17, 40])
    p = np.array([0, 983, 2960])
    case = _make_case("norm_rope_prefill", p + c, c, 8, 2, 128, 12, tables_for(p + c, c, 12, 21), 31)
    case["rope_rows"] = 4096
    out.append(case)
    # Decode, MHA, D 64, kv_lens on and next to page boundaries.
    kv = np.array([1, 16, 17, 640, 1999, 2048])
    case = _make_case("norm_rope_decode_d64", kv, [1] * 6, 4, 4, 64, 10, tables_for(kv, [1] * 6, 10, 22), 32)
    case["rope_rows"] = 2048
    out.append(case)
    return out


def run_reference_norm_rope(case, femtovllm, QwenSelfAttention, VarlenAttnMetadata):
    """The reference's own q_norm / k_norm (nn.RMSNorm), QwenRotaryEmbedding (base 1e6) and KV-write
    loop, with the attention op replaced by a stub that records the q it is given."""
    Hq, Hkv, D = case["Hq"], case["Hkv"], case["D"]
    kv_lens, q_lens = case["kv_lens"], case["q_lens"]
    T = int(q_lens.sum())
    md, padded, raw_cu, raw_pos, is_decoding = _varlen_metadata(kv_lens, q_lens, case["tables"], VarlenAttnMetadata)
    eps = 1e-6
    cfg = types.SimpleNamespace(head_dim=D, rms_norm_eps=eps)
    d_model = D * (Hq + 2 * Hkv)
    attn = QwenSelfAttention(d_model, Hq, Hkv, max_seqlen=case["rope_rows"], dropout_p=0.0, config=cfg)
    attn.w_q = _Slice(0, Hq * D)
    attn.w_k = _Slice(Hq * D, (Hq + Hkv) * D)
    attn.w_v = _Slice((Hq + Hkv) * D, (Hq + 2 * Hkv) * D)
    gen = torch.Generator().manual_seed(int(case["kv_lens"].sum()))
    q_w = (1.0 + 0.25 * torch.randn(D, generator=gen)).to(torch.bfloat16).to(torch.float32)
    k_w = (1.0 + 0.25 * torch.randn(D, generator=gen)).to(torch.bfloat16).to(torch.float32)
    with torch.no_grad():
        attn.q_norm.weight.copy_(q_w)
        attn.k_norm.weight.copy_(k_w)
    attn.o_proj = torch.nn.Identity()
    attn.eval()
    q_tok = case["q"].transpose(0, 1).reshape(T, Hq * D)
    x = torch.cat([q_tok, case["k_new"].reshape(T, Hkv * D), case["v_new"].reshape(T, Hkv * D)], dim=1)
    seen = {}

    def stub(q, **kw):
        seen["q"] = q.detach().clone()
        return torch.zeros_like(q)

    kp, vp = case["k_pool"].clone(), case["v_pool"].clone()
    saved = (femtovllm.ops.paged_attention_gemv, femtovllm.ops.paged_attention_gemm)
    femtovllm.ops.paged_attention_gemv = stub
    femtovllm.ops.paged_attention_gemm = stub
    try:
        with torch.no_grad():
            if is_decoding:
                attn.forward_varlen_custom_gemv(x, kp, vp, md)
            else:
                attn.forward_varlen_custom_gemm(x, kp, vp, md)
    finally:
        femtovllm.ops.paged_attention_gemv, femtovllm.ops.paged_attention_gemm = saved
    pos = torch.tensor(raw_pos, dtype=torch.long)
    return {
        "q_ref": seen["q"].numpy().astype(np.float32),  # (Hq, T, D), as handed to the attention op
        "k_pool": kp,
        "v_pool": vp,
        "q_norm_weight": q_w,
        "k_norm_weight": k_w,
        "eps": eps,
        "cos_rows": attn.rotary_embd.cos[pos].numpy().astype(np.float32),
        "sin_rows": attn.rotary_embd.sin[pos].numpy().astype(np.float32),
        "padded": padded,
        "cu": raw_cu,
        "pos": raw_pos,
    }


def run_reference_routes(ref: Path):
    """Per-step metadata as the reference's ModelRunner builds it (model_runner.py:159-339): its own
    _route_prefill / _route_decode run on a stand-in object whose model records the
    VarlenAttnMetadata it is handed."""
    from femtovllm.engine.model_runner import ModelRunner

    seen = {}

    class _Model:
        def forward_varlen(self, idx_flatten, varlen_attn_metadata, skip_lm_head=True):
            seen["md"] = varlen_attn_metadata
            return None

    runner = types.SimpleNamespace(device="cpu", model=_Model())
    runner.pad_block_tables = lambda t: ModelRunner.pad_block_tables(runner, t)
    rng = np.random.default_rng(41)
    out = {}
    # Prefill route: new chunks over cached prefixes (0, page edges, long), ragged table rows.
    num_computed = np.array([0, 15, 16, 100, 2047, 0, 31], np.int64)
    num_new = np.array([5, 1, 33, 64, 1, 300, 17], np.int64)
    # Decode route: one new token per sequence.
    dec_computed = np.array([0, 15, 16, 17, 1000, 4095], np.int64)
    for route, (pc, pn) in {"prefill": (num_computed, num_new), "decode": (dec_computed, np.ones(6, np.int64))}.items():
        free = [int(b) for b in rng.permutation(4096)]
        tables = []
        for p, n in zip(pc, pn):
            need = (int(p + n) + PAGE - 1) // PAGE + int(rng.integers(0, 3))  # rows may run past kv_len
            tables.append([free.pop() for _ in range(need)])
        scheduled = [(types.SimpleNamespace(num_computed_tokens=int(p), token_ids=list(range(int(p + n)))), int(n))
                     for p, n in zip(pc, pn)]
        if route == "prefill":
            ModelRunner._route_prefill(runner, scheduled, None, None, tables)
        else:
            ModelRunner._route_decode(runner, scheduled, None, None, tables)
        md = seen["md"]
        flat = np.asarray([b for t in tables for b in t], np.int32)
        cu_blocks = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int32)
        out[f"{route}_num_computed"] = pc.astype(np.int32)
        out[f"{route}_num_new"] = pn.astype(np.int32)
        out[f"{route}_flat_blocks"] = flat
        out[f"{route}_cu_blocks"] = cu_blocks
        out[f"{route}_positions"] = md.positions.numpy()
        out[f"{route}_kv_lens"] = md.kv_lens.numpy()
        out[f"{route}_block_tables"] = md.block_tables.numpy()
        out[f"{route}_max_q_len"] = np.int32(md.max_q_len)
        out[f"{route}_max_kv_len"] = np.int32(md.max_kv_len)
        if md.cu_seqlens is not None:
            out[f"{route}_cu_seqlens"] = md.cu_seqlens.numpy()
    np.savez_compressed(HERE / "metadata_routes.npz", **out)
    print("metadata_routes: prefill T=%d, decode B=%d" % (int(num_new.sum()), len(dec_computed)))


def sampler_cases():
    """Logit batches for the reference Sampler: greedy rows (exact ids: ties, penalties that move
    the argmax, negative and tiny penalties) and sampled rows over a small vocabulary (counts of
    many draws, with and without the batch-wide penalty that switches bf16 logits to fp32)."""
    g = torch.Generator().manual_seed(77)
    V = 1000
    out = []
    lg = (torch.randn(6, V, generator=g) * 3).to(torch.bfloat16)
    lg[0, 10] = lg[0, 500] = lg[0].max() + 1  # a tie: the first index wins
    out.append(dict(name="greedy_bf16", logits=lg, temps=[0.0] * 6, pens=[0.0] * 6, tables=[[]] * 6, draws=1))
    lg = torch.randn(6, V, generator=g) * 2
    top = lg.argmax(dim=1).tolist()
    tables = [[top[0], 3, 3, 999], [], [top[2], top[2]], [7, 8, 9], [top[4], 0], [top[5]]]
    lg[3, 8] = lg[3].max() - 0.1  # a negative penalty lifts token 8 over the maximum
    out.append(dict(name="greedy_pen_f32", logits=lg, temps=[0.0] * 6, pens=[1.0, 0.0, 0.5, -0.3, 2.0, 1e-6],
                    tables=tables, draws=1))
    Vs = 12
    base = torch.tensor([2.9, 2.1, 1.3, 0.2, -0.7, 3.3, 1.0, -2.0, 0.55, 2.6, -1.1, 1.9])
    lg = torch.stack([base, base.flip(0), base * 1.7, base - 1.0]).to(torch.bfloat16)
    out.append(dict(name="dist_bf16", logits=lg, temps=[0.7, 1.0, 1.5, 0.3], pens=[0.0] * 4, tables=[[]] * 4,
                    draws=20000))
    out.append(dict(name="dist_pen", logits=lg.clone(), temps=[0.7, 1.0, 1.5, 0.0], pens=[1.0, 0.0, 0.5, 0.0],
                    tables=[[0, 5, Vs, Vs], [1, 2], [5, 9, 0], [3]], draws=20000))
    return out


def run_reference_sampler(ref: Path):
    """The reference's Sampler.forward (femtovllm/engine/sampler.py:15-114) on CPU with stand-in
    sequences: greedy ids of every row and, over `draws` calls, the count of each sampled token."""
    from femtovllm.engine.sampler import Sampler

    torch.manual_seed(5)
    sampler = Sampler()
    out = {}
    for case in sampler_cases():
        lg = case["logits"]
        B, V = lg.shape
        seqs = [(types.SimpleNamespace(token_ids=list(t), sampling_params=types.SimpleNamespace(
            temperature=float(tp), presence_penalty=float(pp))), 1)
            for t, tp, pp in zip(case["tables"], case["temps"], case["pens"])]
        counts = np.zeros((B, V), np.int64)
        for _ in range(case["draws"]):
            ids = sampler(lg.clone(), seqs)
            counts[np.arange(B), ids] += 1
        width = max(1, max(len(t) for t in case["tables"]))
        table = np.full((B, width), V, np.int64)
        for i, t in enumerate(case["tables"]):
            table[i, : len(t)] = t
        n = case["name"]
        out[f"{n}_dtype"] = np.array("bf16" if lg.dtype == torch.bfloat16 else "f32")
        out[f"{n}_logits"] = lg.float().numpy()
        out[f"{n}_temps"] = np.asarray(case["temps"], np.float32)
        out[f"{n}_pens"] = np.asarray(case["pens"], np.float32)
        out[f"{n}_table"] = table
        out[f"{n}_counts"] = counts
        print(f"sampler {n}: B={B} V={V} draws={case['draws']}")
    out["names"] = np.array([c["name"] for c in sampler_cases()])
    np.savez_compressed(HERE / "sampler.npz", **out)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _changed_rows(before, after):
    diff = (before != after).any(dim=-1).nonzero().numpy().astype(np.int32)  # (n, 3): block, head, offset
    rows = after[diff[:, 0], diff[:, 1], diff[:, 2]]
    return diff, _bits(rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--which", choices=["attention", "norm_rope", "metadata", "sampler", "all"], default="all")
    args = ap.parse_args()
    femtovllm, QSA, VAM = _import_reference(args.reference)
    if args.which in ("sampler", "all"):
        run_reference_sampler(args.reference)
        if args.which == "sampler":
            return
    if args.which in ("metadata", "all"):
        run_reference_routes(args.reference)
        if args.which == "metadata":
            return
    if args.which in ("norm_rope", "all"):
        for case in norm_rope_cases():
            r = run_reference_norm_rope(case, femtovllm, QSA, VAM)
            k_idx, _ = _changed_rows(case["k_pool"], r["k_pool"])
            v_idx, v_rows = _changed_rows(case["v_pool"], r["v_pool"])
            k_rows = r["k_pool"][k_idx[:, 0], k_idx[:, 1], k_idx[:, 2]].numpy().astype(np.float32)
            np.savez_compressed(
                HERE / f"{case['name']}.npz",
                n_heads=case["Hq"],
                n_kv_heads=case["Hkv"],
                head_dim=case["D"],
                num_blocks=case["num_blocks"],
                rope_rows=case["rope_rows"],
                eps=np.float32(r["eps"]),
                kv_lens=case["kv_lens"],
                q_lens=case["q_lens"],
                cu_seqlens=np.asarray(r["cu"], np.int32),
                positions=np.asarray(r["pos"], np.int32),
                block_tables=np.asarray(r["padded"], np.int32),
                q_bits=_bits(case["q"].transpose(0, 1).contiguous()),  # (T, Hq, D): the projection output
                k_new_bits=_bits(case["k_new"]),
                v_new_bits=_bits(case["v_new"]),
                q_norm_weight_bits=_bits(r["q_norm_weight"]),
                k_norm_weight_bits=_bits(r["k_norm_weight"]),
                cos_rows=r["cos_rows"],
                sin_rows=r["sin_rows"],
                k_pool_bits=_bits(case["k_pool"]),
                v_pool_bits=_bits(case["v_pool"]),
                k_written_idx=k_idx,
                k_written=k_rows,
                v_written_idx=v_idx,
                v_written_bits=v_rows,
                q_ref=r["q_ref"],
            )
            print(f"{case['name']}: T={int(case['q_lens'].sum())} rows written={len(k_idx)}")
    if args.which == "norm_rope":
        return
    for case in cases():
        out, (kp, vp), (kp2, vp2), padded, cu, pos = run_reference(case, femtovllm, QSA, VAM)
        k_rows_idx, k_rows = _changed_rows(case["k_pool"], kp)
        v_rows_idx, v_rows = _changed_rows(case["v_pool"], vp)
        k2_idx, k2 = _changed_rows(case["k_pool"], kp2)
        v2_idx, v2 = _changed_rows(case["v_pool"], vp2)
        assert np.array_equal(k_rows_idx, k2_idx) and np.array_equal(k_rows, k2), "write loops disagree (K)"
        assert np.array_equal(v_rows_idx, v2_idx) and np.array_equal(v_rows, v2), "write loops disagree (V)"
        np.savez_compressed(
            HERE / f"{case['name']}.npz",
            n_heads=case["Hq"],
            n_kv_heads=case["Hkv"],
            head_dim=case["D"],
            num_blocks=case["num_blocks"],
            kv_lens=case["kv_lens"],
            q_lens=case["q_lens"],
            cu_seqlens=np.asarray(cu, np.int32),
            positions=np.asarray(pos, np.int32),
            block_tables=np.asarray(padded, np.int32),
            q_bits=_bits(case["q"]),
            k_new_bits=_bits(case["k_new"]),
            v_new_bits=_bits(case["v_new"]),
            k_pool_bits=_bits(case["k_pool"]),
            v_pool_bits=_bits(case["v_pool"]),
            k_written_idx=k_rows_idx,
            k_written_bits=k_rows,
            v_written_idx=v_rows_idx,
            v_written_bits=v_rows,
            out_ref=out.numpy().astype(np.float32),
        )
        print(f"{case['name']}: T={int(case['q_lens'].sum())} rows written={len(k_rows_idx)}")


if __name__ == "__main__":
    main()
