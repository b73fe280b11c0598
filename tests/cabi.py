"""Call the C ABI of libfemtovllm_b200.so on torch tensors (test helper)."""

from __future__ import annotations

import ctypes

import torch

from femtovllm_b200 import capi

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = capi.load()
    return _lib


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def store_kvcache(k, v, k_pool, v_pool, slot_mapping):
    assert k.stride() == v.stride() and k.stride(2) == 1
    st = lib().fvb_store_kvcache(
        k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0],
        slot_mapping.data_ptr(), k.shape[0], k.shape[1], k.shape[2], k_pool.shape[2], capi.dtype_code(k.dtype),
        _stream(),
    )
    capi.check(st, "fvb_store_kvcache")


def decode(q, k_pool, v_pool, block_tables, kv_lens, max_kv_len):
    hq, b, d = q.shape
    hkv = k_pool.shape[1]
    out = torch.empty_like(q)
    ws_bytes = lib().fvb_paged_attention_decode_workspace_size(b, hq, hkv, d, int(max_kv_len))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    st = lib().fvb_paged_attention_decode(
        q.data_ptr(), out.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0], hq, hkv, d,
        k_pool.shape[2], b, block_tables.data_ptr(), block_tables.shape[1], kv_lens.data_ptr(), int(max_kv_len),
        capi.dtype_code(q.dtype), ws.data_ptr(), ws_bytes, _stream(),
    )
    capi.check(st, "fvb_paged_attention_decode")
    return out


def prefill(q, k_pool, v_pool, cu_seqlens, max_q_len, block_tables, kv_lens, positions):
    hq, t, d = q.shape
    hkv = k_pool.shape[1]
    b = cu_seqlens.numel() - 1
    out = torch.empty_like(q)
    ws_bytes = lib().fvb_paged_attention_prefill_workspace_size(b, hq, hkv, d, t, int(max_q_len))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    st = lib().fvb_paged_attention_prefill(
        q.data_ptr(), out.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0], hq, hkv, d,
        k_pool.shape[2], b, t, cu_seqlens.data_ptr(), int(max_q_len), block_tables.data_ptr(), block_tables.shape[1],
        kv_lens.data_ptr(), positions.data_ptr(), capi.dtype_code(q.dtype), ws.data_ptr(), ws_bytes, _stream(),
    )
    capi.check(st, "fvb_paged_attention_prefill")
    return out


def read_device_error():
    code, info = ctypes.c_int(0), ctypes.c_int(0)
    capi.check(lib().fvb_read_device_error(ctypes.byref(code), ctypes.byref(info), _stream()), "read_device_error")
    return code.value, info.value


def qk_norm_rope_store_status(q, k, v, q_w, k_w, eps, cos, sin, positions, k_pool, v_pool, slot_mapping, q_out):
    """Raw status of fvb_qk_norm_rope_store (q / k / v: (T, heads, D) strided views)."""
    return lib().fvb_qk_norm_rope_store(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0),
        v.stride(1), q_w.data_ptr(), k_w.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
        positions.data_ptr(), slot_mapping.data_ptr(), q.shape[0], q.shape[1], k.shape[1], q.shape[2],
        q_out.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0], k_pool.shape[2],
        capi.dtype_code(q.dtype), _stream(),
    )


def qk_norm_rope_store(q, k, v, q_w, k_w, eps, cos, sin, positions, k_pool, v_pool, slot_mapping):
    q_out = torch.empty((q.shape[1], q.shape[0], q.shape[2]), dtype=q.dtype, device=q.device)
    st = qk_norm_rope_store_status(q, k, v, q_w, k_w, eps, cos, sin, positions, k_pool, v_pool, slot_mapping, q_out)
    capi.check(st, "fvb_qk_norm_rope_store")
    return q_out


def sample_tokens(logits, temperatures, presence_penalties, token_table, rng_state, workspace=None):
    """fvb_sample_tokens on a (B, vocab) logits view with contiguous rows; returns int64 ids (B,)."""
    B, V = logits.shape
    assert logits.stride(1) == 1
    out = torch.empty(B, dtype=torch.int64, device=logits.device)
    ws_bytes = lib().fvb_sample_workspace_size(B, V)
    if workspace is None:
        workspace = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device=logits.device)
    has_table = token_table is not None and token_table.numel() > 0
    st = lib().fvb_sample_tokens(
        logits.data_ptr(), logits.stride(0), B, V, capi.dtype_code(logits.dtype), temperatures.data_ptr(),
        presence_penalties.data_ptr() if presence_penalties is not None else None,
        token_table.data_ptr() if has_table else None, token_table.stride(0) if has_table else 0,
        token_table.shape[1] if has_table else 0, rng_state.data_ptr(), out.data_ptr(), workspace.data_ptr(),
        workspace.numel(), _stream(),
    )
    capi.check(st, "fvb_sample_tokens")
    return out
