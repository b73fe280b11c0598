"""Python op boundary, mirroring ``femtovllm/ops/__init__.py`` of the reference.

Same function names, argument order and meaning, and error behaviour:

* ``paged_attention_gemv`` (reference ``ops/__init__.py:82-107``): decode,
  ``q`` of shape ``(n_heads, B, d_head)``;
* ``paged_attention_gemm`` (reference ``ops/__init__.py:110-156``): varlen
  chunked prefill, ``q`` of shape ``(n_heads, q_len_flatten, d_head)``;
* ``MAX_KV_LEN_NON_SPLIT``, ``KV_LEN_PER_PAGE``, ``DIM_HEAD`` (reference
  ``ops/__init__.py:21-26``), read from the native module;

plus ``store_kvcache``, the slot-mapped KV write that replaces the Python
loops of ``femtovllm/models/qwen/qwen3.py:240-264, 322-366``,
``build_slot_mapping``, which computes its ``slot_mapping`` on the device, and
``qk_norm_rope_store``, which fuses the q/k RMSNorm and rotary embedding of
``qwen3.py:234-238`` with that write and hands q back head-major, and
``sample_tokens``, the arithmetic of ``femtovllm/engine/sampler.py`` in one
launch (the drop-in ``Sampler`` module is ``femtovllm_b200.sampler``).

The reference routes each op through a Triton/CUDA backend switch
(``femtovllm._DEV``, ``ImplCustomKernel``).  That router is gone: ``impl`` is
accepted for signature compatibility and ignored; every call runs the sm_100a
kernels of ``libfemtovllm_b200.so``.  Non-CUDA tensors raise ``ValueError``
(reference ``ops/__init__.py:36-39``); the native checks raise
``RuntimeError``.
"""

from __future__ import annotations

import torch

from femtovllm_b200 import EXT_PATH

try:
    from femtovllm_b200 import _C as _cuda_backend
except ImportError as e:  # no fallback: the product path is the CUDA extension
    raise ImportError(
        f"femtovllm_b200: native extension not built ({EXT_PATH}). "
        "Run `python -m femtovllm_b200._build` from nano-vllm-practice_b200/."
    ) from e

MAX_KV_LEN_NON_SPLIT = _cuda_backend.kMaxKVLenNonSplit
KV_LEN_PER_PAGE = _cuda_backend.kKVLenPerPage
DIM_HEAD = _cuda_backend.kDimHead


def _ensure_valid_tensor(t: torch.Tensor, name: str) -> torch.Tensor:
    """CUDA check + contiguous copy, as the reference helper (ops/__init__.py:29-44)."""
    if not t.is_cuda:
        raise ValueError(f"Argument '{name}' must be a CUDA tensor. Got device={t.device}")
    if not t.is_contiguous():
        return t.contiguous()
    return t


def _q_view(q: torch.Tensor) -> torch.Tensor:
    """q as the kernels can read it in place: any ``(n_heads, T, d_head)`` view whose
    ``d_head`` is contiguous and whose token / head strides are 16-byte multiples (for
    example ``q_thd.transpose(0, 1)`` of the projection output); anything else is copied,
    as the reference's ``_ensure_valid_tensor`` does (``ops/__init__.py:29-44``)."""
    if not q.is_cuda:
        raise ValueError(f"Argument 'q' must be a CUDA tensor. Got device={q.device}")
    es = q.element_size()
    if q.dim() == 3 and q.stride(2) == 1 and (q.stride(0) * es) % 16 == 0 and (q.stride(1) * es) % 16 == 0 \
            and q.data_ptr() % 16 == 0:
        return q
    return q.contiguous()


def paged_attention_gemv(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    kv_page_tables: torch.Tensor,
    kv_lens: torch.Tensor,
    max_kv_len: int,
    impl=None,
    out_token_major: bool = False,
) -> torch.Tensor:
    """Decode paged attention; returns ``(n_heads, B, d_head)`` in q's dtype.

    ``out_token_major=True`` returns the same shape as a view of a ``(B, n_heads, d_head)``
    buffer, so ``out.transpose(0, 1).reshape(B, n_heads * d_head)`` (the o_proj input,
    ``qwen3.py:278``) is free.  ``q`` may be a transposed view (see ``_q_view``).
    """
    q = _q_view(q)
    for t, n in ((k_pool, "k_pool"), (v_pool, "v_pool"), (kv_page_tables, "kv_page_tables"), (kv_lens, "kv_lens")):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    return _cuda_backend.PagedAttentionGemvCuda(q, k_pool, v_pool, kv_page_tables, kv_lens, int(max_kv_len),
                                                bool(out_token_major))


def paged_attention_gemm(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_q_len: int,
    Q_TILE_SIZE: int,
    cu_q_tiles: torch.Tensor,
    q_tile_to_seq_idx: torch.Tensor,
    kv_page_tables: torch.Tensor,
    kv_lens: torch.Tensor,
    positions: torch.Tensor,
    impl=None,
    out_token_major: bool = False,
) -> torch.Tensor:
    """Varlen chunked-prefill attention; returns ``(n_heads, q_len_flatten, d_head)``.

    ``Q_TILE_SIZE``, ``cu_q_tiles`` and ``q_tile_to_seq_idx`` are the
    reference Triton kernel's tiling metadata (``model_runner.py:174-202``);
    they are accepted and unused, since the kernel tiles the queries itself.
    ``out_token_major`` and strided ``q`` as for ``paged_attention_gemv``.
    """
    q = _q_view(q)
    for t, n in (
        (k_pool, "k_pool"),
        (v_pool, "v_pool"),
        (cu_seqlens, "cu_seqlens"),
        (kv_page_tables, "kv_page_tables"),
        (kv_lens, "kv_lens"),
        (positions, "positions"),
    ):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    return _cuda_backend.PagedAttentionGemmCuda(
        q, k_pool, v_pool, cu_seqlens, int(max_q_len), kv_page_tables, kv_lens, positions, bool(out_token_major)
    )


def store_kvcache(
    k: torch.Tensor,
    v: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Write ``k[t]``, ``v[t]`` (each ``(n_kv_heads, d_head)``) to pool slot ``slot_mapping[t]``.

    ``slot = block_table[s][pos // 16] * 16 + pos % 16`` (int64; ``-1`` skips).
    ``k`` / ``v`` may be strided views ``(T, n_kv_heads, d_head)`` of the
    projection output as long as ``d_head`` is contiguous.
    """
    for t, n in ((k, "k"), (v, "v"), (k_pool, "k_pool"), (v_pool, "v_pool"), (slot_mapping, "slot_mapping")):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    _cuda_backend.StoreKVCacheCuda(k, v, k_pool, v_pool, slot_mapping.contiguous())


def build_slot_mapping(
    positions: torch.Tensor,
    block_tables: torch.Tensor,
    cu_seqlens: torch.Tensor | None = None,
) -> torch.Tensor:
    """int64 slot of every new token: ``table[s][pos // 16] * 16 + pos % 16`` (-1 for a -1 entry).

    ``cu_seqlens`` (int32, ``num_seqs + 1``) maps tokens to sequences; ``None``
    means one token per sequence (decode).  Computed on the device; it is the
    index arithmetic of the reference write loops (``qwen3.py:250-264, 335-361``).
    """
    for t, n in ((positions, "positions"), (block_tables, "block_tables")):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    return _cuda_backend.BuildSlotMappingCuda(positions.contiguous(), cu_seqlens, block_tables.contiguous())


def build_varlen_metadata(
    num_computed: torch.Tensor,
    num_new: torch.Tensor,
    flat_blocks: torch.Tensor,
    cu_blocks: torch.Tensor,
    max_blocks_per_seq: int,
    num_tokens: int,
) -> dict:
    """Attention metadata of one step from per-sequence counts, built on the device.

    For sequence ``s`` with ``num_computed[s]`` cached and ``num_new[s]`` new tokens
    (decode: 1), as ``ModelRunner._route_prefill`` / ``_route_decode`` build them on the
    host (``model_runner.py:186-205, 280-290``) and ``pad_block_tables`` (``:46-72``):
    ``positions`` (``range(p, p + n)`` per sequence), ``cu_seqlens``, ``kv_lens = p + n``,
    ``block_tables`` (``-1``-padded to ``max_blocks_per_seq``) and ``slot_mapping``.
    ``flat_blocks`` holds every sequence's blocks back to back, ``cu_blocks`` (``B + 1``)
    where each row starts; ``num_tokens`` is ``sum(num_new)`` (the scheduler knows it).
    """
    for t, n in ((num_computed, "num_computed"), (num_new, "num_new"), (flat_blocks, "flat_blocks"),
                 (cu_blocks, "cu_blocks")):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    i32 = lambda t: t.to(torch.int32).contiguous()  # noqa: E731
    pos, cu, kv, tables, slots = _cuda_backend.BuildVarlenMetadataCuda(
        i32(num_computed), i32(num_new), i32(flat_blocks), i32(cu_blocks), int(max_blocks_per_seq), int(num_tokens)
    )
    return {"positions": pos, "cu_seqlens": cu, "kv_lens": kv, "block_tables": tables, "slot_mapping": slots}


def qk_norm_rope_store(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    eps: float,
    rope_cos: torch.Tensor,
    rope_sin: torch.Tensor,
    positions: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> torch.Tensor:
    """q/k RMSNorm + rotary embedding + KV write in one pass; returns q as ``(n_heads, T, d_head)``.

    Does what ``QwenSelfAttention`` does between its projections and the
    attention op (``qwen3.py:234-238`` then the write loops ``:240-264`` /
    ``:322-366`` and ``q.transpose(0, 1)``): ``q``/``k`` are normalised over
    ``d_head`` (``x / sqrt(mean(x^2) + eps) * weight``), rotated with the
    rotary module's ``cos``/``sin`` buffers (``(rows, d_head)``) at
    ``positions[t]``, k and v land in ``slot_mapping[t]`` (``-1`` skips) and
    the returned q is ready for ``paged_attention_gemv`` / ``_gemm``.
    ``q``, ``k``, ``v`` are ``(T, heads, d_head)`` views (e.g. of the
    projection outputs) with ``d_head`` contiguous and 16-byte aligned rows.
    """
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (k_pool, "k_pool"), (v_pool, "v_pool"), (positions, "positions"),
                 (slot_mapping, "slot_mapping"), (rope_cos, "rope_cos"), (rope_sin, "rope_sin")):
        if not t.is_cuda:
            raise ValueError(f"Argument '{n}' must be a CUDA tensor. Got device={t.device}")
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    if positions.dtype != torch.int32:
        positions = positions.to(torch.int32)
    return _cuda_backend.QKNormRopeStoreCuda(
        q, k, v, q_norm_weight.contiguous(), k_norm_weight.contiguous(), float(eps), rope_cos.contiguous(),
        rope_sin.contiguous(), positions.contiguous(), k_pool, v_pool, slot_mapping.contiguous()
    )


def new_rng_state(seed: int | None = None, device: torch.device | str = "cuda") -> torch.Tensor:
    """Device RNG state ``{seed, offset}`` (int64, 2) for :func:`sample_tokens`; a seed drawn from
    torch's global CPU generator when none is given (so ``torch.manual_seed`` makes runs repeat)."""
    if seed is None:
        seed = int(torch.randint(0, 2**62, (1,)).item())
    return torch.tensor([seed, 0], dtype=torch.int64, device=device)


def sample_workspace(num_rows: int, vocab: int, device: torch.device | str = "cuda") -> torch.Tensor:
    """Zeroed workspace for :func:`sample_tokens`, reusable across calls (each call leaves it zero)."""
    return torch.zeros(max(int(_cuda_backend.SampleWorkspaceSize(num_rows, vocab)), 1), dtype=torch.uint8,
                       device=device)


def sample_tokens(
    logits: torch.Tensor,
    temperatures: torch.Tensor,
    presence_penalties: torch.Tensor | None = None,
    token_table: torch.Tensor | None = None,
    rng_state: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Next-token ids ``(B,)`` int64 from ``logits`` ``(B, vocab)``, on the device (one pass over the logits).

    The arithmetic of the reference's ``Sampler.forward`` (``femtovllm/engine/sampler.py:15-114``):
    when any ``|presence_penalties| > 1e-5``, every token that occurs in a row of ``token_table``
    (``(B, L)`` int64; entries outside ``[0, vocab)`` are padding, as the reference's pad id
    ``vocab``) loses that row's penalty; rows with ``temperatures < 1e-5`` take the first argmax,
    the others one draw from ``softmax(logits / T)``.  ``rng_state`` (:func:`new_rng_state`) is
    advanced on the device by every call, so the op can be captured in a CUDA graph together
    with a persistent ``workspace`` (:func:`sample_workspace`).
    """
    if not logits.is_cuda:
        raise ValueError(f"Argument 'logits' must be a CUDA tensor. Got device={logits.device}")
    dev = logits.device
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    temperatures = temperatures.to(device=dev, dtype=torch.float32).contiguous()
    if presence_penalties is not None:
        presence_penalties = presence_penalties.to(device=dev, dtype=torch.float32).contiguous()
    if token_table is not None:
        token_table = token_table.to(device=dev, dtype=torch.int64)
        if token_table.stride(-1) != 1:
            token_table = token_table.contiguous()
    if rng_state is None:
        rng_state = new_rng_state(device=dev)
    return _cuda_backend.SampleTokensCuda(logits, temperatures, presence_penalties, token_table, rng_state,
                                          workspace)


def read_device_error() -> tuple[int, int]:
    """(code, info) of the first bad page / slot / timeout a kernel recorded; clears it. Synchronizes."""
    return tuple(_cuda_backend.ReadDeviceError())
