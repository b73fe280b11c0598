"""numpy restatement of the reference's per-step attention metadata (test infrastructure).

``ModelRunner._route_prefill`` (``femtovllm/engine/model_runner.py:186-205``) and
``_route_decode`` (``:280-290``) walk the scheduled sequences on the host: for a
sequence with ``p`` computed tokens and ``n`` new ones they append
``range(p, p + n)`` to the positions, ``cu_seqlens[-1] + n`` to the cumulative
query lengths and ``p + n`` to the kv lengths (decode: ``n = 1``, no
cu_seqlens); ``pad_block_tables`` (``:46-72``) pads every block-table row with
``-1`` to the longest row.  Pinned by ``tests/golden/metadata_routes.npz``,
captured from those reference methods by ``tests/golden/make_golden.py``.
"""

from __future__ import annotations

import numpy as np

from oracle.paged_attention import build_slot_mapping


def varlen_metadata(num_computed, num_new, raw_block_tables):
    """``{positions, cu_seqlens, kv_lens, block_tables, slot_mapping, max_q_len, max_kv_len}`` (int32 / int64)."""
    positions, cu, kv = [], [0], []
    for p, n in zip(num_computed, num_new):
        p, n = int(p), int(n)
        positions.extend(range(p, p + n))
        cu.append(cu[-1] + n)
        kv.append(p + n)
    width = max(len(t) for t in raw_block_tables)
    tables = np.full((len(raw_block_tables), width), -1, dtype=np.int32)
    for i, row in enumerate(raw_block_tables):
        tables[i, : len(row)] = row
    positions = np.asarray(positions, np.int32)
    seq_of_token = np.repeat(np.arange(len(num_new)), np.asarray(num_new, np.int64))
    return {
        "positions": positions,
        "cu_seqlens": np.asarray(cu, np.int32),
        "kv_lens": np.asarray(kv, np.int32),
        "block_tables": tables,
        "slot_mapping": build_slot_mapping(positions, seq_of_token, tables),
        "max_q_len": int(max(num_new)),
        "max_kv_len": int(max(kv)),
    }
