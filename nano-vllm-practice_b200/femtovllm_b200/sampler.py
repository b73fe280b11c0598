"""Drop-in for the reference's ``femtovllm.engine.sampler.Sampler``.

Same module interface (``femtovllm/engine/sampler.py:8-114``): ``forward(logits_next,
scheduled_const)`` takes lm_head's ``(B, vocab)`` output and the scheduler's
``[(Sequence, n), ...]`` and returns the next token id of every row as a Python list.
The reference turns the sampling parameters into Python lists, builds a ``(B, vocab)``
count matrix with ``scatter_add`` for the presence penalty and samples greedy and
temperature rows in separate gathers, ``argmax``, ``softmax`` and ``multinomial`` calls.
Here the per-row parameters go to the device once and one kernel
(:func:`femtovllm_b200.ops.sample_tokens`) applies the penalty, takes the greedy argmax or
draws the sample for every row.  Random numbers come from a device Philox state seeded
from torch's global generator, so ``torch.manual_seed`` makes runs repeat; the draws are
the same distribution as ``torch.multinomial``'s, not the same numbers.
"""

from __future__ import annotations

import numpy as np
import torch

from femtovllm_b200 import ops


class Sampler(torch.nn.Module):
    def __init__(self, seed: int | None = None):
        super().__init__()
        self._seed = seed
        self._rng: dict[torch.device, torch.Tensor] = {}
        self._workspace: dict[torch.device, torch.Tensor] = {}

    def _state(self, device: torch.device, rows: int, vocab: int) -> tuple[torch.Tensor, torch.Tensor]:
        if device not in self._rng:
            self._rng[device] = ops.new_rng_state(self._seed, device)
        need = int(ops._cuda_backend.SampleWorkspaceSize(rows, vocab))
        ws = self._workspace.get(device)
        if ws is None or ws.numel() < need:
            ws = ops.sample_workspace(rows, vocab, device)
            self._workspace[device] = ws
        return self._rng[device], ws

    def forward(self, logits_next: torch.Tensor, scheduled_const: list) -> list[int]:
        B, vocab_size = logits_next.shape
        device = logits_next.device
        params = [x.sampling_params for x, _ in scheduled_const]
        temperatures = torch.tensor([p.temperature for p in params], dtype=torch.float32)
        penalties = [p.presence_penalty for p in params]
        pens = table = None
        # The reference applies the penalty to the whole batch when any row asks for one
        # (sampler.py:31-35, 56-76); rows without a table entry are padded with vocab_size.
        if any(abs(x) > 1e-5 for x in penalties):
            histories = [x.token_ids for x, _ in scheduled_const]
            width = max(1, max(len(h) for h in histories))
            host = np.full((B, width), vocab_size, dtype=np.int64)
            for i, h in enumerate(histories):
                host[i, : len(h)] = h
            table = torch.from_numpy(host).to(device, non_blocking=True)
            pens = torch.tensor(penalties, dtype=torch.float32).to(device, non_blocking=True)
        rng, ws = self._state(device, B, vocab_size)
        ids = ops.sample_tokens(logits_next, temperatures.to(device, non_blocking=True), pens, table, rng, ws)
        return ids.tolist()
