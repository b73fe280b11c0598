"""numpy restatement of the reference's next-token sampler (test infrastructure).

``Sampler.forward`` (``femtovllm/engine/sampler.py:15-114``), row by row:

* ``apply = any(|presence_penalty| > 1e-5)`` over the batch (``:31-35``);
* if ``apply``: ``counts`` is a ``scatter_add`` of the row's token ids padded with
  ``vocab`` (the pad column is dropped) and ``logits - p[:, None] * (counts > 0)``
  (``:56-76``): a token that occurs loses ``p``; the result is fp32;
* ``temperature < 1e-5`` (``:41-46``): ``argmax`` (the first maximal index, ``:88-95``);
* otherwise ``logits / T`` in place (``:97-104``; in the logits' own dtype, so
  bf16 / fp16 rounding, when ``apply`` is off, fp32 when on), ``softmax`` and one
  ``multinomial`` draw (``:106-109``).

The device kernel draws by inverse CDF over vocabulary order with one
Philox4x32-10 uniform per row (Salmon et al., SC 2011; restated below and checked
against the published known-answer vectors in the tests), so :func:`sample`
reproduces its choice for comparison, and :func:`probabilities` gives the
distribution against which the reference's own ``multinomial`` frequencies are
tested.  Pinned by ``tests/golden/sampler.npz`` (reference ids of greedy rows, and
reference sample counts), made by ``tests/golden/make_golden.py``.
"""

from __future__ import annotations

import numpy as np

GREEDY_BELOW = 1e-5
PENALTY_ABOVE = 1e-5

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(counters, key):
    """Philox4x32-10 of ``counters`` ``(N, 4)`` uint32 under ``key`` ``(k0, k1)`` -> ``(N, 4)`` uint32."""
    c = [np.asarray(counters, np.uint64)[:, i].copy() for i in range(4)]
    k0, k1 = int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF
    for r in range(10):
        if r:
            k0, k1 = (k0 + _W0) & 0xFFFFFFFF, (k1 + _W1) & 0xFFFFFFFF
        p0 = _M0 * c[0]
        p1 = _M1 * c[2]
        c = [((p1 >> np.uint64(32)) ^ c[1] ^ np.uint64(k0)) & _MASK, p1 & _MASK,
             ((p0 >> np.uint64(32)) ^ c[3] ^ np.uint64(k1)) & _MASK, p0 & _MASK]
    return np.stack(c, axis=1).astype(np.uint32)


def uniforms(num_rows: int, seed: int, offset: int) -> np.ndarray:
    """The kernel's per-row uniform in [0, 1): 53 bits of Philox(counter {row, 0, offset}, key seed)."""
    seed, offset = int(seed) & (2**64 - 1), int(offset) & (2**64 - 1)
    ctr = np.zeros((num_rows, 4), np.uint64)
    ctr[:, 0] = np.arange(num_rows)
    ctr[:, 2] = offset & 0xFFFFFFFF
    ctr[:, 3] = offset >> 32
    r = philox4x32_10(ctr, (seed & 0xFFFFFFFF, seed >> 32)).astype(np.uint64)
    bits = (r[:, 0] << np.uint64(21)) | (r[:, 1] >> np.uint64(11))
    return bits.astype(np.float64) * 2.0**-53


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> ``dtype`` (round to nearest even) -> fp32, as torch's in-place division stores it."""
    x = np.asarray(x, np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)) << np.uint64(16)
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isfinite(x), out, x).astype(np.float32)


def penalized(logits, penalties, token_table):
    """(x, apply): the logits after the presence penalty (fp32), and whether it applied."""
    x = np.asarray(logits, np.float32).copy()
    B, V = x.shape
    pens = None if penalties is None else np.asarray(penalties, np.float32)
    apply = pens is not None and bool(np.any(np.abs(pens.astype(np.float64)) > PENALTY_ABOVE))
    if apply and token_table is not None:
        table = np.asarray(token_table, np.int64)
        for b in range(B):
            ids = table[b]
            ids = ids[(ids >= 0) & (ids < V)]
            present = np.zeros(V, bool)
            present[ids] = True
            x[b, present] = x[b, present] - pens[b]
    return x, apply


def scaled(x_row, temperature, apply: bool, dtype: str):
    """``x / T`` as the reference leaves it before softmax (fp32 division, rounded to the
    logits' dtype when the penalty did not turn them into fp32)."""
    xs = (np.asarray(x_row, np.float32) / np.float32(temperature)).astype(np.float32)
    return xs if apply else round_to(xs, dtype)


def probabilities(logits, dtype, temperatures, penalties=None, token_table=None):
    """``(B, V)`` float64 sampling distribution of every row (one-hot at the argmax for greedy rows)."""
    x, apply = penalized(logits, penalties, token_table)
    B, V = x.shape
    out = np.zeros((B, V), np.float64)
    for b in range(B):
        t = float(np.float32(temperatures[b]))
        if t < GREEDY_BELOW:
            out[b, int(np.argmax(x[b]))] = 1.0
            continue
        xs = scaled(x[b], t, apply, dtype).astype(np.float64)
        m = xs.max()
        if not np.isfinite(m):
            out[b, 0] = 1.0
            continue
        e = np.exp(xs - m)
        out[b] = e / e.sum()
    return out


def sample(logits, dtype, temperatures, penalties=None, token_table=None, seed=0, offset=0):
    """``(ids, margin)``: each row's token as the kernel picks it (argmax for greedy rows, the
    inverse CDF of :func:`probabilities` at the Philox uniform for sampled rows) and, for sampled
    rows, the distance of the uniform from the nearest CDF edge (``inf`` for greedy rows): a
    kernel whose fp32 sums differ in the last bits may pick the neighbour only when it is tiny."""
    p = probabilities(logits, dtype, temperatures, penalties, token_table)
    B = p.shape[0]
    u = uniforms(B, seed, offset)
    ids = np.zeros(B, np.int64)
    margin = np.full(B, np.inf)
    x, _ = penalized(logits, penalties, token_table)
    for b in range(B):
        if float(np.float32(temperatures[b])) < GREEDY_BELOW:
            ids[b] = int(np.argmax(x[b]))
            continue
        cdf = np.cumsum(p[b])
        cdf /= cdf[-1]
        k = int(np.searchsorted(cdf, u[b], side="right"))
        k = min(k, len(cdf) - 1)
        ids[b] = k
        lo = cdf[k - 1] if k > 0 else 0.0
        margin[b] = min(u[b] - lo, cdf[k] - u[b])
    return ids, margin
