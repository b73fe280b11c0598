"""CPU oracle for the FemtoVLLM attention hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the reference
algorithm of fishAndShrimp/nano-vllm-practice ("FemtoVLLM") for the three
parts of the attention hot path:

* the KV-cache write (the reference's per-sequence block-walk loops, and the
  equivalent ``slot_mapping`` scatter),
* decode paged attention over ``block_tables`` with GQA,
* varlen chunked-prefill causal attention over prefix-cached paged KV,
* the stage before them: q/k RMSNorm, rotary embedding and the KV write
  (``oracle/qk_norm_rope.py``),
* the per-step metadata (positions, cu_seqlens, kv_lens, padded block tables)
  the engine builds for them (``oracle/metadata.py``),
* the next-token sampler that consumes the step's logits: presence penalty,
  greedy argmax, temperature sampling (``oracle/sampler.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline.  The product path
(``femtovllm_b200``) never imports it and has no CPU fallback.

Parity pin: ``tests/golden/*.npz`` were produced by running the reference's
own ``QwenSelfAttention.forward_varlen_pytorch`` and its KV-write loops
(``femtovllm/models/qwen/qwen3.py:240-264, 322-366, 389-544``) on CPU, by
``tests/golden/make_golden.py``; the ``norm_rope_*`` fixtures record the
reference's q_norm / k_norm / QwenRotaryEmbedding and write loop
(``qwen3.py:17-138, 181-183, 228-264, 308-366``); ``sampler.npz`` records the
reference's ``Sampler`` (``femtovllm/engine/sampler.py``).  ``tests/test_oracle_golden.py``
checks this package against every one of those fixtures.
"""

from oracle.paged_attention import (  # noqa: F401
    build_slot_mapping,
    decode_attention,
    gather_seq_kv,
    prefill_attention,
    store_kvcache,
    store_kvcache_decode_loop,
    store_kvcache_prefill_loop,
)
from oracle.qk_norm_rope import (  # noqa: F401
    apply_rope,
    qk_norm_rope_store,
    rms_norm,
    rope_tables,
)
from oracle.metadata import varlen_metadata  # noqa: F401,E402
from oracle import sampler  # noqa: F401,E402
