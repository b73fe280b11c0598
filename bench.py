"""Benchmark of the B200 attention hot path: KV write, paged decode, chunked prefill.

Contract: ``python bench.py --gpus N --steps K --warmup W`` prints ONE JSON line.
For N > 1 it runs under torchrun, one process per GPU; the work is sharded by
request with no collective on the data path (every rank owns its own KV pool
and sequences).  NCCL carries only the timing barriers and the gathers of the
per-rank timings.

The line's headline (``value``) is the decode step: bf16, B=256 sequences per
GPU, 16 query heads / 8 KV heads, head_dim 128, 16-token pages, kv_len
U[512,4096], random non-contiguous block tables over a 1.2x pool.  One step =
the slot-mapped write of one new token per sequence (store_kvcache) + decode
attention over the paged KV (split-KV kernel + split combine).  ``value`` is the
step's algorithmic HBM bytes (K/V read once per kv head, q, out, tables, and the
store's rows + slots) / step time, summed over ranks (``scaling`` "weak").

The same line carries one block per further workload of the north star, each
with its own timing, roofline, clocks and (where the op returns a result)
end-to-end figure through the public ops with host buffers:

* ``prefill_config3``: varlen chunked prefill, 64 sequences per GPU, chunks
  U[128,2048] over cached prefixes U[0,8192] (TFLOP/s, tensor roofline);
  beside it the reference's own default prefill (its Triton kernel, through the
  reference's ``femtovllm.ops``) on the same inputs when the reference is
  installed under ``baseline/_ref``;
* ``mixed_config4``: 24 decode + 8 prefill requests sharing a 4096-token prefix,
  one launch;
* ``long_config5``: 64 sequences of U[32768,131072] tokens in total, split over
  the ranks longest-first (strong scaling: tokens/s and GB/s over all ranks);
* ``store_65k``: store_kvcache of 65,536 tokens; ``qk_norm_rope_config3``: the
  fused q/k RMSNorm + rotary + KV write over config 3's new tokens.

Timing: W warm-up steps, then blocks of exactly K steps, each between two CUDA
events on the launch stream.  The first block is the contract's timed region
(``ms_per_step``); blocks repeat until ``--min-seconds`` have passed so that the
nvidia-smi sampler sees the load, and their median is reported as
``sustained_ms_per_step`` (the power cap acts on long tensor-core loops).

``--impl reference`` times the reference's PyTorch attention path on the host
cores instead (its own ``forward_varlen_pytorch`` when the reference is
installed, else the ``oracle/`` restatement), on a bounded sample of the
default workload.  ``--workload`` runs one workload alone (development).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "nano-vllm-practice_b200"))
sys.path.insert(0, str(REPO))

METRIC = "paged decode attn HBM GB/s (% peak); chunked-prefill attn TFLOP/s; tok/s"
REF_DIR = REPO / "baseline" / "_ref"


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _sustained_tflops():
    """cuBLAS bf16 throughput held for seconds under the power cap (the denominator for a kernel
    timed over a long back-to-back loop)."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        v = json.loads(p.read_text()).get("bf16_tflops_sustained")
        return float(v) if v else None
    return 1400.0


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers GPUs physically; address this process's device by UUID.
        try:
            import torch

            self.gpu_index = f"GPU-{torch.cuda.get_device_properties(gpu_index).uuid}"
        except Exception:
            self.gpu_index = str(gpu_index)
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"fvb_clocks_{os.getpid()}_{id(self)}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": float(max(power))}


def _profile_traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(kernel_key)
    return None


def _reference_installed() -> bool:
    return (REF_DIR / "femtovllm" / "__init__.py").exists()


# ---------------------------------------------------------------------------
# CPU baseline: the reference's PyTorch attention path on the host cores
# ---------------------------------------------------------------------------


def _decode_step_bytes(batch, seqs=None) -> int:
    import torch

    es = torch.finfo(batch.dtype).bits // 8
    lens = batch.kv_lens if seqs is None else batch.kv_lens[seqs]
    n = len(lens)
    kv = 2 * int(lens.astype(np.int64).sum()) * batch.n_kv_heads * batch.head_dim * es
    qo = 2 * n * batch.n_heads * batch.head_dim * es
    tables = 4 * int(((lens + 15) // 16).sum()) + 4 * n
    store = 2 * 2 * n * batch.n_kv_heads * batch.head_dim * es + 8 * n
    return kv + qo + tables + store


def _cpu_sample(n_seqs: int, dtype):
    """A bounded sample of config 2 (the sampled sequences' lengths, heads and scale), drawn on the host."""
    import torch

    from femtovllm_b200 import workloads

    full = workloads.config2(seed=2)
    rng = np.random.default_rng(0)
    seqs = sorted(rng.choice(full.num_seqs, size=min(n_seqs, full.num_seqs), replace=False).tolist())
    small = workloads.custom(full.kv_lens[seqs], np.ones(len(seqs)), full.n_heads, full.n_kv_heads, full.head_dim,
                             dtype, seed=2, pool_factor=1.2, qkv_scale=full.qkv_scale)
    small.materialize("cpu")
    return small, full.num_seqs


def _time_cpu(fn, steps: int, warmup: int):
    for _ in range(warmup):
        fn()
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        t.append(time.perf_counter() - t0)
    return float(np.median(t))


def _port_step_fn(small):
    """The oracle restatement (numpy, fp32) of the write loop + decode attention."""
    import oracle
    from femtovllm_b200 import workloads

    sub = workloads.subset_for_oracle(small, list(range(small.num_seqs)))
    sub["k_new"] = small.k_new.float().numpy()
    sub["v_new"] = small.v_new.float().numpy()

    def step():
        kp, vp = sub["k_pool"], sub["v_pool"]
        slots = oracle.build_slot_mapping(sub["positions"], np.arange(len(sub["kv_lens"])), sub["block_tables"])
        oracle.store_kvcache(sub["k_new"], sub["v_new"], kp, vp, slots)
        oracle.decode_attention(sub["q"], kp, vp, sub["block_tables"], sub["kv_lens"], acc_dtype=np.float32)

    return step


def _reference_step_fn(small):
    """The reference's own QwenSelfAttention.forward_varlen_pytorch (femtovllm/models/qwen/qwen3.py:389-544:
    its KV write loop, page gather, GQA replication and SDPA) on the host, in the sample's dtype."""
    import torch

    from oracle import reference_module

    attn = reference_module.attention_module(small.n_heads, small.n_kv_heads, small.head_dim)
    md = reference_module.metadata(small.kv_lens, small.q_lens, small.block_tables, "cpu")
    x = reference_module.packed_input(small.q, small.k_new, small.v_new)
    kp, vp = small.k_pool, small.v_pool

    def step():
        with torch.no_grad():
            attn.forward_varlen_pytorch(x, kp, vp, md)

    return step


def cpu_baseline(n_seqs: int, steps: int = 3, warmup: int = 1) -> dict:
    """The CPU figure reported beside the GPU arm (config-2 sample, same GB/s formula).

    With the reference installed (``baseline/_ref``) the headline is its own PyTorch path in fp32
    (``kind: reference``) with a bf16 leg beside it; the numpy port is always timed as well."""
    import torch

    import contextlib

    threads = os.cpu_count() or 1
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    stack = contextlib.ExitStack()
    try:
        from threadpoolctl import threadpool_limits

        stack.enter_context(threadpool_limits(limits=threads))  # numpy's BLAS on every core too
    except Exception:
        pass
    try:
        small32, total = _cpu_sample(n_seqs, torch.float32)
        nbytes32 = _decode_step_bytes(small32)
        port_s = _time_cpu(_port_step_fn(small32), steps, warmup)
        out = {"port": {"value": round(nbytes32 / port_s / 1e9, 4), "unit": "GB/s", "ms_per_step": round(port_s * 1e3, 2),
                        "dtype": "f32", "what": "numpy restatement (oracle/) of qwen3.py:240-264 + 430-542"}}
        ref_err = None
        if _reference_installed():
            try:
                ref32_s = _time_cpu(_reference_step_fn(small32), steps, warmup)
                small16, _ = _cpu_sample(n_seqs, torch.bfloat16)
                ref16_s = _time_cpu(_reference_step_fn(small16), steps, warmup)
                nbytes16 = _decode_step_bytes(small16)
                out.update({
                    "value": round(nbytes32 / ref32_s / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "reference",
                    "ms_per_step": round(ref32_s * 1e3, 2),
                    "sample": f"{small32.num_seqs} of {total} config-2 sequences per step: the reference's own "
                              f"QwenSelfAttention.forward_varlen_pytorch (KV write loop + page gather + SDPA, "
                              f"qwen3.py:389-544) in fp32 on {threads} threads, median of {steps} steps "
                              f"({ref32_s * 1e3:.1f} ms/step)",
                    "bf16": {"value": round(nbytes16 / ref16_s / 1e9, 4), "unit": "GB/s",
                             "ms_per_step": round(ref16_s * 1e3, 2)},
                })
            except Exception as e:  # the reference's own code failed here: report the port instead
                ref_err = f"{type(e).__name__}: {e}"[:200]
        if "value" not in out:
            out.update({"value": out["port"]["value"], "unit": "GB/s", "cores": threads, "kind": "port",
                        "ms_per_step": out["port"]["ms_per_step"],
                        "sample": f"{small32.num_seqs} of {total} config-2 sequences per step (store + decode), "
                                  f"fp32 numpy restatement on {threads} threads, median of {steps} steps "
                                  f"({port_s * 1e3:.1f} ms/step)"})
            if ref_err:
                out["reference_error"] = ref_err
        out["host_cpu_count"] = threads
        out["torch_threads"] = torch.get_num_threads()
        return out
    finally:
        torch.set_num_threads(old)
        stack.close()


# ---------------------------------------------------------------------------
# GPU arm: timing helpers
# ---------------------------------------------------------------------------


class Ctx:
    """Per-process state shared by the workload blocks."""

    def __init__(self, args, rank, world, local_rank):
        import torch

        self.args, self.rank, self.world, self.local_rank = args, rank, world, local_rank
        self.dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(self.dev)
        self.hbm_peak, self.tflops_peak, self.peak_src = _peaks()
        self.tflops_sustained = _sustained_tflops()

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def gather(self, obj):
        if self.world == 1:
            return [obj]
        import torch.distributed as dist

        out = [None] * self.world
        dist.all_gather_object(out, obj)
        return out

    def timed(self, fn, steps=None, min_s=None, clocks=True):
        """W warm-up calls, then blocks of exactly K calls between CUDA events on the current stream,
        repeated until min_s seconds have passed.  Returns (first block ms/call, median ms/call,
        blocks, clock summary)."""
        import torch

        steps = steps or self.args.steps
        min_s = self.args.min_seconds if min_s is None else min_s
        for _ in range(self.args.warmup):
            fn()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        times = []
        sampler = ClockSampler(self.local_rank) if clocks else None
        if sampler:
            sampler.__enter__()
        try:
            t_start = time.perf_counter()
            while True:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(steps):
                    fn()
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b) / steps)
                if time.perf_counter() - t_start >= min_s or len(times) >= 100000:
                    break
        finally:
            if sampler:
                sampler.__exit__(None, None, None)
        torch.cuda.synchronize()
        self.barrier()
        return times[0], float(np.median(times)), len(times), (sampler.summary() if sampler else None)


class HostPipeline:
    """End-to-end steps from pinned host memory: every step's inputs cross PCIe as one staging copy
    into one of two device buffers (each input a fixed view of it), the op runs on the compute
    stream, and its output is copied back into one of two pinned host buffers.  The copies run on
    their own streams, so step i+1's inputs arrive while step i computes and step i's output returns
    while step i+1 computes; every copy of every timed step lies inside the timed region (the
    compute stream waits for the last read-back before the end event)."""

    def __init__(self, dev, srcs, out_shape, out_dtype):
        import torch

        self.dev = dev
        self.srcs = srcs
        offs, total = [], 0
        for t in srcs:
            offs.append(total)
            total += -(-t.numel() * t.element_size() // 256) * 256
        self.offs, self.total = offs, total
        self.h_flat = torch.empty(total, dtype=torch.uint8).pin_memory()
        for hv, t in zip(self._views(self.h_flat), srcs):
            hv.copy_(t.cpu())
        self.d_flat = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]
        self.dbuf = [self._views(f) for f in self.d_flat]
        self.h_outs = [torch.empty(out_shape, dtype=out_dtype).pin_memory() for _ in range(2)]
        self.h2d_s, self.d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_used = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]
        self.h2d_bytes = total
        self.d2h_bytes = self.h_outs[0].numel() * self.h_outs[0].element_size()

    def _views(self, flat):
        return [flat[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                for o, t in zip(self.offs, self.srcs)]

    def _copy_in(self, i):
        import torch

        b = i % 2
        with torch.cuda.stream(self.h2d_s):
            self.h2d_s.wait_event(self.ev_used[b])  # step i-2 is done reading this buffer
            self.d_flat[b].copy_(self.h_flat, non_blocking=True)
            self.ev_in[b].record(self.h2d_s)

    def run(self, n, compute):
        import torch

        stream = torch.cuda.current_stream()
        self._copy_in(0)
        for i in range(n):
            b = i % 2
            stream.wait_event(self.ev_in[b])
            out = compute(self.dbuf[b])
            self.ev_used[b].record(stream)
            if i + 1 < n:
                self._copy_in(i + 1)
            with torch.cuda.stream(self.d2h_s):
                self.d2h_s.wait_event(self.ev_used[b])
                self.d2h_s.wait_event(self.ev_out[b])  # the read-back of step i-2 into the same host buffer
                self.h_outs[b].copy_(out, non_blocking=True)
                out.record_stream(self.d2h_s)
                self.ev_out[b].record(self.d2h_s)
        stream.wait_stream(self.d2h_s)

    def timed(self, ctx, compute, min_s=0.5):
        """(first block ms/step, median ms/step) over blocks of K end-to-end steps."""
        import torch

        self.run(ctx.args.warmup, compute)
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        times = []
        t_start = time.perf_counter()
        while True:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            self.run(ctx.args.steps, compute)
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b) / ctx.args.steps)
            if time.perf_counter() - t_start >= min_s:
                break
        torch.cuda.synchronize()
        ctx.barrier()
        return times[0], float(np.median(times))


def _free():
    import gc

    import torch

    gc.collect()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# GPU arm: workload blocks (each returns this rank's figures; rank 0 aggregates)
# ---------------------------------------------------------------------------


def block_decode_config2(ctx):
    """The contract step: store_kvcache of 1 token per sequence + decode attention (config 2)."""
    from femtovllm_b200 import capi, ops, workloads

    batch = workloads.config2(seed=2 + ctx.rank, num_seqs=ctx.args.num_seqs).materialize(ctx.dev)
    md = batch.device_metadata(ctx.dev)
    q, kp, vp = batch.q, batch.k_pool, batch.v_pool
    tables, lens, slots = md["block_tables"], md["kv_lens"], md["slot_mapping"]
    max_kv = batch.max_kv_len

    def step():
        ops.store_kvcache(batch.k_new, batch.v_new, kp, vp, slots)
        return ops.paged_attention_gemv(q, kp, vp, tables, lens, max_kv)

    first, med, blocks, clocks = ctx.timed(step)
    dec_first, dec_med, _, _ = ctx.timed(lambda: ops.paged_attention_gemv(q, kp, vp, tables, lens, max_kv),
                                         min_s=0.3, clocks=False)
    st_first, _, _, _ = ctx.timed(lambda: ops.store_kvcache(batch.k_new, batch.v_new, kp, vp, slots), min_s=0.1,
                                  clocks=False)

    pipe = HostPipeline(ctx.dev, (q, batch.k_new, batch.v_new, tables, lens, slots), q.shape, q.dtype)

    def e2e_step(v):
        dq, dk, dv, dt, dl, ds = v
        ops.store_kvcache(dk, dv, kp, vp, ds)
        return ops.paged_attention_gemv(dq, kp, vp, dt, dl, max_kv)

    e2e_first, e2e_med = pipe.timed(ctx, e2e_step)
    lib = capi.load()
    plan_ws = lib.fvb_paged_attention_decode_workspace_size(batch.num_seqs, batch.n_heads, batch.n_kv_heads,
                                                            batch.head_dim, max_kv)
    return {"step_ms": first, "step_ms_median": med, "blocks": blocks, "decode_ms": dec_first,
            "decode_ms_median": dec_med, "store_ms": st_first, "e2e_ms": e2e_first, "e2e_ms_median": e2e_med,
            "bytes": _decode_step_bytes(batch), "decode_bytes": batch.decode_bytes(), "tokens": batch.num_seqs,
            "clocks": clocks, "h2d": pipe.h2d_bytes, "d2h": pipe.d2h_bytes,
            "launches_per_step": 2 + (1 if plan_ws > 0 else 0), "num_blocks": batch.num_blocks}


def _reference_ops():
    """The reference's femtovllm.ops (from baseline/_ref) with this repository's extension as its
    femtovllm._C, or None.  Imported here rather than from oracle/: it is timed on the GPU."""
    if not _reference_installed():
        return None
    from femtovllm_b200 import _C as this_extension

    sys.modules.setdefault("femtovllm._C", this_extension)
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import femtovllm.ops
    from femtovllm.protocol import ImplCustomKernel

    return femtovllm.ops, ImplCustomKernel


def _q_tiles(q_lens, tile=32):
    """The reference Triton prefill's tile metadata (model_runner.py:174-202): cu_q_tiles, q_tile_to_seq_idx."""
    n = (np.asarray(q_lens, np.int64) + tile - 1) // tile
    cu = np.concatenate([[0], np.cumsum(n)]).astype(np.int32)
    seq = np.repeat(np.arange(len(n)), n).astype(np.int32)
    return cu, seq


def _prefill_like_block(ctx, batch, key, with_reference_triton):
    """Chunked prefill (or a mixed batch) in one launch of paged_attention_gemm."""
    import torch

    from femtovllm_b200 import ops

    batch.materialize(ctx.dev)
    md = batch.device_metadata(ctx.dev)
    cu, tab, lens, pos = md["cu_seqlens"], md["block_tables"], md["kv_lens"], md["positions"]

    def call(q, c=cu, t=tab, kl=lens, p=pos):
        return ops.paged_attention_gemm(q, batch.k_pool, batch.v_pool, c, batch.max_q_len, 32, None, None, t, kl, p)

    first, med, blocks, clocks = ctx.timed(lambda: call(batch.q))
    pipe = HostPipeline(ctx.dev, (batch.q, cu, tab, lens, pos), batch.q.shape, batch.q.dtype)
    e2e_first, e2e_med = pipe.timed(ctx, lambda v: call(v[0], v[1], v[2], v[3], v[4]))
    res = {"ms": first, "ms_median": med, "blocks": blocks, "clocks": clocks, "flops": batch.attn_flops(),
           "kv_bytes": batch.kv_bytes(), "kv_bytes_unique": batch.unique_kv_bytes(), "tokens": batch.num_tokens, "e2e_ms": e2e_first, "e2e_ms_median": e2e_med,
           "h2d": pipe.h2d_bytes, "d2h": pipe.d2h_bytes, "name": batch.name}
    del pipe
    if with_reference_triton:
        try:
            ref = _reference_ops()
        except Exception as e:
            ref = None
            res["reference_triton"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
        if ref is None and "reference_triton" not in res:
            res["reference_triton"] = {"unavailable": "the reference is not installed under baseline/_ref"}
        if ref is not None:
            rops, Impl = ref
            cu_t, seq_t = _q_tiles(batch.q_lens)
            cu_t, seq_t = torch.from_numpy(cu_t).to(ctx.dev), torch.from_numpy(seq_t).to(ctx.dev)

            def via_ref(impl):
                return rops.paged_attention_gemm(batch.q, batch.k_pool, batch.v_pool, cu, batch.max_q_len, 32, cu_t,
                                                 seq_t, tab, lens, pos, impl=impl)

            try:
                t_first, t_med, _, _ = ctx.timed(lambda: via_ref(Impl.TRITON), min_s=0.0, clocks=False)
                o_first, _, _, _ = ctx.timed(lambda: via_ref(Impl.CUDA), min_s=0.0, clocks=False)
                diff = (via_ref(Impl.TRITON).float() - call(batch.q).float()).abs()
                res["reference_triton"] = {
                    "ms": t_first, "ms_median": t_med, "this_via_reference_ops_ms": o_first,
                    "max_abs_diff_vs_this": float(diff.max()), "mean_abs_diff_vs_this": float(diff.mean())}
            except Exception as e:
                res["reference_triton"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    return res


def block_prefill_config3(ctx):
    from femtovllm_b200 import workloads

    # The reference's Triton prefill is timed at N = 1 only (its import could fail on one rank
    # alone, and every rank takes the same barriers).
    return _prefill_like_block(ctx, workloads.config3(seed=3 + ctx.rank), "prefill_config3",
                               with_reference_triton=ctx.world == 1 and not ctx.args.no_reference_gpu)


def block_mixed_config4(ctx):
    from femtovllm_b200 import workloads

    return _prefill_like_block(ctx, workloads.config4(seed=4 + ctx.rank), "mixed_config4",
                               with_reference_triton=False)


def block_long_config5(ctx):
    """Config 5's 64 sequences split longest-first over the ranks (strong scaling)."""
    from femtovllm_b200 import ops, workloads

    b = workloads.config5(rank=ctx.rank, world=ctx.world, total=ctx.args.long_total).materialize(ctx.dev)
    md = b.device_metadata(ctx.dev)
    tab, lens = md["block_tables"], md["kv_lens"]

    def call(q, t=tab, kl=lens):
        return ops.paged_attention_gemv(q, b.k_pool, b.v_pool, t, kl, b.max_kv_len)

    first, med, blocks, clocks = ctx.timed(lambda: call(b.q))
    pipe = HostPipeline(ctx.dev, (b.q, tab, lens), b.q.shape, b.q.dtype)
    e2e_first, e2e_med = pipe.timed(ctx, lambda v: call(v[0], v[1], v[2]))
    return {"ms": first, "ms_median": med, "blocks": blocks, "clocks": clocks, "bytes": b.decode_bytes(),
            "tokens": b.num_seqs, "e2e_ms": e2e_first, "e2e_ms_median": e2e_med, "h2d": pipe.h2d_bytes,
            "d2h": pipe.d2h_bytes, "kv_tokens": int(b.kv_lens.astype(np.int64).sum())}


def block_store_65k(ctx):
    """store_kvcache alone at prefill size: 65,536 new tokens of config 2's heads (Hkv 8, D 128, bf16)
    scattered through a random slot permutation into a pool with room for 131,072 tokens (> L2)."""
    import torch

    from femtovllm_b200 import ops

    T, hkv, D = 65536, 8, 128
    g = torch.Generator(device=ctx.dev).manual_seed(11 + ctx.rank)
    k = torch.randn(T, hkv, D, generator=g, device=ctx.dev).to(torch.bfloat16)
    v = torch.randn(T, hkv, D, generator=g, device=ctx.dev).to(torch.bfloat16)
    blocks_ = (2 * T + 15) // 16
    k_pool = torch.zeros(blocks_, hkv, 16, D, device=ctx.dev, dtype=torch.bfloat16)
    v_pool = torch.zeros_like(k_pool)
    rng = np.random.default_rng(11 + ctx.rank)
    slots = torch.from_numpy(rng.permutation(blocks_ * 16)[:T].astype(np.int64)).to(ctx.dev)
    first, med, blocks, clocks = ctx.timed(lambda: ops.store_kvcache(k, v, k_pool, v_pool, slots), min_s=1.0)
    return {"ms": first, "ms_median": med, "blocks": blocks, "clocks": clocks,
            "bytes": 2 * 2 * T * hkv * D * 2 + 8 * T, "tokens": T}


def block_qk_norm_rope_config3(ctx):
    """The fused q/k RMSNorm + rotary + KV write over config 3's new tokens, read from the projection
    output (T, (Hq + 2 Hkv) D) in place."""
    import torch

    from femtovllm_b200 import ops, workloads

    batch = workloads.config3(seed=3 + ctx.rank)
    T, Hq, Hkv, D = batch.num_tokens, batch.n_heads, batch.n_kv_heads, batch.head_dim
    dev = ctx.dev
    g = torch.Generator(device=dev).manual_seed(7 + ctx.rank)
    x = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g, device=dev).to(batch.dtype)
    qv = x[:, : Hq * D].view(T, Hq, D)
    kv = x[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D)
    vv = x[:, (Hq + Hkv) * D :].view(T, Hkv, D)
    q_w = (1 + 0.25 * torch.randn(D, generator=g, device=dev)).to(batch.dtype)
    k_w = (1 + 0.25 * torch.randn(D, generator=g, device=dev)).to(batch.dtype)
    rows = int(batch.kv_lens.max())
    inv = 1e-6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
    theta = torch.arange(rows, device=dev, dtype=torch.float32)[:, None] * inv[None]
    theta = torch.cat([theta, theta], -1)
    cos, sin = theta.cos().to(batch.dtype), theta.sin().to(batch.dtype)
    shape = (batch.num_blocks, Hkv, 16, D)
    k_pool = torch.empty(shape, device=dev, dtype=batch.dtype)
    v_pool = torch.empty(shape, device=dev, dtype=batch.dtype)
    md = batch.device_metadata(dev)
    pos, slots = md["positions"], md["slot_mapping"]

    def step():
        return ops.qk_norm_rope_store(qv, kv, vv, q_w, k_w, 1e-6, cos, sin, pos, k_pool, v_pool, slots)

    first, med, blocks, clocks = ctx.timed(step, min_s=1.0)
    es = x.element_size()
    return {"ms": first, "ms_median": med, "blocks": blocks, "clocks": clocks,
            "bytes": 2 * T * (Hq + 2 * Hkv) * D * es + 12 * T, "tokens": T}


# ---------------------------------------------------------------------------
# GPU arm: aggregation into the JSON line
# ---------------------------------------------------------------------------


def _r(x, n=5):
    return None if x is None else round(float(x), n)


def _e2e(g, key_units, unit, scale):
    """End-to-end figure: the median over blocks of K host-pipelined steps (the first block after the
    warm-up also carries the host's one-time costs; it is reported beside it)."""
    t = max(x["e2e_ms"] for x in g)
    tm = max(x["e2e_ms_median"] for x in g)
    units = sum(x[key_units] for x in g)
    return {"value": _r(units / (tm * 1e-3) / scale, 2), "unit": unit, "ms_per_step": _r(tm),
            "value_first_block": _r(units / (t * 1e-3) / scale, 2),
            "h2d_bytes_per_step": sum(x["h2d"] for x in g), "d2h_bytes_per_step": sum(x["d2h"] for x in g)}


def line_prefill(ctx, g, workload, config):
    t = max(x["ms"] for x in g)
    tm = max(x["ms_median"] for x in g)
    flops = sum(x["flops"] for x in g)
    tokens = sum(x["tokens"] for x in g)
    r0 = g[0]
    ach = r0["flops"] / (r0["ms"] * 1e-3) / 1e12
    ach_s = r0["flops"] / (r0["ms_median"] * 1e-3) / 1e12
    out = {
        "workload": workload, "config": config, "unit": "TFLOP/s",
        "value": _r(flops / (t * 1e-3) / 1e12, 2), "ms_per_step": _r(t),
        "sustained": {"value": _r(flops / (tm * 1e-3) / 1e12, 2), "ms_per_step": _r(tm),
                      "blocks": min(x["blocks"] for x in g)},
        "tokens_per_s": _r(tokens / (t * 1e-3), 1),
        "gbs_kv": _r(sum(x["kv_bytes"] for x in g) / (t * 1e-3) / 1e9, 1),
        "gbs_kv_unique": _r(sum(x["kv_bytes_unique"] for x in g) / (t * 1e-3) / 1e9, 1),
        "flops_per_step_per_gpu": r0["flops"],
        "roofline": {
            "kernel": ("prefill_plan_kernel + prefill_tc_kernel + decode_split_kernel + decode_combine_kernel (one "
                       "paged_attention_gemm call; the decode kernels take its single-token sequences)"),
            "bound": "tensor", "achieved": _r(ach, 1), "peak": ctx.tflops_peak, "unit": "TFLOP/s",
            "frac": _r(ach / ctx.tflops_peak, 4),
            "peak_source": f"{ctx.peak_src} burst (MEASURED_PEAKS.json bf16_tflops): the first block of K calls",
            "traffic": _profile_traffic(workload),
            "sustained": {"achieved": _r(ach_s, 1), "peak": ctx.tflops_sustained,
                          "frac": _r(ach_s / ctx.tflops_sustained, 4) if ctx.tflops_sustained else None,
                          "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained: median over the blocks"},
        },
        "e2e": _e2e(g, "flops", "TFLOP/s", 1e12),
        "clocks": g[0]["clocks"],
        # plan + tensor-core kernel + split-KV decode (single-token sequences; it exits at once when there are
        # none) + its combine (the workload's block tables span more than one split)
        "gpu_launches": 4 * ctx.args.steps,
    }
    out["e2e"]["api"] = ("femtovllm_b200.ops.paged_attention_gemm: q and the step metadata copied in from pinned "
                         "host memory, the output copied back, every step (the K/V pools stay resident)")
    if "reference_triton" in r0:
        rt = r0["reference_triton"]
        if "ms" in rt:
            rt = dict(rt)
            rt["tflops"] = _r(r0["flops"] / (rt["ms"] * 1e-3) / 1e12, 2)
            rt["this_over_reference"] = _r(rt["ms"] / r0["ms"], 2)
            rt["what"] = ("the reference's default prefill: femtovllm.ops.paged_attention_gemm(impl=TRITON) from "
                          "baseline/_ref (paged_attention_gemm.py:6-235) on the same device tensors; "
                          "this_via_reference_ops_ms = this repository's kernel through the same reference op "
                          "(impl=CUDA, its femtovllm._C replaced by this extension)")
        out["reference_gpu"] = rt
    return out


def run_contract(args, rank, world, local_rank, cpu):
    ctx = Ctx(args, rank, world, local_rank)
    only = set(args.blocks.split(",")) if args.blocks else None

    def want(name):
        return only is None or name in only

    d = None
    if only is None:
        d = ctx.gather(block_decode_config2(ctx))
        _free()
    blocks = {}
    if want("prefill_config3"):
        blocks["prefill_config3"] = ctx.gather(block_prefill_config3(ctx))
        _free()
    if want("mixed_config4"):
        blocks["mixed_config4"] = ctx.gather(block_mixed_config4(ctx))
        _free()
    if want("long_config5"):
        blocks["long_config5"] = ctx.gather(block_long_config5(ctx))
        _free()
    if want("store_65k"):
        blocks["store_65k"] = ctx.gather(block_store_65k(ctx))
        _free()
    if want("qk_norm_rope_config3"):
        blocks["qk_norm_rope_config3"] = ctx.gather(block_qk_norm_rope_config3(ctx))
        _free()
    if rank != 0:
        return None
    hbm = ctx.hbm_peak
    line = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup}
    if d is not None:
        line.update(_line_decode(ctx, d, cpu))
    _add_blocks(ctx, line, blocks)
    return line


def _line_decode(ctx, d, cpu):
    args, world, hbm = ctx.args, ctx.world, ctx.hbm_peak
    t_step = max(x["step_ms"] for x in d)
    t_med = max(x["step_ms_median"] for x in d)
    t_dec = d[0]["decode_ms"]
    total_bytes = sum(x["bytes"] for x in d)
    tokens = sum(x["tokens"] for x in d)
    value = total_bytes / (t_step * 1e-3) / 1e9
    achieved = d[0]["decode_bytes"] / (t_dec * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1)/sqrt(128) q/k/v, random non-contiguous block tables)",
        "config": {
            "workload": "config2: decode paged attention + 1-token store_kvcache per sequence",
            "num_seqs_per_gpu": args.num_seqs, "n_heads": 16, "n_kv_heads": 8, "head_dim": 128, "block_size": 16,
            "kv_len": "U[512,4096]", "pool_blocks_per_gpu": d[0]["num_blocks"],
            "parallelism": f"request-sharded x{world}, no collective",
            "l2": "inputs larger than L2 (K/V ~2.4 GB per GPU), no flush",
            "timing": f"first block of exactly {args.steps} steps after {args.warmup} warm-up steps (CUDA events on "
                      f"the launch stream, max over ranks); blocks repeated for {args.min_seconds} s "
                      "for the clock sampler, their median in sustained_ms_per_step",
        },
        "sustained_ms_per_step": round(t_med, 5),
        "tokens_per_s": round(tokens / (t_step * 1e-3), 1),
        "pct_hbm_peak": round(100 * value / (hbm * world), 2),
        "kernel_ms": {"decode_attention": round(t_dec, 5), "decode_attention_median": round(d[0]["decode_ms_median"], 5),
                      "store_kvcache": round(d[0]["store_ms"], 5)},
        "roofline": {
            "kernel": "decode attention (decode_split_kernel + decode_combine_kernel)",
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": hbm,
            "unit": "GB/s",
            "frac": round(achieved / hbm, 4),
            "peak_source": f"{ctx.peak_src} (MEASURED_PEAKS.json hbm_gbs)" if ctx.peak_src == "measured" else ctx.peak_src,
            "traffic": _profile_traffic("decode_config2"),
        },
        "cpu_baseline": cpu,
        "e2e": {
            "value": round(total_bytes / (max(x["e2e_ms_median"] for x in d) * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "ms_per_step": round(max(x["e2e_ms_median"] for x in d), 5),
            "value_first_block": round(total_bytes / (max(x["e2e_ms"] for x in d) * 1e-3) / 1e9, 2),
            "timing": "median over blocks of K end-to-end steps (>= 0.5 s), max over ranks",
            "h2d_bytes_per_step": sum(x["h2d"] for x in d),
            "d2h_bytes_per_step": sum(x["d2h"] for x in d),
            "api": "femtovllm_b200.ops.store_kvcache + paged_attention_gemv from pinned host buffers "
                   "(the step's inputs copied in as one staging copy and the output copied out every step, "
                   "on copy streams overlapping the neighbouring steps' compute)",
        },
        "gpu_launches": d[0]["launches_per_step"] * args.steps,
        "clocks": d[0]["clocks"],
        "clocks_per_rank": [x["clocks"] for x in d] if world > 1 else None,
    }
    return line


def _add_blocks(ctx, line, blocks):
    args, world, hbm = ctx.args, ctx.world, ctx.hbm_peak
    if "prefill_config3" in blocks:
        line["prefill_config3"] = line_prefill(
            ctx, blocks["prefill_config3"], "prefill_config3",
            {"seqs_per_gpu": 64, "n_heads": 16, "n_kv_heads": 8, "head_dim": 128, "chunk": "U[128,2048]",
             "cached_prefix": "U[0,8192]", "scaling": "weak (one config-3 batch per GPU)"})
    if "mixed_config4" in blocks:
        line["mixed_config4"] = line_prefill(
            ctx, blocks["mixed_config4"], "mixed_config4",
            {"requests_per_gpu": 32, "decode": 24, "prefill": "8 x 512-token chunks", "shared_prefix": 4096,
             "suffix": "U[64,1024]", "n_heads": 32, "n_kv_heads": 8, "head_dim": 128, "launches": "one call",
             "scaling": "weak"})
    if "long_config5" in blocks:
        g = blocks["long_config5"]
        t = max(x["ms"] for x in g)
        tm = max(x["ms_median"] for x in g)
        nbytes = sum(x["bytes"] for x in g)
        toks = sum(x["tokens"] for x in g)
        slow = max(range(world), key=lambda r: g[r]["ms"])
        ach = g[slow]["bytes"] / (g[slow]["ms"] * 1e-3) / 1e9
        line["long_config5"] = {
            "workload": "long_config5", "unit": "tokens/s",
            "config": {"total_seqs": args.long_total, "n_heads": 32, "n_kv_heads": 8, "head_dim": 128, "kv_len": "U[32768,131072]",
                       "sharding": f"longest-first over {world} rank(s), each with its own pool (strong scaling)",
                       "seqs_per_rank": [x["tokens"] for x in g], "kv_tokens_per_rank": [x["kv_tokens"] for x in g]},
            "value": _r(toks / (t * 1e-3), 1), "ms_per_step": _r(t),
            "gbs": _r(nbytes / (t * 1e-3) / 1e9, 1), "pct_hbm_peak_aggregate": _r(100 * nbytes / (t * 1e-3) / 1e9 / (hbm * world), 2),
            "sustained": {"value": _r(toks / (tm * 1e-3), 1), "ms_per_step": _r(tm), "gbs": _r(nbytes / (tm * 1e-3) / 1e9, 1)},
            "ms_per_rank": [_r(x["ms"]) for x in g],
            "roofline": {"kernel": "decode attention on the slowest rank (decode_split_kernel + decode_combine_kernel)",
                         "bound": "hbm", "achieved": _r(ach, 1), "peak": hbm, "unit": "GB/s", "frac": _r(ach / hbm, 4),
                         "traffic": _profile_traffic("long_config5")},
            "e2e": _e2e(g, "tokens", "tokens/s", 1.0),
            "clocks": g[0]["clocks"],
            "gpu_launches": 2 * args.steps,
        }
    if "store_65k" in blocks:
        g = blocks["store_65k"]
        t = max(x["ms"] for x in g)
        ach = g[0]["bytes"] / (g[0]["ms"] * 1e-3) / 1e9
        line["store_65k"] = {
            "workload": "store_kvcache of 65,536 tokens per GPU (Hkv 8, D 128, bf16, random slots)", "unit": "GB/s",
            "value": _r(sum(x["bytes"] for x in g) / (t * 1e-3) / 1e9, 1), "ms_per_step": _r(t),
            "sustained_ms_per_step": _r(max(x["ms_median"] for x in g)),
            "roofline": {"kernel": "store_kvcache_bulk_kernel", "bound": "hbm", "achieved": _r(ach, 1), "peak": hbm,
                         "unit": "GB/s", "frac": _r(ach / hbm, 4), "traffic": _profile_traffic("store_65k")},
            "clocks": g[0]["clocks"], "gpu_launches": args.steps,
        }
    if "qk_norm_rope_config3" in blocks:
        g = blocks["qk_norm_rope_config3"]
        t = max(x["ms"] for x in g)
        ach = g[0]["bytes"] / (g[0]["ms"] * 1e-3) / 1e9
        line["qk_norm_rope_config3"] = {
            "workload": "qk_norm_rope_store over config 3's new tokens per GPU", "unit": "GB/s",
            "tokens_per_gpu": g[0]["tokens"],
            "value": _r(sum(x["bytes"] for x in g) / (t * 1e-3) / 1e9, 1), "ms_per_step": _r(t),
            "sustained_ms_per_step": _r(max(x["ms_median"] for x in g)),
            "roofline": {"kernel": "qk_norm_rope_ws_kernel", "bound": "hbm", "achieved": _r(ach, 1), "peak": hbm,
                         "unit": "GB/s", "frac": _r(ach / hbm, 4), "traffic": _profile_traffic("qk_norm_rope_config3")},
            "clocks": g[0]["clocks"], "gpu_launches": args.steps,
        }


# ---------------------------------------------------------------------------
# development workloads (one block alone, or the graph / sampler measurements)
# ---------------------------------------------------------------------------


def _reference_sampler_ops(logits, temps, pens, table):
    """The tensor ops of the reference's Sampler.forward (femtovllm/engine/sampler.py:56-109) for a
    batch whose rows all sample with a presence penalty, restated with torch on the same device
    tensors: (B, vocab + 1) count matrix by scatter_add, penalty, in-place division, softmax,
    multinomial.  Timed beside the fused kernel; its host list building is not included."""
    import torch

    B, V = logits.shape
    counts = torch.zeros((B, V + 1), dtype=torch.long, device=logits.device)
    counts.scatter_add_(dim=1, index=table, src=torch.ones_like(table))
    x = logits - pens[:, None] * (counts[:, :V] > 0)
    x /= temps[:, None]
    return torch.multinomial(torch.softmax(x, dim=-1), num_samples=1).squeeze(-1)


def run_sampler(args, rank, local_rank, hbm_peak, peak_src):
    """Next-token sampling of a decode batch: B = 256 rows (config 2's batch) of Qwen3's 151,936-entry
    vocabulary in bf16, the reference's default SamplingParams (temperature 1.0, presence penalty 1.0)
    and token histories of config 2's context lengths U[512, 4096].  Four logits buffers are rotated
    (311 MB > L2).  Algorithmic bytes: the logits once, the token tables once, ids written."""
    import torch

    from femtovllm_b200 import ops

    if rank != 0:
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B = args.num_seqs
    V = 151936
    g = torch.Generator(device=dev).manual_seed(21)
    bufs = [(torch.randn(B, V, generator=g, device=dev) * 3).to(torch.bfloat16) for _ in range(4)]
    rng = np.random.default_rng(21)
    lens = rng.integers(512, 4097, B)
    table_h = np.full((B, int(lens.max())), V, np.int64)
    for b in range(B):
        table_h[b, : lens[b]] = rng.integers(0, V, lens[b])
    table = torch.from_numpy(table_h).to(dev)
    temps = torch.ones(B, device=dev)
    pens = torch.ones(B, device=dev)
    state = ops.new_rng_state(7, dev)
    ws = ops.sample_workspace(B, V, dev)
    steps = min(args.steps, 200)

    def timed(fn):
        for i in range(max(args.warmup, 3)):
            fn(bufs[i % 4])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(bufs[i % 4])
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    with ClockSampler(local_rank) as clk:
        ms = timed(lambda lg: ops.sample_tokens(lg, temps, pens, table, state, ws))
    ms_ref = timed(lambda lg: _reference_sampler_ops(lg, temps, pens, table))
    nbytes = B * V * 2 + int(table.numel()) * 8 + B * (4 + 4 + 8)
    line = {"metric": "sampler GB/s", "workload": "sampler", "rows": B, "vocab": V, "dtype": "bf16",
            "table_len": int(table.shape[1]), "steps": steps, "ms_per_step": round(ms, 5),
            "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "pct_hbm_peak": round(100 * nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 2), "peak_source": peak_src,
            "reference_ops_ms_per_step": round(ms_ref, 5), "speedup_vs_reference_ops": round(ms_ref / ms, 2),
            "data": "synthetic (seeded N(0, 9) bf16 logits, uniform token histories)", "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def run_decode_graph(args, rank, local_rank):
    """Per-step latency of a small-batch decode step (config 2's heads, context U[512,4096]):
    slot mapping + fused q/k norm / rotary / KV write + split-KV attention, launched eagerly
    through femtovllm_b200.ops versus replayed from one captured CUDA graph."""
    import torch

    from femtovllm_b200 import ops, workloads

    if rank != 0:
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B = args.num_seqs if args.num_seqs != 256 else 8
    b = workloads.config2(num_seqs=B).materialize(dev)
    md = b.device_metadata(dev)
    T, Hq, Hkv, D = B, b.n_heads, b.n_kv_heads, b.head_dim
    x = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).to(b.dtype)
    qv, kv, vv = x[:, : Hq * D].view(T, Hq, D), x[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D), x[:, (Hq + Hkv) * D :].view(T, Hkv, D)
    w = torch.ones(D, device=dev, dtype=b.dtype)
    rows = int(b.kv_lens.max()) + 1
    inv = 1e-6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
    th = torch.arange(rows, device=dev, dtype=torch.float32)[:, None] * inv[None]
    th = torch.cat([th, th], -1)
    cos, sin = th.cos().to(b.dtype), th.sin().to(b.dtype)
    pos = (md["kv_lens"] - 1).contiguous()

    def step():
        slots = ops.build_slot_mapping(pos, md["block_tables"])
        q_hm = ops.qk_norm_rope_store(qv, kv, vv, w, w, 1e-6, cos, sin, pos, b.k_pool, b.v_pool, slots)
        return ops.paged_attention_gemv(q_hm, b.k_pool, b.v_pool, md["block_tables"], md["kv_lens"], b.max_kv_len)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps * 1e3

    eager_us = timed(step)
    graph_us = timed(g.replay)
    del g
    line = {"metric": "decode step latency (us), eager vs CUDA graph", "workload": "decode_graph", "num_seqs": B,
            "n_heads": Hq, "n_kv_heads": Hkv, "head_dim": D, "kv_len": "U[512,4096]", "steps": args.steps,
            "eager_us": round(eager_us, 2), "graph_us": round(graph_us, 2),
            "speedup": round(eager_us / graph_us, 2), "kv_bytes": int(b.decode_bytes()),
            "graph_gbs": round(b.decode_bytes() / (graph_us * 1e-6) / 1e9, 1),
            "launches_per_step": 4, "data": "synthetic (seeded)"}
    print(json.dumps(line), flush=True)


def run_reference_arm(args, rank: int, world: int):
    """The reference's PyTorch attention path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    cpu = cpu_baseline(args.cpu_seqs, steps=args.steps, warmup=args.warmup)
    value = cpu["value"]
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": cpu["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16-valued inputs); bf16 leg in cpu_baseline.bf16" if cpu["kind"] == "reference"
        else "f32 (bf16-valued inputs)",
        "data": "synthetic",
        "config": {"workload": "config2: decode paged attention + 1-token store_kvcache per sequence (sampled)"},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seqs", type=int, default=24)
    ap.add_argument("--num-seqs", type=int, default=256, help="decode sequences per GPU (256 = config 2)")
    ap.add_argument("--min-seconds", type=float, default=1.5,
                    help="repeat each workload's K-step block until this many seconds have passed")
    ap.add_argument("--blocks", default="",
                    help="comma list of the extra blocks to run (default all): prefill_config3, mixed_config4, "
                         "long_config5, store_65k, qk_norm_rope_config3")
    ap.add_argument("--workload", default="all",
                    choices=["all", "prefill", "mixed", "long", "store", "qk_norm_rope", "decode_graph", "sampler"],
                    help="all = the contract line (config 2 + every block); the others run one measurement alone")
    ap.add_argument("--long-total", type=int, default=64,
                    help="config 5's total sequences over all ranks (64; fewer only for profiling captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true", help="skip the reference Triton prefill timing")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    # The CPU baseline runs before any GPU work and before the process group exists, so it
    # overlaps nothing (the other ranks wait in the rendezvous).
    cpu = None
    if rank == 0 and args.workload == "all" and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seqs)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "decode_graph":
            run_decode_graph(args, rank, local_rank)
        elif args.workload == "sampler":
            hbm, _, src = _peaks()
            run_sampler(args, rank, local_rank, hbm, src)
        elif args.workload == "all":
            line = run_contract(args, rank, world, local_rank, cpu)
            if rank == 0:
                print(json.dumps(line), flush=True)
        else:
            one = {"prefill": "prefill_config3", "mixed": "mixed_config4", "long": "long_config5",
                   "store": "store_65k", "qk_norm_rope": "qk_norm_rope_config3"}[args.workload]
            args.blocks = one
            line = run_contract(args, rank, world, local_rank, None)
            if rank == 0:
                print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
