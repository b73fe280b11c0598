"""Benchmark of the B200 attention hot path (KV write + paged decode attention).

Contract: ``python bench.py --gpus N --steps K --warmup W`` prints ONE JSON line.
For N > 1 it runs under torchrun, one process per GPU; the work is sharded by
request with no collective on the data path (every rank owns its own KV pool
and sequences), so ``scaling`` is "weak" and ``value`` aggregates all ranks.

Default workload: decode, bf16, B=256 sequences per GPU,
16 query heads / 8 KV heads, head_dim 128, 16-token pages, kv_len U[512,4096],
random non-contiguous block tables over a 1.2x pool.  One step = the slot-mapped
write of one new token per sequence (store_kvcache) + decode attention over the
paged KV (split-KV kernel + split combine).  ``value`` is the step's
algorithmic HBM bytes (K/V read once per kv head, q, out, tables, and the
store's rows + slots) / step time.

``--impl reference`` times the reference's CPU attention path (the oracle
restatement, ``oracle/``) on the host cores instead, on a bounded sample of
the same workload, and prints the same metric.  ``--workload`` selects other
configurations for development measurements (prefill, mixed, long).
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


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _sustained_tflops():
    """cuBLAS bf16 throughput held for seconds under the power cap (the denominator for a kernel
    timed over a long back-to-back loop, as the prefill workloads are); None without the file."""
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
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"fvb_clocks_{os.getpid()}.csv"

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
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
                "samples": len(sm)}


def _profile_traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(kernel_key)
    return None


# ---------------------------------------------------------------------------
# CPU baseline: the reference attention path restated (oracle), on host cores
# ---------------------------------------------------------------------------


def cpu_decode_sample(batch, n_seqs: int, seed: int = 0):
    """A bounded sample of a decode batch, copied to numpy fp32 (pages renumbered)."""
    from femtovllm_b200 import workloads

    rng = np.random.default_rng(seed)
    seqs = sorted(rng.choice(batch.num_seqs, size=min(n_seqs, batch.num_seqs), replace=False).tolist())
    sub = workloads.subset_for_oracle(batch, seqs)
    sub["k_new"] = batch.k_new[seqs].float().cpu().numpy()
    sub["v_new"] = batch.v_new[seqs].float().cpu().numpy()
    sub["bytes"] = _decode_step_bytes(batch, seqs)
    return sub


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


def cpu_decode_step(sub) -> None:
    import oracle

    kp, vp = sub["k_pool"], sub["v_pool"]
    slots = oracle.build_slot_mapping(sub["positions"], np.arange(len(sub["kv_lens"])), sub["block_tables"])
    oracle.store_kvcache(sub["k_new"], sub["v_new"], kp, vp, slots)
    oracle.decode_attention(sub["q"], kp, vp, sub["block_tables"], sub["kv_lens"], acc_dtype=np.float32)


def time_cpu_baseline(sub, steps: int, warmup: int) -> tuple[float, float]:
    for _ in range(warmup):
        cpu_decode_step(sub)
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        cpu_decode_step(sub)
        t.append(time.perf_counter() - t0)
    med = float(np.median(t))
    return sub["bytes"] / med / 1e9, med


def _cpu_threads():
    """Let numpy's BLAS use every host core (torchrun sets OMP_NUM_THREADS=1 for its workers)."""
    try:
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=os.cpu_count() or 1)
    except Exception:
        import contextlib

        return contextlib.nullcontext()


def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


def run_gpu(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from femtovllm_b200 import ops, workloads

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    batch = workloads.config2(seed=2 + rank, num_seqs=args.num_seqs).materialize(dev)
    md = batch.device_metadata(dev)
    q, kp, vp = batch.q, batch.k_pool, batch.v_pool
    tables, lens, slots = md["block_tables"], md["kv_lens"], md["slot_mapping"]
    max_kv = batch.max_kv_len
    stream = torch.cuda.current_stream()

    def step():
        ops.store_kvcache(batch.k_new, batch.v_new, kp, vp, slots)
        return ops.paged_attention_gemv(q, kp, vp, tables, lens, max_kv)

    def barrier():
        if world > 1:
            dist.barrier()

    # --- device-resident timing of whole steps ---
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    step_ms = ev0.elapsed_time(ev1) / args.steps

    # --- the dominant kernel alone: decode attention launches (split + combine) ---
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(args.steps):
        ops.paged_attention_gemv(q, kp, vp, tables, lens, max_kv)
    d1.record(stream)
    torch.cuda.synchronize()
    decode_ms = d0.elapsed_time(d1) / args.steps
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        ops.store_kvcache(batch.k_new, batch.v_new, kp, vp, slots)
    s1.record(stream)
    torch.cuda.synchronize()
    store_ms = s0.elapsed_time(s1) / args.steps

    # --- end to end through the public API with host buffers ---
    # The step's six inputs (q, new K/V, tables, lens, slots) sit in one pinned staging buffer and
    # cross PCIe as one copy per step into one of two device buffers, each input a fixed view of it.
    srcs = (q, batch.k_new, batch.v_new, tables, lens, slots)
    offs, total = [], 0
    for t in srcs:
        offs.append(total)
        total += -(-t.numel() * t.element_size() // 256) * 256
    h_flat = torch.empty(total, dtype=torch.uint8).pin_memory()

    def views(flat):
        return [flat[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for o, t in zip(offs, srcs)]

    for hv, t in zip(views(h_flat), srcs):
        hv.copy_(t.cpu())
    h_q = views(h_flat)[0]
    h_out = torch.empty_like(h_q).pin_memory()
    h2d = total
    d2h = h_out.numel() * h_out.element_size()

    # Each step copies its inputs host -> device and its output back, through the public ops.  The
    # copies run on their own streams, double-buffered, so step i+1's inputs cross PCIe while step i
    # computes and step i's output returns while step i+1 computes; every copy of every step is
    # inside the timed region (the compute stream waits for the last read-back before the end event).
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    d_flat = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]
    dbuf = [views(f) for f in d_flat]
    h_outs = [h_out, torch.empty_like(h_q).pin_memory()]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def copy_in(i):
        b = i % 2
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(ev_used[b])  # step i-2 is done reading this buffer
            d_flat[b].copy_(h_flat, non_blocking=True)
            ev_in[b].record(h2d_s)

    def run_steps(n):
        copy_in(0)
        for i in range(n):
            b = i % 2
            stream.wait_event(ev_in[b])
            dq, dk, dv, dt, dl, ds = dbuf[b]
            ops.store_kvcache(dk, dv, kp, vp, ds)
            out = ops.paged_attention_gemv(dq, kp, vp, dt, dl, max_kv)
            ev_used[b].record(stream)
            if i + 1 < n:
                copy_in(i + 1)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ev_used[b])
                d2h_s.wait_event(ev_out[b])  # the read-back of step i-2 into the same host buffer
                h_outs[b].copy_(out, non_blocking=True)
                out.record_stream(d2h_s)
                ev_out[b].record(d2h_s)
        stream.wait_stream(d2h_s)

    run_steps(args.warmup)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    step_bytes = _decode_step_bytes(batch)
    decode_bytes = batch.decode_bytes()
    res = {"step_ms": step_ms, "decode_ms": decode_ms, "store_ms": store_ms, "e2e_ms": e2e_ms,
           "bytes": step_bytes, "tokens": batch.num_seqs}
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
    else:
        gathered = [res]
    clocks = clk.summary()
    from femtovllm_b200 import capi

    lib = capi.load()
    plan_ws = lib.fvb_paged_attention_decode_workspace_size(batch.num_seqs, batch.n_heads, batch.n_kv_heads,
                                                            batch.head_dim, max_kv)
    launches_per_step = 2 + (1 if plan_ws > 0 else 0)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        sub = cpu_decode_sample(batch, args.cpu_seqs)
        with _cpu_threads():
            gbs, med = time_cpu_baseline(sub, steps=3, warmup=1)
            cores = _blas_threads()
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"{len(sub['kv_lens'])} of {batch.num_seqs} config-2 sequences (store + decode), "
                         f"fp32 numpy oracle, median of 3 steps ({med * 1e3:.1f} ms/step)"}
    return gathered, clocks, decode_bytes, launches_per_step, cpu, (h2d, d2h), batch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seqs", type=int, default=24)
    ap.add_argument("--num-seqs", type=int, default=256, help="sequences per GPU (256 = BASELINE config 2)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "mixed", "long", "qk_norm_rope", "decode_graph", "store",
                                                       "sampler"],
                    help="decode = config 2 (the contract line); prefill = config 3; mixed = config 4; "
                         "long = config 5 sharded over the ranks; qk_norm_rope = the fused q/k norm + rotary + "
                         "KV write over config 3's new tokens; decode_graph = one small-batch decode step "
                         "(slots + fused norm/rope/write + attention) eager vs replayed from a CUDA graph; "
                         "store = store_kvcache of 65,536 new tokens (config 2's heads); "
                         "sampler = next-token sampling of 256 rows of a 151,936-token vocabulary")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    hbm_peak, tflops_peak, peak_src = _peaks()

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    if args.workload == "decode_graph":
        run_decode_graph(args, rank, local_rank)
        return
    if args.workload == "store":
        run_store(args, rank, local_rank, hbm_peak, peak_src)
        return
    if args.workload == "sampler":
        run_sampler(args, rank, local_rank, hbm_peak, peak_src)
        return
    if args.workload != "decode":
        run_other(args, rank, world, local_rank, hbm_peak, tflops_peak, peak_src)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    gathered, clocks, decode_bytes, launches, cpu, (h2d, d2h), batch = run_gpu(args, rank, world, local_rank)
    if rank == 0:
        t_step = max(g["step_ms"] for g in gathered)
        t_e2e = max(g["e2e_ms"] for g in gathered)
        t_dec = max(g["decode_ms"] for g in gathered)
        total_bytes = sum(g["bytes"] for g in gathered)
        tokens = sum(g["tokens"] for g in gathered)
        value = total_bytes / (t_step * 1e-3) / 1e9
        achieved = decode_bytes / (gathered[0]["decode_ms"] * 1e-3) / 1e9
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
                "num_seqs_per_gpu": batch.num_seqs, "n_heads": batch.n_heads, "n_kv_heads": batch.n_kv_heads,
                "head_dim": batch.head_dim, "block_size": 16, "kv_len": "U[512,4096]",
                "pool_blocks_per_gpu": batch.num_blocks, "parallelism": f"request-sharded x{world}, no collective",
                "l2": "inputs larger than L2 (K/V ~2.4 GB per GPU), no flush",
            },
            "tokens_per_s": round(tokens / (t_step * 1e-3), 1),
            "pct_hbm_peak": round(100 * value / (hbm_peak * world), 2),
            "kernel_ms": {"decode_attention": round(t_dec, 5), "store_kvcache": round(gathered[0]["store_ms"], 5)},
            "roofline": {
                "kernel": "decode attention (decode_split_kernel + decode_combine_kernel)",
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                "traffic": _profile_traffic("decode_config2"),
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": round(total_bytes / (t_e2e * 1e-3) / 1e9, 2),
                "unit": "GB/s",
                "ms_per_step": round(t_e2e, 5),
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "femtovllm_b200.ops.store_kvcache + paged_attention_gemv from pinned host buffers "
                       "(the step's inputs copied in as one staging copy and the output copied out every step, "
                       "on copy streams overlapping the neighbouring steps' compute)",
            },
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_other(args, rank, world, local_rank, hbm_peak, tflops_peak, peak_src):
    """Development measurements: prefill (config 3), mixed (config 4), long decode (config 5), and the
    fused q/k norm + rotary + KV write over config 3's new tokens."""
    import torch
    import torch.distributed as dist

    from femtovllm_b200 import ops, workloads

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.workload in ("prefill", "qk_norm_rope"):
        batch = workloads.config3(seed=3 + rank, num_seqs=args.num_seqs if args.num_seqs != 256 else 64)
    elif args.workload == "mixed":
        batch = workloads.config4(seed=4 + rank)
    else:
        total = args.num_seqs if args.num_seqs != 256 else 64  # config 5: 64 sequences over all ranks
        batch = workloads.config5(rank=rank, world=world, total=total)
    batch.materialize(dev)
    md = batch.device_metadata(dev)
    stream = torch.cuda.current_stream()
    if args.workload == "long":
        def step():
            return ops.paged_attention_gemv(batch.q, batch.k_pool, batch.v_pool, md["block_tables"], md["kv_lens"],
                                            batch.max_kv_len)
    elif args.workload == "qk_norm_rope":
        # The projection output (T, (Hq + 2 Hkv) D) as the Linear layers emit it; q / k / v are views of it.
        T, Hq, Hkv, D = batch.num_tokens, batch.n_heads, batch.n_kv_heads, batch.head_dim
        x = torch.cat([batch.q.transpose(0, 1).reshape(T, -1), batch.k_new.reshape(T, -1),
                       batch.v_new.reshape(T, -1)], dim=1)
        batch.q = None
        qv = x[:, : Hq * D].view(T, Hq, D)
        kv = x[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D)
        vv = x[:, (Hq + Hkv) * D :].view(T, Hkv, D)
        g = torch.Generator(device=dev).manual_seed(7)
        q_w = (1 + 0.25 * torch.randn(D, generator=g, device=dev)).to(batch.dtype)
        k_w = (1 + 0.25 * torch.randn(D, generator=g, device=dev)).to(batch.dtype)
        rows = int(batch.kv_lens.max())
        inv = 1e-6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
        theta = torch.arange(rows, device=dev, dtype=torch.float32)[:, None] * inv[None]
        theta = torch.cat([theta, theta], -1)
        cos, sin = theta.cos().to(batch.dtype), theta.sin().to(batch.dtype)
        es = x.element_size()

        def step():
            return ops.qk_norm_rope_store(qv, kv, vv, q_w, k_w, 1e-6, cos, sin, md["positions"], batch.k_pool,
                                          batch.v_pool, md["slot_mapping"])
    else:
        def step():
            return ops.paged_attention_gemm(batch.q, batch.k_pool, batch.v_pool, md["cu_seqlens"], batch.max_q_len, 32,
                                            None, None, md["block_tables"], md["kv_lens"], md["positions"])
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    if args.workload == "long":
        nbytes = batch.decode_bytes()
    elif args.workload == "qk_norm_rope":
        # q, k, v read once and q_out, k, v written once, plus position and slot per token
        nbytes = 2 * batch.num_tokens * (batch.n_heads + 2 * batch.n_kv_heads) * batch.head_dim * es + 12 * batch.num_tokens
    else:
        nbytes = batch.kv_bytes()
    res = {"ms": ms, "flops": 0 if args.workload == "qk_norm_rope" else batch.attn_flops(), "bytes": nbytes,
           "tokens": batch.num_tokens}
    gathered = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, res)
    else:
        gathered = [res]
    if rank != 0:
        return
    t = max(g["ms"] for g in gathered)
    flops = sum(g["flops"] for g in gathered)
    nbytes = sum(g["bytes"] for g in gathered)
    tokens = sum(g["tokens"] for g in gathered)
    line = {"metric": METRIC, "workload": args.workload, "n_gpus": world, "steps": args.steps, "ms_per_step": round(t, 5),
            "tflops": round(flops / (t * 1e-3) / 1e12, 2), "gbs": round(nbytes / (t * 1e-3) / 1e9, 1),
            "tokens_per_s": round(tokens / (t * 1e-3), 1),
            "pct_tensor_peak": round(100 * flops / (t * 1e-3) / 1e12 / (tflops_peak * world), 2),
            "pct_hbm_peak": round(100 * nbytes / (t * 1e-3) / 1e9 / (hbm_peak * world), 2),
            "peak_source": peak_src, "config": batch.name, "clocks": clk.summary()}
    sus = _sustained_tflops()
    if flops and sus:
        line["pct_tensor_peak_sustained"] = round(100 * flops / (t * 1e-3) / 1e12 / (sus * world), 2)
    print(json.dumps(line), flush=True)


def run_store(args, rank, local_rank, hbm_peak, peak_src):
    """store_kvcache alone at prefill size: T new tokens (65,536 unless --num-seqs gives another T) of
    config 2's heads (Hkv 8, D 128, bf16) scattered through a random slot mapping into a pool with room
    for 2 T tokens.  Inputs and pool exceed L2."""
    import numpy as np
    import torch

    from femtovllm_b200 import ops

    if rank != 0:
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T = args.num_seqs if args.num_seqs != 256 else 65536
    hkv, D = 8, 128
    g = torch.Generator(device=dev).manual_seed(11)
    k = torch.randn(T, hkv, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(T, hkv, D, generator=g, device=dev).to(torch.bfloat16)
    blocks = (2 * T + 15) // 16
    k_pool = torch.zeros(blocks, hkv, 16, D, device=dev, dtype=torch.bfloat16)
    v_pool = torch.zeros_like(k_pool)
    rng = np.random.default_rng(11)
    slots = torch.from_numpy(rng.permutation(blocks * 16)[:T].astype(np.int64)).to(dev)

    def step():
        ops.store_kvcache(k, v, k_pool, v_pool, slots)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = 2 * 2 * T * hkv * D * 2 + 8 * T  # K and V rows read and written, slots read
    line = {"metric": "store_kvcache GB/s", "workload": "store", "tokens": T, "n_kv_heads": hkv, "head_dim": D,
            "steps": args.steps, "ms_per_step": round(ms, 5), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "pct_hbm_peak": round(100 * nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 2), "peak_source": peak_src,
            "data": "synthetic (seeded N(0,1), random slot permutation)", "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


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
    import numpy as np
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
    import numpy as np
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
    """The reference's CPU attention path (oracle restatement) on host cores."""
    if rank != 0:
        return
    import torch

    from femtovllm_b200 import workloads

    torch.set_num_threads(os.cpu_count() or 1)
    batch = workloads.config2(seed=2)
    # Host copy of only the sampled sequences' pages: draw the pools on the CPU.
    rng = np.random.default_rng(0)
    seqs = sorted(rng.choice(batch.num_seqs, size=min(args.cpu_seqs, batch.num_seqs), replace=False).tolist())
    small = workloads.custom(batch.kv_lens[seqs], np.ones(len(seqs)), batch.n_heads, batch.n_kv_heads,
                             batch.head_dim, torch.bfloat16, seed=2, pool_factor=1.2, qkv_scale=batch.qkv_scale)
    small.materialize("cpu")
    sub = workloads.subset_for_oracle(small, list(range(len(seqs))))
    sub["k_new"] = small.k_new.float().numpy()
    sub["v_new"] = small.v_new.float().numpy()
    sub["bytes"] = _decode_step_bytes(small)
    with _cpu_threads():
        for _ in range(args.warmup):
            cpu_decode_step(sub)
        t = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            cpu_decode_step(sub)
            t.append(time.perf_counter() - t0)
        cores = _blas_threads()
    mean = float(np.mean(t))
    value = sub["bytes"] / mean / 1e9
    sample = (f"{len(seqs)} of 256 config-2 sequences per step (store + decode, fp32 numpy restatement of "
              f"qwen3.py:240-264 + 430-542)")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(mean * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16-valued inputs)",
        "data": "synthetic",
        "config": {"workload": "config2: decode paged attention + 1-token store_kvcache per sequence (sampled)"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
