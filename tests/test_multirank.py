"""world_size-2 gloo tests (CPU) of the multi-rank host logic.

The hot path shards by request with no collective on the data path: every rank
owns its KV pool, block tables and sequences.  These tests check, across real
processes, that the LPT request sharding of config 5 partitions the batch, that
every rank's metadata is self-consistent, and that a rank failing before a
collective is detected by its peer through the process group's timeout (host
side only; no GPU is involved).
"""

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    sys.path[:0] = [str(REPO), str(REPO / "nano-vllm-practice_b200")]
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    return dist


def _shard_worker(rank, world, port, out):
    dist = _init(rank, world, port, 60)
    import oracle
    from femtovllm_b200 import workloads

    lengths = workloads.config5_lengths()
    mine = workloads.shard_lpt(lengths, world)[rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine.tolist())
    b = workloads.config5(rank=rank, world=world)
    ok_tables = bool(
        (b.kv_lens == lengths[mine]).all()
        and np.array_equal(oracle.build_slot_mapping(b.positions, b.seq_of_token, b.block_tables), b.slot_mapping)
        and b.block_tables.max() < b.num_blocks
    )
    dist.barrier()
    dist.destroy_process_group()
    out[rank] = (gathered, int(lengths[mine].sum()), ok_tables)


def _failing_worker(rank, world, port, out):
    dist = _init(rank, world, port, 5)
    import torch

    if rank == 1:
        # A rank that dies between steps: it never joins the next collective.
        dist.destroy_process_group()
        out[rank] = "exited"
        return
    try:
        dist.all_reduce(torch.ones(4))
        out[rank] = "no error"
    except Exception as e:  # the peer learns of the failure on the host
        out[rank] = type(e).__name__
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run(target, world=2):
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=target, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
        return dict(out)


def test_lpt_sharding_partitions_config5_across_ranks():
    out = _run(_shard_worker)
    assert set(out) == {0, 1}
    gathered = out[0][0]
    assert gathered == out[1][0]
    allidx = sorted(sum(gathered, []))
    assert allidx == list(range(64))  # every request on exactly one rank
    loads = [out[r][1] for r in (0, 1)]
    assert max(loads) <= 1.05 * min(loads)  # LPT keeps the token loads within a few percent
    assert out[0][2] and out[1][2]


@pytest.mark.timeout(120)
def test_peer_failure_surfaces_as_an_error_not_a_hang():
    out = _run(_failing_worker)
    assert out.get(1) == "exited"
    assert out.get(0) not in (None, "no error")
