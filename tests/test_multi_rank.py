"""The N > 1 host logic on CPU with two gloo ranks (no GPU): config 1's N-split. Each rank builds
its shard of the sweep image (bench.build_gemm: the vocabulary shape's output columns split over
the ranks, the other shapes whole on every rank), computes its outputs with the oracle, the ranks
all-gather their output regions, and the reassembled full outputs (split columns in rank order,
replicated shapes from rank 0) must hash to the reference golden Machine's
(tests/golden/gemm_sweep.json, M = 4). Also the max-over-ranks time of bench.py and the queue
segments the overlapped all-gathers follow."""
import json
import os
import socket

import pytest


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import numpy as np
    import torch
    import torch.distributed as dist
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        import bench
        from oracle.machine import OracleMachine
        p = bench.build_gemm(world, rank, ms=(4,))
        assert p["split"] == {2} and [seg[:2] for seg in p["segments"]] == [(4, "split"), (None, "rest")]
        assert p["nl"][2] == 151936 // world and p["nl"][0] == 3072
        o = OracleMachine(bytearray(p["ddr"].tobytes()))
        assert o.run_queue(p["q_setup"], p["n_setup"]).done
        assert o.run_queue(p["q_main"], p["n_main"]).done
        y0, yn = p["y_region"]
        mine = torch.frombuffer(bytearray(bytes(o.ddr[y0:y0 + yn])), dtype=torch.uint8)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        slow = bench.max_over_ranks(float(rank + 1), world)
        if rank == 0:
            regions = [t.numpy() for t in parts]
            out.put((bench.gemm_hashes(bench.gemm_outputs(p, regions)), slow))
    finally:
        dist.destroy_process_group()


def test_gemm_sweep_n_split_over_two_ranks_matches_reference():
    import multiprocessing as mp
    from tests import fixtures as FX
    want = json.loads((FX.GOLDEN / "gemm_sweep.json").read_text())["sha256"]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got, slow = q.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert got == {k: want[k] for k in got}
    assert slow == 2.0
