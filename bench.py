#!/usr/bin/env python
"""Benchmark of the tars_mini hot path on B200s (one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload decode|decode-gemma|gemv|w4|gemm|vision|qwen35]
                    [--batch B] [--impl ours|reference]

Workloads (synthetic seeded data with the configs' distributions):
  decode        (default) config 3: Qwen3-0.6B shapes, random-init weights, B sequences per GPU
                (default 64) with seeded 20-token prompts prefilled in chunks of 4, then greedy
                decode; a step = one token for every sequence; value in tok/s (all GPUs). The
                default K = 236 timed steps decode the whole context once (positions 20 -> 255),
                each step timed with its own pair of events; ms_per_step_at_position gives the
                steps near positions 32, 128 and 250. Sequence 0 is checked bit for bit against
                the reference's logits (committed fixture). The line also carries config0_gemv
                and config2_w4: the GEMV workloads below, 50 timed steps each, and on one GPU
                config1_gemm (the sweep, 20 steps) and config4_gemma3_decode (Gemma-3-1B decode,
                positions 20 -> 60) (--decode-only skips them).
  decode-gemma  config 4: the same for Gemma-3-1B shapes
  gemv  config 0: one unit = ROW_QUANT of x [1, 1024] + W8A8 GEMV (QM_ROWCOL) against W [3072, 1024];
        a step runs R units on R distinct weight copies (R * 3 MiB > the 126 MB L2)
  w4    config 2: one unit = W4A16 GEMV, M=1, K=8192, N=16384 (64 MiB of packed weights);
        a step runs R units on distinct weight copies
  gemm  config 1: the W8A8 prefill GEMM sweep, M in {4, 16, 64, 256} x (K, N) in {(1024, 3072),
        (3072, 1024), (1024, 151936), (6912, 1152) as K blocks 4096 + 2816}; a step = every GEMM of
        the sweep (one queue); value in int8 TOPS (2 M N K per GEMM); on N GPUs the vocabulary
        shape's N is split over the ranks (each keeps its output columns, as a greedy pick over a
        shard would), the small shapes run whole on every rank (strong scaling); each M's split
        outputs are all-gathered with NCCL while the later segments compute (--gemm-gather after:
        once the step's GEMMs are done; none: outside the timed steps)
gemv / w4 value: algorithmic bytes of all units of all ranks / device time of the timed steps
(max over ranks), in GB/s. e2e: the same metric through the board-runtime API (opentars_b200.board.Cuda:
host writes x into pinned memory, to_dev, run, from_dev of y) timed on the host clock.
--impl reference: the reference's numpy golden path restated in oracle/ (the reference itself is
Python and cannot travel), on all host cores, over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] if (ROOT / "BASELINE.json").exists() else \
    "W8A8/W4A16 GEMV HBM GB/s vs peak; Qwen3-0.6B-shape decode tok/s, bit-exact"
QA_ALIGN = 128


# ----------------------------------------------------------------------------- programs
def _desc(**f):
    from opentars_b200 import contract as C
    return C.encode(dict(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1, **f))


def _align(x, a=QA_ALIGN):
    return -(-x // a) * a


def build_gemv(R: int, seed: int, M: int = 1, K: int = 1024, N: int = 3072):
    """R independent config-0 GEMVs (quant + GEMM) in one image; returns the program and layout."""
    from opentars_b200 import contract as C
    rng = np.random.default_rng(seed)
    w0 = 0x1000
    s0 = _align(w0 + R * N * K)
    x0 = _align(s0 + R * 4 * N)
    q0 = _align(x0 + R * 4 * M * K)
    r0 = _align(q0 + R * M * K)
    y0 = _align(r0 + R * 16)
    qa = _align(y0 + R * 4 * M * N)
    size = _align(qa + 64 * 2 * R + 4096, 1 << 16)
    ddr = np.zeros(size, np.uint8)
    for r in range(R):
        ddr[w0 + r * N * K:w0 + (r + 1) * N * K] = rng.integers(-127, 128, N * K, dtype=np.int8).view(np.uint8)
    ddr[s0:s0 + R * 4 * N] = rng.uniform(1e-3, 1e-2, R * N).astype("<f4").view(np.uint8)
    ddr[x0:x0 + R * 4 * M * K] = rng.normal(0, 1, R * M * K).astype("<f4").view(np.uint8)
    for r in range(R):
        q, sr = q0 + r * M * K, r0 + r * 16
        d0 = _desc(OPCODE=C.OP_ROW, CTRL=C.ROW_QUANT, EPI=C.epi(C.ACT_NONE, C.OUT_INT8),
                   A_OFF=x0 + r * 4 * M * K, Y_OFF=q, SCALE_OFF=sr, M=M, N=K)
        d1 = _desc(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_ROWCOL), EPI=C.epi(), A_OFF=q, W_OFF=w0 + r * N * K,
                   SCALE_OFF=s0 + r * 4 * N, Y_OFF=y0 + r * 4 * M * N, M=M, N=N, K=K, HDR_RSV=sr // 16)
        ddr[qa + 128 * r:qa + 128 * r + 64] = np.frombuffer(d0, np.uint8)
        ddr[qa + 128 * r + 64:qa + 128 * (r + 1)] = np.frombuffer(d1, np.uint8)
    gemm_bytes = N * K + 4 * N + M * K + 4 * M + 4 * M * N          # 3,171,332 bytes at config 0
    quant_bytes = 4 * M * K + M * K + 4 * M
    return dict(ddr=ddr, qa=qa, qlen=2 * R, units=R, unit_bytes=gemm_bytes + quant_bytes,
                kernel_bytes=R * gemm_bytes, roof=(2, lambda i: i == 1),
                kernel=f"k_gemv8_group (W8A8 GEMV, {R} units in one launch)",
                inputs=(x0, R * 4 * M * K), outputs=(y0, R * 4 * M * N),
                config=dict(workload="config0_w8a8_gemv", M=M, K=K, N=N, units_per_step=R,
                            weights_bytes_per_step=R * N * K,
                            l2="inputs larger than L2: each step streams R distinct weight copies"))


def build_w4(R: int, seed: int, M: int = 1, K: int = 8192, N: int = 16384):
    from opentars_b200 import contract as C
    rng = np.random.default_rng(seed)
    G = K // 128
    w0 = 0x1000
    s0 = _align(w0 + R * N * K // 2)
    x0 = _align(s0 + R * 2 * N * G)
    y0 = _align(x0 + R * 4 * M * K)
    qa = _align(y0 + R * 4 * M * N)
    size = _align(qa + 64 * R + 4096, 1 << 16)
    ddr = np.zeros(size, np.uint8)
    for r in range(R):
        ddr[w0 + r * N * K // 2:w0 + (r + 1) * N * K // 2] = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    ddr[s0:s0 + R * 2 * N * G] = rng.uniform(1e-3, 2e-2, R * N * G).astype("<f2").view(np.uint8)
    ddr[x0:x0 + R * 4 * M * K] = rng.normal(0, 1, R * M * K).astype("<f4").view(np.uint8)
    for r in range(R):
        d = _desc(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_GROUP, a_dtype=C.DT_FP32, w_dtype=C.DT_INT4), EPI=C.epi(),
                  A_OFF=x0 + r * 4 * M * K, W_OFF=w0 + r * N * K // 2, SCALE_OFF=s0 + r * 2 * N * G,
                  Y_OFF=y0 + r * 4 * M * N, M=M, N=N, K=K, GROUP_SIZE=128)
        ddr[qa + 64 * r:qa + 64 * (r + 1)] = np.frombuffer(d, np.uint8)
    unit = N * K // 2 + 2 * N * G + 4 * M * K + 4 * M * N               # 69,304,320 bytes here
    return dict(ddr=ddr, qa=qa, qlen=R, units=R, unit_bytes=unit, kernel_bytes=R * unit, roof=(2, lambda i: i == 0),
                kernel="k_w4_align + k_gemv_w4t: the step's R W4A16 GEMVs as one grouped launch (one dependency level)",
                inputs=(x0, R * 4 * M * K), outputs=(y0, R * 4 * M * N),
                config=dict(workload="config2_w4a16_gemv", M=M, K=K, N=N, units_per_step=R,
                            weights_bytes_per_step=R * N * K // 2,
                            l2="inputs larger than L2: each step streams R distinct weight copies"))


WORKLOADS = {"gemv": (build_gemv, 64), "w4": (build_w4, 4)}


# ----------------------------------------------------------------------------- clocks (NVML)
class Clocks:
    """Samples SM clock and throttle reasons of one GPU every 5 ms while running."""

    def __init__(self, index: int):
        self.index, self.samples, self.reasons, self.max_mhz = index, [], set(), None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            names = {getattr(N, k): k for k in dir(N) if k.startswith("nvmlClocksEventReason")
                     and k not in ("nvmlClocksEventReasonAll", "nvmlClocksEventReasonNone")}

            def loop():
                while not self._stop.is_set():
                    self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                    r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for bit, name in names.items():
                        if isinstance(bit, int) and r & bit:
                            self.reasons.add(name.replace("nvmlClocksEventReason", ""))
                    time.sleep(0.005)
            self._t = threading.Thread(target=loop, daemon=True)
            self._t.start()
        except Exception as e:                      # no NVML: report that instead of numbers
            self.error = str(e)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "note": getattr(self, "error", "no samples")}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU oracle timing
def _oracle_unit_worker(args):
    """Runs the oracle on one-unit images for `seconds`; returns (units, elapsed)."""
    workload, seed, seconds = args
    sys.path.insert(0, str(ROOT))
    from oracle.machine import OracleMachine
    p = WORKLOADS[workload][0](1, seed)
    ddr = bytearray(p["ddr"].tobytes())
    n, t0 = 0, time.perf_counter()
    while True:
        m = OracleMachine(bytearray(ddr))
        assert m.run_queue(p["qa"], p["qlen"]).done
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    return n, time.perf_counter() - t0


def cpu_oracle_gbs(workload: str, seconds: float, procs: int) -> dict:
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    unit_bytes = WORKLOADS[workload][0](1, 0)["unit_bytes"]
    t0 = time.perf_counter()
    with ctx.Pool(procs) as pool:
        res = pool.map(_oracle_unit_worker, [(workload, 100 + i, seconds) for i in range(procs)])
    wall = time.perf_counter() - t0
    units = sum(n for n, _ in res)
    span = max(t for _, t in res)
    return dict(value=units * unit_bytes / span / 1e9, unit="GB/s", cores=procs, kind="port",
                sample=f"{units} units of {workload} (one per image) on {procs} processes, {span:.1f}s each",
                wall_s=round(wall, 1))


# ----------------------------------------------------------------------------- distributed plumbing
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------- our arm
def run_ours(a, world, rank, local) -> dict | None:
    m = measure_units(a.workload, a.units, a.steps, a.warmup, world, rank, local)
    if rank != 0:
        return None
    out = {
        "metric": METRIC, "value": round(m["value"], 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": m["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8" if a.workload == "gemv" else "int4xint16",
        "data": "synthetic, seeded (BASELINE config distributions)",
        "config": gemv_config(m["config"], world),
        "roofline": m["roofline"], "e2e": m["e2e"],
        "gpu_launches": m["gpu_launches"], "clocks": m["clocks"], "bit_exact_unit0": m["bit_exact"],
    }
    if world == 1 and not a.no_cpu:
        out["cpu_baseline"] = cpu_oracle_gbs(a.workload, a.cpu_seconds, os.cpu_count() or 1)
    return out


def measure_units(workload: str, units: int, steps: int, warmup: int, world: int, rank: int, local: int,
                  e2e_steps: int | None = None) -> dict:
    """Configs 0 / 2 on this GPU: `steps` timed launches of the captured queue of R units (device
    time, max over ranks), the dominant kernel's roofline, the end-to-end number through the board
    API and rank 0's unit 0 against the oracle."""
    import ctypes

    import torch
    os.environ["TC_DEVICE"] = str(local)
    torch.cuda.set_device(local)
    from opentars_b200._lib import check, lib
    from opentars_b200.board import Cuda
    build, R = WORKLOADS[workload]
    R = units or R
    p = build(R, seed=1234 + rank)
    L = lib()
    ddr = p["ddr"]
    dev = Cuda(len(ddr), device=local, pinned=True)
    dev.mem[:] = ddr
    dev.to_dev(0, len(ddr))
    g, st = dev.graph(p["qa"], p["qlen"])
    assert g is not None and st.done, "the benchmark queue must capture"
    kernels_per_step = check(L.tc_graph_kernels(g), dev.h, "graph_kernels")
    stream = torch.cuda.ExternalStream(L.tc_stream(dev.h), device=local)

    # parity spot check: unit 0 against the oracle happens after timing (rank 0)
    for _ in range(warmup):
        check(L.tc_graph_launch(g, None), dev.h)
    check(L.tc_synchronize(dev.h), dev.h)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            check(L.tc_graph_launch(g, None), dev.h)
        e1.record(stream)
        check(L.tc_synchronize(dev.h), dev.h)
    ms = e0.elapsed_time(e1)
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    total_bytes = world * R * p["unit_bytes"] * steps
    value = total_bytes / (ms_max / 1e3) / 1e9

    # roofline: device times of the dominant kernel from a graph captured with events between
    # dependency levels (config 0: level 1 is the one grouped GEMV launch of all R units; config 2:
    # level 0 is the grouped pre-pass and GEMV launch of all R units)
    from opentars_b200._lib import Status_t
    mode, pick = p["roof"]
    st2, cop, gt = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
    check(L.tc_queue_capture(dev.h, p["qa"], p["qlen"], 0, 0, mode, ctypes.byref(st2), ctypes.byref(cop),
                             ctypes.byref(gt)), dev.h)
    kt = []
    for _ in range(3):
        check(L.tc_graph_launch(gt, None), dev.h)
        check(L.tc_synchronize(dev.h), dev.h)
        arr = (ctypes.c_float * p["qlen"])()
        n = check(L.tc_graph_times(gt, arr, p["qlen"]), dev.h, "graph_times")
        kt += [arr[i] for i in range(n) if pick(i)]
    if not kt:
        raise RuntimeError("no kernel timings")
    L.tc_graph_destroy(gt)
    k_ms = statistics.mean(kt)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = p["kernel_bytes"] / (k_ms / 1e3) / 1e9
    traffic_file = ROOT / "profiles" / f"traffic_{workload}.json"
    traffic = json.loads(traffic_file.read_text()).get("bytes_per_launch") if traffic_file.exists() else None
    roofline = dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s", frac=round(achieved / peak, 4),
                    traffic=traffic, kernel=p["kernel"], kernel_bytes_per_launch=p["kernel_bytes"],
                    kernel_us=round(k_ms * 1e3, 3), peak_source="measured" if peaks else "fallback")

    # e2e through the board API with host (pinned) buffers, host clock
    x0, xn = p["inputs"]
    y0, yn = p["outputs"]
    rng = np.random.default_rng(7 + rank)
    xs = [rng.normal(0, 1, xn // 4).astype("<f4").view(np.uint8) for _ in range(4)]
    for i in range(2):
        dev.mem[x0:x0 + xn] = xs[i % 4]
        dev.to_dev(x0, xn)
        dev.run(p["qa"], p["qlen"])
        dev.from_dev(y0, yn)
    n_e2e = steps if e2e_steps is None else e2e_steps
    barrier(world)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        dev.mem[x0:x0 + xn] = xs[i % 4]
        dev.to_dev(x0, xn)
        dev.run(p["qa"], p["qlen"])
        dev.from_dev(y0, yn)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = dict(value=round(world * R * p["unit_bytes"] * n_e2e / e2e_s / 1e9, 2), unit="GB/s",
               h2d_bytes_per_step=xn, d2h_bytes_per_step=yn,
               api="opentars_b200.board.Cuda: mem write, to_dev, run (cached graph), from_dev")

    # parity: unit 0's output of the last run against the oracle
    bit_exact = None
    if rank == 0:
        from oracle.machine import OracleMachine
        # unit 0 of the benchmark image with the last e2e input
        dev.from_dev(0, len(ddr))
        img = dev.mem.copy()
        o = OracleMachine(bytearray(img.tobytes()))
        qa = p["qa"]
        o.run_queue(qa, 2 if workload == "gemv" else 1)
        bit_exact = bytes(o.ddr[y0:y0 + yn // R]) == img[y0:y0 + yn // R].tobytes()
    dev.close()
    return dict(value=value, ms_per_step=round(ms_max / steps, 4), config=p["config"], roofline=roofline,
                e2e=e2e, gpu_launches=steps * kernels_per_step, clocks=clk.summary(), bit_exact=bit_exact)


# ----------------------------------------------------------------------------- the reference arm
def gemv_config(cfg: dict, world: int) -> dict:
    """The `config` of a GEMV workload's line (both arms print the same)."""
    return dict(cfg, parallelism=f"replicas x{world} (independent GEMV batches per GPU)")


def run_reference(a, world, rank) -> dict | None:
    if rank != 0:
        return None
    procs = os.cpu_count() or 1
    for _ in range(a.warmup):
        cpu_oracle_gbs(a.workload, 0.5, procs)
    vals = [cpu_oracle_gbs(a.workload, a.ref_seconds, procs) for _ in range(a.steps)]
    v = statistics.mean(x["value"] for x in vals)
    build, R = WORKLOADS[a.workload]
    cfg = build(a.units or R, 0)["config"]                    # the workload our arm measures
    return {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8" if a.workload == "gemv" else "int4xint16", "data": "synthetic, seeded",
        "config": gemv_config(cfg, world),
        "cpu_baseline": dict(value=round(v, 4), unit="GB/s", cores=procs, kind="port",
                             sample=vals[-1]["sample"]),
        "e2e": dict(value=round(v, 4), unit="GB/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
        "note": "the reference is Python (numpy golden model); its restatement in oracle/ is timed here",
    }



# ----------------------------------------------------------------------------- config 1: GEMM sweep
GEMM_M = (4, 16, 64, 256)
GEMM_SHAPES = ((1024, 3072, 0), (3072, 1024, 0), (1024, 151936, 0), (6912, 1152, 4096))   # (K, N, first K block)
DESC_N_MAX = 65520                 # the descriptor's N field is 16 bits; blocks are multiples of 16


def _row_blocks(n: int, cap: int = DESC_N_MAX) -> list[tuple[int, int]]:
    parts = -(-n // cap)
    q = -(-n // parts // 16) * 16
    return [(c, min(n, c + q)) for c in range(0, n, q)]


def build_gemm(world: int = 1, rank: int = 0, seed: int = 1234, ms=GEMM_M, shapes=GEMM_SHAPES, split=None):
    """Config 1 on one rank: activations ~N(0,1) quantised per row (a setup queue), int8 weights
    uniform in [-127, 127] with per-channel scales uniform in [1e-3, 1e-2] (seeded, the same full
    operands on every rank). The shapes in `split` (default: those above one descriptor's N, the
    151936-row vocabulary) are N-split: rank r owns output columns [r N / world, (r+1) N / world);
    the others run whole on every rank (replicas: 3 - 20 MB of weights, not worth a collective).
    The split shapes' outputs form one contiguous region per M, and their GEMMs come first in the
    queue, one segment per M ("split"), before one segment of every replicated GEMM ("rest"): each
    M's outputs can be all-gathered while the next segments compute. The (6912, 1152) shape runs as two K blocks (4096 + 2816) sharing the
    scales, their fp32 partial results added by an ELT descriptor. N above the descriptor's 16-bit
    field runs as row blocks. Returns the image, both queues, the output region, the segments and
    per-descriptor metadata."""
    from opentars_b200 import contract as C
    from opentars_b200.program import Image, Linear
    rng = np.random.default_rng(seed)
    Mx = max(ms)
    Ks = sorted({K for K, _, _ in shapes})
    xs = {K: rng.normal(0, 1, (max(GEMM_M), K)).astype(np.float32)[:Mx] for K in Ks}   # row m: the same for any ms
    full = [(rng.integers(-127, 128, (N, K), dtype=np.int8), rng.uniform(1e-3, 1e-2, N).astype(np.float32))
            for K, N, _ in shapes]
    if split is None:
        split = {i for i, (_, N, _) in enumerate(shapes) if N > DESC_N_MAX}
    for i, (K, N, _) in enumerate(shapes):
        assert i not in split or N % (16 * world) == 0, "a split shape's N splits into 16-column multiples"
    nl = [N // world if i in split else N for i, (_, N, _) in enumerate(shapes)]
    own = [(rank * n if i in split else 0) for i, n in enumerate(nl)]      # first owned output column
    need = sum(5 * Mx * K + 4 * Mx + 512 for K in Ks) + sum(n * K + 4 * n + 512 for n, (K, _, _) in zip(nl, shapes))
    need += sum(4 * M * n * (2 if kb else 1) + 512 for M in ms for n, (_, _, kb) in zip(nl, shapes)) + (1 << 16)
    p = Image(need)
    xv = {K: p.constant(xs[K]) for K in Ks}
    qv = {K: p.quantize(xv[K]) for K in Ks}
    _, q_setup, n_setup = p.finish()
    p.descs, p.queue_off = [], None
    lins = []
    for (K, N, kb), (W, sc), n, c0 in zip(shapes, full, nl, own):
        Wl, sl = W[c0:c0 + n], sc[c0:c0 + n]
        s_off = p.store(sl)
        if kb:
            lins.append(("k", [Linear(p.store(np.ascontiguousarray(Wl[:, :kb]), "i1"), s_off, None, n, kb),
                               Linear(p.store(np.ascontiguousarray(Wl[:, kb:]), "i1"), s_off, None, n, K - kb)]))
        else:
            w_off = p.store(Wl, "i1")
            lins.append(("n", [(c0, Linear(w_off + c0 * K, s_off + 4 * c0, None, c1 - c0, K))
                               for c0, c1 in _row_blocks(n)]))
    # outputs: row-block-major for N above one descriptor block (the row stride field is 15 bits
    # of 16 bytes), as the model image lays out the vocabulary head's logits
    y0 = p.top
    order = sorted(range(len(shapes)), key=lambda i: i not in split)          # split shapes first
    ys = {}
    for first in (True, False):
        for M in ms:
            for i in order:
                if (i in split) == first:
                    ys[(M, i)] = [(c0, p.matrix(M, c1 - c0)) for c0, c1 in _row_blocks(nl[i])]
    y1 = p.top
    meta = []                      # per GEMM queue descriptor: (M, shape index, ops, weight bytes) or None
    segments = []                  # (M or None, "split" | "rest", first descriptor, count)
    for first in (True, False):
        for M in ms:
            for i in order:
                if (i in split) != first:
                    continue
                (K, N, kb), (kind, parts), n = shapes[i], lins[i], nl[i]
                key = (M, "split") if first else (None, "rest")
                if not segments or segments[-1][:2] != key:
                    segments.append((*key, len(p.descs), 0))
                xq, xs_off = qv[K]
                xq = xq.rows_at(0, M)
                if kind == "n":
                    for (c0, lin), (_, y) in zip(parts, ys[(M, i)]):
                        p.mm8(xq, xs_off, lin, y)
                        meta.append((M, i, 2 * M * lin.n * K, lin.n * K))
                else:
                    y = ys[(M, i)][0][1]
                    part = p.matrix(M, n)
                    p.mm8(xq.cols_at(0, kb), xs_off, parts[0], y)
                    meta.append((M, i, 2 * M * n * kb, n * kb))
                    p.mm8(xq.cols_at(kb, K - kb), xs_off, parts[1], part)
                    meta.append((M, i, 2 * M * n * (K - kb), n * (K - kb)))
                    p.elt(C.ELT_ADD, y, part, y)
                    meta.append(None)
                M_, sg, first_d, _ = segments[-1]
                segments[-1] = (M_, sg, first_d, len(p.descs) - first_d)
    ddr, q_main, n_main = p.finish()
    split_regions = {}             # M -> (offset, bytes) of its split outputs (contiguous)
    for M in ms:
        blocks = [v for i in order if i in split for _, v in ys[(M, i)]]
        if blocks:
            split_regions[M] = (blocks[0].off, blocks[-1].off + blocks[-1].rows * blocks[-1].ld - blocks[0].off)
    x_first, x_last = min(v.off for v in xv.values()), max(v.off + v.rows * v.ld for v in xv.values())
    return dict(ddr=np.frombuffer(bytes(ddr), np.uint8).copy(), q_setup=q_setup, n_setup=n_setup, q_main=q_main,
                n_main=n_main, y_region=(y0, y1 - y0), x_region=(x_first, x_last - x_first), ys=ys, nl=nl,
                meta=meta, ms=ms, shapes=shapes, world=world, split=split, segments=segments,
                split_regions=split_regions, ops=sum(2 * M * N * K for M in ms for K, N, _ in shapes))


def gemm_outputs(p: dict, gathered: list[np.ndarray]) -> dict:
    """Per (M, shape) the full [M, N] fp32 output from every rank's copy of its output region (a
    split shape's columns from every rank in rank order, a replicated one's from rank 0)."""
    y0 = p["y_region"][0]
    split = p.get("split", set(range(len(p["shapes"]))))
    out = {}
    for (M, i), blocks in p["ys"].items():
        cols = [g[v.off - y0:v.off - y0 + v.rows * v.ld].view("<f4").reshape(M, -1)
                for g in (gathered if i in split else gathered[:1]) for _, v in blocks]
        out[(M, i)] = np.concatenate(cols, axis=1)
    return out


def gemm_hashes(outs: dict) -> dict:
    import hashlib
    return {f"M{M}_s{i}": hashlib.sha256(np.ascontiguousarray(y).tobytes()).hexdigest() for (M, i), y in outs.items()}


class _DevBytes:
    """A device byte range as a CUDA array (for torch.as_tensor without a copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _oracle_gemm_worker(args):
    """Runs one config-1 GEMM descriptor (M=64, K=1024, N=3072) on the oracle for `seconds`."""
    seconds, = args
    sys.path.insert(0, str(ROOT))
    from oracle.machine import OracleMachine
    p = build_gemm(1, 0, seed=99, ms=(64,), shapes=((1024, 3072, 0),))
    o = OracleMachine(bytearray(p["ddr"].tobytes()))
    assert o.run_queue(p["q_setup"], p["n_setup"]).done
    n, t0 = 0, time.perf_counter()
    while True:
        assert o.run_queue(p["q_main"], p["n_main"]).done
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    return n, time.perf_counter() - t0


def cpu_oracle_gemm(seconds: float, procs: int) -> dict:
    import multiprocessing as mp
    with mp.get_context("spawn").Pool(procs) as pool:
        res = pool.map(_oracle_gemm_worker, [(seconds,)] * procs)
    units = sum(n for n, _ in res)
    span = max(t for _, t in res)
    ops = 2 * 64 * 3072 * 1024
    return dict(value=round(units * ops / span / 1e12, 6), unit="TOPS", cores=procs, kind="port",
                sample=f"{units} W8A8 GEMMs of M=64 K=1024 N=3072 (config 1's first shape) on {procs} processes, "
                       f"{span:.1f}s each")


def run_gemm(a, world, rank, local) -> dict | None:
    import ctypes

    import torch
    os.environ["TC_DEVICE"] = str(local)
    torch.cuda.set_device(local)
    from opentars_b200._lib import Status_t, check, lib
    from opentars_b200.board import Cuda
    p = build_gemm(world, rank)
    L = lib()
    ddr = p["ddr"]
    dev = Cuda(len(ddr), device=local, pinned=True)
    dev.mem[:] = ddr
    dev.to_dev(0, len(ddr))
    ok = dev.run(p["q_setup"], p["n_setup"])[0]
    assert ok, "the quantisation queue must run"
    # one graph for the whole queue on one GPU; on N GPUs one per segment (each M's split
    # vocabulary GEMM, then the replicated shapes), each M's outputs all-gathered after its segment
    if world > 1:
        segs = []
        for M, kind, first, count in p["segments"]:
            g, st = dev.graph(p["q_main"] + 64 * first, count)
            assert g is not None and st.done, "every GEMM segment must capture"
            segs.append((M, kind, g))
    else:
        g, st = dev.graph(p["q_main"], p["n_main"])
        assert g is not None and st.done, "the GEMM queue must capture"
        segs = [(None, "rest", g)]
    kernels_per_step = sum(check(L.tc_graph_kernels(g), dev.h, "graph_kernels") for _, _, g in segs)
    stream = torch.cuda.ExternalStream(L.tc_stream(dev.h), device=local)
    y0, yn = p["y_region"]
    base = int(L.tc_device_ptr(dev.h))
    yt = torch.as_tensor(_DevBytes(base + y0, yn), device=f"cuda:{local}")
    side = torch.cuda.Stream(device=local) if world > 1 else None
    mine, gath = {}, {}
    if world > 1:
        for M, (s_off, s_nb) in p["split_regions"].items():
            mine[M] = torch.as_tensor(_DevBytes(base + s_off, s_nb), device=f"cuda:{local}")
            gath[M] = torch.empty(world * s_nb, dtype=torch.uint8, device=f"cuda:{local}")
    gather_ms = []

    def step(timed_gathers: bool = False):
        """The segments in order; after each M's split segment its outputs are all-gathered on a
        second stream (NCCL over NVLink) while the next segments compute."""
        import torch.distributed as dist
        for M, kind, g in segs:
            check(L.tc_graph_launch(g, None), dev.h)
            if world > 1 and kind == "split" and a.gemm_gather == "overlap":
                ev = torch.cuda.Event()
                ev.record(stream)
                side.wait_event(ev)
                with torch.cuda.stream(side):
                    if timed_gathers:
                        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        g0.record(side)
                    dist.all_gather_into_tensor(gath[M], mine[M])
                    if timed_gathers:
                        g1.record(side)
                        gather_ms.append((g0, g1))
        if world > 1 and a.gemm_gather == "after":   # every gather once all GEMMs are done
            with torch.cuda.stream(stream):
                for M in gath:
                    if timed_gathers:
                        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        g0.record(stream)
                    dist.all_gather_into_tensor(gath[M], mine[M])
                    if timed_gathers:
                        g1.record(stream)
                        gather_ms.append((g0, g1))
        if world > 1:
            stream.wait_stream(side)

    for _ in range(a.warmup):
        step()
    check(L.tc_synchronize(dev.h), dev.h)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(a.steps):
            step()
        e1.record(stream)
        check(L.tc_synchronize(dev.h), dev.h)
    ms = e0.elapsed_time(e1)
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    value = p["ops"] * a.steps / (ms_max / 1e3) / 1e12
    collective = None
    if world > 1 and a.gemm_gather != "none":       # the all-gathers' own device time, one more step
        step(timed_gathers=True)
        check(L.tc_synchronize(dev.h), dev.h)
        torch.cuda.synchronize(local)
        g_ms = sum(g0.elapsed_time(g1) for g0, g1 in gather_ms)
        collective = dict(op="all_gather (NCCL) of each M's vocabulary output blocks, " +
                          ("on a second stream while the later segments compute" if a.gemm_gather == "overlap"
                           else "after every GEMM of the step"),
                          bytes_per_rank_per_step=sum(nb for _, nb in p["split_regions"].values()),
                          ms_per_step=round(max_over_ranks(g_ms, world), 4),
                          share_of_step=round(max_over_ranks(g_ms, world) / (ms_max / a.steps), 3),
                          note="share = the gathers' device time / the step's")

    # parity: the full outputs (every rank's output region gathered) against the reference's hashes
    torch.cuda.synchronize(local)
    if world > 1:
        import torch.distributed as dist
        allreg = torch.empty(world * yn, dtype=torch.uint8, device=f"cuda:{local}")
        dist.all_gather_into_tensor(allreg, yt)
        regions = [allreg[r * yn:(r + 1) * yn].cpu().numpy() for r in range(world)]
    else:
        regions = [yt.cpu().numpy()]
    fx = ROOT / "tests" / "golden" / "gemm_sweep.json"
    bit_exact = None
    if rank == 0 and fx.exists():
        want = json.loads(fx.read_text())["sha256"]
        got = gemm_hashes(gemm_outputs(p, regions))
        bit_exact = got == want
        if not bit_exact:
            bit_exact = {k: got[k] == want.get(k) for k in got}

    # roofline: per-descriptor device times (graph captured with events between descriptors)
    st2, cop, gt = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
    check(L.tc_queue_capture(dev.h, p["q_main"], p["n_main"], 0, 0, 1, ctypes.byref(st2), ctypes.byref(cop),
                             ctypes.byref(gt)), dev.h)
    times = np.zeros(p["n_main"])
    reps = 3
    for _ in range(reps):
        check(L.tc_graph_launch(gt, None), dev.h)
        check(L.tc_synchronize(dev.h), dev.h)
        arr = (ctypes.c_float * p["n_main"])()
        check(L.tc_graph_times(gt, arr, p["n_main"]), dev.h, "graph_times")
        times += np.array(arr[:p["n_main"]]) / reps
    L.tc_graph_destroy(gt)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    i8 = 2 * peaks.get("bf16_tflops", 1590.0)
    cases = {}
    for t, m in zip(times, p["meta"]):
        if m is None:
            continue
        M, i, ops, wb = m
        c = cases.setdefault((M, i), [0.0, 0, 0])
        c[0] += t
        c[1] += ops
        c[2] += wb
    rows = []
    for (M, i), (t, ops, wb) in sorted(cases.items()):
        K, N, kb = p["shapes"][i]
        ideal = max(wb / (hbm * 1e9), ops / (i8 * 1e12)) * 1e3
        rows.append(dict(M=M, K=K, N=N // world, ms=round(t, 4), tops=round(ops / (t / 1e3) / 1e12, 1),
                         weight_gbs=round(wb / (t / 1e3) / 1e9, 1), roofline_frac=round(ideal / t, 3)))
    gemm_ms = sum(t for t, m in zip(times, p["meta"]) if m is not None)
    gemm_ops = sum(m[2] for m in p["meta"] if m is not None)
    achieved = gemm_ops / (gemm_ms / 1e3) / 1e12
    roofline = dict(bound="tensor", achieved=round(achieved, 1), peak=round(i8, 1), unit="TOPS",
                    frac=round(achieved / i8, 4), traffic=None,
                    kernel="k_mma_i8 (tcgen05 int8 GEMM) / k_gemv8 for M=4", kernel_ms_per_step=round(gemm_ms, 4),
                    peak_source="2 x measured bf16 burst (int8 dense = 2 x bf16 on B200)", cases=rows)

    # e2e through the board API: fp32 activations up from pinned memory, quantise + GEMMs, outputs back
    x0, xn = p["x_region"]
    for i in range(2):
        dev.to_dev(x0, xn)
        dev.run(p["q_setup"], p["n_setup"])
        dev.run(p["q_main"], p["n_main"])
        dev.from_dev(y0, yn)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        dev.to_dev(x0, xn)
        dev.run(p["q_setup"], p["n_setup"])
        dev.run(p["q_main"], p["n_main"])
        dev.from_dev(y0, yn)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = dict(value=round(p["ops"] / world * world * a.steps / e2e_s / 1e12, 2), unit="TOPS",
               h2d_bytes_per_step=xn, d2h_bytes_per_step=yn,
               api="opentars_b200.board.Cuda: to_dev, run (quant queue, GEMM queue), from_dev")
    if world > 1:
        e2e["note"] = "per-rank output blocks only (the all-gather runs in the device-timed steps)"
    dev.close()
    if rank != 0:
        return None
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic, seeded (config 1 distributions)",
        "config": gemm_config(world, a.gemm_gather, p["n_main"]),
        "roofline": roofline, "e2e": e2e, "gpu_launches": a.steps * kernels_per_step, "clocks": clk.summary(),
        "bit_exact_vs_reference": bit_exact,
    }
    if collective:
        out["collective"] = collective
    if world == 1 and not a.no_cpu:
        out["cpu_baseline"] = cpu_oracle_gemm(a.cpu_seconds, os.cpu_count() or 1)
    return out


def gemm_config(world: int, gather: str, n_main: int) -> dict:
    """The `config` of config 1's line (both arms print the same)."""
    return dict(workload="config1_w8a8_gemm_sweep", M=list(GEMM_M), shapes=[list(s) for s in GEMM_SHAPES],
                descriptors_per_step=n_main,
                parallelism=(f"the 151936-row vocabulary GEMM N-split over {world} GPUs (each keeps its "
                             f"output columns), the other shapes whole on every GPU"
                             + {"overlap": ", the split outputs all-gathered (NCCL, second stream) while "
                                           "the later segments compute",
                                "after": ", the split outputs all-gathered (NCCL) after the step's GEMMs",
                                "none": "; no collective in the timed steps (the outputs are gathered "
                                        "afterwards for the parity check)"}[gather]
                             if world > 1 else "1 GPU"),
                l2="weights (170 MB per step) larger than L2, streamed once per step")


def run_gemm_reference(a, world, rank) -> dict | None:
    if rank != 0:
        return None
    n_main = build_gemm(world, rank)["n_main"]
    procs = os.cpu_count() or 1
    vals = [cpu_oracle_gemm(a.ref_seconds, procs) for _ in range(a.warmup + a.steps)][a.warmup:]
    v = statistics.mean(x["value"] for x in vals)
    return {
        "impl": "reference", "metric": METRIC, "value": round(v, 6), "unit": "TOPS", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic, seeded",
        "config": gemm_config(world, a.gemm_gather, n_main),
        "cpu_baseline": dict(value=round(v, 6), unit="TOPS", cores=procs, kind="port", sample=vals[-1]["sample"]),
        "e2e": dict(value=round(v, 6), unit="TOPS", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
        "note": "the reference is Python (numpy golden model); its restatement in oracle/ is timed here",
    }


# ----------------------------------------------------------------------------- decode (configs 3 / 4)
DECODE_MODELS = {
    # name: (base config, layer types, vocab, fixture name)
    "decode": ("CFG_Q3_06B", None, "VOCAB_Q3_06B", "qwen3_0.6b"),
    "decode-gemma": ("CFG_G3_1B", "LAYERS_G3_1B", "VOCAB_G3_1B", "gemma3_1b"),
}
PROMPT_LEN, CHUNK, CONTEXT = 20, 4, 256


def prompt_ids(seed: int, vocab: int, n: int = PROMPT_LEN) -> list[int]:
    """Configs 3 / 4: a seeded prompt of n token ids uniform over the vocabulary."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def build_decode_model(workload: str):
    """The model lowered exactly as the reference lowers it (random weights, seed 0)."""
    from opentars_b200 import models as Mo
    from opentars_b200.model_image import ModelImage
    base, types, vocab_name, _ = DECODE_MODELS[workload]
    vocab = getattr(Mo, vocab_name)
    cfg = Mo.make_config(getattr(Mo, base), list(getattr(Mo, types)) if types else None, vocab=vocab)
    w = Mo.random_weights(cfg, seed=0, embed=True)
    return ModelImage(cfg, w, max_tokens=CONTEXT, ddr_bytes=3 << 29, head=True, queue_cap=8192)


_CPU: dict = {}


def _cpu_decode_prepare(low) -> None:
    """One decode step's queue (position 0) staged in the image, for the forked oracle workers."""
    tok = prompt_ids(0, low.vocab)[:1]
    ddr = low.p.ddr
    low.put_input(ddr, 0, low.embed(tok))
    a = len(low.p.descs)
    low.chunk(0, 1)
    q, n = low.stage(ddr, a, len(low.p.descs))
    _CPU.update(ddr=ddr, q=q, n=n, pos=0)


def _cpu_decode_tokens(seconds: float):
    """Whole decode steps of the oracle (a restatement of the reference's golden Machine) for at
    least `seconds`: (steps, elapsed)."""
    from oracle.machine import OracleMachine
    t0, k = time.perf_counter(), 0
    while True:
        assert OracleMachine(_CPU["ddr"], gemv_only=True).run_queue(_CPU["q"], _CPU["n"]).done
        k += 1
        if time.perf_counter() - t0 >= seconds:
            return k, time.perf_counter() - t0


def _cpu_decode_slice(count: int):
    """The next `count` descriptors of the decode queue, in order, cycling (the worker keeps its
    place between calls): (descriptors run, elapsed)."""
    from oracle.machine import OracleMachine
    q, n, pos = _CPU["q"], _CPU["n"], _CPU["pos"]
    t0 = time.perf_counter()
    done = 0
    while done < count:
        k = min(count - done, n - pos)
        assert OracleMachine(_CPU["ddr"], gemv_only=True).run_queue(q + 64 * pos, k).done
        pos = (pos + k) % n
        done += k
    _CPU["pos"] = pos
    return done, time.perf_counter() - t0


def _fork_pool(procs: int):
    import multiprocessing as mp
    return mp.get_context("fork").Pool(procs)     # forked before any CUDA context exists


def cpu_decode_baseline(procs: int, seconds: float) -> dict:
    with _fork_pool(procs) as pool:
        t0 = time.perf_counter()
        res = pool.map(_cpu_decode_tokens, [seconds] * procs, chunksize=1)
        wall = time.perf_counter() - t0
    toks = sum(k for k, _ in res)
    return dict(value=round(toks / wall, 4), unit="tok/s", cores=procs, kind="port",
                sample=f"{toks} whole decode steps (one token, one sequence, 1,910-descriptor queue at position 0) "
                       f"of the oracle on {procs} forked processes in {wall:.1f}s")


def run_decode(a, world, rank, local) -> dict | None:
    import torch
    t_build = time.perf_counter()
    low = build_decode_model(a.workload)
    build_s = time.perf_counter() - t_build
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:          # before the GPU is touched: fork is safe
        _cpu_decode_prepare(low)
        cpu = cpu_decode_baseline(os.cpu_count() or 1, a.cpu_seconds)
    os.environ["TC_DEVICE"] = str(local)
    torch.cuda.set_device(local)
    from opentars_b200.engine import DecodeEngine
    B = a.batch
    eng = DecodeEngine(low, batch=B, device=local)
    vocab = low.vocab
    prompts = np.array([prompt_ids(rank * B + b, vocab) for b in range(B)], np.int32)
    stream = torch.cuda.ExternalStream(_engine_stream(eng), device=local)

    def prefill():
        eng.reset()
        for s0 in range(0, PROMPT_LEN, CHUNK):
            eng.step(prompts[:, s0:s0 + CHUNK], CHUNK)
        return PROMPT_LEN

    # parity: sequence 0 of rank 0 is the committed reference fixture's prompt
    fx = None
    fpath = ROOT / "tests" / "golden" / "full_models.json"
    if rank == 0 and fpath.exists():
        fx = json.loads(fpath.read_text()).get(DECODE_MODELS[a.workload][3])
    pos = prefill()
    bit_exact = None
    if fx is not None and fx["prompt"] == prompts[0].tolist():
        import hashlib
        want = [r["logits_sha256"] for r in fx["runs"] if "logits_sha256" in r]
        got = []
        for i in range(len(want)):
            if i:
                eng.step(None)
                pos += 1
            got.append(hashlib.sha256(eng.logits()[0].astype("<f4").tobytes()).hexdigest())
        bit_exact = got == want

    def decode_steps(k: int, events: list | None = None):
        """k one-token steps; when the context is full the batch starts over (a prefill, outside
        the per-step events). With `events`, (position, start, end) of every step."""
        nonlocal pos
        for _ in range(k):
            if pos + 1 > CONTEXT:                         # context full: start the batch over
                pos = prefill()
            if events is None:
                eng.step(None)
            else:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record(stream)
                eng.step(None)
                ev[1].record(stream)
                events.append((pos, *ev))
            pos += 1

    decode_steps(a.warmup)
    pos = prefill()                                       # the timed steps start at the prompt's end
    eng.sync()
    barrier(world)
    events: list = []
    with Clocks(local) as clk:
        decode_steps(a.steps, events)
        eng.sync()
    step_ms = [(p_, e0.elapsed_time(e1)) for p_, e0, e1 in events]
    ms = sum(t for _, t in step_ms)
    barrier(world)
    ms_max = max_over_ranks(ms, world)
    value = world * B * a.steps / (ms_max / 1e3)
    at = {}
    for t in (32, 128, 250):                              # steps whose position is within 2 of t
        near = [ms_ for p_, ms_ in step_ms if abs(p_ - t) <= 2]
        at[str(t)] = round(statistics.mean(near), 4) if near else None

    # roofline: the step's GEMV kernels (the weight stream) from one profiled step
    if pos + 1 > CONTEXT:
        pos = prefill()
    prof = eng.profile()
    pos += 1
    kinds = {}
    for k, t, nb in prof:
        d = kinds.setdefault(k, [0, 0.0, 0])
        d[0] += 1
        d[1] += t
        d[2] += nb
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    g = kinds["gemv"]
    achieved = g[2] / (g[1] / 1e3) / 1e9
    tfile = ROOT / "profiles" / "traffic_decode.json"
    traffic = json.loads(tfile.read_text()).get("bytes_per_step") if tfile.exists() and a.workload == "decode" else None
    roofline = dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s", frac=round(achieved / peak, 4),
                    traffic=traffic, traffic_unit="DRAM bytes per step of the GEMM launches (ncu, B=64)",
                    kernel="k_mma_i8 (tcgen05 W8A8 GEMM; k_eng_gemv below 16 rows): all linears and the head",
                    kernel_bytes_per_step=g[2], kernel_launches_per_step=g[0], kernel_ms_per_step=round(g[1], 4),
                    peak_source="measured" if peaks else "fallback",
                    step_breakdown_ms={k: round(v[1], 4) for k, v in kinds.items()})
    gl = [(t, nb) for k, t, nb in prof if k == "gemv"]
    if len(gl) > 5:   # layer 0's four GEMMs and the head: [ms, algorithmic GB/s]
        roofline["gemv_layer0_and_head"] = [[round(t, 4), round(nb / (t / 1e3) / 1e9, 1)] for t, nb in gl[:4] + gl[-1:]]

    # e2e: the host in the loop as the reference's generate runs it: each step the token ids go up
    # from pinned memory and the greedy picks come back
    host_tok = torch.empty(B, dtype=torch.int32, pin_memory=True).numpy()
    pos = prefill()                                       # the same positions as the timed steps
    host_tok[:] = eng.tokens()
    eng.sync()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        if pos + 1 > CONTEXT:
            pos = prefill()
            host_tok[:] = eng.tokens()
        eng.set_tokens(host_tok)
        eng.step(None)
        pos += 1
        host_tok[:] = eng.tokens()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = dict(value=round(world * B * a.steps / e2e_s, 1), unit="tok/s", h2d_bytes_per_step=4 * B,
               d2h_bytes_per_step=4 * B, api="opentars_b200.engine.DecodeEngine: set_tokens, step, tokens")
    eng.close()
    # configs 0 and 2 beside it (the GEMV kernels alone): GB/s of algorithmic bytes
    units = {}
    if not a.decode_only:
        for key, wl in (("config0_gemv", "gemv"), ("config2_w4", "w4")):
            m = measure_units(wl, 0, 50, 5, world, rank, local, e2e_steps=20)
            units[key] = dict(value=round(m["value"], 1), unit="GB/s", ms_per_step=m["ms_per_step"],
                              roofline_frac=m["roofline"]["frac"], kernel_us=m["roofline"]["kernel_us"],
                              e2e_gbs=m["e2e"]["value"], bit_exact_unit0=m["bit_exact"], config=m["config"],
                              clocks=m["clocks"])
        if world == 1 and a.workload == "decode":
            # config 1 (the GEMM sweep) and config 4 (Gemma-3-1B decode, the first 40 positions)
            # on one GPU, so the default line carries every BASELINE config
            import copy
            ga = copy.copy(a)
            ga.steps, ga.warmup, ga.no_cpu = 20, 3, True
            gm = run_gemm(ga, world, rank, local)
            if gm is not None:
                units["config1_gemm"] = dict(value=gm["value"], unit=gm["unit"], ms_per_step=gm["ms_per_step"],
                                             roofline_frac=gm["roofline"]["frac"], e2e=gm["e2e"]["value"],
                                             bit_exact_vs_reference=gm["bit_exact_vs_reference"],
                                             config=gm["config"], clocks=gm["clocks"])
            da = copy.copy(a)
            da.workload, da.steps, da.warmup, da.no_cpu, da.decode_only = "decode-gemma", 40, 3, True, True
            dm = run_decode(da, world, rank, local)
            if dm is not None:
                units["config4_gemma3_decode"] = dict(
                    value=dm["value"], unit=dm["unit"], ms_per_step=dm["ms_per_step"],
                    ms_per_step_at_position=dm["ms_per_step_at_position"], e2e=dm["e2e"]["value"],
                    bit_exact_seq0_vs_reference=dm["bit_exact_seq0_vs_reference"], config=dm["config"],
                    clocks=dm["clocks"])
    if rank != 0:
        return None
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: random-init weights (seeded, the reference's random_weights), seeded prompts",
        "config": decode_config(a.workload, B, world, a.steps), "model_build_s": round(build_s, 1),
        "ms_per_step_at_position": at,
        "roofline": roofline, "e2e": e2e, "gpu_launches": a.steps * len(prof), "clocks": clk.summary(),
        "bit_exact_seq0_vs_reference": bit_exact,
    }
    for key, m in units.items():
        out[key] = m
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


# ----------------------------------------------------------------------------- Qwen3.5 text model
def run_qwen35(a, world, rank, local) -> dict | None:
    """Qwen3.5-0.8B shapes (18 gated-DeltaNet and 6 gated full-attention layers, vocab 248320,
    random-init seeded weights, its MTP head) on the descriptor path through the board runtime:
    the device time of one decode position's captured queue (one sequence, position PROMPT_LEN,
    replayed a.steps times - the work of that position, the recurrent state advancing each time),
    and of an MTP round (the 2-row verify chunk, then the MTP head over the known rows: two tokens
    when the draft is accepted, one when it is not). Parity of the same queues is pinned at small
    shapes by the reference's fixtures (models.json qwen35_small*, mtp.json)."""
    import ctypes

    import torch
    os.environ["TC_DEVICE"] = str(local)
    torch.cuda.set_device(local)
    from opentars_b200 import models as Mo
    from opentars_b200._lib import check, lib
    from opentars_b200.board import Cuda
    from opentars_b200.model_image import ModelImage
    t_build = time.perf_counter()
    cfg = Mo.make_config(Mo.CFG_08B, Mo.LAYERS_08B, Mo.VOCAB_08B)
    w = {**Mo.random_weights(cfg, seed=0, embed=True), **Mo.random_mtp(cfg)}
    low = ModelImage(cfg, w, max_tokens=CONTEXT, ddr_bytes=3 << 29, head=True, queue_cap=16384, verify_rows=2,
                     mtp=True)
    build_s = time.perf_counter() - t_build
    host = low.p.ddr
    L = lib()
    dev = Cuda(len(host), device=local, pinned=True)
    dev.mem[:] = np.frombuffer(host, np.uint8)
    dev.to_dev(0, len(host))

    def put(t0: int, toks) -> None:                    # input rows t0 .. up to the device
        low.put_input(host, t0, low.embed(toks))
        at = low.p.base + low.x0.off + t0 * low.x0.ld
        n = len(toks) * low.x0.ld
        dev.mem[at:at + n] = np.frombuffer(host, np.uint8, count=n, offset=at)
        dev.to_dev(at, n)

    def queue(record):                                 # the recorded descriptors, staged and uploaded
        a0 = len(low.p.descs)
        record()
        q, n = low.stage(host, a0, len(low.p.descs))
        dev.mem[q:q + 64 * n] = np.frombuffer(host, np.uint8, count=64 * n, offset=q)
        dev.to_dev(q, 64 * n)
        g, st = dev.graph(q, n)
        assert g is not None and st.done, "the queue must capture"
        return g, n

    stream = torch.cuda.ExternalStream(L.tc_stream(dev.h), device=local)

    def timed(graphs) -> float:                        # ms per replay of the graphs, in order
        for _ in range(a.warmup):
            for g in graphs:
                check(L.tc_graph_launch(g, None), dev.h)
        check(L.tc_synchronize(dev.h), dev.h)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            for g in graphs:
                check(L.tc_graph_launch(g, None), dev.h)
        e1.record(stream)
        check(L.tc_synchronize(dev.h), dev.h)
        return e0.elapsed_time(e1) / a.steps

    P = PROMPT_LEN
    prompt = [int(x) for x in np.random.default_rng(3).integers(0, Mo.VOCAB_08B, P)]
    n_pre = 0
    for t0 in range(0, P, CHUNK):                      # the prompt in chunks, as the board runtime feeds it
        n = min(CHUNK, P - t0)
        put(t0, prompt[t0:t0 + n])
        g_pre, k = queue(lambda: low.chunk(t0, n))
        n_pre += k
        check(L.tc_graph_launch(g_pre, None), dev.h)
    put(P, [prompt[-1]])
    g_dec, n_dec = queue(lambda: low.chunk(P, 1))
    ms_dec = timed([g_dec])
    # MTP: the head over the prompt, then rounds at position P (verify 2 rows, MTP over 2 or 1)
    g_m0, _ = queue(lambda: low.mtp_chunk(0, P))
    check(L.tc_graph_launch(g_m0, None), dev.h)
    put(P, [prompt[-1], prompt[0]])
    g_ver, n_ver = queue(lambda: low.chunk(P, 2, all_rows=True, parity=0, spec=True))
    g_hit, n_hit = queue(lambda: low.mtp_chunk(P, 2))
    g_miss, n_miss = queue(lambda: low.mtp_chunk(P, 1))
    ms_hit = timed([g_ver, g_hit])
    ms_miss = timed([g_ver, g_miss])
    kernels = check(L.tc_graph_kernels(g_dec), dev.h, "graph_kernels")
    dev.close()
    if rank != 0:
        return None
    return {
        "metric": METRIC, "value": round(1e3 / ms_dec, 1), "unit": "tok/s (one sequence)", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_dec, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: random-init weights (seeded, the reference's random_weights / random_mtp), seeded prompt",
        "config": dict(workload="f2_f3_qwen35_0.8b_decode_mtp", layers="18 gated DeltaNet + 6 gated attention",
                       position=P, path="descriptor queues (board runtime, captured graphs)",
                       descriptors=dict(decode=n_dec, verify=n_ver, mtp_hit=n_hit, mtp_miss=n_miss, prefill=n_pre)),
        "model_build_s": round(build_s, 1),
        "mtp": dict(ms_per_round_accepted=round(ms_hit, 4), tok_s_all_accepted=round(2e3 / ms_hit, 1),
                    ms_per_round_rejected=round(ms_miss, 4), tok_s_all_rejected=round(1e3 / ms_miss, 1)),
        "gpu_launches": a.steps * kernels,
        "parity": "the same queues at small shapes are pinned by tests/golden/models.json and mtp.json",
    }


# ----------------------------------------------------------------------------- Qwen3.5 vision tower
VISION_SIDE = 448                 # one 448 x 448 image: 28 x 28 patches of 16, 784 patches, 196 tokens


def run_vision(a, world, rank, local) -> dict | None:
    """The Qwen3.5-0.8B vision tower (12 blocks of hidden 768, 12 heads, the 2 x 2 merger to 1024)
    on one seeded 448 x 448 image per GPU: every linear is a W8A8 GEMM with M = 784 patch rows (the
    tensor-core kernel), attention is FDOT / softmax descriptors. A step = one image through the
    captured queue; value in merged visual tokens per second over all GPUs."""
    import ctypes

    import torch
    os.environ["TC_DEVICE"] = str(local)
    torch.cuda.set_device(local)
    from opentars_b200 import vision as OV
    from opentars_b200._lib import check, lib
    from opentars_b200.board import Cuda
    t_build = time.perf_counter()
    cfg = OV.vision_config()
    w = OV.random_vision(cfg, seed=0)
    img = np.random.default_rng(11 + rank).normal(0, 1, (cfg.in_channels, VISION_SIDE, VISION_SIDE)).astype(np.float32)
    px, grid = OV.patchify(img, cfg)
    pos, rope = OV.position_embeddings(cfg, w, grid), OV.rope_table(cfg, grid)
    tower = OV.VisionImage(cfg, w, patches_max=len(px), ddr_bytes=1 << 28)
    out = tower.emit(px, pos, rope)
    ddr, qa, qn = tower.p.finish()
    build_s = time.perf_counter() - t_build
    L = lib()
    dev = Cuda(len(ddr), device=local, pinned=True)
    dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
    dev.to_dev(0, len(ddr))
    g, st = dev.graph(qa, qn)
    assert g is not None and st.done, "the tower's queue must capture"
    kernels_per_step = check(L.tc_graph_kernels(g), dev.h, "graph_kernels")
    stream = torch.cuda.ExternalStream(L.tc_stream(dev.h), device=local)
    for _ in range(a.warmup):
        check(L.tc_graph_launch(g, None), dev.h)
    check(L.tc_synchronize(dev.h), dev.h)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(a.steps):
            check(L.tc_graph_launch(g, None), dev.h)
        e1.record(stream)
        check(L.tc_synchronize(dev.h), dev.h)
    ms_max = max_over_ranks(e0.elapsed_time(e1), world)
    ntok = out.rows
    value = world * ntok * a.steps / (ms_max / 1e3)
    # e2e: the image's patch, position and rotary rows (the first three tensors of the scratch)
    # up from pinned memory, the tower, the merged tokens back
    from opentars_b200.program import GRANULE
    x_lo = tower.p.base + tower.scratch0
    x_n = sum(-(-4 * a.size // GRANULE) * GRANULE for a in (px, pos, rope))
    y_lo, y_n = tower.p.base + out.off, out.rows * out.ld
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        dev.to_dev(x_lo, x_n)
        dev.run(qa, qn)
        dev.from_dev(y_lo, y_n)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    # where the image's time goes: the queue captured with events between descriptors (each time
    # includes a few microseconds of event overhead), summed per op kind and shape
    from opentars_b200 import contract as C
    from opentars_b200._lib import Status_t
    st2, cop, gt = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
    check(L.tc_queue_capture(dev.h, qa, qn, 0, 0, 1, ctypes.byref(st2), ctypes.byref(cop), ctypes.byref(gt)), dev.h)
    arr = (ctypes.c_float * qn)()
    for _ in range(2):
        check(L.tc_graph_launch(gt, None), dev.h)
        check(L.tc_synchronize(dev.h), dev.h)
    nt = check(L.tc_graph_times(gt, arr, qn), dev.h, "graph_times")
    L.tc_graph_destroy(gt)
    names = {C.OP_GEMM: "GEMM", C.OP_ROW: "ROW", C.OP_ELT: "ELT", C.OP_FDOT: "FDOT", C.OP_ROPE: "ROPE"}
    kinds: dict = {}
    for i in range(nt):
        d = C.decode(bytes(ddr[qa + 64 * i:qa + 64 * (i + 1)]))
        op = names.get(d["OPCODE"], str(d["OPCODE"]))
        if d["OPCODE"] == C.OP_FDOT:
            op += " NN" if d["CTRL"] & 1 else " NT"
        key = f"{op} {d['M']}x{d['N']}" + (f"x{d['K']}" if d["K"] else "")
        c, t = kinds.get(key, (0, 0.0))
        kinds[key] = (c + 1, t + arr[i])
    top = sorted(kinds.items(), key=lambda kv: -kv[1][1])[:8]
    descriptor_times = [[k, c, round(1e3 * t / c, 1)] for k, (c, t) in top]     # kind, count, us each
    gemm_ops = 2 * len(px) * sum(lin.n * lin.k for blk in tower.blocks for lin in
                                 (blk["qkv"], blk["proj"], blk["fc1"], blk["fc2"])) + \
        2 * ntok * (tower.m_fc1.n * tower.m_fc1.k + tower.m_fc2.n * tower.m_fc2.k) + 2 * len(px) * tower.pe.n * tower.pe.k
    dev.close()
    if rank != 0:
        return None
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "visual tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic: random-init tower weights (seeded, the reference's random_vision), a seeded image",
        "config": dict(workload="f4_qwen35_0.8b_vision_tower", image=f"{VISION_SIDE}x{VISION_SIDE}", patches=len(px),
                       merged_tokens=ntok, descriptors=qn, parallelism=f"one image per GPU x {world} GPUs",
                       model_build_s=round(build_s, 1)),
        "gemm_tops": round(gemm_ops * a.steps / (ms_max / 1e3) / 1e12, 2),
        "descriptor_us": {"top_kinds": descriptor_times, "note": "events between descriptors: kind, count, "
                          "microseconds each (a few of them event overhead)"},
        "e2e": dict(value=round(world * ntok * a.steps / e2e_s, 1), unit="visual tok/s", h2d_bytes_per_step=x_n,
                    d2h_bytes_per_step=y_n, api="opentars_b200.board.Cuda: to_dev (patch rows), run, from_dev"),
        "gpu_launches": a.steps * kernels_per_step, "clocks": clk.summary(),
        "parity": "the tower's queue and tokens are pinned to the reference at a small config "
                  "(tests/golden/vision.json, tests/test_gpu_vision.py)",
    }


def _engine_stream(eng) -> int:
    from opentars_b200.engine import lib as elib
    return elib().tc_engine_stream(eng.h)


def decode_config(workload: str, B: int, world: int, steps: int) -> dict:
    """The `config` of a decode line (both arms print the same): the timed steps decode positions
    PROMPT_LEN onwards, a full context starting the batch over."""
    last = PROMPT_LEN + steps
    span = (f"{PROMPT_LEN} -> {last}" if last <= CONTEXT else
            f"{PROMPT_LEN} -> {CONTEXT}, then again from {PROMPT_LEN} ({steps} steps)")
    return dict(workload=("config3_qwen3_0.6b_decode" if workload == "decode" else "config4_gemma3_1b_decode"),
                batch_per_gpu=B, prompt=PROMPT_LEN, prefill_chunk=CHUNK, context=CONTEXT,
                timed_positions=span + " (each step one token per sequence; a full context starts the batch "
                                       "over, untimed)",
                parallelism=f"independent sequences, {B} per GPU x {world} GPUs",
                l2="weights (596 MB Qwen3 / 1 GB Gemma-3) larger than L2, streamed once per step")


def run_decode_reference(a, world, rank) -> dict | None:
    """The reference arm for decode: the oracle's golden-Machine restatement on all host cores.
    Each step every worker runs the next 1/16 of a decode step's queue (cycling in order)."""
    if rank != 0:
        return None
    low = build_decode_model(a.workload)
    _cpu_decode_prepare(low)
    procs = os.cpu_count() or 1
    per = -(-_CPU["n"] // 16)
    vals = []
    with _fork_pool(procs) as pool:
        for i in range(a.warmup + a.steps):
            t0 = time.perf_counter()
            res = pool.map(_cpu_decode_slice, [per] * procs, chunksize=1)
            dt = time.perf_counter() - t0
            if i >= a.warmup:
                vals.append(sum(d for d, _ in res) / _CPU["n"] / dt)
    v = statistics.mean(vals)
    cfg = decode_config(a.workload, a.batch, world, a.steps)
    return {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic, seeded", "config": cfg,
        "cpu_baseline": dict(value=round(v, 4), unit="tok/s", cores=procs, kind="port",
                             sample=f"per step {procs} processes each run {per} descriptors of the decode queue "
                                    f"({_CPU['n']} per token), in order"),
        "e2e": dict(value=round(v, 4), unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0),
        "note": "the reference is Python (numpy golden model); its restatement in oracle/ is timed here",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: decode the whole context once, 236 steps; GEMV: 100)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode",
                    choices=sorted(WORKLOADS) + sorted(DECODE_MODELS) + ["gemm", "vision", "qwen35"])
    ap.add_argument("--batch", type=int, default=64, help="decode: sequences per GPU")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--units", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=3.0)
    ap.add_argument("--decode-only", action="store_true", help="decode: skip the config 0 / 2 keys")
    ap.add_argument("--gemm-gather", default="overlap", choices=["overlap", "after", "none"],
                    help="gemm on N GPUs: all-gather the vocabulary outputs after the step's GEMMs, "
                         "overlapped with the later segments, or not in the timed steps")
    a = ap.parse_args()
    if a.steps is None:
        a.steps = CONTEXT - PROMPT_LEN if a.workload in DECODE_MODELS else 100
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":                       # CPU only: no process group, no GPU
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        if a.workload == "gemm":
            out = run_gemm_reference(a, world, rank)
        elif a.workload in DECODE_MODELS:
            out = run_decode_reference(a, world, rank)
        else:
            out = run_reference(a, world, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    world, rank, local = dist_setup(a.gpus)
    if a.workload == "vision":
        out = run_vision(a, world, rank, local)
    elif a.workload == "qwen35":
        out = run_qwen35(a, world, rank, local)
    elif a.workload == "gemm":
        out = run_gemm(a, world, rank, local)
    elif a.workload in DECODE_MODELS:
        out = run_decode(a, world, rank, local)
    else:
        out = run_ours(a, world, rank, local)
    if out is not None:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
