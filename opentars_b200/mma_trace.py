"""Timeline of single tensor-core GEMM launches inside a decode step (a diagnostic).

`tc_mma_trace(k)` arms the k-th k_mma_i8 launch after the call: each of its CTAs records the
global timer at eight points (0 entry, 1 barriers and TMEM ready, 2 first token slice issued after
the dependency wait, 3 first full stage seen by the MMA issuer, 4 last MMA committed, 6 epilogue
done; split-K: 7 accumulator ready in the epilogue, 5 the peers' partial rows received;
persistent: 7 exit). `trace_step` runs one decode step of a DecodeEngine kernel by kernel (the
engine's profile mode: no graph, no programmatic launch overlap) once per armed launch and returns,
per launch, the event-timed duration and each point's min / median / max over the CTAs in
microseconds after the earliest entry.

    python -m opentars_b200.mma_trace --launches 1,2,3,4,113
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

import numpy as np

STAMPS = {0: "entry", 1: "ready", 2: "first_x_issued", 3: "first_stage_at_mma", 4: "last_mma",
          7: "acc_ready (split-K) / exit", 5: "peers_received (split-K)", 6: "epilogue_done"}
_CTAS, _PER = 2048, 8


def trace_step(eng, launches: list[int]) -> list[dict]:
    from ._lib import lib
    L = lib()
    out = []
    for k in launches:
        if L.tc_mma_trace(k, None, 0) != 0:
            raise RuntimeError("tc_mma_trace could not arm the trace")
        prof = eng.profile()
        buf = (ctypes.c_uint64 * (_CTAS * _PER))()
        n = L.tc_mma_trace(0, buf, _CTAS * _PER)
        if n < 0:
            raise RuntimeError("tc_mma_trace could not read the trace")
        a = np.frombuffer(buf, np.uint64)[:n].reshape(-1, _PER).astype(np.int64)
        a = a[a[:, 0] > 0]
        gemms = [t for kind, t, _ in prof if kind == "gemv"]
        rec = dict(launch=k, ctas=int(len(a)), event_us=round(gemms[k - 1] * 1e3, 2) if k <= len(gemms) else None)
        if len(a):
            t0 = a[:, 0].min()
            for i, name in STAMPS.items():
                col = a[:, i]
                col = col[col > 0]
                if len(col):
                    rel = (col - t0) / 1e3
                    rec[name] = [round(float(rel.min()), 2), round(float(np.median(rel)), 2), round(float(rel.max()), 2)]
        out.append(rec)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--launches", default="1,2,3,4", help="k_mma launches of the step to trace (1-based)")
    ap.add_argument("--batch", type=int, default=64)
    a = ap.parse_args()
    import torch

    from . import models as Mo
    from .engine import DecodeEngine
    from .model_image import ModelImage
    cfg = Mo.make_config(Mo.CFG_Q3_06B, None, vocab=Mo.VOCAB_Q3_06B)
    low = ModelImage(cfg, Mo.random_weights(cfg, seed=0, embed=True), max_tokens=256, ddr_bytes=3 << 29,
                       head=True, queue_cap=8192)
    os.environ.setdefault("TC_DEVICE", "0")
    torch.cuda.set_device(int(os.environ["TC_DEVICE"]))
    eng = DecodeEngine(low, batch=a.batch, device=int(os.environ["TC_DEVICE"]))
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, low.vocab, (a.batch, 20)).astype(np.int32)
    for s0 in range(0, 20, 4):
        eng.step(prompts[:, s0:s0 + 4], 4)
    for _ in range(3):
        eng.step(None)
    eng.sync()
    for rec in trace_step(eng, [int(x) for x in a.launches.split(",")]):
        print(json.dumps(rec))


if __name__ == "__main__":
    main()
