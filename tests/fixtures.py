"""Loading the committed golden fixtures (tests/golden/*, made by tests/golden/make_fixtures.py
from the reference implementation)."""
from __future__ import annotations

import functools
import gzip
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


@functools.lru_cache(None)
def queues() -> dict:
    with gzip.open(GOLDEN / "queues.json.gz", "rt") as f:
        return json.load(f)


@functools.lru_cache(None)
def numerics() -> dict:
    with np.load(GOLDEN / "numerics.npz") as z:
        return {k: z[k] for k in z.files}


@functools.lru_cache(None)
def models() -> dict:
    p = GOLDEN / "models.json"
    return json.loads(p.read_text()) if p.exists() else {}


def engine_models() -> dict:
    """The model fixtures the batched decode engine serves (Qwen3, Gemma 3: attention layers only;
    W8A8; Qwen3.5's DeltaNet layers, Gemma 4 and W4A16 models run through the descriptor path)."""
    return {k: v for k, v in models().items()
            if set(v["types"]) <= {"full_attention", "sliding_attention"} and "G4" not in v["base"]
            and v.get("wbits", 8) == 8}


def queue_params():
    """(set name, case) pairs for parametrisation."""
    q = queues()
    return [(name, c) for name, s in q.items() for c in s["cases"]]


def build(name: str, case: dict):
    from tests.golden import cases
    q = queues()[name]
    if name == "chains":
        return cases.build_chain(case["seed"])
    return cases.build_case(case["seed"], tuple(q["kinds"]), q["n_desc"], q["p_corrupt"])
