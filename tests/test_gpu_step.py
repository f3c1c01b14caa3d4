"""The fused decode step (one cooperative kernel per one-token step) against the reference and the
per-kernel engine path, bit for bit.

* The whole 256-token context at the real head dims (tests/golden/context.json, made by the
  reference's lowering and golden Machine): Qwen3's 16 q / 8 kv heads of 128 and Gemma 3's 4 q /
  1 kv head of 256 with 5 sliding layers to 1 full one, decoded to position 255, so the attention
  stages many K / V tiles. 40 sequences share a batch but join it at different steps (slot b
  restarts with tc_engine_reset_seq), so every step mixes positions; each sequence must reproduce
  the reference's logits at every position. Both engine paths are checked.
* Every sequence of a batch against the per-kernel path: the small fixture models at batch 5 and
  33, and the full-size Qwen3-0.6B / Gemma-3-1B shapes at batch 64 (configs 3 and 4), where the
  fixture's sequence must also reproduce the reference's logits.
"""
import functools
import hashlib
import json

import numpy as np
import pytest

from tests import fixtures as FX
from tests.model_runs import build_image, logits_sha

pytestmark = pytest.mark.gpu


@functools.lru_cache(None)
def _context() -> dict:
    return json.loads((FX.GOLDEN / "context.json").read_text())


def _full() -> dict:
    return json.loads((FX.GOLDEN / "full_models.json").read_text())


def _engine(low, batch, fused):
    from opentars_b200.engine import DecodeEngine
    eng = DecodeEngine(low, batch=batch)
    eng.fused(fused)
    assert eng.fused() == fused, eng.fused_why()
    return eng


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("name", ["qwen3_hd128", "gemma3_hd256"])
def test_whole_context_staggered_sequences_match_reference(name, fused):
    fx = _context()[name]
    runs, T = fx["runs"], fx["T"]
    P = len(runs[0]["prompt"])
    low = build_image(dict(base=fx["base"], types=fx["types"], vocab=fx["vocab"], T=T))
    assert hashlib.sha256(bytes(low.p.ddr)).hexdigest() == fx["image_sha256"]
    B = 40
    start = [3 * b for b in range(B)]                 # sequence b joins at step 3 b
    run_of = [runs[b % len(runs)] for b in range(B)]
    eng = _engine(low, B, fused)
    eng.reset()
    picks = np.zeros(B, np.int64)
    checked = 0
    for S in range(max(start) + T):
        tok = np.zeros(B, np.int32)
        for b in range(B):
            i = S - start[b]
            if i == 0 or i == T:
                eng.reset_seq(b)                      # join (or leave: idle from position 0)
            if 0 <= i < P:
                tok[b] = run_of[b]["prompt"][i]
            elif P <= i < T:
                tok[b] = picks[b]
        eng.step(tok.reshape(B, 1), 1)
        pos = eng.positions()
        lg = eng.logits()
        picks = eng.tokens()
        for b in range(B):
            i = S - start[b]
            if P - 1 <= i < T:
                assert pos[b] == i + 1
                r = run_of[b]
                assert logits_sha(lg[b]) == r["logits_sha256"][i - (P - 1)], (b, i)
                if i + 1 < T:
                    assert int(picks[b]) == r["ids"][i + 1], (b, i)
                checked += 1
    eng.close()
    assert checked == B * (T - P + 1)


@pytest.mark.parametrize("batch", [5, 33])
@pytest.mark.parametrize("name", sorted(FX.engine_models()))
def test_fused_step_equals_per_kernel_path(name, batch):
    fx = FX.engine_models()[name]
    rng = np.random.default_rng(21)
    P = len(fx["prompt"])
    prompts = [fx["prompt"]] + [list(map(int, rng.integers(0, fx["vocab"], P))) for _ in range(batch - 1)]
    outs = []
    for fused in (True, False):
        eng = _engine(build_image(fx), batch, fused)
        ids, logits = eng.generate(prompts, fx["new"], chunk=4)
        eng.close()
        outs.append((ids, [lg.view(np.uint32).copy() for lg in logits]))
    assert outs[0][0] == outs[1][0]
    assert all(np.array_equal(a, b) for a, b in zip(outs[0][1], outs[1][1]))
    assert outs[0][0][0] == fx["ids"]


@pytest.mark.parametrize("name", ["qwen3_0.6b", "gemma3_1b"])
def test_full_size_batch64_fused_equals_per_kernel_and_reference(name):
    """Configs 3 / 4 at the benched batch: all 64 sequences equal between the fused step and the
    per-kernel path at every step, and the fixture's sequence equals the reference."""
    fx = _full()[name]
    low = build_image(fx, full=True)
    rng = np.random.default_rng(5)
    prompts = [fx["prompt"]] + [list(map(int, rng.integers(0, fx["vocab"], len(fx["prompt"])))) for _ in range(63)]
    outs = []
    for fused in (True, False):
        eng = _engine(low, 64, fused)
        ids, logits = eng.generate(prompts, fx["new"], chunk=fx["chunk"])
        eng.close()
        outs.append((ids, logits))
    want = [r["logits_sha256"] for r in fx["runs"] if "logits_sha256" in r]
    assert outs[0][0][0] == fx["ids"]
    assert [logits_sha(lg[0]) for lg in outs[0][1]] == want
    assert outs[0][0] == outs[1][0]
    for a, b in zip(outs[0][1], outs[1][1]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_engine_refuses_steps_past_the_context_and_bad_tokens():
    from opentars_b200.engine import DecodeEngine
    fx = FX.engine_models()["qwen3_small"]
    low = build_image(fx)
    eng = DecodeEngine(low, batch=2)
    eng.reset()
    with pytest.raises(RuntimeError):
        eng.step(np.array([[0], [fx["vocab"]]], np.int32), 1)      # id outside the vocabulary
    for _ in range(fx["T"]):
        eng.step(np.zeros((2, 1), np.int32), 1)
    with pytest.raises(RuntimeError):
        eng.step(np.zeros((2, 1), np.int32), 1)                   # position T would pass max_tokens
    eng.reset_seq(1)
    assert list(eng.positions()) == [fx["T"], 0]
    eng.close()
