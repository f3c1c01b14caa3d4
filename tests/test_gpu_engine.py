"""The batched decode engine against the reference golden model (committed fixtures) and the CPU
oracle, bit for bit per sequence: small Qwen3 / Gemma 3 models at batch 1 and 3, and the full-size
Qwen3-0.6B / Gemma-3-1B shapes (configs 3 and 4)."""
import json

import numpy as np
import pytest

from tests import fixtures as FX
from tests.model_runs import build_image, logits_sha, machine_runner

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(FX.engine_models()))
def test_engine_batch1_matches_reference_small(name):
    from opentars_b200.engine import DecodeEngine
    fx = FX.engine_models()[name]
    low = build_image(fx)
    eng = DecodeEngine(low, batch=1)
    ids, logits = eng.generate([fx["prompt"]], fx["new"], chunk=4)
    assert ids[0] == fx["ids"]
    assert [logits_sha(lg[0]) for lg in logits] == fx["logits_sha256"]
    eng.close()


@pytest.mark.parametrize("batch", [3, 33])
@pytest.mark.parametrize("name", sorted(FX.engine_models()))
def test_engine_batch_each_sequence_matches_oracle(name, batch):
    """Prompts decoded together (batch 33: the batched-GEMM path, two row blocks); each sequence
    equals its own single-sequence oracle run."""
    from opentars_b200.engine import DecodeEngine
    from oracle.machine import OracleMachine
    fx = FX.engine_models()[name]
    rng = np.random.default_rng(11)
    P = len(fx["prompt"])
    prompts = [fx["prompt"]] + [list(map(int, rng.integers(0, fx["vocab"], P))) for _ in range(batch - 1)]
    eng = DecodeEngine(build_image(fx), batch=batch)
    ids, logits = eng.generate(prompts, 3, chunk=4)
    eng.close()
    for b, pr in enumerate(prompts):
        low = build_image(fx)
        oids, ologits, _ = low.generate(machine_runner(OracleMachine, []), pr, 3, chunk=4)
        assert ids[b] == oids, b
        assert all(np.array_equal(lg[b].view(np.uint32), ol.view(np.uint32)) for lg, ol in zip(logits, ologits)), b


@pytest.mark.parametrize("name", sorted(FX.engine_models()))
def test_engine_three_launch_attention_matches_fused(name, monkeypatch):
    """TARSCUDA_FUSE_ATTN=0 (q / k norm + RoPE, attention and the output quantiser as three
    launches) and the default single cluster launch give the same tokens and logits bits."""
    from opentars_b200.engine import DecodeEngine
    fx = FX.engine_models()[name]
    rng = np.random.default_rng(5)
    P = len(fx["prompt"])
    prompts = [list(map(int, rng.integers(0, fx["vocab"], P))) for _ in range(5)]
    outs = []
    for fuse in ("1", "0"):
        monkeypatch.setenv("TARSCUDA_FUSE_ATTN", fuse)
        eng = DecodeEngine(build_image(fx), batch=5)
        ids, logits = eng.generate(prompts, 3, chunk=4)
        eng.close()
        outs.append((ids, [lg.view(np.uint32).copy() for lg in logits]))
    assert outs[0][0] == outs[1][0]
    assert all(np.array_equal(a, b) for a, b in zip(outs[0][1], outs[1][1]))


def _full():
    p = FX.GOLDEN / "full_models.json"
    return json.loads(p.read_text()) if p.exists() else {}


@pytest.mark.parametrize("name", ["qwen3_0.6b", "gemma3_1b"])
def test_engine_full_size_logits_bit_exact(name):
    """Config 3 / 4: the full-size model, batch 2 (the fixture's prompt and a second one); the
    fixture's sequence must reproduce the reference golden model's logits at every step."""
    from opentars_b200.engine import DecodeEngine
    fx = _full().get(name)
    if fx is None:
        pytest.skip(f"no {name} fixture")
    low = build_image(fx, full=True)
    rng = np.random.default_rng(5)
    prompts = [fx["prompt"], list(map(int, rng.integers(0, fx["vocab"], len(fx["prompt"]))))]
    eng = DecodeEngine(low, batch=2)
    ids, logits = eng.generate(prompts, fx["new"], chunk=fx["chunk"])
    eng.close()
    want = [r["logits_sha256"] for r in fx["runs"] if "logits_sha256" in r]
    assert ids[0] == fx["ids"]
    assert [logits_sha(lg[0]) for lg in logits] == want
