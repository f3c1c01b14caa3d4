"""The package's model images (opentars_b200.model_image) against the reference's own lowering + golden
model (committed fixtures): identical DDR image, identical descriptor queues, identical logits,
run here through the CPU oracle."""
import json

import numpy as np
import pytest

from tests import fixtures as FX
from tests.model_runs import build_image, check_mtp, logits_sha, machine_runner, sha

MTP = json.loads((FX.GOLDEN / "mtp.json").read_text())


@pytest.mark.parametrize("name", sorted(FX.models()))
def test_lowering_matches_reference_small_models(name):
    from oracle.machine import OracleMachine
    fx = FX.models()[name]
    low = build_image(fx)
    assert sha(low.p.ddr) == fx["image_sha256"]
    queues = []
    ids, logits, counts = low.generate(machine_runner(OracleMachine, queues), fx["prompt"], fx["new"])
    assert queues == fx["queue_sha256"] and counts == fx["counts"]
    assert ids == fx["ids"]
    assert [logits_sha(lg) for lg in logits] == fx["logits_sha256"]


def test_chunked_prefill_equals_whole_prompt_logits():
    """Prefill in chunks of 4 ends at the same last-token logits as one prompt chunk (the
    reference pins chunk == single steps, test_v04.py:370-422)."""
    from oracle.machine import OracleMachine
    fx = FX.models()["qwen3_small"]
    a, b = build_image(fx), build_image(fx)
    ids1, lg1, _ = a.generate(machine_runner(OracleMachine, []), fx["prompt"], 2)
    ids2, lg2, _ = b.generate(machine_runner(OracleMachine, []), fx["prompt"], 2, chunk=4)
    assert ids1 == ids2
    assert all(np.array_equal(x.view(np.uint32), y.view(np.uint32)) for x, y in zip(lg1, lg2))


@pytest.mark.parametrize("name", sorted(MTP))
def test_mtp_speculative_decoding_matches_reference(name):
    """Qwen3.5 with the MTP head, drafts forced to hit and miss: the reference's queues, tokens
    (plain decoding's), verified logits, rounds and swap_state queue, through the CPU oracle."""
    from oracle.machine import OracleMachine
    check_mtp(MTP[name], OracleMachine)
