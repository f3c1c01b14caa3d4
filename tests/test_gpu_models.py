"""Whole-model decode on the GPU against the reference golden model's logits (committed fixtures),
bit for bit: small Qwen3 / Gemma 3 / Qwen3.5 (fp32 and fp16 DeltaNet state) models through the drop-in Machine and the board backend,
and the full-size Qwen3-0.6B / Gemma-3-1B shapes (configs 3 and 4) through the board backend."""
import pytest

from tests import fixtures as FX
from tests.model_runs import BoardRunner, build_image, logits_sha, machine_runner, sha

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(FX.models()))
def test_small_models_through_drop_in_machine(name):
    from opentars_b200.machine import Machine
    fx = FX.models()[name]
    low = build_image(fx)
    queues = []
    ids, logits, counts = low.generate(machine_runner(Machine, queues), fx["prompt"], fx["new"])
    assert queues == fx["queue_sha256"]
    assert ids == fx["ids"]
    assert [logits_sha(lg) for lg in logits] == fx["logits_sha256"]


@pytest.mark.parametrize("name", sorted(FX.models()))
def test_small_models_through_board_backend(name):
    fx = FX.models()[name]
    low = build_image(fx)
    run = BoardRunner(low)
    ids, logits, counts = low.generate(run, fx["prompt"], fx["new"])
    assert run.queues == fx["queue_sha256"]
    assert ids == fx["ids"]
    assert [logits_sha(lg) for lg in logits] == fx["logits_sha256"]
    run.dev.close()


@pytest.mark.parametrize("name", ["qwen35_mtp", "qwen35_mtp_fp16"])
def test_mtp_speculative_decoding_through_drop_in_machine(name):
    """Qwen3.5 with the MTP head (tests/golden/mtp.json): speculative decoding on the GPU gives the
    reference's queues, tokens, verified logits and rounds, bit for bit."""
    import json

    from opentars_b200.machine import Machine
    from tests.model_runs import check_mtp
    check_mtp(json.loads((FX.GOLDEN / "mtp.json").read_text())[name], Machine)


def _full():
    import json
    p = FX.GOLDEN / "full_models.json"
    return json.loads(p.read_text()) if p.exists() else {}


@pytest.mark.parametrize("name", ["qwen3_0.6b", "gemma3_1b"])
def test_full_size_model_logits_bit_exact(name):
    fx = _full().get(name)
    if fx is None:
        pytest.skip(f"no {name} fixture")
    low = build_image(fx, full=True)
    assert sha(low.p.ddr) == fx["image_sha256"]
    run = BoardRunner(low)
    ids, logits, counts = low.generate(run, fx["prompt"], fx["new"], chunk=fx["chunk"])
    want = [r for r in fx["runs"] if "logits_sha256" in r]
    assert run.queues == [r["queue_sha256"] for r in fx["runs"]]
    assert ids == fx["ids"]
    assert [logits_sha(lg) for lg in logits] == [r["logits_sha256"] for r in want]
    run.dev.close()
