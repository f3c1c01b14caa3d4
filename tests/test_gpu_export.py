"""The board export runtime (board.Qwen) on the B200 device backend (board.Cuda) against the
reference's own board runtime's results over the same exports (tests/golden/export_ref.json):
per-run argmax and logits SHA-256, twice (the conversation state reset, the captured graphs
replayed)."""
import json

import pytest

from tests import fixtures as FX
from tests.model_runs import build_export_image
from tests.test_export import run_conversation

pytestmark = pytest.mark.gpu
REF = json.loads((FX.GOLDEN / "export_ref.json").read_text())


@pytest.mark.parametrize("name", sorted(REF))
def test_export_on_cuda_matches_the_reference_runtime(name, tmp_path):
    from opentars_b200.board import Cuda, Qwen, manifest_mem
    from opentars_b200.export import write_export
    write_export(build_export_image(FX.models()[name]), tmp_path)
    dev = Cuda(manifest_mem(tmp_path))
    model = Qwen(dev, tmp_path, log=lambda *a, **k: None)
    want = REF[name]["runs"]
    for _ in range(2):
        model.new_conversation()
        assert run_conversation(model, REF[name]["prompt"], len(want) - 1) == want
    dev.close()
