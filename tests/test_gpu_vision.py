"""The Qwen3.5 vision tower on the B200 through the drop-in Machine: the merged tokens of every
test image (4, 64 and 256 patches: the 64- and 256-row GEMMs run on the tensor cores) equal the
reference VisionLowering's on its golden Machine, bit for bit (tests/golden/vision.json)."""
import pytest

from tests.test_vision import VIS, _sha, host_data

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("size", sorted(VIS["images"], key=int))
def test_tower_on_the_gpu_matches_the_reference(size):
    from opentars_b200 import vision as OV
    from opentars_b200.machine import Machine
    cfg = OV.vision_config(**VIS["config"])
    w = OV.random_vision(cfg, seed=VIS["seed"])
    px, _, pos, rope = host_data(cfg, w, int(size))
    low = OV.VisionImage(cfg, w, patches_max=len(px), ddr_bytes=1 << 23)
    assert _sha(low.run(px, pos, rope, machine=Machine)) == VIS["images"][size]["tokens_sha256"]
    assert _sha(low.run(px, pos, rope, blocks=1, machine=Machine)) == VIS["images"][size]["block1_sha256"]
