"""The Qwen3.5 vision tower (opentars_b200.vision) against the reference: the host tables against
the installed transformers tower's own computations (bit for bit); the lowered program - the
built DDR image, the queue - and its output on the CPU oracle against the reference's
VisionLowering run on its golden Machine (tests/golden/vision.json, made by
tests/golden/make_fixtures.py --models)."""
import hashlib
import json

import numpy as np
import pytest

from tests import fixtures as FX

VIS = json.loads((FX.GOLDEN / "vision.json").read_text())


def vit_image(size: int, seed: int = 3) -> np.ndarray:
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.arange(size), np.arange(size), indexing="ij")
    base = (np.sin(xx / 3.0) + np.cos(yy / 5.0))[:, :, None] / 2.0 + rng.normal(0, 0.3, (size, size, 3))
    return np.ascontiguousarray(base.transpose(2, 0, 1), np.float32)


@pytest.fixture(scope="module")
def tower():
    from opentars_b200 import vision as OV
    cfg = OV.vision_config(**VIS["config"])
    return cfg, OV.random_vision(cfg, seed=VIS["seed"])


def host_data(cfg, w, size):
    from opentars_b200 import vision as OV
    px, grid = OV.patchify(vit_image(size), cfg)
    return px, grid, OV.position_embeddings(cfg, w, grid), OV.rope_table(cfg, grid)


def _sha(*arrays):
    return hashlib.sha256(b"".join(np.asarray(a, "<f4").tobytes() for a in arrays)).hexdigest()


@pytest.mark.parametrize("grid", [[1, 2, 2], [1, 8, 8], [1, 4, 6], [1, 16, 16]])
def test_host_tables_equal_the_towers_own(tower, grid):
    """The position rows and the rotary rows equal what transformers' tower computes in its
    forward (fast_pos_embed_interpolate, rot_pos_emb then cos / sin), bit for bit."""
    import torch
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5VisionModel

    from opentars_b200 import vision as OV
    cfg, w = tower
    m = Qwen3_5VisionModel(cfg).eval()
    m.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()})
    g = torch.tensor([grid])
    with torch.no_grad():
        pe = m.fast_pos_embed_interpolate(g).numpy()
        ang = m.rot_pos_emb(g)
        rope = torch.cat([ang.cos(), ang.sin()], -1).numpy()
    assert np.array_equal(OV.position_embeddings(cfg, w, np.array([grid])), pe)
    assert np.array_equal(OV.rope_table(cfg, np.array([grid])), rope)


@pytest.mark.parametrize("size", sorted(VIS["images"], key=int))
def test_lowering_and_oracle_match_the_reference(tower, size):
    from oracle.machine import OracleMachine
    from opentars_b200 import vision as OV
    cfg, w = tower
    want = VIS["images"][size]
    px, _, pos, rope = host_data(cfg, w, int(size))
    assert len(px) == want["patches"] and _sha(px, pos, rope) == want["host_sha256"]
    low = OV.VisionImage(cfg, w, patches_max=len(px), ddr_bytes=1 << 23)
    one = low.run(px, pos, rope, blocks=1, machine=OracleMachine)
    tokens = low.run(px, pos, rope, machine=OracleMachine)
    ddr, q, n = low.p.finish()
    assert hashlib.sha256(bytes(ddr)).hexdigest() == want["image_sha256"] and [q, n] == want["queue"]
    assert _sha(one) == want["block1_sha256"]
    assert _sha(tokens) == want["tokens_sha256"]


def test_one_program_serves_a_smaller_image(tower):
    """The score-mask rows follow the image: a program sized for 64 patches gives the 4-patch
    image the tokens of the program sized for it."""
    from oracle.machine import OracleMachine
    from opentars_b200 import vision as OV
    cfg, w = tower
    px, _, pos, rope = host_data(cfg, w, 8)
    got = OV.VisionImage(cfg, w, patches_max=64, ddr_bytes=1 << 23).run(px, pos, rope, machine=OracleMachine)
    assert _sha(got) == VIS["images"]["8"]["tokens_sha256"]
