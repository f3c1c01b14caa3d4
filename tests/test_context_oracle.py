"""The whole-context fixtures (tests/golden/context.json: the reference's lowering and golden
Machine at the real head dims, T = 256) against the package's lowering and the CPU oracle: the same
DDR image, and the same logits for the first runs of each prompt fed one token per run. The GPU
engine is checked against every position up to 255 in tests/test_gpu_step.py."""
import json

import numpy as np
import pytest

from tests import fixtures as FX
from tests.model_runs import build_image, logits_sha, sha

CONTEXT = json.loads((FX.GOLDEN / "context.json").read_text())


@pytest.mark.parametrize("name", sorted(CONTEXT))
def test_context_fixture_oracle_first_positions(name):
    from oracle.machine import OracleMachine
    fx = CONTEXT[name]
    run = fx["runs"][0]
    low = build_image(dict(base=fx["base"], types=fx["types"], vocab=fx["vocab"], T=fx["T"]))
    assert sha(low.p.ddr) == fx["image_sha256"]
    P = len(run["prompt"])
    ddr, ids = low.p.ddr, list(run["prompt"])
    for t0 in range(P + 3):                            # the prompt one token per run, then 3 decode runs
        low.put_input(ddr, t0, low.embed(ids[t0:t0 + 1]))
        a = len(low.p.descs)
        low.chunk(t0, 1)
        q, cnt = low.stage(ddr, a, len(low.p.descs))
        m = OracleMachine(ddr, gemv_only=True)
        assert m.run_queue(q, cnt).done
        ddr = m.ddr
        if t0 >= P - 1:
            lg = low.logits_of(ddr)
            assert logits_sha(lg) == run["logits_sha256"][t0 - (P - 1)], t0
            assert int(np.argmax(lg)) == run["ids"][t0 + 1]
            ids.append(int(np.argmax(lg)))
