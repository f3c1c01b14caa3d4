"""Generate tests/golden/export_ref.json by running the REFERENCE's own board runtime over exports
written by opentars_b200.export.

Run in a container that holds the reference checkout (it is never needed at test time):

    PYTHONDONTWRITEBYTECODE=1 python -m tests.golden.make_export_fixture --ref <path to openTARS>

For each small fixture model (tests/golden/models.json; embedding rounded to bf16, as an export
stores it) the export directory is written to a temporary folder, loaded by the reference's
deploy/kv260/sw/tars_board.py `Qwen` on its `Golden` device (the reference golden Machine), and run
as the board runtime runs a conversation: prefill of the fixture's prompt (chunks of 4 where the
export has them), then greedy steps. Stored per model: the manifest's sizes, the SHA-256 of
image.bin, queues.bin and queues_c4.bin, and per run the argmax and the logits' SHA-256.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tests import fixtures as FX  # noqa: E402
from tests.model_runs import build_export_image  # noqa: E402

N_NEW = 4


def file_sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def run_reference(ref: str, data: str, prompt: list[int]) -> list[dict]:
    sys.path.insert(0, str(Path(ref) / "deploy" / "kv260" / "sw"))
    import tars_board as TB
    dev = TB.Golden(TB.manifest_mem(data))
    model = TB.Qwen(dev, data, log=lambda *a, **k: None)
    runs = []
    lg = model.prefill(prompt)
    for i in range(N_NEW + 1):
        tok = int(np.argmax(lg))
        runs.append(dict(pos=model.pos, argmax=tok,
                         logits_sha256=hashlib.sha256(np.asarray(lg, "<f4").tobytes()).hexdigest()))
        if i < N_NEW:
            lg = model.step(tok)
    return runs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference checkout")
    a = ap.parse_args()
    from opentars_b200.export import write_export
    out = {}
    for name, fx in sorted(FX.models().items()):
        low = build_export_image(fx)
        with tempfile.TemporaryDirectory() as d:
            m = write_export(low, d)
            dd = Path(d)
            out[name] = dict(
                image_bytes=m["image_bytes"], state_end=m["state_end"], qbase=m["qbase"], queue_cap=m["queue_cap"],
                x0_off=m["x0_off"], x0_ld=m["x0_ld"], logits_off=m["logits_off"],
                image_sha256=file_sha(dd / "image.bin"), queues_sha256=file_sha(dd / "queues.bin"),
                queues_c4_sha256=file_sha(dd / "queues_c4.bin"), prompt=fx["prompt"],
                runs=run_reference(a.ref, d, fx["prompt"]))
        print(name, [r["argmax"] for r in out[name]["runs"]], flush=True)
    (FX.GOLDEN / "export_ref.json").write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
