"""The board export format (opentars_b200.export writer, board.Qwen runtime) against the
reference's own board runtime: tests/golden/export_ref.json holds what the reference's tars_board
Qwen (Golden device, the reference golden Machine) computed over these exports - file hashes,
per-run argmax and logits SHA-256 (tests/golden/make_export_fixture.py). Here board.Qwen runs the
same export on the CPU oracle device."""
import hashlib
import json

import numpy as np
import pytest

from tests import fixtures as FX
from tests.model_runs import OracleDevice, build_export_image

REF = json.loads((FX.GOLDEN / "export_ref.json").read_text())


@pytest.fixture(scope="module", params=sorted(REF))
def export_dir(request, tmp_path_factory):
    from opentars_b200.export import write_export
    d = tmp_path_factory.mktemp(request.param)
    write_export(build_export_image(FX.models()[request.param]), d)
    return request.param, d


def _sha(p):
    return hashlib.sha256(p.read_bytes()).hexdigest()


def test_export_files_match_the_reference_fixture(export_dir):
    name, d = export_dir
    want = REF[name]
    m = json.loads((d / "manifest.json").read_text())
    for k in ("image_bytes", "state_end", "qbase", "queue_cap", "x0_off", "x0_ld", "logits_off"):
        assert m[k] == want[k], k
    assert _sha(d / "image.bin") == want["image_sha256"]
    assert _sha(d / "queues.bin") == want["queues_sha256"]
    assert _sha(d / "queues_c4.bin") == want["queues_c4_sha256"]


def run_conversation(model, prompt, n_new):
    runs = []
    lg = model.prefill(prompt)
    for i in range(n_new + 1):
        tok = int(np.argmax(lg))
        runs.append(dict(pos=model.pos, argmax=tok,
                         logits_sha256=hashlib.sha256(np.asarray(lg, "<f4").tobytes()).hexdigest()))
        if i < n_new:
            lg = model.step(tok)
    return runs


def test_runtime_on_the_oracle_matches_the_reference_runtime(export_dir):
    from opentars_b200.board import Qwen, manifest_mem
    name, d = export_dir
    model = Qwen(OracleDevice(manifest_mem(d)), d, log=lambda *a, **k: None)
    want = REF[name]["runs"]
    assert run_conversation(model, REF[name]["prompt"], len(want) - 1) == want
    model.new_conversation()                       # the state is reset: the same again
    assert run_conversation(model, REF[name]["prompt"], len(want) - 1) == want


def test_unchunked_prefill_gives_the_same_logits(export_dir):
    from opentars_b200.board import Qwen, manifest_mem
    name, d = export_dir
    prompt = REF[name]["prompt"]
    outs = []
    for chunked in (True, False):
        model = Qwen(OracleDevice(manifest_mem(d)), d, log=lambda *a, **k: None)
        outs.append(model.prefill(prompt, chunked=chunked).view(np.uint32))
    assert np.array_equal(outs[0], outs[1])


def test_runtime_refuses_mismatched_or_unsupported_exports(tmp_path, export_dir):
    import shutil

    from opentars_b200.board import Qwen
    _, d = export_dir
    bad = tmp_path / "bad"
    shutil.copytree(d, bad)
    m = json.loads((bad / "manifest.json").read_text())
    (bad / "manifest.json").write_text(json.dumps(dict(m, image_bytes=m["image_bytes"] + 64)))
    with pytest.raises(RuntimeError, match="image.bin"):
        Qwen(OracleDevice(m["image_bytes"] + 64), bad, log=lambda *a, **k: None)
    (bad / "manifest.json").write_text(json.dumps(dict(m, spec={"m1": []})))
    with pytest.raises(ValueError, match="speculative"):
        Qwen(OracleDevice(m["image_bytes"]), bad, log=lambda *a, **k: None)


def test_writer_refuses_what_an_export_cannot_hold(tmp_path):
    """write_export stores the embedding tables as bf16 and needs the head and a queue region."""
    from opentars_b200.export import bf16_exact, write_export
    from tests.model_runs import build_image
    low = build_image(FX.models()["qwen3_small"])             # fp32 embedding, not bf16-exact
    with pytest.raises(ValueError, match="bf16-exact"):
        write_export(low, tmp_path / "a")
    g4 = build_export_image(FX.models()["gemma4_small"])
    g4.w["embed_tokens_per_layer.weight"] = g4.w["embed_tokens_per_layer.weight"] + np.float32(1e-3)
    assert not np.array_equal(bf16_exact(g4.w["embed_tokens_per_layer.weight"]), g4.w["embed_tokens_per_layer.weight"])
    with pytest.raises(ValueError, match="per-layer"):
        write_export(g4, tmp_path / "b")
    low.head = False
    with pytest.raises(ValueError, match="head"):
        write_export(low, tmp_path / "c")
