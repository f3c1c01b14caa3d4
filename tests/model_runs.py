"""Shared drivers for the model-level parity tests: build a fixture's model with the package's
image builder (opentars_b200.model_image) and run its greedy decode through a given backend."""
from __future__ import annotations

import hashlib

import numpy as np


# fixture bases that are a named config with a few fields changed: name -> (config, changes)
DERIVED = {"G3_SMALL_K2": ("CFG_G3_SMALL", dict(intermediate_size=4608)),
           # the whole-context cases: the real head layouts of Qwen3-0.6B (16 q / 8 kv heads of 128)
           # and Gemma-3-1B (4 q / 1 kv head of 256, down_proj in two K blocks) on a narrow residual
           "Q3_HD128": ("CFG_Q3_06B", dict(hidden_size=256, intermediate_size=512)),
           "G3_HD256": ("CFG_G3_1B", dict(hidden_size=256, intermediate_size=4608)),
           # W4A16 needs K >= 256 on every linear: the per-layer-input projection's K is ple_dim
           "G4_SMALL_P256": ("CFG_G4_SMALL", dict(hidden_size_per_layer_input=256))}


def base_config(mod, name: str, rename: dict | None = None) -> dict:
    """The base config `name` of a fixture from module `mod` (opentars_b200.models, or the
    reference's qwen_ref with its own names in `rename`)."""
    rename = rename or {}
    if name in DERIVED:
        b, changes = DERIVED[name]
        return dict(getattr(mod, rename.get(b, b)), **changes)
    return getattr(mod, rename.get(name, name))


def build_image(fx: dict, full: bool = False):
    from opentars_b200 import models as Mo
    from opentars_b200.model_image import ModelImage as ModelImage
    if full:
        base = getattr(Mo, fx["base"])
        types = list(getattr(Mo, fx["types"])) if fx["types"] else None
        cfg = Mo.make_config(base, types, vocab=fx["vocab"])
        w = Mo.random_weights(cfg, seed=0, embed=True)
        return ModelImage(cfg, w, max_tokens=fx["T"], ddr_bytes=3 << 29, head=True, queue_cap=8192)
    cfg = Mo.make_config(base_config(Mo, fx["base"]), fx["types"], vocab=fx["vocab"])
    w = Mo.random_weights(cfg, seed=0, embed=True)
    return ModelImage(cfg, w, max_tokens=fx["T"], ddr_bytes=1 << 26, head=True, queue_cap=4096,
                        state_dtype=fx.get("state_dtype", "fp32"), wbits=fx.get("wbits", 8))


def build_export_image(fx: dict):
    """A fixture's small model with its embedding table rounded to bf16 (an export stores the table
    as bf16), for the export-format tests."""
    from opentars_b200 import models as Mo
    from opentars_b200.export import bf16_exact
    from opentars_b200.model_image import ModelImage as ModelImage
    cfg = Mo.make_config(base_config(Mo, fx["base"]), fx["types"], vocab=fx["vocab"])
    w = Mo.random_weights(cfg, seed=0, embed=True)
    w["embed_tokens.weight"] = bf16_exact(w["embed_tokens.weight"])
    if "embed_tokens_per_layer.weight" in w:
        w["embed_tokens_per_layer.weight"] = bf16_exact(w["embed_tokens_per_layer.weight"])
    return ModelImage(cfg, w, max_tokens=fx["T"], ddr_bytes=1 << 26, head=True, queue_cap=4096,
                        wbits=fx.get("wbits", 8))


class OracleDevice:
    """The CPU oracle as a board device (mem / to_dev / from_dev / run), as tars_board's Golden
    backend is the reference golden model: test infrastructure only."""
    params = dict(backend="oracle")

    def __init__(self, mem: int):
        self.buf = bytearray(mem)
        self.mem = np.frombuffer(self.buf, np.uint8)

    def to_dev(self, a, n):
        pass

    def from_dev(self, a, n):
        pass

    def run(self, q, n, timeout=None):
        from oracle.machine import OracleMachine
        m = OracleMachine(self.buf)
        st = m.run_queue(q, n)
        if m.ddr is not self.buf:
            self.mem[:] = np.frombuffer(bytes(m.ddr), np.uint8)
        return st.done, st.err_code, st.op_idx, 0


def mtp_oracle(plain_ids: list[int], vocab: int, seed: int = 2):
    """The draft replacement of the speculative tests: each draft at random the right token (plain
    decoding's next token) or a wrong one, so rounds both hit and miss."""
    rng = np.random.default_rng(seed)

    def oracle(t, d):
        right = rng.random() < 0.5 and t + 1 < len(plain_ids)
        return plain_ids[t + 1] if right else (plain_ids[min(t + 1, len(plain_ids) - 1)] + 1) % vocab
    return oracle


def build_mtp_image(fx: dict, **kw):
    """A tests/golden/mtp.json case's Qwen3.5 model (with the MTP head weights)."""
    from opentars_b200 import models as Mo
    from opentars_b200.model_image import ModelImage as ModelImage
    cfg = Mo.make_config(Mo.CFG_Q35_SMALL, fx["types"], vocab=fx["vocab"])
    w = {**Mo.random_weights(cfg, embed=True), **Mo.random_mtp(cfg)}
    return ModelImage(cfg, w, max_tokens=fx["T"], ddr_bytes=1 << 25, head=True, queue_cap=8192,
                        state_dtype=fx["state_dtype"], **kw)


def check_mtp(fx: dict, machine_cls) -> None:
    """Speculative decoding through machine_cls against the reference's run (mtp.json): the image,
    every queue, the tokens (those of plain decoding), every verified position's logits, the
    rounds and swap_state's queue."""
    low = build_mtp_image(fx, verify_rows=2, mtp=True)
    assert sha(low.p.ddr) == fx["image_sha256"]
    queues = []
    ids, lg, rounds = low.generate_mtp(machine_runner(machine_cls, queues, gemv_only=False), fx["prompt"],
                                       fx["new"], mtp_oracle(fx["plain_ids"], fx["vocab"]))
    assert queues == fx["queue_sha256"]
    assert ids == fx["ids"] and ids == fx["plain_ids"][:len(ids)]
    assert rounds == fx["rounds"]
    assert {str(k): logits_sha(v) for k, v in sorted(lg.items())} == fx["logits_sha256"]
    a = len(low.p.descs)
    low.swap_state()
    assert sha(b"".join(bytes(d) for d in low.p.descs[a:])) == fx["swap_sha256"]


def sha(a) -> str:
    return hashlib.sha256(bytes(a)).hexdigest()


def logits_sha(lg: np.ndarray) -> str:
    return hashlib.sha256(np.asarray(lg, "<f4").tobytes()).hexdigest()


def machine_runner(machine_cls, queues: list, gemv_only: bool = True):
    def run(ddr, q, n):
        queues.append(sha(ddr[q:q + 64 * n]))
        m = machine_cls(ddr, gemv_only=gemv_only)
        assert m.run_queue(q, n).done
        return m.ddr
    return run


class BoardRunner:
    """run(ddr, q, n) over the board backend: the image uploaded once, then per run only the
    input rows (Gemma 4: and the per-layer input rows) and the queue go up and the logits come
    back (as the board runtime moves data)."""

    def __init__(self, low, graphs: bool = True):
        from opentars_b200.board import Cuda
        self.low = low
        self.dev = Cuda(len(low.p.ddr), graphs=graphs, gemv_only=True)
        self.dev.mem[:] = np.frombuffer(bytes(low.p.ddr), np.uint8)
        self.dev.to_dev(0, len(low.p.ddr))
        self.queues = []

    def __call__(self, ddr, q, n):
        low, dev = self.low, self.dev
        x0, ld, T = low.p.base + low.x0.off, low.x0.ld, low.T
        dev.mem[x0:x0 + ld * T] = np.frombuffer(bytes(ddr[x0:x0 + ld * T]), np.uint8)
        dev.to_dev(x0, ld * T)
        if low.ple_dim:
            p0, pld = low.p.base + low.ple0.off, low.ple0.ld
            dev.mem[p0:p0 + pld * T] = np.frombuffer(bytes(ddr[p0:p0 + pld * T]), np.uint8)
            dev.to_dev(p0, pld * T)
        dev.mem[q:q + 64 * n] = np.frombuffer(bytes(ddr[q:q + 64 * n]), np.uint8)
        dev.to_dev(q, 64 * n)
        self.queues.append(sha(ddr[q:q + 64 * n]))
        done, err, op, _ = dev.run(q, n)
        assert done, (err, op)
        la = low.p.base + low.logits.off
        nb = 4 * low.vocab * low.verify_rows
        dev.from_dev(la, nb)
        ddr[la:la + nb] = dev.mem[la:la + nb].tobytes()
        return ddr
