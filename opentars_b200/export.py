"""Writes a ModelImage as a board export directory - the file set that
tools/export_kv260.py:14-33 describes (the PLE fields: 234-237) and tars_board.py:212-435 (and board.Qwen) reads:

    image.bin        the DDR image from address 0: the zeroed state, the queue region, scratch,
                     the quantised weights
    embed_bf16.bin   the embedding table [vocab, H] as bf16 (the table must be bf16-exact)
    ple_bf16.bin     Gemma 4: the per-layer token table [vocab, L * ple_dim] as bf16 (bf16-exact),
                     scaled on the host by the manifest's ple_scale
    queues.bin       one descriptor queue per token position t (t0 = t, one token), back to back
    queues_c<n>.bin  prefill: one queue per chunk of n tokens at t0 = 0, align, 2 align, ...
    manifest.json    the addresses and sizes the runtime needs and the queue indexes

The queues are the model image's own chunk(t0, n) descriptors (byte-identical to the reference
lowering's), so an export of the same weights and configuration holds the same queues as the
reference exporter's. Checkpoint loading, the tokenizer files and the golden check of
expected.json belong to the reference's exporter and are not part of this writer.

    low = ModelImage(cfg, weights, max_tokens=T, head=True, queue_cap=4096)
    write_export(low, "out/")
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from . import contract as C


def bf16_exact(a: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (ties to even), as fp32: a table the export can
    store exactly."""
    b = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def write_export(low, out, chunks=(4,), align: int = 4, bos_ids=(), eos_ids=(), chat_prefix: str = "",
                 chat_suffix: str = "") -> dict:
    """Writes the export of `low` (a ModelImage built with head=True and a queue region) into
    `out`; returns the manifest. Every position 0 .. T-1 gets a one-token queue; chunk sizes in
    `chunks` get a queue at every t0 that is a multiple of `align` with t0 + n <= T."""
    if not low.head or not low.queue_cap:
        raise ValueError("the model image needs the head and a queue region (head=True, queue_cap > 0)")
    if low.p.base:
        raise ValueError("an export's image starts at address 0 (base_addr = 0)")
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    p = low.p
    emb = np.ascontiguousarray(low.w["embed_tokens.weight"], np.float32)
    bits = emb.view(np.uint32)
    if (bits & 0xFFFF).any():
        raise ValueError("the embedding table is not bf16-exact (round it with bf16_exact first)")
    (bits >> 16).astype("<u2").tofile(out / "embed_bf16.bin")
    if low.ple_dim:
        ple = np.ascontiguousarray(low.w["embed_tokens_per_layer.weight"], np.float32)
        pbits = ple.view(np.uint32)
        if (pbits & 0xFFFF).any():
            raise ValueError("the per-layer embedding table is not bf16-exact (round it with bf16_exact first)")
        (pbits >> 16).astype("<u2").tofile(out / "ple_bf16.bin")

    def queue(t0: int, n: int) -> tuple[bytes, int]:
        a = len(p.descs)
        low.chunk(t0, n)
        raw = b"".join(bytes(d) for d in p.descs[a:])
        del p.descs[a:]
        return raw, len(raw) // 64

    index, off = [], 0
    with open(out / "queues.bin", "wb") as f:
        for t in range(low.T):
            raw, k = queue(t, 1)
            f.write(raw)
            index.append([off, k])
            off += len(raw)
    chunk_index = {}
    for n in chunks:
        entries, off = [], 0
        with open(out / f"queues_c{n}.bin", "wb") as f:
            for t0 in range(0, low.T - n + 1, align):
                raw, k = queue(t0, n)
                f.write(raw)
                entries.append([t0, off, k])
                off += len(raw)
        chunk_index[str(n)] = entries
    image = bytes(p.ddr[:low.end])
    (out / "image.bin").write_bytes(image)
    m = dict(
        model_type=getattr(low.cfg, "model_type", ""), max_tokens=low.T, hidden=low.H, vocab=low.vocab,
        wbits=int(low.wbits), state_dtype="fp16" if (low.state_fmt == C.OUT_FP16 and "linear_attention" in low.types) else "fp32",
        keep_layers=bool(low.keep_layers),
        turn_end="<turn|>\n" if low.gemma4 else ("<end_of_turn>\n" if low.gemma else "<|im_end|>\n"),
        image_bytes=len(image), mem_bytes=len(image), state_end=int(low.qbase),
        x0_off=int(low.x0.off), x0_ld=int(low.x0.ld), qbase=int(low.qbase), queue_cap=int(low.queue_cap),
        logits_off=int(low.logits.off), head_blocks=[int(lin.n) for lin in low.head_lins],
        queue_index=index, chunks=chunk_index, bos_ids=list(bos_ids), eos_ids=list(eos_ids),
        chat_prefix=chat_prefix, chat_suffix=chat_suffix)
    if low.gemma:
        m["embed_scale"] = float(np.float32(low.H ** 0.5))
    if low.ple_dim:
        from .models import ple_embedding
        m.update(ple_cols=len(low.types) * low.ple_dim,
                 ple_scale=float(ple_embedding(low.cfg, np.ones((1, 1), np.float32))[0, 0]),
                 ple0_off=int(low.ple0.off), ple0_ld=int(low.ple0.ld))
    (out / "manifest.json").write_text(json.dumps(m))
    return m
