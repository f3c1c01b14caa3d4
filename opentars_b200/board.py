"""The board runtime's device backend on a B200 (the `Cuda` twin of tars_board's Fpga / Golden).

Mirrors deploy/kv260/sw/tars_board.py:1-13, 155-178:

    dev = Cuda(mem_bytes)
    dev.mem[a:a + n] = ...      # numpy uint8 view of the host side of the image
    dev.to_dev(a, n)            # make host writes to [a, a + n) visible to the device
    dev.run(q, n)               # -> (done, err, op_idx, cycles)
    dev.from_dev(a, n)          # make the device's writes to [a, a + n) visible to the host

Unlike the drop-in Machine, nothing is diffed or copied implicitly: the caller moves exactly the
bytes it needs, as the board runtime already does. Each distinct queue (address, length,
descriptor bytes) is checked and captured once as a CUDA graph, then replayed. `cycles` is the
run's device time in 10 ns units (the board's 100 MHz cycle), so the runtime's cycles / 100e6
stays seconds.

`Qwen` is the board runtime's model over an export directory (tars_board.py:212-435): image.bin,
the per-position and prefill-chunk queues and the bf16 embedding table, run on any of these
devices (`Cuda`, or the reference's own devices, which have the same interface).
"""
from __future__ import annotations

import ctypes
import json
import time
from collections import OrderedDict
from pathlib import Path

import numpy as np

from ._lib import Status_t, TC_CONTRACT, check, lib
from .machine import ContractError, default_device


class Cuda:
    params = dict(backend="cuda (B200, libtarscuda)")

    def __init__(self, mem: int = 1 << 30, device: int | None = None, graphs: bool = True,
                 core_id: int = 0, gemv_only: bool = False, pinned: bool = False):
        self.device = default_device() if device is None else device
        self.n = int(mem)
        if pinned:                                   # page-locked host memory: direct DMA both ways
            import torch
            self._pinned = torch.zeros(self.n, dtype=torch.uint8, pin_memory=True)
            self.buf = self._pinned.numpy()
        else:
            self.buf = np.zeros(self.n, np.uint8)
        self.mem = self.buf
        self.core_id, self.gemv_only, self.graphs = core_id, gemv_only, graphs
        h = ctypes.c_void_p()
        if lib().tc_open(self.device, self.n, ctypes.byref(h)) != 0:
            raise RuntimeError(f"libtarscuda: cannot open a {self.n}-byte image on device {self.device}")
        self.h = h
        # captured graphs by (address, length, descriptor bytes), least recently used dropped first
        self._cache: OrderedDict[tuple[int, int, bytes], tuple[ctypes.c_void_p, Status_t]] = OrderedDict()
        self._t0 = self._t1 = None

    # ------------------------------------------------------------------ memory
    def _ptr(self, a: int):
        return ctypes.c_void_p(self.buf.ctypes.data + a)

    def to_dev(self, a: int, n: int) -> None:
        check(lib().tc_upload(self.h, a, self._ptr(a), n), self.h, "to_dev")

    def from_dev(self, a: int, n: int) -> None:
        check(lib().tc_download(self.h, a, self._ptr(a), n), self.h, "from_dev")

    # ------------------------------------------------------------------ running a queue
    GRAPHS = 512                                   # captured graphs kept (one per distinct queue)

    def graph(self, q: int, n: int):
        """The captured graph of the queue at q (captured on the first run of these descriptor bytes
        at this address; a runtime that stages each position's queue at the same address keeps one
        graph per position)."""
        L = lib()
        key = (int(q), int(n), self.buf[q:q + 64 * n].tobytes())
        hit = self._cache.get(key)
        if hit is not None:
            self._cache.move_to_end(key)
            return hit
        st, cop, g = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
        rc = L.tc_queue_capture(self.h, key[0], key[1], self.core_id, int(self.gemv_only), 0, ctypes.byref(st),
                                ctypes.byref(cop), ctypes.byref(g))
        if rc == TC_CONTRACT:
            raise ContractError(L.tc_last_error(self.h).decode())
        if rc != 0:
            return None, None                      # not capturable (e.g. the queue rewrites itself)
        self._cache[key] = (g, st)
        while len(self._cache) > self.GRAPHS:
            _, (old, _) = self._cache.popitem(last=False)
            L.tc_graph_destroy(old)
        return g, st

    def run(self, q: int, n: int, timeout: float | None = None) -> tuple[bool, int, int, int]:
        import torch
        L = lib()
        g, st = self.graph(q, n) if self.graphs else (None, None)
        stream = torch.cuda.ExternalStream(L.tc_stream(self.h), device=self.device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        if g is not None:
            check(L.tc_graph_launch(g, None), self.h, "run")
        else:
            st, cop = Status_t(), ctypes.c_int32(-1)
            rc = L.tc_run_queue(self.h, int(q), int(n), self.core_id, int(self.gemv_only), ctypes.byref(st),
                                ctypes.byref(cop))
            if rc == TC_CONTRACT:
                raise ContractError(L.tc_last_error(self.h).decode())
            check(rc, self.h, "run")
        t1.record(stream)
        check(L.tc_synchronize(self.h), self.h, "run")
        cycles = int(t0.elapsed_time(t1) * 1e5)    # ms -> 10 ns ticks
        return bool(st.done), int(st.err_code), int(st.op_idx), cycles

    def close(self) -> None:
        L = lib()
        for g, _ in self._cache.values():
            L.tc_graph_destroy(g)
        self._cache.clear()
        if self.h:
            L.tc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------- the model (an export directory)
ERRORS = {0: "OK", 1: "E_MAGIC", 2: "E_VERSION", 3: "E_CRC", 4: "E_VALID", 5: "E_OPCODE", 6: "E_FIELD",
          7: "E_ALIGN", 8: "E_RANGE"}


class Qwen:
    """The board runtime's model over an export directory (tars_board.py:212-435, the format of
    tools/export_kv260.py:14-33): image.bin loaded at address 0 of the device, one descriptor queue
    per token position (queues.bin, manifest queue_index) and prefill chunk queues
    (queues_c<n>.bin, manifest chunks), the bf16 embedding table (embed_bf16.bin). The host looks
    up the embeddings and takes the argmax; the device runs everything in between. A queue is
    staged at the manifest's qbase in parts of queue_cap descriptors.

        dev = Cuda(manifest_mem(data)); model = Qwen(dev, data)
        logits = model.prefill(prompt_ids); logits = model.step(token)

    Gemma 4 exports add the per-layer token table (ple_bf16.bin). Exports with speculative-decoding
    queues are refused."""

    def __init__(self, dev, data, log=print):
        self.dev, self.d = dev, Path(data)
        m = json.loads((self.d / "manifest.json").read_text())
        if m.get("spec"):
            raise ValueError(f"{self.d}: speculative-decoding queues are not supported")
        self.m = m
        self.T, self.H, self.vocab = int(m["max_tokens"]), int(m["hidden"]), int(m["vocab"])
        t = time.time()
        img = self.d / "image.bin"
        size = img.stat().st_size
        if size != m["image_bytes"]:
            raise RuntimeError(f"{img}: {size} bytes, the manifest says {m['image_bytes']}")
        if len(dev.mem) < max(size, int(m.get("mem_bytes", size))):
            raise RuntimeError(f"device buffer is {len(dev.mem) >> 20} MiB, the export needs "
                               f"{max(size, int(m.get('mem_bytes', size))) >> 20} MiB")
        with open(img, "rb") as f:                    # straight into the device's host buffer
            mv = memoryview(dev.mem)
            pos = 0
            while pos < size:
                k = f.readinto(mv[pos:min(size, pos + (64 << 20))])
                if not k:
                    raise IOError("short read of image.bin")
                pos += k
        dev.mem[size:] = 0
        dev.to_dev(0, len(dev.mem))
        self.state_end = int(m["state_end"])
        self.state0 = dev.mem[:self.state_end].copy() if np.any(dev.mem[:self.state_end]) else None
        self.embed = np.memmap(self.d / "embed_bf16.bin", np.uint16, "r", shape=(self.vocab, self.H))
        self.qidx = np.asarray(m["queue_index"], np.int64)         # [T, 2]: byte offset, descriptors
        self.queues = np.memmap(self.d / "queues.bin", np.uint8, "r")
        self.chunks = {}                                           # n -> (queues, {t0: (offset, count)})
        for n, index in m.get("chunks", {}).items():
            if (self.d / f"queues_c{n}.bin").exists():
                self.chunks[int(n)] = (np.memmap(self.d / f"queues_c{n}.bin", np.uint8, "r"),
                                       {int(t0): (int(o), int(k)) for t0, o, k in index})
        s = m.get("embed_scale")
        self.embed_scale = None if s is None else np.float32(s)
        self.ple_cols = int(m.get("ple_cols", 0))         # Gemma 4: per-layer token rows
        self.ple = np.memmap(self.d / "ple_bf16.bin", np.uint16, "r", shape=(self.vocab, self.ple_cols)) \
            if self.ple_cols else None
        self.ple_scale = np.float32(m["ple_scale"]) if self.ple_cols else None
        self.bos = [int(v) for v in m.get("bos_ids", [])]
        self.turn_end = m.get("turn_end", "<|im_end|>\n")
        self.cycles = 0
        self.pos = 0
        log(f"  ready in {time.time() - t:.1f} s ({size >> 20} MiB image, {self.T} positions, "
            f"prefill chunks {sorted(self.chunks) or 'none'})")

    def new_conversation(self) -> None:
        if self.state0 is None:
            self.dev.mem[:self.state_end] = 0
        else:
            self.dev.mem[:self.state_end] = self.state0
        self.dev.to_dev(0, self.state_end)
        self.pos = 0

    def encode(self, tk, text: str, chat: bool = True) -> list[int]:
        """Token ids of `text` at the next position (in the export's chat template with `chat`; a
        later turn first closes the model's turn; the BOS tokens at position 0)."""
        if chat:
            text = self.m["chat_prefix"] + text + self.m["chat_suffix"]
            if self.pos:
                text = self.turn_end + text
        ids = tk.encode(text, add_special_tokens=False).ids
        return (self.bos if self.pos == 0 else []) + ids

    def _put(self, t: int, tokens) -> None:
        """The input rows t, t + 1, ...: each token's bf16 embedding widened exactly (Gemma: times
        the manifest's fp32 embed_scale); Gemma 4 also writes the token's per-layer row (bf16
        widened, times ple_scale) at ple0 (tars_board.py:298-314)."""
        if t + len(tokens) > self.T:
            raise OverflowError(f"context full ({self.T} tokens)")
        x0, ld = int(self.m["x0_off"]), int(self.m["x0_ld"])
        for i, token in enumerate(tokens):
            x = (self.embed[int(token)].astype(np.uint32) << 16).view(np.float32)
            if self.embed_scale is not None:
                x = x * self.embed_scale
            a = x0 + (t + i) * ld
            self.dev.mem[a:a + 4 * self.H] = np.frombuffer(np.asarray(x, "<f4").tobytes(), np.uint8)
            self.dev.to_dev(a, 4 * self.H)
            if self.ple is not None:
                pr = (self.ple[int(token)].astype(np.uint32) << 16).view(np.float32) * self.ple_scale
                pa = int(self.m["ple0_off"]) + (t + i) * int(self.m["ple0_ld"])
                self.dev.mem[pa:pa + 4 * self.ple_cols] = np.frombuffer(np.asarray(pr, "<f4").tobytes(), np.uint8)
                self.dev.to_dev(pa, 4 * self.ple_cols)

    def _run(self, queues, off: int, n: int, what: str) -> int:
        q, cap, cyc = int(self.m["qbase"]), int(self.m["queue_cap"]), 0
        for s in range(0, n, cap):
            k = min(cap, n - s)
            self.dev.mem[q:q + 64 * k] = queues[off + 64 * s:off + 64 * (s + k)]
            self.dev.to_dev(q, 64 * k)
            done, err, op, c = self.dev.run(q, k)
            if not done or err:
                raise RuntimeError(f"{what}: the device stopped at descriptor {s + op} with error "
                                   f"{ERRORS.get(err, err)}")
            cyc += c
        return cyc

    def _logits(self) -> np.ndarray:
        lo = int(self.m["logits_off"])
        self.dev.from_dev(lo, 4 * self.vocab)
        return self.dev.mem[lo:lo + 4 * self.vocab].view(np.float32).copy()

    def step(self, token: int) -> np.ndarray:
        """`token` at the next position; returns the logits (fp32, vocab)."""
        t = self.pos
        self._put(t, [token])
        off, n = (int(v) for v in self.qidx[t])
        self.cycles = self._run(self.queues, off, n, f"position {t}")
        self.pos += 1
        return self._logits()

    def prefill(self, tokens, chunked: bool = True) -> np.ndarray:
        """`tokens` at the next positions; returns the logits after the last one. chunked: the
        largest chunk queue the export has for the position (bit-identical to single steps, the
        weights read once per chunk), single steps elsewhere."""
        tokens = [int(v) for v in tokens]
        if not tokens:
            raise ValueError("no tokens")
        i, cyc, lg = 0, 0, None
        while i < len(tokens):
            t = self.pos
            n = next((n for n in sorted(self.chunks, reverse=True)
                      if chunked and i + n <= len(tokens) and t in self.chunks[n][1]), 1)
            if n == 1:
                lg = self.step(tokens[i])
                cyc += self.cycles
            else:
                self._put(t, tokens[i:i + n])
                queues, index = self.chunks[n]
                off, k = index[t]
                cyc += self._run(queues, off, k, f"positions {t}..{t + n - 1}")
                self.pos += n
                lg = None
            i += n
        self.cycles = cyc
        return lg if lg is not None else self._logits()


def manifest_mem(data) -> int:
    """The device buffer an export needs (manifest mem_bytes, at least the image)."""
    m = json.loads((Path(data) / "manifest.json").read_text())
    return max(int(m["image_bytes"]), int(m.get("mem_bytes", 0)))
