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
"""
from __future__ import annotations

import ctypes

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
        self._cache: dict[tuple[int, int], tuple[bytes, ctypes.c_void_p, Status_t]] = {}
        self._t0 = self._t1 = None

    # ------------------------------------------------------------------ memory
    def _ptr(self, a: int):
        return ctypes.c_void_p(self.buf.ctypes.data + a)

    def to_dev(self, a: int, n: int) -> None:
        check(lib().tc_upload(self.h, a, self._ptr(a), n), self.h, "to_dev")

    def from_dev(self, a: int, n: int) -> None:
        check(lib().tc_download(self.h, a, self._ptr(a), n), self.h, "from_dev")

    # ------------------------------------------------------------------ running a queue
    def graph(self, q: int, n: int):
        """The captured graph of the queue at q (captured on first use, or when its bytes changed)."""
        L = lib()
        key = (int(q), int(n))
        raw = self.buf[q:q + 64 * n].tobytes()
        hit = self._cache.get(key)
        if hit is not None and hit[0] == raw:
            return hit[1], hit[2]
        if hit is not None:
            L.tc_graph_destroy(hit[1])
        st, cop, g = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
        rc = L.tc_queue_capture(self.h, key[0], key[1], self.core_id, int(self.gemv_only), 0, ctypes.byref(st),
                                ctypes.byref(cop), ctypes.byref(g))
        if rc == TC_CONTRACT:
            raise ContractError(L.tc_last_error(self.h).decode())
        if rc != 0:
            return None, None                      # not capturable (e.g. the queue rewrites itself)
        self._cache[key] = (raw, g, st)
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
        for _, g, _ in self._cache.values():
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
