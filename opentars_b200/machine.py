"""The golden executor's call surface on a B200: a drop-in for tars_mini.golden.Machine.

    from opentars_b200.machine import Machine, ContractError, Status
    m = Machine(ddr)                      # ddr: the caller's bytearray (the DDR image)
    st = m.run_queue(queue_addr, n)       # Status(done, err_code, op_idx); m.ddr mutated in place

Same constructor, attributes and errors as golden.py:41-56, 450-492: run_queue(queue_addr,
queue_len) -> Status, read(addr, n) / write(addr, data) on the host bytes, .ddr (the caller's own
object, updated in place), .status, .stats (list of OpStat), validate(raw) -> (err, fields), the
static strides / bstride / segments / extra_out, and ContractError for illegal programs (an
output overlapping an input) raised before that descriptor runs, earlier writes kept.

Execution happens in libtarscuda on the GPU: the image is mirrored in HBM, one mirror per
bytearray, reused by later Machines on the same bytearray. Before a run, every 64 KiB block the
host changed since the last sync is uploaded (so host writes between runs, e.g. a model image's
put_input, are seen); after it, every byte range the queue wrote is copied back into the caller's
bytearray. There is no CPU execution path.
"""
from __future__ import annotations

import ctypes
import os
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

from . import contract as C
from ._lib import OpStat_t, Seg_t, Status_t, TC_CONTRACT, check, lib


class ContractError(Exception):
    """An illegal program the compiler must not emit (golden.py:18-19)."""


@dataclass
class Status:
    """How a queue run ended: finished or not, the first error code, the op it stopped at."""
    done: bool = False
    err_code: int = C.E_OK
    op_idx: int = 0

    def __str__(self) -> str:
        return f"done={int(self.done)} err={C.ERR_NAMES[self.err_code]} op_idx={self.op_idx}"


@dataclass
class OpStat:
    opcode: int
    macs: int
    bytes_read: int
    bytes_written: int


def default_device() -> int:
    return int(os.environ.get("TC_DEVICE", os.environ.get("LOCAL_RANK", "0")))


class DeviceImage:
    """The HBM copy of one host DDR buffer and the shadow of the bytes it holds."""

    def __init__(self, host, device: int):
        self.host = host                                  # keeps the object (and its id) alive
        self.n = len(host)
        self.device = device
        h = ctypes.c_void_p()
        L = lib()
        rc = L.tc_open(device, self.n, ctypes.byref(h))
        if rc != 0:
            raise RuntimeError(f"libtarscuda: cannot open a {self.n}-byte image on CUDA device {device}")
        self.h = h
        self.shadow = np.zeros(self.n, np.uint8)          # tc_open zero-fills the image

    def host_ptr(self):
        return (ctypes.c_char * self.n).from_buffer(self.host)

    def close(self) -> None:
        if self.h:
            lib().tc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_IMAGES: OrderedDict[int, DeviceImage] = OrderedDict()
_MAX_IMAGES = int(os.environ.get("TC_MAX_IMAGES", "4"))


def image_for(ddr, device: int) -> DeviceImage:
    key = id(ddr)
    img = _IMAGES.get(key)
    if img is not None and (img.host is not ddr or img.n != len(ddr) or img.device != device):
        _IMAGES.pop(key).close()
        img = None
    if img is None:
        while len(_IMAGES) >= _MAX_IMAGES:
            _IMAGES.popitem(last=False)[1].close()
        img = DeviceImage(ddr, device)
        _IMAGES[key] = img
    _IMAGES.move_to_end(key)
    return img


def release_images() -> None:
    while _IMAGES:
        _IMAGES.popitem()[1].close()


def _fields_to_raw(d: dict) -> bytes:
    return C.encode({k: d[k] for k in C.LAYOUT}, fix_crc=False)


@dataclass
class Machine:
    """The drop-in executor: the caller's DDR bytearray, run on the GPU (golden.py:40-57 surface)."""
    ddr: bytearray
    core_id: int = 0
    gemv_only: bool = field(default_factory=lambda: os.environ.get("TM_GEMV_ONLY") == "1")
    status: Status = field(default_factory=Status)
    stats: list = field(default_factory=list)
    device: int = field(default_factory=default_device)

    # ------------------------------------------------------------------ memory (host bytes)
    def read(self, addr: int, n: int) -> bytes:
        return bytes(memoryview(self.ddr)[addr:addr + n])

    def write(self, addr: int, data: bytes) -> None:
        end = addr + len(data)
        self.ddr[addr:end] = data

    # ------------------------------------------------------------------ checks
    def validate(self, raw: bytes) -> tuple[int, dict]:
        f = (ctypes.c_uint64 * 23)()
        err = lib().tc_validate(bytes(raw), self.core_id, int(bool(self.gemv_only)), f)
        return err, dict(zip(C.FIELD_ORDER, (int(v) for v in f)))

    @staticmethod
    def bstride(d: dict) -> tuple[int, int]:
        """(row stride, dense row bytes) of an FDOT's B or an ELT's b operand."""
        if d["OPCODE"] != C.OP_FDOT:
            dense = 0 if d["HDR_RSV"] & 3 != C.BM_DENSE else 4 * d["N"]
        else:
            es = 2 if d["HDR_RSV"] & C.STATE_FP16 else 4
            dense = es * (d["N"] if d["CTRL"] & 1 else d["K"])
        ld = 16 * d["GROUP_SIZE"] or dense
        return ld, dense

    @staticmethod
    def strides(d: dict) -> tuple[int, int, int, int]:
        out, op = d["EPI"] >> 2 & 3, d["OPCODE"]
        w4 = op == C.OP_GEMM and d["CTRL"] & 7 == C.QM_GROUP and d["CTRL"] >> 8 & 15 == C.DT_INT4
        if w4:
            arow = (4 if d["CTRL"] >> 4 & 15 == C.DT_FP32 else 2) * d["K"]
        elif op == C.OP_GEMM:
            arow = d["K"]
        elif op in C.CONV_OPS:
            arow = C.conv_params(d)["Cin"]
        elif op == C.OP_FDOT:
            arow = 4 * d["K"]
        else:
            arow = (2 if op == C.OP_ELT and d["HDR_RSV"] & C.STATE_FP16 else 4) * d["N"]
        yrow = d["N"] * C.ESIZE.get(out, 4)
        return (16 * d["LDA16"] if d["LDA16"] else arow), (16 * d["LDY16"] if d["LDY16"] else yrow), arow, yrow

    @staticmethod
    def _footprint(d: dict) -> list:
        raw = _fields_to_raw(d)
        cap = 64
        segs = (Seg_t * cap)()
        n = ctypes.c_uint32()
        lib().tc_footprint(raw, segs, cap, ctypes.byref(n))
        out = []
        for s in segs[:n.value]:
            base = s.base_lo | (s.base_hi << 64)
            out.append((s.kind, [(base + i * s.ld, base + i * s.ld + s.nbytes) for i in range(s.count)]))
        return out

    @classmethod
    def segments(cls, d: dict):
        """([read segments per tensor], [one segment per output row]), golden.py:195-248."""
        fp = cls._footprint(d)
        reads = [segs for k, segs in fp if k >= 0]
        y = next(segs for k, segs in fp if k == -1)
        return reads, y

    @classmethod
    def extra_out(cls, d: dict):
        """ROW_QUANT's row scales (golden.py:250-256)."""
        return next((segs for k, segs in cls._footprint(d) if k == -2), [])

    # ------------------------------------------------------------------ the queue
    def run_queue(self, queue_addr: int, queue_len: int) -> Status:
        self.status, self.stats = Status(), []
        if queue_len <= 0:
            self.status = Status(True, C.E_OK, queue_len if queue_len > 0 else 0)
            return self.status
        if queue_addr + C.DESC_BYTES > len(self.ddr):
            self.status = Status(False, C.E_RANGE, 0)
            return self.status
        L = lib()
        img = image_for(self.ddr, self.device)
        hp = img.host_ptr()
        sp = img.shadow.ctypes.data_as(ctypes.c_void_p)
        check(L.tc_sync_up(img.h, hp, sp, img.n, None), img.h, "sync_up")
        st, cop = Status_t(), ctypes.c_int32(-1)
        qlen = min(int(queue_len), 0xFFFFFFFF)
        rc = L.tc_run_queue(img.h, int(queue_addr), qlen, int(self.core_id), int(bool(self.gemv_only)),
                            ctypes.byref(st), ctypes.byref(cop))
        msg = L.tc_last_error(img.h).decode()
        check(L.tc_sync_down(img.h, hp, sp), img.h, "sync_down")
        del hp
        ns = L.tc_stats(img.h, None, 0)
        arr = (OpStat_t * max(ns, 1))()
        L.tc_stats(img.h, arr, ns)
        self.stats = [OpStat(int(s.opcode), int(s.macs), int(s.bytes_read), int(s.bytes_written)) for s in arr[:ns]]
        if rc == TC_CONTRACT:
            raise ContractError(msg)
        check(rc, img.h, "run_queue")
        self.status = Status(bool(st.done), int(st.err_code), int(st.op_idx))
        return self.status


CudaMachine = Machine
