"""DDR images and descriptor queues of the tars_mini v0.4 contract, as the golden executor takes them.

An Image is a byte arena (tensors placed one after another on 128-byte boundaries, offset 0 left
unused) plus the list of descriptors recorded against it; finish() places the queue after the last
tensor. A Buf names a matrix inside the image (offset from the image base, shape, row stride in
bytes, element format); views of rows, columns or attention heads are Bufs too. The recording
methods take Bufs and fill the descriptor fields of tars_mini/contract.py:14-38 the way the golden
executor reads them (golden.py:59-435): row strides as 16-byte units (0 for dense rows), the row
scales of a QM_ROWCOL GEMM in HDR_RSV, the broadcast mode and fp16 state flag of an ELT in HDR_RSV.

The layout rule (a bump arena on 128-byte boundaries from offset 128) and the field encodings are
the contract's: images and queues built here are byte-identical to the reference's for the same
model (pinned by the committed fixtures).
"""
from __future__ import annotations

from typing import NamedTuple

import numpy as np

from . import contract as C

F32 = np.float32
GRANULE = 128


class Buf(NamedTuple):
    """A matrix in the image: offset from the image base, rows, columns, row stride (bytes), format."""
    off: int
    rows: int
    cols: int
    ld: int
    fmt: int = C.OUT_FP32

    @property
    def esize(self) -> int:
        return C.ESIZE[self.fmt]

    @property
    def row_bytes(self) -> int:
        return self.cols * self.esize

    def rows_at(self, r0: int, n: int) -> "Buf":
        return self._replace(off=self.off + r0 * self.ld, rows=n)

    def cols_at(self, c0: int, n: int) -> "Buf":
        return self._replace(off=self.off + c0 * self.esize, cols=n)

    def as_heads(self, width: int) -> "Buf":
        """Dense rows of several heads as one row per head."""
        assert self.ld == self.row_bytes and self.cols % width == 0
        return Buf(self.off, self.rows * (self.cols // width), width, width * self.esize, self.fmt)

    def column_of(self, j: int, width: int) -> "Buf":
        """Column block j of `width` columns, rows kept (a head of a [rows, heads * width] matrix)."""
        return self._replace(off=self.off + j * width * self.esize, cols=width)


class Linear(NamedTuple):
    """A quantised weight in the image: weight bytes, scales (fp32 per row, or fp16 per 128-group for
    W4), optional fp32 bias, output rows n, input columns k, weight bits."""
    w_off: int
    s_off: int
    b_off: int | None
    n: int
    k: int
    bits: int = 8


def stride16(ld: int, row_bytes: int) -> int:
    """A row-stride field: 0 for dense rows, else the stride in 16-byte units."""
    if ld == row_bytes:
        return 0
    if ld % 16 or ld < row_bytes:
        raise ValueError(f"row stride {ld} for rows of {row_bytes} bytes")
    return ld // 16


class Image:
    """A DDR image under construction and the descriptors recorded against it."""

    def __init__(self, size: int = 1 << 24, base: int = 0):
        self.base = base
        self.ddr = bytearray(base + size)
        self.top = GRANULE
        self.descs: list[bytes] = []
        self.queue_off: int | None = None

    # ---------------------------------------------------------------- placement
    def reserve(self, nbytes: int) -> int:
        off = self.top
        self.top = (off + nbytes + GRANULE - 1) // GRANULE * GRANULE
        if self.base + self.top > len(self.ddr):
            raise MemoryError(f"the image needs {self.top} bytes, it has {len(self.ddr) - self.base}")
        return off

    def store(self, array, dtype: str = "<f4") -> int:
        raw = np.ascontiguousarray(array).astype(dtype).tobytes()
        off = self.reserve(len(raw))
        self.ddr[self.base + off:self.base + off + len(raw)] = raw
        return off

    def matrix(self, rows: int, cols: int, fmt: int = C.OUT_FP32) -> Buf:
        es = C.ESIZE[fmt]
        return Buf(self.reserve(rows * cols * es), rows, cols, cols * es, fmt)

    def constant(self, values) -> Buf:
        """fp32 values as a matrix (a vector as one row)."""
        v = np.asarray(values, F32)
        if v.ndim < 2:
            v = v.reshape(1, -1)
        return Buf(self.store(v), v.shape[0], v.shape[1], 4 * v.shape[1])

    def finish(self) -> tuple[bytearray, int, int]:
        """Places the recorded queue after the tensors (once); returns (ddr, queue address, count)."""
        if self.queue_off is None:
            self.queue_off = self.reserve(C.DESC_BYTES * len(self.descs))
            at = self.base + self.queue_off
            for i, d in enumerate(self.descs):
                self.ddr[at + 64 * i:at + 64 * (i + 1)] = d
        return self.ddr, self.base + self.queue_off, len(self.descs)

    # ---------------------------------------------------------------- recording
    def _record(self, **fields) -> None:
        fields.update(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1, BASE_ADDR=self.base)
        self.descs.append(C.encode(fields))

    @staticmethod
    def _io(x: Buf, y: Buf, xbytes: int | None = None) -> dict:
        return dict(A_OFF=x.off, Y_OFF=y.off, LDA16=stride16(x.ld, x.row_bytes if xbytes is None else xbytes),
                    LDY16=stride16(y.ld, y.row_bytes))

    def row_op(self, fn: int, x: Buf, y: Buf, gamma: Buf | None = None, eps: float = 0.0, start: int = 0,
               scale_out: int = 0, beta: Buf | None = None) -> None:
        """OPCODE ROW (golden.py:358-380): fn over each row of fp32 x into y."""
        if x.fmt != C.OUT_FP32 or y.fmt == C.OUT_FP16 or (x.rows, x.cols) != (y.rows, y.cols):
            raise ValueError("a row op maps fp32 rows onto rows of the same shape")
        self._record(OPCODE=C.OP_ROW, CTRL=fn, EPI=C.epi(C.ACT_NONE, y.fmt, int(beta is not None)),
                     M=x.rows, N=x.cols, K=start, SCALE_OFF=scale_out if gamma is None else gamma.off,
                     BIAS_OFF=0 if beta is None else beta.off, W_OFF=0 if gamma is None else C.f32_bits(eps),
                     **self._io(x, y))

    def rms_norm(self, x: Buf, gamma: Buf, eps: float, y: Buf, l2: bool = False) -> None:
        self.row_op(C.ROW_L2NORM if l2 else C.ROW_RMSNORM, x, y, gamma, eps)

    def quantize(self, x: Buf, q: Buf | None = None, scales: int | None = None) -> tuple[Buf, int]:
        """ROW_QUANT of x: the int8 rows (a new matrix unless given) and their fp32 row scales."""
        if q is None:
            q = self.matrix(x.rows, x.cols, C.OUT_INT8)
        if scales is None:
            scales = self.reserve(4 * x.rows)
        self.row_op(C.ROW_QUANT, x, q, scale_out=scales)
        return q, scales

    def mm8(self, xq: Buf, srow: int, w: Linear, y: Buf, act: int = C.ACT_NONE) -> None:
        """W8A8 GEMM, QM_ROWCOL (golden.py:326-349): y = act(i2f(xq . w^T) * srow * scale [+ bias])."""
        if xq.fmt != C.OUT_INT8 or xq.cols != w.k or y.cols != w.n or srow % 16 or y.fmt == C.OUT_FP16:
            raise ValueError("mm8 operands")
        self._record(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_ROWCOL, fusion=int(act != C.ACT_NONE)),
                     EPI=C.epi(act, y.fmt, int(w.b_off is not None)), W_OFF=w.w_off, SCALE_OFF=w.s_off,
                     BIAS_OFF=w.b_off or 0, M=xq.rows, N=w.n, K=w.k, HDR_RSV=srow // 16, **self._io(xq, y))

    def mm4(self, x: Buf, w: Linear, y: Buf, act: int = C.ACT_NONE) -> None:
        """W4A16 GEMM, QM_GROUP (golden.py:295-324) on fp32 or bf16 activations."""
        if x.fmt not in (C.OUT_FP32, C.OUT_BF16) or x.cols != w.k or y.cols != w.n or w.bits != 4:
            raise ValueError("mm4 operands")
        if w.k < 256 or w.k % 256 or w.w_off % 128 or y.fmt == C.OUT_FP16:
            raise ValueError("mm4 needs K a multiple of 256 and 128-byte aligned weights")
        a_dt = C.DT_FP32 if x.fmt == C.OUT_FP32 else C.DT_BF16
        self._record(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_GROUP, a_dtype=a_dt, w_dtype=C.DT_INT4,
                                                   fusion=int(act != C.ACT_NONE)),
                     EPI=C.epi(act, y.fmt, int(w.b_off is not None)), W_OFF=w.w_off, SCALE_OFF=w.s_off,
                     BIAS_OFF=w.b_off or 0, M=x.rows, N=w.n, K=w.k, GROUP_SIZE=C.W4_GROUP, **self._io(x, y))

    def fdot(self, a: Buf, b: Buf, y: Buf, nn: bool) -> None:
        """FDOT (golden.py:426-435): y = a . b^T (NT) or a . b (NN), b fp32 or fp16 (NN)."""
        n_out, k_in = (b.cols, b.rows) if nn else (b.rows, b.cols)
        if k_in != a.cols or y.cols != n_out or y.rows != a.rows:
            raise ValueError("fdot operands")
        self._record(OPCODE=C.OP_FDOT, CTRL=int(nn), EPI=C.epi(C.ACT_NONE, y.fmt), W_OFF=b.off, M=a.rows,
                     N=n_out, K=a.cols, GROUP_SIZE=stride16(b.ld, b.row_bytes),
                     HDR_RSV=C.STATE_FP16 if b.fmt == C.OUT_FP16 else 0, **self._io(a, y))

    def elt(self, op: int, a: Buf, b: Buf, y: Buf, bmode: int = C.BM_DENSE, arow: bool = False,
            act: int = C.ACT_NONE, c: Buf | None = None) -> None:
        """ELT (golden.py:393-418): y = act(a) op b, b dense or broadcast (row, column, scalar); a
        may be one row for every output row (arow); MULADD adds c."""
        flags = bmode | (int(arow) << 2) | (C.STATE_FP16 if a.fmt == C.OUT_FP16 else 0)
        self._record(OPCODE=C.OP_ELT, CTRL=op, EPI=C.epi(act, y.fmt, int(c is not None)), A_OFF=a.off,
                     W_OFF=b.off, Y_OFF=y.off, BIAS_OFF=0 if c is None else c.off, M=y.rows, N=y.cols,
                     HDR_RSV=flags, GROUP_SIZE=stride16(b.ld, 4 * y.cols) if bmode == C.BM_DENSE else 0,
                     LDA16=0 if arow else stride16(a.ld, a.esize * y.cols), LDY16=stride16(y.ld, y.row_bytes))

    def activation(self, x: Buf, act: int, y: Buf) -> None:
        """The RELU opcode with an activation code (golden.py:351-356): y = act(x)."""
        self._record(OPCODE=C.OP_RELU, CTRL=0, EPI=C.epi(act, y.fmt), M=x.rows, N=x.cols, **self._io(x, y))

    def rotary(self, x: Buf, table: Buf, rows_per_pos: int, rot: int, y: Buf) -> None:
        """ROPE (golden.py:420-424) of the first `rot` columns; row r uses table row r // rows_per_pos."""
        self._record(OPCODE=C.OP_ROPE, CTRL=0, EPI=C.epi(C.ACT_NONE, y.fmt), W_OFF=table.off, M=x.rows, N=x.cols,
                     K=rot, GROUP_SIZE=rows_per_pos, **self._io(x, y))
