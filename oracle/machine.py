"""CPU oracle, part 3: the golden executor (tars_mini/golden.py) restated over a DDR bytearray.

TEST INFRASTRUCTURE ONLY (see oracle/numerics.py's header for who may use it).

OracleMachine has the call surface of the reference's golden Machine (golden.py:41-56,
450-492): run_queue(queue_addr, queue_len) -> Status, read/write, .ddr (mutated in place),
.status, .stats; validate(raw) and the static strides/bstride/segments/extra_out.
"""
from __future__ import annotations

import bisect
from dataclasses import dataclass, field

import numpy as np

from . import contract as C
from . import numerics as F


class ContractError(Exception):
    """golden.py:18-19 - an illegal program (an output overlapping an input, or two outputs)."""


@dataclass
class Status:
    done: bool = False
    err_code: int = C.E_OK
    op_idx: int = 0


@dataclass
class OpStat:
    opcode: int
    macs: int
    bytes_read: int
    bytes_written: int


def is_w4(d: dict) -> bool:
    return d["OPCODE"] == C.OP_GEMM and d["CTRL"] & 7 == C.QM_GROUP and d["CTRL"] >> 8 & 15 == C.DT_INT4


def check(d: dict, raw: bytes, core_id: int, gemv_only: bool) -> int:
    """golden.py:59-169 - the first failing check in contract order, or E_OK."""
    if d["MAGIC"] != C.MAGIC:
        return C.E_MAGIC
    if d["VERSION"] != C.VERSION:
        return C.E_VERSION
    if not C.crc_ok(raw):
        return C.E_CRC
    if d["VALID"] != 1:
        return C.E_VALID
    op = d["OPCODE"]
    if op not in (C.OP_GEMM, C.OP_RELU, C.OP_ROW) + C.CONV_OPS + C.V04_OPS:
        return C.E_OPCODE
    if gemv_only and (op in C.CONV_OPS or (op == C.OP_GEMM and d["K"] > 4096)):
        return C.E_OPCODE
    conv = op in C.CONV_OPS
    c, e = d["CTRL"], d["EPI"]
    qm, sym, adt, wdt, fus = c & 7, c >> 3 & 1, c >> 4 & 15, c >> 8 & 15, c >> 12 & 1
    act, out, bias = C.act_of(e), e >> 2 & 3, e >> 4 & 1
    w4 = is_w4(d)
    hdr_ok = conv or (op == C.OP_GEMM and qm == C.QM_ROWCOL and not w4) \
        or (op == C.OP_ELT and d["HDR_RSV"] < 16) \
        or (op == C.OP_FDOT and c & 1 and d["HDR_RSV"] == C.STATE_FP16)
    grp_ok = conv or op in C.V04_OPS or w4
    if d["CORE_ID"] != core_id or d["DEP_SIG"] or (d["HDR_RSV"] and not hdr_ok) \
            or (d["GROUP_SIZE"] and not grp_ok):
        return C.E_FIELD
    if c >> 13 or e >> 6 or (out == C.OUT_FP16 and op != C.OP_ELT):
        return C.E_FIELD
    if out != C.OUT_INT8 and d["OUT_SCALE"]:
        return C.E_FIELD
    gemm = op == C.OP_GEMM or conv
    if gemm:
        if w4:
            if sym != 1 or adt not in (C.DT_FP32, C.DT_BF16) or d["HDR_RSV"] != 0 \
                    or d["GROUP_SIZE"] != C.W4_GROUP:
                return C.E_FIELD
        elif qm not in (C.QM_TENSOR, C.QM_CHANNEL, C.QM_ROWCOL) or sym != 1 \
                or adt != C.DT_INT8 or wdt != C.DT_INT8 or (conv and qm == C.QM_ROWCOL):
            return C.E_FIELD
        if (act != C.ACT_NONE) != (fus == 1):
            return C.E_FIELD
        if op == C.OP_CONV_ACT and act == C.ACT_NONE:
            return C.E_FIELD
        if conv:
            g = C.conv_params(d)
            if not (g["H"] and g["W"] and g["KH"] and g["KW"]) or g["OH"] < 1 or g["OW"] < 1 \
                    or d["M"] != g["OH"] * g["OW"]:
                return C.E_FIELD
    elif op == C.OP_RELU:
        if c or bias or d["K"] or d["W_OFF"] or d["SCALE_OFF"] or d["BIAS_OFF"] or act == C.ACT_NONE:
            return C.E_FIELD
    elif op == C.OP_ROW:
        fn = c & 7
        if c >> 3 or fn > C.ROW_QUANT or act != C.ACT_NONE or (d["K"] and fn != C.ROW_SOFTMAX):
            return C.E_FIELD
        if fn == C.ROW_SOFTMAX and (bias or d["W_OFF"] or d["SCALE_OFF"] or d["BIAS_OFF"]):
            return C.E_FIELD
        if fn == C.ROW_QUANT and (bias or d["W_OFF"] or d["BIAS_OFF"] or out != C.OUT_INT8 or d["OUT_SCALE"]):
            return C.E_FIELD
        if not bias and d["BIAS_OFF"]:
            return C.E_FIELD
    elif op == C.OP_ELT:
        eop = c & 3
        if c >> 2 or d["K"] or d["SCALE_OFF"] or bias != (eop == C.ELT_MULADD) \
                or (eop == C.ELT_MULADD and out not in (C.OUT_FP32, C.OUT_FP16)) or (not bias and d["BIAS_OFF"]):
            return C.E_FIELD
    elif op == C.OP_ROPE:
        if c or act != C.ACT_NONE or bias or d["SCALE_OFF"] or d["BIAS_OFF"] or d["GROUP_SIZE"] == 0:
            return C.E_FIELD
    else:
        if c >> 1 or act != C.ACT_NONE or bias or d["SCALE_OFF"] or d["BIAS_OFF"]:
            return C.E_FIELD
    M, N, K = d["M"], d["N"], d["K"]
    if M == 0 or N == 0 or N % 16 or ((gemm or op == C.OP_FDOT) and (K == 0 or K % 16)):
        return C.E_ALIGN
    if w4 and (K < 256 or K % 256 or K > 8192 or d["W_OFF"] % 128):
        return C.E_ALIGN
    if op == C.OP_ROPE and (K == 0 or K % 32 or K > N):
        return C.E_ALIGN
    if conv:
        g = C.conv_params(d)
        if K % (g["KH"] * g["KW"]) or g["Cin"] % 16:
            return C.E_ALIGN
    offs = ("A_OFF", "Y_OFF", "SCALE_OFF", "BIAS_OFF") + (() if op == C.OP_ROW else ("W_OFF",))
    for o in offs:
        al = 4 if (o == "W_OFF" and op == C.OP_ELT and d["HDR_RSV"] & 3 in (C.BM_COL, C.BM_SCALAR)) else 16
        if d[o] % al:
            return C.E_ALIGN
    lda, ldy, arow, yrow = strides(d)
    if lda < arow or ldy < yrow:
        return C.E_ALIGN
    if op in (C.OP_ELT, C.OP_FDOT):
        ldb, brow = bstride(d)
        if ldb < brow:
            return C.E_ALIGN
    return C.E_OK


def bstride(d: dict) -> tuple[int, int]:
    """golden.py:171-178."""
    if d["OPCODE"] == C.OP_FDOT:
        brow = (2 if d["HDR_RSV"] & C.STATE_FP16 else 4) * (d["N"] if d["CTRL"] & 1 else d["K"])
    else:
        brow = 4 * d["N"] if (d["HDR_RSV"] & 3) == C.BM_DENSE else 0
    return (16 * d["GROUP_SIZE"] if d["GROUP_SIZE"] else brow), brow


def strides(d: dict) -> tuple[int, int, int, int]:
    """golden.py:180-193 - (lda, ldy, input row bytes, output row bytes)."""
    out = d["EPI"] >> 2 & 3
    op = d["OPCODE"]
    if is_w4(d):
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


def segments(d: dict):
    """golden.py:195-248 - ([read segments per tensor], [write segment per output row])."""
    B, M, N, K = d["BASE_ADDR"], d["M"], d["N"], d["K"]
    lda, ldy, arow, yrow = strides(d)

    def rows(off, ld, nb, count=None):
        return [(B + off + m * ld, B + off + m * ld + nb) for m in range(M if count is None else count)]

    y = rows(d["Y_OFF"], ldy, yrow)
    op = d["OPCODE"]
    if op in C.V04_OPS:
        if op == C.OP_ELT and d["HDR_RSV"] >> 2 & 1:
            reads = [[(B + d["A_OFF"], B + d["A_OFF"] + arow)]]
        else:
            reads = [rows(d["A_OFF"], lda, arow)]
        w0 = B + d["W_OFF"]
        if op == C.OP_ELT:
            bm = d["HDR_RSV"] & 3
            if bm == C.BM_DENSE:
                ldb = bstride(d)[0]
                reads.append([(w0 + m * ldb, w0 + m * ldb + 4 * N) for m in range(M)])
            else:
                reads.append([(w0, w0 + {C.BM_ROW: 4 * N, C.BM_COL: 4 * M, C.BM_SCALAR: 4}[bm])])
            if d["CTRL"] & 3 == C.ELT_MULADD:
                reads.append(rows(d["BIAS_OFF"], ldy, yrow))
        elif op == C.OP_ROPE:
            reads.append([(w0, w0 + 4 * K * ((M - 1) // d["GROUP_SIZE"] + 1))])
        else:
            ldb, brow = bstride(d)
            nb = K if d["CTRL"] & 1 else N
            reads.append([(w0 + i * ldb, w0 + i * ldb + brow) for i in range(nb)])
        return reads, y
    if op in C.CONV_OPS:
        npx = C.conv_params(d)["H"] * C.conv_params(d)["W"]
        a0 = B + d["A_OFF"]
        reads = [[(a0, a0 + npx * arow)] if lda == arow else
                 [(a0 + p * lda, a0 + p * lda + arow) for p in range(npx)]]
    else:
        reads = [rows(d["A_OFF"], lda, arow)]
    if op in (C.OP_GEMM,) + C.CONV_OPS:
        w4 = is_w4(d)
        ns = 1 if d["CTRL"] & 7 == C.QM_TENSOR else N
        reads.append([(B + d["W_OFF"], B + d["W_OFF"] + N * K // (2 if w4 else 1))])
        reads.append([(B + d["SCALE_OFF"], B + d["SCALE_OFF"] + (2 * N * (K // C.W4_GROUP) if w4 else 4 * ns))])
        if d["EPI"] >> 4 & 1:
            reads.append([(B + d["BIAS_OFF"], B + d["BIAS_OFF"] + 4 * N)])
        if d["CTRL"] & 7 == C.QM_ROWCOL and not w4:
            r0 = B + 16 * d["HDR_RSV"]
            reads.append([(r0, r0 + 4 * M)])
    elif op == C.OP_ROW and d["CTRL"] & 7 in (C.ROW_LAYERNORM, C.ROW_RMSNORM, C.ROW_L2NORM):
        reads.append([(B + d["SCALE_OFF"], B + d["SCALE_OFF"] + 4 * N)])
        if d["EPI"] >> 4 & 1:
            reads.append([(B + d["BIAS_OFF"], B + d["BIAS_OFF"] + 4 * N)])
    return reads, y


def extra_out(d: dict):
    """golden.py:250-256 - ROW_QUANT's row scales: 4 M bytes at SCALE_OFF."""
    if d["OPCODE"] == C.OP_ROW and d["CTRL"] & 7 == C.ROW_QUANT:
        a = d["BASE_ADDR"] + d["SCALE_OFF"]
        return [(a, a + 4 * d["M"])]
    return []


def overlaps(segs, y) -> bool:
    """golden.py:258-266 - y is ascending and disjoint."""
    ends = [hi for _, hi in y]
    for lo, hi in segs:
        i = bisect.bisect_right(ends, lo)
        if i < len(y) and y[i][0] < hi:
            return True
    return False


def in_place(d: dict, i: int) -> bool:
    """golden.py:437-447 - read i of an ELT may be its own output: A (0) or C (2)."""
    out = d["EPI"] >> 2 & 3
    if d["OPCODE"] != C.OP_ELT or out not in (C.OUT_FP32, C.OUT_FP16):
        return False
    lda, ldy = strides(d)[:2]
    if i == 0:
        afmt = C.OUT_FP16 if d["HDR_RSV"] & C.STATE_FP16 else C.OUT_FP32
        return afmt == out and not (d["HDR_RSV"] >> 2 & 1) and d["A_OFF"] == d["Y_OFF"] and lda == ldy
    return i == 2 and d["BIAS_OFF"] == d["Y_OFF"]


class OracleMachine:
    """The golden executor over `ddr` (mutated in place), golden.py:41-492."""

    def __init__(self, ddr: bytearray, core_id: int = 0, gemv_only: bool = False):
        self.ddr = ddr
        self.core_id = core_id
        self.gemv_only = gemv_only
        self.status = Status()
        self.stats: list[OpStat] = []

    def read(self, addr: int, n: int) -> bytes:
        return bytes(self.ddr[addr:addr + n])

    def write(self, addr: int, data: bytes) -> None:
        self.ddr[addr:addr + len(data)] = data

    def validate(self, raw: bytes):
        d = C.decode(raw)
        return check(d, raw, self.core_id, self.gemv_only), d

    strides = staticmethod(strides)
    bstride = staticmethod(bstride)
    segments = staticmethod(segments)
    extra_out = staticmethod(extra_out)

    # ------------------------------------------------------------ tensors out of DDR
    def _f32_rows(self, addr, ld, m, n):
        return np.stack([np.frombuffer(self.read(addr + i * ld, 4 * n), "<f4") for i in range(m)]).astype(F.F32)

    def _float_rows(self, addr, ld, m, n, half):
        if not half:
            return self._f32_rows(addr, ld, m, n)
        return np.stack([F.from_fp16_bits(np.frombuffer(self.read(addr + i * ld, 2 * n), "<u2")) for i in range(m)])

    def _vec(self, addr, n):
        return np.frombuffer(self.read(addr, 4 * n), "<f4").astype(F.F32)

    @staticmethod
    def convert(y, out: int, out_scale_bits: int) -> np.ndarray:
        """golden.py:269-280 - [M, N] -> [M, row bytes] uint8."""
        if out == C.OUT_FP32:
            b = F.ftz(y).astype("<f4").tobytes()
        elif out == C.OUT_BF16:
            b = F.to_bf16_bits(y).astype("<u2").tobytes()
        elif out == C.OUT_FP16:
            b = F.to_fp16_bits(y).astype("<u2").tobytes()
        else:
            b = F.q8(y, C.bits_f32(out_scale_bits)).tobytes()
        return np.frombuffer(b, np.uint8).reshape(y.shape[0], -1)

    # ------------------------------------------------------------ opcode semantics
    def _gemm(self, d, A=None):
        """golden.py:326-349."""
        if is_w4(d):
            return self._gemm_w4(d)
        B, M, N, K, e = d["BASE_ADDR"], d["M"], d["N"], d["K"], d["EPI"]
        lda = strides(d)[0]
        if A is None:
            A = np.stack([np.frombuffer(self.read(B + d["A_OFF"] + m * lda, K), np.int8)
                          for m in range(M)]).astype(np.int64)
        W = np.frombuffer(self.read(B + d["W_OFF"], N * K), np.int8).reshape(N, K).astype(np.int64)
        acc = A @ W.T
        assert np.abs(acc).max(initial=0) < 2 ** 31
        qm = d["CTRL"] & 7
        s = self._vec(B + d["SCALE_OFF"], 1 if qm == C.QM_TENSOR else N)
        y = F.i2f(acc)
        if qm == C.QM_ROWCOL:
            y = F.fmul(y, self._vec(B + 16 * d["HDR_RSV"], M)[:, None])
        y = F.fmul(y, np.broadcast_to(s, (M, N)))
        if e >> 4 & 1:
            y = F.fadd(y, np.broadcast_to(self._vec(B + d["BIAS_OFF"], N), (M, N)))
        y = F.act_fn(y, C.act_of(e))
        return self.convert(y, e >> 2 & 3, d["OUT_SCALE"])

    def _gemm_w4(self, d):
        """golden.py:295-324."""
        B, M, N, K, e = d["BASE_ADDR"], d["M"], d["N"], d["K"], d["EPI"]
        lda = strides(d)[0]
        G = K // C.W4_GROUP
        if d["CTRL"] >> 4 & 15 == C.DT_FP32:
            a = self._f32_rows(B + d["A_OFF"], lda, M, K)
        else:
            a = np.stack([F.bf16_bits_to_f32(np.frombuffer(self.read(B + d["A_OFF"] + m * lda, 2 * K), "<u2"))
                          for m in range(M)])
        aq, asc = F.align_w4_groups(a)
        aq = aq.reshape(M, G, C.W4_GROUP).astype(np.int64)
        pk = np.frombuffer(self.read(B + d["W_OFF"], N * K // 2), np.uint8).reshape(N, K // 2)
        lo, hi = (pk & 15).astype(np.int64), (pk >> 4).astype(np.int64)
        lo, hi = np.where(lo >= 8, lo - 16, lo), np.where(hi >= 8, hi - 16, hi)
        w = np.stack((lo, hi), axis=2).reshape(N, G, C.W4_GROUP)
        ws = F.from_fp16_bits(np.frombuffer(self.read(B + d["SCALE_OFF"], 2 * N * G), "<u2").reshape(N, G))
        banks = np.zeros((4, M, N), F.F32)
        for g in range(G):
            dot = aq[:, g] @ w[:, g].T
            term = F.fmul(F.fmul(F.i2f(dot), ws[None, :, g]), asc[:, None, g])
            banks[g % 4] = F.fadd(banks[g % 4], term)
        y = F.fadd(F.fadd(banks[0], banks[1]), F.fadd(banks[2], banks[3]))
        if e >> 4 & 1:
            y = F.fadd(y, np.broadcast_to(self._vec(B + d["BIAS_OFF"], N), (M, N)))
        y = F.act_fn(y, C.act_of(e))
        return self.convert(y, e >> 2 & 3, d["OUT_SCALE"])

    def _conv(self, d):
        """golden.py:282-293 - implicit GEMM over an NHWC INT8 image, zero padding."""
        g = C.conv_params(d)
        lda = strides(d)[0]
        a0, cin = d["BASE_ADDR"] + d["A_OFF"], g["Cin"]
        img = np.zeros((g["H"] + 2 * g["P"], g["W"] + 2 * g["P"], cin), np.int64)
        for p in range(g["H"] * g["W"]):
            img[g["P"] + p // g["W"], g["P"] + p % g["W"]] = np.frombuffer(self.read(a0 + p * lda, cin), np.int8)
        S, KH, KW = g["S"], g["KH"], g["KW"]
        A = np.stack([img[oy * S:oy * S + KH, ox * S:ox * S + KW].reshape(-1)
                      for oy in range(g["OH"]) for ox in range(g["OW"])])
        return self._gemm(d, A)

    def _relu(self, d):
        """golden.py:351-356."""
        x = self._f32_rows(d["BASE_ADDR"] + d["A_OFF"], strides(d)[0], d["M"], d["N"])
        return self.convert(F.act_fn(x, C.act_of(d["EPI"])), d["EPI"] >> 2 & 3, d["OUT_SCALE"])

    def _row(self, d):
        """golden.py:358-380."""
        B, M, N = d["BASE_ADDR"], d["M"], d["N"]
        x = self._f32_rows(B + d["A_OFF"], strides(d)[0], M, N)
        fn = d["CTRL"] & 7
        if fn == C.ROW_SOFTMAX:
            y = F.softmax_rows_causal(x, np.minimum(N, d["K"] + np.arange(M))) if d["K"] else F.softmax_rows(x)
        elif fn == C.ROW_QUANT:
            q, s = F.quant_rows(x)
            self._extra = (B + d["SCALE_OFF"], F.ftz(s).astype("<f4").tobytes())
            return q.view(np.uint8)
        else:
            gamma = self._vec(B + d["SCALE_OFF"], N)
            beta = self._vec(B + d["BIAS_OFF"], N) if d["EPI"] >> 4 & 1 else None
            fnc = {C.ROW_LAYERNORM: F.layernorm_rows, C.ROW_RMSNORM: F.rmsnorm_rows,
                   C.ROW_L2NORM: F.l2norm_rows}[fn]
            y = fnc(x, gamma, beta, C.bits_f32(d["W_OFF"]))
        return self.convert(y, d["EPI"] >> 2 & 3, d["OUT_SCALE"])

    def _elt(self, d):
        """golden.py:393-418."""
        B, M, N, e = d["BASE_ADDR"], d["M"], d["N"], d["EPI"]
        lda, ldy = strides(d)[:2]
        a = self._float_rows(B + d["A_OFF"], 0 if d["HDR_RSV"] >> 2 & 1 else lda, M, N,
                             bool(d["HDR_RSV"] & C.STATE_FP16))
        bm = d["HDR_RSV"] & 3
        w0 = B + d["W_OFF"]
        if bm == C.BM_DENSE:
            b = self._f32_rows(w0, bstride(d)[0], M, N)
        else:
            v = self._vec(w0, {C.BM_ROW: N, C.BM_COL: M, C.BM_SCALAR: 1}[bm])
            b = np.broadcast_to(v[None, :] if bm == C.BM_ROW else v[:, None] if bm == C.BM_COL else v[None, :1],
                                (M, N))
        a = F.act_fn(a, C.act_of(e))
        eop = d["CTRL"] & 3
        if eop == C.ELT_MUL:
            y = F.fmul(a, b)
        elif eop == C.ELT_ADD:
            y = F.fadd(a, b)
        elif eop == C.ELT_SUB:
            y = F.fadd(a, F.neg(F.ftz(b)))
        else:
            c = self._float_rows(B + d["BIAS_OFF"], ldy, M, N, e >> 2 & 3 == C.OUT_FP16)
            y = F.fadd(c, F.fmul(a, b))
        return self.convert(y, e >> 2 & 3, d["OUT_SCALE"])

    def _rope(self, d):
        """golden.py:420-424."""
        B, M, N, R, G = d["BASE_ADDR"], d["M"], d["N"], d["K"], d["GROUP_SIZE"]
        x = self._f32_rows(B + d["A_OFF"], strides(d)[0], M, N)
        tab = self._f32_rows(B + d["W_OFF"], 4 * R, (M - 1) // G + 1, R)
        return self.convert(F.rope_rows(x, tab, G, R), d["EPI"] >> 2 & 3, d["OUT_SCALE"])

    def _fdot(self, d):
        """golden.py:426-435."""
        B, M, N, K = d["BASE_ADDR"], d["M"], d["N"], d["K"]
        a = self._f32_rows(B + d["A_OFF"], strides(d)[0], M, K)
        ldb = bstride(d)[0]
        if d["CTRL"] & 1:
            y = F.fdot_nn(a, self._float_rows(B + d["W_OFF"], ldb, K, N, bool(d["HDR_RSV"] & C.STATE_FP16)))
        else:
            y = F.fdot_nt(a, self._f32_rows(B + d["W_OFF"], ldb, N, K))
        return self.convert(y, d["EPI"] >> 2 & 3, d["OUT_SCALE"])

    # ------------------------------------------------------------ the queue
    def run_queue(self, queue_addr: int, queue_len: int) -> Status:
        """golden.py:450-492 - in order; all checks of a descriptor before any of its writes; an
        error stops the queue and keeps the earlier writes."""
        self.status, self.stats = Status(), []
        table = {C.OP_GEMM: self._gemm, C.OP_RELU: self._relu, C.OP_ROW: self._row,
                 C.OP_CONV: self._conv, C.OP_CONV_ACT: self._conv, C.OP_ELT: self._elt,
                 C.OP_ROPE: self._rope, C.OP_FDOT: self._fdot}
        for i in range(queue_len):
            qa = queue_addr + C.DESC_BYTES * i
            if qa + C.DESC_BYTES > len(self.ddr):
                self.status = Status(False, C.E_RANGE, i)
                return self.status
            raw = self.read(qa, C.DESC_BYTES)
            err, d = self.validate(raw)
            if err == C.E_OK:
                reads, y = segments(d)
                extra = extra_out(d)
                if any(hi > len(self.ddr) for seg in reads + [y, extra] for _, hi in seg):
                    err = C.E_RANGE
            if err != C.E_OK:
                self.status = Status(False, err, i)
                return self.status
            for j, seg in enumerate(reads):
                if overlaps(seg, y) and not in_place(d, j):
                    raise ContractError(f"descriptor {i}: output overlaps an input")
                if extra and overlaps(seg, extra):
                    raise ContractError(f"descriptor {i}: output overlaps an input")
            if extra and overlaps(extra, y):
                raise ContractError(f"descriptor {i}: the two outputs overlap")
            self._extra = None
            rows = table[d["OPCODE"]](d)
            for m in range(rows.shape[0]):
                self.write(y[m][0], rows[m].tobytes())
            if self._extra:
                self.write(*self._extra)
            macs = d["M"] * d["N"] * d["K"] if d["OPCODE"] in (C.OP_GEMM, C.OP_FDOT) + C.CONV_OPS else 0
            self.stats.append(OpStat(d["OPCODE"], macs, sum(hi - lo for seg in reads for lo, hi in seg), rows.size))
        self.status = Status(True, C.E_OK, queue_len)
        return self.status
