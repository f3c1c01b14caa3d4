"""CPU oracle, part 3: the golden executor (tars_mini/golden.py) restated over a DDR bytearray.

TEST INFRASTRUCTURE ONLY (see oracle/numerics.py's header for who may use it).

OracleMachine has the call surface of the reference's golden Machine (golden.py:41-56,
450-492): run_queue(queue_addr, queue_len) -> Status, read/write, .ddr (mutated in place),
.status, .stats; validate(raw) and the static strides/bstride/segments/extra_out.
"""
from __future__ import annotations

import bisect
from dataclasses import dataclass

import numpy as np

from . import contract as C
from . import numerics as F


class ContractError(Exception):
    """golden.py:18-19 - an illegal program (an output overlapping an input, or two outputs)."""


@dataclass
class Status:
    """golden.py:21-26 - whether the queue finished, the error code, the index it stopped at."""
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
        # W4A16: symmetric, fp32 or bf16 activations, groups of 128, no row-scale word; else
        # symmetric int8 x int8 in the tensor / channel / row-col modes (row-col not for CONV)
        w4_bad = (sym, d["HDR_RSV"], d["GROUP_SIZE"]) != (1, 0, C.W4_GROUP) or adt not in (C.DT_FP32, C.DT_BF16)
        i8_bad = (sym, adt, wdt) != (1, C.DT_INT8, C.DT_INT8) or qm not in (C.QM_TENSOR, C.QM_CHANNEL, C.QM_ROWCOL) \
            or (conv and qm == C.QM_ROWCOL)
        if (w4 and w4_bad) or (not w4 and i8_bad):
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
    """golden.py:171-178 - (row stride, row bytes) of B: an FDOT's [K][N] (NN, fp32 or fp16) or
    [N][K] (NT) matrix, an ELT's dense b rows (0 bytes when b is broadcast); GROUP_SIZE, when set,
    is the stride in 16-byte units."""
    fdot = d["OPCODE"] == C.OP_FDOT
    if fdot:
        width = d["N"] if d["CTRL"] & 1 else d["K"]
        nbytes = width * (2 if d["HDR_RSV"] & C.STATE_FP16 else 4)
    else:
        nbytes = 4 * d["N"] * int(d["HDR_RSV"] & 3 == C.BM_DENSE)
    return (d["GROUP_SIZE"] * 16 or nbytes), nbytes


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
    def span(off, nbytes):                      # one contiguous read at base + off
        return [(B + off, B + off + nbytes)]

    if op in C.CONV_OPS:
        g = C.conv_params(d)
        pixels = g["H"] * g["W"]                # the input image, one row of Cin per pixel
        reads = [span(d["A_OFF"], pixels * arow) if lda == arow else rows(d["A_OFF"], lda, arow, pixels)]
    else:
        reads = [rows(d["A_OFF"], lda, arow)]
    has_bias = bool(d["EPI"] >> 4 & 1)
    if op == C.OP_GEMM or op in C.CONV_OPS:
        qm, w4 = d["CTRL"] & 7, is_w4(d)
        if w4:
            wbytes, sbytes = N * K // 2, 2 * N * (K // C.W4_GROUP)      # nibbles, binary16 per group
        else:
            wbytes, sbytes = N * K, 4 * (1 if qm == C.QM_TENSOR else N)
        reads += [span(d["W_OFF"], wbytes), span(d["SCALE_OFF"], sbytes)]
        if has_bias:
            reads.append(span(d["BIAS_OFF"], 4 * N))
        if qm == C.QM_ROWCOL and not w4:
            reads.append(span(16 * d["HDR_RSV"], 4 * M))                 # the activation row scales
    elif op == C.OP_ROW and d["CTRL"] & 7 in (C.ROW_LAYERNORM, C.ROW_RMSNORM, C.ROW_L2NORM):
        reads.append(span(d["SCALE_OFF"], 4 * N))
        if has_bias:
            reads.append(span(d["BIAS_OFF"], 4 * N))
    return reads, y


def extra_out(d: dict):
    """golden.py:250-256 - ROW_QUANT's row scales: 4 M bytes at SCALE_OFF."""
    quant = d["OPCODE"] == C.OP_ROW and d["CTRL"] & 7 == C.ROW_QUANT
    lo = d["BASE_ADDR"] + d["SCALE_OFF"]
    return [(lo, lo + 4 * d["M"])] if quant else []


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
    if i == 2:
        return d["BIAS_OFF"] == d["Y_OFF"]
    if i != 0:
        return False
    lda, ldy = strides(d)[:2]
    a_fp16 = bool(d["HDR_RSV"] & C.STATE_FP16)
    same_format = out == (C.OUT_FP16 if a_fp16 else C.OUT_FP32)
    one_row = bool(d["HDR_RSV"] >> 2 & 1)
    return same_format and not one_row and (d["A_OFF"], lda) == (d["Y_OFF"], ldy)


def _check_overlaps(i: int, d: dict, reads, y, extra) -> None:
    """An output may overlap no input (except an ELT's in-place A or C), the row scales of
    ROW_QUANT no input and not the output rows."""
    for j, seg in enumerate(reads):
        if (overlaps(seg, y) and not in_place(d, j)) or (extra and overlaps(seg, extra)):
            raise ContractError(f"descriptor {i}: output overlaps an input")
    if extra and overlaps(extra, y):
        raise ContractError(f"descriptor {i}: the two outputs overlap")


class OracleMachine:
    """The golden executor over `ddr` (mutated in place), golden.py:41-492."""

    def __init__(self, ddr: bytearray, core_id: int = 0, gemv_only: bool = False):
        self.ddr = ddr
        self.core_id = core_id
        self.gemv_only = gemv_only
        self.status = Status()
        self.stats: list[OpStat] = []

    def read(self, addr: int, n: int) -> bytes:
        view = memoryview(self.ddr)
        return view[addr:addr + n].tobytes()

    def write(self, addr: int, data: bytes) -> None:
        n = len(data)
        self.ddr[addr:addr + n] = data

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
        fn = d["CTRL"] & 3
        if fn == C.ELT_MULADD:                  # c (at BIAS_OFF, the output's layout) + a b
            c = self._float_rows(B + d["BIAS_OFF"], ldy, M, N, e >> 2 & 3 == C.OUT_FP16)
            y = F.fadd(c, F.fmul(a, b))
        else:
            binop = {C.ELT_MUL: F.fmul, C.ELT_ADD: F.fadd,
                     C.ELT_SUB: lambda p, q: F.fadd(p, F.neg(F.ftz(q)))}[fn]
            y = binop(a, b)
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
        end = len(self.ddr)
        for i in range(queue_len):
            at = queue_addr + C.DESC_BYTES * i
            if at + C.DESC_BYTES > end:
                return self._stop(C.E_RANGE, i)
            err, d = self.validate(self.read(at, C.DESC_BYTES))
            if err != C.E_OK:
                return self._stop(err, i)
            reads, y = segments(d)
            extra = extra_out(d)
            if max((hi for seg in (*reads, y, extra) for _, hi in seg), default=0) > end:
                return self._stop(C.E_RANGE, i)
            _check_overlaps(i, d, reads, y, extra)
            self._extra = None
            out = table[d["OPCODE"]](d)
            for m, row in enumerate(out):
                self.write(y[m][0], row.tobytes())
            if self._extra:
                self.write(*self._extra)
            contraction = d["OPCODE"] == C.OP_GEMM or d["OPCODE"] == C.OP_FDOT or d["OPCODE"] in C.CONV_OPS
            read_bytes = sum(hi - lo for seg in reads for lo, hi in seg)
            self.stats.append(OpStat(d["OPCODE"], d["M"] * d["N"] * d["K"] * contraction, read_bytes, out.size))
        self.status = Status(True, C.E_OK, queue_len)
        return self.status

    def _stop(self, err: int, i: int) -> Status:
        self.status = Status(False, err, i)
        return self.status
