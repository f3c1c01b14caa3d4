"""Seeded random programs (a DDR image + a descriptor queue) covering every opcode and mode.

The same seed builds the same bytes on any machine (numpy's default_rng), so the reference's
results are stored once as fixtures (make_fixtures.py) and every implementation is run on
regenerated inputs. Uses only numpy and the oracle's descriptor encoder.
"""
from __future__ import annotations

import numpy as np

from oracle import contract as C

F32 = np.float32
DDR_BYTES = 1 << 17           # 128 KiB image per case
QADDR = 0x1F000               # the queue region (64 descriptors at most)
HEAP0 = 0x100


def _special_f32(rng, shape, scale=2.0, p_special=0.02):
    x = rng.normal(0, scale, shape).astype(F32)
    if p_special:
        mask = rng.random(shape) < p_special
        pool = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38, 1e-38],
                        F32)
        x = np.where(mask, pool[rng.integers(0, len(pool), shape)], x).astype(F32)
    return x


class Heap:
    """A bump allocator over the image with 16-byte (sometimes 128-byte) alignment."""

    def __init__(self, ddr: bytearray, rng):
        self.ddr, self.rng, self.top = ddr, rng, HEAP0

    def alloc(self, n: int, align: int = 16) -> int:
        off = -(-self.top // align) * align
        self.top = off + n
        if self.top > QADDR:
            raise MemoryError
        return off

    def put(self, data: bytes, align: int = 16) -> int:
        off = self.alloc(len(data), align)
        self.ddr[off:off + len(data)] = data
        return off

    def rows(self, m: int, rowbytes: int, extra16: int = 0) -> tuple[int, int]:
        """[m rows] with a row stride of rowbytes (+ 16 * extra16): (offset, stride)."""
        ld = rowbytes + 16 * extra16
        return self.alloc(ld * m), ld


def _base(**f):
    return dict(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1, **f)


def _ld16(ld, row):
    return 0 if ld == row else ld // 16


def gen_gemm(rng, h: Heap):
    M = int(rng.integers(1, 9))
    N = 16 * int(rng.integers(1, 5))
    K = 16 * int(rng.integers(1, 9))
    qm = int(rng.choice([C.QM_TENSOR, C.QM_CHANNEL, C.QM_ROWCOL]))
    act = int(rng.integers(0, 8))
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    bias = int(rng.integers(0, 2))
    a_off, lda = h.rows(M, K, int(rng.integers(0, 2)) * int(rng.integers(1, 3)))
    for m in range(M):
        h.ddr[a_off + m * lda:a_off + m * lda + K] = rng.integers(-128, 128, K, dtype=np.int8).tobytes()
    w_off = h.put(rng.integers(-128, 128, N * K, dtype=np.int8).tobytes())
    ns = 1 if qm == C.QM_TENSOR else N
    s = rng.uniform(1e-4, 1e-2, ns).astype(F32)
    if rng.random() < 0.1:
        s[0] = np.inf
    s_off = h.put(s.astype("<f4").tobytes())
    f = _base(OPCODE=C.OP_GEMM, CTRL=C.ctrl(qm, fusion=int(act != 0)), EPI=C.epi(act, out, bias),
              A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, M=M, N=N, K=K, LDA16=_ld16(lda, K))
    if bias:
        f["BIAS_OFF"] = h.put(_special_f32(rng, N, 4.0, 0.05).astype("<f4").tobytes())
    if qm == C.QM_ROWCOL:
        sr = rng.uniform(1e-3, 5e-2, M).astype(F32)
        f["HDR_RSV"] = h.put(sr.astype("<f4").tobytes()) // 16
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def gen_w4(rng, h: Heap):
    M = int(rng.integers(1, 4))
    N = 16 * int(rng.integers(1, 4))
    K = 256 * int(rng.integers(1, 4))
    adt = int(rng.choice([C.DT_FP32, C.DT_BF16]))
    act = int(rng.integers(0, 8))
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    bias = int(rng.integers(0, 2))
    aes = 4 if adt == C.DT_FP32 else 2
    a_off, lda = h.rows(M, aes * K, int(rng.integers(0, 2)))
    x = _special_f32(rng, (M, K), 2.0, 0.002)
    if rng.random() < 0.3:                        # wide dynamic range inside a group
        x *= (2.0 ** rng.integers(-30, 30, (M, K))).astype(F32)
    for m in range(M):
        if adt == C.DT_FP32:
            row = x[m].astype("<f4").tobytes()
        else:
            row = (x[m].view(np.uint32) >> 16).astype("<u2").tobytes()
        h.ddr[a_off + m * lda:a_off + m * lda + len(row)] = row
    w_off = h.put(rng.integers(0, 256, N * K // 2, dtype=np.uint8).tobytes(), align=128)
    ws = rng.uniform(1e-3, 2e-2, (N, K // 128)).astype(np.float16).view(np.uint16)
    s_off = h.put(ws.astype("<u2").tobytes())
    f = _base(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_GROUP, a_dtype=adt, w_dtype=C.DT_INT4, fusion=int(act != 0)),
              EPI=C.epi(act, out, bias), A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, M=M, N=N, K=K,
              GROUP_SIZE=128, LDA16=_ld16(lda, aes * K))
    if bias:
        f["BIAS_OFF"] = h.put(rng.normal(0, 1, N).astype("<f4").tobytes())
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def _f32_rows(rng, h: Heap, M, N, extra=0, scale=2.0, p_special=0.01):
    off, ld = h.rows(M, 4 * N, extra)
    x = _special_f32(rng, (M, N), scale, p_special)
    for m in range(M):
        h.ddr[off + m * ld:off + m * ld + 4 * N] = x[m].astype("<f4").tobytes()
    return off, ld


def gen_relu(rng, h: Heap):
    M, N = int(rng.integers(1, 9)), 16 * int(rng.integers(1, 5))
    act = int(rng.integers(1, 8))
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    a_off, lda = _f32_rows(rng, h, M, N, int(rng.integers(0, 2)), 6.0, 0.03)
    f = _base(OPCODE=C.OP_RELU, EPI=C.epi(act, out), A_OFF=a_off, M=M, N=N, LDA16=_ld16(lda, 4 * N))
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def gen_row(rng, h: Heap):
    fn = int(rng.integers(0, 5))
    M, N = int(rng.integers(1, 9)), 16 * int(rng.integers(1, 9))
    a_off, lda = _f32_rows(rng, h, M, N, int(rng.integers(0, 2)), 3.0, 0.005 if rng.random() < 0.3 else 0)
    if fn == C.ROW_QUANT:
        out = C.OUT_INT8
        f = _base(OPCODE=C.OP_ROW, CTRL=fn, EPI=C.epi(C.ACT_NONE, out), A_OFF=a_off, M=M, N=N,
                  LDA16=_ld16(lda, 4 * N), SCALE_OFF=h.alloc(4 * M))
        if rng.random() < 0.3:                    # an all-zero row
            h.ddr[a_off:a_off + 4 * N] = bytes(4 * N)
    else:
        out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
        f = _base(OPCODE=C.OP_ROW, CTRL=fn, A_OFF=a_off, M=M, N=N, LDA16=_ld16(lda, 4 * N))
        beta = 0
        if fn == C.ROW_SOFTMAX:
            if rng.random() < 0.6:
                f["K"] = int(rng.integers(1, N + 1))
        else:
            f["SCALE_OFF"] = h.put(rng.normal(1, 0.3, N).astype("<f4").tobytes())
            f["W_OFF"] = C.f32_bits(float(rng.choice([1e-6, 1e-5, 0.0, 1.0])))
            beta = int(rng.integers(0, 2))
            if beta:
                f["BIAS_OFF"] = h.put(rng.normal(0, 0.5, N).astype("<f4").tobytes())
        f["EPI"] = C.epi(C.ACT_NONE, out, beta)
        if out == C.OUT_INT8:
            f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def gen_elt(rng, h: Heap):
    M, N = int(rng.integers(1, 9)), 16 * int(rng.integers(1, 5))
    eop = int(rng.integers(0, 4))
    bm = int(rng.integers(0, 4))
    arow = int(rng.random() < 0.2)
    a16 = int(rng.random() < 0.25)
    act = int(rng.integers(0, 8))
    outs = [C.OUT_FP32, C.OUT_FP16] if eop == C.ELT_MULADD else [C.OUT_FP32, C.OUT_BF16, C.OUT_INT8, C.OUT_FP16]
    out = int(rng.choice(outs))
    aes = 2 if a16 else 4
    inplace_a = (not arow) and ((a16 and out == C.OUT_FP16) or (not a16 and out == C.OUT_FP32)) and rng.random() < 0.3
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    if inplace_a:
        a_off, lda = y_off, ldy
        xs = _special_f32(rng, (M, N), 2.0, 0.01)
        for m in range(M):
            row = xs[m].astype("<f4").tobytes() if not a16 else xs[m].astype("<f2").tobytes()
            h.ddr[a_off + m * ldy:a_off + m * ldy + len(row)] = row
    else:
        rows_a = 1 if arow else M
        a_off, lda = h.rows(rows_a, aes * N, int(rng.integers(0, 2)))
        xs = _special_f32(rng, (rows_a, N), 2.0, 0.01)
        for m in range(rows_a):
            row = xs[m].astype("<f4").tobytes() if not a16 else xs[m].astype("<f2").tobytes()
            h.ddr[a_off + m * lda:a_off + m * lda + len(row)] = row
    if bm == C.BM_DENSE:
        b_off, ldb = _f32_rows(rng, h, M, N, int(rng.integers(0, 2)), 2.0, 0.01)
        g = _ld16(ldb, 4 * N)
    else:
        cnt = {C.BM_ROW: N, C.BM_COL: M, C.BM_SCALAR: 1}[bm]
        base = h.put(_special_f32(rng, cnt + 3, 2.0, 0.01).astype("<f4").tobytes())
        b_off = base + (4 * int(rng.integers(0, 4)) if bm in (C.BM_COL, C.BM_SCALAR) else 0)
        g = 0
    f = _base(OPCODE=C.OP_ELT, CTRL=eop, EPI=C.epi(act, out, int(eop == C.ELT_MULADD)), A_OFF=a_off,
              W_OFF=b_off, Y_OFF=y_off, M=M, N=N, GROUP_SIZE=g,
              HDR_RSV=bm | arow << 2 | (C.STATE_FP16 if a16 else 0),
              LDA16=0 if arow else _ld16(lda, aes * N), LDY16=_ld16(ldy, yrow))
    if eop == C.ELT_MULADD:
        if rng.random() < 0.4:                    # C is the output itself
            f["BIAS_OFF"] = y_off
            cs = _special_f32(rng, (M, N), 2.0, 0.01)
            for m in range(M):
                row = cs[m].astype("<f4").tobytes() if out == C.OUT_FP32 else cs[m].astype("<f2").tobytes()
                if not inplace_a:
                    h.ddr[y_off + m * ldy:y_off + m * ldy + len(row)] = row
        else:
            c_off = h.alloc(ldy * M)
            cs = _special_f32(rng, (M, N), 2.0, 0.01)
            for m in range(M):
                row = cs[m].astype("<f4").tobytes() if out == C.OUT_FP32 else cs[m].astype("<f2").tobytes()
                h.ddr[c_off + m * ldy:c_off + m * ldy + len(row)] = row
            f["BIAS_OFF"] = c_off
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    return f


def gen_rope(rng, h: Heap):
    R = 32 * int(rng.integers(1, 3))
    N = R + 16 * int(rng.integers(0, 3))
    G = int(rng.integers(1, 4))
    M = int(rng.integers(1, 9))
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    a_off, lda = _f32_rows(rng, h, M, N, int(rng.integers(0, 2)), 2.0, 0.005)
    rows = (M - 1) // G + 1
    pos = np.arange(rows, dtype=F32) + F32(rng.integers(0, 50))
    inv = (1.0 / (F32(10000.0) ** (np.arange(0, R, 2, dtype=F32) / F32(R)))).astype(F32)
    fr = (pos[:, None] * inv[None, :]).astype(F32)
    tab = np.concatenate([np.cos(fr), np.sin(fr)], 1).astype(F32)
    t_off = h.put(tab.astype("<f4").tobytes())
    f = _base(OPCODE=C.OP_ROPE, EPI=C.epi(C.ACT_NONE, out), A_OFF=a_off, W_OFF=t_off, M=M, N=N, K=R,
              GROUP_SIZE=G, LDA16=_ld16(lda, 4 * N))
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def gen_fdot(rng, h: Heap):
    nn = int(rng.integers(0, 2))
    M, N, K = int(rng.integers(1, 7)), 16 * int(rng.integers(1, 4)), 16 * int(rng.integers(1, 5))
    b16 = int(nn and rng.random() < 0.3)
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    a_off, lda = _f32_rows(rng, h, M, K, int(rng.integers(0, 2)), 2.0, 0.003)
    brows, bcols = (K, N) if nn else (N, K)
    bes = 2 if b16 else 4
    b_off, ldb = h.rows(brows, bes * bcols, int(rng.integers(0, 2)))
    bv = _special_f32(rng, (brows, bcols), 2.0, 0.003)
    for r in range(brows):
        row = bv[r].astype("<f2").tobytes() if b16 else bv[r].astype("<f4").tobytes()
        h.ddr[b_off + r * ldb:b_off + r * ldb + len(row)] = row
    f = _base(OPCODE=C.OP_FDOT, CTRL=nn, EPI=C.epi(C.ACT_NONE, out), A_OFF=a_off, W_OFF=b_off, M=M, N=N, K=K,
              GROUP_SIZE=_ld16(ldb, bes * bcols), HDR_RSV=C.STATE_FP16 if b16 else 0, LDA16=_ld16(lda, 4 * K))
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(M, yrow, int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=_ld16(ldy, yrow))
    return f


def gen_conv(rng, h: Heap):
    H, W = int(rng.integers(2, 7)), int(rng.integers(2, 7))
    KH, KW = int(rng.integers(1, 4)), int(rng.integers(1, 4))
    S, P = int(rng.integers(1, 3)), int(rng.integers(0, 2))
    cin = 16 * int(rng.integers(1, 3))
    OH, OW = (H + 2 * P - KH) // S + 1, (W + 2 * P - KW) // S + 1
    if OH < 1 or OW < 1:
        H, W, KH, KW, S, P = 4, 4, 3, 3, 1, 1
        OH, OW = 4, 4
    N = 16 * int(rng.integers(1, 3))
    K = KH * KW * cin
    act = int(rng.integers(0, 8))
    out = int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8]))
    a_off, lda = h.rows(H * W, cin, int(rng.integers(0, 2)))
    for p in range(H * W):
        h.ddr[a_off + p * lda:a_off + p * lda + cin] = rng.integers(-128, 128, cin, dtype=np.int8).tobytes()
    w_off = h.put(rng.integers(-128, 128, N * K, dtype=np.int8).tobytes())
    qm = int(rng.choice([C.QM_TENSOR, C.QM_CHANNEL]))
    s_off = h.put(rng.uniform(1e-4, 1e-2, 1 if qm == C.QM_TENSOR else N).astype("<f4").tobytes())
    f = _base(OPCODE=C.OP_CONV_ACT if act else C.OP_CONV, CTRL=C.ctrl(qm, fusion=int(act != 0)),
              EPI=C.epi(act, out, 0), A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, M=OH * OW, N=N, K=K,
              LDA16=_ld16(lda, cin), GROUP_SIZE=W, HDR_RSV=H << 12 | KH << 8 | KW << 4 | (S - 1) << 2 | P)
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    yrow = N * C.ESIZE[out]
    y_off, ldy = h.rows(OH * OW, yrow, 0)
    f.update(Y_OFF=y_off, LDY16=0)
    return f


GENS = {"gemm": gen_gemm, "w4": gen_w4, "relu": gen_relu, "row": gen_row, "elt": gen_elt,
        "rope": gen_rope, "fdot": gen_fdot, "conv": gen_conv}


def corrupt(rng, f: dict, raw: bytes) -> bytes:
    """One injected fault: a CRC bit flip, a field, alignment, range or opcode error, or an output
    placed over an input (an illegal program)."""
    k = int(rng.integers(0, 8))
    if k == 0:
        b = bytearray(raw)
        b[int(rng.integers(0, 64))] ^= 1 << int(rng.integers(0, 8))
        return bytes(b)
    g = dict(f)
    if k == 1:
        g["DEP_SIG"] = 1
    elif k == 2:
        g["N"] = g["N"] + 8
    elif k == 3:
        g["A_OFF"] = g["A_OFF"] + 4
    elif k == 4:
        g["Y_OFF"] = DDR_BYTES - 16
    elif k == 5:
        g["OPCODE"] = 0x0F
    else:                                          # an output over an input: ContractError
        g["Y_OFF"] = g["A_OFF"] + 16 * int(rng.integers(0, 2))
    return C.encode(g)


def build_case(seed: int, kinds: tuple[str, ...] = tuple(GENS), n_desc: int | None = None,
               p_corrupt: float = 0.06):
    """(ddr bytearray, queue address, queue length) for a seed."""
    with np.errstate(all="ignore"):
        return _build_case(seed, kinds, n_desc, p_corrupt)


def _build_case(seed, kinds, n_desc, p_corrupt):
    rng = np.random.default_rng(seed)
    ddr = bytearray(rng.integers(0, 256, DDR_BYTES, dtype=np.uint8).tobytes()) if rng.random() < 0.3 \
        else bytearray(DDR_BYTES)
    h = Heap(ddr, rng)
    n = n_desc or int(rng.integers(1, 7))
    descs = []
    for _ in range(n):
        kind = kinds[int(rng.integers(0, len(kinds)))]
        try:
            f = GENS[kind](rng, h)
        except MemoryError:
            break
        raw = C.encode(f)
        if rng.random() < p_corrupt:
            raw = corrupt(rng, f, raw)
        descs.append(raw)
    for i, r in enumerate(descs):
        ddr[QADDR + 64 * i:QADDR + 64 * (i + 1)] = r
    return ddr, QADDR, len(descs)


# ----------------------------------------------------------- chained programs (RAW/WAR/WAW)
def build_chain(seed: int):
    """A queue whose descriptors read earlier outputs: quant -> GEMM(ROWCOL) -> ELT add -> norm
    -> quant -> GEMM, with the second quant writing over the first's rows (WAW) and a RELU
    overwriting the first GEMM's input (WAR)."""
    rng = np.random.default_rng(seed)
    ddr = bytearray(DDR_BYTES)
    h = Heap(ddr, rng)
    M, K, N = int(rng.integers(1, 6)), 64, 64
    x_off, _ = _f32_rows(rng, h, M, K, 0, 2.0, 0)
    q_off, s_off = h.alloc(M * K), h.alloc(4 * M)
    w_off = h.put(rng.integers(-127, 128, N * K, dtype=np.int8).tobytes())
    sc_off = h.put(rng.uniform(1e-3, 1e-2, N).astype("<f4").tobytes())
    y_off = h.alloc(4 * M * N)
    r_off, _ = _f32_rows(rng, h, M, N, 0, 1.0, 0)
    z_off = h.alloc(4 * M * N)
    g_off = h.put(rng.normal(1, 0.2, N).astype("<f4").tobytes())
    n_off = h.alloc(4 * M * N)
    y2_off = h.alloc(4 * M * N)
    d = [
        _base(OPCODE=C.OP_ROW, CTRL=C.ROW_QUANT, EPI=C.epi(C.ACT_NONE, C.OUT_INT8), A_OFF=x_off, Y_OFF=q_off,
              SCALE_OFF=s_off, M=M, N=K),
        _base(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_ROWCOL, fusion=1), EPI=C.epi(C.ACT_SILU, C.OUT_FP32),
              A_OFF=q_off, W_OFF=w_off, SCALE_OFF=sc_off, Y_OFF=y_off, M=M, N=N, K=K, HDR_RSV=s_off // 16),
        _base(OPCODE=C.OP_ELT, CTRL=C.ELT_ADD, EPI=C.epi(), A_OFF=y_off, W_OFF=r_off, Y_OFF=z_off, M=M, N=N),
        _base(OPCODE=C.OP_ROW, CTRL=C.ROW_RMSNORM, EPI=C.epi(), A_OFF=z_off, Y_OFF=n_off, SCALE_OFF=g_off,
              W_OFF=C.f32_bits(1e-6), M=M, N=N),
        _base(OPCODE=C.OP_ROW, CTRL=C.ROW_QUANT, EPI=C.epi(C.ACT_NONE, C.OUT_INT8), A_OFF=n_off, Y_OFF=q_off,
              SCALE_OFF=s_off, M=M, N=N),
        _base(OPCODE=C.OP_RELU, EPI=C.epi(C.ACT_RELU, C.OUT_FP32), A_OFF=z_off, Y_OFF=x_off, M=M, N=N),
        _base(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_ROWCOL), EPI=C.epi(C.ACT_NONE, C.OUT_BF16),
              A_OFF=q_off, W_OFF=w_off, SCALE_OFF=sc_off, Y_OFF=y2_off, M=M, N=N, K=K, HDR_RSV=s_off // 16),
    ]
    for i, f in enumerate(d):
        ddr[QADDR + 64 * i:QADDR + 64 * (i + 1)] = C.encode(f)
    return ddr, QADDR, len(d)
