"""CPU oracle, part 1: the tars_mini fp32 numeric contract restated in numpy.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module; only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it, and only as
the checker (or the timed CPU baseline), never as the thing measured or shipped.

Every function restates one function of the reference's tars_mini/numerics.py (cited per
function). The contract: each fp step rounds once to nearest-even, inputs and outputs of
every step are flushed (denormal -> signed zero), no fused multiply-add, and every NaN a
step produces is the canonical 0x7FC00000. numpy's float32 add/mul are IEEE RNE with
gradual underflow, so a step is "flush the operands, one numpy op, flush, canonicalise".

Two reductions are vectorised without changing a single bit:
  * sum16 keeps the contract's lane order (lane j mod 16, sequential per lane, then the
    pairwise fold) but advances all 16 lanes of all rows per numpy call;
  * max16 folds pairwise instead of left to right; fmax is commutative and associative by
    construction (its answer for every pair is fixed), so any fold order gives the same bits.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
U32 = np.uint32
_SIGN = np.uint32(0x80000000)
_EXPM = np.uint32(0x7F800000)
CANON_NAN_BITS = 0x7FC00000


def bits(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, F32)).view(U32)


def from_bits(b) -> np.ndarray:
    return np.asarray(b, dtype=np.uint64).astype(U32).view(F32)


def f32c(b: int) -> np.float32:
    """A float32 constant from its bit pattern."""
    return np.array([b], U32).view(F32)[0]


# ---------------------------------------------------------------- step primitives
def ftz(x) -> np.ndarray:
    """numerics.py:26-31 - a denormal becomes the zero of its sign."""
    x = np.asarray(x, F32)
    b = x.view(U32) if x.flags.c_contiguous else bits(x)
    return np.where((b & _EXPM) == 0, (b & _SIGN).view(F32), x).astype(F32)


def canon(x) -> np.ndarray:
    """numerics.py:34-37 - any NaN becomes 0x7FC00000."""
    x = np.asarray(x, F32)
    return np.where(np.isnan(x), f32c(CANON_NAN_BITS), x).astype(F32)


def fmul(a, b) -> np.ndarray:
    """numerics.py:40-42."""
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        return canon(ftz(ftz(a) * ftz(b)))


def fadd(a, b) -> np.ndarray:
    """numerics.py:45-47."""
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        return canon(ftz(ftz(a) + ftz(b)))


def i2f(i) -> np.ndarray:
    """numerics.py:50-52 - integer to fp32, ties to even."""
    return np.asarray(i, np.int64).astype(F32)


def neg(x) -> np.ndarray:
    """numerics.py:111-113 - exact sign flip (not an fp operation)."""
    return (bits(x) ^ _SIGN).view(F32)


def fabs(x) -> np.ndarray:
    """numerics.py:265-267 - flush, then clear the sign bit."""
    return (bits(ftz(x)) & U32(0x7FFFFFFF)).view(F32)


def to_fp16_bits(x) -> np.ndarray:
    """numerics.py:14-18 - IEEE binary16, RNE, gradual underflow; NaN -> 0x7E00."""
    x = np.asarray(x, F32)
    with np.errstate(over="ignore", invalid="ignore"):
        h = x.astype(np.float16).view(np.uint16)
    return np.where(np.isnan(x), 0x7E00, h).astype(np.uint16)


def from_fp16_bits(h) -> np.ndarray:
    """numerics.py:21-23 - exact widening (binary16 subnormals included), NaN canonical."""
    return canon(np.asarray(h, np.uint16).view(np.float16).astype(F32))


def to_bf16_bits(x) -> np.ndarray:
    """numerics.py:270-275 - flush, then RNE to the top 16 bits; NaN -> 0x7FC0."""
    b = bits(ftz(x)).astype(np.uint64)
    isnan = ((b & 0x7F800000) == 0x7F800000) & ((b & 0x007FFFFF) != 0)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    return np.where(isnan, 0x7FC0, r).astype(np.uint16)


def bf16_bits_to_f32(h) -> np.ndarray:
    """numerics.py:278-279."""
    return (np.asarray(h, np.uint32) << 16).view(F32)


def q8(x, inv) -> np.ndarray:
    """numerics.py:282-286 - rint(fmul(x, inv)) ties-even, NaN -> 0, saturate to +-127."""
    r = np.rint(fmul(x, inv))
    return np.where(np.isnan(r), F32(0), np.clip(r, F32(-127), F32(127))).astype(np.int8)


# ---------------------------------------------------------------- contract constants
ONE, TWO, HALF = f32c(0x3F800000), f32c(0x40000000), f32c(0x3F000000)
LOG2E = f32c(0x3FB8AA3B)
NEG_LN2_HI, NEG_LN2_LO = f32c(0xBF317200), f32c(0xB5BFBE8E)
EXP_POLY = [f32c(b) for b in (0x3AB60B61, 0x3C088889, 0x3D2AAAAB, 0x3E2AAAAB,
                              0x3F000000, 0x3F800000, 0x3F800000)]
EXP_HI, EXP_LO = f32c(0x42B20000), f32c(0xC2D00000)          # 89, -104
RECIP_MAGIC, RSQRT_MAGIC = 0x7EF311C7, 0x5F3759DF
GELU_A, GELU_C = f32c(0x3D372713), f32c(0x3F4C422A)
LOG1P_POLY = [f32c(b) for b in (0x3D70F0F1, 0x3D888889, 0x3D9D89D9, 0x3DBA2E8C, 0x3DE38E39,
                                0x3E124925, 0x3E4CCCCD, 0x3EAAAAAB, 0x3F800000)]
SP_HI = f32c(0x41A00000)                                     # 20
Q127, INV127 = f32c(0x42FE0000), f32c(0x3C010204)             # 127, fp32(1/127)


def add_to_exponent(y, e) -> np.ndarray:
    """numerics.py:126-132 - e added to the biased exponent of a positive normal y, exactly;
    >= 255 gives +inf, <= 0 gives +0. The sign of y is not kept."""
    yb = bits(y).astype(np.int64)
    ne = ((yb >> 23) & 0xFF) + np.asarray(e, np.int64)
    out = np.where(ne >= 255, 0x7F800000, np.where(ne <= 0, 0, (ne << 23) | (yb & 0x7FFFFF)))
    return from_bits(out)


def _horner(coeffs, z) -> np.ndarray:
    """c0 z^k + ... + ck with one fmul and one fadd per step, highest power first."""
    acc = np.full_like(z, coeffs[0])
    for c in coeffs[1:]:
        acc = fadd(fmul(acc, z), c)
    return acc


def exp_f(x) -> np.ndarray:
    """numerics.py:135-150 - n = rint(x log2 e) clamped to +-200, r = x - n ln2 (two-part ln2),
    the degree-6 polynomial of r, n added to its exponent; +inf from 89 up, +0 from -104 down."""
    x = ftz(x)
    with np.errstate(invalid="ignore"):
        n = np.clip(np.rint(fmul(x, LOG2E)), -200, 200).astype(F32)
        over, under = x >= EXP_HI, x <= EXP_LO
    r = fadd(fadd(x, fmul(n, NEG_LN2_HI)), fmul(n, NEG_LN2_LO))
    y = add_to_exponent(_horner(EXP_POLY, r), np.nan_to_num(n, nan=0).astype(np.int64))
    y = np.select([np.isnan(x), over, under], [F32(np.nan), F32(np.inf), F32(0)], y)
    return canon(y.astype(F32))


def recip_f(x) -> np.ndarray:
    """numerics.py:153-168 - magic seed on the mantissa scaled to [1, 2), three Newton steps in
    correction form, then the exponent put back exactly."""
    x = ftz(x)
    b = bits(x).astype(np.int64)
    sgn, a = b & 0x80000000, b & 0x7FFFFFFF
    mb = (a & 0x7FFFFF) | (127 << 23)
    m = from_bits(mb)
    y = from_bits(np.int64(RECIP_MAGIC) - mb)
    for _ in range(3):
        y = fadd(y, fmul(y, fadd(ONE, neg(fmul(m, y)))))
    y = from_bits(bits(add_to_exponent(y, -((a >> 23) - 127))).astype(np.int64) | sgn)
    y = np.where(a == 0, from_bits(sgn | 0x7F800000), y)
    y = np.where(a == 0x7F800000, from_bits(sgn), y)
    return canon(np.where(np.isnan(x), F32(np.nan), y).astype(F32))


def rsqrt_f(x) -> np.ndarray:
    """numerics.py:171-191 - exponent split E = 2k + j, mantissa scaled to [1, 4), magic seed,
    three Newton steps, k subtracted from the exponent."""
    x = ftz(x)
    b = bits(x).astype(np.int64)
    E = ((b >> 23) & 0xFF) - 127
    j, k = E & 1, E >> 1
    mb = (b & 0x7FFFFF) | ((127 + j) << 23)
    m = from_bits(mb)
    y = from_bits(np.int64(RSQRT_MAGIC) - (mb >> 1))
    for _ in range(3):
        y = fadd(y, fmul(y, fadd(HALF, neg(fmul(HALF, fmul(fmul(m, y), y))))))
    with np.errstate(invalid="ignore"):
        nan_out = np.isnan(x) | (x < F32(0))
    signed_inf = from_bits((b & 0x80000000) | 0x7F800000)
    y = np.select([nan_out, b == 0x7F800000, (b & 0x7FFFFFFF) == 0], [F32(np.nan), F32(0), signed_inf],
                  add_to_exponent(y, -k))
    return canon(y.astype(F32))


def gelu_f(x) -> np.ndarray:
    """numerics.py:194-201 - tanh-form GELU with tanh(u) = 1 - 2 recip(exp(2u) + 1)."""
    x = ftz(x)
    x3 = fmul(fmul(x, x), x)
    u = fmul(GELU_C, fadd(x, fmul(GELU_A, x3)))
    t = fadd(ONE, neg(fmul(TWO, recip_f(fadd(exp_f(fmul(TWO, u)), ONE)))))
    return fmul(fmul(HALF, x), fadd(ONE, t))


def sigmoid_f(x) -> np.ndarray:
    """numerics.py:241-244."""
    x = ftz(x)
    return recip_f(fadd(ONE, exp_f(neg(x))))


def silu_f(x) -> np.ndarray:
    """numerics.py:204-207."""
    x = ftz(x)
    return fmul(x, recip_f(fadd(ONE, exp_f(neg(x)))))


def softplus_f(x) -> np.ndarray:
    """numerics.py:247-262."""
    x = ftz(x)
    t = exp_f(neg(fabs(x)))
    s = fmul(t, recip_f(fadd(t, TWO)))
    p = _horner(LOG1P_POLY, fmul(s, s))
    y = fadd(np.where(x > F32(0), x, F32(0)).astype(F32), fmul(fmul(TWO, s), p))
    with np.errstate(invalid="ignore"):
        big = x > SP_HI
    return canon(np.select([np.isnan(x), big], [F32(np.nan), x], y).astype(F32))


def act_fn(x, act: int) -> np.ndarray:
    """numerics.py:210-230 - the epilogue activation codes 0..7."""
    x = ftz(x)
    if act == 0:
        return x
    if act in (1, 2):
        r = np.where(x > F32(0), x, F32(0)).astype(F32)
        return r if act == 1 else np.where(r > F32(6), F32(6), r).astype(F32)
    return {3: gelu_f, 4: silu_f, 5: sigmoid_f, 6: softplus_f, 7: exp_f}[act](x)


# ---------------------------------------------------------------- row reductions
def fmax(a, b) -> np.ndarray:
    """numerics.py:293-303 - NaN wins (canonical); of two equal values the sign bit is the AND
    of both signs."""
    a, b = ftz(a), ftz(b)
    with np.errstate(invalid="ignore"):
        eq = a == b
        m = np.where(a > b, a, b)
    ab, bb = bits(a), bits(b)
    tie = ((ab & bb & _SIGN) | (ab & U32(0x7FFFFFFF))).view(F32)
    m = np.where(eq, tie, m)
    return canon(np.where(np.isnan(a) | np.isnan(b), F32(np.nan), m).astype(F32))


def sum16(v) -> np.ndarray:
    """numerics.py:306-316 - element j to lane j mod 16, each lane a sequential fadd chain from
    +0, then four pairwise folds (0+1, 2+3, ...)."""
    v = np.asarray(v, F32)
    M, N = v.shape
    assert N % 16 == 0
    lanes = np.zeros((M, 16), F32)
    blocks = v.reshape(M, N // 16, 16)
    for c in range(N // 16):
        lanes = fadd(lanes, blocks[:, c, :])
    for half in (8, 4, 2, 1):                   # lane 2i + lane 2i+1 into lane i
        pairs = lanes.reshape(M, half, 2)
        lanes = fadd(pairs[:, :, 0], pairs[:, :, 1])
    return lanes[:, 0]


def max16(v) -> np.ndarray:
    """numerics.py:319-325 - row maxima under fmax (pairwise fold; fmax is order-free)."""
    v = np.asarray(v, F32)
    while v.shape[1] > 1:
        if v.shape[1] % 2:
            v = np.concatenate([fmax(v[:, :1], v[:, -1:]), v[:, 1:-1]], axis=1)
            continue
        v = fmax(v[:, 0::2], v[:, 1::2])
    return v[:, 0]


def inv_n(n: int) -> np.float32:
    """numerics.py:336-338 - 1/N = recip(i2f(N))."""
    return recip_f(i2f(np.array([n])))[0]


def softmax_rows(x) -> np.ndarray:
    """numerics.py:328-333."""
    x = ftz(x)
    mx = max16(x)[:, None]
    e = exp_f(fadd(x, neg(mx)))
    return fmul(e, recip_f(sum16(e))[:, None])


def softmax_rows_causal(x, valid) -> np.ndarray:
    """numerics.py:362-371 - row m: the first valid[m] elements; the rest output +0 and add +0."""
    x = ftz(x)
    M, N = x.shape
    valid = np.asarray(valid)
    keep = np.arange(N)[None, :] < valid[:, None]
    mx = np.array([max16(x[m:m + 1, :valid[m]])[0] for m in range(M)], F32)[:, None]
    e = np.where(keep, exp_f(fadd(x, neg(mx))), F32(0)).astype(F32)
    return fmul(e, recip_f(sum16(e))[:, None])


def _normalise(v, sq_sum, eps, gamma, beta) -> np.ndarray:
    """The tail the three norms share: v * rsqrt(sq_sum + eps) * gamma [+ beta], per row."""
    rs = rsqrt_f(fadd(sq_sum, eps))
    out = fmul(fmul(v, rs[:, None]), gamma[None, :])
    if beta is not None:
        out = fadd(out, beta[None, :])
    return out


def layernorm_rows(x, gamma, beta, eps) -> np.ndarray:
    """numerics.py:341-350 - mean = sum16(x) / N, d = x - mean, variance = sum16(d d) / N."""
    x = ftz(x)
    k = inv_n(x.shape[1])
    d = fadd(x, neg(fmul(sum16(x), k)[:, None]))
    return _normalise(d, fmul(sum16(fmul(d, d)), k), eps, gamma, beta)


def rmsnorm_rows(x, gamma, beta, eps) -> np.ndarray:
    """numerics.py:353-358 - mean square sum16(x x) / N."""
    x = ftz(x)
    return _normalise(x, fmul(sum16(fmul(x, x)), inv_n(x.shape[1])), eps, gamma, beta)


def l2norm_rows(x, gamma, beta, eps) -> np.ndarray:
    """numerics.py:374-380 - RMSNorm without the 1/N."""
    x = ftz(x)
    return _normalise(x, sum16(fmul(x, x)), eps, gamma, beta)


def quant_rows(x) -> tuple[np.ndarray, np.ndarray]:
    """numerics.py:383-390 - per-row symmetric INT8: amax = max16(|x|), q = q8(x, 127 recip(amax)),
    s = amax * fp32(1/127)."""
    x = ftz(x)
    amax = max16(fabs(x))
    row_scale = fmul(amax, INV127)
    return q8(x, fmul(Q127, recip_f(amax))[:, None]), row_scale


def fdot_nt(a, b) -> np.ndarray:
    """numerics.py:393-399 - y[m][n] = sum16 over k of a[m][k] b[n][k]."""
    a, b = ftz(a), ftz(b)
    M, K = a.shape
    N = b.shape[0]
    return sum16(fmul(a[:, None, :], b[None, :, :]).reshape(M * N, K)).reshape(M, N)


def fdot_nn(a, b) -> np.ndarray:
    """numerics.py:402-409 - y[m][n] = (((+0 + a[m][0] b[0][n]) + a[m][1] b[1][n]) + ...)."""
    a, b = ftz(a), ftz(b)
    y = np.zeros((a.shape[0], b.shape[1]), F32)
    for k in range(a.shape[1]):
        y = fadd(y, fmul(a[:, k:k + 1], b[k:k + 1, :]))
    return y


def rope_rows(x, tab, rows_per_pos: int, rot: int) -> np.ndarray:
    """numerics.py:412-424."""
    x = ftz(x)
    h = rot // 2
    t = ftz(tab)[np.arange(x.shape[0]) // rows_per_pos]
    c, s = t[:, :h], t[:, h:rot]
    y = x.copy()
    y[:, :h] = fadd(fmul(x[:, :h], c), neg(fmul(x[:, h:rot], s)))
    y[:, h:rot] = fadd(fmul(x[:, h:rot], c), fmul(x[:, :h], s))
    return y


def align_w4_groups(x) -> tuple[np.ndarray, np.ndarray]:
    """numerics.py:55-98 - per (row, 128-group) block-FP alignment to INT16 mantissas and an fp32
    group scale: emax_eff = max(emax, 14), shift 10 + emax_eff - e with RNE, scale bits
    (emax_eff - 13) << 23; NaN group -> zero mantissas + canonical NaN scale; inf group (no NaN)
    -> +-16384 at the infinities, 0 elsewhere, +inf scale; all-zero group -> scale 0."""
    b = bits(ftz(x)).astype(np.int64)
    M, K = b.shape
    if K == 0 or K % 128:
        raise ValueError("W4A16 activations need [M, K], K a nonzero multiple of 128")
    b = b.reshape(M, K // 128, 128)
    neg_sign = (b & 0x80000000) != 0
    e = (b >> 23) & 0xFF
    fr = b & 0x7FFFFF
    isnan = (e == 255) & (fr != 0)
    isinf = (e == 255) & (fr == 0)
    gnan = isnan.any(axis=2)
    ginf = isinf.any(axis=2) & ~gnan
    emax = np.where(e == 0, 0, e).max(axis=2)
    eff = np.maximum(emax, 14)
    sh = 10 + eff[:, :, None] - e
    u = (1 << 23) | fr
    s = np.clip(sh, 0, 31)
    kept = u >> s
    rem = u & ((np.int64(1) << s) - 1)
    half = np.int64(1) << np.clip(s - 1, 0, 30)
    up = (s > 0) & ((rem > half) | ((rem == half) & ((kept & 1) != 0)))
    mag = np.where((e == 0) | (sh >= 25) | (e == 255), 0, kept + up)
    mag = np.where(isinf & ~gnan[:, :, None], 16384, mag)
    mag = np.where(gnan[:, :, None], 0, mag)
    q = np.where(neg_sign, -mag, mag).astype(np.int16).reshape(M, K)
    sb = (np.clip(eff - 13, 0, 255).astype(np.int64) << 23)
    sb = np.where(emax == 0, 0, sb)
    sb = np.where(ginf, 0x7F800000, sb)
    sb = np.where(gnan, CANON_NAN_BITS, sb)
    return q, from_bits(sb)
