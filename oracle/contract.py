"""CPU oracle, part 2: the 512-bit descriptor of contract v0.4, restated.

TEST INFRASTRUCTURE ONLY (see oracle/numerics.py's header for who may use it).

Restates the reference's tars_mini/contract.py: the field table (contract.py:14-38), the codes
(contract.py:40-114), ctrl/epi/act_of (131-143), encode/decode/crc_ok (154-181). A descriptor is
64 bytes little endian (byte i holds bits 8i+7..8i); the CRC-32/ISO-HDLC covers all 64 bytes with
bytes 4..7 zeroed.
"""
from __future__ import annotations

import zlib

import numpy as np

# name: (hi, lo) - bit 511 is the top bit of byte 63
FIELDS = {
    "MAGIC": (511, 496), "VERSION": (495, 480), "CORE_ID": (479, 472), "HDR_RSV": (471, 448),
    "OPCODE": (447, 432), "CTRL": (431, 416), "GROUP_SIZE": (415, 400), "EPI": (399, 384),
    "BASE_ADDR": (383, 320), "A_OFF": (319, 288), "W_OFF": (287, 256), "Y_OFF": (255, 224),
    "SCALE_OFF": (223, 192), "BIAS_OFF": (191, 160), "M": (159, 144), "N": (143, 128),
    "K": (127, 112), "LDA16": (111, 96), "OUT_SCALE": (95, 64), "CRC32": (63, 32),
    "VALID": (31, 31), "LDY16": (30, 16), "DEP_SIG": (15, 0),
}
DESC_BYTES = 64
MAGIC, VERSION = 0xAA55, 0x0002

OP_CONV, OP_GEMM, OP_RELU, OP_ROW, OP_CONV_ACT = 0x01, 0x02, 0x03, 0x04, 0x05
OP_ELT, OP_ROPE, OP_FDOT = 0x06, 0x07, 0x08
CONV_OPS = (OP_CONV, OP_CONV_ACT)
V04_OPS = (OP_ELT, OP_ROPE, OP_FDOT)
ROW_SOFTMAX, ROW_LAYERNORM, ROW_RMSNORM, ROW_L2NORM, ROW_QUANT = 0, 1, 2, 3, 4
ELT_MUL, ELT_ADD, ELT_MULADD, ELT_SUB = 0, 1, 2, 3
BM_DENSE, BM_ROW, BM_COL, BM_SCALAR = 0, 1, 2, 3
QM_NONE, QM_TENSOR, QM_CHANNEL, QM_ROWCOL = 0, 1, 2, 3
QM_GROUP = QM_ROWCOL
DT_BF16, DT_INT8, DT_INT4, DT_FP8, DT_FP32 = 0, 1, 2, 3, 4
W4_GROUP = 128
ACT_NONE, ACT_RELU, ACT_RELU6, ACT_GELU, ACT_SILU, ACT_SIGMOID, ACT_SOFTPLUS, ACT_EXP = range(8)
OUT_FP32, OUT_BF16, OUT_INT8, OUT_FP16 = 0, 1, 2, 3
ESIZE = {OUT_FP32: 4, OUT_BF16: 2, OUT_INT8: 1, OUT_FP16: 2}
STATE_FP16 = 1 << 3
E_OK, E_MAGIC, E_VERSION, E_CRC, E_VALID, E_OPCODE, E_FIELD, E_ALIGN, E_RANGE = range(9)
K_MAX = 65535
CANON_NAN = 0x7FC00000


# sub-fields of CTRL and EPI: name -> (first bit, width) (contract.py:131-143); the 3-bit
# activation code is split, its bit 2 stored at EPI bit 5
CTRL_BITS = {"qmode": (0, 3), "symmetric": (3, 1), "a_dtype": (4, 4), "w_dtype": (8, 4), "fusion": (12, 1)}
EPI_BITS = {"act_lo": (0, 2), "out": (2, 2), "bias": (4, 1), "act_hi": (5, 1)}
# the CONV geometry word in HDR_RSV (contract.py:72-85)
CONV_BITS = {"pad": (0, 2), "stride_m1": (2, 2), "kw": (4, 4), "kh": (8, 4), "h": (12, 12)}


def _put(table: dict, **vals) -> int:
    return sum((v & ((1 << table[k][1]) - 1)) << table[k][0] for k, v in vals.items())


def _get(table: dict, word: int, key: str) -> int:
    at, w = table[key]
    return (word >> at) % (1 << w)


def ctrl(qmode=QM_TENSOR, symmetric=1, a_dtype=DT_INT8, w_dtype=DT_INT8, fusion=0) -> int:
    """contract.py:131-134."""
    return _put(CTRL_BITS, qmode=qmode, symmetric=symmetric, a_dtype=a_dtype, w_dtype=w_dtype, fusion=fusion)


def epi(act=ACT_NONE, out=OUT_FP32, bias=0) -> int:
    """contract.py:137-138."""
    return _put(EPI_BITS, act_lo=act, out=out, bias=bias, act_hi=act >> 2)


def act_of(e: int) -> int:
    """contract.py:141-143."""
    return _get(EPI_BITS, e, "act_lo") + 4 * _get(EPI_BITS, e, "act_hi")


def f32_bits(x: float) -> int:
    return int(np.float32(x).view(np.uint32))


def bits_f32(b: int) -> np.float32:
    return np.uint32(b & 0xFFFFFFFF).view(np.float32)


def crc32_desc(raw: bytes) -> int:
    """CRC-32/ISO-HDLC of the descriptor with bytes 4..7 taken as zero."""
    return zlib.crc32(b"".join((bytes(raw[:4]), b"\0" * 4, bytes(raw[8:DESC_BYTES]))))


def _bit_array(raw: bytes) -> np.ndarray:
    """The 512 bits, bit i = bit i % 8 of byte i // 8."""
    return np.unpackbits(np.frombuffer(bytes(raw), np.uint8), bitorder="little")


def encode(fields: dict, *, fix_crc: bool = True) -> bytes:
    """contract.py:154-170, built bit by bit."""
    bits = np.zeros(8 * DESC_BYTES, np.uint8)
    for name, val in fields.items():
        hi, lo = FIELDS[name]
        n = hi - lo + 1
        val = int(val)
        if val < 0 or val.bit_length() > n:
            raise ValueError(f"{name}={val} does not fit {n} bits")
        bits[lo:hi + 1] = [(val >> i) & 1 for i in range(n)]
    raw = bytearray(np.packbits(bits, bitorder="little").tobytes())
    if fix_crc:
        raw[4:8] = crc32_desc(raw).to_bytes(4, "little")
    return bytes(raw)


def decode(raw: bytes) -> dict:
    """contract.py:173-175, read bit by bit."""
    bits = _bit_array(raw)
    weights = [1 << i for i in range(64)]
    return {name: sum(w for w, b in zip(weights, bits[lo:hi + 1]) if b) for name, (hi, lo) in FIELDS.items()}


def crc_ok(raw: bytes) -> bool:
    """contract.py:178-181."""
    return int.from_bytes(bytes(raw[4:8]), "little") == crc32_desc(raw)


def conv_params(d: dict) -> dict:
    """contract.py:79-85 - conv geometry from HDR_RSV / GROUP_SIZE."""
    g = {k: _get(CONV_BITS, d["HDR_RSV"], k) for k in CONV_BITS}
    h, w, kh, kw, p, s = g["h"], d["GROUP_SIZE"], g["kh"], g["kw"], g["pad"], g["stride_m1"] + 1
    return dict(H=h, W=w, KH=kh, KW=kw, S=s, P=p, Cin=d["K"] // (kh * kw) if kh * kw else 0,
                OH=(h - kh + 2 * p) // s + 1, OW=(w - kw + 2 * p) // s + 1)
