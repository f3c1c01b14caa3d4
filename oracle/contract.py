"""CPU oracle, part 2: the 512-bit descriptor of contract v0.4, restated.

TEST INFRASTRUCTURE ONLY (see oracle/numerics.py's header for who may use it).

Restates the reference's tars_mini/contract.py: the field table (contract.py:14-38), the codes
(contract.py:40-114), ctrl/epi/act_of (131-143), encode/decode/crc_ok (154-181). A descriptor is
64 bytes little endian (byte i holds bits 8i+7..8i); the CRC-32/ISO-HDLC covers all 64 bytes with
bytes 4..7 zeroed.
"""
from __future__ import annotations

import struct
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


def ctrl(qmode=QM_TENSOR, symmetric=1, a_dtype=DT_INT8, w_dtype=DT_INT8, fusion=0) -> int:
    """contract.py:131-134."""
    return (qmode & 7) | (symmetric & 1) << 3 | (a_dtype & 15) << 4 | (w_dtype & 15) << 8 | (fusion & 1) << 12


def epi(act=ACT_NONE, out=OUT_FP32, bias=0) -> int:
    """contract.py:137-138 - the 3-bit activation code is EPI[1:0] | EPI[5] << 2."""
    return (act & 3) | (out & 3) << 2 | (bias & 1) << 4 | (act >> 2 & 1) << 5


def act_of(e: int) -> int:
    """contract.py:141-143."""
    return (e & 3) | (e >> 5 & 1) << 2


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bits_f32(b: int) -> np.float32:
    return np.frombuffer(struct.pack("<I", b & 0xFFFFFFFF), "<f4")[0]


def crc32_desc(raw: bytes) -> int:
    z = bytearray(raw)
    z[4:8] = b"\0\0\0\0"
    return zlib.crc32(bytes(z)) & 0xFFFFFFFF


def encode(fields: dict, *, fix_crc: bool = True) -> bytes:
    """contract.py:154-170."""
    v = 0
    for name, val in fields.items():
        hi, lo = FIELDS[name]
        if not 0 <= val < (1 << (hi - lo + 1)):
            raise ValueError(f"{name}={val} does not fit {hi - lo + 1} bits")
        v |= val << lo
    raw = bytearray(v.to_bytes(DESC_BYTES, "little"))
    if fix_crc:
        raw[4:8] = struct.pack("<I", crc32_desc(bytes(raw)))
    return bytes(raw)


def decode(raw: bytes) -> dict:
    """contract.py:173-175."""
    v = int.from_bytes(raw, "little")
    return {n: (v >> lo) & ((1 << (hi - lo + 1)) - 1) for n, (hi, lo) in FIELDS.items()}


def crc_ok(raw: bytes) -> bool:
    """contract.py:178-181."""
    return struct.unpack("<I", bytes(raw[4:8]))[0] == crc32_desc(raw)


def conv_params(d: dict) -> dict:
    """contract.py:79-85 - conv geometry from HDR_RSV / GROUP_SIZE."""
    g = d["HDR_RSV"]
    h, kh, kw, s, p, w = g >> 12, g >> 8 & 15, g >> 4 & 15, (g >> 2 & 3) + 1, g & 3, d["GROUP_SIZE"]
    cin = d["K"] // (kh * kw) if kh and kw else 0
    return dict(H=h, W=w, KH=kh, KW=kw, S=s, P=p, Cin=cin,
                OH=(h + 2 * p - kh) // s + 1, OW=(w + 2 * p - kw) // s + 1)
