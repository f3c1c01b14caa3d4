"""The tars_mini v0.4 descriptor contract on the host: field table, codes, encode/decode.

Mirrors the reference's tars_mini/contract.py call surface (contract.py:14-181) so descriptor
emitters (the compiler and the program builders) and tests written against it run unchanged. The device
side decodes and validates in C++ (libtarscuda); this module only builds and reads descriptors.
"""
from __future__ import annotations

import zlib

import numpy as np

# (hi, lo) bit positions, little endian: byte i holds bits 8i+7..8i (contract.py:14-38)
LAYOUT = {
    "MAGIC": (511, 496), "VERSION": (495, 480), "CORE_ID": (479, 472), "HDR_RSV": (471, 448),
    "OPCODE": (447, 432), "CTRL": (431, 416), "GROUP_SIZE": (415, 400), "EPI": (399, 384),
    "BASE_ADDR": (383, 320), "A_OFF": (319, 288), "W_OFF": (287, 256), "Y_OFF": (255, 224),
    "SCALE_OFF": (223, 192), "BIAS_OFF": (191, 160), "M": (159, 144), "N": (143, 128), "K": (127, 112),
    "LDA16": (111, 96), "OUT_SCALE": (95, 64), "CRC32": (63, 32), "VALID": (31, 31), "LDY16": (30, 16),
    "DEP_SIG": (15, 0),
}
FIELD_ORDER = tuple(LAYOUT)            # the order libtarscuda's tc_validate returns fields in

DESC_BYTES = 64
MAGIC, VERSION = 0xAA55, 0x0002
OP_GEMM, OP_RELU, OP_ROW = 0x02, 0x03, 0x04
ROW_SOFTMAX, ROW_LAYERNORM, ROW_RMSNORM = 0, 1, 2
OP_CONV, OP_CONV_ACT = 0x01, 0x05
CONV_OPS = (OP_CONV, OP_CONV_ACT)
OP_ELT, OP_ROPE, OP_FDOT = 0x06, 0x07, 0x08
V04_OPS = (OP_ELT, OP_ROPE, OP_FDOT)
ELT_MUL, ELT_ADD, ELT_MULADD, ELT_SUB = 0, 1, 2, 3
BM_DENSE, BM_ROW, BM_COL, BM_SCALAR = 0, 1, 2, 3
AM_DENSE, AM_ROW = 0, 1
FDOT_NT, FDOT_NN = 0, 1
ROW_L2NORM, ROW_QUANT = 3, 4
QM_NONE, QM_TENSOR, QM_CHANNEL, QM_ROWCOL = 0, 1, 2, 3
QM_GROUP = QM_ROWCOL
DT_BF16, DT_INT8, DT_INT4, DT_FP8, DT_FP32 = 0, 1, 2, 3, 4
W4_GROUP = 128
W4A16_MIN_VERSION = 0x00040001
ACT_NONE, ACT_RELU, ACT_RELU6, ACT_GELU, ACT_SILU = 0, 1, 2, 3, 4
ACT_SIGMOID, ACT_SOFTPLUS, ACT_EXP = 5, 6, 7
OUT_FP32, OUT_BF16, OUT_INT8, OUT_FP16 = 0, 1, 2, 3
ESIZE = {OUT_FP32: 4, OUT_BF16: 2, OUT_INT8: 1, OUT_FP16: 2}
STATE_FP16 = 1 << 3
FP16_MIN_VERSION = 0x00030400
E_OK, E_MAGIC, E_VERSION, E_CRC, E_VALID, E_OPCODE, E_FIELD, E_ALIGN, E_RANGE = range(9)
ERR_NAMES = {E_OK: "OK", E_MAGIC: "E_MAGIC", E_VERSION: "E_VERSION", E_CRC: "E_CRC", E_VALID: "E_VALID",
             E_OPCODE: "E_OPCODE", E_FIELD: "E_FIELD", E_ALIGN: "E_ALIGN", E_RANGE: "E_RANGE"}
K_MAX = 65535
CANON_NAN = 0x7FC00000


def _span(name: str) -> tuple[int, int]:
    """(first bit, width) of a field."""
    hi, lo = LAYOUT[name]
    return lo, hi - lo + 1


def _pack(*parts: tuple[int, int]) -> int:
    """Packs (value, width) pairs from bit 0 upwards, each value masked to its width."""
    word, at = 0, 0
    for val, w in parts:
        word |= (val & ((1 << w) - 1)) << at
        at += w
    return word


def _unpack(word: int, *widths: int) -> list[int]:
    out, at = [], 0
    for w in widths:
        out.append(word >> at & ((1 << w) - 1))
        at += w
    return out


def check_layout() -> None:
    """Every bit of the 512-bit descriptor belongs to exactly one field."""
    nxt = 0
    for lo, w in sorted(_span(n) for n in LAYOUT):
        if lo != nxt or w < 1:
            raise AssertionError("fields overlap or leave holes")
        nxt = lo + w
    if nxt != 8 * DESC_BYTES:
        raise AssertionError("fields overlap or leave holes")


def width(name: str) -> int:
    return _span(name)[1]


def conv_geom(h: int, kh: int, kw: int, stride: int = 1, pad: int = 0) -> int:
    """The CONV geometry word in HDR_RSV: pad (2 bits), stride - 1 (2), KW (4), KH (4), H (12)."""
    if not (0 < h < 4096 and 0 < kh < 16 and 0 < kw < 16 and 1 <= stride <= 4 and 0 <= pad <= 3):
        raise AssertionError(f"conv geometry h={h} kh={kh} kw={kw} stride={stride} pad={pad}")
    return _pack((pad, 2), (stride - 1, 2), (kw, 4), (kh, 4), (h, 12))


def conv_params(d: dict) -> dict:
    """A CONV descriptor's geometry: input H x W (W in GROUP_SIZE), kernel, stride, pad, input
    channels (K / (KH KW)) and the output size."""
    p, s1, kw, kh, h = _unpack(d["HDR_RSV"], 2, 2, 4, 4, 12)
    s, w = s1 + 1, d["GROUP_SIZE"]
    taps = kh * kw
    return dict(H=h, W=w, KH=kh, KW=kw, S=s, P=p, Cin=d["K"] // taps if taps else 0,
                OH=(h + 2 * p - kh) // s + 1, OW=(w + 2 * p - kw) // s + 1)


def ctrl(qmode: int = QM_TENSOR, symmetric: int = 1, a_dtype: int = DT_INT8, w_dtype: int = DT_INT8,
         fusion: int = 0) -> int:
    """CTRL of a GEMM: quant mode (3 bits), symmetric (1), A type (4), W type (4), fusion (1)."""
    return _pack((qmode, 3), (symmetric, 1), (a_dtype, 4), (w_dtype, 4), (fusion, 1))


def epi(act: int = ACT_NONE, out: int = OUT_FP32, bias: int = 0) -> int:
    """EPI: activation bits 0-1, output format (2), bias flag (1), activation bit 2 (1)."""
    return _pack((act, 2), (out, 2), (bias, 1), (act >> 2, 1))


def act_of(e: int) -> int:
    lo2, _, _, hi1 = _unpack(e, 2, 2, 1, 1)
    return lo2 | hi1 << 2


def f32_bits(x: float) -> int:
    return int(np.array(x, np.float32).view(np.uint32))


def bits_f32(b: int) -> np.float32:
    return np.array(b & 0xFFFFFFFF, np.uint32).view(np.float32)[()]


def _crc(raw: bytes) -> int:
    """CRC-32/ISO-HDLC of the 64 bytes with the CRC field (bytes 4..7) read as zero."""
    raw = bytes(raw)
    return zlib.crc32(raw[8:], zlib.crc32(raw[:4] + bytes(4)))


def encode(fields: dict, *, fix_crc: bool = True) -> bytes:
    """64 bytes, little endian; fields not given are 0; the CRC (CRC-32/ISO-HDLC over all 64
    bytes with bytes 4..7 zeroed) is filled in unless fix_crc is False."""
    word = 0
    for name, val in fields.items():
        lo, w = _span(name)
        val = int(val)
        if val < 0 or val >> w:
            raise ValueError(f"{name}={val} does not fit {w} bits")
        word |= val << lo
    raw = bytearray(word.to_bytes(DESC_BYTES, "little"))
    if fix_crc:
        raw[4:8] = _crc(raw).to_bytes(4, "little")
    return bytes(raw)


def decode(raw: bytes) -> dict:
    word = int.from_bytes(raw, "little")
    return {name: word >> lo & ((1 << w) - 1) for name, (lo, w) in ((n, _span(n)) for n in LAYOUT)}


def crc_ok(raw: bytes) -> bool:
    return int.from_bytes(bytes(raw[4:8]), "little") == _crc(raw)
