// Contract codes shared by host and device code (contract.py:40-114 of the reference).
#pragma once

namespace tc {

enum : int { MAGIC = 0xAA55, VERSION = 0x0002 };
enum : int { OP_CONV = 1, OP_GEMM = 2, OP_RELU = 3, OP_ROW = 4, OP_CONV_ACT = 5, OP_ELT = 6, OP_ROPE = 7, OP_FDOT = 8 };
enum : int { ROW_SOFTMAX = 0, ROW_LAYERNORM = 1, ROW_RMSNORM = 2, ROW_L2NORM = 3, ROW_QUANT = 4 };
enum : int { ELT_MUL = 0, ELT_ADD = 1, ELT_MULADD = 2, ELT_SUB = 3 };
enum : int { BM_DENSE = 0, BM_ROW = 1, BM_COL = 2, BM_SCALAR = 3 };
enum : int { QM_NONE = 0, QM_TENSOR = 1, QM_CHANNEL = 2, QM_ROWCOL = 3 };
enum : int { DT_BF16 = 0, DT_INT8 = 1, DT_INT4 = 2, DT_FP8 = 3, DT_FP32 = 4 };
enum : int { OUT_FP32 = 0, OUT_BF16 = 1, OUT_INT8 = 2, OUT_FP16 = 3 };
enum : int { STATE_FP16 = 8, W4_GROUP = 128 };
enum : int { E_OK = 0, E_MAGIC, E_VERSION, E_CRC, E_VALID, E_OPCODE, E_FIELD, E_ALIGN, E_RANGE };

}  // namespace tc
