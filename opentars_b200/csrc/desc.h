// Descriptor decode, CRC-32 and contract validation for the tars_mini v0.4 queue (host side).
//
// Restates the reference's tars_mini/contract.py (field table, codes) and the checks of
// tars_mini/golden.py Machine.validate / strides / bstride / segments / extra_out / _overlaps /
// _in_place (golden.py:59-266, 437-447). All address arithmetic is done in 128-bit integers:
// BASE_ADDR is a 64-bit field and the reference computes in unbounded Python integers, so a
// footprint that wraps 2^64 must still be judged out of range.
#pragma once
#include <cstdint>
#include <cstddef>
#include <vector>

#include "codes.h"

namespace tc {

typedef unsigned __int128 u128;

enum Field {
  F_MAGIC, F_VERSION, F_CORE_ID, F_HDR_RSV, F_OPCODE, F_CTRL, F_GROUP_SIZE, F_EPI, F_BASE_ADDR,
  F_A_OFF, F_W_OFF, F_Y_OFF, F_SCALE_OFF, F_BIAS_OFF, F_M, F_N, F_K, F_LDA16, F_OUT_SCALE,
  F_CRC32, F_VALID, F_LDY16, F_DEP_SIG, F_COUNT
};

struct Desc {
  uint64_t f[F_COUNT];
  uint64_t operator[](int i) const { return f[i]; }
  int op() const { return (int)f[F_OPCODE]; }
  int ctrl() const { return (int)f[F_CTRL]; }
  int epi() const { return (int)f[F_EPI]; }
  int act() const { return (int)((f[F_EPI] & 3) | ((f[F_EPI] >> 5 & 1) << 2)); }
  int out() const { return (int)(f[F_EPI] >> 2 & 3); }
  bool bias() const { return f[F_EPI] >> 4 & 1; }
  int qmode() const { return (int)(f[F_CTRL] & 7); }
  bool w4() const { return op() == OP_GEMM && qmode() == QM_ROWCOL && ((f[F_CTRL] >> 8) & 15) == DT_INT4; }
  bool conv() const { return op() == OP_CONV || op() == OP_CONV_ACT; }
};

struct ConvGeom { int H, W, KH, KW, S, P, Cin, OH, OW; };
ConvGeom conv_geom(const Desc& d);

uint32_t crc32_iso_hdlc(const uint8_t* p, size_t n);
void decode(const uint8_t raw[64], Desc* d);
// The first failing check in contract order (E_MAGIC .. E_ALIGN); E_RANGE is judged by the
// footprint against the image size, in run_queue.
int validate(const uint8_t raw[64], const Desc& d, int core_id, int gemv_only);

struct Strides { uint64_t lda, ldy, arow, yrow; };
Strides strides(const Desc& d);
void bstride(const Desc& d, uint64_t* ldb, uint64_t* brow);

// A set of byte segments [base + i*ld, base + i*ld + nbytes), i < count (count >= 1).
struct Seg { u128 base, ld, nbytes, count; };
struct Footprint {
  std::vector<std::vector<Seg>> reads;   // per input tensor, in the reference's order
  Seg y;                                 // the output rows (ascending, disjoint: ld >= nbytes)
  bool has_extra = false;
  Seg extra{};                           // ROW_QUANT's second output (its row scales)
};
Footprint footprint(const Desc& d);
u128 seg_end(const Seg& s);              // one past the last byte
u128 seg_bytes(const Seg& s);
// Whether any segment of `a` intersects any row of `y` (y ascending and disjoint).
bool overlaps(const Seg& a, const Seg& y);
bool in_place(const Desc& d, int read_index);

}  // namespace tc
