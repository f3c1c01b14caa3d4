// Descriptor decode / CRC / validation / footprints (see desc.h for the reference citations).
#include "desc.h"

#include <cstring>

namespace tc {

namespace {
// (hi, lo) bit positions of each field, contract.py:14-38
const int kBits[F_COUNT][2] = {
    {511, 496}, {495, 480}, {479, 472}, {471, 448}, {447, 432}, {431, 416}, {415, 400}, {399, 384},
    {383, 320}, {319, 288}, {287, 256}, {255, 224}, {223, 192}, {191, 160}, {159, 144}, {143, 128},
    {127, 112}, {111, 96},  {95, 64},   {63, 32},   {31, 31},   {30, 16},   {15, 0}};

struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      t[i] = c;
    }
  }
};
const CrcTable kCrc;

uint64_t field(const uint8_t* raw, int hi, int lo) {
  uint64_t v = 0;
  int w = hi - lo + 1;
  for (int b = 0; b < w; ++b) {
    int bit = lo + b;
    v |= (uint64_t)((raw[bit >> 3] >> (bit & 7)) & 1) << b;
  }
  return v;
}
}  // namespace

uint32_t crc32_iso_hdlc(const uint8_t* p, size_t n) {
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = kCrc.t[(c ^ p[i]) & 0xFF] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

void decode(const uint8_t raw[64], Desc* d) {
  for (int i = 0; i < F_COUNT; ++i) d->f[i] = field(raw, kBits[i][0], kBits[i][1]);
}

ConvGeom conv_geom(const Desc& d) {
  ConvGeom g;
  uint64_t h = d[F_HDR_RSV];
  g.H = (int)(h >> 12);
  g.KH = (int)(h >> 8 & 15);
  g.KW = (int)(h >> 4 & 15);
  g.S = (int)((h >> 2 & 3) + 1);
  g.P = (int)(h & 3);
  g.W = (int)d[F_GROUP_SIZE];
  g.Cin = (g.KH && g.KW) ? (int)(d[F_K] / (uint64_t)(g.KH * g.KW)) : 0;
  // Python floor division: (H + 2P - KH) // S + 1 can be <= 0
  auto fdiv = [](int a, int b) { int q = a / b; if ((a % b != 0) && ((a < 0) != (b < 0))) --q; return q; };
  g.OH = fdiv(g.H + 2 * g.P - g.KH, g.S) + 1;
  g.OW = fdiv(g.W + 2 * g.P - g.KW, g.S) + 1;
  return g;
}

Strides strides(const Desc& d) {
  Strides s;
  static const uint64_t esize[4] = {4, 2, 1, 2};
  int op = d.op();
  if (d.w4()) s.arow = (((d[F_CTRL] >> 4) & 15) == DT_FP32 ? 4 : 2) * d[F_K];
  else if (op == OP_GEMM) s.arow = d[F_K];
  else if (d.conv()) s.arow = (uint64_t)conv_geom(d).Cin;
  else if (op == OP_FDOT) s.arow = 4 * d[F_K];
  else s.arow = ((op == OP_ELT && (d[F_HDR_RSV] & STATE_FP16)) ? 2 : 4) * d[F_N];
  s.yrow = d[F_N] * esize[d.out()];
  s.lda = d[F_LDA16] ? 16 * d[F_LDA16] : s.arow;
  s.ldy = d[F_LDY16] ? 16 * d[F_LDY16] : s.yrow;
  return s;
}

void bstride(const Desc& d, uint64_t* ldb, uint64_t* brow) {
  if (d.op() == OP_FDOT)
    *brow = ((d[F_HDR_RSV] & STATE_FP16) ? 2 : 4) * ((d[F_CTRL] & 1) ? d[F_N] : d[F_K]);
  else
    *brow = ((d[F_HDR_RSV] & 3) == BM_DENSE) ? 4 * d[F_N] : 0;
  *ldb = d[F_GROUP_SIZE] ? 16 * d[F_GROUP_SIZE] : *brow;
}

int validate(const uint8_t raw[64], const Desc& d, int core_id, int gemv_only) {
  if (d[F_MAGIC] != MAGIC) return E_MAGIC;
  if (d[F_VERSION] != VERSION) return E_VERSION;
  {
    uint8_t z[64];
    std::memcpy(z, raw, 64);
    std::memset(z + 4, 0, 4);
    if (crc32_iso_hdlc(z, 64) != (uint32_t)d[F_CRC32]) return E_CRC;
  }
  if (d[F_VALID] != 1) return E_VALID;
  const int op = d.op();
  const bool known = op == OP_GEMM || op == OP_RELU || op == OP_ROW || op == OP_CONV || op == OP_CONV_ACT ||
                     op == OP_ELT || op == OP_ROPE || op == OP_FDOT;
  if (!known) return E_OPCODE;
  if (gemv_only && (d.conv() || (op == OP_GEMM && d[F_K] > 4096))) return E_OPCODE;

  const bool conv = d.conv();
  const uint64_t c = d[F_CTRL], e = d[F_EPI];
  const int qm = (int)(c & 7), sym = (int)(c >> 3 & 1), adt = (int)(c >> 4 & 15), wdt = (int)(c >> 8 & 15);
  const int fus = (int)(c >> 12 & 1);
  const int act = d.act(), out = d.out();
  const bool bias = d.bias();
  const bool w4 = d.w4();
  const bool v04 = op == OP_ELT || op == OP_ROPE || op == OP_FDOT;
  const bool hdr_ok = conv || (op == OP_GEMM && qm == QM_ROWCOL && !w4) || (op == OP_ELT && d[F_HDR_RSV] < 16) ||
                      (op == OP_FDOT && (c & 1) && d[F_HDR_RSV] == STATE_FP16);
  const bool grp_ok = conv || v04 || w4;
  if (d[F_CORE_ID] != (uint64_t)core_id || d[F_DEP_SIG] || (d[F_HDR_RSV] && !hdr_ok) ||
      (d[F_GROUP_SIZE] && !grp_ok))
    return E_FIELD;
  if ((c >> 13) || (e >> 6) || (out == OUT_FP16 && op != OP_ELT)) return E_FIELD;
  if (out != OUT_INT8 && d[F_OUT_SCALE]) return E_FIELD;
  const bool gemm = op == OP_GEMM || conv;
  if (gemm) {
    if (w4) {
      if (sym != 1 || (adt != DT_FP32 && adt != DT_BF16) || d[F_HDR_RSV] != 0 || d[F_GROUP_SIZE] != W4_GROUP)
        return E_FIELD;
    } else if ((qm != QM_TENSOR && qm != QM_CHANNEL && qm != QM_ROWCOL) || sym != 1 || adt != DT_INT8 ||
               wdt != DT_INT8 || (conv && qm == QM_ROWCOL)) {
      return E_FIELD;
    }
    if ((act != 0) != (fus == 1)) return E_FIELD;
    if (op == OP_CONV_ACT && act == 0) return E_FIELD;
    if (conv) {
      ConvGeom g = conv_geom(d);
      if (!(g.H && g.W && g.KH && g.KW) || g.OH < 1 || g.OW < 1 || d[F_M] != (uint64_t)g.OH * (uint64_t)g.OW)
        return E_FIELD;
    }
  } else if (op == OP_RELU) {
    if (c || bias || d[F_K] || d[F_W_OFF] || d[F_SCALE_OFF] || d[F_BIAS_OFF] || act == 0) return E_FIELD;
  } else if (op == OP_ROW) {
    const int fn = (int)(c & 7);
    if ((c >> 3) || fn > ROW_QUANT || act != 0 || (d[F_K] && fn != ROW_SOFTMAX)) return E_FIELD;
    if (fn == ROW_SOFTMAX && (bias || d[F_W_OFF] || d[F_SCALE_OFF] || d[F_BIAS_OFF])) return E_FIELD;
    if (fn == ROW_QUANT && (bias || d[F_W_OFF] || d[F_BIAS_OFF] || out != OUT_INT8 || d[F_OUT_SCALE]))
      return E_FIELD;
    if (!bias && d[F_BIAS_OFF]) return E_FIELD;
  } else if (op == OP_ELT) {
    const int eop = (int)(c & 3);
    if ((c >> 2) || d[F_K] || d[F_SCALE_OFF] || bias != (eop == ELT_MULADD) ||
        (eop == ELT_MULADD && out != OUT_FP32 && out != OUT_FP16) || (!bias && d[F_BIAS_OFF]))
      return E_FIELD;
  } else if (op == OP_ROPE) {
    if (c || act != 0 || bias || d[F_SCALE_OFF] || d[F_BIAS_OFF] || d[F_GROUP_SIZE] == 0) return E_FIELD;
  } else {  // FDOT
    if ((c >> 1) || act != 0 || bias || d[F_SCALE_OFF] || d[F_BIAS_OFF]) return E_FIELD;
  }
  // E_ALIGN: shapes and offsets
  const uint64_t M = d[F_M], N = d[F_N], K = d[F_K];
  if (M == 0 || N == 0 || N % 16 || ((gemm || op == OP_FDOT) && (K == 0 || K % 16))) return E_ALIGN;
  if (w4 && (K < 256 || K % 256 || K > 8192 || d[F_W_OFF] % 128)) return E_ALIGN;
  if (op == OP_ROPE && (K == 0 || K % 32 || K > N)) return E_ALIGN;
  if (conv) {
    ConvGeom g = conv_geom(d);
    if (K % (uint64_t)(g.KH * g.KW) || g.Cin % 16) return E_ALIGN;
  }
  const int offs[5] = {F_A_OFF, F_Y_OFF, F_SCALE_OFF, F_BIAS_OFF, F_W_OFF};
  const int noffs = op == OP_ROW ? 4 : 5;
  for (int i = 0; i < noffs; ++i) {
    uint64_t al = 16;
    if (offs[i] == F_W_OFF && op == OP_ELT) {
      int bm = (int)(d[F_HDR_RSV] & 3);
      if (bm == BM_COL || bm == BM_SCALAR) al = 4;
    }
    if (d[offs[i]] % al) return E_ALIGN;
  }
  Strides s = strides(d);
  if (s.lda < s.arow || s.ldy < s.yrow) return E_ALIGN;
  if (op == OP_ELT || op == OP_FDOT) {
    uint64_t ldb, brow;
    bstride(d, &ldb, &brow);
    if (ldb < brow) return E_ALIGN;
  }
  return E_OK;
}

static Seg one(u128 lo, u128 n) { return Seg{lo, n, n, 1}; }
static Seg rows(u128 lo, u128 ld, u128 n, u128 count) { return Seg{lo, ld, n, count}; }

u128 seg_end(const Seg& s) { return s.base + (s.count - 1) * s.ld + s.nbytes; }
u128 seg_bytes(const Seg& s) { return s.count * s.nbytes; }

Footprint footprint(const Desc& d) {
  Footprint fp;
  const u128 B = d[F_BASE_ADDR], M = d[F_M], N = d[F_N], K = d[F_K];
  const Strides s = strides(d);
  const int op = d.op();
  fp.y = rows(B + d[F_Y_OFF], s.ldy, s.yrow, M);
  if (op == OP_ELT || op == OP_ROPE || op == OP_FDOT) {
    if (op == OP_ELT && (d[F_HDR_RSV] >> 2 & 1))
      fp.reads.push_back({one(B + d[F_A_OFF], s.arow)});
    else
      fp.reads.push_back({rows(B + d[F_A_OFF], s.lda, s.arow, M)});
    const u128 w0 = B + d[F_W_OFF];
    if (op == OP_ELT) {
      const int bm = (int)(d[F_HDR_RSV] & 3);
      if (bm == BM_DENSE) {
        uint64_t ldb, brow;
        bstride(d, &ldb, &brow);
        fp.reads.push_back({rows(w0, ldb, 4 * N, M)});
      } else {
        const u128 n = bm == BM_ROW ? 4 * N : bm == BM_COL ? 4 * M : 4;
        fp.reads.push_back({one(w0, n)});
      }
      if ((d[F_CTRL] & 3) == ELT_MULADD) fp.reads.push_back({rows(B + d[F_BIAS_OFF], s.ldy, s.yrow, M)});
    } else if (op == OP_ROPE) {
      const u128 nrows = (M - 1) / d[F_GROUP_SIZE] + 1;
      fp.reads.push_back({one(w0, 4 * K * nrows)});
    } else {
      uint64_t ldb, brow;
      bstride(d, &ldb, &brow);
      const u128 nb = (d[F_CTRL] & 1) ? K : N;
      fp.reads.push_back({rows(w0, ldb, brow, nb)});
    }
    return fp;
  }
  if (d.conv()) {
    ConvGeom g = conv_geom(d);
    const u128 npx = (u128)g.H * (u128)g.W;
    const u128 a0 = B + d[F_A_OFF];
    if (s.lda == s.arow)
      fp.reads.push_back({one(a0, npx * s.arow)});
    else
      fp.reads.push_back({rows(a0, s.lda, s.arow, npx)});
  } else {
    fp.reads.push_back({rows(B + d[F_A_OFF], s.lda, s.arow, M)});
  }
  if (op == OP_GEMM || d.conv()) {
    const bool w4 = d.w4();
    const u128 ns = d.qmode() == QM_TENSOR ? 1 : N;
    fp.reads.push_back({one(B + d[F_W_OFF], N * K / (w4 ? 2 : 1))});
    fp.reads.push_back({one(B + d[F_SCALE_OFF], w4 ? 2 * N * (K / W4_GROUP) : 4 * ns)});
    if (d.bias()) fp.reads.push_back({one(B + d[F_BIAS_OFF], 4 * N)});
    if (d.qmode() == QM_ROWCOL && !w4) fp.reads.push_back({one(B + 16 * (u128)d[F_HDR_RSV], 4 * M)});
  } else if (op == OP_ROW) {
    const int fn = (int)(d[F_CTRL] & 7);
    if (fn == ROW_LAYERNORM || fn == ROW_RMSNORM || fn == ROW_L2NORM) {
      fp.reads.push_back({one(B + d[F_SCALE_OFF], 4 * N)});
      if (d.bias()) fp.reads.push_back({one(B + d[F_BIAS_OFF], 4 * N)});
    }
    if (fn == ROW_QUANT) {
      fp.has_extra = true;
      fp.extra = one(B + d[F_SCALE_OFF], 4 * M);
    }
  }
  return fp;
}

bool overlaps(const Seg& a, const Seg& y) {
  const u128 yend0 = y.base + y.nbytes;  // end of output row 0
  for (u128 i = 0; i < a.count; ++i) {
    const u128 lo = a.base + i * a.ld, hi = lo + a.nbytes;
    // first output row whose end is after lo
    u128 r;
    if (lo < yend0) r = 0;
    else r = (lo - yend0) / y.ld + 1;
    if (r < y.count && y.base + r * y.ld < hi) return true;
  }
  return false;
}

bool in_place(const Desc& d, int i) {
  const int out = d.out();
  if (d.op() != OP_ELT || (out != OUT_FP32 && out != OUT_FP16)) return false;
  const Strides s = strides(d);
  if (i == 0) {
    const int afmt = (d[F_HDR_RSV] & STATE_FP16) ? OUT_FP16 : OUT_FP32;
    return afmt == out && !(d[F_HDR_RSV] >> 2 & 1) && d[F_A_OFF] == d[F_Y_OFF] && s.lda == s.ldy;
  }
  return i == 2 && d[F_BIAS_OFF] == d[F_Y_OFF];
}

}  // namespace tc
