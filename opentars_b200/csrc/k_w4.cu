// W4A16 GEMV (golden.py:295-324) for sm_100a.
//
// Prologue (per block, in shared memory): the block-FP alignment of numerics.py:55-98 for the
// block's activation rows: per (row, 128-group) the largest exponent, emax_eff = max(emax, 14),
// each significand shifted right by 10 + emax_eff - e with round-to-nearest-even, the sign
// applied; group scale bits (emax_eff - 13) << 23; the NaN / inf / all-zero group rules.
//
// Main loop: one warp per output column; lane L owns groups L, L + 32. A group's 64 packed
// bytes (128 int4) are four 16-byte loads. The nibbles become unsigned (u = nibble ^ 8 = w + 8,
// 0..15): the even and odd nibbles of a word are two byte masks. The aligned mantissas are split
// as q = 256 qh + ql (qh signed, ql unsigned bytes) and stored per 8 elements in the matching
// (even, odd) order, one 16-byte shared load per 8 weights, so four dp4a per 8 weights give
// sum(u qh) and sum(u ql); dot = 256 sum(u qh) + sum(u ql) - 8 sum(q), exact in int32, with
// sum(q) per activation group computed once. term_g = fmul(fmul(i2f(dot_g),
// ws[n,g]), xs[m,g]) runs in parallel across lanes; the four fp32 banks (g mod 4) then add their
// terms in increasing g on lanes 0..3 (unrolled: the shuffles issue ahead of the dependent adds),
// and y = (b0 + b1) + (b2 + b3), bias, activation and the output conversion follow.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "fp32.cuh"
#include "mma.h"
#include "ops.h"
#include "pdl.cuh"
#include "umma.cuh"

namespace tc {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// int16 slots per group in shared memory: 128 mantissas + 8 of padding, so consecutive groups
// start 272 bytes apart and the 8 lanes of a 16-byte load phase (one group each) cover 32
// different banks
constexpr int kQStride = 136;

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// The dp4a kernels' layout of a group's mantissas: one 256-byte block of 16 chunks (chunk c:
// k = 8c .. 8c + 7 as qh of k = 8c + 0, 2, 4, 6 | qh of k = 8c + 1, 3, 5, 7 | ql of the even k | ql
// of the odd k, q = 256 qh + ql with qh = q >> 8 in [-64, 64] and ql = q & 255). Element k = 4 lane
// + j lies in chunk c = lane / 2 at k = 8c + 4h + j with h = lane & 1: this lane's even / odd
// elements are bytes 2h, 2h + 1 of the chunk's four words.
__device__ __forceinline__ void put_dp4a_chunks(uint8_t* block, int lane, const int (&qv)[4]) {
  uint8_t* dst = block + 16 * (lane >> 1) + 2 * (lane & 1);
  auto hi = [](int q) { return (uint32_t)(uint8_t)(int8_t)(q >> 8); };
  auto lo = [](int q) { return (uint32_t)(q & 0xFF); };
  *reinterpret_cast<uint16_t*>(dst + 0) = (uint16_t)(hi(qv[0]) | hi(qv[2]) << 8);     // qh even
  *reinterpret_cast<uint16_t*>(dst + 4) = (uint16_t)(hi(qv[1]) | hi(qv[3]) << 8);     // qh odd
  *reinterpret_cast<uint16_t*>(dst + 8) = (uint16_t)(lo(qv[0]) | lo(qv[2]) << 8);     // ql even
  *reinterpret_cast<uint16_t*>(dst + 12) = (uint16_t)(lo(qv[1]) | lo(qv[3]) << 8);    // ql odd
}

// Block-FP alignment of four (row, group) pairs p0 .. p0 + 3 (pairs >= total are not written) by
// one warp, four elements of each group per lane (lane L: elements 4L .. 4L + 3). bits(p) gives
// the lane's four fp32 bit patterns of pair p. The sink receives, per pair, each lane's four
// aligned mantissas (sink.put(p, lane, q[4])), the group's scale bits (sink.scale(p, bits)) and
// the sum of its mantissas (sink.sum(p, s)). The four groups' shuffle reductions overlap.
template <class Bits, class Sink>
__device__ __forceinline__ void align_quad(int p0, int total, Bits bits, Sink& sink) {
  const int lane = threadIdx.x & 31;
  uint32_t b[4][4];
  int e[4][4], emax[4];
  bool nan[4], inf[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint4 v4 = bits(min(p0 + u, total - 1));
    const uint32_t vv[4] = {v4.x, v4.y, v4.z, v4.w};
    nan[u] = false;
    inf[u] = false;
    emax[u] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t v = vv[j];
      if ((v & 0x7F800000u) == 0) v &= 0x80000000u;          // ftz
      b[u][j] = v;
      e[u][j] = (int)((v >> 23) & 0xFF);
      nan[u] |= e[u][j] == 255 && (v & 0x7FFFFFu);
      inf[u] |= e[u][j] == 255 && !(v & 0x7FFFFFu);
      emax[u] = max(emax[u], e[u][j]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 4; ++u) emax[u] = max(emax[u], __shfl_xor_sync(0xFFFFFFFFu, emax[u], o));
  int qs[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const bool gnan = __any_sync(0xFFFFFFFFu, nan[u]);
    const bool ginf = __any_sync(0xFFFFFFFFu, inf[u]) && !gnan;
    const int eff = max(emax[u], 14);
    int qv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sh = 10 + eff - e[u][j];
      const uint32_t uu = (1u << 23) | (b[u][j] & 0x7FFFFFu);
      const int s = min(max(sh, 0), 31);
      const uint32_t kept = uu >> s;
      const uint32_t rem = uu & ((1u << s) - 1u);
      const uint32_t half = 1u << min(max(s - 1, 0), 30);
      const bool up = s > 0 && (rem > half || (rem == half && (kept & 1u)));
      int mag = (e[u][j] == 0 || sh >= 25 || e[u][j] == 255) ? 0 : (int)(kept + (up ? 1u : 0u));
      const bool isinf_j = e[u][j] == 255 && !(b[u][j] & 0x7FFFFFu);
      if (isinf_j && !gnan) mag = 16384;
      if (gnan) mag = 0;
      qv[j] = (b[u][j] >> 31) ? -mag : mag;
    }
    qs[u] = qv[0] + qv[1] + qv[2] + qv[3];
    const int p = p0 + u;
    if (p < total) {
      sink.put(p, lane, qv);
      if (lane == 0) {
        uint32_t sb = (uint32_t)min(max(eff - 13, 0), 255) << 23;
        if (emax[u] == 0) sb = 0;
        if (ginf) sb = 0x7F800000u;
        if (gnan) sb = 0x7FC00000u;
        sink.scale(p, sb);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < 4; ++u) qs[u] += __shfl_xor_sync(0xFFFFFFFFu, qs[u], o);
  if (lane == 0) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (p0 + u < total) sink.sum(p0 + u, qs[u]);
  }
}

// Aligns rows [m0, m0 + mb) from their fp32 bit patterns in sX [MB][K] into sQ [MB][64][kQStride]
// int16, sS [MB][64] fp32 scale bits and sSum [MB][64].
struct SmemSink {
  int16_t* sQ;
  uint32_t* sS;
  int* sSum;
  int G;
  __device__ void put(int p, int lane, const int (&qv)[4]) const {
    put_dp4a_chunks(reinterpret_cast<uint8_t*>(sQ + ((p / G) * 64 + p % G) * kQStride), lane, qv);
  }
  __device__ void scale(int p, uint32_t v) const { sS[(p / G) * 64 + p % G] = v; }
  __device__ void sum(int p, int v) const { sSum[(p / G) * 64 + p % G] = v; }
};
template <int MB>
__device__ void align_rows(const W4Args& g, int mb, const uint32_t* sX, int16_t* sQ, uint32_t* sS, int* sSum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = g.K / W4_GROUP;
  const int nwarps = blockDim.x >> 5;
  const int total = mb * G;
  SmemSink sink{sQ, sS, sSum, G};
  for (int p0 = 4 * warp; p0 < total; p0 += 4 * nwarps)
    align_quad(p0, total, [&](int p) {
      const int m = p / G, gi = p - m * G;
      return *reinterpret_cast<const uint4*>(sX + m * g.K + gi * W4_GROUP + lane * 4);
    }, sink);
}

// Mixed-sign 4-way byte dots (PTX dp4a with an unsigned first operand): d = c + sum a.b[i] * b.b[i].
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// The exact dot of one 128-group: 16 words of packed nibbles against 16 chunks (in word order)
// of the aligned mantissas split as q = 256 qh + ql; u = nibble ^ 8 = w + 8, so
// sum(w q) = 256 sum(u qh) + sum(u ql) - 8 sum(q). Four independent accumulator chains. The odd
// nibbles stay in the high half of each byte (16 u), so their sums are 16 times their value and
// are shifted back exactly (multiples of 16): two logic operations per packed word.
template <class WordOf, class ChunkOf>
__device__ __forceinline__ int group_dot(WordOf word, ChunkOf chunk, int qsum) {
  int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const uint32_t w = word(c) ^ 0x88888888u;                      // u = nibble ^ 8 in every nibble
    const uint32_t ev = w & 0x0F0F0F0Fu;                          // u of k = 8c + 0, 2, 4, 6
    const uint32_t od = w & 0xF0F0F0F0u;                          // 16 u of k = 8c + 1, 3, 5, 7
    const uint4 qc = chunk(c);
    h0 = dp4a_us(ev, qc.x, h0);
    h1 = dp4a_us(od, qc.y, h1);
    l0 = dp4a_uu(ev, qc.z, l0);
    l1 = dp4a_uu(od, qc.w, l1);
  }
  return 256 * (h0 + (h1 >> 4)) + (l0 + (l1 >> 4)) - 8 * qsum;
}

// term = fmul(fmul(i2f(dot), ws), xs) without the input flushes: i2f of an int, a widened fp16 and
// a block-FP scale (2^e, 0, inf or NaN) are never denormal; a NaN stays a NaN through the products
// and the bank's final canon makes it 0x7FC00000.
__device__ __forceinline__ float group_term(int dot, float ws, float xs) { return fmul_ff(fmul_ff(i2f(dot), ws), xs); }

// One persistent block stages its activation rows once (16-byte loads when aligned), aligns them
// in shared memory, then its warps stream columns n = gw, gw + nw, ...; each lane keeps the
// packed weights of its groups (lane, lane + 32) for this column and the next one in registers.
template <int MB>
__global__ void __launch_bounds__(kThreads) k_gemv_w4(W4Args g, bool vec) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* sX = reinterpret_cast<uint32_t*>(smem);                                 // [MB][K] fp32 bits
  int16_t* sQ = reinterpret_cast<int16_t*>(smem + (size_t)MB * g.K * 4);             // [MB][64][kQStride]
  uint32_t* sS = reinterpret_cast<uint32_t*>(smem + (size_t)MB * g.K * 4 + (size_t)MB * 64 * kQStride * 2);
  int* sSum = reinterpret_cast<int*>(sS + MB * 64);                                  // [MB][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int G = g.K / W4_GROUP;
  const int nw = gridDim.x * kWarps;
  int n = blockIdx.x * kWarps + warp;
  uint4 w[2][4], wn[2][4];
  uint16_t wsh[2], wsn[2];
  auto load_col = [&](int col, uint4 (*dst)[4], uint16_t (&h)[2]) {
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int gi = lane + 32 * slot;
      h[slot] = gi < G ? ld_u16(g.scale + 2 * ((uint64_t)col * G + gi)) : (uint16_t)0;
      const uint8_t* wp = g.W + (uint64_t)col * (g.K / 2) + gi * 64;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (gi >= G) dst[slot][i] = make_uint4(0, 0, 0, 0);
        else if (vec) dst[slot][i] = ldg_stream(wp + 16 * i);
        else dst[slot][i] = make_uint4(ld_u32(wp + 16 * i), ld_u32(wp + 16 * i + 4), ld_u32(wp + 16 * i + 8),
                                       ld_u32(wp + 16 * i + 12));
      }
    }
  };
  if (n < g.N) load_col(n, w, wsh);
  // the block's activation rows as fp32 bit patterns (bf16 widened exactly)
  for (int m = 0; m < mb; ++m) {
    const uint8_t* row = g.A + (uint64_t)(m0 + m) * g.lda;
    uint32_t* dst = sX + m * g.K;
    if (!g.a_bf16 && ((uintptr_t)row & 15) == 0) {
      for (int i = threadIdx.x; i < g.K / 4; i += kThreads) cp16(dst + 4 * i, row + 16 * (uint64_t)i);
      cp_wait_all();
    } else {
      for (int k = threadIdx.x; k < g.K; k += kThreads)
        dst[k] = g.a_bf16 ? ((uint32_t)ld_u16(row + 2 * (uint64_t)k) << 16) : ld_u32(row + 4 * (uint64_t)k);
    }
  }
  __syncthreads();
  align_rows<MB>(g, mb, sX, sQ, sS, sSum);
  __syncthreads();

  for (; n < g.N; n += nw) {
    const int nn = n + nw;
    if (nn < g.N) load_col(nn, wn, wsn);
    float term[MB][2];
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int gi = lane + 32 * slot;
#pragma unroll
      for (int m = 0; m < MB; ++m) term[m][slot] = 0.0f;
      if (gi < G) {
        const float ws = from_fp16(wsh[slot]);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m < mb) {
            const uint4* q = reinterpret_cast<const uint4*>(sQ + (m * 64 + gi) * kQStride);
            const int dot = group_dot(
                [&](int c) {
                  const uint4& v = w[slot][c >> 2];
                  return (c & 3) == 0 ? v.x : (c & 3) == 1 ? v.y : (c & 3) == 2 ? v.z : v.w;
                },
                [&](int c) { return q[c]; }, sSum[m * 64 + gi]);
            term[m][slot] = group_term(dot, ws, bf(sS[m * 64 + gi]));
          }
        }
      }
    }
    // banks: lane b (< 4) adds terms g = b, b + 4, ... in order (G <= 64: at most 16 terms)
    const int b = lane & 3;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      float t[16];                                                // group b + 4 i: lane (b + 4 i) mod 32
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = __shfl_sync(0xFFFFFFFFu, term[m][i < 8 ? 0 : 1], (b + 4 * i) & 31);
      float bank = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (b + 4 * i < G) bank = fadd_nc(bank, t[i]);
      bank = canon(bank);
      const float b1 = __shfl_sync(0xFFFFFFFFu, bank, 1);
      const float b2 = __shfl_sync(0xFFFFFFFFu, bank, 2);
      const float b3 = __shfl_sync(0xFFFFFFFFu, bank, 3);
      if (lane == 0 && m < mb) {
        float y = fadd(fadd(bank, b1), fadd(b2, b3));
        if (g.bias) y = fadd(y, ld_f32(g.bias + 4 * (uint64_t)n));
        y = act_fn(y, g.act);
        store_out(g.Y + (uint64_t)(m0 + m) * g.ldy, n, y, g.out, g.out_scale);
      }
    }
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
#pragma unroll
      for (int i = 0; i < 4; ++i) w[slot][i] = wn[slot][i];
      wsh[slot] = wsn[slot];
    }
  }
}

// The same GEMV with the weights streamed through shared memory: warp 0's lane 0 copies chunks of
// kW4Cols consecutive columns (kW4Cols * K/2 contiguous bytes) with 1-D bulk copies into a ring of
// stages (completing on mbarriers, full-line DRAM reads, up to kW4Stages chunks in flight per
// block); compute warp w (1..kW4Cols) takes column w - 1 of a chunk. Lane L reads the 64 bytes of its groups L
// and L + 32 from shared memory as four 16-byte pieces in the order (i + L/2) mod 4, which puts
// the 8 lanes of each load phase on 8 different 16-byte bank groups. Every wait is bounded; after
// a timeout the block stops streaming and skips its remaining columns.
constexpr int kW4Cols = 16, kW4Stages = 2, kW4Threads = 32 * (1 + kW4Cols);

template <int MB>
__global__ void __launch_bounds__(kW4Threads, 1) k_gemv_w4s(W4Args g) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kW4Stages], empty[kW4Stages];
  __shared__ int s_stop;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int G = g.K / W4_GROUP;
  const uint32_t colb = g.K / 2;                                  // bytes per column
  const uint32_t stage_b = kW4Cols * colb;
  uint8_t* ring = smem;                                           // [kW4Stages][kW4Cols columns]
  uint32_t* sX = reinterpret_cast<uint32_t*>(smem + kW4Stages * stage_b);               // [MB][K]
  int16_t* sQ = reinterpret_cast<int16_t*>(smem + kW4Stages * stage_b + (size_t)MB * g.K * 4);
  uint32_t* sS = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sQ) + (size_t)MB * 64 * kQStride * 2);
  int* sSum = reinterpret_cast<int*>(sS + MB * 64);
  const int nchunk = (g.N + kW4Cols - 1) / kW4Cols;
  auto chunk_bytes = [&](int c) { return (uint32_t)(min(kW4Cols, g.N - c * kW4Cols)) * colb; };
  // the activation rows first, then the first weight chunks
  for (int m = 0; m < mb; ++m) {
    const uint8_t* row = g.A + (uint64_t)(m0 + m) * g.lda;
    uint32_t* dst = sX + m * g.K;
    if (!g.a_bf16 && ((uintptr_t)row & 15) == 0) {
      for (int i = threadIdx.x; i < g.K / 4; i += blockDim.x) cp16(dst + 4 * i, row + 16 * (uint64_t)i);
    } else {
      for (int k = threadIdx.x; k < g.K; k += blockDim.x)
        dst[k] = g.a_bf16 ? ((uint32_t)ld_u16(row + 2 * (uint64_t)k) << 16) : ld_u32(row + 4 * (uint64_t)k);
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kW4Stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kW4Cols);
    }
    s_stop = 0;
    mbar_fence_init();
  }
  __syncthreads();
  int issued = 0;
  if (threadIdx.x == 0) {
    for (int c = blockIdx.x; c < nchunk && issued < kW4Stages; c += gridDim.x, ++issued) {
      mbar_expect_tx(&full[issued], chunk_bytes(c));
      bulk_load(ring + issued * stage_b, g.W + (uint64_t)c * stage_b, chunk_bytes(c), &full[issued]);
    }
  }
  cp_wait_all();
  __syncthreads();
  align_rows<MB>(g, mb, sX, sQ, sS, sSum);
  __syncthreads();

  // consumer warp cw + 1 computes column cw of every chunk
  auto compute = [&](const int cw) {
    // the fp16 group scales of this warp's next column are loaded one column ahead
    auto load_ws = [&](int col, uint16_t (&h)[2]) {
#pragma unroll
      for (int slot = 0; slot < 2; ++slot) {
        const int gi = lane + 32 * slot;
        h[slot] = (col < g.N && gi < G) ? ld_u16(g.scale + 2 * ((uint64_t)col * G + gi)) : (uint16_t)0;
      }
    };
    uint16_t wsh[2], wsn[2];
    load_ws(blockIdx.x * kW4Cols + cw, wsh);
    int t = 0;
    for (int c = blockIdx.x; c < nchunk; c += gridDim.x, ++t) {
      const int st = t % kW4Stages;
      load_ws((c + gridDim.x) * kW4Cols + cw, wsn);
      const bool ok = !*(volatile int*)&s_stop && mbar_wait(&full[st], (t / kW4Stages) & 1, g.err, 12, g.spin);
      if (!__all_sync(0xFFFFFFFFu, ok)) {                           // the whole warp stops together
        s_stop = 1;
        break;
      }
      const int n = c * kW4Cols + cw;
      if (n < g.N) {
        const uint8_t* colp = ring + st * stage_b + cw * colb;
        float term[MB][2];
#pragma unroll
        for (int slot = 0; slot < 2; ++slot) {
          const int gi = lane + 32 * slot;
#pragma unroll
          for (int m = 0; m < MB; ++m) term[m][slot] = 0.0f;
          if (gi < G) {
            const float ws = from_fp16(wsh[slot]);
            uint4 wv[4];
            int pc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              pc[i] = (i + (lane >> 1)) & 3;
              wv[i] = *reinterpret_cast<const uint4*>(colp + gi * 64 + 16 * pc[i]);
            }
#pragma unroll
            for (int m = 0; m < MB; ++m) {
              if (m < mb) {
                const uint4* q = reinterpret_cast<const uint4*>(sQ + (m * 64 + gi) * kQStride);
                const int dot = group_dot(
                    [&](int c) {
                      const uint4& v = wv[c >> 2];
                      return (c & 3) == 0 ? v.x : (c & 3) == 1 ? v.y : (c & 3) == 2 ? v.z : v.w;
                    },
                    [&](int c) { return q[pc[c >> 2] * 4 + (c & 3)]; }, sSum[m * 64 + gi]);
                term[m][slot] = group_term(dot, ws, bf(sS[m * 64 + gi]));
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);                     // the weights are in registers
        const int b = lane & 3;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          float tt[16];                                             // group b + 4 i: lane (b + 4 i) mod 32
#pragma unroll
          for (int i = 0; i < 16; ++i) tt[i] = __shfl_sync(0xFFFFFFFFu, term[m][i < 8 ? 0 : 1], (b + 4 * i) & 31);
          float bank = 0.0f;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (b + 4 * i < G) bank = fadd_nc(bank, tt[i]);
          bank = canon(bank);
          const float b1 = __shfl_sync(0xFFFFFFFFu, bank, 1);
          const float b2 = __shfl_sync(0xFFFFFFFFu, bank, 2);
          const float b3 = __shfl_sync(0xFFFFFFFFu, bank, 3);
          if (lane == 0 && m < mb) {
            float y = fadd(fadd(bank, b1), fadd(b2, b3));
            if (g.bias) y = fadd(y, ld_f32(g.bias + 4 * (uint64_t)n));
            y = act_fn(y, g.act);
            store_out(g.Y + (uint64_t)(m0 + m) * g.ldy, n, y, g.out, g.out_scale);
          }
        }
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      wsh[0] = wsn[0];
      wsh[1] = wsn[1];
    }
  };
  __shared__ int s_issued;
  if (warp == 0) {
    if (lane == 0) {
      // producer: chunk t of this block into stage t % kW4Stages once its 8 columns are done
      int t = issued;
      for (int c = blockIdx.x + issued * gridDim.x; c < nchunk; c += gridDim.x, ++t) {
        const int st = t % kW4Stages;
        if (!mbar_wait(&empty[st], ((t / kW4Stages) & 1) ^ 1, g.err, 11, g.spin)) {
          s_stop = 1;
          break;
        }
        mbar_expect_tx(&full[st], chunk_bytes(c));
        bulk_load(ring + st * stage_b, g.W + (uint64_t)c * stage_b, chunk_bytes(c), &full[st]);
      }
      s_issued = t;
    }
  } else {
    compute(warp - 1);
  }
  // After a wait gave up, copies of the last chunks issued may still be in flight: the block does
  // not exit before they land (these waits always have the full limit).
  __syncthreads();
  if (threadIdx.x == 0 && s_stop)
    for (int u = s_issued > kW4Stages ? s_issued - kW4Stages : 0; u < s_issued; ++u)
      mbar_wait(&full[u % kW4Stages], (u / kW4Stages) & 1, nullptr, 0);
}

// ---------------------------------------------------------------------------------------------
// The tiled W4A16 GEMV (M <= 4) for up to kW4GroupMax independent GEMVs of one row block and one K
// at once: a pre-pass aligns every GEMV's activation rows, then one persistent kernel streams the
// weights of all of them through TMA tiles.
//
// Pre-pass (k_w4_align): one warp per four (row, group) pairs of one GEMV writes, per row m, the
// aligned mantissas as [G][256 bytes] (put_s8_planes' lo / hi byte planes) followed by [G][scale
// bits, mantissa sum] into that GEMV's scratch. It lets the main kernel start at once
// (griddepcontrol.launch_dependents); the main kernel is launched with programmatic stream
// serialisation and copies from the scratch only after griddepcontrol.wait.
//
// Main kernel (k_gemv_w4t): a tile is 64 output columns of one GEMV x all of K; the tiles of the
// group's GEMVs are numbered one after another, each block takes a contiguous run of them, and its
// two quads split the run's stages in halves (W4Plan: the tile cut at the midpoint hands its
// partial bank sums from one quad to the other through shared memory). A quad is four compute
// warps, warp b adding the terms of the groups g = b (mod 4) - exactly the bank b of the
// reference's four-bank sum, in increasing g - so no term crosses a warp until the four banks are
// combined. A producer warp per quad fills
// the quad's ring with stages of four groups: two TMA boxes of 64 rows x 128 bytes of weights
// (128-byte swizzle: the lanes' 16-byte reads of one row chunk land on eight different bank
// groups) and, per activation row, the four groups' aligned mantissas (1 KB) and scale / sum
// words (32 bytes), bulk copies from the scratch. The weights of the first ring-full are requested
// before the pre-pass has finished; their activation copies follow griddepcontrol.wait.
//
// The exact group dots run on the warp MMA (mma.sync m16n8k32, u8 x s8 -> s32; the tcgen05 MMA
// wants its operands in shared memory in its own layout and its accumulator in TMEM, which a
// per-group scale would have to read back every 128 k). A operand: the nibbles made unsigned
// (u = nibble ^ 8 = w + 8), the even nibbles of a word as four bytes, the odd ones as 16 u in the
// high halves (a second accumulator, shifted back exactly). B operand: q = lo + 256 hi as two
// signed-byte planes in the same even / odd split, B column n = plane n & 1, so
// sum(w q) = C_lo + 256 C_hi - 8 sum(q), exact in int32. The MMA's k order is a permutation of the
// group's k applied alike to A and B (lane t: words 4 t .. 4 t + 3 of the row and of the planes),
// which leaves the integer sum unchanged. Per group a warp issues four MMAs per block of 16
// columns; MMA rows i and i + 8 are tile rows 16 cb + r(i) and + 8 with r = 0 4 1 5 2 6 3 7, so the
// eight lanes of each 16-byte read phase hit eight different bank groups of the swizzled rows. B
// columns 2..7 repeat the two planes, so every lane holds whole dots; lane (i, t) owns the columns
// of block t (rows r(i), r(i) + 8). The fp16 group scales of the next piece's tile are copied
// into shared memory (4-byte cp.async, one warp per column, columns padded to an odd number of
// words) while the current piece computes; the ring slot and its phase advance without integer
// divisions, and the barrier polls sleep (suspend-time hint). Every wait is bounded; after a give-up the warps skip their remaining
// work but keep the quad's barrier count, the producers stop issuing (the activation copies of
// stages whose weights were requested are still issued), and the block drains the copies in
// flight.
constexpr int kTQuads = 2, kTBanks = 4, kTCols = 64;
constexpr int kTThreads = 32 * (kTQuads + kTQuads * kTBanks);      // 2 producer warps + 8 compute warps
constexpr int kTStageB = 2 * kTCols * 128;                            // four groups of 64 columns
constexpr int kTActRow = 4 * 256 + 4 * 8;                             // a stage's mantissas + words, one row
constexpr int kTMaxStages = 16;

// Scratch bytes of one activation row: [G][256] mantissas, then [G][scale bits, sum].
__host__ __device__ constexpr uint32_t w4_scratch_row(int G) { return (uint32_t)G * (256 + 8); }

// A group's mantissas for the tensor-core dot: q = lo + 256 hi with lo in [-128, 127] and hi in
// [-64, 64] (|q| <= 16384), both signed bytes. Word w of the group (k = 8 w .. 8 w + 7) is split
// like the weights' nibbles: the bytes of its even k (8 w + 0, 2, 4, 6) lie at 64 p + 4 w of the
// 256-byte block (p = 0 for lo, 1 for hi), those of its odd k 128 bytes further on - so MMA lane t
// reads its four words' even (odd) parts of plane p as one 16-byte load at 64 p + 16 t (+ 128),
// and the eight lanes of a load phase read 128 contiguous bytes.
__device__ __forceinline__ void put_s8_planes(uint8_t* block, int lane, const int (&qv)[4]) {
  const int w = lane >> 1, h = lane & 1;                  // elements k = 8 w + 4 h + j, j = 0..3
  uint8_t* at = block + 4 * w + 2 * h;
  auto lo = [](int q) { return (uint32_t)(q & 0xFF); };
  auto hi = [](int q) { return (uint32_t)(((q + 128) >> 8) & 0xFF); };
  *reinterpret_cast<uint16_t*>(at) = (uint16_t)(lo(qv[0]) | lo(qv[2]) << 8);           // lo, even k
  *reinterpret_cast<uint16_t*>(at + 128) = (uint16_t)(lo(qv[1]) | lo(qv[3]) << 8);     // lo, odd k
  *reinterpret_cast<uint16_t*>(at + 64) = (uint16_t)(hi(qv[0]) | hi(qv[2]) << 8);      // hi, even k
  *reinterpret_cast<uint16_t*>(at + 192) = (uint16_t)(hi(qv[1]) | hi(qv[3]) << 8);     // hi, odd k
}

// D += A B for one m16n8k32 tile (A 16 x 32 unsigned bytes row-major, B 32 x 8 signed bytes
// column-major, s32 D).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A B (zero accumulator) for one m16n8k32 tile.
__device__ __forceinline__ void mma_u8s8_first(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// u = nibble ^ 8 of the even nibbles of w as bytes, and 16 u of the odd ones in the high halves:
// one three-input logic operation each ((w ^ 0x88888888) & mask).
__device__ __forceinline__ uint32_t nib_even(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x28;" : "=r"(d) : "r"(w), "n"(0x88888888u), "n"(0x0F0F0F0Fu));
  return d;
}
__device__ __forceinline__ uint32_t nib_odd(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x28;" : "=r"(d) : "r"(w), "n"(0x88888888u), "n"(0xF0F0F0F0u));
  return d;
}

// The waits of the tiled W4A16 kernel sleep in the poll (up to about this many nanoseconds).
constexpr uint32_t kW4WaitNs = 1000;

struct AlignSink {
  uint8_t* base;
  int G;
  __device__ uint8_t* row(int p) const { return base + (uint64_t)(p / G) * w4_scratch_row(G); }
  __device__ void put(int p, int lane, const int (&qv)[4]) const {
    put_s8_planes(row(p) + (uint64_t)(p % G) * 256, lane, qv);
  }
  __device__ void scale(int p, uint32_t v) const {
    reinterpret_cast<uint32_t*>(row(p) + (uint64_t)G * 256)[2 * (p % G)] = v;
  }
  __device__ void sum(int p, int v) const { reinterpret_cast<int*>(row(p) + (uint64_t)G * 256)[2 * (p % G) + 1] = v; }
};

// The GEMVs of one tiled launch (one row block, one K) and their tiles: GEMV j owns tiles
// tile0[j] .. tile0[j + 1] - 1.
struct W4Group {
  W4Args e[kW4GroupMax];
  int tile0[kW4GroupMax + 1];
  int n;
};
struct W4Maps {
  CUtensorMap m[kW4GroupMax];
};

// blockIdx.y: the GEMV; eight warps per block, four (row, group) pairs per warp.
__global__ void __launch_bounds__(256) k_w4_align(const __grid_constant__ W4Group grp) {
  griddep_launch();
  const W4Args& g = grp.e[blockIdx.y];
  const int G = g.K / W4_GROUP, total = g.M * G;
  const int lane = threadIdx.x & 31;
  const int p0 = 4 * (blockIdx.x * 8 + (threadIdx.x >> 5));
  if (p0 >= total) return;
  AlignSink sink{g.scratch, G};
  align_quad(p0, total, [&](int p) {
    const int m = p / G, gi = p - m * G;
    const uint8_t* row = g.A + (uint64_t)m * g.lda;
    const uint64_t k = (uint64_t)gi * W4_GROUP + 4 * lane;
    if (g.a_bf16)
      return make_uint4((uint32_t)ld_u16(row + 2 * k) << 16, (uint32_t)ld_u16(row + 2 * k + 2) << 16,
                        (uint32_t)ld_u16(row + 2 * k + 4) << 16, (uint32_t)ld_u16(row + 2 * k + 6) << 16);
    if (((uintptr_t)(row + 4 * k) & 15) == 0) return *reinterpret_cast<const uint4*>(row + 4 * k);
    return make_uint4(ld_u32(row + 4 * k), ld_u32(row + 4 * k + 4), ld_u32(row + 4 * k + 8), ld_u32(row + 4 * k + 12));
  }, sink);
}

// Row stride (bytes) of one column's group scales in shared memory: at least 2 G, a multiple of 4
// with an odd number of words, so the 32 lanes' 2-byte reads of one group hit 32 different banks.
__host__ __device__ constexpr uint32_t w4t_scale_stride(int G) { return (uint32_t)((G + 1) / 2) % 2 ? 2 * G : 2 * G + 4; }

// The work of one quad of a block, in order. Block b takes the contiguous tiles
// [ntiles * b / nblk, ntiles * (b + 1) / nblk) and its two quads half of their stages each: quad 0
// the first stages of the tile cut at the midpoint (kind 1: its bank sums are handed to quad 1)
// and then the whole tiles before it (kind 0); quad 1 the whole tiles after it and then the cut
// tile's remaining stages (kind 2: starting from the handed-over sums, so every bank still adds
// its groups in increasing g).
struct W4Piece {
  int t, s0, s1, kind;
};
struct W4Plan {
  int t_lo, t_hi, ts, r, nstage;
  __device__ W4Plan(int ntiles, int nstage_, int blk, int nblk) : nstage(nstage_) {
    t_lo = (int)((int64_t)ntiles * blk / nblk);
    t_hi = (int)((int64_t)ntiles * (blk + 1) / nblk);
    const int half = (t_hi - t_lo) * nstage / 2;
    ts = t_lo + half / nstage;
    r = half % nstage;
  }
  __device__ int count(int q) const { return q == 0 ? (r > 0) + (ts - t_lo) : t_hi - ts; }
  __device__ W4Piece piece(int q, int p) const {
    if (q == 0) {
      if (r > 0) {
        if (p == 0) return {ts, 0, r, 1};
        --p;
      }
      return {t_lo + p, 0, nstage, 0};
    }
    const int f0 = ts + (r > 0);
    if (p < t_hi - f0) return {f0 + p, 0, nstage, 0};
    return {ts, r, nstage, 2};
  }
};

template <int MB>
__global__ void __launch_bounds__(kTThreads, 1) k_gemv_w4t(const __grid_constant__ W4Group grp,
                                                            const __grid_constant__ W4Maps maps, int stages) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kTQuads][kTMaxStages], empty[kTQuads][kTMaxStages];
  __shared__ float sbank[2][kTQuads][kTBanks][MB][kTCols];
  __shared__ float xbank[kTBanks][MB][kTCols];                      // the cut tile's bank sums
  __shared__ uint64_t xbar;
  __shared__ int s_stop, s_issued[kTQuads];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = grp.e[0].K / W4_GROUP, nstage = (G + 3) / 4;
  const int ntiles = grp.tile0[grp.n];
  const uint32_t row_b = w4_scratch_row(G), sstr = w4t_scale_stride(G);
  int* const err = grp.e[0].err;
  const uint32_t spin = grp.e[0].spin;
  uint8_t* ring = smem;                                             // [quad][stage][2 boxes][64][128]
  uint8_t* aring = ring + (size_t)kTQuads * stages * kTStageB;     // [quad][stage][MB][kTActRow]
  uint8_t* sscl = aring + (size_t)kTQuads * stages * MB * kTActRow; // [quad][2][64 columns][sstr]
  if (threadIdx.x == 0) {
    for (int q = 0; q < kTQuads; ++q)
      for (int i = 0; i < stages; ++i) {
        mbar_init(&full[q][i], 1);
        mbar_init(&empty[q][i], kTBanks);
      }
    mbar_init(&xbar, kTBanks);
    s_stop = 0;
    mbar_fence_init();
  }
  __syncthreads();
  // the GEMV of global tile t
  auto entry_of = [&](int t) {
    int j = 0;
    while (j + 1 < grp.n && t >= grp.tile0[j + 1]) ++j;
    return j;
  };
  const W4Plan plan(ntiles, nstage, blockIdx.x, gridDim.x);
  if (warp < kTQuads) {
    if (lane == 0) {
      const int q = warp, np = plan.count(q);
      // the activation rows of stage s of GEMV j into ring slot st (after griddepcontrol.wait)
      auto issue_acts = [&](int j, int s, int st) {
        const W4Args& e = grp.e[j];
        const bool two = 4 * s + 2 < G;
        uint8_t* dst = aring + ((size_t)q * stages + st) * MB * kTActRow;
        for (int m = 0; m < min(e.M, MB); ++m) {
          const uint8_t* src = e.scratch + (uint64_t)m * row_b;
          bulk_load(dst + m * kTActRow, src + (uint64_t)s * 1024, two ? 1024 : 512, &full[q][st]);
          bulk_load(dst + m * kTActRow + 1024, src + (uint64_t)G * 256 + (uint64_t)s * 32, two ? 32 : 16, &full[q][st]);
        }
      };
      // the first ring-full went out without its activations: wait for the pre-pass, then send them
      auto catch_up = [&](int upto) {
        griddep_wait();
        int k = 0;
        for (int p = 0; p < np && k < upto; ++p) {
          const W4Piece pc = plan.piece(q, p);
          const int j = entry_of(pc.t);
          for (int s = pc.s0; s < pc.s1 && k < upto; ++s, ++k) issue_acts(j, s, k);
        }
      };
      int it = 0, st = 0, ph = 0;                  // stages issued; ring slot and its phase
      bool waited = false;
      for (int p = 0; p < np; ++p) {
        const W4Piece pc = plan.piece(q, p);
        const int t = pc.t, j = entry_of(t), lt = t - grp.tile0[j];
        const int mrows = min(grp.e[j].M, MB);
        for (int s = pc.s0; s < pc.s1; ++s, ++it, st = st + 1 < stages ? st + 1 : (ph ^= 1, 0)) {
          if (!waited && it == stages) {
            catch_up(stages);
            waited = true;
          }
          if (*(volatile int*)&s_stop ||
              !mbar_wait_hint(&empty[q][st], ph ^ 1, err, 13, spin, kW4WaitNs)) {
            s_stop = 1;
            goto producer_done;
          }
          const bool two = 4 * s + 2 < G;
          mbar_expect_tx(&full[q][st], (two ? kTStageB : kTStageB / 2) + mrows * (two ? 1024 + 32 : 512 + 16));
          uint8_t* dst = ring + ((size_t)q * stages + st) * kTStageB;
          tma_load_2d(dst, &maps.m[j], 256 * s, kTCols * lt, &full[q][st]);
          if (two) tma_load_2d(dst + kTStageB / 2, &maps.m[j], 256 * s + 128, kTCols * lt, &full[q][st]);
          if (waited) issue_acts(j, s, st);
        }
      }
    producer_done:
      if (!waited) catch_up(min(it, stages));     // every stage requested gets its activations
      s_issued[warp] = it;
    }
  } else {
    const int cw = warp - kTQuads, q = cw / kTBanks, b = cw % kTBanks;
    // MMA lane roles: row i = lane / 4 (tile row ri = 0 4 1 5 2 6 3 7 of it), tg = lane % 4; the
    // lane's result columns cA = 16 tg + ri and cA + 8
    const int mr = lane >> 2, tg = lane & 3;
    const int ri = (mr >> 1) | ((mr & 1) << 2), cA = 16 * tg + ri;
    const uint32_t woff = 16u * ((4 * (b & 1) + tg) ^ ri);
    // the group scales of tile t into buffer `buf` of this quad (4-byte copies): warp b copies
    // columns b, b + 4, ..., its lanes consecutive words of one column
    auto fetch_scales = [&](int t, int buf) {
      const int j = entry_of(t);
      const W4Args& e = grp.e[j];
      const int lt = t - grp.tile0[j], nc = min(kTCols, e.N - lt * kTCols);
      uint8_t* dst = sscl + ((size_t)q * 2 + buf) * kTCols * sstr;
      for (int c = b; c < nc; c += kTBanks) {
        const uint8_t* src = e.scale + 2 * ((uint64_t)(lt * kTCols + c) * G);
        for (int jw = lane; jw < G / 2; jw += 32)
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst + c * sstr + 4 * jw)),
                       "l"(src + 4 * jw)
                       : "memory");
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int np = plan.count(q);
    if (np > 0) fetch_scales(plan.piece(q, 0).t, 0);
    // the first piece's scales, copied by all four warps, before any warp reads them (later
    // pieces' scales are waited for at the end of the piece before)
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("bar.sync %0, %1;" ::"r"(2 + q), "n"(32 * kTBanks) : "memory");
    int st = 0, ph = 0;                              // ring slot and its phase
    for (int tl = 0; tl < np; ++tl) {
      const W4Piece pc = plan.piece(q, tl);
      const int t = pc.t, j = entry_of(t), lt = t - grp.tile0[j];
      const W4Args& e = grp.e[j];
      const int eM = e.M;                              // (kept in a register across the stage loop)
      if (tl + 1 < np) fetch_scales(plan.piece(q, tl + 1).t, (tl + 1) & 1);
      const uint8_t* scl = sscl + ((size_t)q * 2 + (tl & 1)) * kTCols * sstr;
      float bank[2][MB];
      bool from_x = false;
      if (pc.kind == 2) {                            // continue the bank sums quad 0 handed over
        from_x = !*(volatile int*)&s_stop && mbar_wait_hint(&xbar, 0, err, 15, spin, kW4WaitNs);
        from_x = __all_sync(0xFFFFFFFFu, from_x);
        if (!from_x) s_stop = 1;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < MB; ++m) bank[h][m] = from_x ? xbank[b][m][cA + 8 * h] : 0.0f;
      for (int s = pc.s0; s < pc.s1; ++s, st = st + 1 < stages ? st + 1 : (ph ^= 1, 0)) {
        const int gi = 4 * s + b;
        bool ok = !*(volatile int*)&s_stop && mbar_wait_hint(&full[q][st], ph, err, 14, spin, kW4WaitNs);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) {
          s_stop = 1;
          continue;                                  // skip the work, keep the barrier count
        }
        if (gi < G) {
          uint4 wa[4], wb[4];                                       // MMA rows i, i + 8 of each block
          // group gi = 4 s + b: box b / 2, 16-byte piece 4 (b & 1) + tg of rows 16 cb + ri (+ 8), swizzled
          const uint8_t* box = ring + ((size_t)q * stages + st) * kTStageB + (b >> 1) * (kTStageB / 2) + woff;
#pragma unroll
          for (int cb = 0; cb < 4; ++cb) {
            wa[cb] = *reinterpret_cast<const uint4*>(box + (16 * cb + ri) * 128);
            wb[cb] = *reinterpret_cast<const uint4*>(box + (16 * cb + ri + 8) * 128);
          }
          float ws[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) ws[h] = from_fp16(*reinterpret_cast<const uint16_t*>(scl + (cA + 8 * h) * sstr + 2 * gi));
          const uint8_t* arow0 = aring + ((size_t)q * stages + st) * MB * kTActRow;
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            if (m < eM) {
              const uint8_t* arow = arow0 + m * kTActRow;
              // B column n = plane n & 1 (lo, hi; columns 2..7 repeat 0, 1): the even-k bytes (de)
              // and odd-k bytes (dd) of lane tg's words 4 tg .. 4 tg + 3
              const uint8_t* pl = arow + b * 256 + 64 * (mr & 1) + 16 * tg;
              const uint4 de = *reinterpret_cast<const uint4*>(pl), dd = *reinterpret_cast<const uint4*>(pl + 128);
              int pa[4], pb[4];
#pragma unroll
              for (int cb = 0; cb < 4; ++cb) {
                // u = nibble ^ 8 = w + 8: even nibbles as bytes, odd nibbles as 16 u in the high halves
                const uint4 va = wa[cb], vb = wb[cb];
                int ce[4], co[4];
                mma_u8s8_first(ce, nib_even(va.x), nib_even(vb.x), nib_even(va.y), nib_even(vb.y), de.x, de.y);
                mma_u8s8(ce, nib_even(va.z), nib_even(vb.z), nib_even(va.w), nib_even(vb.w), de.z, de.w);
                mma_u8s8_first(co, nib_odd(va.x), nib_odd(vb.x), nib_odd(va.y), nib_odd(vb.y), dd.x, dd.y);
                mma_u8s8(co, nib_odd(va.z), nib_odd(vb.z), nib_odd(va.w), nib_odd(vb.w), dd.z, dd.w);
                // sum(u q) of rows i, i + 8: columns 2 tg (lo) and 2 tg + 1 (hi); the odd sums are
                // multiples of 16, shifted back exactly
                pa[cb] = ce[0] + (co[0] >> 4) + 256 * (ce[1] + (co[1] >> 4));
                pb[cb] = ce[2] + (co[2] >> 4) + 256 * (ce[3] + (co[3] >> 4));
              }
              const uint2 wd = *reinterpret_cast<const uint2*>(arow + 1024 + 8 * b);   // scale bits, sum
              const float xs = bf(wd.x);
              // dot = sum(w q) = sum(u q) - 8 sum(q), for the block this lane owns (cb = tg)
              const int qs8 = 8 * (int)wd.y;
              const int dota = (tg == 0 ? pa[0] : tg == 1 ? pa[1] : tg == 2 ? pa[2] : pa[3]) - qs8;
              const int dotb = (tg == 0 ? pb[0] : tg == 1 ? pb[1] : tg == 2 ? pb[2] : pb[3]) - qs8;
              bank[0][m] = fadd_nc(bank[0][m], group_term(dota, ws[0], xs));
              bank[1][m] = fadd_nc(bank[1][m], group_term(dotb, ws[1], xs));
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q][st]);   // the stage's weights and rows are read
      }
      if (pc.kind == 1) {                            // hand the bank sums (as they are) to quad 1
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int m = 0; m < MB; ++m) xbank[b][m][cA + 8 * h] = bank[h][m];
        __syncwarp();
        if (lane == 0) mbar_arrive(&xbar);
        asm volatile("cp.async.wait_group 0;" ::: "memory");   // the next piece's scales have landed
        asm volatile("bar.sync %0, %1;" ::"r"(2 + q), "n"(32 * kTBanks) : "memory");
        continue;
      }
      // the four banks of the tile's columns: (b0 + b1) + (b2 + b3)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < MB; ++m) sbank[tl & 1][q][b][m][cA + 8 * h] = canon(bank[h][m]);
      asm volatile("cp.async.wait_group 0;" ::: "memory");     // the next tile's scales have landed
      asm volatile("bar.sync %0, %1;" ::"r"(2 + q), "n"(32 * kTBanks) : "memory");
      if (b < 2 && !*(volatile int*)&s_stop) {                // warps 0 / 1: columns lane / lane + 32
        const int c = lane + 32 * b, n = lt * kTCols + c;
        if (n < e.N) {
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            if (m < e.M) {
              const float(&bk)[kTBanks][MB][kTCols] = sbank[tl & 1][q];
              float y = fadd(fadd(bk[0][m][c], bk[1][m][c]), fadd(bk[2][m][c], bk[3][m][c]));
              if (e.bias) y = fadd(y, ld_f32(e.bias + 4 * (uint64_t)n));
              y = act_fn(y, e.act);
              store_out(e.Y + (uint64_t)m * e.ldy, n, y, e.out, e.out_scale);
            }
          }
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  }
  // after a give-up, the copies of the last stages issued may still be in flight: they land
  // before the block exits (these waits always have the full limit)
  __syncthreads();
  if (threadIdx.x < kTQuads && s_stop) {
    const int q = threadIdx.x, n_is = s_issued[q];
    for (int u = n_is > stages ? n_is - stages : 0; u < n_is; ++u)
      mbar_wait(&full[q][u % stages], (u / stages) & 1, nullptr, 0);
  }
}

// Dynamic shared memory the tiled kernel may use beside its static arrays (the banks of two tiles
// per quad and of the cut tile, the barriers).
size_t w4t_smem_cap(int MB) { return 227 * 1024 - (size_t)5120 * MB - 1024; }

// Shared memory of the tiled kernel for MB rows: the weight and activation rings, the scales of
// two tiles per quad, alignment slack.
size_t w4t_smem(int MB, int G, int stages) {
  return (size_t)kTQuads * stages * (kTStageB + (size_t)MB * kTActRow) + (size_t)kTQuads * 2 * kTCols * w4t_scale_stride(G) +
         1024;
}

template <int MB>
cudaError_t launch_w4t(const W4Args* gs, int n, cudaStream_t st) {
  W4Group grp{};
  W4Maps maps{};
  grp.n = n;
  grp.tile0[0] = 0;
  for (int j = 0; j < n; ++j) {
    grp.e[j] = gs[j];
    grp.e[j].err = wait_error_flag();
    grp.e[j].spin = spin_limit();
    grp.tile0[j + 1] = grp.tile0[j] + (gs[j].N + kTCols - 1) / kTCols;
    if (!make_map_u8(&maps.m[j], gs[j].W, gs[j].K / 2, gs[j].N, gs[j].K / 2, 128, kTCols)) return cudaErrorInvalidValue;
  }
  const int G = gs[0].K / W4_GROUP;
  int stages = kTMaxStages;
  while (stages > 2 && w4t_smem(MB, G, stages) > w4t_smem_cap(MB)) --stages;
  const size_t smem = w4t_smem(MB, G, stages);
  int pre = 1;
  for (int j = 0; j < n; ++j) pre = std::max(pre, (gs[j].M * G + 31) / 32);
  k_w4_align<<<dim3(pre, n), 256, 0, st>>>(grp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  auto kern = k_gemv_w4t<MB>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(std::min(grp.tile0[n], 148));
  cfg.blockDim = dim3(kTThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, grp, maps, stages);
}

template <int MB>
cudaError_t launch_w4s(const W4Args& g0, cudaStream_t st) {
  W4Args g = g0;
  g.err = wait_error_flag();
  g.spin = spin_limit();
  const size_t smem = (size_t)kW4Stages * kW4Cols * (g.K / 2) + (size_t)MB * g.K * 4 +
                      (size_t)MB * 64 * kQStride * 2 + (size_t)MB * 64 * 8;
  auto kern = k_gemv_w4s<MB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int nchunk = (g.N + kW4Cols - 1) / kW4Cols;
  kern<<<dim3(std::min(nchunk, 148), (g.M + MB - 1) / MB), kW4Threads, smem, st>>>(g);
  return cudaGetLastError();
}

template <int MB>
cudaError_t launch_w4(const W4Args& g, cudaStream_t st) {
  const size_t smem = (size_t)MB * g.K * 4 + (size_t)MB * 64 * kQStride * 2 + (size_t)MB * 64 * 8;
  auto kern = k_gemv_w4<MB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int nblk = std::min((g.N + kWarps - 1) / kWarps, 148 * 2);
  dim3 grid(nblk, (g.M + MB - 1) / MB);
  kern<<<grid, kThreads, smem, st>>>(g, (uintptr_t)g.W % 16 == 0);
  return cudaGetLastError();
}
}  // namespace

// TARSCUDA_W4_PATH=legacy keeps the streamed dp4a kernel that aligns in every block (for
// comparisons); the default is the tiled kernel with the alignment pre-pass.
int w4_path() {
  static const int v = [] {
    const char* e = getenv("TARSCUDA_W4_PATH");
    return e && !strcmp(e, "legacy") ? 0 : 1;
  }();
  return v;
}

bool w4_tiled_ok(const W4Args& g) {
  const int G = g.K / W4_GROUP;
  const int mb = g.M <= 1 ? 1 : (g.M <= 2 ? 2 : 4);
  return g.scratch && g.M >= 1 && g.M <= 4 && g.K % 256 == 0 && (uintptr_t)g.W % 16 == 0 &&
         ((uintptr_t)g.scratch & 15) == 0 && w4t_smem(mb, G, 3) <= w4t_smem_cap(mb) && w4_path() >= 1;
}

uint64_t w4_scratch_bytes(int M, int K) { return (uint64_t)M * w4_scratch_row(K / W4_GROUP); }

int w4_group_class(const W4Args& g) {
  if (!w4_tiled_ok(g)) return -1;
  const int mb = g.M <= 1 ? 1 : (g.M <= 2 ? 2 : 4);
  return mb << 16 | g.K / 256;
}

cudaError_t launch_w4_group(const W4Args* gs, int n, cudaStream_t st) {
  if (n < 1 || n > kW4GroupMax) return cudaErrorInvalidValue;
  const int cls = w4_group_class(gs[0]);
  for (int j = 0; j < n; ++j)
    if (cls < 0 || w4_group_class(gs[j]) != cls) return cudaErrorInvalidValue;
  if (cls >> 16 == 1) return launch_w4t<1>(gs, n, st);
  if (cls >> 16 == 2) return launch_w4t<2>(gs, n, st);
  return launch_w4t<4>(gs, n, st);
}

cudaError_t launch_gemm_w4a16(const W4Args& g, cudaStream_t st) {
  if (w4_tiled_ok(g)) return launch_w4_group(&g, 1, st);
  // streamed through shared memory when the packed weights are 16-byte aligned (K % 256 == 0
  // makes every column a multiple of 128 bytes) and the ring fits next to the activations
  const size_t ring = (size_t)kW4Stages * kW4Cols * (g.K / 2);
  const int mbk = g.M <= 1 ? 1 : (g.M <= 2 ? 2 : 4);
  if ((uintptr_t)g.W % 16 == 0 && g.M <= 4 &&
      ring + (size_t)mbk * g.K * 4 + (size_t)mbk * 64 * (kQStride * 2 + 8) <= 200 * 1024) {
    if (g.M == 1) return launch_w4s<1>(g, st);
    if (g.M == 2) return launch_w4s<2>(g, st);
    return launch_w4s<4>(g, st);
  }
  if (g.M == 1) return launch_w4<1>(g, st);
  if (g.M == 2) return launch_w4<2>(g, st);
  return launch_w4<4>(g, st);
}

}  // namespace tc
