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

#include "fp32.cuh"
#include "mma.h"
#include "ops.h"
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

// Aligns rows [m0, m0 + mb) from their fp32 bit patterns in sX [MB][K] into sQ [MB][64][kQStride]
// int16 (chunks of 8 in the order k = 8c + 0, 2, 4, 6, 1, 3, 5, 7), sS [MB][64] fp32 scale bits and
// sSum [MB][64] (the sum of each group's mantissas). A warp aligns 4 groups at once (4 elements of
// each per lane), so the shuffle reductions of the 4 groups overlap.
template <int MB>
__device__ void align_rows(const W4Args& g, int mb, const uint32_t* sX, int16_t* sQ, uint32_t* sS, int* sSum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = g.K / W4_GROUP;
  const int nwarps = blockDim.x >> 5;
  const int total = mb * G;
  for (int p0 = 4 * warp; p0 < total; p0 += 4 * nwarps) {
    uint32_t b[4][4];
    int e[4][4], emax[4];
    bool nan[4], inf[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int p = min(p0 + u, total - 1);
      const int m = p / G, gi = p - m * G;
      const uint4 v4 = *reinterpret_cast<const uint4*>(sX + m * g.K + gi * W4_GROUP + lane * 4);
      const uint32_t vv[4] = {v4.x, v4.y, v4.z, v4.w};
      nan[u] = false;
      inf[u] = false;
      emax[u] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t v = vv[j];
        if ((v & 0x7F800000u) == 0) v &= 0x80000000u;        // ftz
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
        const int m = p / G, gi = p - m * G;
        // element k = 4 lane + j: chunk c = lane / 2, k = 8c + 4h + j with h = lane & 1. A chunk is
        // 16 bytes: qh of k = 8c + 0, 2, 4, 6 | qh of k = 8c + 1, 3, 5, 7 | ql (even k) | ql (odd k),
        // q = 256 qh + ql with qh = q >> 8 in [-64, 64] and ql = q & 255; this lane's even / odd
        // elements are bytes 2h, 2h + 1 of those words.
        uint8_t* dst = reinterpret_cast<uint8_t*>(sQ + (m * 64 + gi) * kQStride) + 16 * (lane >> 1) + 2 * (lane & 1);
        auto hi = [](int q) { return (uint32_t)(uint8_t)(int8_t)(q >> 8); };
        auto lo = [](int q) { return (uint32_t)(q & 0xFF); };
        *reinterpret_cast<uint16_t*>(dst + 0) = (uint16_t)(hi(qv[0]) | hi(qv[2]) << 8);     // qh even
        *reinterpret_cast<uint16_t*>(dst + 4) = (uint16_t)(hi(qv[1]) | hi(qv[3]) << 8);     // qh odd
        *reinterpret_cast<uint16_t*>(dst + 8) = (uint16_t)(lo(qv[0]) | lo(qv[2]) << 8);     // ql even
        *reinterpret_cast<uint16_t*>(dst + 12) = (uint16_t)(lo(qv[1]) | lo(qv[3]) << 8);    // ql odd
        if (lane == 0) {
          uint32_t sb = (uint32_t)min(max(eff - 13, 0), 255) << 23;
          if (emax[u] == 0) sb = 0;
          if (ginf) sb = 0x7F800000u;
          if (gnan) sb = 0x7FC00000u;
          sS[m * 64 + gi] = sb;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) qs[u] += __shfl_xor_sync(0xFFFFFFFFu, qs[u], o);
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + u;
        if (p < total) sSum[(p / G) * 64 + (p % G)] = qs[u];
      }
    }
  }
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

cudaError_t launch_gemm_w4a16(const W4Args& g, cudaStream_t st) {
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
