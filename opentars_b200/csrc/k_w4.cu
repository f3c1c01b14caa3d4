// W4A16 GEMV (golden.py:295-324) for sm_100a.
//
// Prologue (per block, in shared memory): the block-FP alignment of numerics.py:55-98 for the
// block's activation rows: per (row, 128-group) the largest exponent, emax_eff = max(emax, 14),
// each significand shifted right by 10 + emax_eff - e with round-to-nearest-even, the sign
// applied; group scale bits (emax_eff - 13) << 23; the NaN / inf / all-zero group rules.
//
// Main loop: one warp per output column; lane L owns groups L, L + 32. A group's 64 packed
// bytes (128 int4) are four 16-byte loads; the nibbles are sign-extended to int8 in registers
// (__vsub4 on x ^ 0x08) and dotted with the int16 mantissas by dp2a, exactly in int32
// (|dot| <= 128 * 16384 * 8 = 2^24). term_g = fmul(fmul(i2f(dot_g), ws[n,g]), xs[m,g]) runs in
// parallel across lanes; the four fp32 banks (g mod 4) then add their terms in increasing g on
// lanes 0..3, and y = (b0 + b1) + (b2 + b3), bias, activation and the output conversion follow.
#include <cuda_runtime.h>

#include <algorithm>

#include "fp32.cuh"
#include "ops.h"

namespace tc {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// int16 slots per group in shared memory: 128 mantissas + 2 of padding, so a group starts 65 words
// after the previous one and the 32 lanes (one group each) read 32 different banks
constexpr int kQStride = 130;

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Aligns rows [m0, m0 + mb) from their fp32 bit patterns in sX [MB][K] into sQ [MB][K] int16 and
// sS [MB][64] fp32 bits; one warp per (row, group), four elements per lane.
template <int MB>
__device__ void align_rows(const W4Args& g, int mb, const uint32_t* sX, int16_t* sQ, uint32_t* sS) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = g.K / W4_GROUP;
  for (int p = warp; p < mb * G; p += kWarps) {
    const int m = p / G, gi = p - m * G;
    uint32_t b[4];
    int e[4];
    bool nan = false, inf = false;
    int emax = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t v = sX[m * g.K + gi * W4_GROUP + lane * 4 + j];
      if ((v & 0x7F800000u) == 0) v &= 0x80000000u;        // ftz
      b[j] = v;
      e[j] = (int)((v >> 23) & 0xFF);
      nan |= e[j] == 255 && (v & 0x7FFFFFu);
      inf |= e[j] == 255 && !(v & 0x7FFFFFu);
      emax = max(emax, e[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) emax = max(emax, __shfl_xor_sync(0xFFFFFFFFu, emax, o));
    const bool gnan = __any_sync(0xFFFFFFFFu, nan);
    const bool ginf = __any_sync(0xFFFFFFFFu, inf) && !gnan;
    const int eff = max(emax, 14);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sh = 10 + eff - e[j];
      const uint32_t u = (1u << 23) | (b[j] & 0x7FFFFFu);
      const int s = min(max(sh, 0), 31);
      const uint32_t kept = u >> s;
      const uint32_t rem = u & ((1u << s) - 1u);
      const uint32_t half = 1u << min(max(s - 1, 0), 30);
      const bool up = s > 0 && (rem > half || (rem == half && (kept & 1u)));
      int mag = (e[j] == 0 || sh >= 25 || e[j] == 255) ? 0 : (int)(kept + (up ? 1u : 0u));
      const bool isinf_j = e[j] == 255 && !(b[j] & 0x7FFFFFu);
      if (isinf_j && !gnan) mag = 16384;
      if (gnan) mag = 0;
      sQ[(m * 64 + gi) * kQStride + lane * 4 + j] = (int16_t)((b[j] >> 31) ? -mag : mag);
    }
    if (lane == 0) {
      uint32_t sb = (uint32_t)min(max(eff - 13, 0), 255) << 23;
      if (emax == 0) sb = 0;
      if (ginf) sb = 0x7F800000u;
      if (gnan) sb = 0x7FC00000u;
      sS[m * 64 + gi] = sb;
    }
  }
}

// int4 nibbles of one 32-bit word (8 elements) -> two words of 4 sign-extended int8 in k order
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t ev = __vsub4((w & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);         // k = 0,2,4,6
  const uint32_t od = __vsub4(((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);  // k = 1,3,5,7
  lo = __byte_perm(ev, od, 0x5140);
  hi = __byte_perm(ev, od, 0x7362);
}

// One persistent block stages its activation rows once (16-byte loads when aligned), aligns them
// in shared memory, then its warps stream columns n = gw, gw + nw, ...; each lane keeps the
// packed weights of its groups (lane, lane + 32) for this column and the next one in registers.
template <int MB>
__global__ void __launch_bounds__(kThreads) k_gemv_w4(W4Args g, bool vec) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* sX = reinterpret_cast<uint32_t*>(smem);                                 // [MB][K] fp32 bits
  int16_t* sQ = reinterpret_cast<int16_t*>(smem + (size_t)MB * g.K * 4);             // [MB][64][kQStride]
  uint32_t* sS = reinterpret_cast<uint32_t*>(smem + (size_t)MB * g.K * 4 + (size_t)MB * 64 * kQStride * 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int G = g.K / W4_GROUP;
  const int nw = gridDim.x * kWarps;
  int n = blockIdx.x * kWarps + warp;
  uint4 w[2][4], wn[2][4];
  auto load_col = [&](int col, uint4 (*dst)[4]) {
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int gi = lane + 32 * slot;
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
  if (n < g.N) load_col(n, w);
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
  align_rows<MB>(g, mb, sX, sQ, sS);
  __syncthreads();

  for (; n < g.N; n += nw) {
    const int nn = n + nw;
    if (nn < g.N) load_col(nn, wn);
    float term[MB][2];
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int gi = lane + 32 * slot;
#pragma unroll
      for (int m = 0; m < MB; ++m) term[m][slot] = 0.0f;
      if (gi < G) {
        const float ws = from_fp16(ld_u16(g.scale + 2 * ((uint64_t)n * G + gi)));
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m < mb) {
            const uint32_t* q = reinterpret_cast<const uint32_t*>(sQ + (m * 64 + gi) * kQStride);
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t words[4] = {w[slot][i].x, w[slot][i].y, w[slot][i].z, w[slot][i].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint32_t lo, hi;
                unpack8(words[j], lo, hi);
                const int base = (i * 4 + j) * 4;  // 8 elements = 4 words of int16 pairs
                dot = __dp2a_lo((int)q[base + 0], (int)lo, dot);
                dot = __dp2a_hi((int)q[base + 1], (int)lo, dot);
                dot = __dp2a_lo((int)q[base + 2], (int)hi, dot);
                dot = __dp2a_hi((int)q[base + 3], (int)hi, dot);
              }
            }
            term[m][slot] = fmul(fmul(i2f(dot), ws), bf(sS[m * 64 + gi]));
          }
        }
      }
    }
    // banks: lane b (< 4) adds terms g = b, b + 4, ... in order
    const int b = lane & 3;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      float bank = 0.0f;
      for (int i = 0; 4 * i < G; ++i) {
        const int gi = b + 4 * i;
        const float t0 = __shfl_sync(0xFFFFFFFFu, term[m][0], gi & 31);
        const float t1 = __shfl_sync(0xFFFFFFFFu, term[m][1], gi & 31);
        if (gi < G) bank = fadd_nc(bank, gi < 32 ? t0 : t1);
      }
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
    for (int slot = 0; slot < 2; ++slot)
#pragma unroll
      for (int i = 0; i < 4; ++i) w[slot][i] = wn[slot][i];
  }
}

template <int MB>
cudaError_t launch_w4(const W4Args& g, cudaStream_t st) {
  const size_t smem = (size_t)MB * g.K * 4 + (size_t)MB * 64 * kQStride * 2 + (size_t)MB * 64 * 4;
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
  if (g.M == 1) return launch_w4<1>(g, st);
  if (g.M == 2) return launch_w4<2>(g, st);
  return launch_w4<4>(g, st);
}

}  // namespace tc
