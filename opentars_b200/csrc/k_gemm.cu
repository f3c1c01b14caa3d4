// W8A8 GEMV / GEMM (golden.py:326-349) and the conv's im2col (golden.py:282-293) for sm_100a.
//
// Integer part: int8 x int8 products summed in int32 with dp4a. Two's-complement int32 sums are
// exact in any order when the final value fits (|acc| <= 128*128*65535 < 2^31 for every legal K),
// so the reduction order is free. Epilogue, in the reference's order and rounding:
//   y = i2f(acc); [y = fmul(y, srow[m])]; y = fmul(y, scale[n or 0]); [y = fadd(y, bias[n])];
//   y = act(y); store in the output format.
//
// Layout: W rows [N, K] int8 stream from HBM once per pass through 16-byte non-allocating loads,
// 32 lanes x 16 B = one 512 B coalesced line per warp instruction; the M activation rows of a pass
// are staged in shared memory in K-chunks of KC bytes. One warp owns NCW output columns.
#include <cuda_runtime.h>

#include <algorithm>

#include "fp32.cuh"
#include "gemm_epi.cuh"
#include "mma.h"
#include "ops.h"

namespace tc {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int KC = 4096;

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

template <bool VEC>
__device__ __forceinline__ uint4 load16(const uint8_t* p) {
  if (VEC) return ldg_stream(p);
  return make_uint4(ld_u32(p), ld_u32(p + 4), ld_u32(p + 8), ld_u32(p + 12));
}

// One pass: rows [m0, m0 + mb) of A (mb <= MB), NCW columns per warp.
template <int MB, int NCW, bool VEC>
__global__ void __launch_bounds__(kThreads) k_gemv_i8(GemmArgs g) {
  __shared__ __align__(16) uint8_t sA[MB * KC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int nbase = (blockIdx.x * kWarps + warp) * NCW;
  int acc[NCW][MB];
#pragma unroll
  for (int c = 0; c < NCW; ++c)
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[c][m] = 0;

  for (int k0 = 0; k0 < g.K; k0 += KC) {
    const int kc = min(KC, g.K - k0);
    __syncthreads();
    for (int i = threadIdx.x * 4; i < mb * kc; i += kThreads * 4) {
      const int m = i / kc, k = i - m * kc;
      *reinterpret_cast<uint32_t*>(&sA[m * KC + k]) = ld_u32(g.A + (uint64_t)(m0 + m) * g.lda + k0 + k);
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < NCW; ++c) {
      const int n = nbase + c;
      if (n >= g.N) break;
      const uint8_t* wrow = g.W + (uint64_t)n * g.K + k0;
#pragma unroll 4
      for (int k = lane * 16; k < kc; k += 512) {
        const uint4 w = load16<VEC>(wrow + k);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m < mb) {
            const uint4 a = *reinterpret_cast<const uint4*>(&sA[m * KC + k]);
            int s = acc[c][m];
            s = __dp4a((int)a.x, (int)w.x, s);
            s = __dp4a((int)a.y, (int)w.y, s);
            s = __dp4a((int)a.z, (int)w.z, s);
            s = __dp4a((int)a.w, (int)w.w, s);
            acc[c][m] = s;
          }
        }
      }
    }
  }
  int mine = 0;
#pragma unroll
  for (int c = 0; c < NCW; ++c)
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      int v = acc[c][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      if (lane == c * MB + m) mine = v;
    }
  if (lane < NCW * MB) {
    const int c = lane / MB, m = lane - c * MB;
    const int n = nbase + c;
    if (n < g.N && m < mb) gemm_epilogue(g, m0 + m, n, mine);
  }
}

template <int MB, int NCW>
cudaError_t launch_gemv(const GemmArgs& g, bool vec, cudaStream_t st) {
  dim3 grid((g.N + kWarps * NCW - 1) / (kWarps * NCW), (g.M + MB - 1) / MB);
  if (vec) k_gemv_i8<MB, NCW, true><<<grid, kThreads, 0, st>>>(g);
  else k_gemv_i8<MB, NCW, false><<<grid, kThreads, 0, st>>>(g);
  return cudaGetLastError();
}

// Decode GEMV (M <= 8, K <= 512 * KU, 16-byte aligned operands). Persistent warps: each warp owns
// output columns gw, gw + nw, ...; a lane holds the 16-byte slices k = lane*16 + 512u of one
// column's weights in registers. The first column's loads are issued before the block stages its
// activation rows in shared memory, and each next column's loads before the current one is
// reduced, so every warp keeps two columns of weights in flight.
template <int MB, int KU>
__global__ void __launch_bounds__(kThreads) k_gemv8(GemmArgs g) {
  __shared__ __align__(16) uint8_t sA[MB * 512 * KU];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int nw = gridDim.x * kWarps;
  int n = blockIdx.x * kWarps + warp;
  uint4 w[KU], wn[KU];
  auto load_col = [&](int col, uint4* dst) {
    const uint8_t* row = g.W + (uint64_t)col * g.K;
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = lane * 16 + 512 * u;
      dst[u] = k < g.K ? ldg_stream(row + k) : make_uint4(0, 0, 0, 0);
    }
  };
  if (n < g.N) load_col(n, w);
  const int kv = g.K / 16;
  for (int i = threadIdx.x; i < mb * kv; i += kThreads) {
    const int m = i / kv, kk = (i - m * kv) * 16;
    cp16(&sA[m * 512 * KU + kk], g.A + (uint64_t)(m0 + m) * g.lda + kk);
  }
  cp_wait_all();
  __syncthreads();
  for (; n < g.N; n += nw) {
    const int nn = n + nw;
    if (nn < g.N) load_col(nn, wn);
    int acc[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[m] = 0;
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = lane * 16 + 512 * u;
      if (k < g.K) {
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (m < mb) {
            const uint4 a = *reinterpret_cast<const uint4*>(&sA[m * 512 * KU + k]);
            int s = acc[m];
            s = __dp4a((int)a.x, (int)w[u].x, s);
            s = __dp4a((int)a.y, (int)w[u].y, s);
            s = __dp4a((int)a.z, (int)w[u].z, s);
            s = __dp4a((int)a.w, (int)w[u].w, s);
            acc[m] = s;
          }
        }
      }
    }
    int mine = 0;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      int v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      if (lane == m) mine = v;
    }
    if (lane < mb) gemm_epilogue(g, m0 + lane, n, mine);
#pragma unroll
    for (int u = 0; u < KU; ++u) w[u] = wn[u];
  }
}

template <int MB, int KU>
cudaError_t launch_gemv8(const GemmArgs& g, cudaStream_t st) {
  const int blocks = std::min((g.N + kWarps - 1) / kWarps, 148 * 4);
  k_gemv8<MB, KU><<<dim3(blocks, (g.M + MB - 1) / MB), kThreads, 0, st>>>(g);
  return cudaGetLastError();
}

template <int MB>
cudaError_t launch_gemv8_k(const GemmArgs& g, cudaStream_t st) {
  if (g.K <= 1024) return launch_gemv8<MB, 2>(g, st);
  if (g.K <= 2048) return launch_gemv8<MB, 4>(g, st);
  return launch_gemv8<MB, 8>(g, st);
}

__global__ void k_im2col(Im2colArgs a) {
  const int K = a.KH * a.KW * a.Cin;
  const uint64_t total = (uint64_t)a.OH * a.OW * K;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / K), kk = (int)(i - (uint64_t)r * K);
    const int ky = kk / (a.KW * a.Cin), kx = (kk / a.Cin) % a.KW, ci = kk % a.Cin;
    const int oy = r / a.OW, ox = r - oy * a.OW;
    const int iy = oy * a.S - a.P + ky, ix = ox * a.S - a.P + kx;
    uint8_t v = 0;
    if (iy >= 0 && iy < a.H && ix >= 0 && ix < a.W) v = a.img[(uint64_t)(iy * a.W + ix) * a.ld + ci];
    a.out[i] = v;
  }
}
}  // namespace

cudaError_t launch_gemm_w8a8(const GemmArgs& g, cudaStream_t st) {
  if (g.M >= mma_min_rows() && mma_machine_ok(g)) return gemm_mma(g, st);
  const bool vec = ((uintptr_t)g.A % 16 == 0) && (g.lda % 16 == 0) && ((uintptr_t)g.W % 16 == 0) && (g.K % 16 == 0);
  if (vec && g.K <= 4096 && g.M <= 8) {
    if (g.M == 1) return launch_gemv8_k<1>(g, st);
    if (g.M == 2) return launch_gemv8_k<2>(g, st);
    if (g.M <= 4) return launch_gemv8_k<4>(g, st);
    return launch_gemv8_k<8>(g, st);
  }
  if (g.M == 1) return launch_gemv<1, 4>(g, vec, st);
  if (g.M == 2) return launch_gemv<2, 4>(g, vec, st);
  if (g.M <= 4) return launch_gemv<4, 4>(g, vec, st);
  return launch_gemv<8, 4>(g, vec, st);
}

cudaError_t launch_im2col(const Im2colArgs& a, cudaStream_t st) {
  const uint64_t total = (uint64_t)a.OH * a.OW * a.KH * a.KW * a.Cin;
  const int blocks = (int)std::min<uint64_t>((total + 255) / 256, 148 * 16);
  k_im2col<<<blocks, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace tc
