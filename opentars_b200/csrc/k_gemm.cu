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
#include "umma.cuh"

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
// Column block bx of nbx, token-row pass by.
template <int MB, int KU>
__device__ __forceinline__ void gemv8_body(const GemmArgs& g, int bx, int nbx, int by, uint8_t* sA) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = by * MB;
  const int mb = min(MB, g.M - m0);
  const int nw = nbx * kWarps;
  int n = bx * kWarps + warp;
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
__global__ void __launch_bounds__(kThreads) k_gemv8(GemmArgs g) {
  __shared__ __align__(16) uint8_t sA[MB * 512 * KU];
  gemv8_body<MB, KU>(g, blockIdx.x, gridDim.x, blockIdx.y, sA);
}

// The GEMVs of one dependency level in one launch, with the weights streamed through shared
// memory. Work unit: a chunk of 16 consecutive output columns (16 * K contiguous weight bytes; N is
// a multiple of 16) for one pass of MB token rows. The group's chunks form one list (entry by
// entry) that is cut into gridDim.x equal contiguous ranges, one per block. Warp 0's lane 0 copies
// each chunk's weights, and its 16 scales and biases, with 1-D bulk copies into a ring of
// kSStages stages (completing on the stage's mbarrier). Consumer warp w (1..kSStages) owns stage
// w - 1 and takes every kSStages-th chunk, so it waits for the stage's phases strictly in order.
// A warp computes the 16 columns of a chunk in batches of CB = 16 / MB columns: lane L holds the
// partial int32 dots of k in {16L + 512u}; the 16 (row, column) sums of a batch are reduced
// across the warp by one transpose reduction (16 shuffles; lanes 2i and 2i + 1 end with sum i)
// and 16 lanes run the epilogue of k_gemv8 at once. int32 sums are exact in any order.
// Every wait is bounded; after a timeout the block skips its remaining chunks.
constexpr int kSCols = 16;
// The group's waits sleep in the poll (up to about this many nanoseconds).
constexpr uint32_t kGroupWaitNs = 1000;

template <int KU>
__host__ __device__ constexpr int s_stages() { return KU <= 2 ? 6 : (KU <= 4 ? 3 : 2); }

__device__ __forceinline__ uint4 ldg_l1(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ int dot16(const uint4& a, const uint4& w, int s) {
  s = __dp4a((int)a.x, (int)w.x, s);
  s = __dp4a((int)a.y, (int)w.y, s);
  s = __dp4a((int)a.z, (int)w.z, s);
  return __dp4a((int)a.w, (int)w.w, s);
}

template <int MB, int KU>
__global__ void __launch_bounds__(32 * (1 + s_stages<KU>()), 2)
    k_gemv8_group(const __grid_constant__ GemvGroup grp) {
  constexpr int S = s_stages<KU>();
  constexpr int CB = MB >= kSCols ? 1 : kSCols / MB;          // columns per batch; MB * CB == 16
  constexpr uint32_t kWB = kSCols * 512 * KU;                 // weight bytes of a stage (largest K)
  constexpr uint32_t kStage = kWB + 128;                      // + 16 scales + 16 biases
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[S], empty[S];
  __shared__ int s_stop;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = grp.c0[grp.n];
  const int c_begin = (int)((long long)blockIdx.x * total / gridDim.x);
  const int c_end = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    s_stop = 0;
    mbar_fence_init();
  }
  __syncthreads();
  int j = 0;                                                  // the entry of chunk c_begin
  while (c_begin >= grp.c0[j + 1] && j + 1 < grp.n) ++j;
  __shared__ int s_issued;
  // consumer warp st + 1 owns stage st and takes every S-th chunk
  auto consume = [&](const int st) {
    const uint8_t* stage = smem + (size_t)st * kStage;
    uint4 areg[MB == 1 ? KU : 1];                               // M = 1: the activation row in registers
    int areg_j = -1;
    for (int c = c_begin + st, t = st; c < c_end; c += S, t += S) {
      const bool ok = !*(volatile int*)&s_stop && mbar_wait_hint(&full[st], (t / S) & 1, grp.err, 22, grp.spin, kGroupWaitNs);
      if (!__all_sync(0xFFFFFFFFu, ok)) {                           // the whole warp stops together
        s_stop = 1;
        break;
      }
      while (c >= grp.c0[j + 1]) ++j;
      const GemmArgs& g = grp.g[j];
      const int local = c - grp.c0[j], ncx = grp.ncx[j];
      const int by = local / ncx, cx = local - by * ncx;
      const int m0 = by * MB, mb = min(MB, g.M - m0);
      const uint8_t* arow = g.A + (uint64_t)m0 * g.lda;
      if constexpr (MB == 1) {
        if (areg_j != j) {
#pragma unroll
          for (int u = 0; u < KU; ++u) {
            const int k = lane * 16 + 512 * u;
            areg[u] = k < g.K ? ldg_l1(arow + k) : make_uint4(0, 0, 0, 0);
          }
          areg_j = j;
        }
      }
      const float* ssc = reinterpret_cast<const float*>(stage + kWB);
      const float* sbi = reinterpret_cast<const float*>(stage + kWB + 64);
      // the epilogue lanes' scale and bias before the stage is released
      const int i_mine = lane >> 1, m_mine = i_mine / CB, c_mine = i_mine - m_mine * CB;
      float sc[kSCols / CB], bi[kSCols / CB];
#pragma unroll
      for (int b = 0; b < kSCols / CB; ++b) {
        sc[b] = g.per_channel ? ssc[b * CB + c_mine] : 0.0f;
        bi[b] = g.bias ? sbi[b * CB + c_mine] : 0.0f;
      }
      int res[kSCols / CB];
#pragma unroll
      for (int b = 0; b < kSCols / CB; ++b) {
        int acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0;
#pragma unroll
        for (int u = 0; u < KU; ++u) {
          const int k = lane * 16 + 512 * u;
          if (k < g.K) {
            uint4 a[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m) {
              if constexpr (MB == 1) a[m] = areg[u];
              else a[m] = m < mb ? ldg_l1(arow + (uint64_t)m * g.lda + k) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int cc = 0; cc < CB; ++cc) {
              const uint4 w = *reinterpret_cast<const uint4*>(stage + (size_t)(b * CB + cc) * g.K + k);
#pragma unroll
              for (int m = 0; m < MB; ++m) acc[m * CB + cc] = dot16(a[m], w, acc[m * CB + cc]);
            }
          }
        }
        // transpose reduction: after the step with offset o, lane bit o selects which half it keeps
#pragma unroll
        for (int o = 16, v = 16; o >= 2; o >>= 1, v >>= 1) {
          const bool hi = (lane & o) != 0;
#pragma unroll
          for (int i = 0; i < v / 2; ++i) {
            const int send = hi ? acc[i] : acc[i + v / 2];
            const int keep = hi ? acc[i + v / 2] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
          }
        }
        res[b] = acc[0] + __shfl_xor_sync(0xFFFFFFFFu, acc[0], 1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);                   // the stage's bytes are consumed
      const float sc0 = g.per_channel ? 0.0f : ld_f32(g.scale);
      if ((lane & 1) == 0 && m_mine < mb) {
#pragma unroll
        for (int b = 0; b < kSCols / CB; ++b)
          gemm_epilogue_v(g, m0 + m_mine, cx * kSCols + b * CB + c_mine, res[b], g.per_channel ? sc[b] : sc0, bi[b]);
      }
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      int t = 0;
      for (int c = c_begin; c < c_end; ++c, ++t) {
        const int st = t % S;
        if (!mbar_wait_hint(&empty[st], ((t / S) & 1) ^ 1, grp.err, 21, grp.spin, kGroupWaitNs)) {
          s_stop = 1;
          break;
        }
        while (c >= grp.c0[j + 1]) ++j;
        const GemmArgs& g = grp.g[j];
        const int cx = (c - grp.c0[j]) % grp.ncx[j];
        const uint32_t wb = kSCols * (uint32_t)g.K;
        uint8_t* dst = smem + (size_t)st * kStage;
        mbar_expect_tx(&full[st], wb + (g.per_channel ? 64 : 0) + (g.bias ? 64 : 0));
        bulk_load(dst, g.W + (uint64_t)cx * wb, wb, &full[st]);
        if (g.per_channel) bulk_load(dst + kWB, g.scale + 64 * (uint64_t)cx, 64, &full[st]);
        if (g.bias) bulk_load(dst + kWB + 64, g.bias + 64 * (uint64_t)cx, 64, &full[st]);
      }
      s_issued = t;
    }
  } else {
    consume(warp - 1);
  }
  // After a wait gave up, copies of the last chunks issued may still be in flight: the block does
  // not exit before they land (these waits always have the full limit).
  __syncthreads();
  if (threadIdx.x == 0 && s_stop)
    for (int u = s_issued > S ? s_issued - S : 0; u < s_issued; ++u) mbar_wait(&full[u % S], (u / S) & 1, nullptr, 0);
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
    if (iy >= 0 && iy < a.H && ix >= 0 && ix < a.W) v = a.img[((uint64_t)iy * a.W + ix) * a.ld + ci];
    a.out[i] = v;
  }
}

bool gemv8_ok(const GemmArgs& g) {
  return ((uintptr_t)g.A % 16 == 0) && (g.lda % 16 == 0) && ((uintptr_t)g.W % 16 == 0) && (g.K % 16 == 0);
}

template <int MB, int KU>
cudaError_t launch_group(GemvGroup& grp, cudaStream_t st) {
  constexpr int S = s_stages<KU>();
  constexpr int threads = 32 * (1 + S);
  const int smem = S * (kSCols * 512 * KU + 128);
  auto kern = k_gemv8_group<MB, KU>;
  static int resident = 0;                                  // blocks resident on the GPU at once
  if (!resident) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
    if (e != cudaSuccess) return e;
    resident = std::max(per_sm, 1) * 148;
  }
  grp.c0[0] = 0;
  for (int j = 0; j < grp.n; ++j) {
    const GemmArgs& g = grp.g[j];
    grp.ncx[j] = g.N / kSCols;
    grp.c0[j + 1] = grp.c0[j] + grp.ncx[j] * ((g.M + MB - 1) / MB);
  }
  const int blocks = std::min(grp.c0[grp.n], resident);
  kern<<<blocks, threads, smem, st>>>(grp);
  return cudaGetLastError();
}
}  // namespace

int gemv8_class(const GemmArgs& g) {
  if (g.M >= mma_min_rows() && mma_machine_ok(g)) return -1;
  if (!gemv8_ok(g) || g.K > 4096 || g.M > 8 || g.M < 1 || g.N < kSCols || g.N % kSCols) return -1;
  if ((g.per_channel && (uintptr_t)g.scale % 16) || (g.bias && (uintptr_t)g.bias % 16)) return -1;
  const int mb = g.M == 1 ? 1 : g.M == 2 ? 2 : g.M <= 4 ? 4 : 8;
  const int ku = g.K <= 1024 ? 2 : g.K <= 2048 ? 4 : 8;
  return mb * 16 + ku;
}

cudaError_t launch_gemv8_group(GemvGroup& grp, cudaStream_t st) {
  grp.err = wait_error_flag();
  grp.spin = spin_limit();
  switch (grp.mb * 16 + grp.ku) {
    case 1 * 16 + 2: return launch_group<1, 2>(grp, st);
    case 1 * 16 + 4: return launch_group<1, 4>(grp, st);
    case 1 * 16 + 8: return launch_group<1, 8>(grp, st);
    case 2 * 16 + 2: return launch_group<2, 2>(grp, st);
    case 2 * 16 + 4: return launch_group<2, 4>(grp, st);
    case 2 * 16 + 8: return launch_group<2, 8>(grp, st);
    case 4 * 16 + 2: return launch_group<4, 2>(grp, st);
    case 4 * 16 + 4: return launch_group<4, 4>(grp, st);
    case 4 * 16 + 8: return launch_group<4, 8>(grp, st);
    case 8 * 16 + 2: return launch_group<8, 2>(grp, st);
    case 8 * 16 + 4: return launch_group<8, 4>(grp, st);
    case 8 * 16 + 8: return launch_group<8, 8>(grp, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm_w8a8(const GemmArgs& g, cudaStream_t st) {
  if (g.M >= mma_min_rows() && mma_machine_ok(g)) {
    // A transcendental activation (GELU, SiLU, sigmoid, softplus, exp: about 200 dependent steps
    // per element) on fp32 output runs as its own elementwise pass over the whole GPU instead of in
    // the tensor-core GEMM's few epilogue warps: the GEMM stores the fp32 pre-activation values in
    // the output, the pass applies the activation in place - the same value per element.
    if (g.act >= 3 && g.out == OUT_FP32) {
      GemmArgs g2 = g;
      g2.act = 0;
      cudaError_t e = gemm_mma(g2, st);
      if (e != cudaSuccess) return e;
      ActArgs a{};
      a.X = g.Y; a.lda = g.ldy; a.Y = g.Y; a.ldy = g.ldy;
      a.M = g.M; a.N = g.N; a.act = g.act; a.out = OUT_FP32; a.out_scale = g.out_scale;
      return launch_act(a, st);
    }
    return gemm_mma(g, st);
  }
  const bool vec = gemv8_ok(g);
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
