// The batched decode engine's kernels (Qwen3 / Gemma 3 full-attention layers), sm_100a.
//
// The engine runs the step that QwenLowering.chunk lowers to descriptors (tars_mini/llm.py:548-571,
// 582-593, 614-640, 705-782) for B independent sequences at once: every row-wise op and every
// GEMM takes the B sequences' rows together (one weight stream for the whole batch), attention
// runs per (sequence, query head) on that sequence's own KV cache. Each kernel computes exactly
// the values the descriptors would write (same steps, same rounding, same reduction orders), so
// each sequence's logits equal the golden model's for that sequence alone, bit for bit. Rows are
// ordered sequence-major: row r = b * n + m is token t0 + m of sequence b.
#include <cuda_runtime.h>

#include <algorithm>

#include "engine.h"
#include "mma.h"
#include "fp32.cuh"
#include "umma.cuh"
#include "pdl.cuh"

namespace tc {
namespace {

constexpr int kT = 256;

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float sum16_fold(float v, unsigned mask = 0xFFFFFFFFu) {
  v = fadd(v, __shfl_xor_sync(mask, v, 1));
  v = fadd(v, __shfl_xor_sync(mask, v, 2));
  v = fadd(v, __shfl_xor_sync(mask, v, 4));
  v = fadd(v, __shfl_xor_sync(mask, v, 8));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = fmax_c(r, red[i]);
  return r;
}
// sum16 of v[0..N) (shared memory) in the contract's order, broadcast to the block. Each chain
// loads 8 of its values before their 8 dependent adds (the order of the adds is unchanged).
__device__ __forceinline__ float block_sum16(const float* v, int N, float* red) {
  __syncthreads();
  if (threadIdx.x < 16) {
    float acc = 0.0f;
    int j = threadIdx.x;
    for (; j + 16 * 7 < N; j += 16 * 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = v[j + 16 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = fadd_nc(acc, t[u]);
    }
    for (; j < N; j += 16) acc = fadd_nc(acc, v[j]);
    acc = sum16_fold(canon(acc), 0x0000FFFFu);
    if (threadIdx.x == 0) red[32] = acc;
  }
  __syncthreads();
  return red[32];
}

// ------------------------------------------------------------------------------- embedding
// x[r] = E[tok[r]] (Gemma: times fp32(sqrt(H)) in IEEE fp32, as the host's numpy does), llm.py:198-204
__global__ void k_embed(const float* E, const int* tok, float* x, int H, int scale_on, float scale, int rows) {
  griddep_launch();
  griddep_wait();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* e = E + (uint64_t)tok[r] * H;
  for (int j = threadIdx.x; j < H; j += blockDim.x) x[(uint64_t)r * H + j] = scale_on ? __fmul_rn(e[j], scale) : e[j];
}

// ------------------------------------------------------------------------------- row kernels
// Optional pre-step, then RMSNorm(x, gamma) and ROW_QUANT of the normalised row:
//   mode 0: x = in                                          (a layer's ln_in, the final norm)
//   mode 1: x = fadd(res, in)          and x is written out (Qwen3: after o / down)
//   mode 2: x = fadd(res, rmsnorm(in, pre_gamma)), written   (Gemma 3: attn_norm / mlp_norm)
// Outputs the int8 row and its row scale (llm.py:97-104, numerics.py:353-390).
__global__ void __launch_bounds__(256) k_norm_quant(NormQuantArgs a) {
  griddep_launch();
  extern __shared__ float sm[];
  float* sx = sm;
  float* sv = sm + a.H;
  float* sg = sm + 2 * a.H;                      // gamma, then pre_gamma (mode 2)
  float* spg = sm + 3 * a.H;
  __shared__ float red[33];
  const int r = blockIdx.x, H = a.H, t = threadIdx.x;
  // the norms' weights do not depend on the previous kernel: staged before the dependency wait
  if ((((uintptr_t)a.gamma | (uintptr_t)a.pre_gamma) & 15) == 0 && H % 4 == 0) {
    for (int j4 = t; j4 < H / 4; j4 += blockDim.x) {
      cp16(sg + 4 * j4, a.gamma + 4 * j4);
      if (a.mode == 2) cp16(spg + 4 * j4, a.pre_gamma + 4 * j4);
    }
  } else {
    for (int j = t; j < H; j += blockDim.x) {
      sg[j] = a.gamma[j];
      if (a.mode == 2) spg[j] = a.pre_gamma[j];
    }
  }
  griddep_wait();
  const float kinv = recip_f(i2f(H));
  const float* in = a.in + (uint64_t)r * a.ld_in;
  const float* res = a.res + (uint64_t)r * H;
  float* sres = sm + 4 * H;                      // the residual row, staged with the input row
  const bool res_v = a.mode >= 1 && ((uintptr_t)a.res & 15) == 0 && H % 4 == 0;
  for (int j4 = t; j4 < H / 4; j4 += blockDim.x) {
    cp16(sx + 4 * j4, in + 4 * j4);
    if (res_v) cp16(sres + 4 * j4, res + 4 * j4);
  }
  cp_wait_all();
  __syncthreads();
  for (int j = t; j < H; j += blockDim.x) sx[j] = ftz(sx[j]);
  if (a.mode == 2) {
    __syncthreads();
    for (int j = t; j < H; j += blockDim.x) sv[j] = fmul(sx[j], sx[j]);
    const float s = block_sum16(sv, H, red);
    const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
    for (int j = t; j < H; j += blockDim.x) sx[j] = ftz(fmul(fmul(sx[j], rs), spg[j]));
  }
  if (a.mode >= 1) {
    for (int j = t; j < H; j += blockDim.x) {
      const float v = fadd(res_v ? sres[j] : res[j], sx[j]);
      sx[j] = ftz(v);
      a.x_out[(uint64_t)r * H + j] = ftz(v);
    }
  }
  __syncthreads();
  for (int j = t; j < H; j += blockDim.x) sv[j] = fmul(sx[j], sx[j]);
  const float s = block_sum16(sv, H, red);
  const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
  float amax = 0.0f;
  for (int j = t; j < H; j += blockDim.x) {
    const float h = ftz(fmul(fmul(sx[j], rs), sg[j]));
    sv[j] = h;
    amax = fmax_c(amax, fabs_c(h));
  }
  amax = block_max(amax, red);
  const float inv = fmul(127.0f, recip_f(amax));
  int8_t* q = a.q + (uint64_t)r * a.ldq;
  for (int j = t; j < H; j += blockDim.x) q[j] = q8(sv[j], inv);
  if (t == 0) a.qs[r] = ftz(fmul(amax, bf(0x3C010204u)));
}

// ROW_QUANT alone (attention output, gate * up), numerics.py:383-390
// Row quantisation with a row spread over a cluster of kQCluster CTAs (every SM busy at batch
// 64): CTA c takes a contiguous quarter of the row (for the gated MLP computing its elements
// v = ftz(fmul(ftz(act(gate)), up)) first), the CTAs exchange their partial absmax through
// distributed shared memory (max is order-free), then each quantises its slice.
constexpr int kQCluster = 4;
template <int ACT, bool GATED>
__global__ void __launch_bounds__(256) k_quant_cl(const float* x, const float* up, int ld, int N, int act, int8_t* q,
                                                  int ldq, float* qs) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float4 qrow4[];
  float* row = reinterpret_cast<float*>(qrow4);
  __shared__ float red[33];
  __shared__ float s_part;
  const int r = blockIdx.x / kQCluster, c = (int)cluster_rank();
  const int S = ((N + kQCluster - 1) / kQCluster + 3) / 4 * 4;
  const int j0 = min(N, c * S), j1 = min(N, j0 + S);
  const float* src = x + (uint64_t)r * ld;
  float amax = 0.0f;
  if constexpr (GATED) {
    const float* us = up + (uint64_t)r * ld;
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
      float a;
      if constexpr (ACT == 4) a = silu_f(src[j]);
      else if constexpr (ACT == 3) a = gelu_f(src[j]);
      else a = act_fn(src[j], act);
      const float v = ftz(fmul(ftz(a), us[j]));
      row[j - j0] = v;
      amax = fmax_c(amax, fabs_c(v));
    }
  } else {
    for (int j4 = j0 / 4 + threadIdx.x; j4 < j1 / 4; j4 += blockDim.x) cp16(row + 4 * j4 - j0, src + 4 * j4);
    cp_wait_all();
    __syncthreads();
    for (int j = threadIdx.x; j < j1 - j0; j += blockDim.x) amax = fmax_c(amax, fabs_c(row[j]));
  }
  amax = block_max(amax, red);
  if (threadIdx.x == 0) s_part = amax;
  cluster_sync();
  amax = s_part;
  for (int p = 0; p < kQCluster; ++p)
    if (p != c) amax = fmax_c(amax, __int_as_float(dsmem_ld_s32(smem_u32(&s_part), p)));
  const float inv = fmul(127.0f, recip_f(amax));
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) q[(uint64_t)r * ldq + j] = q8(row[j - j0], inv);
  if (c == 0 && threadIdx.x == 0) qs[r] = ftz(fmul(amax, bf(0x3C010204u)));
  cluster_sync();                                 // the peers have read s_part
}

template <class Kern>
static cudaError_t launch_quant_cl(Kern kern, const float* x, const float* up, int ld, int N, int act, int8_t* q,
                                   int ldq, float* qs, int rows, cudaStream_t st) {
  const int S = ((N + kQCluster - 1) / kQCluster + 3) / 4 * 4;
  const int smem = S * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  return launch_ex(kern, dim3(rows * kQCluster), dim3(256), smem, st, kQCluster, x, up, ld, N, act, q, ldq, qs);
}

// ------------------------------------------------------------------------------- GEMV
// y[m][col] over the concatenated output columns of up to kMaxSegs weight blocks. Epilogue per
// output: y = fmul(fmul(i2f(acc), srow[m]), scale[n]) (golden.py:336-344), then by mode:
//   kEpiStore   store y (flushed) to the segment's output
//   kEpiResid   store fadd(res[m][col], y)
//   kEpiGated   segments 0 (gate) and 1 (up) of equal width: out = fmul(act(y_gate), y_up)
//   kEpiKSplit  K blocks of kb: y = fadd(ep(acc_0), ep(acc_1)), then store (or add res if given)
template <int MB, int KU>
__global__ void __launch_bounds__(256) k_eng_gemv(EngGemvArgs g) {
  __shared__ __align__(16) int8_t sA[MB * 512 * KU];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MB;
  const int mb = min(MB, g.M - m0);
  const int nw = gridDim.x * 8;
  const int ncols = g.mode == kEpiGated ? g.seg[0].n : g.ncols;
  const int kv = g.K / 16;
  griddep_launch();
  griddep_wait();
  for (int i = threadIdx.x; i < mb * kv; i += blockDim.x) {
    const int m = i / kv, kk = (i - m * kv) * 16;
    cp16(&sA[m * 512 * KU + kk], g.A + (uint64_t)(m0 + m) * g.lda + kk);
  }
  cp_wait_all();
  __syncthreads();
  for (int col = blockIdx.x * 8 + warp; col < ncols; col += nw) {
    int s = 0;
    while (s + 1 < g.nseg && col >= g.seg[s + 1].n0) ++s;
    const int c = col - g.seg[s].n0;
    const int nrows = g.mode == kEpiGated ? 2 : 1;
    int acc[2][2][MB];                       // [weight row][K block][m]
#pragma unroll
    for (int w = 0; w < 2; ++w)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[w][h][m] = 0;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      if (w >= nrows) break;
      const EngSeg& sg = g.seg[w == 0 ? s : 1];
      const int8_t* w1 = sg.W + (uint64_t)c * g.kb;
      const int8_t* w2 = sg.W2 + (uint64_t)c * (g.K - g.kb) - g.kb;
      uint4 wv[KU];
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        const int k = lane * 16 + 512 * u;
        wv[u] = k >= g.K ? make_uint4(0, 0, 0, 0) : ldg_stream(k < g.kb ? w1 + k : w2 + k);
      }
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        const int k = lane * 16 + 512 * u;
        if (k < g.K) {
          const int h = k >= g.kb ? 1 : 0;
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            if (m < mb) {
              const uint4 av = *reinterpret_cast<const uint4*>(&sA[m * 512 * KU + k]);
              int v = acc[w][h][m];
              v = __dp4a((int)av.x, (int)wv[u].x, v);
              v = __dp4a((int)av.y, (int)wv[u].y, v);
              v = __dp4a((int)av.z, (int)wv[u].z, v);
              v = __dp4a((int)av.w, (int)wv[u].w, v);
              acc[w][h][m] = v;
            }
          }
        }
      }
    }
    // reduce the partial sums over the 32 lanes; lane m keeps row m
    int mine[2][2] = {{0, 0}, {0, 0}};
    const int nsplit = g.kb < g.K ? 2 : 1;
#pragma unroll
    for (int w = 0; w < 2; ++w)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          if (w >= nrows || h >= nsplit || m >= mb) continue;   // warp-uniform
          int v = acc[w][h][m];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
          if (lane == m) mine[w][h] = v;
        }
    if (lane < mb) {
      const int m = m0 + lane;
      const float sr = g.srow[m];
      auto ep = [&](int acc_v, const EngSeg& sg) { return fmul(fmul(i2f(acc_v), sr), sg.scale[c]); };
      const EngSeg& sg = g.seg[s];
      float y;
      if (g.mode == kEpiGated) {
        const float yg = ftz(act_fn(ep(mine[0][0], g.seg[0]), g.act));
        const float yu = ep(mine[1][0], g.seg[1]);
        g.seg[0].out[(uint64_t)m * g.seg[0].ldo + c] = ftz(fmul(yg, yu));
        continue;
      }
      if (g.mode == kEpiKSplit) y = fadd(ftz(ep(mine[0][0], sg)), ftz(ep(mine[0][1], sg)));
      else y = ep(mine[0][0], sg);
      if (g.res) y = fadd(g.res[(uint64_t)m * g.ldres + col], y);
      sg.out[(uint64_t)m * sg.ldo + c] = ftz(y);
    }
  }
}

// Batched GEMM for M > 8 token rows: one lane per token row. A block stages 32 rows of A in shared
// memory (row stride K + 16 bytes, so the 8 lanes of each 16-byte access phase hit 8 different
// bank groups) and its warps stream output columns: each lane holds the 16-byte weight slices
// k = lane*16 + 512u of the column, and the slices are broadcast to the warp with shuffles, so
// every lane accumulates its own row's exact int32 dot product with no cross-lane reduction.
// Same segments and epilogue modes as k_eng_gemv.
template <int KU>
__global__ void __launch_bounds__(128) k_eng_gemm_tl(EngGemvArgs g) {
  griddep_launch();
  griddep_wait();
  extern __shared__ __align__(16) int8_t sAt[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * 32;
  const int mb = min(32, g.M - m0);
  const int ld = g.K + 16;
  const int nw = gridDim.x * 4;
  const int ncols = g.mode == kEpiGated ? g.seg[0].n : g.ncols;
  const int kv = g.K / 16;
  for (int i = threadIdx.x; i < mb * kv; i += blockDim.x) {
    const int m = i / kv, kk = (i - m * kv) * 16;
    cp16(&sAt[m * ld + kk], g.A + (uint64_t)(m0 + m) * g.lda + kk);
  }
  cp_wait_all();
  __syncthreads();
  const int nrows = g.mode == kEpiGated ? 2 : 1;
  const int8_t* arow = sAt + (lane < mb ? lane : 0) * ld;
  for (int col = blockIdx.x * 4 + warp; col < ncols; col += nw) {
    int s = 0;
    while (s + 1 < g.nseg && col >= g.seg[s + 1].n0) ++s;
    const int c = col - g.seg[s].n0;
    int acc[2][2] = {{0, 0}, {0, 0}};          // [weight row][K block]
    for (int w = 0; w < nrows; ++w) {
      const EngSeg& sg = g.seg[w == 0 ? s : 1];
      const int8_t* w1 = sg.W + (uint64_t)c * g.kb;
      const int8_t* w2 = sg.W2 + (uint64_t)c * (g.K - g.kb) - g.kb;
      uint4 wv[KU];
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        const int k = lane * 16 + 512 * u;
        wv[u] = k >= g.K ? make_uint4(0, 0, 0, 0) : ldg_stream(k < g.kb ? w1 + k : w2 + k);
      }
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        if (512 * u >= g.K) break;
#pragma unroll 4
        for (int src = 0; src < 32; ++src) {
          const int k = src * 16 + 512 * u;
          if (k >= g.K) break;
          const uint32_t x = __shfl_sync(0xFFFFFFFFu, wv[u].x, src);
          const uint32_t y = __shfl_sync(0xFFFFFFFFu, wv[u].y, src);
          const uint32_t z = __shfl_sync(0xFFFFFFFFu, wv[u].z, src);
          const uint32_t q = __shfl_sync(0xFFFFFFFFu, wv[u].w, src);
          const uint4 av = *reinterpret_cast<const uint4*>(arow + k);
          const int h = k >= g.kb ? 1 : 0;
          int v = acc[w][h];
          v = __dp4a((int)av.x, (int)x, v);
          v = __dp4a((int)av.y, (int)y, v);
          v = __dp4a((int)av.z, (int)z, v);
          v = __dp4a((int)av.w, (int)q, v);
          acc[w][h] = v;
        }
      }
    }
    if (lane < mb) {
      const int m = m0 + lane;
      const float sr = g.srow[m];
      auto ep = [&](int acc_v, const EngSeg& sg) { return fmul(fmul(i2f(acc_v), sr), sg.scale[c]); };
      const EngSeg& sg = g.seg[s];
      if (g.mode == kEpiGated) {
        const float yg = ftz(act_fn(ep(acc[0][0] + acc[0][1], g.seg[0]), g.act));
        const float yu = ep(acc[1][0] + acc[1][1], g.seg[1]);
        g.seg[0].out[(uint64_t)m * g.seg[0].ldo + c] = ftz(fmul(yg, yu));
        continue;
      }
      float y;
      if (g.mode == kEpiKSplit) y = fadd(ftz(ep(acc[0][0], sg)), ftz(ep(acc[0][1], sg)));
      else y = ep(acc[0][0] + acc[0][1], sg);
      if (g.res) y = fadd(g.res[(uint64_t)m * g.ldres + col], y);
      sg.out[(uint64_t)m * sg.ldo + c] = ftz(y);
    }
  }
}

// ------------------------------------------------------------------------------- q / k heads
// Per row and head: RMSNorm over the head (gamma = q_norm * scaling or k_norm), then RoPE with the
// table row of the token's position (llm.py:718-734, numerics.py:353-358, 412-424). q -> qr;
// k -> the K cache row of (sequence, position). One half-warp per (row, head).
__global__ void __launch_bounds__(128) k_qk_rope(QkRopeArgs a) {
  griddep_launch();
  griddep_wait();
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int heads = a.nh + a.nkv;
  const int item = blockIdx.x * 8 + hw;
  const bool live = item < a.rows * heads;
  const int r = live ? item / heads : 0, h = live ? item % heads : 0;
  const bool isq = h < a.nh;
  const int b = r / a.n, m = r - b * a.n;
  const int t = a.pos[b] + m;
  const int hd = a.hd;
  const float* src = isq ? a.q + (uint64_t)r * a.nh * hd + h * hd : a.k + (uint64_t)r * a.nkv * hd + (h - a.nh) * hd;
  const float* gam = isq ? a.qn : a.kn;
  float v[16];                                 // hd <= 256: 16 elements per lane, j = l + 16 i
  float s = 0.0f;
  for (int i = 0; i < hd / 16; ++i) {
    v[i] = ftz(src[l + 16 * i]);
    s = fadd_nc(s, fmul(v[i], v[i]));
  }
  s = sum16_fold(canon(s));
  const float rs = rsqrt_f(fadd(fmul(s, recip_f(i2f(hd))), a.eps));
  __shared__ float sn[8][256];
  for (int i = 0; i < hd / 16; ++i) sn[hw][l + 16 * i] = ftz(fmul(fmul(v[i], rs), gam[l + 16 * i]));
  __syncwarp();
  if (!live) return;
  const float* tab = a.tab + (uint64_t)t * a.rot;
  float* dst = isq ? a.qr + (uint64_t)r * a.nh * hd + h * hd
                   : a.kc + (((uint64_t)b * a.Tp + t) * a.nkv + (h - a.nh)) * hd;
  const int half = a.rot / 2;
  for (int j = l; j < hd; j += 16) {
    float y;
    if (j < half) y = fadd(fmul(sn[hw][j], ftz(tab[j])), neg(fmul(sn[hw][j + half], ftz(tab[half + j]))));
    else if (j < a.rot) y = fadd(fmul(sn[hw][j], ftz(tab[j - half])), fmul(sn[hw][j - half], ftz(tab[j])));
    else y = sn[hw][j];
    dst[j] = ftz(y);
  }
  if (!isq) {                                  // V goes to the cache as the GEMM wrote it (llm.py:731)
    const int kh = h - a.nh;
    const float* vs = a.v + (uint64_t)r * a.nkv * hd + kh * hd;
    float* vd = a.vc + (((uint64_t)b * a.Tp + t) * a.nkv + kh) * hd;
    for (int j = l; j < hd; j += 16) vd[j] = vs[j];
  }
}

// ------------------------------------------------------------------------------- attention
// One block per (sequence, KV head), serving the G = nh / nkv query heads that share it: FDOT NT of
// each head's n query rows against the sequence's K cache rows 0 .. nk-1 (nk = pad16(t0 + n), the
// rows beyond the tokens written are zeros), the causal softmax of each row over its first
// t0 + 1 + m keys, FDOT NN against the V cache in key order (llm.py:735-746; numerics.py:362-371,
// 393-409). K and V are staged in shared memory in tiles of up to kTile keys (all threads load,
// many 16-byte loads in flight); the per-output FDOT NN chain carries its accumulator across tiles.
constexpr int kAttnThreads = 256;
constexpr int kMaxRows = 16;                 // G * n query rows per block
// K / V rows in shared memory are padded by 4 floats: a warp's 32 threads read 32 different rows
// at the same column, and the padding puts each 16-byte access of a phase in its own bank group.
// FUSED: the block first runs k_qk_rope's work for its rows - the G query heads into shared
// memory, the kv head's K row (normalised, rotated) and V row into the caches - and ends with the
// ROW_QUANT of the attention output rows (k_quant_cl's steps): each block's absmax per token row,
// the order-free max over the cluster's blocks (the sequence's kv heads) through distributed
// shared memory, then each block quantises its own columns and rank 0 writes the row scales.
template <int HD, bool FUSED>
__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnArgs a, int tile, AttnQuantArgs f) {
  griddep_launch();
  griddep_wait();
  constexpr int LD = HD + 4;
  extern __shared__ float4 smem4[];
  const int n = a.n, G = a.nh / a.nkv, R = G * n;
  float* sq = reinterpret_cast<float*>(smem4);   // [R][HD] query rows (flushed)
  float* sp = sq + R * HD;                        // [R][kT] scores, then probabilities
  float* skv = sp + R * kT;                       // [tile][LD] K or V rows
  __shared__ float srow[2][kMaxRows];             // per row: max, then 1 / sum
  const int b = blockIdx.x / a.nkv, kvh = blockIdx.x - b * a.nkv;
  const int t0 = a.pos[b];
  const int nk = ((t0 + n) + 15) / 16 * 16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if constexpr (FUSED) {
    // one half-warp per (query head, row) or (kv head, row); the K / V tile area is free yet and
    // holds each half-warp's normalised row. Dead half-warps still join the shuffles.
    const QkRopeArgs& q = f.r;
    const int hw = tid >> 4, l = tid & 15;
    float* sn = skv + hw * HD;
    const int items = (G + 1) * n;
    for (int base = 0; base < items; base += kAttnThreads / 16) {
      const int item = base + hw;
      const bool live = item < items;
      const int it = live ? item : 0;
      const bool isq = it < G * n;
      const int g = isq ? it / n : 0, m = isq ? it - g * n : it - G * n;
      const int r = b * n + m, t = t0 + m;
      const float* src = isq ? q.q + (uint64_t)r * a.nh * HD + (kvh * G + g) * HD : q.k + ((uint64_t)r * a.nkv + kvh) * HD;
      const float* gam = isq ? q.qn : q.kn;
      float v[HD / 16];
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < HD / 16; ++i) {
        v[i] = ftz(src[l + 16 * i]);
        s = fadd_nc(s, fmul(v[i], v[i]));
      }
      s = sum16_fold(canon(s));
      const float rs = rsqrt_f(fadd(fmul(s, recip_f(i2f(HD))), q.eps));
#pragma unroll
      for (int i = 0; i < HD / 16; ++i) sn[l + 16 * i] = ftz(fmul(fmul(v[i], rs), gam[l + 16 * i]));
      __syncwarp();
      if (live) {
        const float* tab = q.tab + (uint64_t)t * q.rot;
        const int half = q.rot / 2;
        float* dst = isq ? sq + (g * n + m) * HD : q.kc + (((uint64_t)b * a.Tp + t) * a.nkv + kvh) * HD;
        for (int j = l; j < HD; j += 16) {
          float y;
          if (j < half) y = fadd(fmul(sn[j], ftz(tab[j])), neg(fmul(sn[j + half], ftz(tab[half + j]))));
          else if (j < q.rot) y = fadd(fmul(sn[j], ftz(tab[j - half])), fmul(sn[j - half], ftz(tab[j])));
          else y = sn[j];
          dst[j] = ftz(y);
        }
        if (!isq) {                                // V goes to the cache as the GEMM wrote it
          const float* vs = q.v + ((uint64_t)r * a.nkv + kvh) * HD;
          float* vd = q.vc + (((uint64_t)b * a.Tp + t) * a.nkv + kvh) * HD;
          for (int j = l; j < HD; j += 16) vd[j] = vs[j];
        }
      }
      __syncwarp();
    }
    __threadfence_block();                         // the cache rows before the tiles read them
  } else {
    for (int i = tid; i < R * HD; i += kAttnThreads) {
      const int r = i / HD, d = i - r * HD, g = r / n, m = r - g * n;
      sq[i] = ftz(a.qr[((uint64_t)(b * n + m) * a.nh + kvh * G + g) * HD + d]);
    }
  }
  const uint64_t kstride = (uint64_t)a.nkv * HD;
  const float* K = a.kc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  const float* V = a.vc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  auto stage = [&](const float* src, int j0, int tk) {
    __syncthreads();
    for (int i = tid; i < tk * (HD / 4); i += kAttnThreads) {
      const int j = i / (HD / 4), d4 = i - j * (HD / 4);
      cp16(skv + j * LD + 4 * d4, src + (uint64_t)(j0 + j) * kstride + 4 * d4);
    }
    cp_wait_all();
    __syncthreads();
  };
  // scores: one thread per (row, key) runs the 16 lane chains of sum16 (element d to chain d mod 16,
  // in d order) and their pairwise fold itself
  for (int j0 = 0; j0 < nk; j0 += tile) {
    const int tk = min(tile, nk - j0);
    stage(K, j0, tk);
    for (int p = tid; p < R * tk; p += kAttnThreads) {
      const int r = p / tk, j = p - r * tk;
      const float* qr = sq + r * HD;
      const float* kr = skv + j * LD;
      float c[16];
#pragma unroll
      for (int l = 0; l < 16; ++l) c[l] = 0.0f;
#pragma unroll
      for (int d = 0; d < HD; d += 16) {
#pragma unroll
        for (int l4 = 0; l4 < 4; ++l4) {
          const float4 qv = *reinterpret_cast<const float4*>(qr + d + 4 * l4);
          const float4 kv = *reinterpret_cast<const float4*>(kr + d + 4 * l4);
          c[4 * l4 + 0] = fadd_nc(c[4 * l4 + 0], fmul_ff(qv.x, kv.x));
          c[4 * l4 + 1] = fadd_nc(c[4 * l4 + 1], fmul_ff(qv.y, kv.y));
          c[4 * l4 + 2] = fadd_nc(c[4 * l4 + 2], fmul_ff(qv.z, kv.z));
          c[4 * l4 + 3] = fadd_nc(c[4 * l4 + 3], fmul_ff(qv.w, kv.w));
        }
      }
#pragma unroll
      for (int w = 1; w < 16; w *= 2)
#pragma unroll
        for (int l = 0; l < 16; l += 2 * w) c[l] = fadd_nc(c[l], c[l + w]);
      sp[r * kT + j0 + j] = ftz(canon(c[0]));
    }
  }
  __syncthreads();
  // causal softmax (numerics.py:362-371): row maxima, exps over the block, ordered sums, scaling
  for (int r = warp; r < R; r += kAttnThreads / 32) {
    const int valid = min(nk, t0 + 1 + r % n);
    float mx = bf(0xFF800000u);
    for (int j = lane; j < valid; j += 32) mx = fmax_c(mx, sp[r * kT + j]);
    mx = warp_max(mx);
    if (lane == 0) srow[0][r] = mx;
  }
  __syncthreads();
  for (int p = tid; p < R * nk; p += kAttnThreads) {
    const int r = p / nk, j = p - r * nk;
    const int valid = min(nk, t0 + 1 + r % n);
    sp[r * kT + j] = j < valid ? exp_f(fadd(sp[r * kT + j], neg(srow[0][r]))) : 0.0f;
  }
  __syncthreads();
  for (int r = warp; r < R; r += kAttnThreads / 32) {
    float acc = 0.0f;                                     // lanes 16..31 repeat lanes 0..15
    for (int j = lane & 15; j < nk; j += 16) acc = fadd_nc(acc, sp[r * kT + j]);
    const float rinv = recip_f(sum16_fold(canon(acc)));
    if (lane == 0) srow[1][r] = rinv;
  }
  __syncthreads();
  for (int p = tid; p < R * nk; p += kAttnThreads) {
    const int r = p / nk, j = p - r * nk;
    sp[r * kT + j] = ftz(fmul(sp[r * kT + j], srow[1][r]));
  }
  // FDOT NN: out[r][d] = k-order chain over the nk keys, V staged tile by tile
  constexpr int kPer = (kMaxRows * HD + kAttnThreads - 1) / kAttnThreads;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
  for (int j0 = 0; j0 < nk; j0 += tile) {
    const int tk = min(tile, nk - j0);
    stage(V, j0, tk);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = tid + i * kAttnThreads;
      if (o < R * HD) {
        const int r = o / HD, d = o - r * HD;
        const float* pr = sp + r * kT + j0;
        float v = acc[i];
#pragma unroll 8
        for (int j = 0; j < tk; ++j) v = fadd_nc(v, fmul_ff(pr[j], skv[j * LD + d]));
        acc[i] = v;
      }
    }
  }
  if constexpr (!FUSED) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = tid + i * kAttnThreads;
      if (o < R * HD) {
        const int r = o / HD, d = o - r * HD, g = r / n, m = r - g * n;
        a.att[((uint64_t)(b * n + m) * a.nh + kvh * G + g) * HD + d] = ftz(canon(acc[i]));
      }
    }
  } else {
    __shared__ float red[33];
    __shared__ float s_amax[kMaxRows];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = ftz(canon(acc[i]));   // the values the att rows held
    for (int m = 0; m < n; ++m) {
      float mx = 0.0f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int o = tid + i * kAttnThreads;
        if (o < R * HD && (o / HD) % n == m) mx = fmax_c(mx, fabs_c(acc[i]));
      }
      mx = block_max(mx, red);
      if (tid == 0) s_amax[m] = mx;
    }
    __shared__ float s_inv[kMaxRows];
    cluster_sync();
    if (tid < n) {                                  // thread m: row m's max over the cluster
      const int m = tid;
      const uint32_t crank = cluster_rank();
      float mx = s_amax[m];
      for (int p = 0; p < a.nkv; ++p)
        if (p != (int)crank) mx = fmax_c(mx, __int_as_float(dsmem_ld_s32(smem_u32(&s_amax[m]), p)));
      s_inv[m] = fmul(127.0f, recip_f(mx));
      if (crank == 0) f.qs[b * n + m] = ftz(fmul(mx, bf(0x3C010204u)));
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = tid + i * kAttnThreads;
      if (o < R * HD) {
        const int r = o / HD, d = o - r * HD, g = r / n, m = r - g * n;
        f.q8[(uint64_t)(b * n + m) * f.ldq + (kvh * G + g) * HD + d] = q8(acc[i], s_inv[m]);
      }
    }
    cluster_sync();                                 // the peers have read s_amax
  }
}

template <int HD, bool FUSED>
static cudaError_t attention_hd(const AttnArgs& a, const AttnQuantArgs& f, int batch, cudaStream_t st) {
  const int R = (a.nh / a.nkv) * a.n;
  const int fixed = (R * HD + R * kT) * 4;
  // K / V tiles of about 40 KB: several blocks share an SM (all (sequence, kv head) blocks of a
  // batch of 64 in one wave) instead of one block streaming all keys at once
  const int tile = std::min(kT, (40 * 1024) / ((HD + 4) * 4)) / 16 * 16;
  if (tile < 16) return cudaErrorInvalidValue;                // (the fused prologue needs 16 rows)
  const int smem = fixed + tile * (HD + 4) * 4;
  cudaError_t e = cudaFuncSetAttribute(k_attention<HD, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_ex(k_attention<HD, FUSED>, dim3(batch * a.nkv), dim3(kAttnThreads), smem, st, FUSED ? a.nkv : 1, a,
                   tile, f);
}

// ------------------------------------------------------------------------------- greedy pick
// np.argmax of each sequence's logits: the first maximum; the first NaN wins over numbers. A row
// is spread over a cluster of kPickCluster CTAs (every SM busy at batch 64): CTA c scans a
// contiguous slice with 16-byte loads, each thread keeping four candidates (one per vector lane)
// so four independent compare chains overlap the loads; candidates combine under a rule that is
// order-free (NaN first, then the larger value, then the smaller index), per warp by shuffles, per
// CTA in shared memory, and across the cluster through distributed shared memory.
constexpr int kPickCluster = 8, kPickThreads = 256;

struct Pick {
  float v;
  int i;       // -1: no element yet
  int nan;
};
// elements of one chain arrive in increasing index order, so a tie keeps the earlier one
__device__ __forceinline__ void pick_step(Pick& p, float v, int j) {
  const int vn = is_nan(v);
  const bool take = (p.i < 0) | (vn & !p.nan) | (!p.nan & !vn & (v > p.v));
  p.v = take ? v : p.v;
  p.i = take ? j : p.i;
  p.nan = take ? vn : p.nan;
}
__device__ __forceinline__ Pick pick_comb(Pick a, Pick b) {
  bool take_b;
  if (b.i < 0) take_b = false;
  else if (a.i < 0) take_b = true;
  else if (a.nan != b.nan) take_b = b.nan;
  else if (a.nan) take_b = b.i < a.i;
  else take_b = b.v > a.v || (b.v == a.v && b.i < a.i);
  return take_b ? b : a;
}
__device__ __forceinline__ Pick pick_shfl(Pick p, int o) {
  Pick q;
  q.v = __shfl_xor_sync(0xFFFFFFFFu, p.v, o);
  q.i = __shfl_xor_sync(0xFFFFFFFFu, p.i, o);
  q.nan = __shfl_xor_sync(0xFFFFFFFFu, p.nan, o);
  return q;
}

__global__ void __launch_bounds__(kPickThreads) k_argmax(const float* logits, int vocab, int* tok_out, int tok_stride) {
  griddep_launch();
  griddep_wait();
  __shared__ Pick s_warp[kPickThreads / 32];
  __shared__ int s_cand[3];                      // this CTA's candidate: value bits, index, nan
  const int b = blockIdx.x / kPickCluster, c = (int)cluster_rank();
  const int S = ((vocab + kPickCluster - 1) / kPickCluster + 3) / 4 * 4;
  const int lo = min(vocab, c * S), hi = min(vocab, lo + S);
  const float* row = logits + (uint64_t)b * vocab;
  Pick p[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) p[u] = Pick{0.0f, -1, 0};
  if ((vocab & 3) == 0 && ((uintptr_t)logits & 15) == 0) {
    // lo and hi are multiples of 4: vectors only, two in flight per thread
    const float4* r4 = reinterpret_cast<const float4*>(row);
    int j4 = lo / 4 + threadIdx.x;
    const int e4 = hi / 4;
    for (; j4 + kPickThreads < e4; j4 += 2 * kPickThreads) {
      const float4 x = __ldg(r4 + j4), y = __ldg(r4 + j4 + kPickThreads);
      pick_step(p[0], x.x, 4 * j4);
      pick_step(p[1], x.y, 4 * j4 + 1);
      pick_step(p[2], x.z, 4 * j4 + 2);
      pick_step(p[3], x.w, 4 * j4 + 3);
      const int k4 = j4 + kPickThreads;
      pick_step(p[0], y.x, 4 * k4);
      pick_step(p[1], y.y, 4 * k4 + 1);
      pick_step(p[2], y.z, 4 * k4 + 2);
      pick_step(p[3], y.w, 4 * k4 + 3);
    }
    if (j4 < e4) {
      const float4 x = __ldg(r4 + j4);
      pick_step(p[0], x.x, 4 * j4);
      pick_step(p[1], x.y, 4 * j4 + 1);
      pick_step(p[2], x.z, 4 * j4 + 2);
      pick_step(p[3], x.w, 4 * j4 + 3);
    }
  } else {
    for (int j = lo + threadIdx.x; j < hi; j += kPickThreads) pick_step(p[0], row[j], j);
  }
  Pick m = pick_comb(pick_comb(p[0], p[1]), pick_comb(p[2], p[3]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = pick_comb(m, pick_shfl(m, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_warp[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    Pick t = s_warp[0];
#pragma unroll
    for (int w = 1; w < kPickThreads / 32; ++w) t = pick_comb(t, s_warp[w]);
    s_cand[0] = __float_as_int(t.v);
    s_cand[1] = t.i;
    s_cand[2] = t.nan;
  }
  cluster_sync();
  if (c == 0 && threadIdx.x == 0) {
    Pick t{__int_as_float(s_cand[0]), s_cand[1], s_cand[2]};
    for (int r = 1; r < kPickCluster; ++r) {
      const Pick u{__int_as_float(dsmem_ld_s32(smem_u32(&s_cand[0]), r)), dsmem_ld_s32(smem_u32(&s_cand[1]), r),
                   dsmem_ld_s32(smem_u32(&s_cand[2]), r)};
      t = pick_comb(t, u);
    }
    tok_out[b * tok_stride] = t.i;
  }
  cluster_sync();                                 // the peers' candidates have been read
}

__global__ void k_advance(int* pos, int n, int batch) {
  griddep_wait();
  for (int b = threadIdx.x; b < batch; b += blockDim.x) pos[b] += n;
}

}  // namespace

// --------------------------------------------------------------------------------- launchers
cudaError_t eng_embed(const float* E, const int* tok, float* x, int H, int scale_on, float scale, int rows, cudaStream_t st) {
  cudaError_t e = launch_ex(k_embed, dim3(rows), dim3(256), 0, st, 1, E, tok, x, H, scale_on, scale, rows);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
cudaError_t eng_norm_quant(const NormQuantArgs& a, cudaStream_t st) {
  const int smem = 5 * a.H * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_norm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e2 = launch_ex(k_norm_quant, dim3(a.rows), dim3(256), smem, st, 1, a);
  if (e2 != cudaSuccess) return e2;
  return cudaGetLastError();
}
cudaError_t eng_quant(const float* x, int ldx, int N, int8_t* q, int ldq, float* qs, int rows, cudaStream_t st) {
  if (N % 4 || ldx % 4 || (uintptr_t)x % 16) return cudaErrorInvalidValue;
  return launch_quant_cl(k_quant_cl<0, false>, x, nullptr, ldx, N, 0, q, ldq, qs, rows, st);
}
cudaError_t eng_quant_gated(const float* gate, const float* up, int ld, int N, int act, int8_t* q, int ldq, float* qs,
                            int rows, cudaStream_t st) {
  if (act == 4) return launch_quant_cl(k_quant_cl<4, true>, gate, up, ld, N, act, q, ldq, qs, rows, st);
  if (act == 3) return launch_quant_cl(k_quant_cl<3, true>, gate, up, ld, N, act, q, ldq, qs, rows, st);
  return launch_quant_cl(k_quant_cl<-1, true>, gate, up, ld, N, act, q, ldq, qs, rows, st);
}
template <int MB, int KU>
static cudaError_t gemv_mk(const EngGemvArgs& g, cudaStream_t st) {
  const int ncols = g.mode == kEpiGated ? g.seg[0].n : g.ncols;
  const int blocks = std::min((ncols + 7) / 8, 148 * 4);
  cudaError_t e = launch_ex(k_eng_gemv<MB, KU>, dim3(blocks, (g.M + MB - 1) / MB), dim3(256), 0, st, 1, g);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
template <int MB>
static cudaError_t gemv_m(const EngGemvArgs& g, cudaStream_t st) {
  if (g.K <= 1024) return gemv_mk<MB, 2>(g, st);
  if (g.K <= 2048) return gemv_mk<MB, 4>(g, st);
  if (g.K <= 4096) return gemv_mk<MB, 8>(g, st);
  if constexpr (MB <= 4) return gemv_mk<MB, 14>(g, st);
  return cudaErrorInvalidValue;
}
template <int KU>
static cudaError_t gemm_tl(const EngGemvArgs& g, cudaStream_t st) {
  const int ncols = g.mode == kEpiGated ? g.seg[0].n : g.ncols;
  const int smem = 32 * (g.K + 16);
  cudaError_t e = cudaFuncSetAttribute(k_eng_gemm_tl<KU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int yb = (g.M + 31) / 32;
  const int blocks = std::min((ncols + 3) / 4, std::max(1, 148 * 8 / yb));
  e = launch_ex(k_eng_gemm_tl<KU>, dim3(blocks, yb), dim3(128), smem, st, 1, g);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t eng_gemv(const EngGemvArgs& g, cudaStream_t st) {
  if (g.M >= mma_min_rows() && mma_engine_ok(g)) return eng_gemm_mma(g, st);
  if (g.K > 14 * 512 || g.K % 16) return cudaErrorInvalidValue;
  if (g.M > 8) {
    if (g.K <= 1024) return gemm_tl<2>(g, st);
    if (g.K <= 2048) return gemm_tl<4>(g, st);
    if (g.K <= 4096) return gemm_tl<8>(g, st);
    return gemm_tl<14>(g, st);
  }
  if (g.M == 1) return gemv_m<1>(g, st);
  if (g.M == 2) return gemv_m<2>(g, st);
  if (g.M <= 4 || g.K > 4096) return gemv_m<4>(g, st);   // 8 rows of K > 4096 exceed static shared memory
  return gemv_m<8>(g, st);
}
cudaError_t eng_qk_rope(const QkRopeArgs& a, cudaStream_t st) {
  const int items = a.rows * (a.nh + a.nkv);
  cudaError_t e = launch_ex(k_qk_rope, dim3((items + 7) / 8), dim3(128), 0, st, 1, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
cudaError_t eng_attention(const AttnArgs& a, int batch, cudaStream_t st) {
  const int R = (a.nh / a.nkv) * a.n;
  if (a.nh % a.nkv || R > kMaxRows) return cudaErrorInvalidValue;
  const AttnQuantArgs f{};
  switch (a.hd) {
    case 64: return attention_hd<64, false>(a, f, batch, st);
    case 128: return attention_hd<128, false>(a, f, batch, st);
    case 256: return attention_hd<256, false>(a, f, batch, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t eng_attention_quant(const AttnArgs& a, const AttnQuantArgs& f, int batch, cudaStream_t st) {
  const int R = (a.nh / a.nkv) * a.n;
  if (a.nh % a.nkv || R > kMaxRows || a.nkv > 8 || a.n > kMaxRows || f.r.hd != a.hd || f.r.rot > a.hd ||
      f.r.rot % 2)
    return cudaErrorInvalidValue;
  switch (a.hd) {
    case 64: return attention_hd<64, true>(a, f, batch, st);
    case 128: return attention_hd<128, true>(a, f, batch, st);
    case 256: return attention_hd<256, true>(a, f, batch, st);
    default: return cudaErrorInvalidValue;
  }
}
cudaError_t eng_argmax(const float* logits, int vocab, int batch, int* tok_out, int tok_stride, cudaStream_t st) {
  cudaError_t e = launch_ex(k_argmax, dim3(batch * kPickCluster), dim3(kPickThreads), 0, st, kPickCluster, logits,
                            vocab, tok_out, tok_stride);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
cudaError_t eng_advance(int* pos, int n, int batch, cudaStream_t st) {
  cudaError_t e = launch_ex(k_advance, dim3(1), dim3(256), 0, st, 1, pos, n, batch);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace tc
