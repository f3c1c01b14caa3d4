// Row ops (golden.py:358-380), the RELU/activation op (351-356), ELT (393-418), ROPE (420-424)
// and FDOT (426-435) for sm_100a, bit-exact to numerics.py.
//
// Reductions keep the contract's order: sum16 = 16 lanes (a half-warp), lane j mod 16, each a
// sequential fadd chain from +0, then the pairwise fold (0+1),(2+3).. done as xor-shuffles 1,2,4,8
// (IEEE addition is commutative, so lane l and lane l^1 compute the same pair sum). max16 uses
// fmax, which is order-free by construction. FDOT NN is the strict k-order chain, one thread per
// output. Elementwise ops are one thread per element: in-place ELT (A or C is the output itself)
// reads an element before the same thread writes it.
#include <cuda_runtime.h>

#include "fp32.cuh"
#include "ops.h"

namespace tc {

namespace {

__device__ __forceinline__ float sum16_fold(float v, unsigned mask = 0xFFFFFFFFu) {
  v = fadd(v, __shfl_xor_sync(mask, v, 1));
  v = fadd(v, __shfl_xor_sync(mask, v, 2));
  v = fadd(v, __shfl_xor_sync(mask, v, 4));
  v = fadd(v, __shfl_xor_sync(mask, v, 8));
  return v;
}
__device__ __forceinline__ float max_fold(float v) {
  v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
  v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
  return v;
}

// Long rows (N > kRowSmem floats): one half-warp per row, loads straight from global memory.
__global__ void __launch_bounds__(128) k_rowop_long(RowArgs a) {
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int m = blockIdx.x * 8 + hw;
  const bool live = m < a.M;            // dead half-warps still join the shuffles
  const int mm = live ? m : 0;
  const uint8_t* x = a.X + (uint64_t)mm * a.lda;
  uint8_t* y = a.Y + (uint64_t)mm * a.ldy;
  const int N = a.N;
  auto X = [&](int j) { return ftz(ld_f32(x + 4 * (uint64_t)j)); };

  if (a.fn == ROW_QUANT) {
    float amax = 0.0f;
    for (int j = l; j < N; j += 16) amax = fmax_c(amax, fabs_c(X(j)));
    amax = max_fold(amax);
    const float inv = fmul(127.0f, recip_f(amax));
    if (live) {
      for (int j = l; j < N; j += 16) y[j] = (uint8_t)q8(X(j), inv);
      if (l == 0) st_u32(a.scale_out + 4 * (uint64_t)m, fb(ftz(fmul(amax, bf(0x3C010204u)))));
    }
    return;
  }
  if (a.fn == ROW_SOFTMAX) {
    const int valid = a.K ? min(N, a.K + m) : N;
    float mx = bf(0xFF800000u);          // -inf: the identity of fmax
    for (int j = l; j < valid; j += 16) mx = fmax_c(mx, X(j));
    mx = max_fold(mx);
    float s = 0.0f;
    for (int j = l; j < N; j += 16) s = fadd(s, j < valid ? exp_f(fadd(X(j), neg(mx))) : 0.0f);
    const float r = recip_f(sum16_fold(s));
    if (live)
      for (int j = l; j < N; j += 16)
        store_out(y, j, fmul(j < valid ? exp_f(fadd(X(j), neg(mx))) : 0.0f, r), a.out, a.out_scale);
    return;
  }
  const float kinv = recip_f(i2f(N));
  float mean = 0.0f;
  if (a.fn == ROW_LAYERNORM) {
    float s = 0.0f;
    for (int j = l; j < N; j += 16) s = fadd(s, X(j));
    mean = fmul(sum16_fold(s), kinv);
  }
  float s = 0.0f;
  for (int j = l; j < N; j += 16) {
    const float v = a.fn == ROW_LAYERNORM ? fadd(X(j), neg(mean)) : X(j);
    s = fadd(s, fmul(v, v));
  }
  s = sum16_fold(s);
  const float rs = rsqrt_f(a.fn == ROW_L2NORM ? fadd(s, a.eps) : fadd(fmul(s, kinv), a.eps));
  if (!live) return;
  for (int j = l; j < N; j += 16) {
    const float v = a.fn == ROW_LAYERNORM ? fadd(X(j), neg(mean)) : X(j);
    float o = fmul(fmul(v, rs), ld_f32(a.gamma + 4 * (uint64_t)j));
    if (a.beta) o = fadd(o, ld_f32(a.beta + 4 * (uint64_t)j));
    store_out(y, j, o, a.out, a.out_scale);
  }
}

constexpr int kRT = 256;                 // threads per row block
constexpr int kRowSmem = 16384;          // rows up to this many floats are staged in shared memory

// Block-wide fmax (order-free) of one value per thread; every thread gets the result.
__device__ __forceinline__ float block_max(float v, float* red) {
  v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, 16));
  v = max_fold(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kRT / 32; ++i) r = fmax_c(r, red[i]);
  return r;
}

// sum16 of v[0..N) in the contract's order: threads 0..15 run the lane chains over shared memory
// (hardware flush-to-zero adds, canonicalised once), then the pairwise fold; broadcast to all.
__device__ __forceinline__ float block_sum16(const float* v, int N, float* red) {
  __syncthreads();
  if (threadIdx.x < 16) {
    float acc = 0.0f;
    for (int j = threadIdx.x; j < N; j += 16) acc = fadd_nc(acc, v[j]);
    acc = sum16_fold(canon(acc), 0x0000FFFFu);
    if (threadIdx.x == 0) red[kRT / 32] = acc;
  }
  __syncthreads();
  return red[kRT / 32];
}

// One block per row: the row (flushed) is staged in shared memory with 16-byte loads when
// aligned; elementwise work is spread over the block, the ordered sums run on 16 threads.
// `sm` holds 2 * a.N floats.
__device__ __forceinline__ void rowop_body(const RowArgs& a, int m, float* sm, float* red) {
  float* sx = sm;                  // the row
  float* sv = sm + a.N;            // per-element terms (x*x, d*d, e)
  const int N = a.N, t = threadIdx.x;
  const uint8_t* x = a.X + (uint64_t)m * a.lda;
  uint8_t* y = a.Y + (uint64_t)m * a.ldy;
  if (((uintptr_t)x & 15) == 0) {
    for (int i = t; i < N / 4; i += kRT) cp16(sx + 4 * i, x + 16 * (uint64_t)i);
    cp_wait_all();
    __syncthreads();
    for (int j = t; j < N; j += kRT) sx[j] = ftz(sx[j]);
  } else {
    for (int j = t; j < N; j += kRT) sx[j] = ftz(ld_f32(x + 4 * (uint64_t)j));
  }
  __syncthreads();
  if (a.fn == ROW_QUANT) {
    float amax = 0.0f;
    for (int j = t; j < N; j += kRT) amax = fmax_c(amax, fabs_c(sx[j]));
    amax = block_max(amax, red);
    const float inv = fmul(127.0f, recip_f(amax));
    if (((uintptr_t)y & 3) == 0) {
      for (int i = t; i < N / 4; i += kRT) {
        const uint32_t b = (uint32_t)(uint8_t)q8(sx[4 * i], inv) | (uint32_t)(uint8_t)q8(sx[4 * i + 1], inv) << 8 |
                           (uint32_t)(uint8_t)q8(sx[4 * i + 2], inv) << 16 | (uint32_t)(uint8_t)q8(sx[4 * i + 3], inv) << 24;
        reinterpret_cast<uint32_t*>(y)[i] = b;
      }
    } else {
      for (int j = t; j < N; j += kRT) y[j] = (uint8_t)q8(sx[j], inv);
    }
    if (t == 0) st_u32(a.scale_out + 4 * (uint64_t)m, fb(ftz(fmul(amax, bf(0x3C010204u)))));
    return;
  }
  if (a.fn == ROW_SOFTMAX) {
    const int valid = a.K ? min(N, a.K + m) : N;
    float mx = bf(0xFF800000u);
    for (int j = t; j < valid; j += kRT) mx = fmax_c(mx, sx[j]);
    mx = block_max(mx, red);
    for (int j = t; j < N; j += kRT) sv[j] = j < valid ? exp_f(fadd(sx[j], neg(mx))) : 0.0f;
    const float r = recip_f(block_sum16(sv, N, red));
    for (int j = t; j < N; j += kRT) store_out(y, j, fmul(sv[j], r), a.out, a.out_scale);
    return;
  }
  const float kinv = recip_f(i2f(N));
  if (a.fn == ROW_LAYERNORM) {
    const float mean = fmul(block_sum16(sx, N, red), kinv);
    __syncthreads();
    for (int j = t; j < N; j += kRT) sx[j] = fadd(sx[j], neg(mean));     // d
  }
  __syncthreads();
  for (int j = t; j < N; j += kRT) sv[j] = fmul(sx[j], sx[j]);
  const float s = block_sum16(sv, N, red);
  const float rs = rsqrt_f(a.fn == ROW_L2NORM ? fadd(s, a.eps) : fadd(fmul(s, kinv), a.eps));
  for (int j = t; j < N; j += kRT) {
    float o = fmul(fmul(sx[j], rs), ld_f32(a.gamma + 4 * (uint64_t)j));
    if (a.beta) o = fadd(o, ld_f32(a.beta + 4 * (uint64_t)j));
    store_out(y, j, o, a.out, a.out_scale);
  }
}

__global__ void __launch_bounds__(kRT) k_rowop(RowArgs a) {
  extern __shared__ float sm[];
  __shared__ float red[kRT / 32 + 1];
  rowop_body(a, blockIdx.x, sm, red);
}

// Independent row ops of one dependency level in one launch: block b runs row b - row0[j] of
// entry j, where row0[j] <= b < row0[j + 1] (a block-uniform search over at most kGroupMax
// entries). Each row is computed exactly as k_rowop computes it.
__global__ void __launch_bounds__(kRT) k_rowop_group(const __grid_constant__ RowGroup grp) {
  extern __shared__ float sm[];
  __shared__ float red[kRT / 32 + 1];
  const int b = blockIdx.x;
  int lo = 0, hi = grp.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (grp.row0[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  rowop_body(grp.a[lo], b - grp.row0[lo], sm, red);
}

// The row of flat element i of an M x N matrix: M and N are 16-bit descriptor fields, so i < 2^32
// and a 32-bit division is exact.
__device__ __forceinline__ int row_of(uint64_t i, int N) { return (int)((uint32_t)i / (uint32_t)N); }

__global__ void k_act(ActArgs a) {
  const uint64_t total = (uint64_t)a.M * a.N;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const int m = row_of(i, a.N), n = (int)((uint32_t)i - (uint32_t)m * (uint32_t)a.N);
    const float v = ld_f32(a.X + (uint64_t)m * a.lda + 4 * (uint64_t)n);
    store_out(a.Y + (uint64_t)m * a.ldy, n, act_fn(v, a.act), a.out, a.out_scale);
  }
}

__global__ void k_elt(EltArgs a) {
  const uint64_t total = (uint64_t)a.M * a.N;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const int m = row_of(i, a.N), n = (int)((uint32_t)i - (uint32_t)m * (uint32_t)a.N);
    const uint8_t* ap = a.A + (uint64_t)m * a.lda;
    float av = a.a_fp16 ? from_fp16(ld_u16(ap + 2 * (uint64_t)n)) : ld_f32(ap + 4 * (uint64_t)n);
    float bv;
    switch (a.bmode) {
      case BM_DENSE: bv = ld_f32(a.B + (uint64_t)m * a.ldb + 4 * (uint64_t)n); break;
      case BM_ROW: bv = ld_f32(a.B + 4 * (uint64_t)n); break;
      case BM_COL: bv = ld_f32(a.B + 4 * (uint64_t)m); break;
      default: bv = ld_f32(a.B); break;
    }
    uint8_t* yrow = a.Y + (uint64_t)m * a.ldy;
    float cv = 0.0f;
    if (a.op == ELT_MULADD)
      cv = a.out == OUT_FP16 ? from_fp16(ld_u16(a.C + (uint64_t)m * a.ldy + 2 * (uint64_t)n))
                             : ld_f32(a.C + (uint64_t)m * a.ldy + 4 * (uint64_t)n);
    av = act_fn(av, a.act);
    float r;
    switch (a.op) {
      case ELT_MUL: r = fmul(av, bv); break;
      case ELT_ADD: r = fadd(av, bv); break;
      case ELT_SUB: r = fadd(av, neg(ftz(bv))); break;
      default: r = fadd(cv, fmul(av, bv)); break;
    }
    store_out(yrow, n, r, a.out, a.out_scale);
  }
}

__global__ void k_rope(RopeArgs a) {
  const uint64_t total = (uint64_t)a.M * a.N;
  const int h = a.R / 2;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const int m = row_of(i, a.N), n = (int)((uint32_t)i - (uint32_t)m * (uint32_t)a.N);
    const uint8_t* x = a.X + (uint64_t)m * a.lda;
    const uint8_t* t = a.tab + (uint64_t)(m / a.G) * 4 * a.R;
    float r;
    if (n < h) {
      const float c = ftz(ld_f32(t + 4 * n)), s = ftz(ld_f32(t + 4 * (h + n)));
      r = fadd(fmul(ld_f32(x + 4 * n), c), neg(fmul(ld_f32(x + 4 * (n + h)), s)));
    } else if (n < a.R) {
      const int i0 = n - h;
      const float c = ftz(ld_f32(t + 4 * i0)), s = ftz(ld_f32(t + 4 * (h + i0)));
      r = fadd(fmul(ld_f32(x + 4 * n), c), fmul(ld_f32(x + 4 * i0), s));
    } else {
      r = ftz(ld_f32(x + 4 * (uint64_t)n));
    }
    store_out(a.Y + (uint64_t)m * a.ldy, n, r, a.out, a.out_scale);
  }
}

// FDOT NT (numerics.py:393-399), tiled: a block computes a 16 x 16 tile of outputs, one per
// thread. The tile's 16 A rows and 16 B rows are staged in shared memory (flushed once) in chunks
// of kFdKC k; each thread runs the 16 lane chains of sum16 (element k to chain k mod 16, in k order,
// each from +0) and their pairwise fold in registers. Products are flushed; sums use the
// flush-to-zero add; a NaN, once made, stays a NaN through every later product and sum, so making
// it canonical once at the end gives the bits of the reference's per-step canonicalisation.
constexpr int kFdT = 16, kFdKC = 256, kFdLD = kFdKC + 4;    // +4: a row's float4 reads in their own banks
__global__ void __launch_bounds__(256) k_fdot_nt(FdotArgs a) {
  __shared__ __align__(16) float sa[kFdT][kFdLD];
  __shared__ __align__(16) float sb[kFdT][kFdLD];
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const int m0 = blockIdx.y * kFdT, n0 = blockIdx.x * kFdT;
  float c[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) c[i] = 0.0f;
  for (int k0 = 0; k0 < a.K; k0 += kFdKC) {
    const int kc = min(kFdKC, a.K - k0);                     // a multiple of 16
    __syncthreads();
    // float4 i of the chunk: row i / 64, k 4 (i % 64); four per thread and matrix
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, r = i >> 6, k = 4 * (i & 63);
      if (k < kc) {
        const int m = m0 + r, n = n0 + r;
        float4 va = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vb = va;
        const uint8_t* ap = a.A + (uint64_t)m * a.lda + 4 * (uint64_t)(k0 + k);
        const uint8_t* bp = a.B + (uint64_t)n * a.ldb + 4 * (uint64_t)(k0 + k);
        if (m < a.M)
          va = a.vec ? *reinterpret_cast<const float4*>(ap)
                     : make_float4(ld_f32(ap), ld_f32(ap + 4), ld_f32(ap + 8), ld_f32(ap + 12));
        if (n < a.N)
          vb = a.vec ? *reinterpret_cast<const float4*>(bp)
                     : make_float4(ld_f32(bp), ld_f32(bp + 4), ld_f32(bp + 8), ld_f32(bp + 12));
        *reinterpret_cast<float4*>(&sa[r][k]) = make_float4(ftz(va.x), ftz(va.y), ftz(va.z), ftz(va.w));
        *reinterpret_cast<float4*>(&sb[r][k]) = make_float4(ftz(vb.x), ftz(vb.y), ftz(vb.z), ftz(vb.w));
      }
    }
    __syncthreads();
    const float* ar = sa[tr];
    const float* br = sb[tc];
    for (int k = 0; k < kc; k += 16) {
#pragma unroll
      for (int l4 = 0; l4 < 4; ++l4) {
        const float4 av = *reinterpret_cast<const float4*>(ar + k + 4 * l4);
        const float4 bv = *reinterpret_cast<const float4*>(br + k + 4 * l4);
        c[4 * l4 + 0] = fadd_nc(c[4 * l4 + 0], fmul_ff(av.x, bv.x));
        c[4 * l4 + 1] = fadd_nc(c[4 * l4 + 1], fmul_ff(av.y, bv.y));
        c[4 * l4 + 2] = fadd_nc(c[4 * l4 + 2], fmul_ff(av.z, bv.z));
        c[4 * l4 + 3] = fadd_nc(c[4 * l4 + 3], fmul_ff(av.w, bv.w));
      }
    }
  }
#pragma unroll
  for (int w = 1; w < 16; w *= 2)                              // lane 2i + lane 2i + 1 into lane i
#pragma unroll
    for (int l = 0; l < 16; l += 2 * w) c[l] = fadd_nc(c[l], c[l + w]);
  const int m = m0 + tr, n = n0 + tc;
  if (m < a.M && n < a.N) store_out(a.Y + (uint64_t)m * a.ldy, n, canon(c[0]), a.out, a.out_scale);
}

// FDOT NN (numerics.py:402-409), tiled: a block computes 4 rows x 64 columns of outputs, one per
// thread, each the sequential chain (((+0 + a0 b0) + a1 b1) + ...) in k order; the 4 A rows and
// kNnK rows of B at a time are staged in shared memory (flushed once). NaN as in k_fdot_nt.
constexpr int kNnR = 4, kNnC = 64, kNnK = 128;
__global__ void __launch_bounds__(256) k_fdot_nn(FdotArgs a) {
  __shared__ __align__(16) float sa[kNnR][kNnK];
  __shared__ __align__(16) float sb[kNnK][kNnC];
  const int tid = threadIdx.x, tr = tid >> 6, tc = tid & 63;
  const int m0 = blockIdx.y * kNnR, n0 = blockIdx.x * kNnC;
  float s = 0.0f;
  for (int k0 = 0; k0 < a.K; k0 += kNnK) {
    const int kc = min(kNnK, a.K - k0);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {                             // the 4 x 128 A tile
      const int i = tid + 256 * j, r = i >> 7, k = i & 127, m = m0 + r;
      sa[r][k] = (k < kc && m < a.M) ? ftz(ld_f32(a.A + (uint64_t)m * a.lda + 4 * (uint64_t)(k0 + k))) : 0.0f;
    }
    if (a.vec && !a.b_fp16 && n0 + kNnC <= a.N) {             // 128 x 64 fp32: eight float4 per thread
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = tid + 256 * j, k = i >> 4, c4 = 4 * (i & 15);
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < kc) v = *reinterpret_cast<const float4*>(a.B + (uint64_t)(k0 + k) * a.ldb + 4 * (uint64_t)(n0 + c4));
        *reinterpret_cast<float4*>(&sb[k][c4]) = make_float4(ftz(v.x), ftz(v.y), ftz(v.z), ftz(v.w));
      }
    } else {
      for (int i = tid; i < kNnK * kNnC; i += 256) {
        const int k = i >> 6, cc = i & 63, n = n0 + cc;
        float v = 0.0f;
        if (k < kc && n < a.N) {
          const uint8_t* bp = a.B + (uint64_t)(k0 + k) * a.ldb;
          v = ftz(a.b_fp16 ? from_fp16(ld_u16(bp + 2 * (uint64_t)n)) : ld_f32(bp + 4 * (uint64_t)n));
        }
        sb[k][cc] = v;
      }
    }
    __syncthreads();
    const float* ar = sa[tr];
#pragma unroll 8
    for (int k = 0; k < kc; ++k) s = fadd_nc(s, fmul_ff(ar[k], sb[k][tc]));
  }
  const int m = m0 + tr, n = n0 + tc;
  if (m < a.M && n < a.N) store_out(a.Y + (uint64_t)m * a.ldy, n, canon(s), a.out, a.out_scale);
}

inline int grid_for(uint64_t total, int threads) {
  const uint64_t b = (total + threads - 1) / threads;
  return (int)std::min<uint64_t>(std::max<uint64_t>(b, 1), 148ull * 32);
}
}  // namespace

cudaError_t launch_rowop(const RowArgs& a, cudaStream_t st) {
  if (a.N > kRowSmem) {
    k_rowop_long<<<(a.M + 7) / 8, 128, 0, st>>>(a);
    return cudaGetLastError();
  }
  const int smem = 2 * a.N * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_rowop, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kRowSmem * 4);
    if (e != cudaSuccess) return e;
  }
  k_rowop<<<a.M, kRT, smem, st>>>(a);
  return cudaGetLastError();
}
bool rowop_groupable(const RowArgs& a) { return a.N <= kRowSmem && a.M > 0; }
cudaError_t launch_rowop_group(const RowGroup& g, cudaStream_t st) {
  const int smem = 2 * g.nmax * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_rowop_group, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kRowSmem * 4);
    if (e != cudaSuccess) return e;
  }
  k_rowop_group<<<g.row0[g.n], kRT, smem, st>>>(g);
  return cudaGetLastError();
}
cudaError_t launch_act(const ActArgs& a, cudaStream_t st) {
  k_act<<<grid_for((uint64_t)a.M * a.N, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_elt(const EltArgs& a, cudaStream_t st) {
  k_elt<<<grid_for((uint64_t)a.M * a.N, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_rope(const RopeArgs& a, cudaStream_t st) {
  k_rope<<<grid_for((uint64_t)a.M * a.N, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_fdot(const FdotArgs& a0, cudaStream_t st) {
  FdotArgs a = a0;
  a.vec = (((uintptr_t)a.A | a.lda | (uintptr_t)a.B | a.ldb) & 15) == 0;
  if (a.nn) {
    k_fdot_nn<<<dim3((a.N + kNnC - 1) / kNnC, (a.M + kNnR - 1) / kNnR), 256, 0, st>>>(a);
  } else {
    k_fdot_nt<<<dim3((a.N + kFdT - 1) / kFdT, (a.M + kFdT - 1) / kFdT), 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace tc
