// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8) for M > 1 token rows:
// the prefill / batched-decode contraction of golden.py:326-349 and of the decode engine.
//
// Roles in a 128-thread CTA: thread 0 streams 128-byte K slices of a 128-row weight tile (UMMA
// operand A) and of the token tile (operand B, NT rows) into a ring of shared-memory stages with
// TMA (128-byte swizzle, zero fill past every edge); thread 32 issues 4 MMAs of K = 32 per stage
// into int32 accumulators in TMEM (lane = weight row, column = token) and releases each stage with
// tcgen05.commit; then all four warps read the accumulators back (warp w: lanes 32w..32w+31) and
// run the caller's exact fp32 epilogue. int32 sums are exact in any order (|acc| < 2^31 for every
// legal K), so tiling and split-K change nothing in the result.
//
// Split-K: a tile's K slices are shared by the `split` CTAs of a thread-block cluster. Each CTA
// writes its int32 partial tile into its own shared memory; after a cluster barrier CTA r sums
// rows [r*128/split, (r+1)*128/split) over all peers through distributed shared memory and runs
// the epilogue for them. No global workspace, so concurrent launches never share state.
//
// Two accumulators per tile: the gated MLP (gate rows -> acc 0, up rows -> acc 1 from one staged
// token slice) and the K-split linear (first K block -> acc 0, second -> acc 1).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "engine.h"
#include "fp32.cuh"
#include "gemm_epi.cuh"
#include "mma.h"
#include "ops.h"
#include "umma.cuh"

namespace tc {

namespace {
constexpr int kRows = 128;          // weight rows per tile (UMMA M)
constexpr int kSlice = 128;         // K bytes per stage (one swizzle row)
constexpr int kThreads = 128;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 200 * 1024;
constexpr int kSmemPerSM = 228 * 1024;     // shared memory of one SM (1 KB of it reserved per CTA)

struct MmaMaps {
  CUtensorMap x;                    // token rows [M, K] int8
  CUtensorMap w[2 * kMaxSegs];      // segment s: w[2s] first K block, w[2s+1] second K block
};

struct MmaShape {
  int M, NT, ntt;                   // token rows, token tile (multiple of 16, <= 256), token tiles
  int nseg, tile0[kMaxSegs + 1];    // row tiles of segment s: [tile0[s], tile0[s+1])
  int nrow[kMaxSegs];
  int nkb1, nkb2, kb;               // K slices of the two K blocks; kb = first token column of block 2
  int gated, nacc, split, stages;
  int* err;
};

// The decode engine's epilogue (k_eng_gemv's, restated per element): acc0 is the (first K block's)
// dot of segment s's row c with token row m; acc1 the second K block's (kEpiKSplit) or the up
// row's (kEpiGated).
struct EngEpi {
  EngGemvArgs g;
  __device__ __forceinline__ void operator()(int s, int c, int m, int acc0, int acc1) const {
    const float sr = g.srow[m];
    auto ep = [&](int a, const EngSeg& sg) { return fmul(fmul(i2f(a), sr), sg.scale[c]); };
    if (g.mode == kEpiGated) {
      const float yg = ftz(act_fn(ep(acc0, g.seg[0]), g.act));
      const float yu = ep(acc1, g.seg[1]);
      g.seg[0].out[(uint64_t)m * g.seg[0].ldo + c] = ftz(fmul(yg, yu));
      return;
    }
    const EngSeg& sg = g.seg[s];
    float y = g.mode == kEpiKSplit ? fadd(ftz(ep(acc0, sg)), ftz(ep(acc1, sg))) : ep(acc0 + acc1, sg);
    if (g.res) y = fadd(g.res[(uint64_t)m * g.ldres + sg.n0 + c], y);
    sg.out[(uint64_t)m * sg.ldo + c] = ftz(y);
  }
};

// The descriptor path's epilogue (one segment, one K block).
struct MachEpi {
  GemmArgs g;
  __device__ __forceinline__ void operator()(int, int c, int m, int acc0, int acc1) const {
    gemm_epilogue(g, m, c, acc0 + acc1);
  }
};

template <class Epi>
__global__ void __launch_bounds__(kThreads, 1) k_mma_i8(const __grid_constant__ MmaMaps maps, const MmaShape sh,
                                                        const Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kMaxStages], bar_empty[kMaxStages], bar_acc;
  __shared__ uint32_t s_tmem;
  // the swizzled tiles want 1024-byte aligned shared addresses
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = sh.split;
  const int crank = split > 1 ? (int)cluster_rank() : 0;
  const int item = blockIdx.x / split;
  const int tt = item % sh.ntt, rt = item / sh.ntt;
  int s = 0;
  while (s + 1 < sh.nseg && rt >= sh.tile0[s + 1]) ++s;
  const int row0 = (rt - sh.tile0[s]) * kRows;
  const int tok0 = tt * sh.NT;
  const int NT = sh.NT;
  const int nkb = sh.nkb1 + sh.nkb2;
  const int per = (nkb + split - 1) / split;
  const int k_lo = min(nkb, crank * per), k_hi = min(nkb, k_lo + per);
  const int nk = k_hi - k_lo;
  const int nacc = sh.nacc;
  const bool used0 = nk > 0 && (sh.gated || k_lo < sh.nkb1);
  const bool used1 = nk > 0 && (sh.gated || k_hi > sh.nkb1);
  const uint32_t a_bytes = kRows * kSlice, b_bytes = (uint32_t)NT * kSlice;
  const int na = sh.gated ? 2 : 1;
  const uint32_t stage_bytes = na * a_bytes + b_bytes;
  const int S = sh.stages;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(nacc * NT)) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], 1);
    }
    mbar_init(&bar_acc, 1);
    mbar_fence_init();
    tma_prefetch_desc(&maps.x);
  }
  if (warp == 0) tmem_alloc(&s_tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (threadIdx.x == 0) {
    // producer: K slice i of this CTA's range into stage i % S
    for (int i = 0; i < nk; ++i) {
      const int st = i % S;
      const uint32_t use = i / S;
      if (i >= S && !mbar_wait(&bar_empty[st], (use & 1) ^ 1, sh.err, 1)) break;
      uint8_t* sa = smem + st * stage_bytes;
      const int k = k_lo + i;
      int xk;
      mbar_expect_tx(&bar_full[st], stage_bytes);
      if (sh.gated) {
        tma_load_2d(sa, &maps.w[0], k * kSlice, row0, &bar_full[st]);
        tma_load_2d(sa + a_bytes, &maps.w[2], k * kSlice, row0, &bar_full[st]);
        xk = k * kSlice;
      } else if (k < sh.nkb1) {
        tma_load_2d(sa, &maps.w[2 * s], k * kSlice, row0, &bar_full[st]);
        xk = k * kSlice;
      } else {
        tma_load_2d(sa, &maps.w[2 * s + 1], (k - sh.nkb1) * kSlice, row0, &bar_full[st]);
        xk = sh.kb + (k - sh.nkb1) * kSlice;
      }
      tma_load_2d(sa + na * a_bytes, &maps.x, xk, tok0, &bar_full[st]);
    }
  } else if (threadIdx.x == 32 && nk > 0) {
    // MMA issuer
    const uint32_t idesc = idesc_i8(kRows, NT);
    bool first0 = true, first1 = true;
    for (int i = 0; i < nk; ++i) {
      const int st = i % S;
      if (!mbar_wait(&bar_full[st], (i / S) & 1, sh.err, 2)) break;
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + st * stage_bytes);
      const uint32_t sb = sa + na * a_bytes;
      const int k = k_lo + i;
      auto run = [&](uint32_t a_addr, uint32_t d, bool& first) {
#pragma unroll
        for (int kk = 0; kk < kSlice / 32; ++kk)
          mma_i8(d, sdesc_k128(a_addr + 32 * kk), sdesc_k128(sb + 32 * kk), idesc, (first && kk == 0) ? 0u : 1u);
        first = false;
      };
      if (sh.gated) {
        run(sa, tmem, first0);
        run(sa + a_bytes, tmem + NT, first1);
      } else if (k < sh.nkb1) {
        run(sa, tmem, first0);
      } else {
        run(sa, tmem + NT, first1);
      }
      mma_commit(&bar_empty[st]);
    }
    mma_commit(&bar_acc);
  }
  __syncwarp();
  bool ok = true;
  if (nk > 0) ok = mbar_wait(&bar_acc, 0, sh.err, 3);
  if (threadIdx.x == 0 && !ok) {   // after a timeout: wait (bounded) for copies still in flight
    for (int i = max(0, nk - S); i < nk; ++i) mbar_wait(&bar_full[i % S], (i / S) & 1, nullptr, 0);
  }
  __syncwarp();
  tc_fence_after();
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const int r = warp * 32 + lane;               // this thread's TMEM lane = weight row in the tile
  const int nrow = sh.nrow[s];

  if (split == 1) {
    const int c = row0 + r;
    for (int j0 = 0; j0 < NT; j0 += 16) {
      uint32_t v0[16], v1[16];
      tmem_ld16(trow + j0, v0);
      if (nacc == 2) tmem_ld16(trow + NT + j0, v1);
      tmem_wait_ld();
      if (ok && c < nrow) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = tok0 + j0 + j;
          if (m < sh.M) epi(s, c, m, used0 ? (int)v0[j] : 0, (nacc == 2 && used1) ? (int)v1[j] : 0);
        }
      }
    }
  } else {
    // The partial tile goes to shared memory (P[a][token][row], int32, in the drained stages) and
    // the TMEM columns are freed before the first cluster barrier: a CTA that holds TMEM never
    // waits on another CTA, so CTAs of concurrent launches blocked in tcgen05.alloc always
    // progress.
    int* P = reinterpret_cast<int*>(smem);
    for (int j0 = 0; j0 < NT; j0 += 16) {
      uint32_t v0[16], v1[16];
      tmem_ld16(trow + j0, v0);
      if (nacc == 2) tmem_ld16(trow + NT + j0, v1);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        P[(j0 + j) * kRows + r] = used0 ? (int)v0[j] : 0;
        if (nacc == 2) P[(NT + j0 + j) * kRows + r] = used1 ? (int)v1[j] : 0;
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
    cluster_sync();
    const int rs = kRows / split, r0 = crank * rs;
    const uint32_t pbase = smem_u32(P);
    for (int idx = threadIdx.x; idx < rs * NT; idx += kThreads) {
      const int rr = r0 + idx % rs, j = idx / rs;
      const uint32_t off = (uint32_t)(j * kRows + rr) * 4;
      int a0 = 0, a1 = 0;
      for (int p = 0; p < split; ++p) {
        a0 += dsmem_ld_s32(pbase + off, p);
        if (nacc == 2) a1 += dsmem_ld_s32(pbase + NT * kRows * 4 + off, p);
      }
      const int c = row0 + rr, m = tok0 + j;
      if (ok && c < nrow && m < sh.M) epi(s, c, m, a0, a1);
    }
    cluster_sync();      // peers have read this CTA's partials
    return;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ------------------------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// int8 matrix [rows, cols] with row stride ld bytes, boxes of 128 bytes x box_rows rows.
bool make_map(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn || (uintptr_t)ptr % 16 || ld % 16 || cols == 0 || rows == 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld};
  const cuuint32_t box[2] = {(cuuint32_t)kSlice, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Error code of the bounded waits (static device memory: the kernel allocates nothing).
__device__ int g_mma_err;
int* err_flag() {
  static int* p = nullptr;
  if (!p) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_mma_err) == cudaSuccess) p = static_cast<int*>(a);
  }
  return p;
}

// Token tile, split factor, stages and shared memory for a GEMM of `tiles` row tiles.
bool plan(MmaShape& sh, int tiles, int* smem) {
  sh.NT = std::min(256, (sh.M + 15) / 16 * 16);
  sh.ntt = (sh.M + sh.NT - 1) / sh.NT;
  const int nkb = sh.nkb1 + sh.nkb2;
  int split = 1;
  while (split < 8 && tiles * sh.ntt * split * 2 <= 2 * 148 && nkb >= split * 2 * 2) split *= 2;
  if (split > 1 && sh.nacc * sh.NT * kRows * 4 > kSmemBudget) {   // the partial tile must fit
    sh.NT = 128;
    sh.ntt = (sh.M + sh.NT - 1) / sh.NT;
  }
  sh.split = split;
  const int per = (nkb + split - 1) / split;
  const int na = sh.gated ? 2 : 1;
  const int stage = na * kRows * kSlice + sh.NT * kSlice;
  sh.stages = std::max(1, std::min({kMaxStages, per, kSmemBudget / stage}));
  const int part = split > 1 ? sh.nacc * sh.NT * kRows * 4 : 0;
  *smem = std::max(sh.stages * stage, part) + 1024;
  // CTAs that share an SM must fit in its 512 TMEM columns together: a CTA blocked in
  // tcgen05.alloc must never wait on a cluster peer that holds the columns it needs.
  int ncols = 32;
  while (ncols < sh.nacc * sh.NT) ncols <<= 1;
  const int max_res = 512 / ncols;
  *smem = std::max(*smem, kSmemPerSM / (max_res + 1) + 64 - 1024);
  sh.err = err_flag();
  return sh.stages >= 1 && sh.err != nullptr;
}

template <class Epi>
cudaError_t launch(const MmaMaps& maps, const MmaShape& sh, const Epi& epi, int tiles, int smem, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(k_mma_i8<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles * sh.ntt * sh.split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = sh.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_mma_i8<Epi>, maps, sh, epi);
}
}  // namespace

bool mma_engine_ok(const EngGemvArgs& g) {
  if (g.M < 2 || g.K % 16 || g.kb % 16 || (uintptr_t)g.A % 16 || g.lda % 16 || !encode_fn()) return false;
  for (int s = 0; s < g.nseg; ++s) {
    if ((uintptr_t)g.seg[s].W % 16 || (g.kb < g.K && (uintptr_t)g.seg[s].W2 % 16)) return false;
  }
  return true;
}

cudaError_t eng_gemm_mma(const EngGemvArgs& g, cudaStream_t st) {
  MmaMaps maps;
  MmaShape sh{};
  sh.M = g.M;
  sh.gated = g.mode == kEpiGated;
  const bool two = g.kb < g.K;
  if (sh.gated && two) return cudaErrorInvalidValue;
  sh.kb = g.kb;
  sh.nkb1 = (g.kb + kSlice - 1) / kSlice;
  sh.nkb2 = two ? (g.K - g.kb + kSlice - 1) / kSlice : 0;
  sh.nacc = (sh.gated || two) ? 2 : 1;
  const int nseg = sh.gated ? 1 : g.nseg;
  sh.nseg = nseg;
  int tiles = 0;
  for (int s = 0; s < nseg; ++s) {
    sh.tile0[s] = tiles;
    sh.nrow[s] = g.seg[s].n;
    tiles += (g.seg[s].n + kRows - 1) / kRows;
  }
  sh.tile0[nseg] = tiles;
  int smem = 0;
  if (!plan(sh, tiles, &smem)) return cudaErrorInvalidValue;
  if (!make_map(&maps.x, g.A, g.K, g.M, g.lda, sh.NT)) return cudaErrorInvalidValue;
  for (int s = 0; s < g.nseg; ++s) {
    if (!make_map(&maps.w[2 * s], g.seg[s].W, g.kb, g.seg[s].n, g.kb, kRows)) return cudaErrorInvalidValue;
    if (two && !make_map(&maps.w[2 * s + 1], g.seg[s].W2, g.K - g.kb, g.seg[s].n, g.K - g.kb, kRows))
      return cudaErrorInvalidValue;
  }
  return launch(maps, sh, EngEpi{g}, tiles, smem, st);
}

bool mma_machine_ok(const GemmArgs& g) {
  return g.M >= 2 && g.K % 16 == 0 && (uintptr_t)g.A % 16 == 0 && g.lda % 16 == 0 && (uintptr_t)g.W % 16 == 0 &&
         encode_fn() != nullptr;
}

cudaError_t gemm_mma(const GemmArgs& g, cudaStream_t st) {
  MmaMaps maps;
  MmaShape sh{};
  sh.M = g.M;
  sh.kb = g.K;
  sh.nkb1 = (g.K + kSlice - 1) / kSlice;
  sh.nacc = 1;
  sh.nseg = 1;
  const int tiles = (g.N + kRows - 1) / kRows;
  sh.tile0[0] = 0;
  sh.tile0[1] = tiles;
  sh.nrow[0] = g.N;
  int smem = 0;
  if (!plan(sh, tiles, &smem)) return cudaErrorInvalidValue;
  if (!make_map(&maps.x, g.A, g.K, g.M, g.lda, sh.NT)) return cudaErrorInvalidValue;
  if (!make_map(&maps.w[0], g.W, g.K, g.N, g.K, kRows)) return cudaErrorInvalidValue;
  return launch(maps, sh, MachEpi{g}, tiles, smem, st);
}

std::atomic<int> g_min_rows{-1};
int mma_min_rows() {
  int v = g_min_rows.load();
  if (v < 0) {
    const char* e = getenv("TARSCUDA_MMA_MIN_M");
    v = e ? std::max(2, atoi(e)) : 16;
    g_min_rows.store(v);
  }
  return v;
}

int mma_error_code() {
  int* p = err_flag();
  int v = 0;
  if (p) cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  return v;
}

}  // namespace tc

extern "C" int tc_set_mma_min_rows(int32_t rows) {
  const int prev = tc::mma_min_rows();
  tc::g_min_rows.store(rows < 2 ? 2 : rows);
  return prev;
}
