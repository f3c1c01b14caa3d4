// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8) for M > 1 token rows:
// the prefill / batched-decode contraction of golden.py:326-349 and of the decode engine.
//
// A tile is 128 weight rows (UMMA operand A, M = 128) x NT token rows (operand B, N = NT <= 256);
// its accumulator is int32 in TMEM (lane = weight row, column = token). int32 sums are exact in
// any order (|acc| < 2^31 for every legal K), so tiling and split-K change nothing in the result.
// Warp roles in a 320-thread CTA:
//   warp 0     TMA producer: 128-byte K slices of the weight tile(s) and of the token tile into a
//              ring of shared-memory stages (128-byte swizzle, zero fill past every edge)
//   warp 1     TMEM owner and MMA issuer: 4 MMAs of K = 32 per stage, tcgen05.commit releases
//              the stage; a finished accumulator is committed to the epilogue
//   warps 2-9  epilogue: tcgen05.ld of the accumulator (warp w reads lanes 32(w%4).., warps
//              2-5 the even 16-column chunks, 6-9 the odd ones), the caller's exact fp32
//              epilogue, coalesced stores (consecutive lanes = consecutive output columns)
// Two modes:
//   persistent  CTAs loop over tiles; two TMEM accumulators, so the epilogue of one tile overlaps
//               the loads and MMAs of the next
//   split-K     few tiles: the K slices of one tile are shared by the `split` CTAs of a thread-
//               block cluster. CTA r owns rows [r*128/split, (r+1)*128/split) of the tile; every
//               CTA pushes each owner its partial rows with st.async into a slot of the owner's
//               shared memory (completing on the owner's mbarrier), frees its TMEM, waits for its
//               own slots, sums them and runs the epilogue for its rows. No global workspace, so
//               concurrent launches never share state, and no CTA holds TMEM while it waits on
//               another CTA.
// Two accumulators per tile: the gated MLP (gate rows -> acc 0, up rows -> acc 1 from one staged
// token slice) and the K-split linear (first K block -> acc 0, second -> acc 1).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "../../include/tarscuda.h"
#include "engine.h"
#include "fp32.cuh"
#include "gemm_epi.cuh"
#include "mma.h"
#include "ops.h"
#include "umma.cuh"
#include "pdl.cuh"

namespace tc {

namespace {
constexpr int kRows = 128;          // weight rows per tile (UMMA M)
constexpr int kSlice = 128;         // K bytes per stage (one swizzle row)
constexpr int kEpiWarps = 8;                // two per TMEM lane quarter, alternating 16-column chunks
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 144 * 1024;
constexpr int kSmemPerSM = 228 * 1024;     // shared memory of one SM (1 KB of it reserved per CTA)
constexpr int kSMs = 148;

struct MmaMaps {
  CUtensorMap x;                    // token rows [M, K] int8
  CUtensorMap w[2 * kMaxSegs];      // segment s: w[2s] first K block, w[2s+1] second K block
};

// Phase trace (tc_mma_trace): per CTA, globaltimer stamps of kernel entry, setup done, first TMA
// issued, first stage consumed by the MMA thread, last MMA issued, first accumulator seen by the
// epilogue, epilogue done, exit. Off unless enabled; it changes no work.
constexpr int kTraceCtas = 2048, kTraceStamps = 8;
__device__ unsigned long long g_mma_trace[kTraceCtas * kTraceStamps];
std::atomic<int> g_trace_on{0};     // 0 off, n > 0: trace the n-th tensor-core launch from now on
std::atomic<int> g_trace_count{0};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct MmaShape {
  int M, NT, ntt;                   // token rows, token tile (multiple of 16, <= 256), token tiles
  int nseg, tile0[kMaxSegs + 1];    // row tiles of segment s: [tile0[s], tile0[s+1])
  int nrow[kMaxSegs];
  int nkb1, nkb2, kb;               // K slices of the two K blocks; kb = first token column of block 2
  int gated, nacc, split, stages, items, nbuf, trace;
  int* err;
  uint32_t spin;                    // poll limit of the bounded waits for work
};

// Epilogues. row() holds what depends on the weight row only (scales pre-flushed), tok() the
// per-token factor (the row scale of the token's int8 row; staged flushed in shared memory once
// per tile), put16() 16 consecutive tokens of one weight row: first the 16 values, branch-free
// (the choices that are uniform over the launch - output format, activation, residual, mode -
// are template instances picked outside the loop), then the stores, predicated on the token
// count. A branch per element would split the unrolled loop into blocks whose dependent chains
// (convert, multiply, flush, store) the scheduler could not overlap.
// ep(a, s) = fmul(fmul(i2f(a), sr), s) is computed as canon(ftz(ftz(i2f(a) * sr) * s)): i2f of an
// int is never denormal, sr and s are flushed once, and a NaN stays a NaN through a product, so
// canonicalising once at the end gives the same bits.
__device__ __forceinline__ float ep_fast(int a, float sr, float sc) { return canon(fmul_ff(fmul_ff(i2f(a), sr), sc)); }

// ACT 0-2 without a branch; -1: any code through act_fn_lean
template <int ACT>
__device__ __forceinline__ float act_static(float x, int act) {
  if constexpr (ACT == 3) return gelu_f(x);
  else if constexpr (ACT == 4) return silu_f(x);
  else if constexpr (ACT == 0) {
    x = ftz(x);
    const float r = x > 0.0f ? x : 0.0f;
    const float r6 = r > 6.0f ? 6.0f : r;
    return act == 0 ? x : (act == 1 ? r : r6);
  } else {
    return act_fn_lean(x, act);
  }
}

// The decode engine's epilogue (k_eng_gemv's): acc0 is the (first K block's) dot of segment s's row
// c with a token row; acc1 the second K block's (kEpiKSplit) or the up row's (kEpiGated).
struct EngEpi {
  EngGemvArgs g;
  struct Row {
    float s0, s1;
    float* out;
    uint64_t ldo;
    int col;
  };
  __device__ __forceinline__ Row row(int s, int c) const {
    Row r;
    if (g.mode == kEpiGated) {
      r.s0 = ftz(g.seg[0].scale[c]);
      r.s1 = ftz(g.seg[1].scale[c]);
      r.out = g.seg[0].out + c;
      r.ldo = g.seg[0].ldo;
      r.col = c;
    } else {
      const EngSeg& sg = g.seg[s];
      r.s0 = r.s1 = ftz(sg.scale[c]);
      r.out = sg.out + c;
      r.ldo = sg.ldo;
      r.col = sg.n0 + c;
    }
    return r;
  }
  __device__ __forceinline__ float tok(int m) const { return g.srow[m]; }

  template <int ACT, int N>
  __device__ __forceinline__ void gated(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                        const uint32_t (&v1)[N]) const {
    float y[N];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float yg = ep_fast((int)v0[j], tk[j], r.s0);
      const float yu = ep_fast((int)v1[j], tk[j], r.s1);
      y[j] = ftz(fmul(ftz(act_static<ACT>(yg, g.act)), yu));
    }
    store<N>(r, m0, mc, y);
  }
  template <bool RES, bool KSPLIT, int N>
  __device__ __forceinline__ void plain(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                        const uint32_t (&v1)[N], bool two) const {
    float y[N];
    float pre[N];
    if constexpr (RES) {
      const float* rp = g.res + r.col;
#pragma unroll
      for (int j = 0; j < N; ++j) pre[j] = rp[(uint64_t)(m0 + min(j, mc - 1)) * g.ldres];
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const int a0 = (int)v0[j], a1 = two ? (int)v1[j] : 0;
      float v;
      if constexpr (KSPLIT) v = fadd(ftz(ep_fast(a0, tk[j], r.s0)), ftz(ep_fast(a1, tk[j], r.s0)));
      else v = ep_fast(a0 + a1, tk[j], r.s0);
      if constexpr (RES) v = fadd(pre[j], v);
      y[j] = ftz(v);
    }
    store<N>(r, m0, mc, y);
  }
  template <int N>
  __device__ __forceinline__ void store(const Row& r, int m0, int mc, const float (&y)[N]) const {
    float* o = r.out + (uint64_t)m0 * r.ldo;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < mc) o[(uint64_t)j * r.ldo] = y[j];
  }
  // N consecutive tokens m0.. (mc of them real) of one weight row
  template <int N>
  __device__ __forceinline__ void put(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                      const uint32_t (&v1)[N], bool two) const {
    if (mc <= 0) return;
    if (g.mode == kEpiGated) {
      if (g.act == 4) gated<4, N>(r, tk, m0, mc, v0, v1);
      else if (g.act == 3) gated<3, N>(r, tk, m0, mc, v0, v1);
      else gated<-1, N>(r, tk, m0, mc, v0, v1);
    } else if (g.mode == kEpiKSplit) {
      if (g.res) plain<true, true, N>(r, tk, m0, mc, v0, v1, two);
      else plain<false, true, N>(r, tk, m0, mc, v0, v1, two);
    } else {
      if (g.res) plain<true, false, N>(r, tk, m0, mc, v0, v1, two);
      else plain<false, false, N>(r, tk, m0, mc, v0, v1, two);
    }
  }
};

// The descriptor path's epilogue (gemm_epilogue, golden.py:326-349).
struct MachEpi {
  GemmArgs g;
  struct Row {
    float sc, bias;
    int n;
  };
  __device__ __forceinline__ Row row(int, int c) const {
    Row r;
    r.n = c;
    r.sc = ftz(ld_f32(g.scale + (g.per_channel ? 4 * (uint64_t)c : 0)));
    r.bias = g.bias ? ld_f32(g.bias + 4 * (uint64_t)c) : 0.0f;
    return r;
  }
  __device__ __forceinline__ float tok(int m) const { return g.srow ? ld_f32(g.srow + 4 * (uint64_t)m) : 1.0f; }

  template <int ACT, int OUT, int N>
  __device__ __forceinline__ void run(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                      const uint32_t (&v1)[N], bool two) const {
    const bool srow = g.srow != nullptr, bias = g.bias != nullptr;
    uint32_t bits[N];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float y = i2f((int)v0[j] + (two ? (int)v1[j] : 0));
      const float ys = fmul_ff(y, tk[j]);
      y = srow ? ys : y;
      y = canon(fmul_ff(y, r.sc));
      const float yb = fadd(y, r.bias);
      y = bias ? yb : y;
      y = act_static<ACT>(y, g.act);
      if constexpr (OUT == 0) bits[j] = fb(ftz(y));
      else if constexpr (OUT == 1) bits[j] = to_bf16(y);
      else if constexpr (OUT == 2) bits[j] = (uint8_t)q8(y, g.out_scale);
      else bits[j] = to_fp16(y);
    }
    uint8_t* yrow = g.Y + (uint64_t)m0 * g.ldy;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (j < mc) {
        uint8_t* p = yrow + (uint64_t)j * g.ldy;
        if constexpr (OUT == 0) st_u32(p + 4 * (uint64_t)r.n, bits[j]);
        else if constexpr (OUT == 2) p[r.n] = (uint8_t)bits[j];
        else st_u16(p + 2 * (uint64_t)r.n, (uint16_t)bits[j]);
      }
    }
  }
  template <int ACT, int N>
  __device__ __forceinline__ void run_act(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                          const uint32_t (&v1)[N], bool two) const {
    switch (g.out) {
      case 0: run<ACT, 0, N>(r, tk, m0, mc, v0, v1, two); break;
      case 1: run<ACT, 1, N>(r, tk, m0, mc, v0, v1, two); break;
      case 2: run<ACT, 2, N>(r, tk, m0, mc, v0, v1, two); break;
      default: run<ACT, 3, N>(r, tk, m0, mc, v0, v1, two); break;
    }
  }
  template <int N>
  __device__ __forceinline__ void put(const Row& r, const float* tk, int m0, int mc, const uint32_t (&v0)[N],
                                      const uint32_t (&v1)[N], bool two) const {
    if (mc <= 0) return;
    if (g.act <= 2) run_act<0, N>(r, tk, m0, mc, v0, v1, two);
    else if (g.act == 4 && g.out == 0) run<4, 0, N>(r, tk, m0, mc, v0, v1, two);    // prefill's SiLU gate
    else if (g.act == 3 && g.out == 0) run<3, 0, N>(r, tk, m0, mc, v0, v1, two);    // and GELU gate
    else run_act<-1, N>(r, tk, m0, mc, v0, v1, two);
  }
};

__device__ __forceinline__ bool aborted(const int* flag) { return *(volatile const int*)flag != 0; }

template <class Epi>
__global__ void __launch_bounds__(kThreads, 1) k_mma_i8(const __grid_constant__ MmaMaps maps, const MmaShape sh,
                                                        const Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kMaxStages], bar_empty[kMaxStages], bar_accf[2], bar_acce[2], bar_recv, bar_drain;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ float s_tok[2][256];             // the tile's token factors (double buffered per tile)
  // barrier of the epilogue warps that also ORs a flag over them, so all of them take the same
  // branch after it
  auto epi_sync_or = [](bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(32 * kEpiWarps)
        : "memory");
    return r != 0;
  };
  // the swizzled tiles want 1024-byte aligned shared addresses
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = sh.stages, NT = sh.NT, split = sh.split, nacc = sh.nacc;
  const int crank = split > 1 ? (int)cluster_rank() : 0;
  const int nkb = sh.nkb1 + sh.nkb2;
  const int per = (nkb + split - 1) / split;
  const int k_lo = min(nkb, crank * per), k_hi = min(nkb, k_lo + per);
  const int nk = k_hi - k_lo;
  const bool used0 = nk > 0 && (sh.gated || k_lo < sh.nkb1);
  const bool used1 = nk > 0 && (sh.gated || k_hi > sh.nkb1);
  const int na = sh.gated ? 2 : 1;
  const uint32_t a_bytes = kRows * kSlice;
  const uint32_t stage_bytes = na * a_bytes + (uint32_t)NT * kSlice;
  const uint32_t acc_cols = nacc * NT;
  uint32_t ncols = 32;
  while (ncols < sh.nbuf * acc_cols) ncols <<= 1;
  const int item0 = blockIdx.x / split, istride = gridDim.x / split;
  auto stamp = [&](int k) {
    if (sh.trace && blockIdx.x < kTraceCtas) g_mma_trace[blockIdx.x * kTraceStamps + k] = gtimer();
  };
  if (threadIdx.x == 0) stamp(0);
  auto coords = [&](int item, int& s, int& row0, int& tok0) {
    const int tt = item % sh.ntt, rt = item / sh.ntt;
    s = 0;
    while (s + 1 < sh.nseg && rt >= sh.tile0[s + 1]) ++s;
    row0 = (rt - sh.tile0[s]) * kRows;
    tok0 = tt * NT;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_accf[i], 1);
      mbar_init(&bar_acce[i], kEpiWarps);
    }
    mbar_init(&bar_drain, 1);
    s_abort = 0;
    if (split > 1) {
      // the owner's slots receive (split - 1) peers' partial rows
      mbar_init(&bar_recv, 1);
      mbar_expect_tx(&bar_recv, (uint32_t)((split - 1) * (kRows / split) * NT * 4 * nacc));
    }
    mbar_fence_init();
    tma_prefetch_desc(&maps.x);
    for (int i = 0; i < 2 * sh.nseg; ++i) tma_prefetch_desc(&maps.w[i]);   // descriptors used by this launch
    if (sh.gated) tma_prefetch_desc(&maps.w[2]);
  }
  if (warp == 1) tmem_alloc(&s_tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // split-K: the barriers of every CTA are initialised before any peer pushes into them
  if (split > 1) cluster_arrive_relaxed();
  const int RL = NT + 4;                         // slot row: NT int32 + 16 bytes of padding
  int* R = reinterpret_cast<int*>(smem + S * stage_bytes);   // slots [acc][sender][row][RL]
  if (threadIdx.x == 0) stamp(1);

  uint32_t issued = 0;                           // the producer's count of K slices issued
  if (warp == 0) {
    if (lane == 0 && nk > 0) {
      // producer: K slice q (counted over all items of this CTA) into stage q % S
      auto load_w = [&](int st, int s, int row0, int k) {   // the weight box(es) of K slice k
        uint8_t* sa = smem + st * stage_bytes;
        if (sh.gated) {
          tma_load_2d(sa, &maps.w[0], k * kSlice, row0, &bar_full[st]);
          tma_load_2d(sa + a_bytes, &maps.w[2], k * kSlice, row0, &bar_full[st]);
        } else if (k < sh.nkb1) {
          tma_load_2d(sa, &maps.w[2 * s], k * kSlice, row0, &bar_full[st]);
        } else {
          tma_load_2d(sa, &maps.w[2 * s + 1], (k - sh.nkb1) * kSlice, row0, &bar_full[st]);
        }
      };
      auto load_x = [&](int st, int tok0, int k) {           // the token box of K slice k
        const int xk = k < sh.nkb1 || sh.gated ? k * kSlice : sh.kb + (k - sh.nkb1) * kSlice;
        tma_load_2d(smem + st * stage_bytes + na * a_bytes, &maps.x, xk, tok0, &bar_full[st]);
      };
      // the weights do not depend on the previous kernel: the first stages' weight boxes are
      // in flight before the wait for its outputs (programmatic dependent launch)
      const int pre = min(S, nk);
      {
        int s, row0, tok0;
        coords(item0, s, row0, tok0);
        for (int i = 0; i < pre; ++i) {
          mbar_expect_tx(&bar_full[i], stage_bytes);
          load_w(i, s, row0, k_lo + i);
        }
      }
      griddep_wait();
      uint32_t q = 0, ph = 0;                  // slices issued; stage st = q mod S, ph its phase bit
      int st = 0;
      bool stop = false;
      for (int item = item0; item < sh.items && !stop; item += istride) {
        int s, row0, tok0;
        coords(item, s, row0, tok0);
        for (int i = 0; i < nk; ++i, ++q, st = st + 1 < S ? st + 1 : (ph ^= 1, 0)) {
          const int k = k_lo + i;
          if (q < (uint32_t)pre) {
            load_x(st, tok0, k);
            if (q == 0) stamp(2);
            continue;
          }
          if (!mbar_wait(&bar_empty[st], ph ^ 1, sh.err, 1, sh.spin)) {
            s_abort = 1;
            stop = true;
            break;
          }
          if (aborted(&s_abort)) {
            stop = true;
            break;
          }
          mbar_expect_tx(&bar_full[st], stage_bytes);
          load_w(st, s, row0, k);
          load_x(st, tok0, k);
        }
      }
      issued = q;
    }
  } else if (warp == 1) {
    if (lane == 0 && nk > 0) {
      // MMA issuer
      const uint32_t idesc = idesc_i8(kRows, NT);
      uint32_t q = 0, ph = 0;                  // slices consumed; stage st = q mod S, ph its phase bit
      int st = 0;
      int t = 0;
      bool stop = false;
      for (int item = item0; item < sh.items && !stop; item += istride, ++t) {
        const int buf = sh.nbuf == 2 ? (t & 1) : 0;
        const uint32_t use = sh.nbuf == 2 ? (t >> 1) : t;
        if (use > 0 && !mbar_wait(&bar_acce[buf], (use & 1) ^ 1, sh.err, 2, sh.spin)) {
          s_abort = 1;
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + buf * acc_cols;
        bool first0 = true, first1 = true;
        for (int i = 0; i < nk; ++i, ++q, st = st + 1 < S ? st + 1 : (ph ^= 1, 0)) {
          if (!mbar_wait(&bar_full[st], ph, sh.err, 3, sh.spin) || aborted(&s_abort)) {
            s_abort = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          if (q == 0) stamp(3);
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
            run(sa, d0, first0);
            run(sa + a_bytes, d0 + NT, first1);
          } else if (k < sh.nkb1) {
            run(sa, d0, first0);
          } else {
            run(sa, d0 + NT, first1);
          }
          mma_commit(&bar_empty[st]);
        }
        mma_commit(&bar_accf[buf]);
      }
      if (q > 0) {
        // every MMA issued has completed before the block frees TMEM or exits, also when a wait
        // elsewhere gave up (this wait always has the full limit)
        mma_commit(&bar_drain);
        mbar_wait(&bar_drain, 0, nullptr, 0);
      }
      stamp(4);
    }
  } else {
    // epilogue warps
    const int ew = warp & 3, half = (warp - 2) >> 2;
    const int r = ew * 32 + lane;
    const int et = threadIdx.x - 64;             // 0..255
    const uint32_t tlane = tmem + ((uint32_t)(ew * 32) << 16);
    griddep_wait();                              // token factors and residuals come from predecessors
    int t = 0;
    bool waited = false;
    // the next tile's token factor (one per thread: NT <= 256 epilogue threads) and weight-row
    // constants are loaded while this tile is written out, so their latency is hidden
    float tk_next = 0.0f;
    typename Epi::Row rw_next{};
    bool live_next = false;
    for (int item = item0; item < sh.items; item += istride, ++t) {
      const int buf = sh.nbuf == 2 ? (t & 1) : 0;
      const uint32_t use = sh.nbuf == 2 ? (t >> 1) : t;
      int s, row0, tok0;
      coords(item, s, row0, tok0);
      float* tk = s_tok[t & 1];
      if (t == 0) {
        for (int j = et; j < NT; j += 32 * kEpiWarps) tk[j] = ftz(epi.tok(min(tok0 + j, sh.M - 1)));
      } else if (et < NT) {
        tk[et] = tk_next;
      }
      // the first tile's weight-row constants load while its MMAs run (later tiles take them from
      // the previous iteration's prefetch): split-K, the rows of this thread's first two units
      typename Epi::Row rw_first{}, rw_unit0{}, rw_unit1{};
      if (t == 0) {
        if (split > 1) {
          const int rs = kRows / split;
          const int u0 = et, u1 = et + 32 * kEpiWarps;
          if (u0 < rs * (NT / 4) && row0 + crank * rs + u0 % rs < sh.nrow[s]) rw_unit0 = epi.row(s, row0 + crank * rs + u0 % rs);
          if (u1 < rs * (NT / 4) && row0 + crank * rs + u1 % rs < sh.nrow[s]) rw_unit1 = epi.row(s, row0 + crank * rs + u1 % rs);
        } else if (row0 + r < sh.nrow[s]) {
          rw_first = epi.row(s, row0 + r);
        }
      }
      // (split-K: every CTA pushes its rows even after a give-up, so no owner waits in vain)
      if (split == 1 && epi_sync_or(aborted(&s_abort))) break;
      bool ok = true;
      if (nk > 0) {
        ok = mbar_wait(&bar_accf[buf], use & 1, sh.err, 4, sh.spin);
        if (!ok) s_abort = 1;
        if (split > 1 && threadIdx.x == 64) stamp(7);   // split-K: the accumulator is ready
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t tb = tlane + buf * acc_cols;
      if (split > 1) {
        // push this CTA's partial rows to their owners (16 tokens of one row per 4 st.async)
        cluster_wait();
        waited = true;
        const int rs = kRows / split, owner = r / rs, rl = r % rs;
        const uint32_t slot = smem_u32(R) + (uint32_t)(((crank * rs + rl) * RL) * 4);
        const uint32_t accb = (uint32_t)(split * rs * RL * 4);
        const uint32_t rbar = cluster_map(smem_u32(&bar_recv), owner);
        for (int j0 = 16 * half; j0 < NT; j0 += 32) {
          uint32_t v[2][16];
          tmem_ld16(tb + j0, v[0]);
          if (nacc == 2) tmem_ld16(tb + NT + j0, v[1]);
          tmem_wait_ld();
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            if (a >= nacc) break;
            const bool used = a == 0 ? used0 : used1;
            const uint32_t dst = slot + a * accb + (uint32_t)j0 * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t x0 = used ? v[a][4 * q] : 0u, x1 = used ? v[a][4 * q + 1] : 0u;
              const uint32_t x2 = used ? v[a][4 * q + 2] : 0u, x3 = used ? v[a][4 * q + 3] : 0u;
              if (owner == crank) {
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + 16 * q), "r"(x0), "r"(x1),
                             "r"(x2), "r"(x3)
                             : "memory");
              } else {
                st_async_v4(cluster_map(dst + 16 * q, owner), x0, x1, x2, x3, rbar);
              }
            }
          }
        }
        // TMEM is read: hand it back (warp 1 frees it) before waiting on the peers
        tc_fence_before();
        asm volatile("bar.arrive 2, %0;" ::"n"(32 + 32 * kEpiWarps) : "memory");
        // every peer pushes its rows, so this wait ends; it has the full limit because the
        // block must not exit while a peer's stores into its shared memory are in flight
        const bool got = mbar_wait(&bar_recv, 0, sh.err, 5);
        if (threadIdx.x == 64) stamp(5);                // the peers' partial rows have arrived
        if (epi_sync_or(!got || !ok)) {
          s_abort = 1;
          break;
        }
        // sum the slots of this CTA's rows and run the epilogue: one row x 4 tokens per unit, so
        // every epilogue thread has work and a few short chains to interleave
        const int units = rs * (NT / 4);
        for (int u = et, ui = 0; u < units; u += 32 * kEpiWarps, ++ui) {
          const int url = u % rs, uj0 = 4 * (u / rs);
          const int cc = row0 + crank * rs + url;
          uint32_t a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
          for (int p = 0; p < split; ++p) {
            const int* src = R + (p * rs + url) * RL + uj0;
            const int4 x = *reinterpret_cast<const int4*>(src);
            a0[0] += x.x;
            a0[1] += x.y;
            a0[2] += x.z;
            a0[3] += x.w;
            if (nacc == 2) {
              const int4 y = *reinterpret_cast<const int4*>(src + split * rs * RL);
              a1[0] += y.x;
              a1[1] += y.y;
              a1[2] += y.z;
              a1[3] += y.w;
            }
          }
          if (cc < sh.nrow[s]) {
            const typename Epi::Row rw2 = ui == 0 ? rw_unit0 : (ui == 1 ? rw_unit1 : epi.row(s, cc));
            epi.template put<4>(rw2, tk + uj0, tok0 + uj0, min(4, sh.M - tok0 - uj0), a0, a1, nacc == 2);
          }
        }
        break;                                   // one tile per CTA in this mode
      }
      const int c = row0 + r;
      typename Epi::Row rw{};
      bool live;
      if (t == 0) {
        live = c < sh.nrow[s];
        rw = rw_first;
      } else {
        live = live_next;
        rw = rw_next;
      }
      live = live && ok;
      if (item + istride < sh.items) {           // prefetch for the next tile
        int s2, row2, tok2;
        coords(item + istride, s2, row2, tok2);
        if (et < NT) tk_next = ftz(epi.tok(min(tok2 + et, sh.M - 1)));
        live_next = row2 + r < sh.nrow[s2];
        if (live_next) rw_next = epi.row(s2, row2 + r);
      }
      const int last = (NT - 16 - 16 * half) / 32 * 32 + 16 * half;   // this warp's last chunk
      for (int j0 = 16 * half; j0 < NT; j0 += 32) {
        uint32_t v0[16], v1[16];
        tmem_ld16(tb + j0, v0);
        if (nacc == 2) tmem_ld16(tb + NT + j0, v1);
        tmem_wait_ld();
        if (j0 == last && sh.nbuf == 2) {        // the accumulator is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_acce[buf]);
        }
        if (live) epi.template put<16>(rw, tk + j0, tok0 + j0, min(16, sh.M - tok0 - j0), v0, v1, nacc == 2);
      }
      if (NT <= 16 * half && sh.nbuf == 2) {     // no chunk for this warp: release at once
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_acce[buf]);
      }
    }
    if (split > 1 && !waited) {                  // aborted before the push: keep the barriers paired
      cluster_wait();
      asm volatile("bar.arrive 2, %0;" ::"n"(32 + 32 * kEpiWarps) : "memory");
    }
  }

  __syncwarp();                              // lanes 1-31 of warps 0 / 1 wait for their lane 0
  if (threadIdx.x == 64) stamp(6);
  if (split > 1 && warp < 2) cluster_wait();
  if (split > 1) {
    // warp 1 frees TMEM once the epilogue warps have read it (named barrier 2), not at the end
    if (warp == 1) {
      asm volatile("bar.sync 2, %0;" ::"n"(32 + 32 * kEpiWarps) : "memory");
      tc_fence_after();
      tmem_dealloc(tmem, ncols);
    }
  } else {
    tc_fence_before();
  }
  __syncthreads();
  if (split == 1 && warp == 1) tmem_dealloc(tmem, ncols);
  if (threadIdx.x == 0) {
    if (split == 1) stamp(7);
    // after a give-up, the last K slices issued may still be in flight: they land before the
    // block exits (these waits always have the full limit)
    if (aborted(&s_abort))
      for (uint32_t i = issued > (uint32_t)S ? issued - S : 0; i < issued; ++i)
        mbar_wait(&bar_full[i % S], (i / S) & 1, nullptr, 0);
  }
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

// Error code of the bounded waits (static device memory: the kernel allocates nothing). The
// symbol has its own address on every device, so the address is looked up (once) per device,
// with that device current.
__device__ int g_mma_err;
constexpr int kMaxDevices = 64;
std::mutex g_err_mutex;
int* g_err_ptr[kMaxDevices] = {};
int* err_flag() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mutex);
  if (!g_err_ptr[dev]) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_mma_err) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(a);
  }
  return g_err_ptr[dev];
}
std::atomic<uint32_t> g_spin{kSpinLimit};

// Token tile, mode (split-K factor or persistent), stages, shared memory and grid.
bool plan(MmaShape& sh, int tiles, int* smem, int* grid) {
  sh.NT = std::min(256, (sh.M + 15) / 16 * 16);
  int ntt = (sh.M + sh.NT - 1) / sh.NT;
  const int nkb = sh.nkb1 + sh.nkb2;
  int split = 1;
  if (tiles * ntt >= 16 && tiles * ntt < kSMs / 2) {
    // 16 or more weight tiles: split-K first (it divides the weight bytes per CTA; at most 4 here,
    // a cluster of 8 with 2-3 K slices per CTA measured slower), then narrower token tiles.
    // Measured at M = 64: qkv (32 tiles) 17.7 -> 16.8 us, gate|up (48 tiles) 20.9 -> 16.8 us.
    while (split < 8 && tiles * ntt * split * 2 <= kSMs && nkb >= split * 2 * 2) split *= 2;
    while (tiles * ntt * split * 2 <= kSMs && sh.NT > 16) {
      sh.NT = std::max(16, (sh.NT / 2 + 15) / 16 * 16);
      ntt = (sh.M + sh.NT - 1) / sh.NT;
    }
  } else {
    // too few tiles for the SMs: narrower token tiles first (their weight tiles are shared through
    // L2), then split-K over a cluster
    while (tiles * ntt < kSMs && sh.NT > 16) {
      sh.NT = std::max(16, (sh.NT / 2 + 15) / 16 * 16);
      ntt = (sh.M + sh.NT - 1) / sh.NT;
    }
    if (tiles * ntt < kSMs / 2)
      while (split < 8 && tiles * ntt * split * 2 <= kSMs && nkb >= split * 4) split *= 2;   // one wave
  }
  sh.split = split;
  sh.nbuf = split > 1 ? 1 : 2;
  // the slots (split-K) with a stage, or both accumulators (persistent), must fit
  const int na0 = sh.gated ? 2 : 1;
  auto slots = [&](int nt) { return sh.nacc * kRows * (nt + 4) * 4; };
  if ((split > 1 && slots(sh.NT) + na0 * kRows * kSlice + sh.NT * kSlice > kSmemBudget) ||
      sh.nbuf * sh.nacc * sh.NT > 512)
    sh.NT = std::min(sh.NT, 128);
  sh.ntt = (sh.M + sh.NT - 1) / sh.NT;
  sh.items = tiles * sh.ntt;
  const int per = (nkb + split - 1) / split;
  const int na = sh.gated ? 2 : 1;
  const int stage = na * kRows * kSlice + sh.NT * kSlice;
  const int part = split > 1 ? slots(sh.NT) : 0;
  sh.stages = std::max(1, std::min(kMaxStages, (kSmemBudget - part) / stage));
  if (split > 1) sh.stages = std::min(sh.stages, per);
  *smem = sh.stages * stage + part + 1024;
  // CTAs that share an SM must fit in its 512 TMEM columns together, so a CTA never waits in
  // tcgen05.alloc
  int ncols = 32;
  while (ncols < sh.nbuf * sh.nacc * sh.NT) ncols <<= 1;
  const int max_res = 512 / ncols;
  *smem = std::max(*smem, kSmemPerSM / (max_res + 1) + 64 - 1024);
  const int res = std::max(1, std::min(max_res, kSmemPerSM / (*smem + 1024 + 256)));
  *grid = split > 1 ? sh.items * split : std::min(sh.items, kSMs * res);
  const int want = g_trace_on.load();
  sh.trace = want > 0 && g_trace_count.fetch_add(1) + 1 == want;
  sh.err = err_flag();
  sh.spin = spin_limit();
  return sh.err != nullptr;
}

template <class Epi>
cudaError_t launch(const MmaMaps& maps, const MmaShape& sh, const Epi& epi, int grid, int smem, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(k_mma_i8<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_ex(k_mma_i8<Epi>, dim3(grid), dim3(kThreads), smem, st, sh.split, maps, sh, epi);
}
}  // namespace

// uint8 matrix [rows, cols] (row stride ld bytes) in boxes of box_cols bytes x box_rows rows, with
// the 128-byte swizzle (box_cols <= 128) or dense rows, zero fill past the edges.
bool make_map_u8(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle) {
  auto fn = encode_fn();
  if (!fn || (uintptr_t)ptr % 16 || ld % 16 || cols == 0 || rows == 0 || box_cols % 16 || box_cols > 128)
    return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


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
  int smem = 0, grid = 0;
  if (!plan(sh, tiles, &smem, &grid)) return cudaErrorInvalidValue;
  if (!make_map(&maps.x, g.A, g.K, g.M, g.lda, sh.NT)) return cudaErrorInvalidValue;
  for (int s = 0; s < g.nseg; ++s) {
    if (!make_map(&maps.w[2 * s], g.seg[s].W, g.kb, g.seg[s].n, g.kb, kRows)) return cudaErrorInvalidValue;
    if (two && !make_map(&maps.w[2 * s + 1], g.seg[s].W2, g.K - g.kb, g.seg[s].n, g.K - g.kb, kRows))
      return cudaErrorInvalidValue;
  }
  return launch(maps, sh, EngEpi{g}, grid, smem, st);
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
  int smem = 0, grid = 0;
  if (!plan(sh, tiles, &smem, &grid)) return cudaErrorInvalidValue;
  if (!make_map(&maps.x, g.A, g.K, g.M, g.lda, sh.NT)) return cudaErrorInvalidValue;
  if (!make_map(&maps.w[0], g.W, g.K, g.N, g.K, kRows)) return cudaErrorInvalidValue;
  return launch(maps, sh, MachEpi{g}, grid, smem, st);
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

int* wait_error_flag() { return err_flag(); }

uint32_t spin_limit() { return g_spin.load(); }

}  // namespace tc

extern "C" uint32_t tc_set_spin_limit(uint32_t polls) {
  return tc::g_spin.exchange(polls == 0 ? 0u : std::min(polls, tc::kSpinLimit));
}

extern "C" int tc_wait_error(int32_t clear) {
  int* p = tc::wait_error_flag();
  if (!p) return TC_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return TC_ERR_CUDA;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return TC_ERR_CUDA;
  }
  return v;
}

extern "C" int tc_mma_trace(int32_t enable, uint64_t* out, uint32_t cap) {
  if (enable > 0) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, tc::g_mma_trace) != cudaSuccess ||
        cudaMemset(a, 0, sizeof(tc::g_mma_trace)) != cudaSuccess)
      return TC_ERR_CUDA;
  }
  tc::g_trace_on.store(enable > 0 ? enable : 0);
  tc::g_trace_count.store(0);
  if (!out || !cap) return 0;
  const uint32_t n = std::min<uint32_t>(cap, tc::kTraceCtas * tc::kTraceStamps);
  if (cudaDeviceSynchronize() != cudaSuccess) return TC_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, tc::g_mma_trace, n * sizeof(uint64_t)) != cudaSuccess) return TC_ERR_CUDA;
  return (int)n;
}

extern "C" int tc_set_mma_min_rows(int32_t rows) {
  const int prev = tc::mma_min_rows();
  tc::g_min_rows.store(rows < 2 ? 2 : rows);
  return prev;
}
