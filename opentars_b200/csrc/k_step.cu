// The fused decode step: every layer of a Qwen3 / Gemma 3 decode step for B <= 64 sequences in one
// cooperative launch (one CTA per SM), bit-exact with the per-kernel engine path (k_engine.cu,
// k_mma.cu) and so with the reference's descriptor queues (tars_mini/llm.py:548-571, 614-640,
// 705-782; golden.py:326-349, 358-435; numerics.py).
//
// Roles in a 320-thread CTA:
//   warp 0, lane 0   weight producer: walks the step's GEMMs in order and bulk-copies the 128-row x
//                    128-byte weight slices of this CTA's share into a ring of kStages slots as
//                    soon as a slot is free - the weights do not depend on the step's data, so the
//                    next GEMM's slices are on chip before its phase starts
//   warp 1           TMEM owner; lane 0 issues the MMAs of a GEMM phase (tcgen05.mma kind::i8,
//                    weights as operand A: M = 128 rows; the step's int8 rows as operand B: N =
//                    ntok) after copying the phase's K chunk of the rows into shared memory
//   warps 2-9        workers: the GEMM epilogue (TMEM -> int32 partial sums), the row phases
//                    (norm + quant, gated quant), attention
// Every operand slice is one contiguous block in HBM laid out as the MMA reads it (step.h), so each
// copy is one 1-D bulk copy. Phases are separated by a grid barrier (a global arrival count).
// Every wait is bounded in time (globaltimer): one that gives up records where (err, diag), the
// step is abandoned by every CTA, and copies or MMAs still in flight finish before a block exits.
// A GEMM phase writes int32 partial sums per K chunk, part[chunk][m][col]: int32 sums are exact in
// any order, so the consumer phase adds the chunks and runs the GEMM's fp32 epilogue itself with
// the same steps as the per-kernel path. The attention output's row quantisation needs the row's
// absmax over all kv heads: each (sequence, kv head) unit publishes its part, and the unit that
// arrives last for a sequence quantises the whole row (max is order-free).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "fp32.cuh"
#include "step.h"
#include "umma.cuh"

namespace tc {
namespace {

constexpr int kThreads = 320;
constexpr int kStages = 8;
constexpr int kSliceB = kStepSliceBytes;    // one weight slice: 128 rows x 128 bytes of K
constexpr int kRegion = 80 * 1024;          // the rows' K chunk / attention tiles / row staging
constexpr int kT = 256;                     // longest context
// trace layout: [0, kTraceArrive) CTA 0's barrier exits (stamp 0: the kernel's start), then per
// barrier every CTA's arrival
constexpr int kTraceArrive = 1024;

// named barriers (the non-aligned form: a warp may reach them with its lanes apart)
__device__ __forceinline__ void sync_main() { asm volatile("barrier.sync 1, 288;" ::: "memory"); }     // warps 1-9
__device__ __forceinline__ void sync_workers() { asm volatile("barrier.sync 2, 256;" ::: "memory"); }  // warps 2-9
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_vol(const int* p) { return *(volatile const int*)p; }
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ep(a) = fmul(fmul(i2f(a), sr), sc) with sr, sc flushed: the engine GEMM epilogue's product
__device__ __forceinline__ float ep_fast(int a, float sr, float sc) { return canon(fmul_ff(fmul_ff(i2f(a), sr), sc)); }

__device__ __forceinline__ float sum16_fold(float v) {
  v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
  v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax_c(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

struct Ctl {
  int abort;                  // set by any role whose wait gave up (or saw another CTA give up)
  int go;                     // written only by the barrier leader: every thread of warps 1-9
                              // reads the same value after a barrier, so they leave together
  unsigned gen;
};

// A non-blocking test of an mbarrier phase (mbarrier.try_wait may suspend the thread for a time
// the hardware chooses; these loops bound their waits by the clock instead).
__device__ __forceinline__ bool mbar_ready(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// The first give-up of the step records its code, CTA, barrier count and detail.
__device__ void give_up(const StepArgs& a, Ctl* ctl, int code, uint32_t detail) {
  if (atomicCAS(a.err, 0, code) == 0) {
    a.diag[0] = code;
    a.diag[1] = (int)blockIdx.x;
    a.diag[2] = (int)ctl->gen;
    a.diag[3] = (int)detail;
  }
  ctl->abort = 1;
}
__device__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const StepArgs& a, Ctl* ctl, int code) {
  if (mbar_ready(bar, parity)) return true;
  const uint64_t t0 = gtime();
  for (uint32_t i = 1;; ++i) {
    if (mbar_ready(bar, parity)) return true;
    if ((i & 31) == 0) {
      if (*(volatile int*)&ctl->abort || ld_vol(a.err)) {
        ctl->abort = 1;
        return false;
      }
      if (gtime() - t0 >= a.wait_ns) {
        give_up(a, ctl, code, parity);
        return false;
      }
    }
    if (i > 64) __nanosleep(32);
  }
}
// Waits (up to limit_ns) for copies or MMAs in flight before a block leaves after a give-up.
__device__ void drain_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = gtime();
  while (!mbar_ready(bar, parity)) {
    if (gtime() - t0 >= limit_ns) return;
    __nanosleep(64);
  }
}

// Grid barrier over warps 1-9 of every CTA: what the phase wrote is visible to every CTA after it.
// (The bulk copies that read what a phase wrote are ordered after it by the MMA thread's own proxy
// fences in mma_phase.)
__device__ bool grid_sync(const StepArgs& a, Ctl* ctl) {
  sync_main();
  if (threadIdx.x == 64) {
    const unsigned gen = ctl->gen + 1;
    ctl->gen = gen;
    bool ok = !*(volatile int*)&ctl->abort;
    if (ok) {
      if (a.trace) a.trace[(uint64_t)gen * gridDim.x + blockIdx.x + kTraceArrive] = gtime();
      __threadfence();
      red_release(a.sync, 1u);
      const unsigned target = gen * gridDim.x;
      const uint64_t t0 = gtime();
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire(a.sync) >= target) break;
        if ((i & 15) == 15) {
          if (ld_vol(a.err)) {
            ctl->abort = 1;
            ok = false;
            break;
          }
          if (gtime() - t0 >= a.wait_ns) {
            give_up(a, ctl, 31, ld_acquire(a.sync));
            ok = false;
            break;
          }
        }
      }
      if (a.trace && blockIdx.x == 0) a.trace[gen] = gtime();          // CTA 0 leaves the barrier
    }
    ctl->go = ok;
  }
  sync_main();
  return *(volatile int*)&ctl->go != 0;
}

// trace mode, CTA 0: the first time a point is reached in the step (points 700..: inside phases),
// by the first worker (stamp) or by the MMA thread (stamp1)
__device__ __forceinline__ void stamp(const StepArgs& a, int k) {
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 64 && a.trace[k] == 0) a.trace[k] = gtime();
}
__device__ __forceinline__ void stamp1(const StepArgs& a, int k) {
  if (a.trace && blockIdx.x == 0 && a.trace[k] == 0) a.trace[k] = gtime();
}

__device__ __forceinline__ bool my_chunk(const StepGemm& g, int& ks, int& grp) {
  ks = (int)blockIdx.x % g.ksplit;
  grp = (int)blockIdx.x / g.ksplit;
  return grp < g.groups && grp < g.tile0[g.nseg];
}
__device__ __forceinline__ int seg_of(const StepGemm& g, int t) {
  int s = 0;
  while (s + 1 < g.nseg && t >= g.tile0[s + 1]) ++s;
  return s;
}

// ------------------------------------------------------------------------------ weight producer
__device__ __noinline__ uint32_t produce(const StepArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty, Ctl* ctl) {
  uint32_t q = 0;
  // gs: the barrier after which the GEMM's phase runs; its slices are issued once this CTA has
  // entered barrier gs - lead (so the stream does not crowd the latency-bound phases before it)
  auto gemm = [&](const StepGemm& g, unsigned gs) -> bool {
    int ks, grp;
    if (!my_chunk(g, ks, grp)) return true;
    if ((unsigned)a.lead < gs) {
      const uint64_t t0 = gtime();
      while (*(volatile unsigned*)&ctl->gen + (unsigned)a.lead < gs) {
        if (*(volatile int*)&ctl->abort) return false;
        if (gtime() - t0 >= a.wait_ns) {
          give_up(a, ctl, 45, gs);
          return false;
        }
      }
    }
    const int k0 = ks * g.KC, k1 = min(g.nslices, k0 + g.KC);
    const int ntiles = g.tile0[g.nseg];
    for (int t = grp; t < ntiles; t += g.groups) {
      for (int k = k0; k < k1; ++k, ++q) {
        const int slot = q % kStages;
        if (!wait_or_abort(&empty[slot], ((q / kStages) & 1) ^ 1, a, ctl, 41)) return false;
        mbar_expect_tx(&full[slot], kSliceB);
        bulk_load(ring + slot * kSliceB, g.wt + ((uint64_t)t * g.nslices + k) * kSliceB, kSliceB, &full[slot]);
      }
    }
    return true;
  };
  bool ok = true;
  for (int l = 0; l < a.L && ok; ++l) {
    const StepLayer& Ly = a.layers[l];
    const unsigned g0 = 8u * l;                        // a layer's phases end at barriers 8l + 1 .. 8l + 8
    ok = gemm(Ly.qkv, g0 + 1) && gemm(Ly.o, g0 + 3) && gemm(Ly.gu, g0 + 5) && gemm(Ly.down, g0 + 7);
  }
  if (ok) gemm(a.head, 8u * a.L + 1);
  return q;
}

// ------------------------------------------------------------------------------ GEMM phase
struct MmaState {
  uint32_t q = 0, tiles = 0, nact = 0;
};

// warp 1, lane 0: the K chunk of the rows into shared memory, then per row tile the chunk's MMAs
// trace mode, CTA 0, the head GEMM: pipeline stamps at kTraceHead.. (rows copy issued / landed; per
// tile: its first and last weight slice ready, its MMAs issued; then per tile in the epilogue: the
// accumulator seen, its stores issued)
constexpr int kTraceHead = 600;
__device__ __noinline__ bool mma_phase(const StepArgs& a, const StepGemm& g, uint8_t* ring, uint8_t* region, uint64_t* full,
                          uint64_t* empty, uint64_t* accf, uint64_t* acce, uint64_t* actb, uint32_t tmem, MmaState& st,
                          Ctl* ctl, bool head) {
  int ks, grp;
  if (!my_chunk(g, ks, grp)) return true;
  unsigned long long* tr = (a.trace && head && blockIdx.x == 0) ? a.trace + kTraceHead : nullptr;
  const int k0 = ks * g.KC, kc = min(g.nslices, k0 + g.KC) - k0;
  const uint32_t xb = (uint32_t)a.ntok * 128;
  // what the phases before wrote through the generic proxy (the rows in global memory, the staging
  // region in shared memory) is ordered before this thread's bulk copy
  fence_proxy_async();
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_expect_tx(actb, kc * xb);
  bulk_load(region, a.q8t + (uint64_t)k0 * xb, kc * xb, actb);
  if (tr) tr[0] = gtime();
  if (!head) stamp1(a, 735);
  const uint32_t par = st.nact & 1;
  ++st.nact;
  if (!wait_or_abort(actb, par, a, ctl, 42)) {
    drain_wait(actb, par, a.drain_ns);                  // the rows' copy lands before anything else
    return false;
  }
  if (tr) tr[1] = gtime();
  if (!head) stamp1(a, 736);
  int ti = 0;
  const uint32_t idesc = idesc_i8(128, a.ntok);
  const int ntiles = g.tile0[g.nseg];
  for (int t = grp; t < ntiles; t += g.groups, ++st.tiles) {
    const int buf = st.tiles & 1;
    const uint32_t use = st.tiles >> 1;
    if (use > 0 && !wait_or_abort(&acce[buf], (use & 1) ^ 1, a, ctl, 43)) return false;
    tc_fence_after();
    const uint32_t d = tmem + buf * a.ntok;
    for (int i = 0; i < kc; ++i, ++st.q) {
      const int slot = st.q % kStages;
      if (!wait_or_abort(&full[slot], (st.q / kStages) & 1, a, ctl, 44)) return false;
      if (tr && ti < 8 && (i == 0 || i == kc - 1)) tr[2 + 3 * ti + (i ? 1 : 0)] = gtime();
      tc_fence_after();
      const uint32_t sa = smem_u32(ring + slot * kSliceB), sb = smem_u32(region + i * xb);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_i8(d, sdesc_k128(sa + 32 * kk), sdesc_k128(sb + 32 * kk), idesc, (i | kk) ? 1u : 0u);
      mma_commit(&empty[slot]);
    }
    mma_commit(&accf[buf]);
    if (tr && ti < 8) tr[4 + 3 * ti] = gtime();
    if (!head) stamp1(a, 737);
    ++ti;
  }
  return true;
}

// warps 2-9: each accumulator to the partial sums (or, for the head, through the epilogue to the
// logits). Warp w reads TMEM lanes 32 (w % 4) .. (weight rows); warps 2-5 the even 16-token
// chunks, 6-9 the odd ones.
__device__ __noinline__ bool epi_phase(const StepArgs& a, const StepGemm& g, bool fused, uint32_t tmem, uint64_t* accf,
                          uint64_t* acce, uint32_t& tiles, Ctl* ctl, float* s_tok) {
  int ks, grp;
  if (!my_chunk(g, ks, grp)) return true;
  if (fused) {                                         // the tokens' row scales, once per phase
    const int wt = threadIdx.x - 64;
    if (wt < a.ntok) s_tok[wt] = wt < a.B ? ftz(a.qsa[wt]) : 0.0f;
    sync_workers();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp & 3, half = (warp - 2) >> 2, r = ew * 32 + lane;
  const uint32_t tlane = tmem + ((uint32_t)(ew * 32) << 16);
  const int ntiles = g.tile0[g.nseg];
  const int ldp = g.col0[g.nseg];
  const int last = (a.ntok - 16 - 16 * half) / 32 * 32 + 16 * half;
  unsigned long long* tr = (a.trace && fused && blockIdx.x == 0 && threadIdx.x == 64) ? a.trace + kTraceHead + 40 : nullptr;
  int ti = 0;
  // the head's per-row scale, loaded a tile ahead so its latency hides behind the previous tile
  auto row_scale = [&](int t) {
    if (!fused || t >= ntiles) return 0.0f;
    const int s = seg_of(g, t);
    const int rr = (t - g.tile0[s]) * 128 + r;
    return rr < g.col0[s + 1] - g.col0[s] ? g.scale[s][rr] : 0.0f;
  };
  float sc_next = row_scale(grp);
  for (int t = grp; t < ntiles; t += g.groups, ++tiles, ++ti) {
    const int buf = tiles & 1;
    const uint32_t use = tiles >> 1;
    const int s = seg_of(g, t);
    const int rr = (t - g.tile0[s]) * 128 + r;
    const bool live = rr < g.col0[s + 1] - g.col0[s];
    const int col = g.col0[s] + rr;
    const float sc = ftz(sc_next);
    sc_next = row_scale(t + g.groups);
    const bool ok = wait_or_abort(&accf[buf], use & 1, a, ctl, 45);
    if (!__all_sync(0xFFFFFFFFu, ok)) return false;
    if (tr && ti < 8) tr[2 * ti] = gtime();
    if (!fused && ti == 0) stamp(a, 730);
    tc_fence_after();
    for (int j0 = 16 * half; j0 < a.ntok; j0 += 32) {
      uint32_t v[16];
      tmem_ld16(tlane + buf * a.ntok + j0, v);
      tmem_wait_ld();
      if (j0 == last) {                                 // the accumulator is in registers
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
      }
      if (!live) continue;
      if (fused) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = j0 + j;
          if (m < a.B) a.logits[(uint64_t)m * a.vocab + col] = ftz(ep_fast((int)v[j], s_tok[m], sc));
        }
      } else {
        int* p = a.part + (uint64_t)ks * a.B * ldp + col;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = j0 + j;
          if (m < a.B) p[(uint64_t)m * ldp] = (int)v[j];
        }
      }
    }
    if (a.ntok <= 16 * half) {                          // no chunk for this warp: release at once
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
    }
    if (tr && ti < 8) tr[2 * ti + 1] = gtime();
    if (!fused && ti == 0) stamp(a, 731);
  }
  return true;
}

// ------------------------------------------------------------------------------ worker reductions
// sum16 of v[0..N) in shared memory in the contract's order (numerics.py:306-316), broadcast
__device__ float wsum16(const float* v, int N, float* red) {
  const int tid = threadIdx.x - 64;
  sync_workers();
  if (tid < 16) {
    float acc = 0.0f;
    int j = tid;
    for (; j + 16 * 7 < N; j += 16 * 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = v[j + 16 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = fadd_nc(acc, t[u]);
    }
    for (; j < N; j += 16) acc = fadd_nc(acc, v[j]);
    acc = canon(acc);
    acc = fadd(acc, __shfl_xor_sync(0x0000FFFFu, acc, 1));
    acc = fadd(acc, __shfl_xor_sync(0x0000FFFFu, acc, 2));
    acc = fadd(acc, __shfl_xor_sync(0x0000FFFFu, acc, 4));
    acc = fadd(acc, __shfl_xor_sync(0x0000FFFFu, acc, 8));
    if (tid == 0) red[32] = acc;
  }
  sync_workers();
  return red[32];
}
// the order-free absmax (numerics.py:293-303) over the workers
__device__ float wmax(float v, float* red) {
  const int tid = threadIdx.x - 64;
  v = warp_max(v);
  sync_workers();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  sync_workers();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) r = fmax_c(r, red[i]);
  return r;
}

// element (row m, column k) of the step's int8 rows, in the operand layout (step.h)
__device__ __forceinline__ void put_q8(const StepArgs& a, int m, int k, int8_t v) {
  a.q8t[(uint64_t)(k >> 7) * a.ntok * 128 + step_swz((uint32_t)m, (uint32_t)(k & 127))] = (uint8_t)v;
}
// ROW_QUANT's q8 of columns [16 c, 16 c + 16) of row m (x: their fp32 values), one 16-byte store:
// the 16 columns are one chunk of the operand layout
__device__ __forceinline__ void put_q8x16(const StepArgs& a, int m, int c, const float4 (&x)[4], float inv) {
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    w[q] = (uint32_t)(uint8_t)q8(x[q].x, inv) | (uint32_t)(uint8_t)q8(x[q].y, inv) << 8 |
           (uint32_t)(uint8_t)q8(x[q].z, inv) << 16 | (uint32_t)(uint8_t)q8(x[q].w, inv) << 24;
  const int k = 16 * c;
  *reinterpret_cast<uint4*>(a.q8t + (uint64_t)(k >> 7) * a.ntok * 128 + step_swz((uint32_t)m, (uint32_t)(k & 127))) =
      make_uint4(w[0], w[1], w[2], w[3]);
}
// ROW_QUANT of the n fp32 values at src (L2, written by other CTAs) into row m, by nt threads
// (thread t): two 16-column chunks' loads in flight per thread before they are used
__device__ __forceinline__ void quant_row_from(const StepArgs& a, int m, const float* src, int n, float inv, int t,
                                               int nt) {
  const int nc = n / 16;
  for (int c0 = t; c0 < nc; c0 += 2 * nt) {
    float4 x[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (c0 + h * nt < nc)
#pragma unroll
        for (int q = 0; q < 4; ++q) x[h][q] = __ldcg(reinterpret_cast<const float4*>(src + 16 * (c0 + h * nt)) + q);
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (c0 + h * nt < nc) put_q8x16(a, m, c0 + h * nt, x[h], inv);
  }
}

// ------------------------------------------------------------------------------ row phases
// Row m of the residual stream, then its RMSNorm (gamma) and ROW_QUANT (llm.py:97-104;
// numerics.py:353-390):
//   kind 0  x = E[tok] (Gemma: times fp32(sqrt(H)), in IEEE fp32 as the host computes it)
//   kind 1  x = res + ep(the GEMM's partials)                       (Qwen3: after o / down)
//   kind 2  x = res + rmsnorm(y, pre_gamma), y the GEMM's output    (Gemma 3: attn / mlp norm)
// x is written to xout. The K-split GEMM (two K blocks sharing the scales): y = ep(acc_1) + ep(acc_2).
__device__ __noinline__ void norm_row(const StepArgs& a, int m, int kind, const StepGemm* g, const float* srow, const float* res,
                         float* xout, const float* pre_gamma, const float* gamma, float* qs_out, float* sm, float* red) {
  const int H = a.H, tid = threadIdx.x - 64;
  const bool st = kind != 0;
  if (st) stamp(a, 700);
  float* sx = sm;
  float* sv = sm + H;
  float* sg = sm + 2 * H;                              // gamma, pre_gamma and the residual row,
  float* spg = sm + 3 * H;                             // staged before the partial sums are read
  float* sres = sm + 4 * H;
  for (int j4 = tid; j4 < H / 4; j4 += 256) {
    cp16(sg + 4 * j4, gamma + 4 * j4);
    if (kind == 2) cp16(spg + 4 * j4, pre_gamma + 4 * j4);
    if (kind >= 1) cp16(sres + 4 * j4, res + (uint64_t)m * H + 4 * j4);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const float kinv = recip_f(i2f(H));
  if (kind == 0) {
    const float* e = a.E + (uint64_t)a.tok[m] * H;
    for (int j = tid; j < H; j += 256) {
      const float v = a.gemma ? __fmul_rn(e[j], a.embed_scale) : e[j];
      xout[(uint64_t)m * H + j] = v;
      sx[j] = ftz(v);
    }
  } else {
    const float sr = ftz(srow[m]);
    const uint64_t ldp = g->col0[g->nseg], slab = (uint64_t)a.B * ldp;
    const bool two = g->kb < g->nslices;
    const int nb1 = two ? g->kb / g->KC : g->ksplit, ksplit = g->ksplit;
    const float* scale = g->scale[0];
    for (int j4 = tid; j4 < H / 4; j4 += 256) {
      const int j = 4 * j4;
      const int* p = a.part + (uint64_t)m * ldp + j;
      int4 v[8];                                       // every chunk's load issued before the sums
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        if (ks < ksplit) v[ks] = *reinterpret_cast<const int4*>(p + ks * slab);
      int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (ks >= ksplit) continue;
        if (ks < nb1) {
          a0[0] += v[ks].x; a0[1] += v[ks].y; a0[2] += v[ks].z; a0[3] += v[ks].w;
        } else {
          a1[0] += v[ks].x; a1[1] += v[ks].y; a1[2] += v[ks].z; a1[3] += v[ks].w;
        }
      }
      if (st && j4 == tid) stamp(a, 706);               // the partial sums have arrived
      const float4 sc4 = *reinterpret_cast<const float4*>(scale + j);
      const float scs[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
      float y[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float sc = ftz(scs[u]);
        y[u] = two ? ftz(fadd(ftz(ep_fast(a0[u], sr, sc)), ftz(ep_fast(a1[u], sr, sc)))) : ep_fast(a0[u], sr, sc);
      }
      if (st && j4 == tid) stamp(a, 707);               // the scales have arrived
      if (kind == 1) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");    // this thread's residual quad
        if (st && j4 == tid) stamp(a, 708);
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = ftz(fadd(sres[j + u], y[u]));
        *reinterpret_cast<float4*>(xout + (uint64_t)m * H + j) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(sx + j) = make_float4(x[0], x[1], x[2], x[3]);
      } else {
        *reinterpret_cast<float4*>(sx + j) = make_float4(ftz(y[0]), ftz(y[1]), ftz(y[2]), ftz(y[3]));
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (st) stamp(a, 701);
  sync_workers();
  if (kind == 2) {
    for (int j = tid; j < H; j += 256) sv[j] = fmul(sx[j], sx[j]);
    const float s = wsum16(sv, H, red);
    const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
    for (int j = tid; j < H; j += 256) {
      const float x = ftz(fadd(sres[j], ftz(fmul(fmul(sx[j], rs), spg[j]))));
      sx[j] = x;
      xout[(uint64_t)m * H + j] = x;
    }
    sync_workers();
  }
  if (st) stamp(a, 702);
  for (int j = tid; j < H; j += 256) sv[j] = fmul(sx[j], sx[j]);
  const float s = wsum16(sv, H, red);
  if (st) stamp(a, 703);
  const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
  float amax = 0.0f;
  for (int j = tid; j < H; j += 256) {
    const float h = ftz(fmul(fmul(sx[j], rs), sg[j]));
    sv[j] = h;
    amax = fmax_c(amax, fabs_c(h));
  }
  amax = wmax(amax, red);
  const float inv = fmul(127.0f, recip_f(amax));
  if (st) stamp(a, 704);
  for (int j = tid; j < H; j += 256) put_q8(a, m, j, q8(sv[j], inv));
  if (tid == 0) qs_out[m] = ftz(fmul(amax, bf(0x3C010204u)));
  sync_workers();                                      // sm is free again
  if (st) stamp(a, 705);
}

// Unit (row m, columns [c0, c0 + cw)) of the gated MLP: g = ep(gate), u = ep(up) from the gate|up
// GEMM's partials, v = ftz(fmul(ftz(act(g)), u)) into gv (llm.py:614-640; the engine's k_quant_cl);
// the unit's absmax into gmax. The unit that arrives last for its row runs the ROW_QUANT of the
// whole row with the row's absmax (max is order-free).
template <int ACT>
__device__ __noinline__ void gated_unit(const StepArgs& a, int m, int c, const StepGemm& g, const float* srow,
                                        float* qs_out, float* red) {
  const int I = a.I, tid = threadIdx.x - 64, nch = a.gchunks;
  const int cw = (I / nch + 1) & ~1, c0 = c * cw, c1 = min(I, c0 + cw);
  const uint64_t ldp = g.col0[g.nseg], slab = (uint64_t)a.B * ldp;
  const int ksplit = g.ksplit;
  const float sr = ftz(srow[m]);
  stamp(a, 710);
  float amax = 0.0f;
  for (int j = c0 + 2 * tid; j < c1; j += 512) {
    const int* p = a.part + (uint64_t)m * ldp + j;
    int ag[2] = {0, 0}, au[2] = {0, 0};
#pragma unroll
    for (int k0 = 0; k0 < 8; k0 += 4) {                // four chunks' loads in flight before their sums
      if (k0 >= ksplit) break;
      int2 vg[4], vu[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (k0 + u < ksplit) {
          vg[u] = *reinterpret_cast<const int2*>(p + (k0 + u) * slab);
          vu[u] = *reinterpret_cast<const int2*>(p + (k0 + u) * slab + I);
        }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (k0 + u < ksplit) {
          ag[0] += vg[u].x; ag[1] += vg[u].y;
          au[0] += vu[u].x; au[1] += vu[u].y;
        }
    }
    const float2 sg2 = *reinterpret_cast<const float2*>(g.scale[0] + j);
    const float2 su2 = *reinterpret_cast<const float2*>(g.scale[1] + j);
    const float sgs[2] = {sg2.x, sg2.y}, sus[2] = {su2.x, su2.y};
    float out[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float gvv = ftz(ep_fast(ag[u], sr, ftz(sgs[u])));
      const float uv = ftz(ep_fast(au[u], sr, ftz(sus[u])));
      float av;
      if constexpr (ACT == 4) av = silu_f(gvv);
      else if constexpr (ACT == 3) av = gelu_f(gvv);
      else av = act_fn(gvv, a.act);
      out[u] = ftz(fmul(ftz(av), uv));
      amax = fmax_c(amax, fabs_c(out[u]));
    }
    *reinterpret_cast<float2*>(a.gv + (uint64_t)m * I + j) = make_float2(out[0], out[1]);
  }
  stamp(a, 711);
  amax = wmax(amax, red);
  stamp(a, 712);
  __shared__ int s_last;
  // every worker's stores are ordered before the counting thread's fence by wmax's barrier, and the
  // fence is cumulative: one fence before the count publishes them all
  if (tid == 0) {
    a.gmax[m * nch + c] = amax;
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync[1 + a.B + m], 1u);
    s_last = (prev + 1) % (unsigned)nch == 0;
  }
  sync_workers();
  stamp(a, 713);
  if (s_last) {                                        // every unit of row m is done
    __threadfence();
    float mx = __ldcg(&a.gmax[m * nch]);
    for (int p = 1; p < nch; ++p) mx = fmax_c(mx, __ldcg(&a.gmax[m * nch + p]));
    const float inv = fmul(127.0f, recip_f(mx));
    quant_row_from(a, m, a.gv + (uint64_t)m * I, I, inv, tid, 256);
    if (tid == 0) qs_out[m] = ftz(fmul(mx, bf(0x3C010204u)));
  }
  sync_workers();
  stamp(a, 714);
}

// ------------------------------------------------------------------------------ attention
// A group of the workers (gt = 256 / ngroups threads, named barrier 3 + group) runs one unit at a
// time; the CTA's groups run their units at the same time, so their memory latencies overlap.
struct Grp {
  int g, gt, tid;                                      // group, its threads, thread in the group
  __device__ __forceinline__ void sync() const {
    asm volatile("barrier.sync %0, %1;" ::"r"(3 + g), "r"(gt) : "memory");
  }
};
// per group: row maxima / reciprocal sums of the softmax, the warps' absmax, the last-arrival flag
struct GrpCtl {
  float rowv[2][16];
  float wred[8];
  int last;
};

// Unit (sequence b, kv head kvh), one token at position t0 = pos[b]: the q | k | v GEMM's epilogue
// for the unit's G query heads and its K / V rows; q / k RMSNorm and RoPE (llm.py:718-734); the
// K / V rows into the caches; scores over keys 0 .. t0 (FDOT NT, 16 lane chains per key), the
// causal softmax, FDOT NN as k-order chains (llm.py:735-746; numerics.py:362-409). Keys past t0
// are masked (probability +0) in the reference; they add nothing to any sum, so they are skipped.
// The output rows go to att, the unit's absmax to amax; the last unit of a sequence to arrive
// quantises the sequence's whole attention row.
template <int HD>
__device__ __noinline__ void attn_unit(const StepArgs& a, const StepLayer& Ly, int b, int kvh, const Grp& gr, float* sm,
                          int tile, GrpCtl* gc) {
  constexpr int LD = HD + 4;
  constexpr int Q4 = HD / 4;
  const int G = a.nh / a.nkv;
  const int tid = gr.tid, gt = gr.gt, warp = tid >> 5, lane = tid & 31, nwarps = gt >> 5;
  float* sq = sm;                                     // [G][HD]
  float* sp = sq + G * HD;                            // [G][kT]
  float* skv = sp + G * kT;                           // [tile][LD]; first the prologue's rows
  const int t0 = a.pos[b];
  const int valid = t0 + 1;
  const StepGemm& g = Ly.qkv;
  const uint64_t ldp = g.col0[g.nseg], slab = (uint64_t)a.B * ldp;
  const float sr = ftz(a.qsa[b]);
  stamp(a, 720);
  float* stab = skv + (2 * G + 3) * HD;               // the RoPE table row of t0, the q / k norm
  float* sgq = stab + HD;                              // gammas: staged while the partials load
  float* sgk = sgq + HD;
  for (int i = tid; i < a.rot / 4; i += gt) cp16(stab + 4 * i, Ly.tab + (uint64_t)t0 * a.rot + 4 * i);
  for (int i = tid; i < Q4; i += gt) {
    cp16(sgq + 4 * i, Ly.qn + 4 * i);
    cp16(sgk + 4 * i, Ly.kn + 4 * i);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // 1. the unit's q | k | v values (G query heads, the K row, the V row) from the partial sums,
  //    four columns per thread with every chunk's load issued before the sums
  const int nq = (G + 2) * Q4;
  for (int i0 = tid; i0 < nq; i0 += 2 * gt) {
    int4 v[2][8];                                      // two quads' chunk loads in flight at once
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = i0 + h * gt;
      if (i >= nq) break;
      const int it = i / Q4, d = 4 * (i - it * Q4);
      const int seg = it < G ? 0 : (it == G ? 1 : 2);
      const int cis = (it < G ? (kvh * G + it) * HD : kvh * HD) + d;
      const int* p = a.part + (uint64_t)b * ldp + g.col0[seg] + cis;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        if (ks < g.ksplit) v[h][ks] = *reinterpret_cast<const int4*>(p + ks * slab);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = i0 + h * gt;
      if (i >= nq) break;
      const int it = i / Q4, d = 4 * (i - it * Q4);
      const int seg = it < G ? 0 : (it == G ? 1 : 2);
      const int cis = (it < G ? (kvh * G + it) * HD : kvh * HD) + d;
      int4 acc = make_int4(0, 0, 0, 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        if (ks < g.ksplit) {
          acc.x += v[h][ks].x;
          acc.y += v[h][ks].y;
          acc.z += v[h][ks].z;
          acc.w += v[h][ks].w;
        }
      const float4 sc = *reinterpret_cast<const float4*>(g.scale[seg] + cis);
      float* dst = skv + it * HD + d;
      dst[0] = ftz(ep_fast(acc.x, sr, ftz(sc.x)));
      dst[1] = ftz(ep_fast(acc.y, sr, ftz(sc.y)));
      dst[2] = ftz(ep_fast(acc.z, sr, ftz(sc.z)));
      dst[3] = ftz(ep_fast(acc.w, sr, ftz(sc.w)));
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  stamp(a, 721);
  gr.sync();
  // 2. per q / K row a half-warp: RMSNorm over the head (16 lane chains, element d to chain
  //    d mod 16), then RoPE with the table row of t0; the V row to the cache as it is
  float* vrow = skv + (G + 1) * HD;
  float* sn = skv + (G + 2) * HD;                      // the normalised rows [G + 1][HD]
  for (int base = 0; base < G + 1; base += gt / 16) {
    const int hw = tid >> 4, l = tid & 15, it = base + hw;
    const bool live = it < G + 1;
    const float* src = skv + (live ? it : 0) * HD;
    float v[HD / 16];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) {
      v[i] = src[l + 16 * i];
      s = fadd_nc(s, fmul(v[i], v[i]));
    }
    s = sum16_fold(canon(s));
    const float rs = rsqrt_f(fadd(fmul(s, recip_f(i2f(HD))), a.eps));
    const float* gam = it < G ? sgq : sgk;
    if (live) {
#pragma unroll
      for (int i = 0; i < HD / 16; ++i) sn[it * HD + l + 16 * i] = ftz(fmul(fmul(v[i], rs), gam[l + 16 * i]));
    }
  }
  gr.sync();
  {
    const float* tab = stab;
    const int half = a.rot / 2;
    float* kdst = Ly.kc + (((uint64_t)b * a.Tp + t0) * a.nkv + kvh) * HD;
    float* vdst = Ly.vc + (((uint64_t)b * a.Tp + t0) * a.nkv + kvh) * HD;
    for (int i = tid; i < (G + 2) * HD; i += gt) {
      const int it = i / HD, j = i - it * HD;
      if (it == G + 1) {
        vdst[j] = vrow[j];
        continue;
      }
      const float* r = sn + it * HD;
      float y;
      if (j < half) y = fadd(fmul(r[j], ftz(tab[j])), neg(fmul(r[j + half], ftz(tab[half + j]))));
      else if (j < a.rot) y = fadd(fmul(r[j], ftz(tab[j - half])), fmul(r[j - half], ftz(tab[j])));
      else y = r[j];
      if (it < G) sq[it * HD + j] = ftz(y);
      else kdst[j] = ftz(y);
    }
  }
  __threadfence_block();                               // the cache rows before the tiles read them
  stamp(a, 722);
  const uint64_t kstride = (uint64_t)a.nkv * HD;
  const float* K = Ly.kc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  const float* V = Ly.vc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  auto stage = [&](const float* src, int j0, int tk) {
    gr.sync();
    for (int i = tid; i < tk * Q4; i += gt) {
      const int j = i / Q4, d4 = i - j * Q4;
      cp16(skv + j * LD + 4 * d4, src + (uint64_t)(j0 + j) * kstride + 4 * d4);
    }
    cp_wait_all();
    gr.sync();
  };
  for (int j0 = 0; j0 < valid; j0 += tile) {
    const int tk = min(tile, valid - j0);
    stage(K, j0, tk);
    for (int p = tid; p < G * tk; p += gt) {
      const int r = p / tk, j = p - r * tk;
      const float* qr = sq + r * HD;
      const float* kr = skv + j * LD;
      float c[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) c[u] = 0.0f;
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
        for (int u = 0; u < 16; u += 2 * w) c[u] = fadd_nc(c[u], c[u + w]);
      sp[r * kT + j0 + j] = ftz(canon(c[0]));
    }
  }
  gr.sync();
  stamp(a, 723);
  // causal softmax over keys 0 .. t0 (numerics.py:362-371)
  for (int r = warp; r < G; r += nwarps) {
    float mx = bf(0xFF800000u);
    for (int j = lane; j < valid; j += 32) mx = fmax_c(mx, sp[r * kT + j]);
    mx = warp_max(mx);
    if (lane == 0) gc->rowv[0][r] = mx;
  }
  gr.sync();
  for (int p = tid; p < G * valid; p += gt) {
    const int r = p / valid, j = p - r * valid;
    sp[r * kT + j] = exp_f(fadd(sp[r * kT + j], neg(gc->rowv[0][r])));
  }
  gr.sync();
  for (int r = warp; r < G; r += nwarps) {
    float acc = 0.0f;                                  // lanes 16..31 repeat lanes 0..15
    for (int j = lane & 15; j < valid; j += 16) acc = fadd_nc(acc, sp[r * kT + j]);
    const float rinv = recip_f(sum16_fold(canon(acc)));
    if (lane == 0) gc->rowv[1][r] = rinv;
  }
  gr.sync();
  for (int p = tid; p < G * valid; p += gt) {
    const int r = p / valid, j = p - r * valid;
    sp[r * kT + j] = ftz(fmul(sp[r * kT + j], gc->rowv[1][r]));
  }
  stamp(a, 724);
  // FDOT NN: out[r][d] = the k-order chain over keys 0 .. t0, V staged tile by tile
  constexpr int kPer = 8;                              // outputs per thread (the host keeps G * HD <= 8 gt)
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
  for (int j0 = 0; j0 < valid; j0 += tile) {
    const int tk = min(tile, valid - j0);
    stage(V, j0, tk);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = tid + i * gt;
      if (o < G * HD) {
        const int r = o / HD, d = o - r * HD;
        const float* pr = sp + r * kT + j0;
        float v = acc[i];
#pragma unroll 8
        for (int j = 0; j < tk; ++j) v = fadd_nc(v, fmul_ff(pr[j], skv[j * LD + d]));
        acc[i] = v;
      }
    }
  }
  stamp(a, 725);
  // the unit's output rows and absmax
  float mx = 0.0f;
  const int qw = a.nh * HD;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = tid + i * gt;
    if (o < G * HD) {
      const float y = ftz(canon(acc[i]));
      const int r = o / HD, d = o - r * HD;
      a.att[(uint64_t)b * qw + (kvh * G + r) * HD + d] = y;
      mx = fmax_c(mx, fabs_c(y));
    }
  }
  mx = warp_max(mx);
  if (lane == 0) gc->wred[warp] = mx;
  gr.sync();
  if (tid == 0) {                                      // (one cumulative fence, as in gated_unit)
    float m = gc->wred[0];
    for (int w = 1; w < nwarps; ++w) m = fmax_c(m, gc->wred[w]);
    a.amax[b * a.nkv + kvh] = m;
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync[1 + b], 1u);
    gc->last = (prev + 1) % (unsigned)a.nkv == 0;
  }
  gr.sync();
  stamp(a, 726);
  if (gc->last) {                                      // every kv head of sequence b is done
    __threadfence();
    float m2 = __ldcg(&a.amax[b * a.nkv]);
    for (int p = 1; p < a.nkv; ++p) m2 = fmax_c(m2, __ldcg(&a.amax[b * a.nkv + p]));
    const float inv = fmul(127.0f, recip_f(m2));
    quant_row_from(a, b, a.att + (uint64_t)b * qw, qw, inv, tid, gt);
    if (tid == 0) a.qsb[b] = ftz(fmul(m2, bf(0x3C010204u)));
  }
  gr.sync();
  stamp(a, 727);
}

// ------------------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) k_step(const __grid_constant__ StepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], accf[2], acce[2], actb, drain;
  __shared__ uint32_t s_tmem;
  __shared__ Ctl ctl;
  __shared__ GrpCtl gctl[4];
  __shared__ float s_tok[kStepMaxTok];
  __shared__ float red[40];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ring = smem;
  uint8_t* region = smem + kStages * kSliceB;
  float* sm = reinterpret_cast<float*>(region);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t ncols = 32;
  while (ncols < 2u * a.ntok) ncols <<= 1;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 8);
    }
    mbar_init(&actb, 1);
    mbar_init(&drain, 1);
    ctl.abort = 0;
    ctl.go = 1;
    ctl.gen = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 64) a.trace[0] = gtime();

  uint32_t issued = 0;
  MmaState ms;
  uint32_t etiles = 0;
  if (warp == 0) {
    if (lane == 0) issued = produce(a, ring, full, empty, &ctl);
  } else {
    const bool mma_lane = warp == 1 && lane == 0;
    auto gemm = [&](const StepGemm& g, bool fused) {
      if (warp == 1) {
        if (mma_lane) mma_phase(a, g, ring, region, full, empty, accf, acce, &actb, tmem, ms, &ctl, fused);
        __syncwarp();
      } else {
        epi_phase(a, g, fused, tmem, accf, acce, etiles, &ctl, s_tok);
      }
    };
    const int grid = gridDim.x;
    const bool worker = warp >= 2;
    bool alive = true;                                 // the same in every thread of warps 1-9
    auto barrier = [&]() { return alive = grid_sync(a, &ctl); };
    for (int l = 0; l < a.L; ++l) {
      const StepLayer& Ly = a.layers[l];
      const StepLayer* Lp = l ? &a.layers[l - 1] : nullptr;
      // ln_in + quant of the residual stream (after the previous layer's down projection)
      if (worker)
        for (int m = blockIdx.x; m < a.B; m += grid)
          norm_row(a, m, l == 0 ? 0 : (a.gemma ? 2 : 1), Lp ? &Lp->down : nullptr, a.qsb, a.x1, a.x,
                   Lp ? Lp->mlp_norm : nullptr, Ly.ln_in, a.qsa, sm, red);
      if (!barrier()) break;
      gemm(Ly.qkv, false);
      if (!barrier()) break;
      if (worker) {
        // the CTA's ngroups groups each take units blockIdx.x * ngroups + group, + grid * ngroups ..
        const int ng = a.agroups, wt = threadIdx.x - 64;
        const Grp gr{wt / (256 / ng), 256 / ng, wt % (256 / ng)};
        float* gsm = sm + gr.g * (kRegion / 4 / ng);
        for (int u = blockIdx.x * ng + gr.g; u < a.B * a.nkv; u += grid * ng) {
          if (a.hd == 128) attn_unit<128>(a, Ly, u / a.nkv, u % a.nkv, gr, gsm, a.tile, &gctl[gr.g]);
          else if (a.hd == 256) attn_unit<256>(a, Ly, u / a.nkv, u % a.nkv, gr, gsm, a.tile, &gctl[gr.g]);
          else attn_unit<64>(a, Ly, u / a.nkv, u % a.nkv, gr, gsm, a.tile, &gctl[gr.g]);
        }
      }
      if (!barrier()) break;
      gemm(Ly.o, false);
      if (!barrier()) break;
      // x1 = x + o (Gemma: x + attn_norm(o)), then ln_post + quant
      if (worker)
        for (int m = blockIdx.x; m < a.B; m += grid)
          norm_row(a, m, a.gemma ? 2 : 1, &Ly.o, a.qsb, a.x, a.x1, Ly.attn_norm, Ly.ln_post, a.qsa, sm, red);
      if (!barrier()) break;
      gemm(Ly.gu, false);
      if (!barrier()) break;
      if (worker)
        for (int u = blockIdx.x; u < a.B * a.gchunks; u += grid) {
          const int m = u / a.gchunks, c = u - m * a.gchunks;
          if (a.act == 4) gated_unit<4>(a, m, c, Ly.gu, a.qsa, a.qsb, red);
          else if (a.act == 3) gated_unit<3>(a, m, c, Ly.gu, a.qsa, a.qsb, red);
          else gated_unit<-1>(a, m, c, Ly.gu, a.qsa, a.qsb, red);
        }
      if (!barrier()) break;
      gemm(Ly.down, false);
      if (!barrier()) break;
    }
    if (alive) {
      // the last layer's residual, the final norm + quant, the head (logits through its epilogue)
      const StepLayer& Lp = a.layers[a.L - 1];
      if (worker)
        for (int m = blockIdx.x; m < a.B; m += grid)
          norm_row(a, m, a.gemma ? 2 : 1, &Lp.down, a.qsb, a.x1, a.x, Lp.mlp_norm, a.final_norm, a.qsa, sm, red);
      if (barrier()) {
        gemm(a.head, true);
        if (a.trace)                                   // the head's end; then four empty phases
          for (int i = 0; i < 5 && barrier(); ++i) {
          }
      }
    }
    if (mma_lane && ms.q > 0) {
      // every MMA issued completes before TMEM is freed
      mma_commit(&drain);
      drain_wait(&drain, 0, a.drain_ns);
    }
  }
  __syncwarp();                                        // lane 0 of warps 0 / 1 rejoins its warp
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  if (threadIdx.x == 0 && *(volatile int*)&ctl.abort) {
    // after a give-up, weight slices issued but never consumed land before the block exits
    for (uint32_t i = issued > (uint32_t)kStages ? issued - kStages : 0; i < issued; ++i)
      drain_wait(&full[i % kStages], (i / kStages) & 1, a.drain_ns);
  }
}

// One thread per 16-byte chunk of the re-laid-out weight (step.h's [tile][slice] blocks).
__global__ void k_retile(const int8_t* w, const int8_t* w2, int n, int K, int kb, uint8_t* out) {
  const int nslices = K / 128, ntiles = (n + 127) / 128;
  const uint64_t total = (uint64_t)ntiles * nslices * 128 * 8;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t chunk = (uint32_t)(i & 7), r = (uint32_t)((i >> 3) & 127);
    const uint64_t ts = i >> 10;                          // tile * nslices + slice
    const int k = (int)(ts % nslices), t = (int)(ts / nslices);
    const int row = t * 128 + (int)r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < n) {
      const int kk = k * 128 + (int)chunk * 16;
      const int8_t* src = kk < kb ? w + (uint64_t)row * kb + kk : w2 + (uint64_t)row * (K - kb) + (kk - kb);
      v = *reinterpret_cast<const uint4*>(src);
    }
    *reinterpret_cast<uint4*>(out + ts * kSliceB + step_swz(r, chunk * 16)) = v;
  }
}

}  // namespace

size_t step_smem_bytes() { return (size_t)kStages * kSliceB + kRegion + 1024; }
int step_region_bytes() { return kRegion; }

int step_attn_tile(int hd, int G, int ngroups) {
  const int region = kRegion / ngroups;
  const int fixed = (G * hd + G * kT) * 4;
  const int per = (hd + 4) * 4;
  const int scratch = (2 * G + 6) * hd * 4;            // the prologue's rows, RoPE row and norm gammas
  int tile = (region - fixed) / per / 16 * 16;
  tile = std::min(tile, kT);
  if (tile < 16 || tile * per < scratch || G * hd > 8 * (256 / ngroups)) return 0;
  return tile;
}

bool step_plan_gemm(StepGemm& g, int ntok, int grid, bool fused) {
  const int ntiles = g.tile0[g.nseg];
  const int maxkc = kRegion / (ntok * 128);
  if (ntiles < 1 || g.nslices < 1 || maxkc < 1) return false;
  const bool two = g.kb < g.nslices;
  int KC;
  if (fused) {
    if (two || g.nslices > maxkc) return false;
    KC = g.nslices;
  } else {
    // enough K chunks to give every CTA work (at most 8 partial sums per output), K chunks of at
    // most maxkc slices that never straddle the boundary of two K blocks
    // TARSCUDA_STEP_KSPLIT caps the partial sums per output (fewer chunks: fewer CTAs stream the
    // weights, less int32 traffic for the phase after the GEMM)
    static const int cap = [] {
      const char* v = getenv("TARSCUDA_STEP_KSPLIT");
      const int c = v ? atoi(v) : 8;
      return c >= 1 && c <= 8 ? c : 8;
    }();
    const int want = std::min(cap, std::max(1, (grid + ntiles - 1) / ntiles));
    KC = std::min(maxkc, (g.nslices + want - 1) / want);
    if (two) {
      int up = KC;
      while (up <= maxkc && g.kb % up) ++up;            // the next divisor of the first block
      if (up <= maxkc) KC = up;
      else
        while (KC > 1 && g.kb % KC) --KC;
    }
  }
  g.KC = KC;
  g.ksplit = (g.nslices + KC - 1) / KC;
  g.groups = grid / g.ksplit;
  return g.groups >= 1 && g.ksplit <= 8;
}

cudaError_t step_occupancy(int* per_sm) {
  const size_t smem = step_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_step, kThreads, smem);
}

cudaError_t step_retile(const int8_t* w, const int8_t* w2, int n, int K, int kb, uint8_t* out, cudaStream_t st) {
  if (n < 1 || K % 128 || kb % 128 || kb < 128 || kb > K || (kb < K && !w2) || ((uintptr_t)w | (uintptr_t)w2) % 16)
    return cudaErrorInvalidValue;
  const uint64_t total = (uint64_t)((n + 127) / 128) * (K / 128) * 1024;
  const int blocks = (int)std::min<uint64_t>((total + 255) / 256, 148 * 16);
  k_retile<<<blocks, 256, 0, st>>>(w, w2, n, K, kb, out);
  return cudaGetLastError();
}

cudaError_t step_launch(const StepArgs& a, int grid, cudaStream_t st) {
  const size_t smem = step_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_step, a);
}

}  // namespace tc
