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
  int last;
  float rowv[2][16];
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
__device__ bool grid_sync(const StepArgs& a, Ctl* ctl) {
  fence_proxy_async();                                   // generic writes, later read by bulk copies
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // shared memory that copies overwrite next
  sync_main();
  if (threadIdx.x == 64) {
    const unsigned gen = ctl->gen + 1;
    ctl->gen = gen;
    bool ok = !*(volatile int*)&ctl->abort;
    if (ok) {
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
      if (a.trace && blockIdx.x == 0) a.trace[gen] = gtime();
    }
    ctl->go = ok;
  }
  sync_main();
  return *(volatile int*)&ctl->go != 0;
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
__device__ uint32_t produce(const StepArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty, Ctl* ctl) {
  uint32_t q = 0;
  auto gemm = [&](const StepGemm& g) -> bool {
    int ks, grp;
    if (!my_chunk(g, ks, grp)) return true;
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
    ok = gemm(Ly.qkv) && gemm(Ly.o) && gemm(Ly.gu) && gemm(Ly.down);
  }
  if (ok) gemm(a.head);
  return q;
}

// ------------------------------------------------------------------------------ GEMM phase
struct MmaState {
  uint32_t q = 0, tiles = 0, nact = 0;
};

// warp 1, lane 0: the K chunk of the rows into shared memory, then per row tile the chunk's MMAs
__device__ bool mma_phase(const StepArgs& a, const StepGemm& g, uint8_t* ring, uint8_t* region, uint64_t* full,
                          uint64_t* empty, uint64_t* accf, uint64_t* acce, uint64_t* actb, uint32_t tmem, MmaState& st,
                          Ctl* ctl) {
  int ks, grp;
  if (!my_chunk(g, ks, grp)) return true;
  const int k0 = ks * g.KC, kc = min(g.nslices, k0 + g.KC) - k0;
  const uint32_t xb = (uint32_t)a.ntok * 128;
  fence_proxy_async();
  mbar_expect_tx(actb, kc * xb);
  bulk_load(region, a.q8t + (uint64_t)k0 * xb, kc * xb, actb);
  const uint32_t par = st.nact & 1;
  ++st.nact;
  if (!wait_or_abort(actb, par, a, ctl, 42)) {
    drain_wait(actb, par, a.drain_ns);                  // the rows' copy lands before anything else
    return false;
  }
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
      tc_fence_after();
      const uint32_t sa = smem_u32(ring + slot * kSliceB), sb = smem_u32(region + i * xb);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_i8(d, sdesc_k128(sa + 32 * kk), sdesc_k128(sb + 32 * kk), idesc, (i | kk) ? 1u : 0u);
      mma_commit(&empty[slot]);
    }
    mma_commit(&accf[buf]);
  }
  return true;
}

// warps 2-9: each accumulator to the partial sums (or, for the head, through the epilogue to the
// logits). Warp w reads TMEM lanes 32 (w % 4) .. (weight rows); warps 2-5 the even 16-token
// chunks, 6-9 the odd ones.
__device__ bool epi_phase(const StepArgs& a, const StepGemm& g, bool fused, uint32_t tmem, uint64_t* accf,
                          uint64_t* acce, uint32_t& tiles, Ctl* ctl) {
  int ks, grp;
  if (!my_chunk(g, ks, grp)) return true;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp & 3, half = (warp - 2) >> 2, r = ew * 32 + lane;
  const uint32_t tlane = tmem + ((uint32_t)(ew * 32) << 16);
  const int ntiles = g.tile0[g.nseg];
  const int ldp = g.col0[g.nseg];
  const int last = (a.ntok - 16 - 16 * half) / 32 * 32 + 16 * half;
  for (int t = grp; t < ntiles; t += g.groups, ++tiles) {
    const int buf = tiles & 1;
    const uint32_t use = tiles >> 1;
    const int s = seg_of(g, t);
    const int rr = (t - g.tile0[s]) * 128 + r;
    const bool live = rr < g.col0[s + 1] - g.col0[s];
    const int col = g.col0[s] + rr;
    const float sc = (fused && live) ? ftz(g.scale[s][rr]) : 0.0f;
    const bool ok = wait_or_abort(&accf[buf], use & 1, a, ctl, 45);
    if (!__all_sync(0xFFFFFFFFu, ok)) return false;
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
          if (m < a.B) a.logits[(uint64_t)m * a.vocab + col] = ftz(ep_fast((int)v[j], ftz(a.qsa[m]), sc));
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

// ------------------------------------------------------------------------------ row phases
// Row m of the residual stream, then its RMSNorm (gamma) and ROW_QUANT (llm.py:97-104;
// numerics.py:353-390):
//   kind 0  x = E[tok] (Gemma: times fp32(sqrt(H)), in IEEE fp32 as the host computes it)
//   kind 1  x = res + ep(the GEMM's partials)                       (Qwen3: after o / down)
//   kind 2  x = res + rmsnorm(y, pre_gamma), y the GEMM's output    (Gemma 3: attn / mlp norm)
// x is written to xout. The K-split GEMM (two K blocks sharing the scales): y = ep(acc_1) + ep(acc_2).
__device__ void norm_row(const StepArgs& a, int m, int kind, const StepGemm* g, const float* srow, const float* res,
                         float* xout, const float* pre_gamma, const float* gamma, float* qs_out, float* sm, float* red) {
  const int H = a.H, tid = threadIdx.x - 64;
  float* sx = sm;
  float* sv = sm + H;
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
    const int ldp = g->col0[g->nseg];
    const bool two = g->kb < g->nslices;
    const int nb1 = two ? g->kb / g->KC : g->ksplit;
    const float* scale = g->scale[0];
    for (int j = tid; j < H; j += 256) {
      int a0 = 0, a1 = 0;
      for (int ks = 0; ks < g->ksplit; ++ks) {
        const int v = a.part[((uint64_t)ks * a.B + m) * ldp + j];
        if (ks < nb1) a0 += v;
        else a1 += v;
      }
      const float sc = ftz(scale[j]);
      const float y = two ? ftz(fadd(ftz(ep_fast(a0, sr, sc)), ftz(ep_fast(a1, sr, sc)))) : ep_fast(a0, sr, sc);
      if (kind == 1) {
        const float x = ftz(fadd(res[(uint64_t)m * H + j], y));
        xout[(uint64_t)m * H + j] = x;
        sx[j] = x;
      } else {
        sx[j] = ftz(y);
      }
    }
  }
  sync_workers();
  if (kind == 2) {
    for (int j = tid; j < H; j += 256) sv[j] = fmul(sx[j], sx[j]);
    const float s = wsum16(sv, H, red);
    const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
    for (int j = tid; j < H; j += 256) {
      const float x = ftz(fadd(res[(uint64_t)m * H + j], ftz(fmul(fmul(sx[j], rs), pre_gamma[j]))));
      sx[j] = x;
      xout[(uint64_t)m * H + j] = x;
    }
    sync_workers();
  }
  for (int j = tid; j < H; j += 256) sv[j] = fmul(sx[j], sx[j]);
  const float s = wsum16(sv, H, red);
  const float rs = rsqrt_f(fadd(fmul(s, kinv), a.eps));
  float amax = 0.0f;
  for (int j = tid; j < H; j += 256) {
    const float h = ftz(fmul(fmul(sx[j], rs), gamma[j]));
    sv[j] = h;
    amax = fmax_c(amax, fabs_c(h));
  }
  amax = wmax(amax, red);
  const float inv = fmul(127.0f, recip_f(amax));
  for (int j = tid; j < H; j += 256) put_q8(a, m, j, q8(sv[j], inv));
  if (tid == 0) qs_out[m] = ftz(fmul(amax, bf(0x3C010204u)));
  sync_workers();                                      // sm is free again
}

// Row m of the gated MLP: g = ep(gate), u = ep(up) from the gate|up GEMM's partials, v =
// ftz(fmul(ftz(act(g)), u)), then ROW_QUANT of v (llm.py:614-640; the engine's k_quant_cl)
template <int ACT>
__device__ void gated_row(const StepArgs& a, int m, const StepGemm& g, const float* srow, float* qs_out, float* sm,
                          float* red) {
  const int I = a.I, tid = threadIdx.x - 64;
  const int ldp = g.col0[g.nseg];
  const float sr = ftz(srow[m]);
  float amax = 0.0f;
  for (int j = tid; j < I; j += 256) {
    int ag = 0, au = 0;
    for (int ks = 0; ks < g.ksplit; ++ks) {
      const int* p = a.part + ((uint64_t)ks * a.B + m) * ldp;
      ag += p[j];
      au += p[I + j];
    }
    const float gv = ftz(ep_fast(ag, sr, ftz(g.scale[0][j])));
    const float uv = ftz(ep_fast(au, sr, ftz(g.scale[1][j])));
    float av;
    if constexpr (ACT == 4) av = silu_f(gv);
    else if constexpr (ACT == 3) av = gelu_f(gv);
    else av = act_fn(gv, a.act);
    const float v = ftz(fmul(ftz(av), uv));
    sm[j] = v;
    amax = fmax_c(amax, fabs_c(v));
  }
  amax = wmax(amax, red);
  const float inv = fmul(127.0f, recip_f(amax));
  for (int j = tid; j < I; j += 256) put_q8(a, m, j, q8(sm[j], inv));
  if (tid == 0) qs_out[m] = ftz(fmul(amax, bf(0x3C010204u)));
  sync_workers();
}

// ------------------------------------------------------------------------------ attention
// Unit (sequence b, kv head kvh), one token at position t0 = pos[b]: the q | k | v GEMM's epilogue
// for the unit's G query heads and its K / V rows; q / k RMSNorm and RoPE (llm.py:718-734); the
// K / V rows into the caches; scores over keys 0 .. t0 (FDOT NT, 16 lane chains per key), the
// causal softmax, FDOT NN as k-order chains (llm.py:735-746; numerics.py:362-409). Keys past t0
// are masked (probability +0) in the reference; they add nothing to any sum, so they are skipped.
// The output rows go to att, the unit's absmax to amax; the last unit of a sequence to arrive
// quantises the sequence's whole attention row.
template <int HD>
__device__ void attn_unit(const StepArgs& a, const StepLayer& Ly, int b, int kvh, float* sm, float* red, Ctl* ctl) {
  constexpr int LD = HD + 4;
  const int G = a.nh / a.nkv;
  const int tid = threadIdx.x - 64, warp = tid >> 5, lane = tid & 31;
  float* sq = sm;                                     // [G][HD]
  float* sp = sq + G * HD;                            // [G][kT]
  float* skv = sp + G * kT;                           // [tile][LD]
  const int t0 = a.pos[b];
  const int valid = t0 + 1;
  const StepGemm& g = Ly.qkv;
  const int ldp = g.col0[g.nseg];
  const float sr = ftz(a.qsa[b]);
  {
    // half-warp hw: item hw = query head kvh * G + hw (hw < G), the K row (G), the V row (G + 1)
    const int hw = tid >> 4, l = tid & 15;
    const int items = G + 2;
    const bool live = hw < items;
    const int it = live ? hw : 0;
    const int seg = it < G ? 0 : (it == G ? 1 : 2);
    const int cis = it < G ? (kvh * G + it) * HD : kvh * HD;
    float v[HD / 16];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) {
      const int d = l + 16 * i;
      const int col = g.col0[seg] + cis + d;
      int acc = 0;
      for (int ks = 0; ks < g.ksplit; ++ks) acc += a.part[((uint64_t)ks * a.B + b) * ldp + col];
      v[i] = ftz(ep_fast(acc, sr, ftz(g.scale[seg][cis + d])));
      s = fadd_nc(s, fmul(v[i], v[i]));
    }
    s = sum16_fold(canon(s));
    // the two half-warps of a warp may take different branches below: both __syncwarp calls stay
    // outside them, so every lane of the warp meets at the same two points
    float* sn = skv + hw * HD;
    const bool qk = it <= G;                           // a query head or the K row: norm + RoPE
    if (qk) {
      const float rs = rsqrt_f(fadd(fmul(s, recip_f(i2f(HD))), a.eps));
      const float* gam = it < G ? Ly.qn : Ly.kn;
#pragma unroll
      for (int i = 0; i < HD / 16; ++i) sn[l + 16 * i] = ftz(fmul(fmul(v[i], rs), gam[l + 16 * i]));
    }
    __syncwarp();
    if (live && qk) {
      const float* tab = Ly.tab + (uint64_t)t0 * a.rot;
      const int half = a.rot / 2;
      float* dst = it < G ? sq + it * HD : Ly.kc + (((uint64_t)b * a.Tp + t0) * a.nkv + kvh) * HD;
      for (int j = l; j < HD; j += 16) {
        float y;
        if (j < half) y = fadd(fmul(sn[j], ftz(tab[j])), neg(fmul(sn[j + half], ftz(tab[half + j]))));
        else if (j < a.rot) y = fadd(fmul(sn[j], ftz(tab[j - half])), fmul(sn[j - half], ftz(tab[j])));
        else y = sn[j];
        dst[j] = ftz(y);
      }
    } else if (live) {                                 // V goes to the cache as the GEMM gave it
      float* vd = Ly.vc + (((uint64_t)b * a.Tp + t0) * a.nkv + kvh) * HD;
#pragma unroll
      for (int i = 0; i < HD / 16; ++i) vd[l + 16 * i] = v[i];
    }
    __syncwarp();
  }
  __threadfence_block();                               // the cache rows before the tiles read them
  const int tile = a.tile;
  const uint64_t kstride = (uint64_t)a.nkv * HD;
  const float* K = Ly.kc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  const float* V = Ly.vc + ((uint64_t)b * a.Tp * a.nkv + kvh) * HD;
  auto stage = [&](const float* src, int j0, int tk) {
    sync_workers();
    for (int i = tid; i < tk * (HD / 4); i += 256) {
      const int j = i / (HD / 4), d4 = i - j * (HD / 4);
      cp16(skv + j * LD + 4 * d4, src + (uint64_t)(j0 + j) * kstride + 4 * d4);
    }
    cp_wait_all();
    sync_workers();
  };
  for (int j0 = 0; j0 < valid; j0 += tile) {
    const int tk = min(tile, valid - j0);
    stage(K, j0, tk);
    for (int p = tid; p < G * tk; p += 256) {
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
  sync_workers();
  // causal softmax over keys 0 .. t0 (numerics.py:362-371)
  for (int r = warp; r < G; r += 8) {
    float mx = bf(0xFF800000u);
    for (int j = lane; j < valid; j += 32) mx = fmax_c(mx, sp[r * kT + j]);
    mx = warp_max(mx);
    if (lane == 0) ctl->rowv[0][r] = mx;
  }
  sync_workers();
  for (int p = tid; p < G * valid; p += 256) {
    const int r = p / valid, j = p - r * valid;
    sp[r * kT + j] = exp_f(fadd(sp[r * kT + j], neg(ctl->rowv[0][r])));
  }
  sync_workers();
  for (int r = warp; r < G; r += 8) {
    float acc = 0.0f;                                  // lanes 16..31 repeat lanes 0..15
    for (int j = lane & 15; j < valid; j += 16) acc = fadd_nc(acc, sp[r * kT + j]);
    const float rinv = recip_f(sum16_fold(canon(acc)));
    if (lane == 0) ctl->rowv[1][r] = rinv;
  }
  sync_workers();
  for (int p = tid; p < G * valid; p += 256) {
    const int r = p / valid, j = p - r * valid;
    sp[r * kT + j] = ftz(fmul(sp[r * kT + j], ctl->rowv[1][r]));
  }
  // FDOT NN: out[r][d] = the k-order chain over keys 0 .. t0, V staged tile by tile
  constexpr int kPer = (16 * HD + 255) / 256;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
  for (int j0 = 0; j0 < valid; j0 += tile) {
    const int tk = min(tile, valid - j0);
    stage(V, j0, tk);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int o = tid + i * 256;
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
  // the unit's output rows and absmax
  float mx = 0.0f;
  const int qw = a.nh * HD;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int o = tid + i * 256;
    if (o < G * HD) {
      const float y = ftz(canon(acc[i]));
      const int r = o / HD, d = o - r * HD;
      a.att[(uint64_t)b * qw + (kvh * G + r) * HD + d] = y;
      mx = fmax_c(mx, fabs_c(y));
    }
  }
  mx = wmax(mx, red);
  if (tid == 0) {
    a.amax[b * a.nkv + kvh] = mx;
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync[1 + b], 1u);
    ctl->last = (prev + 1) % (unsigned)a.nkv == 0;
  } else {
    __threadfence();
  }
  sync_workers();
  if (ctl->last) {                                     // every kv head of sequence b is done
    __threadfence();
    float m2 = __ldcg(&a.amax[b * a.nkv]);
    for (int p = 1; p < a.nkv; ++p) m2 = fmax_c(m2, __ldcg(&a.amax[b * a.nkv + p]));
    const float inv = fmul(127.0f, recip_f(m2));
    for (int c = tid; c < qw; c += 256) put_q8(a, b, c, q8(__ldcg(&a.att[(uint64_t)b * qw + c]), inv));
    if (tid == 0) a.qsb[b] = ftz(fmul(m2, bf(0x3C010204u)));
  }
  sync_workers();
}

// ------------------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) k_step(const __grid_constant__ StepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], accf[2], acce[2], actb, drain;
  __shared__ uint32_t s_tmem;
  __shared__ Ctl ctl;
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
    ctl.last = 0;
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
        if (mma_lane) mma_phase(a, g, ring, region, full, empty, accf, acce, &actb, tmem, ms, &ctl);
        __syncwarp();
      } else {
        epi_phase(a, g, fused, tmem, accf, acce, etiles, &ctl);
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
      if (worker)
        for (int u = blockIdx.x; u < a.B * a.nkv; u += grid) {
          if (a.hd == 128) attn_unit<128>(a, Ly, u / a.nkv, u % a.nkv, sm, red, &ctl);
          else if (a.hd == 256) attn_unit<256>(a, Ly, u / a.nkv, u % a.nkv, sm, red, &ctl);
          else attn_unit<64>(a, Ly, u / a.nkv, u % a.nkv, sm, red, &ctl);
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
        for (int m = blockIdx.x; m < a.B; m += grid) {
          if (a.act == 4) gated_row<4>(a, m, Ly.gu, a.qsa, a.qsb, sm, red);
          else if (a.act == 3) gated_row<3>(a, m, Ly.gu, a.qsa, a.qsb, sm, red);
          else gated_row<-1>(a, m, Ly.gu, a.qsa, a.qsb, sm, red);
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
        if (a.trace) barrier();                        // the head's end, for the phase times
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

int step_attn_tile(int hd, int G) {
  const int fixed = (G * hd + G * kT) * 4;
  const int per = (hd + 4) * 4;
  const int scratch = 16 * hd * 4;                     // the prologue's 16 half-warp rows
  int tile = (kRegion - fixed) / per / 16 * 16;
  tile = std::min(tile, kT);
  if (tile * per < scratch) return 0;
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
    const int want = std::min(8, std::max(1, (grid + ntiles - 1) / ntiles));
    KC = std::min(maxkc, (g.nslices + want - 1) / want);
    if (two) {
      while (KC > 1 && g.kb % KC) --KC;
    }
  }
  g.KC = KC;
  g.ksplit = (g.nslices + KC - 1) / KC;
  g.groups = grid / g.ksplit;
  return g.groups >= 1;
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
