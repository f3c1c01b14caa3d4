// The batched decode engine (host side): resident model, per-sequence KV caches, one CUDA graph
// per chunk length, a device-side position counter and greedy pick.
//
// It replaces, for B sequences at once, the per-step path of the reference's QwenLowering.generate
// (tars_mini/llm.py:815-836) and the board runtime's Qwen.step / prefill (deploy/kv260/sw/
// tars_board.py:400-435): embedding lookup, every layer, the final norm, the head and the argmax
// run on the GPU; the host only moves token ids (and logits when asked). The weights are read
// from the DDR image the lowering laid out (the same bytes the descriptor path executes).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/tarscuda.h"
#include "../../include/tarscuda_engine.h"
#include "engine.h"
#include "pdl.cuh"
#include "mma.h"
#include "step.h"

using namespace tc;

struct tc_machine;
extern "C" uint64_t tc_device_ptr(tc_machine* m);

namespace tc {
bool& pdl_launches() {
  static thread_local bool on = false;
  return on;
}
}  // namespace tc

namespace {
struct Lin { const int8_t* W; const float* s; int n, k; };
struct Layer {
  const float *ln_in, *ln_post, *attn_norm, *mlp_norm, *qn, *kn, *tab;
  Lin q, k, v, o, gate, up;
  Lin down[4];
  int n_down;
};
}  // namespace

struct tc_engine {
  int device = 0;
  cudaStream_t st = nullptr;
  tc_model_desc md{};
  std::vector<Layer> layers;
  std::vector<Lin> head;
  const float* final_norm = nullptr;
  int B = 0, T = 0, Tp = 0, nmax = 4, H = 0, I = 0, qw = 0, kvw = 0;
  // device buffers
  float* E = nullptr;                       // fp32 embedding table [vocab][H]
  int *tok = nullptr, *next = nullptr, *pos = nullptr;
  float *x = nullptr, *x1 = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *att = nullptr;
  float *o = nullptr, *g = nullptr, *u = nullptr, *d = nullptr, *logits = nullptr;
  int8_t* q8 = nullptr;                      // quantised rows [M][max(H, I, qw)]
  float* qs = nullptr;
  float *kc = nullptr, *vc = nullptr;        // [L][B][Tp][kvw]
  cudaGraphExec_t graph[5] = {};
  // q / k norm + RoPE, attention and the output quantiser as one cluster launch
  // (TARSCUDA_FUSE_ATTN=0: three launches, the same bits)
  bool fuse_attn = true;
  std::string err;
  // the fused decode step (step.h) for one-token steps, when the model and batch fit it
  bool step_ok = false;
  int grid = 0;
  StepArgs sa{};
  std::vector<StepLayer> slayers;
  StepLayer* d_layers = nullptr;
  uint8_t* wt = nullptr;                     // the weights re-laid out for the fused step
  uint8_t* q8t = nullptr;                    // its int8 rows in the operand layout
  int* sdiag = nullptr;
  float* qs2 = nullptr;
  int* part = nullptr;
  float *satt = nullptr, *samax = nullptr, *sgv = nullptr, *sgmax = nullptr;
  unsigned* ssync = nullptr;
  unsigned long long* strace = nullptr;
  int ntrace = 0;
  std::string step_why;                      // why the fused step is not used, when it is not
  std::vector<int> hpos;                     // the host's copy of every sequence's position
  // profiling (tc_engine_profile): events around every kernel of one uncaptured step
  bool prof = false;
  std::vector<cudaEvent_t> pev;
  std::vector<int> pkind;
  std::vector<uint64_t> pbytes;
};

namespace {
constexpr bool kFusedDefault = false;
int fail(tc_engine* e, const char* what, cudaError_t c) {
  e->err = std::string(what) + ": " + cudaGetErrorString(c);
  return TC_ERR_CUDA;
}
// A step of n tokens per sequence may run only while every sequence has room for them: the KV
// caches and RoPE tables hold max_tokens positions. Advances the host's copy of the positions.
bool take_positions(tc_engine* e, int n) {
  for (int p : e->hpos)
    if (p + n > e->T) {
      e->err = "a sequence would pass max_tokens (reset it first)";
      return false;
    }
  for (int& p : e->hpos) p += n;
  return true;
}
#define TRY(expr)                                   \
  do {                                              \
    cudaError_t _c = (expr);                        \
    if (_c != cudaSuccess) return fail(e, #expr, _c); \
  } while (0)

// A kernel launch of the step; when profiling, bracketed by events and tagged with its kind and
// algorithmic bytes.
enum { kKEmbed, kKNormQuant, kKGemv, kKQkRope, kKAttention, kKQuant, kKArgmax, kKAdvance };
#define KERNEL(kind, bytes, expr)                                              \
  do {                                                                         \
    if (e->prof) {                                                             \
      cudaEvent_t _a, _b;                                                      \
      cudaEventCreate(&_a);                                                    \
      cudaEventCreate(&_b);                                                    \
      cudaEventRecordWithFlags(_a, e->st, cudaEventRecordExternal);            \
      TRY(expr);                                                               \
      cudaEventRecordWithFlags(_b, e->st, cudaEventRecordExternal);            \
      e->pev.push_back(_a);                                                    \
      e->pev.push_back(_b);                                                    \
      e->pkind.push_back(kind);                                                \
      e->pbytes.push_back(bytes);                                              \
    } else {                                                                   \
      TRY(expr);                                                               \
    }                                                                          \
  } while (0)

Lin lin_of(const uint8_t* base, const tc_lin& l) {
  return Lin{(const int8_t*)(base + l.w_off), (const float*)(base + l.s_off), l.n, l.k};
}
const float* vec_of(const uint8_t* base, uint64_t off) { return off ? (const float*)(base + off) : nullptr; }

EngGemvArgs gemv_args(const int8_t* A, uint64_t lda, const float* srow, int M, int K) {
  EngGemvArgs g{};
  g.A = A; g.lda = lda; g.srow = srow; g.M = M; g.K = K; g.kb = K;
  return g;
}
void add_seg(EngGemvArgs& g, const Lin& l, float* out, uint64_t ldo) {
  EngSeg& s = g.seg[g.nseg++];
  s.W = l.W; s.scale = l.s; s.out = out; s.ldo = ldo; s.n0 = g.ncols; s.n = l.n;
  g.ncols += l.n;
}

// The algorithmic bytes of one engine GEMV: every weight row and scale once, the int8 rows and
// their scales, the fp32 outputs (and residual rows read).
uint64_t gemv_bytes(const EngGemvArgs& g) {
  uint64_t b = (uint64_t)g.M * g.K + 4ull * g.M;
  for (int s = 0; s < g.nseg; ++s) b += (uint64_t)g.seg[s].n * g.K + 4ull * g.seg[s].n;
  const uint64_t ncols = g.mode == kEpiGated ? g.seg[0].n : g.ncols;
  b += 4ull * g.M * ncols * (g.res ? 2 : 1);
  return b;
}

// Enqueues one step for chunks of n tokens per sequence, starting at the device position.
int enqueue_step(tc_engine* e, int n, const int* tok_in) {
  const tc_model_desc& md = e->md;
  const int B = e->B, M = B * n, H = e->H, I = e->I, qw = e->qw, kvw = e->kvw;
  const int ldq = std::max(std::max(H, I), qw);
  cudaStream_t st = e->st;
  KERNEL(kKEmbed, (uint64_t)M * H * 8, eng_embed(e->E, tok_in, e->x, H, md.gemma, md.embed_scale, M, st));
  const float eps = md.eps;
  for (int li = 0; li < md.n_layers; ++li) {
    const Layer& L = e->layers[li];
    float* kc = e->kc + (uint64_t)li * B * e->Tp * kvw;
    float* vc = e->vc + (uint64_t)li * B * e->Tp * kvw;
    // ln_in + quant (for li > 0 on Gemma this was fused into the previous layer's tail)
    if (li == 0 || !md.gemma) {
      NormQuantArgs a{};
      a.in = e->x; a.ld_in = H; a.gamma = L.ln_in; a.eps = eps; a.q = e->q8; a.ldq = ldq; a.qs = e->qs;
      a.H = H; a.rows = M; a.mode = 0;
      KERNEL(kKNormQuant, (uint64_t)a.rows * a.H * (a.mode ? 13 : 5), eng_norm_quant(a, st));
    }
    {  // q | k | v
      EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, M, H);
      add_seg(g, L.q, e->q, qw);
      add_seg(g, L.k, e->k, kvw);
      add_seg(g, L.v, e->v, kvw);
      g.mode = kEpiStore;
      KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
    }
    {
      QkRopeArgs r{};
      r.q = e->q; r.k = e->k; r.v = e->v; r.qr = e->qr; r.kc = kc; r.vc = vc; r.qn = L.qn; r.kn = L.kn;
      r.tab = L.tab; r.pos = e->pos; r.rows = M; r.n = n; r.nh = md.n_heads; r.nkv = md.n_kv; r.hd = md.head_dim;
      r.rot = md.rot; r.Tp = e->Tp; r.eps = eps;
      AttnArgs a{};
      a.qr = e->qr; a.kc = kc; a.vc = vc; a.att = e->att; a.pos = e->pos; a.n = n; a.nh = md.n_heads;
      a.nkv = md.n_kv; a.hd = md.head_dim; a.Tp = e->Tp;
      if (e->fuse_attn && md.n_kv <= 8) {
        // q / k norm + RoPE, attention and the output quantiser in one cluster launch
        const AttnQuantArgs f{r, e->q8, (uint64_t)ldq, e->qs};
        KERNEL(kKAttention, (uint64_t)M * (qw + 3 * kvw) * 8, eng_attention_quant(a, f, B, st));
      } else {
        KERNEL(kKQkRope, (uint64_t)M * (qw + 3 * kvw) * 8, eng_qk_rope(r, st));
        KERNEL(kKAttention, 0, eng_attention(a, B, st));
        KERNEL(kKQuant, (uint64_t)M * qw * 5, eng_quant(e->att, qw, qw, e->q8, ldq, e->qs, M, st));
      }
    }
    {  // o; Qwen3 adds the residual in the epilogue
      EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, M, qw);
      add_seg(g, L.o, md.gemma ? e->o : e->x1, H);
      if (md.gemma) g.mode = kEpiStore;
      else { g.mode = kEpiResid; g.res = e->x; g.ldres = H; }
      KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
    }
    {  // [Gemma: attn_norm + residual] + ln_post + quant
      NormQuantArgs a{};
      a.eps = eps; a.q = e->q8; a.ldq = ldq; a.qs = e->qs; a.H = H; a.rows = M; a.gamma = L.ln_post;
      if (md.gemma) { a.mode = 2; a.in = e->o; a.ld_in = H; a.pre_gamma = L.attn_norm; a.res = e->x; a.x_out = e->x1; }
      else { a.mode = 0; a.in = e->x1; a.ld_in = H; }
      KERNEL(kKNormQuant, (uint64_t)a.rows * a.H * (a.mode ? 13 : 5), eng_norm_quant(a, st));
    }
    // gate, up. On the tensor cores (M >= the MMA threshold) as one plain GEMM of two segments,
    // act(gate) * up fused into the row quantiser (its 1024-thread rows hide the activation's
    // latency); on the GEMV path act(gate) * up in the GEMM epilogue, then the plain quantiser.
    if (M >= mma_min_rows()) {
      EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, M, H);
      add_seg(g, L.gate, e->g, I);
      add_seg(g, L.up, e->u, I);
      g.mode = kEpiStore;
      KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
      KERNEL(kKQuant, (uint64_t)M * I * 9, eng_quant_gated(e->g, e->u, I, I, md.act, e->q8, ldq, e->qs, M, st));
    } else {
      EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, M, H);
      add_seg(g, L.gate, e->g, I);
      add_seg(g, L.up, e->g, I);
      g.mode = kEpiGated;
      g.act = md.act;
      KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
      KERNEL(kKQuant, (uint64_t)M * I * 5, eng_quant(e->g, I, I, e->q8, ldq, e->qs, M, st));
    }
    {  // down (K blocks on Gemma); Qwen3 adds the residual into x
      EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, M, I);
      Lin dl = L.down[0];
      if (L.n_down == 2) {
        g.kb = L.down[0].k;
        dl.k = I;
      }
      if (md.gemma) {
        add_seg(g, dl, e->d, H);
        g.mode = L.n_down == 2 ? kEpiKSplit : kEpiStore;
      } else {
        add_seg(g, dl, e->x, H);
        g.mode = kEpiResid;
        g.res = e->x1;
        g.ldres = H;
      }
      if (L.n_down == 2) g.seg[0].W2 = L.down[1].W;   // the second K block's rows
      KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
    }
    if (md.gemma) {  // mlp_norm + residual, fused with the next layer's ln_in (or the final norm)
      NormQuantArgs a{};
      a.mode = 2; a.in = e->d; a.ld_in = H; a.pre_gamma = L.mlp_norm; a.res = e->x1; a.x_out = e->x;
      a.gamma = li + 1 < md.n_layers ? e->layers[li + 1].ln_in : e->final_norm;
      a.eps = eps; a.q = e->q8; a.ldq = ldq; a.qs = e->qs; a.H = H; a.rows = M;
      KERNEL(kKNormQuant, (uint64_t)a.rows * a.H * (a.mode ? 13 : 5), eng_norm_quant(a, st));
    }
  }
  {  // final norm + quant of each sequence's last row, the head, the greedy pick
    NormQuantArgs a{};
    a.mode = 0; a.in = e->x + (uint64_t)(n - 1) * H; a.ld_in = (uint64_t)n * H; a.gamma = e->final_norm;
    a.eps = eps; a.q = e->q8; a.ldq = ldq; a.qs = e->qs; a.H = H; a.rows = B;
    KERNEL(kKNormQuant, (uint64_t)a.rows * a.H * (a.mode ? 13 : 5), eng_norm_quant(a, st));
    EngGemvArgs g = gemv_args(e->q8, ldq, e->qs, B, H);
    for (const Lin& l : e->head) {
      EngSeg& s = g.seg[g.nseg++];
      s.W = l.W; s.scale = l.s; s.out = e->logits + g.ncols; s.ldo = md.vocab; s.n0 = g.ncols; s.n = l.n;
      g.ncols += l.n;
    }
    g.mode = kEpiStore;
    KERNEL(kKGemv, gemv_bytes(g), eng_gemv(g, st));
    KERNEL(kKArgmax, (uint64_t)B * md.vocab * 4, eng_argmax(e->logits, md.vocab, B, e->next, 1, st));
  }
  KERNEL(kKAdvance, 0, eng_advance(e->pos, n, B, st));
  return TC_OK;
}

// ------------------------------------------------------------------------------ the fused step
// Sets up the fused decode step (step.h): the weights re-laid out per GEMM, the per-layer table,
// the GEMM plans and the step's buffers. Leaves step_ok false (and step_why) when the model or the
// batch does not fit it; the per-kernel path then serves every step.
bool setup_step(tc_engine* e) {
  const tc_model_desc& md = e->md;
  auto no = [&](const char* why) {
    e->step_why = why;
    return false;
  };
  const char* env = getenv("TARSCUDA_STEP");
  if (env && env[0] == '0') return no("TARSCUDA_STEP=0");
  const int B = e->B, ntok = (B + 15) / 16 * 16;
  if (B > kStepMaxTok) return no("batch above 64");
  if (e->H % 128 || e->qw % 128 || e->I % 128) return no("a K dimension is not a multiple of 128");
  if (md.head_dim != 64 && md.head_dim != 128 && md.head_dim != 256) return no("head dim");
  // the attention prologue gives each of 16 half-warps one row: G query heads, the K and the V row
  if (md.n_heads % md.n_kv || md.n_heads / md.n_kv > 14 || md.rot > md.head_dim || md.rot % 2) return no("heads");
  if (md.n_head_blocks < 1 || md.n_head_blocks > kStepSegs) return no("head blocks");
  const int G = md.n_heads / md.n_kv;
  int nsm0 = 0, dev0 = 0;
  cudaGetDevice(&dev0);
  cudaDeviceGetAttribute(&nsm0, cudaDevAttrMultiProcessorCount, dev0);
  // concurrent attention units per CTA: enough groups for every (sequence, kv head) in one pass
  int agroups = 1;
  while (agroups < 4 && B * md.n_kv > nsm0 * agroups && step_attn_tile(md.head_dim, G, agroups * 2) >= 16)
    agroups *= 2;
  const int tile = step_attn_tile(md.head_dim, G, agroups);
  if (tile < 16) return no("attention tile");
  if (5 * e->H * 4 > step_region_bytes() || md.rot % 4) return no("row staging");
  int dev = 0, coop = 0, nsm = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (!coop || nsm < 1) return no("no cooperative launch");
  if (step_occupancy(&per_sm) != cudaSuccess || per_sm < 1) return no("occupancy");
  const int grid = nsm;
  uint64_t part_bytes = 0;
  // plan every GEMM; its weights are re-laid out as [tile][slice] blocks (step.h) below
  struct Pending { StepGemm* g; std::vector<Lin> segs; const Lin* second; int K; };
  std::vector<Pending> todo;
  auto gemm = [&](StepGemm& g, const std::vector<Lin>& segs, const Lin* second, int K, bool fused) {
    g = StepGemm{};
    g.nseg = (int)segs.size();
    int tiles = 0, cols = 0;
    for (int s = 0; s < g.nseg; ++s) {
      const Lin& l = segs[s];
      if (l.k != (second ? segs[0].k : K)) return false;
      g.tile0[s] = tiles;
      g.col0[s] = cols;
      g.scale[s] = l.s;
      tiles += (l.n + 127) / 128;
      cols += l.n;
    }
    g.tile0[g.nseg] = tiles;
    g.col0[g.nseg] = cols;
    g.nslices = K / 128;
    g.kb = second ? segs[0].k / 128 : g.nslices;
    if (second && (segs[0].k % 128 || second->k != K - segs[0].k)) return false;
    if (!step_plan_gemm(g, ntok, grid, fused)) return false;
    if (!fused) part_bytes = std::max(part_bytes, (uint64_t)g.ksplit * B * cols * 4);
    todo.push_back(Pending{&g, segs, second, K});
    return true;
  };
  e->slayers.assign(md.n_layers, StepLayer{});
  for (int li = 0; li < md.n_layers; ++li) {
    const Layer& L = e->layers[li];
    StepLayer& S = e->slayers[li];
    if (L.n_down > 2) return no("down in more than two K blocks");
    if (!gemm(S.qkv, {L.q, L.k, L.v}, nullptr, e->H, false)) return no("q|k|v plan");
    if (!gemm(S.o, {L.o}, nullptr, e->qw, false)) return no("o plan");
    if (!gemm(S.gu, {L.gate, L.up}, nullptr, e->H, false)) return no("gate|up plan");
    if (!gemm(S.down, {L.down[0]}, L.n_down == 2 ? &L.down[1] : nullptr, e->I, false)) return no("down plan");
    S.ln_in = L.ln_in; S.ln_post = L.ln_post; S.attn_norm = L.attn_norm; S.mlp_norm = L.mlp_norm;
    S.qn = L.qn; S.kn = L.kn; S.tab = L.tab;
    S.kc = e->kc + (uint64_t)li * e->B * e->Tp * e->kvw;
    S.vc = e->vc + (uint64_t)li * e->B * e->Tp * e->kvw;
  }
  StepArgs& a = e->sa;
  if (!gemm(a.head, e->head, nullptr, e->H, true)) return no("head plan");
  uint64_t wt_bytes = 0;
  for (const Pending& p : todo) wt_bytes += (uint64_t)p.g->tile0[p.g->nseg] * p.g->nslices * kStepSliceBytes;
  cudaError_t c = cudaMalloc((void**)&e->wt, wt_bytes);
  uint64_t off = 0;
  for (const Pending& p : todo) {
    if (c != cudaSuccess) break;
    StepGemm& g = *p.g;
    g.wt = e->wt + off;
    for (int s = 0; s < g.nseg && c == cudaSuccess; ++s) {
      const Lin& l = p.segs[s];
      uint8_t* out = e->wt + off + (uint64_t)g.tile0[s] * g.nslices * kStepSliceBytes;
      c = step_retile(l.W, p.second ? p.second->W : nullptr, l.n, p.K, p.second ? l.k : p.K, out, e->st);
    }
    off += (uint64_t)g.tile0[g.nseg] * g.nslices * kStepSliceBytes;
  }
  const int ldq = std::max(std::max(e->H, e->I), e->qw);
  const size_t q8t_bytes = (size_t)(ldq / 128) * ntok * 128;
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->d_layers, e->slayers.size() * sizeof(StepLayer));
  if (c == cudaSuccess)
    c = cudaMemcpy(e->d_layers, e->slayers.data(), e->slayers.size() * sizeof(StepLayer), cudaMemcpyHostToDevice);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->q8t, q8t_bytes);
  if (c == cudaSuccess) c = cudaMemsetAsync(e->q8t, 0, q8t_bytes, e->st);   // the padding rows stay zero
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->qs2, (size_t)B * 4);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->part, std::max<uint64_t>(part_bytes, 16));
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->satt, (size_t)B * e->qw * 4);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->samax, (size_t)B * md.n_kv * 4);
  // gated MLP units of 512 columns (the last one of a row may be shorter)
  const int gchunks = std::max(1, (e->I + 511) / 512);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->sgv, (size_t)B * e->I * 4);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->sgmax, (size_t)B * gchunks * 4);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->ssync, (size_t)(1 + 2 * B) * 4);
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->sdiag, 4 * sizeof(int));
  if (c == cudaSuccess) c = cudaMemsetAsync(e->sdiag, 0, 4 * sizeof(int), e->st);
  e->ntrace = 1024 + (9 * md.n_layers + 8) * grid;
  if (c == cudaSuccess) c = cudaMalloc((void**)&e->strace, (size_t)e->ntrace * 8);
  if (c == cudaSuccess) c = cudaStreamSynchronize(e->st);
  if (c != cudaSuccess) return no("allocation or weight layout");
  a.layers = e->d_layers;
  a.L = md.n_layers; a.B = B; a.ntok = ntok; a.H = e->H; a.I = e->I; a.nh = md.n_heads; a.nkv = md.n_kv;
  a.hd = md.head_dim; a.rot = md.rot; a.Tp = e->Tp; a.vocab = md.vocab; a.gemma = md.gemma; a.act = md.act;
  a.ldq = ldq; a.tile = tile; a.agroups = agroups; a.gchunks = gchunks;
  a.gv = e->sgv; a.gmax = e->sgmax;
  a.eps = md.eps; a.embed_scale = md.embed_scale;
  a.E = e->E; a.pos = e->pos; a.final_norm = e->final_norm;
  a.x = e->x; a.x1 = e->x1; a.q8t = e->q8t; a.qsa = e->qs; a.qsb = e->qs2;
  a.part = e->part; a.att = e->satt; a.amax = e->samax; a.logits = e->logits; a.sync = e->ssync;
  a.diag = e->sdiag;
  a.err = wait_error_flag();
  if (!a.err) return no("error word");
  e->grid = grid;
  return true;
}

// One fused decode step (tokens already on the device at tok), then the greedy pick and the
// positions' advance.
int step_fused(tc_engine* e, const int* tok, bool trace) {
  StepArgs a = e->sa;
  a.tok = tok;
  // time limits: the poll limit's scale (2^22 polls: about 0.2 s; 0: give up at once)
  a.wait_ns = (uint64_t)spin_limit() * 50;
  a.drain_ns = 20000000ull;
  static const int lead = [] {                         // a tuning knob: how early weights stream
    const char* v = getenv("TARSCUDA_STEP_LEAD");
    return v ? atoi(v) : 1 << 20;
  }();
  a.lead = lead;
  a.trace = trace ? e->strace : nullptr;
  TRY(cudaMemsetAsync(e->ssync, 0, (size_t)(1 + 2 * e->B) * 4, e->st));
  if (trace) TRY(cudaMemsetAsync(e->strace, 0, (size_t)e->ntrace * 8, e->st));
  TRY(step_launch(a, e->grid, e->st));
  TRY(eng_argmax(e->logits, e->md.vocab, e->B, e->next, 1, e->st));
  TRY(eng_advance(e->pos, 1, e->B, e->st));
  return TC_OK;
}
}  // namespace

extern "C" {

int tc_engine_create(tc_machine* image, const tc_model_desc* md, const tc_layer_desc* layers, const float* embed_host,
                     int32_t batch, tc_engine** out) {
  if (!out) return TC_ERR_ARG;
  *out = nullptr;
  if (!image || !md || !layers || !embed_host || md->n_layers < 1 || md->vocab < 1) return TC_ERR_ARG;
  tc_engine* e = new tc_engine();
  {
    const char* fa = getenv("TARSCUDA_FUSE_ATTN");
    e->fuse_attn = !(fa && fa[0] == '0');
  }
  e->md = *md;
  const uint8_t* base = (const uint8_t*)(uintptr_t)tc_device_ptr(image);
  e->B = batch;
  e->T = md->max_tokens;
  e->Tp = (md->max_tokens + 15) / 16 * 16;
  e->H = md->hidden;
  e->I = md->inter;
  e->qw = md->n_heads * md->head_dim;
  e->kvw = md->n_kv * md->head_dim;
  if (md->n_head_blocks > kMaxSegs || md->head_dim > 256 || md->max_tokens > 256 || batch < 1) {
    delete e;
    return TC_ERR_ARG;
  }
  for (int i = 0; i < md->n_layers; ++i) {
    const tc_layer_desc& ld = layers[i];
    Layer L{};
    L.ln_in = vec_of(base, ld.ln_in); L.ln_post = vec_of(base, ld.ln_post);
    L.attn_norm = vec_of(base, ld.attn_norm); L.mlp_norm = vec_of(base, ld.mlp_norm);
    L.qn = vec_of(base, ld.qn); L.kn = vec_of(base, ld.kn); L.tab = vec_of(base, ld.rope_tab);
    L.q = lin_of(base, ld.q); L.k = lin_of(base, ld.k); L.v = lin_of(base, ld.v); L.o = lin_of(base, ld.o);
    L.gate = lin_of(base, ld.gate); L.up = lin_of(base, ld.up);
    L.n_down = ld.n_down;
    for (int j = 0; j < ld.n_down; ++j) L.down[j] = lin_of(base, ld.down[j]);
    e->layers.push_back(L);
  }
  for (int j = 0; j < md->n_head_blocks; ++j) e->head.push_back(lin_of(base, md->head[j]));
  e->final_norm = vec_of(base, md->final_norm);
  cudaGetDevice(&e->device);
  const int M = e->B * e->nmax, ldq = std::max(std::max(e->H, e->I), e->qw);
  auto alloc = [&](void** p, size_t n) { return cudaMalloc(p, std::max<size_t>(n, 16)); };
  cudaError_t c = cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking);
  if (c == cudaSuccess) c = alloc((void**)&e->E, (size_t)md->vocab * e->H * 4);
  if (c == cudaSuccess) c = cudaMemcpy(e->E, embed_host, (size_t)md->vocab * e->H * 4, cudaMemcpyHostToDevice);
  if (c == cudaSuccess) c = alloc((void**)&e->tok, (size_t)M * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->next, (size_t)e->B * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->pos, (size_t)e->B * 4);
  float** fbufs[] = {&e->x, &e->x1, &e->o, &e->d};
  for (auto p : fbufs) if (c == cudaSuccess) c = alloc((void**)p, (size_t)M * e->H * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->q, (size_t)M * e->qw * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->qr, (size_t)M * e->qw * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->att, (size_t)M * e->qw * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->k, (size_t)M * e->kvw * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->v, (size_t)M * e->kvw * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->g, (size_t)M * e->I * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->u, (size_t)M * e->I * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->logits, (size_t)e->B * md->vocab * 4);
  if (c == cudaSuccess) c = alloc((void**)&e->q8, (size_t)M * ldq);
  if (c == cudaSuccess) c = alloc((void**)&e->qs, (size_t)M * 4);
  const size_t cache = (size_t)md->n_layers * e->B * e->Tp * e->kvw * 4;
  if (c == cudaSuccess) c = alloc((void**)&e->kc, cache);
  if (c == cudaSuccess) c = alloc((void**)&e->vc, cache);
  if (c != cudaSuccess) {
    tc_engine_destroy(e);
    return TC_ERR_CUDA;
  }
  // set up where the model fits; on by default only once validated (tc_engine_fused switches it)
  e->step_ok = setup_step(e) && kFusedDefault;
  cudaGetLastError();                        // a refused setup leaves no error state behind
  *out = e;
  return tc_engine_reset(e);
}

int tc_engine_destroy(tc_engine* e) {
  if (!e) return TC_OK;
  if (e->st) cudaStreamSynchronize(e->st);
  for (auto& gx : e->graph) if (gx) cudaGraphExecDestroy(gx);
  void* bufs[] = {e->E, e->tok, e->next, e->pos, e->x, e->x1, e->q, e->k, e->v, e->qr, e->att, e->o, e->g, e->u, e->d,
                  e->logits, e->q8, e->qs, e->kc, e->vc, e->d_layers, e->wt, e->q8t, e->sdiag, e->qs2, e->part,
                  e->satt, e->samax, e->sgv, e->sgmax, e->ssync, e->strace};
  for (void* p : bufs) if (p) cudaFree(p);
  if (e->st) cudaStreamDestroy(e->st);
  delete e;
  return TC_OK;
}

const char* tc_engine_error(tc_engine* e) { return e ? e->err.c_str() : ""; }
void* tc_engine_stream(tc_engine* e) { return (void*)e->st; }

int tc_engine_reset(tc_engine* e) {
  const size_t cache = (size_t)e->md.n_layers * e->B * e->Tp * e->kvw * 4;
  TRY(cudaMemsetAsync(e->kc, 0, cache, e->st));
  TRY(cudaMemsetAsync(e->vc, 0, cache, e->st));
  TRY(cudaMemsetAsync(e->pos, 0, (size_t)e->B * 4, e->st));
  TRY(cudaStreamSynchronize(e->st));
  e->hpos.assign(e->B, 0);
  return TC_OK;
}

int tc_engine_reset_seq(tc_engine* e, int32_t b) {
  if (!e || b < 0 || b >= e->B) return TC_ERR_ARG;
  const size_t rows = (size_t)e->Tp * e->kvw * 4;
  for (int li = 0; li < e->md.n_layers; ++li) {
    const uint64_t off = ((uint64_t)li * e->B + b) * e->Tp * e->kvw;
    TRY(cudaMemsetAsync(e->kc + off, 0, rows, e->st));
    TRY(cudaMemsetAsync(e->vc + off, 0, rows, e->st));
  }
  TRY(cudaMemsetAsync(e->pos + b, 0, 4, e->st));
  e->hpos[b] = 0;
  return TC_OK;
}

int tc_engine_positions(tc_engine* e, int32_t* pos_host) {
  TRY(cudaMemcpyAsync(pos_host, e->pos, (size_t)e->B * 4, cudaMemcpyDeviceToHost, e->st));
  TRY(cudaStreamSynchronize(e->st));
  return TC_OK;
}

int tc_engine_fused(tc_engine* e, int32_t enable) {
  if (!e) return TC_ERR_ARG;
  const bool was = e->step_ok;
  if (enable >= 0) {
    if (enable && !e->d_layers) return TC_ERR_ARG;       // never set up for this model / batch
    e->step_ok = enable != 0;
  }
  return was ? 1 : 0;
}

const char* tc_engine_fused_why(tc_engine* e) { return e ? e->step_why.c_str() : ""; }

int tc_engine_fused_diag(tc_engine* e, int32_t* out4) {
  if (!e || !e->sdiag || !out4) return TC_ERR_ARG;
  TRY(cudaStreamSynchronize(e->st));
  TRY(cudaMemcpy(out4, e->sdiag, 4 * sizeof(int), cudaMemcpyDeviceToHost));
  return TC_OK;
}

int tc_engine_phase_times(tc_engine* e, uint64_t* stamps, uint32_t cap) {
  if (!e || !e->step_ok) return TC_ERR_ARG;
  if (!take_positions(e, 1)) return TC_ERR_ARG;
  const int rc = step_fused(e, e->next, true);
  if (rc != TC_OK) return rc;
  TRY(cudaStreamSynchronize(e->st));
  const uint32_t n = std::min<uint32_t>(cap, (uint32_t)e->ntrace);
  if (stamps && n) TRY(cudaMemcpy(stamps, e->strace, (size_t)n * 8, cudaMemcpyDeviceToHost));
  return (int)n;
}

// Runs one chunk of n tokens per sequence (tokens_host: [B][n] ids, or NULL to feed each
// sequence's greedy pick of the previous step, n = 1). The step is captured as a CUDA graph on
// first use for that n and replayed afterwards; the position advances on the device.
int tc_engine_step(tc_engine* e, const int32_t* tokens_host, int32_t n) {
  if (n < 1 || n > e->nmax || (!tokens_host && n != 1)) { e->err = "bad chunk"; return TC_ERR_ARG; }
  if (tokens_host)
    for (int i = 0; i < e->B * n; ++i)
      if (tokens_host[i] < 0 || tokens_host[i] >= e->md.vocab) {
        e->err = "token id outside the vocabulary";
        return TC_ERR_ARG;
      }
  if (!take_positions(e, n)) return TC_ERR_ARG;
  const int* src = e->next;
  if (tokens_host) {
    TRY(cudaMemcpyAsync(e->tok, tokens_host, (size_t)e->B * n * 4, cudaMemcpyHostToDevice, e->st));
    src = e->tok;
  }
  if (n == 1 && e->step_ok) return step_fused(e, src, false);
  const int slot = tokens_host ? n : 0;
  if (!e->graph[slot]) {
    cudaGraph_t graph;
    TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeRelaxed));
    // programmatic dependent launch between the step's kernels when its GEMMs run on the tensor
    // cores (measured: neutral to slightly faster there, slower for the GEMV path at batch 1);
    // TARSCUDA_PDL=0 turns it off
    const char* pdl = getenv("TARSCUDA_PDL");
    pdl_launches() = !(pdl && pdl[0] == '0') && e->B * n >= mma_min_rows();
    const int rc = enqueue_step(e, n, src);
    pdl_launches() = false;
    cudaError_t c = cudaStreamEndCapture(e->st, &graph);
    if (rc != TC_OK) return rc;
    if (c != cudaSuccess) return fail(e, "end capture", c);
    c = cudaGraphInstantiate(&e->graph[slot], graph, 0);
    cudaGraphDestroy(graph);
    if (c != cudaSuccess) return fail(e, "instantiate", c);
  }
  TRY(cudaGraphLaunch(e->graph[slot], e->st));
  return TC_OK;
}

int tc_engine_profile(tc_engine* e, float* ms, int32_t* kind, uint64_t* bytes, uint32_t cap) {
  // The step is captured with an event node on each side of every kernel and launched once, so
  // the times are the kernels' own (no host work between the events, as in the timed graphs).
  if (!take_positions(e, 1)) return TC_ERR_ARG;
  e->prof = true;
  e->pev.clear(); e->pkind.clear(); e->pbytes.clear();
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaError_t c = cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal);
  int rc = c == cudaSuccess ? enqueue_step(e, 1, e->next) : TC_OK;
  if (c == cudaSuccess) {
    const cudaError_t c2 = cudaStreamEndCapture(e->st, &graph);
    if (rc == TC_OK && c2 != cudaSuccess) c = c2;
  }
  e->prof = false;
  if (c == cudaSuccess && rc == TC_OK) c = cudaGraphInstantiate(&exec, graph, 0);
  if (c == cudaSuccess && rc == TC_OK) c = cudaGraphLaunch(exec, e->st);
  if (c == cudaSuccess && rc == TC_OK) c = cudaStreamSynchronize(e->st);
  const int n = (int)e->pkind.size();
  for (int i = 0; i < n && i < (int)cap && c == cudaSuccess && rc == TC_OK; ++i) {
    cudaEventElapsedTime(&ms[i], e->pev[2 * i], e->pev[2 * i + 1]);
    kind[i] = e->pkind[i];
    bytes[i] = e->pbytes[i];
  }
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  for (auto ev : e->pev) cudaEventDestroy(ev);
  e->pev.clear();
  if (rc != TC_OK) return rc;
  if (c != cudaSuccess) return fail(e, "profile", c);
  return n;
}

int tc_engine_set_tokens(tc_engine* e, const int32_t* tokens_host) {
  TRY(cudaMemcpyAsync(e->next, tokens_host, (size_t)e->B * 4, cudaMemcpyHostToDevice, e->st));
  return TC_OK;
}
int tc_engine_tokens(tc_engine* e, int32_t* tokens_host) {
  TRY(cudaMemcpyAsync(tokens_host, e->next, (size_t)e->B * 4, cudaMemcpyDeviceToHost, e->st));
  TRY(cudaStreamSynchronize(e->st));
  return TC_OK;
}
int tc_engine_logits(tc_engine* e, float* logits_host) {
  TRY(cudaMemcpyAsync(logits_host, e->logits, (size_t)e->B * e->md.vocab * 4, cudaMemcpyDeviceToHost, e->st));
  TRY(cudaStreamSynchronize(e->st));
  return TC_OK;
}
int tc_engine_sync(tc_engine* e) {
  TRY(cudaStreamSynchronize(e->st));
  return TC_OK;
}

int tc_argmax(const float* logits, int32_t vocab, int32_t rows, int32_t* tok_out, void* stream) {
  if (!logits || !tok_out || vocab <= 0 || rows <= 0 || rows > (1 << 24)) return TC_ERR_ARG;
  return tc::eng_argmax(logits, vocab, rows, tok_out, 1, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? TC_OK
             : TC_ERR_CUDA;
}

}  // extern "C"
