// libtarscuda: the DDR image in HBM and the in-order descriptor queue executor (C-ABI).
//
// Replaces the execution half of the reference's golden Machine (tars_mini/golden.py:450-492):
// descriptors run strictly in queue order; every check of a descriptor (decode, CRC, field,
// alignment, range; overlap refusal) happens on the host before anything of it is launched; a
// failing descriptor stops the queue with its error code and keeps the earlier descriptors'
// writes. The arithmetic runs as sm_100a kernels on one CUDA stream, so descriptor i+1 sees
// every write of descriptor i (RAW/WAR/WAW in queue order).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tarscuda.h"
#include "desc.h"
#include "ops.h"

using namespace tc;

struct tc_machine {
  int device = 0;
  uint8_t* dev = nullptr;
  uint64_t size = 0;
  cudaStream_t stream = nullptr;
  std::vector<tc_opstat> stats;
  std::vector<std::pair<uint64_t, uint64_t>> written;  // [lo, hi) of the last run's outputs
  uint8_t* scratch = nullptr;
  uint64_t scratch_size = 0;
  uint8_t* w4s = nullptr;                              // the W4A16 GEMV's aligned activation rows
  uint64_t w4s_size = 0;
  uint64_t w4s_slice = 0;                              // bytes per W4 GEMV of one capture level
  std::string err;
  std::vector<cudaStream_t> lanes;                     // extra capture streams (one level's launches)
};

// A validated queue captured as one CUDA graph (tc_queue_capture).
struct tc_graph {
  tc_machine* m = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<cudaEvent_t> events;                     // before each descriptor, and one after the last
  std::vector<tc_opstat> stats;
  std::vector<std::pair<uint64_t, uint64_t>> written;
  tc_status status{};
  int kernels = 0;                                     // kernel nodes of the graph
};

namespace {

int fail(tc_machine* m, const char* what, cudaError_t e) {
  if (m) m->err = std::string(what) + ": " + cudaGetErrorString(e);
  return TC_ERR_CUDA;
}

float f32(uint64_t bits) {
  uint32_t b = (uint32_t)bits;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// Grows a device buffer of the machine (after the machine's stream drained: queued work may still
// use the old one).
cudaError_t grow(tc_machine* m, uint8_t*& buf, uint64_t& size, uint64_t n) {
  if (n <= size) return cudaSuccess;
  if (buf) {
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return e;
    cudaFree(buf);
    buf = nullptr;
    size = 0;
  }
  cudaError_t e = cudaMalloc(&buf, n);
  if (e == cudaSuccess) size = n;
  return e;
}
cudaError_t ensure_scratch(tc_machine* m, uint64_t n) { return grow(m, m->scratch, m->scratch_size, n); }
cudaError_t ensure_w4s(tc_machine* m, uint64_t n) { return grow(m, m->w4s, m->w4s_size, n); }

// The kernel arguments of a W8A8 GEMM descriptor (A as the descriptor names it; a conv's gather
// buffer replaces it at launch) and of a row-op descriptor.
void gemm_args(tc_machine* mc, const Desc& d, GemmArgs* g) {
  uint8_t* B = mc->dev + d[F_BASE_ADDR];
  const Strides s = strides(d);
  g->A = B + d[F_A_OFF]; g->lda = s.lda;
  g->W = B + d[F_W_OFF]; g->scale = B + d[F_SCALE_OFF];
  g->per_channel = d.qmode() != QM_TENSOR;
  g->srow = (d.qmode() == QM_ROWCOL) ? mc->dev + d[F_BASE_ADDR] + 16 * d[F_HDR_RSV] : nullptr;
  g->bias = d.bias() ? B + d[F_BIAS_OFF] : nullptr;
  g->Y = B + d[F_Y_OFF]; g->ldy = s.ldy;
  g->M = (int)d[F_M]; g->N = (int)d[F_N]; g->K = (int)d[F_K];
  g->act = d.act(); g->out = d.out(); g->out_scale = f32(d[F_OUT_SCALE]);
}
// The kernel arguments of a W4A16 GEMV descriptor; its aligned rows go to the W4 scratch at
// `w4_off` (nullptr scratch when it cannot be had: the kernels then align in every block).
W4Args w4_args(tc_machine* mc, const Desc& d, uint64_t w4_off) {
  uint8_t* B = mc->dev + d[F_BASE_ADDR];
  const Strides s = strides(d);
  W4Args g{};
  g.A = B + d[F_A_OFF]; g.lda = s.lda;
  g.a_bf16 = ((d[F_CTRL] >> 4) & 15) == DT_BF16;
  g.W = B + d[F_W_OFF]; g.scale = B + d[F_SCALE_OFF];
  g.bias = d.bias() ? B + d[F_BIAS_OFF] : nullptr;
  g.Y = B + d[F_Y_OFF]; g.ldy = s.ldy;
  g.M = (int)d[F_M]; g.N = (int)d[F_N]; g.K = (int)d[F_K];
  g.act = d.act(); g.out = d.out(); g.out_scale = f32(d[F_OUT_SCALE]);
  if (g.M <= 4 && ensure_w4s(mc, w4_off + w4_scratch_bytes(g.M, g.K)) == cudaSuccess) g.scratch = mc->w4s + w4_off;
  return g;
}
void row_args(tc_machine* mc, const Desc& d, RowArgs* a) {
  uint8_t* B = mc->dev + d[F_BASE_ADDR];
  const Strides s = strides(d);
  a->X = B + d[F_A_OFF]; a->lda = s.lda; a->Y = B + d[F_Y_OFF]; a->ldy = s.ldy;
  a->fn = (int)(d[F_CTRL] & 7);
  a->M = (int)d[F_M]; a->N = (int)d[F_N]; a->K = (int)d[F_K]; a->out = d.out(); a->out_scale = f32(d[F_OUT_SCALE]);
  if (a->fn == ROW_QUANT) a->scale_out = B + d[F_SCALE_OFF];
  if (a->fn == ROW_LAYERNORM || a->fn == ROW_RMSNORM || a->fn == ROW_L2NORM) {
    a->gamma = B + d[F_SCALE_OFF];
    a->beta = d.bias() ? B + d[F_BIAS_OFF] : nullptr;
    a->eps = f32(d[F_W_OFF]);
  }
}

// Enqueues the kernels of one validated, in-range descriptor.
// `w4_off`: where in the W4 row scratch a W4A16 GEMV keeps its aligned activation rows (W4 GEMVs
// that may run at the same time use different slices).
cudaError_t launch_on(tc_machine* mc, const Desc& d, cudaStream_t stream, uint64_t w4_off = 0);
cudaError_t launch(tc_machine* mc, const Desc& d) { return launch_on(mc, d, mc->stream); }

cudaError_t launch_on(tc_machine* mc, const Desc& d, cudaStream_t stream, uint64_t w4_off) {
  uint8_t* B = mc->dev + d[F_BASE_ADDR];
  const Strides s = strides(d);
  const int op = d.op();
  const float osc = f32(d[F_OUT_SCALE]);
  if (op == OP_GEMM || d.conv()) {
    if (d.w4()) return launch_gemm_w4a16(w4_args(mc, d, w4_off), stream);
    GemmArgs g{};
    gemm_args(mc, d, &g);
    if (d.conv()) {
      const ConvGeom cg = conv_geom(d);
      const uint64_t need = d[F_M] * d[F_K];
      cudaError_t e = ensure_scratch(mc, need);
      if (e != cudaSuccess) return e;
      Im2colArgs ia{};
      ia.img = B + d[F_A_OFF]; ia.ld = s.lda; ia.out = mc->scratch;
      ia.H = cg.H; ia.W = cg.W; ia.KH = cg.KH; ia.KW = cg.KW; ia.S = cg.S; ia.P = cg.P;
      ia.Cin = cg.Cin; ia.OH = cg.OH; ia.OW = cg.OW;
      e = launch_im2col(ia, stream);
      if (e != cudaSuccess) return e;
      g.A = mc->scratch; g.lda = d[F_K];
    }
    return launch_gemm_w8a8(g, stream);
  }
  if (op == OP_RELU) {
    ActArgs a{};
    a.X = B + d[F_A_OFF]; a.lda = s.lda; a.Y = B + d[F_Y_OFF]; a.ldy = s.ldy;
    a.M = (int)d[F_M]; a.N = (int)d[F_N]; a.act = d.act(); a.out = d.out(); a.out_scale = osc;
    return launch_act(a, stream);
  }
  if (op == OP_ROW) {
    RowArgs a{};
    row_args(mc, d, &a);
    return launch_rowop(a, stream);
  }
  if (op == OP_ELT) {
    EltArgs a{};
    const uint64_t hdr = d[F_HDR_RSV];
    a.A = B + d[F_A_OFF]; a.lda = (hdr >> 2 & 1) ? 0 : s.lda; a.a_fp16 = (hdr & STATE_FP16) != 0;
    uint64_t ldb, brow;
    bstride(d, &ldb, &brow);
    a.B = B + d[F_W_OFF]; a.ldb = ldb; a.bmode = (int)(hdr & 3);
    a.op = (int)(d[F_CTRL] & 3);
    a.C = a.op == ELT_MULADD ? B + d[F_BIAS_OFF] : nullptr;
    a.Y = B + d[F_Y_OFF]; a.ldy = s.ldy;
    a.M = (int)d[F_M]; a.N = (int)d[F_N]; a.act = d.act(); a.out = d.out(); a.out_scale = osc;
    return launch_elt(a, stream);
  }
  if (op == OP_ROPE) {
    RopeArgs a{};
    a.X = B + d[F_A_OFF]; a.lda = s.lda; a.tab = B + d[F_W_OFF]; a.Y = B + d[F_Y_OFF]; a.ldy = s.ldy;
    a.M = (int)d[F_M]; a.N = (int)d[F_N]; a.R = (int)d[F_K]; a.G = (int)d[F_GROUP_SIZE];
    a.out = d.out(); a.out_scale = osc;
    return launch_rope(a, stream);
  }
  // FDOT
  FdotArgs a{};
  uint64_t ldb, brow;
  bstride(d, &ldb, &brow);
  a.A = B + d[F_A_OFF]; a.lda = s.lda; a.B = B + d[F_W_OFF]; a.ldb = ldb;
  a.nn = (int)(d[F_CTRL] & 1); a.b_fp16 = (d[F_HDR_RSV] & STATE_FP16) != 0;
  a.Y = B + d[F_Y_OFF]; a.ldy = s.ldy;
  a.M = (int)d[F_M]; a.N = (int)d[F_N]; a.K = (int)d[F_K]; a.out = d.out(); a.out_scale = osc;
  return launch_fdot(a, stream);
}

bool in_range(const Footprint& fp, u128 size) {
  for (const auto& t : fp.reads)
    for (const auto& sg : t)
      if (seg_end(sg) > size) return false;
  if (seg_end(fp.y) > size) return false;
  if (fp.has_extra && seg_end(fp.extra) > size) return false;
  return true;
}

// golden.py:473-479: an output over an input (except the in-place ELT reads) or over the other output
const char* illegal(const Desc& d, const Footprint& fp) {
  for (size_t j = 0; j < fp.reads.size(); ++j)
    for (const auto& sg : fp.reads[j]) {
      if (overlaps(sg, fp.y) && !in_place(d, (int)j)) return "output overlaps an input";
      if (fp.has_extra && overlaps(sg, fp.extra)) return "output overlaps an input";
    }
  if (fp.has_extra && overlaps(fp.extra, fp.y)) return "the two outputs overlap";
  return nullptr;
}

uint64_t read_bytes(const Footprint& fp) {
  u128 s = 0;
  for (const auto& t : fp.reads)
    for (const auto& sg : t) s += seg_bytes(sg);
  return (uint64_t)s;
}

// The in-order loop shared by tc_run_queue and tc_queue_capture. `before(i)` runs before
// `run(d)` enqueues (or records) the kernels of descriptor i; `capturing` forbids host
// synchronisation (a queue that rewrites its own later descriptors cannot be captured).
template <class Before, class After, class Run>
int execute(tc_machine* m, uint64_t qaddr, uint32_t qlen, int32_t core_id, int32_t gemv_only, tc_status* st,
            int32_t* contract_op, const std::vector<uint8_t>& q0, bool capturing, Before before, After after,
            Run run) {
  std::vector<uint8_t> q = q0;
  const u128 size = m->size;
  auto fetch = [&](uint32_t from) -> cudaError_t {
    uint64_t n_ok = 0;
    if ((u128)qaddr + 64 * (u128)from < size) n_ok = (uint64_t)((size - qaddr) / 64);
    n_ok = std::min<uint64_t>(n_ok, qlen);
    if (n_ok <= from) return cudaSuccess;
    cudaError_t e = cudaMemcpyAsync(q.data() + 64 * (size_t)from, m->dev + qaddr + 64 * (uint64_t)from,
                                    64 * (n_ok - from), cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    return e;
  };
  const u128 qend = (u128)qaddr + 64 * (u128)qlen;
  int rc = TC_OK;
  uint32_t i = 0;
  for (; i < qlen; ++i) {
    const u128 qa = (u128)qaddr + 64 * (u128)i;
    if (qa + 64 > size) { st->err_code = E_RANGE; st->op_idx = (int32_t)i; break; }
    const uint8_t* raw = q.data() + 64 * (size_t)i;
    Desc d;
    decode(raw, &d);
    int err = validate(raw, d, core_id, gemv_only);
    Footprint fp;
    if (err == E_OK) {
      fp = footprint(d);
      if (!in_range(fp, size)) err = E_RANGE;
    }
    if (err != E_OK) { st->err_code = err; st->op_idx = (int32_t)i; break; }
    if (const char* why = illegal(d, fp)) {
      *contract_op = (int32_t)i;
      m->err = std::string("descriptor ") + std::to_string(i) + ": " + why;
      rc = TC_CONTRACT;
      break;
    }
    before(i, d, fp);
    cudaError_t e = run(d);
    if (e != cudaSuccess) { rc = fail(m, "launch", e); break; }
    after(i);
    const int op = d.op();
    const uint64_t macs = (op == OP_GEMM || op == OP_FDOT || d.conv()) ? d[F_M] * d[F_N] * d[F_K] : 0;
    const Strides s = strides(d);
    m->stats.push_back(tc_opstat{(uint64_t)op, macs, read_bytes(fp), d[F_M] * s.yrow});
    const u128 ylo = fp.y.base, yhi = seg_end(fp.y);
    m->written.push_back({(uint64_t)ylo, (uint64_t)yhi});
    u128 xlo = 0, xhi = 0;
    if (fp.has_extra) {
      xlo = fp.extra.base; xhi = seg_end(fp.extra);
      m->written.push_back({(uint64_t)xlo, (uint64_t)xhi});
    }
    // a descriptor that rewrites later descriptors of this queue: read them again
    const u128 rest = qa + 64;
    if (i + 1 < qlen && ((ylo < qend && yhi > rest) || (fp.has_extra && xlo < qend && xhi > rest))) {
      if (capturing) { m->err = "the queue rewrites its own descriptors: not capturable"; rc = TC_ERR_ARG; break; }
      e = fetch(i + 1);
      if (e != cudaSuccess) { rc = fail(m, "queue refetch", e); break; }
    }
  }
  if (rc == TC_OK && i == qlen) { st->done = 1; st->err_code = E_OK; st->op_idx = (int32_t)qlen; }
  return rc;
}

cudaError_t fetch_queue(tc_machine* m, uint64_t qaddr, uint32_t qlen, std::vector<uint8_t>& q) {
  q.assign((size_t)qlen * 64, 0);
  uint64_t n_ok = 0;
  if ((u128)qaddr < (u128)m->size) n_ok = std::min<uint64_t>((m->size - qaddr) / 64, qlen);
  if (!n_ok) return cudaSuccess;
  cudaError_t e = cudaMemcpyAsync(q.data(), m->dev + qaddr, 64 * n_ok, cudaMemcpyDeviceToHost, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  return e;
}

// At most this many W4A16 GEMVs share a capture level (each with its own scratch slice, and one
// grouped launch for those of one class); more move to later levels.
constexpr int kW4Slices = kW4GroupMax;

// The conv gather scratch, and the W4A16 row scratch a queue needs as (slice bytes, slices), so
// that capture never allocates.
struct ScratchNeed { uint64_t conv, w4_slice; int w4_slices; };
ScratchNeed scratch_need(const std::vector<uint8_t>& q, uint32_t qlen, int core_id, int gemv_only) {
  uint64_t conv = 0, w4 = 0;
  int nw4 = 0;
  for (uint32_t i = 0; i < qlen; ++i) {
    const uint8_t* raw = q.data() + 64 * (size_t)i;
    Desc d;
    decode(raw, &d);
    if (validate(raw, d, core_id, gemv_only) != E_OK) continue;
    if (d.conv()) conv = std::max<uint64_t>(conv, d[F_M] * d[F_K]);
    if (d.op() == OP_GEMM && d.w4() && d[F_M] <= 4) {
      w4 = std::max<uint64_t>(w4, w4_scratch_bytes((int)d[F_M], (int)d[F_K]));
      ++nw4;
    }
  }
  return {conv, (w4 + 255) / 256 * 256, std::min(nw4, kW4Slices)};
}
// Captures a queue as a graph of dependency levels. Every descriptor's byte footprint (bounding
// interval per input tensor and per output) is compared with those of the earlier descriptors; a
// read-after-write, write-after-read or write-after-write overlap orders the pair. A descriptor's
// level is one more than the highest level among the earlier descriptors it overlaps, so the
// descriptors of one level are pairwise independent and every hazard points to a lower level.
// Each level runs after the previous one; inside a level the row ops, and (in a level of nothing
// but GEMVs and row ops) the decode GEMVs of one kernel class, become one launch each (up to
// kGroupMax entries), and the remaining descriptors and groups run side by side on the capture
// streams. The conv gather buffer counts as a written input of every conv; the W4A16 GEMVs of a
// level each align their activation rows into a scratch slice of their own (at most kW4Slices
// per level) and those of one row block and K become one grouped launch. Independent work
// commutes, so the bytes written are those of the in-order run.
struct Iv { u128 lo, hi; };

bool hits(const std::vector<Iv>& a, const std::vector<Iv>& b) {
  for (const Iv& x : a)
    for (const Iv& y : b)
      if (x.lo < y.hi && y.lo < x.hi) return true;
  return false;
}

struct LevelNode {
  Desc d;
  std::vector<Iv> r, w;
  int level;
  uint64_t w4_off = 0;                              // the W4A16 GEMV's scratch slice
};

int capture_grouped(tc_machine* m, uint64_t qaddr, uint32_t qlen, int32_t core_id, int32_t gemv_only, tc_status* st,
                    int32_t* contract_op, const std::vector<uint8_t>& q, std::vector<cudaEvent_t>& evs,
                    std::vector<cudaEvent_t>* marks) {
  const int kLanes = 16;
  while ((int)m->lanes.size() < kLanes) {
    cudaStream_t s;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) return fail(m, "capture streams", e);
    m->lanes.push_back(s);
  }
  std::vector<LevelNode> nodes;
  std::vector<int> w4_in_level;                     // W4A16 GEMVs (scratch slices) per level
  int top = -1;                                     // highest level so far
  const u128 kScratch = ((u128)1) << 120;          // a key outside every image for the gather buffer
  int rc = execute(m, qaddr, qlen, core_id, gemv_only, st, contract_op, q, true,
                   [&](uint32_t, const Desc& d, const Footprint& fp) {
    LevelNode nd;
    nd.d = d;
    for (const auto& t : fp.reads)
      for (const auto& sg : t) nd.r.push_back(Iv{sg.base, seg_end(sg)});
    nd.w.push_back(Iv{fp.y.base, seg_end(fp.y)});
    if (fp.has_extra) nd.w.push_back(Iv{fp.extra.base, seg_end(fp.extra)});
    if (d.conv()) nd.w.push_back(Iv{kScratch, kScratch + 1});
    int lvl = 0;
    for (int k = (int)nodes.size() - 1; k >= 0 && lvl <= top; --k) {
      const LevelNode& o = nodes[k];
      if (o.level < lvl) continue;                  // cannot raise the level
      if (hits(o.w, nd.r) || hits(o.w, nd.w) || hits(o.r, nd.w)) lvl = o.level + 1;
    }
    if (d.op() == OP_GEMM && d.w4() && d[F_M] <= 4) {
      // a scratch slice of its own in the level; a full level sends it to a later one
      while ((int)w4_in_level.size() <= lvl) w4_in_level.push_back(0);
      while (w4_in_level[lvl] >= kW4Slices) {
        ++lvl;
        if ((int)w4_in_level.size() <= lvl) w4_in_level.push_back(0);
      }
      nd.w4_off = (uint64_t)w4_in_level[lvl]++ * m->w4s_slice;
    }
    nd.level = lvl;
    top = std::max(top, lvl);
    nodes.push_back(std::move(nd));
  }, [](uint32_t) {}, [](const Desc&) { return cudaSuccess; });
  if (rc != TC_OK) return rc;

  auto new_event = [&]() {
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    evs.push_back(ev);
    return ev;
  };
  std::vector<std::vector<int>> levels(top + 1);
  for (int i = 0; i < (int)nodes.size(); ++i) levels[nodes[i].level].push_back(i);
  // marks: an external (timing) event before each level and one after the last
  auto mark = [&]() {
    if (!marks) return;
    cudaEvent_t ev;
    cudaEventCreate(&ev);
    marks->push_back(ev);
    cudaEventRecordWithFlags(ev, m->stream, cudaEventRecordExternal);
  };
  for (const auto& lv : levels) {
    mark();
    // the level's launch units: GEMV groups per class, row-op groups, single descriptors
    std::vector<std::function<cudaError_t(cudaStream_t)>> units;
    std::vector<std::pair<int, std::vector<GemmArgs>>> gemvs;   // class -> entries
    std::vector<std::pair<int, std::vector<W4Args>>> w4g;      // W4A16 class -> entries
    std::vector<RowArgs> rows;
    for (int i : lv) {
      const Desc& d = nodes[i].d;
      if (d.op() == OP_GEMM && !d.conv() && d.w4()) {
        const W4Args g = w4_args(m, d, nodes[i].w4_off);
        const int cls = w4_group_class(g);
        if (cls >= 0) {
          auto it = std::find_if(w4g.begin(), w4g.end(), [&](const auto& c) { return c.first == cls; });
          if (it == w4g.end()) w4g.push_back({cls, {g}});
          else it->second.push_back(g);
          continue;
        }
      } else if (d.op() == OP_GEMM && !d.conv()) {
        GemmArgs g{};
        gemm_args(m, d, &g);
        const int cls = gemv8_class(g);
        if (cls >= 0) {
          auto it = std::find_if(gemvs.begin(), gemvs.end(), [&](const auto& c) { return c.first == cls; });
          if (it == gemvs.end()) gemvs.push_back({cls, {g}});
          else it->second.push_back(g);
          continue;
        }
      } else if (d.op() == OP_ROW) {
        RowArgs a{};
        row_args(m, d, &a);
        if (rowop_groupable(a)) {
          rows.push_back(a);
          continue;
        }
      }
      const uint64_t w4_off = nodes[i].w4_off;
      units.push_back([m, d, w4_off](cudaStream_t s) { return launch_on(m, d, s, w4_off); });
    }
    // the streaming GEMV group fills every SM's shared memory; beside other work in the level (a
    // tensor-core GEMM, a W4A16 GEMV, ...) the GEMVs run as launches of their own instead
    const bool alone = units.empty();
    for (size_t ci = 0; ci < gemvs.size(); ++ci) {
      const int cls = gemvs[ci].first;
      const auto& gs = gemvs[ci].second;
      if (!alone) {
        for (const GemmArgs& g : gs) units.push_back([g](cudaStream_t s) { return launch_gemm_w8a8(g, s); });
        continue;
      }
      for (size_t j0 = 0; j0 < gs.size(); j0 += kGroupMax) {
        const int n = (int)std::min<size_t>(kGroupMax, gs.size() - j0);
        if (n == 1) {
          const GemmArgs g = gs[j0];
          units.push_back([g](cudaStream_t s) { return launch_gemm_w8a8(g, s); });
          continue;
        }
        auto grp = std::make_shared<GemvGroup>();
        grp->n = n; grp->mb = cls >> 4; grp->ku = cls & 15;
        for (int j = 0; j < n; ++j) grp->g[j] = gs[j0 + j];
        units.push_back([grp](cudaStream_t s) { return launch_gemv8_group(*grp, s); });
      }
    }
    // the tiled W4A16 GEMVs of one class: one pre-pass and one streaming launch per kW4GroupMax
    for (const auto& c : w4g)
      for (size_t j0 = 0; j0 < c.second.size(); j0 += kW4GroupMax) {
        auto grp = std::make_shared<std::vector<W4Args>>(
            c.second.begin() + j0, c.second.begin() + std::min(c.second.size(), j0 + kW4GroupMax));
        units.push_back([grp](cudaStream_t s) { return launch_w4_group(grp->data(), (int)grp->size(), s); });
      }
    for (size_t j0 = 0; j0 < rows.size(); j0 += kGroupMax) {
      const int n = (int)std::min<size_t>(kGroupMax, rows.size() - j0);
      if (n == 1) {
        const RowArgs a = rows[j0];
        units.push_back([a](cudaStream_t s) { return launch_rowop(a, s); });
        continue;
      }
      auto grp = std::make_shared<RowGroup>();
      grp->n = n; grp->nmax = 0; grp->row0[0] = 0;
      for (int j = 0; j < n; ++j) {
        grp->a[j] = rows[j0 + j];
        grp->nmax = std::max(grp->nmax, grp->a[j].N);
        grp->row0[j + 1] = grp->row0[j] + grp->a[j].M;
      }
      units.push_back([grp](cudaStream_t s) { return launch_rowop_group(*grp, s); });
    }
    if (units.size() == 1) {
      cudaError_t e = units[0](m->stream);
      if (e != cudaSuccess) return fail(m, "launch", e);
      continue;
    }
    // fork: the lanes start after everything before this level; join: the next level waits for all
    cudaEvent_t fork = new_event();
    cudaEventRecord(fork, m->stream);
    const int used = (int)std::min<size_t>(units.size(), kLanes);
    for (int l = 0; l < used; ++l) cudaStreamWaitEvent(m->lanes[l], fork, 0);
    for (size_t u = 0; u < units.size(); ++u) {
      cudaError_t e = units[u](m->lanes[u % kLanes]);
      if (e != cudaSuccess) return fail(m, "launch", e);
    }
    for (int l = 0; l < used; ++l) {
      cudaEvent_t join = new_event();
      cudaEventRecord(join, m->lanes[l]);
      cudaStreamWaitEvent(m->stream, join, 0);
    }
  }
  if (!levels.empty()) mark();
  return rc;
}
}  // namespace

extern "C" {

int tc_run_queue(tc_machine* m, uint64_t qaddr, uint32_t qlen, int32_t core_id, int32_t gemv_only,
                 tc_status* st, int32_t* contract_op) {
  cudaSetDevice(m->device);
  m->stats.clear();
  m->written.clear();
  m->err.clear();
  st->done = 0; st->err_code = E_OK; st->op_idx = 0;
  *contract_op = -1;
  std::vector<uint8_t> q;
  cudaError_t e = fetch_queue(m, qaddr, qlen, q);
  if (e != cudaSuccess) return fail(m, "queue fetch", e);
  int rc = execute(m, qaddr, qlen, core_id, gemv_only, st, contract_op, q, false,
                   [](uint32_t, const Desc&, const Footprint&) {}, [](uint32_t) {},
                   [m](const Desc& d) { return launch(m, d); });
  cudaError_t se = cudaStreamSynchronize(m->stream);
  if (se != cudaSuccess && rc >= 0) rc = fail(m, "queue run", se);
  return rc;
}

int tc_queue_capture(tc_machine* m, uint64_t qaddr, uint32_t qlen, int32_t core_id, int32_t gemv_only,
                     int32_t timing, tc_status* st, int32_t* contract_op, tc_graph** out) {
  *out = nullptr;
  cudaSetDevice(m->device);
  m->stats.clear();
  m->written.clear();
  m->err.clear();
  st->done = 0; st->err_code = E_OK; st->op_idx = 0;
  *contract_op = -1;
  std::vector<uint8_t> q;
  cudaError_t e = fetch_queue(m, qaddr, qlen, q);
  if (e == cudaSuccess) {
    const ScratchNeed need = scratch_need(q, qlen, core_id, gemv_only);
    m->w4s_slice = need.w4_slice;
    e = ensure_scratch(m, need.conv);
    if (e == cudaSuccess) e = ensure_w4s(m, need.w4_slice * (uint64_t)need.w4_slices);
  }
  if (e != cudaSuccess) return fail(m, "capture setup", e);
  tc_graph* g = new tc_graph();
  g->m = m;
  if (timing == 1) {
    g->events.resize((size_t)qlen + 1);
    for (auto& ev : g->events) cudaEventCreate(&ev);
  }
  e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) { delete g; return fail(m, "begin capture", e); }
  uint32_t last = 0;
  int rc;
  std::vector<cudaEvent_t> dag_events;
  if (timing == 1) {
    rc = execute(m, qaddr, qlen, core_id, gemv_only, st, contract_op, q, true,
                 [&](uint32_t i, const Desc&, const Footprint&) {
      // an external record node: a plain cudaEventRecord inside a capture only orders work
      cudaEventRecordWithFlags(g->events[i], m->stream, cudaEventRecordExternal);
      last = i + 1;
    }, [](uint32_t) {}, [m](const Desc& d) { return launch(m, d); });
    if (last) cudaEventRecordWithFlags(g->events[last], m->stream, cudaEventRecordExternal);
  } else {
    rc = capture_grouped(m, qaddr, qlen, core_id, gemv_only, st, contract_op, q, dag_events,
                         timing == 2 ? &g->events : nullptr);
  }
  cudaGraph_t graph = nullptr;
  cudaError_t ce = cudaStreamEndCapture(m->stream, &graph);
  if (rc == TC_OK && ce != cudaSuccess) rc = fail(m, "end capture", ce);
  if (rc == TC_OK) {
    size_t nn = 0;
    ce = cudaGraphGetNodes(graph, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    if (ce == cudaSuccess && nn) ce = cudaGraphGetNodes(graph, nodes.data(), &nn);
    for (size_t k = 0; ce == cudaSuccess && k < nn; ++k) {
      cudaGraphNodeType t;
      ce = cudaGraphNodeGetType(nodes[k], &t);
      if (ce == cudaSuccess && t == cudaGraphNodeTypeKernel) ++g->kernels;
    }
    if (ce != cudaSuccess) rc = fail(m, "graph nodes", ce);
  }
  if (rc == TC_OK) {
    ce = cudaGraphInstantiate(&g->exec, graph, 0);
    if (ce != cudaSuccess) rc = fail(m, "instantiate", ce);
  }
  if (graph) cudaGraphDestroy(graph);
  for (auto ev : dag_events) cudaEventDestroy(ev);
  if (rc != TC_OK) {
    for (auto& ev : g->events) cudaEventDestroy(ev);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    delete g;
    return rc;
  }
  if (timing == 1) g->events.resize(last + (last ? 1 : 0));
  g->stats = m->stats;
  g->written = m->written;
  g->status = *st;
  *out = g;
  return TC_OK;
}

int tc_graph_launch(tc_graph* g, void* stream) {
  tc_machine* m = g->m;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  cudaError_t e = cudaGraphLaunch(g->exec, s);
  if (e != cudaSuccess) return fail(m, "graph launch", e);
  m->stats = g->stats;
  m->written = g->written;
  return TC_OK;
}

int tc_graph_times(tc_graph* g, float* ms, uint32_t cap) {
  if (g->events.size() < 2) return 0;
  const uint32_t n = (uint32_t)g->events.size() - 1;
  for (uint32_t i = 0; i < std::min(cap, n); ++i) {
    cudaError_t e = cudaEventElapsedTime(&ms[i], g->events[i], g->events[i + 1]);
    if (e != cudaSuccess) return fail(g->m, "event time", e);
  }
  return (int)n;
}

int tc_graph_kernels(tc_graph* g) { return g ? g->kernels : TC_ERR_ARG; }

int tc_graph_destroy(tc_graph* g) {
  if (!g) return TC_OK;
  cudaSetDevice(g->m->device);
  for (auto& ev : g->events) cudaEventDestroy(ev);
  if (g->exec) cudaGraphExecDestroy(g->exec);
  delete g;
  return TC_OK;
}

int tc_synchronize(tc_machine* m) {
  cudaSetDevice(m->device);
  cudaError_t e = cudaStreamSynchronize(m->stream);
  return e == cudaSuccess ? TC_OK : fail(m, "synchronize", e);
}


int tc_version(void) { return TC_ABI_VERSION; }

int tc_open(int device, uint64_t ddr_bytes, tc_machine** out) {
  *out = nullptr;
  tc_machine* m = new tc_machine();
  m->device = device;
  m->size = ddr_bytes;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&m->dev, std::max<uint64_t>(ddr_bytes, 256));
  if (e == cudaSuccess) e = cudaMemsetAsync(m->dev, 0, std::max<uint64_t>(ddr_bytes, 256), m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) {
    if (m->dev) cudaFree(m->dev);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return TC_ERR_CUDA;
  }
  *out = m;
  return TC_OK;
}

int tc_close(tc_machine* m) {
  if (!m) return TC_OK;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (auto s : m->lanes) cudaStreamDestroy(s);
  if (m->scratch) cudaFree(m->scratch);
  if (m->w4s) cudaFree(m->w4s);
  if (m->dev) cudaFree(m->dev);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
  return TC_OK;
}

const char* tc_last_error(tc_machine* m) { return m ? m->err.c_str() : ""; }

uint64_t tc_device_ptr(tc_machine* m) { return (uint64_t)(uintptr_t)m->dev; }
void* tc_stream(tc_machine* m) { return (void*)m->stream; }

int tc_upload(tc_machine* m, uint64_t addr, const void* src, uint64_t n) {
  if (addr > m->size || n > m->size - addr) { m->err = "upload out of range"; return TC_ERR_ARG; }
  cudaSetDevice(m->device);
  cudaError_t e = cudaMemcpyAsync(m->dev + addr, src, n, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  return e == cudaSuccess ? TC_OK : fail(m, "upload", e);
}

int tc_download(tc_machine* m, uint64_t addr, void* dst, uint64_t n) {
  if (addr > m->size || n > m->size - addr) { m->err = "download out of range"; return TC_ERR_ARG; }
  cudaSetDevice(m->device);
  cudaError_t e = cudaMemcpyAsync(dst, m->dev + addr, n, cudaMemcpyDeviceToHost, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  return e == cudaSuccess ? TC_OK : fail(m, "download", e);
}

int tc_sync_up(tc_machine* m, const void* host, void* shadow, uint64_t n, uint64_t* uploaded) {
  if (n != m->size) { m->err = "image size mismatch"; return TC_ERR_ARG; }
  const uint8_t* h = (const uint8_t*)host;
  uint8_t* s = (uint8_t*)shadow;
  const uint64_t blk = 1 << 16;
  const uint64_t nblk = (n + blk - 1) / blk;
  std::vector<uint8_t> dirty(nblk, 0);
  const unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  auto work = [&](unsigned t) {
    for (uint64_t b = t; b < nblk; b += nt) {
      const uint64_t lo = b * blk, len = std::min(blk, n - lo);
      if (std::memcmp(h + lo, s + lo, len) != 0) {
        dirty[b] = 1;
        std::memcpy(s + lo, h + lo, len);
      }
    }
  };
  if (n >= (32u << 20) && nt > 1) {
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t) th.emplace_back(work, t);
    for (auto& t : th) t.join();
  } else {
    work(0);
    for (unsigned t = 1; t < nt; ++t) work(t);
  }
  cudaSetDevice(m->device);
  uint64_t total = 0;
  for (uint64_t b = 0; b < nblk;) {
    if (!dirty[b]) { ++b; continue; }
    uint64_t e = b;
    while (e < nblk && dirty[e]) ++e;
    const uint64_t lo = b * blk, hi = std::min(n, e * blk);
    cudaError_t err = cudaMemcpyAsync(m->dev + lo, s + lo, hi - lo, cudaMemcpyHostToDevice, m->stream);
    if (err != cudaSuccess) return fail(m, "sync_up", err);
    total += hi - lo;
    b = e;
  }
  cudaError_t err = cudaStreamSynchronize(m->stream);
  if (err != cudaSuccess) return fail(m, "sync_up", err);
  if (uploaded) *uploaded = total;
  return TC_OK;
}

int tc_sync_down(tc_machine* m, void* host, void* shadow) {
  cudaSetDevice(m->device);
  auto& w = m->written;
  std::sort(w.begin(), w.end());
  std::vector<std::pair<uint64_t, uint64_t>> merged;
  for (auto& r : w) {
    if (!merged.empty() && r.first <= merged.back().second) merged.back().second = std::max(merged.back().second, r.second);
    else merged.push_back(r);
  }
  uint8_t* h = (uint8_t*)host;
  for (auto& r : merged) {
    cudaError_t e = cudaMemcpyAsync(h + r.first, m->dev + r.first, r.second - r.first, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) return fail(m, "sync_down", e);
  }
  cudaError_t e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return fail(m, "sync_down", e);
  if (shadow)
    for (auto& r : merged) std::memcpy((uint8_t*)shadow + r.first, h + r.first, r.second - r.first);
  w.clear();
  return TC_OK;
}

int tc_validate(const uint8_t* raw, int32_t core_id, int32_t gemv_only, uint64_t* fields) {
  Desc d;
  decode(raw, &d);
  if (fields) std::memcpy(fields, d.f, sizeof(d.f));
  return validate(raw, d, core_id, gemv_only);
}

int tc_footprint(const uint8_t* raw, tc_seg* out, uint32_t cap, uint32_t* count) {
  Desc d;
  decode(raw, &d);
  Footprint fp = footprint(d);
  std::vector<tc_seg> v;
  auto put = [&](int kind, const Seg& s) {
    tc_seg t;
    t.kind = kind;
    t.base_lo = (uint64_t)s.base;
    t.base_hi = (uint64_t)(s.base >> 64);
    t.ld = (uint64_t)s.ld;
    t.nbytes = (uint64_t)s.nbytes;
    t.count = (uint64_t)s.count;
    v.push_back(t);
  };
  for (size_t j = 0; j < fp.reads.size(); ++j)
    for (auto& s : fp.reads[j]) put((int)j, s);
  put(-1, fp.y);
  if (fp.has_extra) put(-2, fp.extra);
  *count = (uint32_t)v.size();
  for (uint32_t i = 0; i < std::min<uint32_t>(cap, *count); ++i) out[i] = v[i];
  return TC_OK;
}

uint32_t tc_stats(tc_machine* m, tc_opstat* out, uint32_t cap) {
  const uint32_t n = (uint32_t)m->stats.size();
  for (uint32_t i = 0; i < std::min(cap, n); ++i) out[i] = m->stats[i];
  return n;
}

}  // extern "C"
