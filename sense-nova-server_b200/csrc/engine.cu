// The engine: the reference's Engine (src/engine.rs) on one B200.
//
// It owns every device buffer (weights, KV caches, DeltaNet states, activations),
// runs the op graph of engine.rs:383-493 in the same order, and keeps the same
// bookkeeping (pos, hid rows, hlast, checkpoints, snapshots). Differences by design:
//   * the embedding rows are dequantized on the device from token ids (the reference
//     does it on the host and uploads x);
//   * steps of 1 and 2 token rows (decode, speculative verify) are captured once into
//     CUDA graphs that read the step descriptor from device memory, so a decode token
//     is one graph launch plus a 4-byte (greedy) or vocab-float logits read-back;
//   * greedy callers get the argmax on the device (snl_engine_forward_greedy).
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemv_mma.cuh"
#include "synth.h"
#include "tp.cuh"
#include "synth_model.h"

namespace snl {

static thread_local std::string g_err;
static std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { g_err = msg; }
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  g_err = std::string(what) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) return SNL_E_OOM;
  return SNL_E_CUDA;
}
void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int launch_argmax_with(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, unsigned long long* part,
                       cudaStream_t s);

namespace {

constexpr size_t MAX_M = 512;      // engine.rs:18
constexpr size_t SNAPSHOTS = 4;    // engine.rs:20
constexpr size_t LOGIT_ROWS = 2;   // engine.rs:22
constexpr uint32_t MAX_PARTS = 64;  // engine.rs:827 clamp

struct QT {
  int dtype = 0;
  size_t rows = 0, cols = 0;
  void* q = nullptr;
  void* s = nullptr;
  int s_f16 = 0;
  // the same matrix in the tile layout of the decode GEMV (gemv_mma.cu)
  void* tiles = nullptr;
  void* tscales = nullptr;
  int tscale_f16 = 0;  // the tile scales are fp16 (every block scale is an fp16 number), else f32
  uint32_t pair_half = 0;  // tiles pair gate row i with up row i (a layer's gate_up)
  __half* wplanes = nullptr;  // fp16 hi/lo weight planes for the prefill GEMM (optional)
};
struct FT {
  float* p = nullptr;
  size_t n = 0;
};

uint32_t parts_for(size_t m, size_t total, uint32_t cap) {
  // engine.rs:827: split-K attention only for short steps. The reference splits every
  // 256 keys; here a part is kAttKeysPerPart keys (one 8-key group per warp of
  // attend_kernel), so short contexts spread over more CTAs, up to cap parts. The split
  // changes only the summation order.
  if (m > 4) return 1;
  size_t p = (total + kAttKeysPerPart - 1) / kAttKeysPerPart;
  return (uint32_t)std::min<size_t>(std::max<size_t>(p, 1), cap);
}

}  // namespace
}  // namespace snl

struct snl_engine {
  snl_model_config cfg;
  // This rank's shard of the model: cfg with the head counts and intermediate size
  // divided by the tensor-parallel size (cfg itself when it is 1).
  snl_model_config lc;
  uint32_t vocab_l = 0;  // LM-head rows on this rank
  snl::TpHost tp;
  unsigned long long* step_ctr = nullptr;  // steps run (exchange epochs), bumped by the embedding
  uint32_t att_parts = 0;  // split-key parts of a decode step's attention (att_parts())
  float* logits_full = nullptr;            // tensor parallel: gathered logits [2][vocab]
  float* head_out = nullptr;               // where the LM head writes [rows][vocab_l]
  uint32_t tp_sites = 0;                   // exchanges per step: 2 per layer visit + 2 (head)
  size_t ctx = 0;
  int device = 0;
  uint32_t flags = 0;
  bool has_mtp = false;
  bool finalized = false;
  cudaStream_t stream = nullptr;
  std::map<std::string, snl::QT> qw;
  std::map<std::string, snl::FT> fv;
  std::vector<size_t> plan;
  std::vector<void*> allocs;
  size_t bytes = 0;

  // activations (engine.rs:243-273)
  float *x = nullptr, *xn = nullptr, *proj = nullptr, *act = nullptr, *attn_out = nullptr, *branch = nullptr,
        *qbuf = nullptr, *coef = nullptr, *partial = nullptr, *logits = nullptr, *hid = nullptr, *hlast = nullptr,
        *mhc_raw = nullptr;
  uint32_t *rpos = nullptr, *tokens = nullptr, *amax = nullptr;
  unsigned long long* amax_part = nullptr;
  snl_step_u *step_d = nullptr, *mstep_d = nullptr;
  // caches (engine.rs:275-297)
  float *lin_state = nullptr, *conv_state = nullptr, *lin_ckpt = nullptr, *conv_ckpt = nullptr;
  size_t state_elems = 0, conv_elems = 0, n_lin = 0, n_full = 0;
  std::vector<uint32_t*> kc, vc;
  std::vector<float*> snap_lin, snap_conv, snap_h;
  // MTP (engine.rs:495-580)
  float *mx = nullptr, *hn = nullptr, *m_logits = nullptr;
  uint32_t *m_kc = nullptr, *m_vc = nullptr;
  uint64_t mtp_drafts = 0;  // tensor parallel: drafts run (their argmax key sets alternate)
  // pinned host staging
  uint32_t* h_tokens = nullptr;
  uint32_t* h_rpos = nullptr;
  snl_step_u* h_step = nullptr;
  float* h_logits = nullptr;
  uint32_t* h_amax = nullptr;
  int* h_err = nullptr;  // the device error word, read back with each call's results

  size_t pos = 0, hid_rows = 0, head_rows = 1;
  // captured step graphs keyed by (m, head rows, ckpt, greedy)
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;
  };
  std::map<uint32_t, Graph> graphs;
  bool use_graphs = true;
  // Steps of <= 4 rows run their projections on the tensor-core GEMV, whose x operand is
  // these planes ([8][pstride] halves), written by the kernel that produces each input.
  bool use_tc = true;
  bool use_fused_norm = true;
  // On-device sampling (snl_engine_sample): logit rows of the last forward, scratch, the
  // history copied per call (grown on demand) and the result words.
  size_t last_logit_rows = 0;
  void* sample_scratch = nullptr;
  uint32_t* sample_out = nullptr;
  uint32_t* h_sample_out = nullptr;
  uint32_t* hist_d = nullptr;
  size_t hist_cap = 0;
  bool tiles_on = false;      // every quantized matrix has its tile-layout copy
  int* tile_flag = nullptr;   // scale check scratch: set when a block scale is not an fp16 number
  uint32_t tiles_f16 = 0, tiles_f32 = 0;  // matrices whose tile scales are fp16 / f32
  __half* xpl = nullptr;
  __half* xpl_act = nullptr;  // planes of the SwiGLU output, written by the gate_up GEMV
  __half* xpl_norm = nullptr;  // both residual streams x the next norm weight (fused norms)
  uint32_t pstride = 0;
  // Router partial sums written by the residual-merging GEMV for the next mHC norm.
  float* rpart = nullptr;
  float* dn_scratch = nullptr;  // chunk records of the chunked delta rule (prefill)
  bool rpart_ready = false;

  // Per-op timing of one eager step (snl_engine_profile).
  struct ProfRec {
    std::string label;
    double bytes;
    cudaEvent_t a, b;
  };
  std::vector<ProfRec>* prof = nullptr;

  size_t h() const { return cfg.hidden; }
};

namespace snl {
namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <class T>
int dalloc(snl_engine* e, T** p, size_t count) {
  void* ptr = nullptr;
  const size_t nbytes = std::max<size_t>(count * sizeof(T), 256);
  cudaError_t err = cudaMalloc(&ptr, nbytes);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc");
  err = cudaMemsetAsync(ptr, 0, nbytes, e->stream);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
  e->allocs.push_back(ptr);
  e->bytes += nbytes;
  *p = static_cast<T*>(ptr);
  return SNL_OK;
}

snl_layer_p layer_p(const snl_engine* e, uint32_t mode, bool last_row) {
  snl_layer_p p;
  p.h = e->cfg.hidden;
  p.mode = mode;
  p.last_row = last_row ? 1 : 0;
  p.eps = e->cfg.eps;
  p.weight_one = 1.0f;
  p.iterations = e->cfg.mhc_start >= 0 ? e->cfg.mhc_iterations : 0;
  p.inter = e->lc.intermediate;
  p.x_stride = 0;
  return p;
}

// The attention of this rank's shard (lc), or of the whole model (cfg: the MTP layer,
// which every rank runs in full).
snl_attn_p attn_p(const snl_engine* e, bool whole = false) {
  const snl_model_config& c = whole ? e->cfg : e->lc;
  snl_attn_p a;
  a.n_heads = c.n_heads;
  a.n_kv = c.n_kv_heads;
  a.rot_dim = e->cfg.rot_dim;
  a.proj_stride = (uint32_t)snl_synth::attn_proj_rows(c);
  a.rope_theta = e->cfg.rope_theta;
  a.eps = e->cfg.eps;
  a.scale = 1.0f / sqrtf((float)e->cfg.head_dim);
  a.mrope = ((3 * e->cfg.mrope_section[1]) << 16) | (3 * e->cfg.mrope_section[2]);
  return a;
}

snl_lin_p lin_p(const snl_engine* e) {
  snl_lin_p l;
  l.conv_dim = (uint32_t)snl_synth::conv_dim(e->lc);
  l.proj_stride = (uint32_t)snl_synth::lin_proj_rows(e->lc);
  l.n_k = e->lc.lin_k_heads;
  l.n_v = e->lc.lin_v_heads;
  l.eps = e->cfg.eps;
  l.pad[0] = l.pad[1] = l.pad[2] = 0;
  return l;
}

const QT* find_q(const snl_engine* e, const std::string& n) {
  auto it = e->qw.find(n);
  return it == e->qw.end() ? nullptr : &it->second;
}
const float* find_f(const snl_engine* e, const std::string& n) {
  auto it = e->fv.find(n);
  return it == e->fv.end() ? nullptr : it->second.p;
}

// Runs `fn` (one launch) and, while profiling, brackets it with CUDA events on the
// engine stream under `label` with its algorithmic byte count.
template <class F>
int timed(snl_engine* e, const std::string& label, double bytes, F&& fn) {
  if (!e->prof) return fn();
  snl_engine::ProfRec r{label, bytes, nullptr, nullptr};
  cudaEventCreate(&r.a);
  cudaEventCreate(&r.b);
  cudaEventRecord(r.a, e->stream);
  int rc = fn();
  cudaEventRecord(r.b, e->stream);
  e->prof->push_back(r);
  return rc;
}

// Bytes the GEMV streams for w: codes plus a block scale per 32 weights (fp16 or f32).
double qbytes(const QT& w) {
  const double n = (double)w.rows * w.cols;
  return (w.dtype == SNL_Q8_0 ? n : n / 2) + n / 32 * (w.tiles ? (w.tscale_f16 ? 2 : 4) : (w.s_f16 ? 2 : 4));
}

// One matrix op (engine.rs:336-363): y[r, y_stride] for rows_m token rows.
int mat(snl_engine* e, StepRef st, const QT& w, const float* x, size_t x_stride, float* y, size_t y_stride,
        uint32_t rows_m, uint32_t m_one = 0, uint32_t x_off = 0) {
  snl_mat_p p;
  p.n = (uint32_t)w.rows;
  p.k = (uint32_t)w.cols;
  p.x_off = x_off;
  p.x_stride = (uint32_t)x_stride;
  p.y_off = 0;
  p.y_stride = (uint32_t)y_stride;
  p.n_off = 0;
  p.m_one = m_one;
  const double bytes = qbytes(w) + 4.0 * rows_m * (w.cols + w.rows);
  const std::string label = "mat n=" + std::to_string(w.rows) + (m_one ? " (head)" : "");
  return timed(e, label, bytes,
               [&] { return launch_mat(w.dtype, st, p, x, w.q, w.s, w.s_f16, y, e->stream, rows_m, w.wplanes); });
}

// One projection of an eager step (the MTP layer and head) with 1-4 token rows: x packed
// into fp16 hi/lo planes and the tile GEMV, when the matrix has its tile copy; else mat().
int mat_tile(snl_engine* e, StepRef st, const QT& w, const float* x, size_t x_stride, float* y, size_t y_stride,
             uint32_t rows_m) {
  if (!w.tiles || !e->use_tc || rows_m == 0 || rows_m > 4) return mat(e, st, w, x, x_stride, y, y_stride, rows_m);
  SNL_TRY(timed(e, "XPack", 6.0 * rows_m * w.cols, [&] {
    return launch_xpack(x, rows_m, (uint32_t)w.cols, (uint32_t)x_stride, e->xpl, e->pstride, e->stream);
  }));
  GemvArgs a{};
  a.n = (uint32_t)w.rows;
  a.k = (uint32_t)w.cols;
  a.xplanes = e->xpl;
  a.plane_stride = e->pstride;
  a.mode = 0;
  a.y = y;
  a.y_stride = (uint32_t)y_stride;
  const double bytes = qbytes(w) + 4.0 * rows_m * (w.cols + w.rows);
  return timed(e, "mat n=" + std::to_string(w.rows), bytes,
               [&] { return launch_gemv_tile(w.dtype, a, rows_m, w.tiles, w.tscales, w.tscale_f16, e->stream); });
}

int push_norm(snl_engine* e, StepRef st, uint32_t m, const float* router, const float* norm_w, XOut xo = XOut()) {
  const double h = e->cfg.hidden;
  if (router && e->rpart_ready) {
    // The router sums were produced by the GEMV that merged the residual.
    e->rpart_ready = false;
    snl_layer_p p = layer_p(e, 1, false);
    const uint32_t nparts = (e->cfg.hidden + 15) / 16;
    return timed(e, "BranchNorm+Router", 4.0 * (m * 3 * h + h + 9.0 * nparts * m), [&] {
      return launch_branch_norm_router(st, p, e->x, e->coef, norm_w, e->xn, m, e->stream, xo, e->rpart, nparts, router);
    });
  }
  e->rpart_ready = false;
  if (router) {
    snl_layer_p p0 = layer_p(e, 0, false);
    SNL_TRY(timed(e, "MhcRouter", 4.0 * (16 * h + 8 + m * 2 * h),
                  [&] { return launch_mhc_router(p0, e->x, router, e->mhc_raw, e->coef, m, e->stream); }));
  }
  snl_layer_p p = layer_p(e, router ? 1 : 0, false);
  return timed(e, "BranchNorm", 4.0 * (m * 3 * h + h),
               [&] { return launch_branch_norm(st, p, e->x, e->coef, norm_w, e->xn, m, e->stream, xo); });
}

// One projection on the tensor-core GEMV (x = the planes). mode 0 writes y; mode 1
// merges into the residual x like `merge` (engine.rs:471-480) and can expand stream 0
// into stream 1 (the merge mode 3 that opens an mHC range).
// A norm folded into the GEMV that consumes it (see GemvArgs::fused_norm): `on` when the
// producing GEMV left the weighted streams in xpl_norm and the partials in rpart.
struct NormFuse {
  bool on = false;
  const float* router = nullptr;
};

int matx(snl_engine* e, const QT& w, uint32_t rows, int mode, float* y, size_t y_stride, uint32_t merge_mode = 0,
         int expand = 0, const float* rnext = nullptr, const __half* planes = nullptr, int tp_site = -1,
         const NormFuse& nf_in = NormFuse(), const float* nw_out = nullptr) {
  GemvArgs a{};
  a.n = (uint32_t)w.rows;
  a.k = (uint32_t)w.cols;
  a.xplanes = planes ? planes : e->xpl;
  a.act_planes = e->xpl_act;
  a.act_stride = e->pstride;
  uint32_t launch_rows = rows;
  if (nf_in.on) {  // the x operand is the two weighted streams of each token
    a.xplanes = e->xpl_norm;
    a.fused_norm = 1;
    a.nrpart = e->rpart;
    a.nparts = (uint32_t)((e->cfg.hidden + 15) / 16);
    a.nrouter = nf_in.router;
    a.neps = e->cfg.eps;
    a.niter = e->cfg.mhc_start >= 0 ? e->cfg.mhc_iterations : 0;
    a.ncoef = e->coef;
    launch_rows = 2 * rows;
  }
  if (nw_out) {  // leave the next norm's input for a fused consumer
    a.nplanes = e->xpl_norm;
    a.nstride = e->pstride;
    a.nw = nw_out;
    a.weight_one = 1.0f;
  }
  if (tp_site >= 0 && e->tp.size > 1) {
    a.tp = e->tp.comm;
    a.tp_site = (uint32_t)tp_site;
  }
  a.plane_stride = e->pstride;
  a.wq = static_cast<const uint8_t*>(w.q);
  a.mode = mode;
  a.y = y;
  a.y_stride = (uint32_t)y_stride;
  a.resid = e->x;
  a.coef = e->coef;
  a.h = e->cfg.hidden;
  a.merge_mode = (int)merge_mode;
  a.expand = expand;
  a.rnext = rnext;
  a.rpart = mode == 1 && (rnext || nw_out) ? e->rpart : nullptr;
  const double bytes = qbytes(w) + 4.0 * rows * (w.cols + w.rows);
  const std::string label = "mat n=" + std::to_string(w.rows) + (y == e->head_out ? " (head)" : "");
  SNL_TRY(timed(e, label, bytes, [&] {
    if (w.tiles) return launch_gemv_tile(w.dtype, a, launch_rows, w.tiles, w.tscales, w.tscale_f16, e->stream);
    if (nf_in.on) return fail(SNL_E_STATE, "fused norm needs the tile layout");
    return launch_gemv_mma(w.dtype, a, rows, w.s, w.s_f16, e->stream);
  }));
  e->rpart_ready = rnext != nullptr;
  return SNL_OK;
}

// Element offset of this rank's o_proj input inside the attention output (non-zero
// only when ranks outnumber KV heads and a rank computes a whole GQA group).
size_t o_proj_offset(const snl_engine* e) {
  const auto& c = e->cfg;
  const size_t N = (size_t)e->tp.size;
  if (N <= c.n_kv_heads) return 0;
  const size_t nq = c.n_heads / N;
  return ((size_t)e->tp.rank % (N / c.n_kv_heads)) * nq * c.head_dim;
}

// The layer loop of engine.rs:389-481 for one step of m rows.
// Part slots of a decode step's attention (the captured graphs use all of them): one
// attend CTA per (local KV head, part) and at most one wave of them, since an attend CTA
// holds an SM's registers (189 per thread): 37 parts for 4 KV heads on 148 SMs, against
// 64 before (two waves at long contexts: 246.8 -> 252.4 tok/s at a 32K context).
// SNL_ATT_PARTS overrides it; at most MAX_PARTS (the partial buffer's slots).
uint32_t att_parts(snl_engine* e) {
  if (!e->att_parts) {
    const char* v = getenv("SNL_ATT_PARTS");
    long p = v ? strtol(v, nullptr, 10) : (long)sm_count() / (long)std::max<uint32_t>(e->lc.n_kv_heads, 1);
    e->att_parts = (uint32_t)std::min<long>(std::max<long>(p, 1), (long)MAX_PARTS);
  }
  return e->att_parts;
}

int run_layers(snl_engine* e, StepRef st, uint32_t m, uint32_t parts_grid) {
  const auto& c = e->lc;
  const size_t h = c.hidden;
  size_t lin_slot = 0, full_slot = 0;
  const snl_attn_p ap = attn_p(e);
  const snl_lin_p lp = lin_p(e);
  const bool tc = e->use_tc && m <= 4;
  const XOut xo = tc ? XOut{e->xpl, e->pstride} : XOut{};
  const double hb = 4.0 * m * h;
  // in-projection (x = normed residual) into y
  // Fused norms (1-2 token rows on the tile path): a residual-merging GEMV leaves the next
  // norm's weighted streams and partials, and the next projection finishes the norm.
  const bool fuse = tc && m <= 2 && e->use_fused_norm && e->tiles_on;
  bool fused_ready = false;  // xpl_norm and rpart hold the inputs of the upcoming norm
  NormFuse pending;          // a norm deferred into the next projection
  auto norm_step = [&](const float* router, const float* norm_w) -> int {
    if (fuse && fused_ready) {
      pending.on = true;
      pending.router = router;
      fused_ready = false;
      return SNL_OK;
    }
    pending.on = false;
    return push_norm(e, st, m, router, norm_w, xo);
  };
  auto take_pending = [&]() {
    NormFuse f = pending;
    pending.on = false;
    return f;
  };
  auto proj_in = [&](const QT& w, float* y, size_t y_stride) -> int {
    if (tc) return matx(e, w, m, 0, y, y_stride, 0, 0, nullptr, nullptr, -1, take_pending());
    return mat(e, st, w, e->xn, h, y, y_stride, m);
  };
  // out-projection of `src` (K = src_dim) merged into the residual
  // Under tensor parallelism the out-projections are row-parallel: the tensor-core GEMV
  // trades partials with the peers in its epilogue; the prefill GEMM writes this rank's
  // partial into the exchange region and an allreduce kernel sums the ranks' partials.
  auto proj_out = [&](const QT& w, const float* src, size_t src_dim, uint32_t merge_mode, bool expand,
                      const float* rnext, const __half* planes, uint32_t site, const float* next_norm_w) -> int {
    if (tc) {
      const float* nw = fuse ? next_norm_w : nullptr;
      SNL_TRY(matx(e, w, m, 1, nullptr, 0, merge_mode, expand ? 1 : 0, rnext, planes, (int)site, NormFuse(), nw));
      fused_ready = nw != nullptr;
      return SNL_OK;
    }
    if (e->tp.size > 1) {
      const uint64_t par = (((uint64_t)site + 1) & 1) * e->tp.comm.bp_elems;  // tp_sites is even
      float* part = e->tp.comm.bparts[e->tp.rank] + par;
      SNL_TRY(mat(e, st, w, src, src_dim, part, h, m));
      SNL_TRY(timed(e, "TpAllreduce", 4.0 * m * h * e->tp.size,
                    [&] { return launch_tp_allreduce(e->tp.comm, site, (uint64_t)m * h, e->branch, e->stream); }));
    } else {
      SNL_TRY(mat(e, st, w, src, src_dim, e->branch, h, m));
    }
    SNL_TRY(timed(e, "Merge", 5 * hb, [&] {
      return launch_merge(st, layer_p(e, merge_mode, false), e->x, e->coef, e->branch, m, e->stream);
    }));
    if (expand)
      SNL_TRY(timed(e, "Merge", 2 * hb, [&] { return launch_merge(st, layer_p(e, 3, false), e->x, e->coef, e->branch, m, e->stream); }));
    return SNL_OK;
  };
  bool expanded = false;  // the previous visit's last merge already opened the mHC range
  e->rpart_ready = false;
  for (size_t vi = 0; vi < e->plan.size(); vi++) {
    const size_t li = e->plan[vi];
    const std::string L = "l" + std::to_string(li) + ".";
    const bool mhc = snl_synth::is_mhc(c, li);
    if (mhc && (int32_t)li == c.mhc_start && !expanded) {
      SNL_TRY(timed(e, "Merge", 2 * hb, [&] { return launch_merge(st, layer_p(e, 3, false), e->x, e->coef, e->branch, m, e->stream); }));
      fused_ready = false;  // the streams changed after the fused inputs were written
    }
    SNL_TRY(norm_step(mhc ? find_f(e, L + "mhc_attn") : nullptr, find_f(e, L + "in_ln")));
    if (c.full_attention[li]) {
      SNL_TRY(proj_in(*find_q(e, L + "qkv"), e->proj, ap.proj_stride));
      const double kvd = (double)snl_synth::kv_dim(c), qd = (double)snl_synth::q_dim(c);
      SNL_TRY(timed(e, "AttnPrep", 4.0 * m * (qd + 2 * kvd) + 4.0 * m * qd + 2.0 * m * 2 * kvd, [&] {
        return launch_attn_prep(st, ap, e->proj, e->qbuf, e->kc[full_slot], e->vc[full_slot], find_f(e, L + "qk_norm"),
                                e->rpos, m, e->stream);
      }));
      const double keys = (double)st.val.pos0 + m;
      SNL_TRY(timed(e, "Attend", 2.0 * 2 * kvd * keys + 4.0 * m * 2 * qd, [&] {
        return launch_attend(st, ap, e->proj, e->qbuf, e->kc[full_slot], e->vc[full_slot], e->attn_out, e->partial, m,
                             parts_grid, e->stream, xo);
      }));
      if (parts_grid > 1)
        SNL_TRY(timed(e, "Combine", 4.0 * m * qd * 2, [&] {
          return launch_attn_combine(st, ap, e->proj, e->partial, e->attn_out, m, e->stream, parts_grid, xo);
        }));
      // o_proj's K shard: this rank's query heads within the attention it computed.
      const size_t xo_off = o_proj_offset(e);
      SNL_TRY(proj_out(*find_q(e, L + "o_proj"), e->attn_out + xo_off, snl_synth::q_dim(c), mhc ? 1 : 0, false,
                       mhc ? find_f(e, L + "mhc_ffn") : nullptr, tc ? e->xpl + xo_off : nullptr, (uint32_t)(2 * vi),
                       find_f(e, L + "post_ln")));
      full_slot++;
    } else {
      SNL_TRY(proj_in(*find_q(e, L + "in_proj"), e->proj, lp.proj_stride));
      float* cs = e->conv_state + lin_slot * e->conv_elems;
      float* ss = e->lin_state + lin_slot * e->state_elems;
      float* cc = e->conv_ckpt + lin_slot * e->conv_elems;
      float* sc = e->lin_ckpt + lin_slot * e->state_elems;
      const float* lw = find_f(e, L + "lin");
      const double cdim = (double)lp.conv_dim;
      if (!tc && m >= kChunkedMinRows && st.val.ckpt == 0) {
        // Prefill step: the chunked delta rule (conv_out in act, chunk records in dn_scratch).
        SNL_TRY(timed(e, "ConvDeltaChunked", 4.0 * (2.0 * e->state_elems + m * (3.0 * cdim + 2 * 4096.0)), [&] {
          return launch_conv_delta_chunked(m, lp, e->proj, cs, ss, lw, e->attn_out, e->act, e->dn_scratch, e->stream);
        }));
      } else {
        SNL_TRY(timed(e, "ConvDelta", 4.0 * (2.0 * e->state_elems + 10.0 * cdim + m * (cdim + 2 * 4096.0)), [&] {
          return launch_conv_delta(st, lp, e->proj, cs, ss, lw, e->attn_out, cc, sc, e->stream, xo);
        }));
      }
      SNL_TRY(proj_out(*find_q(e, L + "out_proj"), e->attn_out, snl_synth::lin_value_dim(c), mhc ? 1 : 0, false,
                       mhc ? find_f(e, L + "mhc_ffn") : nullptr, nullptr, (uint32_t)(2 * vi), find_f(e, L + "post_ln")));
      lin_slot++;
    }
    SNL_TRY(norm_step(mhc ? find_f(e, L + "mhc_ffn") : nullptr, find_f(e, L + "post_ln")));
    const QT& gu = *find_q(e, L + "gate_up");
    const bool fused_swiglu = tc && gu.tiles && gu.pair_half;
    if (fused_swiglu) {
      // The gate_up GEMV finishes SwiGLU in its epilogue and writes the planes of act.
      SNL_TRY(matx(e, gu, m, 2, nullptr, c.intermediate, 0, 0, nullptr, nullptr, -1, take_pending()));
    } else {
      SNL_TRY(proj_in(gu, e->proj, 2 * (size_t)c.intermediate));
      SNL_TRY(timed(e, "Swiglu", 12.0 * m * c.intermediate,
                    [&] { return launch_swiglu(st, layer_p(e, 0, false), e->proj, e->act, m, e->stream, xo); }));
    }
    const uint32_t mode = !mhc ? 0 : ((int32_t)(li + 1) == c.mhc_end ? 2 : 1);
    const bool expand_next = vi + 1 < e->plan.size() && snl_synth::is_mhc(c, e->plan[vi + 1]) &&
                             (int32_t)e->plan[vi + 1] == c.mhc_start;
    const bool next_mhc = vi + 1 < e->plan.size() && snl_synth::is_mhc(c, e->plan[vi + 1]);
    const float* rnext = next_mhc ? find_f(e, "l" + std::to_string(e->plan[vi + 1]) + ".mhc_attn") : nullptr;
    const float* next_ln = vi + 1 < e->plan.size() ? find_f(e, "l" + std::to_string(e->plan[vi + 1]) + ".in_ln") : nullptr;
    SNL_TRY(proj_out(*find_q(e, L + "down"), e->act, c.intermediate, mode, expand_next, rnext,
                     fused_swiglu ? e->xpl_act : nullptr, (uint32_t)(2 * vi + 1), next_ln));
    expanded = expand_next;
  }
  return SNL_OK;
}

// Everything a step does on the device after its inputs (tokens, rpos, step) are
// resident: embedding, layers, final norm, optional head and argmax, hlast update.
int device_step(snl_engine* e, StepRef st, uint32_t m, uint32_t parts_grid, uint32_t rows, bool greedy,
                bool embed = true) {
  const size_t h = e->h();
  if (embed) {
    const QT* emb = find_q(e, "embed");
    SNL_TRY(timed(e, "Embed", (double)m * h * 13, [&] {
      return launch_embed(e->tokens, m, (const int8_t*)emb->q, (const float*)emb->s, (uint32_t)h, e->cfg.vocab, e->x,
                          nullptr, e->stream, e->step_ctr);
    }));
  }
  // Row 0 of hid is the hidden state of the token before this step (engine.rs:889-890).
  SNL_CUDA_TRY(cudaMemcpyAsync(e->hid, e->hlast, h * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
  SNL_TRY(run_layers(e, st, m, parts_grid));
  const bool tc = e->use_tc && m <= 4 && rows > 0;
  const XOut xo = (tc && rows == m) ? XOut{e->xpl, e->pstride} : XOut{};
  SNL_TRY(timed(e, "BranchNorm", 12.0 * m * h, [&] {
    return launch_branch_norm(st, layer_p(e, 0, false), e->x, e->coef, find_f(e, "norm"), e->hid + h, m, e->stream, xo);
  }));
  const uint32_t vl = e->vocab_l;
  if (rows > 0) {
    if (tc) {
      // The head reads the last `rows` hidden rows (engine.rs:835-842).
      if (rows != m)
        SNL_TRY(launch_xpack(e->hid + (size_t)(m - rows + 1) * h, rows, (uint32_t)h, (uint32_t)h, e->xpl, e->pstride,
                             e->stream));
      SNL_TRY(matx(e, *find_q(e, "lm_head"), rows, 0, e->head_out, vl));
    } else {
      SNL_TRY(mat(e, st, *find_q(e, "lm_head"), e->hid, h, e->head_out, vl, rows, rows,
                  (uint32_t)((m - rows + 1) * h)));
    }
  }
  if (e->tp.size > 1 && rows > 0) {
    // The last two exchange sites of a step: the logits shards are gathered when the
    // caller wants logits; the greedy token is the largest of the ranks' shard maxima
    // (first index on ties, as one scan of the whole row would find).
    const uint32_t site = e->tp_sites - 2;
    if (!greedy)
      SNL_TRY(timed(e, "TpGather", 4.0 * rows * e->cfg.vocab,
                    [&] { return launch_tp_gather_logits(e->tp.comm, site, rows, vl, e->logits_full, e->stream); }));
    else
      SNL_TRY(timed(e, "Argmax", 4.0 * rows * vl, [&] {
        return launch_argmax_tp(e->head_out, rows, vl, e->amax, e->amax_part, e->tp.comm, site + 1, e->stream);
      }));
  } else if (rows > 0 && greedy) {
    SNL_TRY(timed(e, "Argmax", 4.0 * rows * vl,
                  [&] { return launch_argmax_with(e->head_out, rows, vl, e->amax, e->amax_part, e->stream); }));
  }
  SNL_CUDA_TRY(cudaMemcpyAsync(e->hlast, e->hid + (size_t)m * h, h * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
  return SNL_OK;
}

// Run one step, through a captured graph for m <= 2.
int run_step(snl_engine* e, const snl_step_u& sh, uint32_t m, uint32_t rows, bool greedy) {
  StepRef st = step_dev(e->step_d, sh);
  const bool graphable = e->use_graphs && m <= 2;
  if (!graphable) {
    const uint32_t parts_grid = sh.parts;
    return device_step(e, st, m, parts_grid, rows, greedy);
  }
  const uint32_t key = (m << 8) | (rows << 4) | ((sh.ckpt ? 1u : 0u) << 1) | (greedy ? 1u : 0u);
  auto it = e->graphs.find(key);
  if (it == e->graphs.end()) {
    const uint64_t before = g_launches.load();
    SNL_CUDA_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = device_step(e, st, m, att_parts(e), rows, greedy);
    cudaGraph_t graph = nullptr;
    cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    snl_engine::Graph g;
    ce = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    g.launches = g_launches.load() - before;
    g_launches.fetch_sub(g.launches);  // captured, not executed
    it = e->graphs.emplace(key, g).first;
  }
  SNL_CUDA_TRY(cudaGraphLaunch(it->second.exec, e->stream));
  count_launch(it->second.launches);
  return SNL_OK;
}

// Queues the read-back of the device error word behind the call's work on the engine
// stream; take_device_error() reads it after the stream synchronizes.
int queue_error_read(snl_engine* e) {
  if (!e->h_err) return SNL_OK;
  int* w = nullptr;
  SNL_TRY(device_error_word(&w));
  SNL_CUDA_TRY(cudaMemcpyAsync(e->h_err, w, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  return SNL_OK;
}
// After the stream synchronized: a bounded device-side wait that gave up during the call
// (bit 1: a tensor-parallel peer never answered; bit 0: an asynchronous copy never
// landed) left the call's results undefined, so the call fails with SNL_E_TIMEOUT. The
// word is cleared, so the next call starts clean.
int take_device_error(snl_engine* e) {
  if (!e->h_err) return SNL_OK;
  const int v = *e->h_err;
  if (!v) return SNL_OK;
  *e->h_err = 0;
  int* w = nullptr;
  SNL_TRY(device_error_word(&w));
  SNL_CUDA_TRY(cudaMemsetAsync(w, 0, sizeof(int), e->stream));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  return fail(SNL_E_TIMEOUT, (v & 2) ? "a tensor-parallel peer did not answer within the wait bound "
                                       "(device error word " + std::to_string(v) + "); recreate the engines of every rank"
                                     : "a device-side wait gave up (device error word " + std::to_string(v) + ")");
}

int check_tokens(const snl_engine* e, const uint32_t* toks, size_t n) {
  for (size_t i = 0; i < n; i++)
    if (toks[i] >= e->cfg.vocab) return fail(SNL_E_RANGE, "token id " + std::to_string(toks[i]) + " out of range");
  return SNL_OK;
}

// forward_mm (engine.rs:801-936), leaving the logits (or the argmax) on the device.
int forward_impl(snl_engine* e, const uint32_t* tokens, size_t n, const uint32_t* pos3, const uint32_t* embed_idx,
                 const float* embeds, size_t n_embeds, size_t logit_rows, int ckpt, bool greedy, size_t* rows_out) {
  if (!e->finalized) return fail(SNL_E_STATE, "engine not finalized");
  if (logit_rows > LOGIT_ROWS || (ckpt && n != 2)) return fail(SNL_E_INVALID, "forward: unsupported logits or checkpoint request");
  if (n == 0 || !tokens) return fail(SNL_E_INVALID, "forward called with no tokens");
  for (size_t i = 0; i < n_embeds; i++)
    if (embed_idx[i] >= n) return fail(SNL_E_INVALID, "forward: positions or embeddings do not match the tokens");
  if (e->pos + n > e->ctx)
    return fail(SNL_E_RANGE, "context length exceeded (" + std::to_string(e->pos + n) + " > " + std::to_string(e->ctx) + ")");
  SNL_TRY(check_tokens(e, tokens, n));
  const size_t h = e->h();
  const size_t chunk = MAX_M;
  const size_t n_chunks = (n + chunk - 1) / chunk;
  *rows_out = 0;
  for (size_t ci = 0; ci < n_chunks; ci++) {
    const bool last = ci + 1 == n_chunks;
    const size_t c0 = ci * chunk;
    const size_t m = std::min(chunk, n - c0);
    const size_t total = e->pos + m;
    snl_step_u sh = {(uint32_t)m, (uint32_t)e->pos, parts_for(m, total, att_parts(e)), (uint32_t)(ckpt ? 1 : 0)};
    const size_t rows = (last && logit_rows > 0) ? std::min(logit_rows, m) : 0;
    if (rows) e->head_rows = rows;
    // Stage the step inputs through pinned memory.
    *e->h_step = sh;
    memcpy(e->h_tokens, tokens + c0, m * sizeof(uint32_t));
    for (size_t i = 0; i < m; i++)
      for (int k = 0; k < 4; k++)
        e->h_rpos[i * 4 + k] = pos3 ? (k < 3 ? pos3[(c0 + i) * 3 + k] : 0u) : (uint32_t)(e->pos + i);
    SNL_CUDA_TRY(cudaMemcpyAsync(e->step_d, e->h_step, sizeof(snl_step_u), cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(e->tokens, e->h_tokens, m * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(e->rpos, e->h_rpos, m * 4 * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
    bool has_embeds = false;
    for (size_t i = 0; i < n_embeds; i++) has_embeds |= embed_idx[i] >= c0 && embed_idx[i] < c0 + m;
    if (has_embeds) {
      // Vision features replace embedding rows: run the embedding first, then
      // overwrite, outside any graph.
      StepRef st = step_dev(e->step_d, sh);
      const QT* emb = find_q(e, "embed");
      SNL_TRY(launch_embed(e->tokens, (uint32_t)m, (const int8_t*)emb->q, (const float*)emb->s, (uint32_t)h,
                           e->cfg.vocab, e->x, nullptr, e->stream, e->step_ctr));
      for (size_t i = 0; i < n_embeds; i++) {
        const size_t r = embed_idx[i];
        if (r < c0 || r >= c0 + m) continue;
        SNL_CUDA_TRY(cudaMemcpyAsync(e->x + (r - c0) * 2 * h, embeds + i * h, h * sizeof(float), cudaMemcpyHostToDevice,
                                     e->stream));
      }
      SNL_TRY(device_step(e, st, (uint32_t)m, sh.parts, (uint32_t)rows, greedy, false));
    } else {
      SNL_TRY(run_step(e, sh, (uint32_t)m, (uint32_t)rows, greedy));
    }
    if (!last) SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));  // pinned staging is reused by the next chunk
    e->pos += m;
    e->hid_rows = m;
    if (rows) *rows_out = rows;
  }
  return SNL_OK;
}

}  // namespace
}  // namespace snl

using namespace snl;

// ---------------------------------------------------------------------------
// C ABI: errors, config
// ---------------------------------------------------------------------------

extern "C" const char* snl_last_error(void) { return snl::g_err.c_str(); }
extern "C" const char* snl_version(void) { return "snl_b200 0.1 (sm_100a)"; }
extern "C" uint64_t snl_launch_count(void) { return snl::g_launches.load(); }

extern "C" int snl_config_validate(const snl_model_config* c) {
  if (!c) return fail(SNL_E_INVALID, "null config");
  // ModelConfig::validate (config.rs:194-240)
  if (c->head_dim != 256) return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: head_dim must be 256");
  if (c->lin_k_dim != 128 || c->lin_v_dim != 128)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear head dims must be 128");
  if (c->conv_kernel != 4) return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear conv kernel must be 4");
  if (c->hidden == 0 || c->hidden % 256)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: hidden size must be a multiple of 256");
  if (c->n_layers == 0 || c->n_layers > SNL_MAX_LAYERS)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: layer_types length mismatch");
  if (c->n_kv_heads == 0 || c->n_heads != 4 * c->n_kv_heads)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: attention must have 4 query heads per KV head");
  if (c->lin_k_heads == 0 || c->lin_v_heads % c->lin_k_heads)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear value heads must be a multiple of key heads");
  if (c->rot_dim % 2 || c->rot_dim > c->head_dim || c->rot_dim == 0)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: invalid rotary dim");
  if (c->mrope_section[0] + c->mrope_section[1] + c->mrope_section[2] != c->rot_dim / 2)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: M-RoPE sections must cover the rotary dims");
  if (!(c->loop_start < c->loop_end && c->loop_end <= c->n_layers && c->loop_count >= 1))
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: invalid loop range");
  if (c->intermediate == 0 || c->intermediate % 32 || c->vocab == 0)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: intermediate/vocab");
  if (c->mhc_start >= 0) {
    if (c->mhc_streams != 2)
      return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: only 2 mHC streams are supported");
    auto inside = [&](uint32_t a, uint32_t b) { return a <= (uint32_t)c->mhc_start && (uint32_t)c->mhc_end <= b; };
    if (!(inside(0, c->loop_start) || inside(c->loop_start, c->loop_end) || inside(c->loop_end, c->n_layers)))
      return fail(SNL_E_UNSUPPORTED, "mHC range crosses a loop boundary");
  }
  return SNL_OK;
}

// ---------------------------------------------------------------------------
// C ABI: engine
// ---------------------------------------------------------------------------

extern "C" int snl_engine_create(const snl_model_config* cfg, size_t ctx, int device, uint32_t flags, snl_engine** out) {
  if (!out) return fail(SNL_E_INVALID, "snl_engine_create: null out");
  *out = nullptr;
  if (int rc = snl_config_validate(cfg)) return rc;
  int ndev = 0;
  cudaError_t ce = cudaGetDeviceCount(&ndev);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(SNL_E_INVALID, "snl_engine_create: no such device");
  DeviceGuard dg(device);
  snl_engine* e = new snl_engine();
  e->cfg = *cfg;
  e->lc = *cfg;
  e->vocab_l = cfg->vocab;
  e->ctx = std::min<size_t>(ctx, cfg->max_position);
  e->device = device;
  e->flags = flags;
  e->has_mtp = (flags & SNL_ENGINE_MTP) != 0;
  if (getenv("SNL_NO_GRAPHS")) e->use_graphs = false;
  ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    delete e;
    return cuda_fail(ce, "cudaStreamCreate");
  }
  const auto& c = e->cfg;
  for (size_t i = 0; i < c.loop_start; i++) e->plan.push_back(i);
  for (size_t r = 0; r < c.loop_count; r++)
    for (size_t i = c.loop_start; i < c.loop_end; i++) e->plan.push_back(i);
  for (size_t i = c.loop_end; i < c.n_layers; i++) e->plan.push_back(i);
  *out = e;
  return SNL_OK;
}

// ---------------------------------------------------------------------------
// Tensor parallelism (the Megatron split): column-parallel in-projections
// (qkv by head, in_proj by key/value head, gate_up by intermediate slice) and LM head
// (by vocabulary rows); row-parallel out-projections (o_proj, out_proj, down: K split)
// whose partial sums are exchanged over NVLink peer memory (tp.cuh). Norms, mHC and the
// embedding are replicated.
// ---------------------------------------------------------------------------
namespace {

struct RowRange {
  size_t a, n;
};

void dfree(snl_engine* e, void* p) {
  if (!p) return;
  auto it = std::find(e->allocs.begin(), e->allocs.end(), p);
  if (it != e->allocs.end()) e->allocs.erase(it);
  cudaFree(p);
}

// Keeps the rows `rs` (in order) of a quantized matrix.
int shard_rows(snl_engine* e, snl::QT& t, const std::vector<RowRange>& rs) {
  size_t rows = 0;
  for (const auto& r : rs) rows += r.n;
  const size_t qrow = t.dtype == SNL_Q8_0 ? t.cols : t.cols / 2, srow = t.cols / 32;
  uint8_t* q = nullptr;
  float* sc = nullptr;
  SNL_TRY(snl::dalloc(e, &q, rows * qrow));
  SNL_TRY(snl::dalloc(e, &sc, rows * srow));
  size_t o = 0;
  for (const auto& r : rs) {
    SNL_CUDA_TRY(cudaMemcpyAsync(q + o * qrow, (const uint8_t*)t.q + r.a * qrow, r.n * qrow, cudaMemcpyDeviceToDevice,
                                 e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(sc + o * srow, (const float*)t.s + r.a * srow, r.n * srow * sizeof(float),
                                 cudaMemcpyDeviceToDevice, e->stream));
    o += r.n;
  }
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  dfree(e, t.q);
  dfree(e, t.s);
  t.q = q;
  t.s = sc;
  t.rows = rows;
  return SNL_OK;
}

// Keeps columns [c0, c0 + cn) (multiples of 32) of a quantized matrix.
int shard_cols(snl_engine* e, snl::QT& t, size_t c0, size_t cn) {
  const bool q8 = t.dtype == SNL_Q8_0;
  const size_t qrow = q8 ? t.cols : t.cols / 2, qw = q8 ? cn : cn / 2, qo = q8 ? c0 : c0 / 2;
  uint8_t* q = nullptr;
  float* sc = nullptr;
  SNL_TRY(snl::dalloc(e, &q, t.rows * qw));
  SNL_TRY(snl::dalloc(e, &sc, t.rows * (cn / 32)));
  SNL_CUDA_TRY(cudaMemcpy2DAsync(q, qw, (const uint8_t*)t.q + qo, qrow, qw, t.rows, cudaMemcpyDeviceToDevice, e->stream));
  SNL_CUDA_TRY(cudaMemcpy2DAsync(sc, cn / 32 * sizeof(float), (const float*)t.s + c0 / 32, t.cols / 32 * sizeof(float),
                                 cn / 32 * sizeof(float), t.rows, cudaMemcpyDeviceToDevice, e->stream));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  dfree(e, t.q);
  dfree(e, t.s);
  t.q = q;
  t.s = sc;
  t.cols = cn;
  return SNL_OK;
}

// Keeps the element ranges `rs` of an f32 vector.
int shard_f32(snl_engine* e, snl::FT& f, const std::vector<RowRange>& rs) {
  size_t n = 0;
  for (const auto& r : rs) n += r.n;
  float* p = nullptr;
  SNL_TRY(snl::dalloc(e, &p, n));
  size_t o = 0;
  for (const auto& r : rs) {
    SNL_CUDA_TRY(cudaMemcpyAsync(p + o, f.p + r.a, r.n * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
    o += r.n;
  }
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  dfree(e, f.p);
  f.p = p;
  f.n = n;
  return SNL_OK;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// The shard plan of one tensor for rank r of N: kind SNL_TP_ROWS keeps the listed row
// ranges of a matrix (in order), SNL_TP_COLS one column range, SNL_TP_ELEMS the listed
// element ranges of an f32 vector, SNL_TP_FULL the whole tensor.
int tp_plan(const snl_model_config& c, size_t r, size_t N, const std::string& nm, int* kind,
            std::vector<RowRange>* rs) {
  rs->clear();
  *kind = SNL_TP_FULL;
  if (N <= 1 || nm == "embed" || nm.compare(0, 4, "mtp.") == 0) return SNL_OK;
  const size_t HD = c.head_dim;
  const size_t nq = c.n_heads / N, q0 = r * nq;  // the query heads whose o_proj columns this rank holds
  const size_t nkv = N <= c.n_kv_heads ? c.n_kv_heads / N : 1;
  const size_t G = c.n_heads / c.n_kv_heads;
  const size_t kv0 = N <= c.n_kv_heads ? r * nkv : q0 / G;
  // With more ranks than KV heads, a rank computes the attention of its whole GQA group
  // (G query heads over one KV head) and keeps its nq heads' share for o_proj.
  const size_t aq = N <= c.n_kv_heads ? nq : G, aq0 = N <= c.n_kv_heads ? q0 : kv0 * G;
  const size_t q_dim = (size_t)c.n_heads * HD, kv_dim = (size_t)c.n_kv_heads * HD;
  const size_t nk = c.lin_k_heads / N, nv = c.lin_v_heads / N, k0 = r * nk, v0 = r * nv;
  const size_t key_dim = (size_t)c.lin_k_heads * c.lin_k_dim, cdim = snl_synth::conv_dim(c);
  const size_t DKh = c.lin_k_dim, DVh = c.lin_v_dim;
  const size_t Il = c.intermediate / N, I = c.intermediate, vl = c.vocab / N;
  if (ends_with(nm, ".qkv")) {
    *kind = SNL_TP_ROWS;
    *rs = {{aq0 * 2 * HD, aq * 2 * HD}, {2 * q_dim + kv0 * HD, nkv * HD}, {2 * q_dim + kv_dim + kv0 * HD, nkv * HD}};
  } else if (ends_with(nm, ".in_proj")) {
    const size_t zb = cdim, bb = cdim + (size_t)c.lin_v_heads * DVh, ab = bb + c.lin_v_heads;
    *kind = SNL_TP_ROWS;
    *rs = {{k0 * DKh, nk * DKh}, {key_dim + k0 * DKh, nk * DKh}, {2 * key_dim + v0 * DVh, nv * DVh},
           {zb + v0 * DVh, nv * DVh}, {bb + v0, nv}, {ab + v0, nv}};
  } else if (ends_with(nm, ".gate_up")) {
    *kind = SNL_TP_ROWS;
    *rs = {{r * Il, Il}, {I + r * Il, Il}};
  } else if (nm == "lm_head") {
    *kind = SNL_TP_ROWS;
    *rs = {{r * vl, vl}};
  } else if (ends_with(nm, ".o_proj")) {
    *kind = SNL_TP_COLS;
    *rs = {{q0 * HD, nq * HD}};
  } else if (ends_with(nm, ".out_proj")) {
    *kind = SNL_TP_COLS;
    *rs = {{v0 * DVh, nv * DVh}};
  } else if (ends_with(nm, ".down")) {
    *kind = SNL_TP_COLS;
    *rs = {{r * Il, Il}};
  } else if (ends_with(nm, ".lin")) {
    // conv w [conv_dim][4] | A_log [n_v] | dt_bias [n_v] | norm w [128] (linear.wgsl bindings)
    const size_t tail = cdim * 4;
    *kind = SNL_TP_ELEMS;
    *rs = {{k0 * DKh * 4, nk * DKh * 4},        {(key_dim + k0 * DKh) * 4, nk * DKh * 4},
           {(2 * key_dim + v0 * DVh) * 4, nv * DVh * 4}, {tail + v0, nv},
           {tail + c.lin_v_heads + v0, nv},     {tail + 2 * (size_t)c.lin_v_heads, DVh}};
  }
  return SNL_OK;
}

// Replaces every tensor by this rank's shard (the global shapes were checked before).
int shard_weights(snl_engine* e) {
  const size_t N = (size_t)e->tp.size, r = (size_t)e->tp.rank;
  std::vector<RowRange> rs;
  int kind = 0;
  for (auto& kv : e->qw) {
    SNL_TRY(tp_plan(e->cfg, r, N, kv.first, &kind, &rs));
    if (kind == SNL_TP_ROWS) SNL_TRY(shard_rows(e, kv.second, rs));
    else if (kind == SNL_TP_COLS) SNL_TRY(shard_cols(e, kv.second, rs[0].a, rs[0].n));
  }
  for (auto& kv : e->fv) {
    SNL_TRY(tp_plan(e->cfg, r, N, kv.first, &kind, &rs));
    if (kind == SNL_TP_ELEMS) SNL_TRY(shard_f32(e, kv.second, rs));
  }
  return SNL_OK;
}

}  // namespace

extern "C" int snl_engine_create_tp(const snl_model_config* cfg, size_t ctx, int device, uint32_t flags, int tp_rank,
                                    int tp_size, snl_engine** out) {
  if (!out) return fail(SNL_E_INVALID, "snl_engine_create_tp: null out");
  *out = nullptr;
  if (tp_size < 1 || tp_size > snl::kTpMax || (tp_size & (tp_size - 1)) || tp_rank < 0 || tp_rank >= tp_size)
    return fail(SNL_E_INVALID, "snl_engine_create_tp: tp_size must be 1, 2, 4 or 8 and 0 <= tp_rank < tp_size");
  if (int rc = snl_config_validate(cfg)) return rc;
  const uint32_t N = (uint32_t)tp_size;
  if (cfg->n_heads % N || cfg->lin_k_heads % N || cfg->lin_v_heads % N || cfg->intermediate % (32 * N) ||
      cfg->vocab % N || (N > cfg->n_kv_heads && N % cfg->n_kv_heads) ||
      (N > cfg->n_kv_heads && (cfg->n_heads / cfg->n_kv_heads) % (cfg->n_heads / N)))
    return fail(SNL_E_UNSUPPORTED, "tensor parallel: heads, intermediate and vocab must divide by tp_size");
  snl_engine* e = nullptr;
  SNL_TRY(snl_engine_create(cfg, ctx, device, flags, &e));
  if (tp_size == 1) {
    *out = e;
    return SNL_OK;
  }
  DeviceGuard dg(device);
  e->tp.rank = tp_rank;
  e->tp.size = tp_size;
  e->lc.n_heads = N <= cfg->n_kv_heads ? cfg->n_heads / N : cfg->n_heads / cfg->n_kv_heads;
  e->lc.n_kv_heads = N <= cfg->n_kv_heads ? cfg->n_kv_heads / N : 1;
  e->lc.lin_k_heads = cfg->lin_k_heads / N;
  e->lc.lin_v_heads = cfg->lin_v_heads / N;
  e->lc.intermediate = cfg->intermediate / N;
  e->vocab_l = cfg->vocab / N;
  // The exchange region: flags, GEMV partials, bulk partials, argmax keys, LM-head shard.
  const size_t h = cfg->hidden;
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  TpHost& t = e->tp;
  t.off_flags = 0;
  t.off_bparts = al(t.off_flags + (size_t)snl::kTpSlots * snl::kTpMax * 8);
  t.off_ll = al(t.off_bparts + 2 * MAX_M * h * sizeof(float));
  t.off_llkeys = al(t.off_ll + (size_t)2 * snl::kTpMax * 4 * h * 8);
  static_assert(LOGIT_ROWS <= snl::kTpKeyRows, "argmax key slots per set");
  t.off_logits = al(t.off_llkeys + (size_t)snl::kTpKeySets * snl::kTpKeyRows * snl::kTpMax * 2 * 8);
  t.region_bytes = al(t.off_logits + LOGIT_ROWS * (size_t)e->vocab_l * sizeof(float));
  cudaError_t ce = cudaMalloc(&t.region, t.region_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(t.region, 0, t.region_bytes);
  if (ce != cudaSuccess) {
    snl_engine_destroy(e);
    return cuda_fail(ce, "tensor parallel: exchange region");
  }
  e->bytes += t.region_bytes;
  t.peer_base[tp_rank] = t.region;
  *out = e;
  return SNL_OK;
}

extern "C" int snl_tp_plan(const snl_model_config* cfg, int tp_rank, int tp_size, const char* name, int* kind,
                           size_t* ranges, size_t cap, size_t* n_ranges) {
  if (!cfg || !name || !kind || !n_ranges) return fail(SNL_E_INVALID, "snl_tp_plan: null argument");
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail(SNL_E_INVALID, "snl_tp_plan: bad rank");
  std::vector<RowRange> rs;
  SNL_TRY(tp_plan(*cfg, (size_t)tp_rank, (size_t)tp_size, name, kind, &rs));
  *n_ranges = rs.size();
  if (rs.size() > cap || (!ranges && !rs.empty())) return fail(SNL_E_RANGE, "snl_tp_plan: ranges buffer too small");
  for (size_t i = 0; i < rs.size(); i++) {
    ranges[2 * i] = rs[i].a;
    ranges[2 * i + 1] = rs[i].n;
  }
  return SNL_OK;
}

extern "C" int snl_engine_tp_handle(snl_engine* e, void* handle_out) {
  if (!e || !handle_out) return fail(SNL_E_INVALID, "snl_engine_tp_handle: null argument");
  if (e->tp.size < 2) return fail(SNL_E_STATE, "snl_engine_tp_handle: not a tensor parallel engine");
  DeviceGuard dg(e->device);
  cudaIpcMemHandle_t hd;
  SNL_CUDA_TRY(cudaIpcGetMemHandle(&hd, e->tp.region));
  memcpy(handle_out, &hd, sizeof(hd));
  return SNL_OK;
}

extern "C" int snl_engine_tp_connect(snl_engine* e, const void* handles) {
  if (!e || !handles) return fail(SNL_E_INVALID, "snl_engine_tp_connect: null argument");
  if (e->tp.size < 2) return fail(SNL_E_STATE, "snl_engine_tp_connect: not a tensor parallel engine");
  if (e->tp.connected) return SNL_OK;
  DeviceGuard dg(e->device);
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (int q = 0; q < e->tp.size; q++) {
    if (q == e->tp.rank) continue;
    cudaIpcMemHandle_t hd;
    memcpy(&hd, hs + (size_t)q * SNL_TP_HANDLE_BYTES, sizeof(hd));
    void* p = nullptr;
    cudaError_t ce = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) return cuda_fail(ce, "tensor parallel: cudaIpcOpenMemHandle");
    e->tp.peer_base[q] = p;
  }
  e->tp.connected = true;
  return SNL_OK;
}

static int store_q(snl_engine* e, const std::string& name, int dtype, size_t rows, size_t cols) {
  snl::QT t;
  t.dtype = dtype;
  t.rows = rows;
  t.cols = cols;
  const size_t n = rows * cols;
  const size_t qbytes = dtype == SNL_Q8_0 ? n : n / 2;
  void* q = nullptr;
  float* s = nullptr;
  SNL_TRY(dalloc(e, (uint8_t**)&q, qbytes));
  SNL_TRY(dalloc(e, &s, n / 32));
  t.q = q;
  t.s = s;
  e->qw[name] = t;
  return SNL_OK;
}

extern "C" int snl_engine_set_tensor(snl_engine* e, const char* name, int dtype, size_t rows, size_t cols, const void* q,
                                     const void* s) {
  if (!e || !name || !q) return fail(SNL_E_INVALID, "snl_engine_set_tensor: null argument");
  if (e->finalized) return fail(SNL_E_STATE, "snl_engine_set_tensor: engine already finalized");
  DeviceGuard dg(e->device);
  const std::string nm(name);
  if (dtype == SNL_F32) {
    snl::FT f;
    f.n = rows * cols;
    SNL_TRY(dalloc(e, &f.p, f.n));
    SNL_CUDA_TRY(cudaMemcpyAsync(f.p, q, f.n * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    e->fv[nm] = f;
  } else if (dtype == SNL_Q8_0 || dtype == SNL_Q4_0) {
    if (!s) return fail(SNL_E_INVALID, "snl_engine_set_tensor: quantized tensor without scales");
    if (cols % 32) return fail(SNL_E_INVALID, std::string(name) + ": columns not divisible by 32");
    SNL_TRY(store_q(e, nm, dtype, rows, cols));
    const snl::QT& t = e->qw[nm];
    const size_t n = rows * cols;
    SNL_CUDA_TRY(cudaMemcpyAsync(t.q, q, dtype == SNL_Q8_0 ? n : n / 2, cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(t.s, s, n / 32 * sizeof(float), cudaMemcpyHostToDevice, e->stream));
  } else {
    return fail(SNL_E_INVALID, "snl_engine_set_tensor: unknown dtype");
  }
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));  // host buffers may go away after return
  return SNL_OK;
}

extern "C" int snl_engine_fill_synthetic(snl_engine* e, uint64_t seed, int quant) {
  if (!e) return fail(SNL_E_INVALID, "null engine");
  if (e->finalized) return fail(SNL_E_STATE, "snl_engine_fill_synthetic: engine already finalized");
  if (quant != SNL_Q8_0 && quant != SNL_Q4_0) return fail(SNL_E_INVALID, "snl_engine_fill_synthetic: quant");
  DeviceGuard dg(e->device);
  int rc = SNL_OK;
  snl_synth::for_each_tensor(
      e->cfg, e->has_mtp, quant,
      [&](const std::string& name, int dtype, size_t rows, size_t cols) {
        if (rc) return;
        rc = store_q(e, name, dtype, rows, cols);
        if (rc) return;
        const snl::QT& t = e->qw[name];
        rc = launch_gen_quant(seed, name.c_str(), dtype, rows, cols, t.q, (float*)t.s, e->stream);
      },
      [&](const std::string& name, const snl_synth::Seg* segs, int nseg) {
        if (rc) return;
        snl::FT f;
        for (int i = 0; i < nseg; i++) f.n += segs[i].n;
        rc = dalloc(e, &f.p, f.n);
        if (rc) return;
        size_t off = 0;
        for (int i = 0; i < nseg && !rc; i++) {
          rc = launch_gen_f32(seed, name.c_str(), segs[i].sub, segs[i].n, segs[i].mult, segs[i].offset, f.p + off,
                              e->stream);
          off += segs[i].n;
        }
        e->fv[name] = f;
      });
  if (rc) return rc;
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  return SNL_OK;
}

extern "C" int snl_engine_finalize(snl_engine* e) {
  if (!e) return fail(SNL_E_INVALID, "null engine");
  if (e->finalized) return SNL_OK;
  DeviceGuard dg(e->device);
  const auto& c = e->lc;  // this rank's shard of the model
  const size_t h = c.hidden, I = c.intermediate;
  // Every tensor the op graph binds must be present (WeightFile::info, weights.rs:108-113).
  std::string missing;
  snl_synth::for_each_tensor(
      e->cfg, e->has_mtp, SNL_Q8_0,
      [&](const std::string& name, int, size_t rows, size_t cols) {
        auto it = e->qw.find(name);
        if (it == e->qw.end()) {
          if (missing.empty()) missing = name;
        } else if (it->second.rows != rows || it->second.cols != cols) {
          if (missing.empty()) missing = name + " (shape)";
        }
      },
      [&](const std::string& name, const snl_synth::Seg* segs, int nseg) {
        size_t n = 0;
        for (int i = 0; i < nseg; i++) n += segs[i].n;
        auto it = e->fv.find(name);
        if (it == e->fv.end()) {
          if (missing.empty()) missing = name;
        } else if (it->second.n != n) {
          if (missing.empty()) missing = name + " (shape)";
        }
      });
  if (!missing.empty()) return fail(SNL_E_INVALID, "weight file is missing tensor `" + missing + "`");
  if (e->tp.size > 1) {
    if (!e->tp.connected) return fail(SNL_E_STATE, "tensor parallel engine: snl_engine_tp_connect first");
    SNL_TRY(shard_weights(e));
  }
  // Tile-layout copies for the decode GEMV (embed is only gathered, not multiplied). A
  // matrix's block scales are kept as fp16 when every one is an fp16 number, else as f32.
  if (!getenv("SNL_NO_TILES")) {
    SNL_TRY(dalloc(e, &e->tile_flag, 1));
    for (auto& kv : e->qw) {
      if (kv.first == "embed") continue;
      snl::QT& t = kv.second;
      size_t tb = 0, sf = 0;
      tile_sizes(t.dtype, (uint32_t)t.rows, (uint32_t)t.cols, &tb, &sf);
      bool f16 = false;
      SNL_TRY(scales_fp16_exact((const float*)t.s, (uint64_t)t.rows * (t.cols / 32), e->tile_flag, &f16, e->stream));
      uint8_t* tiles = nullptr;
      void* ts = nullptr;
      SNL_TRY(dalloc(e, &tiles, tb));
      if (f16) {
        __half* p = nullptr;
        SNL_TRY(dalloc(e, &p, sf));
        ts = p;
      } else {
        float* p = nullptr;
        SNL_TRY(dalloc(e, &p, sf));
        ts = p;
      }
      // A layer's [gate; up] matrix pairs gate row i with up row i for the SwiGLU epilogue.
      const std::string& nm = kv.first;
      const bool pair = nm.size() > 8 && nm[0] == 'l' && nm.compare(nm.size() - 8, 8, ".gate_up") == 0 &&
                        t.rows % 16 == 0;
      t.pair_half = pair ? (uint32_t)(t.rows / 2) : 0;
      SNL_TRY(launch_repack_tiles(t.dtype, (uint32_t)t.rows, (uint32_t)t.cols, t.q, (const float*)t.s, tiles, ts,
                                  f16 ? 1 : 0, e->stream, t.pair_half));
      t.tiles = tiles;
      t.tscales = ts;
      t.tscale_f16 = f16 ? 1 : 0;
      (f16 ? e->tiles_f16 : e->tiles_f32)++;
    }
    e->tiles_on = true;
  }
  // The MTP layer runs unsharded on every rank: with it, the step buffers also fit the
  // whole model's attention and FFN (mc == c without tensor parallelism).
  const snl_model_config& mc = e->has_mtp ? e->cfg : c;
  const size_t proj_w = std::max({2 * I, snl_synth::lin_proj_rows(c), snl_synth::attn_proj_rows(c),
                                  2 * (size_t)mc.intermediate, snl_synth::attn_proj_rows(mc)});
  const size_t act_w = std::max({I, snl_synth::conv_dim(c), (size_t)mc.intermediate});
  const size_t attn_w = std::max({snl_synth::q_dim(c), snl_synth::lin_value_dim(c), snl_synth::q_dim(mc)});
  SNL_TRY(dalloc(e, &e->x, MAX_M * 2 * h));
  SNL_TRY(dalloc(e, &e->xn, MAX_M * h));
  SNL_TRY(dalloc(e, &e->proj, MAX_M * proj_w));
  SNL_TRY(dalloc(e, &e->act, MAX_M * act_w));
  SNL_TRY(dalloc(e, &e->attn_out, MAX_M * attn_w));
  SNL_TRY(dalloc(e, &e->branch, MAX_M * h));
  SNL_TRY(dalloc(e, &e->qbuf, MAX_M * std::max(snl_synth::q_dim(c), snl_synth::q_dim(mc))));
  SNL_TRY(dalloc(e, &e->coef, MAX_M * 8));
  const size_t heads_w = std::max(c.n_heads, mc.n_heads);
  SNL_TRY(dalloc(e, &e->partial, std::max<size_t>(heads_w * MAX_M, heads_w * 4 * MAX_PARTS) * (c.head_dim + 2)));
  SNL_TRY(dalloc(e, &e->rpos, MAX_M * 4));
  SNL_TRY(dalloc(e, &e->tokens, MAX_M));
  SNL_TRY(dalloc(e, &e->logits, LOGIT_ROWS * (size_t)c.vocab));
  SNL_TRY(dalloc(e, &e->hid, (MAX_M + 1) * h));
  SNL_TRY(dalloc(e, &e->hlast, h));
  SNL_TRY(dalloc(e, &e->mhc_raw, MAX_M * 16 * 9));
  SNL_TRY(dalloc(e, &e->amax, LOGIT_ROWS));
  SNL_TRY(dalloc(e, &e->amax_part, LOGIT_ROWS * 128));
  e->pstride = (uint32_t)((std::max({h, I, snl_synth::q_dim(c), snl_synth::lin_value_dim(c),
                                      (size_t)mc.intermediate, snl_synth::q_dim(mc)}) + 7) / 8 * 8);
  SNL_TRY(dalloc(e, &e->xpl, (size_t)8 * e->pstride));
  SNL_TRY(dalloc(e, &e->xpl_act, (size_t)8 * e->pstride));
  SNL_TRY(dalloc(e, &e->xpl_norm, (size_t)8 * e->pstride));
  if (getenv("SNL_NO_FUSED_NORM")) e->use_fused_norm = false;
  SNL_TRY(dalloc(e, &e->rpart, (size_t)4 * ((h + 15) / 16) * kRpStride));
  SNL_TRY(dalloc(e, &e->dn_scratch, conv_delta_chunked_scratch(lin_p(e), (uint32_t)MAX_M)));
  if (getenv("SNL_NO_TC")) e->use_tc = false;
  SNL_TRY(dalloc(e, &e->step_d, 1));
  SNL_TRY(dalloc(e, &e->mstep_d, 1));
  for (size_t l : e->plan) (c.full_attention[l] ? e->n_full : e->n_lin)++;
  e->state_elems = (size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim;
  e->conv_elems = (3 * snl_synth::conv_dim(c) + 63) / 64 * 64;  // 256-byte aligned slots (engine.rs:284)
  SNL_TRY(dalloc(e, &e->lin_state, e->state_elems * std::max<size_t>(e->n_lin, 1)));
  SNL_TRY(dalloc(e, &e->conv_state, e->conv_elems * std::max<size_t>(e->n_lin, 1)));
  SNL_TRY(dalloc(e, &e->lin_ckpt, e->state_elems * std::max<size_t>(e->n_lin, 1)));
  SNL_TRY(dalloc(e, &e->conv_ckpt, e->conv_elems * std::max<size_t>(e->n_lin, 1)));
  const size_t kv_words = e->ctx * snl_synth::kv_dim(c) / 2;
  e->kc.resize(e->n_full);
  e->vc.resize(e->n_full);
  for (size_t i = 0; i < e->n_full; i++) {
    SNL_TRY(dalloc(e, &e->kc[i], kv_words));
    SNL_TRY(dalloc(e, &e->vc[i], kv_words));
  }
  e->snap_lin.resize(SNAPSHOTS);
  e->snap_conv.resize(SNAPSHOTS);
  e->snap_h.resize(SNAPSHOTS);
  for (size_t i = 0; i < SNAPSHOTS; i++) {
    SNL_TRY(dalloc(e, &e->snap_lin[i], e->state_elems * std::max<size_t>(e->n_lin, 1)));
    SNL_TRY(dalloc(e, &e->snap_conv[i], e->conv_elems * std::max<size_t>(e->n_lin, 1)));
    SNL_TRY(dalloc(e, &e->snap_h[i], h));
  }
  if (e->has_mtp) {
    SNL_TRY(dalloc(e, &e->mx, MAX_M * 2 * h));
    SNL_TRY(dalloc(e, &e->hn, MAX_M * h));
    SNL_TRY(dalloc(e, &e->m_logits, (size_t)c.vocab));
    const size_t m_kv_words = e->ctx * snl_synth::kv_dim(mc) / 2;  // the MTP layer's cache is unsharded
    SNL_TRY(dalloc(e, &e->m_kc, m_kv_words));
    SNL_TRY(dalloc(e, &e->m_vc, m_kv_words));
  }
  SNL_CUDA_TRY(cudaMallocHost(&e->h_tokens, MAX_M * sizeof(uint32_t)));
  SNL_CUDA_TRY(cudaMallocHost(&e->h_rpos, MAX_M * 4 * sizeof(uint32_t)));
  SNL_CUDA_TRY(cudaMallocHost(&e->h_step, sizeof(snl_step_u)));
  SNL_CUDA_TRY(cudaMallocHost(&e->h_logits, LOGIT_ROWS * (size_t)c.vocab * sizeof(float)));
  SNL_CUDA_TRY(cudaMallocHost(&e->h_amax, LOGIT_ROWS * sizeof(uint32_t)));
  SNL_CUDA_TRY(cudaMallocHost(&e->h_err, sizeof(int)));
  *e->h_err = 0;
  SNL_TRY(dalloc(e, &e->step_ctr, 1));
  e->tp_sites = (uint32_t)(2 * e->plan.size() + 2);
  e->head_out = e->logits;
  if (e->tp.size > 1) {
    SNL_TRY(dalloc(e, &e->logits_full, LOGIT_ROWS * (size_t)e->cfg.vocab));
    int* err = nullptr;
    SNL_TRY(device_error_word(&err));
    snl::TpComm& cm = e->tp.comm;
    cm.rank = e->tp.rank;
    cm.size = e->tp.size;
    for (int q = 0; q < e->tp.size; q++) {
      uint8_t* b = static_cast<uint8_t*>(e->tp.peer_base[q]);
      cm.flags[q] = reinterpret_cast<uint64_t*>(b + e->tp.off_flags);
      cm.bparts[q] = reinterpret_cast<float*>(b + e->tp.off_bparts);
      cm.ll[q] = reinterpret_cast<unsigned long long*>(b + e->tp.off_ll);
      cm.llkeys[q] = reinterpret_cast<unsigned long long*>(b + e->tp.off_llkeys);
      cm.logits[q] = reinterpret_cast<float*>(b + e->tp.off_logits);
    }
    cm.gp_rows = (uint32_t)h;
    cm.bp_elems = MAX_M * h;
    cm.step = e->step_ctr;
    cm.sites = e->tp_sites;
    cm.err = err;
    if (const char* ms = getenv("SNL_TP_WAIT_MS")) {
      const double v = atof(ms);
      if (v > 0) cm.wait_ns = (unsigned long long)(v * 1e6);
    }
    e->head_out = cm.logits[e->tp.rank];
  }
  // Weight planes for the prefill GEMM (4 bytes per weight: fp16 hi and lo of each value),
  // made last and only when they fit with kPlanesHeadroom to spare; otherwise the GEMM
  // dequantizes the file layout itself (the same values). SNL_NO_WPLANES skips them.
  if (!getenv("SNL_NO_WPLANES") && gemm_tc_enabled()) {
    constexpr size_t kPlanesHeadroom = (size_t)8 << 30;
    size_t need = 0;
    for (auto& kv : e->qw)
      if (kv.first != "embed" && !kv.second.s_f16) need += kv.second.rows * kv.second.cols * 2 * sizeof(__half);
    size_t fr = 0, tot = 0;
    SNL_CUDA_TRY(cudaMemGetInfo(&fr, &tot));
    if (fr > need + kPlanesHeadroom) {
      for (auto& kv : e->qw) {
        if (kv.first == "embed" || kv.second.s_f16) continue;
        snl::QT& t = kv.second;
        __half* pl = nullptr;
        SNL_TRY(dalloc(e, &pl, 2 * t.rows * t.cols));
        SNL_TRY(launch_weight_planes(t.dtype, (uint32_t)t.rows, (uint32_t)t.cols, t.q, (const float*)t.s, pl,
                                     e->stream));
        t.wplanes = pl;
      }
    }
  }
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  e->finalized = true;
  e->pos = 0;
  e->hid_rows = 0;
  return SNL_OK;
}

extern "C" void snl_engine_destroy(snl_engine* e) {
  if (!e) return;
  {
    DeviceGuard dg(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (auto& kv : e->graphs)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    for (void* p : e->allocs) cudaFree(p);
    for (int q = 0; q < e->tp.size; q++)
      if (q != e->tp.rank && e->tp.peer_base[q]) cudaIpcCloseMemHandle(e->tp.peer_base[q]);
    if (e->tp.region) cudaFree(e->tp.region);
    if (e->h_tokens) cudaFreeHost(e->h_tokens);
    if (e->h_rpos) cudaFreeHost(e->h_rpos);
    if (e->h_step) cudaFreeHost(e->h_step);
    if (e->h_logits) cudaFreeHost(e->h_logits);
    if (e->h_amax) cudaFreeHost(e->h_amax);
    if (e->h_err) cudaFreeHost(e->h_err);
    if (e->h_sample_out) cudaFreeHost(e->h_sample_out);
    if (e->sample_scratch) cudaFree(e->sample_scratch);
    if (e->sample_out) cudaFree(e->sample_out);
    if (e->hist_d) cudaFree(e->hist_d);
    if (e->stream) cudaStreamDestroy(e->stream);
  }
  delete e;
}

extern "C" int snl_engine_forward_mm(snl_engine* e, const uint32_t* tokens, size_t n, const uint32_t* pos,
                                     const uint32_t* embed_idx, const float* embeds, size_t n_embeds, size_t logit_rows,
                                     int ckpt, float* logits_out) {
  if (!e) return fail(SNL_E_INVALID, "null engine");
  if (n_embeds && (!embed_idx || !embeds)) return fail(SNL_E_INVALID, "forward: embeds without rows");
  DeviceGuard dg(e->device);
  size_t rows = 0;
  e->last_logit_rows = 0;
  SNL_TRY(forward_impl(e, tokens, n, pos, embed_idx, embeds, n_embeds, logit_rows, ckpt, false, &rows));
  e->last_logit_rows = rows;
  if (rows && logits_out) {
    const size_t nbytes = rows * e->cfg.vocab * sizeof(float);
    const float* src = e->tp.size > 1 ? e->logits_full : e->head_out;
    SNL_CUDA_TRY(cudaMemcpyAsync(e->h_logits, src, nbytes, cudaMemcpyDeviceToHost, e->stream));
    SNL_TRY(queue_error_read(e));
    SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
    SNL_TRY(take_device_error(e));
    memcpy(logits_out, e->h_logits, nbytes);
  } else {
    // Keep the host from running far ahead of the device (engine.rs:933-934).
    SNL_TRY(queue_error_read(e));
    SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
    SNL_TRY(take_device_error(e));
  }
  return SNL_OK;
}

extern "C" int snl_engine_forward_greedy(snl_engine* e, const uint32_t* tokens, size_t n, const uint32_t* pos,
                                         size_t logit_rows, int ckpt, uint32_t* argmax_out) {
  if (!e) return fail(SNL_E_INVALID, "null engine");
  if (logit_rows == 0 || !argmax_out) return fail(SNL_E_INVALID, "forward_greedy: needs logit_rows >= 1 and an output");
  DeviceGuard dg(e->device);
  size_t rows = 0;
  SNL_TRY(forward_impl(e, tokens, n, pos, nullptr, nullptr, 0, logit_rows, ckpt, true, &rows));
  SNL_CUDA_TRY(cudaMemcpyAsync(e->h_amax, e->amax, rows * sizeof(uint32_t), cudaMemcpyDeviceToHost, e->stream));
  SNL_TRY(queue_error_read(e));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  SNL_TRY(take_device_error(e));
  memcpy(argmax_out, e->h_amax, rows * sizeof(uint32_t));
  return SNL_OK;
}

// Sampler::sample / verify (sampler.rs:54-167) on row `row` of the last forward's logits,
// on the device: only the token and two flags come back, not the 1 MB row.
extern "C" int snl_engine_sample(snl_engine* e, size_t row, const snl_sample_p* p, const uint32_t* hist_tok,
                                 const uint32_t* hist_cnt, size_t n_hist, const float* u, int64_t draft, uint32_t* out3) {
  if (!e || !p || !u || !out3) return fail(SNL_E_INVALID, "sample: null argument");
  if (n_hist && (!hist_tok || !hist_cnt)) return fail(SNL_E_INVALID, "sample: history arrays missing");
  if (row >= e->last_logit_rows) return fail(SNL_E_STATE, "sample: the last forward kept no logits for that row");
  DeviceGuard dg(e->device);
  if (!e->sample_scratch) {
    SNL_CUDA_TRY(cudaMalloc(&e->sample_scratch, sample_scratch_bytes()));
    SNL_CUDA_TRY(cudaMalloc(&e->sample_out, 4 * sizeof(uint32_t)));
    SNL_CUDA_TRY(cudaMallocHost(&e->h_sample_out, 4 * sizeof(uint32_t)));
  }
  if (n_hist > e->hist_cap) {
    if (e->hist_d) cudaFree(e->hist_d);
    e->hist_d = nullptr;
    e->hist_cap = 0;
    SNL_CUDA_TRY(cudaMalloc(&e->hist_d, 2 * n_hist * sizeof(uint32_t)));
    e->hist_cap = n_hist;
  }
  if (n_hist) {
    SNL_CUDA_TRY(cudaMemcpyAsync(e->hist_d, hist_tok, n_hist * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(e->hist_d + e->hist_cap, hist_cnt, n_hist * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                 e->stream));
  }
  float* src = (e->tp.size > 1 ? e->logits_full : e->head_out) + row * (size_t)e->cfg.vocab;
  SNL_TRY(launch_sample(*p, src, e->cfg.vocab, e->hist_d, e->hist_d + e->hist_cap, (uint32_t)n_hist, u[0], u[1], draft,
                        e->sample_out, e->sample_scratch, e->stream));
  SNL_CUDA_TRY(cudaMemcpyAsync(e->h_sample_out, e->sample_out, 3 * sizeof(uint32_t), cudaMemcpyDeviceToHost, e->stream));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  memcpy(out3, e->h_sample_out, 3 * sizeof(uint32_t));
  return SNL_OK;
}

// mtp (engine.rs:708-774). Under tensor parallelism every rank runs the MTP layer in
// full on its copy of the hidden rows (the layer's weights are not sharded), so the ranks
// need no exchange until the head: that is split by vocabulary like the model's, and the
// draft is the argmax agreed over the ranks' shards. Each call's embedding advances the
// step counter, so the draft's exchange has an epoch of its own.
extern "C" int snl_engine_mtp(snl_engine* e, size_t r0, const uint32_t* tokens, size_t n, const uint32_t* pos, size_t slot0,
                              int draft, uint32_t* draft_out) {
  if (!e) return fail(SNL_E_INVALID, "null engine");
  if (!e->has_mtp) return fail(SNL_E_STATE, "mtp: the model has no MTP head");
  if (n == 0 || !tokens || !pos || r0 + n > e->hid_rows + 1) return fail(SNL_E_RANGE, "mtp: rows out of range");
  if (slot0 + n > e->ctx) return fail(SNL_E_RANGE, "mtp: rows out of range");
  SNL_TRY(check_tokens(e, tokens, n));
  DeviceGuard dg(e->device);
  const size_t h = e->h();
  const auto& c = e->cfg;
  const snl_attn_p ap = attn_p(e, true);
  const bool tp = e->tp.size > 1;
  for (size_t c0 = 0; c0 < n; c0 += MAX_M) {
    const size_t c1 = std::min(c0 + MAX_M, n);
    const uint32_t m = (uint32_t)(c1 - c0);
    snl_step_u sh = {m, (uint32_t)(slot0 + c0), parts_for(m, slot0 + c1, att_parts(e)), 0};
    *e->h_step = sh;
    memcpy(e->h_tokens, tokens + c0, m * sizeof(uint32_t));
    for (size_t i = 0; i < m; i++) {
      for (int k = 0; k < 3; k++) e->h_rpos[i * 4 + k] = pos[(c0 + i) * 3 + k];
      e->h_rpos[i * 4 + 3] = 0;
    }
    SNL_CUDA_TRY(cudaMemcpyAsync(e->mstep_d, e->h_step, sizeof(snl_step_u), cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(e->tokens, e->h_tokens, m * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
    SNL_CUDA_TRY(cudaMemcpyAsync(e->rpos, e->h_rpos, m * 4 * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
    StepRef st = step_dev(e->mstep_d, sh);
    const bool last = c1 == n;
    const QT* emb = find_q(e, "embed");
    SNL_TRY(launch_embed(e->tokens, m, (const int8_t*)emb->q, (const float*)emb->s, (uint32_t)h, c.vocab, e->mx, nullptr,
                         e->stream, tp ? e->step_ctr : nullptr));
    snl_layer_p p0 = layer_p(e, 0, false);
    p0.inter = c.intermediate;  // the MTP FFN is unsharded
    SNL_TRY(launch_branch_norm(st, p0, e->mx, e->coef, find_f(e, "mtp.norm_e"), e->xn, m, e->stream));
    snl_layer_p ph = p0;
    ph.x_stride = (uint32_t)h;
    SNL_TRY(launch_branch_norm(st, ph, e->hid + (r0 + c0) * h, e->coef, find_f(e, "mtp.norm_h"), e->hn, m, e->stream));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.fc_e"), e->xn, h, e->mx, 2 * h, m));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.fc_h"), e->hn, h, e->branch, h, m));
    SNL_TRY(launch_merge(st, p0, e->mx, e->coef, e->branch, m, e->stream));
    SNL_TRY(launch_branch_norm(st, p0, e->mx, e->coef, find_f(e, "mtp.in_ln"), e->xn, m, e->stream));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.qkv"), e->xn, h, e->proj, ap.proj_stride, m));
    SNL_TRY(launch_attn_prep(st, ap, e->proj, e->qbuf, e->m_kc, e->m_vc, find_f(e, "mtp.qk_norm"), e->rpos, m, e->stream));
    SNL_TRY(launch_attend(st, ap, e->proj, e->qbuf, e->m_kc, e->m_vc, e->attn_out, e->partial, m, sh.parts, e->stream));
    if (sh.parts > 1) SNL_TRY(launch_attn_combine(st, ap, e->proj, e->partial, e->attn_out, m, e->stream, sh.parts));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.o_proj"), e->attn_out, snl_synth::q_dim(c), e->branch, h, m));
    SNL_TRY(launch_merge(st, p0, e->mx, e->coef, e->branch, m, e->stream));
    SNL_TRY(launch_branch_norm(st, p0, e->mx, e->coef, find_f(e, "mtp.post_ln"), e->xn, m, e->stream));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.gate_up"), e->xn, h, e->proj, 2 * (size_t)c.intermediate, m));
    SNL_TRY(launch_swiglu(st, p0, e->proj, e->act, m, e->stream));
    SNL_TRY(mat_tile(e, st, *find_q(e, "mtp.down"), e->act, c.intermediate, e->branch, h, m));
    SNL_TRY(launch_merge(st, p0, e->mx, e->coef, e->branch, m, e->stream));
    if (last && draft) {
      snl_layer_p pl = layer_p(e, 0, true);
      SNL_TRY(launch_branch_norm(st, pl, e->mx, e->coef, find_f(e, "mtp.norm"), e->xn, 1, e->stream));
      SNL_TRY(mat_tile(e, st, *find_q(e, "lm_head"), e->xn, h, e->m_logits, e->vocab_l, 1));
      if (tp) {
        const uint32_t key_set = 1 + (uint32_t)(e->mtp_drafts++ & 1);
        SNL_TRY(launch_argmax_tp(e->m_logits, 1, e->vocab_l, e->amax, e->amax_part, e->tp.comm, e->tp_sites - 1,
                                 e->stream, key_set));
      } else {
        SNL_TRY(launch_argmax_with(e->m_logits, 1, c.vocab, e->amax, e->amax_part, e->stream));
      }
    }
    SNL_TRY(queue_error_read(e));
    SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
    SNL_TRY(take_device_error(e));
  }
  if (draft && draft_out) {
    SNL_CUDA_TRY(cudaMemcpy(draft_out, e->amax, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  }
  return SNL_OK;
}

extern "C" int snl_engine_generate(snl_engine* e, uint32_t first_token, size_t n, uint32_t* out_tokens, float* device_ms) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "generate: engine not finalized");
  if (!out_tokens || n == 0) return fail(SNL_E_INVALID, "generate: needs n >= 1 and an output buffer");
  if (e->pos + n > e->ctx)
    return fail(SNL_E_RANGE, "context length exceeded (" + std::to_string(e->pos + n) + " > " + std::to_string(e->ctx) + ")");
  if (first_token >= e->cfg.vocab) return fail(SNL_E_RANGE, "token id " + std::to_string(first_token) + " out of range");
  DeviceGuard dg(e->device);
  // Every step's descriptor and rotary positions go to device memory first, so the
  // timed loop reads only device-resident inputs.
  std::vector<snl_step_u> steps(n);
  std::vector<uint32_t> rp(4 * n);
  for (size_t i = 0; i < n; i++) {
    const size_t p = e->pos + i;
    steps[i] = snl_step_u{1u, (uint32_t)p, parts_for(1, p + 1, att_parts(e)), 0u};
    for (int k = 0; k < 4; k++) rp[4 * i + k] = (uint32_t)p;
  }
  snl_step_u* steps_d = nullptr;
  uint32_t *rp_d = nullptr, *gen_d = nullptr;
  SNL_CUDA_TRY(cudaMalloc(&steps_d, n * sizeof(snl_step_u)));
  SNL_CUDA_TRY(cudaMalloc(&rp_d, 4 * n * sizeof(uint32_t)));
  SNL_CUDA_TRY(cudaMalloc(&gen_d, n * sizeof(uint32_t)));
  int rc = SNL_OK;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  do {
    cudaError_t ce;
    if ((ce = cudaMemcpy(steps_d, steps.data(), n * sizeof(snl_step_u), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (ce = cudaMemcpy(rp_d, rp.data(), 4 * n * sizeof(uint32_t), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (ce = cudaMemcpy(e->tokens, &first_token, sizeof(uint32_t), cudaMemcpyHostToDevice)) != cudaSuccess) {
      rc = cuda_fail(ce, "generate: staging");
      break;
    }
    cudaEventCreate(&t0);
    cudaEventCreate(&t1);
    cudaEventRecord(t0, e->stream);
    for (size_t i = 0; i < n && !rc; i++) {
      if ((ce = cudaMemcpyAsync(e->step_d, steps_d + i, sizeof(snl_step_u), cudaMemcpyDeviceToDevice, e->stream)) ||
          (ce = cudaMemcpyAsync(e->rpos, rp_d + 4 * i, 4 * sizeof(uint32_t), cudaMemcpyDeviceToDevice, e->stream))) {
        rc = cuda_fail(ce, "generate: step copy");
        break;
      }
      rc = run_step(e, steps[i], 1, 1, true);
      if (rc) break;
      if ((ce = cudaMemcpyAsync(e->tokens, e->amax, sizeof(uint32_t), cudaMemcpyDeviceToDevice, e->stream)) ||
          (ce = cudaMemcpyAsync(gen_d + i, e->amax, sizeof(uint32_t), cudaMemcpyDeviceToDevice, e->stream))) {
        rc = cuda_fail(ce, "generate: token copy");
        break;
      }
      e->pos += 1;
      e->hid_rows = 1;
    }
    cudaEventRecord(t1, e->stream);
    if (!rc) rc = queue_error_read(e);
    if ((ce = cudaStreamSynchronize(e->stream)) != cudaSuccess) {
      rc = cuda_fail(ce, "generate");
      break;
    }
    if (!rc) rc = take_device_error(e);
    if (!rc && device_ms) cudaEventElapsedTime(device_ms, t0, t1);
    if (!rc && (ce = cudaMemcpy(out_tokens, gen_d, n * sizeof(uint32_t), cudaMemcpyDeviceToHost)) != cudaSuccess)
      rc = cuda_fail(ce, "generate: read-back");
  } while (0);
  if (t0) cudaEventDestroy(t0);
  if (t1) cudaEventDestroy(t1);
  cudaFree(steps_d);
  cudaFree(rp_d);
  cudaFree(gen_d);
  return rc;
}

extern "C" int snl_engine_profile(snl_engine* e, uint32_t token, snl_op_stat* out, size_t cap, size_t* n_out) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "profile: engine not finalized");
  if (e->pos + 1 > e->ctx) return fail(SNL_E_RANGE, "context length exceeded");
  if (token >= e->cfg.vocab) return fail(SNL_E_RANGE, "token id " + std::to_string(token) + " out of range");
  DeviceGuard dg(e->device);
  std::vector<snl_engine::ProfRec> recs;
  snl_step_u sh = {1u, (uint32_t)e->pos, parts_for(1, e->pos + 1, att_parts(e)), 0u};
  *e->h_step = sh;
  *e->h_tokens = token;
  for (int k = 0; k < 4; k++) e->h_rpos[k] = (uint32_t)e->pos;
  SNL_CUDA_TRY(cudaMemcpyAsync(e->step_d, e->h_step, sizeof(snl_step_u), cudaMemcpyHostToDevice, e->stream));
  SNL_CUDA_TRY(cudaMemcpyAsync(e->tokens, e->h_tokens, sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
  SNL_CUDA_TRY(cudaMemcpyAsync(e->rpos, e->h_rpos, 4 * sizeof(uint32_t), cudaMemcpyHostToDevice, e->stream));
  e->prof = &recs;
  int rc = device_step(e, step_dev(e->step_d, sh), 1, sh.parts, 1, true);
  e->prof = nullptr;
  cudaError_t ce = cudaStreamSynchronize(e->stream);
  std::map<std::string, snl_op_stat> agg;
  std::vector<std::string> order;
  for (auto& r : recs) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
    auto it = agg.find(r.label);
    if (it == agg.end()) {
      snl_op_stat z;
      memset(&z, 0, sizeof(z));
      snprintf(z.label, sizeof(z.label), "%s", r.label.c_str());
      it = agg.emplace(r.label, z).first;
      order.push_back(r.label);
    }
    it->second.calls += 1;
    it->second.ms += ms;
    it->second.bytes += r.bytes;
  }
  if (rc) return rc;
  if (ce != cudaSuccess) return cuda_fail(ce, "profile");
  e->pos += 1;
  e->hid_rows = 1;
  size_t k = 0;
  for (auto& l : order) {
    if (k >= cap) break;
    if (out) out[k] = agg[l];
    k++;
  }
  if (n_out) *n_out = k;
  return SNL_OK;
}

extern "C" int snl_engine_reset(snl_engine* e) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "reset: engine not finalized");
  DeviceGuard dg(e->device);
  const size_t nl = std::max<size_t>(e->n_lin, 1);
  SNL_CUDA_TRY(cudaMemsetAsync(e->lin_state, 0, e->state_elems * nl * sizeof(float), e->stream));
  SNL_CUDA_TRY(cudaMemsetAsync(e->conv_state, 0, e->conv_elems * nl * sizeof(float), e->stream));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  e->pos = 0;
  e->hid_rows = 0;
  return SNL_OK;
}

static int copy_state(snl_engine* e, float* dl, const float* sl, float* dc, const float* sc, float* dh, const float* sh_) {
  const size_t nl = std::max<size_t>(e->n_lin, 1);
  SNL_CUDA_TRY(cudaMemcpyAsync(dl, sl, e->state_elems * nl * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
  SNL_CUDA_TRY(cudaMemcpyAsync(dc, sc, e->conv_elems * nl * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
  SNL_CUDA_TRY(cudaMemcpyAsync(dh, sh_, e->h() * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  return SNL_OK;
}

extern "C" int snl_engine_snapshot(snl_engine* e, size_t slot) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "snapshot: engine not finalized");
  if (slot >= SNAPSHOTS) return fail(SNL_E_RANGE, "snapshot slot out of range");
  DeviceGuard dg(e->device);
  return copy_state(e, e->snap_lin[slot], e->lin_state, e->snap_conv[slot], e->conv_state, e->snap_h[slot], e->hlast);
}

extern "C" int snl_engine_restore(snl_engine* e, size_t slot, size_t pos) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "restore: engine not finalized");
  if (slot >= SNAPSHOTS) return fail(SNL_E_RANGE, "snapshot slot out of range");
  if (pos > e->ctx) return fail(SNL_E_RANGE, "restore: position beyond the context");
  DeviceGuard dg(e->device);
  SNL_TRY(copy_state(e, e->lin_state, e->snap_lin[slot], e->conv_state, e->snap_conv[slot], e->hlast, e->snap_h[slot]));
  e->pos = pos;
  e->hid_rows = 0;
  return SNL_OK;
}

extern "C" int snl_engine_rollback(snl_engine* e) {
  if (!e || !e->finalized) return fail(SNL_E_STATE, "rollback: engine not finalized");
  if (e->pos == 0) return fail(SNL_E_STATE, "rollback: nothing to undo");
  DeviceGuard dg(e->device);
  SNL_TRY(copy_state(e, e->lin_state, e->lin_ckpt, e->conv_state, e->conv_ckpt, e->hlast, e->hid + e->h()));
  e->pos -= 1;
  e->hid_rows = 1;
  return SNL_OK;
}

extern "C" size_t snl_engine_hid_rows(const snl_engine* e) { return e ? e->hid_rows : 0; }
extern "C" int snl_engine_has_mtp(const snl_engine* e) { return e && e->has_mtp ? 1 : 0; }
extern "C" int snl_engine_tile_scales(const snl_engine* e, uint32_t* fp16_matrices, uint32_t* f32_matrices) {
  if (!e || !fp16_matrices || !f32_matrices) return snl::fail(SNL_E_INVALID, "snl_engine_tile_scales: null argument");
  *fp16_matrices = e->tiles_f16;
  *f32_matrices = e->tiles_f32;
  return SNL_OK;
}
extern "C" size_t snl_engine_pos(const snl_engine* e) { return e ? e->pos : 0; }
extern "C" size_t snl_engine_ctx(const snl_engine* e) { return e ? e->ctx : 0; }
extern "C" size_t snl_engine_device_bytes(const snl_engine* e) { return e ? e->bytes : 0; }

extern "C" int snl_engine_read_hidden(const snl_engine* e, size_t row0, size_t rows, float* out) {
  if (!e || !e->finalized || !out) return fail(SNL_E_INVALID, "read_hidden: bad argument");
  if (row0 + rows > MAX_M + 1) return fail(SNL_E_RANGE, "read_hidden: rows out of range");
  DeviceGuard dg(e->device);
  SNL_CUDA_TRY(cudaStreamSynchronize(e->stream));
  SNL_CUDA_TRY(cudaMemcpy(out, e->hid + row0 * e->h(), rows * e->h() * sizeof(float), cudaMemcpyDeviceToHost));
  return SNL_OK;
}

extern "C" size_t snl_engine_prefill_chunk(const snl_engine* e) { return e ? MAX_M : 0; }

namespace snl {
size_t engine_hidden(const snl_engine* e) { return e ? e->cfg.hidden : 0; }
}  // namespace snl
