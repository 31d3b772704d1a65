// C ABI and host orchestration of the DenseGPA b200 core (see include/gpa_b200.h).
//
// Schedule (level-major, every lag block of the call at once):
//   input -> for each level j: prep, paired inner/outer chunked GDN scans over
//   the whole call (block-boundary states), writes / residuals from the
//   frozen snapshots, counts and logits -> relation scans (all edges, grouped
//   by target) -> dense reader per level -> outer reads -> level mix.
// The backward runs the same schedule in reverse; boundary-state gradients
// coming from the writes and residuals enter the reverse GDN sweeps as
// external terms.  Workspaces are caller-owned; nothing here allocates.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gpa_b200.h"
#include "decode.cuh"
#include "gdn.cuh"
#include "level.cuh"

namespace gpa {

// ---------------------------------------------------------- launch accounting
namespace {
std::atomic<long long> g_launches{0};
std::atomic<bool> g_profiling{false};
std::mutex g_prof_mu;
struct ProfRec {
  const char* name;
  cudaEvent_t a, b;
};
std::vector<ProfRec> g_recs;
size_t g_used = 0;
}  // namespace

Launch::Launch(const char* name, cudaStream_t s) : slot(-1), st(s) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_profiling.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (g_used == g_recs.size()) {
    ProfRec r{name, nullptr, nullptr};
    if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return;
    g_recs.push_back(r);
  }
  slot = (int)g_used++;
  g_recs[slot].name = name;
  cudaEventRecord(g_recs[slot].a, st);
}

Launch::~Launch() {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  cudaEventRecord(g_recs[slot].b, st);
}

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

struct Geo {
  int B, T, H, D, Dv, L, E, C, offset, post, dt, pos_none, U;
  int reader;  // GPA_B200_READER_*
  int moments;     // positional moments
  int64_t pos0;    // absolute position of the call's first token
  int M[kMaxLevels];
  int es[kMaxEdges], ed[kMaxEdges];
  float rs, qs, bm;
  Blocks bl;
  int Mmax;
  int fast;  // tensor-core GDN kernels (bf16 / fp16 inputs, widths multiples of 16)
};

// whether level j reads relation messages (some edge ends at it)
bool has_incoming(const Geo& g, int j) {
  for (int e = 0; e < g.E; ++e)
    if (g.ed[e] == j) return true;
  return false;
}

int make_geo(const GpaDims* d, Geo* g, std::string* why) {
  if (!d) {
    *why = "dims is NULL";
    return GPA_B200_BAD_ARGUMENT;
  }
  g->B = d->batch;
  g->T = d->length;
  g->H = d->heads;
  g->D = d->key_dim;
  g->Dv = d->value_dim;
  g->L = d->levels;
  g->C = d->chunk_size;
  g->offset = d->chunk_offset;
  g->dt = d->input_dtype;
  g->pos_none = d->positional_none;
  g->rs = d->read_scale;
  g->qs = d->query_scale;
  g->bm = d->beta_max;
  g->reader = d->reader_mode;
  g->moments = d->positional_moments != 0;
  g->pos0 = d->position;
  if (g->moments && (d->key_dim % 2 || d->position < 0)) {
    *why = "positional moments need an even key_dim and a non-negative position";
    return GPA_B200_BAD_ARGUMENT;
  }
  if (g->reader < GPA_B200_READER_TANH || g->reader > GPA_B200_READER_MARGINAL) {
    *why = "reader_mode must be GPA_B200_READER_TANH, _PRODUCT or _MARGINAL";
    return GPA_B200_BAD_ARGUMENT;
  }
  if (g->B <= 0 || g->T < 0 || g->H <= 0 || g->D <= 0 || g->Dv <= 0 || g->L <= 0) {
    *why = "dimensions must be positive";
    return GPA_B200_BAD_ARGUMENT;
  }
  if (g->L > kMaxLevels) {
    *why = "at most 8 levels are supported";
    return GPA_B200_UNSUPPORTED;
  }
  if (g->C < 1 || g->C > kMaxChunk) {
    *why = "chunk_size must be in [1, 64] for the b200 backend";
    return GPA_B200_UNSUPPORTED;
  }
  if (g->offset < 0 || g->offset >= g->C) {
    *why = "chunk_offset must be in [0, chunk_size)";
    return GPA_B200_BAD_ARGUMENT;
  }
  if (g->dt < 0 || g->dt > 2) {
    *why = "input_dtype must be F32, BF16 or F16";
    return GPA_B200_BAD_ARGUMENT;
  }
  if (g->D > 128 || g->Dv > 128) {
    *why = "key_dim and value_dim must be <= 128";
    return GPA_B200_UNSUPPORTED;
  }
  g->Mmax = 0;
  for (int j = 0; j < g->L; ++j) {
    g->M[j] = d->slots[j];
    if (g->M[j] <= 0) {
      *why = "slots must be positive";
      return GPA_B200_BAD_ARGUMENT;
    }
    if (g->M[j] > 128) {
      *why = "slot counts must be <= 128";
      return GPA_B200_UNSUPPORTED;
    }
    g->Mmax = g->M[j] > g->Mmax ? g->M[j] : g->Mmax;
  }
  g->E = 0;
  for (int i = 0; i < g->L; ++i)
    for (int j = 0; j < g->L; ++j)
      if (i != j) {
        g->es[g->E] = i;
        g->ed[g->E] = j;
        ++g->E;
      }
  g->U = g->B * g->H;
  g->post = g->C == 1;
  g->fast = g->dt != GPA_B200_F32 && tc_supported(g->D, g->Dv);
  for (int j = 0; j < g->L; ++j) g->fast = g->fast && tc_supported(g->M[j], g->M[j]);
  g->bl = make_blocks(g->T, g->C, g->offset);
  return GPA_B200_OK;
}

// Bump layout over a caller buffer; with base == nullptr it only measures.
struct Bump {
  char* base;
  size_t off = 0;
  explicit Bump(void* b) : base(static_cast<char*>(b)) {}
  float* take(size_t nfloat) {
    off = (off + 255) & ~size_t(255);
    float* p = base ? reinterpret_cast<float*>(base + off) : nullptr;
    off += nfloat * sizeof(float);
    return p;
  }
};

struct Saved {
  float *qf, *qh, *qn;
  float *key[kMaxLevels + 1], *val[kMaxLevels + 1];
  float *nk[kMaxLevels], *kn[kMaxLevels], *slot[kMaxLevels], *ns[kMaxLevels], *sn[kMaxLevels];
  float *raw4[kMaxLevels], *gates[kMaxLevels];
  float *Abnd[kMaxLevels], *WA[kMaxLevels], *Bbnd[kMaxLevels], *WB[kMaxLevels];
  float *raw[kMaxLevels], *write[kMaxLevels], *counts[kMaxLevels], *logits[kMaxLevels];
  float *lh[kMaxLevels], *ln[kMaxLevels], *wh[kMaxLevels], *wn[kMaxLevels], *bsum[kMaxLevels];
  float *r[kMaxLevels], *hp[kMaxLevels], *mlp[kMaxLevels], *route[kMaxLevels];
  float *qoh[kMaxLevels], *qon[kMaxLevels], *y[kMaxLevels];
  float *Rbnd[kMaxEdges], *WR[kMaxEdges], *msg[kMaxEdges];
  float *ge, *be;
  // chunk WY terms of every scan (U = T diag(b) V, Wk = T diag(b e^G) K), kept for the backward
  float *UA[kMaxLevels], *KA[kMaxLevels], *UB[kMaxLevels], *KB[kMaxLevels];
  float *UR[kMaxEdges], *KR[kMaxEdges];
  // T = (I + A)^-1 of every block of every scan (tensor-core path only; the backward forms A
  // again from K and the gates, exactly as the forward did)
  float *TA[kMaxLevels], *TB[kMaxLevels];
  float *TR[kMaxEdges];
  // positional moments: the state at every block start and the end [U, nb+1, D, M], and the
  // moment reads corr [U,T,M] of every level
  float *Pb[kMaxLevels], *corr[kMaxLevels];
  size_t bytes;
};

void layout_saved(const Geo& g, void* base, Saved* s) {
  Bump b(base);
  const size_t UT = (size_t)g.U * g.T, nb1 = (size_t)g.bl.nb + 1;
  s->qf = b.take(UT * g.D);
  s->qh = b.take(UT * g.D);
  s->qn = b.take(UT);
  for (int j = 0; j < g.L; ++j) {
    const size_t M = g.M[j];
    s->key[j] = b.take(UT * g.D);
    s->val[j] = b.take(UT * g.Dv);
    s->nk[j] = b.take(UT * g.D);
    s->kn[j] = b.take(UT);
    s->slot[j] = b.take(UT * M);
    s->ns[j] = b.take(UT * M);
    s->sn[j] = b.take(UT);
    s->raw4[j] = b.take(UT * 4);
    s->gates[j] = b.take(UT * 4);
    s->Abnd[j] = b.take((size_t)g.U * nb1 * g.D * M);
    const size_t wsz = g.fast ? (UT + 1) / 2 : UT;  // W is bf16 on the tensor-core path
    s->WA[j] = b.take(wsz * M);
    s->Bbnd[j] = b.take((size_t)g.U * nb1 * M * g.Dv);
    s->WB[j] = b.take(wsz * g.Dv);
    s->raw[j] = b.take(UT * M);
    s->write[j] = b.take(UT * M);
    s->counts[j] = b.take(UT * M);
    s->logits[j] = b.take(UT * M);
    s->lh[j] = b.take(UT * M);
    s->ln[j] = b.take(UT);
    s->wh[j] = b.take(UT * M);
    s->wn[j] = b.take(UT);
    s->bsum[j] = b.take((size_t)g.U * g.bl.nb * M);
    s->r[j] = b.take(UT * M);
    s->hp[j] = b.take(UT * 2 * M);
    s->mlp[j] = b.take(UT * M);
    s->route[j] = b.take(UT * M);
    s->qoh[j] = b.take(UT * M);
    s->qon[j] = b.take(UT);
    s->y[j] = b.take(UT * g.Dv);
  }
  for (int e = 0; e < g.E; ++e) {
    const size_t Mi = g.M[g.es[e]], Mj = g.M[g.ed[e]];
    s->Rbnd[e] = b.take((size_t)g.U * nb1 * Mi * Mj);
    s->WR[e] = b.take((g.fast ? (UT + 1) / 2 : UT) * Mj);
    s->msg[e] = b.take(UT * Mj);
  }
  s->ge = b.take((size_t)g.E * g.U);
  s->be = b.take((size_t)g.E * g.U);
  for (int j = 0; j < g.L; ++j) {
    s->UA[j] = b.take(UT * g.M[j]);
    s->KA[j] = b.take(UT * g.D);
    s->UB[j] = b.take(UT * g.Dv);
    s->KB[j] = b.take(UT * g.M[j]);
  }
  for (int e = 0; e < g.E; ++e) {
    s->UR[e] = b.take(UT * g.M[g.ed[e]]);
    s->KR[e] = b.take(UT * g.M[g.es[e]]);
  }
  const size_t nAT = g.fast ? (size_t)g.U * g.bl.nb * kMaxChunk * kMaxChunk : 0;
  for (int j = 0; j < g.L; ++j) {
    s->TA[j] = g.fast ? b.take(nAT) : nullptr;
    s->TB[j] = g.fast ? b.take(nAT) : nullptr;
  }
  for (int j = 0; j < g.L; ++j) {
    s->Pb[j] = g.moments ? b.take((size_t)g.U * nb1 * g.D * g.M[j]) : nullptr;
    s->corr[j] = g.moments ? b.take(UT * g.M[j]) : nullptr;
  }
  for (int e = 0; e < g.E; ++e) {
    s->TR[e] = g.fast ? b.take(nAT) : nullptr;
  }
  s->bytes = b.off + 256;
}

// Backward scratch.
struct Scratch {
  float *dout_f, *ow_scale, *dqh, *dq_direct, *dkey, *dval;
  double *scal, *scalE;
  float *dqoh[kMaxLevels], *dqo[kMaxLevels], *droute[kMaxLevels], *dhp[kMaxLevels];
  float *dlogits[kMaxLevels], *dlh[kMaxLevels], *dwh[kMaxLevels], *dwrite[kMaxLevels];
  float *odK[kMaxLevels], *odW[kMaxLevels], *odG[kMaxLevels];
  float* dln[kMaxLevels];  // gradient of |softmax(logits_j)| per row (product reader)
  float *Gend, *dcorr, *dmk;  // positional moments: G at block ends, dcorr, unit-key gradient
  float* dmsg[kMaxEdges];
  float *draw, *dn, *dnsum, *extA, *extB, *dnk, *dslot, *dns, *dgates, *d4;
  float *dfzA, *dfzB;
  // GDN group slots
  float *dWk[kMaxScans], *db[kMaxScans], *dA[kMaxScans];
  float *Dend[kMaxScans], *dK[kMaxScans], *dW[kMaxScans], *dG[kMaxScans];
  size_t bytes;
};

void layout_scratch(const Geo& g, void* base, Scratch* s) {
  Bump b(base);
  const size_t UT = (size_t)g.U * g.T, nb = g.bl.nb, nb1 = nb + 1;
  const size_t Mx = g.Mmax;
  s->dout_f = b.take(UT * g.Dv);
  s->ow_scale = b.take((size_t)g.L * g.U);
  s->dqh = b.take(UT * g.D);
  s->dq_direct = b.take(UT * g.D);
  s->dkey = b.take(UT * g.D);
  s->dval = b.take(UT * g.Dv);
  s->scal = reinterpret_cast<double*>(b.take((size_t)g.U * g.L * kNScal * 2));
  s->scalE = reinterpret_cast<double*>(b.take((size_t)g.U * (g.E ? g.E : 1) * kNEdge * 2));
  for (int j = 0; j < g.L; ++j) {
    const size_t M = g.M[j];
    s->dqoh[j] = b.take(UT * M);
    s->dqo[j] = b.take(UT * M);
    s->droute[j] = b.take(UT * M);
    s->dhp[j] = b.take(UT * 2 * M);
    s->dlogits[j] = b.take(UT * M);
    s->dlh[j] = b.take(UT * M);
    s->dwh[j] = b.take(UT * M);
    s->dwrite[j] = b.take(UT * M);
    s->odK[j] = b.take(UT * M);
    s->odW[j] = b.take(UT * g.Dv);
    s->odG[j] = b.take(UT);
    s->dln[j] = b.take(UT);
  }
  for (int e = 0; e < g.E; ++e) s->dmsg[e] = b.take(UT * g.M[g.ed[e]]);
  s->Gend = g.moments ? b.take((size_t)g.U * g.bl.nb * g.D * Mx) : nullptr;
  s->dcorr = g.moments ? b.take(UT * Mx) : nullptr;
  s->dmk = g.moments ? b.take(UT * g.D) : nullptr;
  s->draw = b.take(UT * Mx);
  s->dn = b.take(UT * Mx);
  s->dnsum = b.take((size_t)g.U * nb * Mx);
  s->extA = b.take((size_t)g.U * nb1 * g.D * Mx);
  s->extB = b.take((size_t)g.U * nb1 * Mx * g.Dv);
  s->dnk = b.take(UT * g.D);
  s->dslot = b.take(UT * Mx);
  s->dns = b.take(UT * Mx);
  s->dgates = b.take(UT * 4);
  s->d4 = b.take(UT * 4);
  s->dfzA = b.take((size_t)g.U * g.D * Mx);
  s->dfzB = b.take((size_t)g.U * Mx * g.Dv);
  const size_t K = g.D > Mx ? g.D : Mx, V = g.Dv > Mx ? g.Dv : Mx;
  const int slots = g.L - 1 > 2 ? g.L - 1 : 2;
  for (int i = 0; i < slots; ++i) {
    s->dWk[i] = b.take(UT * K);
    // per-block dA and db round trips exist only on the SIMT path (the tensor-core backward
    // chunk kernel keeps them in shared memory)
    s->db[i] = g.fast ? nullptr : b.take(UT);
    s->dA[i] = g.fast ? nullptr : b.take((size_t)g.U * nb * kMaxChunk * kMaxChunk);
    s->Dend[i] = b.take((size_t)g.U * nb * K * V);
    s->dK[i] = b.take(UT * K);
    s->dW[i] = b.take(UT * V);
    s->dG[i] = b.take(UT);
  }
  s->bytes = b.off + 256;
}

#define CK(x)                                                                        \
  do {                                                                               \
    cudaError_t e_ = (x);                                                            \
    if (e_ != cudaSuccess)                                                           \
      return fail(GPA_B200_LAUNCH_FAILURE, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// parameter-gradient reduction: tensor-core variant when the widths allow it
cudaError_t head_outer(const Geo& g, int B, int T, int H, const float* X, int P, int xmode,
                       const float* Y, int Q, const float* scale, int64_t scale_stride,
                       float cscale, float* out, cudaStream_t st) {
  if (g.fast && xmode != 2 && P % 16 == 0 && Q % 16 == 0)
    return tc_head_outer(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, st);
  return launch_head_outer(B, T, H, X, P, xmode, Y, Q, scale, scale_stride, cscale, out, st);
}

cudaError_t zero(float* p, size_t n, cudaStream_t st) {
  return n ? cudaMemsetAsync(p, 0, n * sizeof(float), st) : cudaSuccess;
}

ScanDesc blank_scan() {
  ScanDesc d;
  std::memset(&d, 0, sizeof(d));
  return d;
}

int check_params(const Geo& g, const GpaParams* p) {
  if (!p) return fail(GPA_B200_BAD_ARGUMENT, "params is NULL");
  for (int j = 0; j < g.L; ++j)
    if (!p->center[j] || !p->route_weight[j] || !p->query_weight[j] || !p->route_up[j] ||
        !p->route_down[j] || !p->gate_weight[j] || !p->gate_bias[j])
      return fail(GPA_B200_BAD_ARGUMENT, "missing per-level parameter pointer");
  if (!p->residual_raw || !p->count_gain_raw || !p->route_mlp_gain || !p->output_logits ||
      !p->relation_gain)
    return fail(GPA_B200_BAD_ARGUMENT, "missing level scalar parameter pointer");
  if (g.E && (!p->edge_logits || !p->relation_decay_raw || !p->relation_beta_raw))
    return fail(GPA_B200_BAD_ARGUMENT, "missing edge parameter pointer");
  if (g.moments && !p->moment_gain)
    return fail(GPA_B200_BAD_ARGUMENT, "positional moments need moment_gain");
  return GPA_B200_OK;
}

int check_state(const Geo& g, const GpaStateRef* s, bool need_frozen, const char* what) {
  if (!s) return fail(GPA_B200_BAD_ARGUMENT, std::string(what) + " is NULL");
  for (int j = 0; j < g.L; ++j) {
    if (!s->inner[j] || !s->outer[j] || !s->count[j])
      return fail(GPA_B200_BAD_ARGUMENT, std::string(what) + ": missing level tensor");
    if (need_frozen && (!s->frozen_inner[j] || !s->frozen_outer[j]))
      return fail(GPA_B200_BAD_ARGUMENT, std::string(what) + ": missing frozen snapshot");
    if (g.moments && !s->moment[j])
      return fail(GPA_B200_BAD_ARGUMENT, std::string(what) + ": missing moment state");
  }
  for (int e = 0; e < g.E; ++e)
    if (!s->relation[e]) return fail(GPA_B200_BAD_ARGUMENT, std::string(what) + ": missing relation");
  return GPA_B200_OK;
}

int forward_impl(const Geo& g, const GpaParams* p, const void* q, const void* k, const void* v,
                 const GpaStateRef* si, GpaStateRef* so, void* out, void* saved,
                 size_t saved_bytes, cudaStream_t st) {
  Saved s;
  layout_saved(g, nullptr, &s);
  if (!saved || saved_bytes < s.bytes)
    return fail(GPA_B200_BAD_ARGUMENT, "saved buffer too small (gpa_b200_saved_bytes)");
  layout_saved(g, saved, &s);
  const int U = g.U, T = g.T, D = g.D, Dv = g.Dv;
  const Blocks& bl = g.bl;
  const bool fz_in = g.offset != 0;
  CK(launch_input(q, k, v, g.dt, g.B, T, g.H, D, Dv, s.qf, s.qh, s.qn, s.key[0], s.val[0],
                  g.moments ? g.pos0 : -1, st));
  for (int j = 0; j < g.L; ++j) {
    const int M = g.M[j];
    CK((g.fast ? tc_level_prep : launch_level_prep)(U, T, g.H, D, M, s.key[j], p->center[j], p->gate_weight[j],
                         p->gate_bias[j], g.bm, g.pos_none, s.nk[j], s.kn[j], s.slot[j], s.ns[j],
                         s.sn[j], s.raw4[j], s.gates[j], st));
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = 2;
    ScanDesc& in = sb.s[0];
    ScanDesc& ou = sb.s[1];
    in = blank_scan();
    in.K = D;
    in.V = M;
    in.q = s.qh;
    in.k = s.nk[j];
    in.v = s.slot[j];
    in.g = s.gates[j] + 0;
    in.beta = s.gates[j] + 1;
    in.g_su = (int64_t)T * 4;
    in.g_st = 4;
    in.S0 = si->inner[j];
    in.Sb = s.Abnd[j];
    in.W = s.WA[j];
    in.Ub = s.UA[j];
    in.Wk = s.KA[j];
    in.Tsv = s.TA[j];
    in.O = s.raw[j];
    in.S_final = so->inner[j];
    ou = blank_scan();
    ou.K = M;
    ou.V = Dv;
    ou.k = s.ns[j];
    ou.v = s.val[j];
    ou.g = s.gates[j] + 2;
    ou.beta = s.gates[j] + 3;
    ou.g_su = (int64_t)T * 4;
    ou.g_st = 4;
    ou.S0 = si->outer[j];
    ou.Sb = s.Bbnd[j];
    ou.W = s.WB[j];
    ou.Ub = s.UB[j];
    ou.Wk = s.KB[j];
    ou.Tsv = s.TB[j];
    ou.S_final = so->outer[j];
    CK(gdn_forward(sb, U, bl, true, st));
    const int with_res = j + 1 < g.L;
    CK((g.fast ? tc_level_post : launch_level_post)(U, bl, g.post, g.H, D, Dv, M, with_res, s.nk[j], s.key[j], s.val[j],
                         s.Abnd[j], s.Bbnd[j], fz_in ? si->frozen_inner[j] : nullptr,
                         fz_in ? si->frozen_outer[j] : nullptr, p->residual_raw, j, s.write[j],
                         s.bsum[j], with_res ? s.key[j + 1] : nullptr,
                         with_res ? s.val[j + 1] : nullptr, st));
    if (g.moments)
      CK(launch_moments_fwd(U, bl, D, M, g.pos0, s.qh, s.nk[j], s.write[j], si->moment[j],
                            s.Pb[j], s.corr[j], so->moment[j], st));
    CK(launch_counts(U, bl, g.H, M, g.rs, p->count_gain_raw, j, si->count[j], s.bsum[j],
                     s.write[j], s.raw[j], s.counts[j], s.logits[j], s.lh[j], s.ln[j], s.wh[j],
                     s.wn[j], so->count[j], s.corr[j], p->moment_gain, st));
  }
  CK(launch_rel_gates(U, g.H, g.E, g.pos_none, p->relation_decay_raw, p->relation_beta_raw, s.ge,
                      s.be, st));
  for (int tj = 0; tj < g.L; ++tj) {
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = 0;
    for (int e = 0; e < g.E; ++e) {
      if (g.ed[e] != tj) continue;
      const int i = g.es[e];
      ScanDesc& d = sb.s[sb.n];
      d = blank_scan();
      d.K = g.M[i];
      d.V = g.M[tj];
      d.q = s.lh[i];
      d.k = s.wh[i];
      d.v = s.write[tj];
      d.g = s.ge + (size_t)e * U;
      d.beta = s.be + (size_t)e * U;
      d.g_su = 1;
      d.g_st = 0;
      d.S0 = si->relation[e];
      d.Sb = s.Rbnd[e];
      d.W = s.WR[e];
      d.Ub = s.UR[e];
      d.Wk = s.KR[e];
      d.Tsv = s.TR[e];
      d.O = s.msg[e];
      d.S_final = so->relation[e];
      ++sb.n;
    }
    if (sb.n) CK(gdn_forward(sb, U, bl, true, st));
  }
  for (int j = 0; j < g.L; ++j) {
    BridgeIn bi;
    bi.n = 0;
    bi.mode = g.reader;
    bi.counts = s.counts[j];
    for (int e = 0; e < g.E; ++e)
      if (g.ed[e] == j) {
        bi.edge[bi.n] = e;
        bi.msg[bi.n] = s.msg[e];
        bi.dmsg[bi.n] = nullptr;
        bi.ln[bi.n] = s.ln[g.es[e]];
        bi.dln[bi.n] = nullptr;
        ++bi.n;
      }
    CK((g.fast ? tc_bridge : launch_bridge)(U, T, g.H, D, g.M[j], g.L, j, bi, p->edge_logits, p->relation_gain,
                     p->route_up[j], p->route_down[j], p->route_mlp_gain, p->route_weight[j],
                     p->query_weight[j], g.qs, s.logits[j], s.qf, s.r[j], s.hp[j], s.mlp[j],
                     s.route[j], s.qoh[j], s.qon[j], st));
  }
  {
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = g.L;
    for (int j = 0; j < g.L; ++j) {
      ScanDesc& d = sb.s[j];
      d = blank_scan();
      d.K = g.M[j];
      d.V = Dv;
      d.q = s.qoh[j];
      d.k = s.ns[j];
      d.g = s.gates[j] + 2;
      d.beta = s.gates[j] + 3;
      d.g_su = (int64_t)T * 4;
      d.g_st = 4;
      d.Sb = s.Bbnd[j];
      d.W = s.WB[j];
      d.O = s.y[j];
    }
    CK(gdn_output(sb, U, bl, st));
  }
  std::vector<const float*> ys(s.y, s.y + g.L);
  CK(launch_mix(g.B, T, g.H, Dv, g.L, p->output_logits, ys.data(), out, g.dt, st));
  const int new_off = (g.offset + T) % g.C;
  if (new_off) {
    for (int j = 0; j < g.L; ++j) {
      const size_t na = (size_t)U * D * g.M[j], nbv = (size_t)U * g.M[j] * Dv;
      if (!so->frozen_inner[j] || !so->frozen_outer[j])
        return fail(GPA_B200_BAD_ARGUMENT, "state_out needs frozen snapshots for a partial block");
      const int last = bl.nb - 1;
      if (last == 0 && fz_in) {
        CK(launch_copy(so->frozen_inner[j], si->frozen_inner[j], na, st));
        CK(launch_copy(so->frozen_outer[j], si->frozen_outer[j], nbv, st));
      } else {
        CK(launch_gather_boundary(so->frozen_inner[j], s.Abnd[j], U, bl.nb + 1, last,
                                  (int64_t)D * g.M[j], st));
        CK(launch_gather_boundary(so->frozen_outer[j], s.Bbnd[j], U, bl.nb + 1, last,
                                  (int64_t)g.M[j] * Dv, st));
      }
    }
  }
  return GPA_B200_OK;
}

int backward_impl(const Geo& g, const GpaParams* p, const GpaStateRef* si, const void* saved,
                  const void* dout, const GpaStateRef* dso, void* dq, void* dk, void* dv,
                  GpaStateRef* dsi, GpaParamGrads* gp, void* scratch, size_t scratch_bytes,
                  cudaStream_t st) {
  Saved s;
  layout_saved(g, const_cast<void*>(saved), &s);
  Scratch x;
  layout_scratch(g, nullptr, &x);
  if (!scratch || scratch_bytes < x.bytes)
    return fail(GPA_B200_BAD_ARGUMENT, "scratch buffer too small (gpa_b200_scratch_bytes)");
  layout_scratch(g, scratch, &x);
  const int U = g.U, T = g.T, D = g.D, Dv = g.Dv, L = g.L, E = g.E, H = g.H;
  const Blocks& bl = g.bl;
  const size_t UT = (size_t)U * T;
  const bool fz_in = g.offset != 0;
  const int new_off = (g.offset + T) % g.C;
  GpaStateRef none;
  std::memset(&none, 0, sizeof(none));
  const GpaStateRef& ds = dso ? *dso : none;

  CK(zero(x.dqh, UT * D, st));
  CK(zero(x.dq_direct, UT * D, st));
  CK(zero(x.dkey, UT * D, st));
  CK(zero(x.dval, UT * Dv, st));
  CK(zero(reinterpret_cast<float*>(x.scal), (size_t)U * L * kNScal * 2, st));
  CK(zero(reinterpret_cast<float*>(x.scalE), (size_t)U * (E ? E : 1) * kNEdge * 2, st));
  for (int j = 0; j < L; ++j) {
    const size_t M = g.M[j];
    CK(zero(x.dqoh[j], UT * M, st));
    CK(zero(x.dlh[j], UT * M, st));
    CK(zero(x.dwh[j], UT * M, st));
    CK(zero(x.dwrite[j], UT * M, st));
    CK(zero(x.odK[j], UT * M, st));
    CK(zero(x.odG[j], UT, st));
    if (g.reader != GPA_B200_READER_TANH) CK(zero(x.dln[j], UT, st));
  }
  CK(launch_scales(U, H, L, p->output_logits, x.ow_scale, st));
  std::vector<const float*> ys(s.y, s.y + L);
  CK(launch_mix_bwd(g.B, T, H, Dv, L, dout, g.dt, ys.data(), x.dout_f, x.scal, st));

  auto outer_desc = [&](int j) {
    ScanDesc d = blank_scan();
    d.K = g.M[j];
    d.V = Dv;
    d.q = s.qoh[j];
    d.k = s.ns[j];
    d.v = s.val[j];
    d.g = s.gates[j] + 2;
    d.beta = s.gates[j] + 3;
    d.g_su = (int64_t)T * 4;
    d.g_st = 4;
    d.Sb = s.Bbnd[j];
    d.W = s.WB[j];
    d.dO = x.dout_f;
    d.dO_scale = x.ow_scale + (size_t)j * U;
    d.sc_dK = x.odK[j];
    d.sc_dW = x.odW[j];
    d.sc_dG = x.odG[j];
    return d;
  };
  {
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = L;
    for (int j = 0; j < L; ++j) {
      sb.s[j] = outer_desc(j);
      sb.s[j].dq = x.dqoh[j];
    }
    CK(gdn_backward_local(sb, U, bl, st));
  }
  for (int j = 0; j < L; ++j) {
    BridgeIn bi;
    bi.n = 0;
    bi.mode = g.reader;
    bi.counts = s.counts[j];
    for (int e = 0; e < E; ++e)
      if (g.ed[e] == j) {
        bi.edge[bi.n] = e;
        bi.msg[bi.n] = s.msg[e];
        bi.dmsg[bi.n] = x.dmsg[e];
        bi.ln[bi.n] = s.ln[g.es[e]];
        bi.dln[bi.n] = x.dln[g.es[e]];
        ++bi.n;
      }
    const int M = g.M[j];
    CK((g.fast ? tc_bridge_bwd : launch_bridge_bwd)(U, T, H, D, M, L, j, bi, p->edge_logits, p->relation_gain,
                         p->route_up[j], p->route_down[j], p->route_mlp_gain, p->route_weight[j],
                         p->query_weight[j], g.qs, s.logits[j], s.r[j], s.hp[j], s.mlp[j],
                         s.qoh[j], s.qon[j], x.dqoh[j], x.dqo[j], x.droute[j], x.dhp[j],
                         x.dlogits[j], x.dq_direct, x.scal, x.scalE, E ? E : 1, st));
    CK(head_outer(g, g.B, T, H, s.route[j], M, 0, x.dqo[j], M, nullptr, 0, 1.f,
                         gp->route_weight[j], st));
    CK(head_outer(g, g.B, T, H, s.qf, D, 0, x.dqo[j], M, nullptr, 0, g.qs,
                         gp->query_weight[j], st));
    CK(head_outer(g, g.B, T, H, s.r[j], M, 0, x.dhp[j], 2 * M, nullptr, 0, 1.f,
                         gp->route_up[j], st));
    CK(head_outer(g, g.B, T, H, s.hp[j], 2 * M, 1, x.droute[j], M,
                         p->route_mlp_gain + (size_t)j * H, 1, 1.f, gp->route_down[j], st));
  }
  // relation scans, grouped by target level
  for (int tj = 0; tj < L; ++tj) {
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = 0;
    for (int e = 0; e < E; ++e) {
      if (g.ed[e] != tj) continue;
      const int i = g.es[e], slot = sb.n;
      ScanDesc& d = sb.s[slot];
      d = blank_scan();
      d.K = g.M[i];
      d.V = g.M[tj];
      d.q = s.lh[i];
      d.k = s.wh[i];
      d.v = s.write[tj];
      d.g = s.ge + (size_t)e * U;
      d.beta = s.be + (size_t)e * U;
      d.g_su = 1;
      d.g_st = 0;
      d.Sb = s.Rbnd[e];
      d.W = s.WR[e];
      d.Ub = s.UR[e];
      d.Wk = s.KR[e];
      d.Tsv = s.TR[e];
      d.dO = x.dmsg[e];
      d.dS_final = ds.relation[e];
      d.dq = x.dlh[i];
      d.dk = x.dwh[i];
      d.dv = x.dwrite[tj];
      d.dg64 = x.scalE + (size_t)e * kNEdge + kE_G;
      d.dbeta64 = x.scalE + (size_t)e * kNEdge + kE_B;
      d.dg_su = (int64_t)E * kNEdge;
      d.dg_st = 0;
      d.dS0 = dsi->relation[e];
      d.sc_dW = x.dW[slot];
      d.sc_dK = x.dK[slot];
      d.sc_dWk = x.dWk[slot];
      d.sc_dG = x.dG[slot];
      d.sc_db = x.db[slot];
      d.sc_dA = x.dA[slot];
      d.Dend = x.Dend[slot];
      const size_t K = d.K, V = d.V;
      if (!g.fast) {  // the SIMT kernels accumulate into these; the tensor-core ones overwrite
        CK(zero(x.dK[slot], UT * K, st));
        CK(zero(x.dWk[slot], UT * K, st));
        CK(zero(x.dG[slot], UT, st));
        CK(zero(x.db[slot], UT, st));
        CK(zero(x.dA[slot], (size_t)U * bl.nb * kMaxChunk * kMaxChunk, st));
      }
      (void)V;
      ++sb.n;
    }
    if (!sb.n) continue;
    CK(gdn_backward_local(sb, U, bl, st));
    CK(gdn_backward_rest(sb, U, bl, st));
  }
  for (int j = L - 1; j >= 0; --j) {
    const int M = g.M[j];
    const int with_res = j + 1 < L;
    CK(zero(x.dnsum, (size_t)U * bl.nb * M, st));
    CK(launch_logits_bwd(U, bl, H, M, L, j, g.rs, p->count_gain_raw, s.logits[j], s.counts[j],
                         s.lh[j], s.ln[j], s.wh[j], s.wn[j], x.dlh[j], x.dwh[j], x.dlogits[j],
                         x.dwrite[j], x.draw, x.dn, x.dnsum, x.scal,
                         ProductBwd{g.reader != GPA_B200_READER_TANH ? x.dln[j] : nullptr,
                                    p->relation_gain,
                                    g.reader == GPA_B200_READER_MARGINAL && has_incoming(g, j)},
                         MomentBwd{s.corr[j], p->moment_gain, x.dcorr}, st));
    CK(launch_counts_bwd(U, bl, M, x.dn, x.dnsum, ds.count[j], x.dwrite[j], dsi->count[j], st));
    if (g.moments)  // dq and dwrite now; the unit-key part joins dnk after the post backward
      CK(launch_moments_bwd(U, bl, D, M, g.pos0, s.qh, s.nk[j], s.write[j], s.Pb[j], x.dcorr,
                            ds.moment[j], x.Gend, dsi->moment[j], x.dqh, x.dwrite[j], x.dmk,
                            st));
    const size_t szA = (size_t)D * M, szB = (size_t)M * Dv;
    CK(zero(x.extA, (size_t)U * (bl.nb + 1) * szA, st));
    CK(zero(x.extB, (size_t)U * (bl.nb + 1) * szB, st));
    if (fz_in) {
      CK(zero(dsi->frozen_inner[j], (size_t)U * szA, st));
      CK(zero(dsi->frozen_outer[j], (size_t)U * szB, st));
    }
    if (new_off && ds.frozen_inner[j]) {
      const int last = bl.nb - 1;
      if (last == 0 && fz_in) {
        CK(launch_add(dsi->frozen_inner[j], ds.frozen_inner[j], (int64_t)U * szA, st));
        CK(launch_add(dsi->frozen_outer[j], ds.frozen_outer[j], (int64_t)U * szB, st));
      } else {
        CK(launch_scatter_add_boundary(x.extA, ds.frozen_inner[j], U, bl.nb + 1,
                                       last + g.post, (int64_t)szA, st));
        CK(launch_scatter_add_boundary(x.extB, ds.frozen_outer[j], U, bl.nb + 1,
                                       last + g.post, (int64_t)szB, st));
      }
    }
    CK((g.fast ? tc_post_bwd : launch_post_bwd)(U, bl, g.post, g.offset, H, D, Dv, M, L, j, with_res, s.nk[j], s.write[j],
                       s.Abnd[j], s.Bbnd[j], fz_in ? si->frozen_inner[j] : nullptr,
                       fz_in ? si->frozen_outer[j] : nullptr, p->residual_raw, x.dkey, x.dval,
                       x.dwrite[j], x.dnk, x.extA, x.extB, fz_in ? dsi->frozen_inner[j] : nullptr,
                       fz_in ? dsi->frozen_outer[j] : nullptr, x.scal, st));
    if (g.moments) CK(launch_add(x.dnk, x.dmk, (int64_t)UT * D, st));
    CK(zero(x.dslot, UT * M, st));
    CK(zero(x.dns, UT * M, st));
    CK(zero(x.dgates, UT * 4, st));
    if (!g.fast) {  // the SIMT kernels accumulate into these; the tensor-core ones overwrite
      for (int sl = 0; sl < 2; ++sl) {
        CK(zero(x.dWk[sl], UT * (D > M ? D : M), st));
        CK(zero(x.db[sl], UT, st));
        CK(zero(x.dA[sl], (size_t)U * bl.nb * kMaxChunk * kMaxChunk, st));
      }
      CK(zero(x.dK[0], UT * D, st));
      CK(zero(x.dG[0], UT, st));
    }
    ScanBatch sb;
    sb.tc = g.fast;
    sb.n = 1;
    ScanDesc& in = sb.s[0];
    in = blank_scan();
    in.K = D;
    in.V = M;
    in.q = s.qh;
    in.k = s.nk[j];
    in.v = s.slot[j];
    in.g = s.gates[j] + 0;
    in.beta = s.gates[j] + 1;
    in.g_su = (int64_t)T * 4;
    in.g_st = 4;
    in.Sb = s.Abnd[j];
    in.W = s.WA[j];
    in.Ub = s.UA[j];
    in.Wk = s.KA[j];
    in.Tsv = s.TA[j];
    in.dO = x.draw;
    in.ext = x.extA;
    in.dS_final = ds.inner[j];
    in.dq = x.dqh;
    in.dk = x.dnk;
    in.dv = x.dslot;
    in.dg = x.dgates + 0;
    in.dbeta = x.dgates + 1;
    in.dg_su = (int64_t)T * 4;
    in.dg_st = 4;
    in.dS0 = dsi->inner[j];
    in.sc_dW = x.dW[0];
    in.sc_dK = x.dK[0];
    in.sc_dWk = x.dWk[0];
    in.sc_dG = x.dG[0];
    in.sc_db = x.db[0];
    in.sc_dA = x.dA[0];
    in.Dend = x.Dend[0];
    CK(gdn_backward_local(sb, U, bl, st));
    sb.n = 2;
    ScanDesc& ou = sb.s[1];
    ou = outer_desc(j);
    ou.Ub = s.UB[j];
    ou.Wk = s.KB[j];
    ou.Tsv = s.TB[j];
    ou.ext = x.extB;
    ou.dS_final = ds.outer[j];
    ou.dk = x.dns;
    ou.dv = x.dval;
    ou.dg = x.dgates + 2;
    ou.dbeta = x.dgates + 3;
    ou.dg_su = (int64_t)T * 4;
    ou.dg_st = 4;
    ou.dS0 = dsi->outer[j];
    ou.sc_dWk = x.dWk[1];
    ou.sc_db = x.db[1];
    ou.sc_dA = x.dA[1];
    ou.Dend = x.Dend[1];
    CK(gdn_backward_rest(sb, U, bl, st));
    CK((g.fast ? tc_prep_bwd : launch_prep_bwd)(U, T, H, D, M, p->center[j], p->gate_weight[j], g.bm, g.pos_none,
                       s.raw4[j], s.nk[j], s.kn[j], s.ns[j], s.sn[j], x.dgates, x.dnk, x.dns,
                       x.dslot, x.d4, x.dkey, st));
    CK(head_outer(g, g.B, T, H, x.dslot, M, 0, s.key[j], D, nullptr, 0, 1.f, gp->center[j],
                         st));
    CK(launch_gate_grad(g.B, T, H, s.nk[j], D, x.d4, gp->gate_weight[j], gp->gate_bias[j], st));
  }
  CK(launch_input_bwd(g.B, T, H, D, Dv, g.dt, s.qh, s.qn, x.dqh, x.dq_direct, x.dkey, x.dval, dq,
                      dk, dv, g.moments ? g.pos0 : -1, st));
  FoldArgs fa;
  std::memset(&fa, 0, sizeof(fa));
  fa.B = g.B;
  fa.H = H;
  fa.L = L;
  fa.E = E;
  fa.pos_none = g.pos_none;
  for (int e = 0; e < E; ++e) {
    fa.edge_src[e] = g.es[e];
    fa.edge_dst[e] = g.ed[e];
  }
  fa.residual_raw = p->residual_raw;
  fa.count_gain_raw = p->count_gain_raw;
  fa.output_logits = p->output_logits;
  fa.edge_logits = p->edge_logits;
  fa.relation_decay_raw = p->relation_decay_raw;
  fa.relation_beta_raw = p->relation_beta_raw;
  fa.scal = x.scal;
  fa.scalE = x.scalE;
  fa.g_residual_raw = gp->residual_raw;
  fa.g_count_gain_raw = gp->count_gain_raw;
  fa.g_route_mlp_gain = gp->route_mlp_gain;
  fa.g_relation_gain = gp->relation_gain;
  fa.g_output_logits = gp->output_logits;
  fa.g_edge_logits = gp->edge_logits;
  fa.g_relation_decay_raw = gp->relation_decay_raw;
  fa.g_relation_beta_raw = gp->relation_beta_raw;
  fa.g_moment_gain = g.moments ? gp->moment_gain : nullptr;
  CK(launch_fold(fa, st));
  return GPA_B200_OK;
}

}  // namespace
}  // namespace gpa

using namespace gpa;

extern "C" {

size_t gpa_b200_saved_bytes(const GpaDims* dims) {
  Geo g;
  std::string why;
  if (make_geo(dims, &g, &why) != GPA_B200_OK) return 0;
  Saved s;
  layout_saved(g, nullptr, &s);
  return s.bytes;
}

size_t gpa_b200_scratch_bytes(const GpaDims* dims) {
  Geo g;
  std::string why;
  if (make_geo(dims, &g, &why) != GPA_B200_OK) return 0;
  Scratch x;
  layout_scratch(g, nullptr, &x);
  return x.bytes;
}

int gpa_b200_forward(const GpaDims* dims, const GpaParams* params, const void* q, const void* k,
                     const void* v, const GpaStateRef* state_in, GpaStateRef* state_out,
                     void* out, void* saved, size_t saved_bytes, void* stream) {
  g_last_error.clear();
  Geo g;
  std::string why;
  int rc = make_geo(dims, &g, &why);
  if (rc) return fail(rc, why);
  if ((rc = check_params(g, params))) return rc;
  if ((rc = check_state(g, state_in, g.offset != 0, "state_in"))) return rc;
  if ((rc = check_state(g, state_out, false, "state_out"))) return rc;
  if (g.T == 0) return fail(GPA_B200_BAD_ARGUMENT, "length must be positive (empty calls are host-side)");
  if (!q || !k || !v || !out) return fail(GPA_B200_BAD_ARGUMENT, "q/k/v/out must not be NULL");
  return forward_impl(g, params, q, k, v, state_in, state_out, out, saved, saved_bytes,
                      static_cast<cudaStream_t>(stream));
}

int gpa_b200_step(const GpaDims* dims, const GpaParams* params, const void* q, const void* k,
                  const void* v, const GpaStateRef* state, int32_t* offset, void* out,
                  void* stream) {
  g_last_error.clear();
  Geo g;
  std::string why;
  int rc = make_geo(dims, &g, &why);
  if (rc) return fail(rc, why);
  if (g.T != 1) return fail(GPA_B200_BAD_ARGUMENT, "gpa_b200_step takes one token (length 1)");
  if (g.C < 2)
    return fail(GPA_B200_UNSUPPORTED, "gpa_b200_step needs lag blocks (chunk_size >= 2)");
  if (g.D % 4 || g.Dv % 4)
    return fail(GPA_B200_UNSUPPORTED, "gpa_b200_step needs key/value widths that are multiples of 4");
  for (int j = 0; j < g.L; ++j)
    if (g.M[j] % 4) return fail(GPA_B200_UNSUPPORTED, "gpa_b200_step needs slot counts that are multiples of 4");
  if ((rc = check_params(g, params))) return rc;
  if ((rc = check_state(g, state, true, "state"))) return rc;
  if (!q || !k || !v || !out || !offset)
    return fail(GPA_B200_BAD_ARGUMENT, "q/k/v/out/offset must not be NULL");
  StepArgs a;
  a.U = g.U;
  a.H = g.H;
  a.D = g.D;
  a.Dv = g.Dv;
  a.L = g.L;
  a.E = g.E;
  a.C = g.C;
  for (int j = 0; j < kMaxLevels; ++j) a.M[j] = j < g.L ? g.M[j] : 0;
  for (int e = 0; e < kMaxEdges; ++e) {
    a.es[e] = e < g.E ? g.es[e] : 0;
    a.ed[e] = e < g.E ? g.ed[e] : 0;
  }
  a.dt = g.dt;
  a.pos_none = g.pos_none;
  a.reader = g.reader;
  a.moments = g.moments;
  a.query_scale = g.qs;
  a.beta_max = g.bm;
  a.read_scale = g.rs;
  a.p = *params;
  a.s = *state;
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.offset = offset;
  if (decode_step_smem(a) > 227 * 1024)
    return fail(GPA_B200_UNSUPPORTED, "gpa_b200_step: widths too large for one CTA");
  const cudaError_t e = launch_decode_step(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(GPA_B200_LAUNCH_FAILURE, std::string("decode step: ") + cudaGetErrorString(e));
  return GPA_B200_OK;
}

int gpa_b200_backward(const GpaDims* dims, const GpaParams* params, const GpaStateRef* state_in,
                      const void* saved, const void* dout, const GpaStateRef* dstate_out,
                      void* dq, void* dk, void* dv, GpaStateRef* dstate_in,
                      GpaParamGrads* dparams, void* scratch, size_t scratch_bytes, void* stream) {
  g_last_error.clear();
  Geo g;
  std::string why;
  int rc = make_geo(dims, &g, &why);
  if (rc) return fail(rc, why);
  if ((rc = check_params(g, params))) return rc;
  if ((rc = check_state(g, state_in, g.offset != 0, "state_in"))) return rc;
  if ((rc = check_state(g, dstate_in, g.offset != 0, "dstate_in"))) return rc;
  if (g.T == 0) return fail(GPA_B200_BAD_ARGUMENT, "length must be positive");
  if (!saved || !dout || !dq || !dk || !dv || !dparams)
    return fail(GPA_B200_BAD_ARGUMENT, "saved/dout/dq/dk/dv/dparams must not be NULL");
  return backward_impl(g, params, state_in, saved, dout, dstate_out, dq, dk, dv, dstate_in,
                       dparams, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------- no-allocation forward
// Scratch of gpa_b200_forward_noalloc: one file-scope device array per GPU that
// loads this library (held until the process exits).  Host code only sees a
// host-side stand-in under this name; the device address is looked up per
// device with cudaGetSymbolAddress and cached.
constexpr size_t kNoAllocBytes = size_t(64) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
constexpr int kMaxDevices = 64;
void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GPA_B200_LAUNCH_FAILURE, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(GPA_B200_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(GPA_B200_LAUNCH_FAILURE,
                  std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GPA_B200_OK;
}
}  // namespace

size_t gpa_b200_noalloc_capacity(void) { return kNoAllocBytes; }

int gpa_b200_device_status(int clear) {
  const int a = gpa::tc5_device_status(clear != 0), b = gpa::decode_device_status(clear != 0);
  const int c = gpa::outer_device_status(clear != 0);
  if (a < 0 || b < 0 || c < 0) return -1;
  return a ? a : b ? b : c;
}

int gpa_b200_umma_selftest(int M, int mma_m, int N, int Kd, int a_mn, int b_mn, int flags,
                           const void* A, const void* B, const void* A_tiled, float* D,
                           int* status, void* stream) {
  g_last_error.clear();
  if (!gpa::umma_probe_shape_ok(M, mma_m, N, Kd, flags))
    return fail(GPA_B200_UNSUPPORTED, "umma self-test: unsupported shape or flags");
  const bool a_bulk = flags & GPA_B200_UMMA_BULK_A;
  if (!B || !D || !status || (a_bulk ? !A_tiled : !A))
    return fail(GPA_B200_BAD_ARGUMENT, "umma self-test: NULL operand");
  if (a_bulk && (reinterpret_cast<uintptr_t>(A_tiled) & 15))
    return fail(GPA_B200_BAD_ARGUMENT, "umma self-test: A_tiled must be 16-byte aligned");
  const int rc = gpa::umma_probe(M, mma_m, N, Kd, a_mn, b_mn, flags, A, B, A_tiled, D, status,
                                 static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "umma self-test: launch failed") : GPA_B200_OK;
}

int gpa_b200_forward_noalloc(const GpaDims* dims, const GpaParams* params, const void* q,
                             const void* k, const void* v, const GpaStateRef* state_in,
                             GpaStateRef* state_out, void* out, void* stream) {
  g_last_error.clear();
  Geo g;
  std::string why;
  int rc = make_geo(dims, &g, &why);
  if (rc) return fail(rc, why);
  if ((rc = check_params(g, params))) return rc;
  if ((rc = check_state(g, state_in, g.offset != 0, "state_in"))) return rc;
  if ((rc = check_state(g, state_out, false, "state_out"))) return rc;
  if (g.T == 0) return fail(GPA_B200_BAD_ARGUMENT, "length must be positive (empty calls are host-side)");
  if (!q || !k || !v || !out) return fail(GPA_B200_BAD_ARGUMENT, "q/k/v/out must not be NULL");
  Saved sz;
  layout_saved(g, nullptr, &sz);
  if (sz.bytes > kNoAllocBytes)
    return fail(GPA_B200_UNSUPPORTED,
                "this call needs " + std::to_string(sz.bytes) + " bytes of scratch; the "
                "no-allocation entry point holds " + std::to_string(kNoAllocBytes) +
                " (use gpa_b200_forward with a caller buffer)");
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  return forward_impl(g, params, q, k, v, state_in, state_out, out, scratch, kNoAllocBytes,
                      static_cast<cudaStream_t>(stream));
}

int gpa_b200_routes(const GpaDims* dims, const void* saved, void* const* routes, void* stream) {
  g_last_error.clear();
  Geo g;
  std::string why;
  int rc = make_geo(dims, &g, &why);
  if (rc) return fail(rc, why);
  if (!saved || !routes) return fail(GPA_B200_BAD_ARGUMENT, "saved/routes must not be NULL");
  Saved s;
  layout_saved(g, const_cast<void*>(saved), &s);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int j = 0; j < g.L; ++j) {
    if (!routes[j]) return fail(GPA_B200_BAD_ARGUMENT, "routes[j] must not be NULL");
    CK(launch_to_bthx(s.route[j], routes[j], g.dt, g.B, g.T, g.H, g.M[j], st));
  }
  return GPA_B200_OK;
}

int gpa_b200_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::snprintf(buf, len, "%s", g_last_error.c_str());
  }
  return g_last_error.empty() ? 0 : 1;
}

int gpa_b200_abi_version(void) { return 2; }

long long gpa_b200_launch_count(void) { return g_launches.load(); }

int gpa_b200_profile_start(void) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  g_used = 0;
  g_profiling.store(true);
  return GPA_B200_OK;
}

int gpa_b200_profile_stop(char* buf, size_t len) {
  g_profiling.store(false);
  std::lock_guard<std::mutex> lock(g_prof_mu);
  std::map<std::string, std::pair<long long, double>> acc;
  for (size_t i = 0; i < g_used; ++i) {
    float ms = 0.f;
    if (cudaEventSynchronize(g_recs[i].b) != cudaSuccess ||
        cudaEventElapsedTime(&ms, g_recs[i].a, g_recs[i].b) != cudaSuccess)
      return fail(GPA_B200_LAUNCH_FAILURE, "profile events could not be read");
    auto& e = acc[g_recs[i].name];
    e.first += 1;
    e.second += ms;
  }
  std::string out = "{";
  for (auto& kv : acc) {
    char item[160];
    std::snprintf(item, sizeof(item), "%s\"%s\": [%lld, %.6f]", out.size() > 1 ? ", " : "",
                  kv.first.c_str(), kv.second.first, kv.second.second);
    out += item;
  }
  out += "}";
  g_used = 0;
  if (buf && len) std::snprintf(buf, len, "%s", out.c_str());
  return out.size() + 1 <= len ? GPA_B200_OK : GPA_B200_BAD_ARGUMENT;
}

}  // extern "C"
