// Per-token level, relation-reader and output kernels of the DenseGPA core.
// Launchers are declared here and defined in level.cu; all are stream-ordered
// and allocate nothing.  Buffers are fp32, unit-major [U, T, X] (see common.cuh).
#pragma once
#include "../../include/gpa_b200.h"
#include "common.cuh"

namespace gpa {

constexpr int kMaxLevels = 8;
constexpr int kMaxEdges = kMaxLevels * (kMaxLevels - 1);
constexpr int kMaxIn = kMaxLevels - 1;

// cos / sin of the rotary angle of element d (pair d / 2) at position pos,
// pos * 10000^(-2i/D) (src/gpa/ops.py:117-132), in double precision (positions reach 2^31)
__device__ __forceinline__ void rope_cs(int64_t pos, int d, int D, float& c, float& s) {
  const double ang = (double)pos * exp(-log(10000.0) * (double)(d & ~1) / (double)D);
  double sd, cd;
  sincos(ang, &sd, &cd);
  c = (float)cd;
  s = (float)sd;
}

// per-(unit, level) scalar gradient accumulators
enum ScalarSlot {
  kS_EtaK = 0, kS_EtaV, kS_CountGain, kS_MlpGain, kS_RelGain, kS_OutW, kS_MomentGain, kNScal = 8
};
// per-(unit, edge) accumulators
enum EdgeSlot { kE_W = 0, kE_G, kE_B, kNEdge = 3 };

struct BridgeIn {
  int n;                      // incoming edges
  int edge[kMaxIn];           // edge ids
  const float* msg[kMaxIn];   // [U,T,M]
  float* dmsg[kMaxIn];        // [U,T,M] (backward)
  // product reader (mode GPA_B200_READER_PRODUCT / _MARGINAL): each message times the norm of
  // its source level's route softmax, ln [U,T]; the backward adds the gradient of that norm
  // into dln [U,T] (one writer per row and source level in a launch)
  int mode;
  const float* ln[kMaxIn];
  float* dln[kMaxIn];
  const float* counts;        // [U,T,M] counts of the target level (marginal term)
};

// rope_pos0 >= 0: the queries are rotated (positional moments), token t at rope_pos0 + t
cudaError_t launch_input(const void* q, const void* k, const void* v, int dt, int B, int T, int H,
                         int D, int Dv, float* qf, float* qh, float* qn, float* key0, float* val0,
                         int64_t rope_pos0, cudaStream_t st);
cudaError_t launch_level_prep(int U, int T, int H, int D, int M, const float* key, const float* C,
                              const float* Wg, const float* gbias, float beta_max, int pos_none,
                              float* nk, float* kn, float* slot, float* ns, float* sn, float* raw4,
                              float* gates, cudaStream_t st);
cudaError_t launch_level_post(int U, const Blocks& bl, int post, int H, int D, int Dv, int M,
                              int with_residual, const float* nk, const float* key, const float* val,
                              const float* Abnd, const float* Bbnd, const float* fzA,
                              const float* fzB, const float* residual_raw, int j, float* write,
                              float* bsum, float* key_next, float* val_next, cudaStream_t st);
cudaError_t launch_counts(int U, const Blocks& bl, int H, int M, float read_scale,
                          const float* count_gain_raw, int j, const float* n0, const float* bsum,
                          const float* write, const float* raw, float* counts, float* logits,
                          float* lh, float* ln, float* wh, float* wn, float* n_final,
                          const float* corr, const float* moment_gain, cudaStream_t st);
cudaError_t launch_rel_gates(int U, int H, int E, int pos_none, const float* decay_raw,
                             const float* beta_raw, float* ge, float* be, cudaStream_t st);
cudaError_t launch_bridge(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                          const float* edge_logits, const float* relation_gain,
                          const float* route_up, const float* route_down,
                          const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                          float qs, const float* logits, const float* qf, float* r, float* hp,
                          float* mlp, float* route, float* qoh, float* qon, cudaStream_t st);
cudaError_t launch_mix(int B, int T, int H, int Dv, int L, const float* output_logits,
                       const float* const* y, void* out, int dt, cudaStream_t st);
cudaError_t launch_copy(float* dst, const float* src, int64_t n, cudaStream_t st);
// dst [B,T,H,X] (dtype dt) <- src [U,T,X] fp32
cudaError_t launch_to_bthx(const float* src, void* dst, int dt, int B, int T, int H, int X,
                           cudaStream_t st);
cudaError_t launch_add(float* dst, const float* src, int64_t n, cudaStream_t st);
// dst[u] = src[u, idx] for src laid out [U, nb1, sz]
cudaError_t launch_gather_boundary(float* dst, const float* src, int U, int nb1, int idx,
                                   int64_t sz, cudaStream_t st);
// dst[u, idx] += src[u] for dst laid out [U, nb1, sz]
cudaError_t launch_scatter_add_boundary(float* dst, const float* src, int U, int nb1, int idx,
                                        int64_t sz, cudaStream_t st);

// ---- backward ----
cudaError_t launch_scales(int U, int H, int L, const float* output_logits, float* ow_scale,
                          cudaStream_t st);
cudaError_t launch_mix_bwd(int B, int T, int H, int Dv, int L, const void* dout, int dt,
                           const float* const* y, float* dout_f, double* scal, cudaStream_t st);
cudaError_t launch_bridge_bwd(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                              const float* edge_logits, const float* relation_gain,
                              const float* route_up, const float* route_down,
                              const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                              float qs, const float* logits, const float* r, const float* hp,
                              const float* mlp, const float* qoh, const float* qon,
                              const float* dqoh, float* dqo, float* droute, float* dhp,
                              float* dlogits, float* dq_direct, double* scal, double* scalE, int E,
                              cudaStream_t st);
// Product-reader terms of a level's logits backward: dln [U,T] (gradient of the norm of the
// level's route softmax, from the readers it feeds; null: none) and, for the marginal reader
// on a level with incoming edges, the count term -e^{clamp(relation_gain)} dlogits / (1 + n).
struct ProductBwd {
  const float* dln;
  const float* relation_gain;  // [L,H]
  int marginal;
};
// Positional-moment terms of a level's logits backward (corr null: none): the level's moment
// reads corr [U,T,M] and their gradient dcorr (written).
struct MomentBwd {
  const float* corr;
  const float* moment_gain;  // [L,H]
  float* dcorr;
};
cudaError_t launch_logits_bwd(int U, const Blocks& bl, int H, int M, int L, int j,
                              float read_scale, const float* count_gain_raw, const float* logits,
                              const float* counts, const float* lh, const float* ln,
                              const float* wh, const float* wn, const float* dlh,
                              const float* dwh, const float* dlogits, float* dwrite, float* draw,
                              float* dn, float* dnsum, double* scal, ProductBwd pb, MomentBwd mb,
                              cudaStream_t st);
cudaError_t launch_counts_bwd(int U, const Blocks& bl, int M, const float* dn, const float* dnsum,
                              const float* dn_final, float* dwrite, float* dn0, cudaStream_t st);
cudaError_t launch_post_bwd(int U, const Blocks& bl, int post, int offset, int H, int D, int Dv,
                            int M, int L, int j, int with_residual, const float* nk,
                            const float* write, const float* Abnd, const float* Bbnd,
                            const float* fzA, const float* fzB, const float* residual_raw,
                            const float* dkey, const float* dval, float* dwrite, float* dnk,
                            float* extA, float* extB, float* dfzA, float* dfzB, double* scal,
                            cudaStream_t st);
cudaError_t launch_prep_bwd(int U, int T, int H, int D, int M, const float* C, const float* Wg,
                            float beta_max, int pos_none, const float* raw4, const float* nk,
                            const float* kn, const float* ns, const float* sn, const float* dgates,
                            const float* dnk, const float* dns, float* dslot, float* d4,
                            float* dkey, cudaStream_t st);
// out[h] (P x Q) += scale[h] * sum over units of head h and tokens of X^T Y.
// xmode: 0 identity, 1 gelu(X), 2 X is all ones (P must be 1).
// gate parameter gradients of one level: gw[h] (D x 4) += sum_{b,t} X^T Y and gb[h] (4) +=
// sum_{b,t} Y over the rows of head h; X [U,T,D] (D <= 128), Y [U,T,4]
cudaError_t launch_gate_grad(int B, int T, int H, const float* X, int D, const float* Y, float* gw,
                             float* gb, cudaStream_t st);
cudaError_t launch_head_outer(int B, int T, int H, const float* X, int P, int xmode,
                              const float* Y, int Q, const float* scale, int64_t scale_stride,
                              float cscale, float* out, cudaStream_t st);
cudaError_t launch_input_bwd(int B, int T, int H, int D, int Dv, int dt, const float* qh,
                             const float* qn, const float* dqh, const float* dq_direct,
                             const float* dkey, const float* dval, void* dq, void* dk, void* dv,
                             int64_t rope_pos0, cudaStream_t st);

// Tensor-core variants (level_tc.cu): bf16 operands, fp32 accumulation; widths
// (key_dim, value_dim, slots) multiples of 16 and <= 128.  Same arguments as the
// SIMT launchers above.
cudaError_t tc_level_prep(int U, int T, int H, int D, int M, const float* key, const float* C,
                          const float* Wg, const float* gbias, float beta_max, int pos_none,
                          float* nk, float* kn, float* slot, float* ns, float* sn, float* raw4,
                          float* gates, cudaStream_t st);
cudaError_t tc_level_post(int U, const Blocks& bl, int post, int H, int D, int Dv, int M,
                          int with_residual, const float* nk, const float* key, const float* val,
                          const float* Abnd, const float* Bbnd, const float* fzA, const float* fzB,
                          const float* residual_raw, int j, float* write, float* bsum,
                          float* key_next, float* val_next, cudaStream_t st);
cudaError_t tc_bridge(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                      const float* edge_logits, const float* relation_gain, const float* route_up,
                      const float* route_down, const float* route_mlp_gain, const float* Wrs,
                      const float* Wqs, float qs, const float* logits, const float* qf, float* r,
                      float* hp, float* mlp, float* route, float* qoh, float* qon,
                      cudaStream_t st);
cudaError_t tc_bridge_bwd(int U, int T, int H, int D, int M, int L, int j, const BridgeIn& in,
                          const float* edge_logits, const float* relation_gain,
                          const float* route_up, const float* route_down,
                          const float* route_mlp_gain, const float* Wrs, const float* Wqs,
                          float qs, const float* logits, const float* r, const float* hp,
                          const float* mlp, const float* qoh, const float* qon, const float* dqoh,
                          float* dqo, float* droute, float* dhp, float* dlogits, float* dq_direct,
                          double* scal, double* scalE, int E, cudaStream_t st);
cudaError_t tc_post_bwd(int U, const Blocks& bl, int post, int offset, int H, int D, int Dv,
                        int M, int L, int j, int with_residual, const float* nk,
                        const float* write, const float* Abnd, const float* Bbnd,
                        const float* fzA, const float* fzB, const float* residual_raw,
                        const float* dkey, const float* dval, float* dwrite, float* dnk,
                        float* extA, float* extB, float* dfzA, float* dfzB, double* scal,
                        cudaStream_t st);
cudaError_t tc_prep_bwd(int U, int T, int H, int D, int M, const float* C, const float* Wg,
                        float beta_max, int pos_none, const float* raw4, const float* nk,
                        const float* kn, const float* ns, const float* sn, const float* dgates,
                        const float* dnk, const float* dns, float* dslot, float* d4, float* dkey,
                        cudaStream_t st);
// P, Q multiples of 16; xmode 0 or 1
cudaError_t tc_head_outer(int B, int T, int H, const float* X, int P, int xmode, const float* Y,
                          int Q, const float* scale, int64_t scale_stride, float cscale,
                          float* out, cudaStream_t st);

struct FoldArgs {
  int B, H, L, E, pos_none;
  int edge_src[kMaxEdges], edge_dst[kMaxEdges];
  const float *residual_raw, *count_gain_raw, *output_logits, *edge_logits, *relation_decay_raw,
      *relation_beta_raw;
  const double *scal, *scalE;
  float *g_residual_raw, *g_count_gain_raw, *g_route_mlp_gain, *g_relation_gain,
      *g_output_logits, *g_edge_logits, *g_relation_decay_raw, *g_relation_beta_raw;
  float* g_moment_gain;  // null without positional moments
};
cudaError_t launch_fold(const FoldArgs& a, cudaStream_t st);

// Parameter-gradient reductions on tcgen05 (outer_tc5.cu), selected in tc_head_outer by
// GPA_B200_OUTER=tc5 (the mma.sync kernel is the default).  P, Q multiples of 8, <= 256.
bool tc5_outer_enabled();
cudaError_t tc5_head_outer_launch(int B, int T, int H, const float* X, int P, int xmode,
                                  const float* Y, int Q, const float* scale,
                                  int64_t scale_stride, float cscale, float* out,
                                  cudaStream_t st);
// device status word of that kernel (GPA_B200_DEVICE_TIMEOUT after a wait gave up)
int outer_device_status(bool clear);

// Positional moments of one level (moments.cu): forward P snapshots at every block start and
// the end, corr [U,T,M] and the final state; backward dq (+=), dw (+=), the unit-key gradient
// dkey (written) and dP_0 (written), with G_end [U, nb, D, M] as workspace.  pos0: absolute
// position of the call's first token.
cudaError_t launch_moments_fwd(int U, const Blocks& bl, int D, int M, int64_t pos0,
                               const float* qh, const float* nk, const float* w, const float* P0,
                               float* Pb, float* corr, float* Pout, cudaStream_t st);
cudaError_t launch_moments_bwd(int U, const Blocks& bl, int D, int M, int64_t pos0,
                               const float* qh, const float* nk, const float* w, const float* Pb,
                               const float* dcorr, const float* dPfinal, float* Gend, float* dP0,
                               float* dq, float* dw, float* dkey, cudaStream_t st);

}  // namespace gpa
