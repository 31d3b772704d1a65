// Chunked gated-delta-rule (GDN) scans over lag blocks: forward and backward.
//
// Recurrence (key-major, src/gpa/ops.py:29-46, docs/EQUATIONS.md:7-28):
//   S_t = a_t S_{t-1} + b_t k_t (v_t - a_t k_t^T S_{t-1})^T,   y_t = q_t^T S_t,
// with unit-normalised q, k supplied by the caller and a_t = exp(g_t).
//
// Chunk form (the WY / UT representation of Yang et al. 2024, "Parallelizing
// Linear Transformers with the Delta Rule over Sequence Length"), per block of
// c <= 64 tokens with G = inclusive cumsum of g inside the block:
//   A_ts = b_t exp(G_t - G_s) k_t.k_s  (s < t),   (I + A) [U | Wk] = [b V | b e^G K]
//   W = U - Wk S_0,   O = e^G (Q S_0) + ((Q K^T) o Gamma) W,
//   S_c = e^{G_c} S_0 + K^T diag(e^{G_c - G}) W.
// The triangular system is solved by column-parallel forward substitution
// (one thread per right-hand-side column), so T = (I + A)^-1 is never formed;
// the backward uses back substitution with (I + A)^T the same way.
//
// Kernels (SIMT fp32 in this file; every launch covers a batch of scans that
// may have different K, V):
//   gdn_fwd_chunk   chunk-parallel:  A, U, Wk                        (also backward recompute)
//   gdn_fwd_state   sequential over blocks, V-sliced: boundary states, W
//   gdn_fwd_out     chunk-parallel, V-sliced: O
//   gdn_bwd_local   chunk-parallel, V-sliced: dQ, dK (read part), dW_local, dG (read part)
//   gdn_bwd_state   sequential reverse over blocks, V-sliced: D (dS) at block ends, dW
//   gdn_bwd_chunk_v chunk-parallel, V-sliced: state-update + U-path terms
//   gdn_bwd_chunk_k chunk-parallel: Wk-path terms, dA consequences, dg = revcumsum(dG)
#pragma once
#include "common.cuh"

namespace gpa {

constexpr int kMaxScans = 8;
constexpr int kVSlice = 64;
constexpr int kAStride = 65;  // padded row stride of c x c tiles in shared memory

struct ScanDesc {
  int K, V;
  const float* q;     // [U,T,K] unit-normalised queries (null: no output)
  const float* k;     // [U,T,K] unit-normalised keys
  const float* v;     // [U,T,V]
  const float* g;     // log decay, element (u,t) at g[u*g_su + t*g_st]
  const float* beta;  // same indexing as g
  int64_t g_su, g_st;
  const float* S0;    // [U,K,V] initial state
  float* Sb;          // [U,NB+1,K,V] block-boundary states
  float* W;           // [U,T,V] pseudo-values: fp32 (SIMT path) or bf16 (tensor-core path,
                      // whose every consumer reads W as single bf16 operands)
  float* Ub;          // [U,T,V] T diag(b) V (may alias W in the forward)
  float* Wk;          // [U,T,K] T diag(b e^G) K
  float* O;           // [U,T,V] output (null: none)
  float* S_final;     // [U,K,V] copy of the final state (null: none)
  // ---- backward ----
  const float* dO;        // [U,T,V] output gradient (null: zero)
  const float* dO_scale;  // per-unit scale of dO (null: 1)
  const float* ext;       // [U,NB+1,K,V] external gradients of boundary states (null: zero)
  const float* dS_final;  // [U,K,V] gradient of the final state (null: zero)
  float* dq;              // [U,T,K] += (null: skip)
  float* dk;              // [U,T,K] +=
  float* dv;              // [U,T,V] +=
  float* dg;              // += at dg[u*dg_su + t*dg_st]
  float* dbeta;           // += with dg's indexing
  int64_t dg_su, dg_st;
  double* dg64;           // if set: dg / dbeta are summed over t into dg64 / dbeta64 [u*dg_su]
  double* dbeta64;
  float* dS0;             // [U,K,V] gradient of the initial state (written)
  float* sc_dW;           // [U,T,V] scratch
  float* sc_dK;           // [U,T,K] scratch (zeroed by the caller)
  float* sc_dWk;          // [U,T,K] scratch (zeroed)
  float* sc_dG;           // [U,T]   scratch (zeroed)
  float* sc_db;           // [U,T]   scratch (zeroed)
  float* sc_dA;           // [U,NB,64,64] scratch (zeroed)
  float* Dend;            // [U,NB,K,V] dS at each block end
  float* Tsv;             // [U,NB,64,64] T = (I + A)^-1 of every block (same)
};

struct ScanBatch {
  int n;
  int tc;  // 1: tensor-core kernels (bf16 operands); 0: SIMT fp32 kernels
  ScanDesc s[kMaxScans];
};

// Host launchers (gdn.cu).  All are stream-ordered and allocate nothing.
cudaError_t gdn_forward(const ScanBatch& b, int U, const Blocks& bl, bool with_output,
                        cudaStream_t st);
cudaError_t gdn_output(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
cudaError_t gdn_backward_local(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
cudaError_t gdn_backward_rest(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
int gdn_max_smem_bytes();

// tensor-core variants (gdn_tc.cu); widths must be multiples of 16 and <= 128
bool tc_supported(int K, int V);
cudaError_t tc_forward(const ScanBatch& b, int U, const Blocks& bl, bool with_output,
                       cudaStream_t st);
cudaError_t tc_output(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
cudaError_t tc_backward_local(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
cudaError_t tc_backward_rest(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);

// tcgen05 state sweeps (gdn_tc5.cu); GPA_B200_SWEEPS=mma in the environment selects the
// mma.sync sweeps instead (kept for comparison)
bool tc5_sweeps_enabled();
cudaError_t tc5_fwd_state_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
cudaError_t tc5_bwd_state_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
// tcgen05 WY / UT transform of every block (gdn_tc5.cu): A, T (kept), U, Wk;
// GPA_B200_WY=mma selects the mma.sync kernel instead
bool tc5_wy_enabled();
cudaError_t tc5_fwd_chunk_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
// tcgen05 block outputs O = e^G Q S_n + P W (gdn_tc5.cu), selected by GPA_B200_OUT=tc5 (the
// mma.sync kernel is the default)
bool tc5_out_enabled();
cudaError_t tc5_fwd_out_launch(const ScanBatch& b, int U, const Blocks& bl, cudaStream_t st);
// device status word of the tcgen05 kernels (GPA_B200_DEVICE_TIMEOUT after a wait gave up);
// synchronous read, optionally clearing it; -1 if the read failed
int tc5_device_status(bool clear);

// tcgen05 self-test (tc5_probe.cu): D = A B on one CTA; returns a GPA_B200_* status
int umma_probe(int M, int mma_m, int N, int Kd, int a_mn, int b_mn, int flags, const void* A,
               const void* B, const void* A_tiled, float* D, int* status, cudaStream_t st);
bool umma_probe_shape_ok(int M, int mma_m, int N, int Kd, int flags);

}  // namespace gpa
