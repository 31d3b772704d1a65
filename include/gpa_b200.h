/* gpa_b200.h -- C ABI of the B200-native DenseGPA attention core.
 *
 * The library (gpa_b200/libgpa_b200.so, sm_100a) computes the forward and the
 * backward of fisalt/GPA's DenseGPA core on CUDA device buffers.  Every entry
 * point is stream-ordered on the caller's stream, allocates no device memory
 * (the caller passes the workspaces it sized with the *_bytes queries), never
 * synchronises the device and never traps: failures return a nonzero status
 * and a message readable with gpa_b200_last_error().
 *
 * Reference interfaces replaced (paths relative to the fisalt/GPA project):
 *   gpa_b200_forward  - DenseGPA.forward            src/gpa/attention.py:347-414
 *                       (block loop :376-405, lag block :299-345, token :264-297,
 *                        and the FLA GDN dispatch in gdn_scan src/gpa/ops.py:58-77)
 *   gpa_b200_backward - autograd through the above (FLA chunk_gated_delta_rule
 *                       backward plus ATen autograd of src/gpa/attention.py:161-345)
 *
 * Conventions: q, k [B,T,H,Dk] and v, out [B,T,H,Dv] are contiguous in the
 * input dtype (fp32 / bf16 / fp16).  Parameters, states and their gradients
 * are contiguous fp32 tensors with the reference's shapes
 * (src/gpa/attention.py:104-135, src/gpa/state.py:30-58).  Status codes:
 * 0 ok, 1 bad argument, 2 unsupported configuration, 3 CUDA launch failure,
 * 4 device timeout (a bounded wait inside a tensor-core kernel gave up; the
 * kernel returned without its result and the context stays usable).
 */
#ifndef GPA_B200_H
#define GPA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPA_B200_MAX_LEVELS 8
#define GPA_B200_MAX_EDGES 56

enum { GPA_B200_OK = 0, GPA_B200_BAD_ARGUMENT = 1, GPA_B200_UNSUPPORTED = 2,
       GPA_B200_LAUNCH_FAILURE = 3, GPA_B200_DEVICE_TIMEOUT = 4 };
enum { GPA_B200_F32 = 0, GPA_B200_BF16 = 1, GPA_B200_F16 = 2 };

/* Shapes and the scalar GPAConfig fields the core reads (src/gpa/attention.py:17-43). */
typedef struct GpaDims {
  int32_t batch, length, heads, key_dim, value_dim, levels;
  int32_t slots[GPA_B200_MAX_LEVELS];
  int32_t chunk_size;      /* 1 = exact token recurrence, 2..64 = lag blocks */
  int32_t chunk_offset;    /* GPAState.chunk_offset of the incoming cache */
  int32_t input_dtype;     /* GPA_B200_F32 / _BF16 / _F16 */
  int32_t positional_none; /* positional_mode == "none": zero decays */
  float read_scale, query_scale, beta_max;
  int32_t reader_mode;     /* dense reader: GPA_B200_READER_TANH (centred tanh,
                              src/gpa/attention.py:238-241), _PRODUCT
                              (paper_product_read, :231-234) or _MARGINAL
                              (product and relation_marginal, :235-236) */
  int32_t positional_moments; /* positional_mode == "moments": rotated queries and
                                 the per-level moment state (:277-283, :318-322) */
  int32_t position;        /* GPAState.position: absolute index of the call's first
                              token (rotary angles of positional moments) */
} GpaDims;

#define GPA_B200_READER_TANH 0
#define GPA_B200_READER_PRODUCT 1
#define GPA_B200_READER_MARGINAL 2

/* Parameter pointers (per-level lists by level, edges in the reference order
 * (i, j) for i != j, row-major).  The learned prefixes are not listed: they
 * enter through the incoming state. */
typedef struct GpaParams {
  const float* center[GPA_B200_MAX_LEVELS];       /* [H,M,Dk] */
  const float* route_weight[GPA_B200_MAX_LEVELS]; /* [H,M,M] */
  const float* query_weight[GPA_B200_MAX_LEVELS]; /* [H,Dk,M] */
  const float* route_up[GPA_B200_MAX_LEVELS];     /* [H,M,2M] */
  const float* route_down[GPA_B200_MAX_LEVELS];   /* [H,2M,M] */
  const float* gate_weight[GPA_B200_MAX_LEVELS];  /* [H,Dk,4] */
  const float* gate_bias[GPA_B200_MAX_LEVELS];    /* [H,4] */
  const float* residual_raw;       /* [L,H,2] */
  const float* count_gain_raw;     /* [L,H] */
  const float* route_mlp_gain;     /* [L,H] */
  const float* output_logits;      /* [L,H] */
  const float* edge_logits;        /* [E,H] */
  const float* relation_gain;      /* [L,H] */
  const float* relation_decay_raw; /* [E,H] */
  const float* relation_beta_raw;  /* [E,H] */
  const float* moment_gain;        /* [L,H] (positional moments; else unused) */
} GpaParams;

/* Same layout, writable: parameter gradients (accumulated with +=). */
typedef struct GpaParamGrads {
  float* center[GPA_B200_MAX_LEVELS];
  float* route_weight[GPA_B200_MAX_LEVELS];
  float* query_weight[GPA_B200_MAX_LEVELS];
  float* route_up[GPA_B200_MAX_LEVELS];
  float* route_down[GPA_B200_MAX_LEVELS];
  float* gate_weight[GPA_B200_MAX_LEVELS];
  float* gate_bias[GPA_B200_MAX_LEVELS];
  float* residual_raw;
  float* count_gain_raw;
  float* route_mlp_gain;
  float* output_logits;
  float* edge_logits;
  float* relation_gain;
  float* relation_decay_raw;
  float* relation_beta_raw;
  float* moment_gain;  /* NULL unless positional moments */
} GpaParamGrads;

/* Recurrent cache tensors, GPAState layout (src/gpa/state.py:30-58).
 * frozen_* are the lag-block residual snapshots; NULL when absent. */
typedef struct GpaStateRef {
  float* inner[GPA_B200_MAX_LEVELS];  /* A [B,H,Dk,M] */
  float* outer[GPA_B200_MAX_LEVELS];  /* B [B,H,M,Dv] */
  float* count[GPA_B200_MAX_LEVELS];  /* n [B,H,M] */
  float* relation[GPA_B200_MAX_EDGES];/* R [B,H,M_i,M_j] */
  float* frozen_inner[GPA_B200_MAX_LEVELS];
  float* frozen_outer[GPA_B200_MAX_LEVELS];
  float* moment[GPA_B200_MAX_LEVELS]; /* P [B,H,Dk,M]: positional moments (else NULL) */
} GpaStateRef;

/* Bytes of the forward's saved buffer (kept alive until gpa_b200_backward). */
size_t gpa_b200_saved_bytes(const GpaDims* dims);
/* Bytes of the backward scratch buffer. */
size_t gpa_b200_scratch_bytes(const GpaDims* dims);

/* Forward of one call: out [B,T,H,Dv]; state_out receives the final cache
 * (frozen_* written when (chunk_offset + T) % chunk_size != 0).
 * Replaces DenseGPA.forward (src/gpa/attention.py:347-414). */
int gpa_b200_forward(const GpaDims* dims, const GpaParams* params, const void* q, const void* k,
                     const void* v, const GpaStateRef* state_in, GpaStateRef* state_out,
                     void* out, void* saved, size_t saved_bytes, void* stream);

/* Backward of one forward call.  dstate_out holds the gradients of the
 * returned cache tensors (NULL members count as zero).  Writes dq, dk, dv
 * (input dtype), the incoming-cache gradients dstate_in (every member of
 * state_in that is non-NULL), and accumulates the parameter gradients. */
int gpa_b200_backward(const GpaDims* dims, const GpaParams* params, const GpaStateRef* state_in,
                      const void* saved, const void* dout, const GpaStateRef* dstate_out,
                      void* dq, void* dk, void* dv, GpaStateRef* dstate_in,
                      GpaParamGrads* dparams, void* scratch, size_t scratch_bytes, void* stream);

/* Forward of one call (same results as gpa_b200_forward) for callers that
 * cannot allocate device memory: code running inside another runtime's
 * stream capture or memory pool, or a decode loop whose memory is fixed up
 * front.  No counterpart in the reference, which allocates through PyTorch.
 * The workspace is a file-scope device array of gpa_b200_noalloc_capacity()
 * bytes (64 MiB) that every GPU loading this library holds until the process
 * exits; calls whose workspace would exceed it return GPA_B200_UNSUPPORTED.
 * The first call on a device looks the array's address up (with that device
 * current) and keeps it for the life of the process; make that first call before
 * any stream capture, and do not call this entry point on a device after its
 * primary context was destroyed (cudaDeviceReset), which would leave the kept
 * address stale.  Every call shares
 * the array and overwrites all of it that it reads, so nothing needs clearing,
 * but calls that overlap on the GPU (other streams, other threads) race.  The
 * array is reused by the next call, so this entry point has no backward. */
int gpa_b200_forward_noalloc(const GpaDims* dims, const GpaParams* params, const void* q,
                             const void* k, const void* v, const GpaStateRef* state_in,
                             GpaStateRef* state_out, void* out, void* stream);
size_t gpa_b200_noalloc_capacity(void);

/* One-token decode step of a lag-block cache (chunk_size >= 2; dims->length == 1),
 * replacing a one-token DenseGPA.forward call (src/gpa/attention.py:347-414 with
 * T = 1, which runs _block_segment :299-345 on a one-token block).  The cache is
 * updated IN PLACE (state->frozen_* required: the snapshots of the current lag
 * block, written by this call when the token opens a block).  offset points to three
 * device int32: offset[0] is the cache's chunk_offset, advanced to
 * (offset[0] + 1) % chunk_size on the device; offset[1] is the step's completion
 * counter, which must be 0 before the first step and is left at 0 by every step
 * (steps on the same offset buffer must not overlap on the GPU); offset[2] is the
 * cache's position (GPAState.position), advanced by one (the rotary angle of
 * positional moments).  dims->chunk_offset and dims->position are ignored.  out: [B,1,H,Dv] in the input dtype.  One kernel launch, stream-ordered,
 * allocates nothing and never synchronizes with the host, so a sequence of steps can
 * be captured in a CUDA graph.  Widths must be multiples of 4. */
int gpa_b200_step(const GpaDims* dims, const GpaParams* params, const void* q, const void* k,
                  const void* v, const GpaStateRef* state, int32_t* offset, void* out,
                  void* stream);

/* Diagnostics: copy the per-level post-MLP routes of a forward call out of its
 * saved buffer into routes[j] ([B,T,H,M_j], input dtype).  Replaces the
 * return_diagnostics routes of DenseGPA.forward (src/gpa/attention.py:407-413). */
int gpa_b200_routes(const GpaDims* dims, const void* saved, void* const* routes, void* stream);

/* Device status of the kernels that wait on mbarriers, the tensor-core kernels and
 * the decode step's bulk state loads (no counterpart in the reference): 0, or
 * GPA_B200_DEVICE_TIMEOUT once a bounded wait inside one of them gave up since the
 * last clear (that kernel returned without a usable result).  Reads the device
 * words synchronously (the device must be current); clear != 0 resets them.  -1 if
 * a read failed. */
int gpa_b200_device_status(int clear);

/* Self-test of the tensor-core building blocks (no counterpart in the reference):
 * one CTA computes D = A B on the 5th-generation tensor cores (tcgen05.mma, bf16
 * operands in shared memory, fp32 accumulator in tensor memory).  A [M x Kd] and
 * B [Kd x N] are row-major bf16 device arrays, D [M x N] fp32; mma_m (64 or 128)
 * is the instruction's M (rows >= M are zero); a_mn / b_mn select the MN-major
 * operand layouts (b_mn == 2: B stored as its own K-major tile, rows k, and
 * read through an MN-major view of it).  flags: GPA_B200_UMMA_BULK_A reads A
 * instead from A_tiled, its 128-row K-major or MN-major shared-memory image, by
 * one bulk (TMA) copy; GPA_B200_UMMA_LD16 (mma_m 64, N a multiple of 16) reads D
 * back through the 16-lane tcgen05.ld shape instead of the 32-lane one.  *status
 * (device int) is set to GPA_B200_DEVICE_TIMEOUT if a wait gave up.  Returns
 * GPA_B200_UNSUPPORTED for shapes outside M <= mma_m, 16 <= N <= 256,
 * 16 <= Kd <= 128 (multiples of 16), or unknown flags. */
#define GPA_B200_UMMA_BULK_A 1
#define GPA_B200_UMMA_LD16 2
int gpa_b200_umma_selftest(int M, int mma_m, int N, int Kd, int a_mn, int b_mn, int flags,
                           const void* A, const void* B, const void* A_tiled, float* D,
                           int* status, void* stream);

/* Message of the last failure on the calling thread (0 if none). */
int gpa_b200_last_error(char* buf, size_t len);

/* ABI version of this header: 2 (GpaDims.reader_mode, positional_moments and
 * position; GpaParams / GpaParamGrads.moment_gain; GpaStateRef.moment; a third
 * offset word of gpa_b200_step). */
int gpa_b200_abi_version(void);

/* Kernel accounting (no counterpart in the reference, which has no native
 * code): the number of kernels this library has launched in this process, and
 * optional per-kernel device timing with CUDA events on the launch streams.
 * Profiling is off by default; profile_stop synchronises on the recorded
 * events and writes {"kernel": [launches, total_ms], ...} as JSON into buf. */
long long gpa_b200_launch_count(void);
int gpa_b200_profile_start(void);
int gpa_b200_profile_stop(char* buf, size_t len);

#ifdef __cplusplus
}
#endif
#endif /* GPA_B200_H */
