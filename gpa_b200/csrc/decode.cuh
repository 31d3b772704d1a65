// One-token decode step (decode.cu): host interface used by the C ABI (api.cu).
#pragma once
#include "../../include/gpa_b200.h"
#include "common.cuh"
#include "level.cuh"

namespace gpa {

struct StepArgs {
  int U, H, D, Dv, L, E;
  int C;  // lag-block length (>= 2)
  int M[kMaxLevels];
  int es[kMaxEdges], ed[kMaxEdges];
  int dt, pos_none;
  int reader;  // GPA_B200_READER_* (dense reader form)
  int moments;  // positional moments (rotated query, per-level moment state)
  float query_scale, beta_max, read_scale;
  GpaParams p;
  GpaStateRef s;  // updated in place; frozen_* required
  const void *q, *k, *v;
  void* out;
  int* offset;  // device int[3]: the cache's chunk offset (advanced by the step), the step's
                // completion counter (0 between steps) and the cache position (advanced)
};

// Shared memory the step kernel needs for these widths (bytes).
size_t decode_step_smem(const StepArgs& a);
// Stream-ordered, one kernel (its last CTA advances the offset).  No allocation, no host
// synchronization (capturable in a CUDA graph).
cudaError_t launch_decode_step(const StepArgs& a, cudaStream_t st);
// device status word of the step kernel (GPA_B200_DEVICE_TIMEOUT after a bulk-load wait gave
// up); synchronous read, optionally clearing it; -1 if the read failed
int decode_device_status(bool clear);

}  // namespace gpa
