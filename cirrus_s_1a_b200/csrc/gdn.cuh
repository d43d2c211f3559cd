// Internal launch interface of the Gated DeltaNet step (gdn.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

struct GdnParams {
  const float* proj;   // in_proj output, row b*T + t, stride ldp: q | k | v at channel offsets, gate, a, b
  int ldp;
  int off_gate, off_a, off_b;
  const float* conv_w;
  const float* A_log;
  const float* dt_bias;
  const float* o_norm;
  float* state;        // sequence 0 of this layer: [H][Dk][Dv]
  int64_t state_stride;
  float* conv;         // sequence 0 of this layer: [KC-1][C]
  int64_t conv_stride;
  float* snap_state;   // per-token snapshots (null = off): + t * snap_state_t, same offsets as state
  int64_t snap_state_t;
  float* snap_conv;    // + t * snap_conv_t, same offsets as conv
  int64_t snap_conv_t;
  float* out;          // [batch*T][ldo]
  int ldo;
  int batch, T, H, Dk, Dv, C, KC;
  float eps, scale;
};

size_t gdn_smem_bytes(int Dk, int Dv);
int launch_gdn_step(const GdnParams& p, cudaStream_t st);

}  // namespace cb
