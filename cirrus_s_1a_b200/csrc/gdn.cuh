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

// Chunked form of the recurrence (gdn_chunk.cu), Dk = Dv = 64.
// Token (b, t) of head h reads q/k/v at base + (b * T + t) * ld_qkv + h * 64 and
// writes its output at out + (b * T + t) * ld_out + h * 64.
//   standalone (cb_gdn_chunk_prefill): q, k, v [B][T][H][64], g and beta [B][T][H], raw o out;
//   model (a prompt chunk of cb_forward): q | k | v after the short conv (channels
//     of one row), the decay and beta computed here from the raw a / b projections
//     (layers.py:161-162), q and k L2-normalised here (layers.py:158-159), and the
//     output RMS-normalised over Dv times o_norm times silu(gate) (layers.py:171).
struct GdnChunkParams {
  const float *q, *k, *v;
  int64_t ld_qkv;
  const float *g, *beta;              // standalone: [B][T][H]
  const float *a_raw, *b_raw;         // model: row (b, t) + h, stride ld_ab
  int64_t ld_ab;
  const float *A_log, *dt_bias;       // model: [H]
  float* state;                       // [H][Dk][Dv] per sequence, in/out
  int64_t state_seq;                  // sequence stride of state (elements)
  float* out;
  int64_t ld_out;
  const float* gate;                  // model: row (b, t) + h * Dv, stride ld_gate (null: raw o)
  int64_t ld_gate;
  const float* o_norm;                // model: [Dv]
  float eps;
  int B, T, H;
  float scale;
};

int launch_gdn_chunk(const GdnChunkParams& p, cudaStream_t st);

// Prompt chunks: the short conv over T tokens of every channel (gdn_prefill.cu):
// proj rows (b * T + t, stride ldp) -> silu(conv) rows of C channels (stride ldo),
// the conv window of each sequence advanced by T tokens.
int launch_gdn_conv(const float* proj, int ldp, const float* conv_w, float* conv, int64_t conv_stride, int batch,
                    int T, int C, int KC, float* out, int ldo, cudaStream_t st);

}  // namespace cb
