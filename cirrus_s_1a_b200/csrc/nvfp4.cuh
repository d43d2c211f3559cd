// Internal launch interface of the NVFP4 kernels (nvfp4.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

enum { PRE_NONE = 0, PRE_RMSNORM = 1, PRE_SWIGLU = 2 };
enum { EPI_STORE = 0, EPI_ADD = 1 };

// y[m, n] (=|+=) tensor_scale * sum_k W[n, k] * pre(x)[m, k]
//   PRE_RMSNORM: pre(x) = x * rsqrt(mean(x^2) + eps) * norm_w     (layers.py:39-44)
//   PRE_SWIGLU:  pre(x)[k] = silu(x[k]) * x[K + k]                 (layers.py:52-54)
struct GemvParams {
  const uint8_t* tiles;
  const float* tile_scale;
  int rows;       // padded rows of W (multiple of 16)
  int K;
  const float* x;
  int ldx;
  int m_rows;
  const float* norm_w;
  float eps;
  float* y;
  int ldy;
  int rows_out;   // rows of y written (<= rows)
  int ksplit;     // warps sharing a row pair over K (1, 2, 4; set by the launcher, 0 = 1)
};

int launch_gemv(const GemvParams& p, int pre, int epi, cudaStream_t st);
int launch_embed(const CbMatrix& tab, int vocab, const int64_t* ids, int64_t ids_ld, int batch, int T, int c0,
                 float* h, int32_t* status, cudaStream_t st);
int launch_argmax(const float* x, int rows, int n, int ld, int32_t* out, cudaStream_t st);

}  // namespace cb
