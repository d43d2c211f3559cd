// Internal launch interface of the tensor-core NVFP4 GEMM (gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

enum { GEMM_PRE_NONE = CB_GEMM_PRE_NONE, GEMM_PRE_RMSNORM = CB_GEMM_PRE_RMSNORM };
enum { GEMM_EPI_STORE = CB_GEMM_EPI_STORE, GEMM_EPI_ADD = CB_GEMM_EPI_ADD, GEMM_EPI_SWIGLU = CB_GEMM_EPI_SWIGLU };

// y[m][r] (=, +=) tile_scale * sum_k W[r][k] * pre(x)[m][k] for m < m_rows:
//   GEMM_PRE_RMSNORM  pre(x) = x * rsqrt(mean(x^2) + eps) * norm_w      (layers.py:39-44)
//   GEMM_EPI_SWIGLU   W = [gate; up] (2F rows), y[m][r] = silu(g_r) * u_r for r < F  (layers.py:52-54)
struct GemmParams {
  const uint8_t* tiles;
  const float* tile_scale;
  int rows;        // rows of W (multiple of 16)
  int K;           // multiple of 64 (RMSNorm inputs: any such K)
  const float* x;  // [m_rows][ldx] float32, 16-byte aligned rows
  int ldx, m_rows;
  int pre;
  const float* norm_w;
  float eps;
  float* y;
  int ldy, rows_out, epi;
  uint8_t* xb;      // scratch for the prepared inputs (gemm_scratch_bytes)
  size_t xb_bytes;
  int32_t* status;  // CB_ERR_TIMEOUT when a bounded wait gives up (may be null)
};

// Bytes of prepared-input scratch for m_rows token rows of K inputs.
size_t gemm_scratch_bytes(int K, int m_rows);
int launch_gemm(const GemmParams& p, cudaStream_t st);

}  // namespace cb
