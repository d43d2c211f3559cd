// Short causal conv of the Gated DeltaNet over a prompt chunk
// (ShortConv.forward, cirrus/model/layers.py:95-104): for every channel c of
// every sequence, y_t = sum_j w[c][j] * xx[t + j] over xx = [window (KC - 1
// previous inputs); x_0 .. x_{T-1}], then silu; the window keeps the last
// KC - 1 inputs.  One thread per (sequence, channel, group of kConvTok
// tokens): its inputs (the group and the KC - 1 before it) are all loaded
// before the first output is formed, so the group costs one memory round trip.
// The thread of the first group reads the old window and writes the new one.
#include "common.cuh"
#include "gdn.cuh"

namespace cb {
namespace {

constexpr int kConvThreads = 256;
constexpr int kConvTok = 16;

__global__ void __launch_bounds__(kConvThreads) gdn_conv_kernel(const float* __restrict__ proj, int ldp,
                                                               const float* __restrict__ conv_w, float* conv,
                                                               int64_t conv_stride, int T, int C,
                                                               float* __restrict__ out, int ldo) {
  const int c = blockIdx.x * kConvThreads + threadIdx.x, grp = blockIdx.y, b = blockIdx.z;
  if (c >= C) return;
  const int t0 = grp * kConvTok, n = min(kConvTok, T - t0);
  const float4 w = *reinterpret_cast<const float4*>(conv_w + (int64_t)c * 4);
  float* win = conv + (int64_t)b * conv_stride + c;
  const float* x = proj + (int64_t)b * T * ldp + c;
  // xx[0..2] = the three inputs before t0, xx[3 + i] = input t0 + i
  float xx[kConvTok + 3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = t0 - 3 + j;
    xx[j] = t >= 0 ? x[(int64_t)t * ldp] : win[(int64_t)(3 + t) * C];
  }
#pragma unroll
  for (int i = 0; i < kConvTok; ++i) xx[3 + i] = i < n ? x[(int64_t)(t0 + i) * ldp] : 0.0f;
  float* y = out + (int64_t)b * T * ldo + c;
#pragma unroll
  for (int i = 0; i < kConvTok; ++i) {
    if (i < n) {
      float acc = xx[i] * w.x;
      acc += xx[i + 1] * w.y;
      acc += xx[i + 2] * w.z;
      acc += xx[i + 3] * w.w;
      y[(int64_t)(t0 + i) * ldo] = silu(acc);
    }
  }
  if (grp == 0) {
    // the window after the chunk: inputs T-3, T-2, T-1 (from the old window when T < 3)
    float nw[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int t = T - 3 + j;
      // t < 0 only when T < 3: input t is the old window entry 3 + t, i.e. xx[3 + t]
      nw[j] = t >= 0 ? x[(int64_t)t * ldp] : (t == -3 ? xx[0] : (t == -2 ? xx[1] : xx[2]));
    }
    win[0] = nw[0];
    win[C] = nw[1];
    win[2 * (int64_t)C] = nw[2];
  }
}

}  // namespace

int launch_gdn_conv(const float* proj, int ldp, const float* conv_w, float* conv, int64_t conv_stride, int batch,
                    int T, int C, int KC, float* out, int ldo, cudaStream_t st) {
  if (KC != 4 || T < 1 || batch < 1 || C < 1) return CB_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(conv_w) & 15) return CB_ERR_ARG;
  const dim3 grid(ceil_div(C, kConvThreads), ceil_div(T, kConvTok), batch);
  gdn_conv_kernel<<<grid, kConvThreads, 0, st>>>(proj, ldp, conv_w, conv, conv_stride, T, C, out, ldo);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb
