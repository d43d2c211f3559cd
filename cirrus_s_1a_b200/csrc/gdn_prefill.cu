// Short causal conv of the Gated DeltaNet over a prompt chunk
// (ShortConv.forward, cirrus/model/layers.py:95-104): for every channel c of
// every sequence, y_t = sum_j w[c][j] * xx[t + j] over xx = [window (KC - 1
// previous inputs); x_0 .. x_{T-1}], then silu; the window keeps the last
// KC - 1 inputs.  One thread per (sequence, channel) walks the chunk's tokens;
// for a fixed token the threads of a warp read consecutive channels.
#include "common.cuh"
#include "gdn.cuh"

namespace cb {
namespace {

constexpr int kConvThreads = 256;

__global__ void __launch_bounds__(kConvThreads) gdn_conv_kernel(const float* __restrict__ proj, int ldp,
                                                               const float* __restrict__ conv_w, float* conv,
                                                               int64_t conv_stride, int T, int C,
                                                               float* __restrict__ out, int ldo) {
  const int c = blockIdx.x * kConvThreads + threadIdx.x, b = blockIdx.y;
  if (c >= C) return;
  const float4 w = *reinterpret_cast<const float4*>(conv_w + (int64_t)c * 4);
  float* win = conv + (int64_t)b * conv_stride + c;
  float c0 = win[0], c1 = win[C], c2 = win[2 * (int64_t)C];
  const float* x = proj + (int64_t)b * T * ldp + c;
  float* y = out + (int64_t)b * T * ldo + c;
#pragma unroll 8
  for (int t = 0; t < T; ++t) {
    const float xt = x[(int64_t)t * ldp];
    float acc = c0 * w.x;
    acc += c1 * w.y;
    acc += c2 * w.z;
    acc += xt * w.w;
    y[(int64_t)t * ldo] = silu(acc);
    c0 = c1;
    c1 = c2;
    c2 = xt;
  }
  win[0] = c0;
  win[C] = c1;
  win[2 * (int64_t)C] = c2;
}

}  // namespace

int launch_gdn_conv(const float* proj, int ldp, const float* conv_w, float* conv, int64_t conv_stride, int batch,
                    int T, int C, int KC, float* out, int ldo, cudaStream_t st) {
  if (KC != 4 || T < 1 || batch < 1 || C < 1) return CB_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(conv_w) & 15) return CB_ERR_ARG;
  gdn_conv_kernel<<<dim3(ceil_div(C, kConvThreads), batch), kConvThreads, 0, st>>>(proj, ldp, conv_w, conv,
                                                                                  conv_stride, T, C, out, ldo);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb
