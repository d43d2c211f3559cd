// Device helpers shared by the cirrus-b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

// Host-side count of kernel launches issued by this library (cb_launch_count).
void count_launch();

// Per-device launch state (devstate.cu): the dynamic shared-memory opt-in of a
// kernel on the current device (CB_OK or CB_ERR_CUDA), its resident CTAs per SM
// at that size, and the current device's SM count.
int ensure_smem_attr(const void* fn, int bytes);
int resident_ctas(const void* fn, int threads, int smem_bytes);
int num_sms();
// Clusters of `cluster` CTAs of a kernel that fit on the current device at once
// (cudaOccupancyMaxActiveClusters, cached per kernel and device; 0 on error).
int resident_clusters(const void* fn, int threads, int smem_bytes, int cluster);
// Whether a cooperative launch may carry a cluster dimension on the current
// device (true until a launch of that form has been refused there).
bool cooperative_clusters_ok();
void note_cooperative_clusters_refused();

constexpr int kTileRows = CB_TILE_ROWS;
constexpr int kWarp = 32;

__host__ __device__ inline int64_t tile_bytes(int K) { return (int64_t)kTileRows * (K / 2 + K / 16); }
__host__ __device__ inline int pad16(int x) { return (x + 15) / 16 * 16; }
__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// E4M3 byte -> float (exact: every E4M3 value is a normal half).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// float -> E4M3 byte, round to nearest even, saturating to +-448.
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

// Two E2M1 codes (low nibble -> .x) to two exact floats.
__device__ __forceinline__ float2 e2m1x2_to_f32x2(uint32_t byte) {
  __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)(byte & 0xFF), __NV_E2M1);
  return __half22float2(__half2(h));
}

// E2M1 code of q: nearest of {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even
// code, saturating; bit 3 carries the sign bit of q.
__device__ __forceinline__ uint32_t e2m1_encode(float q) {
  const uint32_t sign = (__float_as_uint(q) >> 31) << 3;
  const float a = fabsf(q);
  uint32_t m;
  if (a <= 0.25f) m = 0;
  else if (a < 0.75f) m = 1;
  else if (a <= 1.25f) m = 2;
  else if (a < 1.75f) m = 3;
  else if (a <= 2.5f) m = 4;
  else if (a < 3.5f) m = 5;
  else if (a <= 5.0f) m = 6;
  else m = 7;
  return sign | m;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
// torch.nn.functional.softplus(beta=1, threshold=20)
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ uint16_t f32_to_bf16(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float bf16_to_f32(uint32_t b) { return __uint_as_float((b & 0xFFFFu) << 16); }

// Orderable key of a float score: larger score <-> larger key; -0 maps to +0.
__device__ __forceinline__ uint32_t score_key(float s) {
  uint32_t u = __float_as_uint(s + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide sum over all threads (blockDim.x multiple of 32, <= 1024).
// `red` is shared scratch of >= 33 floats; the result is returned to every thread.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Partial interleaved RoPE (layers.py:72-82) on one pair (x[2j], x[2j+1]) at position p.
__device__ __forceinline__ void rope_pair(float& x1, float& x2, int p, float inv_freq_j) {
  const float f = (float)p * inv_freq_j;
  float s, c;
  sincosf(f, &s, &c);
  const float a = x1 * c - x2 * s;
  const float b = x1 * s + x2 * c;
  x1 = a;
  x2 = b;
}

// Device status word helpers (first int of the workspace).
__device__ __forceinline__ void set_status(int32_t* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace cb
