// NVFP4 weight path: quantiser, tile packer, CUDA-core GEMV (warp per row
// pair, warp-shuffle reduction), embedding gather and row argmax.
//
// Format: E2M1 codes with an E4M3 scale per 16 elements and a float32 tensor
// scale (cirrus/perf/bench_kernels.cu:141-145).  Weights are stored in
// 16-row tiles: [16 rows x K/2 code bytes][16 rows x K/16 scale bytes], so a
// tile is one contiguous 9*K-byte block that a single bulk copy can move.
#include <algorithm>

#include "common.cuh"
#include "nvfp4.cuh"

namespace cb {

// ------------------------------------------------------------- quantiser
__global__ void quantize_kernel(const float* __restrict__ w, int n, int k, float tscale, uint8_t* __restrict__ codes,
                                uint8_t* __restrict__ scales) {
  const int64_t nb = (int64_t)n * (k / 16);
  const int64_t bi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (bi >= nb) return;
  const int row = (int)(bi / (k / 16)), kb = (int)(bi % (k / 16));
  const float* src = w + (int64_t)row * k + kb * 16;
  float v[16];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = __fdiv_rn(src[i], tscale);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  const uint8_t sc = f32_to_e4m3(__fdiv_rn(amax, 6.0f));
  const float sv = e4m3_to_f32(sc);
  uint8_t* dst = codes + (int64_t)row * (k / 2) + kb * 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = e2m1_encode(sv > 0.0f ? __fdiv_rn(v[2 * i], sv) : 0.0f);
    const uint32_t hi = e2m1_encode(sv > 0.0f ? __fdiv_rn(v[2 * i + 1], sv) : 0.0f);
    dst[i] = (uint8_t)(lo | (hi << 4));
  }
  scales[(int64_t)row * (k / 16) + kb] = sc;
}

__global__ void pack_tiles_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, int n, int k,
                                  uint8_t* __restrict__ tiles) {
  const int64_t tb = tile_bytes(k);
  const int64_t total = (int64_t)ceil_div(n, kTileRows) * tb;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / tb, off = i % tb;
    const int64_t code_bytes = (int64_t)kTileRows * (k / 2);
    uint8_t val;
    if (off < code_bytes) {
      const int row = (int)(t * kTileRows + off / (k / 2)), col = (int)(off % (k / 2));
      val = row < n ? codes[(int64_t)row * (k / 2) + col] : 0;
    } else {
      const int64_t o2 = off - code_bytes;
      const int row = (int)(t * kTileRows + o2 / (k / 16)), col = (int)(o2 % (k / 16));
      val = row < n ? scales[(int64_t)row * (k / 16) + col] : 0;
    }
    tiles[i] = val;
  }
}

// ------------------------------------------------------------------ GEMV
// One warp computes two adjacent weight rows; lane l owns the 8-code chunks
// l, l+32, ... of the row (one 32-bit code word and half a scale byte each),
// so a warp reads 128 contiguous code bytes per step.  The input rows sit in
// shared memory after the fused pre-op (RMSNorm, SwiGLU or copy).
constexpr int kGemvThreads = 256;
constexpr int kGemvUnroll = 4;

template <int EPI>
__device__ __forceinline__ void gemv_store(const GemvParams& p, int m, int r0, float a0, float a1) {
  float* yr = p.y + (int64_t)m * p.ldy;
  if (r0 < p.rows_out) {
    if (EPI == EPI_ADD) yr[r0] += a0;
    else yr[r0] = a0;
  }
  if (r0 + 1 < p.rows_out) {
    if (EPI == EPI_ADD) yr[r0 + 1] += a1;
    else yr[r0 + 1] = a1;
  }
}

template <int M, int PRE, int EPI>
__global__ void __launch_bounds__(kGemvThreads) gemv_nvfp4_kernel(GemvParams p) {
  extern __shared__ __align__(16) float xs[];  // [M][K]
  __shared__ float rs[M];
  const int K = p.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (PRE == PRE_RMSNORM) {
    for (int m = warp; m < M; m += kGemvThreads / 32) {
      float ss = 0.0f;
      if (m < p.m_rows)
        for (int k = lane; k < K; k += 32) {
          const float v = p.x[(int64_t)m * p.ldx + k];
          ss += v * v;
        }
      ss = warp_sum(ss);
      if (lane == 0) rs[m] = rsqrtf(ss / (float)K + p.eps);
    }
    __syncthreads();
  }
  // Stage the inputs: 16-byte vectors, four in flight per thread (a loop of
  // single loads would wait out one memory latency per element it stages).
  const bool vec = ((reinterpret_cast<uintptr_t>(p.x) | (uintptr_t)p.ldx * 4u) & 15u) == 0 &&
                   (PRE != PRE_RMSNORM || (reinterpret_cast<uintptr_t>(p.norm_w) & 15u) == 0);
  if (vec) {
    const int K4 = K >> 2, n4 = M * K4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * kGemvThreads) {
      float4 xa[4], xb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * kGemvThreads, m = i / K4, k4 = i - m * K4;
        xa[j] = xb[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < n4 && m < p.m_rows) {
          const float4* xr = reinterpret_cast<const float4*>(p.x + (int64_t)m * p.ldx);
          xa[j] = xr[k4];
          if (PRE == PRE_SWIGLU) xb[j] = xr[K4 + k4];
          else if (PRE == PRE_RMSNORM) xb[j] = reinterpret_cast<const float4*>(p.norm_w)[k4];
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * kGemvThreads, m = i / K4;
        if (i < n4) {
          float4 v = xa[j];
          if (m < p.m_rows) {
            const float4 a = xa[j], b = xb[j];
            if (PRE == PRE_RMSNORM) {
              const float r = rs[m];
              v = make_float4(a.x * r * b.x, a.y * r * b.y, a.z * r * b.z, a.w * r * b.w);
            } else if (PRE == PRE_SWIGLU) {
              v = make_float4(silu(a.x) * b.x, silu(a.y) * b.y, silu(a.z) * b.z, silu(a.w) * b.w);
            }
          }
          reinterpret_cast<float4*>(xs)[i] = v;
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < M * K; i += kGemvThreads) {
      const int m = i / K, k = i - m * K;
      float v = 0.0f;
      if (m < p.m_rows) {
        const float* xr = p.x + (int64_t)m * p.ldx;
        if (PRE == PRE_RMSNORM) v = xr[k] * rs[m] * p.norm_w[k];
        else if (PRE == PRE_SWIGLU) v = silu(xr[k]) * xr[K + k];
        else v = xr[k];
      }
      xs[i] = v;
    }
  }
  __syncthreads();

  const int kc = K >> 3;
  const int64_t tb = tile_bytes(K);
  // S warps share a row pair, each over kc / S of the 8-code chunks; their
  // partial sums meet in shared memory and are added in part order.
  const int S = M >= 4 && p.ksplit > 1 ? p.ksplit : 1;  // 1 and 2 row launches compile without the split
  const int ppc = (kGemvThreads / 32) / S;  // row pairs per CTA pass
  const int slot = warp % ppc, part = warp / ppc;
  const int c_lo = part * (kc / S), c_hi = c_lo + kc / S;
  __shared__ float red[kGemvThreads / 32][2][M];
  // rows % (2 * ppc) == 0, so every pair of a pass exists and the pass count is CTA-uniform
  for (int base = blockIdx.x * ppc * 2; base < p.rows; base += gridDim.x * ppc * 2) {
    const int r0 = base + slot * 2;
    const uint8_t* tile = p.tiles + (int64_t)(r0 >> 4) * tb;
    const int rr = r0 & 15;
    const uint32_t* cw0 = reinterpret_cast<const uint32_t*>(tile + rr * (K / 2));
    const uint32_t* cw1 = reinterpret_cast<const uint32_t*>(tile + (rr + 1) * (K / 2));
    const uint8_t* sb0 = tile + kTileRows * (K / 2) + rr * (K / 16);
    const uint8_t* sb1 = sb0 + K / 16;
    float acc0[M], acc1[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc0[m] = acc1[m] = 0.0f;

    for (int cbase = c_lo; cbase < c_hi; cbase += 32 * kGemvUnroll) {
      uint32_t w0[kGemvUnroll], w1[kGemvUnroll], s0[kGemvUnroll], s1[kGemvUnroll];
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = cbase + u * 32 + lane;
        const bool ok = c < c_hi;
        w0[u] = ok ? __ldg(cw0 + c) : 0u;
        w1[u] = ok ? __ldg(cw1 + c) : 0u;
        s0[u] = ok ? __ldg(sb0 + (c >> 1)) : 0u;
        s1[u] = ok ? __ldg(sb1 + (c >> 1)) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = cbase + u * 32 + lane;
        if (c < c_hi) {
          const float sc0 = e4m3_to_f32(s0[u]), sc1 = e4m3_to_f32(s1[u]);
          float2 f0[4], f1[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            f0[j] = e2m1x2_to_f32x2(w0[u] >> (8 * j));
            f1[j] = e2m1x2_to_f32x2(w1[u] >> (8 * j));
          }
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float4 xa = *reinterpret_cast<const float4*>(xs + m * K + c * 8);
            const float4 xb = *reinterpret_cast<const float4*>(xs + m * K + c * 8 + 4);
            float p0 = f0[0].x * xa.x;
            p0 = fmaf(f0[0].y, xa.y, p0);
            p0 = fmaf(f0[1].x, xa.z, p0);
            p0 = fmaf(f0[1].y, xa.w, p0);
            p0 = fmaf(f0[2].x, xb.x, p0);
            p0 = fmaf(f0[2].y, xb.y, p0);
            p0 = fmaf(f0[3].x, xb.z, p0);
            p0 = fmaf(f0[3].y, xb.w, p0);
            float p1 = f1[0].x * xa.x;
            p1 = fmaf(f1[0].y, xa.y, p1);
            p1 = fmaf(f1[1].x, xa.z, p1);
            p1 = fmaf(f1[1].y, xa.w, p1);
            p1 = fmaf(f1[2].x, xb.x, p1);
            p1 = fmaf(f1[2].y, xb.y, p1);
            p1 = fmaf(f1[3].x, xb.z, p1);
            p1 = fmaf(f1[3].y, xb.w, p1);
            acc0[m] = fmaf(p0, sc0, acc0[m]);
            acc1[m] = fmaf(p1, sc1, acc1[m]);
          }
        }
      }
    }
    const float ts = p.tile_scale[r0 >> 4];
    if (S == 1) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float a0 = warp_sum(acc0[m]) * ts;
        const float a1 = warp_sum(acc1[m]) * ts;
        if (lane == 0 && m < p.m_rows) gemv_store<EPI>(p, m, r0, a0, a1);
      }
    } else {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float a0 = warp_sum(acc0[m]), a1 = warp_sum(acc1[m]);
        if (lane == 0) {
          red[warp][0][m] = a0;
          red[warp][1][m] = a1;
        }
      }
      __syncthreads();
      if (part == 0 && lane == 0) {
        for (int m = 0; m < p.m_rows; ++m) {
          float a0 = red[slot][0][m], a1 = red[slot][1][m];
          for (int q = 1; q < S; ++q) {
            a0 += red[q * ppc + slot][0][m];
            a1 += red[q * ppc + slot][1][m];
          }
          gemv_store<EPI>(p, m, r0, a0 * ts, a1 * ts);
        }
      }
      __syncthreads();
    }
  }
}

// K split of a matrix for launches of 4..16 input rows: doubled (up to 4)
// while its 16-row tiles leave SMs idle and the split CTAs still fit one wave
// at 16 input rows.  Launches of 1 or 2 rows keep S = 1: there the shared-
// memory meeting of the partial sums costs more than the extra CTAs save
// (74-matrix weight stream at M = 1: 290 us unsplit, 304 us split; at M = 16:
// 1006 us unsplit, 965 us split).
static int gemv_ksplit(int rows, int K) {
  const int kc = K / 8, tiles = rows / 16;
  const size_t smem16 = (size_t)16 * K * sizeof(float) + 2048;
  const int per_sm = std::max(1, (int)((size_t)227 * 1024 / smem16));
  int S = 1;
  while (S < 4 && tiles * S < num_sms() && tiles * S * 2 <= num_sms() * per_sm && kc % (2 * S) == 0) S *= 2;
  return S;
}

template <int M, int PRE, int EPI>
static int launch_gemv_m(const GemvParams& p, cudaStream_t st) {
  const size_t smem = (size_t)M * p.K * sizeof(float);
  if (ensure_smem_attr((const void*)gemv_nvfp4_kernel<M, PRE, EPI>, 200 * 1024) != CB_OK) return CB_ERR_CUDA;
  const int S = M >= 4 ? gemv_ksplit(p.rows, p.K) : 1;
  const int pairs_per_cta = kGemvThreads / 32 / S;
  const int want = ceil_div(p.rows / 2, pairs_per_cta);
  const int grid = std::max(1, std::min(want, num_sms() * 4));
  GemvParams q = p;
  q.ksplit = S;
  gemv_nvfp4_kernel<M, PRE, EPI><<<grid, kGemvThreads, smem, st>>>(q);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

template <int PRE, int EPI>
static int launch_gemv_pe(GemvParams p, cudaStream_t st) {
  int rc = CB_OK;
  // up to 16 rows per launch (the input rows are staged in shared memory:
  // 16 x K floats, 128 KB at K = 2048), so a batch reads each matrix M / 16 times
  const int step = p.K <= 2048 ? 16 : 8;
  for (int m0 = 0; m0 < p.m_rows && rc == CB_OK; m0 += step) {
    GemvParams q = p;
    q.m_rows = std::min(step, p.m_rows - m0);
    q.x = p.x + (int64_t)m0 * p.ldx;
    q.y = p.y + (int64_t)m0 * p.ldy;
    if (q.m_rows == 1) rc = launch_gemv_m<1, PRE, EPI>(q, st);
    else if (q.m_rows == 2) rc = launch_gemv_m<2, PRE, EPI>(q, st);
    else if (q.m_rows <= 4) rc = launch_gemv_m<4, PRE, EPI>(q, st);
    else if (q.m_rows <= 8) rc = launch_gemv_m<8, PRE, EPI>(q, st);
    else rc = launch_gemv_m<16, PRE, EPI>(q, st);
  }
  return rc;
}

int launch_gemv(const GemvParams& p, int pre, int epi, cudaStream_t st) {
  if (!p.tiles || !p.tile_scale || !p.x || !p.y || p.K <= 0 || p.K % 16 || p.rows % kTileRows || p.m_rows <= 0 ||
      p.rows_out > p.rows || (pre == PRE_RMSNORM && !p.norm_w))
    return CB_ERR_ARG;
  if (p.K > 6144) return CB_ERR_SHAPE;
  if (pre == PRE_RMSNORM) return epi == EPI_ADD ? launch_gemv_pe<PRE_RMSNORM, EPI_ADD>(p, st)
                                                : launch_gemv_pe<PRE_RMSNORM, EPI_STORE>(p, st);
  if (pre == PRE_SWIGLU) return epi == EPI_ADD ? launch_gemv_pe<PRE_SWIGLU, EPI_ADD>(p, st)
                                               : launch_gemv_pe<PRE_SWIGLU, EPI_STORE>(p, st);
  return epi == EPI_ADD ? launch_gemv_pe<PRE_NONE, EPI_ADD>(p, st) : launch_gemv_pe<PRE_NONE, EPI_STORE>(p, st);
}

// ------------------------------------------------------------- embedding
__global__ void embed_kernel(const uint8_t* __restrict__ tiles, const float* __restrict__ tile_scale, int K, int vocab,
                             const int64_t* __restrict__ ids, int64_t ids_ld, int T, int c0, float* __restrict__ h,
                             int32_t* status) {
  const int r = blockIdx.x, b = r / T, t = r % T;
  const int64_t id = ids[(int64_t)b * ids_ld + c0 + t];
  float* out = h + (int64_t)r * K;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(status, CB_ERR_TOKEN);
    for (int k = threadIdx.x; k < K; k += blockDim.x) out[k] = 0.0f;
    return;
  }
  const uint8_t* tile = tiles + (id >> 4) * tile_bytes(K);
  const int rr = (int)(id & 15);
  const uint8_t* code = tile + rr * (K / 2);
  const uint8_t* sc = tile + kTileRows * (K / 2) + rr * (K / 16);
  const float ts = tile_scale[id >> 4];
  for (int j = threadIdx.x; j < K / 2; j += blockDim.x) {
    const float2 f = e2m1x2_to_f32x2(code[j]);
    const float s = e4m3_to_f32(sc[j >> 3]);
    out[2 * j] = (f.x * s) * ts;
    out[2 * j + 1] = (f.y * s) * ts;
  }
}

int launch_embed(const CbMatrix& tab, int vocab, const int64_t* ids, int64_t ids_ld, int batch, int T, int c0,
                 float* h, int32_t* status, cudaStream_t st) {
  embed_kernel<<<batch * T, 128, 0, st>>>(tab.tiles, tab.tile_scale, tab.k, vocab, ids, ids_ld, T, c0, h, status);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// ---------------------------------------------------------------- argmax
__global__ void argmax_kernel(const float* __restrict__ x, int n, int ld, int32_t* __restrict__ out) {
  const float* row = x + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = row[i];
    if (v > best) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

int launch_argmax(const float* x, int rows, int n, int ld, int32_t* out, cudaStream_t st) {
  if (rows <= 0) return CB_OK;
  argmax_kernel<<<rows, 1024, 0, st>>>(x, n, ld, out);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

// ------------------------------------------------------------------ C ABI
using namespace cb;

extern "C" int cb_nvfp4_quantize(const float* w, int32_t n, int32_t k, float tensor_scale, uint8_t* codes,
                                 uint8_t* scales, void* stream) {
  if (!w || !codes || !scales || n <= 0 || k <= 0 || k % 16 || !(tensor_scale > 0.0f)) return CB_ERR_ARG;
  const int64_t nb = (int64_t)n * (k / 16);
  quantize_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, (cudaStream_t)stream>>>(w, n, k, tensor_scale, codes,
                                                                                   scales);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

namespace cb {
// Column slices of `width` columns: slice s = [n][width/2 code bytes] then
// [n][1 scale byte] (the E4M3 scale of the 16-column block holding the slice).
__global__ void pack_slices_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, int n, int k,
                                   int width, int64_t slice_bytes, uint8_t* __restrict__ out) {
  const int cb = width / 2, ns = k / width;
  const int64_t total = (int64_t)ns * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(i / n), r = (int)(i - (int64_t)s * n);
    uint8_t* dst = out + s * slice_bytes;
    for (int j = 0; j < cb; ++j) dst[(int64_t)r * cb + j] = codes[(int64_t)r * (k / 2) + s * cb + j];
    dst[(int64_t)n * cb + r] = scales[(int64_t)r * (k / 16) + (s * width) / 16];
    if (r == 0)  // zero the padding after the scales
      for (int64_t j = (int64_t)n * (cb + 1); j < slice_bytes; ++j) dst[j] = 0;
  }
}
}  // namespace cb

extern "C" int64_t cb_nvfp4_slice_bytes(int32_t n, int32_t width) {
  if (n <= 0 || (width != 2 && width != 4 && width != 8 && width != 16)) return 0;
  return ((int64_t)n * (width / 2 + 1) + 15) / 16 * 16;
}

extern "C" int cb_nvfp4_pack_slices(const uint8_t* codes, const uint8_t* scales, int32_t n, int32_t k, int32_t width,
                                    uint8_t* out, void* stream) {
  const int64_t sb = cb_nvfp4_slice_bytes(n, width);
  if (!codes || !scales || !out || sb == 0 || k <= 0 || k % 16 || k % width) return CB_ERR_ARG;
  pack_slices_kernel<<<num_sms() * 4, 256, 0, (cudaStream_t)stream>>>(codes, scales, n, k, width, sb, out);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_nvfp4_pack_tiles(const uint8_t* codes, const uint8_t* scales, int32_t n, int32_t k, uint8_t* tiles,
                                   void* stream) {
  if (!codes || !scales || !tiles || n <= 0 || k <= 0 || k % 16) return CB_ERR_ARG;
  pack_tiles_kernel<<<num_sms() * 4, 256, 0, (cudaStream_t)stream>>>(codes, scales, n, k, tiles);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_gemv_nvfp4(const CbMatrix* w, const float* x, int32_t ldx, int32_t m_rows, float* y, int32_t ldy,
                             int32_t rows_out, void* stream) {
  if (!w) return CB_ERR_ARG;
  GemvParams p{};
  p.tiles = w->tiles;
  p.tile_scale = w->tile_scale;
  p.rows = w->rows;
  p.K = w->k;
  p.x = x;
  p.ldx = ldx;
  p.m_rows = m_rows;
  p.y = y;
  p.ldy = ldy;
  p.rows_out = rows_out;
  return launch_gemv(p, PRE_NONE, EPI_STORE, (cudaStream_t)stream);
}

extern "C" int cb_embed(const CbMatrix* table, const int64_t* ids, int32_t n_rows, float* h, int32_t* status,
                        void* stream) {
  if (!table || !ids || !h || n_rows <= 0) return CB_ERR_ARG;
  return launch_embed(*table, table->rows, ids, 1, n_rows, 1, 0, h, status, (cudaStream_t)stream);
}

extern "C" int cb_argmax(const float* x, int32_t rows, int32_t n, int32_t ld, int32_t* out, void* stream) {
  if (!x || !out || rows < 0 || n <= 0 || ld < n) return CB_ERR_ARG;
  return launch_argmax(x, rows, n, ld, out, (cudaStream_t)stream);
}
