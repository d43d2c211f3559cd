// NVFP4 weight stream: every projection of a decode step as one persistent
// launch, y = x . dequant(W)^T for M <= 8 token rows and every matrix of a list
// (the reference's decode-step weight stream, cirrus/perf/bench_kernels.cu
// :1079-1300 and scripts/bench_spark.py decode_stream_v5, where the matrices
// are independent and share one input).
//
// One CTA per SM walks the 16-row tiles of all matrices round-robin.  A
// producer warp keeps kStRing tiles in flight: each tile (9 * K contiguous
// bytes: codes then E4M3 scales) arrives by one bulk copy (cp.async.bulk,
// completion on the slot's mbarrier).  Sixteen compute warps take one row of
// the tile each: a lane's 32-bit code words and scale bytes from shared memory,
// E2M1 pairs to floats, products with the staged input rows in fp32, a warp
// shuffle reduction, and each warp releases the slot on its "empty" mbarrier.
// Every wait is bounded (%globaltimer); a timeout sets the status word and
// ends the launch.
#include "common.cuh"

namespace cb {
namespace {

constexpr int kStCompute = 16;                   // compute warps: one per tile row
constexpr int kStThreads = (kStCompute + 1) * 32; // + the producer warp
constexpr int kStRing = 8;                       // tiles in flight per CTA
constexpr int kStMaxK = 2048;
constexpr int kStSlot = kTileRows * kStMaxK * 9 / 16;  // 18 KB: one tile of K = 2048
constexpr int kStMaxMats = 128;
// Staged input rows keep 16 bytes of padding after every 32 floats, so the
// 128-bit loads of lanes 0-7 (8-float chunks 32 bytes apart) hit 32 distinct banks.
__host__ __device__ inline int st_xpad(int K) { return K + K / 8; }
__device__ __forceinline__ int st_xoff(int k) { return k + (k >> 5) * 4; }
constexpr unsigned long long kStTimeoutNs = 200ull * 1000 * 1000;

struct StreamMat {
  const uint8_t* tiles;
  const float* tile_scale;
  int32_t K, n_tiles;
  int64_t row_off;  // first output row of the matrix in y
};

struct StreamParams {
  const StreamMat* mats;  // device [n_mats]
  int n_mats, total_tiles;
  const float* x;  // [m_rows][ldx]
  int ldx, m_rows, kmax;
  float* y;  // [m_rows][ldy]
  int64_t ldy;
  int32_t* status;
};

__device__ __forceinline__ uint32_t st_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long st_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool st_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool st_wait(uint32_t bar, uint32_t parity, const int* abort_flag) {
  if (st_try(bar, parity)) return true;
  const unsigned long long t0 = st_timer();
  while (!st_try(bar, parity)) {
    if (*(volatile const int*)abort_flag) return false;
    if (st_timer() - t0 > kStTimeoutNs) return false;
  }
  return true;
}

// Matrix and local tile of global tile g; a CTA visits its tiles in increasing
// order, so the cursor (matrix mi, its first global tile base) only moves forward.
__device__ __forceinline__ int st_find(const StreamMat* mats, int n, int g, int& mi, int& base) {
  while (mi + 1 < n && g >= base + mats[mi].n_tiles) {
    base += mats[mi].n_tiles;
    ++mi;
  }
  return g - base;
}

template <int M>
__global__ void __launch_bounds__(kStThreads, 1) weight_stream_kernel(const __grid_constant__ StreamParams p) {
  extern __shared__ __align__(128) uint8_t ssm[];
  uint8_t* ring = ssm;                                           // [kStRing][kStSlot]
  float* xs = reinterpret_cast<float*>(ssm + kStRing * kStSlot);  // [M][st_xpad(kmax)]
  __shared__ __align__(8) unsigned long long full[kStRing], empty[kStRing];
  __shared__ StreamMat mats[kStMaxMats];
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < p.n_mats; i += kStThreads) mats[i] = p.mats[i];
  if (tid == 0) {
    for (int s = 0; s < kStRing; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st_smem(full + s)));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(st_smem(empty + s)), "r"(kStCompute));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  for (int i = tid; i < M * p.kmax; i += kStThreads) {
    const int m = i / p.kmax, k = i - m * p.kmax;
    xs[m * st_xpad(p.kmax) + st_xoff(k)] = m < p.m_rows ? p.x[(int64_t)m * p.ldx + k] : 0.0f;
  }
  __syncthreads();
  const int n_mine = p.total_tiles > (int)blockIdx.x ? (p.total_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (warp == kStCompute) {
    // producer: tile i of this CTA into slot i % kStRing once the slot's previous tile is released
    if (lane == 0) {
      int mi = 0, base = 0;
      for (int i = 0; i < n_mine; ++i) {
        const int s = i % kStRing;
        if (i >= kStRing) {
          if (!st_wait(st_smem(empty + s), ((i / kStRing) - 1) & 1, &s_abort)) {
            s_abort = 1;
            break;
          }
          // the slot's previous tile was read through the generic proxy
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        const int local = st_find(mats, p.n_mats, (int)blockIdx.x + i * (int)gridDim.x, mi, base);
        const unsigned bytes = (unsigned)(kTileRows * mats[mi].K * 9 / 16);
        const uint32_t bar = st_smem(full + s);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                st_smem(ring + s * kStSlot)),
            "l"(mats[mi].tiles + (int64_t)local * kTileRows * mats[mi].K * 9 / 16), "r"(bytes), "r"(bar)
            : "memory");
      }
    }
  } else {
    int mi = 0, base = 0;
    for (int i = 0; i < n_mine; ++i) {
      const int s = i % kStRing;
      // the tile scale is loaded before the wait, so its latency overlaps the wait and the dot products
      const int local = st_find(mats, p.n_mats, (int)blockIdx.x + i * (int)gridDim.x, mi, base);
      const float ts = __ldg(mats[mi].tile_scale + local);
      if (!st_wait(st_smem(full + s), (i / kStRing) & 1, &s_abort)) {
        s_abort = 1;
        break;
      }
      const int K = mats[mi].K, kc = K >> 3;
      const uint8_t* tile = ring + s * kStSlot;
      const uint32_t* cw = reinterpret_cast<const uint32_t*>(tile + warp * (K / 2));
      const uint8_t* sb = tile + kTileRows * (K / 2) + warp * (K / 16);
      float acc[M];
#pragma unroll
      for (int m = 0; m < M; ++m) acc[m] = 0.0f;
      for (int c = lane; c < kc; c += 32) {
        const uint32_t w = cw[c];
        const float sc = e4m3_to_f32(sb[c >> 1]);
        float2 f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = e2m1x2_to_f32x2(w >> (8 * j));
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float* xc = xs + m * st_xpad(p.kmax) + st_xoff(c * 8);
          const float4 xa = *reinterpret_cast<const float4*>(xc);
          const float4 xb = *reinterpret_cast<const float4*>(xc + 4);
          float d = f[0].x * xa.x;
          d = fmaf(f[0].y, xa.y, d);
          d = fmaf(f[1].x, xa.z, d);
          d = fmaf(f[1].y, xa.w, d);
          d = fmaf(f[2].x, xb.x, d);
          d = fmaf(f[2].y, xb.y, d);
          d = fmaf(f[3].x, xb.z, d);
          d = fmaf(f[3].y, xb.w, d);
          acc[m] = fmaf(d, sc, acc[m]);
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(st_smem(empty + s)) : "memory");
      const int64_t row = mats[mi].row_off + (int64_t)local * kTileRows + warp;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float v = warp_sum(acc[m]) * ts;
        if (lane == m && m < p.m_rows) p.y[(int64_t)m * p.ldy + row] = v;
      }
    }
  }
  if (s_abort && tid == 0 && p.status) atomicCAS(p.status, 0, CB_ERR_TIMEOUT);
  // copies still in flight land before the CTA exits (bounded)
  __syncthreads();
  if (tid == 0 && n_mine > 0) {
    const int last = n_mine - 1;
    for (int i = (last >= kStRing ? last - kStRing + 1 : 0); i <= last; ++i)
      st_wait(st_smem(full + i % kStRing), (i / kStRing) & 1, &s_abort);
  }
}

}  // namespace

}  // namespace cb

using namespace cb;

extern "C" size_t cb_stream_plan_bytes(int32_t n_mats) {
  return n_mats > 0 && n_mats <= kStMaxMats ? sizeof(StreamMat) * (size_t)n_mats : 0;
}

extern "C" int cb_stream_plan(const CbMatrix* mats, int32_t n_mats, void* plan, size_t plan_bytes, int64_t* rows_total,
                              void* stream) {
  if (!mats || !plan || n_mats <= 0 || n_mats > kStMaxMats || plan_bytes < cb_stream_plan_bytes(n_mats))
    return CB_ERR_ARG;
  StreamMat host[kStMaxMats];
  int64_t off = 0;
  for (int i = 0; i < n_mats; ++i) {
    const CbMatrix& w = mats[i];
    if (!w.tiles || !w.tile_scale || w.rows <= 0 || w.rows % kTileRows || w.k < 256 || w.k % 256 || w.k > kStMaxK ||
        (reinterpret_cast<uintptr_t>(w.tiles) & 15))
      return CB_ERR_SHAPE;
    host[i] = StreamMat{w.tiles, w.tile_scale, w.k, w.rows / kTileRows, off};
    off += w.rows;
  }
  if (rows_total) *rows_total = off;
  // pageable source: the copy is complete when the call returns
  if (cudaMemcpyAsync(plan, host, sizeof(StreamMat) * n_mats, cudaMemcpyHostToDevice, (cudaStream_t)stream) !=
      cudaSuccess)
    return CB_ERR_CUDA;
  return cudaStreamSynchronize((cudaStream_t)stream) == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_weight_stream_nvfp4(const void* plan, int32_t n_mats, int32_t total_tiles, const float* x,
                                      int32_t ldx, int32_t kmax, int32_t m_rows, float* y, int64_t ldy, int32_t* status,
                                      void* stream) {
  if (!plan || !x || !y || n_mats <= 0 || n_mats > kStMaxMats || total_tiles <= 0 || m_rows < 1 || m_rows > 8 ||
      kmax < 256 || kmax > kStMaxK || kmax % 256 || ldx < kmax || ldy < 1)
    return CB_ERR_ARG;
  StreamParams p{static_cast<const StreamMat*>(plan), n_mats, total_tiles, x, ldx, m_rows, kmax, y, ldy, status};
  const int M = m_rows <= 1 ? 1 : m_rows <= 2 ? 2 : m_rows <= 4 ? 4 : 8;
  const size_t smem = (size_t)kStRing * kStSlot + sizeof(float) * (size_t)M * st_xpad(kmax);
  const void* fn = M == 1 ? (const void*)weight_stream_kernel<1>
                 : M == 2 ? (const void*)weight_stream_kernel<2>
                 : M == 4 ? (const void*)weight_stream_kernel<4>
                          : (const void*)weight_stream_kernel<8>;
  if (ensure_smem_attr(fn, (int)((size_t)kStRing * kStSlot + sizeof(float) * 8 * st_xpad(kStMaxK))) != CB_OK)
    return CB_ERR_CUDA;
  void* args[] = {&p};
  const cudaError_t e = cudaLaunchKernel(fn, dim3(num_sms()), dim3(kStThreads), args, smem, (cudaStream_t)stream);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}
