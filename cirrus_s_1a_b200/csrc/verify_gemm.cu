// Multi-token verify GEMM on the 5th-generation tensor cores (tcgen05):
//   y[t][r] = sum_k x[t][k] * dequant(W)[r][k]      t < m_rows <= 16
//
// The reference runs this contraction for a verify of 1 + draft tokens
// (draft width 2-8) as nvfp4_gemv with M > 1 (cirrus/perf/bench_kernels.cu
// :202-227, mma.sync f16 in its v4/v5 kernels).  Here one CTA owns a 128-row
// tile of W:
//   * W: each K chunk of 64 (128 rows x 32 code bytes + 4 scale bytes) comes
//     by cp.async into a ring of 6 raw stages, 5 chunks ahead; all 256 threads
//     dequantise it (E2M1 code x E4M3 block scale is exact in bf16) into a
//     shared-memory stage in the canonical K-major layout (8-row x 16-byte core
//     matrices, no swizzle); two such stages alternate;
//   * x: staged once as bf16, 16 rows (tokens; rows >= m_rows are zero);
//   * one thread issues tcgen05.mma.kind::f16 (M 128, N 16, K 16) x 4 per
//     chunk into an fp32 accumulator in tensor memory and commits to the
//     stage's mbarrier, which frees the stage for the chunk after next;
//   * the epilogue reads the accumulator with tcgen05.ld (warp w owns rows
//     32w .. 32w + 31) and applies the fp32 tile scale;
//   * a tile with few rows per SM splits K over a cluster of up to 8 CTAs; the
//     partials meet in distributed shared memory and cluster rank 0 adds them
//     in rank order (deterministic, no atomics).
// Every wait is bounded (%globaltimer); on timeout the launch sets its status
// word and skips the remaining work, and still frees its tensor memory.
#include <cuda_bf16.h>

#include "common.cuh"

namespace cb {
namespace {

constexpr int kVgThreads = 256;
constexpr int kVgM = 128;        // W rows per CTA (MMA M)
constexpr int kVgN = 16;         // token columns (MMA N)
constexpr int kVgKc = 64;        // K per stage
constexpr int kVgStageBytes = kVgM * kVgKc * 2;  // 16 KB
constexpr int kVgRing = 6;                         // raw NVFP4 chunks in flight
constexpr int kVgRawBytes = kVgM * (kVgKc / 2) + kVgM * (kVgKc / 16);  // 4 KB codes + 512 B scales
constexpr unsigned long long kVgTimeoutNs = 200ull * 1000 * 1000;

struct VerifyParams {
  const uint8_t* tiles;
  const float* tile_scale;
  int rows, K;
  const uint16_t* x;  // bf16 [m_rows][ldx]
  int ldx, m_rows;
  float* y;
  int ldy, rows_out;
  int32_t* status;    // set to CB_ERR_TIMEOUT when a bounded wait gives up (may be null)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long vg_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Matrix descriptor of a K-major, no-swizzle operand: start address, leading
// byte offset (between the two 8-element K halves of a K=16 step), stride byte
// offset (between 8-row groups), version 1 (bits 46-47), layout type 0.
__device__ __forceinline__ uint64_t vg_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B bf16
// (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
constexpr uint32_t kVgIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kVgN >> 3) << 17) |
                              ((uint32_t)(kVgM >> 4) << 24);

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase; false after the time limit.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = vg_timer();
  while (!mbar_try(bar, parity))
    if (vg_timer() - t0 > kVgTimeoutNs) return false;
  return true;
}

// bf16 bits of an E2M1 code (exact): magnitude code m = 2e + f (e exponent,
// f mantissa bit) is (1 + f/2) * 2^(e-1) for m >= 2 -> biased exponent e + 126,
// mantissa bit f at bit 6; m = 1 is 0.5; bit 3 is the sign.
__device__ __forceinline__ uint32_t e2m1_bf16(uint32_t c) {
  const uint32_t m = c & 7;
  const uint32_t mag = m >= 2 ? ((((m >> 1) + 126u) << 7) | ((m & 1u) << 6)) : (m == 1 ? 0x3F00u : 0u);
  return mag | ((c & 8u) << 12);
}

__global__ void __launch_bounds__(kVgThreads, 1) verify_gemm_kernel(const __grid_constant__ VerifyParams p) {
  extern __shared__ __align__(1024) uint8_t vsm[];
  __shared__ __align__(8) unsigned long long bar_mma[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // split K over the CTAs of a cluster (csize 1 without clusters): this CTA owns
  // chunks [cbeg, cbeg + nchunks) of its 128-row tile
  uint32_t crank, csize;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int K = p.K, nall = K / kVgKc, row0 = (int)(blockIdx.x / csize) * kVgM;
  const int cbeg = (int)crank * nall / (int)csize, nchunks = ((int)crank + 1) * nall / (int)csize - cbeg;
  uint8_t* A = vsm;                          // [2][16 row groups][8 k-blocks][8 rows][16 B]
  uint8_t* B = vsm + 2 * kVgStageBytes;      // [2 row groups][K/8 k-blocks][8 rows][16 B]
  const uint32_t sbo_b = (uint32_t)(K / 8) * 128u;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar_mma + b)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(smem_u32(&tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // x -> B (bf16, 16 token rows, zero beyond m_rows)
  for (int i = tid; i < kVgN * (K / 8); i += kVgThreads) {
    const int n = i / (K / 8), kb = i - n * (K / 8);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (n < p.m_rows) v = *reinterpret_cast<const uint4*>(p.x + (int64_t)n * p.ldx + kb * 8);
    *reinterpret_cast<uint4*>(B + (n >> 3) * sbo_b + kb * 128 + (n & 7) * 16) = v;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  // this thread's share of a chunk: row r of the tile, 32 K values (half h).
  // Raw chunks travel by cp.async into a ring of kVgRing stages, kVgRing - 1
  // chunks ahead of the one being converted.
  const int r = tid >> 1, h = tid & 1, grow = row0 + r;
  const bool rvalid = grow < p.rows;
  const int64_t tb = 9ll * K;
  const uint8_t* codes = p.tiles + (int64_t)(grow >> 4) * tb + (grow & 15) * (K / 2) + 16 * h;
  const uint8_t* sc = p.tiles + (int64_t)(grow >> 4) * tb + kTileRows * (K / 2) + (grow & 15) * (K / 16);
  uint8_t* raw = B + (size_t)kVgN * K * 2;  // [kVgRing][codes 128 x 32 | scales 128 x 4]
  auto issue = [&](int c) {
    if (rvalid && c < nchunks) {
      uint8_t* rs = raw + (c % kVgRing) * kVgRawBytes;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(rs + r * 32 + 16 * h)),
                   "l"(codes + (cbeg + c) * 32)
                   : "memory");
      if (h == 0)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(rs + kVgM * 32 + r * 4)),
                     "l"(sc + (cbeg + c) * 4)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int j = 0; j < kVgRing - 1; ++j) issue(j);
  unsigned par[2] = {0u, 0u};
  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c & 1;
    uint8_t* As = A + st * kVgStageBytes;
    issue(c + kVgRing - 1);  // its stage held chunk c - 1, converted before the last barrier
    asm volatile("cp.async.wait_group %0;" ::"n"(kVgRing - 1) : "memory");
    // the MMA of chunk c - 2 read this A stage: wait for its commit
    if (c >= 2 && tid == 0 && !mbar_wait(smem_u32(bar_mma + st), par[st])) s_abort = 1;
    __syncthreads();  // chunk c's raw bytes (all threads' copies) visible; abort flag
    if (s_abort) {
      ok = false;
      break;
    }
    if (c >= 2) {
      mbar_wait(smem_u32(bar_mma + st), par[st]);  // completed: returns at once
      par[st] ^= 1u;
    }
    const uint8_t* rs = raw + (c % kVgRing) * kVgRawBytes;
    uint4 cw = make_uint4(0u, 0u, 0u, 0u);
    uint32_t s2 = 0;
    if (rvalid) {
      cw = *reinterpret_cast<const uint4*>(rs + r * 32 + 16 * h);
      s2 = (uint32_t)rs[kVgM * 32 + r * 4 + 2 * h] | ((uint32_t)rs[kVgM * 32 + r * 4 + 2 * h + 1] << 8);
    }
    // 32 codes -> bf16 x E4M3 scale (exact), into k-blocks 4h .. 4h + 3 of row r
    const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 s = __floats2bfloat162_rn(e4m3_to_f32((s2 >> (8 * (j >> 1))) & 0xFF),
                                                     e4m3_to_f32((s2 >> (8 * (j >> 1))) & 0xFF));
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t byte = (w4[j] >> (8 * q)) & 0xFF;
        const uint32_t pr = e2m1_bf16(byte & 15) | (e2m1_bf16(byte >> 4) << 16);
        __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&pr);
        v = __hmul2(v, s);
        o[q] = *reinterpret_cast<uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(As + (r >> 3) * 1024 + (4 * h + j) * 128 + (r & 7) * 16) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
    // generic-proxy stores -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int s = 0; s < kVgKc / 16; ++s) {
        const uint64_t da = vg_desc(smem_u32(As) + s * 256, 128, 1024);
        const uint64_t db = vg_desc(smem_u32(B) + ((cbeg + c) * (kVgKc / 8) + 2 * s) * 128, 128, sbo_b);
        const uint32_t acc = (c > 0 || s > 0) ? 1u : 0u;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
            "l"(da), "l"(db), "r"(kVgIdesc), "r"(acc)
            : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(bar_mma + st))
                   : "memory");
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA
  // the last commit covers every MMA issued before it
  if (ok && nchunks > 0) {
    const int st = (nchunks - 1) & 1;
    if (tid == 0 && !mbar_wait(smem_u32(bar_mma + st), par[st])) s_abort = 1;
    __syncthreads();
    ok = !s_abort;
    if (ok) mbar_wait(smem_u32(bar_mma + st), par[st]);
  } else if (!ok) {
    // give the MMAs already issued a bounded time to finish before freeing their memory
    if (tid == 0) {
      for (int st = 0; st < 2; ++st) mbar_wait(smem_u32(bar_mma + st), par[st]);
    }
    __syncthreads();
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  uint32_t d[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) d[t] = 0u;
  if (ok && warp < 4) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
          "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
        : "r"(tmem + ((uint32_t)(warp * 32) << 16)));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  }
  const int row = row0 + warp * 32 + lane;
  if (csize == 1) {
    if (ok && warp < 4 && row < p.rows_out) {
      const float ts = p.tile_scale[row >> 4];
#pragma unroll
      for (int t = 0; t < kVgN; ++t)
        if (t < p.m_rows) p.y[(int64_t)t * p.ldy + row] = __uint_as_float(d[t]) * ts;
    }
  } else {
    // split K: every CTA parks its partial in shared memory (the A stages are
    // idle now); rank 0 adds the partials of ranks 0 .. csize-1 in that order
    float* red = reinterpret_cast<float*>(A);  // [128][17]
    if (warp < 4)
#pragma unroll
      for (int t = 0; t < kVgN; ++t) red[(warp * 32 + lane) * 17 + t] = __uint_as_float(d[t]);
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (crank == 0 && warp < 4 && row < p.rows_out) {
      const float ts = p.tile_scale[row >> 4];
      for (int t = 0; t < p.m_rows; ++t) {
        float acc = 0.0f;
        for (uint32_t rk = 0; rk < csize; ++rk) {
          uint32_t ra;
          float v;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(red + (warp * 32 + lane) * 17 + t)), "r"(rk));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
          acc += v;
        }
        p.y[(int64_t)t * p.ldy + row] = acc * ts;
      }
    }
    // rank 0 has read every partial before any CTA of the cluster exits
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  if (!ok && tid == 0 && p.status) atomicCAS(p.status, 0, CB_ERR_TIMEOUT);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem));
}

}  // namespace

size_t verify_gemm_smem(int K) { return (size_t)2 * kVgStageBytes + (size_t)kVgN * K * 2 + (size_t)kVgRing * kVgRawBytes; }

}  // namespace cb

using namespace cb;

extern "C" int cb_verify_gemm_nvfp4(const CbMatrix* w, const uint16_t* x, int32_t ldx, int32_t m_rows, float* y,
                                    int32_t ldy, int32_t rows_out, int32_t* status, void* stream) {
  if (!w || !x || !y || !w->tiles || !w->tile_scale) return CB_ERR_ARG;
  if (m_rows < 1 || m_rows > kVgN || rows_out < 1 || rows_out > w->rows || ldy < rows_out || ldx < w->k)
    return CB_ERR_ARG;
  const int K = w->k;
  if (K < kVgKc || K % kVgKc || K > 2048 || w->rows % kTileRows) return CB_ERR_SHAPE;
  // 16-byte vector loads of x rows and of the packed code rows
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx % 8) || (reinterpret_cast<uintptr_t>(w->tiles) & 15))
    return CB_ERR_ARG;
  const size_t smem = verify_gemm_smem(K);
  if (ensure_smem_attr((const void*)verify_gemm_kernel, (int)verify_gemm_smem(2048)) != CB_OK) return CB_ERR_CUDA;
  VerifyParams p{};
  p.tiles = w->tiles;
  p.tile_scale = w->tile_scale;
  p.rows = w->rows;
  p.K = K;
  p.x = x;
  p.ldx = ldx;
  p.m_rows = m_rows;
  p.y = y;
  p.ldy = ldy;
  p.rows_out = rows_out;
  p.status = status;
  // split K over a cluster of up to 8 CTAs while the grid stays within two CTAs per SM
  const int tiles = (rows_out + kVgM - 1) / kVgM, nall = K / kVgKc;
  const int sms = num_sms();
  int S = 1;
  while (S < 8 && tiles * S * 2 <= 2 * sms && S * 2 <= nall) S *= 2;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles * S);
  cfg.blockDim = dim3(kVgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, verify_gemm_kernel, p);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}
