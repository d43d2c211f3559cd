// Many-token NVFP4 GEMM on the 5th-generation tensor cores (tcgen05):
//   y[m][r] (=, +=) sum_k pre(x)[m][k] * dequant(W)[r][k]        m < m_rows
//
// This is the contraction of a step that carries many token rows at once:
// batched decode (B sequences x 1 token), batched verify (B x (1 + draft)) and
// prompt chunks.  The CUDA-core GEMV re-reads the weights for every 16 token
// rows; here each weight tile is read once per 64 tokens and the products run
// on the tensor pipe.  Two launches:
//
// gemm_prep_kernel: each input row once -- RMSNorm when asked (layers.py:39-44),
//   then split into an f16 head and an f16 tail, hi = f16(x), lo = f16(x - hi),
//   written in the tensor core's K-major operand layout (8-row x 16-byte core
//   matrices), one contiguous 16 KB block per (64-token tile, K chunk of 64):
//   rows 0-63 the heads, rows 64-127 the tails.
// gemm_nvfp4_kernel: one CTA owns a 128-row tile of W and a 64-token tile (a
//   cluster of up to 8 CTAs splits K):
//   * W: each K chunk of 64 (128 rows x 32 code bytes, 4 scale bytes per row)
//     comes by cp.async into a ring of kGRing raw stages, kGRing - 1 chunks
//     ahead; each thread copies exactly the bytes it converts.  E2M1 pairs go
//     to f16x2 by the hardware converter and are multiplied by the E4M3 block
//     scale, also f16: every E2M1 x E4M3 product has at most 6 significant bits
//     and lies in [2^-10, 2688], so the f16 operand is exact.  Two A stages.
//   * B: the prepared 16 KB block of each chunk comes by one bulk copy
//     (cp.async.bulk, completion on an mbarrier) into a ring of kGBRing stages,
//     two chunks ahead; a stage is refilled once the MMAs that read it commit.
//   * one thread issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N 128,
//     K 16) x 4 per chunk into an fp32 accumulator in tensor memory; the
//     epilogue adds the head and tail columns, so every input carries about 22
//     bits into fp32 accumulation.
//   * epilogue: tcgen05.ld -> shared memory; with split K the cluster's
//     partials are added in rank order through distributed shared memory, each
//     rank finishing a slice of the rows; then the tile scale and the store /
//     residual add / SwiGLU (gate row r and up row F + r in one tile).
// Both kernels are launched as programmatic dependents: the GEMM's set-up and
// its first weight copies overlap the kernel before it, and it waits
// (griddepcontrol.wait) before it reads the prepared inputs or writes y.
// Every mbarrier wait is bounded (%globaltimer); on timeout the launch sets its
// status word, skips the rest of the work, and still frees its tensor memory.
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemm.cuh"

namespace cb {
namespace {

constexpr int kGT = 256;                   // threads
constexpr int kGM = 128;                   // W rows per CTA (MMA M)
constexpr int kGN = 64;                    // token rows per CTA
constexpr int kGNm = 2 * kGN;              // MMA N: head and tail rows
constexpr int kGKc = 64;                   // K per chunk
constexpr int kGRing = 4;                  // raw weight chunks in flight
constexpr int kGBRing = 3;                 // prepared input chunks (bulk copies)
constexpr int kGAStage = kGM * kGKc * 2;   // 16 KB f16
constexpr int kGBStage = kGNm * kGKc * 2;  // 16 KB f16
constexpr int kGRawCodes = kGM * kGKc / 2;  // 4 KB
constexpr int kGRawScales = kGT * 4;        // 1 KB: each thread its row's 4 scale bytes
constexpr int kGRawStage = kGRawCodes + kGRawScales;
constexpr int kGSmem = 2 * kGAStage + kGBRing * kGBStage + kGRing * kGRawStage;
constexpr int kGPartLd = kGN + 1;
constexpr int kGTmemCols = kGNm;
constexpr unsigned long long kGTimeoutNs = 200ull * 1000 * 1000;
static_assert(kGM * kGPartLd * 4 <= 2 * kGAStage + kGBRing * kGBStage, "partials live in the A and B stages");

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B f16 (0),
// both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kGIdesc = (1u << 4) | ((uint32_t)(kGNm >> 3) << 17) | ((uint32_t)(kGM >> 4) << 24);

__device__ __forceinline__ uint32_t g_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long g_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Shared-memory matrix descriptor, K-major without swizzle: start address,
// leading byte offset (K-adjacent 8x16-byte core matrices), stride byte offset
// (8-row groups), descriptor version 1 at bits 46-47.
__device__ __forceinline__ uint64_t g_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

__device__ __forceinline__ bool g_mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool g_mbar_wait(uint32_t bar, uint32_t parity) {
  if (g_mbar_try(bar, parity)) return true;
  const unsigned long long t0 = g_timer();
  while (!g_mbar_try(bar, parity))
    if (g_timer() - t0 > kGTimeoutNs) return false;
  return true;
}

__device__ __forceinline__ void g_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void g_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void g_cp4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Programmatic dependent launch: wait for the kernels this one depends on
// (a no-op without the launch attribute), and let the next one start.
__device__ __forceinline__ void g_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void g_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Offset of (row n, 8-element K block kb) in a K-major no-swizzle operand stage of 64 K.
__device__ __forceinline__ uint32_t g_off(int n, int kb) { return (uint32_t)((n >> 3) * 1024 + kb * 128 + (n & 7) * 16); }

// Two E2M1 codes (one byte, low nibble first) times an f16x2 scale -> f16x2 bits (exact).
__device__ __forceinline__ uint32_t g_dq2(uint32_t byte, __half2 s) {
  __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)(byte & 0xFF), __NV_E2M1);
  __half2 v = __hmul2(__half2(h), s);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// ------------------------------------------------------------------ input preparation
// Two token rows of the padded token range per CTA, 128 threads per row:
// RMSNorm factor (block reduction over K), then 8-element K blocks as head and
// tail f16 into the prepared operand blocks.  Rows >= m_rows are written as zeros.
constexpr int kPrepRowThreads = kGT / 2;

__global__ void __launch_bounds__(kGT) gemm_prep_kernel(const __grid_constant__ GemmParams p) {
  g_dep_wait();
  g_dep_launch();
  __shared__ float s_part[kGT / 32];
  const int half = threadIdx.x / kPrepRowThreads, t = threadIdx.x - half * kPrepRowThreads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 2 + half;
  const int K = p.K, nall = K / kGKc;
  const bool valid = row < p.m_rows;
  const float* xr = p.x + (int64_t)row * p.ldx;
  constexpr int kMaxBlk = 8;  // 8-element blocks per thread: K <= 8192
  float4 va[kMaxBlk], vb[kMaxBlk];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    const int kb8 = t + j * kPrepRowThreads;
    va[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    vb[j] = va[j];
    if (valid && kb8 < K / 8) {
      va[j] = __ldcg(reinterpret_cast<const float4*>(xr + kb8 * 8));
      vb[j] = __ldcg(reinterpret_cast<const float4*>(xr + kb8 * 8 + 4));
    }
  }
  float rn = 1.0f;
  if (p.pre == GEMM_PRE_RMSNORM) {
#pragma unroll
    for (int j = 0; j < kMaxBlk; ++j) {
      ss = fmaf(va[j].x, va[j].x, ss);
      ss = fmaf(va[j].y, va[j].y, ss);
      ss = fmaf(va[j].z, va[j].z, ss);
      ss = fmaf(va[j].w, va[j].w, ss);
      ss = fmaf(vb[j].x, vb[j].x, ss);
      ss = fmaf(vb[j].y, vb[j].y, ss);
      ss = fmaf(vb[j].z, vb[j].z, ss);
      ss = fmaf(vb[j].w, vb[j].w, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) s_part[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < kPrepRowThreads / 32; ++w) tot += s_part[half * (kPrepRowThreads / 32) + w];
    rn = rsqrtf(tot / (float)K + p.eps);
  }
  const int nt = row / kGN, n = row - nt * kGN;
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    const int kb8 = t + j * kPrepRowThreads;
    if (kb8 >= K / 8) continue;
    float v[8] = {va[j].x, va[j].y, va[j].z, va[j].w, vb[j].x, vb[j].y, vb[j].z, vb[j].w};
    if (valid && p.pre == GEMM_PRE_RMSNORM) {
      const float4 n0 = __ldg(reinterpret_cast<const float4*>(p.norm_w + kb8 * 8));
      const float4 n1 = __ldg(reinterpret_cast<const float4*>(p.norm_w + kb8 * 8 + 4));
      const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] * rn * nw[i];
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half h0 = __float2half_rn(v[2 * i]), h1 = __float2half_rn(v[2 * i + 1]);
      const __half l0 = __float2half_rn(v[2 * i] - __half2float(h0));
      const __half l1 = __float2half_rn(v[2 * i + 1] - __half2float(h1));
      hi[i] = pack_h2(h0, h1);
      lo[i] = pack_h2(l0, l1);
    }
    const int kc = kb8 >> 3, kb = kb8 & 7;
    uint8_t* blk = p.xb + ((int64_t)nt * nall + kc) * kGBStage;
    *reinterpret_cast<uint4*>(blk + g_off(n, kb)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(blk + g_off(kGN + n, kb)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// ------------------------------------------------------------------ GEMM
__global__ void __launch_bounds__(kGT, 2) gemm_nvfp4_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  __shared__ __align__(8) unsigned long long bar_mma[2];
  __shared__ __align__(8) unsigned long long bar_bfull[kGBRing];
  __shared__ __align__(8) unsigned long long bar_bfree[kGBRing];
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  __shared__ float s_ts[kGM / kTileRows];  // tile scales of the CTA's rows (SwiGLU: 4 gate tiles, then 4 up tiles)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t crank, csize;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int K = p.K, nall = K / kGKc;
  const int tile = (int)(blockIdx.x / csize);
  const int ntile = (int)blockIdx.y, m0 = ntile * kGN;
  const int cbeg = (int)crank * nall / (int)csize, nch = ((int)crank + 1) * nall / (int)csize - cbeg;
  const bool swiglu = p.epi == GEMM_EPI_SWIGLU;
  const int half_rows = p.rows / 2;  // SwiGLU: gate rows [0, F), up rows [F, 2F)
  uint8_t* A = gsm;                            // [2][16 KB]
  uint8_t* Bs = gsm + 2 * kGAStage;            // [kGBRing][16 KB]
  uint8_t* raw = Bs + kGBRing * kGBStage;      // [kGRing][codes | scales]

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g_smem_u32(bar_mma + b)));
    for (int b = 0; b < kGBRing; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g_smem_u32(bar_bfull + b)));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g_smem_u32(bar_bfree + b)));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g_smem_u32(&tmem_base)),
                 "n"(kGTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }

  // this thread's weight row (r) and K half (h) of every chunk
  const int r = tid >> 1, h = tid & 1;
  int grow;
  if (swiglu) grow = r < 64 ? tile * 64 + r : half_rows + tile * 64 + (r - 64);
  else grow = tile * kGM + r;
  const bool rvalid = swiglu ? (tile * 64 + (r & 63)) < half_rows : grow < p.rows;
  const int64_t tb = 9ll * K;
  const uint8_t* codes = p.tiles + (int64_t)(grow >> 4) * tb + (grow & 15) * (K / 2) + 16 * h;
  const uint8_t* scl = p.tiles + (int64_t)(grow >> 4) * tb + kTileRows * (K / 2) + (grow & 15) * (K / 16);
  const uint32_t raw_s = g_smem_u32(raw);

  auto issue = [&](int c) {  // weights only: nothing another kernel writes
    if (c < nch && rvalid) {
      const uint32_t rs = raw_s + (uint32_t)((c % kGRing) * kGRawStage);
      const int kc = cbeg + c;
      g_cp16(rs + r * 32 + 16 * h, codes + kc * 32);
      g_cp4(rs + kGRawCodes + tid * 4, scl + kc * 4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int j = 0; j < kGRing - 1; ++j) issue(j);
  if (tid < kGM / kTileRows) {
    int tr;
    if (swiglu) tr = tid < 4 ? tile * 64 + tid * kTileRows : half_rows + tile * 64 + (tid - 4) * kTileRows;
    else tr = tile * kGM + tid * kTileRows;
    s_ts[tid] = tr < p.rows ? __ldg(p.tile_scale + tr / kTileRows) : 0.0f;
  }

  // the prepared inputs come from the kernel before this one
  g_dep_wait();
  const uint8_t* xb = p.xb + ((int64_t)ntile * nall + cbeg) * kGBStage;
  auto issue_b = [&](int c) {  // thread 0: chunk c's prepared block into B stage c % kGBRing
    const uint32_t bar = g_smem_u32(bar_bfull + c % kGBRing);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kGBStage) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            g_smem_u32(Bs + (c % kGBRing) * kGBStage)),
        "l"(xb + (int64_t)c * kGBStage), "r"(kGBStage), "r"(bar)
        : "memory");
  };
  if (tid == 0)
    for (int c = 0; c < 2 && c < nch; ++c) issue_b(c);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int st = c & 1;
    issue(c + kGRing - 1);  // its ring slot held chunk c - 1, which this thread converted already
    asm volatile("cp.async.wait_group %0;" ::"n"(kGRing - 1) : "memory");
    // the MMAs of chunk c - 2 read this A stage: wait for their commit
    if (c >= 2 && !g_mbar_wait(g_smem_u32(bar_mma + st), ((c - 2) >> 1) & 1)) s_abort = 1;
    const uint8_t* rsp = raw + (c % kGRing) * kGRawStage;
    // A: 32 codes of row r -> f16 (exact) into K blocks 4h .. 4h + 3
    {
      uint4 cw = make_uint4(0u, 0u, 0u, 0u);
      uint32_t s4 = 0;
      if (rvalid) {
        cw = *reinterpret_cast<const uint4*>(rsp + r * 32 + 16 * h);
        s4 = *reinterpret_cast<const uint32_t*>(rsp + kGRawCodes + tid * 4);
      }
      const uint32_t w4[4] = {cw.x, cw.y, cw.z, cw.w};
      uint8_t* As = A + st * kGAStage;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // K block 4h + j covers elements 8j .. 8j + 7 of this half: scale byte 2h + j / 2
        const uint32_t sb = (s4 >> (8 * (2 * h + (j >> 1)))) & 0xFF;
        __half_raw sh = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)sb, __NV_E4M3);
        const __half2 s2 = __half2(__half(sh), __half(sh));
        uint4 o;
        o.x = g_dq2(w4[j], s2);
        o.y = g_dq2(w4[j] >> 8, s2);
        o.z = g_dq2(w4[j] >> 16, s2);
        o.w = g_dq2(w4[j] >> 24, s2);
        *reinterpret_cast<uint4*>(As + g_off(r, 4 * h + j)) = o;
      }
    }
    // generic-proxy stores -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (s_abort) {
      ok = false;
      break;
    }
    if (tid == 0) {
      // refill the B stage of chunk c - 1 with chunk c + 2 once chunk c - 1's MMAs are done
      if (c >= 1 && c + 2 < nch) {
        if (!g_mbar_wait(g_smem_u32(bar_bfree + (c - 1) % kGBRing), ((c - 1) / kGBRing) & 1)) s_abort = 1;
        else issue_b(c + 2);
      } else if (c == 0 && 2 < nch) {
        issue_b(2);
      }
      if (!g_mbar_wait(g_smem_u32(bar_bfull + c % kGBRing), (c / kGBRing) & 1)) s_abort = 1;
      if (!s_abort) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t as = g_smem_u32(A + st * kGAStage), bs = g_smem_u32(Bs + (c % kGBRing) * kGBStage);
#pragma unroll
        for (int s = 0; s < kGKc / 16; ++s) {
          const uint64_t da = g_desc(as + s * 256, 128, 1024);
          const uint64_t db = g_desc(bs + s * 256, 128, 1024);
          const uint32_t acc = (c > 0 || s > 0) ? 1u : 0u;
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
              "l"(da), "l"(db), "r"(kGIdesc), "r"(acc)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         g_smem_u32(bar_mma + st))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         g_smem_u32(bar_bfree + c % kGBRing))
                     : "memory");
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA
  __syncthreads();
  if (s_abort) ok = false;
  if (ok && nch > 0) {
    // the last commit covers every MMA issued before it
    if (!g_mbar_wait(g_smem_u32(bar_mma + ((nch - 1) & 1)), ((nch - 1) >> 1) & 1)) s_abort = 1;
    __syncthreads();
    ok = !s_abort;
  }
  if (!ok && tid == 0) {
    // give the copies and MMAs already issued a bounded time to finish before their memory is reused or freed
    for (int b = 0; b < 2; ++b) g_mbar_wait(g_smem_u32(bar_mma + b), 0);
    for (int b = 0; b < kGBRing; ++b) g_mbar_wait(g_smem_u32(bar_bfull + b), 0);
  }
  __syncthreads();
  g_dep_launch();  // the next kernel may start its set-up
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  // accumulator -> partials [128][kGPartLd] in the (idle) A and B stages: head + tail
  float* part = reinterpret_cast<float*>(A);
  const int prow = (warp & 3) * 32 + lane;
  for (int half = 0; half < 2; ++half) {
    uint32_t d[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) d[t] = 0u;
    if (ok && nch > 0) {
      const uint32_t taddr =
          tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * kGN + half * 32);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
          "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
            "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15]),
            "=r"(d[16]), "=r"(d[17]), "=r"(d[18]), "=r"(d[19]), "=r"(d[20]), "=r"(d[21]), "=r"(d[22]), "=r"(d[23]),
            "=r"(d[24]), "=r"(d[25]), "=r"(d[26]), "=r"(d[27]), "=r"(d[28]), "=r"(d[29]), "=r"(d[30]), "=r"(d[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    }
    if (warp < 4) {
#pragma unroll
      for (int t = 0; t < 32; ++t) part[prow * kGPartLd + half * 32 + t] = __uint_as_float(d[t]);
    }
    __syncthreads();
    if (warp >= 4) {
#pragma unroll
      for (int t = 0; t < 32; ++t) part[prow * kGPartLd + half * 32 + t] += __uint_as_float(d[t]);
    }
  }
  if (csize > 1) g_cluster_sync();  // every rank's partials complete before any rank reads them
  else __syncthreads();

  // epilogue: this rank finishes output rows [o0, o1) of the tile, adding the
  // ranks' partials in rank order
  const int nout = swiglu ? 64 : kGM;
  const int o0 = (int)crank * nout / (int)csize, o1 = ((int)crank + 1) * nout / (int)csize, no = o1 - o0;
  if (ok) {
    // the partials' base address in every rank's shared memory
    uint32_t base[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      base[q] = 0;
      if (q < (int)csize) asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(base[q]) : "r"(g_smem_u32(part)), "r"(q));
    }
    // kGE outputs per thread and round: every rank's partials of all of them in
    // flight (and the old values for a residual add), then each summed in rank order
    constexpr int kGE = 4;
    for (int i0 = tid; i0 < no * kGN; i0 += kGE * kGT) {
      float va[kGE], vb[kGE], yo[kGE];
      float xa[kGE][8], xv[kGE][8];
#pragma unroll
      for (int e = 0; e < kGE; ++e) {
        const int i = i0 + e * kGT;
        const int t = i / no, o = o0 + (i - t * no);
        const bool live = i < no * kGN && m0 + t < p.m_rows;
        const int gr = swiglu ? tile * 64 + o : tile * kGM + o;
        yo[e] = 0.0f;
        if (live && p.epi == GEMM_EPI_ADD && gr < p.rows_out) yo[e] = p.y[(int64_t)(m0 + t) * p.ldy + gr];
        const uint32_t off = (uint32_t)((o * kGPartLd + t) * 4);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          xa[e][q] = 0.0f;
          xv[e][q] = 0.0f;
          if (live && q < (int)csize) {
            if (csize == 1) {
              xa[e][q] = part[o * kGPartLd + t];
              if (swiglu) xv[e][q] = part[(o + 64) * kGPartLd + t];
            } else {
              asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(xa[e][q]) : "r"(base[q] + off));
              if (swiglu)
                asm volatile("ld.shared::cluster.f32 %0, [%1];"
                             : "=f"(xv[e][q])
                             : "r"(base[q] + off + 64 * kGPartLd * 4));
            }
          }
        }
      }
#pragma unroll
      for (int e = 0; e < kGE; ++e) {
        va[e] = 0.0f;
        vb[e] = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < (int)csize) {
            va[e] += xa[e][q];
            vb[e] += xv[e][q];
          }
        const int i = i0 + e * kGT;
        const int t = i / no, o = o0 + (i - t * no);
        if (i >= no * kGN || m0 + t >= p.m_rows) continue;
        float* yr = p.y + (int64_t)(m0 + t) * p.ldy;
        if (swiglu) {
          const int gr = tile * 64 + o;
          if (gr < p.rows_out) yr[gr] = silu(va[e] * s_ts[o >> 4]) * (vb[e] * s_ts[4 + (o >> 4)]);
        } else {
          const int gr = tile * kGM + o;
          if (gr < p.rows_out) {
            const float v = va[e] * s_ts[o >> 4];
            yr[gr] = p.epi == GEMM_EPI_ADD ? yo[e] + v : v;
          }
        }
      }
    }
  }
  // no rank leaves (and frees its shared memory) while another still reads it
  if (csize > 1) g_cluster_sync();
  if (!ok && tid == 0 && p.status) atomicCAS(p.status, 0, CB_ERR_TIMEOUT);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kGTmemCols));
}

cudaError_t launch_pdl(const void* fn, dim3 grid, int smem, cudaStream_t st, int cluster, const GemmParams& p) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = cluster;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  void* args[] = {const_cast<GemmParams*>(&p)};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

size_t gemm_scratch_bytes(int K, int m_rows) {
  if (K <= 0 || m_rows <= 0 || K % kGKc) return 0;
  return (size_t)ceil_div(m_rows, kGN) * (size_t)(K / kGKc) * kGBStage;
}

int launch_gemm(const GemmParams& p, cudaStream_t st) {
  if (!p.tiles || !p.tile_scale || !p.x || !p.y || !p.xb || p.m_rows < 1 || p.rows_out < 1) return CB_ERR_ARG;
  if (p.pre != GEMM_PRE_NONE && p.pre != GEMM_PRE_RMSNORM) return CB_ERR_ARG;
  if (p.epi != GEMM_EPI_STORE && p.epi != GEMM_EPI_ADD && p.epi != GEMM_EPI_SWIGLU) return CB_ERR_ARG;
  if (p.pre == GEMM_PRE_RMSNORM && !p.norm_w) return CB_ERR_ARG;
  const int K = p.K;
  if (K < kGKc || K % kGKc || K > 8192 || p.rows % kTileRows || p.rows < kTileRows) return CB_ERR_SHAPE;
  if (p.epi == GEMM_EPI_SWIGLU) {
    // gate rows [0, F) and up rows [F, 2F): F a multiple of 64 so that a tile's two halves are whole 16-row tiles
    if ((p.rows / 2) % 64 || p.rows_out > p.rows / 2) return CB_ERR_SHAPE;
  } else if (p.rows_out > p.rows) {
    return CB_ERR_ARG;
  }
  // 16-byte loads of x rows, packed code rows and norm weights; 16-byte bulk copies of the prepared blocks
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.ldx % 4) || p.ldx < K ||
      (reinterpret_cast<uintptr_t>(p.tiles) & 15) || (reinterpret_cast<uintptr_t>(p.xb) & 15) ||
      (p.norm_w && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)))
    return CB_ERR_ARG;
  if (p.xb_bytes < gemm_scratch_bytes(K, p.m_rows)) return CB_ERR_WORKSPACE;
  if (ensure_smem_attr((const void*)gemm_nvfp4_kernel, kGSmem) != CB_OK) return CB_ERR_CUDA;
  const int tiles = p.epi == GEMM_EPI_SWIGLU ? ceil_div(p.rows_out, 64) : ceil_div(p.rows_out, kGM);
  const int ntok = ceil_div(p.m_rows, kGN), nall = K / kGKc;
  if (ntok > 65535) return CB_ERR_SHAPE;
  // inputs: one warp per padded token row
  cudaError_t e = launch_pdl((const void*)gemm_prep_kernel, dim3(ntok * kGN / 2), 0, st, 1, p);
  count_launch();
  if (e != cudaSuccess) return CB_ERR_CUDA;
  // split K over a cluster of up to 8 CTAs while the grid stays within two CTAs per SM
  const int slots = 2 * num_sms();
  int S = 1;
  while (S < 8 && tiles * ntok * S * 2 <= slots && S * 2 <= nall) S *= 2;
  e = launch_pdl((const void*)gemm_nvfp4_kernel, dim3(tiles * S, ntok), kGSmem, st, S, p);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

using namespace cb;

extern "C" size_t cb_gemm_scratch_bytes(int32_t k, int32_t m_rows) { return gemm_scratch_bytes(k, m_rows); }

extern "C" int cb_gemm_nvfp4(const CbMatrix* w, const float* x, int32_t ldx, int32_t m_rows, int32_t pre,
                             const float* norm_w, float eps, float* y, int32_t ldy, int32_t rows_out, int32_t epi,
                             void* scratch, size_t scratch_bytes, int32_t* status, void* stream) {
  if (!w || !w->tiles || !w->tile_scale || !scratch) return CB_ERR_ARG;
  if (ldy < rows_out) return CB_ERR_ARG;
  GemmParams p{};
  p.tiles = w->tiles;
  p.tile_scale = w->tile_scale;
  p.rows = w->rows;
  p.K = w->k;
  p.x = x;
  p.ldx = ldx;
  p.m_rows = m_rows;
  p.pre = pre;
  p.norm_w = norm_w;
  p.eps = eps;
  p.y = y;
  p.ldy = ldy;
  p.rows_out = rows_out;
  p.epi = epi;
  p.xb = static_cast<uint8_t*>(scratch);
  p.xb_bytes = scratch_bytes;
  p.status = status;
  return launch_gemm(p, (cudaStream_t)stream);
}
