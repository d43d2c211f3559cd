// Many-token NVFP4 GEMM on the 5th-generation tensor cores (tcgen05):
//   y[m][r] (=, +=) sum_k pre(x)[m][k] * dequant(W)[r][k]        m < m_rows
//
// This is the contraction of a step that carries many token rows at once:
// batched decode (B sequences x 1 token), batched verify (B x (1 + draft)) and
// prompt chunks.  The CUDA-core GEMV re-reads the weights for every 16 token
// rows; here each weight tile is read once per 32 tokens and the products run
// on the tensor pipe.
//
// One CTA owns a 128-row tile of W and 32 token rows of x (a cluster of up to
// 8 CTAs splits K):
//   * W: every K chunk of 64 (128 rows x 32 code bytes, 4 scale bytes per row)
//     and the chunk's 32 x 64 float inputs come by cp.async into a ring of
//     kGRing raw stages, kGRing - 1 chunks ahead.  Each thread copies exactly
//     the bytes it converts, so no barrier sits between copy and conversion.
//   * A (weights): E2M1 pairs go to f16x2 by the hardware converter and are
//     multiplied by the E4M3 block scale, also f16: every E2M1 x E4M3 product
//     has at most 6 significant bits and lies in [2^-10, 2688], so the f16
//     operand is exact.
//   * B (activations): each input x (RMSNorm applied when asked) is split into
//     an f16 head and an f16 tail, hi = f16(x), lo = f16(x - hi): the MMA's
//     N = 64 columns are 32 head rows and 32 tail rows, and the epilogue adds
//     the two, so the products carry about 22 bits of every input.
//   * one thread issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N 64,
//     K 16) x 4 per chunk into an fp32 accumulator in tensor memory and
//     commits to the stage's mbarrier; two A/B stages alternate.
//   * epilogue: tcgen05.ld (warps 0-3 the head columns, 4-7 the tail columns
//     of their lane quarter) -> shared memory; with split K the cluster's
//     partials are added in rank order through distributed shared memory,
//     each rank finishing a slice of the rows; then the tile scale and the
//     store / residual add / SwiGLU (gate row r and up row F + r in one tile).
// RMSNorm (layers.py:39-44): the CTA first reduces the sums of squares of its
// 32 token rows over the whole K, then stages x * rsqrt(mean + eps) * norm_w.
// Every mbarrier wait is bounded (%globaltimer); on timeout the launch sets its
// status word, skips the rest of the work, and still frees its tensor memory.
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemm.cuh"

namespace cb {
namespace {

constexpr int kGT = 256;                  // threads
constexpr int kGM = 128;                  // W rows per CTA (MMA M)
constexpr int kGN = 32;                   // token rows per CTA
constexpr int kGNm = 2 * kGN;             // MMA N: head and tail rows
constexpr int kGKc = 64;                  // K per chunk
constexpr int kGRing = 4;                 // raw chunks in flight
constexpr int kGAStage = kGM * kGKc * 2;  // 16 KB f16
constexpr int kGBStage = kGNm * kGKc * 2; // 8 KB f16
constexpr int kGRawCodes = kGM * kGKc / 2;         // 4 KB
constexpr int kGRawScales = kGT * 4;               // 1 KB: each thread its row's 4 scale bytes
constexpr int kGRawX = kGN * kGKc * 4;             // 8 KB
constexpr int kGRawStage = kGRawCodes + kGRawScales + kGRawX;
constexpr int kGSmem = 2 * (kGAStage + kGBStage) + kGRing * kGRawStage;
constexpr int kGPartLd = kGN + 1;
constexpr int kGTmemCols = 64;
constexpr unsigned long long kGTimeoutNs = 200ull * 1000 * 1000;
static_assert(kGM * kGPartLd * 4 <= 2 * kGAStage, "partials live in the A stages");

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

__global__ void __launch_bounds__(kGT, 2) gemm_nvfp4_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  __shared__ __align__(8) unsigned long long bar_mma[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  __shared__ float s_rn[kGN];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t crank, csize;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  const int K = p.K, nall = K / kGKc;
  const int tile = (int)(blockIdx.x / csize);
  const int m0 = (int)blockIdx.y * kGN;
  const int cbeg = (int)crank * nall / (int)csize, nch = ((int)crank + 1) * nall / (int)csize - cbeg;
  const bool swiglu = p.epi == GEMM_EPI_SWIGLU;
  const int half_rows = p.rows / 2;  // SwiGLU: gate rows [0, F), up rows [F, 2F)
  uint8_t* A = gsm;                               // [2][16 KB]
  uint8_t* Bs = gsm + 2 * kGAStage;               // [2][8 KB]
  uint8_t* raw = Bs + 2 * kGBStage;               // [kGRing][codes | scales | x]

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(g_smem_u32(bar_mma + b)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g_smem_u32(&tmem_base)),
                 "n"(kGTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }

  // this thread's weight row (r) and K half (h) of every chunk, and its x pair (token xt, K block xkb)
  const int r = tid >> 1, h = tid & 1;
  int grow;
  if (swiglu) grow = r < 64 ? tile * 64 + r : half_rows + tile * 64 + (r - 64);
  else grow = tile * kGM + r;
  const bool rvalid = swiglu ? (tile * 64 + (r & 63)) < half_rows : grow < p.rows;
  const int64_t tb = 9ll * K;
  const uint8_t* codes = p.tiles + (int64_t)(grow >> 4) * tb + (grow & 15) * (K / 2) + 16 * h;
  const uint8_t* scl = p.tiles + (int64_t)(grow >> 4) * tb + kTileRows * (K / 2) + (grow & 15) * (K / 16);
  const int xt = tid >> 3, xkb = tid & 7;
  const bool xvalid = m0 + xt < p.m_rows;
  const float* xrow = p.x + (int64_t)(m0 + xt) * p.ldx + xkb * 8;
  const uint32_t raw_s = g_smem_u32(raw);

  auto issue = [&](int c) {
    if (c < nch) {
      const uint32_t rs = raw_s + (uint32_t)((c % kGRing) * kGRawStage);
      const int kc = cbeg + c;
      if (rvalid) {
        g_cp16(rs + r * 32 + 16 * h, codes + kc * 32);
        g_cp4(rs + kGRawCodes + tid * 4, scl + kc * 4);
      }
      if (xvalid) {
        const float* src = xrow + kc * kGKc;
        g_cp16(rs + kGRawCodes + kGRawScales + tid * 32, src);
        g_cp16(rs + kGRawCodes + kGRawScales + tid * 32 + 16, src + 4);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int j = 0; j < kGRing - 1; ++j) issue(j);

  // RMSNorm factors of the CTA's token rows over the whole K (rows in L2)
  if (p.pre == GEMM_PRE_RMSNORM) {
    for (int t = warp; t < kGN; t += kGT / 32) {
      float ss = 0.0f;
      if (m0 + t < p.m_rows) {
        const float4* xr = reinterpret_cast<const float4*>(p.x + (int64_t)(m0 + t) * p.ldx);
        for (int i = lane; i < K / 4; i += 32) {
          const float4 v = __ldcg(xr + i);
          ss = fmaf(v.x, v.x, ss);
          ss = fmaf(v.y, v.y, ss);
          ss = fmaf(v.z, v.z, ss);
          ss = fmaf(v.w, v.w, ss);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_rn[t] = rsqrtf(ss / (float)K + p.eps);
    }
  } else if (tid < kGN) {
    s_rn[tid] = 1.0f;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const float rn = s_rn[xt];

  unsigned par[2] = {0u, 0u};
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int st = c & 1;
    issue(c + kGRing - 1);  // its ring slot held chunk c - 1, which this thread converted already
    asm volatile("cp.async.wait_group %0;" ::"n"(kGRing - 1) : "memory");
    // the MMAs of chunk c - 2 read this stage: wait for their commit
    if (c >= 2) {
      if (!g_mbar_wait(g_smem_u32(bar_mma + st), par[st])) s_abort = 1;
      par[st] ^= 1u;
    }
    const uint8_t* rsp = raw + (c % kGRing) * kGRawStage;
    const int kc = cbeg + c;
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
    // B: token xt, K block xkb -> head row xt and tail row kGN + xt
    {
      float v[8];
      if (xvalid) {
        const float4 a = *reinterpret_cast<const float4*>(rsp + kGRawCodes + kGRawScales + tid * 32);
        const float4 b = *reinterpret_cast<const float4*>(rsp + kGRawCodes + kGRawScales + tid * 32 + 16);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        if (p.pre == GEMM_PRE_RMSNORM) {
          const float4 n0 = __ldg(reinterpret_cast<const float4*>(p.norm_w + kc * kGKc + xkb * 8));
          const float4 n1 = __ldg(reinterpret_cast<const float4*>(p.norm_w + kc * kGKc + xkb * 8 + 4));
          const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = v[i] * rn * nw[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
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
      uint8_t* Bst = Bs + st * kGBStage;
      *reinterpret_cast<uint4*>(Bst + g_off(xt, xkb)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(Bst + g_off(kGN + xt, xkb)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    // generic-proxy stores -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (s_abort) {
      ok = false;
      break;
    }
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t as = g_smem_u32(A + st * kGAStage), bs = g_smem_u32(Bs + st * kGBStage);
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
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA
  if (ok && nch > 0) {
    // the last commit covers every MMA issued before it
    const int st = (nch - 1) & 1;
    if (!g_mbar_wait(g_smem_u32(bar_mma + st), par[st])) s_abort = 1;
    __syncthreads();
    ok = !s_abort;
  } else if (!ok) {
    // give the MMAs already issued a bounded time to finish before their memory is reused or freed
    if (tid == 0)
      for (int st = 0; st < 2; ++st) g_mbar_wait(g_smem_u32(bar_mma + st), par[st]);
    __syncthreads();
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  // accumulator -> partials [128][kGPartLd] in the (idle) A stages: head + tail
  float* part = reinterpret_cast<float*>(A);
  uint32_t d[32];
#pragma unroll
  for (int t = 0; t < 32; ++t) d[t] = 0u;
  if (ok && nch > 0) {
    const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * kGN);
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
  const int prow = (warp & 3) * 32 + lane;
  if (warp < 4) {
#pragma unroll
    for (int t = 0; t < kGN; ++t) part[prow * kGPartLd + t] = __uint_as_float(d[t]);
  }
  __syncthreads();
  if (warp >= 4) {
#pragma unroll
    for (int t = 0; t < kGN; ++t) part[prow * kGPartLd + t] += __uint_as_float(d[t]);
  }
  if (csize > 1) g_cluster_sync();  // every rank's partials complete before any rank reads them
  else __syncthreads();

  // epilogue: this rank finishes output rows [o0, o1) of the tile, adding the
  // ranks' partials in rank order
  const int nout = swiglu ? 64 : kGM;
  const int o0 = (int)crank * nout / (int)csize, o1 = ((int)crank + 1) * nout / (int)csize, no = o1 - o0;
  if (ok) {
    for (int i = tid; i < no * kGN; i += kGT) {
      const int t = i / no, o = o0 + (i - t * no);
      if (m0 + t >= p.m_rows) continue;
      float va = 0.0f, vb = 0.0f;
      for (uint32_t q = 0; q < csize; ++q) {
        const float* pa = part + o * kGPartLd + t;
        if (csize == 1) {
          va += *pa;
          if (swiglu) vb += pa[64 * kGPartLd];
        } else {
          uint32_t ra;
          float x;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(g_smem_u32(pa)), "r"(q));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(ra) : "memory");
          va += x;
          if (swiglu) {
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(g_smem_u32(pa + 64 * kGPartLd)), "r"(q));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(ra) : "memory");
            vb += x;
          }
        }
      }
      float* yr = p.y + (int64_t)(m0 + t) * p.ldy;
      if (swiglu) {
        const int gr = tile * 64 + o;
        if (gr < p.rows_out) {
          const float g = va * p.tile_scale[gr >> 4];
          const float u = vb * p.tile_scale[(half_rows + gr) >> 4];
          yr[gr] = silu(g) * u;
        }
      } else {
        const int gr = tile * kGM + o;
        if (gr < p.rows_out) {
          const float v = va * p.tile_scale[gr >> 4];
          if (p.epi == GEMM_EPI_ADD) yr[gr] += v;
          else yr[gr] = v;
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

}  // namespace

int gemm_tokens_per_cta() { return kGN; }

int launch_gemm(const GemmParams& p, cudaStream_t st) {
  if (!p.tiles || !p.tile_scale || !p.x || !p.y || p.m_rows < 1 || p.rows_out < 1) return CB_ERR_ARG;
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
  // 16-byte copies of x rows and of the packed code rows
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.ldx % 4) || p.ldx < K ||
      (reinterpret_cast<uintptr_t>(p.tiles) & 15) || (p.norm_w && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)))
    return CB_ERR_ARG;
  if (ensure_smem_attr((const void*)gemm_nvfp4_kernel, kGSmem) != CB_OK) return CB_ERR_CUDA;
  const int tiles = p.epi == GEMM_EPI_SWIGLU ? ceil_div(p.rows_out, 64) : ceil_div(p.rows_out, kGM);
  const int ntok = ceil_div(p.m_rows, kGN), nall = K / kGKc;
  if (ntok > 65535) return CB_ERR_SHAPE;
  // split K over a cluster of up to 8 CTAs while the grid stays within two CTAs per SM
  const int slots = 2 * num_sms();
  int S = 1;
  while (S < 8 && tiles * ntok * S * 2 <= slots && S * 2 <= nall) S *= 2;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles * S, ntok);
  cfg.blockDim = dim3(kGT);
  cfg.dynamicSmemBytes = kGSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_nvfp4_kernel, p);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_gemm_nvfp4(const CbMatrix* w, const float* x, int32_t ldx, int32_t m_rows, int32_t pre,
                             const float* norm_w, float eps, float* y, int32_t ldy, int32_t rows_out, int32_t epi,
                             int32_t* status, void* stream) {
  if (!w || !w->tiles || !w->tile_scale) return CB_ERR_ARG;
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
  p.status = status;
  return launch_gemm(p, (cudaStream_t)stream);
}
