// Persistent decode kernel: one launch runs a whole forward chunk of
// M = batch * T <= 8 rows (a tau=1 decode step, or a verify of 1 + draft
// tokens), with every CTA resident, walking the model phase by phase.
//
// The grid is a set of 8-CTA thread-block clusters.  Phases, each ended by a
// grid barrier (bounded waits on one monotonic counter):
//   GDN layer:  [mixer]  one cluster per head: in-projection rows of the head
//                        (2 tiles per CTA) -> distributed shared memory ->
//                        short conv, L2 norms, decay / beta -> the recurrence on
//                        the CTA's Dv/8 value columns -> gated RMSNorm (sums of
//                        squares exchanged in the cluster) -> split-K o-projection
//                        on the CTA's columns -> partials summed in the cluster
//                        -> added to the residual stream
//               [FFN]    split K: each CTA one 16-wide slice of the hidden layer
//                        (its gate and up tiles, SwiGLU, the matching 16 columns
//                        of the down projection) -> partials summed in the cluster
//                        -> added to the residual stream
//   SWA layer:  [mixer]  one cluster per query head: the head's q, k, v and gate
//                        rows -> distributed shared memory -> q / k RMSNorm +
//                        RoPE (ring append) -> each CTA attends over an eighth of
//                        the window -> partials merged in the cluster -> the
//                        head's column block of the o-projection on the CTA's
//                        d/8 output rows -> added to the residual stream
//               [FFN]
//   shared KV:  projection GEMV -> K/V/indexer-key append + indexer scores with a
//               2048-bin histogram (and the cross residual stream initialised)
//               -> threshold bin + compaction -> exact selection (one CTA per
//               query row)
//   cross layer: [mixer] as the SWA mixer, q and gate rows only, over the
//               selected keys of the shared cache -> [FFN]
//   head:       LM-head GEMV (final norm fused) with a per-row argmax
//
// The residual streams are kept in 64-bit fixed point (value * 2^32) and every
// update is an integer atomic add, so the split-K sums are exact and the
// result does not depend on the order in which CTAs finish.  Each phase's
// weights are staged into one of two shared-memory slots by bulk copies
// (cp.async.bulk, completion on an mbarrier) issued one phase ahead.
//
// Every wait is bounded (%globaltimer): on timeout a CTA sets CB_ERR_TIMEOUT and
// an abort bit in the barrier counter; from then on every CTA skips the work
// but still takes its cluster barriers, so no CTA is left waiting for a
// cluster peer, and the launch ends without advancing the cache.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "mk.cuh"
#include "nvfp4.cuh"

namespace cb {
namespace {

constexpr int kT = kMkThreads;
constexpr int kW = kMkThreads / 32;   // 16 warps: one per row of a weight tile
constexpr int kCl = kMkCluster;
constexpr int kSlot = kMkSlotBytes;
constexpr int kWork = kMkWorkBytes;
// Parameter region at the end of the work area: each phase's small operands
// (norm vector, tile and tensor scales, gate constants, conv taps and windows)
// are copied here between the arrival at the barrier before the phase and the
// wait there.  No other CTA writes it, and no phase that needs parameters
// uses it as scratch.
constexpr int kPreOff = kWork - 21 * 1024;
constexpr int kParNorm = 0;                      // [kMkMaxD] norm vector
constexpr int kParSmall = kMkMaxD;               // [64] scales and constants
constexpr int kParConv = kMkMaxD + 80;           // conv taps [NC][4], then windows [B][3][NC]
constexpr int kParTs = 48;                       // tile scales held for the first 48 units of a GEMV
enum { PS_A_LOG = 48, PS_DT_BIAS = 49, PS_TSCALE = 50, PS_O_NORM = 52 };  // indices in the small block (80)
constexpr int kMarkBase = 256;                   // trace entries kMarkBase + 6 p + i: sub-phase marks of CTA 0
constexpr int kSmem = 2 * kSlot + kWork;
constexpr int kMaxSort = 4096;
constexpr int kMkBitmapWords = 4096;  // selection bitmap: up to 131072 keys
constexpr int kMaxPhases = 4 * CB_MAX_SELF + 4 * CB_MAX_CROSS + 8;
constexpr unsigned kAbortBit = 1u << 30;
constexpr float kFix = 4294967296.0f;              // 2^32
constexpr float kFixInv = 2.3283064365386963e-10f;  // 2^-32

enum { PRE_NONE_ = 0, PRE_RMS_ = 1, PRE_EMBED_ = 2 };
enum { EPI_STORE_ = 0, EPI_RED_ = 1 };
enum : int {
  PH_GDN = 0, PH_FFN_SELF, PH_SWA_HEAD, PH_SH_PROJ, PH_SH_SCORE, PH_SH_COMPACT, PH_CR_RESOLVE, PH_CR_HEAD,
  PH_FFN_CROSS, PH_LM_HEAD
};

// ------------------------------------------------------------------ timers, sync
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Per-CTA copy of the launch's wait limit and stall hook (thread 0 reads them at start).
__shared__ unsigned long long s_wait_limit;
__shared__ unsigned s_stall_barrier;

__shared__ int s_mark_base;  // trace entry of this phase's first sub-phase mark

// %globaltimer at a point inside the current phase (CTA 0 only; i < 6).
__device__ __forceinline__ void mark(const MkArgs& a, int i) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && s_mark_base + i < kMkTrace) a.trace[s_mark_base + i] = gtimer();
}

__device__ __forceinline__ void raise_abort(const MkArgs& a) {
  atomicOr(a.sync, kAbortBit);
  atomicCAS(a.status, 0, CB_ERR_TIMEOUT);
}

// Grid barrier on a monotonic arrival counter, split in two: grid_arrive
// publishes this CTA's writes and counts it in; grid_wait waits for every CTA.
// Work that does not depend on the other CTAs' writes (the next phase's weight
// copies, recurrent state) goes between the two.  The abort bit in the counter
// ends every wait at once; grid_wait returns false when the launch is aborted.
// The barrier is taken by lane 0 of the last warp and the weight copies are
// issued by another warp, so that neither waits for the arrival to drain this
// CTA's writes.
constexpr int kBarThread = kT - 32;
constexpr int kCopyWarp = kW - 2;  // issues the weight copies (warp 0 carries the most preload work)

__device__ __forceinline__ void grid_arrive(const MkArgs& a, unsigned& gen) {
  __syncthreads();
  gen += 1;
  if (threadIdx.x == kBarThread) {
    if (blockIdx.x == 0 && 2 * gen < (unsigned)kMkTrace) a.trace[2 * gen - 1] = gtimer();
    // a release add at GPU scope: the CTA's writes (ordered before it by the
    // CTA barrier) are visible to every CTA that acquires the count
    // the test hook leaves this barrier one arrival short, so every wait on it runs out
    if (!(blockIdx.x == 0 && gen == s_stall_barrier))
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync) : "memory");
  }
}

__device__ __forceinline__ bool grid_wait(const MkArgs& a, unsigned gen, int* s_ok) {
  if (threadIdx.x == kBarThread) {
    const unsigned target = gen * gridDim.x;
    int ok = 1;
    const unsigned long long t0 = gtimer();
    unsigned spin = 0;
    for (;;) {
      const unsigned v = ld_acquire_u32(a.sync);
      if (v & kAbortBit) {
        ok = 0;
        break;
      }
      if (v >= target) break;
      if ((++spin & 63) == 0 && gtimer() - t0 > s_wait_limit) {
        raise_abort(a);
        ok = 0;
        break;
      }
    }
    if (blockIdx.x == 0 && 2 * gen < (unsigned)kMkTrace) a.trace[2 * gen] = gtimer();
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// ------------------------------------------------------------------ clusters
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cluster_index() {
  unsigned r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Cluster barrier: orders this CTA's shared-memory stores to the cluster's CTAs
// before every CTA's later reads.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem(const void* p, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ------------------------------------------------------------------ bulk copies
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_arrive(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for an mbarrier phase (every thread waits, so every thread sees the copied bytes).
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (!mbar_try(bar, parity))
    if (gtimer() - t0 > s_wait_limit) return false;
  return true;
}
// Global -> this CTA's shared memory, completion counted on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Asynchronous global -> shared copies of small pieces (no registers held while they fly)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Every committed group but the most recent one complete.
__device__ __forceinline__ void cp_async_wait_prior() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// ------------------------------------------------------------------ fixed point
__device__ __forceinline__ float from_fix(long long q) { return __ll2float_rn(q) * kFixInv; }
__device__ __forceinline__ void red_fix(long long* p, float v) {
  const unsigned long long q = (unsigned long long)__float2ll_rn(v * kFix);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(q) : "memory");
}

// ------------------------------------------------------------------ staged inputs
// A staged input row of K floats keeps 16 bytes of padding after every 32
// floats: the 8-float chunks that lanes 0-7 of a warp read with 128-bit loads
// (chunks 32 bytes apart) then fall on 32 distinct banks.
__host__ __device__ inline int xpad(int K) { return K + K / 8; }           // floats per staged row
__host__ __device__ inline int xoff(int k) { return k + (k >> 5) * 4; }    // position of element k in its row

// ------------------------------------------------------------------ weight rows
// One weight row as seen by one lane: the 8-code chunks lane, lane+32, ...
// (K <= 2048, so at most 8 chunks), code words and scale bytes.
template <int NU>
struct RowW {
  uint32_t w[NU];
  uint32_t s[NU];
};

// Row `w` of a 16-row tile (codes of the 16 rows, then their scales), in shared
// or global memory.
template <int NU>
__device__ __forceinline__ void tile_row(const uint8_t* tile, int K, int w, bool valid, bool global, RowW<NU>& r,
                                         int trows = kTileRows) {
  const int lane = threadIdx.x & 31, kc = K >> 3;
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(tile + w * (K / 2));
  const uint8_t* sb = tile + trows * (K / 2) + w * (K / 16);
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int c = u * 32 + lane;
    const bool ok = valid && c < kc;
    if (global) {
      r.w[u] = ok ? __ldg(cw + c) : 0u;
      r.s[u] = ok ? (uint32_t)__ldg(sb + (c >> 1)) : 0u;
    } else {
      r.w[u] = ok ? cw[c] : 0u;
      r.s[u] = ok ? (uint32_t)sb[c >> 1] : 0u;
    }
  }
}

template <int M, int NU>
__device__ __forceinline__ void dot_row(const RowW<NU>& r, int K, const float* xs, float (&acc)[M]) {
  const int lane = threadIdx.x & 31, kc = K >> 3;
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int c = u * 32 + lane;
    if (c < kc) {
      const float sc = e4m3_to_f32(r.s[u]);
      float2 f[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = e2m1x2_to_f32x2(r.w[u] >> (8 * j));
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float* xc = xs + m * xpad(K) + xoff(c * 8);
        const float4 x0 = *reinterpret_cast<const float4*>(xc);
        const float4 x1 = *reinterpret_cast<const float4*>(xc + 4);
        float p = f[0].x * x0.x;
        p = fmaf(f[0].y, x0.y, p);
        p = fmaf(f[1].x, x0.z, p);
        p = fmaf(f[1].y, x0.w, p);
        p = fmaf(f[2].x, x1.x, p);
        p = fmaf(f[2].y, x1.y, p);
        p = fmaf(f[3].x, x1.z, p);
        p = fmaf(f[3].y, x1.w, p);
        acc[m] = fmaf(p, sc, acc[m]);
      }
    }
  }
}

// Dot products of one tile row with the M staged input rows: acc[m] holds the
// warp-reduced sum on every lane.  A tile holds trows rows (codes, then scales).
template <int M>
__device__ __forceinline__ void row_dot(const uint8_t* tile, int K, int w, bool valid, bool global, const float* xs,
                                        float (&acc)[M], int trows = kTileRows) {
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.0f;
  if (K <= 768) {
    RowW<3> r;
    tile_row<3>(tile, K, w, valid, global, r, trows);
    dot_row<M, 3>(r, K, xs, acc);
  } else {
    RowW<8> r;
    tile_row<8>(tile, K, w, valid, global, r, trows);
    dot_row<M, 8>(r, K, xs, acc);
  }
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = warp_sum(acc[m]);
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, int idx) {
  return ((unsigned long long)score_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}

// ------------------------------------------------------------------ RMSNorm staging
// xs[m][xoff(k)] = x[m][k] * norm_w[k] (rows xpad(K) floats apart) for m < m_rows
// (zeros above); rn[m] receives the RMSNorm factor of each row (1 when norm_w is
// null).  x comes from a fixed-point residual row (xq, row rowmap[m]), float rows
// (x) or the token embeddings (embed_from).  The sums of squares are reduced in a
// fixed order.
template <int M>
__device__ void stage_rows(const long long* xq, const float* x, int ldx, const int* rowmap, int m_rows, int K,
                           const float* norm_w, float eps, float* xs, float (&rn)[M], long long* copy_q,
                           long long* embed_add, const MkArgs* embed_from) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ float wsq[kW][kMkMaxRows];
  float sq[M];
#pragma unroll
  for (int m = 0; m < M; ++m) sq[m] = 0.0f;
  const bool norm = norm_w != nullptr;
  for (int i = tid; i < M * K; i += kT) {
    const int mr = i / K, k = i - mr * K;
    float v = 0.0f;
    if (mr < m_rows) {
      if (embed_from) {  // the token's embedding row (tied with the LM head, gathered from its tiles)
        const MkArgs& a = *embed_from;
        const CbMatrix& E = a.m.lm_head;
        const int b = mr / a.T, t = mr - b * a.T;
        const int64_t id = a.ids[(int64_t)b * a.ids_ld + a.c0 + t];
        if (id >= 0 && id < a.m.vocab_size) {
          const uint8_t* tile = E.tiles + (id >> 4) * tile_bytes(K);
          const int rr = (int)(id & 15);
          const float2 f = e2m1x2_to_f32x2(tile[rr * (K / 2) + (k >> 1)]);
          const float s = e4m3_to_f32(tile[kTileRows * (K / 2) + rr * (K / 16) + (k >> 4)]);
          v = ((k & 1 ? f.y : f.x) * s) * E.tile_scale[id >> 4];
        } else if (k == 0) {
          set_status(a.status, CB_ERR_TOKEN);
        }
        if (embed_add) red_fix(embed_add + (int64_t)mr * K + k, v);
      } else {
        const int xr = rowmap ? rowmap[mr] : mr;
        if (xq) {
          const long long q = __ldcg(xq + (int64_t)xr * ldx + k);
          v = from_fix(q);
          if (copy_q) copy_q[(int64_t)mr * ldx + k] = q;
        } else {
          v = __ldcg(x + (int64_t)xr * ldx + k);
        }
      }
    }
    if (norm) {
#pragma unroll
      for (int q = 0; q < M; ++q)
        if (q == mr) sq[q] += v * v;
      v *= norm_w[k];
    }
    xs[mr * xpad(K) + xoff(k)] = v;
  }
  if (norm) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float t = warp_sum(sq[m]);
      if (lane == 0) wsq[warp][m] = t;
    }
  }
  __syncthreads();
#pragma unroll
  for (int m = 0; m < M; ++m) {
    rn[m] = 1.0f;
    if (norm) {
      float t = 0.0f;
      for (int w = 0; w < kW; ++w) t += wsq[w][m];
      rn[m] = rsqrtf(t / (float)K + eps);
    }
  }
}

// ------------------------------------------------------------------ GEMV over tiles
struct GemvJob {
  CbMatrix W;
  const long long* xq;  // fixed-point input rows (or null)
  const float* x;       // float input rows (when xq is null)
  int ldx;
  int pre;
  const float* norm_w;
  float* y;             // EPI_STORE_
  long long* yq;        // EPI_RED_: y is added to this fixed-point stream
  int ldy, rows_out, epi;
  bool argmax;
  int ucta, uncta;      // this CTA's index among the phase's CTAs and their count (units ucta + i * uncta)
};

__device__ __forceinline__ int gemv_mine(const GemvJob& g) {
  const int units = g.W.rows / kTileRows;
  if (g.ucta < 0 || g.ucta >= units || g.uncta <= 0) return 0;
  return (units - 1 - g.ucta) / g.uncta + 1;
}
__device__ __forceinline__ int gemv_staged(const GemvJob& g) {
  return min(gemv_mine(g), (int)(kSlot / tile_bytes(g.W.k)));
}
// Tiles after the staged ones that the last phase copies into the other slot
// (free once the phase before it is done).
__device__ __forceinline__ int gemv_extra(const GemvJob& g) {
  return max(0, min(gemv_mine(g) - gemv_staged(g), (int)(kSlot / tile_bytes(g.W.k))));
}

__device__ __forceinline__ float* par_norm(float* work) { return work + kPreOff / 4 + kParNorm; }
__device__ __forceinline__ float* par_small(float* work) { return work + kPreOff / 4 + kParSmall; }

template <int M>
__device__ void gemv_phase(const MkArgs& a, const GemvJob& g, int m_rows, const uint8_t* slot, const uint8_t* slot2,
                           int nst2, float* work) {
  const int n_mine = gemv_mine(g);
  if (n_mine == 0) return;
  const float* ps = par_small(work);
  const int K = g.W.k, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tb = tile_bytes(K);
  const int nst = gemv_staged(g);
  float* xs = work;  // [M][xpad(K)]
  __shared__ unsigned long long s_best[kMkMaxRows];
  __shared__ int s_rowmap[kMkMaxRows];
  if (g.argmax && tid < kMkMaxRows) s_best[tid] = 0ull;
  if (tid < kMkMaxRows) s_rowmap[tid] = tid;
  __syncthreads();
  float rn[M];
  const bool first = g.ucta == 0;
  stage_rows<M>(g.xq, g.x, g.ldx, s_rowmap, m_rows, K, g.pre == PRE_NONE_ ? nullptr : par_norm(work), a.m.norm_eps,
                xs, rn, nullptr, (g.pre == PRE_EMBED_ && first) ? a.hq : nullptr,
                g.pre == PRE_EMBED_ ? &a : nullptr);
  mark(a, 0);

  unsigned long long best[M];
#pragma unroll
  for (int mr = 0; mr < M; ++mr) best[mr] = 0ull;
  for (int i = 0; i < n_mine; i += 2) {
    const int ua = g.ucta + i * g.uncta, ub = ua + g.uncta;
    const bool hb = i + 1 < n_mine;
    const int ra = ua * kTileRows + warp, rb = ub * kTileRows + warp;
    // tile i: the phase's slot, then the second slot, then global memory
    const bool ga = i >= nst + nst2, gb = i + 1 >= nst + nst2;
    const uint8_t* ta = ga ? g.W.tiles + ua * tb : (i < nst ? slot + i * tb : slot2 + (i - nst) * tb);
    const uint8_t* tbb = gb ? g.W.tiles + ub * tb : (i + 1 < nst ? slot + (i + 1) * tb : slot2 + (i + 1 - nst) * tb);
    float aa[M], ab[M];
    row_dot<M>(ta, K, warp, true, ga, xs, aa);
    if (hb) row_dot<M>(tbb, K, warp, true, gb, xs, ab);
    const float tsa = i < kParTs ? ps[i] : g.W.tile_scale[ua];
    const float tsb = hb ? (i + 1 < kParTs ? ps[i + 1] : g.W.tile_scale[ub]) : 0.0f;
#pragma unroll
    for (int mr = 0; mr < M; ++mr) {
      const float va = aa[mr] * tsa * rn[mr];
      const float vb = hb ? ab[mr] * tsb * rn[mr] : 0.0f;
      if (g.argmax) {
        if (ra < g.rows_out) best[mr] = max(best[mr], pack_argmax(va, ra));
        if (hb && rb < g.rows_out) best[mr] = max(best[mr], pack_argmax(vb, rb));
      }
      if (lane == mr && mr < m_rows) {  // one lane per input row writes
        if (g.epi == EPI_RED_) {
          long long* yr = g.yq + (int64_t)mr * g.ldy;
          if (ra < g.rows_out) red_fix(yr + ra, va);
          if (hb && rb < g.rows_out) red_fix(yr + rb, vb);
        } else {
          float* yr = g.y + (int64_t)mr * g.ldy;
          if (ra < g.rows_out) yr[ra] = va;
          if (hb && rb < g.rows_out) yr[rb] = vb;
        }
      }
    }
  }
  if (g.argmax) {
    if (lane == 0)
#pragma unroll
      for (int mr = 0; mr < M; ++mr)
        if (mr < m_rows) atomicMax(&s_best[mr], best[mr]);
    __syncthreads();
    if (tid < m_rows) atomicMax(&a.amax[tid], s_best[tid]);
  }
}

// ------------------------------------------------------------------ GDN (cluster per head)
struct GdnGeo {
  int H, Dk, Dv, vpr, v0, HP, ntile, NC, RC, d;
};

__device__ __forceinline__ GdnGeo gdn_geo(const CbModel& m, int rank) {
  GdnGeo g;
  g.H = m.gdn_heads;
  g.Dk = m.gdn_dk;
  g.Dv = m.gdn_dv;
  g.vpr = g.Dv / kCl;
  g.v0 = rank * g.vpr;
  g.HP = 2 * g.Dk + 2 * g.Dv + 2;
  g.ntile = (2 * g.Dk + 2 * g.Dv) / kTileRows;
  g.NC = 2 * g.Dk + g.vpr;
  g.RC = m.d_model / kCl;
  g.d = m.d_model;
  return g;
}

// In-projection tile of entry j of head h's tile list (q tiles, k tiles, v tiles,
// gate tiles), and the offset of its first row in the head's output vector.
__device__ __forceinline__ int gdn_head_tile(const CbModel& m, const GdnGeo& g, int h, int j, int& hp_off) {
  const int qt = g.Dk / kTileRows, vt = g.Dv / kTileRows;
  if (j < qt) {
    hp_off = j * kTileRows;
    return (h * g.Dk) / kTileRows + j;
  }
  j -= qt;
  if (j < qt) {
    hp_off = g.Dk + j * kTileRows;
    return (g.H * g.Dk + h * g.Dk) / kTileRows + j;
  }
  j -= qt;
  if (j < vt) {
    hp_off = 2 * g.Dk + j * kTileRows;
    return (2 * g.H * g.Dk + h * g.Dv) / kTileRows + j;
  }
  j -= vt;
  hp_off = 2 * g.Dk + g.Dv + j * kTileRows;
  return (m.gdn_off_gate + h * g.Dv) / kTileRows + j;
}

// Global channel of conv channel c of this rank (q: Dk, k: Dk, v: the rank's vpr columns).
__device__ __forceinline__ int gdn_channel(const GdnGeo& g, int h, int c) {
  if (c < g.Dk) return h * g.Dk + c;
  if (c < 2 * g.Dk) return g.H * g.Dk + h * g.Dk + (c - g.Dk);
  return 2 * g.H * g.Dk + h * g.Dv + g.v0 + (c - 2 * g.Dk);
}

// Shared-memory plan of the GDN phase inside the work area (hp, ssq and red
// are written by the cluster's CTAs; the preload region is written only by
// this CTA, before the barrier that starts the phase).
struct GdnSmem {
  float *hp, *ssq, *red, *xs, *qk, *vv, *og, *rs, *pv, *gb, *stb, *pconv_w, *pconv_s;
};
__host__ __device__ inline int pad4(int n) { return (n + 3) & ~3; }  // floats to a 16-byte multiple

template <int M>
__device__ __forceinline__ GdnSmem gdn_smem(float* work, const GdnGeo& g) {
  GdnSmem s;  // every array starts on a 16-byte boundary (xs is read as float4)
  s.xs = work;                          // [M][xpad(d)]
  s.hp = s.xs + pad4(M * xpad(g.d));    // [M][HP]
  s.ssq = s.hp + pad4(M * g.HP);        // [kCl][M]
  s.red = s.ssq + pad4(kCl * M);        // [kCl][M][RC]
  s.qk = s.red + pad4(kCl * M * g.RC);  // [M][2 Dk]
  s.vv = s.qk + pad4(M * 2 * g.Dk);     // [M][vpr]
  s.og = s.vv + pad4(M * g.vpr);        // [M][vpr]
  s.rs = s.og + pad4(M * g.vpr);        // [kT] reduction scratch
  s.pv = s.rs + kT;                     // [kW]
  s.gb = s.pv + kW;                     // [M][2] decay log, beta
  s.stb = s.gb + pad4(M * 2);           // [M][kT] state columns copied before the barrier
  s.pconv_w = work + kPreOff / 4 + kParConv;  // [NC][4] conv taps (parameter region)
  s.pconv_s = s.pconv_w + g.NC * 4;     // [B][3][NC] conv window
  return s;
}

// Before the barrier: this rank's state columns into the work area (read into
// registers once the phase starts) and its conv taps / conv window into the
// preload region; all by cp.async (they do not depend on the step).
template <int M>
__device__ __forceinline__ void gdn_preload(const MkArgs& a, const CbSelfLayer& L, int h, int rank, float (&st)[M],
                            float* work) {
  const CbModel& m = a.m;
  const GdnGeo g = gdn_geo(m, rank);
  const GdnSmem s = gdn_smem<M>(work, g);
  const int tid = threadIdx.x, C = 2 * g.H * g.Dk + g.H * g.Dv;
  const bool holds = tid < g.Dk * g.vpr;
  const int k = tid / g.vpr, v = tid - k * g.vpr;
  // first group (needed as the phase starts): norm vector, tile scales of this rank's tiles
  float* pn = par_norm(work);
  float* ps = par_small(work);
  for (int i = tid; i < m.d_model / 4; i += kT) cp_async16(pn + 4 * i, L.norm1 + 4 * i);
  if (tid == 0) {
    int q = 0;
    for (int j = rank; j < g.ntile; j += kCl, ++q) {
      int hp_off;
      cp_async4(ps + q, L.in_proj.tile_scale + gdn_head_tile(m, g, h, j, hp_off));
    }
    if (rank == kCl - 1) {
      cp_async4(ps + 16, L.in_proj.tile_scale + (m.gdn_off_a + h) / kTileRows);
      cp_async4(ps + 17, L.in_proj.tile_scale + (m.gdn_off_b + h) / kTileRows);
    }
  }
  cp_async_commit();
  // second group (needed after the in-projection): state columns, gate constants,
  // tensor scale, o_norm columns, conv taps and window
#pragma unroll
  for (int b = 0; b < M; ++b) {
    if (b < a.B && holds) {
      const int64_t slot = (int64_t)b * a.c.n_gdn + L.slot;
      cp_async4(s.stb + b * kT + tid, a.c.gdn_state + ((slot * g.H + h) * g.Dk + k) * g.Dv + g.v0 + v);
    }
  }
  if (tid == 0) {
    cp_async4(ps + PS_A_LOG, L.A_log + h);
    cp_async4(ps + PS_DT_BIAS, L.dt_bias + h);
    cp_async4(ps + PS_TSCALE, L.o_proj_ks.tensor_scale);
  }
  for (int v2 = tid; v2 < g.vpr; v2 += kT) cp_async4(ps + PS_O_NORM + v2, L.o_norm + g.v0 + v2);
  for (int c = tid; c < g.NC; c += kT) cp_async16(s.pconv_w + c * 4, L.conv_w + (int64_t)gdn_channel(g, h, c) * 4);
  for (int i = tid; i < a.B * 3 * g.NC; i += kT) {
    const int b = i / (3 * g.NC), r = i - b * 3 * g.NC, j = r / g.NC, c = r - j * g.NC;
    const int64_t slot = (int64_t)b * a.c.n_gdn + L.slot;
    cp_async4(s.pconv_s + i, a.c.gdn_conv + (slot * 3 + j) * C + gdn_channel(g, h, c));
  }
  cp_async_commit();
}

__device__ __forceinline__ int64_t slice_bytes(const CbSliced& S) {
  return ((int64_t)S.rows * (S.width / 2 + 1) + 15) / 16 * 16;
}

// Weight chunks of the GDN phase for cluster rank `rank` of head h: the rank's
// in-projection tiles (entries rank, rank + 8, ... of the head's list), the a
// and b tiles on the last rank, then the rank's o-projection slice.  Returns
// the chunk count; *oslice receives the slot offset of the o-projection slice.
template <typename F>
__device__ __forceinline__ int gdn_chunks(const CbSelfLayer& L, const CbModel& m, int h, int rank, F&& f,
                                          int* oslice = nullptr) {
  const GdnGeo g = gdn_geo(m, rank);
  const int64_t tb = tile_bytes(L.in_proj.k);
  int n = 0, off = 0;
  for (int j = rank; j < g.ntile; j += kCl) {
    int hp_off;
    const int t = gdn_head_tile(m, g, h, j, hp_off);
    f(n++, L.in_proj.tiles + t * tb, (unsigned)tb, off);
    off += (int)tb;
  }
  if (rank == kCl - 1) {
    f(n++, L.in_proj.tiles + ((m.gdn_off_a + h) / kTileRows) * tb, (unsigned)tb, off);
    off += (int)tb;
    f(n++, L.in_proj.tiles + ((m.gdn_off_b + h) / kTileRows) * tb, (unsigned)tb, off);
    off += (int)tb;
  }
  if (oslice) *oslice = off;
  const int64_t sb = slice_bytes(L.o_proj_ks);
  f(n++, L.o_proj_ks.data + (int64_t)(h * kCl + rank) * sb, (unsigned)sb, off);
  return n;
}

// One cluster per head: in-projection -> conv -> recurrence -> gated norm -> o-projection.
template <int M>
__device__ __forceinline__ void gdn_phase(const MkArgs& a, const CbSelfLayer& L, bool first, bool live, int h, int rank,
                          float (&st)[M], const uint8_t* slot, float* work) {
  const CbModel& m = a.m;
  const GdnGeo g = gdn_geo(m, rank);
  const GdnSmem s = gdn_smem<M>(work, g);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = a.B, T = a.T, Mr = B * T, d = g.d, K = L.in_proj.k, C = 2 * g.H * g.Dk + g.H * g.Dv;
  const int64_t tb = tile_bytes(K);
  const bool snap = a.c.snap_state != nullptr && a.c.snap_conv != nullptr && T > 1;
  if (live) {
    __shared__ int s_rows[kMkMaxRows];
    if (tid < kMkMaxRows) s_rows[tid] = tid;
    __syncthreads();
    float rn[M];
    stage_rows<M>(a.hq, nullptr, d, s_rows, Mr, K, par_norm(work), m.norm_eps, s.xs, rn, nullptr,
                  (first && h == 0 && rank == 0) ? a.hq : nullptr, first ? &a : nullptr);
    mark(a, 0);
    const float* ps = par_small(work);
    // this rank's rows: tiles rank, rank + 8, ... then (last rank) the a and b rows;
    // lane r < 8 of each warp sends the row's values to cluster rank r
    int off = 0, q = 0;
    for (int j = rank; j < g.ntile; j += kCl, ++q) {
      int hp_off;
      gdn_head_tile(m, g, h, j, hp_off);
      float acc[M];
      row_dot<M>(slot + off, K, warp, true, false, s.xs, acc);
      off += (int)tb;
      const float ts = ps[q];
      if (lane < kCl)
#pragma unroll
        for (int mr = 0; mr < M; ++mr)
          if (mr < Mr) st_dsmem(dsmem(s.hp + mr * g.HP + hp_off + warp, lane), acc[mr] * ts * rn[mr]);
    }
    if (rank == kCl - 1) {
      for (int e = 0; e < 2; ++e) {
        const int row = (e == 0 ? m.gdn_off_a : m.gdn_off_b) + h;
        if (warp == (row & 15)) {
          float acc[M];
          row_dot<M>(slot + off, K, warp, true, false, s.xs, acc);
          const float ts = ps[16 + e];
          if (lane < kCl)
#pragma unroll
            for (int mr = 0; mr < M; ++mr)
              if (mr < Mr) st_dsmem(dsmem(s.hp + mr * g.HP + 2 * g.Dk + 2 * g.Dv + e, lane), acc[mr] * ts * rn[mr]);
        }
        off += (int)tb;
      }
    }
  }
  cp_async_wait_all();  // the preload's second group (state, conv, constants); the cluster barrier publishes it
  cluster_sync();  // every rank's in-projection rows are in every rank's hp
  mark(a, 1);
#pragma unroll
  for (int b = 0; b < M; ++b) st[b] = (b < B && tid < g.Dk * g.vpr) ? s.stb[b * kT + tid] : 0.0f;
  if (live) {
    const float* ps = par_small(work);
    // short conv (4 taps) on q, k and this rank's v channels; the new window goes back to the cache
    for (int c = tid; c < g.NC; c += kT) {
      const float w0 = s.pconv_w[c * 4], w1 = s.pconv_w[c * 4 + 1], w2 = s.pconv_w[c * 4 + 2],
                  w3 = s.pconv_w[c * 4 + 3];
      const int hpi = c < 2 * g.Dk ? c : 2 * g.Dk + g.v0 + (c - 2 * g.Dk);
      const bool own = c >= 2 * g.Dk || (c % kCl) == rank;
      for (int b = 0; b < B; ++b) {
        float c0 = s.pconv_s[(b * 3 + 0) * g.NC + c], c1 = s.pconv_s[(b * 3 + 1) * g.NC + c],
              c2 = s.pconv_s[(b * 3 + 2) * g.NC + c];
        for (int t = 0; t < T; ++t) {
          const int mr = b * T + t;
          const float x = s.hp[mr * g.HP + hpi];
          float y = c0 * w0;
          y += c1 * w1;
          y += c2 * w2;
          y += x * w3;
          const float o = silu(y);
          if (c < 2 * g.Dk) s.qk[mr * 2 * g.Dk + c] = o;
          else s.vv[mr * g.vpr + (c - 2 * g.Dk)] = o;
          c0 = c1;
          c1 = c2;
          c2 = x;
          if (snap && own && t < T - 1) {  // the window after token t (verify rewind)
            float* sw = a.c.snap_conv + (int64_t)t * B * a.c.n_gdn * 3 * C +
                        ((int64_t)b * a.c.n_gdn + L.slot) * 3 * C + gdn_channel(g, h, c);
            sw[0] = c0;
            sw[C] = c1;
            sw[2 * (int64_t)C] = c2;
          }
        }
        if (own) {
          const int64_t slot_i = (int64_t)b * a.c.n_gdn + L.slot;
          float* cw = a.c.gdn_conv + slot_i * 3 * C + gdn_channel(g, h, c);
          cw[0] = c0;
          cw[C] = c1;
          cw[2 * (int64_t)C] = c2;
        }
      }
    }
    if (tid < Mr) {
      const float av = s.hp[tid * g.HP + 2 * g.Dk + 2 * g.Dv], bv = s.hp[tid * g.HP + 2 * g.Dk + 2 * g.Dv + 1];
      s.gb[tid * 2] = -expf(ps[PS_A_LOG]) * softplus(av + ps[PS_DT_BIAS]);
      s.gb[tid * 2 + 1] = sigmoid(bv);
    }
    __syncthreads();
    for (int job = warp; job < 2 * Mr; job += kW) {  // L2 norms of q and k
      float* x = s.qk + (job >> 1) * 2 * g.Dk + (job & 1) * g.Dk;
      float ss = 0.0f;
      for (int i = lane; i < g.Dk; i += 32) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
      for (int i = lane; i < g.Dk; i += 32) x[i] *= inv;
    }
    __syncthreads();
  }
  // the recurrence on this rank's columns: thread (k, v) holds S[k][v0 + v] of every sequence
  const bool holds = tid < g.Dk * g.vpr;
  const int k = tid / g.vpr, v = tid - k * g.vpr;
  if (live) {
    const float scale = rsqrtf((float)g.Dk);
    auto reduce_k = [&](float part, float* out, float mul) {  // out[v] = mul * sum_k part(k, v), fixed order
      s.rs[tid] = part;
      __syncthreads();
      if (warp < g.vpr) {
        float t = 0.0f;
        for (int kk = lane; kk < g.Dk; kk += 32) t += s.rs[kk * g.vpr + warp];
        t = warp_sum(t);
        if (lane == 0) out[warp] = t * mul;
      }
      __syncthreads();
    };
#pragma unroll
    for (int b = 0; b < M; ++b) {
      if (b < B) {
        for (int t = 0; t < T; ++t) {
          const int mr = b * T + t;
          const float* qq = s.qk + mr * 2 * g.Dk;
          const float* kk = qq + g.Dk;
          const float decay = expf(s.gb[mr * 2]), beta = s.gb[mr * 2 + 1];
          float part = 0.0f;
          if (holds) {
            st[b] *= decay;
            part = st[b] * kk[k];
          }
          reduce_k(part, s.pv, 1.0f);
          part = 0.0f;
          if (holds) {
            const float delta = beta * (s.vv[mr * g.vpr + v] - s.pv[v]);
            st[b] = fmaf(kk[k], delta, st[b]);
            part = st[b] * qq[k];
          }
          reduce_k(part, s.og + mr * g.vpr, scale);
          if (snap && holds && t < T - 1)  // the state after token t (verify rewind)
            a.c.snap_state[(int64_t)t * B * a.c.n_gdn * g.H * g.Dk * g.Dv +
                           ((((int64_t)b * a.c.n_gdn + L.slot) * g.H + h) * g.Dk + k) * g.Dv + g.v0 + v] = st[b];
        }
        if (holds) {
          const int64_t slot_i = (int64_t)b * a.c.n_gdn + L.slot;
          a.c.gdn_state[((slot_i * g.H + h) * g.Dk + k) * g.Dv + g.v0 + v] = st[b];
        }
      }
    }
    // this rank's part of each row's sum of squares, to every rank
    if (tid < Mr) {
      float ss = 0.0f;
      for (int vv = 0; vv < g.vpr; ++vv) ss += s.og[tid * g.vpr + vv] * s.og[tid * g.vpr + vv];
      for (int r = 0; r < kCl; ++r) st_dsmem(dsmem(s.ssq + rank * M + tid, r), ss);
    }
  }
  cluster_sync();
  mark(a, 2);
  if (live) {
    const float* ps = par_small(work);
    for (int i = tid; i < Mr * g.vpr; i += kT) {
      const int mr = i / g.vpr, vc = i - mr * g.vpr;
      float ss = 0.0f;
      for (int r = 0; r < kCl; ++r) ss += s.ssq[r * M + mr];
      const float rr = rsqrtf(ss / (float)g.Dv + m.norm_eps);
      const float gate = s.hp[mr * g.HP + 2 * g.Dk + g.Dv + g.v0 + vc];
      s.og[i] = s.og[i] * rr * ps[PS_O_NORM + vc] * silu(gate);
    }
    __syncthreads();
    // split-K o-projection on this rank's columns; the partial of output n goes to rank n / RC
    int soff = 0;
    gdn_chunks(L, m, h, rank, [](int, const uint8_t*, unsigned, int) {}, &soff);
    const uint8_t* sl = slot + soff;
    const int cbytes = g.vpr / 2;
    const float ts = ps[PS_TSCALE];
    for (int n = tid; n < d; n += kT) {
      const float sc = e4m3_to_f32(sl[(int64_t)d * cbytes + n]) * ts;
      float acc[M];
#pragma unroll
      for (int mr = 0; mr < M; ++mr) acc[mr] = 0.0f;
      for (int j = 0; j < cbytes; ++j) {
        const float2 w = e2m1x2_to_f32x2(sl[n * cbytes + j]);
#pragma unroll
        for (int mr = 0; mr < M; ++mr)
          acc[mr] = fmaf(w.y, s.og[mr * g.vpr + 2 * j + 1], fmaf(w.x, s.og[mr * g.vpr + 2 * j], acc[mr]));
      }
      const int q = n / g.RC, nl = n - q * g.RC;
#pragma unroll
      for (int mr = 0; mr < M; ++mr)
        if (mr < Mr) st_dsmem(dsmem(s.red + (rank * M + mr) * g.RC + nl, q), acc[mr] * sc);
    }
  }
  cluster_sync();
  mark(a, 3);
  if (live) {
    for (int i = tid; i < Mr * g.RC; i += kT) {
      const int mr = i / g.RC, nl = i - mr * g.RC;
      float t = 0.0f;
      for (int r = 0; r < kCl; ++r) t += s.red[(r * M + mr) * g.RC + nl];
      red_fix(a.hq + (int64_t)mr * d + rank * g.RC + nl, t);
    }
  }
}

// ------------------------------------------------------------------ FFN (split K)
// Slices of 16 hidden units: slice j = the gate tile j, the up tile F/16 + j and
// the 16 columns j of the down projection.  CTA c owns slices c, c + ncta, ...
// When the slices outnumber the CTAs by at most one per cluster, CTA c owns
// slice c only and slice ncta + q is split over cluster q instead: its CTA r
// takes hidden units 2r and 2r + 1 (gate and up rows 2r, 2r + 1 and down
// columns 2r, 2r + 1), so that no CTA holds two slices.
__device__ __forceinline__ bool ffn_split(int F, int K, int ncta) {
  const int nsl = F / kTileRows;
  return nsl > ncta && nsl - ncta <= ncta / kCl && K % 128 == 0;
}
__device__ __forceinline__ int ffn_mine(int F, int K, int cta, int ncta) {
  const int nsl = F / kTileRows;
  if (ffn_split(F, K, ncta)) return 1;
  return cta < nsl ? (nsl - 1 - cta) / ncta + 1 : 0;
}
// The slice split over this CTA's cluster, or -1.
__device__ __forceinline__ int ffn_extra(int F, int K, int cta, int ncta) {
  if (!ffn_split(F, K, ncta)) return -1;
  const int q = cta / kCl;
  return q < F / kTileRows - ncta ? ncta + q : -1;
}
__device__ __forceinline__ int ffn_staged(const CbMatrix& GU, const CbSliced& D, int F, int cta, int ncta) {
  const int64_t per = 2 * tile_bytes(GU.k) + slice_bytes(D);
  return min(ffn_mine(F, GU.k, cta, ncta), (int)(kSlot / per));
}

// Slot layout: the staged slices (gate tile, up tile, down slice each), then for
// a split slice: gate rows 2r, 2r + 1 (codes, then scales), the same up rows, the down slice.
template <typename F>
__device__ __forceinline__ int ffn_chunks(const CbMatrix& GU, const CbSliced& D, int Fh, int cta, int ncta, F&& f) {
  const int K = GU.k;
  const int64_t tb = tile_bytes(K), dsb = slice_bytes(D);
  const int nst = ffn_staged(GU, D, Fh, cta, ncta);
  int n = 0, off = 0;
  for (int i = 0; i < nst; ++i) {
    const int j = cta + i * ncta;
    f(n++, GU.tiles + j * tb, (unsigned)tb, off);
    off += (int)tb;
    f(n++, GU.tiles + (Fh / kTileRows + j) * tb, (unsigned)tb, off);
    off += (int)tb;
    f(n++, D.data + j * dsb, (unsigned)dsb, off);
    off += (int)dsb;
  }
  const int x = ffn_extra(Fh, K, cta, ncta);
  if (x >= 0) {
    const int r = cta % kCl;
    for (int t = 0; t < 2; ++t) {
      const uint8_t* tile = GU.tiles + (t == 0 ? x : Fh / kTileRows + x) * tb;
      f(n++, tile + 2 * r * (K / 2), (unsigned)K, off);
      off += K;
      f(n++, tile + kTileRows * (K / 2) + 2 * r * (K / 16), (unsigned)(K / 8), off);
      off += K / 8;
    }
    f(n++, D.data + x * dsb, (unsigned)dsb, off);
  }
  return n;
}

template <int M>
__device__ __forceinline__ void ffn_phase(const MkArgs& a, const CbMatrix& GU, const CbSliced& D, const float* norm2,
                                          long long* resid, int Mr, bool live, int rank, int cid, const uint8_t* slot,
                                          float* work) {
  const CbModel& m = a.m;
  const int d = m.d_model, Fh = m.ffn_hidden, RC = d / kCl, K = GU.k;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x, ncta = gridDim.x;
  float* red = work;                   // [kCl][M][RC]  (written by the cluster's CTAs)
  float* xs = red + kCl * M * RC;      // [M][xpad(d)]
  float* act = xs + M * xpad(d);       // [M][16]
  float* gux = act + M * kTileRows;    // [4][M] split slice: gate 2r, gate 2r + 1, up 2r, up 2r + 1
  constexpr int kNE = (kMkMaxD + kT - 1) / kT;  // outputs per thread
  float acc[kNE][M];
#pragma unroll
  for (int e = 0; e < kNE; ++e)
#pragma unroll
    for (int mr = 0; mr < M; ++mr) acc[e][mr] = 0.0f;
  const int n_mine = ffn_mine(Fh, K, cta, ncta);
  const int xsl = ffn_extra(Fh, K, cta, ncta);
  // a cluster adds its sums only when one of its CTAs owns a slice (cluster-uniform)
  const bool cluster_has = cid * kCl < Fh / kTileRows;
  if (live && n_mine > 0) {
    __shared__ int s_rows[kMkMaxRows];
    if (tid < kMkMaxRows) s_rows[tid] = tid;
    __syncthreads();
    float rn[M];
    stage_rows<M>(resid, nullptr, d, s_rows, Mr, K, par_norm(work), m.norm_eps, xs, rn, nullptr, nullptr, nullptr);
    mark(a, 0);
    const float* ps = par_small(work);
    const int64_t tb = tile_bytes(K), dsb = slice_bytes(D);
    const int nst = ffn_staged(GU, D, Fh, cta, ncta);
    const float ts_d = ps[PS_TSCALE];
    for (int i = 0; i < n_mine; ++i) {
      const int j = cta + i * ncta;
      const bool glob = i >= nst;
      const uint8_t* tg = glob ? GU.tiles + j * tb : slot + i * (2 * tb + dsb);
      const uint8_t* tu = glob ? GU.tiles + (Fh / kTileRows + j) * tb : tg + tb;
      const uint8_t* ds = glob ? D.data + j * dsb : tg + 2 * tb;
      float gv[M], uv[M];
      row_dot<M>(tg, K, warp, true, glob, xs, gv);
      row_dot<M>(tu, K, warp, true, glob, xs, uv);
      const float tsg = i < 16 ? ps[i] : GU.tile_scale[j];
      const float tsu = i < 16 ? ps[16 + i] : GU.tile_scale[Fh / kTileRows + j];
      if (i == 0 && xsl >= 0 && warp < 4) {  // the split slice's rows: warp w takes row w & 1 of gate (w < 2) or up
        const uint8_t* xt = slot + nst * (2 * tb + dsb) + (warp >> 1) * (K + K / 8);
        float xv[M];
        row_dot<M>(xt, K, warp & 1, true, false, xs, xv, 2);
        const float tsx = ps[32 + (warp >> 1)];
        if (lane < M && lane < Mr) {
          float v = 0.0f;
#pragma unroll
          for (int mr = 0; mr < M; ++mr)
            if (mr == lane) v = xv[mr] * tsx * rn[mr];
          gux[warp * M + lane] = v;
        }
      }
      if (i == 0) mark(a, 1);
      if (lane < M && lane < Mr) {
        float g0 = 0.0f, u0 = 0.0f;
#pragma unroll
        for (int mr = 0; mr < M; ++mr)
          if (mr == lane) {
            g0 = gv[mr] * tsg * rn[mr];
            u0 = uv[mr] * tsu * rn[mr];
          }
        act[lane * kTileRows + warp] = silu(g0) * u0;
      }
      __syncthreads();
      const bool with_x = i == 0 && xsl >= 0;
      float ax[M][2];  // the split slice's two activations per row
#pragma unroll
      for (int mr = 0; mr < M; ++mr) {
        ax[mr][0] = ax[mr][1] = 0.0f;
        if (with_x && mr < Mr) {
          ax[mr][0] = silu(gux[mr]) * gux[2 * M + mr];
          ax[mr][1] = silu(gux[M + mr]) * gux[3 * M + mr];
        }
      }
      const uint8_t* dsx = slot + nst * (2 * tb + dsb) + 2 * (K + K / 8);
#pragma unroll
      for (int e = 0; e < kNE; ++e) {
        const int n = tid + e * kT;
        if (n < d && with_x) {
          const float2 fx = e2m1x2_to_f32x2(dsx[(int64_t)n * 8 + rank]);
          const float scx = e4m3_to_f32(dsx[(int64_t)d * 8 + n]) * ts_d;
#pragma unroll
          for (int mr = 0; mr < M; ++mr) acc[e][mr] = fmaf(fmaf(fx.x, ax[mr][0], fx.y * ax[mr][1]), scx, acc[e][mr]);
        }
        if (n < d) {
          const uint2 cw = glob ? __ldg(reinterpret_cast<const uint2*>(ds + (int64_t)n * 8))
                                : *reinterpret_cast<const uint2*>(ds + (int64_t)n * 8);
          const float sc = e4m3_to_f32(glob ? __ldg(ds + (int64_t)d * 8 + n) : ds[(int64_t)d * 8 + n]) * ts_d;
          float w[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 lo = e2m1x2_to_f32x2(cw.x >> (8 * q)), hi = e2m1x2_to_f32x2(cw.y >> (8 * q));
            w[2 * q] = lo.x;
            w[2 * q + 1] = lo.y;
            w[8 + 2 * q] = hi.x;
            w[8 + 2 * q + 1] = hi.y;
          }
#pragma unroll
          for (int mr = 0; mr < M; ++mr) {
            float p = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) p = fmaf(w[c], act[mr * kTileRows + c], p);
            acc[e][mr] = fmaf(p, sc, acc[e][mr]);
          }
        }
      }
      __syncthreads();
      if (i == 0) mark(a, 2);
    }
  }
  mark(a, 3);
  if (live && cluster_has) {
#pragma unroll
    for (int e = 0; e < kNE; ++e) {
      const int n = tid + e * kT;
      if (n < d) {
        const int q = n / RC, nl = n - q * RC;
#pragma unroll
        for (int mr = 0; mr < M; ++mr)
          if (mr < Mr) st_dsmem(dsmem(red + (rank * M + mr) * RC + nl, q), acc[e][mr]);
      }
    }
  }
  mark(a, 4);
  cluster_sync();
  mark(a, 5);
  if (live && cluster_has) {
    for (int i = tid; i < Mr * RC; i += kT) {
      const int mr = i / RC, nl = i - mr * RC;
      float t = 0.0f;
      for (int r = 0; r < kCl; ++r) t += red[(r * M + mr) * RC + nl];
      red_fix(resid + (int64_t)mr * d + rank * RC + nl, t);
    }
  }
}

// ------------------------------------------------------- RMSNorm + RoPE
// One warp: RMSNorm(x) * w (over hd) then partial interleaved RoPE at position
// p; lane owns the pairs j = lane, lane + 32, ...  Results to out (smem).
// When bf16 is set the values are rounded to bfloat16 and the bits also go to bits_out.
__device__ void norm_rope_warp(const float* x, const float* w, int hd, int rot2, int p, const float* inv_freq,
                               float eps, float* out, bool bf16, uint16_t* bits_out) {
  const int lane = threadIdx.x & 31, npairs = hd / 2;
  float ss = 0.0f;
  for (int j = lane; j < npairs; j += 32) {
    const float a0 = __ldcg(x + 2 * j), a1 = __ldcg(x + 2 * j + 1);
    ss += a0 * a0 + a1 * a1;
  }
  ss = warp_sum(ss);
  const float rn = rsqrtf(ss / (float)hd + eps);
  for (int j = lane; j < npairs; j += 32) {
    float x1 = __ldcg(x + 2 * j) * rn * w[2 * j];
    float x2 = __ldcg(x + 2 * j + 1) * rn * w[2 * j + 1];
    if (j < rot2) rope_pair(x1, x2, p, inv_freq[j]);
    if (bf16) {
      const uint16_t b1 = f32_to_bf16(x1), b2 = f32_to_bf16(x2);
      x1 = bf16_to_f32(b1);
      x2 = bf16_to_f32(b2);
      if (bits_out) {
        bits_out[2 * j] = b1;
        bits_out[2 * j + 1] = b2;
      }
    }
    out[2 * j] = x1;
    out[2 * j + 1] = x2;
  }
}

// ------------------------------------------------------ shared KV + indexer
__device__ __forceinline__ void query_row(const MkArgs& a, int r, int& b, int& t, int& p, int& n) {
  b = r / a.nq;
  t = a.T - a.nq + (r - b * a.nq);
  p = a.c.pos[b] + a.c0 + t;
  n = max(0, min(p + 1, a.c.max_ctx));
}

// New rows of the shared cache: k = RoPE(RMSNorm(k)), v, indexer key (E4M3).
__device__ void shared_append(const MkArgs& a, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int Mrows = a.B * a.T, hd = m.head_dim, Hkv = m.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int mr = blockIdx.x; mr < Mrows; mr += gridDim.x) {
    const int b = mr / a.T, t = mr - b * a.T, p = c.pos[b] + a.c0 + t;
    if (p < 0 || p >= c.max_ctx) {
      if (threadIdx.x == 0) set_status(a.status, CB_ERR_CTX_FULL);
      continue;
    }
    const float* row = a.proj + (int64_t)mr * a.ldp;
    const int64_t base = ((int64_t)b * c.max_ctx + p) * Hkv * hd;
    const int items = 2 * Hkv + (m.sparse_topk > 0 ? 1 : 0);
    for (int it = warp; it < items; it += kW) {
      if (it < Hkv) {
        float* tmp = smem + it * hd;
        norm_rope_warp(row + it * hd, m.shared_k_norm, hd, m.rot_dim / 2, p, m.inv_freq, m.norm_eps, tmp, true,
                       c.kv_k + base + it * hd);
      } else if (it < 2 * Hkv) {
        const int hh = it - Hkv;
        for (int dd = lane; dd < hd; dd += 32)
          c.kv_v[base + hh * hd + dd] = f32_to_bf16(__ldcg(row + Hkv * hd + hh * hd + dd));
      } else {
        uint8_t* ik = c.kv_ik + ((int64_t)b * c.max_ctx + p) * m.indexer_dim;
        for (int dd = lane; dd < m.indexer_dim; dd += 32) ik[dd] = f32_to_e4m3(__ldcg(row + m.sh_off_ik + dd));
      }
    }
    __syncthreads();
  }
}

// Fixed-order float32 indexer score (the order of indexer.cu and oracle/indexer.py).
__device__ __forceinline__ float indexer_score_bytes(const uint8_t* kr, const float* q, const float* w, int Hi, int Di) {
  float score = 0.0f;
  for (int h = 0; h < Hi; ++h) {
    const float* qh = q + h * Di;
    float pr[8];
    for (int i = 0; i < Di / 8; ++i) {
      const uint2 raw = *reinterpret_cast<const uint2*>(kr + 8 * i);
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const uint32_t byte = ((rr < 4 ? raw.x : raw.y) >> (8 * (rr & 3))) & 0xFF;
        const float prod = __fmul_rn(e4m3_to_f32(byte), qh[8 * i + rr]);
        pr[rr] = i == 0 ? prod : __fadd_rn(pr[rr], prod);
      }
    }
    const float dsum = __fadd_rn(__fadd_rn(__fadd_rn(pr[0], pr[1]), __fadd_rn(pr[2], pr[3])),
                                 __fadd_rn(__fadd_rn(pr[4], pr[5]), __fadd_rn(pr[6], pr[7])));
    const float rl = dsum > 0.0f ? dsum : 0.0f;
    const float term = __fmul_rn(rl, w[h]);
    score = h == 0 ? term : __fadd_rn(score, term);
  }
  return score;
}

__device__ __forceinline__ void key_range(int n, int cta, int ncta, int& js, int& je) {
  const int per = ceil_div(n, ncta);
  js = min(n, cta * per);
  je = min(n, js + per);
}

// Scores of this CTA's key range for every query row + histogram of the top 11
// key bits.  All rows at once: their queries, the chunk's new keys and the
// histograms are staged together, and the rows' score loops run back to back
// (a key read for one row is in L1 for the next rows of its sequence).
__device__ void score_phase(const MkArgs& a, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int RQ = a.B * a.nq, Hi = m.indexer_heads, Di = m.indexer_dim, k = m.sparse_topk, HD = Hi * Di;
  const int Mrows = a.B * a.T;
  const int tid = threadIdx.x, cta = blockIdx.x, ncta = gridDim.x;
  unsigned* hist = reinterpret_cast<unsigned*>(smem);        // [RQ][2048]
  float* q = smem + RQ * kMkHistBins;                         // [RQ][Hi * Di]
  float* w = q + RQ * HD;                                     // [RQ][16]
  uint8_t* newk = reinterpret_cast<uint8_t*>(w + RQ * 16);    // [Mrows][Di] keys of this chunk's tokens
  __shared__ int r_b[kMkMaxRows], r_p0[kMkMaxRows], r_js[kMkMaxRows], r_je[kMkMaxRows];
  if (tid < RQ) {
    int b, t, p, n;
    query_row(a, tid, b, t, p, n);
    int js = 0, je = 0;
    if (n > k) key_range(n, cta, ncta, js, je);
    r_b[tid] = b;
    r_p0[tid] = c.pos[b] + a.c0;
    r_js[tid] = js;
    r_je[tid] = je;
  }
  for (int i = tid; i < RQ * HD; i += kT) {
    const int r = i / HD, e = i - r * HD, b = r / a.nq, t = a.T - a.nq + (r - b * a.nq);
    q[i] = __ldcg(a.proj + ((int64_t)b * a.T + t) * a.ldp + m.sh_off_iq + e);
  }
  for (int i = tid; i < RQ * Hi; i += kT) {
    const int r = i / Hi, h = i - r * Hi, b = r / a.nq, t = a.T - a.nq + (r - b * a.nq);
    w[r * 16 + h] = __ldcg(a.proj + ((int64_t)b * a.T + t) * a.ldp + m.sh_off_iw + h);
  }
  for (int i = tid; i < Mrows * Di; i += kT) {
    const int mr = i / Di, dd = i - mr * Di;
    newk[i] = f32_to_e4m3(__ldcg(a.proj + (int64_t)mr * a.ldp + m.sh_off_ik + dd));
  }
  for (int i = tid; i < RQ * kMkHistBins; i += kT) hist[i] = 0u;
  __syncthreads();
  for (int r = 0; r < RQ; ++r) {
    const int js = r_js[r], je = r_je[r], b = r_b[r], p0 = r_p0[r];
    const uint8_t* ikb = c.kv_ik + (int64_t)b * c.max_ctx * Di;
    float* out = a.scores + (int64_t)r * c.max_ctx;
    for (int j = js + tid; j < je; j += kT) {
      const uint8_t* kr = j < p0 ? ikb + (int64_t)j * Di : newk + (b * a.T + (j - p0)) * Di;
      const float sc = indexer_score_bytes(kr, q + r * HD, w + r * 16, Hi, Di);
      out[j] = sc;
      atomicAdd(&hist[r * kMkHistBins + (score_key(sc) >> 21)], 1u);
    }
  }
  __syncthreads();
  for (int i = tid; i < RQ * kMkHistBins; i += kT)
    if (hist[i]) atomicAdd(&a.hist[i], hist[i]);
}

// Block-wide exclusive prefix sum of one unsigned per thread (kT threads).
__device__ unsigned block_excl_scan(unsigned v, unsigned* wsum, unsigned* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned x = lane < kW ? wsum[lane] : 0u;
    unsigned xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned t = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += t;
    }
    if (lane < kW) wsum[lane] = xi - x;
    if (lane == kW - 1) *total = xi;
  }
  __syncthreads();
  return wsum[warp] + incl - v;
}

// Threshold bin of the k-th largest key, then this CTA's keys above it to hi_list and in it to cand.
__device__ void compact_phase(const MkArgs& a) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int RQ = a.B * a.nq, k = m.sparse_topk;
  const int tid = threadIdx.x, lane = tid & 31, cta = blockIdx.x, ncta = gridDim.x;
  __shared__ unsigned wsum[32], s_total;
  __shared__ int s_b1;
  for (int r = 0; r < RQ; ++r) {
    int b, t, p, n;
    query_row(a, r, b, t, p, n);
    if (n <= k) continue;
    int js, je;
    key_range(n, cta, ncta, js, je);
    if (js >= je) continue;
    // thread tid owns bins 2047-4*tid .. 2044-4*tid (descending)
    const unsigned* hg = a.hist + (int64_t)r * kMkHistBins;
    unsigned h4[4], sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h4[i] = __ldcg(hg + kMkHistBins - 1 - 4 * tid - i);
      sum += h4[i];
    }
    const unsigned excl = block_excl_scan(sum, wsum, &s_total);
    if (excl < (unsigned)k && excl + sum >= (unsigned)k) {
      unsigned cum = excl;
      for (int i = 0; i < 4; ++i) {
        if (cum + h4[i] >= (unsigned)k) {
          s_b1 = kMkHistBins - 1 - 4 * tid - i;
          break;
        }
        cum += h4[i];
      }
    }
    __syncthreads();
    const unsigned b1 = (unsigned)s_b1;
    const float* sc = a.scores + (int64_t)r * c.max_ctx;
    for (int base = js; base < je; base += kT) {
      const int j = base + tid;
      unsigned u = 0;
      if (j < je) u = score_key(__ldcg(sc + j));
      const unsigned bin = u >> 21;
      const bool hi = j < je && bin > b1, eq = j < je && bin == b1;
      const unsigned bh = __ballot_sync(0xffffffffu, hi), be = __ballot_sync(0xffffffffu, eq);
      int basehi = 0, baseeq = 0;
      if (lane == 0) {
        if (bh) basehi = atomicAdd(&a.hi_cnt[r], __popc(bh));
        if (be) baseeq = atomicAdd(&a.cand_cnt[r], __popc(be));
      }
      basehi = __shfl_sync(0xffffffffu, basehi, 0);
      baseeq = __shfl_sync(0xffffffffu, baseeq, 0);
      const unsigned lt = (1u << lane) - 1u;
      const int shi = basehi + __popc(bh & lt), seq = baseeq + __popc(be & lt);
      if (hi && shi < k) a.hi_list[(int64_t)r * k + shi] = j;
      if (eq && seq < c.max_ctx) a.cand[(int64_t)r * c.max_ctx + seq] = ((unsigned long long)u << 32) | (unsigned)j;
    }
    __syncthreads();
  }
}

// Exact selection of one query row: the keys above the threshold bin, the top
// `need` threshold-bin candidates by (key, index) -- all of them share the top
// 11 bits, so a 7-pass radix select over the low 53 bits -- and the diagonal.
// The selection is marked in a bitmap over the row's keys and written out in
// ascending order by a block-wide scan of the bitmap.
__device__ void resolve_row(const MkArgs& a, int r, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int k = m.sparse_topk, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int b, t, p, n;
  query_row(a, r, b, t, p, n);
  int32_t* out = a.sel_idx + (int64_t)r * a.sel_ld;
  if (n <= k) {
    for (int j = tid; j < n; j += kT) out[j] = j;
    if (tid == 0) a.sel_cnt[r] = n;
    return;
  }
  __shared__ unsigned hist256[256];
  __shared__ unsigned wsum[32], s_total;
  __shared__ int s_digit, s_rem, s_done;
  unsigned* bits = reinterpret_cast<unsigned*>(smem);  // [kMkBitmapWords]
  unsigned long long* cs = reinterpret_cast<unsigned long long*>(smem) + kMkBitmapWords / 2;
  const int cap = (kPreOff - kMkBitmapWords * (int)sizeof(unsigned)) / (int)sizeof(unsigned long long);
  const int nw = (n + 31) / 32;
  const int above = min(max(__ldcg(a.hi_cnt + r), 0), k - 1);
  const int nc = min(max(__ldcg(a.cand_cnt + r), 0), c.max_ctx);
  const int need = k - above;
  const unsigned long long* cg = a.cand + (int64_t)r * c.max_ctx;
  const unsigned long long* cand = cg;
  for (int i = tid; i < nw; i += kT) bits[i] = 0u;
  if (nc <= cap) {
#pragma unroll 4
    for (int i = tid; i < nc; i += kT) cs[i] = __ldcg(cg + i);
    cand = cs;
  }
  __syncthreads();
  mark(a, 0);
#pragma unroll 2
  for (int i = tid; i < above; i += kT) {
    const int j = __ldcg(a.hi_list + (int64_t)r * k + i);
    if (j >= 0 && j < n) atomicOr(&bits[j >> 5], 1u << (j & 31));
  }
  unsigned long long prefix = 0ull, pmask = 0ull;
  int remaining = need;
  // radix select of the need-th largest candidate; it stops as soon as the chosen
  // digit's bucket holds exactly the remaining count (then every candidate with
  // the prefix so far is selected: the threshold is the prefix with zero low bits)
#pragma unroll 1
  for (int ps = 0; ps < 7 && nc > need; ++ps) {  // digits of 8 bits from bit 45 down, then the low 5 bits
    const int shift = ps < 6 ? 45 - 8 * ps : 0;
    const unsigned dm = ps < 6 ? 0xFFu : 0x1Fu;
    for (int i = tid; i < 256; i += kT) hist256[i] = 0u;
    __syncthreads();
    for (int i = tid; i < nc; i += kT) {
      const unsigned long long v = cand[i];
      if ((v & pmask) == prefix) atomicAdd(&hist256[(v >> shift) & dm], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      unsigned c8[8], sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c8[i] = hist256[255 - 8 * lane - i];
        sum += c8[i];
      }
      unsigned incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned tt = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += tt;
      }
      const unsigned excl = incl - sum;
      if (excl < (unsigned)remaining && incl >= (unsigned)remaining) {
        unsigned cum = excl;
        for (int i = 0; i < 8; ++i) {
          if (cum + c8[i] >= (unsigned)remaining) {
            s_digit = 255 - 8 * lane - i;
            s_rem = remaining - (int)cum;
            s_done = c8[i] == (unsigned)(remaining - (int)cum);
            break;
          }
          cum += c8[i];
        }
      }
    }
    __syncthreads();
    prefix |= (unsigned long long)s_digit << shift;
    pmask |= (unsigned long long)dm << shift;
    remaining = s_rem;
    const bool done = s_done != 0;
    __syncthreads();
    if (done) break;
  }
  mark(a, 1);
  // candidates at or above the need-th largest (low 53 bits; the top 11 are equal)
  const unsigned long long thr = prefix;
  const unsigned long long low = (1ull << 53) - 1;
  for (int i = tid; i < nc; i += kT) {
    const unsigned long long v = cand[i];
    if ((v & low) >= thr) {
      const int j = (int)(v & 0xFFFFFFFFull);
      if (j >= 0 && j < n) atomicOr(&bits[j >> 5], 1u << (j & 31));
    }
  }
  if (tid == 0) atomicOr(&bits[p >> 5], 1u << (p & 31));  // the diagonal
  __syncthreads();
  mark(a, 2);
  // ascending output: thread tid owns words [tid * wpt, (tid + 1) * wpt)
  const int wpt = (nw + kT - 1) / kT;
  unsigned cnt = 0;
  for (int wi = tid * wpt; wi < min(nw, (tid + 1) * wpt); ++wi) cnt += __popc(bits[wi]);
  unsigned pos = block_excl_scan(cnt, wsum, &s_total);
  for (int wi = tid * wpt; wi < min(nw, (tid + 1) * wpt); ++wi) {
    unsigned wv = bits[wi];
    while (wv) {
      const int bpos = __ffs(wv) - 1;
      wv &= wv - 1;
      if (pos < (unsigned)a.sel_ld) out[pos] = wi * 32 + bpos;
      ++pos;
    }
  }
  if (tid == 0) a.sel_cnt[r] = (int)min(s_total, (unsigned)a.sel_ld);
  __syncthreads();
}

// ------------------------------------------------- attention (cluster per query head)
// One cluster per query head h (KV head g = h / G) runs the whole attention
// mixer of an SWA or cross layer:
//   in-projection rows of the head (q; SWA also k and v of its KV head; the
//   head gate), tiles rank, rank + 8, ... per CTA -> distributed shared memory
//   -> q RMSNorm + RoPE (SWA: k too, and the first head of each KV group
//   appends this step's k / v to the window ring) -> each CTA attends over its
//   eighth of every query's keys (8-lane key groups, running softmax) -> the
//   CTA partials (max, sum, o) are merged by every CTA of the cluster -> the
//   gated head output times the head's column block of the o-projection for
//   this CTA's d/8 output rows -> added to the residual stream.
// Before the barrier that starts the phase (nothing there depends on the
// step's earlier phases): the o-projection block, norms, RoPE frequencies, and
// the K/V rows of this CTA's keys (SWA: the window's earlier positions; cross:
// the selected keys, except in the first cross layer, whose selection is
// resolved by the phase just before it) into shared memory.
constexpr int kParHeadO = kParConv;                      // [d/8 rows][hd/2 code bytes + scale words]
constexpr int kParHeadQn = kParHeadO + kMkMaxD / 8 * (128 / 2 + 8) / 4;  // q_norm [hd]
constexpr int kParHeadKn = kParHeadQn + 128;             // k_norm [hd]
constexpr int kParHeadInv = kParHeadKn + 128;            // RoPE inverse frequencies [rot/2]
constexpr int kHeadOTs = 8;                              // small-block index of the o-projection tile scales

struct HeadGeo {
  int hd, G, g, qt, ntile, HP, RC, d, nsw, os, sb0, gate_row;
  bool swa;
};

__device__ __forceinline__ HeadGeo head_geo(const CbModel& m, bool swa, int h) {
  HeadGeo e;
  e.swa = swa;
  e.hd = m.head_dim;
  e.G = m.n_q_heads / m.n_kv_heads;
  e.g = h / e.G;
  e.qt = e.hd / kTileRows;
  e.ntile = (swa ? 3 : 1) * e.qt + 1;
  e.HP = (swa ? 3 : 1) * e.hd + 1;
  e.d = m.d_model;
  e.RC = e.d / kCl;
  e.nsw = e.hd >= 128 ? 2 : 1;   // scale words per o-projection row slice
  e.os = e.hd / 2 + 4 * e.nsw;    // bytes per row slice
  e.sb0 = h * e.hd / 16;          // first scale byte of the head's columns in an o-projection row
  e.gate_row = (swa ? m.swa_off_gate : m.cr_off_gate) + h;
  return e;
}

// Entry j of head h's in-projection tile list: q tiles, (SWA) k tiles, v tiles, then the gate tile.
__device__ __forceinline__ int head_tile(const CbModel& m, const HeadGeo& e, int h, int j, int& hp_off) {
  if (j < e.qt) {
    hp_off = j * kTileRows;
    return (h * e.hd) / kTileRows + j;
  }
  j -= e.qt;
  if (e.swa) {
    if (j < e.qt) {
      hp_off = e.hd + j * kTileRows;
      return (m.swa_off_kv + e.g * e.hd) / kTileRows + j;
    }
    j -= e.qt;
    if (j < e.qt) {
      hp_off = 2 * e.hd + j * kTileRows;
      return (m.swa_off_kv + m.n_kv_heads * e.hd + e.g * e.hd) / kTileRows + j;
    }
  }
  hp_off = e.HP - 1;
  return e.gate_row / kTileRows;
}

template <typename F>
__device__ __forceinline__ int head_chunks(const CbMatrix& W, const CbModel& m, bool swa, int h, int rank, F&& f) {
  const HeadGeo e = head_geo(m, swa, h);
  const int64_t tb = tile_bytes(W.k);
  int n = 0, off = 0;
  for (int j = rank; j < e.ntile; j += kCl) {
    int hp_off;
    const int t = head_tile(m, e, h, j, hp_off);
    f(n++, W.tiles + t * tb, (unsigned)tb, off);
    off += (int)tb;
  }
  return n;
}

// Shared-memory plan of a head phase inside the work area.  xs (the
// in-projection input) is dead after the first cluster barrier and the
// attention scratch overlays it; hp and part are read by the cluster; the
// prefetched K/V rows take what is left below the parameter region.
template <int M>
struct HeadSmem {
  static constexpr int QG = M <= 5 ? M : 4;  // queries per pass over the keys
  float *xs, *qs, *og, *wpart, *hp, *part;
  uint16_t *kc, *vc, *kvb;
  int nbuf_max;
};

template <int M>
__device__ __forceinline__ HeadSmem<M> head_smem(float* work, const HeadGeo& e) {
  HeadSmem<M> s;
  const int hd = e.hd;
  s.xs = work;                                               // [M][xpad(d)]
  s.qs = work;                                               // [M][hd] scaled queries
  s.kc = reinterpret_cast<uint16_t*>(s.qs + M * hd);         // [M][hd] this step's keys (bf16)
  s.vc = s.kc + M * hd;                                      // [M][hd] this step's values (bf16)
  s.og = s.qs + 2 * M * hd;                                  // [M][hd] gated head output
  s.wpart = s.og + M * hd;                                   // [kW][QG][hd + 2] warp partials
  const int over = pad4(3 * M * hd + kW * HeadSmem<M>::QG * (hd + 2));
  s.hp = work + max(pad4(M * xpad(e.d)), over);             // [M][HP]
  s.part = s.hp + pad4(M * e.HP);                            // [M][hd + 2] this CTA's partial per row
  const int used = (int)(s.part - work) + pad4(M * (hd + 2));
  s.nbuf_max = max(0, (kPreOff / 4 - used) / hd);            // a key row pair is hd floats
  s.kvb = reinterpret_cast<uint16_t*>(work + kPreOff / 4 - s.nbuf_max * hd);  // [nbuf_max][K hd | V hd]
  return s;
}

// The phase's rows and key segments (per CTA; kept from the preload to the phase).
// The first cross layer's plan is kept for the later ones (same rows, same
// selections): g_cross_ready marks it, g_keys holds this rank's selected key
// indices.  s_self_pos: positions of the self-decoder rows, read at launch start.
constexpr int kHeadKeys = 512;
__shared__ int h_pos[kMkMaxRows], h_seq[kMkMaxRows], h_n[kMkMaxRows], s_self_pos[kMkMaxRows];
__shared__ int g_keys[kHeadKeys], g_nkeys, g_cross_ready;
__shared__ int g_lo[kMkMaxRows], g_n[kMkMaxRows], g_c0[kMkMaxRows], g_s0[kMkMaxRows], g_b[kMkMaxRows],
    g_row[kMkMaxRows], g_p0[kMkMaxRows];
__shared__ int g_nseg, g_tot, g_nbuf;

// Row r < Mr (thread r): position, sequence and, for cross rows, the key count.
__device__ __forceinline__ void head_rows(const MkArgs& a, bool swa, int Mr) {
  const int r = threadIdx.x;
  if (r < Mr) {
    int b, t, p, n = 0;
    if (swa) {
      b = r / a.T;
      p = s_self_pos[r];
    } else {
      query_row(a, r, b, t, p, n);
      if (a.m.sparse_topk > 0) n = min(__ldcg(a.sel_cnt + r), a.sel_ld);
    }
    h_pos[r] = p;
    h_seq[r] = b;
    h_n[r] = n;
  }
}

// Thread 0: the key segments of the pass over rows r0 .. r0 + nq - 1 (SWA: one per
// sequence, the union of its queries' windows; cross: one per row, its
// selection) and this rank's eighth of each, concatenated.
__device__ __forceinline__ void head_segments(const MkArgs& a, bool swa, int r0, int nq, int rank) {
  int ns = 0, tot = 0;
  for (int j = 0; j < nq; ++j) {
    const int r = r0 + j;
    int lo, hi;
    if (swa) {
      lo = max(0, h_pos[r] - a.m.swa_window + 1);
      hi = h_pos[r];
      if (ns > 0 && g_b[ns - 1] == h_seq[r]) {  // a later token of the same sequence extends its segment
        g_n[ns - 1] = hi - g_lo[ns - 1] + 1;
        continue;
      }
    } else {
      lo = 0;
      hi = h_n[r] - 1;
    }
    g_lo[ns] = lo;
    g_n[ns] = hi - lo + 1;
    g_b[ns] = h_seq[r];
    g_row[ns] = r;
    g_p0[ns] = h_pos[r] - (r - h_seq[r] * a.T);  // position of the sequence's first token of this step
    ++ns;
  }
  for (int s = 0; s < ns; ++s) {
    const int n = max(0, g_n[s]);
    const int a0 = n * rank / kCl, a1 = n * (rank + 1) / kCl;
    g_s0[s] = a0;
    g_c0[s] = tot;
    tot += a1 - a0;
  }
  g_nseg = ns;
  g_tot = tot;
}

// Key i of this rank's list: segment, position, and where its K/V rows are:
// 0 = global memory (ks / vs), 1 = this step's SWA token (row of kc / vc).
__device__ __forceinline__ int head_key(const MkArgs& a, const HeadGeo& e, bool swa, int layer, int i, bool need_src,
                                        int& seg, int& kp, const uint16_t*& ks, const uint16_t*& vs, int& mr) {
  int s = 0;
  while (s + 1 < g_nseg && i >= g_c0[s + 1]) ++s;
  seg = s;
  const int li = g_s0[s] + (i - g_c0[s]), b = g_b[s];
  const CbCache& c = a.c;
  const int hd = e.hd, Hkv = a.m.n_kv_heads;
  if (swa) {
    kp = g_lo[s] + li;
    if (kp >= g_p0[s]) {
      mr = b * a.T + (kp - g_p0[s]);
      return 1;
    }
    if (need_src) {
      const int64_t off = (((int64_t)(b * c.n_swa + a.m.self_layers[layer].slot) * c.swa_slots + kp % c.swa_slots) *
                               Hkv + e.g) * hd;
      ks = c.swa_k + off;
      vs = c.swa_v + off;
    }
    return 0;
  }
  kp = 0;
  if (need_src) {
    kp = a.m.sparse_topk == 0 ? li : i < g_nkeys ? g_keys[i] : __ldcg(a.sel_idx + (int64_t)g_row[s] * a.sel_ld + li);
    const int64_t off = (((int64_t)b * c.max_ctx + kp) * Hkv + e.g) * hd;
    ks = c.kv_k + off;
    vs = c.kv_v + off;
  }
  return 0;
}

// This rank's first nbuf keys (those in global memory) into kvb[i] = (K row, V row), 16 bytes per copy.
__device__ void head_prefetch(const MkArgs& a, const HeadGeo& e, bool swa, int layer, uint16_t* kvb, int nbuf) {
  const int hd = e.hd, per = hd / 8;
  for (int x = threadIdx.x; x < nbuf * per; x += kT) {
    const int i = x / per, q = x - i * per;
    int seg, kp, mr;
    const uint16_t *ks, *vs;
    if (head_key(a, e, swa, layer, i, true, seg, kp, ks, vs, mr) == 0) {
      cp_async16(kvb + (int64_t)i * 2 * hd + q * 8, ks + q * 8);
      cp_async16(kvb + (int64_t)i * 2 * hd + hd + q * 8, vs + q * 8);
    }
  }
}

// The first pass's rows, segments and K/V prefetch (every thread of the CTA).
template <int M>
__device__ void head_plan(const MkArgs& a, const HeadGeo& e, bool swa, int layer, int rank, float* work) {
  const int Mr = swa ? a.B * a.T : a.B * a.nq;
  if (swa || !g_cross_ready) {
    head_rows(a, swa, Mr);
    __syncthreads();
    if (threadIdx.x == 0) {
      head_segments(a, swa, 0, min(HeadSmem<M>::QG, Mr), rank);
      g_nbuf = min(g_tot, head_smem<M>(work, e).nbuf_max);
    }
    __syncthreads();
    if (!swa && Mr <= HeadSmem<M>::QG) {  // one pass: keep the plan and this rank's keys for the later layers
      const int nk = a.m.sparse_topk > 0 ? min(g_tot, kHeadKeys) : 0;
      for (int i = threadIdx.x; i < nk; i += kT) {
        int s = 0;
        while (s + 1 < g_nseg && i >= g_c0[s + 1]) ++s;
        g_keys[i] = __ldcg(a.sel_idx + (int64_t)g_row[s] * a.sel_ld + g_s0[s] + (i - g_c0[s]));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        g_nkeys = nk;
        g_cross_ready = 1;
      }
      __syncthreads();
    }
  }
  head_prefetch(a, e, swa, layer, head_smem<M>(work, e).kvb, g_nbuf);
}

// Before the barrier: norm vector, in-projection tile scales, q/k norms, RoPE
// frequencies, this rank's o-projection rows restricted to the head's
// columns, and (SWA, later cross layers) the plan and K/V prefetch.
template <int M>
__device__ void head_preload(const MkArgs& a, bool swa, int layer, int h, int rank, float* work) {
  const CbModel& m = a.m;
  const HeadGeo e = head_geo(m, swa, h);
  const CbMatrix& W = swa ? m.self_layers[layer].in_proj : m.cross_layers[layer].q_gate;
  const CbMatrix& O = swa ? m.self_layers[layer].o_proj : m.cross_layers[layer].o_proj;
  const float* norm1 = swa ? m.self_layers[layer].norm1 : m.cross_layers[layer].norm1;
  const float* qn = swa ? m.self_layers[layer].q_norm : m.cross_layers[layer].q_norm;
  const int tid = threadIdx.x;
  float* pn = par_norm(work);
  float* ps = par_small(work);
  for (int i = tid; i < e.d / 4; i += kT) cp_async16(pn + 4 * i, norm1 + 4 * i);
  if (tid == 0) {
    int q = 0;
    for (int j = rank; j < e.ntile; j += kCl, ++q) {
      int hp_off;
      cp_async4(ps + q, W.tile_scale + head_tile(m, e, h, j, hp_off));
    }
  }
  cp_async_commit();  // the first group: what the in-projection needs; the rest is waited after it
  const int n0 = rank * e.RC, t0 = n0 / kTileRows, nt = (n0 + e.RC - 1) / kTileRows - t0 + 1;
  for (int i = tid; i < nt; i += kT) cp_async4(ps + kHeadOTs + i, O.tile_scale + t0 + i);
  float* pq = work + kPreOff / 4 + kParHeadQn;
  float* pk = work + kPreOff / 4 + kParHeadKn;
  float* pf = work + kPreOff / 4 + kParHeadInv;
  for (int i = tid; i < e.hd; i += kT) {
    cp_async4(pq + i, qn + i);
    if (swa) cp_async4(pk + i, m.self_layers[layer].k_norm + i);
  }
  for (int i = tid; i < m.rot_dim / 2; i += kT) cp_async4(pf + i, m.inv_freq + i);
  uint8_t* ob = reinterpret_cast<uint8_t*>(work + kPreOff / 4 + kParHeadO);
  const int K = O.k, wpr = e.hd / 8 + e.nsw;  // words per row slice
  const int64_t tb = tile_bytes(K);
  for (int i = tid; i < e.RC * wpr; i += kT) {
    const int row = i / wpr, wd = i - row * wpr, n = n0 + row, w = n & (kTileRows - 1);
    const uint8_t* tile = O.tiles + (int64_t)(n / kTileRows) * tb;
    const uint8_t* src = wd < e.hd / 8 ? tile + w * (K / 2) + h * (e.hd / 2) + wd * 4
                                       : tile + kTileRows * (K / 2) + w * (K / 16) + (e.sb0 & ~3) + (wd - e.hd / 8) * 4;
    cp_async4(ob + row * e.os + wd * 4, src);
  }
  if (swa || layer > 0) head_plan<M>(a, e, swa, layer, rank, work);
  cp_async_commit();
}

// RMSNorm over hd (weights w) + partial interleaved RoPE at position p of a
// shared-memory vector, one warp; out = result * oscale.  When bits is set the
// result is rounded to bfloat16 first and the bits are stored there too.
__device__ __forceinline__ void head_norm_rope(const float* x, const float* w, int hd, int rot2, int p,
                                               const float* inv_freq, float eps, float oscale, float* out,
                                               uint16_t* bits) {
  const int lane = threadIdx.x & 31;
  float ss = 0.0f;
  for (int i = lane; i < hd; i += 32) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float rn = rsqrtf(ss / (float)hd + eps);
  for (int j = lane; j < hd / 2; j += 32) {
    float x1 = x[2 * j] * rn * w[2 * j];
    float x2 = x[2 * j + 1] * rn * w[2 * j + 1];
    if (j < rot2) rope_pair(x1, x2, p, inv_freq[j]);
    if (bits) {
      const uint16_t b1 = f32_to_bf16(x1), b2 = f32_to_bf16(x2);
      bits[2 * j] = b1;
      bits[2 * j + 1] = b2;
      x1 = bf16_to_f32(b1);
      x2 = bf16_to_f32(b2);
    }
    out[2 * j] = x1 * oscale;
    out[2 * j + 1] = x2 * oscale;
  }
}

__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Running-softmax update of one query with one key score.
__device__ __forceinline__ void soft_update(float sc, const float (&vf)[8], float& mq, float& lq, float (&o)[8]) {
  const float mn = fmaxf(mq, sc);
  const float c = mq == -INFINITY ? 0.0f : expf(mq - mn);
  const float pe = expf(sc - mn);
  lq = lq * c + pe;
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = fmaf(pe, vf[e], o[e] * c);
  mq = mn;
}

template <int M>
__device__ void head_phase(const MkArgs& a, bool swa, int layer, bool first, bool live, int h, int rank,
                           const uint8_t* slot, float* work) {
  constexpr int QG = HeadSmem<M>::QG;
  constexpr int KU = QG == 1 ? 1 : 2;  // keys per key group in flight (one row: a compact loop)
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const HeadGeo e = head_geo(m, swa, h);
  const HeadSmem<M> sm = head_smem<M>(work, e);
  const CbMatrix& W = swa ? m.self_layers[layer].in_proj : m.cross_layers[layer].q_gate;
  long long* resid = swa ? a.hq : a.xq;
  const int Mr = swa ? a.B * a.T : a.B * a.nq;
  const int hd = e.hd, HP = e.HP, d = e.d, K = W.k;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tb = tile_bytes(K);
  float* xs = sm.xs;
  float* qs = sm.qs;
  uint16_t* kc = sm.kc;
  uint16_t* vc = sm.vc;
  float* og = sm.og;
  float* wpart = sm.wpart;
  float* hp = sm.hp;
  float* part = sm.part;
  const float* ps = par_small(work);
  const float* qn = work + kPreOff / 4 + kParHeadQn;
  const float* kn = work + kPreOff / 4 + kParHeadKn;
  const float* inv = work + kPreOff / 4 + kParHeadInv;
  const uint8_t* ob = reinterpret_cast<const uint8_t*>(work + kPreOff / 4 + kParHeadO);
  const bool planned = swa || layer > 0;  // plan and K/V prefetch done before the barrier
  if (live) {
    if (!planned) head_plan<M>(a, e, swa, layer, rank, work);  // the first cross layer: selections are new
    __shared__ int s_rows[kMkMaxRows];
    if (tid < kMkMaxRows) s_rows[tid] = tid;
    __syncthreads();
    float rn[M];
    stage_rows<M>(resid, nullptr, d, s_rows, Mr, K, par_norm(work), m.norm_eps, xs, rn, nullptr,
                  (swa && first && h == 0 && rank == 0) ? a.hq : nullptr, (swa && first) ? &a : nullptr);
    mark(a, 0);
    int off = 0, q = 0;
    for (int j = rank; j < e.ntile; j += kCl, ++q) {
      int hp_off;
      head_tile(m, e, h, j, hp_off);
      const bool gate_tile = j == e.ntile - 1;
      if (!gate_tile || warp == (e.gate_row & (kTileRows - 1))) {  // the gate tile: the head's row only
        float acc[M];
        row_dot<M>(slot + off, K, warp, true, false, xs, acc);
        const float ts = ps[q];
        const int col = gate_tile ? HP - 1 : hp_off + warp;
        if (lane < kCl)
#pragma unroll
          for (int mr = 0; mr < M; ++mr)
            if (mr < Mr) st_dsmem(dsmem(hp + mr * HP + col, lane), acc[mr] * ts * rn[mr]);
      }
      off += (int)tb;
    }
  }
  cp_async_wait_all();  // the preload's second group; the cluster barrier publishes it
  cluster_sync();  // every rank's in-projection rows are in every rank's hp
  mark(a, 1);
  if (live) {
    const int rot2 = m.rot_dim / 2;
    const float scale = rsqrtf((float)hd);
    const bool writer = swa && h % e.G == 0 && rank == 0;  // appends this step's k / v to the ring
    const int nj = swa ? 3 : 1;                            // q; SWA also k and v, one warp each
    for (int job = warp; job < Mr * nj; job += kW) {
      const int mr = job / nj, kind = job - mr * nj, p = h_pos[mr];
      int64_t roff = 0;
      if (writer)
        roff = (((int64_t)(h_seq[mr] * c.n_swa + m.self_layers[layer].slot) * c.swa_slots + p % c.swa_slots) *
                    m.n_kv_heads + e.g) * hd;
      if (kind == 0) {
        head_norm_rope(hp + mr * HP, qn, hd, rot2, p, inv, m.norm_eps, scale, qs + mr * hd, nullptr);
      } else if (kind == 1) {
        head_norm_rope(hp + mr * HP + hd, kn, hd, rot2, p, inv, m.norm_eps, 1.0f, og + mr * hd, kc + mr * hd);
        if (writer) {
          __syncwarp();
          for (int dd = lane; dd < hd; dd += 32) c.swa_k[roff + dd] = kc[mr * hd + dd];
        }
      } else {
        for (int dd = lane; dd < hd; dd += 32) {
          const uint16_t v = f32_to_bf16(hp[mr * HP + 2 * hd + dd]);
          vc[mr * hd + dd] = v;
          if (writer) c.swa_v[roff + dd] = v;
        }
      }
    }
    __syncthreads();
    mark(a, 2);
    // ---- attention: groups of LK lanes hold one key (8 dims per lane)
    const int LK = hd / 8, KG = 32 / LK, NG = kW * KG;
    const int grp = warp * KG + lane / LK, sub = lane % LK;
    for (int r0 = 0; r0 < Mr; r0 += QG) {
      const int nq = min(QG, Mr - r0);
      int nbuf = 0;
      if (r0 == 0) {
        cp_async_wait_all();  // the prefetched keys
        nbuf = g_nbuf;
      } else if (tid == 0) {
        head_segments(a, swa, r0, nq, rank);
      }
      __syncthreads();
      const int tot = g_tot;
      float o[QG][8], mq[QG], lq[QG];
#pragma unroll
      for (int j = 0; j < QG; ++j) {
        mq[j] = -INFINITY;
        lq[j] = 0.0f;
#pragma unroll
        for (int x = 0; x < 8; ++x) o[j][x] = 0.0f;
      }
      for (int base = 0; base < tot; base += NG * KU) {
        uint4 kq[KU], vq[KU];
        int kpos[KU], kseg[KU];
#pragma unroll
        for (int u = 0; u < KU; ++u) {
          const int i = base + u * NG + grp;
          kseg[u] = -1;
          kpos[u] = 0;
          kq[u] = make_uint4(0u, 0u, 0u, 0u);
          vq[u] = kq[u];
          if (i < tot) {
            int seg, kp, mr;
            const uint16_t *ks, *vs;
            const int where = head_key(a, e, swa, layer, i, i >= nbuf, seg, kp, ks, vs, mr);
            if (where == 1) {
              kq[u] = *reinterpret_cast<const uint4*>(kc + mr * hd + sub * 8);
              vq[u] = *reinterpret_cast<const uint4*>(vc + mr * hd + sub * 8);
            } else if (i < nbuf) {
              kq[u] = *reinterpret_cast<const uint4*>(sm.kvb + (int64_t)i * 2 * hd + sub * 8);
              vq[u] = *reinterpret_cast<const uint4*>(sm.kvb + (int64_t)i * 2 * hd + hd + sub * 8);
            } else {
              kq[u] = __ldcg(reinterpret_cast<const uint4*>(ks + sub * 8));
              vq[u] = __ldcg(reinterpret_cast<const uint4*>(vs + sub * 8));
            }
            kpos[u] = kp;
            kseg[u] = seg;
          }
        }
#pragma unroll
        for (int u = 0; u < KU; ++u) {
          const uint32_t kw[4] = {kq[u].x, kq[u].y, kq[u].z, kq[u].w}, vw[4] = {vq[u].x, vq[u].y, vq[u].z, vq[u].w};
          float kf[8], vf[8];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            kf[2 * x] = bf16_to_f32(kw[x]);
            kf[2 * x + 1] = bf16_to_f32(kw[x] >> 16);
            vf[2 * x] = bf16_to_f32(vw[x]);
            vf[2 * x + 1] = bf16_to_f32(vw[x] >> 16);
          }
          if constexpr (QG == 1) {  // one query row
#pragma unroll
            for (int j = 0; j < QG; ++j) {
              if (j < nq) {
                const float4 q0 = *reinterpret_cast<const float4*>(qs + (r0 + j) * hd + sub * 8);
                const float4 q1 = *reinterpret_cast<const float4*>(qs + (r0 + j) * hd + sub * 8 + 4);
                float sc = q0.x * kf[0];
                sc = fmaf(q0.y, kf[1], sc);
                sc = fmaf(q0.z, kf[2], sc);
                sc = fmaf(q0.w, kf[3], sc);
                sc = fmaf(q1.x, kf[4], sc);
                sc = fmaf(q1.y, kf[5], sc);
                sc = fmaf(q1.z, kf[6], sc);
                sc = fmaf(q1.w, kf[7], sc);
                for (int x = LK / 2; x > 0; x >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, x);
                const int s = kseg[u];
                bool ok = s >= 0;
                if (ok) {
                  if (swa) {
                    const int pj = h_pos[r0 + j];
                    ok = g_b[s] == h_seq[r0 + j] && kpos[u] <= pj && kpos[u] > pj - m.swa_window;
                  } else {
                    ok = g_row[s] == r0 + j;
                  }
                }
                if (ok) soft_update(sc, vf, mq[j], lq[j], o[j]);
              }
            }
          } else {
            auto score = [&](int j) {  // this lane's part of q_j . k, reduced over the key group
              const float4 q0 = *reinterpret_cast<const float4*>(qs + (r0 + j) * hd + sub * 8);
              const float4 q1 = *reinterpret_cast<const float4*>(qs + (r0 + j) * hd + sub * 8 + 4);
              float sc = q0.x * kf[0];
              sc = fmaf(q0.y, kf[1], sc);
              sc = fmaf(q0.z, kf[2], sc);
              sc = fmaf(q0.w, kf[3], sc);
              sc = fmaf(q1.x, kf[4], sc);
              sc = fmaf(q1.y, kf[5], sc);
              sc = fmaf(q1.z, kf[6], sc);
              sc = fmaf(q1.w, kf[7], sc);
              for (int x = LK / 2; x > 0; x >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, x);
              return sc;
            };
            const int s = kseg[u];
            if (swa) {  // every query of the pass may see the key (window and causal masks)
#pragma unroll
              for (int j = 0; j < QG; ++j) {
                if (j < nq) {
                  const float sc = score(j);
                  const int pj = h_pos[r0 + j];
                  if (s >= 0 && g_b[s] == h_seq[r0 + j] && kpos[u] <= pj && kpos[u] > pj - m.swa_window)
                    soft_update(sc, vf, mq[j], lq[j], o[j]);
                }
              }
            } else {  // a selected key belongs to one query row: score it against that row only
              const int jr = s >= 0 ? g_row[s] - r0 : 0;
              const float sc = score(jr);
#pragma unroll
              for (int j = 0; j < QG; ++j)
                if (s >= 0 && j == jr) soft_update(sc, vf, mq[j], lq[j], o[j]);
            }
          }
        }
      }
      if (r0 == 0) mark(a, 3);
      // merge the key groups of the warp, then the warps
      for (int x = LK; x < 32; x <<= 1) {
#pragma unroll
        for (int j = 0; j < QG; ++j) {
          const float m2 = __shfl_xor_sync(0xffffffffu, mq[j], x), l2 = __shfl_xor_sync(0xffffffffu, lq[j], x);
          const float mn = fmaxf(mq[j], m2);
          const float c1 = mq[j] == -INFINITY ? 0.0f : expf(mq[j] - mn);
          const float c2 = m2 == -INFINITY ? 0.0f : expf(m2 - mn);
          lq[j] = lq[j] * c1 + l2 * c2;
#pragma unroll
          for (int y = 0; y < 8; ++y) {
            const float o2 = __shfl_xor_sync(0xffffffffu, o[j][y], x);
            o[j][y] = o[j][y] * c1 + o2 * c2;
          }
          mq[j] = mn;
        }
      }
      if (lane < LK) {
#pragma unroll
        for (int j = 0; j < QG; ++j) {
          float* wp = wpart + (warp * QG + j) * (hd + 2);
          if (lane == 0) {
            wp[0] = mq[j];
            wp[1] = lq[j];
          }
#pragma unroll
          for (int y = 0; y < 8; ++y) wp[2 + sub * 8 + y] = o[j][y];
        }
      }
      __syncthreads();
      for (int i = tid; i < nq * (hd + 2); i += kT) {
        const int j = i / (hd + 2), x = i - j * (hd + 2);
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kW; ++w) mx = fmaxf(mx, wpart[(w * QG + j) * (hd + 2)]);
        float v = mx;
        if (x > 0) {
          v = 0.0f;
#pragma unroll
          for (int w = 0; w < kW; ++w) {
            const float* wp = wpart + (w * QG + j) * (hd + 2);
            if (wp[0] != -INFINITY) v += wp[x] * expf(wp[0] - mx);
          }
        }
        part[(r0 + j) * (hd + 2) + x] = v;
      }
      __syncthreads();
    }
  }
  mark(a, 4);
  cluster_sync();  // every rank's partials are complete
  mark(a, 5);
  if (live) {
    // merge the cluster's partials (every rank, all rows) into the gated head output
    for (int i = tid; i < Mr * hd; i += kT) {
      const int mr = i / hd, dd = i - mr * hd;
      float mr_[kCl], lr[kCl], orr[kCl];
#pragma unroll
      for (int r = 0; r < kCl; ++r) {
        const float* pp = part + mr * (hd + 2);
        mr_[r] = ld_dsmem(dsmem(pp, r));
        lr[r] = ld_dsmem(dsmem(pp + 1, r));
        orr[r] = ld_dsmem(dsmem(pp + 2 + dd, r));
      }
      float mx = -INFINITY;
#pragma unroll
      for (int r = 0; r < kCl; ++r) mx = fmaxf(mx, mr_[r]);
      float L = 0.0f, O = 0.0f;
#pragma unroll
      for (int r = 0; r < kCl; ++r) {
        if (mr_[r] == -INFINITY) continue;
        const float w = expf(mr_[r] - mx);
        L = fmaf(lr[r], w, L);
        O = fmaf(orr[r], w, O);
      }
      og[i] = L > 0.0f ? (O / L) * sigmoid(hp[mr * HP + HP - 1]) : 0.0f;
    }
    __syncthreads();
    // o-projection: output rows rank * RC ... of the head's hd columns, hd / 16 lanes per row
    const int LQ = hd / 16, total = e.RC * LQ, n0 = rank * e.RC, t0 = n0 / kTileRows;
    for (int base = 0; base < total; base += kT) {
      const int i = base + tid, row = i / LQ, qb = i - row * LQ;
      const bool valid = i < total;
      float acc[M];
#pragma unroll
      for (int mr = 0; mr < M; ++mr) acc[mr] = 0.0f;
      if (valid) {
        const uint8_t* rb = ob + row * e.os;
        const uint32_t c0 = *reinterpret_cast<const uint32_t*>(rb + qb * 8);
        const uint32_t c1 = *reinterpret_cast<const uint32_t*>(rb + qb * 8 + 4);
        const int n = n0 + row;
        const float sc = e4m3_to_f32(rb[e.hd / 2 + (e.sb0 & 3) + qb]) * ps[kHeadOTs + n / kTileRows - t0];
        float w[16];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float2 lo = e2m1x2_to_f32x2(c0 >> (8 * x)), hi = e2m1x2_to_f32x2(c1 >> (8 * x));
          w[2 * x] = lo.x;
          w[2 * x + 1] = lo.y;
          w[8 + 2 * x] = hi.x;
          w[8 + 2 * x + 1] = hi.y;
        }
#pragma unroll
        for (int mr = 0; mr < M; ++mr) {
          if (mr < Mr) {
            const float* ov = og + mr * hd + qb * 16;
            float p = 0.0f;
#pragma unroll
            for (int x = 0; x < 16; ++x) p = fmaf(w[x], ov[x], p);
            acc[mr] = p * sc;
          }
        }
      }
#pragma unroll
      for (int mr = 0; mr < M; ++mr)
        for (int x = LQ / 2; x > 0; x >>= 1) acc[mr] += __shfl_xor_sync(0xffffffffu, acc[mr], x);
      if (valid && qb == 0)
#pragma unroll
        for (int mr = 0; mr < M; ++mr)
          if (mr < Mr) red_fix(resid + (int64_t)mr * d + n0 + row, acc[mr]);
    }
  }
}

// ------------------------------------------------------------------ phase plan
__device__ int build_plan(const CbModel& m, uint16_t* plan) {
  int n = 0;
  auto push = [&](int kind, int layer) { plan[n++] = (uint16_t)((kind << 8) | layer); };
  for (int i = 0; i < m.n_self_layers; ++i) {
    if (m.self_layers[i].kind == CB_LAYER_GDN) {
      push(PH_GDN, i);
    } else {
      push(PH_SWA_HEAD, i);
    }
    push(PH_FFN_SELF, i);
  }
  push(PH_SH_PROJ, 0);
  push(PH_SH_SCORE, 0);
  if (m.sparse_topk > 0) {
    push(PH_SH_COMPACT, 0);
    push(PH_CR_RESOLVE, 0);
  }
  for (int j = 0; j < m.n_cross_layers; ++j) {
    push(PH_CR_HEAD, j);
    push(PH_FFN_CROSS, j);
  }
  push(PH_LM_HEAD, 0);
  return n;
}

// The GEMV of a GEMV phase (input, output, this CTA's units).
__device__ GemvJob gemv_job(const MkArgs& a, int kind, int layer) {
  const CbModel& m = a.m;
  const int d = m.d_model;
  GemvJob g{};
  g.ucta = blockIdx.x;
  g.uncta = gridDim.x;
  g.ldx = d;
  g.epi = EPI_STORE_;
  switch (kind) {
    case PH_SH_PROJ:
      g.W = m.shared_proj;
      g.xq = a.hq;
      g.pre = PRE_RMS_;
      g.norm_w = m.shared_norm;
      g.y = a.proj;
      g.ldy = a.ldp;
      g.rows_out = m.shared_proj.rows;
      break;
    default:  // PH_LM_HEAD
      g.W = m.lm_head;
      g.xq = a.xq;
      g.pre = PRE_RMS_;
      g.norm_w = m.final_norm;
      g.y = a.logits ? a.logits : a.ws_logits;
      g.ldy = m.vocab_size;
      g.rows_out = m.vocab_size;
      g.argmax = true;
      break;
  }
  return g;
}

__device__ __forceinline__ bool is_gemv(int kind) {
  return kind == PH_SH_PROJ || kind == PH_LM_HEAD;
}

// Weight chunks of phase (kind, layer) for this CTA, in slot order: f(i, src, bytes, slot offset).
template <typename F>
__device__ int phase_chunks(const MkArgs& a, int kind, int layer, F&& f) {
  const CbModel& m = a.m;
  if (is_gemv(kind)) {
    const GemvJob g = gemv_job(a, kind, layer);
    const int nst = gemv_staged(g);
    const int64_t tb = tile_bytes(g.W.k);
    for (int i = 0; i < nst; ++i) f(i, g.W.tiles + (int64_t)(g.ucta + i * g.uncta) * tb, (unsigned)tb, (int)(i * tb));
    return nst;
  }
  if (kind == PH_GDN) {
    const int cid = (int)cluster_index();
    if (cid >= m.gdn_heads) return 0;
    return gdn_chunks(m.self_layers[layer], m, cid, (int)cluster_rank(), f);
  }
  if (kind == PH_FFN_SELF) {
    const CbSelfLayer& L = m.self_layers[layer];
    return ffn_chunks(L.gate_up, L.down_ks, m.ffn_hidden, blockIdx.x, gridDim.x, f);
  }
  if (kind == PH_FFN_CROSS) {
    const CbCrossLayer& L = m.cross_layers[layer];
    return ffn_chunks(L.gate_up, L.down_ks, m.ffn_hidden, blockIdx.x, gridDim.x, f);
  }
  if (kind == PH_SWA_HEAD || kind == PH_CR_HEAD) {
    const int cid = (int)cluster_index();
    if (cid >= m.n_q_heads) return 0;
    const bool swa = kind == PH_SWA_HEAD;
    return head_chunks(swa ? m.self_layers[layer].in_proj : m.cross_layers[layer].q_gate, m, swa, cid,
                       (int)cluster_rank(), f);
  }
  return 0;
}

// Between the arrival at the barrier before a GEMV or FFN phase and the wait
// there: the phase's norm vector, tile scales and tensor scale into the
// parameter region (cp.async; completed after the wait).  The GDN phase has
// its own (gdn_preload).
template <int M>
__device__ void phase_params(const MkArgs& a, int kind, int layer, float* work) {
  const CbModel& m = a.m;
  const int tid = threadIdx.x;
  float* pn = par_norm(work);
  float* ps = par_small(work);
  if (is_gemv(kind)) {
    const GemvJob g = gemv_job(a, kind, layer);
    const int n = min(gemv_mine(g), kParTs);
    if (n == 0) return;
    if (g.pre == PRE_RMS_ || g.pre == PRE_EMBED_)
      for (int i = tid; i < g.W.k / 4; i += kT) cp_async16(pn + 4 * i, g.norm_w + 4 * i);
    for (int i = tid; i < n; i += kT) cp_async4(ps + i, g.W.tile_scale + g.ucta + i * g.uncta);
  } else if (kind == PH_FFN_SELF || kind == PH_FFN_CROSS) {
    const bool self = kind == PH_FFN_SELF;
    const CbMatrix& GU = self ? m.self_layers[layer].gate_up : m.cross_layers[layer].gate_up;
    const CbSliced& D = self ? m.self_layers[layer].down_ks : m.cross_layers[layer].down_ks;
    const float* norm2 = self ? m.self_layers[layer].norm2 : m.cross_layers[layer].norm2;
    const int n = min(ffn_mine(m.ffn_hidden, GU.k, blockIdx.x, gridDim.x), 16);
    if (n == 0) return;
    const int x = ffn_extra(m.ffn_hidden, GU.k, blockIdx.x, gridDim.x);
    if (x >= 0 && tid < 2) cp_async4(ps + 32 + tid, GU.tile_scale + (tid == 0 ? x : m.ffn_hidden / kTileRows + x));
    for (int i = tid; i < m.d_model / 4; i += kT) cp_async16(pn + 4 * i, norm2 + 4 * i);
    for (int i = tid; i < n; i += kT) {
      const int j = blockIdx.x + i * gridDim.x;
      cp_async4(ps + i, GU.tile_scale + j);
      cp_async4(ps + 16 + i, GU.tile_scale + m.ffn_hidden / kTileRows + j);
    }
    if (tid == 0) cp_async4(ps + PS_TSCALE, D.tensor_scale);
  } else if (kind == PH_SWA_HEAD || kind == PH_CR_HEAD) {
    const int cid = (int)cluster_index();
    if (cid < m.n_q_heads) head_preload<M>(a, kind == PH_SWA_HEAD, layer, cid, (int)cluster_rank(), work);
  }
}

// The copy warp: arm the slot's mbarrier with the phase's byte count and start its copies.
__device__ void stage_issue(const MkArgs& a, int kind, int layer, uint8_t* slot, unsigned long long* bar) {
  const int lane = threadIdx.x & 31;
  unsigned total = 0;
  phase_chunks(a, kind, layer, [&](int, const uint8_t*, unsigned bytes, int) { total += bytes; });
  if (lane == 0) {
    fence_proxy_async();  // the slot's previous contents were read by ordinary loads
    mbar_expect_arrive(bar, total);
  }
  __syncwarp();
  phase_chunks(a, kind, layer, [&](int i, const uint8_t* src, unsigned bytes, int off) {
    if ((i & 31) == lane) bulk_copy(slot + off, src, bytes, bar);
  });
}

// The copy warp, last phase only: the GEMV tiles after the staged ones into the other slot.
__device__ void stage_issue_extra(const MkArgs& a, int kind, int layer, uint8_t* slot, unsigned long long* bar) {
  const int lane = threadIdx.x & 31;
  const GemvJob g = gemv_job(a, kind, layer);
  const int nst = gemv_staged(g), nx = gemv_extra(g);
  if (nx == 0) return;
  const int64_t tb = tile_bytes(g.W.k);
  if (lane == 0) {
    fence_proxy_async();
    mbar_expect_arrive(bar, (unsigned)(nx * tb));
  }
  __syncwarp();
  for (int i = lane; i < nx; i += 32)
    bulk_copy(slot + i * tb, g.W.tiles + (int64_t)(g.ucta + (nst + i) * g.uncta) * tb, (unsigned)tb, bar);
}

// ------------------------------------------------------------------ kernel
template <int M>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) unsigned long long s_bar[2];
  __shared__ uint16_t s_plan[kMaxPhases];
  __shared__ int s_np, s_ok, s_live;
  float* work = reinterpret_cast<float*>(smem + 2 * kSlot);
  unsigned gen = 0;
  const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x, warp = tid >> 5;
  const int rank = (int)cluster_rank(), cid = (int)cluster_index();
  const CbModel& m = a.m;
  const int d = m.d_model, Mrows = a.B * a.T, RQ = a.B * a.nq;

  if (tid == 0) {
    s_np = build_plan(m, s_plan);
    mbar_init(&s_bar[0], 1);
    mbar_init(&s_bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const unsigned long long lim = __ldcg(&a.ctl->limit_ns);
    s_wait_limit = lim ? lim : kDefaultWaitNs;
    const int stall = __ldcg(&a.ctl->stall_barrier);
    s_stall_barrier = stall > 0 ? (unsigned)stall : 0u;
    s_live = 1;
    g_nkeys = 0;
    g_cross_ready = 0;
    if (cta == 0) a.trace[0] = gtimer();
  }
  if (tid < Mrows) s_self_pos[tid] = a.c.pos[tid / a.T] + a.c0 + tid % a.T;
  if (cta == 0) {
    // the histogram exists only with a top-k (dense cross attention carves it empty)
    if (m.sparse_topk > 0)
      for (int i = tid; i < RQ * kMkHistBins; i += kT) a.hist[i] = 0u;
    for (int i = tid; i < RQ; i += kT) {
      a.hi_cnt[i] = 0;
      a.cand_cnt[i] = 0;
      a.amax[i] = 0ull;
    }
    for (int i = tid; i < Mrows * d; i += kT) a.hq[i] = 0;  // the embedding is added in the first phase
  }
  __syncthreads();
  // bulk-copy phases issued and waited per slot (uniform in the CTA)
  unsigned issued0 = 0u, issued1 = 0u, waited0 = 0u, waited1 = 0u;
  const int P = s_np;
  if (warp == kCopyWarp) stage_issue(a, s_plan[0] >> 8, s_plan[0] & 0xFF, smem, &s_bar[0]);
  issued0 = 1;
  grid_arrive(a, gen);
  bool live = true;

  for (int p = 0; p < P; ++p) {
    const int kind = s_plan[p] >> 8, layer = s_plan[p] & 0xFF, sl = p & 1;
    int nst2 = 0;  // tiles of this phase in the other slot (last phase only)
    if (live && p + 1 < P) {  // the next phase's weights, into the other slot
      if (warp == kCopyWarp)
        stage_issue(a, s_plan[p + 1] >> 8, s_plan[p + 1] & 0xFF, smem + (sl ^ 1) * kSlot, &s_bar[sl ^ 1]);
      if (sl) issued0 += 1;
      else issued1 += 1;
    } else if (live && is_gemv(kind)) {  // the last phase: its later tiles into the free slot
      nst2 = gemv_extra(gemv_job(a, kind, layer));
      if (nst2 > 0) {
        if (warp == kCopyWarp) stage_issue_extra(a, kind, layer, smem + (sl ^ 1) * kSlot, &s_bar[sl ^ 1]);
        if (sl) issued0 += 1;
        else issued1 += 1;
      }
    }
    float st[M];  // the recurrent state of this thread's GDN columns, one value per sequence
    const bool gdn_here = kind == PH_GDN && cid < m.gdn_heads;
    if (tid == 0) s_mark_base = kMarkBase + 6 * p;
    if (live) {
      if (gdn_here) gdn_preload<M>(a, m.self_layers[layer], cid, rank, st, work);
      else phase_params<M>(a, kind, layer, work);
    }
    live = grid_wait(a, gen, &s_ok) && live;
    // this phase's parameters (GDN and attention phases: the first of their two groups)
    if (gdn_here || ((kind == PH_SWA_HEAD || kind == PH_CR_HEAD) && cid < m.n_q_heads)) cp_async_wait_prior();
    else cp_async_wait_all();
    __syncthreads();
    const unsigned iss = sl ? issued1 : issued0, wtd = sl ? waited1 : waited0;
    if (live && iss > wtd) {
      const bool ok = mbar_wait(&s_bar[sl], wtd & 1u);
      if (sl) waited1 += 1;
      else waited0 += 1;
      if (!ok && tid == 0) {
        raise_abort(a);
        s_live = 0;
      }
      __syncthreads();
      live = s_live != 0;
    }
    const uint8_t* slot = smem + sl * kSlot;
    switch (kind) {
      case PH_GDN:
        if (gdn_here) gdn_phase<M>(a, m.self_layers[layer], layer == 0, live, cid, rank, st, slot, work);
        break;
      case PH_FFN_SELF: {
        const CbSelfLayer& L = m.self_layers[layer];
        ffn_phase<M>(a, L.gate_up, L.down_ks, L.norm2, a.hq, Mrows, live, rank, cid, slot, work);
        break;
      }
      case PH_FFN_CROSS: {
        const CbCrossLayer& L = m.cross_layers[layer];
        ffn_phase<M>(a, L.gate_up, L.down_ks, L.norm2, a.xq, RQ, live, rank, cid, slot, work);
        break;
      }
      case PH_SWA_HEAD:
        if (cid < m.n_q_heads) head_phase<M>(a, true, layer, layer == 0, live, cid, rank, slot, work);
        break;
      case PH_CR_HEAD:
        if (cid < m.n_q_heads) head_phase<M>(a, false, layer, false, live, cid, rank, slot, work);
        break;
      case PH_SH_SCORE:
        if (live) {
          // the query rows of the self-decoder's output start the cross residual stream
          for (int i = cta * kT + tid; i < RQ * d; i += ncta * kT) {
            const int r = i / d, k = i - r * d, b = r / a.nq;
            a.xq[i] = __ldcg(a.hq + ((int64_t)b * a.T + (a.T - a.nq) + (r - b * a.nq)) * d + k);
          }
          shared_append(a, work);
          if (m.sparse_topk > 0) score_phase(a, work);
        }
        break;
      case PH_SH_COMPACT:
        if (live) compact_phase(a);
        break;
      case PH_CR_RESOLVE:
        if (live && cta < RQ) resolve_row(a, cta, work);
        break;
      default: {  // GEMV phases
        if (!live) break;
        const GemvJob g = gemv_job(a, kind, layer);
        const int rows = kind == PH_LM_HEAD ? RQ : Mrows;
        if (nst2 > 0) {  // the second slot's tiles (copies started before the barrier)
          const unsigned iss2 = sl ? issued0 : issued1, wtd2 = sl ? waited0 : waited1;
          if (iss2 > wtd2) {
            const bool ok = mbar_wait(&s_bar[sl ^ 1], wtd2 & 1u);
            if (sl) waited0 += 1;
            else waited1 += 1;
            if (!ok && tid == 0) {
              raise_abort(a);
              s_live = 0;
            }
            __syncthreads();
            if (s_live == 0) {
              live = false;
              break;
            }
          }
        }
        gemv_phase<M>(a, g, rows, slot, smem + (sl ^ 1) * kSlot, nst2, work);
        if (kind == PH_LM_HEAD && a.hidden != nullptr && cta == ncta - 1)
          for (int i = tid; i < RQ * d; i += kT) a.hidden[i] = from_fix(__ldcg(a.xq + i));
        break;
      }
    }
    grid_arrive(a, gen);
  }
  live = grid_wait(a, gen, &s_ok) && live;
  if (live && cta == 0) {
    if (a.argmax != nullptr)
      for (int r = tid; r < RQ; r += kT)
        a.argmax[r] = (int32_t)(0xFFFFFFFFu - (unsigned)(__ldcg(a.amax + r) & 0xFFFFFFFFull));
    for (int b = tid; b < a.B; b += kT) a.c.pos[b] += a.T;
  }
  // copies still in flight after an abort land before the CTA exits (bounded)
  for (; waited0 < issued0; ++waited0) mbar_wait(&s_bar[0], waited0 & 1u);
  for (; waited1 < issued1; ++waited1) mbar_wait(&s_bar[1], waited1 & 1u);
}

}  // namespace

size_t mk_smem_bytes() { return kSmem; }

int mk_swa_splits(const CbModel& m) { return ceil_div(m.swa_window + CB_MAX_T, kMkSwaSplit); }

static bool sliced_ok(const CbSliced& s, int rows, int k, int width) {
  return s.data != nullptr && s.tensor_scale != nullptr && s.rows == rows && s.k == k && s.width == width &&
         (reinterpret_cast<uintptr_t>(s.data) & 15) == 0;
}

bool mk_supported(const CbModel& m, const CbCache& c, int T, int nq) {
  const int G = m.n_q_heads / m.n_kv_heads, d = m.d_model;
  if (c.batch * T > kMkMaxRows || T > CB_MAX_T || nq < 1 || nq > T) return false;
  if (m.head_dim > 128 || m.head_dim % 8 || G * T > kMkMaxQ) return false;
  if (d > kMkMaxD || d % 16 || m.ffn_hidden % kTileRows || m.ffn_hidden > 2048) return false;
  if (m.n_q_heads * m.head_dim > kMkMaxD) return false;
  if (m.conv_size != 4) return false;
  if (m.sparse_topk > 0 && c.max_ctx > kMkBitmapWords * 32) return false;
  if (m.sparse_topk > 0 && (m.sparse_topk + 1 > kMaxSort || m.indexer_dim % 8 || m.indexer_dim > 256 ||
                            m.indexer_heads > 16 ||
                            kMkMaxRows * (m.indexer_heads * m.indexer_dim + 16 + kMkHistBins) * 4 +
                                    kMkMaxRows * m.indexer_dim > kPreOff))
    return false;
  // attention phases (a cluster per query head): hd / 8 lanes per key, 16-row
  // tiles of q / k / v, the o-projection's column block of each head on 4-byte words
  const int hd = m.head_dim;
  if (hd % 16 || 32 % (hd / 8) || d % kCl || (m.n_q_heads * hd) % 64 || m.rot_dim / 2 > 64) return false;
  {
    const int HP = 3 * hd + 1, QGm = 5;
    const size_t w = sizeof(float) * ((size_t)std::max(pad4(kMkMaxRows * xpad(d)),
                                                       pad4(3 * kMkMaxRows * hd + kW * QGm * (hd + 2))) +
                                      pad4(kMkMaxRows * HP) + (size_t)kMkMaxRows * (hd + 2));
    if (w > (size_t)kPreOff) return false;
    if ((int64_t)ceil_div(3 * hd / kTileRows + 1, kCl) * tile_bytes(d) > kSlot) return false;
  }
  // GEMV staging: [M][xpad(K)] inputs
  if ((size_t)kMkMaxRows * xpad(kMkMaxD) * sizeof(float) > (size_t)kPreOff) return false;
  // FFN: [8][M][d/8] partials + [M][xpad(d)] inputs + [M][16] + [4][M]
  if ((size_t)kMkMaxRows * (d + xpad(d) + 20) * sizeof(float) > (size_t)kPreOff) return false;
  const int64_t tb = tile_bytes(d);
  for (int i = 0; i < m.n_self_layers; ++i) {
    const CbSelfLayer& L = m.self_layers[i];
    if (L.in_proj.k != d || L.gate_up.k != d || L.o_proj.rows < d || L.down.rows < d) return false;
    if (L.kind != CB_LAYER_GDN && L.o_proj.k != m.n_q_heads * hd) return false;
    if (!sliced_ok(L.down_ks, d, m.ffn_hidden, 16)) return false;
    if (L.kind == CB_LAYER_GDN) {
      const int Dk = m.gdn_dk, Dv = m.gdn_dv, vpr = Dv / kCl;
      if (Dk % 16 || Dv % 16 || Dk > 64 || Dk * vpr > kMkThreads || vpr > kW) return false;
      if (m.gdn_off_gate % 16 || m.gdn_off_a % 16 || m.gdn_off_b % 16) return false;
      if (!sliced_ok(L.o_proj_ks, d, m.gdn_heads * Dv, vpr)) return false;
      const int ntile = (2 * Dk + 2 * Dv) / kTileRows;
      const int64_t slice = ((int64_t)d * (vpr / 2 + 1) + 15) / 16 * 16;
      if ((int64_t)(ceil_div(ntile, kCl) + 2) * tb + slice > kSlot) return false;
      // GDN working memory before the preload region; conv taps and windows after it
      const size_t w = sizeof(float) * ((size_t)kMkMaxRows * (2 * Dk + 2 * Dv + 2) + kCl * kMkMaxRows +
                                        (size_t)kMkMaxRows * (d + xpad(d)) + (size_t)kMkMaxRows * (2 * Dk + 2 * vpr) +
                                        kT + kW + 2 * kMkMaxRows + (size_t)kMkMaxRows * kT +
                                        36);  // + 16-byte padding of each array
      const size_t pre = sizeof(float) * ((size_t)kParConv + (size_t)(2 * Dk + vpr) * (4 + 3 * c.batch));
      if (w > (size_t)kPreOff || pre > (size_t)(kWork - kPreOff) || vpr > 16) return false;
    }
  }
  for (int j = 0; j < m.n_cross_layers; ++j) {
    const CbCrossLayer& L = m.cross_layers[j];
    if (L.q_gate.k != d || L.gate_up.k != d || L.o_proj.rows < d || L.o_proj.k != m.n_q_heads * hd) return false;
    if (!sliced_ok(L.down_ks, d, m.ffn_hidden, 16)) return false;
  }
  if (m.lm_head.k != d || m.shared_proj.k != d) return false;
  return true;
}

int launch_mk(const MkArgs& a, cudaStream_t st) {
  const int M = a.B * a.T;
  void (*fn)(MkArgs);
  if (M <= 1) fn = decode_mk_kernel<1>;
  else if (M <= 2) fn = decode_mk_kernel<2>;
  else if (M <= 4) fn = decode_mk_kernel<4>;
  else if (M <= 5) fn = decode_mk_kernel<5>;  // a verify of 1 + 4 drafts: fewer live registers than <8>
  else fn = decode_mk_kernel<8>;
  if (ensure_smem_attr((const void*)fn, kSmem) != CB_OK) return CB_ERR_CUDA;
  const int ncl = std::min(resident_clusters((const void*)fn, kMkThreads, kSmem, kCl), kMkMaxClusters);
  // every GDN head and every query head needs a cluster; one CTA resolves each query row's selection
  if (ncl < a.m.gdn_heads || ncl < a.m.n_q_heads || ncl * kCl < a.B * a.nq) return CB_ERR_SHAPE;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ncl * kCl);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = kCl;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeCooperative;
  attrs[1].val.cooperative = 1;
  cfg.attrs = attrs;
  // A cooperative launch guarantees co-residency.  Where the runtime does not
  // combine it with clusters, the plain cluster launch runs the same grid: every
  // cluster fits at once (the count comes from the occupancy query), and the
  // bounded waits end a launch whose CTAs are not all resident.
  const bool coop = cooperative_clusters_ok();
  cfg.numAttrs = coop ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
  if (e != cudaSuccess && coop) {
    (void)cudaGetLastError();
    note_cooperative_clusters_refused();
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, fn, a);
  }
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb
