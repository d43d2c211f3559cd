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
//   SWA layer:  in-projection GEMV -> split attention over the window ring ->
//               o-projection (merging the split partials) -> FFN
//   shared KV:  projection GEMV -> K/V/indexer-key append + indexer scores with a
//               2048-bin histogram -> threshold bin + compaction -> exact
//               selection (one CTA per query row, beside the first q GEMV)
//   cross layer: q|gate GEMV -> selected-key attention -> o-projection -> FFN
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
constexpr int kMarkBase = 256;                   // trace entries kMarkBase + 4 p + i: sub-phase marks of CTA 0
constexpr int kSmem = 2 * kSlot + kWork;
constexpr int kMaxSort = 4096;
constexpr int kMkBitmapWords = 4096;  // selection bitmap: up to 131072 keys
constexpr int kMaxPhases = 4 * CB_MAX_SELF + 4 * CB_MAX_CROSS + 8;
constexpr unsigned kAbortBit = 1u << 30;
constexpr float kFix = 4294967296.0f;              // 2^32
constexpr float kFixInv = 2.3283064365386963e-10f;  // 2^-32

enum { PRE_NONE_ = 0, PRE_RMS_ = 1, PRE_EMBED_ = 2, PRE_COMBINE_ = 3 };
enum { EPI_STORE_ = 0, EPI_RED_ = 1 };
enum : int {
  PH_GDN = 0, PH_FFN_SELF, PH_SWA_IN, PH_SWA_ATT, PH_SWA_O, PH_SH_PROJ, PH_SH_SCORE, PH_SH_COMPACT, PH_CR_Q,
  PH_CR_ATT, PH_CR_O, PH_FFN_CROSS, PH_LM_HEAD
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

// %globaltimer at a point inside the current phase (CTA 0 only; i < 4).
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
__device__ __forceinline__ void grid_arrive(const MkArgs& a, unsigned& gen) {
  __syncthreads();
  gen += 1;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0 && 2 * gen < (unsigned)kMkTrace) a.trace[2 * gen - 1] = gtimer();
    __threadfence();
    // the test hook leaves this barrier one arrival short, so every wait on it runs out
    if (!(blockIdx.x == 0 && gen == s_stall_barrier)) atomicAdd(a.sync, 1u);
  }
}

__device__ __forceinline__ bool grid_wait(const MkArgs& a, unsigned gen, int* s_ok) {
  if (threadIdx.x == 0) {
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

// ------------------------------------------------------------------ fixed point
__device__ __forceinline__ float from_fix(long long q) { return __ll2float_rn(q) * kFixInv; }
__device__ __forceinline__ void red_fix(long long* p, float v) {
  const unsigned long long q = (unsigned long long)__float2ll_rn(v * kFix);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(q) : "memory");
}

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
__device__ __forceinline__ void tile_row(const uint8_t* tile, int K, int w, bool valid, bool global, RowW<NU>& r) {
  const int lane = threadIdx.x & 31, kc = K >> 3;
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(tile + w * (K / 2));
  const uint8_t* sb = tile + kTileRows * (K / 2) + w * (K / 16);
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
        const float4 x0 = *reinterpret_cast<const float4*>(xs + m * K + c * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + m * K + c * 8 + 4);
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
// warp-reduced sum on every lane.
template <int M>
__device__ __forceinline__ void row_dot(const uint8_t* tile, int K, int w, bool valid, bool global, const float* xs,
                                        float (&acc)[M]) {
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.0f;
  if (K <= 768) {
    RowW<3> r;
    tile_row<3>(tile, K, w, valid, global, r);
    dot_row<M, 3>(r, K, xs, acc);
  } else {
    RowW<8> r;
    tile_row<8>(tile, K, w, valid, global, r);
    dot_row<M, 8>(r, K, xs, acc);
  }
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = warp_sum(acc[m]);
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, int idx) {
  return ((unsigned long long)score_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}

// ------------------------------------------------------------------ RMSNorm staging
// xs[m][k] = x[m][k] * norm_w[k] for m < m_rows (zeros above); rn[m] receives
// the RMSNorm factor of each row (1 when norm_w is null).  x comes from a
// fixed-point residual row (xq, row rowmap[m]), float rows (x) or the token
// embeddings (embed_from).  The sums of squares are reduced in a fixed order.
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
    xs[i] = v;
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
  int xmap_nq, xmap_T, xmap_off;  // input row of m = (m / nq) * T + off + m % nq when xmap_nq > 0
  int pre;
  const float* norm_w;
  float* y;             // EPI_STORE_
  long long* yq;        // EPI_RED_: y is added to this fixed-point stream
  int ldy, rows_out, epi;
  long long* copy_q;    // the first CTA of the phase copies the (mapped) fixed-point input rows here
  bool argmax;
  // PRE_COMBINE_: the input is the gated merge of split-softmax attention
  // partials, part[((m * H + h) * S + s) * (hd + 2)] = (max, sum, o[hd]), with
  // the output gate sigmoid(gate_x[m * gate_ld + gate_off + h])
  const float* part;
  int S, hd;
  const float* gate_x;
  int gate_ld, gate_off;
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

__device__ __forceinline__ float* par_norm(float* work) { return work + kPreOff / 4 + kParNorm; }
__device__ __forceinline__ float* par_small(float* work) { return work + kPreOff / 4 + kParSmall; }

template <int M>
__device__ void gemv_phase(const MkArgs& a, const GemvJob& g, int m_rows, const uint8_t* slot, float* work) {
  const int n_mine = gemv_mine(g);
  if (n_mine == 0) return;
  const float* ps = par_small(work);
  const int K = g.W.k, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tb = tile_bytes(K);
  const int nst = gemv_staged(g);
  float* xs = work;  // [M][K]
  __shared__ unsigned long long s_best[kMkMaxRows];
  __shared__ int s_rowmap[kMkMaxRows];
  if (g.argmax && tid < kMkMaxRows) s_best[tid] = 0ull;
  if (tid < kMkMaxRows)
    s_rowmap[tid] = g.xmap_nq > 0 ? (tid / g.xmap_nq) * g.xmap_T + g.xmap_off + tid % g.xmap_nq : tid;
  __syncthreads();
  float rn[M];
  if (g.pre == PRE_COMBINE_) {
    // Merge the S <= 32 split partials of every (row, head): a warp per pair,
    // a lane per split: w_s = exp(m_s - max m), coef_s = w_s * gate / sum_s w_s l_s;
    // then x = sum_s coef_s o_s with the loads of 8 splits in flight at a time.
    const int hd = g.hd, H = K / hd, S = g.S, per = hd + 2;
    float* coef = work + M * K;  // [M][H][32]
    for (int i = warp; i < m_rows * H; i += kW) {
      const int mr = i / H, h = i - mr * H;
      const float* pb = g.part + (int64_t)i * S * per + lane * per;
      const float ms = lane < S ? __ldcg(pb) : -INFINITY;
      const float ls = lane < S ? __ldcg(pb + 1) : 0.0f;
      const float gt = __ldcg(g.gate_x + (int64_t)mr * g.gate_ld + g.gate_off + h);
      const float mx = warp_max(ms);
      const float w = ms == -INFINITY ? 0.0f : expf(ms - mx);
      const float L = warp_sum(w * ls);
      coef[i * 32 + lane] = w * (sigmoid(gt) / L);
    }
    __syncthreads();
    for (int i = tid; i < M * K; i += kT) {
      const int mr = i / K, k = i - mr * K;
      float v = 0.0f;
      if (mr < m_rows) {
        const int h = k / hd, dd = k - h * hd;
        const float* pb = g.part + (int64_t)(mr * H + h) * S * per + 2 + dd;
        const float* cf = coef + (mr * H + h) * 32;
        for (int s0 = 0; s0 < S; s0 += 8) {
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = s0 + e < S ? __ldcg(pb + (s0 + e) * per) : 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) v = fmaf(cf[s0 + e], o[e], v);
        }
      }
      xs[i] = v;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < M; ++m) rn[m] = 1.0f;
  } else {
    const bool first = g.ucta == 0;
    stage_rows<M>(g.xq, g.x, g.ldx, s_rowmap, m_rows, K, g.pre == PRE_NONE_ ? nullptr : par_norm(work), a.m.norm_eps,
                  xs, rn, first ? g.copy_q : nullptr, (g.pre == PRE_EMBED_ && first) ? a.hq : nullptr,
                  g.pre == PRE_EMBED_ ? &a : nullptr);
  }
  mark(a, 0);

  unsigned long long best[M];
#pragma unroll
  for (int mr = 0; mr < M; ++mr) best[mr] = 0ull;
  for (int i = 0; i < n_mine; i += 2) {
    const int ua = g.ucta + i * g.uncta, ub = ua + g.uncta;
    const bool hb = i + 1 < n_mine;
    const int ra = ua * kTileRows + warp, rb = ub * kTileRows + warp;
    const bool ga = i >= nst, gb = i + 1 >= nst;
    const uint8_t* ta = ga ? g.W.tiles + ua * tb : slot + i * tb;
    const uint8_t* tbb = gb ? g.W.tiles + ub * tb : slot + (i + 1) * tb;
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
  float *hp, *ssq, *red, *xs, *qk, *vv, *og, *rs, *pv, *gb, *pconv_w, *pconv_s;
};
__device__ __forceinline__ int pad4(int n) { return (n + 3) & ~3; }  // floats to a 16-byte multiple

template <int M>
__device__ __forceinline__ GdnSmem gdn_smem(float* work, const GdnGeo& g) {
  GdnSmem s;  // every array starts on a 16-byte boundary (xs is read as float4)
  s.xs = work;                          // [M][d]
  s.hp = s.xs + pad4(M * g.d);          // [M][HP]
  s.ssq = s.hp + pad4(M * g.HP);        // [kCl][M]
  s.red = s.ssq + pad4(kCl * M);        // [kCl][M][RC]
  s.qk = s.red + pad4(kCl * M * g.RC);  // [M][2 Dk]
  s.vv = s.qk + pad4(M * 2 * g.Dk);     // [M][vpr]
  s.og = s.vv + pad4(M * g.vpr);        // [M][vpr]
  s.rs = s.og + pad4(M * g.vpr);        // [kT] reduction scratch
  s.pv = s.rs + kT;                     // [kW]
  s.gb = s.pv + kW;                     // [M][2] decay log, beta
  s.pconv_w = work + kPreOff / 4 + kParConv;  // [NC][4] conv taps (parameter region)
  s.pconv_s = s.pconv_w + g.NC * 4;     // [B][3][NC] conv window
  return s;
}

// Before the barrier: this rank's state columns into registers and its conv
// taps / conv window into the preload region (they do not depend on the step).
template <int M>
__device__ __forceinline__ void gdn_preload(const MkArgs& a, const CbSelfLayer& L, int h, int rank, float (&st)[M],
                            float* work) {
  const CbModel& m = a.m;
  const GdnGeo g = gdn_geo(m, rank);
  const GdnSmem s = gdn_smem<M>(work, g);
  const int tid = threadIdx.x, C = 2 * g.H * g.Dk + g.H * g.Dv;
  const bool holds = tid < g.Dk * g.vpr;
  const int k = tid / g.vpr, v = tid - k * g.vpr;
#pragma unroll
  for (int b = 0; b < M; ++b) {
    st[b] = 0.0f;
    if (b < a.B && holds) {
      const int64_t slot = (int64_t)b * a.c.n_gdn + L.slot;
      st[b] = __ldcg(a.c.gdn_state + ((slot * g.H + h) * g.Dk + k) * g.Dv + g.v0 + v);
    }
  }
  // norm vector, tile scales of this rank's tiles, gate constants, tensor scale, o_norm columns
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
  cluster_sync();  // every rank's in-projection rows are in every rank's hp
  mark(a, 1);
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
__device__ __forceinline__ int ffn_mine(int F, int cta, int ncta) {
  const int nsl = F / kTileRows;
  return cta < nsl ? (nsl - 1 - cta) / ncta + 1 : 0;
}
__device__ __forceinline__ int ffn_staged(const CbMatrix& GU, const CbSliced& D, int F, int cta, int ncta) {
  const int64_t per = 2 * tile_bytes(GU.k) + slice_bytes(D);
  return min(ffn_mine(F, cta, ncta), (int)(kSlot / per));
}

template <typename F>
__device__ __forceinline__ int ffn_chunks(const CbMatrix& GU, const CbSliced& D, int Fh, int cta, int ncta, F&& f) {
  const int64_t tb = tile_bytes(GU.k), dsb = slice_bytes(D);
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
  return n;
}

template <int M>
__device__ void ffn_phase(const MkArgs& a, const CbMatrix& GU, const CbSliced& D, const float* norm2, long long* resid,
                          int Mr, bool live, int rank, int cid, const uint8_t* slot, float* work) {
  const CbModel& m = a.m;
  const int d = m.d_model, Fh = m.ffn_hidden, RC = d / kCl, K = GU.k;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x, ncta = gridDim.x;
  float* red = work;                   // [kCl][M][RC]  (written by the cluster's CTAs)
  float* xs = red + kCl * M * RC;      // [M][d]
  float* act = xs + M * d;             // [M][16]
  constexpr int kNE = (kMkMaxD + kT - 1) / kT;  // outputs per thread
  float acc[kNE][M];
#pragma unroll
  for (int e = 0; e < kNE; ++e)
#pragma unroll
    for (int mr = 0; mr < M; ++mr) acc[e][mr] = 0.0f;
  const int n_mine = ffn_mine(Fh, cta, ncta);
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
#pragma unroll
      for (int e = 0; e < kNE; ++e) {
        const int n = tid + e * kT;
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
    }
  }
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
  mark(a, 1);
  cluster_sync();
  mark(a, 2);
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

// ------------------------------------------- attention helpers (split softmax)
// Scores of nq queries (Qs [nq][hd]) against n keys (Ks [n][hd+1]) into Sc [nq][ldsc],
// masked entries -inf; then per query max / exp / sum (qm, ql) and o += e V into oacc.
__device__ void attend_chunk(const float* Qs, const float* Ks, const float* Vs, float* Sc, int ldsc, int nq, int n,
                             int hd, float scale, float* qm, float* ql, float* corr, float* oacc,
                             const int* key_pos, const int* q_pos, int window) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < nq * n; i += kT) {
    const int q = i / n, key = i - q * n;
    bool ok = true;
    if (window > 0) {
      const int kp = key_pos[key], pt = q_pos[q];
      ok = kp <= pt && kp > pt - window;
    }
    float sc = -INFINITY;
    if (ok) {  // four independent chains over d (hd % 8 == 0), summed in a fixed order
      const float* qq = Qs + q * hd;
      const float* kk = Ks + key * (hd + 1);
      float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 2
      for (int dd = 0; dd < hd; dd += 4) {
        a0 = fmaf(qq[dd], kk[dd], a0);
        a1 = fmaf(qq[dd + 1], kk[dd + 1], a1);
        a2 = fmaf(qq[dd + 2], kk[dd + 2], a2);
        a3 = fmaf(qq[dd + 3], kk[dd + 3], a3);
      }
      sc = ((a0 + a1) + (a2 + a3)) * scale;
    }
    Sc[q * ldsc + key] = sc;
  }
  __syncthreads();
  for (int q = warp; q < nq; q += kW) {
    float mx = -INFINITY;
    for (int key = lane; key < n; key += 32) mx = fmaxf(mx, Sc[q * ldsc + key]);
    mx = warp_max(mx);
    const float mnew = fmaxf(qm[q], mx);
    float l = 0.0f;
    for (int key = lane; key < n; key += 32) {
      const float sc = Sc[q * ldsc + key];
      const float e = sc == -INFINITY ? 0.0f : expf(sc - mnew);
      Sc[q * ldsc + key] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      const float cr = qm[q] == -INFINITY ? 0.0f : expf(qm[q] - mnew);
      corr[q] = cr;
      ql[q] = ql[q] * cr + l;
      qm[q] = mnew;
    }
  }
  __syncthreads();
  for (int i = tid; i < nq * hd; i += kT) {
    const int q = i / hd, dd = i - q * hd;
    const float* e = Sc + q * ldsc;
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;  // keys mod 4, summed in a fixed order
    int key = 0;
#pragma unroll 2
    for (; key + 4 <= n; key += 4) {
      o0 = fmaf(e[key], Vs[key * hd + dd], o0);
      o1 = fmaf(e[key + 1], Vs[(key + 1) * hd + dd], o1);
      o2 = fmaf(e[key + 2], Vs[(key + 2) * hd + dd], o2);
      o3 = fmaf(e[key + 3], Vs[(key + 3) * hd + dd], o3);
    }
    for (; key < n; ++key) o0 = fmaf(e[key], Vs[key * hd + dd], o0);
    oacc[i] = fmaf(oacc[i], corr[q], (o0 + o1) + (o2 + o3));
  }
  __syncthreads();
}

// ------------------------------------------------------------------- SWA
__device__ void swa_item(const MkArgs& a, const CbSelfLayer& L, int b, int g, int s, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int hd = m.head_dim, Hq = m.n_q_heads, Hkv = m.n_kv_heads, G = Hq / Hkv, T = a.T;
  const int W = m.swa_window, Ls = kMkSwaSplit, S = a.swa_splits, nqry = G * T;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int p0 = c.pos[b] + a.c0;
  const int lo = max(0, p0 - W + 1), last = p0 + T - 1;
  const int ks = lo + s * Ls, ke = min(ks + Ls, last + 1), n = max(0, ke - ks);
  float* Ks = smem;                    // [Ls][hd + 1]
  float* Vs = Ks + Ls * (hd + 1);      // [Ls][hd]
  float* Qs = Vs + Ls * hd;            // [kMkMaxQ][hd]
  float* Sc = Qs + kMkMaxQ * hd;       // [kMkMaxQ][Ls]
  float* oacc = Sc + kMkMaxQ * Ls;     // [kMkMaxQ][hd]
  __shared__ float qm[kMkMaxQ], ql[kMkMaxQ], corr[kMkMaxQ];
  __shared__ int kpos[kMkSwaSplit], qpos[kMkMaxQ];
  const int64_t ring = (int64_t)(b * c.n_swa + L.slot) * c.swa_slots * Hkv * hd;
  uint16_t* kr = c.swa_k + ring;
  uint16_t* vr = c.swa_v + ring;

  uint16_t* raw = reinterpret_cast<uint16_t*>(oacc + kMkMaxQ * hd);  // [2][Ls][hd] bf16 ring rows
  const int vpk = hd / 8;  // 16-byte vectors per key row
  // the window's ring rows do not depend on this step: start their copies first
  for (int i = tid; i < n * vpk; i += kT) {
    const int key = i / vpk, e8 = (i - key * vpk) * 8, kp = ks + key;
    if (kp < p0) {
      const int64_t off = ((int64_t)(kp % c.swa_slots) * Hkv + g) * hd + e8;
      cp_async16(raw + key * hd + e8, kr + off);
      cp_async16(raw + (Ls + key) * hd + e8, vr + off);
    }
  }
  for (int q = warp; q < nqry; q += kW) {
    const int t = q / G, j = q - t * G;
    norm_rope_warp(a.proj + ((int64_t)b * T + t) * a.ldp + (g * G + j) * hd, L.q_norm, hd, m.rot_dim / 2, p0 + t,
                   m.inv_freq, m.norm_eps, Qs + q * hd, false, nullptr);
  }
  // keys of this chunk's own tokens come from the projection (and are appended
  // to the ring here), on the warps after the query ones
  const int new0 = max(ks, p0), wk = (warp + kW - nqry % kW) % kW;
  for (int kp = new0 + wk; kp < ke; kp += kW) {
    const int idx = kp - ks, t2 = kp - p0;
    const float* row = a.proj + ((int64_t)b * T + t2) * a.ldp;
    const int64_t off = ((int64_t)(kp % c.swa_slots) * Hkv + g) * hd;
    norm_rope_warp(row + m.swa_off_kv + g * hd, L.k_norm, hd, m.rot_dim / 2, kp, m.inv_freq, m.norm_eps,
                   Ks + idx * (hd + 1), true, kr + off);
    const int lane = tid & 31;
    for (int dd = lane; dd < hd; dd += 32) {
      const uint16_t bits = f32_to_bf16(__ldcg(row + m.swa_off_kv + Hkv * hd + g * hd + dd));
      vr[off + dd] = bits;
      Vs[idx * hd + dd] = bf16_to_f32(bits);
    }
  }
  cp_async_wait_all();
  __syncthreads();
#pragma unroll 2
  for (int i = tid; i < n * vpk; i += kT) {
    const int key = i / vpk, e8 = (i - key * vpk) * 8, kp = ks + key;
    if (kp < p0) {
      const uint4 kq = *reinterpret_cast<const uint4*>(raw + key * hd + e8);
      const uint4 vq = *reinterpret_cast<const uint4*>(raw + (Ls + key) * hd + e8);
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, vw[4] = {vq.x, vq.y, vq.z, vq.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        Ks[key * (hd + 1) + e8 + 2 * e] = bf16_to_f32(kw[e]);
        Ks[key * (hd + 1) + e8 + 2 * e + 1] = bf16_to_f32(kw[e] >> 16);
        Vs[key * hd + e8 + 2 * e] = bf16_to_f32(vw[e]);
        Vs[key * hd + e8 + 2 * e + 1] = bf16_to_f32(vw[e] >> 16);
      }
    }
  }
  for (int i = tid; i < n; i += kT) kpos[i] = ks + i;
  for (int i = tid; i < nqry; i += kT) {
    qpos[i] = p0 + i / G;
    qm[i] = -INFINITY;
    ql[i] = 0.0f;
  }
  for (int i = tid; i < nqry * hd; i += kT) oacc[i] = 0.0f;
  __syncthreads();
  if (n > 0) attend_chunk(Qs, Ks, Vs, Sc, Ls, nqry, n, hd, rsqrtf((float)hd), qm, ql, corr, oacc, kpos, qpos, W);
  for (int i = tid; i < nqry * (hd + 2); i += kT) {
    const int q = i / (hd + 2), e = i - q * (hd + 2);
    const int t = q / G, j = q - t * G;
    float* pp = a.part + ((((int64_t)b * T + t) * Hq + g * G + j) * S + s) * (hd + 2);
    pp[e] = e == 0 ? qm[q] : (e == 1 ? ql[q] : oacc[q * hd + e - 2]);
  }
  __syncthreads();
  // the o projection merges the partials (PRE_COMBINE)
}

__device__ void swa_phase(const MkArgs& a, const CbSelfLayer& L, float* smem) {
  const int Hkv = a.m.n_kv_heads, S = a.swa_splits;
  for (int it = blockIdx.x; it < a.B * Hkv * S; it += gridDim.x) {
    const int s = it % S, g = (it / S) % Hkv, b = it / (S * Hkv);
    swa_item(a, L, b, g, s, smem);
  }
}

// -------------------------------------------------------- cross attention
__device__ void cross_item(const MkArgs& a, const CbCrossLayer& L, int r, int g, int s, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int hd = m.head_dim, Hq = m.n_q_heads, Hkv = m.n_kv_heads, G = Hq / Hkv, S = a.cross_splits;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = r / a.nq, jr = r - b * a.nq;
  const int position = c.pos[b] + a.c0 + (a.T - a.nq) + jr;
  const bool dense = m.sparse_topk == 0;
  const int n_all = dense ? max(0, min(position + 1, c.max_ctx)) : min(__ldcg(a.sel_cnt + r), a.sel_ld);
  const int per = dense ? ceil_div(n_all, S) : kMkCrossSplit;
  const int ks = s * per, ke = min(ks + per, n_all);
  const int Lc = kMkSwaSplit;  // keys per sub-chunk
  float* Ks = smem;                 // [Lc][hd + 1]
  float* Vs = Ks + Lc * (hd + 1);   // [Lc][hd]
  float* Qs = Vs + Lc * hd;         // [G][hd]
  float* Sc = Qs + kMkMaxQ * hd;    // [G][Lc]
  float* oacc = Sc + kMkMaxQ * Lc;  // [G][hd]
  __shared__ float qm[kMkMaxQ], ql[kMkMaxQ], corr[kMkMaxQ];
  __shared__ int kid[kMkSwaSplit];
  const float* row = a.cproj + (int64_t)r * a.cr_ld;
  for (int j = warp; j < G; j += kW)
    norm_rope_warp(row + (g * G + j) * hd, L.q_norm, hd, m.rot_dim / 2, position, m.inv_freq, m.norm_eps, Qs + j * hd,
                   false, nullptr);
  for (int i = tid; i < G; i += kT) {
    qm[i] = -INFINITY;
    ql[i] = 0.0f;
  }
  for (int i = tid; i < G * hd; i += kT) oacc[i] = 0.0f;
  const uint16_t* kb = c.kv_k + (int64_t)b * c.max_ctx * Hkv * hd;
  const uint16_t* vb = c.kv_v + (int64_t)b * c.max_ctx * Hkv * hd;
  for (int c0 = ks; c0 < ke; c0 += Lc) {
    const int cn = min(Lc, ke - c0);
    // (the previous chunk's attend_chunk ended with a barrier; kid is free)
    // on the warps after the query ones, so the first chunk's ids load beside the q RoPE
    for (int i = (tid + kT - 32 * (G % kW)) % kT; i < cn; i += kT)
      kid[i] = dense ? c0 + i : __ldcg(a.sel_idx + (int64_t)r * a.sel_ld + c0 + i);
    __syncthreads();
    const int vpk = hd / 8;
#pragma unroll 4
    for (int i = tid; i < cn * vpk; i += kT) {
      const int key = i / vpk, e8 = (i - key * vpk) * 8;
      const int64_t off = ((int64_t)kid[key] * Hkv + g) * hd + e8;
      const uint4 kq = __ldcg(reinterpret_cast<const uint4*>(kb + off));
      const uint4 vq = __ldcg(reinterpret_cast<const uint4*>(vb + off));
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, vw[4] = {vq.x, vq.y, vq.z, vq.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        Ks[key * (hd + 1) + e8 + 2 * e] = bf16_to_f32(kw[e]);
        Ks[key * (hd + 1) + e8 + 2 * e + 1] = bf16_to_f32(kw[e] >> 16);
        Vs[key * hd + e8 + 2 * e] = bf16_to_f32(vw[e]);
        Vs[key * hd + e8 + 2 * e + 1] = bf16_to_f32(vw[e] >> 16);
      }
    }
    __syncthreads();
    attend_chunk(Qs, Ks, Vs, Sc, Lc, G, cn, hd, rsqrtf((float)hd), qm, ql, corr, oacc, nullptr, nullptr, 0);
  }
  __syncthreads();
  for (int i = tid; i < G * (hd + 2); i += kT) {
    const int j = i / (hd + 2), e = i - j * (hd + 2);
    float* pp = a.part2 + (((int64_t)r * Hq + g * G + j) * S + s) * (hd + 2);
    pp[e] = e == 0 ? qm[j] : (e == 1 ? ql[j] : oacc[j * hd + e - 2]);
  }
  __syncthreads();
  // the o projection merges the partials (PRE_COMBINE)
}

__device__ void cross_phase(const MkArgs& a, const CbCrossLayer& L, float* smem) {
  const int Hkv = a.m.n_kv_heads, S = a.cross_splits, RQ = a.B * a.nq;
  for (int it = blockIdx.x; it < RQ * Hkv * S; it += gridDim.x) {
    const int s = it % S, g = (it / S) % Hkv, r = it / (S * Hkv);
    cross_item(a, L, r, g, s, smem);
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

// Scores of this CTA's key range for every query row + histogram of the top 11 key bits.
__device__ void score_phase(const MkArgs& a, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int RQ = a.B * a.nq, Hi = m.indexer_heads, Di = m.indexer_dim, k = m.sparse_topk;
  const int tid = threadIdx.x, cta = blockIdx.x, ncta = gridDim.x;
  unsigned* hist = reinterpret_cast<unsigned*>(smem);             // [2048]
  float* q = smem + kMkHistBins;                                   // [Hi*Di]
  float* w = q + Hi * Di;                                          // [Hi]
  uint8_t* newk = reinterpret_cast<uint8_t*>(w + 16);              // [8][Di] keys of this chunk's tokens
  for (int r = 0; r < RQ; ++r) {
    int b, t, p, n;
    query_row(a, r, b, t, p, n);
    if (n <= k) continue;
    int js, je;
    key_range(n, cta, ncta, js, je);
    if (js >= je) continue;
    const float* qrow = a.proj + ((int64_t)b * a.T + t) * a.ldp;
    const int p0 = c.pos[b] + a.c0;
    for (int i = tid; i < Hi * Di; i += kT) q[i] = __ldcg(qrow + m.sh_off_iq + i);
    for (int i = tid; i < Hi; i += kT) w[i] = __ldcg(qrow + m.sh_off_iw + i);
    for (int i = tid; i < a.T * Di; i += kT) {
      const int t2 = i / Di, dd = i - t2 * Di;
      newk[i] = f32_to_e4m3(__ldcg(a.proj + ((int64_t)b * a.T + t2) * a.ldp + m.sh_off_ik + dd));
    }
    for (int i = tid; i < kMkHistBins; i += kT) hist[i] = 0u;
    __syncthreads();
    const uint8_t* ikb = c.kv_ik + (int64_t)b * c.max_ctx * Di;
    float* out = a.scores + (int64_t)r * c.max_ctx;
    for (int j = js + tid; j < je; j += kT) {
      const uint8_t* kr = j < p0 ? ikb + (int64_t)j * Di : newk + (j - p0) * Di;
      const float sc = indexer_score_bytes(kr, q, w, Hi, Di);
      out[j] = sc;
      atomicAdd(&hist[score_key(sc) >> 21], 1u);
    }
    __syncthreads();
    for (int i = tid; i < kMkHistBins; i += kT)
      if (hist[i]) atomicAdd(&a.hist[(int64_t)r * kMkHistBins + i], hist[i]);
    __syncthreads();
  }
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
  __shared__ int s_digit, s_rem;
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
#pragma unroll 2
  for (int i = tid; i < above; i += kT) {
    const int j = __ldcg(a.hi_list + (int64_t)r * k + i);
    if (j >= 0 && j < n) atomicOr(&bits[j >> 5], 1u << (j & 31));
  }
  unsigned long long prefix = 0ull, pmask = 0ull;
  int remaining = need;
#pragma unroll 1
  for (int ps = 0; ps < 7; ++ps) {  // digits of 8 bits from bit 45 down, then the low 5 bits
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
    __syncthreads();
  }
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

// ------------------------------------------------------------------ phase plan
__device__ int build_plan(const CbModel& m, uint16_t* plan) {
  int n = 0;
  auto push = [&](int kind, int layer) { plan[n++] = (uint16_t)((kind << 8) | layer); };
  for (int i = 0; i < m.n_self_layers; ++i) {
    if (m.self_layers[i].kind == CB_LAYER_GDN) {
      push(PH_GDN, i);
    } else {
      push(PH_SWA_IN, i);
      push(PH_SWA_ATT, i);
      push(PH_SWA_O, i);
    }
    push(PH_FFN_SELF, i);
  }
  push(PH_SH_PROJ, 0);
  push(PH_SH_SCORE, 0);
  if (m.sparse_topk > 0) push(PH_SH_COMPACT, 0);
  for (int j = 0; j < m.n_cross_layers; ++j) {
    push(PH_CR_Q, j);
    push(PH_CR_ATT, j);
    push(PH_CR_O, j);
    push(PH_FFN_CROSS, j);
  }
  push(PH_LM_HEAD, 0);
  return n;
}

// The GEMV of a GEMV phase (input, output, this CTA's units).
__device__ GemvJob gemv_job(const MkArgs& a, int kind, int layer) {
  const CbModel& m = a.m;
  const int d = m.d_model, RQ = a.B * a.nq;
  GemvJob g{};
  g.ucta = blockIdx.x;
  g.uncta = gridDim.x;
  g.ldx = d;
  g.epi = EPI_STORE_;
  switch (kind) {
    case PH_SWA_IN: {
      const CbSelfLayer& L = m.self_layers[layer];
      g.W = L.in_proj;
      g.xq = a.hq;
      g.pre = layer == 0 ? PRE_EMBED_ : PRE_RMS_;
      g.norm_w = L.norm1;
      g.y = a.proj;
      g.ldy = a.ldp;
      g.rows_out = L.in_proj.rows;
      break;
    }
    case PH_SWA_O: {
      const CbSelfLayer& L = m.self_layers[layer];
      g.W = L.o_proj;
      g.pre = PRE_COMBINE_;
      g.part = a.part;
      g.S = a.swa_splits;
      g.hd = m.head_dim;
      g.gate_x = a.proj;
      g.gate_ld = a.ldp;
      g.gate_off = m.swa_off_gate;
      g.yq = a.hq;
      g.ldy = d;
      g.rows_out = d;
      g.epi = EPI_RED_;
      break;
    }
    case PH_SH_PROJ:
      g.W = m.shared_proj;
      g.xq = a.hq;
      g.pre = PRE_RMS_;
      g.norm_w = m.shared_norm;
      g.y = a.proj;
      g.ldy = a.ldp;
      g.rows_out = m.shared_proj.rows;
      break;
    case PH_CR_Q: {
      const CbCrossLayer& L = m.cross_layers[layer];
      g.W = L.q_gate;
      g.xq = layer == 0 ? a.hq : a.xq;
      if (layer == 0) {  // the query rows of the self-decoder's output start the cross residual stream
        g.xmap_nq = a.nq;
        g.xmap_T = a.T;
        g.xmap_off = a.T - a.nq;
        g.copy_q = a.xq;
        if (m.sparse_topk > 0) {  // the first RQ CTAs resolve the selections beside this GEMV
          g.ucta = (int)blockIdx.x - RQ;
          g.uncta = (int)gridDim.x - RQ;
        }
      }
      g.pre = PRE_RMS_;
      g.norm_w = L.norm1;
      g.y = a.cproj;
      g.ldy = a.cr_ld;
      g.rows_out = L.q_gate.rows;
      break;
    }
    case PH_CR_O: {
      const CbCrossLayer& L = m.cross_layers[layer];
      g.W = L.o_proj;
      g.pre = PRE_COMBINE_;
      g.part = a.part2;
      g.S = a.cross_splits;
      g.hd = m.head_dim;
      g.gate_x = a.cproj;
      g.gate_ld = a.cr_ld;
      g.gate_off = m.cr_off_gate;
      g.yq = a.xq;
      g.ldy = d;
      g.rows_out = d;
      g.epi = EPI_RED_;
      break;
    }
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
  return kind == PH_SWA_IN || kind == PH_SWA_O || kind == PH_SH_PROJ || kind == PH_CR_Q || kind == PH_CR_O ||
         kind == PH_LM_HEAD;
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
  return 0;
}

// Between the arrival at the barrier before a GEMV or FFN phase and the wait
// there: the phase's norm vector, tile scales and tensor scale into the
// parameter region (cp.async; completed after the wait).  The GDN phase has
// its own (gdn_preload).
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
    const int n = min(ffn_mine(m.ffn_hidden, blockIdx.x, gridDim.x), 16);
    if (n == 0) return;
    for (int i = tid; i < m.d_model / 4; i += kT) cp_async16(pn + 4 * i, norm2 + 4 * i);
    for (int i = tid; i < n; i += kT) {
      const int j = blockIdx.x + i * gridDim.x;
      cp_async4(ps + i, GU.tile_scale + j);
      cp_async4(ps + 16 + i, GU.tile_scale + m.ffn_hidden / kTileRows + j);
    }
    if (tid == 0) cp_async4(ps + PS_TSCALE, D.tensor_scale);
  }
}

// Warp 0: arm the slot's mbarrier with the phase's byte count and start its copies.
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
    if (cta == 0) a.trace[0] = gtimer();
  }
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
  if (warp == 0) stage_issue(a, s_plan[0] >> 8, s_plan[0] & 0xFF, smem, &s_bar[0]);
  issued0 = 1;
  grid_arrive(a, gen);
  bool live = true;

  for (int p = 0; p < P; ++p) {
    const int kind = s_plan[p] >> 8, layer = s_plan[p] & 0xFF, sl = p & 1;
    if (live && p + 1 < P) {  // the next phase's weights, into the other slot
      if (warp == 0) stage_issue(a, s_plan[p + 1] >> 8, s_plan[p + 1] & 0xFF, smem + (sl ^ 1) * kSlot, &s_bar[sl ^ 1]);
      if (sl) issued0 += 1;
      else issued1 += 1;
    }
    float st[M];  // the recurrent state of this thread's GDN columns, one value per sequence
    const bool gdn_here = kind == PH_GDN && cid < m.gdn_heads;
    if (tid == 0) s_mark_base = kMarkBase + 4 * p;
    if (live) {
      if (gdn_here) gdn_preload<M>(a, m.self_layers[layer], cid, rank, st, work);
      else phase_params(a, kind, layer, work);
    }
    live = grid_wait(a, gen, &s_ok) && live;
    cp_async_wait_all();  // this phase's parameters
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
      case PH_SWA_ATT:
        if (live) swa_phase(a, m.self_layers[layer], work);
        break;
      case PH_SH_SCORE:
        if (live) {
          shared_append(a, work);
          if (m.sparse_topk > 0) score_phase(a, work);
        }
        break;
      case PH_SH_COMPACT:
        if (live) compact_phase(a);
        break;
      case PH_CR_ATT:
        if (live) cross_phase(a, m.cross_layers[layer], work);
        break;
      default: {  // GEMV phases
        if (!live) break;
        const GemvJob g = gemv_job(a, kind, layer);
        const int rows = (kind == PH_CR_Q || kind == PH_CR_O || kind == PH_LM_HEAD) ? RQ : Mrows;
        if (kind == PH_CR_Q && layer == 0 && m.sparse_topk > 0 && cta < RQ) resolve_row(a, cta, work);
        else gemv_phase<M>(a, g, rows, slot, work);
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
                            m.indexer_heads > 16 || (m.indexer_heads * m.indexer_dim + 16 + kMkHistBins) * 4 +
                            CB_MAX_T * m.indexer_dim > kWork))
    return false;
  const size_t att = sizeof(float) * ((size_t)kMkSwaSplit * (2 * m.head_dim + 1) + (size_t)kMkMaxQ * m.head_dim * 2 +
                                      (size_t)kMkMaxQ * kMkSwaSplit) +
                     sizeof(uint16_t) * 2 * kMkSwaSplit * m.head_dim;
  if (att > (size_t)kWork) return false;
  if (mk_swa_splits(m) > 32) return false;
  if (m.sparse_topk > 0 && ceil_div(m.sparse_topk + 1, kMkCrossSplit) > 32) return false;
  // GEMV staging: [M][K] inputs (+ [M][H][32] split weights for the o projections)
  if ((size_t)kMkMaxRows * (kMkMaxD + m.n_q_heads * 32) * sizeof(float) > (size_t)kPreOff) return false;
  // FFN: [8][M][d/8] partials + [M][d] inputs + [M][16]
  if ((size_t)kMkMaxRows * (2 * d + 16) * sizeof(float) > (size_t)kPreOff) return false;
  const int64_t tb = tile_bytes(d);
  for (int i = 0; i < m.n_self_layers; ++i) {
    const CbSelfLayer& L = m.self_layers[i];
    if (L.in_proj.k != d || L.gate_up.k != d || L.o_proj.rows < d || L.down.rows < d) return false;
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
                                        (size_t)kMkMaxRows * 2 * d + (size_t)kMkMaxRows * (2 * Dk + 2 * vpr) +
                                        kT + kW + 2 * kMkMaxRows + 32);  // + 16-byte padding of each array
      const size_t pre = sizeof(float) * ((size_t)kParConv + (size_t)(2 * Dk + vpr) * (4 + 3 * c.batch));
      if (w > (size_t)kPreOff || pre > (size_t)(kWork - kPreOff) || vpr > 16) return false;
    }
  }
  for (int j = 0; j < m.n_cross_layers; ++j) {
    const CbCrossLayer& L = m.cross_layers[j];
    if (L.q_gate.k != d || L.gate_up.k != d) return false;
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
  // every GDN head needs a cluster, and the first cross layer needs CTAs beyond the query rows
  if (ncl < a.m.gdn_heads || ncl * kCl <= a.B * a.nq) return CB_ERR_SHAPE;
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
