// Persistent decode kernel: one cooperative launch runs a whole forward chunk
// of M = batch * T <= 8 rows (a tau=1 decode step, or a verify of 1 + draft
// tokens) with every CTA resident, walking the model layer by layer.
//
// Phases (each followed by a grid barrier):
//   self layer:  in-proj GEMV (norm1 fused; layer 0 gathers the embedding)
//                -> GDN heads | SWA (q/k norm + RoPE + ring append + split
//                   attention partials)
//                -> o-proj GEMV (+ residual; after SWA its input staging merges
//                   the split partials and applies the output gate)
//                -> gate_up GEMV producing silu(g)*u
//                -> down GEMV (+ residual)
//   shared KV:   projection GEMV -> K/V/indexer-key append + indexer scores with
//                a 2048-bin histogram of the score keys -> threshold bin and
//                compaction -> exact selection (one CTA per query row, run
//                alongside the first cross layer's q GEMV)
//   cross layer: q|gate GEMV -> selected-key attention (split partials)
//                -> o-proj (merging the partials) -> gate_up -> down
//   head:        LM-head GEMV (final norm fused) with a per-row argmax
// Each GEMV's first weight rows are copied to shared memory between the
// arrival at the barrier before it and the wait there; there is no separate
// L2 prefetch (measured: it costs more in issue and queueing than it saves).
// Every wait is bounded
// (%globaltimer); on timeout the launch sets CB_ERR_TIMEOUT and all CTAs exit.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "mk.cuh"
#include "nvfp4.cuh"

namespace cb {
namespace {

constexpr int kT = kMkThreads;
constexpr int kW = kMkThreads / 32;
constexpr int kSmem = 160 * 1024;
constexpr int kMaxSort = 4096;
constexpr int kMkBitmapWords = 4096;  // selection bitmap: up to 131072 keys

enum { PRE_NONE_ = 0, PRE_RMS_ = 1, PRE_EMBED_ = 2, PRE_COMBINE_ = 3 };
enum { EPI_STORE_ = 0, EPI_ADD_ = 1, EPI_ACT_ = 2 };

// ------------------------------------------------------------------ sync
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile_i32(const int32_t* p) { return *(volatile const int32_t*)p; }

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid barrier on a monotonic arrival counter, split in two: grid_arrive
// publishes this CTA's writes and counts it in; grid_wait waits for every CTA.
// Work that does not depend on the other CTAs' writes (the next phase's
// weight loads) goes between the two.  grid_wait returns false when the launch
// must stop (this CTA's wait timed out, or another CTA's did).
// Per-CTA copy of the launch's wait limit and stall hook (thread 0 reads them at start).
__shared__ unsigned long long s_wait_limit;
__shared__ unsigned s_stall_barrier;

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
    while (ld_acquire_u32(a.sync) < target) {
      if ((++spin & 127) == 0) {
        if (ld_volatile_i32(a.abort_flag)) {
          ok = 0;
          break;
        }
        if (gtimer() - t0 > s_wait_limit) {
          atomicExch(a.abort_flag, 1);
          atomicCAS(a.status, 0, CB_ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    if (blockIdx.x == 0 && 2 * gen < (unsigned)kMkTrace) a.trace[2 * gen] = gtimer();
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

__device__ __forceinline__ bool grid_sync(const MkArgs& a, unsigned& gen, int* s_ok) {
  grid_arrive(a, gen);
  return grid_wait(a, gen, s_ok);
}

// Asynchronous global -> shared copies (no registers held while they fly)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------------------------------ GEMV
struct GemvJob {
  CbMatrix W;
  const float* x;
  int ldx;
  int xmap_nq, xmap_T, xmap_off;  // x row of m = (m / nq) * T + off + m % nq when xmap_nq > 0
  int pre;
  const float* norm_w;
  float* y;
  int ldy, rows_out, epi;
  float* copy_x;                  // local CTA 0 stores the raw input rows here ([m][K])
  bool argmax;
  // PRE_COMBINE: the input is the gated merge of split-softmax attention
  // partials, part[((m * H + h) * S + s) * (hd + 2)] = (max, sum, o[hd]), with
  // the output gate sigmoid(gate_x[m * gate_ld + gate_off + h])
  const float* part;
  int S, hd;
  const float* gate_x;
  int gate_ld, gate_off;
};

// One weight row as seen by one lane: the 8-code chunks lane, lane+32, ...
// (K <= 2048, so at most 8 chunks), code words and scale bytes.
template <int NU>
struct RowW {
  uint32_t w[NU];
  uint32_t s[NU];
};

template <int NU>
__device__ __forceinline__ void load_row(const CbMatrix& W, int64_t tb, int K, int row, bool valid, RowW<NU>& r) {
  const int lane = threadIdx.x & 31, kc = K >> 3;
  const uint8_t* t = W.tiles + (int64_t)(row >> 4) * tb;
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(t + (row & 15) * (K / 2));
  const uint8_t* sb = t + kTileRows * (K / 2) + (row & 15) * (K / 16);
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int c = u * 32 + lane;
    const bool ok = valid && c < kc;
    r.w[u] = ok ? __ldg(cw + c) : 0u;
    r.s[u] = ok ? (uint32_t)__ldg(sb + (c >> 1)) : 0u;
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

__device__ __forceinline__ unsigned long long pack_argmax(float v, int idx) {
  return ((unsigned long long)score_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}

// Rows of unit u for this warp: ACT pairs gate row ra with up row rb; the
// other epilogues pair units u and u + ncta (rb valid when hb).
__device__ __forceinline__ void gemv_rows(const GemvJob& g, int units, int ncta, int u, int& ra, int& rb, bool& hb) {
  const int warp = threadIdx.x >> 5;
  if (g.epi == EPI_ACT_) {
    ra = u * kTileRows + warp;
    rb = g.W.rows / 2 + u * kTileRows + warp;
    hb = true;
  } else {
    const int ub = u + ncta;
    ra = u * kTileRows + warp;
    hb = ub < units;
    rb = ub * kTileRows + warp;
  }
}

__device__ __forceinline__ int gemv_units(const GemvJob& g) {
  return g.epi == EPI_ACT_ ? g.W.rows / 32 : g.W.rows / kTileRows;
}

// The first unit's weights and, for a residual add, the old outputs: they do
// not depend on the previous phase, so they are fetched between the arrival at
// its barrier and the wait there.  The weight rows go by asynchronous copies
// into a per-warp shared-memory slot at kPreOff (two rows of codes + scales),
// so no registers stay live across the barrier; the residuals are registers.
constexpr int kPreOff = 96 * 1024;
__host__ __device__ constexpr int pre_row_bytes(int K) { return ((9 * K / 16) + 15) & ~15; }
static_assert(kPreOff + kW * 2 * pre_row_bytes(2048) <= kSmem, "preload slots exceed the scratch");

template <int M>
struct GemvPre {
  float resa[M], resb[M];
};

// The copies move 16-byte code chunks and 4-byte scale chunks: K % 64 == 0.
// Other K load the first unit directly after the barrier.
__device__ __forceinline__ bool pre_staged(int K) { return K % 64 == 0; }

__device__ __forceinline__ uint8_t* pre_slot(float* smem, int K) {
  return reinterpret_cast<uint8_t*>(smem) + kPreOff + (threadIdx.x >> 5) * 2 * pre_row_bytes(K);
}

__device__ __forceinline__ void pre_copy_row(const CbMatrix& W, int K, int row, uint8_t* dst) {
  const int lane = threadIdx.x & 31;
  const uint8_t* t = W.tiles + (int64_t)(row >> 4) * tile_bytes(K);
  const uint8_t* codes = t + (row & 15) * (K / 2);
  const uint8_t* sc = t + kTileRows * (K / 2) + (row & 15) * (K / 16);
  for (int i = lane; i < K / 32; i += 32) cp_async16(dst + 16 * i, codes + 16 * i);
  for (int i = lane; i < K / 64; i += 32) cp_async4(dst + K / 2 + 4 * i, sc + 4 * i);
}

// The lane's view of a preloaded row (the layout load_row produces).
template <int NU>
__device__ __forceinline__ void pre_read_row(const uint8_t* src, int K, bool valid, RowW<NU>& r) {
  const int lane = threadIdx.x & 31, kc = K >> 3;
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(src);
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int c = u * 32 + lane;
    const bool ok = valid && c < kc;
    r.w[u] = ok ? cw[c] : 0u;
    r.s[u] = ok ? (uint32_t)src[K / 2 + (c >> 1)] : 0u;
  }
}

template <int M>
__device__ __forceinline__ void gemv_pre(const GemvJob& g, int m_rows, int cta, int ncta, float* smem,
                                         GemvPre<M>& p) {
  const int units = gemv_units(g);
  if (cta < 0 || cta >= units || ncta <= 0) return;
  const int K = g.W.k, lane = threadIdx.x & 31;
  int ra, rb;
  bool hb;
  gemv_rows(g, units, ncta, cta, ra, rb, hb);
  if (pre_staged(K)) {
    uint8_t* slot = pre_slot(smem, K);
    pre_copy_row(g.W, K, ra, slot);
    if (hb) pre_copy_row(g.W, K, rb, slot + pre_row_bytes(K));
  }
#pragma unroll
  for (int mr = 0; mr < M; ++mr) {
    p.resa[mr] = p.resb[mr] = 0.0f;
    if (g.epi == EPI_ADD_ && lane == 0 && mr < m_rows) {
      if (ra < g.rows_out) p.resa[mr] = __ldcg(g.y + (int64_t)mr * g.ldy + ra);
      if (hb && rb < g.rows_out) p.resb[mr] = __ldcg(g.y + (int64_t)mr * g.ldy + rb);
    }
  }
}

template <int M>
__device__ void gemv_phase(const MkArgs& a, const GemvJob& g, int m_rows, int cta, int ncta, float* smem,
                           GemvPre<M>& p) {
  const int units = gemv_units(g);
  if (cta < 0 || cta >= units || ncta <= 0) return;
  const int K = g.W.k, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* xs = smem;  // [M][K]
  __shared__ unsigned long long s_best[kMkMaxRows];
  const int64_t tb = tile_bytes(K);
  const int step = g.epi == EPI_ACT_ ? ncta : 2 * ncta;
  auto rows_of = [&](int u, int& ra, int& rb, bool& hb) { gemv_rows(g, units, ncta, u, ra, rb, hb); };
  cp_async_wait_all();  // this warp's preloaded rows (read after the staging barrier)
  float(&resa)[M] = p.resa;
  float(&resb)[M] = p.resb;
  auto load_res = [&](int ra, int rb, bool hb) {
#pragma unroll
    for (int mr = 0; mr < M; ++mr) {
      resa[mr] = resb[mr] = 0.0f;
      if (g.epi == EPI_ADD_ && lane == 0 && mr < m_rows) {
        if (ra < g.rows_out) resa[mr] = __ldcg(g.y + (int64_t)mr * g.ldy + ra);
        if (hb && rb < g.rows_out) resb[mr] = __ldcg(g.y + (int64_t)mr * g.ldy + rb);
      }
    }
  };

  // Stage pre(x) = x * norm_w (RMSNorm's per-row scale is applied to the dot
  // products at the end); the sum of squares of each row is reduced on the way.
  __shared__ float wsq[kW][kMkMaxRows];  // per-warp partial sums of squares (summed in a fixed order)
  if (g.argmax && tid < kMkMaxRows) s_best[tid] = 0ull;
  __syncthreads();
  const bool norm = g.pre == PRE_RMS_ || g.pre == PRE_EMBED_;
  const bool copy = g.copy_x != nullptr && cta == 0;
  float sq[M];
#pragma unroll
  for (int mr = 0; mr < M; ++mr) sq[mr] = 0.0f;
  if (g.pre == PRE_EMBED_) {
    const CbMatrix& E = a.m.lm_head;
    const int64_t etb = tile_bytes(K);
    for (int i = tid; i < M * (K / 2); i += kT) {
      const int mr = i / (K / 2), j = i - mr * (K / 2);
      float v0 = 0.0f, v1 = 0.0f;
      if (mr < m_rows) {
        const int b = mr / a.T, t = mr - b * a.T;
        const int64_t id = a.ids[(int64_t)b * a.ids_ld + a.c0 + t];
        if (id >= 0 && id < a.m.vocab_size) {
          const uint8_t* tile = E.tiles + (id >> 4) * etb;
          const int rr = (int)(id & 15);
          const float2 f = e2m1x2_to_f32x2(tile[rr * (K / 2) + j]);
          const float s = e4m3_to_f32(tile[kTileRows * (K / 2) + rr * (K / 16) + (j >> 3)]);
          const float ts = E.tile_scale[id >> 4];
          v0 = (f.x * s) * ts;
          v1 = (f.y * s) * ts;
        } else if (j == 0) {
          set_status(a.status, CB_ERR_TOKEN);
        }
      }
      if (copy && mr < m_rows) {
        g.copy_x[mr * K + 2 * j] = v0;
        g.copy_x[mr * K + 2 * j + 1] = v1;
      }
#pragma unroll
      for (int q = 0; q < M; ++q)
        if (q == mr) sq[q] += v0 * v0 + v1 * v1;
      xs[mr * K + 2 * j] = v0 * g.norm_w[2 * j];
      xs[mr * K + 2 * j + 1] = v1 * g.norm_w[2 * j + 1];
    }
  } else if (g.pre == PRE_COMBINE_) {
    // Merge the S <= 32 split partials of every (row, head): a warp per pair,
    // a lane per split: w_s = exp(m_s - max m), coef_s = w_s * gate / sum_s w_s l_s;
    // then x = sum_s coef_s o_s with the loads of 8 splits in flight at a time.
    const int hd = g.hd, H = K / hd, S = g.S, per = hd + 2;
    float* coef = smem + M * K;  // [M][H][32]
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
        const int h = k / hd, d = k - h * hd;
        const float* pb = g.part + (int64_t)(mr * H + h) * S * per + 2 + d;
        const float* cf = coef + (mr * H + h) * 32;
        for (int s0 = 0; s0 < S; s0 += 8) {  // 8 loads in flight per batch
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = s0 + e < S ? __ldcg(pb + (s0 + e) * per) : 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) v = fmaf(cf[s0 + e], o[e], v);
        }
      }
      xs[i] = v;
    }
  } else {
#pragma unroll 4
    for (int i = tid; i < M * K; i += kT) {
      const int mr = i / K, k = i - mr * K;
      float v = 0.0f;
      if (mr < m_rows) {
        const int xr = g.xmap_nq > 0 ? (mr / g.xmap_nq) * g.xmap_T + g.xmap_off + mr % g.xmap_nq : mr;
        v = __ldcg(g.x + (int64_t)xr * g.ldx + k);
        if (copy) g.copy_x[mr * K + k] = v;
      }
      if (norm) {
#pragma unroll
        for (int q = 0; q < M; ++q)
          if (q == mr) sq[q] += v * v;
        v *= g.norm_w[k];
      }
      xs[i] = v;
    }
  }
  if (norm) {
#pragma unroll
    for (int mr = 0; mr < M; ++mr) {
      const float t = warp_sum(sq[mr]);
      if (lane == 0) wsq[warp][mr] = t;
    }
  }
  __syncthreads();
  float rn[M];
#pragma unroll
  for (int mr = 0; mr < M; ++mr) {
    rn[mr] = 1.0f;
    if (norm) {
      float t = 0.0f;
      for (int w = 0; w < kW; ++w) t += wsq[w][mr];
      rn[mr] = rsqrtf(t / (float)K + a.m.norm_eps);
    }
  }

  unsigned long long best[M];
#pragma unroll
  for (int mr = 0; mr < M; ++mr) best[mr] = 0ull;
  // the row loop, compiled for K <= 768 (3 chunks of 256 codes per lane) and K <= 2048 (8)
  auto row_loop = [&](auto nu) {
  constexpr int NU = decltype(nu)::value;
  RowW<NU> A0, B0;
  for (int u = cta; u < units; u += step) {
    int ra, rb;
    bool hb;
    rows_of(u, ra, rb, hb);
    if (u != cta || !pre_staged(K)) {
      load_row(g.W, tb, K, ra, true, A0);
      load_row(g.W, tb, K, rb, hb, B0);
      if (u != cta) load_res(ra, rb, hb);
    } else {  // the first unit's rows were copied to shared memory before the barrier
      const uint8_t* slot = pre_slot(smem, K);
      pre_read_row(slot, K, true, A0);
      pre_read_row(slot + pre_row_bytes(K), K, hb, B0);
    }
    float aa[M], ab[M];
#pragma unroll
    for (int mr = 0; mr < M; ++mr) aa[mr] = ab[mr] = 0.0f;
    dot_row<M>(A0, K, xs, aa);
    if (hb) dot_row<M>(B0, K, xs, ab);
    const float tsa = g.W.tile_scale[ra >> 4];
    const float tsb = hb ? g.W.tile_scale[rb >> 4] : 0.0f;
#pragma unroll
    for (int mr = 0; mr < M; ++mr) {
      const float va = warp_sum(aa[mr]) * tsa * rn[mr];
      const float vb = hb ? warp_sum(ab[mr]) * tsb * rn[mr] : 0.0f;
      if (lane == 0 && mr < m_rows) {
        float* yr = g.y + (int64_t)mr * g.ldy;
        if (g.epi == EPI_ACT_) {
          if (ra < g.rows_out) yr[ra] = silu(va) * vb;
        } else {
          if (ra < g.rows_out) {
            if (g.epi == EPI_ADD_) yr[ra] = resa[mr] + va;
            else yr[ra] = va;
            if (g.argmax) best[mr] = max(best[mr], pack_argmax(va, ra));
          }
          if (hb && rb < g.rows_out) {
            if (g.epi == EPI_ADD_) yr[rb] = resb[mr] + vb;
            else yr[rb] = vb;
            if (g.argmax) best[mr] = max(best[mr], pack_argmax(vb, rb));
          }
        }
      }
    }
  }
  };
  if (K <= 768) row_loop(std::integral_constant<int, 3>{});
  else row_loop(std::integral_constant<int, 8>{});
  if (g.argmax) {
    if (lane == 0)
#pragma unroll
      for (int mr = 0; mr < M; ++mr)
        if (mr < m_rows) atomicMax(&s_best[mr], best[mr]);
    __syncthreads();
    if (tid < m_rows) atomicMax(&a.amax[tid], s_best[tid]);
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

// ------------------------------------------------------------------- GDN
template <int KPT>
__device__ void gdn_item(const MkArgs& a, const CbSelfLayer& L, int h, int b, float* smem) {
  const CbModel& m = a.m;
  const int H = m.gdn_heads, Dk = m.gdn_dk, Dv = m.gdn_dv, T = a.T, KC = m.conv_size;
  const int C = 2 * H * Dk + H * Dv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_kg = Dk / KPT;  // thread groups that hold state rows
  const int v = tid % Dv, kg = tid / Dv;
  const bool holds = kg < n_kg;
  float* qs = smem;                  // [8][Dk]
  float* ks = qs + kMkMaxRows * Dk;  // [8][Dk]
  float* vs = ks + kMkMaxRows * Dk;  // [8][Dv]
  float* red = vs + kMkMaxRows * Dv; // [kT]
  float* os = red + kT;              // [8][Dv]
  __shared__ float gs[kMkMaxRows], bs[kMkMaxRows], scratch[33];
  const int64_t slot = (int64_t)b * a.c.n_gdn + L.slot;
  float* conv = a.c.gdn_conv + slot * (KC - 1) * C;
  float* S = a.c.gdn_state + slot * H * Dk * Dv + (int64_t)h * Dk * Dv;
  const float* proj = a.proj + (int64_t)b * T * a.ldp;
  float s[KPT];  // state rows of this thread, loaded first (they do not depend on the step's input)
  if (holds) {
#pragma unroll
    for (int i = 0; i < KPT; ++i) s[i] = S[(int64_t)(kg * KPT + i) * Dv + v];
  }

  for (int c = tid; c < 2 * Dk + Dv; c += kT) {
    int ch, di;
    float* dst;
    int dstride;
    if (c < Dk) { ch = h * Dk + c; dst = qs; dstride = Dk; di = c; }
    else if (c < 2 * Dk) { ch = H * Dk + h * Dk + (c - Dk); dst = ks; dstride = Dk; di = c - Dk; }
    else { ch = 2 * H * Dk + h * Dv + (c - 2 * Dk); dst = vs; dstride = Dv; di = c - 2 * Dk; }
    // causal conv with 4 taps (the persistent path requires conv_size == 4): y_t = sum_j w[j] * xx[t + j]
    float w0 = L.conv_w[(int64_t)ch * 4 + 0], w1 = L.conv_w[(int64_t)ch * 4 + 1];
    float w2 = L.conv_w[(int64_t)ch * 4 + 2], w3 = L.conv_w[(int64_t)ch * 4 + 3];
    float c0 = conv[ch], c1 = conv[(int64_t)C + ch], c2 = conv[(int64_t)2 * C + ch];
    float xin[kMkMaxRows];
#pragma unroll
    for (int t = 0; t < kMkMaxRows; ++t) xin[t] = t < T ? __ldcg(proj + (int64_t)t * a.ldp + ch) : 0.0f;
#pragma unroll
    for (int t = 0; t < kMkMaxRows; ++t) {
      if (t < T) {
        const float x = xin[t];
        float y = c0 * w0;
        y += c1 * w1;
        y += c2 * w2;
        y += x * w3;
        dst[t * dstride + di] = silu(y);
        c0 = c1;
        c1 = c2;
        c2 = x;
      }
    }
    conv[ch] = c0;
    conv[(int64_t)C + ch] = c1;
    conv[(int64_t)2 * C + ch] = c2;
  }
  if (tid < T) {
    const float av = __ldcg(proj + (int64_t)tid * a.ldp + m.gdn_off_a + h);
    const float bv = __ldcg(proj + (int64_t)tid * a.ldp + m.gdn_off_b + h);
    gs[tid] = -expf(L.A_log[h]) * softplus(av + L.dt_bias[h]);
    bs[tid] = sigmoid(bv);
  }
  __syncthreads();
  for (int job = warp; job < 2 * T; job += kW) {
    float* x = (job < T ? qs : ks) + (job % T) * Dk;
    float ss = 0.0f;
    for (int i = lane; i < Dk; i += 32) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
    for (int i = lane; i < Dk; i += 32) x[i] *= inv;
  }
  __syncthreads();
  const float scale = rsqrtf((float)Dk);
  for (int t = 0; t < T; ++t) {
    const float decay = expf(gs[t]);
    float part = 0.0f;
    if (holds) {
      const float* kt = ks + t * Dk + kg * KPT;
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        s[i] *= decay;
        part = fmaf(s[i], kt[i], part);
      }
    }
    red[tid] = part;
    __syncthreads();
    float pred = 0.0f;
    for (int g2 = 0; g2 < n_kg; ++g2) pred += red[g2 * Dv + v];
    __syncthreads();
    const float delta = bs[t] * (vs[t * Dv + v] - pred);
    part = 0.0f;
    if (holds) {
      const float* kt = ks + t * Dk + kg * KPT;
      const float* qt = qs + t * Dk + kg * KPT;
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        s[i] = fmaf(kt[i], delta, s[i]);
        part = fmaf(s[i], qt[i], part);
      }
    }
    red[tid] = part;
    __syncthreads();
    if (kg == 0) {
      float o = 0.0f;
      for (int g2 = 0; g2 < n_kg; ++g2) o += red[g2 * Dv + v];
      os[t * Dv + v] = o * scale;
    }
    __syncthreads();
  }
  if (holds) {
#pragma unroll
    for (int i = 0; i < KPT; ++i) S[(int64_t)(kg * KPT + i) * Dv + v] = s[i];
  }
  for (int t = 0; t < T; ++t) {
    const float o = tid < Dv ? os[t * Dv + tid] : 0.0f;
    const float ss = block_sum(o * o, scratch);
    if (tid < Dv) {
      const float r = rsqrtf(ss / (float)Dv + m.norm_eps);
      const float gate = __ldcg(proj + (int64_t)t * a.ldp + m.gdn_off_gate + h * Dv + tid);
      a.attn[((int64_t)b * T + t) * a.att_ld + h * Dv + tid] = o * r * L.o_norm[tid] * silu(gate);
    }
  }
  __syncthreads();
}

__device__ void gdn_phase(const MkArgs& a, const CbSelfLayer& L, int cta, int ncta, float* smem) {
  const int H = a.m.gdn_heads;
  const int kpt = max(1, a.m.gdn_dk * a.m.gdn_dv / kT);
  for (int it = cta; it < H * a.B; it += ncta) {
    const int h = it % H, b = it / H;
    switch (kpt) {
      case 1: gdn_item<1>(a, L, h, b, smem); break;
      case 2: gdn_item<2>(a, L, h, b, smem); break;
      case 4: gdn_item<4>(a, L, h, b, smem); break;
      case 8: gdn_item<8>(a, L, h, b, smem); break;
      case 16: gdn_item<16>(a, L, h, b, smem); break;
      default: gdn_item<32>(a, L, h, b, smem); break;
    }
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
      for (int d = 0; d < hd; d += 4) {
        a0 = fmaf(qq[d], kk[d], a0);
        a1 = fmaf(qq[d + 1], kk[d + 1], a1);
        a2 = fmaf(qq[d + 2], kk[d + 2], a2);
        a3 = fmaf(qq[d + 3], kk[d + 3], a3);
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
    const int q = i / hd, d = i - q * hd;
    const float* e = Sc + q * ldsc;
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;  // keys mod 4, summed in a fixed order
    int key = 0;
#pragma unroll 2
    for (; key + 4 <= n; key += 4) {
      o0 = fmaf(e[key], Vs[key * hd + d], o0);
      o1 = fmaf(e[key + 1], Vs[(key + 1) * hd + d], o1);
      o2 = fmaf(e[key + 2], Vs[(key + 2) * hd + d], o2);
      o3 = fmaf(e[key + 3], Vs[(key + 3) * hd + d], o3);
    }
    for (; key < n; ++key) o0 = fmaf(e[key], Vs[key * hd + d], o0);
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
    for (int d = lane; d < hd; d += 32) {
      const uint16_t bits = f32_to_bf16(__ldcg(row + m.swa_off_kv + Hkv * hd + g * hd + d));
      vr[off + d] = bits;
      Vs[idx * hd + d] = bf16_to_f32(bits);
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
  // the o projection merges the partials (PRE_COMBINE)
}

__device__ void swa_phase(const MkArgs& a, const CbSelfLayer& L, int cta, int ncta, float* smem) {
  const int Hkv = a.m.n_kv_heads, S = a.swa_splits;
  for (int it = cta; it < a.B * Hkv * S; it += ncta) {
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
  // the o projection merges the partials (PRE_COMBINE)
}

__device__ void cross_phase(const MkArgs& a, const CbCrossLayer& L, int cta, int ncta, float* smem) {
  const int Hkv = a.m.n_kv_heads, S = a.cross_splits, RQ = a.B * a.nq;
  for (int it = cta; it < RQ * Hkv * S; it += ncta) {
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
__device__ void shared_append(const MkArgs& a, int cta, int ncta, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int Mrows = a.B * a.T, hd = m.head_dim, Hkv = m.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int mr = cta; mr < Mrows; mr += ncta) {
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
        for (int d = lane; d < hd; d += 32) c.kv_v[base + hh * hd + d] = f32_to_bf16(__ldcg(row + Hkv * hd + hh * hd + d));
      } else {
        uint8_t* ik = c.kv_ik + ((int64_t)b * c.max_ctx + p) * m.indexer_dim;
        for (int d = lane; d < m.indexer_dim; d += 32) ik[d] = f32_to_e4m3(__ldcg(row + m.sh_off_ik + d));
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
    const float d = __fadd_rn(__fadd_rn(__fadd_rn(pr[0], pr[1]), __fadd_rn(pr[2], pr[3])),
                              __fadd_rn(__fadd_rn(pr[4], pr[5]), __fadd_rn(pr[6], pr[7])));
    const float rl = d > 0.0f ? d : 0.0f;
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
__device__ void score_phase(const MkArgs& a, int cta, int ncta, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int RQ = a.B * a.nq, Hi = m.indexer_heads, Di = m.indexer_dim, k = m.sparse_topk;
  const int tid = threadIdx.x;
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
      const int t2 = i / Di, d = i - t2 * Di;
      newk[i] = f32_to_e4m3(__ldcg(a.proj + ((int64_t)b * a.T + t2) * a.ldp + m.sh_off_ik + d));
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
__device__ void compact_phase(const MkArgs& a, int cta, int ncta, float* smem) {
  const CbModel& m = a.m;
  const CbCache& c = a.c;
  const int RQ = a.B * a.nq, k = m.sparse_topk;
  const int tid = threadIdx.x, lane = tid & 31;
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
  const int cap = (kSmem - kMkBitmapWords * (int)sizeof(unsigned)) / (int)sizeof(unsigned long long);
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
  const int shifts[7] = {45, 37, 29, 21, 13, 5, 0};
  const unsigned widths[7] = {0xFF, 0xFF, 0xFF, 0xFF, 0xFF, 0xFF, 0x1F};
#pragma unroll 1
  for (int ps = 0; ps < 7; ++ps) {
    const int shift = shifts[ps];
    const unsigned dm = widths[ps];
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

// ------------------------------------------------------------------ kernel
template <int M>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkArgs a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ int s_ok;
  unsigned gen = 0;
  const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
  const CbModel& m = a.m;
  const int d = m.d_model, Mrows = a.B * a.T, RQ = a.B * a.nq, F = m.ffn_hidden;
  const bool sparse = m.sparse_topk > 0;

  if (cta == 0) {
    // the histogram exists only with a top-k (dense cross attention carves it empty)
    if (sparse)
      for (int i = tid; i < RQ * kMkHistBins; i += kT) a.hist[i] = 0u;
    for (int i = tid; i < RQ; i += kT) {
      a.hi_cnt[i] = 0;
      a.cand_cnt[i] = 0;
      a.amax[i] = 0ull;
    }
  }
  if (cta == 0 && tid == 0) a.trace[0] = gtimer();
  if (tid == 0) {
    const unsigned long long lim = __ldcg(&a.ctl->limit_ns);
    s_wait_limit = lim ? lim : kDefaultWaitNs;
    const int stall = __ldcg(&a.ctl->stall_barrier);
    s_stall_barrier = stall > 0 ? (unsigned)stall : 0u;
  }
  // Each GEMV's first weights (and residual) are loaded between the arrival at
  // the barrier before it and the wait there (GemvPre): they do not depend on
  // the previous phase, so their latency hides behind the barrier.
  grid_arrive(a, gen);

  for (int i = 0; i < m.n_self_layers; ++i) {
    const CbSelfLayer& L = m.self_layers[i];
    GemvJob in{};
    in.W = L.in_proj;
    in.x = a.h;
    in.ldx = d;
    in.pre = i == 0 ? PRE_EMBED_ : PRE_RMS_;
    in.norm_w = L.norm1;
    in.y = a.proj;
    in.ldy = a.ldp;
    in.rows_out = L.in_proj.rows;
    in.epi = EPI_STORE_;
    in.copy_x = i == 0 ? a.h : nullptr;
    {
      GemvPre<M> p;
      gemv_pre<M>(in, Mrows, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, in, Mrows, cta, ncta, smem, p);
    }
    if (!grid_sync(a, gen, &s_ok)) return;
    if (L.kind == CB_LAYER_GDN) gdn_phase(a, L, cta, ncta, smem);
    else swa_phase(a, L, cta, ncta, smem);
    grid_arrive(a, gen);
    GemvJob o{};
    o.W = L.o_proj;
    o.x = a.attn;
    o.ldx = a.att_ld;
    if (L.kind == CB_LAYER_SWA) {
      o.pre = PRE_COMBINE_;
      o.part = a.part;
      o.S = a.swa_splits;
      o.hd = m.head_dim;
      o.gate_x = a.proj;
      o.gate_ld = a.ldp;
      o.gate_off = m.swa_off_gate;
    }
    o.y = a.h;
    o.ldy = d;
    o.rows_out = d;
    o.epi = EPI_ADD_;
    {
      GemvPre<M> p;
      gemv_pre<M>(o, Mrows, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, o, Mrows, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
    GemvJob gu{};
    gu.W = L.gate_up;
    gu.x = a.h;
    gu.ldx = d;
    gu.pre = PRE_RMS_;
    gu.norm_w = L.norm2;
    gu.y = a.act;
    gu.ldy = F;
    gu.rows_out = F;
    gu.epi = EPI_ACT_;
    {
      GemvPre<M> p;
      gemv_pre<M>(gu, Mrows, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, gu, Mrows, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
    GemvJob dn{};
    dn.W = L.down;
    dn.x = a.act;
    dn.ldx = F;
    dn.y = a.h;
    dn.ldy = d;
    dn.rows_out = d;
    dn.epi = EPI_ADD_;
    {
      GemvPre<M> p;
      gemv_pre<M>(dn, Mrows, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, dn, Mrows, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
  }

  {
    GemvJob sh{};
    sh.W = m.shared_proj;
    sh.x = a.h;
    sh.ldx = d;
    sh.pre = PRE_RMS_;
    sh.norm_w = m.shared_norm;
    sh.y = a.proj;
    sh.ldy = a.ldp;
    sh.rows_out = m.shared_proj.rows;
    sh.epi = EPI_STORE_;
    GemvPre<M> p;
    gemv_pre<M>(sh, Mrows, cta, ncta, smem, p);
    if (!grid_wait(a, gen, &s_ok)) {
      cp_async_wait_all();
      return;
    }
    gemv_phase<M>(a, sh, Mrows, cta, ncta, smem, p);
  }
  if (!grid_sync(a, gen, &s_ok)) return;
  shared_append(a, cta, ncta, smem);
  if (sparse) score_phase(a, cta, ncta, smem);
  grid_arrive(a, gen);
  if (sparse) {
    if (!grid_wait(a, gen, &s_ok)) return;
    compact_phase(a, cta, ncta, smem);
    grid_arrive(a, gen);
  }

  for (int j = 0; j < m.n_cross_layers; ++j) {
    const CbCrossLayer& L = m.cross_layers[j];
    GemvJob q{};
    q.W = L.q_gate;
    q.x = j == 0 ? a.h : a.xc;
    q.ldx = d;
    if (j == 0) {
      q.xmap_nq = a.nq;
      q.xmap_T = a.T;
      q.xmap_off = a.T - a.nq;
      q.copy_x = a.xc;
    }
    q.pre = PRE_RMS_;
    q.norm_w = L.norm1;
    q.y = a.cproj;
    q.ldy = a.cr_ld;
    q.rows_out = L.q_gate.rows;
    q.epi = EPI_STORE_;
    {
      // the exact selection of each query row runs beside the first q projection
      const bool beside = j == 0 && sparse;
      const int qc = beside ? cta - RQ : cta, qn = beside ? ncta - RQ : ncta;
      GemvPre<M> p;
      gemv_pre<M>(q, RQ, qc, qn, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      if (beside && cta < RQ) resolve_row(a, cta, smem);
      else gemv_phase<M>(a, q, RQ, qc, qn, smem, p);
    }
    if (!grid_sync(a, gen, &s_ok)) return;
    cross_phase(a, L, cta, ncta, smem);
    grid_arrive(a, gen);
    GemvJob o{};
    o.W = L.o_proj;
    o.x = a.attn;
    o.ldx = a.att_ld;
    o.pre = PRE_COMBINE_;
    o.part = a.part2;
    o.S = a.cross_splits;
    o.hd = m.head_dim;
    o.gate_x = a.cproj;
    o.gate_ld = a.cr_ld;
    o.gate_off = m.cr_off_gate;
    o.y = a.xc;
    o.ldy = d;
    o.rows_out = d;
    o.epi = EPI_ADD_;
    {
      GemvPre<M> p;
      gemv_pre<M>(o, RQ, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, o, RQ, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
    GemvJob gu{};
    gu.W = L.gate_up;
    gu.x = a.xc;
    gu.ldx = d;
    gu.pre = PRE_RMS_;
    gu.norm_w = L.norm2;
    gu.y = a.act;
    gu.ldy = F;
    gu.rows_out = F;
    gu.epi = EPI_ACT_;
    {
      GemvPre<M> p;
      gemv_pre<M>(gu, RQ, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, gu, RQ, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
    GemvJob dn{};
    dn.W = L.down;
    dn.x = a.act;
    dn.ldx = F;
    dn.y = a.xc;
    dn.ldy = d;
    dn.rows_out = d;
    dn.epi = EPI_ADD_;
    {
      GemvPre<M> p;
      gemv_pre<M>(dn, RQ, cta, ncta, smem, p);
      if (!grid_wait(a, gen, &s_ok)) {
        cp_async_wait_all();
        return;
      }
      gemv_phase<M>(a, dn, RQ, cta, ncta, smem, p);
    }
    grid_arrive(a, gen);
  }

  {
    GemvJob hd{};
    hd.W = m.lm_head;
    hd.x = a.xc;
    hd.ldx = d;
    hd.pre = PRE_RMS_;
    hd.norm_w = m.final_norm;
    hd.y = a.logits ? a.logits : a.ws_logits;
    hd.ldy = m.vocab_size;
    hd.rows_out = m.vocab_size;
    hd.epi = EPI_STORE_;
    hd.argmax = true;
    GemvPre<M> p;
    gemv_pre<M>(hd, RQ, cta, ncta, smem, p);
    if (!grid_wait(a, gen, &s_ok)) {
      cp_async_wait_all();
      return;
    }
    gemv_phase<M>(a, hd, RQ, cta, ncta, smem, p);
    if (a.hidden != nullptr && cta == ncta - 1)
      for (int i = tid; i < RQ * d; i += kT) a.hidden[i] = __ldcg(a.xc + i);
  }
  if (!grid_sync(a, gen, &s_ok)) return;
  if (cta == 0) {
    if (a.argmax != nullptr)
      for (int r = tid; r < RQ; r += kT)
        a.argmax[r] = (int32_t)(0xFFFFFFFFu - (unsigned)(__ldcg(a.amax + r) & 0xFFFFFFFFull));
    for (int b = tid; b < a.B; b += kT) a.c.pos[b] += a.T;
  }
}

}  // namespace

size_t mk_smem_bytes() { return kSmem; }

bool mk_supported(const CbModel& m, const CbCache& c, int T, int nq) {
  const int G = m.n_q_heads / m.n_kv_heads;
  if (c.batch * T > kMkMaxRows || T > CB_MAX_T || nq < 1 || nq > T) return false;
  if (m.head_dim > 128 || m.head_dim % 8 || G * T > kMkMaxQ) return false;
  if (m.gdn_dv > kMkThreads || kMkThreads % m.gdn_dv || m.gdn_dk * m.gdn_dv / kMkThreads > 32) return false;
  if ((m.gdn_dk * m.gdn_dv) % kMkThreads && m.gdn_dk * m.gdn_dv > kMkThreads) return false;
  if (m.conv_size != 4) return false;
  if (m.d_model > 2048 || m.ffn_hidden > 2048 || m.d_model % 16 || m.ffn_hidden % 16) return false;
  if (m.sparse_topk > 0 && c.max_ctx > kMkBitmapWords * 32) return false;
  if (m.sparse_topk > 0 && (m.sparse_topk + 1 > kMaxSort || m.indexer_dim % 8 || m.indexer_dim > 256 ||
                            m.indexer_heads > 16 || (m.indexer_heads * m.indexer_dim + 16 + kMkHistBins) * 4 +
                            CB_MAX_T * m.indexer_dim > kSmem))
    return false;
  const size_t att = sizeof(float) * ((size_t)kMkSwaSplit * (2 * m.head_dim + 1) + (size_t)kMkMaxQ * m.head_dim * 2 +
                                      (size_t)kMkMaxQ * kMkSwaSplit) +
                     sizeof(uint16_t) * 2 * kMkSwaSplit * m.head_dim;
  if (att > (size_t)kSmem) return false;
  if ((size_t)kMkMaxRows * 2048 * sizeof(float) > (size_t)kSmem) return false;
  {  // GEMV staging ([M][K] inputs, K <= 2048) stays below the preload slots at kPreOff
    int kmax = std::max(m.lm_head.k, m.shared_proj.k);
    for (int i = 0; i < m.n_self_layers; ++i) {
      const CbSelfLayer& L = m.self_layers[i];
      kmax = std::max({kmax, L.in_proj.k, L.o_proj.k, L.gate_up.k, L.down.k});
    }
    for (int j = 0; j < m.n_cross_layers; ++j) {
      const CbCrossLayer& L = m.cross_layers[j];
      kmax = std::max({kmax, L.q_gate.k, L.o_proj.k, L.gate_up.k, L.down.k});
    }
    if (kmax > 2048 || (size_t)kMkMaxRows * (kmax + m.n_q_heads * 32) * sizeof(float) > (size_t)kPreOff) return false;
  }
  {  // o projection staging with the split merge: [M][K] inputs + [M][H][32] weights, S <= 32 splits
    const int sw = ceil_div(m.swa_window + CB_MAX_T, kMkSwaSplit);
    const int sc = m.sparse_topk > 0 ? ceil_div(m.sparse_topk + 1, kMkCrossSplit) : 32;
    const size_t need = (size_t)kMkMaxRows * m.n_q_heads * (m.head_dim + 32) * sizeof(float);
    if (need > (size_t)kSmem || sw > 32 || sc > 32) return false;
  }
  return true;
}

int launch_mk(const MkArgs& a, int grid, cudaStream_t st) {
  const int M = a.B * a.T;
  void (*fn)(MkArgs);
  if (M <= 1) fn = decode_mk_kernel<1>;
  else if (M <= 2) fn = decode_mk_kernel<2>;
  else if (M <= 4) fn = decode_mk_kernel<4>;
  else fn = decode_mk_kernel<8>;
  if (ensure_smem_attr((const void*)fn, kSmem) != CB_OK) return CB_ERR_CUDA;
  if (resident_ctas((const void*)fn, kMkThreads, kSmem) < 1) return CB_ERR_SHAPE;  // the grid could not be co-resident
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb
