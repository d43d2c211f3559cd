// Chunked Gated DeltaNet for prefill: the recurrence of gated_delta_rule_ref
// (cirrus/model/layers.py:108-129; S[k, v], per token t:
//   S <- e^{g_t} S;  d_t = beta_t (v_t - S^T k_t);  S <- S + k_t d_t^T;
//   o_t = S^T (q_t * scale))
// evaluated 64 tokens at a time, the form the reference delegates to fla's
// chunk_gated_delta_rule on CUDA (layers.py:165-170).
//
// Within a chunk with start state S0 and cumulative log decay G_t = sum_{s<=t} g_s,
// unrolling the recurrence gives S_t = e^{G_t} S0 + sum_{i<=t} e^{G_t - G_i} k_i d_i^T, so
//   d_t = beta_t (v_t - e^{G_t} S0^T k_t - sum_{i<t} e^{G_t - G_i} (k_i . k_t) d_i),
// i.e. (I + diag(beta) A) D = diag(beta) V - diag(beta e^G) K S0 with the strictly
// lower A[t][i] = e^{G_t - G_i} (k_t . k_i).  Solving for U (right-hand side
// diag(beta) V) and W (diag(beta e^G) K) gives D = U - W S0, and
//   O   = diag(e^G) Q~ S0 + (Q~ K^T o M) D,   M[t][i] = e^{G_t - G_i} for i <= t,
//   S_C = e^{G_C} S0 + K^T diag(e^{G_C - G}) D,           Q~ = q * scale.
// All exponents are <= 0 (g <= 0), so nothing overflows.
//
// The value columns of S, V, U, D and O never mix: a cluster of NS CTAs per
// (sequence, head) splits them (4 when the grid is small, 1 with many
// sequences), each CTA owning 64 / NS columns of the state in shared memory
// and walking the chunks in order.  Every CTA also forms the
// column-free parts (the normalised K and Q, the decays, A, P and W) itself.
// The products are fp32 (4 x 4 or 4 x 1 outputs per thread); the triangular
// solve goes in 16-row blocks: a parallel update from the finished blocks, then
// one thread per right-hand-side column inside the block.  The gated RMSNorm of
// an output row needs all 64 columns: the CTAs exchange their rows' sums of
// squares through distributed shared memory.
#include "common.cuh"
#include "gdn.cuh"

namespace cb {
namespace {

constexpr int kGc = 64;         // chunk length
constexpr int kGd = 64;         // Dk = Dv
constexpr int kGp = kGd + 1;    // padded row stride of 64-wide arrays (floats)
constexpr int kGThreads = 256;

// acc[r][c] += sum_{k < n} X[(r0 + r) * xr + k * xk] * Y[k * yk + (c0 + c) * yc]
__device__ __forceinline__ void mm44(const float* X, int xr, int xk, const float* Y, int yk, int yc, int n, int r0,
                                     int c0, float (&acc)[4][4]) {
#pragma unroll 4
  for (int k = 0; k < n; ++k) {
    float a[4], b[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r] = X[(r0 + r) * xr + k * xk];
#pragma unroll
    for (int c = 0; c < 4; ++c) b[c] = Y[k * yk + (c0 + c) * yc];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], b[c], acc[r][c]);
  }
}

// acc[r][j] += sum_{k < n} X[(r0 + r) * xr + k * xk] * Y[k * yk + c0 + j]
template <int CW>
__device__ __forceinline__ void mm4c(const float* X, int xr, int xk, const float* Y, int yk, int n, int r0, int c0,
                                     float (&acc)[4][CW]) {
#pragma unroll 4
  for (int k = 0; k < n; ++k) {
    float a[4], bb[CW];
#pragma unroll
    for (int r = 0; r < 4; ++r) a[r] = X[(r0 + r) * xr + k * xk];
#pragma unroll
    for (int j = 0; j < CW; ++j) bb[j] = Y[k * yk + c0 + j];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < CW; ++j) acc[r][j] = fmaf(a[r], bb[j], acc[r][j]);
  }
}

// NS CTAs per (sequence, head), each owning 64 / NS value columns.
template <int NS>
__global__ void __launch_bounds__(kGThreads, 1) gdn_chunk_kernel(const __grid_constant__ GdnChunkParams p) {
  constexpr int kGns = NS;
  constexpr int kGcw = kGd / NS;   // value columns of this CTA
  constexpr int kGq = kGcw + 1;    // padded row stride of the column arrays
  constexpr int CW = kGcw / 16;    // columns per thread in the 64 x kGcw products
  extern __shared__ __align__(16) float gsm[];
  float* Kc = gsm;                  // [C][kGp]
  float* Qc = Kc + kGc * kGp;       // [C][kGp]    q * scale
  float* A = Qc + kGc * kGp;        // [C][kGp]    strictly lower e^{G_t-G_i} k_t.k_i
  float* P = A + kGc * kGp;         // [C][kGp]    lower-inclusive e^{G_t-G_i} q~_t.k_i
  float* W = P + kGc * kGp;         // [C][kGp]    solve of diag(beta e^G) K
  float* S = W + kGc * kGp;         // [Dk][kGq]   this CTA's state columns
  float* Vc = S + kGd * kGq;        // [C][kGq]
  float* U = Vc + kGc * kGq;        // [C][kGq]    then D
  float* X = U + kGc * kGq;         // [C][kGq]    D scaled for the state update; output rows
  __shared__ float Gs[kGc], bs[kGc];
  __shared__ float ssq[2][NS][kGc];  // rows' partial sums of squares, from every rank (by chunk parity)
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15, r0 = 4 * ty, c0 = 4 * tx;
  const int cs = (int)(blockIdx.x % kGns), bh = (int)(blockIdx.x / kGns);
  const int b = bh / p.H, h = bh - b * p.H, H = p.H, v0 = cs * kGcw;
  const bool model = p.a_raw != nullptr;
  float* Sg = p.state + (int64_t)b * p.state_seq + (int64_t)h * kGd * kGd;
  for (int i = tid; i < kGd * kGcw; i += kGThreads) S[(i / kGcw) * kGq + (i % kGcw)] = Sg[(i / kGcw) * kGd + v0 + i % kGcw];

  for (int t0 = 0, chunk = 0; t0 < p.T; t0 += kGc, ++chunk) {
    const int tc = min(kGc, p.T - t0);
    __syncthreads();  // S written by the previous chunk; chunk buffers free
    for (int i = tid; i < kGc * kGd; i += kGThreads) {
      const int t = i / kGd, d = i - t * kGd;
      float kv = 0.0f, qv = 0.0f;
      if (t < tc) {
        const int64_t off = ((int64_t)b * p.T + t0 + t) * p.ld_qkv + (int64_t)h * kGd + d;
        kv = p.k[off];
        qv = p.q[off];
      }
      Kc[t * kGp + d] = kv;
      Qc[t * kGp + d] = qv;
    }
    for (int i = tid; i < kGc * kGcw; i += kGThreads) {
      const int t = i / kGcw, d = i - t * kGcw;
      Vc[t * kGq + d] = t < tc ? p.v[((int64_t)b * p.T + t0 + t) * p.ld_qkv + (int64_t)h * kGd + v0 + d] : 0.0f;
    }
    if (model) {
      // L2-normalise the chunk's q and k rows (x / max(||x||, 1e-12)); a warp per row
      __syncthreads();
      const int warp = tid >> 5, lane = tid & 31;
      for (int j = warp; j < 2 * kGc; j += kGThreads / 32) {
        float* x = (j < kGc ? Qc : Kc) + (j & (kGc - 1)) * kGp;
        const float a0 = x[lane], a1 = x[lane + 32];
        const float ss = warp_sum(a0 * a0 + a1 * a1);
        const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
        x[lane] = a0 * inv;
        x[lane + 32] = a1 * inv;
      }
      __syncthreads();
    }
    for (int i = tid; i < kGc * kGd; i += kGThreads) Qc[(i / kGd) * kGp + (i % kGd)] *= p.scale;
    if (tid < 32) {  // G = inclusive prefix sum of g (padded tokens: g = 0, beta = 0)
      float g0 = 0.0f, g1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
      if (model) {
        const float Ah = -expf(p.A_log[h]), dtb = p.dt_bias[h];
        const int64_t rr = (int64_t)b * p.T + t0;
        if (tid < tc) {
          g0 = Ah * softplus(p.a_raw[(rr + tid) * p.ld_ab + h] + dtb);
          b0 = sigmoid(p.b_raw[(rr + tid) * p.ld_ab + h]);
        }
        if (tid + 32 < tc) {
          g1 = Ah * softplus(p.a_raw[(rr + tid + 32) * p.ld_ab + h] + dtb);
          b1 = sigmoid(p.b_raw[(rr + tid + 32) * p.ld_ab + h]);
        }
      } else {
        const int64_t o0 = ((int64_t)b * p.T + t0) * H + h;
        g0 = tid < tc ? p.g[o0 + (int64_t)tid * H] : 0.0f;
        g1 = tid + 32 < tc ? p.g[o0 + (int64_t)(tid + 32) * H] : 0.0f;
        b0 = tid < tc ? p.beta[o0 + (int64_t)tid * H] : 0.0f;
        b1 = tid + 32 < tc ? p.beta[o0 + (int64_t)(tid + 32) * H] : 0.0f;
      }
      bs[tid] = b0;
      bs[tid + 32] = b1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float a0 = __shfl_up_sync(0xffffffffu, g0, o), a1 = __shfl_up_sync(0xffffffffu, g1, o);
        if (tid >= o) {
          g0 += a0;
          g1 += a1;
        }
      }
      g1 += __shfl_sync(0xffffffffu, g0, 31);
      Gs[tid] = g0;
      Gs[tid + 32] = g1;
    }
    __syncthreads();
    // A (strictly lower) and P (lower inclusive)
    {
      float a[4][4] = {}, q[4][4] = {};
      mm44(Kc, kGp, 1, Kc, 1, kGp, kGd, r0, c0, a);
      mm44(Qc, kGp, 1, Kc, 1, kGp, kGd, r0, c0, q);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int t = r0 + r, i = c0 + c;
          const float e = i <= t ? expf(Gs[t] - Gs[i]) : 0.0f;
          A[t * kGp + i] = i < t ? e * a[r][c] : 0.0f;
          P[t * kGp + i] = e * q[r][c];
        }
    }
    __syncthreads();
    // forward substitution X_t = beta_t (R_t - sum_{i<t} A[t][i] X_i) for U (R = this
    // CTA's V columns) and W (R = e^G K, all 64 columns), in 4 row blocks of 16:
    // all threads subtract the finished blocks, then one thread per column finishes
    // the block's rows in order
    constexpr int kNcol = kGcw + kGd;
    for (int blk = 0; blk < kGc / 16; ++blk) {
      const int tb0 = 16 * blk;
      for (int e = tid; e < 16 * kNcol; e += kGThreads) {
        const int t = tb0 + e / kNcol, col = e % kNcol;
        const bool isu = col < kGcw;
        const int c = isu ? col : col - kGcw;
        float* Xs = isu ? U : W;
        const int ld = isu ? kGq : kGp;
        float y = isu ? Vc[t * kGq + c] : expf(Gs[t]) * Kc[t * kGp + c];
        for (int i = 0; i < tb0; ++i) y = fmaf(-A[t * kGp + i], Xs[i * ld + c], y);
        Xs[t * ld + c] = y;
      }
      __syncthreads();
      if (tid < kNcol) {
        const bool isu = tid < kGcw;
        const int c = isu ? tid : tid - kGcw;
        float* Xs = isu ? U : W;
        const int ld = isu ? kGq : kGp;
        for (int t = tb0; t < tb0 + 16; ++t) {
          float y = Xs[t * ld + c];
          for (int i = tb0; i < t; ++i) y = fmaf(-A[t * kGp + i], Xs[i * ld + c], y);
          Xs[t * ld + c] = bs[t] * y;
        }
      }
      __syncthreads();
    }
    // thread (rows rr0 .. rr0 + 3, columns cc .. cc + CW - 1) of every 64 x kGcw product
    const int rr0 = 4 * (tid >> 4), cc = CW * (tid & 15);
    // D = U - W S0 (into U), and O = diag(e^G) Q~ S0 + P D
    float o[4][CW] = {};
    {
      float ws[4][CW] = {};
      mm4c<CW>(W, kGp, 1, S, kGq, kGd, rr0, cc, ws);
      mm4c<CW>(Qc, kGp, 1, S, kGq, kGd, rr0, cc, o);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          U[(rr0 + r) * kGq + cc + j] -= ws[r][j];
          o[r][j] *= expf(Gs[rr0 + r]);
        }
    }
    __syncthreads();
    mm4c<CW>(P, kGp, 1, U, kGq, kGc, rr0, cc, o);
    if (p.gate == nullptr) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = rr0 + r;
        if (t < tc)
#pragma unroll
          for (int j = 0; j < CW; ++j)
            p.out[((int64_t)b * p.T + t0 + t) * p.ld_out + (int64_t)h * kGd + v0 + cc + j] = o[r][j];
      }
    } else {
      // gated RMSNorm of each output row over all 64 columns: this CTA's rows through
      // X, their sums of squares to every rank of the cluster
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < CW; ++j) X[(rr0 + r) * kGq + cc + j] = o[r][j];
      __syncthreads();
      const int par = chunk & 1;
      if (tid < kGc) {
        float ss = 0.0f;
#pragma unroll
        for (int c = 0; c < kGcw; ++c) ss = fmaf(X[tid * kGq + c], X[tid * kGq + c], ss);
        for (int q = 0; q < kGns; ++q) {
          uint32_t ra;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                       : "=r"(ra)
                       : "r"((uint32_t)__cvta_generic_to_shared(&ssq[par][cs][tid])), "r"(q));
          asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(ss) : "memory");
        }
      }
      asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
      for (int i = tid; i < tc * kGcw; i += kGThreads) {
        const int t = i / kGcw, c = i - t * kGcw;
        float tot = 0.0f;
        for (int q = 0; q < kGns; ++q) tot += ssq[par][q][t];
        const float rr = rsqrtf(tot / (float)kGd + p.eps);
        const int64_t row = (int64_t)b * p.T + t0 + t;
        const float gt = p.gate[row * p.ld_gate + (int64_t)h * kGd + v0 + c];
        p.out[row * p.ld_out + (int64_t)h * kGd + v0 + c] = X[t * kGq + c] * rr * p.o_norm[v0 + c] * silu(gt);
      }
      __syncthreads();  // X is rewritten below
    }
    // S = e^{G_C} S0 + K^T diag(e^{G_C - G}) D
    {
      const float gC = Gs[kGc - 1];
      for (int i = tid; i < kGc * kGcw; i += kGThreads) {
        const int t = i / kGcw, d = i - t * kGcw;
        X[t * kGq + d] = expf(gC - Gs[t]) * U[t * kGq + d];
      }
      __syncthreads();
      float sn[4][CW] = {};
      mm4c<CW>(Kc, 1, kGp, X, kGq, kGc, rr0, cc, sn);
      __syncthreads();  // all reads of S0 finished
      const float eC = expf(gC);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          float* sp = S + (rr0 + r) * kGq + cc + j;
          *sp = fmaf(eC, *sp, sn[r][j]);
        }
    }
  }
  __syncthreads();
  for (int i = tid; i < kGd * kGcw; i += kGThreads) Sg[(i / kGcw) * kGd + v0 + i % kGcw] = S[(i / kGcw) * kGq + (i % kGcw)];
}

}  // namespace

size_t gdn_chunk_smem(int ns) {
  const size_t q = kGd / ns + 1;
  return sizeof(float) * (size_t)(5 * kGc * kGp + kGd * q + 3 * kGc * q);
}

int launch_gdn_chunk(const GdnChunkParams& p, cudaStream_t st) {
  if (p.B < 1 || p.T < 1 || p.H < 1) return CB_ERR_ARG;
  // split the value columns over 4 CTAs per head while that keeps the grid within
  // about two waves; with many sequences one CTA per head does less redundant work
  const int kGns = p.B * p.H * 4 <= 2 * num_sms() ? 4 : 1;
  const void* fn = kGns == 4 ? (const void*)gdn_chunk_kernel<4> : (const void*)gdn_chunk_kernel<1>;
  const size_t smem = gdn_chunk_smem(kGns);
  if (ensure_smem_attr(fn, (int)smem) != CB_OK) return CB_ERR_CUDA;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.B * p.H * kGns);
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kGns;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<GdnChunkParams*>(&p)};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  count_launch();
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_gdn_chunk_prefill(const float* q, const float* k, const float* v, const float* g, const float* beta,
                                    int32_t B, int32_t T, int32_t H, int32_t Dk, int32_t Dv, float scale,
                                    float* state, float* out, void* stream) {
  if (!q || !k || !v || !g || !beta || !state || !out || B < 1 || T < 1 || H < 1) return CB_ERR_ARG;
  if (Dk != kGd || Dv != kGd) return CB_ERR_SHAPE;
  GdnChunkParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.ld_qkv = (int64_t)H * kGd;
  p.g = g;
  p.beta = beta;
  p.state = state;
  p.state_seq = (int64_t)H * kGd * kGd;
  p.out = out;
  p.ld_out = (int64_t)H * kGd;
  p.B = B;
  p.T = T;
  p.H = H;
  p.scale = scale;
  return launch_gdn_chunk(p, (cudaStream_t)stream);
}
