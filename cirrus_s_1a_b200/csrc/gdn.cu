// Gated DeltaNet decode / verify step (cirrus/model/layers.py:95-174).
//
// One CTA per (head, sequence).  The head's state S[k][v] (float32) lives in
// registers for the whole T-token step: thread (kg, v) holds rows
// kg*KPT .. kg*KPT+KPT-1 of column v.  Every column of S updates
// independently (pred[v] = sum_k S[k][v] k[k], then S[:, v] += k * delta[v]),
// so the only cross-thread traffic is the k-reduction through shared memory.
#include "common.cuh"
#include "gdn.cuh"

namespace cb {

constexpr int kGdnThreads = 256;

template <int KPT>
__global__ void __launch_bounds__(kGdnThreads) gdn_step_kernel(GdnParams p) {
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int H = p.H, Dk = p.Dk, Dv = p.Dv, T = p.T, KC = p.KC;
  const int n_kg = kGdnThreads / Dv;
  const int v = tid % Dv, kg = tid / Dv;

  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                    // [T][Dk]
  float* ks = qs + CB_MAX_T * Dk;    // [T][Dk]
  float* vs = ks + CB_MAX_T * Dk;    // [T][Dv]
  float* red = vs + CB_MAX_T * Dv;   // [n_kg][Dv]  (= 256 floats)
  float* os = red + kGdnThreads;     // [T][Dv]
  __shared__ float gs[CB_MAX_T], bs[CB_MAX_T], scratch[33];

  float* conv = p.conv + (int64_t)b * p.conv_stride;  // [KC-1][C]
  const float* proj = p.proj + (int64_t)b * T * p.ldp;

  // ---- short conv + SiLU over this head's q, k, v channels (layers.py:95-104)
  const int nch = 2 * Dk + Dv;
  for (int c = tid; c < nch; c += kGdnThreads) {
    int ch;
    float* dst;
    int dstride, di;
    if (c < Dk) { ch = h * Dk + c; dst = qs; dstride = Dk; di = c; }
    else if (c < 2 * Dk) { ch = H * Dk + h * Dk + (c - Dk); dst = ks; dstride = Dk; di = c - Dk; }
    else { ch = 2 * H * Dk + h * Dv + (c - 2 * Dk); dst = vs; dstride = Dv; di = c - 2 * Dk; }
    float w[8], win[8];
    for (int j = 0; j < KC; ++j) w[j] = p.conv_w[(int64_t)ch * KC + j];
    for (int j = 0; j < KC - 1; ++j) win[j] = conv[(int64_t)j * p.C + ch];
    for (int t = 0; t < T; ++t) {
      win[KC - 1] = proj[(int64_t)t * p.ldp + ch];
      float y = 0.0f;
      for (int j = 0; j < KC; ++j) y += win[j] * w[j];
      dst[t * dstride + di] = silu(y);
      for (int j = 0; j < KC - 1; ++j) win[j] = win[j + 1];
      if (p.snap_conv && t < T - 1)  // the window after token t
        for (int j = 0; j < KC - 1; ++j)
          p.snap_conv[t * p.snap_conv_t + (int64_t)b * p.conv_stride + (int64_t)j * p.C + ch] = win[j];
    }
    for (int j = 0; j < KC - 1; ++j) conv[(int64_t)j * p.C + ch] = win[j];
  }
  if (tid < T) {
    const float a = proj[(int64_t)tid * p.ldp + p.off_a + h];
    const float bb = proj[(int64_t)tid * p.ldp + p.off_b + h];
    gs[tid] = -expf(p.A_log[h]) * softplus(a + p.dt_bias[h]);  // layers.py:162
    bs[tid] = sigmoid(bb);                                     // layers.py:163
  }
  __syncthreads();

  // ---- L2-normalise q and k per token (F.normalize, eps 1e-12)
  const int warp = tid >> 5, lane = tid & 31;
  for (int job = warp; job < 2 * T; job += kGdnThreads / 32) {
    float* x = (job < T ? qs : ks) + (job % T) * Dk;
    float ss = 0.0f;
    for (int i = lane; i < Dk; i += 32) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
    for (int i = lane; i < Dk; i += 32) x[i] *= inv;
  }

  // ---- recurrence (layers.py:122-128)
  float* S = p.state + (int64_t)b * p.state_stride + (int64_t)h * Dk * Dv;
  float s[KPT];
#pragma unroll
  for (int i = 0; i < KPT; ++i) s[i] = S[(int64_t)(kg * KPT + i) * Dv + v];
  __syncthreads();

  for (int t = 0; t < T; ++t) {
    const float decay = expf(gs[t]);
    const float* kt = ks + t * Dk + kg * KPT;
    const float* qt = qs + t * Dk + kg * KPT;
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      s[i] *= decay;
      part = fmaf(s[i], kt[i], part);
    }
    red[kg * Dv + v] = part;
    __syncthreads();
    float pred = 0.0f;
    for (int g = 0; g < n_kg; ++g) pred += red[g * Dv + v];
    __syncthreads();
    const float delta = bs[t] * (vs[t * Dv + v] - pred);
    part = 0.0f;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      s[i] = fmaf(kt[i], delta, s[i]);
      part = fmaf(s[i], qt[i], part);
    }
    red[kg * Dv + v] = part;
    __syncthreads();
    if (kg == 0) {
      float o = 0.0f;
      for (int g = 0; g < n_kg; ++g) o += red[g * Dv + v];
      os[t * Dv + v] = o * p.scale;
    }
    if (p.snap_state && t < T - 1) {  // the state after token t
      float* Sn = p.snap_state + t * p.snap_state_t + (int64_t)b * p.state_stride + (int64_t)h * Dk * Dv;
#pragma unroll
      for (int i = 0; i < KPT; ++i) Sn[(int64_t)(kg * KPT + i) * Dv + v] = s[i];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < KPT; ++i) S[(int64_t)(kg * KPT + i) * Dv + v] = s[i];

  // ---- o_norm (RMSNorm over Dv) * silu(gate)  (layers.py:173)
  for (int t = 0; t < T; ++t) {
    const float o = tid < Dv ? os[t * Dv + tid] : 0.0f;
    const float ss = block_sum(o * o, scratch);
    if (tid < Dv) {
      const float r = rsqrtf(ss / (float)Dv + p.eps);
      const float gate = proj[(int64_t)t * p.ldp + p.off_gate + h * Dv + tid];
      p.out[((int64_t)b * T + t) * p.ldo + h * Dv + tid] = o * r * p.o_norm[tid] * silu(gate);
    }
  }
}

size_t gdn_smem_bytes(int Dk, int Dv) {
  return sizeof(float) * ((size_t)CB_MAX_T * (2 * Dk + Dv) + kGdnThreads + (size_t)CB_MAX_T * Dv);
}

int launch_gdn_step(const GdnParams& p, cudaStream_t st) {
  if (p.T < 1 || p.T > CB_MAX_T || p.KC < 1 || p.KC > 8) return CB_ERR_SHAPE;
  if (p.Dv > kGdnThreads || kGdnThreads % p.Dv || (p.Dk * p.Dv) % kGdnThreads) return CB_ERR_SHAPE;
  const int kpt = p.Dk * p.Dv / kGdnThreads;
  const size_t smem = gdn_smem_bytes(p.Dk, p.Dv);
  dim3 grid(p.H, p.batch);
#define CB_GDN_CASE(K)                                                                                   \
  case K: {                                                                                              \
    if (ensure_smem_attr((const void*)gdn_step_kernel<K>, 160 * 1024) != CB_OK) return CB_ERR_CUDA;      \
    gdn_step_kernel<K><<<grid, kGdnThreads, smem, st>>>(p);                                              \
    break;                                                                                               \
  }
  switch (kpt) {
    CB_GDN_CASE(1)
    CB_GDN_CASE(2)
    CB_GDN_CASE(4)
    CB_GDN_CASE(8)
    CB_GDN_CASE(16)
    CB_GDN_CASE(32)
    CB_GDN_CASE(64)
    default:
      return CB_ERR_SHAPE;
  }
#undef CB_GDN_CASE
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_gdn_step(const CbModel* m, int32_t layer, const float* proj, int32_t ldp, int32_t batch, int32_t T,
                           float* state, int64_t state_stride, float* conv, int64_t conv_stride, float* out,
                           int32_t ldo, void* stream) {
  if (!m || layer < 0 || layer >= m->n_self_layers || !proj || !state || !conv || !out || batch <= 0)
    return CB_ERR_ARG;
  const CbSelfLayer& L = m->self_layers[layer];
  if (L.kind != CB_LAYER_GDN) return CB_ERR_ARG;
  GdnParams p{};
  p.proj = proj;
  p.ldp = ldp;
  p.off_a = m->gdn_off_a;
  p.off_b = m->gdn_off_b;
  p.off_gate = m->gdn_off_gate;
  p.conv_w = L.conv_w;
  p.A_log = L.A_log;
  p.dt_bias = L.dt_bias;
  p.o_norm = L.o_norm;
  p.state = state;
  p.state_stride = state_stride;
  p.conv = conv;
  p.conv_stride = conv_stride;
  p.out = out;
  p.ldo = ldo;
  p.batch = batch;
  p.T = T;
  p.H = m->gdn_heads;
  p.Dk = m->gdn_dk;
  p.Dv = m->gdn_dv;
  p.C = 2 * m->gdn_heads * m->gdn_dk + m->gdn_heads * m->gdn_dv;
  p.KC = m->conv_size;
  p.eps = m->norm_eps;
  p.scale = 1.0f / sqrtf((float)m->gdn_dk);
  return launch_gdn_step(p, (cudaStream_t)stream);
}
