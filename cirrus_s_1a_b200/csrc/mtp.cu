// MTP draft head on the device (cirrus/model/model.py:230-245 with the MTP
// module of cirrus/model/layers.py:351-370):
//   for each pass: x = proj(cat(RMSNorm(h) * norm_h, RMSNorm(embed(tok)) * norm_e))
//                  h = x + down(silu(gate(x')) * up(x')), x' = RMSNorm(x) * ffn_norm
//                  tok = draft_ids[argmax(RMSNorm(h) * final_norm . draft_head^T)]
// as a short chain of launches on one stream: an input kernel (both norms and
// the embedding gather from the tied NVFP4 LM head), the NVFP4 GEMVs of the
// decode path for the projections, and a pick kernel that maps the argmax
// through draft_ids and feeds the next pass.
#include "common.cuh"
#include "nvfp4.cuh"

namespace cb {

constexpr int kMtpThreads = 256;

// x[0:d) = RMSNorm(h) * norm_h, x[d:2d) = RMSNorm(embed(tok)) * norm_e
__global__ void __launch_bounds__(kMtpThreads) mtp_input_kernel(const float* __restrict__ h, const int32_t* tok,
                                                                CbMatrix E, int vocab, const float* __restrict__ norm_h,
                                                                const float* __restrict__ norm_e, float eps, int d,
                                                                float* __restrict__ x, int32_t* status) {
  __shared__ float red[33];
  const int tid = threadIdx.x;
  const int id = tok[0];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && tid == 0) set_status(status, CB_ERR_TOKEN);
  const uint8_t* tile = E.tiles + (int64_t)(ok ? id >> 4 : 0) * tile_bytes(d);
  const int rr = ok ? (id & 15) : 0;
  const float ts = E.tile_scale[ok ? id >> 4 : 0];
  float sh = 0.0f, se = 0.0f;
  for (int k = tid; k < d; k += kMtpThreads) {
    const float hv = h[k];
    const float2 f = e2m1x2_to_f32x2(tile[rr * (d / 2) + (k >> 1)]);
    const float s = e4m3_to_f32(tile[kTileRows * (d / 2) + rr * (d / 16) + (k >> 4)]);
    const float ev = ok ? ((k & 1 ? f.y : f.x) * s) * ts : 0.0f;
    x[k] = hv;
    x[d + k] = ev;
    sh += hv * hv;
    se += ev * ev;
  }
  const float th = block_sum(sh, red);
  const float te = block_sum(se, red);
  const float rh = rsqrtf(th / (float)d + eps), re = rsqrtf(te / (float)d + eps);
  for (int k = tid; k < d; k += kMtpThreads) {
    x[k] = x[k] * rh * norm_h[k];
    x[d + k] = x[d + k] * re * norm_e[k];
  }
}

// tok = draft_ids[first argmax of logits[0:n)]; out[i] = tok; the next pass reads tok
__global__ void __launch_bounds__(1024) mtp_pick_kernel(const float* __restrict__ logits, int n,
                                                        const int32_t* __restrict__ draft_ids, int32_t* tok,
                                                        int32_t* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < n; i += blockDim.x) {
    const float v = logits[i];
    if (v > best) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
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
    if (lane == 0) {
      const int t = draft_ids[bi == 0x7fffffff ? 0 : bi];
      tok[0] = t;
      out[0] = t;
    }
  }
}

struct MtpScratch {
  int32_t* status;
  int32_t* tok;
  float *x, *y, *act, *logits;
  size_t bytes;
};

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

static MtpScratch mtp_carve(const CbModel& m, const CbMtp& t, char* base) {
  MtpScratch s{};
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off += al256(b);
    return base ? base + o : nullptr;
  };
  s.status = (int32_t*)take(sizeof(int32_t));
  s.tok = (int32_t*)take(sizeof(int32_t));
  s.x = (float*)take(sizeof(float) * 2 * m.d_model);
  s.y = (float*)take(sizeof(float) * m.d_model);
  s.act = (float*)take(sizeof(float) * 2 * m.ffn_hidden);
  s.logits = (float*)take(sizeof(float) * (size_t)t.draft_head.rows);
  s.bytes = off;
  return s;
}

static int mtp_gemv(const CbMatrix& W, const float* x, int ldx, const float* norm_w, float eps, int pre, int epi, float* y,
                    int ldy, int rows_out, cudaStream_t st) {
  GemvParams p{};
  p.tiles = W.tiles;
  p.tile_scale = W.tile_scale;
  p.rows = W.rows;
  p.K = W.k;
  p.x = x;
  p.ldx = ldx;
  p.m_rows = 1;
  p.norm_w = norm_w;
  p.eps = eps;
  p.y = y;
  p.ldy = ldy;
  p.rows_out = rows_out;
  return launch_gemv(p, pre, epi, st);
}

}  // namespace cb

using namespace cb;

extern "C" size_t cb_mtp_workspace_bytes(const CbModel* m, const CbMtp* mtp) {
  if (!m || !mtp) return 0;
  return mtp_carve(*m, *mtp, nullptr).bytes;
}

extern "C" int cb_mtp_draft(const CbModel* mp, const CbMtp* tp, const float* h_last, const int32_t* token, int32_t n,
                            int32_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!mp || !tp || !h_last || !token || !out || !workspace || n < 0) return CB_ERR_ARG;
  const CbModel& m = *mp;
  const CbMtp& t = *tp;
  if (!t.proj.tiles || !t.gate_up.tiles || !t.down.tiles || !t.draft_head.tiles || !t.draft_ids || t.n_draft <= 0 ||
      !t.norm_h || !t.norm_e || !t.ffn_norm || !m.final_norm || !m.lm_head.tiles)
    return CB_ERR_ARG;
  const int d = m.d_model, F2 = 2 * m.ffn_hidden;
  if (t.proj.k != 2 * d || t.gate_up.k != d || t.down.k != m.ffn_hidden || t.draft_head.k != d ||
      t.draft_head.rows < t.n_draft || d % 16)
    return CB_ERR_SHAPE;
  const MtpScratch s = mtp_carve(m, t, (char*)workspace);
  if (workspace_bytes < s.bytes) return CB_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 0) return CB_OK;
  if (cudaMemsetAsync(s.status, 0, sizeof(int32_t), st) != cudaSuccess ||
      cudaMemcpyAsync(s.tok, token, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(s.y, h_last, sizeof(float) * d, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return CB_ERR_CUDA;
  for (int i = 0; i < n; ++i) {
    mtp_input_kernel<<<1, kMtpThreads, 0, st>>>(s.y, s.tok, m.lm_head, m.vocab_size, t.norm_h, t.norm_e, m.norm_eps, d,
                                                s.x, s.status);
    count_launch();
    if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
    int rc = mtp_gemv(t.proj, s.x, 2 * d, nullptr, 0.0f, PRE_NONE, EPI_STORE, s.y, d, d, st);
    if (rc == CB_OK)
      rc = mtp_gemv(t.gate_up, s.y, d, t.ffn_norm, m.norm_eps, PRE_RMSNORM, EPI_STORE, s.act, F2, F2, st);
    if (rc == CB_OK) rc = mtp_gemv(t.down, s.act, F2, nullptr, 0.0f, PRE_SWIGLU, EPI_ADD, s.y, d, d, st);
    if (rc == CB_OK)
      rc = mtp_gemv(t.draft_head, s.y, d, m.final_norm, m.norm_eps, PRE_RMSNORM, EPI_STORE, s.logits, t.n_draft,
                    t.n_draft, st);
    if (rc != CB_OK) return rc;
    mtp_pick_kernel<<<1, 1024, 0, st>>>(s.logits, t.n_draft, t.draft_ids, s.tok, out + i);
    count_launch();
    if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
  }
  return CB_OK;
}
