// cb_forward: one CirrusModel.forward (cirrus/model/model.py:99-176) for a
// batch of sequences, as a fixed sequence of launches on one stream.
//
// Per chunk of <= CB_MAX_T tokens per sequence:
//   embed -> 12 x [in-proj GEMV (norm1 fused) -> GDN step | SWA prep + attention
//              -> o-proj GEMV (+residual) -> gate_up GEMV (norm2 fused)
//              -> down GEMV (SwiGLU fused, +residual)]
//   -> shared projection GEMV (norm fused) -> K/V/indexer-key append
//   -> (rows that need logits) indexer scores + top-k
//   -> 6 x [q|gate GEMV -> sparse attention -> o-proj -> FFN] -> final norm + LM head
// Dynamic values (positions) are read on the device, so the whole sequence
// can be captured once in a CUDA graph and replayed every step.
#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstring>

#include "attn.cuh"
#include "common.cuh"
#include "gdn.cuh"
#include "gemm.cuh"
#include "mk.cuh"
#include "nvfp4.cuh"

namespace cb {

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

struct Workspace {
  int32_t* status;
  long long* hq;   // persistent kernel: fixed-point residual streams
  long long* xq;
  float* h;
  float* proj;
  float* attn;
  float* gu;
  float* qbuf;
  float* part;
  float* xc;
  float* cproj;
  float* scores;
  int32_t* sel_idx;
  int32_t* sel_cnt;
  float* logits;
  int32_t* amax;
  // persistent kernel
  float* part2;
  unsigned* hist;
  int32_t* hi_list;
  int32_t* hi_cnt;
  unsigned long long* cand;
  int32_t* cand_cnt;
  unsigned long long* amax64;
  unsigned* sync;     // [0] barrier counter, [32] abort flag
  unsigned long long* trace;
  uint8_t* gemm_x;     // prepared GEMM inputs (cb_gemm scratch)
  size_t gemm_x_bytes;
  size_t bytes;
  int ldp, att_ld, cr_ld, n_splits, sel_ld, cross_splits;
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Token rows from which a projection runs on the tensor cores (cb_gemm_nvfp4)
// instead of the CUDA-core GEMV.
constexpr int kGemmMinRows = 17;
// Query rows (batch * tokens) from which SWA and cross attention run on the
// many-row kernels (lane groups over keys, block-wise SWA for several tokens).
constexpr int kSwaBlockRows = 32;

static int swa_splits(const CbModel& m) { return ceil_div(m.swa_window + CB_MAX_T, kSwaSplit); }
static int cross_splits(const CbModel& m) {
  return m.sparse_topk > 0 ? ceil_div(m.sparse_topk + 1, kMkCrossSplit) : 32;
}

// Whether prompt chunks longer than CB_MAX_T tokens can run on the prefill
// kernels: the chunked GDN (Dk = Dv = 64), block-wise SWA, and the tensor-core
// GEMM for every projection (K multiples of 64, F a multiple of 64).
static bool prefill_ok(const CbModel& m) {
  bool gdn = false, swa = false;
  for (int i = 0; i < m.n_self_layers; ++i) (m.self_layers[i].kind == CB_LAYER_GDN ? gdn : swa) = true;
  if (gdn && (m.gdn_dk != 64 || m.gdn_dv != 64 || m.conv_size != 4)) return false;
  if (swa && !swa_prefill_supported(m.n_q_heads, m.n_kv_heads, m.head_dim)) return false;
  return m.d_model % 64 == 0 && m.ffn_hidden % 64 == 0 && (m.n_q_heads * m.head_dim) % 64 == 0 &&
         (m.gdn_heads * m.gdn_dv) % 64 == 0;
}

// Tokens per sequence of one chunk of a T-token forward: the whole forward up
// to CB_MAX_T (decode, verify), CB_PREFILL_CHUNK for prompts on the prefill
// kernels, CB_MAX_T otherwise.
static int chunk_tokens(const CbModel& m, int T) {
  T = std::max(T, 1);
  if (T <= CB_MAX_T) return T;
  return prefill_ok(m) ? std::min(T, CB_PREFILL_CHUNK) : CB_MAX_T;
}

static Workspace carve(const CbModel& m, int batch, int T, int max_ctx, char* base) {
  Workspace w{};
  const int R = batch * chunk_tokens(m, T);
  int ldp = m.shared_proj.rows;
  for (int i = 0; i < m.n_self_layers; ++i) ldp = std::max(ldp, m.self_layers[i].in_proj.rows);
  w.ldp = ldp;
  w.att_ld = std::max(m.gdn_heads * m.gdn_dv, m.n_q_heads * m.head_dim);
  w.cr_ld = m.n_cross_layers > 0 ? m.cross_layers[0].q_gate.rows : 16;
  w.n_splits = std::max(swa_splits(m), mk_swa_splits(m));  // the larger of the two paths' split counts
  w.sel_ld = std::max(m.sparse_topk, 1) + 1;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return base ? base + o : nullptr;
  };
  w.status = (int32_t*)take(256);
  w.hq = (long long*)take(sizeof(long long) * R * m.d_model);
  w.xq = (long long*)take(sizeof(long long) * R * m.d_model);
  w.h = (float*)take(sizeof(float) * R * m.d_model);
  w.proj = (float*)take(sizeof(float) * R * ldp);
  w.attn = (float*)take(sizeof(float) * R * w.att_ld);
  w.gu = (float*)take(sizeof(float) * R * 2 * m.ffn_hidden);
  w.qbuf = (float*)take(sizeof(float) * R * m.n_q_heads * m.head_dim);
  w.part = (float*)take(sizeof(float) * R * m.n_q_heads * w.n_splits * (m.head_dim + 2));
  w.xc = (float*)take(sizeof(float) * R * m.d_model);
  w.cproj = (float*)take(sizeof(float) * R * w.cr_ld);
  w.scores = (float*)take(m.sparse_topk > 0 ? sizeof(float) * R * (size_t)max_ctx : 0);
  w.sel_idx = (int32_t*)take(m.sparse_topk > 0 ? sizeof(int32_t) * R * (size_t)w.sel_ld : 0);
  w.sel_cnt = (int32_t*)take(sizeof(int32_t) * R);
  w.logits = (float*)take(sizeof(float) * R * (size_t)m.vocab_size);
  w.amax = (int32_t*)take(sizeof(int32_t) * R);
  w.cross_splits = cross_splits(m);
  w.part2 = (float*)take(sizeof(float) * R * m.n_q_heads * w.cross_splits * (m.head_dim + 2));
  const bool sp = m.sparse_topk > 0;
  w.hist = (unsigned*)take(sp ? sizeof(unsigned) * R * kMkHistBins : 0);
  w.hi_list = (int32_t*)take(sp ? sizeof(int32_t) * R * (size_t)m.sparse_topk : 0);
  w.hi_cnt = (int32_t*)take(sizeof(int32_t) * R);
  w.cand = (unsigned long long*)take(sp ? sizeof(unsigned long long) * R * (size_t)max_ctx : 0);
  w.cand_cnt = (int32_t*)take(sizeof(int32_t) * R);
  w.amax64 = (unsigned long long*)take(sizeof(unsigned long long) * R);
  w.sync = (unsigned*)take(256);
  w.trace = (unsigned long long*)take(sizeof(unsigned long long) * kMkTrace);
  // the tensor-core GEMM's prepared inputs: the widest projection input of R rows
  const int kmax = std::max(std::max(m.d_model, m.ffn_hidden), w.att_ld);
  w.gemm_x_bytes = R >= kGemmMinRows ? gemm_scratch_bytes((kmax + 63) / 64 * 64, R) : 0;
  w.gemm_x = (uint8_t*)take(w.gemm_x_bytes);
  w.bytes = off;
  return w;
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int src_T, int t_off, int nq, int cols,
                                   float* __restrict__ dst) {
  const int r = blockIdx.x, b = r / nq, j = r % nq;
  const float* s = src + ((int64_t)b * src_T + t_off + j) * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[(int64_t)r * cols + c] = s[c];
}

template <typename Tv>
__global__ void scatter_rows_kernel(const Tv* __restrict__ src, int cols, int nqc, int nq, int off, Tv* __restrict__ dst) {
  const int r = blockIdx.x, b = r / nqc, j = r % nqc;
  Tv* d = dst + ((int64_t)b * nq + off + j) * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) d[c] = src[(int64_t)r * cols + c];
}

__global__ void advance_pos_kernel(int32_t* pos, int batch, int T) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) pos[b] += T;
}

#define CB_TRY(x)               \
  do {                          \
    const int rc_ = (x);        \
    if (rc_ != CB_OK) return rc_; \
  } while (0)

static int gemv(const CbMatrix& W, const float* x, int ldx, int m_rows, const float* norm_w, float eps, int pre, int epi,
                float* y, int ldy, int rows_out, cudaStream_t st) {
  GemvParams p{};
  p.tiles = W.tiles;
  p.tile_scale = W.tile_scale;
  p.rows = W.rows;
  p.K = W.k;
  p.x = x;
  p.ldx = ldx;
  p.m_rows = m_rows;
  p.norm_w = norm_w;
  p.eps = eps;
  p.y = y;
  p.ldy = ldy;
  p.rows_out = rows_out;
  return launch_gemv(p, pre, epi, st);
}


static bool use_gemm(const CbMatrix& W, int m_rows) { return m_rows >= kGemmMinRows && W.k % 64 == 0; }

static int gemm(const Workspace& w, const CbMatrix& W, const float* x, int ldx, int m_rows, const float* norm_w,
                float eps, int pre, int epi, float* y, int ldy, int rows_out, cudaStream_t st) {
  int32_t* status = w.status;
  GemmParams p{};
  p.xb = w.gemm_x;
  p.xb_bytes = w.gemm_x_bytes;
  p.tiles = W.tiles;
  p.tile_scale = W.tile_scale;
  p.rows = W.rows;
  p.K = W.k;
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
  return launch_gemm(p, st);
}

// One projection of m_rows token rows: the tensor-core GEMM for many rows, the GEMV otherwise.
static int proj(const Workspace& w, const CbMatrix& W, const float* x, int ldx, int m_rows, const float* norm_w,
                float eps, int pre, int epi, float* y, int ldy, int rows_out, cudaStream_t st) {
  if (use_gemm(W, m_rows))
    return gemm(w, W, x, ldx, m_rows, norm_w, eps, pre == PRE_RMSNORM ? GEMM_PRE_RMSNORM : GEMM_PRE_NONE,
                epi == EPI_ADD ? GEMM_EPI_ADD : GEMM_EPI_STORE, y, ldy, rows_out, st);
  return gemv(W, x, ldx, m_rows, norm_w, eps, pre, epi, y, ldy, rows_out, st);
}

static int ffn(const CbMatrix& gate_up, const CbMatrix& down, const float* norm2, const CbModel& m, float* x, int rows,
               const Workspace& w, cudaStream_t st) {
  const int d = m.d_model, F = m.ffn_hidden, F2 = 2 * F;
  if (use_gemm(gate_up, rows) && use_gemm(down, rows) && F % 64 == 0 && gate_up.rows == F2) {
    // gate_up with the SwiGLU epilogue -> [rows][F]; down adds into the residual stream
    CB_TRY(gemm(w, gate_up, x, d, rows, norm2, m.norm_eps, GEMM_PRE_RMSNORM, GEMM_EPI_SWIGLU, w.gu, F, F, st));
    return gemm(w, down, w.gu, F, rows, nullptr, 0.f, GEMM_PRE_NONE, GEMM_EPI_ADD, x, d, d, st);
  }
  CB_TRY(gemv(gate_up, x, d, rows, norm2, m.norm_eps, PRE_RMSNORM, EPI_STORE, w.gu, F2, F2, st));
  return gemv(down, w.gu, F2, rows, nullptr, 0.f, PRE_SWIGLU, EPI_ADD, x, d, d, st);
}

static int launch_persistent(const CbModel& m, const CbCache& c, const Workspace& w, const int64_t* ids, int T, int nq,
                             float* logits, float* hidden, int32_t* argmax, cudaStream_t st) {
  MkArgs a{};
  a.m = m;
  a.c = c;
  a.hq = w.hq;
  a.xq = w.xq;
  a.proj = w.proj;
  a.act = w.gu;
  a.cproj = w.cproj;
  a.part = w.part;
  a.part2 = w.part2;
  a.scores = w.scores;
  a.ws_logits = w.logits;
  a.hist = w.hist;
  a.hi_list = w.hi_list;
  a.hi_cnt = w.hi_cnt;
  a.cand = w.cand;
  a.cand_cnt = w.cand_cnt;
  a.sel_idx = w.sel_idx;
  a.sel_cnt = w.sel_cnt;
  a.amax = w.amax64;
  a.sync = w.sync;
  a.trace = w.trace;
  a.status = w.status;
  a.ldp = w.ldp;
  a.att_ld = w.att_ld;
  a.cr_ld = w.cr_ld;
  a.sel_ld = w.sel_ld;
  a.swa_splits = mk_swa_splits(m);
  a.cross_splits = w.cross_splits;
  a.ids = ids;
  a.ids_ld = T;
  a.c0 = 0;
  a.B = c.batch;
  a.T = T;
  a.nq = nq;
  a.logits = logits;
  a.hidden = hidden;
  a.argmax = argmax;
  a.ctl = reinterpret_cast<const WaitCtl*>(w.status);
  if (cudaMemsetAsync(w.sync, 0, 256, st) != cudaSuccess) return CB_ERR_CUDA;
  return launch_mk(a, st);
}

static int validate(const CbModel& m, const CbCache& c) {
  if (m.n_self_layers <= 0 || m.n_self_layers > CB_MAX_SELF || m.n_cross_layers <= 0 ||
      m.n_cross_layers > CB_MAX_CROSS || m.d_model <= 0 || m.d_model % 16 || m.vocab_size <= 0)
    return CB_ERR_ARG;
  if (m.n_q_heads % m.n_kv_heads || m.head_dim % 8 || m.rot_dim > m.head_dim) return CB_ERR_SHAPE;
  if (!c.pos || !c.kv_k || !c.kv_v || (m.sparse_topk > 0 && !c.kv_ik) || c.batch <= 0 || c.max_ctx <= 0)
    return CB_ERR_ARG;
  if (c.swa_slots < m.swa_window + CB_SWA_EXTRA) return CB_ERR_SHAPE;
  if (!m.lm_head.tiles || !m.shared_proj.tiles || !m.inv_freq) return CB_ERR_ARG;
  return CB_OK;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_abi_version(void) { return CB_ABI_VERSION; }

extern "C" int64_t cb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" const char* cb_status_string(int code) {
  switch (code) {
    case CB_OK: return "ok";
    case CB_ERR_ARG: return "invalid argument";
    case CB_ERR_SHAPE: return "shape not supported";
    case CB_ERR_CUDA: return "CUDA launch failed";
    case CB_ERR_WORKSPACE: return "workspace too small";
    case CB_ERR_CTX_FULL: return "context full (position >= max_ctx)";
    case CB_ERR_TOKEN: return "token id outside the vocabulary";
    case CB_ERR_TOO_LARGE: return "rows * max_ctx exceeds the static scratch of cb_indexer_topk_noalloc";
    case CB_ERR_TIMEOUT: return "a bounded wait in the persistent kernel timed out";
    default: return "unknown status";
  }
}

extern "C" size_t cb_workspace_bytes(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx) {
  if (!m || batch <= 0 || max_ctx <= 0) return 0;
  return carve(*m, batch, T, max_ctx, nullptr).bytes;
}

extern "C" int cb_workspace_layout(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx,
                                   CbWorkspaceLayout* out) {
  if (!m || !out || batch <= 0 || max_ctx <= 0 || T <= 0) return CB_ERR_ARG;
  const Workspace w = carve(*m, batch, T, max_ctx, nullptr);
  const Workspace z = carve(*m, batch, T, max_ctx, reinterpret_cast<char*>(256));  // any non-null base
  auto off = [&](const void* p) { return (uint64_t)(reinterpret_cast<const char*>(p) - reinterpret_cast<char*>(256)); };
  out->bytes = w.bytes;
  out->proj = off(z.proj);
  out->sel_idx = off(z.sel_idx);
  out->sel_cnt = off(z.sel_cnt);
  out->ld_proj = z.ldp;
  out->sel_ld = z.sel_ld;
  out->rows = batch * chunk_tokens(*m, T);
  return CB_OK;
}

extern "C" int cb_read_status(const void* workspace, int32_t* status, void* stream) {
  if (!workspace || !status) return CB_ERR_ARG;
  if (cudaMemcpyAsync(status, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream) !=
      cudaSuccess)
    return CB_ERR_CUDA;
  return cudaStreamSynchronize((cudaStream_t)stream) == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_read_trace(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx, const void* workspace,
                             uint64_t* out, int32_t n, void* stream) {
  if (!m || !workspace || !out || n <= 0 || batch <= 0 || max_ctx <= 0) return -CB_ERR_ARG;
  const Workspace w = carve(*m, batch, T, max_ctx, (char*)workspace);
  const int cnt = std::min(n, kMkTrace);
  if (cudaMemcpyAsync(out, w.trace, sizeof(uint64_t) * cnt, cudaMemcpyDeviceToHost, (cudaStream_t)stream) !=
      cudaSuccess)
    return -CB_ERR_CUDA;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return -CB_ERR_CUDA;
  return cnt;
}

extern "C" int cb_set_wait_limit(void* workspace, uint64_t limit_ns, int32_t stall_barrier, void* stream) {
  if (!workspace || stall_barrier < 0) return CB_ERR_ARG;
  const unsigned long long lim = limit_ns;
  cudaStream_t st = (cudaStream_t)stream;
  char* base = static_cast<char*>(workspace);
  if (cudaMemcpyAsync(base + offsetof(WaitCtl, stall_barrier), &stall_barrier, sizeof(int32_t),
                      cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(base + offsetof(WaitCtl, limit_ns), &lim, sizeof(lim), cudaMemcpyHostToDevice, st) !=
          cudaSuccess)
    return CB_ERR_CUDA;
  return cudaStreamSynchronize(st) == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_clear_status(void* workspace, void* stream) {
  if (!workspace) return CB_ERR_ARG;
  return cudaMemsetAsync(workspace, 0, sizeof(int32_t), (cudaStream_t)stream) == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_forward(const CbModel* mp, const CbCache* cp, void* workspace, size_t workspace_bytes,
                          const int64_t* ids, int32_t T, int32_t n_logits, float* logits, float* hidden,
                          int32_t* argmax, void* stream) {
  if (!mp || !cp || !workspace || !ids || T <= 0) return CB_ERR_ARG;
  const CbModel& m = *mp;
  const CbCache& c = *cp;
  CB_TRY(validate(m, c));
  const int B = c.batch;
  const Workspace w = carve(m, B, T, c.max_ctx, (char*)workspace);
  if (workspace_bytes < w.bytes) return CB_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const int d = m.d_model;
  const int nq = (n_logits <= 0 || n_logits > T) ? T : n_logits;
  int Tc = chunk_tokens(m, T);
  // a prompt chunk appends all its keys to the SWA ring before its attention:
  // the ring must hold window + Tc - 1 positions
  if (Tc > CB_MAX_T) Tc = std::max(CB_MAX_T, std::min(Tc, c.swa_slots - m.swa_window + 1));
  const int H = m.gdn_heads, C = 2 * H * m.gdn_dk + H * m.gdn_dv;
  const int64_t gdn_S_layer = (int64_t)H * m.gdn_dk * m.gdn_dv;
  const int64_t gdn_conv_layer = (int64_t)(m.conv_size - 1) * C;
  const int64_t swa_layer = (int64_t)c.swa_slots * m.n_kv_heads * m.head_dim;
  const int64_t kv_seq = (int64_t)c.max_ctx * m.n_kv_heads * m.head_dim;

  if (m.forward_path != CB_PATH_MULTI_KERNEL && T <= CB_MAX_T && mk_supported(m, c, T, nq)) {
    const int rc = launch_persistent(m, c, w, ids, T, nq, logits, hidden, argmax, st);
    if (rc != CB_ERR_SHAPE) return rc;  // CB_ERR_SHAPE: not co-resident on this device, use one launch per op
  }

  for (int c0 = 0; c0 < T; c0 += Tc) {
    const int tc = std::min(Tc, T - c0);
    const int R = B * tc;
    CB_TRY(launch_embed(m.lm_head, m.vocab_size, ids, T, B, tc, c0, w.h, w.status, st));

    // ------------------------------------------------------ self-decoder
    for (int i = 0; i < m.n_self_layers; ++i) {
      const CbSelfLayer& L = m.self_layers[i];
      const int ldp = L.in_proj.rows;
      CB_TRY(proj(w, L.in_proj, w.h, d, R, L.norm1, m.norm_eps, PRE_RMSNORM, EPI_STORE, w.proj, ldp, ldp, st));
      if (L.kind == CB_LAYER_GDN && tc > CB_MAX_T) {
        // prompt chunk: the conv over the chunk into w.gu (free until the FFN), then
        // the chunked recurrence with the gating and the gated RMSNorm fused
        CB_TRY(launch_gdn_conv(w.proj, ldp, L.conv_w, c.gdn_conv + (int64_t)L.slot * gdn_conv_layer,
                               (int64_t)c.n_gdn * gdn_conv_layer, B, tc, C, m.conv_size, w.gu, C, st));
        GdnChunkParams g{};
        g.q = w.gu;
        g.k = w.gu + H * m.gdn_dk;
        g.v = w.gu + 2 * H * m.gdn_dk;
        g.ld_qkv = C;
        g.a_raw = w.proj + m.gdn_off_a;
        g.b_raw = w.proj + m.gdn_off_b;
        g.ld_ab = ldp;
        g.A_log = L.A_log;
        g.dt_bias = L.dt_bias;
        g.state = c.gdn_state + (int64_t)L.slot * gdn_S_layer;
        g.state_seq = (int64_t)c.n_gdn * gdn_S_layer;
        g.out = w.attn;
        g.ld_out = w.att_ld;
        g.gate = w.proj + m.gdn_off_gate;
        g.ld_gate = ldp;
        g.o_norm = L.o_norm;
        g.eps = m.norm_eps;
        g.B = B;
        g.T = tc;
        g.H = H;
        g.scale = 1.0f / sqrtf((float)m.gdn_dk);
        CB_TRY(launch_gdn_chunk(g, st));
      } else if (L.kind == CB_LAYER_GDN) {
        GdnParams g{};
        g.proj = w.proj;
        g.ldp = ldp;
        g.off_gate = m.gdn_off_gate;
        g.off_a = m.gdn_off_a;
        g.off_b = m.gdn_off_b;
        g.conv_w = L.conv_w;
        g.A_log = L.A_log;
        g.dt_bias = L.dt_bias;
        g.o_norm = L.o_norm;
        g.state = c.gdn_state + (int64_t)L.slot * gdn_S_layer;
        g.state_stride = (int64_t)c.n_gdn * gdn_S_layer;
        g.conv = c.gdn_conv + (int64_t)L.slot * gdn_conv_layer;
        g.conv_stride = (int64_t)c.n_gdn * gdn_conv_layer;
        g.out = w.attn;
        g.ldo = w.att_ld;
        if (c.snap_state && c.snap_conv && tc > 1 && T <= CB_MAX_T) {
          g.snap_state = c.snap_state + (int64_t)L.slot * gdn_S_layer;
          g.snap_state_t = (int64_t)B * c.n_gdn * gdn_S_layer;
          g.snap_conv = c.snap_conv + (int64_t)L.slot * gdn_conv_layer;
          g.snap_conv_t = (int64_t)B * c.n_gdn * gdn_conv_layer;
        }
        g.batch = B;
        g.T = tc;
        g.H = H;
        g.Dk = m.gdn_dk;
        g.Dv = m.gdn_dv;
        g.C = C;
        g.KC = m.conv_size;
        g.eps = m.norm_eps;
        g.scale = 1.0f / sqrtf((float)m.gdn_dk);
        CB_TRY(launch_gdn_step(g, st));
      } else {
        HeadPrepParams hp{};
        hp.proj = w.proj;
        hp.ldp = ldp;
        hp.T = tc;
        hp.c0 = c0;
        hp.pos = c.pos;
        hp.Hq = m.n_q_heads;
        hp.Hkv = m.n_kv_heads;
        hp.hd = m.head_dim;
        hp.rot2 = m.rot_dim / 2;
        hp.off_q = 0;
        hp.off_k = m.swa_off_kv;
        hp.off_v = m.swa_off_kv + m.n_kv_heads * m.head_dim;
        hp.q_norm = L.q_norm;
        hp.k_norm = L.k_norm;
        hp.inv_freq = m.inv_freq;
        hp.eps = m.norm_eps;
        hp.qout = w.qbuf;
        hp.ldq = m.n_q_heads * m.head_dim;
        hp.kdst = c.swa_k + (int64_t)L.slot * swa_layer;
        hp.vdst = c.swa_v + (int64_t)L.slot * swa_layer;
        hp.seq_stride = (int64_t)c.n_swa * swa_layer;
        hp.slots = c.swa_slots;
        hp.ring = true;
        hp.status = w.status;
        CB_TRY(launch_head_prep(hp, R, st));
        SwaParams sp{};
        sp.q = w.qbuf;
        sp.ldq = hp.ldq;
        sp.kring = hp.kdst;
        sp.vring = hp.vdst;
        sp.seq_stride = hp.seq_stride;
        sp.slots = c.swa_slots;
        sp.pos = c.pos;
        sp.T = tc;
        sp.c0 = c0;
        sp.Hq = m.n_q_heads;
        sp.Hkv = m.n_kv_heads;
        sp.hd = m.head_dim;
        sp.window = m.swa_window;
        sp.split_len = kSwaSplit;
        sp.n_splits = w.n_splits;
        sp.scale = 1.0f / sqrtf((float)m.head_dim);
        sp.part = w.part;
        sp.gate = w.proj + m.swa_off_gate;
        sp.ldg = ldp;
        sp.out = w.attn;
        sp.ldo = w.att_ld;
        // prompt chunks, and decode / verify steps of many sequences: the block-wise
        // kernel (one CTA per sequence, KV head and 8 tokens) instead of the
        // split-window kernel, whose launch grows with the window
        const bool blockwise = swa_prefill_supported(m.n_q_heads, m.n_kv_heads, m.head_dim) &&
                               c.swa_slots >= m.swa_window + tc - 1 && (tc > CB_MAX_T || R >= kSwaBlockRows);
        if (tc == 1 && R >= kSwaBlockRows && decode_attn_supported(m.n_q_heads, m.n_kv_heads, m.head_dim))
          CB_TRY(launch_swa_decode(sp, B, st));
        else if (blockwise)
          CB_TRY(launch_swa_prefill(sp, B, st));
        else
          CB_TRY(launch_swa(sp, B, st));
      }
      CB_TRY(proj(w, L.o_proj, w.attn, w.att_ld, R, nullptr, 0.f, PRE_NONE, EPI_ADD, w.h, d, d, st));
      CB_TRY(ffn(L.gate_up, L.down, L.norm2, m, w.h, R, w, st));
    }

    // ------------------------------------------------ shared KV (YOCO)
    // row stride w.ldp, as in the persistent kernel (cb_workspace_layout reports it)
    const int lds = w.ldp;
    CB_TRY(proj(w, m.shared_proj, w.h, d, R, m.shared_norm, m.norm_eps, PRE_RMSNORM, EPI_STORE, w.proj, lds,
                m.shared_proj.rows, st));
    {
      HeadPrepParams hp{};
      hp.proj = w.proj;
      hp.ldp = lds;
      hp.T = tc;
      hp.c0 = c0;
      hp.pos = c.pos;
      hp.Hq = 0;
      hp.Hkv = m.n_kv_heads;
      hp.hd = m.head_dim;
      hp.rot2 = m.rot_dim / 2;
      hp.off_k = 0;
      hp.off_v = m.n_kv_heads * m.head_dim;
      hp.k_norm = m.shared_k_norm;
      hp.inv_freq = m.inv_freq;
      hp.eps = m.norm_eps;
      hp.kdst = c.kv_k;
      hp.vdst = c.kv_v;
      hp.seq_stride = kv_seq;
      hp.slots = c.max_ctx;
      hp.ring = false;
      if (m.sparse_topk > 0) {
        hp.off_ik = m.sh_off_ik;
        hp.Di = m.indexer_dim;
        hp.ikdst = c.kv_ik;
        hp.ik_seq_stride = (int64_t)c.max_ctx * m.indexer_dim;
      }
      hp.status = w.status;
      CB_TRY(launch_head_prep(hp, R, st));
    }

    // --------------------------------------------------- cross-decoder
    const int nqc = std::max(0, std::min(tc, c0 + tc - (T - nq)));
    if (nqc == 0) continue;
    const int RQ = B * nqc, t_off = tc - nqc;
    gather_rows_kernel<<<RQ, 256, 0, st>>>(w.h, tc, t_off, nqc, d, w.xc);
    count_launch();
    if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
    if (m.sparse_topk > 0) {
      IndexerParams ip{};
      ip.iq = w.proj + m.sh_off_iq;
      ip.iw = w.proj + m.sh_off_iw;
      ip.ld_q = lds;
      ip.iq_T = tc;
      ip.iq_off = t_off;
      ip.ik = c.kv_ik;
      ip.ik_seq_stride = (int64_t)c.max_ctx * m.indexer_dim;
      ip.Hi = m.indexer_heads;
      ip.Di = m.indexer_dim;
      ip.max_ctx = c.max_ctx;
      ip.pos = c.pos;
      ip.c0 = c0;
      ip.t_off = t_off;
      ip.nq = nqc;
      ip.rows = RQ;
      ip.k = m.sparse_topk;
      ip.scores = w.scores;
      ip.sel_idx = w.sel_idx;
      ip.sel_ld = w.sel_ld;
      ip.sel_cnt = w.sel_cnt;
      CB_TRY(launch_indexer_topk(ip, st));
    }
    for (int j = 0; j < m.n_cross_layers; ++j) {
      const CbCrossLayer& L = m.cross_layers[j];
      const int ldc = L.q_gate.rows;
      CB_TRY(proj(w, L.q_gate, w.xc, d, RQ, L.norm1, m.norm_eps, PRE_RMSNORM, EPI_STORE, w.cproj, ldc, ldc, st));
      CrossParams cpp{};
      cpp.proj = w.cproj;
      cpp.ldp = ldc;
      cpp.off_gate = m.cr_off_gate;
      cpp.q_norm = L.q_norm;
      cpp.inv_freq = m.inv_freq;
      cpp.rot2 = m.rot_dim / 2;
      cpp.eps = m.norm_eps;
      cpp.scale = 1.0f / sqrtf((float)m.head_dim);
      cpp.pos = c.pos;
      cpp.c0 = c0;
      cpp.t_off = t_off;
      cpp.nq = nqc;
      cpp.kk = c.kv_k;
      cpp.vv = c.kv_v;
      cpp.seq_stride = kv_seq;
      cpp.Hq = m.n_q_heads;
      cpp.Hkv = m.n_kv_heads;
      cpp.hd = m.head_dim;
      cpp.sel_idx = m.sparse_topk > 0 ? w.sel_idx : nullptr;
      cpp.sel_cnt = w.sel_cnt;
      cpp.sel_ld = w.sel_ld;
      cpp.max_ctx = c.max_ctx;
      cpp.out = w.attn;
      cpp.ldo = w.att_ld;
      if (RQ >= kSwaBlockRows && decode_attn_supported(m.n_q_heads, m.n_kv_heads, m.head_dim))
        CB_TRY(launch_cross_decode(cpp, RQ, st));
      else
        CB_TRY(launch_cross(cpp, RQ, st));
      CB_TRY(proj(w, L.o_proj, w.attn, w.att_ld, RQ, nullptr, 0.f, PRE_NONE, EPI_ADD, w.xc, d, d, st));
      CB_TRY(ffn(L.gate_up, L.down, L.norm2, m, w.xc, RQ, w, st));
    }

    // --------------------------------------------------- LM head + outputs
    const int V = m.vocab_size;
    const int out_off = c0 + t_off - (T - nq);  // first logits row of this chunk, per sequence
    const bool direct = (tc == T) && logits != nullptr;
    float* lg = direct ? logits : w.logits;
    CB_TRY(proj(w, m.lm_head, w.xc, d, RQ, m.final_norm, m.norm_eps, PRE_RMSNORM, EPI_STORE, lg, V, V, st));
    if (logits && !direct) {
      scatter_rows_kernel<float><<<RQ, 256, 0, st>>>(lg, V, nqc, nq, out_off, logits);
      count_launch();
      if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
    }
    if (argmax) {
      if (tc == T) {
        CB_TRY(launch_argmax(lg, RQ, V, V, argmax, st));
      } else {
        CB_TRY(launch_argmax(lg, RQ, V, V, w.amax, st));
        scatter_rows_kernel<int32_t><<<RQ, 32, 0, st>>>(w.amax, 1, nqc, nq, out_off, argmax);
        count_launch();
        if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
      }
    }
    if (hidden) {
      scatter_rows_kernel<float><<<RQ, 256, 0, st>>>(w.xc, d, nqc, nq, out_off, hidden);
      count_launch();
      if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
    }
  }
  advance_pos_kernel<<<ceil_div(B, 128), 128, 0, st>>>(c.pos, B, T);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}
