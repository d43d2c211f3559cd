// Speculative decoding on the device: prompt-lookup drafts and greedy
// acceptance with a rewind to the accepted prefix (the draft -> verify ->
// accept loop of cirrus/model/generate.py:43-89 with the drafter and the
// acceptance rule of cirrus/decoding/prompt_lookup.py:19-74), so that a whole
// decoding step is three launches on one stream and the host reads tokens only
// when it wants them.
//
// Drafter: instead of the reference's incremental n-gram index, every
// candidate position of the sequence's token history is compared with the
// last n tokens in parallel (one CTA per sequence, a block-wide max of the
// matching positions), from n = max_ngram down: at 32K tokens that is 32K
// comparisons per n, a few microseconds, and it needs no per-sequence index
// state on the device.
#include <algorithm>

#include "common.cuh"

namespace cb {

constexpr int kDraftThreads = 512;
constexpr int kAcceptThreads = 256;

// draft_len[b] and the verify input ids[b][0..T): the pending token, the draft, padding.
__global__ void __launch_bounds__(kDraftThreads) prompt_lookup_kernel(const int32_t* __restrict__ tokens, int ld,
                                                                      const int32_t* __restrict__ lens,
                                                                      const int32_t* __restrict__ budget, int min_ngram,
                                                                      int max_ngram, int max_draft, int64_t* ids, int T,
                                                                      int32_t* draft_len) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t* tok = tokens + (int64_t)b * ld;
  const int L = lens[b];
  __shared__ int s_best;
  __shared__ int key[16];
  if (tid == 0) s_best = -1;
  const int cap = min(min(max_draft, T - 1), budget[b] - 1);
  __syncthreads();
  for (int n = max_ngram; n >= min_ngram && cap > 0 && L >= 1; --n) {
    if (L < n + 1) continue;
    if (tid < n) key[tid] = tok[L - n + tid];
    __syncthreads();
    // the latest position p in [n, L - 1] whose preceding n tokens equal the last n
    int best = -1;
    for (int p = L - 1 - tid; p >= n; p -= kDraftThreads) {
      bool eq = true;
      for (int i = 0; i < n && eq; ++i) eq = tok[p - n + i] == key[i];
      if (eq) {
        best = p;
        break;  // this thread's later candidates are all smaller
      }
    }
    if (best >= 0) atomicMax(&s_best, best);
    __syncthreads();
    if (s_best >= 0) break;  // the longest n-gram with an earlier occurrence wins
    __syncthreads();
  }
  __syncthreads();
  const int start = s_best;
  int dl = 0;
  if (start >= 0 && cap > 0) dl = min(cap, L - start);
  const int64_t pending = L >= 1 ? tok[L - 1] : 0;
  for (int t = tid; t < T; t += kDraftThreads) {
    int64_t v = pending;
    if (t >= 1 && t - 1 < dl) v = tok[start + t - 1];
    ids[(int64_t)b * T + t] = v;
  }
  if (tid == 0) draft_len[b] = dl;
}

// Accept, append, rewind.  Grid (batch, copy splits): split 0 does the
// bookkeeping; every split copies its share of the snapshot back.
struct AcceptParams {
  const int32_t* argmax;
  const int64_t* ids;
  const int32_t* draft_len;
  int T;
  int32_t* tokens;
  int ld;
  int32_t* lens;
  int32_t* budget;
  int64_t* emitted;
  int32_t* pos;
  float* state;        // [batch][per_state]
  const float* snap_state;  // [T-1][batch][per_state]
  int64_t per_state;
  float* conv;
  const float* snap_conv;
  int64_t per_conv;
  int batch;
};

__device__ __forceinline__ int accepted_prefix(const AcceptParams& p, int b) {
  const int dl = p.draft_len[b];
  int n = 0;
  while (n < dl && p.ids[(int64_t)b * p.T + 1 + n] == (int64_t)p.argmax[(int64_t)b * p.T + n]) ++n;
  return n;
}

__global__ void __launch_bounds__(kAcceptThreads) spec_accept_kernel(AcceptParams p) {
  const int b = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y, tid = threadIdx.x;
  // (a sequence that finishes in this step may look finished to a split that runs
  // after split 0's update and skip its copy: its state is not used again)
  const bool active = p.budget[b] > 0;
  const int n = active ? accepted_prefix(p, b) : 0;
  __syncthreads();
  // the snapshot after token n replaces the state the verify left behind (all T tokens)
  if (active && n < p.T - 1 && p.snap_state) {
    const float* ss = p.snap_state + ((int64_t)n * p.batch + b) * p.per_state;
    float* ds = p.state + (int64_t)b * p.per_state;
    for (int64_t i = split * (int64_t)kAcceptThreads + tid; i < p.per_state; i += (int64_t)nsplit * kAcceptThreads)
      ds[i] = ss[i];
    const float* sc = p.snap_conv + ((int64_t)n * p.batch + b) * p.per_conv;
    float* dc = p.conv + (int64_t)b * p.per_conv;
    for (int64_t i = split * (int64_t)kAcceptThreads + tid; i < p.per_conv; i += (int64_t)nsplit * kAcceptThreads)
      dc[i] = sc[i];
  }
  if (split != 0 || tid != 0) return;
  if (!active) {
    p.pos[b] -= p.T;  // a finished sequence keeps its position
    return;
  }
  const int L = p.lens[b];
  int32_t* tok = p.tokens + (int64_t)b * p.ld;
  for (int i = 0; i < n; ++i) tok[L + i] = (int32_t)p.ids[(int64_t)b * p.T + 1 + i];
  tok[L + n] = p.argmax[(int64_t)b * p.T + n];
  p.lens[b] = L + n + 1;
  p.budget[b] -= n + 1;
  p.pos[b] -= p.T - 1 - n;
  atomicAdd(reinterpret_cast<unsigned long long*>(p.emitted), (unsigned long long)(n + 1));
}

}  // namespace cb

using namespace cb;

extern "C" int cb_prompt_lookup_draft(const int32_t* tokens, int32_t ld, const int32_t* lens, const int32_t* budget,
                                      int32_t batch, int32_t min_ngram, int32_t max_ngram, int32_t max_draft,
                                      int64_t* ids, int32_t T, int32_t* draft_len, void* stream) {
  if (!tokens || !lens || !budget || !ids || !draft_len || batch <= 0 || T <= 0 || ld <= 0) return CB_ERR_ARG;
  if (min_ngram < 1 || max_ngram < min_ngram || max_ngram > 16 || max_draft < 0) return CB_ERR_ARG;
  prompt_lookup_kernel<<<batch, kDraftThreads, 0, (cudaStream_t)stream>>>(tokens, ld, lens, budget, min_ngram,
                                                                          max_ngram, max_draft, ids, T, draft_len);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C" int cb_spec_accept(const CbModel* m, const CbCache* c, const int32_t* argmax, const int64_t* ids,
                              const int32_t* draft_len, int32_t T, int32_t* tokens, int32_t ld, int32_t* lens,
                              int32_t* budget, int64_t* emitted, void* stream) {
  if (!m || !c || !argmax || !ids || !draft_len || !tokens || !lens || !budget || !emitted || T <= 0 || ld <= 0)
    return CB_ERR_ARG;
  if (T > CB_MAX_T || !c->pos) return CB_ERR_SHAPE;
  if (T > 1 && (!c->snap_state || !c->snap_conv)) return CB_ERR_ARG;
  AcceptParams p{};
  p.argmax = argmax;
  p.ids = ids;
  p.draft_len = draft_len;
  p.T = T;
  p.tokens = tokens;
  p.ld = ld;
  p.lens = lens;
  p.budget = budget;
  p.emitted = emitted;
  p.pos = c->pos;
  const int C = 2 * m->gdn_heads * m->gdn_dk + m->gdn_heads * m->gdn_dv;
  p.per_state = (int64_t)c->n_gdn * m->gdn_heads * m->gdn_dk * m->gdn_dv;
  p.per_conv = (int64_t)c->n_gdn * (m->conv_size - 1) * C;
  p.state = c->gdn_state;
  p.conv = c->gdn_conv;
  p.snap_state = T > 1 ? c->snap_state : nullptr;
  p.snap_conv = T > 1 ? c->snap_conv : nullptr;
  p.batch = c->batch;
  const int nsplit = (int)std::max<int64_t>(1, std::min<int64_t>(32, p.per_state / (kAcceptThreads * 64)));
  spec_accept_kernel<<<dim3(c->batch, nsplit), kAcceptThreads, 0, (cudaStream_t)stream>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}
