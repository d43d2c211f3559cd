// Lightning-indexer scores and exact stable top-k (cirrus/model/layers.py:282-309).
//
// Scores use one fixed float32 order (no fused multiply-add), so equal
// inputs give bit-identical scores on any device:
//   per head: p[r] = sum_i q[8i+r]*k[8i+r] (i ascending, r = 0..7),
//             d = ((p0+p1)+(p2+p3)) + ((p4+p5)+(p6+p7)),  relu(d) = d > 0 ? d : +0
//   score = w0*r0, then score += w_h*r_h for h = 1, 2, ...
// Selection: the k keys with the largest (score, index) pairs -- a key with a
// higher index wins a tie, as the reference's stable sort of the flipped row
// does -- plus the query's own key; every key when there are at most k.
// The k-th largest score is found by a 4-pass 8-bit radix select over the
// order-preserving 32-bit key of each score; the ties at that score are then
// taken from the highest index down.
#include <algorithm>
#include <mutex>

#include "attn.cuh"
#include "common.cuh"
#include "nvfp4.cuh"

namespace cb {

constexpr int kScoreThreads = 256;
constexpr int kTopkThreads = 1024;
constexpr int kMaxDi = 256;
constexpr int kMaxHi = 16;

__device__ __forceinline__ void row_seq_pos(const IndexerParams& p, int r, int& b, int& qp, int& iq_row) {
  if (p.seq_arr) {
    b = p.seq_arr[r];
    qp = p.qpos_arr[r];
    iq_row = r;
  } else {
    b = r / p.nq;
    const int j = r % p.nq;
    qp = p.pos[b] + p.c0 + p.t_off + j;
    iq_row = b * p.iq_T + p.iq_off + j;
  }
}

__global__ void __launch_bounds__(kScoreThreads) indexer_score_kernel(IndexerParams p) {
  const int r = blockIdx.y;
  int b, qp, iq_row;
  row_seq_pos(p, r, b, qp, iq_row);
  const int n = min(qp + 1, p.max_ctx);
  if (n <= p.k) return;  // every key is selected; no scores needed
  __shared__ float q[kMaxHi * kMaxDi];
  __shared__ float w[kMaxHi];
  const int Hi = p.Hi, Di = p.Di;
  for (int i = threadIdx.x; i < Hi * Di; i += kScoreThreads) q[i] = p.iq[(int64_t)iq_row * p.ld_q + i];
  for (int i = threadIdx.x; i < Hi; i += kScoreThreads) w[i] = p.iw[(int64_t)iq_row * p.ld_q + i];
  __syncthreads();
  const uint8_t* ikb = p.ik + (int64_t)b * p.ik_seq_stride;
  float* out = p.scores + (int64_t)r * p.max_ctx;
  // Each key's 8-byte groups are read and converted once and feed every head
  // (up to kHiFast heads in registers; more heads take the per-head loop).
  constexpr int kHiFast = 4;
  for (int j = blockIdx.x * kScoreThreads + threadIdx.x; j < n; j += gridDim.x * kScoreThreads) {
    const uint8_t* kr = ikb + (int64_t)j * Di;
    float score = 0.0f;
    if (Hi <= kHiFast) {
      float pr[kHiFast][8];
      for (int i = 0; i < Di / 8; ++i) {
        const uint2 raw = *reinterpret_cast<const uint2*>(kr + 8 * i);
        float kv[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // pairs of E4M3 codes -> exact halves -> floats
          const uint32_t w2 = ((e < 2 ? raw.x : raw.y) >> (16 * (e & 1))) & 0xFFFF;
          const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)w2, __NV_E4M3);
          const float2 f = __half22float2(__half2(hr));
          kv[2 * e] = f.x;
          kv[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int h = 0; h < kHiFast; ++h) {
          if (h < Hi) {
            const float* qh = q + h * Di + 8 * i;
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
              const float prod = __fmul_rn(kv[rr], qh[rr]);
              pr[h][rr] = i == 0 ? prod : __fadd_rn(pr[h][rr], prod);
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < kHiFast; ++h) {
        if (h < Hi) {
          const float d = __fadd_rn(__fadd_rn(__fadd_rn(pr[h][0], pr[h][1]), __fadd_rn(pr[h][2], pr[h][3])),
                                    __fadd_rn(__fadd_rn(pr[h][4], pr[h][5]), __fadd_rn(pr[h][6], pr[h][7])));
          const float rl = d > 0.0f ? d : 0.0f;
          const float term = __fmul_rn(rl, w[h]);
          score = h == 0 ? term : __fadd_rn(score, term);
        }
      }
      out[j] = score;
      continue;
    }
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
    out[j] = score;
  }
}

// Block-wide exclusive prefix count of `flag` in thread order; returns the
// prefix for this thread and writes the block total to *total.
__device__ __forceinline__ int block_excl_count(bool flag, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(bal & ((1u << lane) - 1u));
  __syncthreads();
  if (lane == 0) wsum[w] = __popc(bal);
  __syncthreads();
  if (w == 0) {
    const int v = wsum[lane];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    wsum[lane] = incl - v;
    if (lane == 31) *total = incl;
  }
  __syncthreads();
  return wsum[w] + in_warp;
}

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(IndexerParams p, int nsort) {
  const int r = blockIdx.x, tid = threadIdx.x;
  int b, qp, iq_row;
  row_seq_pos(p, r, b, qp, iq_row);
  const int n = min(qp + 1, p.max_ctx);
  int32_t* out = p.sel_idx + (int64_t)r * p.sel_ld;
  if (n <= p.k) {
    for (int j = tid; j < n; j += kTopkThreads) out[j] = j;
    if (tid == 0) p.sel_cnt[r] = n;
    return;
  }
  extern __shared__ int list[];  // [nsort]
  __shared__ unsigned hist[256];
  __shared__ int wsum[32];
  __shared__ int s_total, s_cnt, s_digit, s_remaining;
  const float* sc = p.scores + (int64_t)r * p.max_ctx;

  uint32_t prefix = 0, mask = 0;
  int remaining = p.k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    for (int j = tid; j < n; j += kTopkThreads) {
      const uint32_t u = score_key(sc[j]);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns digits 255-8l .. 248-8l (descending)
      unsigned c8[8], sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c8[i] = hist[255 - 8 * tid - i];
        sum += c8[i];
      }
      unsigned incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += t;
      }
      const unsigned excl = incl - sum;
      const bool here = excl < (unsigned)remaining && incl >= (unsigned)remaining;
      if (here) {
        unsigned cum = excl;
        for (int i = 0; i < 8; ++i) {
          if (cum + c8[i] >= (unsigned)remaining) {
            s_digit = 255 - 8 * tid - i;
            s_remaining = remaining - (int)cum;
            break;
          }
          cum += c8[i];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s_digit << shift;
    mask |= 0xFFu << shift;
    remaining = s_remaining;
    __syncthreads();
  }
  const uint32_t thr = prefix;  // key of the k-th largest score
  const int need = remaining;   // keys equal to thr that are taken (>= 1)

  if (tid == 0) s_cnt = 0;
  __syncthreads();
  for (int j = tid; j < n; j += kTopkThreads)
    if (score_key(sc[j]) > thr) list[atomicAdd(&s_cnt, 1)] = j;
  __syncthreads();
  const int above = s_cnt;  // == k - need
  int taken = 0;
  for (int base = n - 1; base >= 0 && taken < need; base -= kTopkThreads) {
    const int j = base - tid;
    const bool flag = j >= 0 && score_key(sc[j]) == thr;
    const int rank = block_excl_count(flag, wsum, &s_total);
    if (flag && taken + rank < need) list[above + taken + rank] = j;
    taken += s_total;  // uniform across the block
    __syncthreads();
  }
  int cnt = p.k;
  if (score_key(sc[n - 1]) < thr) {  // the diagonal was not selected
    if (tid == 0) list[p.k] = n - 1;
    cnt = p.k + 1;
  }
  for (int i = cnt + tid; i < nsort; i += kTopkThreads) list[i] = 0x7fffffff;
  __syncthreads();
  // bitonic sort ascending
  for (int size = 2; size <= nsort; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < nsort / 2; i += kTopkThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const int a = list[lo], c = list[hi];
        if ((a > c) == up) {
          list[lo] = c;
          list[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < cnt; i += kTopkThreads) out[i] = list[i];
  if (tid == 0) p.sel_cnt[r] = cnt;
}

int launch_indexer_topk(const IndexerParams& p, cudaStream_t st) {
  if (p.Di % 8 || p.Di > kMaxDi || p.Hi > kMaxHi || p.Hi < 1 || p.k < 1 || p.rows <= 0) return CB_ERR_SHAPE;
  int nsort = 1;
  while (nsort < p.k + 1) nsort <<= 1;
  if (nsort > 16384) return CB_ERR_SHAPE;
  const int blocks_per_row = std::max(1, std::min(num_sms(), ceil_div(p.max_ctx, kScoreThreads)));
  indexer_score_kernel<<<dim3(blocks_per_row, p.rows), kScoreThreads, 0, st>>>(p);
  count_launch();
  if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
  if (ensure_smem_attr((const void*)topk_kernel, 64 * 1024) != CB_OK) return CB_ERR_CUDA;
  topk_kernel<<<p.rows, kTopkThreads, nsort * sizeof(int), st>>>(p, nsort);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb

using namespace cb;

extern "C" int cb_indexer_topk(const float* iq, const float* iw, int32_t ld_q, const uint8_t* ik, int32_t max_ctx,
                               int32_t Hi, int32_t Di, const int32_t* seq, const int32_t* qpos, int32_t rows, int32_t k,
                               float* scores, int32_t* sel_idx, int32_t* sel_cnt, void* stream) {
  if (!iq || !iw || !ik || !seq || !qpos || !scores || !sel_idx || !sel_cnt || rows <= 0 || k <= 0 || max_ctx <= 0)
    return CB_ERR_ARG;
  IndexerParams p{};
  p.iq = iq;
  p.iw = iw;
  p.ld_q = ld_q;
  p.ik = ik;
  p.ik_seq_stride = (int64_t)max_ctx * Di;
  p.Hi = Hi;
  p.Di = Di;
  p.max_ctx = max_ctx;
  p.seq_arr = seq;
  p.qpos_arr = qpos;
  p.rows = rows;
  p.k = k;
  p.scores = scores;
  p.sel_idx = sel_idx;
  p.sel_ld = k + 1;
  p.sel_cnt = sel_cnt;
  return launch_indexer_topk(p, (cudaStream_t)stream);
}

// ------------------------------------------------ no-allocation variant
// Score scratch owned by the library for cb_indexer_topk_noalloc, for callers
// that cannot allocate device memory.  In host code the name of this array is
// only a host-side stand-in, never a device address: the device address is
// looked up per device with cudaGetSymbolAddress (with that device current)
// and passed to the kernels.
static __device__ __align__(256) float g_noalloc_scores[CB_NOALLOC_MAX_SCORES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_addr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scores on the current device (looked up once per device).
int noalloc_scratch(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return CB_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_scores) != cudaSuccess || addr == nullptr) return CB_ERR_CUDA;
    g_noalloc_addr[dev] = static_cast<float*>(addr);
  }
  *out = g_noalloc_addr[dev];
  return CB_OK;
}
}  // namespace

extern "C" int cb_indexer_topk_noalloc(const float* iq, const float* iw, int32_t ld_q, const uint8_t* ik,
                                       int32_t max_ctx, int32_t Hi, int32_t Di, const int32_t* seq,
                                       const int32_t* qpos, int32_t rows, int32_t k, int32_t* sel_idx,
                                       int32_t* sel_cnt, void* stream) {
  if (!iq || !iw || !ik || !seq || !qpos || !sel_idx || !sel_cnt || rows <= 0 || k <= 0 || max_ctx <= 0)
    return CB_ERR_ARG;
  if ((int64_t)rows * max_ctx > (int64_t)CB_NOALLOC_MAX_SCORES) return CB_ERR_TOO_LARGE;
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != CB_OK) return rc;
  IndexerParams p{};
  p.iq = iq;
  p.iw = iw;
  p.ld_q = ld_q;
  p.ik = ik;
  p.ik_seq_stride = (int64_t)max_ctx * Di;
  p.Hi = Hi;
  p.Di = Di;
  p.max_ctx = max_ctx;
  p.seq_arr = seq;
  p.qpos_arr = qpos;
  p.rows = rows;
  p.k = k;
  p.scores = scratch;
  p.sel_idx = sel_idx;
  p.sel_ld = k + 1;
  p.sel_cnt = sel_cnt;
  return launch_indexer_topk(p, (cudaStream_t)stream);
}
