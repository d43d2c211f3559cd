// Attention kernels of the decode step.
//
//  head_prep   q/k RMSNorm + partial interleaved RoPE, bf16 K/V cache append,
//              E4M3 indexer-key append        (layers.py:227-235, 265-279)
//  swa_attn    sliding-window attention over the ring, split over key ranges
//  swa_combine merges the splits, applies the sigmoid head gate (layers.py:243)
//  cross_attn  cross-decoder attention over the selected shared-KV rows
//              (layers.py:325-331) with the q norm/RoPE and head gate fused in
#include <algorithm>

#include "attn.cuh"
#include "common.cuh"

namespace cb {

// ------------------------------------------------------------- head prep
__global__ void __launch_bounds__(256) head_prep_kernel(HeadPrepParams p) {
  const int r = blockIdx.x, b = r / p.T, t = r % p.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int position = p.pos[b] + p.c0 + t;
  // a position outside the cache (context full, or a corrupted pos) writes nothing
  const bool linear_full = position < 0 || (!p.ring && position >= p.slots);
  if (linear_full && threadIdx.x == 0) set_status(p.status, CB_ERR_CTX_FULL);
  const int slot = position < 0 ? 0 : (p.ring ? position % p.slots : position);
  const float* row = p.proj + (int64_t)r * p.ldp;
  const int items = p.Hq + 2 * p.Hkv + (p.Di > 0 ? 1 : 0);
  const int npairs = p.hd / 2;
  for (int it = warp; it < items; it += 8) {
    if (it < p.Hq + p.Hkv) {
      const bool is_q = it < p.Hq;
      const int hh = is_q ? it : it - p.Hq;
      const float* x = row + (is_q ? p.off_q : p.off_k) + hh * p.hd;
      const float* nw = is_q ? p.q_norm : p.k_norm;
      float ss = 0.0f;
      for (int j = lane; j < npairs; j += 32) ss += x[2 * j] * x[2 * j] + x[2 * j + 1] * x[2 * j + 1];
      ss = warp_sum(ss);
      const float rn = rsqrtf(ss / (float)p.hd + p.eps);
      for (int j = lane; j < npairs; j += 32) {
        float x1 = x[2 * j] * rn * nw[2 * j];
        float x2 = x[2 * j + 1] * rn * nw[2 * j + 1];
        if (j < p.rot2) rope_pair(x1, x2, position, p.inv_freq[j]);
        if (is_q) {
          float* q = p.qout + (int64_t)r * p.ldq + hh * p.hd;
          q[2 * j] = x1;
          q[2 * j + 1] = x2;
        } else if (!linear_full) {
          uint16_t* k = p.kdst + (int64_t)b * p.seq_stride + ((int64_t)slot * p.Hkv + hh) * p.hd;
          k[2 * j] = f32_to_bf16(x1);
          k[2 * j + 1] = f32_to_bf16(x2);
        }
      }
    } else if (it < p.Hq + 2 * p.Hkv) {
      if (linear_full) continue;
      const int hh = it - p.Hq - p.Hkv;
      const float* x = row + p.off_v + hh * p.hd;
      uint16_t* v = p.vdst + (int64_t)b * p.seq_stride + ((int64_t)slot * p.Hkv + hh) * p.hd;
      for (int d = lane; d < p.hd; d += 32) v[d] = f32_to_bf16(x[d]);
    } else {
      if (linear_full) continue;
      const float* x = row + p.off_ik;
      uint8_t* ik = p.ikdst + (int64_t)b * p.ik_seq_stride + (int64_t)slot * p.Di;
      for (int d = lane; d < p.Di; d += 32) ik[d] = f32_to_e4m3(x[d]);
    }
  }
}

int launch_head_prep(const HeadPrepParams& p, int rows, cudaStream_t st) {
  if (p.hd % 2 || p.hd > 256) return CB_ERR_SHAPE;
  head_prep_kernel<<<rows, 256, 0, st>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// ------------------------------------------------------------------ SWA
constexpr int kSwaThreads = 128;

__global__ void __launch_bounds__(kSwaThreads) swa_attn_kernel(SwaParams p) {
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int hd = p.hd, G = p.Hq / p.Hkv, L = p.split_len;
  extern __shared__ __align__(16) float sm[];
  float* Ks = sm;                            // [L][hd + 1]
  float* Vs = Ks + L * (hd + 1);             // [L][hd]
  float* qsh = Vs + L * hd;                  // [hd]
  float* es = qsh + hd;                      // [L]
  float* ored = es + L;                      // [kSwaThreads]
  __shared__ float red[33];

  const int p0 = p.pos[b] + p.c0;
  const int lo = max(0, p0 - p.window + 1), last = p0 + p.T - 1;
  const int ks = lo + s * L, ke = min(ks + L, last + 1);
  const int n = ke - ks;

  auto part_ptr = [&](int t, int qh) {
    return p.part + ((((int64_t)b * p.T + t) * p.Hq + qh) * p.n_splits + s) * (hd + 2);
  };
  if (n <= 0) {
    for (int t = 0; t < p.T; ++t)
      for (int j = 0; j < G; ++j) {
        float* pp = part_ptr(t, g * G + j);
        for (int d = tid; d < hd + 2; d += kSwaThreads) pp[d] = d == 0 ? -INFINITY : 0.0f;
      }
    return;
  }
  const uint16_t* kr = p.kring + (int64_t)b * p.seq_stride;
  const uint16_t* vr = p.vring + (int64_t)b * p.seq_stride;
  // the split's K/V rows: 16-byte vectors, four of each in flight per thread
  const int vpk = hd / 8, nv = n * vpk;
  for (int i0 = tid; i0 < nv; i0 += 4 * kSwaThreads) {
    uint4 kq[4], vq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j * kSwaThreads;
      if (i < nv) {
        const int key = i / vpk, e8 = (i - key * vpk) * 8;
        const int64_t off = ((int64_t)((ks + key) % p.slots) * p.Hkv + g) * hd + e8;
        kq[j] = *reinterpret_cast<const uint4*>(kr + off);
        vq[j] = *reinterpret_cast<const uint4*>(vr + off);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j * kSwaThreads;
      if (i < nv) {
        const int key = i / vpk, e8 = (i - key * vpk) * 8;
        const uint32_t kw[4] = {kq[j].x, kq[j].y, kq[j].z, kq[j].w}, vw[4] = {vq[j].x, vq[j].y, vq[j].z, vq[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          Ks[key * (hd + 1) + e8 + 2 * e] = bf16_to_f32(kw[e]);
          Ks[key * (hd + 1) + e8 + 2 * e + 1] = bf16_to_f32(kw[e] >> 16);
          Vs[key * hd + e8 + 2 * e] = bf16_to_f32(vw[e]);
          Vs[key * hd + e8 + 2 * e + 1] = bf16_to_f32(vw[e] >> 16);
        }
      }
    }
  }
  __syncthreads();

  for (int t = 0; t < p.T; ++t) {
    const int pt = p0 + t;
    for (int j = 0; j < G; ++j) {
      const int qh = g * G + j;
      const float* qrow = p.q + ((int64_t)b * p.T + t) * p.ldq + qh * hd;
      for (int d = tid; d < hd; d += kSwaThreads) qsh[d] = qrow[d];
      __syncthreads();
      float sc = -INFINITY;
      if (tid < n) {
        const int kp = ks + tid;
        if (kp <= pt && kp > pt - p.window) {
          float acc = 0.0f;
          const float* kk = Ks + tid * (hd + 1);
          for (int d = 0; d < hd; ++d) acc = fmaf(qsh[d], kk[d], acc);
          sc = acc * p.scale;
        }
      }
      const float m = block_max(sc, red);
      float* pp = part_ptr(t, qh);
      if (m == -INFINITY) {
        for (int d = tid; d < hd + 2; d += kSwaThreads) pp[d] = d == 0 ? -INFINITY : 0.0f;
        __syncthreads();
        continue;
      }
      const float e = sc == -INFINITY ? 0.0f : expf(sc - m);
      if (tid < L) es[tid] = e;
      const float l = block_sum(e, red);
      // o[d] = sum_i e_i V[i][d]; kSwaThreads / hd groups of keys
      const int groups = kSwaThreads / hd;
      float o = 0.0f;
      const int d = tid % hd, grp = tid / hd;
      if (grp < groups)
        for (int i = grp; i < n; i += groups) o = fmaf(es[i], Vs[i * hd + d], o);
      ored[tid] = o;
      __syncthreads();
      if (tid < hd) {
        float acc = 0.0f;
        for (int q2 = 0; q2 < groups; ++q2) acc += ored[q2 * hd + tid];
        pp[2 + tid] = acc;
      }
      if (tid == 0) {
        pp[0] = m;
        pp[1] = l;
      }
      __syncthreads();
    }
  }
}

__global__ void swa_combine_kernel(SwaParams p) {
  const int r = blockIdx.x;
  const int hd = p.hd;
  for (int i = threadIdx.x; i < p.Hq * hd; i += blockDim.x) {
    const int qh = i / hd, d = i - qh * hd;
    const float* base = p.part + ((int64_t)r * p.Hq + qh) * p.n_splits * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < p.n_splits; ++s) M = fmaxf(M, base[s * (hd + 2)]);
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < p.n_splits; ++s) {
      const float ms = base[s * (hd + 2)];
      if (ms == -INFINITY) continue;
      const float w = expf(ms - M);
      L += base[s * (hd + 2) + 1] * w;
      O += base[s * (hd + 2) + 2 + d] * w;
    }
    const float gate = sigmoid(p.gate[(int64_t)r * p.ldg + qh]);
    p.out[(int64_t)r * p.ldo + qh * hd + d] = (O / L) * gate;
  }
}

int launch_swa(const SwaParams& p, int batch, cudaStream_t st) {
  if (p.hd > kSwaThreads || kSwaThreads % p.hd || p.hd % 8 || p.split_len != kSwaSplit) return CB_ERR_SHAPE;
  const size_t smem = sizeof(float) * ((size_t)p.split_len * (2 * p.hd + 1) + p.hd + p.split_len + kSwaThreads);
  if (ensure_smem_attr((const void*)swa_attn_kernel, 160 * 1024) != CB_OK) return CB_ERR_CUDA;
  swa_attn_kernel<<<dim3(p.n_splits, p.Hkv, batch), kSwaThreads, smem, st>>>(p);
  count_launch();
  if (cudaGetLastError() != cudaSuccess) return CB_ERR_CUDA;
  swa_combine_kernel<<<batch * p.T, std::min(1024, p.Hq * p.hd), 0, st>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// ------------------------------------------------------- decode attention, many rows
// One query token: one CTA per (KV head, query row), 8 warps over the keys.
// In a warp, groups of hd/8 lanes take one key each (a lane owns 8 dimensions:
// one 16-byte K load and one V load per key), so a warp reads 32 x 16 bytes of
// K and of V per step; each group keeps a running (max, sum, o) per query head
// of the KV head, and the groups, then the warps, are merged in a fixed order.
// Scores are partial dot products summed over the group's lanes by shuffles.
constexpr int kSdThreads = 256;
constexpr int kSdMaxG = 4;

// Keys key_of(i) for i < n of this CTA's (KV head g, row) against qs [G][hd]
// (already scaled), into out[row][(g * G + j) * hd + d] = o / l * sigmoid(gate[j]).
template <typename KeyOf>
__device__ __forceinline__ void decode_attend(const float* qs, int G, int hd, int g, int Hkv, int n, KeyOf key_of,
                                              const uint16_t* kr, const uint16_t* vr, const float* gate, float* out) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int LK = hd / 8, KG = 32 / LK, kg = lane / LK, sub = lane - kg * LK;
  const int k0 = warp * n / (kSdThreads / 32), k1 = (warp + 1) * n / (kSdThreads / 32);
  float q[kSdMaxG][8], o[kSdMaxG][8], m[kSdMaxG], l[kSdMaxG];
#pragma unroll
  for (int j = 0; j < kSdMaxG; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      q[j][e] = j < G ? qs[j * hd + sub * 8 + e] : 0.0f;
      o[j][e] = 0.0f;
    }
  }
  for (int kb = k0; kb < k1; kb += KG) {
    const int i = kb + kg;
    const bool valid = i < k1;
    uint4 kq = make_uint4(0u, 0u, 0u, 0u), vq = kq;
    if (valid) {
      const int64_t off = ((int64_t)key_of(i) * Hkv + g) * hd + sub * 8;
      kq = *reinterpret_cast<const uint4*>(kr + off);
      vq = *reinterpret_cast<const uint4*>(vr + off);
    }
    const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, vw[4] = {vq.x, vq.y, vq.z, vq.w};
    float kf[8], vf[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      kf[2 * e] = bf16_to_f32(kw[e]);
      kf[2 * e + 1] = bf16_to_f32(kw[e] >> 16);
      vf[2 * e] = bf16_to_f32(vw[e]);
      vf[2 * e + 1] = bf16_to_f32(vw[e] >> 16);
    }
#pragma unroll
    for (int j = 0; j < kSdMaxG; ++j) {
      if (j < G) {
        float sc = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) sc = fmaf(q[j][e], kf[e], sc);
        for (int off = LK / 2; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
        if (valid) {
          const float mn = fmaxf(m[j], sc);
          const float c = m[j] == -INFINITY ? 0.0f : expf(m[j] - mn);
          const float pe = expf(sc - mn);
          l[j] = l[j] * c + pe;
#pragma unroll
          for (int e = 0; e < 8; ++e) o[j][e] = fmaf(pe, vf[e], o[j][e] * c);
          m[j] = mn;
        }
      }
    }
  }
  // merge the key groups of the warp (lanes sub, sub + LK, ...), then the warps
  for (int off = LK; off < 32; off <<= 1) {
#pragma unroll
    for (int j = 0; j < kSdMaxG; ++j) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m[j], off), l2 = __shfl_xor_sync(0xffffffffu, l[j], off);
      const float mn = fmaxf(m[j], m2);
      const float c1 = m[j] == -INFINITY ? 0.0f : expf(m[j] - mn), c2 = m2 == -INFINITY ? 0.0f : expf(m2 - mn);
      l[j] = l[j] * c1 + l2 * c2;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float o2 = __shfl_xor_sync(0xffffffffu, o[j][e], off);
        o[j][e] = o[j][e] * c1 + o2 * c2;
      }
      m[j] = mn;
    }
  }
  __shared__ float wm[kSdThreads / 32][kSdMaxG], wl[kSdThreads / 32][kSdMaxG];
  __shared__ float wo[kSdThreads / 32][kSdMaxG][256];
  if (kg == 0) {
#pragma unroll
    for (int j = 0; j < kSdMaxG; ++j) {
      if (sub == 0) {
        wm[warp][j] = m[j];
        wl[warp][j] = l[j];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) wo[warp][j][sub * 8 + e] = o[j][e];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += kSdThreads) {
    const int j = i / hd, d = i - j * hd;
    float M = -INFINITY;
    for (int w = 0; w < kSdThreads / 32; ++w) M = fmaxf(M, wm[w][j]);
    float L = 0.0f, O = 0.0f;
    for (int w = 0; w < kSdThreads / 32; ++w) {
      if (wm[w][j] == -INFINITY) continue;
      const float c = expf(wm[w][j] - M);
      L += wl[w][j] * c;
      O += wo[w][j][d] * c;
    }
    out[(g * G + j) * hd + d] = (O / L) * sigmoid(gate[g * G + j]);
  }
}

bool decode_attn_supported(int Hq, int Hkv, int hd) {
  const int G = Hkv > 0 ? Hq / Hkv : 0;
  return hd >= 8 && hd <= 256 && hd % 8 == 0 && 32 % (hd / 8) == 0 && G >= 1 && G <= kSdMaxG && G * Hkv == Hq;
}

// SWA, one token per sequence: the window's keys (positions, ring slots).
__global__ void __launch_bounds__(kSdThreads) swa_decode_kernel(SwaParams p) {
  const int g = blockIdx.x, b = blockIdx.y;
  const int hd = p.hd, G = p.Hq / p.Hkv;
  __shared__ float qs[kSdMaxG * 256];
  const float* qrow = p.q + (int64_t)b * p.ldq;
  for (int i = threadIdx.x; i < G * hd; i += kSdThreads) qs[i] = qrow[g * G * hd + i] * p.scale;
  __syncthreads();
  const int P0 = p.pos[b] + p.c0;
  const int lo = max(0, P0 - p.window + 1), slots = p.slots;
  decode_attend(qs, G, hd, g, p.Hkv, P0 - lo + 1, [&](int i) { return (lo + i) % slots; },
                p.kring + (int64_t)b * p.seq_stride, p.vring + (int64_t)b * p.seq_stride,
                p.gate + (int64_t)b * p.ldg, p.out + (int64_t)b * p.ldo);
}

int launch_swa_decode(const SwaParams& p, int batch, cudaStream_t st) {
  if (!decode_attn_supported(p.Hq, p.Hkv, p.hd) || p.T != 1) return CB_ERR_SHAPE;
  swa_decode_kernel<<<dim3(p.Hkv, batch), kSdThreads, 0, st>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// Cross attention of one query row over its selected keys (or all keys at or
// before its position when dense), q RMSNorm + RoPE and the head gate fused.
__global__ void __launch_bounds__(kSdThreads) cross_decode_kernel(CrossParams p) {
  const int g = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int hd = p.hd, G = p.Hq / p.Hkv, warp = tid >> 5, lane = tid & 31;
  const int b = r / p.nq, j0 = r % p.nq;
  const int position = p.pos[b] + p.c0 + p.t_off + j0;
  __shared__ float qs[kSdMaxG * 256];
  const float* row = p.proj + (int64_t)r * p.ldp;
  for (int j = warp; j < G; j += kSdThreads / 32) {
    const float* x = row + (g * G + j) * hd;
    float ss = 0.0f;
    for (int d = lane; d < hd; d += 32) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float rn = rsqrtf(ss / (float)hd + p.eps);
    for (int jj = lane; jj < hd / 2; jj += 32) {
      float x1 = x[2 * jj] * rn * p.q_norm[2 * jj];
      float x2 = x[2 * jj + 1] * rn * p.q_norm[2 * jj + 1];
      if (jj < p.rot2) rope_pair(x1, x2, position, p.inv_freq[jj]);
      qs[j * hd + 2 * jj] = x1 * p.scale;
      qs[j * hd + 2 * jj + 1] = x2 * p.scale;
    }
  }
  __syncthreads();
  const bool dense = p.sel_idx == nullptr;
  const int n = dense ? max(0, min(position + 1, p.max_ctx)) : min(p.sel_cnt[r], p.sel_ld);
  const int32_t* sel = dense ? nullptr : p.sel_idx + (int64_t)r * p.sel_ld;
  decode_attend(qs, G, hd, g, p.Hkv, n, [&](int i) { return dense ? i : sel[i]; }, p.kk + (int64_t)b * p.seq_stride,
                p.vv + (int64_t)b * p.seq_stride, row + p.off_gate, p.out + (int64_t)r * p.ldo);
}

int launch_cross_decode(const CrossParams& p, int rows, cudaStream_t st) {
  if (!decode_attn_supported(p.Hq, p.Hkv, p.hd)) return CB_ERR_SHAPE;
  cross_decode_kernel<<<dim3(p.Hkv, rows), kSdThreads, 0, st>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// ------------------------------------------------------------- SWA prefill
// Block-wise sliding-window attention for a prompt chunk (the reference's
// _sliding_window_attend, layers.py:195-210, over the ring instead of a padded
// key tensor).  One CTA takes kSpQ consecutive tokens of one sequence and the
// G query heads of one KV head (rows r = t * G + j) and walks the keys of their
// windows 64 at a time with a running (max, sum) per row:
//   S = q K^T * scale (masked to 0 <= pos - key < window), m' = max(m, max S),
//   p = exp(S - m'), l = l e^{m - m'} + sum p, o = o e^{m - m'} + p V,
// then writes o / l times the head gate sigmoid(gate) (layers.py:243).  The
// chunk's own keys are already in the ring, which must hold window + T - 1
// positions so that no key a query of the chunk needs is overwritten.
constexpr int kSpThreads = 256;
constexpr int kSpQ = 8;      // tokens per CTA
constexpr int kSpKeys = 64;  // keys per tile
constexpr int kSpMaxRows = kSpQ * 4;  // G <= 4 query heads per KV head

// PER = output rows per thread (kSpMaxRows * hd / kSpThreads)
template <int PER>
__global__ void __launch_bounds__(kSpThreads) swa_prefill_kernel(SwaParams p) {
  const int qb = blockIdx.x, g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int hd = p.hd, G = p.Hq / p.Hkv;
  const int t0 = qb * kSpQ, nq = min(kSpQ, p.T - t0), rows = nq * G;
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;                           // [rows][hd]
  float* Ks = Qs + kSpMaxRows * hd;         // [kSpKeys][hd + 1]
  float* Vs = Ks + kSpKeys * (hd + 1);      // [kSpKeys][hd]
  float* Ps = Vs + kSpKeys * hd;            // [rows][kSpKeys + 1]
  __shared__ float m_run[kSpMaxRows], l_run[kSpMaxRows], corr[kSpMaxRows];
  const int P0 = p.pos[b] + p.c0 + t0;      // position of the block's first token
  const int klo = max(0, P0 - p.window + 1), khi = P0 + nq - 1;
  for (int i = tid; i < rows * hd; i += kSpThreads) {
    const int r = i / hd, d = i - r * hd, t = r / G, j = r - t * G;
    Qs[i] = p.q[((int64_t)b * p.T + t0 + t) * p.ldq + (g * G + j) * hd + d];
  }
  for (int r = tid; r < rows; r += kSpThreads) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.0f;
  }
  // output accumulators: column d, rows rg, rg + groups, ...
  const int groups = kSpThreads / hd, d = tid % hd, rg = tid / hd;
  constexpr int kMaxPer = PER;
  float o[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) o[i] = 0.0f;
  const uint16_t* kr = p.kring + (int64_t)b * p.seq_stride;
  const uint16_t* vr = p.vring + (int64_t)b * p.seq_stride;
  const int warp = tid >> 5, lane = tid & 31, vpk = hd / 8;
  // K/V tiles: the next tile's 16-byte vectors are loaded into registers while
  // the current tile is processed, then converted into shared memory
  constexpr int kSpLd = kSpKeys * 16 / kSpThreads;  // vectors per thread (head_dim <= 128)
  uint4 pk[kSpLd], pv[kSpLd];
  auto fetch = [&](int kt) {
    const int nn = min(kSpKeys, khi + 1 - kt);
#pragma unroll
    for (int e = 0; e < kSpLd; ++e) {
      const int i = tid + e * kSpThreads;
      if (kt <= khi && i < nn * vpk) {
        const int key = i / vpk, e8 = (i - key * vpk) * 8;
        const int64_t off = ((int64_t)((kt + key) % p.slots) * p.Hkv + g) * hd + e8;
        pk[e] = *reinterpret_cast<const uint4*>(kr + off);
        pv[e] = *reinterpret_cast<const uint4*>(vr + off);
      }
    }
  };
  fetch(klo);
  for (int kt0 = klo; kt0 <= khi; kt0 += kSpKeys) {
    const int n = min(kSpKeys, khi + 1 - kt0);
    __syncthreads();  // the previous tile's K, V and P are consumed
#pragma unroll
    for (int e = 0; e < kSpLd; ++e) {
      const int i = tid + e * kSpThreads;
      if (i < n * vpk) {
        const int key = i / vpk, e8 = (i - key * vpk) * 8;
        const uint32_t kw[4] = {pk[e].x, pk[e].y, pk[e].z, pk[e].w}, vw[4] = {pv[e].x, pv[e].y, pv[e].z, pv[e].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          Ks[key * (hd + 1) + e8 + 2 * q] = bf16_to_f32(kw[q]);
          Ks[key * (hd + 1) + e8 + 2 * q + 1] = bf16_to_f32(kw[q] >> 16);
          Vs[key * hd + e8 + 2 * q] = bf16_to_f32(vw[q]);
          Vs[key * hd + e8 + 2 * q + 1] = bf16_to_f32(vw[q] >> 16);
        }
      }
    }
    __syncthreads();
    fetch(kt0 + kSpKeys);
    // scores: thread (key j, rows r0, r0 + 4, ...)
    {
      const int j = tid & (kSpKeys - 1), kp = kt0 + j;
      for (int r = tid >> 6; r < rows; r += kSpThreads / kSpKeys) {
        const int qp = P0 + r / G;
        float sc = -INFINITY;
        if (j < n && kp <= qp && kp > qp - p.window) {
          const float* qq = Qs + r * hd;
          const float* kk = Ks + j * (hd + 1);
          float acc = 0.0f;
          for (int e = 0; e < hd; ++e) acc = fmaf(qq[e], kk[e], acc);
          sc = acc * p.scale;
        }
        Ps[r * (kSpKeys + 1) + j] = sc;
      }
    }
    __syncthreads();
    // running max / sum per row (a warp per row)
    for (int r = warp; r < rows; r += kSpThreads / 32) {
      float* pr = Ps + r * (kSpKeys + 1);
      const float s0 = pr[lane], s1 = pr[lane + 32];
      const float mt = warp_max(fmaxf(s0, s1));
      const float mo = m_run[r], mn = fmaxf(mo, mt);
      const float e0 = s0 == -INFINITY ? 0.0f : expf(s0 - mn), e1 = s1 == -INFINITY ? 0.0f : expf(s1 - mn);
      const float ls = warp_sum(e0 + e1);
      pr[lane] = e0;
      pr[lane + 32] = e1;
      if (lane == 0) {
        const float c = mo == -INFINITY ? 0.0f : expf(mo - mn);
        corr[r] = c;
        l_run[r] = l_run[r] * c + ls;
        m_run[r] = mn;
      }
    }
    __syncthreads();
    // o = o * corr + P V
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int r = rg + i * groups;
      if (r < rows) {
        const float* pr = Ps + r * (kSpKeys + 1);
        float acc = o[i] * corr[r];
        for (int jj = 0; jj < n; ++jj) acc = fmaf(pr[jj], Vs[jj * hd + d], acc);
        o[i] = acc;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int r = rg + i * groups;
    if (r < rows) {
      const int t = r / G, j = r - t * G, qh = g * G + j;
      const int64_t row = (int64_t)b * p.T + t0 + t;
      const float gate = sigmoid(p.gate[row * p.ldg + qh]);
      p.out[row * p.ldo + qh * hd + d] = (o[i] / l_run[r]) * gate;
    }
  }
}

bool swa_prefill_supported(int Hq, int Hkv, int hd) {
  const int G = Hkv > 0 ? Hq / Hkv : 0;
  return hd >= 8 && hd <= 128 && kSpThreads % hd == 0 && hd % 8 == 0 && (kSpMaxRows * hd) % kSpThreads == 0 &&
         G >= 1 && G <= 4 && G * Hkv == Hq;
}

int launch_swa_prefill(const SwaParams& p, int batch, cudaStream_t st) {
  if (!swa_prefill_supported(p.Hq, p.Hkv, p.hd)) return CB_ERR_SHAPE;
  if (p.slots < p.window + p.T - 1) return CB_ERR_SHAPE;  // the chunk would overwrite keys it still needs
  const size_t smem =
      sizeof(float) * ((size_t)kSpMaxRows * p.hd + (size_t)kSpKeys * (2 * p.hd + 1) + (size_t)kSpMaxRows * (kSpKeys + 1));
  const dim3 grid(ceil_div(p.T, kSpQ), p.Hkv, batch);
  const int per = kSpMaxRows * p.hd / kSpThreads;
#define CB_SP_CASE(N)                                                                              \
  case N:                                                                                          \
    if (ensure_smem_attr((const void*)swa_prefill_kernel<N>, (int)smem) != CB_OK) return CB_ERR_CUDA; \
    swa_prefill_kernel<N><<<grid, kSpThreads, smem, st>>>(p);                                      \
    break;
  switch (per) {
    CB_SP_CASE(1)
    CB_SP_CASE(2)
    CB_SP_CASE(4)
    CB_SP_CASE(8)
    CB_SP_CASE(16)
    CB_SP_CASE(32)
    default:
      return CB_ERR_SHAPE;
  }
#undef CB_SP_CASE
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

// ---------------------------------------------------------- cross attention
constexpr int kCrossThreads = 256;
constexpr int kCrossChunk = 256;
constexpr int kCrossMaxG = 8;

__global__ void __launch_bounds__(kCrossThreads) cross_attn_kernel(CrossParams p) {
  const int g = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int hd = p.hd, G = p.Hq / p.Hkv;
  const int warp = tid >> 5, lane = tid & 31;
  const int b = r / p.nq, j0 = r % p.nq;
  const int position = p.pos[b] + p.c0 + p.t_off + j0;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                          // [G][hd]
  float* es = qs + G * hd;                 // [G][kCrossChunk]
  const int kvld = hd + 8;                 // bf16 row stride of the staged rows (16-byte vector reads spread over banks)
  uint16_t* Kc = reinterpret_cast<uint16_t*>(es + G * kCrossChunk);  // [kCrossChunk][kvld]
  uint16_t* Vc = Kc + kCrossChunk * kvld;                             // [kCrossChunk][kvld]
  __shared__ int keys[kCrossChunk];
  __shared__ float red[33];
  __shared__ float mrun[kCrossMaxG], lrun[kCrossMaxG], corr[kCrossMaxG];

  // q: RMSNorm (q_norm) + RoPE per head of this KV group
  const float* row = p.proj + (int64_t)r * p.ldp;
  for (int j = warp; j < G; j += kCrossThreads / 32) {
    const float* x = row + (g * G + j) * hd;
    float ss = 0.0f;
    for (int d = lane; d < hd; d += 32) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float rn = rsqrtf(ss / (float)hd + p.eps);
    for (int jj = lane; jj < hd / 2; jj += 32) {
      float x1 = x[2 * jj] * rn * p.q_norm[2 * jj];
      float x2 = x[2 * jj + 1] * rn * p.q_norm[2 * jj + 1];
      if (jj < p.rot2) rope_pair(x1, x2, position, p.inv_freq[jj]);
      qs[j * hd + 2 * jj] = x1;
      qs[j * hd + 2 * jj + 1] = x2;
    }
  }
  if (tid < G) {
    mrun[tid] = -INFINITY;
    lrun[tid] = 0.0f;
  }
  const bool dense = p.sel_idx == nullptr;
  const int n = dense ? max(0, min(position + 1, p.max_ctx)) : min(p.sel_cnt[r], p.sel_ld);
  const uint16_t* kb = p.kk + (int64_t)b * p.seq_stride;
  const uint16_t* vb = p.vv + (int64_t)b * p.seq_stride;
  // each thread accumulates up to two (head, dim) outputs
  float o_acc[2] = {0.0f, 0.0f};
  __syncthreads();

  for (int c = 0; c < n; c += kCrossChunk) {
    const int cn = min(kCrossChunk, n - c);
    if (tid < cn) keys[tid] = dense ? c + tid : p.sel_idx[(int64_t)r * p.sel_ld + c + tid];
    __syncthreads();
    // the chunk's K/V rows into shared memory: 16-byte vectors, four of each in flight per thread
    const int vpk = hd / 8, nv = cn * vpk;
    for (int i0 = tid; i0 < nv; i0 += 4 * kCrossThreads) {
      uint4 kq[4], vq[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * kCrossThreads;
        if (i < nv) {
          const int key = i / vpk, e8 = (i - key * vpk) * 8;
          const int64_t src = ((int64_t)keys[key] * p.Hkv + g) * hd + e8;
          kq[j] = *reinterpret_cast<const uint4*>(kb + src);
          vq[j] = *reinterpret_cast<const uint4*>(vb + src);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j * kCrossThreads;
        if (i < nv) {
          const int key = i / vpk, e8 = (i - key * vpk) * 8;
          *reinterpret_cast<uint4*>(Kc + key * kvld + e8) = kq[j];
          *reinterpret_cast<uint4*>(Vc + key * kvld + e8) = vq[j];
        }
      }
    }
    __syncthreads();
    // scores for this chunk
    for (int i = tid; i < cn; i += kCrossThreads) {
      const uint16_t* kr = Kc + i * kvld;
      float acc[kCrossMaxG];
#pragma unroll
      for (int j = 0; j < kCrossMaxG; ++j) acc[j] = 0.0f;
      for (int d = 0; d < hd; d += 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kr + d);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          kf[2 * e] = bf16_to_f32(w[e]);
          kf[2 * e + 1] = bf16_to_f32(w[e] >> 16);
        }
#pragma unroll
        for (int j = 0; j < kCrossMaxG; ++j)
          if (j < G)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[j] = fmaf(qs[j * hd + d + e], kf[e], acc[j]);
      }
      for (int j = 0; j < G; ++j) es[j * kCrossChunk + i] = acc[j] * p.scale;
    }
    __syncthreads();
    // running max / sum per head
    for (int j = 0; j < G; ++j) {
      const float v = tid < cn ? es[j * kCrossChunk + tid] : -INFINITY;
      const float cm = block_max(v, red);
      const float mnew = fmaxf(mrun[j], cm);
      const float e = tid < cn ? expf(v - mnew) : 0.0f;
      if (tid < cn) es[j * kCrossChunk + tid] = e;
      const float cs = block_sum(e, red);
      if (tid == 0) {
        corr[j] = mrun[j] == -INFINITY ? 0.0f : expf(mrun[j] - mnew);
        lrun[j] = lrun[j] * corr[j] + cs;
        mrun[j] = mnew;
      }
      __syncthreads();
    }
    // o[j][d] += sum_i e[j][i] * V[key_i][g][d]
#pragma unroll
    for (int q2 = 0; q2 < 2; ++q2) {
      const int idx = tid + q2 * kCrossThreads;
      if (idx < G * hd) {
        const int j = idx / hd, d = idx - j * hd;
        float acc = o_acc[q2] * corr[j];
        const float* ej = es + j * kCrossChunk;
        for (int i = 0; i < cn; ++i) acc = fmaf(ej[i], bf16_to_f32(Vc[i * kvld + d]), acc);
        o_acc[q2] = acc;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int q2 = 0; q2 < 2; ++q2) {
    const int idx = tid + q2 * kCrossThreads;
    if (idx < G * hd) {
      const int j = idx / hd, d = idx - j * hd;
      const int qh = g * G + j;
      const float gate = sigmoid(row[p.off_gate + qh]);
      p.out[(int64_t)r * p.ldo + qh * hd + d] = (o_acc[q2] / lrun[j]) * gate;
    }
  }
}

int launch_cross(const CrossParams& p, int rows, cudaStream_t st) {
  const int G = p.Hq / p.Hkv;
  if (G > kCrossMaxG || G * p.hd > 2 * kCrossThreads || p.hd % 8) return CB_ERR_SHAPE;
  const size_t smem = sizeof(float) * ((size_t)G * p.hd + (size_t)G * kCrossChunk) +
                      sizeof(uint16_t) * 2 * kCrossChunk * (size_t)(p.hd + 8);
  if (smem > 200 * 1024) return CB_ERR_SHAPE;
  if (ensure_smem_attr((const void*)cross_attn_kernel, 200 * 1024) != CB_OK) return CB_ERR_CUDA;
  cross_attn_kernel<<<dim3(p.Hkv, rows), kCrossThreads, smem, st>>>(p);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

}  // namespace cb
