// Internal launch interface of the attention kernels (attn.cu) and the
// indexer / top-k kernels (indexer.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

// Per-token head preparation: q heads (RMSNorm + RoPE -> qout), k heads
// (RMSNorm + RoPE -> bf16 cache row), v heads (-> bf16 cache row) and
// optionally the indexer key (-> E4M3 cache row).
struct HeadPrepParams {
  const float* proj;
  int ldp;
  int T, c0;                 // rows b*T + t; position pos[b] + c0 + t
  const int32_t* pos;
  int Hq, Hkv, hd, rot2;     // rot2 = rotary pairs per head
  int off_q, off_k, off_v;
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;
  float eps;
  float* qout;               // [rows][Hq*hd] (unused when Hq == 0)
  int ldq;
  uint16_t* kdst;            // sequence 0 of the cache (ring or linear)
  uint16_t* vdst;
  int64_t seq_stride;        // elements between sequences in kdst / vdst
  int slots;                 // ring length (SWA) or max_ctx (shared)
  bool ring;                 // SWA ring (slot = position % slots) or linear (bounds-checked)
  int off_ik, Di;            // indexer key (Di == 0: none)
  uint8_t* ikdst;
  int64_t ik_seq_stride;
  int32_t* status;
};

// Sliding-window attention over the ring, split over key ranges.
struct SwaParams {
  const float* q;            // [rows][ldq] prepared queries
  int ldq;
  const uint16_t* kring;     // sequence 0 of this layer's ring
  const uint16_t* vring;
  int64_t seq_stride;
  int slots;
  const int32_t* pos;
  int T, c0;
  int Hq, Hkv, hd, window;
  int split_len, n_splits;
  float scale;
  float* part;               // [rows][Hq][n_splits][hd + 2]
  const float* gate;         // proj + off_gate (row stride ldg)
  int ldg;
  float* out;                // [rows][ldo]
  int ldo;
};

// Cross attention over the shared KV: selected keys (sparse) or all keys <= position (dense).
struct CrossParams {
  const float* proj;         // cross q | gate output, row r, stride ldp
  int ldp, off_gate;
  const float* q_norm;
  const float* inv_freq;
  int rot2;
  float eps, scale;
  const int32_t* pos;
  int c0, t_off, nq;         // row r -> sequence r / nq, position pos[b] + c0 + t_off + r % nq
  const uint16_t* kk;        // shared K, sequence 0
  const uint16_t* vv;
  int64_t seq_stride;
  int Hq, Hkv, hd;
  const int32_t* sel_idx;    // null -> dense
  const int32_t* sel_cnt;
  int sel_ld;
  int max_ctx;
  float* out;
  int ldo;
};

struct IndexerParams {
  const float* iq;           // query rows of the indexer projections
  const float* iw;
  int ld_q;
  int iq_T, iq_off;          // iq row of query row r: (r / nq) * iq_T + iq_off + r % nq
  const uint8_t* ik;         // sequence 0 of the E4M3 key cache
  int64_t ik_seq_stride;
  int Hi, Di, max_ctx;
  const int32_t* seq_arr;    // explicit mode: sequence and position of every row
  const int32_t* qpos_arr;
  const int32_t* pos;        // forward mode (seq_arr == null)
  int c0, t_off, nq;
  int rows, k;
  float* scores;             // [rows][max_ctx]
  int32_t* sel_idx;          // [rows][sel_ld]
  int sel_ld;
  int32_t* sel_cnt;
};

int launch_head_prep(const HeadPrepParams& p, int rows, cudaStream_t st);
int launch_swa(const SwaParams& p, int batch, cudaStream_t st);
// Prompt chunks: block-wise SWA (rows b * T + t), gated output straight into out.
int launch_swa_prefill(const SwaParams& p, int batch, cudaStream_t st);
bool swa_prefill_supported(int Hq, int Hkv, int hd);
// Steps of many query rows: one CTA per (KV head, row), lane groups over keys
// (SWA for one token per sequence, cross attention for any rows).
int launch_swa_decode(const SwaParams& p, int batch, cudaStream_t st);
int launch_cross_decode(const CrossParams& p, int rows, cudaStream_t st);
bool decode_attn_supported(int Hq, int Hkv, int hd);
int launch_cross(const CrossParams& p, int rows, cudaStream_t st);
int launch_indexer_topk(const IndexerParams& p, cudaStream_t st);

constexpr int kSwaSplit = 128;

}  // namespace cb
