// Persistent decode kernel: launch interface (decode_mk.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

constexpr int kMkThreads = 512;
constexpr int kMkCluster = 8;          // CTAs per thread-block cluster
constexpr int kMkMaxClusters = 18;     // 144 CTAs at most
constexpr int kMkSlotBytes = 56 * 1024;   // two weight-staging slots (8 tiles of K = 768 each)
constexpr int kMkWorkBytes = 108 * 1024;  // per-phase working memory, parameter region at its end
constexpr int kMkHistBins = 2048;      // top 11 bits of the score key
constexpr int kMkSwaSplit = 80;        // window keys per SWA work item (and key chunk of cross attention)
constexpr int kMkCrossSplit = 64;      // selected keys per cross-attention work item
constexpr int kMkMaxRows = 8;          // batch * T handled by one persistent launch
constexpr int kMkMaxQ = 24;            // (q heads per KV head) * T per attention work item
constexpr int kMkMaxD = 1024;          // d_model and every GEMV K the kernel stages
constexpr int kMkTrace = 512;          // phase timestamps
constexpr unsigned long long kDefaultWaitNs = 200ull * 1000 * 1000;  // bounded-wait limit when none is set

// The first bytes of a cb_forward workspace: the device status word and the
// control words that cb_set_wait_limit writes (zero = defaults).
struct WaitCtl {
  int32_t status;               // CB_OK or the first device-side error
  int32_t stall_barrier;        // > 0: CTA 0 skips its arrival at this barrier (fault injection for tests)
  unsigned long long limit_ns;  // limit of every bounded wait of the persistent kernel; 0 = kDefaultWaitNs
};

// Everything one persistent launch needs, passed by value (__grid_constant__).
struct MkArgs {
  CbModel m;
  CbCache c;
  // workspace
  long long* hq;     // [M][d] self-decoder residual stream, fixed point (value * 2^32)
  long long* xq;     // [RQ][d] cross-decoder residual stream, fixed point
  float* proj;       // [M][ldp] in-projection outputs (SWA, shared KV)
  float* act;        // unused scratch kept for the workspace layout
  float* cproj;      // [RQ][cr_ld]
  float* part;       // SWA partials [M][Hq][swa_splits][hd + 2]
  float* part2;      // cross partials [RQ][Hq][cross_splits][hd + 2]
  float* scores;     // [RQ][max_ctx]
  float* ws_logits;  // [RQ][vocab] when the caller passes no logits buffer
  unsigned* hist;    // [RQ][kMkHistBins]
  int32_t* hi_list;  // [RQ][k]  keys above the threshold bin
  int32_t* hi_cnt;   // [RQ]
  unsigned long long* cand;  // [RQ][max_ctx]  (key << 32 | index) in the threshold bin
  int32_t* cand_cnt; // [RQ]
  int32_t* sel_idx;  // [RQ][sel_ld]
  int32_t* sel_cnt;  // [RQ]
  unsigned long long* amax;  // [RQ] packed argmax
  unsigned* sync;    // grid barrier counter (zeroed before every launch)
  unsigned long long* trace;  // [kMkTrace] phase timestamps of CTA 0
  int32_t* status;
  int ldp, att_ld, cr_ld, sel_ld, swa_splits, cross_splits;
  // this launch
  const int64_t* ids;
  int ids_ld, c0, B, T, nq;  // rows b*T + t; cross rows = last nq of each sequence
  float* logits;     // [RQ][vocab] or null
  float* hidden;     // [RQ][d] or null
  int32_t* argmax;   // [RQ] or null
  const WaitCtl* ctl;  // wait limit and test hook (read once per launch)
};

size_t mk_smem_bytes();
int mk_swa_splits(const CbModel& m);
bool mk_supported(const CbModel& m, const CbCache& c, int T, int nq);
int launch_mk(const MkArgs& a, cudaStream_t st);

}  // namespace cb
