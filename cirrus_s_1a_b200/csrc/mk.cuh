// Persistent decode kernel: launch interface (decode_mk.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cirrus_b200.h"

namespace cb {

constexpr int kMkThreads = 512;
constexpr int kMkHistBins = 2048;      // top 11 bits of the score key
constexpr int kMkSwaSplit = 128;       // window keys per SWA work item
constexpr int kMkCrossSplit = 64;      // selected keys per cross-attention work item
constexpr int kMkMaxRows = 8;          // batch * T handled by one persistent launch
constexpr int kMkMaxQ = 24;            // (q heads per KV head) * T per SWA work item
constexpr int kMkArrive = 512;         // last-arriver counters
constexpr int kMkTrace = 512;          // phase timestamps

constexpr int kMkMaxPhases = 128;

enum { MK_PRE_NONE = 0, MK_PRE_RMS = 1, MK_PRE_EMBED = 2 };
enum { MK_EPI_STORE = 0, MK_EPI_ADD = 1, MK_EPI_ACT = 2 };
enum { MK_PH_GEMV = 0, MK_PH_GDN = 1, MK_PH_SWA = 2, MK_PH_SHARED = 3, MK_PH_COMPACT = 4, MK_PH_CROSS = 5 };

// One NVFP4 GEMV phase: y[m, :rows_out] (=, += or silu-gated) W . pre(x[m, :]).
struct GemvJob {
  CbMatrix W;
  const float* x;
  int32_t ldx;
  int32_t xmap_nq, xmap_T, xmap_off;  // x row of m = (m / nq) * T + off + m % nq when xmap_nq > 0
  int32_t pre;                        // MK_PRE_*
  const float* norm_w;
  float* y;
  int32_t ldy, rows_out, epi;         // MK_EPI_*; ACT pairs row r (gate) with row rows/2 + r (up)
  int32_t argmax;                     // per-row argmax of y into MkArgs::amax
  float* copy_x;                      // the phase's first CTA stores the raw input rows here ([m][K])
};

// One step of the plan the persistent kernel interprets; a grid barrier follows every phase.
struct MkPhase {
  int32_t type;           // MK_PH_*
  int32_t layer;          // self or cross layer index
  int32_t resolve_ctas;   // GEMV phase: CTAs [0, resolve_ctas) resolve the top-k rows instead
  int32_t m_rows;         // GEMV input rows
  int32_t prefetch_unit;  // L2 prefetch issued when the phase starts (-1: none)
  int32_t copy_hidden;    // copy the cross-decoder rows to the hidden output
  GemvJob g;
};

// Everything one persistent launch needs, passed by value (__grid_constant__).
struct MkArgs {
  CbModel m;
  CbCache c;
  // workspace
  float* h;          // [M][d] residual stream of the self-decoder
  float* proj;       // [M][ldp]
  float* attn;       // [M][att_ld]
  float* act;        // [M][ffn]   silu(gate) * up
  float* xc;         // [RQ][d]   cross-decoder residual stream
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
  unsigned* arrive;  // [kMkArrive]
  unsigned long long* amax;  // [RQ] packed argmax
  unsigned* sync;    // grid barrier counter (zeroed before every launch)
  unsigned long long* trace;  // [kMkTrace] phase timestamps of CTA 0
  int32_t* abort_flag;
  int32_t* status;
  int ldp, att_ld, cr_ld, sel_ld, swa_splits, cross_splits;
  // this launch
  const int64_t* ids;
  int ids_ld, c0, B, T, nq;  // rows b*T + t; cross rows = last nq of each sequence
  float* logits;     // [RQ][vocab] or null
  float* hidden;     // [RQ][d] or null
  int32_t* argmax;   // [RQ] or null
  unsigned long long timeout_ns;
  int32_t n_phases;
  MkPhase phases[kMkMaxPhases];
};

static_assert(sizeof(MkArgs) < 32000, "persistent kernel arguments must fit the kernel parameter space");

size_t mk_smem_bytes();
// Fill a.phases with the step's plan (the fields above must be set); false if it does not fit.
bool mk_build_plan(MkArgs& a);
bool mk_supported(const CbModel& m, const CbCache& c, int T, int nq);
int launch_mk(const MkArgs& a, int grid, cudaStream_t st);

}  // namespace cb
