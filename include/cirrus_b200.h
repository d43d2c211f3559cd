/*
 * cirrus_b200.h -- C ABI of the B200 (sm_100a) decode path of cirrus-s-1a.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches work on that stream only, allocates nothing,
 * never synchronises the device and never throws.  Each returns CB_OK or a
 * CB_ERR_* code for a host-side argument error (nothing is launched then).
 * Errors found on the device (context full, bad token id) are written to the
 * status word of the workspace (cb_forward) and read with cb_read_status.
 *
 * Reference interfaces these replace (paths inside the reference project):
 *   cb_forward            CirrusModel.forward            cirrus/model/model.py:99-176
 *   cb_nvfp4_quantize     (no quantiser in the reference; the NVFP4 format is
 *                          cirrus/perf/bench_kernels.cu:141-145)
 *   cb_nvfp4_pack_tiles   pack_nvfp4_mma / pack_nvfp4_v3  scripts/bench_spark.py:369-391, 639-660
 *   cb_nvfp4_pack_slices  (same packers: a column-sliced layout of the standard format)
 *   cb_gemv_nvfp4         nvfp4_gemv                     cirrus/perf/bench_kernels.cu:202-227
 *   cb_gemm_nvfp4         nvfp4_gemv, M > 1 (verify, batched, prefill)  cirrus/perf/bench_kernels.cu:202-227,
 *                         1079-1300; the dense nn.Linear products of CirrusModel.forward
 *   cb_gdn_chunk_prefill  chunk_gated_delta_rule (fla)    cirrus/model/layers.py:165-170 (recurrence :108-129)
 *                         (and every nn.Linear of the model, layers.py)
 *   cb_gdn_step           GatedDeltaNet.forward          cirrus/model/layers.py:151-174
 *   cb_indexer_topk       indexer_scores + topk_mask     cirrus/model/layers.py:282-309
 *   cb_embed              nn.Embedding (tied to lm_head) cirrus/model/model.py:124, 75-77
 *   cb_argmax             logits.argmax                  cirrus/model/generate.py:33, 74
 */
#ifndef CIRRUS_B200_H
#define CIRRUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CB_ABI_VERSION 3
#define CB_MAX_SELF 32   /* self-decoder layers */
#define CB_MAX_CROSS 16  /* cross-decoder layers */
#define CB_MAX_T 8       /* tokens per sequence per launch chunk (1 + draft) */
#define CB_TILE_ROWS 16  /* rows per NVFP4 weight tile */
#define CB_SWA_EXTRA 16  /* SWA ring slots beyond the window (minimum) */
#define CB_PREFILL_CHUNK 128  /* tokens per sequence of one prompt chunk on the prefill kernels */

enum {
  CB_OK = 0,
  CB_ERR_ARG = 1,         /* null pointer or bad size */
  CB_ERR_SHAPE = 2,       /* shape not supported by the kernels */
  CB_ERR_CUDA = 3,        /* a launch failed (cudaGetLastError) */
  CB_ERR_WORKSPACE = 4,   /* workspace smaller than cb_workspace_bytes */
  CB_ERR_CTX_FULL = 5,    /* device status: a position reached max_ctx */
  CB_ERR_TOKEN = 6,       /* device status: token id outside the vocabulary */
  CB_ERR_TOO_LARGE = 7,   /* request larger than the static scratch of cb_indexer_topk_noalloc */
  CB_ERR_TIMEOUT = 8      /* device status: a bounded wait in the persistent kernel gave up */
};

enum { CB_PATH_AUTO = 0, CB_PATH_MULTI_KERNEL = 1 };

enum { CB_LAYER_GDN = 0, CB_LAYER_SWA = 1 };

/* One NVFP4 weight matrix in tile layout: ceil(rows/16) tiles, each tile is
 * 16 rows of E2M1 codes (K/2 bytes per row, low nibble = even k) followed by
 * the 16 rows of E4M3 block scales (K/16 bytes per row): 9*K bytes a tile.
 * Several matrices that read the same input are concatenated row-wise, each
 * padded to a multiple of 16 rows; tile_scale holds the float32 tensor scale
 * of every tile. */
typedef struct CbMatrix {
  const uint8_t* tiles;
  const float* tile_scale;
  int32_t rows;         /* rows including padding (multiple of 16) */
  int32_t k;            /* multiple of 16 */
} CbMatrix;

/* A second copy of an NVFP4 matrix cut into column slices of `width` columns
 * (width 2, 4, 8 or 16), for the split-K phases of the persistent kernel: slice
 * s holds, for every row r, the width/2 code bytes of columns [s*width,
 * (s+1)*width) of row r, then for every row the E4M3 scale byte of the 16-column
 * block that contains those columns; each slice is padded to a multiple of 16
 * bytes (cb_nvfp4_slice_bytes).  tensor_scale points at the float32 tensor scale. */
typedef struct CbSliced {
  const uint8_t* data;
  const float* tensor_scale;
  int32_t rows, k, width;
} CbSliced;

typedef struct CbSelfLayer {
  int32_t kind;         /* CB_LAYER_GDN or CB_LAYER_SWA */
  int32_t slot;         /* index among the GDN layers, or among the SWA layers */
  const float* norm1;   /* [d_model] */
  const float* norm2;   /* [d_model] */
  CbMatrix in_proj;     /* GDN: qkv | gate | ab ;  SWA: q | kv | gate */
  CbMatrix o_proj;
  CbMatrix gate_up;     /* [2*ffn_hidden rows] gate rows first, then up rows */
  CbMatrix down;
  const float* conv_w;  /* GDN [C, conv_size], C = 2*H*dk + H*dv */
  const float* A_log;   /* GDN [H] */
  const float* dt_bias; /* GDN [H] */
  const float* o_norm;  /* GDN [dv] */
  const float* q_norm;  /* SWA [head_dim] */
  const float* k_norm;  /* SWA [head_dim] */
  CbSliced o_proj_ks;   /* GDN: o_proj in slices of gdn_dv/8 columns (the persistent kernel's split-K o-projection) */
  CbSliced down_ks;     /* down in slices of 16 columns (the persistent kernel's split-K FFN) */
} CbSelfLayer;

typedef struct CbCrossLayer {
  const float* norm1;
  const float* norm2;
  CbMatrix q_gate;      /* q | gate */
  CbMatrix o_proj;
  CbMatrix gate_up;
  CbMatrix down;
  const float* q_norm;  /* [head_dim] */
  CbSliced down_ks;     /* down in slices of 16 columns */
} CbCrossLayer;

typedef struct CbModel {
  int32_t d_model, vocab_size, n_self_layers, n_cross_layers;
  int32_t gdn_heads, gdn_dk, gdn_dv, conv_size;
  int32_t n_q_heads, n_kv_heads, head_dim, rot_dim;
  int32_t swa_window, sparse_topk;            /* sparse_topk 0 = dense cross attention */
  int32_t indexer_heads, indexer_dim, ffn_hidden;
  float norm_eps;
  int32_t forward_path;                       /* CB_PATH_AUTO: one persistent launch per chunk when
                                                 batch*T <= 8, else one launch per op; CB_PATH_MULTI_KERNEL:
                                                 always one launch per op */
  const float* inv_freq;                      /* [rot_dim/2], as layers.py:69 computes it */
  /* column offsets inside the concatenated projection outputs (each segment
   * starts on a multiple of 16) */
  int32_t gdn_off_gate, gdn_off_a, gdn_off_b;  /* q at 0, k at H*dk, v at 2*H*dk */
  int32_t swa_off_kv, swa_off_gate;            /* q at 0; k at off_kv, v at off_kv + kv_dim */
  int32_t sh_off_ik, sh_off_iq, sh_off_iw;     /* k at 0, v at kv_dim */
  int32_t cr_off_gate;                         /* q at 0 */
  CbSelfLayer self_layers[CB_MAX_SELF];
  const float* shared_norm;
  const float* shared_k_norm;
  CbMatrix shared_proj;                        /* kv | idx_k | idx_q | idx_w */
  CbCrossLayer cross_layers[CB_MAX_CROSS];
  const float* final_norm;
  CbMatrix lm_head;                            /* tied with the embedding */
} CbModel;

/* Decode state of `batch` independent sequences (the reference Cache,
 * model.py:41-51).  pos[b] = tokens already in the cache.  SWA keys live in a
 * ring of swa_slots >= swa_window + CB_SWA_EXTRA rows, slot = position % swa_slots
 * (prompt chunks of up to swa_slots - swa_window + 1 tokens run on the prefill
 * kernels, so swa_window + CB_PREFILL_CHUNK slots give full-size chunks);
 * the shared KV rows are indexed by position.  Rows at positions >= pos[b]
 * are scratch: a forward that is later discarded may write them.
 * snap_state / snap_conv (may be null): when set, a forward of T > 1 tokens
 * also writes the GDN state and conv window after each of its first T - 1
 * tokens, [CB_MAX_T - 1][batch][n_gdn][...] in the layouts of gdn_state /
 * gdn_conv, so that a verify can be rewound to any accepted prefix
 * (cb_spec_accept) without running it again. */
typedef struct CbCache {
  int32_t batch, max_ctx, swa_slots, n_gdn, n_swa;
  int32_t* pos;        /* device [batch] */
  float* gdn_state;    /* [batch][n_gdn][H][dk][dv] float32 (S[k][v], layers.py:120) */
  float* gdn_conv;     /* [batch][n_gdn][conv_size-1][C] float32 */
  uint16_t* swa_k;     /* bf16 [batch][n_swa][swa_slots][n_kv_heads][head_dim] */
  uint16_t* swa_v;
  uint16_t* kv_k;      /* bf16 [batch][max_ctx][n_kv_heads][head_dim] */
  uint16_t* kv_v;
  uint8_t* kv_ik;      /* E4M3 [batch][max_ctx][indexer_dim] */
  float* snap_state;   /* [CB_MAX_T-1][batch][n_gdn][H][dk][dv] or null */
  float* snap_conv;    /* [CB_MAX_T-1][batch][n_gdn][conv_size-1][C] or null */
} CbCache;

int cb_abi_version(void);
const char* cb_status_string(int code);

/* ---------------------------------------------------------------- NVFP4 */
/* w float32 [n, k] (k % 16 == 0) -> standard NVFP4: codes [n, k/2] (low nibble
 * = even k), scales E4M3 [n, k/16].  Block scale = absmax(w/tensor_scale)/6
 * rounded to E4M3 (nearest-even, saturating); codes = E2M1 nearest-even of
 * (w/tensor_scale)/scale, saturating; zero scale -> zero codes. */
int cb_nvfp4_quantize(const float* w, int32_t n, int32_t k, float tensor_scale, uint8_t* codes,
                      uint8_t* scales, void* stream);

/* Bytes of one column slice of an [n, k] matrix (see CbSliced); the whole
 * sliced copy is (k / width) slices. */
int64_t cb_nvfp4_slice_bytes(int32_t n, int32_t width);

/* standard NVFP4 [n, k] -> (k / width) column slices (see CbSliced). */
int cb_nvfp4_pack_slices(const uint8_t* codes, const uint8_t* scales, int32_t n, int32_t k, int32_t width,
                         uint8_t* out, void* stream);

/* standard NVFP4 [n, k] -> ceil(n/16) tiles (see CbMatrix); pad rows are zero. */
int cb_nvfp4_pack_tiles(const uint8_t* codes, const uint8_t* scales, int32_t n, int32_t k, uint8_t* tiles,
                        void* stream);

/* y[m, :rows_out] = x[m, :k] @ dequant(W)^T for m < m_rows (rows_out <= W.rows);
 * x row stride ldx, y row stride ldy (elements).  Any m_rows >= 1. */
int cb_gemv_nvfp4(const CbMatrix* w, const float* x, int32_t ldx, int32_t m_rows, float* y, int32_t ldy,
                  int32_t rows_out, void* stream);

/* Many-token GEMM on the tensor cores (tcgen05.mma kind::f16 into tensor memory)
 * for steps that carry many token rows (batched decode, batched verify, prompt
 * chunks): y[m, r] (=, +=) pre(x)[m, :k] . dequant(W)[r, :] for m < m_rows (any
 * count), r < rows_out.  x float32 [m_rows][ldx] (16-byte aligned rows, ldx % 4
 * == 0), y float32 [m_rows][ldy].  W.k a multiple of 64.  The dequantised
 * weights are exact in f16; each input is carried as an f16 head + tail pair
 * (about 22 bits), accumulation fp32.
 *   pre CB_GEMM_PRE_RMSNORM: x * rsqrt(mean(x^2) + eps) * norm_w (norm_w 16-byte aligned)
 *   epi CB_GEMM_EPI_STORE / _ADD (y += ...) / _SWIGLU: W = [gate; up] with 2F rows,
 *       F % 64 == 0, y[m, r] = silu(gate_r) * up_r for r < rows_out <= F.
 * scratch: device memory of at least cb_gemm_scratch_bytes(W.k, m_rows) bytes
 * (16-byte aligned) for the inputs prepared as f16 operand blocks; two launches
 * (input preparation, GEMM), both as programmatic dependents of the kernel
 * before them.  status (device int32, may be null) receives CB_ERR_TIMEOUT if a
 * bounded wait on the tensor-core pipeline gives up.
 * Replaces the nn.Linear products of CirrusModel.forward for T > 1 token rows
 * (cirrus/model/model.py:99-176, layers.py:49-54 for the fused SwiGLU) that the
 * reference runs as dense matmuls, and nvfp4_gemv with M > 1
 * (cirrus/perf/bench_kernels.cu:202-227). */
#define CB_GEMM_PRE_NONE 0
#define CB_GEMM_PRE_RMSNORM 1
#define CB_GEMM_EPI_STORE 0
#define CB_GEMM_EPI_ADD 1
#define CB_GEMM_EPI_SWIGLU 2
size_t cb_gemm_scratch_bytes(int32_t k, int32_t m_rows);
int cb_gemm_nvfp4(const CbMatrix* w, const float* x, int32_t ldx, int32_t m_rows, int32_t pre, const float* norm_w,
                  float eps, float* y, int32_t ldy, int32_t rows_out, int32_t epi, void* scratch,
                  size_t scratch_bytes, int32_t* status, void* stream);

/* The NVFP4 weight stream of a step as one persistent launch: for every matrix
 * of a list (independent projections sharing one input, as in the reference's
 * decode-step weight stream) y[m, row_off(i) + r] = x[m, :k_i] . dequant(W_i)[r, :]
 * for m < m_rows <= 8.  cb_stream_plan writes the list (k a multiple of 256, at
 * most 2048; at most 128 matrices) into a caller-allocated device buffer of
 * cb_stream_plan_bytes(n_mats) bytes and returns the total rows (matrix i's rows
 * start where matrix i-1's end); it synchronises the stream.  x float32
 * [m_rows][ldx] with kmax <= ldx (every matrix reads x[:, :k_i]), y float32
 * [m_rows][ldy], ldy >= total rows.  status (device int32, may be null) receives
 * CB_ERR_TIMEOUT if a bounded wait gives up.
 * Replaces the reference's persistent weight-stream kernels decode_stream_v4/v5
 * (cirrus/perf/bench_kernels.cu:1079-1300, scripts/bench_spark.py:885-930). */
size_t cb_stream_plan_bytes(int32_t n_mats);
int cb_stream_plan(const CbMatrix* mats, int32_t n_mats, void* plan, size_t plan_bytes, int64_t* rows_total,
                   void* stream);
int cb_weight_stream_nvfp4(const void* plan, int32_t n_mats, int32_t total_tiles, const float* x, int32_t ldx,
                           int32_t kmax, int32_t m_rows, float* y, int64_t ldy, int32_t* status, void* stream);

/* h[r, :] = dequant(lm_head row ids[r]) for r < n_rows (float32 [n_rows, d]). */
int cb_embed(const CbMatrix* table, const int64_t* ids, int32_t n_rows, float* h, int32_t* status, void* stream);

/* out[r] = first index of the maximum of x[r, :n] for r < rows. */
int cb_argmax(const float* x, int32_t rows, int32_t n, int32_t ld, int32_t* out, void* stream);

/* ------------------------------------------------------------ GDN step */
/* One Gated DeltaNet mixer step for T tokens of `batch` sequences, from the
 * in_proj output (qkv | gate | ab, row = b*T + t, row stride ldp) to the
 * gated, normalised output [batch*T, H*dv]: short conv with its rolling
 * cache, L2-norm of q and k, decay g = -exp(A_log)*softplus(a + dt_bias),
 * beta = sigmoid(b), the exact recurrence on S (updated in place), o_norm and
 * the silu(gate) product.  state/conv point at this layer's slot of sequence
 * 0; state_stride / conv_stride are the element strides between sequences. */
int cb_gdn_step(const CbModel* m, int32_t layer, const float* proj, int32_t ldp, int32_t batch, int32_t T,
                float* state, int64_t state_stride, float* conv, int64_t conv_stride, float* out, int32_t ldo,
                void* stream);

/* Chunked Gated DeltaNet recurrence for prefill (64-token chunks, Dk = Dv = 64),
 * the exact recurrence of layers.py:108-129 evaluated chunk-wise:
 * q, k [B][T][H][64] (q, k L2-normalised by the caller), v [B][T][H][64],
 * g [B][T][H] (log decay, <= 0), beta [B][T][H]; state S [B][H][Dk][Dv] fp32 is
 * read and replaced by the state after token T-1; out [B][T][H][Dv] = S_t^T (q_t scale).
 * Replaces fla's chunk_gated_delta_rule at layers.py:165-170. */
int cb_gdn_chunk_prefill(const float* q, const float* k, const float* v, const float* g, const float* beta, int32_t B,
                         int32_t T, int32_t H, int32_t Dk, int32_t Dv, float scale, float* state, float* out,
                         void* stream);

/* -------------------------------------------------- indexer + top-k */
/* For each of `rows` query rows: scores over keys 0..qpos[r] of sequence
 * seq[r] (s = sum_h iw_h * relu(iq_h . ik_s), one fixed float32 order), then
 * the stable top-k of layers.py:291-309 (most recent key wins ties, the
 * query's own key always kept, all keys kept when qpos+1 <= k).
 * iq [rows][Hi*Di] (stride ld_q), iw [rows][Hi] (stride ld_q), ik E4M3
 * [batch][max_ctx][Di].  scores: scratch [rows][max_ctx] float32.
 * sel_idx [rows][k+1] ascending key indices, sel_cnt [rows]. */
int cb_indexer_topk(const float* iq, const float* iw, int32_t ld_q, const uint8_t* ik, int32_t max_ctx,
                    int32_t Hi, int32_t Di, const int32_t* seq, const int32_t* qpos, int32_t rows, int32_t k,
                    float* scores, int32_t* sel_idx, int32_t* sel_cnt, void* stream);

/* cb_indexer_topk for callers that cannot allocate device memory when they
 * call: for example a serving process whose memory planner hands out every
 * device byte at start-up and forbids allocation afterwards, or a binding in
 * another language that receives only the input and output buffers from its
 * host runtime and has no device allocator to call.  No counterpart in the
 * reference: it is cb_indexer_topk with the `scores` scratch taken from a
 * static array inside the library (CB_NOALLOC_MAX_SCORES float32 values =
 * 4 MiB per GPU that loads the library, held until the process exits), so the
 * caller passes only inputs and outputs and nothing is allocated.
 *   - rows * max_ctx must be <= CB_NOALLOC_MAX_SCORES, else CB_ERR_TOO_LARGE and
 *     nothing is launched (e.g. 8 query rows at 128K context, 32 at 32K);
 *   - the first call on each device looks the array up on that device (make
 *     that first call before any stream capture on the device);
 *   - every call on a device shares the one array and it keeps the last call's
 *     scores; nothing in it needs to start at zero (each call writes every
 *     score it reads), but calls that overlap on the GPU (other streams, or
 *     other threads' streams) race on it and must be serialised by the caller. */
#define CB_NOALLOC_MAX_SCORES (1 << 20)
int cb_indexer_topk_noalloc(const float* iq, const float* iw, int32_t ld_q, const uint8_t* ik, int32_t max_ctx,
                            int32_t Hi, int32_t Di, const int32_t* seq, const int32_t* qpos, int32_t rows,
                            int32_t k, int32_t* sel_idx, int32_t* sel_cnt, void* stream);

/* ------------------------------------------------------- whole forward */
/* Workspace bytes cb_forward needs for `batch` sequences and up to T tokens
 * per sequence.  Longer inputs run in chunks: up to CB_MAX_T tokens on the
 * decode kernels; prompts (T > CB_MAX_T) in chunks of up to CB_PREFILL_CHUNK
 * tokens on the prefill kernels (tensor-core GEMMs, chunked Gated DeltaNet,
 * block-wise SWA) when the model's shapes allow them (GDN Dk = Dv = 64, every
 * projection K a multiple of 64), else in chunks of CB_MAX_T. */
size_t cb_workspace_bytes(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx);

/* CirrusModel.forward(input_ids[batch, T], cache, n_logits) for a batch of
 * sequences sharing T: embeds, runs the self-decoder (updating GDN / conv /
 * SWA state), appends T shared-KV rows per sequence, runs the cross-decoder
 * and LM head for the last n_logits positions (n_logits <= 0 means T), and
 * advances cache->pos by T on the device.  ids: device int64 [batch, T].
 * Outputs (any may be NULL): logits [batch][n][vocab], hidden [batch][n][d]
 * (pre-final-norm), argmax [batch][n].  Launch-only: capturable in a CUDA graph. */
int cb_forward(const CbModel* m, const CbCache* c, void* workspace, size_t workspace_bytes, const int64_t* ids,
               int32_t T, int32_t n_logits, float* logits, float* hidden, int32_t* argmax, void* stream);

/* Where cb_forward keeps its intermediate results inside a workspace sized for
 * (batch, T, max_ctx), as byte offsets from the workspace start, for reading
 * them back after a forward (tests, debugging):
 *   proj     float32 [rows][ld_proj], rows = batch * Tc (Tc the chunk length): the shared
 *            projection of the last chunk's rows (k | v | idx_k | idx_q | idx_w at
 *            the CbModel offsets; row b*Tc + t);
 *   sel_idx  int32 [batch*nq][sel_ld]: the keys each query row of the last chunk
 *            selected (ascending, sel_cnt[r] of them), nq = query rows per sequence;
 *   sel_cnt  int32 [batch*nq].
 * The reference computes these inside CirrusModel.forward (model.py:136-156). */
typedef struct CbWorkspaceLayout {
  uint64_t bytes, proj, sel_idx, sel_cnt;
  int32_t ld_proj, sel_ld;
  int32_t rows;  /* batch * Tc: rows of proj */
} CbWorkspaceLayout;
int cb_workspace_layout(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx, CbWorkspaceLayout* out);

/* ------------------------------------------------------------ MTP draft */
/* The first multi-token-prediction module and the FR-Spec restricted draft
 * head (cirrus/model/layers.py:351-370, cirrus/model/model.py:230-245). */
typedef struct CbMtp {
  const float* norm_h;      /* [d] */
  const float* norm_e;      /* [d] */
  const float* ffn_norm;    /* [d] */
  CbMatrix proj;            /* [d rows][2d]: cat(norm_h(h), norm_e(e)) -> d */
  CbMatrix gate_up;         /* [2*ffn_hidden rows][d] */
  CbMatrix down;            /* [d rows][ffn_hidden] */
  CbMatrix draft_head;      /* the embedding rows of draft_ids, [n_draft rows][d] */
  const int32_t* draft_ids; /* device [n_draft] */
  int32_t n_draft;
} CbMtp;

/* Scratch bytes cb_mtp_draft needs. */
size_t cb_mtp_workspace_bytes(const CbModel* m, const CbMtp* mtp);

/* CirrusModel.mtp_draft(h_last, token, n) (model.py:230-245): n passes of
 * h = mtp(h, embed(tok)); tok = draft_ids[argmax(final_norm(h) . draft_head^T)],
 * starting from the hidden state h_last (device float [d], the pre-final-norm
 * hidden that predicted `token`) and token (device int32 [1]); the n drafted
 * tokens go to out (device int32 [n]). */
int cb_mtp_draft(const CbModel* m, const CbMtp* mtp, const float* h_last, const int32_t* token, int32_t n,
                 int32_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------- speculative decoding */
/* Prompt-lookup drafts for `batch` sequences, on the device.  Sequence b's
 * tokens so far are tokens[b*ld .. b*ld + lens[b]) (prompt, then generated
 * tokens; the last one is the pending token not yet in the cache).  The draft
 * is the reference rule (cirrus/decoding/prompt_lookup.py:19-58): for n from
 * max_ngram down to min_ngram, the tokens that followed the most recent earlier
 * occurrence of the last n tokens, at most min(max_draft, T - 1, budget[b] - 1)
 * of them (budget = tokens still to generate; <= 0 marks a finished sequence).
 * Writes the verify input ids[b][0..T) = pending token, draft, then the pending
 * token again as padding, and draft_len[b]. */
int cb_prompt_lookup_draft(const int32_t* tokens, int32_t ld, const int32_t* lens, const int32_t* budget,
                           int32_t batch, int32_t min_ngram, int32_t max_ngram, int32_t max_draft, int64_t* ids,
                           int32_t T, int32_t* draft_len, void* stream);

/* Greedy acceptance after a verify forward of T = 1 + draft tokens per
 * sequence (cirrus/decoding/prompt_lookup.py:61-74 and the bookkeeping of
 * cirrus/model/generate.py:66-88): n = the leading draft tokens equal to the
 * model's argmax[b][t]; the n accepted tokens and the model's next token are
 * appended to tokens/lens, budget[b] drops by n + 1, *emitted (device int64)
 * grows by n + 1; the cache is rewound to the accepted prefix: pos[b] drops by
 * T - 1 - n and, when n < T - 1, the GDN state and conv window are restored
 * from the snapshot after token n (the cache must have snap_state/snap_conv).
 * A finished sequence (budget <= 0) only gets its position rewound by T. */
int cb_spec_accept(const CbModel* m, const CbCache* c, const int32_t* argmax, const int64_t* ids,
                   const int32_t* draft_len, int32_t T, int32_t* tokens, int32_t ld, int32_t* lens,
                   int32_t* budget, int64_t* emitted, void* stream);

/* Copy the workspace's device status word into *status (synchronises on the stream). */
int cb_read_status(const void* workspace, int32_t* status, void* stream);
/* Clear the status word (stream-ordered). */
int cb_clear_status(void* workspace, void* stream);

/* Limit of every bounded wait of the persistent kernel that runs on this
 * workspace (limit_ns = 0 restores the default, 200 ms): a wait that lasts
 * longer sets CB_ERR_TIMEOUT in the status word, and every CTA of that launch
 * returns without advancing the cache.  stall_barrier > 0 is a fault-injection
 * hook for tests: CTA 0 then skips its arrival at that grid barrier, so the
 * waits on it run out (0 = off).  Synchronises on the stream.  No reference
 * counterpart: the reference's grid barrier spins without a limit
 * (cirrus/perf/bench_kernels.cu:116-117). */
int cb_set_wait_limit(void* workspace, uint64_t limit_ns, int32_t stall_barrier, void* stream);

/* Number of kernels this library has launched in this process (all entry points). */
int64_t cb_launch_count(void);

/* Phase trace of the last persistent launch that used this workspace: out[0] =
 * %globaltimer (ns) at kernel start, then for barrier i >= 1: out[2i-1] = when
 * CTA 0 arrived at barrier i, out[2i] = when it left.  Returns the number of
 * values written (<= n) or a negative CB_ERR code (synchronises on the stream).
 * (The reference's per-stage clock / globaltimer stamps, bench_kernels.cu:904-988.) */
int cb_read_trace(const CbModel* m, int32_t batch, int32_t T, int32_t max_ctx, const void* workspace, uint64_t* out,
                  int32_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CIRRUS_B200_H */
