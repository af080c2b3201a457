/*
 * wl_attn.h — C ABI of the B200 (sm_100a) GLM-5.2 attention substep:
 * DSA lightning-indexer scoring over fp8-e4m3 index keys, exact per-query
 * top-k key selection, and absorbed-MLA attention over the bf16 latent cache,
 * for decode and chunked prefill, optionally with the KV sequence sharded
 * across the GPUs of one node (NCCL).
 *
 * Drop-in boundary. The reference runs this substep inside
 *     run_attention(const Config&, const LayerWeights&, uint32_t layer,
 *                   uint32_t pos, float* d_hidden, IndexShare&, cudaStream_t)
 * at src/glm_layer_runner.cuh:525-527, specifically the block
 * src/glm_layer_runner.cuh:582-644 (indexer -> index mask -> absorbed
 * attention). Every entry point below replaces one piece of that block; the
 * reference function each one stands in for is cited beside it.
 *
 * Conventions
 *  - Plain pointers and sizes only. Every pointer argument named "device" is
 *    device memory owned by the caller; nothing here allocates on a hot path.
 *  - Every call is stream-ordered on the caller's `stream` (a cudaStream_t
 *    passed as void*; NULL is the legacy default stream) and returns a status
 *    code instead of aborting (the reference aborts: GLM_CUDA_OK at
 *    src/glm_loader.cuh:24-26, IndexShare::require at
 *    src/glm_layer_runner.cuh:507-516, T > max_seq at :576-580).
 *  - Shapes are GLM-5.2's (Config at src/glm_loader.cuh:33-69): 64 attention
 *    heads, kv_lora 512 + rope 64 = 576-wide absorbed query and latent row,
 *    32 indexer heads x 128. Other shapes return WL_ERR_UNSUPPORTED.
 *  - Index selections ("sel") are int32 key positions. Lists this library
 *    writes are canonical: strictly ascending, unique, inside [0, T).
 */
#ifndef WL_ATTN_H
#define WL_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WL_ABI_VERSION 1

/* ---- status codes --------------------------------------------------------- */
enum {
    WL_OK                = 0,
    WL_ERR_ARG           = 1,  /* null pointer, bad size or stride                */
    WL_ERR_T_EXCEEDS_MAX = 2,  /* T > cfg.T_max (reference: abort at :576-580)     */
    WL_ERR_NO_INDICES    = 3,  /* consumer layer with nothing published (:507-516) */
    WL_ERR_CUDA          = 4,  /* a CUDA runtime call failed                       */
    WL_ERR_NCCL          = 5,  /* an NCCL call failed                              */
    WL_ERR_TIMEOUT       = 6,  /* a bounded device-side wait ran out               */
    WL_ERR_WORKSPACE     = 7,  /* workspace missing or smaller than required       */
    WL_ERR_UNSUPPORTED   = 8,  /* shape outside the compiled GLM-5.2 dimensions    */
    WL_ERR_DEVICE        = 9   /* a device-side bounds check fired                 */
};

/* Human-readable text for a status code (never NULL). */
const char* wl_strerror(int status);

/* ---- configuration (subset of Config, src/glm_loader.cuh:33-69) ----------- */
typedef struct wl_attn_cfg {
    int32_t n_heads;       /* num_attention_heads          = 64   */
    int32_t kv_lora;       /* kv_lora_rank                 = 512  */
    int32_t rope_dim;      /* qk_rope_head_dim             = 64   */
    int32_t idx_heads;     /* index_n_heads                = 32   */
    int32_t idx_dim;       /* index_head_dim               = 128  */
    int32_t index_topk;    /* index_topk                   = 2048 */
    float   softmax_scale; /* qk_head_dim^-0.5 = 1/16 (glm_layer_runner.cuh:641) */
    float   idx_qk_scale;  /* index_head_dim^-0.5 (glm_kernels.cuh:463)         */
    int32_t T_max;         /* Config::max_seq: rows the caller's caches hold    */
} wl_attn_cfg;

/* Fill `cfg` with GLM-5.2's values and the given cache capacity. */
void wl_attn_cfg_glm52(wl_attn_cfg* cfg, int32_t T_max);

/* ---- cache views ------------------------------------------------------------
 * Latent cache: the reference keeps kv_c_cache [max_seq,512] and k_rot_cache
 * [max_seq,64] in fp32, row = absolute position (glm_loader.cuh:282-283). Here
 * the same two-pointer addressing holds bf16 rows. A packed [T,576] row is the
 * case k_rot = c_kv + 512 with both row strides 576. Strides are in elements;
 * row strides must be multiples of 8 and both pointers 16-byte aligned.
 * `*_seq_stride` steps between independent sequences of a batch. */
typedef struct wl_latent_cache {
    const void* c_kv;   int64_t c_kv_row_stride;  int64_t c_kv_seq_stride;
    const void* k_rot;  int64_t k_rot_row_stride; int64_t k_rot_seq_stride;
} wl_latent_cache;

/* Indexer key cache of an owning layer: the reference stores bf16 [max_seq,128]
 * (glm_loader.cuh:307, written by indexer_store_k_bf16 at glm_kernels.cuh:280).
 * Here: fp8-e4m3 [T, idx_dim] packed rows (128 bytes each) plus one fp32
 * dequantisation scale per key; key t's value is e4m3(keys[t]) * scale[t].
 * `keys` must be 16-byte aligned. Seq strides: bytes for keys, floats for scale. */
typedef struct wl_index_cache {
    const void*  keys;  int64_t keys_seq_stride;
    const float* scale; int64_t scale_seq_stride;
} wl_index_cache;

/* Query rows of one call. Row r belongs to sequence r / rows_per_seq and sees
 * keys [0, len0 + (r % rows_per_seq) * len_step), clamped to T. Decode:
 * rows_per_seq = 1, len0 = T, len_step = 0. Chunked prefill of n_q rows after
 * a pos0-token prefix: rows_per_seq = n_q, len0 = pos0 + 1, len_step = 1 (the
 * causal rule of run_prefill_layer_major, glm_layer_runner.cuh:963-973). */
typedef struct wl_rows {
    int32_t n_rows;
    int32_t rows_per_seq;
    int32_t len0;
    int32_t len_step;
} wl_rows;

/* ---- IndexShare (glm_layer_runner.cuh:485-517; ref_glm_chain.py:445-462) --
 * Owner layers publish their raw top-k; "shared" layers read it unchanged;
 * a shared layer with nothing published fails with WL_ERR_NO_INDICES. `dense`
 * is the standalone-layer test mode: attend every key, never fail. */
typedef struct wl_index_share {
    const int32_t* idx;       /* device [n_rows, stride] canonical lists     */
    const int32_t* n_dev;     /* device [n_rows] counts (may be NULL)        */
    int64_t        stride;    /* elements between rows of idx                */
    int32_t        n;         /* count when n_dev is NULL                    */
    uint32_t       producer;  /* layer that published; UINT32_MAX = none     */
    int32_t        dense;
} wl_index_share;

void wl_index_share_reset(wl_index_share* s);                 /* IndexShare::reset   */
void wl_index_share_publish(wl_index_share* s, uint32_t layer, /* IndexShare::publish */
                            const int32_t* idx, const int32_t* n_dev,
                            int64_t stride, int32_t n);
int  wl_index_share_require(const wl_index_share* s, uint32_t layer); /* ::require */

/* ---- decode (one query token per sequence) ------------------------------- */
enum { WL_MODE_OWNER = 0, WL_MODE_CONSUMER = 1, WL_MODE_DENSE = 2 };
enum { WL_SEL_CANONICAL = 1 };  /* consumer asserts sel_in is already canonical */

typedef struct wl_attn_decode_io {
    int32_t batch;              /* independent sequences                       */
    int32_t T;                  /* keys per sequence (= pos + 1)               */
    wl_latent_cache latent;
    wl_index_cache  index;      /* owner only                                  */
    const void*  q_abs;         /* bf16 [batch, n_heads, kv_lora+rope_dim]     */
    const void*  q_idx;         /* bf16 [batch, idx_heads, idx_dim], post-RoPE */
    const float* w_idx;         /* fp32 [batch, idx_heads], x idx_heads^-0.5   */
    int32_t  mode;              /* WL_MODE_*                                   */
    int32_t  sel_flags;         /* WL_SEL_CANONICAL                            */
    int32_t* sel_out;           /* owner: [batch, sel_stride] (may be NULL)    */
    int32_t* sel_n_out;         /* owner: [batch] counts (may be NULL)         */
    const int32_t* sel_in;      /* consumer: [batch, sel_stride]               */
    const int32_t* sel_n_in;    /* consumer: [batch] counts, or NULL -> sel_n  */
    int32_t  sel_n;             /* consumer count when sel_n_in is NULL        */
    int64_t  sel_stride;        /* >= min(index_topk, T)                       */
    float*   index_out;         /* owner, optional: [batch, index_stride] fp32 */
    int64_t  index_stride;
    float*   ctx;               /* out: fp32 [batch, n_heads, kv_lora]         */
    float*   lse;               /* out, optional: fp32 [batch, n_heads]        */
} wl_attn_decode_io;

/* Workspace needed by wl_attn_decode / wl_attn_decode_sharded for up to
 * `batch` sequences of up to T_max keys (bytes, 256-byte aligned base). */
size_t wl_attn_workspace_bytes(const wl_attn_cfg* cfg, int32_t T_max, int32_t batch);

/* The attention substep for one decode token per sequence. Replaces
 * glm_layer_runner.cuh:582-644: owner -> indexer scores (glm_kernels.cuh:
 * 453-477) + top-k (:344-414) + sparse absorbed attention (glm_layer_runner.cuh:
 * 251-298) over the selected keys; consumer -> the same attention over sel_in;
 * dense -> attention over every key. Output ctx is the reference's s_ctx. */
int wl_attn_decode(const wl_attn_cfg* cfg, const wl_attn_decode_io* io,
                   void* workspace, size_t workspace_bytes, void* stream);

/* The same substep with run_attention's IndexShare dispatch
 * (glm_layer_runner.cuh:594-619): if `owner`, run the indexer and publish the
 * selection (io->sel_out, which must be set) into *share; otherwise require
 * *share and consume it (or attend densely if share->dense). */
int wl_attn_layer_decode(const wl_attn_cfg* cfg, wl_attn_decode_io* io,
                         int32_t owner, uint32_t layer, wl_index_share* share,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---- chunked prefill ------------------------------------------------------
 * n_q new rows for one sequence whose cache already holds the pos0-token
 * prefix AND the n_q new rows (T = pos0 + n_q). Row i is causal over keys
 * [0, pos0 + i]. The reference has no batched prefill attention: it calls the
 * decode form once per row in ascending order (glm_layer_runner.cuh:963-983);
 * this computes exactly those per-row results in one call. */
typedef struct wl_attn_prefill_io {
    int32_t n_q;
    int32_t pos0;
    wl_latent_cache latent;
    wl_index_cache  index;
    const void*  q_abs;         /* bf16 [n_q, n_heads, 576]                   */
    const void*  q_idx;         /* bf16 [n_q, idx_heads, idx_dim]             */
    const float* w_idx;         /* fp32 [n_q, idx_heads]                      */
    int32_t  mode;
    int32_t  sel_flags;
    int32_t* sel_out;           /* owner: [n_q, sel_stride]                   */
    int32_t* sel_n_out;         /* owner: [n_q]                               */
    const int32_t* sel_in;      /* consumer: [n_q, sel_stride]                */
    const int32_t* sel_n_in;    /* consumer: [n_q] or NULL -> min(topk, row len) */
    int64_t  sel_stride;
    float*   index_out;         /* optional [n_q, index_stride]               */
    int64_t  index_stride;
    float*   ctx;               /* out: fp32 [n_q, n_heads, kv_lora]          */
    float*   lse;               /* out, optional: fp32 [n_q, n_heads]         */
} wl_attn_prefill_io;

size_t wl_attn_prefill_workspace_bytes(const wl_attn_cfg* cfg, int32_t n_q, int32_t T);
int wl_attn_prefill(const wl_attn_cfg* cfg, const wl_attn_prefill_io* io,
                    void* workspace, size_t workspace_bytes, void* stream);

/* wl_attn_prefill with run_prefill_layer_major's IndexShare dispatch
 * (glm_layer_runner.cuh:954-983): an owner layer publishes every row's
 * selection (io->sel_out / sel_n_out, which must be set: row i is query
 * position pos0 + i) into *share; a shared layer requires *share and attends
 * each row over its own published row (or densely if share->dense). */
int wl_attn_layer_prefill(const wl_attn_cfg* cfg, wl_attn_prefill_io* io,
                          int32_t owner, uint32_t layer, wl_index_share* share,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---- the individual hot-path kernels ------------------------------------- */

/* a1+a2 fused: index[r][t] = sum_h w[r][h] * relu(idx_qk_scale * scale[t] *
 * (q[r][h] . e4m3(keys[t]))) for t < len(r). Replaces indexer_scores_relu +
 * indexer_combine (glm_kernels.cuh:308-340); no [H,T] intermediate. */
int wl_indexer_scores(const wl_attn_cfg* cfg, const wl_index_cache* cache,
                      int32_t T, const wl_rows* rows,
                      const void* q_idx, const float* w_idx,
                      float* index_out, int64_t index_stride, void* stream);

/* a3: exact top-min(k, len(r)) per row, ties to the lowest index, written
 * canonical (ascending); k >= len(r) writes the identity 0..len-1. Replaces
 * indexer_topk (glm_kernels.cuh:344-414) / ref_glm_chain.py:504-515.
 * `cand_idx` (may be NULL) maps positions to output indices: row r's element
 * j is reported as cand_idx[r*index_stride + j] (used to merge candidates). */
int wl_indexer_topk(const float* index, int64_t index_stride, const wl_rows* rows,
                    int32_t T, int32_t k, const int32_t* cand_idx,
                    int32_t* sel_out, int64_t sel_stride, int32_t* sel_n_out,
                    void* workspace, size_t workspace_bytes, void* stream);
/* Workspace that lets wl_indexer_topk spread a row over many CTAs: rows of
 * 8 193 - 196 608 keys select on an 8-CTA thread-block cluster, longer ones in
 * a multi-CTA partition pass (without it every row runs on one CTA). */
size_t wl_indexer_topk_workspace_bytes(int32_t n_rows, int32_t T);

/* a5 semantics: turn an arbitrary index list (any order, duplicates, entries
 * outside [0, len(r))) into the canonical list of the keys it keeps. Same
 * selection as index_mask_fill/scatter (glm_kernels.cuh:526-537): out-of-range
 * entries unmask nothing, duplicates count once. */
int wl_sel_normalize(const int32_t* sel_in, int64_t in_stride,
                     const int32_t* n_in_dev, int32_t n_in,
                     const wl_rows* rows, int32_t T,
                     int32_t* sel_out, int64_t out_stride, int32_t* n_out_dev,
                     void* stream);

/* a7: sparse absorbed-MLA attention over canonical lists (NULL = every key),
 * restricted to the key window [win_lo, win_hi) whose first key is cache row 0,
 * split into CTAs of `split_keys` selected keys (multiple of 64; 0 = the whole
 * list in one CTA). Writes per split the normalised partial output and its
 * log-sum-exp: o_part[(r*max_splits + s)*n_heads*kv_lora ...],
 * lse_part[(r*max_splits + s)*n_heads ...]. A split with no keys writes lse =
 * -inf only and leaves its o untouched (wl_lse_merge never reads it).
 * Replaces mla_decode_absorbed (glm_layer_runner.cuh:251-298) with its mask
 * (glm_kernels.cuh:526-545). */
int wl_mla_sparse_attn(const wl_attn_cfg* cfg, const wl_latent_cache* cache,
                       int32_t T, const wl_rows* rows, const void* q_abs,
                       const int32_t* sel, int64_t sel_stride,
                       const int32_t* sel_n_dev, int32_t sel_n,
                       int64_t win_lo, int64_t win_hi, int32_t split_keys,
                       float* o_part, float* lse_part, int32_t max_splits,
                       void* stream);

/* (o, lse) merge of `n_parts` partials per row: o = sum_s e^(lse_s - L) o_s,
 * L = log sum_s e^(lse_s). Part s of row r lives at o_part + r*row_stride +
 * s*part_stride (floats; lse likewise with lse_row_stride / lse_part_stride). */
int wl_lse_merge(const float* o_part, const float* lse_part, int32_t n_rows,
                 int32_t n_parts, int64_t row_stride, int64_t part_stride,
                 int64_t lse_row_stride, int64_t lse_part_stride,
                 int32_t n_heads, int32_t kv_lora,
                 float* ctx, float* lse, void* stream);

/* ---- KV-sequence sharding over the GPUs of one node ------------------------
 * Rank r holds keys [t0, t0 + io->T) of every cache. Each rank scores and
 * selects locally; an all-gather of the (score, global index) candidates
 * gives every rank the exact single-GPU selection, each rank attends over its
 * part of it, and the (o, lse) partials are combined: over peer memory as a
 * reduce-scatter by heads (each rank merges 64/N heads of every row) and an
 * all-gather of the merged slices; over NCCL as an all-gather of the partials
 * and a merge on every rank. Every rank returns the full ctx/lse and (owner)
 * the global selection. No reference counterpart: the reference is
 * single-GPU (README.md:88).
 * The all-gathers run over NVLink peer memory (each rank writes into every
 * rank's exchange region; wl_comm_create maps them, collectively, through CUDA
 * IPC; N must divide 64), or over NCCL when that is unavailable, disabled
 * (WL_NO_P2P=1) or a call exceeds the regions' capacity (32 rows,
 * index_topk 4096). Creation and destruction are collective. */
typedef struct wl_comm wl_comm;
int wl_comm_unique_id(uint8_t id_out[128]);
int wl_comm_create(const uint8_t id[128], int32_t nranks, int32_t rank,
                   wl_comm** out);
int wl_comm_destroy(wl_comm* comm);
/* 1 when this communicator exchanges over NVLink peer memory, 0 over NCCL. */
int wl_comm_p2p(const wl_comm* comm);

typedef struct wl_shard {
    int64_t t0;        /* global position of this rank's cache row 0 */
    int64_t T_global;  /* keys across all ranks                      */
} wl_shard;

size_t wl_attn_sharded_workspace_bytes(const wl_attn_cfg* cfg, int32_t T_local_max,
                                       int32_t batch, int32_t nranks);
int wl_attn_decode_sharded(const wl_attn_cfg* cfg, const wl_attn_decode_io* io,
                           const wl_shard* shard, wl_comm* comm,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Decode attention (consumer with a canonical list, or dense) for callers
 * that cannot allocate device memory: no workspace argument, no allocation.
 * No counterpart in the reference. Its split-K scratch is a fixed array
 * inside the library (about 8.4 MB on every GPU that loads it, for at most 4
 * sequences per call); larger batches return WL_ERR_WORKSPACE, owner mode
 * and non-canonical lists WL_ERR_UNSUPPORTED. The first call on a device
 * looks up the array's device address, so make that first call before any
 * stream capture. All calls share the array: calls that overlap on the GPU
 * (different streams, or different host threads) race and must not. */
int wl_attn_decode_noalloc(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, void* stream);

/* ---- the indexer's query side --------------------------------------------------
 * For n query rows: q_idx[r] = RoPE(wq_b @ q_resid[r]) (RoPE on dims [0, 64)
 * of each of the 32 heads, interleaved pairs in, halves out, with the row's
 * table cos/sin [n, 32]) stored bf16 [n, 32, 128]; and w_idx[r][h] =
 * (weights_proj @ x[r])[h] * 32^-0.5 stored fp32 [n, 32] — the inputs the
 * scoring entry points take. q_resid: fp32 [n, 2048] (the shared q-LoRA
 * residual); wq_b: bf16 [32*128, 2048]; x: fp32 [n, hidden] (the
 * input_layernorm output; hidden a multiple of 1024); weights_proj: fp32
 * [32, hidden]. Row strides in elements, multiples of 4; matrices 16-byte
 * aligned. Replaces the query half of launch_indexer_query
 * (glm_kernels.cuh:469-472: launch_matvec_bf16, rope_interleave_slice,
 * indexer_head_weights). */
int wl_indexer_query(const wl_attn_cfg* cfg, int32_t n, const float* q_resid, int64_t q_resid_row_stride,
                     const void* wq_b, const float* x, int64_t x_row_stride, int32_t hidden,
                     const float* weights_proj, const float* cos, const float* sin,
                     void* q_idx, float* w_idx, void* stream);

/* ---- the absorption around the attention ------------------------------------
 * kv_b = kv_b_proj, device bf16 [n_heads * (qk_nope 192 + v_head 256), kv_lora]
 * (per head: 192 W_UK rows, then 256 W_UV rows), 16-byte aligned.
 *
 * wl_mla_absorb_q: for n query rows, q fp32 [n][n_heads][256] (qk_nope 192 |
 * roped qk_rope 64; 16-byte aligned, row stride q_row_stride floats, a
 * multiple of 4) ->
 *   q_abs[r][h][c]       = sum_{d<192} q[r][h][d] * kv_b[h*448 + d][c]   (c < 512)
 *   q_abs[r][h][512 + j] = q[r][h][192 + j]                              (j < 64)
 * in bf16 (row stride q_abs_row_stride elements): the absorbed query the
 * attention entry points read. Replaces mla_absorb_q (glm_layer_runner.cuh:
 * 196-215) plus the q_rot half of the reference's mla_decode_absorbed input.
 *
 * wl_mla_project_v: ctx fp32 [n][n_heads][512] (row stride ctx_row_stride
 * floats, a multiple of 4) -> out[r][h][v] = sum_c ctx[r][h][c] *
 * kv_b[h*448 + 192 + v][c], fp32 [n][n_heads][256] (row stride out_row_stride).
 * Replaces mla_project_v (glm_layer_runner.cuh:217-234). fp32 accumulation.
 *
 * Both run on the tensor cores: the bf16 weight slice is the MMA's A operand
 * and each fp32 activation enters as three bf16 terms (hi + mid + lo, 24
 * significant bits), so the products accumulate in fp32 as exactly as the
 * reference's fp32 FMA loop (wl_indexer_query's projection likewise).
 * Under programmatic launch the weights (kv_b, wq_b) are fetched before the
 * wait on the previous kernel: a kernel that writes them must not signal an
 * early launch of its dependents (ordinary kernels do not). */
int wl_mla_absorb_q(const wl_attn_cfg* cfg, int32_t n, const float* q, int64_t q_row_stride,
                    const void* kv_b, void* q_abs, int64_t q_abs_row_stride, void* stream);
int wl_mla_project_v(const wl_attn_cfg* cfg, int32_t n, const float* ctx, int64_t ctx_row_stride,
                     const void* kv_b, float* out, int64_t out_row_stride, void* stream);

/* ---- the cache write path ---------------------------------------------------
 * Appends n tokens to the caches: for token i at row pos[i] of sequence seq[i]
 * (seq NULL: sequence 0), given the projections' outputs,
 *  - index key (owner layers; skipped when k_raw is NULL): LayerNorm of
 *    wk(x) with weight/bias (eps ln_eps), RoPE on its leading rope_dim dims,
 *    rounded to bf16 (the value the reference caches), then stored as
 *    fp8-e4m3 with the per-key scale amax / 448 into `index`;
 *  - latent row (skipped when kv_raw is NULL): the first kv_lora of
 *    kv_a_proj_with_mqa(x) RMS-normalised with the kv_a_layernorm weight (eps
 *    rms_eps), the trailing rope_dim roped, both stored as bf16 into `latent`.
 * RoPE is the interleaved-in, halves-out form with the token's table row
 * cos/sin [n][rope_dim/2] (the caller's table, as in the reference).
 * Replaces launch_indexer_key (glm_kernels.cuh:432-448) and the latent row
 * write of run_attention (glm_layer_runner.cuh:544-570). Rows outside
 * [0, cfg->T_max), and sequences outside [0, n_seq), set the device error
 * word and are skipped. The caches'
 * pointers are written through (their `const` is the readers' view). */
typedef struct wl_cache_append_io {
    int32_t n;                  /* tokens                                      */
    const int32_t* pos;         /* device [n]: cache row of each token         */
    const int32_t* seq;         /* device [n] or NULL: sequence of each token  */
    const float* cos;           /* device fp32 [n, rope_dim/2]                 */
    const float* sin;           /* device fp32 [n, rope_dim/2]                 */
    const float* k_raw;         /* device fp32 [n, idx_dim]: wk(x), or NULL    */
    const void*  k_norm_w;      /* device bf16 [idx_dim] LayerNorm weight      */
    const void*  k_norm_b;      /* device bf16 [idx_dim] LayerNorm bias        */
    float        ln_eps;        /* 1e-6 (INDEXER_LN_EPS)                       */
    wl_index_cache index;
    const float* kv_raw;        /* device fp32 [n, kv_lora + rope_dim], or NULL */
    const void*  kv_norm_w;     /* device bf16 [kv_lora] kv_a_layernorm weight */
    float        rms_eps;       /* 1e-6 (LORA_NORM_EPS)                        */
    wl_latent_cache latent;
    int32_t n_seq;              /* sequences the caches hold: every seq[i] must
                                   lie in [0, n_seq); 1 when seq is NULL        */
} wl_cache_append_io;

int wl_cache_append(const wl_attn_cfg* cfg, const wl_cache_append_io* io, void* stream);

/* ---- diagnostics ------------------------------------------------------------ */
/* Device-side error word of the calling thread's current device: bounds-check
 * failures and bounded-wait timeouts of any kernel of this library set it.
 * Synchronises the device. `clear` resets it to 0. Returns the WL_ERR_* code
 * (WL_OK when clean); *detail (may be NULL) receives the raw word. */
int wl_device_error(int32_t clear, uint32_t* detail);

/* Limit of every bounded device-side wait of this library on the current
 * device, in SM clock cycles (about 1 s by default; <= 0 restores the
 * default). Waits that run past it set the device error word (read by
 * wl_device_error as WL_ERR_TIMEOUT) and unwind; tests shorten it to make a
 * wait run out without hanging anything. */
int wl_diag_set_wait_limit(int64_t cycles);

/* Phase timeline of wl_attn_decode and wl_attn_decode_sharded. With a device
 * buffer set, every later call (or graph replay of one captured meanwhile)
 * writes the global timer (ns) into dev_buf[i] at its i-th phase boundary, up
 * to `cap` stamps in all; wl_diag_phase_count returns how many were issued
 * since the buffer was set. NULL turns stamping off. Boundaries of
 * wl_attn_decode: start | indexer | top-k | attention | merge (owner; a
 * consumer has no indexer or top-k stamps). Of wl_attn_decode_sharded over
 * peer memory: start | indexer | local top-k | candidate exchange | global
 * top-k | attention | (o, lse) reduce-scatter | all-gather; over
 * NCCL: start | indexer | local top-k | candidate exchange | global top-k |
 * attention | local merge | all-gather | merge. Stamping adds one tiny launch per
 * boundary and breaks the overlap between phases: a diagnostic, not a
 * measurement of the unstamped step. Not thread-safe across concurrent calls. */
int wl_diag_phase_stamps(uint64_t* dev_buf, int32_t cap);
int32_t wl_diag_phase_count(void);

/* The final (o, lse) merge of the sharded decode, run over a caller-provided
 * region in the peer-exchange wire format (8-byte words {payload, epoch}; part
 * s of row r at word s*slot_words + r*(64*512+64), its lse 64*512 words
 * further) with the epoch read from *epoch_ctr (device). Test hook for the
 * exchange's consumer: words whose epoch never matches make its bounded waits
 * run out. */
int wl_diag_merge_exchange(const void* region, int64_t slot_words, const uint32_t* epoch_ctr, int32_t n_rows,
                           int32_t n_parts, float* ctx, float* lse, void* stream);

/* The sharded decode's peer-memory (o, lse) combination (reduce-scatter by
 * heads, then all-gather) for `nranks` ranks emulated on the current GPU:
 * every stage runs for every emulated rank before the next stage starts, so
 * no wait depends on a kernel still to come. o_part [nranks][batch][nsplit]
 * [64][512] and lse_part [nranks][batch][nsplit][64] are each rank's split
 * partials; ctx [nranks][batch][64][512] and lse [nranks][batch][64] receive
 * every rank's result (all equal). `regions`: zeroed device memory of
 * wl_diag_xmerge_bytes(nranks) bytes (every rank's exchange region and
 * counters), 16-byte aligned. A test hook for the exchange's layout. */
size_t wl_diag_xmerge_bytes(int32_t nranks);
int wl_diag_xmerge(int32_t nranks, int32_t batch, int32_t nsplit, const float* o_part, const float* lse_part,
                   void* regions, size_t regions_bytes, float* ctx, float* lse, void* stream);

/* sizeof of each public struct, for binding checks: fills up to n entries in
 * the order cfg, latent_cache, index_cache, rows, index_share, decode_io,
 * prefill_io, shard, cache_append_io; returns how many exist. */
int32_t wl_struct_sizes(int64_t* out, int32_t n);
int32_t wl_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* WL_ATTN_H */
