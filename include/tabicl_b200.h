/*
 * tabicl_b200.h - C ABI of the B200 backend for tabicl-anywhere's prediction hot path.
 *
 * The entry points are what a Rust shim crate would bind to implement tabicl-anywhere's accelerator hook
 * `predict::AttendCached` (src/predict.rs:63-79) and the card tier around it (src/gpu.rs:2495-2701), reading the
 * same `.tirs` bundles byte for byte (src/store.rs:1-11). Plain pointers and sizes only. Every call returns a
 * status: TCU_OK (0), TCU_DECLINED (1, the caller's CPU path answers, as `Ok(None)` in predict.rs:58-61), or a
 * negative error; `tcu_last_error` then says why (gpu.rs:2525-2527).
 *
 * Threading: a context serialises the calls made on it (one in flight at a time); use one context per thread for
 * concurrency. Handles must not be used after they are freed; a model must be freed before its weights, and
 * weights before their context.
 */
#ifndef TABICL_B200_H
#define TABICL_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TCU_API __attribute__((visibility("default")))
#else
#define TCU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TCU_OK = 0,
    TCU_DECLINED = 1,
    TCU_ERR_ARG = -1,    /* bad argument (shape, pointer, range) */
    TCU_ERR_FORMAT = -2, /* bundle or tensor not as tabicl-anywhere writes it */
    TCU_ERR_CUDA = -3,   /* a CUDA call failed */
    TCU_ERR_MEMORY = -4, /* device or host memory exhausted */
    TCU_ERR_STATE = -5,  /* handle not ready (weights or layers missing) */
    TCU_ERR_IO = -6,     /* file could not be read */
};

/* Stored number format of the in-context keys and values: the codes of `fit::Kv` (src/fit.rs:103-122), which a
 * fitted member stores in `m{i}/meta[4]`. */
enum { TCU_KV_F32 = 0, TCU_KV_I16 = 1, TCU_KV_I8 = 2 };

typedef struct tcu_ctx tcu_ctx;         /* one device and its stream: gpu::Gpu (src/gpu.rs:725-747) */
typedef struct tcu_weights tcu_weights; /* in-context weights on the device: gpu::GpuWeights (src/gpu.rs:1838-2028) */
typedef struct tcu_model tcu_model;     /* one fitted problem's cache on the device: gpu::VramModel (src/gpu.rs:2033-2116) */

/* Sizes of the in-context stage (src/model.rs:110-143): width d, heads, layers, feed-forward width ff
 * (linear1 rows), scalable-softmax hidden width hid (query_mlp.0 rows), decoder hidden dec_ff (decoder.0 rows),
 * decoder outputs outs (decoder.2 rows), max_classes (0 for a regression model). */
typedef struct {
    int32_t d, heads, layers, ff, hid, dec_ff, outs, max_classes;
} tcu_icl_shape;

/* Sizes of the column and row stages (src/model.rs:199-245): width e, features per group, inducing points, class
 * tokens, heads of the column stage's attention and of the row blocks, column blocks (ISABs) and row blocks, and
 * their feed-forward widths (linear1 rows). */
typedef struct {
    int32_t e, group, inds, cls, col_heads, row_heads, col_blocks, row_blocks, col_ff, row_ff;
} tcu_rows_shape;

/* ---- context ---------------------------------------------------------------------------------------------- */

/* Open device `device` (gpu::Gpu::new_async, src/gpu.rs:930-971). */
TCU_API int tcu_open(int device, tcu_ctx **out);
TCU_API void tcu_close(tcu_ctx *ctx);
/* Why the last failing call on this context failed ("" if none): VramTier::last_error (src/gpu.rs:2525-2527). */
TCU_API const char *tcu_last_error(const tcu_ctx *ctx);
/* Kernels this context has launched so far (each of this library's own kernels counts once per launch). */
TCU_API uint64_t tcu_launches(const tcu_ctx *ctx);

/* ---- weights (GpuWeights::new, src/gpu.rs:1876; tensor names of src/model.rs:52-98, 236-270) --------------- */

/* Empty weights of this shape; `for_fit` also keeps what fitting needs (key/value rows of in_proj, the
 * scalable softmax's base MLP, the target embedding). */
TCU_API int tcu_weights_new(tcu_ctx *ctx, const tcu_icl_shape *shape, int for_fit, tcu_weights **out);
/* One tensor by its bundle name (e.g. "icl_predictor.tf_icl.blocks.3.linear1.weight"), `count` elements of
 * dtype 0 = float32 or 1 = float16 (widened exactly, src/store.rs:363-375). Names the stage does not use are
 * ignored; a layer norm bias never put is zero (src/model.rs:56-57, 261-266). */
TCU_API int tcu_weights_put(tcu_weights *w, const char *name, int dtype, const void *data, size_t count);
/* Upload to the device; every needed tensor must have been put. */
TCU_API int tcu_weights_ready(tcu_weights *w);
/* The whole of the above from a weight bundle file (Model::load, src/model.rs:202-272, in-context part). */
TCU_API int tcu_weights_from_bundle(tcu_ctx *ctx, const char *path, int for_fit, tcu_weights **out);
TCU_API int tcu_weights_shape(const tcu_weights *w, tcu_icl_shape *out);
/* Also keep the column and row stages of this shape (their tensors "col_embedder.*" and "row_interactor.*" put with
 * tcu_weights_put; only the column blocks' second attention is needed, src/model.rs:226-231): call before
 * tcu_weights_ready. tcu_weights_from_bundle does this itself when the bundle has them. */
TCU_API int tcu_weights_set_rows_shape(tcu_weights *w, const tcu_rows_shape *shape);
/* The column and row stages' sizes; TCU_DECLINED when the weights have none. */
TCU_API int tcu_weights_rows_shape(const tcu_weights *w, tcu_rows_shape *out);
TCU_API void tcu_weights_free(tcu_weights *w);

/* ---- resident caches (VramTier::preload / Gpu::load, src/gpu.rs:2546-2556, 2062-2116) ------------------------ */

/* A problem of a fitted member: `meta` is the member's `m{i}/meta` ([rows, features, classes, chunk, kv, digits,
 * nodes], src/fit.rs:291); node_rows / node_k the problem's rows and outputs from `m{i}/tree`
 * (src/predict.rs:137-161). */
TCU_API int tcu_model_new(tcu_weights *w, const int32_t meta[7], int32_t node_rows, int32_t node_k, tcu_model **out);
/* `n{node}_scale`, [layers][d] floats (src/fit.rs:746). */
TCU_API int tcu_model_put_scales(tcu_model *m, const float *scales, size_t count);
/* Bytes [offset, offset + nbytes) of `n{node}_kv{layer}`, exactly as stored (no repacking; src/fit.rs:224-241). */
TCU_API int tcu_model_put_layer(tcu_model *m, int layer, size_t offset, const void *bytes, size_t nbytes);
/* The column stage's cache `m{i}/col_kv` (src/fit.rs:230): [features][digits][column blocks][2][e][inds] floats, the
 * keys then the values ([e][inds] each) of every feature group's inducing points. Needed by the `rows` hook. A cache
 * made by tcu_fit_icl_device takes its feature count from `count` (one label digit). */
TCU_API int tcu_model_put_col_kv(tcu_model *m, const float *col_kv, size_t count);
/* The member's feature count and label digits (meta[1] and meta[5]) for a cache made by tcu_fit_icl_device, before
 * its col_kv is put (a member of more classes than the model tells apart has several digits, src/fit.rs:159-184). */
TCU_API int tcu_model_set_columns(tcu_model *m, int features, int digits);
/* The whole of the above from a fitted bundle file, member `prefix` ("m0/", or "" for a raw fit), problem node
 * (col_kv too when the bundle holds it). */
TCU_API int tcu_model_from_bundle(tcu_weights *w, const char *path, const char *prefix, int node, tcu_model **out);
/* Device bytes the cache holds (Gpu::model_bytes, src/gpu.rs:2064-2068, for tier budgets): the stored records,
 * scales, column cache and tables, and the tensor-core attention's pre-split copy of the keys and values (head width
 * 128), counted from creation although the first call builds it. Working memory that grows with the rows of a call
 * is not counted. */
TCU_API size_t tcu_model_bytes(const tcu_model *m);
/* Copy back a layer's stored bytes / the scales (for writing a bundle after a device fit). */
TCU_API int tcu_model_get_layer(const tcu_model *m, int layer, void *bytes, size_t nbytes);
TCU_API int tcu_model_get_scales(const tcu_model *m, float *scales, size_t count);
TCU_API void tcu_model_free(tcu_model *m);

/* ---- AttendCached (src/predict.rs:63-79) --------------------------------------------------------------------- */

/* `attend`: attention outputs [rows][d] (before the output projection) for scaled queries q [rows][d] against
 * in-context layer `layer`. Host buffers. */
TCU_API int tcu_attend(tcu_model *m, int layer, const float *q, int rows, int d, int heads, float *out);
/* `stage`: the whole in-context stage, row representations h [rows][d] to the first out_n decoder outputs per
 * row [rows][out_n]. Host buffers; h is not modified. */
TCU_API int tcu_stage(tcu_model *m, const float *h, int rows, int d, int out_n, float *out);
/* The same two on device buffers, queued on `stream` (a cudaStream_t; NULL = the context's stream); inputs are
 * not modified. Their kernels run after the call returns: a kernel that gives up a bounded wait (a lost matrix
 * unit, a copy that never lands) marks the outputs of the calls queued since as invalid, and that is reported by
 * the next call on the context, by tcu_sync, or by a host-buffer form (TCU_ERR_CUDA, `tcu_last_error` naming the
 * wait). The context stays usable: the next call starts clean. */
TCU_API int tcu_attend_device(tcu_model *m, int layer, const float *q, int rows, float *out, void *stream);
TCU_API int tcu_stage_device(tcu_model *m, const float *h, int rows, int out_n, float *out, void *stream);
/* `rows`: all three stages for normalised rows x [rows][features] (prep's output, missing cells -100): the column stage
 * (predict::embed, src/predict.rs:282-353; with several label digits, once per digit and averaged), the row stage
 * (predict::represent, src/predict.rs:356-372), then the in-context stage; the first out_n decoder outputs per row
 * [rows][out_n]. Host buffers. TCU_DECLINED when the weights have no column and row stages or the cache no col_kv
 * (the caller's CPU path answers, as for `stage`). The reference calls this hook only for a member of one node
 * (src/predict.rs:642-652). */
TCU_API int tcu_rows(tcu_model *m, const float *x, int rows, int features, int out_n, float *out);
/* The same on device buffers, queued on `stream` (NULL = the context's stream). */
TCU_API int tcu_rows_device(tcu_model *m, const float *x, int rows, int out_n, float *out, void *stream);
/* Its two first stages alone, on device buffers: tokens tok [rows][cls + features][e] of normalised rows x, and row
 * representations rep [rows][cls e] of tokens (tok is used as scratch). */
TCU_API int tcu_embed_device(tcu_model *m, const float *x, int rows, float *tok, void *stream);
TCU_API int tcu_represent_device(tcu_model *m, float *tok, int rows, float *rep, void *stream);
/* Wait for `stream` (NULL = the context's stream) and report kernels that gave up since the last report
 * (TCU_ERR_CUDA), as cudaStreamSynchronize plus a check; no counterpart in the reference, whose card calls block. */
TCU_API int tcu_sync(tcu_ctx *ctx, void *stream);
/* Test hook (no counterpart in the reference): the next one-kernel stage launch on this context starts as if a
 * wait had given up, so that the give-up path (every CTA leaving at its next barrier after its copies land) and
 * its report can be exercised without making any wait run out. */
TCU_API int tcu_debug_abort_next(tcu_ctx *ctx);

/* ---- a whole member: its problems and the class tree (src/predict.rs:638-699) ----------------------------------- */

typedef struct tcu_member tcu_member;
/* A member of n_nodes problems, node i = nodes[i] (each made on the same weights), with its tree `m{i}/tree`
 * ([leaf, rows, k, map[k]] per node, src/fit.rs:217-220) over `classes` classes. A
 * leaf's map holds classes, an inner node's its children; the walk starts at node 0; every node's k is at most the
 * decoder's outputs (its stage returns its first k). Node 0 holds the column stage's
 * cache (col_kv) for tcu_member_rows. On success the member owns the nodes (tcu_member_free frees them); on failure
 * they stay the caller's. TCU_ERR_FORMAT for a tree that is damaged, reaches a node twice or names a class or node
 * out of range. */
TCU_API int tcu_member_new(tcu_model *const *nodes, int n_nodes, const int32_t *tree, size_t tree_len, int classes,
                           tcu_member **out);
/* Every problem of member `prefix` of a fitted bundle (src/predict.rs:138-161), col_kv into node 0. */
TCU_API int tcu_member_from_bundle(tcu_weights *w, const char *path, const char *prefix, tcu_member **out);
TCU_API int tcu_member_nodes(const tcu_member *m);
TCU_API int tcu_member_classes(const tcu_member *m);
/* Problem `node` (owned by the member), for the per-problem `stage` hook; NULL when out of range. */
TCU_API tcu_model *tcu_member_node(tcu_member *m, int node);
TCU_API size_t tcu_member_bytes(const tcu_member *m);
/* predict_raw's pass (src/predict.rs:638-699) for normalised rows x [rows][features]: the column and row stages once,
 * the in-context stage of every problem, then for a tree each problem's scores as probabilities (temperature 0.9)
 * multiplied down the tree and back to scores 0.9 ln(p + 1e-6); a member of one problem returns its decoder outputs
 * as they are. out [rows][classes]. Host buffers (the `_device` form: device buffers queued on `stream`). */
TCU_API int tcu_member_rows(tcu_member *m, const float *x, int rows, int features, float *out);
TCU_API int tcu_member_rows_device(tcu_member *m, const float *x, int rows, float *out, void *stream);
/* The tree step alone (src/predict.rs:664-692): every problem's scores laid end to end (problem i's [rows][k_i]
 * after those of problems 0..i-1) to class scores out [rows][classes]. Device buffers. */
TCU_API int tcu_member_combine_device(tcu_member *m, const float *scores, int rows, float *out, void *stream);
TCU_API void tcu_member_free(tcu_member *m);

/* ---- the card tier (gpu::VramTier and its handle, src/gpu.rs:2450-2701; the ledger of src/warm.rs:28-115) ------- */

typedef struct tcu_tier tcu_tier;     /* fitted problems resident on one device for many tenants */
typedef struct tcu_handle tcu_handle; /* one tenant's use of the tier for one fitted bundle: an AttendCached */
typedef struct tcu_pin tcu_pin;       /* test hook: a problem held as a prediction holds it */
/* A bundle read through the caller's positional reads (ReadAt, src/store.rs:45-50: a file, memory, object storage,
 * a sealed bundle decrypted as it is read): read_at fills buf with n bytes at offset and returns 0, nonzero on failure.
 * Called from the tier's loading threads, possibly at once: it must be safe to call concurrently, and `user` must
 * outlive the handle and every load it started. */
typedef struct {
    void *user;
    int (*read_at)(void *user, uint64_t offset, void *buf, size_t n);
    uint64_t size;
} tcu_source;

/* VramTier::new (gpu.rs:2512-2514): `budget` bytes of fitted problems on the device in all, `tenant_budget` (at most
 * `budget`) per tenant. background nonzero: a first prediction starts its problem's load on a thread of its own and
 * declines meanwhile (natively, gpu.rs:2690-2698); zero: the load runs in that call, which then answers (gpu.rs:
 * 2683-2689). ctx NULL: a tier that only keeps its books (the tcu_tier_debug_* entry points), without a device. */
TCU_API int tcu_tier_new(tcu_ctx *ctx, size_t budget, size_t tenant_budget, int background, tcu_tier **out);
/* Waits for loads in flight, then releases every problem not in use (handles must be freed before the tier). */
TCU_API void tcu_tier_free(tcu_tier *t);
/* Wait until no load started by a prediction is still running. */
TCU_API void tcu_tier_wait(tcu_tier *t);
/* Bytes the tier holds, in all and by `tenant` (problems being loaded included) (gpu.rs:2517-2519). */
TCU_API void tcu_tier_held(tcu_tier *t, const char *tenant, size_t *all, size_t *mine);
/* Bytes of `tenant`'s problems that are loaded and ready (gpu.rs:2522-2524). */
TCU_API size_t tcu_tier_ready(tcu_tier *t, const char *tenant);
/* Bytes really on the device, in all and of `tenant`: what the tier holds plus what was evicted but is still in use
 * by a prediction; never more than the budgets (gpu.rs:2528-2531). */
TCU_API void tcu_tier_on_card(tcu_tier *t, const char *tenant, size_t *all, size_t *mine);
/* Predictions the device was asked for but declined because it failed, and the last reason (gpu.rs:2504-2506,
 * 2534-2536): the reason's length (0: none), copied NUL-terminated into buf[n]. */
TCU_API uint64_t tcu_tier_fallbacks(const tcu_tier *t);
TCU_API size_t tcu_tier_last_error(tcu_tier *t, char *buf, size_t n);
/* Release everything `tenant` holds (for `model` only, if not NULL); problems in use by a prediction are released
 * when it finishes (gpu.rs:2538-2542). */
TCU_API void tcu_tier_evict(tcu_tier *t, const char *tenant, const char *model);
/* VramTier::handle (gpu.rs:2545-2547): tenant `tenant`'s use of fitted bundle `model` (a name of the caller's) read
 * from a file or a source, with weights w (which must outlive the handle and its loads). */
TCU_API int tcu_tier_handle(tcu_tier *t, const char *tenant, const char *model, const char *bundle_path, tcu_weights *w,
                            tcu_handle **out);
TCU_API int tcu_tier_handle_source(tcu_tier *t, const char *tenant, const char *model, const tcu_source *src,
                                   tcu_weights *w, tcu_handle **out);
TCU_API void tcu_handle_free(tcu_handle *h);
/* VramTier::preload (gpu.rs:2550-2558) of problem `node` of member `prefix`, now: 1 resident afterwards, 0 the budgets
 * do not allow it (now, or ever), < 0 the load failed (tcu_tier_last_error says why). */
TCU_API int tcu_handle_preload(tcu_handle *h, const char *prefix, int node);
/* The handle's AttendCached hooks (gpu.rs:2636-2656), host buffers, as tcu_attend / tcu_stage / tcu_rows: TCU_OK, or
 * TCU_DECLINED when the problem is not resident (its load is started), too large for its tenant, without the column
 * cache (rows: kept only for a member of one problem and one label digit), or when the device failed (counted in
 * fallbacks, the reason kept). */
TCU_API int tcu_handle_attend(tcu_handle *h, const char *prefix, int node, int layer, const float *q, int rows, int d,
                              int heads, float *out);
TCU_API int tcu_handle_stage(tcu_handle *h, const char *prefix, int node, const float *x, int rows, int d, int out_n,
                             float *out);
TCU_API int tcu_handle_rows(tcu_handle *h, const char *prefix, const float *x, int rows, int features, int out_n,
                            float *out);
/* Test hooks (no counterpart in the reference), the tier's books without a device: admit a ready entry of `bytes`
 * for (tenant, model, prefix, node) through the same claim as a load (1 admitted, 0 no room); hold a ready entry as a
 * prediction holds its problem (1, or 0 when it is not ready) until unpinned. */
TCU_API int tcu_tier_debug_admit(tcu_tier *t, const char *tenant, const char *model, const char *prefix, int node,
                                 size_t bytes);
TCU_API int tcu_tier_debug_pin(tcu_tier *t, const char *tenant, const char *model, const char *prefix, int node,
                               tcu_pin **out);
TCU_API void tcu_tier_debug_unpin(tcu_pin *p);

/* ---- heads (src/table.rs) ------------------------------------------------------------------------------------ */

/* Classifier::logit_sums_async (src/table.rs:265-269) for one member: sums[r][c] += logits[r][classes_of[c]]
 * in f64; then finish_proba (src/table.rs:70-78) when `finish` is nonzero (members, temperature). Device
 * buffers on the context stream. */
TCU_API int tcu_class_head_device(tcu_ctx *ctx, const float *logits, int rows, int classes, int stride,
                          const int32_t *member_classes, double *sums, int finish, int members, double temperature);
/* Regressor::predict_async (src/table.rs:457-496) for one member: each row's nq quantile outputs read as a
 * QuantileDist (src/table.rs:292-346); mean, variance, median and the quantiles at alphas, back-transformed,
 * ADDED to the f64 outputs (divide by the member count at the end). Device buffers. */
TCU_API int tcu_regression_head_device(tcu_ctx *ctx, const float *qout, int rows, int nq, int stride, const double *alphas,
                               int na, double target_mean, double target_scale, double *mean, double *variance,
                               double *median, double *quantiles);

/* ---- fitting on the device (src/fit.rs:285-747) ------------------------------------------------------------- */

/* The accelerator hooks of fit::Attend (src/fit.rs:25-74), host buffers in and out. */
/* fit::Attend::column_batch (src/fit.rs:54-56): feature groups tcu_fit_columns takes at once for `rows` training rows
 * (0: not offered, as for weights without the column stage's fit tensors). */
TCU_API int tcu_fit_column_batch(const tcu_weights *w, int rows);
/* fit::Attend::columns (src/fit.rs:33-38, 57-59, called at 426-448): the column stage of `groups` feature groups for
 * one label digit. cells [rows][groups][e] (through the input layer, the target's embedding added) is replaced by the
 * cells after the stage; ind_q [column blocks][inds][e] holds each block's inducing-point queries, scaled; rec
 * receives [groups][column blocks][2][e][inds]. */
TCU_API int tcu_fit_columns(tcu_weights *w, float *cells, int rows, int groups, const float *ind_q, float *rec);
/* fit::Attend::row_batch (src/fit.rs:60-62): rows tcu_fit_rows takes at once for tables of `features` features. */
TCU_API int tcu_fit_row_batch(const tcu_weights *w, int features);
/* fit::Attend::rows (src/fit.rs:39, 63-65, called at 493-518): the row stage of n rows, cells [n][features][e] to
 * reps [n][d]. */
TCU_API int tcu_fit_rows(tcu_weights *w, const float *cells, int n, int features, float *reps);
/* Receives layer `layer`'s keys and values, [rows][d] each (host, valid during the call); nonzero stops the pass. */
typedef int (*tcu_layer_sink)(void *user, int layer, const float *k, const float *v);
/* fit::Attend::in_context (src/fit.rs:66-71, called at 622): the whole in-context stage of one problem. h
 * [rows][d] (host): the row representations with the target's embedding added; scales [layers][d] (host): each
 * layer's query scale. `sink` is called once per layer, in order. Weights made with for_fit. */
TCU_API int tcu_fit_in_context(tcu_weights *w, const float *h, int rows, const float *scales, tcu_layer_sink sink,
                               void *user);

/* The column and row stages of fitting one member (src/fit.rs:298-540; fit_raw_async's column stage 300-481 and row
 * stage 487-540). x: normalised training rows (device [rows][features]); y: their labels (device [rows]: class
 * indices as floats, or standardised targets); `digits` label digits of mixed-radix `bases` (host [digits], each at
 * least 2; unused for one digit: the label itself). Writes col_kv (device [features][digits][column blocks][2][e]
 * [inds]: the member's `m{i}/col_kv`, src/fit.rs:230) and rep (device [rows][d]: the training rows' representations,
 * which tcu_fit_icl_device takes per node of the class tree). `w` made with for_fit from a bundle that holds the
 * column stage's first attention and label embedding; TCU_DECLINED otherwise. Working memory is taken and freed in
 * the call; returns once the results are written. */
TCU_API int tcu_fit_rows_device(tcu_weights *w, const float *x, const float *y, int rows, int features, int digits,
                                const int32_t *bases, float *col_kv, float *rep, void *stream);

/* Training rows h [rows][d] (device; consumed) with targets y [rows] (device; class index or standardised
 * value) to a resident cache: every layer's keys and values packed as `kv` in chunks of `chunk` rows
 * (src/fit.rs:549-576) and the query scales. `w` must have been made with for_fit. */
TCU_API int tcu_fit_icl_device(tcu_weights *w, float *h, const float *y, int rows, int chunk, int kv, tcu_model **out);

/* Pack one chunk: c [2d][rc] floats (device) to its stored record (device, tcu_record bytes): src/fit.rs:549-576. */
TCU_API int tcu_pack_device(tcu_ctx *ctx, int kv, int d, int rc, const float *c, void *rec);
/* Bytes of a stored chunk of rc rows (src/fit.rs:124-126). */
TCU_API size_t tcu_record(int kv, int d, int rc);
/* The accelerator load helper `layer_rows` (src/predict.rs:590-629) on the device: one layer's stored chunks
 * `layer` (device, `rows` cached rows in chunks of `chunk`, format kv) widened to keys k and values v [rows][d]
 * (device floats; integers times their coordinate's scale), with the same vector widening the attention kernels
 * read the cache through. Synchronises the context stream. */
TCU_API int tcu_layer_rows_device(tcu_ctx *ctx, int kv, int d, const void *layer, int rows, int chunk, float *k, float *v);

/* Few-row attention that allocates nothing (no counterpart in the reference; an addition for callers that cannot
 * call cudaMalloc: code running while a CUDA graph is captured, hosts whose device memory belongs to an arena or
 * another runtime's allocator, and real-time paths that cannot accept an allocation's latency or failure).
 * Same result as tcu_attend_device: the attention outputs out [nq][d] (device) of scaled queries q [nq][d]
 * (device) against one layer's stored keys/values `layer` (device, the n{j}_kv{l} bytes of `rows` cached rows in
 * chunks of `chunk`, format kv), queued on `stream` (a cudaStream_t; NULL = the legacy default stream). No
 * context or handle is needed. Its scratch is one static device array of TCU_NOALLOC_SCRATCH_BYTES (16 MiB) in
 * every context that loads this library, kept until the process exits; a call is refused with TCU_ERR_ARG (and a
 * message in `err`, if given) when nq > TCU_NOALLOC_MAX_ROWS, when the cache has more than TCU_NOALLOC_MAX_ITEMS
 * key slices of 32-64 rows, or when the work does not fit the scratch (it fits 32 query rows at 10,000 cached
 * rows of width 512 stored as i16, about 4 at 100,000), or when `layer`, `q` or `out` is not 4-byte aligned (the
 * chunk records' scales and the queries are read as floats). The first call on each device looks the scratch's
 * address up (with that device current): make it before any stream capture. Every call shares the scratch and it keeps the last call's contents (each call
 * writes all it reads, so nothing must start at zero): calls that overlap on the GPU - on two streams, or from
 * two threads - race and give wrong answers; serialise them. */
#define TCU_NOALLOC_SCRATCH_BYTES (16 << 20)
#define TCU_NOALLOC_MAX_ROWS 32
#define TCU_NOALLOC_MAX_ITEMS 8192
TCU_API int tcu_attend_noalloc(int kv, int d, int heads, const void *layer, int rows, int chunk, const float *q, int nq,
                               float *out, void *stream, char *err, size_t err_cap);

/* Self-test of the tensor-core path (no counterpart in the reference): small exact products on the tcgen05 units
 * against CUDA cores, for every operand layout the attention uses. *max_err is the largest difference (0 when
 * the layouts are right), or -1 if the matrix units never answered. */
TCU_API int tcu_selftest_mma(tcu_ctx *ctx, double *max_err);

/* Measurement hook (no counterpart in the reference, which times stages with wall clocks, src/predict.rs:20-56):
 * while enabled, every attention pass (one layer's attention kernels) is bracketed by CUDA events on its stream.
 * A call reads the total device time and count of the passes since the last call (when the pointers are set,
 * after synchronising the device), then enables or disables timing and starts a new count. Stages replayed from
 * a CUDA graph re-record the same events each replay, so for them the count covers the last replay. */
TCU_API int tcu_profile(tcu_ctx *ctx, int enable, double *attend_ms, uint64_t *attend_launches);

/* ---- several devices (no counterpart in the reference, which runs on one device) ----------------------------------
 *
 * A cache too large for one device, or wanted faster, is split along its training rows: device g holds whole chunks
 * [c0_g, c1_g) of every layer (tcu_model_slice). The chunk records are unchanged, so a shard is an ordinary cache of
 * fewer rows; it keeps the full cache's query scales (they depend on the full row count, src/nn.rs:97-107). In the
 * stage each device attends over its own rows and the partial softmax states (max, weight sum, weighted values;
 * src/nn.rs:187-286) are merged over all devices after every layer: an all-reduce (max) of the maxima, a rescale to
 * the common max, an all-reduce (sum) of the states, a division. Everything else runs on every device alike.
 *
 * tcu_comm wraps an NCCL communicator over the devices (libnccl.so.2 is loaded when the first one is made). Rank 0
 * makes the id with tcu_comm_unique_id and passes it to the other ranks out of band (torch.distributed, MPI, a
 * file); every rank then calls tcu_comm_init with it, which returns once all have joined. Every rank must take the
 * same collective steps in the same order: call the sharded stage with the same rows and out_n everywhere. */
typedef struct tcu_comm tcu_comm;
#define TCU_COMM_ID_BYTES 128
TCU_API int tcu_comm_unique_id(uint8_t id[TCU_COMM_ID_BYTES]);
TCU_API int tcu_comm_init(tcu_ctx *ctx, const uint8_t id[TCU_COMM_ID_BYTES], int nranks, int rank, tcu_comm **out);
TCU_API void tcu_comm_free(tcu_comm *c);
/* Sum `count` doubles over all ranks in place (device buffer), e.g. per-rank class-logit sums of ensemble members
 * placed one per device. Queued on `stream` (NULL: the context's stream). */
/* Abort the communicator now (ncclCommAbort): for a rank that learned on the host that a peer has left, so that
 * nothing waits on it; every later collective on it fails with TCU_ERR_STATE. */
TCU_API int tcu_comm_abort(tcu_comm *c);
TCU_API int tcu_comm_allreduce_f64(tcu_comm *c, double *buf, size_t count, void *stream);
/* Wait up to timeout_ms for `stream` (NULL: the context's stream); on timeout the communicator is aborted, so that
 * collectives still waiting for a lost rank end, and TCU_ERR_CUDA is returned. The communicator is unusable after. */
TCU_API int tcu_comm_wait(tcu_comm *c, void *stream, int timeout_ms);

/* A new resident cache holding chunks [first_chunk, first_chunk + nchunks) of `m` (device-to-device copies) with
 * m's query scales. */
TCU_API int tcu_model_slice(const tcu_model *m, int first_chunk, int nchunks, tcu_model **out);
/* The stage of `rows` rows (h, out device buffers as in tcu_stage_device, the same rows on every rank) with `m`
 * holding this rank's shard of the training rows (predict.rs:398-409, 521-532 with the readers on separate devices).
 * The rows are padded to equal slices of ceil(rows / ranks), one per rank. Every layer, each rank attends all rows
 * over its shard; the partial states (max, weight sum, weighted values per row and head) of each slice go to the rank
 * owning it, which merges them (nn.rs:261-286) and runs the rest of the layer and the next layer's query for its
 * slice only; every rank then receives all queries. The exchanges are stores into the peers' memory over NVLink
 * (CUDA IPC mappings set up at the first call, flags with bounded waits; a wait that gives up is reported as for the
 * other kernels), or, where the mappings are not available on every rank (or with TCU_SHARD_P2P=0), NCCL: an
 * all-reduce of the maxima, a reduce-scatter of the states scaled to them and an all-gather of the queries. Every rank
 * ends with all rows' outputs. Queued on `stream` (NULL: the context's stream). */
TCU_API int tcu_stage_sharded_device(tcu_model *m, tcu_comm *c, const float *h, int rows, int out_n, float *out,
                                     void *stream);
/* Phases of tcu_stage_sharded_device timed by tcu_comm_breakdown: attention over the shard; merge of its splits (and
 * the states' maxima); the exchange of states (peer stores and the wait for every rank's, or the all-reduce of the
 * maxima, the scaling and the reduce-scatter); the merge over ranks (or the division of the summed states); the rest
 * of each layer and the next query; the exchange of queries; the decoder and the gather of outputs. */
enum { TCU_SHARD_PHASES = 7 };
/* ms (NULL: only switch): the device time of each phase in the last sharded call made while timing was on (summed
 * over layers; waits for that call); then timing on for the following calls when `enable` is nonzero. */
TCU_API int tcu_comm_breakdown(tcu_comm *c, int enable, double *ms);

#ifdef __cplusplus
}
#endif
#endif
