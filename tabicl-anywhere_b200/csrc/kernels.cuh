// Launch interface of the prediction-path kernels (kernels.cu). All launches are asynchronous on `stream`.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <vector_types.h>

namespace tcu {

// y (=|+=) act(W LN?(x) + b): x [M][K] (row stride ldx), W [N][K], y [M][N] (row stride ldy).
struct LinArgs {
    const float *x = nullptr;
    int ldx = 0, M = 0, K = 0;
    const float *lnw = nullptr, *lnb = nullptr;  // LayerNorm of each input row first (eps 1e-5), if set
    const float *stats = nullptr;                // [M][2] mean, 1/sigma of the input rows (tiled path)
    const float *W = nullptr, *bias = nullptr;
    int N = 0;
    float *y = nullptr;
    int ldy = 0;
    int act = 0;         // 1: GELU (kern.rs:285-290)
    int accumulate = 0;  // 1: y += result (residual)
    int bias_on_m = 0;   // bias indexed by the row of y (used when y is a transposed product)
    int transpose_out = 0;  // write y[n][m] (row stride ldy) instead of y[m][n]
    // tensor-core path: W split once into f16 hi + lo, scaled per output row by 1 / unscale[n], in 128 x 64 blocks
    // ([N / 128][K / 64][hi 128 x 64][lo 128 x 64], core-matrix order); tc_atiles: scratch of tc_split_bytes(M, K)
    // bytes for the split input rows
    const void *tc_wtiles = nullptr;
    const float *tc_wunscale = nullptr;
    void *tc_atiles = nullptr;
    size_t tc_atiles_bytes = 0;
    int *err = nullptr;  // report slot (host memory, mapped): set to 1 when the kernel gave up waiting
};

// The query MLP of many rows (nn.rs:138-149) in one tensor-core kernel: q [pairs][hd] as (row, head) pairs, in place.
struct QmlpArgs {
    float *q = nullptr;
    int pairs = 0, heads = 0, hd = 0, hid = 0;
    const void *w0_tiles = nullptr, *w2_tiles = nullptr;  // W0 [hid][hd], W2 [hd][hid] split as for the linear layers
    const float *w0_unscale = nullptr, *w2_unscale = nullptr, *b0 = nullptr, *b2 = nullptr;
    const float *scale = nullptr;  // [heads * hd] the layer's fit-time query scale
    int *err = nullptr;  // report slot (host memory, mapped): set to 1 when the kernel gave up waiting
};

// Attention of scaled queries against one layer's stored chunks (fit.rs:6-11 layout, read in place).
struct AttnArgs {
    const uint8_t *layer = nullptr;
    int rows = 0, chunk = 0, d = 0, heads = 0;
    size_t full = 0;               // bytes of a full chunk record
    const int2 *items = nullptr;   // decode: (chunk, first key) per item
    int nitems = 0;
    const int4 *tiles = nullptr;   // flash: (chunk, first key, keys) per 64-key tile
    int ntiles = 0, tiles_per_split = 0, splits = 1;
    const float *q = nullptr;      // [R][d] scaled queries (row stride ldq)
    int ldq = 0, R = 0;
    float *part_ms = nullptr;      // [parts][R][heads][2]: running max, weight sum
    float *part_acc = nullptr;     // [parts][R][d]: weighted value sums
    float *out = nullptr;          // [R][d] finished outputs (row stride ldo)
    int ldo = 0;
    int tc_eK = 0, tc_eV = 0;      // tensor-core path: power-of-two scalings of the keys and values
    int *err = nullptr;            // report slot (host memory, mapped): set to 1 when the kernel gave up waiting
    int parts_only = 0;            // 1: always leave parts (no merge), even with a single split
    // tensor-core path: when set, the result is the merged state left unnormalised: out [R][ldo] the weighted values,
    // state_ms [R][heads][2] the (max, weight sum) they are relative to (one split, or splits merged in the kernel)
    float *state_ms = nullptr;
    const void *tc_tiles = nullptr;  // tensor-core path: the layer's tiles pre-split by launch_tc_tiles
    int *merge_cnt = nullptr;  // tensor-core path: [R / 128][heads] arrival counters (zero between launches); when
                               // set, the last split of each (row block, head) merges the parts itself
};

// The few-row stage in one persistent kernel: per layer, the pointers it reads.
struct RowsLayer {
    const float *n1w, *n1b, *wq, *bq, *q0w, *q0b, *q2w, *q2b, *wo, *bo, *n2w, *n2b, *w1, *b1, *w2, *b2;
    const uint8_t *cache;  // the layer's stored chunks (fit.rs:6-11 layout)
    const float *scale;    // [d] fit-time query scale of the layer (nn.rs:97-107)
};

constexpr int ROWS_MAX_HEADS = 16;
constexpr int ROWS_MAX_LAYERS = 16;
constexpr int ROWS_MAX_GRID = 160;

struct RowsArgs {
    const RowsLayer *layers = nullptr;  // [L], device memory
    int L = 0, d = 0, heads = 0, ff = 0, dff = 0, out_n = 0, R = 0;
    const float *lnw = nullptr, *lnb = nullptr, *dec0w = nullptr, *dec0b = nullptr, *dec2w = nullptr, *dec2b = nullptr;
    int rows = 0, chunk = 0;
    size_t full = 0;                    // bytes of a full chunk record
    // key tiles, head-major: (chunk, first key, keys, head | 1 << 16 when its rows can be bulk-copied)
    const int4 *tiles = nullptr;
    int ntiles = 0, tiles_per_head = 0;
    int slots = 0;                      // tiles of shared memory per CTA
    // TMA tensor maps per layer, device memory: [L][2] CUtensorMap (the full chunks as bytes x coordinates x chunks,
    // then the last, shorter chunk as bytes x coordinates); tiles flagged aligned are loaded through them
    const void *tmaps = nullptr;
    int nfull = 0;                      // full chunks per layer
    float *h = nullptr, *q = nullptr, *att = nullptr, *mid = nullptr, *out = nullptr;
    // per CTA (each holds tiles of one head: CTA c of grid G takes head c / (G / heads)): [grid][R] (max, weight
    // sum) and [grid][R][head width]
    float *part_ms = nullptr, *part_acc = nullptr;
    unsigned *bar = nullptr;            // grid barrier word (zero low bits between launches)
    int *err = nullptr;                 // abort word (device memory, zeroed before each launch): set when a wait
                                        // gave up, every CTA then leaves at its next barrier
    int *err_report = nullptr;          // report slots (host memory, mapped): [0] a grid barrier gave up, [1] a
                                        // tile's copy did not arrive, [2] the CTA left because another gave up
    // diagnostics (null: off): [grid][ROWS_TRACE_MARKS] global-timer nanoseconds, thread 0 of each CTA recording
    // its entry into and exit from every grid barrier wait, in order
    unsigned long long *trace = nullptr;
};
constexpr int ROWS_TRACE_MARKS = 512;

// Keys per tile of the one-kernel stage for a stored format (f32 32, i16 64, i8 64).
int rows_tile_keys(int kv);
// Shared memory of the one-kernel stage for R rows with `slots` tiles; slots_for gives the most that fit.
size_t rows_smem(int kv, int hd, int R, int slots);
int rows_slots_for(int kv, int hd, int R, size_t smem_max);
// Largest co-resident grid for that shared memory (0: not launchable).
int rows_max_grid(int kv, int hd, int R, size_t smem, int sms);
// Cooperative launch of the one-kernel stage (grid CTAs, all resident at once).
cudaError_t launch_stage_rows(int kv, int hd, const RowsArgs &a, int grid, size_t smem, cudaStream_t s,
                              uint64_t *launches);

#ifdef __CUDACC__
#define TCU_HD __host__ __device__
#else
#define TCU_HD
#endif

// fit.rs:124-126 record: bytes of one stored chunk of rc rows
TCU_HD inline size_t record_bytes(int kv, int d, int rc) {
    int w = kv == 0 ? 4 : (kv == 1 ? 2 : 1);
    return (size_t)2 * d * rc * w + (kv == 0 ? 0 : (size_t)8 * d);
}

// Rows of keys per decode item for a stored format (f32 32, i16 64, i8 64).
int decode_keys_per_item(int kv);
constexpr int FLASH_KEYS = 64;  // keys per flash tile
constexpr int FLASH_ROWS = 64;  // query rows per flash block

// stats_scratch: 4 floats per row
cudaError_t launch_linear(const LinArgs &a, float *stats_scratch, cudaStream_t s, uint64_t *launches);
// the tensor-core path of launch_linear (M > 8, K a multiple of 64, split weights given)
cudaError_t launch_gemm_tc(const LinArgs &a, float4 *stats, cudaStream_t s, uint64_t *launches);
// bytes of rows x K values split into f16 hi + lo blocks of 128 rows x 64 (rows rounded up to 128)
size_t tc_split_bytes(int rows, int K);
// element offset of (n, k) inside one 128 x 64 block of the tiled weights: 8-row groups outermost, then 8-wide
// groups of K, then the 8 x 8 core matrix
inline size_t tc_block_off(int n, int k) { return (size_t)((((n & 127) >> 3) * 8 + ((k & 63) >> 3)) * 64 + (n & 7) * 8 + (k & 7)); }
size_t gemm_tc_smem();
bool gemm_tc_enabled();
cudaError_t launch_ln_apply(const float *x, int M, int K, const float *w, const float *b, float *y, cudaStream_t s,
                            uint64_t *launches);
cudaError_t launch_ssmax(float *q, int R, int d, int heads, int hid, const float *q0w, const float *q0b,
                         const float *q2w, const float *q2b, const float *scale, cudaStream_t s, uint64_t *launches);
// q *= scale (1 + tanh(m)) elementwise over [R][d] (scale indexed by coordinate)
// hd 128 and hid 64 only (cudaErrorInvalidValue otherwise)
cudaError_t launch_qmlp_tc(const QmlpArgs &a, cudaStream_t s, uint64_t *launches);
cudaError_t launch_ssmax_apply(float *q, const float *m, const float *scale, int R, int d, cudaStream_t s,
                               uint64_t *launches);
// keys-parallel split attention for few rows, then the merge into out
cudaError_t launch_attend_decode(int kv, int hd, const AttnArgs &a, cudaStream_t s, uint64_t *launches);
// row-blocked attention for many rows; merges itself when splits == 1, else writes parts
cudaError_t launch_attend_flash(int kv, int hd, const AttnArgs &a, cudaStream_t s, uint64_t *launches);
cudaError_t launch_attend_merge(const AttnArgs &a, int parts, cudaStream_t s, uint64_t *launches);
// Attention over training rows split across devices (nn.rs:261-286 merge): this device's parts of each (row, head)
// into one unnormalised state laid out as a single part (ms_out [R][H][2] = max, weight sum; acc_out [R][d]); its
// maxima m_out [R][H]; the state scaled to the maxima over devices m_all, packed [R][d + H] (values, then weight
// sums) for a sum over devices; the summed states divided (out [R][d]).
cudaError_t launch_merge_state(const AttnArgs &a, int parts, float *ms_out, float *acc_out, cudaStream_t s,
                               uint64_t *launches);
cudaError_t launch_state_max(const float *ms, int R, int H, float *m_out, cudaStream_t s, uint64_t *launches);
cudaError_t launch_state_pack(const float *ms, const float *acc, const float *m_all, int R, int H, int d, float *packed,
                              cudaStream_t s, uint64_t *launches);
cudaError_t launch_state_finish(const float *packed, int R, int H, int d, float *out, int ldo, cudaStream_t s,
                                uint64_t *launches);
cudaError_t launch_pack(const float *kvT, int ld, int d, int rows, int chunk, int kv, uint8_t *out, cudaStream_t s,
                        uint64_t *launches);
// predict.rs:590-629: a layer's stored chunks widened to k, v [rows][d] (integers times their scales)
cudaError_t launch_layer_rows(int kv, const uint8_t *layer, int rows, int chunk, int d, float *k, float *v, cudaStream_t s,
                              uint64_t *launches);
cudaError_t launch_add_y(float *h, const float *y, int rows, int d, int max_classes, const float *table,
                         cudaStream_t s, uint64_t *launches);
cudaError_t launch_class_head(const float *logits, int rows, int classes, int stride, const int32_t *member_classes,
                              double *sums, int finish, int members, double temperature, cudaStream_t s,
                              uint64_t *launches);
cudaError_t launch_regression_head(const float *qout, int rows, int nq, int stride, const double *alphas, int na,
                                   double tmean, double tscale, double *mean, double *var, double *median,
                                   double *quant, cudaStream_t s, uint64_t *launches);
cudaError_t kernels_init();

// The column and row stages (rows.cu; src/predict.rs:282-372).
// Cells X [R * F][e] of normalised rows x [R][F]: in_linear of each feature group, -100 when all are missing.
cudaError_t launch_col_cells(const float *x, int R, int F, int group, const float *in_w, const float *in_b, int e,
                             float *X, cudaStream_t s, uint64_t *launches);
// Attention of the cells' raw query projections Q [R * F][e] (times scale) against group g's cached keys and values
// ([e][n] each, at kv + g * gstride): att [R * F][e].
cudaError_t launch_col_attend(const float *Q, int R, int F, const float *kv, size_t gstride, int e, int n, int heads,
                              float scale, float *att, cudaStream_t s, uint64_t *launches);
// Rotary attention of the first nq of each row's T tokens over all T: QKV [R * T][3e] -> att [R * nq][e]; position
// tables cs, sn [T][head width / 2]; `work` (row_attend_workspace floats) when row_attend_smem is 0.
size_t row_attend_smem(int e, int T, int heads);
size_t row_attend_workspace(int R, int T, int e);
// Whether a row attention of nq queries over T tokens needs that workspace.
bool row_attend_needs_workspace(int e, int T, int nq, int heads);
cudaError_t launch_row_attend(const float *QKV, int R, int T, int nq, int e, int heads, const float *cs, const float *sn,
                              float *work, float *att, cudaStream_t s, uint64_t *launches);
// tok [R][cls + F][e]: the class tokens, then the cells.
cudaError_t launch_tokens(const float *X, const float *cls_tokens, int R, int F, int cls, int e, float *tok, cudaStream_t s,
                          uint64_t *launches);
// y [R][nq][e] += x [R][T][e] (first nq tokens of each row); x [R][T][e] = y for those tokens.
cudaError_t launch_add_rows(float *y, const float *x, int R, int nq, int T, int e, cudaStream_t s, uint64_t *launches);
cudaError_t launch_copy_rows(float *x, const float *y, int R, int nq, int T, int e, cudaStream_t s, uint64_t *launches);
// y = a x (+ y when accumulate); y = x / a.
cudaError_t launch_scale_add(float *y, const float *x, size_t n, float a, int accumulate, cudaStream_t s,
                             uint64_t *launches);
cudaError_t launch_divide(float *y, const float *x, size_t n, float a, cudaStream_t s, uint64_t *launches);
// The column stage of fitting (fitcol.cu; src/fit.rs:298-420).
// Training cells X [n * F][e] += the label's embedding (digit ((int)y / divisor) % base of a class label when base > 0).
cudaError_t launch_col_add_y(float *X, const float *y, int n, int F, int e, int max_classes, const float *table,
                             int divisor, int base, cudaStream_t s, uint64_t *launches);
// How many splits of the training cells the inducing points' attention takes (the part buffers hold
// F * heads * splits * inds states: 2 floats in part_ms, head width floats in part_acc).
int ind_attend_splits(int n, int F, int heads, int inds);
// Whether the inducing points' attention takes this width and head count (head widths 4, 8, 16, 32, 64).
bool ind_attend_takes(int e, int heads);
// The inducing points' scaled queries q [inds][e] against each group's training cells (keys and values the rows
// r * F + g of kv [n * F][2e]): att [F * inds][e].
cudaError_t launch_ind_attend(const float *q, const float *kv, int n, int F, int e, int inds, int heads, int splits,
                              float *part_ms, float *part_acc, float *att, cudaStream_t s, uint64_t *launches);
// dst [times][count] = src [count], repeated.
cudaError_t launch_repeat(float *dst, const float *src, size_t count, int times, cudaStream_t s, uint64_t *launches);
// kv2 [F * inds][2e] (keys, values) into col_kv: group g's [2][e][inds] at col_kv + g * gstride + off.
cudaError_t launch_col_kv_scatter(const float *kv2, int F, int e, int inds, size_t gstride, size_t off, float *col_kv,
                                  cudaStream_t s, uint64_t *launches);
// The class tree (tree.cu; src/predict.rs:661-692): nodes' scores (node t's [R][k] at logits + nodes[t].z * R) to
// class scores out [R][classes]; nodes in walk order {k, leaf, score offset, map offset}; wbuf [n_nodes][R].
cudaError_t launch_tree_combine(const float *logits, const int4 *nodes, const int *map, int n_nodes, int R, int classes,
                                float *wbuf, float *out, cudaStream_t s, uint64_t *launches);
// The sharded stage's exchanges by peer stores (peer.cu): for every destination rank j, segment s's count[s] floats
// at src[s] + j * src_step[s] go to peer[j] + dst_off[s] (bytes); once all of j's blocks are done, this rank's flag
// in j's buffer (at flag_off, one u32 per source rank) becomes `epoch`. done: ranks counters in this rank's memory,
// zero between pushes.
constexpr int PUSH_MAX_RANKS = 8;
struct PushArgs {
    uint8_t *peer[PUSH_MAX_RANKS] = {};
    const float *src[2] = {};
    size_t src_step[2] = {}, count[2] = {}, dst_off[2] = {};
    size_t flag_off = 0;
    unsigned *done = nullptr;
    int segments = 0, ranks = 0, me = 0;
    unsigned epoch = 0;
};
cudaError_t launch_push(const PushArgs &a, int blocks_per_dest, cudaStream_t s, uint64_t *launches);
// Wait (one thread, bounded by max_cycles) until flags[0..n) have all reached epoch; on giving up, 1 into *err.
cudaError_t launch_wait_flags(const unsigned *flags, int n, unsigned epoch, long long max_cycles, int *err,
                              cudaStream_t s, uint64_t *launches);
// Opt `kernel` in to `bytes` of dynamic shared memory on the current device (the attribute is per function and
// device); remembered per (device, kernel), so repeated calls cost a map lookup.
cudaError_t allow_dynamic_smem(const void *kernel, size_t bytes);

// Tensor-core attention (head width 128, many rows): merges itself when splits == 1, else writes parts.
cudaError_t launch_attend_tc(int kv, const AttnArgs &a, cudaStream_t s, uint64_t *launches);
size_t attend_tc_smem();
// The layer's keys and values as pre-split operand tiles for the tensor-core attention: one per (64-key tile of
// a.tiles, head), tc_tile_bytes() each, [tile][head] order (uses a.layer, rows, chunk, d, heads, full, tiles,
// ntiles, tc_eK, tc_eV).
cudaError_t launch_tc_tiles(int kv, const AttnArgs &a, void *out, cudaStream_t s, uint64_t *launches);
size_t tc_tile_bytes();
// Largest |key| and |value| of a layer, as float bits, into out[0], out[1].
cudaError_t launch_absmax_layer(const uint8_t *layer, int rows, int chunk, int d, int kv, unsigned *out, cudaStream_t s,
                                uint64_t *launches);
// Power-of-two exponent e with mx * 2^e < 2^14 (0 for mx = 0).
int tc_exponent(float mx);
// Self-test of the tensor-core operand layouts: result[0] = largest error (float), result[1] = 1 if a wait gave up.
cudaError_t launch_tc_selftest(float *result, cudaStream_t s);

}  // namespace tcu
