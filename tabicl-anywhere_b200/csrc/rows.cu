// Kernels of the column and row stages of prediction (src/predict.rs:282-372, src/nn.rs:289-429 of tabicl-anywhere):
// the test cells from the feature groups, the column stage's attention against a group's cached inducing points,
// the row stage's rotary attention over a row's tokens, and the elementwise steps between the linear layers (which
// run through launch_linear).
#include "kernels.cuh"
#include "device.cuh"

#include <algorithm>
#include <cfloat>

namespace tcu {

namespace {

// predict.rs:300-315 and nn.rs:422-429: cell (r, g) = in_linear of the features g+1, g+2, g+4, ... (circular), or
// -100 everywhere when all of them are missing (-100); X [R * F][e]. Products and sums unfused, as the CPU's short dot.
__global__ void k_col_cells1(const float *x, int R, int F, int group, const float *in_w, const float *in_b, int e, float *X) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * F * e) return;
    const int k = (int)(i % e);
    const size_t cell = i / e;
    const int g = (int)(cell % F), r = (int)(cell / F);
    const float *row = x + (size_t)r * F;
    bool missing = true;
    float s = 0.f;
    for (int j = 0; j < group; j++) {
        const float v = row[(g + (1 << j)) % F];
        missing &= v == -100.0f;
        s = __fadd_rn(s, __fmul_rn(in_w[k * group + j], v));
    }
    X[i] = missing ? -100.0f : __fadd_rn(s, in_b[k]);
}

// The same, four consecutive outputs of a cell per thread (e a multiple of 4, X 16-byte aligned): the cell's feature
// values are read once for them.
__global__ void k_col_cells(const float *x, int R, int F, int group, const float *in_w, const float *in_b, int e, float *X) {
    const size_t i4 = (size_t)blockIdx.x * blockDim.x + threadIdx.x, e4 = e / 4;
    if (i4 >= (size_t)R * F * e4) return;
    const int k0 = (int)(i4 % e4) * 4;
    const size_t cell = i4 / e4;
    const int g = (int)(cell % F), r = (int)(cell / F);
    const float *row = x + (size_t)r * F;
    bool missing = true;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < group; j++) {
        const float v = row[(g + (1 << j)) % F];
        missing &= v == -100.0f;
#pragma unroll
        for (int c = 0; c < 4; c++) s[c] = __fadd_rn(s[c], __fmul_rn(in_w[(k0 + c) * group + j], v));
    }
    float4 o;
    o.x = missing ? -100.0f : __fadd_rn(s[0], in_b[k0]);
    o.y = missing ? -100.0f : __fadd_rn(s[1], in_b[k0 + 1]);
    o.z = missing ? -100.0f : __fadd_rn(s[2], in_b[k0 + 2]);
    o.w = missing ? -100.0f : __fadd_rn(s[3], in_b[k0 + 3]);
    reinterpret_cast<float4 *>(X)[i4] = o;
}

// nn.rs:187-228, 280-286 for one query against n fixed keys: the column stage's attention of cell (r, g) against the
// cached inducing points of group g. Q [M][e] (rows of the cells, g = row % F), already the raw projection: each
// query element is multiplied by `scale` first (nn.rs:139-141); K and V of group g are [e][n] at kv + g * gstride
// (V e * n floats after K). One block per (group, run of cells of that group); the group's keys and values sit in
// shared memory, V transposed to [n][e]; one warp per (cell, head).
__global__ void __launch_bounds__(256) k_col_attend(const float *Q, int R, int F, const float *kv, size_t gstride, int e,
                                                    int n, int heads, float scale, float *att, int rows_per_block) {
    extern __shared__ float sm[];
    const int g = blockIdx.x, hd = e / heads, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *Ks = sm, *Vt = sm + (size_t)e * n, *scr = Vt + (size_t)e * n;  // scr: per warp, n scores + hd query
    const float *Kg = kv + (size_t)g * gstride, *Vg = Kg + (size_t)e * n;
    for (int i = threadIdx.x; i < e * n; i += blockDim.x) {
        Ks[i] = Kg[i];
        const int j = i / n, k = i - j * n;
        Vt[(size_t)k * e + j] = Vg[i];
    }
    __syncthreads();
    float *ps = scr + (size_t)warp * (n + hd), *qs = ps + n;
    const int r0 = blockIdx.y * rows_per_block, r1 = min(R, r0 + rows_per_block);
    for (int task = warp; task < (r1 - r0) * heads; task += blockDim.x >> 5) {
        const int r = r0 + task / heads, h = task % heads;
        const size_t cell = (size_t)r * F + g;
        for (int j = lane; j < hd; j += 32) qs[j] = Q[cell * e + h * hd + j] * scale;
        __syncwarp();
        float mx = -FLT_MAX;
        for (int k = lane; k < n; k += 32) {
            float s = 0.f;
            for (int j = 0; j < hd; j++) s = fmaf(qs[j], Ks[(size_t)(h * hd + j) * n + k], s);
            ps[k] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        float sum = 0.f;
        for (int k = lane; k < n; k += 32) {
            const float p = exp1(ps[k] - mx);
            ps[k] = p;
            sum += p;
        }
        sum = warp_sum(sum);
        __syncwarp();
        const float inv = 1.0f / sum;
        for (int j = lane; j < hd; j += 32) {
            float o = 0.f;
            for (int k = 0; k < n; k++) o = fmaf(Vt[(size_t)k * e + h * hd + j], ps[k], o);
            att[cell * e + h * hd + j] = o * inv;
        }
        __syncwarp();
    }
}

// Queries per thread (each key and value row read from shared memory serves all of them) and keys per chunk (as
// many independent chains as the queries and the weighted values leave registers for), by head width.
__host__ __device__ constexpr int attend_nq(int hd) { return hd <= 32 ? 2 : 1; }
__host__ __device__ constexpr int attend_chunk(int hd, int nq) {
    return nq == 2 ? (hd <= 8 ? 16 : hd == 16 ? 8 : 4) : (hd <= 16 ? 16 : hd == 32 ? 8 : 4);
}

// nn.rs:187-228, 280-286 for NQ queries (scaled, in registers) against n keys and values held in shared memory as
// [n][HD] rows, read by every lane at once: the online softmax over chunks of KC keys, each query's running maximum
// replaced (and its sums rescaled) only when a chunk's maximum exceeds it, as Soft::update does. A chunk's scores are
// independent chains, each added in coordinate order. acc[i] (HD) receives query i's weighted values, sum[i] its
// weights' sum. Key (and value) rows are ld floats apart.
template <int HD, int KC, int NQ>
__device__ __forceinline__ void attend_queries(const float (&q)[NQ][HD], const float *Ks, const float *Vs, int n,
                                               float (&acc)[NQ][HD], float (&sum)[NQ], int ld = HD) {
    float m[NQ];
#pragma unroll
    for (int i = 0; i < NQ; i++) m[i] = -FLT_MAX, sum[i] = 0.f;
    for (int k0 = 0; k0 < n; k0 += KC) {
        float sc[NQ][KC];
#pragma unroll
        for (int i = 0; i < NQ; i++)
#pragma unroll
            for (int c = 0; c < KC; c++) sc[i][c] = 0.f;
#pragma unroll
        for (int j4 = 0; j4 < HD / 4; j4++) {
#pragma unroll
            for (int c = 0; c < KC; c++) {
                const float4 kk = reinterpret_cast<const float4 *>(Ks + (size_t)min(k0 + c, n - 1) * ld)[j4];
#pragma unroll
                for (int i = 0; i < NQ; i++) {
                    sc[i][c] = fmaf(q[i][4 * j4], kk.x, sc[i][c]), sc[i][c] = fmaf(q[i][4 * j4 + 1], kk.y, sc[i][c]);
                    sc[i][c] = fmaf(q[i][4 * j4 + 2], kk.z, sc[i][c]), sc[i][c] = fmaf(q[i][4 * j4 + 3], kk.w, sc[i][c]);
                }
            }
        }
        float p[NQ][KC];
#pragma unroll
        for (int i = 0; i < NQ; i++) {
            float cm = -FLT_MAX;
#pragma unroll
            for (int c = 0; c < KC; c++)
                if (k0 + c < n) cm = fmaxf(cm, sc[i][c]);
            if (cm > m[i]) {
                const float corr = exp1(m[i] - cm);
                m[i] = cm, sum[i] *= corr;
#pragma unroll
                for (int j = 0; j < HD; j++) acc[i][j] *= corr;
            }
#pragma unroll
            for (int c = 0; c < KC; c++) {
                p[i][c] = k0 + c < n ? exp1(sc[i][c] - m[i]) : 0.f;
                sum[i] += p[i][c];
            }
        }
#pragma unroll
        for (int c = 0; c < KC; c++) {
            const float4 *vr = reinterpret_cast<const float4 *>(Vs + (size_t)min(k0 + c, n - 1) * ld);
#pragma unroll
            for (int j4 = 0; j4 < HD / 4; j4++) {
                const float4 vv = vr[j4];
#pragma unroll
                for (int i = 0; i < NQ; i++) {
                    acc[i][4 * j4] = fmaf(vv.x, p[i][c], acc[i][4 * j4]);
                    acc[i][4 * j4 + 1] = fmaf(vv.y, p[i][c], acc[i][4 * j4 + 1]);
                    acc[i][4 * j4 + 2] = fmaf(vv.z, p[i][c], acc[i][4 * j4 + 2]);
                    acc[i][4 * j4 + 3] = fmaf(vv.w, p[i][c], acc[i][4 * j4 + 3]);
                }
            }
        }
    }
}

// The same attention with one query per thread, or two: block (group g, head h, run of NQ * blockDim rows); the
// head's keys and values of group g in shared memory as [n][HD] rows, read by every lane at once (broadcast); the
// queries, then the weighted values, in registers (attend_queries). Thread t takes rows t and t + blockDim of the run.
template <int HD>
__global__ void __launch_bounds__(128) k_col_attend_q(const float *Q, int R, int F, const float *kv, size_t gstride,
                                                      int e, int n, float scale, float *att) {
    constexpr int NQ = attend_nq(HD);
    extern __shared__ __align__(16) float sm[];
    const int g = blockIdx.x, h = blockIdx.y;
    const float *Kg = kv + (size_t)g * gstride, *Vg = Kg + (size_t)e * n;
    // rows padded to HD + 4 floats: the turn-round's stores (consecutive keys, one coordinate) fall in eight banks
    // instead of one, and every row still starts on 16 bytes
    constexpr int LD = HD + 4;
    float *Ks = sm, *Vs = sm + (size_t)n * LD;
#pragma unroll 8
    for (int i = threadIdx.x; i < n * HD; i += blockDim.x) {
        const int j = i / n, k = i - j * n;
        Ks[k * LD + j] = Kg[(size_t)(h * HD + j) * n + k];
        Vs[k * LD + j] = Vg[(size_t)(h * HD + j) * n + k];
    }
    __syncthreads();
    const int r0 = blockIdx.z * NQ * blockDim.x + threadIdx.x;
    if (r0 >= R) return;
    float q[NQ][HD], acc[NQ][HD], sum[NQ];
    int rr[NQ];
#pragma unroll
    for (int i = 0; i < NQ; i++) {
        rr[i] = r0 + i * blockDim.x;
        const float *qp = Q + ((size_t)min(rr[i], R - 1) * F + g) * e + h * HD;  // a row past R repeats the last one
#pragma unroll
        for (int j = 0; j < HD; j++) q[i][j] = qp[j] * scale, acc[i][j] = 0.f;
    }
    attend_queries<HD, attend_chunk(HD, NQ), NQ>(q, Ks, Vs, n, acc, sum, LD);
#pragma unroll
    for (int i = 0; i < NQ; i++) {
        if (rr[i] >= R) break;
        const float inv = 1.0f / sum[i];
        float *op = att + ((size_t)rr[i] * F + g) * e + h * HD;
#pragma unroll
        for (int j = 0; j < HD; j++) op[j] = acc[i][j] * inv;
    }
}

// The rotary rotation (nn.rs:380-395) of element j of a head's key or query row x (head width hd), position t.
__device__ __forceinline__ float rope(const float *x, int j, int half, const float *cs, const float *sn, int t) {
    if (j < half) return x[j] * cs[t * half + j] - x[j + half] * sn[t * half + j];
    const int jj = j - half;
    return x[j] * cs[t * half + jj] + x[jj] * sn[t * half + jj];
}

// Rotated keys of every token, transposed per row: Kt [R][e][T] (for rows too long to keep in shared memory).
__global__ void k_row_keys(const float *QKV, int R, int T, int e, int heads, const float *cs, const float *sn, float *Kt) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * T * e) return;
    const int hd = e / heads, c = (int)(i % e);
    const size_t rt = i / e;
    const int t = (int)(rt % T), r = (int)(rt / T), h = c / hd;
    const float *kr = QKV + rt * 3 * e + e + h * hd;
    Kt[((size_t)r * e + c) * T + t] = rope(kr, c - h * hd, hd / 2, cs, sn, t);
}

// nn.rs:369-404 for one row: tokens' projections QKV [R * T][3e] (queries, keys, values), the rotary rotation of the
// queries (times 1/sqrt(head width)) and keys by the position tables cs, sn [T][hd / 2], then attention of the
// first nq tokens over all T; att [R * nq][e]. One block per row, one warp per (token, head). SMEM: the row's rotated
// keys [e][T] and values [T][e] in shared memory; otherwise keys from Kt (k_row_keys) and values from QKV.
template <bool SMEM>
__global__ void __launch_bounds__(256) k_row_attend(const float *QKV, int R, int T, int nq, int e, int heads,
                                                    const float *cs, const float *sn, const float *KtG, float *att) {
    extern __shared__ float sm[];
    const int r = blockIdx.x, hd = e / heads, half = hd / 2, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5;
    const float *base = QKV + (size_t)r * T * 3 * e;
    const float *Kt = SMEM ? nullptr : KtG + (size_t)r * e * T, *V = base + 2 * e;  // V[k][c] at V + k * 3e + c
    size_t vstride = (size_t)3 * e;
    float *scr = sm;
    if constexpr (SMEM) {
        float *Ks = sm, *Vs = sm + (size_t)e * T;
        scr = Vs + (size_t)e * T;
        for (int i = threadIdx.x; i < T * e; i += blockDim.x) {
            const int t = i / e, c = i - t * e, h = c / hd;
            Ks[(size_t)c * T + t] = rope(base + (size_t)t * 3 * e + e + h * hd, c - h * hd, half, cs, sn, t);
            Vs[i] = base[(size_t)t * 3 * e + 2 * e + c];
        }
        __syncthreads();
        Kt = Ks, V = Vs, vstride = e;
    }
    const float inv = 1.0f / sqrtf((float)hd);
    float *ps = scr + (size_t)warp * (T + hd), *qs = ps + T;
    for (int task = warp; task < nq * heads; task += nw) {
        const int t = task / heads, h = task % heads;
        const float *qr = base + (size_t)t * 3 * e + h * hd;
        for (int j = lane; j < hd; j += 32) qs[j] = rope(qr, j, half, cs, sn, t) * inv;
        __syncwarp();
        float mx = -FLT_MAX;
        for (int k = lane; k < T; k += 32) {
            float s = 0.f;
            for (int j = 0; j < hd; j++) s = fmaf(qs[j], Kt[(size_t)(h * hd + j) * T + k], s);
            ps[k] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        float sum = 0.f;
        for (int k = lane; k < T; k += 32) {
            const float p = exp1(ps[k] - mx);
            ps[k] = p;
            sum += p;
        }
        sum = warp_sum(sum);
        __syncwarp();
        const float s = 1.0f / sum;
        for (int j = lane; j < hd; j += 32) {
            float o = 0.f;
            for (int k = 0; k < T; k++) o = fmaf(V[(size_t)k * vstride + h * hd + j], ps[k], o);
            att[((size_t)r * nq + t) * e + h * hd + j] = o * s;
        }
        __syncwarp();
    }
}

// k_row_attend with one query token per thread: block (row r, head h), the head's rotated keys and values of the row
// in shared memory as [T][HD] rows, read by every lane at once; the query and the weighted values in registers
// (attend_queries).
template <int HD>
__global__ void __launch_bounds__(512) k_row_attend_q(const float *QKV, int R, int T, int nq, int e, const float *cs,
                                                       const float *sn, float *att) {
    constexpr int NQ = 1;  // two tokens a thread measured slower: the row's blocks are bound by loading its keys
    extern __shared__ __align__(16) float sm[];
    const int r = blockIdx.x, h = blockIdx.y, half = HD / 2;
    const float *base = QKV + (size_t)r * T * 3 * e;
    float *Ks = sm, *Vs = sm + (size_t)T * HD;
#pragma unroll 8
    for (int i = threadIdx.x; i < T * HD; i += blockDim.x) {
        const int t = i / HD, j = i - t * HD;
        Ks[i] = rope(base + (size_t)t * 3 * e + e + h * HD, j, half, cs, sn, t);
        Vs[i] = base[(size_t)t * 3 * e + 2 * e + h * HD + j];
    }
    __syncthreads();
    if ((int)threadIdx.x >= nq) return;
    const float inv = 1.0f / sqrtf((float)HD);
    float q[NQ][HD], acc[NQ][HD], sum[NQ];
    int tt[NQ];
#pragma unroll
    for (int i = 0; i < NQ; i++) {
        tt[i] = threadIdx.x + i * blockDim.x;
        const int t = min(tt[i], nq - 1);  // a token past nq repeats the last one
        const float *qr = base + (size_t)t * 3 * e + h * HD;
#pragma unroll
        for (int j = 0; j < HD; j++) q[i][j] = rope(qr, j, half, cs, sn, t) * inv, acc[i][j] = 0.f;
    }
    attend_queries<HD, attend_chunk(HD, NQ), NQ>(q, Ks, Vs, T, acc, sum);
#pragma unroll
    for (int i = 0; i < NQ; i++) {
        if (tt[i] >= nq) break;
        const float s = 1.0f / sum[i];
        float *op = att + ((size_t)r * nq + tt[i]) * e + h * HD;
#pragma unroll
        for (int j = 0; j < HD; j++) op[j] = acc[i][j] * s;
    }
}

// tok [R][T][e]: rows t < cls are the class tokens, rows cls + g the cells X [R * F][e] (T = cls + F).
__global__ void k_tokens1(const float *X, const float *cls_tokens, int R, int F, int cls, int e, float *tok) {
    const int T = cls + F;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * T * e) return;
    const int k = (int)(i % e);
    const size_t rt = i / e;
    const int t = (int)(rt % T), r = (int)(rt / T);
    tok[i] = t < cls ? cls_tokens[t * e + k] : X[((size_t)r * F + (t - cls)) * e + k];
}

// The same, four values a thread (e a multiple of 4, the buffers 16-byte aligned).
__global__ void k_tokens(const float *X, const float *cls_tokens, int R, int F, int cls, int e, float *tok) {
    const int T = cls + F, e4 = e / 4;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * T * e4) return;
    const int k = (int)(i % e4);
    const size_t rt = i / e4;
    const int t = (int)(rt % T), r = (int)(rt / T);
    reinterpret_cast<float4 *>(tok)[i] =
        t < cls ? reinterpret_cast<const float4 *>(cls_tokens)[t * e4 + k]
                : reinterpret_cast<const float4 *>(X)[((size_t)r * F + (t - cls)) * e4 + k];
}

// y[r][t] (nq rows of each of R) += x[r][t] (T rows of each): the residual of the row stage's query tokens.
__global__ void k_add_rows(float *y, const float *x, int R, int nq, int T, int e) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * nq * e) return;
    const int k = (int)(i % e);
    const size_t rt = i / e;
    const int t = (int)(rt % nq), r = (int)(rt / nq);
    y[i] += x[((size_t)r * T + t) * e + k];
}

// x[r][t] (T rows of each of R) = y[r][t] (nq rows of each) for t < nq.
__global__ void k_copy_rows(float *x, const float *y, int R, int nq, int T, int e) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * nq * e) return;
    const int k = (int)(i % e);
    const size_t rt = i / e;
    const int t = (int)(rt % nq), r = (int)(rt / nq);
    x[((size_t)r * T + t) * e + k] = y[i];
}

// y = a * x (+ y when accumulate): the digits' running sum and its average (predict.rs:326-346).
__global__ void k_scale_add(float *y, const float *x, size_t n, float a, int accumulate) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    y[i] = accumulate ? y[i] + a * x[i] : a * x[i];
}

// y = x / a: the digits' average (predict.rs:344, a division as the CPU does it).
__global__ void k_divide(float *y, const float *x, size_t n, float a) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = x[i] / a;
}

inline unsigned blocks_for(size_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace

cudaError_t launch_col_cells(const float *x, int R, int F, int group, const float *in_w, const float *in_b, int e,
                             float *X, cudaStream_t s, uint64_t *launches) {
    if (e % 4 || reinterpret_cast<uintptr_t>(X) % 16)
        k_col_cells1<<<blocks_for((size_t)R * F * e), 256, 0, s>>>(x, R, F, group, in_w, in_b, e, X);
    else
        k_col_cells<<<blocks_for((size_t)R * F * e / 4), 256, 0, s>>>(x, R, F, group, in_w, in_b, e, X);
    if (launches) ++*launches;
    return cudaGetLastError();
}

size_t col_attend_smem(int e, int n, int heads) { return sizeof(float) * ((size_t)2 * e * n + 8 * (size_t)(n + e / heads)); }

template <int HD>
static cudaError_t col_attend_q(const float *Q, int R, int F, const float *kv, size_t gstride, int e, int n, int heads,
                                float scale, float *att, cudaStream_t s) {
    const size_t smem = sizeof(float) * 2 * (size_t)n * (HD + 4);
    cudaError_t err = allow_dynamic_smem((const void *)k_col_attend_q<HD>, smem);
    if (err != cudaSuccess) return err;
    constexpr int NQ = attend_nq(HD), TH = 128;
    dim3 grid(F, heads, (R + NQ * TH - 1) / (NQ * TH));
    k_col_attend_q<HD><<<grid, TH, smem, s>>>(Q, R, F, kv, gstride, e, n, scale, att);
    return cudaGetLastError();
}

cudaError_t launch_col_attend(const float *Q, int R, int F, const float *kv, size_t gstride, int e, int n, int heads,
                              float scale, float *att, cudaStream_t s, uint64_t *launches) {
    const int hd = e / heads;
    if (sizeof(float) * 2 * (size_t)n * (hd + 4) <= 200 * 1024 && (hd == 8 || hd == 16 || hd == 32 || hd == 64)) {
        const cudaError_t err = hd == 8    ? col_attend_q<8>(Q, R, F, kv, gstride, e, n, heads, scale, att, s)
                                : hd == 16 ? col_attend_q<16>(Q, R, F, kv, gstride, e, n, heads, scale, att, s)
                                : hd == 32 ? col_attend_q<32>(Q, R, F, kv, gstride, e, n, heads, scale, att, s)
                                           : col_attend_q<64>(Q, R, F, kv, gstride, e, n, heads, scale, att, s);
        if (launches) ++*launches;
        return err;
    }
    const size_t smem = col_attend_smem(e, n, heads);
    cudaError_t err = allow_dynamic_smem((const void *)k_col_attend, smem);
    if (err != cudaSuccess) return err;
    // enough row runs for about four blocks per SM over all groups, at least 32 cells per block
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int runs = (4 * sms + F - 1) / F;
    runs = std::max(1, std::min(runs, (R + 31) / 32));
    const int per = (R + runs - 1) / runs;
    dim3 grid(F, (R + per - 1) / per);
    k_col_attend<<<grid, 256, smem, s>>>(Q, R, F, kv, gstride, e, n, heads, scale, att, per);
    if (launches) ++*launches;
    return cudaGetLastError();
}

// Shared memory of the row attention when the row's keys and values are held (0: too long, they stay in global
// memory and the keys go through a workspace of row_attend_workspace floats).
size_t row_attend_smem(int e, int T, int heads) {
    const size_t need = sizeof(float) * ((size_t)2 * e * T + 8 * (size_t)(T + e / heads));
    return need <= 200 * 1024 ? need : 0;
}
size_t row_attend_workspace(int R, int T, int e) { return (size_t)R * T * e; }

template <int HD>
static cudaError_t row_attend_q(const float *QKV, int R, int T, int nq, int e, int heads, const float *cs,
                                const float *sn, float *att, cudaStream_t s) {
    const size_t smem = sizeof(float) * 2 * (size_t)T * HD;
    cudaError_t err = allow_dynamic_smem((const void *)k_row_attend_q<HD>, smem);
    if (err != cudaSuccess) return err;
    k_row_attend_q<HD><<<dim3(R, heads), (nq + 31) / 32 * 32, smem, s>>>(QKV, R, T, nq, e, cs, sn, att);
    return cudaGetLastError();
}

// Whether the one-query-per-thread row attention takes the shape (else k_row_attend).
static bool row_attend_by_query(int e, int T, int nq, int heads) {
    const int hd = e / heads;
    return nq <= 512 && sizeof(float) * 2 * (size_t)T * hd <= 200 * 1024 && (hd == 8 || hd == 16 || hd == 32 || hd == 64);
}

bool row_attend_needs_workspace(int e, int T, int nq, int heads) {
    return !row_attend_by_query(e, T, nq, heads) && !row_attend_smem(e, T, heads);
}

cudaError_t launch_row_attend(const float *QKV, int R, int T, int nq, int e, int heads, const float *cs, const float *sn,
                              float *work, float *att, cudaStream_t s, uint64_t *launches) {
    if (row_attend_by_query(e, T, nq, heads)) {
        const int hd = e / heads;
        const cudaError_t err = hd == 8    ? row_attend_q<8>(QKV, R, T, nq, e, heads, cs, sn, att, s)
                                : hd == 16 ? row_attend_q<16>(QKV, R, T, nq, e, heads, cs, sn, att, s)
                                : hd == 32 ? row_attend_q<32>(QKV, R, T, nq, e, heads, cs, sn, att, s)
                                           : row_attend_q<64>(QKV, R, T, nq, e, heads, cs, sn, att, s);
        if (launches) ++*launches;
        return err;
    }
    const size_t smem = row_attend_smem(e, T, heads);
    cudaError_t err;
    if (smem) {
        err = allow_dynamic_smem((const void *)k_row_attend<true>, smem);
        if (err != cudaSuccess) return err;
        k_row_attend<true><<<R, 256, smem, s>>>(QKV, R, T, nq, e, heads, cs, sn, nullptr, att);
    } else {
        if (!work) return cudaErrorInvalidValue;
        k_row_keys<<<blocks_for((size_t)R * T * e), 256, 0, s>>>(QKV, R, T, e, heads, cs, sn, work);
        if (launches) ++*launches;
        const size_t scratch = sizeof(float) * 8 * (size_t)(T + e / heads);
        err = allow_dynamic_smem((const void *)k_row_attend<false>, scratch);
        if (err != cudaSuccess) return err;
        k_row_attend<false><<<R, 256, scratch, s>>>(QKV, R, T, nq, e, heads, cs, sn, work, att);
    }
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_tokens(const float *X, const float *cls_tokens, int R, int F, int cls, int e, float *tok, cudaStream_t s,
                          uint64_t *launches) {
    if (e % 4 || (reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(cls_tokens) | reinterpret_cast<uintptr_t>(tok)) % 16)
        k_tokens1<<<blocks_for((size_t)R * (cls + F) * e), 256, 0, s>>>(X, cls_tokens, R, F, cls, e, tok);
    else
        k_tokens<<<blocks_for((size_t)R * (cls + F) * e / 4), 256, 0, s>>>(X, cls_tokens, R, F, cls, e, tok);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_add_rows(float *y, const float *x, int R, int nq, int T, int e, cudaStream_t s, uint64_t *launches) {
    k_add_rows<<<blocks_for((size_t)R * nq * e), 256, 0, s>>>(y, x, R, nq, T, e);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_copy_rows(float *x, const float *y, int R, int nq, int T, int e, cudaStream_t s, uint64_t *launches) {
    k_copy_rows<<<blocks_for((size_t)R * nq * e), 256, 0, s>>>(x, y, R, nq, T, e);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_scale_add(float *y, const float *x, size_t n, float a, int accumulate, cudaStream_t s,
                             uint64_t *launches) {
    k_scale_add<<<blocks_for(n), 256, 0, s>>>(y, x, n, a, accumulate);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_divide(float *y, const float *x, size_t n, float a, cudaStream_t s, uint64_t *launches) {
    k_divide<<<blocks_for(n), 256, 0, s>>>(y, x, n, a);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
