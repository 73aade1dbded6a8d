// Hand-written sm_100a kernels of tabicl-anywhere's in-context prediction stage (src/predict.rs:381-586):
// LayerNorm + linear layers with fused GELU / residual epilogues, the query MLP of the scalable softmax,
// attention over the stored key/value chunks with the integer dequantisation fused into the loads, the
// log-sum-exp merge, fitting's chunk packer, and the classification / regression heads.
#include "kernels.cuh"
#include "pdl.cuh"
#include "device.cuh"

#include <cfloat>
#include <map>
#include <mutex>

namespace tcu {

#define TCU_LAUNCHED(l) \
    do {                \
        if (l) ++*(l);  \
    } while (0)

// ---- linear layers -----------------------------------------------------------------------------------------

// Few rows (M <= 8): the rows sit in shared memory (LayerNorm applied there, two-pass as kern.rs:357-376), one
// warp per output reads that output's weight row once with 16-byte loads and serves every row.
template <int RM>
__global__ void __launch_bounds__(128) k_gemv(LinArgs a) {
    extern __shared__ __align__(16) float xs[];  // [RM][K]
    constexpr int WARPS = 4, MAXV = 8;           // a lane holds up to 8 16-byte pieces of its weight row (K <= 1024)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int R = a.M, K = a.K;
    for (int i = tid; i < R * K; i += blockDim.x) {
        int r = i / K, k = i - r * K;
        xs[i] = a.x[(size_t)r * a.ldx + k];
    }
    __syncthreads();
    if (a.lnw) {
        for (int r = warp; r < R; r += WARPS) {
            float *row = xs + r * K;
            float s = 0.f;
            for (int k = lane; k < K; k += 32) s += row[k];
            float mean = warp_sum(s) / (float)K;
            float q = 0.f;
            for (int k = lane; k < K; k += 32) {
                float dd = row[k] - mean;
                q = fmaf(dd, dd, q);
            }
            float inv = 1.0f / sqrtf(warp_sum(q) / (float)K + 1e-5f);
            for (int k = lane; k < K; k += 32) row[k] = (row[k] - mean) * inv * a.lnw[k] + a.lnb[k];
        }
        __syncthreads();
    }
    const uint64_t pol = policy_evict_last();
    for (int o = blockIdx.x * WARPS + warp; o < a.N; o += gridDim.x * WARPS) {
        float acc[RM];
#pragma unroll
        for (int r = 0; r < RM; r++) acc[r] = 0.f;
        const float *w = a.W + (size_t)o * K;
        auto step = [&](const float4 &wv, int k) {
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r < R) {
                    float4 xv = *reinterpret_cast<const float4 *>(xs + r * K + k);
                    acc[r] = fmaf(wv.x, xv.x, acc[r]);
                    acc[r] = fmaf(wv.y, xv.y, acc[r]);
                    acc[r] = fmaf(wv.z, xv.z, acc[r]);
                    acc[r] = fmaf(wv.w, xv.w, acc[r]);
                }
            }
        };
        if (K <= 128 * MAXV) {
            // every load of the row issued before the first multiply
            float4 wv[MAXV];
#pragma unroll
            for (int v = 0; v < MAXV; v++)
                if (lane * 4 + v * 128 < K) wv[v] = ld_weight4(w + lane * 4 + v * 128, pol);
#pragma unroll
            for (int v = 0; v < MAXV; v++)
                if (lane * 4 + v * 128 < K) step(wv[v], lane * 4 + v * 128);
        } else {
            for (int k = lane * 4; k < K; k += 128) step(ld_weight4(w + k, pol), k);
        }
#pragma unroll
        for (int r = 0; r < RM; r++) acc[r] = warp_sum(acc[r]);
        if (lane == 0) {
            float b = a.bias ? a.bias[o] : 0.f;
#pragma unroll
            for (int r = 0; r < RM; r++) {
                if (r < R) {
                    float v = acc[r] + b;
                    if (a.act) v = gelu1(v);
                    float *dst = a.transpose_out ? a.y + (size_t)o * a.ldy + r : a.y + (size_t)r * a.ldy + o;
                    *dst = a.accumulate ? *dst + v : v;
                }
            }
        }
    }
}

// Per-row mean and 1/sigma (kern.rs:357-376): one warp per row, two passes.
__global__ void k_ln_stats(const float *x, int ldx, int M, int K, float *stats) {
    int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const float *p = x + (size_t)row * ldx;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += p[k];
    float mean = warp_sum(s) / (float)K;
    float q = 0.f;
    for (int k = lane; k < K; k += 32) {
        float dd = p[k] - mean;
        q = fmaf(dd, dd, q);
    }
    float inv = 1.0f / sqrtf(warp_sum(q) / (float)K + 1e-5f);
    if (lane == 0) stats[2 * row] = mean, stats[2 * row + 1] = inv;
}

__global__ void k_ln_apply(const float *x, int M, int K, const float *w, const float *b, float *y) {
    int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const float *p = x + (size_t)row * K;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += p[k];
    float mean = warp_sum(s) / (float)K;
    float q = 0.f;
    for (int k = lane; k < K; k += 32) {
        float dd = p[k] - mean;
        q = fmaf(dd, dd, q);
    }
    float inv = 1.0f / sqrtf(warp_sum(q) / (float)K + 1e-5f);
    for (int k = lane; k < K; k += 32) y[(size_t)row * K + k] = (p[k] - mean) * inv * w[k] + b[k];
}

// Many rows: 128 x 128 output tiles, k-steps of 8, double-buffered shared memory, 8 x 8 outputs per thread in
// four 4 x 4 quadrants. The LayerNorm of the input rows is applied as the tile is loaded (stats precomputed).
__global__ void __launch_bounds__(256, 2) k_gemm(LinArgs a) {
    __shared__ __align__(16) float As[2][8][128];
    __shared__ __align__(16) float Bs[2][8][128];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
    const int lr = tid >> 1, lk = (tid & 1) * 4;
    const int am = m0 + lr, bn = n0 + lr;
    float mean = 0.f, rstd = 1.f;
    if (a.stats && am < a.M) mean = a.stats[2 * am], rstd = a.stats[2 * am + 1];
    const float *ap = a.x + (size_t)(am < a.M ? am : 0) * a.ldx;
    const float *bp = a.W + (size_t)(bn < a.N ? bn : 0) * a.K;
    const uint64_t pol = policy_evict_last();
    auto loadA = [&](int k0) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        int k = k0 + lk;
        if (am < a.M && k < a.K) {
            v = *reinterpret_cast<const float4 *>(ap + k);
            if (a.stats) {
                v.x = (v.x - mean) * rstd * a.lnw[k] + a.lnb[k];
                v.y = (v.y - mean) * rstd * a.lnw[k + 1] + a.lnb[k + 1];
                v.z = (v.z - mean) * rstd * a.lnw[k + 2] + a.lnb[k + 2];
                v.w = (v.w - mean) * rstd * a.lnw[k + 3] + a.lnb[k + 3];
            }
        }
        return v;
    };
    auto loadB = [&](int k0) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        int k = k0 + lk;
        if (bn < a.N && k < a.K) v = ld_weight4(bp + k, pol);
        return v;
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
    float4 ra = loadA(0), rb = loadB(0);
    As[0][lk + 0][lr] = ra.x, As[0][lk + 1][lr] = ra.y, As[0][lk + 2][lr] = ra.z, As[0][lk + 3][lr] = ra.w;
    Bs[0][lk + 0][lr] = rb.x, Bs[0][lk + 1][lr] = rb.y, Bs[0][lk + 2][lr] = rb.z, Bs[0][lk + 3][lr] = rb.w;
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < a.K; k0 += 8) {
        const bool more = k0 + 8 < a.K;
        if (more) ra = loadA(k0 + 8), rb = loadB(k0 + 8);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4 + 64]);
            float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4 + 64]);
            float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) {
            buf ^= 1;
            As[buf][lk + 0][lr] = ra.x, As[buf][lk + 1][lr] = ra.y, As[buf][lk + 2][lr] = ra.z, As[buf][lk + 3][lr] = ra.w;
            Bs[buf][lk + 0][lr] = rb.x, Bs[buf][lk + 1][lr] = rb.y, Bs[buf][lk + 2][lr] = rb.z, Bs[buf][lk + 3][lr] = rb.w;
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (n >= a.N) continue;
            float v = acc[i][j] + (a.bias ? a.bias[a.bias_on_m ? m : n] : 0.f);
            if (a.act) v = gelu1(v);
            float *dst = a.transpose_out ? a.y + (size_t)n * a.ldy + m : a.y + (size_t)m * a.ldy + n;
            *dst = a.accumulate ? *dst + v : v;
        }
    }
}

// ---- the scalable softmax's query modulation (nn.rs:138-149) ------------------------------------------------

// For each row and head: m = q2 . GELU(q0 . q_h + b0) + b2, then q_h *= scale_h * (1 + tanh(m)). The two small
// matrices sit in shared memory (rows padded by one float so threads walking rows do not share banks).
__global__ void __launch_bounds__(256) k_ssmax(float *q, int R, int d, int heads, int hid, const float *q0w,
                                               const float *q0b, const float *q2w, const float *q2b,
                                               const float *scale, int rows_per_block) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    extern __shared__ float sm[];
    const int hd = d / heads, h = blockIdx.y, r0 = blockIdx.x * rows_per_block;
    const int RB = rows_per_block;
    float *w0 = sm;                         // [hid][hd + 1]
    float *w2 = w0 + hid * (hd + 1);        // [hd][hid + 1]
    float *qs = w2 + hd * (hid + 1);        // [RB][hd]
    float *hs = qs + RB * hd;               // [RB][hid]
    const int tid = threadIdx.x, bd = blockDim.x;
    for (int i = tid; i < hid * hd; i += bd) w0[(i / hd) * (hd + 1) + i % hd] = q0w[i];
    for (int i = tid; i < hd * hid; i += bd) w2[(i / hid) * (hid + 1) + i % hid] = q2w[i];
    for (int i = tid; i < RB * hd; i += bd) {
        int r = i / hd, j = i % hd;
        qs[i] = r0 + r < R ? q[(size_t)(r0 + r) * d + h * hd + j] : 0.f;
    }
    __syncthreads();
    for (int i = tid; i < RB * hid; i += bd) {
        int r = i / hid, t = i % hid;
        const float *w = w0 + t * (hd + 1), *x = qs + r * hd;
        float s = 0.f;
        for (int j = 0; j < hd; j++) s = fmaf(w[j], x[j], s);
        hs[i] = gelu1(s + q0b[t]);
    }
    __syncthreads();
    for (int i = tid; i < RB * hd; i += bd) {
        int r = i / hd, j = i % hd;
        if (r0 + r >= R) continue;
        const float *w = w2 + j * (hid + 1), *x = hs + r * hid;
        float s = 0.f;
        for (int t = 0; t < hid; t++) s = fmaf(w[t], x[t], s);
        float mm = s + q2b[j];
        q[(size_t)(r0 + r) * d + h * hd + j] = qs[i] * (scale[h * hd + j] * (1.0f + tanh1(mm)));
    }
}

// Few rows: one block per (row, head), weights read straight from L2 by warps (one output per warp step).
__global__ void __launch_bounds__(256) k_ssmax_rows(float *q, int d, int heads, int hid, const float *q0w,
                                                    const float *q0b, const float *q2w, const float *q2b,
                                                    const float *scale) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    extern __shared__ float sm[];
    const int hd = d / heads, r = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float *qs = sm, *hs = sm + hd;
    float *qp = q + (size_t)r * d + h * hd;
    if (hd == 128 && hid == 64) {
        // the configs' shape: every weight a warp needs is loaded before q, all in flight at once; each output's
        // sum is taken in the same order as the general loops below
        float w0[8][4], w2[16][2], b0[8], b2[16], sc[16];
#pragma unroll
        for (int i = 0; i < 8; i++) {
#pragma unroll
            for (int k = 0; k < 4; k++) w0[i][k] = __ldg(q0w + (size_t)(warp + 8 * i) * 128 + lane + 32 * k);
            b0[i] = __ldg(q0b + warp + 8 * i);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
#pragma unroll
            for (int k = 0; k < 2; k++) w2[i][k] = __ldg(q2w + (size_t)(warp + 8 * i) * 64 + lane + 32 * k);
            b2[i] = __ldg(q2b + warp + 8 * i);
            sc[i] = __ldg(scale + h * 128 + warp + 8 * i);
        }
        if (tid < 128) qs[tid] = qp[tid];
        __syncthreads();
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; k++) x[k] = qs[lane + 32 * k];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) s = fmaf(w0[i][k], x[k], s);
            s = warp_sum(s);
            if (lane == 0) hs[warp + 8 * i] = gelu1(s + b0[i]);
        }
        __syncthreads();
        const float y0 = hs[lane], y1 = hs[lane + 32];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            float s = fmaf(w2[i][0], y0, 0.f);
            s = fmaf(w2[i][1], y1, s);
            s = warp_sum(s);
            const int j = warp + 8 * i;
            if (lane == 0) qp[j] = qs[j] * (sc[i] * (1.0f + tanh1(s + b2[i])));
        }
        return;
    }
    for (int j = tid; j < hd; j += blockDim.x) qs[j] = qp[j];
    __syncthreads();
    for (int t = warp; t < hid; t += 8) {
        float s = 0.f;
        for (int j = lane; j < hd; j += 32) s = fmaf(q0w[(size_t)t * hd + j], qs[j], s);
        s = warp_sum(s);
        if (lane == 0) hs[t] = gelu1(s + q0b[t]);
    }
    __syncthreads();
    for (int j = warp; j < hd; j += 8) {
        float s = 0.f;
        for (int t = lane; t < hid; t += 32) s = fmaf(q2w[(size_t)j * hid + t], hs[t], s);
        s = warp_sum(s);
        if (lane == 0) qp[j] = qs[j] * (scale[h * hd + j] * (1.0f + tanh1(s + q2b[j])));
    }
}

// q_h *= scale_h * (1 + tanh(m)) for every (row, coordinate), m the query MLP's output (nn.rs:148).
__global__ void k_ssmax_apply(float *q, const float *m, const float *scale, int R, int d) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * d) return;
    q[i] = q[i] * (scale[i % d] * (1.0f + tanh1(m[i])));
}

// ---- attention over the stored cache ------------------------------------------------------------------------

// A 16-byte vector of stored elements from any alignment, zero past `len` (ragged chunk tails).
template <int KV, int EPV>
__device__ __forceinline__ uint4 gather_vec(const uint8_t *row, int k, int len) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < EPV; e++) {
        if (k + e < len) {
            if (KV == 0) {
                w[e] = __float_as_uint(__ldg(reinterpret_cast<const float *>(row) + k + e));
            } else if (KV == 1) {
                uint32_t v = (uint16_t)__ldg(reinterpret_cast<const short *>(row) + k + e);
                w[e >> 1] |= v << (16 * (e & 1));
            } else {
                uint32_t v = (uint8_t)__ldg(reinterpret_cast<const signed char *>(row) + k + e);
                w[e >> 2] |= v << (8 * (e & 3));
            }
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Keys-parallel attention for few rows (flash-decoding). One block per (item, head); an item is KS = 8 * EPV
// consecutive keys of one stored chunk (32 KB of keys and values at head width 128, whatever the format). Lane
// v = tid & 7 holds one 16-byte vector (EPV keys) of each of its dims j = (tid >> 3) + 16 t, for keys and for
// values, loaded once and kept in registers while the rows go through in sub-blocks of RSB. Integer keys: the
// query is multiplied by the chunk's key scales (predict.rs:486-497); integer values: the weighted sum is
// multiplied by the value scales afterwards (nn.rs:253-256). Each (item, row, head) leaves (max, weight sum,
// weighted values) for the merge.
template <int KV, int HD, int RSB>
__global__ void __launch_bounds__(128) k_attend_decode(AttnArgs a) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    // 8-byte vectors for 8-bit values keep a lane at 8 keys, as 16-byte vectors do for 16-bit ones
    constexpr int W = KvFmt<KV>::W, VB = KV == 2 ? 8 : 16, EPV = VB / W, KS = 8 * EPV, DG = 16;
    constexpr int DPT = HD >= DG ? HD / DG : 1;
    __shared__ __align__(16) float qsm[RSB][HD];
    __shared__ __align__(16) float red[4][RSB][KS];
    __shared__ __align__(16) float psm[RSB][KS];
    const int item = blockIdx.x, h = blockIdx.y, H = gridDim.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, v = tid & 7, jg = tid >> 3;
    const int2 it = a.items[item];
    const int ci = it.x, k0 = it.y;
    const int rc = min(a.chunk, a.rows - ci * a.chunk);
    const int len = min(KS, rc - k0);
    const uint8_t *rec = a.layer + (size_t)ci * a.full;
    const float *sc = reinterpret_cast<const float *>(rec);
    const uint8_t *body = rec + (KV ? 8 * (size_t)a.d : 0);
    const uint8_t *kb = body + ((size_t)h * HD * rc + k0) * W;
    const uint8_t *vb = body + ((size_t)(a.d + h * HD) * rc + k0) * W;
    const size_t rowb = (size_t)rc * W;
    const bool fast = len == KS && ((((uintptr_t)kb) | ((uintptr_t)vb) | rowb) & (VB - 1)) == 0;
    const uint64_t pol = policy_evict_first();
    uint4 kr[DPT], vr[DPT];
#pragma unroll
    for (int t = 0; t < DPT; t++) {
        const int j = jg + DG * t;
        if (j < HD) {
            if (fast && VB == 16) {
                kr[t] = ld_stream16(kb + j * rowb + v * 16, pol);
                vr[t] = ld_stream16(vb + j * rowb + v * 16, pol);
            } else if (fast) {
                kr[t] = ld_stream8(kb + j * rowb + v * 8, pol);
                vr[t] = ld_stream8(vb + j * rowb + v * 8, pol);
            } else {
                kr[t] = gather_vec<KV, EPV>(kb + j * rowb, v * EPV, len);
                vr[t] = gather_vec<KV, EPV>(vb + j * rowb, v * EPV, len);
            }
        } else {
            kr[t] = make_uint4(0u, 0u, 0u, 0u);
            vr[t] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    for (int rb0 = 0; rb0 < a.R; rb0 += RSB) {
        const int nr = min(RSB, a.R - rb0);
        __syncthreads();
        for (int i = tid; i < RSB * HD; i += 128) {
            int r = i / HD, j = i % HD;
            float qv = r < nr ? a.q[(size_t)(rb0 + r) * a.ldq + h * HD + j] : 0.f;
            if (KV) qv *= sc[h * HD + j];
            qsm[r][j] = qv;
        }
        __syncthreads();
        float sp[RSB][EPV];
#pragma unroll
        for (int r = 0; r < RSB; r++)
#pragma unroll
            for (int e = 0; e < EPV; e++) sp[r][e] = 0.f;
#pragma unroll
        for (int t = 0; t < DPT; t++) {
            const int j = min(jg + DG * t, HD - 1);  // rows past HD hold zeros
#pragma unroll
            for (int e = 0; e < EPV; e++) {
                const float kv = unpack<KV>(kr[t], e);
#pragma unroll
                for (int r = 0; r < RSB; r++) sp[r][e] = fmaf(qsm[r][j], kv, sp[r][e]);
            }
        }
#pragma unroll
        for (int r = 0; r < RSB; r++)
#pragma unroll
            for (int e = 0; e < EPV; e++) {
                float x = sp[r][e];
                x += __shfl_xor_sync(0xffffffffu, x, 8);
                x += __shfl_xor_sync(0xffffffffu, x, 16);
                sp[r][e] = x;
            }
        if (lane < 8) {
#pragma unroll
            for (int r = 0; r < RSB; r++)
#pragma unroll
                for (int e = 0; e < EPV; e++) red[warp][r][v * EPV + e] = sp[r][e];
        }
        __syncthreads();
        for (int r = warp; r < nr; r += 4) {
            float mx = -FLT_MAX;
            for (int k = lane; k < KS; k += 32) {
                float s = (red[0][r][k] + red[1][r][k]) + (red[2][r][k] + red[3][r][k]);
                psm[r][k] = s;
                if (k < len) mx = fmaxf(mx, s);
            }
            mx = warp_max(mx);
            float sum = 0.f;
            for (int k = lane; k < KS; k += 32) {
                float p = k < len ? exp1(psm[r][k] - mx) : 0.f;
                psm[r][k] = p;
                sum += p;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                float *ms = a.part_ms + (((size_t)item * a.R + rb0 + r) * H + h) * 2;
                ms[0] = mx, ms[1] = sum;
            }
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < DPT; t++) {
            const int j = jg + DG * t;
#pragma unroll
            for (int r = 0; r < RSB; r++) {
                float pv = 0.f;
#pragma unroll
                for (int e = 0; e < EPV; e++) pv = fmaf(psm[r][v * EPV + e], unpack<KV>(vr[t], e), pv);
                pv += __shfl_xor_sync(0xffffffffu, pv, 1);
                pv += __shfl_xor_sync(0xffffffffu, pv, 2);
                pv += __shfl_xor_sync(0xffffffffu, pv, 4);
                if (v == (r & 7) && r < nr && j < HD)
                    a.part_acc[((size_t)item * a.R + rb0 + r) * a.d + h * HD + j] = KV ? pv * sc[a.d + h * HD + j] : pv;
            }
        }
    }
}

// Row-blocked attention for many rows (one block: 64 rows x one head x a range of 64-key tiles). Keys and
// values are widened (and scaled, for integer formats) into shared memory as they arrive, scores and weighted
// sums run on 4 x 4 / 4 x (head width / 16) register tiles, and the softmax is kept online across tiles with
// the reference's rescaling rule (nn.rs:207-215).
template <int KV, int HD>
__global__ void __launch_bounds__(256, 2) k_attend_flash(AttnArgs a) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    constexpr int W = KvFmt<KV>::W, EPV = KvFmt<KV>::EPV, BQ = FLASH_ROWS, KT = FLASH_KEYS;
    constexpr int OD = HD >= 16 ? HD / 16 : 1;
    constexpr int VPR = KT / EPV;
    extern __shared__ __align__(16) float sm[];
    float *Qt = sm;              // [HD][BQ]
    float *Kt = Qt + HD * BQ;    // [HD][KT]
    float *Vt = Kt + HD * KT;    // [KT][HD]
    float *Pt = Vt + KT * HD;    // [KT][BQ]
    const int tid = threadIdx.x, tr = tid >> 4, tk = tid & 15;
    const int h = blockIdx.y, split = blockIdx.z, r0 = blockIdx.x * BQ, d = a.d, H = gridDim.y;
    for (int i = tid; i < BQ * HD; i += 256) {
        int r = i % BQ, j = i / BQ;
        Qt[j * BQ + r] = r0 + r < a.R ? a.q[(size_t)(r0 + r) * a.ldq + h * HD + j] : 0.f;
    }
    float mrun[4], lrun[4], o[4][OD];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        mrun[i] = -FLT_MAX, lrun[i] = 0.f;
#pragma unroll
        for (int e = 0; e < OD; e++) o[i][e] = 0.f;
    }
    const int t0 = split * a.tiles_per_split, t1 = min(a.ntiles, t0 + a.tiles_per_split);
    const uint64_t pol = policy_evict_first();
    for (int t = t0; t < t1; t++) {
        const int4 tile = a.tiles[t];
        const int ci = tile.x, k0 = tile.y, len = tile.z;
        const int rc = min(a.chunk, a.rows - ci * a.chunk);
        const uint8_t *rec = a.layer + (size_t)ci * a.full;
        const float *sc = reinterpret_cast<const float *>(rec);
        const uint8_t *body = rec + (KV ? 8 * (size_t)d : 0);
        const uint8_t *kb = body + ((size_t)h * HD * rc + k0) * W;
        const uint8_t *vb = body + ((size_t)(d + h * HD) * rc + k0) * W;
        const size_t rowb = (size_t)rc * W;
        const bool fast = len == KT && ((((uintptr_t)kb) | ((uintptr_t)vb) | rowb) & 15) == 0;
        __syncthreads();
        if (fast) {
            for (int i = tid; i < HD * VPR; i += 256) {
                int j = i / VPR, vv = i % VPR;
                uint4 raw = ld_stream16(kb + j * rowb + vv * 16, pol);
                float s = KV ? sc[h * HD + j] : 1.f;
#pragma unroll
                for (int e = 0; e < EPV; e++) Kt[j * KT + vv * EPV + e] = KV ? unpack<KV>(raw, e) * s : unpack<KV>(raw, e);
            }
            for (int i = tid; i < HD * VPR; i += 256) {
                int j = i % HD, vv = i / HD;
                uint4 raw = ld_stream16(vb + j * rowb + vv * 16, pol);
                float s = KV ? sc[d + h * HD + j] : 1.f;
#pragma unroll
                for (int e = 0; e < EPV; e++) Vt[(vv * EPV + e) * HD + j] = KV ? unpack<KV>(raw, e) * s : unpack<KV>(raw, e);
            }
        } else {
            for (int i = tid; i < HD * KT; i += 256) {
                int j = i / KT, k = i % KT;
                float val = 0.f;
                if (k < len) {
                    val = load_elem<KV>(body, (size_t)(h * HD + j) * rc + k0 + k);
                    if (KV) val *= sc[h * HD + j];
                }
                Kt[j * KT + k] = val;
            }
            for (int i = tid; i < HD * KT; i += 256) {
                int j = i % HD, k = i / HD;
                float val = 0.f;
                if (k < len) {
                    val = load_elem<KV>(body, (size_t)(d + h * HD + j) * rc + k0 + k);
                    if (KV) val *= sc[d + h * HD + j];
                }
                Vt[k * HD + j] = val;
            }
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int k = 0; k < 4; k++) s[i][k] = 0.f;
#pragma unroll 8
        for (int j = 0; j < HD; j++) {
            float4 qa = *reinterpret_cast<const float4 *>(&Qt[j * BQ + 4 * tr]);
            float4 kk = *reinterpret_cast<const float4 *>(&Kt[j * KT + 4 * tk]);
            float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int k = 0; k < 4; k++) s[i][k] = fmaf(qv[i], kv[k], s[i][k]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float mx = -FLT_MAX;
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (4 * tk + k < len) mx = fmaxf(mx, s[i][k]);
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mnew = fmaxf(mrun[i], mx);
            const float f = lrun[i] > 0.f ? exp1(mrun[i] - mnew) : 0.f;
            float ps = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float p = 4 * tk + k < len ? exp1(s[i][k] - mnew) : 0.f;
                s[i][k] = p;
                ps += p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            lrun[i] = lrun[i] * f + ps;
            mrun[i] = mnew;
#pragma unroll
            for (int e = 0; e < OD; e++) o[i][e] *= f;
        }
#pragma unroll
        for (int k = 0; k < 4; k++)
            *reinterpret_cast<float4 *>(&Pt[(4 * tk + k) * BQ + 4 * tr]) = make_float4(s[0][k], s[1][k], s[2][k], s[3][k]);
        __syncthreads();
        if (tk * OD < HD) {
#pragma unroll 4
            for (int k = 0; k < KT; k++) {
                float4 pa = *reinterpret_cast<const float4 *>(&Pt[k * BQ + 4 * tr]);
                float pv[4] = {pa.x, pa.y, pa.z, pa.w};
                float vv[OD];
#pragma unroll
                for (int e = 0; e < OD; e++) vv[e] = Vt[k * HD + tk * OD + e];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int e = 0; e < OD; e++) o[i][e] = fmaf(pv[i], vv[e], o[i][e]);
            }
        }
    }
    if (tk * OD >= HD) return;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = r0 + 4 * tr + i;
        if (r >= a.R) continue;
        if (a.splits == 1 && !a.parts_only) {
            const float inv = 1.0f / lrun[i];
#pragma unroll
            for (int e = 0; e < OD; e++) a.out[(size_t)r * a.ldo + h * HD + tk * OD + e] = o[i][e] * inv;
        } else {
#pragma unroll
            for (int e = 0; e < OD; e++) a.part_acc[((size_t)split * a.R + r) * d + h * HD + tk * OD + e] = o[i][e];
            if (tk == 0) {
                float *ms = a.part_ms + (((size_t)split * a.R + r) * H + h) * 2;
                ms[0] = mrun[i], ms[1] = lrun[i];
            }
        }
    }
}

// Log-sum-exp merge of the parts of each (row, head) (nn.rs:261-276 merge, then 280-286 finish). One block of
// 256 threads per (row, head): the part weights e^(m_p - M) first, then each warp sums a share of the parts
// with 16-byte loads along the head's values, and the warps' sums meet in shared memory.
__global__ void __launch_bounds__(256) k_attend_merge(const float *ms, const float *acc, int P, int R, int H, int d,
                                                      float *out, int ldo) {
    pdl_trigger();
    pdl_wait();  // the inputs come from the kernel before
    extern __shared__ __align__(16) float wsm[];  // [P] part weights, then [8][hd] warp sums
    __shared__ float red[8];
    const int r = blockIdx.x / H, h = blockIdx.x % H, hd = d / H, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = -FLT_MAX;
    for (int p = tid; p < P; p += blockDim.x) {
        const float *q = ms + (((size_t)p * R + r) * H + h) * 2;
        if (q[1] > 0.f) mx = fmaxf(mx, q[0]);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < 8; w++) M = fmaxf(M, red[w]);
    __syncthreads();
    float ssum = 0.f;
    for (int p = tid; p < P; p += blockDim.x) {
        const float *q = ms + (((size_t)p * R + r) * H + h) * 2;
        float w = q[1] > 0.f ? exp1(q[0] - M) : 0.f;
        wsm[p] = w;
        ssum = fmaf(q[1], w, ssum);
    }
    ssum = warp_sum(ssum);
    if (lane == 0) red[warp] = ssum;
    __syncthreads();
    float S = 0.f;
    for (int w = 0; w < 8; w++) S += red[w];
    const float inv = 1.0f / S;
    float *wsum = wsm + ((P + 3) & ~3);  // [8][hd]
    const float *base = acc + (size_t)r * d + h * hd;
    const size_t pstride = (size_t)R * d;
    if ((hd & 3) == 0 && ((d & 3) == 0)) {
        // lanes along the head's values four at a time; warps over the parts
        for (int j0 = lane * 4; j0 < hd; j0 += 128) {
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            int p = warp;
#pragma unroll 4
            for (; p < P; p += 8) {
                const float4 v = *reinterpret_cast<const float4 *>(base + p * pstride + j0);
                const float w = wsm[p];
                o.x = fmaf(v.x, w, o.x), o.y = fmaf(v.y, w, o.y), o.z = fmaf(v.z, w, o.z), o.w = fmaf(v.w, w, o.w);
            }
            *reinterpret_cast<float4 *>(wsum + warp * hd + j0) = o;
        }
    } else {
        for (int j = lane; j < hd; j += 32) {
            float o = 0.f;
            for (int p = warp; p < P; p += 8) o = fmaf(base[p * pstride + j], wsm[p], o);
            wsum[warp * hd + j] = o;
        }
    }
    __syncthreads();
    for (int j = tid; j < hd; j += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < 8; w++) o += wsum[w * hd + j];
        out[(size_t)r * ldo + h * hd + j] = o * inv;
    }
}

// Training rows split across devices: this device's parts of each (row, head) into one unnormalised state, as the
// merge above but without the division, written as one part of the merge (ms_out [R][H][2] = max, weight sum;
// acc_out [R][d] = weighted values), so that the states of all devices for a row are merged by k_attend_merge.
__global__ void __launch_bounds__(256) k_merge_state(const float *ms, const float *acc, int P, int R, int H, int d,
                                                     float *ms_out, float *acc_out) {
    extern __shared__ __align__(16) float wsm[];  // [P] part weights, then [8][hd] warp sums
    __shared__ float red[8];
    const int r = blockIdx.x / H, h = blockIdx.x % H, hd = d / H, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = -FLT_MAX;
    for (int p = tid; p < P; p += blockDim.x) {
        const float *q = ms + (((size_t)p * R + r) * H + h) * 2;
        if (q[1] > 0.f) mx = fmaxf(mx, q[0]);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < 8; w++) M = fmaxf(M, red[w]);
    __syncthreads();
    float ssum = 0.f;
    for (int p = tid; p < P; p += blockDim.x) {
        const float *q = ms + (((size_t)p * R + r) * H + h) * 2;
        const float w = q[1] > 0.f ? exp1(q[0] - M) : 0.f;
        wsm[p] = w;
        ssum = fmaf(q[1], w, ssum);
    }
    ssum = warp_sum(ssum);
    if (lane == 0) red[warp] = ssum;
    __syncthreads();
    float S = 0.f;
    for (int w = 0; w < 8; w++) S += red[w];
    float *wsum = wsm + ((P + 3) & ~3);  // [8][hd]
    const float *base = acc + (size_t)r * d + h * hd;
    const size_t pstride = (size_t)R * d;
    for (int j = lane; j < hd; j += 32) {
        float o = 0.f;
        for (int p = warp; p < P; p += 8) o = fmaf(base[p * pstride + j], wsm[p], o);
        wsum[warp * hd + j] = o;
    }
    __syncthreads();
    float *dst = acc_out + (size_t)r * d + h * hd;
    for (int j = tid; j < hd; j += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < 8; w++) o += wsum[w * hd + j];
        dst[j] = o;
    }
    if (tid == 0) {
        float *q = ms_out + ((size_t)r * H + h) * 2;
        q[0] = S > 0.f ? M : -FLT_MAX;
        q[1] = S;
    }
}

// The sharded stage's merge across devices, around two collectives (an all-reduce of the maxima, a reduce-scatter of
// the scaled states): one state per (row, head), ms [R][H][2] = (max, weight sum), acc [R][d] weighted values.
// m_out[r][h]: the state's max (-FLT_MAX without weight).
__global__ void k_state_max(const float *ms, int n, float *m_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) m_out[i] = ms[2 * (size_t)i + 1] > 0.f ? ms[2 * (size_t)i] : -FLT_MAX;
}

// packed[r] = (acc[r] w_h, s_h w_h over h) with w_h = e^(m - M), M the maximum over devices (0 without weight).
__global__ void k_state_pack(const float *ms, const float *acc, const float *m_all, int R, int H, int d, float *packed) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x, w = (size_t)d + H;
    if (i >= (size_t)R * w) return;
    const int r = (int)(i / w), c = (int)(i % w), h = c < d ? c / (d / H) : c - d;
    const float *st = ms + ((size_t)r * H + h) * 2;
    const float f = st[1] > 0.f ? exp1(st[0] - m_all[(size_t)r * H + h]) : 0.f;
    packed[i] = (c < d ? acc[(size_t)r * d + c] : st[1]) * f;
}

// nn.rs:280-286 finish of the summed states: weighted values / weight sum.
__global__ void k_state_finish(const float *packed, int R, int H, int d, float *out, int ldo) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)R * d) return;
    const int r = (int)(i / d), c = (int)(i % d);
    const float *p = packed + (size_t)r * (d + H);
    out[(size_t)r * ldo + c] = p[c] / p[d + c / (d / H)];
}

// ---- fitting's chunk packer (fit.rs:549-576) ---------------------------------------------------------------

__device__ __forceinline__ int16_t sat16(float v) {
    if (v != v) return 0;
    if (v >= 32767.f) return 32767;
    if (v <= -32768.f) return -32768;
    return (int16_t)v;
}
__device__ __forceinline__ int8_t sat8(float v) {
    if (v != v) return 0;
    if (v >= 127.f) return 127;
    if (v <= -128.f) return -128;
    return (int8_t)v;
}

// One block per (chunk, coordinate): kvT is [2d][rows] (keys' coordinates, then values'); the coordinate's
// values over the chunk's rows get one scale max|x| / 32767 (or / 127), 1 if all zero, and are rounded half away
// from zero with saturation, exactly as the CPU writes them.
__global__ void __launch_bounds__(256) k_pack(const float *kvT, int ld, int d, int rows, int chunk, int kv,
                                              uint8_t *out) {
    const int ci = blockIdx.x, j = blockIdx.y, tid = threadIdx.x;
    const int r0 = ci * chunk, rc = min(chunk, rows - r0);
    const float *row = kvT + (size_t)j * ld + r0;
    uint8_t *rec = out + (size_t)ci * record_bytes(kv, d, chunk);
    if (kv == 0) {
        float *o = reinterpret_cast<float *>(rec) + (size_t)j * rc;
        for (int i = tid; i < rc; i += blockDim.x) o[i] = row[i];
        return;
    }
    __shared__ float red[8];
    float big = 0.f;
    for (int i = tid; i < rc; i += blockDim.x) big = fmaxf(big, fabsf(row[i]));
    big = warp_max(big);
    if ((tid & 31) == 0) red[tid >> 5] = big;
    __syncthreads();
    big = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) big = fmaxf(big, red[w]);
    const float top = kv == 1 ? 32767.f : 127.f;
    const float s = big > 0.f ? big / top : 1.f;
    const float inv = 1.f / s;
    if (tid == 0) reinterpret_cast<float *>(rec)[j] = s;
    uint8_t *body = rec + 8 * (size_t)d;
    if (kv == 1) {
        int16_t *o = reinterpret_cast<int16_t *>(body) + (size_t)j * rc;
        for (int i = tid; i < rc; i += blockDim.x) o[i] = sat16(roundf(row[i] * inv));
    } else {
        int8_t *o = reinterpret_cast<int8_t *>(body) + (size_t)j * rc;
        for (int i = tid; i < rc; i += blockDim.x) o[i] = sat8(roundf(row[i] * inv));
    }
}

// model.rs:185-200 add_y: a class row of the table, or weight * y + bias for regression
__global__ void k_add_y(float *h, const float *y, int rows, int d, int max_classes, const float *table) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)rows * d) return;
    const int r = (int)(i / d), c = (int)(i % d);
    if (max_classes > 0) {
        const float yc = y[r];
        // a label outside the class table poisons the row instead of reading past the table
        if (!(yc >= 0.f && yc < (float)max_classes)) {
            h[i] = __int_as_float(0x7fc00000);
            return;
        }
        h[i] += table[(size_t)(int)yc * d + c];
    } else
        h[i] += table[c] * y[r] + table[d + c];
}

// ---- heads (table.rs) -----------------------------------------------------------------------------------------

// table.rs:265-269 and 70-78: one member's logits added to the f64 sums in its class order, then optionally the
// temperature softmax. One thread per row.
__global__ void k_class_head(const float *logits, int rows, int classes, int stride, const int32_t *mc, double *sums,
                             int finish, int members, double temperature) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    double *row = sums + (size_t)r * classes;
    for (int c = 0; c < classes; c++) {
        const int src = mc[c];
        // a class index outside the logits poisons the sum instead of reading past the row
        row[c] += (src >= 0 && src < stride) ? (double)logits[(size_t)r * stride + src] : __longlong_as_double(0x7ff8000000000000ll);
    }
    if (!finish) return;
    const double inv = 1.0 / ((double)members * temperature);
    double top = -DBL_MAX;
    for (int c = 0; c < classes; c++) top = fmax(top, row[c]);
    double sum = 0.0;
    for (int c = 0; c < classes; c++) row[c] = exp((row[c] - top) * inv);
    for (int c = 0; c < classes; c++) sum += row[c];
    for (int c = 0; c < classes; c++) row[c] /= sum;
}

__device__ __forceinline__ uint32_t total_key(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_key(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// table.rs:292-346 QuantileDist for one row (f32 arithmetic, sums in index order as iter().sum does).
struct QDist {
    const float *q;
    int n;
    float tl0, tl1, tr0, tr1;
    __device__ float level(int i) const { return (float)(i + 1) / (float)(n + 1); }
    __device__ float icdf(float alpha) const {
        if (alpha < level(0)) return tl0 * logf(fmaxf(alpha, 1e-6f)) + tl1;
        if (alpha > level(n - 1)) return tr0 * logf(fmaxf(1.0f - alpha, 1e-6f)) + tr1;
        if (alpha >= level(n - 1)) return q[n - 1];
        // partition_point over levels[..n-1] of (l <= alpha): levels rise, so binary search
        int lo = 0, hi = n - 1;
        while (lo < hi) {
            int mid = (lo + hi) >> 1;
            if (level(mid) <= alpha)
                lo = mid + 1;
            else
                hi = mid;
        }
        int i = lo > 0 ? lo - 1 : 0;
        if (i > n - 2) i = n - 2;
        float t = (alpha - level(i)) / fmaxf(level(i + 1) - level(i), 1e-6f);
        t = fminf(fmaxf(t, 0.f), 1.f);
        return q[i] + t * (q[i + 1] - q[i]);
    }
};

// One block per row: bitonic sort of the row's outputs in total order (padding sorts last), then one thread
// reads the distribution off as the reference does and adds the back-transformed numbers to the outputs.
__global__ void __launch_bounds__(1024) k_regression_head(const float *qout, int rows, int nq, int stride,
                                                          const double *alphas, int na, double tmean, double tscale,
                                                          double *mean, double *var, double *median, double *quant,
                                                          int npow2) {
    extern __shared__ uint32_t keys[];  // [npow2]
    const int r = blockIdx.x, tid = threadIdx.x;
    for (int i = tid; i < npow2; i += blockDim.x) keys[i] = i < nq ? total_key(qout[(size_t)r * stride + i]) : 0xffffffffu;
    __syncthreads();
    for (int k = 2; k <= npow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < npow2; i += blockDim.x) {
                int p = i ^ j;
                if (p > i) {
                    uint32_t a = keys[i], b = keys[p];
                    bool up = (i & k) == 0;
                    if ((a > b) == up) keys[i] = b, keys[p] = a;
                }
            }
            __syncthreads();
        }
    }
    float *q = reinterpret_cast<float *>(keys);
    for (int i = tid; i < nq; i += blockDim.x) q[i] = from_key(keys[i]);
    __syncthreads();
    if (tid != 0) return;
    const int n = nq;
    QDist dd;
    dd.q = q, dd.n = n;
    int k = min(20, n / 4);
    if (k < 1) k = 1;
    float sl[2];
    for (int side = 0; side < 2; side++) {
        float sx = 0.f, sy = 0.f;
        for (int i = 0; i < k; i++) {
            float x = side == 0 ? logf(fmaxf(dd.level(i), 1e-6f)) : logf(fmaxf(1.0f - dd.level(n - k + i), 1e-6f));
            sx += x;
            sy += side == 0 ? q[i] : q[n - k + i];
        }
        float mx = sx / (float)k, my = sy / (float)k, cov = 0.f, vr = 0.f;
        for (int i = 0; i < k; i++) {
            float x = side == 0 ? logf(fmaxf(dd.level(i), 1e-6f)) : logf(fmaxf(1.0f - dd.level(n - k + i), 1e-6f));
            float y = side == 0 ? q[i] : q[n - k + i];
            cov += (x - mx) * (y - my);
        }
        cov /= (float)k;
        for (int i = 0; i < k; i++) {
            float x = side == 0 ? logf(fmaxf(dd.level(i), 1e-6f)) : logf(fmaxf(1.0f - dd.level(n - k + i), 1e-6f));
            vr += (x - mx) * (x - mx);
        }
        vr /= (float)k;
        sl[side] = fminf(fmaxf(fabsf(cov / fmaxf(vr, 1e-6f)), 0.01f), 100.f);
    }
    dd.tl0 = sl[0];
    dd.tl1 = q[0] - sl[0] * logf(fmaxf(dd.level(0), 1e-6f));
    dd.tr0 = -sl[1];
    dd.tr1 = q[n - 1] + sl[1] * logf(1.0f - fminf(dd.level(n - 1), 1.0f - 1e-6f));
    float s = 0.f;
    for (int i = 0; i < n; i++) s += q[i];
    const float m = s / (float)n;
    float v2 = 0.f;
    for (int i = 0; i < n; i++) v2 += (q[i] - m) * (q[i] - m);
    const float variance = v2 / (float)(n - 1);
    auto back = [&](float v) { return (double)v * tscale + tmean; };
    mean[r] += back(m);
    var[r] += back(variance);
    median[r] += back(dd.icdf(0.5f));
    for (int a = 0; a < na; a++) quant[(size_t)r * na + a] += back(dd.icdf((float)alphas[a]));
}

// ---- launchers ----------------------------------------------------------------------------------------------

int decode_keys_per_item(int kv) { return kv == 0 ? 32 : 64; }

static int g_max_smem_optin = 0;

cudaError_t kernels_init() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&g_max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    return cudaSuccess;
}

// Opt a kernel in to more than 48 KB of dynamic shared memory, once per (device, kernel) and size: the attribute
// belongs to the function on the current device, so a second device of the same process needs its own.
cudaError_t allow_dynamic_smem(const void *kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, size_t> done;
    std::lock_guard<std::mutex> lock(mu);
    size_t &have = done[{dev, kernel}];
    if (bytes <= have) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}
template <typename K>
static cudaError_t allow_smem(K kernel, size_t bytes) {
    return allow_dynamic_smem((const void *)kernel, bytes);
}

cudaError_t launch_linear(const LinArgs &a, float *stats_scratch, cudaStream_t s, uint64_t *launches) {
    if (a.M <= 0 || a.N <= 0) return cudaSuccess;
    if (a.M <= 8 && !a.bias_on_m) {
        const size_t smem = (size_t)a.M * a.K * sizeof(float);
        const int grid = (a.N + 3) / 4;
        if (a.M == 1) {
            cudaError_t e = allow_smem(k_gemv<1>, smem);
            if (e != cudaSuccess) return e;
            k_gemv<1><<<grid, 128, smem, s>>>(a);
        } else {
            cudaError_t e = allow_smem(k_gemv<8>, smem);
            if (e != cudaSuccess) return e;
            k_gemv<8><<<grid, 128, smem, s>>>(a);
        }
        TCU_LAUNCHED(launches);
        return cudaGetLastError();
    }
    if (a.tc_wtiles && a.tc_atiles && a.tc_atiles_bytes >= tc_split_bytes(a.M, a.K) && !a.bias_on_m && a.K % 64 == 0 &&
        a.K <= 2048 &&
        a.ldx % 4 == 0 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && gemm_tc_enabled())
        return launch_gemm_tc(a, reinterpret_cast<float4 *>(stats_scratch), s, launches);
    LinArgs b = a;
    if (a.lnw) {
        k_ln_stats<<<(a.M + 7) / 8, 256, 0, s>>>(a.x, a.ldx, a.M, a.K, stats_scratch);
        TCU_LAUNCHED(launches);
        b.stats = stats_scratch;
    }
    dim3 grid((a.N + 127) / 128, (a.M + 127) / 128);
    k_gemm<<<grid, 256, 0, s>>>(b);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_ln_apply(const float *x, int M, int K, const float *w, const float *b, float *y, cudaStream_t s,
                            uint64_t *launches) {
    k_ln_apply<<<(M + 7) / 8, 256, 0, s>>>(x, M, K, w, b, y);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_ssmax(float *q, int R, int d, int heads, int hid, const float *q0w, const float *q0b,
                         const float *q2w, const float *q2b, const float *scale, cudaStream_t s, uint64_t *launches) {
    const int hd = d / heads;
    // one block per (row, head) for few rows, and up to 128 rows at the shape whose weights it loads all at once
    if (R <= 16 || (R <= 128 && hd == 128 && hid == 64)) {
        const cudaError_t e = launch_pdl(k_ssmax_rows, dim3(R, heads), dim3(256), sizeof(float) * (hd + hid), s, q, d, heads, hid, q0w, q0b, q2w, q2b, scale);
        if (e != cudaSuccess) return e;
        TCU_LAUNCHED(launches);
        return cudaGetLastError();
    }
    const int rb = 16;
    const size_t smem = sizeof(float) * ((size_t)hid * (hd + 1) + (size_t)hd * (hid + 1) + (size_t)rb * hd + (size_t)rb * hid);
    cudaError_t e = allow_smem(k_ssmax, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((R + rb - 1) / rb, heads);
    e = launch_pdl(k_ssmax, grid, dim3(256), smem, s, q, R, d, heads, hid, q0w, q0b, q2w, q2b, scale, rb);
    if (e != cudaSuccess) return e;
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_ssmax_apply(float *q, const float *m, const float *scale, int R, int d, cudaStream_t s,
                               uint64_t *launches) {
    const size_t n = (size_t)R * d;
    const cudaError_t e = launch_pdl(k_ssmax_apply, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, q, m, scale, R, d);
    if (e != cudaSuccess) return e;
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

template <int KV, int HD>
static cudaError_t decode_hd(const AttnArgs &a, cudaStream_t s) {
    dim3 grid(a.nitems, a.heads);
    cudaError_t e;
    if (a.R == 1)
        e = launch_pdl(k_attend_decode<KV, HD, 1>, grid, dim3(128), 0, s, a);
    else
        e = launch_pdl(k_attend_decode<KV, HD, 8>, grid, dim3(128), 0, s, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int KV>
static cudaError_t decode_kv(int hd, const AttnArgs &a, cudaStream_t s) {
    switch (hd) {
        case 8: return decode_hd<KV, 8>(a, s);
        case 16: return decode_hd<KV, 16>(a, s);
        case 32: return decode_hd<KV, 32>(a, s);
        case 64: return decode_hd<KV, 64>(a, s);
        case 128: return decode_hd<KV, 128>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attend_merge(const AttnArgs &a, int parts, cudaStream_t s, uint64_t *launches) {
    const size_t smem = sizeof(float) * ((size_t)((parts + 3) & ~3) + 8 * (size_t)(a.d / a.heads));
    cudaError_t e = allow_smem(k_attend_merge, smem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_attend_merge, dim3(a.R * a.heads), dim3(256), smem, s, (const float *)a.part_ms, (const float *)a.part_acc, parts, a.R, a.heads, a.d, a.out, a.ldo);
    if (e != cudaSuccess) return e;
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_attend_decode(int kv, int hd, const AttnArgs &a, cudaStream_t s, uint64_t *launches) {
    cudaError_t e = kv == 0 ? decode_kv<0>(hd, a, s) : kv == 1 ? decode_kv<1>(hd, a, s) : decode_kv<2>(hd, a, s);
    if (e != cudaSuccess) return e;
    TCU_LAUNCHED(launches);
    if (a.parts_only) return cudaSuccess;
    return launch_attend_merge(a, a.nitems, s, launches);
}

template <int KV, int HD>
static cudaError_t flash_hd(const AttnArgs &a, cudaStream_t s) {
    const size_t smem = sizeof(float) * ((size_t)HD * FLASH_ROWS + (size_t)HD * FLASH_KEYS * 2 + (size_t)FLASH_KEYS * FLASH_ROWS);
    cudaError_t e = allow_smem(k_attend_flash<KV, HD>, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.R + FLASH_ROWS - 1) / FLASH_ROWS, a.heads, a.splits);
    e = launch_pdl(k_attend_flash<KV, HD>, grid, dim3(256), smem, s, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int KV>
static cudaError_t flash_kv(int hd, const AttnArgs &a, cudaStream_t s) {
    switch (hd) {
        case 8: return flash_hd<KV, 8>(a, s);
        case 16: return flash_hd<KV, 16>(a, s);
        case 32: return flash_hd<KV, 32>(a, s);
        case 64: return flash_hd<KV, 64>(a, s);
        case 128: return flash_hd<KV, 128>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attend_flash(int kv, int hd, const AttnArgs &a, cudaStream_t s, uint64_t *launches) {
    cudaError_t e = kv == 0 ? flash_kv<0>(hd, a, s) : kv == 1 ? flash_kv<1>(hd, a, s) : flash_kv<2>(hd, a, s);
    if (e != cudaSuccess) return e;
    TCU_LAUNCHED(launches);
    if (a.splits > 1 && !a.parts_only) return launch_attend_merge(a, a.splits, s, launches);
    return cudaSuccess;
}

cudaError_t launch_merge_state(const AttnArgs &a, int parts, float *ms_out, float *acc_out, cudaStream_t s,
                               uint64_t *launches) {
    if (a.R <= 0) return cudaSuccess;
    const size_t smem = sizeof(float) * ((size_t)((parts + 3) & ~3) + 8 * (size_t)(a.d / a.heads));
    cudaError_t e = allow_smem(k_merge_state, smem);
    if (e != cudaSuccess) return e;
    k_merge_state<<<a.R * a.heads, 256, smem, s>>>(a.part_ms, a.part_acc, parts, a.R, a.heads, a.d, ms_out, acc_out);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_state_max(const float *ms, int R, int H, float *m_out, cudaStream_t s, uint64_t *launches) {
    const int n = R * H;
    if (n <= 0) return cudaSuccess;
    k_state_max<<<(n + 255) / 256, 256, 0, s>>>(ms, n, m_out);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_state_pack(const float *ms, const float *acc, const float *m_all, int R, int H, int d, float *packed,
                              cudaStream_t s, uint64_t *launches) {
    const size_t n = (size_t)R * (d + H);
    if (!n) return cudaSuccess;
    k_state_pack<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ms, acc, m_all, R, H, d, packed);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_state_finish(const float *packed, int R, int H, int d, float *out, int ldo, cudaStream_t s,
                                uint64_t *launches) {
    const size_t n = (size_t)R * d;
    if (!n) return cudaSuccess;
    k_state_finish<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(packed, R, H, d, out, ldo);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

// predict.rs:590-629 layer_rows on the device: one layer's stored chunks widened to keys and values [rows][d]
// (value times its coordinate's scale for integer formats, one f32 multiply as the CPU does). Block (chunk,
// coordinate); each thread widens one 16-byte vector of the coordinate's row with the attention kernels' own
// unpack<KV>, or single elements where the row is not 16-byte aligned or ends inside the vector.
template <int KV>
__global__ void k_layer_rows(const uint8_t *layer, int rows, int chunk, int d, size_t full, float *k, float *v) {
    constexpr int W = KvFmt<KV>::W, EPV = 16 / W;
    const int ci = blockIdx.x, j = blockIdx.y;
    const int r0 = ci * chunk, rc = min(chunk, rows - r0);
    const uint8_t *rec = layer + (size_t)ci * full;
    const float scale = KV ? reinterpret_cast<const float *>(rec)[j] : 1.f;
    const uint8_t *row = rec + (KV ? 8 * (size_t)d : 0) + (size_t)j * rc * W;
    float *dst = j < d ? k + (size_t)r0 * d + j : v + (size_t)r0 * d + (j - d);
    for (int e0 = threadIdx.x * EPV; e0 < rc; e0 += blockDim.x * EPV) {
        const uint8_t *p = row + (size_t)e0 * W;
        if (e0 + EPV <= rc && ((uintptr_t)p & 15) == 0) {
            const uint4 vec = __ldg(reinterpret_cast<const uint4 *>(p));
#pragma unroll
            for (int e = 0; e < EPV; e++) {
                const float x = unpack<KV>(vec, e);
                dst[(size_t)(e0 + e) * d] = KV ? x * scale : x;
            }
        } else {
            for (int e = e0; e < min(e0 + EPV, rc); e++) {
                const float x = load_elem<KV>(row, e);
                dst[(size_t)e * d] = KV ? x * scale : x;
            }
        }
    }
}

cudaError_t launch_layer_rows(int kv, const uint8_t *layer, int rows, int chunk, int d, float *k, float *v, cudaStream_t s,
                              uint64_t *launches) {
    if (rows < 1 || chunk < 1 || d < 1 || kv < 0 || kv > 2) return cudaErrorInvalidValue;
    const dim3 grid((rows + chunk - 1) / chunk, 2 * d);
    const size_t full = record_bytes(kv, d, chunk);
    if (kv == 0) k_layer_rows<0><<<grid, 64, 0, s>>>(layer, rows, chunk, d, full, k, v);
    else if (kv == 1) k_layer_rows<1><<<grid, 64, 0, s>>>(layer, rows, chunk, d, full, k, v);
    else k_layer_rows<2><<<grid, 64, 0, s>>>(layer, rows, chunk, d, full, k, v);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_pack(const float *kvT, int ld, int d, int rows, int chunk, int kv, uint8_t *out, cudaStream_t s,
                        uint64_t *launches) {
    dim3 grid((rows + chunk - 1) / chunk, 2 * d);
    k_pack<<<grid, 256, 0, s>>>(kvT, ld, d, rows, chunk, kv, out);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_add_y(float *h, const float *y, int rows, int d, int max_classes, const float *table,
                         cudaStream_t s, uint64_t *launches) {
    const size_t n = (size_t)rows * d;
    k_add_y<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h, y, rows, d, max_classes, table);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_class_head(const float *logits, int rows, int classes, int stride, const int32_t *member_classes,
                              double *sums, int finish, int members, double temperature, cudaStream_t s,
                              uint64_t *launches) {
    k_class_head<<<(rows + 127) / 128, 128, 0, s>>>(logits, rows, classes, stride, member_classes, sums, finish, members,
                                                     temperature);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

cudaError_t launch_regression_head(const float *qout, int rows, int nq, int stride, const double *alphas, int na,
                                   double tmean, double tscale, double *mean, double *var, double *median,
                                   double *quant, cudaStream_t s, uint64_t *launches) {
    int npow2 = 1;
    while (npow2 < nq) npow2 <<= 1;
    const size_t smem = sizeof(uint32_t) * (size_t)npow2;
    cudaError_t e = allow_smem(k_regression_head, smem);
    if (e != cudaSuccess) return e;
    const int threads = npow2 < 1024 ? (npow2 < 32 ? 32 : npow2) : 1024;
    k_regression_head<<<rows, threads, smem, s>>>(qout, rows, nq, stride, alphas, na, tmean, tscale, mean, var, median,
                                                  quant, npow2);
    TCU_LAUNCHED(launches);
    return cudaGetLastError();
}

}  // namespace tcu
