// Kernels of the column stage of fitting (src/fit.rs:298-420 of tabicl-anywhere): the training cells' labels, the
// inducing points' attention over one feature group's training cells (split over the rows, then merged), and the
// scatter of the inducing points' keys and values into the member's column cache. The linear layers between them run
// through launch_linear; the cells' own pass through a block reuses the prediction's column attention.
#include "kernels.cuh"
#include "device.cuh"

#include <algorithm>
#include <cfloat>

namespace tcu {

namespace {

constexpr int IND_THREADS = 128;  // inducing points per block (one query per thread)
constexpr int IND_KEYS = 32;      // training cells per shared-memory tile

// model.rs:185-200 add_y for the training cells (fit.rs:316-324): cell (r, g) of X [n * F][e] gets the row of label
// digit ((int)y[r] / divisor) % base (the plain label when base is 0), or weight * y + bias for a regression model.
// A label outside the class table poisons the cell instead of reading past the table.
__global__ void k_col_add_y(float *X, const float *y, int n, int F, int e, int max_classes, const float *table,
                            int divisor, int base) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)n * F * e) return;
    const int c = (int)(i % e), r = (int)(i / e / F);
    const float yv = y[r];
    if (max_classes > 0) {
        if (!(yv >= 0.f && yv < 2147483648.f)) {
            X[i] = __int_as_float(0x7fc00000);
            return;
        }
        const int lab = base > 0 ? ((int)yv / divisor) % base : (int)yv;
        if (lab >= max_classes) {
            X[i] = __int_as_float(0x7fc00000);
            return;
        }
        X[i] += table[(size_t)lab * e + c];
    } else
        X[i] += table[c] * yv + table[e + c];
}

// fit.rs:330-352 with nn.rs:187-228: the inducing points' scaled queries q [inds][e] (the same for every group)
// attend to group g's training cells, whose keys and values are the rows r * F + g of kv [n * F][2e] (keys, then
// values). Block (g, head h, z): split z / itiles of the cells ([z0, z0 + per)), inducing points of tile z % itiles,
// one per thread; the cells' head slices pass through shared memory a tile at a time, read by every thread at once.
// Each split leaves its (max, weight sum) and unnormalised weighted values per inducing point.
template <int HD>
__global__ void __launch_bounds__(IND_THREADS) k_ind_attend(const float *q, const float *kv, int n, int F, int e,
                                                           int inds, int per, int splits, float *part_ms,
                                                           float *part_acc) {
    __shared__ __align__(16) float Ks[IND_KEYS * HD], Vs[IND_KEYS * HD];
    const int g = blockIdx.x, h = blockIdx.y, heads = gridDim.y, itiles = gridDim.z / splits;
    const int sp = blockIdx.z / itiles, i = (blockIdx.z % itiles) * IND_THREADS + threadIdx.x;
    const int z0 = sp * per, z1 = min(n, z0 + per);
    float qr[HD], acc[HD];
    const float *qp = q + (size_t)min(i, inds - 1) * e + h * HD;
#pragma unroll
    for (int j = 0; j < HD; j++) qr[j] = qp[j], acc[j] = 0.f;
    float mx = -FLT_MAX, sum = 0.f;
    constexpr int V4 = HD / 4;
    for (int k0 = z0; k0 < z1; k0 += IND_KEYS) {
        const int nk = min(IND_KEYS, z1 - k0);
        for (int t = threadIdx.x; t < IND_KEYS * V4; t += IND_THREADS) {
            const int k = t / V4, j4 = t % V4;
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (k < nk) {
                const float *row = kv + ((size_t)(k0 + k) * F + g) * 2 * e + h * HD + 4 * j4;
                kk = *reinterpret_cast<const float4 *>(row);
                vv = *reinterpret_cast<const float4 *>(row + e);
            }
            reinterpret_cast<float4 *>(Ks)[t] = kk;
            reinterpret_cast<float4 *>(Vs)[t] = vv;
        }
        __syncthreads();
        float sc[IND_KEYS];
        float tm = -FLT_MAX;
#pragma unroll
        for (int k = 0; k < IND_KEYS; k++) {
            const float4 *kr = reinterpret_cast<const float4 *>(Ks + k * HD);
            float s = 0.f;
#pragma unroll
            for (int j4 = 0; j4 < V4; j4++) {
                const float4 kk = kr[j4];
                s = fmaf(qr[4 * j4], kk.x, s), s = fmaf(qr[4 * j4 + 1], kk.y, s);
                s = fmaf(qr[4 * j4 + 2], kk.z, s), s = fmaf(qr[4 * j4 + 3], kk.w, s);
            }
            sc[k] = k < nk ? s : -FLT_MAX;
            tm = fmaxf(tm, sc[k]);
        }
        const float nm = fmaxf(mx, tm), corr = exp1(mx - nm);
        sum *= corr;
#pragma unroll
        for (int j = 0; j < HD; j++) acc[j] *= corr;
#pragma unroll
        for (int k = 0; k < IND_KEYS; k++) {
            const float p = k < nk ? exp1(sc[k] - nm) : 0.f;
            sum += p;
            const float4 *vr = reinterpret_cast<const float4 *>(Vs + k * HD);
#pragma unroll
            for (int j4 = 0; j4 < V4; j4++) {
                const float4 vv = vr[j4];
                acc[4 * j4] = fmaf(p, vv.x, acc[4 * j4]), acc[4 * j4 + 1] = fmaf(p, vv.y, acc[4 * j4 + 1]);
                acc[4 * j4 + 2] = fmaf(p, vv.z, acc[4 * j4 + 2]), acc[4 * j4 + 3] = fmaf(p, vv.w, acc[4 * j4 + 3]);
            }
        }
        mx = nm;
        __syncthreads();
    }
    if (i >= inds) return;
    const size_t slot = (((size_t)g * heads + h) * splits + sp) * inds + i;
    part_ms[2 * slot] = mx, part_ms[2 * slot + 1] = sum;
    float4 *out = reinterpret_cast<float4 *>(part_acc + slot * HD);
#pragma unroll
    for (int j4 = 0; j4 < V4; j4++) out[j4] = make_float4(acc[4 * j4], acc[4 * j4 + 1], acc[4 * j4 + 2], acc[4 * j4 + 3]);
}

// nn.rs:261-286 merge and finish: the splits' states of each (group, inducing point, head) into att [F * inds][e]
// (the heads side by side), in split order.
__global__ void k_ind_merge(const float *part_ms, const float *part_acc, int F, int heads, int hd, int inds, int splits,
                            float *att) {
    const int e = heads * hd;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)F * inds * e) return;
    const int c = (int)(t % e), i = (int)(t / e % inds), g = (int)(t / e / inds), h = c / hd, j = c % hd;
    const size_t base = ((size_t)g * heads + h) * splits * inds + i;
    float M = -FLT_MAX;
    for (int s = 0; s < splits; s++) M = fmaxf(M, part_ms[2 * (base + (size_t)s * inds)]);
    float tot = 0.f, val = 0.f;
    for (int s = 0; s < splits; s++) {
        const size_t slot = base + (size_t)s * inds;
        const float w = exp1(part_ms[2 * slot] - M);
        tot += part_ms[2 * slot + 1] * w;
        val += part_acc[slot * hd + j] * w;
    }
    att[t] = val / tot;
}

// dst [times][count] = src [count], repeated: the inducing points under every group's attention output (the residual).
__global__ void k_repeat(float *dst, const float *src, size_t count, int times) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < count * times) dst[t] = src[t % count];
}

// fit.rs:392-404: the inducing points' keys and values for the second attention, kv2 [F * inds][2e], into the member's
// column cache: group g's block b of digit dg at col_kv + g * gstride + off, keys [e][inds] then values [e][inds].
__global__ void k_col_kv_scatter(const float *kv2, int F, int e, int inds, size_t gstride, size_t off, float *col_kv) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)F * inds * 2 * e) return;
    const int j = (int)(t % (2 * e)), i = (int)(t / (2 * e) % inds), g = (int)(t / (2 * e) / inds);
    const int which = j / e, c = j % e;
    col_kv[(size_t)g * gstride + off + ((size_t)which * e + c) * inds + i] = kv2[t];
}

inline unsigned blocks_of(size_t n) { return (unsigned)((n + 255) / 256); }

template <int HD>
cudaError_t ind_attend(const float *q, const float *kv, int n, int F, int e, int inds, int heads, int splits,
                       float *part_ms, float *part_acc, cudaStream_t s) {
    const int itiles = (inds + IND_THREADS - 1) / IND_THREADS, per = (n + splits - 1) / splits;
    k_ind_attend<HD><<<dim3(F, heads, splits * itiles), IND_THREADS, 0, s>>>(q, kv, n, F, e, inds, per, splits, part_ms,
                                                                          part_acc);
    return cudaGetLastError();
}

}  // namespace

bool ind_attend_takes(int e, int heads) {
    const int hd = heads > 0 && e % heads == 0 ? e / heads : 0;
    return hd == 4 || hd == 8 || hd == 16 || hd == 32 || hd == 64;
}

int ind_attend_splits(int n, int F, int heads, int inds) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int itiles = (inds + IND_THREADS - 1) / IND_THREADS;
    const long base = (long)F * heads * itiles;
    // about eight blocks per SM in all, each split at least a few tiles of cells
    const long want = (8L * sms + base - 1) / base;
    const long most = std::max(1, (n + 4 * IND_KEYS - 1) / (4 * IND_KEYS));
    int splits = (int)std::max(1L, std::min(want, most));
    const int per = (n + splits - 1) / splits;
    return (n + per - 1) / per;  // no empty split
}

cudaError_t launch_ind_attend(const float *q, const float *kv, int n, int F, int e, int inds, int heads, int splits,
                              float *part_ms, float *part_acc, float *att, cudaStream_t s, uint64_t *launches) {
    const int hd = e / heads;
    if (n < 1 || F < 1 || inds < 1 || splits < 1 || e % heads || e % 4) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(part_acc)) % 16) return cudaErrorInvalidValue;
    cudaError_t err = hd == 4    ? ind_attend<4>(q, kv, n, F, e, inds, heads, splits, part_ms, part_acc, s)
                      : hd == 8  ? ind_attend<8>(q, kv, n, F, e, inds, heads, splits, part_ms, part_acc, s)
                      : hd == 16 ? ind_attend<16>(q, kv, n, F, e, inds, heads, splits, part_ms, part_acc, s)
                      : hd == 32 ? ind_attend<32>(q, kv, n, F, e, inds, heads, splits, part_ms, part_acc, s)
                      : hd == 64 ? ind_attend<64>(q, kv, n, F, e, inds, heads, splits, part_ms, part_acc, s)
                                 : cudaErrorInvalidValue;
    if (err != cudaSuccess) return err;
    if (launches) ++*launches;
    k_ind_merge<<<blocks_of((size_t)F * inds * e), 256, 0, s>>>(part_ms, part_acc, F, heads, hd, inds, splits, att);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_col_add_y(float *X, const float *y, int n, int F, int e, int max_classes, const float *table,
                             int divisor, int base, cudaStream_t s, uint64_t *launches) {
    k_col_add_y<<<blocks_of((size_t)n * F * e), 256, 0, s>>>(X, y, n, F, e, max_classes, table, divisor, base);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_repeat(float *dst, const float *src, size_t count, int times, cudaStream_t s, uint64_t *launches) {
    k_repeat<<<blocks_of(count * times), 256, 0, s>>>(dst, src, count, times);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_col_kv_scatter(const float *kv2, int F, int e, int inds, size_t gstride, size_t off, float *col_kv,
                                  cudaStream_t s, uint64_t *launches) {
    k_col_kv_scatter<<<blocks_of((size_t)F * inds * 2 * e), 256, 0, s>>>(kv2, F, e, inds, gstride, off, col_kv);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
