// The query's scalable-softmax MLP (nn.rs:138-149) for many rows, in one tensor-core kernel: for every (row, head)
// pair, q_h *= scale_h (1 + tanh(W2 GELU(W0 q_h + b0) + b2)), in place.
//
// A CTA takes 128 pairs (the rows of q viewed as [R * heads][hd]; a row's heads are contiguous). Head width 128 and
// 64 hidden units. The arithmetic is that of the two linear layers and the modulation kernel it replaces: each pair
// is scaled by a power of two and split into f16 hi + lo (as k_split_rows does), multiplied by the weights' split
// blocks (from the upload: rows scaled by powers of two, 128 x 64 blocks in blk_off order) with hi*hi + hi*lo +
// lo*hi per K chunk in a fresh TMEM accumulator, the chunks summed in registers, unscaled, biased and passed through
// GELU; the hidden units split the same way for the second product; the modulation then uses the reference's tanh.
#include <cfloat>

#include "device.cuh"
#include "kernels.cuh"
#include "pdl.cuh"
#include "tc.cuh"

namespace tcu {

using namespace tc;

namespace {

constexpr long long QM_WAIT_CYCLES = 2000000000ll;
constexpr int QM_ROWS = 128, QM_HD = 128, QM_HID = 64, QM_THREADS = 512;  // four warps per TMEM lane quarter
constexpr int QM_BLK = 128 * 64;  // halves of a 128-row block of 64 K values (hi or lo)

__device__ __forceinline__ float p2(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }
// e such that max * 2^e < 2^14 (0 for a zero row), as the row split of the linear layers computes it
__device__ __forceinline__ int row_exponent(float mx) {
    if (!(mx > 0.f)) return 0;
    const int e = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xff) - 126);
    return e < -120 ? -120 : (e > 120 ? 120 : e);
}

__device__ __forceinline__ void qm_bulk(void *dst, const void *src, uint32_t bytes, uint64_t *mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(mbar))
                 : "memory");
}
__device__ __forceinline__ void qm_expect(uint64_t *mbar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(
                     smem_addr(mbar)),
                 "r"(bytes)
                 : "memory");
}

// Eight values of row r (columns k0..k0+7 of a 64-wide block) into the hi and lo blocks.
__device__ __forceinline__ void put_split8(__half *hi, int r, int k0, const float *v, float sc) {
    __align__(16) __half hh[8], ll[8];
#pragma unroll
    for (int e = 0; e < 8; e++) split_f16(v[e] * sc, hh[e], ll[e]);
    const int off = blk_off(r, k0);
    *reinterpret_cast<uint4 *>(hi + off) = *reinterpret_cast<const uint4 *>(hh);
    *reinterpret_cast<uint4 *>(hi + QM_BLK + off) = *reinterpret_cast<const uint4 *>(ll);
}

}  // namespace

__global__ void __launch_bounds__(QM_THREADS, 1) k_qmlp_tc(QmlpArgs a) {
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Aq = reinterpret_cast<__half *>(smraw);  // 2 chunks x [hi 128 x 64][lo 128 x 64]: the pairs, split
    __half *W0 = Aq + 4 * QM_BLK;                      // 2 chunks x [hi 64 x 64][lo 64 x 64]
    __half *W2 = W0 + 2 * QM_BLK;                      // [hi 128 x 64][lo 128 x 64]
    __half *Ah = W2 + 2 * QM_BLK;                      // [hi 128 x 64][lo 128 x 64]: the hidden units, split
    float *xch = reinterpret_cast<float *>(Ah + 2 * QM_BLK);  // [4][128] quarter-row maxima
    float *un1 = xch + 4 * QM_ROWS, *un2 = un1 + QM_ROWS;    // [128] row unscales of the two products
    uint64_t *mb = reinterpret_cast<uint64_t *>(un2 + QM_ROWS);
    uint64_t *mW = mb, *mD1 = mb + 1, *mD2 = mb + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mb + 3);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    // per-column constants, read once: W0's unscale and bias (64 each), W2's (128 each), the query scale [heads][128]
    float *c_w0u = reinterpret_cast<float *>(tslot + 4), *c_b0 = c_w0u + QM_HID, *c_w2u = c_b0 + QM_HID,
          *c_b2 = c_w2u + QM_HD, *c_scl = c_b2 + QM_HD;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int p0 = blockIdx.x * QM_ROWS;
    if (warp == 0) {
        tmem_alloc(tslot, 256);  // the first product's two chunk accumulators (64 columns each), the second's 128
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(mW, 1), mbar_init(mD1, 1), mbar_init(mD2, 1);
        mbar_init_fence();
        *abort_flag = 0;
        // weights: the first 64 rows of each of W0's two K chunks (hi and lo), W2's one chunk
        const __half *w0 = reinterpret_cast<const __half *>(a.w0_tiles), *w2 = reinterpret_cast<const __half *>(a.w2_tiles);
        qm_expect(mW, 4 * (QM_BLK / 2) * 2 + 2 * QM_BLK * 2);
        for (int c = 0; c < 2; c++) {
            qm_bulk(W0 + c * QM_BLK, w0 + (size_t)c * 2 * QM_BLK, QM_BLK, mW);                      // hi rows 0-63
            qm_bulk(W0 + c * QM_BLK + QM_BLK / 2, w0 + (size_t)c * 2 * QM_BLK + QM_BLK, QM_BLK, mW);  // lo rows 0-63
        }
        qm_bulk(W2, w2, 2 * QM_BLK * 2, mW);
    }
    for (int i = threadIdx.x; i < QM_HID; i += QM_THREADS) c_w0u[i] = a.w0_unscale[i], c_b0[i] = a.b0[i];
    for (int i = threadIdx.x; i < QM_HD; i += QM_THREADS) c_w2u[i] = a.w2_unscale[i], c_b2[i] = a.b2[i];
    for (int i = threadIdx.x; i < a.heads * QM_HD; i += QM_THREADS) c_scl[i] = a.scale[i];
    __syncthreads();
    pdl_trigger();  // every block holds its tensor memory
    pdl_wait();     // the queries come from the kernel before
    // 1. the pairs: thread (row m, quarter c) holds head columns 32c..32c+31 of pair p0 + m
    const int m = tid & (QM_ROWS - 1), c = tid >> 7, p = p0 + m;
    const bool real = p < a.pairs;
    {
        float v[32];
        float mx = 0.f;
        if (real) {
            const float4 *src = reinterpret_cast<const float4 *>(a.q + (size_t)p * QM_HD + 32 * c);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 x = src[j];
                v[4 * j] = x.x, v[4 * j + 1] = x.y, v[4 * j + 2] = x.z, v[4 * j + 3] = x.w;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = 0.f;
        }
        xch[c * QM_ROWS + m] = mx;
        __syncthreads();
        const int e = row_exponent(fmaxf(fmaxf(xch[m], xch[QM_ROWS + m]), fmaxf(xch[2 * QM_ROWS + m], xch[3 * QM_ROWS + m])));
        if (c == 0) un1[m] = p2(-e);
        const float sc = p2(e);
#pragma unroll
        for (int g = 0; g < 4; g++) put_split8(Aq + (c >> 1) * 2 * QM_BLK, m, 32 * (c & 1) + 8 * g, v + 8 * g, sc);
    }
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    // 2. first product: two K chunks, each into a fresh accumulator (hi*hi, hi*lo, lo*hi per K step)
    if (tid == 0) {
        if (!mbar_wait(mW, 0, QM_WAIT_CYCLES)) *abort_flag = 1;
        if (!*abort_flag) {
            fence_after_sync();
            const uint32_t id = idesc_f16(QM_ROWS, QM_HID, 0, 0);
            const uint64_t st = 256 >> 4;
#pragma unroll
            for (int ch = 0; ch < 2; ch++) {
                const uint64_t dAh = smem_desc(smem_addr(Aq + ch * 2 * QM_BLK), 128, 1024), dAl = dAh + ((QM_BLK * 2) >> 4);
                const uint64_t dWh = smem_desc(smem_addr(W0 + ch * QM_BLK), 128, 1024), dWl = dWh + ((QM_BLK / 2 * 2) >> 4);
                const uint32_t t = tmem + 64 * ch;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    mma_f16(t, dAh + k * st, dWh + k * st, id, k > 0 ? 1u : 0u);
                    mma_f16(t, dAh + k * st, dWl + k * st, id, 1);
                    mma_f16(t, dAl + k * st, dWh + k * st, id, 1);
                }
            }
            mma_commit(mD1);
        }
    }
    __syncthreads();
    // 3. hidden units: thread (row r, quarter h2) takes 16 of the 64; GELU; split into the second product's A
    const int r = (warp & 3) * 32 + lane, h2 = warp >> 2;
    bool ok = !*abort_flag && mbar_wait(mD1, 0, QM_WAIT_CYCLES);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) *abort_flag = 1;
    fence_after_sync();
    {
        float x0[16], x1[16];
        if (ok) {
            tmem_ld16(tmem + lane_base + 16 * h2, x0);
            tmem_ld16(tmem + lane_base + 64 + 16 * h2, x1);
            tmem_wait_ld();
        }
        const float un = un1[r];
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const int n = 16 * h2 + e;
            float v = (ok ? (x0[e] + x1[e]) * un : 0.f) * c_w0u[n] + c_b0[n];
            v = gelu1(v);
            x0[e] = v;
            mx = fmaxf(mx, fabsf(v));
        }
        __syncthreads();  // every quarter-row maximum of phase 1 has been read
        xch[h2 * QM_ROWS + r] = mx;
        __syncthreads();
        const int e2 = row_exponent(fmaxf(fmaxf(xch[r], xch[QM_ROWS + r]), fmaxf(xch[2 * QM_ROWS + r], xch[3 * QM_ROWS + r])));
        if (h2 == 0) un2[r] = p2(-e2);
        const float sc = p2(e2);
#pragma unroll
        for (int g = 0; g < 2; g++) put_split8(Ah, r, 16 * h2 + 8 * g, x0 + 8 * g, sc);
    }
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    // 4. second product: one K chunk of 64 into a 128-column accumulator
    if (tid == 0 && !*abort_flag) {
        const uint32_t id = idesc_f16(QM_ROWS, QM_HD, 0, 0);
        const uint64_t st = 256 >> 4;
        const uint64_t dAh = smem_desc(smem_addr(Ah), 128, 1024), dAl = dAh + ((QM_BLK * 2) >> 4);
        const uint64_t dWh = smem_desc(smem_addr(W2), 128, 1024), dWl = dWh + ((QM_BLK * 2) >> 4);
        const uint32_t t = tmem + 128;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            mma_f16(t, dAh + k * st, dWh + k * st, id, k > 0 ? 1u : 0u);
            mma_f16(t, dAh + k * st, dWl + k * st, id, 1);
            mma_f16(t, dAl + k * st, dWh + k * st, id, 1);
        }
        mma_commit(mD2);
    }
    __syncthreads();
    // 5. modulation: thread (row r, quarter h2) takes head columns 32 h2 .. 32 h2 + 31 of pair p0 + r
    ok = !*abort_flag && mbar_wait(mD2, 0, QM_WAIT_CYCLES);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) *abort_flag = 1;
    fence_after_sync();
    if (ok) {
        const int pr = p0 + r, hh = pr % a.heads;
        const float un = un2[r];
        {
            float x[32];
            tmem_ld32(tmem + lane_base + 128 + 32 * h2, x);
            tmem_wait_ld();
            if (pr < a.pairs) {
                float4 *qp = reinterpret_cast<float4 *>(a.q + (size_t)pr * QM_HD + 32 * h2);
                const float *scl = c_scl + hh * QM_HD + 32 * h2;
                const float *ws = c_w2u + 32 * h2, *bb = c_b2 + 32 * h2;
                float4 qv[8];
#pragma unroll
                for (int e4 = 0; e4 < 8; e4++) qv[e4] = qp[e4];  // every load before any store
#pragma unroll
                for (int e4 = 0; e4 < 8; e4++) {
                    float o[4] = {qv[e4].x, qv[e4].y, qv[e4].z, qv[e4].w};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int e = 4 * e4 + u;
                        const float mv = (x[e] * un) * ws[e] + bb[e];
                        o[u] = o[u] * (scl[e] * (1.0f + tanh1(mv)));
                    }
                    qv[e4] = make_float4(o[0], o[1], o[2], o[3]);
                }
#pragma unroll
                for (int e4 = 0; e4 < 8; e4++) qp[e4] = qv[e4];
            }
        }
    }
    if (*abort_flag && tid == 0 && a.err) *reinterpret_cast<volatile int *>(a.err) = 1;  // a report slot in host memory
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

size_t qmlp_tc_smem(int heads) {
    return sizeof(__half) * 10 * QM_BLK + sizeof(float) * 6 * QM_ROWS + 3 * sizeof(uint64_t) + 16 +
           sizeof(float) * (2 * QM_HID + 2 * QM_HD + (size_t)heads * QM_HD);
}

cudaError_t launch_qmlp_tc(const QmlpArgs &a, cudaStream_t s, uint64_t *launches) {
    if (a.hd != QM_HD || a.hid != QM_HID || !a.w0_tiles || !a.w2_tiles) return cudaErrorInvalidValue;
    const size_t smem = qmlp_tc_smem(a.heads);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = allow_dynamic_smem((const void *)k_qmlp_tc, smem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(k_qmlp_tc, dim3((a.pairs + QM_ROWS - 1) / QM_ROWS), dim3(QM_THREADS), smem, s, a);
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
