// Linear layers of many rows on the tensor cores (tcgen05) at f32 accuracy: y (=|+=) act(W LN?(x) + b).
//
// A CTA computes a 128-row x 128-output tile, K in chunks of 64 staged twice-buffered in shared memory.
// Activations are split into f16 hi + lo on the fly after a power-of-two scaling per row (from a stats pass that
// also gives the LayerNorm's mean and 1/sigma); weights were split once at upload with a scaling per output row.
// The product is taken as hi*hi + hi*lo + lo*hi in one f32 accumulator in tensor memory; the epilogue undoes the
// two scalings, adds the bias, applies GELU and the residual, and writes through shared memory so that stores
// are coalesced (also when the output is written transposed).
#include <cfloat>
#include <cstdlib>

#include "device.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace tcu {

using namespace tc;

constexpr long long GEMM_WAIT_CYCLES = 2000000000ll;

__device__ __forceinline__ float p2(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Per row: LayerNorm mean and 1/sigma (when lnw is set, else 0 and 1), then the power-of-two scale that keeps the
// row's largest transformed magnitude below 2^14 and its inverse: stats[m] = {mean, rstd, scale, unscale}.
__global__ void k_row_stats_tc(const float *x, int ldx, int M, int K, const float *lnw, const float *lnb, float4 *stats) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const float *p = x + (size_t)row * ldx;
    float mean = 0.f, inv = 1.f;
    if (lnw) {
        float s = 0.f;
        for (int k = lane; k < K; k += 32) s += p[k];
        mean = warp_sum(s) / (float)K;
        float q = 0.f;
        for (int k = lane; k < K; k += 32) {
            float dd = p[k] - mean;
            q = fmaf(dd, dd, q);
        }
        inv = 1.0f / sqrtf(warp_sum(q) / (float)K + 1e-5f);
    }
    float mx = 0.f;
    for (int k = lane; k < K; k += 32) {
        const float v = lnw ? (p[k] - mean) * inv * lnw[k] + lnb[k] : p[k];
        mx = fmaxf(mx, fabsf(v));
    }
    mx = warp_max(mx);
    if (lane == 0) {
        int e = 0;
        if (mx > 0.f) {
            const int ex = (int)((__float_as_uint(mx) >> 23) & 0xff) - 126;
            e = 14 - ex;
            e = e < -120 ? -120 : (e > 120 ? 120 : e);
        }
        stats[row] = make_float4(mean, inv, p2(e), p2(-e));
    }
}

// The tensor cores' f32 accumulation is not rounded to nearest, so a long run of accumulations into one
// accumulator drifts by about an ulp per step. Each 64-wide chunk of K therefore gets fresh accumulators - the
// large hi*hi products in one, the small cross terms in another - and the chunks are added in registers with
// ordinary f32 arithmetic: at most four truncating steps on the large terms.
__global__ void __launch_bounds__(256, 1) k_gemm_tc(LinArgs a, const float4 *stats) {
    constexpr int BM = 128, BN = 128, BK = 64;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Ah = reinterpret_cast<__half *>(smraw);  // [2 stages][BM][BK] K-major, hi
    __half *Al = Ah + 2 * BM * BK;                    // lo
    __half *Wh = Al + 2 * BM * BK;                    // [2][BN][BK]
    __half *Wl = Wh + 2 * BN * BK;
    uint64_t *mbar = reinterpret_cast<uint64_t *>(Wl + 2 * BN * BK);  // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (warp == 0) {
        tmem_alloc(tslot, 512);  // [2 chunks] x (hi*hi accumulator, cross-term accumulator) x 128 columns
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
        *abort_flag = 0;
    }
    // this thread's staging row (A) and output row (W) stay fixed: 256 threads, 128 rows
    const int sm = tid % BM, kq = tid / BM;  // kq: which 8-column groups (kq, kq + 2, ...)
    const int am = m0 + sm, wn = n0 + sm;
    float4 st = make_float4(0.f, 1.f, 0.f, 0.f);
    if (am < a.M) st = stats[am];
    const float *arow = a.x + (size_t)(am < a.M ? am : 0) * a.ldx;
    const __half *wh_row = reinterpret_cast<const __half *>(a.tc_whi) + (size_t)(wn < a.N ? wn : 0) * a.K;
    const __half *wl_row = reinterpret_cast<const __half *>(a.tc_wlo) + (size_t)(wn < a.N ? wn : 0) * a.K;
    auto stage = [&](int c, int buf) {
        __half *ah = Ah + buf * BM * BK, *al = Al + buf * BM * BK, *wh = Wh + buf * BN * BK, *wl = Wl + buf * BN * BK;
#pragma unroll
        for (int g = kq; g < BK / 8; g += 2) {
            const int k = c * BK + g * 8;
            float v[8];
            if (am < a.M) {
                const float4 x0 = *reinterpret_cast<const float4 *>(arow + k), x1 = *reinterpret_cast<const float4 *>(arow + k + 4);
                v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w, v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
                if (a.lnw) {
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = (v[e] - st.x) * st.y * a.lnw[k + e] + a.lnb[k + e];
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = 0.f;
            }
            __align__(16) __half hh[8], ll[8];
#pragma unroll
            for (int e = 0; e < 8; e++) split_f16(v[e] * st.z, hh[e], ll[e]);
            const int off = kmajor_off(sm, g * 8, BM);
            *reinterpret_cast<uint4 *>(ah + off) = *reinterpret_cast<const uint4 *>(hh);
            *reinterpret_cast<uint4 *>(al + off) = *reinterpret_cast<const uint4 *>(ll);
            uint4 whv = make_uint4(0u, 0u, 0u, 0u), wlv = whv;
            if (wn < a.N) {
                whv = __ldg(reinterpret_cast<const uint4 *>(wh_row + k));
                wlv = __ldg(reinterpret_cast<const uint4 *>(wl_row + k));
            }
            const int woff = kmajor_off(sm, g * 8, BN);
            *reinterpret_cast<uint4 *>(wh + woff) = whv;
            *reinterpret_cast<uint4 *>(wl + woff) = wlv;
        }
    };
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot;
    const uint32_t id = idesc_f16(BM, BN, 0, 0);
    const int nk = a.K / BK;
    // this thread's share of the accumulators: lane (row) warp%4 * 32 + lane, columns (warp / 4) * 64 + [0, 64)
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int col0 = (warp >> 2) * 64;
    float sum[64];
#pragma unroll
    for (int e = 0; e < 64; e++) sum[e] = 0.f;
    uint32_t parity[2] = {0u, 0u};
    bool ok = true;
    stage(0, 0);
    fence_async_smem();
    __syncthreads();
    for (int c = 0; c < nk; c++) {
        const int buf = c & 1;
        const uint32_t t_hh = tmem + buf * 128, t_x = tmem + 256 + buf * 128;
        if (tid == 0) {
            fence_after_sync();
            const __half *ah = Ah + buf * BM * BK, *al = Al + buf * BM * BK, *wh = Wh + buf * BN * BK, *wl = Wl + buf * BN * BK;
#pragma unroll
            for (int s = 0; s < BK / 16; s++)
                mma_f16(t_hh, kstep_desc(ah, BM, s), kstep_desc(wh, BN, s), id, s > 0 ? 1u : 0u);
#pragma unroll
            for (int s = 0; s < BK / 16; s++) {
                mma_f16(t_x, kstep_desc(ah, BM, s), kstep_desc(wl, BN, s), id, s > 0 ? 1u : 0u);
                mma_f16(t_x, kstep_desc(al, BM, s), kstep_desc(wh, BN, s), id, 1);
            }
            mma_commit(&mbar[buf]);
        }
        // the next chunk is staged while this one multiplies (its buffer's last readers finished last round)
        if (c + 1 < nk) {
            stage(c + 1, (c + 1) & 1);
            fence_async_smem();
        }
        ok = mbar_wait(&mbar[buf], parity[buf], GEMM_WAIT_CYCLES);
        parity[buf] ^= 1;
        if (!ok) *abort_flag = 1;
        fence_after_sync();
        if (ok) {
#pragma unroll
            for (int h2 = 0; h2 < 2; h2++) {
                float x[32], y[32];
                tmem_ld32(t_hh + lane_base + col0 + 32 * h2, x);
                tmem_ld32(t_x + lane_base + col0 + 32 * h2, y);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; e++) sum[32 * h2 + e] += x[e] + y[e];
            }
        }
        fence_before_sync();
        __syncthreads();
        if (*abort_flag) break;
    }
    ok = !*abort_flag;
    // epilogue through shared memory (reusing the operand buffers) so that global stores are coalesced
    float *ostage = reinterpret_cast<float *>(smraw);  // [BM][BN + 1]
    {
        const int m = (warp & 3) * 32 + (tid & 31);
        const float un = m0 + m < a.M ? stats[m0 + m].w : 0.f;
#pragma unroll
        for (int e = 0; e < 64; e++) ostage[m * (BN + 1) + col0 + e] = sum[e] * un;
    }
    __syncthreads();
    if (ok) {
        for (int i = tid; i < BM * BN; i += 256) {
            int m, e;
            if (a.transpose_out) {
                m = i % BM, e = i / BM;  // consecutive threads: consecutive rows -> consecutive addresses
            } else {
                e = i % BN, m = i / BN;
            }
            const int gm = m0 + m, gn = n0 + e;
            if (gm >= a.M || gn >= a.N) continue;
            float v = ostage[m * (BN + 1) + e] * a.tc_wunscale[gn] + (a.bias ? a.bias[gn] : 0.f);
            if (a.act) v = gelu1(v);
            float *dst = a.transpose_out ? a.y + (size_t)gn * a.ldy + gm : a.y + (size_t)gm * a.ldy + gn;
            *dst = a.accumulate ? *dst + v : v;
        }
    }
    if (!ok && tid == 0 && a.err) atomicExch(a.err, 1);
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

bool gemm_tc_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_TENSOR_CORES");
        return !(e && e[0] == '0');
    }();
    return on;
}

size_t gemm_tc_smem() { return sizeof(__half) * (4 * 128 * 64 + 4 * 128 * 64) + 64; }

cudaError_t launch_gemm_tc(const LinArgs &a, float4 *stats, cudaStream_t s, uint64_t *launches) {
    k_row_stats_tc<<<(a.M + 7) / 8, 256, 0, s>>>(a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats);
    if (launches) ++*launches;
    const size_t smem = gemm_tc_smem();
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    dim3 grid((a.N + 127) / 128, (a.M + 127) / 128);
    k_gemm_tc<<<grid, 256, smem, s>>>(a, stats);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
