// Linear layers of many rows on the tensor cores (tcgen05) at f32 accuracy: y (=|+=) act(W LN?(x) + b).
//
// Both operands reach the kernel already split into f16 hi + lo (x = hi + lo, about 22 significant bits) and laid
// out in blocks of 128 rows x 64 of K exactly as the MMAs read them from shared memory (tc_block_off: groups of 8
// rows outermost, so any 64-row half of a block is contiguous):
//   weights - once, at upload, with a power-of-two scaling per output row (the engine's weight upload);
//   activations - per call by k_split_rows, which also applies the LayerNorm (kern.rs:357-376) and a power-of-two
//   scaling per row.
// A CTA computes a 128-row x BN-output tile (BN 128, or 64 when 128-wide tiles would leave most SMs idle).
// Warp-specialised: one thread bulk-copies each 64-wide chunk of K (the activation and weight blocks) into a ring;
// one thread issues the chunk's MMAs (hi*hi, hi*lo, lo*hi) into a fresh accumulator (one of four in TMEM: the tensor
// cores' f32 accumulation is not round-to-nearest, so no accumulator sees more than 12 steps); eight warps add each
// chunk's accumulator into registers with ordinary f32 arithmetic while later chunks multiply. The epilogue undoes
// the scalings, adds the bias, applies GELU and the residual, and writes through shared memory so that stores are
// coalesced (also when transposed).
#include <cfloat>
#include <cstdlib>

#include "device.cuh"
#include "kernels.cuh"
#include "pdl.cuh"
#include "tc.cuh"

namespace tcu {

using namespace tc;

constexpr long long GEMM_WAIT_CYCLES = 2000000000ll;
constexpr int GBM = 128, GBK = 64, GTHREADS = 320, GBUFS = 4;
constexpr size_t GBLOCK = (size_t)GBM * GBK;  // halves in one operand block (hi or lo)
// STAGES: slots of the copy ring (0: the default for the tile width)
template <int BN, int SLOTS = 0>
struct GemmShape {
    static constexpr int STAGES = SLOTS ? SLOTS : (BN == 128 ? 3 : 4);
    static constexpr uint32_t A_BYTES = 2 * GBLOCK * sizeof(__half);            // hi + lo of 128 rows
    static constexpr uint32_t W_BYTES = 2 * (uint32_t)BN * GBK * sizeof(__half);  // hi + lo of BN rows
    static constexpr uint32_t SLOT = A_BYTES + W_BYTES;
    static constexpr size_t SMEM = (size_t)STAGES * SLOT + 1024;  // + barriers, TMEM slot, flag, row unscales
};


__device__ __forceinline__ float p2(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

size_t tc_split_bytes(int rows, int K) { return (size_t)((rows + GBM - 1) / GBM) * (size_t)(K / GBK) * 2 * GBLOCK * 2; }

// Eight rows per block, one warp per row. Each lane holds 8 consecutive values of its row per 256 of K, read once:
// the LayerNorm's mean and 1/sigma (when lnw is set; kern.rs:357-376, two passes over the held values), the
// power-of-two scale that keeps the row's largest transformed magnitude below 2^14 (stats[m] = {mean, rstd, scale,
// 1 / scale}), and the row, transformed and scaled, split into f16 hi + lo in its 128 x 64 blocks:
// tiles[(m / 128) * (K / 64) + k / 64] = [hi block][lo block], element (m % 128, k % 64) at blk_off. Rows from M up
// to the next multiple of 128 are written as zeros. NJ = K / 256 rounded up (K up to 2048). With RPW = 2 (K up to 128)
// each half-warp takes a row of its own: the lanes a whole warp would leave idle (they hold zeros there), so every sum
// and maximum is the same, added in the same order.
template <int LW>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = LW / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
template <int LW>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
    for (int o = LW / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int NJ, int RPW = 1>
__global__ void __launch_bounds__(256) k_split_rows(const float *x, int ldx, int M, int K, const float *lnw,
                                                    const float *lnb, float4 *stats, __half *tiles) {
    constexpr int LW = 32 / RPW;  // lanes per row
    const int warp = threadIdx.x >> 5, lane = (threadIdx.x & 31) % LW;
    const int row = (blockIdx.x * 8 + warp) * RPW + (int)(threadIdx.x & 31) / LW;
    const bool real = row < M;
    pdl_trigger();
    pdl_wait();
    const float *p = x + (size_t)(real ? row : 0) * ldx;
    float v[NJ][8];
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int k = 256 * j + 8 * lane;
        if (real && k < K) {
            const float4 x0 = *reinterpret_cast<const float4 *>(p + k), x1 = *reinterpret_cast<const float4 *>(p + k + 4);
            v[j][0] = x0.x, v[j][1] = x0.y, v[j][2] = x0.z, v[j][3] = x0.w;
            v[j][4] = x1.x, v[j][5] = x1.y, v[j][6] = x1.z, v[j][7] = x1.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[j][e] = 0.f;
        }
    }
    float mean = 0.f, inv = 1.f;
    if (lnw) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; j++)
#pragma unroll
            for (int e = 0; e < 8; e++) s += v[j][e];
        mean = group_sum<LW>(s) / (float)K;
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (256 * j + 8 * lane < K) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float dd = v[j][e] - mean;
                    q = fmaf(dd, dd, q);
                }
            }
        }
        inv = 1.0f / sqrtf(group_sum<LW>(q) / (float)K + 1e-5f);
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int k = 256 * j + 8 * lane;
            if (k < K) {
                const float4 w0 = *reinterpret_cast<const float4 *>(lnw + k), w1 = *reinterpret_cast<const float4 *>(lnw + k + 4);
                const float4 b0 = *reinterpret_cast<const float4 *>(lnb + k), b1 = *reinterpret_cast<const float4 *>(lnb + k + 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int e = 0; e < 8; e++) v[j][e] = real ? (v[j][e] - mean) * inv * w[e] + bb[e] : 0.f;
            }
        }
    }
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++)
#pragma unroll
        for (int e = 0; e < 8; e++) mx = fmaxf(mx, fabsf(v[j][e]));
    mx = group_max<LW>(mx);
    int ex = 0;
    if (mx > 0.f) {
        ex = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xff) - 126);  // mx < 2^(14 - ex)
        ex = ex < -120 ? -120 : (ex > 120 ? 120 : ex);
    }
    const float sc = p2(ex);
    if (lane == 0 && real) stats[row] = make_float4(mean, inv, sc, p2(-ex));
    const int nk = K / GBK, mt = row / GBM;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int k = 256 * j + 8 * lane;
        if (k < K) {
            __align__(16) __half hh[8], ll[8];
#pragma unroll
            for (int e = 0; e < 8; e++) split_f16(v[j][e] * sc, hh[e], ll[e]);
            __half *blk = tiles + ((size_t)mt * nk + k / GBK) * 2 * GBLOCK;
            const int off = blk_off(row % GBM, k % GBK);
            *reinterpret_cast<uint4 *>(blk + off) = *reinterpret_cast<const uint4 *>(hh);
            *reinterpret_cast<uint4 *>(blk + GBLOCK + off) = *reinterpret_cast<const uint4 *>(ll);
        }
    }
}

__device__ __forceinline__ void g_bulk(void *dst, const void *src, uint32_t bytes, uint64_t *mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(mbar))
                 : "memory");
}
__device__ __forceinline__ void g_expect(uint64_t *mbar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(
                     smem_addr(mbar)),
                 "r"(bytes)
                 : "memory");
}

template <int BN, int SLOTS = 0>
__global__ void __launch_bounds__(GTHREADS, 1) k_gemm_tc(LinArgs a, const float4 *stats) {
    using G = GemmShape<BN, SLOTS>;
    constexpr int S = G::STAGES, HALF = BN / 2;
    extern __shared__ __align__(1024) uint8_t smraw[];
    // ring of S slots: [A hi][A lo][W hi][W lo]
    uint64_t *mb = reinterpret_cast<uint64_t *>(smraw + (size_t)S * G::SLOT);
    uint64_t *mFull = mb, *mEmpty = mb + S, *mT = mb + 2 * S, *mTfree = mT + GBUFS, *mDone = mTfree + GBUFS;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mDone + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    float *un_row = reinterpret_cast<float *>(tslot + 2);  // [GBM]: the rows' unscale (epilogue)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nt = blockIdx.x, mt = blockIdx.y, m0 = mt * GBM, n0 = nt * BN;
    const int nk = a.K / GBK;
    if (warp == 0) {
        tmem_alloc(tslot, GBUFS * BN);  // four chunk accumulators of BN columns
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < S; i++) mbar_init(&mFull[i], 1), mbar_init(&mEmpty[i], 1);
        for (int i = 0; i < GBUFS; i++) mbar_init(&mT[i], 1), mbar_init(&mTfree[i], 256);
        mbar_init(mDone, 1);
        mbar_init_fence();
        *abort_flag = 0;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    pdl_trigger();  // every block holds its tensor memory
    const uint32_t tmem = *tslot;
    const uint8_t *A = reinterpret_cast<const uint8_t *>(a.tc_atiles) + (size_t)mt * nk * G::A_BYTES;
    // weights are stored in 128-row blocks; a 64-wide tile is the first or second half of each hi and lo block
    const uint8_t *Wt = reinterpret_cast<const uint8_t *>(a.tc_wtiles) + (size_t)(n0 / GBM) * nk * 2 * GBLOCK * 2 +
                        (size_t)(n0 % GBM) * GBK * 2;
    auto wait = [&](uint64_t *m, uint32_t parity) {
        if (*abort_flag) return false;
        if (!mbar_wait(m, parity, GEMM_WAIT_CYCLES)) {
            *abort_flag = 1;
            return false;
        }
        return true;
    };
    float sum[HALF];
#pragma unroll
    for (int e = 0; e < HALF; e++) sum[e] = 0.f;
    const int col0 = ((warp >> 2) & 1) * HALF;
    if (warp == 9) {
        // the load thread: chunk c into slot c % S once the MMAs of chunk c - S have read it. The weights of the first
        // S chunks are asked for before the kernel before has finished (no kernel writes them); the rows after.
        if (lane == 0) {
            auto load_w = [&](int c) {
                const int s = c % S;
                uint8_t *dst = smraw + (size_t)s * G::SLOT;
                const uint8_t *wsrc = Wt + (size_t)c * 2 * GBLOCK * 2;
                g_expect(&mFull[s], G::SLOT);
                if (BN == GBM) {
                    g_bulk(dst + G::A_BYTES, wsrc, G::W_BYTES, &mFull[s]);
                } else {
                    g_bulk(dst + G::A_BYTES, wsrc, G::W_BYTES / 2, &mFull[s]);
                    g_bulk(dst + G::A_BYTES + G::W_BYTES / 2, wsrc + GBLOCK * 2, G::W_BYTES / 2, &mFull[s]);
                }
            };
            const int pre = min(nk, S);
            for (int c = 0; c < pre; c++) load_w(c);
            pdl_wait();
            for (int c = 0; c < pre; c++)
                g_bulk(smraw + (size_t)(c % S) * G::SLOT, A + (size_t)c * G::A_BYTES, G::A_BYTES, &mFull[c % S]);
            int issued = pre;
            for (int c = pre; c < nk; c++) {
                const int s = c % S;
                if (!wait(&mEmpty[s], (uint32_t)((c / S) - 1) & 1u)) break;
                load_w(c);
                g_bulk(smraw + (size_t)s * G::SLOT, A + (size_t)c * G::A_BYTES, G::A_BYTES, &mFull[s]);
                issued = c + 1;
            }
            // the last loads land before the block lets go of shared memory
            for (int c = max(0, issued - S); c < issued; c++)
                mbar_wait(&mFull[c % S], (uint32_t)(c / S) & 1u, GEMM_WAIT_CYCLES);
        }
    } else if (warp == 8) {
        // the MMA thread (its bounded waits start once the kernel before has finished)
        pdl_wait();
        if (lane == 0) {
            const uint32_t id = idesc_f16(GBM, BN, 0, 0);
            // K-major, no swizzle: core matrices 128 B apart along K (LBO), 8-row groups 1024 B apart (SBO)
            const uint64_t d0 = smem_desc(smem_addr(smraw), 128, 1024);
            const uint64_t st = 256 >> 4;  // one K-step of 16: two core matrices along K
            for (int c = 0; c < nk; c++) {
                const int s = c % S, b = c % GBUFS;
                if (!wait(&mFull[s], (uint32_t)(c / S) & 1u)) break;
                if (c >= GBUFS && !wait(&mTfree[b], (uint32_t)((c / GBUFS) - 1) & 1u)) break;
                fence_after_sync();
                const uint64_t dAh = d0 + ((s * G::SLOT) >> 4), dAl = dAh + ((GBLOCK * 2) >> 4);
                const uint64_t dWh = dAh + (G::A_BYTES >> 4), dWl = dWh + ((G::W_BYTES / 2) >> 4);
                const uint32_t t = tmem + b * BN;
#pragma unroll
                for (int k = 0; k < GBK / 16; k++) {
                    mma_f16(t, dAh + k * st, dWh + k * st, id, k > 0 ? 1u : 0u);
                    mma_f16(t, dAh + k * st, dWl + k * st, id, 1);
                    mma_f16(t, dAl + k * st, dWh + k * st, id, 1);
                }
                mma_commit(&mEmpty[s]);
                mma_commit(&mT[b]);
            }
            mma_commit(mDone);
            mbar_wait(mDone, 0, GEMM_WAIT_CYCLES);
        }
    } else {
        // eight warps: lane (row) (warp % 4) * 32 + lane, columns col0 + [0, BN / 2) of every chunk's accumulator
        pdl_wait();
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        for (int c = 0; c < nk; c++) {
            const int b = c % GBUFS;
            bool okc = !*abort_flag && mbar_wait(&mT[b], (uint32_t)(c / GBUFS) & 1u, GEMM_WAIT_CYCLES);
            okc = __all_sync(0xffffffffu, okc);  // tcgen05.ld is warp-wide
            if (!okc) *abort_flag = 1;
            fence_after_sync();
            if (okc) {
#pragma unroll
                for (int h2 = 0; h2 < HALF / 32; h2++) {
                    float x[32];
                    tmem_ld32(tmem + b * BN + lane_base + col0 + 32 * h2, x);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++) sum[32 * h2 + e] += x[e];
                }
            }
            fence_before_sync();
            mbar_arrive(&mTfree[b]);
            if (!okc) break;
        }
    }
    pdl_wait();  // the rows' scalings and the residual come from earlier kernels
    if (tid < GBM) un_row[tid] = m0 + tid < a.M ? stats[m0 + tid].w : 0.f;
    fence_before_sync();
    __syncthreads();
    const bool ok = !*abort_flag;
    // epilogue through shared memory (the ring: every load has landed and every MMA finished)
    float *ostage = reinterpret_cast<float *>(smraw);  // [GBM][BN + 1]
    if (warp < 8) {
        const int m = (warp & 3) * 32 + lane;
        const float un = un_row[m];
#pragma unroll
        for (int e = 0; e < HALF; e++) ostage[m * (BN + 1) + col0 + e] = sum[e] * un;
    }
    __syncthreads();
    if (ok && warp < 8) {
        if (a.transpose_out) {
            // thread: row m (consecutive threads, consecutive addresses), columns e0, e0 + 2, ...
            const int m = tid & (GBM - 1), gm = m0 + m;
            if (gm < a.M) {
                // eight columns at a time: the residual values are all loaded before any result is stored
                for (int e0 = tid >> 7; e0 < BN; e0 += 16) {
                    float old[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int gn = n0 + e0 + 2 * j;
                        old[j] = a.accumulate && e0 + 2 * j < BN && gn < a.N ? a.y[(size_t)gn * a.ldy + gm] : 0.f;
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int e = e0 + 2 * j, gn = n0 + e;
                        if (e >= BN || gn >= a.N) break;
                        float v = ostage[m * (BN + 1) + e] * a.tc_wunscale[gn] + (a.bias ? a.bias[gn] : 0.f);
                        if (a.act) v = gelu1(v);
                        a.y[(size_t)gn * a.ldy + gm] = a.accumulate ? old[j] + v : v;
                    }
                }
            }
        } else {
            // thread: column e (consecutive threads, consecutive addresses), rows r0, r0 + 256 / BN, ...
            constexpr int RSTEP = 256 / BN;
            const int e = tid % BN, gn = n0 + e;
            if (gn < a.N) {
                const float ws = a.tc_wunscale[gn], bs = a.bias ? a.bias[gn] : 0.f;
                const int mend = min(GBM, a.M - m0);
                // eight rows at a time: the residual values are all loaded before any result is stored
                for (int mb = tid / BN; mb < mend; mb += 8 * RSTEP) {
                    float old[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int m = mb + j * RSTEP;
                        old[j] = a.accumulate && m < mend ? a.y[(size_t)(m0 + m) * a.ldy + gn] : 0.f;
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int m = mb + j * RSTEP;
                        if (m >= mend) break;
                        float v = ostage[m * (BN + 1) + e] * ws + bs;
                        if (a.act) v = gelu1(v);
                        a.y[(size_t)(m0 + m) * a.ldy + gn] = a.accumulate ? old[j] + v : v;
                    }
                }
            }
        }
    }
    if (!ok && tid == 0 && a.err) *reinterpret_cast<volatile int *>(a.err) = 1;  // a report slot in host memory
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, GBUFS * BN);
}

bool gemm_tc_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_TENSOR_CORES");
        return !(e && e[0] == '0');
    }();
    return on;
}

size_t gemm_tc_smem() { return GemmShape<128>::SMEM; }

// 64-wide tiles when 128-wide ones would fill at most half of the SMs
static int gemm_bn(int M, int N) {
    static const int forced = [] {
        const char *e = getenv("TCU_GEMM_BN");
        return e ? atoi(e) : 0;
    }();
    if (forced == 64 || forced == 128) return forced;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return (long)((M + GBM - 1) / GBM) * ((N + 127) / 128) * 2 <= sms ? 64 : 128;
}

template <int BN, int SLOTS = 0>
static cudaError_t launch_bn(const LinArgs &a, float4 *stats, cudaStream_t s) {
    using G = GemmShape<BN, SLOTS>;
    cudaError_t e = allow_dynamic_smem((const void *)k_gemm_tc<BN, SLOTS>, G::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((a.N + BN - 1) / BN, (a.M + GBM - 1) / GBM);
    return launch_pdl(k_gemm_tc<BN, SLOTS>, grid, dim3(GTHREADS), G::SMEM, s, a, (const float4 *)stats);
}

cudaError_t launch_gemm_tc(const LinArgs &a, float4 *stats, cudaStream_t s, uint64_t *launches) {
    if (!a.tc_wtiles || !a.tc_atiles || a.K % GBK || a.K > 2048) return cudaErrorInvalidValue;
    const int sblocks = (a.M + GBM - 1) / GBM * (GBM / 8);
    __half *at = reinterpret_cast<__half *>(a.tc_atiles);
    cudaError_t e0;
    if (a.K <= 128)
        e0 = launch_pdl(k_split_rows<1, 2>, dim3(sblocks / 2), dim3(256), 0, s, a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats, at);
    else if (a.K <= 256)
        e0 = launch_pdl(k_split_rows<1>, dim3(sblocks), dim3(256), 0, s, a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats, at);
    else if (a.K <= 512)
        e0 = launch_pdl(k_split_rows<2>, dim3(sblocks), dim3(256), 0, s, a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats, at);
    else if (a.K <= 1024)
        e0 = launch_pdl(k_split_rows<4>, dim3(sblocks), dim3(256), 0, s, a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats, at);
    else
        e0 = launch_pdl(k_split_rows<8>, dim3(sblocks), dim3(256), 0, s, a.x, a.ldx, a.M, a.K, a.lnw, a.lnb, stats, at);
    if (e0 != cudaSuccess) return e0;
    if (launches) ++*launches;
    // many tiles of at most four K chunks (the column and row stages): 64-wide tiles with a two-slot ring, so that two
    // CTAs share an SM and one's set-up and epilogue overlap the other's copies and MMAs (TCU_GEMM_PAIR=0: never)
    static const bool pair = [] {
        const char *v = getenv("TCU_GEMM_PAIR");
        return !(v && v[0] == '0');
    }();
    if (pair && a.K <= 256 && (long)((a.M + GBM - 1) / GBM) * ((a.N + 63) / 64) >= 4L * 148) {
        const cudaError_t e = launch_bn<64, 2>(a, stats, s);
        if (launches) ++*launches;
        return e;
    }
    const cudaError_t e = gemm_bn(a.M, a.N) == 64 ? launch_bn<64>(a, stats, s) : launch_bn<128>(a, stats, s);
    if (launches) ++*launches;
    return e;
}

}  // namespace tcu
