// Attention of many query rows on the 5th-generation tensor cores (tcgen05), at f32 accuracy.
//
// Every f32 operand is split into two f16 values (x = hi + lo, about 22 significant bits) after a power-of-two
// scaling that keeps it inside the f16 range, and each product is taken as hi*hi + hi*lo + lo*hi with f32
// accumulators in tensor memory. The stored keys and values are widened and split once per model into 64-key tiles
// in exactly the layout the MMAs read (k_tc_tiles); the attention kernel moves them with bulk copies.
#include <cfloat>
#include <cmath>

#include "device.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace tcu {

using namespace tc;

constexpr long long TC_WAIT_CYCLES = 2000000000ll;  // about a second at boost clock

__device__ __forceinline__ float pow2f(int e) {  // 2^e for |e| < 127, exact
    return __uint_as_float((uint32_t)(e + 127) << 23);
}
// e such that |x| * 2^e < 2^14 for the largest |x| = mx (0 when mx is 0)
__device__ __forceinline__ int f16_exponent(float mx) {
    if (!(mx > 0.f)) return 0;
    int ex = (int)((__float_as_uint(mx) >> 23) & 0xff) - 126;  // mx < 2^ex
    int e = 14 - ex;
    return e < -120 ? -120 : (e > 120 ? 120 : e);
}

// Write one 16-byte group (8 values) of hi and lo halves.
__device__ __forceinline__ void put8(__half *hi, __half *lo, int off, const float (&v)[8], float scale) {
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; e++) split_f16(v[e] * scale, h[e], l[e]);
    *reinterpret_cast<uint4 *>(hi + off) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(lo + off) = *reinterpret_cast<const uint4 *>(l);
}

// e^x on the special-function unit: 2^(x log2 e), relative error about 1e-6 for the softmax's arguments (x <= 0,
// |x| < 30 where the weight matters). The tensor-core path's softmax uses it to keep the FMA pipe free; its results
// stay within the stage bar of the reference's exp (kern.rs:220-235).
__device__ __forceinline__ float exp_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.44269504088896340736f));
    return y;
}

// Eight values as f16 hi + lo (x = hi + lo), two at a time.
__device__ __forceinline__ void put8x2(__half *hi, __half *lo, int off, const float (&v)[8]) {
    __align__(16) __half2 h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
        const float2 b = __half22float2(h[e]);
        l[e] = __floats2half2_rn(v[2 * e] - b.x, v[2 * e + 1] - b.y);
    }
    *reinterpret_cast<uint4 *>(hi + off) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(lo + off) = *reinterpret_cast<const uint4 *>(l);
}

constexpr int TC_HD = 128, TC_BQ = 128, TC_BK = FLASH_KEYS;
constexpr size_t TC_BLOCK = (size_t)TC_BK * TC_HD;  // halves of one operand block (keys hi, keys lo, values hi, lo)

size_t tc_tile_bytes() { return 4 * TC_BLOCK * sizeof(__half); }

// One tile (64 keys x one head) of a stored layer in the tensor cores' operand form, written once per model:
// [keys hi][keys lo][values hi][values lo], each 64 x 128 f16 in the core-matrix layout the MMAs read from shared
// memory, both K-major (a key's coordinates together for S = Q K^T; a coordinate's keys together for P V). Integers are widened exactly and multiplied by their chunk's scale
// (predict.rs:486-497 for keys; nn.rs:253-256 for values, the same product taken per element), then by the layer's
// power of two and split into hi + lo. Keys past a ragged tile's end are zero.
template <int KV>
__global__ void __launch_bounds__(256) k_tc_tiles(AttnArgs a, __half *out) {
    constexpr int HD = TC_HD, BK = TC_BK, W = KvFmt<KV>::W, EPV = KvFmt<KV>::EPV, VPR = BK / EPV;
    const int t = blockIdx.x, h = blockIdx.y, H = gridDim.y, tid = threadIdx.x, d = a.d;
    __half *Khi = out + ((size_t)t * H + h) * 4 * TC_BLOCK, *Klo = Khi + TC_BLOCK, *Vhi = Klo + TC_BLOCK,
           *Vlo = Vhi + TC_BLOCK;
    const int4 tile = a.tiles[t];
    const int ci = tile.x, k0 = tile.y, len = tile.z;
    const int rc = min(a.chunk, a.rows - ci * a.chunk);
    const uint8_t *rec = a.layer + (size_t)ci * a.full;
    const float *sc = reinterpret_cast<const float *>(rec);
    const uint8_t *body = rec + (KV ? 8 * (size_t)d : 0);
    const uint8_t *kb = body + ((size_t)h * HD * rc + k0) * W;
    const uint8_t *vb = body + ((size_t)(d + h * HD) * rc + k0) * W;
    const size_t rowb = (size_t)rc * W;
    const float kscale = pow2f(a.tc_eK), vscale = pow2f(a.tc_eV);
    const bool fast = len == BK && ((((uintptr_t)kb) | ((uintptr_t)vb) | rowb) & 15) == 0;
    if (fast) {
        for (int i = tid; i < HD * VPR / 2; i += 256) {
            const int j = i % HD, vp = i / HD;
            const float ks = (KV ? sc[h * HD + j] : 1.f) * kscale;
            const float vs = (KV ? sc[d + h * HD + j] : 1.f) * vscale;
            const uint4 rk0 = *reinterpret_cast<const uint4 *>(kb + j * rowb + vp * 32);
            const uint4 rk1 = *reinterpret_cast<const uint4 *>(kb + j * rowb + vp * 32 + 16);
            const uint4 rv0 = *reinterpret_cast<const uint4 *>(vb + j * rowb + vp * 32);
            const uint4 rv1 = *reinterpret_cast<const uint4 *>(vb + j * rowb + vp * 32 + 16);
#pragma unroll
            for (int g = 0; g < 2 * EPV; g += 8) {
                float fk[8], fv[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int x = g + e;
                    fk[e] = (x < EPV ? unpack<KV>(rk0, x) : unpack<KV>(rk1, x - EPV)) * ks;
                    fv[e] = (x < EPV ? unpack<KV>(rv0, x) : unpack<KV>(rv1, x - EPV)) * vs;
                }
                const int key = vp * 2 * EPV + g;
#pragma unroll
                for (int e = 0; e < 8; e++)
                    split_f16(fk[e], Khi[kmajor_off(key + e, j, BK)], Klo[kmajor_off(key + e, j, BK)]);
                put8(Vhi, Vlo, kmajor_off(j, key, HD), fv, 1.f);
            }
        }
    } else {
        for (int i = tid; i < HD * BK; i += 256) {
            const int j = i / BK, key = i % BK;
            float fk = 0.f, fv = 0.f;
            if (key < len) {
                fk = load_elem<KV>(body, (size_t)(h * HD + j) * rc + k0 + key) * (KV ? sc[h * HD + j] : 1.f);
                fv = load_elem<KV>(body, (size_t)(d + h * HD + j) * rc + k0 + key) * (KV ? sc[d + h * HD + j] : 1.f);
            }
            split_f16(fk * kscale, Khi[kmajor_off(key, j, BK)], Klo[kmajor_off(key, j, BK)]);
            split_f16(fv * vscale, Vhi[kmajor_off(j, key, HD)], Vlo[kmajor_off(j, key, HD)]);
        }
    }
}

// 16-byte aligned contiguous bytes into shared memory, completing on the mbarrier (async proxy).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(mbar))
                 : "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t *mbar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(
                     smem_addr(mbar)),
                 "r"(bytes)
                 : "memory");
}

// Attention of 128 query rows x one head over a range of 64-key tiles, with the tiles pre-split (k_tc_tiles):
//   S = Q K^T: Q [128 x 128] K-major, K [64 keys x 128] MN-major; two S buffers in TMEM (columns 0-127, 128-255),
//              hi*hi in the first 64 columns of a buffer, cross terms in the next 64
//   O += P V^T: P [128 x 64 keys] K-major, V [128 x 64 keys] K-major; per tile hi*hi in 256-383, cross 384-511
// Warp-specialised: warps 0-7 compute (the online softmax, nn.rs:207-215 rule, two threads per query row; the fold
// of each tile's P V into O held in registers), one thread of warp 8 issues every MMA, one thread of warp 9 the bulk
// copies of the key and value halves of each tile into two-slot rings. They hand over through mbarriers only (the
// two producers in separate warps, so neither's waiting holds the other up), and the tensor cores work on tile
// i + 1's scores while the softmax of tile i runs. Every f32 sum of tensor-core results is taken
// in registers (fresh accumulators per tile: the units' own f32 accumulation is not round-to-nearest). Every wait
// is bounded; a wait that gives up raises the block's abort flag and everyone leaves.
constexpr int TC_THREADS = 320;  // eight compute warps, an MMA warp and a load warp

// Named barrier 1 over the 256 compute threads, returning the AND of p over them (every compute thread takes the
// same branch after it).
__device__ __forceinline__ bool compute_all(bool p) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}\n"
                 : "=r"(r)
                 : "r"((uint32_t)p)
                 : "memory");
    return r != 0;
}

template <int KV>
__global__ void __launch_bounds__(TC_THREADS, 1) k_attend_tc(AttnArgs a) {
    constexpr int HD = TC_HD, BQ = TC_BQ, BK = TC_BK;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Qhi = reinterpret_cast<__half *>(smraw);  // [BQ][HD] K-major
    __half *Qlo = Qhi + BQ * HD;
    __half *Kring = Qlo + BQ * HD;                    // two slots of [keys hi][keys lo]
    __half *Vring = Kring + 2 * 2 * TC_BLOCK;         // two slots of [values hi][values lo]
    __half *Phi = Vring + 2 * 2 * TC_BLOCK;           // [BQ][BK keys] K-major
    __half *Plo = Phi + BQ * BK;
    float *fr = reinterpret_cast<float *>(Plo + BQ * BK);  // [BQ] this tile's rescale factor of each row
    float *redm = fr + BQ;                                 // [2][BQ] half-row maxima
    float *reds = redm + 2 * BQ;                           // [2][BQ] half-row weight sums
    uint64_t *mb = reinterpret_cast<uint64_t *>(reds + 2 * BQ);
    uint64_t *mS = mb, *mSfree = mb + 2, *mK = mb + 4, *mV = mb + 6, *mP = mb + 8, *mPV = mb + 9, *mO = mb + 10,
             *mDone = mb + 11;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mb + 12);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    float *qscale = reinterpret_cast<float *>(Phi);  // [BQ] 2^e of each row's query (until the first P)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, split = blockIdx.z, r0 = blockIdx.x * BQ, d = a.d, H = gridDim.y;
    const int t0 = split * a.tiles_per_split, t1 = min(a.ntiles, t0 + a.tiles_per_split), nt = t1 - t0;
    const __half *tiles = reinterpret_cast<const __half *>(a.tc_tiles);
    const bool producer = warp >= 8;
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&mS[i], 1);
            mbar_init(&mSfree[i], 256);
            mbar_init(&mK[i], 1);
            mbar_init(&mV[i], 1);
        }
        mbar_init(mP, 256);
        mbar_init(mPV, 1);
        mbar_init(mO, 256);
        mbar_init(mDone, 1);
        mbar_init_fence();
        *abort_flag = 0;
    }
    // each row's query scale: its largest |q| maps below 2^14
    if (tid < BQ) {
        float mx = 0.f;
        const int r = r0 + tid;
        if (r < a.R) {
            const float4 *qp = reinterpret_cast<const float4 *>(a.q + (size_t)r * a.ldq + h * HD);
#pragma unroll 4
            for (int j = 0; j < HD / 4; j++) {
                float4 v = qp[j];
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        }
        qscale[tid] = pow2f(f16_exponent(mx));
    }
    __syncthreads();
    const uint32_t half_bytes = (uint32_t)(2 * TC_BLOCK * sizeof(__half));
    auto load = [&](int i, bool values) {  // producer thread: the key or value halves of tile t0 + i into slot i & 1
        const __half *src = tiles + ((size_t)(t0 + i) * H + h) * 4 * TC_BLOCK + (values ? 2 * TC_BLOCK : 0);
        __half *dst = (values ? Vring : Kring) + (size_t)(i & 1) * 2 * TC_BLOCK;
        uint64_t *m = values ? &mV[i & 1] : &mK[i & 1];
        expect_tx(m, half_bytes);
        bulk_g2s(dst, src, half_bytes / 2, m);
        bulk_g2s(dst + TC_BLOCK, src + TC_BLOCK, half_bytes / 2, m);
    };
    if (warp == 9 && lane == 0) {
        for (int i = 0; i < min(nt, 2); i++) load(i, false), load(i, true);
    }
    for (int i = tid; i < BQ * (HD / 8); i += TC_THREADS) {
        const int m = i % BQ, j0 = (i / BQ) * 8, r = r0 + m;
        float v[8];
        if (r < a.R) {
            const float4 *qp = reinterpret_cast<const float4 *>(a.q + (size_t)r * a.ldq + h * HD + j0);
            float4 x = qp[0], y = qp[1];
            v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w, v[4] = y.x, v[5] = y.y, v[6] = y.z, v[7] = y.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.f;
        }
        put8(Qhi, Qlo, kmajor_off(m, j0, BQ), v, qscale[m]);
    }
    const int row = (warp & 3) * 32 + lane, half = (warp >> 2) & 1;
    const float rs = producer ? 1.f : (1.0f / qscale[row]) * pow2f(-a.tc_eK);  // undoes both scalings
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot, tO = tmem + 256;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    float o[64];
#pragma unroll
    for (int e = 0; e < 64; e++) o[e] = 0.f;
    float mrun = -FLT_MAX, lrun = 0.f;
    bool any = false;

    if (producer) {
        auto wait = [&](uint64_t *m, uint32_t parity) {
            if (*abort_flag) return false;
            if (!mbar_wait(m, parity, TC_WAIT_CYCLES)) {
                *abort_flag = 1;
                return false;
            }
            return true;
        };
        if (warp == 8 && lane == 0) {
            // the MMA thread: waits only for what its next MMAs read
            const uint32_t idS = idesc_f16(BQ, BK, 0, 0), idO = idesc_f16(BQ, HD, 0, 0);
            // Descriptors: K-step k of an operand is its k = 0 descriptor plus k times the step of its start address
            // (the address sits in the low bits, in 16-byte units), so each MMA costs one add, not a recomputation.
            const uint64_t dQh = kstep_desc(Qhi, BQ, 0), dQl = kstep_desc(Qlo, BQ, 0);
            const uint64_t dK0 = kstep_desc(Kring, BK, 0), dV0 = kstep_desc(Vring, HD, 0);
            const uint64_t dPh = kstep_desc(Phi, BQ, 0), dPl = kstep_desc(Plo, BQ, 0);
            const uint64_t stQ = (2 * (BQ / 8) * 128) >> 4, stK = (2 * (BK / 8) * 128) >> 4, stV = (2 * (HD / 8) * 128) >> 4;
            const uint64_t lo_off = (TC_BLOCK * sizeof(__half)) >> 4, slot_off = (2 * TC_BLOCK * sizeof(__half)) >> 4;
            auto issue_S = [&](int i) {
                const uint32_t tS = tmem + 128 * (i & 1);
                const uint64_t dKh = dK0 + (i & 1) * slot_off, dKl = dKh + lo_off;
                fence_after_sync();
#pragma unroll
                for (int k = 0; k < HD / 16; k++) {
                    mma_f16(tS, dQh + k * stQ, dKh + k * stK, idS, k > 0 ? 1u : 0u);
                    mma_f16(tS + 64, dQh + k * stQ, dKl + k * stK, idS, k > 0 ? 1u : 0u);
                    mma_f16(tS + 64, dQl + k * stQ, dKh + k * stK, idS, 1);
                }
                mma_commit(&mS[i & 1]);
            };
            bool ok = true;
            for (int i = 0; i < min(nt, 2) && ok; i++) {
                ok = wait(&mK[i & 1], 0);
                if (ok) issue_S(i);
            }
            for (int i = 0; i < nt && ok; i++) {
                const int b = i & 1;
                const uint32_t ph = (uint32_t)(i >> 1) & 1u;
                // P V of tile i: its P written, its values here, O's accumulators folded
                if (!(ok = wait(mP, (uint32_t)i & 1u))) break;
                if (!(ok = wait(&mV[b], ph))) break;
                if (i > 0 && !(ok = wait(mO, (uint32_t)(i - 1) & 1u))) break;
                fence_after_sync();
                {
                    const uint64_t dVh = dV0 + b * slot_off, dVl = dVh + lo_off;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) {
                        mma_f16(tO, dPh + k * stQ, dVh + k * stV, idO, k > 0 ? 1u : 0u);
                        mma_f16(tO + 128, dPh + k * stQ, dVl + k * stV, idO, k > 0 ? 1u : 0u);
                        mma_f16(tO + 128, dPl + k * stQ, dVh + k * stV, idO, 1);
                    }
                    mma_commit(mPV);
                }
                // S of tile i + 2 into the buffer the softmax of tile i has read, from its keys
                if (i + 2 < nt) {
                    if (!(ok = wait(&mSfree[b], ph))) break;
                    if (!(ok = wait(&mK[b], (uint32_t)((i + 2) >> 1) & 1u))) break;
                    issue_S(i + 2);
                }
            }
            // every MMA completes before the block lets go of tensor memory
            mma_commit(mDone);
            mbar_wait(mDone, 0, TC_WAIT_CYCLES);
        } else if (warp == 9 && lane == 0) {
            // the load thread: tile i + 2's keys where tile i's were once S(i) is done, its values once P V(i) is
            int ki = min(nt, 2), vi = min(nt, 2);  // key / value loads started
            for (int i = 0; i + 2 < nt; i++) {
                const int b = i & 1;
                if (!wait(&mS[b], (uint32_t)(i >> 1) & 1u)) break;
                load(i + 2, false);
                ki = i + 3;
                if (!wait(mPV, (uint32_t)i & 1u)) break;
                load(i + 2, true);
                vi = i + 3;
            }
            // the last load into each slot lands before the block lets go of shared memory
            for (int j = max(0, ki - 2); j < ki; j++) mbar_wait(&mK[j & 1], (uint32_t)(j >> 1) & 1u, TC_WAIT_CYCLES);
            for (int j = max(0, vi - 2); j < vi; j++) mbar_wait(&mV[j & 1], (uint32_t)(j >> 1) & 1u, TC_WAIT_CYCLES);
        }
    } else {
        bool alive = true;
        for (int i = 0; i < nt; i++) {
            const int b = i & 1;
            const uint32_t ph = (uint32_t)(i >> 1) & 1u;
            const int len = a.tiles[t0 + i].z;
            // (1) the online softmax of S(i), two threads per row; the compute warps leave together or not at all
            const bool okS = alive && !*abort_flag && mbar_wait(&mS[b], ph, TC_WAIT_CYCLES);
            if (!compute_all(okS)) {
                if (tid == 0) *abort_flag = 1;
                alive = false;
                break;
            }
            fence_after_sync();
            __syncwarp();
            float s[32];
            {
                float x[32], y[32];
                const uint32_t tS = tmem + 128 * b + lane_base + 32 * half;
                tmem_ld32(tS, x);
                tmem_ld32(tS + 64, y);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) s[k] = (x[k] + y[k]) * rs;
            }
            fence_before_sync();
            mbar_arrive(&mSfree[b]);
            float mx = -FLT_MAX;
#pragma unroll
            for (int k = 0; k < 32; k++)
                if (32 * half + k < len) mx = fmaxf(mx, s[k]);
            redm[half * BQ + row] = mx;
            asm volatile("bar.sync 1, 256;" ::: "memory");
            const float mnew = fmaxf(mrun, fmaxf(redm[row], redm[BQ + row]));
            const float f = lrun > 0.f ? exp_sfu(mrun - mnew) : 0.f;
            float psum = 0.f;
#pragma unroll
            for (int k = 0; k < 32; k++) {
                const float p = 32 * half + k < len ? exp_sfu(s[k] - mnew) : 0.f;
                s[k] = p * 16384.f;  // 2^14: small weights stay normal in f16
                psum += p;
            }
            reds[half * BQ + row] = psum;
            if (half == 0) fr[row] = f;
#pragma unroll
            for (int g = 0; g < 4; g++) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = s[g * 8 + e];
                put8x2(Phi, Plo, kmajor_off(row, 32 * half + g * 8, BQ), v);
            }
            fence_async_smem();
            mbar_arrive(mP);
            asm volatile("bar.sync 1, 256;" ::: "memory");
            lrun = lrun * f + (reds[row] + reds[BQ + row]);
            mrun = mnew;
            // (2) fold P V(i) into O: O = O * f + (hi*hi + cross terms); a failed wait is voted on at the next step
            alive = mbar_wait(mPV, (uint32_t)i & 1u, TC_WAIT_CYCLES);
            fence_after_sync();
            __syncwarp();
            if (alive) {
                const float fo = fr[row];
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float x[32], y[32];
                    tmem_ld32(tO + lane_base + 64 * half + 32 * c, x);
                    tmem_ld32(tO + 128 + lane_base + 64 * half + 32 * c, y);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; k++) o[32 * c + k] = fmaf(o[32 * c + k], fo, x[k] + y[k]);
                }
            }
            fence_before_sync();
            mbar_arrive(mO);
            any = true;
        }
        if (!compute_all(alive)) {
            if (tid == 0) *abort_flag = 1;
        }
    }
    fence_before_sync();
    __syncthreads();
    const bool ok = any && !*abort_flag;
    const int r = r0 + row;
    if (!producer && r < a.R) {
        const float oun = pow2f(-14 - a.tc_eV);
        const int col = 64 * half;
        if (a.splits == 1 && !a.parts_only) {
            const float inv = ok ? 1.0f / lrun : 0.f;
            float *dst = a.out + (size_t)r * a.ldo + h * HD + col;
#pragma unroll
            for (int k = 0; k < 64; k++) dst[k] = o[k] * oun * inv;
        } else {
            float *dst = a.part_acc + ((size_t)split * a.R + r) * d + h * HD + col;
#pragma unroll
            for (int k = 0; k < 64; k++) dst[k] = ok ? o[k] * oun : 0.f;
            if (half == 0) {
                float *ms = a.part_ms + (((size_t)split * a.R + r) * H + h) * 2;
                ms[0] = ok ? mrun : -FLT_MAX, ms[1] = ok ? lrun : 0.f;
            }
        }
    }
    if (*abort_flag && tid == 0 && a.err) atomicExch(a.err, 1);
    if (warp == 0) tmem_dealloc(tmem, 512);
}

size_t attend_tc_smem() {
    return sizeof(__half) * (2 * TC_BQ * TC_HD + 2 * 4 * TC_BLOCK + 2 * TC_BQ * TC_BK) + sizeof(float) * 5 * TC_BQ +
           12 * sizeof(uint64_t) + 16;
}

cudaError_t launch_tc_tiles(int kv, const AttnArgs &a, void *out, cudaStream_t s, uint64_t *launches) {
    dim3 grid(a.ntiles, a.heads);
    __half *o = reinterpret_cast<__half *>(out);
    if (kv == 0)
        k_tc_tiles<0><<<grid, 256, 0, s>>>(a, o);
    else if (kv == 1)
        k_tc_tiles<1><<<grid, 256, 0, s>>>(a, o);
    else
        k_tc_tiles<2><<<grid, 256, 0, s>>>(a, o);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_attend_tc(int kv, const AttnArgs &a, cudaStream_t s, uint64_t *launches) {
    if (!a.tc_tiles) return cudaErrorInvalidValue;
    const size_t smem = attend_tc_smem();
    dim3 grid((a.R + 127) / 128, a.heads, a.splits);
    cudaError_t e = cudaSuccess;
    if (kv == 0) {
        e = cudaFuncSetAttribute(k_attend_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_attend_tc<0><<<grid, TC_THREADS, smem, s>>>(a);
    } else if (kv == 1) {
        e = cudaFuncSetAttribute(k_attend_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_attend_tc<1><<<grid, TC_THREADS, smem, s>>>(a);
    } else {
        e = cudaFuncSetAttribute(k_attend_tc<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_attend_tc<2><<<grid, TC_THREADS, smem, s>>>(a);
    }
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
    if (a.splits > 1 && !a.parts_only) return launch_attend_merge(a, a.splits, s, launches);
    return cudaSuccess;
}

// ---- largest magnitude of a layer's keys and of its values (for the tensor-core scaling) ----------------------

__global__ void k_absmax_layer(const uint8_t *layer, int rows, int chunk, int d, int kv, unsigned *out) {
    const int ci = blockIdx.x, tid = threadIdx.x;
    const int rc = min(chunk, rows - ci * chunk);
    const uint8_t *rec = layer + (size_t)ci * record_bytes(kv, d, chunk);
    float mk = 0.f, mv = 0.f;
    if (kv == 0) {
        const float *p = reinterpret_cast<const float *>(rec);
        const size_t n = (size_t)d * rc;
        for (size_t i = tid; i < n; i += blockDim.x) mk = fmaxf(mk, fabsf(p[i]));
        for (size_t i = tid; i < n; i += blockDim.x) mv = fmaxf(mv, fabsf(p[n + i]));
    } else {
        // a coordinate's largest stored value is its scale times the integer maximum (fit.rs:560-561)
        const float *sc = reinterpret_cast<const float *>(rec);
        const float top = kv == 1 ? 32767.f : 127.f;
        for (int j = tid; j < d; j += blockDim.x) mk = fmaxf(mk, sc[j] * top), mv = fmaxf(mv, sc[d + j] * top);
    }
    mk = warp_max(mk), mv = warp_max(mv);
    if ((tid & 31) == 0) {
        atomicMax(out, __float_as_uint(mk));  // non-negative floats order as their bits
        atomicMax(out + 1, __float_as_uint(mv));
    }
}

cudaError_t launch_absmax_layer(const uint8_t *layer, int rows, int chunk, int d, int kv, unsigned *out, cudaStream_t s,
                                uint64_t *launches) {
    cudaError_t e = cudaMemsetAsync(out, 0, 2 * sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    k_absmax_layer<<<(rows + chunk - 1) / chunk, 256, 0, s>>>(layer, rows, chunk, d, kv, out);
    if (launches) ++*launches;
    return cudaGetLastError();
}

int tc_exponent(float mx) {
    if (!(mx > 0.f)) return 0;
    int ex = 0;
    std::frexp(mx, &ex);  // mx < 2^ex
    int e = 14 - ex;
    return e < -120 ? -120 : (e > 120 ? 120 : e);
}

// ---- self-test of the operand layouts and descriptors ------------------------------------------------------

// D[128][N] = A[128][128] B[N][128]^T with small-integer f16 values (exact in f32), B K-major or MN-major, on the
// tensor cores and on CUDA cores; writes the largest difference and whether every wait finished.
template <int N>
__global__ void __launch_bounds__(128) k_tc_selftest(int b_mn_major, float *result) {
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *A = reinterpret_cast<__half *>(smraw);  // [128][128] K-major
    __half *B = A + 128 * 128;                       // [N][128]
    uint64_t *mbar = reinterpret_cast<uint64_t *>(B + N * 128);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    auto av = [](int m, int k) { return (float)(((m * 7 + k * 3) % 13) - 6); };
    auto bv = [](int n, int k) { return (float)(((n * 5 + k * 11) % 9) - 4); };
    for (int i = tid; i < 128 * 128; i += 128) {
        const int m = i / 128, k = i % 128;
        A[kmajor_off(m, k, 128)] = __float2half_rn(av(m, k));
    }
    for (int i = tid; i < N * 128; i += 128) {
        const int n = i / 128, k = i % 128;
        B[b_mn_major ? mnmajor_off(n, k, N) : kmajor_off(n, k, N)] = __float2half_rn(bv(n, k));
    }
    if (warp == 0) {
        tmem_alloc(tslot, 256);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(mbar, 1);
        mbar_init_fence();
    }
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot;
    if (tid == 0) {
        const uint32_t id = idesc_f16(128, N, 0, b_mn_major);
        for (int s = 0; s < 8; s++) mma_f16(tmem, kstep_desc(A, 128, s), kstep_desc(B, N, s), id, s > 0);
        mma_commit(mbar);
    }
    const bool ok = mbar_wait(mbar, 0, TC_WAIT_CYCLES);
    fence_after_sync();
    float worst = 0.f;
    if (ok) {
        const int m = tid;
        for (int c = 0; c < N / 32; c++) {
            float o[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 32 * c, o);
            tmem_wait_ld();
            for (int e = 0; e < 32; e++) {
                const int n = 32 * c + e;
                float want = 0.f;
                for (int k = 0; k < 128; k++) want += av(m, k) * bv(n, k);
                worst = fmaxf(worst, fabsf(o[e] - want));
            }
        }
    }
    worst = warp_max(worst);
    if ((tid & 31) == 0) atomicMax(reinterpret_cast<unsigned *>(result), __float_as_uint(worst));
    if (!ok && tid == 0) atomicExch(reinterpret_cast<unsigned *>(result) + 1, 1u);
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

cudaError_t launch_tc_selftest(float *result, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(result, 0, 2 * sizeof(float), s);
    if (e != cudaSuccess) return e;
    const size_t smem64 = sizeof(__half) * (128 * 128 + 64 * 128) + 64;
    const size_t smem128 = sizeof(__half) * (128 * 128 + 128 * 128) + 64;
    e = cudaFuncSetAttribute(k_tc_selftest<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem64);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_tc_selftest<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem128);
    if (e != cudaSuccess) return e;
    for (int mn = 0; mn < 2; mn++) {
        k_tc_selftest<64><<<1, 128, smem64, s>>>(mn, result);
        k_tc_selftest<128><<<1, 128, smem128, s>>>(mn, result);
    }
    return cudaGetLastError();
}

}  // namespace tcu
