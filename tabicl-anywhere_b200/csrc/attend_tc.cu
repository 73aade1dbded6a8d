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
#include "pdl.cuh"
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

// Attention of 128 query rows x one head over a range of 64-key tiles, with the tiles pre-split (k_tc_tiles).
// Tensor memory, 512 columns, one query row per lane:
//   [0, 128)    Q: hi in 0-63, lo in 64-127 (f16 pairs, element 2c in the low half of column c): the A operand of
//               S = Q K^T (K [64 keys x 128] K-major in shared memory)
//   [128, 320)  three S slots of 64 columns. The softmax overwrites S(i) in place with P(i) (hi in the first 32
//               columns, lo in the next 32, f16 pairs): the A operand of P V^T (V [128 x 64 keys] K-major in shared
//               memory)
//   [384, 512)  P V^T of the latest tile
// Roles: warps 0-3 run the online softmax (one thread per query row, the nn.rs:207-215 rule), warps 4-7 fold each
// tile's P V into O held in registers (O = O f + P V), one thread each of warps 8 and 11 issues the S MMAs of even
// and odd tiles and one of warp 10 the P V MMAs (one thread alone cannot keep the tensor pipe fed), one thread of
// warp 9 bulk-copies keys and values into three-slot rings. They hand over through mbarriers only: S(i + 2) runs on the
// tensor cores while the softmax of tile i + 1 runs, and the fold of tile i while S(i + 2) runs. With both A
// operands in TMEM the MMAs read only K and V from shared memory. Each product is hi*hi + hi*lo + lo*hi with the
// two cross terms accumulated first, so the tensor cores' f32 accumulation (not round-to-nearest) adds only 8 (S)
// or 4 (P V) steps of full magnitude; every sum across tiles is taken in registers. Every wait is bounded; a wait
// that gives up raises the block's abort flag and everyone leaves.
// four softmax warps, four fold warps, two S-issuing warps (even and odd tiles), the load warp and the P V-issuing
// warp
constexpr int TC_THREADS = 384;
constexpr int TC_SLOTS = 3;      // S/P slots in TMEM, key and value slots in shared memory
constexpr uint32_t TM_Q = 0, TM_SP = 128, TM_O = 384;

template <int KV>
__global__ void __launch_bounds__(TC_THREADS, 1) k_attend_tc(AttnArgs a) {
    constexpr int HD = TC_HD, BQ = TC_BQ, BK = TC_BK, NS = TC_SLOTS;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Kring = reinterpret_cast<__half *>(smraw);                 // NS slots of [keys hi][keys lo]
    __half *Vring = Kring + NS * 2 * TC_BLOCK;                         // NS slots of [values hi][values lo]
    float *fr = reinterpret_cast<float *>(Vring + NS * 2 * TC_BLOCK);  // [4][BQ]: tile i's rescale factors in i % 4
    float *rowx = fr + 4 * BQ;  // [3][BQ]: each row's m, l and 1 / l at the end
    uint64_t *mb = reinterpret_cast<uint64_t *>(rowx + 3 * BQ);
    uint64_t *mK = mb, *mV = mb + NS, *mKfree = mb + 2 * NS, *mVfree = mb + 3 * NS;
    uint64_t *mS = mb + 4 * NS, *mP = mb + 5 * NS, *mSlot = mb + 6 * NS;  // S done, P written, P V done, per slot
    uint64_t *mPV = mb + 7 * NS, *mOfree = mPV + 1, *mF = mPV + 2, *mDone = mPV + 6;  // mDone[3]: per issuer
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mPV + 9);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    float *qmax = fr;                                  // [2][BQ] query halves' maxima, before the first factor
    float *ostage = reinterpret_cast<float *>(Kring);  // [BQ][HD + 1] after the last fold

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, split = blockIdx.z, r0 = blockIdx.x * BQ, d = a.d, H = gridDim.y;
    const int t0 = split * a.tiles_per_split, t1 = min(a.ntiles, t0 + a.tiles_per_split), nt = max(0, t1 - t0);
    const __half *tiles = reinterpret_cast<const __half *>(a.tc_tiles);
    const int row = tid & (BQ - 1), part = (tid >> 7) & 1;  // compute threads: query row; softmax (0) or fold (1)
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&mK[i], 1), mbar_init(&mV[i], 1), mbar_init(&mKfree[i], 1), mbar_init(&mVfree[i], 1);
            mbar_init(&mS[i], 1), mbar_init(&mP[i], BQ), mbar_init(&mSlot[i], 1);
        }
        mbar_init(mPV, 1), mbar_init(mOfree, BQ);
        for (int i = 0; i < 4; i++) mbar_init(&mF[i], BQ);
        mbar_init(&mDone[0], 1), mbar_init(&mDone[1], 1), mbar_init(&mDone[2], 1);
        mbar_init_fence();
        *abort_flag = 0;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    pdl_trigger();  // every block holds its tensor memory
    const uint32_t tmem = *tslot;
    const uint32_t half_bytes = (uint32_t)(2 * TC_BLOCK * sizeof(__half));
    auto load = [&](int i, bool values) {  // the load thread: keys or values of tile t0 + i into slot i % NS
        const __half *src = tiles + ((size_t)(t0 + i) * H + h) * 4 * TC_BLOCK + (values ? 2 * TC_BLOCK : 0);
        __half *dst = (values ? Vring : Kring) + (size_t)(i % NS) * 2 * TC_BLOCK;
        uint64_t *m = values ? &mV[i % NS] : &mK[i % NS];
        expect_tx(m, half_bytes);
        bulk_g2s(dst, src, half_bytes, m);
    };
    // the first tiles before the kernel before has finished: the split keys and values are written only by kernels
    // launched the ordinary way (at load, or per layer of a fit), which every later kernel starts after
    if (warp == 9 && lane == 0) {
        for (int i = 0; i < min(nt, NS); i++) load(i, false), load(i, true);
    }
    pdl_wait();  // the queries come from the kernel before
    // each compute thread: half of its row's query (head columns 64 * part + [0, 64)) and its largest magnitude
    float qv[64];
    if (tid < 2 * BQ) {
        const int r = r0 + row;
        float mx = 0.f;
        if (r < a.R) {
            const float4 *qp = reinterpret_cast<const float4 *>(a.q + (size_t)r * a.ldq + h * HD + 64 * part);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float4 v = qp[j];
                qv[4 * j] = v.x, qv[4 * j + 1] = v.y, qv[4 * j + 2] = v.z, qv[4 * j + 3] = v.w;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 64; j++) qv[j] = 0.f;
        }
        qmax[part * BQ + row] = mx;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    // the row's query scale (its largest |q| maps below 2^14); Q split into TMEM
    float rs = 1.f;
    if (tid < 2 * BQ) {
        const float qs = pow2f(f16_exponent(fmaxf(qmax[row], qmax[BQ + row])));
        rs = (1.0f / qs) * pow2f(-a.tc_eK);  // undoes both scalings of S
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int c = 0; c < 32; c++) split_pair(qv[2 * c] * qs, qv[2 * c + 1] * qs, hi[c], lo[c]);
        tmem_st32u(tmem + lane_base + TM_Q + 32 * part, hi);
        tmem_st32u(tmem + lane_base + TM_Q + 64 + 32 * part, lo);
        tmem_wait_st();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();

    auto wait = [&](uint64_t *m, uint32_t parity) {
        if (mbar_test_wait(m, parity)) return true;
        if (*abort_flag) return false;
        if (!mbar_wait(m, parity, TC_WAIT_CYCLES)) {
            *abort_flag = 1;
            return false;
        }
        return true;
    };
    // warp-uniform wait (the tcgen05 loads and stores after it are warp-wide)
    auto wait_warp = [&](uint64_t *m, uint32_t parity) {
        bool okw = mbar_test_wait(m, parity) || (!*abort_flag && mbar_wait(m, parity, TC_WAIT_CYCLES));
        okw = __all_sync(0xffffffffu, okw);
        if (!okw) *abort_flag = 1;
        return okw;
    };

    if (warp == 8 || warp == 10 || warp == 11) {
        if (lane == 0) {
            // the three MMA threads: each waits only for what its next MMAs read or overwrite
            const uint32_t idS = idesc_f16(BQ, BK, 0, 0), idO = idesc_f16(BQ, HD, 0, 0);
            const uint64_t dK0 = kstep_desc(Kring, BK, 0), dV0 = kstep_desc(Vring, HD, 0);
            const uint64_t stK = (2 * (BK / 8) * 128) >> 4, stV = (2 * (HD / 8) * 128) >> 4;
            const uint64_t lo_off = (TC_BLOCK * sizeof(__half)) >> 4, slot_off = (2 * TC_BLOCK * sizeof(__half)) >> 4;
            auto issue_S = [&](int i) {  // S(i) into TMEM slot i % NS from key slot i % NS
                const int sl = i % NS;
                const uint32_t tS = tmem + TM_SP + 64 * sl;
                const uint64_t dKh = dK0 + sl * slot_off, dKl = dKh + lo_off;
                fence_after_sync();
#pragma unroll
                for (int k = 0; k < HD / 16; k++) mma_f16_ta(tS, tmem + TM_Q + 8 * k, dKl + k * stK, idS, k > 0 ? 1u : 0u);
#pragma unroll
                for (int k = 0; k < HD / 16; k++) mma_f16_ta(tS, tmem + TM_Q + 64 + 8 * k, dKh + k * stK, idS, 1);
#pragma unroll
                for (int k = 0; k < HD / 16; k++) mma_f16_ta(tS, tmem + TM_Q + 8 * k, dKh + k * stK, idS, 1);
                mma_commit(&mS[sl]);
                mma_commit(&mKfree[sl]);
            };
            auto issue_PV = [&](int i) {  // P V(i) from P in TMEM slot i % NS and value slot i % NS
                const int sl = i % NS;
                const uint32_t pA = tmem + TM_SP + 64 * sl, tO = tmem + TM_O;
                const uint64_t dVh = dV0 + sl * slot_off, dVl = dVh + lo_off;
                fence_after_sync();
#pragma unroll
                for (int k = 0; k < BK / 16; k++) mma_f16_ta(tO, pA + 8 * k, dVl + k * stV, idO, k > 0 ? 1u : 0u);
#pragma unroll
                for (int k = 0; k < BK / 16; k++) mma_f16_ta(tO, pA + 32 + 8 * k, dVh + k * stV, idO, 1);
#pragma unroll
                for (int k = 0; k < BK / 16; k++) mma_f16_ta(tO, pA + 8 * k, dVh + k * stV, idO, 1);
                mma_commit(mPV);
                mma_commit(&mVfree[sl]);
                mma_commit(&mSlot[sl]);
            };
            bool ok = true;
            if (warp != 10) {
                // S(j) into slot j % NS once P V(j - NS) has read that slot, from its keys; even j by warp 8, odd j
                // by warp 11
                for (int j = warp == 8 ? 0 : 1; j < nt && ok; j += 2) {
                    const int sj = j % NS;
                    const uint32_t pj = (uint32_t)(j / NS) & 1u;
                    const bool f = j < NS || mbar_test_wait(&mSlot[sj], pj ^ 1u), k = mbar_test_wait(&mK[sj], pj);
                    if (!f && !(ok = wait(&mSlot[sj], pj ^ 1u))) break;
                    if (!k && !(ok = wait(&mK[sj], pj))) break;
                    issue_S(j);
                }
            } else {
                // P V of tile i: its P written, its values here, the fold of P V(i - 1) done (the three tests issued
                // together; a blocking wait only for one that is not complete yet)
                for (int i = 0; i < nt && ok; i++) {
                    const int sl = i % NS;
                    const uint32_t ph = (uint32_t)(i / NS) & 1u;
                    const bool p = mbar_test_wait(&mP[sl], ph), v = mbar_test_wait(&mV[sl], ph);
                    const bool o = i < 1 || mbar_test_wait(mOfree, (uint32_t)(i - 1) & 1u);
                    if (!p && !(ok = wait(&mP[sl], ph))) break;
                    if (!v && !(ok = wait(&mV[sl], ph))) break;
                    if (!o && !(ok = wait(mOfree, (uint32_t)(i - 1) & 1u))) break;
                    issue_PV(i);
                }
            }
            // every MMA this thread issued completes before the block lets go of tensor memory
            uint64_t *done = &mDone[warp == 8 ? 0 : warp == 10 ? 1 : 2];
            mma_commit(done);
            mbar_wait(done, 0, TC_WAIT_CYCLES);
        }
    } else if (warp == 9) {
        if (lane == 0) {
            // the load thread: tile i + NS's keys into tile i's slot once S(i) is done, its values once P V(i) is
            int kl = min(nt, NS), vl = kl;  // key / value loads started
            for (int i = 0; i + NS < nt; i++) {
                const uint32_t ph = (uint32_t)(i / NS) & 1u;
                if (!wait(&mKfree[i % NS], ph)) break;
                load(i + NS, false);
                kl = i + NS + 1;
                if (!wait(&mVfree[i % NS], ph)) break;
                load(i + NS, true);
                vl = i + NS + 1;
            }
            // the last load into each slot lands before the block lets go of shared memory
            for (int j = max(0, kl - NS); j < kl; j++) mbar_wait(&mK[j % NS], (uint32_t)(j / NS) & 1u, TC_WAIT_CYCLES);
            for (int j = max(0, vl - NS); j < vl; j++) mbar_wait(&mV[j % NS], (uint32_t)(j / NS) & 1u, TC_WAIT_CYCLES);
        }
    } else if (part == 0) {
        // softmax: S(i) -> P(i) = e^(S - m) (scaled by 2^14 so small weights stay normal in f16), written over S(i)
        // in its TMEM slot, and the factor f
        float mrun = -FLT_MAX, lrun = 0.f;
        for (int i = 0; i < nt; i++) {
            const int sl = i % NS;
            const int len = a.tiles[t0 + i].z;
            if (!wait_warp(&mS[sl], (uint32_t)(i / NS) & 1u)) break;
            fence_after_sync();
            const uint32_t tsp = tmem + lane_base + TM_SP + 64 * sl;
            float s[64];
            {
                float x[32], y[32];
                tmem_ld32(tsp, x);
                tmem_ld32(tsp + 32, y);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) s[k] = x[k], s[32 + k] = y[k];
            }
            // the scores are s * rs (rs > 0, so the largest raw score gives the largest score)
            float mx = -FLT_MAX;
            if (len == BK) {
#pragma unroll
                for (int k = 0; k < 64; k++) mx = fmaxf(mx, s[k]);
            } else {
#pragma unroll
                for (int k = 0; k < 64; k++)
                    if (k < len) mx = fmaxf(mx, s[k]);
            }
            const float mnew = fmaxf(mrun, mx * rs);
            const float f = lrun > 0.f ? exp_sfu(mrun - mnew) : 0.f;
            // p 2^14 = 2^(s rs log2 e - (mnew log2 e - 14)): one FMA and one ex2 per weight (2^14 keeps small
            // weights normal in f16)
            const float c1 = rs * 1.44269504088896340736f, c0 = mnew * 1.44269504088896340736f - 14.f;
            float psum = 0.f;
#pragma unroll
            for (int k = 0; k < 64; k++) {
                float p;
                asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(fmaf(s[k], c1, -c0)));
                s[k] = (len == BK || k < len) ? p : 0.f;
                psum += s[k];
            }
            psum *= 1.0f / 16384.f;
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int c = 0; c < 32; c++) split_pair(s[2 * c], s[2 * c + 1], hi[c], lo[c]);
            tmem_st32u(tsp, hi);
            tmem_st32u(tsp + 32, lo);
            tmem_wait_st();
            fr[(i & 3) * BQ + row] = f;
            fence_before_sync();
            mbar_arrive(&mP[sl]);
            mbar_arrive(&mF[i & 3]);
            lrun = lrun * f + psum;
            mrun = mnew;
        }
        rowx[row] = mrun, rowx[BQ + row] = lrun, rowx[2 * BQ + row] = lrun > 0.f ? 1.0f / lrun : 0.f;
    } else if (warp < 8) {
        // fold: O = O f(i) + P V(i), in registers
        float o[128];
#pragma unroll
        for (int e = 0; e < 128; e++) o[e] = 0.f;
        for (int i = 0; i < nt; i++) {
            if (!wait_warp(mPV, (uint32_t)i & 1u)) break;
            if (!wait_warp(&mF[i & 3], (uint32_t)(i >> 2) & 1u)) break;
            fence_after_sync();
            const float f = fr[(i & 3) * BQ + row];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float x[32];
                tmem_ld32(tmem + lane_base + TM_O + 32 * c, x);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) o[32 * c + k] = fmaf(o[32 * c + k], f, x[k]);
            }
            fence_before_sync();
            mbar_arrive(mOfree);
        }
        // after the last fold no MMA or load touches the key and value rings (on an abort the rows are not used)
#pragma unroll
        for (int k = 0; k < HD; k++) ostage[row * (HD + 1) + k] = o[k];
    }
    fence_before_sync();
    __syncthreads();
    const bool ok = nt > 0 && !*abort_flag;
    if (tid < 2 * BQ) {
        const float oun = pow2f(-14 - a.tc_eV);
        const bool whole = a.splits == 1 && !a.parts_only;
        for (int idx = tid; idx < BQ * HD; idx += 2 * BQ) {
            const int m = idx / HD, k = idx % HD, r = r0 + m;
            if (r >= a.R) break;  // rows grow with idx
            const float v = ostage[m * (HD + 1) + k] * oun;
            if (whole && a.state_ms) {
                a.out[(size_t)r * a.ldo + h * HD + k] = ok ? v : 0.f;
                if (k == 0) {
                    float *ms = a.state_ms + ((size_t)r * H + h) * 2;
                    ms[0] = ok ? rowx[m] : -FLT_MAX, ms[1] = ok ? rowx[BQ + m] : 0.f;
                }
            } else if (whole) {
                a.out[(size_t)r * a.ldo + h * HD + k] = ok ? v * rowx[2 * BQ + m] : 0.f;
            } else {
                a.part_acc[((size_t)split * a.R + r) * d + h * HD + k] = ok ? v : 0.f;
                if (k == 0) {
                    float *ms = a.part_ms + (((size_t)split * a.R + r) * H + h) * 2;
                    ms[0] = ok ? rowx[m] : -FLT_MAX, ms[1] = ok ? rowx[BQ + m] : 0.f;
                }
            }
        }
    }
    if (*abort_flag && tid == 0 && a.err) *reinterpret_cast<volatile int *>(a.err) = 1;  // a report slot in host memory
    // split parts: the last of a (row block, head)'s splits to finish merges them (the log-sum-exp merge of
    // k_attend_merge, predict.rs:455-478, with the same products and order of sums)
    if (a.splits > 1 && !a.parts_only && a.merge_cnt) {
        volatile int *last = abort_flag + 1;
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            int *cnt = a.merge_cnt + blockIdx.x * H + h;
            const int prev = atomicAdd(cnt, 1);
            *last = prev == a.splits - 1;
            if (prev == a.splits - 1) *cnt = 0;  // every split has arrived: ready for the next launch
        }
        __syncthreads();
        if (*last) {
            __threadfence();
            const int P = a.splits;
            float *wts = reinterpret_cast<float *>(Vring);  // [P][BQ] part weights, then [BQ] 1 / sums
            float *winv = wts + P * BQ;
            if (tid < BQ && r0 + tid < a.R) {
                // eight parts' (max, weight sum) pairs in flight at a time
                const int r = r0 + tid;
                const float2 *msr = reinterpret_cast<const float2 *>(a.part_ms) + (size_t)r * H + h;
                const size_t mstep = (size_t)a.R * H;
                float M = -FLT_MAX;
                for (int p0 = 0; p0 < P; p0 += 8) {
                    float2 ms[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (p0 + u < P) ms[u] = __ldcg(msr + (p0 + u) * mstep);
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (p0 + u < P && ms[u].y > 0.f) M = fmaxf(M, ms[u].x);
                }
                float S = 0.f;
                for (int p0 = 0; p0 < P; p0 += 8) {
                    float2 ms[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (p0 + u < P) ms[u] = __ldcg(msr + (p0 + u) * mstep);
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        if (p0 + u < P) {
                            const float l = ms[u].y, w = l > 0.f ? exp1(ms[u].x - M) : 0.f;
                            wts[(p0 + u) * BQ + tid] = w;
                            S = __fadd_rn(S, __fmul_rn(l, w));
                        }
                    }
                }
                winv[tid] = a.state_ms ? 1.0f : 1.0f / S;
                if (a.state_ms) {
                    float *st = a.state_ms + ((size_t)r * H + h) * 2;
                    st[0] = S > 0.f ? M : -FLT_MAX, st[1] = S;
                }
            }
            __syncthreads();
            const size_t pstride = (size_t)a.R * d;
            const float oun = pow2f(-14 - a.tc_eV);
            if (tid < 2 * BQ) {
                // four values of a row per thread and step, two steps at a time; the parts in groups of eight, every
                // load of a group issued before any is used, summed in part order; this block's own part is still in
                // shared memory
                constexpr int STEPS = BQ * HD / 4 / (2 * BQ);
#pragma unroll 1
                for (int st = 0; st < STEPS; st += 2) {
                    float4 o[2], ownv[2];
                    const float *base[2];
                    int mm[2];
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const int e4 = tid + (st + u) * 2 * BQ, m = e4 / (HD / 4), k0 = (e4 % (HD / 4)) * 4;
                        const int r = min(r0 + m, a.R - 1);
                        base[u] = a.part_acc + (size_t)r * d + h * HD + k0;
                        mm[u] = m;
                        const float *own = ostage + m * (HD + 1) + k0;
                        ownv[u] = make_float4(own[0] * oun, own[1] * oun, own[2] * oun, own[3] * oun);
                        o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll 1
                    for (int p0 = 0; p0 < P; p0 += 8) {
                        float4 v[2][8];
#pragma unroll
                        for (int u = 0; u < 2; u++)
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                const int p = p0 + q;
                                if (p < P && p != split) v[u][q] = __ldcg(reinterpret_cast<const float4 *>(base[u] + p * pstride));
                            }
#pragma unroll
                        for (int u = 0; u < 2; u++)
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                const int p = p0 + q;
                                if (p < P) {
                                    const float4 x = p == split ? ownv[u] : v[u][q];
                                    const float w = wts[p * BQ + mm[u]];
                                    o[u].x = __fadd_rn(o[u].x, __fmul_rn(x.x, w)), o[u].y = __fadd_rn(o[u].y, __fmul_rn(x.y, w));
                                    o[u].z = __fadd_rn(o[u].z, __fmul_rn(x.z, w)), o[u].w = __fadd_rn(o[u].w, __fmul_rn(x.w, w));
                                }
                            }
                    }
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const int e4 = tid + (st + u) * 2 * BQ, m = mm[u], k0 = (e4 % (HD / 4)) * 4, r = r0 + m;
                        if (r >= a.R) continue;
                        const float iv = winv[m];
                        *reinterpret_cast<float4 *>(a.out + (size_t)r * a.ldo + h * HD + k0) =
                            make_float4(o[u].x * iv, o[u].y * iv, o[u].z * iv, o[u].w * iv);
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

size_t attend_tc_smem() {
    return sizeof(__half) * (2 * TC_SLOTS * 2 * TC_BLOCK) + sizeof(float) * 7 * TC_BQ +
           (7 * TC_SLOTS + 9) * sizeof(uint64_t) + 16;  // + the TMEM slot, the abort flag and the last-split flag
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
        e = allow_dynamic_smem((const void *)k_attend_tc<0>, smem);
        if (e == cudaSuccess) e = launch_pdl(k_attend_tc<0>, grid, dim3(TC_THREADS), smem, s, a);
    } else if (kv == 1) {
        e = allow_dynamic_smem((const void *)k_attend_tc<1>, smem);
        if (e == cudaSuccess) e = launch_pdl(k_attend_tc<1>, grid, dim3(TC_THREADS), smem, s, a);
    } else {
        e = allow_dynamic_smem((const void *)k_attend_tc<2>, smem);
        if (e == cudaSuccess) e = launch_pdl(k_attend_tc<2>, grid, dim3(TC_THREADS), smem, s, a);
    }
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
    if (a.splits > 1 && !a.parts_only && !a.merge_cnt) return launch_attend_merge(a, a.splits, s, launches);
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
__global__ void __launch_bounds__(128) k_tc_selftest(int b_mn_major, int a_tmem, float *result) {
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
    if (a_tmem) {
        // A into columns 128-191, one row per lane: column c holds k = 2c (low half) and 2c + 1
        const int m = tid;
        for (int h = 0; h < 2; h++) {
            uint32_t v[32];
            for (int c = 0; c < 32; c++) {
                const int k = 2 * (32 * h + c);
                const __half2 p = __floats2half2_rn(av(m, k), av(m, k + 1));
                v[c] = *reinterpret_cast<const uint32_t *>(&p);
            }
            tmem_st32u(tmem + ((uint32_t)(warp * 32) << 16) + 128 + 32 * h, v);
        }
        tmem_wait_st();
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
    }
    if (tid == 0) {
        const uint32_t id = idesc_f16(128, N, 0, b_mn_major);
        for (int s = 0; s < 8; s++) {
            if (a_tmem)
                mma_f16_ta(tmem, tmem + 128 + 8 * s, kstep_desc(B, N, s), id, s > 0);
            else
                mma_f16(tmem, kstep_desc(A, 128, s), kstep_desc(B, N, s), id, s > 0);
        }
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
        for (int at = 0; at < 2; at++) {
            k_tc_selftest<64><<<1, 128, smem64, s>>>(mn, at, result);
            k_tc_selftest<128><<<1, 128, smem128, s>>>(mn, at, result);
        }
    }
    return cudaGetLastError();
}

}  // namespace tcu
