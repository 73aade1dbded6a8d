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
// memory (keys MN-major, values K-major). Integers are widened exactly and multiplied by their chunk's scale
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
                put8(Khi, Klo, mnmajor_off(key, j, BK), fk, 1.f);
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
            split_f16(fk * kscale, Khi[mnmajor_off(key, j, BK)], Klo[mnmajor_off(key, j, BK)]);
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
//   S = Q K^T: Q [128 x 128] K-major, K [64 keys x 128] MN-major; hi*hi in TMEM columns 0-63, cross terms 64-127
//   O += P V^T: P [128 x 64 keys] K-major, V [128 x 64 keys] K-major; per tile hi*hi in 128-255, cross 256-383
// Each tile's four operand blocks arrive by bulk copies into one of two shared-memory stages, two tiles ahead. The
// online softmax (nn.rs:207-215 rule) runs on all eight warps, two threads per query row (one per half of the
// keys). While a tile's P V is folded into the registers' O, the next tile's S is already on the tensor cores.
// Every f32 sum of tensor-core results is taken in registers (fresh accumulators per tile: the units' own f32
// accumulation is not round-to-nearest). One thread issues the MMAs and copies; every wait is bounded.
template <int KV>
__global__ void __launch_bounds__(256, 1) k_attend_tc(AttnArgs a) {
    constexpr int HD = TC_HD, BQ = TC_BQ, BK = TC_BK;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Qhi = reinterpret_cast<__half *>(smraw);  // [BQ][HD] K-major
    __half *Qlo = Qhi + BQ * HD;
    __half *stage0 = Qlo + BQ * HD;                   // two stages of [keys hi][keys lo][values hi][values lo]
    __half *Phi = stage0 + 2 * 4 * TC_BLOCK;          // [BQ][BK keys] K-major
    __half *Plo = Phi + BQ * BK;
    float *fr = reinterpret_cast<float *>(Plo + BQ * BK);  // [BQ] this tile's rescale factor of each row
    float *redm = fr + BQ;                                 // [2][BQ] half-row maxima
    float *reds = redm + 2 * BQ;                           // [2][BQ] half-row weight sums
    uint64_t *mbar = reinterpret_cast<uint64_t *>(reds + 2 * BQ);  // S ready, P V ready, stage 0 loaded, stage 1
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    float *qscale = reinterpret_cast<float *>(Phi);  // [BQ] 2^e of each row's query (until the first P)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, split = blockIdx.z, r0 = blockIdx.x * BQ, d = a.d, H = gridDim.y;
    // a query row per (warp % 4, lane); keys / output columns by warp / 4
    const int row = (warp & 3) * 32 + lane, half = warp >> 2;
    const int t0 = split * a.tiles_per_split, t1 = min(a.ntiles, t0 + a.tiles_per_split), nt = t1 - t0;
    const __half *tiles = reinterpret_cast<const __half *>(a.tc_tiles);
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 4; i++) mbar_init(&mbar[i], 1);
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
    // the first two tiles start loading while the queries are split
    auto load_tile = [&](int i) {  // thread 0: tile t0 + i into stage i & 1
        const __half *src = tiles + ((size_t)(t0 + i) * H + h) * 4 * TC_BLOCK;
        __half *dst = stage0 + (size_t)(i & 1) * 4 * TC_BLOCK;
        uint64_t *mb = &mbar[2 + (i & 1)];
        expect_tx(mb, (uint32_t)(4 * TC_BLOCK * sizeof(__half)));
#pragma unroll
        for (int b = 0; b < 4; b++) bulk_g2s(dst + b * TC_BLOCK, src + b * TC_BLOCK, (uint32_t)(TC_BLOCK * sizeof(__half)), mb);
    };
    if (tid == 0) {
        if (nt > 0) load_tile(0);
        if (nt > 1) load_tile(1);
    }
    for (int i = tid; i < BQ * (HD / 8); i += 256) {
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
    const float rs = (1.0f / qscale[row]) * pow2f(-a.tc_eK);  // undoes the query's and the keys' scalings
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot, tShh = tmem, tSx = tmem + 64, tOhh = tmem + 128, tOx = tmem + 256;
    const uint32_t idS = idesc_f16(BQ, BK, 0, 1), idO = idesc_f16(BQ, HD, 0, 0);
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    auto issue_S = [&](int i) {  // thread 0: S of tile t0 + i from its stage
        const __half *K = stage0 + (size_t)(i & 1) * 4 * TC_BLOCK;
#pragma unroll
        for (int s = 0; s < HD / 16; s++) mma_f16(tShh, kstep_desc(Qhi, BQ, s), kstep_desc(K, BK, s), idS, s > 0 ? 1u : 0u);
#pragma unroll
        for (int s = 0; s < HD / 16; s++) {
            mma_f16(tSx, kstep_desc(Qhi, BQ, s), kstep_desc(K + TC_BLOCK, BK, s), idS, s > 0 ? 1u : 0u);
            mma_f16(tSx, kstep_desc(Qlo, BQ, s), kstep_desc(K, BK, s), idS, 1);
        }
        mma_commit(&mbar[0]);
    };
    uint32_t pS = 0, pO = 0, pK = 0;  // mbarrier parities (pK: bit per stage)
    int issued = min(nt, 2);  // tiles whose loads were started
    if (tid == 0 && nt > 0) {
        if (mbar_wait(&mbar[2], 0, TC_WAIT_CYCLES)) {
            fence_after_sync();
            issue_S(0);
        } else {
            *abort_flag = 1;
        }
        pK = 1;
    }
    float o[64];
#pragma unroll
    for (int e = 0; e < 64; e++) o[e] = 0.f;
    float mrun = -FLT_MAX, lrun = 0.f;
    bool any = false;
    int consumed = 0;
    for (int i = 0; i < nt; i++) {
        __syncthreads();
        if (*abort_flag) break;
        const int len = a.tiles[t0 + i].z;
        // (1) the online softmax of S, two threads per row
        const bool okS = mbar_wait(&mbar[0], pS, TC_WAIT_CYCLES);
        pS ^= 1;
        if (!okS) *abort_flag = 1;
        fence_after_sync();
        __syncwarp();
        float s[32];
        {
            float x[32], y[32];
            tmem_ld32(tShh + lane_base + 32 * half, x);
            tmem_ld32(tSx + lane_base + 32 * half, y);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; k++) s[k] = (x[k] + y[k]) * rs;
        }
        float mx = -FLT_MAX;
#pragma unroll
        for (int k = 0; k < 32; k++)
            if (32 * half + k < len) mx = fmaxf(mx, s[k]);
        redm[half * BQ + row] = mx;
        fence_before_sync();
        __syncthreads();
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
        fence_before_sync();
        __syncthreads();
        lrun = lrun * f + (reds[row] + reds[BQ + row]);
        mrun = mnew;
        // (2) this tile's P V, then the next tile's S (its stage loaded)
        if (tid == 0) {
            fence_after_sync();
            const __half *V = stage0 + (size_t)(i & 1) * 4 * TC_BLOCK + 2 * TC_BLOCK;
#pragma unroll
            for (int s2 = 0; s2 < BK / 16; s2++)
                mma_f16(tOhh, kstep_desc(Phi, BQ, s2), kstep_desc(V, HD, s2), idO, s2 > 0 ? 1u : 0u);
#pragma unroll
            for (int s2 = 0; s2 < BK / 16; s2++) {
                mma_f16(tOx, kstep_desc(Phi, BQ, s2), kstep_desc(V + TC_BLOCK, HD, s2), idO, s2 > 0 ? 1u : 0u);
                mma_f16(tOx, kstep_desc(Plo, BQ, s2), kstep_desc(V, HD, s2), idO, 1);
            }
            mma_commit(&mbar[1]);
            if (i + 1 < nt) {
                const int st = (i + 1) & 1;
                if (mbar_wait(&mbar[2 + st], (pK >> st) & 1u, TC_WAIT_CYCLES)) {
                    fence_after_sync();
                    issue_S(i + 1);
                } else {
                    *abort_flag = 1;
                }
                pK ^= 1u << st;
            }
        }
        // (3) fold this tile's P V into O: O = O * f + (hi*hi + cross terms)
        const bool okO = mbar_wait(&mbar[1], pO, TC_WAIT_CYCLES);
        pO ^= 1;
        if (!okO) *abort_flag = 1;
        fence_after_sync();
        __syncwarp();
        if (okO) {
            const float fo = fr[row];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float x[32], y[32];
                tmem_ld32(tOhh + lane_base + 64 * half + 32 * c, x);
                tmem_ld32(tOx + lane_base + 64 * half + 32 * c, y);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) o[32 * c + k] = fmaf(o[32 * c + k], fo, x[k] + y[k]);
            }
        }
        any = true;
        consumed = i + 1;
        fence_before_sync();
        __syncthreads();
        // (4) this tile's stage is free (its S and P V are done): the tile two ahead goes there
        if (tid == 0 && i + 2 < nt && !*abort_flag) {
            load_tile(i + 2);
            issued = i + 3;
        }
    }
    // leaving early: loads still in flight land before the shared memory is given up
    if (tid == 0) {
        for (int i = max(consumed + 1, 1); i < issued; i++) {
            const int st = i & 1;
            mbar_wait(&mbar[2 + st], (pK >> st) & 1u, TC_WAIT_CYCLES);
            pK ^= 1u << st;
        }
    }
    const bool ok = any && !*abort_flag;
    const int r = r0 + row;
    if (r < a.R) {
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
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

size_t attend_tc_smem() {
    return sizeof(__half) * (2 * TC_BQ * TC_HD + 2 * 4 * TC_BLOCK + 2 * TC_BQ * TC_BK) + sizeof(float) * 5 * TC_BQ +
           4 * sizeof(uint64_t) + 16;
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
        if (e == cudaSuccess) k_attend_tc<0><<<grid, 256, smem, s>>>(a);
    } else if (kv == 1) {
        e = cudaFuncSetAttribute(k_attend_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_attend_tc<1><<<grid, 256, smem, s>>>(a);
    } else {
        e = cudaFuncSetAttribute(k_attend_tc<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_attend_tc<2><<<grid, 256, smem, s>>>(a);
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
