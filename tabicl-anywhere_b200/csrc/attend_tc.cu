// Attention of many query rows on the 5th-generation tensor cores (tcgen05), at f32 accuracy.
//
// One CTA takes 128 query rows of one head and a range of 64-key tiles of the stored cache (chunks read in place,
// integer formats dequantised as they are staged). Every f32 operand is split into two f16 values (x = hi + lo,
// about 22 significant bits) after a power-of-two scaling that keeps it inside the f16 range, and each product is
// taken as hi*hi + hi*lo + lo*hi in f32 accumulators in tensor memory:
//   S = Q K^T: Q [128 rows x 128] K-major, K [64 keys x 128] keys-contiguous (as stored), S in TMEM columns 0-63;
//   O += P V^T: P [128 x 64 keys] K-major, V [128 dims x 64 keys] keys-contiguous (as stored), O in columns 64-191.
// The softmax is online across tiles (nn.rs:207-215 rule): each of the 128 threads of warps 0-3 owns one query
// row (its TMEM lane), so a row's maximum and sum need no shuffles; O is rescaled in TMEM only when the running
// maximum rises. One thread issues the MMAs; mbarrier waits are bounded and record a failure instead of hanging.
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

template <int KV>
__global__ void __launch_bounds__(256, 1) k_attend_tc(AttnArgs a) {
    constexpr int HD = 128, BQ = 128, BK = FLASH_KEYS, W = KvFmt<KV>::W, EPV = KvFmt<KV>::EPV, VPR = BK / EPV;
    extern __shared__ __align__(1024) uint8_t smraw[];
    __half *Qhi = reinterpret_cast<__half *>(smraw);  // [BQ][HD] K-major
    __half *Qlo = Qhi + BQ * HD;
    __half *Khi = Qlo + BQ * HD;                      // [BK keys][HD] MN-major
    __half *Klo = Khi + BK * HD;
    __half *Vhi = Klo + BK * HD;                      // [HD][BK keys] K-major
    __half *Vlo = Vhi + HD * BK;
    __half *Phi = Vlo + HD * BK;                      // [BQ][BK keys] K-major
    __half *Plo = Phi + BQ * BK;
    uint64_t *mbar = reinterpret_cast<uint64_t *>(Plo + BQ * BK);  // [0] S ready, [1] P V ready
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    float *qscale = reinterpret_cast<float *>(tslot + 4);  // [BQ] 2^e of each row's query
    float *fr = qscale + BQ;                               // [BQ] this tile's rescale factor of each row
    float *lrow = fr + BQ;                                 // [BQ] final weight sums
    float *mrow = lrow + BQ;                               // [BQ] final maxima

    const int tid = threadIdx.x, warp = tid >> 5;
    const int h = blockIdx.y, split = blockIdx.z, r0 = blockIdx.x * BQ, d = a.d, H = gridDim.y;
    if (warp == 0) {
        // S: hi*hi in columns 0-63, cross terms 64-127; one tile's P V: hi*hi 128-255, cross terms 256-383
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
        *abort_flag = 0;
    }
    // each row's query scale: its largest |q| maps below 2^14
    int erow = 0;
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
        erow = f16_exponent(mx);
        qscale[tid] = pow2f(erow);
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot, tShh = tmem, tSx = tmem + 64, tOhh = tmem + 128, tOx = tmem + 256;
    // queries, split; consecutive threads take consecutive rows so their 16-byte stores are contiguous
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
    const float kscale = pow2f(a.tc_eK), vscale = pow2f(a.tc_eV);
    const float row_unscale = tid < BQ ? pow2f(-erow) * pow2f(-a.tc_eK) : 1.f;
    const uint32_t idS = idesc_f16(BQ, BK, 0, 1), idO = idesc_f16(BQ, HD, 0, 0);
    // every thread's share of O: row (warp % 4) * 32 + lane, columns (warp / 4) * 64 + [0, 64)
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int orow = (warp & 3) * 32 + (tid & 31), ocol = (warp >> 2) * 64;
    float o[64];
#pragma unroll
    for (int e = 0; e < 64; e++) o[e] = 0.f;
    float mrun = -FLT_MAX, lrun = 0.f;
    uint32_t ps = 0, po = 0;
    const int t0 = split * a.tiles_per_split, t1 = min(a.ntiles, t0 + a.tiles_per_split);
    const uint64_t pol = policy_evict_first();
    bool any = false;
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
        const bool fast = len == BK && ((((uintptr_t)kb) | ((uintptr_t)vb) | rowb) & 15) == 0;
        if (fast) {
            // consecutive threads take consecutive dims (contiguous shared-memory stores in both layouts), each
            // reading a 32-byte run of its dim's keys
            for (int i = tid; i < HD * VPR / 2; i += 256) {
                const int j = i % HD, vp = i / HD;
                const float ks = (KV ? sc[h * HD + j] : 1.f) * kscale;
                const float vs = (KV ? sc[d + h * HD + j] : 1.f) * vscale;
                const uint4 rk0 = ld_stream16(kb + j * rowb + vp * 32, pol), rk1 = ld_stream16(kb + j * rowb + vp * 32 + 16, pol);
                const uint4 rv0 = ld_stream16(vb + j * rowb + vp * 32, pol), rv1 = ld_stream16(vb + j * rowb + vp * 32 + 16, pol);
#pragma unroll
                for (int g = 0; g < 2 * EPV; g += 8) {
                    float fk[8], fv[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const int x = g + e;  // element within the 32-byte run
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
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            fence_after_sync();
#pragma unroll
            for (int s = 0; s < HD / 16; s++)
                mma_f16(tShh, kstep_desc(Qhi, BQ, s), kstep_desc(Khi, BK, s), idS, s > 0 ? 1u : 0u);
#pragma unroll
            for (int s = 0; s < HD / 16; s++) {
                mma_f16(tSx, kstep_desc(Qhi, BQ, s), kstep_desc(Klo, BK, s), idS, s > 0 ? 1u : 0u);
                mma_f16(tSx, kstep_desc(Qlo, BQ, s), kstep_desc(Khi, BK, s), idS, 1);
            }
            mma_commit(&mbar[0]);
        }
        if (warp < 4) {
            const bool ok = mbar_wait(&mbar[0], ps, TC_WAIT_CYCLES);
            if (!ok) *abort_flag = 1;
            fence_after_sync();
            float s[64];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float x[32], y[32];
                tmem_ld32(tShh + lane_base + 32 * c, x);
                tmem_ld32(tSx + lane_base + 32 * c, y);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) s[32 * c + k] = (x[k] + y[k]) * row_unscale;
            }
            float mx = -FLT_MAX;
#pragma unroll
            for (int k = 0; k < 64; k++)
                if (k < len) mx = fmaxf(mx, s[k]);
            const float mnew = fmaxf(mrun, mx);
            const float f = lrun > 0.f ? exp1(mrun - mnew) : 0.f;
            float psum = 0.f;
#pragma unroll
            for (int k = 0; k < 64; k++) {
                const float p = k < len ? exp1(s[k] - mnew) : 0.f;
                s[k] = p * 16384.f;  // 2^14: small weights stay normal in f16
                psum += p;
            }
            lrun = lrun * f + psum;
            mrun = mnew;
            fr[tid] = f;
#pragma unroll
            for (int g = 0; g < 8; g++) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = s[g * 8 + e];
                put8(Phi, Plo, kmajor_off(tid, g * 8, BQ), v, 1.f);
            }
        }
        ps ^= 1;
        fence_async_smem();
        fence_before_sync();
        __syncthreads();
        if (*abort_flag) break;
        if (tid == 0) {
            fence_after_sync();
#pragma unroll
            for (int s = 0; s < BK / 16; s++)
                mma_f16(tOhh, kstep_desc(Phi, BQ, s), kstep_desc(Vhi, HD, s), idO, s > 0 ? 1u : 0u);
#pragma unroll
            for (int s = 0; s < BK / 16; s++) {
                mma_f16(tOx, kstep_desc(Phi, BQ, s), kstep_desc(Vlo, HD, s), idO, s > 0 ? 1u : 0u);
                mma_f16(tOx, kstep_desc(Plo, BQ, s), kstep_desc(Vhi, HD, s), idO, 1);
            }
            mma_commit(&mbar[1]);
        }
        // every thread folds this tile's P V into its share of O: O = O * f + (hi*hi + cross terms)
        const bool okO = mbar_wait(&mbar[1], po, TC_WAIT_CYCLES);
        po ^= 1;
        if (!okO) *abort_flag = 1;
        fence_after_sync();
        if (okO) {
            const float f = fr[orow];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float x[32], y[32];
                tmem_ld32(tOhh + lane_base + ocol + 32 * c, x);
                tmem_ld32(tOx + lane_base + ocol + 32 * c, y);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++) o[32 * c + k] = fmaf(o[32 * c + k], f, x[k] + y[k]);
            }
        }
        any = true;
        fence_before_sync();
        __syncthreads();
        if (*abort_flag) break;
    }
    if (tid < BQ) lrow[tid] = lrun, mrow[tid] = mrun;
    __syncthreads();
    const bool ok = any && !*abort_flag;
    const int r = r0 + orow;
    if (r < a.R) {
        const float oun = pow2f(-14 - a.tc_eV);
        if (a.splits == 1 && !a.parts_only) {
            const float inv = ok ? 1.0f / lrow[orow] : 0.f;
            float *dst = a.out + (size_t)r * a.ldo + h * HD + ocol;
#pragma unroll
            for (int k = 0; k < 64; k++) dst[k] = o[k] * oun * inv;
        } else {
            float *dst = a.part_acc + ((size_t)split * a.R + r) * d + h * HD + ocol;
#pragma unroll
            for (int k = 0; k < 64; k++) dst[k] = ok ? o[k] * oun : 0.f;
            if (ocol == 0) {
                float *ms = a.part_ms + (((size_t)split * a.R + r) * H + h) * 2;
                ms[0] = ok ? mrow[orow] : -FLT_MAX, ms[1] = ok ? lrow[orow] : 0.f;
            }
        }
    }
    if (*abort_flag && tid == 0 && a.err) atomicExch(a.err, 1);
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

size_t attend_tc_smem() {
    return sizeof(__half) * (2 * 128 * 128 + 2 * 64 * 128 + 2 * 128 * 64 + 2 * 128 * 64) + 64 + sizeof(float) * 4 * 128 + 64;
}

cudaError_t launch_attend_tc(int kv, const AttnArgs &a, cudaStream_t s, uint64_t *launches) {
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
