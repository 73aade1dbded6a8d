// Device-side scalar math of tabicl-anywhere's CPU path, restated from its own published formulas (not CUDA's
// math library): the reference's exponential, erf, GELU and tanh (src/kern.rs:214-297). Using the same
// formulas on both sides keeps the device within rounding of the CPU path.
#pragma once
#include <cstdint>

namespace tcu {

// kern.rs:220-235: Cody-Waite reduction by ln 2 (split in two parts) and a degree-7 Taylor polynomial, the
// argument clamped to [-87, 88] so the result is never zero, denormal or infinite.
__device__ __forceinline__ float exp1(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    float n = floorf(x * 1.44269504088896340736f + 0.5f);
    float r = (x - n * 0.6933594f) - n * -2.1219444e-4f;
    float p = 1.0f / 5040.0f;
    p = p * r + 1.0f / 720.0f;
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    return p * __int_as_float(((int)n + 127) << 23);
}

// kern.rs:256-282: erf by Abramowitz and Stegun 7.1.26 for |x| >= 0.5, its power series below.
__device__ __forceinline__ float erf1(float x) {
    float a = fabsf(x);
    float t = 1.0f / (1.0f + 0.3275911f * a);
    float p = 1.0614054f;
    p = p * t - 1.4531521f;
    p = p * t + 1.4214138f;
    p = p * t - 0.28449674f;
    p = p * t + 0.2548296f;
    float far = copysignf(1.0f - p * t * exp1(-a * a), x);
    float x2 = x * x;
    float q = -1.0f / 1320.0f;
    q = q * x2 + 1.0f / 216.0f;
    q = q * x2 - 1.0f / 42.0f;
    q = q * x2 + 0.1f;
    q = q * x2 - 1.0f / 3.0f;
    q = q * x2 + 1.0f;
    float near = q * x * 1.12837916709551257390f;
    return a < 0.5f ? near : far;
}

// kern.rs:285-290: GELU as PyTorch defines it, x/2 (1 + erf(x / sqrt 2))
__device__ __forceinline__ float gelu1(float v) { return 0.5f * v * (1.0f + erf1(v * 0.70710678118654752440f)); }

// kern.rs:292-297: tanh through one exponential, argument clamped to [-10, 10]
__device__ __forceinline__ float tanh1(float x) {
    float e = exp1(2.0f * fminf(fmaxf(x, -10.0f), 10.0f));
    return (e - 1.0f) / (e + 1.0f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// L2 cache policies: cache bytes are read once per call (evict first); weights are re-read every layer and
// call and should keep their place in the 126 MB L2 (evict last).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Streaming 16-byte load of cache bytes: read-only path, no L1 allocation, L2 policy as given.
__device__ __forceinline__ uint4 ld_stream16(const void *p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// 8-byte streaming load (into .x, .y).
__device__ __forceinline__ uint4 ld_stream8(const void *p, uint64_t pol) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p), "l"(pol));
    return v;
}

// Weights: read-only path with an L2 policy (evict last).
__device__ __forceinline__ float4 ld_weight4(const float *p, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// Stored element e of a 16-byte vector of the cache, widened to float exactly (fit.rs:103-122 formats:
// 0 = f32 (4 per vector), 1 = i16 (8), 2 = i8 (16)).
template <int KV>
__device__ __forceinline__ float unpack(const uint4 &v, int e);
template <>
__device__ __forceinline__ float unpack<0>(const uint4 &v, int e) {
    uint32_t w = e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
    return __uint_as_float(w);
}
// Integers are widened without the conversion unit (a quarter-rate pipe): with the sign bit flipped, an n-bit
// value v becomes the unsigned v + 2^(n-1); placed in the low mantissa bits of 2^23 it is the float
// 2^23 + v + 2^(n-1), and subtracting 2^23 + 2^(n-1) leaves v. Every step is exact (integers below 2^24), so the
// result equals (float)v bit for bit.
template <>
__device__ __forceinline__ float unpack<1>(const uint4 &v, int e) {
    const uint32_t w = ((e >> 1) == 0 ? v.x : (e >> 1) == 1 ? v.y : (e >> 1) == 2 ? v.z : v.w) ^ 0x80008000u;
    const uint32_t f = __byte_perm(w, 0x4B000000u, (e & 1) ? 0x7632u : 0x7610u);
    return __uint_as_float(f) - 8421376.0f;  // 2^23 + 2^15
}
template <>
__device__ __forceinline__ float unpack<2>(const uint4 &v, int e) {
    const uint32_t w = ((e >> 2) == 0 ? v.x : (e >> 2) == 1 ? v.y : (e >> 2) == 2 ? v.z : v.w) ^ 0x80808080u;
    const uint32_t f = __byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)(e & 3));
    return __uint_as_float(f) - 8388736.0f;  // 2^23 + 2^7
}

// One stored element by index (any alignment), for ragged chunk tails.
template <int KV>
__device__ __forceinline__ float load_elem(const uint8_t *base, size_t i) {
    if (KV == 0) return __ldg((const float *)base + i);
    if (KV == 1) return (float)__ldg((const int16_t *)base + i);
    return (float)(int8_t)__ldg((const signed char *)base + i);
}

template <int KV>
struct KvFmt {
    static constexpr int W = KV == 0 ? 4 : (KV == 1 ? 2 : 1);  // bytes per element
    static constexpr int EPV = 16 / W;                          // elements per 16-byte vector
};

}  // namespace tcu
