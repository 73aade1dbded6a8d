// Pieces of the few-row stage kernel (stage_rows.cu) kept apart from its phases: the layout of a key/value tile in
// shared memory, GPU-scope flag loads, and the bulk and tensor copies that fill shared memory.
#pragma once
#include <cstdint>

#include "device.cuh"
#include "tc.cuh"

namespace tcu {

// One tile of a head's stored keys and values as a few-row kernel keeps it in shared memory: TK keys of each of the
// head's HD key coordinates (ROWB bytes per coordinate), then the same of the values, then (integer formats) the
// chunk's HD key scales and HD value scales. A lane reads VB bytes (EPV keys) of a coordinate's row at a time.
template <int KV, int HD>
struct TileFmt {
    static constexpr int W = KvFmt<KV>::W;
    static constexpr int VB = KV == 2 ? 8 : 16;  // bytes of a coordinate's row a lane reads
    static constexpr int EPV = VB / W;            // keys per lane vector: 4, 8, 8
    static constexpr int TK = 8 * EPV;            // keys per tile: 32, 64, 64
    static constexpr int ROWB = TK * W;           // bytes of one coordinate's keys in a tile: 128, 128, 64
    static constexpr int DPT = HD / 32;           // coordinates per thread
    static constexpr int SLOT = 2 * HD * ROWB + (KV ? 8 * HD : 0);  // keys, values, then key and value scales
    static_assert(SLOT % 128 == 0 && (HD * ROWB) % 128 == 0, "tensor-load destinations must be 128-byte aligned");
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_s32(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *mbar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n" ::"r"(
                     tc::smem_addr(mbar)),
                 "r"(bytes)
                 : "memory");
}
// Box of a 3-D / 2-D tensor map (coordinates innermost first) into shared memory, completing on the mbarrier.
__device__ __forceinline__ void tma_load3(void *dst, const void *tmap, int x, int y, int z, uint64_t *mbar,
                                          uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(tc::smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(tc::smem_addr(mbar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load2(void *dst, const void *tmap, int x, int y, uint64_t *mbar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(tc::smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(tc::smem_addr(mbar)), "l"(pol)
        : "memory");
}
// Contiguous bytes (16-byte aligned, a multiple of 16) into shared memory, completing on the mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *mbar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            tc::smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_addr(mbar)), "l"(pol)
        : "memory");
}

template <int VB>
__device__ __forceinline__ uint4 lds_vec(const uint8_t *p) {
    if (VB == 16) return *reinterpret_cast<const uint4 *>(p);
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    return make_uint4(v.x, v.y, 0u, 0u);
}

// x[0..7] are this lane's partial sums for rows 0..7; lanes v = 0..7 (low three lane bits) end with the full sum of
// row v.
__device__ __forceinline__ float reduce_scatter8(const float (&x)[8], int v) {
    float y[4], z[2];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float send = (v & 4) ? x[i] : x[i + 4], keep = (v & 4) ? x[i + 4] : x[i];
        y[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float send = (v & 2) ? y[i] : y[i + 2], keep = (v & 2) ? y[i + 2] : y[i];
        z[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    const float send = (v & 1) ? z[0] : z[1], keep = (v & 1) ? z[1] : z[0];
    return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

}  // namespace tcu
