// The sharded stage's exchanges over NVLink without a collective library: each rank stores its data straight into
// its peers' memory (plain peer stores through CUDA IPC mappings; no multicast), then raises a flag in the peer's
// memory; the receiver waits for every rank's flag (a bounded wait) before the kernels that read the data.
#include <cstdint>

#include "kernels.cuh"

namespace tcu {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Block (b, j): its share of every segment for destination rank j, 16-byte pieces, then the flag once all of j's
// blocks are done (the last to arrive raises it).
__global__ void __launch_bounds__(256) k_push(PushArgs a) {
    const int j = blockIdx.y, nb = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
    uint8_t *dst = a.peer[j];
    for (int sg = 0; sg < a.segments; sg++) {
        const float4 *src = reinterpret_cast<const float4 *>(a.src[sg] + (size_t)j * a.src_step[sg]);
        float4 *out = reinterpret_cast<float4 *>(dst + a.dst_off[sg]);
        const size_t n4 = a.count[sg] / 4;
        for (size_t i = (size_t)b * blockDim.x + tid; i < n4; i += (size_t)nb * blockDim.x) out[i] = src[i];
        if (b == 0 && tid < (int)(a.count[sg] % 4))  // a count that is not a multiple of four: its last values
            reinterpret_cast<float *>(out)[4 * n4 + tid] = reinterpret_cast<const float *>(src)[4 * n4 + tid];
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.done + j, 1u);
        if (prev == (unsigned)nb - 1) {
            a.done[j] = 0;  // ready for the next push
            __threadfence_system();
            st_release_sys(reinterpret_cast<unsigned *>(dst + a.flag_off) + a.me, a.epoch);
        }
    }
}

// One thread: every rank's flag in this rank's memory has reached `epoch`; gives up after max_cycles (storing 1 into
// the report slot: the data that follows is not valid).
__global__ void k_wait_flags(const unsigned *flags, int n, unsigned epoch, long long max_cycles, int *err) {
    const long long t0 = clock64();
    for (int s = 0; s < n; s++) {
        while ((int)(ld_acquire_sys(flags + s) - epoch) < 0) {
            if (clock64() - t0 > max_cycles) {
                if (err) *reinterpret_cast<volatile int *>(err) = 1;
                return;
            }
            __nanosleep(64);
        }
    }
    __threadfence_system();
}

}  // namespace

cudaError_t launch_push(const PushArgs &a, int blocks_per_dest, cudaStream_t s, uint64_t *launches) {
    if (a.ranks <= 0 || a.ranks > PUSH_MAX_RANKS) return cudaErrorInvalidValue;
    for (int sg = 0; sg < a.segments; sg++)
        if (a.dst_off[sg] % 16 || reinterpret_cast<uintptr_t>(a.src[sg]) % 16 || a.src_step[sg] % 4)
            return cudaErrorInvalidValue;
    k_push<<<dim3(blocks_per_dest, a.ranks), 256, 0, s>>>(a);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_wait_flags(const unsigned *flags, int n, unsigned epoch, long long max_cycles, int *err,
                              cudaStream_t s, uint64_t *launches) {
    k_wait_flags<<<1, 1, 0, s>>>(flags, n, epoch, max_cycles, err);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
