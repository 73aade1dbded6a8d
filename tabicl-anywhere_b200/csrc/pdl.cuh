// Programmatic dependent launch: a kernel of the stage may be launched while the kernel before it on the stream is
// still running, so that its launch, its prologue (tensor-memory allocation, barrier set-up) and its loads of data
// no kernel writes (weights, a resident cache) overlap the other's tail.
//
// The rules every kernel launched this way keeps:
//  * pdl_wait() before it reads anything an earlier kernel of the stream writes and before it writes any global
//    memory (it returns once the kernel before has completed and its writes are visible; that kernel waited for the
//    one before it, and so on);
//  * pdl_trigger() once every resource the kernel will wait for is held (after its tensor-memory allocation), so a
//    later kernel's blocks never hold tensor memory that one of this kernel's blocks still has to allocate.
// Both are no-ops in a kernel launched the ordinary way. TCU_PDL=0 launches every kernel the ordinary way.
#pragma once
#include <cstdlib>
#include <cuda_runtime.h>

namespace tcu {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// kernel<<<grid, block, smem, s>>>(args...), allowed to overlap the kernel before it on s.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at, cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace tcu
