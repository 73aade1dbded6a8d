// Few-row attention over one layer's stored keys/values that allocates no device memory at call time, for
// callers that cannot call cudaMalloc: code that runs while a CUDA graph is being captured (an allocation would
// break the capture), hosts whose device memory is owned by a fixed arena or another runtime's allocator, and
// real-time paths where an allocation's latency or its chance of failing is not acceptable. Its scratch - the
// work list and the per-item partial softmax states - lives in one file-scope device array instead.
#include "../../include/tabicl_b200.h"
#include "kernels.cuh"

#include <atomic>
#include <cstdio>

namespace tcu {

// The scratch: TCU_NOALLOC_SCRATCH_BYTES (16 MiB) of global memory in every context that loads this library,
// held until the process exits. Every call shares it and it keeps the last call's contents; each call writes
// every entry it reads before reading it, so nothing has to start at zero.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TCU_NOALLOC_SCRATCH_BYTES];

// The work list of the decode kernel, (chunk, first key) per item, made on the device into the scratch.
__global__ void k_fill_items(int2 *items, int rows, int chunk, int ks, int per_chunk) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_chunks = (rows + chunk - 1) / chunk;
    if (i >= n_chunks * per_chunk) return;
    const int ci = i / per_chunk, k0 = (i % per_chunk) * ks;
    items[i] = make_int2(ci, k0);
}

// The scratch's device address, looked up once per device with that device current (a host-side name for a
// __device__ array is only a stand-in, never a device address).
static std::atomic<void *> g_scratch_addr[64];

static int scratch_address(void **out, char *err, size_t cap) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        if (err && cap) snprintf(err, cap, "attend_noalloc: no current CUDA device (%s)", cudaGetErrorString(e));
        return TCU_ERR_CUDA;
    }
    void *p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            if (err && cap) snprintf(err, cap, "attend_noalloc: cannot find the scratch on device %d (%s)", dev, cudaGetErrorString(e));
            return TCU_ERR_CUDA;
        }
        g_scratch_addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return TCU_OK;
}

}  // namespace tcu

using namespace tcu;

extern "C" int tcu_attend_noalloc(int kv, int d, int heads, const void *layer, int rows, int chunk, const float *q,
                                  int nq, float *out, void *stream, char *err, size_t err_cap) {
    auto bad = [&](const char *msg) {
        if (err && err_cap) snprintf(err, err_cap, "attend_noalloc: %s", msg);
        return TCU_ERR_ARG;
    };
    if (kv < 0 || kv > 2) return bad("kv must be 0 (f32), 1 (i16) or 2 (i8)");
    if (d <= 0 || heads <= 0 || d % heads || d % 4) return bad("d must be a positive multiple of 4 and of heads");
    const int hd = d / heads;
    if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128) return bad("head width must be 8, 16, 32, 64 or 128");
    if (rows < 1 || chunk < 1) return bad("rows and chunk must be at least 1");
    if (nq < 1 || nq > TCU_NOALLOC_MAX_ROWS) return bad("query rows must be 1..32");
    if (!layer || !q || !out) return bad("null pointer");
    // chunk records are read through float pointers (their scales) and so are the queries and outputs: a
    // misaligned pointer would fault the context instead of being refused
    if (((uintptr_t)layer | (uintptr_t)q | (uintptr_t)out) & 3) return bad("layer, q and out must be 4-byte aligned");
    // the scratch holds the work list and, per item and query row, (max, sum) per head plus d weighted values
    const int ks = decode_keys_per_item(kv);
    const int per_chunk = (chunk + ks - 1) / ks;
    const long long n_chunks = (rows + (long long)chunk - 1) / chunk;
    const long long nitems_full = n_chunks * per_chunk;
    if (nitems_full > TCU_NOALLOC_MAX_ITEMS) return bad("more than 8192 key slices (about 500,000 cached rows); use tcu_attend_device");
    const size_t items_bytes = ((size_t)nitems_full * sizeof(int2) + 255) / 256 * 256;
    const size_t ms_bytes = ((size_t)nitems_full * nq * heads * 2 * sizeof(float) + 255) / 256 * 256;
    const size_t acc_bytes = (size_t)nitems_full * nq * d * sizeof(float);
    if (items_bytes + ms_bytes + acc_bytes > (size_t)TCU_NOALLOC_SCRATCH_BYTES) {
        if (err && err_cap)
            snprintf(err, err_cap, "attend_noalloc: %zu bytes of scratch needed for %d query rows over %d cached rows, "
                                   "more than the %d available; use tcu_attend_device", items_bytes + ms_bytes + acc_bytes,
                     nq, rows, TCU_NOALLOC_SCRATCH_BYTES);
        return TCU_ERR_ARG;
    }
    void *base = nullptr;
    int r = scratch_address(&base, err, err_cap);
    if (r != TCU_OK) return r;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *sp = reinterpret_cast<uint8_t *>(base);
    int2 *items = reinterpret_cast<int2 *>(sp);
    // items past a ragged last chunk's keys would read outside the chunk: the list covers only real slices, and
    // the ragged chunk's missing slices are dropped by counting exactly
    const int last_rc = (int)(rows - (n_chunks - 1) * chunk);
    const int last_items = (last_rc + ks - 1) / ks;
    const int nitems = (int)((n_chunks - 1) * per_chunk + last_items);
    k_fill_items<<<(unsigned)((nitems_full + 255) / 256), 256, 0, s>>>(items, rows, chunk, ks, per_chunk);
    cudaError_t e = cudaGetLastError();
    AttnArgs a;
    a.layer = reinterpret_cast<const uint8_t *>(layer), a.rows = rows, a.chunk = chunk, a.d = d, a.heads = heads;
    a.full = record_bytes(kv, d, chunk);
    a.items = items, a.nitems = nitems;
    a.q = q, a.ldq = d, a.R = nq, a.out = out, a.ldo = d;
    a.part_ms = reinterpret_cast<float *>(sp + items_bytes);
    a.part_acc = reinterpret_cast<float *>(sp + items_bytes + ms_bytes);
    if (e == cudaSuccess) e = launch_attend_decode(kv, hd, a, s, nullptr);
    if (e != cudaSuccess) {
        if (err && err_cap) snprintf(err, err_cap, "attend_noalloc: launch failed (%s)", cudaGetErrorString(e));
        return TCU_ERR_CUDA;
    }
    return TCU_OK;
}
