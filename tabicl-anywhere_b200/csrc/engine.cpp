// Host side of the B200 backend: the context, the in-context weights on the device, resident caches, the stage
// and attention drivers (the AttendCached hook, src/predict.rs:63-79 of tabicl-anywhere), fitting's in-context
// stage on the device, and the C ABI of include/tabicl_b200.h.
#include "../../include/tabicl_b200.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>

#include <cmath>
#include <cstdlib>
#include <algorithm>
#include <array>
#include <atomic>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "engine.hpp"
#include "tirs.hpp"

namespace tcu {

#define CU(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) throw Error{e_ == cudaErrorMemoryAllocation ? TCU_ERR_MEMORY : TCU_ERR_CUDA, \
                                           std::string(#call) + ": " + cudaGetErrorString(e_)};      \
    } while (0)

static void fail(int code, const std::string &m) { throw Error{code, m}; }

// Device memory owned by a handle.
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr, bytes = 0;
    }
    // grow to at least n bytes; true when the buffer moved (its old contents and address are gone)
    bool ensure(size_t n) {
        if (n <= bytes) return false;
        release();
        CU(cudaMalloc(&p, n));
        bytes = n;
        return true;
    }
    template <typename T>
    T *as() const {
        return reinterpret_cast<T *>(p);
    }
};

}  // namespace tcu

using namespace tcu;

struct tcu_ctx {
    std::atomic<int> refs{1};  // the caller's handle plus one per live weights object
    int device = 0;
    int sms = 148;
    int coop = 0;          // cooperative launches supported
    size_t smem_optin = 0; // dynamic shared memory a CTA may opt in to
    cudaStream_t stream = nullptr;
    std::string err;
    std::recursive_mutex mu;
    uint64_t launches = 0;
    // optional event timing of the attention launches (tcu_profile): pairs of events, read after the fact
    bool prof = false;
    std::vector<cudaEvent_t> prof_events;
    size_t prof_used = 0;
    // Report slots of kernels that gave up a bounded wait, in pinned host memory mapped into the device (kernels
    // store 1 into their slot; the host reads them without synchronising): ERR_SLOTS ints, see err_slot_names.
    int *err_host = nullptr;
    int *err_mapped = nullptr;     // the same slots' device address
    bool abort_next = false;       // test hook: the next one-kernel stage launch starts aborted
    unsigned *dev_scan = nullptr;  // scratch of the per-layer magnitude scan
    // uploads from bundles: two pinned staging buffers and a stream of their own (a piece is read from the source
    // while the one before is copied), used by one upload at a time and not under `mu`
    std::mutex upload_mu;
    cudaStream_t upload_stream = nullptr;
    void *pin[2] = {nullptr, nullptr};
    cudaEvent_t pin_ev[2] = {nullptr, nullptr};
};

// Which wait each report slot stands for.
enum { ERR_ATTEND_TC = 0, ERR_GEMM_TC = 1, ERR_QMLP_TC = 2, ERR_ROWS = 3, ERR_PEER = 6, ERR_SLOTS = 8 };
static const char *const err_slot_names[7] = {
    "tensor-core attention (matrix-unit or copy wait)", "tensor-core linear layer (matrix-unit or copy wait)",
    "tensor-core query MLP (matrix-unit wait)", "one-kernel stage (grid barrier)", "one-kernel stage (key tile copy)",
    "one-kernel stage (left after another CTA gave up)", "cross-device exchange (a peer's data never arrived)"};

// A weight matrix [N][K] split once for the tensor cores: f16 hi + lo (bit patterns) of W * 2^e(n) in 128 x 64
// blocks (tc_block_off), and 2^-e(n). No blocks when K is not a multiple of 64.
struct SplitW {
    const uint16_t *tiles = nullptr;
    const float *unscale = nullptr;
};

// Device pointers of one in-context block (src/model.rs:27-98), plus what fitting adds.
struct LayerPtrs {
    const float *n1w, *n1b, *wq, *bq, *q0w, *q0b, *q2w, *q2b, *wo, *bo, *n2w, *n2b, *w1, *b1, *w2, *b2;
    const float *wkv, *bkv;  // fit only: in_proj rows d..3d
    SplitW tq, to, t1, t2, tkv, tq0, tq2;  // tq0 / tq2: the query MLP (hid x hd, hd x hid)
};

// One pre-norm block of the column or row stage on the device (src/model.rs:27-98): in_proj's query rows (column
// blocks) or all three projections (row blocks), no scalable softmax.
struct CBlockPtrs {
    const float *n1w, *n1b, *inw, *inb, *ow, *ob, *n2w, *n2b, *w1, *b1, *w2, *b2;
    SplitW tin, to, t1, t2;
    int ff;
};

// A column block's first attention for fitting (multihead_attn1): on the device its LayerNorm, key/value rows of
// in_proj, out-projection and feed-forward (`b`, `b.inw` [2e][e]) and the inducing points; on the host what the
// inducing points' queries need (the query rows of in_proj and the scalable softmax's MLPs).
struct Isab1 {
    CBlockPtrs b;
    const float *ind = nullptr;      // [inds][e]
    const float *kv2w = nullptr, *kv2b = nullptr;  // the second attention's key/value rows of in_proj [2e][e]
    SplitW tkv2;
    std::vector<float> n1w, n1b, wq, bq, q0w, q0b, q2w, q2b, sb0w, sb0b, sb2w, sb2b, ind_h;
    int hid = 0;
};

// The column and row stages' weights (src/model.rs:199-245), when the bundle has them.
struct RowsWeights {
    bool on = false;
    tcu_rows_shape shape{};
    const float *in_w = nullptr, *in_b = nullptr, *cls_tokens = nullptr, *out_lnw = nullptr, *out_lnb = nullptr;
    std::vector<float> rope_freqs;  // host copy: the position tables are made per token count
    std::vector<CBlockPtrs> col, row;
    // fitting (weights made for_fit with the column stage's first attention present)
    bool fit = false;
    std::vector<Isab1> col1;
    const float *col_y = nullptr;  // the label's embedding table (model.rs:163-177)
    int max_classes = 0;
    DevBuf dev, dev16;
};

struct tcu_weights {
    std::atomic<int> refs{1};  // the caller's handle plus one per live model
    tcu_ctx *ctx = nullptr;
    tcu_icl_shape shape{};
    bool for_fit = false;
    std::map<std::string, std::vector<float>> host;  // as put, widened to f32
    DevBuf dev, dev16;
    std::vector<LayerPtrs> layer;
    const float *lnw = nullptr, *lnb = nullptr, *dec0w = nullptr, *dec0b = nullptr, *dec2w = nullptr, *dec2b = nullptr;
    SplitW tdec0, tdec2;
    const float *icl_y = nullptr;  // fit: class table (model.rs:163-177)
    bool ready = false;
    // fit-time query scale pieces (the base MLP of the scalable softmax), kept on the host: nn.rs:97-107
    std::vector<std::vector<float>> sb0w, sb0b, sb2w, sb2b;
    RowsWeights rows;
};

struct tcu_model {
    tcu_weights *w = nullptr;
    int rows = 0, chunk = 0, kv = 0, classes = 0, features = 0, digits = 1, nodes = 1;
    DevBuf col_kv;  // the column stage's cache [features][digits][blocks][2][e][inds] (fit.rs:230)
    // the column and row stages' working memory: cells (and the digits' sum), projections, attention, hidden,
    // tokens, the row stage's projections and key workspace, the position tables of the last token count
    DevBuf cin, cx, cx0, csum, cq, catt, cmid, ctok, cqkv, ckt, cnew, crope;
    int crope_T = -1;
    size_t full = 0, layer_bytes = 0, layer_stride = 0;
    DevBuf layers, scales, items, tiles;
    int nitems = 0, ntiles = 0;
    std::vector<bool> have_layer;
    bool have_scales = false;
    // tensor-core attention: per layer, power-of-two scalings that keep keys and values inside f16
    std::vector<int> tc_eK, tc_eV;
    bool tc_scanned = false;
    DevBuf tctiles;  // every layer's keys and values as pre-split tensor-core tiles (head width 128)
    // working memory, grown to the largest call so far
    // ssm: the query MLP's hidden units and outputs; atiles: rows split for the tensor cores; mcnt: per (128-row
    // block, head) arrival counters of the tensor-core attention's splits, zero between launches
    DevBuf h, q, att, mid, stats, out, part_ms, part_acc, ssm, atiles, mcnt;
    DevBuf sh_m, sh_mall, sh_packed;  // the cross-device merge: local maxima, their maximum, (values, weight sums)
    // the one-kernel few-row stage: key tiles (head-major), per-layer pointer table, barrier words, partials
    DevBuf rtiles, rlayers, rsync, rparts_ms, rparts_acc, rtmaps;
    int rtiles_n = 0, rtiles_per_head = 0;
    bool rows_built = false;
    struct RowsPlan {
        bool done = false;
        int grid = 0, slots = 0;
        size_t smem = 0;
    } rows_plans[2];  // one row, 2..8 rows
    // the stage captured as CUDA graphs, one per (rows, outputs, profiling), over the buffers above
    struct Graph {
        int R, out_n;
        bool prof;
        cudaGraphExec_t exec;
        uint64_t launches;  // kernels one replay runs
        size_t prof_events; // timing events it records (from index 0 of the context's events), when profiling
    };
    std::vector<Graph> graphs;
    ~tcu_model() {
        for (auto &g : graphs) cudaGraphExecDestroy(g.exec);
    }
};

// NCCL, loaded when the first communicator is made (the library does not link it).
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*reduce_scatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    std::string why;
};
static const NcclApi &nccl_api() {
    static const NcclApi api = [] {
        NcclApi a;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
            return a;
        }
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(dlsym(h, "ncclCommAbort"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        a.send = reinterpret_cast<decltype(a.send)>(dlsym(h, "ncclSend"));
        a.recv = reinterpret_cast<decltype(a.recv)>(dlsym(h, "ncclRecv"));
        a.group_start = reinterpret_cast<decltype(a.group_start)>(dlsym(h, "ncclGroupStart"));
        a.group_end = reinterpret_cast<decltype(a.group_end)>(dlsym(h, "ncclGroupEnd"));
        a.reduce_scatter = reinterpret_cast<decltype(a.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.comm_abort || !a.all_reduce || !a.error_string ||
            !a.send || !a.recv || !a.group_start || !a.group_end || !a.reduce_scatter || !a.all_gather)
            a.why = "libnccl.so.2 lacks an entry point";
        return a;
    }();
    return api;
}

struct tcu_comm {
    tcu_ctx *ctx = nullptr;
    ncclComm_t comm = nullptr;
    int nranks = 1, rank = 0;
    bool aborted = false;
    // optional timing of the sharded stage's phases (tcu_comm_breakdown): an event at the start of each phase,
    // read after the call
    bool prof = false;
    std::vector<cudaEvent_t> events;
    std::vector<int> marks;  // the phase each recorded event starts
    // the sharded stage's collectives run on a stream of their own, ordered against the compute stream by events
    cudaStream_t cstream = nullptr;
    cudaEvent_t sync[10] = {};
    // exchanges by peer stores: this rank's exchange buffer (mapped by every peer through CUDA IPC) and the peers'
    // buffers mapped here; per exchange kind an epoch that every rank advances in step
    int p2p = -1;  // -1 not tried yet, 0 not available (every rank agreed), 1 set up
    void *pbuf = nullptr;
    size_t pbytes = 0;
    std::vector<void *> ppeer;
    unsigned *pdone = nullptr;
    unsigned epoch_q = 0, epoch_s = 0;
};

// ---- handle lifetimes: a context lives while its weights do, weights while their models do --------------------

static void ctx_release(tcu_ctx *ctx) {
    if (--ctx->refs > 0) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    for (auto e : ctx->prof_events) cudaEventDestroy(e);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    if (ctx->dev_scan) cudaFree(ctx->dev_scan);
    for (int i = 0; i < 2; i++) {
        if (ctx->pin[i]) cudaFreeHost(ctx->pin[i]);
        if (ctx->pin_ev[i]) cudaEventDestroy(ctx->pin_ev[i]);
    }
    if (ctx->upload_stream) cudaStreamDestroy(ctx->upload_stream);
    delete ctx;
}

static void weights_release(tcu_weights *w) {
    if (--w->refs > 0) return;
    tcu_ctx *ctx = w->ctx;
    {
        std::lock_guard<std::recursive_mutex> lock(ctx->mu);
        cudaSetDevice(ctx->device);
        delete w;
    }
    ctx_release(ctx);
}

struct ModelDel {
    void operator()(tcu_model *m) const {
        tcu_weights *w = m->w;
        delete m;
        if (w) weights_release(w);
    }
};
using ModelPtr = std::unique_ptr<tcu_model, ModelDel>;
struct WeightsDel {
    void operator()(tcu_weights *w) const { weights_release(w); }
};
using WeightsPtr = std::unique_ptr<tcu_weights, WeightsDel>;

namespace tcu {

static int status_of(tcu_ctx *ctx, const Error &e) {
    if (ctx) ctx->err = e.msg;
    return e.code;
}

template <typename F>
static int guarded(tcu_ctx *ctx, F f) {
    if (!ctx) return TCU_ERR_ARG;
    std::lock_guard<std::recursive_mutex> lock(ctx->mu);
    try {
        CU(cudaSetDevice(ctx->device));
        int r = f();
        return r;
    } catch (const Error &e) {
        return status_of(ctx, e);
    } catch (const BundleError &e) {
        ctx->err = e.what();
        return e.code;
    } catch (const std::bad_alloc &) {
        ctx->err = "host memory exhausted";
        return TCU_ERR_MEMORY;
    } catch (const std::exception &e) {
        ctx->err = e.what();
        return TCU_ERR_ARG;
    }
}

// ---- host restatement of the fit-time query scale (nn.rs:97-107), with the reference's own formulas --------

static float h_exp1(float x) {
    x = x < -87.0f ? -87.0f : (x > 88.0f ? 88.0f : x);
    volatile float t = x * 1.44269504088896340736f;  // keep the multiply and add unfused, as the reference does
    float n = std::floor(t + 0.5f);
    volatile float a = n * 0.6933594f;
    volatile float b = n * -2.1219444e-4f;
    float r = (x - a) - b;
    float p = 1.0f / 5040.0f;
    p = p * r + 1.0f / 720.0f;
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    uint32_t bits = ((uint32_t)((int32_t)n + 127)) << 23;
    float sc;
    std::memcpy(&sc, &bits, 4);
    return p * sc;
}
static float h_erf1(float x) {
    float a = std::fabs(x);
    float t = 1.0f / (1.0f + 0.3275911f * a);
    float p = 1.0614054f;
    p = p * t - 1.4531521f;
    p = p * t + 1.4214138f;
    p = p * t - 0.28449674f;
    p = p * t + 0.2548296f;
    float far = std::copysign(1.0f - p * t * h_exp1(-a * a), x);
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
static float h_gelu(float v) { return 0.5f * v * (1.0f + h_erf1(v * 0.70710678118654752440f)); }

static float h_tanh1(float x) {  // kern.rs:292-297
    const float e = h_exp1(2.0f * (x < -10.0f ? -10.0f : (x > 10.0f ? 10.0f : x)));
    return (e - 1.0f) / (e + 1.0f);
}

// kern.rs:42-61 dot: four running sums of fused products, then the remainder
static float h_dot(const float *a, const float *b, int n) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
        s0 = std::fma(a[i], b[i], s0);
        s1 = std::fma(a[i + 1], b[i + 1], s1);
        s2 = std::fma(a[i + 2], b[i + 2], s2);
        s3 = std::fma(a[i + 3], b[i + 3], s3);
    }
    float s = (s0 + s1) + (s2 + s3);
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

// kern.rs:154-159 linear, y = w x + b with w [out][in]
static void h_linear(const float *w, const float *b, const float *x, int in, int out, float *y) {
    for (int o = 0; o < out; o++) y[o] = h_dot(w + (size_t)o * in, x, in) + (b ? b[o] : 0.f);
}

// kern.rs:357-376 layer norm: eps 1e-5, biased variance
static void h_layer_norm(const float *x, const float *w, const float *b, int n, float *y) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += x[i];
    const float mean = s / (float)n;
    float q = 0.f;
    for (int i = 0; i < n; i++) q = std::fma(x[i] - mean, x[i] - mean, q);
    const float inv = 1.0f / std::sqrt(q / (float)n + 1e-5f);
    for (int i = 0; i < n; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}

static std::vector<float> query_scale(const tcu_weights *w, int l, int n) {
    const int d = w->shape.d, hd = d / w->shape.heads;
    const auto &b0w = w->sb0w[l], &b0b = w->sb0b[l], &b2w = w->sb2w[l], &b2b = w->sb2b[l];
    const int hid = (int)b0b.size();
    float inv = 1.0f / std::sqrt((float)hd);
    float logn = std::log((float)(n > 1 ? n : 1));
    std::vector<float> h(hid), out(d);
    for (int i = 0; i < hid; i++) h[i] = h_gelu(b0w[i] * logn + b0b[i]);
    for (int o = 0; o < d; o++) {
        // kern.rs:42-61 dot: four running sums of fused products, then the remainder
        const float *w = b2w.data() + (size_t)o * hid;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        int i = 0;
        for (; i + 4 <= hid; i += 4) {
            s0 = std::fma(w[i], h[i], s0);
            s1 = std::fma(w[i + 1], h[i + 1], s1);
            s2 = std::fma(w[i + 2], h[i + 2], s2);
            s3 = std::fma(w[i + 3], h[i + 3], s3);
        }
        float s = (s0 + s1) + (s2 + s3);
        for (; i < hid; i++) s += w[i] * h[i];
        out[o] = (s + b2b[o]) * inv;
    }
    return out;
}

// ---- weights ---------------------------------------------------------------------------------------------------

static std::string blk(int l, const char *name) { return "icl_predictor.tf_icl.blocks." + std::to_string(l) + "." + name; }

static const std::vector<float> &need(const tcu_weights *w, const std::string &name, size_t count) {
    auto it = w->host.find(name);
    if (it == w->host.end()) fail(TCU_ERR_STATE, "weights: tensor " + name + " was never put");
    if (it->second.size() != count)
        fail(TCU_ERR_FORMAT, "weights: " + name + " has " + std::to_string(it->second.size()) + " values, expected " + std::to_string(count));
    return it->second;
}

static std::vector<float> opt_zero(const tcu_weights *w, const std::string &name, size_t count) {
    auto it = w->host.find(name);
    if (it == w->host.end()) return std::vector<float>(count, 0.f);  // a layer norm trained without bias
    if (it->second.size() != count) fail(TCU_ERR_FORMAT, "weights: " + name + " has the wrong length");
    return it->second;
}

// Weights gathered for one upload: every tensor in device order, each 256-byte aligned (`flat`), and the f16 hi + lo
// copies of the matrices the tensor cores take (`half`): W * 2^e(n) per output row n, in 128 x 64 blocks
// (tc_block_off), rows past N zero; 2^-e(n) beside it in `flat`. No blocks when K is not a multiple of 64.
struct Packer {
    std::vector<float> flat;
    std::vector<uint16_t> half;
    std::vector<size_t> offs;
    struct SplitIdx {
        size_t tiles = 0, unscale = 0;
        bool on = false;
    };
    size_t add(const std::vector<float> &v) {
        size_t at = (flat.size() + 63) / 64 * 64;
        flat.resize(at + v.size());
        std::memcpy(flat.data() + at, v.data(), v.size() * sizeof(float));
        offs.push_back(at);
        return offs.size() - 1;
    }
    const float *host(size_t idx) const { return flat.data() + offs[idx]; }
    SplitIdx split(size_t idx, int N, int K) {
        SplitIdx ix;
        ix.on = K % 64 == 0;
        if (!ix.on) return ix;
        const std::vector<float> src(host(idx), host(idx) + (size_t)N * K);  // add() below may move `flat`
        const int nts = (N + 127) / 128, nk = K / 64;
        const size_t blk = 128 * 64;
        ix.tiles = (half.size() + 127) / 128 * 128;
        half.resize(ix.tiles + (size_t)nts * nk * 2 * blk, 0);
        std::vector<float> un(N);
        for (int n = 0; n < N; n++) {
            const float *row = src.data() + (size_t)n * K;
            float mx = 0.f;
            for (int k = 0; k < K; k++) mx = std::max(mx, std::fabs(row[k]));
            const int e = tc_exponent(mx);
            const float sc = std::ldexp(1.0f, e);
            un[n] = std::ldexp(1.0f, -e);
            for (int k = 0; k < K; k++) {
                const float x = row[k] * sc;  // exact: a power of two
                const uint16_t h = f32_to_f16(x);
                uint16_t *b = half.data() + ix.tiles + ((size_t)(n / 128) * nk + k / 64) * 2 * blk;
                const size_t off = tc_block_off(n, k);
                b[off] = h;
                b[blk + off] = f32_to_f16(x - f16_to_f32(h));
            }
        }
        ix.unscale = add(un);
        return ix;
    }
    // copy both to the device; the pointer of an added tensor is then P(idx), of a split matrix S(ix)
    void upload(DevBuf &dev, DevBuf &dev16) {
        dev.ensure(flat.size() * sizeof(float));
        CU(cudaMemcpy(dev.p, flat.data(), flat.size() * sizeof(float), cudaMemcpyHostToDevice));
        dev16.ensure(std::max<size_t>(half.size(), 1) * sizeof(uint16_t));
        if (!half.empty()) CU(cudaMemcpy(dev16.p, half.data(), half.size() * sizeof(uint16_t), cudaMemcpyHostToDevice));
        base = dev.as<float>(), hbase = dev16.as<uint16_t>();
    }
    const float *base = nullptr;
    const uint16_t *hbase = nullptr;
    const float *P(size_t idx) const { return base + offs[idx]; }
    SplitW S(const SplitIdx &ix) const { return ix.on ? SplitW{hbase + ix.tiles, base + offs[ix.unscale]} : SplitW(); }
};

static int rows_ready(tcu_weights *w);

static int weights_ready(tcu_weights *w) {
    const auto &s = w->shape;
    const int d = s.d, L = s.layers, ff = s.ff, hid = s.hid, hd = d / s.heads, dff = s.dec_ff, outs = s.outs;
    Packer pk;
    auto add = [&](const std::vector<float> &v) { return pk.add(v); };
    struct LIdx {
        size_t n1w, n1b, wq, bq, q0w, q0b, q2w, q2b, wo, bo, n2w, n2b, w1, b1, w2, b2, wkv, bkv;
    };
    std::vector<LIdx> li(L);
    w->sb0w.assign(L, {}), w->sb0b.assign(L, {}), w->sb2w.assign(L, {}), w->sb2b.assign(L, {});
    for (int l = 0; l < L; l++) {
        const auto &inw = need(w, blk(l, "attn.in_proj_weight"), (size_t)3 * d * d);
        const auto &inb = need(w, blk(l, "attn.in_proj_bias"), (size_t)3 * d);
        LIdx &x = li[l];
        x.n1w = add(need(w, blk(l, "norm1.weight"), d));
        x.n1b = add(opt_zero(w, blk(l, "norm1.bias"), d));
        x.wq = add(std::vector<float>(inw.begin(), inw.begin() + (size_t)d * d));
        x.bq = add(std::vector<float>(inb.begin(), inb.begin() + d));
        x.q0w = add(need(w, blk(l, "attn.ssmax_layer.query_mlp.0.weight"), (size_t)hid * hd));
        x.q0b = add(need(w, blk(l, "attn.ssmax_layer.query_mlp.0.bias"), hid));
        x.q2w = add(need(w, blk(l, "attn.ssmax_layer.query_mlp.2.weight"), (size_t)hd * hid));
        x.q2b = add(need(w, blk(l, "attn.ssmax_layer.query_mlp.2.bias"), hd));
        x.wo = add(need(w, blk(l, "attn.out_proj.weight"), (size_t)d * d));
        x.bo = add(need(w, blk(l, "attn.out_proj.bias"), d));
        x.n2w = add(need(w, blk(l, "norm2.weight"), d));
        x.n2b = add(opt_zero(w, blk(l, "norm2.bias"), d));
        x.w1 = add(need(w, blk(l, "linear1.weight"), (size_t)ff * d));
        x.b1 = add(need(w, blk(l, "linear1.bias"), ff));
        x.w2 = add(need(w, blk(l, "linear2.weight"), (size_t)d * ff));
        x.b2 = add(need(w, blk(l, "linear2.bias"), d));
        if (w->for_fit) {
            x.wkv = add(std::vector<float>(inw.begin() + (size_t)d * d, inw.end()));
            x.bkv = add(std::vector<float>(inb.begin() + d, inb.end()));
            auto b0b = w->host.find(blk(l, "attn.ssmax_layer.base_mlp.0.bias"));
            if (b0b == w->host.end()) fail(TCU_ERR_STATE, "weights: the scalable softmax's base MLP is needed to fit");
            const size_t bh = b0b->second.size();
            w->sb0w[l] = need(w, blk(l, "attn.ssmax_layer.base_mlp.0.weight"), bh);
            w->sb0b[l] = b0b->second;
            w->sb2w[l] = need(w, blk(l, "attn.ssmax_layer.base_mlp.2.weight"), (size_t)d * bh);
            w->sb2b[l] = need(w, blk(l, "attn.ssmax_layer.base_mlp.2.bias"), d);
        }
    }
    size_t i_lnw = add(need(w, "icl_predictor.ln.weight", d));
    size_t i_lnb = add(opt_zero(w, "icl_predictor.ln.bias", d));
    size_t i_d0w = add(need(w, "icl_predictor.decoder.0.weight", (size_t)dff * d));
    size_t i_d0b = add(need(w, "icl_predictor.decoder.0.bias", dff));
    size_t i_d2w = add(need(w, "icl_predictor.decoder.2.weight", (size_t)outs * dff));
    size_t i_d2b = add(need(w, "icl_predictor.decoder.2.bias", outs));
    size_t i_y = 0;
    if (w->for_fit) {
        // model.rs:163-177 class_table: one embedding row per class, or [weight][bias] for regression
        const int mc = s.max_classes;
        const auto &yw = need(w, "icl_predictor.y_encoder.weight", (size_t)d * (mc > 0 ? mc : 1));
        const auto &yb = need(w, "icl_predictor.y_encoder.bias", d);
        std::vector<float> t;
        if (mc == 0) {
            t = yw;
            t.insert(t.end(), yb.begin(), yb.end());
        } else {
            t.assign((size_t)mc * d, 0.f);
            for (int c = 0; c < mc; c++)
                for (int o = 0; o < d; o++) t[(size_t)c * d + o] = yw[(size_t)o * mc + c] + yb[o];
        }
        i_y = add(t);
    }
    // tensor-core copies of the linear layers' weights: f16 hi + lo per row, scaled to stay inside f16
    using SplitIdx = Packer::SplitIdx;
    std::vector<std::array<SplitIdx, 7>> lsplit(L);
    for (int l = 0; l < L; l++) {
        const LIdx &x = li[l];
        lsplit[l][0] = pk.split(x.wq, d, d);
        lsplit[l][1] = pk.split(x.wo, d, d);
        lsplit[l][2] = pk.split(x.w1, ff, d);
        lsplit[l][3] = pk.split(x.w2, d, ff);
        if (w->for_fit) lsplit[l][4] = pk.split(x.wkv, 2 * d, d);
        lsplit[l][5] = pk.split(x.q0w, hid, hd);
        lsplit[l][6] = pk.split(x.q2w, hd, hid);
    }
    const SplitIdx s_dec0 = pk.split(i_d0w, dff, d);
    const SplitIdx s_dec2 = pk.split(i_d2w, outs, dff);
    pk.upload(w->dev, w->dev16);
    auto P = [&](size_t idx) { return pk.P(idx); };
    auto S = [&](const SplitIdx &ix) { return pk.S(ix); };
    w->layer.resize(L);
    for (int l = 0; l < L; l++) {
        const LIdx &x = li[l];
        LayerPtrs &p = w->layer[l];
        p = LayerPtrs{P(x.n1w), P(x.n1b), P(x.wq), P(x.bq), P(x.q0w), P(x.q0b), P(x.q2w), P(x.q2b), P(x.wo), P(x.bo),
                      P(x.n2w), P(x.n2b), P(x.w1), P(x.b1), P(x.w2), P(x.b2), nullptr, nullptr};
        if (w->for_fit) p.wkv = P(x.wkv), p.bkv = P(x.bkv);
        p.tq = S(lsplit[l][0]), p.to = S(lsplit[l][1]), p.t1 = S(lsplit[l][2]), p.t2 = S(lsplit[l][3]);
        if (w->for_fit) p.tkv = S(lsplit[l][4]);
        p.tq0 = S(lsplit[l][5]), p.tq2 = S(lsplit[l][6]);
    }
    w->lnw = P(i_lnw), w->lnb = P(i_lnb), w->dec0w = P(i_d0w), w->dec0b = P(i_d0b), w->dec2w = P(i_d2w), w->dec2b = P(i_d2b);
    w->tdec0 = S(s_dec0), w->tdec2 = S(s_dec2);
    w->icl_y = w->for_fit ? P(i_y) : nullptr;
    if (w->rows.on) rows_ready(w);
    w->host.clear();
    w->ready = true;
    return TCU_OK;
}

// The column and row stages' tensors (model.rs:199-245; the column blocks' second attention, whose in_proj query
// rows are all prediction uses, model.rs:226-231) to the device, with tensor-core copies of their matrices.
static int rows_ready(tcu_weights *w) {
    RowsWeights &rw = w->rows;
    const auto &s = rw.shape;
    const int e = s.e;
    Packer pk;
    struct BIdx {
        size_t n1w, n1b, inw, inb, ow, ob, n2w, n2b, w1, b1, w2, b2;
        Packer::SplitIdx tin, to, t1, t2;
        int ff;
    };
    // in_proj rows: the query's only (q_only 1), the keys' and values' only (2), or all three (0)
    auto block = [&](const std::string &p, int q_only, int ff) {
        BIdx x;
        const int nin = q_only == 1 ? e : (q_only == 2 ? 2 * e : 3 * e), first = q_only == 2 ? e : 0;
        const auto &inw = need(w, p + "attn.in_proj_weight", (size_t)3 * e * e);
        const auto &inb = need(w, p + "attn.in_proj_bias", (size_t)3 * e);
        x.n1w = pk.add(need(w, p + "norm1.weight", e));
        x.n1b = pk.add(opt_zero(w, p + "norm1.bias", e));
        x.inw = pk.add(std::vector<float>(inw.begin() + (size_t)first * e, inw.begin() + (size_t)(first + nin) * e));
        x.inb = pk.add(std::vector<float>(inb.begin() + first, inb.begin() + first + nin));
        x.ow = pk.add(need(w, p + "attn.out_proj.weight", (size_t)e * e));
        x.ob = pk.add(need(w, p + "attn.out_proj.bias", e));
        x.n2w = pk.add(need(w, p + "norm2.weight", e));
        x.n2b = pk.add(opt_zero(w, p + "norm2.bias", e));
        x.w1 = pk.add(need(w, p + "linear1.weight", (size_t)ff * e));
        x.b1 = pk.add(need(w, p + "linear1.bias", ff));
        x.w2 = pk.add(need(w, p + "linear2.weight", (size_t)e * ff));
        x.b2 = pk.add(need(w, p + "linear2.bias", e));
        x.tin = pk.split(x.inw, nin, e), x.to = pk.split(x.ow, e, e);
        x.t1 = pk.split(x.w1, ff, e), x.t2 = pk.split(x.w2, e, ff);
        x.ff = ff;
        return x;
    };
    std::vector<BIdx> cb, rb, c1, c2kv;
    for (int i = 0; i < s.col_blocks; i++)
        cb.push_back(block("col_embedder.tf_col.blocks." + std::to_string(i) + ".multihead_attn2.", 1, s.col_ff));
    for (int i = 0; i < s.row_blocks; i++)
        rb.push_back(block("row_interactor.tf_row.blocks." + std::to_string(i) + ".", 0, s.row_ff));
    // fitting: the first attention of each column block (its key/value rows on the device, its query on the host),
    // the inducing points, the second attention's key/value rows, and the label's embedding table
    rw.fit = w->for_fit && w->host.count("col_embedder.tf_col.blocks.0.multihead_attn1.attn.in_proj_weight") &&
             w->host.count("col_embedder.y_encoder.weight");
    std::vector<size_t> i_ind;
    size_t i_coly = 0;
    rw.col1.clear();
    if (rw.fit) {
        for (int i = 0; i < s.col_blocks; i++) {
            const std::string p = "col_embedder.tf_col.blocks." + std::to_string(i) + ".";
            c1.push_back(block(p + "multihead_attn1.", 2, s.col_ff));
            c2kv.push_back(block(p + "multihead_attn2.", 2, s.col_ff));
            const auto &ind = need(w, p + "ind_vectors", (size_t)s.inds * e);
            i_ind.push_back(pk.add(ind));
            Isab1 a;
            const std::string q = p + "multihead_attn1.", ss = q + "attn.ssmax_layer.";
            const auto &inw = need(w, q + "attn.in_proj_weight", (size_t)3 * e * e);
            const auto &inb = need(w, q + "attn.in_proj_bias", (size_t)3 * e);
            a.n1w = need(w, q + "norm1.weight", e), a.n1b = opt_zero(w, q + "norm1.bias", e);
            a.wq.assign(inw.begin(), inw.begin() + (size_t)e * e), a.bq.assign(inb.begin(), inb.begin() + e);
            a.sb0b = w->host.at(ss + "base_mlp.0.bias");
            a.hid = (int)a.sb0b.size();
            const int hd = e / s.col_heads;
            a.sb0w = need(w, ss + "base_mlp.0.weight", a.hid), a.sb2w = need(w, ss + "base_mlp.2.weight", (size_t)e * a.hid);
            a.sb2b = need(w, ss + "base_mlp.2.bias", e);
            a.q0w = need(w, ss + "query_mlp.0.weight", (size_t)a.hid * hd), a.q0b = need(w, ss + "query_mlp.0.bias", a.hid);
            a.q2w = need(w, ss + "query_mlp.2.weight", (size_t)hd * a.hid), a.q2b = need(w, ss + "query_mlp.2.bias", hd);
            a.ind_h = ind;
            rw.col1.push_back(std::move(a));
        }
        rw.max_classes = w->shape.max_classes;
        const auto &yw = w->host.at("col_embedder.y_encoder.weight");
        const auto &yb = need(w, "col_embedder.y_encoder.bias", e);
        std::vector<float> table;
        if (rw.max_classes > 0) {
            // model.rs:163-177: a class's row is the one-hot layer's weight column plus its bias
            const int mc = rw.max_classes;
            if (yw.size() != (size_t)e * mc) fail(TCU_ERR_FORMAT, "weights: col_embedder.y_encoder.weight has the wrong length");
            table.resize((size_t)mc * e);
            for (int c = 0; c < mc; c++)
                for (int o = 0; o < e; o++) table[(size_t)c * e + o] = yw[(size_t)o * mc + c] + yb[o];
        } else {
            table = yw;
            table.insert(table.end(), yb.begin(), yb.end());
        }
        i_coly = pk.add(table);
    }
    const size_t i_inw = pk.add(need(w, "col_embedder.in_linear.weight", (size_t)e * s.group));
    const size_t i_inb = pk.add(need(w, "col_embedder.in_linear.bias", e));
    const size_t i_cls = pk.add(need(w, "row_interactor.cls_tokens", (size_t)s.cls * e));
    const size_t i_lnw = pk.add(need(w, "row_interactor.out_ln.weight", e));
    const size_t i_lnb = pk.add(opt_zero(w, "row_interactor.out_ln.bias", e));
    rw.rope_freqs = need(w, "row_interactor.tf_row.rope.freqs", (size_t)e / s.row_heads / 2);
    pk.upload(rw.dev, rw.dev16);
    auto ptrs = [&](const BIdx &x) {
        return CBlockPtrs{pk.P(x.n1w), pk.P(x.n1b), pk.P(x.inw), pk.P(x.inb), pk.P(x.ow), pk.P(x.ob),
                          pk.P(x.n2w), pk.P(x.n2b), pk.P(x.w1), pk.P(x.b1), pk.P(x.w2), pk.P(x.b2),
                          pk.S(x.tin), pk.S(x.to), pk.S(x.t1), pk.S(x.t2), x.ff};
    };
    rw.col.clear(), rw.row.clear();
    for (const auto &x : cb) rw.col.push_back(ptrs(x));
    for (const auto &x : rb) rw.row.push_back(ptrs(x));
    for (size_t i = 0; i < rw.col1.size(); i++) {
        rw.col1[i].b = ptrs(c1[i]);
        rw.col1[i].ind = pk.P(i_ind[i]);
        rw.col1[i].kv2w = pk.P(c2kv[i].inw), rw.col1[i].kv2b = pk.P(c2kv[i].inb), rw.col1[i].tkv2 = pk.S(c2kv[i].tin);
    }
    if (rw.fit) rw.col_y = pk.P(i_coly);
    rw.in_w = pk.P(i_inw), rw.in_b = pk.P(i_inb), rw.cls_tokens = pk.P(i_cls), rw.out_lnw = pk.P(i_lnw), rw.out_lnb = pk.P(i_lnb);
    return TCU_OK;
}

// model.rs:157-161 cfg_value: the text after "key": up to the next comma or brace, quotes trimmed
static std::string cfg_value(const std::string &cfg, const std::string &key) {
    size_t at = cfg.find("\"" + key + "\"");
    if (at == std::string::npos) return "(missing)";
    size_t colon = cfg.find(':', at);
    if (colon == std::string::npos) return "(missing)";
    size_t end = cfg.find_first_of(",}", colon + 1);
    std::string v = cfg.substr(colon + 1, end == std::string::npos ? std::string::npos : end - colon - 1);
    size_t a = v.find_first_not_of(" \t\n\""), b = v.find_last_not_of(" \t\n\"");
    return a == std::string::npos ? "" : v.substr(a, b - a + 1);
}

// ---- resident caches ------------------------------------------------------------------------------------------

static size_t layer_bytes_of(int kv, int d, int rows, int chunk) {
    // fit.rs:234 raw_entries: full chunks, then the remainder's record
    return (size_t)(rows / chunk) * record_bytes(kv, d, chunk) + (rows % chunk ? record_bytes(kv, d, rows % chunk) : 0);
}

static bool tc_enabled();

// Everything a problem of `rows` training rows holds on the device once it has answered a call of each kind: the
// stored records (each layer on a 256-byte boundary), the query scales, the decode items and key tiles, the column
// cache, the tensor-core attention's pre-split keys and values (head width 128) and the one-kernel stage's tables.
static size_t model_bytes_of(const tcu_weights *w, int rows, int chunk, int kv, size_t col_floats) {
    const int d = w->shape.d, L = w->shape.layers, heads = w->shape.heads;
    const size_t stride = (layer_bytes_of(kv, d, rows, chunk) + 255) / 256 * 256;
    const int ks = decode_keys_per_item(kv), tk = rows_tile_keys(kv);
    size_t nitems = 0, ntiles = 0, nrt = 0;
    for (int r0 = 0; r0 < rows; r0 += chunk) {
        const int rc = std::min(chunk, rows - r0);
        nitems += (rc + ks - 1) / ks, ntiles += (rc + FLASH_KEYS - 1) / FLASH_KEYS, nrt += (rc + tk - 1) / tk;
    }
    size_t n = stride * L + sizeof(float) * (size_t)L * d + nitems * sizeof(int2) + ntiles * sizeof(int4) +
               sizeof(float) * col_floats;
    if (d / heads == 128 && tc_enabled()) n += ntiles * heads * tc_tile_bytes() * L;
    n += nrt * heads * sizeof(int4) + 2 * (size_t)L * sizeof(CUtensorMap) + L * sizeof(RowsLayer) + 256;
    return n;
}

static void model_init(tcu_model *m, tcu_weights *w, int rows, int chunk, int kv, int classes) {
    m->w = w;
    w->refs++;  // released by tcu_model_free, or by ModelDel when creation fails
    const int d = w->shape.d, L = w->shape.layers;
    if (rows <= 0 || chunk < 1 || kv < 0 || kv > 2) fail(TCU_ERR_ARG, "cache: bad rows, chunk or kv format");
    m->rows = rows, m->chunk = chunk, m->kv = kv, m->classes = classes;
    m->full = record_bytes(kv, d, chunk);
    m->layer_bytes = layer_bytes_of(kv, d, rows, chunk);
    m->layer_stride = (m->layer_bytes + 255) / 256 * 256;
    m->layers.ensure(m->layer_stride * L);
    m->scales.ensure(sizeof(float) * (size_t)L * d);
    m->have_layer.assign(L, false);
    // decode items and flash tiles: the same for every layer and head
    const int ks = decode_keys_per_item(kv);
    std::vector<int2> items;
    std::vector<int4> tiles;
    for (int ci = 0, r0 = 0; r0 < rows; ci++, r0 += chunk) {
        int rc = std::min(chunk, rows - r0);
        for (int k0 = 0; k0 < rc; k0 += ks) items.push_back(make_int2(ci, k0));
        for (int k0 = 0; k0 < rc; k0 += FLASH_KEYS) tiles.push_back(make_int4(ci, k0, std::min(FLASH_KEYS, rc - k0), 0));
    }
    m->nitems = (int)items.size(), m->ntiles = (int)tiles.size();
    m->items.ensure(items.size() * sizeof(int2));
    m->tiles.ensure(tiles.size() * sizeof(int4));
    CU(cudaMemcpy(m->items.p, items.data(), items.size() * sizeof(int2), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(m->tiles.p, tiles.data(), tiles.size() * sizeof(int4), cudaMemcpyHostToDevice));
}

static const uint8_t *layer_ptr(const tcu_model *m, int l) { return m->layers.as<uint8_t>() + m->layer_stride * (size_t)l; }

static void check_ready(const tcu_model *m) {
    if (!m->w->ready) fail(TCU_ERR_STATE, "weights not ready");
    if (!m->have_scales) fail(TCU_ERR_STATE, "cache: query scales were never put");
    for (size_t l = 0; l < m->have_layer.size(); l++)
        if (!m->have_layer[l]) fail(TCU_ERR_STATE, "cache: layer " + std::to_string(l) + " was never put");
}

// ---- the in-context stage -----------------------------------------------------------------------------------

struct Launch {
    tcu_ctx *ctx;
    cudaStream_t s;
    void operator()(cudaError_t e, const char *what) const {
        if (e != cudaSuccess) fail(TCU_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    }
};

// flash-path splits of the training rows: enough blocks for two per SM, at most 64 parts
static int flash_splits(const tcu_ctx *ctx, int R, int heads, int ntiles) {
    const int blocks = (R + FLASH_ROWS - 1) / FLASH_ROWS * heads;
    int splits = (2 * ctx->sms + blocks - 1) / blocks;
    splits = std::max(1, std::min({splits, ntiles, 64}));
    const int per = (ntiles + splits - 1) / splits;
    return (ntiles + per - 1) / per;
}

// Which attention kernel takes R rows, and in how many parts of the training rows.
enum class Path { Decode, Flash, Tensor };
struct Plan {
    Path path;
    int splits;  // parts (decode: items)
};
static bool tc_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_TENSOR_CORES");
        return !(e && e[0] == '0');
    }();
    return on;
}
static Plan attend_plan(const tcu_ctx *ctx, int R, int heads, int hd, int nitems, int ntiles) {
    // the tensor-core kernel from 9 rows (head width 128); the split-K decode kernel below that, and up to 32 rows
    // at other head widths
    const bool tensor = hd == 128 && tc_enabled();
    if (R <= (tensor ? 8 : 32)) return {Path::Decode, nitems};
    if (tensor) {
        // one block per SM at a time: (128 rows x head) blocks, each over a share of the key tiles; the split count
        // that minimises waves x (tiles per block + a block's fixed cost, about 4 tiles: staging its queries,
        // writing and merging its part); ties: fewer splits
        const int blocks = (R + 127) / 128 * heads;
        int best = 1;
        long long best_cost = -1;
        for (int sp = 1; sp <= std::min(ntiles, 64); sp++) {
            const int per = (ntiles + sp - 1) / sp, used = (ntiles + per - 1) / per;
            const long long waves = ((long long)blocks * used + ctx->sms - 1) / ctx->sms;
            const long long cost = waves * (per + (used > 1 ? 4 : 0));
            if (best_cost < 0 || cost < best_cost) best_cost = cost, best = used;
        }
        return {Path::Tensor, best};
    }
    return {Path::Flash, flash_splits(ctx, R, heads, ntiles)};
}

static void drop_graphs(tcu_model *m) {
    for (auto &g : m->graphs) cudaGraphExecDestroy(g.exec);
    m->graphs.clear();
}

// Grow the working memory for R rows; captured graphs point into it, so they go when any buffer moves.
static void ensure_work(tcu_model *m, int R) {
    const auto &s = m->w->shape;
    const size_t d = s.d, H = s.heads;
    const size_t wide = (size_t)std::max(s.ff, s.dec_ff);
    bool moved = false;
    moved |= m->q.ensure(sizeof(float) * R * d);
    moved |= m->att.ensure(sizeof(float) * R * d);
    moved |= m->mid.ensure(sizeof(float) * R * wide);
    moved |= m->stats.ensure(sizeof(float) * R * 4 * std::max<size_t>(H, 1));  // per row, or per (row, head)
    if (R > 16) moved |= m->ssm.ensure(sizeof(float) * R * (H * (size_t)s.hid + d));
    if (R > 8) {
        size_t at = tc_split_bytes(R, (int)std::max<size_t>(d, wide));
        if (R > 16) at = std::max(at, tc_split_bytes(R * (int)H, std::max(s.d / s.heads, s.hid)));
        moved |= m->atiles.ensure(at);
    }
    const Plan plan = attend_plan(m->w->ctx, R, s.heads, s.d / s.heads, m->nitems, m->ntiles);
    const size_t pr = plan.path == Path::Decode ? (size_t)m->nitems : (size_t)plan.splits;  // parts, when left
    if (m->mcnt.ensure(sizeof(int) * ((size_t)(R + 127) / 128) * std::max<size_t>(H, 1))) {
        CU(cudaMemset(m->mcnt.p, 0, m->mcnt.bytes));
        moved = true;
    }
    if (pr) {
        moved |= m->part_ms.ensure(sizeof(float) * pr * R * H * 2);
        moved |= m->part_acc.ensure(sizeof(float) * pr * R * d);
    }
    if (moved) drop_graphs(m);
}

// attention of R scaled queries q (device, [R][d]) against a layer given in stored form; out [R][d]
// Returns the number of parts left in part_ms / part_acc when parts_only (the outputs are not finished then). With
// state_ms (and parts_only), the tensor-core path leaves the merged state itself when it can (out the unnormalised
// values, state_ms their (max, weight sum)) and returns 0; otherwise the parts are left as above.
static int attend_layer(tcu_ctx *ctx, tcu_model *m, const uint8_t *layer, int rows, int chunk, int kv, const int2 *items,
                        int nitems, const int4 *tiles, int ntiles, const float *q, int R, float *out, cudaStream_t s,
                        int eK = 0, int eV = 0, bool parts_only = false, const void *tc_tiles = nullptr,
                        float *state_ms = nullptr) {
    const auto &sh = m->w->shape;
    AttnArgs a;
    a.layer = layer, a.rows = rows, a.chunk = chunk, a.d = sh.d, a.heads = sh.heads;
    a.full = record_bytes(kv, sh.d, chunk);
    a.q = q, a.ldq = sh.d, a.R = R, a.out = out, a.ldo = sh.d;
    a.part_ms = m->part_ms.as<float>(), a.part_acc = m->part_acc.as<float>();
    a.parts_only = parts_only ? 1 : 0;
    const int hd = sh.d / sh.heads;
    Launch ck{ctx, s};
    cudaEvent_t ev_end = nullptr;
    unsigned ev_flags = cudaEventRecordDefault;
    if (ctx->prof) {
        if (ctx->prof_used + 2 > ctx->prof_events.size()) {
            for (int i = 0; i < 64; i++) {
                cudaEvent_t e;
                CU(cudaEventCreate(&e));
                ctx->prof_events.push_back(e);
            }
        }
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        CU(cudaStreamIsCapturing(s, &cs));
        ev_flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
        CU(cudaEventRecordWithFlags(ctx->prof_events[ctx->prof_used], s, ev_flags));
        ev_end = ctx->prof_events[ctx->prof_used + 1];
        ctx->prof_used += 2;
    }
    struct End {
        cudaEvent_t e;
        cudaStream_t s;
        unsigned flags;
        ~End() {
            if (e) cudaEventRecordWithFlags(e, s, flags);
        }
    } end_mark{ev_end, s, ev_flags};
    const Plan plan = attend_plan(ctx, R, sh.heads, hd, nitems, ntiles);
    if (plan.path == Path::Decode) {
        a.items = items, a.nitems = nitems;
        ck(launch_attend_decode(kv, hd, a, s, &ctx->launches), "attend (decode)");
        return parts_only ? nitems : 0;
    }
    a.tiles = tiles, a.ntiles = ntiles;
    // a merged state is left by the kernel itself for up to eight splits: keep to eight when one is asked for
    const int splits = state_ms && plan.path == Path::Tensor ? std::min(plan.splits, 8) : plan.splits;
    a.tiles_per_split = (ntiles + splits - 1) / splits;
    a.splits = (ntiles + a.tiles_per_split - 1) / a.tiles_per_split;
    if (plan.path == Path::Tensor) {
        if (!tc_tiles) fail(TCU_ERR_STATE, "attend: tensor-core tiles were not built");
        a.tc_eK = eK, a.tc_eV = eV, a.err = ctx->err_mapped + ERR_ATTEND_TC, a.tc_tiles = tc_tiles;
        // up to eight splits the last split of a (row block, head) merges them inside the kernel; more parts are
        // merged by k_attend_merge, one block per (row, head), instead of by a few CTAs reading them all
        if (a.splits <= 8 && m->mcnt.bytes >= sizeof(int) * ((size_t)(R + 127) / 128) * sh.heads)
            a.merge_cnt = m->mcnt.as<int>();
        const bool state = state_ms && (a.splits == 1 || a.merge_cnt);
        if (state) a.parts_only = 0, a.state_ms = state_ms;
        ck(launch_attend_tc(kv, a, s, &ctx->launches), "attend (tensor cores)");
        if (state) return 0;
    } else {
        ck(launch_attend_flash(kv, hd, a, s, &ctx->launches), "attend (flash)");
    }
    return parts_only ? a.splits : 0;
}

static void linear(tcu_ctx *ctx, tcu_model *m, const float *x, int ldx, int R, int K, const float *lnw, const float *lnb,
                   const float *W, const float *b, int N, float *y, int ldy, int act, int accumulate, cudaStream_t s,
                   const SplitW &tw = SplitW(), int transpose_out = 0) {
    LinArgs a;
    a.x = x, a.ldx = ldx, a.M = R, a.K = K, a.lnw = lnw, a.lnb = lnb, a.W = W, a.bias = b, a.N = N, a.y = y, a.ldy = ldy;
    a.act = act, a.accumulate = accumulate, a.transpose_out = transpose_out;
    a.tc_wtiles = tw.tiles, a.tc_wunscale = tw.unscale, a.err = ctx->err_mapped + ERR_GEMM_TC;
    a.tc_atiles = m->atiles.p, a.tc_atiles_bytes = m->atiles.bytes;
    Launch{ctx, s}(launch_linear(a, m->stats.as<float>(), s, &ctx->launches), "linear");
}

// Kernels that gave up a bounded wait stored 1 into their report slots: report them once (naming the waits), and
// clear them. The slots are host memory, so this needs no synchronisation; a call still running on the device
// reports at a later check.
static void check_device_error(tcu_ctx *ctx) {
    volatile int *slot = ctx->err_host;
    std::string which;
    for (int i = 0; i < 7; i++) {
        if (slot[i]) {
            slot[i] = 0;
            which += (which.empty() ? "" : "; ") + std::string(err_slot_names[i]);
        }
    }
    if (!which.empty())
        fail(TCU_ERR_CUDA, "kernels gave up a bounded wait: " + which +
                               ". Outputs of the calls queued since the last report are invalid");
}

// Largest |key| and |value| of a stored layer -> the tensor cores' power-of-two scalings (synchronises).
static void scan_layer(tcu_ctx *ctx, const uint8_t *layer, int rows, int chunk, int d, int kv, cudaStream_t s, int &eK,
                       int &eV) {
    Launch{ctx, s}(launch_absmax_layer(layer, rows, chunk, d, kv, ctx->dev_scan, s, &ctx->launches), "scan");
    unsigned bits[2];
    CU(cudaMemcpyAsync(bits, ctx->dev_scan, sizeof(bits), cudaMemcpyDeviceToHost, s));
    CU(cudaStreamSynchronize(s));
    float mk, mv;
    std::memcpy(&mk, &bits[0], 4), std::memcpy(&mv, &bits[1], 4);
    if (!std::isfinite(mk) || !std::isfinite(mv)) fail(TCU_ERR_FORMAT, "cache holds a non-finite key or value");
    eK = tc_exponent(mk), eV = tc_exponent(mv);
}

// The tensor-core tiles of one stored layer (its scalings eK, eV) into out: tc_tile_bytes() per (tile, head).
static void build_tc_tiles(tcu_ctx *ctx, const tcu_model *m, const uint8_t *layer, int kv, int eK, int eV, void *out,
                           cudaStream_t s) {
    const auto &sh = m->w->shape;
    AttnArgs a;
    a.layer = layer, a.rows = m->rows, a.chunk = m->chunk, a.d = sh.d, a.heads = sh.heads;
    a.full = record_bytes(kv, sh.d, m->chunk);
    a.tiles = m->tiles.as<int4>(), a.ntiles = m->ntiles, a.tc_eK = eK, a.tc_eV = eV;
    Launch{ctx, s}(launch_tc_tiles(kv, a, out, s, &ctx->launches), "tensor-core tiles");
}

static bool tc_shape(const tcu_model *m) { return m->w->shape.d / m->w->shape.heads == 128 && tc_enabled(); }
static size_t tc_layer_bytes(const tcu_model *m) { return (size_t)m->ntiles * m->w->shape.heads * tc_tile_bytes(); }
static const void *tc_tiles_of(const tcu_model *m, int l) {
    return m->tctiles.p ? m->tctiles.as<uint8_t>() + tc_layer_bytes(m) * l : nullptr;
}

static void scan_model(tcu_ctx *ctx, tcu_model *m, cudaStream_t s) {
    if (m->tc_scanned) return;
    const int L = m->w->shape.layers;
    m->tc_eK.assign(L, 0), m->tc_eV.assign(L, 0);
    for (int l = 0; l < L; l++)
        scan_layer(ctx, layer_ptr(m, l), m->rows, m->chunk, m->w->shape.d, m->kv, s, m->tc_eK[l], m->tc_eV[l]);
    if (tc_shape(m)) {
        m->tctiles.ensure(tc_layer_bytes(m) * L);
        for (int l = 0; l < L; l++)
            build_tc_tiles(ctx, m, layer_ptr(m, l), m->kv, m->tc_eK[l], m->tc_eV[l],
                           m->tctiles.as<uint8_t>() + tc_layer_bytes(m) * l, s);
        CU(cudaStreamSynchronize(s));
    }
    m->tc_scanned = true;
}

// predict.rs:413-568 one layer for R rows whose representations are h (device, [R][d], updated in place)
static void query_rows(tcu_ctx *ctx, tcu_model *m, int l, const float *scale, const float *h, int R, float *q, cudaStream_t s) {
    const auto &sh = m->w->shape;
    const LayerPtrs &p = m->w->layer[l];
    const int d = sh.d;
    linear(ctx, m, h, d, R, d, p.n1w, p.n1b, p.wq, p.bq, d, q, d, 0, 0, s, p.tq);  // nn.rs:136-137
    if (R <= 128) {
        // up to 128 rows: the SIMT kernels (one block per (row, head), or per 16 rows and a head) spread over more SMs
        // than the tensor-core kernel's 128-pair CTAs would
        Launch{ctx, s}(launch_ssmax(q, R, d, sh.heads, sh.hid, p.q0w, p.q0b, p.q2w, p.q2b, scale, s, &ctx->launches), "ssmax");
        return;
    }
    // nn.rs:138-149 over all (row, head) pairs at once: q viewed as [R * heads][hd] (a row's heads are contiguous),
    // m = W2 GELU(W0 q_h + b0) + b2 as two linear layers, then q_h *= scale_h (1 + tanh m)
    const int H = sh.heads, hd = d / H, hid = sh.hid;
    if (hd == 128 && hid == 64 && p.tq0.tiles && p.tq2.tiles && gemm_tc_enabled()) {
        // the whole MLP and the modulation in one tensor-core kernel
        QmlpArgs qa;
        qa.q = q, qa.pairs = R * H, qa.heads = H, qa.hd = hd, qa.hid = hid;
        qa.w0_tiles = p.tq0.tiles, qa.w2_tiles = p.tq2.tiles, qa.w0_unscale = p.tq0.unscale, qa.w2_unscale = p.tq2.unscale;
        qa.b0 = p.q0b, qa.b2 = p.q2b, qa.scale = scale, qa.err = ctx->err_mapped + ERR_QMLP_TC;
        Launch{ctx, s}(launch_qmlp_tc(qa, s, &ctx->launches), "query MLP (tensor cores)");
        return;
    }
    float *hs = m->ssm.as<float>(), *mm = hs + (size_t)R * H * hid;
    linear(ctx, m, q, hd, R * H, hd, nullptr, nullptr, p.q0w, p.q0b, hid, hs, hid, 1, 0, s, p.tq0);
    linear(ctx, m, hs, hid, R * H, hid, nullptr, nullptr, p.q2w, p.q2b, hd, mm, hd, 0, 0, s, p.tq2);
    Launch{ctx, s}(launch_ssmax_apply(q, mm, scale, R, d, s, &ctx->launches), "ssmax (apply)");
}

static void block_tail(tcu_ctx *ctx, tcu_model *m, int l, float *h, const float *att, int R, cudaStream_t s) {
    const auto &sh = m->w->shape;
    const LayerPtrs &p = m->w->layer[l];
    const int d = sh.d, ff = sh.ff;
    linear(ctx, m, att, d, R, d, nullptr, nullptr, p.wo, p.bo, d, h, d, 0, 1, s, p.to);                    // predict.rs:542-551
    linear(ctx, m, h, d, R, d, p.n2w, p.n2b, p.w1, p.b1, ff, m->mid.as<float>(), ff, 1, 0, s, p.t1);      // predict.rs:552-559
    linear(ctx, m, m->mid.as<float>(), ff, R, ff, nullptr, nullptr, p.w2, p.b2, d, h, d, 0, 1, s, p.t2);   // predict.rs:560-568
}

static void stage(tcu_ctx *ctx, tcu_model *m, float *h, int R, int out_n, float *out, cudaStream_t s) {
    check_ready(m);
    const auto &sh = m->w->shape;
    const int d = sh.d, L = sh.layers, dff = sh.dec_ff;
    if (out_n < 1 || out_n > sh.outs) fail(TCU_ERR_ARG, "stage: out_n must be 1..decoder outputs");
    ensure_work(m, R);
    const float *scales = m->scales.as<float>();
    for (int l = 0; l < L; l++) {
        query_rows(ctx, m, l, scales + (size_t)l * d, h, R, m->q.as<float>(), s);
        attend_layer(ctx, m, layer_ptr(m, l), m->rows, m->chunk, m->kv, m->items.as<int2>(), m->nitems, m->tiles.as<int4>(),
                     m->ntiles, m->q.as<float>(), R, m->att.as<float>(), s, m->tc_eK[l], m->tc_eV[l], false, tc_tiles_of(m, l));
        block_tail(ctx, m, l, h, m->att.as<float>(), R, s);
    }
    // predict.rs:570-584 decoder: only the first out_n outputs are computed (each output is its own row)
    linear(ctx, m, h, d, R, d, m->w->lnw, m->w->lnb, m->w->dec0w, m->w->dec0b, dff, m->mid.as<float>(), dff, 1, 0, s, m->w->tdec0);
    linear(ctx, m, m->mid.as<float>(), dff, R, dff, nullptr, nullptr, m->w->dec2w, m->w->dec2b, out_n, out, out_n, 0, 0, s,
           m->w->tdec2);
}

// ---- the few-row stage as one kernel -------------------------------------------------------------------------

static bool rows_kernel_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_ROWS_KERNEL");
        return !(e && e[0] == '0');
    }();
    return on;
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// Key tiles (head-major), the per-layer pointer table, TMA tensor maps and the barrier words, once per model.
// A stored layer is read in place (fit.rs:6-11): the full chunks as a 3-D byte tensor (a coordinate's keys, the
// 2d coordinates, the chunks; strides chunk * width and the record size) and the last, shorter chunk as a 2-D one.
// Boxes are one tile: the tile's keys (in bytes) x one head's coordinates. A chunk whose rows are not a multiple of
// 16 bytes cannot be described so; its tiles are copied element by element instead.
static void rows_build(tcu_model *m) {
    if (m->rows_built) return;
    const auto &sh = m->w->shape;
    const int tk = rows_tile_keys(m->kv), w = m->kv == 0 ? 4 : (m->kv == 1 ? 2 : 1), hd = sh.d / sh.heads;
    const int nfull = m->rows / m->chunk, rem = m->rows % m->chunk;
    const size_t head = m->kv ? 8 * (size_t)sh.d : 0;
    bool full_ok = nfull > 0 && (m->chunk * w) % 16 == 0 && m->full % 16 == 0;
    bool rem_ok = rem > 0 && (rem * w) % 16 == 0 && m->full % 16 == 0;
    std::vector<CUtensorMap> maps(2 * (size_t)sh.layers);
    std::memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
    auto encode = tensor_map_encoder();
    if (!encode) full_ok = rem_ok = false;
    for (int l = 0; l < sh.layers && (full_ok || rem_ok); l++) {
        const uint8_t *base = layer_ptr(m, l) + head;
        const cuuint32_t box[3] = {(cuuint32_t)(tk * w), (cuuint32_t)hd, 1}, one[3] = {1, 1, 1};
        if (full_ok) {
            const cuuint64_t dims[3] = {(cuuint64_t)m->chunk * w, 2 * (cuuint64_t)sh.d, (cuuint64_t)nfull};
            const cuuint64_t strides[2] = {(cuuint64_t)m->chunk * w, (cuuint64_t)m->full};
            full_ok = encode(&maps[2 * l], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides,
                             box, one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
        if (rem_ok) {
            const cuuint64_t dims[2] = {(cuuint64_t)rem * w, 2 * (cuuint64_t)sh.d};
            const cuuint64_t strides[1] = {(cuuint64_t)rem * w};
            rem_ok = encode(&maps[2 * l + 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                            const_cast<uint8_t *>(base + (size_t)nfull * m->full), dims, strides, box, one,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
    }
    m->rtmaps.ensure(maps.size() * sizeof(CUtensorMap));
    CU(cudaMemcpy(m->rtmaps.p, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
    std::vector<int4> tiles;
    for (int h = 0; h < sh.heads; h++) {
        for (int ci = 0, r0 = 0; r0 < m->rows; ci++, r0 += m->chunk) {
            const int rc = std::min(m->chunk, m->rows - r0);
            const int tma = (ci < nfull ? full_ok : rem_ok) ? 1 : 0;
            for (int k0 = 0; k0 < rc; k0 += tk) tiles.push_back(make_int4(ci, k0, std::min(tk, rc - k0), h | tma << 16));
        }
    }
    m->rtiles_n = (int)tiles.size();
    m->rtiles_per_head = m->rtiles_n / sh.heads;
    m->rtiles.ensure(tiles.size() * sizeof(int4));
    CU(cudaMemcpy(m->rtiles.p, tiles.data(), tiles.size() * sizeof(int4), cudaMemcpyHostToDevice));
    std::vector<RowsLayer> layers(sh.layers);
    const float *scales = m->scales.as<float>();
    for (int l = 0; l < sh.layers; l++) {
        const LayerPtrs &p = m->w->layer[l];
        layers[l] = RowsLayer{p.n1w, p.n1b, p.wq, p.bq, p.q0w, p.q0b, p.q2w, p.q2b, p.wo, p.bo, p.n2w, p.n2b,
                              p.w1, p.b1, p.w2, p.b2, layer_ptr(m, l), scales + (size_t)l * sh.d};
    }
    m->rlayers.ensure(layers.size() * sizeof(RowsLayer));
    CU(cudaMemcpy(m->rlayers.p, layers.data(), layers.size() * sizeof(RowsLayer), cudaMemcpyHostToDevice));
    m->rsync.ensure(256);
    CU(cudaMemset(m->rsync.p, 0, 256));
    m->rows_built = true;
}

// Whether R rows take the one-kernel stage, and its launch shape: one CTA per SM, the same number for every head
// (at most one per key tile of a head), as many tiles of shared memory as fit.
static const tcu_model::RowsPlan *rows_plan(tcu_ctx *ctx, tcu_model *m, int R) {
    const auto &sh = m->w->shape;
    const int hd = sh.d / sh.heads;
    if (!rows_kernel_enabled() || !ctx->coop || R < 1 || R > 8) return nullptr;
    if ((hd != 64 && hd != 128) || sh.hid != 64 || sh.heads > ROWS_MAX_HEADS || sh.layers > ROWS_MAX_LAYERS) return nullptr;
    for (int k : {sh.d, sh.ff, sh.dec_ff})
        if (k % 128 || k > 1024) return nullptr;
    auto &p = m->rows_plans[R > 1 ? 1 : 0];
    if (!p.done) {
        p.done = true;
        rows_build(m);
        // one head per CTA: the grid is a multiple of the heads, with at least one tile per CTA
        const int per = std::min(std::min(ctx->sms, ROWS_MAX_GRID) / sh.heads, m->rtiles_per_head);
        const int want = per * sh.heads;
        for (int slots = rows_slots_for(m->kv, hd, R, ctx->smem_optin); want > 0 && slots >= 2; slots--) {
            const size_t smem = rows_smem(m->kv, hd, R, slots);
            if (rows_max_grid(m->kv, hd, R, smem, ctx->sms) >= want) {
                p.grid = want, p.slots = slots, p.smem = smem;
                break;
            }
        }
    }
    return p.grid ? &p : nullptr;
}

// The stage of R rows (m->h in, m->out out) as one cooperative launch.
static void stage_rows(tcu_ctx *ctx, tcu_model *m, const tcu_model::RowsPlan &p, int R, int out_n, cudaStream_t s) {
    const auto &sh = m->w->shape;
    const int hd = sh.d / sh.heads;
    ensure_work(m, R);
    m->rparts_ms.ensure(sizeof(float) * (size_t)p.grid * 8 * 2);
    m->rparts_acc.ensure(sizeof(float) * (size_t)p.grid * 8 * hd);
    RowsArgs a;
    a.layers = m->rlayers.as<RowsLayer>();
    a.L = sh.layers, a.d = sh.d, a.heads = sh.heads, a.ff = sh.ff, a.dff = sh.dec_ff, a.out_n = out_n, a.R = R;
    a.lnw = m->w->lnw, a.lnb = m->w->lnb, a.dec0w = m->w->dec0w, a.dec0b = m->w->dec0b;
    a.dec2w = m->w->dec2w, a.dec2b = m->w->dec2b;
    a.rows = m->rows, a.chunk = m->chunk, a.full = m->full;
    a.tiles = m->rtiles.as<int4>(), a.ntiles = m->rtiles_n, a.tiles_per_head = m->rtiles_per_head, a.slots = p.slots;
    a.tmaps = m->rtmaps.p, a.nfull = m->rows / m->chunk;
    a.h = m->h.as<float>(), a.q = m->q.as<float>(), a.att = m->att.as<float>(), a.mid = m->mid.as<float>();
    a.out = m->out.as<float>();
    a.part_ms = m->rparts_ms.as<float>(), a.part_acc = m->rparts_acc.as<float>();
    // the barrier word at byte 0, the launch's abort word at byte 128 (its own line); every launch starts from
    // zeros, so one that gave up leaves nothing behind
    a.bar = m->rsync.as<unsigned>(), a.err = reinterpret_cast<int *>(m->rsync.as<uint8_t>() + 128);
    a.err_report = ctx->err_mapped + ERR_ROWS;
    CU(cudaMemsetAsync(m->rsync.p, 0, 256, s));
    if (ctx->abort_next) {
        // test hook: start with the abort word set, as if a wait had given up; every CTA leaves at its first
        // barrier after its first phase and waits for its copies in flight
        CU(cudaMemsetAsync(a.err, 1, sizeof(int), s));
        ctx->abort_next = false;
    }
    cudaEvent_t ev_end = nullptr;
    if (ctx->prof) {
        if (ctx->prof_used + 2 > ctx->prof_events.size()) {
            for (int i = 0; i < 64; i++) {
                cudaEvent_t e;
                CU(cudaEventCreate(&e));
                ctx->prof_events.push_back(e);
            }
        }
        CU(cudaEventRecord(ctx->prof_events[ctx->prof_used], s));
        ev_end = ctx->prof_events[ctx->prof_used + 1];
        ctx->prof_used += 2;
    }
    // diagnostics: TCU_ROWS_TRACE=<file> writes each CTA's barrier entry and exit times of this launch there
    const char *trace_path = getenv("TCU_ROWS_TRACE");
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    CU(cudaStreamIsCapturing(s, &capturing));
    if (capturing != cudaStreamCaptureStatusNone) trace_path = nullptr;  // eager calls only (TCU_GRAPHS=0)
    DevBuf trace;
    if (trace_path) {
        trace.ensure(sizeof(unsigned long long) * (size_t)p.grid * ROWS_TRACE_MARKS);
        CU(cudaMemsetAsync(trace.p, 0, trace.bytes, s));
        a.trace = trace.as<unsigned long long>();
    }
    Launch{ctx, s}(launch_stage_rows(m->kv, hd, a, p.grid, p.smem, s, &ctx->launches), "stage (one kernel)");
    if (ev_end) CU(cudaEventRecord(ev_end, s));
    if (trace_path) {
        std::vector<unsigned long long> t(trace.bytes / sizeof(unsigned long long));
        CU(cudaMemcpyAsync(t.data(), trace.p, trace.bytes, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        if (FILE *f = std::fopen(trace_path, "wb")) {
            const int32_t head[2] = {p.grid, ROWS_TRACE_MARKS};
            std::fwrite(head, sizeof(head), 1, f);
            std::fwrite(t.data(), sizeof(unsigned long long), t.size(), f);
            std::fclose(f);
        }
    }
}

// The stage on the model's own buffers (m->h in, m->out out), replayed from a CUDA graph captured on the context
// stream the first time a (rows, outputs, profiling) combination is seen. TCU_GRAPHS=0 runs it eagerly.
static void stage_replay(tcu_ctx *ctx, tcu_model *m, int R, int out_n, cudaStream_t s) {
    static const bool use_graphs = [] {
        const char *e = getenv("TCU_GRAPHS");
        return !(e && e[0] == '0');
    }();
    if (m->out.ensure(sizeof(float) * (size_t)R * out_n)) drop_graphs(m);
    if (const auto *p = rows_plan(ctx, m, R)) {
        stage_rows(ctx, m, *p, R, out_n, s);
        return;
    }
    scan_model(ctx, m, ctx->stream);  // once per model, before any capture
    ensure_work(m, R);
    if (!use_graphs) {
        stage(ctx, m, m->h.as<float>(), R, out_n, m->out.as<float>(), s);
        return;
    }
    for (auto &g : m->graphs) {
        if (g.R == R && g.out_n == out_n && g.prof == ctx->prof) {
            CU(cudaGraphLaunch(g.exec, s));
            ctx->launches += g.launches;
            // a profiled graph re-records its own events: the profile then holds its last replay's passes
            if (g.prof) ctx->prof_used = std::max(ctx->prof_used, g.prof_events);
            return;
        }
    }
    cudaStream_t cs = ctx->stream;
    const uint64_t before = ctx->launches;
    if (ctx->prof) ctx->prof_used = 0;  // a profiled graph owns the first events of the context
    CU(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    cudaGraph_t graph = nullptr;
    try {
        stage(ctx, m, m->h.as<float>(), R, out_n, m->out.as<float>(), cs);
    } catch (...) {
        cudaStreamEndCapture(cs, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
    }
    CU(cudaStreamEndCapture(cs, &graph));
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    CU(e);
    tcu_model::Graph g{R, out_n, ctx->prof, exec, ctx->launches - before, ctx->prof ? ctx->prof_used : 0};
    // a profiled graph keeps its events for good: drop other profiled graphs, which used the same ones
    if (g.prof) {
        for (auto it = m->graphs.begin(); it != m->graphs.end();) {
            if (it->prof) {
                cudaGraphExecDestroy(it->exec);
                it = m->graphs.erase(it);
            } else {
                ++it;
            }
        }
    }
    m->graphs.push_back(g);
    // the capture itself ran nothing: count the replay's kernels
    ctx->launches = before + g.launches;
    CU(cudaGraphLaunch(exec, s));
}

// ---- the column and row stages (predict.rs:282-372) -------------------------------------------------------------

static void check_rows_weights(const tcu_weights *w) {
    const RowsWeights &rw = w->rows;
    if (!rw.on) fail(TCU_DECLINED, "rows: the weights have no column and row stages");
    if (rw.shape.cls * rw.shape.e != w->shape.d) fail(TCU_ERR_FORMAT, "rows: class tokens times width differ from the in-context width");
}

static void check_rows_ready(const tcu_model *m) {
    check_rows_weights(m->w);
    if (!m->col_kv.p) fail(TCU_DECLINED, "rows: the cache has no column-stage keys and values (col_kv was never put)");
}

// Grow the linear layers' scratch (row statistics, split rows) for M rows of width up to K; graphs that used the old
// buffers are dropped.
static void ensure_linear(tcu_model *m, size_t M, int K) {
    bool moved = m->stats.ensure(sizeof(float) * 4 * M);
    moved |= m->atiles.ensure(tc_split_bytes((int)M, K));
    if (moved) drop_graphs(m);
}

// nn.rs:289-302 cached_block for every cell of X [R * F][e] (in place): the second attention of a column block against
// group g's inducing points (keys and values at kv + g * gstride), then the block's feed-forward. Q, A [R * F][e] and
// H [R * F][ff] are scratch.
static void cached_block(tcu_ctx *ctx, tcu_model *m, const CBlockPtrs &B, float *X, float *Q, float *A, float *H, int R,
                         int F, const float *kv, size_t gstride, cudaStream_t s) {
    const auto &rs = m->w->rows.shape;
    const int e = rs.e, ff = B.ff, M = R * F;
    const float scale = 1.0f / std::sqrt((float)(e / rs.col_heads));
    linear(ctx, m, X, e, M, e, B.n1w, B.n1b, B.inw, B.inb, e, Q, e, 0, 0, s, B.tin);
    Launch{ctx, s}(launch_col_attend(Q, R, F, kv, gstride, e, rs.inds, rs.col_heads, scale, A, s, &ctx->launches),
                   "column attention");
    linear(ctx, m, A, e, M, e, nullptr, nullptr, B.ow, B.ob, e, X, e, 0, 1, s, B.to);
    linear(ctx, m, X, e, M, e, B.n2w, B.n2b, B.w1, B.b1, ff, H, ff, 1, 0, s, B.t1);
    linear(ctx, m, H, ff, M, ff, nullptr, nullptr, B.w2, B.b2, e, X, e, 0, 1, s, B.t2);
}

// predict.rs:282-353 embed: normalised rows x (device [R][F]) to tokens tok (device [R][cls + F][e]). Every cell
// goes through every column block's second attention against its group's cached inducing points (cached_block,
// nn.rs:289-302); with several label digits, once per digit from the same starting cell, then the average.
static void embed(tcu_ctx *ctx, tcu_model *m, const float *x, int R, float *tok, cudaStream_t s) {
    check_rows_ready(m);
    const RowsWeights &rw = m->w->rows;
    const auto &rs = rw.shape;
    const int e = rs.e, F = m->features, D = m->digits, nb = rs.col_blocks, inds = rs.inds, ff = rs.col_ff;
    const size_t M = (size_t)R * F, per = (size_t)2 * e * inds, gstride = (size_t)D * nb * per;
    m->cx.ensure(sizeof(float) * M * e), m->cq.ensure(sizeof(float) * M * e), m->catt.ensure(sizeof(float) * M * e);
    m->cmid.ensure(sizeof(float) * M * ff);
    if (D > 1) m->cx0.ensure(sizeof(float) * M * e), m->csum.ensure(sizeof(float) * M * e);
    ensure_linear(m, M, std::max(e, ff));
    float *X = m->cx.as<float>(), *Q = m->cq.as<float>(), *A = m->catt.as<float>(), *H = m->cmid.as<float>();
    Launch ck{ctx, s};
    ck(launch_col_cells(x, R, F, rs.group, rw.in_w, rw.in_b, e, D > 1 ? m->cx0.as<float>() : X, s, &ctx->launches), "cells");
    for (int dg = 0; dg < D; dg++) {
        if (D > 1) CU(cudaMemcpyAsync(X, m->cx0.p, sizeof(float) * M * e, cudaMemcpyDeviceToDevice, s));
        for (int b = 0; b < nb; b++)
            cached_block(ctx, m, rw.col[b], X, Q, A, H, R, F, m->col_kv.as<float>() + (dg * nb + b) * per, gstride, s);
        if (D > 1) ck(launch_scale_add(m->csum.as<float>(), X, M * e, 1.0f, dg > 0, s, &ctx->launches), "digit sum");
    }
    if (D > 1) ck(launch_divide(X, m->csum.as<float>(), M * e, (float)D, s, &ctx->launches), "digit average");
    ck(launch_tokens(X, rw.cls_tokens, R, F, rs.cls, e, tok, s, &ctx->launches), "tokens");
}

// predict.rs:356-372 represent: tokens (device [R][T][e], consumed) to row representations rep (device [R][cls e]):
// the row blocks (nn.rs:357-419; the last one only for the class tokens), then the class tokens' LayerNorm.
static void represent(tcu_ctx *ctx, tcu_model *m, float *tok, int R, float *rep, cudaStream_t s) {
    check_rows_weights(m->w);
    const RowsWeights &rw = m->w->rows;
    const auto &rs = rw.shape;
    const int e = rs.e, T = rs.cls + m->features, heads = rs.row_heads, half = e / heads / 2, ff = rs.row_ff;
    const size_t M = (size_t)R * T;
    m->cqkv.ensure(sizeof(float) * M * 3 * e), m->catt.ensure(sizeof(float) * M * e);
    m->cnew.ensure(sizeof(float) * (size_t)R * rs.cls * e);  // the last block's class tokens
    m->cmid.ensure(sizeof(float) * M * ff);
    if (row_attend_needs_workspace(e, T, T, heads) || row_attend_needs_workspace(e, T, rs.cls, heads))
        m->ckt.ensure(sizeof(float) * row_attend_workspace(R, T, e));
    ensure_linear(m, M, std::max(e, ff));
    if (m->crope_T != T) {
        // nn.rs:309-321: cos and sin of position times frequency, in f32
        std::vector<float> tab((size_t)2 * T * half);
        for (int t = 0; t < T; t++)
            for (int i = 0; i < half; i++) {
                const float a = (float)t * rw.rope_freqs[i];
                tab[(size_t)t * half + i] = std::cos(a), tab[(size_t)(T + t) * half + i] = std::sin(a);
            }
        m->crope.ensure(sizeof(float) * tab.size());
        CU(cudaMemcpy(m->crope.p, tab.data(), sizeof(float) * tab.size(), cudaMemcpyHostToDevice));
        m->crope_T = T;
    }
    const float *cs = m->crope.as<float>(), *sn = cs + (size_t)T * half;
    float *cur = tok, *nxt = m->cnew.as<float>(), *QKV = m->cqkv.as<float>(), *A = m->catt.as<float>(), *H = m->cmid.as<float>();
    Launch ck{ctx, s};
    for (int bi = 0; bi < rs.row_blocks; bi++) {
        const CBlockPtrs &B = rw.row[bi];
        const bool last = bi + 1 == rs.row_blocks;
        const int nq = last ? rs.cls : T, MQ = R * nq;
        linear(ctx, m, cur, e, (int)M, e, B.n1w, B.n1b, B.inw, B.inb, 3 * e, QKV, 3 * e, 0, 0, s, B.tin);
        ck(launch_row_attend(QKV, R, T, nq, e, heads, cs, sn, m->ckt.as<float>(), A, s, &ctx->launches), "row attention");
        if (!last) {
            // every token is a query: the out-projection adds onto the tokens themselves (the residual, the same sum
            // as adding the tokens onto it), and the feed-forward updates them in place for the next block
            linear(ctx, m, A, e, MQ, e, nullptr, nullptr, B.ow, B.ob, e, cur, e, 0, 1, s, B.to);
            linear(ctx, m, cur, e, MQ, e, B.n2w, B.n2b, B.w1, B.b1, ff, H, ff, 1, 0, s, B.t1);
            linear(ctx, m, H, ff, MQ, ff, nullptr, nullptr, B.w2, B.b2, e, cur, e, 0, 1, s, B.t2);
            continue;
        }
        linear(ctx, m, A, e, MQ, e, nullptr, nullptr, B.ow, B.ob, e, nxt, e, 0, 0, s, B.to);
        ck(launch_add_rows(nxt, cur, R, nq, T, e, s, &ctx->launches), "row residual");
        linear(ctx, m, nxt, e, MQ, e, B.n2w, B.n2b, B.w1, B.b1, ff, H, ff, 1, 0, s, B.t1);
        linear(ctx, m, H, ff, MQ, ff, nullptr, nullptr, B.w2, B.b2, e, nxt, e, 0, 1, s, B.t2);
    }
    // the last block left the class tokens [R][cls][e] in nxt: their LayerNorm, laid end to end, is the representation
    ck(launch_ln_apply(nxt, R * rs.cls, e, rw.out_lnw, rw.out_lnb, rep, s, &ctx->launches), "row LayerNorm");
}

// predict.rs:638-652: the three stages of a member with one node (the `rows` hook): x (device [R][F]) to the model's
// out buffer (m->out, [R][out_n]).
static void rows_stage(tcu_ctx *ctx, tcu_model *m, const float *x, int R, int out_n, cudaStream_t s) {
    check_ready(m);
    check_rows_ready(m);
    if (m->nodes != 1) fail(TCU_DECLINED, "rows: the member has several problems (the class tree); its nodes run one by one");
    if (out_n < 1 || out_n > m->w->shape.outs) fail(TCU_ERR_ARG, "rows: out_n must be 1..decoder outputs");
    const auto &rs = m->w->rows.shape;
    m->ctok.ensure(sizeof(float) * (size_t)R * (rs.cls + m->features) * rs.e);
    if (m->h.ensure(sizeof(float) * (size_t)R * m->w->shape.d)) drop_graphs(m);
    embed(ctx, m, x, R, m->ctok.as<float>(), s);
    represent(ctx, m, m->ctok.as<float>(), R, m->h.as<float>(), s);
    stage_replay(ctx, m, R, out_n, s);
}

// ---- the column and row stages of fitting (fit.rs:298-540) ---------------------------------------------------------

// fit.rs:300-314: the inducing points' queries of a column block's first attention for n training rows, [inds][e]:
// nn.rs:130-152 query (LayerNorm, the query rows of in_proj, the per-head query MLP) times nn.rs:97-107 query_scale.
static std::vector<float> ind_queries(const Isab1 &a, const tcu_rows_shape &rs, int n) {
    const int e = rs.e, heads = rs.col_heads, hd = e / heads, hid = a.hid;
    std::vector<float> scale(e), h(hid), t(e), mm(hd), out((size_t)rs.inds * e);
    const float logn = std::log((float)(n > 1 ? n : 1)), inv = 1.0f / std::sqrt((float)hd);
    for (int i = 0; i < hid; i++) h[i] = h_gelu(a.sb0w[i] * logn + a.sb0b[i]);
    h_linear(a.sb2w.data(), a.sb2b.data(), h.data(), hid, e, scale.data());
    for (int i = 0; i < e; i++) scale[i] *= inv;
    for (int i = 0; i < rs.inds; i++) {
        float *q = out.data() + (size_t)i * e;
        h_layer_norm(a.ind_h.data() + (size_t)i * e, a.n1w.data(), a.n1b.data(), e, t.data());
        h_linear(a.wq.data(), a.bq.data(), t.data(), e, e, q);
        for (int hh = 0; hh < heads; hh++) {
            float *qh = q + hh * hd;
            h_linear(a.q0w.data(), a.q0b.data(), qh, hd, hid, h.data());
            for (int j = 0; j < hid; j++) h[j] = h_gelu(h[j]);
            h_linear(a.q2w.data(), a.q2b.data(), h.data(), hid, hd, mm.data());
            for (int j = 0; j < hd; j++) qh[j] *= scale[hh * hd + j] * (1.0f + h_tanh1(mm[j]));
        }
    }
    return out;
}

// fit.rs:326-420 col_one for F feature groups at once (the `columns` hook of fit::Attend, fit.rs:33-38): the training
// cells X (device [n * F][e], cell (r, g) at row r * F + g, through the input layer with the label's embedding added;
// replaced by the cells after the stage) through every column block. Per block: the cells' keys and values for the
// first attention, the inducing points' attention over every group's cells (queries iq, device [blocks][inds][e],
// scaled), its out-projection with the inducing points as residual and the feed-forward, the result's keys and values
// for the second attention (block b's cache of group g at col_kv + g * gstride + off + b * 2 e inds), then every cell
// through the second attention against them. The reference walks the cells `chunk` rows at a time only to bound its
// memory; the attention here takes every row of a group at once, split for parallelism: the same up to rounding.
static void column_blocks(tcu_ctx *ctx, tcu_model *m, float *X, int n, int F, const float *iq, float *col_kv,
                          size_t gstride, size_t off, cudaStream_t s) {
    const RowsWeights &rw = m->w->rows;
    const auto &rs = rw.shape;
    const int e = rs.e, nb = rs.col_blocks, inds = rs.inds, heads = rs.col_heads, hd = e / heads, ff = rs.col_ff;
    const size_t M = (size_t)n * F, per = (size_t)2 * e * inds, I = (size_t)F * inds;
    if (M > (size_t)INT32_MAX / 4 || I > (size_t)INT32_MAX / 4) fail(TCU_ERR_ARG, "fit: too many training cells for one call");
    const int splits = ind_attend_splits(n, F, heads, inds);
    m->cq.ensure(sizeof(float) * M * 2 * e), m->catt.ensure(sizeof(float) * M * e), m->cmid.ensure(sizeof(float) * M * ff);
    ensure_linear(m, std::max(M, I), std::max(e, ff));
    DevBuf pms, pacc, hid, hmid, kv2;
    pms.ensure(sizeof(float) * 2 * (size_t)F * heads * splits * inds);
    pacc.ensure(sizeof(float) * (size_t)F * heads * splits * inds * hd);
    hid.ensure(sizeof(float) * I * e), hmid.ensure(sizeof(float) * I * std::max(e, ff));
    kv2.ensure(sizeof(float) * I * 2 * e);
    float *KV = m->cq.as<float>(), *A = m->catt.as<float>(), *H = m->cmid.as<float>();
    float *hb = hid.as<float>(), *hm = hmid.as<float>();
    Launch ck{ctx, s};
    for (int b = 0; b < nb; b++) {
        const Isab1 &a1 = rw.col1[b];
        // the cells' keys and values for the first attention [M][2e]
        linear(ctx, m, X, e, (int)M, e, a1.b.n1w, a1.b.n1b, a1.b.inw, a1.b.inb, 2 * e, KV, 2 * e, 0, 0, s, a1.b.tin);
        // the attention [F * inds][e] goes into the feed-forward's buffer, which it leaves before the feed-forward
        ck(launch_ind_attend(iq + (size_t)b * inds * e, KV, n, F, e, inds, heads, splits, pms.as<float>(), pacc.as<float>(),
                             hm, s, &ctx->launches),
           "inducing attention");
        ck(launch_repeat(hb, a1.ind, (size_t)inds * e, F, s, &ctx->launches), "inducing residual");
        linear(ctx, m, hm, e, (int)I, e, nullptr, nullptr, a1.b.ow, a1.b.ob, e, hb, e, 0, 1, s, a1.b.to);
        linear(ctx, m, hb, e, (int)I, e, a1.b.n2w, a1.b.n2b, a1.b.w1, a1.b.b1, a1.b.ff, hm, a1.b.ff, 1, 0, s, a1.b.t1);
        linear(ctx, m, hm, a1.b.ff, (int)I, a1.b.ff, nullptr, nullptr, a1.b.w2, a1.b.b2, e, hb, e, 0, 1, s, a1.b.t2);
        // their keys and values for the second attention: the cache prediction reads (fit.rs:392-404)
        const CBlockPtrs &B = rw.col[b];
        linear(ctx, m, hb, e, (int)I, e, B.n1w, B.n1b, a1.kv2w, a1.kv2b, 2 * e, kv2.as<float>(), 2 * e, 0, 0, s, a1.tkv2);
        ck(launch_col_kv_scatter(kv2.as<float>(), F, e, inds, gstride, off + b * per, col_kv, s, &ctx->launches),
           "cache scatter");
        cached_block(ctx, m, B, X, KV, A, H, n, F, col_kv + off + b * per, gstride, s);
    }
    // the locals above are freed on return: finish with them first
    CU(cudaStreamSynchronize(s));
}

static void check_fit_weights(const tcu_weights *w) {
    check_rows_weights(w);
    if (!w->rows.fit) fail(TCU_DECLINED, "fit: the weights were not made for fitting, or have no column-stage fit tensors");
    if (!ind_attend_takes(w->rows.shape.e, w->rows.shape.col_heads))
        fail(TCU_DECLINED, "fit: the column stage's head width is not one of 4, 8, 16, 32, 64");
}

// fit.rs:300-314: every column block's inducing-point queries for n training rows, on the device [blocks][inds][e].
static void put_ind_queries(const tcu_weights *w, int n, DevBuf &iq, cudaStream_t s) {
    const RowsWeights &rw = w->rows;
    const auto &rs = rw.shape;
    const size_t one = (size_t)rs.inds * rs.e;
    std::vector<float> q_all(one * rs.col_blocks);
    for (int b = 0; b < rs.col_blocks; b++) {
        auto q = ind_queries(rw.col1[b], rs, n);
        std::copy(q.begin(), q.end(), q_all.begin() + b * one);
    }
    iq.ensure(sizeof(float) * q_all.size());
    CU(cudaMemcpyAsync(iq.p, q_all.data(), sizeof(float) * q_all.size(), cudaMemcpyHostToDevice, s));
    CU(cudaStreamSynchronize(s));
}

// fit.rs:298-481 on the device: normalised training rows x (device [n][F]) and labels y (device [n]) to the member's
// column cache col_kv (device [F][D][blocks][2][e][inds]) and the training tokens tok (device [n][cls + F][e]): the
// cells through the input layer, then per label digit (fit.rs:316-324: digit ((int)y / divisor) % base of the class
// label) the label's embedding and the column blocks; with several digits the cells' average over them.
static void fit_columns(tcu_ctx *ctx, tcu_model *m, const float *x, const float *y, int n, int F, int D,
                        const int32_t *bases, float *col_kv, float *tok, cudaStream_t s) {
    const tcu_weights *w = m->w;
    check_fit_weights(w);
    const RowsWeights &rw = w->rows;
    const auto &rs = rw.shape;
    const int e = rs.e, nb = rs.col_blocks, inds = rs.inds;
    if (n < 1 || F < 1 || D < 1) fail(TCU_ERR_ARG, "fit: rows, features and digits must be positive");
    for (int dg = 0; D > 1 && dg < D; dg++)
        if (bases[dg] < 2) fail(TCU_ERR_ARG, "fit: every digit's base must be at least 2");
    const size_t M = (size_t)n * F, per = (size_t)2 * e * inds, gstride = (size_t)D * nb * per;
    m->cx.ensure(sizeof(float) * M * e);
    if (D > 1) m->cx0.ensure(sizeof(float) * M * e), m->csum.ensure(sizeof(float) * M * e);
    DevBuf iq;
    put_ind_queries(w, n, iq, s);
    float *X = m->cx.as<float>();
    Launch ck{ctx, s};
    ck(launch_col_cells(x, n, F, rs.group, rw.in_w, rw.in_b, e, D > 1 ? m->cx0.as<float>() : X, s, &ctx->launches), "cells");
    for (int dg = 0; dg < D; dg++) {
        if (D > 1) CU(cudaMemcpyAsync(X, m->cx0.p, sizeof(float) * M * e, cudaMemcpyDeviceToDevice, s));
        int divisor = 1;
        for (int b = dg + 1; b < D; b++) divisor *= bases[b];
        ck(launch_col_add_y(X, y, n, F, e, rw.max_classes, rw.col_y, divisor, D > 1 ? bases[dg] : 0, s, &ctx->launches),
           "cell labels");
        column_blocks(ctx, m, X, n, F, iq.as<float>(), col_kv, gstride, (size_t)dg * nb * per, s);
        if (D > 1) ck(launch_scale_add(m->csum.as<float>(), X, M * e, 1.0f, dg > 0, s, &ctx->launches), "digit sum");
    }
    if (D > 1) ck(launch_divide(X, m->csum.as<float>(), M * e, (float)D, s, &ctx->launches), "digit average");
    ck(launch_tokens(X, rw.cls_tokens, n, F, rs.cls, e, tok, s, &ctx->launches), "tokens");
}

// fit.rs:487-540: the training tokens (device [n][cls + F][e], consumed) through the row stage to the training rows'
// representations rep (device [n][d]), a block of rows at a time to bound the working memory.
static void fit_rows(tcu_ctx *ctx, tcu_model *m, float *tok, int n, int F, float *rep, cudaStream_t s) {
    const auto &rs = m->w->rows.shape;
    const size_t T = (size_t)rs.cls + F;
    const int block = (int)std::max<size_t>(256, std::min<size_t>(n, (size_t)(1u << 22) / T));
    for (int r0 = 0; r0 < n; r0 += block) {
        const int rb = std::min(block, n - r0);
        represent(ctx, m, tok + (size_t)r0 * T * rs.e, rb, rep + (size_t)r0 * m->w->shape.d, s);
    }
    CU(cudaStreamSynchronize(s));
}

// ---- a member's problems and the class tree (predict.rs:638-699) -------------------------------------------------

// One node of `m{i}/tree` (fit.rs:217-220): [leaf, rows, k, map[k]].
struct TreeNode {
    bool leaf;
    int rows, k;
    std::vector<int> map;
};

static std::vector<TreeNode> parse_tree(const int32_t *tree, size_t len, int n_nodes) {
    if (n_nodes < 1) fail(TCU_ERR_FORMAT, "tree: no nodes");
    std::vector<TreeNode> out;
    size_t at = 0;
    for (int i = 0; i < n_nodes; i++) {
        if (at + 3 > len || tree[at + 2] < 1 || at + 3 + (size_t)tree[at + 2] > len) fail(TCU_ERR_FORMAT, "tree is damaged");
        TreeNode n{tree[at] != 0, tree[at + 1], tree[at + 2], {}};
        n.map.assign(tree + at + 3, tree + at + 3 + n.k);
        at += 3 + (size_t)n.k;
        out.push_back(std::move(n));
    }
    return out;
}

}  // namespace tcu

struct tcu_member {
    tcu_ctx *ctx = nullptr;
    std::vector<tcu_model *> nodes;  // owned
    std::vector<TreeNode> tree;
    int classes = 0;
    std::vector<int> walk;   // node indices in the order predict.rs:676-687's walk visits them
    std::vector<int> koff;   // per node: offset of its scores among all problems' [R][k] blocks, in units of R
    int ksum = 0;
    DevBuf tnodes, tmap;     // the walk as the combine kernel reads it
    DevBuf rep, tok, scores, wbuf, out;
};

namespace tcu {

// The walk of predict.rs:676-687 from node 0: a node, then each child in map order. Checks every target (a leaf's
// against the classes, an inner node's against the nodes, none reached twice) and lays the walk out for the kernel.
static void member_tables(tcu_member *mb) {
    const int n = (int)mb->tree.size();
    std::vector<int> pos(n, -1);
    std::function<void(int, int)> visit = [&](int ni, int depth) {
        if (depth > n || pos[ni] >= 0) fail(TCU_ERR_FORMAT, "tree: node " + std::to_string(ni) + " is reached twice");
        pos[ni] = (int)mb->walk.size();
        mb->walk.push_back(ni);
        const TreeNode &t = mb->tree[ni];
        for (int c : t.map) {
            if (t.leaf) {
                if (c < 0 || c >= mb->classes) fail(TCU_ERR_FORMAT, "tree: class " + std::to_string(c) + " out of range");
            } else {
                if (c < 0 || c >= n) fail(TCU_ERR_FORMAT, "tree: child " + std::to_string(c) + " out of range");
                visit(c, depth + 1);
            }
        }
    };
    visit(0, 0);
    mb->koff.assign(n, 0);
    mb->ksum = 0;
    for (int i = 0; i < n; i++) mb->koff[i] = mb->ksum, mb->ksum += mb->tree[i].k;
    std::vector<int4> tn;
    std::vector<int> tm;
    for (int ni : mb->walk) {
        const TreeNode &t = mb->tree[ni];
        tn.push_back(make_int4(t.k, t.leaf ? 1 : 0, mb->koff[ni], (int)tm.size()));
        for (int c : t.map) tm.push_back(t.leaf ? c : pos[c]);
    }
    mb->tnodes.ensure(tn.size() * sizeof(int4));
    mb->tmap.ensure(tm.size() * sizeof(int));
    CU(cudaMemcpy(mb->tnodes.p, tn.data(), tn.size() * sizeof(int4), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(mb->tmap.p, tm.data(), tm.size() * sizeof(int), cudaMemcpyHostToDevice));
}

// predict.rs:664-692: every problem's scores (mb->scores, or `scores` laid out the same way) to class scores
static void member_combine(tcu_ctx *ctx, tcu_member *mb, const float *scores, int R, float *out, cudaStream_t s) {
    mb->wbuf.ensure(sizeof(float) * (size_t)mb->tree.size() * R);
    Launch{ctx, s}(launch_tree_combine(scores, mb->tnodes.as<int4>(), mb->tmap.as<int>(), (int)mb->walk.size(), R,
                                       mb->classes, mb->wbuf.as<float>(), out, s, &ctx->launches),
                   "class tree");
}

// predict.rs:638-699 for R normalised rows x (device [R][F]): the column and row stages once (node 0's column cache),
// every problem's in-context stage, then the tree; the result is left in mb->out [R][classes], or for a member of
// one problem in node 0's out buffer (returned).
static const float *member_rows(tcu_ctx *ctx, tcu_member *mb, const float *x, int R, cudaStream_t s) {
    tcu_model *m0 = mb->nodes[0];
    for (auto *m : mb->nodes) check_ready(m);
    check_rows_ready(m0);
    const auto &rs = m0->w->rows.shape;
    const size_t hd = sizeof(float) * (size_t)R * m0->w->shape.d;
    mb->tok.ensure(sizeof(float) * (size_t)R * (rs.cls + m0->features) * rs.e);
    if (mb->nodes.size() == 1) {
        if (m0->h.ensure(hd)) drop_graphs(m0);
        embed(ctx, m0, x, R, mb->tok.as<float>(), s);
        represent(ctx, m0, mb->tok.as<float>(), R, m0->h.as<float>(), s);
        stage_replay(ctx, m0, R, mb->tree[0].k, s);
        return m0->out.as<float>();
    }
    mb->rep.ensure(hd);
    embed(ctx, m0, x, R, mb->tok.as<float>(), s);
    represent(ctx, m0, mb->tok.as<float>(), R, mb->rep.as<float>(), s);
    mb->scores.ensure(sizeof(float) * (size_t)R * mb->ksum);
    for (int ni : mb->walk) {
        tcu_model *m = mb->nodes[ni];
        const int k = mb->tree[ni].k;
        if (m->h.ensure(hd)) drop_graphs(m);
        CU(cudaMemcpyAsync(m->h.p, mb->rep.p, hd, cudaMemcpyDeviceToDevice, s));  // the stage consumes its rows
        stage_replay(ctx, m, R, k, s);
        CU(cudaMemcpyAsync(mb->scores.as<float>() + (size_t)mb->koff[ni] * R, m->out.p, sizeof(float) * (size_t)R * k,
                           cudaMemcpyDeviceToDevice, s));
    }
    mb->out.ensure(sizeof(float) * (size_t)R * mb->classes);
    member_combine(ctx, mb, mb->scores.as<float>(), R, mb->out.as<float>(), s);
    return mb->out.as<float>();
}

// ---- training rows split across devices -----------------------------------------------------------------------

static void nccl_check(ncclResult_t r, const char *what) {
    if (r != ncclSuccess) fail(TCU_ERR_CUDA, std::string(what) + ": " + nccl_api().error_string(r));
}

// The stage with every layer's attention merged over the ranks of c (m holds this rank's rows; m->h in, m->out out).
static bool p2p_enabled() {
    static const bool on = [] {
        const char *e = getenv("TCU_SHARD_P2P");
        return !(e && e[0] == '0');
    }();
    return on;
}

// This rank's exchange buffer of at least `bytes`, mapped by every peer, and theirs mapped here (all ranks call this
// with the same size, in step). The buffer is made anew when it must grow; the handles are exchanged by an NCCL
// all-gather and every rank agrees (all-reduce of the outcome) whether the mappings work everywhere: false, for good,
// when they do not.
static bool ensure_peer(tcu_comm *c, size_t bytes, cudaStream_t s) {
    if (c->p2p == 0 || !p2p_enabled() || c->nranks > PUSH_MAX_RANKS) return false;
    if (c->p2p == 1 && bytes <= c->pbytes) return true;
    const auto &api = nccl_api();
    const int N = c->nranks, me = c->rank;
    CU(cudaStreamSynchronize(s));
    DevBuf hd, okd;
    okd.ensure(sizeof(int));
    if (c->pbuf) {
        // a buffer that must grow: every rank lets go of its mappings of the others' before any is freed
        for (int j = 0; j < (int)c->ppeer.size(); j++)
            if (j != me && c->ppeer[j]) cudaIpcCloseMemHandle(c->ppeer[j]);
        nccl_check(api.all_reduce(okd.p, okd.p, 1, ncclInt32, ncclMin, c->comm, s), "all-reduce (exchange buffers)");
        CU(cudaStreamSynchronize(s));
        CU(cudaFree(c->pbuf));
    }
    c->ppeer.assign(N, nullptr);
    c->pbuf = nullptr, c->pbytes = 0;
    bytes = (bytes + 4095) / 4096 * 4096;
    CU(cudaMalloc(&c->pbuf, bytes));
    CU(cudaMemset(c->pbuf, 0, bytes));
    if (!c->pdone) CU(cudaMalloc(&c->pdone, sizeof(unsigned) * PUSH_MAX_RANKS));
    CU(cudaMemset(c->pdone, 0, sizeof(unsigned) * PUSH_MAX_RANKS));
    cudaIpcMemHandle_t mine;
    CU(cudaIpcGetMemHandle(&mine, c->pbuf));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    hd.ensure(hb * N);
    CU(cudaMemcpy(hd.as<uint8_t>() + hb * me, &mine, hb, cudaMemcpyHostToDevice));
    nccl_check(api.all_gather(hd.as<uint8_t>() + hb * me, hd.p, hb, ncclUint8, c->comm, s), "all-gather (exchange handles)");
    CU(cudaStreamSynchronize(s));
    std::vector<cudaIpcMemHandle_t> hs(N);
    CU(cudaMemcpy(hs.data(), hd.p, hb * N, cudaMemcpyDeviceToHost));
    int ok = 1;
    for (int j = 0; j < N; j++) {
        if (j == me) {
            c->ppeer[j] = c->pbuf;
            continue;
        }
        if (cudaIpcOpenMemHandle(&c->ppeer[j], hs[j], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            c->ppeer[j] = nullptr, ok = 0;
        }
    }
    CU(cudaMemcpy(okd.p, &ok, sizeof(int), cudaMemcpyHostToDevice));
    nccl_check(api.all_reduce(okd.p, okd.p, 1, ncclInt32, ncclMin, c->comm, s), "all-reduce (exchange mappings)");
    CU(cudaMemcpyAsync(&ok, okd.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    CU(cudaStreamSynchronize(s));
    c->epoch_q = c->epoch_s = 0;
    if (!ok) {
        for (int j = 0; j < N; j++)
            if (j != me && c->ppeer[j]) cudaIpcCloseMemHandle(c->ppeer[j]);
        c->ppeer.assign(N, nullptr);
        CU(cudaFree(c->pbuf));
        c->pbuf = nullptr, c->p2p = 0;
        return false;
    }
    c->pbytes = bytes, c->p2p = 1;
    return true;
}

// The sharded stage with its exchanges as peer stores (NVLink) instead of collectives. The rows are padded to N
// equal slices of Rs rows, rank j owning rows [j Rs, (j + 1) Rs). Every layer: every rank attends all rows over its
// own chunks (the kernel leaving the merged state of its splits, unnormalised); it stores the states of rank j's rows
// into j's exchange buffer; each rank, once every rank's states have arrived, merges them in rank order
// (k_attend_merge: nn.rs:261-286) and runs the rest of the layer and the next query for its slice, whose queries it
// stores into every rank's query buffer. Per layer and rank: R (d + 2H) floats and R d floats leave, as many arrive.
// Nothing overwrites data still being read: a rank's next stores into a peer need the peer's own next step first.
// False (nothing queued) when peer mappings are not available; the caller then takes the collective path.
static bool stage_sharded_p2p(tcu_ctx *ctx, tcu_model *m, tcu_comm *c, int R, int out_n, cudaStream_t s) {
    const auto &sh = m->w->shape;
    const int d = sh.d, H = sh.heads, L = sh.layers, dff = sh.dec_ff, N = c->nranks, me = c->rank;
    const int Rs = (R + N - 1) / N, Rp = Rs * N, r0 = me * Rs;
    auto a16 = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t off_q = 256, off_ms = off_q + a16(sizeof(float) * (size_t)Rp * d);
    const size_t off_acc = off_ms + a16(sizeof(float) * (size_t)N * Rs * H * 2);
    const size_t bytes = off_acc + a16(sizeof(float) * (size_t)N * Rs * d);
    if (!ensure_peer(c, bytes, s)) return false;
    check_ready(m);
    if (out_n < 1 || out_n > sh.outs) fail(TCU_ERR_ARG, "stage: out_n must be 1..decoder outputs");
    scan_model(ctx, m, ctx->stream);
    ensure_work(m, Rp);
    if (m->out.ensure(sizeof(float) * (size_t)Rp * out_n)) drop_graphs(m);
    m->sh_mall.ensure(sizeof(float) * (size_t)Rp * H * 2);
    uint8_t *base = static_cast<uint8_t *>(c->pbuf);
    float *qbuf = reinterpret_cast<float *>(base + off_q), *rms = reinterpret_cast<float *>(base + off_ms);
    float *racc = reinterpret_cast<float *>(base + off_acc);
    const unsigned *flags_q = reinterpret_cast<unsigned *>(base), *flags_s = flags_q + PUSH_MAX_RANKS;
    const float *scales = m->scales.as<float>();
    float *h = m->h.as<float>(), *att = m->att.as<float>(), *om = m->out.as<float>(), *ms1 = m->sh_mall.as<float>();
    float *hm = h + (size_t)r0 * d, *am = att + (size_t)r0 * d, *qm = qbuf + (size_t)r0 * d;
    Launch ck{ctx, s};
    const long long wait_cycles = 4000000000ll;  // about two seconds at boost clock
    int *err = ctx->err_mapped + ERR_PEER;
    PushArgs pa;
    for (int j = 0; j < N; j++) pa.peer[j] = static_cast<uint8_t *>(c->ppeer[j]);
    pa.done = c->pdone, pa.ranks = N, pa.me = me;
    const int bpd = std::max(1, std::min(32, ctx->sms / std::max(1, N)));  // blocks per destination
    c->marks.clear();
    auto mark = [&](int phase) {
        if (!c->prof) return;
        const size_t i = c->marks.size();
        if (i == c->events.size()) {
            cudaEvent_t e;
            CU(cudaEventCreate(&e));
            c->events.push_back(e);
        }
        CU(cudaEventRecord(c->events[i], s));
        c->marks.push_back(phase);
    };
    // this rank's slice of the queries to every rank, then all of them here
    auto push_q = [&]() {
        mark(5);
        PushArgs a = pa;
        a.segments = 1, a.epoch = ++c->epoch_q, a.flag_off = 0;
        a.src[0] = qm, a.src_step[0] = 0, a.count[0] = (size_t)Rs * d, a.dst_off[0] = off_q + sizeof(float) * (size_t)r0 * d;
        ck(launch_push(a, bpd, s, &ctx->launches), "push (queries)");
        ck(launch_wait_flags(flags_q, N, a.epoch, wait_cycles, err, s, &ctx->launches), "wait (queries)");
    };
    mark(4);
    query_rows(ctx, m, 0, scales, hm, Rs, qm, s);
    push_q();
    for (int l = 0; l < L; l++) {
        mark(0);
        const int parts = attend_layer(ctx, m, layer_ptr(m, l), m->rows, m->chunk, m->kv, m->items.as<int2>(), m->nitems,
                                       m->tiles.as<int4>(), m->ntiles, qbuf, Rp, att, s, m->tc_eK[l], m->tc_eV[l], true,
                                       tc_tiles_of(m, l), ms1);
        mark(1);
        const float *sms = parts == 0 ? ms1 : m->part_ms.as<float>(), *sacc = parts == 0 ? att : m->part_acc.as<float>();
        if (parts > 1) {
            AttnArgs a;
            a.R = Rp, a.heads = H, a.d = d, a.part_ms = m->part_ms.as<float>(), a.part_acc = m->part_acc.as<float>();
            ck(launch_merge_state(a, parts, ms1, att, s, &ctx->launches), "merge (local)");
            sms = ms1, sacc = att;
        }
        // the states of rank j's rows into rank j's buffer, block `me`; then every rank's here
        mark(2);
        PushArgs a = pa;
        a.segments = 2, a.epoch = ++c->epoch_s, a.flag_off = sizeof(unsigned) * PUSH_MAX_RANKS;
        a.src[0] = sms, a.src_step[0] = (size_t)Rs * H * 2, a.count[0] = (size_t)Rs * H * 2;
        a.dst_off[0] = off_ms + sizeof(float) * (size_t)me * Rs * H * 2;
        a.src[1] = sacc, a.src_step[1] = (size_t)Rs * d, a.count[1] = (size_t)Rs * d;
        a.dst_off[1] = off_acc + sizeof(float) * (size_t)me * Rs * d;
        ck(launch_push(a, bpd, s, &ctx->launches), "push (states)");
        ck(launch_wait_flags(flags_s, N, a.epoch, wait_cycles, err, s, &ctx->launches), "wait (states)");
        mark(3);
        AttnArgs b;
        b.R = Rs, b.heads = H, b.d = d, b.part_ms = rms, b.part_acc = racc, b.out = am, b.ldo = d;
        ck(launch_attend_merge(b, N, s, &ctx->launches), "merge (ranks)");
        mark(4);
        block_tail(ctx, m, l, hm, am, Rs, s);
        if (l + 1 < L) {
            query_rows(ctx, m, l + 1, scales + (size_t)(l + 1) * d, hm, Rs, qm, s);
            push_q();
        }
    }
    mark(6);
    linear(ctx, m, hm, d, Rs, d, m->w->lnw, m->w->lnb, m->w->dec0w, m->w->dec0b, dff, m->mid.as<float>(), dff, 1, 0, s, m->w->tdec0);
    linear(ctx, m, m->mid.as<float>(), dff, Rs, dff, nullptr, nullptr, m->w->dec2w, m->w->dec2b, out_n,
           om + (size_t)r0 * out_n, out_n, 0, 0, s, m->w->tdec2);
    nccl_check(nccl_api().all_gather(om + (size_t)r0 * out_n, om, (size_t)Rs * out_n, ncclFloat32, c->comm, s),
               "all-gather (outputs)");
    mark(7);
    return true;
}

// predict.rs:398-409, 521-532 (training rows split over readers, partial states merged by nn.rs:261-286) with the
// readers on separate devices. The rows are split into G groups (two when each rank's slice of a group keeps at least
// 2048 rows, else one: the rest of a layer on fewer rows costs about as much, so splitting smaller calls loses more
// than the overlap wins), each padded to N equal slices of Rs rows (padding rows start at zero); in group g rank j owns rows
// g Rg + [j Rs, (j + 1) Rs), Rg = N Rs. Every layer, every rank attends each group's rows over its own chunks; the
// maxima of the states are all-reduced (max), each rank scales its states to them, and a reduce-scatter (sum) hands
// each rank the summed states of its own slice, which it divides and runs through the rest of the layer and the next
// layer's query; an all-gather gives every rank all of the group's queries. Per layer and rank: R H floats all-reduced,
// R (d + H) reduce-scattered, R d gathered. The compute runs on the caller's stream, the collectives (with the small
// kernels between them) on the communicator's own stream, so that one group's collectives run while the other group
// computes; with timing on (tcu_comm_breakdown) everything runs on the caller's stream, one phase after another.
static void stage_sharded(tcu_ctx *ctx, tcu_model *m, tcu_comm *c, int R, int out_n, cudaStream_t s) {
    if (c->aborted) fail(TCU_ERR_STATE, "communicator was aborted");
    if (stage_sharded_p2p(ctx, m, c, R, out_n, s)) return;
    check_ready(m);
    const auto &sh = m->w->shape;
    const int d = sh.d, H = sh.heads, L = sh.layers, dff = sh.dec_ff, N = c->nranks, me = c->rank;
    if (out_n < 1 || out_n > sh.outs) fail(TCU_ERR_ARG, "stage: out_n must be 1..decoder outputs");
    if (c->aborted) fail(TCU_ERR_STATE, "communicator was aborted");
    const int G = R >= 4096 * N ? 2 : 1;
    const int Rs = (R + G * N - 1) / (G * N), Rg = Rs * N, Rp = Rg * G;
    scan_model(ctx, m, ctx->stream);
    ensure_work(m, Rg);
    ensure_work(m, Rp);
    if (m->out.ensure(sizeof(float) * (size_t)Rp * out_n)) drop_graphs(m);
    const size_t w = (size_t)d + H;
    m->sh_m.ensure(sizeof(float) * (size_t)Rp * H * 2);     // per group: this rank's maxima, then the maxima over ranks
    m->sh_mall.ensure(sizeof(float) * (size_t)Rp * H * 2);  // the merged (max, weight sum) of every row
    m->sh_packed.ensure(sizeof(float) * ((size_t)Rp + (size_t)G * Rs) * w);
    const auto &api = nccl_api();
    const float *scales = m->scales.as<float>();
    float *h = m->h.as<float>(), *q = m->q.as<float>(), *att = m->att.as<float>(), *om = m->out.as<float>();
    const bool serial = c->prof;
    cudaStream_t cs = serial ? s : c->cstream;
    Launch ck{ctx, s}, cc{ctx, cs};
    c->marks.clear();
    auto mark = [&](int phase) {
        if (!c->prof) return;
        const size_t i = c->marks.size();
        if (i == c->events.size()) {
            cudaEvent_t e;
            CU(cudaEventCreate(&e));
            c->events.push_back(e);
        }
        CU(cudaEventRecord(c->events[i], s));
        c->marks.push_back(phase);
    };
    // cross-stream order (nothing to do on one stream): event e marks what `from` has queued so far; `to` waits for it
    auto signal = [&](cudaStream_t from, int e) {
        if (!serial) CU(cudaEventRecord(c->sync[e], from));
    };
    auto wait = [&](cudaStream_t to, int e) {
        if (!serial) CU(cudaStreamWaitEvent(to, c->sync[e], 0));
    };
    enum { EV_INPUT = 0, EV_QUERY = 1, EV_GATHERED = 3, EV_ATTENDED = 5, EV_MERGED = 7, EV_OUTPUT = 9 };
    struct Group {
        float *h, *q, *att, *hm, *qm, *am, *ms, *mloc, *mall, *packed, *mine;
        int parts;
    };
    std::vector<Group> gs(G);
    for (int g = 0; g < G; g++) {
        Group &x = gs[g];
        const size_t o = (size_t)g * Rg;
        x.h = h + o * d, x.q = q + o * d, x.att = att + o * d;
        x.hm = x.h + (size_t)me * Rs * d, x.qm = x.q + (size_t)me * Rs * d, x.am = x.att + (size_t)me * Rs * d;
        x.ms = m->sh_mall.as<float>() + o * H * 2;
        x.mloc = m->sh_m.as<float>() + o * H * 2, x.mall = x.mloc + (size_t)Rg * H;
        x.packed = m->sh_packed.as<float>() + o * w;
        x.mine = m->sh_packed.as<float>() + (size_t)Rp * w + (size_t)g * Rs * w;
    }
    // group g's queries from this rank's slice to every rank, once they are computed on s
    auto gather = [&](int g) {
        signal(s, EV_QUERY + g);
        wait(cs, EV_QUERY + g);
        mark(5);
        nccl_check(api.all_gather(gs[g].qm, gs[g].q, (size_t)Rs * d, ncclFloat32, c->comm, cs), "all-gather (queries)");
        signal(cs, EV_GATHERED + g);
    };
    for (int g = 0; g < G; g++) {
        mark(4);
        query_rows(ctx, m, 0, scales, gs[g].hm, Rs, gs[g].qm, s);
        gather(g);
    }
    for (int l = 0; l < L; l++) {
        // attention of each group (after its queries are gathered), its state then merged on the collective stream
        for (int g = 0; g < G; g++) {
            Group &x = gs[g];
            wait(s, EV_GATHERED + g);
            mark(0);
            x.parts = attend_layer(ctx, m, layer_ptr(m, l), m->rows, m->chunk, m->kv, m->items.as<int2>(), m->nitems,
                                   m->tiles.as<int4>(), m->ntiles, x.q, Rg, x.att, s, m->tc_eK[l], m->tc_eV[l], true,
                                   tc_tiles_of(m, l), x.ms);
            mark(1);
            // the kernel left the merged state (parts 0), or one part is it, or several are merged into one first
            const float *sms = x.parts == 0 ? x.ms : m->part_ms.as<float>(), *sacc = x.parts == 0 ? x.att : m->part_acc.as<float>();
            if (x.parts > 1) {
                AttnArgs a;
                a.R = Rg, a.heads = H, a.d = d, a.part_ms = m->part_ms.as<float>(), a.part_acc = m->part_acc.as<float>();
                ck(launch_merge_state(a, x.parts, x.ms, x.att, s, &ctx->launches), "merge (local)");
                sms = x.ms, sacc = x.att;
            } else if (x.parts == 1) {
                // the parts are reused by the next group's attention: the state moves out of them first
                CU(cudaMemcpyAsync(x.ms, sms, sizeof(float) * Rg * H * 2, cudaMemcpyDeviceToDevice, s));
                CU(cudaMemcpyAsync(x.att, sacc, sizeof(float) * Rg * d, cudaMemcpyDeviceToDevice, s));
                sms = x.ms, sacc = x.att;
            }
            signal(s, EV_ATTENDED + g);
            wait(cs, EV_ATTENDED + g);
            mark(2);
            cc(launch_state_max(sms, Rg, H, x.mloc, cs, &ctx->launches), "merge (maxima)");
            nccl_check(api.all_reduce(x.mloc, x.mall, (size_t)Rg * H, ncclFloat32, ncclMax, c->comm, cs), "all-reduce (max)");
            cc(launch_state_pack(sms, sacc, x.mall, Rg, H, d, x.packed, cs, &ctx->launches), "merge (scale)");
            nccl_check(api.reduce_scatter(x.packed, x.mine, (size_t)Rs * w, ncclFloat32, ncclSum, c->comm, cs), "reduce-scatter (states)");
            mark(3);
            cc(launch_state_finish(x.mine, Rs, H, d, x.am, d, cs, &ctx->launches), "merge (finish)");
            signal(cs, EV_MERGED + g);
        }
        // the rest of the layer and the next query for this rank's slice of each group, its queries then gathered
        for (int g = 0; g < G; g++) {
            Group &x = gs[g];
            wait(s, EV_MERGED + g);
            mark(4);
            block_tail(ctx, m, l, x.hm, x.am, Rs, s);
            if (l + 1 < L) {
                query_rows(ctx, m, l + 1, scales + (size_t)(l + 1) * d, x.hm, Rs, x.qm, s);
                gather(g);
            }
        }
    }
    mark(6);
    for (int g = 0; g < G; g++) {
        Group &x = gs[g];
        float *og = om + (size_t)g * Rg * out_n, *mo = og + (size_t)me * Rs * out_n;
        linear(ctx, m, x.hm, d, Rs, d, m->w->lnw, m->w->lnb, m->w->dec0w, m->w->dec0b, dff, m->mid.as<float>(), dff, 1, 0, s, m->w->tdec0);
        linear(ctx, m, m->mid.as<float>(), dff, Rs, dff, nullptr, nullptr, m->w->dec2w, m->w->dec2b, out_n, mo, out_n, 0, 0, s,
               m->w->tdec2);
    }
    signal(s, EV_OUTPUT);
    wait(cs, EV_OUTPUT);
    for (int g = 0; g < G; g++) {
        float *og = om + (size_t)g * Rg * out_n, *mo = og + (size_t)me * Rs * out_n;
        nccl_check(api.all_gather(mo, og, (size_t)Rs * out_n, ncclFloat32, c->comm, cs), "all-gather (outputs)");
    }
    signal(cs, EV_INPUT);
    wait(s, EV_INPUT);
    mark(7);
}

// fit.rs:577-747 in-memory path on the device. With `scales_in` (host [layers][d]) those query scales are used instead
// of the ones worked out for `rows`; without y, h already carries the target's embedding; with `sink`, every layer's
// keys and values ([rows][d] each, host) are handed to it in layer order (the in_context hook of fit::Attend).
struct LayerSink {
    tcu_layer_sink fn = nullptr;
    void *user = nullptr;
};
static tcu_model *fit_icl(tcu_weights *w, float *h, const float *y, int rows, int chunk, int kv,
                          const float *scales_in = nullptr, LayerSink sink = LayerSink()) {
    tcu_ctx *ctx = w->ctx;
    if (!w->for_fit || !w->ready) fail(TCU_ERR_STATE, "fit: weights must be made with for_fit and be ready");
    if (chunk < 8) chunk = 8;  // fit.rs:226
    ModelPtr m(new tcu_model());
    model_init(m.get(), w, rows, chunk, kv, w->shape.outs);
    const auto &sh = w->shape;
    const int d = sh.d, L = sh.layers;
    cudaStream_t s = ctx->stream;
    ensure_work(m.get(), rows);
    DevBuf kvT, kvf, fit_tiles, fit_items;
    kvT.ensure(sizeof(float) * (size_t)rows * 2 * d);
    kvf.ensure(layer_bytes_of(0, d, rows, chunk));
    // the f32 view's decode items (the few-row attention of a small node reads them): f32 chunking
    const int2 *items = m->items.as<int2>();
    int nitems = m->nitems;
    if (kv != 0) {
        std::vector<int2> it;
        const int ks = decode_keys_per_item(0);
        for (int ci = 0, r0 = 0; r0 < rows; ci++, r0 += chunk)
            for (int k0 = 0; k0 < std::min(chunk, rows - r0); k0 += ks) it.push_back(make_int2(ci, k0));
        fit_items.ensure(it.size() * sizeof(int2));
        CU(cudaMemcpy(fit_items.p, it.data(), it.size() * sizeof(int2), cudaMemcpyHostToDevice));
        items = fit_items.as<int2>(), nitems = (int)it.size();
    }
    Launch ck{ctx, s};
    if (y) ck(launch_add_y(h, y, rows, d, sh.max_classes, w->icl_y, s, &ctx->launches), "add_y");
    DevBuf kvr;
    std::vector<float> hk, hv;
    if (sink.fn) kvr.ensure(sizeof(float) * (size_t)rows * 2 * d), hk.resize((size_t)rows * d), hv.resize((size_t)rows * d);
    // the float view of a layer (for the training rows' own attention) has its own items/tiles: same chunking
    std::vector<float> scales((size_t)L * d);
    for (int l = 0; l < L; l++) {
        const LayerPtrs &p = w->layer[l];
        auto sc = scales_in ? std::vector<float>(scales_in + (size_t)l * d, scales_in + (size_t)(l + 1) * d) : query_scale(w, l, rows);
        std::memcpy(scales.data() + (size_t)l * d, sc.data(), sizeof(float) * d);
        CU(cudaMemcpyAsync(m->scales.as<float>() + (size_t)l * d, sc.data(), sizeof(float) * d, cudaMemcpyHostToDevice, s));
        // keys and values, coordinate-major: kvT[j][r] = Wkv[j] . LN1(h_r) + bkv[j] (fit.rs:633-647)
        linear(ctx, m.get(), h, d, rows, d, p.n1w, p.n1b, p.wkv, p.bkv, 2 * d, kvT.as<float>(), rows, 0, 0, s, p.tkv, 1);
        if (sink.fn) {
            // the same keys and values row by row for the caller: [rows][2d], keys then values of each row
            linear(ctx, m.get(), h, d, rows, d, p.n1w, p.n1b, p.wkv, p.bkv, 2 * d, kvr.as<float>(), 2 * d, 0, 0, s, p.tkv);
            const size_t row = sizeof(float) * d;
            CU(cudaMemcpy2DAsync(hk.data(), row, kvr.p, 2 * row, row, rows, cudaMemcpyDeviceToHost, s));
            CU(cudaMemcpy2DAsync(hv.data(), row, kvr.as<float>() + d, 2 * row, row, rows, cudaMemcpyDeviceToHost, s));
            CU(cudaStreamSynchronize(s));
            if (sink.fn(sink.user, l, hk.data(), hv.data()) != 0) fail(TCU_ERR_ARG, "fit_in_context: the layer sink failed");
        }
        ck(launch_pack(kvT.as<float>(), rows, d, rows, chunk, kv, m->layers.as<uint8_t>() + m->layer_stride * l, s, &ctx->launches), "pack");
        m->have_layer[l] = true;
        if (l + 1 == L) break;  // fit.rs:664-666
        if (kv != 0) ck(launch_pack(kvT.as<float>(), rows, d, rows, chunk, 0, kvf.as<uint8_t>(), s, &ctx->launches), "pack f32");
        const uint8_t *fl = kv == 0 ? layer_ptr(m.get(), l) : kvf.as<uint8_t>();
        int eK = 0, eV = 0;
        scan_layer(ctx, fl, rows, chunk, d, 0, s, eK, eV);
        const void *ft = nullptr;
        if (tc_shape(m.get())) {
            fit_tiles.ensure(tc_layer_bytes(m.get()));
            build_tc_tiles(ctx, m.get(), fl, 0, eK, eV, fit_tiles.p, s);
            ft = fit_tiles.p;
        }
        query_rows(ctx, m.get(), l, m->scales.as<float>() + (size_t)l * d, h, rows, m->q.as<float>(), s);
        // the f32 view has the same chunking, and flash tiles depend only on chunking
        attend_layer(ctx, m.get(), fl, rows, chunk, 0, items, nitems, m->tiles.as<int4>(), m->ntiles, m->q.as<float>(), rows,
                     m->att.as<float>(), s, eK, eV, false, ft);
        block_tail(ctx, m.get(), l, h, m->att.as<float>(), rows, s);
    }
    CU(cudaStreamSynchronize(s));
    check_device_error(ctx);
    m->have_scales = true;
    return m.release();
}

}  // namespace tcu

// ---- C ABI ------------------------------------------------------------------------------------------------------

extern "C" {

int tcu_open(int device, tcu_ctx **out) {
    if (!out) return TCU_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return TCU_ERR_CUDA;
    std::unique_ptr<tcu_ctx> ctx(new tcu_ctx());
    ctx->device = device;
    int r = guarded(ctx.get(), [&]() -> int {
        CU(cudaDeviceGetAttribute(&ctx->sms, cudaDevAttrMultiProcessorCount, device));
        CU(cudaDeviceGetAttribute(&ctx->coop, cudaDevAttrCooperativeLaunch, device));
        int optin = 0;
        CU(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
        ctx->smem_optin = (size_t)optin;
        CU(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
        CU(cudaHostAlloc((void **)&ctx->err_host, ERR_SLOTS * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
        std::memset(ctx->err_host, 0, ERR_SLOTS * sizeof(int));
        CU(cudaHostGetDevicePointer((void **)&ctx->err_mapped, ctx->err_host, 0));
        CU(cudaMalloc(&ctx->dev_scan, 2 * sizeof(unsigned)));
        CU(kernels_init());
        return TCU_OK;
    });
    if (r != TCU_OK) return r;
    *out = ctx.release();
    return TCU_OK;
}

void tcu_close(tcu_ctx *ctx) {
    if (ctx) ctx_release(ctx);
}

const char *tcu_last_error(const tcu_ctx *ctx) { return ctx ? ctx->err.c_str() : "no context"; }

uint64_t tcu_launches(const tcu_ctx *ctx) { return ctx ? ctx->launches : 0; }

int tcu_weights_new(tcu_ctx *ctx, const tcu_icl_shape *shape, int for_fit, tcu_weights **out) {
    return guarded(ctx, [&]() -> int {
        if (!shape || !out) fail(TCU_ERR_ARG, "weights_new: null argument");
        const auto &s = *shape;
        if (s.d <= 0 || s.heads <= 0 || s.d % s.heads || s.layers <= 0 || s.ff <= 0 || s.hid <= 0 || s.dec_ff <= 0 || s.outs <= 0)
            fail(TCU_ERR_ARG, "weights_new: bad shape");
        const int hd = s.d / s.heads;
        if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128) fail(TCU_ERR_ARG, "weights_new: head width must be 8, 16, 32, 64 or 128");
        if (s.d % 4 || s.ff % 4 || s.dec_ff % 4) fail(TCU_ERR_ARG, "weights_new: widths must be multiples of 4");
        auto *w = new tcu_weights();
        w->ctx = ctx, w->shape = s, w->for_fit = for_fit != 0;
        ctx->refs++;
        *out = w;
        return TCU_OK;
    });
}

int tcu_weights_put(tcu_weights *w, const char *name, int dtype, const void *data, size_t count) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!name || (!data && count)) fail(TCU_ERR_ARG, "weights_put: null argument");
        if (w->ready) fail(TCU_ERR_STATE, "weights_put: weights already uploaded");
        std::vector<float> v(count);
        if (dtype == 0)
            std::memcpy(v.data(), data, count * sizeof(float));
        else if (dtype == 1)
            for (size_t i = 0; i < count; i++) v[i] = f16_to_f32(reinterpret_cast<const uint16_t *>(data)[i]);
        else
            fail(TCU_ERR_ARG, "weights_put: dtype must be 0 (float32) or 1 (float16)");
        w->host[name] = std::move(v);
        return TCU_OK;
    });
}

int tcu_weights_ready(tcu_weights *w) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int { return weights_ready(w); });
}

int tcu_weights_from_bundle(tcu_ctx *ctx, const char *path, int for_fit, tcu_weights **out) {
    return guarded(ctx, [&]() -> int {
        if (!path || !out) fail(TCU_ERR_ARG, "weights_from_bundle: null argument");
        auto b = Bundle::open(path);
        auto cfgb = b->bytes("config.json");
        std::string cfg(cfgb.begin(), cfgb.end());
        // model.rs:204-219: only the TabICLv2 layout this path implements
        const char *want[][2] = {{"col_feature_group", "same"}, {"col_affine", "false"}, {"col_target_aware", "true"},
                                 {"col_ssmax", "qassmax-mlp-elementwise"}, {"icl_ssmax", "qassmax-mlp-elementwise"},
                                 {"row_rope_interleaved", "false"}, {"norm_first", "true"}, {"activation", "gelu"}};
        for (auto &kv : want) {
            std::string got = cfg_value(cfg, kv[0]);
            if (got != kv[1]) fail(TCU_ERR_FORMAT, std::string("unsupported checkpoint: ") + kv[0] + " is " + got + ", this backend implements " + kv[1]);
        }
        auto num = [&](const char *k) {
            std::string v = cfg_value(cfg, k);
            char *end = nullptr;
            long x = std::strtol(v.c_str(), &end, 10);
            if (v.empty() || *end) fail(TCU_ERR_FORMAT, std::string("config has no number ") + k);
            return (int)x;
        };
        tcu_icl_shape s{};
        s.heads = num("icl_nhead"), s.layers = num("icl_num_blocks"), s.max_classes = num("max_classes");
        s.d = (int)b->entry("icl_predictor.ln.weight").len();
        s.ff = (int)b->entry(blk(0, "linear1.bias")).len();
        s.hid = (int)b->entry(blk(0, "attn.ssmax_layer.query_mlp.0.bias")).len();
        s.dec_ff = (int)b->entry("icl_predictor.decoder.0.bias").len();
        s.outs = (int)b->entry("icl_predictor.decoder.2.bias").len();
        tcu_weights *w = nullptr;
        int r = tcu_weights_new(ctx, &s, for_fit, &w);
        if (r != TCU_OK) return r;
        WeightsPtr guard(w);
        const bool rows = b->has("col_embedder.in_linear.weight") && b->has("row_interactor.cls_tokens");
        if (rows) {
            // model.rs:220-244: the column and row stages' sizes
            tcu_rows_shape rs{};
            rs.e = (int)b->entry("col_embedder.in_linear.bias").len();
            rs.group = num("col_feature_group_size"), rs.inds = num("col_num_inds"), rs.cls = num("row_num_cls");
            rs.col_heads = num("col_nhead"), rs.row_heads = num("row_nhead");
            rs.col_blocks = num("col_num_blocks"), rs.row_blocks = num("row_num_blocks");
            rs.col_ff = (int)b->entry("col_embedder.tf_col.blocks.0.multihead_attn2.linear1.bias").len();
            rs.row_ff = (int)b->entry("row_interactor.tf_row.blocks.0.linear1.bias").len();
            r = tcu_weights_set_rows_shape(w, &rs);
            if (r != TCU_OK) return r;
        }
        for (const auto &e : b->entries()) {
            const bool want = e.name.rfind("icl_predictor.", 0) == 0 ||
                              (rows && (e.name.rfind("col_embedder.", 0) == 0 || e.name.rfind("row_interactor.", 0) == 0));
            if (want && (e.dtype == "float32" || e.dtype == "float16")) w->host[e.name] = b->f32s(e.name);
        }
        weights_ready(w);
        *out = guard.release();
        return TCU_OK;
    });
}

int tcu_weights_shape(const tcu_weights *w, tcu_icl_shape *out) {
    if (!w || !out) return TCU_ERR_ARG;
    *out = w->shape;
    return TCU_OK;
}

int tcu_weights_set_rows_shape(tcu_weights *w, const tcu_rows_shape *shape) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!shape) fail(TCU_ERR_ARG, "set_rows_shape: null argument");
        if (w->ready) fail(TCU_ERR_STATE, "set_rows_shape: weights already uploaded");
        const auto &s = *shape;
        if (s.e <= 0 || s.group < 1 || s.group > 8 || s.inds < 1 || s.cls < 1 || s.col_heads < 1 || s.row_heads < 1 ||
            s.e % s.col_heads || s.e % s.row_heads || (s.e / s.row_heads) % 2 || s.col_blocks < 1 || s.row_blocks < 1 ||
            s.col_ff < 1 || s.row_ff < 1 || s.e % 4)
            fail(TCU_ERR_ARG, "set_rows_shape: bad shape");
        if (s.cls * s.e != w->shape.d) fail(TCU_ERR_ARG, "set_rows_shape: class tokens times width must be the in-context width");
        w->rows.shape = s, w->rows.on = true;
        return TCU_OK;
    });
}

int tcu_weights_rows_shape(const tcu_weights *w, tcu_rows_shape *out) {
    if (!w || !out) return TCU_ERR_ARG;
    if (!w->rows.on) return TCU_DECLINED;
    *out = w->rows.shape;
    return TCU_OK;
}

void tcu_weights_free(tcu_weights *w) {
    if (w) weights_release(w);
}

int tcu_model_new(tcu_weights *w, const int32_t meta[7], int32_t node_rows, int32_t node_k, tcu_model **out) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!meta || !out) fail(TCU_ERR_ARG, "model_new: null argument");
        if (!w->ready) fail(TCU_ERR_STATE, "model_new: weights not ready");
        ModelPtr m(new tcu_model());
        // meta = [rows, features, classes, chunk, kv, digits, nodes] (fit.rs:291)
        if (meta[4] < 0 || meta[4] > 2) fail(TCU_ERR_FORMAT, "meta: unknown key/value format " + std::to_string(meta[4]));
        model_init(m.get(), w, node_rows, meta[3], meta[4], node_k);
        m->features = meta[1];
        m->digits = std::max(1, (int)meta[5]), m->nodes = std::max(1, (int)meta[6]);
        *out = m.release();
        return TCU_OK;
    });
}

int tcu_model_put_scales(tcu_model *m, const float *scales, size_t count) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        const size_t want = (size_t)m->w->shape.layers * m->w->shape.d;
        if (!scales || count != want) fail(TCU_ERR_ARG, "model_put_scales: expected layers * d floats");
        CU(cudaMemcpy(m->scales.p, scales, sizeof(float) * want, cudaMemcpyHostToDevice));
        m->have_scales = true;
        return TCU_OK;
    });
}

int tcu_model_put_layer(tcu_model *m, int layer, size_t offset, const void *bytes, size_t nbytes) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        if (layer < 0 || layer >= m->w->shape.layers) fail(TCU_ERR_ARG, "model_put_layer: no such layer");
        if (!bytes || offset + nbytes > m->layer_bytes) fail(TCU_ERR_ARG, "model_put_layer: range past the layer's " + std::to_string(m->layer_bytes) + " bytes");
        CU(cudaMemcpy(m->layers.as<uint8_t>() + m->layer_stride * layer + offset, bytes, nbytes, cudaMemcpyHostToDevice));
        if (offset + nbytes == m->layer_bytes) m->have_layer[layer] = true;
        m->tc_scanned = false;
        return TCU_OK;
    });
}

}  // extern "C"

namespace tcu {

static constexpr size_t STAGING_BYTES = 8u << 20;

// The context's staging buffers and upload stream, made at the first upload (with upload_mu held).
static void ensure_staging(tcu_ctx *ctx) {
    if (ctx->upload_stream) return;
    CU(cudaStreamCreateWithFlags(&ctx->upload_stream, cudaStreamNonBlocking));
    for (int i = 0; i < 2; i++) {
        CU(cudaHostAlloc(&ctx->pin[i], STAGING_BYTES, cudaHostAllocPortable));
        CU(cudaEventCreateWithFlags(&ctx->pin_ev[i], cudaEventDisableTiming));
    }
}

// Copy `n` bytes to device memory `dst`, the pieces produced by read(piece, offset, len) into alternating pinned
// buffers: a buffer is refilled only after its previous copy has landed, so reading and copying overlap. Returns with
// every copy landed.
template <typename Read>
static void staged_upload(tcu_ctx *ctx, void *dst, size_t n, Read read) {
    std::lock_guard<std::mutex> lk(ctx->upload_mu);
    ensure_staging(ctx);
    int i = 0;
    for (size_t off = 0; off < n; off += STAGING_BYTES, i ^= 1) {
        const size_t len = std::min(STAGING_BYTES, n - off);
        CU(cudaEventSynchronize(ctx->pin_ev[i]));
        read(ctx->pin[i], off, len);
        CU(cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, ctx->pin[i], len, cudaMemcpyHostToDevice, ctx->upload_stream));
        CU(cudaEventRecord(ctx->pin_ev[i], ctx->upload_stream));
    }
    CU(cudaStreamSynchronize(ctx->upload_stream));
}

static void upload_tensor(tcu_ctx *ctx, const Bundle &b, const std::string &name, void *dst, size_t n) {
    staged_upload(ctx, dst, n, [&](void *buf, size_t off, size_t len) { b.read_bytes_at(name, off, buf, len); });
}

static void upload_host(tcu_ctx *ctx, const void *src, void *dst, size_t n) {
    staged_upload(ctx, dst, n, [&](void *buf, size_t off, size_t len) { std::memcpy(buf, static_cast<const uint8_t *>(src) + off, len); });
}

static size_t col_kv_floats(const tcu_model *m) {
    const auto &rs = m->w->rows.shape;
    return (size_t)m->features * m->digits * rs.col_blocks * 2 * rs.e * rs.inds;
}

struct NodeMeta {
    std::vector<int32_t> meta;
    std::vector<TreeNode> tree;
};

static NodeMeta node_meta(const Bundle &b, const std::string &p) {
    NodeMeta nm{b.i32s(p + "meta"), {}};
    if (nm.meta.size() != 7) fail(TCU_ERR_FORMAT, p + "meta is damaged");
    if (nm.meta[4] < 0 || nm.meta[4] > 2) fail(TCU_ERR_FORMAT, "meta: unknown key/value format " + std::to_string(nm.meta[4]));
    auto tree = b.i32s(p + "tree");
    nm.tree = parse_tree(tree.data(), tree.size(), nm.meta[6]);
    return nm;
}

MemberInfo member_info(const Bundle &b, const std::string &p) {
    auto nm = node_meta(b, p);
    return MemberInfo{std::max(1, (int)nm.meta[6]), std::max(1, (int)nm.meta[5])};
}

tcu_ctx *ctx_of(const tcu_weights *w) {
    CU(cudaSetDevice(w->ctx->device));
    return w->ctx;
}

bool has_col(const tcu_model *m) { return m->col_kv.p != nullptr; }

tcu_ctx *ctx_of_weights(const tcu_weights *w) { return w->ctx; }

size_t node_bytes(const tcu_weights *w, const Bundle &b, const std::string &p, int node, bool with_col) {
    auto nm = node_meta(b, p);
    if (node < 0 || node >= (int)nm.tree.size()) fail(TCU_ERR_ARG, "no such node");
    const size_t col = with_col && w->rows.on && b.has(p + "col_kv") ? b.entry(p + "col_kv").len() : 0;
    return model_bytes_of(w, nm.tree[node].rows, std::max(1, (int)nm.meta[3]), nm.meta[4], col);
}

tcu_model *load_node(tcu_weights *w, const Bundle &b, const std::string &p, int node, bool with_col) {
    tcu_ctx *ctx = ctx_of(w);
    auto nm = node_meta(b, p);
    const auto &meta = nm.meta;
    if (node < 0 || node >= (int)nm.tree.size()) fail(TCU_ERR_ARG, "model_from_bundle: no such node");
    ModelPtr m(new tcu_model());
    {
        // creation touches the weights' reference count and the context's tables: under the lock; the uploads not
        std::lock_guard<std::recursive_mutex> lk(ctx->mu);
        if (!w->ready) fail(TCU_ERR_STATE, "model_from_bundle: weights not ready");
        model_init(m.get(), w, nm.tree[node].rows, meta[3], meta[4], nm.tree[node].k);
        m->features = meta[1];
        m->digits = std::max(1, (int)meta[5]), m->nodes = std::max(1, (int)meta[6]);
    }
    const int L = w->shape.layers, d = w->shape.d;
    auto sc = b.f32s(p + "n" + std::to_string(node) + "_scale");
    if (sc.size() != (size_t)L * d) fail(TCU_ERR_FORMAT, p + "n" + std::to_string(node) + "_scale: expected layers * d floats");
    upload_host(ctx, sc.data(), m->scales.p, sizeof(float) * sc.size());
    m->have_scales = true;
    if (with_col && w->rows.on && b.has(p + "col_kv")) {
        const std::string name = p + "col_kv";
        const Entry &e = b.entry(name);
        const size_t want = col_kv_floats(m.get());
        if (e.len() != want || m->features < 1) fail(TCU_ERR_FORMAT, name + ": expected features * digits * column blocks * 2 * e * inducing points = " + std::to_string(want) + " floats");
        m->col_kv.ensure(sizeof(float) * want);
        if (e.dtype == "float32") {
            upload_tensor(ctx, b, name, m->col_kv.p, sizeof(float) * want);
        } else {
            auto v = b.f32s(name);
            upload_host(ctx, v.data(), m->col_kv.p, sizeof(float) * want);
        }
    }
    for (int l = 0; l < L; l++) {
        const std::string name = p + "n" + std::to_string(node) + "_kv" + std::to_string(l);
        const Entry &e = b.entry(name);
        if (e.nbytes != m->layer_bytes) fail(TCU_ERR_FORMAT, name + ": " + std::to_string(e.nbytes) + " bytes, expected " + std::to_string(m->layer_bytes));
        upload_tensor(ctx, b, name, m->layers.as<uint8_t>() + m->layer_stride * l, m->layer_bytes);
        m->have_layer[l] = true;
    }
    return m.release();
}

}  // namespace tcu

extern "C" {

int tcu_model_from_bundle(tcu_weights *w, const char *path, const char *prefix, int node, tcu_model **out) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!path || !prefix || !out) fail(TCU_ERR_ARG, "model_from_bundle: null argument");
        auto b = Bundle::open(path);
        *out = load_node(w, *b, prefix, node, true);
        return TCU_OK;
    });
}

size_t tcu_model_bytes(const tcu_model *m) {
    if (!m) return 0;
    // what the model will hold, its lazily built copies and tables included: a budget charged at load time holds
    return model_bytes_of(m->w, m->rows, m->chunk, m->kv, m->col_kv.bytes / sizeof(float));
}

int tcu_model_set_columns(tcu_model *m, int features, int digits) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        if (features < 1 || digits < 1) fail(TCU_ERR_ARG, "model_set_columns: features and digits must be positive");
        if (m->col_kv.p) fail(TCU_ERR_STATE, "model_set_columns: the column cache is already put");
        m->features = features, m->digits = digits;
        return TCU_OK;
    });
}

int tcu_model_put_col_kv(tcu_model *m, const float *col_kv, size_t count) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        const RowsWeights &rw = m->w->rows;
        if (!rw.on) fail(TCU_ERR_STATE, "model_put_col_kv: the weights have no column and row stages");
        const auto &rs = rw.shape;
        const size_t per_feature = (size_t)m->digits * rs.col_blocks * 2 * rs.e * rs.inds;
        // a cache fitted on the device does not know its features: the column cache says how many
        if (m->features < 1 && count % per_feature == 0) m->features = (int)(count / per_feature);
        const size_t want = (size_t)m->features * per_feature;
        if (!col_kv || count != want || m->features < 1)
            fail(TCU_ERR_ARG, "model_put_col_kv: expected features * digits * column blocks * 2 * e * inducing points = " +
                                  std::to_string(want) + " floats");
        m->col_kv.ensure(sizeof(float) * want);
        CU(cudaMemcpy(m->col_kv.p, col_kv, sizeof(float) * want, cudaMemcpyHostToDevice));
        return TCU_OK;
    });
}

int tcu_embed_device(tcu_model *m, const float *x, int rows, float *tok, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (rows < 0 || (rows && (!x || !tok))) fail(TCU_ERR_ARG, "embed: bad argument");
        if (rows == 0) return TCU_OK;
        embed(ctx, m, x, rows, tok, stream ? (cudaStream_t)stream : ctx->stream);
        return TCU_OK;
    });
}

int tcu_represent_device(tcu_model *m, float *tok, int rows, float *rep, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (rows < 0 || (rows && (!tok || !rep))) fail(TCU_ERR_ARG, "represent: bad argument");
        if (rows == 0) return TCU_OK;
        represent(ctx, m, tok, rows, rep, stream ? (cudaStream_t)stream : ctx->stream);
        return TCU_OK;
    });
}

int tcu_rows_device(tcu_model *m, const float *x, int rows, int out_n, float *out, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (rows < 0 || (rows && (!x || !out))) fail(TCU_ERR_ARG, "rows: bad argument");
        if (rows == 0) return TCU_OK;
        cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        rows_stage(ctx, m, x, rows, out_n, s);
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * (size_t)rows * out_n, cudaMemcpyDeviceToDevice, s));
        return TCU_OK;
    });
}

int tcu_rows(tcu_model *m, const float *x, int rows, int features, int out_n, float *out) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (features != m->features) fail(TCU_ERR_ARG, "rows: features differ from the cache's " + std::to_string(m->features));
        if (rows < 0 || (rows && (!x || !out))) fail(TCU_ERR_ARG, "rows: bad argument");
        if (rows == 0) return TCU_OK;
        check_rows_ready(m);
        cudaStream_t s = ctx->stream;
        const size_t n = (size_t)rows * features;
        m->cin.ensure(sizeof(float) * n);
        CU(cudaMemcpyAsync(m->cin.p, x, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        rows_stage(ctx, m, m->cin.as<float>(), rows, out_n, s);
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * (size_t)rows * out_n, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_model_get_layer(const tcu_model *m, int layer, void *bytes, size_t nbytes) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        if (layer < 0 || layer >= m->w->shape.layers || nbytes != m->layer_bytes || !bytes) fail(TCU_ERR_ARG, "model_get_layer: bad layer or size");
        CU(cudaMemcpy(bytes, layer_ptr(m, layer), nbytes, cudaMemcpyDeviceToHost));
        return TCU_OK;
    });
}

int tcu_model_get_scales(const tcu_model *m, float *scales, size_t count) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        const size_t want = (size_t)m->w->shape.layers * m->w->shape.d;
        if (!scales || count != want) fail(TCU_ERR_ARG, "model_get_scales: expected layers * d floats");
        CU(cudaMemcpy(scales, m->scales.p, sizeof(float) * want, cudaMemcpyDeviceToHost));
        return TCU_OK;
    });
}

void tcu_model_free(tcu_model *m) {
    if (!m) return;
    tcu_weights *w = m->w;
    {
        std::lock_guard<std::recursive_mutex> lock(w->ctx->mu);
        cudaSetDevice(w->ctx->device);
        delete m;
    }
    weights_release(w);
}

int tcu_attend_device(tcu_model *m, int layer, const float *q, int rows, float *out, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);  // an earlier call's kernels that gave up are reported by the next call
        check_ready(m);
        if (layer < 0 || layer >= m->w->shape.layers || rows < 0 || (rows && (!q || !out))) fail(TCU_ERR_ARG, "attend: bad argument");
        if (rows == 0) return TCU_OK;
        cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        scan_model(ctx, m, ctx->stream);
        ensure_work(m, rows);
        attend_layer(ctx, m, layer_ptr(m, layer), m->rows, m->chunk, m->kv, m->items.as<int2>(), m->nitems, m->tiles.as<int4>(),
                     m->ntiles, q, rows, out, s, m->tc_eK[layer], m->tc_eV[layer], false, tc_tiles_of(m, layer));
        return TCU_OK;
    });
}

int tcu_stage_device(tcu_model *m, const float *h, int rows, int out_n, float *out, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (rows < 0 || (rows && (!h || !out))) fail(TCU_ERR_ARG, "stage: bad argument");
        if (rows == 0) return TCU_OK;
        cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        check_ready(m);
        if (out_n < 1 || out_n > m->w->shape.outs) fail(TCU_ERR_ARG, "stage: out_n must be 1..decoder outputs");
        const size_t n = (size_t)rows * m->w->shape.d;
        if (m->h.ensure(sizeof(float) * n)) drop_graphs(m);
        CU(cudaMemcpyAsync(m->h.p, h, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
        stage_replay(ctx, m, rows, out_n, s);
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * (size_t)rows * out_n, cudaMemcpyDeviceToDevice, s));
        return TCU_OK;
    });
}

int tcu_attend(tcu_model *m, int layer, const float *q, int rows, int d, int heads, float *out) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (d != m->w->shape.d || heads != m->w->shape.heads) fail(TCU_ERR_ARG, "attend: d or heads differ from the weights'");
        if (rows < 0 || (rows && (!q || !out))) fail(TCU_ERR_ARG, "attend: bad argument");
        if (rows == 0) return TCU_OK;
        check_ready(m);
        const size_t n = (size_t)rows * d;
        m->h.ensure(sizeof(float) * n);
        m->out.ensure(sizeof(float) * n);
        cudaStream_t s = ctx->stream;
        CU(cudaMemcpyAsync(m->h.p, q, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        int r = tcu_attend_device(m, layer, m->h.as<float>(), rows, m->out.as<float>(), s);
        if (r != TCU_OK) return r;
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_stage(tcu_model *m, const float *h, int rows, int d, int out_n, float *out) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (d != m->w->shape.d) fail(TCU_ERR_ARG, "stage: d differs from the weights'");
        if (rows < 0 || (rows && (!h || !out))) fail(TCU_ERR_ARG, "stage: bad argument");
        if (rows == 0) return TCU_OK;
        check_ready(m);
        if (out_n < 1 || out_n > m->w->shape.outs) fail(TCU_ERR_ARG, "stage: out_n must be 1..decoder outputs");
        if (m->h.ensure(sizeof(float) * (size_t)rows * d)) drop_graphs(m);
        cudaStream_t s = ctx->stream;
        CU(cudaMemcpyAsync(m->h.p, h, sizeof(float) * (size_t)rows * d, cudaMemcpyHostToDevice, s));
        stage_replay(ctx, m, rows, out_n, s);
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * (size_t)rows * out_n, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_class_head_device(tcu_ctx *ctx, const float *logits, int rows, int classes, int stride,
                          const int32_t *member_classes, double *sums, int finish, int members, double temperature) {
    return guarded(ctx, [&]() -> int {
        if (rows < 0 || classes < 1 || stride < classes || (rows && (!logits || !member_classes || !sums))) fail(TCU_ERR_ARG, "class_head: bad argument");
        if (finish && (members < 1 || !(temperature > 0))) fail(TCU_ERR_ARG, "class_head: members and temperature must be positive");
        if (rows == 0) return TCU_OK;
        Launch{ctx, ctx->stream}(launch_class_head(logits, rows, classes, stride, member_classes, sums, finish, members, temperature,
                                                   ctx->stream, &ctx->launches),
                                 "class head");
        CU(cudaStreamSynchronize(ctx->stream));
        return TCU_OK;
    });
}

int tcu_regression_head_device(tcu_ctx *ctx, const float *qout, int rows, int nq, int stride, const double *alphas,
                               int na, double target_mean, double target_scale, double *mean, double *variance,
                               double *median, double *quantiles) {
    return guarded(ctx, [&]() -> int {
        if (rows < 0 || nq < 2 || nq > 4096 || stride < nq || na < 0) fail(TCU_ERR_ARG, "regression_head: bad sizes (2 <= nq <= 4096)");
        if (rows && (!qout || !mean || !variance || !median || (na && (!alphas || !quantiles)))) fail(TCU_ERR_ARG, "regression_head: null argument");
        if (rows == 0) return TCU_OK;
        Launch{ctx, ctx->stream}(launch_regression_head(qout, rows, nq, stride, alphas, na, target_mean, target_scale, mean, variance,
                                                        median, quantiles, ctx->stream, &ctx->launches),
                                 "regression head");
        CU(cudaStreamSynchronize(ctx->stream));
        return TCU_OK;
    });
}

int tcu_fit_icl_device(tcu_weights *w, float *h, const float *y, int rows, int chunk, int kv, tcu_model **out) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!h || !y || !out || rows < 1 || kv < 0 || kv > 2) fail(TCU_ERR_ARG, "fit_icl: bad argument");
        *out = fit_icl(w, h, y, rows, chunk, kv);
        return TCU_OK;
    });
}

int tcu_fit_rows_device(tcu_weights *w, const float *x, const float *y, int rows, int features, int digits,
                        const int32_t *bases, float *col_kv, float *rep, void *stream) {
    if (!w) return TCU_ERR_ARG;
    tcu_ctx *ctx = w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (!x || !y || !col_kv || !rep || rows < 1 || features < 1 || digits < 1 || (digits > 1 && !bases))
            fail(TCU_ERR_ARG, "fit_rows: bad argument");
        if (!w->ready) fail(TCU_ERR_STATE, "fit_rows: weights not ready");
        const cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        // working memory only (no cache): freed on return
        std::unique_ptr<tcu_model> sc(new tcu_model());
        sc->w = w, sc->features = features, sc->digits = digits;
        const auto &rs = w->rows.shape;
        DevBuf tok;
        tok.ensure(sizeof(float) * (size_t)rows * (rs.cls + features) * rs.e);
        fit_columns(ctx, sc.get(), x, y, rows, features, digits, bases, col_kv, tok.as<float>(), s);
        fit_rows(ctx, sc.get(), tok.as<float>(), rows, features, rep, s);
        check_device_error(ctx);
        return TCU_OK;
    });
}

// Working memory the fit's column and row stages may take per call (the hooks size their batches by it).
static constexpr size_t FIT_WORK_BYTES = (size_t)16 << 30;

int tcu_fit_column_batch(const tcu_weights *w, int rows) {
    if (!w || rows < 1 || !w->ready || !w->rows.on || !w->rows.fit) return 0;
    const auto &rs = w->rows.shape;
    const size_t wide = std::max(rs.e, rs.col_ff);
    // per cell: the cells, their keys and values, attention, hidden units, split rows (two f16 halves)
    const size_t per_cell = sizeof(float) * (4 * (size_t)rs.e + rs.col_ff + wide);
    return (int)std::max<size_t>(1, std::min<size_t>(1 << 20, FIT_WORK_BYTES / per_cell / (size_t)rows));
}

int tcu_fit_columns(tcu_weights *w, float *cells, int rows, int groups, const float *ind_q, float *rec) {
    if (!w) return TCU_ERR_ARG;
    tcu_ctx *ctx = w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (!cells || !ind_q || !rec || rows < 1 || groups < 1) fail(TCU_ERR_ARG, "fit_columns: bad argument");
        if (!w->ready) fail(TCU_ERR_STATE, "fit_columns: weights not ready");
        check_fit_weights(w);
        const auto &rs = w->rows.shape;
        const cudaStream_t s = ctx->stream;
        const size_t M = (size_t)rows * groups, per = (size_t)2 * rs.e * rs.inds, nq = (size_t)rs.col_blocks * rs.inds * rs.e;
        std::unique_ptr<tcu_model> sc(new tcu_model());
        sc->w = w, sc->features = groups;
        DevBuf iq, out;
        sc->cx.ensure(sizeof(float) * M * rs.e), iq.ensure(sizeof(float) * nq);
        out.ensure(sizeof(float) * groups * rs.col_blocks * per);
        CU(cudaMemcpyAsync(sc->cx.p, cells, sizeof(float) * M * rs.e, cudaMemcpyHostToDevice, s));
        CU(cudaMemcpyAsync(iq.p, ind_q, sizeof(float) * nq, cudaMemcpyHostToDevice, s));
        column_blocks(ctx, sc.get(), sc->cx.as<float>(), rows, groups, iq.as<float>(), out.as<float>(), rs.col_blocks * per, 0, s);
        CU(cudaMemcpyAsync(cells, sc->cx.p, sizeof(float) * M * rs.e, cudaMemcpyDeviceToHost, s));
        CU(cudaMemcpyAsync(rec, out.p, out.bytes, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_fit_row_batch(const tcu_weights *w, int features) {
    if (!w || features < 1 || !w->ready || !w->rows.on) return 0;
    const auto &rs = w->rows.shape;
    const size_t T = (size_t)rs.cls + features, wide = std::max(rs.e, rs.row_ff);
    // per row: its tokens, their projections, attention, new tokens, hidden units, split rows
    const size_t per_row = sizeof(float) * T * (6 * (size_t)rs.e + rs.row_ff + wide);
    return (int)std::max<size_t>(1, std::min<size_t>(1 << 16, FIT_WORK_BYTES / per_row));
}

int tcu_fit_rows(tcu_weights *w, const float *cells, int n, int features, float *reps) {
    if (!w) return TCU_ERR_ARG;
    tcu_ctx *ctx = w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (!cells || !reps || n < 1 || features < 1) fail(TCU_ERR_ARG, "fit_rows: bad argument");
        if (!w->ready) fail(TCU_ERR_STATE, "fit_rows: weights not ready");
        check_rows_weights(w);
        const auto &rs = w->rows.shape;
        const cudaStream_t s = ctx->stream;
        const size_t M = (size_t)n * features, d = w->shape.d;
        std::unique_ptr<tcu_model> sc(new tcu_model());
        sc->w = w, sc->features = features;
        DevBuf x, tok, rep;
        x.ensure(sizeof(float) * M * rs.e), tok.ensure(sizeof(float) * (size_t)n * (rs.cls + features) * rs.e);
        rep.ensure(sizeof(float) * n * d);
        CU(cudaMemcpyAsync(x.p, cells, sizeof(float) * M * rs.e, cudaMemcpyHostToDevice, s));
        Launch{ctx, s}(launch_tokens(x.as<float>(), w->rows.cls_tokens, n, features, rs.cls, rs.e, tok.as<float>(), s,
                                     &ctx->launches),
                       "tokens");
        fit_rows(ctx, sc.get(), tok.as<float>(), n, features, rep.as<float>(), s);
        CU(cudaMemcpy(reps, rep.p, sizeof(float) * n * d, cudaMemcpyDeviceToHost));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_fit_in_context(tcu_weights *w, const float *h, int rows, const float *scales, tcu_layer_sink sink, void *user) {
    if (!w) return TCU_ERR_ARG;
    tcu_ctx *ctx = w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (!h || !scales || !sink || rows < 1) fail(TCU_ERR_ARG, "fit_in_context: bad argument");
        const size_t n = (size_t)rows * w->shape.d;
        DevBuf hd;
        hd.ensure(sizeof(float) * n);
        CU(cudaMemcpy(hd.p, h, sizeof(float) * n, cudaMemcpyHostToDevice));
        // the stored form is not asked for: the cache the pass keeps on the way is f32 in chunks of 256 rows
        ModelPtr m(fit_icl(w, hd.as<float>(), nullptr, rows, 256, 0, scales, LayerSink{sink, user}));
        return TCU_OK;
    });
}

int tcu_pack_device(tcu_ctx *ctx, int kv, int d, int rc, const float *c, void *rec) {
    return guarded(ctx, [&]() -> int {
        if (kv < 0 || kv > 2 || d < 1 || rc < 1 || !c || !rec) fail(TCU_ERR_ARG, "pack: bad argument");
        Launch{ctx, ctx->stream}(launch_pack(c, rc, d, rc, rc, kv, reinterpret_cast<uint8_t *>(rec), ctx->stream, &ctx->launches), "pack");
        CU(cudaStreamSynchronize(ctx->stream));
        return TCU_OK;
    });
}

size_t tcu_record(int kv, int d, int rc) { return record_bytes(kv, d, rc); }

int tcu_layer_rows_device(tcu_ctx *ctx, int kv, int d, const void *layer, int rows, int chunk, float *k, float *v) {
    return guarded(ctx, [&]() -> int {
        if (kv < 0 || kv > 2 || d < 4 || d % 4 || rows < 1 || chunk < 1 || !layer || !k || !v)
            fail(TCU_ERR_ARG, "layer_rows: bad argument");
        if ((uintptr_t)layer & 3) fail(TCU_ERR_ARG, "layer_rows: layer must be 4-byte aligned");
        Launch{ctx, ctx->stream}(launch_layer_rows(kv, reinterpret_cast<const uint8_t *>(layer), rows, chunk, d, k, v,
                                                   ctx->stream, &ctx->launches),
                                 "layer_rows");
        CU(cudaStreamSynchronize(ctx->stream));
        return TCU_OK;
    });
}

int tcu_selftest_mma(tcu_ctx *ctx, double *max_err) {
    return guarded(ctx, [&]() -> int {
        if (!max_err) fail(TCU_ERR_ARG, "selftest: null argument");
        float *res = nullptr;
        CU(cudaMalloc(&res, 2 * sizeof(float)));
        cudaError_t e = launch_tc_selftest(res, ctx->stream);
        unsigned bits[2] = {0, 0};
        if (e == cudaSuccess) e = cudaMemcpyAsync(bits, res, sizeof(bits), cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        cudaFree(res);
        CU(e);
        float worst;
        std::memcpy(&worst, &bits[0], 4);
        *max_err = bits[1] ? -1.0 : (double)worst;
        return TCU_OK;
    });
}

int tcu_comm_unique_id(uint8_t id[TCU_COMM_ID_BYTES]) {
    if (!id) return TCU_ERR_ARG;
    const auto &api = nccl_api();
    if (!api.why.empty()) return TCU_ERR_STATE;
    static_assert(sizeof(ncclUniqueId) == TCU_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    if (api.get_unique_id(&u) != ncclSuccess) return TCU_ERR_CUDA;
    std::memcpy(id, &u, sizeof(u));
    return TCU_OK;
}

int tcu_comm_init(tcu_ctx *ctx, const uint8_t id[TCU_COMM_ID_BYTES], int nranks, int rank, tcu_comm **out) {
    return guarded(ctx, [&]() -> int {
        if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks) fail(TCU_ERR_ARG, "comm_init: bad argument");
        const auto &api = nccl_api();
        if (!api.why.empty()) fail(TCU_ERR_STATE, api.why);
        std::unique_ptr<tcu_comm> c(new tcu_comm());
        c->ctx = ctx, c->nranks = nranks, c->rank = rank;
        ncclUniqueId u;
        std::memcpy(&u, id, sizeof(u));
        nccl_check(api.comm_init_rank(&c->comm, nranks, u, rank), "comm_init");
        CU(cudaStreamCreateWithFlags(&c->cstream, cudaStreamNonBlocking));
        for (auto &e : c->sync) CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        ctx->refs++;  // released by tcu_comm_free
        *out = c.release();
        return TCU_OK;
    });
}

void tcu_comm_free(tcu_comm *c) {
    if (!c) return;
    tcu_ctx *ctx = c->ctx;
    {
        std::lock_guard<std::recursive_mutex> lock(ctx->mu);
        cudaSetDevice(ctx->device);
        if (c->comm) (c->aborted ? nccl_api().comm_abort : nccl_api().comm_destroy)(c->comm);
        for (auto e : c->events) cudaEventDestroy(e);
        for (auto e : c->sync)
            if (e) cudaEventDestroy(e);
        for (size_t j = 0; j < c->ppeer.size(); j++)
            if ((int)j != c->rank && c->ppeer[j]) cudaIpcCloseMemHandle(c->ppeer[j]);
        if (c->pbuf) cudaFree(c->pbuf);
        if (c->pdone) cudaFree(c->pdone);
        if (c->cstream) cudaStreamDestroy(c->cstream);
        delete c;
    }
    ctx_release(ctx);
}

int tcu_comm_abort(tcu_comm *c) {
    if (!c) return TCU_ERR_ARG;
    return guarded(c->ctx, [&]() -> int {
        if (c->comm) nccl_api().comm_abort(c->comm);
        c->comm = nullptr, c->aborted = true;
        return TCU_OK;
    });
}

int tcu_comm_allreduce_f64(tcu_comm *c, double *buf, size_t count, void *stream) {
    if (!c) return TCU_ERR_ARG;
    return guarded(c->ctx, [&]() -> int {
        if (!buf && count) fail(TCU_ERR_ARG, "allreduce: null buffer");
        if (c->aborted) fail(TCU_ERR_STATE, "communicator was aborted");
        cudaStream_t s = stream ? (cudaStream_t)stream : c->ctx->stream;
        nccl_check(nccl_api().all_reduce(buf, buf, count, ncclFloat64, ncclSum, c->comm, s), "all-reduce (f64)");
        return TCU_OK;
    });
}

int tcu_comm_wait(tcu_comm *c, void *stream, int timeout_ms) {
    if (!c) return TCU_ERR_ARG;
    return guarded(c->ctx, [&]() -> int {
        cudaStream_t s = stream ? (cudaStream_t)stream : c->ctx->stream;
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            const cudaError_t e = cudaStreamQuery(s);
            if (e == cudaSuccess) return TCU_OK;
            if (e != cudaErrorNotReady) CU(e);
            if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
                // a rank that never arrives leaves NCCL's kernels waiting: aborting the communicator ends them
                nccl_api().comm_abort(c->comm);
                c->comm = nullptr, c->aborted = true;
                fail(TCU_ERR_CUDA, "collective did not complete within " + std::to_string(timeout_ms) + " ms; communicator aborted");
            }
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    });
}

int tcu_model_slice(const tcu_model *m, int first_chunk, int nchunks, tcu_model **out) {
    if (!m) return TCU_ERR_ARG;
    return guarded(m->w->ctx, [&]() -> int {
        const int total = (m->rows + m->chunk - 1) / m->chunk;
        if (!out || first_chunk < 0 || nchunks < 1 || first_chunk + nchunks > total) fail(TCU_ERR_ARG, "model_slice: chunk range outside the cache");
        check_ready(m);
        const int r0 = first_chunk * m->chunk, r1 = std::min(m->rows, (first_chunk + nchunks) * m->chunk);
        ModelPtr s(new tcu_model());
        model_init(s.get(), m->w, r1 - r0, m->chunk, m->kv, m->classes);
        s->features = m->features;
        const auto &sh = m->w->shape;
        for (int l = 0; l < sh.layers; l++) {
            // whole chunk records: a shard's bytes are one contiguous range of the layer
            CU(cudaMemcpy(s->layers.as<uint8_t>() + s->layer_stride * l, layer_ptr(m, l) + (size_t)first_chunk * m->full,
                          s->layer_bytes, cudaMemcpyDeviceToDevice));
            s->have_layer[l] = true;
        }
        CU(cudaMemcpy(s->scales.p, m->scales.p, sizeof(float) * (size_t)sh.layers * sh.d, cudaMemcpyDeviceToDevice));
        s->have_scales = true;
        *out = s.release();
        return TCU_OK;
    });
}

int tcu_comm_breakdown(tcu_comm *c, int enable, double *ms) {
    if (!c) return TCU_ERR_ARG;
    return guarded(c->ctx, [&]() -> int {
        if (ms) {
            for (int i = 0; i < TCU_SHARD_PHASES; i++) ms[i] = 0.0;
            const size_t n = c->marks.size();
            if (n > 1) {
                CU(cudaEventSynchronize(c->events[n - 1]));
                for (size_t k = 0; k + 1 < n; k++) {
                    float t = 0.f;
                    CU(cudaEventElapsedTime(&t, c->events[k], c->events[k + 1]));
                    if (c->marks[k] >= 0 && c->marks[k] < TCU_SHARD_PHASES) ms[c->marks[k]] += t;
                }
            }
        }
        c->prof = enable != 0;
        return TCU_OK;
    });
}

int tcu_stage_sharded_device(tcu_model *m, tcu_comm *c, const float *h, int rows, int out_n, float *out, void *stream) {
    if (!m || !c) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->w->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (c->ctx != ctx) fail(TCU_ERR_ARG, "stage_sharded: communicator and cache belong to different contexts");
        if (rows < 0 || (rows && (!h || !out))) fail(TCU_ERR_ARG, "stage_sharded: bad argument");
        if (rows == 0) return TCU_OK;
        cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        const size_t n = (size_t)rows * m->w->shape.d;
        // the rows padded to equal slices (in one or two groups, as stage_sharded splits them), the padding rows zero
        const int G = rows >= 4096 * c->nranks ? 2 : 1;
        const size_t np = (size_t)((rows + G * c->nranks - 1) / (G * c->nranks)) * G * c->nranks * m->w->shape.d;
        if (m->h.ensure(sizeof(float) * np)) drop_graphs(m);
        CU(cudaMemcpyAsync(m->h.p, h, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
        if (np > n) CU(cudaMemsetAsync(m->h.as<float>() + n, 0, sizeof(float) * (np - n), s));
        stage_sharded(ctx, m, c, rows, out_n, s);
        CU(cudaMemcpyAsync(out, m->out.p, sizeof(float) * (size_t)rows * out_n, cudaMemcpyDeviceToDevice, s));
        return TCU_OK;
    });
}

int tcu_member_new(tcu_model *const *nodes, int n_nodes, const int32_t *tree, size_t tree_len, int classes,
                   tcu_member **out) {
    if (!nodes || n_nodes < 1 || !nodes[0]) return TCU_ERR_ARG;
    tcu_ctx *ctx = nodes[0]->w->ctx;
    return guarded(ctx, [&]() -> int {
        if (!tree || !out || classes < 1) fail(TCU_ERR_ARG, "member_new: bad argument");
        std::unique_ptr<tcu_member> mb(new tcu_member());
        mb->ctx = ctx, mb->classes = classes;
        mb->tree = parse_tree(tree, tree_len, n_nodes);
        for (int i = 0; i < n_nodes; i++) {
            tcu_model *m = nodes[i];
            if (!m || m->w != nodes[0]->w) fail(TCU_ERR_ARG, "member_new: every node needs the same weights");
            if (mb->tree[i].k > m->w->shape.outs)
                fail(TCU_ERR_ARG, "member_new: node " + std::to_string(i) + " has " + std::to_string(mb->tree[i].k) +
                                      " outputs, more than the decoder's " + std::to_string(m->w->shape.outs));
            for (int j = 0; j < i; j++)
                if (nodes[j] == m) fail(TCU_ERR_ARG, "member_new: a node is given twice");
        }
        member_tables(mb.get());
        mb->nodes.assign(nodes, nodes + n_nodes);  // owned from here on
        *out = mb.release();
        return TCU_OK;
    });
}

int tcu_member_from_bundle(tcu_weights *w, const char *path, const char *prefix, tcu_member **out) {
    if (!w) return TCU_ERR_ARG;
    return guarded(w->ctx, [&]() -> int {
        if (!path || !prefix || !out) fail(TCU_ERR_ARG, "member_from_bundle: null argument");
        auto b = Bundle::open(path);
        const std::string p(prefix);
        auto meta = b->i32s(p + "meta");
        auto tree = b->i32s(p + "tree");
        if (meta.size() != 7) fail(TCU_ERR_FORMAT, p + "meta is damaged");
        std::unique_ptr<tcu_member> mb(new tcu_member());
        mb->ctx = w->ctx, mb->classes = meta[2];
        mb->tree = parse_tree(tree.data(), tree.size(), meta[6]);
        member_tables(mb.get());
        std::vector<ModelPtr> nodes;
        for (int i = 0; i < meta[6]; i++) nodes.emplace_back(load_node(w, *b, p, i, i == 0));
        for (auto &n : nodes) mb->nodes.push_back(n.release());
        *out = mb.release();
        return TCU_OK;
    });
}

int tcu_member_nodes(const tcu_member *m) { return m ? (int)m->nodes.size() : 0; }
int tcu_member_classes(const tcu_member *m) { return m ? m->classes : 0; }
tcu_model *tcu_member_node(tcu_member *m, int node) {
    return m && node >= 0 && node < (int)m->nodes.size() ? m->nodes[node] : nullptr;
}

size_t tcu_member_bytes(const tcu_member *m) {
    if (!m) return 0;
    size_t n = m->tnodes.bytes + m->tmap.bytes;
    for (auto *x : m->nodes) n += tcu_model_bytes(x);
    return n;
}

int tcu_member_rows_device(tcu_member *m, const float *x, int rows, float *out, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        if (rows < 0 || (rows && (!x || !out))) fail(TCU_ERR_ARG, "member_rows: bad argument");
        if (rows == 0) return TCU_OK;
        cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
        const float *res = member_rows(ctx, m, x, rows, s);
        CU(cudaMemcpyAsync(out, res, sizeof(float) * (size_t)rows * m->classes, cudaMemcpyDeviceToDevice, s));
        return TCU_OK;
    });
}

int tcu_member_rows(tcu_member *m, const float *x, int rows, int features, float *out) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->ctx;
    return guarded(ctx, [&]() -> int {
        check_device_error(ctx);
        tcu_model *m0 = m->nodes[0];
        if (features != m0->features) fail(TCU_ERR_ARG, "member_rows: features differ from the cache's " + std::to_string(m0->features));
        if (rows < 0 || (rows && (!x || !out))) fail(TCU_ERR_ARG, "member_rows: bad argument");
        if (rows == 0) return TCU_OK;
        check_rows_ready(m0);
        cudaStream_t s = ctx->stream;
        const size_t n = (size_t)rows * features;
        m0->cin.ensure(sizeof(float) * n);
        CU(cudaMemcpyAsync(m0->cin.p, x, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        const float *res = member_rows(ctx, m, m0->cin.as<float>(), rows, s);
        CU(cudaMemcpyAsync(out, res, sizeof(float) * (size_t)rows * m->classes, cudaMemcpyDeviceToHost, s));
        CU(cudaStreamSynchronize(s));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_member_combine_device(tcu_member *m, const float *scores, int rows, float *out, void *stream) {
    if (!m) return TCU_ERR_ARG;
    tcu_ctx *ctx = m->ctx;
    return guarded(ctx, [&]() -> int {
        if (rows < 0 || (rows && (!scores || !out))) fail(TCU_ERR_ARG, "member_combine: bad argument");
        if (rows == 0) return TCU_OK;
        member_combine(ctx, m, scores, rows, out, stream ? (cudaStream_t)stream : ctx->stream);
        return TCU_OK;
    });
}

void tcu_member_free(tcu_member *m) {
    if (!m) return;
    std::vector<tcu_model *> nodes;
    nodes.swap(m->nodes);
    {
        std::lock_guard<std::recursive_mutex> lock(m->ctx->mu);
        cudaSetDevice(m->ctx->device);
        delete m;
    }
    // each node lets go of the weights (and they of the context) after the member's own buffers are gone
    for (auto *x : nodes) tcu_model_free(x);
}

int tcu_sync(tcu_ctx *ctx, void *stream) {
    return guarded(ctx, [&]() -> int {
        CU(cudaStreamSynchronize(stream ? (cudaStream_t)stream : ctx->stream));
        check_device_error(ctx);
        return TCU_OK;
    });
}

int tcu_debug_abort_next(tcu_ctx *ctx) {
    return guarded(ctx, [&]() -> int {
        ctx->abort_next = true;
        return TCU_OK;
    });
}

int tcu_profile(tcu_ctx *ctx, int enable, double *attend_ms, uint64_t *attend_launches) {
    return guarded(ctx, [&]() -> int {
        if (attend_ms || attend_launches) {
            CU(cudaDeviceSynchronize());
            double ms = 0;
            for (size_t i = 0; i + 1 < ctx->prof_used; i += 2) {
                float t = 0;
                CU(cudaEventElapsedTime(&t, ctx->prof_events[i], ctx->prof_events[i + 1]));
                ms += t;
            }
            if (attend_ms) *attend_ms = ms;
            if (attend_launches) *attend_launches = ctx->prof_used / 2;
        }
        ctx->prof = enable != 0;
        ctx->prof_used = 0;
        return TCU_OK;
    });
}

}  // extern "C"
