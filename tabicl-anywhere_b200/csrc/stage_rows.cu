// The in-context stage (src/predict.rs:381-586) for up to 8 query rows as ONE persistent kernel: one CTA per SM,
// all resident (cooperative launch), the phases of each layer separated by grid barriers.
//
//   A  q = Wq LN1(h) + bq                   (nn.rs:130-137; outputs spread over the CTAs)
//   B  the query MLP of the scalable softmax (nn.rs:138-149) for this CTA's head, then attention over its share
//      of the head's key tiles with the online softmax (nn.rs:187-258), leaving one partial state per CTA
//   C  att = the log-sum-exp merge of each head's partial states (nn.rs:261-286), outputs spread over the CTAs
//   D  h += Wo att + bo                     (predict.rs:542-551)
//   E  mid = GELU(W1 LN2(h) + b1)           (predict.rs:552-559)
//   F  h += W2 mid + b2                     (predict.rs:560-568)
//   then the decoder (predict.rs:570-584).
//
// Few rows are latency-bound: each phase is a few microseconds of dependent work. What the kernel overlaps is the
// cache stream. Every CTA owns a fixed share of each layer's key tiles and keeps a ring of them in shared memory,
// filled by the tensor memory accelerator: one thread starts two tensor loads (keys, values) and two bulk copies
// (their scales) per tile, completing on the slot's mbarrier. A slot is refilled with the next tile of the CTA's
// sequence as soon as it has been used, so the next layer's keys and values arrive while phases D, E, F and A of
// this layer run. Loads that do
// not depend on a barrier (weight rows, biases, LayerNorm and query-MLP weights) are issued before it. Every grid
// barrier is bounded: one that does not complete within about a second sets the error flag, and every CTA then
// leaves at its next barrier.
#include "kernels.cuh"
#include "device.cuh"
#include "stage_common.cuh"
#include "tc.cuh"

#include <algorithm>
#include <cfloat>
#include <mutex>

namespace tcu {

namespace {

constexpr int THREADS = 256, WARPS = 8;
constexpr int HID = 64;                       // hidden width of the query MLP (nn.rs:124)
constexpr int KMAX = 1024;                    // widest input of a linear phase
constexpr long long SPIN_LIMIT = 2000000000;  // cycles, about a second
constexpr int TCACHE = 96;                    // a CTA's tile descriptors kept in shared memory

template <int KV, int HD, int RM>
struct Cfg : TileFmt<KV, HD> {
    using F = TileFmt<KV, HD>;
    using F::W, F::VB, F::EPV, F::TK, F::ROWB, F::DPT, F::SLOT;
    static constexpr int BMAX = RM == 1 ? 8 : 1;  // tiles under one softmax step
    static constexpr int BT = BMAX * TK;
    // scratch (floats), shared by the linear phases and the attention phase
    static constexpr int QH = 0, QM = QH + RM * HD, RED = QM + RM * HD, PSM = RED + WARPS * RM * BT,
                         HS = PSM + RM * BT, ALPHA = HS + RM * HID, LENS = ALPHA + 8, BMS = LENS + 8,
                         ATT_END = BMS + 16;
    static constexpr int XS = 0, LNW = RM * KMAX, LNB = LNW + KMAX, LRED = LNB + KMAX, LIN_END = LRED + 2 * WARPS;
    static constexpr int SCRATCH = ATT_END > LIN_END ? ATT_END : LIN_END;
    static_assert(WARPS * TK >= 4 * HID && WARPS * TK >= 256, "reduction scratch too small for the query MLP");
};

// Grid barrier on a counter zeroed before the launch, in two halves. arrive(): after a phase's stores, one thread per
// CTA adds one (release). wait(): one thread waits (acquire) until the counter reaches G times the barrier's number.
// Work that neither reads what other CTAs write in the phase nor writes what they read (loads of weights, copies
// of key tiles) goes between the two. The wait is bounded: false (for the whole CTA) when it gave up or another CTA
// raised the error flag.
__device__ __forceinline__ void grid_arrive(const RowsArgs &a, unsigned &target) {
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    }
}
__device__ bool grid_wait(const RowsArgs &a, unsigned target, int *flag_s) {
    if (threadIdx.x == 0) {
        const long long t0 = clock64();
        int ok = 1;
        while (ld_acquire_u32(a.bar) < target) {
            if (ld_relaxed_s32(a.err) != 0) {
                // another CTA gave up (or the launch was started aborted): leave, and say why
                if (a.err_report) reinterpret_cast<volatile int *>(a.err_report)[2] = 1;
                ok = 0;
                break;
            }
            if (clock64() - t0 > SPIN_LIMIT) {
                atomicExch(a.err, 1);
                if (a.err_report) reinterpret_cast<volatile int *>(a.err_report)[0] = 1;
                ok = 0;
                break;
            }
        }
        *flag_s = ok;
    }
    __syncthreads();
    return *flag_s != 0;
}

template <int KV, int HD, int RM>
struct Stage {
    using C = Cfg<KV, HD, RM>;
    const RowsArgs &a;
    const RowsLayer *lay;  // the per-layer pointers, in shared memory
    const int4 *tcache;    // this CTA's tile descriptors (the first TCACHE), in shared memory
    uint8_t *ring;
    uint64_t *mbar;
    float *scr;
    int *flag_s;
    int head;             // the head whose tiles this CTA holds
    int t0, n, total;     // this CTA's tiles [t0, t0 + n) of every layer; total = L n tiles in its sequence
    int consumed = 0;     // next tile of the sequence to use
    int issued = 0;       // tiles of the sequence whose copies have started (at most consumed + slots)
    // kept step by step instead of divided out: consumed's slot; issued's layer, index in its layer and slot
    int cons_s = 0, iss_l = 0, iss_i = 0, iss_s = 0;
    unsigned phase = 0;   // per slot, the parity of its mbarrier's next phase
    unsigned target = 0;  // the grid barrier's latest target
    uint64_t pol_kv, pol_w;

    __device__ Stage(const RowsArgs &a_, uint8_t *smem_in, int *flag, const RowsLayer *lay_, const int4 *tcache_)
        : a(a_), lay(lay_), tcache(tcache_), flag_s(flag) {
        // tensor loads want 128-byte aligned destinations
        uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_in) + 127) & ~(uintptr_t)127);
        ring = smem;
        mbar = reinterpret_cast<uint64_t *>(smem + (size_t)a.slots * C::SLOT);
        scr = reinterpret_cast<float *>(smem + (size_t)a.slots * C::SLOT + 128);
        // G / heads CTAs per head; CTA c takes an equal share of head c / (G / heads)'s tiles (head-major list)
        const int per = gridDim.x / a.heads, i = blockIdx.x % per, Th = a.tiles_per_head;
        head = blockIdx.x / per;
        t0 = head * Th + (int)((long long)Th * i / per);
        n = head * Th + (int)((long long)Th * (i + 1) / per) - t0;
        total = a.L * n;
        pol_kv = policy_evict_first();
        pol_w = policy_evict_last();
    }

    // Descriptor of this CTA's tile i of a layer.
    __device__ __forceinline__ int4 tile_at(int i) const { return i < TCACHE ? tcache[i] : a.tiles[t0 + i]; }
    __device__ __forceinline__ int4 tile_of(int g) const { return tile_at(g % n); }
    // Slot s + b of the ring (b < slots).
    __device__ __forceinline__ int slot_add(int s, int b) const { return s + b >= a.slots ? s + b - a.slots : s + b; }
    __device__ __forceinline__ void arrive() { grid_arrive(a, target); }
    __device__ __forceinline__ bool wait() {
        mark();
        const bool r = grid_wait(a, target, flag_s);
        mark();
        return r;
    }
    int nmark = 0;
    __device__ __forceinline__ void mark() {
        if (a.trace && threadIdx.x == 0 && nmark < ROWS_TRACE_MARKS) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            a.trace[(size_t)blockIdx.x * ROWS_TRACE_MARKS + nmark++] = t;
        }
    }
    // Start the copies of the next tiles of the sequence, up to `limit`, into the slots that are free.
    __device__ void issue_upto(int limit) {
        limit = min(limit, min(total, consumed + a.slots));
        for (; issued < limit; issued++) {
            issue(iss_l, iss_i, iss_s);
            if (++iss_i == n) iss_i = 0, iss_l++;
            iss_s = slot_add(iss_s, 1);
        }
    }

    // Thread 0: start the loads of tile i of layer l into slot s (tiles whose rows are not 16-byte aligned are copied
    // when used instead).
    __device__ void issue(int l, int i, int s) {
        if (threadIdx.x != 0) return;
        const int4 tl = tile_at(i);
        if (!(tl.w >> 16)) return;
        const int h = tl.w & 0xffff, ci = tl.x, x = tl.y * C::W;
        const uint8_t *rec = lay[l].cache + (size_t)ci * a.full;
        uint8_t *slot = ring + (size_t)s * C::SLOT;
        uint64_t *mb = mbar + s;
        // no proxy fence: the slot was only read (ordinary loads, done before the CTA barrier that freed it); a proxy
        // fence here would wait for every copy still in flight, so that the tiles would arrive one after another
        mbar_expect_tx(mb, 2u * HD * C::ROWB + (KV ? 8u * HD : 0u));
        const uint8_t *maps = reinterpret_cast<const uint8_t *>(a.tmaps) + (size_t)l * 256;
        if (ci < a.nfull) {
            tma_load3(slot, maps, x, h * HD, ci, mb, pol_kv);
            tma_load3(slot + HD * C::ROWB, maps, x, a.d + h * HD, ci, mb, pol_kv);
        } else {
            tma_load2(slot, maps + 128, x, h * HD, mb, pol_kv);
            tma_load2(slot + HD * C::ROWB, maps + 128, x, a.d + h * HD, mb, pol_kv);
        }
        if (KV) {
            bulk_load(slot + 2 * HD * C::ROWB, rec + (size_t)h * HD * 4, HD * 4, mb, pol_kv);
            bulk_load(slot + 2 * HD * C::ROWB + 4 * HD, rec + ((size_t)a.d + h * HD) * 4, HD * 4, mb, pol_kv);
        }
    }

    // All threads: wait for the next nb tiles to use, tiles i0.. of layer l in the slots from cons_s (thread b waits on
    // tile b's mbarrier, the CTA barrier below passes the completed copies on to the other threads); then copy those
    // that could not be copied asynchronously.
    __device__ bool acquire(int l, int i0, int nb) {
        bool ok = true;
        for (int b = 0; b < nb; b++) {
            const int s = slot_add(cons_s, b);
            const int4 tl = tile_at(i0 + b);
            if (tl.w >> 16) {
                if (threadIdx.x == b) ok = tc::mbar_wait(mbar + s, (phase >> s) & 1u, SPIN_LIMIT);
                phase ^= 1u << s;
            } else {
                copy_now(l, s, tl);
            }
        }
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) {
                atomicExch(a.err, 1);
                if (a.err_report) reinterpret_cast<volatile int *>(a.err_report)[1] = 1;
            }
            return false;
        }
        return true;
    }

    __device__ void copy_now(int l, int s, const int4 &tl) {
        // rows not 16-byte aligned: element copies by all threads
        const int h = tl.w & 0xffff, ci = tl.x, k0 = tl.y, len = tl.z;
        const int rc = min(a.chunk, a.rows - ci * a.chunk);
        const uint8_t *rec = lay[l].cache + (size_t)ci * a.full;
        const uint8_t *body = rec + (KV ? 8 * (size_t)a.d : 0);
        uint8_t *slot = ring + (size_t)s * C::SLOT;
        for (int i = threadIdx.x; i < 2 * HD * len; i += THREADS) {
            const int row = i / len, e = i - row * len;
            const int coord = row < HD ? h * HD + row : a.d + h * HD + (row - HD);
            const uint8_t *src = body + ((size_t)coord * rc + k0 + e) * C::W;
            uint8_t *dst = slot + (size_t)row * C::ROWB + e * C::W;
            if (C::W == 4)
                *reinterpret_cast<uint32_t *>(dst) = __ldg(reinterpret_cast<const uint32_t *>(src));
            else if (C::W == 2)
                *reinterpret_cast<uint16_t *>(dst) = __ldg(reinterpret_cast<const unsigned short *>(src));
            else
                *dst = __ldg(src);
        }
        if (KV) {
            float *sc = reinterpret_cast<float *>(slot + 2 * HD * C::ROWB);
            const float *ks = reinterpret_cast<const float *>(rec);
            for (int i = threadIdx.x; i < 2 * HD; i += THREADS)
                sc[i] = __ldg(ks + (i < HD ? h * HD + i : a.d + h * HD + (i - HD)));
        }
    }

    // Leaving early: wait (bounded) for this CTA's loads still in flight.
    __device__ void drain() {
        for (int g = consumed; g < issued; g++) {
            if (!(tile_of(g).w >> 16)) continue;
            const int s = g % a.slots;
            tc::mbar_wait(mbar + s, (phase >> s) & 1u, SPIN_LIMIT);
            phase ^= 1u << s;
        }
    }

    // One linear phase: y[r][o] (=|+=) act(W[o] . LN?(x[r]) + b[o]) for this CTA's outputs o (a contiguous share of
    // N), one warp per output; the lanes hold 4-float pieces k = 4 lane + 128 v of the weight row, as the few-row
    // linear kernel does, so both give the same sums. The first output's weights, its bias and the LayerNorm weights
    // are loaded before the barrier (when `wait`) that makes x ready; x (rows written by other CTAs in this launch)
    // is read through L2.
    __device__ bool linear(bool LN, bool wait_first, const float *x, int K, const float *lnw, const float *lnb,
                           const float *W, const float *b, int N, int act, float *y, int ldy, bool residual) {
        float *xs = scr + C::XS, *lw_s = scr + C::LNW, *lb_s = scr + C::LNB;
        const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, R = a.R;
        const int n0 = (int)((long long)N * blockIdx.x / gridDim.x), n1 = (int)((long long)N * (blockIdx.x + 1) / gridDim.x);
        const int nv = K >> 7;  // K is a multiple of 128, at most KMAX
        float4 wv[KMAX / 128];
        float bias = 0.f;
        int o = n0 + warp;
        if (o < n1) {
            const float *wr = W + (size_t)o * K + lane * 4;
#pragma unroll
            for (int v = 0; v < KMAX / 128; v++)
                if (v < nv) wv[v] = ld_weight4(wr + v * 128, pol_w);
            if (b) bias = b[o];
        }
        float lw[KMAX / THREADS], lb[KMAX / THREADS];
        if (LN) {
#pragma unroll
            for (int i = 0; i < KMAX / THREADS; i++)
                if (tid + i * THREADS < K) lw[i] = lnw[tid + i * THREADS], lb[i] = lnb[tid + i * THREADS];
        }
        if (wait_first && !wait()) return false;
        const int k4 = K >> 2;
        for (int i = tid; i < R * k4; i += THREADS) {
            const int r = i / k4, c = i - r * k4;
            reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(x + (size_t)r * K) + c);
        }
        if (LN) {
#pragma unroll
            for (int i = 0; i < KMAX / THREADS; i++)
                if (tid + i * THREADS < K) lw_s[tid + i * THREADS] = lw[i], lb_s[tid + i * THREADS] = lb[i];
        }
        __syncthreads();
        if (LN && RM == 1) {
            // kern.rs:357-376 for the one row, by all warps: mean, then the mean square deviation, then the scaling
            float *lred = scr + C::LRED;
            float sum = 0.f;
            for (int k = tid; k < K; k += THREADS) sum += xs[k];
            sum = warp_sum(sum);
            if (lane == 0) lred[warp] = sum;
            __syncthreads();
            const float mean = (((lred[0] + lred[1]) + (lred[2] + lred[3])) + ((lred[4] + lred[5]) + (lred[6] + lred[7]))) / (float)K;
            float q = 0.f;
            for (int k = tid; k < K; k += THREADS) {
                const float dd = xs[k] - mean;
                q = fmaf(dd, dd, q);
            }
            q = warp_sum(q);
            if (lane == 0) lred[WARPS + warp] = q;
            __syncthreads();
            const float *lq = lred + WARPS;
            const float var = (((lq[0] + lq[1]) + (lq[2] + lq[3])) + ((lq[4] + lq[5]) + (lq[6] + lq[7]))) / (float)K;
            const float inv = 1.0f / sqrtf(var + 1e-5f);
            for (int k = tid; k < K; k += THREADS) xs[k] = (xs[k] - mean) * inv * lw_s[k] + lb_s[k];
            __syncthreads();
        } else if (LN) {
            // kern.rs:357-376, as the few-row linear kernel computes it
            for (int r = warp; r < R; r += WARPS) {
                float *row = xs + r * K;
                float s = 0.f;
                for (int k = lane; k < K; k += 32) s += row[k];
                const float mean = warp_sum(s) / (float)K;
                float q = 0.f;
                for (int k = lane; k < K; k += 32) {
                    const float dd = row[k] - mean;
                    q = fmaf(dd, dd, q);
                }
                const float inv = 1.0f / sqrtf(warp_sum(q) / (float)K + 1e-5f);
                for (int k = lane; k < K; k += 32) row[k] = (row[k] - mean) * inv * lw_s[k] + lb_s[k];
            }
            __syncthreads();
        }
        for (bool first = true; o < n1; o += WARPS, first = false) {
            if (!first) {
                const float *wr = W + (size_t)o * K + lane * 4;
#pragma unroll
                for (int v = 0; v < KMAX / 128; v++)
                    if (v < nv) wv[v] = ld_weight4(wr + v * 128, pol_w);
                bias = b ? b[o] : 0.f;
            }
            float acc[RM];
#pragma unroll
            for (int r = 0; r < RM; r++) acc[r] = 0.f;
#pragma unroll
            for (int v = 0; v < KMAX / 128; v++) {
                if (v < nv) {
#pragma unroll
                    for (int r = 0; r < RM; r++) {
                        if (r < R) {
                            const float4 xv = *reinterpret_cast<const float4 *>(xs + r * K + lane * 4 + v * 128);
                            acc[r] = fmaf(wv[v].x, xv.x, acc[r]);
                            acc[r] = fmaf(wv[v].y, xv.y, acc[r]);
                            acc[r] = fmaf(wv[v].z, xv.z, acc[r]);
                            acc[r] = fmaf(wv[v].w, xv.w, acc[r]);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RM; r++) acc[r] = warp_sum(acc[r]);
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < RM; r++) {
                    if (r < R) {
                        float v = acc[r] + bias;
                        if (act) v = gelu1(v);
                        float *dst = y + (size_t)r * ldy + o;
                        *dst = residual ? __ldcg(dst) + v : v;
                    }
                }
            }
        }
        arrive();
        return true;
    }

    // Registers of the query MLP for one head, loaded ahead of use.
    struct QueryW {
        float4 w0[HD / 16];       // hidden unit tid % 64, coordinates (tid / 64) HD/4 + [0, HD/4)
        float4 w2[HID * HD / 1024];  // coordinate tid % HD, hidden units (tid / HD) 64 HD/256 + [0, 64 HD/256)
        float b0, b2, sc;
    };
    __device__ void query_load(const RowsLayer &Ly, int h, QueryW &w) {
        const int tid = threadIdx.x, u = tid & (HID - 1), p = tid >> 6, j = tid % HD, p2 = tid / HD;
        constexpr int QJ = HD / 4, QU = HID * HD / THREADS;
#pragma unroll
        for (int i = 0; i < QJ / 4; i++) w.w0[i] = ld_weight4(Ly.q0w + (size_t)u * HD + p * QJ + 4 * i, pol_w);
#pragma unroll
        for (int i = 0; i < QU / 4; i++) w.w2[i] = ld_weight4(Ly.q2w + (size_t)j * HID + p2 * QU + 4 * i, pol_w);
        w.b0 = Ly.q0b[u];
        w.b2 = Ly.q2b[j];
        w.sc = Ly.scale[h * HD + j];
    }

    // The query MLP of the scalable softmax for head h (nn.rs:138-149): qm = q_h * scale_h * (1 + tanh(m)).
    __device__ void query_head(int h, const QueryW &w) {
        float *qh = scr + C::QH, *qm = scr + C::QM, *red = scr + C::RED, *hs = scr + C::HS;
        const int tid = threadIdx.x, R = a.R, d = a.d;
        constexpr int QJ = HD / 4, P2 = THREADS / HD, QU = HID / P2;
        for (int i = tid; i < RM * HD; i += THREADS) {
            const int r = i / HD, j = i - r * HD;
            qh[i] = r < R ? __ldcg(a.q + (size_t)r * d + h * HD + j) : 0.f;
        }
        __syncthreads();
        {
            const int u = tid & (HID - 1), p = tid >> 6;
            float acc[RM];
#pragma unroll
            for (int r = 0; r < RM; r++) acc[r] = 0.f;
#pragma unroll
            for (int i = 0; i < QJ / 4; i++) {
#pragma unroll
                for (int r = 0; r < RM; r++) {
                    const float4 xv = *reinterpret_cast<const float4 *>(qh + r * HD + p * QJ + 4 * i);
                    acc[r] = fmaf(w.w0[i].x, xv.x, acc[r]);
                    acc[r] = fmaf(w.w0[i].y, xv.y, acc[r]);
                    acc[r] = fmaf(w.w0[i].z, xv.z, acc[r]);
                    acc[r] = fmaf(w.w0[i].w, xv.w, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < RM; r++) red[(p * RM + r) * HID + u] = acc[r];
        }
        __syncthreads();
        for (int i = tid; i < RM * HID; i += THREADS) {
            const int r = i / HID, u = i - r * HID;  // u = tid % 64: this thread's b0
            const float s = (red[(0 * RM + r) * HID + u] + red[(1 * RM + r) * HID + u]) +
                            (red[(2 * RM + r) * HID + u] + red[(3 * RM + r) * HID + u]);
            hs[i] = gelu1(s + w.b0);
        }
        __syncthreads();
        {
            const int j = tid % HD, p2 = tid / HD;
            float acc[RM];
#pragma unroll
            for (int r = 0; r < RM; r++) acc[r] = 0.f;
#pragma unroll
            for (int i = 0; i < QU / 4; i++) {
#pragma unroll
                for (int r = 0; r < RM; r++) {
                    const float4 xv = *reinterpret_cast<const float4 *>(hs + r * HID + p2 * QU + 4 * i);
                    acc[r] = fmaf(w.w2[i].x, xv.x, acc[r]);
                    acc[r] = fmaf(w.w2[i].y, xv.y, acc[r]);
                    acc[r] = fmaf(w.w2[i].z, xv.z, acc[r]);
                    acc[r] = fmaf(w.w2[i].w, xv.w, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < RM; r++) red[(p2 * RM + r) * HD + j] = acc[r];
        }
        __syncthreads();
        for (int i = tid; i < RM * HD; i += THREADS) {
            const int r = i / HD, j = i - r * HD;  // j = tid % HD: this thread's b2 and scale
            float s = 0.f;
#pragma unroll
            for (int q = 0; q < P2; q++) s += red[(q * RM + r) * HD + j];
            qm[i] = qh[i] * (w.sc * (1.0f + tanh1(s + w.b2)));
        }
        __syncthreads();
    }

    // Phase C: the log-sum-exp merge of the partial states (nn.rs:261-286) into att, spread over the CTAs: CTA c takes
    // the outputs (row, coordinate) [R d c / G, R d (c + 1) / G). TPO threads share an output, each with every
    // TPO-th part of the output's head (the first MPT of them loaded all at once, any further ones after); M is the
    // largest part maximum and att = sum_p e^(m_p - M) acc_p / sum_p e^(m_p - M) s_p. A part of no keys
    // (m -FLT_MAX, s 0, acc 0) adds zero.
    __device__ bool merge_parts() {
        constexpr int TPO = 8, OPP = THREADS / TPO, MPT = 6;
        if (!wait()) return false;  // every partial state is written
        const int tid = threadIdx.x, sub = tid % TPO, G = gridDim.x, R = a.R, d = a.d, per = G / a.heads;
        const int nout = R * d, o0 = (int)((long long)nout * blockIdx.x / G),
                  o1 = (int)((long long)nout * (blockIdx.x + 1) / G);
        for (int ob = o0; ob < o1; ob += OPP) {
            const int o = ob + tid / TPO;
            const bool live = o < o1;
            const int r = live ? o / d : 0, coord = live ? o - r * d : 0, h = coord / HD, j = coord - h * HD;
            const int p0 = h * per;
            float mv[MPT], sv[MPT], av[MPT];
            float M = -FLT_MAX;
#pragma unroll
            for (int k = 0; k < MPT; k++) {
                const int p = sub + TPO * k;
                mv[k] = -FLT_MAX, sv[k] = 0.f, av[k] = 0.f;
                if (live && p < per) {
                    const float *ms = a.part_ms + ((size_t)(p0 + p) * R + r) * 2;
                    mv[k] = __ldcg(ms), sv[k] = __ldcg(ms + 1);
                    av[k] = __ldcg(a.part_acc + ((size_t)(p0 + p) * R + r) * HD + j);
                }
            }
#pragma unroll
            for (int k = 0; k < MPT; k++) M = fmaxf(M, mv[k]);
            const float *ms_r = a.part_ms + (size_t)r * 2;
            const float *acc_r = a.part_acc + (size_t)r * HD + j;
            for (int p = sub + TPO * MPT; live && p < per; p += TPO) M = fmaxf(M, __ldcg(ms_r + (size_t)(p0 + p) * R * 2));
#pragma unroll
            for (int m = 1; m < TPO; m <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, m));
            float S = 0.f, O = 0.f;
#pragma unroll
            for (int k = 0; k < MPT; k++) {
                if (sub + TPO * k < per) {
                    const float w = exp1(mv[k] - M);
                    S = fmaf(sv[k], w, S);
                    O = fmaf(av[k], w, O);
                }
            }
            for (int p = sub + TPO * MPT; live && p < per; p += TPO) {
                const float w = exp1(__ldcg(ms_r + (size_t)(p0 + p) * R * 2) - M);
                S = fmaf(__ldcg(ms_r + (size_t)(p0 + p) * R * 2 + 1), w, S);
                O = fmaf(__ldcg(acc_r + (size_t)(p0 + p) * R * HD), w, O);
            }
#pragma unroll
            for (int m = 1; m < TPO; m <<= 1) {
                S += __shfl_xor_sync(0xffffffffu, S, m);
                O += __shfl_xor_sync(0xffffffffu, O, m);
            }
            if (live && sub == 0) a.att[(size_t)r * d + coord] = O * (1.0f / S);
        }
        arrive();
        return true;
    }

    // Phase B of layer l: the query MLP of this CTA's head (its weights qw loaded before phase A), attention over its
    // tiles, its partial state.
    __device__ bool attend(int l, const QueryW &qw) {
        if (!wait()) return false;  // q is ready
        query_head(head, qw);
        float *qm = scr + C::QM, *red = scr + C::RED, *psm = scr + C::PSM, *alpha = scr + C::ALPHA;
        int *lens = reinterpret_cast<int *>(scr + C::LENS);
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, v = tid & 7, jg = tid >> 3, R = a.R;
        {
            const int te = t0 + n;
            int t = t0;
            float m_run = -FLT_MAX, s_run = 0.f;  // row `warp`'s running state, in every lane of that warp
            float acc[C::DPT];                    // row v (RM 8) or row 0 (lanes v = 0), coordinates jg + 32 i
#pragma unroll
            for (int i = 0; i < C::DPT; i++) acc[i] = 0.f;
            for (bool first = true; t < te; first = false) {
                // a batch of resident tiles under one softmax step
                const int nb = min(min(C::BMAX, a.slots), te - t);
                const int g0 = l * n + (t - t0);
                if (tid < nb) lens[tid] = tile_at(t - t0 + tid).z;
                if (!acquire(l, t - t0, nb)) return false;
                // scores: integer keys take the query times the chunk's key scales (predict.rs:486-497)
                for (int b = 0; b < nb; b++) {
                    const uint8_t *slot = ring + (size_t)slot_add(cons_s, b) * C::SLOT;
                    const float *ksc = reinterpret_cast<const float *>(slot + 2 * HD * C::ROWB);
                    float sp[RM][C::EPV];
#pragma unroll
                    for (int r = 0; r < RM; r++)
#pragma unroll
                        for (int e = 0; e < C::EPV; e++) sp[r][e] = 0.f;
#pragma unroll
                    for (int i = 0; i < C::DPT; i++) {
                        const int j = jg + 32 * i;
                        const uint4 kv = lds_vec<C::VB>(slot + (size_t)j * C::ROWB + v * C::VB);
                        float qs[RM];
#pragma unroll
                        for (int r = 0; r < RM; r++) qs[r] = KV ? qm[r * HD + j] * ksc[j] : qm[r * HD + j];
#pragma unroll
                        for (int e = 0; e < C::EPV; e++) {
                            const float kf = unpack<KV>(kv, e);
#pragma unroll
                            for (int r = 0; r < RM; r++) sp[r][e] = fmaf(qs[r], kf, sp[r][e]);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < RM; r++)
#pragma unroll
                        for (int e = 0; e < C::EPV; e++) {
                            float x = sp[r][e];
                            x += __shfl_xor_sync(0xffffffffu, x, 8);
                            x += __shfl_xor_sync(0xffffffffu, x, 16);
                            sp[r][e] = x;
                        }
                    if (lane < 8) {
#pragma unroll
                        for (int r = 0; r < RM; r++)
#pragma unroll
                            for (int e = 0; e < C::EPV; e++)
                                red[(warp * RM + r) * C::BT + b * C::TK + v * C::EPV + e] = sp[r][e];
                    }
                }
                __syncthreads();
                // online softmax with the reference's rescaling rule (nn.rs:207-215): one row over all eight warps, or
                // one warp per row
                float al_one = 1.f;
                if constexpr (RM == 1) {
                    float *bm = scr + C::BMS, *bs = bm + 8;
                    constexpr int KPT = C::BT / THREADS > 0 ? C::BT / THREADS : 1;
                    float sc[KPT];
                    bool ok[KPT];
                    float mx = -FLT_MAX;
#pragma unroll
                    for (int q = 0; q < KPT; q++) {
                        const int k = tid + THREADS * q;
                        ok[q] = k < C::BT && k < nb * C::TK && (k % C::TK) < lens[k / C::TK];
                        float s = 0.f;
                        if (k < C::BT) {
                            const float *rr = red + k;
                            s = ((rr[0] + rr[C::BT]) + (rr[2 * C::BT] + rr[3 * C::BT])) +
                                ((rr[4 * C::BT] + rr[5 * C::BT]) + (rr[6 * C::BT] + rr[7 * C::BT]));
                        }
                        sc[q] = s;
                        if (ok[q]) mx = fmaxf(mx, s);
                    }
                    mx = warp_max(mx);
                    if (lane == 0) bm[warp] = mx;
                    __syncthreads();
                    mx = fmaxf(fmaxf(fmaxf(bm[0], bm[1]), fmaxf(bm[2], bm[3])), fmaxf(fmaxf(bm[4], bm[5]), fmaxf(bm[6], bm[7])));
                    if (first) {
                        m_run = mx, s_run = 0.f, al_one = 0.f;
                    } else if (mx > m_run) {
                        al_one = exp1(m_run - mx), m_run = mx;
                    }
                    float sum = 0.f;
#pragma unroll
                    for (int q = 0; q < KPT; q++) {
                        const int k = tid + THREADS * q;
                        const float pk = ok[q] ? exp1(sc[q] - m_run) : 0.f;
                        if (k < C::BT) psm[k] = pk;
                        sum += pk;
                    }
                    sum = warp_sum(sum);
                    if (lane == 0) bs[warp] = sum;
                    __syncthreads();
                    s_run = s_run * al_one + (((bs[0] + bs[1]) + (bs[2] + bs[3])) + ((bs[4] + bs[5]) + (bs[6] + bs[7])));
                } else {
                    if (warp < RM) {
                        const int r = warp;
                        if (r < R) {
                            float sc[C::BT / 32];
                            float mx = -FLT_MAX;
#pragma unroll
                            for (int kk = 0; kk < C::BT / 32; kk++) {
                                const int k = lane + 32 * kk;
                                const float *rr = red + r * C::BT + k;
                                const int ws = RM * C::BT;
                                const float s = ((rr[0] + rr[ws]) + (rr[2 * ws] + rr[3 * ws])) +
                                                ((rr[4 * ws] + rr[5 * ws]) + (rr[6 * ws] + rr[7 * ws]));
                                sc[kk] = s;
                                if (k < nb * C::TK && (k % C::TK) < lens[k / C::TK]) mx = fmaxf(mx, s);
                            }
                            mx = warp_max(mx);
                            float al;
                            if (first) {
                                m_run = mx, s_run = 0.f, al = 0.f;
                            } else if (mx > m_run) {
                                al = exp1(m_run - mx), m_run = mx;
                            } else {
                                al = 1.f;
                            }
                            float sum = 0.f;
#pragma unroll
                            for (int kk = 0; kk < C::BT / 32; kk++) {
                                const int k = lane + 32 * kk;
                                const bool valid = k < nb * C::TK && (k % C::TK) < lens[k / C::TK];
                                const float pk = valid ? exp1(sc[kk] - m_run) : 0.f;
                                psm[r * C::BT + k] = pk;
                                sum += pk;
                            }
                            s_run = s_run * al + warp_sum(sum);
                            if (lane == 0) alpha[r] = al;
                        } else {
#pragma unroll
                            for (int kk = 0; kk < C::BT / 32; kk++) psm[r * C::BT + lane + 32 * kk] = 0.f;
                            if (lane == 0) alpha[r] = 1.f;
                        }
                    }
                    __syncthreads();
                }
                // weighted values; integer values take the chunk's value scales after the sum (nn.rs:253-256)
                {
                    float x[C::DPT][RM];
#pragma unroll
                    for (int i = 0; i < C::DPT; i++)
#pragma unroll
                        for (int r = 0; r < RM; r++) x[i][r] = 0.f;
                    for (int b = 0; b < nb; b++) {
                        const uint8_t *slot = ring + (size_t)slot_add(cons_s, b) * C::SLOT;
                        const float *vsc = reinterpret_cast<const float *>(slot + 2 * HD * C::ROWB) + HD;
                        const int len = lens[b];
                        float p[RM][C::EPV];
#pragma unroll
                        for (int r = 0; r < RM; r++)
#pragma unroll
                            for (int e = 0; e < C::EPV; e += 4) {
                                const float4 pv =
                                    *reinterpret_cast<const float4 *>(psm + r * C::BT + b * C::TK + v * C::EPV + e);
                                p[r][e] = pv.x, p[r][e + 1] = pv.y, p[r][e + 2] = pv.z, p[r][e + 3] = pv.w;
                            }
#pragma unroll
                        for (int i = 0; i < C::DPT; i++) {
                            const int j = jg + 32 * i;
                            const uint4 vv = lds_vec<C::VB>(slot + (size_t)(HD + j) * C::ROWB + v * C::VB);
                            float vf[C::EPV];
#pragma unroll
                            for (int e = 0; e < C::EPV; e++) vf[e] = v * C::EPV + e < len ? unpack<KV>(vv, e) : 0.f;
                            const float vs = KV ? vsc[j] : 1.f;
#pragma unroll
                            for (int r = 0; r < RM; r++) {
                                float s = 0.f;
#pragma unroll
                                for (int e = 0; e < C::EPV; e++) s = fmaf(p[r][e], vf[e], s);
                                x[i][r] = KV ? fmaf(s, vs, x[i][r]) : x[i][r] + s;
                            }
                        }
                    }
#pragma unroll
                    for (int i = 0; i < C::DPT; i++) {
                        float tot;
                        if constexpr (RM == 8) {
                            tot = reduce_scatter8(x[i], v);
                        } else {
                            tot = x[i][0];
                            tot += __shfl_xor_sync(0xffffffffu, tot, 1);
                            tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                            tot += __shfl_xor_sync(0xffffffffu, tot, 4);
                        }
                        const int r = RM == 8 ? v : 0;
                        if (r < R && (RM == 8 || v == 0)) acc[i] = acc[i] * (RM == 1 ? al_one : alpha[r]) + tot;
                    }
                }
                __syncthreads();  // the slots and the scratch are free again
                consumed = g0 + nb;
                cons_s = slot_add(cons_s, nb);
                t += nb;
                issue_upto((l + 1) * n);  // this layer's later tiles now; the next layer's after the barrier arrival
            }
            // this CTA's partial state
            const int pi = blockIdx.x;
            if (warp < R && lane == 0) {
                float *ms = a.part_ms + ((size_t)pi * R + warp) * 2;
                ms[0] = m_run, ms[1] = s_run;
            }
            {
                const int r = RM == 8 ? v : 0;
                if (r < R && (RM == 8 || v == 0)) {
#pragma unroll
                    for (int i = 0; i < C::DPT; i++) a.part_acc[((size_t)pi * R + r) * HD + jg + 32 * i] = acc[i];
                }
            }
        }
        arrive();
        issue_upto(total);
        return true;
    }
};

template <int KV, int HD, int RM>
__global__ void __launch_bounds__(THREADS, 1) k_stage_rows(const RowsArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int flag_s;
    __shared__ RowsLayer lay[ROWS_MAX_LAYERS];
    __shared__ int4 tcache[TCACHE];
    Stage<KV, HD, RM> st(a, smem, &flag_s, lay, tcache);
    const int tid = threadIdx.x, d = a.d;
    if (tid == 0) {
        for (int i = 0; i < a.slots; i++) tc::mbar_init(st.mbar + i, 1);
        tc::mbar_init_fence();
    }
    // the pointer table and this CTA's tile descriptors, read once
    {
        const unsigned long long *src = reinterpret_cast<const unsigned long long *>(a.layers);
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(lay);
        for (int i = tid; i < a.L * (int)(sizeof(RowsLayer) / 8); i += THREADS) dst[i] = src[i];
        for (int i = tid; i < min(st.n, TCACHE); i += THREADS) tcache[i] = a.tiles[st.t0 + i];
    }
    __syncthreads();
    st.issue_upto(st.total);
    // Every linear phase (A, D, E, F of each layer, then the decoder's two layers) runs the one inlined linear body
    // from this loop, so the loop's code stays small.
    bool ok = true;
    typename Stage<KV, HD, RM>::QueryW qw;
    const int L = a.L;
    for (int step = 0; step < 4 * L + 2 && ok; step++) {
        const int l = step >> 2, ph = step & 3;
        if (step < 4 * L) {
            const RowsLayer &Ly = lay[l];
            if (ph == 0) st.query_load(Ly, st.head, qw);  // the query MLP's weights load while phase A runs
            if (ph == 1) {
                ok = st.attend(l, qw) && st.merge_parts();
                if (!ok) break;
            }
            const float *x = ph == 1 ? a.att : ph == 3 ? a.mid : a.h;
            const float *W = ph == 0 ? Ly.wq : ph == 1 ? Ly.wo : ph == 2 ? Ly.w1 : Ly.w2;
            const float *b = ph == 0 ? Ly.bq : ph == 1 ? Ly.bo : ph == 2 ? Ly.b1 : Ly.b2;
            const int N = ph == 2 ? a.ff : d;
            float *y = ph == 0 ? a.q : ph == 2 ? a.mid : a.h;
            ok = st.linear(ph == 0 || ph == 2, step > 0, x, ph == 3 ? a.ff : d, ph == 0 ? Ly.n1w : Ly.n2w,
                           ph == 0 ? Ly.n1b : Ly.n2b, W, b, N, ph == 2, y, N, ph == 1 || ph == 3);
        } else {
            const bool first = ph == 0;
            const int N = first ? a.dff : a.out_n;
            ok = st.linear(first, true, first ? a.h : a.mid, first ? d : a.dff, a.lnw, a.lnb, first ? a.dec0w : a.dec2w,
                           first ? a.dec0b : a.dec2b, N, first, first ? a.mid : a.out, N, false);
        }
    }
    if (!ok) st.drain();
}

template <int KV, int HD, int RM>
size_t smem_of(int slots) {
    using C = Cfg<KV, HD, RM>;
    return 128 + (size_t)slots * C::SLOT + 128 + sizeof(float) * (size_t)C::SCRATCH;
}

template <int KV, int HD, int RM>
cudaError_t launch_one(const RowsArgs &a, int grid, size_t smem, cudaStream_t s) {
    auto kern = k_stage_rows<KV, HD, RM>;
    cudaError_t e = allow_dynamic_smem((const void *)kern, smem);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<RowsArgs *>(&a)};
    return cudaLaunchCooperativeKernel((const void *)kern, dim3(grid), dim3(THREADS), args, smem, s);
}

template <int KV, int HD, int RM>
int max_grid_one(size_t smem, int sms) {
    auto kern = k_stage_rows<KV, HD, RM>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, THREADS, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per * sms;
}

#define TCU_ROWS_CASES(X)                                                                                      \
    X(0, 128, 1) X(0, 128, 8) X(1, 128, 1) X(1, 128, 8) X(2, 128, 1) X(2, 128, 8) X(0, 64, 1) X(0, 64, 8) X(1, 64, 1) \
        X(1, 64, 8) X(2, 64, 1) X(2, 64, 8)

}  // namespace

int rows_tile_keys(int kv) { return kv == 0 ? 32 : 64; }

size_t rows_smem(int kv, int hd, int R, int slots) {
    const int rm = R > 1 ? 8 : 1;
#define X(K, H, M) \
    if (kv == K && hd == H && rm == M) return smem_of<K, H, M>(slots);
    TCU_ROWS_CASES(X)
#undef X
    return 0;
}

int rows_slots_for(int kv, int hd, int R, size_t smem_max) {
    const size_t base = rows_smem(kv, hd, R, 0), one = rows_smem(kv, hd, R, 1) - base;
    if (base == 0 || smem_max < base + one) return 0;
    return (int)std::min<size_t>(16, (smem_max - base) / one);
}

int rows_max_grid(int kv, int hd, int R, size_t smem, int sms) {
    const int rm = R > 1 ? 8 : 1;
#define X(K, H, M) \
    if (kv == K && hd == H && rm == M) return max_grid_one<K, H, M>(smem, sms);
    TCU_ROWS_CASES(X)
#undef X
    return 0;
}

cudaError_t launch_stage_rows(int kv, int hd, const RowsArgs &a, int grid, size_t smem, cudaStream_t s,
                              uint64_t *launches) {
    const int R = a.R, rm = R > 1 ? 8 : 1;
    if (R < 1 || R > 8 || grid < 1 || grid > ROWS_MAX_GRID || a.heads > ROWS_MAX_HEADS) return cudaErrorInvalidValue;
    cudaError_t e = cudaErrorInvalidValue;
#define X(K, H, M) \
    if (kv == K && hd == H && rm == M) e = launch_one<K, H, M>(a, grid, smem, s);
    TCU_ROWS_CASES(X)
#undef X
    if (e == cudaSuccess && launches) ++*launches;
    return e;
}

}  // namespace tcu
