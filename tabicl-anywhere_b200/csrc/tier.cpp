// The card tier (gpu::VramTier and VramHandle, src/gpu.rs:2450-2701) over the ownership ledger of src/warm.rs:28-115:
// fitted problems resident on one device for many tenants, within an overall byte budget and one per tenant. The
// least recently used problem makes room; one in use by a prediction is released only when that prediction has
// finished; a load is started by the first prediction that needs it, on a thread of its own, while that prediction
// declines (the caller's CPU path answers it).
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <system_error>
#include <thread>
#include <tuple>
#include <vector>

#include "engine.hpp"

using namespace tcu;

namespace {

// warm.rs:22: tenant, model, a name within the model (the member prefix) and a number within it (the problem)
struct Key {
    std::string tenant, model, prefix;
    int node;
    bool operator<(const Key &o) const {
        return std::tie(tenant, model, prefix, node) < std::tie(o.tenant, o.model, o.prefix, o.node);
    }
};

// warm.rs:28-115 Ledger: what is held for whom, the bytes in all and per tenant, when each entry was last used, and
// the one rule for making room. Removed values are handed back in `gone`; the caller lets go of them.
template <typename V>
struct Ledger {
    struct E {
        V v;
        size_t bytes;
        uint64_t used;
    };
    std::map<Key, E> entries;
    size_t bytes = 0;
    std::map<std::string, size_t> by_tenant;
    uint64_t clock = 0;

    // the entry, marked as just used
    V *get(const Key &k) {
        ++clock;
        auto it = entries.find(k);
        if (it == entries.end()) return nullptr;
        it->second.used = clock;
        return &it->second.v;
    }
    bool contains(const Key &k) const { return entries.count(k) != 0; }
    size_t tenant_bytes(const std::string &t) const {
        auto it = by_tenant.find(t);
        return it == by_tenant.end() ? 0 : it->second;
    }
    bool remove(const Key &k, std::vector<V> &gone) {
        auto it = entries.find(k);
        if (it == entries.end()) return false;
        bytes -= it->second.bytes;
        by_tenant[k.tenant] -= it->second.bytes;
        gone.push_back(std::move(it->second.v));
        entries.erase(it);
        return true;
    }
    // warm.rs:62-88: hold v (n bytes) under k, first making room within both budgets: while the tenant would be over
    // its share its own least recently used entry goes, otherwise the least recently used of anyone's; only entries
    // may_go allows ever go. False, with nothing held under k, when room cannot be made (what went stays gone).
    template <typename MayGo>
    bool admit(const Key &k, size_t n, V v, size_t budget, size_t tenant_budget, MayGo may_go, std::vector<V> &gone) {
        if (n > std::min(tenant_budget, budget)) return false;
        for (;;) {
            const bool over_tenant = tenant_bytes(k.tenant) + n > tenant_budget;
            if (!over_tenant && bytes + n <= budget) break;
            const Key *victim = nullptr;
            uint64_t oldest = UINT64_MAX;
            for (auto &e : entries)
                if ((!over_tenant || e.first.tenant == k.tenant) && may_go(e.second.v) && e.second.used < oldest)
                    oldest = e.second.used, victim = &e.first;
            if (!victim) return false;
            const Key vk = *victim;
            remove(vk, gone);
        }
        ++clock;
        bytes += n;
        by_tenant[k.tenant] += n;
        remove(k, gone);  // an entry replaced gives its bytes back once
        entries.emplace(k, E{std::move(v), n, clock});
        return true;
    }
    // everything `tenant` holds (for `model` only, if given)
    std::vector<V> evict(const std::string &tenant, const char *model) {
        std::vector<Key> keys;
        for (auto &e : entries)
            if (e.first.tenant == tenant && (!model || e.first.model == model)) keys.push_back(e.first);
        std::vector<V> gone;
        for (auto &k : keys) remove(k, gone);
        return gone;
    }
};

// gpu.rs:2464-2490 Live and Lease: device memory really taken by the models loaded through the tier, from the start
// of a load until the model's buffers are released (models evicted but still in use by a prediction included).
struct Live {
    std::mutex mu;
    size_t bytes = 0;
    std::map<std::string, size_t> by_tenant;
};

struct Lease {
    std::shared_ptr<Live> live;
    std::string tenant;
    size_t bytes;
    ~Lease() {
        std::lock_guard<std::mutex> lk(live->mu);
        live->bytes -= bytes;
        live->by_tenant[tenant] -= bytes;
    }
};

// A loaded problem with its share of Live: the model is freed first, then the share is given back.
struct Resident {
    tcu_model *m = nullptr;
    std::unique_ptr<Lease> lease;
    ~Resident() {
        if (m) tcu_model_free(m);
    }
};

// gpu.rs:2450-2457: being uploaded (its bytes already counted), ready, or larger than its tenant's whole budget
struct Slot {
    enum Kind { LOADING, READY, TOO_BIG } kind;
    std::shared_ptr<Resident> ready;
};

using Loader = std::function<tcu_model *()>;

}  // namespace

struct tcu_tier {
    tcu_ctx *ctx = nullptr;  // null: bookkeeping only (the debug entry points)
    size_t budget = 0, tenant_budget = 0;
    bool background = true;
    std::mutex mu;  // the ledger; taken before a context's lock or Live's, never after
    Ledger<Slot> state;
    std::shared_ptr<Live> live = std::make_shared<Live>();
    std::atomic<uint64_t> fallbacks{0};
    std::mutex err_mu;
    std::string last_error;
    std::mutex load_mu;
    std::condition_variable load_cv;
    int loading = 0;  // loads running on threads of their own
};

// VramHandle (gpu.rs:2628-2634): one tenant's use of the tier for one fitted bundle and set of weights
struct tcu_handle {
    tcu_tier *tier = nullptr;
    std::string tenant, model;
    std::function<std::unique_ptr<Bundle>()> open;
    tcu_weights *w = nullptr;
};

struct tcu_pin {
    std::shared_ptr<Resident> r;
};

namespace {

void set_error(tcu_tier *t, const std::string &e) {
    std::lock_guard<std::mutex> lk(t->err_mu);
    t->last_error = e;
}

// gpu.rs:2560-2593 claim: a place for the problem and its bytes counted, before anything is uploaded; null when the
// budgets leave no room (a problem larger than its tenant's budget is marked so, and never tried again).
std::unique_ptr<Lease> claim(tcu_tier *t, const Key &key, size_t bytes) {
    std::vector<Slot> gone;
    std::lock_guard<std::mutex> lk(t->mu);
    if (t->state.contains(key)) return nullptr;
    // only ready problems may make room; one being loaded keeps its place
    if (!t->state.admit(key, bytes, Slot{Slot::LOADING, nullptr}, t->budget, t->tenant_budget,
                        [](const Slot &s) { return s.kind == Slot::READY; }, gone)) {
        if (bytes > t->tenant_budget)
            t->state.admit(key, 0, Slot{Slot::TOO_BIG, nullptr}, t->budget, t->tenant_budget, [](const Slot &) { return false; }, gone);
        gone.clear();
        return nullptr;
    }
    // what was evicted is released here, unless a prediction is still using it
    gone.clear();
    std::lock_guard<std::mutex> ll(t->live->mu);
    const size_t mine = t->live->by_tenant[key.tenant];
    if (t->live->bytes + bytes > t->budget || mine + bytes > t->tenant_budget) {
        // the room is promised to problems still in use: not this time
        t->state.remove(key, gone);
        return nullptr;
    }
    t->live->bytes += bytes;
    t->live->by_tenant[key.tenant] += bytes;
    return std::unique_ptr<Lease>(new Lease{t->live, key.tenant, bytes});
}

// gpu.rs:2595-2626 finish: upload a claimed problem and make it ready, unless it was evicted meanwhile. 1 ready,
// 0 evicted meanwhile, < 0 the load failed (its place is given up and the reason kept).
int finish(tcu_tier *t, const Key &key, std::unique_ptr<Lease> lease, const Loader &load) {
    tcu_model *m = nullptr;
    int code = TCU_OK;
    std::string err;
    try {
        m = load();
        if (m && tcu_model_bytes(m) != lease->bytes) {
            tcu_model_free(m);
            m = nullptr;
            throw Error{TCU_ERR_STATE, "tier: a loaded problem holds other bytes than were charged for it"};
        }
    } catch (const Error &e) {
        code = e.code, err = e.msg;
    } catch (const BundleError &e) {
        code = e.code, err = e.what();
    } catch (const std::bad_alloc &) {
        code = TCU_ERR_MEMORY, err = "host memory exhausted";
    } catch (const std::exception &e) {
        code = TCU_ERR_ARG, err = e.what();
    }
    std::shared_ptr<Resident> r;  // released (outside the lock) when the problem was evicted meanwhile
    std::vector<Slot> gone;
    std::lock_guard<std::mutex> lk(t->mu);
    if (code == TCU_OK) {
        r = std::make_shared<Resident>();
        r->m = m, r->lease = std::move(lease);
        Slot *s = t->state.get(key);
        if (s && s->kind == Slot::LOADING) {
            s->kind = Slot::READY, s->ready = r;
            return 1;
        }
        return s && s->kind == Slot::READY ? 1 : 0;
    }
    Slot *s = t->state.get(key);
    if (s && s->kind == Slot::LOADING) t->state.remove(key, gone);
    set_error(t, err);
    return code;
}

// Run `finish` on a thread of its own (VramHandle::resident natively, gpu.rs:2690-2698).
void start_load(tcu_tier *t, const Key &key, std::unique_ptr<Lease> lease, Loader load) {
    {
        std::lock_guard<std::mutex> lk(t->load_mu);
        t->loading++;
    }
    auto done = [t] {
        std::lock_guard<std::mutex> lk(t->load_mu);
        if (--t->loading == 0) t->load_cv.notify_all();
    };
    try {
        std::thread([t, key, lease = std::move(lease), load = std::move(load), done]() mutable {
            finish(t, key, std::move(lease), load);
            done();
        }).detach();
    } catch (const std::system_error &e) {
        // no thread: the claimed place is given up (the lease went with the thread's state)
        std::vector<Slot> gone;
        {
            std::lock_guard<std::mutex> lk(t->mu);
            Slot *s = t->state.get(key);
            if (s && s->kind == Slot::LOADING) t->state.remove(key, gone);
        }
        set_error(t, std::string("tier: cannot start a load: ") + e.what());
        done();
    }
}

bool with_col(const Bundle &b, const std::string &prefix) {
    // the column stage's cache is kept only where the `rows` hook is called: one problem, one label digit
    // (gpu.rs:2087-2090, predict.rs:642)
    const MemberInfo mi = member_info(b, prefix);
    return mi.nodes == 1 && mi.digits == 1;
}

// VramHandle::resident (gpu.rs:2674-2700): the problem if it is ready; otherwise its load is started (once) and the
// call declines; in the tier's foreground mode the load runs right here and this call already uses it.
std::shared_ptr<Resident> resident(tcu_handle *h, const std::string &prefix, int node) {
    tcu_tier *t = h->tier;
    const Key key{h->tenant, h->model, prefix, node};
    {
        std::lock_guard<std::mutex> lk(t->mu);
        if (Slot *s = t->state.get(key)) return s->kind == Slot::READY ? s->ready : nullptr;
    }
    size_t bytes = 0;
    try {
        auto b = h->open();
        ctx_of(h->w);
        bytes = node_bytes(h->w, *b, prefix, node, with_col(*b, prefix));
    } catch (...) {
        return nullptr;  // as claim(...).ok()?? does: a bundle that cannot be read declines
    }
    auto lease = claim(t, key, bytes);
    if (!lease) return nullptr;
    auto open = h->open;
    tcu_weights *w = h->w;
    Loader load = [open, w, prefix, node]() -> tcu_model * {
        auto b = open();
        return load_node(w, *b, prefix, node, with_col(*b, prefix));
    };
    if (t->background) {
        start_load(t, key, std::move(lease), std::move(load));
        return nullptr;
    }
    finish(t, key, std::move(lease), load);
    std::lock_guard<std::mutex> lk(t->mu);
    Slot *s = t->state.get(key);
    return s && s->kind == Slot::READY ? s->ready : nullptr;
}

// VramHandle::or_cpu (gpu.rs:2658-2671): a card that fails does not fail the prediction: it declines, counted, with
// the reason kept.
int or_cpu(tcu_handle *h, int rc) {
    if (rc >= 0) return rc;
    h->tier->fallbacks++;
    set_error(h->tier, tcu_last_error(h->tier->ctx));
    return TCU_DECLINED;
}

}  // namespace

extern "C" {

int tcu_tier_new(tcu_ctx *ctx, size_t budget, size_t tenant_budget, int background, tcu_tier **out) {
    if (!out) return TCU_ERR_ARG;
    try {
        tcu_tier *t = new tcu_tier();
        t->ctx = ctx, t->budget = budget, t->tenant_budget = std::min(tenant_budget, budget);
        t->background = background != 0;
        *out = t;
        return TCU_OK;
    } catch (const std::bad_alloc &) {
        return TCU_ERR_MEMORY;
    }
}

void tcu_tier_wait(tcu_tier *t) {
    if (!t) return;
    std::unique_lock<std::mutex> lk(t->load_mu);
    t->load_cv.wait(lk, [t] { return t->loading == 0; });
}

void tcu_tier_free(tcu_tier *t) {
    if (!t) return;
    tcu_tier_wait(t);
    std::vector<Slot> gone;
    {
        std::lock_guard<std::mutex> lk(t->mu);
        for (auto &e : t->state.entries) gone.push_back(std::move(e.second.v));
        t->state.entries.clear();
    }
    gone.clear();  // problems still pinned by a prediction are released when it lets go
    delete t;
}

void tcu_tier_held(tcu_tier *t, const char *tenant, size_t *all, size_t *mine) {
    if (!t) return;
    std::lock_guard<std::mutex> lk(t->mu);
    if (all) *all = t->state.bytes;
    if (mine) *mine = tenant ? t->state.tenant_bytes(tenant) : 0;
}

size_t tcu_tier_ready(tcu_tier *t, const char *tenant) {
    if (!t || !tenant) return 0;
    std::lock_guard<std::mutex> lk(t->mu);
    size_t n = 0;
    for (auto &e : t->state.entries)
        if (e.first.tenant == tenant && e.second.v.kind == Slot::READY) n += e.second.bytes;
    return n;
}

void tcu_tier_on_card(tcu_tier *t, const char *tenant, size_t *all, size_t *mine) {
    if (!t) return;
    std::lock_guard<std::mutex> lk(t->live->mu);
    if (all) *all = t->live->bytes;
    if (mine) *mine = tenant ? t->live->by_tenant[tenant] : 0;
}

uint64_t tcu_tier_fallbacks(const tcu_tier *t) { return t ? t->fallbacks.load() : 0; }

size_t tcu_tier_last_error(tcu_tier *t, char *buf, size_t n) {
    if (!t) return 0;
    std::lock_guard<std::mutex> lk(t->err_mu);
    if (buf && n) {
        const size_t k = std::min(n - 1, t->last_error.size());
        std::memcpy(buf, t->last_error.data(), k);
        buf[k] = 0;
    }
    return t->last_error.size();
}

void tcu_tier_evict(tcu_tier *t, const char *tenant, const char *model) {
    if (!t || !tenant) return;
    std::vector<Slot> gone;
    {
        std::lock_guard<std::mutex> lk(t->mu);
        gone = t->state.evict(tenant, model);
    }
    // released here, unless a prediction is still using them
}

static int make_handle(tcu_tier *t, const char *tenant, const char *model, tcu_weights *w,
                       std::function<std::unique_ptr<Bundle>()> open, tcu_handle **out) {
    if (!t || !tenant || !model || !w || !out || !t->ctx || ctx_of_weights(w) != t->ctx) return TCU_ERR_ARG;
    try {
        tcu_handle *h = new tcu_handle();
        h->tier = t, h->tenant = tenant, h->model = model, h->w = w, h->open = std::move(open);
        *out = h;
        return TCU_OK;
    } catch (const std::bad_alloc &) {
        return TCU_ERR_MEMORY;
    }
}

int tcu_tier_handle(tcu_tier *t, const char *tenant, const char *model, const char *bundle_path, tcu_weights *w,
                    tcu_handle **out) {
    if (!bundle_path) return TCU_ERR_ARG;
    std::string path(bundle_path);
    return make_handle(t, tenant, model, w, [path] { return Bundle::open(path); }, out);
}

int tcu_tier_handle_source(tcu_tier *t, const char *tenant, const char *model, const tcu_source *src, tcu_weights *w,
                           tcu_handle **out) {
    if (!src || !src->read_at) return TCU_ERR_ARG;
    const tcu_source s = *src;
    return make_handle(t, tenant, model, w, [s] {
        return Bundle::from_reader(
            [s](void *buf, uint64_t n, uint64_t off) {
                if (s.read_at(s.user, off, buf, n) != 0) throw BundleError(TCU_ERR_IO, "bundle source: read failed");
            },
            s.size);
    }, out);
}

void tcu_handle_free(tcu_handle *h) { delete h; }

int tcu_handle_preload(tcu_handle *h, const char *prefix, int node) {
    if (!h || !prefix) return TCU_ERR_ARG;
    tcu_tier *t = h->tier;
    const Key key{h->tenant, h->model, prefix, node};
    {
        std::lock_guard<std::mutex> lk(t->mu);
        Slot *s = t->state.get(key);
        if (s && s->kind == Slot::READY) return 1;
    }
    size_t bytes = 0;
    try {
        auto b = h->open();
        ctx_of(h->w);
        bytes = node_bytes(h->w, *b, prefix, node, with_col(*b, prefix));
    } catch (const Error &e) {
        set_error(t, e.msg);
        return e.code;
    } catch (const BundleError &e) {
        set_error(t, e.what());
        return e.code;
    } catch (const std::exception &e) {
        set_error(t, e.what());
        return TCU_ERR_ARG;
    }
    auto lease = claim(t, key, bytes);
    if (!lease) return 0;
    auto open = h->open;
    tcu_weights *w = h->w;
    const std::string p(prefix);
    return finish(t, key, std::move(lease), [open, w, p, node]() -> tcu_model * {
        auto b = open();
        return load_node(w, *b, p, node, with_col(*b, p));
    });
}

int tcu_handle_attend(tcu_handle *h, const char *prefix, int node, int layer, const float *q, int rows, int d, int heads,
                      float *out) {
    if (!h || !prefix) return TCU_ERR_ARG;
    auto r = resident(h, prefix, node);
    if (!r || !r->m) return TCU_DECLINED;
    return or_cpu(h, tcu_attend(r->m, layer, q, rows, d, heads, out));
}

int tcu_handle_stage(tcu_handle *h, const char *prefix, int node, const float *x, int rows, int d, int out_n, float *out) {
    if (!h || !prefix) return TCU_ERR_ARG;
    auto r = resident(h, prefix, node);
    if (!r || !r->m) return TCU_DECLINED;
    return or_cpu(h, tcu_stage(r->m, x, rows, d, out_n, out));
}

int tcu_handle_rows(tcu_handle *h, const char *prefix, const float *x, int rows, int features, int out_n, float *out) {
    if (!h || !prefix) return TCU_ERR_ARG;
    auto r = resident(h, prefix, 0);
    if (!r || !r->m || !has_col(r->m)) return TCU_DECLINED;
    return or_cpu(h, tcu_rows(r->m, x, rows, features, out_n, out));
}

int tcu_tier_debug_admit(tcu_tier *t, const char *tenant, const char *model, const char *prefix, int node, size_t bytes) {
    if (!t || !tenant || !model || !prefix) return TCU_ERR_ARG;
    const Key key{tenant, model, prefix, node};
    auto lease = claim(t, key, bytes);
    if (!lease) return 0;
    return finish(t, key, std::move(lease), []() -> tcu_model * { return nullptr; });
}

int tcu_tier_debug_pin(tcu_tier *t, const char *tenant, const char *model, const char *prefix, int node, tcu_pin **out) {
    if (!t || !tenant || !model || !prefix || !out) return TCU_ERR_ARG;
    std::lock_guard<std::mutex> lk(t->mu);
    Slot *s = t->state.get(Key{tenant, model, prefix, node});
    if (!s || s->kind != Slot::READY) return 0;
    *out = new tcu_pin{s->ready};
    return 1;
}

void tcu_tier_debug_unpin(tcu_pin *p) { delete p; }

}  // extern "C"
