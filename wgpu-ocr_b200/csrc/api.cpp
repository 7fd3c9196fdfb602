// The C ABI of include/wocr.h: status codes at the boundary, exceptions inside.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "exec.h"
#include "layout.h"

using namespace wocr;

namespace wocr {
const std::string &last_error();
}

// The context lives until the caller's handle and every detector / recogniser / graph made
// from it are destroyed, in any order.
struct wocr_ctx {
    Ctx c;
    int refs = 1;
};

static void ctx_release(wocr_ctx *ctx);

struct Stats {
    double flops = 0;
    int64_t launches = 0;
    int64_t h2d = 0, d2h = 0;  // bytes copied between host and device
};

// One detection pass (detect_pages_dev) captured as a CUDA graph for a given page count, size,
// threshold and pair of device buffers, then replayed with one launch: the executor's host work
// (lowering lookups, stream-ordered allocations, twenty-odd launches) is paid at capture only.
struct DetGraph {
    int n = 0, w = 0, h = 0;
    float thr = 0;
    const int2 *rows = nullptr;  // compacted pages: the row table (null: whole pages)
    const uint8_t *rgb = nullptr;
    uint32_t *mask = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    double flops = 0;
    int64_t launches = 0;
    uint64_t used = 0;  // last use (least recently used is replaced)
    void reset() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        exec = nullptr;
        graph = nullptr;
        n = 0;
    }
};

// The source rows the detector's grey/resize reads (src/gpu.rs:533-561): output row oy of the
// 800 x 600 model input interpolates rows y1 = floor(iy) and y2 = min(y1 + 1, ph - 1) of the page,
// iy = clamp(sy (oy + 0.5) - 0.5, 0, ph - 1), sy = ph / 800.  For a tall page (h > 1600) that is
// under half of it, so wocr_detect_pages uploads only those rows: page row pairs (y1, y1 + 1)
// whose positions repeat with a period of k output rows and P page rows go up as k strided
// copies per page (cudaMemcpy2DAsync), the rest (the last rows, where y2 is clamped) one row at a
// time, into rows 2 oy and 2 oy + 1 of a compacted page (k_grey_rows).  Pages with no period up
// to 64 output rows, or not taller than 1600, upload whole.
struct RowPlan {
    int w = 0, h = 0;
    bool ok = false;
    int k = 0, P = 0, regular = 0;     // period; output rows [0, regular) are (y1, y1 + 1) pairs
    std::vector<int> y1, y2;
    std::vector<int> first, count;     // per phase j < k: first page row, number of periods
    BufP table;                        // rows[oy] for k_grey_rows
    size_t bytes = 0;                  // compacted page bytes
};

struct wocr_detector {
    wocr_ctx *ctx;
    std::unique_ptr<Executor> graph;
    Stats last;
    DetGraph graphs[4];
    uint64_t uses = 0;
    // wocr_detect_pages: two upload slots and two mask slots, kept between calls (stable
    // addresses, so each slot's detection pass is one cached graph)
    BufP up_buf[2], mask_buf[2];
    RowPlan plan;                      // of the last page size seen
    // page uploads on their own stream and mask read-backs on another, both overlapped with
    // detection: ready (buffers allocated), up[slot] (chunk uploaded), done[slot] (chunk
    // detected), back[slot] (chunk mask read back)
    cudaStream_t copy = nullptr, copy_back = nullptr;
    cudaEvent_t ready = nullptr, up[2] = {nullptr, nullptr}, done[2] = {nullptr, nullptr},
                back[2] = {nullptr, nullptr}, fin = nullptr;
    ~wocr_detector() {
        for (auto &g : graphs) g.reset();
        if (copy) cudaStreamDestroy(copy);
        if (copy_back) cudaStreamDestroy(copy_back);
        for (cudaEvent_t e : {ready, up[0], up[1], done[0], done[1], back[0], back[1], fin})
            if (e) cudaEventDestroy(e);
    }
};

struct GruLayer {
    DevW w_t, wb, r, rb;  // w_t [in][1536], wb [2][768] (input bias), r [2][768][256], rb [2][768]
    int input = 0;
    std::shared_ptr<k::UmmaW> uw;  // the projection on the tensor cores
};

// One wocr_recognize layout (batch sizes and widths, which outputs) replayed from a CUDA graph:
// the batches are uploaded into a persistent buffer, the captured trunks, GRU layers, output
// layer and arg-max write persistent outputs.  The first call of a layout runs directly.
struct RecReplay {
    std::vector<int32_t> bn, bw;
    int want = -1;  // bit 0 logits, bit 1 arg-max
    int ntot = 0, tmax = 0;
    std::vector<int> lens;
    BufP in, lens_d, logits, best;
    std::vector<size_t> in_off;  // element offset of each batch in `in`
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    double flops = 0;
    int64_t launches = 0;
    uint64_t used = 0;
    void reset() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        exec = nullptr;
        graph = nullptr;
        want = -1;
        in.reset();
        lens_d.reset();
        logits.reset();
        best.reset();
    }
};

struct wocr_recognizer {
    wocr_ctx *ctx;
    RecReplay replays[4];
    uint64_t uses = 0;
    // the width buckets' trunks run on these streams inside a captured pass (parallel graph
    // branches): fork from the context stream, join back before the time-major pooling
    static constexpr int kSide = 4;
    cudaStream_t side[kSide] = {};
    cudaEvent_t fork = nullptr, join[kSide] = {};
    std::unique_ptr<Executor> trunk;
    int pool_kh = 1;
    GruLayer layers[2];
    DevW lin_w, lin_b;  // [512][ldw], bias [ldw]
    std::shared_ptr<k::UmmaW> lin_uw;
    int classes = 0, ldw = 0;
    int lines = 8;
    ~wocr_recognizer() {
        for (auto &r : replays) r.reset();
        for (int i = 0; i < kSide; i++) {
            if (side[i]) cudaStreamDestroy(side[i]);
            if (join[i]) cudaEventDestroy(join[i]);
        }
        if (fork) cudaEventDestroy(fork);
    }
    Stats last;
};

// One NdGraph call for one input shape, replayed from a CUDA graph: the input is uploaded into a
// persistent buffer, the captured run writes persistent outputs (the full output, or the row
// arg-max with its maximum and log-sum-exp).  The first call of a shape runs directly and
// records the output shape; the second captures.
struct NdReplay {
    std::vector<int64_t> in_shape, out_shape;
    // 0 wocr_ndgraph_run, 1 wocr_ndgraph_run_argmax, 4 the same without the log-sum-exp (a
    // caller that reads only the classes and maxima), 2 / 3 PP detection
    int mode = -1;
    int64_t rows = 0, len = 0;
    BufP in, out, best, mx, lse;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    double flops = 0;
    int64_t launches = 0;
    uint64_t used = 0;
    void reset() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        exec = nullptr;
        graph = nullptr;
        mode = -1;
        in.reset();
        out.reset();
        best.reset();
        mx.reset();
        lse.reset();
    }
};

struct wocr_ndgraph {
    wocr_ctx *ctx;
    std::unique_ptr<Executor> graph;
    Stats last;
    // captured runs per input shape: config 3 recognises 16 width buckets a step and a page of
    // the page pipeline up to ~50 line batches of different widths, so the cache holds far more
    // than that (an LRU of fewer entries than a cycle's shapes misses on every call of it)
    NdReplay replays[256];
    uint64_t uses = 0;
    // the probability map of the last wocr_ppdet_page ([map_h][map_w] fp32) for the DB steps
    BufP map_buf;
    const float *map = nullptr;
    int map_w = 0, map_h = 0;
    float map_to_page[2] = {1.f, 1.f};
    ~wocr_ndgraph() {
        for (auto &r : replays) r.reset();
    }
};

namespace {

struct RunScope {
    Ctx *c;
    Stats *out;
    double f0;
    int64_t l0;
    RunScope(Ctx *ctx, Stats *s) : c(ctx), out(s), f0(ctx->flops), l0(ctx->launches) {
        WOCR_CUDA(cudaSetDevice(ctx->device));
        out->h2d = out->d2h = 0;
    }
    ~RunScope() {
        out->flops = c->flops - f0;
        out->launches = c->launches - l0;
    }
};

}  // namespace

namespace wocr {
// The device error word of bounded kernel waits: read (and cleared) after a synchronisation.
void check_status(Ctx *c) {
    if (!c->status) return;
    int v = 0;
    WOCR_CUDA(cudaMemcpy(&v, c->status, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
        WOCR_CUDA(cudaMemset(c->status, 0, sizeof(int)));
        fail(WOCR_ERR_TIMEOUT, "a kernel wait gave up (code " + std::to_string(v) + "); its results are invalid");
    }
}

void wait_stream(Ctx *c) {
    if (!c->sync_ev) {
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
        return;
    }
    // a short wait polls (a blocking wait's wake-up costs tens of microseconds), a long one
    // sleeps on the event
    WOCR_CUDA(cudaEventRecord(c->sync_ev, c->stream));
    const auto t0 = std::chrono::steady_clock::now();
    while (std::chrono::steady_clock::now() - t0 < std::chrono::microseconds(100)) {
        const cudaError_t e = cudaEventQuery(c->sync_ev);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) WOCR_CUDA(e);
    }
    WOCR_CUDA(cudaEventSynchronize(c->sync_ev));
}

void sync_bounded(Ctx *c, int timeout_ms) {
    if (timeout_ms <= 0) {
        wait_stream(c);
        check_status(c);
        return;
    }
    auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaStreamQuery(c->stream);
        if (e == cudaSuccess) {
            check_status(c);
            return;
        }
        if (e != cudaErrorNotReady) WOCR_CUDA(e);
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) fail(WOCR_ERR_TIMEOUT, "stream did not finish within " + std::to_string(timeout_ms) + " ms");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

Ctx *ctx_of(wocr_ctx *h) { return h ? &h->c : nullptr; }
}  // namespace wocr

namespace {

void d2h(Ctx *c, void *dst, const void *src, size_t bytes) {
    if (bytes) WOCR_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream));
}

}  // namespace

static void ctx_release(wocr_ctx *ctx) {
    if (--ctx->refs > 0) return;
    Ctx &c = ctx->c;
    cudaSetDevice(c.device);
    cudaStreamSynchronize(c.stream);
    // everything freed on the stream goes before the stream itself
    c.status_buf.reset();
    c.status = nullptr;
    for (auto &r : c.recs) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (auto e : c.spare) cudaEventDestroy(e);
    if (c.sync_ev) cudaEventDestroy(c.sync_ev);
    c.recs.clear();
    c.spare.clear();
    cudaStreamSynchronize(c.stream);
    cudaStreamDestroy(c.stream);
    c.stream = nullptr;
    delete ctx;
}

extern "C" {

const char *wocr_last_error(void) { return last_error().c_str(); }

int32_t wocr_ctx_create(int32_t device, int32_t lines, wocr_ctx **out) {
    return guard([&] {
        if (!out) fail(WOCR_ERR_INVALID, "null out");
        int n = 0;
        WOCR_CUDA(cudaGetDeviceCount(&n));
        if (device < 0 || device >= n) fail(WOCR_ERR_INVALID, "no CUDA device " + std::to_string(device));
        WOCR_CUDA(cudaSetDevice(device));
        cudaDeviceProp prop;
        WOCR_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major < 10) fail(WOCR_ERR_UNSUPPORTED, std::string("sm_100a kernels need a B200-class GPU, found ") + prop.name);
        auto *h = new wocr_ctx();
        h->c.device = device;
        h->c.lines = lines > 0 ? lines : 8;
        h->c.sm_count = prop.multiProcessorCount;
        h->c.name = std::string(prop.name) + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ", " +
                    std::to_string(prop.multiProcessorCount) + " SMs)";
        cudaError_t e = cudaStreamCreateWithFlags(&h->c.stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete h;
            WOCR_CUDA(e);
        }
        cudaMemPool_t pool;
        WOCR_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
        uint64_t thr = UINT64_MAX;
        WOCR_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
        h->c.pool = pool;
        if (!std::getenv("WOCR_SPIN_SYNC"))
            WOCR_CUDA(cudaEventCreateWithFlags(&h->c.sync_ev, cudaEventBlockingSync | cudaEventDisableTiming));
        // the device error word of bounded waits, allocated before any graph capture
        h->c.status_buf = alloc(&h->c, 16);
        h->c.status = (int *)h->c.status_buf->p;
        WOCR_CUDA(cudaMemsetAsync(h->c.status, 0, 16, h->c.stream));
        WOCR_CUDA(cudaStreamSynchronize(h->c.stream));
        *out = h;
    });
}

void wocr_ctx_destroy(wocr_ctx *ctx) {
    if (!ctx) return;
    ctx_release(ctx);
}

int32_t wocr_ctx_describe(wocr_ctx *ctx, char *buf, int32_t cap) {
    return guard([&] {
        if (!ctx || !buf || cap <= 0) fail(WOCR_ERR_INVALID, "null argument");
        std::snprintf(buf, (size_t)cap, "%s", ctx->c.name.c_str());
    });
}

void *wocr_ctx_stream(wocr_ctx *ctx) { return ctx ? (void *)ctx->c.stream : nullptr; }

int32_t wocr_ctx_sync(wocr_ctx *ctx, int32_t timeout_ms) {
    return guard([&] {
        if (!ctx) fail(WOCR_ERR_INVALID, "null ctx");
        WOCR_CUDA(cudaSetDevice(ctx->c.device));
        sync_bounded(&ctx->c, timeout_ms);
    });
}

int64_t wocr_ctx_pool_bytes(wocr_ctx *ctx) {
    if (!ctx) return -1;
    uint64_t v = 0;
    if (cudaMemPoolGetAttribute(ctx->c.pool, cudaMemPoolAttrReservedMemCurrent, &v) != cudaSuccess) return -1;
    return (int64_t)v;
}

int64_t wocr_ctx_launches(wocr_ctx *ctx) { return ctx ? ctx->c.launches : -1; }

int32_t wocr_ctx_profile(wocr_ctx *ctx, int32_t on) {
    return guard([&] {
        if (!ctx) fail(WOCR_ERR_INVALID, "null ctx");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
        for (auto &r : c->recs) {
            c->spare.push_back(r.a);
            c->spare.push_back(r.b);
        }
        c->recs.clear();
        c->prof = on != 0;
    });
}

int32_t wocr_ctx_profile_report(wocr_ctx *ctx, char *buf, int32_t cap) {
    return guard([&] {
        if (!ctx || !buf || cap <= 0) fail(WOCR_ERR_INVALID, "null argument");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
        struct Agg {
            int64_t n = 0;
            double ms = 0, flops = 0, bytes = 0;
        };
        std::map<std::string, Agg> agg;
        for (auto &r : c->recs) {
            float ms = 0;
            WOCR_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
            Agg &a = agg[r.name];
            a.n++;
            a.ms += ms;
            a.flops += r.flops;
            a.bytes += r.bytes;
        }
        std::string s = "[";
        for (auto &kv : agg) {
            char tmp[512];
            std::snprintf(tmp, sizeof tmp, "%s{\"kernel\": \"%s\", \"launches\": %lld, \"ms\": %.6f, \"flops\": %.6e, \"bytes\": %.6e}",
                          s.size() > 1 ? ", " : "", kv.first.c_str(), (long long)kv.second.n, kv.second.ms,
                          kv.second.flops, kv.second.bytes);
            s += tmp;
        }
        s += "]";
        if ((int64_t)s.size() + 1 > cap) fail(WOCR_ERR_CAPACITY, "report needs " + std::to_string(s.size() + 1) + " bytes");
        std::memcpy(buf, s.c_str(), s.size() + 1);
    });
}

int32_t wocr_ctx_profile_launches(wocr_ctx *ctx, char *buf, int32_t cap) {
    return guard([&] {
        if (!ctx || !buf || cap <= 0) fail(WOCR_ERR_INVALID, "null argument");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
        std::string s = "[";
        for (auto &r : c->recs) {
            float ms = 0;
            WOCR_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
            char tmp[256];
            std::snprintf(tmp, sizeof tmp, "%s{\"kernel\": \"%s\", \"ms\": %.6f, \"flops\": %.6e, \"bytes\": %.6e}",
                          s.size() > 1 ? ", " : "", r.name, ms, r.flops, r.bytes);
            s += tmp;
        }
        s += "]";
        if ((int64_t)s.size() + 1 > cap) fail(WOCR_ERR_CAPACITY, "report needs " + std::to_string(s.size() + 1) + " bytes");
        std::memcpy(buf, s.c_str(), s.size() + 1);
    });
}

int32_t wocr_host_alloc(size_t bytes, void **out) {
    return guard([&] {
        if (!out) fail(WOCR_ERR_INVALID, "null out");
        WOCR_CUDA(cudaHostAlloc(out, bytes ? bytes : 16, cudaHostAllocPortable));
    });
}

void wocr_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

// ---- detector ---------------------------------------------------------------------------
}  // extern "C"

// Detector::new from a parsed model (wocr_detector_create, and the lanes of the ocrs page
// pipeline, which rebuild their detectors from the model kept at create time).
static wocr_detector *detector_from_model(wocr_ctx *ctx, const Model &m) {
    WOCR_CUDA(cudaSetDevice(ctx->c.device));
    auto *d = new wocr_detector();
    d->ctx = ctx;
    ctx->refs++;
    try {
        d->graph = build_graph(&ctx->c, m, nullptr, nullptr);
        WOCR_CUDA(cudaStreamSynchronize(ctx->c.stream));
    } catch (...) {
        delete d;
        ctx_release(ctx);
        throw;
    }
    return d;
}

extern "C" {

int32_t wocr_detector_create(wocr_ctx *ctx, const wocr_model *model, wocr_detector **out) {
    return guard([&] {
        if (!ctx || !out) fail(WOCR_ERR_INVALID, "null argument");
        WOCR_CUDA(cudaSetDevice(ctx->c.device));
        *out = detector_from_model(ctx, model_from_c(model));
    });
}

void wocr_detector_destroy(wocr_detector *det) {
    if (!det) return;
    wocr_ctx *ctx = det->ctx;
    cudaSetDevice(ctx->c.device);
    cudaStreamSynchronize(ctx->c.stream);
    delete det;
    ctx_release(ctx);
}

static void detect_pages_dev(wocr_detector *det, const uint8_t *d_rgb, int n, int w, int h, float thr,
                             uint32_t *d_mask, const int2 *rows = nullptr) {
    Ctx *c = &det->ctx->c;
    if (n <= 0 || w <= 0 || h <= 0) fail(WOCR_ERR_INVALID, "empty page");
    const int mh = 800, mw = 600;  // the model size (src/gpu.rs:1394)
    int ph = std::max(h, mh), pw = std::max(w, mw);
    DT in = new_nhwc(c, n, 1, mh, mw);
    if (rows) k::grey_resize_rows(c, d_rgb, rows, n, w, mh, mw, in.p);
    else k::grey_resize(c, d_rgb, (int64_t)w * h * 3, n, w, h, mh, mw, in.p);
    DT m = det->graph->run(in);
    if (m.rank() != 4 || m.shape[0] != n || m.shape[1] != 1)
        fail(WOCR_ERR_SHAPE, "detection output " + shape_str(m.shape));
    int vh = mh - (ph - h) * mh / ph, vw = mw - (pw - w) * mw / pw;
    if (m.shape[2] < vh || m.shape[3] < vw) fail(WOCR_ERR_SHAPE, "detection output " + shape_str(m.shape));
    // C = 1: row stride strides[2], plane strides[0]
    k::mask_up(c, m.p, (int)m.strides[2], m.strides[0], n, vw, vh, w, h, thr, d_mask);
}

// detect_pages_dev through the detector's graph cache (direct when profiling, or with
// WOCR_NO_GRAPH set).
static void detect_pages_run(wocr_detector *det, const uint8_t *d_rgb, int n, int w, int h, float thr,
                             uint32_t *d_mask, const int2 *rows = nullptr) {
    Ctx *c = &det->ctx->c;
    if (c->prof || std::getenv("WOCR_NO_GRAPH")) {
        detect_pages_dev(det, d_rgb, n, w, h, thr, d_mask, rows);
        return;
    }
    DetGraph *g = nullptr;
    for (auto &e : det->graphs)
        if (e.exec && e.n == n && e.w == w && e.h == h && e.thr == thr && e.rgb == d_rgb && e.mask == d_mask &&
            e.rows == rows)
            g = &e;
    if (!g) {
        g = &det->graphs[0];
        for (auto &e : det->graphs)
            if (!e.exec || e.used < g->used) g = &e;
        g->reset();
        const double f0 = c->flops;
        const int64_t l0 = c->launches;
        WOCR_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
        try {
            detect_pages_dev(det, d_rgb, n, w, h, thr, d_mask, rows);
        } catch (...) {
            cudaGraph_t dead = nullptr;
            cudaStreamEndCapture(c->stream, &dead);
            if (dead) cudaGraphDestroy(dead);
            throw;
        }
        WOCR_CUDA(cudaStreamEndCapture(c->stream, &g->graph));
        WOCR_CUDA(cudaGraphInstantiate(&g->exec, g->graph, 0));
        g->n = n;
        g->w = w;
        g->h = h;
        g->thr = thr;
        g->rgb = d_rgb;
        g->mask = d_mask;
        g->rows = rows;
        g->flops = c->flops - f0;
        g->launches = c->launches - l0;
        c->flops = f0;
        c->launches = l0;
    }
    g->used = ++det->uses;
    WOCR_CUDA(cudaGraphLaunch(g->exec, c->stream));
    c->flops += g->flops;
    c->launches += g->launches;
}

int32_t wocr_detect_pages_device(wocr_detector *det, const uint8_t *d_rgb, int32_t n, int32_t w, int32_t h,
                                 float threshold, uint32_t *d_mask_out) {
    return guard([&] {
        if (!det || !d_rgb || !d_mask_out) fail(WOCR_ERR_INVALID, "null argument");
        RunScope rs(&det->ctx->c, &det->last);
        detect_pages_run(det, d_rgb, n, w, h, threshold, d_mask_out);
    });
}

// The row plan of a page size (RowPlan), built on its first use.
static const RowPlan &row_plan(wocr_detector *det, int w, int h) {
    RowPlan &pl = det->plan;
    if (pl.w == w && pl.h == h) return pl;
    pl = RowPlan();
    pl.w = w;
    pl.h = h;
    const int mh = 800;  // the model height (src/gpu.rs:1394)
    const int ph = std::max(h, mh);
    const float sy = (float)ph / (float)mh;
    pl.y1.resize(mh);
    pl.y2.resize(mh);
    std::vector<int2> table(mh);
    for (int oy = 0; oy < mh; oy++) {
        volatile float t = sy * ((float)oy + 0.5f);  // rounded before the subtraction, as K13 states it
        const float iy = std::fmin(std::fmax(t - 0.5f, 0.f), (float)ph - 1.f);
        const int y1 = (int)iy, y2 = std::min(y1 + 1, ph - 1);
        const float wy = iy - (float)y1;
        pl.y1[oy] = y1;
        pl.y2[oy] = y2;
        int wb;
        std::memcpy(&wb, &wy, 4);
        table[oy] = make_int2(wb, (y1 >= h ? 1 : 0) | (y2 >= h ? 2 : 0));
    }
    pl.bytes = (size_t)2 * mh * w * 3;
    if (h <= 2 * mh) return pl;  // the compacted page would not be smaller
    int R = 0;  // the regular prefix: (y1, y1 + 1) pairs inside the page
    while (R < mh && pl.y1[R] + 1 < h && pl.y2[R] == pl.y1[R] + 1) R++;
    for (int k = 1; k <= 64 && k < R; k++) {
        const int P = pl.y1[k] - pl.y1[0];
        bool good = P >= 2;
        for (int oy = 0; good && oy + k < R; oy++) good = pl.y1[oy + k] - pl.y1[oy] == P;
        if (good) {
            pl.k = k;
            pl.P = P;
            break;
        }
    }
    if (!pl.k) return pl;
    pl.regular = R;
    pl.first.assign(pl.k, 0);
    pl.count.assign(pl.k, 0);
    for (int j = 0; j < pl.k && j < R; j++) {
        pl.first[j] = pl.y1[j];
        pl.count[j] = (R - 1 - j) / pl.k + 1;
    }
    Ctx *c = &det->ctx->c;
    pl.table = alloc(c, mh * sizeof(int2));
    WOCR_CUDA(cudaMemcpyAsync(pl.table->p, table.data(), mh * sizeof(int2), cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaStreamSynchronize(c->stream));
    pl.ok = true;
    return pl;
}

// Pages per chunk of wocr_detect_pages: the upload of one chunk overlaps the detection of the
// previous one and the read-back of the mask before, so what is left exposed is the PCIe upload
// or the detection, whichever is longer, plus one chunk of the other.  Whole pages (the upload
// the longer part): one page per chunk up to 12.  Compacted pages (the two about even): six
// chunks, two pages each for 12, since a pass over one page fills the SMs poorly in the deep
// layers (measured on 12-page steps: 2850 pages/s against 2420).  WOCR_DETECT_CHUNK overrides
// (0 = one chunk).
static int detect_chunk(int n, bool compact) {
    if (const char *e = std::getenv("WOCR_DETECT_CHUNK")) {
        int v = std::atoi(e);
        return v <= 0 ? n : std::min(v, n);
    }
    return compact ? std::max(1, (n + 5) / 6) : std::max(1, (n + 11) / 12);
}

int32_t wocr_detect_pages(wocr_detector *det, const uint8_t *rgb, int32_t n, int32_t w, int32_t h, float threshold,
                          uint32_t *mask_out) {
    return guard([&] {
        if (!det || !rgb || !mask_out) fail(WOCR_ERR_INVALID, "null argument");
        if (n <= 0 || w <= 0 || h <= 0) fail(WOCR_ERR_INVALID, "empty page");
        Ctx *c = &det->ctx->c;
        RunScope rs(c, &det->last);
        const size_t page_bytes = (size_t)w * h * 3, page_words = (size_t)h * ((w + 31) / 32);
        // tall pages go up compacted: only the rows the grey/resize reads (RowPlan)
        const RowPlan &pl = row_plan(det, w, h);
        const bool compact = pl.ok && !std::getenv("WOCR_WHOLE_PAGES");
        const int chunk = detect_chunk(n, compact), nchunks = (n + chunk - 1) / chunk;
        const size_t up_page = compact ? pl.bytes : page_bytes, rb = (size_t)w * 3;
        if (!det->copy) {
            WOCR_CUDA(cudaStreamCreateWithFlags(&det->copy, cudaStreamNonBlocking));
            WOCR_CUDA(cudaStreamCreateWithFlags(&det->copy_back, cudaStreamNonBlocking));
            for (cudaEvent_t *e : {&det->ready, &det->up[0], &det->up[1], &det->done[0], &det->done[1], &det->back[0],
                                   &det->back[1], &det->fin})
                WOCR_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
        }
        for (int b = 0; b < std::min(nchunks, 2); b++) {
            if (!det->up_buf[b] || det->up_buf[b]->bytes < (size_t)chunk * up_page)
                det->up_buf[b] = alloc(c, (size_t)chunk * up_page);
            if (!det->mask_buf[b] || det->mask_buf[b]->bytes < (size_t)chunk * page_words * 4)
                det->mask_buf[b] = alloc(c, (size_t)chunk * page_words * 4);
        }
        BufP src[2] = {det->up_buf[0], det->up_buf[1]}, dst[2] = {det->mask_buf[0], det->mask_buf[1]};
        // nothing of the copy streams may still run when the buffers go back to the pool
        struct Drain {
            cudaStream_t s[2];
            ~Drain() {
                cudaStreamSynchronize(s[0]);
                cudaStreamSynchronize(s[1]);
            }
        } drain{{det->copy, det->copy_back}};
        WOCR_CUDA(cudaEventRecord(det->ready, c->stream));
        WOCR_CUDA(cudaStreamWaitEvent(det->copy, det->ready, 0));
        WOCR_CUDA(cudaStreamWaitEvent(det->copy_back, det->ready, 0));
        for (int i = 0; i < nchunks; i++) {
            const int slot = i & 1, k0 = i * chunk, kn = std::min(chunk, n - k0);
            // the slot's upload buffer is free once the detection of chunk i - 2 has read it,
            // its mask buffer once that chunk's mask is back on the host
            if (i >= 2) {
                WOCR_CUDA(cudaStreamWaitEvent(det->copy, det->done[slot], 0));
                WOCR_CUDA(cudaStreamWaitEvent(c->stream, det->back[slot], 0));
            }
            if (compact) {
                for (int pg = 0; pg < kn; pg++) {
                    const uint8_t *page = rgb + (size_t)(k0 + pg) * page_bytes;
                    uint8_t *cp = (uint8_t *)src[slot]->p + (size_t)pg * pl.bytes;
                    // the row pairs of phase j: output rows j, j + k, ... -> compacted rows 2 oy, 2 oy + 1
                    for (int j = 0; j < pl.k; j++)
                        if (pl.count[j]) {
                            WOCR_CUDA(cudaMemcpy2DAsync(cp + 2 * (size_t)j * rb, 2 * (size_t)pl.k * rb,
                                                        page + (size_t)pl.first[j] * rb, (size_t)pl.P * rb, 2 * rb,
                                                        pl.count[j], cudaMemcpyHostToDevice, det->copy));
                            det->last.h2d += (int64_t)(2 * rb * pl.count[j]);
                        }
                    for (int oy = pl.regular; oy < 800; oy++)
                        for (int r = 0; r < 2; r++) {
                            const int yy = r ? pl.y2[oy] : pl.y1[oy];
                            if (yy >= h) continue;  // padding: not read
                            WOCR_CUDA(cudaMemcpyAsync(cp + (2 * (size_t)oy + r) * rb, page + (size_t)yy * rb, rb,
                                                      cudaMemcpyHostToDevice, det->copy));
                            det->last.h2d += (int64_t)rb;
                        }
                }
            } else {
                WOCR_CUDA(cudaMemcpyAsync(src[slot]->p, rgb + (size_t)k0 * page_bytes, (size_t)kn * page_bytes,
                                          cudaMemcpyHostToDevice, det->copy));
                det->last.h2d += (int64_t)(kn * page_bytes);
            }
            WOCR_CUDA(cudaEventRecord(det->up[slot], det->copy));
            WOCR_CUDA(cudaStreamWaitEvent(c->stream, det->up[slot], 0));
            detect_pages_run(det, (const uint8_t *)src[slot]->p, kn, w, h, threshold, (uint32_t *)dst[slot]->p,
                             compact ? (const int2 *)pl.table->p : nullptr);
            WOCR_CUDA(cudaEventRecord(det->done[slot], c->stream));
            WOCR_CUDA(cudaStreamWaitEvent(det->copy_back, det->done[slot], 0));
            WOCR_CUDA(cudaMemcpyAsync(mask_out + (size_t)k0 * page_words, dst[slot]->p, (size_t)kn * page_words * 4,
                                      cudaMemcpyDeviceToHost, det->copy_back));
            det->last.d2h += (int64_t)(kn * page_words * 4);
            WOCR_CUDA(cudaEventRecord(det->back[slot], det->copy_back));
        }
        // the context stream ends after the last read-back, so the bounded wait covers it
        WOCR_CUDA(cudaEventRecord(det->fin, det->copy_back));
        WOCR_CUDA(cudaStreamWaitEvent(c->stream, det->fin, 0));
        sync_bounded(c, 0);
    });
}

int32_t wocr_detect_page(wocr_detector *det, const uint8_t *rgb, int32_t w, int32_t h, float threshold,
                         uint32_t *mask_out) {
    return wocr_detect_pages(det, rgb, 1, w, h, threshold, mask_out);
}

int32_t wocr_detect(wocr_detector *det, const float *input, int32_t h, int32_t w, float *prob_out, int64_t cap,
                    int32_t *out_h, int32_t *out_w) {
    return guard([&] {
        if (!det || !input || h <= 0 || w <= 0) fail(WOCR_ERR_INVALID, "bad argument");
        Ctx *c = &det->ctx->c;
        RunScope rs(c, &det->last);
        DT x = from_host(c, input, {1, 1, h, w});
        DT out = to_rowmajor(c, det->graph->run(x));
        if (out.rank() != 4) fail(WOCR_ERR_SHAPE, "detection output " + shape_str(out.shape));
        if (out_h) *out_h = (int32_t)out.shape[2];
        if (out_w) *out_w = (int32_t)out.shape[3];
        if (prob_out) {
            if (cap < out.numel()) fail(WOCR_ERR_CAPACITY, "output buffer too small for " + shape_str(out.shape));
            d2h(c, prob_out, out.p, (size_t)out.numel() * 4);
        }
        sync_bounded(c, 0);
    });
}

// ---- recogniser -------------------------------------------------------------------------
}  // extern "C"

// Recognizer::new from a parsed model (wocr_recognizer_create and the ocrs pipeline's lanes).
static wocr_recognizer *recognizer_from_model(wocr_ctx *ctx, const Model &m, int32_t lines) {
    Ctx *c = &ctx->c;
    WOCR_CUDA(cudaSetDevice(c->device));
    auto *r = new wocr_recognizer();
    r->ctx = ctx;
    ctx->refs++;
    r->lines = lines > 0 ? lines : c->lines;
    try {
        Node pool;
        r->trunk = build_graph(c, m, "AveragePool", &pool);
        if (pool.op.empty()) fail(WOCR_ERR_UNSUPPORTED, "no AveragePool in the recognition model");
        auto kv = pool.ints("kernel_shape");
        if (!kv) fail(WOCR_ERR_UNSUPPORTED, "AveragePool without kernel_shape");
        auto sv = pool.ints("strides");
        if (kv->size() != 2 || (*kv)[1] != 1 || !sv || *sv != *kv)
            fail(WOCR_ERR_UNSUPPORTED, "unsupported AveragePool " + shape_str(*kv));
        r->pool_kh = (int)(*kv)[0];
        int nl = 0;
        for (auto &n : m.nodes) {
            if (n.op != "GRU") continue;
            if (n.int_("hidden_size").value_or(0) != 256 || n.int_("linear_before_reset").value_or(0) != 1 ||
                n.str("direction").value_or("") != "bidirectional")
                fail(WOCR_ERR_UNSUPPORTED, "unsupported GRU attributes");
            if (nl >= 2) {
                nl++;
                continue;
            }
            const HostW &W = m.weight(n.in(1)), &R = m.weight(n.in(2)), &B = m.weight(n.in(3));
            if (W.dims.size() != 3 || W.dims[0] != 2 || W.dims[1] != 768 || R.data.size() != 2 * 768 * 256 ||
                B.data.size() != 2 * 1536)
                fail(WOCR_ERR_SHAPE, "GRU weights " + shape_str(W.dims));
            int input = (int)W.dims[2];
            // W [2][768][in] as rows of the projection -> [in][1536] (src/gpu.rs:1466-1472)
            std::vector<float> wt((size_t)input * 1536);
            for (int row = 0; row < 1536; row++)
                for (int i = 0; i < input; i++) wt[(size_t)i * 1536 + row] = W.data[(size_t)row * input + i];
            std::vector<float> wb, rb;
            for (int dir = 0; dir < 2; dir++) {
                wb.insert(wb.end(), B.data.begin() + dir * 1536, B.data.begin() + dir * 1536 + 768);
                rb.insert(rb.end(), B.data.begin() + dir * 1536 + 768, B.data.begin() + dir * 1536 + 1536);
            }
            GruLayer &L = r->layers[nl];
            L.input = input;
            L.w_t = upload(c, wt);
            L.uw = linear_umma(c, wt.data(), input, 1536);
            L.wb = upload(c, wb);
            L.r = upload(c, R.data);
            L.rb = upload(c, rb);
            nl++;
        }
        if (nl != 2) fail(WOCR_ERR_UNSUPPORTED, std::to_string(nl) + " GRU layers");
        const Node *mm = nullptr;
        for (auto &n : m.nodes)
            if (n.op == "MatMul") {
                mm = &n;
                break;
            }
        if (!mm) fail(WOCR_ERR_UNSUPPORTED, "no MatMul");
        const HostW &lin = m.weight(mm->in(1));  // [512][classes]
        if (lin.dims.size() != 2 || lin.dims[0] != 512) fail(WOCR_ERR_SHAPE, "output layer " + shape_str(lin.dims));
        const Node *add = nullptr;
        for (auto &n : m.nodes)
            if (n.op == "Add" && std::find(n.inputs.begin(), n.inputs.end(), mm->outputs[0]) != n.inputs.end()) {
                add = &n;
                break;
            }
        if (!add) fail(WOCR_ERR_UNSUPPORTED, "no bias Add");
        const HostW *bias = nullptr;
        for (auto &i : add->inputs)
            if (m.weights.count(i)) {
                bias = &m.weights.at(i);
                break;
            }
        if (!bias) fail(WOCR_ERR_UNSUPPORTED, "no bias weight");
        r->classes = (int)lin.dims[1];
        r->ldw = (r->classes + 3) / 4 * 4;
        std::vector<float> lw((size_t)512 * r->ldw, 0.f), lb(r->ldw, 0.f);
        for (int i = 0; i < 512; i++)
            for (int q = 0; q < r->classes; q++) lw[(size_t)i * r->ldw + q] = lin.data[(size_t)i * r->classes + q];
        for (int q = 0; q < r->classes && q < (int)bias->data.size(); q++) lb[q] = bias->data[q];
        r->lin_w = upload(c, lw);
        r->lin_uw = linear_umma(c, lin.data.data(), 512, r->classes);
        r->lin_b = upload(c, lb);
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
    } catch (...) {
        delete r;
        ctx_release(ctx);
        throw;
    }
    return r;
}

extern "C" {

int32_t wocr_recognizer_create(wocr_ctx *ctx, const wocr_model *model, int32_t lines, wocr_recognizer **out) {
    return guard([&] {
        if (!ctx || !out) fail(WOCR_ERR_INVALID, "null argument");
        WOCR_CUDA(cudaSetDevice(ctx->c.device));
        *out = recognizer_from_model(ctx, model_from_c(model), lines);
    });
}

void wocr_recognizer_destroy(wocr_recognizer *rec) {
    if (!rec) return;
    wocr_ctx *ctx = rec->ctx;
    cudaSetDevice(ctx->c.device);
    cudaStreamSynchronize(ctx->c.stream);
    delete rec;
    ctx_release(ctx);
}

// Trunk output width of a batch of width w: follows the trunk's pooling/strides exactly by
// running shape arithmetic of the lowered steps.
static int trunk_width(wocr_recognizer *rec, int w, int *h_out) {
    int64_t h = 64, wd = w;
    for (auto &s : rec->trunk->steps) {
        switch (s.kind) {
        case Step::G_DIRECT:
            h = (h + 2 * s.conv.pads[0] - s.conv.kh + 1) / s.conv.pool_h;
            wd = (wd + 2 * s.conv.pads[0] - s.conv.kw + 1) / s.conv.pool_w;
            break;
        case Step::G_CONV:
        case Step::G_DEPTHWISE:
            h = (h + 2 * s.conv.pads[0] - s.conv.kh) / s.conv.sh + 1;
            wd = (wd + 2 * s.conv.pads[0] - s.conv.kw) / s.conv.sw + 1;
            break;
        case Step::G_CONVT:
            h = (h - 1) * s.convt.s + s.convt.kh;
            wd = (wd - 1) * s.convt.s + s.convt.kw;
            break;
        case Step::G_MAXPOOL:
            h /= s.conv.kh;
            wd /= s.conv.kw;
            break;
        default:
            break;
        }
    }
    if (h_out) *h_out = (int)h;
    return (int)wd;
}

int32_t wocr_recognizer_dims(wocr_recognizer *rec, const int32_t *batch_n, const int32_t *batch_w, int32_t n_batches,
                             int32_t *tmax, int32_t *ntot, int32_t *classes) {
    return guard([&] {
        if (!rec || (n_batches > 0 && (!batch_n || !batch_w))) fail(WOCR_ERR_INVALID, "null argument");
        int tm = 0, nt = 0;
        for (int b = 0; b < n_batches; b++) {
            tm = std::max(tm, trunk_width(rec, batch_w[b], nullptr));
            nt += batch_n[b];
        }
        if (tmax) *tmax = tm;
        if (ntot) *ntot = nt;
        if (classes) *classes = rec->classes;
    });
}

// The recognition pass on device batches (src/gpu.rs:1510-1602): trunks, time-major pooling, two
// GRU layers, the output layer, the arg-max.  `lens_d` (optional) holds the line lengths already.
// Returns the logits [tmax][ntot][classes] (and, with want_best, the arg-max [tmax][ntot], into
// d_best when given).
struct RecResult {
    DT logits;
    BufP best;
    int ntot = 0, tmax = 0;
    std::vector<int> lens;
};

static RecResult recognize_dev(wocr_recognizer *rec, const std::vector<DT> &xs, const int *lens_d_in, bool want_best,
                               uint32_t *d_best, bool branches = false) {
    Ctx *c = &rec->ctx->c;
    std::vector<DT> trunks;
    if (branches && xs.size() > 1) {
        // trunks on the side streams (captured as parallel branches of the graph)
        cudaStream_t main = c->stream;
        WOCR_CUDA(cudaEventRecord(rec->fork, main));
        const int ns = std::min<int>(wocr_recognizer::kSide, (int)xs.size());
        for (int i = 0; i < ns; i++) WOCR_CUDA(cudaStreamWaitEvent(rec->side[i], rec->fork, 0));
        struct Restore {
            Ctx *c;
            cudaStream_t s;
            ~Restore() { c->stream = s; }
        } restore{c, main};
        for (size_t b = 0; b < xs.size(); b++) {
            c->stream = rec->side[b % ns];
            trunks.push_back(rec->trunk->run(xs[b]));
        }
        c->stream = main;
        for (int i = 0; i < ns; i++) {
            WOCR_CUDA(cudaEventRecord(rec->join[i], rec->side[i]));
            WOCR_CUDA(cudaStreamWaitEvent(main, rec->join[i], 0));
        }
    } else {
        for (auto &x : xs) trunks.push_back(rec->trunk->run(x));
    }
    int ntot = 0, tmax = 0;
    for (auto &t : trunks) {
        ntot += (int)t.shape[0];
        tmax = std::max(tmax, (int)t.shape[3]);
    }
    int ch = (int)trunks[0].shape[1];
    if (ch != rec->layers[0].input)
        fail(WOCR_ERR_SHAPE, "trunk gives " + std::to_string(ch) + " features, GRU takes " +
                                 std::to_string(rec->layers[0].input));
    int64_t m = (int64_t)tmax * ntot;
    DT x = new_rowmajor(c, {tmax, ntot, ch});
    WOCR_CUDA(cudaMemsetAsync(x.p, 0, (size_t)x.numel() * 4, c->stream));
    std::vector<int> hl;
    int noff = 0;
    for (auto &t : trunks) {
        int n = (int)t.shape[0], tc = (int)t.shape[1], h = (int)t.shape[2], w = (int)t.shape[3];
        if (tc != ch) fail(WOCR_ERR_SHAPE, "trunk channels differ between batches");
        if ((h - rec->pool_kh) / rec->pool_kh + 1 != 1 || h < rec->pool_kh)
            fail(WOCR_ERR_SHAPE, "trunk height " + std::to_string(h) + " does not pool to one row");
        DT tn = to_nhwc(c, t);
        k::avgpool_t(c, tn.p, tn.strides[0], tn.pix(), n, ch, h, w, rec->pool_kh, ntot, noff, x.p);
        for (int q = 0; q < n; q++) hl.push_back(w);
        noff += n;
    }
    BufP lens_own;
    const int *lens_d = lens_d_in;
    if (!lens_d) {
        lens_own = alloc(c, hl.size() * sizeof(int));
        WOCR_CUDA(cudaMemcpyAsync(lens_own->p, hl.data(), hl.size() * sizeof(int), cudaMemcpyHostToDevice,
                                  c->stream));
        lens_d = (const int *)lens_own->p;
    }
    DT in = x;
    for (int l = 0; l < 2; l++) {
        GruLayer &L = rec->layers[l];
        DT gates = linear_run(c, in, L.w_t, L.wb, L.input, 1536, 1536, 0, L.uw.get());
        DT yo = new_rowmajor(c, {tmax, ntot, 512});
        WOCR_CUDA(cudaMemsetAsync(yo.p, 0, (size_t)yo.numel() * 4, c->stream));
        k::gru_layer(c, gates.p, L.r.p, L.rb.p, lens_d, tmax, ntot, yo.p);
        in = yo;
    }
    RecResult res;
    res.logits = linear_run(c, in, rec->lin_w, rec->lin_b, 512, rec->classes, rec->ldw, 0, rec->lin_uw.get());
    if (want_best) {
        if (!d_best) {
            res.best = alloc(c, (size_t)std::max<int64_t>(m, 1) * 4);
            d_best = (uint32_t *)res.best->p;
        }
        k::argmax(c, res.logits.p, m, rec->classes, rec->classes, d_best, nullptr, nullptr, 1);
    }
    res.ntot = ntot;
    res.tmax = tmax;
    res.lens = hl;
    return res;
}

int32_t wocr_recognize(wocr_recognizer *rec, const float *const *batches, const int32_t *batch_n,
                       const int32_t *batch_w, int32_t n_batches, float *logits, int64_t logits_cap, int32_t *lens,
                       uint32_t *best, int32_t *tmax_out) {
    return guard([&] {
        if (!rec || n_batches <= 0 || !batches || !batch_n || !batch_w) fail(WOCR_ERR_INVALID, "no batches");
        Ctx *c = &rec->ctx->c;
        RunScope rs(c, &rec->last);
        for (int b = 0; b < n_batches; b++)
            if (batch_n[b] <= 0 || batch_w[b] <= 0 || !batches[b]) fail(WOCR_ERR_INVALID, "empty batch");
        std::vector<int32_t> bn(batch_n, batch_n + n_batches), bw(batch_w, batch_w + n_batches);
        const int want = (logits ? 1 : 0) | (best ? 2 : 0);
        // the replay entry of this layout
        RecReplay *r = nullptr;
        bool first = false;
        if (!c->prof && !std::getenv("WOCR_NO_GRAPH")) {
            for (auto &e : rec->replays)
                if (e.want == want && e.bn == bn && e.bw == bw) r = &e;
            if (!r) {
                r = &rec->replays[0];
                for (auto &e : rec->replays)
                    if (e.want < 0 || e.used < r->used) r = &e;
                r->reset();
                r->want = want;
                r->bn = bn;
                r->bw = bw;
                first = true;
            }
            r->used = ++rec->uses;
        }
        int ntot = 0, tmax = 0;
        std::vector<int> hl;
        if (!r || first) {
            std::vector<DT> xs;
            for (int b = 0; b < n_batches; b++) xs.push_back(from_host(c, batches[b], {bn[b], 1, 64, bw[b]}));
            RecResult res = recognize_dev(rec, xs, nullptr, best != nullptr, nullptr);
            ntot = res.ntot;
            tmax = res.tmax;
            hl = res.lens;
            const int64_t m = (int64_t)tmax * ntot;
            if (logits) {
                if (logits_cap < m * rec->classes) fail(WOCR_ERR_CAPACITY, "logits buffer too small");
                d2h(c, logits, res.logits.p, (size_t)m * rec->classes * 4);
            }
            if (best) d2h(c, best, res.best->p, (size_t)m * 4);
            sync_bounded(c, 0);
            if (r) {
                r->ntot = ntot;
                r->tmax = tmax;
                r->lens = hl;
            }
        } else {
            ntot = r->ntot;
            tmax = r->tmax;
            hl = r->lens;
            const int64_t m = (int64_t)tmax * ntot;
            if (logits && logits_cap < m * rec->classes) fail(WOCR_ERR_CAPACITY, "logits buffer too small");
            if (!r->exec) {
                size_t total = 0;
                r->in_off.clear();
                for (int b = 0; b < n_batches; b++) {
                    r->in_off.push_back(total);
                    total += (size_t)bn[b] * 64 * bw[b];
                }
                r->in = alloc(c, total * 4);
                r->lens_d = alloc(c, hl.size() * sizeof(int));
                WOCR_CUDA(cudaMemcpyAsync(r->lens_d->p, hl.data(), hl.size() * sizeof(int), cudaMemcpyHostToDevice,
                                          c->stream));
                if (logits) r->logits = alloc(c, (size_t)m * rec->classes * 4);
                if (best) r->best = alloc(c, (size_t)m * 4);
                WOCR_CUDA(cudaStreamSynchronize(c->stream));  // lens uploaded before capture
                if (!rec->fork) {
                    for (int i = 0; i < wocr_recognizer::kSide; i++) {
                        WOCR_CUDA(cudaStreamCreateWithFlags(&rec->side[i], cudaStreamNonBlocking));
                        WOCR_CUDA(cudaEventCreateWithFlags(&rec->join[i], cudaEventDisableTiming));
                    }
                    WOCR_CUDA(cudaEventCreateWithFlags(&rec->fork, cudaEventDisableTiming));
                }
                const double f0 = c->flops;
                const int64_t l0 = c->launches;
                WOCR_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
                try {
                    std::vector<DT> xs;
                    for (int b = 0; b < n_batches; b++) {
                        DT x;
                        x.buf = r->in;
                        x.p = (float *)r->in->p + r->in_off[b];
                        x.shape = {bn[b], 1, 64, bw[b]};
                        x.strides = rowmajor_strides(x.shape);
                        xs.push_back(x);
                    }
                    RecResult res = recognize_dev(rec, xs, (const int *)r->lens_d->p, best != nullptr,
                                                  best ? (uint32_t *)r->best->p : nullptr, true);
                    if (res.ntot != ntot || res.tmax != tmax)
                        fail(WOCR_ERR_SHAPE, "recognition sizes changed between calls");
                    if (logits)
                        WOCR_CUDA(cudaMemcpyAsync(r->logits->p, res.logits.p, (size_t)m * rec->classes * 4,
                                                  cudaMemcpyDeviceToDevice, c->stream));
                } catch (...) {
                    cudaGraph_t dead = nullptr;
                    cudaStreamEndCapture(c->stream, &dead);
                    if (dead) cudaGraphDestroy(dead);
                    r->reset();
                    throw;
                }
                WOCR_CUDA(cudaStreamEndCapture(c->stream, &r->graph));
                WOCR_CUDA(cudaGraphInstantiate(&r->exec, r->graph, 0));
                r->flops = c->flops - f0;
                r->launches = c->launches - l0;
                c->flops = f0;
                c->launches = l0;
            }
            for (int b = 0; b < n_batches; b++)
                WOCR_CUDA(cudaMemcpyAsync((float *)r->in->p + r->in_off[b], batches[b],
                                          (size_t)bn[b] * 64 * bw[b] * 4, cudaMemcpyHostToDevice, c->stream));
            WOCR_CUDA(cudaGraphLaunch(r->exec, c->stream));
            c->flops += r->flops;
            c->launches += r->launches;
            if (logits) d2h(c, logits, r->logits->p, (size_t)m * rec->classes * 4);
            if (best) d2h(c, best, r->best->p, (size_t)m * 4);
            sync_bounded(c, 0);
        }
        if (lens) std::memcpy(lens, hl.data(), hl.size() * sizeof(int));
        if (tmax_out) *tmax_out = tmax;
    });
}

// ---- N-D graph ----------------------------------------------------------------------------
}  // extern "C"

// An N-D graph handle on `ctx` from a parsed model (wocr_ndgraph_create, and the extra lanes of
// the page pipeline, which rebuild their graphs from the models kept at create time).
static wocr_ndgraph *ndgraph_from_model(wocr_ctx *ctx, const Model &m, bool stop_before_softmax) {
    WOCR_CUDA(cudaSetDevice(ctx->c.device));
    auto *g = new wocr_ndgraph();
    g->ctx = ctx;
    ctx->refs++;
    try {
        g->graph = build_ndgraph(&ctx->c, m, stop_before_softmax);
        WOCR_CUDA(cudaStreamSynchronize(ctx->c.stream));
    } catch (...) {
        delete g;
        ctx_release(ctx);
        throw;
    }
    return g;
}

extern "C" {

int32_t wocr_ndgraph_create(wocr_ctx *ctx, const wocr_model *model, int32_t stop_before_softmax, wocr_ndgraph **out) {
    return guard([&] {
        if (!ctx || !out) fail(WOCR_ERR_INVALID, "null argument");
        WOCR_CUDA(cudaSetDevice(ctx->c.device));
        *out = ndgraph_from_model(ctx, model_from_c(model), stop_before_softmax != 0);
    });
}

void wocr_ndgraph_destroy(wocr_ndgraph *g) {
    if (!g) return;
    wocr_ctx *ctx = g->ctx;
    cudaSetDevice(ctx->c.device);
    cudaStreamSynchronize(ctx->c.stream);
    delete g;
    ctx_release(ctx);
}

static DT nd_input(Ctx *c, const float *x, const int64_t *shape, int32_t rank) {
    if (!x || !shape || rank <= 0 || rank > kMaxRank) fail(WOCR_ERR_INVALID, "bad input tensor");
    std::vector<int64_t> s(shape, shape + rank);
    for (auto d : s)
        if (d <= 0) fail(WOCR_ERR_INVALID, "empty input tensor");
    return from_host(c, x, s);
}

static void put_shape(const DT &t, int64_t *out_shape, int32_t *out_rank) {
    if (out_rank) *out_rank = t.rank();
    if (out_shape)
        for (int d = 0; d < t.rank(); d++) out_shape[d] = t.shape[d];
}

// The replay entry of (shape, mode), or null on a first call (which then records one).
static NdReplay *nd_replay(wocr_ndgraph *g, const std::vector<int64_t> &shape, int mode, bool *first) {
    *first = false;
    if (g->ctx->c.prof || std::getenv("WOCR_NO_GRAPH")) return nullptr;
    for (auto &r : g->replays)
        if (r.mode == mode && r.in_shape == shape) {
            r.used = ++g->uses;
            return &r;
        }
    NdReplay *r = &g->replays[0];
    for (auto &e : g->replays)
        if (e.mode < 0 || e.used < r->used) r = &e;
    r->reset();
    r->mode = mode;
    r->in_shape = shape;
    r->used = ++g->uses;
    *first = true;
    return r;
}

// Capture the run (+ arg-max) from r->in into r's persistent outputs, once.
static void nd_capture(wocr_ndgraph *g, NdReplay *r) {
    if (r->exec) return;
    Ctx *c = &g->ctx->c;
    int64_t n = 1;
    for (auto d : r->in_shape) n *= d;
    r->in = alloc(c, (size_t)n * 4);
    if (r->mode == 0) {
        int64_t m = 1;
        for (auto d : r->out_shape) m *= d;
        r->out = alloc(c, (size_t)std::max<int64_t>(m, 1) * 4);
    } else {
        r->best = alloc(c, (size_t)r->rows * 4);
        r->mx = alloc(c, (size_t)r->rows * 4);
        r->lse = alloc(c, (size_t)r->rows * 4);
    }
    const double f0 = c->flops;
    const int64_t l0 = c->launches;
    WOCR_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
    try {
        DT x;
        x.buf = r->in;
        x.p = (float *)r->in->p;
        x.shape = r->in_shape;
        x.strides = rowmajor_strides(x.shape);
        Executor &ex = *g->graph;
        float *lse = r->mode == 1 ? (float *)r->lse->p : nullptr;  // run (0) and no-lse (4): none
        if (r->mode != 0 && ex.ends_in_linear() && !std::getenv("WOCR_UNFUSED_ARGMAX")) {
            DT xl = ex.run_to(x, (int)ex.steps.size() - 1);
            if (ex.linear_argmax(xl, (uint32_t *)r->best->p, (float *)r->mx->p, lse) != r->out_shape)
                fail(WOCR_ERR_SHAPE, "NdGraph output shape changed between runs");
        } else {
            DT y = to_rowmajor(c, ex.run(x));
            if (y.shape != r->out_shape) fail(WOCR_ERR_SHAPE, "NdGraph output shape changed between runs");
            if (r->mode == 0) {
                if (y.numel() > 0)
                    WOCR_CUDA(cudaMemcpyAsync(r->out->p, y.p, (size_t)y.numel() * 4, cudaMemcpyDeviceToDevice,
                                              c->stream));
            } else {
                k::argmax(c, y.p, r->rows, r->len, r->len, (uint32_t *)r->best->p, (float *)r->mx->p, lse, 0);
            }
        }
    } catch (...) {
        cudaGraph_t dead = nullptr;
        cudaStreamEndCapture(c->stream, &dead);
        if (dead) cudaGraphDestroy(dead);
        r->reset();
        throw;
    }
    WOCR_CUDA(cudaStreamEndCapture(c->stream, &r->graph));
    WOCR_CUDA(cudaGraphInstantiate(&r->exec, r->graph, 0));
    r->flops = c->flops - f0;
    r->launches = c->launches - l0;
    c->flops = f0;
    c->launches = l0;
}

static void nd_replay_launch(wocr_ndgraph *g, NdReplay *r, const float *x) {
    Ctx *c = &g->ctx->c;
    WOCR_CUDA(cudaMemcpyAsync(r->in->p, x, r->in->bytes, cudaMemcpyDefault, c->stream));
    WOCR_CUDA(cudaGraphLaunch(r->exec, c->stream));
    c->flops += r->flops;
    c->launches += r->launches;
}

static void put_dims(const std::vector<int64_t> &s, int64_t *out_shape, int32_t *out_rank) {
    if (out_rank) *out_rank = (int32_t)s.size();
    if (out_shape)
        for (size_t d = 0; d < s.size(); d++) out_shape[d] = s[d];
}

}  // extern "C"

// The bodies of NdGraph::run and NdGraph::run + argmax.  `read(dst, device src, bytes)` brings a
// result to the host: at once for the synchronous entry points (then a wait), or staged into a
// wocr_batch for the enqueue variants (NdGraph::argmax_record, src/nd.rs:1372-1380, read later by
// wocr_wait as Gpu::read_many reads, src/gpu.rs:1011-1037).
template <typename Read>
static void nd_run_core(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank, float *out,
                        int64_t out_cap, int64_t *out_shape, int32_t *out_rank, Read &&read) {
    Ctx *c = &g->ctx->c;
    if (!x || !shape || rank <= 0 || rank > kMaxRank) fail(WOCR_ERR_INVALID, "bad input tensor");
    bool first = false;
    NdReplay *r = nd_replay(g, std::vector<int64_t>(shape, shape + rank), 0, &first);
    if (!r || first) {
        DT y = g->graph->run(nd_input(c, x, shape, rank));
        put_shape(y, out_shape, out_rank);
        if (r) r->out_shape = y.shape;
        if (out) {
            if (out_cap < y.numel()) fail(WOCR_ERR_CAPACITY, "output buffer too small for " + shape_str(y.shape));
            y = to_rowmajor(c, y);
            read(out, y.p, (size_t)y.numel() * 4);
        }
        return;
    }
    put_dims(r->out_shape, out_shape, out_rank);
    int64_t m = 1;
    for (auto d : r->out_shape) m *= d;
    if (!out) return;
    if (out_cap < m) fail(WOCR_ERR_CAPACITY, "output buffer too small for " + shape_str(r->out_shape));
    nd_capture(g, r);
    nd_replay_launch(g, r, x);
    read(out, r->out->p, (size_t)m * 4);
}

template <typename Read>
static void nd_argmax_core(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank, uint32_t *best,
                           float *row_max, float *row_lse, int64_t cap, int64_t *rows_out, int64_t *out_shape,
                           int32_t *out_rank, Read &&read) {
    Ctx *c = &g->ctx->c;
    if (!x || !shape || rank <= 0 || rank > kMaxRank) fail(WOCR_ERR_INVALID, "bad input tensor");
    bool first = false;
    // without a log-sum-exp to read, the fused arg-max skips the exponentials' sums
    NdReplay *r = nd_replay(g, std::vector<int64_t>(shape, shape + rank), row_lse ? 1 : 4, &first);
    if (!r || first) {
        Executor &ex = *g->graph;
        DT in = nd_input(c, x, shape, rank);
        // a final linear layer (the CTC head) takes the arg-max into its epilogue
        const bool fused = ex.ends_in_linear() && !std::getenv("WOCR_UNFUSED_ARGMAX");
        DT y = fused ? ex.run_to(in, (int)ex.steps.size() - 1) : to_rowmajor(c, ex.run(in));
        std::vector<int64_t> oshape = y.shape;
        if (fused && !oshape.empty()) oshape.back() = ex.steps.back().ln;
        put_dims(oshape, out_shape, out_rank);
        int64_t len = oshape.empty() ? 1 : oshape.back(), rows = 1;
        for (auto d : oshape) rows *= d;
        rows /= std::max<int64_t>(len, 1);
        if (rows_out) *rows_out = rows;
        if (r) {
            r->out_shape = oshape;
            r->rows = rows;
            r->len = len;
        }
        if (cap < rows) fail(WOCR_ERR_CAPACITY, "argmax buffers too small");
        BufP b = alloc(c, (size_t)rows * 4), mx = alloc(c, (size_t)rows * 4), ls = alloc(c, (size_t)rows * 4);
        if (fused)
            ex.linear_argmax(y, (uint32_t *)b->p, (float *)mx->p, row_lse ? (float *)ls->p : nullptr);
        else
            k::argmax(c, y.p, rows, len, len, (uint32_t *)b->p, (float *)mx->p, row_lse ? (float *)ls->p : nullptr,
                      0);
        read(best, b->p, (size_t)rows * 4);
        read(row_max, mx->p, (size_t)rows * 4);
        read(row_lse, ls->p, (size_t)rows * 4);
        return;
    }
    put_dims(r->out_shape, out_shape, out_rank);
    if (rows_out) *rows_out = r->rows;
    if (cap < r->rows) fail(WOCR_ERR_CAPACITY, "argmax buffers too small");
    nd_capture(g, r);
    nd_replay_launch(g, r, x);
    read(best, r->best->p, (size_t)r->rows * 4);
    read(row_max, r->mx->p, (size_t)r->rows * 4);
    read(row_lse, r->lse->p, (size_t)r->rows * 4);
}

// ---- record, then read in one wait ------------------------------------------------------------
// The reference records NdGraph::run and argmax_record into one command encoder and reads every
// recorded buffer with one Gpu::read_many (src/bin/ocr-bench.rs:240-253).  A wocr_batch is that
// encoder's read list: each enqueue queues its work on the context stream and a device-to-host
// copy of its results into page-locked staging owned by the batch; wocr_wait waits once and
// copies the staged results to the callers' buffers.
struct wocr_batch {
    wocr_ctx *ctx = nullptr;
    struct Chunk {
        uint8_t *p = nullptr;
        size_t bytes = 0;
    };
    std::vector<Chunk> chunks;  // staging, kept for reuse across waits
    size_t cur = 0, off = 0;
    struct Out {
        void *dst;
        const uint8_t *src;
        size_t bytes;
    };
    std::vector<Out> outs;
    int64_t recorded = 0;
    ~wocr_batch() {
        for (auto &ch : chunks) cudaFreeHost(ch.p);
    }
};

static uint8_t *batch_stage(wocr_batch *b, size_t bytes) {
    bytes = (bytes + 255) / 256 * 256;
    while (b->cur < b->chunks.size() && b->off + bytes > b->chunks[b->cur].bytes) {
        b->cur++;
        b->off = 0;
    }
    if (b->cur == b->chunks.size()) {
        const size_t sz = std::max<size_t>(bytes, (size_t)4 << 20);
        void *p = nullptr;
        WOCR_CUDA(cudaHostAlloc(&p, sz, cudaHostAllocPortable));
        b->chunks.push_back({(uint8_t *)p, sz});
        b->off = 0;
    }
    uint8_t *p = b->chunks[b->cur].p + b->off;
    b->off += bytes;
    return p;
}

// A reader for the cores above that stages into `b`.
struct BatchRead {
    wocr_batch *b;
    Ctx *c;
    void operator()(void *dst, const void *src, size_t bytes) const {
        if (!dst || !bytes) return;
        uint8_t *s = batch_stage(b, bytes);
        WOCR_CUDA(cudaMemcpyAsync(s, src, bytes, cudaMemcpyDeviceToHost, c->stream));
        b->outs.push_back({dst, s, bytes});
    }
};

// Waits for everything recorded in `b` (bounded) and hands the staged results to their buffers.
static void batch_wait(wocr_batch *b, int timeout_ms) {
    Ctx *c = &b->ctx->c;
    WOCR_CUDA(cudaSetDevice(c->device));
    try {
        sync_bounded(c, timeout_ms);
    } catch (const Error &e) {
        // a wait that ran out while the stream still works keeps the reads pending (a later
        // wocr_wait may finish them); any other failure drops them
        if (!(e.code == WOCR_ERR_TIMEOUT && cudaStreamQuery(c->stream) == cudaErrorNotReady)) {
            b->outs.clear();
            b->cur = b->off = 0;
            b->recorded = 0;
        }
        throw;
    }
    for (const auto &o : b->outs) std::memcpy(o.dst, o.src, o.bytes);
    b->outs.clear();
    b->cur = b->off = 0;
    b->recorded = 0;
}

extern "C" {

int32_t wocr_ndgraph_run(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank, float *out,
                         int64_t out_cap, int64_t *out_shape, int32_t *out_rank) {
    return guard([&] {
        if (!g) fail(WOCR_ERR_INVALID, "null graph");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        nd_run_core(g, x, shape, rank, out, out_cap, out_shape, out_rank,
                    [&](void *dst, const void *src, size_t bytes) { d2h(c, dst, src, bytes); });
        sync_bounded(c, 0);
    });
}

int32_t wocr_ndgraph_run_argmax(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank, uint32_t *best,
                                float *row_max, float *row_lse, int64_t cap, int64_t *rows_out, int64_t *out_shape,
                                int32_t *out_rank) {
    return guard([&] {
        if (!g) fail(WOCR_ERR_INVALID, "null graph");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        nd_argmax_core(g, x, shape, rank, best, row_max, row_lse, cap, rows_out, out_shape, out_rank,
                       [&](void *dst, const void *src, size_t bytes) {
                           if (dst) d2h(c, dst, src, bytes);
                       });
        sync_bounded(c, 0);
    });
}

int32_t wocr_batch_create(wocr_ctx *ctx, wocr_batch **out) {
    return guard([&] {
        if (!ctx || !out) fail(WOCR_ERR_INVALID, "null argument");
        auto *b = new wocr_batch();
        b->ctx = ctx;
        ctx->refs++;
        *out = b;
    });
}

void wocr_batch_destroy(wocr_batch *b) {
    if (!b) return;
    wocr_ctx *ctx = b->ctx;
    cudaSetDevice(ctx->c.device);
    cudaStreamSynchronize(ctx->c.stream);  // no staged copy may still be writing
    delete b;
    ctx_release(ctx);
}

int64_t wocr_batch_pending(wocr_batch *b) { return b ? b->recorded : -1; }

int32_t wocr_ndgraph_run_enqueue(wocr_ndgraph *g, wocr_batch *b, const float *x, const int64_t *shape, int32_t rank,
                                 float *out, int64_t out_cap, int64_t *out_shape, int32_t *out_rank) {
    return guard([&] {
        if (!g || !b) fail(WOCR_ERR_INVALID, "null graph or batch");
        if (b->ctx != g->ctx) fail(WOCR_ERR_INVALID, "the batch belongs to another context");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        nd_run_core(g, x, shape, rank, out, out_cap, out_shape, out_rank, BatchRead{b, c});
        b->recorded++;
    });
}

int32_t wocr_ndgraph_argmax_enqueue(wocr_ndgraph *g, wocr_batch *b, const float *x, const int64_t *shape,
                                    int32_t rank, uint32_t *best, float *row_max, float *row_lse, int64_t cap,
                                    int64_t *rows_out, int64_t *out_shape, int32_t *out_rank) {
    return guard([&] {
        if (!g || !b) fail(WOCR_ERR_INVALID, "null graph or batch");
        if (b->ctx != g->ctx) fail(WOCR_ERR_INVALID, "the batch belongs to another context");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        nd_argmax_core(g, x, shape, rank, best, row_max, row_lse, cap, rows_out, out_shape, out_rank,
                       BatchRead{b, c});
        b->recorded++;
    });
}

int32_t wocr_wait(wocr_batch *b, int32_t timeout_ms) {
    return guard([&] {
        if (!b) fail(WOCR_ERR_INVALID, "null batch");
        batch_wait(b, timeout_ms);
    });
}

static void det_input_sizes(int w, int h, int max_side, int *ow, int *oh) {
    float ratio = std::max(w, h) > max_side ? (float)max_side / (float)std::max(w, h) : 1.0f;
    auto rnd = [](float v) { return std::max((int)std::round(v / 32.0f) * 32, 32); };
    *ow = rnd((float)w * ratio);
    *oh = rnd((float)h * ratio);
}

int32_t wocr_det_input(wocr_ctx *ctx, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side, float *out,
                       int64_t out_cap, int32_t *ow_out, int32_t *oh_out, float *to_page) {
    return guard([&] {
        if (!ctx || !rgb || w <= 0 || h <= 0 || max_side <= 0) fail(WOCR_ERR_INVALID, "bad argument");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        int ow, oh;
        det_input_sizes(w, h, max_side, &ow, &oh);
        if (ow_out) *ow_out = ow;
        if (oh_out) *oh_out = oh;
        if (to_page) {
            to_page[0] = (float)w / (float)ow;
            to_page[1] = (float)h / (float)oh;
        }
        if (!out) return;
        if (out_cap < (int64_t)3 * ow * oh) fail(WOCR_ERR_CAPACITY, "det_input buffer too small");
        BufP src = alloc(c, (size_t)w * h * 3);
        WOCR_CUDA(cudaMemcpyAsync(src->p, rgb, (size_t)w * h * 3, cudaMemcpyHostToDevice, c->stream));
        DT y = new_rowmajor(c, {1, 3, oh, ow});
        k::det_prep(c, (const uint8_t *)src->p, w, h, ow, oh, 1, y.p);
        d2h(c, out, y.p, (size_t)y.numel() * 4);
        sync_bounded(c, 0);
    });
}

int32_t wocr_ppdet_page(wocr_ndgraph *g, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side, float *prob,
                        int64_t prob_cap, int32_t *ow_out, int32_t *oh_out, float *to_page) {
    return guard([&] {
        if (!g || !rgb || w <= 0 || h <= 0 || max_side <= 0) fail(WOCR_ERR_INVALID, "bad argument");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        int ow, oh;
        det_input_sizes(w, h, max_side, &ow, &oh);
        if (ow_out) *ow_out = ow;
        if (oh_out) *oh_out = oh;
        g->map_to_page[0] = (float)w / (float)ow;
        g->map_to_page[1] = (float)h / (float)oh;
        if (to_page) {
            to_page[0] = (float)w / (float)ow;
            to_page[1] = (float)h / (float)oh;
        }
        // replayed from a CUDA graph after the first call of a page size (mode 2 of the cache)
        bool first = false;
        NdReplay *r = nd_replay(g, {h, w, 3, max_side}, 2, &first);
        if (!r || first) {
            BufP src = alloc(c, (size_t)w * h * 3);
            WOCR_CUDA(cudaMemcpyAsync(src->p, rgb, (size_t)w * h * 3, cudaMemcpyDefault, c->stream));
            DT x = new_nhwc(c, 1, 3, oh, ow);
            k::det_prep(c, (const uint8_t *)src->p, w, h, ow, oh, 0, x.p);
            DT y = to_rowmajor(c, g->graph->run(x));
            if (r) r->out_shape = y.shape;
            g->map_buf = y.buf;
            g->map = y.p;
            g->map_w = (int)y.shape.back();
            g->map_h = (int)(y.numel() / std::max<int64_t>(y.shape.back(), 1));
            if (prob) {
                if (prob_cap < y.numel()) fail(WOCR_ERR_CAPACITY, "probability buffer too small");
                d2h(c, prob, y.p, (size_t)y.numel() * 4);
            }
            sync_bounded(c, 0);
            return;
        }
        int64_t m = 1;
        for (auto d : r->out_shape) m *= d;
        if (!r->exec) {
            r->in = alloc(c, (size_t)w * h * 3);
            r->out = alloc(c, (size_t)std::max<int64_t>(m, 1) * 4);
            const double f0 = c->flops;
            const int64_t l0 = c->launches;
            WOCR_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
            try {
                DT x = new_nhwc(c, 1, 3, oh, ow);
                k::det_prep(c, (const uint8_t *)r->in->p, w, h, ow, oh, 0, x.p);
                DT y = to_rowmajor(c, g->graph->run(x));
                if (y.shape != r->out_shape) fail(WOCR_ERR_SHAPE, "NdGraph output shape changed between runs");
                WOCR_CUDA(cudaMemcpyAsync(r->out->p, y.p, (size_t)m * 4, cudaMemcpyDeviceToDevice, c->stream));
            } catch (...) {
                cudaGraph_t dead = nullptr;
                cudaStreamEndCapture(c->stream, &dead);
                if (dead) cudaGraphDestroy(dead);
                r->reset();
                throw;
            }
            WOCR_CUDA(cudaStreamEndCapture(c->stream, &r->graph));
            WOCR_CUDA(cudaGraphInstantiate(&r->exec, r->graph, 0));
            r->flops = c->flops - f0;
            r->launches = c->launches - l0;
            c->flops = f0;
            c->launches = l0;
        }
        nd_replay_launch(g, r, reinterpret_cast<const float *>(rgb));
        g->map_buf = r->out;
        g->map = (const float *)r->out->p;
        g->map_w = (int)r->out_shape.back();
        g->map_h = (int)(m / std::max<int64_t>(r->out_shape.back(), 1));
        if (prob) {
            if (prob_cap < m) fail(WOCR_ERR_CAPACITY, "probability buffer too small");
            d2h(c, prob, r->out->p, (size_t)m * 4);
        }
        sync_bounded(c, 0);
    });
}

int32_t wocr_ppdet_mask(wocr_ndgraph *g, float thresh, uint32_t *mask, int64_t cap, int32_t *ow, int32_t *oh) {
    return guard([&] {
        if (!g) fail(WOCR_ERR_INVALID, "null argument");
        if (!g->map) fail(WOCR_ERR_INVALID, "no probability map: call wocr_ppdet_page first");
        const int w = g->map_w, h = g->map_h, words = (w + 31) / 32;
        if (ow) *ow = w;
        if (oh) *oh = h;
        if (!mask && cap == 0) return;  // size query
        if (!mask) fail(WOCR_ERR_INVALID, "null argument");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        if (cap < (int64_t)words * h) fail(WOCR_ERR_CAPACITY, "mask buffer too small");
        BufP bits = alloc(c, (size_t)words * h * 4);
        k::db_mask(c, g->map, w, h, thresh, (uint32_t *)bits->p);
        d2h(c, mask, bits->p, (size_t)words * h * 4);
        g->last.d2h += (int64_t)words * h * 4;
        sync_bounded(c, 0);
    });
}

namespace {

// The score boxes of rects [n][6] on a w x h map: the scan rectangle is the box's bounding
// rectangle (its four corners), floor / ceil, clamped to the map as score() clamps it.
std::vector<k::DbBox> db_make_boxes(const float *rects, int n, int w, int h) {
    std::vector<k::DbBox> bx((size_t)n);
    for (int i = 0; i < n; i++) {
        const float *r = rects + 6 * (size_t)i;
        k::DbBox &b = bx[i];
        b.cx = r[0];
        b.cy = r[1];
        b.ux = r[2];
        b.uy = r[3];
        b.hw = r[4] / 2.0f;
        b.hh = r[5] / 2.0f;
        float lo_x = INFINITY, hi_x = -INFINITY, lo_y = INFINITY, hi_y = -INFINITY;
        for (int sa = -1; sa <= 1; sa += 2)
            for (int sb = -1; sb <= 1; sb += 2) {
                const float px = b.cx + sa * b.hh * b.ux + sb * b.hw * -b.uy;
                const float py = b.cy + sa * b.hh * b.uy + sb * b.hw * b.ux;
                lo_x = std::min(lo_x, px), hi_x = std::max(hi_x, px);
                lo_y = std::min(lo_y, py), hi_y = std::max(hi_y, py);
            }
        // one pixel wider on every side than floor / ceil of the corners: the pixels that pass
        // the inside test lie in the box's bounding rectangle whatever the corner rounding
        // `as usize`: saturating, NaN to 0
        auto to_idx = [](float v) -> int64_t { return v > 0.f ? (v < 4e9f ? (int64_t)v : (int64_t)4e9) : 0; };
        b.x0 = (int)std::min<int64_t>(to_idx(std::floor(lo_x) - 1.f), w);
        b.y0 = (int)std::min<int64_t>(to_idx(std::floor(lo_y) - 1.f), h);
        b.x1 = (int)std::min<int64_t>(to_idx(std::ceil(hi_x) + 1.f), std::max(w - 1, 0));
        b.y1 = (int)std::min<int64_t>(to_idx(std::ceil(hi_y) + 1.f), std::max(h - 1, 0));
        b.map = 0;
    }
    return bx;
}

// `score` (src/ppdet.rs:63-83) of rects [n][6] on the device map prob (w x h), into host scores.
void db_score_boxes(Ctx *c, const float *prob, int w, int h, const float *rects, int n, float *scores) {
    if (n == 0) return;
    const std::vector<k::DbBox> bx = db_make_boxes(rects, n, w, h);
    BufP db = alloc(c, bx.size() * sizeof(k::DbBox)), ds = alloc(c, (size_t)n * 4);
    WOCR_CUDA(cudaMemcpyAsync(db->p, bx.data(), bx.size() * sizeof(k::DbBox), cudaMemcpyHostToDevice, c->stream));
    k::db_scores(c, prob, w, h, (const k::DbBox *)db->p, n, (float *)ds->p);
    d2h(c, scores, ds->p, (size_t)n * 4);
    sync_bounded(c, 0);
}

// A box's left and top (the minimum of its four corners) for the reading-order sort.
void db_bounds(const float *r, float *left, float *top) {
    const float hw = r[4] / 2.0f, hh = r[5] / 2.0f;
    float lx = INFINITY, ty = INFINITY;
    for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
            const float px = r[0] + sa * hh * r[2] + sb * hw * -r[3];
            const float py = r[1] + sa * hh * r[3] + sb * hw * r[2];
            lx = px < lx ? px : lx;
            ty = py < ty ? py : ty;
        }
    *left = lx;
    *top = ty;
}

// `ppdet::boxes` (src/ppdet.rs:87-132) on n device maps of one size, stacked [n][h][w]: the
// p > thresh masks, their external contours' minimum-area rectangles (simplified, epsilon 2) and
// the box scores on the device, every page in the same launches; the size checks, unclip, page
// scaling and reading order on the host, page by page, as the reference orders them.
std::vector<std::vector<float>> db_boxes_pages(Ctx *c, const float *maps, int npages, int w, int h,
                                               const float *to_page, float thresh, float box_thresh,
                                               float unclip_ratio, float min_size) {
    const int words = (w + 31) / 32;
    const int64_t plane = (int64_t)w * h;
    BufP bits = alloc(c, (size_t)words * h * npages * 4);
    // the stacked maps threshold as one tall map: rows are independent
    k::db_mask(c, maps, w, h * npages, thresh, (uint32_t *)bits->p);
    k::WordRects wr = k::word_rects(c, (const uint32_t *)bits->p, npages, w, h, 0.f, 0.f, -INFINITY);
    std::vector<float> rs((size_t)wr.n * 6);
    std::vector<int32_t> counts((size_t)npages);
    d2h(c, rs.data(), wr.rects->p, rs.size() * 4);
    d2h(c, counts.data(), wr.page_count->p, counts.size() * 4);
    sync_bounded(c, 0);
    std::vector<float> cand;
    std::vector<int> cand_page;
    {
        size_t r0 = 0;
        for (int q = 0; q < npages; q++) {
            for (int i = 0; i < counts[q]; i++) {
                const float *r = rs.data() + 6 * (r0 + (size_t)i);
                if (std::min(r[4], r[5]) >= min_size) {
                    cand.insert(cand.end(), r, r + 6);
                    cand_page.push_back(q);
                }
            }
            r0 += (size_t)counts[q];
        }
    }
    const int nc = (int)(cand.size() / 6);
    // `score < box_thresh` per candidate.  The ordered f32 sum S of a box's n inside values lies
    // within gamma(n - 1) * sum |v| of their exact sum (gamma(k) = k u / (1 - k u), u = 2^-24),
    // and the division by n adds a rounding; an order-free pass (sum in double) settles every box
    // whose mean is clear of box_thresh by that margin, and only the rest get the ordered score.
    std::vector<char> below((size_t)nc, 0);
    if (nc > 0) {
        std::vector<k::DbBox> bx = db_make_boxes(cand.data(), nc, w, h);
        for (int i = 0; i < nc; i++) bx[i].map = plane * cand_page[i];
        BufP db = alloc(c, bx.size() * sizeof(k::DbBox)), dsum = alloc(c, (size_t)nc * 16),
             dcnt = alloc(c, (size_t)nc * 8);
        WOCR_CUDA(cudaMemcpyAsync(db->p, bx.data(), bx.size() * sizeof(k::DbBox), cudaMemcpyHostToDevice, c->stream));
        int max_rows = 1;
        for (const k::DbBox &b : bx) max_rows = std::max(max_rows, b.y1 - b.y0 + 1);
        k::db_bounds(c, maps, w, (const k::DbBox *)db->p, nc, max_rows, (double *)dsum->p, (long long *)dcnt->p);
        std::vector<double> sums((size_t)nc * 2);
        std::vector<long long> cnts((size_t)nc);
        d2h(c, sums.data(), dsum->p, sums.size() * 8);
        d2h(c, cnts.data(), dcnt->p, cnts.size() * 8);
        sync_bounded(c, 0);
        std::vector<k::DbBox> amb;
        std::vector<int> amb_idx;
        const double u = std::ldexp(1.0, -24);
        for (int i = 0; i < nc; i++) {
            const long long n = cnts[i];
            if (n == 0) {  // no pixel inside: the score is 0
                below[i] = 0.f < box_thresh;
                continue;
            }
            const double S = sums[2 * (size_t)i], A = sums[2 * (size_t)i + 1], ku = (double)(n - 1) * u;
            bool settled = std::isfinite(S) && std::isfinite(A) && ku < 0.25;
            if (settled) {
                // f32 ordering error, plus the double pass's own (far below it), doubled for safety
                const double err = 2.0 * (ku / (1.0 - ku) + (double)n * std::ldexp(1.0, -52)) * A;
                double lo = (S - err) / (double)n, hi = (S + err) / (double)n;
                lo -= std::fabs(lo) * 4.0 * u;  // the f32 division (and n's conversion past 2^24)
                hi += std::fabs(hi) * 4.0 * u;
                if (hi < (double)box_thresh)
                    below[i] = 1;
                else if (lo >= (double)box_thresh)
                    below[i] = 0;
                else
                    settled = false;
            }
            if (!settled) {
                amb.push_back(bx[i]);
                amb_idx.push_back(i);
            }
        }
        if (!amb_idx.empty()) {
            const int na = (int)amb.size();
            BufP da = alloc(c, amb.size() * sizeof(k::DbBox)), ds = alloc(c, (size_t)na * 4);
            WOCR_CUDA(cudaMemcpyAsync(da->p, amb.data(), amb.size() * sizeof(k::DbBox), cudaMemcpyHostToDevice,
                                      c->stream));
            k::db_scores(c, maps, w, h, (const k::DbBox *)da->p, na, (float *)ds->p);
            std::vector<float> sc((size_t)na);
            d2h(c, sc.data(), ds->p, (size_t)na * 4);
            sync_bounded(c, 0);
            for (size_t j = 0; j < amb_idx.size(); j++) below[amb_idx[j]] = sc[j] < box_thresh;
        }
    }
    std::vector<std::vector<float>> pages((size_t)npages);
    std::vector<std::vector<float>> outs((size_t)npages);
    const float s = (to_page[0] + to_page[1]) / 2.0f;
    for (int i = 0; i < nc; i++) {
        const float *r = cand.data() + 6 * (size_t)i;
        if (below[i]) continue;
        const float rw = r[4], rh = r[5];
        const float per = 2.0f * (rw + rh);
        const float d = rw * rh * unclip_ratio / (per > 1e-6f ? per : 1e-6f);
        const float nw = rw + 2.0f * d, nh = rh + 2.0f * d;
        if (std::min(nw, nh) < min_size + 2.0f) continue;
        const float o[6] = {r[0] * to_page[0], r[1] * to_page[1], r[2], r[3], nw * s, nh * s};
        outs[cand_page[i]].insert(outs[cand_page[i]].end(), o, o + 6);
    }
    for (int q = 0; q < npages; q++) {
        const std::vector<float> &out = outs[q];
        // stable by the top of the bounding rectangle, then boxes whose tops are within 10 px of
        // their predecessor's by the left edge (one insertion pass)
        const int n = (int)(out.size() / 6);
        std::vector<int> idx((size_t)n);
        std::vector<float> top((size_t)n), left((size_t)n);
        for (int i = 0; i < n; i++) {
            idx[i] = i;
            db_bounds(out.data() + 6 * (size_t)i, &left[i], &top[i]);
        }
        std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return top[a] < top[b]; });
        for (int i = 0; i < n; i++)
            for (int j = i; j > 0; j--) {
                const int a = idx[j - 1], b = idx[j];
                if (std::fabs(top[b] - top[a]) < 10.0f && left[b] < left[a])
                    std::swap(idx[j - 1], idx[j]);
                else
                    break;
            }
        std::vector<float> &sorted = pages[q];
        sorted.resize(out.size());
        for (int i = 0; i < n; i++)
            std::memcpy(sorted.data() + 6 * (size_t)i, out.data() + 6 * (size_t)idx[i], 24);
    }
    return pages;
}

std::vector<float> db_boxes(Ctx *c, const float *prob, int w, int h, const float *to_page, float thresh,
                            float box_thresh, float unclip_ratio, float min_size) {
    return db_boxes_pages(c, prob, 1, w, h, to_page, thresh, box_thresh, unclip_ratio, min_size)[0];
}

void put_boxes(const std::vector<float> &b, float *boxes, int32_t cap, int32_t *n) {
    const int nb = (int)(b.size() / 6);
    *n = nb;
    if (!boxes && cap == 0) return;
    if (cap < nb) fail(WOCR_ERR_CAPACITY, "boxes holds " + std::to_string(cap) + " of " + std::to_string(nb));
    if (nb) std::memcpy(boxes, b.data(), b.size() * 4);
}

}  // namespace

int32_t wocr_ppdet_scores(wocr_ndgraph *g, const float *rects, int32_t n, float *scores) {
    return guard([&] {
        if (!g || (n > 0 && (!rects || !scores)) || n < 0) fail(WOCR_ERR_INVALID, "bad argument");
        if (!g->map) fail(WOCR_ERR_INVALID, "no probability map: call wocr_ppdet_page first");
        if (n == 0) return;
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        db_score_boxes(c, g->map, g->map_w, g->map_h, rects, n, scores);
    });
}

int32_t wocr_ppdet_boxes(wocr_ndgraph *g, float thresh, float box_thresh, float unclip_ratio, float min_size,
                         float *boxes, int32_t cap, int32_t *n) {
    return guard([&] {
        if (!g || !n || cap < 0 || (cap > 0 && !boxes)) fail(WOCR_ERR_INVALID, "bad argument");
        if (!g->map) fail(WOCR_ERR_INVALID, "no probability map: call wocr_ppdet_page first");
        Ctx *c = &g->ctx->c;
        RunScope rs(c, &g->last);
        put_boxes(db_boxes(c, g->map, g->map_w, g->map_h, g->map_to_page, thresh, box_thresh, unclip_ratio, min_size),
                  boxes, cap, n);
    });
}

int32_t wocr_db_boxes(wocr_ctx *ctx, const float *prob, int32_t w, int32_t h, int32_t prob_on_device,
                      const float *to_page, float thresh, float box_thresh, float unclip_ratio, float min_size,
                      float *boxes, int32_t cap, int32_t *n) {
    return guard([&] {
        if (!ctx || !prob || !to_page || !n || cap < 0 || (cap > 0 && !boxes)) fail(WOCR_ERR_INVALID, "bad argument");
        if (w <= 0 || h <= 0 || w > 32767 || h > 32767) fail(WOCR_ERR_INVALID, "bad map size");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        const float *dp = prob;
        BufP up;
        if (!prob_on_device) {
            up = alloc(c, (size_t)w * h * 4);
            WOCR_CUDA(cudaMemcpyAsync(up->p, prob, (size_t)w * h * 4, cudaMemcpyHostToDevice, c->stream));
            dp = (const float *)up->p;
        }
        put_boxes(db_boxes(c, dp, w, h, to_page, thresh, box_thresh, unclip_ratio, min_size), boxes, cap, n);
    });
}

int32_t wocr_word_rects(wocr_ctx *ctx, const uint32_t *mask, int32_t n, int32_t w, int32_t h,
                        int32_t mask_on_device, float expand, float expand_x, float min_area, float *rects,
                        int64_t cap, int32_t *counts) {
    return guard([&] {
        if (!ctx || !mask || !counts || (cap > 0 && !rects)) fail(WOCR_ERR_INVALID, "null argument");
        if (n < 0 || w <= 0 || h <= 0 || cap < 0) fail(WOCR_ERR_INVALID, "bad page count or size");
        if (w > 32767 || h > 32767) fail(WOCR_ERR_INVALID, "pages wider or taller than 32767 pixels");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        const int64_t words = (w + 31) / 32, page_words = words * h;
        // page groups small enough for 32-bit run and point counts
        const int group = (int)std::max<int64_t>(1, ((int64_t)1 << 28) / ((int64_t)w * h));
        int64_t total = 0;
        std::vector<float> host;
        for (int p0 = 0; p0 < n; p0 += group) {
            const int pn = std::min(group, n - p0);
            const uint32_t *dm = mask + p0 * page_words;
            BufP up;
            if (!mask_on_device) {
                up = alloc(c, (size_t)(pn * page_words * 4));
                WOCR_CUDA(cudaMemcpyAsync(up->p, dm, (size_t)(pn * page_words * 4), cudaMemcpyHostToDevice, c->stream));
                dm = (const uint32_t *)up->p;
            }
            k::WordRects wr = k::word_rects(c, dm, pn, w, h, expand, expand_x, min_area);
            d2h(c, counts + p0, wr.page_count->p, (size_t)pn * 4);
            const size_t o = host.size();
            host.resize(o + (size_t)wr.n * 6);
            d2h(c, host.data() + o, wr.rects->p, (size_t)wr.n * 24);
            sync_bounded(c, 0);
            total += wr.n;
        }
        if (!rects && cap == 0) return;
        if (cap < total) fail(WOCR_ERR_CAPACITY, "rects holds " + std::to_string(cap) + " of " + std::to_string(total));
        if (total) std::memcpy(rects, host.data(), (size_t)total * 24);
    });
}

int32_t wocr_pp_lines(wocr_ctx *ctx, const uint8_t *d_rgb, int32_t w, int32_t h, const float *rects, int32_t n,
                      int32_t per_batch, float *d_out, int64_t cap, int32_t *order, int32_t *batch_n,
                      int32_t *batch_w, int32_t *n_batches, int64_t *total) {
    return guard([&] {
        if (!ctx || (n > 0 && !rects)) fail(WOCR_ERR_INVALID, "null argument");
        if (n < 0 || w <= 0 || h <= 0 || per_batch <= 0) fail(WOCR_ERR_INVALID, "bad page size, line count or batch");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        // each box as ppocr::line_input clamps and sizes it
        auto clampb = [](float v, int hi) -> int {
            if (!(v > 0.f)) v = 0.f;  // f32::max ignores NaN
            if (v > (float)hi) v = (float)hi;
            return (int)(unsigned)v;
        };
        std::vector<k::PpLine> ln((size_t)n);
        for (int i = 0; i < n; i++) {
            const float *r = rects + 4 * (size_t)i;
            const int l = clampb(r[0], w), t = clampb(r[1], h), rr = clampb(r[2], w), b = clampb(r[3], h);
            k::PpLine &L = ln[i];
            L.l = l;
            L.t = t;
            L.cw = std::max(rr - l, 1);
            L.ch = std::max(b - t, 1);
            volatile float q = 48.f * (float)L.cw;  // rounded before the division, as the oracle
            const float fw = std::ceil(q / (float)L.ch);
            L.ow = fw < 8.f ? 8 : (fw > 3200.f ? 3200 : (int)fw);
        }
        // sorted by width (stable), cut into batches of per_batch, widths rounded up to 8
        std::vector<int> idx((size_t)n);
        for (int i = 0; i < n; i++) idx[i] = i;
        std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return ln[a].ow < ln[b].ow; });
        std::vector<k::PpLine> plan((size_t)n);
        int64_t off = 0;
        int nb = 0;
        for (int k0 = 0; k0 < n; k0 += per_batch, nb++) {
            const int kn = std::min(per_batch, n - k0);
            int width = 0;
            for (int j = 0; j < kn; j++) width = std::max(width, ln[idx[k0 + j]].ow);
            width = (width + 7) / 8 * 8;
            for (int j = 0; j < kn; j++) {
                plan[k0 + j] = ln[idx[k0 + j]];
                plan[k0 + j].width = width;
                plan[k0 + j].off = off + (int64_t)j * 3 * 48 * width;
                if (order) order[k0 + j] = idx[k0 + j];
            }
            if (batch_n) batch_n[nb] = kn;
            if (batch_w) batch_w[nb] = width;
            off += (int64_t)kn * 3 * 48 * width;
        }
        if (n_batches) *n_batches = nb;
        if (total) *total = off;
        if (!d_out || n == 0) return;
        if (!d_rgb) fail(WOCR_ERR_INVALID, "null page");
        if (cap < off) fail(WOCR_ERR_CAPACITY, "line batches need " + std::to_string(off) + " floats");
        // tall crops (a vertical downscale of 8 or more) go through the two-pass kernels
        std::vector<k::PpLine> normal, tall;
        std::vector<int64_t> toff;
        int64_t tmp_total = 0;
        int max_w_n = 0, max_w_t = 0, max_cw = 0;
        double bytes_n = 0, bytes_t = 0;
        for (const k::PpLine &L : plan) {
            const double b = 3.0 * L.cw * L.ch + 4.0 * 3 * 48 * L.width;
            if (L.ch >= k::kPpTallRows) {
                tall.push_back(L);
                toff.push_back(tmp_total);
                tmp_total += (int64_t)48 * L.cw * 3;
                max_w_t = std::max(max_w_t, L.width);
                max_cw = std::max(max_cw, L.cw);
                bytes_t += b;
            } else {
                normal.push_back(L);
                max_w_n = std::max(max_w_n, L.width);
                bytes_n += b;
            }
        }
        if (!normal.empty()) {
            BufP dl = alloc(c, normal.size() * sizeof(k::PpLine));
            WOCR_CUDA(cudaMemcpyAsync(dl->p, normal.data(), normal.size() * sizeof(k::PpLine), cudaMemcpyHostToDevice,
                                      c->stream));
            k::pp_lines(c, d_rgb, w, h, (const k::PpLine *)dl->p, (int)normal.size(), max_w_n, d_out, bytes_n);
        }
        if (!tall.empty()) {
            BufP dl = alloc(c, tall.size() * sizeof(k::PpLine)), dt = alloc(c, toff.size() * 8);
            BufP tmp = alloc(c, (size_t)tmp_total * 4);
            WOCR_CUDA(cudaMemcpyAsync(dl->p, tall.data(), tall.size() * sizeof(k::PpLine), cudaMemcpyHostToDevice,
                                      c->stream));
            WOCR_CUDA(cudaMemcpyAsync(dt->p, toff.data(), toff.size() * 8, cudaMemcpyHostToDevice, c->stream));
            k::pp_lines_tall(c, d_rgb, w, h, (const k::PpLine *)dl->p, (int)tall.size(), max_cw, max_w_t,
                             (const int64_t *)dt->p, (float *)tmp->p, d_out, bytes_t);
        }
        sync_bounded(c, 0);  // the plan's host copy is read until the upload completes
    });
}

int32_t wocr_last_transfer_bytes(void *handle, int32_t kind, int64_t *h2d, int64_t *d2h) {
    return guard([&] {
        if (!handle) fail(WOCR_ERR_INVALID, "null handle");
        Stats *s = nullptr;
        if (kind == 1) s = &((wocr_detector *)handle)->last;
        else if (kind == 2) s = &((wocr_recognizer *)handle)->last;
        else if (kind == 3) s = &((wocr_ndgraph *)handle)->last;
        else fail(WOCR_ERR_INVALID, "kind must be 1 (detector), 2 (recogniser) or 3 (N-D graph)");
        if (h2d) *h2d = s->h2d;
        if (d2h) *d2h = s->d2h;
    });
}

int32_t wocr_last_run_stats(void *handle, int32_t kind, double *flops, int64_t *launches) {
    return guard([&] {
        if (!handle) fail(WOCR_ERR_INVALID, "null handle");
        Stats *s = nullptr;
        if (kind == 1) s = &((wocr_detector *)handle)->last;
        else if (kind == 2) s = &((wocr_recognizer *)handle)->last;
        else if (kind == 3) s = &((wocr_ndgraph *)handle)->last;
        else fail(WOCR_ERR_INVALID, "kind must be 1 (detector), 2 (recogniser) or 3 (N-D graph)");
        if (flops) *flops = s->flops;
        if (launches) *launches = s->launches;
    });
}

}  // extern "C"

// ---- the PP-OCRv6 page pipeline --------------------------------------------------------------
//
// The reference's bench runs a page in two halves on two threads (src/bin/ocr-bench.rs:133-310,
// 458-585): its GPU thread detects page k + 1 while the CPU turns page k's map into boxes and
// line images; recognition jobs wait until MERGE pages are held and then run every batch in one
// encoder, read with one wait.  Here both halves run on the device, so the overlap is between
// pages on the device: a pipeline owns `lanes` workers on one GPU, each a context (stream, pool,
// graph caches) with its own detector and recogniser graphs and a host thread.  Lane j takes
// pages j, j + lanes, ...; while one lane's page is in its latency-bound steps (the contour of a
// large component, a small recognition batch), the others' kernels fill the SMs.  Each lane holds
// the line batches of `merge` of its pages and recognises them together: every batch queued on
// its stream with its arg-max read staged (wocr_ndgraph_argmax_enqueue), then one wait.
struct PpLane {
    wocr_ctx *ctx = nullptr;
    wocr_ndgraph *det = nullptr, *rec = nullptr;
    wocr_batch *batch = nullptr;
    // two chunk buffers (pages back to back: the detection batch's input): the next chunk's pages
    // go up on the copy stream while the current chunk computes.  up[b]: chunk in b uploaded;
    // freed[b]: the compute stream is done with b (and b's allocation is ordered before reuse)
    BufP page[2];
    size_t page_bytes[2] = {0, 0};
    cudaStream_t copy = nullptr;
    cudaEvent_t up[2] = {nullptr, nullptr}, freed[2] = {nullptr, nullptr};
    BufP maps_tmp;  // the maps of a batch that ran without a captured graph
    ~PpLane() {
        if (ctx) cudaStreamSynchronize(ctx->c.stream);
        if (copy) {
            cudaStreamSynchronize(copy);
            cudaStreamDestroy(copy);
        }
        for (cudaEvent_t e : {up[0], up[1], freed[0], freed[1]})
            if (e) cudaEventDestroy(e);
        if (batch) wocr_batch_destroy(batch);
        if (det) wocr_ndgraph_destroy(det);
        if (rec) wocr_ndgraph_destroy(rec);
        if (ctx) wocr_ctx_destroy(ctx);  // the lane's own reference
    }
};

struct wocr_pp {
    wocr_ctx *ctx = nullptr;  // lane 0's context (the caller's)
    Model det_m, rec_m;       // kept to build further lanes
    std::vector<std::unique_ptr<PpLane>> lanes;
};

namespace {
// a failing inner entry point: its status and message, rethrown
void check_st(int32_t st) {
    if (st != WOCR_OK) fail(st, wocr_last_error());
}

// One page between its two halves: boxes in reading order, the line batches on the device,
// then the arg-max classes of each line.
struct PpPage {
    std::vector<float> boxes;  // [n][6]
    std::vector<int32_t> order, bn, bw;
    int32_t nb = 0;
    BufP lines;                // the batches, one after another, [bn, 3, 48, bw] each
    std::vector<std::vector<uint32_t>> best;  // per line
    int64_t h2d = 0, d2h = 0;
};

struct PpArgs {
    int max_side;
    const float *db;
    float relv;
    int per_batch;
    bool want_rec;
};

bool on_device(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice;
}

// The line rectangles of a page's boxes: each box grown by relv x its height across the text
// (src/bin/ocr-bench.rs:534-558: a line of one box, whose median height is its own), then its
// bounding rectangle [left, top, right, bottom].
std::vector<float> pp_line_rects(const std::vector<float> &boxes, float relv) {
    const int n = (int)(boxes.size() / 6);
    std::vector<float> lr((size_t)n * 4);
    for (int i = 0; i < n; i++) {
        const float *r = boxes.data() + 6 * (size_t)i;
        const bool upright = std::fabs(r[3]) >= std::fabs(r[2]);
        const float across = relv * (upright ? r[5] : r[4]);
        const float rw = upright ? r[4] : r[4] + 2.f * across, rh = upright ? r[5] + 2.f * across : r[5];
        const float hw = rw / 2.0f, hh = rh / 2.0f;
        float lx = INFINITY, ty = INFINITY, rx = -INFINITY, by = -INFINITY;
        for (int sa = -1; sa <= 1; sa += 2)
            for (int sb = -1; sb <= 1; sb += 2) {
                const float px = r[0] + sa * hh * r[2] + sb * hw * -r[3];
                const float py = r[1] + sa * hh * r[3] + sb * hw * r[2];
                lx = std::min(lx, px), rx = std::max(rx, px);
                ty = std::min(ty, py), by = std::max(by, py);
            }
        float *o = lr.data() + 4 * (size_t)i;
        o[0] = lx;
        o[1] = ty;
        o[2] = rx;
        o[3] = by;
    }
    return lr;
}

// NdGraph::det_input + the DB detector on n device pages of one size, back to back at d_pages,
// in one batch [n, 3, oh, ow] (each image's results are those of a batch of one: every kernel
// computes an image's outputs from that image alone, in the same order).  Replayed from a CUDA
// graph per (n, size, input buffer) after the first call.  Returns the maps [n][mh][mw].
const float *ppdet_batch(PpLane &ln, const uint8_t *d_pages, int n, int w, int h, int max_side, int *mw, int *mh) {
    wocr_ndgraph *g = ln.det;
    Ctx *c = &g->ctx->c;
    RunScope rs(c, &g->last);
    int ow, oh;
    det_input_sizes(w, h, max_side, &ow, &oh);
    const size_t page_bytes = (size_t)w * h * 3;
    auto pass = [&]() {
        DT x = new_nhwc(c, n, 3, oh, ow);
        for (int q = 0; q < n; q++)
            k::det_prep(c, d_pages + page_bytes * q, w, h, ow, oh, 0, x.p + (int64_t)q * oh * ow * 3);
        return to_rowmajor(c, g->graph->run(x));
    };
    auto dims = [&](const std::vector<int64_t> &shape) {
        int64_t m = 1;
        for (auto d : shape) m *= d;
        *mw = (int)shape.back();
        *mh = (int)(m / std::max<int64_t>((int64_t)n * shape.back(), 1));
        return m;
    };
    bool first = false;
    NdReplay *r = nd_replay(g, {n, h, w, max_side, (int64_t)(intptr_t)d_pages}, 3, &first);
    if (!r || first) {
        DT y = pass();
        if (r) r->out_shape = y.shape;
        dims(y.shape);
        ln.maps_tmp = y.buf;
        return y.p;
    }
    const int64_t m = dims(r->out_shape);
    if (!r->exec) {
        r->out = alloc(c, (size_t)std::max<int64_t>(m, 1) * 4);
        const double f0 = c->flops;
        const int64_t l0 = c->launches;
        WOCR_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
        try {
            DT y = pass();
            if (y.shape != r->out_shape) fail(WOCR_ERR_SHAPE, "NdGraph output shape changed between runs");
            WOCR_CUDA(cudaMemcpyAsync(r->out->p, y.p, (size_t)m * 4, cudaMemcpyDeviceToDevice, c->stream));
        } catch (...) {
            cudaGraph_t dead = nullptr;
            cudaStreamEndCapture(c->stream, &dead);
            if (dead) cudaGraphDestroy(dead);
            r->reset();
            throw;
        }
        WOCR_CUDA(cudaStreamEndCapture(c->stream, &r->graph));
        WOCR_CUDA(cudaGraphInstantiate(&r->exec, r->graph, 0));
        r->flops = c->flops - f0;
        r->launches = c->launches - l0;
        c->flops = f0;
        c->launches = l0;
    }
    WOCR_CUDA(cudaGraphLaunch(r->exec, c->stream));
    c->flops += r->flops;
    c->launches += r->launches;
    return (const float *)r->out->p;
}

// The first half of a chunk of pages of one size: the pages gathered on the device (uploads
// for host pages), their detection in one batch, the DB boxes of all their maps in the same
// launches, each page's line cuts.
// The pages of a chunk into chunk buffer b on the lane's copy stream (after the compute stream is
// done with b); up[b] marks their arrival.
void pp_upload_chunk(PpLane &ln, int b, const uint8_t *const *pages, const std::vector<int> &ks, int w, int h,
                     std::vector<PpPage> &out) {
    Ctx *c = &ln.ctx->c;
    const int n = (int)ks.size();
    const size_t bytes = (size_t)w * h * 3;
    if (ln.page_bytes[b] < bytes * n) {
        ln.page[b] = alloc(c, bytes * n);
        ln.page_bytes[b] = bytes * n;
    }
    WOCR_CUDA(cudaEventRecord(ln.freed[b], c->stream));
    WOCR_CUDA(cudaStreamWaitEvent(ln.copy, ln.freed[b], 0));
    uint8_t *dp = (uint8_t *)ln.page[b]->p;
    for (int q = 0; q < n; q++) {
        const uint8_t *src = pages[ks[q]];
        const bool dev = on_device(src);
        WOCR_CUDA(cudaMemcpyAsync(dp + bytes * q, src, bytes, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                  ln.copy));
        if (!dev) out[ks[q]].h2d += (int64_t)bytes;
    }
    WOCR_CUDA(cudaEventRecord(ln.up[b], ln.copy));
}

void pp_front_chunk(PpLane &ln, int buf, const std::vector<int> &ks, int w, int h, const PpArgs &a,
                    std::vector<PpPage> &out) {
    Ctx *c = &ln.ctx->c;
    WOCR_CUDA(cudaSetDevice(c->device));
    const int n = (int)ks.size();
    const size_t bytes = (size_t)w * h * 3;
    WOCR_CUDA(cudaStreamWaitEvent(c->stream, ln.up[buf], 0));
    const uint8_t *dp = (const uint8_t *)ln.page[buf]->p;
    int mw = 0, mh = 0, ow = 0, oh = 0;
    const float *maps = ppdet_batch(ln, dp, n, w, h, a.max_side, &mw, &mh);
    det_input_sizes(w, h, a.max_side, &ow, &oh);
    const float tp[2] = {(float)w / (float)ow, (float)h / (float)oh};
    std::vector<std::vector<float>> bx = db_boxes_pages(c, maps, n, mw, mh, tp, a.db[0], a.db[1], a.db[2], a.db[3]);
    for (int q = 0; q < n; q++) {
        PpPage &pg = out[ks[q]];
        pg.boxes = std::move(bx[q]);
        const int nb = (int)(pg.boxes.size() / 6);
        if (!a.want_rec || nb == 0) continue;
        const std::vector<float> lr = pp_line_rects(pg.boxes, a.relv);
        const uint8_t *dpage = dp + bytes * q;
        pg.order.assign((size_t)nb, 0);
        pg.bn.assign((size_t)nb, 0);
        pg.bw.assign((size_t)nb, 0);
        int64_t total = 0;
        check_st(wocr_pp_lines(ln.ctx, dpage, w, h, lr.data(), nb, a.per_batch, nullptr, 0, pg.order.data(),
                               pg.bn.data(), pg.bw.data(), &pg.nb, &total));
        pg.lines = alloc(c, (size_t)std::max<int64_t>(total, 1) * 4);
        check_st(wocr_pp_lines(ln.ctx, dpage, w, h, lr.data(), nb, a.per_batch, (float *)pg.lines->p, total,
                               pg.order.data(), pg.bn.data(), pg.bw.data(), &pg.nb, &total));
    }
}

// The second half of the held pages: every batch's recognition and arg-max queued on the lane's
// stream with its read staged, one wait, then the classes handed to their lines.
void pp_recognize(PpLane &ln, const std::vector<PpPage *> &held) {
    // The held pages' batches, grouped by width: batches of one width (of one page or several)
    // run as one batch of all their lines.  A line's recognition depends only on its own image
    // and its batch's width (the padding it is decoded over), not on the other lines of its
    // batch, so the classes are those of the reference's 16-line batches (src/bin/ocr-bench.rs:
    // 322-333), with fewer, larger launches.
    struct Part {
        PpPage *pg;
        int first;   // the batch's first slot in pg->order
        int n;
        int64_t off;  // its float offset in pg->lines
    };
    std::map<int, std::vector<Part>> groups;
    for (PpPage *pg : held) {
        pg->best.assign(pg->boxes.size() / 6, {});
        int k = 0;
        int64_t off = 0;
        for (int b = 0; b < pg->nb; b++) {
            groups[pg->bw[b]].push_back({pg, k, pg->bn[b], off});
            k += pg->bn[b];
            off += (int64_t)pg->bn[b] * 3 * 48 * pg->bw[b];
        }
    }
    if (groups.empty()) return;
    Ctx *c = &ln.ctx->c;
    struct Job {
        const std::vector<Part> *parts;
        int n = 0;
        std::vector<uint32_t> best;
        int64_t rows = 0;
    };
    std::vector<Job> jobs;
    std::vector<BufP> merged;  // kept until the wait: the enqueued runs read them
    for (const auto &g : groups) {
        const int W = g.first;
        Job jb;
        jb.parts = &g.second;
        for (const Part &p : g.second) jb.n += p.n;
        const int64_t line_floats = (int64_t)3 * 48 * W;
        const float *x = nullptr;
        if (g.second.size() == 1) {
            x = (const float *)g.second[0].pg->lines->p + g.second[0].off;
        } else {
            BufP m = alloc(c, (size_t)(jb.n * line_floats) * 4);
            int64_t o = 0;
            for (const Part &p : g.second) {
                WOCR_CUDA(cudaMemcpyAsync((float *)m->p + o, (const float *)p.pg->lines->p + p.off,
                                          (size_t)(p.n * line_floats) * 4, cudaMemcpyDeviceToDevice, c->stream));
                o += p.n * line_floats;
            }
            x = (const float *)m->p;
            merged.push_back(m);
        }
        const int64_t shape[4] = {jb.n, 3, 48, W};
        const int64_t bcap = (int64_t)jb.n * W;
        jb.best.resize((size_t)bcap);
        jobs.push_back(std::move(jb));
        Job &jr = jobs.back();
        int64_t oshape[kMaxRank];
        int32_t orank = 0;
        check_st(wocr_ndgraph_argmax_enqueue(ln.rec, ln.batch, x, shape, 4, jr.best.data(), nullptr, nullptr, bcap,
                                             &jr.rows, oshape, &orank));
    }
    check_st(wocr_wait(ln.batch, 0));
    for (Job &jb : jobs) {
        const int64_t T = jb.rows / std::max(jb.n, 1);
        int64_t line = 0;
        for (const Part &p : *jb.parts) {
            for (int q = 0; q < p.n; q++, line++)
                p.pg->best[p.pg->order[p.first + q]].assign(jb.best.begin() + line * T, jb.best.begin() + (line + 1) * T);
            p.pg->d2h += (int64_t)p.n * T * 4;
        }
    }
}

PpLane *pp_lane(wocr_pp *p, int i) {
    while ((int)p->lanes.size() <= i) {
        auto ln = std::make_unique<PpLane>();
        if (p->lanes.empty()) {
            ln->ctx = p->ctx;
            p->ctx->refs++;
        } else {
            check_st(wocr_ctx_create(p->ctx->c.device, p->ctx->c.lines, &ln->ctx));
        }
        ln->det = ndgraph_from_model(ln->ctx, p->det_m, false);
        ln->rec = ndgraph_from_model(ln->ctx, p->rec_m, true);
        check_st(wocr_batch_create(ln->ctx, &ln->batch));
        WOCR_CUDA(cudaSetDevice(ln->ctx->c.device));
        WOCR_CUDA(cudaStreamCreateWithFlags(&ln->copy, cudaStreamNonBlocking));
        for (int b = 0; b < 2; b++) {
            WOCR_CUDA(cudaEventCreateWithFlags(&ln->up[b], cudaEventDisableTiming));
            WOCR_CUDA(cudaEventCreateWithFlags(&ln->freed[b], cudaEventDisableTiming));
        }
        p->lanes.push_back(std::move(ln));
    }
    return p->lanes[i].get();
}

// Pages [0, n) over `lanes` lanes, recognitions merged `merge` pages at a time per lane.
void pp_run(wocr_pp *p, const uint8_t *const *pages, const int32_t *w, const int32_t *h, int n, const PpArgs &a,
            int merge, int lanes, std::vector<PpPage> &out) {
    lanes = std::max(1, std::min(lanes, n));
    merge = std::max(1, merge);
    for (int i = 0; i < lanes; i++) pp_lane(p, i);
    out.assign((size_t)n, PpPage{});
    std::vector<std::exception_ptr> errs((size_t)lanes);
    auto work = [&](int L) {
        try {
            PpLane &ln = *p->lanes[L];
            WOCR_CUDA(cudaSetDevice(ln.ctx->c.device));
            // chunks: up to `merge` of this lane's pages in a row of one size, detected in one batch
            // and recognised with one wait; chunk j + 1 uploads while chunk j computes
            std::vector<std::vector<int>> chunks(1);
            for (int k = L; k < n; k += lanes) {
                chunks.back().push_back(k);
                const int nx = k + lanes;
                const bool last = nx >= n || (int)chunks.back().size() >= merge || w[nx] != w[k] || h[nx] != h[k];
                if (last && nx < n) chunks.emplace_back();
            }
            if (chunks.back().empty()) chunks.pop_back();
            if (!chunks.empty()) pp_upload_chunk(ln, 0, pages, chunks[0], w[chunks[0][0]], h[chunks[0][0]], out);
            for (size_t j = 0; j < chunks.size(); j++) {
                const std::vector<int> &ks = chunks[j];
                if (j + 1 < chunks.size()) {
                    const std::vector<int> &nk = chunks[j + 1];
                    pp_upload_chunk(ln, (int)((j + 1) & 1), pages, nk, w[nk[0]], h[nk[0]], out);
                }
                pp_front_chunk(ln, (int)(j & 1), ks, w[ks[0]], h[ks[0]], a, out);
                if (a.want_rec) {
                    std::vector<PpPage *> held;
                    for (int q : ks) held.push_back(&out[q]);
                    pp_recognize(ln, held);
                }
            }
        } catch (...) {
            errs[L] = std::current_exception();
        }
    };
    std::vector<std::thread> th;
    for (int L = 1; L < lanes; L++) th.emplace_back(work, L);
    work(0);
    for (auto &t : th) t.join();
    for (auto &e : errs)
        if (e) std::rethrow_exception(e);
}
}  // namespace

extern "C" {

int32_t wocr_pp_create(wocr_ctx *ctx, const wocr_model *det, const wocr_model *rec, wocr_pp **out) {
    return guard([&] {
        if (!ctx || !det || !rec || !out) fail(WOCR_ERR_INVALID, "null argument");
        auto p = std::make_unique<wocr_pp>();
        p->ctx = ctx;
        p->det_m = model_from_c(det);
        p->rec_m = model_from_c(rec);
        pp_lane(p.get(), 0);
        *out = p.release();
    });
}

void wocr_pp_destroy(wocr_pp *p) { delete p; }

int64_t wocr_pp_launches(wocr_pp *p) {
    if (!p) return -1;
    int64_t n = 0;
    for (const auto &ln : p->lanes) n += ln->ctx->c.launches;
    return n;
}

int32_t wocr_pp_page(wocr_pp *p, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side, const float *db,
                     float relv, int32_t per_batch, float *boxes, int32_t box_cap, int32_t *n_lines, uint32_t *best,
                     int64_t cap, int32_t *steps) {
    return guard([&] {
        if (!p || !rgb || !db || !n_lines || box_cap < 0 || cap < 0) fail(WOCR_ERR_INVALID, "bad argument");
        if (w <= 0 || h <= 0 || max_side <= 0 || per_batch <= 0) fail(WOCR_ERR_INVALID, "bad page size or batch");
        const bool want_rec = !(!best && cap == 0);
        if (want_rec && (!best || !steps)) fail(WOCR_ERR_INVALID, "null outputs");
        std::vector<PpPage> out;
        const uint8_t *pages[1] = {rgb};
        pp_run(p, pages, &w, &h, 1, PpArgs{max_side, db, relv, per_batch, want_rec}, 1, 1, out);
        const PpPage &pg = out[0];
        const int n = (int)(pg.boxes.size() / 6);
        *n_lines = n;
        if (boxes) {
            if (box_cap < n) fail(WOCR_ERR_CAPACITY, "boxes holds " + std::to_string(box_cap) + " of " + std::to_string(n));
            if (n) std::memcpy(boxes, pg.boxes.data(), pg.boxes.size() * 4);
        }
        if (!want_rec) return;
        int64_t need = 0;
        for (const auto &v : pg.best) need += (int64_t)v.size();
        if (cap < need) fail(WOCR_ERR_CAPACITY, "best holds " + std::to_string(cap) + " of " + std::to_string(need));
        int64_t o = 0;
        for (int i = 0; i < n; i++) {
            steps[i] = (int32_t)pg.best[i].size();
            std::copy(pg.best[i].begin(), pg.best[i].end(), best + o);
            o += (int64_t)pg.best[i].size();
        }
    });
}

int32_t wocr_pp_pages(wocr_pp *p, const uint8_t *const *pages, const int32_t *w, const int32_t *h, int32_t n,
                      int32_t max_side, const float *db, float relv, int32_t per_batch, int32_t merge, int32_t lanes,
                      float *boxes, int64_t box_cap, int32_t *n_lines, uint32_t *best, int64_t cap, int32_t *steps,
                      int64_t *bytes) {
    return guard([&] {
        if (!p || !pages || !w || !h || !db || !n_lines || n < 0 || box_cap < 0 || cap < 0)
            fail(WOCR_ERR_INVALID, "bad argument");
        if (max_side <= 0 || per_batch <= 0 || merge <= 0 || lanes <= 0 || lanes > 64)
            fail(WOCR_ERR_INVALID, "bad max_side, batch, merge or lane count");
        for (int k = 0; k < n; k++)
            if (!pages[k] || w[k] <= 0 || h[k] <= 0) fail(WOCR_ERR_INVALID, "bad page " + std::to_string(k));
        const bool want_rec = !(!best && cap == 0);
        if (want_rec && (!best || !steps)) fail(WOCR_ERR_INVALID, "null outputs");
        std::vector<PpPage> out;
        pp_run(p, pages, w, h, n, PpArgs{max_side, db, relv, per_batch, want_rec}, merge, lanes, out);
        int64_t nl = 0, need = 0, h2d = 0, d2h = 0;
        for (int k = 0; k < n; k++) {
            n_lines[k] = (int32_t)(out[k].boxes.size() / 6);
            nl += n_lines[k];
            for (const auto &v : out[k].best) need += (int64_t)v.size();
            h2d += out[k].h2d;
            d2h += out[k].d2h;
        }
        if (bytes) {
            bytes[0] = h2d;
            bytes[1] = d2h;
        }
        if (boxes || box_cap) {
            if (box_cap < nl) fail(WOCR_ERR_CAPACITY, "boxes holds " + std::to_string(box_cap) + " of " + std::to_string(nl));
            int64_t o = 0;
            for (int k = 0; k < n; k++) {
                if (!out[k].boxes.empty()) std::memcpy(boxes + o, out[k].boxes.data(), out[k].boxes.size() * 4);
                o += (int64_t)out[k].boxes.size();
            }
        }
        if (!want_rec) return;
        if (cap < need) fail(WOCR_ERR_CAPACITY, "best holds " + std::to_string(cap) + " of " + std::to_string(need));
        int64_t o = 0, li = 0;
        for (int k = 0; k < n; k++)
            for (const auto &v : out[k].best) {
                steps[li++] = (int32_t)v.size();
                std::copy(v.begin(), v.end(), best + o);
                o += (int64_t)v.size();
            }
    });
}

}  // extern "C"

// ---- the ocrs page pipeline -----------------------------------------------------------------
//
// The reference's default page loop (src/bin/ocr-bench.rs:458-585, no DET / REC): the GPU thread
// detects a page into its thresholded mask (Detector::detect_page); the CPU finds its words
// (word_rects), lines (ocrs find_text_lines), pads them and cuts ocrs line images
// (line_batches); the GPU thread recognises the batches of MERGE pages in one
// Recognizer::recognize call; the CPU decodes.  Here the mask, the words and the line images stay
// on the device (wocr_detect_pages' kernels, wocr_word_rects' kernels, k_ocrs_lines); only the
// word rectangles come to the host for the line grouping (layout.cpp) and only the arg-max
// classes for the decode.  As in the PP pipeline, a pipeline owns `lanes` workers on one GPU,
// each its own context, detector, recogniser and host thread; a lane detects `merge` of its pages
// in one batched pass and recognises all their lines in one recogniser pass.

namespace {

// Batches of one page's lines as line_batches forms them: grouped by image width rounded up to
// 50 (ascending), 20 lines a batch in line order.  Fills slots (line index per slot), and the
// batches' line counts and widths.
void ocrs_batching(const std::vector<LineCut> &cuts, std::vector<int> &slots, std::vector<int> &bn,
                   std::vector<int> &bw) {
    std::map<int, std::vector<int>> groups;
    for (int i = 0; i < (int)cuts.size(); i++)
        groups[(cuts[i].W + kLineBucket - 1) / kLineBucket * kLineBucket].push_back(i);
    for (auto &g : groups)
        for (size_t k = 0; k < g.second.size(); k += kLinesPerBatch) {
            const size_t e = std::min(g.second.size(), k + kLinesPerBatch);
            bn.push_back((int)(e - k));
            bw.push_back(g.first);
            slots.insert(slots.end(), g.second.begin() + k, g.second.begin() + e);
        }
}

// One page's lines: grouping and padding on the host; its crops and polygons.
struct OcrsPageLines {
    std::vector<float> words;     // padded, line by line
    std::vector<int> line_len;
    std::vector<LineCut> cuts;
    std::vector<int> vxy;         // polygons, x y pairs
    std::vector<int> v0;          // each line's first vertex
};

void ocrs_page_lines(const float *rects, int n, int pw, int ph, float relv, float relend, OcrsPageLines &out) {
    std::vector<int> order;
    text_lines(rects, n, order, out.line_len);
    out.words.resize(order.size() * 6);
    for (size_t i = 0; i < order.size(); i++) std::memcpy(out.words.data() + 6 * i, rects + 6 * (size_t)order[i], 24);
    size_t w0 = 0;
    for (int len : out.line_len) {
        float *lw = out.words.data() + 6 * w0;
        if (4 * len > kMaxLineVerts)
            fail(WOCR_ERR_UNSUPPORTED, "a text line of " + std::to_string(len) + " words (at most " +
                                           std::to_string(kMaxLineVerts / 4) + ")");
        pad_line(lw, len, relv, relend);
        out.v0.push_back((int)(out.vxy.size() / 2));
        out.cuts.push_back(line_cut(lw, len, pw, ph, out.vxy));
        w0 += (size_t)len;
    }
}

}  // namespace

extern "C" {

int32_t wocr_text_lines(const float *words, int32_t n, int32_t *order, int32_t *line_len, int32_t *n_lines) {
    return guard([&] {
        if (n < 0 || (n > 0 && (!words || !order || !line_len)) || !n_lines) fail(WOCR_ERR_INVALID, "bad argument");
        std::vector<int> o, l;
        text_lines(words, n, o, l);
        std::copy(o.begin(), o.end(), order);
        std::copy(l.begin(), l.end(), line_len);
        *n_lines = (int32_t)l.size();
    });
}

int32_t wocr_pad_line(float *words, int32_t n, float relv, float relend) {
    return guard([&] {
        if (n < 0 || (n > 0 && !words)) fail(WOCR_ERR_INVALID, "bad argument");
        pad_line(words, n, relv, relend);
    });
}

int32_t wocr_ocrs_lines(wocr_ctx *ctx, const uint8_t *d_rgb, int32_t w, int32_t h, const float *words,
                        const int32_t *line_len, int32_t n_lines, float *d_out, int64_t cap, int32_t *slots,
                        int32_t *widths, int32_t *batch_n, int32_t *batch_w, int32_t *n_batches, int64_t *total) {
    return guard([&] {
        if (!ctx || n_lines < 0 || (n_lines > 0 && (!words || !line_len)) || w <= 0 || h <= 0)
            fail(WOCR_ERR_INVALID, "bad argument");
        Ctx *c = &ctx->c;
        WOCR_CUDA(cudaSetDevice(c->device));
        std::vector<LineCut> cuts;
        std::vector<int> vxy, v0;
        size_t w0 = 0;
        for (int i = 0; i < n_lines; i++) {
            if (line_len[i] <= 0 || 4 * line_len[i] > kMaxLineVerts)
                fail(WOCR_ERR_INVALID, "line " + std::to_string(i) + " has " + std::to_string(line_len[i]) + " words");
            v0.push_back((int)(vxy.size() / 2));
            cuts.push_back(line_cut(words + 6 * w0, line_len[i], w, h, vxy));
            w0 += (size_t)line_len[i];
        }
        std::vector<int> sl, bn, bw;
        ocrs_batching(cuts, sl, bn, bw);
        int64_t off = 0;
        std::vector<k::OcrsLine> plan;
        size_t q = 0;
        for (size_t b = 0; b < bn.size(); b++) {
            for (int j = 0; j < bn[b]; j++, q++) {
                const int i = sl[q];
                const LineCut &lc = cuts[i];
                plan.push_back({d_rgb, w, h, lc.l, lc.t, lc.cw, lc.ch, lc.W, bw[b], v0[i],
                                4 * line_len[i], off + (int64_t)j * 64 * bw[b]});
                if (slots) slots[q] = i;
                if (widths) widths[q] = lc.W;
            }
            if (batch_n) batch_n[b] = bn[b];
            if (batch_w) batch_w[b] = bw[b];
            off += (int64_t)bn[b] * 64 * bw[b];
        }
        if (n_batches) *n_batches = (int32_t)bn.size();
        if (total) *total = off;
        if (!d_out || n_lines == 0) return;
        if (!d_rgb) fail(WOCR_ERR_INVALID, "null page");
        if (cap < off) fail(WOCR_ERR_CAPACITY, "line batches need " + std::to_string(off) + " floats");
        double bytes = 0;
        for (const auto &L : plan) bytes += 3.0 * L.cw * L.ch + 4.0 * 64 * L.bw;
        BufP dl = alloc(c, plan.size() * sizeof(k::OcrsLine)), dv = alloc(c, std::max<size_t>(vxy.size(), 2) * 4);
        WOCR_CUDA(cudaMemcpyAsync(dl->p, plan.data(), plan.size() * sizeof(k::OcrsLine), cudaMemcpyHostToDevice,
                                  c->stream));
        WOCR_CUDA(cudaMemcpyAsync(dv->p, vxy.data(), vxy.size() * 4, cudaMemcpyHostToDevice, c->stream));
        k::ocrs_lines(c, (const k::OcrsLine *)dl->p, (int)plan.size(), (const int2 *)dv->p, d_out, bytes);
        sync_bounded(c, 0);  // the plan's host copies are read until the uploads complete
    });
}

}  // extern "C"

struct OcrsLane {
    wocr_ctx *ctx = nullptr;
    wocr_detector *det = nullptr;
    wocr_recognizer *rec = nullptr;
    BufP pages, masks;  // a chunk of pages back to back, their masks
    size_t pages_bytes = 0, masks_bytes = 0;
    ~OcrsLane() {
        if (det) wocr_detector_destroy(det);
        if (rec) wocr_recognizer_destroy(rec);
        if (ctx) wocr_ctx_destroy(ctx);
    }
};

struct wocr_ocrs {
    wocr_ctx *ctx = nullptr;
    Model det_m, rec_m;
    std::vector<std::unique_ptr<OcrsLane>> lanes;
};

namespace {

// One page's results: the padded words of its lines, each line's image width and arg-max classes.
struct OcrsPage {
    OcrsPageLines lines;
    std::vector<int> widths;                 // per line
    std::vector<std::vector<uint32_t>> best;  // per line, its steps t < len
    int64_t h2d = 0, d2h = 0;
};

struct OcrsArgs {
    int w, h;
    float thr, relv, relend;
};

OcrsLane *ocrs_lane(wocr_ocrs *p, int i) {
    while ((int)p->lanes.size() <= i) {
        auto ln = std::make_unique<OcrsLane>();
        if (p->lanes.empty()) {
            ln->ctx = p->ctx;
            p->ctx->refs++;
        } else {
            check_st(wocr_ctx_create(p->ctx->c.device, p->ctx->c.lines, &ln->ctx));
        }
        ln->det = detector_from_model(ln->ctx, p->det_m);
        ln->rec = recognizer_from_model(ln->ctx, p->rec_m, ln->ctx->c.lines);
        p->lanes.push_back(std::move(ln));
    }
    return p->lanes[i].get();
}

// A chunk of pages on one lane: batched detection, word rectangles, lines (host), line images,
// one recognition pass, classes back.
void ocrs_chunk(OcrsLane &ln, const uint8_t *const *pages, const std::vector<int> &ks, const OcrsArgs &a,
                std::vector<OcrsPage> &out) {
    Ctx *c = &ln.ctx->c;
    WOCR_CUDA(cudaSetDevice(c->device));
    const int n = (int)ks.size(), words = (a.w + 31) / 32;
    const size_t page_bytes = (size_t)a.w * a.h * 3, mask_bytes = (size_t)words * a.h * 4;
    if (ln.pages_bytes < page_bytes * n) {
        ln.pages = alloc(c, page_bytes * n);
        ln.pages_bytes = page_bytes * n;
    }
    if (ln.masks_bytes < mask_bytes * n) {
        ln.masks = alloc(c, mask_bytes * n);
        ln.masks_bytes = mask_bytes * n;
    }
    uint8_t *dp = (uint8_t *)ln.pages->p;
    for (int q = 0; q < n; q++) {
        const uint8_t *src = pages[ks[q]];
        const bool dev = on_device(src);
        WOCR_CUDA(cudaMemcpyAsync(dp + page_bytes * q, src, page_bytes,
                                  dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
        if (!dev) out[ks[q]].h2d += (int64_t)page_bytes;
    }
    uint32_t *dm = (uint32_t *)ln.masks->p;
    detect_pages_run(ln.det, dp, n, a.w, a.h, a.thr, dm);
    // words: ocrs' word rectangles (expand 3, min area 100, src/bin/ocr-bench.rs:38-60)
    k::WordRects wr = k::word_rects(c, dm, n, a.w, a.h, 3.0f, 0.0f, 100.0f);
    std::vector<int32_t> counts((size_t)n);
    std::vector<float> rects((size_t)wr.n * 6);
    d2h(c, counts.data(), wr.page_count->p, (size_t)n * 4);
    d2h(c, rects.data(), wr.rects->p, rects.size() * 4);
    sync_bounded(c, 0);
    // lines, padding and crops on the host; every page's batches after the previous page's
    std::vector<k::OcrsLine> plan;
    std::vector<int> vxy;
    struct Batch {
        int page, n, w;
        int64_t off;
    };
    std::vector<Batch> batches;
    std::vector<std::pair<int, int>> slot_line;  // (page, line) of each batch slot, in order
    int64_t off = 0;
    size_t r0 = 0;
    for (int q = 0; q < n; q++) {
        OcrsPage &pg = out[ks[q]];
        ocrs_page_lines(rects.data() + 6 * r0, counts[q], a.w, a.h, a.relv, a.relend, pg.lines);
        r0 += (size_t)counts[q];
        std::vector<int> sl, bn, bw;
        ocrs_batching(pg.lines.cuts, sl, bn, bw);
        pg.widths.assign(pg.lines.cuts.size(), 0);
        size_t s = 0;
        const int vbase = (int)(vxy.size() / 2);
        vxy.insert(vxy.end(), pg.lines.vxy.begin(), pg.lines.vxy.end());
        for (size_t b = 0; b < bn.size(); b++) {
            batches.push_back({ks[q], bn[b], bw[b], off});
            for (int j = 0; j < bn[b]; j++, s++) {
                const int i = sl[s];
                const LineCut &lc = pg.lines.cuts[i];
                plan.push_back({dp + page_bytes * q, a.w, a.h, lc.l, lc.t, lc.cw, lc.ch, lc.W, bw[b],
                                vbase + pg.lines.v0[i], 4 * pg.lines.line_len[i], off + (int64_t)j * 64 * bw[b]});
                pg.widths[i] = lc.W;
                slot_line.push_back({ks[q], i});
            }
            off += (int64_t)bn[b] * 64 * bw[b];
        }
    }
    if (plan.empty()) return;
    BufP lines = alloc(c, (size_t)off * 4);
    BufP dl = alloc(c, plan.size() * sizeof(k::OcrsLine)), dv = alloc(c, std::max<size_t>(vxy.size(), 2) * 4);
    WOCR_CUDA(cudaMemcpyAsync(dl->p, plan.data(), plan.size() * sizeof(k::OcrsLine), cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaMemcpyAsync(dv->p, vxy.data(), vxy.size() * 4, cudaMemcpyHostToDevice, c->stream));
    double bytes = 0;
    for (const auto &L : plan) bytes += 3.0 * L.cw * L.ch + 4.0 * 64 * L.bw;
    k::ocrs_lines(c, (const k::OcrsLine *)dl->p, (int)plan.size(), (const int2 *)dv->p, (float *)lines->p, bytes);
    // every batch of the chunk in one recogniser pass (the reference's merged recognize)
    std::vector<DT> xs;
    for (const Batch &b : batches) {
        DT x;
        x.buf = lines;
        x.p = (float *)lines->p + b.off;
        x.shape = {b.n, 1, 64, b.w};
        x.strides = rowmajor_strides(x.shape);
        xs.push_back(x);
    }
    RecResult rr = recognize_dev(ln.rec, xs, nullptr, true, nullptr);
    std::vector<uint32_t> best((size_t)rr.tmax * rr.ntot);
    d2h(c, best.data(), rr.best->p, best.size() * 4);
    sync_bounded(c, 0);
    for (int line = 0; line < rr.ntot; line++) {
        OcrsPage &pg = out[slot_line[line].first];
        if (pg.best.empty()) pg.best.assign(pg.lines.cuts.size(), {});
        std::vector<uint32_t> &dst = pg.best[slot_line[line].second];
        const int len = rr.lens[line];
        dst.resize((size_t)len);
        for (int t = 0; t < len; t++) dst[t] = best[(size_t)t * rr.ntot + line];
        pg.d2h += (int64_t)len * 4;
    }
}

void ocrs_run(wocr_ocrs *p, const uint8_t *const *pages, int n, const OcrsArgs &a, int merge, int lanes,
              std::vector<OcrsPage> &out) {
    lanes = std::max(1, std::min(lanes, n));
    merge = std::max(1, merge);
    for (int i = 0; i < lanes; i++) ocrs_lane(p, i);
    out.assign((size_t)n, OcrsPage{});
    std::vector<std::exception_ptr> errs((size_t)lanes);
    auto work = [&](int L) {
        try {
            std::vector<int> ks;
            for (int k = L; k < n; k += lanes) {
                ks.push_back(k);
                if ((int)ks.size() >= merge || k + lanes >= n) {
                    ocrs_chunk(*p->lanes[L], pages, ks, a, out);
                    ks.clear();
                }
            }
        } catch (...) {
            errs[L] = std::current_exception();
        }
    };
    std::vector<std::thread> th;
    for (int L = 1; L < lanes; L++) th.emplace_back(work, L);
    work(0);
    for (auto &t : th) t.join();
    for (auto &e : errs)
        if (e) std::rethrow_exception(e);
}

}  // namespace

extern "C" {

int32_t wocr_ocrs_create(wocr_ctx *ctx, const wocr_model *det, const wocr_model *rec, wocr_ocrs **out) {
    return guard([&] {
        if (!ctx || !det || !rec || !out) fail(WOCR_ERR_INVALID, "null argument");
        auto p = std::make_unique<wocr_ocrs>();
        p->ctx = ctx;
        p->det_m = model_from_c(det);
        p->rec_m = model_from_c(rec);
        ocrs_lane(p.get(), 0);
        *out = p.release();
    });
}

void wocr_ocrs_destroy(wocr_ocrs *p) { delete p; }

int64_t wocr_ocrs_launches(wocr_ocrs *p) {
    if (!p) return -1;
    int64_t n = 0;
    for (const auto &ln : p->lanes) n += ln->ctx->c.launches;
    return n;
}

int32_t wocr_ocrs_pages(wocr_ocrs *p, const uint8_t *const *pages, int32_t n, int32_t w, int32_t h, float threshold,
                        float relv, float relend, int32_t merge, int32_t lanes, int32_t *n_lines, int32_t *line_words,
                        int64_t lines_cap, float *words, int64_t words_cap, int32_t *widths, int32_t *steps,
                        uint32_t *best, int64_t cap, int64_t *bytes) {
    return guard([&] {
        if (!p || !pages || !n_lines || n < 0 || lines_cap < 0 || words_cap < 0 || cap < 0)
            fail(WOCR_ERR_INVALID, "bad argument");
        if (w <= 0 || h <= 0 || merge <= 0 || lanes <= 0 || lanes > 64)
            fail(WOCR_ERR_INVALID, "bad page size, merge or lane count");
        for (int k = 0; k < n; k++)
            if (!pages[k]) fail(WOCR_ERR_INVALID, "null page " + std::to_string(k));
        std::vector<OcrsPage> out;
        ocrs_run(p, pages, n, OcrsArgs{w, h, threshold, relv, relend}, merge, lanes, out);
        int64_t nl = 0, nw = 0, need = 0, h2d = 0, d2h_ = 0;
        for (int k = 0; k < n; k++) {
            n_lines[k] = (int32_t)out[k].lines.line_len.size();
            nl += n_lines[k];
            nw += (int64_t)out[k].lines.words.size() / 6;
            for (const auto &v : out[k].best) need += (int64_t)v.size();
            h2d += out[k].h2d;
            d2h_ += out[k].d2h;
        }
        if (bytes) {
            bytes[0] = h2d;
            bytes[1] = d2h_;
        }
        if (lines_cap < nl || words_cap < nw || cap < need)
            fail(WOCR_ERR_CAPACITY, "outputs hold " + std::to_string(lines_cap) + " lines, " + std::to_string(words_cap) +
                                        " words, " + std::to_string(cap) + " classes; the pages need " +
                                        std::to_string(nl) + ", " + std::to_string(nw) + ", " + std::to_string(need));
        int64_t li = 0, wi = 0, o = 0;
        for (int k = 0; k < n; k++) {
            const OcrsPage &pg = out[k];
            for (size_t i = 0; i < pg.lines.line_len.size(); i++, li++) {
                if (line_words) line_words[li] = pg.lines.line_len[i];
                if (widths) widths[li] = pg.widths[i];
                const size_t t = i < pg.best.size() ? pg.best[i].size() : 0;
                if (steps) steps[li] = (int32_t)t;
                if (best && t) std::copy(pg.best[i].begin(), pg.best[i].end(), best + o);
                o += (int64_t)t;
            }
            if (words && !pg.lines.words.empty())
                std::memcpy(words + 6 * wi, pg.lines.words.data(), pg.lines.words.size() * 4);
            wi += (int64_t)pg.lines.words.size() / 6;
        }
    });
}

}  // extern "C"
