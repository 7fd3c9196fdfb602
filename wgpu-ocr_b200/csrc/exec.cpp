// The two graph executors of the reference, lowered to the sm_100a kernels.
#include "exec.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <set>

namespace wocr {

// =========================================================================================
// weights
// =========================================================================================
DevW upload(Ctx *c, const float *v, int64_t n) {
    DevW d;
    d.buf = alloc(c, (size_t)std::max<int64_t>(n, 4) * sizeof(float));
    d.p = (float *)d.buf->p;
    d.n = n;
    if (n > 0) WOCR_CUDA(cudaMemcpyAsync(d.p, v, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    return d;
}
DevW upload(Ctx *c, const std::vector<float> &v) { return upload(c, v.data(), (int64_t)v.size()); }

static int round4(int v) { return (v + 3) / 4 * 4; }

// Dense convolutions and matrix products run on the tcgen05 tensor-core kernel; WOCR_SIMT_GEMM=1
// selects the CUDA-core fp32 kernel instead (a diagnosis switch for comparing the two).
static bool use_umma() {
    static const bool v = [] {
        const char *e = std::getenv("WOCR_SIMT_GEMM");
        return !(e && e[0] == '1');
    }();
    return v;
}

std::shared_ptr<k::UmmaW> linear_umma(Ctx *c, const float *w_kn, int K, int N) {
    if (!use_umma()) return nullptr;
    std::vector<float> nk((size_t)N * K);
    for (int kk = 0; kk < K; kk++)
        for (int n = 0; n < N; n++) nk[(size_t)n * K + kk] = w_kn[(size_t)kk * N + n];
    return std::make_shared<k::UmmaW>(k::make_umma_weights(c, nk, N, K));
}

// [cout][cin/g][kh][kw] -> the layout of the kernel the conv runs on.
ConvW lower_conv_dense(Ctx *c, const HostW &w, const std::vector<float> &bias, int group) {
    if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "conv weight not 4D");
    ConvW cw;
    int cout = (int)w.dims[0], cin_g = (int)w.dims[1], kh = (int)w.dims[2], kw = (int)w.dims[3];
    cw.cout = cout;
    cw.kh = kh;
    cw.kw = kw;
    cw.group = group;
    std::vector<float> b = bias;
    b.resize(round4(cout), 0.f);
    if (group == 1) {
        cw.kind = ConvW::DENSE;
        cw.cin = cin_g;
        cw.ldw = round4(cout);
        int K = kh * kw * cin_g;
        std::vector<float> t((size_t)K * cw.ldw, 0.f);
        for (int co = 0; co < cout; co++)
            for (int ci = 0; ci < cin_g; ci++)
                for (int ky = 0; ky < kh; ky++)
                    for (int kx = 0; kx < kw; kx++)
                        t[(size_t)((ky * kw + kx) * cin_g + ci) * cw.ldw + co] =
                            w.data[(((size_t)co * cin_g + ci) * kh + ky) * kw + kx];
        cw.w = upload(c, t);
        if (use_umma()) {
            std::vector<float> nk((size_t)cout * K);
            for (int co = 0; co < cout; co++)
                for (int ci = 0; ci < cin_g; ci++)
                    for (int ky = 0; ky < kh; ky++)
                        for (int kx = 0; kx < kw; kx++)
                            nk[(size_t)co * K + (ky * kw + kx) * cin_g + ci] =
                                w.data[(((size_t)co * cin_g + ci) * kh + ky) * kw + kx];
            cw.uw = std::make_shared<k::UmmaW>(k::make_umma_weights(c, nk, cout, K));
        }
    } else {
        // depthwise: [kh][kw][c]
        cw.kind = ConvW::DEPTHWISE;
        cw.cin = group;
        std::vector<float> t((size_t)kh * kw * round4(cout), 0.f);
        for (int co = 0; co < cout; co++)
            for (int ky = 0; ky < kh; ky++)
                for (int kx = 0; kx < kw; kx++)
                    t[(size_t)(ky * kw + kx) * cout + co] = w.data[((size_t)co * kh + ky) * kw + kx];
        cw.w = upload(c, t);
    }
    cw.b = upload(c, b);
    return cw;
}

static ConvW lower_conv_direct(Ctx *c, const HostW &w, const std::vector<float> &bias) {
    ConvW cw;
    cw.kind = ConvW::DIRECT;
    int cout = (int)w.dims[0], kh = (int)w.dims[2], kw = (int)w.dims[3];
    cw.cout = cout;
    cw.cin = 1;
    cw.kh = kh;
    cw.kw = kw;
    std::vector<float> t((size_t)kh * kw * cout);
    for (int co = 0; co < cout; co++)
        for (int ky = 0; ky < kh; ky++)
            for (int kx = 0; kx < kw; kx++) t[(size_t)(ky * kw + kx) * cout + co] = w.data[((size_t)co * kh + ky) * kw + kx];
    cw.w = upload(c, t);
    cw.b = upload(c, bias);
    return cw;
}

ConvTW lower_convt(Ctx *c, const HostW &w, const std::vector<float> &bias, int stride) {
    if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "ConvTranspose weight not 4D");
    ConvTW t;
    t.cin = (int)w.dims[0];
    t.cout = (int)w.dims[1];
    t.kh = (int)w.dims[2];
    t.kw = (int)w.dims[3];
    t.s = stride;
    t.gemm = t.kh == stride && t.kw == stride;
    if (t.gemm) {
        // one GEMM over input pixels: column (ky*s + kx)*cout + co
        int N = t.cout * stride * stride;
        t.ldw = round4(N);
        std::vector<float> m((size_t)t.cin * t.ldw, 0.f);
        for (int ci = 0; ci < t.cin; ci++)
            for (int co = 0; co < t.cout; co++)
                for (int ky = 0; ky < t.kh; ky++)
                    for (int kx = 0; kx < t.kw; kx++)
                        m[(size_t)ci * t.ldw + (ky * stride + kx) * t.cout + co] =
                            w.data[(((size_t)ci * t.cout + co) * t.kh + ky) * t.kw + kx];
        t.w = upload(c, m);
        if (use_umma()) {
            std::vector<float> nk((size_t)N * t.cin);
            for (int ci = 0; ci < t.cin; ci++)
                for (int j = 0; j < N; j++) nk[(size_t)j * t.cin + ci] = m[(size_t)ci * t.ldw + j];
            t.uw = std::make_shared<k::UmmaW>(k::make_umma_weights(c, nk, N, t.cin));
        }
    } else {
        t.w = upload(c, w.data);
    }
    t.b = upload(c, bias);
    return t;
}

// The tap-convolution operand of a stride-1 dense convolution: [cout][ky][kx][ci].
void attach_tconv(Ctx *c, ConvW &cw, const HostW &w) {
    const int cout = (int)w.dims[0], cin = (int)w.dims[1], kh = (int)w.dims[2], kw = (int)w.dims[3];
    std::vector<float> nk((size_t)cout * kh * kw * cin);
    for (int co = 0; co < cout; co++)
        for (int ci = 0; ci < cin; ci++)
            for (int ky = 0; ky < kh; ky++)
                for (int kx = 0; kx < kw; kx++)
                    nk[(((size_t)co * kh + ky) * kw + kx) * cin + ci] = w.data[(((size_t)co * cin + ci) * kh + ky) * kw + kx];
    cw.tw = std::make_shared<k::TconvW>(k::make_tconv_weights(c, nk, cout, kh * kw, cin));
}

// ... of a ConvTranspose with kernel == stride s: one 1 x 1 tap, row (ky*s + kx)*cout + co.
void attach_tconv(Ctx *c, ConvTW &t, const HostW &w) {
    const int s = t.s, N = t.cout * s * s;
    std::vector<float> nk((size_t)N * t.cin);
    for (int ci = 0; ci < t.cin; ci++)
        for (int co = 0; co < t.cout; co++)
            for (int ky = 0; ky < s; ky++)
                for (int kx = 0; kx < s; kx++)
                    nk[(size_t)((ky * s + kx) * t.cout + co) * t.cin + ci] =
                        w.data[(((size_t)ci * t.cout + co) * t.kh + ky) * t.kw + kx];
    t.tw = std::make_shared<k::TconvW>(k::make_tconv_weights(c, nk, N, 1, t.cin));
    // the narrow 2 x 2 ones also on the row kernel (taps stacked along N)
    if (s == 2 && t.cout <= 32 && t.cin <= 64) k::add_convt_rows(c, *t.tw, nk, t.cout, t.cin);
}

// =========================================================================================
// tensor helpers
// =========================================================================================
static k::Strided strided_of(const DT &x, const DT &y) {
    k::Strided s;
    s.rank = x.rank();
    if (s.rank > kMaxRank) fail(WOCR_ERR_UNSUPPORTED, "rank " + std::to_string(s.rank) + " > 6");
    for (int d = 0; d < s.rank; d++) {
        s.dims[d] = x.shape[d];
        s.xs[d] = x.strides[d];
        s.ys[d] = y.strides[d];
    }
    return s;
}

static void copy_into(Ctx *c, const DT &x, const DT &y) { k::copy(c, x.p, y.p, strided_of(x, y)); }

DT to_nhwc(Ctx *c, const DT &x) {
    if (x.nhwc()) return x;
    if (x.rank() != 4) fail(WOCR_ERR_SHAPE, "expected a 4D tensor, got " + shape_str(x.shape));
    DT y = new_nhwc(c, x.shape[0], x.shape[1], x.shape[2], x.shape[3]);
    copy_into(c, x, y);
    return y;
}

DT to_rowmajor(Ctx *c, const DT &x) {
    if (x.rowmajor()) return x;
    DT y = new_rowmajor(c, x.shape);
    copy_into(c, x, y);
    return y;
}

DT from_host(Ctx *c, const float *x, const std::vector<int64_t> &shape) {
    DT t = new_rowmajor(c, shape);
    if (t.numel() > 0)
        WOCR_CUDA(cudaMemcpyAsync(t.p, x, (size_t)t.numel() * sizeof(float), cudaMemcpyDefault, c->stream));
    return t;
}

static DT view(const DT &x, std::vector<int64_t> shape, std::vector<int64_t> strides, int64_t offset = 0) {
    DT v;
    v.buf = x.buf;
    v.p = x.split ? reinterpret_cast<float *>(reinterpret_cast<uint16_t *>(x.p) + offset) : x.p + offset;
    v.shape = std::move(shape);
    v.strides = std::move(strides);
    v.split = x.split;
    return v;
}

static void strides4(const DT &t, int64_t (&s)[4]) {
    for (int d = 0; d < 4; d++) s[d] = t.strides[d];
}

// x (any format, 4-D) into the same-shaped view y (any format).
static void copy_any(Ctx *c, const DT &x, const DT &y) {
    if (!x.split && !y.split) {
        copy_into(c, x, y);
        return;
    }
    int64_t xs[4], ys[4], dims[4] = {x.shape[0], x.shape[1], x.shape[2], x.shape[3]};
    if (x.split && y.split) {
        DT t = new_nhwc(c, x.shape[0], x.shape[1], x.shape[2], x.shape[3]);
        copy_any(c, x, t);
        copy_any(c, t, y);
        return;
    }
    strides4(x, xs);
    strides4(y, ys);
    if (x.split)
        k::unsplit(c, reinterpret_cast<const uint16_t *>(x.p), xs, x.strides[3] / 2, y.p, ys, dims);
    else
        k::resplit(c, x.p, xs, reinterpret_cast<uint16_t *>(y.p), ys, y.strides[3] / 2, dims);
}

DT to_f32(Ctx *c, const DT &x) {
    if (!x.split) return x;
    DT y = new_nhwc(c, x.shape[0], x.shape[1], x.shape[2], x.shape[3]);
    copy_any(c, x, y);
    return y;
}

// The output of a kernel that may or may not write split tensors: `y` is what it writes (the
// step's own output when formats agree, else an fp32 temporary converted into it by done()).
struct KOut {
    DT y, target;
    bool convert = false;
};

static KOut kout(Ctx *c, const OutAlloc *out, int64_t n, int64_t ch, int64_t h, int64_t w, bool kernel_splits) {
    KOut o;
    o.target = out ? (*out)(n, ch, h, w) : new_nhwc(c, n, ch, h, w);
    if (o.target.split && !kernel_splits) {
        o.y = new_nhwc(c, n, ch, h, w);
        o.convert = true;
    } else {
        o.y = o.target;
    }
    return o;
}

static DT done(Ctx *c, const KOut &o) {
    if (o.convert) copy_any(c, o.y, o.target);
    return o.target;
}

// =========================================================================================
// convolution runs
// =========================================================================================
// MaxPool with kernel == stride, no padding (src/gpu.rs:462-482), on a split or fp32 input; the
// output split when `split_out`.
static DT maxpool_run(Ctx *ctx, DT x, int kh, int kw, bool split_out) {
    if (x.rank() != 4) fail(WOCR_ERR_SHAPE, "MaxPool input " + shape_str(x.shape));
    if (x.split && !x.nhwc()) x = to_f32(ctx, x);
    int64_t n = x.shape[0], ch = x.shape[1], h = x.shape[2], w = x.shape[3];
    int64_t oh = h / kh, ow = w / kw;
    if (x.split) {
        DT y = split_out ? new_nhwc_split(ctx, n, ch, oh, ow) : new_nhwc(ctx, n, ch, oh, ow);
        k::maxpool_split(ctx, reinterpret_cast<const uint16_t *>(x.p), x.strides[0], x.pix(), (int)n, (int)h, (int)w,
                         (int)ch, kh, kw, (int)oh, (int)ow, y.p, y.strides[0], y.pix(), y.split ? 1 : 0);
        return y;
    }
    x = to_nhwc(ctx, x);
    KOut o = kout(ctx, nullptr, n, ch, oh, ow, false);
    if (split_out) o.target = new_nhwc_split(ctx, n, ch, oh, ow), o.y = new_nhwc(ctx, n, ch, oh, ow), o.convert = true;
    k::pool(ctx, x.p, x.strides[0], x.pix(), (int)n, (int)h, (int)w, (int)ch, kh, kw, kh, kw, 0, 0, (int)oh, (int)ow,
            0, o.y.p, o.y.strides[0], o.y.pix());
    return done(ctx, o);
}

// A convolution whose input is a split tensor: the tap convolution (stride 1, dense) or the
// pointwise kernel; false when neither applies (the caller converts the input to fp32).
static bool conv_split(Ctx *c, const DT &x, const ConvW &cw, int act, const DT *res, const DT *scale,
                       const OutAlloc *out, DT &y, PoolReq *pool, HeadReq *head) {
    if (res || scale || cw.kind != ConvW::DENSE || !x.nhwc()) return false;
    int64_t n = x.shape[0], cin = x.shape[1], h = x.shape[2], w = x.shape[3];
    if (cw.cin != cin)
        fail(WOCR_ERR_SHAPE, "Conv expects " + std::to_string(cw.cin) + " channels, has " + std::to_string(cin));
    int pt, pl, pb, pr;
    if (cw.same_upper) {
        int64_t oh = (h + cw.sh - 1) / cw.sh, ow = (w + cw.sw - 1) / cw.sw;
        int64_t th = std::max<int64_t>((oh - 1) * cw.sh + cw.kh - h, 0);
        int64_t tw = std::max<int64_t>((ow - 1) * cw.sw + cw.kw - w, 0);
        pt = (int)(th / 2), pl = (int)(tw / 2), pb = (int)(th - th / 2), pr = (int)(tw - tw / 2);
    } else {
        pt = cw.pads[0], pl = cw.pads[1], pb = cw.pads[2], pr = cw.pads[3];
    }
    if (h + pt + pb < cw.kh || w + pl + pr < cw.kw)
        fail(WOCR_ERR_SHAPE, "conv input " + shape_str(x.shape) + " smaller than its kernel");
    const uint16_t *xp = reinterpret_cast<const uint16_t *>(x.p);
    if (cw.cout < 16 && cw.kh == 1 && cw.kw == 1 && cw.sh == 1 && cw.sw == 1 && pt == 0 && pl == 0 && pb == 0 &&
        pr == 0 && cin <= 4096) {
        KOut o = kout(c, out, n, cw.cout, h, w, false);
        k::pointwise(c, xp, x.strides[0], x.pix(), h * w, (int)n, (int)cin, cw.w.p, cw.ldw, cw.b.p, cw.cout, act,
                     o.y.p, o.y.strides[0], o.y.pix(), 1);
        y = done(c, o);
        return true;
    }
    if (!cw.tw || cw.sh != 1 || cw.sw != 1 || !k::tconv_input_ok(xp, x.strides[0], x.pix())) return false;
    const int64_t oh = h + pt + pb - cw.kh + 1, ow = w + pl + pr - cw.kw + 1;
    k::TconvP p;
    if (head && !pool && head->cw->cin == cw.cout && head->cw->cout <= 4) {
        // the head from the row kernel's epilogue; this convolution's output is never stored
        p.x = xp;
        p.x_n = x.strides[0];
        p.x_pix = x.pix();
        p.n = (int)n;
        p.h = (int)h;
        p.w = (int)w;
        p.cin = (int)cin;
        p.kh = cw.kh;
        p.kw = cw.kw;
        p.pt = pt;
        p.pl = pl;
        p.oh = (int)oh;
        p.ow = (int)ow;
        p.bias = cw.b.p;
        p.act = act;
        if (k::tconv_rows_eligible(*cw.tw, p)) {
            head->out = new_nhwc(c, n, head->cw->cout, oh, ow);
            p.head_w = head->cw->w.p;
            p.head_b = head->cw->b.p;
            p.head_ldw = head->cw->ldw;
            p.head_n = head->cw->cout;
            p.head_act = head->act;
            p.head_y = head->out.p;
            p.head_y_n = head->out.strides[0];
            p.head_y_pix = head->out.pix();
            k::tconv(c, *cw.tw, p);
            head->done = true;
            y = DT();
            return true;
        }
        p = k::TconvP();
    }
    KOut o = kout(c, out, n, cw.cout, oh, ow, true);
    p.x = xp;
    p.x_n = x.strides[0];
    p.x_pix = x.pix();
    p.n = (int)n;
    p.h = (int)h;
    p.w = (int)w;
    p.cin = (int)cin;
    p.kh = cw.kh;
    p.kw = cw.kw;
    p.pt = pt;
    p.pl = pl;
    p.oh = (int)oh;
    p.ow = (int)ow;
    p.bias = cw.b.p;
    p.act = act;
    p.y = o.y.p;
    p.split_out = o.y.split;
    p.y_n = o.y.strides[0];
    p.y_pix = o.y.pix();
    if (pool && !o.convert && cw.cout % 16 == 0) {
        // the 2 x 2 MaxPool of this output, from the epilogue
        pool->out = pool->split ? new_nhwc_split(c, n, cw.cout, oh / 2, ow / 2) : new_nhwc(c, n, cw.cout, oh / 2, ow / 2);
        p.pool_y = pool->out.p;
        p.pool_split = pool->out.split ? 1 : 0;
        p.pool_n = pool->out.strides[0];
        p.pool_pix = pool->out.pix();
        pool->done = true;
    }
    k::tconv(c, *cw.tw, p);
    y = done(c, o);
    return true;
}

static DT conv_run_body(Ctx *c, const DT &xin, const ConvW &cw, int act, const DT *res, const DT *scale,
                        const OutAlloc *out, PoolReq *pool, HeadReq *head);

DT conv_run(Ctx *c, const DT &xin, const ConvW &cw, int act, const DT *res, const DT *scale, const OutAlloc *out,
            PoolReq *pool, HeadReq *head) {
    DT y = conv_run_body(c, xin, cw, act, res, scale, out, pool, head);
    if (head && !head->done) {
        // not from the epilogue: the head as its own convolution of the stored output
        head->out = conv_run_body(c, y, *head->cw, head->act, nullptr, nullptr, nullptr, nullptr, nullptr);
        head->done = true;
    }
    return y;
}

static DT conv_run_body(Ctx *c, const DT &xin, const ConvW &cw, int act, const DT *res, const DT *scale,
                        const OutAlloc *out, PoolReq *pool, HeadReq *head) {
    if (xin.split) {
        DT y;
        if (conv_split(c, xin, cw, act, res, scale, out, y, pool, head)) {
            if (pool && !pool->done) pool->out = maxpool_run(c, y, 2, 2, pool->split), pool->done = true;
            return y;
        }
        return conv_run(c, to_f32(c, xin), cw, act, res, scale, out, pool);
    }
    if (pool) {
        DT y = conv_run(c, xin, cw, act, res, scale, out, nullptr);
        pool->out = maxpool_run(c, y, 2, 2, pool->split);
        pool->done = true;
        return y;
    }
    DT x = to_nhwc(c, xin);
    int64_t n = x.shape[0], cin = x.shape[1], h = x.shape[2], w = x.shape[3];
    int pt, pl, pb, pr;
    if (cw.same_upper) {
        int64_t oh = (h + cw.sh - 1) / cw.sh, ow = (w + cw.sw - 1) / cw.sw;
        int64_t th = std::max<int64_t>((oh - 1) * cw.sh + cw.kh - h, 0);
        int64_t tw = std::max<int64_t>((ow - 1) * cw.sw + cw.kw - w, 0);
        pt = (int)(th / 2), pl = (int)(tw / 2), pb = (int)(th - th / 2), pr = (int)(tw - tw / 2);
    } else {
        pt = cw.pads[0], pl = cw.pads[1], pb = cw.pads[2], pr = cw.pads[3];
    }
    if (cw.kind == ConvW::DIRECT) {
        int64_t ch = h + 2 * pt - cw.kh + 1, cwd = w + 2 * pt - cw.kw + 1;
        if (ch <= 0 || cwd <= 0) fail(WOCR_ERR_SHAPE, "conv input " + shape_str(x.shape) + " smaller than its kernel");
        if (cin != 1) fail(WOCR_ERR_SHAPE, "direct conv expects 1 channel, has " + std::to_string(cin));
        int64_t oh = ch / cw.pool_h, ow = cwd / cw.pool_w;
        const bool splits = (cw.cout == 16 || cw.cout == 32) && cw.kh * cw.kw <= 49;
        KOut o = kout(c, out, n, cw.cout, oh, ow, splits);
        k::conv_direct(c, x.p, x.strides[0], x.pix(), (int)n, (int)h, (int)w, cw.w.p, cw.b.p, cw.cout, cw.kh, cw.kw,
                       pt, act, cw.pool_h, cw.pool_w, o.y.p, o.y.strides[0], o.y.pix(), (int)oh, (int)ow,
                       o.y.split ? 1 : 0);
        return done(c, o);
    }
    if (h + pt + pb < cw.kh || w + pl + pr < cw.kw)
        fail(WOCR_ERR_SHAPE, "conv input " + shape_str(x.shape) + " smaller than its kernel");
    int64_t oh = (h + pt + pb - cw.kh) / cw.sh + 1;
    int64_t ow = (w + pl + pr - cw.kw) / cw.sw + 1;
    if (res && res->shape != std::vector<int64_t>{n, cw.cout, oh, ow})
        fail(WOCR_ERR_SHAPE, "residual " + shape_str(res->shape) + " for a conv giving " +
                                 shape_str({n, cw.cout, oh, ow}));
    if (scale && scale->numel() != n * cin)
        fail(WOCR_ERR_SHAPE, "input scale " + shape_str(scale->shape) + " for " + shape_str(x.shape));
    if ((res || scale) && cw.kind != ConvW::DENSE) fail(WOCR_ERR_UNSUPPORTED, "residual after a grouped conv");
    KOut o = kout(c, out, n, cw.cout, oh, ow, false);
    const DT &y = o.y;
    if (cw.kind == ConvW::DEPTHWISE) {
        if (cin != cw.cout || cw.group != cin)
            fail(WOCR_ERR_UNSUPPORTED, "grouped conv with group " + std::to_string(cw.group));
        k::depthwise(c, x.p, x.strides[0], x.pix(), (int)n, (int)h, (int)w, (int)cin, cw.w.p, cw.b.p, cw.kh, cw.kw,
                     cw.sh, cw.sw, pt, pl, (int)oh, (int)ow, act, y.p, y.strides[0], y.pix());
        return done(c, o);
    }
    if (cw.cin != cin)
        fail(WOCR_ERR_SHAPE, "Conv expects " + std::to_string(cw.cin) + " channels, has " + std::to_string(cin));
    if (cw.cout < 16 && cw.kh == 1 && cw.kw == 1 && cw.sh == 1 && cw.sw == 1 && pt == 0 && pl == 0 && pb == 0 && pr == 0 && !res && !scale &&
        cin <= 4096) {
        // too narrow for a tensor-core tile: a memory-bound pass over the pixels
        k::pointwise(c, x.p, x.strides[0], x.pix(), h * w, (int)n, (int)cin, cw.w.p, cw.ldw, cw.b.p, cw.cout, act, y.p,
                     y.strides[0], y.pix());
        return done(c, o);
    }
    DT r, s;
    k::ConvP p;
    p.x = x.p;
    p.x_n = x.strides[0];
    p.x_pix = x.pix();
    p.n = (int)n;
    p.h = (int)h;
    p.w = (int)w;
    p.cin = (int)cin;
    p.wt = cw.w.p;
    p.ldw = cw.ldw;
    p.bias = cw.b.p;
    p.cout = cw.cout;
    p.kh = cw.kh;
    p.kw = cw.kw;
    p.sh = cw.sh;
    p.sw = cw.sw;
    p.pt = pt;
    p.pl = pl;
    p.oh = (int)oh;
    p.ow = (int)ow;
    p.y = y.p;
    p.y_n = y.strides[0];
    p.y_pix = y.pix();
    p.act = act;
    if (res) {
        r = to_nhwc(c, *res);
        p.res = r.p;
        p.res_n = r.strides[0];
        p.res_pix = r.pix();
    }
    if (scale) {
        s = to_rowmajor(c, *scale);
        p.insc = s.p;
    }
    if (k::conv_narrow_ok(p) && !std::getenv("WOCR_NO_NARROW")) {
        k::conv_narrow(c, p);
        return done(c, o);
    }
    if (cw.uw) {
        k::UmmaP u;
        u.mode = 1;
        u.x = p.x;
        u.x_n = p.x_n;
        u.x_pix = p.x_pix;
        u.n = p.n;
        u.h = p.h;
        u.w = p.w;
        u.cin = p.cin;
        u.kh = p.kh;
        u.kw = p.kw;
        u.sh = p.sh;
        u.sw = p.sw;
        u.pt = p.pt;
        u.pl = p.pl;
        u.oh = p.oh;
        u.ow = p.ow;
        u.insc = p.insc;
        u.vec = (p.cin % 8 == 0) && (p.x_pix % 4 == 0) && (p.x_n % 4 == 0) &&
                ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
        u.M = (int64_t)p.n * p.oh * p.ow;
        u.bias = p.bias;
        u.act = p.act;
        u.y = p.y;
        u.y_n = p.y_n;
        u.y_pix = p.y_pix;
        u.res = p.res;
        u.res_n = p.res_n;
        u.res_pix = p.res_pix;
        k::umma_gemm(c, *cw.uw, u);
        return done(c, o);
    }
    k::conv_gemm(c, p);
    return done(c, o);
}

static DT convt_run(Ctx *c, const DT &xin, const ConvTW &t, int act, const OutAlloc *out = nullptr) {
    if (xin.split) {
        const uint16_t *xp = reinterpret_cast<const uint16_t *>(xin.p);
        if (!t.tw || !xin.nhwc() || !k::tconv_input_ok(xp, xin.strides[0], xin.pix()))
            return convt_run(c, to_f32(c, xin), t, act, out);
        int64_t n = xin.shape[0], cin = xin.shape[1], h = xin.shape[2], w = xin.shape[3];
        if (cin != t.cin) fail(WOCR_ERR_SHAPE, "ConvTranspose expects " + std::to_string(t.cin) + " channels, has " +
                                                   std::to_string(cin));
        KOut o = kout(c, out, n, t.cout, h * t.s, w * t.s, true);
        k::TconvP p;
        p.x = xp;
        p.x_n = xin.strides[0];
        p.x_pix = xin.pix();
        p.n = (int)n;
        p.h = (int)h;
        p.w = (int)w;
        p.cin = (int)cin;
        p.oh = (int)h;
        p.ow = (int)w;
        p.bias = t.b.p;
        p.act = act;
        p.y = o.y.p;
        p.split_out = o.y.split;
        p.y_n = o.y.strides[0];
        p.y_pix = o.y.pix();
        p.scatter = t.s;
        p.scat_cout = t.cout;
        k::tconv(c, *t.tw, p);
        return done(c, o);
    }
    DT x = to_nhwc(c, xin);
    int64_t n = x.shape[0], cin = x.shape[1], h = x.shape[2], w = x.shape[3];
    if (cin != t.cin) fail(WOCR_ERR_SHAPE, "ConvTranspose expects " + std::to_string(t.cin) + " channels, has " +
                                               std::to_string(cin));
    int64_t oh = (h - 1) * t.s + t.kh, ow = (w - 1) * t.s + t.kw;
    KOut o = kout(c, out, n, t.cout, oh, ow, false);
    const DT &y = o.y;
    if (t.gemm) {
        k::ConvP p;
        p.x = x.p;
        p.x_n = x.strides[0];
        p.x_pix = x.pix();
        p.n = (int)n;
        p.h = (int)h;
        p.w = (int)w;
        p.cin = (int)cin;
        p.wt = t.w.p;
        p.ldw = t.ldw;
        p.bias = t.b.p;
        p.cout = t.cout * t.s * t.s;
        p.oh = (int)h;
        p.ow = (int)w;
        p.y = y.p;
        p.y_n = y.strides[0];
        p.y_pix = y.pix();
        p.act = act;
        p.scatter = t.s;
        p.scat_cout = t.cout;
        if (t.uw) {
            k::UmmaP u;
            u.mode = 1;
            u.x = p.x;
            u.x_n = p.x_n;
            u.x_pix = p.x_pix;
            u.n = p.n;
            u.h = p.h;
            u.w = p.w;
            u.cin = p.cin;
            u.oh = p.oh;
            u.ow = p.ow;
            u.vec = (p.cin % 8 == 0) && (p.x_pix % 4 == 0) && (p.x_n % 4 == 0) &&
                    ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
            u.M = (int64_t)p.n * p.oh * p.ow;
            u.bias = p.bias;
            u.act = p.act;
            u.y = p.y;
            u.y_n = p.y_n;
            u.y_pix = p.y_pix;
            u.scatter = t.s;
            u.scat_cout = t.cout;
            k::umma_gemm(c, *t.uw, u);
        } else {
            k::conv_gemm(c, p);
        }
    } else {
        k::convt_gather(c, x.p, x.strides[0], x.pix(), (int)n, (int)h, (int)w, (int)cin, t.w.p, t.b.p, t.cout, t.kh,
                        t.kw, t.s, act, y.p, y.strides[0], y.pix(), (int)oh, (int)ow);
    }
    return done(c, o);
}

DT linear_run(Ctx *c, const DT &xin, const DevW &w, const DevW &b, int K, int N, int ldw, int act,
              const k::UmmaW *uw) {
    if (xin.shape.empty() || xin.shape.back() != K)
        fail(WOCR_ERR_SHAPE, "MatMul: " + shape_str(xin.shape) + " by [" + std::to_string(K) + ", " +
                                 std::to_string(N) + "]");
    DT x = to_rowmajor(c, xin);
    int64_t M = x.numel() / K;
    std::vector<int64_t> shape = x.shape;
    shape.back() = N;
    DT y = new_rowmajor(c, shape);
    k::ConvP p;
    p.x = x.p;
    p.x_n = M * K;
    p.x_pix = K;
    p.n = 1;
    p.h = 1;
    p.w = (int)M;
    p.cin = K;
    p.wt = w.p;
    p.ldw = ldw;
    p.bias = b.p;
    p.cout = N;
    p.oh = 1;
    p.ow = (int)M;
    p.y = y.p;
    p.y_n = M * N;
    p.y_pix = N;
    p.act = act;
    if (uw) {
        k::UmmaP u;
        u.mode = 0;
        u.x = x.p;
        u.lda = K;
        u.vec = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(x.p) & 15) == 0);
        u.M = M;
        u.bias = b.p;
        u.act = act;
        u.y = y.p;
        u.ldy = N;
        k::umma_gemm(c, *uw, u);
        return y;
    }
    k::conv_gemm(c, p);
    return y;
}

// =========================================================================================
// Executor
// =========================================================================================
Value Executor::get(std::map<std::string, Value> &vals, const std::string &name) {
    auto it = vals.find(name);
    if (it != vals.end()) return it->second;
    auto wi = weights.find(name);
    if (wi != weights.end()) {
        Value v;
        v.f = wi->second;
        return v;
    }
    auto ii = model.ints.find(name);
    if (ii != model.ints.end()) {
        Value v;
        v.is_int = true;
        v.iv = ii->second;
        v.ishape = {(int64_t)ii->second.size()};
        return v;
    }
    fail(WOCR_ERR_MISSING, "missing value " + name);
}

DT Executor::getx(std::map<std::string, Value> &vals, const std::string &name) {
    Value v = get(vals, name);
    if (v.is_int) fail(WOCR_ERR_SHAPE, name + " is not float");
    return v.f;
}

DT Executor::getf(std::map<std::string, Value> &vals, const std::string &name) {
    return to_f32(ctx, getx(vals, name));
}

// Which step outputs are stored split: those whose kernel can write them so (a Cin = 1 direct
// conv, a tap convolution or tap ConvTranspose fed split, a MaxPool, Concat or Identity of split
// values) and whose every reader takes them (tap convolutions, the pointwise head, MaxPool,
// split Concats and Identities).  The graph output never is.  Fixed point from above.
void Executor::plan_split() {
    for (auto &st : steps) st.split_out = false;
    if (!allow_split) return;
    std::map<std::string, std::vector<int>> readers;
    for (int i = 0; i < (int)steps.size(); i++)
        for (auto &nm : steps[i].inputs) readers[nm].push_back(i);
    auto pointwise_head = [](const ConvW &cw) {
        return cw.kind == ConvW::DENSE && cw.cout < 16 && cw.kh == 1 && cw.kw == 1 && cw.sh == 1 && cw.sw == 1 &&
               !cw.same_upper && cw.pads[0] == 0 && cw.pads[1] == 0 && cw.pads[2] == 0 && cw.pads[3] == 0;
    };
    std::set<std::string> sp;
    for (auto &st : steps) {
        bool capable = false;
        switch (st.kind) {
        case Step::G_DIRECT: capable = (st.conv.cout == 16 || st.conv.cout == 32) && st.conv.kh * st.conv.kw <= 49; break;
        case Step::G_CONV: capable = (bool)st.conv.tw; break;
        case Step::G_CONVT: capable = (bool)st.convt.tw; break;
        case Step::G_MAXPOOL:
        case Step::G_CONCAT:
        case Step::G_IDENTITY: capable = true; break;
        default: break;
        }
        if (capable && st.output != output && st.output != input) sp.insert(st.output);
    }
    auto accepts = [&](const Step &st) {
        switch (st.kind) {
        case Step::G_CONV: return (bool)st.conv.tw || pointwise_head(st.conv);
        case Step::G_CONVT: return (bool)st.convt.tw;
        case Step::G_MAXPOOL: return true;
        case Step::G_CONCAT:
        case Step::G_IDENTITY: return sp.count(st.output) > 0;
        default: return false;
        }
    };
    for (bool changed = true; changed;) {
        changed = false;
        for (auto &st : steps) {
            if (!sp.count(st.output)) continue;
            bool ok = true;
            if (st.kind != Step::G_DIRECT)
                for (auto &nm : st.inputs) ok = ok && sp.count(nm) > 0;
            for (int r : readers[st.output]) ok = ok && accepts(steps[r]);
            if (!ok) {
                sp.erase(st.output);
                changed = true;
            }
        }
    }
    for (auto &st : steps) st.split_out = sp.count(st.output) > 0;
}

void Executor::finalize() {
    // float initializers read at run time by steps that are not fused away
    std::set<std::string> needed;
    for (auto &s : steps)
        for (auto &i : s.inputs) needed.insert(i);
    for (auto &name : needed) {
        auto it = model.weights.find(name);
        if (it == model.weights.end() || weights.count(name)) continue;
        DT t;
        DevW d = upload(ctx, it->second.data);
        t.buf = d.buf;
        t.p = d.p;
        t.shape = it->second.dims;
        if (t.shape.empty()) t.shape = {1};
        t.strides = rowmajor_strides(t.shape);
        weights[name] = t;
    }
    last_use.clear();
    for (int i = 0; i < (int)steps.size(); i++)
        for (auto &n : steps[i].inputs) last_use[n] = i;
    // Channel Concats whose parts all come from convolution steps: those steps write straight
    // into their channel slice of the Concat output, and the Concat itself copies nothing.
    concat_slot.clear();
    std::map<std::string, int> producer;
    for (int i = 0; i < (int)steps.size(); i++) producer[steps[i].output] = i;
    for (auto &st : steps) {
        bool channel_concat = st.kind == Step::G_CONCAT;
        if (st.kind == Step::N_GENERIC) {
            const Node &n = model.nodes[st.node];
            channel_concat = n.op == "Concat" && n.int_("axis").value_or(0) == 1;
        }
        if (!channel_concat) continue;
        std::vector<std::pair<std::string, int>> parts;
        bool ok = true;
        std::set<std::string> seen;
        for (auto &nm : st.inputs) {
            auto pi = producer.find(nm);
            if (pi == producer.end() || nm == input || nm == output || !seen.insert(nm).second ||
                concat_slot.count(nm)) {
                ok = false;
                break;
            }
            const Step &ps = steps[pi->second];
            int c = 0;
            if (ps.kind == Step::G_CONV || ps.kind == Step::G_DIRECT || ps.kind == Step::G_DEPTHWISE ||
                ps.kind == Step::N_CONV)
                c = ps.conv.cout;
            else if (ps.kind == Step::G_CONVT || ps.kind == Step::N_CONVT)
                c = ps.convt.cout;
            if (c <= 0) {
                ok = false;
                break;
            }
            parts.push_back({nm, c});
        }
        if (!ok || parts.size() < 2) continue;
        int64_t ctot = 0;
        for (auto &pp : parts) ctot += pp.second;
        int64_t off = 0;
        for (auto &pp : parts) {
            concat_slot[pp.first] = {st.output, off, ctot};
            off += pp.second;
        }
    }
    plan_split();
    // 2 x 2 MaxPools computed in the epilogue of the tap convolution producing their input
    for (auto &st : steps) st.pool_output.clear(), st.pool_fused_away = false;
    if (allow_split) {
        for (auto &mp : steps) {
            if (mp.kind != Step::G_MAXPOOL || mp.conv.kh != 2 || mp.conv.kw != 2) continue;
            auto pi = producer.find(mp.inputs[0]);
            if (pi == producer.end()) continue;
            Step &cs = steps[pi->second];
            if (cs.kind != Step::G_CONV || !cs.conv.tw || !cs.pool_output.empty() || cs.conv.cout % 16) continue;
            cs.pool_output = mp.output;
            cs.pool_split = mp.split_out;
            mp.pool_fused_away = true;
        }
    }
    // 1 x 1 heads (at most 4 outputs, fp32) computed in the epilogue of the 3 x 3 tap convolution
    // they read, when nothing else reads its output
    for (auto &st : steps) st.head_output.clear(), st.head_step = -1, st.head_fused_away = false;
    if (allow_split) {
        for (size_t hi = 0; hi < steps.size(); hi++) {
            Step &hs = steps[hi];
            const ConvW &h = hs.conv;
            if (hs.kind != Step::G_CONV || h.kind != ConvW::DENSE || h.kh != 1 || h.kw != 1 || h.sh != 1 ||
                h.sw != 1 || h.cout > 4 || h.same_upper || h.pads[0] || h.pads[1] || h.pads[2] || h.pads[3] ||
                hs.split_out || concat_slot.count(hs.output))
                continue;
            auto readers = [&](const std::string &v) {
                int r = 0;
                for (const Step &o : steps)
                    for (const std::string &in : o.inputs) r += in == v;
                return r;
            };
            // through identity steps (a zero Pad) with one reader each
            std::string src = hs.inputs[0];
            std::vector<int> between;
            auto pi = producer.find(src);
            bool ok = pi != producer.end();
            while (ok && steps[pi->second].kind == Step::G_IDENTITY) {
                const Step &id = steps[pi->second];
                ok = readers(id.output) == 1 && id.output != output && !concat_slot.count(id.output);
                between.push_back(pi->second);
                src = id.inputs[0];
                pi = producer.find(src);
                ok = ok && pi != producer.end();
            }
            if (!ok) continue;
            Step &cs = steps[pi->second];
            if (cs.kind != Step::G_CONV || !cs.conv.tw || !cs.conv.tw->x3 || cs.conv.kh != 3 || cs.conv.kw != 3 ||
                !cs.pool_output.empty() || !cs.head_output.empty() || cs.conv.cout != h.cin || cs.output == output ||
                concat_slot.count(cs.output) || readers(cs.output) != 1)
                continue;
            cs.head_output = hs.output;
            cs.head_step = (int)hi;
            hs.head_fused_away = true;
            for (int b : between) steps[b].head_fused_away = true;
        }
    }
}

// The output of a step registered in concat_slot: a channel slice of the Concat buffer (made on
// first use with the producing step's batch and spatial size).
DT Executor::slot_output(const std::string &name, int64_t n, int64_t c, int64_t h, int64_t w, bool split) {
    auto fresh = [&](int64_t ch) { return split ? new_nhwc_split(ctx, n, ch, h, w) : new_nhwc(ctx, n, ch, h, w); };
    auto si = concat_slot.find(name);
    if (si == concat_slot.end() || !cbufs) return fresh(c);
    const ConcatSlot &sl = si->second;
    auto bi = cbufs->find(sl.concat);
    if (bi == cbufs->end()) bi = cbufs->emplace(sl.concat, fresh(sl.ctot)).first;
    const DT &b = bi->second;
    if (b.shape[0] != n || b.shape[2] != h || b.shape[3] != w || sl.offset + c > sl.ctot || b.split != split)
        return fresh(c);  // shapes or formats differ: the Concat will copy this part
    return view(b, {n, c, h, w}, b.strides, sl.offset);
}

DT Executor::run(const DT &x) { return run_to(x, (int)steps.size()); }

DT Executor::run_to(const DT &x, int upto) {
    if (upto < 0 || upto > (int)steps.size()) fail(WOCR_ERR_INVALID, "step index out of range");
    std::map<std::string, DT> concat_bufs;
    cbufs = &concat_bufs;
    struct Reset {
        std::map<std::string, DT> **p;
        ~Reset() { *p = nullptr; }
    } reset{&cbufs};
    std::map<std::string, Value> vals;
    Value in;
    in.f = x;
    vals[input] = in;
    for (int i = 0; i < upto; i++) {
        exec_step(steps[i], vals);
        for (auto &n : steps[i].inputs) {
            auto lu = last_use.find(n);
            if (lu != last_use.end() && lu->second == i && n != output && n != input) vals.erase(n);
        }
    }
    // the whole graph: its output; a prefix: the first input of step `upto`
    const std::string &want = upto == (int)steps.size() ? output : steps[upto].inputs[0];
    auto it = vals.find(want);
    if (it == vals.end()) fail(WOCR_ERR_MISSING, "value " + want + " not computed");
    if (it->second.is_int) fail(WOCR_ERR_SHAPE, "value " + want + " is not float");
    return to_f32(ctx, it->second.f);
}

bool Executor::ends_in_linear() const {
    if (steps.empty()) return false;
    const Step &s = steps.back();
    // the fused arg-max epilogue exists for tiles of 64 columns or more (more than 32 classes)
    return s.kind == Step::N_LINEAR && s.act == 0 && s.luw && s.luw->bn >= 64 && s.output == output;
}

// The final linear layer with the row arg-max in its epilogue: per N tile partials, then one
// merge pass; the logits are never stored (the CTC head, src/nd.rs:291 + 360-391).
std::vector<int64_t> Executor::linear_argmax(const DT &xin, uint32_t *best, float *row_max, float *row_lse) {
    const Step &s = steps.back();
    if (xin.shape.empty() || xin.shape.back() != s.lk)
        fail(WOCR_ERR_SHAPE, "MatMul: " + shape_str(xin.shape) + " by [" + std::to_string(s.lk) + ", " +
                                 std::to_string(s.ln) + "]");
    DT x = to_rowmajor(ctx, xin);
    const int64_t M = x.numel() / s.lk;
    const int ntn = k::umma_part_slots(*s.luw);
    // no log-sum-exp wanted: no exponentials' sums (the epilogue's second pass is skipped)
    BufP pm = alloc(ctx, (size_t)std::max<int64_t>(M, 1) * ntn * 4),
         ps = row_lse ? alloc(ctx, (size_t)std::max<int64_t>(M, 1) * ntn * 4) : nullptr,
         pi = alloc(ctx, (size_t)std::max<int64_t>(M, 1) * ntn * 4);
    k::UmmaP u;
    u.mode = 0;
    u.x = x.p;
    u.lda = s.lk;
    u.vec = (s.lk % 4 == 0) && ((reinterpret_cast<uintptr_t>(x.p) & 15) == 0);
    u.M = M;
    u.bias = s.lb.p;
    u.act = 0;
    u.part_max = (float *)pm->p;
    u.part_sum = ps ? (float *)ps->p : nullptr;
    u.part_idx = (uint32_t *)pi->p;
    u.part_ld = ntn;
    k::umma_gemm(ctx, *s.luw, u);
    k::argmax_merge(ctx, (const float *)pm->p, ps ? (const float *)ps->p : nullptr, (const uint32_t *)pi->p, M, ntn,
                    best, row_max, row_lse);
    std::vector<int64_t> shape = x.shape;
    shape.back() = s.ln;
    return shape;
}

// Channel Concat of NHWC parts: parts already written into their slice of the registered
// buffer are not copied again (src/gpu.rs:1317-1330 copies every part).
DT Executor::concat_channels(const std::vector<DT> &parts, const std::string &out_name, bool split) {
    const DT &a = parts[0];
    int64_t ctot = 0;
    for (auto &t : parts) ctot += t.shape[1];
    DT y;
    bool reuse = false;
    if (cbufs) {
        auto bi = cbufs->find(out_name);
        if (bi != cbufs->end() && bi->second.shape == std::vector<int64_t>{a.shape[0], ctot, a.shape[2], a.shape[3]}) {
            y = bi->second;
            reuse = true;
        }
    }
    if (!reuse)
        y = split ? new_nhwc_split(ctx, a.shape[0], ctot, a.shape[2], a.shape[3])
                  : new_nhwc(ctx, a.shape[0], ctot, a.shape[2], a.shape[3]);
    int64_t off = 0;
    for (auto &t : parts) {
        DT dst = view(y, t.shape, y.strides, off);
        if (!(reuse && t.p == dst.p && t.strides == dst.strides && t.split == dst.split)) copy_any(ctx, t, dst);
        off += t.shape[1];
    }
    return y;
}

void Executor::exec_step(const Step &s, std::map<std::string, Value> &vals) {
    Value out;
    const OutAlloc alloc_out = [&](int64_t n, int64_t c, int64_t h, int64_t w) {
        return slot_output(s.output, n, c, h, w, s.split_out);
    };
    switch (s.kind) {
    case Step::G_CONV:
    case Step::G_DIRECT:
    case Step::G_DEPTHWISE:
        if (s.head_fused_away) return;  // computed with the convolution it reads
        if (!s.head_output.empty()) {
            const Step &hs = steps[s.head_step];
            HeadReq hr;
            hr.cw = &hs.conv;
            hr.act = hs.act;
            conv_run(ctx, getx(vals, s.inputs[0]), s.conv, s.act, nullptr, nullptr, &alloc_out, nullptr, &hr);
            Value hv;
            hv.f = hr.out;
            vals[s.head_output] = hv;
            return;  // this step's own output has no other reader
        }
        if (!s.pool_output.empty()) {
            PoolReq pr;
            pr.split = s.pool_split;
            out.f = conv_run(ctx, getx(vals, s.inputs[0]), s.conv, s.act, nullptr, nullptr, &alloc_out, &pr);
            Value pv;
            pv.f = pr.out;
            vals[s.pool_output] = pv;
            break;
        }
        out.f = conv_run(ctx, getx(vals, s.inputs[0]), s.conv, s.act, nullptr, nullptr, &alloc_out);
        break;
    case Step::N_CONV: {
        DT r, sc;
        const DT *rp = nullptr, *sp = nullptr;
        if (!s.residual.empty()) {
            r = getf(vals, s.residual);
            rp = &r;
        }
        if (!s.scale.empty()) {
            sc = getf(vals, s.scale);
            sp = &sc;
        }
        DT x = getf(vals, s.inputs[0]);
        if (x.rank() != 4) fail(WOCR_ERR_SHAPE, "Conv input " + shape_str(x.shape));
        out.f = conv_run(ctx, x, s.conv, s.act, rp, sp, &alloc_out);
        break;
    }
    case Step::G_CONVT:
    case Step::N_CONVT: {
        DT x = getx(vals, s.inputs[0]);
        if (x.rank() != 4) fail(WOCR_ERR_SHAPE, "ConvTranspose input " + shape_str(x.shape));
        out.f = convt_run(ctx, x, s.convt, s.act, &alloc_out);
        break;
    }
    case Step::G_MAXPOOL: {
        if (s.pool_fused_away) return;  // computed by the producing convolution's epilogue
        out.f = maxpool_run(ctx, getx(vals, s.inputs[0]), s.conv.kh, s.conv.kw, s.split_out);
        break;
    }
    case Step::G_SLICE: {
        // 4-D box (src/gpu.rs:1303-1315)
        DT a = getx(vals, s.inputs[0]);
        if (a.rank() != 4) fail(WOCR_ERR_SHAPE, "Slice input " + shape_str(a.shape));
        std::vector<int64_t> lo(4, 0), shp = a.shape;
        for (size_t q = 0; q < s.starts.size() && q < s.ends.size() && q < s.axes.size(); q++) {
            int64_t ax = s.axes[q] < 0 ? s.axes[q] + 4 : s.axes[q];
            if (ax < 0 || ax >= 4) fail(WOCR_ERR_SHAPE, "Slice axis out of range");
            int64_t dim = a.shape[ax];
            auto cl = [&](int64_t v) { return std::min(std::max(v < 0 ? v + dim : v, (int64_t)0), dim); };
            int64_t s0 = cl(s.starts[q]), e0 = cl(s.ends[q]);
            lo[ax] = s0;
            shp[ax] = std::max<int64_t>(e0 - s0, 0);
        }
        int64_t off = 0;
        for (int d = 0; d < 4; d++) off += lo[d] * a.strides[d];
        out.f = view(a, shp, a.strides, off);
        break;
    }
    case Step::G_CONCAT: {
        std::vector<DT> parts;
        for (auto &nm : s.inputs) parts.push_back(getx(vals, nm));
        DT a = parts[0];
        int64_t ctot = 0;
        for (auto &t : parts) {
            if (t.rank() != 4 || t.shape[0] != a.shape[0] || t.shape[2] != a.shape[2] || t.shape[3] != a.shape[3]) {
                std::string m = "Concat shapes differ:";
                for (auto &q : parts) m += " " + shape_str(q.shape);
                fail(WOCR_ERR_SHAPE, m);
            }
            ctot += t.shape[1];
        }
        out.f = concat_channels(parts, s.output, s.split_out);
        break;
    }
    case Step::G_ACT: {
        DT x = getf(vals, s.inputs[0]);
        if (!x.dense()) x = to_rowmajor(ctx, x);
        DT y = x;
        y.buf = alloc(ctx, (size_t)std::max<int64_t>(x.numel(), 1) * sizeof(float));
        y.p = (float *)y.buf->p;
        // dense input: the minimum-stride element is at p, output shares the strides
        k::unary(ctx, s.act, x.p, y.p, x.numel(), 0.2f, 0.5f);
        out.f = y;
        break;
    }
    case Step::G_IDENTITY:
        if (s.head_fused_away) return;  // between a convolution and the head fused into it
        out = get(vals, s.inputs[0]);
        break;
    case Step::N_LINEAR:
        out.f = linear_run(ctx, getf(vals, s.inputs[0]), s.lw, s.lb, s.lk, s.ln, s.ldw, s.act, s.luw.get());
        break;
    case Step::N_AFFINE: {
        DT x = getf(vals, s.inputs[0]);
        if (!x.dense()) x = to_rowmajor(ctx, x);
        int64_t C = x.rank() > 1 ? x.shape[1] : 1;
        if (C * 2 != s.st.n) fail(WOCR_ERR_SHAPE, "BatchNormalization over " + shape_str(x.shape));
        DT y = x;
        y.buf = alloc(ctx, (size_t)std::max<int64_t>(x.numel(), 1) * sizeof(float));
        y.p = (float *)y.buf->p;
        int64_t cdiv = x.rank() > 1 && C > 1 ? x.strides[1] : 1;
        k::affine(ctx, x.p, y.p, x.numel(), (int)C, cdiv, s.st.p);
        out.f = y;
        break;
    }
    case Step::N_LAYERNORM: {
        DT x = getf(vals, s.inputs[0]);
        if (x.shape.empty() || x.shape.back() != s.ln_len)
            fail(WOCR_ERR_SHAPE, "LayerNorm over " + shape_str(x.shape) + ", expects " + std::to_string(s.ln_len));
        x = to_rowmajor(ctx, x);
        DT y = new_rowmajor(ctx, x.shape);
        k::layer_norm(ctx, x.p, y.p, x.numel() / s.ln_len, s.ln_len, s.st.p, s.eps);
        out.f = y;
        break;
    }
    case Step::N_GENERIC:
        exec_generic(model.nodes[s.node], vals);
        return;
    }
    vals[s.output] = out;
}

// ---- N-D generic nodes (src/nd.rs:888-1164) -------------------------------------------------
static int64_t axis_of(int64_t a, int64_t rank) {
    int64_t r = a < 0 ? a + rank : a;
    if (r < 0 || r >= std::max<int64_t>(rank, 1))
        fail(WOCR_ERR_SHAPE, "axis " + std::to_string(a) + " out of range for rank " + std::to_string(rank));
    return r;
}

static void pads_of(const Node &n, int64_t h, int64_t w, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t &pt,
                    int64_t &pl, int64_t &pb, int64_t &pr) {
    if (n.str("auto_pad").value_or("") == "SAME_UPPER") {
        int64_t oh = (h + sh - 1) / sh, ow = (w + sw - 1) / sw;
        int64_t th = std::max<int64_t>((oh - 1) * sh + kh - h, 0);
        int64_t tw = std::max<int64_t>((ow - 1) * sw + kw - w, 0);
        pt = th / 2, pl = tw / 2, pb = th - th / 2, pr = tw - tw / 2;
    } else {
        auto p = n.ints("pads").value_or(std::vector<int64_t>{0, 0, 0, 0});
        if (p.size() < 4) p.resize(4, 0);
        pt = p[0], pl = p[1], pb = p[2], pr = p[3];
    }
}

void Executor::exec_generic(const Node &n, std::map<std::string, Value> &vals) {
    const std::string &op = n.op;
    Value out;
    auto ints_of = [&](size_t k) -> std::vector<int64_t> {
        Value v = get(vals, n.in(k));
        if (!v.is_int) fail(WOCR_ERR_SHAPE, op + ": input " + std::to_string(k) + " is not an integer constant");
        return v.iv;
    };
    if (op == "Resize") {
        DT a = getf(vals, n.in(0));
        if (n.str("mode").value_or("") != "nearest" ||
            n.str("coordinate_transformation_mode").value_or("") != "asymmetric")
            fail(WOCR_ERR_UNSUPPORTED, "Resize other than nearest/asymmetric");
        auto sw = model.weights.find(n.in(2));
        if (sw == model.weights.end() || sw->second.data.size() > 8) fail(WOCR_ERR_MISSING, "Resize scales");
        const auto &sc = sw->second.data;
        if (a.rank() != 4) fail(WOCR_ERR_SHAPE, "Resize input " + shape_str(a.shape));
        if (sc.size() != 4 || sc[0] != 1.0f || sc[1] != 1.0f) fail(WOCR_ERR_UNSUPPORTED, "Resize scales");
        a = to_nhwc(ctx, a);
        int64_t nb = a.shape[0], ch = a.shape[1], h = a.shape[2], w = a.shape[3];
        int64_t oh = (int64_t)std::floor((float)h * sc[2]), ow = (int64_t)std::floor((float)w * sc[3]);
        DT y = new_nhwc(ctx, nb, ch, oh, ow);
        k::resize_nearest(ctx, a.p, a.strides[0], a.pix(), (int)nb, (int)h, (int)w, (int)ch, (int)oh, (int)ow, sc[2],
                          sc[3], y.p, y.strides[0], y.pix());
        out.f = y;
    } else if (op == "GlobalAveragePool") {
        DT a = getf(vals, n.in(0));
        if (a.rank() < 3) fail(WOCR_ERR_SHAPE, "GlobalAveragePool on " + shape_str(a.shape));
        std::vector<int64_t> shape = a.shape;
        for (size_t d = 2; d < shape.size(); d++) shape[d] = 1;
        DT y = new_rowmajor(ctx, shape);
        if (a.rank() == 4 && a.nhwc()) {
            k::gap(ctx, a.p, a.strides[0], a.pix(), (int)a.shape[0], (int)(a.shape[2] * a.shape[3]), (int)a.shape[1],
                   y.p);
        } else {
            a = to_rowmajor(ctx, a);
            int64_t inner = 1;
            for (size_t d = 2; d < a.shape.size(); d++) inner *= a.shape[d];
            k::reduce_mean(ctx, a.p, y.p, a.numel() / std::max<int64_t>(inner, 1), inner);
        }
        out.f = y;
    } else if (op == "MatMul") {
        DT a = getf(vals, n.in(0)), b = getf(vals, n.in(1));
        int r = a.rank();
        bool ok = r >= 2 && b.rank() == r && a.shape[r - 1] == b.shape[r - 2];
        for (int d = 0; ok && d < r - 2; d++) ok = a.shape[d] == b.shape[d];
        if (!ok) fail(WOCR_ERR_SHAPE, "MatMul shapes " + shape_str(a.shape) + " x " + shape_str(b.shape));
        int64_t m = a.shape[r - 2], kk = a.shape[r - 1], nn = b.shape[r - 1];
        int64_t batch = 1;
        for (int d = 0; d < r - 2; d++) batch *= a.shape[d];
        a = to_rowmajor(ctx, a);
        b = to_rowmajor(ctx, b);
        std::vector<int64_t> shape = a.shape;
        shape[r - 1] = nn;
        DT y = new_rowmajor(ctx, shape);
        k::bmm(ctx, a.p, b.p, y.p, batch, (int)m, (int)kk, (int)nn);
        ctx->flops += 2.0 * batch * m * kk * nn;
        out.f = y;
    } else if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div" || op == "Pow") {
        Value va = get(vals, n.in(0)), vb = get(vals, n.in(1));
        if (va.is_int && vb.is_int) {
            auto f = [&](int64_t x, int64_t y) -> int64_t {
                if (op == "Add") return x + y;
                if (op == "Sub") return x - y;
                if (op == "Mul") return x * y;
                if (op == "Div") return y == 0 ? 0 : x / y;
                return x;
            };
            std::vector<int64_t> v;
            if (vb.iv.size() == 1)
                for (auto x : va.iv) v.push_back(f(x, vb.iv[0]));
            else
                for (size_t i = 0; i < std::min(va.iv.size(), vb.iv.size()); i++) v.push_back(f(va.iv[i], vb.iv[i]));
            out.is_int = true;
            out.iv = v;
            out.ishape = va.ishape;
        } else if (va.is_int || vb.is_int) {
            fail(WOCR_ERR_SHAPE, op + ": mixed integer and float inputs");
        } else {
            DT a = va.f, b = vb.f;
            int r = std::max(a.rank(), b.rank());
            if (r > kMaxRank) fail(WOCR_ERR_UNSUPPORTED, "rank " + std::to_string(r) + " > 6");
            std::vector<int64_t> sa(r, 1), sb(r, 1), ta(r, 0), tb(r, 0);
            for (int d = 0; d < a.rank(); d++) sa[r - a.rank() + d] = a.shape[d], ta[r - a.rank() + d] = a.strides[d];
            for (int d = 0; d < b.rank(); d++) sb[r - b.rank() + d] = b.shape[d], tb[r - b.rank() + d] = b.strides[d];
            std::vector<int64_t> shape(r);
            for (int d = 0; d < r; d++) {
                if (sa[d] != sb[d] && sa[d] != 1 && sb[d] != 1)
                    fail(WOCR_ERR_SHAPE, op + ": shapes " + shape_str(a.shape) + " and " + shape_str(b.shape) +
                                             " do not broadcast");
                shape[d] = std::max(sa[d], sb[d]);
                if (sa[d] == 1) ta[d] = 0;
                if (sb[d] == 1) tb[d] = 0;
            }
            // keep a channels-last layout when a full-size operand has it
            bool nh = r == 4 && ((a.shape == shape && a.nhwc() && a.shape[1] > 1) ||
                                 (b.shape == shape && b.nhwc() && b.shape[1] > 1));
            DT y = nh ? new_nhwc(ctx, shape[0], shape[1], shape[2], shape[3]) : new_rowmajor(ctx, shape);
            k::Strided st;
            st.rank = r;
            for (int d = 0; d < r; d++) {
                st.dims[d] = shape[d];
                st.xs[d] = ta[d];
                st.bs[d] = tb[d];
                st.ys[d] = y.strides[d];
            }
            int code = op == "Add" ? 0 : op == "Sub" ? 1 : op == "Mul" ? 2 : op == "Div" ? 3 : 4;
            k::binary(ctx, code, a.p, b.p, y.p, st);
            out.f = y;
        }
    } else if (op == "Relu" || op == "Sigmoid" || op == "HardSigmoid" || op == "Erf" || op == "Sqrt") {
        DT x = getf(vals, n.in(0));
        if (!x.dense()) x = to_rowmajor(ctx, x);
        int code = op == "Relu" ? 1 : op == "Sigmoid" ? 2 : op == "HardSigmoid" ? 3 : op == "Erf" ? 4 : 5;
        DT y = x;
        y.buf = alloc(ctx, (size_t)std::max<int64_t>(x.numel(), 1) * sizeof(float));
        y.p = (float *)y.buf->p;
        k::unary(ctx, code, x.p, y.p, x.numel(), n.f32("alpha").value_or(0.2f), n.f32("beta").value_or(0.5f));
        out.f = y;
    } else if (op == "ReduceMean") {
        DT a = getf(vals, n.in(0));
        int64_t r = a.rank();
        std::vector<int64_t> axes;
        auto ax = n.ints("axes");
        if (ax)
            for (auto v : *ax) axes.push_back(axis_of(v, r));
        else
            for (int64_t d = 0; d < r; d++) axes.push_back(d);
        std::sort(axes.begin(), axes.end());
        for (size_t k2 = 0; k2 < axes.size(); k2++)
            if (axes[k2] != r - (int64_t)axes.size() + (int64_t)k2)
                fail(WOCR_ERR_UNSUPPORTED, "ReduceMean over non-trailing axes");
        int64_t inner = 1;
        for (auto d : axes) inner *= a.shape[d];
        bool keep = n.int_("keepdims").value_or(1) == 1;
        std::vector<int64_t> shape;
        for (int64_t d = 0; d < r; d++) {
            bool red = std::find(axes.begin(), axes.end(), d) != axes.end();
            if (!red) shape.push_back(a.shape[d]);
            else if (keep) shape.push_back(1);
        }
        a = to_rowmajor(ctx, a);
        DT y = new_rowmajor(ctx, shape);
        k::reduce_mean(ctx, a.p, y.p, a.numel() / std::max<int64_t>(inner, 1), inner);
        out.f = y;
    } else if (op == "Softmax") {
        DT a = getf(vals, n.in(0));
        int64_t ax = axis_of(n.int_("axis").value_or(-1), a.rank());
        int64_t len = 1;
        for (int64_t d = ax; d < a.rank(); d++) len *= a.shape[d];
        a = to_rowmajor(ctx, a);
        DT y = new_rowmajor(ctx, a.shape);
        k::softmax(ctx, a.p, y.p, a.numel() / std::max<int64_t>(len, 1), len);
        out.f = y;
    } else if (op == "Transpose") {
        DT a = getf(vals, n.in(0));
        int r = a.rank();
        std::vector<int64_t> perm;
        auto pv = n.ints("perm");
        if (pv) perm = *pv;
        else
            for (int d = r - 1; d >= 0; d--) perm.push_back(d);
        if ((int)perm.size() != r) fail(WOCR_ERR_SHAPE, "Transpose perm of rank " + std::to_string(perm.size()));
        std::vector<int64_t> shape(r), strides(r);
        for (int d = 0; d < r; d++) {
            if (perm[d] < 0 || perm[d] >= r) fail(WOCR_ERR_SHAPE, "Transpose perm out of range");
            shape[d] = a.shape[perm[d]];
            strides[d] = a.strides[perm[d]];
        }
        out.f = view(a, shape, strides);
    } else if (op == "Slice") {
        std::vector<int64_t> starts = ints_of(1), ends = ints_of(2);
        Value data = get(vals, n.in(0));
        std::vector<int64_t> shape = data.is_int ? data.ishape : data.f.shape;
        int64_t r = (int64_t)shape.size();
        std::vector<int64_t> axes;
        if (n.inputs.size() > 3 && !n.inputs[3].empty()) axes = ints_of(3);
        else
            for (size_t q = 0; q < starts.size(); q++) axes.push_back((int64_t)q);
        if (n.inputs.size() > 4 && !n.inputs[4].empty()) {
            for (auto st : ints_of(4))
                if (st != 1) fail(WOCR_ERR_UNSUPPORTED, "Slice with steps");
        }
        std::vector<int64_t> lo(r, 0), oshape = shape;
        for (size_t q = 0; q < starts.size() && q < ends.size() && q < axes.size(); q++) {
            int64_t a = axis_of(axes[q], r);
            int64_t dim = shape[a];
            auto cl = [&](int64_t v) { return std::min(std::max(v < 0 ? v + dim : v, (int64_t)0), dim); };
            int64_t s0 = cl(starts[q]), e0 = cl(ends[q]);
            lo[a] = s0;
            oshape[a] = std::max<int64_t>(e0 - s0, 0);
        }
        if (data.is_int) {
            out.is_int = true;
            int64_t a0 = lo.empty() ? 0 : lo[0], n0 = oshape.empty() ? 0 : oshape[0];
            for (int64_t q = a0; q < a0 + n0 && q < (int64_t)data.iv.size(); q++) out.iv.push_back(data.iv[q]);
            out.ishape = oshape;
        } else {
            int64_t off = 0;
            for (int64_t d = 0; d < r; d++) off += lo[d] * data.f.strides[d];
            out.f = view(data.f, oshape, data.f.strides, off);
        }
    } else if (op == "Concat") {
        std::vector<Value> parts;
        for (size_t k2 = 0; k2 < n.inputs.size(); k2++) parts.push_back(get(vals, n.inputs[k2]));
        bool all_int = std::all_of(parts.begin(), parts.end(), [](const Value &v) { return v.is_int; });
        if (all_int) {
            out.is_int = true;
            for (auto &p : parts) out.iv.insert(out.iv.end(), p.iv.begin(), p.iv.end());
            out.ishape = {(int64_t)out.iv.size()};
        } else {
            for (auto &p : parts)
                if (p.is_int) fail(WOCR_ERR_SHAPE, "Concat of mixed values");
            int64_t r = parts[0].f.rank();
            int64_t ax = axis_of(n.int_("axis").value_or(0), r);
            std::vector<int64_t> shape = parts[0].f.shape;
            shape[ax] = 0;
            for (auto &p : parts) {
                if (p.f.rank() != r) fail(WOCR_ERR_SHAPE, "Concat ranks differ");
                shape[ax] += p.f.shape[ax];
            }
            bool nh = r == 4 && ax == 1;
            if (nh) {
                std::vector<DT> ts;
                for (auto &p : parts) ts.push_back(p.f);
                out.f = concat_channels(ts, n.outputs[0], false);
                vals[n.outputs[0]] = out;
                return;
            }
            DT y = nh ? new_nhwc(ctx, shape[0], shape[1], shape[2], shape[3]) : new_rowmajor(ctx, shape);
            int64_t off = 0;
            for (auto &p : parts) {
                DT dst = view(y, p.f.shape, y.strides, off * y.strides[ax]);
                copy_into(ctx, p.f, dst);
                off += p.f.shape[ax];
            }
            out.f = y;
        }
    } else if (op == "MaxPool" || op == "AveragePool") {
        DT a = getf(vals, n.in(0));
        if (a.rank() != 4) fail(WOCR_ERR_SHAPE, "pool input " + shape_str(a.shape));
        auto kv = n.ints("kernel_shape");
        if (!kv || kv->size() < 2) fail(WOCR_ERR_UNSUPPORTED, "pool without kernel_shape");
        auto sv = n.ints("strides").value_or(std::vector<int64_t>{1, 1});
        if (n.int_("ceil_mode").value_or(0) != 0) fail(WOCR_ERR_UNSUPPORTED, "pool with ceil_mode");
        if (op == "AveragePool" && n.int_("count_include_pad").value_or(0) != 0)
            fail(WOCR_ERR_UNSUPPORTED, "AveragePool counting padding");
        a = to_nhwc(ctx, a);
        int64_t nb = a.shape[0], ch = a.shape[1], h = a.shape[2], w = a.shape[3];
        int64_t kh = (*kv)[0], kw = (*kv)[1], sh = sv[0], sw = sv[1];
        int64_t pt, pl, pb, pr;
        pads_of(n, h, w, kh, kw, sh, sw, pt, pl, pb, pr);
        if (h + pt + pb < kh || w + pl + pr < kw) fail(WOCR_ERR_SHAPE, "pool input " + shape_str(a.shape));
        int64_t oh = (h + pt + pb - kh) / sh + 1, ow = (w + pl + pr - kw) / sw + 1;
        DT y = new_nhwc(ctx, nb, ch, oh, ow);
        k::pool(ctx, a.p, a.strides[0], a.pix(), (int)nb, (int)h, (int)w, (int)ch, (int)kh, (int)kw, (int)sh, (int)sw,
                (int)pt, (int)pl, (int)oh, (int)ow, op == "AveragePool", y.p, y.strides[0], y.pix());
        out.f = y;
    } else if (op == "Reshape") {
        DT a = getf(vals, n.in(0));
        std::vector<int64_t> want = ints_of(1);
        int64_t total = a.numel();
        std::vector<int64_t> shape(want.size());
        for (size_t d = 0; d < want.size(); d++)
            shape[d] = want[d] == 0 ? (d < a.shape.size() ? a.shape[d] : 1) : std::max<int64_t>(want[d], 1);
        auto neg = std::find(want.begin(), want.end(), -1);
        if (neg != want.end()) {
            size_t p = neg - want.begin();
            int64_t known = 1;
            for (size_t d = 0; d < shape.size(); d++)
                if (d != p) known *= shape[d];
            shape[p] = total / std::max<int64_t>(known, 1);
        }
        int64_t prod = 1;
        for (auto s : shape) prod *= s;
        if (prod != total) fail(WOCR_ERR_SHAPE, "Reshape " + shape_str(a.shape) + " to " + shape_str(want));
        a = to_rowmajor(ctx, a);
        out.f = view(a, shape, rowmajor_strides(shape));
    } else if (op == "Squeeze" || op == "Unsqueeze") {
        std::vector<int64_t> axes;
        auto av = n.ints("axes");
        if (av) axes = *av;
        else axes = ints_of(1);
        Value v = get(vals, n.in(0));
        if (v.is_int) {
            out = v;
            if (op == "Squeeze") {
                std::vector<int64_t> s;
                for (auto d : v.ishape)
                    if (d != 1) s.push_back(d);
                out.ishape = s;
            } else {
                out.ishape = {(int64_t)v.iv.size()};
            }
        } else {
            DT a = v.f;
            std::vector<int64_t> shape, strides;
            if (op == "Squeeze") {
                std::vector<int64_t> ax;
                for (auto x : axes) ax.push_back(axis_of(x, a.rank()));
                for (int d = 0; d < a.rank(); d++)
                    if (std::find(ax.begin(), ax.end(), d) == ax.end()) {
                        shape.push_back(a.shape[d]);
                        strides.push_back(a.strides[d]);
                    }
            } else {
                int64_t r = a.rank() + (int64_t)axes.size();
                std::vector<int64_t> ax;
                for (auto x : axes) ax.push_back(axis_of(x, r));
                int src = 0;
                for (int64_t d = 0; d < r; d++) {
                    if (std::find(ax.begin(), ax.end(), d) != ax.end()) {
                        shape.push_back(1);
                        strides.push_back(0);
                    } else {
                        shape.push_back(src < a.rank() ? a.shape[src] : 1);
                        strides.push_back(src < a.rank() ? a.strides[src] : 0);
                        src++;
                    }
                }
            }
            out.f = view(a, shape, strides);
        }
    } else if (op == "Shape") {
        Value v = get(vals, n.in(0));
        std::vector<int64_t> s = v.is_int ? v.ishape : v.f.shape;
        out.is_int = true;
        out.iv = s;
        out.ishape = {(int64_t)s.size()};
    } else if (op == "Gather") {
        std::vector<int64_t> data = ints_of(0), idx = ints_of(1);
        out.is_int = true;
        for (auto i : idx) {
            int64_t j = i < 0 ? i + (int64_t)data.size() : i;
            out.iv.push_back(j >= 0 && j < (int64_t)data.size() ? data[j] : 0);
        }
        out.ishape = out.iv.size() == 1 ? std::vector<int64_t>{} : std::vector<int64_t>{(int64_t)out.iv.size()};
    } else if (op == "Cast") {
        out = get(vals, n.in(0));
    } else if (op == "Identity") {
        out = get(vals, n.in(0));
    } else {
        fail(WOCR_ERR_UNSUPPORTED, "unsupported op " + op);
    }
    vals[n.outputs[0]] = out;
}

// =========================================================================================
// Graph::build (src/gpu.rs:1104-1240)
// =========================================================================================
static int act_of(const std::string &op) { return op == "Relu" ? 1 : op == "Sigmoid" ? 2 : 0; }

// One value of a symmetric 2-D attribute (src/gpu.rs:1111-1118).
static int64_t symmetric(const Node &n, const std::string &name, int64_t dflt) {
    auto v = n.ints(name);
    if (!v || v->empty()) return dflt;
    for (auto x : *v)
        if (x != (*v)[0] || x < 0) fail(WOCR_ERR_UNSUPPORTED, n.op + ": asymmetric " + name);
    return (*v)[0];
}

static std::vector<float> bias_or_zero(const Model &m, const Node &n, size_t idx, int count) {
    if (idx < n.inputs.size() && !n.inputs[idx].empty()) return m.weight(n.inputs[idx]).data;
    return std::vector<float>(count, 0.f);
}

std::unique_ptr<Executor> build_graph(Ctx *c, const Model &m, const char *stop, Node *stop_node) {
    auto ex = std::make_unique<Executor>(c);
    ex->model = m;
    const auto &nodes = m.nodes;
    bool stopped = false;
    Node sn;
    size_t i = 0;
    while (i < nodes.size()) {
        const Node &n = nodes[i];
        if (stop && n.op == stop) {
            sn = n;
            stopped = true;
            break;
        }
        std::string output = n.outputs[0];
        int fused = 0;
        if ((n.op == "Conv" || n.op == "ConvTranspose") && i + 1 < nodes.size()) {
            const Node &next = nodes[i + 1];
            if (act_of(next.op) && !next.inputs.empty() && next.inputs[0] == output && m.readers(output) == 1) {
                fused = act_of(next.op);
                output = next.outputs[0];
                i++;
            }
        }
        Step st;
        st.output = output;
        st.inputs = {n.in(0)};
        if (n.op == "Conv") {
            const HostW &w = m.weight(n.in(1));
            if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "conv weight not 4D");
            int cout = (int)w.dims[0], cin_g = (int)w.dims[1];
            int group = (int)n.int_("group").value_or(1);
            if (symmetric(n, "dilations", 1) != 1) fail(WOCR_ERR_UNSUPPORTED, "dilated conv");
            int pad = (int)symmetric(n, "pads", 0), stride = (int)symmetric(n, "strides", 1);
            std::vector<float> b = bias_or_zero(m, n, 2, cout);
            if (group == 1 && cin_g == 1 && stride == 1) {
                st.kind = Step::G_DIRECT;
                st.conv = lower_conv_direct(c, w, b);
                // a MaxPool right after, reading only this output, is fused in (src/gpu.rs:1146-1159)
                if (i + 1 < nodes.size()) {
                    const Node &next = nodes[i + 1];
                    auto kv = next.ints("kernel_shape");
                    auto sv = next.ints("strides");
                    if (next.op == "MaxPool" && !next.inputs.empty() && next.inputs[0] == output &&
                        m.readers(output) == 1 && kv && kv->size() >= 2 && (!sv || *sv == *kv) &&
                        symmetric(next, "pads", 0) == 0 && next.int_("ceil_mode").value_or(0) == 0) {
                        st.conv.pool_h = (int)(*kv)[0];
                        st.conv.pool_w = (int)(*kv)[1];
                        output = next.outputs[0];
                        st.output = output;
                        i++;
                    }
                }
            } else if (group == 1) {
                st.kind = Step::G_CONV;
                st.conv = lower_conv_dense(c, w, b, 1);
            } else if (cin_g == 1 && group == cout) {
                st.kind = Step::G_DEPTHWISE;
                st.conv = lower_conv_dense(c, w, b, group);
            } else {
                fail(WOCR_ERR_UNSUPPORTED, "grouped conv with group " + std::to_string(group));
            }
            st.conv.sh = st.conv.sw = stride;
            for (int q = 0; q < 4; q++) st.conv.pads[q] = pad;
            if (st.kind == Step::G_CONV && stride == 1 && cin_g >= 16 && use_umma()) attach_tconv(c, st.conv, w);
            st.act = fused;
        } else if (n.op == "ConvTranspose") {
            const HostW &w = m.weight(n.in(1));
            if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "convT weight not 4D");
            if (n.int_("group").value_or(1) != 1 || symmetric(n, "pads", 0) != 0 ||
                symmetric(n, "output_padding", 0) != 0)
                fail(WOCR_ERR_UNSUPPORTED, "unsupported ConvTranspose attributes");
            st.kind = Step::G_CONVT;
            st.convt = lower_convt(c, w, bias_or_zero(m, n, 2, (int)w.dims[1]), (int)symmetric(n, "strides", 1));
            if (st.convt.gemm && st.convt.cin >= 16 && use_umma()) attach_tconv(c, st.convt, w);
            st.act = fused;
        } else if (n.op == "MaxPool") {
            auto kv = n.ints("kernel_shape");
            if (!kv || kv->size() < 2) fail(WOCR_ERR_UNSUPPORTED, "MaxPool without kernel_shape");
            auto sv = n.ints("strides").value_or(*kv);
            if (sv != *kv || symmetric(n, "pads", 0) != 0 || n.int_("ceil_mode").value_or(0) != 0)
                fail(WOCR_ERR_UNSUPPORTED, "unsupported MaxPool attributes");
            st.kind = Step::G_MAXPOOL;
            st.conv.kh = (int)(*kv)[0];
            st.conv.kw = (int)(*kv)[1];
        } else if (n.op == "Slice") {
            auto get = [&](size_t idx) -> const std::vector<int64_t> * {
                if (idx >= n.inputs.size()) return nullptr;
                auto it = m.ints.find(n.inputs[idx]);
                return it == m.ints.end() ? nullptr : &it->second;
            };
            if (auto stp = get(4))
                for (auto v : *stp)
                    if (v != 1) fail(WOCR_ERR_UNSUPPORTED, "Slice with steps");
            if (!get(1)) fail(WOCR_ERR_UNSUPPORTED, "Slice starts not constant");
            if (!get(2)) fail(WOCR_ERR_UNSUPPORTED, "Slice ends not constant");
            st.kind = Step::G_SLICE;
            st.starts = *get(1);
            st.ends = *get(2);
            if (get(3)) st.axes = *get(3);
            else
                for (size_t q = 0; q < st.starts.size(); q++) st.axes.push_back((int64_t)q);
        } else if (n.op == "Concat") {
            if (n.int_("axis").value_or(-999) != 1) fail(WOCR_ERR_UNSUPPORTED, "Concat not on channels");
            st.kind = Step::G_CONCAT;
            st.inputs = n.inputs;
        } else if (n.op == "Pad") {
            bool nonzero = false;
            if (n.inputs.size() > 1) {
                auto it = m.ints.find(n.inputs[1]);
                if (it != m.ints.end()) {
                    for (auto v : it->second) nonzero |= v != 0;
                } else {
                    auto wt = m.weights.find(n.inputs[1]);
                    if (wt != m.weights.end())
                        for (auto v : wt->second.data) nonzero |= (int64_t)v != 0;
                }
            }
            if (nonzero) fail(WOCR_ERR_UNSUPPORTED, "non-zero Pad");
            st.kind = Step::G_IDENTITY;
        } else if (act_of(n.op)) {
            st.kind = Step::G_ACT;
            st.act = act_of(n.op);
        } else {
            fail(WOCR_ERR_UNSUPPORTED, "unsupported op " + n.op);
        }
        ex->steps.push_back(st);
        i++;
    }
    ex->input = m.input;
    ex->output = stopped ? sn.in(0) : m.output;
    ex->allow_split = use_umma() && !std::getenv("WOCR_NO_SPLIT");
    if (stop_node && stopped) *stop_node = sn;
    if (stop && !stopped && stop_node) stop_node->op.clear();
    ex->finalize();
    return ex;
}

// =========================================================================================
// NdGraph::new (src/nd.rs:505-817)
// =========================================================================================
std::unique_ptr<Executor> build_ndgraph(Ctx *c, const Model &m, bool stop_before_softmax) {
    auto ex = std::make_unique<Executor>(c);
    // Identity nodes: every reader reads their input instead
    std::map<std::string, std::string> alias;
    for (auto &n : m.nodes)
        if (n.op == "Identity" && !n.inputs.empty()) {
            auto it = alias.find(n.inputs[0]);
            alias[n.outputs[0]] = it != alias.end() ? it->second : n.inputs[0];
        }
    auto resolve = [&](const std::string &s) {
        auto it = alias.find(s);
        return it != alias.end() ? it->second : s;
    };
    std::vector<Node> nodes;
    for (auto &n : m.nodes) {
        if (n.op == "Identity") continue;
        Node q = n;
        for (auto &i : q.inputs) i = resolve(i);
        nodes.push_back(q);
    }
    std::string output = resolve(m.output);
    if (stop_before_softmax) {
        int last = -1;
        for (int k2 = (int)nodes.size() - 1; k2 >= 0; k2--)
            if (!nodes[k2].outputs.empty() && nodes[k2].outputs[0] == output) {
                last = k2;
                break;
            }
        if (last >= 0 && nodes[last].op == "Softmax") {
            output = nodes[last].in(0);
            nodes.resize(last);
        }
    }
    auto scalar = [&](const std::string &name) -> std::optional<float> {
        auto it = m.weights.find(name);
        if (it == m.weights.end() || it->second.data.size() != 1) return std::nullopt;
        return it->second.data[0];
    };
    auto is_weight = [&](const std::string &name) { return m.weights.count(name) > 0; };
    std::vector<bool> skip(nodes.size(), false);
    auto count_readers = [&]() {
        std::map<std::string, int> cnt;
        for (size_t k2 = 0; k2 < nodes.size(); k2++)
            if (!skip[k2])
                for (auto &i : nodes[k2].inputs) cnt[i]++;
        return cnt;
    };
    std::map<std::string, int> counts = count_readers();
    auto readers = [&](const std::string &name) {
        auto it = counts.find(name);
        return (it == counts.end() ? 0 : it->second) + (name == output ? 1 : 0);
    };
    // Squeeze-excitation: Mul(x, s) read only by a dense Conv becomes its input scale
    std::map<size_t, std::string> in_scale;
    struct SE {
        size_t mi, ci;
        std::string x, sc;
    };
    std::vector<SE> se;
    for (size_t mi = 0; mi < nodes.size(); mi++) {
        const Node &mn = nodes[mi];
        if (mn.op != "Mul" || readers(mn.outputs[0]) != 1 || mn.inputs.size() < 2) continue;
        size_t ci = nodes.size();
        for (size_t q = 0; q < nodes.size(); q++)
            if (nodes[q].op == "Conv" && nodes[q].in(0) == mn.outputs[0] && nodes[q].int_("group").value_or(1) == 1) {
                ci = q;
                break;
            }
        if (ci == nodes.size()) continue;
        auto gate = [&](const std::string &name) {
            for (auto &g : nodes)
                if (g.op == "HardSigmoid" && g.outputs[0] == name) return true;
            return false;
        };
        if (gate(mn.inputs[1])) se.push_back({mi, ci, mn.inputs[0], mn.inputs[1]});
        else if (gate(mn.inputs[0])) se.push_back({mi, ci, mn.inputs[1], mn.inputs[0]});
    }
    for (auto &e : se) {
        in_scale[e.ci] = e.sc;
        skip[e.mi] = true;
        nodes[e.ci].inputs[0] = e.x;
    }
    counts = count_readers();

    std::vector<std::pair<size_t, std::string>> renames;
    std::vector<Step> steps;
    size_t i = 0;
    while (i < nodes.size()) {
        if (skip[i]) {
            i++;
            continue;
        }
        const Node &n = nodes[i];
        // LayerNorm: ReduceMean, Sub, Pow 2, ReduceMean, Add eps, Sqrt, Div, Mul gamma, Add beta
        if (n.op == "ReduceMean" && i + 9 <= nodes.size()) {
            const Node &mean = nodes[i], &sub = nodes[i + 1], &pw = nodes[i + 2], &var = nodes[i + 3],
                       &add = nodes[i + 4], &sq = nodes[i + 5], &dv = nodes[i + 6], &mul = nodes[i + 7],
                       &beta = nodes[i + 8];
            auto axes_last = [](const Node &q) {
                auto a = q.ints("axes");
                return a && a->size() == 1 && (*a)[0] == -1;
            };
            bool ok = axes_last(n) && sub.op == "Sub" && sub.in(0) == mean.in(0) && sub.in(1) == mean.outputs[0] &&
                      pw.op == "Pow" && pw.in(0) == sub.outputs[0] && scalar(pw.in(1)) == 2.0f &&
                      var.op == "ReduceMean" && var.in(0) == pw.outputs[0] && axes_last(var) && add.op == "Add" &&
                      add.in(0) == var.outputs[0] && scalar(add.in(1)).has_value() && sq.op == "Sqrt" &&
                      sq.in(0) == add.outputs[0] && dv.op == "Div" && dv.in(0) == sub.outputs[0] &&
                      dv.in(1) == sq.outputs[0] && mul.op == "Mul" && mul.in(0) == dv.outputs[0] &&
                      is_weight(mul.in(1)) && beta.op == "Add" && beta.in(0) == mul.outputs[0] &&
                      is_weight(beta.in(1)) && readers(mean.outputs[0]) == 1 && readers(sub.outputs[0]) == 2;
            for (auto *o : {&pw.outputs[0], &var.outputs[0], &add.outputs[0], &sq.outputs[0], &dv.outputs[0],
                            &mul.outputs[0]})
                ok = ok && readers(*o) == 1;
            if (ok) {
                const HostW &g = m.weight(mul.in(1)), &b = m.weight(beta.in(1));
                std::vector<float> gb = g.data;
                gb.insert(gb.end(), b.data.begin(), b.data.end());
                Step st;
                st.kind = Step::N_LAYERNORM;
                st.st = upload(c, gb);
                st.ln_len = (int)g.data.size();
                st.eps = scalar(add.in(1)).value_or(1e-5f);
                st.inputs = {n.in(0)};
                st.output = beta.outputs[0];
                steps.push_back(st);
                for (size_t k2 = i + 1; k2 < i + 9; k2++) skip[k2] = true;
                renames.push_back({i, beta.outputs[0]});
                i += 9;
                continue;
            }
        }
        size_t j = i + 1;
        std::string out = n.outputs[0];
        // a following Add of a constant bias, read only here (src/nd.rs:619-625)
        auto takes_bias = [&](const Node &next, const std::string &o, size_t want) -> std::optional<std::string> {
            if (next.op != "Add" || readers(o) != 1 || next.inputs.size() < 2) return std::nullopt;
            std::string other;
            if (next.inputs[0] == o) other = next.inputs[1];
            else if (next.inputs[1] == o) other = next.inputs[0];
            else return std::nullopt;
            auto it = m.weights.find(other);
            if (it == m.weights.end()) return std::nullopt;
            int non1 = 0;
            for (auto d : it->second.dims) non1 += d != 1;
            if (it->second.data.size() != want || non1 > 1) return std::nullopt;
            return other;
        };
        Step st;
        bool fused_step = false;
        if (n.op == "Conv") {
            const HostW &w = m.weight(n.in(1));
            if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "conv weight not 4D");
            int cout = (int)w.dims[0];
            std::vector<float> b = bias_or_zero(m, n, 2, cout);
            int act = 0;
            if (j < nodes.size()) {
                if (auto name = takes_bias(nodes[j], out, cout)) {
                    const auto &bw = m.weight(*name).data;
                    for (int q = 0; q < cout; q++) b[q] += bw[q];
                    out = nodes[j].outputs[0];
                    j++;
                }
            }
            if (j < nodes.size() && nodes[j].op == "Relu" && nodes[j].in(0) == out && readers(out) == 1) {
                act = 1;
                out = nodes[j].outputs[0];
                j++;
            }
            // GELU as the exporter writes it: x * (erf(x / sqrt 2) + 1) * 0.5 (src/nd.rs:674-701)
            if (act == 0 && j + 4 < nodes.size()) {
                {
                    const Node &dv = nodes[j], &ef = nodes[j + 1], &ad = nodes[j + 2], &mu = nodes[j + 3],
                               &hf = nodes[j + 4];
                    auto has = [](const Node &q, const std::string &s) {
                        return std::find(q.inputs.begin(), q.inputs.end(), s) != q.inputs.end();
                    };
                    auto any_scalar = [&](const Node &q, float v, float tol) {
                        for (auto &x : q.inputs) {
                            auto s = scalar(x);
                            if (s && std::fabs(*s - v) < tol) return true;
                        }
                        return false;
                    };
                    auto sq2 = scalar(dv.in(1));
                    bool ok = dv.op == "Div" && dv.in(0) == out && sq2 && std::fabs(*sq2 - 1.41421356f) < 1e-4f &&
                              ef.op == "Erf" && ef.in(0) == dv.outputs[0] && ad.op == "Add" &&
                              has(ad, ef.outputs[0]) && any_scalar(ad, 1.0f, 1e-6f) && mu.op == "Mul" &&
                              has(mu, out) && has(mu, ad.outputs[0]) && hf.op == "Mul" && has(hf, mu.outputs[0]) &&
                              any_scalar(hf, 0.5f, 1e-6f) && readers(out) == 2;
                    for (auto *o : {&dv.outputs[0], &ef.outputs[0], &ad.outputs[0], &mu.outputs[0]})
                        ok = ok && readers(*o) == 1;
                    if (ok) {
                        act = 3;
                        out = hf.outputs[0];
                        j += 5;
                    }
                }
            }
            // a residual Add of another computed tensor (src/nd.rs:703-716)
            std::string residual;
            if (j < nodes.size()) {
                const Node &nx = nodes[j];
                if (nx.op == "Add" && readers(out) == 1 &&
                    std::find(nx.inputs.begin(), nx.inputs.end(), out) != nx.inputs.end()) {
                    for (auto &o : nx.inputs)
                        if (o != out) {
                            if (!m.weights.count(o) && !m.ints.count(o)) {
                                residual = o;
                                out = nx.outputs[0];
                                j++;
                            }
                            break;
                        }
                }
            }
            int group = (int)n.int_("group").value_or(1);
            auto strides = n.ints("strides").value_or(std::vector<int64_t>{1, 1});
            auto dil = n.ints("dilations");
            if (dil)
                for (auto d : *dil)
                    if (d != 1) fail(WOCR_ERR_UNSUPPORTED, "dilated conv");
            st.kind = Step::N_CONV;
            st.conv = lower_conv_dense(c, w, b, group);
            st.conv.sh = (int)strides[0];
            st.conv.sw = (int)strides[1];
            auto pads = n.ints("pads");
            if (pads && pads->size() >= 4)
                for (int q = 0; q < 4; q++) st.conv.pads[q] = (int)(*pads)[q];
            st.conv.same_upper = n.str("auto_pad").value_or("") == "SAME_UPPER";
            st.act = act;
            st.residual = residual;
            auto sc = in_scale.find(i);
            if (sc != in_scale.end()) st.scale = sc->second;
            st.inputs = {n.in(0)};
            if (!residual.empty()) st.inputs.push_back(residual);
            if (!st.scale.empty()) st.inputs.push_back(st.scale);
            fused_step = true;
        } else if (n.op == "MatMul" && m.weights.count(n.in(1)) && m.weights.at(n.in(1)).dims.size() == 2) {
            const HostW &w = m.weight(n.in(1));
            int K = (int)w.dims[0], N = (int)w.dims[1];
            std::vector<float> b(N, 0.f);
            if (j < nodes.size())
                if (auto name = takes_bias(nodes[j], out, N)) {
                    b = m.weight(*name).data;
                    out = nodes[j].outputs[0];
                    j++;
                }
            int act = 0;
            if (j + 1 < nodes.size()) {
                const Node &sg = nodes[j], &mu = nodes[j + 1];
                auto has = [](const Node &q, const std::string &s) {
                    return std::find(q.inputs.begin(), q.inputs.end(), s) != q.inputs.end();
                };
                if (sg.op == "Sigmoid" && sg.in(0) == out && mu.op == "Mul" && has(mu, out) && has(mu, sg.outputs[0]) &&
                    readers(out) == 2 && readers(sg.outputs[0]) == 1) {
                    act = 4;
                    out = mu.outputs[0];
                    j += 2;
                }
            }
            st.kind = Step::N_LINEAR;
            st.lk = K;
            st.ln = N;
            st.ldw = round4(N);
            std::vector<float> t((size_t)K * st.ldw, 0.f);
            for (int r = 0; r < K; r++)
                for (int q = 0; q < N; q++) t[(size_t)r * st.ldw + q] = w.data[(size_t)r * N + q];
            st.lw = upload(c, t);
            st.luw = linear_umma(c, w.data.data(), K, N);
            b.resize(st.ldw, 0.f);
            st.lb = upload(c, b);
            st.act = act;
            st.inputs = {n.in(0)};
            fused_step = true;
        } else if (n.op == "ConvTranspose") {
            const HostW &w = m.weight(n.in(1));
            if (w.dims.size() != 4) fail(WOCR_ERR_UNSUPPORTED, "ConvTranspose weight not 4D");
            int cout = (int)w.dims[1];
            auto strides = n.ints("strides").value_or(std::vector<int64_t>{1, 1});
            auto nz = [&](const char *a) {
                auto v = n.ints(a);
                if (!v) return false;
                for (auto x : *v)
                    if (x != 0) return true;
                return false;
            };
            if (n.int_("group").value_or(1) != 1 || nz("pads") || nz("output_padding") || strides[0] != strides[1])
                fail(WOCR_ERR_UNSUPPORTED, "unsupported ConvTranspose attributes");
            std::vector<float> b = bias_or_zero(m, n, 2, cout);
            if (j < nodes.size())
                if (auto name = takes_bias(nodes[j], out, cout)) {
                    const auto &bw = m.weight(*name).data;
                    for (int q = 0; q < cout; q++) b[q] += bw[q];
                    out = nodes[j].outputs[0];
                    j++;
                }
            int act = 0;
            if (j < nodes.size() && (nodes[j].op == "Relu" || nodes[j].op == "Sigmoid") && nodes[j].in(0) == out &&
                readers(out) == 1) {
                act = nodes[j].op == "Relu" ? 1 : 2;
                out = nodes[j].outputs[0];
                j++;
            }
            st.kind = Step::N_CONVT;
            st.convt = lower_convt(c, w, b, (int)strides[0]);
            st.act = act;
            st.inputs = {n.in(0)};
            fused_step = true;
        } else if (n.op == "BatchNormalization") {
            const auto &g = m.weight(n.in(1)).data, &sh = m.weight(n.in(2)).data, &mn = m.weight(n.in(3)).data,
                       &vr = m.weight(n.in(4)).data;
            float eps = n.f32("epsilon").value_or(1e-5f);
            size_t C = g.size();
            std::vector<float> stv(2 * C);
            for (size_t q = 0; q < C; q++) {
                float s = g[q] / std::sqrt(vr[q] + eps);
                stv[q] = s;
                stv[C + q] = sh[q] - mn[q] * s;
            }
            st.kind = Step::N_AFFINE;
            st.st = upload(c, stv);
            st.inputs = {n.in(0)};
            fused_step = true;
        }
        for (size_t k2 = i + 1; k2 < j; k2++) skip[k2] = true;
        if (j > i + 1) renames.push_back({i, out});
        if (fused_step) {
            st.node = (int)i;
            st.output = out;
            steps.push_back(st);
        } else {
            Step g;
            g.kind = Step::N_GENERIC;
            g.node = (int)i;
            g.inputs = n.inputs;
            g.output = n.outputs[0];
            steps.push_back(g);
        }
        i = j;
    }
    for (auto &r : renames) nodes[r.first].outputs[0] = r.second;
    ex->model = m;
    ex->model.nodes = nodes;
    ex->steps = steps;
    ex->input = m.input;
    ex->output = output;
    ex->finalize();
    return ex;
}

}  // namespace wocr
