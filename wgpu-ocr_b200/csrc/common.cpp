// Status handling, device buffers, device tensors, model parsing.
#include "common.h"

#include <algorithm>
#include <cstring>
#include <sstream>

#include "model.h"

namespace wocr {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string &msg) { g_last_error = msg; }
const std::string &last_error() { return g_last_error; }

[[noreturn]] void fail(int32_t code, const std::string &msg) { throw Error(code, msg); }

static cudaEvent_t take_event(Ctx *c) {
    if (!c->spare.empty()) {
        cudaEvent_t e = c->spare.back();
        c->spare.pop_back();
        return e;
    }
    cudaEvent_t e;
    WOCR_CUDA(cudaEventCreate(&e));
    return e;
}

Prof::Prof(Ctx *ctx, const char *name, double flops, double bytes) : c(ctx), on(ctx->prof) {
    if (!on) return;
    r.name = name;
    r.flops = flops;
    r.bytes = bytes;
    r.a = take_event(c);
    r.b = take_event(c);
    cudaEventRecord(r.a, c->stream);
}

Prof::~Prof() {
    if (!on) return;
    cudaEventRecord(r.b, c->stream);
    c->recs.push_back(r);
}

Buf::Buf(Ctx *c, size_t b) : ctx(c), p(nullptr), bytes(b) {
    size_t n = b == 0 ? 16 : (b + 15) / 16 * 16;
    cudaError_t e = cudaMallocAsync(&p, n, c->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        p = nullptr;
        fail(e == cudaErrorMemoryAllocation ? WOCR_ERR_OOM : WOCR_ERR_CUDA,
             std::string("device allocation of ") + std::to_string(n) + " bytes: " + cudaGetErrorString(e));
    }
}

Buf::~Buf() {
    if (p) cudaFreeAsync(p, ctx->stream);
}

std::vector<int64_t> rowmajor_strides(const std::vector<int64_t> &shape) {
    std::vector<int64_t> s(shape.size(), 1);
    for (int d = (int)shape.size() - 2; d >= 0; d--) s[d] = s[d + 1] * shape[d + 1];
    return s;
}

bool DT::rowmajor() const {
    int64_t expect = 1;
    for (int d = rank() - 1; d >= 0; d--) {
        if (shape[d] != 1 && strides[d] != expect) return false;
        expect *= shape[d];
    }
    return true;
}

bool DT::nhwc() const {
    if (rank() != 4) return false;
    if (shape[1] > 1 && strides[1] != 1) return false;
    if (strides[3] < shape[1]) return false;
    if (shape[2] > 1 && strides[2] != shape[3] * strides[3]) return false;
    return true;
}

bool DT::dense() const {
    // a permutation of a contiguous block: sort dims by stride and check
    std::vector<std::pair<int64_t, int64_t>> v;
    for (int d = 0; d < rank(); d++)
        if (shape[d] != 1) v.push_back({strides[d], shape[d]});
    std::sort(v.begin(), v.end());
    int64_t expect = 1;
    for (auto &e : v) {
        if (e.first != expect) return false;
        expect *= e.second;
    }
    return true;
}

DT new_rowmajor(Ctx *c, const std::vector<int64_t> &shape) {
    DT t;
    t.shape = shape;
    t.strides = rowmajor_strides(shape);
    int64_t n = t.numel();
    t.buf = alloc(c, (size_t)std::max<int64_t>(n, 1) * sizeof(float));
    t.p = (float *)t.buf->p;
    return t;
}

DT new_nhwc(Ctx *c, int64_t n, int64_t ch, int64_t h, int64_t w) {
    DT t;
    t.shape = {n, ch, h, w};
    t.strides = {h * w * ch, 1, w * ch, ch};
    t.buf = alloc(c, (size_t)std::max<int64_t>(n * ch * h * w, 1) * sizeof(float));
    t.p = (float *)t.buf->p;
    return t;
}

DT new_nhwc_split(Ctx *c, int64_t n, int64_t ch, int64_t h, int64_t w) {
    DT t;
    t.shape = {n, ch, h, w};
    t.strides = {h * w * 2 * ch, 1, w * 2 * ch, 2 * ch};
    t.buf = alloc(c, (size_t)std::max<int64_t>(n * ch * h * w, 1) * 2 * sizeof(uint16_t));
    t.p = (float *)t.buf->p;
    t.split = true;
    return t;
}

std::string shape_str(const std::vector<int64_t> &s) {
    std::ostringstream o;
    o << "[";
    for (size_t i = 0; i < s.size(); i++) o << (i ? ", " : "") << s[i];
    o << "]";
    return o.str();
}

// ---- model -----------------------------------------------------------------------------
std::optional<std::vector<int64_t>> Node::ints(const std::string &name) const {
    auto it = attrs.find(name);
    if (it == attrs.end()) return std::nullopt;
    return it->second.ints;
}
std::optional<int64_t> Node::int_(const std::string &name) const {
    auto it = attrs.find(name);
    if (it == attrs.end() || it->second.kind != WOCR_ATTR_INT) return std::nullopt;
    return it->second.i;
}
std::optional<std::string> Node::str(const std::string &name) const {
    auto it = attrs.find(name);
    if (it == attrs.end() || it->second.kind != WOCR_ATTR_STRING) return std::nullopt;
    return it->second.s;
}
std::optional<float> Node::f32(const std::string &name) const {
    auto it = attrs.find(name);
    if (it == attrs.end() || it->second.kind != WOCR_ATTR_FLOAT) return std::nullopt;
    return it->second.f;
}
const std::string &Node::in(size_t k) const {
    static const std::string empty;
    return k < inputs.size() ? inputs[k] : empty;
}

const HostW &Model::weight(const std::string &name) const {
    auto it = weights.find(name);
    if (it == weights.end()) fail(WOCR_ERR_MISSING, "missing weight " + name);
    return it->second;
}

int Model::readers(const std::string &name) const {
    int c = 0;
    for (auto &n : nodes)
        for (auto &i : n.inputs)
            if (i == name) {
                c++;
                break;
            }
    return c;
}

Model model_from_c(const wocr_model *m) {
    if (!m) fail(WOCR_ERR_INVALID, "null model");
    Model out;
    auto str = [](const char *s) { return std::string(s ? s : ""); };
    for (int i = 0; i < m->n_inits; i++) {
        const wocr_initializer &t = m->inits[i];
        int64_t count = 1;
        std::vector<int64_t> dims;
        for (int d = 0; d < t.rank; d++) {
            if (t.dims[d] < 0) fail(WOCR_ERR_INVALID, "negative dimension");
            dims.push_back(t.dims[d]);
            count *= t.dims[d];
        }
        if (count > 0 && !t.data) fail(WOCR_ERR_INVALID, "initializer " + str(t.name) + " without data");
        if (t.dtype == 1) {
            HostW w;
            w.dims = dims;
            w.data.assign((const float *)t.data, (const float *)t.data + count);
            out.weights[str(t.name)] = std::move(w);
        } else if (t.dtype == 7) {
            out.ints[str(t.name)] = std::vector<int64_t>((const int64_t *)t.data, (const int64_t *)t.data + count);
        }
        // other element types are ignored, as src/onnx.rs:80-83 does
    }
    for (int i = 0; i < m->n_nodes; i++) {
        const wocr_node &cn = m->nodes[i];
        Node n;
        n.op = str(cn.op);
        for (int k = 0; k < cn.n_inputs; k++) n.inputs.push_back(str(cn.inputs[k]));
        for (int k = 0; k < cn.n_outputs; k++) n.outputs.push_back(str(cn.outputs[k]));
        if (n.outputs.empty()) fail(WOCR_ERR_INVALID, "node " + n.op + " without outputs");
        for (int k = 0; k < cn.n_attrs; k++) {
            const wocr_attr &a = cn.attrs[k];
            Attr at;
            at.kind = a.kind;
            at.i = a.i;
            at.f = a.f;
            at.s = str(a.s);
            if (a.kind == WOCR_ATTR_INTS && a.count > 0) at.ints.assign(a.ints, a.ints + a.count);
            if (a.kind == WOCR_ATTR_FLOATS && a.count > 0) at.floats.assign(a.floats, a.floats + a.count);
            n.attrs[str(a.name)] = at;
        }
        out.nodes.push_back(std::move(n));
    }
    out.input = str(m->input);
    out.output = str(m->output);
    if (out.input.empty()) fail(WOCR_ERR_INVALID, "no graph input");
    if (out.output.empty()) fail(WOCR_ERR_INVALID, "no graph output");
    return out;
}

}  // namespace wocr
