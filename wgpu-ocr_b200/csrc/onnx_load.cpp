// ONNX model files read into a wocr_model, as the reference's loader reads them (Onnx::load,
// src/onnx.rs:57-123, over rten-onnx =0.26.0's protobuf reader).  The protobuf wire format of
// onnx.proto is decoded directly, for the fields that loader uses:
//   ModelProto.graph (7); GraphProto.node (1), initializer (5), input (11), output (12);
//   NodeProto.input (1), output (2), op_type (4), attribute (5);
//   AttributeProto.name (1), f (2), i (3), s (4), t (5), floats (7), ints (8), type (20);
//   TensorProto.dims (1), data_type (2), float_data (4), int64_data (7), name (8), raw_data (9);
//   ValueInfoProto.name (1).
// Everything else is skipped by wire type.  Repeated numeric fields are read packed or not.
// Semantics of Onnx::load: float (1) initializers become weights (their value count must match
// the dimensions), int64 (7) ones integer lists, other types are dropped; a Constant node's
// first tensor attribute becomes an initializer named after its first output and the node is
// dropped; the graph input is the first input that is not a float weight; the output is the
// first graph output.
#include <cstdio>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace {

using wocr::fail;

// One length-delimited region of the buffer.
struct Reader {
    const uint8_t *p, *end;
    bool done() const { return p >= end; }
    uint64_t varint() {
        uint64_t v = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            if (p >= end) fail(WOCR_ERR_INVALID, "truncated varint");
            const uint8_t b = *p++;
            v |= (uint64_t)(b & 0x7f) << shift;
            if (!(b & 0x80)) return v;
        }
        fail(WOCR_ERR_INVALID, "varint longer than 10 bytes");
        return 0;
    }
    Reader sub() {
        const uint64_t n = varint();
        if (n > (uint64_t)(end - p)) fail(WOCR_ERR_INVALID, "truncated length-delimited field");
        Reader r{p, p + n};
        p += n;
        return r;
    }
    std::string str() {
        Reader r = sub();
        return std::string((const char *)r.p, (size_t)(r.end - r.p));
    }
    uint32_t fixed32() {
        if (end - p < 4) fail(WOCR_ERR_INVALID, "truncated fixed32");
        uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }
    void skip(int wire) {
        switch (wire) {
        case 0: varint(); break;
        case 1:
            if (end - p < 8) fail(WOCR_ERR_INVALID, "truncated fixed64");
            p += 8;
            break;
        case 2: sub(); break;
        case 5: fixed32(); break;
        default: fail(WOCR_ERR_INVALID, "unsupported wire type " + std::to_string(wire));
        }
    }
};

float as_f32(uint32_t bits) {
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// a repeated varint field, packed (wire type 2) or one value (wire type 0)
void read_ints(Reader &r, int wire, std::vector<int64_t> &out) {
    if (wire == 2) {
        Reader s = r.sub();
        while (!s.done()) out.push_back((int64_t)s.varint());
    } else if (wire == 0) {
        out.push_back((int64_t)r.varint());
    } else {
        r.skip(wire);
    }
}

// a repeated float field, packed (wire type 2) or one value (wire type 5)
void read_floats(Reader &r, int wire, std::vector<float> &out) {
    if (wire == 2) {
        Reader s = r.sub();
        while (!s.done()) out.push_back(as_f32(s.fixed32()));
    } else if (wire == 5) {
        out.push_back(as_f32(r.fixed32()));
    } else {
        r.skip(wire);
    }
}

struct Tensor {
    std::string name;
    bool has_name = false, has_type = false, has_raw = false;
    int32_t type = 0;
    std::vector<int64_t> dims, i64;
    std::vector<float> f32;
    std::string raw;
};

Tensor read_tensor(Reader r) {
    Tensor t;
    while (!r.done()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        switch (field) {
        case 1: read_ints(r, wire, t.dims); break;
        case 2:
            if (wire != 0) fail(WOCR_ERR_INVALID, "TensorProto.data_type: wire type");
            t.type = (int32_t)r.varint();
            t.has_type = true;
            break;
        case 4: read_floats(r, wire, t.f32); break;
        case 7: read_ints(r, wire, t.i64); break;
        case 8:
            if (wire != 2) fail(WOCR_ERR_INVALID, "TensorProto.name: wire type");
            t.name = r.str();
            t.has_name = true;
            break;
        case 9:
            if (wire != 2) fail(WOCR_ERR_INVALID, "TensorProto.raw_data: wire type");
            t.raw = r.str();
            t.has_raw = true;
            break;
        default: r.skip(wire);
        }
    }
    return t;
}

struct Attr {
    std::string name;
    bool has_f = false, has_i = false, has_s = false, has_t = false;
    int type = 0;
    float f = 0;
    int64_t i = 0;
    std::string s;
    Tensor t;
    std::vector<float> floats;
    std::vector<int64_t> ints;
    bool has_floats = false, has_ints = false;
};

Attr read_attr(Reader r) {
    Attr a;
    while (!r.done()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        if ((field == 1 || field == 4 || field == 5) && wire != 2) {
            r.skip(wire);  // not the length-delimited field onnx.proto defines
            continue;
        }
        switch (field) {
        case 1: a.name = r.str(); break;
        case 2:
            if (wire != 5) fail(WOCR_ERR_INVALID, "AttributeProto.f: wire type");
            a.f = as_f32(r.fixed32());
            a.has_f = true;
            break;
        case 3:
            if (wire != 0) fail(WOCR_ERR_INVALID, "AttributeProto.i: wire type");
            a.i = (int64_t)r.varint();
            a.has_i = true;
            break;
        case 4:
            a.s = r.str();
            a.has_s = true;
            break;
        case 5:
            a.t = read_tensor(r.sub());
            a.has_t = true;
            break;
        case 7:
            read_floats(r, wire, a.floats);
            a.has_floats = true;
            break;
        case 8:
            read_ints(r, wire, a.ints);
            a.has_ints = true;
            break;
        case 20: a.type = (int)r.varint(); break;
        default: r.skip(wire);
        }
    }
    return a;
}

struct NodeP {
    std::string op;
    std::vector<std::string> inputs, outputs;
    std::vector<Attr> attrs;
};

NodeP read_node(Reader r) {
    NodeP n;
    while (!r.done()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        if (wire != 2) r.skip(wire);  // NodeProto's fields read here are all length-delimited
        else if (field == 1) n.inputs.push_back(r.str());
        else if (field == 2) n.outputs.push_back(r.str());
        else if (field == 4) n.op = r.str();
        else if (field == 5) n.attrs.push_back(read_attr(r.sub()));
        else r.skip(wire);
    }
    return n;
}

// ValueInfoProto.name, if present
bool read_value_name(Reader r, std::string &name) {
    bool has = false;
    while (!r.done()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        if (field == 1 && wire == 2) {
            name = r.str();
            has = true;
        } else {
            r.skip(wire);
        }
    }
    return has;
}

// The storage a loaded model's C view points into.
struct Owned {
    std::deque<std::string> strs;
    std::deque<std::vector<const char *>> name_lists;
    std::vector<wocr_node> nodes;
    std::deque<std::vector<wocr_attr>> attrs;
    std::deque<std::vector<int64_t>> i64;
    std::deque<std::vector<float>> f32;
    std::vector<wocr_initializer> inits;
    const char *keep(const std::string &s) {
        strs.push_back(s);
        return strs.back().c_str();
    }
};

// What wocr_model_load hands out: the model first (standard layout, so wocr_model_free can cast
// the model pointer back), then its storage.
struct Holder {
    wocr_model m;
    Owned *o;
};

struct Values {
    std::vector<int64_t> dims;
    int kind = 0;  // 1 float, 7 int64, 0 dropped
    std::vector<float> f;
    std::vector<int64_t> i;
};

// values() of src/onnx.rs:61-86
Values values(const Tensor &t) {
    Values v;
    int64_t count = 1;
    for (int64_t d : t.dims) {
        if (d < 0) fail(WOCR_ERR_INVALID, "negative dimension");
        count *= d;
        v.dims.push_back(d);
    }
    const int32_t type = t.has_type ? t.type : 0;
    if (type == 1) {
        if (t.has_raw) {
            const size_t n = t.raw.size() / 4;
            v.f.resize(n);
            std::memcpy(v.f.data(), t.raw.data(), n * 4);
        } else {
            v.f = t.f32;
        }
        if ((int64_t)v.f.size() != count) {
            const std::string nm = t.has_name ? "Some(\"" + t.name + "\")" : "None";
            fail(WOCR_ERR_INVALID, nm + ": " + std::to_string(v.f.size()) + " values for " + std::to_string(count));
        }
        v.kind = 1;
    } else if (type == 7) {
        if (t.has_raw) {
            const size_t n = t.raw.size() / 8;
            v.i.resize(n);
            std::memcpy(v.i.data(), t.raw.data(), n * 8);
        } else {
            v.i = t.i64;
        }
        // Onnx::load keeps an int64 list whatever its length; the C view's dims then describe
        // the list itself (prod(dims) values, as wocr_initializer promises)
        if ((int64_t)v.i.size() != count) v.dims = {(int64_t)v.i.size()};
        v.kind = 7;
    }
    return v;
}

wocr_model *parse(const uint8_t *bytes, size_t n) {
    Reader top{bytes, bytes + n};
    bool has_graph = false;
    Reader graph{nullptr, nullptr};
    while (!top.done()) {
        const uint64_t key = top.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        if (field == 7 && wire == 2) {
            graph = top.sub();  // a later graph field replaces an earlier one
            has_graph = true;
        } else {
            top.skip(wire);
        }
    }
    if (!has_graph) fail(WOCR_ERR_INVALID, "model has no graph");
    std::vector<NodeP> nodes;
    std::vector<Tensor> inits;
    std::vector<std::pair<bool, std::string>> inputs, outputs;
    while (!graph.done()) {
        const uint64_t key = graph.varint();
        const int field = (int)(key >> 3), wire = (int)(key & 7);
        if (field == 1 && wire == 2) nodes.push_back(read_node(graph.sub()));
        else if (field == 5 && wire == 2) inits.push_back(read_tensor(graph.sub()));
        else if ((field == 11 || field == 12) && wire == 2) {
            std::string nm;
            const bool has = read_value_name(graph.sub(), nm);
            (field == 11 ? inputs : outputs).push_back({has, nm});
        } else {
            graph.skip(wire);
        }
    }
    // weights and integer lists by name (a later one of the same name replaces an earlier one)
    std::map<std::string, Values> weights, ints;
    std::vector<std::string> worder, iorder;
    auto add = [&](const std::string &name, const Tensor &t) {
        Values v = values(t);
        if (v.kind == 1) {
            if (!weights.count(name)) worder.push_back(name);
            weights[name] = std::move(v);
        } else if (v.kind == 7) {
            if (!ints.count(name)) iorder.push_back(name);
            ints[name] = std::move(v);
        }
    };
    for (const Tensor &t : inits) add(t.has_name ? t.name : std::string(), t);
    std::unique_ptr<Owned> o(new Owned());
    std::vector<const NodeP *> kept;
    for (const NodeP &nd : nodes) {
        if (nd.op == "Constant") {
            if (!nd.outputs.empty())
                for (const Attr &a : nd.attrs)
                    if (a.has_t) {
                        add(nd.outputs[0], a.t);
                        break;
                    }
            continue;
        }
        kept.push_back(&nd);
    }
    const char *input = nullptr, *output = nullptr;
    for (const auto &in : inputs)
        if (in.first && !weights.count(in.second)) {
            input = o->keep(in.second);
            break;
        }
    if (!input) fail(WOCR_ERR_INVALID, "no graph input");
    if (outputs.empty() || !outputs[0].first) fail(WOCR_ERR_INVALID, "no graph output");
    output = o->keep(outputs[0].second);

    o->nodes.resize(kept.size());
    for (size_t k = 0; k < kept.size(); k++) {
        const NodeP &nd = *kept[k];
        wocr_node &cn = o->nodes[k];
        cn.op = o->keep(nd.op);
        o->name_lists.emplace_back();
        for (const std::string &s : nd.inputs) o->name_lists.back().push_back(o->keep(s));
        cn.inputs = o->name_lists.back().data();
        cn.n_inputs = (int32_t)nd.inputs.size();
        o->name_lists.emplace_back();
        for (const std::string &s : nd.outputs) o->name_lists.back().push_back(o->keep(s));
        cn.outputs = o->name_lists.back().data();
        cn.n_outputs = (int32_t)nd.outputs.size();
        o->attrs.emplace_back();
        std::vector<wocr_attr> &ca = o->attrs.back();
        for (const Attr &a : nd.attrs) {
            // the kind from AttributeProto.type (FLOAT 1, INT 2, STRING 3, FLOATS 6, INTS 7), or
            // from the field present when the type is missing.  An attribute with none of these
            // (a tensor or graph attribute, or an empty list without a type) becomes an empty
            // integer list: the reference's Node::ints gives Some([]) for it and its other
            // accessors None (src/onnx.rs:24-42)
            int kind = WOCR_ATTR_INTS;
            switch (a.type) {
            case 1: kind = WOCR_ATTR_FLOAT; break;
            case 2: kind = WOCR_ATTR_INT; break;
            case 3: kind = WOCR_ATTR_STRING; break;
            case 6: kind = WOCR_ATTR_FLOATS; break;
            case 7: kind = WOCR_ATTR_INTS; break;
            case 0:
                kind = a.has_ints ? WOCR_ATTR_INTS
                       : a.has_floats ? WOCR_ATTR_FLOATS
                       : a.has_s      ? WOCR_ATTR_STRING
                       : a.has_f      ? WOCR_ATTR_FLOAT
                       : a.has_i      ? WOCR_ATTR_INT
                                      : WOCR_ATTR_INTS;
                break;
            default: break;
            }
            wocr_attr x{};
            x.name = o->keep(a.name);
            x.kind = kind;
            x.i = a.i;
            x.f = a.f;
            if (kind == WOCR_ATTR_STRING) x.s = o->keep(a.s);
            if (kind == WOCR_ATTR_INTS) {
                o->i64.push_back(a.ints);
                x.ints = o->i64.back().data();
                x.count = (int64_t)a.ints.size();
            }
            if (kind == WOCR_ATTR_FLOATS) {
                o->f32.push_back(a.floats);
                x.floats = o->f32.back().data();
                x.count = (int64_t)a.floats.size();
            }
            ca.push_back(x);
        }
        cn.attrs = ca.data();
        cn.n_attrs = (int32_t)ca.size();
    }
    auto put = [&](const std::string &name, const Values &v, int32_t dtype) {
        wocr_initializer in{};
        in.name = o->keep(name);
        in.dtype = dtype;
        o->i64.push_back(v.dims);
        in.dims = o->i64.back().data();
        in.rank = (int32_t)v.dims.size();
        if (dtype == 1) {
            o->f32.push_back(v.f);
            in.data = o->f32.back().data();
        } else {
            o->i64.push_back(v.i);
            in.data = o->i64.back().data();
        }
        o->inits.push_back(in);
    };
    for (const std::string &nm : worder) put(nm, weights[nm], 1);
    for (const std::string &nm : iorder) put(nm, ints[nm], 7);
    Holder *h = new Holder();
    h->m.nodes = o->nodes.data();
    h->m.n_nodes = (int32_t)o->nodes.size();
    h->m.inits = o->inits.data();
    h->m.n_inits = (int32_t)o->inits.size();
    h->m.input = input;
    h->m.output = output;
    h->o = o.release();
    return &h->m;
}

}  // namespace

extern "C" {

int32_t wocr_model_parse(const uint8_t *bytes, int64_t n, wocr_model **out) {
    return wocr::guard([&] {
        if (!out || (n > 0 && !bytes) || n < 0) fail(WOCR_ERR_INVALID, "null argument");
        *out = parse(bytes, (size_t)n);
    });
}

int32_t wocr_model_load(const char *path, wocr_model **out) {
    return wocr::guard([&] {
        if (!path || !out) fail(WOCR_ERR_INVALID, "null argument");
        FILE *f = std::fopen(path, "rb");
        if (!f) fail(WOCR_ERR_INVALID, std::string(path) + ": cannot open");
        std::vector<uint8_t> buf;
        uint8_t chunk[1 << 16];
        size_t got;
        while ((got = std::fread(chunk, 1, sizeof chunk, f)) > 0) buf.insert(buf.end(), chunk, chunk + got);
        std::fclose(f);
        try {
            *out = parse(buf.data(), buf.size());
        } catch (const wocr::Error &e) {
            fail(e.code, std::string(path) + ": " + e.what());
        }
    });
}

void wocr_model_free(wocr_model *m) {
    if (!m) return;
    Holder *h = reinterpret_cast<Holder *>(m);
    delete h->o;
    delete h;
}

}  // extern "C"
