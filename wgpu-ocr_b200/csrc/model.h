// The loaded ONNX graph as the executors see it: `Onnx` of src/onnx.rs:44-56.
#pragma once

#include <map>
#include <optional>
#include <string>
#include <vector>

#include "common.h"

namespace wocr {

struct Attr {
    int kind = 0;
    int64_t i = 0;
    float f = 0.f;
    std::string s;
    std::vector<int64_t> ints;
    std::vector<float> floats;
};

// One node (src/onnx.rs:16-42): op type, input/output names, attributes.
struct Node {
    std::string op;
    std::vector<std::string> inputs, outputs;
    std::map<std::string, Attr> attrs;

    std::optional<std::vector<int64_t>> ints(const std::string &name) const;
    std::optional<int64_t> int_(const std::string &name) const;
    std::optional<std::string> str(const std::string &name) const;
    std::optional<float> f32(const std::string &name) const;
    const std::string &in(size_t k) const;  // "" when absent
};

struct HostW {
    std::vector<int64_t> dims;
    std::vector<float> data;
};

struct Model {
    std::vector<Node> nodes;
    std::map<std::string, HostW> weights;
    std::map<std::string, std::vector<int64_t>> ints;
    std::string input, output;

    const HostW &weight(const std::string &name) const;  // WOCR_ERR_MISSING if absent
    int readers(const std::string &name) const;          // src/onnx.rs:129-132
};

Model model_from_c(const wocr_model *m);

}  // namespace wocr
