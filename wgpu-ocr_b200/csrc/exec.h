// Graph executors: the lowering and fusion passes of the reference's two executors and the
// run loop that issues the sm_100a kernels.
//   Graph   - src/gpu.rs:1058-1378 (4-D convolutional graphs of the ocrs models)
//   NdGraph - src/nd.rs:428-1394  (N-D graphs of PP-OCR, with load-time fusions)
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"
#include "model.h"
#include "tconv.h"
#include "umma.h"

namespace wocr {

// A weight uploaded to the device.
struct DevW {
    BufP buf;
    float *p = nullptr;
    int64_t n = 0;
};
DevW upload(Ctx *c, const std::vector<float> &v);
DevW upload(Ctx *c, const float *v, int64_t n);

// A lowered convolution (dense, depthwise or Cin = 1 direct), weights laid out for its kernel.
struct ConvW {
    enum Kind { DENSE, DEPTHWISE, DIRECT } kind = DENSE;
    DevW w, b;
    int cout = 0, cin = 0, group = 1, kh = 1, kw = 1, sh = 1, sw = 1;
    int pads[4] = {0, 0, 0, 0};  // top, left, bottom, right
    bool same_upper = false;
    int ldw = 0;                 // DENSE: columns of the [K][ldw] weight matrix
    int pool_h = 1, pool_w = 1;  // DIRECT: fused MaxPool
    std::shared_ptr<k::UmmaW> uw;  // DENSE: the tensor-core operand (split bf16, TMA maps)
    std::shared_ptr<k::TconvW> tw;  // DENSE, stride 1: the tap-convolution operand (split inputs)
};

// A lowered ConvTranspose: kernel == stride runs as one GEMM with a scatter epilogue.
struct ConvTW {
    DevW w, b;  // gemm: [cin][ldw] with column (ky*s + kx)*cout + co; else [cin][cout][kh][kw]
    int cin = 0, cout = 0, kh = 0, kw = 0, s = 1, ldw = 0;
    bool gemm = false;
    std::shared_ptr<k::UmmaW> uw;  // gemm: the tensor-core operand
    std::shared_ptr<k::TconvW> tw;  // gemm: the tap-convolution operand (split inputs)
};

ConvW lower_conv_dense(Ctx *c, const HostW &w, const std::vector<float> &bias, int group);
ConvTW lower_convt(Ctx *c, const HostW &w, const std::vector<float> &bias, int stride);
// Tap-convolution operands (split inputs): a stride-1 dense convolution, a kernel == stride
// ConvTranspose.
void attach_tconv(Ctx *c, ConvW &cw, const HostW &w);
void attach_tconv(Ctx *c, ConvTW &t, const HostW &w);

// A value while a graph runs: a device float tensor or a host integer tensor (src/nd.rs:448).
struct Value {
    bool is_int = false;
    DT f;
    std::vector<int64_t> iv;
    std::vector<int64_t> ishape;
};

// One executed step of a lowered graph.
struct Step {
    enum Kind {
        // Graph (src/gpu.rs:1088-1098)
        G_CONV, G_DIRECT, G_DEPTHWISE, G_CONVT, G_MAXPOOL, G_SLICE, G_CONCAT, G_ACT, G_IDENTITY,
        // NdGraph fused kinds (src/nd.rs:467-479); other NdGraph nodes run as N_GENERIC
        N_CONV, N_CONVT, N_LINEAR, N_AFFINE, N_LAYERNORM, N_GENERIC
    } kind;
    int node = -1;                        // index into the (rewritten) node list
    std::vector<std::string> inputs;
    std::string output;
    ConvW conv;
    ConvTW convt;
    int act = 0;
    std::string residual, scale;          // N_CONV fusions
    DevW lw, lb;                          // N_LINEAR [K][ldw] + bias
    int lk = 0, ln = 0, ldw = 0;
    std::shared_ptr<k::UmmaW> luw;        // N_LINEAR tensor-core operand
    DevW st;                              // N_AFFINE scale|shift, N_LAYERNORM gamma|beta
    int ln_len = 0;
    float eps = 1e-5f;
    std::vector<int64_t> starts, ends, axes;  // G_SLICE
    bool split_out = false;               // the output is stored as a split tensor
    // a 2 x 2 MaxPool of this convolution's output computed by its epilogue (pool_output named,
    // split when pool_split); the MaxPool step itself is then skipped (pool_fused_away)
    std::string pool_output;
    bool pool_split = false, pool_fused_away = false;
    // a 1 x 1 head convolution (head_step, output head_output) computed by this convolution's
    // epilogue: this step's own output is then never stored, and the head step is skipped
    // (head_fused_away)
    std::string head_output;
    int head_step = -1;
    bool head_fused_away = false;
};

class Executor {
  public:
    Ctx *ctx;
    Model model;                          // nodes rewritten by the fusion pass
    std::vector<Step> steps;
    std::map<std::string, DT> weights;    // float initializers read by generic steps
    std::string input, output;
    std::map<std::string, int> last_use;  // value -> last step reading it
    struct ConcatSlot {
        std::string concat;               // the Concat output this value is a channel slice of
        int64_t offset, ctot;
    };
    std::map<std::string, ConcatSlot> concat_slot;
    std::map<std::string, DT> *cbufs = nullptr;  // Concat buffers of the current run
    // Values between the convolutional steps of a Graph may be stored split (bf16 hi | lo, as
    // the tap convolution reads them); plan_split() marks the steps whose output is.
    bool allow_split = false;

    explicit Executor(Ctx *c) : ctx(c) {}
    // Run on `x`; returns the output tensor.
    DT run(const DT &x);
    // Run steps [0, upto); returns the first input of step `upto` (the output when upto = all).
    DT run_to(const DT &x, int upto);
    // The last step is a linear layer without activation producing the output (a CTC head).
    bool ends_in_linear() const;
    // That linear layer on x (its input) with the row arg-max fused; returns the logits' shape.
    std::vector<int64_t> linear_argmax(const DT &x, uint32_t *best, float *row_max, float *row_lse);
    void finalize();  // uploads generic weights, computes last uses

  protected:
    void plan_split();
    DT slot_output(const std::string &name, int64_t n, int64_t c, int64_t h, int64_t w, bool split);
    DT concat_channels(const std::vector<DT> &parts, const std::string &out_name, bool split);
    Value get(std::map<std::string, Value> &vals, const std::string &name);
    DT getf(std::map<std::string, Value> &vals, const std::string &name);  // fp32 (converts split)
    DT getx(std::map<std::string, Value> &vals, const std::string &name);  // as stored
    void exec_step(const Step &s, std::map<std::string, Value> &vals);
    void exec_generic(const Node &n, std::map<std::string, Value> &vals);
};

// Graph::build (src/gpu.rs:1104-1240): the graph up to (not including) the first node of type
// `stop`, if given; `stop_node` receives that node.
std::unique_ptr<Executor> build_graph(Ctx *c, const Model &m, const char *stop, Node *stop_node);
// NdGraph::new (src/nd.rs:505-817).
std::unique_ptr<Executor> build_ndgraph(Ctx *c, const Model &m, bool stop_before_softmax);

// Helpers shared with the API layer.
DT to_nhwc(Ctx *c, const DT &x);
DT to_f32(Ctx *c, const DT &x);  // a split tensor as fp32 NHWC; others unchanged
DT to_rowmajor(Ctx *c, const DT &x);
using OutAlloc = std::function<DT(int64_t n, int64_t c, int64_t h, int64_t w)>;
// A 2 x 2 / stride 2 MaxPool wanted of a convolution's output: `out` receives it.
struct PoolReq {
    bool split = false;
    bool done = false;
    DT out;
};
// A 1 x 1 convolution with at most 4 outputs (cw, act) that reads only the convolution being run:
// computed by that convolution's epilogue when the row kernel runs it (done), else after it.
struct HeadReq {
    const ConvW *cw = nullptr;
    int act = 0;
    bool done = false;
    DT out;
};
DT conv_run(Ctx *c, const DT &x, const ConvW &cw, int act, const DT *res, const DT *scale,
            const OutAlloc *out = nullptr, PoolReq *pool = nullptr, HeadReq *head = nullptr);
DT linear_run(Ctx *c, const DT &x, const DevW &w, const DevW &b, int K, int N, int ldw, int act,
              const k::UmmaW *uw = nullptr);
// [K][N] row-major fp32 weights -> the tensor-core operand of y = x W.
std::shared_ptr<k::UmmaW> linear_umma(Ctx *c, const float *w_kn, int K, int N);
DT from_host(Ctx *c, const float *x, const std::vector<int64_t> &shape);

}  // namespace wocr
