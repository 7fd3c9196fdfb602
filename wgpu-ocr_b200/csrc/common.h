// Shared internals of libwocr: status handling, the device context, device tensors.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/wocr.h"

namespace wocr {

// An error carried as a C++ exception inside the library and turned into a status code plus
// a thread-local message at the C ABI (the reference returns Err(String) in these places).
struct Error : std::runtime_error {
    int32_t code;
    Error(int32_t c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int32_t code, const std::string &msg);
void set_last_error(const std::string &msg);

// Runs an ABI entry point's body: a status code and the thread-local message from what it threw.
template <typename F>
int32_t guard(F &&f) {
    try {
        f();
        set_last_error("");
        return WOCR_OK;
    } catch (const Error &e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc &) {
        set_last_error("host out of memory");
        return WOCR_ERR_OOM;
    } catch (const std::exception &e) {
        set_last_error(e.what());
        return WOCR_ERR_INVALID;
    }
}

#define WOCR_CUDA(call)                                                                          \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess)                                                                   \
            ::wocr::fail(e_ == cudaErrorMemoryAllocation ? WOCR_ERR_OOM : WOCR_ERR_CUDA,         \
                         std::string(#call) + ": " + cudaGetErrorString(e_));                    \
    } while (0)

// Kernel launch bookkeeping: every launch goes through here, so the context can count them.
#define WOCR_LAUNCHED(ctx)                                                                       \
    do {                                                                                         \
        cudaError_t e_ = cudaGetLastError();                                                     \
        if (e_ != cudaSuccess) ::wocr::fail(WOCR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e_)); \
        (ctx)->launches++;                                                                       \
    } while (0)

// One timed kernel launch (profiling mode): CUDA events on the launching stream.
struct ProfRec {
    const char *name;
    cudaEvent_t a, b;
    double flops, bytes;
};

// The device context: `Gpu` of src/gpu.rs:825-846.  One stream; buffers come from the
// device's stream-ordered memory pool (cudaMallocAsync), which plays the reference's
// recycle-by-size pool (src/gpu.rs:938-966) without its cap bookkeeping.
struct Ctx {
    int device = 0;
    int lines = 8;
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    cudaMemPool_t pool = nullptr;
    int64_t launches = 0;
    double flops = 0;  // algorithmic FLOPs of the current run (2 per multiply-add)
    std::string name;
    // per-kernel timing with CUDA events (the reference's OPPROFILE / NDPROFILE, src/gpu.rs:1247,
    // src/nd.rs:18-27, without its wait after every node)
    bool prof = false;
    std::vector<ProfRec> recs;
    std::vector<cudaEvent_t> spare;
    // device error word written by kernels whose bounded waits gave up (0 = fine)
    int *status = nullptr;
    std::shared_ptr<struct Buf> status_buf;
    // unbounded waits poll this event briefly, then block on it (the host thread sleeps until
    // the stream reaches it) instead of spinning: several contexts per GPU, each with its own
    // host thread, share the host's cores with the other GPUs' processes
    cudaEvent_t sync_ev = nullptr;
};

// Brackets one kernel launch with events when the context profiles; records its algorithmic
// FLOPs and bytes.
struct Prof {
    Ctx *c;
    ProfRec r;
    bool on;
    Prof(Ctx *ctx, const char *name, double flops, double bytes);
    ~Prof();
};

// A device buffer owned jointly by the tensors that view it.  Freed on the context stream
// (stream order keeps later kernels safe), like recycle() returning it to the pool.
struct Buf {
    Ctx *ctx;
    void *p;
    size_t bytes;
    Buf(Ctx *c, size_t b);
    ~Buf();
    Buf(const Buf &) = delete;
    Buf &operator=(const Buf &) = delete;
};
using BufP = std::shared_ptr<Buf>;

inline BufP alloc(Ctx *c, size_t bytes) { return std::make_shared<Buf>(c, bytes); }

constexpr int kMaxRank = 6;  // src/nd.rs:30

// A float tensor on the device: logical shape with element strides into `buf`.  4-D image
// tensors produced by the convolution kernels are channels-last (NHWC): strides
// {H*W*P, 1, W*P, P} with the pixel stride P >= C (P > C when the tensor is a channel slice
// of a wider buffer, e.g. one part of a Concat).
//
// A split tensor (`split`) is an NHWC activation stored for the tensor cores: per pixel the bf16
// hi parts (bf16(v)) of all channels of its buffer, then their lo parts (bf16(v - hi)), the same
// 4 bytes a value as fp32.  Its strides count bf16 elements, `p` addresses the hi part of the
// view's first channel, and a channel's lo part lies pix() / 2 elements after its hi part.
struct DT {
    float *p = nullptr;
    std::vector<int64_t> shape;
    std::vector<int64_t> strides;
    BufP buf;
    bool split = false;

    int rank() const { return (int)shape.size(); }
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
    bool rowmajor() const;      // contiguous in logical order
    bool nhwc() const;          // rank 4, channels-last (pixel stride may exceed C)
    bool dense() const;         // covers numel() consecutive elements
    int64_t pix() const { return strides[3]; }  // NHWC pixel stride
};

// Waits for the context stream (bounded when timeout_ms > 0) and raises the device error word.
void sync_bounded(Ctx *c, int timeout_ms);
// Waits for the context stream (unbounded, on the context's blocking event when it has one).
void wait_stream(Ctx *c);
// The context behind a C-ABI handle.
Ctx *ctx_of(wocr_ctx *h);

std::vector<int64_t> rowmajor_strides(const std::vector<int64_t> &shape);
DT new_rowmajor(Ctx *c, const std::vector<int64_t> &shape);
DT new_nhwc(Ctx *c, int64_t n, int64_t ch, int64_t h, int64_t w);
DT new_nhwc_split(Ctx *c, int64_t n, int64_t ch, int64_t h, int64_t w);
std::string shape_str(const std::vector<int64_t> &s);

}  // namespace wocr
