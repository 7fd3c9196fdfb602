// Row arg-max for callers that cannot allocate device memory.
//
// wocr_ndgraph_run_argmax stages its per-row results (best class, row maximum, log-sum-exp) in
// device buffers it allocates for every call, then copies them to the caller.  Some callers
// cannot have the library allocate: a host program whose own allocator owns the whole GPU
// (it sized its arena at start-up and nothing else may take memory), a process under a device
// memory cap where an allocation failing in the middle of a request is not acceptable, or a
// latency-critical path that avoids cudaMalloc because it can synchronise the device.  This
// variant runs the same arg-max kernel with its scratch in a fixed array in the library's
// device memory instead.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"

namespace {

// Scratch of wocr_argmax_rows_noalloc: per row the best index (u32), the row maximum (f32) and
// the log-sum-exp (f32), for at most kMaxRows rows (768 KiB).  Every GPU that loads the library
// holds this array until the process exits.  All calls share it and it keeps the contents of the
// last call; the kernel writes every entry it later reads, so nothing needs clearing.
constexpr int64_t kMaxRows = 65536;
static __device__ __align__(256) uint8_t g_argmax_scratch[kMaxRows * 12];

// Device address of the array per device.  In host code `g_argmax_scratch` names a host-side
// stand-in, not device memory, so the kernel gets this address instead.
std::mutex g_mu;
void *g_addr[64] = {nullptr};

void *scratch_address(int device) {
    if (device < 0 || device >= 64) wocr::fail(WOCR_ERR_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);  // with `device` current
        if (e != cudaSuccess || !p)
            wocr::fail(WOCR_ERR_CUDA, std::string("cudaGetSymbolAddress of the arg-max scratch: ") +
                                          cudaGetErrorString(e));
        g_addr[device] = p;
    }
    return g_addr[device];
}

}  // namespace

extern "C" int32_t wocr_argmax_rows_noalloc(wocr_ctx *ctx, const float *d_logits, int64_t rows, int64_t len,
                                            uint32_t *best, float *row_max, float *row_lse) {
    try {
        wocr::Ctx *c = wocr::ctx_of(ctx);
        if (!c || !d_logits || rows <= 0 || len <= 0 || !best) wocr::fail(WOCR_ERR_INVALID, "bad argument");
        if (rows > kMaxRows)
            wocr::fail(WOCR_ERR_CAPACITY, "wocr_argmax_rows_noalloc handles at most " + std::to_string(kMaxRows) +
                                              " rows, got " + std::to_string(rows));
        WOCR_CUDA(cudaSetDevice(c->device));
        uint8_t *s = static_cast<uint8_t *>(scratch_address(c->device));
        uint32_t *d_best = reinterpret_cast<uint32_t *>(s);
        float *d_max = reinterpret_cast<float *>(s + kMaxRows * 4);
        float *d_lse = reinterpret_cast<float *>(s + kMaxRows * 8);
        wocr::k::argmax(c, d_logits, rows, len, len, d_best, d_max, row_lse ? d_lse : nullptr, 0);
        WOCR_CUDA(cudaMemcpyAsync(best, d_best, (size_t)rows * 4, cudaMemcpyDeviceToHost, c->stream));
        if (row_max)
            WOCR_CUDA(cudaMemcpyAsync(row_max, d_max, (size_t)rows * 4, cudaMemcpyDeviceToHost, c->stream));
        if (row_lse)
            WOCR_CUDA(cudaMemcpyAsync(row_lse, d_lse, (size_t)rows * 4, cudaMemcpyDeviceToHost, c->stream));
        wocr::sync_bounded(c, 0);
        wocr::set_last_error("");
        return WOCR_OK;
    } catch (const wocr::Error &e) {
        wocr::set_last_error(e.what());
        return e.code;
    } catch (const std::exception &e) {
        wocr::set_last_error(e.what());
        return WOCR_ERR_INVALID;
    }
}
