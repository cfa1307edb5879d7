// kq_noalloc.cu -- routed-expert decode for callers that cannot allocate.
//
// kq_moe_decode needs a scratch workspace (a status word, the routing, the
// gate/up activations and their per-tile scales) that the caller allocates
// once.  Some callers cannot do that: runtimes that hand a plugin
// only its input and output buffers and own every other byte of device memory
// in their own pool, and hosts that reach this library through a plain FFI
// (ctypes, cgo) with no device allocator at hand.  kq_moe_decode_static runs
// the same kernels with the scratch taken from one fixed array in this file:
//
//   * the array is a file-scope __device__ buffer of KQ_STATIC_WS_BYTES bytes;
//     every GPU that loads libkq.so holds it until the process exits;
//   * host code cannot use the array's name as a device address, so the first
//     call on each device (with that device current) resolves it with
//     cudaGetSymbolAddress and caches it; make that first call before any
//     stream capture;
//   * every call shares the array and it keeps the last call's contents: each
//     call clears the status word (the only part that must start at zero; the
//     rest is written before it is read) before its kernels;
//     calls that overlap on the GPU (two streams, two threads) race on it;
//   * a call whose workspace would exceed the array is rejected with
//     KQ_ERR_WORKSPACE and a message on stderr; nothing is allocated;
//   * the stream must belong to the current device (checked); a context reset
//     (cudaDeviceReset) invalidates the cached address until the process
//     restarts;
//   * kq_moe_decode_static_status reads the status word the last call on the
//     current device left (bad expert ids, wait timeouts), synchronising the
//     stream it is given.
#include <cstdio>
#include <mutex>

#include "kq_internal.h"

#define KQ_STATIC_WS_BYTES (8u << 20)

static __device__ __align__(256) uint8_t kq_static_ws[KQ_STATIC_WS_BYTES];

namespace {
std::mutex g_mu;
void* g_ws[64] = {nullptr};

// the array's device address for the current device (resolved on first use)
int static_ws(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KQ_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ws[dev]) {
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, kq_static_ws);
        if (rc != cudaSuccess || !p) {
            fprintf(stderr, "[kq] kq_moe_decode_static: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(rc));
            return KQ_ERR_CUDA;
        }
        g_ws[dev] = p;
    }
    *out = g_ws[dev];
    return KQ_OK;
}

// a stream of another device would run the kernels on addresses of this one
bool stream_on_current_device(cudaStream_t s) {
    if (!s) return true;
    int dev = 0, sdev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaStreamGetDevice(s, &sdev) != cudaSuccess) return false;
    return dev == sdev;
}
}  // namespace

extern "C" int kq_moe_decode_static(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                                    const float* logits, int32_t* idx, float* weights, int K,
                                    void* out_per_k, void* out, int out_dtype, const void* residual,
                                    void* stream) {
    if (!t || T < 0 || K <= 0) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    const kq::MoeWs L = kq::moe_ws_layout(t, T, K);
    if (L.total > KQ_STATIC_WS_BYTES) {
        fprintf(stderr,
                "[kq] kq_moe_decode_static: T=%d K=%d needs %zu bytes of scratch; the static buffer holds "
                "%u bytes (use kq_moe_decode with a caller workspace, or fewer tokens per call)\n",
                T, K, L.total, (unsigned)KQ_STATIC_WS_BYTES);
        return KQ_ERR_WORKSPACE;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!stream_on_current_device(s)) return KQ_ERR_ARG;
    void* ws = nullptr;
    if (int rc = static_ws(&ws)) return rc;
    uint8_t* w = static_cast<uint8_t*>(ws);
    if (cudaMemsetAsync(w + L.status, 0, L.idx - L.status, s) != cudaSuccess) return KQ_ERR_CUDA;
    return kq_moe_decode(t, layer, x, x_dtype, T, logits, idx, weights, K, out_per_k, out, out_dtype,
                         residual, ws, KQ_STATIC_WS_BYTES, stream);
}

extern "C" int kq_moe_decode_static_status(uint32_t* status_out, void* stream) {
    if (!status_out) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!stream_on_current_device(s)) return KQ_ERR_ARG;
    void* ws = nullptr;
    if (int rc = static_ws(&ws)) return rc;
    return kq_status_read(ws, status_out, stream);
}
