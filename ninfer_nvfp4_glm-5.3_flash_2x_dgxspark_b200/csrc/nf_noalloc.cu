// nf_noalloc.cu -- nf_router_topk_noalloc (include/nf_moe.h): the router's
// top-k selection from caller-owned device buffers with no device memory
// allocation.  It has no counterpart in the reference.
//
// Who needs it: a caller that cannot allocate device memory -- a serving
// runtime whose memory pool reserved the device's free memory up front, a
// path where a cudaMalloc would synchronise the device, a process under a
// hard memory budget -- and so cannot create an nf_moe handle (which owns
// weights and a workspace).  The routes are the same bit-exact ones as
// nf_moe_route: the router kernels of nf_kernels.cu run unchanged, only their
// intermediate logits, scores and choices go to a fixed static device array
// compiled into this file instead of a handle's workspace.
#include "nf_moe.h"

#include "nf_internal.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>

using namespace nf;

namespace {

// tokens x experts scores one call may hold (e.g. 256 tokens at 64 experts)
constexpr int kMaxScores = NF_NOALLOC_MAX_SCORES;
// float layout: logits [kMaxScores] | scores [kMaxScores] | choices [kMaxScores] | error word + pad
constexpr int kErrOffset = 3 * kMaxScores;
constexpr int kScratchFloats = 3 * kMaxScores + 64;

}  // namespace

// The scratch: 3 x 64 KB of scores and one error word, about 192 KB per device.
// Only the error word has to start at zero; each call clears it on its stream.
static __device__ __align__(256) float g_route_scratch[kScratchFloats];

namespace {

std::mutex g_setup_mutex;
float* g_scratch[kMaxDevices] = {};  // device address of g_route_scratch per device

// A call whose logits stage gave up on a bounded wait has no valid routes:
// mark every index -1 (and every weight NaN) so the caller sees it.
__global__ void mark_failed_routes_kernel(const int* __restrict__ err, int32_t* __restrict__ idx,
                                          float* __restrict__ w, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && *err != 0) {
        idx[i] = -1;
        w[i] = __int_as_float(0x7fc00000);
    }
}

int report(char* msg, int msg_len, int status, const char* fmt, ...) {
    if (msg && msg_len > 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(msg, static_cast<size_t>(msg_len), fmt, ap);
        va_end(ap);
    }
    return status;
}

// One-time set-up of the current device: the scratch array's device address
// and the sigmoid lookup index the logits kernel reads.  Synchronises the
// device the first time, which is why the first call must not be captured.
int scratch_for_current_device(float** out, char* msg, int msg_len) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return report(msg, msg_len, NF_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return report(msg, msg_len, NF_ERR_UNSUPPORTED, "device %d is beyond the %d devices this build tracks", dev,
                      kMaxDevices);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch[dev]) {
        e = prepare_device_tables();
        if (e != cudaSuccess)
            return report(msg, msg_len, NF_ERR_CUDA, "sigmoid table set-up: %s", cudaGetErrorString(e));
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p)
            return report(msg, msg_len, NF_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        g_scratch[dev] = static_cast<float*>(p);
    }
    *out = g_scratch[dev];
    return NF_OK;
}

}  // namespace

int nf_router_topk_noalloc(const uint16_t* x, const uint16_t* router_w, const float* bias, int tokens, int hidden,
                           int experts, int top_k, int n_group, int topk_group, int normalize, float routed_scaling,
                           int32_t* topk_idx, float* topk_w, char* msg, int msg_len, void* stream) {
    if (msg && msg_len > 0) msg[0] = '\0';
    // every check runs before any CUDA call
    if (!x || !router_w || !bias || !topk_idx || !topk_w)
        return report(msg, msg_len, NF_ERR_INVALID, "null device pointer");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) % 16 != 0)
        return report(msg, msg_len, NF_ERR_LAYOUT, "x and router weights must be 16-byte aligned");
    if (tokens < 0) return report(msg, msg_len, NF_ERR_INVALID, "tokens must be >= 0");
    if (hidden <= 0 || hidden % 8 != 0) return report(msg, msg_len, NF_ERR_SHAPE, "hidden must be a positive multiple of 8");
    if (experts < 1 || experts > 1024) return report(msg, msg_len, NF_ERR_INVALID, "experts must be in [1, 1024]");
    if (top_k < 1 || top_k > 32 || top_k > experts)
        return report(msg, msg_len, NF_ERR_INVALID, "top_k must be in [1, min(32, experts)]");
    if (n_group < 1) return report(msg, msg_len, NF_ERR_INVALID, "n_group must be >= 1");
    if (n_group > 1 && (n_group > 32 || experts % n_group != 0 || topk_group < 1 || topk_group > n_group ||
                        top_k > topk_group * (experts / n_group)))
        return report(msg, msg_len, NF_ERR_UNSUPPORTED,
                      "group-limited routing needs n_group <= 32 dividing experts and enough eligible experts");
    if (!std::isfinite(routed_scaling)) return report(msg, msg_len, NF_ERR_INVALID, "routed_scaling must be finite");
    const long long scores = static_cast<long long>(tokens) * experts;
    if (scores > kMaxScores)
        return report(msg, msg_len, NF_ERR_CAPACITY,
                      "tokens x experts = %lld exceeds the %d scores of the static scratch; split the batch", scores,
                      kMaxScores);
    if (tokens == 0) return NF_OK;

    float* scratch = nullptr;
    const int st = scratch_for_current_device(&scratch, msg, msg_len);
    if (st != NF_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* err = reinterpret_cast<int*>(scratch + kErrOffset);
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), s);
    // w_safe = 0: the caller's weights are not range-checked on the host, so
    // the chain always runs the separately rounded multiply and add
    if (e == cudaSuccess)
        e = launch_router(x, router_w, /*w_chunked32=*/nullptr, /*w_chunked16=*/nullptr, bias, tokens, hidden, experts, top_k, routed_scaling,
                          normalize, n_group, topk_group, /*w_safe=*/0, scratch, scratch + kMaxScores,
                          scratch + 2 * kMaxScores, topk_idx, topk_w, err, s);
    if (e == cudaSuccess) {
        const int n = tokens * top_k;
        mark_failed_routes_kernel<<<(n + 255) / 256, 256, 0, s>>>(err, topk_idx, topk_w, n);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return report(msg, msg_len, NF_ERR_CUDA, "router launch: %s", cudaGetErrorString(e));
    return NF_OK;
}
