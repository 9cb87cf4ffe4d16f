// nf_tp.cu -- tensor-parallel BF16 linears: the reference's TP2 row split of
// every BF16 projection, rebuilt for 1-8 GPUs of one node.
//
// The reference (src/text_forward.cpp) runs one process per rank; for a BF16
// linear each rank computes a contiguous block of output rows with gemv_bf16
// (:497-508; apply_rows :803-819 gives rank 0 rows [0, rows/2) and rank 1
// [rows/2, rows)), then gather_rows (:242-256) swaps the halves over a
// socket so that both ranks hold the whole output vector.  linear_bf16
// (:821-830) and the lm_head logits (:656-667, :760-767) use it.
//
// Here one call does both steps on the GPU: each rank's CTAs compute their
// rows of the product -- the reference's exact arithmetic: a sequential fp32
// chain over the columns with the product and the sum rounded separately, so
// every output is bit-identical to gemv_bf16 -- and store them straight into
// every rank's gather buffer over NVLink (CUDA IPC mappings), closed by an
// epoch flag per source with a bounded wait.  The gather buffers alternate
// by epoch, and a rank writes into a peer's buffer only after that peer has
// acknowledged consuming the epoch that last used it, so consecutive calls
// never overwrite a result that is still being read.  With world = 1 the
// same kernels run without peers.  When the ranks cannot map each other's
// buffers (or NF_TP_TRANSPORT=nccl), each rank stores its rows locally and
// NCCL point-to-point calls exchange the row blocks.
//
// Rank r of `world` owns rows [r rows / world, (r+1) rows / world) (integer
// division; for world = 2 the reference's split).
#include "nf_moe.h"

#include "nf_common.cuh"
#include "nf_internal.h"
#include "nf_nccl.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace nf;

namespace {

constexpr int kTpMaxRanks = 8;
constexpr int kGemvRows = 256;   // output rows per CTA, one per thread
constexpr int kGemvKc = 64;      // columns per staged chunk
constexpr int kWPitch = 68;      // BF16 per staged row: 136 B, 8-byte aligned; the two
                                 // half-warps of a 64-bit read never share a bank
constexpr int kPieces = kGemvRows * kGemvKc / 4 / kGemvRows;  // 8-byte pieces per thread per chunk (16)
constexpr size_t kTpRecBytes = 256;
constexpr int64_t kFlagsBytes = 256;  // [0,64) row flags from each source, [64,128) acks from each source

struct TpPeers {
    uint8_t* mbox[kTpMaxRanks];
};

__device__ __forceinline__ void tp_st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tp_ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until the epoch at *flag reaches `want` (epochs only grow).
__device__ bool tp_wait_flag(const uint32_t* flag, uint32_t want) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (static_cast<int32_t>(tp_ld_acquire_sys(flag) - want) >= 0) return true;
        if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) return false;
        __nanosleep(100);
    }
}

// Start of call e = *epoch + 1: tell every rank that this rank has consumed
// every result up to e - 1 (everything before this kernel in the stream has
// completed), then wait until every rank has consumed e - 2, the last epoch
// that used the gather buffer call e writes into.
__global__ void tp_begin_kernel(TpPeers peers, int world, int me, const uint32_t* __restrict__ epoch,
                                int* __restrict__ err) {
    const uint32_t e = *epoch + 1u;
    const int p = threadIdx.x;
    if (p < world) tp_st_release_sys(reinterpret_cast<uint32_t*>(peers.mbox[p] + 64) + me, e - 1u);
    __syncwarp();
    if (p < world && e >= 3u &&
        !tp_wait_flag(reinterpret_cast<const uint32_t*>(peers.mbox[me] + 64) + p, e - 2u))
        atomicCAS(err, 0, NF_DEVERR_EP_WAIT);
}

// y[t, row0 + i] = sum_c bf16(W[i, c]) * x[t, c] for this rank's rows i, as
// gemv_bf16 computes it: acc starts at +0 and adds each rounded product in
// column order.  One thread per row and up to TPT tokens; W streams through
// shared memory in 64-column chunks (the next chunk's loads in flight during
// the current chunk's chains), x chunks are broadcast from shared memory.
// The rows go to every destination's gather buffer (peers; one of them is
// this rank's own), `stage` (contiguous [T][nrows], the NCCL transport) or
// both; the grid's last CTA publishes this rank's flag on every destination.
template <int TPT>
__global__ void __launch_bounds__(kGemvRows) tp_gemv_kernel(const uint16_t* __restrict__ W, const float* __restrict__ x,
                                                            int64_t rows_total, int64_t row0, int nrows, int cols,
                                                            int T, TpPeers peers, int world, int me, int64_t cap,
                                                            float* __restrict__ stage,
                                                            const uint32_t* __restrict__ epoch,
                                                            int* __restrict__ done) {
    __shared__ __align__(16) uint16_t sW[kGemvRows * kWPitch];
    __shared__ __align__(16) float sX[TPT * kGemvKc];
    const int tid = threadIdx.x;
    const int64_t rbase = static_cast<int64_t>(blockIdx.x) * kGemvRows;
    const int t0 = blockIdx.y * TPT;
    const int tn = min(TPT, T - t0);
    float acc[TPT];
#pragma unroll
    for (int t = 0; t < TPT; ++t) acc[t] = 0.f;
    uint2 pre[kPieces];
    // piece j of thread tid: staged row (tid + 256 j) / 16, 8-byte piece (tid + 256 j) % 16
    auto load_chunk = [&](int k0) {
#pragma unroll
        for (int j = 0; j < kPieces; ++j) {
            const int i = tid + kGemvRows * j;
            const int r = i >> 4, pc = i & 15;
            const int64_t row = rbase + r;
            const int col = k0 + pc * 4;
            pre[j] = (row < nrows && col < cols)
                         ? __ldg(reinterpret_cast<const uint2*>(W + row * cols + col))
                         : make_uint2(0u, 0u);
        }
    };
    load_chunk(0);
    for (int k0 = 0; k0 < cols; k0 += kGemvKc) {
        const int kc = min(kGemvKc, cols - k0);
        __syncthreads();  // the previous chunk's chains are done with sW / sX
#pragma unroll
        for (int j = 0; j < kPieces; ++j) {
            const int i = tid + kGemvRows * j;
            *reinterpret_cast<uint2*>(sW + (i >> 4) * kWPitch + (i & 15) * 4) = pre[j];
        }
        for (int i = tid; i < TPT * kGemvKc; i += kGemvRows) {
            const int t = i / kGemvKc, c = i % kGemvKc;
            sX[i] = (t < tn && k0 + c < cols) ? __ldg(x + static_cast<int64_t>(t0 + t) * cols + k0 + c) : 0.f;
        }
        __syncthreads();
        if (k0 + kGemvKc < cols) load_chunk(k0 + kGemvKc);
        const uint16_t* wr = sW + tid * kWPitch;
        // kc is a multiple of 4 (cols % 4 == 0)
        for (int c = 0; c < kc; c += 4) {
            const uint2 wp = *reinterpret_cast<const uint2*>(wr + c);
            const float w0 = __uint_as_float(wp.x << 16), w1 = __uint_as_float(wp.x & 0xffff0000u);
            const float w2 = __uint_as_float(wp.y << 16), w3 = __uint_as_float(wp.y & 0xffff0000u);
#pragma unroll
            for (int t = 0; t < TPT; ++t) {
                const float4 xv = *reinterpret_cast<const float4*>(sX + t * kGemvKc + c);
                float a = acc[t];
                a = __fadd_rn(a, __fmul_rn(w0, xv.x));
                a = __fadd_rn(a, __fmul_rn(w1, xv.y));
                a = __fadd_rn(a, __fmul_rn(w2, xv.z));
                a = __fadd_rn(a, __fmul_rn(w3, xv.w));
                acc[t] = a;
            }
        }
    }
    const int64_t row = rbase + tid;
    if (row < nrows) {
        const uint32_t e = *epoch + 1u;
        const int64_t buf = kFlagsBytes + static_cast<int64_t>(e & 1u) * cap;
        for (int p = 0; p < world; ++p) {
            float* out = reinterpret_cast<float*>(peers.mbox[p] + buf);
#pragma unroll
            for (int t = 0; t < TPT; ++t)
                if (t < tn) out[static_cast<int64_t>(t0 + t) * rows_total + row0 + row] = acc[t];
        }
        if (stage) {
#pragma unroll
            for (int t = 0; t < TPT; ++t)
                if (t < tn) stage[static_cast<int64_t>(t0 + t) * nrows + row] = acc[t];
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        const int total = static_cast<int>(gridDim.x * gridDim.y);
        if (atomicAdd(done, 1) == total - 1) {
            const uint32_t e = *epoch + 1u;
            __threadfence_system();
            for (int p = 0; p < world; ++p) tp_st_release_sys(reinterpret_cast<uint32_t*>(peers.mbox[p]) + me, e);
            *done = 0;  // ready for the next call (which follows this kernel in stream order)
        }
    }
}

// Waits until every source's rows of this call have arrived, then advances
// the epoch: the gather buffer of parity (epoch & 1) holds the result.
__global__ void tp_wait_kernel(const uint8_t* __restrict__ mbox, int world, uint32_t* __restrict__ epoch,
                               int* __restrict__ err) {
    const uint32_t e = *epoch + 1u;
    if (threadIdx.x < world && !tp_wait_flag(reinterpret_cast<const uint32_t*>(mbox) + threadIdx.x, e))
        atomicCAS(err, 0, NF_DEVERR_EP_WAIT);
    __syncthreads();
    if (threadIdx.x == 0) *epoch = e;
}

// NCCL transport: the row blocks received from every source ([src][T][n_src])
// scattered into the gather buffer of the current call, then the epoch.
__global__ void tp_scatter_kernel(const float* __restrict__ recv, int64_t rows_total, int T, int world,
                                  uint8_t* __restrict__ mbox, int64_t cap, uint32_t* __restrict__ epoch) {
    const uint32_t e = *epoch + 1u;
    float* out = reinterpret_cast<float*>(mbox + kFlagsBytes + static_cast<int64_t>(e & 1u) * cap);
    const int64_t n = static_cast<int64_t>(T) * rows_total;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // source block: rows [r0, r1) of every token, stored contiguously
        const int64_t t = i / rows_total, row = i % rows_total;
        int src = static_cast<int>((row * world) / rows_total);
        while (src + 1 < world && row >= ((src + 1) * rows_total) / world) ++src;
        while (src > 0 && row < (src * rows_total) / world) --src;
        const int64_t r0 = (src * rows_total) / world, r1 = ((src + 1) * rows_total) / world;
        const int64_t base = T * r0;  // blocks are [src][T][n_src], n_src = r1 - r0: earlier blocks hold T * r0 values
        out[i] = recv[base + t * (r1 - r0) + (row - r0)];
    }
}
__global__ void tp_advance_kernel(uint32_t* __restrict__ epoch) {
    if (threadIdx.x == 0) *epoch = *epoch + 1u;
}

// y = the current result [T, rows] (gather buffer of parity epoch & 1).
__global__ void tp_copy_kernel(const uint8_t* __restrict__ mbox, int64_t cap, const uint32_t* __restrict__ epoch,
                               int64_t n, float* __restrict__ y) {
    const float* src = reinterpret_cast<const float*>(mbox + kFlagsBytes + static_cast<int64_t>(*epoch & 1u) * cap);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = src[i];
}

// The reference's argmax over a token's logits (TextModel::argmax,
// src/text_forward.cpp:668-681): best = row 0; a later row replaces it only
// when its value compares strictly greater.  So a NaN never wins, a NaN at
// row 0 is never replaced, and among equal values (+0 and -0 included) the
// lowest row wins.  One CTA per token; per-thread bests reduced with that rule.
struct ArgBest {
    float v;
    int i;  // -1: no candidate yet
};
__device__ __forceinline__ ArgBest arg_pick(ArgBest a, ArgBest b) {
    if (a.i < 0) return b;
    if (b.i < 0) return a;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return a.i < b.i ? a : b;  // equal values: the lower row
}
__global__ void __launch_bounds__(1024) tp_argmax_kernel(const uint8_t* __restrict__ mbox, int64_t cap,
                                                         const uint32_t* __restrict__ epoch, int64_t rows,
                                                         int32_t* __restrict__ idx) {
    const float* lg = reinterpret_cast<const float*>(mbox + kFlagsBytes + static_cast<int64_t>(*epoch & 1u) * cap) +
                      static_cast<int64_t>(blockIdx.x) * rows;
    __shared__ ArgBest s_best[32];
    ArgBest b{0.f, -1};
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
        const float v = lg[r];
        if (isnan(v)) continue;  // never wins (row 0 handled below)
        b = arg_pick(b, ArgBest{v, static_cast<int>(r)});
    }
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest c;
        c.v = __shfl_down_sync(0xffffffffu, b.v, o);
        c.i = __shfl_down_sync(0xffffffffu, b.i, o);
        b = arg_pick(b, c);
    }
    if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = b;
    __syncthreads();
    if (threadIdx.x < 32) {
        b = threadIdx.x < (blockDim.x >> 5) ? s_best[threadIdx.x] : ArgBest{0.f, -1};
        for (int o = 16; o > 0; o >>= 1) {
            ArgBest c;
            c.v = __shfl_down_sync(0xffffffffu, b.v, o);
            c.i = __shfl_down_sync(0xffffffffu, b.i, o);
            b = arg_pick(b, c);
        }
        if (threadIdx.x == 0) idx[blockIdx.x] = isnan(lg[0]) || b.i < 0 ? 0 : b.i;
    }
}

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

struct nf_tp {
    int device = 0, rank = 0, world = 1;
    int max_tokens = 0;
    int64_t max_rows = 0;
    int64_t cap = 0;                 // bytes of one gather buffer
    bool p2p = false;                // NVLink peer stores (else NCCL, or world == 1)
    void* nccl = nullptr;            // ncclComm_t
    cudaStream_t stream = nullptr;   // set-up exchanges
    uint8_t* mbox = nullptr;         // flags + two gather buffers (exported over IPC when p2p)
    TpPeers peers{};                 // every rank's mailbox mapped here (own included)
    uint8_t* stage = nullptr;        // set-up records, then (NCCL) this rank's rows [T][n]
    float* recv = nullptr;           // NCCL: every source's rows [src][T][n_src]
    uint32_t* epoch = nullptr;       // calls completed (device counter, equal on every rank)
    int* done = nullptr;             // last-CTA counter of the GEMV kernel
    int* err = nullptr;              // device error word
    std::vector<void*> allocs;
    std::string msg;

    int fail(int status, const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        msg = buf;
        return status;
    }
    template <typename T>
    bool alloc(T** p, size_t count) {
        void* q = nullptr;
        if (cudaMalloc(&q, count * sizeof(T) > 0 ? count * sizeof(T) : 16) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return true;
    }
};

namespace {

thread_local std::string g_tp_create_error;

void tp_release(nf_tp* h) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    for (int p = 0; p < kTpMaxRanks; ++p)
        if (h->peers.mbox[p] && h->peers.mbox[p] != h->mbox) cudaIpcCloseMemHandle(h->peers.mbox[p]);
    if (h->nccl) nccl().comm_destroy(static_cast<ncclComm_t>(h->nccl));
    for (void* q : h->allocs) cudaFree(q);
    if (h->stream) cudaStreamDestroy(h->stream);
    cudaSetDevice(prev);
    delete h;
}

// The collective set-up of a group with world > 1: mailboxes exported and
// mapped over CUDA IPC (or the NCCL transport), with every rank taking the
// same exchanges whatever fails locally (as for expert parallelism).
int tp_setup_group(nf_tp* h, bool mbox_ok, std::string* err) {
    const int R = h->world, me = h->rank;
    struct Rec {
        cudaIpcMemHandle_t handle;
        int32_t ok;      // mailbox exported
        int32_t sound;   // local set-up succeeded (a zeroed record: failed)
        int32_t pad[14];
    };
    static_assert(sizeof(Rec) <= kTpRecBytes && sizeof(Rec) % 16 == 0, "record size");
    const char* tr = std::getenv("NF_TP_TRANSPORT");
    const bool want = tr ? std::strcmp(tr, "nccl") != 0 : true;
    Rec mine{};
    mine.sound = mbox_ok ? 1 : 0;
    mine.ok = mbox_ok && want && cudaIpcGetMemHandle(&mine.handle, h->mbox) == cudaSuccess;
    cudaGetLastError();
    std::vector<Rec> all(static_cast<size_t>(R));
    if (!nccl_allgather_records(h->nccl, h->stage, h->stream, R, &mine, sizeof(Rec), all.data())) {
        *err = "gather buffer handle exchange failed";
        return NF_ERR_CUDA;
    }
    for (int p = 0; p < R; ++p)
        if (!all[static_cast<size_t>(p)].sound) {
            char m[96];
            std::snprintf(m, sizeof(m), "tensor-parallel set-up failed on rank %d (device allocation)", p);
            *err = m;
            return NF_ERR_NOMEM;
        }
    int opened = 1;
    for (int p = 0; p < R; ++p) opened &= all[static_cast<size_t>(p)].ok ? 1 : 0;
    h->peers.mbox[me] = h->mbox;
    for (int p = 0; p < R && opened; ++p) {
        if (p == me) continue;
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[static_cast<size_t>(p)].handle, cudaIpcMemLazyEnablePeerAccess) !=
            cudaSuccess) {
            cudaGetLastError();
            opened = 0;
            break;
        }
        h->peers.mbox[p] = static_cast<uint8_t*>(ptr);
    }
    Rec done{};
    done.ok = opened;
    done.sound = 1;
    if (!nccl_allgather_records(h->nccl, h->stage, h->stream, R, &done, sizeof(Rec), all.data())) {
        *err = "gather buffer mapping agreement failed";
        return NF_ERR_CUDA;
    }
    int every = 1;
    for (int p = 0; p < R; ++p) every &= all[static_cast<size_t>(p)].ok ? 1 : 0;
    if (every) {
        h->p2p = true;
        return NF_OK;
    }
    for (int p = 0; p < R; ++p)
        if (p != me && h->peers.mbox[p]) cudaIpcCloseMemHandle(h->peers.mbox[p]);
    for (int p = 0; p < kTpMaxRanks; ++p) h->peers.mbox[p] = nullptr;
    h->peers.mbox[0] = h->mbox;  // the NCCL transport's GEMV stores locally only
    // NCCL transport: every source's row blocks are received here
    struct Ok {
        int32_t ok;
        int32_t pad[3];
    } ok_mine{h->alloc(&h->recv, static_cast<size_t>(h->max_tokens) * h->max_rows) ? 1 : 0, {}};
    std::vector<Ok> oks(static_cast<size_t>(R));
    if (!nccl_allgather_records(h->nccl, h->stage, h->stream, R, &ok_mine, sizeof(Ok), oks.data())) {
        *err = "allocation agreement failed";
        return NF_ERR_CUDA;
    }
    for (const Ok& o : oks)
        if (!o.ok) {
            *err = "device allocation failed";
            return NF_ERR_NOMEM;
        }
    return NF_OK;
}

template <int TPT>
cudaError_t launch_gemv(const uint16_t* w, const float* x, int64_t rows, int64_t row0, int nrows, int cols, int T,
                        const TpPeers& peers, int world, int me, int64_t cap, float* stage, const uint32_t* epoch,
                        int* done, cudaStream_t st) {
    const dim3 grid(static_cast<unsigned>(std::max(1, (nrows + kGemvRows - 1) / kGemvRows)),
                    static_cast<unsigned>((T + TPT - 1) / TPT));
    tp_gemv_kernel<TPT><<<grid, kGemvRows, 0, st>>>(w, x, rows, row0, nrows, cols, T, peers, world, me, cap, stage,
                                                    epoch, done);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

int nf_tp_split(int64_t rows, int rank, int world, int64_t* row0, int64_t* row1) {
    if (!row0 || !row1 || rows < 0 || world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world)
        return NF_ERR_INVALID;
    *row0 = rows * rank / world;
    *row1 = rows * (rank + 1) / world;
    return NF_OK;
}

int nf_tp_create(int device, int rank, int world, const uint8_t* group_id, int id_len, int max_tokens,
                 int64_t max_rows, nf_tp** out) {
    std::string& err = g_tp_create_error;
    err.clear();
    if (!out) {
        err = "null output handle";
        return NF_ERR_INVALID;
    }
    *out = nullptr;
    if (world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world) {
        err = "tensor parallelism needs 1 <= world <= 8 and 0 <= rank < world";
        return NF_ERR_UNSUPPORTED;
    }
    if (world > 1 && (!group_id || id_len < NF_EP_ID_BYTES)) {
        err = "a group of more than one rank needs a group id (nf_ep_unique_id)";
        return NF_ERR_INVALID;
    }
    if (max_tokens < 1 || max_rows < 1 || max_rows > (int64_t(1) << 31)) {
        err = "max_tokens and max_rows must be positive (max_rows < 2^31)";
        return NF_ERR_INVALID;
    }
    if (world > 1 && !nccl().ok) {
        err = nccl().why;
        return NF_ERR_UNSUPPORTED;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        err = "cannot use the requested device";
        return NF_ERR_CUDA;
    }
    nf_tp* h = new nf_tp();
    h->device = device;
    h->rank = rank;
    h->world = world;
    h->max_tokens = max_tokens;
    h->max_rows = max_rows;
    h->cap = align256(static_cast<int64_t>(max_tokens) * max_rows * 4);
    // small buffers first (before any collective); the gather buffers' failure is
    // reported through the set-up exchange so that no rank is left waiting
    const int64_t shard = (max_rows + world - 1) / world + 1;
    bool ok = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) == cudaSuccess &&
              h->alloc(&h->epoch, 1) && h->alloc(&h->done, 1) && h->alloc(&h->err, 1) &&
              h->alloc(&h->stage, std::max<size_t>(kTpRecBytes * (world + 1),
                                                   world > 1 ? static_cast<size_t>(max_tokens) * shard * 4 : 0));
    if (!ok) {
        cudaGetLastError();
        tp_release(h);
        cudaSetDevice(prev);
        err = "device allocation failed";
        return NF_ERR_NOMEM;
    }
    const bool mbox_ok = h->alloc(&h->mbox, static_cast<size_t>(kFlagsBytes + 2 * h->cap)) &&
                         cudaMemset(h->mbox, 0, kFlagsBytes) == cudaSuccess &&
                         cudaMemset(h->epoch, 0, 4) == cudaSuccess && cudaMemset(h->done, 0, 4) == cudaSuccess &&
                         cudaMemset(h->err, 0, 4) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    if (!mbox_ok) cudaGetLastError();
    int st = NF_OK;
    if (world == 1) {
        if (!mbox_ok) {
            st = NF_ERR_NOMEM;
            err = "device allocation failed";
        } else {
            h->peers.mbox[0] = h->mbox;
            h->p2p = true;
        }
    } else {
        ncclUniqueId id;
        std::memcpy(&id, group_id, sizeof(id));
        ncclComm_t comm = nullptr;
        const ncclResult_t r = nccl().comm_init_rank(&comm, world, id, rank);
        if (r != ncclSuccess) {
            err = std::string("ncclCommInitRank: ") + nccl_str(r);
            st = NF_ERR_CUDA;
        } else {
            h->nccl = comm;
            st = tp_setup_group(h, mbox_ok, &err);
        }
    }
    cudaSetDevice(prev);
    if (st != NF_OK) {
        tp_release(h);
        return st;
    }
    *out = h;
    return NF_OK;
}

void nf_tp_destroy(nf_tp* h) {
    if (h) tp_release(h);
}

const char* nf_tp_last_error(const nf_tp* h) { return h ? h->msg.c_str() : g_tp_create_error.c_str(); }

int nf_tp_transport(const nf_tp* h) {
    if (!h || h->world == 1) return NF_EP_NONE;
    return h->p2p ? NF_EP_NVLINK : NF_EP_NCCL;
}

int nf_tp_linear_bf16(nf_tp* h, const uint16_t* w, int64_t rows, int64_t cols, const float* x, int tokens, float* y,
                      void* stream) {
    if (!h) return NF_ERR_INVALID;
    h->msg.clear();
    int64_t r0 = 0, r1 = 0;
    if (rows >= 0) nf_tp_split(rows, h->rank, h->world, &r0, &r1);
    // (a rank whose row block is empty -- rows < world -- reads no weights)
    if ((!w && r1 > r0) || !x) return h->fail(NF_ERR_INVALID, "null weight or input pointer");
    if (rows < 1 || cols < 4 || cols % 4 != 0 || cols > (int64_t(1) << 30))
        return h->fail(NF_ERR_SHAPE, "BF16 linear layout: rows must be positive and cols a positive multiple of 4");
    if (rows > h->max_rows) return h->fail(NF_ERR_CAPACITY, "rows %lld exceed the handle's max_rows %lld",
                                            static_cast<long long>(rows), static_cast<long long>(h->max_rows));
    if (tokens < 0 || tokens > h->max_tokens)
        return h->fail(NF_ERR_CAPACITY, "tokens must be in [0, max_tokens = %d]", h->max_tokens);
    if (reinterpret_cast<uintptr_t>(w) % 8 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
        (y && reinterpret_cast<uintptr_t>(y) % 4 != 0))
        return h->fail(NF_ERR_LAYOUT, "weights must be 8-byte and x 16-byte aligned");
    if (tokens == 0) return NF_OK;
    const int nrows = static_cast<int>(r1 - r0);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    const int wdst = h->p2p ? h->world : 1;
    float* stage = h->p2p ? nullptr : reinterpret_cast<float*>(h->stage);
    if (h->p2p) {
        tp_begin_kernel<<<1, 32, 0, s>>>(h->peers, h->world, h->rank, h->epoch, h->err);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        // (a rank with no rows -- rows < world -- still launches one CTA, which
        // publishes its flag)
        const int T = tokens, ci = static_cast<int>(cols);
        if (T >= 8) e = launch_gemv<8>(w, x, rows, r0, nrows, ci, T, h->peers, wdst, h->rank, h->cap, stage, h->epoch, h->done, s);
        else if (T >= 4) e = launch_gemv<4>(w, x, rows, r0, nrows, ci, T, h->peers, wdst, h->rank, h->cap, stage, h->epoch, h->done, s);
        else if (T >= 2) e = launch_gemv<2>(w, x, rows, r0, nrows, ci, T, h->peers, wdst, h->rank, h->cap, stage, h->epoch, h->done, s);
        else e = launch_gemv<1>(w, x, rows, r0, nrows, ci, T, h->peers, wdst, h->rank, h->cap, stage, h->epoch, h->done, s);
    }
    if (e == cudaSuccess && h->p2p) {
        tp_wait_kernel<<<1, 32, 0, s>>>(h->mbox, h->world, h->epoch, h->err);
        e = cudaGetLastError();
    } else if (e == cudaSuccess) {
        // NCCL transport: exchange the row blocks, scatter them into the gather buffer
        NcclApi& api = nccl();
        ncclComm_t comm = static_cast<ncclComm_t>(h->nccl);
        ncclResult_t r = api.group_start();
        for (int p = 0; p < h->world && r == ncclSuccess; ++p) {
            int64_t q0 = 0, q1 = 0;
            nf_tp_split(rows, p, h->world, &q0, &q1);
            const size_t n_mine = static_cast<size_t>(tokens) * nrows, n_src = static_cast<size_t>(tokens) * (q1 - q0);
            if (n_mine) r = api.send(stage, n_mine, ncclFloat32, p, comm, s);
            if (r == ncclSuccess && n_src)
                r = api.recv(h->recv + static_cast<int64_t>(tokens) * q0, n_src, ncclFloat32, p, comm, s);
        }
        const ncclResult_t r2 = api.group_end();
        if (r == ncclSuccess) r = r2;
        if (r != ncclSuccess) {
            cudaSetDevice(prev);
            return h->fail(NF_ERR_CUDA, "row exchange: %s", nccl_str(r));
        }
        const int64_t n = static_cast<int64_t>(tokens) * rows;
        tp_scatter_kernel<<<static_cast<unsigned>(std::min<int64_t>(1184, (n + 255) / 256)), 256, 0, s>>>(
            h->recv, rows, tokens, h->world, h->mbox, h->cap, h->epoch);
        tp_advance_kernel<<<1, 32, 0, s>>>(h->epoch);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && y) {
        const int64_t n = static_cast<int64_t>(tokens) * rows;
        tp_copy_kernel<<<static_cast<unsigned>(std::min<int64_t>(1184, (n + 255) / 256)), 256, 0, s>>>(
            h->mbox, h->cap, h->epoch, n, y);
        e = cudaGetLastError();
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->fail(NF_ERR_CUDA, "tensor-parallel linear launch: %s", cudaGetErrorString(e));
    return NF_OK;
}

int nf_tp_argmax(nf_tp* h, int tokens, int64_t rows, int32_t* idx, void* stream) {
    if (!h) return NF_ERR_INVALID;
    h->msg.clear();
    if (!idx) return h->fail(NF_ERR_INVALID, "null index pointer");
    if (tokens < 0 || tokens > h->max_tokens || rows < 1 || rows > h->max_rows)
        return h->fail(NF_ERR_CAPACITY, "tokens or rows beyond the handle's capacity");
    if (tokens == 0) return NF_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    tp_argmax_kernel<<<tokens, 1024, 0, static_cast<cudaStream_t>(stream)>>>(h->mbox, h->cap, h->epoch, rows, idx);
    const cudaError_t e = cudaGetLastError();
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->fail(NF_ERR_CUDA, "argmax launch: %s", cudaGetErrorString(e));
    return NF_OK;
}

int nf_tp_result(nf_tp* h, const float** out_dev) {
    if (!h || !out_dev) return NF_ERR_INVALID;
    // the host cannot read the device epoch without synchronising: report both
    // buffers' base via the parity the device holds after a sync
    uint32_t ep = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    const cudaError_t e = cudaMemcpy(&ep, h->epoch, 4, cudaMemcpyDeviceToHost);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->fail(NF_ERR_CUDA, "epoch read: %s", cudaGetErrorString(e));
    *out_dev = reinterpret_cast<const float*>(h->mbox + kFlagsBytes + static_cast<int64_t>(ep & 1u) * h->cap);
    return NF_OK;
}

int nf_tp_sync(nf_tp* h, void* stream) {
    if (!h) return NF_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    int dev_err = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&dev_err, h->err, 4, cudaMemcpyDeviceToHost);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->fail(NF_ERR_CUDA, "synchronise: %s", cudaGetErrorString(e));
    if (dev_err != 0)
        return h->fail(NF_ERR_TIMEOUT, "a peer's rows or acknowledgement never arrived (bounded wait, code %d); "
                                       "the group is out of step and must be recreated", dev_err);
    return NF_OK;
}

}  // extern "C"
