// nf_kernels.cu -- router, token permutation / dispatch (with the fused
// NVFP4 activation quantiser), weighted combine + residual, and the
// stand-alone format kernels (dequantise, quantise, reference sigmoid).
//
// These kernels are HBM- or latency-bound integer/byte and scalar work; they
// use plain coalesced loads, shared-memory staging and grids sized from the
// SM count.  The contractions live in nf_gemm.cu.
#include "nf_common.cuh"
#include "nf_gemm_shared.cuh"
#include "nf_internal.h"

#include "_gen/sigmoid_table.inc"

#include <algorithm>

namespace nf {

// ---------------------------------------------------------------------------
// Sigmoid exactly as the reference computes it (src/text_forward.cpp:42-49).
// exp is evaluated in double and rounded once (a correctly rounded expf).
// libm's expf can only differ from that next to a float rounding boundary,
// so the arguments whose exp lies within a relative NF_SIG_NEAR_EPS of one
// (checked by rounding the double value nudged both ways) look themselves up
// in the build-time exception table, found through a 2^20-bucket index over
// the key bits (bucket = bits >> 12; at most a few dozen keys, one or two
// cache lines, per bucket).  The generator proves that every table entry is
// caught by this screen.
// ---------------------------------------------------------------------------
constexpr int kSigBucketShift = 12;
constexpr int kSigBuckets = 1 << (32 - kSigBucketShift);
__device__ uint32_t g_sig_index[kSigBuckets + 1];

__global__ void sig_index_kernel() {
    for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b <= kSigBuckets;
         b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // first key >= b << shift (lower bound)
        const uint64_t target = static_cast<uint64_t>(b) << kSigBucketShift;
        int lo = 0, hi = NF_SIG_TABLE_N;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (static_cast<uint64_t>(g_sig_keys[mid]) < target) lo = mid + 1;
            else hi = mid;
        }
        g_sig_index[b] = static_cast<uint32_t>(lo);
    }
}

__device__ __noinline__ float sigmoid_lookup(float x, float r) {
    const uint32_t key = __float_as_uint(x);
    const uint32_t b = key >> kSigBucketShift;
    const uint32_t hi = g_sig_index[b + 1];
    for (uint32_t j = g_sig_index[b]; j < hi; ++j)
        if (g_sig_keys[j] == key) return __uint_as_float(g_sig_vals[j]);
    return r;
}

__device__ __forceinline__ float sigmoid_ref(float x) {
    const double zd = exp(x >= 0.f ? -static_cast<double>(x) : static_cast<double>(x));
    const float z = __double2float_rn(zd);
    const float r = x >= 0.f ? __fdiv_rn(1.f, __fadd_rn(1.f, z)) : __fdiv_rn(z, __fadd_rn(1.f, z));
    const bool near = !(zd > NF_SIG_TINY) || __double2float_rn(zd * (1.0 + NF_SIG_NEAR_EPS)) != z ||
                      __double2float_rn(zd * (1.0 - NF_SIG_NEAR_EPS)) != z;
    return near ? sigmoid_lookup(x, r) : r;
}

__global__ void sigmoid_ref_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = sigmoid_ref(x[i]);
}

cudaError_t prepare_device_tables() {
    static int ready[kMaxDevices] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (ready[dev]) return cudaSuccess;
    sig_index_kernel<<<1024, 256>>>();
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) ready[dev] = 1;
    return e;
}

// ---------------------------------------------------------------------------
// Router logits: gemv_bf16 (src/text_forward.cpp:497-508) for every token:
// logits[t, e] = sum_c bf16(W[e, c]) * x[t, c], accumulated sequentially in
// fp32 in column order with the product rounded before the add, which is
// what makes the result bit-identical to the reference.
//
// A CTA owns kRtExp experts x kRtTok tokens: it stages those router rows and
// token rows in shared memory with 1-D bulk copies (row pitch padded by 16
// bytes so the 8 rows a warp reads fall in distinct banks), then each thread
// runs the chain of one (token, expert) pair: two unpack operations and one
// fused multiply-add per step, so the warp issues fast enough for the chain
// of H dependent adds -- the kernel's latency floor -- to be the bound.
// A product of two BF16 values has at most 16 significant bits, so it is
// exact in fp32 unless it leaves fp32's range; when every nonzero |w| and |x|
// lies in [2^-67, 2^63) (router weights checked at bind, token rows checked
// here in shared memory) the product is exact and fma(w, x, acc) equals the
// reference's round(acc + round(w * x)).  Otherwise the CTA runs the
// separately rounded multiply and add.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

constexpr int kRtExp = 8;    // experts per CTA
constexpr int kRtTok = 8;    // tokens per CTA
constexpr int kRtThreads = kRtExp * kRtTok;
constexpr int kRtMaxChunk = 4096;  // K elements staged at a time

// true when a BF16 pair holds a value whose product with another in-range
// BF16 value could leave fp32's exact range (nonzero |v| outside
// [2^-67, 2^63), inf or NaN)
__device__ __forceinline__ bool bf16x2_unsafe(uint32_t u) {
    const uint32_t e0 = (u >> 7) & 0xffu, e1 = (u >> 23) & 0xffu;
    const bool nz0 = (u & 0x7fffu) != 0u, nz1 = (u & 0x7fff0000u) != 0u;
    return (nz0 && (e0 < 60u || e0 > 189u)) || (nz1 && (e1 < 60u || e1 > 189u));
}

template <bool kFma>
__device__ __forceinline__ float chain_step2(uint32_t wv, uint32_t xv, float acc) {
    if (kFma) {
        acc = fmaf(bf16_lo(wv), bf16_lo(xv), acc);
        acc = fmaf(bf16_hi(wv), bf16_hi(xv), acc);
    } else {
        acc = __fadd_rn(acc, __fmul_rn(bf16_lo(wv), bf16_lo(xv)));
        acc = __fadd_rn(acc, __fmul_rn(bf16_hi(wv), bf16_hi(xv)));
    }
    return acc;
}

// One chain over n8 groups of 8 elements from shared memory; the next
// group's two 16-byte loads are issued before the current group's 8
// dependent steps, so the load latency hides behind the chain.
template <bool kFma>
__device__ __forceinline__ float chain(const uint4* __restrict__ wr, const uint4* __restrict__ xr, int n8, float acc) {
    uint4 w = wr[0], a = xr[0];
    for (int c = 0; c < n8; ++c) {
        const int nx = c + 1 < n8 ? c + 1 : c;
        const uint4 wn = wr[nx], an = xr[nx];
        acc = chain_step2<kFma>(w.x, a.x, acc);
        acc = chain_step2<kFma>(w.y, a.y, acc);
        acc = chain_step2<kFma>(w.z, a.z, acc);
        acc = chain_step2<kFma>(w.w, a.w, acc);
        w = wn;
        a = an;
    }
    return acc;
}

__global__ void __launch_bounds__(kRtThreads) router_logits_kernel(const uint16_t* __restrict__ x,
                                                                   const uint16_t* __restrict__ w,
                                                                   const float* __restrict__ bias, int T, int H, int E,
                                                                   int w_safe, float* __restrict__ logits,
                                                                   float* __restrict__ scores,
                                                                   float* __restrict__ choices,
                                                                   int* __restrict__ err) {
    pdl_wait();  // no-op unless launched dependent
    pdl_trigger();  // let the permutation launch
    extern __shared__ __align__(128) uint8_t rt_smem[];
    __shared__ uint64_t bar;
    const int chunk = min(H, kRtMaxChunk);
    const int pitch = chunk * 2 + 16;  // bytes
    uint8_t* ws = rt_smem;
    uint8_t* xs = rt_smem + kRtExp * pitch;
    const int t0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp;
    const int nt = min(kRtTok, T - t0), ne = min(kRtExp, E - e0);
    const int el = threadIdx.x % kRtExp, tl = threadIdx.x / kRtExp;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    float acc = 0.f;
    int ok = 1;
    for (int k0 = 0, phase = 0; k0 < H; k0 += chunk, phase ^= 1) {
        const int kc = min(chunk, H - k0);
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(&bar, static_cast<uint32_t>((ne + nt) * kc * 2));
            for (int r = 0; r < ne; ++r)
                bulk_load(ws + r * pitch, w + static_cast<int64_t>(e0 + r) * H + k0, kc * 2, &bar);
            for (int r = 0; r < nt; ++r)
                bulk_load(xs + r * pitch, x + static_cast<int64_t>(t0 + r) * H + k0, kc * 2, &bar);
        }
        // bounded wait; every thread polls the same barrier
        const uint64_t start = globaltimer_ns();
        while (!mbar_try_wait_sleep(&bar, static_cast<uint32_t>(phase), 20000u)) {
            if (globaltimer_ns() - start > NF_WAIT_BUDGET_NS) {
                ok = 0;
                break;
            }
        }
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
            return;
        }
        // range check of the staged token rows
        int unsafe = 0;
        for (int r = 0; r < nt; ++r) {
            const uint4* row = reinterpret_cast<const uint4*>(xs + r * pitch);
            for (int c = threadIdx.x; c < kc / 8; c += blockDim.x) {
                const uint4 q = row[c];
                unsafe |= (bf16x2_unsafe(q.x) | bf16x2_unsafe(q.y) | bf16x2_unsafe(q.z) | bf16x2_unsafe(q.w)) ? 1 : 0;
            }
        }
        const bool use_fma = w_safe && !__syncthreads_or(unsafe);
        const uint4* wr = reinterpret_cast<const uint4*>(ws + el * pitch);
        const uint4* xr = reinterpret_cast<const uint4*>(xs + tl * pitch);
        acc = use_fma ? chain<true>(wr, xr, kc / 8, acc) : chain<false>(wr, xr, kc / 8, acc);
        __syncthreads();  // the next chunk overwrites the staged rows
    }
    if (el < ne && tl < nt) {
        // router_select's per-expert part (src/text_forward.cpp:1453-1456):
        // score = sigmoid(logit), choice = score + correction bias
        const int64_t o = static_cast<int64_t>(t0 + tl) * E + e0 + el;
        const float sc = sigmoid_ref(acc);
        logits[o] = acc;
        scores[o] = sc;
        choices[o] = __fadd_rn(sc, bias[e0 + el]);
    }
}

// ---------------------------------------------------------------------------
// Router selection: router_select (src/text_forward.cpp:1447-1471) on the
// scores and choices the logits kernel wrote.  One warp per token.  With n_group > 1 the group-limited
// form (a group scores the sum of its two best choices, topk_group groups
// stay eligible, lower group index on ties) masks the other experts first;
// the reference has no group limit.
// ---------------------------------------------------------------------------
constexpr int kSelectWarps = 4;

// One warp selects the top-k experts of one token from its scores and
// choices (global or shared memory) and writes K indices and weights.
// `excl` is a 32-word scratch of the warp (shared memory).
__device__ __forceinline__ void warp_select(const float* score, const float* choice, int E, int K, float scaling,
                                            int normalize, int n_group, int topk_group, uint32_t* excl,
                                            int32_t* __restrict__ idx_row, float* __restrict__ w_row) {
    const int lane = threadIdx.x & 31;
    // experts excluded by the group limit (computed by lane 0, rare path)
    excl[lane] = 0u;
    __syncwarp();
    if (n_group > 1 && topk_group < n_group) {
        if (lane == 0) {
            const int per = E / n_group;
            uint32_t keep = 0u;  // n_group <= 32
            for (int r = 0; r < topk_group; ++r) {
                int best = -1;
                float best_score = 0.f;
                for (int g = 0; g < n_group; ++g) {
                    if (keep & (1u << g)) continue;
                    float b1 = -INFINITY, b2 = -INFINITY;
                    for (int j = 0; j < per; ++j) {
                        const float c = choice[g * per + j];
                        if (c > b1) {
                            b2 = b1;
                            b1 = c;
                        } else if (c > b2) {
                            b2 = c;
                        }
                    }
                    const float s = per >= 2 ? __fadd_rn(b1, b2) : b1;
                    if (best < 0 || s > best_score) {
                        best = g;
                        best_score = s;
                    }
                }
                keep |= 1u << best;
            }
            for (int e = 0; e < E; ++e)
                if (!(keep & (1u << (e / per)))) excl[e >> 5] |= 1u << (e & 31);
        }
        __syncwarp();
    }
    // The reference scans from the first unused expert and moves on a strict
    // '>' only: so a NaN first choice is kept, NaN choices are never taken
    // otherwise, and the pick is the largest non-NaN choice with the lowest
    // index among equals.  Lane l owns experts l, l + 32, ... and the warp
    // reduces (first unused, best non-NaN) per pick.
    const int jn = (E + 31) / 32;
    uint32_t used = 0u;  // bit j: expert lane + 32 j taken or excluded
    for (int j = 0; j < jn; ++j) {
        const int e = lane + 32 * j;
        if (e >= E || ((excl[e >> 5] >> (e & 31)) & 1u)) used |= 1u << j;
    }
    int picks[32];
    float wts[32];
    for (int p = 0; p < K; ++p) {
        int first = 0x7fffffff, best = -1;
        float bv = 0.f;
        for (int j = 0; j < jn; ++j) {
            if (used & (1u << j)) continue;
            const int e = lane + 32 * j;
            if (e < first) first = e;
            const float c = choice[e];
            if (!isnan(c) && (best < 0 || c > bv)) {
                best = e;
                bv = c;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            first = min(first, __shfl_xor_sync(0xffffffffu, first, off));
            const int ob = __shfl_xor_sync(0xffffffffu, best, off);
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            if (ob >= 0 && (best < 0 || ov > bv || (ov == bv && ob < best))) {
                best = ob;
                bv = ov;
            }
        }
        int pick = 0;
        if (first != 0x7fffffff) pick = (isnan(choice[first]) || best < 0) ? first : best;
        if ((pick & 31) == lane) used |= 1u << (pick >> 5);
        picks[p] = pick;
        wts[p] = score[pick];
    }
    if (lane != 0) return;
    if (normalize) {
        float sum = 1e-20f;
        for (int p = 0; p < K; ++p) sum = __fadd_rn(sum, wts[p]);
        for (int p = 0; p < K; ++p) wts[p] = __fmul_rn(__fdiv_rn(wts[p], sum), scaling);
    }
    for (int p = 0; p < K; ++p) {
        idx_row[p] = picks[p];
        w_row[p] = wts[p];
    }
}

// warp_select with the token's scores and choices held in registers (lane l
// owns experts l + 32 j, j < JN, so E <= 32 JN): each pick is two ballots
// (the first eligible expert) and one 64-bit max-reduction over keys
// (order-preserving bits of the choice, then the complement of the expert
// index: the largest non-NaN choice, lowest index among equals), instead of
// re-reading shared memory and reducing three values per level.  Lane p
// keeps pick p (K <= 32), so the weights are normalised by K lanes at once
// after a sum taken in pick order.  Same results as warp_select.
__device__ __forceinline__ uint32_t float_order_bits(float c) {
    const uint32_t u = __float_as_uint(__fadd_rn(c, 0.f));  // -0 -> +0: equal choices get equal keys
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int JN>
__device__ __forceinline__ void warp_select_reg(const float* score, const float* choice, int E, int K, float scaling,
                                                int normalize, int n_group, int topk_group, uint32_t* excl,
                                                int32_t* __restrict__ idx_row, float* __restrict__ w_row) {
    const int lane = threadIdx.x & 31;
    excl[lane] = 0u;
    __syncwarp();
    if (n_group > 1 && topk_group < n_group) {
        if (lane == 0) {
            const int per = E / n_group;
            uint32_t keep = 0u;
            for (int r = 0; r < topk_group; ++r) {
                int best = -1;
                float best_score = 0.f;
                for (int g = 0; g < n_group; ++g) {
                    if (keep & (1u << g)) continue;
                    float b1 = -INFINITY, b2 = -INFINITY;
                    for (int j = 0; j < per; ++j) {
                        const float c = choice[g * per + j];
                        if (c > b1) {
                            b2 = b1;
                            b1 = c;
                        } else if (c > b2) {
                            b2 = c;
                        }
                    }
                    const float s = per >= 2 ? __fadd_rn(b1, b2) : b1;
                    if (best < 0 || s > best_score) {
                        best = g;
                        best_score = s;
                    }
                }
                keep |= 1u << best;
            }
            for (int e = 0; e < E; ++e)
                if (!(keep & (1u << (e / per)))) excl[e >> 5] |= 1u << (e & 31);
        }
        __syncwarp();
    }
    float ch[JN], sc[JN];
    uint32_t avail = 0u;  // bit j: expert lane + 32 j exists, is not excluded and not yet taken
#pragma unroll
    for (int j = 0; j < JN; ++j) {
        const int e = lane + 32 * j;
        ch[j] = 0.f;
        sc[j] = 0.f;
        if (e < E) {
            ch[j] = choice[e];
            sc[j] = score[e];
            if (!((excl[e >> 5] >> (e & 31)) & 1u)) avail |= 1u << j;
        }
    }
    int my_pick = 0;
    float my_w = 0.f;
    for (int p = 0; p < K; ++p) {
        int first = -1;
#pragma unroll
        for (int j = JN - 1; j >= 0; --j) {
            const uint32_t b = __ballot_sync(0xffffffffu, (avail >> j) & 1u);
            if (b) first = 32 * j + __ffs(b) - 1;
        }
        uint64_t key = 0;
#pragma unroll
        for (int j = 0; j < JN; ++j) {
            if (((avail >> j) & 1u) && !isnan(ch[j])) {
                const uint64_t k = (static_cast<uint64_t>(float_order_bits(ch[j])) << 32) |
                                   (0xffffffffu - static_cast<uint32_t>(lane + 32 * j));
                key = k > key ? k : key;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, key, off);
            key = o > key ? o : key;
        }
        int pick = 0;
        if (first >= 0) {
            float cf = ch[0];
#pragma unroll
            for (int j = 1; j < JN; ++j)
                if ((first >> 5) == j) cf = ch[j];
            cf = __shfl_sync(0xffffffffu, cf, first & 31);
            pick = (isnan(cf) || key == 0) ? first : static_cast<int>(0xffffffffu - static_cast<uint32_t>(key));
        }
        if ((pick & 31) == lane) avail &= ~(1u << (pick >> 5));
        float w = sc[0];
#pragma unroll
        for (int j = 1; j < JN; ++j)
            if ((pick >> 5) == j) w = sc[j];
        w = __shfl_sync(0xffffffffu, w, pick & 31);
        if (lane == p) my_pick = pick, my_w = w;
    }
    if (normalize) {
        float sum = 1e-20f;
        for (int p = 0; p < K; ++p) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_w, p));
        my_w = __fmul_rn(__fdiv_rn(my_w, sum), scaling);
    }
    if (lane < K) {
        idx_row[lane] = my_pick;
        w_row[lane] = my_w;
    }
}

__global__ void __launch_bounds__(kSelectWarps * 32) router_select_kernel(
    const float* __restrict__ scores, const float* __restrict__ choices, int T, int E, int K, float scaling,
    int normalize, int n_group, int topk_group, int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
    __shared__ uint32_t s_excl[kSelectWarps][32];  // E <= 1024 bits
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.x * kSelectWarps + warp;
    if (t >= T) return;
    warp_select(scores + static_cast<int64_t>(t) * E, choices + static_cast<int64_t>(t) * E, E, K, scaling, normalize,
                n_group, topk_group, s_excl[warp], idx_out + static_cast<int64_t>(t) * K,
                w_out + static_cast<int64_t>(t) * K);
}

// One thread selects the top-k experts of one token, scanning its choices
// (shared memory) in expert order exactly as router_select does: each pick
// starts from the first unused expert and moves on a strict '>' only (lowest
// index wins ties, a NaN first choice is kept, later NaNs are never taken).
// The group limit, when on, first marks the experts of the groups that lose.
// `used` is a per-token byte scratch of E entries.
__device__ __forceinline__ void thread_select(const float* score, const float* choice, int E, int K, float scaling,
                                              int normalize, int n_group, int topk_group, uint8_t* used,
                                              int32_t* __restrict__ idx_row, float* __restrict__ w_row) {
    const bool grouped = n_group > 1 && topk_group < n_group;
    const int per = grouped ? E / n_group : E;
    uint32_t keep = 0xffffffffu;
    if (grouped) {
        keep = 0u;
        for (int r = 0; r < topk_group; ++r) {
            int best = -1;
            float best_score = 0.f;
            for (int gi = 0; gi < n_group; ++gi) {
                if (keep & (1u << gi)) continue;
                float b1 = -INFINITY, b2 = -INFINITY;
                for (int j = 0; j < per; ++j) {
                    const float c = choice[gi * per + j];
                    if (c > b1) {
                        b2 = b1;
                        b1 = c;
                    } else if (c > b2) {
                        b2 = c;
                    }
                }
                const float sg = per >= 2 ? __fadd_rn(b1, b2) : b1;
                if (best < 0 || sg > best_score) {
                    best = gi;
                    best_score = sg;
                }
            }
            keep |= 1u << best;
        }
    }
    for (int e = 0; e < E; ++e) used[e] = grouped ? static_cast<uint8_t>(((keep >> (e / per)) & 1u) ^ 1u) : 0;
    int picks[32];
    float wts[32];
    for (int p = 0; p < K; ++p) {
        int best = -1;
        float bc = 0.f;
        for (int e = 0; e < E; ++e) {
            if (used[e]) continue;
            const float c = choice[e];
            if (best < 0 || c > bc) {
                best = e;
                bc = c;
            }
        }
        best = max(best, 0);
        used[best] = 1;
        picks[p] = best;
        wts[p] = score[best];
    }
    if (normalize) {
        float sum = 1e-20f;
        for (int p = 0; p < K; ++p) sum = __fadd_rn(sum, wts[p]);
        for (int p = 0; p < K; ++p) wts[p] = __fmul_rn(__fdiv_rn(wts[p], sum), scaling);
    }
    for (int p = 0; p < K; ++p) {
        idx_row[p] = picks[p];
        w_row[p] = wts[p];
    }
}

// ---------------------------------------------------------------------------
// Fused router for E <= 128 (every configuration of the benchmark): one CTA
// owns `tc` tokens and all experts, so it runs the logits, the sigmoid, the
// bias and the selection without a second launch or a round trip through
// global memory.
//
// Warp-specialised.  The router rows stream through a ring of NS shared-
// memory slots: the producer warp copies the chunk of every row with one bulk
// copy per stage (rows laid out chunk-major at bind, 16 bytes of padding per
// row so the rows a warp reads fall in distinct banks), and the consumer warps
// run the chains without a CTA-wide barrier -- a slot is handed over by its
// `full` mbarrier and handed back by `empty`.  A bulk copy costs a fixed
// latency of several hundred cycles on top of its bytes, so each stage is one
// large copy and token rows never travel by bulk copy:
//   - small batches (kXRes): the CTA's few token rows are loaded once with
//     coalesced loads by every thread, range-checked and widened to fp32 in
//     shared memory for the whole of H; one chain per thread over BF16 router
//     rows (half the bytes to stream; the unpack is free next to the chain of
//     H dependent adds, which is the floor), loads four groups ahead.
//   - large batches: the producer lanes load the next stage's token rows into
//     registers while the consumers work, then widen them into the stage's
//     slot; 8 tokens x 2 experts per consumer thread over fp32 router rows,
//     64 independent FMAs per 10 loads (2 distinct rows, 8 broadcasts).
// ---------------------------------------------------------------------------
constexpr int kFzConsumers = 4;                    // consumer warps
constexpr int kFzCThreads = kFzConsumers * 32;
constexpr int kFzKc = kRouterKc;                   // K elements per chunk
constexpr int kFzXPitch = kFzKc * 4 + 16;          // bytes per widened token row chunk
constexpr int kFzMaxE = kRouterMaxE;
constexpr int kFzMaxResH = 4096;                   // resident token rows: H limit

__host__ __device__ constexpr int fz_group_threads(int E, int ept) { return ((E + 32 * ept - 1) / (32 * ept)) * 32; }
__host__ __device__ constexpr int fz_tokens(int E, int ept, int tpt) { return (kFzCThreads / fz_group_threads(E, ept)) * tpt; }
__host__ __device__ constexpr int fz_wpitch(bool w16) { return w16 ? kRouterPitch16 * 2 : kRouterPitch * 4; }
// kXRes: slot = SUB router chunks; token rows resident after the ring
// (tc rows of H fp32, + 16 bytes).  Else: slot = router chunk + widened token chunk.
__host__ __device__ constexpr size_t fz_slot(int E, int ept, int tpt, int sub, bool w16, bool xres) {
    return static_cast<size_t>(sub) * E * fz_wpitch(w16) +
           (xres ? 0 : static_cast<size_t>(fz_tokens(E, ept, tpt)) * kFzXPitch);
}
__host__ __device__ constexpr size_t fz_smem(int E, int ept, int tpt, int sub, int ns, bool w16, bool xres, int H) {
    return ns * fz_slot(E, ept, tpt, sub, w16, xres) +
           (xres ? static_cast<size_t>(fz_tokens(E, ept, tpt)) * (static_cast<size_t>(H) * 4 + 16) : 0);
}

template <bool kFma>
__device__ __forceinline__ float fz_step(float acc, float w, float x) {
    return kFma ? fmaf(w, x, acc) : __fadd_rn(acc, __fmul_rn(w, x));
}

// One chain over one chunk of BF16 router weights (8 per 16-byte load) and
// widened tokens, loads kAhead groups ahead in a register ring.
template <bool kFma>
__device__ __forceinline__ float chain_fz16(const uint4* __restrict__ wr, const float4* __restrict__ xr, float a) {
    constexpr int kN8 = kFzKc / 8, kAhead = 4;
    uint4 wq[kAhead];
    float4 xq[kAhead][2];
#pragma unroll
    for (int i = 0; i < kAhead; ++i) {
        wq[i] = wr[i];
        xq[i][0] = xr[2 * i];
        xq[i][1] = xr[2 * i + 1];
    }
#pragma unroll
    for (int q = 0; q < kN8; ++q) {
        const uint4 wv = wq[q % kAhead];
        const float4 xa = xq[q % kAhead][0], xb = xq[q % kAhead][1];
        if (q + kAhead < kN8) {
            wq[q % kAhead] = wr[q + kAhead];
            xq[q % kAhead][0] = xr[2 * (q + kAhead)];
            xq[q % kAhead][1] = xr[2 * (q + kAhead) + 1];
        }
        a = fz_step<kFma>(a, bf16_lo(wv.x), xa.x);
        a = fz_step<kFma>(a, bf16_hi(wv.x), xa.y);
        a = fz_step<kFma>(a, bf16_lo(wv.y), xa.z);
        a = fz_step<kFma>(a, bf16_hi(wv.y), xa.w);
        a = fz_step<kFma>(a, bf16_lo(wv.z), xb.x);
        a = fz_step<kFma>(a, bf16_hi(wv.z), xb.y);
        a = fz_step<kFma>(a, bf16_lo(wv.w), xb.z);
        a = fz_step<kFma>(a, bf16_hi(wv.w), xb.w);
    }
    return a;
}

// TPT x EPT chains over one chunk of fp32 router weights and widened tokens.
template <bool kFma, int EPT, int TPT>
__device__ __forceinline__ void chain_fz32(const float4* const (&wr)[EPT], const float4* __restrict__ xr,
                                           float (&acc)[TPT][EPT]) {
    constexpr int kN4 = kFzKc / 4, kXs = kFzXPitch / 16;
#pragma unroll 4
    for (int q = 0; q < kN4; ++q) {
        float4 wv[EPT], xv[TPT];
#pragma unroll
        for (int j = 0; j < EPT; ++j) wv[j] = wr[j][q];
#pragma unroll
        for (int t = 0; t < TPT; ++t) xv[t] = xr[t * kXs + q];
#pragma unroll
        for (int t = 0; t < TPT; ++t)
#pragma unroll
            for (int j = 0; j < EPT; ++j) acc[t][j] = fz_step<kFma>(acc[t][j], wv[j].x, xv[t].x);
#pragma unroll
        for (int t = 0; t < TPT; ++t)
#pragma unroll
            for (int j = 0; j < EPT; ++j) acc[t][j] = fz_step<kFma>(acc[t][j], wv[j].y, xv[t].y);
#pragma unroll
        for (int t = 0; t < TPT; ++t)
#pragma unroll
            for (int j = 0; j < EPT; ++j) acc[t][j] = fz_step<kFma>(acc[t][j], wv[j].z, xv[t].z);
#pragma unroll
        for (int t = 0; t < TPT; ++t)
#pragma unroll
            for (int j = 0; j < EPT; ++j) acc[t][j] = fz_step<kFma>(acc[t][j], wv[j].w, xv[t].w);
    }
}

// Bounded wait on a slot barrier that also gives up once the CTA aborted.
__device__ __forceinline__ bool fz_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
        if (abort && *abort) return false;
        if (globaltimer_ns() - start > NF_WAIT_BUDGET_NS) return false;
    }
}

__device__ __forceinline__ int bf16x8_unsafe(uint4 u) {
    return (bf16x2_unsafe(u.x) | bf16x2_unsafe(u.y) | bf16x2_unsafe(u.z) | bf16x2_unsafe(u.w)) ? 1 : 0;
}

template <int EPT, int TPT, int SUB, int NS, int PW, bool kW16, bool kXRes>
__global__ void __launch_bounds__(kFzCThreads + 32 * PW, 1) router_fused_kernel(
    const uint16_t* __restrict__ x, const void* __restrict__ wz, const float* __restrict__ bias, int T, int H, int E,
    int K, float scaling, int normalize, int n_group, int topk_group, int w_safe, float* __restrict__ logits,
    int32_t* __restrict__ idx_out, float* __restrict__ w_out, int* __restrict__ err) {
    pdl_wait();  // no-op unless launched dependent
    pdl_trigger();  // let the permutation launch
    static_assert(!kW16 || (EPT == 1 && TPT == 1), "BF16 staging serves the one-chain form");
    static_assert(!kXRes || (EPT == 1 && TPT == 1), "resident token rows serve small batches");
    static_assert(kXRes || SUB == 1, "streamed token rows come one chunk per stage");
    constexpr int kThreads = kFzCThreads + 32 * PW;       // consumers + PW producer warps
    constexpr int kXRegs = 16 / PW;  // token pieces a producer thread carries per stage (tc <= 32)
    extern __shared__ __align__(128) uint8_t fz_smem_buf[];
    __shared__ uint64_t full[NS], empty[NS];
    __shared__ int s_unsafe[NS][PW];
    __shared__ int s_abort, s_x_unsafe;
    const int gt = fz_group_threads(E, EPT), tg = kFzCThreads / gt, tc = tg * TPT;
    const int wchunk = E * fz_wpitch(kW16);
    const int wbytes = SUB * wchunk;  // router bytes per stage
    const int slot_bytes = static_cast<int>(fz_slot(E, EPT, TPT, SUB, kW16, kXRes));
    const int t0 = blockIdx.x * tc, nt = min(tc, T - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = H / kFzKc, nstages = (nchunks + SUB - 1) / SUB;
    const int xres_pitch = H * 4 + 16;
    uint8_t* xres = fz_smem_buf + NS * slot_bytes;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], kXRes ? 1 : 32 * PW);
            mbar_init(&empty[i], kFzConsumers);
        }
        s_abort = 0;
        s_x_unsafe = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if constexpr (kXRes) {
        // the first router copies go out at once from the producer thread,
        // while the consumer threads widen the resident token rows (zero past
        // the batch), their loads issued four at a time before the stores
        if (threadIdx.x == kFzCThreads)
            for (int c = 0; c < NS && c < nstages; ++c) {
                const int bytes = min(SUB, nchunks - c * SUB) * wchunk;
                mbar_arrive_expect_tx(&full[c], static_cast<uint32_t>(bytes));
                bulk_load(fz_smem_buf + c * slot_bytes, static_cast<const uint8_t*>(wz) + static_cast<int64_t>(c) * wbytes,
                          static_cast<uint32_t>(bytes), &full[c]);
            }
        int unsafe = 0;
        const int q8 = H / 8;
        constexpr int kB = 4;
        if (threadIdx.x < kFzCThreads)
            for (int i0 = threadIdx.x; i0 < tc * q8; i0 += kB * kFzCThreads) {
                uint4 u[kB];
#pragma unroll
                for (int j = 0; j < kB; ++j) {
                    const int i = i0 + j * kFzCThreads, r = i / q8, q = i - r * q8;
                    u[j] = make_uint4(0u, 0u, 0u, 0u);
                    if (i < tc * q8 && r < nt)
                        u[j] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + r) * H) + q);
                }
#pragma unroll
                for (int j = 0; j < kB; ++j) {
                    const int i = i0 + j * kFzCThreads, r = i / q8, q = i - r * q8;
                    if (i >= tc * q8) break;
                    unsafe |= bf16x8_unsafe(u[j]);
                    float4* dst = reinterpret_cast<float4*>(xres + r * xres_pitch) + 2 * q;
                    dst[0] = make_float4(bf16_lo(u[j].x), bf16_hi(u[j].x), bf16_lo(u[j].y), bf16_hi(u[j].y));
                    dst[1] = make_float4(bf16_lo(u[j].z), bf16_hi(u[j].z), bf16_lo(u[j].w), bf16_hi(u[j].w));
                }
            }
        if (__syncthreads_or(unsafe) && threadIdx.x == 0) s_x_unsafe = 1;
        __syncthreads();
    }
    const int el = threadIdx.x % gt, g = threadIdx.x / gt;
    const bool active = warp < kFzConsumers && g < tg;
    float acc[TPT][EPT];
#pragma unroll
    for (int t = 0; t < TPT; ++t)
#pragma unroll
        for (int j = 0; j < EPT; ++j) acc[t][j] = 0.f;
    if (warp >= kFzConsumers) {
        // producer warps (thread pl of 32 * PW)
        const int pl = threadIdx.x - kFzCThreads, pw = warp - kFzConsumers;
        uint4 xv[kXRegs];
        auto load_x = [&](int c) {  // stage c's token chunk into registers
#pragma unroll
            for (int j = 0; j < kXRegs; ++j) {
                const int i = pl + 32 * PW * j, r = i / (kFzKc / 8), q = i % (kFzKc / 8);
                xv[j] = make_uint4(0u, 0u, 0u, 0u);
                if (i < tc * (kFzKc / 8) && r < nt)
                    xv[j] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + r) * H + c * kFzKc) + q);
            }
        };
        int issued = 0;
        bool ok = true;
        if (!kXRes) load_x(0);
        for (int c = kXRes ? min(NS, nstages) : 0; c < nstages; ++c) {
            const int s = c % NS;
            if (c >= NS && !fz_wait(&empty[s], static_cast<uint32_t>((c / NS - 1) & 1), &s_abort)) {
                ok = false;
                break;
            }
            uint8_t* slot = fz_smem_buf + s * slot_bytes;
            const int bytes = min(SUB, nchunks - c * SUB) * wchunk;
            if (pl == 0) {
                if (kXRes) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(bytes));
                else mbar_expect_tx(&full[s], static_cast<uint32_t>(bytes));
                bulk_load(slot, static_cast<const uint8_t*>(wz) + static_cast<int64_t>(c) * wbytes,
                          static_cast<uint32_t>(bytes), &full[s]);
            }
            issued = c + 1;
            if constexpr (!kXRes) {
                int unsafe = 0;
#pragma unroll
                for (int j = 0; j < kXRegs; ++j) {
                    const int i = pl + 32 * PW * j;
                    if (i < tc * (kFzKc / 8)) {
                        const int r = i / (kFzKc / 8), q = i % (kFzKc / 8);
                        const uint4 u = xv[j];
                        unsafe |= bf16x8_unsafe(u);
                        float4* dst = reinterpret_cast<float4*>(slot + wchunk + r * kFzXPitch) + 2 * q;
                        dst[0] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
                        dst[1] = make_float4(bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w));
                    }
                }
                unsafe = __any_sync(0xffffffffu, unsafe);
                if (lane == 0) s_unsafe[s][pw] = unsafe;
                mbar_arrive(&full[s]);  // releases this thread's token stores (and its warp's flag)
                if (c + 1 < nstages) load_x(c + 1);
            }
        }
        if (!ok && pl == 0 && atomicExch(const_cast<int*>(&s_abort), 1) == 0) atomicCAS(err, 0, NF_DEVERR_WAIT_EMPTY);
        // every router copy issued has to land before the CTA leaves (each
        // issued stage already has all its arrivals: they follow the issue)
        for (int c = max(0, issued - NS); c < issued; ++c)
            fz_wait(&full[c % NS], static_cast<uint32_t>((c / NS) & 1), nullptr);
    } else {
        for (int c = 0; c < nstages; ++c) {
            const int s = c % NS;
            if (!fz_wait(&full[s], static_cast<uint32_t>((c / NS) & 1), &s_abort)) {
                if (lane == 0 && atomicExch(const_cast<int*>(&s_abort), 1) == 0) atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
                break;
            }
            const uint8_t* slot = fz_smem_buf + s * slot_bytes;
            int unsafe_stage = kXRes ? s_x_unsafe : 0;
            if constexpr (!kXRes) {
#pragma unroll
                for (int i = 0; i < PW; ++i) unsafe_stage |= s_unsafe[s][i];
            }
            const bool use_fma = w_safe && !unsafe_stage;
            if (active) {
                if constexpr (kXRes) {
#pragma unroll
                    for (int sub = 0; sub < SUB; ++sub) {
                        const int chunk = c * SUB + sub;
                        if (chunk < nchunks) {
                            const float4* xr = reinterpret_cast<const float4*>(xres + g * xres_pitch) + chunk * (kFzKc / 4);
                            const uint4* wr = reinterpret_cast<const uint4*>(slot + sub * wchunk + el * fz_wpitch(kW16));
                            acc[0][0] = use_fma ? chain_fz16<true>(wr, xr, acc[0][0]) : chain_fz16<false>(wr, xr, acc[0][0]);
                        }
                    }
                } else {
                    const float4* xr = reinterpret_cast<const float4*>(slot + wchunk + g * TPT * kFzXPitch);
                    const float4* wr[EPT];
#pragma unroll
                    for (int j = 0; j < EPT; ++j)
                        wr[j] = reinterpret_cast<const float4*>(slot + min(el + j * gt, E - 1) * fz_wpitch(false));
                    if (use_fma) chain_fz32<true, EPT, TPT>(wr, xr, acc);
                    else chain_fz32<false, EPT, TPT>(wr, xr, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();
    if (s_abort) return;
    // router_select's per-expert part (src/text_forward.cpp:1453-1456):
    // score = sigmoid(logit), choice = score + correction bias; rows padded
    // to E + 1 so the per-token scans below hit distinct banks
    const int rs = E + 1;
    float* s_sc = reinterpret_cast<float*>(fz_smem_buf);  // [tc][E + 1]
    float* s_ch = s_sc + tc * rs;
    uint8_t* s_used = reinterpret_cast<uint8_t*>(s_ch + tc * rs);  // [tc][E]
    if (active) {
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int e = el + j * gt;
            if (e < E) {
                const float b = bias[e];
#pragma unroll
                for (int t = 0; t < TPT; ++t) {
                    const int tok = g * TPT + t;
                    if (tok < nt) {
                        const float sc = sigmoid_ref(acc[t][j]);
                        logits[static_cast<int64_t>(t0 + tok) * E + e] = acc[t][j];
                        s_sc[tok * rs + e] = sc;
                        s_ch[tok * rs + e] = __fadd_rn(sc, b);
                    }
                }
            }
        }
    }
    __syncthreads();
    if constexpr (TPT == 1) {
        // a few tokens: a warp per token, lanes split the experts
        __shared__ uint32_t s_excl[kThreads / 32][32];
        for (int t = warp; t < nt; t += kThreads / 32)
            warp_select_reg<(kFzMaxE + 31) / 32>(s_sc + t * rs, s_ch + t * rs, E, K, scaling, normalize, n_group,
                                                 topk_group, s_excl[warp], idx_out + static_cast<int64_t>(t0 + t) * K,
                                                 w_out + static_cast<int64_t>(t0 + t) * K);
    } else {
        // many tokens: a thread per token
        for (int t = threadIdx.x; t < nt; t += kThreads)
            thread_select(s_sc + t * rs, s_ch + t * rs, E, K, scaling, normalize, n_group, topk_group, s_used + t * E,
                          idx_out + static_cast<int64_t>(t0 + t) * K, w_out + static_cast<int64_t>(t0 + t) * K);
    }
}

// ---------------------------------------------------------------------------
// Permutation.  Output order is (expert, token): each expert owns a
// contiguous segment of permuted rows that starts on a multiple of 128 (the
// GEMM tile height and the scale-factor atom height); inside a segment rows
// follow token order.  The order is fully deterministic.
// Small batches (T * K <= kSmallPairs) run with the dispatch in one kernel
// whose every CTA rebuilds the permutation; large batches use per-chunk
// histograms, a scan and a per-chunk scatter.  Picks with expert -1 (empty
// slots of expert-parallel receive buffers) get no row (pair_row -1).
// ---------------------------------------------------------------------------
constexpr int kChunkTok = 128;
constexpr int kSmallPairs = 2048;
constexpr int kScanCtas = 16;  // CTAs of the large-batch scan (each writes a share of its outputs)

// Segment offsets of the permuted rows (each expert's segment padded to a
// multiple of 128) and m-tile offsets from per-expert counts in shared memory
// (s_cnt [E]); s_off and s_mt get [E + 1] entries.  Warp 0 scans; ends with
// the CTA synchronised.
__device__ void segment_scan(const int32_t* s_cnt, int32_t* s_off, int32_t* s_mt, int E) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int32_t base_mt = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int32_t m = e < E ? (s_cnt[e] + 127) / 128 : 0;
            int32_t inc = m;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t v = __shfl_up_sync(0xffffffffu, inc, d);
                if (lane >= d) inc += v;
            }
            if (e < E) {
                s_mt[e] = base_mt + inc - m;
                s_off[e] = (base_mt + inc - m) * 128;
            }
            base_mt += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) {
            s_mt[E] = base_mt;
            s_off[E] = base_mt * 128;
        }
    }
    __syncthreads();
}

// The permutation's global outputs that follow from the scan: meta, segment
// offsets and counts, padding rows (-1 in row_token), the two GEMM tile lists
// and the zeroed per-m-tile counters.  Work item i of each list is done by
// thread (i mod stride) of part i / blockDim.x mod parts: one CTA (part 0 of
// 1) or every CTA of a grid (blockIdx.x of gridDim.x) sharing the lists.
__device__ void segment_outputs(const int32_t* s_cnt, const int32_t* s_off, const int32_t* s_mt, int E, int nb_gu,
                                int nb_down, int part, int parts, int32_t* __restrict__ counts,
                                int32_t* __restrict__ seg_off, int32_t* __restrict__ row_token,
                                NfTile* __restrict__ tiles_gu, NfTile* __restrict__ tiles_down,
                                int32_t* __restrict__ meta, int32_t* __restrict__ mt_done) {
    const int32_t mt_total = s_mt[E];
    const int first = part * blockDim.x + threadIdx.x, stride = parts * blockDim.x;
    if (part == 0 && threadIdx.x == 0) {
        meta[0] = s_off[E];
        meta[1] = mt_total * nb_gu;
        meta[2] = mt_total * nb_down;
        meta[3] = mt_total;
        meta[4] = 0;  // tile counters of the two grouped GEMMs
        meta[5] = 0;
    }
    for (int e = first; e <= E; e += stride) {
        seg_off[e] = s_off[e];
        if (e < E) counts[e] = s_cnt[e];
    }
    // padding rows (at most 127 per expert)
    for (int i = first; i < E * 128; i += stride) {
        const int e = i >> 7, j = i & 127;
        const int32_t r = s_off[e] + s_cnt[e] + j;
        if (r < s_off[e + 1]) row_token[r] = -1;
    }
    for (int32_t i = first; i < mt_total; i += stride) mt_done[i] = 0;
    // tile lists, ordered (expert, n_block, m_tile): CTAs that run at the same
    // time share the weight block through L2
    for (int pass = 0; pass < 2; ++pass) {
        const int nb = pass == 0 ? nb_gu : nb_down;
        NfTile* tiles = pass == 0 ? tiles_gu : tiles_down;
        for (int32_t i = first; i < mt_total * nb; i += stride) {
            const int32_t mi = i / nb;  // any tile of m-tile group mi's expert
            int lo = 0, hi = E - 1;     // expert e with s_mt[e] <= mi < s_mt[e + 1]
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (s_mt[mid] <= mi) lo = mid;
                else hi = mid - 1;
            }
            const int e = lo;
            const int32_t mtiles = s_mt[e + 1] - s_mt[e];
            const int32_t local = i - s_mt[e] * nb;
            const int n = local / mtiles, m = local % mtiles;
            NfTile t;
            t.expert = e;
            t.row0 = s_off[e] + m * 128;
            t.n_block = n;
            t.m_valid = min(128, s_cnt[e] - m * 128);
            tiles[i] = t;
        }
    }
}

__global__ void permute_hist_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                    int32_t* __restrict__ chunk_counts) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    extern __shared__ int32_t cnt[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int t0 = blockIdx.x * kChunkTok;
    const int n = min(kChunkTok, T - t0) * K;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = idx[static_cast<int64_t>(t0) * K + i];
        if (e >= 0) atomicAdd(&cnt[e], 1);  // e < 0: an empty slot (expert-parallel receive buffers)
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[static_cast<int64_t>(blockIdx.x) * E + e] = cnt[e];
}

__global__ void __launch_bounds__(1024) permute_scan_kernel(const int32_t* __restrict__ chunk_counts, int nchunks,
                                                            int E, int nb_gu, int nb_down,
                                                            int32_t* __restrict__ chunk_base,
                                                            int32_t* __restrict__ counts,
                                                            int32_t* __restrict__ seg_off,
                                                            int32_t* __restrict__ row_token,
                                                            NfTile* __restrict__ tiles_gu,
                                                            NfTile* __restrict__ tiles_down,
                                                            int32_t* __restrict__ meta,
                                                            int32_t* __restrict__ mt_done) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    extern __shared__ int32_t sh[];
    int32_t* s_cnt = sh;
    int32_t* s_off = s_cnt + E;
    int32_t* s_mt = s_off + E + 1;
    // Every CTA scans all the counts (a few thousand integers) and writes its
    // share of the outputs: the chunk bases of chunks c = blockIdx.x mod
    // gridDim.x, and a part of the segment outputs and tile lists.
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        // the loads are independent: unrolled, eight are in flight at a time
        int32_t run = 0;
#pragma unroll 8
        for (int c = 0; c < nchunks; ++c) {
            const int32_t n = chunk_counts[static_cast<int64_t>(c) * E + e];
            if (c % static_cast<int>(gridDim.x) == static_cast<int>(blockIdx.x))
                chunk_base[static_cast<int64_t>(c) * E + e] = run;
            run += n;
        }
        s_cnt[e] = run;
    }
    __syncthreads();
    segment_scan(s_cnt, s_off, s_mt, E);
    segment_outputs(s_cnt, s_off, s_mt, E, nb_gu, nb_down, blockIdx.x, gridDim.x, counts, seg_off, row_token, tiles_gu,
                    tiles_down, meta, mt_done);
}

// Rows of a chunk of kChunkTok tokens.  A token's picks are distinct experts,
// so the rank of pick (t, e) inside expert e's share of the chunk is the
// number of earlier tokens of the chunk that picked e: each expert keeps a
// kChunkTok-bit mask of the tokens that picked it, and the rank is a
// popcount of the bits below t.
constexpr int kChunkWords = kChunkTok / 32;

__global__ void __launch_bounds__(256) permute_rows_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                                           const int32_t* __restrict__ chunk_base,
                                                           const int32_t* __restrict__ seg_off,
                                                           int32_t* __restrict__ pair_row,
                                                           int32_t* __restrict__ row_token) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    extern __shared__ uint32_t s_mask[];  // [E][kChunkWords]
    const int t0 = blockIdx.x * kChunkTok;
    const int n = min(kChunkTok, T - t0) * K;
    for (int i = threadIdx.x; i < E * kChunkWords; i += blockDim.x) s_mask[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = idx[static_cast<int64_t>(t0) * K + i], t = i / K;
        if (e >= 0) atomicOr(&s_mask[e * kChunkWords + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = idx[static_cast<int64_t>(t0) * K + i], t = i / K;
        if (e < 0) {
            pair_row[static_cast<int64_t>(t0) * K + i] = -1;
            continue;
        }
        const uint32_t* m = s_mask + e * kChunkWords;
        int rank = __popc(m[t >> 5] & ((1u << (t & 31)) - 1u));
        for (int wd = 0; wd < (t >> 5); ++wd) rank += __popc(m[wd]);
        const int row = seg_off[e] + chunk_base[static_cast<int64_t>(blockIdx.x) * E + e] + rank;
        pair_row[static_cast<int64_t>(t0) * K + i] = row;
        row_token[row] = t0 + t;
    }
}

// ---------------------------------------------------------------------------
// Dispatch: x rows into the permuted activation buffer.  NVFP4 experts: the
// row of pick (t, p) is x[t] quantised with the gate input_scale of expert
// idx[t, p] (quant_dequant_nvfp4_activation, src/text_forward.cpp:527-550),
// stored as E2M1 codes plus E4M3 scales in the tcgen05 atom layout.  BF16
// experts: plain row copies.  Large batches: one thread per (token,
// 16-element group), which quantises the group once and writes it to each
// pick's row (again only for a pick whose expert has another input scale), so
// the work is per token, not per pick.  Small batches (permute_dispatch_kernel):
// one thread per (pick, group), so a decode step still covers the GPU.
// ---------------------------------------------------------------------------
// Elements [16 g, 16 g + 16) of token t's row into the permuted row of each of
// its K picks (pair_row[t K + p], -1 = an empty slot), quantised once with
// the gate input scale of the first pick and again only for a pick whose
// expert has another scale (each row's codes are those of its own expert).
__device__ __forceinline__ void dispatch_token_group(const uint16_t* __restrict__ x, int t, int g, int K,
                                                     const int32_t* __restrict__ pick_e,
                                                     const int32_t* __restrict__ pick_row,
                                                     const float* __restrict__ gscale,
                                                     const float* __restrict__ os_tab_g, int H, int bf16_mode,
                                                     uint8_t* __restrict__ a_codes, uint8_t* __restrict__ a_sf,
                                                     uint16_t* __restrict__ a_bf16) {
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * H + g * 16);
    const uint4 r0 = __ldg(src), r1 = __ldg(src + 1);
    float v[16];
    if (!bf16_mode) {
        const uint32_t u[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[2 * j] = bf16_lo(u[j]);
            v[2 * j + 1] = bf16_hi(u[j]);
        }
    }
    uint32_t codes[2] = {0u, 0u}, sf = 0u;
    float have = 0.f;  // the scale the held codes were made with (0: none yet)
    for (int p = 0; p < K; ++p) {
        const int row = pick_row[p];
        if (row < 0) continue;
        if (bf16_mode) {
            uint4* dst = reinterpret_cast<uint4*>(a_bf16 + static_cast<int64_t>(row) * H + g * 16);
            dst[0] = r0;
            dst[1] = r1;
            continue;
        }
        const int e = pick_e[p];
        const float gs = gscale[e];
        if (!(have == gs)) {
            float w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = v[j];
            // (the expert's table of output scales per scale code, when given:
            // the same values without the three divisions)
            sf = os_tab_g ? quantize_group16_tab(w, gs, os_tab_g + 256 * e, codes) : quantize_group16_fast<true>(w, gs, codes);
            have = gs;
        }
        *reinterpret_cast<uint2*>(a_codes + static_cast<int64_t>(row) * (H / 2) + g * 8) = make_uint2(codes[0], codes[1]);
        a_sf[sf_atom_offset(row, g, H / 16)] = static_cast<uint8_t>(sf);
    }
}

__global__ void dispatch_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ idx,
                                const int32_t* __restrict__ pair_row, const float* __restrict__ gscale,
                                const float* __restrict__ os_tab_g, int T, int K,
                                int H, int bf16_mode, uint8_t* __restrict__ a_codes, uint8_t* __restrict__ a_sf,
                                uint16_t* __restrict__ a_bf16) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    const int gq = H / 16;
    const int64_t item = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (item >= static_cast<int64_t>(T) * gq) return;
    const int64_t t = item / gq;
    const int g = static_cast<int>(item - t * gq);
    dispatch_token_group(x, static_cast<int>(t), g, K, idx + t * K, pair_row + t * K, gscale, os_tab_g, H,
                         bf16_mode, a_codes, a_sf, a_bf16);
}

// The dense MLP's dispatch: its rows are the tokens in order (one segment at
// row 0, no permutation), so it quantises token t into row t with the one
// gate input scale, writes the identity pick -> row map for the combine, and
// block 0 zeroes the GEMMs' tile counters (meta[4..5]), the fused split-K
// reduction's slice counters; with rep64 (T <= 64) token t is also written to
// row t + 64
// and the per-128-row hand-off counters the permutation would otherwise reset.
__global__ void dense_dispatch_kernel(const uint16_t* __restrict__ x, int T, int H, const float* __restrict__ gscale,
                                      const float* __restrict__ os_tab_g,
                                      uint8_t* __restrict__ a_codes, uint8_t* __restrict__ a_sf,
                                      int32_t* __restrict__ pair_row, int32_t* __restrict__ meta,
                                      int32_t* __restrict__ mt_done, int m_tiles, int* __restrict__ splitk_cnt,
                                      int n_splitk_cnt, int rep64) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    if (blockIdx.x == 0) {
        if (threadIdx.x < 2) meta[4 + threadIdx.x] = 0;
        for (int i = threadIdx.x; i < m_tiles; i += blockDim.x) mt_done[i] = 0;
        for (int i = threadIdx.x; i < n_splitk_cnt; i += blockDim.x) splitk_cnt[i] = 0;
    }
    const int gq = H / 16;
    const int64_t item = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (item >= static_cast<int64_t>(T) * gq) return;
    const int t = static_cast<int>(item / gq), g = static_cast<int>(item - static_cast<int64_t>(t) * gq);
    const int32_t e0 = 0, row = t, row2 = t + 64;
    if (g == 0) pair_row[t] = t;  // the combine's pick -> row map
    dispatch_token_group(x, t, g, 1, &e0, &row, gscale, os_tab_g, H, 0, a_codes, a_sf, nullptr);
    if (rep64) dispatch_token_group(x, t, g, 1, &e0, &row2, gscale, os_tab_g, H, 0, a_codes, a_sf, nullptr);
}

cudaError_t launch_dense_dispatch(const uint16_t* x, int T, int H, const float* gscale, const float* os_tab_g,
                                  PermuteBuffers& b, int* splitk_cnt, int n_splitk_cnt, bool rep64, cudaStream_t st) {
    if (rep64 && T > 64) return cudaErrorInvalidValue;
    const int64_t items = static_cast<int64_t>(T) * (H / 16);
    const int m_tiles = (T + 127) / 128;
    return launch_dependent(dense_dispatch_kernel, dim3(static_cast<unsigned>(std::max<int64_t>(1, (items + 127) / 128))),
                            dim3(128), 0, st, x, T, H, gscale, os_tab_g, b.a_codes, b.a_sf, b.pair_row, b.meta, b.mt_done,
                            m_tiles, splitk_cnt, splitk_cnt ? n_splitk_cnt : 0, rep64 ? 1 : 0);
}

// Permutation and dispatch of a small batch (T * K <= kSmallPairs) in one
// launch: every CTA rebuilds the permutation in shared memory from idx (a
// few hundred picks: cheaper than a kernel boundary), writes its share of the
// permutation's global outputs (segment_outputs over the grid, pair rows by
// pick) and quantises its share of the dispatch items.
__global__ void __launch_bounds__(256) permute_dispatch_kernel(
    const int32_t* __restrict__ idx, const uint16_t* __restrict__ x, int T, int K, int E, int H, int nb_gu, int nb_down,
    const float* __restrict__ gscale, const float* __restrict__ os_tab_g, int bf16_mode, int32_t* __restrict__ counts,
    int32_t* __restrict__ seg_off,
    int32_t* __restrict__ pair_row, int32_t* __restrict__ row_token, NfTile* __restrict__ tiles_gu,
    NfTile* __restrict__ tiles_down, int32_t* __restrict__ meta, int32_t* __restrict__ mt_done,
    uint8_t* __restrict__ a_codes, uint8_t* __restrict__ a_sf, uint16_t* __restrict__ a_bf16) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    extern __shared__ int32_t sh[];
    const int n = T * K, words = (T + 31) / 32;
    int32_t* s_cnt = sh;
    int32_t* s_off = s_cnt + E;
    int32_t* s_mt = s_off + E + 1;
    int32_t* s_idx = s_mt + E + 1;   // [n]
    int32_t* s_row = s_idx + n;      // [n] permuted row of each pick
    uint32_t* s_mask = reinterpret_cast<uint32_t*>(s_row + n);  // [E][words]: tokens that picked e
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    for (int i = threadIdx.x; i < E * words; i += blockDim.x) s_mask[i] = 0u;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s_idx[i] = idx[i];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = s_idx[i], t = i / K;
        if (e < 0) continue;  // an empty slot (expert-parallel receive buffers)
        atomicAdd(&s_cnt[e], 1);
        atomicOr(&s_mask[e * words + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    segment_scan(s_cnt, s_off, s_mt, E);
    // the rank of pick (t, e) in expert e's segment: e's tokens below t
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = s_idx[i], t = i / K;
        if (e < 0) {
            s_row[i] = -1;
            continue;
        }
        const uint32_t* m = s_mask + e * words;
        int rank = __popc(m[t >> 5] & ((1u << (t & 31)) - 1u));
        for (int wd = 0; wd < (t >> 5); ++wd) rank += __popc(m[wd]);
        s_row[i] = s_off[e] + rank;
    }
    __syncthreads();
    segment_outputs(s_cnt, s_off, s_mt, E, nb_gu, nb_down, blockIdx.x, gridDim.x, counts, seg_off, row_token, tiles_gu,
                    tiles_down, meta, mt_done);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        pair_row[i] = s_row[i];
        if (s_row[i] >= 0) row_token[s_row[i]] = i / K;
    }
    // small batches: one thread per (pick, group), so a decode step still
    // covers the GPU (a group shared by a token's picks is quantised per pick)
    const int gq = H / 16;
    for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < n * gq; item += gridDim.x * blockDim.x) {
        const int pair = item / gq, g = item - pair * gq;
        dispatch_token_group(x, pair / K, g, 1, s_idx + pair, s_row + pair, gscale, os_tab_g, H, bf16_mode,
                             a_codes, a_sf, a_bf16);
    }
}

// ---------------------------------------------------------------------------
// Self-check of the hardware format conversions against the reference's
// rules over every 32-bit pattern: E2M1 (cast_to_e2m1 after the +-6 clamp),
// E4M3 on [2^-6, inf) (f32_to_e4m3 after the 448 clamp) and BF16 rounding
// (f32_to_bf16 on every non-NaN input).
// ---------------------------------------------------------------------------
__global__ void format_selfcheck_kernel(unsigned long long* __restrict__ mismatches) {
    unsigned long long bad_e2m1 = 0, bad_e4m3 = 0, bad_bf16 = 0;
    for (uint64_t b = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; b < (1ull << 32);
         b += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float x = __uint_as_float(static_cast<uint32_t>(b));
        if (isnan(x)) continue;
        if (__float_as_uint(bf16_round_hw(x)) != __float_as_uint(bf16_round(x))) ++bad_bf16;
        const uint32_t pair = bf16x2_hw(x, -x);
        if ((pair << 16) != __float_as_uint(bf16_round(x)) || (pair & 0xffff0000u) != __float_as_uint(bf16_round(-x)))
            ++bad_bf16;
        const float c = x > 6.f ? 6.f : (x < -6.f ? -6.f : x);
        const uint32_t want = e2m1_code(c);
        if ((e2m1x2_hw(c, 0.f) & 0xfu) != want || (e2m1x2_hw(x, 0.f) & 0xfu) != want) ++bad_e2m1;
        if ((e2m1x2_hw(0.f, c) >> 4) != want) ++bad_e2m1;
        if (x >= 0.015625f) {
            const float m = x > 448.f ? 448.f : x;
            const uint32_t w8 = f32_to_e4m3(m);
            if (e4m3_hw(m) != w8 || e4m3_hw(x) != w8) ++bad_e4m3;
        }
    }
    atomicAdd(&mismatches[0], bad_e2m1);
    atomicAdd(&mismatches[1], bad_e4m3);
    atomicAdd(&mismatches[2], bad_bf16);
}

// ---------------------------------------------------------------------------
// Combine: y[t] = sum_p w[t,p] * down[row(t,p)] in pick order starting from
// 0 (src/text_forward.cpp:951,958-959), + shared[t] (:962), + residual[t]
// (mhc_combine with hc = 1, :906/1646-1657).  Separate multiply and add, in
// the reference's order; `down` holds BF16-exact values (NVFP4 path) or F32
// (BF16 experts).  One CTA per token, 8 dims per thread.
// ---------------------------------------------------------------------------
template <typename DownT>
__global__ void __launch_bounds__(256) combine_kernel(const DownT* __restrict__ down, const int32_t* __restrict__ pair_row,
                                                      const float* __restrict__ topk_w, const float* __restrict__ shared,
                                                      const float* __restrict__ residual, int T, int K, int H,
                                                      float* __restrict__ y) {
    pdl_wait();  // launched dependent on the previous kernel
    pdl_trigger();
    const int t = blockIdx.x;
    for (int d0 = threadIdx.x * 8; d0 < H; d0 += blockDim.x * 8) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int p = 0; p < K; ++p) {
            const int row = pair_row[static_cast<int64_t>(t) * K + p];
            const float w = topk_w[static_cast<int64_t>(t) * K + p];
            float dv[8];
            if constexpr (sizeof(DownT) == 2) {
                const uint4 q = *reinterpret_cast<const uint4*>(down + static_cast<int64_t>(row) * H + d0);
                const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    dv[2 * i] = __uint_as_float((u[i] & 0xffffu) << 16);
                    dv[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
                }
            } else {
                const float4* s = reinterpret_cast<const float4*>(down + static_cast<int64_t>(row) * H + d0);
                const float4 a = s[0], b = s[1];
                dv[0] = a.x; dv[1] = a.y; dv[2] = a.z; dv[3] = a.w;
                dv[4] = b.x; dv[5] = b.y; dv[6] = b.z; dv[7] = b.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(w, dv[i]));
        }
        if (shared) {
            const float4* s = reinterpret_cast<const float4*>(shared + static_cast<int64_t>(t) * H + d0);
            const float4 a = s[0], b = s[1];
            const float sv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], sv[i]);
        }
        if (residual) {
            const float4* s = reinterpret_cast<const float4*>(residual + static_cast<int64_t>(t) * H + d0);
            const float4 a = s[0], b = s[1];
            const float rv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], rv[i]);
        }
        float4* o = reinterpret_cast<float4*>(y + static_cast<int64_t>(t) * H + d0);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// ---------------------------------------------------------------------------
// Format kernels
// ---------------------------------------------------------------------------
// Nvfp4MatrixView::at (src/nvfp4_decode.cpp:88-97): double product, one
// rounding to float.
__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales, float gscale,
                               int64_t rows, int64_t cols, float* __restrict__ out) {
    const int64_t n = rows * cols / 2;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / (cols / 2), cb = i % (cols / 2);
        const uint32_t byte = packed[i];
        const double s = static_cast<double>(e4m3_to_f32(scales[r * (cols / 16) + (cb * 2) / 16]));
        const uint32_t lo = byte & 0xfu, hi = byte >> 4;
        const double vlo = (lo & 8u) ? -static_cast<double>(e2m1_mag(lo)) : static_cast<double>(e2m1_mag(lo));
        const double vhi = (hi & 8u) ? -static_cast<double>(e2m1_mag(hi)) : static_cast<double>(e2m1_mag(hi));
        out[r * cols + cb * 2] = static_cast<float>(vlo * s * static_cast<double>(gscale));
        out[r * cols + cb * 2 + 1] = static_cast<float>(vhi * s * static_cast<double>(gscale));
    }
}

// quant_dequant_nvfp4_activation over rows, one thread per 16-group.
__global__ void quantize_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, float gscale,
                                uint8_t* __restrict__ codes, uint8_t* __restrict__ scales, float* __restrict__ fake) {
    const int64_t groups = rows * (cols / 16);
    for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = x[g * 16 + i];
        uint32_t c[2];
        const uint32_t sc = quantize_group16_fast<false>(v, gscale, c);
        reinterpret_cast<uint2*>(codes)[g] = make_uint2(c[0], c[1]);
        scales[g] = static_cast<uint8_t>(sc);
        if (fake) {
            const float s = e4m3_to_f32(sc);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t code = (c[i >> 3] >> (4 * (i & 7))) & 0xfu;
                const float m = e2m1_mag(code);
                fake[g * 16 + i] = __fmul_rn((code & 8u) ? -m : m, s);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
// Sets a kernel's dynamic shared memory limit once per device.
template <typename Kernel>
static cudaError_t smem_attr_once(Kernel kernel, int bytes, bool (&done)[kMaxDevices]) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (done[dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[dev] = true;
    return e;
}

template <int EPT, int TPT, int SUB, int NS, int PW, bool kW16, bool kXRes>
static cudaError_t launch_fused(const uint16_t* x, const void* wz, const float* bias, int T, int H, int E, int K,
                                float scaling, int normalize, int n_group, int topk_group, int w_safe, float* logits,
                                int32_t* idx, float* wts, int* err, cudaStream_t st) {
    static bool attr[kMaxDevices] = {};
    const cudaError_t e = smem_attr_once(router_fused_kernel<EPT, TPT, SUB, NS, PW, kW16, kXRes>,
                                         static_cast<int>(fz_smem(kFzMaxE, EPT, TPT, SUB, NS, kW16, kXRes, kFzMaxResH)),
                                         attr);
    if (e != cudaSuccess) return e;
    const int tc = fz_tokens(E, EPT, TPT);
    router_fused_kernel<EPT, TPT, SUB, NS, PW, kW16, kXRes>
        <<<(T + tc - 1) / tc, kFzCThreads + 32 * PW, fz_smem(E, EPT, TPT, SUB, NS, kW16, kXRes, H), st>>>(
            x, wz, bias, T, H, E, K, scaling, normalize, n_group, topk_group, w_safe, logits, idx, wts, err);
    return cudaGetLastError();
}

cudaError_t launch_router(const uint16_t* x, const uint16_t* w, const float* w_chunked32, const uint16_t* w_chunked16,
                          const float* bias, int T, int H, int E, int K, float scaling, int normalize, int n_group,
                          int topk_group, int w_safe, float* logits, float* scores, float* choices, int32_t* idx,
                          float* wts, int* err, cudaStream_t st) {
    if (w_chunked32 && w_chunked16 && E <= kFzMaxE && H % kFzKc == 0) {
        // one chain per thread over resident token rows while the batch gives
        // each CTA a couple of tokens; 8 tokens x 2 experts per thread once it
        // fills the GPU
        if (T < 2048 && H <= kFzMaxResH)
            return launch_fused<1, 1, 2, 3, 1, true, true>(x, w_chunked16, bias, T, H, E, K, scaling, normalize, n_group,
                                                         topk_group, w_safe, logits, idx, wts, err, st);
        if (E > 32)
            return launch_fused<2, 8, 1, 2, 2, false, false>(x, w_chunked32, bias, T, H, E, K, scaling, normalize, n_group,
                                                          topk_group, w_safe, logits, idx, wts, err, st);
        return launch_fused<1, 8, 1, 2, 2, false, false>(x, w_chunked32, bias, T, H, E, K, scaling, normalize, n_group,
                                                      topk_group, w_safe, logits, idx, wts, err, st);
    }
    const int chunk = H < kRtMaxChunk ? H : kRtMaxChunk;
    const size_t smem = static_cast<size_t>(kRtExp + kRtTok) * (chunk * 2 + 16);
    static bool attr[kMaxDevices] = {};
    cudaError_t e = smem_attr_once(router_logits_kernel, static_cast<int>((kRtExp + kRtTok) * (kRtMaxChunk * 2 + 16)), attr);
    if (e != cudaSuccess) return e;
    const dim3 grid((T + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp);
    router_logits_kernel<<<grid, kRtThreads, smem, st>>>(x, w, bias, T, H, E, w_safe, logits, scores, choices, err);
    router_select_kernel<<<(T + kSelectWarps - 1) / kSelectWarps, kSelectWarps * 32, 0, st>>>(
        scores, choices, T, E, K, scaling, normalize, n_group, topk_group, idx, wts);
    return cudaGetLastError();
}

cudaError_t launch_permute(const int32_t* idx, const uint16_t* x, int T, int K, int E, int H, int nb_gu, int nb_down,
                           const float* gscale, const float* os_tab_g, int bf16_mode, PermuteBuffers& b, cudaStream_t st,
                           bool* one_kernel) {
    const size_t small_smem = (3 * E + 2 + 2 * T * K + static_cast<size_t>(E) * ((T + 31) / 32)) * sizeof(int32_t);
    if (T * K <= kSmallPairs && small_smem <= 48 * 1024) {
        const int64_t items = static_cast<int64_t>(T) * K * (H / 16);
        const int blocks = static_cast<int>(std::min<int64_t>(256, (items + 255) / 256));
        *one_kernel = true;
        return launch_dependent(permute_dispatch_kernel, dim3(blocks), dim3(256), small_smem, st, idx, x, T, K, E, H,
                                nb_gu, nb_down, gscale, os_tab_g, bf16_mode, b.counts, b.seg_off, b.pair_row, b.row_token,
                                b.tiles_gu, b.tiles_down, b.meta, b.mt_done, b.a_codes, b.a_sf, b.a_bf16);
    } else {
        *one_kernel = false;
        const int nchunks = (T + kChunkTok - 1) / kChunkTok;
        cudaError_t e = launch_dependent(permute_hist_kernel, dim3(nchunks), dim3(256), E * sizeof(int32_t), st, idx, T,
                                         K, E, b.chunk_counts);
        if (e == cudaSuccess)
            e = launch_dependent(permute_scan_kernel, dim3(kScanCtas), dim3(1024), (3 * E + 2) * sizeof(int32_t), st,
                                 static_cast<const int32_t*>(b.chunk_counts), nchunks, E, nb_gu, nb_down, b.chunk_base,
                                 b.counts, b.seg_off, b.row_token, b.tiles_gu, b.tiles_down, b.meta, b.mt_done);
        if (e == cudaSuccess)
            e = launch_dependent(permute_rows_kernel, dim3(nchunks), dim3(256),
                                 static_cast<size_t>(E) * kChunkWords * sizeof(uint32_t), st, idx, T, K, E,
                                 static_cast<const int32_t*>(b.chunk_base), static_cast<const int32_t*>(b.seg_off),
                                 b.pair_row, b.row_token);
        if (e != cudaSuccess) return e;
    }
    const int64_t items = static_cast<int64_t>(T) * (H / 16);
    return launch_dependent(dispatch_kernel, dim3(static_cast<unsigned>((items + 127) / 128)), dim3(128), 0, st, x, idx,
                            static_cast<const int32_t*>(b.pair_row), gscale, os_tab_g, T, K, H, bf16_mode, b.a_codes, b.a_sf,
                            b.a_bf16);
}

cudaError_t launch_format_selfcheck(unsigned long long* mismatches_dev, cudaStream_t st) {
    format_selfcheck_kernel<<<148 * 8, 256, 0, st>>>(mismatches_dev);
    return cudaGetLastError();
}

cudaError_t launch_combine(const void* down, bool down_bf16, const int32_t* pair_row, const float* topk_w,
                           const float* shared, const float* residual, int T, int K, int H, float* y,
                           cudaStream_t st) {
    const int threads = min(256, H / 8);
    if (down_bf16)
        return launch_dependent(combine_kernel<uint16_t>, dim3(T), dim3(threads), 0, st,
                                static_cast<const uint16_t*>(down), pair_row, topk_w, shared, residual, T, K, H, y);
    return launch_dependent(combine_kernel<float>, dim3(T), dim3(threads), 0, st, static_cast<const float*>(down),
                            pair_row, topk_w, shared, residual, T, K, H, y);
}

// ---------------------------------------------------------------------------
// Split-K reduction of a dense down projection: linear_nvfp4's output
// (src/text_forward.cpp:852-855: accumulator x alpha, rounded to BF16) from
// the fp32 partial accumulators of S K slices, summed in slice order, then
// the hc = 1 residual (src/text_forward.cpp:906).  Four columns per thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) splitk_store_kernel(const float* __restrict__ part, int S, int64_t stride, int T,
                                                           int H, const float* __restrict__ alpha,
                                                           const float* __restrict__ residual, float* __restrict__ y) {
    pdl_wait();  // launched dependent on the GEMM that writes the slices
    pdl_trigger();
    const int64_t n4 = static_cast<int64_t>(T) * H / 4;
    const float a = alpha[0];
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // slices in order; four loads in flight before their adds
        float4 acc = reinterpret_cast<const float4*>(part)[i];
        auto add = [&](const float4 v) {
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        };
        int s = 1;
        for (; s + 3 < S; s += 4) {
            const float4 v0 = reinterpret_cast<const float4*>(part + s * stride)[i];
            const float4 v1 = reinterpret_cast<const float4*>(part + (s + 1) * stride)[i];
            const float4 v2 = reinterpret_cast<const float4*>(part + (s + 2) * stride)[i];
            const float4 v3 = reinterpret_cast<const float4*>(part + (s + 3) * stride)[i];
            add(v0);
            add(v1);
            add(v2);
            add(v3);
        }
        for (; s < S; ++s) add(reinterpret_cast<const float4*>(part + s * stride)[i]);
        float4 o = make_float4(bf16_round_hw(__fmul_rn(acc.x, a)), bf16_round_hw(__fmul_rn(acc.y, a)),
                               bf16_round_hw(__fmul_rn(acc.z, a)), bf16_round_hw(__fmul_rn(acc.w, a)));
        if (residual) {
            const float4 r = reinterpret_cast<const float4*>(residual)[i];
            o.x = __fadd_rn(o.x, r.x);
            o.y = __fadd_rn(o.y, r.y);
            o.z = __fadd_rn(o.z, r.z);
            o.w = __fadd_rn(o.w, r.w);
        }
        reinterpret_cast<float4*>(y)[i] = o;
    }
}

cudaError_t launch_splitk_store(const float* part, int S, int64_t stride, int T, int H, const float* alpha,
                                const float* residual, float* y, int grid_cap, cudaStream_t st) {
    const int64_t n4 = static_cast<int64_t>(T) * H / 4;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid_cap, (n4 + 255) / 256)));
    return launch_dependent(splitk_store_kernel, dim3(blocks), dim3(256), 0, st, part, S, stride, T, H, alpha, residual,
                            y);
}

// ---------------------------------------------------------------------------
// Expert parallelism.  Pick (t, p) goes to rank d = idx[t, p] / e_per_rank.
// ep_pack lays the picks out in (destination, token, pick) order -- the
// order the exchange sends them in, fully deterministic -- and writes, per
// pick, its send slot (the combine's pair_row at the source), per slot its
// token and destination-local expert, and per destination its count.  One
// CTA of 1024 threads walks the picks in chunks of 1024: per chunk, each
// warp ballots its lanes per destination and a scan over the warps gives
// every pick its rank.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) ep_pack_kernel(const int32_t* __restrict__ idx, int n, int K,
                                                       const int32_t* __restrict__ route, int experts,
                                                       int world, int32_t* __restrict__ slot,
                                                       int32_t* __restrict__ send_tok, int32_t* __restrict__ send_e,
                                                       int32_t* __restrict__ counts) {
    __shared__ int32_t s_base[kEpMaxRanks];
    __shared__ int32_t s_w[32][kEpMaxRanks];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < kEpMaxRanks) s_base[threadIdx.x] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&s_base[route[idx[i]]], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int d = 0; d < world; ++d) {
            const int c = s_base[d];
            counts[d] = c;
            s_base[d] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int c0 = 0; c0 < n; c0 += blockDim.x) {
        const int i = c0 + threadIdx.x;
        const int d = i < n ? route[idx[i]] : -1;
        int in_warp = 0;
        for (int dd = 0; dd < world; ++dd) {
            const uint32_t m = __ballot_sync(0xffffffffu, d == dd);
            if (lane == 0) s_w[warp][dd] = __popc(m);
            if (d == dd) in_warp = __popc(m & ((1u << lane) - 1u));
        }
        __syncthreads();
        if (d >= 0) {
            int r = s_base[d] + in_warp;
            for (int w = 0; w < warp; ++w) r += s_w[w][d];
            slot[i] = r;
            send_tok[r] = i / K;
            send_e[r] = route[experts + idx[i]];
        }
        __syncthreads();
        if (threadIdx.x < world) {
            int total = 0;
            for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += s_w[w][threadIdx.x];
            s_base[threadIdx.x] += total;
        }
        __syncthreads();
    }
}

// dst row i = src row map[i]; rows of row_bytes (a multiple of 16) bytes.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, const int32_t* __restrict__ map, int n,
                                   int row_bytes, uint8_t* __restrict__ dst) {
    const int per_row = row_bytes / 16;
    const int64_t total = static_cast<int64_t>(n) * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c = i - r * per_row;
        reinterpret_cast<uint4*>(dst + r * row_bytes)[c] =
            __ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(map[r]) * row_bytes) + c);
    }
}

cudaError_t launch_ep_pack(const int32_t* idx, int T, int K, const int32_t* route, int experts, int world, int32_t* slot,
                           int32_t* send_tok, int32_t* send_e, int32_t* counts, cudaStream_t st) {
    if (world < 1 || world > kEpMaxRanks) return cudaErrorInvalidValue;
    ep_pack_kernel<<<1, 1024, 0, st>>>(idx, T * K, K, route, experts, world, slot, send_tok, send_e, counts);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const void* src, const int32_t* map, int n, int row_bytes, void* dst, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int64_t total = static_cast<int64_t>(n) * (row_bytes / 16);
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    gather_rows_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(src), map, n, row_bytes,
                                               static_cast<uint8_t*>(dst));
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Expert parallelism over NVLink peer memory.  Every rank exports one
// "mailbox" allocation (EpLayout) that its peers map with CUDA IPC; rows go
// to their owners and outputs come back by plain stores into the peer's
// mailbox, each direction closed by a flag the writer sets to the forward's
// epoch (st.release.sys after a system-scope fence) and the reader waits for
// (ld.acquire.sys, bounded by NF_WAIT_BUDGET_NS).  The epoch is a device
// counter (every rank runs the same forwards, so the counters agree), which
// keeps the forward free of host synchronisation and capturable in a graph.
// One buffer per direction is enough: a rank sends epoch e + 1 only after it
// received every owner's epoch-e outputs, which each owner returns after its
// GEMMs consumed all of epoch e's rows.
// ---------------------------------------------------------------------------
// Bounded wait until *flag >= want (epochs only grow); false after the budget.
__device__ bool ep_wait_flag(const uint32_t* flag, uint32_t want) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (static_cast<int32_t>(ld_acquire_sys(flag) - want) >= 0) return true;
        if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) return false;
        __nanosleep(100);
    }
}

// Rows of this rank's picks (send order: destination-major) from x into
// their owners' mailboxes: grid (blocks, world), one destination per y.
// The last block of a destination publishes the count, this rank's send
// offset for it, and the flag.
__global__ void __launch_bounds__(256) ep_p2p_send_kernel(const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ send_tok,
                                                          const int32_t* __restrict__ send_e,
                                                          const int32_t* __restrict__ counts, int H, int me,
                                                          EpPeers peers, EpLayout lay,
                                                          const uint32_t* __restrict__ epoch, int32_t* __restrict__ done) {
    const int p = blockIdx.y;
    int soff = 0;
    for (int q = 0; q < p; ++q) soff += counts[q];
    const int cnt = counts[p];
    const uint32_t ep = *epoch + 1u;
    uint8_t* dst = peers.mbox[p];
    const int per_row = H / 8;  // 16-byte pieces of a BF16 row
    uint4* rows = reinterpret_cast<uint4*>(dst + lay.rows) + static_cast<int64_t>(me) * lay.cap * per_row;
    int32_t* dst_e = reinterpret_cast<int32_t*>(dst + lay.e) + static_cast<int64_t>(me) * lay.cap;
    for (int r = blockIdx.x; r < cnt; r += gridDim.x) {
        const int slot = soff + r;
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(send_tok[slot]) * H);
        for (int c = threadIdx.x; c < per_row; c += blockDim.x) rows[static_cast<int64_t>(r) * per_row + c] = __ldg(src + c);
        if (threadIdx.x == 0) dst_e[r] = send_e[slot];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(&done[p], 1) == static_cast<int>(gridDim.x) - 1) {
            reinterpret_cast<int32_t*>(dst + lay.cnt)[me] = cnt;
            reinterpret_cast<int32_t*>(dst + lay.off)[me] = soff;
            __threadfence_system();
            st_release_sys(reinterpret_cast<uint32_t*>(dst + lay.flags_recv) + me, ep);
            done[p] = 0;  // ready for the next forward (which follows this kernel in stream order)
        }
    }
}

// Waits for every source's rows of this epoch, records the counts it saw in
// seen[] (0 for a source that never arrived: the wait gave up and set *err)
// and marks the unused slots of the receive buffer as empty (expert -1).
__global__ void __launch_bounds__(256) ep_p2p_recv_wait_kernel(uint8_t* __restrict__ mbox, EpLayout lay, int world,
                                                               const uint32_t* __restrict__ epoch,
                                                               int32_t* __restrict__ seen, int* __restrict__ err) {
    __shared__ int s_cnt[kEpMaxRanks];
    const uint32_t ep = *epoch + 1u;
    if (threadIdx.x < world) {
        int c = 0;
        if (ep_wait_flag(reinterpret_cast<const uint32_t*>(mbox + lay.flags_recv) + threadIdx.x, ep)) {
            c = reinterpret_cast<volatile int32_t*>(mbox + lay.cnt)[threadIdx.x];
            c = max(0, min(c, lay.cap));
        } else {
            atomicCAS(err, 0, NF_DEVERR_EP_WAIT);
        }
        s_cnt[threadIdx.x] = c;
        if (blockIdx.x == 0) seen[threadIdx.x] = c;
    }
    __syncthreads();
    int32_t* e = reinterpret_cast<int32_t*>(mbox + lay.e);
    for (int src = 0; src < world; ++src)
        for (int j = s_cnt[src] + blockIdx.x * blockDim.x + threadIdx.x; j < lay.cap; j += gridDim.x * blockDim.x)
            e[static_cast<int64_t>(src) * lay.cap + j] = -1;
}

// Each received row's expert output (down, in the inner handle's permuted
// order, pair_row over the [world][cap] receive slots) back into its
// source's mailbox at the source's send position: grid (blocks, world), one
// source per y.  Every source gets its flag, also with no rows.
__global__ void __launch_bounds__(256) ep_p2p_return_kernel(const uint8_t* __restrict__ down,
                                                            const int32_t* __restrict__ pair_row, int out_bytes, int me,
                                                            EpPeers peers, EpLayout lay,
                                                            const uint8_t* __restrict__ mbox,
                                                            const int32_t* __restrict__ seen,
                                                            const uint32_t* __restrict__ epoch,
                                                            int32_t* __restrict__ done) {
    const int src = blockIdx.y;
    const int cnt = seen[src];
    const int off = reinterpret_cast<const int32_t*>(mbox + lay.off)[src];
    const uint32_t ep = *epoch + 1u;
    uint8_t* dst = peers.mbox[src];
    const int per_row = out_bytes / 16;
    uint4* ret = reinterpret_cast<uint4*>(dst + lay.ret);
    for (int r = blockIdx.x; r < cnt; r += gridDim.x) {
        const int row = pair_row[static_cast<int64_t>(src) * lay.cap + r];
        const uint4* from = reinterpret_cast<const uint4*>(down + static_cast<int64_t>(row) * out_bytes);
        for (int c = threadIdx.x; c < per_row; c += blockDim.x)
            ret[static_cast<int64_t>(off + r) * per_row + c] = __ldg(from + c);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(&done[kEpMaxRanks + src], 1) == static_cast<int>(gridDim.x) - 1) {
            __threadfence_system();
            st_release_sys(reinterpret_cast<uint32_t*>(dst + lay.flags_ret) + me, ep);
            done[kEpMaxRanks + src] = 0;
        }
    }
}

// Waits for every owner's outputs of this epoch, then advances the epoch.
__global__ void ep_p2p_ret_wait_kernel(const uint8_t* __restrict__ mbox, EpLayout lay, int world,
                                       uint32_t* __restrict__ epoch, int* __restrict__ err) {
    const uint32_t ep = *epoch + 1u;
    if (threadIdx.x < world &&
        !ep_wait_flag(reinterpret_cast<const uint32_t*>(mbox + lay.flags_ret) + threadIdx.x, ep))
        atomicCAS(err, 0, NF_DEVERR_EP_WAIT);
    __syncthreads();
    if (threadIdx.x == 0) *epoch = ep;
}

// Blocks per peer of the row copies: 64 for decode-sized mailboxes, up to
// 512 (one per 64 rows) for prefill-sized ones.
static int ep_copy_blocks(int cap) { return std::max(1, std::min(cap, std::max(64, std::min(512, cap / 64)))); }

cudaError_t launch_ep_p2p_send(const uint16_t* x, const int32_t* send_tok, const int32_t* send_e,
                               const int32_t* counts, int H, int world, int me, const EpPeers& peers,
                               const EpLayout& lay, const uint32_t* epoch, int32_t* done, cudaStream_t st) {
    const int blocks = ep_copy_blocks(lay.cap);
    ep_p2p_send_kernel<<<dim3(blocks, world), 256, 0, st>>>(x, send_tok, send_e, counts, H, me, peers, lay, epoch, done);
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_recv_wait(uint8_t* mbox, const EpLayout& lay, int world, const uint32_t* epoch,
                                    int32_t* seen, int* err, cudaStream_t st) {
    const int blocks = std::max(1, std::min(32, (lay.cap + 255) / 256));
    ep_p2p_recv_wait_kernel<<<blocks, 256, 0, st>>>(mbox, lay, world, epoch, seen, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_return(const void* down, const int32_t* pair_row, int out_bytes, int world, int me,
                                 const EpPeers& peers, const EpLayout& lay, const uint8_t* mbox, const int32_t* seen,
                                 const uint32_t* epoch, int32_t* done, cudaStream_t st) {
    const int blocks = ep_copy_blocks(lay.cap);
    ep_p2p_return_kernel<<<dim3(blocks, world), 256, 0, st>>>(static_cast<const uint8_t*>(down), pair_row, out_bytes,
                                                              me, peers, lay, mbox, seen, epoch, done);
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_ret_wait(const uint8_t* mbox, const EpLayout& lay, int world, uint32_t* epoch, int* err,
                                   cudaStream_t st) {
    ep_p2p_ret_wait_kernel<<<1, 32, 0, st>>>(mbox, lay, world, epoch, err);
    return cudaGetLastError();
}

cudaError_t launch_dequant(const uint8_t* packed, const uint8_t* scales, float gscale, int64_t rows, int64_t cols,
                           float* out, cudaStream_t st) {
    dequant_kernel<<<1184, 256, 0, st>>>(packed, scales, gscale, rows, cols, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize(const float* x, int64_t rows, int64_t cols, float gscale, uint8_t* codes,
                            uint8_t* scales, float* fake, cudaStream_t st) {
    quantize_kernel<<<1184, 256, 0, st>>>(x, rows, cols, gscale, codes, scales, fake);
    return cudaGetLastError();
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ y) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = f32_to_bf16_bits(x[i]);
}

cudaError_t launch_f32_to_bf16(const float* x, int64_t n, uint16_t* y, cudaStream_t st) {
    f32_to_bf16_kernel<<<1184, 256, 0, st>>>(x, n, y);
    return cudaGetLastError();
}

cudaError_t launch_sigmoid_ref(const float* x, int64_t n, float* y, cudaStream_t st) {
    sigmoid_ref_kernel<<<1184, 256, 0, st>>>(x, n, y);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Screened router for large batches: the reference's exact logit chains
// (gemv_bf16, src/text_forward.cpp:497-508) only where they can change the
// selection (router_select :1447-1471).
//
// 1. Approximate logits l~[t, e] come from a tensor-core GEMM of the BF16
//    tokens and router rows (fp32 accumulation in the MMA's order).
// 2. route_screen_kernel bounds |l~ - l| for the exact chain l:
//      |l - s| <= gamma_H sum|w x|  (the reference's sequential sum, exact
//                                     products: one rounding per step)
//      |l~ - s| <= H 2^-21 sum|w x| (the tensor core's accumulation, taken
//                                     eight times fp32's unit roundoff per step)
//    with s the real dot product and sum|w x| <= ||x||_2 ||w_e||_2 (the
//    norms rounded up).  choice(l) = sigmoid_ref(l) + bias is non-decreasing
//    in l (each step is a correctly rounded monotone function), so
//    [choice(l~ - B), choice(l~ + B)] (endpoints rounded outward) encloses the
//    exact choice.  At least k experts have an exact choice >= the k-th
//    largest lower end, so an expert whose upper end lies below it can never
//    be picked: the candidates are the experts whose upper end reaches it.
//    A token with a non-finite approximate logit, a token value outside
//    [2^-67, 2^20) in magnitude (products inexact, or sums near overflow), or
//    more than 32 candidates, is marked for every chain.
// 3. route_exact_kernel runs the exact chains of the candidates (all E for a
//    marked token), the exact sigmoid and bias, and the reference's selection
//    with every other expert's choice set to -inf: such an expert is below k
//    exact choices, so it is never picked, and -inf is not a NaN, so the
//    first-unused rule for NaN never reaches it.  Routes and weights are
//    therefore bit-identical to the full exact router.
// ---------------------------------------------------------------------------
constexpr int kScreenMaxCand = kScreenMaxCandHost;

__device__ __forceinline__ bool bf16_screen_unsafe(uint32_t u) {
    // a nonzero BF16 half outside [2^-67, 2^20) in magnitude, inf or NaN
    const uint32_t e0 = (u >> 7) & 0xffu, e1 = (u >> 23) & 0xffu;
    const bool nz0 = (u & 0x7fffu) != 0u, nz1 = (u & 0x7fff0000u) != 0u;
    return (nz0 && (e0 < 60u || e0 > 146u)) || (nz1 && (e1 < 60u || e1 > 146u));
}

// The exact chains of the screened candidates, packed densely over the
// threads (a chain's cost is H dependent steps whoever runs it, so a lane
// must not idle on a token with few candidates).  A CTA takes kExTok tokens
// and lists their (token, expert) chains in shared memory -- each candidate,
// or every expert of a marked token -- and thread i runs chains i, i + 256,
// i + 512, i + 768 of the list at once (further passes for longer lists),
// each sequential over the columns: fused multiply-add when the weights
// passed the bind-time range check and the token is in range (products
// exact), else the separately rounded multiply and add.  The router rows
// (the fused router's BF16 chunk-major copy, rows padded to kRouterPitch16)
// and the tokens' BF16 columns stream through shared memory in 128-column
// chunks, three stages of cp.async; the padded pitches put the rows that
// neighbouring lanes read in different banks.  The CTA's token rows are
// prefetched into L2 as one bulk request each before the first chunk, so
// the chunks' token columns come from L2 rather than from DRAM one chunk
// ahead.  Then one warp per token
// applies the exact sigmoid and bias and the reference's selection with
// every non-candidate's choice at -inf.
// Token columns of a 128-column chunk staged by TMA as two 64-column boxes
// of 32 rows with the 128-byte swizzle: row r of box b at b * 4 KB + r * 128
// bytes, its 16-byte piece q stored at piece q ^ (r & 7) (so that the rows
// eight lanes read at one column land in different banks).
constexpr int kRtXStage = 2 * 32 * 64;  // BF16 elements per stage
__device__ __forceinline__ int rt_xpiece(int tok, int q) {  // element offset of 16-byte piece q (0..15) of row tok
    return (q >> 3) * 2048 + tok * 64 + (((q & 7) ^ (tok & 7)) << 3);
}
constexpr int kExTok = 32;
constexpr int kExThreads = 256;
constexpr int kExWarps = kExThreads / 32;
constexpr int kExSlots = 4;
constexpr int kExStages = 3;
constexpr int kExMaxK = 8;  // picks per token (the screened path serves K <= 8)
// The stages are issued by lane 0 of the last warp: chains fill the threads
// from 0 up, so that warp computes only for long lists.
constexpr int kExIssuer = kExThreads - 32;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// One 128-column chunk of a chain.  MODE 0: fused multiply-add; 1: the
// separately rounded multiply and add; 2: per lane, by `fma`.
template <int MODE>
__device__ __forceinline__ float exact_chunk(const uint16_t* wr, const uint16_t* xb, int tok, float a, bool fma) {
#pragma unroll 4
    for (int k = 0; k < kRouterKc; k += 8) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wr + k);
        const uint4 xv = *reinterpret_cast<const uint4*>(xb + rt_xpiece(tok, k >> 3));
        if (MODE == 0 || (MODE == 2 && fma)) {
            a = chain_step2<true>(wv.x, xv.x, a);
            a = chain_step2<true>(wv.y, xv.y, a);
            a = chain_step2<true>(wv.z, xv.z, a);
            a = chain_step2<true>(wv.w, xv.w, a);
        } else {
            a = chain_step2<false>(wv.x, xv.x, a);
            a = chain_step2<false>(wv.y, xv.y, a);
            a = chain_step2<false>(wv.z, xv.z, a);
            a = chain_step2<false>(wv.w, xv.w, a);
        }
    }
    return a;
}

// NS chains at once, each sequential over the chunk's columns (fused
// multiply-add: every chain of the warp is in range): the chains are
// independent, so their loads and steps interleave.
template <int NS>
__device__ __forceinline__ void exact_chunk_multi(const uint16_t* wb, const uint16_t* xb, const int (&wofs)[kExSlots],
                                                  const int (&xtok)[kExSlots], float (&acc)[kExSlots]) {
#pragma unroll 2
    for (int k = 0; k < kRouterKc; k += 8) {
        uint4 wv[NS], xv[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            wv[s] = *reinterpret_cast<const uint4*>(wb + wofs[s] + k);
            xv[s] = *reinterpret_cast<const uint4*>(xb + rt_xpiece(xtok[s], k >> 3));
        }
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            float a = acc[s];
            a = chain_step2<true>(wv[s].x, xv[s].x, a);
            a = chain_step2<true>(wv[s].y, xv[s].y, a);
            a = chain_step2<true>(wv[s].z, xv[s].z, a);
            a = chain_step2<true>(wv[s].w, xv[s].w, a);
            acc[s] = a;
        }
    }
}

__global__ void __launch_bounds__(kExThreads, 2) route_exact_kernel(
    const __grid_constant__ CUtensorMap tmx, const uint16_t* __restrict__ x, const uint16_t* __restrict__ wz16,
    const float* __restrict__ bias, int T, int H,
    int E, int K, float scaling, int normalize, int w_safe, const int32_t* __restrict__ cand,
    const int32_t* __restrict__ cnt, int32_t* __restrict__ idx_out, float* __restrict__ w_out, int* __restrict__ err) {
    extern __shared__ uint8_t rx_smem_raw[];
    uint8_t* rx_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rx_smem_raw) + 1023) & ~uintptr_t(1023));
    const int wchunk = E * kRouterPitch16;  // BF16 elements of one chunk of every row
    uint16_t* sx = reinterpret_cast<uint16_t*>(rx_smem);                         // [stages][kRtXStage] (swizzled)
    uint16_t* sw = sx + kExStages * kRtXStage;                                   // [stages][wchunk]
    int32_t* s_chain = reinterpret_cast<int32_t*>(sw + kExStages * wchunk);      // [kExTok * E] token << 8 | expert
    float* s_val = reinterpret_cast<float*>(s_chain + kExTok * E);               // [kExTok * E] exact logits
    float* s_sc = s_val + kExTok * E;                                            // [kExWarps][E]
    float* s_ch = s_sc + kExWarps * E;                                           // [kExWarps][E]
    __shared__ int s_base[kExTok + 1];
    __shared__ int s_marked[kExTok];
    __shared__ int s_fma[kExTok];
    __shared__ uint32_t s_excl[kExWarps][32];
    __shared__ uint64_t full[kExStages];  // chunk stage landed (router rows + token columns)
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kExTok;
    const int ntok = min(kExTok, T - t0);
    if (threadIdx.x < ntok) prefetch_l2_bulk(x + static_cast<int64_t>(t0 + threadIdx.x) * H, static_cast<uint32_t>(H) * 2u);
    const int nchunks = H / kRouterKc;
    // Chunk g of the staging sequence (all passes) lands in buffer g % stages
    // with barrier parity (g / stages) & 1: the router rows of the chunk as
    // one bulk copy (the chunk-major copy keeps a chunk's rows contiguous, in
    // the staged pitch) and the tokens' columns as two TMA boxes (rows past
    // the batch read as zeros).
    const uint32_t wbytes = static_cast<uint32_t>(wchunk) * 2u;
    auto issue = [&](int c, int g) {
        const int buf = g % kExStages;
        mbar_arrive_expect_tx(&full[buf], wbytes + static_cast<uint32_t>(kRtXStage) * 2u);
        bulk_load(sw + buf * wchunk, wz16 + static_cast<int64_t>(c) * wchunk, wbytes, &full[buf]);
        tma_load_2d(sx + buf * kRtXStage, &tmx, &full[buf], c * kRouterKc, t0);
        tma_load_2d(sx + buf * kRtXStage + kRtXStage / 2, &tmx, &full[buf], c * kRouterKc + 64, t0);
    };
    // the first pass's first two chunks go out before the chain list is built
    // (the issuing thread initialises the barriers; the others first touch
    // them after the __syncthreads below)
    if (threadIdx.x == kExIssuer) {
        for (int i = 0; i < kExStages; ++i) mbar_init(&full[i], 1);
        s_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmx);
        issue(0, 0);
        if (nchunks > 1) issue(1, 1);
    }

    // the chain list: per-token counts, their prefix, then the entries
    if (warp == 0) {
        const int c = lane < ntok ? cnt[t0 + lane] : 0;
        const int n = c < 0 ? E : c;
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane < kExTok) {
            s_base[lane] = incl - n;
            s_marked[lane] = c < 0 ? 1 : 0;
        }
        if (lane == 31) s_base[kExTok] = incl;
    }
    __syncthreads();  // (also publishes the barrier initialisation)
    {
        // a warp's tokens tl = warp + 8 i; their candidate loads go out together
        constexpr int kPer = kExTok / kExWarps;
        int cv[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int tl = warp + i * kExWarps;
            cv[i] = 0;
            if (tl < ntok && !s_marked[tl] && lane < s_base[tl + 1] - s_base[tl])
                cv[i] = cand[static_cast<int64_t>(t0 + tl) * kScreenMaxCand + lane];
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int tl = warp + i * kExWarps;
            if (tl >= ntok) break;  // (warp-uniform)
            const int t = t0 + tl;
            const int base = s_base[tl], n = s_base[tl + 1] - base;
            const bool marked = s_marked[tl] != 0;
            if (marked) {
                for (int j = lane; j < n; j += 32) s_chain[base + j] = (tl << 8) | j;
            } else if (lane < n) {
                s_chain[base + lane] = (tl << 8) | cv[i];
            }
            // a token the screen passed is in range; a marked one may not be
            int xbad = 0;
            if (marked)
                for (int q = lane; q < H / 2; q += 32)
                    xbad |= bf16x2_unsafe(reinterpret_cast<const uint32_t*>(x + static_cast<int64_t>(t) * H)[q]) ? 1 : 0;
            xbad = __any_sync(0xffffffffu, xbad);
            if (lane == 0) s_fma[tl] = (w_safe && !xbad) ? 1 : 0;
        }
    }
    __syncthreads();
    const int total = s_base[kExTok];
    int staged = 0;  // chunks staged by earlier passes
    for (int p0 = 0; p0 < total; p0 += kExThreads * kExSlots) {
        int wofs[kExSlots], xtok[kExSlots];
        bool fm[kExSlots];
        float acc[kExSlots];
#pragma unroll
        for (int j = 0; j < kExSlots; ++j) {
            const int ci = p0 + j * kExThreads + threadIdx.x;
            const int ch = ci < total ? s_chain[ci] : 0;  // a lane past the list runs token 0 / expert 0, unused
            wofs[j] = (ch & 0xff) * kRouterPitch16;
            xtok[j] = ch >> 8;
            fm[j] = ci < total ? s_fma[ch >> 8] != 0 : true;
            acc[j] = 0.f;
        }
        // this warp's live slots, and whether all their chains take the fused form
        int ns = 0;
        bool all_fma = true;
#pragma unroll
        for (int j = 0; j < kExSlots; ++j) {
            if (p0 + j * kExThreads + warp * 32 < total) {
                ns = j + 1;
                all_fma = all_fma && __all_sync(0xffffffffu, fm[j]);
            }
        }
        if (threadIdx.x == kExIssuer && p0 > 0) {
            issue(0, staged);
            if (nchunks > 1) issue(1, staged + 1);
        }
        for (int c = 0; c < nchunks; ++c) {
            const int g = staged + c, buf = g % kExStages;
            const bool landed = mbar_wait(&full[buf], static_cast<uint32_t>((g / kExStages) & 1), &s_abort, err);
            // chunk c is in place for every thread, and every thread is done with chunk c - 1
            if (!__syncthreads_and(landed ? 1 : 0)) {
                // a stage never landed: record it, let every issued copy land, leave
                if (threadIdx.x == 0) {
                    atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
                    const int issued_end = staged + min(nchunks, c + 2);
                    for (int q = g; q < issued_end; ++q) {
                        const uint64_t tw = globaltimer_ns();
                        while (!mbar_try_wait(&full[q % kExStages], static_cast<uint32_t>((q / kExStages) & 1))) {
                            if (globaltimer_ns() - tw > NF_WAIT_BUDGET_NS) {
                                atomicCAS(err, 0, NF_DEVERR_DRAIN);
                                break;
                            }
                        }
                    }
                }
                __syncthreads();
                return;
            }
            if (threadIdx.x == kExIssuer && c + 2 < nchunks) issue(c + 2, g + 2);
            const uint16_t* wb = sw + buf * wchunk;
            const uint16_t* xb = sx + buf * kRtXStage;
            if (all_fma) {
                switch (ns) {
                    case 1: exact_chunk_multi<1>(wb, xb, wofs, xtok, acc); break;
                    case 2: exact_chunk_multi<2>(wb, xb, wofs, xtok, acc); break;
                    case 3: exact_chunk_multi<3>(wb, xb, wofs, xtok, acc); break;
                    case 4: exact_chunk_multi<4>(wb, xb, wofs, xtok, acc); break;
                    default: break;
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < kExSlots; ++j) {
                if (p0 + j * kExThreads + warp * 32 >= total) break;  // (warp-uniform) no chain in this slot
                const bool all_f = __all_sync(0xffffffffu, fm[j]);
                const bool none_f = __all_sync(0xffffffffu, !fm[j]);
                if (all_f)
                    acc[j] = exact_chunk<0>(wb + wofs[j], xb, xtok[j], acc[j], true);
                else if (none_f)
                    acc[j] = exact_chunk<1>(wb + wofs[j], xb, xtok[j], acc[j], false);
                else
                    acc[j] = exact_chunk<2>(wb + wofs[j], xb, xtok[j], acc[j], fm[j]);
            }
        }
        staged += nchunks;
#pragma unroll
        for (int j = 0; j < kExSlots; ++j) {
            const int ci = p0 + j * kExThreads + threadIdx.x;
            if (ci < total) s_val[ci] = acc[j];
        }
        __syncthreads();  // the buffers are restaged by the next pass; s_val complete
    }

    // selection.  Every chain's score and choice (one thread per chain, into
    // the staging buffers, free now), then one thread per token over its
    // candidates in expert order: each pick is the largest choice among the
    // unused candidates, lowest index among equals -- the reference's rule,
    // since every other expert's choice is -inf and a screened token's
    // choices are finite.  Tokens that run every chain (possibly NaN
    // choices) take the warp form of the full rule.
    float* c_sc = reinterpret_cast<float*>(sw);  // [total]
    float* c_ch = c_sc + kExTok * E;             // [total]
    for (int ci = threadIdx.x; ci < total; ci += kExThreads) {
        const float sg = sigmoid_ref(s_val[ci]);
        c_sc[ci] = sg;
        c_ch[ci] = __fadd_rn(sg, bias[s_chain[ci] & 0xff]);
    }
    __syncthreads();
    if (threadIdx.x < ntok && !s_marked[threadIdx.x]) {
        const int tl = threadIdx.x, t = t0 + tl;
        const int base = s_base[tl], n = s_base[tl + 1] - base;  // K <= n <= kScreenMaxCand
        uint32_t used = 0u;
        int pk[kExMaxK];
        float wt[kExMaxK];
#pragma unroll
        for (int p = 0; p < kExMaxK; ++p) {
            pk[p] = 0;
            wt[p] = 0.f;
            if (p < K) {
                int best = -1;
                float bc = 0.f;
                for (int j = 0; j < n; ++j) {
                    if ((used >> j) & 1u) continue;
                    const float cj = c_ch[base + j];
                    if (best < 0 || cj > bc) {
                        best = j;
                        bc = cj;
                    }
                }
                best = max(best, 0);
                used |= 1u << best;
                pk[p] = s_chain[base + best] & 0xff;
                wt[p] = c_sc[base + best];
            }
        }
        if (normalize) {
            float sum = 1e-20f;
#pragma unroll
            for (int p = 0; p < kExMaxK; ++p)
                if (p < K) sum = __fadd_rn(sum, wt[p]);
#pragma unroll
            for (int p = 0; p < kExMaxK; ++p)
                if (p < K) wt[p] = __fmul_rn(__fdiv_rn(wt[p], sum), scaling);
        }
#pragma unroll
        for (int p = 0; p < kExMaxK; ++p) {
            if (p < K) {
                idx_out[static_cast<int64_t>(t) * K + p] = pk[p];
                w_out[static_cast<int64_t>(t) * K + p] = wt[p];
            }
        }
    }
    float* sc = s_sc + warp * E;
    float* chv = s_ch + warp * E;
    for (int tl = warp; tl < ntok; tl += kExWarps) {
        if (!s_marked[tl]) continue;  // (warp-uniform)
        const int t = t0 + tl;
        const int base = s_base[tl];  // every expert, in order
        for (int e = lane; e < E; e += 32) {
            sc[e] = c_sc[base + e];
            chv[e] = c_ch[base + e];
        }
        __syncwarp();
        warp_select_reg<(kRouterMaxE + 31) / 32>(sc, chv, E, K, scaling, normalize, 1, 1, s_excl[warp],
                                                 idx_out + static_cast<int64_t>(t) * K,
                                                 w_out + static_cast<int64_t>(t) * K);
        __syncwarp();
    }
}

size_t route_exact_smem(int E) {
    return 1024 + static_cast<size_t>(kExStages) * E * kRouterPitch16 * 2 + static_cast<size_t>(kExStages) * kRtXStage * 2 +
           static_cast<size_t>(2) * kExTok * E * 4 + static_cast<size_t>(2) * kExWarps * E * 4;
}

// bf16_screen_unsafe for both halves at once, as flags (bit 15: low half,
// bit 31: high half) from the magnitudes m (15 bits per 16-bit lane, so no
// carry crosses lanes): m >= 147 << 7 sets bit 15 of m + 0x3680; 0 < m <
// 60 << 7 leaves bit 15 of m + 0x6200 clear and sets that of m + 0x7fff.
__device__ __forceinline__ uint32_t bf16x2_screen_flags(uint32_t u) {
    const uint32_t m = u & 0x7fff7fffu;
    return ((m + 0x36803680u) | (~(m + 0x62006200u) & (m + 0x7fff7fffu))) & 0x80008000u;
}
// (lo, hi) += (a_lo^2, a_hi^2) per lane, rounded toward +inf (fmaf_ru on each lane)
__device__ __forceinline__ void sq_acc_ru2(uint64_t& acc, float lo, float hi) {
    const uint64_t a = (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
    asm("fma.rp.f32x2 %0, %1, %1, %0;" : "+l"(acc) : "l"(a));
}

// Fused screen: 32 tokens per CTA, 4 warps.  The token rows and the router
// rows ([E, H] BF16) stream through shared memory in 128-column chunks
// (three cp.async stages, rows padded to 272 bytes so that ldmatrix is
// conflict-free); warp w multiplies tokens 16 (w & 1) .. + 16 by experts
// (w >> 1) E / 2 .. + E / 2 with mma.sync m16n8k16 (BF16 in, fp32
// accumulate).  Meanwhile four threads per token sum the token's squares
// (fused multiply-adds rounded upward, so the sum bounds the exact one from
// above) and check its range.  Then four threads per token bound the logits
// and list the candidates, a quarter of the experts each.
constexpr int kScTok = 32;
constexpr int kScThreads = 128;
constexpr int kScStages = 3;
constexpr int kScPitch = kRouterKc + 8;  // BF16 elements per staged row (272 bytes)
constexpr int kScMaxK = 8;

// The interval ends use a float sigmoid: expf is within 2 ulp of e^x and
// __fdividef within 2 ulp of the quotient for a divisor in [1, 2] (CUDA's
// documented bounds).  With z = e^-|x| <= 1: |z~ - z| <= 2^-22, the rounded
// 1 + z~ adds 2^-24, and the quotient (at most 1) 2^-23, so
// |sig_screen(x) - sigma(x)| <= 2^-22 + 2^-24 + 2^-23 < 2^-21; sigmoid_ref,
// the reference's float evaluation, is within 2^-22 of sigma.  Widening by
// kSigMargin = 2^-19 and adding the bias with outward rounding therefore
// keeps [lo, hi] around fadd_rn(sigmoid_ref(l), bias) for every l in
// [la, ha] (sigmoid_ref and round-to-nearest are non-decreasing).
__device__ __forceinline__ float sig_screen(float x) {
    const float z = expf(-fabsf(x));
    const float d = __fadd_rn(1.f, z);
    return __fdividef(x >= 0.f ? 1.f : z, d);
}
constexpr float kSigMargin = 1.9073486328125e-06f;  // 2^-19

__global__ void __launch_bounds__(kScThreads) route_screen_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                  const uint16_t* __restrict__ x, int T, int H,
                                                                  const uint16_t* __restrict__ wz16, int E, int K,
                                                                  const float* __restrict__ bias,
                                                                  const float* __restrict__ wnorm, float c,
                                                                  int32_t* __restrict__ cand,
                                                                  int32_t* __restrict__ cnt,
                                                                  float* __restrict__ approx, int* __restrict__ err) {
    extern __shared__ uint8_t sc_smem_raw[];
    uint8_t* sc_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint16_t* sx = reinterpret_cast<uint16_t*>(sc_smem);                // [stages][kRtXStage] (swizzled)
    uint16_t* sw = sx + kScStages * kRtXStage;                          // [stages][E][kScPitch]
    float* slog = reinterpret_cast<float*>(sw + kScStages * E * kScPitch);  // [kScTok][E + 1]
    __shared__ uint64_t full[kScStages];  // chunk stage landed (token columns + router rows)
    __shared__ float s_wn[kRouterMaxE], s_bias[kRouterMaxE];
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kScTok;
    const int ntok = min(kScTok, T - t0);
    const int nchunks = H / kRouterKc;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kScStages; ++i) mbar_init(&full[i], 1);
        s_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmx);
    }
    for (int e = threadIdx.x; e < E; e += kScThreads) {
        s_wn[e] = wnorm[e];
        s_bias[e] = bias[e];
    }
    __syncthreads();
    // Chunk ch lands in buffer ch % stages with barrier parity (ch / stages) & 1:
    // the tokens' columns as two TMA boxes (rows past the batch read as
    // zeros) and the router rows of the chunk as one bulk copy (the
    // chunk-major copy keeps them contiguous, in the staged pitch).  Thread 0
    // issues.
    const int wchunk = E * kScPitch;
    const uint32_t wbytes = static_cast<uint32_t>(wchunk) * 2u;
    auto issue = [&](int ch) {
        const int buf = ch % kScStages;
        mbar_arrive_expect_tx(&full[buf], wbytes + static_cast<uint32_t>(kRtXStage) * 2u);
        tma_load_2d(sx + buf * kRtXStage, &tmx, &full[buf], ch * kRouterKc, t0);
        tma_load_2d(sx + buf * kRtXStage + kRtXStage / 2, &tmx, &full[buf], ch * kRouterKc + 64, t0);
        bulk_load(sw + buf * wchunk, wz16 + static_cast<int64_t>(ch) * wchunk, wbytes, &full[buf]);
    };
    // warp tile: 16 tokens x E / 2 experts (nt n-tiles of 8)
    const int tok0 = 16 * (warp & 1);
    const int ex0 = (warp >> 1) * (E / 2);
    const int nt = E / 16;  // n-tiles per warp (E % 16 == 0, E <= 128)
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    // thread -> token tid / 4 and quarter tid % 4 (norm: columns 32 q .. + 32 of each chunk)
    const int tl = threadIdx.x >> 2, tq = threadIdx.x & 3;
    uint64_t ss2 = 0;  // (sum of the low halves' squares, of the high halves')
    uint32_t badf = 0u;
    int bad = 0;
    if (threadIdx.x == 0) {
        issue(0);
        if (nchunks > 1) issue(1);
    }
    for (int ch = 0; ch < nchunks; ++ch) {
        const int buf = ch % kScStages;
        const bool landed = mbar_wait(&full[buf], static_cast<uint32_t>((ch / kScStages) & 1), &s_abort, err);
        // chunk ch is in place for every thread, and every thread is done with chunk ch - 1
        if (!__syncthreads_and(landed ? 1 : 0)) {
            // a stage never landed: record it, let every issued copy land, leave
            if (threadIdx.x == 0) {
                atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
                for (int q = ch; q < min(nchunks, ch + 2); ++q) {
                    const uint64_t tw = globaltimer_ns();
                    while (!mbar_try_wait(&full[q % kScStages], static_cast<uint32_t>((q / kScStages) & 1))) {
                        if (globaltimer_ns() - tw > NF_WAIT_BUDGET_NS) {
                            atomicCAS(err, 0, NF_DEVERR_DRAIN);
                            break;
                        }
                    }
                }
            }
            __syncthreads();
            if (threadIdx.x < ntok) cnt[t0 + threadIdx.x] = -1;  // every chain for these tokens
            return;
        }
        if (threadIdx.x == 0 && ch + 2 < nchunks) issue(ch + 2);
        const uint16_t* xb = sx + buf * kRtXStage;
        const uint16_t* wb = sw + buf * wchunk;
        if (tl < ntok) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 v = *reinterpret_cast<const uint4*>(xb + rt_xpiece(tl, 4 * tq + i));
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    badf |= bf16x2_screen_flags(w4[j]);
                    sq_acc_ru2(ss2, bf16_lo(w4[j]), bf16_hi(w4[j]));
                }
            }
        }
        // A: lanes 0-15 give rows tok0 + 0..15 at the k-step's first 8 columns,
        // lanes 16-31 the same rows at its second 8 (pieces 2 s, 2 s + 1)
        const int arow = tok0 + (lane & 15);
        const uint32_t xb_u32 = smem_u32(xb);
        const uint32_t b_addr =
            smem_u32(wb + (ex0 + (lane & 7) + 8 * (lane >> 4)) * kScPitch + 8 * ((lane >> 3) & 1));
#pragma unroll
        for (int s = 0; s < kRouterKc / 16; ++s) {
            uint32_t a[4];
            ldsm_x4(xb_u32 + 2 * rt_xpiece(arow, 2 * s + (lane >> 4)), a);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                if (2 * p >= nt) break;
                uint32_t b[4];
                ldsm_x4(b_addr + 16 * p * kScPitch * 2 + 32 * s, b);
                mma_16816(acc[2 * p], a[0], a[1], a[2], a[3], b[0], b[1]);
                mma_16816(acc[2 * p + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
            }
        }
    }
    // logits to shared memory (row g and g + 8 of the warp's tile, columns 2 (lane % 4) + {0, 1})
    const int g = lane >> 2, q2 = 2 * (lane & 3);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i >= nt) break;
        float* r0 = slog + (tok0 + g) * (E + 1) + ex0 + 8 * i + q2;
        float* r1 = r0 + 8 * (E + 1);
        r0[0] = acc[i][0];
        r0[1] = acc[i][1];
        r1[0] = acc[i][2];
        r1[1] = acc[i][3];
    }
    // ||x_t||_2 over the four threads of a token, rounded up at every step
    bad |= badf != 0u ? 1 : 0;
    float ss = __fadd_ru(__uint_as_float(static_cast<uint32_t>(ss2)), __uint_as_float(static_cast<uint32_t>(ss2 >> 32)));
    ss = __fadd_ru(ss, __shfl_xor_sync(0xffffffffu, ss, 1));
    ss = __fadd_ru(ss, __shfl_xor_sync(0xffffffffu, ss, 2));
    bad |= __shfl_xor_sync(0xffffffffu, bad, 1);
    bad |= __shfl_xor_sync(0xffffffffu, bad, 2);
    const float nx = __fsqrt_ru(ss);
    __syncthreads();
    // Choice intervals of this thread's quarter of the experts; the K largest
    // lower ends (with multiplicity) by insertion, merged over the token's four
    // threads; the upper ends overwrite the logits in shared memory.
    const int t = t0 + tl;
    const bool live = tl < ntok;
    float* lrow = slog + tl * (E + 1);
    const int per = E / 4;
    const float cn = __fmul_ru(c, nx);
    float top[kScMaxK];
#pragma unroll
    for (int i = 0; i < kScMaxK; ++i) top[i] = -INFINITY;
#pragma unroll 4
    for (int j = 0; j < per; ++j) {
        const int e = tq * per + j;
        const float l = lrow[e];
        if (live && approx) approx[static_cast<int64_t>(t) * E + e] = l;  // (kept for inspection)
        const float B = __fmul_ru(cn, s_wn[e]);
        const float la = __fsub_rd(l, B), ha = __fadd_ru(l, B);
        if (!isfinite(l) || !isfinite(la) || !isfinite(ha)) {
            bad = 1;
            continue;
        }
        float v = __fadd_rd(__fsub_rd(sig_screen(la), kSigMargin), s_bias[e]);
        lrow[e] = __fadd_ru(__fadd_ru(sig_screen(ha), kSigMargin), s_bias[e]);
#pragma unroll
        for (int i = 0; i < kScMaxK; ++i) {
            if (i >= K) break;
            const float a = top[i];
            const bool gt = v > a;
            top[i] = gt ? v : a;
            v = gt ? a : v;
        }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        float other[kScMaxK];
#pragma unroll
        for (int i = 0; i < kScMaxK; ++i) other[i] = __shfl_xor_sync(0xffffffffu, top[i], o);
#pragma unroll
        for (int m = 0; m < kScMaxK; ++m) {
            if (m >= K) break;
            float v = other[m];
#pragma unroll
            for (int i = 0; i < kScMaxK; ++i) {
                if (i >= K) break;
                const float a = top[i];
                const bool gt = v > a;
                top[i] = gt ? v : a;
                v = gt ? a : v;
            }
        }
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    float kth = top[0];
#pragma unroll
    for (int i = 1; i < kScMaxK; ++i)
        if (i < K) kth = top[i];
    // candidates: the experts whose upper end reaches the k-th largest lower end
    int n = 0;
    if (!bad)
        for (int j = 0; j < per; ++j) n += lrow[tq * per + j] >= kth ? 1 : 0;
    const int base_lane = lane & ~3;
    int before = 0, total = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int nq = __shfl_sync(0xffffffffu, n, base_lane + q);
        before += q < tq ? nq : 0;
        total += nq;
    }
    if (!live) return;
    if (bad) {
        if (tq == 0) cnt[t] = -1;
        return;
    }
    int32_t* out = cand + static_cast<int64_t>(t) * kScreenMaxCand;
    int slot = before;
    for (int j = 0; j < per && slot < kScreenMaxCand; ++j) {
        const int e = tq * per + j;
        if (lrow[e] >= kth) out[slot++] = e;
    }
    if (tq == 0) cnt[t] = total <= kScreenMaxCand ? total : -1;
}

size_t route_screen_smem(int E) {
    return 1024 + static_cast<size_t>(kScStages) * (kRtXStage + E * kScPitch) * 2 + static_cast<size_t>(kScTok) * (E + 1) * 4;
}

cudaError_t launch_route_screen(const CUtensorMap& tmx, const uint16_t* x, int T, int H, const uint16_t* wz16, int E,
                                int K, const float* bias, const float* wnorm, float c, int32_t* cand, int32_t* cnt,
                                float* approx, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (E % 16 != 0 || E > kRouterMaxE || H % kRouterKc != 0 || K < 1 || K > kScMaxK) return cudaErrorInvalidValue;
    static bool attr[kMaxDevices] = {};
    cudaError_t e = smem_attr_once(route_screen_kernel, static_cast<int>(route_screen_smem(kRouterMaxE)), attr);
    if (e != cudaSuccess) return e;
    route_screen_kernel<<<(T + kScTok - 1) / kScTok, kScThreads, route_screen_smem(E), st>>>(
        tmx, x, T, H, wz16, E, K, bias, wnorm, c, cand, cnt, approx, err);
    return cudaGetLastError();
}

cudaError_t launch_route_exact(const CUtensorMap& tmx, const uint16_t* x, const uint16_t* wz16, const float* bias, int T,
                               int H, int E, int K,
                               float scaling, int normalize, int w_safe, const int32_t* cand, const int32_t* cnt,
                               int32_t* idx, float* wts, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (K < 1 || K > kExMaxK || E > kRouterMaxE) return cudaErrorInvalidValue;
    const size_t smem = route_exact_smem(E);
    static bool attr[kMaxDevices] = {};
    cudaError_t e = smem_attr_once(route_exact_kernel, static_cast<int>(route_exact_smem(kRouterMaxE)), attr);
    if (e != cudaSuccess) return e;
    route_exact_kernel<<<(T + kExTok - 1) / kExTok, kExThreads, smem, st>>>(
        tmx, x, wz16, bias, T, H, E, K, scaling, normalize, w_safe, cand, cnt, idx, wts, err);
    return cudaGetLastError();
}

}  // namespace nf
