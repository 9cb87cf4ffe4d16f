// nf_kernels.cu -- router, token permutation / dispatch (with the fused
// NVFP4 activation quantiser), weighted combine + residual, and the
// stand-alone format kernels (dequantise, quantise, reference sigmoid).
//
// These kernels are HBM- or latency-bound integer/byte and scalar work; they
// use plain coalesced loads, shared-memory staging and grids sized from the
// SM count.  The contractions live in nf_gemm.cu.
#include "nf_common.cuh"
#include "nf_internal.h"

#include "_gen/sigmoid_table.inc"

namespace nf {

// ---------------------------------------------------------------------------
// Sigmoid exactly as the reference computes it (src/text_forward.cpp:42-49).
// exp is evaluated in double and rounded once (a correctly rounded expf);
// the arguments where libm's expf gives a different sigmoid come from the
// build-time exception table.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid_ref(float x) {
    float r;
    if (x >= 0.f) {
        const float z = static_cast<float>(exp(-static_cast<double>(x)));
        r = __fdiv_rn(1.f, __fadd_rn(1.f, z));
    } else {
        const float z = static_cast<float>(exp(static_cast<double>(x)));
        r = __fdiv_rn(z, __fadd_rn(1.f, z));
    }
    const uint32_t key = __float_as_uint(x);
    int lo = 0, hi = NF_SIG_TABLE_N - 1;
    while (lo <= hi) {
        const int mid = (lo + hi) >> 1;
        const uint32_t k = g_sig_keys[mid];
        if (k == key) return __uint_as_float(g_sig_vals[mid]);
        if (k < key) lo = mid + 1;
        else hi = mid - 1;
    }
    return r;
}

__global__ void sigmoid_ref_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = sigmoid_ref(x[i]);
}

// ---------------------------------------------------------------------------
// Router logits: gemv_bf16 (src/text_forward.cpp:497-508) for every token:
// logits[t, e] = sum_c bf16(W[e, c]) * x[t, c], accumulated sequentially in
// fp32 with separate multiply and add (no fused multiply-add), which is what
// makes the result bit-identical to the reference.  A CTA stages
// kRouterTok tokens of x in shared memory; each thread runs 4 independent
// chains (4 tokens of one expert) for instruction-level parallelism.
// ---------------------------------------------------------------------------
constexpr int kRouterTok = 16;

__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w, int T, int H, int E,
                                                            float* __restrict__ logits) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);  // [kRouterTok][H]
    const int t0 = blockIdx.x * kRouterTok;
    const int nt = min(kRouterTok, T - t0);
    // stage x rows (16-byte vectors; H % 8 == 0)
    const int vec_per_row = H / 8;
    for (int i = threadIdx.x; i < kRouterTok * vec_per_row; i += blockDim.x) {
        const int r = i / vec_per_row, c = i % vec_per_row;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < nt) v = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + r) * H)[c];
        reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * H)[c] = v;
    }
    __syncthreads();
    const int items = E * (kRouterTok / 4);
    for (int item = threadIdx.x; item < items; item += blockDim.x) {
        const int e = item % E, tq = item / E;
        const uint16_t* wr = w + static_cast<int64_t>(e) * H;
        const uint16_t* x0 = xs + static_cast<int64_t>(tq * 4) * H;
        float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
        for (int c = 0; c < H; c += 8) {
            const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
            const uint4 a = *reinterpret_cast<const uint4*>(x0 + c);
            const uint4 b = *reinterpret_cast<const uint4*>(x0 + H + c);
            const uint4 d = *reinterpret_cast<const uint4*>(x0 + 2 * H + c);
            const uint4 f = *reinterpret_cast<const uint4*>(x0 + 3 * H + c);
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
            const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
            const uint32_t dd[4] = {d.x, d.y, d.z, d.w}, ff[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int sh = 16 * h;
                    const float wf = __uint_as_float(((ww[j] >> sh) & 0xffffu) << 16);
                    acc0 = __fadd_rn(acc0, __fmul_rn(wf, __uint_as_float(((aa[j] >> sh) & 0xffffu) << 16)));
                    acc1 = __fadd_rn(acc1, __fmul_rn(wf, __uint_as_float(((bb[j] >> sh) & 0xffffu) << 16)));
                    acc2 = __fadd_rn(acc2, __fmul_rn(wf, __uint_as_float(((dd[j] >> sh) & 0xffffu) << 16)));
                    acc3 = __fadd_rn(acc3, __fmul_rn(wf, __uint_as_float(((ff[j] >> sh) & 0xffffu) << 16)));
                }
            }
        }
        const int tb = t0 + tq * 4;
        if (tb + 0 < T) logits[static_cast<int64_t>(tb + 0) * E + e] = acc0;
        if (tb + 1 < T) logits[static_cast<int64_t>(tb + 1) * E + e] = acc1;
        if (tb + 2 < T) logits[static_cast<int64_t>(tb + 2) * E + e] = acc2;
        if (tb + 3 < T) logits[static_cast<int64_t>(tb + 3) * E + e] = acc3;
    }
}

// ---------------------------------------------------------------------------
// Router selection: router_select (src/text_forward.cpp:1447-1471).  One warp
// per token: the lanes evaluate score = sigmoid(logit) and choice = score +
// bias for every expert into shared memory, then lane 0 runs the reference's
// sequential scan (strict '>' from the lowest unused index), so ties and NaN
// behave exactly as in the reference.  With n_group > 1 the group-limited
// form (a group scores the sum of its two best choices, topk_group groups
// stay eligible, lower group index on ties) masks the other experts first;
// the reference has no group limit.
// ---------------------------------------------------------------------------
constexpr int kSelectWarps = 4;

__global__ void __launch_bounds__(kSelectWarps * 32) router_select_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int T, int E, int K, float scaling,
    int normalize, int n_group, int topk_group, int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
    extern __shared__ float s_sel[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* score = s_sel + static_cast<int64_t>(warp) * 2 * E;
    float* choice = score + E;
    const int t = blockIdx.x * kSelectWarps + warp;
    if (t >= T) return;
    const float* lg = logits + static_cast<int64_t>(t) * E;
    for (int e = lane; e < E; e += 32) {
        const float s = sigmoid_ref(lg[e]);
        score[e] = s;
        choice[e] = __fadd_rn(s, bias[e]);
    }
    __syncwarp();
    if (lane != 0) return;
    uint32_t used[32];  // E <= 1024
    for (int i = 0; i < 32; ++i) used[i] = 0u;
    if (n_group > 1 && topk_group < n_group) {
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
            if (!(keep & (1u << (e / per)))) used[e >> 5] |= 1u << (e & 31);
    }
    int picks[32];
    float wts[32];
    for (int p = 0; p < K; ++p) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
            if (used[e >> 5] & (1u << (e & 31))) continue;
            if (best < 0 || choice[e] > choice[best]) best = e;
        }
        if (best < 0) best = 0;
        used[best >> 5] |= 1u << (best & 31);
        picks[p] = best;
        wts[p] = score[best];
    }
    if (normalize) {
        float sum = 1e-20f;
        for (int p = 0; p < K; ++p) sum = __fadd_rn(sum, wts[p]);
        for (int p = 0; p < K; ++p) wts[p] = __fmul_rn(__fdiv_rn(wts[p], sum), scaling);
    }
    for (int p = 0; p < K; ++p) {
        idx_out[static_cast<int64_t>(t) * K + p] = picks[p];
        w_out[static_cast<int64_t>(t) * K + p] = wts[p];
    }
}

// ---------------------------------------------------------------------------
// Permutation.  Output order is (expert, token): each expert owns a
// contiguous segment of permuted rows that starts on a multiple of 128 (the
// GEMM tile height and the scale-factor atom height), and within a segment
// rows follow token order.  The order is fully deterministic.
//   hist    : per chunk of kChunkTok tokens, tokens routed to each expert
//   scan    : per-expert totals, chunk bases, 128-aligned segment offsets,
//             padding rows marked -1, GEMM tile lists
//   scatter : row of every (token, pick), token of every row, and the
//             dispatch of x into the permuted activation buffer (NVFP4
//             quantised with the expert's gate input_scale, or BF16 copied)
// ---------------------------------------------------------------------------
constexpr int kChunkTok = 128;

__global__ void permute_hist_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                    int32_t* __restrict__ chunk_counts) {
    extern __shared__ int32_t cnt[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int t0 = blockIdx.x * kChunkTok;
    const int n = min(kChunkTok, T - t0) * K;
    for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[idx[static_cast<int64_t>(t0) * K + i]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[static_cast<int64_t>(blockIdx.x) * E + e] = cnt[e];
}

__global__ void __launch_bounds__(1024) permute_scan_kernel(const int32_t* __restrict__ chunk_counts, int nchunks,
                                                            int E, int nb_gu, int nb_down,
                                                            int32_t* __restrict__ chunk_base,
                                                            int32_t* __restrict__ counts,
                                                            int32_t* __restrict__ seg_off,
                                                            int32_t* __restrict__ row_token, NfTile* __restrict__ tiles_gu,
                                                            NfTile* __restrict__ tiles_down,
                                                            int32_t* __restrict__ meta) {
    extern __shared__ int32_t sh[];
    int32_t* s_cnt = sh;             // [E]
    int32_t* s_off = sh + E;         // [E + 1]
    int32_t* s_mt = sh + 2 * E + 1;  // [E + 1] m-tile prefix
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int32_t run = 0;
        for (int c = 0; c < nchunks; ++c) {
            chunk_base[static_cast<int64_t>(c) * E + e] = run;
            run += chunk_counts[static_cast<int64_t>(c) * E + e];
        }
        s_cnt[e] = run;
        counts[e] = run;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t off = 0, mt = 0;
        for (int e = 0; e < E; ++e) {
            s_off[e] = off;
            s_mt[e] = mt;
            const int32_t m = (s_cnt[e] + 127) / 128;
            off += m * 128;
            mt += m;
        }
        s_off[E] = off;
        s_mt[E] = mt;
        meta[0] = off;             // rows in use
        meta[1] = mt * nb_gu;      // gate/up tiles
        meta[2] = mt * nb_down;    // down tiles
        meta[3] = mt;              // m-tiles
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= E; e += blockDim.x) seg_off[e] = s_off[e];
    // padding rows of every segment
    for (int e = 0; e < E; ++e) {
        const int32_t beg = s_off[e] + s_cnt[e], end = s_off[e + 1];
        for (int r = beg + threadIdx.x; r < end; r += blockDim.x) row_token[r] = -1;
    }
    // tile lists, ordered (expert, n_block, m_tile) so that CTAs working at
    // the same time share the weight block through L2
    for (int e = 0; e < E; ++e) {
        const int32_t mtiles = s_mt[e + 1] - s_mt[e];
        if (mtiles == 0) continue;
        const int32_t base_gu = s_mt[e] * nb_gu, base_dn = s_mt[e] * nb_down;
        for (int i = threadIdx.x; i < mtiles * nb_gu; i += blockDim.x) {
            const int n = i / mtiles, m = i % mtiles;
            NfTile t;
            t.expert = e;
            t.row0 = s_off[e] + m * 128;
            t.n_block = n;
            t.m_valid = min(128, s_cnt[e] - m * 128);
            tiles_gu[base_gu + i] = t;
        }
        for (int i = threadIdx.x; i < mtiles * nb_down; i += blockDim.x) {
            const int n = i / mtiles, m = i % mtiles;
            NfTile t;
            t.expert = e;
            t.row0 = s_off[e] + m * 128;
            t.n_block = n;
            t.m_valid = min(128, s_cnt[e] - m * 128);
            tiles_down[base_dn + i] = t;
        }
    }
}

// One CTA per chunk of kChunkTok tokens, 256 threads.
__global__ void __launch_bounds__(256) permute_scatter_kernel(
    const int32_t* __restrict__ idx, const uint16_t* __restrict__ x, int T, int K, int E, int H,
    const int32_t* __restrict__ chunk_base, const int32_t* __restrict__ seg_off,
    const float* __restrict__ gscale,  // [E] 1 / gate input_scale (NVFP4 mode)
    int bf16_mode, int32_t* __restrict__ pair_row, int32_t* __restrict__ row_token, uint8_t* __restrict__ a_codes,
    uint8_t* __restrict__ a_sf, uint16_t* __restrict__ a_bf16) {
    extern __shared__ int32_t sh[];
    int32_t* s_run = sh;                        // [E] running count inside the chunk
    int32_t* s_rows = sh + E;                   // [kChunkTok * K] permuted row of each pick
    int32_t* s_pe = s_rows + kChunkTok * K;     // [kChunkTok * K] expert of each pick
    const int t0 = blockIdx.x * kChunkTok;
    const int nt = min(kChunkTok, T - t0);
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_run[e] = 0;
    for (int i = threadIdx.x; i < nt * K; i += blockDim.x) s_pe[i] = idx[static_cast<int64_t>(t0) * K + i];
    __syncthreads();
    // ranks inside the chunk, in token order (one warp, rounds of 32 tokens)
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        for (int r0 = 0; r0 < nt; r0 += 32) {
            const int tl = r0 + lane;
            const bool valid = tl < nt;
            const int lanes = min(32, nt - r0);
            if (valid) {
                for (int p = 0; p < K; ++p) {
                    const int e = s_pe[tl * K + p];
                    int rank = 0;
                    for (int l = 0; l < lane; ++l)
                        for (int q = 0; q < K; ++q) rank += (s_pe[(r0 + l) * K + q] == e) ? 1 : 0;
                    s_rows[tl * K + p] =
                        seg_off[e] + chunk_base[static_cast<int64_t>(blockIdx.x) * E + e] + s_run[e] + rank;
                }
            }
            __syncwarp();
            if (lane == 0)
                for (int i = 0; i < lanes * K; ++i) s_run[s_pe[r0 * K + i]] += 1;
            __syncwarp();
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nt * K; i += blockDim.x) {
        const int row = s_rows[i];
        pair_row[static_cast<int64_t>(t0) * K + i] = row;
        row_token[row] = t0 + i / K;
    }
    // dispatch: one warp per token
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = H / 16;
    for (int tl = warp; tl < nt; tl += 8) {
        const int t = t0 + tl;
        const uint16_t* xr = x + static_cast<int64_t>(t) * H;
        if (bf16_mode) {
            for (int p = 0; p < K; ++p) {
                const int row = s_rows[tl * K + p];
                const uint4* src = reinterpret_cast<const uint4*>(xr);
                uint4* dst = reinterpret_cast<uint4*>(a_bf16 + static_cast<int64_t>(row) * H);
                for (int v = lane; v < H / 8; v += 32) dst[v] = src[v];
            }
            continue;
        }
        // each lane quantises 4 consecutive groups (64 elements) per pass;
        // one quantisation serves every pick whose expert shares the scale
        for (int g0 = lane * 4; g0 < groups; g0 += 128) {
            float v[4][16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4* src = reinterpret_cast<const uint4*>(xr + (g0 + j) * 16);
                const uint4 q0 = src[0], q1 = src[1];
                const uint32_t u[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[j][2 * i] = __uint_as_float((u[i] & 0xffffu) << 16);
                    v[j][2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
                }
            }
            float cur_gs = 0.f;
            bool have = false;
            uint32_t codes[4][2];
            uint32_t sfw = 0u;
            for (int p = 0; p < K; ++p) {
                const int e = s_pe[tl * K + p];
                const int row = s_rows[tl * K + p];
                const float gs = gscale[e];
                if (!have || gs != cur_gs) {
                    sfw = 0u;
#pragma unroll
                    for (int j = 0; j < 4; ++j) sfw |= quantize_group16(v[j], gs, codes[j]) << (8 * j);
                    cur_gs = gs;
                    have = true;
                }
                uint4* dst = reinterpret_cast<uint4*>(a_codes + static_cast<int64_t>(row) * (H / 2) + g0 * 8);
                dst[0] = make_uint4(codes[0][0], codes[0][1], codes[1][0], codes[1][1]);
                dst[1] = make_uint4(codes[2][0], codes[2][1], codes[3][0], codes[3][1]);
                *reinterpret_cast<uint32_t*>(a_sf + sf_atom_offset(row, g0, groups)) = sfw;
            }
        }
    }
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
        const uint32_t sc = quantize_group16(v, gscale, c);
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
cudaError_t launch_router(const uint16_t* x, const uint16_t* w, const float* bias, int T, int H, int E, int K,
                          float scaling, int normalize, int n_group, int topk_group, float* logits, int32_t* idx,
                          float* wts, cudaStream_t st) {
    const size_t smem = static_cast<size_t>(kRouterTok) * H * sizeof(uint16_t);
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(200 * 1024));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    router_logits_kernel<<<(T + kRouterTok - 1) / kRouterTok, 256, smem, st>>>(x, w, T, H, E, logits);
    router_select_kernel<<<(T + kSelectWarps - 1) / kSelectWarps, kSelectWarps * 32,
                           kSelectWarps * 2 * E * sizeof(float), st>>>(logits, bias, T, E, K, scaling, normalize,
                                                                      n_group, topk_group, idx, wts);
    return cudaGetLastError();
}

cudaError_t launch_permute(const int32_t* idx, const uint16_t* x, int T, int K, int E, int H, int nb_gu, int nb_down,
                           const float* gscale, int bf16_mode, PermuteBuffers& b, cudaStream_t st) {
    const int nchunks = (T + kChunkTok - 1) / kChunkTok;
    permute_hist_kernel<<<nchunks, 256, E * sizeof(int32_t), st>>>(idx, T, K, E, b.chunk_counts);
    permute_scan_kernel<<<1, 1024, (3 * E + 2) * sizeof(int32_t), st>>>(b.chunk_counts, nchunks, E, nb_gu, nb_down,
                                                                       b.chunk_base, b.counts, b.seg_off, b.row_token,
                                                                       b.tiles_gu, b.tiles_down, b.meta);
    const size_t smem = (E + 2 * kChunkTok * K) * sizeof(int32_t);
    permute_scatter_kernel<<<nchunks, 256, smem, st>>>(idx, x, T, K, E, H, b.chunk_base, b.seg_off, gscale,
                                                       bf16_mode, b.pair_row, b.row_token, b.a_codes, b.a_sf,
                                                       b.a_bf16);
    return cudaGetLastError();
}

cudaError_t launch_combine(const void* down, bool down_bf16, const int32_t* pair_row, const float* topk_w,
                           const float* shared, const float* residual, int T, int K, int H, float* y,
                           cudaStream_t st) {
    const int threads = min(256, H / 8);
    if (down_bf16)
        combine_kernel<uint16_t><<<T, threads, 0, st>>>(static_cast<const uint16_t*>(down), pair_row, topk_w, shared,
                                                        residual, T, K, H, y);
    else
        combine_kernel<float><<<T, threads, 0, st>>>(static_cast<const float*>(down), pair_row, topk_w, shared,
                                                     residual, T, K, H, y);
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

}  // namespace nf
