// nf_attn.cu -- the attention side of a decoder layer for the synthetic
// decoder stack (nf_stack.cu): embedding gather, RMSNorm, per-head q/k
// RMSNorm + RoPE with the KV-cache append, and GQA decode attention.
//
// The reference has no GQA attention for the target model; its closest CPU
// path is the DFlash draft's attention, draft_attention
// (src/text_forward.cpp:1216-1289): q/k/v projections, per-head RMSNorm of q
// and k (eps 1e-5, weights q_norm / k_norm), RoPE with theta 10000 on the
// two halves of each head (rope_heads :1169-1184), scores q.k * 1/sqrt(dim),
// softmax with the running max subtracted, and the weighted sum of v.  These
// kernels follow that math for one new token per sequence against a cache
// of earlier keys and values; rmsnorm / rmsnorm_stash follow :258-276 and
// the embedding row embed_row :753-757.
//
// Layouts: q F32 [T][nq][D]; the caches BF16 [seq][nkv][L_max][D] (K and V
// apart), so that one sequence's keys of one KV head are contiguous and a
// tile of them is one bulk copy; D = 128.
#include "nf_common.cuh"
#include "nf_internal.h"

#include <algorithm>

namespace nf {

namespace {

constexpr int kHd = 128;            // head dimension
constexpr int kAttnTile = 32;        // keys per pipeline stage
constexpr int kAttnStages = 4;
constexpr int kAttnWarps = 2;        // consumer warps (16 keys of every stage each)
constexpr int kAttnThreads = 32 * (kAttnWarps + 1);
constexpr int kBoxBytes = kAttnTile * 128;  // one TMA box: 32 keys x 64 dims (128-byte rows, swizzled)
constexpr int kStageBytes = 4 * kBoxBytes;  // K dims 0-63 | K 64-127 | V 0-63 | V 64-127
constexpr int kAttnMaxSplits = kAttnMaxSplitsHost;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace

// ---------------------------------------------------------------------------
// Embedding rows (embed_row, src/text_forward.cpp:753-757): x[t] = embed[tok[t]]
// widened to F32.  A token outside the vocabulary (the reference fails with
// "prompt token is outside the vocabulary", :626) records an error and
// writes a NaN row.
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const uint16_t* __restrict__ table, int64_t vocab, int H, const int32_t* __restrict__ tok,
                             float* __restrict__ x, int* __restrict__ err) {
    const int t = blockIdx.x;
    const int32_t id = tok[t];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && threadIdx.x == 0) atomicCAS(err, 0, NF_DEVERR_BAD_TOKEN);
    const uint16_t* row = table + (ok ? static_cast<int64_t>(id) : 0) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        x[static_cast<int64_t>(t) * H + i] = ok ? bf16_bits_to_f32(row[i]) : __int_as_float(0x7fc00000);
}

// ---------------------------------------------------------------------------
// RMSNorm of one row per CTA (rmsnorm :258-263, rmsnorm_stash :267-276):
//   h = a (+ the sum of b's S slices, slice s at b + s * b_stride, when b !=
//   NULL: a split-K projection's partials; h_out receives h),
//   inv = 1 / sqrt(sum(h^2)/n + eps)
//   stash = 0: y = h * inv * w;      stash = 1: y = bf16(bf16(h) * inv * w)
// y goes to y_bf16 (rounded) and/or y_f32.  The sum of squares is a tree
// sum (the reference adds sequentially): the norm agrees within rounding.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float slice_sum(const float* __restrict__ b, int S, int64_t stride, int64_t i) {
    float v = b[i];
    for (int s = 1; s < S; ++s) v = __fadd_rn(v, b[s * stride + i]);
    return v;
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ a, const float* __restrict__ b, int S,
                                                      int64_t b_stride, float* __restrict__ h_out,
                                                      const float* __restrict__ w, int n, float eps, int stash,
                                                      uint16_t* __restrict__ y_bf16, float* __restrict__ y_f32) {
    __shared__ float s_part[8];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = a[base + i];
        if (b) v = __fadd_rn(v, slice_sum(b, S, b_stride, base + i));
        if (h_out) h_out[base + i] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += s_part[i];
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(n)), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = h_out ? h_out[base + i] : a[base + i];
        if (b && !h_out) v = __fadd_rn(v, slice_sum(b, S, b_stride, base + i));
        if (stash) v = bf16_round(v);
        const float y = __fmul_rn(__fmul_rn(v, inv), w ? w[i] : 1.f);
        if (y_bf16) y_bf16[base + i] = f32_to_bf16_bits(y);
        if (y_f32) y_f32[base + i] = stash ? bf16_round(y) : y;
    }
}

// ---------------------------------------------------------------------------
// q/k RMSNorm + RoPE + cache append.  qkv F32 [T][(nq + 2 nkv) D] from the
// fused projection (the sum of S split-K slices, slice s at qkv + s * stride); one warp per (token, head); lane l holds dims l, l+32,
// l+64, l+96, so both halves of RoPE's pairs (i, i + D/2) are in one lane.
// q heads -> q F32; k heads -> K cache, v heads -> V cache (BF16) at the
// token's position.  rope_heads (:1169-1184): freq_i = theta^(-2i/D),
// angle = pos * freq_i, (x_i, x_{i+D/2}) rotated by angle.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(const float* __restrict__ qkv, int S, int64_t stride,
                                                           int T, int nq, int nkv,
                                                           const float* __restrict__ q_norm,
                                                           const float* __restrict__ k_norm, float eps, float theta,
                                                           const int32_t* __restrict__ pos, int L_max,
                                                           float* __restrict__ q_out, uint16_t* __restrict__ kc,
                                                           uint16_t* __restrict__ vc, int* __restrict__ err) {
    const int heads = nq + 2 * nkv;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= T * heads) return;
    const int lane = threadIdx.x & 31;
    const int t = gw / heads, hh = gw % heads;
    const int64_t src = static_cast<int64_t>(t) * heads * kHd + static_cast<int64_t>(hh) * kHd;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = slice_sum(qkv, S, stride, src + lane + 32 * j);
    const int p = pos[t];
    if (p < 0 || p >= L_max) {
        if (lane == 0) atomicCAS(err, 0, NF_DEVERR_BAD_TOKEN);
        return;
    }
    const bool is_q = hh < nq, is_k = !is_q && hh < nq + nkv;
    if (is_q || is_k) {
        const float* nw = is_q ? q_norm : k_norm;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss = __fmaf_rn(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(kHd)), eps)));
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], inv), nw ? nw[lane + 32 * j] : 1.f);
        // rotate pairs (i, i + 64) for i = lane and lane + 32
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = lane + 32 * j;
            const float freq = powf(theta, __fdiv_rn(-2.f * static_cast<float>(i), static_cast<float>(kHd)));
            const float ang = __fmul_rn(static_cast<float>(p), freq);
            const float c = cosf(ang), s = sinf(ang);
            const float first = v[j], second = v[j + 2];
            v[j] = __fsub_rn(__fmul_rn(first, c), __fmul_rn(second, s));
            v[j + 2] = __fadd_rn(__fmul_rn(first, s), __fmul_rn(second, c));
        }
    }
    if (is_q) {
        float* dst = q_out + (static_cast<int64_t>(t) * nq + hh) * kHd;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = v[j];
    } else {
        const int g = is_k ? hh - nq : hh - nq - nkv;
        uint16_t* dst = (is_k ? kc : vc) + ((static_cast<int64_t>(t) * nkv + g) * L_max + p) * kHd;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = f32_to_bf16_bits(v[j]);
    }
}

// ---------------------------------------------------------------------------
// GQA decode attention, flash-decoding split over the context.
// grid (T * nkv, splits), kAttnThreads threads: warp kAttnWarps is the
// producer (TMA tiles of 32 keys x 64 dims, 128-byte swizzled, two per K
// tile and two per V tile, into a 4-stage ring), warps 0..1 consume 16 keys
// of every stage each.  The two contractions run on the tensor cores as
// warp-level MMAs (m16n8k16, BF16 in, F32 accumulate): S = Q K^T with the G
// = 8 query heads of the KV head as rows (rows 8-15 zero) and 8 keys per
// n-tile, then O += P V with P from S's accumulator fragments.  The kernel
// is bound by the cache's HBM bytes (8 flops per byte), so the MMAs only
// remove the ~200 scalar instructions a key cost on the CUDA cores; the
// swizzled tiles make every ldmatrix conflict-free.  Softmax runs online per
// 16-key chunk (max over the chunk, rescale, exp).  The warps' partial (max,
// sum, acc) merge in shared memory; with one split the CTA writes the
// output, else its partial goes to part_* and attn_combine_kernel merges the
// splits.  q is rounded to BF16 for the MMA, P too (as flash attention
// does); scores and sums stay F32.
// ---------------------------------------------------------------------------
// shared-memory address of 16-byte chunk `c` (0..7) of row `r` in a 128-byte
// swizzled box (the box base is 1024-byte aligned)
__device__ __forceinline__ uint32_t sw128(uint32_t box, int r, int c) {
    return box + static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kAttnThreads) gqa_decode_kernel(const __grid_constant__ CUtensorMap tmk,
                                                                  const __grid_constant__ CUtensorMap tmv,
                                                                  const float* __restrict__ q,
                                                                  const int32_t* __restrict__ pos, int nkv, int L_max,
                                                                  int chunk, float scale, uint16_t* __restrict__ out,
                                                                  AttnPart* __restrict__ part_ml,
                                                                  float* __restrict__ part_acc, int* __restrict__ err) {
    static_assert(G == 8, "the 8 query heads of a KV head are the MMA's rows 0-7");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stages = smem;  // [kAttnStages][K dims 0-63 | K dims 64-127 | V dims 0-63 | V dims 64-127]
    // the warps' partials reuse the stage ring once every tile is consumed
    float* s_acc = reinterpret_cast<float*>(stages);                      // [kAttnWarps][G][kHd]
    float* s_ml = s_acc + kAttnWarps * G * kHd;                           // [kAttnWarps][G][2]
    static_assert(kAttnWarps * G * (kHd + 2) * 4 <= kAttnStages * kStageBytes, "partials fit in the ring");
    uint64_t* full = reinterpret_cast<uint64_t*>(stages + kAttnStages * kStageBytes);
    uint64_t* empty = full + kAttnStages;
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = blockIdx.x / nkv, g = blockIdx.x % nkv;
    const int nq = nkv * G;
    const int len = pos[seq] + 1;  // keys 0 .. pos (the new token's key included)
    const int k0 = blockIdx.y * chunk;
    const int k1 = min(len, k0 + chunk);
    const int ntiles = k1 > k0 ? (k1 - k0 + kAttnTile - 1) / kAttnTile : 0;
    const int cache_row = (seq * nkv + g) * L_max;  // tensor-map row of key 0

    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAttnWarps);
        }
        s_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmk);
        prefetch_tensormap(&tmv);
    }
    __syncthreads();
    volatile int* abort_flag = &s_abort;

    if (warp == kAttnWarps) {
        // ------------------------- producer -------------------------
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % kAttnStages;
                const uint32_t ph = (i / kAttnStages) & 1u;
                if (i >= kAttnStages && !mbar_wait(&empty[s], ph ^ 1u, abort_flag, err)) {
                    *abort_flag = 1;
                    atomicCAS(err, 0, NF_DEVERR_WAIT_EMPTY);
                    break;
                }
                const int y = cache_row + k0 + i * kAttnTile;
                uint8_t* st = stages + s * kStageBytes;
                mbar_arrive_expect_tx(&full[s], kStageBytes);  // whole boxes (zero-filled past the tensor)
                tma_load_2d(st, &tmk, &full[s], 0, y);
                tma_load_2d(st + kBoxBytes, &tmk, &full[s], 64, y);
                tma_load_2d(st + 2 * kBoxBytes, &tmv, &full[s], 0, y);
                tma_load_2d(st + 3 * kBoxBytes, &tmv, &full[s], 64, y);
                issued = i + 1;
            }
            if (*abort_flag) {
                // drain: the copies of the last tiles issued land before the CTA moves on
                for (int i = max(0, issued - kAttnStages); i < issued; ++i) {
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(&full[i % kAttnStages], (i / kAttnStages) & 1u))
                        if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) break;
                }
            }
        }
    }
    const int grp = lane >> 2, t4 = lane & 3;  // MMA fragment coordinates: row group, thread in group
    float o[16][4];                            // O fragments: head grp (c0, c1) x dims 8 n + 2 t4 (+1)
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m = -INFINITY, l = 0.f;  // head grp's running max and (this lane's part of the) sum
    if (warp < kAttnWarps) {
        // ------------------------- consumers -------------------------
        // Q fragments (rows 8-15 of the MMA are zero): k-step s holds dims 16 s + 2 t4 (+1) and + 8
        uint32_t qa[8][2];
        const float* qrow = q + (static_cast<int64_t>(seq) * nq + g * G + grp) * kHd;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            qa[s][0] = pack_bf16x2(qrow[16 * s + 2 * t4], qrow[16 * s + 2 * t4 + 1]);
            qa[s][1] = pack_bf16x2(qrow[16 * s + 2 * t4 + 8], qrow[16 * s + 2 * t4 + 9]);
        }
        const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: this lane's matrix and row
        for (int i = 0; i < ntiles; ++i) {
            const int s = i % kAttnStages;
            const uint32_t ph = (i / kAttnStages) & 1u;
            if (!mbar_wait(&full[s], ph, abort_flag, err)) {
                *abort_flag = 1;
                atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
                break;
            }
            const uint32_t st = smem_u32(stages + s * kStageBytes);
            const int kk = k0 + i * kAttnTile;
            const int nv = min(16, max(0, min(kAttnTile, k1 - kk) - 16 * warp));  // valid keys of my 16
            if (nv > 0) {
                if (nv < 16) {
                    // V rows past the sequence hold whatever the cache holds there: zero
                    // them, so their zero weights cannot meet a NaN in the MMA
                    for (int r = 16 * warp + nv + (lane >> 3); r < 16 * warp + 16; r += 4)
                        for (int b = 0; b < 2; ++b)
                            *reinterpret_cast<uint4*>(stages + s * kStageBytes + (2 + b) * kBoxBytes + r * 128 +
                                                      (lane & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
                    __syncwarp();
                }
                // S = Q K^T: n-tile j holds keys 16 warp + 8 j .. + 7
                float sc[2][4];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
                    const int key = 16 * warp + 8 * j + mr;
#pragma unroll
                    for (int s2 = 0; s2 < 8; s2 += 2) {
                        // matrices: dims 16 s2 + 8 (mi & 1) of k-step s2 + (mi >> 1)
                        const int dc = 16 * (s2 + (mi >> 1)) + 8 * (mi & 1);
                        uint32_t b[4];
                        ldsm_x4(sw128(st + (dc >> 6) * kBoxBytes, key, (dc & 63) >> 3), b);
                        mma_16816(sc[j], qa[s2][0], 0u, qa[s2][1], 0u, b[0], b[1]);
                        mma_16816(sc[j], qa[s2 + 1][0], 0u, qa[s2 + 1][1], 0u, b[2], b[3]);
                    }
                }
                // online softmax over this chunk for head grp (rows 8-15, c2 / c3, are padding)
                float v[4];
                v[0] = (8 * 0 + 2 * t4 < nv) ? sc[0][0] * scale : -INFINITY;
                v[1] = (8 * 0 + 2 * t4 + 1 < nv) ? sc[0][1] * scale : -INFINITY;
                v[2] = (8 * 1 + 2 * t4 < nv) ? sc[1][0] * scale : -INFINITY;
                v[3] = (8 * 1 + 2 * t4 + 1 < nv) ? sc[1][1] * scale : -INFINITY;
                float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mn = fmaxf(m, mx);
                if (mn != -INFINITY) {
                    const float corr = __expf(m - mn);  // m = -inf on the first chunk: 0
                    float p[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) p[e] = __expf(v[e] - mn);
                    l = l * corr + ((p[0] + p[1]) + (p[2] + p[3]));
                    m = mn;
#pragma unroll
                    for (int n = 0; n < 16; ++n) {
                        o[n][0] *= corr;
                        o[n][1] *= corr;
                    }
                    // O += P V: P (row grp) = keys 2 t4 (+1) and 8 + 2 t4 (+1) of my 16
                    const uint32_t pa0 = pack_bf16x2(p[0], p[1]), pa2 = pack_bf16x2(p[2], p[3]);
                    const int key = 16 * warp + 8 * (mi & 1) + mr;
#pragma unroll
                    for (int n = 0; n < 16; n += 2) {
                        // matrices: keys 8 (mi & 1) .. + 7 of dims 8 (n + (mi >> 1)) .. + 7, transposed
                        const int dc = 8 * (n + (mi >> 1));
                        uint32_t b[4];
                        ldsm_x4_t(sw128(st + (2 + (dc >> 6)) * kBoxBytes, key, (dc & 63) >> 3), b);
                        mma_16816(o[n], pa0, 0u, pa2, 0u, b[0], b[1]);
                        mma_16816(o[n + 1], pa0, 0u, pa2, 0u, b[2], b[3]);
                    }
                }
                if (nv < 16) fence_proxy_async();  // the zeroed rows before the next TMA write into the stage
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
    }
    __syncthreads();  // every tile consumed: the ring is free for the partials
    if (warp < kAttnWarps) {
        float* sa = s_acc + (warp * G + grp) * kHd;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            sa[8 * n + 2 * t4] = o[n][0];
            sa[8 * n + 2 * t4 + 1] = o[n][1];
        }
        if (t4 == 0) {
            s_ml[(warp * G + grp) * 2] = m;
            s_ml[(warp * G + grp) * 2 + 1] = l;
        }
    }
    __syncthreads();
    // merge the consumer warps: thread i of the CTA handles (head h, dim d) pairs
    for (int i = threadIdx.x; i < G * kHd; i += blockDim.x) {
        const int hh = i / kHd, d = i % kHd;
        float mm = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, s_ml[(w * G + hh) * 2]);
        float ll = 0.f, aa = 0.f;
        if (mm != -INFINITY) {
            for (int w = 0; w < kAttnWarps; ++w) {
                const float mw = s_ml[(w * G + hh) * 2];
                if (mw == -INFINITY) continue;
                const float f = __expf(mw - mm);
                ll += s_ml[(w * G + hh) * 2 + 1] * f;
                aa += s_acc[(w * G + hh) * kHd + d] * f;
            }
        }
        const int head = g * G + hh;
        if (gridDim.y == 1) {
            out[(static_cast<int64_t>(seq) * nq + head) * kHd + d] = f32_to_bf16_bits(ll > 0.f ? aa / ll : 0.f);
        } else {
            const int64_t pi = (static_cast<int64_t>(seq) * nq + head) * gridDim.y + blockIdx.y;
            part_acc[pi * kHd + d] = aa;
            if (d == 0) part_ml[pi] = AttnPart{mm, ll};
        }
    }
}

// Merges the splits of every (token, head): one warp per pair, 4 dims a lane.
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnPart* __restrict__ part_ml,
                                                           const float* __restrict__ part_acc, int pairs, int splits,
                                                           uint16_t* __restrict__ out) {
    const int pw = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (pw >= pairs) return;
    const int lane = threadIdx.x & 31;
    const AttnPart* pm = part_ml + static_cast<int64_t>(pw) * splits;
    float mm = -INFINITY;
    for (int s = 0; s < splits; ++s) mm = fmaxf(mm, pm[s].m);
    float ll = 0.f, a[4] = {0.f, 0.f, 0.f, 0.f};
    if (mm != -INFINITY) {
        for (int s = 0; s < splits; ++s) {
            if (pm[s].m == -INFINITY) continue;
            const float f = __expf(pm[s].m - mm);
            ll += pm[s].l * f;
            const float* pa = part_acc + (static_cast<int64_t>(pw) * splits + s) * kHd;
#pragma unroll
            for (int j = 0; j < 4; ++j) a[j] += pa[lane + 32 * j] * f;
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        out[static_cast<int64_t>(pw) * kHd + lane + 32 * j] = f32_to_bf16_bits(ll > 0.f ? a[j] / ll : 0.f);
}

// Deterministic pseudo-random BF16 values in (-1, 1) from a 64-bit hash of
// (seed, index): a stand-in history for a cache, filled on the device.
__global__ void fill_bf16_hash_kernel(uint16_t* __restrict__ p, int64_t n, uint64_t seed) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        uint64_t z = seed + 0x9e3779b97f4a7c15ull * static_cast<uint64_t>(i + 1);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        z ^= z >> 31;
        const float u = static_cast<float>(static_cast<uint32_t>(z >> 40)) * (1.f / 16777216.f);  // [0, 1)
        p[i] = f32_to_bf16_bits(2.f * u - 1.f);
    }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_fill_bf16_hash(uint16_t* p, int64_t n, uint64_t seed, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fill_bf16_hash_kernel<<<2048, 256, 0, st>>>(p, n, seed);
    return cudaGetLastError();
}

cudaError_t launch_embed(const uint16_t* table, int64_t vocab, int H, const int32_t* tok, int T, float* x, int* err,
                         cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    embed_kernel<<<T, 256, 0, st>>>(table, vocab, H, tok, x, err);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* a, const float* b, int b_slices, int64_t b_stride, float* h_out, const float* w,
                           int rows, int n, float eps, int stash, uint16_t* y_bf16, float* y_f32, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    rmsnorm_kernel<<<rows, 256, 0, st>>>(a, b, std::max(1, b_slices), b_stride, h_out, w, n, eps, stash, y_bf16, y_f32);
    return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const float* qkv, int slices, int64_t stride, int T, int nq, int nkv,
                                const float* q_norm, const float* k_norm, float eps, float theta, const int32_t* pos,
                                int L_max, float* q_out, uint16_t* kc, uint16_t* vc, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int warps = T * (nq + 2 * nkv);
    qk_norm_rope_kernel<<<(warps + 3) / 4, 128, 0, st>>>(qkv, std::max(1, slices), stride, T, nq, nkv, q_norm, k_norm,
                                                         eps, theta, pos, L_max, q_out, kc, vc, err);
    return cudaGetLastError();
}

int attn_splits(int T, int nkv, int L_max, int sms) {
    const int pairs = std::max(1, T * nkv);
    const int want = (2 * sms + pairs - 1) / pairs;
    const int max_splits = std::max(1, (L_max + kAttnTile - 1) / kAttnTile);
    return std::max(1, std::min(want, std::min(max_splits, kAttnMaxSplits)));
}

size_t attn_smem_bytes() { return 1024 + static_cast<size_t>(kAttnStages) * kStageBytes + 2 * kAttnStages * 8; }

cudaError_t launch_gqa_decode(const CUtensorMap& tmk, const CUtensorMap& tmv, const float* q, const int32_t* pos,
                              int T, int nq, int nkv, int L_max, int splits, AttnPart* part_ml, float* part_acc,
                              uint16_t* out, int* err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (nq != 8 * nkv) return cudaErrorInvalidValue;
    // the context is cut into `splits` chunks of whole 32-key tiles
    const int chunk = ((L_max + splits - 1) / splits + kAttnTile - 1) / kAttnTile * kAttnTile;
    const size_t smem = attn_smem_bytes();
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(gqa_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const float scale = 1.f / sqrtf(static_cast<float>(kHd));
    gqa_decode_kernel<8><<<dim3(T * nkv, splits), kAttnThreads, smem, st>>>(tmk, tmv, q, pos, nkv, L_max, chunk, scale,
                                                                          out, part_ml, part_acc, err);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && splits > 1) {
        const int pairs = T * nq;
        attn_combine_kernel<<<(pairs + 3) / 4, 128, 0, st>>>(part_ml, part_acc, pairs, splits, out);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace nf
