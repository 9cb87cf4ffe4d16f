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
constexpr int kAttnWarps = 4;        // consumer warps (8 keys of every stage each)
constexpr int kAttnThreads = 32 * (kAttnWarps + 1);
constexpr int kRowBytes = kHd * 2;   // one BF16 key or value row
constexpr int kStageBytes = 2 * kAttnTile * kRowBytes;  // K tile + V tile
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
// producer (bulk copies of 32-key K and V tiles into a 4-stage ring), warps
// 0..3 consume 8 keys of every stage each.  In a consumer warp lane
// (h = lane / 4, quarter = lane % 4) owns q head g*G + h's dims
// [32 quarter, 32 quarter + 32): a key's score is 32 FMAs per lane plus two
// shuffles, its value row 32 FMAs -- every byte of K and V feeds all G = 8
// query heads of the KV head.  Softmax runs online per 8-key tile (max,
// rescale, exp).  The four warps' partial (max, sum, acc) merge in shared
// memory; with one split the CTA writes the output, else its partial
// goes to part_* and attn_combine_kernel merges the splits.
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(kAttnThreads) gqa_decode_kernel(const float* __restrict__ q,
                                                                  const uint16_t* __restrict__ kc,
                                                                  const uint16_t* __restrict__ vc,
                                                                  const int32_t* __restrict__ pos, int nkv, int L_max,
                                                                  int chunk, float scale, uint16_t* __restrict__ out,
                                                                  AttnPart* __restrict__ part_ml,
                                                                  float* __restrict__ part_acc, int* __restrict__ err) {
    static_assert(G == 8, "lane layout: 8 heads x 4 quarters");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* stages = smem;  // [kAttnStages][K tile | V tile]
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
    const int64_t cache_base = (static_cast<int64_t>(seq) * nkv + g) * L_max;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAttnWarps);
        }
        s_abort = 0;
        fence_barrier_init();
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
                const int kk = k0 + i * kAttnTile;
                const int n = min(kAttnTile, k1 - kk);
                const uint32_t bytes = static_cast<uint32_t>(n) * kRowBytes;
                mbar_arrive_expect_tx(&full[s], 2 * bytes);
                uint8_t* st = stages + s * kStageBytes;
                bulk_load(st, kc + (cache_base + kk) * kHd, bytes, &full[s]);
                bulk_load(st + kAttnTile * kRowBytes, vc + (cache_base + kk) * kHd, bytes, &full[s]);
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
    float acc[32];
    float m = -INFINITY, l = 0.f;
    const int h = lane >> 2, qtr = lane & 3;
    if (warp < kAttnWarps) {
        // ------------------------- consumers -------------------------
        const int head = g * G + h;
        // qv and acc hold the quarter's 32 dims in the rotated piece order the
        // reads below use: element 8c + e is dim 32 qtr + 8 ((c + qtr) % 4) + e,
        // so every register index is a compile-time constant
        float qv[32];
        const float* qsrc = q + (static_cast<int64_t>(seq) * nq + head) * kHd + 32 * qtr;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 8; ++e) qv[8 * c + e] = qsrc[8 * ((c + qtr) & 3) + e];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.f;
        for (int i = 0; i < ntiles; ++i) {
            const int s = i % kAttnStages;
            const uint32_t ph = (i / kAttnStages) & 1u;
            if (!mbar_wait(&full[s], ph, abort_flag, err)) {
                *abort_flag = 1;
                atomicCAS(err, 0, NF_DEVERR_WAIT_FULL);
                break;
            }
            const uint8_t* kt = stages + s * kStageBytes;
            const uint8_t* vt = kt + kAttnTile * kRowBytes;
            const int kk = k0 + i * kAttnTile;
            const int nvalid = min(kAttnTile, k1 - kk);
            float sc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int key = warp * 8 + j;
                float d = 0.f;
                if (key < nvalid) {
                    const uint8_t* row = kt + key * kRowBytes + qtr * 64;
                    // 16-byte pieces in a rotated order: the 4 quarters of a
                    // row then read 4 different bank groups at each step
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int pc = (c + qtr) & 3;
                        const uint4 kw = *reinterpret_cast<const uint4*>(row + pc * 16);
                        const uint32_t w4[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            d = __fmaf_rn(qv[c * 8 + 2 * u], __uint_as_float(w4[u] << 16), d);
                            d = __fmaf_rn(qv[c * 8 + 2 * u + 1], __uint_as_float(w4[u] & 0xffff0000u), d);
                        }
                    }
                }
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                sc[j] = key < nvalid ? d * scale : -INFINITY;
            }
            float tm = m;
#pragma unroll
            for (int j = 0; j < 8; ++j) tm = fmaxf(tm, sc[j]);
            if (tm != -INFINITY) {
                const float corr = __expf(m - tm);  // m = -inf on the first tile: 0
                l *= corr;
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] *= corr;
                m = tm;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int key = warp * 8 + j;
                    if (key >= nvalid) continue;
                    const float p = __expf(sc[j] - m);
                    l += p;
                    const uint8_t* row = vt + key * kRowBytes + qtr * 64;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int pc = (c + qtr) & 3;
                        const uint4 vw = *reinterpret_cast<const uint4*>(row + pc * 16);
                        const uint32_t w4[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc[c * 8 + 2 * u] = __fmaf_rn(p, __uint_as_float(w4[u] << 16), acc[c * 8 + 2 * u]);
                            acc[c * 8 + 2 * u + 1] =
                                __fmaf_rn(p, __uint_as_float(w4[u] & 0xffff0000u), acc[c * 8 + 2 * u + 1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();  // every tile consumed: the ring is free for the partials
    if (warp < kAttnWarps) {
        float* sa = s_acc + (warp * G + h) * kHd + 32 * qtr;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 8; ++e) sa[8 * ((c + qtr) & 3) + e] = acc[8 * c + e];
        if (qtr == 0) {
            s_ml[(warp * G + h) * 2] = m;
            s_ml[(warp * G + h) * 2 + 1] = l;
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

size_t attn_smem_bytes() { return 128 + static_cast<size_t>(kAttnStages) * kStageBytes + 2 * kAttnStages * 8; }

cudaError_t launch_gqa_decode(const float* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int T,
                              int nq, int nkv, int L_max, int splits, AttnPart* part_ml, float* part_acc,
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
    gqa_decode_kernel<8><<<dim3(T * nkv, splits), kAttnThreads, smem, st>>>(q, kc, vc, pos, nkv, L_max, chunk, scale, out,
                                                                          part_ml, part_acc, err);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && splits > 1) {
        const int pairs = T * nq;
        attn_combine_kernel<<<(pairs + 3) / 4, 128, 0, st>>>(part_ml, part_acc, pairs, splits, out);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace nf
