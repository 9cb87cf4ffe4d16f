// nf_stack.cu -- a decoder stack for greedy decode (nf_stack_* in
// include/nf_moe.h): the benchmark's synthetic full model around the MoE
// layer.  The reference's token step is TextModel::step + argmax
// (src/text_forward.cpp:625-698): embed the token (:627-634), run every layer
// (mixer, then feed() :892-907 with the dense MLP :909-915 or the MoE
// :924-963), apply the final norm (:652-654) and take the greedy token over
// the lm_head logits (:656-698).
//
// One decode step here, for a batch of sequences each at its own position:
//   x = embed[token]                                      (embed_row :753)
//   per layer l:
//     a   = bf16(rmsnorm(x; input_layernorm))             (rmsnorm :258)
//     qkv = a . [Wq; Wk; Wv]^T                             tcgen05 BF16 GEMM, split K
//     q, k = per-head rmsnorm + RoPE; k, v appended to the layer's KV cache
//     o   = attention(q, cache) . Wo^T                     GQA decode + GEMM
//     h   = x + o;  f = rmsnorm_stash(h; post_attention_layernorm)  (:267)
//     x   = h + ffn_l(f)                                   the layer's nf_moe handle (dense
//                                                          NVFP4 MLP, NVFP4 MoE or BF16-expert
//                                                          MoE), residual fused in its combine
//   next = argmax(lm_head . rmsnorm(x; norm))              nf_tp (exact gemv_bf16 rows + argmax)
// The attention follows the DFlash draft attention's math (draft_attention
// :1216-1289, the reference's only GQA attention).  Every launch is
// asynchronous on the caller's stream, so a whole step can be captured in a
// CUDA graph.
#include "nf_moe.h"

#include "nf_common.cuh"
#include "nf_internal.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using namespace nf;

namespace {

constexpr int kHeadDim = 128;
constexpr int kMaxSlices = 16;  // split-K slices of a projection

struct StackLayer {
    nf_moe* ffn = nullptr;
    uint8_t* w_qkv = nullptr;  // box order [(nq + 2 nkv) D, H] BF16
    uint8_t* w_o = nullptr;    // box order [H, nq D] BF16
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* q_norm = nullptr;
    float* k_norm = nullptr;
    uint16_t* kc = nullptr;    // [B][nkv][L][D]
    uint16_t* vc = nullptr;
    CUtensorMap tm_qkv{}, tm_o{};
    CUtensorMap tm_kc{}, tm_vc{};  // the caches as [B nkv L, 128] tensors for the attention's TMA tiles
    uint16_t bound = 0;        // bit per NF_STACK_* tensor
};

thread_local std::string g_stack_create_error;

}  // namespace

struct nf_stack {
    nf_stack_desc d{};
    int device = 0;
    int sms = 148;
    std::vector<StackLayer> layers;
    std::vector<std::vector<uint16_t>> qkv_host;  // fused q/k/v rows while binding (freed at finalize)
    std::vector<void*> allocs;
    std::string msg;
    bool finalized = false;
    uint16_t* embed = nullptr;     // [V, H] BF16 row-major
    uint16_t* lm_head = nullptr;   // [V, H] BF16 row-major
    float* final_norm = nullptr;   // [H]
    bool embed_bound = false, head_bound = false, norm_bound = false;
    nf_tp* head = nullptr;         // lm_head: exact rows + greedy pick on this GPU
    // workspace (B = max_batch)
    float* x = nullptr;            // [B, H] residual stream
    float* h = nullptr;            // [B, H]
    uint16_t* a16 = nullptr;       // [B, H] normed layer input (BF16)
    uint16_t* f16 = nullptr;       // [B, H] normed FFN input (BF16)
    float* fin = nullptr;          // [B, H] final norm
    float* qkv_part = nullptr;     // [slices][B, (nq + 2 nkv) D]
    float* q = nullptr;            // [B, nq D]
    uint16_t* att16 = nullptr;     // [B, nq D] attention output (BF16)
    float* o_part = nullptr;       // [slices][B, H]
    AttnPart* part_ml = nullptr;   // attention split partials
    float* part_acc = nullptr;
    int* counters = nullptr;       // GEMM tile counters [2 * layers]
    int* err = nullptr;
    CUtensorMap tm_a{}, tm_a_s{}, tm_att{}, tm_att_s{};

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
        if (cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 16)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return true;
    }
};

namespace {

int qkv_rows(const nf_stack_desc& d) { return (d.q_heads + 2 * d.kv_heads) * kHeadDim; }

void stack_release(nf_stack* s) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    for (auto& L : s->layers)
        if (L.ffn) nf_moe_destroy(L.ffn);
    if (s->head) nf_tp_destroy(s->head);
    for (void* p : s->allocs) cudaFree(p);
    cudaSetDevice(prev);
    delete s;
}

// Split-K slices for a dense BF16 projection of T rows x N outputs over K:
// enough (m, n, k) tiles for every SM while the N / 256 output blocks of a
// decode batch alone would leave most SMs idle.
int proj_slices(int T, int N, int K, int sms, int* kt_per) {
    const int m_tiles = (T + 127) / 128, n_blocks = N / 256, k_tiles = (K + 63) / 64;
    const int base = m_tiles * n_blocks;
    int want = std::max(1, std::min(kMaxSlices, sms / std::max(1, base)));
    *kt_per = std::max(2, (k_tiles + want - 1) / want);
    return (k_tiles + *kt_per - 1) / *kt_per;
}

cudaError_t launch_projection(nf_stack* s, const CUtensorMap& tma, const CUtensorMap& tma_s, const CUtensorMap& tmb,
                              const uint8_t* w, int T, int N, int K, float* part, int* counter, int* slices,
                              cudaStream_t st) {
    int kt_per = 0;
    const int S = proj_slices(T, N, K, s->sms, &kt_per);
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    GemmArgs g{};
    g.err = s->err;
    g.kind = KIND_BF16;
    g.epi = EPI_STORE_F32;
    g.K = K;
    g.dense_rows = T;
    g.n_blocks = N / 256;
    g.b_nb = N / 256;
    g.b = w;
    g.b_kt = static_cast<int>(box_k_blocks(2 * static_cast<int64_t>(K)));
    g.k_split = S;
    g.kt_per = kt_per;
    g.out = part;
    g.out_ld = N;
    g.out_split_stride = static_cast<int64_t>(T) * N;
    g.tile_counter = counter;
    g.early_claim = 1;  // the counter was zeroed above, in stream order
    const int tiles = ((T + 127) / 128) * (N / 256) * S;
    *slices = S;
    return launch_gemm(tma, tma_s, tmb, g, std::min(s->sms, tiles), false, st);
}

}  // namespace

extern "C" {

int nf_stack_create(const nf_stack_desc* desc, int device, nf_stack** out) {
    std::string& err = g_stack_create_error;
    err.clear();
    if (!desc || !out) {
        err = "null descriptor or output";
        return NF_ERR_INVALID;
    }
    *out = nullptr;
    const nf_stack_desc& d = *desc;
    if (d.vocab < 1 || d.hidden < 256 || d.hidden % 256 != 0 || d.layers < 1 || d.dense_layers < 0 ||
        d.bf16_expert_layers < 0 || d.dense_layers + d.bf16_expert_layers > d.layers) {
        err = "stack shape: vocab >= 1, hidden a multiple of 256, layers >= dense + BF16-expert layers";
        return NF_ERR_SHAPE;
    }
    if (d.head_dim != kHeadDim || d.kv_heads < 1 || d.q_heads != 8 * d.kv_heads || qkv_rows(d) % 256 != 0 ||
        (d.q_heads * kHeadDim) % 256 != 0) {
        err = "attention: head_dim 128, q_heads = 8 x kv_heads, (q_heads + 2 kv_heads) x 128 a multiple of 256";
        return NF_ERR_UNSUPPORTED;
    }
    if (d.max_batch < 1 || d.max_batch > 4096 || d.max_context < 1 || d.max_context > (1 << 20)) {
        err = "max_batch in [1, 4096] and max_context in [1, 2^20]";
        return NF_ERR_INVALID;
    }
    if (d.dense_layers > 0 && (d.dense_inter < 128 || d.dense_inter % 128 != 0)) {
        err = "dense_inter must be a positive multiple of 128";
        return NF_ERR_SHAPE;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        err = "cannot use the requested device";
        return NF_ERR_CUDA;
    }
    nf_stack* s = new nf_stack();
    s->d = d;
    s->device = device;
    s->sms = gemm_grid_size(device);
    s->layers.resize(static_cast<size_t>(d.layers));
    s->qkv_host.resize(static_cast<size_t>(d.layers));
    const int64_t B = d.max_batch, H = d.hidden, L = d.max_context, nkv = d.kv_heads;
    const int64_t NQKV = qkv_rows(d), NQ = static_cast<int64_t>(d.q_heads) * kHeadDim;
    int st = NF_OK;
    // the FFN of every layer: dense NVFP4 MLP, NVFP4 MoE, or BF16-expert MoE
    for (int l = 0; l < d.layers && st == NF_OK; ++l) {
        nf_moe* f = nullptr;
        if (l < d.dense_layers) {
            st = nf_moe_create_dense(d.hidden, d.dense_inter, d.moe.swiglu_limit, d.max_batch, device, &f);
        } else {
            nf_moe_desc md = d.moe;
            md.hidden = d.hidden;
            md.max_tokens = d.max_batch;
            md.expert_kind = l >= d.layers - d.bf16_expert_layers ? NF_EXPERTS_BF16 : NF_EXPERTS_NVFP4;
            st = nf_moe_create(&md, device, &f);
        }
        if (st != NF_OK) err = std::string("layer ") + std::to_string(l) + " FFN: " + nf_moe_last_error(nullptr);
        s->layers[static_cast<size_t>(l)].ffn = f;
    }
    bool ok = st == NF_OK;
    for (auto& Ly : s->layers) {
        if (!ok) break;
        ok = s->alloc(&Ly.w_qkv, static_cast<size_t>(box_order_bytes(NQKV, 2 * H))) &&
             s->alloc(&Ly.w_o, static_cast<size_t>(box_order_bytes(H, 2 * NQ))) && s->alloc(&Ly.attn_norm, H) &&
             s->alloc(&Ly.ffn_norm, H) && s->alloc(&Ly.q_norm, kHeadDim) && s->alloc(&Ly.k_norm, kHeadDim) &&
             s->alloc(&Ly.kc, static_cast<size_t>(B * nkv * L * kHeadDim)) &&
             s->alloc(&Ly.vc, static_cast<size_t>(B * nkv * L * kHeadDim));
        if (ok) ok = cudaMemset(Ly.kc, 0, static_cast<size_t>(B * nkv * L * kHeadDim) * 2) == cudaSuccess &&
                     cudaMemset(Ly.vc, 0, static_cast<size_t>(B * nkv * L * kHeadDim) * 2) == cudaSuccess;
    }
    const int64_t max_splits = kAttnMaxSplitsHost;
    ok = ok && s->alloc(&s->embed, static_cast<size_t>(d.vocab) * H) &&
         s->alloc(&s->lm_head, static_cast<size_t>(d.vocab) * H) && s->alloc(&s->final_norm, H) &&
         s->alloc(&s->x, B * H) && s->alloc(&s->h, B * H) && s->alloc(&s->a16, B * H) && s->alloc(&s->f16, B * H) &&
         s->alloc(&s->fin, B * H) && s->alloc(&s->qkv_part, kMaxSlices * B * NQKV) && s->alloc(&s->q, B * NQ) &&
         s->alloc(&s->att16, B * NQ) && s->alloc(&s->o_part, kMaxSlices * B * H) &&
         s->alloc(&s->part_ml, B * d.q_heads * max_splits) &&
         s->alloc(&s->part_acc, B * d.q_heads * max_splits * kHeadDim) &&
         s->alloc(&s->counters, 2 * static_cast<size_t>(d.layers)) && s->alloc(&s->err, 1) &&
         cudaMemset(s->err, 0, 4) == cudaSuccess;
    if (ok)
        ok = make_tmap_2d(&s->tm_a, s->a16, true, H, B, 64, 128) && make_tmap_2d(&s->tm_a_s, s->a16, true, H, B, 64, 32) &&
             make_tmap_2d(&s->tm_att, s->att16, true, NQ, B, 64, 128) &&
             make_tmap_2d(&s->tm_att_s, s->att16, true, NQ, B, 64, 32);
    if (ok && st == NF_OK) {
        st = nf_tp_create(device, 0, 1, nullptr, 0, d.max_batch, d.vocab, &s->head);
        if (st != NF_OK) err = std::string("lm_head: ") + nf_tp_last_error(nullptr);
    }
    cudaSetDevice(prev);
    if (!ok && st == NF_OK) {
        st = NF_ERR_NOMEM;
        err = "device allocation failed";
    }
    if (st != NF_OK) {
        stack_release(s);
        return st;
    }
    *out = s;
    return NF_OK;
}

void nf_stack_destroy(nf_stack* s) {
    if (s) stack_release(s);
}

const char* nf_stack_last_error(const nf_stack* s) { return s ? s->msg.c_str() : g_stack_create_error.c_str(); }

nf_moe* nf_stack_layer_ffn(nf_stack* s, int layer) {
    if (!s || layer < 0 || layer >= s->d.layers) return nullptr;
    return s->layers[static_cast<size_t>(layer)].ffn;
}

int nf_stack_bind_bf16(nf_stack* s, int which, int layer, const uint16_t* data, int64_t rows, int64_t cols) {
    if (!s || !data) return NF_ERR_INVALID;
    s->msg.clear();
    const nf_stack_desc& d = s->d;
    const int64_t H = d.hidden, D = kHeadDim, nq = d.q_heads, nkv = d.kv_heads;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaError_t e = cudaSuccess;
    int st = NF_OK;
    if (which == NF_STACK_EMBED || which == NF_STACK_LM_HEAD) {
        if (rows != d.vocab || cols != H) {
            st = s->fail(NF_ERR_SHAPE, "%s layout", which == NF_STACK_EMBED ? "embed_tokens" : "lm_head");
        } else {
            uint16_t* dst = which == NF_STACK_EMBED ? s->embed : s->lm_head;
            e = cudaMemcpy(dst, data, static_cast<size_t>(rows * cols) * 2, cudaMemcpyHostToDevice);
            if (which == NF_STACK_EMBED) s->embed_bound = e == cudaSuccess;
            else s->head_bound = e == cudaSuccess;
        }
    } else if (layer < 0 || layer >= d.layers) {
        st = s->fail(NF_ERR_INVALID, "layer %d out of range", layer);
    } else {
        StackLayer& Ly = s->layers[static_cast<size_t>(layer)];
        if (which == NF_STACK_Q_PROJ || which == NF_STACK_K_PROJ || which == NF_STACK_V_PROJ) {
            const int64_t want = which == NF_STACK_Q_PROJ ? nq * D : nkv * D;
            if (rows != want || cols != H) {
                st = s->fail(NF_ERR_SHAPE, "BF16 linear layout layers.%d.self_attn.%s_proj.weight", layer,
                             which == NF_STACK_Q_PROJ ? "q" : which == NF_STACK_K_PROJ ? "k" : "v");
            } else {
                // q, k and v are rows [0, nq D), [nq D, (nq + nkv) D) and [(nq + nkv) D, (nq + 2 nkv) D)
                // of the fused projection; the host copy of the fused matrix lives until finalize
                const int64_t NQKV = qkv_rows(d);
                const int64_t off = which == NF_STACK_Q_PROJ ? 0 : which == NF_STACK_K_PROJ ? nq * D : (nq + nkv) * D;
                std::vector<uint16_t>& stg = s->qkv_host[static_cast<size_t>(layer)];
                if (stg.size() != static_cast<size_t>(NQKV * H)) stg.assign(static_cast<size_t>(NQKV * H), 0);
                std::memcpy(stg.data() + off * H, data, static_cast<size_t>(rows * cols) * 2);
                e = upload_box_order(Ly.w_qkv, reinterpret_cast<const uint8_t*>(stg.data()), NQKV, 2 * H);
                if (e == cudaSuccess) Ly.bound |= static_cast<uint16_t>(1u << which);
            }
        } else if (which == NF_STACK_O_PROJ) {
            if (rows != H || cols != nq * D) {
                st = s->fail(NF_ERR_SHAPE, "BF16 linear layout layers.%d.self_attn.o_proj.weight", layer);
            } else {
                e = upload_box_order(Ly.w_o, reinterpret_cast<const uint8_t*>(data), H, 2 * nq * D);
                if (e == cudaSuccess) Ly.bound |= static_cast<uint16_t>(1u << which);
            }
        } else {
            st = s->fail(NF_ERR_INVALID, "unknown BF16 tensor id %d", which);
        }
    }
    cudaSetDevice(prev);
    if (st != NF_OK) return st;
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "upload: %s", cudaGetErrorString(e));
    return NF_OK;
}

int nf_stack_bind_f32(nf_stack* s, int which, int layer, const float* data, int64_t n) {
    if (!s || !data) return NF_ERR_INVALID;
    s->msg.clear();
    const nf_stack_desc& d = s->d;
    float* dst = nullptr;
    int64_t want = 0;
    if (which == NF_STACK_FINAL_NORM) {
        dst = s->final_norm;
        want = d.hidden;
    } else if (layer >= 0 && layer < d.layers) {
        StackLayer& Ly = s->layers[static_cast<size_t>(layer)];
        if (which == NF_STACK_ATTN_NORM) dst = Ly.attn_norm, want = d.hidden;
        else if (which == NF_STACK_FFN_NORM) dst = Ly.ffn_norm, want = d.hidden;
        else if (which == NF_STACK_Q_NORM) dst = Ly.q_norm, want = kHeadDim;
        else if (which == NF_STACK_K_NORM) dst = Ly.k_norm, want = kHeadDim;
    }
    if (!dst) return s->fail(NF_ERR_INVALID, "unknown F32 tensor id %d or layer %d", which, layer);
    if (n != want) return s->fail(NF_ERR_SHAPE, "vector length mismatch");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    const cudaError_t e = cudaMemcpy(dst, data, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "upload: %s", cudaGetErrorString(e));
    if (which == NF_STACK_FINAL_NORM) s->norm_bound = true;
    else s->layers[static_cast<size_t>(layer)].bound |= static_cast<uint16_t>(1u << which);
    return NF_OK;
}

int nf_stack_finalize(nf_stack* s) {
    if (!s) return NF_ERR_INVALID;
    s->msg.clear();
    if (!s->embed_bound || !s->head_bound || !s->norm_bound)
        return s->fail(NF_ERR_STATE, "missing tensor (embed_tokens, lm_head or the final norm)");
    const uint16_t all = (1u << NF_STACK_Q_PROJ) | (1u << NF_STACK_K_PROJ) | (1u << NF_STACK_V_PROJ) |
                        (1u << NF_STACK_O_PROJ) | (1u << NF_STACK_ATTN_NORM) | (1u << NF_STACK_FFN_NORM) |
                        (1u << NF_STACK_Q_NORM) | (1u << NF_STACK_K_NORM);
    const nf_stack_desc& d = s->d;
    const int64_t H = d.hidden, NQ = static_cast<int64_t>(d.q_heads) * kHeadDim;
    for (int l = 0; l < d.layers; ++l) {
        StackLayer& Ly = s->layers[static_cast<size_t>(l)];
        if ((Ly.bound & all) != all) return s->fail(NF_ERR_STATE, "layer %d: missing attention tensors", l);
        const uint64_t cache_rows = static_cast<uint64_t>(d.max_batch) * d.kv_heads * d.max_context;
        if (!make_tmap_blocked(&Ly.tm_qkv, Ly.w_qkv, static_cast<uint64_t>(box_order_bytes(qkv_rows(d), 2 * H))) ||
            !make_tmap_blocked(&Ly.tm_o, Ly.w_o, static_cast<uint64_t>(box_order_bytes(H, 2 * NQ))) ||
            !make_tmap_2d(&Ly.tm_kc, Ly.kc, true, kHeadDim, cache_rows, 64, 32) ||
            !make_tmap_2d(&Ly.tm_vc, Ly.vc, true, kHeadDim, cache_rows, 64, 32))
            return s->fail(NF_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    }
    s->qkv_host.clear();
    s->qkv_host.shrink_to_fit();
    s->finalized = true;
    return NF_OK;
}

int nf_stack_kv_cache(nf_stack* s, int layer, uint16_t** k_dev, uint16_t** v_dev) {
    if (!s || !k_dev || !v_dev || layer < 0 || layer >= s->d.layers) return NF_ERR_INVALID;
    *k_dev = s->layers[static_cast<size_t>(layer)].kc;
    *v_dev = s->layers[static_cast<size_t>(layer)].vc;
    return NF_OK;
}

int nf_stack_load_kv(nf_stack* s, int layer, const uint16_t* k_host, const uint16_t* v_host) {
    if (!s || !k_host || !v_host || layer < 0 || layer >= s->d.layers) return NF_ERR_INVALID;
    const size_t n = static_cast<size_t>(s->d.max_batch) * s->d.kv_heads * s->d.max_context * kHeadDim;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    const StackLayer& Ly = s->layers[static_cast<size_t>(layer)];
    cudaError_t e = cudaMemcpy(Ly.kc, k_host, n * 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(Ly.vc, v_host, n * 2, cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "cache upload: %s", cudaGetErrorString(e));
    return NF_OK;
}

int nf_stack_fill_kv(nf_stack* s, uint64_t seed) {
    if (!s) return NF_ERR_INVALID;
    const int64_t n = static_cast<int64_t>(s->d.max_batch) * s->d.kv_heads * s->d.max_context * kHeadDim;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < s->d.layers && e == cudaSuccess; ++l) {
        const StackLayer& Ly = s->layers[static_cast<size_t>(l)];
        e = launch_fill_bf16_hash(Ly.kc, n, seed * 1000003ull + 2ull * l, nullptr);
        if (e == cudaSuccess) e = launch_fill_bf16_hash(Ly.vc, n, seed * 1000003ull + 2ull * l + 1ull, nullptr);
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaSetDevice(prev);
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "cache fill: %s", cudaGetErrorString(e));
    return NF_OK;
}

int nf_stack_decode(nf_stack* s, const int32_t* tokens, const int32_t* positions, int batch, int32_t* next,
                    float* final_dev, void* stream) {
    if (!s) return NF_ERR_INVALID;
    s->msg.clear();
    if (!s->finalized) return s->fail(NF_ERR_STATE, "nf_stack_finalize has not run");
    if (!tokens || !positions || !next) return s->fail(NF_ERR_INVALID, "null token, position or output pointer");
    if (batch < 0 || batch > s->d.max_batch) return s->fail(NF_ERR_CAPACITY, "batch must be in [0, max_batch]");
    if (batch == 0) return NF_OK;
    const nf_stack_desc& d = s->d;
    const int T = batch, H = d.hidden, nq = d.q_heads, nkv = d.kv_heads, L = d.max_context;
    const int NQKV = qkv_rows(d), NQ = nq * kHeadDim;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_embed(s->embed, d.vocab, H, tokens, T, s->x, s->err, st);
    int status = NF_OK;
    const float eps = d.norm_eps;
    const int splits = attn_splits(T, nkv, L, s->sms);
    for (int l = 0; l < d.layers && e == cudaSuccess && status == NF_OK; ++l) {
        StackLayer& Ly = s->layers[static_cast<size_t>(l)];
        int S1 = 1, S2 = 1;
        e = launch_rmsnorm(s->x, nullptr, 1, 0, nullptr, Ly.attn_norm, T, H, eps, 0, s->a16, nullptr, st);
        if (e == cudaSuccess)
            e = launch_projection(s, s->tm_a, s->tm_a_s, Ly.tm_qkv, Ly.w_qkv, T, NQKV, H, s->qkv_part,
                                  s->counters + 2 * l, &S1, st);
        if (e == cudaSuccess)
            e = launch_qk_norm_rope(s->qkv_part, S1, static_cast<int64_t>(T) * NQKV, T, nq, nkv, Ly.q_norm, Ly.k_norm,
                                    1e-5f, d.rope_theta, positions, L, s->q, Ly.kc, Ly.vc, s->err, st);
        if (e == cudaSuccess)
            e = launch_gqa_decode(Ly.tm_kc, Ly.tm_vc, s->q, positions, T, nq, nkv, L, splits, s->part_ml,
                                  s->part_acc, s->att16, s->err, st);
        if (e == cudaSuccess)
            e = launch_projection(s, s->tm_att, s->tm_att_s, Ly.tm_o, Ly.w_o, T, H, NQ, s->o_part,
                                  s->counters + 2 * l + 1, &S2, st);
        // h = x + o (the o projection's split-K slices summed here); f = rmsnorm_stash(h)
        if (e == cudaSuccess)
            e = launch_rmsnorm(s->x, s->o_part, S2, static_cast<int64_t>(T) * H, s->h, Ly.ffn_norm, T, H, eps, 1,
                               s->f16, nullptr, st);
        if (e != cudaSuccess) break;
        // x = h + ffn(f)
        const int fst = nf_moe_forward(Ly.ffn, s->f16, s->h, T, s->x, nullptr, nullptr, stream);
        if (fst != NF_OK) status = s->fail(fst, "layer %d FFN: %s", l, nf_moe_last_error(Ly.ffn));
    }
    if (e == cudaSuccess && status == NF_OK)
        e = launch_rmsnorm(s->x, nullptr, 1, 0, nullptr, s->final_norm, T, H, eps, 0, nullptr,
                           final_dev ? final_dev : s->fin, st);
    cudaSetDevice(prev);
    if (status != NF_OK) return status;
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
    int tst = nf_tp_linear_bf16(s->head, s->lm_head, d.vocab, H, final_dev ? final_dev : s->fin, T, nullptr, stream);
    if (tst == NF_OK) tst = nf_tp_argmax(s->head, T, d.vocab, next, stream);
    if (tst != NF_OK) return s->fail(tst, "lm_head: %s", nf_tp_last_error(s->head));
    return NF_OK;
}

int nf_stack_sync(nf_stack* s, void* stream) {
    if (!s) return NF_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    int derr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&derr, s->err, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && derr != 0) cudaMemset(s->err, 0, 4);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return s->fail(NF_ERR_CUDA, "synchronise: %s", cudaGetErrorString(e));
    if (derr == NF_DEVERR_BAD_TOKEN)
        return s->fail(NF_ERR_INVALID, "prompt token is outside the vocabulary, or a position outside the cache");
    if (derr != 0) return s->fail(NF_ERR_TIMEOUT, "a device-side bounded wait gave up (code %d)", derr);
    for (int l = 0; l < s->d.layers; ++l) {
        const int fst = nf_moe_sync(s->layers[static_cast<size_t>(l)].ffn, stream);
        if (fst != NF_OK) return s->fail(fst, "layer %d FFN: %s", l, nf_moe_last_error(s->layers[static_cast<size_t>(l)].ffn));
    }
    const int tst = nf_tp_sync(s->head, stream);
    if (tst != NF_OK) return s->fail(tst, "lm_head: %s", nf_tp_last_error(s->head));
    return NF_OK;
}

}  // extern "C"
