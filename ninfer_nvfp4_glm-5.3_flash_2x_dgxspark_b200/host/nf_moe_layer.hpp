// nf_moe_layer.hpp -- C++ host class over the C-ABI of include/nf_moe.h, in the
// shape of the reference's MoE path: tensors looked up by checkpoint name
// from a store (Store::get, src/text_forward.cpp:464-470; kinds 'b' BF16,
// 'f' F32, 'u' U8, '8' F8_E4M3, :408-414), the parameter_schema names of one
// MoE layer (src/parameter_schema.cpp:72-98), and a forward with
// TextModel::moe's arguments (prefix, x, y) (src/text_forward.cpp:924).
// Failures throw std::runtime_error with the library's message, as the
// reference's fail() does (src/text_forward.cpp:40).  Header-only: link
// lib/libnf_moe.so.
#pragma once

#include "nf_moe.h"

#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

namespace nf_host {

// A borrowed tensor: what the reference's Store hands out.
struct TensorView {
    const void* data = nullptr;
    std::vector<int64_t> shape;
    char kind = '?';  // 'b' BF16, 'f' F32, 'u' U8, '8' F8_E4M3
    int64_t dim(int axis) const {
        if (axis < 0 || axis >= static_cast<int>(shape.size())) throw std::runtime_error("tensor rank is short");
        return shape[static_cast<size_t>(axis)];
    }
};

// Name -> tensor; throws "missing tensor <name>" like Store::get.
using StoreLookup = std::function<const TensorView*(const std::string&)>;

namespace detail {

inline const TensorView& get(const StoreLookup& store, const std::string& name) {
    const TensorView* t = store(name);
    if (!t) throw std::runtime_error("missing tensor " + name);
    return *t;
}

// Store::scalar (src/text_forward.cpp:470-476).
inline float scalar(const StoreLookup& store, const std::string& name) {
    const TensorView& t = get(store, name);
    if (t.kind != 'f' || !t.shape.empty()) throw std::runtime_error("expected rank-0 F32 for " + name);
    return *static_cast<const float*>(t.data);
}

// One NVFP4 linear by checkpoint name (linear_nvfp4's lookups,
// src/text_forward.cpp:833-843): <base>.weight U8 [N, K/2],
// <base>.weight_scale F8_E4M3 [N, K/16], rank-0 F32 weight_scale_2 and
// input_scale.  Returns the library's status.  Both tensors must be rank 2
// ("NVFP4 layout") and the scales [N, K/16] for codes [N, K/2] ("NVFP4
// shape"): the library takes N and K only and reads N K/16 scale bytes.
inline int bind_nvfp4_named(nf_moe* h, int expert, int proj, const StoreLookup& store, const std::string& base) {
    const TensorView& w = get(store, base + ".weight");
    const TensorView& s = get(store, base + ".weight_scale");
    if (w.kind != 'u' || s.kind != '8' || w.shape.size() != 2 || s.shape.size() != 2)
        throw std::runtime_error("NVFP4 layout " + base);
    if (s.dim(0) != w.dim(0) || s.dim(1) != w.dim(1) * 2 / 16) throw std::runtime_error("NVFP4 shape " + base);
    return nf_moe_bind_nvfp4(h, expert, proj, static_cast<const uint8_t*>(w.data), static_cast<const uint8_t*>(s.data),
                             scalar(store, base + ".weight_scale_2"), scalar(store, base + ".input_scale"), w.dim(0),
                             w.dim(1) * 2);
}

}  // namespace detail

class MoeLayer {
public:
    // desc: the layer's shapes (from ModelSpec); max_tokens per forward.
    MoeLayer(const nf_moe_desc& desc, int device) {
        if (nf_moe_create(&desc, device, &h_) != NF_OK) throw std::runtime_error(nf_moe_last_error(nullptr));
        d_ = desc;
    }
    // This rank's handle of an expert-parallel group (collective: every rank
    // of the group constructs its handle with the same group id, from
    // nf_ep_unique_id on one rank); max_tokens is per rank.  Binding takes
    // every expert's tensors, as for one GPU, and keeps the rank's own.
    MoeLayer(const nf_moe_desc& desc, int device, int rank, int world, const uint8_t* group_id, int id_len) {
        if (nf_moe_create_ep(&desc, device, rank, world, group_id, id_len, &h_) != NF_OK)
            throw std::runtime_error(nf_moe_last_error(nullptr));
        d_ = desc;
    }
    MoeLayer(const MoeLayer&) = delete;
    MoeLayer& operator=(const MoeLayer&) = delete;
    ~MoeLayer() { nf_moe_destroy(h_); }

    nf_moe* handle() const { return h_; }

    // Binds every tensor of the layer `prefix` (e.g. "model.language_model.layers.3.")
    // by checkpoint name and finalizes.
    void bind_from_store(const StoreLookup& store, const std::string& prefix) {
        auto get = [&](const std::string& name) -> const TensorView& {
            const TensorView* t = store(name);
            if (!t) throw std::runtime_error("missing tensor " + name);
            return *t;
        };
        auto bf16 = [&](int which, int expert, const std::string& name) {
            const TensorView& t = get(name);
            if (t.kind != 'b' || t.shape.size() != 2) throw std::runtime_error("BF16 linear layout " + name);
            check(nf_moe_bind_bf16(h_, which, expert, static_cast<const uint16_t*>(t.data), t.dim(0), t.dim(1)));
        };
        bf16(NF_BF16_ROUTER, 0, prefix + "mlp.gate.weight");
        const TensorView& bias = get(prefix + "mlp.gate.e_score_correction_bias");
        if (bias.kind != 'f' || bias.shape.size() != 1)
            throw std::runtime_error("vector length mismatch for " + prefix + "mlp.gate.e_score_correction_bias");
        check(nf_moe_bind_f32(h_, NF_F32_ROUTER_BIAS, static_cast<const float*>(bias.data), bias.dim(0)));
        if (d_.shared_inter > 0) {
            bf16(NF_BF16_SHARED_GATE, 0, prefix + "mlp.shared_experts.gate_proj.weight");
            bf16(NF_BF16_SHARED_UP, 0, prefix + "mlp.shared_experts.up_proj.weight");
            bf16(NF_BF16_SHARED_DOWN, 0, prefix + "mlp.shared_experts.down_proj.weight");
        }
        static const char* proj[3] = {"gate_proj", "up_proj", "down_proj"};
        for (int e = 0; e < d_.experts; ++e)
            for (int p = 0; p < 3; ++p) {
                const std::string base = prefix + "mlp.experts." + std::to_string(e) + "." + proj[p];
                if (d_.expert_kind == NF_EXPERTS_BF16) {
                    bf16(NF_BF16_EXPERT_GATE + p, e, base + ".weight");
                    continue;
                }
                check(detail::bind_nvfp4_named(h_, e, p, store, base));
            }
        check(nf_moe_finalize(h_));
    }

    // TextModel::moe's contract over `tokens` rows: x fp32 (BF16-valued) in,
    // y fp32 out, host memory; synchronous.
    void moe(const float* x, float* y, int tokens = 1) {
        check(nf_moe_forward_host(h_, x, nullptr, tokens, y, nullptr, nullptr));
    }
    // The same with the routes (indices, weights: tokens x top_k).
    void moe(const float* x, float* y, int tokens, int32_t* idx, float* w) {
        check(nf_moe_forward_host(h_, x, nullptr, tokens, y, idx, w));
    }
    // Device buffers, asynchronous on `stream` (a cudaStream_t): x BF16 bits
    // [tokens, H], residual fp32 or null, y fp32 [tokens, H], routes optional.
    // Every rank of an expert-parallel group calls it each step, also with
    // tokens == 0.
    void forward(const uint16_t* x_dev, const float* residual_dev, int tokens, float* y_dev, void* stream,
                 int32_t* idx_dev = nullptr, float* w_dev = nullptr) {
        check(nf_moe_forward(h_, x_dev, residual_dev, tokens, y_dev, idx_dev, w_dev, stream));
    }
    // "none", "nccl" or "nvlink": the exchange the group agreed on.
    const char* ep_transport() const {
        switch (nf_moe_ep_transport(h_)) {
            case NF_EP_NCCL: return "nccl";
            case NF_EP_NVLINK: return "nvlink";
            default: return "none";
        }
    }

private:
    void check(int status) const {
        if (status != NF_OK) throw std::runtime_error(nf_moe_last_error(h_));
    }
    nf_moe* h_ = nullptr;
    nf_moe_desc d_{};
};

// The dense NVFP4 MLP of the first layers (TextModel::dense_mlp,
// src/text_forward.cpp:909-915), bound by the dense layers' names
// (<prefix>mlp.{gate,up,down}_proj, src/parameter_schema.cpp:187-191).
class DenseMlp {
public:
    DenseMlp(int hidden, int inter, float swiglu_limit, int max_tokens, int device) {
        if (nf_moe_create_dense(hidden, inter, swiglu_limit, max_tokens, device, &h_) != NF_OK)
            throw std::runtime_error(nf_moe_last_error(nullptr));
    }
    DenseMlp(const DenseMlp&) = delete;
    DenseMlp& operator=(const DenseMlp&) = delete;
    ~DenseMlp() { nf_moe_destroy(h_); }

    nf_moe* handle() const { return h_; }

    void bind_from_store(const StoreLookup& store, const std::string& prefix) {
        static const char* proj[3] = {"gate_proj", "up_proj", "down_proj"};
        for (int p = 0; p < 3; ++p) check(detail::bind_nvfp4_named(h_, 0, p, store, prefix + "mlp." + proj[p]));
        check(nf_moe_finalize(h_));
    }

    // dense_mlp's contract over `tokens` rows: x fp32 (BF16-valued) in, y fp32
    // out, host memory; synchronous.
    void dense_mlp(const float* x, float* y, int tokens = 1) {
        check(nf_moe_forward_host(h_, x, nullptr, tokens, y, nullptr, nullptr));
    }

private:
    void check(int status) const {
        if (status != NF_OK) throw std::runtime_error(nf_moe_last_error(h_));
    }
    nf_moe* h_ = nullptr;
};

}  // namespace nf_host
