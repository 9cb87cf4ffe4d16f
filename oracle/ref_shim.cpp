// ref_shim.cpp -- exposes the reference's own MoE primitives through a C ABI.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's sources where they lie (it #includes src/text_forward.cpp,
// whose helpers live in an anonymous namespace, and links nvfp4_decode.cpp,
// model_spec.cpp, speculative.cpp and tiny_layer.cpp) into
// oracle/_ref/libnf_ref.so.  Nothing here re-implements arithmetic: every
// number comes from a reference function.  ref_moe_layer composes those
// functions in the order of TextModel::moe (src/text_forward.cpp:924-963),
// because TextModel itself is pinned to the 4096-wide, 288-expert model spec
// and cannot be constructed at the BASELINE shapes.
#include "text_forward.cpp"  // NOLINT: the reference's own translation unit
#include "ninfer_glm53/tiny_layer.hpp"

#include "nf_oracle.h"  // or_moe_weights (a plain struct of pointers)

#include <span>

namespace R = ninfer::glm53;

extern "C" {

float ref_sigmoid(float x) { return R::sigmoid(x); }
unsigned char ref_f32_to_e4m3(float v) { return R::f32_to_e4m3(v); }
float ref_e4m3_to_f32(unsigned char b) { return R::fp8_e4m3_to_f32(b); }
float ref_e2m1(unsigned char n) { return R::e2m1(n); }
float ref_cast_to_e2m1(float v) { return R::cast_to_e2m1(v); }
unsigned short ref_f32_to_bf16(float v) { return R::f32_to_bf16(v); }

int ref_quant_dequant(const float* x, int cols, float input_scale, float* y) {
    try {
        R::quant_dequant_nvfp4_activation(x, cols, input_scale, y);
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

void ref_gemv_nvfp4_rows(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                         const float* x, int rows, int cols, int row0, int row1, float* y) {
    R::gemv_nvfp4_rows(packed, scales, scale2, input_scale, x, rows, cols, row0, row1, y);
}

void ref_gemv_bf16(const uint16_t* weight, const float* x, int rows, int cols, int row0, int row1, float* y) {
    R::gemv_bf16(weight, x, rows, cols, row0, row1, y);
}

void ref_router_select(const float* logits, const float* bias, int experts, int top_k, float scaling, int normalize,
                       int* indices, float* weights) {
    R::router_select(logits, bias, experts, top_k, scaling, normalize != 0, indices, weights);
}

void ref_swiglu_clamp(const float* g, const float* u, int n, float limit, float* h) {
    R::swiglu_clamp(g, u, n, limit, h);
}
void ref_swiglu_clamp_bf16(const float* g, const float* u, int n, float limit, float* h) {
    R::swiglu_clamp_bf16(g, u, n, limit, h);
}
void ref_mhc_combine(const float* residual, const float* branch, const float* post, const float* comb, int hc,
                     int hidden, float* out) {
    R::mhc_combine(residual, branch, post, comb, hc, hidden, out);
}

// Nvfp4MatrixView validation + at() (src/nvfp4_decode.cpp:56-97, 116-130).
int ref_nvfp4_dequantize(const uint8_t* packed, int64_t packed_len, const uint8_t* scales, int64_t scales_len,
                         float global_scale, int64_t rows, int64_t cols, float* weight, int64_t weight_len) {
    try {
        R::nvfp4_dequantize(std::span<const std::uint8_t>(packed, static_cast<std::size_t>(packed_len)),
                            std::span<const std::uint8_t>(scales, static_cast<std::size_t>(scales_len)),
                            global_scale, static_cast<std::size_t>(rows), static_cast<std::size_t>(cols),
                            std::span<float>(weight, static_cast<std::size_t>(weight_len)));
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

void ref_dense_residual_proj(const float* x, const float* nw, const float* proj, float eps, int width, float* y) {
    R::dense_residual_proj(x, nw, proj, eps, width, y);
}
void ref_rmsnorm(const float* x, const float* w, float eps, int width, float* y) { R::rmsnorm(x, w, eps, width, y); }

// linear_nvfp4 (src/text_forward.cpp:832-856) minus the Store lookup.
static void linear_nvfp4(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                         const float* x, int cols, float* y, int rows) {
    std::vector<float> quantized(static_cast<std::size_t>(cols));
    R::quant_dequant_nvfp4_activation(x, cols, input_scale, quantized.data());
    R::gemv_nvfp4_rows(packed, scales, scale2, input_scale, quantized.data(), rows, cols, 0, rows, y);
    for (int row = 0; row < rows; ++row) y[row] = R::bf16_to_f32(R::f32_to_bf16(y[row]));
}

// mlp_bf16 (src/text_forward.cpp:917-922) over explicit matrices.
static void mlp_bf16(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int hidden, int inter,
                     float limit, const float* x, float* y) {
    std::vector<float> g(static_cast<std::size_t>(inter)), u(g.size()), h(g.size());
    R::gemv_bf16(gate, x, inter, hidden, 0, inter, g.data());
    R::gemv_bf16(up, x, inter, hidden, 0, inter, u.data());
    R::swiglu_clamp(g.data(), u.data(), inter, limit, h.data());
    R::gemv_bf16(down, h.data(), hidden, inter, 0, hidden, y);
}

// TextModel::moe (src/text_forward.cpp:924-963) for `tokens` tokens one at a
// time (OpenMP only inside the GEMVs, as in the reference), then the hc = 1
// residual combine (src/text_forward.cpp:906).  Returns 0, -1 on a reference
// exception, -2 for a descriptor the reference cannot express (group limit).
int ref_moe_layer(const or_moe_weights* w, int tokens, const float* x, const float* residual, float* y,
                  int* indices, float* weights) {
    if (w->n_group > 1 && w->topk_group < w->n_group) return -2;
    const int H = w->hidden, E = w->experts, K = w->top_k, I = w->inter;
    try {
        std::vector<float> logits(static_cast<std::size_t>(E)), g(static_cast<std::size_t>(I)), u(g.size()),
            h(g.size()), down(static_cast<std::size_t>(H)), shared(down.size()), out(down.size());
        std::vector<int> idx(static_cast<std::size_t>(K));
        std::vector<float> wt(static_cast<std::size_t>(K));
        for (int t = 0; t < tokens; ++t) {
            const float* xt = x + static_cast<std::size_t>(t) * H;
            float* yt = y + static_cast<std::size_t>(t) * H;
            R::gemv_bf16(w->router_w, xt, E, H, 0, E, logits.data());
            R::router_select(logits.data(), w->router_bias, E, K, w->scaling, w->normalize != 0, idx.data(),
                             wt.data());
            std::fill(yt, yt + H, 0.f);
            for (int p = 0; p < K; ++p) {
                const int e = idx[static_cast<std::size_t>(p)];
                if (w->bf16_experts) {
                    mlp_bf16(w->gate_bf16 + static_cast<std::size_t>(e) * I * H,
                             w->up_bf16 + static_cast<std::size_t>(e) * I * H,
                             w->down_bf16 + static_cast<std::size_t>(e) * H * I, H, I, w->swiglu_limit, xt,
                             down.data());
                } else {
                    const std::size_t gp = static_cast<std::size_t>(e) * I * (H / 2);
                    const std::size_t gs = static_cast<std::size_t>(e) * I * (H / 16);
                    const std::size_t dp = static_cast<std::size_t>(e) * H * (I / 2);
                    const std::size_t ds = static_cast<std::size_t>(e) * H * (I / 16);
                    linear_nvfp4(w->gate_packed + gp, w->gate_scales + gs, w->gate_ws2[e], w->gate_in[e], xt, H,
                                 g.data(), I);
                    linear_nvfp4(w->up_packed + gp, w->up_scales + gs, w->up_ws2[e], w->up_in[e], xt, H, u.data(),
                                 I);
                    R::swiglu_clamp(g.data(), u.data(), I, w->swiglu_limit, h.data());
                    linear_nvfp4(w->down_packed + dp, w->down_scales + ds, w->down_ws2[e], w->down_in[e], h.data(),
                                 I, down.data(), H);
                }
                const float weight = wt[static_cast<std::size_t>(p)];
                for (int d = 0; d < H; ++d) yt[d] += weight * down[static_cast<std::size_t>(d)];
            }
            if (w->shared_inter > 0) {
                mlp_bf16(w->shared_gate, w->shared_up, w->shared_down, H, w->shared_inter, w->swiglu_limit, xt,
                         shared.data());
                for (int d = 0; d < H; ++d) yt[d] += shared[static_cast<std::size_t>(d)];
            }
            if (residual != nullptr) {
                const float one = 1.f;
                R::mhc_combine(residual + static_cast<std::size_t>(t) * H, yt, &one, &one, 1, H, out.data());
                std::copy(out.begin(), out.end(), yt);
            }
            if (indices) std::copy(idx.begin(), idx.end(), indices + static_cast<std::size_t>(t) * K);
            if (weights) std::copy(wt.begin(), wt.end(), weights + static_cast<std::size_t>(t) * K);
        }
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// TextModel::dense_mlp (src/text_forward.cpp:909-915) for `tokens` tokens one
// at a time, then the hc = 1 residual combine (src/text_forward.cpp:906).
// Returns 0 or -1 on a reference exception.
int ref_dense_mlp(const or_dense_weights* w, int tokens, const float* x, const float* residual, float* y) {
    const int H = w->hidden, I = w->inter;
    try {
        std::vector<float> g(static_cast<std::size_t>(I)), u(g.size()), h(g.size()), out(static_cast<std::size_t>(H));
        for (int t = 0; t < tokens; ++t) {
            const float* xt = x + static_cast<std::size_t>(t) * H;
            float* yt = y + static_cast<std::size_t>(t) * H;
            linear_nvfp4(w->gate_packed, w->gate_scales, w->gate_ws2, w->gate_in, xt, H, g.data(), I);
            linear_nvfp4(w->up_packed, w->up_scales, w->up_ws2, w->up_in, xt, H, u.data(), I);
            R::swiglu_clamp_bf16(g.data(), u.data(), I, w->swiglu_limit, h.data());
            linear_nvfp4(w->down_packed, w->down_scales, w->down_ws2, w->down_in, h.data(), I, yt, H);
            if (residual != nullptr) {
                const float one = 1.f;
                R::mhc_combine(residual + static_cast<std::size_t>(t) * H, yt, &one, &one, 1, H, out.data());
                std::copy(out.begin(), out.end(), yt);
            }
        }
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

}  // extern "C"
