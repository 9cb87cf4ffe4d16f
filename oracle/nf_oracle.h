/*
 * nf_oracle.h -- CPU restatement of the reference's NVFP4 MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this code, and
 * only as the checker.  The product library (libnf_moe.so) never links it.
 *
 * Every function restates one function of the reference
 * (alan70435-vibe/Ninfer_Nvfp4_Glm-5.3_Flash_2x_DgxSpark) in plain C, with the
 * same operation order and the same float rounding points, compiled with
 * -ffp-contract=off so that no multiply-add is fused (the reference's x86-64
 * build emits none).  The citation beside each declaration is the reference
 * function it follows.  Parity of this restatement is pinned bit for bit
 * against the reference's own sources (oracle/_ref, built by oracle/Makefile)
 * and against the known-answer values of the reference's tests.
 */
#ifndef NF_ORACLE_H
#define NF_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar formats ---------------------------------------------------- */
/* src/text_forward.cpp:54-59 */
float or_bf16_to_f32(uint16_t bits);
/* src/text_forward.cpp:87-95 (round to nearest even, NaN passes its top half) */
uint16_t or_f32_to_bf16(float value);
/* src/text_forward.cpp:60-85 (software E4M3FN with the subnormal cap at 7) */
uint8_t or_f32_to_e4m3(float value);
/* src/nvfp4_decode.cpp:42-54 */
float or_e4m3_to_f32(uint8_t bits);
/* src/nvfp4_decode.cpp:37-40 */
float or_e2m1(uint8_t nibble);
/* src/text_forward.cpp:510-522 (snap to the E2M1 grid; returns the value) */
float or_cast_to_e2m1(float value);
/* E2M1 code (sign bit 3) of or_cast_to_e2m1(value). */
uint8_t or_e2m1_code(float value);
/* src/text_forward.cpp:42-49 */
float or_sigmoid(float x);

/* ---- NVFP4 activation quantiser ----------------------------------------
 * src/text_forward.cpp:527-550 quant_dequant_nvfp4_activation.
 * y (nullable) receives e2m1 * block_scale (the reference's fake-quant
 * vector).  codes (nullable, cols/2 bytes, low nibble = even element) and
 * scales (nullable, cols/16 E4M3 codes) receive the encoded form that the
 * tensor-core path consumes.  Returns 0, or -1 for the reference's
 * "NVFP4 input scale" rejection (bad input_scale or cols % 16). */
int or_quant_nvfp4_activation(const float* x, int cols, float input_scale, float* y, uint8_t* codes,
                              uint8_t* scales);

/* ---- GEMVs --------------------------------------------------------------- */
/* src/text_forward.cpp:552-576 gemv_nvfp4_rows, rows [row0,row1). */
void or_gemv_nvfp4_rows(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                        const float* x, int rows, int cols, int row0, int row1, float* y);
/* src/text_forward.cpp:497-508 gemv_bf16, rows [row0,row1). */
void or_gemv_bf16(const uint16_t* weight, const float* x, int rows, int cols, int row0, int row1, float* y);
/* src/text_forward.cpp:832-856 linear_nvfp4 minus the Store lookup: quantise x,
 * GEMV, round every output to BF16.  Returns 0 or -1 (bad input scale). */
int or_linear_nvfp4(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                    const float* x, int cols, float* y, int rows);

/* ---- router / activation / combine -------------------------------------- */
/* src/text_forward.cpp:1447-1471 router_select (ties keep the lower index). */
void or_router_select(const float* logits, const float* bias, int experts, int top_k, float scaling,
                      int normalize, int* indices, float* weights);
/* Group-limited variant (DeepSeek-V3 style noaux_tc): experts split into
 * n_group equal groups, a group scores the sum of its two best choice values,
 * the topk_group best groups stay eligible, then router_select runs over the
 * eligible experts.  The reference has no group limit (its model spec has no
 * n_group), so with n_group == 1 this is exactly or_router_select. */
void or_router_select_grouped(const float* logits, const float* bias, int experts, int top_k, float scaling,
                              int normalize, int n_group, int topk_group, int* indices, float* weights);
/* src/text_forward.cpp:1439-1445 */
void or_swiglu_clamp(const float* gate, const float* up, int n, float limit, float* hidden);
/* src/text_forward.cpp:99-106 (dense layers 0-2) */
void or_swiglu_clamp_bf16(const float* gate, const float* up, int n, float limit, float* hidden);
/* src/text_forward.cpp:1646-1657 */
void or_mhc_combine(const float* residual, const float* branch, const float* post, const float* comb, int hc,
                    int hidden, float* out);

/* ---- NVFP4 dequantisation -------------------------------------------------
 * src/nvfp4_decode.cpp:88-97 Nvfp4MatrixView::at (double product, one
 * rounding) over a whole [rows, cols] matrix.  Validation follows the view
 * constructor (src/nvfp4_decode.cpp:56-79); returns 0 or -1 without writing. */
int or_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales, float global_scale, int64_t rows,
                        int64_t cols, float* weight);

/* ---- tiny layer (src/tiny_layer.cpp:7-26) --------------------------------- */
void or_rmsnorm(const float* x, const float* weight, float eps, int width, float* y);
void or_dense_residual_proj(const float* x, const float* norm_weight, const float* projection, float eps,
                            int width, float* y);

/* ---- the MoE layer --------------------------------------------------------
 * src/text_forward.cpp:924-963 TextModel::moe for every token, followed by
 * the hc = 1 residual form of mhc_combine (src/text_forward.cpp:906,
 * 1646-1657) when residual is not NULL.  Shapes come from the descriptor
 * instead of the pinned model spec.  Weight arrays are contiguous per kind:
 *   gate/up packed [E][I][H/2], scales [E][I][H/16], down packed [E][H][I/2],
 *   scales [E][H][I/16]; per-expert scalars [E]; shared BF16 gate/up [Is][H],
 *   down [H][Is]; BF16 routed experts (bf16_experts = 1, the layer-45 form,
 *   whose oracle is mlp_bf16 src/text_forward.cpp:917-922) gate/up [E][I][H],
 *   down [E][H][I]. */
typedef struct or_moe_weights {
    int hidden, experts, top_k, inter, shared_inter;
    float scaling, swiglu_limit;
    int n_group, topk_group, normalize, bf16_experts;
    const uint16_t* router_w;     /* [E][H] BF16 */
    const float* router_bias;     /* [E] */
    const uint8_t *gate_packed, *gate_scales, *up_packed, *up_scales, *down_packed, *down_scales;
    const float *gate_ws2, *gate_in, *up_ws2, *up_in, *down_ws2, *down_in;
    const uint16_t *gate_bf16, *up_bf16, *down_bf16;             /* bf16_experts only */
    const uint16_t *shared_gate, *shared_up, *shared_down;        /* NULL when shared_inter == 0 */
} or_moe_weights;

/* x: [T][H] fp32 (BF16-valued, as rmsnorm_stash produces), residual
 * nullable [T][H], y [T][H]; indices/weights nullable [T][k].
 * Optional per-token taps (nullable): routed [T][H] (the routed sum before
 * the shared expert), shared [T][H] (shared expert output).
 * Returns 0 or -1 (bad input scale). */
int or_moe_layer(const or_moe_weights* w, int tokens, const float* x, const float* residual, float* y,
                 int* indices, float* weights, float* routed, float* shared);

/* One expert projection output for one token, for stage-level parity tests:
 * h (nullable, [I]) = swiglu(gate, up) for expert e, down (nullable, [H]) =
 * the BF16-rounded down projection of h.  Returns 0 or -1. */
int or_expert_forward(const or_moe_weights* w, int expert, const float* x, float* h, float* down);

/* ---- the dense NVFP4 MLP (layers 0-2) --------------------------------------
 * src/text_forward.cpp:909-915 TextModel::dense_mlp for every token: NVFP4
 * gate and up linears (linear_nvfp4, outputs rounded to BF16),
 * swiglu_clamp_bf16 (:99-106), NVFP4 down linear; then the hc = 1 residual
 * form of mhc_combine (src/text_forward.cpp:906, 1646-1657) when residual is
 * not NULL.  Packed [inter][hidden/2] (gate, up), [hidden][inter/2] (down)
 * with block scales [rows][cols/16]. */
typedef struct or_dense_weights {
    int hidden, inter;
    float swiglu_limit;
    const uint8_t *gate_packed, *gate_scales, *up_packed, *up_scales, *down_packed, *down_scales;
    float gate_ws2, gate_in, up_ws2, up_in, down_ws2, down_in;
} or_dense_weights;

/* x [T][H] fp32 (BF16-valued), residual nullable [T][H], y [T][H]; h
 * (nullable, [T][I]) receives swiglu_clamp_bf16's output.  Returns 0 or -1
 * (bad input scale). */
int or_dense_mlp(const or_dense_weights* w, int tokens, const float* x, const float* residual, float* y, float* h);

/* Router logits for one token: gemv_bf16 over [E][H] (src/text_forward.cpp:926). */
void or_router_logits(const or_moe_weights* w, const float* x, float* logits);

/* Router for T tokens (src/text_forward.cpp:926-931): logits [T][E]
 * (nullable), indices / weights [T][k]; tokens in parallel. */
void or_route_tokens(const or_moe_weights* w, int tokens, const float* x, float* logits, int* indices,
                     float* weights);

/* or_sigmoid over n floats (OpenMP). */
void or_sigmoid_array(const float* x, int64_t n, float* y);

#ifdef __cplusplus
}
#endif
#endif
