/*
 * nf_oracle.c -- CPU restatement of the reference's NVFP4 MoE path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  See
 * nf_oracle.h for the contract and the reference citation of every
 * function.  Build flags matter: -O2 -ffp-contract=off (no fused
 * multiply-add, like the reference's x86-64 build) and -fopenmp.
 */
#include "nf_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/text_forward.cpp:54-59 */
float or_bf16_to_f32(uint16_t bits) {
    uint32_t wide = (uint32_t)bits << 16;
    float out;
    memcpy(&out, &wide, sizeof(out));
    return out;
}

/* src/text_forward.cpp:87-95 */
uint16_t or_f32_to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    const uint32_t lsb = (bits >> 16) & 1u;
    const uint32_t round = 0x7fffu + lsb;
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(bits >> 16);
    bits += round;
    return (uint16_t)(bits >> 16);
}

static float bf16_round(float v) { return or_bf16_to_f32(or_f32_to_bf16(v)); }

/* src/text_forward.cpp:60-85.  Normal codes round the 3-bit mantissa to
 * nearest even; the subnormal band rounds v*2^9 and caps the code at 7, so
 * values in [15*2^-10, 2^-6) give 0x07 where IEEE rounding gives 0x08. */
uint8_t or_f32_to_e4m3(float value) {
    if (isnan(value)) return 0x7f;
    const uint8_t sign = signbit(value) ? 0x80 : 0x00;
    float magnitude = fabsf(value);
    if (magnitude == 0.f) return sign;
    if (magnitude > 448.f) magnitude = 448.f;
    int exponent = 0;
    const float fraction = frexpf(magnitude, &exponent);
    const float normal = fraction * 2.f;
    int biased = exponent - 1 + 7;
    if (biased <= 0) {
        int mantissa = (int)nearbyintf(ldexpf(magnitude, 9));
        if (mantissa > 7) mantissa = 7;
        if (mantissa < 0) mantissa = 0;
        return (uint8_t)(sign | mantissa);
    }
    if (biased > 15) return (uint8_t)(sign | 0x7e);
    int mantissa = (int)nearbyintf((normal - 1.f) * 8.f);
    if (mantissa == 8) {
        mantissa = 0;
        ++biased;
        if (biased > 15) return (uint8_t)(sign | 0x7e);
    }
    if (biased >= 15 && mantissa > 6) return (uint8_t)(sign | 0x7e);
    return (uint8_t)(sign | (biased << 3) | mantissa);
}

/* src/nvfp4_decode.cpp:42-54 */
float or_e4m3_to_f32(uint8_t bits) {
    const int exponent = (bits >> 3) & 0xf;
    const int mantissa = bits & 0x7;
    float magnitude;
    if (exponent == 0) {
        magnitude = ldexpf((float)mantissa, -9);
    } else if (exponent == 15 && mantissa == 7) {
        magnitude = NAN;
    } else {
        magnitude = ldexpf(1.f + (float)mantissa / 8.f, exponent - 7);
    }
    return copysignf(magnitude, (bits & 0x80u) ? -1.f : 1.f);
}

/* src/nvfp4_decode.cpp:35-40 (the 8-entry magnitude table, sign in bit 3) */
static const float kE2M1[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};

float or_e2m1(uint8_t nibble) {
    const float magnitude = kE2M1[nibble & 0x7u];
    return (nibble & 0x8u) ? -magnitude : magnitude;
}

/* src/text_forward.cpp:510-522.  Interval edges: ties at 0.25 and 2.5 and 5
 * go down, ties at 0.75 / 1.25 / 1.75 / 3.5 go to the even neighbour; beyond
 * 5 (and NaN, which fails every comparison) snaps to 6. */
float or_cast_to_e2m1(float value) {
    const float sign = copysignf(1.f, value);
    const float magnitude = fabsf(value);
    float snapped = 6.f;
    if (magnitude <= 0.25f) snapped = 0.f;
    else if (magnitude < 0.75f) snapped = 0.5f;
    else if (magnitude <= 1.25f) snapped = 1.f;
    else if (magnitude < 1.75f) snapped = 1.5f;
    else if (magnitude <= 2.5f) snapped = 2.f;
    else if (magnitude < 3.5f) snapped = 3.f;
    else if (magnitude <= 5.f) snapped = 4.f;
    return sign * snapped;
}

uint8_t or_e2m1_code(float value) {
    const float snapped = or_cast_to_e2m1(value);
    const float magnitude = fabsf(snapped);
    uint8_t code = 7;
    for (uint8_t c = 0; c < 8; ++c) {
        if (kE2M1[c] == magnitude) {
            code = c;
            break;
        }
    }
    return (uint8_t)(code | (signbit(snapped) ? 0x8u : 0x0u));
}

/* src/text_forward.cpp:42-49 (two branches, libm expf) */
float or_sigmoid(float x) {
    if (x >= 0.f) {
        const float z = expf(-x);
        return 1.f / (1.f + z);
    }
    const float z = expf(x);
    return z / (1.f + z);
}

static float silu(float x) { return x * or_sigmoid(x); }

/* src/text_forward.cpp:527-550 */
int or_quant_nvfp4_activation(const float* x, int cols, float input_scale, float* y, uint8_t* codes,
                              uint8_t* scales) {
    if (!(input_scale > 0.f) || !isfinite(input_scale) || cols % 16 != 0) return -1;
    const float global_scale = 1.f / input_scale;
    for (int group = 0; group < cols / 16; ++group) {
        float rounded[16];
        float peak = 0.f;
        for (int lane = 0; lane < 16; ++lane) {
            rounded[lane] = bf16_round(x[group * 16 + lane]);
            /* std::max(peak, v) keeps peak when v is NaN */
            const float a = fabsf(rounded[lane]);
            peak = (peak < a) ? a : peak;
        }
        float scale = global_scale * (peak / 6.f);
        if (scale > 448.f) scale = 448.f;
        if (scale < -448.f) scale = -448.f;
        const uint8_t scale_code = or_f32_to_e4m3(scale);
        scale = or_e4m3_to_f32(scale_code);
        const float reduced = scale / global_scale;
        const float output_scale = 1.f / (reduced + (reduced == 0.f ? 1.0e8f : 0.f));
        if (scales) scales[group] = scale_code;
        for (int lane = 0; lane < 16; ++lane) {
            float clipped = rounded[lane] * output_scale;
            if (clipped > 6.f) clipped = 6.f;
            if (clipped < -6.f) clipped = -6.f;
            if (y) y[group * 16 + lane] = or_cast_to_e2m1(clipped) * scale;
            if (codes) {
                const uint8_t c = or_e2m1_code(clipped);
                uint8_t* byte = &codes[(group * 16 + lane) / 2];
                if (lane % 2 == 0) *byte = (uint8_t)((*byte & 0xf0u) | c);
                else *byte = (uint8_t)((*byte & 0x0fu) | (uint8_t)(c << 4));
            }
        }
    }
    return 0;
}

/* src/text_forward.cpp:552-576 */
void or_gemv_nvfp4_rows(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                        const float* x, int rows, int cols, int row0, int row1, float* y) {
    (void)rows;
    const int packed_cols = cols / 2;
    const int scale_cols = cols / 16;
    const float alpha = scale2 * input_scale;
#pragma omp parallel for schedule(static)
    for (int row = row0; row < row1; ++row) {
        const uint8_t* packed_row = packed + (size_t)row * (size_t)packed_cols;
        const uint8_t* scale_row = scales + (size_t)row * (size_t)scale_cols;
        float acc = 0.f;
        for (int group = 0; group < scale_cols; ++group) {
            const float scale = or_e4m3_to_f32(scale_row[group]);
            const uint8_t* bytes = packed_row + group * 8;
            const float* input = x + group * 16;
            for (int byte = 0; byte < 8; ++byte) {
                const uint8_t value = bytes[byte];
                acc += or_e2m1((uint8_t)(value & 0x0fu)) * scale * input[byte * 2];
                acc += or_e2m1((uint8_t)(value >> 4)) * scale * input[byte * 2 + 1];
            }
        }
        y[row] = acc * alpha;
    }
}

/* src/text_forward.cpp:497-508 */
void or_gemv_bf16(const uint16_t* weight, const float* x, int rows, int cols, int row0, int row1, float* y) {
    (void)rows;
#pragma omp parallel for schedule(static)
    for (int row = row0; row < row1; ++row) {
        const uint16_t* line = weight + (size_t)row * (size_t)cols;
        float acc = 0.f;
        for (int col = 0; col < cols; ++col) acc += or_bf16_to_f32(line[col]) * x[col];
        y[row] = acc;
    }
}

/* src/text_forward.cpp:832-856 (after the Store lookups and shape checks) */
int or_linear_nvfp4(const uint8_t* packed, const uint8_t* scales, float scale2, float input_scale,
                    const float* x, int cols, float* y, int rows) {
    float* quantized = (float*)malloc(sizeof(float) * (size_t)cols);
    if (!quantized) return -1;
    if (or_quant_nvfp4_activation(x, cols, input_scale, quantized, NULL, NULL) != 0) {
        free(quantized);
        return -1;
    }
    or_gemv_nvfp4_rows(packed, scales, scale2, input_scale, quantized, rows, cols, 0, rows, y);
    for (int row = 0; row < rows; ++row) y[row] = bf16_round(y[row]);
    free(quantized);
    return 0;
}

/* src/text_forward.cpp:1447-1471, with an optional eligibility mask that the
 * grouped extension fills (NULL = every expert eligible). */
static void router_select_masked(const float* logits, const float* bias, int experts, int top_k, float scaling,
                                 int normalize, const char* eligible, int* indices, float* weights) {
    float* choice = (float*)malloc(sizeof(float) * (size_t)experts);
    float* scores = (float*)malloc(sizeof(float) * (size_t)experts);
    char* used = (char*)calloc((size_t)experts, 1);
    for (int e = 0; e < experts; ++e) {
        scores[e] = or_sigmoid(logits[e]);
        choice[e] = scores[e] + bias[e];
        if (eligible && !eligible[e]) used[e] = 1;
    }
    for (int pick = 0; pick < top_k; ++pick) {
        int best = -1;
        for (int e = 0; e < experts; ++e) {
            if (used[e]) continue;
            if (best < 0 || choice[e] > choice[best]) best = e;
        }
        if (best < 0) best = 0; /* unreachable when top_k <= eligible experts */
        used[best] = 1;
        indices[pick] = best;
        weights[pick] = scores[best];
    }
    if (normalize) {
        float sum = 1e-20f;
        for (int pick = 0; pick < top_k; ++pick) sum += weights[pick];
        for (int pick = 0; pick < top_k; ++pick) weights[pick] = weights[pick] / sum * scaling;
    }
    free(choice);
    free(scores);
    free(used);
}

void or_router_select(const float* logits, const float* bias, int experts, int top_k, float scaling,
                      int normalize, int* indices, float* weights) {
    router_select_masked(logits, bias, experts, top_k, scaling, normalize, NULL, indices, weights);
}

void or_router_select_grouped(const float* logits, const float* bias, int experts, int top_k, float scaling,
                              int normalize, int n_group, int topk_group, int* indices, float* weights) {
    if (n_group <= 1 || topk_group >= n_group) {
        router_select_masked(logits, bias, experts, top_k, scaling, normalize, NULL, indices, weights);
        return;
    }
    const int per_group = experts / n_group;
    float* group_score = (float*)malloc(sizeof(float) * (size_t)n_group);
    char* keep = (char*)calloc((size_t)n_group, 1);
    char* eligible = (char*)calloc((size_t)experts, 1);
    for (int g = 0; g < n_group; ++g) {
        float best1 = -INFINITY, best2 = -INFINITY;
        for (int j = 0; j < per_group; ++j) {
            const int e = g * per_group + j;
            const float c = or_sigmoid(logits[e]) + bias[e];
            if (c > best1) {
                best2 = best1;
                best1 = c;
            } else if (c > best2) {
                best2 = c;
            }
        }
        group_score[g] = per_group >= 2 ? best1 + best2 : best1;
    }
    for (int r = 0; r < topk_group; ++r) {
        int best = -1;
        for (int g = 0; g < n_group; ++g) {
            if (keep[g]) continue;
            if (best < 0 || group_score[g] > group_score[best]) best = g;
        }
        keep[best] = 1;
    }
    for (int e = 0; e < experts; ++e) eligible[e] = keep[e / per_group];
    router_select_masked(logits, bias, experts, top_k, scaling, normalize, eligible, indices, weights);
    free(group_score);
    free(keep);
    free(eligible);
}

/* src/text_forward.cpp:1439-1445 */
void or_swiglu_clamp(const float* gate, const float* up, int n, float limit, float* hidden) {
    for (int i = 0; i < n; ++i) {
        const float capped_gate = (limit < gate[i]) ? limit : gate[i]; /* std::min(gate, limit) */
        const float lo = (-limit < up[i]) ? up[i] : -limit;             /* std::max(-limit, up) */
        const float capped_up = (lo < limit) ? lo : limit;              /* std::min(limit, .) */
        hidden[i] = silu(capped_gate) * capped_up;
    }
}

/* src/text_forward.cpp:99-106 */
void or_swiglu_clamp_bf16(const float* gate, const float* up, int n, float limit, float* hidden) {
    for (int i = 0; i < n; ++i) {
        const float capped_gate = bf16_round((limit < gate[i]) ? limit : gate[i]);
        const float lo = (-limit < up[i]) ? up[i] : -limit;
        const float capped_up = bf16_round((lo < limit) ? lo : limit);
        const float activated = bf16_round(silu(capped_gate));
        hidden[i] = bf16_round(activated * capped_up);
    }
}

/* src/text_forward.cpp:1646-1657 */
void or_mhc_combine(const float* residual, const float* branch, const float* post, const float* comb, int hc,
                    int hidden, float* out) {
    for (int stream = 0; stream < hc; ++stream) {
        for (int dim = 0; dim < hidden; ++dim) {
            float acc = post[stream] * branch[dim];
            for (int source = 0; source < hc; ++source) acc += comb[source * hc + stream] * residual[source * hidden + dim];
            out[stream * hidden + dim] = acc;
        }
    }
}

/* src/nvfp4_decode.cpp:56-79 (validation) and :88-97 (element value) */
int or_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales, float global_scale, int64_t rows,
                        int64_t cols, float* weight) {
    if (rows <= 0 || cols <= 0 || cols % 16 != 0) return -1;
    if (!packed || !scales || !weight) return -1;
    if (!isfinite(global_scale) || global_scale < FLT_MIN) return -1;
    const int64_t nscale = rows * (cols / 16);
    for (int64_t i = 0; i < nscale; ++i) {
        const float s = or_e4m3_to_f32(scales[i]);
        if (!isfinite(s) || s < 0.f) return -1;
        if (6.0 * (double)s * (double)global_scale > (double)FLT_MAX) return -1;
    }
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            const uint8_t byte = packed[r * (cols / 2) + c / 2];
            const uint8_t nibble = (uint8_t)(c % 2 == 0 ? (byte & 0xfu) : (byte >> 4));
            const float s = or_e4m3_to_f32(scales[r * (cols / 16) + c / 16]);
            weight[r * cols + c] = (float)((double)or_e2m1(nibble) * (double)s * (double)global_scale);
        }
    }
    return 0;
}

/* src/tiny_layer.cpp:7-12 */
void or_rmsnorm(const float* x, const float* weight, float eps, int width, float* y) {
    float square = 0.f;
    for (int i = 0; i < width; ++i) square += x[i] * x[i];
    const float scale = 1.f / sqrtf(square / (float)width + eps);
    for (int i = 0; i < width; ++i) y[i] = x[i] * scale * (weight != NULL ? weight[i] : 1.f);
}

/* src/tiny_layer.cpp:14-26 (silently returns for width > 64) */
void or_dense_residual_proj(const float* x, const float* norm_weight, const float* projection, float eps,
                            int width, float* y) {
    float normed[64];
    if (width > 64) return;
    or_rmsnorm(x, norm_weight, eps, width, normed);
    for (int row = 0; row < width; ++row) {
        float sum = 0.f;
        const float* w = projection + row * width;
        for (int col = 0; col < width; ++col) sum += w[col] * normed[col];
        y[row] = x[row] + sum;
    }
}

/* ---- the layer ------------------------------------------------------------ */

void or_router_logits(const or_moe_weights* w, const float* x, float* logits) {
    or_gemv_bf16(w->router_w, x, w->experts, w->hidden, 0, w->experts, logits);
}

/* mlp_bf16 (src/text_forward.cpp:917-922) over explicit BF16 matrices. */
static void mlp_bf16(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int hidden, int inter,
                     float limit, const float* x, float* h, float* y, float* bg, float* bu) {
    or_gemv_bf16(gate, x, inter, hidden, 0, inter, bg);
    or_gemv_bf16(up, x, inter, hidden, 0, inter, bu);
    or_swiglu_clamp(bg, bu, inter, limit, h);
    or_gemv_bf16(down, h, hidden, inter, 0, hidden, y);
}

int or_expert_forward(const or_moe_weights* w, int e, const float* x, float* h_out, float* down_out) {
    const int H = w->hidden, I = w->inter;
    float* g = (float*)malloc(sizeof(float) * (size_t)I);
    float* u = (float*)malloc(sizeof(float) * (size_t)I);
    float* h = (float*)malloc(sizeof(float) * (size_t)I);
    float* d = (float*)malloc(sizeof(float) * (size_t)H);
    int rc = 0;
    if (w->bf16_experts) {
        mlp_bf16(w->gate_bf16 + (size_t)e * I * H, w->up_bf16 + (size_t)e * I * H, w->down_bf16 + (size_t)e * H * I,
                 H, I, w->swiglu_limit, x, h, d, g, u);
    } else {
        const size_t gp = (size_t)e * I * (H / 2), gs = (size_t)e * I * (H / 16);
        const size_t dp = (size_t)e * H * (I / 2), ds = (size_t)e * H * (I / 16);
        rc |= or_linear_nvfp4(w->gate_packed + gp, w->gate_scales + gs, w->gate_ws2[e], w->gate_in[e], x, H, g, I);
        rc |= or_linear_nvfp4(w->up_packed + gp, w->up_scales + gs, w->up_ws2[e], w->up_in[e], x, H, u, I);
        or_swiglu_clamp(g, u, I, w->swiglu_limit, h);
        rc |= or_linear_nvfp4(w->down_packed + dp, w->down_scales + ds, w->down_ws2[e], w->down_in[e], h, I, d, H);
    }
    if (h_out) memcpy(h_out, h, sizeof(float) * (size_t)I);
    if (down_out) memcpy(down_out, d, sizeof(float) * (size_t)H);
    free(g);
    free(u);
    free(h);
    free(d);
    return rc ? -1 : 0;
}

/* src/text_forward.cpp:924-963 for one token, then the residual. */
static int moe_token(const or_moe_weights* w, const float* x, const float* residual, float* y, int* indices,
                     float* weights, float* routed_tap, float* shared_tap) {
    const int H = w->hidden, E = w->experts, K = w->top_k;
    const int Imax = w->inter > w->shared_inter ? w->inter : w->shared_inter;
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    float* down = (float*)malloc(sizeof(float) * (size_t)H);
    float* bg = (float*)malloc(sizeof(float) * (size_t)Imax);
    float* bu = (float*)malloc(sizeof(float) * (size_t)Imax);
    float* h = (float*)malloc(sizeof(float) * (size_t)Imax);
    int idx[64];
    float wt[64];
    int rc = 0;
    or_router_logits(w, x, logits);
    or_router_select_grouped(logits, w->router_bias, E, K, w->scaling, w->normalize, w->n_group, w->topk_group, idx,
                             wt);
    for (int d = 0; d < H; ++d) y[d] = 0.f;
    for (int p = 0; p < K; ++p) {
        if (or_expert_forward(w, idx[p], x, NULL, down) != 0) rc = -1;
        const float weight = wt[p];
        for (int d = 0; d < H; ++d) y[d] += weight * down[d];
    }
    if (routed_tap) memcpy(routed_tap, y, sizeof(float) * (size_t)H);
    if (w->shared_inter > 0) {
        mlp_bf16(w->shared_gate, w->shared_up, w->shared_down, H, w->shared_inter, w->swiglu_limit, x, h, down, bg,
                 bu);
        if (shared_tap) memcpy(shared_tap, down, sizeof(float) * (size_t)H);
        for (int d = 0; d < H; ++d) y[d] += down[d];
    } else if (shared_tap) {
        memset(shared_tap, 0, sizeof(float) * (size_t)H);
    }
    if (residual) {
        const float one = 1.f;
        float* out = (float*)malloc(sizeof(float) * (size_t)H);
        or_mhc_combine(residual, y, &one, &one, 1, H, out);
        memcpy(y, out, sizeof(float) * (size_t)H);
        free(out);
    }
    if (indices) memcpy(indices, idx, sizeof(int) * (size_t)K);
    if (weights) memcpy(weights, wt, sizeof(float) * (size_t)K);
    free(logits);
    free(down);
    free(bg);
    free(bu);
    free(h);
    return rc;
}

int or_moe_layer(const or_moe_weights* w, int tokens, const float* x, const float* residual, float* y,
                 int* indices, float* weights, float* routed, float* shared) {
    const int H = w->hidden, K = w->top_k;
    if (K > 64 || K > w->experts) return -1;
    int rc = 0;
    /* Tokens are independent; the reference steps them one by one with
     * OpenMP inside each GEMV.  Running tokens in parallel here gives the
     * same bits (every token's arithmetic is sequential and unchanged). */
#pragma omp parallel for schedule(dynamic, 1) reduction(| : rc)
    for (int t = 0; t < tokens; ++t) {
        rc |= moe_token(w, x + (size_t)t * H, residual ? residual + (size_t)t * H : NULL, y + (size_t)t * H,
                        indices ? indices + (size_t)t * K : NULL, weights ? weights + (size_t)t * K : NULL,
                        routed ? routed + (size_t)t * H : NULL, shared ? shared + (size_t)t * H : NULL);
    }
    return rc ? -1 : 0;
}

/* src/text_forward.cpp:909-915 for one token, then the residual (:906). */
static int dense_token(const or_dense_weights* w, const float* x, const float* residual, float* y, float* h_tap) {
    const int H = w->hidden, I = w->inter;
    float* g = (float*)malloc(sizeof(float) * (size_t)I);
    float* u = (float*)malloc(sizeof(float) * (size_t)I);
    float* h = (float*)malloc(sizeof(float) * (size_t)I);
    int rc = 0;
    rc |= or_linear_nvfp4(w->gate_packed, w->gate_scales, w->gate_ws2, w->gate_in, x, H, g, I);
    rc |= or_linear_nvfp4(w->up_packed, w->up_scales, w->up_ws2, w->up_in, x, H, u, I);
    or_swiglu_clamp_bf16(g, u, I, w->swiglu_limit, h);
    rc |= or_linear_nvfp4(w->down_packed, w->down_scales, w->down_ws2, w->down_in, h, I, y, H);
    if (h_tap) memcpy(h_tap, h, sizeof(float) * (size_t)I);
    if (residual) {
        const float one = 1.f;
        float* out = (float*)malloc(sizeof(float) * (size_t)H);
        or_mhc_combine(residual, y, &one, &one, 1, H, out);
        memcpy(y, out, sizeof(float) * (size_t)H);
        free(out);
    }
    free(g);
    free(u);
    free(h);
    return rc;
}

int or_dense_mlp(const or_dense_weights* w, int tokens, const float* x, const float* residual, float* y, float* h) {
    const int H = w->hidden, I = w->inter;
    int rc = 0;
    /* tokens are independent; each token's arithmetic is the reference's */
#pragma omp parallel for schedule(dynamic, 1) reduction(| : rc)
    for (int t = 0; t < tokens; ++t) {
        rc |= dense_token(w, x + (size_t)t * H, residual ? residual + (size_t)t * H : NULL, y + (size_t)t * H,
                          h ? h + (size_t)t * I : NULL);
    }
    return rc ? -1 : 0;
}

void or_route_tokens(const or_moe_weights* w, int tokens, const float* x, float* logits, int* indices,
                     float* weights) {
    const int E = w->experts, K = w->top_k, H = w->hidden;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tokens; ++t) {
        float* lg = (float*)malloc(sizeof(float) * (size_t)E);
        /* gemv_bf16 rows serially inside the token loop (same bits) */
        for (int e = 0; e < E; ++e) {
            const uint16_t* line = w->router_w + (size_t)e * H;
            const float* xt = x + (size_t)t * H;
            float acc = 0.f;
            for (int c = 0; c < H; ++c) acc += or_bf16_to_f32(line[c]) * xt[c];
            lg[e] = acc;
        }
        if (logits) memcpy(logits + (size_t)t * E, lg, sizeof(float) * (size_t)E);
        or_router_select_grouped(lg, w->router_bias, E, K, w->scaling, w->normalize, w->n_group, w->topk_group,
                                 indices + (size_t)t * K, weights + (size_t)t * K);
        free(lg);
    }
}

void or_sigmoid_array(const float* x, int64_t n, float* y) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = or_sigmoid(x[i]);
}
