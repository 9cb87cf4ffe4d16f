// nf_gemm_shared.cuh -- device helpers shared by the 1-SM (nf_gemm.cu) and
// the CTA-pair (nf_gemm2.cu) tcgen05 GEMMs: the epilogues' SwiGLU forms and
// the bounded waits.
#pragma once

#include "nf_common.cuh"

namespace nf {

// swiglu_clamp element (src/text_forward.cpp:1439-1445): min(g, L) into SiLU,
// up clamped to [-L, L] with std::min / std::max semantics, with a fast SiLU
// (x / (1 + e^-x), hardware exp2 and divide).  Used
// where the result feeds a 4-bit quantiser or a BF16 store, so agreement to
// a few ulp with the reference's libm SiLU is all that matters.
__device__ __forceinline__ float swiglu_fast(float g, float u, float L) {
    const float cg = (L < g) ? L : g;
    const float lo = (-L < u) ? u : -L;
    const float cu = (lo < L) ? lo : L;
    return __fmul_rn(__fdividef(cg, 1.f + __expf(-cg)), cu);
}

// swiglu_clamp_bf16 element (src/text_forward.cpp:99-106), the dense layers'
// form: the capped gate, the clamped up, SiLU of the capped gate and the
// product are each rounded to BF16 (the same clamps and SiLU as swiglu_fast).
__device__ __forceinline__ float swiglu_bf16_fast(float g, float u, float L) {
    const float cg = bf16_round_hw((L < g) ? L : g);
    const float lo = (-L < u) ? u : -L;
    const float cu = bf16_round_hw((lo < L) ? lo : L);
    const float act = bf16_round_hw(__fdividef(cg, 1.f + __expf(-cg)));
    return bf16_round_hw(__fmul_rn(act, cu));
}

// ---------------------------------------------------------------------------
// The gate/up epilogue's arithmetic with fewer instructions (the NVFP4
// gate/up GEMM at prefill sizes is bound by its epilogue's issue rate):
// packed fp32x2 multiplies (sm_100 mul.rn.f32x2, the same rounding as two
// separate multiplies), single-instruction clamps with the reference's NaN
// behaviour, and a quantiser that finds the group's peak with a packed
// integer max over the BF16 bit patterns, divides by 6 with an FMA
// correction and looks the output scale up per expert.  Results are bit
// identical to swiglu_fast / quantize_group16_fast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
    return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f32x2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f32x2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// min(g, L) with NaN g giving NaN: (L < g) ? L : g (std::min(g, L)) for any non-NaN L
__device__ __forceinline__ float min_nan(float a, float b) {
    float d;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// swiglu_clamp on two elements (as swiglu_fast): min(g, L) into SiLU, up
// clamped to [-L, L] -- fmaxf(u, -L) is (-L < u) ? u : -L also for a NaN u,
// and fminf of a non-NaN value with L is (lo < L) ? lo : L.
__device__ __forceinline__ uint64_t swiglu_fast2(float g0, float g1, float u0, float u1, float L) {
    const float cg0 = min_nan(g0, L), cg1 = min_nan(g1, L);
    const float cu0 = fminf(fmaxf(u0, -L), L), cu1 = fminf(fmaxf(u1, -L), L);
    const float s0 = __fdividef(cg0, 1.f + __expf(-cg0)), s1 = __fdividef(cg1, 1.f + __expf(-cg1));
    return mul_f32x2(f32x2_pack(s0, s1), f32x2_pack(cu0, cu1));
}

// RN(p / 6) for a finite non-negative BF16 value p by Markstein's FMA
// correction of the product with RN(1/6) (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", 1990): equal
// to the correctly rounded quotient for every such p (checked exhaustively,
// tests/test_fast_quant.py).
__device__ __forceinline__ float div6_rn(float p) {
    const float r6 = 0.16666667163372039794921875f;  // RN(1/6)
    const float q = __fmul_rn(p, r6);
    const float r = __fmaf_rn(-q, 6.f, p);
    return __fmaf_rn(r, r6, q);
}

// quantize_group16_fast<false> with the output scale from os_tab[scale code]
// (a table of 1 / (scale / gs) per code, as quantize_group16 computes it, for
// this expert's gs).  Groups holding an infinity or a NaN take the
// reference-rule path.
__device__ __forceinline__ uint32_t quantize_group16_tab(const float (&x)[16], float global_scale,
                                                         const float* __restrict__ os_tab, uint32_t (&codes)[2]) {
    uint32_t w[8];
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w[i] = bf16x2_hw(x[2 * i], x[2 * i + 1]);
        m = __vmaxu2(m, w[i] & 0x7fff7fffu);
    }
    const uint32_t pb = max(m & 0xffffu, m >> 16);
    if (pb >= 0x7f80u) return quantize_group16_cold(x, global_scale, codes);
    float scale = __fmul_rn(global_scale, div6_rn(__uint_as_float(pb << 16)));
    scale = scale > 448.f ? 448.f : scale;
    const uint32_t scode = scale >= 0.015625f ? e4m3_hw(scale) : f32_to_e4m3(scale);
    const float os = __ldg(os_tab + scode);
    const uint64_t os2 = f32x2_pack(os, os);
    uint32_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint64_t pr = mul_f32x2(f32x2_pack(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u)), os2);
        b[i] = e2m1x2_hw(f32x2_lo(pr), f32x2_hi(pr));
    }
    codes[0] = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
    codes[1] = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
    return scode;
}

// One 16-output group of the NVFP4 gate/up epilogue: accumulators vg / vu
// (16 gate and 16 up columns), alpha multiply and BF16 rounding
// (linear_nvfp4's output, src/text_forward.cpp:852-855), swiglu_clamp (or
// swiglu_clamp_bf16 for the dense layers), then the NVFP4 quantiser of the
// down projection's input.
__device__ __forceinline__ uint32_t swiglu_quant_group(const uint32_t* vg, const uint32_t* vu, float ag, float au,
                                                       float gsd, float L, bool sbf, const float* __restrict__ os_tab,
                                                       uint32_t (&cc)[2]) {
    float h[16];
    const uint64_t ag2 = f32x2_pack(ag, ag), au2 = f32x2_pack(au, au);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const uint64_t gg = mul_f32x2(f32x2_pack(__uint_as_float(vg[j]), __uint_as_float(vg[j + 1])), ag2);
        const uint64_t uu = mul_f32x2(f32x2_pack(__uint_as_float(vu[j]), __uint_as_float(vu[j + 1])), au2);
        const uint32_t g2 = bf16x2_hw(f32x2_lo(gg), f32x2_hi(gg));
        const uint32_t u2 = bf16x2_hw(f32x2_lo(uu), f32x2_hi(uu));
        const float g0 = __uint_as_float(g2 << 16), g1 = __uint_as_float(g2 & 0xffff0000u);
        const float u0 = __uint_as_float(u2 << 16), u1 = __uint_as_float(u2 & 0xffff0000u);
        if (sbf) {
            h[j] = swiglu_bf16_fast(g0, u0, L);
            h[j + 1] = swiglu_bf16_fast(g1, u1, L);
        } else {
            const uint64_t hh = swiglu_fast2(g0, g1, u0, u1, L);
            h[j] = f32x2_lo(hh);
            h[j + 1] = f32x2_hi(hh);
        }
    }
    return os_tab ? quantize_group16_tab(h, gsd, os_tab, cc) : quantize_group16_fast<false>(h, gsd, cc);
}

// Bounded wait, by every lane of the calling warp, until *counter >= target
// (acquire); false once the budget runs out or the CTA or kernel gave up.
__device__ __forceinline__ bool wait_count(const int* counter, int target, volatile int* cta_abort,
                                           volatile int* dev_err) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
        if (v >= target) return true;
        if (*cta_abort != 0 || *dev_err != 0 || globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) return false;
        __nanosleep(64);
    }
}

__device__ __forceinline__ void set_abort(volatile int* cta_abort, int* dev_err, int code) {
    *cta_abort = 1;
    atomicCAS(dev_err, 0, code);
}

}  // namespace nf
