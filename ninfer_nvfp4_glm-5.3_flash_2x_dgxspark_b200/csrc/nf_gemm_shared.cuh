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
