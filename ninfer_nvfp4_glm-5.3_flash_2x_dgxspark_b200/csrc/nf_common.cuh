// nf_common.cuh -- shared device code for the sm_100a MoE kernels:
// number-format helpers that reproduce the reference's host rounding
// bit for bit, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define NF_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// Error word shared by every kernel: a device-side bounded wait that gives up
// records a code here and the host turns it into NF_ERR_TIMEOUT.
// ---------------------------------------------------------------------------
enum : int {
    NF_DEVERR_NONE = 0,
    NF_DEVERR_WAIT_FULL = 1,    // consumer waited too long for a TMA stage
    NF_DEVERR_WAIT_EMPTY = 2,   // producer waited too long for a free stage
    NF_DEVERR_WAIT_ACC = 3,     // MMA / epilogue accumulator hand-off timed out
    NF_DEVERR_DRAIN = 4,        // teardown drain after an abort timed out
    NF_DEVERR_EP_WAIT = 5,      // an expert-parallel peer's rows or outputs never arrived
    NF_DEVERR_BAD_TOKEN = 6     // a token id outside the vocabulary, or a position outside the cache
};

// One second of %globaltimer (ns) per wait; the longest kernel here runs
// well under a millisecond.
#define NF_WAIT_BUDGET_NS 1000000000ull

NF_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Number formats (reference host semantics)
// ---------------------------------------------------------------------------

// f32 -> bf16 -> f32 with the reference's rounding (src/text_forward.cpp:87-95):
// round to nearest even, NaN keeps its top 16 bits.
NF_DEV float bf16_round(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(b & 0xffff0000u);
    b += 0x7fffu + ((b >> 16) & 1u);
    return __uint_as_float(b & 0xffff0000u);
}
NF_DEV float bf16_bits_to_f32(uint16_t bits) { return __uint_as_float(static_cast<uint32_t>(bits) << 16); }

// f32 -> bf16 -> f32 by the hardware conversion (round to nearest even).
// Same as bf16_round for every non-NaN input (checked over all 2^32 inputs
// by nf_format_selfcheck); NaN inputs give the canonical NaN.
NF_DEV float bf16_round_hw(float v) {
    uint16_t b;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(b) : "f"(v));
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
// Two values at once, packed (low half = `lo`).
NF_DEV uint32_t bf16x2_hw(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
NF_DEV uint16_t f32_to_bf16_bits(float v) { return static_cast<uint16_t>(__float_as_uint(bf16_round(v)) >> 16); }

// E4M3FN decode (src/nvfp4_decode.cpp:42-54); exact.
NF_DEV float e4m3_to_f32(uint32_t bits) {
    const int exponent = (bits >> 3) & 0xf;
    const int mantissa = bits & 0x7;
    float magnitude;
    if (exponent == 0) magnitude = ldexpf(static_cast<float>(mantissa), -9);
    else if (exponent == 15 && mantissa == 7) magnitude = __uint_as_float(0x7fc00000u);
    else magnitude = ldexpf(1.f + static_cast<float>(mantissa) * 0.125f, exponent - 7);
    return (bits & 0x80u) ? -magnitude : magnitude;
}

// E4M3FN encode with the reference's rules (src/text_forward.cpp:60-85):
// normal band rounds the 3-bit mantissa to nearest even (rintf), saturates
// at 0x7e; the subnormal band rounds v*2^9 and caps the code at 7.
NF_DEV uint32_t f32_to_e4m3(float value) {
    if (isnan(value)) return 0x7fu;
    const uint32_t sign = signbit(value) ? 0x80u : 0u;
    float magnitude = fabsf(value);
    if (magnitude == 0.f) return sign;
    if (magnitude > 448.f) magnitude = 448.f;
    int exponent = 0;
    const float fraction = frexpf(magnitude, &exponent);
    const float normal = fraction * 2.f;
    int biased = exponent - 1 + 7;
    if (biased <= 0) {
        int mantissa = static_cast<int>(rintf(ldexpf(magnitude, 9)));
        mantissa = mantissa > 7 ? 7 : (mantissa < 0 ? 0 : mantissa);
        return sign | static_cast<uint32_t>(mantissa);
    }
    if (biased > 15) return sign | 0x7eu;
    int mantissa = static_cast<int>(rintf((normal - 1.f) * 8.f));
    if (mantissa == 8) {
        mantissa = 0;
        ++biased;
        if (biased > 15) return sign | 0x7eu;
    }
    if (biased >= 15 && mantissa > 6) return sign | 0x7eu;
    return sign | (static_cast<uint32_t>(biased) << 3) | static_cast<uint32_t>(mantissa);
}

// E2M1 magnitude of a code's low 3 bits.
NF_DEV float e2m1_mag(uint32_t code) {
    const float t[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    return t[code & 7u];
}

// cast_to_e2m1 (src/text_forward.cpp:510-522) returning the 4-bit code
// (sign in bit 3; the sign is copysign(1, v), so -0.1 gives code 8).
NF_DEV uint32_t e2m1_code(float v) {
    const float m = fabsf(v);
    uint32_t c = 7u;  // beyond 5 and NaN snap to 6
    if (m <= 0.25f) c = 0u;
    else if (m < 0.75f) c = 1u;
    else if (m <= 1.25f) c = 2u;
    else if (m < 1.75f) c = 3u;
    else if (m <= 2.5f) c = 4u;
    else if (m < 3.5f) c = 5u;
    else if (m <= 5.f) c = 6u;
    return c | (signbit(v) ? 8u : 0u);
}

// Quantises one group of 16 values exactly like one iteration of
// quant_dequant_nvfp4_activation (src/text_forward.cpp:531-549).
// Returns the E4M3 scale code; codes[0..1] receive the 16 packed nibbles
// (low nibble = even element).  `global_scale` is 1/input_scale as the
// reference computes it (one fp32 division on the host).
NF_DEV uint32_t quantize_group16(const float (&x)[16], float global_scale, uint32_t (&codes)[2]) {
    float r[16];
    float peak = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        r[i] = bf16_round(x[i]);
        const float a = fabsf(r[i]);
        peak = (peak < a) ? a : peak;  // std::max(peak, a): NaN never wins
    }
    float scale = __fmul_rn(global_scale, __fdiv_rn(peak, 6.f));
    scale = scale > 448.f ? 448.f : scale;
    const uint32_t scode = f32_to_e4m3(scale);
    scale = e4m3_to_f32(scode);
    const float reduced = __fdiv_rn(scale, global_scale);
    const float output_scale = __fdiv_rn(1.f, __fadd_rn(reduced, reduced == 0.f ? 1.0e8f : 0.f));
    codes[0] = codes[1] = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float clipped = __fmul_rn(r[i], output_scale);
        clipped = clipped > 6.f ? 6.f : clipped;
        clipped = clipped < -6.f ? -6.f : clipped;
        codes[i >> 3] |= e2m1_code(clipped) << (4 * (i & 7));
    }
    return scode;
}

// Two E2M1 codes from the hardware conversion (round to nearest even on the
// E2M1 grid, saturating at +-6): low nibble = `even`, high nibble = `odd`.
// On finite inputs this is cast_to_e2m1 (the reference's ties -- 0.25, 2.5
// and 5 down, 0.75, 1.25, 1.75 and 3.5 up -- are exactly round-half-even on
// that grid); NaN is not handled here.
NF_DEV uint32_t e2m1x2_hw(float even, float odd) {
    uint16_t r;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}"
        : "=h"(r)
        : "f"(odd), "f"(even));
    return r;
}

// E4M3 code from the hardware conversion (round to nearest even, saturating
// at 448).  Matches f32_to_e4m3 for v in [2^-6, inf); below 2^-6 the
// reference's subnormal rule differs, so callers route that band elsewhere.
NF_DEV uint32_t e4m3_hw(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(v));
    return r & 0xffu;
}

// Out-of-line copy of quantize_group16 for the rare NaN groups, so the
// common path keeps its registers.
static __device__ __noinline__ uint32_t quantize_group16_cold(const float (&x)[16], float global_scale, uint32_t (&codes)[2]) {
    return quantize_group16(x, global_scale, codes);
}

// quantize_group16 with the hardware conversions: identical results (NaN
// groups and scales below 2^-6 take the reference-rule path).  kBf16Input:
// the inputs are BF16 values already, so the BF16 rounding is skipped.
template <bool kBf16Input>
NF_DEV uint32_t quantize_group16_fast(const float (&x)[16], float global_scale, uint32_t (&codes)[2]) {
    float r[16];
    float peak = 0.f;
    bool nan = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        // the hardware rounding equals bf16_round for every non-NaN input,
        // and a NaN sends the whole group to the reference-rule path
        r[i] = kBf16Input ? x[i] : bf16_round_hw(x[i]);
        nan |= isnan(r[i]);
        const float a = fabsf(r[i]);
        peak = (peak < a) ? a : peak;
    }
    if (nan) return quantize_group16_cold(x, global_scale, codes);
    float scale = __fmul_rn(global_scale, __fdiv_rn(peak, 6.f));
    scale = scale > 448.f ? 448.f : scale;
    const uint32_t scode = scale >= 0.015625f ? e4m3_hw(scale) : f32_to_e4m3(scale);
    scale = e4m3_to_f32(scode);
    const float reduced = __fdiv_rn(scale, global_scale);
    const float output_scale = __fdiv_rn(1.f, __fadd_rn(reduced, reduced == 0.f ? 1.0e8f : 0.f));
    uint32_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = e2m1x2_hw(__fmul_rn(r[2 * i], output_scale), __fmul_rn(r[2 * i + 1], output_scale));
    codes[0] = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
    codes[1] = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
    return scode;
}

// Offset of block scale (row, kgroup) inside the tcgen05 scale-factor atom
// layout: 128 rows x 4 scales per 512-byte atom, atoms ordered row-block
// major then K-block; inside an atom byte (row % 32) * 16 + ((row % 128) / 32)
// * 4 + kgroup % 4.  This is the layout tcgen05.cp.32x128b.warpx4 expects.
__host__ __device__ __forceinline__ int64_t sf_atom_offset(int64_t row, int64_t kgroup, int64_t kgroups_total) {
    const int64_t atom = (row >> 7) * (kgroups_total >> 2) + (kgroup >> 2);
    return atom * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (kgroup & 3);
}

// ---------------------------------------------------------------------------
// Shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------
NF_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

NF_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
NF_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
NF_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Orders this thread's generic-proxy global accesses with async-proxy (TMA)
// ones: global data written by st.global in one CTA and read by TMA in another.
NF_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
NF_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Adds `bytes` to the current phase's expected transaction count without
// arriving (the arrivals come separately).
NF_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
NF_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
NF_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread until the phase completes, for at
// most `hint_ns` (the hardware wakes it earlier when the phase completes),
// so a waiting warp does not spin on issue slots the working warps need.
NF_DEV bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity`.  Gives up (returns false) when
// the budget runs out or when another role of the CTA (abort flag in shared
// memory) or another CTA (error word in global memory) has given up.
NF_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* cta_abort, volatile int* dev_err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (*cta_abort != 0 || *dev_err != 0) return false;
        if (globaltimer_ns() - start > NF_WAIT_BUDGET_NS) return false;
    }
}

// Named barrier over `threads` threads (a multiple of 32) with id `id` (1-15;
// id 0 is __syncthreads).
NF_DEV void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor maps, no cluster distribution) and 1-D bulk copies
// ---------------------------------------------------------------------------
NF_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// One 32-byte global store (a whole sector per thread; `p` 32-byte aligned):
// the epilogues write each thread's row segment with these rather than with
// 16-byte stores, which leave every sector half written per instruction.
NF_DEV void st_global_v8(void* p, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t a4, uint32_t a5,
                         uint32_t a6, uint32_t a7) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a0), "r"(a1), "r"(a2),
                 "r"(a3), "r"(a4), "r"(a5), "r"(a6), "r"(a7)
                 : "memory");
}
// A 3-D tiled TMA load (x, y, z) into this CTA's shared memory.
NF_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
NF_DEV void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z,
                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
        : "memory");
}
NF_DEV void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// The same copies with an L2 cache-policy operand (l2_evict_first()): the
// expert weights stream through once per layer step, several times the
// 126 MB L2, and would otherwise evict the small working set that the
// latency-bound kernels re-read every step (router weights, tile lists,
// activations, kernel code).
NF_DEV uint64_t l2_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}
NF_DEV void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
NF_DEV void bulk_load_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// System-scope release store / acquire load (flags between GPUs of an
// expert-parallel group, in peer memory).
NF_DEV void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
NF_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
NF_DEV void prefetch_l2_bulk(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
NF_DEV void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with
// launch_dependent() may start while the kernel before it in the stream is
// still running: pdl_wait() returns once that kernel has completed and its
// writes are visible, so every read of its results (and every write it might
// still read) comes after pdl_wait().  pdl_trigger() lets the next kernel
// launch; each kernel of the layer calls it only after its own pdl_wait(), so
// whatever ran two or more launches earlier has completed when a kernel
// starts.  Both are no-ops for a kernel launched the ordinary way.
// ---------------------------------------------------------------------------
NF_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
NF_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, copies, loads
// ---------------------------------------------------------------------------
NF_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
NF_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
NF_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
NF_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrives once on `bar` when every tcgen05 operation this thread issued so
// far has completed.
NF_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T with E2M1 operands and UE4M3 scales per
// 16 K-elements taken from TMEM; K = 64 per instruction.
NF_DEV void mma_nvfp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa_tmem,
                      uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T with BF16 operands; K = 16 per instruction.
NF_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Copies a 32-row x 16-byte block from shared memory into 4 TMEM columns of
// every lane quadrant (the scale-factor atom form).
NF_DEV void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns.
NF_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
NF_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes, 8-row swizzle atoms 1024 bytes apart (SBO), version 1 (sm_100).
NF_DEV uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3fffu);
    d |= static_cast<uint64_t>(1u) << 16;            // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO
    d |= static_cast<uint64_t>(1u) << 46;            // descriptor version
    d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
    return d;
}
// Descriptor of one 512-byte scale-factor atom: 32 rows of 16 bytes,
// no swizzle, 8-row core matrices 128 bytes apart.
NF_DEV uint64_t sdesc_sf_atom(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3fffu);
    d |= static_cast<uint64_t>(128u >> 4) << 16;     // LBO
    d |= static_cast<uint64_t>(128u >> 4) << 32;     // SBO
    d |= static_cast<uint64_t>(1u) << 46;
    return d;
}

// Instruction descriptors (the 32-bit form the PTX takes).
// kind::mxf4nvf4: A/B E2M1 (format 1), UE4M3 scales, K-major, M, N.
__host__ __device__ constexpr uint32_t idesc_nvfp4(int M, int N) {
    return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
// kind::f16: F32 accumulate, A/B BF16, K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// CTA pairs (clusters of 2) for the 2-SM tcgen05 GEMM (nf_gemm2.cu)
// ---------------------------------------------------------------------------
NF_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the same shared-memory location in CTA
// `rank` of the cluster.
NF_DEV uint32_t smem_in_cta(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrives once on an mbarrier given by its shared::cluster address (possibly
// in the other CTA of the pair), release at cluster scope.
NF_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Whole-cluster barrier (every thread of both CTAs).
// try_wait with cluster-scope acquire, for barriers whose arrivals come from
// the other CTA of the pair.
NF_DEV bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
NF_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* cta_abort, volatile int* dev_err) {
    const uint64_t start = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*cta_abort != 0 || *dev_err != 0) return false;
        if (globaltimer_ns() - start > NF_WAIT_BUDGET_NS) return false;
        __nanosleep(32);
    }
}
NF_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A 2-D TMA tile load whose completion is counted on an mbarrier of either
// CTA of the pair (given by its shared::cluster address): each CTA loads its
// own operand halves into its own shared memory, and both report to the
// leader's barrier.
NF_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x, int32_t y,
                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
NF_DEV void tma_load_2d_pair_nohint(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x,
                                    int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
NF_DEV void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {  // one warp of each CTA
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
NF_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {  // one warp of each CTA
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives once on an mbarrier of either CTA of the pair (its shared::cluster
// address) when every cta_group::2 tcgen05 operation this thread issued so
// far has completed.
NF_DEV void tc_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}
// As tc_commit_pair, arriving on the mbarrier at the same shared-memory offset
// in both CTAs of the pair with one instruction (a commit, not a load).
NF_DEV void tc_commit_pair_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}
// D (M = 256 over the pair) (+)= A * B^T, E2M1 operands, UE4M3 scales per 16.
NF_DEV void mma_nvfp4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa_tmem,
                           uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}
// A 32-row x 16-byte scale-factor block from each CTA's shared memory (the
// same offset) into 4 TMEM columns of every lane quadrant of that CTA.
NF_DEV void tmem_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// ---------------------------------------------------------------------------
// Warp-level BF16 tensor-core tiles (mma.sync m16n8k16 with ldmatrix): the
// decode attention and the prefill router's screen, whose tiles (an 8-head
// GQA group, 16 tokens x the experts) are too small for tcgen05's 64/128-row
// tiles.
// ---------------------------------------------------------------------------
NF_DEV uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
NF_DEV void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
NF_DEV void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// d = a (16 x 16, row) * b (16 x 8, col) + d, BF16 in, F32 accumulate
NF_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                      uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
