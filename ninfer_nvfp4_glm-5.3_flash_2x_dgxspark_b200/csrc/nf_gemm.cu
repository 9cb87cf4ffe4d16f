// nf_gemm.cu -- persistent tcgen05 GEMM for the MoE layer on sm_100a.
//
// One kernel template serves every contraction of the layer:
//   KIND_NVFP4 : tcgen05.mma kind::mxf4nvf4 block16 -- E2M1 A and B with UE4M3
//                scales per 16 K-elements (NVFP4), FP32 accumulation in TMEM;
//   KIND_BF16  : tcgen05.mma kind::f16 with BF16 A and B (shared expert and
//                the BF16 layer-45 experts).
// Tile: 128 rows of A (permuted token rows of one expert, or dense token
// rows) x 256 rows of B (for gate/up: 128 gate rows followed by the 128 up
// rows of the same intermediate block, interleaved at bind time, so the
// epilogue sees gate and up of one output column in one thread).
// Pipeline: 4 shared-memory stages of 128-byte K slices (256 FP4 or 64 BF16
// elements) loaded by TMA with 128-byte swizzle; block-scale atoms arrive by
// 1-D bulk copy and move to TMEM with tcgen05.cp; one elected thread issues
// the MMAs and commits stage release / accumulator-ready to mbarriers.
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-5 epilogue (TMEM lane quadrant = warp % 4).
// The persistent grid walks a device-side tile list, so the launch needs no
// host synchronisation after routing.
// Every wait is bounded (nf_common.cuh mbar_wait); on a timeout the kernel
// records an error code, stops every role, drains and frees TMEM.
#include "nf_common.cuh"
#include "nf_internal.h"

#include <mutex>

namespace nf {

constexpr int BM = 128, BN = 256, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * 128;
constexpr int B_STAGE_BYTES = BN * 128;
constexpr int SFA_STAGE_BYTES = 4 * 512;   // [k-step][512]
constexpr int SFB_STAGE_BYTES = 8 * 512;   // [b-block][k-step][512]
constexpr int TMEM_COLS = 512;
constexpr int ACC_COLS = 256;
constexpr int SF_COLS = 48;                // per stage: 16 for A, 32 for B
constexpr int SMEM_TILES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES + SFA_STAGE_BYTES + SFB_STAGE_BYTES);
constexpr int SMEM_BYTES = 1024 + SMEM_TILES + 256;

struct TileInfo {
    int expert, row0, n_block, m_valid;
};

__device__ __forceinline__ TileInfo get_tile(const GemmArgs& a, int i) {
    TileInfo t;
    if (a.dense_rows > 0) {
        const int m_tiles = (a.dense_rows + BM - 1) / BM;
        const int n = i / m_tiles, m = i % m_tiles;
        t.expert = 0;
        t.row0 = m * BM;
        t.n_block = n;
        t.m_valid = min(BM, a.dense_rows - m * BM);
    } else {
        const NfTile x = a.tiles[i];
        t.expert = x.expert;
        t.row0 = x.row0;
        t.n_block = x.n_block;
        t.m_valid = x.m_valid;
    }
    return t;
}

// Reference sigmoid / SiLU shape (src/text_forward.cpp:42-51) with the CUDA
// expf; the SwiGLU output feeds a 4-bit quantiser, so the last-bit agreement
// the router needs is not required here.
__device__ __forceinline__ float silu_dev(float x) {
    float s;
    if (x >= 0.f) s = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x)));
    else {
        const float z = expf(x);
        s = __fdiv_rn(z, __fadd_rn(1.f, z));
    }
    return __fmul_rn(x, s);
}

// swiglu_clamp element (src/text_forward.cpp:1439-1445): min(g, L) into SiLU,
// up clamped to [-L, L] with std::min/std::max semantics.
__device__ __forceinline__ float swiglu_dev(float g, float u, float L) {
    const float cg = (L < g) ? L : g;
    const float lo = (-L < u) ? u : -L;
    const float cu = (lo < L) ? lo : L;
    return __fmul_rn(silu_dev(cg), cu);
}

__device__ __forceinline__ void set_abort(volatile int* cta_abort, int* dev_err, int code) {
    *cta_abort = 1;
    atomicCAS(dev_err, 0, code);
}

template <int KIND, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, const GemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * A_STAGE_BYTES;
    uint8_t* sSFA = sB + STAGES * B_STAGE_BYTES;
    uint8_t* sSFB = sSFA + STAGES * SFA_STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * SFB_STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* drain = acc_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* dev_err = args.err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        mbar_init(drain, 1);
        *cta_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tma);
        prefetch_tensormap(&tmb);
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int num_tiles = args.dense_rows > 0 ? ((args.dense_rows + BM - 1) / BM) * args.n_blocks : *args.num_tiles_dev;
    const int K = args.K;
    constexpr int kElemsPerStage = KIND == KIND_NVFP4 ? 256 : 64;
    constexpr int kMmaK = KIND == KIND_NVFP4 ? 64 : 16;
    const int k_tiles = (K + kElemsPerStage - 1) / kElemsPerStage;
    const int sf_atoms_per_rowblock = K / 64;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_parity[STAGES];
            bool issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && i < num_tiles; i += gridDim.x) {
                const TileInfo t = get_tile(args, i);
                const int brow0 = t.expert * args.b_rows_per_expert + t.n_block * BN;
                for (int kt = 0; kt < k_tiles; ++kt) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_EMPTY);
                        ok = false;
                        break;
                    }
                    const int k0 = kt * kElemsPerStage;
                    const int steps = min(4, (K - k0) / kMmaK);
                    uint32_t bytes = A_STAGE_BYTES + B_STAGE_BYTES;
                    if (KIND == KIND_NVFP4) bytes += static_cast<uint32_t>(steps) * 512u * 3u;
                    mbar_arrive_expect_tx(&full[stage], bytes);
                    const int xc = KIND == KIND_NVFP4 ? kt * 128 : k0;
                    tma_load_2d(sA + stage * A_STAGE_BYTES, &tma, &full[stage], xc, t.row0);
                    tma_load_2d(sB + stage * B_STAGE_BYTES, &tmb, &full[stage], xc, brow0);
                    if (KIND == KIND_NVFP4) {
                        const int64_t a_atom = static_cast<int64_t>(t.row0 / 128) * sf_atoms_per_rowblock + kt * 4;
                        bulk_load(sSFA + stage * SFA_STAGE_BYTES, args.sfa + a_atom * 512, steps * 512u, &full[stage]);
#pragma unroll
                        for (int b = 0; b < 2; ++b) {
                            const int64_t b_atom =
                                static_cast<int64_t>(brow0 / 128 + b) * sf_atoms_per_rowblock + kt * 4;
                            bulk_load(sSFB + stage * SFB_STAGE_BYTES + b * 2048, args.sfb + b_atom * 512,
                                      steps * 512u, &full[stage]);
                        }
                    }
                    issued[stage] = true;
                    issued_parity[stage] = phase;
                    if (++stage == STAGES) stage = 0, phase ^= 1u;
                }
            }
            if (!ok) {
                // drain: every issued copy lands before the CTA may exit
                for (int s = 0; s < STAGES; ++s) {
                    if (!issued[s]) continue;
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(&full[s], issued_parity[s])) {
                        if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) {
                            atomicCAS(args.err, 0, NF_DEVERR_DRAIN);
                            break;
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, acc_phase = 0;
            const uint32_t idesc = KIND == KIND_NVFP4 ? idesc_nvfp4(BM, BN) : idesc_bf16(BM, BN);
            bool ok = true;
            for (int i = blockIdx.x; ok && i < num_tiles; i += gridDim.x) {
                if (!mbar_wait(acc_empty, acc_phase ^ 1u, cta_abort, dev_err)) {
                    set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kt = 0; kt < k_tiles; ++kt) {
                    if (!mbar_wait(&full[stage], phase, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int k0 = kt * kElemsPerStage;
                    const int steps = min(4, (K - k0) / kMmaK);
                    const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
                    const uint32_t sfa_col = ACC_COLS + stage * SF_COLS;
                    const uint32_t sfb_col = sfa_col + 16;
                    if (KIND == KIND_NVFP4) {
                        for (int s = 0; s < steps; ++s) {
                            tmem_cp_sf(tmem + sfa_col + 4 * s, sdesc_sf_atom(smem_u32(sSFA + stage * SFA_STAGE_BYTES + s * 512)));
                            tmem_cp_sf(tmem + sfb_col + 8 * s,
                                       sdesc_sf_atom(smem_u32(sSFB + stage * SFB_STAGE_BYTES + s * 512)));
                            tmem_cp_sf(tmem + sfb_col + 8 * s + 4,
                                       sdesc_sf_atom(smem_u32(sSFB + stage * SFB_STAGE_BYTES + 2048 + s * 512)));
                        }
                    }
                    for (int s = 0; s < steps; ++s) {
                        const uint64_t adesc = sdesc_sw128(a_base + 32 * s);
                        const uint64_t bdesc = sdesc_sw128(b_base + 32 * s);
                        const uint32_t acc = (kt > 0 || s > 0) ? 1u : 0u;
                        if (KIND == KIND_NVFP4)
                            mma_nvfp4(tmem, adesc, bdesc, idesc, tmem + sfa_col + 4 * s, tmem + sfb_col + 8 * s, acc);
                        else
                            mma_bf16(tmem, adesc, bdesc, idesc, acc);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) stage = 0, phase ^= 1u;
                }
                if (!ok) break;
                tc_commit(acc_full);
                acc_phase ^= 1u;
            }
            if (!ok) {
                // drain: wait for every MMA / copy this thread issued
                tc_commit(drain);
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(drain, 0)) {
                    if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) {
                        atomicCAS(args.err, 0, NF_DEVERR_DRAIN);
                        break;
                    }
                }
            }
        }
    } else {
        // ------------------------------ epilogue ----------------------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int r = q * 32 + lane;
        const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
        uint32_t acc_phase = 0;
        for (int i = blockIdx.x; i < num_tiles; i += gridDim.x) {
            const TileInfo t = get_tile(args, i);
            int ok = 1;
            if (lane == 0) ok = mbar_wait(acc_full, acc_phase, cta_abort, dev_err) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                break;
            }
            tc_fence_after();
            const int row = t.row0 + r;
            const bool valid = r < t.m_valid;
            if (EPI == EPI_SWIGLU_QUANT) {
                const float ag = args.alpha0[t.expert], au = args.alpha1[t.expert];
                const float gsd = args.gscale_next[t.expert], L = args.limit;
                uint32_t codes[16];
                uint32_t sfw0 = 0u, sfw1 = 0u;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t g[16], u[16];
                    tmem_ld16(tbase + 16 * c, g);
                    tmem_ld16(tbase + 128 + 16 * c, u);
                    tmem_wait_ld();
                    float h[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float gv = bf16_round(__fmul_rn(__uint_as_float(g[j]), ag));
                        const float uv = bf16_round(__fmul_rn(__uint_as_float(u[j]), au));
                        h[j] = swiglu_dev(gv, uv, L);
                    }
                    uint32_t cc[2];
                    const uint32_t sc = quantize_group16(h, gsd, cc);
                    codes[2 * c] = cc[0];
                    codes[2 * c + 1] = cc[1];
                    if (c < 4) sfw0 |= sc << (8 * c);
                    else sfw1 |= sc << (8 * (c - 4));
                }
                if (valid) {
                    uint8_t* o = static_cast<uint8_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld + t.n_block * 64;
                    uint4* d = reinterpret_cast<uint4*>(o);
                    d[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
                    d[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
                    d[2] = make_uint4(codes[8], codes[9], codes[10], codes[11]);
                    d[3] = make_uint4(codes[12], codes[13], codes[14], codes[15]);
                    *reinterpret_cast<uint32_t*>(args.out_sf + sf_atom_offset(row, t.n_block * 8, args.out_kgroups)) = sfw0;
                    *reinterpret_cast<uint32_t*>(args.out_sf + sf_atom_offset(row, t.n_block * 8 + 4, args.out_kgroups)) = sfw1;
                }
            } else if (EPI == EPI_STORE_BF16) {
                const float a = args.alpha0[t.expert];
#pragma unroll 1
                for (int c = 0; c < 16; ++c) {
                    uint32_t v[16];
                    tmem_ld16(tbase + 16 * c, v);
                    tmem_wait_ld();
                    uint32_t p[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t lo = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[2 * j]), a));
                        const uint32_t hi = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[2 * j + 1]), a));
                        p[j] = lo | (hi << 16);
                    }
                    if (valid) {
                        uint16_t* o = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                      t.n_block * BN + 16 * c;
                        uint4* d = reinterpret_cast<uint4*>(o);
                        d[0] = make_uint4(p[0], p[1], p[2], p[3]);
                        d[1] = make_uint4(p[4], p[5], p[6], p[7]);
                    }
                }
            } else if (EPI == EPI_SWIGLU_BF16) {
                const float L = args.limit;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t g[16], u[16];
                    tmem_ld16(tbase + 16 * c, g);
                    tmem_ld16(tbase + 128 + 16 * c, u);
                    tmem_wait_ld();
                    uint32_t p[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t lo = f32_to_bf16_bits(swiglu_dev(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j]), L));
                        const uint32_t hi =
                            f32_to_bf16_bits(swiglu_dev(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1]), L));
                        p[j] = lo | (hi << 16);
                    }
                    if (valid) {
                        uint16_t* o = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                      t.n_block * 128 + 16 * c;
                        uint4* d = reinterpret_cast<uint4*>(o);
                        d[0] = make_uint4(p[0], p[1], p[2], p[3]);
                        d[1] = make_uint4(p[4], p[5], p[6], p[7]);
                    }
                }
            } else {  // EPI_STORE_F32
#pragma unroll 1
                for (int c = 0; c < 16; ++c) {
                    uint32_t v[16];
                    tmem_ld16(tbase + 16 * c, v);
                    tmem_wait_ld();
                    if (valid) {
                        float* o = static_cast<float*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                   t.n_block * BN + 16 * c;
                        uint4* d = reinterpret_cast<uint4*>(o);
                        d[0] = make_uint4(v[0], v[1], v[2], v[3]);
                        d[1] = make_uint4(v[4], v[5], v[6], v[7]);
                        d[2] = make_uint4(v[8], v[9], v[10], v[11]);
                        d[3] = make_uint4(v[12], v[13], v[14], v[15]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            acc_phase ^= 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*PfnEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PfnEncodeTiled encode_fn() {
    static PfnEncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PfnEncodeTiled>(p);
    });
    return fn;
}

// 2-D K-major tensor map with 128-byte swizzle: inner dimension in elements
// (bytes for packed FP4, BF16 elements otherwise), box = 128 bytes x box_rows.
bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner_elems, uint64_t rows,
                  uint32_t box_inner, uint32_t box_rows) {
    PfnEncodeTiled fn = encode_fn();
    if (!fn) return false;
    const uint64_t esize = bf16 ? 2 : 1;
    cuuint64_t dims[2] = {inner_elems, rows};
    cuuint64_t strides[1] = {inner_elems * esize};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int gemm_grid_size(int device) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms > 0 ? sms : 148;
}

template <int KIND, int EPI>
static cudaError_t launch_one(const CUtensorMap& tma, const CUtensorMap& tmb, const GemmArgs& args, int grid,
                              cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        const cudaError_t e =
            cudaFuncSetAttribute(gemm_kernel<KIND, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    gemm_kernel<KIND, EPI><<<grid, 192, SMEM_BYTES, st>>>(tma, tmb, args);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const CUtensorMap& tma, const CUtensorMap& tmb, const GemmArgs& args, int grid,
                        cudaStream_t st) {
    if (args.kind == KIND_NVFP4) {
        if (args.epi == EPI_SWIGLU_QUANT) return launch_one<KIND_NVFP4, EPI_SWIGLU_QUANT>(tma, tmb, args, grid, st);
        if (args.epi == EPI_STORE_BF16) return launch_one<KIND_NVFP4, EPI_STORE_BF16>(tma, tmb, args, grid, st);
    } else {
        if (args.epi == EPI_SWIGLU_BF16) return launch_one<KIND_BF16, EPI_SWIGLU_BF16>(tma, tmb, args, grid, st);
        if (args.epi == EPI_STORE_F32) return launch_one<KIND_BF16, EPI_STORE_F32>(tma, tmb, args, grid, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace nf
