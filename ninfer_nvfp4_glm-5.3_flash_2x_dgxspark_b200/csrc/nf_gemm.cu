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
// elements) loaded by TMA with 128-byte swizzle (B from its box-order copy:
// one contiguous 32 KB box per stage); block-scale atoms arrive by 1-D bulk
// copy (B's in tile order: one 4 KB copy per stage) and move to TMEM with
// tcgen05.cp; one elected thread issues the MMAs and commits stage release /
// accumulator-ready to mbarriers.  A tile with at most 32 rows (decode)
// loads only those rows of A (a 32-row box); the MMA's other 96 rows are
// left-over data whose outputs nobody stores.  Each TMA copy costs its SM
// about 280 cycles of fixed overhead, so a stage is kept to four copies.
// A thread completes its tcgen05.cp copies one after another (~150 cycles
// each), and in one thread's stream they also hold up the MMAs behind them:
// the 12 scale-atom copies of a stage cost about three times the stage's 4
// MMAs.  So separate scale warps issue them, split between them, one stage
// ahead of the MMA thread, which waits on a per-stage "scales in TMEM"
// barrier instead.
// Warp roles (640 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-17 epilogue (TMEM lane quadrant = warp % 4, four column
// slices per quadrant), warps 18-19 scale-factor copies (NVFP4).
// The persistent grid walks a device-side tile list, so the launch needs no
// host synchronisation after routing: the producer claims tiles in list
// order with an atomic counter and publishes each to the MMA and epilogue
// warps through a small mbarrier-guarded queue, so CTAs that start late
// (their SM still busy with another kernel) simply take fewer tiles.
// Every wait is bounded (nf_common.cuh mbar_wait); on a timeout the kernel
// records an error code, stops every role, drains and frees TMEM.
#include "nf_common.cuh"
#include "nf_gemm_shared.cuh"
#include "nf_internal.h"

#include <mutex>

namespace nf {

constexpr int BM = 128, BN = 256, STAGES = 4;
constexpr int kEpiWarps = 16;
constexpr int kSfWarps = 2;   // scale-factor copy warps (after the epilogue warps)
constexpr int kSfWarp0 = 2 + kEpiWarps;
constexpr int kTileQ = 4;  // depth of the producer -> consumer tile queue
constexpr int kSmallRows = 32;  // A box height for tiles with few rows (decode)
constexpr int kThreads = 64 + 32 * kEpiWarps + 32 * kSfWarps;
constexpr int B_STAGE_BYTES = BN * 128;
constexpr int SFA_STAGE_BYTES = 4 * 512;   // [k-step][512]
constexpr int SFB_STAGE_BYTES = 8 * 512;   // [b-block][k-step][512]
constexpr int TMEM_COLS = 512;
constexpr int ACC_COLS = 256;
constexpr int SF_COLS = 48;                // per stage: 16 for A, 32 for B

// Geometry of one instantiation.  MT = 2 (BF16 only): a CTA tile is two
// 128-row halves of A sharing each B stage, with the two accumulators in
// TMEM columns 0-255 and 256-511 (all of TMEM: BF16 needs no scale-factor
// columns), so a stage moves 64 KB for twice the MMAs of a 48 KB stage;
// three stages fit in shared memory.
// KS = 2 (grouped NVFP4 at prefill-sized batches): a stage covers 512 of K
// with the same four copies, each twice as large -- A as one 3-D box of two
// 16 KB chunks, B as one 3-D box of two consecutive 32 KB box-order blocks,
// and each scale group as one bulk copy.  A TMA copy costs its SM about 280
// cycles of fixed overhead (measured: a 16 KB box streams from L2 at 43 B per
// cycle per SM, a 32 KB box at 69), so the four copies of a 256-K stage
// (~1,450 cycles) outlast its four MMAs (512 cycles) almost threefold; at 512
// K per stage the same copies feed eight MMAs.  Two stages fit.
template <int KIND, int MT, int KS = 1>
struct Geo {
    static constexpr int kStages = MT == 2 ? 3 : (KS == 2 ? 2 : STAGES);
    static constexpr int kTileM = BM * MT;
    static constexpr int kAStage = kTileM * 128 * KS;
    static constexpr int kBStage = B_STAGE_BYTES * KS;
    static constexpr int kSfaStage = KIND == KIND_NVFP4 ? SFA_STAGE_BYTES * KS : 0;
    static constexpr int kSfbStage = KIND == KIND_NVFP4 ? SFB_STAGE_BYTES * KS : 0;
    static constexpr int kSfCols = SF_COLS * KS;
    static constexpr int kSmem = 1024 + kStages * (kAStage + kBStage + kSfaStage + kSfbStage) + 512;
    static_assert(MT == 1 || KIND == KIND_BF16, "paired row tiles are BF16 only");
    static_assert(KS == 1 || (KIND == KIND_NVFP4 && MT == 1), "512-K stages are NVFP4 only");
    static_assert(kSmem <= 227 * 1024, "shared memory");
    static_assert(KIND == KIND_BF16 || ACC_COLS + kStages * kSfCols <= TMEM_COLS, "TMEM columns");
};

struct TileInfo {
    int expert, row0, n_block, m_valid;
    int ks, kt0, kt1;  // K slice and its stages [kt0, kt1)
};

// Dense tiles are numbered (n block, K slice, m tile) with m fastest.
__device__ __forceinline__ void dense_split(const GemmArgs& a, int i, int k_tiles, int* m, int* n, int* ks, int* kt0,
                                            int* kt1, int tile_m) {
    const int m_tiles = (a.dense_rows + tile_m - 1) / tile_m;
    const int per_n = m_tiles * max(1, a.k_split);
    *n = i / per_n;
    const int r = i - *n * per_n;
    *ks = r / m_tiles;
    *m = r - *ks * m_tiles;
    *kt0 = a.k_split > 1 ? *ks * a.kt_per : 0;
    *kt1 = a.k_split > 1 ? min(k_tiles, *kt0 + a.kt_per) : k_tiles;
}

__device__ __forceinline__ TileInfo get_tile(const GemmArgs& a, int i, int k_tiles, int tile_m = BM) {
    TileInfo t;
    if (a.dense_rows > 0) {
        int m, n;
        dense_split(a, i, k_tiles, &m, &n, &t.ks, &t.kt0, &t.kt1, tile_m);
        t.expert = 0;
        t.row0 = m * tile_m;
        t.n_block = n;
        t.m_valid = min(tile_m, a.dense_rows - m * tile_m);
    } else {
        const NfTile x = a.tiles[i];
        t.expert = x.expert;
        t.row0 = x.row0;
        t.n_block = x.n_block;
        t.m_valid = x.m_valid;
        t.ks = 0;
        t.kt0 = 0;
        t.kt1 = k_tiles;
    }
    return t;
}

// The K stages of tile i, without reading the tile list (grouped tiles run all of K).
__device__ __forceinline__ void tile_krange(const GemmArgs& a, int i, int k_tiles, int* kt0, int* kt1, int tile_m = BM) {
    if (a.dense_rows > 0 && a.k_split > 1) {
        int m, n, ks;
        dense_split(a, i, k_tiles, &m, &n, &ks, kt0, kt1, tile_m);
    } else {
        *kt0 = 0;
        *kt1 = k_tiles;
    }
}

template <int KIND, int EPI, int MT, int KS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tma_small,
                const __grid_constant__ CUtensorMap tmb, const GemmArgs args) {
    using G = Geo<KIND, MT, KS>;
    constexpr int STAGES = G::kStages;  // (shadows the file-wide stage count)
    constexpr int A_STAGE_BYTES = G::kAStage;
    constexpr int B_STAGE_BYTES = G::kBStage;  // (shadows the file-wide 256-K size)
    constexpr int SFA_STAGE_BYTES = G::kSfaStage;
    constexpr int SFB_STAGE_BYTES = G::kSfbStage;
    constexpr int TM = G::kTileM;
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
    uint64_t* tq_full = drain + 1;          // tile queue: slot published
    uint64_t* tq_empty = tq_full + kTileQ;  // tile queue: slot read by every consumer
    uint64_t* sf_ready = tq_empty + kTileQ;  // stage's scale atoms are in TMEM
    uint64_t* sf_drain = sf_ready + STAGES;  // [kSfWarps] teardown after an abort
    int* tileq = reinterpret_cast<int*>(sf_drain + kSfWarps);
    volatile int* epi_mail = tileq + kTileQ;  // [2 slots][tile, ok]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(epi_mail) + 4);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* dev_err = args.err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kTileQ; ++s) {
            mbar_init(&tq_full[s], 1);
            // the MMA thread, the epilogue leader and (NVFP4) the scale warps
            mbar_init(&tq_empty[s], 2 + (KIND == KIND_NVFP4 ? kSfWarps : 0));
        }
        for (int s = 0; s < STAGES; ++s) mbar_init(&sf_ready[s], kSfWarps);
        for (int w = 0; w < kSfWarps; ++w) mbar_init(&sf_drain[w], 1);
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kEpiWarps);
        mbar_init(drain, 1);
        *cta_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tma);
        prefetch_tensormap(&tma_small);
        prefetch_tensormap(&tmb);
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int K = args.K;
    constexpr int kElemsPerStage = (KIND == KIND_NVFP4 ? 256 : 64) * KS;
    constexpr int kMmaK = KIND == KIND_NVFP4 ? 64 : 16;
    const int k_tiles = (K + kElemsPerStage - 1) / kElemsPerStage;
    const int sf_atoms_per_rowblock = K / 64;

    if (warp == 0) {
        // ------------------------------ producer ----------------------------
        // The whole warp runs the loop: lane 0 claims tiles, waits for free
        // stages and sets the expected bytes; the copies of a stage then go
        // out from separate lanes (a thread keeps only a couple of copies in
        // flight).  Lane 0: A; lane 1: the stage's 32 KB B box; lane 2: A's
        // scale atoms; lane 3: the 4 KB group of B's scale atoms.
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued_parity[STAGES];
        bool issued[STAGES];
        for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
        bool ok = true;
        int qslot = 0;
        uint32_t qphase = 0;
        // The next tile is claimed three stages before the current tile's
        // last and its descriptor read at the last, so neither the atomic nor
        // the dependent load sits between two tiles' copies (and a CTA holds
        // no tile long before it can start it).
        int next = 0, num_tiles = 0;
        TileInfo next_t{};
        auto claim_first = [&]() {
            num_tiles = args.dense_rows > 0 ? ((args.dense_rows + TM - 1) / TM) * args.n_blocks * max(1, args.k_split)
                                            : *args.num_tiles_dev;
            if (lane == 0) {
                next = args.static_tiles ? static_cast<int>(blockIdx.x) : atomicAdd(args.tile_counter, 1);
                if (next < num_tiles) next_t = get_tile(args, next, k_tiles, TM);
            }
        };
        if (args.early_claim) claim_first();
        // A: 16 KB, or 4 KB (rows 0-31) for a tile with at most 32 rows
        // B's scale groups of the stage's K blocks that hold MMA steps (a last
        // 512-K stage may cover one 256-K block only)
        auto sfb_bytes = [&](int steps) { return static_cast<uint32_t>((steps + 3) / 4) * (SFB_STAGE_BYTES / KS); };
        auto stage_bytes = [&](int steps, bool small) {
            uint32_t bytes = (small ? kSmallRows * 128 : A_STAGE_BYTES) + B_STAGE_BYTES;
            if (KIND == KIND_NVFP4) bytes += static_cast<uint32_t>(steps) * 512u + sfb_bytes(steps);
            return bytes;
        };
        // The kernel may start while the one that writes A is still running
        // (launch_dependent).  With early_claim the tile list and its counter
        // come from a kernel that has completed by then, and B and its scales
        // are weights, so the first tile's first stages of B go out before
        // pdl_wait(); A and its scales follow it.
        const uint64_t stream_policy = l2_evict_first();  // B and its scales: read once per step
        int pre = 0;
        if (args.early_claim) {
            const int first = __shfl_sync(0xffffffffu, next, 0);
            const int e0 = __shfl_sync(0xffffffffu, next_t.expert, 0);
            const int nb0 = __shfl_sync(0xffffffffu, next_t.n_block, 0);
            const int k00 = __shfl_sync(0xffffffffu, next_t.kt0, 0);
            const int k01 = __shfl_sync(0xffffffffu, next_t.kt1, 0);
            const bool small0 = MT == 1 && KS == 1 && __shfl_sync(0xffffffffu, next_t.m_valid, 0) <= kSmallRows;
            if (first < num_tiles) {
                // stage j holds K stage k00 + j of the first tile
                pre = min(STAGES, k01 - k00);
                for (int j = 0; j < pre; ++j) {
                    const int kt = k00 + j;
                    const int steps_j = min(4 * KS, (K - kt * kElemsPerStage) / kMmaK);
                    if (lane == 0) mbar_arrive_expect_tx(&full[j], stage_bytes(steps_j, small0));
                    __syncwarp();
                    const int blk = (e0 * args.b_nb + nb0) * args.b_kt + kt * KS;
                    if (lane == 1) {
                        if (KS == 2) tma_load_3d_hint(sB + j * B_STAGE_BYTES, &tmb, &full[j], 0, 0, blk, stream_policy);
                        else tma_load_2d_hint(sB + j * B_STAGE_BYTES, &tmb, &full[j], 0, blk * BN, stream_policy);
                    } else if (KIND == KIND_NVFP4 && lane == 3) {
                        bulk_load_hint(sSFB + j * SFB_STAGE_BYTES,
                                       args.sfb + static_cast<int64_t>(blk) * (SFB_STAGE_BYTES / KS), sfb_bytes(steps_j),
                                       &full[j], stream_policy);
                    }
                    issued[j] = true;
                }
            }
        }
        // With mt_wait the tiles wait for their own rows of the gate/up GEMM's
        // output (below) rather than for that whole kernel.
        if (args.mt_wait == 0) pdl_wait();
        if (lane == 0) pdl_trigger();
        if (!args.early_claim) claim_first();
        bool first_tile = true;
        while (ok) {
            // publish the claimed tile to the MMA and epilogue warps (-1 ends
            // the CTA's work)
            int i = 0;
            TileInfo t = next_t;
            if (lane == 0) {
                i = next < num_tiles ? next : -1;
                if (!mbar_wait(&tq_empty[qslot], qphase ^ 1u, cta_abort, dev_err)) {
                    set_abort(cta_abort, args.err, NF_DEVERR_WAIT_EMPTY);
                    ok = false;
                } else {
                    tileq[qslot] = i;
                    mbar_arrive(&tq_full[qslot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            i = __shfl_sync(0xffffffffu, i, 0);
            if (!ok) break;
            if (++qslot == kTileQ) qslot = 0, qphase ^= 1u;
            if (i < 0) break;
            t.expert = __shfl_sync(0xffffffffu, t.expert, 0);
            t.row0 = __shfl_sync(0xffffffffu, t.row0, 0);
            t.n_block = __shfl_sync(0xffffffffu, t.n_block, 0);
            t.m_valid = __shfl_sync(0xffffffffu, t.m_valid, 0);
            t.kt0 = __shfl_sync(0xffffffffu, t.kt0, 0);
            t.kt1 = __shfl_sync(0xffffffffu, t.kt1, 0);
            // tiles with at most 32 rows of the expert load only those rows of A
            const bool small_a = MT == 1 && KS == 1 && t.m_valid <= kSmallRows;
            if (args.mt_wait > 0) {
                // A (and its scales) are the gate/up GEMM's output for these rows:
                // generic stores in other CTAs, ordered before these TMA reads by
                // the counter's release/acquire and the proxy fences
                if (!wait_count(args.mt_done + t.row0 / BM, args.mt_wait, cta_abort, dev_err)) {
                    if (lane == 0) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                    ok = false;
                    break;
                }
                fence_proxy_async_global();
            }
            for (int kt = t.kt0; kt < t.kt1; ++kt) {
                const int k0 = kt * kElemsPerStage;
                const int steps = min(4 * KS, (K - k0) / kMmaK);
                const bool b_issued = first_tile && kt - t.kt0 < pre;  // B of this stage went out before pdl_wait()
                if (lane == 0 && !b_issued) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_EMPTY);
                        ok = false;
                    } else {
                        mbar_arrive_expect_tx(&full[stage], stage_bytes(steps, small_a));
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) break;
                // stage kt of tile (expert, n_block) is box `blk` of B and 4 KB group `blk` of its scales
                // (with KS = 2: boxes and groups blk and blk + 1)
                const int blk = (t.expert * args.b_nb + t.n_block) * args.b_kt + kt * KS;
                const int xc = KIND == KIND_NVFP4 ? kt * 128 : k0;  // A's K coordinate (bytes or BF16 elements)
                if (KS == 2 && lane == 0) {
                    // A's 128 rows x two 256-K chunks: x 0, rows, chunk index
                    tma_load_3d(sA + stage * A_STAGE_BYTES, &tma, &full[stage], 0, t.row0, kt * KS);
                } else if (lane == 0) {
                    tma_load_2d(sA + stage * A_STAGE_BYTES, small_a ? &tma_small : &tma, &full[stage], xc, t.row0);
                } else if (MT == 2 && lane == 4) {
                    // the tile's second 128 rows (zero-filled past the tensor)
                    tma_load_2d(sA + stage * A_STAGE_BYTES + BM * 128, &tma, &full[stage], xc, t.row0 + BM);
                } else if (lane == 1 && !b_issued) {
                    if (KS == 2) tma_load_3d_hint(sB + stage * B_STAGE_BYTES, &tmb, &full[stage], 0, 0, blk, stream_policy);
                    else tma_load_2d_hint(sB + stage * B_STAGE_BYTES, &tmb, &full[stage], 0, blk * BN, stream_policy);
                } else if (KIND == KIND_NVFP4 && lane == 2) {
                    const int64_t a_atom = static_cast<int64_t>(t.row0 / 128) * sf_atoms_per_rowblock + kt * 4 * KS;
                    bulk_load(sSFA + stage * SFA_STAGE_BYTES, args.sfa + a_atom * 512, steps * 512u, &full[stage]);
                } else if (KIND == KIND_NVFP4 && lane == 3 && !b_issued) {
                    bulk_load_hint(sSFB + stage * SFB_STAGE_BYTES,
                                   args.sfb + static_cast<int64_t>(blk) * (SFB_STAGE_BYTES / KS), sfb_bytes(steps),
                                   &full[stage], stream_policy);
                }
                issued[stage] = true;
                issued_parity[stage] = phase;
                if (++stage == STAGES) stage = 0, phase ^= 1u;
                // (with the fused split-K reduction a CTA takes one tile only: its
                // epilogue waits for the tile's other K slices, which must not sit
                // behind it in this CTA's own pipeline)
                if (lane == 0 && kt == max(t.kt0, t.kt1 - 3))
                    next = (args.splitk_fuse || args.static_tiles) ? num_tiles : atomicAdd(args.tile_counter, 1);
                if (lane == 0 && kt == t.kt1 - 1 && next < num_tiles) next_t = get_tile(args, next, k_tiles, TM);
            }
            first_tile = false;
        }
        if (!ok && lane == 0) {
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
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, acc_phase = 0;
            const uint32_t idesc = KIND == KIND_NVFP4 ? idesc_nvfp4(BM, BN) : idesc_bf16(BM, BN);
            bool ok = true;
            int qslot = 0;
            uint32_t qphase = 0;
            while (ok) {
                if (!mbar_wait(&tq_full[qslot], qphase, cta_abort, dev_err)) {
                    set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                    ok = false;
                    break;
                }
                const int i = tileq[qslot];
                mbar_arrive(&tq_empty[qslot]);
                if (++qslot == kTileQ) qslot = 0, qphase ^= 1u;
                if (i < 0) break;
                if (!mbar_wait(acc_empty, acc_phase ^ 1u, cta_abort, dev_err)) {
                    set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                    ok = false;
                    break;
                }
                tc_fence_after();
                int kt0, kt1;
                tile_krange(args, i, k_tiles, &kt0, &kt1, TM);
                for (int kt = kt0; kt < kt1; ++kt) {
                    if (!mbar_wait(&full[stage], phase, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                        ok = false;
                        break;
                    }
                    if (KIND == KIND_NVFP4 && !mbar_wait(&sf_ready[stage], phase, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int k0 = kt * kElemsPerStage;
                    const int steps = min(4 * KS, (K - k0) / kMmaK);
                    const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
                    const uint32_t sfa_col = ACC_COLS + stage * G::kSfCols;
                    const uint32_t sfb_col = sfa_col + 16 * KS;
                    for (int s = 0; s < steps; ++s) {
                        // step s: 256-K block s / 4 of the stage (its own 16 KB of A and 32 KB of B)
                        const int sb = KS == 2 ? (s >> 2) : 0, s4 = KS == 2 ? (s & 3) : s;
                        const uint64_t adesc = sdesc_sw128(a_base + sb * (BM * 128) + 32 * s4);
                        const uint64_t bdesc = sdesc_sw128(b_base + sb * (BN * 128) + 32 * s4);
                        const uint32_t acc = (kt > kt0 || s > 0) ? 1u : 0u;
                        if (KIND == KIND_NVFP4)
                            mma_nvfp4(tmem, adesc, bdesc, idesc, tmem + sfa_col + 4 * s, tmem + sfb_col + 8 * s, acc);
                        else
                            mma_bf16(tmem, adesc, bdesc, idesc, acc);
                        if (MT == 2)  // the second 128 rows into the second accumulator
                            mma_bf16(tmem + ACC_COLS, sdesc_sw128(a_base + BM * 128 + 32 * s), bdesc, idesc, acc);
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
    } else if (warp < kSfWarp0) {
        // ------------------------------ epilogue ----------------------------
        // kEpiWarps warps: a warp may only touch the TMEM lane quadrant
        // warp % 4, and the 4 warps of one quadrant split the tile's columns
        // into slices.  Each warp copies its slice of the accumulator into
        // registers, hands the accumulator back to the MMA warp at once, then
        // does the math and the stores while the next tile's MMAs run.
        const int q = warp & 3;
        const int cs = (warp - 2) >> 2;
        const int r = q * 32 + lane;
        const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
        // One leader thread waits for the next tile and for its accumulator;
        // the other epilogue warps sleep on a hardware named barrier instead
        // of polling.  The leader's verdict travels through a two-slot
        // shared-memory mailbox (a slot is rewritten only after every warp
        // has passed the next barrier, i.e. read it).
        const bool leader = warp == 2 && lane == 0;
        int ep_tiles = 0;  // tiles of a fused expert-parallel return stored by this CTA
        uint32_t acc_phase = 0;
        int qslot = 0;
        uint32_t qphase = 0;
        for (int iter = 0;; ++iter) {
            if (leader) {
                int ok = mbar_wait(&tq_full[qslot], qphase, cta_abort, dev_err) ? 1 : 0;
                const int tile = ok ? tileq[qslot] : -1;
                if (ok) mbar_arrive(&tq_empty[qslot]);
                if (ok && tile >= 0) ok = mbar_wait(acc_full, acc_phase, cta_abort, dev_err) ? 1 : 0;
                if (!ok) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                epi_mail[2 * (iter & 1)] = tile;
                epi_mail[2 * (iter & 1) + 1] = ok;
            }
            named_bar_sync(1, 32 * kEpiWarps);
            const int tile = epi_mail[2 * (iter & 1)];
            const int ok = epi_mail[2 * (iter & 1) + 1];
            if (++qslot == kTileQ) qslot = 0, qphase ^= 1u;
            if (!ok || tile < 0) {
                if (EPI == EPI_STORE_BF16 && args.ep_ret && ok) {
                    // Fused expert-parallel return: once every epilogue warp's
                    // rows are out, one system-scope fence and the CTA's tile
                    // count; the CTA that completes the count (CTA 0 when there
                    // are no tiles) publishes every source's flag.
                    named_bar_sync(2, 32 * kEpiWarps);
                    if (leader) {
                        const int total = *args.num_tiles_dev;
                        bool last = total == 0 && blockIdx.x == 0;
                        if (ep_tiles > 0) {
                            __threadfence_system();
                            last = atomicAdd(args.ep_tiles_done, ep_tiles) + ep_tiles == total;
                        }
                        if (last) {
                            __threadfence_system();
                            const uint32_t ep = *args.ep_epoch + 1u;
                            for (int s2 = 0; s2 < args.ep_world; ++s2)
                                st_release_sys(reinterpret_cast<uint32_t*>(args.ep_mbox[s2] + args.ep_flags_ret) + args.ep_me,
                                               ep);
                            *args.ep_tiles_done = 0;
                        }
                    }
                }
                break;
            }
            const TileInfo t = get_tile(args, tile, k_tiles, TM);
            tc_fence_after();
            if constexpr (MT == 2) {
                // Two 128-row accumulators (TMEM columns 0-255, 256-511); every
                // warp hands the accumulator back once its share of the second
                // one is in registers.
#pragma unroll 1
                for (int mt = 0; mt < 2; ++mt) {
                    const uint32_t tb = tbase + mt * ACC_COLS;
                    const int row = t.row0 + mt * BM + r;
                    const bool valid = mt * BM + r < t.m_valid;
                    const bool live = mt * BM + q * 32 < t.m_valid;
                    uint32_t v[64];
                    if (EPI == EPI_SWIGLU_BF16) {
                        if (live) {
                            tmem_ld16(tb + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                            tmem_ld16(tb + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                            tmem_ld16(tb + 128 + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[32]));
                            tmem_ld16(tb + 128 + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[48]));
                            tmem_wait_ld();
                        }
                        if (mt == 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(acc_empty);
                        }
                        if (live) {
                            const float L = args.limit;
                            uint32_t p[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                p[j] = bf16x2_hw(swiglu_fast(__uint_as_float(v[2 * j]), __uint_as_float(v[32 + 2 * j]), L),
                                                 swiglu_fast(__uint_as_float(v[2 * j + 1]), __uint_as_float(v[32 + 2 * j + 1]), L));
                            if (valid) {
                                uint16_t* d = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                              t.n_block * 128 + 32 * cs;
                                st_global_v8(d, p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7]);
                                st_global_v8(d + 16, p[8], p[9], p[10], p[11], p[12], p[13], p[14], p[15]);
                            }
                        }
                    } else {  // EPI_STORE_F32: 16 columns at a time straight to memory
                        if (live) {
                            float* d = static_cast<float*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                       t.n_block * BN + 64 * cs;
#pragma unroll 1
                            for (int c = 0; c < 4; ++c) {
                                tmem_ld16(tb + 64 * cs + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                                tmem_wait_ld();
                                if (valid) {
                                    st_global_v8(d + 16 * c, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
                                    st_global_v8(d + 16 * c + 8, v[8], v[9], v[10], v[11], v[12], v[13], v[14], v[15]);
                                }
                            }
                        }
                        if (mt == 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(acc_empty);
                        }
                    }
                }
                acc_phase ^= 1u;
                continue;
            }
            // (a tile of at most 32 rows has them in TMEM lane quadrant 0 only:
            // its four warps take the tile's columns, the others idle)
            // rep64 (dense NVFP4 gate/up of 33-64 rows): the tile's rows 64-127
            // repeat rows 0-63, so quadrants 2 and 3 hold the accumulators of 0
            // and 1 again; a warp of quadrant q then stores rows (q & 1) * 32 +
            // lane and takes the 16-column half q >> 1 of its slice, and all
            // sixteen warps share the epilogue
            const bool rep = EPI == EPI_SWIGLU_QUANT && args.rep64 != 0;
            const int rr = rep ? (q & 1) * 32 + lane : r;
            const int hg = rep ? (q >> 1) : 0;
            const int row = t.row0 + rr;
            const bool valid = rr < t.m_valid;
            const bool warp_live = rr - lane < t.m_valid;  // some row of this warp belongs to the expert
            uint32_t v[64];
            if (warp_live) {
                if (EPI == EPI_SWIGLU_QUANT && rep) {
                    // gate columns [32cs + 16hg, +16), up columns 128 further
                    tmem_ld16(tbase + 32 * cs + 16 * hg, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                    tmem_ld16(tbase + 128 + 32 * cs + 16 * hg, *reinterpret_cast<uint32_t(*)[16]>(&v[32]));
                } else if (EPI == EPI_SWIGLU_QUANT || EPI == EPI_SWIGLU_BF16) {
                    // gate columns [32cs, 32cs+32), up columns 128 further
                    tmem_ld16(tbase + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                    tmem_ld16(tbase + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                    tmem_ld16(tbase + 128 + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[32]));
                    tmem_ld16(tbase + 128 + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[48]));
                } else if (EPI == EPI_STORE_F32) {
                    // no math: stream 16 columns at a time straight to memory
                    float* d = static_cast<float*>(args.out) + t.ks * args.out_split_stride +
                               static_cast<int64_t>(row) * args.out_ld + t.n_block * BN + 64 * cs;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        tmem_ld16(tbase + 64 * cs + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                        tmem_wait_ld();
                        if (valid) {
                            st_global_v8(d + 16 * c, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
                            st_global_v8(d + 16 * c + 8, v[8], v[9], v[10], v[11], v[12], v[13], v[14], v[15]);
                        }
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tmem_ld16(tbase + 64 * cs + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]));
                }
                tmem_wait_ld();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            acc_phase ^= 1u;
            if (warp_live) {

            if (EPI == EPI_SWIGLU_QUANT) {
                const float ag = args.alpha0[t.expert], au = args.alpha1[t.expert];
                const float gsd = args.gscale_next[t.expert], L = args.limit;
                const bool sbf = args.swiglu_bf16 != 0;
                const float* os_tab = args.os_table ? args.os_table + 256 * t.expert : nullptr;
                if (rep) {
                    uint32_t c1[2];
                    const uint32_t s1 = swiglu_quant_group(&v[0], &v[32], ag, au, gsd, L, sbf, os_tab, c1);
                    if (valid) {
                        uint8_t* o = static_cast<uint8_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                     t.n_block * 64 + cs * 16 + 8 * hg;
                        *reinterpret_cast<uint2*>(o) = make_uint2(c1[0], c1[1]);
                        args.out_sf[sf_atom_offset(row, t.n_block * 8 + cs * 2 + hg, args.out_kgroups)] =
                            static_cast<uint8_t>(s1);
                    }
                } else {
                uint32_t cc[2][2];
                uint32_t sc[2];
#pragma unroll
                for (int g = 0; g < 2; ++g)
                    sc[g] = swiglu_quant_group(&v[16 * g], &v[32 + 16 * g], ag, au, gsd, L, sbf, os_tab, cc[g]);
                if (valid) {
                    uint8_t* o = static_cast<uint8_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                 t.n_block * 64 + cs * 16;
                    *reinterpret_cast<uint4*>(o) = make_uint4(cc[0][0], cc[0][1], cc[1][0], cc[1][1]);
                    *reinterpret_cast<uint16_t*>(args.out_sf + sf_atom_offset(row, t.n_block * 8 + cs * 2, args.out_kgroups)) =
                        static_cast<uint16_t>(sc[0] | (sc[1] << 8));
                }
                }
            } else if (EPI == EPI_STORE_BF16) {
                const float a = args.alpha0[t.expert];
                uint32_t p[32];
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    p[j] = bf16x2_hw(__fmul_rn(__uint_as_float(v[2 * j]), a), __fmul_rn(__uint_as_float(v[2 * j + 1]), a));
                uint16_t* d = nullptr;
                if (valid && args.ep_ret) {
                    // the row's source rank and slot: its output goes to that rank's mailbox
                    const int j = args.row_token[row];
                    if (j >= 0) {
                        const int src = j / args.ep_cap, k = j - src * args.ep_cap;
                        d = reinterpret_cast<uint16_t*>(args.ep_mbox[src] + args.ep_ret_off) +
                            static_cast<int64_t>(args.ep_src_off[src] + k) * args.out_ld + t.n_block * BN + 64 * cs;
                    }
                } else if (valid) {
                    d = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld + t.n_block * BN +
                        64 * cs;
                }
                if (d) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        st_global_v8(d + 16 * j, p[8 * j], p[8 * j + 1], p[8 * j + 2], p[8 * j + 3], p[8 * j + 4],
                                     p[8 * j + 5], p[8 * j + 6], p[8 * j + 7]);
                }
            } else if (EPI == EPI_SWIGLU_BF16) {
                const float L = args.limit;
                uint32_t p[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    p[j] = bf16x2_hw(swiglu_fast(__uint_as_float(v[2 * j]), __uint_as_float(v[32 + 2 * j]), L),
                                     swiglu_fast(__uint_as_float(v[2 * j + 1]), __uint_as_float(v[32 + 2 * j + 1]), L));
                if (valid) {
                    uint16_t* d = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                  t.n_block * 128 + 32 * cs;
                    st_global_v8(d, p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7]);
                    st_global_v8(d + 16, p[8], p[9], p[10], p[11], p[12], p[13], p[14], p[15]);
                }
            }
            }
            if (EPI == EPI_SWIGLU_QUANT || EPI == EPI_SWIGLU_BF16) {
                if (args.mt_signal) {
                    // count the tile for the down GEMM once every warp's stores are out
                    named_bar_sync(2, 32 * kEpiWarps);
                    if (leader) {
                        __threadfence();
                        fence_proxy_async_global();
                        atomicAdd(args.mt_done + t.row0 / BM, 1);
                    }
                }
            }
            if (EPI == EPI_STORE_BF16 && args.ep_ret) ++ep_tiles;  // counted once, at the CTA's end
            if (EPI == EPI_STORE_F32 && args.splitk_fuse) {
                // Fused split-K reduction: count this slice once every warp's
                // stores are out, wait for the tile's other slices (their CTAs
                // are all running: one tile per CTA), then sum this slice's share
                // of the tile's rows over the slices in order.
                named_bar_sync(2, 32 * kEpiWarps);
                if (leader) {
                    int* cnt = args.splitk_cnt + (t.row0 / BM) * args.n_blocks + t.n_block;
                    __threadfence();
                    atomicAdd(cnt, 1);
                    if (!wait_count(cnt, args.k_split, cta_abort, dev_err)) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                    __threadfence();
                }
                named_bar_sync(2, 32 * kEpiWarps);
                if (*cta_abort == 0) {
                    const int S = args.k_split;
                    const int per = (t.m_valid + S - 1) / S;
                    const int r0 = min(t.m_valid, t.ks * per), r1 = min(t.m_valid, r0 + per);
                    const float a = args.alpha0[0];
                    const int nq = (r1 - r0) * (BN / 4);
                    for (int u = (warp - 2) * 32 + lane; u < nq; u += 32 * kEpiWarps) {
                        const int64_t off = static_cast<int64_t>(t.row0 + r0 + u / (BN / 4)) * args.out_ld +
                                            t.n_block * BN + 4 * (u % (BN / 4));
                        const float* part = static_cast<const float*>(args.out);
                        float4 acc = *reinterpret_cast<const float4*>(part + off);
                        for (int s2 = 1; s2 < S; ++s2) {
                            const float4 v = *reinterpret_cast<const float4*>(part + s2 * args.out_split_stride + off);
                            acc.x = __fadd_rn(acc.x, v.x);
                            acc.y = __fadd_rn(acc.y, v.y);
                            acc.z = __fadd_rn(acc.z, v.z);
                            acc.w = __fadd_rn(acc.w, v.w);
                        }
                        float4 o = make_float4(bf16_round_hw(__fmul_rn(acc.x, a)), bf16_round_hw(__fmul_rn(acc.y, a)),
                                               bf16_round_hw(__fmul_rn(acc.z, a)), bf16_round_hw(__fmul_rn(acc.w, a)));
                        if (args.residual) {
                            const float4 r = *reinterpret_cast<const float4*>(args.residual + off);
                            o.x = __fadd_rn(o.x, r.x);
                            o.y = __fadd_rn(o.y, r.y);
                            o.z = __fadd_rn(o.z, r.z);
                            o.w = __fadd_rn(o.w, r.w);
                        }
                        *reinterpret_cast<float4*>(args.y + off) = o;
                    }
                }
            }
        }
    } else if (KIND == KIND_NVFP4 && lane == 0) {
        // --------------------------- scale-factor copies -----------------------
        // Follows the tile queue and the stage ring like the MMA thread: once a
        // stage has landed, copy this warp's share of its 12 scale atoms (A's
        // 4, then B's two row halves' 4 each) into the stage's TMEM columns and
        // commit to sf_ready.  A stage's columns are rewritten only after the
        // stage was refilled, i.e. after the MMAs that read them completed.
        const int sw = warp - kSfWarp0;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int qslot = 0;
        uint32_t qphase = 0;
        while (ok) {
            if (!mbar_wait(&tq_full[qslot], qphase, cta_abort, dev_err)) {
                set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                ok = false;
                break;
            }
            const int i = tileq[qslot];
            mbar_arrive(&tq_empty[qslot]);
            if (++qslot == kTileQ) qslot = 0, qphase ^= 1u;
            if (i < 0) break;
            int kt0, kt1;
            tile_krange(args, i, k_tiles, &kt0, &kt1);
            for (int kt = kt0; kt < kt1; ++kt) {
                if (!mbar_wait(&full[stage], phase, cta_abort, dev_err)) {
                    set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                    ok = false;
                    break;
                }
                const int steps = min(4 * KS, (K - kt * kElemsPerStage) / kMmaK);
                const uint32_t sfa_col = ACC_COLS + stage * G::kSfCols;
                for (int c = sw; c < 12 * KS; c += kSfWarps) {
                    // atoms 0 .. 4 KS - 1: A's, one per MMA step; then B's, two row halves per step
                    const bool is_a = c < 4 * KS;
                    const int s = is_a ? c : (c - 4 * KS) >> 1, w = is_a ? 0 : ((c - 4 * KS) & 1);
                    if (s >= steps) continue;
                    const uint8_t* src = is_a ? sSFA + stage * SFA_STAGE_BYTES + s * 512
                                              : sSFB + stage * SFB_STAGE_BYTES + (s >> 2) * 4096 + w * 2048 + (s & 3) * 512;
                    const uint32_t col = is_a ? sfa_col + 4 * s : sfa_col + 16 * KS + 8 * s + 4 * w;
                    tmem_cp_sf(tmem + col, sdesc_sf_atom(smem_u32(src)));
                }
                tc_commit(&sf_ready[stage]);
                if (++stage == STAGES) stage = 0, phase ^= 1u;
            }
        }
        if (!ok) {
            tc_commit(&sf_drain[sw]);
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&sf_drain[sw], 0)) {
                if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) {
                    atomicCAS(args.err, 0, NF_DEVERR_DRAIN);
                    break;
                }
            }
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

bool make_tmap_blocked(CUtensorMap* map, const void* base, uint64_t bytes, uint32_t box_rows) {
    PfnEncodeTiled fn = encode_fn();
    if (!fn || bytes % (BN * 128) != 0 || box_rows == 0 || box_rows > 256) return false;
    cuuint64_t dims[2] = {128, bytes / 128};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_a3(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows) {
    PfnEncodeTiled fn = encode_fn();
    if (!fn || row_bytes % 256 != 0) return false;
    // [K / 256 chunks][rows][128 bytes]: x = byte in the chunk, y = row, z = chunk
    cuuint64_t dims[3] = {128, rows, row_bytes / 128};
    cuuint64_t strides[2] = {row_bytes, 128};
    cuuint32_t box[3] = {128, BM, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_b3(CUtensorMap* map, const void* base, uint64_t bytes) {
    PfnEncodeTiled fn = encode_fn();
    if (!fn || bytes % (BN * 128) != 0) return false;
    // box-order blocks [blocks][256 rows][128 bytes]; a box is two consecutive blocks
    cuuint64_t dims[3] = {128, BN, bytes / (BN * 128)};
    cuuint64_t strides[2] = {128, BN * 128};
    cuuint32_t box[3] = {128, BN, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_runs(CUtensorMap* map, const void* base, uint64_t bytes, uint32_t box_rows) {
    PfnEncodeTiled fn = encode_fn();
    if (!fn || bytes % 256 != 0 || box_rows == 0 || box_rows > 256) return false;
    cuuint64_t dims[2] = {256, bytes / 256};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {256, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int gemm_grid_size(int device) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms > 0 ? sms : 148;
}

template <int KIND, int EPI, int MT = 1, int KS = 1>
static cudaError_t launch_one(const CUtensorMap& tma, const CUtensorMap& tma_small, const CUtensorMap& tmb,
                              const GemmArgs& args, int grid, bool dependent, cudaStream_t st) {
    constexpr int SMEM_BYTES = Geo<KIND, MT, KS>::kSmem;
    // the shared memory limit is an attribute of the kernel in each device's context
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(gemm_kernel<KIND, EPI, MT, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    if (dependent)
        return launch_dependent(gemm_kernel<KIND, EPI, MT, KS>, dim3(grid), dim3(kThreads), SMEM_BYTES, st, tma, tma_small,
                                tmb, args);
    gemm_kernel<KIND, EPI, MT, KS><<<grid, kThreads, SMEM_BYTES, st>>>(tma, tma_small, tmb, args);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const CUtensorMap& tma, const CUtensorMap& tma_small, const CUtensorMap& tmb,
                        const GemmArgs& args, int grid, bool dependent, cudaStream_t st) {
    if (args.kind == KIND_NVFP4 && args.wide_stages) {
        // 512-K stages: tma / tmb are the 3-D maps (make_tmap_a3 / make_tmap_b3); no split K
        if (args.dense_rows > 0 && args.k_split > 1) return cudaErrorInvalidValue;
        if (args.epi == EPI_SWIGLU_QUANT) return launch_one<KIND_NVFP4, EPI_SWIGLU_QUANT, 1, 2>(tma, tma_small, tmb, args, grid, dependent, st);
        if (args.epi == EPI_STORE_BF16) return launch_one<KIND_NVFP4, EPI_STORE_BF16, 1, 2>(tma, tma_small, tmb, args, grid, dependent, st);
        return cudaErrorInvalidValue;
    }
    if (args.kind == KIND_NVFP4) {
        if (args.epi == EPI_SWIGLU_QUANT) return launch_one<KIND_NVFP4, EPI_SWIGLU_QUANT>(tma, tma_small, tmb, args, grid, dependent, st);
        if (args.epi == EPI_STORE_BF16) return launch_one<KIND_NVFP4, EPI_STORE_BF16>(tma, tma_small, tmb, args, grid, dependent, st);
        if (args.epi == EPI_STORE_F32) return launch_one<KIND_NVFP4, EPI_STORE_F32>(tma, tma_small, tmb, args, grid, dependent, st);
    } else {
        if (args.m_pair && args.dense_rows > 0) {
            if (args.epi == EPI_SWIGLU_BF16) return launch_one<KIND_BF16, EPI_SWIGLU_BF16, 2>(tma, tma_small, tmb, args, grid, dependent, st);
            if (args.epi == EPI_STORE_F32) return launch_one<KIND_BF16, EPI_STORE_F32, 2>(tma, tma_small, tmb, args, grid, dependent, st);
            return cudaErrorInvalidValue;
        }
        if (args.epi == EPI_SWIGLU_BF16) return launch_one<KIND_BF16, EPI_SWIGLU_BF16>(tma, tma_small, tmb, args, grid, dependent, st);
        if (args.epi == EPI_STORE_F32) return launch_one<KIND_BF16, EPI_STORE_F32>(tma, tma_small, tmb, args, grid, dependent, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace nf
