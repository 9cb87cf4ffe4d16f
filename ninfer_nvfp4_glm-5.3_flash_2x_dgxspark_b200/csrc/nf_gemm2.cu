// nf_gemm2.cu -- the grouped NVFP4 expert GEMMs on CTA pairs (tcgen05
// cta_group::2) with the activation rows resident, for prefill-sized batches.
//
// A pair of CTAs on two SMs of one cluster computes 256 x 256 tiles: 256
// permuted rows of one expert (128 per CTA) x one 256-row block of B.  One
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 64) reads A's rows from
// each CTA's own shared memory and B's 256 rows half from each CTA.
// Work item: one expert's 256-row slice x up to kRange B blocks.  Each CTA
// keeps its 128 A rows for the whole K in shared memory (K / 256 chunks of
// 16 KB, with their scale atoms) and their scale atoms in TMEM, and streams
// only its half of each B block (16 KB per 256 K) and the block's scale
// atoms (4 KB).  So once an item's first block is done, a stage moves 20 KB
// into a CTA's shared memory for 512 MMA cycles, where the one-SM kernel
// (128 x 256 tiles, A and B per stage) moves 54 KB: the layer's expert GEMMs
// are bound by the rate at which L2 fills shared memory, not by the tensor
// pipe (measured: the same pipeline with the MMAs left out runs within 6%).
// The first block of an item streams A chunk kt together with B stage kt.
// Chunk kt is released (and the next item's chunk kt loaded) as soon as the
// item's last block has used it, so items follow one another without a gap.
// Every load is a tiled TMA load with .cta_group::2 that lands in the issuing
// CTA's own shared memory and completes on the LEADER's (rank 0) barrier,
// which expects both CTAs' bytes.  No load reads another GPU's memory and
// none is distributed to several CTAs.
// The leader alone issues the MMAs and the scale-atom copies
// (tcgen05.cp.cta_group::2 copies each CTA's atoms into its own TMEM), and
// commits every release and accumulator hand-off to the barrier at the same
// offset in both CTAs (one tcgen05.commit with a CTA mask: each tcgen05
// instruction holds its issuing thread for about 100 cycles, and a stage's
// four MMAs run for 512).  Each CTA's epilogue reads its own
// 128 x 256 accumulator from its own TMEM and arrives on the leader's
// accumulator-free barrier.
// TMEM: the accumulator (256 columns), A's scale atoms for the whole K
// (16 columns per 256 K) and B's per stage (32 columns each).
// Schedule: static.  Items are ordered (expert, block range, 256-row slice),
// slices fastest, so clusters running at the same time share each weight
// block through L2; cluster c takes items c, c + clusters, ...  The item set
// follows from the permutation's segment offsets and counts, read once per
// CTA into shared memory.
// Warp roles (640 threads, both CTAs): warp 0 TMA producer, warp 1 TMEM owner
// (+ MMA issuer in the leader), warps 2-17 epilogue, warps 18-19 scale-atom
// copies (leader).  Every wait is bounded; a timeout records an error code
// and stops every role of both CTAs (through the device error word).
#include "nf_common.cuh"
#include "nf_gemm_shared.cuh"
#include "nf_internal.h"

#include <mutex>

namespace nf {

namespace {

constexpr int kMaxKt = 8;       // K up to 2048
constexpr int kMaxStages = 5;   // B stages
constexpr int kRange = 4;       // B blocks per work item
constexpr int kEpiWarps = 16;
constexpr int kSfWarps = 2;
constexpr int kSfWarp0 = 2 + kEpiWarps;
constexpr int kThreads = 64 + 32 * kEpiWarps + 32 * kSfWarps;
constexpr int kAChunk = 128 * 128;  // this CTA's A rows x 256 K (FP4)
constexpr int kSfaChunk = 4 * 512;  // their scale atoms
constexpr int kBStage = 128 * 128;  // this CTA's half of a B block x 256 K
constexpr int kSfbStage = 8 * 512;  // the whole block's scale atoms
constexpr uint32_t kATx = 2u * (kAChunk + kSfaChunk);   // both CTAs
constexpr uint32_t kBTx = 2u * (kBStage + kSfbStage);
constexpr int kTmemCols = 512;
constexpr int kAccCols = 256;
constexpr int kMaxE = 128;
constexpr int kTailBytes = 4096;  // barriers, segments
constexpr int kSmemLimit = 232448;

__host__ __device__ constexpr int pair_smem(int kt, int stages) {
    return 1024 + kt * (kAChunk + kSfaChunk) + stages * (kBStage + kSfbStage) + kTailBytes;
}
// B stages for K / 256 = kt: as many as shared memory and TMEM hold
__host__ __device__ constexpr int pair_stages(int kt) {
    int s = kMaxStages;
    while (s > 1 && (pair_smem(kt, s) > kSmemLimit || kAccCols + 16 * kt + 32 * s > kTmemCols)) --s;
    return s;
}
static_assert(pair_stages(kMaxKt) >= 3, "pipeline depth");

struct Item {
    int expert, row0, n0, n1, m_valid;  // m_valid: rows of the 256 that belong to the expert
};

// Item p from the per-expert prefix of items (s_pfx[e], e <= E).
__device__ __forceinline__ Item pair_item(const int* s_pfx, const int* s_off, const int* s_cnt, int E, int nb,
                                          int p) {
    int lo = 0, hi = E - 1;  // expert e with s_pfx[e] <= p < s_pfx[e + 1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_pfx[mid] <= p) lo = mid;
        else hi = mid - 1;
    }
    const int e = lo;
    const int slices = (((s_cnt[e] + 127) >> 7) + 1) >> 1;
    const int local = p - s_pfx[e];
    const int r = local / slices, m = local - r * slices;
    Item t;
    t.expert = e;
    t.row0 = s_off[e] + 256 * m;
    t.n0 = r * kRange;
    t.n1 = min(nb, t.n0 + kRange);
    t.m_valid = min(256, s_cnt[e] - 256 * m);
    return t;
}

}  // namespace

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb_half,
                 const __grid_constant__ CUtensorMap tm_sfa, const __grid_constant__ CUtensorMap tm_sfb,
                 const GemmArgs args) {
    const int KT = args.K / 256;  // (K % 256 == 0, KT <= kMaxKt for this kernel)
    const int S = pair_stages(KT);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                       // [KT][16 KB]
    uint8_t* sSFA = sA + KT * kAChunk;        // [KT][2 KB]
    uint8_t* sB = sSFA + KT * kSfaChunk;      // [S][16 KB]
    uint8_t* sSFB = sB + S * kBStage;         // [S][4 KB]
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sSFB + S * kSfbStage);  // leader: A chunk landed (both CTAs)
    uint64_t* empty_a = full_a + kMaxKt;      // both: chunk free (the item's last MMAs on it completed)
    uint64_t* sfa_ready = empty_a + kMaxKt;   // leader: chunk's scale atoms in TMEM
    uint64_t* full_b = sfa_ready + kMaxKt;    // leader: B stage landed (both CTAs)
    uint64_t* empty_b = full_b + kMaxStages;  // both: stage free
    uint64_t* sfb_ready = empty_b + kMaxStages;  // leader: stage's scale atoms in TMEM
    uint64_t* acc_full = sfb_ready + kMaxStages;  // both: accumulator ready
    uint64_t* acc_empty = acc_full + 1;       // leader: both CTAs' epilogues hold their accumulator in registers
    uint64_t* drain = acc_empty + 1;          // leader: MMA teardown after an abort
    uint64_t* sf_drain = drain + 1;           // leader: [kSfWarps]
    int* s_pfx = reinterpret_cast<int*>(sf_drain + kSfWarps);  // [kMaxE + 1]
    int* s_off = s_pfx + kMaxE + 1;                             // [kMaxE]
    int* s_cnt = s_off + kMaxE;                                 // [kMaxE]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_cnt + kMaxE);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* dev_err = args.err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int E = args.num_experts, nb = args.n_blocks;
    const int sfb_col0 = kAccCols + 16 * KT;

    if (threadIdx.x == 0) {
        for (int k = 0; k < kMaxKt; ++k) {
            mbar_init(&full_a[k], 1);
            mbar_init(&empty_a[k], 1);
            mbar_init(&sfa_ready[k], kSfWarps);
        }
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&full_b[s], 1);
            mbar_init(&empty_b[s], 1);
            mbar_init(&sfb_ready[s], kSfWarps);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * kEpiWarps);
        mbar_init(drain, 1);
        for (int w = 0; w < kSfWarps; ++w) mbar_init(&sf_drain[w], 1);
        *cta_abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tma);
        prefetch_tensormap(&tmb_half);
        prefetch_tensormap(&tm_sfa);
        prefetch_tensormap(&tm_sfb);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
    // The gate/up kernel's A comes from the kernel right before it; the down
    // kernel (mt_wait) waits for its rows' counters instead.  The segment
    // offsets come from the permutation, which has completed in both cases.
    if (args.mt_wait == 0) pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    for (int e = threadIdx.x; e < E; e += kThreads) {
        s_off[e] = args.seg_off[e];
        s_cnt[e] = args.seg_cnt[e];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int ranges = (nb + kRange - 1) / kRange;
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            s_pfx[e] = acc;
            acc += ((((s_cnt[e] + 127) >> 7) + 1) >> 1) * ranges;
        }
        s_pfx[E] = acc;
    }
    tc_fence_before();
    cluster_sync();  // barriers initialised in both CTAs; TMEM allocated; items known
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int num_items = s_pfx[E];
    const int sf_atoms_per_rowblock = args.K / 64;
    const uint32_t full_a_leader = smem_in_cta(full_a, 0);
    const uint32_t full_b_leader = smem_in_cta(full_b, 0);
    const uint32_t acc_empty_leader = smem_in_cta(acc_empty, 0);

    if (warp == 0) {
        // ------------------------------ producer (both CTAs) -----------------
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        uint32_t b_parity[kMaxStages], a_parity[kMaxKt];
        bool b_issued[kMaxStages], a_issued[kMaxKt];
        for (int s = 0; s < kMaxStages; ++s) b_issued[s] = false, b_parity[s] = 0;
        for (int k = 0; k < kMaxKt; ++k) a_issued[k] = false, a_parity[k] = 0;
        const uint64_t stream_policy = l2_evict_first();  // B and its scales: read once per step
        int item_no = 0;
        for (int p = cluster; p < num_items && ok; p += nclusters, ++item_no) {
            const Item t = pair_item(s_pfx, s_off, s_cnt, E, nb, p);
            const uint32_t apar = static_cast<uint32_t>(item_no & 1);
            const int my_row0 = t.row0 + 128 * static_cast<int>(rank);
            const bool my_rows = t.m_valid > 128 * static_cast<int>(rank);
            if (args.mt_wait > 0 && my_rows) {
                // A and its scales are the gate/up kernel's output for these rows
                if (!wait_count(args.mt_done + my_row0 / 128, args.mt_wait, cta_abort, dev_err)) {
                    if (lane == 0) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                    ok = false;
                    break;
                }
                fence_proxy_async_global();
            }
            for (int n = t.n0; n < t.n1 && ok; ++n) {
                const int blk0 = (t.expert * args.b_nb + n) * args.b_kt;
                for (int kt = 0; kt < KT; ++kt) {
                    if (n == t.n0) {
                        // A chunk kt and its scale atoms, once the previous item's MMAs are done with the slot
                        if (lane == 0) {
                            if (!mbar_wait(&empty_a[kt], apar ^ 1u, cta_abort, dev_err)) {
                                set_abort(cta_abort, args.err, NF_DEVERR_WAIT_EMPTY);
                                ok = false;
                            } else if (leader) {
                                mbar_arrive_expect_tx(&full_a[kt], kATx);
                            }
                        }
                        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                        if (!ok) break;
                        const uint32_t bar = full_a_leader + 8u * kt;
                        if (lane == 0) {
                            tma_load_2d_pair_nohint(sA + kt * kAChunk, &tma, bar, kt * 128, my_row0);
                        } else if (lane == 2) {
                            // this CTA's 128-row block, chunk kt: 4 atoms = 8 rows of 256 bytes
                            const int atom = (my_row0 / 128) * sf_atoms_per_rowblock + kt * 4;
                            tma_load_2d_pair_nohint(sSFA + kt * kSfaChunk, &tm_sfa, bar, 0, atom * 2);
                        }
                        a_issued[kt] = true;
                        a_parity[kt] = apar;
                    }
                    if (lane == 0) {
                        if (!mbar_wait(&empty_b[stage], phase ^ 1u, cta_abort, dev_err)) {
                            set_abort(cta_abort, args.err, NF_DEVERR_WAIT_EMPTY);
                            ok = false;
                        } else if (leader) {
                            mbar_arrive_expect_tx(&full_b[stage], kBTx);
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                    if (!ok) break;
                    const uint32_t bar = full_b_leader + 8u * stage;
                    const int blk = blk0 + kt;
                    if (lane == 1) {
                        tma_load_2d_pair(sB + stage * kBStage, &tmb_half, bar, 0, blk * 256 + 128 * static_cast<int>(rank),
                                         stream_policy);
                    } else if (lane == 3) {
                        tma_load_2d_pair(sSFB + stage * kSfbStage, &tm_sfb, bar, 0, blk * 16, stream_policy);
                    }
                    b_issued[stage] = true;
                    b_parity[stage] = phase;
                    if (++stage == S) stage = 0, phase ^= 1u;
                }
            }
        }
        if (!ok && lane == 0) {
            // Teardown after an abort: the leader waits for the loads it
            // expected (their bytes come from both CTAs); the other CTA cannot
            // observe its copies' completion and waits a fixed 50 microseconds
            // for copies in flight to land before the final cluster barrier.
            if (leader) {
                for (int i = 0; i < kMaxStages + kMaxKt; ++i) {
                    uint64_t* b = i < kMaxStages ? &full_b[i] : &full_a[i - kMaxStages];
                    const bool was = i < kMaxStages ? b_issued[i] : a_issued[i - kMaxStages];
                    const uint32_t par = i < kMaxStages ? b_parity[i] : a_parity[i - kMaxStages];
                    if (!was) continue;
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(b, par)) {
                        if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) {
                            atomicCAS(args.err, 0, NF_DEVERR_DRAIN);
                            break;
                        }
                    }
                }
            } else {
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 50000ull) __nanosleep(1000);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (leader) --------------------
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0, acc_phase = 0;
            const uint32_t idesc = idesc_nvfp4(256, 256);
            bool ok = true;
            int item_no = 0;
            for (int p = cluster; p < num_items && ok; p += nclusters, ++item_no) {
                const Item t = pair_item(s_pfx, s_off, s_cnt, E, nb, p);
                const uint32_t apar = static_cast<uint32_t>(item_no & 1);
                for (int n = t.n0; n < t.n1; ++n) {
                    if (!mbar_wait_cluster(acc_empty, acc_phase ^ 1u, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kt = 0; kt < KT; ++kt) {
                        if (n == t.n0 && (!mbar_wait(&full_a[kt], apar, cta_abort, dev_err) ||
                                          !mbar_wait(&sfa_ready[kt], apar, cta_abort, dev_err))) {
                            set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&full_b[stage], phase, cta_abort, dev_err) ||
                            !mbar_wait(&sfb_ready[stage], phase, cta_abort, dev_err)) {
                            set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_base = smem_u32(sA + kt * kAChunk);
                        const uint32_t b_base = smem_u32(sB + stage * kBStage);
                        const uint32_t sfa_col = kAccCols + 16 * kt;
                        const uint32_t sfb_col = sfb_col0 + 32 * stage;
#pragma unroll
                        for (int s = 0; s < 4; ++s)
                            mma_nvfp4_pair(tmem, sdesc_sw128(a_base + 32 * s), sdesc_sw128(b_base + 32 * s), idesc,
                                           tmem + sfa_col + 4 * s, tmem + sfb_col + 8 * s,
                                           (kt > 0 || s > 0) ? 1u : 0u);
                        tc_commit_pair_both(&empty_b[stage]);
                        // the item's last use of A chunk kt (and its scale columns)
                        if (n == t.n1 - 1) tc_commit_pair_both(&empty_a[kt]);
                        if (++stage == S) stage = 0, phase ^= 1u;
                    }
                    if (!ok) break;
                    tc_commit_pair_both(acc_full);
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                tc_commit_pair(smem_u32(drain));
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
        // ------------------------------ epilogue (both CTAs) ---------------------
        // As the 1-SM kernel's 128-row epilogue, on this CTA's rows: a warp
        // reads TMEM lane quadrant warp % 4, four column slices per quadrant;
        // the accumulator goes back to the MMA warp once in registers.
        const int q = warp & 3;
        const int cs = (warp - 2) >> 2;
        const int r = q * 32 + lane;
        const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const bool epi_leader = warp == 2 && lane == 0;
        uint32_t acc_phase = 0;
        bool run = true;
        for (int p = cluster; p < num_items && run; p += nclusters) {
            const Item t = pair_item(s_pfx, s_off, s_cnt, E, nb, p);
            const int my_valid = min(128, max(0, t.m_valid - 128 * static_cast<int>(rank)));
            const int row = t.row0 + 128 * static_cast<int>(rank) + r;
            const bool valid = r < my_valid;
            const bool live = q * 32 < my_valid;
            for (int n = t.n0; n < t.n1; ++n) {
                // every warp waits for the accumulator itself (no hop through a leader)
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait_cluster(acc_full, acc_phase, cta_abort, dev_err) ? 1 : 0;
                    if (!ok) set_abort(cta_abort, args.err, NF_DEVERR_WAIT_ACC);
                }
                if (__shfl_sync(0xffffffffu, ok, 0) == 0) {
                    run = false;
                    break;
                }
                acc_phase ^= 1u;
                tc_fence_after();
                uint32_t v[64];
                if (live) {
                    if (EPI == EPI_SWIGLU_QUANT) {
                        tmem_ld16(tbase + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                        tmem_ld16(tbase + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                        tmem_ld16(tbase + 128 + 32 * cs, *reinterpret_cast<uint32_t(*)[16]>(&v[32]));
                        tmem_ld16(tbase + 128 + 32 * cs + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[48]));
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            tmem_ld16(tbase + 64 * cs + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]));
                    }
                    tmem_wait_ld();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (leader) mbar_arrive(acc_empty);
                    else mbar_arrive_cluster(acc_empty_leader);
                }
                if (live) {
                    if (EPI == EPI_SWIGLU_QUANT) {
                        const float ag = args.alpha0[t.expert], au = args.alpha1[t.expert];
                        const float gsd = args.gscale_next[t.expert], L = args.limit;
                        const bool sbf = args.swiglu_bf16 != 0;
                        const float* os_tab = args.os_table ? args.os_table + 256 * t.expert : nullptr;
                        uint32_t cc[2][2];
                        uint32_t sc[2];
#pragma unroll
                        for (int g = 0; g < 2; ++g)
                            sc[g] = swiglu_quant_group(&v[16 * g], &v[32 + 16 * g], ag, au, gsd, L, sbf, os_tab, cc[g]);
                        if (valid) {
                            uint8_t* o = static_cast<uint8_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                         n * 64 + cs * 16;
                            *reinterpret_cast<uint4*>(o) = make_uint4(cc[0][0], cc[0][1], cc[1][0], cc[1][1]);
                            *reinterpret_cast<uint16_t*>(args.out_sf +
                                                         sf_atom_offset(row, n * 8 + cs * 2, args.out_kgroups)) =
                                static_cast<uint16_t>(sc[0] | (sc[1] << 8));
                        }
                    } else {  // EPI_STORE_BF16
                        const float a = args.alpha0[t.expert];
                        uint32_t pk[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            pk[j] = bf16x2_hw(__fmul_rn(__uint_as_float(v[2 * j]), a),
                                              __fmul_rn(__uint_as_float(v[2 * j + 1]), a));
                        if (valid) {
                            uint16_t* d = static_cast<uint16_t*>(args.out) + static_cast<int64_t>(row) * args.out_ld +
                                          n * 256 + 64 * cs;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                st_global_v8(d + 16 * j, pk[8 * j], pk[8 * j + 1], pk[8 * j + 2], pk[8 * j + 3],
                                             pk[8 * j + 4], pk[8 * j + 5], pk[8 * j + 6], pk[8 * j + 7]);
                        }
                    }
                }
                if (EPI == EPI_SWIGLU_QUANT && args.mt_signal) {
                    // count this CTA's 128 rows for the down GEMM once every warp's stores are out
                    named_bar_sync(2, 32 * kEpiWarps);
                    if (epi_leader && my_valid > 0) {
                        __threadfence();
                        fence_proxy_async_global();
                        atomicAdd(args.mt_done + (t.row0 + 128 * static_cast<int>(rank)) / 128, 1);
                    }
                }
            }
        }
    } else if (leader && lane == 0) {
        // --------------------------- scale-atom copies (leader) -------------------
        // Each CTA's atoms from its own shared memory into its own TMEM: an
        // item's A atoms once (with its first block), every stage's B atoms;
        // the two warps split each group and both commit.
        const int sw = warp - kSfWarp0;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int item_no = 0;
        for (int p = cluster; p < num_items && ok; p += nclusters, ++item_no) {
            const Item t = pair_item(s_pfx, s_off, s_cnt, E, nb, p);
            const uint32_t apar = static_cast<uint32_t>(item_no & 1);
            for (int n = t.n0; n < t.n1 && ok; ++n) {
                for (int kt = 0; kt < KT; ++kt) {
                    if (n == t.n0) {
                        if (!mbar_wait(&full_a[kt], apar, cta_abort, dev_err)) {
                            set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                            ok = false;
                            break;
                        }
                        for (int c = sw; c < 4; c += kSfWarps)
                            tmem_cp_sf_pair(tmem + kAccCols + 16 * kt + 4 * c,
                                            sdesc_sf_atom(smem_u32(sSFA + kt * kSfaChunk + c * 512)));
                        tc_commit_pair(smem_u32(&sfa_ready[kt]));
                    }
                    if (!mbar_wait(&full_b[stage], phase, cta_abort, dev_err)) {
                        set_abort(cta_abort, args.err, NF_DEVERR_WAIT_FULL);
                        ok = false;
                        break;
                    }
                    for (int c = sw; c < 8; c += kSfWarps) {
                        const int s = c & 3, w = c >> 2;  // k-step, B row half
                        tmem_cp_sf_pair(tmem + sfb_col0 + 32 * stage + 8 * s + 4 * w,
                                        sdesc_sf_atom(smem_u32(sSFB + stage * kSfbStage + w * 2048 + s * 512)));
                    }
                    tc_commit_pair(smem_u32(&sfb_ready[stage]));
                    if (++stage == S) stage = 0, phase ^= 1u;
                }
            }
        }
        if (!ok) {
            tc_commit_pair(smem_u32(&sf_drain[sw]));
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&sf_drain[sw], 0)) {
                if (globaltimer_ns() - t0 > NF_WAIT_BUDGET_NS) {
                    atomicCAS(args.err, 0, NF_DEVERR_DRAIN);
                    break;
                }
            }
        }
    }

    // Neither CTA leaves (or frees TMEM) while the other may still signal its
    // barriers or the leader's MMAs may still read its shared memory.
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool gemm2_supported(const GemmArgs& a) {
    return a.kind == KIND_NVFP4 && (a.epi == EPI_SWIGLU_QUANT || a.epi == EPI_STORE_BF16) && a.dense_rows == 0 &&
           a.K % 256 == 0 && a.K / 256 >= 1 && a.K / 256 <= kMaxKt && a.num_experts > 0 && a.num_experts <= kMaxE &&
           a.seg_off && a.seg_cnt;
}

int gemm2_grid(int device) {
    // clusters of 2 that fit at once with one CTA per SM
    static int grid[kMaxDevices] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= kMaxDevices) return 0;
    if (grid[device] == 0) {
        const int smem = pair_smem(kMaxKt, pair_stages(kMaxKt));
        cudaFuncSetAttribute(gemm2_kernel<EPI_SWIGLU_QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        cudaFuncSetAttribute(gemm2_kernel<EPI_STORE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sms / 2));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm2_kernel<EPI_SWIGLU_QUANT>, &cfg) != cudaSuccess ||
            clusters <= 0) {
            cudaGetLastError();
            clusters = sms / 2;
        }
        grid[device] = 2 * std::min(clusters, sms / 2);
    }
    return grid[device];
}

cudaError_t launch_gemm2(const CUtensorMap& tma, const CUtensorMap& tmb_half, const CUtensorMap& tm_sfa,
                         const CUtensorMap& tm_sfb, const GemmArgs& args, int grid, bool dependent, cudaStream_t st) {
    if (!gemm2_supported(args) || grid < 2 || grid % 2 != 0) return cudaErrorInvalidValue;
    const int kt = args.K / 256;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pair_smem(kt, pair_stages(kt));
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    int n = 0;
    if (dependent) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    if (args.epi == EPI_SWIGLU_QUANT)
        return cudaLaunchKernelEx(&cfg, gemm2_kernel<EPI_SWIGLU_QUANT>, tma, tmb_half, tm_sfa, tm_sfb, args);
    return cudaLaunchKernelEx(&cfg, gemm2_kernel<EPI_STORE_BF16>, tma, tmb_half, tm_sfa, tm_sfb, args);
}

}  // namespace nf
