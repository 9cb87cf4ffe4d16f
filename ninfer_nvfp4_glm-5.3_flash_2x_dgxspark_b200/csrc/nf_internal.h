// nf_internal.h -- declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cstring>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nf {

// One GEMM work tile: 128 permuted rows of one expert x one 256-wide block
// of output columns.
struct NfTile {
    int32_t expert;
    int32_t row0;     // first permuted row (a multiple of 128)
    int32_t n_block;  // 256-column output block
    int32_t m_valid;  // rows of the tile that belong to the expert
};

// Device buffers the permutation kernels write.
struct PermuteBuffers {
    int32_t* chunk_counts;  // [nchunks, E]
    int32_t* chunk_base;    // [nchunks, E]
    int32_t* counts;        // [E]
    int32_t* seg_off;       // [E + 1]
    int32_t* pair_row;      // [T, K]
    int32_t* row_token;     // [rows_cap]
    NfTile* tiles_gu;       // gate/up tile list
    NfTile* tiles_down;     // down tile list
    int32_t* meta;          // [0] rows in use, [1] gate/up tiles, [2] down tiles, [3] m-tiles,
                            // [4] / [5] gate/up / down tile counters (reset here)
    int32_t* mt_done;       // [rows_cap / 128] gate/up tiles finished per m-tile (GemmArgs::mt_done; reset here)
    uint8_t* a_codes;       // NVFP4 dispatch: [rows_cap, H/2]
    uint8_t* a_sf;          //                 scale atoms
    uint16_t* a_bf16;       // BF16 dispatch:  [rows_cap, H]
};

// Epilogue kinds of the tcgen05 GEMM.
enum GemmEpi : int {
    EPI_SWIGLU_QUANT = 0,  // NVFP4 gate/up: alpha, BF16 round, clamped SwiGLU, NVFP4 quantise for down
    EPI_STORE_BF16 = 1,    // NVFP4 down: alpha, BF16 round, store BF16
    EPI_SWIGLU_BF16 = 2,   // BF16 gate/up: clamped SwiGLU in fp32, store BF16 h
    EPI_STORE_F32 = 3      // BF16 down: store F32
};

// Operand kinds.
enum GemmKind : int { KIND_NVFP4 = 0, KIND_BF16 = 1 };
constexpr int kEpMaxRanks = 8;  // expert-parallel group size limit

struct GemmArgs {
    int kind;            // GemmKind
    int epi;             // GemmEpi
    int K;               // reduction length in elements
    int b_nb;               // B is stored in box order: 256-row blocks per expert ...
    int b_kt;               // ... each split into b_kt blocks of 128 bytes of K
    const uint8_t* b;       // B in box order (32 KB blocks of 256 rows x 128 bytes); read through `tmb`
    // tile source: grouped (tiles + device tile count) or dense
    const NfTile* tiles;
    const int32_t* num_tiles_dev;
    int dense_rows;      // > 0: dense GEMM over this many A rows
    int n_blocks;        // 256-wide output blocks
    // Split K (dense GEMMs only): every (m, n) output tile is computed as
    // k_split partial sums over slices of kt_per K stages; slice s stores its
    // raw fp32 accumulator (EPI_STORE_F32) at out + s * out_split_stride, and
    // a reduction kernel sums the slices.  k_split = 1: no split.
    int k_split;
    int kt_per;
    int m_pair;                // dense BF16 only: 256-row tiles (two 128-row accumulators)
    int64_t out_split_stride;  // elements
    // Split K with the reduction fused (every tile on its own CTA, so all of a
    // tile's slices are in flight together): after storing its slice a CTA
    // counts it in splitk_cnt[m tile * n_blocks + n block] (zeroed before the
    // launch), waits until all k_split are stored, then sums its share of the
    // tile's rows over the slices in order into y: bf16(alpha0[0] * sum) +
    // residual (residual may be NULL) -- the reduction kernel's arithmetic.
    int splitk_fuse;
    int* splitk_cnt;
    // EPI_SWIGLU_QUANT over dense rows 33-64: A's rows 64-127 repeat rows 0-63
    // (the dispatch writes each token twice), so every epilogue warp has rows
    int rep64;
    // Dense tiles with a CTA each (grid >= tiles): CTA b takes tile b and no
    // other, without the tile counter, so it may claim it (and issue its
    // first B stages) before the previous kernel completes
    int static_tiles;
    // Expert-parallel return fused into the down GEMM (EPI_STORE_BF16 over
    // the [world][cap] receive slots, peer memory): permuted row `row` holds
    // receive slot j = row_token[row] = source * ep_cap + k and its output
    // row goes straight to ep_mbox[source] + ep_ret_off + (ep_src_off[source]
    // + k) * row bytes; the CTA that finishes the last tile (or CTA 0 when
    // there is none) publishes flag ep_flags_ret[ep_me] = *ep_epoch + 1 in
    // every source's mailbox after a system-scope fence.
    int ep_ret;
    int ep_world, ep_me, ep_cap;
    int64_t ep_ret_off, ep_flags_ret;
    uint8_t* ep_mbox[kEpMaxRanks];
    const int32_t* ep_src_off;
    const uint32_t* ep_epoch;
    int32_t* ep_tiles_done;    // zero before the launch; reset by the CTA that publishes
    const float* residual;
    float* y;
    // NVFP4 scale-factor atoms: sfa [128-row block][K/64 atoms]; sfb in tile
    // order, one 4 KB group per (expert, n block, K stage): [2 row halves][4 atoms]
    const uint8_t* sfa;
    const uint8_t* sfb;
    // epilogue
    const float* alpha0;       // [E] gate alpha (SwiGLU) or down alpha
    const float* alpha1;       // [E] up alpha (SwiGLU)
    const float* gscale_next;  // [E] 1 / input_scale of the down projection
    const float* os_table;     // [E][256] the down input quantiser's output scale per E4M3 scale code
                               // (1 / (scale / gscale_next), or NULL: computed per group)
    float limit;               // swiglu_limit
    int swiglu_bf16;           // EPI_SWIGLU_QUANT: swiglu_clamp_bf16 (dense layers: BF16 after the clamps,
                               // SiLU and product) instead of swiglu_clamp
    const int32_t* row_token;  // permuted row -> token (-1 = padding), NULL for dense
    void* out;                 // output rows
    int64_t out_ld;            // output row stride in elements of the output type
    uint8_t* out_sf;           // EPI_SWIGLU_QUANT: down-input scale atoms
    int out_kgroups;           // EPI_SWIGLU_QUANT: 16-groups per output row
    int* err;                  // device error word
    int* tile_counter;         // tiles claimed so far (zero before the launch)
    // Row-block hand-off between the gate/up and the down GEMM (both grouped):
    int* mt_done;              // per 128-row m-tile: gate/up tiles finished (zeroed by the permutation)
    int mt_signal;             // gate/up: count each finished tile in mt_done[row0 / 128]
    int mt_wait;               // down: > 0 loads a tile's A only once mt_done[row0 / 128] >= mt_wait,
                               // instead of waiting for the whole previous kernel (pdl_wait)
    int early_claim;           // the tile list and counter come from two or more launches back: claim
                               // the first tile and issue its first B stages before pdl_wait()
    int wide_stages;           // grouped NVFP4: 512-K stages; tma / tmb are make_tmap_a3 / make_tmap_b3 maps
    // CTA-pair GEMM (nf_gemm2.cu): the permutation's segments, from which it
    // derives its 256-row tiles
    int num_experts;
    const int32_t* seg_off;    // [E + 1] first permuted row of each expert (multiples of 128)
    const int32_t* seg_cnt;    // [E] rows of each expert
};

// Launches `kernel` with programmatic stream serialization: it may begin
// before the previous kernel in `st` has finished and calls pdl_wait()
// (nf_common.cuh) before it touches that kernel's results.
template <typename... P, typename... A>
cudaError_t launch_dependent(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// Host helpers (nf_gemm.cu).
bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner_elems, uint64_t rows,
                  uint32_t box_inner, uint32_t box_rows);
// B in box order as a 2-D byte tensor [bytes / 128 rows, 128] with 256-row
// boxes and 128-byte swizzle: box i is the 32 KB block i.
bool make_tmap_blocked(CUtensorMap* map, const void* base, uint64_t bytes, uint32_t box_rows = 256);
// 3-D maps for 512-K stages: A (FP4 rows of row_bytes) as [K / 256 chunks]
// [rows][128 B] with 128-row x 2-chunk boxes; B in box order as [blocks]
// [256 rows][128 B] with 2-block boxes.  128-byte swizzle.
bool make_tmap_a3(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows);
bool make_tmap_b3(CUtensorMap* map, const void* base, uint64_t bytes);
// A byte tensor [bytes / 256 rows, 256] without swizzle and box_rows-row
// boxes: contiguous runs of box_rows * 256 bytes (the scale-factor atoms).
bool make_tmap_runs(CUtensorMap* map, const void* base, uint64_t bytes, uint32_t box_rows);
// tma_small: the same A tensor with a 32-row box, used for tiles with <= 32
// rows; tmb: B (make_tmap_blocked over args.b).  dependent: launch_dependent
// (the kernel's CTAs may start, and hold their SMs, while the previous
// kernel in `st` still runs), else an ordinary launch.
cudaError_t launch_gemm(const CUtensorMap& tma, const CUtensorMap& tma_small, const CUtensorMap& tmb,
                        const GemmArgs& args, int grid, bool dependent, cudaStream_t st);
int gemm_grid_size(int device);
// The grouped NVFP4 GEMMs on CTA pairs (nf_gemm2.cu), for prefill-sized
// batches: tma as for launch_gemm (128-row boxes); tmb_half: B in box order
// with 128-row boxes; tm_sfa / tm_sfb: args.sfa / args.sfb as make_tmap_runs
// with 8- and 16-row boxes.  Grouped tiles only (args.seg_off / seg_cnt),
// K % 256 == 0, the SwiGLU-quantise and BF16-store epilogues.
bool gemm2_supported(const GemmArgs& args);
int gemm2_grid(int device);
cudaError_t launch_gemm2(const CUtensorMap& tma, const CUtensorMap& tmb_half, const CUtensorMap& tm_sfa,
                         const CUtensorMap& tm_sfb, const GemmArgs& args, int grid, bool dependent, cudaStream_t st);
// Weight matrices the GEMMs stream are kept in "box order" (nf_moe.cu): 32 KB
// blocks of 256 rows x 128 bytes, row-block major, K-block minor.
int64_t box_order_bytes(int64_t rows, int64_t row_bytes);
int64_t box_k_blocks(int64_t row_bytes);
// Host row-major [rows, row_bytes] (rows % 256 == 0) -> device box order.
cudaError_t upload_box_order(uint8_t* dst, const uint8_t* src, int64_t rows, int64_t row_bytes);

// Launchers (nf_kernels.cu).
// w_safe: every nonzero router weight has |w| in [2^-67, 2^63) (checked at
// bind), which lets the exact logit chains use fused multiply-add.
// Router weights in the fused router's chunk-major layouts (may be NULL):
// w_chunked32 (fp32, router_chunked_layout) for large batches, w_chunked16
// (BF16, router_chunked_layout16) for small ones.  With NULL the general
// two-kernel router runs on w.
cudaError_t launch_router(const uint16_t* x, const uint16_t* w, const float* w_chunked32, const uint16_t* w_chunked16,
                          const float* bias, int T, int H, int E, int K, float scaling, int normalize, int n_group,
                          int topk_group, int w_safe, float* logits, float* scores, float* choices, int32_t* idx,
                          float* wts, int* err, cudaStream_t st);

// Fused router (E <= kRouterMaxE, H % kRouterKc == 0): K streams in chunks of
// kRouterKc elements; a staged router row is kRouterPitch fp32 values or
// kRouterPitch16 BF16 values (16 bytes of padding keep the rows a warp reads
// in distinct shared-memory banks).
constexpr int kRouterMaxE = 128;
constexpr int kRouterKc = 128;
constexpr int kRouterPitch = kRouterKc + 4;
constexpr int kRouterPitch16 = kRouterKc + 8;
inline int64_t router_chunks(int H) { return (H + kRouterKc - 1) / kRouterKc; }
inline int64_t router_chunked_elems(int E, int H) { return router_chunks(H) * E * kRouterPitch; }
inline int64_t router_chunked_elems16(int E, int H) { return router_chunks(H) * E * kRouterPitch16; }
// BF16 [E, H] -> fp32 [chunk][E][kRouterPitch], padding zero (host side)
inline void router_chunked_layout(const uint16_t* w, int E, int H, float* out) {
    for (int64_t c = 0; c < router_chunks(H); ++c)
        for (int e = 0; e < E; ++e) {
            float* dst = out + (c * E + e) * kRouterPitch;
            for (int k = 0; k < kRouterPitch; ++k) {
                const int64_t col = c * kRouterKc + k;
                uint32_t bits = 0u;
                if (k < kRouterKc && col < H) bits = static_cast<uint32_t>(w[static_cast<int64_t>(e) * H + col]) << 16;
                std::memcpy(dst + k, &bits, sizeof(float));
            }
        }
}
// BF16 [E, H] -> BF16 [chunk][E][kRouterPitch16], padding zero (host side)
inline void router_chunked_layout16(const uint16_t* w, int E, int H, uint16_t* out) {
    for (int64_t c = 0; c < router_chunks(H); ++c)
        for (int e = 0; e < E; ++e) {
            uint16_t* dst = out + (c * E + e) * kRouterPitch16;
            for (int k = 0; k < kRouterPitch16; ++k) {
                const int64_t col = c * kRouterKc + k;
                dst[k] = (k < kRouterKc && col < H) ? w[static_cast<int64_t>(e) * H + col] : uint16_t(0);
            }
        }
}
// one_kernel: set when the permutation and the dispatch ran as one kernel
// (small batches), so the kernel after it must not read the tile lists before
// pdl_wait().
// The dense MLP's dispatch (rows = tokens, no permutation; resets the GEMMs'
// tile and hand-off counters).
cudaError_t launch_dense_dispatch(const uint16_t* x, int T, int H, const float* gscale, const float* os_tab_g,
                                  PermuteBuffers& b, int* splitk_cnt, int n_splitk_cnt, bool rep64, cudaStream_t st);
// os_tab_g: [E][256] the NVFP4 activation quantiser's output scale per E4M3
// scale code for each expert's gate input scale (NULL: computed per group).
cudaError_t launch_permute(const int32_t* idx, const uint16_t* x, int T, int K, int E, int H, int nb_gu, int nb_down,
                           const float* gscale, const float* os_tab_g, int bf16_mode, PermuteBuffers& b, cudaStream_t st,
                           bool* one_kernel);
cudaError_t launch_combine(const void* down, bool down_bf16, const int32_t* pair_row, const float* topk_w,
                           const float* shared, const float* residual, int T, int K, int H, float* y,
                           cudaStream_t st);
// y [T, H] = bf16(alpha[0] * sum of S fp32 slices part + s * stride) (+ residual):
// the split-K form of a dense down projection and its residual.
cudaError_t launch_splitk_store(const float* part, int S, int64_t stride, int T, int H, const float* alpha,
                                const float* residual, float* y, int grid_cap, cudaStream_t st);
// Expert parallelism (up to kEpMaxRanks ranks): the (destination, token,
// pick) layout of the picks (route [2 experts]: expert e's destination rank,
// then its index there), and a row gather.
cudaError_t launch_ep_pack(const int32_t* idx, int T, int K, const int32_t* route, int experts, int world, int32_t* slot,
                           int32_t* send_tok, int32_t* send_e, int32_t* counts, cudaStream_t st);
cudaError_t launch_gather_rows(const void* src, const int32_t* map, int n, int row_bytes, void* dst, cudaStream_t st);
// Expert parallelism over NVLink peer memory (CUDA IPC mailboxes).  A rank's
// mailbox holds, at these byte offsets: per-source receive flags, per-owner
// return flags (uint32 epochs), per-source row counts and send offsets, the
// received rows' destination-local experts [world][cap] and BF16 rows
// [world][cap][H], and the outputs of this rank's own sent rows [cap][row].
struct EpLayout {
    int64_t flags_recv, flags_ret, cnt, off, e, rows, ret, total;
    int cap;  // rows a source can send to one owner: max_tokens * top_k
};
struct EpPeers {
    uint8_t* mbox[kEpMaxRanks];  // every rank's mailbox mapped into this process (own included)
};
cudaError_t launch_ep_p2p_send(const uint16_t* x, const int32_t* send_tok, const int32_t* send_e,
                               const int32_t* counts, int H, int world, int me, const EpPeers& peers,
                               const EpLayout& lay, const uint32_t* epoch, int32_t* done, cudaStream_t st);
cudaError_t launch_ep_p2p_recv_wait(uint8_t* mbox, const EpLayout& lay, int world, const uint32_t* epoch,
                                    int32_t* seen, int* err, cudaStream_t st);
cudaError_t launch_ep_p2p_return(const void* down, const int32_t* pair_row, int out_bytes, int world, int me,
                                 const EpPeers& peers, const EpLayout& lay, const uint8_t* mbox, const int32_t* seen,
                                 const uint32_t* epoch, int32_t* done, cudaStream_t st);
cudaError_t launch_ep_p2p_ret_wait(const uint8_t* mbox, const EpLayout& lay, int world, uint32_t* epoch, int* err,
                                   cudaStream_t st);
cudaError_t launch_dequant(const uint8_t* packed, const uint8_t* scales, float gscale, int64_t rows, int64_t cols,
                           float* out, cudaStream_t st);
cudaError_t launch_quantize(const float* x, int64_t rows, int64_t cols, float gscale, uint8_t* codes,
                            uint8_t* scales, float* fake, cudaStream_t st);
cudaError_t launch_sigmoid_ref(const float* x, int64_t n, float* y, cudaStream_t st);
cudaError_t launch_f32_to_bf16(const float* x, int64_t n, uint16_t* y, cudaStream_t st);
cudaError_t launch_format_selfcheck(unsigned long long* mismatches_dev, cudaStream_t st);
// Builds the per-device lookup index of the router's sigmoid exception table
// (once per device; the calling thread's current device).
cudaError_t prepare_device_tables();

// Attention side of a decoder layer (nf_attn.cu; head dimension 128).
// A split of the context's partial softmax state: running max and sum.
struct AttnPart {
    float m, l;
};
constexpr int kAttnMaxSplitsHost = 64;  // splits of the context per (sequence, head)
cudaError_t launch_embed(const uint16_t* table, int64_t vocab, int H, const int32_t* tok, int T, float* x, int* err,
                         cudaStream_t st);
// RMSNorm per row; h = a (+ the sum of b's slices), h_out optional; stash:
// the rmsnorm_stash form.
cudaError_t launch_rmsnorm(const float* a, const float* b, int b_slices, int64_t b_stride, float* h_out, const float* w,
                           int rows, int n, float eps, int stash, uint16_t* y_bf16, float* y_f32, cudaStream_t st);
cudaError_t launch_qk_norm_rope(const float* qkv, int slices, int64_t stride, int T, int nq, int nkv,
                                const float* q_norm, const float* k_norm, float eps, float theta, const int32_t* pos,
                                int L_max, float* q_out, uint16_t* kc, uint16_t* vc, int* err, cudaStream_t st);
// splits of the context for T sequences (the partial buffers hold
// T * nq * splits pairs of floats and T * nq * splits * 128 floats)
int attn_splits(int T, int nkv, int L_max, int sms);
// tmk / tmv: the layer's K and V caches as 2-D BF16 tensors [seq * nkv * L_max,
// 128] with 64 x 32 boxes and 128-byte swizzle (make_tmap_2d)
cudaError_t launch_gqa_decode(const CUtensorMap& tmk, const CUtensorMap& tmv, const float* q, const int32_t* pos,
                              int T, int nq, int nkv, int L_max, int splits, AttnPart* part_ml, float* part_acc,
                              uint16_t* out, int* err, cudaStream_t st);

cudaError_t launch_fill_bf16_hash(uint16_t* p, int64_t n, uint64_t seed, cudaStream_t st);

// Screened router (large batches): candidates per token and the batch size
// from which forwards use it.  Both kernels take the router rows as the
// chunk-major BF16 copy (rows padded to kRouterPitch16) with E % 16 == 0,
// E <= kRouterMaxE and H % kRouterKc == 0; a stage that never lands sets
// `err` and the kernel leaves.
constexpr int kScreenMaxCandHost = 32;
constexpr int kScreenMinTokens = 1024;
// `tmx`: the tokens [T, H] BF16 as a 2-D map with 64 x 32 boxes and the
// 128-byte swizzle (make_tmap_2d(.., x, true, H, T, 64, 32)).
cudaError_t launch_route_screen(const CUtensorMap& tmx, const uint16_t* x, int T, int H, const uint16_t* wz16, int E,
                                int K, const float* bias, const float* wnorm, float c, int32_t* cand, int32_t* cnt,
                                float* approx, int* err, cudaStream_t st);
cudaError_t launch_route_exact(const CUtensorMap& tmx, const uint16_t* x, const uint16_t* wz16, const float* bias, int T,
                               int H, int E, int K,
                               float scaling, int normalize, int w_safe, const int32_t* cand, const int32_t* cnt,
                               int32_t* idx, float* wts, int* err, cudaStream_t st);

constexpr int kChunkTokHost = 128;  // tokens per permutation chunk (nf_kernels.cu kChunkTok)
// Per-device one-time state (kernel attributes, lookup tables) is kept in
// arrays of this many devices.
constexpr int kMaxDevices = 64;

}  // namespace nf
