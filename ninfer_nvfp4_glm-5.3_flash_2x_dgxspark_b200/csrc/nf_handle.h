// nf_handle.h -- the nf_moe handle (private to the library's host code) and
// the internal entry points nf_moe.cu shares with nf_ep.cu.
#pragma once

#include "nf_moe.h"

#include "nf_internal.h"

#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

using nf::PermuteBuffers;

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
};

struct nf_moe {
    nf_moe_desc d{};
    int device = 0;
    int grid = 148;
    cudaStream_t stream = nullptr;   // internal stream of the host-buffer path
    cudaStream_t side = nullptr;     // shared expert, forked from the caller's stream
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    int* shared_counters = nullptr;  // tile counters of the two shared-expert GEMMs
    std::string err;
    bool finalized = false;
    std::vector<DevBuf> allocs;

    // sizes
    int rows_cap = 0, nchunks_cap = 0, mtiles_cap = 0;

    // weights
    uint16_t* router_w = nullptr;   // [E, H]
    float* router_wz = nullptr;     // fused router's fp32 chunk-major copy (E <= kRouterMaxE)
    uint16_t* router_wz16 = nullptr;  // and its BF16 chunk-major copy
    float* router_bias = nullptr;   // [E]
    uint8_t* w_gu = nullptr;        // NVFP4 [E * 2I, H/2], 128-row gate/up interleave
    uint8_t* w_gu_sf = nullptr;     // scale atoms in tile order (GemmArgs::sfb)
    uint8_t* w_dn = nullptr;        // NVFP4 [E * H, I/2]
    uint8_t* w_dn_sf = nullptr;     // scale atoms in tile order
    uint16_t* wb_gu = nullptr;      // BF16 experts [E * 2I, H]
    uint16_t* wb_dn = nullptr;      // BF16 experts [E * H, I]
    uint16_t* ws_gu = nullptr;      // shared [2 Is, H]
    uint16_t* ws_dn = nullptr;      // shared [H, Is]
    float* alpha_g = nullptr;       // [E] weight_scale_2 * input_scale
    float* alpha_u = nullptr;
    float* alpha_d = nullptr;
    float* gs_g = nullptr;          // [E] 1 / input_scale
    float* gs_d = nullptr;
    float* os_tab = nullptr;  // [E][256] the down input quantiser's output scale per scale code
    float* os_tab_g = nullptr;  // [E][256] the same for the gate/up input (the dispatch's quantiser)
    std::vector<float> h_alpha_g, h_alpha_u, h_alpha_d, h_in_g, h_in_u, h_in_d;
    std::vector<uint8_t> bound;     // [E * 3] expert projection bound flags
    bool router_bound = false, bias_bound = false, sg_bound = false, su_bound = false, sd_bound = false;
    int router_w_safe = 0;  // every nonzero router weight has |w| in [2^-67, 2^63)
    // screened router for large batches (nf_kernels.cu route_screen_kernel):
    // the router rows' 2-norms rounded up and the candidates of each token
    bool screen = false;
    float* router_wnorm = nullptr;
    int32_t* screen_cand = nullptr;   // [Tm][32]
    int32_t* screen_cnt = nullptr;    // [Tm]: candidates, -1 = every chain
    int last_screened = 0;            // the last forward's router was screened

    // workspace
    float* logits = nullptr;         // router logits, sigmoid scores and choices [Tm, E]
    float* scores = nullptr;
    float* choices = nullptr;
    int32_t* topk_idx = nullptr;
    float* topk_w = nullptr;
    PermuteBuffers pb{};
    uint8_t* h_codes = nullptr;
    uint8_t* h_sf = nullptr;
    uint16_t* h_bf16 = nullptr;
    void* down = nullptr;           // BF16 (NVFP4 experts) or F32 (BF16 experts)
    uint16_t* sh_h = nullptr;       // [Tm, Is]
    float* sh_out = nullptr;        // [Tm, H]
    float* x_f32 = nullptr;         // host-path staging
    uint16_t* x_bf16 = nullptr;
    float* res_f32 = nullptr;
    float* y_f32 = nullptr;
    int* dev_err = nullptr;

    // expert parallelism (nf_moe_create_ep): the outer handle routes, runs
    // the shared expert, packs and exchanges rows and combines; `inner` is an
    // experts-only handle over this rank's experts
    bool ep_outer = false;
    bool experts_only = false;
    // dense MLP (nf_moe_create_dense): an experts-only handle with one expert
    // that every token takes with weight 1, and the swiglu_clamp_bf16 epilogue
    bool dense = false;
    int32_t* dense_idx = nullptr;    // [Tm] zeros: every token's pick is expert 0
    float* dense_w = nullptr;        // [Tm] ones: the pick's combine weight
    float* dense_part = nullptr;     // split-K partial sums of the down projection (small batches)
    int64_t dense_part_elems = 0;
    int* splitk_cnt = nullptr;       // [m tiles][H / 256] slices stored per down tile (fused reduction)
    int splitk_cnt_elems = 0;
    int ep_rank = 0, ep_world = 1, ep_base = 0, ep_local = 0;
    // Replicated experts this rank holds beyond its own (inner handle slots
    // ep_local + j): their picks from this rank's tokens stay here.
    std::vector<int> ep_rep;
    int32_t* ep_route = nullptr;  // [2E]: destination rank of expert e, then its index there
    nf_moe* inner = nullptr;
    void* nccl = nullptr;            // ncclComm_t of the group
    uint16_t* ep_send = nullptr;     // [Tm*K, H] rows in (destination, token, pick) order
    int32_t* ep_send_e = nullptr;    // [Tm*K] destination-local expert of each sent row
    int32_t* ep_send_tok = nullptr;  // [Tm*K] source token of each sent row
    int32_t* ep_slot = nullptr;      // [Tm*K] (t, p) -> send slot: the combine's pair_row
    int32_t* ep_cnt = nullptr;       // [2 * world] send counts, then receive counts
    uint16_t* ep_recv = nullptr;     // [world*Tm*K, H] received rows
    int32_t* ep_recv_e = nullptr;    // [world*Tm*K]
    void* ep_back = nullptr;         // [world*Tm*K, H] expert outputs in receive order
    void* ep_ret = nullptr;          // [Tm*K, H] outputs returned, in send order
    int32_t* ep_hcnt = nullptr;      // pinned host copy of ep_cnt
    uint8_t* ep_stage = nullptr;     // staging of the set-up exchanges' host records
    // NVLink peer-memory transport (the default when every rank can map every
    // other rank's mailbox with CUDA IPC; NCCL point-to-point otherwise)
    bool ep_p2p = false;
    uint8_t* ep_mbox = nullptr;      // this rank's mailbox (nf::EpLayout)
    nf::EpLayout ep_lay{};
    nf::EpPeers ep_peers{};          // every rank's mailbox mapped here (own included)
    uint32_t* ep_epoch = nullptr;    // forwards completed (device counter, equal on every rank)
    int32_t* ep_done = nullptr;      // [2 * kEpMaxRanks] last-block counters (send, return)
    int32_t* ep_seen = nullptr;      // [kEpMaxRanks] rows received from each source this forward

    // tensor maps built at finalize
    CUtensorMap tm_a{}, tm_h{}, tm_shh{};
    CUtensorMap tm_a_s{}, tm_h_s{}, tm_shh_s{};  // 32-row boxes of the A operands
    CUtensorMap tm_b_gu{}, tm_b_dn{}, tm_bs_gu{}, tm_bs_dn{};  // B operands (routed, shared) in box order
    // CTA-pair GEMMs (nf_gemm2.cu, NVFP4 experts at prefill-sized batches):
    // B with 128-row boxes, the A operands' and B's scale atoms as runs
    CUtensorMap tm_b_gu_half{}, tm_b_dn_half{}, tm_sfa_a{}, tm_sfa_h{}, tm_sfb_gu{}, tm_sfb_dn{};
    int gemm_mode = 0;  // nf_moe_set_expert_gemm (NF_GEMM_*)
    // 512-K-stage maps of the one-SM grouped NVFP4 GEMMs (prefill-sized batches)
    CUtensorMap tm_a3{}, tm_h3{}, tm_b_gu3{}, tm_b_dn3{};
    bool wide_ok = false;
    int grid2 = 0;          // CTAs of the pair GEMMs (an even number; 0: not available)
    int last_tokens = 0;

    // graph mode (nf_moe_set_graph_mode): captured forwards by argument set
    struct GraphEntry {
        const void* x;
        const void* res;
        void* y;
        void* idx;
        void* w;
        int T;
        cudaStream_t s;
        cudaGraphExec_t exec;
        bool host;  // a host-buffer forward (copies included; the pointers are host pointers)
    };
    static constexpr size_t kMaxGraphs = 16;
    bool use_graphs = false;
    std::vector<GraphEntry> graphs;

    // per-stage event profile: a ring of event sets (a begin and an end event
    // per stage, recorded on the stream the stage runs on), folded into
    // stage_ms
    static constexpr int kProfSets = 64;
    static constexpr int kEvPerSet = 2 * NF_STAGE_COUNT;
    bool profiling = false;
    std::vector<cudaEvent_t> prof_ev;   // kProfSets * kEvPerSet
    std::vector<uint8_t> prof_used;     // set holds an unfolded forward
    std::vector<uint8_t> prof_mask;     // stages recorded by the set
    int prof_next = 0, prof_forwards = 0;
    double stage_ms[NF_STAGE_COUNT] = {};

    void fold(int set) {
        cudaEvent_t* ev = &prof_ev[static_cast<size_t>(set) * kEvPerSet];
        const uint8_t mask = prof_mask[static_cast<size_t>(set)];
        for (int s = 0; s < NF_STAGE_COUNT; ++s) {
            if (!(mask & (1u << s))) continue;
            cudaEventSynchronize(ev[2 * s + 1]);
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, ev[2 * s], ev[2 * s + 1]) == cudaSuccess) stage_ms[s] += ms;
        }
        prof_used[static_cast<size_t>(set)] = 0;
        ++prof_forwards;
    }
    // events of the set recording the current forward (nullptr when off)
    cudaEvent_t* prof_begin(int* set_out) {
        if (!profiling) return nullptr;
        const int set = prof_next;
        prof_next = (prof_next + 1) % kProfSets;
        if (prof_used[static_cast<size_t>(set)]) fold(set);
        prof_used[static_cast<size_t>(set)] = 1;
        prof_mask[static_cast<size_t>(set)] = 0;
        *set_out = set;
        return &prof_ev[static_cast<size_t>(set) * kEvPerSet];
    }

    int fail(int status, const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        err = buf;
        return status;
    }
    int cuda_fail(cudaError_t e, const char* what) {
        return fail(NF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    template <typename T>
    bool alloc(T** p, size_t count) {
        void* q = nullptr;
        const size_t bytes = count * sizeof(T) > 0 ? count * sizeof(T) : 16;
        if (cudaMalloc(&q, bytes) != cudaSuccess) return false;
        allocs.push_back({q, bytes});
        *p = static_cast<T*>(q);
        return true;
    }
    // frees one allocation of the handle before destroy
    void release(void* p) {
        for (size_t i = 0; i < allocs.size(); ++i)
            if (allocs[i].p == p) {
                cudaFree(p);
                allocs.erase(allocs.begin() + static_cast<std::ptrdiff_t>(i));
                return;
            }
    }
    size_t bytes_of(const void* p) const {
        for (const auto& a : allocs)
            if (a.p == p) return a.bytes;
        return 0;
    }
};

// Handle roles: a full layer, the experts-only engine of an EP rank, the
// outer handle of an EP rank, or a dense MLP.
enum HandleRole { kRoleFull = 0, kRoleExperts = 1, kRoleEpOuter = 2, kRoleDense = 3 };

// Stage timing of one forward (events recorded when profiling is on).
struct StageRec {
    nf_moe* h = nullptr;
    cudaEvent_t* ev = nullptr;
    int set = -1;
    void begin(int stage, cudaStream_t st) {
        if (!ev) return;
        cudaEventRecord(ev[2 * stage], st);
        h->prof_mask[static_cast<size_t>(set)] |= static_cast<uint8_t>(1u << stage);
    }
    void end(int stage, cudaStream_t st) {
        if (ev) cudaEventRecord(ev[2 * stage + 1], st);
    }
};

// nf_moe.cu
int validate_desc(const nf_moe_desc& d, std::string* err);
std::string& create_error();
int create_impl(const nf_moe_desc& d, int device, int role, nf_moe** out, std::string* err);
int launch_shared_expert(nf_moe* h, const uint16_t* x, int T, StageRec& rec, cudaStream_t s);
// The router of a forward (no logits out): the screened router for large
// batches when the handle has one, else the full exact router.
cudaError_t route_tokens(nf_moe* h, const uint16_t* x, int T, int32_t* idx, float* w, cudaStream_t s);
// down_split > 1 (dense handles): the down GEMM runs as a dense split-K GEMM
// into h->dense_part (down_split K slices) instead of writing h->down; when
// dense_splitk_fused(), it also reduces the slices into y (+ residual).
// epr: the expert-parallel return fused into the down GEMM (peer memory).
int launch_routed_experts(nf_moe* h, const uint16_t* x, const int32_t* idx, int T, int K, StageRec& rec,
                          cudaStream_t s, int down_split = 1, const float* residual = nullptr, float* y = nullptr,
                          const nf::GemmArgs* epr = nullptr);
// The dense split-K down GEMM reduces its slices itself when every tile gets
// its own CTA (so all slices of a tile run together).
bool dense_splitk_fused(const nf_moe* h, int T, int down_split);
// nf_ep.cu
int ep_forward(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, int32_t* idx, float* w,
               cudaStream_t s);
void ep_release(nf_moe* h);
