// nf_moe.cu -- the C ABI (include/nf_moe.h): handle, weight binding with the
// reference's validation, device layouts, and the forward pass that chains
// router -> permutation/dispatch -> grouped gate/up GEMM (SwiGLU + NVFP4
// quantisation fused) -> grouped down GEMM -> shared expert -> combine.
#include "nf_handle.h"

#include "nf_common.cuh"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace nf;

namespace {

thread_local std::string g_create_error;

}  // namespace

std::string& create_error() { return g_create_error; }

namespace {

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Batches from which the shared expert's GEMMs use 256-row tiles.
constexpr int kSharedPairTokens = 2048;

float e4m3_host(uint8_t bits) {
    const int exponent = (bits >> 3) & 0xf;
    const int mantissa = bits & 0x7;
    float magnitude;
    if (exponent == 0) magnitude = std::ldexp(static_cast<float>(mantissa), -9);
    else if (exponent == 15 && mantissa == 7) magnitude = NAN;
    else magnitude = std::ldexp(1.f + static_cast<float>(mantissa) / 8.f, exponent - 7);
    return (bits & 0x80u) ? -magnitude : magnitude;
}

int64_t sf_off_host(int64_t row, int64_t kg, int64_t kgroups) {
    const int64_t atom = (row >> 7) * (kgroups >> 2) + (kg >> 2);
    return atom * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (kg & 3);
}

// Validates block scales like Nvfp4MatrixView (src/nvfp4_decode.cpp:70-79)
// and converts row-major [rows, kgroups] E4M3 scales into 128x4 atoms
// (rows % 128 == 0).  -0 (0x80) is canonicalised to +0: both are the value 0
// and the tensor core reads the scale as unsigned.
bool scales_to_atoms(const uint8_t* scales, int64_t rows, int64_t kgroups, float gscale, std::vector<uint8_t>& out) {
    out.assign(static_cast<size_t>(rows * kgroups), 0);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t k = 0; k < kgroups; ++k) {
            uint8_t b = scales[r * kgroups + k];
            const float s = e4m3_host(b);
            if (!std::isfinite(s) || s < 0.f) return false;
            if (6.0 * static_cast<double>(s) * static_cast<double>(gscale) > static_cast<double>(FLT_MAX)) return false;
            if (b == 0x80) b = 0;
            out[static_cast<size_t>(sf_off_host(r, k, kgroups))] = b;
        }
    }
    return true;
}

// Scale atoms in tile order (GemmArgs::sfb): one 4 KB group per 256-row
// tile and 256-element K stage, [row half][4 atoms][512 B], zero padded
// past the last atom.  Places one projection's atoms ([128-row block][katoms]
// from scales_to_atoms) into an expert's groups `out`: a down projection
// fills both halves (row block rb -> tile rb / 2, half rb % 2), the gate or
// up projection (half = 0 / 1) the given half of tile rb.
int64_t sf_tile_bytes(int64_t tiles, int64_t katoms) { return tiles * ((katoms + 3) / 4) * 4096; }

void atoms_to_tiles(const std::vector<uint8_t>& atoms, int64_t rowblocks, int64_t katoms, int half,
                    std::vector<uint8_t>& out) {
    const int64_t kts = (katoms + 3) / 4;
    const int64_t tiles = half < 0 ? rowblocks / 2 : rowblocks;
    out.assign(static_cast<size_t>(sf_tile_bytes(tiles, katoms)), 0);
    for (int64_t rb = 0; rb < rowblocks; ++rb) {
        const int64_t tile = half < 0 ? rb / 2 : rb, b = half < 0 ? rb % 2 : half;
        for (int64_t a = 0; a < katoms; ++a)
            std::memcpy(&out[static_cast<size_t>((((tile * kts + a / 4) * 2 + b) * 4 + a % 4) * 512)],
                        &atoms[static_cast<size_t>((rb * katoms + a) * 512)], 512);
    }
}

const char* proj_name(int proj) { return proj == NF_PROJ_GATE ? "gate_proj" : proj == NF_PROJ_UP ? "up_proj" : "down_proj"; }

// Checkpoint name of a projection in messages: mlp.experts.<e>.<proj> for a
// routed expert, mlp.<proj> for the dense MLP (src/parameter_schema.cpp:187-191).
// K slices of a dense down projection over T tokens: when its (m, n) tiles
// would occupy fewer than half the SMs (small batches), K is split so that
// the slices fill the grid, at least 2 stages of 256 K-elements per slice
// and no empty slice.  Returns 1 for no split; *kt_per gets the stages per slice.
int dense_down_split(int T, int H, int I, int grid, int* kt_per) {
    const int m_tiles = (T + 127) / 128, n_blocks = H / 256, k_tiles = (I + 255) / 256;
    const int base = m_tiles * n_blocks;
    *kt_per = k_tiles;
    if (2 * base > grid || k_tiles < 4) return 1;
    const int want = std::max(1, grid / base);
    *kt_per = std::max(2, (k_tiles + want - 1) / want);
    return (k_tiles + *kt_per - 1) / *kt_per;
}

std::string proj_label(const nf_moe* h, long long expert, int proj) {
    if (h->dense) return std::string("mlp.") + proj_name(proj);
    return "mlp.experts." + std::to_string(expert) + "." + proj_name(proj);
}

// Weight matrices that the GEMMs stream (their B operands) are stored in
// "box order": the matrix is cut into blocks of 256 rows x 128 bytes (one
// pipeline stage of one tile; 256 FP4 or 64 BF16 K-elements), each block is
// 32 KB contiguous with 128-byte rows (zero padded past the row end), blocks
// ordered row-block major, K-block minor.  A stage is then one contiguous
// 32 KB region, which one TMA box (make_tmap_blocked) moves into shared
// memory in the 128-byte swizzled form the MMA operand descriptors read.
constexpr int64_t kBlockRows = 256, kBlockRowBytes = 128, kBlockBytes = kBlockRows * kBlockRowBytes;

int64_t k_blocks(int64_t row_bytes) { return (row_bytes + kBlockRowBytes - 1) / kBlockRowBytes; }
int64_t blocked_bytes(int64_t rows, int64_t row_bytes) { return (rows / kBlockRows) * k_blocks(row_bytes) * kBlockBytes; }

// One row piece (n bytes) into row `row` of a block.
void put_row(uint8_t* block, int64_t row, const uint8_t* src, int64_t n) {
    std::memcpy(block + row * kBlockRowBytes, src, static_cast<size_t>(n));
}

// Copies a row-major [rows, row_bytes] matrix (rows % 256 == 0) into box order.
cudaError_t upload_blocked(uint8_t* dst, const uint8_t* src, int64_t rows, int64_t row_bytes) {
    const int64_t nb = rows / kBlockRows, kt = k_blocks(row_bytes);
    std::vector<uint8_t> stage(static_cast<size_t>(nb * kt * kBlockBytes), 0);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < kt; ++k) {
            const int64_t n = std::min(kBlockRowBytes, row_bytes - k * kBlockRowBytes);
            put_row(&stage[static_cast<size_t>(((r / kBlockRows) * kt + k) * kBlockBytes)], r % kBlockRows,
                    src + r * row_bytes + k * kBlockRowBytes, n);
        }
    return cudaMemcpy(dst, stage.data(), stage.size(), cudaMemcpyHostToDevice);
}

// Copies one of the two halves of a gate/up pair into box order: source row
// j lands in row (j % 128) + 128 * half of row block j / 128 (the 256-row
// blocks hold 128 gate rows then the 128 up rows of the same intermediate
// columns).  `dst` is the expert's first block.
cudaError_t upload_blocked_half(uint8_t* dst, const uint8_t* src, int64_t rows, int64_t row_bytes, int half) {
    const int64_t nb = rows / 128, kt = k_blocks(row_bytes), hb = kBlockBytes / 2;
    std::vector<uint8_t> stage(static_cast<size_t>(nb * kt * hb), 0);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < kt; ++k) {
            const int64_t n = std::min(kBlockRowBytes, row_bytes - k * kBlockRowBytes);
            put_row(&stage[static_cast<size_t>(((r / 128) * kt + k) * hb)], r % 128,
                    src + r * row_bytes + k * kBlockRowBytes, n);
        }
    return cudaMemcpy2D(dst + half * hb, static_cast<size_t>(kBlockBytes), stage.data(), static_cast<size_t>(hb),
                        static_cast<size_t>(hb), static_cast<size_t>(nb * kt), cudaMemcpyHostToDevice);
}

}  // namespace

namespace nf {
int64_t box_order_bytes(int64_t rows, int64_t row_bytes) { return blocked_bytes(rows, row_bytes); }
int64_t box_k_blocks(int64_t row_bytes) { return k_blocks(row_bytes); }
cudaError_t upload_box_order(uint8_t* dst, const uint8_t* src, int64_t rows, int64_t row_bytes) {
    return upload_blocked(dst, src, rows, row_bytes);
}
}  // namespace nf

extern "C" {

const char* nf_status_string(int s) {
    switch (s) {
        case NF_OK: return "ok";
        case NF_ERR_INVALID: return "invalid argument";
        case NF_ERR_SHAPE: return "shape mismatch";
        case NF_ERR_LAYOUT: return "layout mismatch";
        case NF_ERR_SCALE: return "bad scale";
        case NF_ERR_STATE: return "bad state";
        case NF_ERR_CUDA: return "CUDA error";
        case NF_ERR_TIMEOUT: return "device wait timed out";
        case NF_ERR_UNSUPPORTED: return "unsupported";
        case NF_ERR_NOMEM: return "out of device memory";
        case NF_ERR_CAPACITY: return "token capacity exceeded";
        default: return "unknown status";
    }
}

const char* nf_moe_last_error(const nf_moe* h) { return h ? h->err.c_str() : g_create_error.c_str(); }

void nf_moe_destroy(nf_moe* h) {
    if (!h) return;
    if (h->ep_outer) ep_release(h);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    if (h->stream) {
        cudaStreamSynchronize(h->stream);
        cudaStreamDestroy(h->stream);
    }
    if (h->side) {
        cudaStreamSynchronize(h->side);
        cudaStreamDestroy(h->side);
    }
    if (h->ev_fork) cudaEventDestroy(h->ev_fork);
    if (h->ev_join) cudaEventDestroy(h->ev_join);
    for (cudaEvent_t ev : h->prof_ev) cudaEventDestroy(ev);
    for (auto& g : h->graphs) cudaGraphExecDestroy(g.exec);
    for (auto& a : h->allocs) cudaFree(a.p);
    cudaSetDevice(prev);
    delete h;
}

}  // extern "C"

// The descriptor checks of nf_moe_create; NF_OK or a status with *err set.
int validate_desc(const nf_moe_desc& d, std::string* err) {
    auto reject = [&](int st, const char* msg) {
        if (err) *err = msg;
        return st;
    };
    if (d.hidden <= 0 || d.hidden % 256 != 0) return reject(NF_ERR_UNSUPPORTED, "hidden must be a positive multiple of 256");
    if (d.inter <= 0 || d.inter % 128 != 0) return reject(NF_ERR_UNSUPPORTED, "inter must be a positive multiple of 128");
    if (d.shared_inter < 0 || d.shared_inter % 128 != 0)
        return reject(NF_ERR_UNSUPPORTED, "shared_inter must be 0 or a multiple of 128");
    if (d.experts < 1 || d.experts > 1024) return reject(NF_ERR_UNSUPPORTED, "experts must be in [1, 1024]");
    if (d.top_k < 1 || d.top_k > 32 || d.top_k > d.experts) return reject(NF_ERR_UNSUPPORTED, "top_k must be in [1, min(32, experts)]");
    if (d.max_tokens < 1) return reject(NF_ERR_INVALID, "max_tokens must be positive");
    if (d.n_group < 1) return reject(NF_ERR_INVALID, "n_group must be >= 1");
    if (d.n_group > 1 && (d.n_group > 32 || d.experts % d.n_group != 0 || d.topk_group < 1 ||
                          d.topk_group > d.n_group || d.top_k > d.topk_group * (d.experts / d.n_group)))
        return reject(NF_ERR_UNSUPPORTED, "group-limited routing needs n_group <= 32 dividing experts and enough eligible experts");
    if (d.expert_kind != NF_EXPERTS_NVFP4 && d.expert_kind != NF_EXPERTS_BF16)
        return reject(NF_ERR_INVALID, "expert_kind must be NF_EXPERTS_NVFP4 or NF_EXPERTS_BF16");
    return NF_OK;
}

extern "C" {

int nf_moe_create(const nf_moe_desc* desc, int device, nf_moe** out) {
    g_create_error.clear();
    if (!desc || !out) {
        g_create_error = "null descriptor or output";
        return NF_ERR_INVALID;
    }
    *out = nullptr;
    const nf_moe_desc& d = *desc;
    const int st = validate_desc(d, &g_create_error);
    if (st != NF_OK) return st;
    return create_impl(d, device, kRoleFull, out, &g_create_error);
}

// TextModel::dense_mlp (src/text_forward.cpp:909-915) as a one-expert,
// router-less handle: every token takes expert 0 with weight 1, so the
// permutation is the identity (rows padded to 128), the grouped GEMMs run
// one segment, and the combine adds 1 * down to the residual exactly.
int nf_moe_create_dense(int32_t hidden, int32_t inter, float swiglu_limit, int32_t max_tokens, int device,
                        nf_moe** out) {
    g_create_error.clear();
    if (!out) {
        g_create_error = "null output";
        return NF_ERR_INVALID;
    }
    *out = nullptr;
    nf_moe_desc d{};
    d.hidden = hidden;
    d.experts = 1;
    d.top_k = 1;
    d.inter = inter;
    d.shared_inter = 0;
    d.n_group = 1;
    d.topk_group = 1;
    d.normalize = 1;
    d.routed_scaling = 1.f;
    d.swiglu_limit = swiglu_limit;
    d.expert_kind = NF_EXPERTS_NVFP4;
    d.max_tokens = max_tokens;
    const int st = validate_desc(d, &g_create_error);
    if (st != NF_OK) return st;
    return create_impl(d, device, kRoleDense, out, &g_create_error);
}

}  // extern "C"

// Allocates a handle for a validated descriptor.  kRoleExperts (the experts
// of an EP rank) has no router or shared expert; kRoleEpOuter has no routed
// experts or GEMM workspace (its experts live in the inner handle).
int create_impl(const nf_moe_desc& d, int device, int role, nf_moe** out, std::string* err) {
    auto reject = [&](int st, const char* msg) {
        if (err) *err = msg;
        return st;
    };
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return reject(NF_ERR_CUDA, "no such CUDA device");
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return reject(NF_ERR_CUDA, "cudaSetDevice failed");
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) {
        cudaSetDevice(prev);
        return reject(NF_ERR_UNSUPPORTED, "this library is built for sm_100a (B200)");
    }

    if (prepare_device_tables() != cudaSuccess) {
        cudaSetDevice(prev);
        return reject(NF_ERR_CUDA, "could not build the router's device tables");
    }
    nf_moe* h = new nf_moe();
    h->d = d;
    h->device = device;
    h->grid = gemm_grid_size(device);
    h->experts_only = role == kRoleExperts || role == kRoleDense;
    h->dense = role == kRoleDense;
    h->ep_outer = role == kRoleEpOuter;
    const bool routed = role != kRoleEpOuter, router = !h->experts_only;
    const int64_t H = d.hidden, E = d.experts, K = d.top_k, I = d.inter, Is = d.shared_inter, Tm = d.max_tokens;
    const int64_t pairs = Tm * K;
    h->rows_cap = static_cast<int>(round_up(pairs + 127 * E, 128));
    h->nchunks_cap = static_cast<int>((Tm + kChunkTokHost - 1) / kChunkTokHost);
    h->mtiles_cap = h->rows_cap / 128;
    const int64_t R = h->rows_cap;
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    bool ok = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) == cudaSuccess;
    if (router) {
        ok = ok && h->alloc(&h->router_w, E * H) && h->alloc(&h->router_bias, E);
        if (E <= kRouterMaxE)
            ok = ok && h->alloc(&h->router_wz, router_chunked_elems(E, H)) &&
                 h->alloc(&h->router_wz16, router_chunked_elems16(E, H));
        ok = ok && h->alloc(&h->logits, Tm * E) && h->alloc(&h->scores, Tm * E) && h->alloc(&h->choices, Tm * E);
        // the screened router, for handles that take prefill-sized batches
        h->screen = E <= kRouterMaxE && E % 16 == 0 && H % kRouterKc == 0 && Tm >= kScreenMinTokens;
        if (h->screen)
            ok = ok && h->alloc(&h->router_wnorm, E) && h->alloc(&h->screen_cand, Tm * kScreenMaxCandHost) &&
                 h->alloc(&h->screen_cnt, Tm);
    }
    if (routed) {
        if (fp4) {
            ok = ok && h->alloc(&h->w_gu, E * blocked_bytes(2 * I, H / 2)) &&
                 h->alloc(&h->w_gu_sf, E * sf_tile_bytes(I / 128, H / 64)) &&
                 h->alloc(&h->w_dn, E * blocked_bytes(H, I / 2)) && h->alloc(&h->w_dn_sf, E * sf_tile_bytes(H / 256, I / 64));
        } else {
            ok = ok && h->alloc(&h->wb_gu, E * blocked_bytes(2 * I, 2 * H) / 2) &&
                 h->alloc(&h->wb_dn, E * blocked_bytes(H, 2 * I) / 2);
        }
    }
    if (Is > 0) ok = ok && h->alloc(&h->ws_gu, blocked_bytes(2 * Is, 2 * H) / 2) && h->alloc(&h->ws_dn, blocked_bytes(H, 2 * Is) / 2);
    ok = ok && h->alloc(&h->alpha_g, E) && h->alloc(&h->alpha_u, E) && h->alloc(&h->alpha_d, E) &&
         h->alloc(&h->gs_g, E) && h->alloc(&h->gs_d, E) && h->alloc(&h->os_tab, E * 256) &&
         h->alloc(&h->os_tab_g, E * 256);
    ok = ok && h->alloc(&h->topk_idx, Tm * K) && h->alloc(&h->topk_w, Tm * K);
    PermuteBuffers& b = h->pb;
    if (routed) {
        ok = ok && h->alloc(&b.chunk_counts, static_cast<int64_t>(h->nchunks_cap) * E) &&
             h->alloc(&b.chunk_base, static_cast<int64_t>(h->nchunks_cap) * E) && h->alloc(&b.counts, E) &&
             h->alloc(&b.seg_off, E + 1) && h->alloc(&b.pair_row, pairs) && h->alloc(&b.row_token, R) &&
             h->alloc(&b.tiles_gu, static_cast<int64_t>(h->mtiles_cap) * (I / 128)) &&
             h->alloc(&b.tiles_down, static_cast<int64_t>(h->mtiles_cap) * (H / 256)) && h->alloc(&b.meta, 8) &&
             h->alloc(&b.mt_done, h->mtiles_cap);
    }
    ok = ok && h->alloc(&h->shared_counters, 2);
    ok = ok && cudaStreamCreateWithFlags(&h->side, cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreateWithFlags(&h->ev_fork, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&h->ev_join, cudaEventDisableTiming) == cudaSuccess;
    if (routed && fp4) {
        ok = ok && h->alloc(&b.a_codes, R * H / 2) && h->alloc(&b.a_sf, R * H / 16) && h->alloc(&h->h_codes, R * I / 2) &&
             h->alloc(&h->h_sf, R * I / 16);
        uint16_t* dn = nullptr;
        ok = ok && h->alloc(&dn, R * H);
        h->down = dn;
    } else if (routed) {
        ok = ok && h->alloc(&b.a_bf16, R * H) && h->alloc(&h->h_bf16, R * I);
        float* dn = nullptr;
        ok = ok && h->alloc(&dn, R * H);
        h->down = dn;
    }
    if (Is > 0) ok = ok && h->alloc(&h->sh_h, Tm * Is) && h->alloc(&h->sh_out, Tm * H);
    ok = ok && h->alloc(&h->x_f32, Tm * H) && h->alloc(&h->x_bf16, Tm * H) && h->alloc(&h->res_f32, Tm * H) &&
         h->alloc(&h->y_f32, Tm * H) && h->alloc(&h->dev_err, 1);
    if (h->dense) {
        ok = ok && h->alloc(&h->dense_idx, Tm) && h->alloc(&h->dense_w, Tm);
        // the largest split-K partial buffer over every batch size up to Tm
        int64_t part = 0;
        for (int64_t mt = 1; mt <= (Tm + 127) / 128; ++mt) {
            int kt_per = 0;
            const int S = dense_down_split(static_cast<int>(mt * 128), static_cast<int>(H), static_cast<int>(I), h->grid, &kt_per);
            if (S > 1) part = std::max(part, S * mt * 128 * H);
        }
        h->dense_part_elems = part;
        if (part > 0) ok = ok && h->alloc(&h->dense_part, part);
        h->splitk_cnt_elems = static_cast<int>((Tm + 127) / 128 * (H / 256));
        ok = ok && h->alloc(&h->splitk_cnt, h->splitk_cnt_elems);
    }
    if (!ok) {
        cudaGetLastError();
        nf_moe_destroy(h);
        cudaSetDevice(prev);
        return reject(NF_ERR_NOMEM, "device allocation failed");
    }
    cudaMemset(h->dev_err, 0, sizeof(int));
    if (routed) cudaMemset(b.row_token, 0xff, R * sizeof(int32_t));
    if (h->dense) {
        const std::vector<float> ones(static_cast<size_t>(Tm), 1.f);
        if (cudaMemset(h->dense_idx, 0, Tm * sizeof(int32_t)) != cudaSuccess ||
            cudaMemcpy(h->dense_w, ones.data(), Tm * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
            nf_moe_destroy(h);
            cudaSetDevice(prev);
            return reject(NF_ERR_CUDA, "dense MLP set-up copy failed");
        }
    }
    h->bound.assign(static_cast<size_t>(E * 3), 0);
    h->h_alpha_g.assign(E, 0.f);
    h->h_alpha_u.assign(E, 0.f);
    h->h_alpha_d.assign(E, 0.f);
    h->h_in_g.assign(E, 0.f);
    h->h_in_u.assign(E, 0.f);
    h->h_in_d.assign(E, 0.f);
    cudaSetDevice(prev);
    *out = h;
    return NF_OK;
}

extern "C" {

// An EP rank binds only the experts it owns (into its inner handle, with
// local ids); the others belong to other ranks and are skipped.  Inner
// failures come back with the expert's global id.
// The global expert id of inner slot `local` (own experts, then replicas).
static long long ep_global_expert(const nf_moe* h, long long local) {
    if (local < h->ep_local) return local + h->ep_base;
    const long long j = local - h->ep_local;
    return j < static_cast<long long>(h->ep_rep.size()) ? h->ep_rep[static_cast<size_t>(j)] : -1;
}

// The inner slot of global expert e on this rank, -1 when the rank holds none.
static int ep_inner_slot(const nf_moe* h, int e) {
    if (e >= h->ep_base && e < h->ep_base + h->ep_local) return e - h->ep_base;
    for (size_t j = 0; j < h->ep_rep.size(); ++j)
        if (h->ep_rep[j] == e) return h->ep_local + static_cast<int>(j);
    return -1;
}

static int ep_relay(nf_moe* h, int st) {
    if (st == NF_OK) return NF_OK;
    std::string m = h->inner->err;
    const size_t at = m.find("mlp.experts.");
    if (at != std::string::npos) {
        size_t end = at + 12;
        while (end < m.size() && m[end] >= '0' && m[end] <= '9') ++end;
        if (end > at + 12) {
            const long long local = std::atoll(m.substr(at + 12, end - at - 12).c_str());
            m = m.substr(0, at + 12) + std::to_string(ep_global_expert(h, local)) + m.substr(end);
        }
    }
    return h->fail(st, "%s", m.c_str());
}

int nf_moe_bind_nvfp4(nf_moe* h, int expert, int proj, const uint8_t* packed, const uint8_t* scales, float ws2,
                      float in_scale, int64_t rows, int64_t cols) {
    if (!h) return NF_ERR_INVALID;
    const nf_moe_desc& d = h->d;
    if (d.expert_kind != NF_EXPERTS_NVFP4) return h->fail(NF_ERR_STATE, "handle holds BF16 experts");
    if (h->finalized) return h->fail(NF_ERR_STATE, "weights are already finalized");
    if (expert < 0 || expert >= d.experts || proj < 0 || proj > 2) return h->fail(NF_ERR_INVALID, "bad expert or projection id");
    if (h->ep_outer) {
        const int slot = ep_inner_slot(h, expert);
        if (slot < 0) return NF_OK;
        return ep_relay(h, nf_moe_bind_nvfp4(h->inner, slot, proj, packed, scales, ws2, in_scale, rows, cols));
    }
    if (!packed || !scales) return h->fail(NF_ERR_LAYOUT, "NVFP4 layout %s", proj_label(h, expert, proj).c_str());
    const int64_t H = d.hidden, I = d.inter;
    const int64_t want_rows = proj == NF_PROJ_DOWN ? H : I, want_cols = proj == NF_PROJ_DOWN ? I : H;
    if (rows != want_rows || cols != want_cols || cols % 16 != 0)
        return h->fail(NF_ERR_SHAPE, "NVFP4 shape %s", proj_label(h, expert, proj).c_str());
    if (!(in_scale > 0.f) || !std::isfinite(in_scale)) return h->fail(NF_ERR_SCALE, "NVFP4 input scale");
    if (!std::isfinite(ws2) || ws2 < FLT_MIN)
        return h->fail(NF_ERR_SCALE, "NVFP4 global scale must be finite and at least the minimum normal float");
    std::vector<uint8_t> atoms;
    if (!scales_to_atoms(scales, rows, cols / 16, ws2, atoms))
        return h->fail(NF_ERR_SCALE, "NVFP4 block scales must be finite and nonnegative");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaSuccess;
    const int64_t kbytes = cols / 2, katoms = cols / 64;
    std::vector<uint8_t> groups;
    if (proj == NF_PROJ_DOWN) {
        e = upload_blocked(h->w_dn + expert * blocked_bytes(H, kbytes), packed, H, kbytes);
        atoms_to_tiles(atoms, H / 128, katoms, -1, groups);
        if (e == cudaSuccess)
            e = cudaMemcpy(h->w_dn_sf + expert * static_cast<int64_t>(groups.size()), groups.data(), groups.size(),
                           cudaMemcpyHostToDevice);
    } else {
        // gate rows j -> interleaved row (j / 128) * 256 + j % 128, up rows +128
        const int half = proj == NF_PROJ_UP ? 1 : 0;
        e = upload_blocked_half(h->w_gu + expert * blocked_bytes(2 * I, kbytes), packed, I, kbytes, half);
        atoms_to_tiles(atoms, I / 128, katoms, half, groups);
        if (e == cudaSuccess)
            e = cudaMemcpy2D(h->w_gu_sf + expert * static_cast<int64_t>(groups.size()) + half * 2048, 4096,
                             groups.data() + half * 2048, 4096, 2048, groups.size() / 4096, cudaMemcpyHostToDevice);
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->cuda_fail(e, "bind copy");
    const float alpha = ws2 * in_scale;  // gemv_nvfp4_rows: alpha = scale2 * input_scale
    if (proj == NF_PROJ_GATE) h->h_alpha_g[expert] = alpha, h->h_in_g[expert] = in_scale;
    else if (proj == NF_PROJ_UP) h->h_alpha_u[expert] = alpha, h->h_in_u[expert] = in_scale;
    else h->h_alpha_d[expert] = alpha, h->h_in_d[expert] = in_scale;
    h->bound[static_cast<size_t>(expert * 3 + proj)] = 1;
    return NF_OK;
}

int nf_moe_bind_bf16(nf_moe* h, int which, int expert, const uint16_t* data, int64_t rows, int64_t cols) {
    if (!h) return NF_ERR_INVALID;
    if (h->finalized) return h->fail(NF_ERR_STATE, "weights are already finalized");
    const nf_moe_desc& d = h->d;
    const int64_t H = d.hidden, E = d.experts, I = d.inter, Is = d.shared_inter;
    int64_t wr = 0, wc = 0;
    const char* name = "";
    switch (which) {
        case NF_BF16_ROUTER: wr = E, wc = H, name = "mlp.gate.weight"; break;
        case NF_BF16_SHARED_GATE: wr = Is, wc = H, name = "mlp.shared_experts.gate_proj.weight"; break;
        case NF_BF16_SHARED_UP: wr = Is, wc = H, name = "mlp.shared_experts.up_proj.weight"; break;
        case NF_BF16_SHARED_DOWN: wr = H, wc = Is, name = "mlp.shared_experts.down_proj.weight"; break;
        case NF_BF16_EXPERT_GATE: wr = I, wc = H, name = "mlp.experts.<e>.gate_proj.weight"; break;
        case NF_BF16_EXPERT_UP: wr = I, wc = H, name = "mlp.experts.<e>.up_proj.weight"; break;
        case NF_BF16_EXPERT_DOWN: wr = H, wc = I, name = "mlp.experts.<e>.down_proj.weight"; break;
        default: return h->fail(NF_ERR_INVALID, "bad BF16 tensor id %d", which);
    }
    const bool is_expert = which >= NF_BF16_EXPERT_GATE;
    if (is_expert && d.expert_kind != NF_EXPERTS_BF16) return h->fail(NF_ERR_STATE, "handle holds NVFP4 experts");
    if (is_expert && (expert < 0 || expert >= E)) return h->fail(NF_ERR_INVALID, "bad expert id");
    if (is_expert && h->ep_outer) {
        const int slot = ep_inner_slot(h, expert);
        if (slot < 0) return NF_OK;
        return ep_relay(h, nf_moe_bind_bf16(h->inner, which, slot, data, rows, cols));
    }
    if (!is_expert && h->experts_only)
        return h->fail(NF_ERR_STATE, "%s handle holds no %s", h->dense ? "a dense MLP" : "an experts-only", name);
    if ((which >= NF_BF16_SHARED_GATE && which <= NF_BF16_SHARED_DOWN) && Is == 0)
        return h->fail(NF_ERR_STATE, "descriptor has no shared expert");
    if (!data || rows != wr || cols != wc) return h->fail(NF_ERR_SHAPE, "BF16 linear layout %s", name);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaSuccess;
    const size_t rb = static_cast<size_t>(cols) * 2;
    switch (which) {
        case NF_BF16_ROUTER: {
            e = cudaMemcpy(h->router_w, data, rows * rb, cudaMemcpyHostToDevice);
            if (e == cudaSuccess && h->router_wz) {
                std::vector<float> wz(static_cast<size_t>(router_chunked_elems(E, d.hidden)));
                router_chunked_layout(data, E, d.hidden, wz.data());
                e = cudaMemcpy(h->router_wz, wz.data(), wz.size() * sizeof(float), cudaMemcpyHostToDevice);
                if (e == cudaSuccess) {
                    std::vector<uint16_t> wz16(static_cast<size_t>(router_chunked_elems16(E, d.hidden)));
                    router_chunked_layout16(data, E, d.hidden, wz16.data());
                    e = cudaMemcpy(h->router_wz16, wz16.data(), wz16.size() * 2, cudaMemcpyHostToDevice);
                }
            }
            if (e == cudaSuccess && h->screen) {
                // each row's 2-norm, rounded up (a bound on sum |w x| with ||x||_2)
                std::vector<float> nrm(static_cast<size_t>(rows));
                for (int64_t r = 0; r < rows; ++r) {
                    double ss = 0.0;
                    for (int64_t c = 0; c < cols; ++c) {
                        uint32_t b = static_cast<uint32_t>(data[r * cols + c]) << 16;
                        float f;
                        std::memcpy(&f, &b, 4);
                        ss += static_cast<double>(f) * f;
                    }
                    const double n = std::sqrt(ss) * (1.0 + 1e-12);
                    float f = static_cast<float>(n);
                    if (static_cast<double>(f) < n) f = std::nextafter(f, INFINITY);
                    nrm[static_cast<size_t>(r)] = std::isfinite(f) ? f : INFINITY;
                }
                if (e == cudaSuccess) e = cudaMemcpy(h->router_wnorm, nrm.data(), nrm.size() * 4, cudaMemcpyHostToDevice);
            }
            h->router_bound = e == cudaSuccess;
            // products with BF16 activations stay exact in fp32 when every
            // nonzero weight has a biased exponent in [60, 189]
            int safe = 1;
            for (int64_t i = 0; i < rows * cols && safe; ++i) {
                const uint32_t v = data[i], ex = (v >> 7) & 0xffu;
                if ((v & 0x7fffu) != 0u && (ex < 60u || ex > 189u)) safe = 0;
            }
            h->router_w_safe = safe;
            break;
        }
        case NF_BF16_SHARED_GATE:
        case NF_BF16_SHARED_UP: {
            e = upload_blocked_half(reinterpret_cast<uint8_t*>(h->ws_gu), reinterpret_cast<const uint8_t*>(data), Is,
                                    static_cast<int64_t>(rb), which == NF_BF16_SHARED_UP ? 1 : 0);
            if (which == NF_BF16_SHARED_GATE) h->sg_bound = e == cudaSuccess;
            else h->su_bound = e == cudaSuccess;
            break;
        }
        case NF_BF16_SHARED_DOWN:
            e = upload_blocked(reinterpret_cast<uint8_t*>(h->ws_dn), reinterpret_cast<const uint8_t*>(data), H,
                               static_cast<int64_t>(rb));
            h->sd_bound = e == cudaSuccess;
            break;
        case NF_BF16_EXPERT_GATE:
        case NF_BF16_EXPERT_UP: {
            uint8_t* base = reinterpret_cast<uint8_t*>(h->wb_gu) + expert * blocked_bytes(2 * I, H * 2);
            e = upload_blocked_half(base, reinterpret_cast<const uint8_t*>(data), I, static_cast<int64_t>(rb),
                                    which == NF_BF16_EXPERT_UP ? 1 : 0);
            if (e == cudaSuccess) h->bound[static_cast<size_t>(expert * 3 + (which - NF_BF16_EXPERT_GATE))] = 1;
            break;
        }
        case NF_BF16_EXPERT_DOWN:
            e = upload_blocked(reinterpret_cast<uint8_t*>(h->wb_dn) + expert * blocked_bytes(H, I * 2),
                               reinterpret_cast<const uint8_t*>(data), H, static_cast<int64_t>(rb));
            if (e == cudaSuccess) h->bound[static_cast<size_t>(expert * 3 + 2)] = 1;
            break;
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->cuda_fail(e, "bind copy");
    return NF_OK;
}

int nf_moe_bind_f32(nf_moe* h, int which, const float* data, int64_t n) {
    if (!h) return NF_ERR_INVALID;
    if (h->finalized) return h->fail(NF_ERR_STATE, "weights are already finalized");
    if (which != NF_F32_ROUTER_BIAS) return h->fail(NF_ERR_INVALID, "bad F32 tensor id %d", which);
    if (h->experts_only)
        return h->fail(NF_ERR_STATE, "%s handle holds no mlp.gate.e_score_correction_bias",
                       h->dense ? "a dense MLP" : "an experts-only");
    if (!data || n != h->d.experts) return h->fail(NF_ERR_SHAPE, "vector length mismatch for mlp.gate.e_score_correction_bias");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    const cudaError_t e = cudaMemcpy(h->router_bias, data, static_cast<size_t>(n) * sizeof(float), cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->cuda_fail(e, "bind copy");
    h->bias_bound = true;
    return NF_OK;
}

int nf_moe_finalize(nf_moe* h) {
    if (!h) return NF_ERR_INVALID;
    if (h->finalized) return NF_OK;
    const nf_moe_desc& d = h->d;
    const int64_t H = d.hidden, E = d.experts, I = d.inter, Is = d.shared_inter;
    if (!h->experts_only && !h->router_bound) return h->fail(NF_ERR_STATE, "missing tensor mlp.gate.weight");
    if (!h->experts_only && !h->bias_bound)
        return h->fail(NF_ERR_STATE, "missing tensor mlp.gate.e_score_correction_bias");
    if (Is > 0 && !(h->sg_bound && h->su_bound && h->sd_bound)) return h->fail(NF_ERR_STATE, "missing tensor mlp.shared_experts");
    if (h->ep_outer) {
        // the routed experts live in the inner handle (expert ids local to this rank)
        const int st = nf_moe_finalize(h->inner);
        if (st != NF_OK) {
            const char* m = h->inner->err.c_str();
            long long le = -1;
            char proj[32] = {0};
            if (std::sscanf(m, "missing tensor mlp.experts.%lld.%31s", &le, proj) == 2)
                return h->fail(st, "missing tensor mlp.experts.%lld.%s", ep_global_expert(h, le), proj);
            return h->fail(st, "%s", m);
        }
    } else {
        for (int64_t e = 0; e < E; ++e)
            for (int p = 0; p < 3; ++p)
                if (!h->bound[static_cast<size_t>(e * 3 + p)])
                    return h->fail(NF_ERR_STATE, "missing tensor %s", proj_label(h, e, p).c_str());
    }
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    std::vector<float> gs_g(E, 1.f), gs_d(E, 1.f);
    if (fp4 && !h->ep_outer) {
        for (int64_t e = 0; e < E; ++e) {
            if (h->h_in_g[e] != h->h_in_u[e])
                return h->fail(NF_ERR_UNSUPPORTED,
                               "%s gate_proj and up_proj input_scale differ; this build needs one gate/up input scale",
                               h->dense ? "mlp" : ("mlp.experts." + std::to_string(e)).c_str());
            gs_g[e] = 1.f / h->h_in_g[e];  // quant_dequant_nvfp4_activation: global_scale = 1 / input_scale
            gs_d[e] = 1.f / h->h_in_d[e];
        }
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaMemcpy(h->alpha_g, h->h_alpha_g.data(), E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->alpha_u, h->h_alpha_u.data(), E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->alpha_d, h->h_alpha_d.data(), E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->gs_g, gs_g.data(), E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->gs_d, gs_d.data(), E * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        // the down input quantiser's output scale for each E4M3 scale code:
        // 1 / (scale / global_scale), with quant_dequant_nvfp4_activation's
        // guard for a zero scale (src/text_forward.cpp:531-549)
        // (and the same for the gate/up input, the dispatch's quantiser)
        std::vector<float> os(static_cast<size_t>(E) * 256), osg(static_cast<size_t>(E) * 256);
        for (int64_t x = 0; x < E; ++x)
            for (int c = 0; c < 256; ++c) {
                const float reduced = e4m3_host(static_cast<uint8_t>(c)) / gs_d[static_cast<size_t>(x)];
                os[static_cast<size_t>(x * 256 + c)] = 1.f / (reduced + (reduced == 0.f ? 1.0e8f : 0.f));
                const float reduced_g = e4m3_host(static_cast<uint8_t>(c)) / gs_g[static_cast<size_t>(x)];
                osg[static_cast<size_t>(x * 256 + c)] = 1.f / (reduced_g + (reduced_g == 0.f ? 1.0e8f : 0.f));
            }
        e = cudaMemcpy(h->os_tab, os.data(), os.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(h->os_tab_g, osg.data(), osg.size() * 4, cudaMemcpyHostToDevice);
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->cuda_fail(e, "finalize copy");
    const int64_t R = h->rows_cap, Tm = d.max_tokens;
    bool ok = true;
    if (h->ep_outer) {
        // no routed workspace: only the shared expert's maps
    } else if (fp4) {
        ok = ok && make_tmap_blocked(&h->tm_b_gu, h->w_gu, h->bytes_of(h->w_gu)) &&
             make_tmap_blocked(&h->tm_b_dn, h->w_dn, h->bytes_of(h->w_dn));
        ok = ok && make_tmap_2d(&h->tm_a, h->pb.a_codes, false, H / 2, R, 128, 128);
        ok = ok && make_tmap_2d(&h->tm_a_s, h->pb.a_codes, false, H / 2, R, 128, 32);
        ok = ok && make_tmap_2d(&h->tm_h_s, h->h_codes, false, I / 2, R, 128, 32);
        ok = ok && make_tmap_2d(&h->tm_h, h->h_codes, false, I / 2, R, 128, 128);
        // 512-K-stage maps (without them the handle keeps 256-K stages)
        h->wide_ok = H % 512 == 0 && I % 256 == 0 && make_tmap_a3(&h->tm_a3, h->pb.a_codes, H / 2, R) &&
                     make_tmap_a3(&h->tm_h3, h->h_codes, I / 2, R) &&
                     make_tmap_b3(&h->tm_b_gu3, h->w_gu, h->bytes_of(h->w_gu)) &&
                     make_tmap_b3(&h->tm_b_dn3, h->w_dn, h->bytes_of(h->w_dn));
        // the CTA-pair GEMMs' maps (without them the handle keeps the one-SM kernels)
        bool pair_ok = make_tmap_blocked(&h->tm_b_gu_half, h->w_gu, h->bytes_of(h->w_gu), 128) &&
                       make_tmap_blocked(&h->tm_b_dn_half, h->w_dn, h->bytes_of(h->w_dn), 128);
        pair_ok = pair_ok && make_tmap_runs(&h->tm_sfa_a, h->pb.a_sf, h->bytes_of(h->pb.a_sf), 8) &&
                  make_tmap_runs(&h->tm_sfa_h, h->h_sf, h->bytes_of(h->h_sf), 8);
        pair_ok = pair_ok && make_tmap_runs(&h->tm_sfb_gu, h->w_gu_sf, h->bytes_of(h->w_gu_sf), 16) &&
                  make_tmap_runs(&h->tm_sfb_dn, h->w_dn_sf, h->bytes_of(h->w_dn_sf), 16);
        h->grid2 = 0;
        if (ok && pair_ok) {
            int prev_dev = 0;
            cudaGetDevice(&prev_dev);
            cudaSetDevice(h->device);
            h->grid2 = gemm2_grid(h->device);
            cudaSetDevice(prev_dev);
        }
    } else {
        ok = ok && make_tmap_blocked(&h->tm_b_gu, h->wb_gu, h->bytes_of(h->wb_gu)) &&
             make_tmap_blocked(&h->tm_b_dn, h->wb_dn, h->bytes_of(h->wb_dn));
        ok = ok && make_tmap_2d(&h->tm_a, h->pb.a_bf16, true, H, R, 64, 128);
        ok = ok && make_tmap_2d(&h->tm_a_s, h->pb.a_bf16, true, H, R, 64, 32);
        ok = ok && make_tmap_2d(&h->tm_h_s, h->h_bf16, true, I, R, 64, 32);
        ok = ok && make_tmap_2d(&h->tm_h, h->h_bf16, true, I, R, 64, 128);
    }
    if (Is > 0) {
        ok = ok && make_tmap_blocked(&h->tm_bs_gu, h->ws_gu, h->bytes_of(h->ws_gu)) &&
             make_tmap_blocked(&h->tm_bs_dn, h->ws_dn, h->bytes_of(h->ws_dn));
        ok = ok && make_tmap_2d(&h->tm_shh, h->sh_h, true, Is, Tm, 64, 128);
        ok = ok && make_tmap_2d(&h->tm_shh_s, h->sh_h, true, Is, Tm, 64, 32);
    }
    if (!ok) return h->fail(NF_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    h->finalized = true;
    return NF_OK;
}

// A device x may be NULL with tokens == 0: nothing reads it then (an
// expert-parallel rank without tokens still calls the forward for the
// exchanges).  Host-buffer calls always need their arrays.
static int check_forward_args(nf_moe* h, const void* x, int tokens, bool device_x = true) {
    if (!h) return NF_ERR_INVALID;
    if (!h->finalized) return h->fail(NF_ERR_STATE, "nf_moe_finalize has not run");
    if (tokens < 0) return h->fail(NF_ERR_INVALID, "negative token count");
    if (!x && (tokens > 0 || !device_x)) return h->fail(NF_ERR_INVALID, "null input");
    // the router copies and the combine read and write 16-byte pieces of device rows
    if (device_x && reinterpret_cast<uintptr_t>(x) % 16 != 0) return h->fail(NF_ERR_LAYOUT, "x must be 16-byte aligned");
    if (tokens > h->d.max_tokens) return h->fail(NF_ERR_CAPACITY, "tokens %d exceed max_tokens %d", tokens, h->d.max_tokens);
    return NF_OK;
}

int nf_moe_route(nf_moe* h, const uint16_t* x, int tokens, float* logits, int32_t* idx, float* w, void* stream) {
    int st = check_forward_args(h, x, tokens);
    if (st != NF_OK) return st;
    if (h->experts_only) return h->fail(NF_ERR_STATE, "handle has no router");
    if (tokens == 0) return NF_OK;
    const nf_moe_desc& d = h->d;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    const cudaError_t e = launch_router(x, h->router_w, h->router_wz, h->router_wz16, h->router_bias, tokens, d.hidden, d.experts, d.top_k,
                                        d.routed_scaling, d.normalize, d.n_group, d.topk_group, h->router_w_safe,
                                        logits ? logits : h->logits, h->scores, h->choices,
                                        idx ? idx : h->topk_idx, w ? w : h->topk_w, h->dev_err, s);
    cudaSetDevice(prev);
    return e == cudaSuccess ? NF_OK : h->cuda_fail(e, "router launch");
}

}  // extern "C"

// The shared expert (mlp_bf16, src/text_forward.cpp:917-922) on the side
// stream: it does not depend on routing, so it is forked from `s` (before
// or after the router, see forward_impl) and overlaps the rest of the layer
// (the GEMMs' dynamic tile scheduler absorbs the SMs it holds).  Joined by
// ev_join.
int launch_shared_expert(nf_moe* h, const uint16_t* x, int T, StageRec& rec, cudaStream_t s) {
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, Is = d.shared_inter;
    cudaError_t e = cudaSuccess;
    if ((e = cudaEventRecord(h->ev_fork, s)) != cudaSuccess || (e = cudaStreamWaitEvent(h->side, h->ev_fork, 0)) != cudaSuccess)
        return h->cuda_fail(e, "shared expert fork");
    CUtensorMap tm_x, tm_x_s;
    if (!make_tmap_2d(&tm_x, x, true, H, T, 64, 128) || !make_tmap_2d(&tm_x_s, x, true, H, T, 64, 32))
        return h->fail(NF_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    rec.begin(NF_STAGE_SHARED, h->side);
    if ((e = cudaMemsetAsync(h->shared_counters, 0, 2 * sizeof(int), h->side)) != cudaSuccess)
        return h->cuda_fail(e, "shared expert counters");
    GemmArgs sg{};
    sg.err = h->dev_err;
    sg.limit = d.swiglu_limit;
    sg.kind = KIND_BF16;
    sg.epi = EPI_SWIGLU_BF16;
    sg.K = H;
    sg.dense_rows = T;
    sg.n_blocks = Is / 128;
    sg.b_nb = 2 * Is / 256;
    sg.b = reinterpret_cast<const uint8_t*>(h->ws_gu);
    sg.b_kt = static_cast<int>(k_blocks(2 * H));
    sg.out = h->sh_h;
    sg.out_ld = Is;
    sg.tile_counter = h->shared_counters;
    sg.early_claim = 1;  // dense tiles; the counters were zeroed before the first GEMM
    // Large batches: 256-row tiles (two accumulators per B stage, 1.5x fewer
    // shared-memory bytes per MMA); they still give every SM a few tiles.
    sg.m_pair = T >= kSharedPairTokens ? 1 : 0;
    // Few tiles at decode sizes: a grid of one CTA per tile leaves the other
    // SMs to the routed path (the down GEMM's CTAs launch early and hold
    // their SMs while gate/up finishes: few CTAs hold few SMs).
    const int m_tiles = sg.m_pair ? (T + 255) / 256 : (T + 127) / 128;
    e = launch_gemm(tm_x, tm_x_s, h->tm_bs_gu, sg, std::min(h->grid, m_tiles * (Is / 128)), false, h->side);
    if (e != cudaSuccess) return h->cuda_fail(e, "shared gate/up GEMM launch");
    sg.epi = EPI_STORE_F32;
    sg.K = Is;
    sg.n_blocks = H / 256;
    sg.b_nb = H / 256;
    sg.b = reinterpret_cast<const uint8_t*>(h->ws_dn);
    sg.b_kt = static_cast<int>(k_blocks(2 * Is));
    sg.out = h->sh_out;
    sg.out_ld = H;
    sg.tile_counter = h->shared_counters + 1;
    e = launch_gemm(h->tm_shh, h->tm_shh_s, h->tm_bs_dn, sg, std::min(h->grid, m_tiles * (H / 256)), true, h->side);
    if (e != cudaSuccess) return h->cuda_fail(e, "shared down GEMM launch");
    rec.end(NF_STAGE_SHARED, h->side);
    if ((e = cudaEventRecord(h->ev_join, h->side)) != cudaSuccess) return h->cuda_fail(e, "shared expert join");
    return NF_OK;
}

// The routed experts for T rows of x with K expert picks each (idx, global
// to this handle's experts): permutation + NVFP4 dispatch, grouped gate/up
// GEMM (SwiGLU and the down input's quantisation fused), grouped down GEMM.
// The down rows land in h->down in permuted order (h->pb.pair_row maps a
// pick to its row).
bool dense_splitk_fused(const nf_moe* h, int T, int down_split) {
    // (NVFP4 dense handles: their dispatch zeroes the slice counters)
    return down_split > 1 && h->dense && h->d.expert_kind == NF_EXPERTS_NVFP4 &&
           static_cast<int64_t>((T + 127) / 128) * (h->d.hidden / 256) * down_split <= static_cast<int64_t>(h->grid);
}

int launch_routed_experts(nf_moe* h, const uint16_t* x, const int32_t* idx, int T, int K, StageRec& rec,
                          cudaStream_t s, int down_split, const float* residual, float* y, const GemmArgs* epr) {
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, E = d.experts, I = d.inter;
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    cudaError_t e = cudaSuccess;
    rec.begin(NF_STAGE_PERMUTE, s);
    bool one_kernel = false;
    // The dense MLP (every token on expert 0) skips the permutation: its rows
    // are the tokens in order, and both GEMMs run dense tiles over them.
    const bool dense_rows = h->dense && fp4;
    // 33-64 tokens fill two of the four TMEM lane quadrants of the gate/up
    // tile: repeat them in the other two so all the epilogue warps work
    const bool rep64 = dense_rows && T > 32 && T <= 64;
    if (dense_rows) {
        e = launch_dense_dispatch(x, T, H, h->gs_g, h->os_tab_g, h->pb, h->splitk_cnt, h->splitk_cnt_elems, rep64, s);
        one_kernel = true;
    } else {
        e = launch_permute(idx, x, T, K, E, H, I / 128, H / 256, h->gs_g, fp4 ? h->os_tab_g : nullptr, fp4 ? 0 : 1, h->pb,
                           s, &one_kernel);
    }
    if (e != cudaSuccess) return h->cuda_fail(e, "permute launch");
    rec.end(NF_STAGE_PERMUTE, s);
    rec.begin(NF_STAGE_GATE_UP, s);
    GemmArgs g{};
    g.err = h->dev_err;
    g.limit = d.swiglu_limit;
    g.swiglu_bf16 = h->dense ? 1 : 0;  // dense_mlp uses swiglu_clamp_bf16 (src/text_forward.cpp:913)
    // gate/up
    g.kind = fp4 ? KIND_NVFP4 : KIND_BF16;
    g.epi = fp4 ? EPI_SWIGLU_QUANT : EPI_SWIGLU_BF16;
    g.K = H;
    g.b_nb = 2 * I / 256;
    g.b = fp4 ? h->w_gu : reinterpret_cast<const uint8_t*>(h->wb_gu);
    g.b_kt = static_cast<int>(k_blocks(fp4 ? H / 2 : 2 * H));
    g.tiles = h->pb.tiles_gu;
    g.num_tiles_dev = h->pb.meta + 1;
    g.dense_rows = 0;
    g.n_blocks = I / 128;
    g.sfa = h->pb.a_sf;
    g.sfb = h->w_gu_sf;
    g.alpha0 = h->alpha_g;
    g.alpha1 = h->alpha_u;
    g.gscale_next = h->gs_d;
    g.os_table = fp4 ? h->os_tab : nullptr;
    g.row_token = h->pb.row_token;
    g.out = fp4 ? static_cast<void*>(h->h_codes) : static_cast<void*>(h->h_bf16);
    g.out_ld = fp4 ? I / 2 : I;
    g.out_sf = h->h_sf;
    g.out_kgroups = I / 16;
    g.tile_counter = h->pb.meta + 4;
    // Unprofiled forwards hand rows over block by block: the down GEMM's
    // tiles start as soon as the gate/up tiles of their 128 rows are done (so
    // its CTAs work through the gate/up GEMM's tail instead of waiting for the
    // whole kernel); profiled forwards keep the kernels apart to time them.
    const bool handoff = rec.ev == nullptr;
    g.mt_done = h->pb.mt_done;
    g.mt_signal = handoff ? 1 : 0;
    g.early_claim = one_kernel ? 0 : 1;  // the tile list is written by the kernel right before
    if (dense_rows) {
        g.dense_rows = T;
        g.tiles = nullptr;
        g.num_tiles_dev = nullptr;
        g.k_split = 1;
        g.row_token = nullptr;
        g.rep64 = rep64 ? 1 : 0;
        // a CTA per tile: claimed by block index before the dispatch completes,
        // so the first B stages stream while it runs
        if (static_cast<int64_t>((T + 127) / 128) * (I / 128) <= h->grid) {
            g.static_tiles = 1;
            g.early_claim = 1;
        }
    }
    // Prefill-sized batches (on average a pair tile's 256 rows per expert or
    // more) may take the alternative GEMM forms (nf_moe_set_expert_gemm)
    g.num_experts = E;
    g.seg_off = h->pb.seg_off;
    g.seg_cnt = h->pb.counts;
    const bool prefill = static_cast<int64_t>(T) * K >= 256LL * E && down_split <= 1;
    const bool pair = !epr && !dense_rows && fp4 && h->gemm_mode == NF_GEMM_CTA_PAIR && h->grid2 >= 2 && prefill && H % 256 == 0 &&
                      I % 256 == 0 && E <= 256;
    const bool wide = !epr && fp4 && h->gemm_mode == NF_GEMM_WIDE_STAGES && prefill && h->wide_ok;
    g.wide_stages = wide ? 1 : 0;
    e = pair ? launch_gemm2(h->tm_a, h->tm_b_gu_half, h->tm_sfa_a, h->tm_sfb_gu, g, h->grid2, true, s)
        : wide ? launch_gemm(h->tm_a3, h->tm_a3, h->tm_b_gu3, g, h->grid, true, s)
               : launch_gemm(h->tm_a, h->tm_a_s, h->tm_b_gu, g, h->grid, true, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "gate/up GEMM launch");
    rec.end(NF_STAGE_GATE_UP, s);
    rec.begin(NF_STAGE_DOWN, s);
    // down
    g.epi = fp4 ? EPI_STORE_BF16 : EPI_STORE_F32;
    g.K = I;
    g.b_nb = H / 256;
    g.b = fp4 ? h->w_dn : reinterpret_cast<const uint8_t*>(h->wb_dn);
    g.b_kt = static_cast<int>(k_blocks(fp4 ? I / 2 : 2 * I));
    g.tiles = h->pb.tiles_down;
    g.num_tiles_dev = h->pb.meta + 2;
    g.n_blocks = H / 256;
    g.sfa = h->h_sf;
    g.sfb = h->w_dn_sf;
    g.alpha0 = h->alpha_d;
    g.out = h->down;
    g.out_ld = H;
    g.tile_counter = h->pb.meta + 5;
    g.swiglu_bf16 = 0;
    g.mt_signal = 0;
    g.mt_wait = handoff ? I / 128 : 0;
    g.early_claim = 1;
    g.rep64 = 0;
    g.static_tiles = 0;
    if (epr && fp4) {
        // the outputs go to their source ranks' mailboxes from the epilogue
        g.ep_ret = 1;
        g.ep_world = epr->ep_world;
        g.ep_me = epr->ep_me;
        g.ep_cap = epr->ep_cap;
        g.ep_ret_off = epr->ep_ret_off;
        g.ep_flags_ret = epr->ep_flags_ret;
        for (int i = 0; i < kEpMaxRanks; ++i) g.ep_mbox[i] = epr->ep_mbox[i];
        g.ep_src_off = epr->ep_src_off;
        g.ep_epoch = epr->ep_epoch;
        g.ep_tiles_done = epr->ep_tiles_done;
    }
    if (dense_rows) {
        g.dense_rows = T;
        g.tiles = nullptr;
        g.num_tiles_dev = nullptr;
    }
    if (down_split > 1) {
        // dense split-K: tiles (n block, K slice, m tile) over the T rows of h
        // (one segment at row 0), raw fp32 slices into dense_part
        int kt_per = 0;
        const int S = dense_down_split(T, H, I, h->grid, &kt_per);
        const int64_t stride = static_cast<int64_t>((T + 127) / 128) * 128 * H;
        if (S != down_split || S * stride > h->dense_part_elems) return h->fail(NF_ERR_STATE, "split-K workspace");
        g.epi = EPI_STORE_F32;
        g.dense_rows = T;
        g.tiles = nullptr;
        g.num_tiles_dev = nullptr;
        g.k_split = S;
        g.kt_per = kt_per;
        g.out = h->dense_part;
        g.out_ld = H;
        g.out_split_stride = stride;
        if (dense_splitk_fused(h, T, S)) {
            g.splitk_fuse = 1;
            g.static_tiles = 1;
            g.splitk_cnt = h->splitk_cnt;
            g.residual = residual;
            g.y = y;
        }
    }
    e = pair ? launch_gemm2(h->tm_h, h->tm_b_dn_half, h->tm_sfa_h, h->tm_sfb_dn, g, h->grid2, true, s)
        : wide ? launch_gemm(h->tm_h3, h->tm_h3, h->tm_b_dn3, g, h->grid, true, s)
               : launch_gemm(h->tm_h, h->tm_h_s, h->tm_b_dn, g, h->grid, true, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "down GEMM launch");
    rec.end(NF_STAGE_DOWN, s);
    return NF_OK;
}

// TextModel::dense_mlp (src/text_forward.cpp:909-915) + the hc = 1 residual:
// the routed chain with every token on expert 0, then y = 1 * down (+ residual).
static int dense_forward(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, cudaStream_t s) {
    h->last_tokens = T;
    StageRec rec;
    rec.h = h;
    rec.ev = h->prof_begin(&rec.set);
    const int H = h->d.hidden;
    int kt_per = 0;
    const int S = dense_down_split(T, H, h->d.inter, h->grid, &kt_per);
    const bool fused = dense_splitk_fused(h, T, S);
    int st = launch_routed_experts(h, x, h->dense_idx, T, 1, rec, s, S, residual, y);
    if (st != NF_OK) return st;
    if (fused) return NF_OK;  // the down GEMM reduced its K slices into y
    rec.begin(NF_STAGE_COMBINE, s);
    const cudaError_t e =
        S > 1 ? launch_splitk_store(h->dense_part, S, static_cast<int64_t>((T + 127) / 128) * 128 * H, T, H, h->alpha_d,
                                    residual, y, 4 * h->grid, s)
              : launch_combine(h->down, true, h->pb.pair_row, h->dense_w, nullptr, residual, T, 1, H, y, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "combine launch");
    rec.end(NF_STAGE_COMBINE, s);
    return NF_OK;
}

cudaError_t route_tokens(nf_moe* h, const uint16_t* x, int T, int32_t* idx, float* w, cudaStream_t s) {
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, E = d.experts, K = d.top_k;
    const bool grouped = d.n_group > 1 && d.topk_group < d.n_group;
    h->last_screened = 0;
    // The screen's bound needs exact products, which the bind-time range
    // check of the router weights guarantees (router_w_safe).  Weights outside
    // that range can overflow the reference's sequential chain where the
    // tensor cores' order does not; such a layer runs every exact chain.
    if (!h->screen || !h->router_w_safe || T < kScreenMinTokens || grouped || T > d.max_tokens || K > 8)
        return launch_router(x, h->router_w, h->router_wz, h->router_wz16, h->router_bias, T, H, E, K,
                             d.routed_scaling, d.normalize, d.n_group, d.topk_group, h->router_w_safe, h->logits,
                             h->scores, h->choices, idx, w, h->dev_err, s);
    h->last_screened = 1;
    // 1-2. approximate logits on the tensor cores, the bound
    //      |l~ - l| <= (gamma_H + H 2^-22 + 2^-24) ||x||_2 ||w_e||_2 (the tensor
    //      core's accumulation taken as 4 units of fp32 roundoff per product),
    //      and the candidates
    const double u = std::ldexp(1.0, -24);
    const double c = (H * u / (1.0 - H * u) + H * std::ldexp(1.0, -22) + u) * 1.01;
    CUtensorMap tmx;
    if (!make_tmap_2d(&tmx, x, true, H, T, 64, 32)) return cudaErrorInvalidValue;
    cudaError_t e = launch_route_screen(tmx, x, T, H, h->router_wz16, E, K, h->router_bias, h->router_wnorm,
                                        static_cast<float>(c), h->screen_cand, h->screen_cnt, h->logits, h->dev_err, s);
    if (e != cudaSuccess) return e;
    // 3. the exact chains of the candidates and the reference's selection
    return launch_route_exact(tmx, x, h->router_wz16, h->router_bias, T, H, E, K, d.routed_scaling, d.normalize,
                              h->router_w_safe, h->screen_cand, h->screen_cnt, idx, w, h->dev_err, s);
}

static int forward_impl(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, int32_t* idx_user,
                        float* w_user, cudaStream_t s) {
    if (h->ep_outer) return ep_forward(h, x, residual, T, y, idx_user, w_user, s);
    if (h->dense) return dense_forward(h, x, residual, T, y, s);
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, K = d.top_k, Is = d.shared_inter;
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    int32_t* idx = idx_user ? idx_user : h->topk_idx;
    float* w = w_user ? w_user : h->topk_w;
    h->last_tokens = T;
    StageRec rec;
    rec.h = h;
    rec.ev = h->prof_begin(&rec.set);
    int st = NF_OK;
    // The shared expert forks before the router at decode sizes (the router
    // is a few CTAs of latency-bound work that the shared GEMMs run beside);
    // at prefill sizes the screened router fills the GPU and the shared
    // GEMMs' persistent CTAs would hold its SMs, so they fork after it and run
    // beside the permutation and the routed GEMMs instead.
    // (Profiled forwards join the shared expert at once, so that every stage
    // time is its kernels alone.)
    const bool shared_first = !(h->screen && T >= kScreenMinTokens);
    cudaError_t e = cudaSuccess;
    auto shared = [&]() -> int {
        int r = launch_shared_expert(h, x, T, rec, s);
        if (r == NF_OK && rec.ev && (e = cudaStreamWaitEvent(s, h->ev_join, 0)) != cudaSuccess)
            r = h->cuda_fail(e, "shared expert join");
        return r;
    };
    if (Is > 0 && shared_first && (st = shared()) != NF_OK) return st;
    rec.begin(NF_STAGE_ROUTER, s);
    e = route_tokens(h, x, T, idx, w, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "router launch");
    rec.end(NF_STAGE_ROUTER, s);
    if (Is > 0 && !shared_first && (st = shared()) != NF_OK) return st;
    if ((st = launch_routed_experts(h, x, idx, T, K, rec, s)) != NF_OK) return st;
    if (Is > 0 && (e = cudaStreamWaitEvent(s, h->ev_join, 0)) != cudaSuccess) return h->cuda_fail(e, "shared expert join");
    rec.begin(NF_STAGE_COMBINE, s);
    e = launch_combine(h->down, fp4, h->pb.pair_row, w, Is > 0 ? h->sh_out : nullptr, residual, T, K, H, y, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "combine launch");
    rec.end(NF_STAGE_COMBINE, s);
    return NF_OK;
}

extern "C" {

int nf_moe_profile(nf_moe* h, int enable) {
    if (!h) return NF_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    if (h->prof_ev.empty()) {
        h->prof_ev.resize(static_cast<size_t>(nf_moe::kProfSets) * nf_moe::kEvPerSet);
        for (auto& ev : h->prof_ev) {
            if (cudaEventCreate(&ev) != cudaSuccess) {
                cudaSetDevice(prev);
                return h->fail(NF_ERR_CUDA, "cudaEventCreate failed");
            }
        }
        h->prof_used.assign(nf_moe::kProfSets, 0);
        h->prof_mask.assign(nf_moe::kProfSets, 0);
    }
    for (int set = 0; set < nf_moe::kProfSets; ++set) h->prof_used[static_cast<size_t>(set)] = 0;
    for (double& v : h->stage_ms) v = 0.0;
    h->prof_forwards = 0;
    h->prof_next = 0;
    h->profiling = enable != 0;
    cudaSetDevice(prev);
    return NF_OK;
}

int nf_moe_stage_times(nf_moe* h, float* ms_out, int* forwards) {
    if (!h || !ms_out) return NF_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    for (int set = 0; set < static_cast<int>(h->prof_used.size()); ++set)
        if (h->prof_used[static_cast<size_t>(set)]) h->fold(set);
    cudaSetDevice(prev);
    for (int s = 0; s < NF_STAGE_COUNT; ++s) ms_out[s] = static_cast<float>(h->stage_ms[s]);
    if (forwards) *forwards = h->prof_forwards;
    return NF_OK;
}

// Graph mode: the forward's launches for one (buffers, tokens, stream)
// combination are captured once into a CUDA graph and replayed, which
// removes the per-kernel launch gaps that dominate small batches.
static int forward_graph(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, int32_t* idx, float* w,
                         cudaStream_t s) {
    for (auto& g : h->graphs)
        if (!g.host && g.x == x && g.res == residual && g.y == y && g.idx == idx && g.w == w && g.T == T && g.s == s) {
            const cudaError_t e = cudaGraphLaunch(g.exec, s);
            return e == cudaSuccess ? NF_OK : h->cuda_fail(e, "graph launch");
        }
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return h->cuda_fail(e, "stream capture");
    const int st = forward_impl(h, x, residual, T, y, idx, w, s);
    cudaGraph_t graph = nullptr;
    e = cudaStreamEndCapture(s, &graph);
    if (st != NF_OK) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (e != cudaSuccess) return h->cuda_fail(e, "stream capture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return h->cuda_fail(e, "graph instantiate");
    if (h->graphs.size() >= nf_moe::kMaxGraphs) {
        cudaGraphExecDestroy(h->graphs.front().exec);
        h->graphs.erase(h->graphs.begin());
    }
    h->graphs.push_back({x, residual, y, idx, w, T, s, exec, false});
    e = cudaGraphLaunch(exec, s);
    return e == cudaSuccess ? NF_OK : h->cuda_fail(e, "graph launch");
}

int nf_moe_forward(nf_moe* h, const uint16_t* x, const float* residual, int tokens, float* y, int32_t* idx, float* w,
                   void* stream) {
    int st = check_forward_args(h, x, tokens);
    if (st != NF_OK) return st;
    if (!y && tokens > 0) return h->fail(NF_ERR_INVALID, "null output");
    if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(residual)) % 16 != 0)
        return h->fail(NF_ERR_LAYOUT, "y and residual must be 16-byte aligned");
    if (h->dense && (idx || w)) return h->fail(NF_ERR_INVALID, "a dense MLP has no routes: pass NULL top-k pointers");
    if (tokens == 0 && !h->ep_outer) return NF_OK;  // an EP rank still takes part in the exchanges
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    // graphs need a capturable stream, no per-stage events, and a caller
    // that is not capturing already
    const bool graph = h->use_graphs && (!h->ep_outer || h->ep_p2p) && s != nullptr && !h->profiling &&
                       cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
    st = graph ? forward_graph(h, x, residual, tokens, y, idx, w, s) : forward_impl(h, x, residual, tokens, y, idx, w, s);
    cudaSetDevice(prev);
    return st;
}

int nf_moe_set_graph_mode(nf_moe* h, int enable) {
    if (!h) return NF_ERR_INVALID;
    h->use_graphs = enable != 0;
    return NF_OK;
}

int nf_moe_set_expert_gemm(nf_moe* h, int mode) {
    if (!h) return NF_ERR_INVALID;
    if (mode < NF_GEMM_ONE_SM || mode > NF_GEMM_CTA_PAIR) return h->fail(NF_ERR_INVALID, "unknown expert GEMM mode");
    if (h->gemm_mode != mode) {
        // captured forwards hold the other kernels: drop them
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(h->device);
        for (auto& g : h->graphs) cudaGraphExecDestroy(g.exec);
        h->graphs.clear();
        cudaSetDevice(prev);
    }
    h->gemm_mode = mode;
    return NF_OK;
}

int nf_moe_sync(nf_moe* h, void* stream) {
    if (!h) return NF_ERR_INVALID;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    int derr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&derr, h->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && derr != 0) cudaMemset(h->dev_err, 0, sizeof(int));
    if (e == cudaSuccess && derr == 0 && h->inner) {
        // an EP rank's experts report through their own handle
        e = cudaMemcpy(&derr, h->inner->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && derr != 0) cudaMemset(h->inner->dev_err, 0, sizeof(int));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return h->cuda_fail(e, "synchronise");
    if (derr != 0) return h->fail(NF_ERR_TIMEOUT, "device-side wait gave up (code %d)", derr);
    return NF_OK;
}

// The host-buffer forward's device work on s: input copies and BF16
// conversion, the layer (inner_graph: through forward_graph), output copies.
static int host_forward_enqueue(nf_moe* h, const float* x_host, const float* res_host, int tokens, float* y_host,
                                int32_t* idx_host, float* w_host, cudaStream_t s, bool inner_graph) {
    const int64_t n = static_cast<int64_t>(tokens) * h->d.hidden;
    const int64_t nk = static_cast<int64_t>(tokens) * h->d.top_k;
    cudaError_t e = cudaMemcpyAsync(h->x_f32, x_host, n * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && res_host) e = cudaMemcpyAsync(h->res_f32, res_host, n * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = launch_f32_to_bf16(h->x_f32, n, h->x_bf16, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "host input copy");
    const float* res = res_host ? h->res_f32 : nullptr;
    int st = inner_graph ? forward_graph(h, h->x_bf16, res, tokens, h->y_f32, nullptr, nullptr, s)
                         : forward_impl(h, h->x_bf16, res, tokens, h->y_f32, nullptr, nullptr, s);
    if (st != NF_OK) return st;
    e = cudaMemcpyAsync(y_host, h->y_f32, n * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && idx_host) e = cudaMemcpyAsync(idx_host, h->topk_idx, nk * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && w_host) e = cudaMemcpyAsync(w_host, h->topk_w, nk * 4, cudaMemcpyDeviceToHost, s);
    return e == cudaSuccess ? NF_OK : h->cuda_fail(e, "host output copy");
}

static bool page_locked(const void* p) {
    if (!p) return true;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

int nf_moe_forward_host(nf_moe* h, const float* x_host, const float* res_host, int tokens, float* y_host,
                        int32_t* idx_host, float* w_host) {
    int st = check_forward_args(h, x_host, tokens, false);
    if (st != NF_OK) return st;
    if (!y_host) return h->fail(NF_ERR_INVALID, "null output");
    if (h->dense && (idx_host || w_host)) return h->fail(NF_ERR_INVALID, "a dense MLP has no routes: pass NULL top-k pointers");
    if (tokens == 0 && !h->ep_outer) return NF_OK;  // an EP rank still takes part in the exchanges
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaStream_t s = h->stream;
    const bool graphs = h->use_graphs && (!h->ep_outer || h->ep_p2p) && !h->profiling;
    // With page-locked host buffers the copies join the layer in one graph
    // (one launch per call); otherwise they are enqueued around it.
    if (graphs && page_locked(x_host) && page_locked(res_host) && page_locked(y_host) && page_locked(idx_host) &&
        page_locked(w_host)) {
        cudaGraphExec_t exec = nullptr;
        for (auto& g : h->graphs)
            if (g.host && g.x == x_host && g.res == res_host && g.y == y_host && g.idx == idx_host && g.w == w_host &&
                g.T == tokens && g.s == s)
                exec = g.exec;
        cudaError_t e = cudaSuccess;
        if (!exec) {
            e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                st = host_forward_enqueue(h, x_host, res_host, tokens, y_host, idx_host, w_host, s, false);
                cudaGraph_t graph = nullptr;
                e = cudaStreamEndCapture(s, &graph);
                if (st == NF_OK && e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
                if (graph) cudaGraphDestroy(graph);
                if (st == NF_OK && e == cudaSuccess) {
                    if (h->graphs.size() >= nf_moe::kMaxGraphs) {
                        cudaGraphExecDestroy(h->graphs.front().exec);
                        h->graphs.erase(h->graphs.begin());
                    }
                    h->graphs.push_back({x_host, res_host, y_host, idx_host, w_host, tokens, s, exec, true});
                }
            }
        }
        if (st == NF_OK && e == cudaSuccess) e = cudaGraphLaunch(exec, s);
        cudaSetDevice(prev);
        if (st != NF_OK) return st;
        if (e != cudaSuccess) return h->cuda_fail(e, "host-buffer graph");
        return nf_moe_sync(h, s);
    }
    st = host_forward_enqueue(h, x_host, res_host, tokens, y_host, idx_host, w_host, s, graphs);
    cudaSetDevice(prev);
    if (st != NF_OK) return st;
    return nf_moe_sync(h, s);
}

int nf_moe_debug_tensor(nf_moe* h, int which, void** ptr, int64_t* bytes) {
    if (!h || !ptr || !bytes) return NF_ERR_INVALID;
    void* p = nullptr;
    switch (which) {
        case NF_DBG_COUNTS: p = h->pb.counts; break;
        case NF_DBG_SEG_OFFSET: p = h->pb.seg_off; break;
        case NF_DBG_PAIR_ROW: p = h->pb.pair_row; break;
        case NF_DBG_ROW_TOKEN: p = h->pb.row_token; break;
        case NF_DBG_ACT_CODES: p = h->pb.a_codes; break;
        case NF_DBG_ACT_SF: p = h->pb.a_sf; break;
        case NF_DBG_H_CODES: p = h->h_codes; break;
        case NF_DBG_H_SF: p = h->h_sf; break;
        case NF_DBG_DOWN: p = h->down; break;
        case NF_DBG_SHARED: p = h->sh_out; break;
        case NF_DBG_ROWS: p = h->pb.meta; break;
        case NF_DBG_LOGITS: p = h->logits; break;
        case NF_DBG_SCREEN_COUNT: p = h->screen_cnt; break;
        default: return h->fail(NF_ERR_INVALID, "bad debug tensor id %d", which);
    }
    if (!p) return h->fail(NF_ERR_STATE, "debug tensor %d does not exist for this descriptor", which);
    *ptr = p;
    *bytes = static_cast<int64_t>(h->bytes_of(p));
    return NF_OK;
}

int nf_moe_debug_read(nf_moe* h, int which, void* host, int64_t bytes) {
    void* p = nullptr;
    int64_t n = 0;
    const int st = nf_moe_debug_tensor(h, which, &p, &n);
    if (st != NF_OK) return st;
    if (!host || bytes < 0 || bytes > n) return h->fail(NF_ERR_INVALID, "debug read of %lld bytes from a %lld-byte tensor",
                                                       static_cast<long long>(bytes), static_cast<long long>(n));
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(host, p, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost);
    cudaSetDevice(prev);
    return e == cudaSuccess ? NF_OK : h->cuda_fail(e, "debug read");
}

int nf_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales, float gscale, int64_t rows, int64_t cols,
                        float* out, void* stream) {
    if (rows <= 0 || cols <= 0 || cols % 16 != 0 || !packed || !scales || !out) return NF_ERR_SHAPE;
    if (!std::isfinite(gscale) || gscale < FLT_MIN) return NF_ERR_SCALE;
    std::vector<uint8_t> hs(static_cast<size_t>(rows * (cols / 16)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(hs.data(), scales, hs.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return NF_ERR_CUDA;
    for (uint8_t b : hs) {
        const float v = e4m3_host(b);
        if (!std::isfinite(v) || v < 0.f) return NF_ERR_SCALE;
        if (6.0 * static_cast<double>(v) * static_cast<double>(gscale) > static_cast<double>(FLT_MAX)) return NF_ERR_SCALE;
    }
    if (launch_dequant(packed, scales, gscale, rows, cols, out, s) != cudaSuccess) return NF_ERR_CUDA;
    return cudaStreamSynchronize(s) == cudaSuccess ? NF_OK : NF_ERR_CUDA;
}

int nf_nvfp4_quantize(const float* x, int64_t rows, int64_t cols, float in_scale, uint8_t* codes, uint8_t* scales,
                      float* fake, void* stream) {
    if (!(in_scale > 0.f) || !std::isfinite(in_scale) || cols % 16 != 0) return NF_ERR_SCALE;  // "NVFP4 input scale"
    if (rows < 0 || cols <= 0 || !x || !codes || !scales) return NF_ERR_INVALID;
    if (rows == 0) return NF_OK;
    return launch_quantize(x, rows, cols, 1.f / in_scale, codes, scales, fake, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? NF_OK
               : NF_ERR_CUDA;
}

int nf_sigmoid_ref(const float* x, int64_t n, float* y, void* stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return NF_ERR_INVALID;
    if (n == 0) return NF_OK;
    if (prepare_device_tables() != cudaSuccess) return NF_ERR_CUDA;
    return launch_sigmoid_ref(x, n, y, static_cast<cudaStream_t>(stream)) == cudaSuccess ? NF_OK : NF_ERR_CUDA;
}

int nf_format_selfcheck(int64_t* e2m1_mismatches, int64_t* e4m3_mismatches, int64_t* bf16_mismatches) {
    if (!e2m1_mismatches || !e4m3_mismatches || !bf16_mismatches) return NF_ERR_INVALID;
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, 3 * sizeof(unsigned long long)) != cudaSuccess) return NF_ERR_NOMEM;
    unsigned long long h[3] = {0, 0, 0};
    cudaError_t e = cudaMemset(d, 0, sizeof(h));
    if (e == cudaSuccess) e = launch_format_selfcheck(d, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return NF_ERR_CUDA;
    *e2m1_mismatches = static_cast<int64_t>(h[0]);
    *e4m3_mismatches = static_cast<int64_t>(h[1]);
    *bf16_mismatches = static_cast<int64_t>(h[2]);
    return NF_OK;
}

}  // extern "C"
