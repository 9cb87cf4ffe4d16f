// nf_ep.cu -- expert parallelism: the MoE layer sharded by experts over the
// GPUs of one node, one handle per rank (nf_moe_create_ep), exchanging
// token rows with NCCL point-to-point calls on the forward's stream.
//
// Rank r owns experts [r E/R, (r+1) E/R); the router, its bias and the shared
// expert are replicated; every rank routes its own tokens.  One forward:
//   1. shared expert forked onto the side stream (as on one GPU);
//   2. router over the rank's tokens (bit-exact, as on one GPU);
//   3. the picks are laid out in (destination, token, pick) order and their
//      BF16 token rows gathered into that order (ep_pack, gather_rows);
//   4. count exchange, then one host synchronisation: NCCL needs the row
//      counts on the host;
//   5. rows and destination-local expert ids exchanged (ncclSend/ncclRecv);
//   6. the rank's experts run on the received rows as top-1 picks: the same
//      permutation, NVFP4 dispatch and grouped GEMMs as on one GPU, so every
//      row's down output is the one a single GPU computes;
//   7. the down rows (BF16 for NVFP4 experts, F32 for BF16 experts) go back
//      to their source rank in receive order;
//   8. the combine adds them in pick order with the routing weights, plus
//      the shared expert and the residual -- the single-GPU combine, so the
//      layer output is bit-identical to one GPU's.
// NCCL is loaded with dlopen on the first EP handle: a process that already
// loaded NCCL (e.g. through PyTorch) shares that copy, and processes that
// never use EP never load it.
//
// Two transports carry steps 4-7.  The peer-memory one maps every rank's "mailbox"
// allocation into every other rank with CUDA IPC and moves rows and outputs
// by plain stores over NVLink, each direction closed by an epoch flag with a
// bounded wait (nf_kernels.cu ep_p2p_*): only the rows that exist cross the
// link, the forward never synchronises the host, and it can be captured in
// a CUDA graph.  NF_EP_TRANSPORT=nvlink selects it (kEpNvlinkDefault when
// unset); when a mailbox cannot be mapped on some rank, or NCCL is chosen,
// every rank uses NCCL point-to-point, with the host synchronisation for the
// counts.
#include "nf_handle.h"

#include "nf_nccl.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <mutex>

using namespace nf;

namespace {

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

// The transport an EP group uses when NF_EP_TRANSPORT is not set.
constexpr bool kEpNvlinkDefault = true;

// Bytes of one record of the set-up exchanges (ep_allgather_host).
constexpr size_t kEpRecBytes = 256;

// Every rank's copy of a small set-up record (nccl_allgather_records over
// the handle's staging buffer, h->ep_stage).
bool ep_allgather_host(nf_moe* h, const void* mine, size_t bytes, void* all) {
    if (bytes > kEpRecBytes) return false;  // the same on every rank: no exchange is posted anywhere
    return nccl_allgather_records(h->nccl, h->ep_stage, h->stream, h->ep_world, mine, bytes, all);
}

// The words a set-up record's failure status is reported with.
const char* setup_failure_what(int status) {
    return status == NF_ERR_NOMEM ? "device allocation" : status == NF_ERR_CUDA ? "initialisation" : "handle creation";
}

// Peer-memory transport set-up (collective: every rank calls it after the
// communicator exists).  Leaves h->ep_p2p false, with nothing mapped, unless
// every rank exported its mailbox and mapped every other rank's.
// prior_fail: a status (not NF_OK) when this rank's create already failed
// before the communicator existed; the rank then allocates nothing here and
// reports the failure in the first exchange, so every rank fails together.
int ep_p2p_setup(nf_moe* h, std::string* err, int prior_fail) {
    const nf_moe_desc& d = h->d;
    const int R = h->ep_world, me = h->ep_rank;
    const int64_t H = d.hidden, cap = static_cast<int64_t>(d.max_tokens) * d.top_k;
    const int64_t ob = d.expert_kind == NF_EXPERTS_NVFP4 ? 2 : 4;
    EpLayout& L = h->ep_lay;
    L.cap = static_cast<int>(cap);
    L.flags_recv = 0;
    L.flags_ret = 64;
    L.cnt = 128;
    L.off = 192;
    L.e = 256;
    L.rows = align256(L.e + R * cap * 4);
    L.ret = align256(L.rows + R * cap * H * 2);
    L.total = align256(L.ret + cap * H * ob);
    // A local failure here does not return at once: the other ranks are about
    // to enter the handle exchange, so this rank joins it too, reporting the
    // failure, and every rank then fails the create together.
    int local_fail = prior_fail;  // NF_OK, or the failure's status
    // ep_done: the send's and the return's per-peer block counters, then the
    // fused return's finished-tile counter
    if (local_fail != NF_OK) {
        // nothing to allocate: the create already failed on this rank
    } else if (!h->alloc(&h->ep_mbox, L.total) || !h->alloc(&h->ep_epoch, 1) ||
               !h->alloc(&h->ep_done, 2 * kEpMaxRanks + 1) || !h->alloc(&h->ep_seen, kEpMaxRanks)) {
        cudaGetLastError();
        local_fail = NF_ERR_NOMEM;
    } else if (cudaMemset(h->ep_mbox, 0, L.total) != cudaSuccess || cudaMemset(h->ep_epoch, 0, 4) != cudaSuccess ||
               cudaMemset(h->ep_done, 0, (2 * kEpMaxRanks + 1) * 4) != cudaSuccess ||
               cudaMemset(h->ep_seen, 0, kEpMaxRanks * 4) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        local_fail = NF_ERR_CUDA;
    }
    struct Rec {
        cudaIpcMemHandle_t handle;
        int32_t ok;      // the mailbox is exported (a zeroed record: not)
        int32_t sound;   // 1: this rank's set-up succeeded so far (a zeroed record: failed)
        int32_t status;  // the failure's status when sound == 0
        int32_t pad[13];
    };
    static_assert(sizeof(Rec) % 16 == 0 && sizeof(Rec) <= kEpRecBytes, "record size");
    // NF_EP_TRANSPORT=nvlink | nccl chooses; unset: kEpNvlinkDefault
    const char* tr = std::getenv("NF_EP_TRANSPORT");
    const bool want = tr ? std::strcmp(tr, "nvlink") == 0 : kEpNvlinkDefault;
    Rec mine{};
    mine.sound = local_fail == 0;
    mine.status = local_fail;
    mine.ok = !local_fail && want && cudaIpcGetMemHandle(&mine.handle, h->ep_mbox) == cudaSuccess;
    cudaGetLastError();
    std::vector<Rec> all(static_cast<size_t>(R));
    if (!ep_allgather_host(h, &mine, sizeof(Rec), all.data())) {
        *err = "mailbox handle exchange failed";
        return NF_ERR_CUDA;
    }
    // every rank reads the same records, so every rank takes this branch or none
    for (int p = 0; p < R; ++p) {
        const Rec& q = all[static_cast<size_t>(p)];
        if (!q.sound) {
            char msg[128];
            std::snprintf(msg, sizeof(msg), "expert-parallel set-up failed on rank %d (%s)", p,
                          setup_failure_what(q.status));
            *err = msg;
            return q.status != NF_OK ? q.status : NF_ERR_NOMEM;
        }
    }
    int opened = 1;
    for (int p = 0; p < R; ++p) opened &= all[static_cast<size_t>(p)].ok ? 1 : 0;
    h->ep_peers.mbox[me] = h->ep_mbox;
    for (int p = 0; p < R && opened; ++p) {
        if (p == me) continue;
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[static_cast<size_t>(p)].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            opened = 0;
            break;
        }
        h->ep_peers.mbox[p] = static_cast<uint8_t*>(ptr);
    }
    // every rank must have mapped every peer
    Rec done{};
    done.ok = opened;
    if (!ep_allgather_host(h, &done, sizeof(Rec), all.data())) {
        *err = "mailbox mapping agreement failed";
        return NF_ERR_CUDA;
    }
    int every = 1;
    for (int p = 0; p < R; ++p) every &= all[static_cast<size_t>(p)].ok ? 1 : 0;
    if (!every) {
        for (int p = 0; p < R; ++p)
            if (p != me && h->ep_peers.mbox[p]) cudaIpcCloseMemHandle(h->ep_peers.mbox[p]);
        for (int p = 0; p < kEpMaxRanks; ++p) h->ep_peers.mbox[p] = nullptr;
        // every rank falls back together; once all have closed their mappings
        // (the exchange below is the barrier) the mailbox goes
        if (!ep_allgather_host(h, &done, sizeof(Rec), all.data())) {
            *err = "mailbox release agreement failed";
            return NF_ERR_CUDA;
        }
        h->release(h->ep_mbox);
        h->ep_mbox = nullptr;
        return NF_OK;  // NCCL transport
    }
    h->ep_p2p = true;
    return NF_OK;
}

}  // namespace

// One forward over the peer-memory transport: no host synchronisation.
static int ep_forward_p2p(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, int32_t* idx,
                          float* w, StageRec& rec, cudaStream_t s) {
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, K = d.top_k, Is = d.shared_inter, R = h->ep_world, me = h->ep_rank;
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    const int out_bytes = H * (fp4 ? 2 : 4);
    const EpLayout& L = h->ep_lay;
    int st = NF_OK;
    cudaError_t e = cudaSuccess;
    if (T > 0 && Is > 0 && (st = launch_shared_expert(h, x, T, rec, s)) != NF_OK) return st;
    rec.begin(NF_STAGE_ROUTER, s);
    if (T > 0) {
        e = route_tokens(h, x, T, idx, w, s);
        if (e == cudaSuccess)
            e = launch_ep_pack(idx, T, K, h->ep_route, d.experts, R, h->ep_slot, h->ep_send_tok, h->ep_send_e, h->ep_cnt, s);
    } else {
        e = cudaMemsetAsync(h->ep_cnt, 0, R * sizeof(int32_t), s);
    }
    if (e == cudaSuccess)
        e = launch_ep_p2p_send(x, h->ep_send_tok, h->ep_send_e, h->ep_cnt, H, R, me, h->ep_peers, L, h->ep_epoch,
                               h->ep_done, s);
    if (e == cudaSuccess) e = launch_ep_p2p_recv_wait(h->ep_mbox, L, R, h->ep_epoch, h->ep_seen, h->dev_err, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "route and send");
    rec.end(NF_STAGE_ROUTER, s);
    // this rank's experts over the [world][cap] receive slots (empty slots carry
    // expert -1).  NVFP4 experts: the down GEMM's epilogue stores each output
    // row straight into its source's mailbox and its last tile publishes the
    // flags (the return overlaps the GEMM); BF16 experts: a return kernel after it.
    nf_moe* in = h->inner;
    GemmArgs epr{};
    epr.ep_world = R;
    epr.ep_me = me;
    epr.ep_cap = L.cap;
    epr.ep_ret_off = L.ret;
    epr.ep_flags_ret = L.flags_ret;
    for (int p = 0; p < kEpMaxRanks; ++p) epr.ep_mbox[p] = h->ep_peers.mbox[p];
    epr.ep_src_off = reinterpret_cast<const int32_t*>(h->ep_mbox + L.off);
    epr.ep_epoch = h->ep_epoch;
    epr.ep_tiles_done = h->ep_done + 2 * kEpMaxRanks;
    if ((st = launch_routed_experts(in, reinterpret_cast<const uint16_t*>(h->ep_mbox + L.rows),
                                    reinterpret_cast<const int32_t*>(h->ep_mbox + L.e), R * L.cap, 1, rec, s, 1, nullptr,
                                    nullptr, fp4 ? &epr : nullptr)) != NF_OK)
        return h->fail(st, "%s", in->err.c_str());
    rec.begin(NF_STAGE_COMBINE, s);
    if (!fp4)
        e = launch_ep_p2p_return(in->down, in->pb.pair_row, out_bytes, R, me, h->ep_peers, L, h->ep_mbox, h->ep_seen,
                                 h->ep_epoch, h->ep_done, s);
    if (e == cudaSuccess) e = launch_ep_p2p_ret_wait(h->ep_mbox, L, R, h->ep_epoch, h->dev_err, s);
    if (e != cudaSuccess) return h->cuda_fail(e, "output return");
    if (T > 0) {
        if (Is > 0 && (e = cudaStreamWaitEvent(s, h->ev_join, 0)) != cudaSuccess) return h->cuda_fail(e, "shared expert join");
        e = launch_combine(h->ep_mbox + L.ret, fp4, h->ep_slot, w, Is > 0 ? h->sh_out : nullptr, residual, T, K, H, y, s);
        if (e != cudaSuccess) return h->cuda_fail(e, "combine launch");
    }
    rec.end(NF_STAGE_COMBINE, s);
    return NF_OK;
}

// Rows, expert ids and outputs of one forward cross the group in three
// grouped exchanges; `rows` are element counts per peer (host side).
int ep_forward(nf_moe* h, const uint16_t* x, const float* residual, int T, float* y, int32_t* idx_user,
               float* w_user, cudaStream_t s) {
    const nf_moe_desc& d = h->d;
    const int H = d.hidden, K = d.top_k, Is = d.shared_inter, R = h->ep_world;
    const bool fp4 = d.expert_kind == NF_EXPERTS_NVFP4;
    const int out_bytes = H * (fp4 ? 2 : 4);  // a down row: BF16 (NVFP4 experts) or F32 (BF16 experts)
    int32_t* idx = idx_user ? idx_user : h->topk_idx;
    float* w = w_user ? w_user : h->topk_w;
    ncclComm_t comm = static_cast<ncclComm_t>(h->nccl);
    NcclApi& api = nccl();
    h->last_tokens = T;
    StageRec rec;
    rec.h = h;
    rec.ev = h->prof_begin(&rec.set);
    if (h->ep_p2p) return ep_forward_p2p(h, x, residual, T, y, idx, w, rec, s);
    int st = NF_OK;
    cudaError_t e = cudaSuccess;
    ncclResult_t r = ncclSuccess;
    if (T > 0 && Is > 0 && (st = launch_shared_expert(h, x, T, rec, s)) != NF_OK) return st;
    // route, lay out, count
    rec.begin(NF_STAGE_ROUTER, s);
    if (T > 0) {
        e = route_tokens(h, x, T, idx, w, s);
        if (e == cudaSuccess)
            e = launch_ep_pack(idx, T, K, h->ep_route, d.experts, R, h->ep_slot, h->ep_send_tok, h->ep_send_e, h->ep_cnt, s);
        if (e == cudaSuccess) e = launch_gather_rows(x, h->ep_send_tok, T * K, H * 2, h->ep_send, s);
    } else {
        e = cudaMemsetAsync(h->ep_cnt, 0, R * sizeof(int32_t), s);
    }
    if (e != cudaSuccess) return h->cuda_fail(e, "route and pack");
    r = api.group_start();
    for (int p = 0; p < R && r == ncclSuccess; ++p) {
        r = api.send(h->ep_cnt + p, 1, ncclInt32, p, comm, s);
        if (r == ncclSuccess) r = api.recv(h->ep_cnt + R + p, 1, ncclInt32, p, comm, s);
    }
    const ncclResult_t r2 = api.group_end();
    if (r == ncclSuccess) r = r2;
    if (r != ncclSuccess) return h->fail(NF_ERR_CUDA, "count exchange: %s", nccl_str(r));
    if ((e = cudaMemcpyAsync(h->ep_hcnt, h->ep_cnt, 2 * R * sizeof(int32_t), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (e = cudaStreamSynchronize(s)) != cudaSuccess)
        return h->cuda_fail(e, "count exchange");
    int64_t soff[kEpMaxRanks + 1] = {0}, roff[kEpMaxRanks + 1] = {0};
    for (int p = 0; p < R; ++p) {
        soff[p + 1] = soff[p] + h->ep_hcnt[p];
        roff[p + 1] = roff[p] + h->ep_hcnt[R + p];
    }
    const int64_t n_recv = roff[R];
    if (soff[R] != static_cast<int64_t>(T) * K || n_recv > static_cast<int64_t>(R) * d.max_tokens * K)
        return h->fail(NF_ERR_CAPACITY, "expert-parallel exchange: %lld rows received, capacity %lld",
                       static_cast<long long>(n_recv), static_cast<long long>(R) * d.max_tokens * K);
    // rows and their destination-local experts
    r = api.group_start();
    for (int p = 0; p < R && r == ncclSuccess; ++p) {
        const size_t sc = static_cast<size_t>(h->ep_hcnt[p]), rc = static_cast<size_t>(h->ep_hcnt[R + p]);
        if (sc) {
            r = api.send(h->ep_send + soff[p] * H, sc * H * 2, ncclUint8, p, comm, s);
            if (r == ncclSuccess) r = api.send(h->ep_send_e + soff[p], sc, ncclInt32, p, comm, s);
        }
        if (rc && r == ncclSuccess) {
            r = api.recv(h->ep_recv + roff[p] * H, rc * H * 2, ncclUint8, p, comm, s);
            if (r == ncclSuccess) r = api.recv(h->ep_recv_e + roff[p], rc, ncclInt32, p, comm, s);
        }
    }
    const ncclResult_t r3 = api.group_end();
    if (r == ncclSuccess) r = r3;
    if (r != ncclSuccess) return h->fail(NF_ERR_CUDA, "row exchange: %s", nccl_str(r));
    rec.end(NF_STAGE_ROUTER, s);
    // this rank's experts on the received rows (top-1 picks), back in receive order
    nf_moe* in = h->inner;
    if (n_recv > 0) {
        if ((st = launch_routed_experts(in, h->ep_recv, h->ep_recv_e, static_cast<int>(n_recv), 1, rec, s)) != NF_OK)
            return h->fail(st, "%s", in->err.c_str());
        e = launch_gather_rows(in->down, in->pb.pair_row, static_cast<int>(n_recv), out_bytes, h->ep_back, s);
        if (e != cudaSuccess) return h->cuda_fail(e, "expert output gather");
    }
    // outputs back to their source ranks, then the single-GPU combine
    rec.begin(NF_STAGE_COMBINE, s);
    r = api.group_start();
    for (int p = 0; p < R && r == ncclSuccess; ++p) {
        const size_t sc = static_cast<size_t>(h->ep_hcnt[p]), rc = static_cast<size_t>(h->ep_hcnt[R + p]);
        if (rc) r = api.send(static_cast<uint8_t*>(h->ep_back) + roff[p] * out_bytes, rc * out_bytes, ncclUint8, p, comm, s);
        if (sc && r == ncclSuccess)
            r = api.recv(static_cast<uint8_t*>(h->ep_ret) + soff[p] * out_bytes, sc * out_bytes, ncclUint8, p, comm, s);
    }
    const ncclResult_t r4 = api.group_end();
    if (r == ncclSuccess) r = r4;
    if (r != ncclSuccess) return h->fail(NF_ERR_CUDA, "output exchange: %s", nccl_str(r));
    if (T > 0) {
        if (Is > 0 && (e = cudaStreamWaitEvent(s, h->ev_join, 0)) != cudaSuccess) return h->cuda_fail(e, "shared expert join");
        e = launch_combine(h->ep_ret, fp4, h->ep_slot, w, Is > 0 ? h->sh_out : nullptr, residual, T, K, H, y, s);
        if (e != cudaSuccess) return h->cuda_fail(e, "combine launch");
    }
    rec.end(NF_STAGE_COMBINE, s);
    return NF_OK;
}

void ep_release(nf_moe* h) {
    for (int p = 0; p < kEpMaxRanks; ++p)
        if (h->ep_peers.mbox[p] && h->ep_peers.mbox[p] != h->ep_mbox) {
            cudaSetDevice(h->device);
            cudaIpcCloseMemHandle(h->ep_peers.mbox[p]);
            h->ep_peers.mbox[p] = nullptr;
        }
    if (h->nccl) {
        cudaSetDevice(h->device);
        nccl().comm_destroy(static_cast<ncclComm_t>(h->nccl));
        h->nccl = nullptr;
    }
    if (h->inner) {
        nf_moe_destroy(h->inner);
        h->inner = nullptr;
    }
    if (h->ep_hcnt) {
        cudaFreeHost(h->ep_hcnt);
        h->ep_hcnt = nullptr;
    }
}

extern "C" {

int nf_ep_unique_id(uint8_t* out, int len) {
    if (!out || len < NF_EP_ID_BYTES) return NF_ERR_INVALID;
    NcclApi& api = nccl();
    if (!api.ok) {
        create_error() = api.why;
        return NF_ERR_UNSUPPORTED;
    }
    static_assert(sizeof(ncclUniqueId) == NF_EP_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    const ncclResult_t r = api.get_unique_id(&id);
    if (r != ncclSuccess) {
        create_error() = std::string("ncclGetUniqueId: ") + nccl_str(r);
        return NF_ERR_CUDA;
    }
    std::memcpy(out, &id, sizeof(id));
    return NF_OK;
}

int nf_moe_ep_transport(const nf_moe* h) {
    if (!h || !h->ep_outer) return NF_EP_NONE;
    return h->ep_p2p ? NF_EP_NVLINK : NF_EP_NCCL;
}

int nf_moe_create_ep(const nf_moe_desc* desc, int device, int rank, int world, const uint8_t* group_id, int id_len,
                     nf_moe** out) {
    return nf_moe_create_ep_replicated(desc, device, rank, world, group_id, id_len, nullptr, 0, out);
}

int nf_moe_create_ep_replicated(const nf_moe_desc* desc, int device, int rank, int world, const uint8_t* group_id,
                                int id_len, const int32_t* replicas, int n_replicas, nf_moe** out) {
    std::string& err = create_error();
    err.clear();
    if (!desc || !out || !group_id || id_len < NF_EP_ID_BYTES) {
        err = "null descriptor, output or group id";
        return NF_ERR_INVALID;
    }
    if (n_replicas < 0 || (n_replicas > 0 && !replicas)) {
        err = "bad replica list";
        return NF_ERR_INVALID;
    }
    *out = nullptr;
    const nf_moe_desc& d = *desc;
    int st = validate_desc(d, &err);
    if (st != NF_OK) return st;
    if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world) {
        err = "expert parallelism needs 1 <= world <= 8 and 0 <= rank < world";
        return NF_ERR_UNSUPPORTED;
    }
    if (d.experts % world != 0) {
        err = "the experts must divide evenly over the ranks";
        return NF_ERR_UNSUPPORTED;
    }
    std::vector<char> seen(static_cast<size_t>(d.experts), 0);
    for (int j = 0; j < n_replicas; ++j) {
        const int e = replicas[j];
        if (e < 0 || e >= d.experts || seen[static_cast<size_t>(e)]) {
            err = "replicas must be distinct expert ids in [0, experts)";
            return NF_ERR_INVALID;
        }
        seen[static_cast<size_t>(e)] = 1;
    }
    NcclApi& api = nccl();
    if (!api.ok) {
        err = api.why;
        return NF_ERR_UNSUPPORTED;
    }
    nf_moe* h = nullptr;
    if ((st = create_impl(d, device, kRoleEpOuter, &h, &err)) != NF_OK) return st;
    h->ep_rank = rank;
    h->ep_world = world;
    h->ep_local = d.experts / world;
    h->ep_base = rank * h->ep_local;
    for (int j = 0; j < n_replicas; ++j)  // the replicas this rank does not own already
        if (replicas[j] < h->ep_base || replicas[j] >= h->ep_base + h->ep_local) h->ep_rep.push_back(replicas[j]);
    // the rank's experts (its own, then its replicas): top-1 picks over rows
    // received from every rank
    nf_moe_desc di = d;
    di.experts = h->ep_local + static_cast<int>(h->ep_rep.size());
    di.top_k = 1;
    di.shared_inter = 0;
    di.n_group = 1;
    di.topk_group = 1;
    di.normalize = 0;
    di.routed_scaling = 1.f;
    di.max_tokens = world * d.max_tokens * d.top_k;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    // The staging buffer of the set-up exchanges comes first: with it this
    // rank can join them whatever fails next.  Without it the rank cannot,
    // and it returns before the communicator exists (the other ranks' own
    // communicator initialisation then waits for it).
    if (!h->alloc(&h->ep_stage, kEpRecBytes * (world + 1))) {
        cudaGetLastError();
        cudaSetDevice(prev);
        nf_moe_destroy(h);
        err = "device allocation failed";
        return NF_ERR_NOMEM;
    }
    // From here a local failure does not return at once: the other ranks are
    // about to initialise the communicator and enter the first set-up
    // exchange, so this rank joins both and reports the failure there
    // (ep_p2p_setup), and every rank fails the create together.
    int local_fail = NF_OK;
    std::string local_err;
    cudaSetDevice(prev);
    local_fail = create_impl(di, device, kRoleExperts, &h->inner, &local_err);
    cudaSetDevice(device);
    const int64_t H = d.hidden, pairs = static_cast<int64_t>(d.max_tokens) * d.top_k, cap = world * pairs;
    const int64_t ob = d.expert_kind == NF_EXPERTS_NVFP4 ? 2 : 4;
    // the send layout, used by both transports (the NCCL transport's own
    // buffers follow once the group has chosen it)
    bool ok = local_fail == NF_OK && h->alloc(&h->ep_send_e, pairs) && h->alloc(&h->ep_send_tok, pairs) &&
              h->alloc(&h->ep_slot, pairs) && h->alloc(&h->ep_cnt, 2 * world) && h->alloc(&h->ep_route, 2 * d.experts);
    if (ok) {
        // where each expert's picks go: its owner and its index there, or this
        // rank's replica slot
        std::vector<int32_t> route(static_cast<size_t>(2 * d.experts));
        for (int e = 0; e < d.experts; ++e) {
            int dest = e / h->ep_local, loc = e % h->ep_local;
            for (size_t j = 0; j < h->ep_rep.size(); ++j)
                if (h->ep_rep[j] == e) dest = rank, loc = h->ep_local + static_cast<int>(j);
            route[static_cast<size_t>(e)] = dest;
            route[static_cast<size_t>(d.experts + e)] = loc;
        }
        ok = cudaMemcpy(h->ep_route, route.data(), route.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    if (local_fail == NF_OK && !ok) {
        cudaGetLastError();
        local_fail = NF_ERR_NOMEM;
        local_err = "device allocation failed";
    }
    ncclUniqueId id;
    std::memcpy(&id, group_id, sizeof(id));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api.comm_init_rank(&comm, world, id, rank);
    cudaSetDevice(prev);
    if (r != ncclSuccess) {
        nf_moe_destroy(h);
        err = std::string("ncclCommInitRank: ") + nccl_str(r);
        return NF_ERR_CUDA;
    }
    h->nccl = comm;
    cudaSetDevice(device);
    st = ep_p2p_setup(h, &err, local_fail);
    if (local_fail != NF_OK && st == local_fail && !local_err.empty()) err = local_err;  // this rank's own reason
    if (st == NF_OK && !h->ep_p2p) {
        // NCCL transport: packed rows, receive and return buffers, host counts
        uint8_t* back = nullptr;
        uint8_t* ret = nullptr;
        ok = h->alloc(&h->ep_send, pairs * H) && h->alloc(&h->ep_recv, cap * H) && h->alloc(&h->ep_recv_e, cap) &&
             h->alloc(&back, cap * H * ob) && h->alloc(&ret, pairs * H * ob) &&
             cudaMallocHost(&h->ep_hcnt, 2 * world * sizeof(int32_t)) == cudaSuccess;
        h->ep_back = back;
        h->ep_ret = ret;
        if (!ok) cudaGetLastError();
        // the group agrees: a rank that could not allocate must not leave the
        // others waiting in their first exchange
        struct Ok {
            int32_t ok;
            int32_t pad[3];
        } mine{ok ? 1 : 0, {}};
        std::vector<Ok> all(static_cast<size_t>(world));
        if (!ep_allgather_host(h, &mine, sizeof(Ok), all.data())) {
            err = "allocation agreement failed";
            st = NF_ERR_CUDA;
        } else {
            for (const Ok& o : all) ok = ok && o.ok;
            if (!ok) {
                err = mine.ok ? "device allocation failed on another rank" : "device allocation failed";
                st = NF_ERR_NOMEM;
            }
        }
    }
    cudaSetDevice(prev);
    if (st != NF_OK) {
        nf_moe_destroy(h);
        return st;
    }
    *out = h;
    return NF_OK;
}

}  // extern "C"
