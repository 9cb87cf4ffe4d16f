"""Host-side statement of the expert-parallel exchange layout (numpy).

The library's EP forward (csrc/nf_ep.cu, ep_pack_kernel in csrc/nf_kernels.cu)
sends every (token, pick) of a rank to the rank that owns the picked expert,
in (destination, token, pick) order, and combines the returned expert outputs
in pick order.  This module restates that layout so that a host (or a test)
can reason about it without a GPU: which rank owns an expert, the send slot
of every pick, the rows and destination-local experts in send order, the
per-destination counts and the receive offsets.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def owner(expert: np.ndarray, experts: int, world: int) -> np.ndarray:
    """Rank that owns each (global) expert id: experts [r E/R, (r+1) E/R)."""
    if experts % world:
        raise ValueError("the experts must divide evenly over the ranks")
    return np.asarray(expert) // (experts // world)


@dataclass
class SendPlan:
    slot: np.ndarray        # [T, K] send slot of each pick (the combine's pair_row)
    send_token: np.ndarray  # [T*K] source token of each slot
    send_expert: np.ndarray # [T*K] destination-local expert of each slot
    counts: np.ndarray      # [world] picks sent to each rank
    offsets: np.ndarray     # [world + 1] first slot of each destination


def pack(idx: np.ndarray, experts: int, world: int) -> SendPlan:
    """The (destination, token, pick) layout of a rank's picks; idx [T, K]."""
    idx = np.asarray(idx, dtype=np.int64)
    T, K = idx.shape
    per = experts // world
    dest = owner(idx, experts, world).ravel()
    counts = np.bincount(dest, minlength=world).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    order = np.argsort(dest, kind="stable")  # stable: token-major, pick-minor inside a destination
    slot = np.empty(T * K, np.int64)
    slot[order] = np.arange(T * K)
    flat = np.arange(T * K)
    send_token = np.empty(T * K, np.int64)
    send_expert = np.empty(T * K, np.int64)
    send_token[slot] = flat // K
    send_expert[slot] = idx.ravel() - dest * per
    return SendPlan(slot.reshape(T, K), send_token, send_expert, counts, offsets)


def receive_offsets(recv_counts: np.ndarray) -> np.ndarray:
    """First received row of each source rank (rows arrive in rank order)."""
    return np.concatenate([[0], np.cumsum(np.asarray(recv_counts, dtype=np.int64))])


def mailbox_exchange(plans: list, cap: int):
    """The NVLink peer-memory exchange (ep_p2p_* kernels) restated over the
    send plans of every rank (plans[r] = pack(...) of rank r): owner p's
    receive slots [world][cap] hold, for source s, s's rows for p in s's send
    order followed by empty slots (expert -1), plus s's send offset for p.
    Returns, per owner, (expert [world, cap], source slot [world, cap] -- the
    sender's slot of each row, -1 for an empty slot -- and the offsets [world])
    so that a row at (s, j) returns to slot offsets[s] + j of rank s."""
    world = len(plans)
    out = []
    for p in range(world):
        expert = np.full((world, cap), -1, np.int64)
        src_slot = np.full((world, cap), -1, np.int64)
        offs = np.zeros(world, np.int64)
        for s, plan in enumerate(plans):
            lo, n = int(plan.offsets[p]), int(plan.counts[p])
            if n > cap:
                raise ValueError("a source sent more rows than the mailbox holds")
            expert[s, :n] = plan.send_expert[lo:lo + n]
            src_slot[s, :n] = np.arange(lo, lo + n)
            offs[s] = lo
        out.append((expert, src_slot, offs))
    return out


NF_OK, NF_ERR_CUDA, NF_ERR_UNSUPPORTED, NF_ERR_NOMEM = 0, 6, 8, 9


def setup_failure_what(status: int) -> str:
    """The words a set-up record's failure status is reported with
    (setup_failure_what in csrc/nf_ep.cu)."""
    return {NF_ERR_NOMEM: "device allocation", NF_ERR_CUDA: "initialisation"}.get(status, "handle creation")


def setup_agreement(exchange, local_status: int, want_nvlink: bool, export_ok: bool, map_peers) -> tuple:
    """The collective steps of an EP group's transport set-up (ep_p2p_setup in
    csrc/nf_ep.cu), restated so that the protocol can be run by CPU ranks.

    exchange(record) -> every rank's record (an all-gather); local_status is
    this rank's set-up outcome so far: NF_OK, or the status of a failure in
    its handle creation before the communicator existed (the inner experts
    handle or the send buffers: NF_ERR_NOMEM and the like, nf_moe_create_ep)
    or in its mailbox allocation / initialisation (NF_ERR_NOMEM,
    NF_ERR_CUDA); export_ok whether its mailbox could be exported;
    map_peers() maps every peer's mailbox and returns success.

    A rank whose own set-up failed still joins the first exchange and reports
    the failure there, so no rank is left waiting in it; every rank reads the
    same records, so every rank then fails together with the failing rank's
    status (the lowest failing rank's, when several fail).  Otherwise every rank maps its peers, the group agrees on whether
    all did (second exchange), and falls back to NCCL together when one did
    not (a third exchange is the barrier before the mailboxes are released).
    Returns (status, transport or message, exchanges taken)."""
    n = 0
    sound = local_status == NF_OK
    recs = exchange({"ok": bool(sound and want_nvlink and export_ok), "sound": sound, "status": local_status})
    n += 1
    for p, q in enumerate(recs):
        if not q["sound"]:
            return q["status"], f"expert-parallel set-up failed on rank {p} ({setup_failure_what(q['status'])})", n
    opened = all(q["ok"] for q in recs) and bool(map_peers())
    recs = exchange({"ok": opened})
    n += 1
    if not all(q["ok"] for q in recs):
        exchange({"ok": opened})  # every rank has closed its mappings before the mailboxes go
        n += 1
        return NF_OK, "nccl", n
    return NF_OK, "nvlink", n
