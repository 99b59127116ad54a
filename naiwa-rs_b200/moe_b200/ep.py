"""Expert parallelism: experts sharded across ranks, tokens exchanged around the per-rank layer.

No counterpart in the reference (naiwa-rs runs one GPU plus CPU offload). Rank r owns the experts
[r * experts_per_rank, (r + 1) * experts_per_rank) as an ordinary `RoutedExperts` layer with local
ids. A forward on rank r's own tokens:

  1. `ep_dispatch`   (device): one send row per (token, destination rank that owns one of its
                     experts), ordered by rank then token, with the row's k slots re-targeted to
                     local ids (MOE_ID_NONE / weight 0 for slots owned elsewhere);
  2. `ep_pack_rows`  (device): gather the tokens' bf16 rows into the send buffer;
  3. `exchange`      (NCCL): all-to-all of the W row counts, then ragged all-to-alls of the rows
                     and of their (id, weight) slots;
  4. local forward   (device): `RoutedExperts.forward` on the received rows;
  5. `return_rows`   (NCCL): ragged all-to-all of the outputs back to their sources;
  6. `ep_combine`    (device): per token, the shared-expert output (if any) plus the returned
                     rows in rank order, f32, rounded once to bf16.

Steps 3 and 5 are plain torch.distributed collectives (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import ctypes
from typing import Optional

from ._lib import check, lib
from .layer import _ptr, _stream, _torch


# ---- device kernels -----------------------------------------------------------------------------

def ep_dispatch(ids, weights, experts_per_rank: int, world: int, error_word=None, stream=None):
    """Dispatch plan of [T, k] global ids/weights (CUDA). Returns a dict of device tensors:
    rank_counts [world], n_send [1], token_rows [T, world], send_token [cap], send_ids [cap, k] (int32
    view of u32), send_w [cap, k]; cap = T * min(world, k)."""
    torch = _torch()
    ids = ids.to(torch.int32).contiguous()
    weights = weights.to(torch.float32).contiguous()
    T, k = ids.shape
    dev = ids.device
    cap = max(T * min(world, k), 1)
    out = {
        "rank_counts": torch.empty(world, dtype=torch.int32, device=dev),
        "n_send": torch.empty(1, dtype=torch.int32, device=dev),
        "token_rows": torch.empty((max(T, 1), world), dtype=torch.int32, device=dev),
        "send_token": torch.empty(cap, dtype=torch.int32, device=dev),
        "send_ids": torch.empty((cap, k), dtype=torch.int32, device=dev),
        "send_w": torch.empty((cap, k), dtype=torch.float32, device=dev),
        "cap": cap,
    }
    err = error_word if error_word is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().moe_ep_dispatch_plan(_ptr(ids), _ptr(weights), T, k, experts_per_rank, world, _ptr(out["rank_counts"]),
                                     _ptr(out["n_send"]), _ptr(out["token_rows"]), _ptr(out["send_token"]),
                                     _ptr(out["send_ids"]), _ptr(out["send_w"]), _ptr(err),
                                     ctypes.c_void_p(_stream(stream))))
    out["error_word"] = err
    return out


def ep_pack_rows(x, send_token, n_send, cap: int, stream=None):
    """send_x[row] = x[send_token[row]] for row < n_send (device count). x [T, H] bf16 (CUDA)."""
    torch = _torch()
    x = x.contiguous()
    T, H = x.shape
    send_x = torch.empty((max(cap, 1), H), dtype=x.dtype, device=x.device)
    check(lib().moe_ep_pack_rows(_ptr(x), T, H, _ptr(send_token), _ptr(n_send), cap, _ptr(send_x),
                                 ctypes.c_void_p(_stream(stream))))
    return send_x


def ep_combine(y_back, token_rows, T: int, y_add=None, stream=None):
    """y[t] = y_add[t] + sum_r y_back[token_rows[t, r]] (bf16 out, f32 accumulation)."""
    torch = _torch()
    world = token_rows.shape[1]
    H = y_back.shape[1]
    y = torch.empty((T, H), dtype=torch.bfloat16, device=y_back.device)
    check(lib().moe_ep_combine(_ptr(y_back.contiguous()), _ptr(token_rows), T, world, H,
                               _ptr(y_add.contiguous() if y_add is not None else None), _ptr(y),
                               ctypes.c_void_p(_stream(stream))))
    return y


# ---- exchange (torch.distributed) ---------------------------------------------------------------

def _single(group) -> bool:
    import torch.distributed as dist

    return not dist.is_initialized() or dist.get_world_size(group) == 1


def exchange_counts(rank_counts, group=None):
    """All-to-all of the per-destination row counts; returns (send_counts, recv_counts) as lists.
    A single rank (no process group) exchanges with itself."""
    torch = _torch()
    import torch.distributed as dist

    if _single(group):
        c = [int(v) for v in rank_counts.tolist()]
        return c, list(c)
    recv = torch.empty_like(rank_counts)
    dist.all_to_all_single(recv, rank_counts.contiguous(), group=group)
    return [int(v) for v in rank_counts.tolist()], [int(v) for v in recv.tolist()]


def exchange_rows(send, send_counts, recv_counts, group=None):
    """Ragged all-to-all of row-major `send` ([>= sum(send_counts), ...]): rows for rank r are the
    r-th section; returns the received rows [sum(recv_counts), ...] in source-rank order."""
    torch = _torch()
    import torch.distributed as dist

    n = sum(send_counts)
    if _single(group):
        return send[:n]
    recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send[:n].contiguous(), output_split_sizes=recv_counts,
                           input_split_sizes=send_counts, group=group)
    return recv


# ---- the layer -----------------------------------------------------------------------------------

class ExpertParallelMoE:
    """One rank's share of an expert-parallel MoE layer.

    `local` is a RoutedExperts built over this rank's experts (local ids 0 .. experts_per_rank - 1)
    with max_tokens >= the rows it may receive (T * world for T tokens per rank). `shared`, if given,
    is a RoutedExperts with one expert run on this rank's own tokens (replicated weights) and added
    in the combine. forward(x, topk_weights, topk_ids) takes global ids and returns [T, H] bf16."""

    def __init__(self, local, rank: int, world: int, experts_per_rank: int, group=None, shared=None):
        self.local = local
        self.rank = rank
        self.world = world
        self.epr = experts_per_rank
        self.group = group
        self.shared = shared
        self.last_counts: Optional[tuple] = None

    def forward(self, xs, topk_weights, topk_ids, stream=None):
        torch = _torch()
        T, H = xs.shape
        k = topk_ids.shape[1]
        plan = ep_dispatch(topk_ids, topk_weights, self.epr, self.world, stream=stream)
        send_x = ep_pack_rows(xs, plan["send_token"], plan["n_send"], plan["cap"], stream=stream)
        y_shared = None
        if self.shared is not None:
            ones = torch.ones((T, 1), dtype=torch.float32, device=xs.device)
            zeros = torch.zeros((T, 1), dtype=torch.int32, device=xs.device)
            y_shared = self.shared.forward(xs, ones, zeros)
        send_counts, recv_counts = exchange_counts(plan["rank_counts"], self.group)
        self.last_counts = (send_counts, recv_counts)
        recv_x = exchange_rows(send_x, send_counts, recv_counts, self.group)
        meta = torch.cat([plan["send_ids"], plan["send_w"].view(torch.int32)], dim=1)
        recv_meta = exchange_rows(meta, send_counts, recv_counts, self.group)
        R = recv_x.shape[0]
        if R > 0:
            recv_ids = recv_meta[:, :k].contiguous()
            recv_w = recv_meta[:, k:].contiguous().view(torch.float32)
            y_recv = self.local.forward(recv_x, recv_w, recv_ids)
        else:
            y_recv = torch.empty((0, H), dtype=torch.bfloat16, device=xs.device)
        y_back = exchange_rows(y_recv, recv_counts, send_counts, self.group)
        return ep_combine(y_back if y_back.shape[0] else torch.zeros((1, H), dtype=torch.bfloat16, device=xs.device),
                          plan["token_rows"], T, y_add=y_shared, stream=stream)

    __call__ = forward


class PeerExpertParallelMoE:
    """ExpertParallelMoE with the exchange done by the library's NVLink peer-memory kernels instead of
    NCCL all-to-alls: dispatch rows are stored straight into the destination ranks' receive regions,
    outputs straight back into the sources' return regions, with epoch flags and bounded waits in
    between and no host synchronisation (so a step can be captured in a CUDA graph). Needs one process
    per GPU and world >= 2; the handles are exchanged once through torch.distributed.

    `local` must be built with max_tokens >= world * max_tokens (the rows it may receive)."""

    def __init__(self, local, rank: int, world: int, experts_per_rank: int, max_tokens: int, group=None,
                 shared=None, wait_limit_us: Optional[int] = None):
        torch = _torch()
        import torch.distributed as dist

        self.local, self.rank, self.world, self.epr = local, rank, world, experts_per_rank
        self.cap, self.group, self.shared = int(max_tokens), group, shared
        self.H, self.k = local.hidden, local.top_k
        h = ctypes.c_void_p()
        check(lib().moe_ep_peer_create(local.device, rank, world, self.cap, self.H, self.k, ctypes.byref(h)))
        self._h = h
        if wait_limit_us is not None:
            self.set_wait_limit(wait_limit_us)
        nb = int(lib().moe_ep_peer_handle_bytes())
        mine = (ctypes.c_ubyte * nb)()
        check(lib().moe_ep_peer_export(self._h, ctypes.cast(mine, ctypes.c_void_p)))
        gathered = [None] * world
        dist.all_gather_object(gathered, bytes(mine), group=group)
        allh = (ctypes.c_ubyte * (nb * world)).from_buffer_copy(b"".join(gathered))
        check(lib().moe_ep_peer_connect(self._h, ctypes.cast(allh, ctypes.c_void_p)))
        dist.barrier(group=group)
        dev = torch.device("cuda", local.device)
        R = world * self.cap
        self.recv_ids = torch.empty((R, self.k), dtype=torch.int32, device=dev)
        self.recv_w = torch.empty((R, self.k), dtype=torch.float32, device=dev)
        self.y_local = torch.empty((R, self.H), dtype=torch.bfloat16, device=dev)
        self.recv_rows = lib().moe_ep_peer_recv_rows(self._h)
        # the routed dispatch leaves this rank's slots in its own receive regions
        self.region_ids = lib().moe_ep_peer_recv_ids(self._h)
        self.region_w = lib().moe_ep_peer_recv_weights(self._h)
        # the dispatch plan the routed dispatch writes, sized for cap tokens (moe_ep_dispatch_plan's layout)
        self.plan = {
            "rank_counts": torch.empty(world, dtype=torch.int32, device=dev),
            "token_rows": torch.empty((self.cap, world), dtype=torch.int32, device=dev),
            "error_word": torch.zeros(1, dtype=torch.int32, device=dev),
        }
        # the local forward runs world * cap received rows, about 1 / world of whose slots are live
        local.set_live_hint(1.0 / world)
        self.shared_w = torch.ones((self.cap, 1), dtype=torch.float32, device=dev)
        self.shared_ids = torch.zeros((self.cap, 1), dtype=torch.int32, device=dev)

    def forward(self, xs, topk_weights, topk_ids, out=None, stream=None, layer=None, marks=None):
        """[T, H] bf16 of this rank's T <= max_tokens tokens, global ids [T, k]. Every rank calls it the
        same number of times, in the same order. The epoch is held on the device (epoch 0 in the C
        calls), so a captured graph of calls can be replayed; nothing is allocated but the output when
        `out` is not given. `layer` runs this call's local experts instead of the constructor's (one
        exchange object can serve every layer of a stack: calls are ordered on the stream). `marks`:
        four CUDA events recorded after the dispatch (which ends with the receive), the local forward,
        the return and the combine (per-stage timing; the shared expert, if any, runs between the
        return and the combine, while the peers' rows come back)."""
        torch = _torch()
        T, H = xs.shape
        if T > self.cap:
            raise ValueError("PeerExpertParallelMoE.forward: T exceeds max_tokens")
        st = ctypes.c_void_p(_stream(stream))
        xs = xs.contiguous()
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        ids = ids.contiguous()
        w = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.to(torch.float32)
        w = w.contiguous()
        P = self.plan
        L = lib()
        local = layer if layer is not None else self.local

        def mark(i):
            if marks is not None:
                marks[i].record(stream if stream is not None else torch.cuda.current_stream())
        check(L.moe_ep_peer_dispatch_routed(self._h, _ptr(xs), T, _ptr(ids), _ptr(w), self.epr, 0,
                                            _ptr(P["rank_counts"]), _ptr(P["token_rows"]), _ptr(P["error_word"]), st))
        mark(0)
        R = self.world * self.cap
        check(L.moe_forward(local._h, ctypes.c_void_p(self.recv_rows), R, ctypes.c_void_p(self.region_ids),
                            ctypes.c_void_p(self.region_w), self.k, _ptr(self.y_local), st))
        mark(1)
        check(L.moe_ep_peer_return(self._h, _ptr(self.y_local), 0, st))
        mark(2)
        y_shared = None
        if self.shared is not None:
            y_shared = self.shared.forward(xs, self.shared_w[:T], self.shared_ids[:T], stream=stream)
        y = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=xs.device)
        check(L.moe_ep_peer_combine(self._h, 0, T, _ptr(P["rank_counts"]), _ptr(P["token_rows"]),
                                    _ptr(y_shared), _ptr(y), st))
        mark(3)
        return y

    __call__ = forward

    def set_wait_limit(self, timeout_us: int):
        """How long the device-side waits for other ranks last (default five seconds)."""
        check(lib().moe_ep_peer_set_wait_limit(self._h, int(timeout_us)))

    def check(self, stream=None):
        check(lib().moe_ep_peer_check(self._h, ctypes.c_void_p(_stream(stream))))
        self.local.check()
        if int(self.plan["error_word"].item()) != 0:
            self.plan["error_word"].zero_()
            check(5)  # MOE_ERR_BAD_IDS: a routed id beyond experts_per_rank * world

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_ep_peer_destroy(self._h)
            self._h = ctypes.c_void_p()
