"""Expert parallelism for the MoE layer: token -> expert dispatch/combine over the EP group.

The reference (``inference/model/magi2_preview.py:3277-3327``) shards *heads* across the EP
group and swaps the whole activation with one ``all_to_all_single`` each way; with H=12
heads padded to 16 on 8 ranks, two ranks hold only zero "dummy" heads
(``magi2_preview.py:2514-2537``).  Here the flattened experts ``[0, H*E)`` are split into
``ep`` contiguous ranges (the same dim-0 row slices the reference's EP checkpoint loader
reads when ``H % ep == 0``) and only routed token rows move, in NVFP4, once per
destination rank:

  1. quantise each (head, token) row once; mark the ranks owning any of its K experts and
     sort those (row, rank) pairs by rank (stable) -> send order and per-rank counts;
  2. pack one record per (row, rank): NVFP4 data + scales + {row scale, count, the
     rank's (local expert, prob) pairs};
  3. exchange counts (``all_to_all_single`` of n ints, read on the host), then records;
  4. receiver: expand records into (row, local expert) entries, sort them by expert, run
     the NVFP4 FFN reading the received records in place, and sum each record's experts
     in ascending expert order (fp32, rounded once to bf16) -> one row per record;
  5. send those rows back; the source sums each (head, token)'s per-rank rows in
     ascending rank order — i.e. ascending global expert ranges — and rounds to bf16.

Per token, ~min(n, K) records cross the links each way instead of K rows.  The sum is
grouped by rank, so the result matches the single-GPU layer to bf16 rounding of the
per-rank partial sums (not bit for bit); it is deterministic.

Device steps go through a backend object (``CudaBackend``: libmhmoe kernels) so the host
logic (splits, orders, collectives) is testable on CPU ranks with ``gloo`` by substituting
a reference backend.  The reference-compatible head-sharded ``ep_dispatch`` /
``ep_undispatch`` are kept for ``H % ep == 0`` users.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .fwd import _events


# ───────────────────────── reference-compatible head sharding ─────────────────────────

def ep_dispatch(x: torch.Tensor, ep_group) -> torch.Tensor:
    """(S, H, D) -> (S * ep, H / ep, D): scatter heads, gather sequence (magi2_preview.py:3277-3299)."""
    ep = dist.get_world_size(ep_group) if ep_group is not None else 1
    if ep == 1:
        return x
    S, H, D = x.shape
    assert H % ep == 0, f"Number of heads H ({H}) must be divisible by ep_size ({ep})"
    x = x.contiguous().view(S, ep, H // ep, D).permute(1, 0, 2, 3).contiguous()
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=ep_group)
    return out.view(ep * S, H // ep, D)


def ep_undispatch(x: torch.Tensor, ep_group) -> torch.Tensor:
    """(S * ep, H / ep, D) -> (S, H, D) (magi2_preview.py:3303-3327)."""
    ep = dist.get_world_size(ep_group) if ep_group is not None else 1
    if ep == 1:
        return x
    total, hp, D = x.shape
    assert total % ep == 0, f"Total sequence length ({total}) must be divisible by ep_size ({ep})"
    S = total // ep
    x = x.contiguous().view(ep, S, hp, D)
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x, group=ep_group)
    return out.permute(1, 0, 2, 3).contiguous().view(S, hp * ep, D)


# ───────────────────────── token -> expert EP ─────────────────────────

class CudaBackend:
    """libmhmoe kernels for the device steps of the EP layer."""

    def quant_tokens(self, x_heads):
        S, H, dh = x_heads.shape
        dev = x_heads.device
        T = S * H
        xq = torch.empty(T, dh // 2, dtype=torch.uint8, device=dev)
        xsf = torch.empty(T, dh // 16, dtype=torch.uint8, device=dev)
        xg = torch.empty(T, dtype=torch.float32, device=dev)
        x = x_heads if (x_heads.stride(2) == 1 and x_heads.data_ptr() % 16 == 0) else x_heads.contiguous()
        _lib.check(_lib.lib().mhmoe_quant_tokens(x.data_ptr(), x.stride(0), x.stride(1), S, H, dh, xq.data_ptr(),
                                                  xsf.data_ptr(), xg.data_ptr(), _lib.stream_ptr(dev)),
                   "quant_tokens")
        return xq, xsf, xg

    def dest(self, idx, num_experts, n_ranks):
        H, S, K = idx.shape
        dev = idx.device
        d = torch.empty(H * S, n_ranks, dtype=torch.int64, device=dev)
        _lib.check(_lib.lib().mhmoe_ep_dest(idx.data_ptr(), H, S, K, num_experts, n_ranks, d.data_ptr(),
                                             _lib.device_status(dev).data_ptr(), _lib.stream_ptr(dev)), "ep_dest")
        return d

    def row_bytes(self, dh, K):
        return int(_lib.lib().mhmoe_ep_row_bytes(dh, K))

    def pack(self, xq, xsf, xg, H, S, idx, probs, num_experts, n_ranks, send_key, send_offsets, R_send):
        dev = xq.device
        dh = xq.shape[1] * 2
        K = idx.shape[-1]
        send = torch.empty(R_send, self.row_bytes(dh, K), dtype=torch.uint8, device=dev)
        _lib.check(_lib.lib().mhmoe_ep_pack(xq.data_ptr(), xsf.data_ptr(), xg.data_ptr(), H, S, dh, idx.data_ptr(),
                                             probs.data_ptr(), K, num_experts, n_ranks, send_key.data_ptr(),
                                             send_offsets.data_ptr(), R_send, send.data_ptr(), _lib.stream_ptr(dev)),
                   "ep_pack")
        return send

    def unpack(self, recv, dh, K, E_loc):
        R = recv.shape[0]
        dev = recv.device
        le = torch.empty(R, K, dtype=torch.int64, device=dev)
        pr = torch.empty(R, K, dtype=torch.float32, device=dev)
        if R:
            _lib.check(_lib.lib().mhmoe_ep_unpack(recv.data_ptr(), R, dh, K, E_loc, le.data_ptr(), pr.data_ptr(),
                                                   _lib.device_status(dev).data_ptr(), _lib.stream_ptr(dev)),
                       "ep_unpack")
        return le, pr

    def sort(self, probs, idx, num_experts):
        from .route import flash_mh_moe_global_sort_with_inverse
        return flash_mh_moe_global_sort_with_inverse(probs, idx, num_experts)

    def ffn_records(self, recv, dh, K, gather_ids, probs_sorted, expert_offsets, row_of_flat, gu, dn,
                    stage_events=None):
        """Per received record: bf16 sum (ascending expert) of its experts' prob-weighted outputs."""
        T = recv.shape[0]
        dev = recv.device
        y = torch.empty(T, dh, dtype=torch.bfloat16, device=dev)
        if T == 0:
            return y
        n = expert_offsets.numel() - 1
        R = gather_ids.numel()
        rb = recv.shape[1]
        L = _lib.lib()
        ws = torch.empty(max(1, L.mhmoe_ffn_workspace_bytes(R, T, 1, dh, gu.d_expert, n)), dtype=torch.uint8,
                         device=dev)
        base = recv.data_ptr()
        _lib.check(L.mhmoe_ffn_nvfp4_quantized(
            base, rb, base + dh // 2, rb, base + dh // 2 + dh // 16, rb, T, dh, gu.d_expert, n, R,
            gather_ids.data_ptr(), probs_sorted.data_ptr(), expert_offsets.data_ptr(), gu.data.data_ptr(),
            gu.sf.data_ptr(), gu.gscale.data_ptr(), dn.data.data_ptr(), dn.sf.data_ptr(), dn.gscale.data_ptr(),
            row_of_flat.data_ptr(), None, K, ws.data_ptr(), y.data_ptr(), y.stride(0),
            _lib.device_status(dev).data_ptr(), 0, _events(stage_events), _lib.stream_ptr(dev)),
            "ffn_nvfp4_quantized")
        return y

    def combine(self, rows, S, H, row_of_flat, K):
        dev = rows.device
        dh = rows.shape[1]
        y = torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
        _lib.check(_lib.lib().mhmoe_combine(rows.data_ptr() if rows.numel() else None, rows.shape[0], None, dh, S,
                                             H, row_of_flat.data_ptr(), None, K, rows.shape[0], y.data_ptr(),
                                             y.stride(0), y.stride(1), _lib.stream_ptr(dev)), "combine")
        return y


LAST_STATS: dict = {}   # records / rows moved by the last ep_moe_layer call on this process
COLLECT_STATS = False   # peer transport: also count chunk 0's remote records (extra small reductions)


def _a2a_rows(t: torch.Tensor, send_counts: list[int], recv_counts: list[int], group) -> torch.Tensor:
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t, output_split_sizes=recv_counts, input_split_sizes=send_counts, group=group)
    return out


def ep_exchange_counts(send_offsets: torch.Tensor, group) -> tuple[list[int], list[int]]:
    """Per-destination record counts of this rank and what every peer sends us.

    The only host synchronisation of the EP layer: the split sizes of the record
    all-to-alls must be known on the host."""
    send = (send_offsets[1:] - send_offsets[:-1]).to(torch.int64)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    both = torch.stack([send, recv]).cpu()
    return both[0].tolist(), both[1].tolist()


def ep_moe_layer(x_heads: torch.Tensor, probs: torch.Tensor, idx: torch.Tensor, num_experts: int, gu, dn, group,
                 backend=None, stage_events=None, comm_events=None) -> torch.Tensor:
    """Token -> expert EP forward of the routed FFN for this rank's tokens.

    x_heads [S, H, dh]; probs/idx [H, S, K] from this rank's router (per-head expert
    ids); gu/dn: this rank's NVFP4 expert slice (flattened experts
    [rank*E_loc, (rank+1)*E_loc)).  Returns y [S, H, dh] bf16.
    comm_events: optional 4 CUDA events recorded before/after the record all-to-all and
    before/after the return all-to-all (for link-bandwidth measurement).
    """
    be = backend or CudaBackend()
    ep = dist.get_world_size(group)
    S, H, dh = x_heads.shape
    K = idx.shape[-1]
    E = int(num_experts)
    HE = H * E
    if HE % ep:
        raise ValueError(f"H*E ({HE}) must be divisible by ep_size ({ep})")
    E_loc = HE // ep
    T = H * S
    # 1. one record per ((head, token), destination rank), grouped by destination
    xq, xsf, xg = be.quant_tokens(x_heads)
    dest = be.dest(idx, E, ep)                                           # [T, ep], key h*S + s
    zeros = torch.zeros(1, T, ep, dtype=torch.float32, device=dest.device)
    send_key, _, send_offs, send_slot = be.sort(zeros, dest.view(1, T, ep), ep)
    # 2./3. counts, then records
    send_counts, recv_counts = ep_exchange_counts(send_offs, group)
    R_send = int(sum(send_counts))
    send = be.pack(xq, xsf, xg, H, S, idx, probs, E, ep, send_key, send_offs, R_send)
    if comm_events:
        comm_events[0].record()
    recv = _a2a_rows(send, send_counts, recv_counts, group)
    if comm_events:
        comm_events[1].record()
    R_recv = recv.shape[0]
    me = dist.get_rank(group)
    remote_out = R_send - send_counts[me]
    remote_in = R_recv - recv_counts[me]
    LAST_STATS.update(records_sent=R_send, records_received=R_recv, bytes_sent=R_send * send.shape[1],
                      dispatch_remote_bytes=remote_out * send.shape[1],
                      return_remote_bytes=remote_in * dh * 2)
    # 4. local experts on the received records
    lidx, lprobs = be.unpack(recv, dh, K, E_loc)
    lg, lps, loffs, linv = be.sort(lprobs.view(1, R_recv, K), lidx.view(1, R_recv, K), E_loc)
    LAST_STATS.update(rows_received=loffs[-1], transport="nccl")   # device scalar: read it after the step
    out = be.ffn_records(recv, dh, K, lg, lps, loffs, linv, gu, dn, stage_events=stage_events)
    # 5. per-record partial sums back to their sources; combine in ascending rank order
    if comm_events:
        comm_events[2].record()
    back = _a2a_rows(out, recv_counts, send_counts, group)
    if comm_events:
        comm_events[3].record()
    return be.combine(back, S, H, send_slot, ep)


# ───────────────────────── token -> expert EP over peer memory ─────────────────────────

class PeerExchange:
    """Per-rank exchange buffer mapped on every rank of the group (CUDA IPC).

    Holds records from every source (``n * cap`` slots) and the returned sums of this
    rank's own records; the kernels store into peers' buffers over NVLink and raise
    arrival counters there, so a layer call needs no host synchronisation.  Requires
    every rank on its own GPU of one node (checked at creation)."""

    _cache: dict = {}

    def __init__(self, group, device: torch.device, cap: int, dh: int, K: int):
        import ctypes as C
        import socket
        L = _lib.lib()
        self.group, self.device, self.cap, self.dh, self.K = group, device, int(cap), int(dh), int(K)
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        ident = (socket.gethostname(), str(torch.cuda.get_device_properties(device).uuid), self.cap)
        idents = [None] * self.n
        dist.all_gather_object(idents, ident, group=group)
        if len({i[0] for i in idents}) != 1 or len({i[1] for i in idents}) != self.n:
            raise RuntimeError("peer-memory EP needs every rank on its own GPU of one node")
        if len({i[2] for i in idents}) != 1:
            # every rank must pass the same number of (head, token) rows, as the reference's
            # equal-split all-to-all (magi2_preview.py:3277-3299) requires; checked here, at
            # the collective, so that all ranks raise together
            raise ValueError(f"expert-parallel ranks passed different token counts {[i[2] for i in idents]}; "
                             "every rank of the EP group must pass the same S")
        size = int(L.mhmoe_ep_sym_bytes(self.n, self.cap, dh, K))
        ptr = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        with torch.cuda.device(device):
            _lib.check(L.mhmoe_ep_sym_alloc(size, C.byref(ptr), handle), "ep_sym_alloc")
        handles = [None] * self.n
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases, self._opened = [], []
        with torch.cuda.device(device):
            for r in range(self.n):
                if r == self.me:
                    bases.append(ptr.value)
                    continue
                p = C.c_void_p()
                buf = (C.c_ubyte * 64).from_buffer_copy(handles[r])
                _lib.check(L.mhmoe_ep_sym_open(buf, C.byref(p)), "ep_sym_open")
                bases.append(p.value)
                self._opened.append(p.value)
        self.local = ptr.value
        self.peer_bases = (C.c_void_p * self.n)(*bases)
        offs = (C.c_int64 * 5)()
        _lib.check(L.mhmoe_ep_sym_offsets(self.n, self.cap, dh, K, offs), "ep_sym_offsets")
        self.off_back = int(offs[3])
        self.epoch = 0
        self.push_done = [None, None]   # copy-engine transport: last push of records / returns
        dist.barrier(group=group)

    @classmethod
    def get(cls, group, device: torch.device, cap: int, dh: int, K: int, slot: int = 0) -> "PeerExchange":
        """The group's exchange on this device (one per pipeline slot), re-created when a
        larger capacity is needed.  Creation is collective and checks that every rank asks
        for the same ``cap`` (ranks passing different token counts raise together there);
        a later call passes without any collective when its ``cap`` fits, so every rank of
        the group must keep passing the same token count per call."""
        key = (id(group), device.index, int(dh), int(K), int(slot))
        px = cls._cache.get(key)
        if px is None or px.cap < cap:
            if px is not None:
                px.close()
            px = cls(group, device, cap, dh, K)
            cls._cache[key] = px
        return px

    def close(self) -> None:
        """Unmap the peers and free the buffer (collective: all ranks call it)."""
        L = _lib.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                L.mhmoe_ep_sym_close(p)
            self._opened = []
            dist.barrier(group=self.group)
            if self.local:
                L.mhmoe_ep_sym_free(self.local)
                self.local = None


def _ep_timeout_ns() -> int:
    import os
    return int(float(os.environ.get("MHMOE_EP_TIMEOUT_S", "10")) * 1e9)


def ep_moe_layer_peer(x_heads: torch.Tensor, probs: torch.Tensor, idx: torch.Tensor, num_experts: int, gu, dn,
                      group, stage_events=None, comm_events=None, slot: int = 0,
                      out: torch.Tensor | None = None, ffn_after=None, gemms_done=None) -> torch.Tensor:
    """Token -> expert EP forward with the exchange fused into the kernels (peer memory).

    Same records and result as ``ep_moe_layer``; the record kernel stores into the
    destinations' buffers and the receiver's combine stores each record's sum into the
    source's buffer, each followed by a device-side arrival flag, so there is no count
    exchange and no host synchronisation.  comm_events (optional, 4): around the record
    send + wait, and around the wait for the returns.  slot: which exchange buffer
    (pipeline chunk) to use; out: optional [S, H, dh] bf16 destination.  ffn_after: an event
    the expert GEMMs wait for (the previous chunk's GEMMs); gemms_done: an event recorded once
    this call's expert GEMMs are done (its returns still move); with stage_events, their
    fourth event marks that point instead.
    """
    be = CudaBackend()
    L = _lib.lib()
    ep = dist.get_world_size(group)
    S, H, dh = x_heads.shape
    K = idx.shape[-1]
    E = int(num_experts)
    HE = H * E
    if HE % ep:
        raise ValueError(f"H*E ({HE}) must be divisible by ep_size ({ep})")
    E_loc = HE // ep
    T = H * S
    dev = x_heads.device
    px = PeerExchange.get(group, dev, T, dh, K, slot)
    st = _lib.stream_ptr(dev)
    status = _lib.device_status(dev).data_ptr()
    timeout = _ep_timeout_ns()
    px.epoch += 1
    # 1. records, grouped by destination
    xq, xsf, xg = be.quant_tokens(x_heads)
    dest = be.dest(idx, E, ep)
    zeros = torch.zeros(1, T, ep, dtype=torch.float32, device=dev)
    send_key, _, send_offs, send_slot = be.sort(zeros, dest.view(1, T, ep), ep)
    if comm_events:
        comm_events[0].record()
    _lib.check(L.mhmoe_ep_send_records(xq.data_ptr(), xsf.data_ptr(), xg.data_ptr(), H, S, dh, idx.data_ptr(),
                                       probs.data_ptr(), K, E, send_key.data_ptr(), send_offs.data_ptr(), ep,
                                       px.me, px.cap, px.peer_bases, status, st), "ep_send_records")
    _lib.check(L.mhmoe_ep_wait(px.local, 0, ep, px.epoch, timeout, status, st), "ep_wait(records)")
    if comm_events:
        comm_events[1].record()
    # 2. receiver: every slot -> (local expert, prob) entries, sorted by expert
    slots = ep * px.cap
    lidx = torch.empty(slots, K, dtype=torch.int64, device=dev)
    lprobs = torch.empty(slots, K, dtype=torch.float32, device=dev)
    _lib.check(L.mhmoe_ep_unpack_slots(px.local, ep, px.cap, dh, K, E_loc, lidx.data_ptr(), lprobs.data_ptr(),
                                       status, st), "ep_unpack_slots")
    lg, lps, loffs, linv = be.sort(lprobs.view(1, slots, K), lidx.view(1, slots, K), E_loc)
    prev = LAST_STATS.get("rows_received") if slot > 0 else None
    LAST_STATS.update(rows_received=loffs[-1] if prev is None else prev + loffs[-1], transport="peer")
    if COLLECT_STATS and slot == 0:     # device scalars; read them after the step
        own = send_offs[px.me + 1] - send_offs[px.me]
        rb = be.row_bytes(dh, K)
        LAST_STATS.update(records_remote_bytes=(send_offs[-1] - own) * rb,
                          return_remote_bytes=((lidx[:, 0] >= 0).sum() - own) * (dh * 2))
    # 3. FFN on the records in place; its combine returns each record's sum to the source
    R = slots * K
    ws = torch.empty(max(1, L.mhmoe_ffn_workspace_bytes(R, slots, 1, dh, gu.d_expert, E_loc)), dtype=torch.uint8,
                     device=dev)
    if ffn_after is not None:
        torch.cuda.current_stream(dev).wait_event(ffn_after)
    evs = list(stage_events) if stage_events else None
    if gemms_done is not None and not evs:
        evs = [None, None, None, gemms_done, None]   # recorded after the down GEMM
    _lib.check(L.mhmoe_ep_ffn_return(px.local, ep, px.me, px.cap, dh, gu.d_expert, K, E_loc, R, lg.data_ptr(),
                                     lps.data_ptr(), loffs.data_ptr(), gu.data.data_ptr(), gu.sf.data_ptr(),
                                     gu.gscale.data_ptr(), dn.data.data_ptr(), dn.sf.data_ptr(),
                                     dn.gscale.data_ptr(), linv.data_ptr(), ws.data_ptr(), px.peer_bases, status, 0,
                                     _events(evs), st), "ep_ffn_return")
    if comm_events:
        comm_events[2].record()
    _lib.check(L.mhmoe_ep_wait(px.local, 1, ep, px.epoch, timeout, status, st), "ep_wait(returns)")
    if comm_events:
        comm_events[3].record()
    # 4. source: sum each (head, token)'s returned rows in ascending rank order
    y = out if out is not None else torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
    _lib.check(L.mhmoe_combine(px.local + px.off_back, slots, None, dh, S, H, send_slot.data_ptr(), None, ep, slots,
                               y.data_ptr(), y.stride(0), y.stride(1), st), "combine")
    return y


_side_streams: dict = {}


def ep_chunks(default: int = 1) -> int:
    """Pipeline depth of the EP layer (``MHMOE_EP_CHUNKS``; default 1 for the kernel-store
    transport, where two chunks measured slower at 2 GPUs, and 2 for the copy-engine one)."""
    import os
    return max(1, int(os.environ.get("MHMOE_EP_CHUNKS", str(default))))


def ep_moe_layer_peer_pipelined(x_heads: torch.Tensor, probs: torch.Tensor, idx: torch.Tensor, num_experts: int,
                                gu, dn, group, chunks: int = 2, stage_events=None,
                                comm_events=None) -> torch.Tensor:
    """The peer-memory EP layer over ``chunks`` token chunks, each on its own stream with its
    own exchange buffer.  Chunk c's expert GEMMs start after chunk c-1's (an event after its
    down GEMM), so the GEMMs do not compete for the SMs, while chunk c-1's returns and chunk
    c+1's records (link-bound) could move beside them.  Each token's result is
    computed exactly as unchunked (the same records, experts and summation order).  Events,
    if given, time chunk 0.
    """
    S, H, dh = x_heads.shape
    if chunks <= 1 or S < 2 * chunks:
        return ep_moe_layer_peer(x_heads, probs, idx, num_experts, gu, dn, group, stage_events, comm_events)
    dev = x_heads.device
    main = torch.cuda.current_stream(dev)
    streams = _side_streams.setdefault(dev.index, [])
    while len(streams) < chunks:
        streams.append(torch.cuda.Stream(device=dev))
    y = torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
    ready = torch.cuda.Event()
    ready.record(main)
    bounds = [(S * c) // chunks for c in range(chunks + 1)]
    done = []
    prev_gemms = None
    for c in range(chunks):
        a, b = bounds[c], bounds[c + 1]
        s = streams[c]
        s.wait_event(ready)
        ev_stage = stage_events if c == 0 else None
        gemms = None if ev_stage else torch.cuda.Event()
        with torch.cuda.stream(s):
            ep_moe_layer_peer(x_heads[a:b], probs[:, a:b].contiguous(), idx[:, a:b].contiguous(), num_experts, gu,
                              dn, group, ev_stage, comm_events if c == 0 else None, slot=c, out=y[a:b],
                              ffn_after=prev_gemms, gemms_done=gemms)
            ev = torch.cuda.Event()
            ev.record(s)
        prev_gemms = ev_stage[3] if ev_stage else gemms
        done.append(ev)
    for ev in done:
        main.wait_event(ev)
    return y


_copy_streams: dict = {}


def ep_moe_layer_copy(x_heads: torch.Tensor, probs: torch.Tensor, idx: torch.Tensor, num_experts: int, gu, dn,
                      group, chunks: int = 2, stage_events=None, comm_events=None) -> torch.Tensor:
    """Token -> expert EP forward whose NVLink transfers run on the copy engines.

    The same records, experts and summation order as ``ep_moe_layer_peer`` (so the same
    result), but the kernels only write this rank's own memory: each chunk's records are
    staged into per-destination slabs and moved with one ``cudaMemcpyAsync`` per peer on a
    copy stream (``mhmoe_ep_push``), and each chunk's per-record sums are staged per source and
    pushed back the same way.  The SMs stay on compute while the copy engines move data, so
    with ``chunks`` >= 2 chunk c+1's records and chunk c-1's returns cross the links during
    chunk c's expert GEMMs.  Whole cap-row slabs move (the counts stay on the device), so at
    n ranks a record slab carries ~(1 - (1 - 1/n)^K) rows in use per row moved.
    stage_events (7, optional) time chunk 0; comm_events (4): around chunk 0's record wait
    and return wait.
    """
    be = CudaBackend()
    L = _lib.lib()
    ep = dist.get_world_size(group)
    S, H, dh = x_heads.shape
    K = idx.shape[-1]
    E = int(num_experts)
    HE = H * E
    if HE % ep:
        raise ValueError(f"H*E ({HE}) must be divisible by ep_size ({ep})")
    E_loc = HE // ep
    dev = x_heads.device
    chunks = max(1, min(int(chunks), S))
    main = torch.cuda.current_stream(dev)
    if dev.index not in _copy_streams:
        _copy_streams[dev.index] = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
    rec_stream, ret_stream = _copy_streams[dev.index]
    st = _lib.stream_ptr(dev)
    status = _lib.device_status(dev).data_ptr()
    timeout = _ep_timeout_ns()
    y = torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
    bounds = [(S * c) // chunks for c in range(chunks + 1)]
    state = []
    # 1. every chunk's records: quantise, group by destination, stage, push on the copy stream
    for c in range(chunks):
        a, b = bounds[c], bounds[c + 1]
        T = H * (b - a)
        px = PeerExchange.get(group, dev, T, dh, K, 16 + c)
        px.epoch += 1
        if px.push_done[0] is not None:
            main.wait_event(px.push_done[0])          # the previous push has read the slabs
        idx_c, probs_c = idx[:, a:b].contiguous(), probs[:, a:b].contiguous()
        xq, xsf, xg = be.quant_tokens(x_heads[a:b])
        dest = be.dest(idx_c, E, ep)
        zeros = torch.zeros(1, T, ep, dtype=torch.float32, device=dev)
        send_key, _, send_offs, send_slot = be.sort(zeros, dest.view(1, T, ep), ep)
        _lib.check(L.mhmoe_ep_stage_records(xq.data_ptr(), xsf.data_ptr(), xg.data_ptr(), H, b - a, dh,
                                            idx_c.data_ptr(), probs_c.data_ptr(), K, E, send_key.data_ptr(),
                                            send_offs.data_ptr(), ep, px.me, px.cap, px.peer_bases, status, st),
                   "ep_stage_records")
        staged = torch.cuda.Event()
        staged.record(main)
        rec_stream.wait_event(staged)
        _lib.check(L.mhmoe_ep_push(px.local, 0, ep, px.me, px.cap, dh, K, px.peer_bases,
                                   rec_stream.cuda_stream), "ep_push(records)")
        px.push_done[0] = torch.cuda.Event()
        px.push_done[0].record(rec_stream)
        state.append((px, a, b, T, send_offs, send_slot))
    # 2. every chunk: wait for its records, expert FFN, stage the sums, push them back
    for c, (px, a, b, T, send_offs, send_slot) in enumerate(state):
        if comm_events and c == 0:
            comm_events[0].record()
        _lib.check(L.mhmoe_ep_wait(px.local, 0, ep, px.epoch, timeout, status, st), "ep_wait(records)")
        if comm_events and c == 0:
            comm_events[1].record()
        slots = ep * px.cap
        lidx = torch.empty(slots, K, dtype=torch.int64, device=dev)
        lprobs = torch.empty(slots, K, dtype=torch.float32, device=dev)
        _lib.check(L.mhmoe_ep_unpack_slots(px.local, ep, px.cap, dh, K, E_loc, lidx.data_ptr(), lprobs.data_ptr(),
                                           status, st), "ep_unpack_slots")
        lg, lps, loffs, linv = be.sort(lprobs.view(1, slots, K), lidx.view(1, slots, K), E_loc)
        R = slots * K
        ws = torch.empty(max(1, L.mhmoe_ffn_workspace_bytes(R, slots, 1, dh, gu.d_expert, E_loc)),
                         dtype=torch.uint8, device=dev)
        if px.push_done[1] is not None:
            main.wait_event(px.push_done[1])          # the previous push has read the stage area
        _lib.check(L.mhmoe_ep_ffn_stage(px.local, ep, px.me, px.cap, dh, gu.d_expert, K, E_loc, R, lg.data_ptr(),
                                        lps.data_ptr(), loffs.data_ptr(), gu.data.data_ptr(), gu.sf.data_ptr(),
                                        gu.gscale.data_ptr(), dn.data.data_ptr(), dn.sf.data_ptr(),
                                        dn.gscale.data_ptr(), linv.data_ptr(), ws.data_ptr(), px.peer_bases, status,
                                        0, _events(stage_events if c == 0 else None), st), "ep_ffn_stage")
        summed = torch.cuda.Event()
        summed.record(main)
        ret_stream.wait_event(summed)
        _lib.check(L.mhmoe_ep_push(px.local, 1, ep, px.me, px.cap, dh, K, px.peer_bases,
                                   ret_stream.cuda_stream), "ep_push(returns)")
        px.push_done[1] = torch.cuda.Event()
        px.push_done[1].record(ret_stream)
    LAST_STATS.update(transport="copy")
    # 3. every chunk: wait for the returns, sum each (head, token)'s rows in ascending rank order
    for c, (px, a, b, T, send_offs, send_slot) in enumerate(state):
        if comm_events and c == 0:
            comm_events[2].record()
        _lib.check(L.mhmoe_ep_wait(px.local, 1, ep, px.epoch, timeout, status, st), "ep_wait(returns)")
        if comm_events and c == 0:
            comm_events[3].record()
        # send row j of destination d landed at back row d*cap + (j - send_offsets[d])
        d = torch.arange(T * ep, device=dev) % ep
        j = send_slot.to(torch.int64)
        back_rows = torch.where(j >= 0, d * px.cap + j - send_offs[d], -1).to(torch.int32)
        _lib.check(L.mhmoe_combine(px.local + px.off_back, ep * px.cap, None, dh, b - a, H, back_rows.data_ptr(), None,
                                   ep, ep * px.cap, y[a:b].data_ptr(), y.stride(0), y.stride(1), st), "combine")
    return y


def ep_transport(module) -> str:
    """'peer' (kernels store over NVLink; the default), 'copy' (copy engines move staged
    slabs, ``MHMOE_EP_TRANSPORT=copy``) or 'nccl' (``MHMOE_EP_TRANSPORT=nccl``)."""
    import os
    want = getattr(module, "ep_transport", None) or os.environ.get("MHMOE_EP_TRANSPORT", "peer")
    return want if want in ("nccl", "copy") else "peer"


def ep_moe_forward(module, x_heads: torch.Tensor, stage_events=None, comm_events=None) -> torch.Tensor:
    """``CoreMultiHeadMoE`` forward with ``ep_size > 1`` (route locally, EP FFN)."""
    probs, idx = module._route(x_heads)
    gu, dn = module.packed_weights()
    if gu.d_head != x_heads.shape[-1]:
        raise NotImplementedError(f"expert parallelism takes d_head multiples of 256 (got {x_heads.shape[-1]}): "
                                  "its records carry the unpadded NVFP4 rows")
    if ep_transport(module) == "copy":
        return ep_moe_layer_copy(x_heads, probs, idx, module.num_experts, gu, dn, module.ep_group,
                                 chunks=ep_chunks(2), stage_events=stage_events, comm_events=comm_events)
    if ep_transport(module) == "peer":
        return ep_moe_layer_peer_pipelined(x_heads, probs, idx, module.num_experts, gu, dn, module.ep_group,
                                           chunks=ep_chunks(), stage_events=stage_events, comm_events=comm_events)
    return ep_moe_layer(x_heads, probs, idx, module.num_experts, gu, dn, module.ep_group,
                        stage_events=stage_events, comm_events=comm_events)
