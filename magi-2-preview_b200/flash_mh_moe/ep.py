"""Expert parallelism for the MoE layer: token -> expert dispatch/combine over the EP group.

The reference (``inference/model/magi2_preview.py:3277-3327``) shards *heads* across the EP
group and swaps the whole activation with one ``all_to_all_single`` each way; with H=12
heads padded to 16 on 8 ranks, two ranks hold only zero "dummy" heads
(``magi2_preview.py:2514-2537``).  Here the flattened experts ``[0, H*E)`` are split into
``ep`` contiguous ranges (the same dim-0 row slices the reference's EP checkpoint loader
reads when ``H % ep == 0``) and only routed rows move, in NVFP4:

  1. route + stable sort the rank's own tokens (rows come out grouped by destination rank,
     because expert ranges are contiguous);
  2. quantise each token once, pack one NVFP4 row (+ 16-byte meta: row scale, local expert,
     prob) per sorted row;
  3. exchange counts (``all_to_all_single`` of n ints, read on the host), then the rows;
  4. receiver: sort received rows by local expert, run the NVFP4 FFN on them, keep one
     bf16 output row per received row (prob already applied);
  5. send the output rows back; the source combines each (token, head)'s K rows in
     ascending global-expert order — the same order as the single-GPU layer, so the EP
     output equals the single-device output bit for bit.

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

    def pack(self, xq, xsf, xg, H, E, E_loc, gather_ids, probs_sorted, expert_offsets):
        R = gather_ids.numel()
        dev = xq.device
        dh = xq.shape[1] * 2
        sxq = torch.empty(R, dh // 2, dtype=torch.uint8, device=dev)
        sxsf = torch.empty(R, dh // 16, dtype=torch.uint8, device=dev)
        meta = torch.empty(R, 4, dtype=torch.float32, device=dev)
        _lib.check(_lib.lib().mhmoe_ep_pack(xq.data_ptr(), xsf.data_ptr(), xg.data_ptr(), xq.shape[0], dh, H, E,
                                             E_loc, R, gather_ids.data_ptr(), probs_sorted.data_ptr(),
                                             expert_offsets.data_ptr(), sxq.data_ptr(), sxsf.data_ptr(),
                                             meta.data_ptr(), _lib.device_status(dev).data_ptr(),
                                             _lib.stream_ptr(dev)), "ep_pack")
        return sxq, sxsf, meta

    def unpack(self, meta, E_loc):
        R = meta.shape[0]
        dev = meta.device
        g = torch.empty(R, dtype=torch.float32, device=dev)
        le = torch.empty(R, dtype=torch.int64, device=dev)
        pr = torch.empty(R, dtype=torch.float32, device=dev)
        _lib.check(_lib.lib().mhmoe_ep_unpack(meta.data_ptr(), R, E_loc, g.data_ptr(), le.data_ptr(), pr.data_ptr(),
                                               _lib.device_status(dev).data_ptr(), _lib.stream_ptr(dev)),
                   "ep_unpack")
        return g, le, pr

    def sort(self, probs, idx, num_experts):
        from .route import flash_mh_moe_global_sort_with_inverse
        return flash_mh_moe_global_sort_with_inverse(probs, idx, num_experts)

    def ffn_rows(self, xq, xsf, xg, gather_ids, probs_sorted, expert_offsets, row_of_flat, gu, dn,
                 stage_events=None):
        """One bf16 output row per quantised input row (prob applied), in input-row order."""
        T = xq.shape[0]
        dh = xq.shape[1] * 2
        dev = xq.device
        y = torch.empty(T, dh, dtype=torch.bfloat16, device=dev)
        n = expert_offsets.numel() - 1
        R = gather_ids.numel()
        L = _lib.lib()
        ws = torch.empty(max(1, L.mhmoe_ffn_workspace_bytes(R, T, 1, dh, gu.d_expert, n)), dtype=torch.uint8,
                         device=dev)
        _lib.check(L.mhmoe_ffn_nvfp4_quantized(
            xq.data_ptr(), xsf.data_ptr(), xg.data_ptr(), T, dh, gu.d_expert, n, R, gather_ids.data_ptr(),
            probs_sorted.data_ptr(), expert_offsets.data_ptr(), gu.data.data_ptr(), gu.sf.data_ptr(),
            gu.gscale.data_ptr(), dn.data.data_ptr(), dn.sf.data_ptr(), dn.gscale.data_ptr(), row_of_flat.data_ptr(),
            None, 1, ws.data_ptr(), y.data_ptr(), y.stride(0), _lib.device_status(dev).data_ptr(), 0,
            _events(stage_events), _lib.stream_ptr(dev)), "ffn_nvfp4_quantized")
        return y

    def combine(self, rows, S, H, row_of_flat, K):
        dev = rows.device
        dh = rows.shape[1]
        y = torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
        _lib.check(_lib.lib().mhmoe_combine(rows.data_ptr() if rows.numel() else None, rows.shape[0], None, dh, S,
                                             H, row_of_flat.data_ptr(), None, K, rows.shape[0], y.data_ptr(),
                                             y.stride(0), y.stride(1), _lib.stream_ptr(dev)), "combine")
        return y


LAST_STATS: dict = {}   # rows sent / received by the last ep_moe_layer call on this process


def _a2a_rows(t: torch.Tensor, send_counts: list[int], recv_counts: list[int], group) -> torch.Tensor:
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t, output_split_sizes=recv_counts, input_split_sizes=send_counts, group=group)
    return out


def ep_exchange_counts(expert_offsets: torch.Tensor, ep: int, E_loc: int, group) -> tuple[list[int], list[int]]:
    """Per-destination row counts of this rank's sorted rows, and what every peer sends us.

    The only host synchronisation of the EP layer: the split sizes of the row
    all-to-alls must be known on the host."""
    bounds = expert_offsets[torch.arange(0, ep + 1, device=expert_offsets.device) * E_loc]
    send = (bounds[1:] - bounds[:-1]).to(torch.int64)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    both = torch.stack([send, recv]).cpu()
    return both[0].tolist(), both[1].tolist()


def ep_moe_layer(x_heads: torch.Tensor, probs: torch.Tensor, idx: torch.Tensor, num_experts: int, gu, dn, group,
                 backend=None, stage_events=None) -> torch.Tensor:
    """Token -> expert EP forward of the routed FFN for this rank's tokens.

    x_heads [S, H, dh]; probs/idx [H, S, K] from this rank's router (global per-head
    expert ids); gu/dn: this rank's NVFP4 expert slice (flattened experts
    [rank*E_loc, (rank+1)*E_loc)).  Returns y [S, H, dh] bf16.
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
    # 1. stable sort of the local routed rows by global expert (grouped by destination rank)
    gids, ps, offs, inv = be.sort(probs, idx, E)
    # 2. NVFP4 rows + meta, in sorted order
    xq, xsf, xg = be.quant_tokens(x_heads)
    sxq, sxsf, meta = be.pack(xq, xsf, xg, H, E, E_loc, gids, ps, offs)
    # 3. counts, then rows
    send_counts, recv_counts = ep_exchange_counts(offs, ep, E_loc, group)
    rxq = _a2a_rows(sxq, send_counts, recv_counts, group)
    rxsf = _a2a_rows(sxsf, send_counts, recv_counts, group)
    rmeta = _a2a_rows(meta, send_counts, recv_counts, group)
    # 4. local experts on the received rows (one output row per received row)
    Rr = rxq.shape[0]
    LAST_STATS.update(rows_sent=int(sum(send_counts)), rows_received=int(Rr),
                      bytes_sent=int(sum(send_counts)) * (sxq.shape[1] + sxsf.shape[1] + 16))
    rg, rexp, rprob = be.unpack(rmeta, E_loc)
    lg, lps, loffs, linv = be.sort(rprob.view(1, Rr, 1), rexp.view(1, Rr, 1), E_loc)
    if stage_events is not None:
        out_rows = be.ffn_rows(rxq, rxsf, rg, lg, lps, loffs, linv, gu, dn, stage_events=stage_events)
    else:
        out_rows = be.ffn_rows(rxq, rxsf, rg, lg, lps, loffs, linv, gu, dn)
    # 5. rows back to their sources; combine in ascending global-expert order
    back = _a2a_rows(out_rows, recv_counts, send_counts, group)
    return be.combine(back, S, H, inv, K)


def ep_moe_forward(module, x_heads: torch.Tensor, stage_events=None) -> torch.Tensor:
    """``CoreMultiHeadMoE`` forward with ``ep_size > 1`` (route locally, EP FFN)."""
    probs, idx = module._route(x_heads)
    gu, dn = module.packed_weights()
    return ep_moe_layer(x_heads, probs, idx, module.num_experts, gu, dn, module.ep_group,
                        stage_events=stage_events)
