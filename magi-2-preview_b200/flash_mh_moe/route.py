"""Routing and sorting — same call signatures as the reference's ``inference/flash_mh_moe/route.py``.

Both functions run on the B200 through libmhmoe; neither has a CPU path.

* ``compute_topk_probs_and_indices``  (reference ``route.py:157-199``)
* ``flash_mh_moe_global_sort``        (reference ``route.py:209-253``)
* ``router_logits``                   the fp32 einsum of ``CoreMultiHeadMoE._route``
  (``inference/model/magi2_preview.py:2588-2591``)
"""
from __future__ import annotations

from typing import Literal, TypeAlias

import torch

from . import _lib

TopKScoreFunc: TypeAlias = Literal["softmax", "sigmoid"]

score_func_name2id_map = {"softmax": 0, "sigmoid": 1}


def compute_topk_probs_and_indices(
    router_logits: torch.Tensor,
    top_k: int,
    score_func: TopKScoreFunc = "softmax",
    expert_bias: torch.Tensor | None = None,
    num_virtual_group: int = 1,
    topk_virtual_group: int = 0,
    route_norm: bool = True,
    norm_eps: float = 1e-12,
    route_scale: float = 1.0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k probabilities and indices from router logits [H, S, E].

    Returns (topk_probs fp32 [H, S, K], topk_indices int64 [H, S, K]); indices are
    sorted by descending (bias-adjusted) score, ties to the lower expert id.  With
    ``num_virtual_group > 1`` the reference returns the selected set unsorted; this
    returns the same set sorted.  ``route_scale`` (default 1.0, i.e. the reference
    contract) folds in ``CoreMultiHeadMoE._route``'s ``topk_probs * route_scale``.
    """
    if score_func not in score_func_name2id_map:
        raise ValueError(f"Unknown score_func: {score_func}")
    _lib.require_cuda(router_logits)
    H, S, E = router_logits.shape
    K = int(top_k)
    if num_virtual_group > 1:
        assert 0 < topk_virtual_group <= num_virtual_group, (
            f"topk_virtual_group ({topk_virtual_group}) must be in (0, num_virtual_group ({num_virtual_group})]")
        assert E % num_virtual_group == 0, (
            f"num_experts ({E}) must be divisible by num_virtual_group ({num_virtual_group})")
    logits = router_logits.float().contiguous()
    bias = None
    if expert_bias is not None:
        bias = expert_bias.reshape(H, E).float().contiguous()
    dev = logits.device
    probs = torch.empty(H, S, K, dtype=torch.float32, device=dev)
    idx = torch.empty(H, S, K, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mhmoe_topk(
            logits.data_ptr(), _lib.ptr(bias), H, S, E, K, score_func_name2id_map[score_func],
            int(num_virtual_group), int(topk_virtual_group), int(bool(route_norm)), float(norm_eps),
            float(route_scale), probs.data_ptr(), idx.data_ptr(), _lib.stream_ptr(dev)),
            "compute_topk_probs_and_indices")
    return probs, idx


def _global_sort(topk_probs, topk_indices, num_experts, want_row_of_flat):
    _lib.require_cuda(topk_probs, topk_indices)
    H, S, K = topk_indices.shape
    E = int(num_experts)
    dev = topk_indices.device
    idx = topk_indices.to(torch.int64).contiguous()
    probs = topk_probs.float().contiguous()
    R = H * S * K
    gather_ids = torch.empty(R, dtype=torch.int32, device=dev)
    probs_sorted = torch.empty(R, dtype=torch.float32, device=dev)
    offsets = torch.empty(H * E + 1, dtype=torch.int64, device=dev)
    row_of_flat = torch.empty(R, dtype=torch.int32, device=dev) if want_row_of_flat else None
    L = _lib.lib()
    ws = torch.empty(L.mhmoe_global_sort_workspace_bytes(H, S, K, E), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.mhmoe_global_sort(probs.data_ptr(), idx.data_ptr(), H, S, K, E, ws.data_ptr(),
                                       gather_ids.data_ptr(), probs_sorted.data_ptr(), offsets.data_ptr(),
                                       _lib.ptr(row_of_flat), _lib.device_status(dev).data_ptr(),
                                       _lib.stream_ptr(dev)), "flash_mh_moe_global_sort")
    return gather_ids, probs_sorted, offsets, row_of_flat


def flash_mh_moe_global_sort(
    topk_probs: torch.Tensor,
    topk_indices: torch.Tensor,
    num_experts: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Map per-head expert ids to global [0, H*E) and sort stably into CSR form.

    Returns gather_ids int32 [T], probs_sorted fp32 [T], expert_offsets int64 [H*E+1],
    bit-identical to the reference's ``argsort(stable=True)`` construction.
    """
    g, p, o, _ = _global_sort(topk_probs, topk_indices, num_experts, False)
    return g, p, o


def flash_mh_moe_global_sort_with_inverse(topk_probs, topk_indices, num_experts):
    """``flash_mh_moe_global_sort`` plus ``row_of_flat`` int32 [H*S*K]: the sorted
    position of each flat (h, s, k) entry (the combine uses it as token -> rows map)."""
    return _global_sort(topk_probs, topk_indices, num_experts, True)


def router_logits(x_heads: torch.Tensor, gate: torch.Tensor, num_experts: int) -> torch.Tensor:
    """fp32 router logits [H, S, E] for x_heads [S, H, dh] (bf16) and gate [H*E, dh]."""
    _lib.require_cuda(x_heads, gate)
    S, H, dh = x_heads.shape
    x = x_heads if x_heads.dtype == torch.bfloat16 else x_heads.to(torch.bfloat16)
    if x.stride(2) != 1:
        x = x.contiguous()
    g = gate.float().contiguous()
    dev = x.device
    out = torch.empty(H, S, num_experts, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mhmoe_router_logits(x.data_ptr(), x.stride(0), x.stride(1), g.data_ptr(), S, H, dh,
                                                   int(num_experts), out.data_ptr(), _lib.stream_ptr(dev)),
                   "router_logits")
    return out


# ───────────────────────── fused tensor-core router ─────────────────────────

def router_prepare(gate: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Split the fp32 router weight [H*E, dh] into the fewest exact bf16 planes (1..3)
    the fused router needs (load-time work; reads back three flags)."""
    _lib.require_cuda(gate)
    g = gate.detach().float().contiguous()
    n, dh = g.shape
    dev = g.device
    L = _lib.lib()
    flags = torch.zeros(3, dtype=torch.int32, device=dev)
    full = torch.empty(n, 3 * dh, dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.mhmoe_router_prepare(g.data_ptr(), n, dh, 3, full.data_ptr(), flags.data_ptr(),
                                           _lib.stream_ptr(dev)), "router_prepare")
        f = flags.tolist()
        nsplit = 3 if f[2] else (2 if f[1] else 1)
        if nsplit == 3:
            return full, 3
        planes = torch.empty(n, nsplit * dh, dtype=torch.bfloat16, device=dev)
        _lib.check(L.mhmoe_router_prepare(g.data_ptr(), n, dh, nsplit, planes.data_ptr(), None,
                                           _lib.stream_ptr(dev)), "router_prepare")
    return planes, nsplit


def fused_router_supported(E: int, K: int, dh: int) -> bool:
    return E <= 256 and K <= 16 and dh % 64 == 0


def route_fused(x_heads: torch.Tensor, planes: torch.Tensor, nsplit: int, num_experts: int, top_k: int,
                score_func: str = "softmax", expert_bias: torch.Tensor | None = None, route_norm: bool = True,
                norm_eps: float = 1e-12, route_scale: float = 1.0, return_logits: bool = False,
                logit_bias: torch.Tensor | None = None):
    """Router logits + top-k in one tcgen05 kernel (``CoreMultiHeadMoE._route``).

    x_heads [S, H, dh] bf16 (heads contiguous).  Returns (probs fp32 [H,S,K], idx int64
    [H,S,K]) and, with ``return_logits``, the fp32 logits [H,S,E] as a third item.
    ``logit_bias`` [H*E] (optional) is added to the logits before scoring.
    """
    if score_func not in score_func_name2id_map:
        raise ValueError(f"Unknown score_func: {score_func}")
    _lib.require_cuda(x_heads, planes)
    S, H, dh = x_heads.shape
    E, K = int(num_experts), int(top_k)
    x = x_heads if x_heads.dtype == torch.bfloat16 else x_heads.to(torch.bfloat16)
    if x.stride(2) != 1 or x.stride(1) != dh or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    dev = x.device
    probs = torch.empty(H, S, K, dtype=torch.float32, device=dev)
    idx = torch.empty(H, S, K, dtype=torch.int64, device=dev)
    logits = torch.empty(H, S, E, dtype=torch.float32, device=dev) if return_logits else None
    bias = None if expert_bias is None else expert_bias.reshape(-1).float().contiguous()
    lbias = None if logit_bias is None else logit_bias.reshape(-1).float().contiguous()
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mhmoe_route(
            x.data_ptr(), x.stride(0), x.stride(1), planes.data_ptr(), int(nsplit), S, H, dh, E, K,
            score_func_name2id_map[score_func], _lib.ptr(lbias), _lib.ptr(bias), int(bool(route_norm)),
            float(norm_eps),
            float(route_scale), probs.data_ptr(), idx.data_ptr(), _lib.ptr(logits),
            _lib.device_status(dev).data_ptr(), _lib.stream_ptr(dev)), "route")
    return (probs, idx, logits) if return_logits else (probs, idx)
