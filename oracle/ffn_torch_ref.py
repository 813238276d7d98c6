"""The reference layer's CPU path in torch, for the timed CPU baseline.

Test and measurement infrastructure only (``bench.py``'s CPU-baseline leg and its
``--impl reference`` arm; checked against ``oracle.ffn_ref`` in ``tests/test_oracle.py``).

The reference has no CPU implementation of its expert FFN: ``_mh_moe_fwd_kernel`` is
Triton (``inference/flash_mh_moe/triton/mh_moe_fwd.py:50-181``).  Its routing and sort
(``inference/flash_mh_moe/route.py``) and its deterministic scatter (``_scatter_back``,
``mh_moe_fwd.py:189-215``) are plain torch and run on the CPU unchanged; when the
reference package is staged under ``oracle/_ref`` those functions are its own code.
The FFN between them is restated here with the kernel's numerics, per expert:

* operands are bf16 values; products accumulate in fp32 (``tl.dot`` with
  ``ACC_DTYPE=tl.float32``, ``:145-146``): computed as fp32 GEMMs of the bf16 values,
  which are exact products with fp32 accumulation;
* ``hidden = swiglu7(gate_acc, up_acc).to(W_down.dtype)`` (``:148``, ``:24-30``);
* ``y_acc = hidden @ W_down`` in fp32, ``y_acc * probs`` in fp32, cast to bf16
  (``:157-171``), then the sequential bf16 ``scatter_add_`` of ``_scatter_back``.

Everything runs on torch's CPU kernels with all the host threads torch is given.
"""
from __future__ import annotations

import torch

SWIGLU7_ALPHA = 1.702   # mh_moe_fwd.py:18-20
SWIGLU7_LIMIT = 7.0
SWIGLU7_BIAS = 1.0


def swiglu7(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """mh_moe_fwd.py:24-30 in fp32."""
    g = torch.clamp(gate, max=SWIGLU7_LIMIT)
    u = torch.clamp(up, min=-SWIGLU7_LIMIT, max=SWIGLU7_LIMIT)
    return g * torch.sigmoid(SWIGLU7_ALPHA * g) * (u + SWIGLU7_BIAS)


def expert_rows(x: torch.Tensor, gather_ids: torch.Tensor, probs: torch.Tensor, expert_offsets: torch.Tensor,
                W_gate: torch.Tensor, W_up: torch.Tensor, W_down: torch.Tensor) -> torch.Tensor:
    """Per sorted row: bf16(y_acc * prob), the values the reference kernel stores in its
    flat [T, 1, dh] buffer (deterministic mode).  x [S, H, dh] bf16; weights bf16."""
    S, H, dh = x.shape
    T = gather_ids.numel()
    nflat = expert_offsets.numel() - 1
    e_per_h = nflat // H
    out = torch.empty(T, dh, dtype=torch.bfloat16)
    offs = expert_offsets.tolist()
    tok = gather_ids.long()
    for e in range(nflat):
        lo, hi = offs[e], offs[e + 1]
        if hi == lo:
            continue
        h = e // e_per_h
        xe = x[tok[lo:hi], h, :].float()
        gate_acc = xe @ W_gate[e].float()
        up_acc = xe @ W_up[e].float()
        hidden = swiglu7(gate_acc, up_acc).to(W_down.dtype)
        y_acc = hidden.float() @ W_down[e].float()
        out[lo:hi] = (y_acc * probs[lo:hi, None].float()).to(torch.bfloat16)
    return out


def scatter_back(y_sorted: torch.Tensor, x: torch.Tensor, gather_ids: torch.Tensor, expert_offsets: torch.Tensor,
                 num_heads: int) -> torch.Tensor:
    """The deterministic scatter (mh_moe_fwd.py:189-215): sequential bf16 scatter_add_ of
    each row into y[token, head]."""
    S, H, dh = x.shape
    nflat = expert_offsets.numel() - 1
    y = torch.zeros(S * H, dh, dtype=x.dtype)
    head_ids = torch.repeat_interleave(torch.arange(nflat) // (nflat // num_heads), expert_offsets.diff())
    idx = gather_ids.long() * num_heads + head_ids if num_heads > 1 else gather_ids.long()
    y.scatter_add_(0, idx.unsqueeze(-1).expand_as(y_sorted), y_sorted.to(y.dtype))
    return y.view(S, H, dh)


def moe_layer_cpu(x: torch.Tensor, gate: torch.Tensor, W_gate: torch.Tensor, W_up: torch.Tensor,
                  W_down: torch.Tensor, num_experts: int, top_k: int, score_func: str = "softmax",
                  route_scale: float = 1.0, expert_bias: torch.Tensor | None = None, ref=None) -> torch.Tensor:
    """The reference layer path on the CPU (CoreMultiHeadMoE._route + _flash_forward in
    deterministic mode, magi2_preview.py:2588-2613): fp32 einsum router, top-k, global
    sort, expert FFN, scatter.  ``ref``: the staged reference package (its route.py and
    _scatter_back are used verbatim); without it the oracle's restatements stand in.
    x [S, H, dh] bf16."""
    S, H, dh = x.shape
    g = gate.view(H, num_experts, dh).float()
    logits = torch.einsum("shd,hed->hse", x.float(), g)
    bias = expert_bias.view(H, num_experts) if expert_bias is not None else None
    if ref is not None:
        probs, idx = ref.compute_topk_probs_and_indices(logits, top_k, score_func=score_func, expert_bias=bias)
        probs = probs * route_scale
        gids, ps, offs = ref.flash_mh_moe_global_sort(probs, idx, num_experts)
        rows = expert_rows(x, gids, ps, offs, W_gate, W_up, W_down)
        from ref_flash_mh_moe.triton.mh_moe_fwd import _scatter_back
        return _scatter_back(rows, x, gids, offs, H * num_experts, H)
    import numpy as np

    from . import route_ref
    p, i = route_ref.compute_topk_probs_and_indices(logits.numpy(), top_k, score_func,
                                                    None if bias is None else bias.numpy())
    p = (p * np.float32(route_scale)).astype(np.float32)
    gi, pi, oi = route_ref.flash_mh_moe_global_sort(p, i, num_experts)
    gids, ps, offs = torch.from_numpy(gi), torch.from_numpy(pi), torch.from_numpy(oi)
    rows = expert_rows(x, gids, ps, offs, W_gate, W_up, W_down)
    return scatter_back(rows, x, gids, offs, H)
