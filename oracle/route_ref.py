"""numpy restatement of the reference router and global sort — test infrastructure.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this module; the product path is the CUDA router/permute kernels.

Pinned against golden vectors produced by the reference's own ``route.py``
(``tests/golden/make_golden.py`` imports it and records its outputs).

Reference lines restated:
* ``inference/flash_mh_moe/route.py:28-148``  ``_compute_topk_probs_and_indices_torch_impl``
* ``inference/flash_mh_moe/route.py:209-253`` ``flash_mh_moe_global_sort``
* ``inference/model/magi2_preview.py:2588-2601`` ``CoreMultiHeadMoE._route``
"""
from __future__ import annotations

import numpy as np


def scores_from_logits(logits: np.ndarray, score_func: str) -> np.ndarray:
    """route.py:44-50 — softmax or sigmoid over the expert axis, fp32."""
    x = np.asarray(logits, dtype=np.float32)
    if score_func == "softmax":
        m = x.max(axis=-1, keepdims=True)
        e = np.exp((x - m).astype(np.float32)).astype(np.float32)
        return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    if score_func == "sigmoid":
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x).astype(np.float32))).astype(np.float32)
    raise ValueError(f"Unknown score_func: {score_func}")


def _topk_desc(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest along the last axis, descending; ties -> lower index first."""
    order = np.argsort(-v, axis=-1, kind="stable")
    return order[..., :k]


def compute_topk_probs_and_indices(
    router_logits: np.ndarray,
    top_k: int,
    score_func: str = "softmax",
    expert_bias: np.ndarray | None = None,
    num_virtual_group: int = 1,
    topk_virtual_group: int = 0,
    route_norm: bool = True,
    norm_eps: float = 1e-12,
) -> tuple[np.ndarray, np.ndarray]:
    """route.py:157-199 (-> :28-148).  Returns probs fp32 [H,S,K], idx int64 [H,S,K]."""
    H, S, E = router_logits.shape
    K = top_k
    scores = scores_from_logits(router_logits, score_func)
    sel = scores
    if expert_bias is not None:                                     # route.py:54-57
        sel = (sel + np.asarray(expert_bias, np.float32).reshape(H, 1, E)).astype(np.float32)
    if num_virtual_group > 1:                                       # route.py:61-104
        assert 0 < topk_virtual_group <= num_virtual_group
        assert E % num_virtual_group == 0
        epg = E // num_virtual_group
        grp = sel.reshape(H, S, num_virtual_group, epg)
        top2 = -np.sort(-grp, axis=-1)[..., : min(2, epg)]
        gscore = top2.sum(axis=-1, dtype=np.float32)
        gidx = _topk_desc(gscore, topk_virtual_group)
        gmask = np.zeros_like(gscore, dtype=bool)
        np.put_along_axis(gmask, gidx, True, axis=-1)
        emask = np.repeat(gmask, epg, axis=-1)
        sel = np.where(emask, sel, np.float32(0.0)).astype(np.float32)
    idx = _topk_desc(sel, K)                                        # route.py:106
    probs = np.take_along_axis(scores, idx, axis=-1)                # route.py:136
    if route_norm:                                                  # route.py:139-142 (F.normalize p=1)
        denom = np.maximum(np.abs(probs).sum(axis=-1, keepdims=True, dtype=np.float32),
                           np.float32(norm_eps))
        probs = (probs / denom).astype(np.float32)
    return probs.astype(np.float32), idx.astype(np.int64)


def flash_mh_moe_global_sort(topk_probs: np.ndarray, topk_indices: np.ndarray, num_experts: int):
    """route.py:209-253.  Stable sort of flat (h,s,k) entries by global expert h*E+e.

    Returns gather_ids int32 [R], probs_sorted fp32 [R], expert_offsets int64 [H*E+1].
    """
    H, S, K = topk_indices.shape
    E = num_experts
    gidx = (topk_indices + np.arange(H).reshape(H, 1, 1) * E).reshape(-1)
    tok = np.broadcast_to(np.arange(S).reshape(1, S, 1), (H, S, K)).reshape(-1)
    order = np.argsort(gidx, kind="stable")
    gather_ids = tok[order].astype(np.int32)
    probs_sorted = topk_probs.reshape(-1)[order].astype(np.float32)
    counts = np.bincount(gidx, minlength=H * E).astype(np.int64)
    offsets = np.zeros(H * E + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    return gather_ids, probs_sorted, offsets


def router_logits(x_heads: np.ndarray, gate: np.ndarray, num_experts: int) -> np.ndarray:
    """magi2_preview.py:2590-2591 — einsum("shd,hed->hse") in fp32 (accumulated in fp64 here)."""
    S, H, dh = x_heads.shape
    g = np.asarray(gate, np.float64).reshape(H, num_experts, dh)
    x = np.asarray(x_heads, np.float64)
    return np.einsum("shd,hed->hse", x, g).astype(np.float32)
