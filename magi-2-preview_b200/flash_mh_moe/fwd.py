"""Expert FFN forward — same call signature as the reference's ``inference/flash_mh_moe/fwd.py``.

``flash_mh_moe_fwd(x, gather_ids, probs, expert_offsets, W_gate, W_up, W_down)``
(reference ``fwd.py:16-40`` -> ``triton/mh_moe_fwd.py:231-331``): gather ->
gate/up GEMM -> SwiGLU7 -> down GEMM -> weighted scatter, here as the NVFP4 B200 path:

    per-row NVFP4 quantise of the gathered x  ->  tcgen05 block-scaled grouped GEMM
    (gate|up) with SwiGLU7 and NVFP4 re-quantise fused in its epilogue  ->  grouped
    GEMM (down) x prob  ->  scatter into y.

Weights may be the reference's bf16 parameters (packed to NVFP4 on first use and
cached per parameter version) or already-packed ``NVFP4GateUp`` / ``NVFP4Down``.
Scatter: by default partial rows are written and a combine pass sums each token's rows
in fp32 in sorted-row order (run-to-run identical, one bf16 rounding) — the reference's
``MAGI2_DETERMINISTIC=1`` behaviour (``fwd.py:12-13``), and on B200 also the faster one.
``MHMOE_SCATTER=atomic`` (or ``deterministic=False``) selects the reference's default
scatter instead: the down GEMM adds its bf16 rows into y with bf16 atomics (bf16
accumulation in arrival order, not run-to-run reproducible); measured slower here, as
the 16-B vector atomics saturate L2.
"""
from __future__ import annotations

import os
import weakref

import torch

from . import _lib
from .nvfp4 import NVFP4Down, NVFP4GateUp, pack_down, pack_gate_up


def _is_deterministic() -> bool:
    """Combine scatter unless MHMOE_SCATTER=atomic (the combine also satisfies the
    reference's MAGI2_DETERMINISTIC=1)."""
    return os.environ.get("MHMOE_SCATTER", "combine") != "atomic"


# Packed operands, one entry per set of source tensors, keyed by their (address, shape,
# dtype, device) and holding the versions they were packed at: an in-place update repacks
# into the same entry (no stale copies pile up).  An entry lives only as long as every
# source tensor object it was packed from: a weakref callback evicts it when one dies, so a
# new tensor later allocated at the same address can never pick up another tensor's
# packed weights.
_pack_cache: dict[tuple, tuple] = {}


def _key(t: torch.Tensor) -> tuple:
    return (t.data_ptr(), tuple(t.shape), t.dtype, t.device)


def _cached_pack(tag: str, srcs: tuple, pack):
    k = (tag,) + tuple(x for t in srcs for x in _key(t))
    versions = tuple(t._version for t in srcs)
    hit = _pack_cache.get(k)
    if hit is not None and hit[0] == versions:
        return hit[1]
    packed = pack(*srcs)
    if hit is None:
        for t in srcs:
            weakref.finalize(t, _pack_cache.pop, k, None)
    _pack_cache[k] = (versions, packed)
    return packed


def packed_weights(W_gate, W_up, W_down) -> tuple[NVFP4GateUp, NVFP4Down]:
    """Return NVFP4 operands for the given weights, packing (and caching) bf16 ones."""
    gu = W_gate if isinstance(W_gate, NVFP4GateUp) else _cached_pack("gu", (W_gate, W_up), pack_gate_up)
    dn = W_down if isinstance(W_down, NVFP4Down) else _cached_pack("dn", (W_down,), pack_down)
    return gu, dn


def clear_pack_cache() -> None:
    _pack_cache.clear()


def ffn_nvfp4(x_heads: torch.Tensor, gather_ids: torch.Tensor, probs: torch.Tensor, expert_offsets: torch.Tensor,
              gu: NVFP4GateUp, dn: NVFP4Down, tok_rows: torch.Tensor | None = None,
              tok_offsets: torch.Tensor | None = None, k_fixed: int = 0,
              out: torch.Tensor | None = None, stage_events=None,
              deterministic: bool | None = None) -> torch.Tensor:
    """NVFP4 expert FFN on x_heads [S, H, dh] bf16 -> y [S, H, dh] bf16.

    ``deterministic``: None -> ``MHMOE_SCATTER`` (default combine); False -> atomic scatter
    from the down GEMM (tok_rows / tok_offsets / k_fixed unused); True -> partials + combine.
    ``stage_events``: optional 5 ``torch.cuda.Event`` recorded on the current stream
    before the tile tables, gate/up GEMM, down GEMM, combine, and at the end.
    """
    _lib.require_cuda(x_heads, expert_offsets)
    S, H, dh0 = x_heads.shape
    n = expert_offsets.numel() - 1
    if gu.num_experts != n or dn.num_experts != n:
        raise ValueError(f"weights hold {gu.num_experts}/{dn.num_experts} experts, expert_offsets {n}")
    dh, de = gu.d_head, gu.d_expert
    if dh0 not in (gu.shape[1], dh) or gu.shape[1] != dn.shape[2] or dh != dn.d_head or de != dn.d_expert:
        raise ValueError("weight shapes do not match x")
    assert dh % 256 == 0 and de % 256 == 0, "packed dimensions are multiples of 256"
    x = x_heads if x_heads.dtype == torch.bfloat16 else x_heads.to(torch.bfloat16)
    if dh != dh0:
        # a head size the tiles do not take: zero-pad the rows (exact; see nvfp4.py), crop y
        y_pad = ffn_nvfp4(torch.nn.functional.pad(x, (0, dh - dh0)), gather_ids, probs, expert_offsets, gu, dn,
                          tok_rows, tok_offsets, k_fixed, None, stage_events, deterministic)
        y = y_pad[..., :dh0]
        if out is not None:
            out.copy_(y)
            return out
        return y.contiguous()
    if x.stride(2) != 1 or x.stride(0) % 8 or x.stride(1) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    dev = x.device
    R = int(gather_ids.numel())
    y = out if out is not None else torch.empty(S, H, dh, dtype=torch.bfloat16, device=dev)
    gids = gather_ids.to(torch.int32).contiguous()
    ps = probs.float().contiguous()
    offs = expert_offsets.to(torch.int64).contiguous()
    L = _lib.lib()
    ws = torch.empty(max(1, L.mhmoe_ffn_workspace_bytes(R, S, H, dh, de, n)), dtype=torch.uint8, device=dev)
    if deterministic is None:
        deterministic = _is_deterministic()
    with torch.cuda.device(dev):
        if deterministic:
            _lib.check(L.mhmoe_ffn_nvfp4(
                x.data_ptr(), x.stride(0), x.stride(1), S, H, dh, de, n, R, gids.data_ptr(), ps.data_ptr(),
                offs.data_ptr(), gu.data.data_ptr(), gu.sf.data_ptr(), gu.gscale.data_ptr(), dn.data.data_ptr(),
                dn.sf.data_ptr(), dn.gscale.data_ptr(), _lib.ptr(tok_rows), _lib.ptr(tok_offsets), int(k_fixed),
                ws.data_ptr(), y.data_ptr(), y.stride(0), y.stride(1), _lib.device_status(dev).data_ptr(), 0,
                _events(stage_events), _lib.stream_ptr(dev)), "flash_mh_moe_fwd")
        else:
            _lib.check(L.mhmoe_ffn_nvfp4_atomic(
                x.data_ptr(), x.stride(0), x.stride(1), S, H, dh, de, n, R, gids.data_ptr(), ps.data_ptr(),
                offs.data_ptr(), gu.data.data_ptr(), gu.sf.data_ptr(), gu.gscale.data_ptr(), dn.data.data_ptr(),
                dn.sf.data_ptr(), dn.gscale.data_ptr(), ws.data_ptr(), y.data_ptr(), y.stride(0), y.stride(1),
                _lib.device_status(dev).data_ptr(), 0, _events(stage_events), _lib.stream_ptr(dev)),
                "flash_mh_moe_fwd")
    return y


def _events(evs):
    if not evs:
        return None
    import ctypes
    arr = (ctypes.c_void_p * 5)()
    for i, e in enumerate(evs):
        if e is None:         # no event at this stage boundary
            continue
        e.record()            # torch creates the CUDA event lazily; the library re-records it in place
        arr[i] = e.cuda_event
    return ctypes.cast(arr, ctypes.c_void_p)


def flash_mh_moe_fwd(
    x: torch.Tensor,
    gather_ids: torch.Tensor,
    probs: torch.Tensor,
    expert_offsets: torch.Tensor,
    W_gate,
    W_up,
    W_down,
) -> torch.Tensor:
    """Flash-MH-MoE forward: gather -> gate/up GEMM -> SwiGLU7 -> down GEMM -> scatter.

    x [S, H, d_head]; gather_ids int32 [T]; probs fp32 [T]; expert_offsets [H*E+1];
    W_gate/W_up [H*E, d_head, d_expert], W_down [H*E, d_expert, d_head] (bf16, packed
    on first use) or their packed ``NVFP4GateUp`` (as W_gate; W_up ignored) and
    ``NVFP4Down`` forms.  Returns y like x (bf16).
    """
    gu, dn = packed_weights(W_gate, W_up, W_down)
    y = ffn_nvfp4(x, gather_ids, probs, expert_offsets, gu, dn)
    return y if x.dtype == torch.bfloat16 else y.to(x.dtype)
