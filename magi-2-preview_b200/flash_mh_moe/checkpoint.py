"""Checkpoint loading for the MoE layers with NVFP4 quantise-on-load.

MAGI-2 checkpoints are HuggingFace-style safetensors directories whose MoE tensors are
concatenated over (head, expert) along dim 0.  The reference loader
(``inference/infra/checkpoint/magi2_checkpointing.py``) reads, per expert-parallel rank,
only the dim-0 rows that rank owns (``_read_ep_slice``, ``:81-105``: start =
``ep_rank * shard_rows``, rows past the real ones zero-filled), casts to the target dtype
(``:170-173``) and substitutes the EMA router bias (``_apply_router_bias_ema``,
``:132-157``; ``MAGI2_ROUTER_BIAS_SOURCE=main`` keeps the raw bias).

``load_moe_module`` applies the same rules to one ``CoreMultiHeadMoE`` and quantises its
expert weights on the way in: the bf16 rows of a few experts at a time are read from the
file, uploaded and packed to NVFP4 straight into the module's packed operands, so the
full bf16 expert weights never have to sit on the GPU (``release_masters``) — at MAGI-2's
shape a layer's routed experts take 2.01 GB as bf16 and 0.57 GB as NVFP4.

Token -> expert expert parallelism owns contiguous flattened-expert ranges
``[ep_rank * n_local, (ep_rank + 1) * n_local)``: exactly the rows the reference rule gives
a rank whose module holds ``n_local`` experts, so the same rule serves both.  The router
(``gate``, ``router.expert_bias``, ``router.expert_bias_ema``) is replicated here: its
target holds every row, which the rule reads whole.
"""
from __future__ import annotations

import json
import os
from typing import Callable

import torch

EP_SHARDED_SUFFIXES = ("moe_mlp.gate", "moe_mlp.W_gate", "moe_mlp.W_up", "moe_mlp.W_down",
                       "moe_mlp.router.expert_bias", "moe_mlp.router.expert_bias_ema")
_INDEX_NAME = "model.safetensors.index.json"
_SINGLE_NAME = "model.safetensors"


def read_weight_map(checkpoint_dir: str) -> dict[str, str]:
    """Tensor name -> file of a safetensors directory (magi2_checkpointing.py:53-67)."""
    index = os.path.join(checkpoint_dir, _INDEX_NAME)
    if os.path.exists(index):
        with open(index) as f:
            wm = json.load(f)["weight_map"]
        return {k: os.path.join(checkpoint_dir, v) for k, v in wm.items()}
    single = os.path.join(checkpoint_dir, _SINGLE_NAME)
    if not os.path.exists(single):
        raise FileNotFoundError(f"No {_INDEX_NAME} or {_SINGLE_NAME} under {checkpoint_dir}")
    from safetensors import safe_open
    with safe_open(single, framework="pt") as f:
        return {k: single for k in f.keys()}


def ep_rows(real_rows: int, shard_rows: int, ep_rank: int, ep_size: int) -> tuple[int, int, int]:
    """(start, stop, zero rows appended) of the dim-0 rows a rank reads for a tensor with
    ``real_rows`` rows into a target of ``shard_rows`` rows (magi2_checkpointing.py:81-105)."""
    if ep_size <= 1 or shard_rows == real_rows:
        return 0, real_rows, 0
    start = ep_rank * shard_rows
    if start >= real_rows:
        return real_rows, real_rows, shard_rows
    stop = min(start + shard_rows, real_rows)
    return start, stop, shard_rows - (stop - start)


_ST_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "F64": torch.float64,
              "I64": torch.int64, "I32": torch.int32, "U8": torch.uint8}


def _read_rows(handle, key: str, start: int, stop: int, pad: int) -> torch.Tensor:
    """Rows [start, stop) of tensor ``key``, then ``pad`` zero rows."""
    view = handle.get_slice(key)
    shape = view.get_shape()
    if start == 0 and stop == shape[0] and pad == 0:
        return handle.get_tensor(key)
    chunk = view[start:stop] if stop > start else None
    if pad == 0:
        return chunk
    dtype = chunk.dtype if chunk is not None else _ST_DTYPES[view.get_dtype()]
    zeros = torch.zeros((pad, *shape[1:]), dtype=dtype)
    return zeros if chunk is None else torch.cat([chunk, zeros], dim=0)


def router_bias_source() -> str:
    return (os.environ.get("MAGI2_ROUTER_BIAS_SOURCE") or "ema").strip().lower()


class _Files:
    """Opened safetensors files, each opened once."""

    def __init__(self, weight_map: dict[str, str]):
        self.weight_map = weight_map
        self.handles: dict[str, object] = {}

    def handle(self, key: str):
        from safetensors import safe_open
        path = self.weight_map[key]
        h = self.handles.get(path)
        if h is None:
            h = safe_open(path, framework="pt")
            h.__enter__()
            self.handles[path] = h
        return h

    def close(self):
        for h in self.handles.values():
            h.__exit__(None, None, None)
        self.handles.clear()


def load_moe_module(module, checkpoint_dir: str | None = None, prefix: str = "", *,
                    weight_map: dict[str, str] | None = None, quantize: bool = True, release_masters: bool = True,
                    chunk_experts: int = 32) -> dict[str, tuple[int, int, int]]:
    """Load one ``CoreMultiHeadMoE`` (``prefix`` = its name in the model, e.g.
    ``"blocks.3.mlp.moe_mlp."``) from a safetensors directory.

    Router tensors are read whole; ``W_gate``/``W_up``/``W_down`` as this rank's dim-0 rows
    (the reference's EP rule).  ``quantize``: pack to NVFP4 on the module's device while
    reading, ``chunk_experts`` experts at a time; with ``release_masters`` the bf16 expert
    parameters are left empty (``CoreMultiHeadMoE.release_master_weights`` state), else they
    are filled too.  Returns the (start, stop, pad) row ranges read per key."""
    from .nvfp4 import NVFP4Down, NVFP4GateUp, pack_down, pack_gate_up, padded
    wm = weight_map if weight_map is not None else read_weight_map(checkpoint_dir)
    files = _Files(wm)
    ranges: dict[str, tuple[int, int, int]] = {}
    dev = module.gate.device
    try:
        def key_of(name):
            k = prefix + name
            if k not in wm:
                raise KeyError(f"{k} not in the checkpoint")
            return k

        # router: replicated (the whole tensor is this rank's slice)
        with torch.no_grad():
            for name, target in (("gate", module.gate), ("router.expert_bias", module.router.expert_bias),
                                 ("router.expert_bias_ema", module.router.expert_bias_ema)):
                k = key_of(name)
                h = files.handle(k)
                rng = ep_rows(h.get_slice(k).get_shape()[0], target.shape[0], module.ep_rank, module.ep_size)
                ranges[k] = rng
                target.copy_(_read_rows(h, k, *rng).to(target.dtype))
            if router_bias_source() != "main":          # magi2_checkpointing.py:132-157
                module.router.expert_bias.copy_(module.router.expert_bias_ema)

        nl = module.local_flatten_num_experts
        kg, ku, kd = key_of("W_gate"), key_of("W_up"), key_of("W_down")
        rng_e = {}
        for k in (kg, ku, kd):
            rng_e[k] = ep_rows(files.handle(k).get_slice(k).get_shape()[0], nl, module.ep_rank, module.ep_size)
            ranges[k] = rng_e[k]

        def rows(k, a, b):
            """Rows [a, b) of this rank's slice of tensor k (zero rows past the real ones)."""
            start, stop, _ = rng_e[k]
            lo, hi = start + a, min(start + b, stop)
            return _read_rows(files.handle(k), k, lo, max(lo, hi), (b - a) - max(0, hi - lo))

        if not quantize:
            with torch.no_grad():
                for k, p in ((kg, module.W_gate), (ku, module.W_up), (kd, module.W_down)):
                    if p.numel() == 0:
                        p.data = torch.empty(module._master_shapes()[k[len(prefix):]], dtype=p.dtype,
                                             device=p.device)
                    p.copy_(rows(k, 0, nl).to(p.dtype))
            module._masters_released = False
            return ranges

        dh0, de0 = module.d_head, module.d_expert
        dh, de = padded(dh0), padded(de0)          # the packed (tile-multiple) sizes
        gu = NVFP4GateUp(torch.empty(nl, 2 * de, dh // 2, dtype=torch.uint8, device=dev),
                         torch.empty(nl, 2 * de * dh // 16, dtype=torch.uint8, device=dev),
                         torch.empty(2, nl, dtype=torch.float32, device=dev), nl, dh, de, dh0, de0)
        dn = NVFP4Down(torch.empty(nl, dh, de // 2, dtype=torch.uint8, device=dev),
                       torch.empty(nl, dh * de // 16, dtype=torch.uint8, device=dev),
                       torch.empty(nl, dtype=torch.float32, device=dev), nl, dh, de, dh0, de0)
        keep = not release_masters
        if keep:
            for n, p in (("W_gate", module.W_gate), ("W_up", module.W_up), ("W_down", module.W_down)):
                if p.numel() == 0:
                    p.data = torch.empty(module._master_shapes()[n], dtype=p.dtype, device=p.device)
        with torch.no_grad():
            for a in range(0, nl, chunk_experts):
                b = min(nl, a + chunk_experts)
                wg = rows(kg, a, b).to(dev, torch.bfloat16)
                wu = rows(ku, a, b).to(dev, torch.bfloat16)
                wd = rows(kd, a, b).to(dev, torch.bfloat16)
                cg, cd = pack_gate_up(wg, wu), pack_down(wd)
                gu.data[a:b].copy_(cg.data)
                gu.sf[a:b].copy_(cg.sf)
                gu.gscale[:, a:b].copy_(cg.gscale)
                dn.data[a:b].copy_(cd.data)
                dn.sf[a:b].copy_(cd.sf)
                dn.gscale[a:b].copy_(cd.gscale)
                if keep:
                    module.W_gate[a:b].copy_(wg)
                    module.W_up[a:b].copy_(wu)
                    module.W_down[a:b].copy_(wd)
        if release_masters:
            for p in (module.W_gate, module.W_up, module.W_down):
                p.data = torch.empty(0, dtype=p.dtype, device=p.device)
        module.load_packed(gu, dn)
        module._masters_released = release_masters
        return ranges
    finally:
        files.close()


def load_moe_layers(model: torch.nn.Module, checkpoint_dir: str, *, quantize: bool = True,
                    release_masters: bool = True, chunk_experts: int = 32,
                    progress: Callable[[str], None] | None = None) -> int:
    """Quantise-on-load every ``CoreMultiHeadMoE`` inside ``model`` from the checkpoint
    (keys ``<module name>.gate``, ``.W_gate``, ...).  Returns the number of modules loaded.
    The rest of the model loads through the reference's own loader unchanged."""
    from .moe import CoreMultiHeadMoE
    wm = read_weight_map(checkpoint_dir)
    n = 0
    for name, mod in model.named_modules():
        if isinstance(mod, CoreMultiHeadMoE):
            load_moe_module(mod, prefix=name + "." if name else "", weight_map=wm, quantize=quantize,
                            release_masters=release_masters, chunk_experts=chunk_experts)
            n += 1
            if progress:
                progress(name)
    return n
