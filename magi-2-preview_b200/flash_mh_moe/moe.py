"""Module-level drop-in for MAGI-2's routed MoE core.

Mirrors ``CoreMultiHeadMoEConfig`` / ``CoreMultiHeadMoE`` / ``magi2_mh_moe``
(``inference/model/magi2_preview.py:2477-2682``): same config keys, parameter names
(``gate``, ``W_gate``, ``W_up``, ``W_down``, ``router.expert_bias``,
``router.expert_bias_ema``), same ``forward(x[S, H*dh]) -> [S, H*dh]`` and the same
opaque custom-op boundary keyed by a stable integer.  The expert weights stay
``params_dtype`` parameters (so reference checkpoints load unchanged); their NVFP4
form is packed on the GPU at first use after a load (quantise on load) and re-packed
whenever a parameter changes.

Forward on one GPU (ep_size == 1):
  router logits (fp32) -> top-k (+expert_bias, route_norm, route_scale) -> stable
  global sort (+ inverse map) -> NVFP4 FFN (gather/quantise, gate/up GEMM + SwiGLU7 +
  hidden quantise, down GEMM x prob) -> deterministic combine.
With ep_size > 1 the experts are sharded across the EP group by contiguous flattened
expert ranges and tokens travel to their experts (flash_mh_moe.ep).
"""
from __future__ import annotations

import itertools
import weakref
from dataclasses import dataclass

import torch
import torch.nn as nn

from .fwd import ffn_nvfp4
from .nvfp4 import NVFP4Down, NVFP4GateUp, pack_down, pack_gate_up
from .route import (compute_topk_probs_and_indices, flash_mh_moe_global_sort_with_inverse,
                    fused_router_supported, route_fused, router_logits, router_prepare)


def _same_key(a, b) -> bool:
    """Keys are tuples of (parameter object, address, version): same objects (identity, not
    tensor equality), same addresses and versions."""
    return a is not None and len(a) == len(b) and all(
        x[0] is y[0] and x[1:] == y[1:] for x, y in zip(a, b))


@dataclass
class CoreMultiHeadMoEConfig:
    hidden_size: int
    num_heads: int
    num_experts: int
    top_k: int
    expert_intermediate_size: int
    num_layers: int
    params_dtype: torch.dtype
    score_func: str = "sigmoid"
    route_norm: bool = True
    route_scale: float = 1.0
    recompute_once_in_bwd: bool = True


# Modules by their op key.  Weak values: registering a module does not keep it (and its
# weights) alive; keys come from a counter, so a key is never reused after a module dies.
_magi2_moe_registry: "weakref.WeakValueDictionary[int, CoreMultiHeadMoE]" = weakref.WeakValueDictionary()
_magi2_moe_keys = itertools.count()


def _psm_ep() -> tuple[int, int, object]:
    """(ep_size, ep_rank, ep_group) from MAGI-2's process-group manager, read the way the
    reference module reads it (``psm.get_world_size("ep")`` at construction,
    ``psm.get_parallel_group("ep")`` at forward: magi2_preview.py:2509, 2632-2637;
    psm.py:94-128), when ``inference.infra.distributed`` is importable; otherwise one rank."""
    try:
        from inference.infra.distributed import psm
    except ImportError:
        return 1, 0, None
    size = int(psm.get_world_size("ep"))
    if size <= 1:
        return 1, 0, None
    return size, int(psm.get_local_rank("ep")), psm.get_parallel_group("ep")


class CoreMultiHeadMoE(nn.Module):
    def __init__(self, config: CoreMultiHeadMoEConfig, ep_group=None) -> None:
        super().__init__()
        if config.hidden_size % config.num_heads != 0:
            raise ValueError("hidden_size must be divisible by num_heads")
        self._moe_key = next(_magi2_moe_keys)
        _magi2_moe_registry[self._moe_key] = self
        self.config = config
        self.num_heads = config.num_heads
        self.num_experts = config.num_experts
        self.topk = config.top_k
        self.d_head = config.hidden_size // config.num_heads
        self.d_expert = config.expert_intermediate_size
        self.flatten_num_experts = self.num_heads * self.num_experts
        if ep_group is not None:
            self.ep_size = torch.distributed.get_world_size(ep_group)
            self.ep_rank = torch.distributed.get_rank(ep_group)
        else:
            # as the reference: the expert-parallel group comes from the process-group manager
            self.ep_size, self.ep_rank, ep_group = _psm_ep()
        self.ep_group = ep_group
        if self.flatten_num_experts % self.ep_size != 0:
            raise ValueError(f"H*E ({self.flatten_num_experts}) must be divisible by ep_size ({self.ep_size})")
        # token -> expert EP: this rank owns flattened experts [expert_lo, expert_lo + local)
        self.local_flatten_num_experts = self.flatten_num_experts // self.ep_size
        self.expert_lo = self.ep_rank * self.local_flatten_num_experts
        nl = self.local_flatten_num_experts
        # The router is replicated: every rank routes its own tokens over all experts.
        self.gate = nn.Parameter(torch.empty(self.flatten_num_experts, self.d_head, dtype=torch.float32))
        self.W_gate = nn.Parameter(torch.empty(nl, self.d_head, self.d_expert, dtype=config.params_dtype))
        self.W_up = nn.Parameter(torch.empty(nl, self.d_head, self.d_expert, dtype=config.params_dtype))
        self.W_down = nn.Parameter(torch.empty(nl, self.d_expert, self.d_head, dtype=config.params_dtype))
        self.router = nn.Module()
        self.router.register_buffer("expert_bias", torch.zeros(self.flatten_num_experts, dtype=torch.float32))
        self.router.register_buffer("expert_bias_ema", torch.zeros(self.flatten_num_experts, dtype=torch.float32))
        self._packed: tuple | None = None
        self._packed_key: tuple | None = None
        self._router_planes: tuple | None = None
        self._router_key: tuple | None = None
        self._masters_released = False

    # ── NVFP4 weights (quantise on load) ──
    def _weights_key(self):
        # the parameter objects themselves are part of the key (held by the key, so a
        # replaced parameter cannot be freed and its address reused while the key exists)
        return tuple((p, p.data_ptr(), p._version) for p in (self.W_gate, self.W_up, self.W_down))

    def packed_weights(self) -> tuple[NVFP4GateUp, NVFP4Down]:
        if self._masters_released:
            return self._packed
        key = self._weights_key()
        if self._packed is None or not _same_key(self._packed_key, key):
            with torch.no_grad():
                self._packed = (pack_gate_up(self.W_gate, self.W_up), pack_down(self.W_down))
            self._packed_key = key
        return self._packed

    _MASTERS = ("W_gate", "W_up", "W_down")

    def _master_shapes(self) -> dict[str, tuple[int, int, int]]:
        nl, dh, de = self.local_flatten_num_experts, self.d_head, self.d_expert
        return {"W_gate": (nl, dh, de), "W_up": (nl, dh, de), "W_down": (nl, de, dh)}

    def release_master_weights(self) -> None:
        """Pack (if needed), then free the params_dtype expert weights: inference only needs
        the NVFP4 operands (0.56 B/weight instead of 2).  The parameters stay registered
        with zero elements until a state dict holding all three of them is loaded: the load
        gives them back their full shapes, copies the new values in, and the next forward
        packs those."""
        self.packed_weights()
        with torch.no_grad():
            for p in (self.W_gate, self.W_up, self.W_down):
                p.data = torch.empty(0, dtype=p.dtype, device=p.device)
        self._masters_released = True

    def load_packed(self, gu: NVFP4GateUp, dn: NVFP4Down) -> None:
        """Install pre-packed NVFP4 operands (e.g. produced offline); skips packing."""
        self._packed = (gu, dn)
        self._packed_key = self._weights_key()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        restore = self._masters_released and all(prefix + n in state_dict for n in self._MASTERS)
        if restore:
            # released masters have zero elements: give them their shapes back so the load
            # copies into them (a released module whose state dict lacks one of the three
            # keeps serving its packed weights)
            for n, shape in self._master_shapes().items():
                p = getattr(self, n)
                p.data = torch.empty(shape, dtype=p.dtype, device=p.device)
        n_err = len(error_msgs)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)
        if len(error_msgs) != n_err:
            if restore:       # this module's load failed: back to the released state
                for n in self._MASTERS:
                    p = getattr(self, n)
                    p.data = torch.empty(0, dtype=p.dtype, device=p.device)
            return
        if restore or not self._masters_released:
            self._masters_released = False    # new masters: pack again at first use

    def router_planes(self) -> tuple[torch.Tensor, int]:
        key = ((self.gate, self.gate.data_ptr(), self.gate._version),)
        if self._router_planes is None or not _same_key(self._router_key, key):
            self._router_planes = router_prepare(self.gate)
            self._router_key = key
        return self._router_planes

    # ── reference structure ──
    def _route(self, x_heads: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """magi2_preview.py:2588-2601: fp32 logits -> top-k -> x route_scale."""
        bias = self.router.expert_bias.view(self.num_heads, self.num_experts)
        if fused_router_supported(self.num_experts, self.topk, self.d_head):
            planes, nsplit = self.router_planes()
            return route_fused(x_heads, planes, nsplit, self.num_experts, self.topk,
                               score_func=self.config.score_func, expert_bias=bias,
                               route_norm=self.config.route_norm, route_scale=float(self.config.route_scale))
        logits = router_logits(x_heads, self.gate, self.num_experts)
        return compute_topk_probs_and_indices(
            logits, self.topk, score_func=self.config.score_func, expert_bias=bias,
            route_norm=self.config.route_norm, route_scale=float(self.config.route_scale))

    def _flash_forward(self, x_heads, topk_probs, topk_indices) -> torch.Tensor:
        gids, ps, offs, inv = flash_mh_moe_global_sort_with_inverse(topk_probs, topk_indices, self.num_experts)
        gu, dn = self.packed_weights()
        return ffn_nvfp4(x_heads, gids, ps, offs, gu, dn, tok_rows=inv, k_fixed=self.topk)

    def _forward_impl(self, x: torch.Tensor) -> torch.Tensor:
        x_heads = x.view(-1, self.num_heads, self.d_head)
        if self.ep_size > 1:
            if self.ep_group is None:
                raise RuntimeError(f"MAGI-2 EP group is not initialized but ep_size={self.ep_size}")
            from .ep import ep_moe_forward
            out = ep_moe_forward(self, x_heads)
        else:
            topk_probs, topk_indices = self._route(x_heads)
            out = self._flash_forward(x_heads, topk_probs, topk_indices)
        return out.reshape(-1, self.num_heads * self.d_head)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return magi2_mh_moe(x, self._moe_key)


@torch.library.custom_op("magi2_b200::mh_moe", mutates_args=())
def magi2_mh_moe(x: torch.Tensor, moe_key: int) -> torch.Tensor:
    """MoE forward (reference op ``infra::magi2_mh_moe``, magi2_preview.py:2668-2682).

    The module is looked up by the stable integer key assigned at construction, so a
    graph compiler sees one opaque op with int-specialised guards.
    """
    moe_module: CoreMultiHeadMoE = _magi2_moe_registry[moe_key]
    return moe_module._forward_impl(x)


@magi2_mh_moe.register_fake
def _magi2_mh_moe_meta(x: torch.Tensor, moe_key: int) -> torch.Tensor:
    return torch.empty_like(x)


def init_moe_params_(m: CoreMultiHeadMoE, seed: int, std: float = 0.02, gate_std: float = 0.02,
                     device: str | torch.device = "cuda") -> None:
    """Seeded synthetic initialisation (benchmarks / tests): gate ~ N(0, gate_std) rounded
    to bf16 and stored fp32; expert weights ~ N(0, std) generated fp32 then cast."""
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        m.gate.copy_((torch.randn(m.gate.shape, generator=g, device=device) * gate_std).to(torch.bfloat16).float())
        for p in (m.W_gate, m.W_up, m.W_down):
            p.copy_((torch.randn(p.shape, generator=g, device=device) * std).to(p.dtype))
