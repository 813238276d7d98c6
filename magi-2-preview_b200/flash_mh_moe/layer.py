"""MAGI-2's full MoE layer around the routed core, B200-native.

Mirrors ``MultiHeadMoELayer`` / ``MultiHeadMoELayerConfig``
(``inference/model/magi2_preview.py:2685-2806``) with the same config fields and the same
parameter names and shapes (``pre_norm.weight``, ``split_linear.weight``,
``merge_linear.weight``, ``shared_expert_fc1/fc2.weight``,
``modality_specific_shared_expert_fc1/fc2.weight``, ``moe_mlp.*``), so the reference
checkpoint loads unchanged:

    norm   = pre_norm(x)                       multi-modality RMSNorm (mhmoe_rmsnorm kernel)
    moe    = merge(moe_mlp(split(norm)))       split / merge: bf16 library GEMMs
    shared = fc2(swiglu7(fc1(norm))) + fc2_m(swiglu7(fc1_m(norm)))   per modality m
    out    = moe + shared

The two shared experts run on the routed path's NVFP4 expert FFN: each token is a
"routed" row of exactly two experts, the shared one and its modality's, with weight 1.
The reference's interleaved SwiGLU7 over ``concat([fc1(x), fc1_m(x)])``
(``:2775-2795``, ``swiglu7`` at ``:86-98``: even columns gate, odd columns linear) is that
FFN's SwiGLU7 with gate rows ``fc1.weight[0::2]`` and up rows ``fc1.weight[1::2]``, and
``x1 + x2`` is its combine (the bf16 partial rows summed in fp32, rounded once).  The
merge GEMM accumulates onto the shared output (one fused ``addmm``), which is the final
``moe + shared``.  Rows of ``hidden_states`` are grouped by modality, as MAGI-2's
``ModalityDispatcher`` lays them out.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .fwd import ffn_nvfp4
from .moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, _same_key
from .nvfp4 import pack_down, pack_gate_up


class MLPActivationType(Enum):
    """magi2_preview.py:65-68."""
    SWIGLU7 = "swiglu7"


@dataclass
class MoEConfig:
    """The MoE keys of MAGI-2's model config (inference/common/magi2_config.py:107-118)."""
    num_experts: int = 256
    top_k: int = 6
    score_func: str = "sigmoid"
    route_norm: bool = True
    route_scale: float = 4.90
    moe_layers: list = field(default_factory=lambda: list(range(2, 38)))
    expert_intermediate_size: int = 1280
    shared_expert_intermediate_size: int = 1280
    modality_specific_expert_intermediate_size: int = 1280
    num_heads: int = 12
    split_merge_intermediate_size: Optional[int] = None


@dataclass
class MultiHeadMoELayerConfig:
    """magi2_preview.py:2686-2697."""
    hidden_size: int
    num_modality: int
    num_layers: int
    activation_type: MLPActivationType
    params_dtype: torch.dtype
    shared_expert_intermediate_sizes: int
    modality_specific_expert_intermediate_sizes: int
    shared_expert_params_dtype: torch.dtype
    split_merge_intermediate_size: Optional[int]
    moe_config: MoEConfig


def group_layout(modality_dispatcher, rows: int, num_modality: int,
                 device: torch.device) -> tuple[list[int], torch.Tensor]:
    """(host group sizes, device int32 cumulative sizes [n+1]) of the modality groups.

    Accepts MAGI-2's ``ModalityDispatcher`` (``group_size_cpu`` / ``cu_group_sizes``,
    magi2_preview.py:1448-1527), a sequence of group sizes, or None for one modality."""
    if modality_dispatcher is None:
        if num_modality > 1:
            raise AssertionError("modality_dispatcher is required for multi-modality RMSNorm")
        sizes = [rows]
    elif hasattr(modality_dispatcher, "group_size_cpu"):
        sizes = [int(v) for v in modality_dispatcher.group_size_cpu]
    elif isinstance(modality_dispatcher, torch.Tensor):
        sizes = [int(v) for v in modality_dispatcher.tolist()]
    else:
        sizes = [int(v) for v in modality_dispatcher]
    if len(sizes) != num_modality or sum(sizes) != rows or min(sizes) < 0:
        raise ValueError(f"modality group sizes {sizes} do not split {rows} rows into {num_modality} groups")
    cu = [0]
    for v in sizes:
        cu.append(cu[-1] + v)
    return sizes, torch.tensor(cu, dtype=torch.int32).to(device, non_blocking=True)


class MultiModalityRMSNorm(nn.Module):
    """RMSNorm with one fp32 weight row per modality and weight bias 1
    (magi2_preview.py:497-623), computed by the mhmoe_rmsnorm kernel."""

    def __init__(self, dim: int, eps: float = 1e-6, device=None, num_modality: int = 1, num_patterns: int = 1,
                 out_dtype: torch.dtype | None = None):
        super().__init__()
        if num_patterns != 1:
            raise NotImplementedError("num_patterns > 1 (multi-head norms) is not on the MoE layer's path")
        self.dim, self.eps, self.num_modality, self.num_patterns = dim, eps, num_modality, num_patterns
        self.out_dtype = out_dtype
        self.weight_bias = 1.0
        self.weight = nn.Parameter(torch.zeros(num_patterns * dim * num_modality, device=device,
                                               dtype=torch.float32))

    def forward(self, x: torch.Tensor, modality_dispatcher=None, cu_groups: torch.Tensor | None = None
                ) -> torch.Tensor:
        _lib.require_cuda(x)
        if self.out_dtype not in (None, torch.bfloat16) or x.dtype != torch.bfloat16:
            raise NotImplementedError("the fused RMSNorm takes and returns bf16")
        rows = x.numel() // self.dim
        x2 = x.reshape(rows, self.dim)
        if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        if cu_groups is None and self.num_modality > 1:
            _, cu_groups = group_layout(modality_dispatcher, rows, self.num_modality, x.device)
        y = torch.empty(rows, self.dim, dtype=torch.bfloat16, device=x.device)
        w = self.weight.detach()
        if w.dtype != torch.float32 or not w.is_contiguous():
            w = w.float().contiguous()
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().mhmoe_rmsnorm(
                x2.data_ptr(), x2.stride(0), w.data_ptr(), _lib.ptr(cu_groups), self.num_modality, rows, self.dim,
                float(self.eps), float(self.weight_bias), y.data_ptr(), y.stride(0), _lib.stream_ptr(x.device)),
                "rmsnorm")
        return y.view(x.shape)


class CustomGroupedLinear(nn.Module):
    """Parameter container of the reference's (grouped) linear (magi2_preview.py:162-207,
    626-698): weight [num_experts * out_features, in_features]; expert i's rows are the
    i-th ``out_features`` block.  Its forward (a plain library GEMM per group) is kept for
    callers that use the module directly; the MoE layer reads the weights."""

    def __init__(self, in_features: int, out_features: int, num_experts: int = 1, num_patterns: int = 1,
                 num_layers_for_initialization: int = 1, bias: bool = False, device=None,
                 dtype: torch.dtype | None = None) -> None:
        super().__init__()
        if bias:
            raise NotImplementedError("the MoE layer's linears have no bias")
        self.in_features, self.out_features = in_features, out_features
        self.num_experts, self.num_patterns = num_experts, num_patterns
        self.weight = nn.Parameter(torch.empty(num_experts * out_features, in_features, device=device, dtype=dtype))
        self.register_parameter("bias", None)

    def expert_weight(self, i: int) -> torch.Tensor:
        return self.weight.view(self.num_experts, self.out_features, self.in_features)[i]

    def forward(self, input: torch.Tensor, modality_dispatcher=None) -> torch.Tensor:
        if self.num_experts == 1:
            return F.linear(input, self.expert_weight(0))
        sizes, _ = group_layout(modality_dispatcher, input.shape[0], self.num_experts, input.device)
        chunks = torch.split(input, sizes, dim=0)
        return torch.cat([F.linear(c, self.expert_weight(i)) for i, c in enumerate(chunks)], dim=0)


def create_linear(in_features: int, out_features: int, num_layers: int = 1, num_experts: int = 1,
                  num_patterns: int = 1, bias: bool = True, device=None, dtype=None) -> CustomGroupedLinear:
    """magi2_preview.py:672-698."""
    return CustomGroupedLinear(in_features, out_features, num_experts, num_patterns, num_layers, bias, device,
                               dtype)


class MultiHeadMoELayer(nn.Module):
    """magi2_preview.py:2699-2806 (see the module docstring for the B200 data path)."""

    def __init__(self, config: MultiHeadMoELayerConfig, ep_group=None) -> None:
        super().__init__()
        act = config.activation_type
        if (act.value if isinstance(act, Enum) else str(act)) != MLPActivationType.SWIGLU7.value:
            raise ValueError(f"Unknown activation type: {act}")
        self.config = config
        mc = config.moe_config
        moe_hidden = config.split_merge_intermediate_size or config.hidden_size
        self.moe_mlp = CoreMultiHeadMoE(CoreMultiHeadMoEConfig(
            hidden_size=moe_hidden, num_heads=mc.num_heads, num_experts=mc.num_experts, top_k=mc.top_k,
            expert_intermediate_size=mc.expert_intermediate_size, num_layers=config.num_layers,
            params_dtype=config.params_dtype, score_func=mc.score_func, route_norm=mc.route_norm,
            route_scale=mc.route_scale), ep_group=ep_group)
        self.is_swiglu = True
        d, M = config.hidden_size, config.num_modality
        Is, Im = config.shared_expert_intermediate_sizes, config.modality_specific_expert_intermediate_sizes
        sdt = config.shared_expert_params_dtype
        self.shared_expert_fc1 = create_linear(d, 2 * Is, config.num_layers, 1, dtype=sdt, bias=False)
        self.shared_expert_fc2 = create_linear(Is, d, config.num_layers, 1, dtype=sdt, bias=False)
        self.modality_specific_shared_expert_fc1 = create_linear(d, 2 * Im, config.num_layers, M, dtype=sdt,
                                                                 bias=False)
        self.modality_specific_shared_expert_fc2 = create_linear(Im, d, config.num_layers, M, dtype=sdt, bias=False)
        self.pre_norm = MultiModalityRMSNorm(d, num_modality=M)
        mid = config.split_merge_intermediate_size or config.hidden_size
        self.split_linear = create_linear(d, mid, config.num_layers, dtype=sdt, bias=False)
        self.merge_linear = create_linear(mid, d, config.num_layers, dtype=sdt, bias=False)
        self._shared_packed = None
        self._shared_key = None
        self._routing_cache: dict = {}

    # ── shared experts as an NVFP4 expert set: expert 0 = shared, expert 1 + m = modality m ──
    def _shared_params(self):
        return (self.shared_expert_fc1.weight, self.shared_expert_fc2.weight,
                self.modality_specific_shared_expert_fc1.weight, self.modality_specific_shared_expert_fc2.weight)

    def shared_expert_weights(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The shared experts in the routed experts' layout: W_gate / W_up [1+M, d, I] and
        W_down [1+M, I, d] (bf16), I = max of the two intermediate sizes (the smaller one
        zero-padded: zero gate and up columns give a zero SwiGLU7 output)."""
        c = self.config
        d, M = c.hidden_size, c.num_modality
        Is, Im = c.shared_expert_intermediate_sizes, c.modality_specific_expert_intermediate_sizes
        I = max(Is, Im)
        fc1_s, fc2_s, fc1_m, fc2_m = (p.detach() for p in self._shared_params())
        dev = fc1_s.device
        Wg = torch.zeros(1 + M, d, I, dtype=torch.bfloat16, device=dev)
        Wu = torch.zeros_like(Wg)
        Wd = torch.zeros(1 + M, I, d, dtype=torch.bfloat16, device=dev)
        fc1s = [fc1_s] + list(fc1_m.view(M, 2 * Im, d))
        fc2s = [fc2_s] + list(fc2_m.view(M, d, Im))
        for e in range(1 + M):
            n = Is if e == 0 else Im
            Wg[e, :, :n] = fc1s[e][0::2].t()          # swiglu7: even columns gate
            Wu[e, :, :n] = fc1s[e][1::2].t()          #          odd columns linear
            Wd[e, :n, :] = fc2s[e].t()
        return Wg, Wu, Wd

    def shared_packed(self):
        key = tuple((p, p.data_ptr(), p._version) for p in self._shared_params())
        if self._shared_packed is None or not _same_key(self._shared_key, key):
            with torch.no_grad():
                Wg, Wu, Wd = self.shared_expert_weights()
                self._shared_packed = (pack_gate_up(Wg, Wu), pack_down(Wd))
            self._shared_key = key
        return self._shared_packed

    def _shared_routing(self, sizes: Sequence[int], device: torch.device):
        """Sorted rows of the shared FFN: rows [0, S) are every token on expert 0, then each
        modality's tokens on its expert; token s's rows are s and S + s (ascending)."""
        k = (tuple(sizes), device)
        hit = self._routing_cache.get(k)
        if hit is None:
            S = sum(sizes)
            tok = torch.arange(S, dtype=torch.int32)
            gather_ids = torch.cat([tok, tok])
            offs = torch.tensor([0, S] + [S + v for v in torch.tensor(sizes).cumsum(0).tolist()], dtype=torch.int64)
            tok_rows = torch.stack([tok, tok + S], dim=1).reshape(-1)
            hit = tuple(t.to(device) for t in (gather_ids, torch.ones(2 * S, dtype=torch.float32), offs, tok_rows))
            if len(self._routing_cache) > 16:
                self._routing_cache.clear()
            self._routing_cache[k] = hit
        return hit

    def _shared_expert_forward(self, norm_output: torch.Tensor, sizes: Sequence[int]) -> torch.Tensor:
        gids, probs, offs, tok_rows = self._shared_routing(sizes, norm_output.device)
        gu, dn = self.shared_packed()
        S, d = norm_output.shape
        y = ffn_nvfp4(norm_output.view(S, 1, d), gids, probs, offs, gu, dn, tok_rows=tok_rows, k_fixed=2,
                      deterministic=True)
        return y.view(S, d)

    def forward(self, hidden_states: torch.Tensor, modality_dispatcher=None) -> torch.Tensor:
        _lib.require_cuda(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, self.config.hidden_size)
        sizes, cu = group_layout(modality_dispatcher, x.shape[0], self.config.num_modality, x.device)
        norm_output = self.pre_norm(x, cu_groups=cu)
        moe_out = self.moe_mlp(F.linear(norm_output, self.split_linear.weight))
        shared = self._shared_expert_forward(norm_output, sizes)
        # merge_linear(moe_out) + shared in one GEMM (accumulating onto the shared output)
        out = torch.addmm(shared, moe_out, self.merge_linear.weight.t())
        return out.view(shape)
