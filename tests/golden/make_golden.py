"""Generate golden fixtures by running the reference implementation itself.

Run once, in a container that has the reference checkout, with ``MAGI2_REFERENCE``
naming its root directory.  The fixtures are committed; nothing at test time reads the
reference.

    MAGI2_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Produces:
* ``route_cases.npz`` — inputs/outputs of ``compute_topk_probs_and_indices``
  (``inference/flash_mh_moe/route.py:157``) and ``flash_mh_moe_global_sort``
  (``route.py:209``) on seeded logits: softmax/sigmoid, expert_bias, virtual
  groups, route_norm off, a Zipf-skewed bias, the production head shape.
* ``ffn_fp32.npz`` — the reference Triton kernel ``_mh_moe_fwd_kernel``
  (``inference/flash_mh_moe/triton/mh_moe_fwd.py:50-181``) run under
  ``TRITON_INTERPRET=1`` on fp32 tensors (the interpreter does not support bf16),
  atomic and deterministic variants.
* ``layer_cases.npz`` — the MoE layer's pre-norm and shared experts from the reference
  module ``inference/model/magi2_preview.py`` (``MultiModalityRMSNorm`` torch path,
  ``MultiHeadMoELayer._shared_expert_forward``) in bf16 on the CPU, with seeded weights.
* ``ckpt_slices.npz`` — the rows the reference checkpoint reader's expert-parallel rule
  (``inference/infra/checkpoint/magi2_checkpointing.py:81-105``) gives each rank.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
def _reference_root() -> Path:
    root = os.environ.get("MAGI2_REFERENCE")
    if not root:
        raise SystemExit("set MAGI2_REFERENCE to the reference checkout's root directory")
    return Path(root)


def _import_reference():
    sys.path.insert(0, str(_reference_root()))
    import torch  # noqa: F401
    from inference.flash_mh_moe import route  # type: ignore
    return route


ROUTE_CASES = [
    # name, H, S, E, K, score_func, bias, nvg, tvg, route_norm, seed
    ("cfg0_softmax", 1, 512, 8, 2, "softmax", False, 1, 0, True, 0),
    ("sigmoid_bias", 2, 64, 16, 4, "sigmoid", True, 1, 0, True, 11),
    ("softmax_vgroup", 2, 64, 16, 4, "softmax", False, 4, 2, True, 12),
    ("softmax_nonorm", 1, 128, 32, 8, "softmax", False, 1, 0, False, 13),
    ("zipf_logit_bias", 1, 256, 128, 8, "softmax", False, 1, 0, True, 2),
    ("prod_heads_sigmoid", 12, 16, 256, 6, "sigmoid", True, 1, 0, True, 14),
    ("sigmoid_vgroup_bias", 1, 96, 64, 6, "sigmoid", True, 8, 3, True, 15),
]


def make_route(route):
    import torch
    out = {}
    for name, H, S, E, K, sf, use_bias, nvg, tvg, rn, seed in ROUTE_CASES:
        g = torch.Generator().manual_seed(seed)
        if name == "cfg0_softmax":
            # config 0 router: x bf16 N(0,1) [S,1,1024]; gate bf16 N(0,0.02) stored fp32 (magi2_preview.py:2588-2591)
            x = torch.randn(S, 1, 1024, generator=g).to(torch.bfloat16)
            gate = (torch.randn(E, 1024, generator=g) * 0.02).to(torch.bfloat16).float()
            logits = torch.einsum("shd,hed->hse", x.float(), gate.view(1, E, 1024))
        else:
            logits = torch.randn(H, S, E, generator=g) * 1.5
        if name == "zipf_logit_bias":
            e = torch.arange(E, dtype=torch.float32)
            logits = logits + 2.0 * torch.log((e + 1.0) ** -1.2)
        bias = (torch.randn(H, E, generator=g) * 0.05) if use_bias else None
        probs, idx = route.compute_topk_probs_and_indices(
            logits, K, score_func=sf, expert_bias=bias, num_virtual_group=nvg,
            topk_virtual_group=tvg, route_norm=rn)
        gids, psorted, offs = route.flash_mh_moe_global_sort(probs, idx, E)
        p = f"{name}/"
        out[p + "meta"] = np.array([H, S, E, K, nvg, tvg, int(rn), int(use_bias)], np.int64)
        out[p + "score_func"] = np.array(sf)
        out[p + "logits"] = logits.numpy().astype(np.float32)
        if bias is not None:
            out[p + "bias"] = bias.numpy().astype(np.float32)
        out[p + "probs"] = probs.numpy()
        out[p + "idx"] = idx.numpy()
        out[p + "gather_ids"] = gids.numpy()
        out[p + "probs_sorted"] = psorted.numpy()
        out[p + "expert_offsets"] = offs.numpy()
    np.savez_compressed(HERE / "route_cases.npz", **out)
    print("route_cases.npz:", len(ROUTE_CASES), "cases")


def make_ffn(route):
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    torch.cuda.get_device_capability = lambda *a, **k: (10, 0)    # mh_moe_fwd.py:225 on a CPU box
    from inference.flash_mh_moe.triton import mh_moe_fwd as mk  # type: ignore
    out = {}
    cases = [("small", 32, 2, 64, 4, 2, 64, 21), ("ragged", 40, 1, 128, 8, 3, 96, 22)]
    for name, S, H, dh, E, K, de, seed in cases:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(S, H, dh, generator=g)
        logits = torch.randn(H, S, E, generator=g)
        if name == "ragged":
            logits[:, :, 0] += 4.0          # one crowded expert, some empty ones
            logits[:, :, E - 1] -= 8.0
        probs, idx = route.compute_topk_probs_and_indices(logits, K, score_func="softmax")
        gids, ps, offs = route.flash_mh_moe_global_sort(probs, idx, E)
        Wg = torch.randn(H * E, dh, de, generator=g) * 0.05
        Wu = torch.randn(H * E, dh, de, generator=g) * 0.05
        Wd = torch.randn(H * E, de, dh, generator=g) * 0.05
        p = f"{name}/"
        for det in (False, True):
            y = mk.mh_moe_fwd_func(x, gids, ps, offs, Wg, Wu, Wd, deterministic=det)
            out[p + ("y_det" if det else "y_atomic")] = y.numpy()
        out[p + "x"] = x.numpy()
        out[p + "gather_ids"] = gids.numpy()
        out[p + "probs_sorted"] = ps.numpy()
        out[p + "expert_offsets"] = offs.numpy()
        out[p + "W_gate"] = Wg.numpy()
        out[p + "W_up"] = Wu.numpy()
        out[p + "W_down"] = Wd.numpy()
    np.savez_compressed(HERE / "ffn_fp32.npz", **out)
    print("ffn_fp32.npz:", len(cases), "cases")


def _import_reference_model():
    """inference/model/magi2_preview.py on a CPU box: three GPU-only imports it names at
    module level are stubbed (FA3, MagiAttention's FA3-with-sink, MagiCompiler's
    decorators as identities) and torch.compile runs eagerly; nothing on the MoE layer's
    path uses them."""
    import types
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    sys.path.insert(0, str(_reference_root()))
    def _stub(name, value):
        m = types.ModuleType(name)

        def attr(a):
            if a.startswith("__"):
                raise AttributeError(a)
            return value
        m.__getattr__ = attr
        sys.modules.setdefault(name, m)
    _stub("flash_attn_interface", types.SimpleNamespace())
    _stub("magi_attn_extensions", None)
    _stub("magi_attn_extensions.fa3_interface_with_sink", lambda *a, **k: None)
    mc = types.ModuleType("magi_compiler")

    def _identity_decorator(*a, **k):
        if len(a) == 1 and callable(a[0]) and not k:
            return a[0]
        return lambda f: f
    mc.magi_compile = mc.magi_register_custom_op = _identity_decorator
    sys.modules.setdefault("magi_compiler", mc)
    from inference.model import magi2_preview  # type: ignore
    return magi2_preview


LAYER_CASES = [
    # name, modality group sizes, hidden, shared, modality-specific, seed
    ("three_modalities", (40, 24, 32), 256, 128, 128, 31),
    ("empty_modality_unequal", (16, 0, 48), 256, 64, 128, 32),
]


def make_layer(mp):
    """MultiModalityRMSNorm (magi2_preview.py:497-623, torch path) and
    MultiHeadMoELayer._shared_expert_forward (:2775-2795) in bf16, from the reference
    module itself; split/merge are plain F.linear and the routed core is pinned above."""
    import torch
    out = {}
    for name, groups, d, Is, Im, seed in LAYER_CASES:
        g = torch.Generator().manual_seed(seed)
        moe = mp.MoEConfig(num_experts=4, top_k=2, num_heads=1, expert_intermediate_size=64,
                           shared_expert_intermediate_size=Is, modality_specific_expert_intermediate_size=Im) \
            if hasattr(mp, "MoEConfig") else None
        if moe is None:
            from inference.common.magi2_config import MoEConfig  # type: ignore
            moe = MoEConfig(num_experts=4, top_k=2, num_heads=1, expert_intermediate_size=64,
                            shared_expert_intermediate_size=Is, modality_specific_expert_intermediate_size=Im)
        cfg = mp.MultiHeadMoELayerConfig(hidden_size=d, num_modality=len(groups), num_layers=1,
                                         activation_type=mp.MLPActivationType.SWIGLU7, params_dtype=torch.bfloat16,
                                         shared_expert_intermediate_sizes=Is,
                                         modality_specific_expert_intermediate_sizes=Im,
                                         shared_expert_params_dtype=torch.bfloat16,
                                         split_merge_intermediate_size=None, moe_config=moe)
        layer = mp.MultiHeadMoELayer(cfg)
        p = f"{name}/"
        with torch.no_grad():
            for pname, prm in layer.named_parameters():
                if pname.startswith("moe_mlp."):
                    continue
                std = 0.1 if pname == "pre_norm.weight" else 0.05
                prm.copy_((torch.randn(prm.shape, generator=g) * std).to(prm.dtype))
                out[p + pname] = prm.float().numpy()
        mapping = torch.cat([torch.full((n,), m, dtype=torch.int64) for m, n in enumerate(groups)])
        disp = mp.ModalityDispatcher(mapping, len(groups))
        x = torch.randn(sum(groups), d, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            layer.pre_norm.backend = "torch"
            norm = layer.pre_norm(x, modality_dispatcher=disp)
            shared = layer._shared_expert_forward(norm, disp)
        out[p + "groups"] = np.array(groups, np.int64)
        out[p + "x"] = x.float().numpy()
        out[p + "norm"] = norm.float().numpy()
        out[p + "shared"] = shared.float().numpy()
    np.savez_compressed(HERE / "layer_cases.npz", **out)
    print("layer_cases.npz:", len(LAYER_CASES), "cases")


CKPT_CASES = [
    # real rows, target rows, ep size
    (12, 12, 4),        # replicated router tensor: read whole
    (12, 3, 4),         # even split
    (12, 4, 4),         # heads padded up to the EP size: the last rank is all zeros
    (10, 4, 3),         # the last rank partly past the real rows
]


def make_ckpt():
    """The reference's EP row reader (_read_ep_slice, magi2_checkpointing.py:81-105) on a
    safetensors file of numbered rows, for every rank of each case."""
    import tempfile

    import torch
    from safetensors.torch import save_file
    sys.path.insert(0, str(_reference_root()))
    from safetensors import safe_open
    from inference.infra.checkpoint import magi2_checkpointing as ck  # type: ignore
    out = {}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "t.safetensors")
        tensors = {f"layer.moe_mlp.W_gate{i}": (torch.arange(real * 6, dtype=torch.float32).view(real, 2, 3) + 1)
                   .to(torch.bfloat16) for i, (real, _, _) in enumerate(CKPT_CASES)}
        save_file(tensors, path)
        for i, (real, shard, ep) in enumerate(CKPT_CASES):
            for rank in range(ep):
                ck.psm.get_world_size = lambda dim="", _e=ep: _e
                ck.psm.get_local_rank = lambda dim, _r=rank: _r
                ck._is_ep_sharded_key = lambda key: True
                key = f"layer.moe_mlp.W_gate{i}"
                with safe_open(path, framework="pt") as h:
                    got = ck._read_ep_slice(h, key, torch.empty(shard, 2, 3, dtype=torch.bfloat16))
                out[f"case{i}/rank{rank}"] = got.float().numpy()
            out[f"case{i}/meta"] = np.array([real, shard, ep], np.int64)
    np.savez_compressed(HERE / "ckpt_slices.npz", **out)
    print("ckpt_slices.npz:", len(CKPT_CASES), "cases")


if __name__ == "__main__":
    r = _import_reference()
    make_route(r)
    make_ffn(r)
    make_layer(_import_reference_model())
    make_ckpt()
