"""CPU: loading the MoE layers from a MAGI-2 safetensors checkpoint.

* The expert-parallel row rule equals the reference reader's (``_read_ep_slice``,
  inference/infra/checkpoint/magi2_checkpointing.py:81-105) on every rank of the golden
  cases, including zero-filled ranks past the real rows.
* ``load_moe_module`` reads this rank's rows of a two-shard checkpoint, the router whole,
  and substitutes the EMA router bias unless MAGI2_ROUTER_BIAS_SOURCE=main (:132-157).
  (NVFP4 packing on load needs the GPU: tests/test_gpu_checkpoint.py.)
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

GOLD = Path(__file__).resolve().parent / "golden"


def test_ep_row_rule_matches_reference(tmp_path):
    from safetensors import safe_open
    from safetensors.torch import save_file

    from flash_mh_moe.checkpoint import _read_rows, ep_rows
    g = np.load(GOLD / "ckpt_slices.npz")
    cases = sorted({k.split("/")[0] for k in g.files})
    for c in cases:
        real, shard, ep = (int(v) for v in g[c + "/meta"])
        path = tmp_path / f"{c}.safetensors"
        save_file({"t": (torch.arange(real * 6, dtype=torch.float32).view(real, 2, 3) + 1).to(torch.bfloat16)},
                  str(path))
        with safe_open(str(path), framework="pt") as h:
            for r in range(ep):
                got = _read_rows(h, "t", *ep_rows(real, shard, r, ep)).float().numpy()
                np.testing.assert_array_equal(got, g[f"{c}/rank{r}"], err_msg=f"{c} rank {r}")


def _cfg():
    from flash_mh_moe.moe import CoreMultiHeadMoEConfig
    return CoreMultiHeadMoEConfig(hidden_size=512, num_heads=2, num_experts=4, top_k=2, expert_intermediate_size=256,
                                  num_layers=1, params_dtype=torch.bfloat16)


def _write_checkpoint(d: Path, prefix: str):
    """A two-shard safetensors directory holding one MoE layer's full tensors."""
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(0)
    H, E, dh, de = 2, 4, 256, 256
    full = {
        "gate": torch.randn(H * E, dh, generator=g),
        "router.expert_bias": torch.randn(H * E, generator=g),
        "router.expert_bias_ema": torch.randn(H * E, generator=g),
        "W_gate": torch.randn(H * E, dh, de, generator=g).to(torch.bfloat16),
        "W_up": torch.randn(H * E, dh, de, generator=g).to(torch.bfloat16),
        "W_down": torch.randn(H * E, de, dh, generator=g).to(torch.bfloat16),
    }
    shards = {"a.safetensors": ["gate", "W_gate", "router.expert_bias"],
              "b.safetensors": ["W_up", "W_down", "router.expert_bias_ema"]}
    wm = {}
    for f, names in shards.items():
        save_file({prefix + n: full[n].contiguous() for n in names}, str(d / f))
        wm.update({prefix + n: f for n in names})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    return full


@pytest.mark.parametrize("bias_source", ["ema", "main"])
def test_load_moe_module_ep_slices(tmp_path, monkeypatch, bias_source):
    from test_module_registry import _FakePsm, _with_psm

    from flash_mh_moe import checkpoint, moe
    prefix = "blocks.2.mlp.moe_mlp."
    full = _write_checkpoint(tmp_path, prefix)
    monkeypatch.setenv("MAGI2_ROUTER_BIAS_SOURCE", bias_source)
    for rank in range(2):
        _with_psm(monkeypatch, _FakePsm(2, rank, object()))
        m = moe.CoreMultiHeadMoE(_cfg())
        ranges = checkpoint.load_moe_module(m, str(tmp_path), prefix, quantize=False)
        lo, hi = rank * 4, rank * 4 + 4                      # 8 flattened experts over 2 ranks
        assert ranges[prefix + "W_gate"] == (lo, hi, 0)
        for n in ("W_gate", "W_up", "W_down"):
            assert torch.equal(getattr(m, n), full[n][lo:hi]), n
        assert torch.equal(m.gate, full["gate"])                            # router replicated
        assert torch.equal(m.router.expert_bias_ema, full["router.expert_bias_ema"])
        want_bias = full["router.expert_bias_ema" if bias_source == "ema" else "router.expert_bias"]
        assert torch.equal(m.router.expert_bias, want_bias)
