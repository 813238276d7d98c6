"""CPU: the module registry behind the opaque op (keyed by a stable integer, reference
op ``infra::magi2_mh_moe``) hands out unique keys and does not keep modules alive."""
import gc

import torch


def _cfg():
    from flash_mh_moe.moe import CoreMultiHeadMoEConfig
    return CoreMultiHeadMoEConfig(hidden_size=256, num_heads=1, num_experts=4, top_k=2,
                                  expert_intermediate_size=256, num_layers=1, params_dtype=torch.bfloat16)


def test_keys_unique_and_weak():
    from flash_mh_moe import moe
    a = moe.CoreMultiHeadMoE(_cfg())
    b = moe.CoreMultiHeadMoE(_cfg())
    assert a._moe_key != b._moe_key
    assert moe._magi2_moe_registry[a._moe_key] is a
    ka = a._moe_key
    del a
    gc.collect()
    assert ka not in moe._magi2_moe_registry          # the registry did not keep it alive
    c = moe.CoreMultiHeadMoE(_cfg())
    assert c._moe_key not in (ka, b._moe_key)         # keys are never reused
