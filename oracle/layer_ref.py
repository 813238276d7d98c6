"""numpy restatement of MAGI-2's MoE layer around the routed core.

Test infrastructure only (``tests/``).  Restates
``inference/model/magi2_preview.py``:

* ``MultiModalityRMSNorm`` (``:497-623``): per row, in fp32,
  ``x * rsqrt(mean(x^2) + eps) * (w[m] + 1)``, cast to the input dtype (bf16);
* ``swiglu7`` on the interleaved layout (``:86-98``): even columns gate, odd linear;
* ``MultiHeadMoELayer.forward`` (``:2797-2806``) and ``_shared_expert_forward``
  (``:2775-2795``) with bf16 activations between the linears, as the reference runs them.

``layer_ref`` is the reference itself (bf16 shared experts).  ``layer_nvfp4_ref`` is its
NVFP4 twin, the CUDA path's oracle: the shared experts on NVFP4 operands (norm output
quantised per row, the SwiGLU7 output with the static hidden scale; their two bf16
outputs summed in fp32 and rounded once, as the combine does), and the merge GEMM
accumulated onto the shared output in fp32 with one bf16 rounding.
"""
from __future__ import annotations

import numpy as np

from . import ffn_ref, nvfp4_ref as nv

bf = nv.bf16_round


def rmsnorm_ref(x, weight, group_sizes, eps: float = 1e-6, weight_bias: float = 1.0) -> np.ndarray:
    """x [S, d] (bf16 values); weight fp32 [M * d]; rows grouped by modality."""
    x = np.asarray(x, np.float32)
    S, d = x.shape
    w = np.asarray(weight, np.float32).reshape(-1, d)
    ms = (np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / d).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    t = (x * r).astype(np.float32)
    m = np.repeat(np.arange(len(group_sizes)), group_sizes)
    return bf((t * (w[m] + np.float32(weight_bias))).astype(np.float32))


def swiglu7_interleaved(x) -> np.ndarray:
    x = np.asarray(x, np.float32)
    return ffn_ref.swiglu7(x[..., 0::2], x[..., 1::2])


def linear(x, w) -> np.ndarray:
    """bf16 F.linear: fp32 accumulation of bf16 values, bf16 output."""
    return bf((np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32))


def shared_experts_ref(norm, group_sizes, fc1, fc2, fc1_m, fc2_m) -> np.ndarray:
    """_shared_expert_forward with bf16 linears (magi2_preview.py:2775-2795)."""
    M = len(group_sizes)
    d = norm.shape[1]
    x1 = linear(norm, fc1)
    starts = np.cumsum([0] + list(group_sizes))
    w1m = np.asarray(fc1_m).reshape(M, -1, d)
    w2m = np.asarray(fc2_m).reshape(M, d, -1)
    x2 = np.concatenate([linear(norm[starts[m]:starts[m + 1]], w1m[m]) for m in range(M)], axis=0)
    Is, Im = fc1.shape[0] // 2, w1m.shape[1] // 2
    act = bf(swiglu7_interleaved(np.concatenate([x1, x2], axis=-1)))
    a1, a2 = act[:, :Is], act[:, Is:Is + Im]
    y1 = linear(a1, fc2)
    y2 = np.concatenate([linear(a2[starts[m]:starts[m + 1]], w2m[m]) for m in range(M)], axis=0)
    return bf(y1 + y2)


def shared_experts_nvfp4_ref(norm, group_sizes, gu_pack: dict, dn_pack: dict) -> np.ndarray:
    """The shared experts as an NVFP4 expert set (expert 0 shared, 1 + m modality m), every
    token routed to its two experts with weight 1 (packs from the GPU or nvfp4_ref)."""
    S, d = norm.shape
    tok = np.arange(S, dtype=np.int32)
    gather_ids = np.concatenate([tok, tok])
    offs = np.array([0, S] + [S + v for v in np.cumsum(group_sizes)], np.int64)
    probs = np.ones(2 * S, np.float32)
    return ffn_ref.mh_moe_fwd_nvfp4_ref(np.asarray(norm, np.float32).reshape(S, 1, d), gather_ids, probs, offs,
                                        gu_pack, dn_pack).reshape(S, d)


def layer_nvfp4_ref(x, group_sizes, norm_w, w_split, w_merge, core, shared_gu, shared_dn,
                    eps: float = 1e-6) -> tuple[np.ndarray, np.ndarray]:
    """The CUDA layer's oracle.  ``core(moe_input) -> moe_out`` is the routed core's oracle
    (a callable, so a test can run it on the GPU's own router logits).  Returns
    (output, norm_output)."""
    norm = rmsnorm_ref(x, norm_w, group_sizes, eps)
    moe_out = core(linear(norm, w_split))
    shared = shared_experts_nvfp4_ref(norm, group_sizes, shared_gu, shared_dn)
    merged = (np.asarray(moe_out, np.float64) @ np.asarray(w_merge, np.float64).T).astype(np.float32)
    return bf((merged + shared).astype(np.float32)), norm
