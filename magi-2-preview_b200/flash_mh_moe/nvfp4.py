"""NVFP4 packed expert weights (quantise on load) and per-row activation quantisation.

Format (identical to the CPU codec in ``oracle/nvfp4_ref.py``, which states the exact
op sequence): E2M1 values two per byte (low nibble = even k), one UE4M3 scale per 16
elements along K stored in 512-byte "SF atoms" (128 rows x 64 K-elements; row m,
scale column c at byte (m%32)*16 + (m//32)*4 + c; atoms K-fastest), and one fp32
second-level scale per expert matrix (amax/2688).

The reference has no NVFP4 weights (its experts are ``params_dtype`` bf16,
``inference/model/magi2_preview.py:2547-2570``); these containers hold the packed
form of those same parameters, built on the GPU by ``mhmoe_pack_weights_nvfp4``.

* ``NVFP4GateUp``: W_gate and W_up ([H*E, dh, de] reference layout) fused into one
  K-major operand [H*E, 2*de, dh/2]; rows interleave 16 gate rows and the 16
  matching up rows, so each 32-column accumulator chunk of the gate/up GEMM holds
  one 16-wide SwiGLU block.  gscale [2, H*E] (gate, up).
* ``NVFP4Down``: W_down ([H*E, de, dh]) as the K-major operand [H*E, dh, de/2].

Shapes the reference accepts but the tensor-core tiles do not (its kernel asserts only
``d_head % 64 == 0`` and ``d_expert % 32 == 0``, ``triton/mh_moe_fwd.py:264-265``) are packed
zero-padded to multiples of 256: ``d_head`` / ``d_expert`` hold the padded sizes and
``src_d_head`` / ``src_d_expert`` the caller's.  The padding is exact: zero weight rows and
columns contribute nothing to the accumulators, zero gate and up columns give a zero
SwiGLU7 output, and zero blocks leave the per-row and per-block scales of the real data
unchanged.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class NVFP4GateUp:
    data: torch.Tensor       # uint8 [n, 2*de, dh/2]
    sf: torch.Tensor         # uint8 [n, 2*de*dh/16]  (SF atoms per expert)
    gscale: torch.Tensor     # fp32 [2, n]
    num_experts: int         # flattened H*E
    d_head: int              # packed (multiple of 256)
    d_expert: int            # packed (multiple of 256)
    src_d_head: int | None = None
    src_d_expert: int | None = None

    @property
    def shape(self):  # reference W_gate shape
        return (self.num_experts, self.src_d_head or self.d_head, self.src_d_expert or self.d_expert)


@dataclass
class NVFP4Down:
    data: torch.Tensor       # uint8 [n, dh, de/2]
    sf: torch.Tensor         # uint8 [n, dh*de/16]
    gscale: torch.Tensor     # fp32 [n]
    num_experts: int
    d_head: int
    d_expert: int
    src_d_head: int | None = None
    src_d_expert: int | None = None

    @property
    def shape(self):  # reference W_down shape
        return (self.num_experts, self.src_d_expert or self.d_expert, self.src_d_head or self.d_head)


def _bf16c(w: torch.Tensor) -> torch.Tensor:
    return w.detach().to(torch.bfloat16).contiguous()


def padded(n: int) -> int:
    """The tile multiple (256) a head or expert dimension is packed at."""
    return (n + 255) // 256 * 256


def check_dims(dh: int, de: int) -> None:
    """The reference's shape contract (triton/mh_moe_fwd.py:264-265)."""
    assert dh % 64 == 0, f"d_head={dh} must be divisible by 64"
    assert de % 32 == 0, f"d_expert={de} must be divisible by 32"


def _pad_to(w: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    if w.shape[1] == rows and w.shape[2] == cols:
        return w
    return torch.nn.functional.pad(w, (0, cols - w.shape[2], 0, rows - w.shape[1]))


def pack_gate_up(W_gate: torch.Tensor, W_up: torch.Tensor) -> NVFP4GateUp:
    """Quantise reference-layout W_gate/W_up [n, dh, de] (any float dtype, via bf16)."""
    _lib.require_cuda(W_gate, W_up)
    if W_gate.shape != W_up.shape or W_gate.dim() != 3:
        raise ValueError(f"W_gate/W_up must both be [n, dh, de], got {tuple(W_gate.shape)}, {tuple(W_up.shape)}")
    n, dh0, de0 = W_gate.shape
    check_dims(dh0, de0)
    dh, de = padded(dh0), padded(de0)
    wg, wu = _pad_to(_bf16c(W_gate), dh, de), _pad_to(_bf16c(W_up), dh, de)
    dev = wg.device
    data = torch.empty(n, 2 * de, dh // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(n, 2 * de * dh // 16, dtype=torch.uint8, device=dev)
    gscale = torch.empty(2, n, dtype=torch.float32, device=dev)
    amax = torch.empty(2 * n, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mhmoe_pack_weights_nvfp4(0, wg.data_ptr(), wu.data_ptr(), n, dh, de, data.data_ptr(),
                                                        sf.data_ptr(), gscale.data_ptr(), amax.data_ptr(),
                                                        _lib.stream_ptr(dev)), "pack_gate_up")
    return NVFP4GateUp(data, sf, gscale, n, dh, de, dh0, de0)


def pack_down(W_down: torch.Tensor) -> NVFP4Down:
    """Quantise reference-layout W_down [n, de, dh]."""
    _lib.require_cuda(W_down)
    if W_down.dim() != 3:
        raise ValueError(f"W_down must be [n, de, dh], got {tuple(W_down.shape)}")
    n, de0, dh0 = W_down.shape
    check_dims(dh0, de0)
    dh, de = padded(dh0), padded(de0)
    wd = _pad_to(_bf16c(W_down), de, dh)
    dev = wd.device
    data = torch.empty(n, dh, de // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(n, dh * de // 16, dtype=torch.uint8, device=dev)
    gscale = torch.empty(n, dtype=torch.float32, device=dev)
    amax = torch.empty(n, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().mhmoe_pack_weights_nvfp4(1, wd.data_ptr(), None, n, dh, de, data.data_ptr(),
                                                        sf.data_ptr(), gscale.data_ptr(), amax.data_ptr(),
                                                        _lib.stream_ptr(dev)), "pack_down")
    return NVFP4Down(data, sf, gscale, n, dh, de, dh0, de0)


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-row NVFP4 of a bf16 [M, K] tensor: (data [M, K/2], sf atoms, gscale [M])."""
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("quantize_rows expects a bf16 [M, K] tensor with unit inner stride")
    M, K = x.shape
    Mp = (M + 127) // 128 * 128
    data = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
    sf = torch.zeros(Mp * K // 16, dtype=torch.uint8, device=x.device)
    g = torch.empty(M, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().mhmoe_quantize_rows_nvfp4(x.data_ptr(), x.stride(0), M, K, data.data_ptr(),
                                                         sf.data_ptr(), g.data_ptr(), _lib.stream_ptr(x.device)),
                   "quantize_rows")
    return data, sf, g
