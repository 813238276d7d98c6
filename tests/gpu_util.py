"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

from oracle import nvfp4_ref as nv


def bf16_tensor(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(torch.bfloat16)


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.detach().cpu().numpy()


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def seeded_moe(S, H, dh, de, E, K, seed, skew=False, score="softmax"):
    """Seeded layer inputs in the benchmark's distributions (x N(0,1), gate N(0,0.02) bf16,
    expert weights N(0,0.02)), as numpy fp32 values (bf16-exact where the reference is bf16)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(S, H * dh, generator=g).to(torch.bfloat16).float().numpy()
    gate = (torch.randn(H * E, dh, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    Wg = (torch.randn(H * E, dh, de, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    Wu = (torch.randn(H * E, dh, de, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    Wd = (torch.randn(H * E, de, dh, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    return x, gate, Wg, Wu, Wd
