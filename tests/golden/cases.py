"""Seeded input cases shared by the golden-fixture generator and the tests.

Inputs follow the reference's own test recipe (tests/test_attention.py:16-18): a CPU
``torch.Generator().manual_seed(seed)``, ``randn`` in fp32, then a cast to the case dtype.
``layout="bnhd"`` builds a ``[B, N, H, D]`` tensor and transposes it to ``[B, H, N, D]``
(non-contiguous), as BASELINE config 4 and tests/test_attention.py:57-64 do.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Case:
    name: str
    shape: tuple[int, int, int, int]  # [B, H, N, D]
    dtype: str  # "float16" | "float32"
    causal: bool
    seeds: tuple[int, int, int, int]  # q, k, v, dO
    layout: str = "bhnd"  # or "bnhd" (transposed, non-contiguous)
    sm_scale: float | None = None


# BASELINE config 1 plus a subset of the config-4 edge sweep (ragged N, small and large D,
# both dtypes, causal and not, non-contiguous).
CASES: dict[str, Case] = {
    c.name: c
    for c in (
        Case("cfg1_fp32_b1h2n256d64", (1, 2, 256, 64), "float32", False, (1, 2, 3, 4)),
        Case("edge_fp16_d16_n17_causal", (3, 5, 17, 16), "float16", True, (11, 12, 13, 14), "bnhd"),
        Case("edge_fp32_d32_n33", (3, 5, 33, 32), "float32", False, (21, 22, 23, 24), "bnhd"),
        Case("edge_fp16_d64_n70_causal", (3, 5, 70, 64), "float16", True, (31, 32, 33, 34), "bnhd"),
        Case("edge_fp32_d64_n1_causal", (3, 5, 1, 64), "float32", True, (41, 42, 43, 44), "bnhd"),
        Case("edge_fp16_d32_n1", (3, 5, 1, 32), "float16", False, (51, 52, 53, 54), "bnhd"),
        Case("edge_fp32_d16_n70_causal", (3, 5, 70, 16), "float32", True, (61, 62, 63, 64), "bnhd"),
        Case("hd128_fp16_n19_causal", (1, 1, 19, 128), "float16", True, (30, 31, 32, 33)),
        Case("scale03_fp32_n20_d32", (1, 2, 20, 32), "float32", False, (9, 10, 11, 12), "bnhd", 0.3),
    )
}


def make_tensor(case: Case, seed: int) -> torch.Tensor:
    b, h, n, d = case.shape
    g = torch.Generator().manual_seed(seed)
    dt = getattr(torch, case.dtype)
    if case.layout == "bnhd":
        return torch.randn((b, n, h, d), generator=g, dtype=torch.float32).to(dt).transpose(1, 2)
    return torch.randn((b, h, n, d), generator=g, dtype=torch.float32).to(dt)


def make_inputs(case: Case) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q, k, v, dO) on the CPU, in the case's dtype and layout."""
    q, k, v, do = (make_tensor(case, s) for s in case.seeds)
    return q, k, v, do


def digest(t: torch.Tensor) -> str:
    """Stable fingerprint of a tensor's values (in logical [B,H,N,D] order)."""
    a = np.ascontiguousarray(t.detach().cpu().numpy())
    return hashlib.sha256(a.tobytes()).hexdigest()[:16]
