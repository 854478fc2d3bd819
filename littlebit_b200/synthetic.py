"""Seeded synthetic LittleBit weights with the benchmark distributions.

Signs are i.i.d. Bernoulli(0.5) ±1 packed LSB-first (a uniformly random
32-bit word is exactly 32 such signs; pad bits are cleared to +1 as
binary_packer does), scales are |N(1, 0.1)|, dense bf16 weights N(0, 0.02).
Tensors are generated on the CPU with a torch.Generator (deterministic
across machines) and moved to the target device by the caller.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch


def sign_words(rows: int, cols: int, g: torch.Generator) -> torch.Tensor:
    wpr = (cols + 31) // 32
    w = torch.randint(-(2 ** 31), 2 ** 31, (rows, wpr), generator=g, dtype=torch.int64)
    if cols % 32:
        w[:, -1] &= (1 << (cols % 32)) - 1
    return w.to(torch.int32)


def abs_normal(n: int, g: torch.Generator, mean: float = 1.0, std: float = 0.1) -> torch.Tensor:
    return (mean + std * torch.randn(n, generator=g)).abs().to(torch.float32)


def branch(in_f: int, out_f: int, rank: int, g: torch.Generator, shared_v: bool = False) -> Dict:
    """One runtime-layout branch: v_sign, v2, mid, u_sign, u1 (CPU tensors)."""
    d = {"rank": rank}
    if shared_v:
        d["v_sign"], d["v2"] = None, None
    else:
        d["v_sign"] = sign_words(rank, in_f, g)
        d["v2"] = abs_normal(in_f, g)
    d["mid"] = abs_normal(rank, g)
    d["u_sign"] = sign_words(out_f, rank, g)
    d["u1"] = abs_normal(out_f, g)
    return d


def layer(in_f: int, out_f: int, ranks: List[int], g: torch.Generator,
          shared_residual: bool = False) -> List[Dict]:
    out = [branch(in_f, out_f, ranks[0], g)]
    for r in ranks[1:]:
        out.append(branch(in_f, out_f, r, g, shared_v=shared_residual))
    return out


def to_packed_linear(in_f: int, out_f: int, branches: List[Dict], device,
                     bias: Optional[torch.Tensor] = None):
    from .ops import Branch, PackedLinear

    bs = []
    for b in branches:
        mv = lambda t: None if t is None else t.to(device).contiguous()
        bs.append(Branch(mv(b["v_sign"]), mv(b["v2"]), mv(b["mid"]), mv(b["u_sign"]), mv(b["u1"]),
                         int(b["rank"])))
    return PackedLinear(in_f, out_f, bs, None if bias is None else bias.to(device))

