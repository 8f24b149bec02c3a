"""CPU oracle of the on-device token sampler (``nkm_sample_logits``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``; the product path never imports it.

Restates the sampler's semantics in plain Python / torch: the ``top_k`` largest logits of a row
(descending; equal logits ordered by lower token id, -0 equal to +0), logits times
``fp32(1 / temperature)``, a softmax over the k relative to the largest, the shortest prefix
whose probability mass reaches ``top_p``, and an inverse-CDF draw with the row's uniform
``u = top 24 bits of SplitMix64(SplitMix64(seed) ^ (position << 32 | row)) / 2^24``.  SplitMix64 is the
published generator of Steele, Lea and Flood (OOPSLA 2014).  The reference's sampler is NxDI's
on-device sampler configured at ``megakernels/qwen3_moe/qwen_with_megakernel.py:123-127``
(``global_topk`` capped to ``top_k``) and ``main.py:390-398``; it is not in the reference tree,
so the semantics above (Hugging Face's top-k / top-p warpers applied in that order) are the
ones restated.
"""
from __future__ import annotations

from typing import Tuple

import numpy as np
import torch

_M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M64
    return x ^ (x >> 31)


def uniform(seed: int, position: int, row: int) -> float:
    r = splitmix64(splitmix64(seed & _M64) ^ (((position & 0xFFFFFFFF) << 32) | (row & 0xFFFFFFFF)))
    return float(np.float32(r >> 40) * np.float32(1.0 / 16777216.0))


def topk_ids(logits_row: torch.Tensor, k: int) -> torch.Tensor:
    """The k largest logits' token ids, descending, equal values by lower id."""
    l = logits_row.float().clone()
    l[l == 0] = 0.0
    return torch.sort(l, descending=True, stable=True).indices[:k]


def sample_row(logits_row: torch.Tensor, top_k: int, top_p: float, temperature: float, seed: int,
               position: int, row: int) -> Tuple[int, float]:
    """(token, margin): ``margin`` is the smaller of the draw's distance from the nearest CDF
    boundary (relative to the kept mass) and the top-p test's distance from ``top_p`` (1.0 for
    greedy), so a caller can tell a draw that fp32 rounding of the softmax may flip from one it
    may not."""
    ids = topk_ids(logits_row, top_k)
    if top_k == 1:
        return int(ids[0]), 1.0
    f32 = np.float32
    inv_t = f32(1.0) / f32(temperature)
    z = [f32(float(logits_row[i])) * inv_t for i in ids.tolist()]
    e = [f32(np.exp(f32(v - z[0]))) for v in z]
    s = f32(0.0)
    for v in e:
        s = f32(s + v)
    keep, acc, p_margin = len(e), f32(0.0), float("inf")
    for j, v in enumerate(e):
        acc = f32(acc + f32(v / s))
        p_margin = min(p_margin, abs(float(acc) - top_p))
        if acc >= f32(top_p):
            keep = j + 1
            break
    mass = f32(0.0)
    for v in e[:keep]:
        mass = f32(mass + v)
    target = f32(f32(uniform(seed, position, row)) * mass)
    cum, pick, margin = f32(0.0), keep - 1, float("inf")
    for j in range(keep):
        cum = f32(cum + e[j])
        margin = min(margin, abs(float(cum) - float(target)) / float(mass))
        if target < cum:
            pick = j
            break
    return int(ids[pick]), min(margin, p_margin)
