"""CPU model of the decode kernel's top-k selection, checked against the oracle's rule.

The kernel (``routing_prologue`` in ``csrc/nkm_qwen3_kernel.cuh``) gives lane l of a warp the
experts e = 32 q + l, turns each logit into an order-preserving uint32 key (-0 folded into +0),
sorts every lane's keys with an odd-even transposition sort that swaps only strictly smaller
neighbours, and then takes K picks: the largest head key over the warp, the lowest expert index
among equal heads, and a pop of the owning lane's head.  This test restates that scheme in
Python and checks that it selects exactly what the oracle's ``topk_select`` selects (descending
logits, ties toward the lower expert index, ``moe_fused_nki.py:241-250``), in the same order, on
random logits with many exact ties and signed zeros.  The GPU tests check the kernel itself.
"""
import struct

import pytest
import torch

from oracle import qwen3_moe_oracle as O


def _order_key(f: float) -> int:
    u = struct.unpack("<I", struct.pack("<f", 0.0 if f == 0.0 else f))[0]
    return (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)


def _kernel_topk(row, k):
    E = len(row)
    per = (E + 31) // 32
    lanes = []
    for lane in range(32):
        keys, qs = [], []
        for q in range(8):
            e = 32 * q + lane
            ok = q < per and e < E
            keys.append(_order_key(float(row[e])) if ok else 0)
            qs.append(q)
        for r in range(8):  # odd-even transposition, strict swaps only
            for a in range(r & 1, 7, 2):
                if keys[a + 1] > keys[a]:
                    keys[a], keys[a + 1] = keys[a + 1], keys[a]
                    qs[a], qs[a + 1] = qs[a + 1], qs[a]
        lanes.append([keys, qs])
    picks = []
    for _ in range(k):
        wmax = max(l[0][0] for l in lanes)
        bi = min(l[1][0] * 32 + lane for lane, l in enumerate(lanes) if l[0][0] == wmax)
        own = lanes[bi & 31]
        own[0] = own[0][1:] + [0]
        own[1] = own[1][1:] + [own[1][-1]]
        picks.append(bi)
    return picks


@pytest.mark.parametrize("E", [128, 256, 96, 64])
def test_kernel_topk_scheme_matches_oracle(E):
    g = torch.Generator().manual_seed(E)
    K = 8
    for trial in range(40):
        if trial % 3 == 0:
            row = torch.randn(E, generator=g)
        else:  # coarse values: many exact ties, and signed zeros
            row = torch.randint(-3, 4, (E,), generator=g).float() * 0.5
            zero = torch.rand(E, generator=g) < 0.2
            row[zero] = torch.where(torch.rand(E, generator=g)[zero] < 0.5, torch.tensor(-0.0), torch.tensor(0.0))
        want = O.topk_select(row[None, :], K)[0].tolist()
        assert _kernel_topk(row.tolist(), K) == want, (trial, row.tolist())
