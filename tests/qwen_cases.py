"""Seeded synthetic Qwen3-MoE cases shared by the GPU parity tests, smoke() and bench.

Weights ~N(0, 0.02) bf16, norm weights ~1+N(0, 0.02), hidden ~N(0, 1), KV prefix ~N(0, 1)
(the distributions of the benchmark configurations).  KV slots that hold no context are
filled with NaN so that any read of them would poison the output.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from oracle import qwen3_moe_oracle as O

BF16 = torch.bfloat16


def qwen_cfg(**kw) -> O.QwenConfig:
    return O.QwenConfig(**kw)


def make_layers(cfg: O.QwenConfig, n_distinct: int, seed: int) -> List[O.LayerWeights]:
    gen = torch.Generator().manual_seed(seed)
    return [O.random_layer(cfg, gen) for _ in range(n_distinct)]


def skew_bias(cfg: O.QwenConfig, hot: Sequence[int] = (3, 17, 64, 101), value: float = 4.0) -> torch.Tensor:
    """Router bias that sends about half of all top-k slots to 4 hot experts."""
    b = torch.zeros(cfg.n_experts, dtype=torch.float32)
    for e in hot:
        b[e % cfg.n_experts] = value
    return b


def make_kv(cfg: O.QwenConfig, n_layers: int, positions: Sequence[int], num_blocks: int, seed: int,
            nan_fill: bool = True):
    """Paged K/V pools ``[L, NB, nkv, 128, 128]`` bf16 (CPU) and a shuffled block table.

    Sequence ``b`` owns ``ceil((pos_b+1)/128)`` blocks; tokens ``0..pos_b-1`` hold N(0,1) values.
    """
    gen = torch.Generator().manual_seed(seed)
    B = len(positions)
    need = [p // cfg.block_size + 1 for p in positions]
    assert sum(need) <= num_blocks, (need, num_blocks)
    maxb = max(need)
    perm = torch.randperm(num_blocks, generator=gen)
    table = torch.full((B, maxb), -1, dtype=torch.int32)
    nxt = 0
    for b in range(B):
        for j in range(need[b]):
            table[b, j] = int(perm[nxt])
            nxt += 1
    shape = (n_layers, num_blocks, cfg.n_kv_heads, cfg.block_size, cfg.head_dim)
    fill = float("nan") if nan_fill else 0.0
    k = torch.full(shape, fill, dtype=BF16)
    v = torch.full(shape, fill, dtype=BF16)
    for b, p in enumerate(positions):
        for t0 in range(0, p, cfg.block_size):
            n = min(cfg.block_size, p - t0)
            blk = int(table[b, t0 // cfg.block_size])
            k[:, blk, :, :n] = torch.randn(n_layers, cfg.n_kv_heads, n, cfg.head_dim, generator=gen).to(BF16)
            v[:, blk, :, :n] = torch.randn(n_layers, cfg.n_kv_heads, n, cfg.head_dim, generator=gen).to(BF16)
    return k, v, table


def gpu_layers(layers: Sequence[O.LayerWeights], device, attention=True, moe=True,
               router_bias: Optional[torch.Tensor] = None):
    from nki_moe_megakernel_b200.engine import GpuLayer

    out = []
    for lw in layers:
        d = {k: getattr(lw, k).to(device) for k in ("wq", "wk", "wv", "wo", "q_norm", "k_norm", "ln1", "ln2",
                                                     "router", "gate_up", "down")}
        out.append(GpuLayer(d["wq"], d["wk"], d["wv"], d["wo"], d["q_norm"], d["k_norm"], d["ln1"], d["ln2"],
                            d["router"], d["gate_up"], d["down"],
                            router_bias=None if router_bias is None else router_bias.to(device),
                            attention=attention, moe=moe))
    return out


def shape_of(cfg: O.QwenConfig, n_layers: int, vocab: int):
    from nki_moe_megakernel_b200.engine import Qwen3MoeShape

    return Qwen3MoeShape(hidden_size=cfg.hidden, num_attention_heads=cfg.n_q_heads,
                         num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, num_experts=cfg.n_experts,
                         num_experts_per_tok=cfg.top_k, moe_intermediate_size=cfg.moe_inter,
                         num_hidden_layers=n_layers, vocab_size=vocab, rms_norm_eps=cfg.rms_eps,
                         rope_theta=cfg.rope_theta, block_size=cfg.block_size)


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality of two bf16 tensors (NaN payloads included)."""
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))
