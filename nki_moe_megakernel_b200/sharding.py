"""Tensor + expert parallel layout of the decode step across the GPUs of one node.

One process per GPU.  Attention is split over KV-head groups: with N <= n_kv_heads ranks,
rank r holds KV heads [r * nkv / N, (r + 1) * nkv / N) and their query heads; with more ranks
than KV heads (N = 8 for 4 KV heads) the ranks of a KV head share it and split its query
heads.  The O-projection of a rank covers its query heads only, so its output is a partial
sum.  Experts are split into N contiguous ranges (expert parallel); the router, the norms,
the embedding and the LM head are replicated.  Inside the decode kernel every rank stores
its partial sums into the exchange region of every rank and all ranks add them in rank order
(``include/nkimoe.h``: ``n_ranks``, ``xchg``), so the residual streams stay identical.

This replaces the reference's TP/EP configuration of the NxDI model (replica groups of
``megakernels/qwen3_moe/qwen_with_megakernel.py:360-362``, ``moe_ep_degree`` of the neuron
config) for this path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch


@dataclass(frozen=True)
class RankShard:
    rank: int
    world: int
    q_heads: List[int]       # global query heads held by this rank
    kv_heads: List[int]      # global KV heads held by this rank
    expert_begin: int
    n_local_experts: int


def plan_shard(rank: int, world: int, n_q_heads: int, n_kv_heads: int, n_experts: int) -> RankShard:
    """Heads and experts of one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if n_experts % world:
        raise ValueError("n_experts must be a multiple of the number of ranks")
    grp = n_q_heads // n_kv_heads
    if world <= n_kv_heads:
        if n_kv_heads % world:
            raise ValueError("n_kv_heads must be a multiple of the number of ranks")
        per = n_kv_heads // world
        kv = list(range(rank * per, (rank + 1) * per))
        q = [h * grp + j for h in kv for j in range(grp)]
    else:
        if world % n_kv_heads:
            raise ValueError("the number of ranks must be a multiple of n_kv_heads")
        share = world // n_kv_heads           # ranks per KV head
        if grp % share:
            raise ValueError("query heads per KV head must split evenly over the ranks that share it")
        h = rank // share
        qs = grp // share
        kv = [h]
        q = [h * grp + (rank % share) * qs + j for j in range(qs)]
    ne = n_experts // world
    return RankShard(rank, world, q, kv, rank * ne, ne)


def _rows(w: torch.Tensor, heads: List[int], head_dim: int) -> torch.Tensor:
    return torch.cat([w[h * head_dim:(h + 1) * head_dim] for h in heads], 0)


def shard_attention(wq, wk, wv, wo, shard: RankShard, head_dim: int):
    """Local (wq, wk, wv, wo): query/key/value rows of the rank's heads, O-projection columns of
    its query heads."""
    wo_l = torch.cat([wo[:, h * head_dim:(h + 1) * head_dim] for h in shard.q_heads], 1)
    return _rows(wq, shard.q_heads, head_dim), _rows(wk, shard.kv_heads, head_dim), \
        _rows(wv, shard.kv_heads, head_dim), wo_l.contiguous()


def shard_experts(gate_up: torch.Tensor, down: torch.Tensor, shard: RankShard):
    """The rank's experts of ``gate_up [E, 2I, H]`` and ``down [E, H, I]``."""
    sl = slice(shard.expert_begin, shard.expert_begin + shard.n_local_experts)
    return gate_up[sl].contiguous(), down[sl].contiguous()


def xchg_bytes(hidden: int, max_batch: int, world: int, vocab: int) -> int:
    """Bytes of one rank's exchange region (``nkm_qwen3_xchg_bytes``): a 256-byte header (the
    cross-GPU barrier counter), the partials as tagged 8-byte words [2][2][world][max_batch][hidden]
    and, with several ranks, the fp32 logits [max_batch][vocab] of the vocabulary-sharded LM head."""
    n = (256 + 4 * world * max_batch * hidden * 8 + 255) // 256 * 256
    if world > 1:
        n += max_batch * vocab * 4
    return (n + 255) // 256 * 256


class XchgRegion:
    """The exchange region of this rank (``nkm_qwen3_xchg_bytes``), allocated with cudaMalloc
    and shared with the other ranks by CUDA IPC; ``ptrs[q]`` is rank q's region mapped in this
    process.  The handles travel over ``group`` (any torch.distributed backend, gloo works)."""

    def __init__(self, nbytes: int, rank: int, world: int, device: int, group=None):
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart  # noqa: PLC0415

        self._cudart = cudart
        self.rank, self.world, self.nbytes = rank, world, nbytes
        torch.cuda.set_device(device)
        err, ptr = cudart.cudaMalloc(nbytes)
        _check(err, "cudaMalloc")
        _check(cudart.cudaMemset(ptr, 0, nbytes)[0], "cudaMemset")
        _check(cudart.cudaDeviceSynchronize()[0], "cudaDeviceSynchronize")
        self.own = int(ptr)
        err, handle = cudart.cudaIpcGetMemHandle(ptr)
        _check(err, "cudaIpcGetMemHandle")
        handles: List[Optional[bytes]] = [None] * world
        dist.all_gather_object(handles, bytes(handle.reserved), group=group)
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        for q, hb in enumerate(handles):
            if q == rank:
                self.ptrs.append(self.own)
                continue
            h = cudart.cudaIpcMemHandle_t()
            h.reserved = hb
            err, peer = cudart.cudaIpcOpenMemHandle(h, cudart.cudaIpcMemLazyEnablePeerAccess)
            _check(err, f"cudaIpcOpenMemHandle(rank {q})")
            self.ptrs.append(int(peer))
            self._opened.append(int(peer))

    def close(self):
        for p in self._opened:
            self._cudart.cudaIpcCloseMemHandle(p)
        self._opened = []
        if self.own:
            self._cudart.cudaFree(self.own)
            self.own = 0


def _check(err, what):
    code = int(err) if not isinstance(err, tuple) else int(err[0])
    if code != 0:
        raise RuntimeError(f"{what} failed with CUDA error {code}")


def shard_gptoss_layer(t: dict, shard: RankShard, head_dim: int) -> dict:
    """The rank's part of one GPT-OSS layer (the tensor names of ``GptOssGpuLayer``): query,
    key and value rows and biases of its heads, O-projection columns and sink logits of its query
    heads, and its experts' MXFP4 codes, scales and biases.  Norms and router stay whole."""
    o = dict(t)
    o["wq"], o["wk"], o["wv"], o["wo"] = shard_attention(t["wq"], t["wk"], t["wv"], t["wo"], shard, head_dim)
    o["bq"] = _rows(t["bq"], shard.q_heads, head_dim)
    o["bk"] = _rows(t["bk"], shard.kv_heads, head_dim)
    o["bv"] = _rows(t["bv"], shard.kv_heads, head_dim)
    o["sinks"] = t["sinks"][torch.tensor(shard.q_heads, device=t["sinks"].device)].contiguous()
    sl = slice(shard.expert_begin, shard.expert_begin + shard.n_local_experts)
    for k in ("gu_codes", "gu_scales", "gu_b", "dn_codes", "dn_scales", "dn_b"):
        o[k] = t[k][sl].contiguous()
    return o


def gptoss_xchg_bytes(hidden: int, max_batch: int, world: int, vocab: int) -> int:
    """Bytes of one rank's GPT-OSS exchange region (``nkm_gptoss_xchg_bytes``): a 256-byte
    header, the partials as tagged 8-byte words [2 kinds][2 slots][world][max_batch][hidden] and,
    with several ranks, the logits as tagged words [2 slots][max_batch][vocab]."""
    a = lambda n: (n + 255) // 256 * 256  # noqa: E731
    n = a(256 + 4 * world * max_batch * hidden * 8)
    if world > 1:
        n += 2 * max_batch * vocab * 8
    return a(n)
