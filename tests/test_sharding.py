"""CPU tests of the tensor + expert parallel layout (``nki_moe_megakernel_b200.sharding``).

The decomposition the kernel relies on is checked with the oracle on ``gloo`` ranks: every
rank evaluates its attention heads (O-projection partial) and its experts (MoE partial), the
partials are summed across ranks, and the result equals the unsharded decoder layer.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nki_moe_megakernel_b200.sharding import plan_shard, shard_attention, shard_experts
from oracle import qwen3_moe_oracle as O


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_heads_and_experts(world):
    nq, nkv, E = 32, 4, 128
    shards = [plan_shard(r, world, nq, nkv, E) for r in range(world)]
    q_all = sorted(h for s in shards for h in s.q_heads)
    assert q_all == list(range(nq))
    for s in shards:
        assert len(s.q_heads) == nq // world
        grp = nq // nkv
        assert all(h // grp in s.kv_heads for h in s.q_heads)  # every query head sees its KV head
    kv_all = sorted({h for s in shards for h in s.kv_heads})
    assert kv_all == list(range(nkv))
    ex = [(s.expert_begin, s.n_local_experts) for s in shards]
    assert ex[0][0] == 0 and all(a + n == b for (a, n), (b, _) in zip(ex, ex[1:])) and sum(n for _, n in ex) == E


def test_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        plan_shard(0, 3, 32, 4, 128)
    with pytest.raises(ValueError):
        plan_shard(0, 2, 32, 4, 127)


def test_shard_weights_slices():
    D = 128
    s = plan_shard(1, 2, 4, 2, 8)
    wq = torch.arange(4 * D * 3, dtype=torch.float32).view(4 * D, 3)
    wk = torch.arange(2 * D * 3, dtype=torch.float32).view(2 * D, 3)
    wo = torch.arange(3 * 4 * D, dtype=torch.float32).view(3, 4 * D)
    q, k, v, o = shard_attention(wq, wk, wk, wo, s, D)
    assert torch.equal(q, wq[2 * D:]) and torch.equal(k, wk[D:]) and torch.equal(o, wo[:, 2 * D:])
    gu = torch.arange(8 * 2).view(8, 2, 1)
    dn = torch.arange(8 * 3).view(8, 3, 1)
    g, d = shard_experts(gu, dn, s)
    assert torch.equal(g, gu[4:]) and torch.equal(d, dn[4:])


@pytest.mark.parametrize("world", [2, 8])
def test_gptoss_layer_shards_cover_the_layer(world):
    """GPT-OSS (64 query / 8 KV heads of 64, 32 experts): the ranks' query/key/value rows and
    biases, O-projection columns, sinks and experts put back together give the whole layer, and
    each rank's query heads are the ones of its KV heads."""
    from nki_moe_megakernel_b200.sharding import shard_gptoss_layer

    D, H, E = 64, 4, 32
    g = torch.Generator().manual_seed(0)
    t = {"wq": torch.randn(64 * D, H, generator=g), "bq": torch.randn(64 * D, generator=g),
         "wk": torch.randn(8 * D, H, generator=g), "bk": torch.randn(8 * D, generator=g),
         "wv": torch.randn(8 * D, H, generator=g), "bv": torch.randn(8 * D, generator=g),
         "wo": torch.randn(H, 64 * D, generator=g), "sinks": torch.randn(64, generator=g),
         "ln1": torch.randn(H, generator=g)}
    for k in ("gu_codes", "gu_scales", "gu_b", "dn_codes", "dn_scales", "dn_b"):
        t[k] = torch.randn(E, 3, generator=g)
    parts = [shard_gptoss_layer(t, plan_shard(r, world, 64, 8, E), D) for r in range(world)]
    for k in ("wq", "bq", "wk", "bk", "wv", "bv", "sinks", "gu_codes", "gu_scales", "gu_b", "dn_codes", "dn_scales",
              "dn_b"):
        assert torch.equal(torch.cat([p[k] for p in parts], 0), t[k]), k
    assert torch.equal(torch.cat([p["wo"] for p in parts], 1), t["wo"])
    assert all(torch.equal(p["ln1"], t["ln1"]) for p in parts)
    for r, p in enumerate(parts):
        s = plan_shard(r, world, 64, 8, E)
        assert s.q_heads == [h * 8 + j for h in s.kv_heads for j in range(8)]
        assert p["wq"].shape[0] == len(s.q_heads) * D and p["gu_codes"].shape[0] == E // world


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank_layer(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    cfg = O.QwenConfig(hidden=256, n_q_heads=8, n_kv_heads=2, n_experts=8, top_k=2, moe_inter=32, n_layers=1)
    gen = torch.Generator().manual_seed(1)
    lw = O.random_layer(cfg, gen)
    B, positions, NB = 3, [5, 40, 130], 8
    pos = torch.tensor(positions, dtype=torch.int32)
    table = torch.zeros(B, 2, dtype=torch.int32)
    table[:, 0] = torch.tensor([0, 1, 2], dtype=torch.int32)
    table[:, 1] = torch.tensor([3, 4, 5], dtype=torch.int32)
    kc = torch.randn(NB, cfg.n_kv_heads, 128, cfg.head_dim, generator=gen).to(torch.bfloat16)
    vc = torch.randn(NB, cfg.n_kv_heads, 128, cfg.head_dim, generator=gen).to(torch.bfloat16)
    x = torch.randn(B, cfg.hidden, generator=gen).to(torch.bfloat16)
    cos, sin = O.rope_tables(4096, cfg.head_dim, cfg.rope_theta, torch.float32)
    # this rank: heads and experts
    s = plan_shard(rank, world, cfg.n_q_heads, cfg.n_kv_heads, cfg.n_experts)
    wq, wk, wv, wo = shard_attention(lw.wq, lw.wk, lw.wv, lw.wo, s, cfg.head_dim)
    lcfg = O.QwenConfig(**{**cfg.__dict__, "n_q_heads": len(s.q_heads), "n_kv_heads": len(s.kv_heads)})
    llw = O.LayerWeights(**{**lw.__dict__, "wq": wq, "wk": wk, "wv": wv, "wo": wo})
    xn1 = O.rmsnorm_fp32(x.float(), lw.ln1, cfg.rms_eps)
    o = O.attention_layer(xn1, llw, lcfg, kc[:, s.kv_heads].clone(), vc[:, s.kv_heads].clone(), pos, table, cos, sin,
                          "fp32")
    dist.all_reduce(o)
    mid = x.float() + o
    xn2 = O.rmsnorm_fp32(mid, lw.ln2, cfg.rms_eps)
    logits = xn2 @ lw.router.float().t()
    idx, w = O.router_topk(logits, cfg.top_k, "fp32")
    local = (idx >= s.expert_begin) & (idx < s.expert_begin + s.n_local_experts)
    moe = O.experts_forward(xn2, idx, w * local, lw.gate_up, lw.down, "fp32")
    dist.all_reduce(moe)
    out = mid + moe
    if rank == 0:
        ref = O.decoder_layer(x, lw, cfg, kc.clone(), vc.clone(), pos, table, cos, sin, "fp32")
        torch.save({"out": out, "ref": ref}, out_path)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_partial_sums_equal_unsharded_layer(tmp_path, world):
    path = str(tmp_path / "res.pt")
    mp.spawn(_rank_layer, args=(world, _free_port(), path), nprocs=world, join=True)
    r = torch.load(path)
    assert (r["out"] - r["ref"]).abs().max().item() < 1e-4
