#!/usr/bin/env python
"""Benchmark: the full Qwen3-30B-A3B decode step (48 layers + final norm + LM head) at
batch 8, context 2048 (paged KV, block 128), bf16, through the sm_100a megakernel.

Prints ONE JSON line (rank 0).  ``--impl reference`` times the CPU restatement of the
reference's decode path (the oracle, on the host cores) on the same configuration.

Inputs: seeded random-init weights of the Qwen3-30B-A3B architecture (no checkpoints in this
environment), a KV prefix ~N(0,1).  The weights streamed per step (~27 GB) are far larger
than L2 (126 MB), so no L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-30B-A3B decode tokens/s and p50 ms/step at B=8 ctx 2048; % HBM roofline"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--stage-times", action="store_true", help="print a per-stage time breakdown to stderr")
    ap.add_argument("--gptoss-layers", type=int, default=24,
                    help="gpt-oss workload: decoder layers (24 = GPT-OSS-20B; fewer for small profiling cases)")
    ap.add_argument("--weights", choices=["bf16", "mxfp8"], default="bf16",
                    help="expert weights of the tcgen05 workloads (moe-tc, wide): bf16 or MXFP8")
    ap.add_argument("--workload", choices=["qwen3", "gpt-oss", "moe-tc", "wide"], default="qwen3",
                    help="qwen3: the headline (config 2); gpt-oss: GPT-OSS-20B decode (config 4, B=16 ctx 4096); "
                         "moe-tc: the tcgen05 MoE block at config 3's 64 tokens; wide: config 3's whole decode "
                         "step at B=64 on one GPU")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------- model build
def build_engine(args, device, seed, shard=None, xchg=None):
    """Seeded random-init model of the bench shape.  With ``shard`` (tensor + expert parallel
    rank) the replicated tensors (norms, router, embedding, LM head) come from the same seed on
    every rank and the rank's heads and experts from a rank-specific one."""
    import torch

    from nki_moe_megakernel_b200.engine import GpuLayer, Qwen3MoeMegakernel, Qwen3MoeShape

    full = Qwen3MoeShape(num_hidden_layers=args.layers)
    H, D, E, I = full.hidden_size, full.head_dim, full.num_experts, full.moe_intermediate_size
    nq, nkv, V = full.num_attention_heads, full.num_key_value_heads, full.vocab_size
    if shard is not None:
        nq, nkv, El = len(shard.q_heads), len(shard.kv_heads), shard.n_local_experts
    else:
        El = E
    shape = Qwen3MoeShape(num_hidden_layers=args.layers, num_attention_heads=nq, num_key_value_heads=nkv)
    g = torch.Generator(device=device).manual_seed(seed)                       # replicated tensors
    gl = torch.Generator(device=device).manual_seed(seed + 1000 + (shard.rank if shard else 0))  # this rank's

    def n(*s, gen=g):
        return (torch.randn(*s, generator=gen, device=device) * 0.02).to(torch.bfloat16)

    def one(*s, gen=g):
        return (1.0 + torch.randn(*s, generator=gen, device=device) * 0.02).to(torch.bfloat16)

    layers = []
    for _ in range(args.layers):
        layers.append(GpuLayer(n(nq * D, H, gen=gl), n(nkv * D, H, gen=gl), n(nkv * D, H, gen=gl),
                               n(H, nq * D, gen=gl), one(D), one(D), one(H), one(H), n(E, H),
                               n(El, 2 * I, H, gen=gl), n(El, H, I, gen=gl)))
        torch.cuda.empty_cache()
    lm_head = n(V, H)
    embed = torch.randn(V, H, generator=g, device=device).to(torch.bfloat16)
    B = args.batch
    blocks_per_seq = args.ctx // shape.block_size + 1
    NB = B * blocks_per_seq
    eng = Qwen3MoeMegakernel(shape, layers, max_batch=B, num_blocks=NB, final_norm=one(H), lm_head=lm_head,
                             embed=embed, rope_max_pos=max(4096, args.ctx + 1), device=device, shard=shard,
                             xchg=xchg)
    del lm_head
    eng.k_pool.normal_(generator=gl)
    eng.v_pool.normal_(generator=gl)
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(seed))
    table = perm.view(B, blocks_per_seq).to(torch.int32)
    positions = torch.full((B,), args.ctx, dtype=torch.int32)
    ids = torch.randint(0, V, (B,), generator=torch.Generator().manual_seed(seed + 1), dtype=torch.int32)
    return eng, shape, table, positions, ids


def algorithmic_bytes(shape, args, distinct_per_layer):
    H, D, E, I = shape.hidden_size, shape.head_dim, shape.num_experts, shape.moe_intermediate_size
    nq, nkv, V = shape.num_attention_heads, shape.num_key_value_heads, shape.vocab_size
    B, ctx = args.batch, args.ctx
    attn_w = ((nq + 2 * nkv) * D * H + H * nq * D) * 2 + (2 * H + 2 * D) * 2
    router = E * H * 2
    expert = (2 * I * H + H * I) * 2
    kv_read = B * ctx * nkv * D * 2 * 2
    kv_write = B * nkv * D * 2 * 2
    per_layer_fixed = attn_w + router + kv_read + kv_write
    total = sum(per_layer_fixed + d * expert for d in distinct_per_layer)
    total += V * H * 2 + H * 2 + B * H * 2  # LM head, final norm, embedding rows
    return total


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """``nvidia-smi`` clock/throttle samples of this process's GPU during the timed region.

    The GPU is named by its UUID (the local rank's index need not be nvidia-smi's index when
    CUDA_VISIBLE_DEVICES is set), and ``__enter__`` returns only once the first sample has
    arrived (several ranks starting nvidia-smi at once can take a second), so a short timed
    region still has samples."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = str(gpu_index)
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
            if uuid:
                self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        self.proc = None
        self.lines = []

    def _reader(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._reader, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 10 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        self.skip = len(self.lines)  # samples taken before the timed region
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.06)  # one more sample period
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        rows = []
        lines = self.lines[self.skip:] or self.lines
        for line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- CPU legs
def config_of(args, world):
    """The ``config`` object of both arms (same keys, so the driver can match the lines)."""
    return {"workload": "qwen3-30b-a3b decode step (48 layers + final norm + LM head)",
            "global_batch": args.batch, "ctx": args.ctx, "kv_block": 128, "layers": args.layers,
            "parallelism": "single GPU" if world == 1 else
            f"tp{world} over KV-head groups + ep{world} over experts, in-kernel exchange over NVLink",
            "l2": "no flush: ~27 GB of weights streamed per step >> 126 MB L2"}


def cpu_steps(args, warmup: int, steps: int):
    """Time the oracle (the faithful CPU restatement of the reference's decode path) over whole
    decode steps of the bench shape: all ``args.layers`` layers, each with its own paged K/V
    cache, the final norm and the LM head.  The layers share one layer's weight tensors (48
    distinct bf16 layers, ~61 GB, do not fit host memory; one layer's 1.2 GB of experts exceeds
    the last-level cache, so the sharing gives no cache advantage).

    Returns (seconds of every timed step, threads)."""
    import torch

    from oracle import qwen3_moe_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = O.QwenConfig(n_layers=args.layers)
    gen = torch.Generator().manual_seed(args.seed)
    lw = O.random_layer(cfg, gen)
    B, ctx = args.batch, args.ctx
    nb = ctx // 128 + 1
    NB = B * nb
    kcs = [torch.randn(NB, cfg.n_kv_heads, 128, cfg.head_dim, generator=gen).to(torch.bfloat16)
           for _ in range(args.layers)]
    vcs = [torch.randn(NB, cfg.n_kv_heads, 128, cfg.head_dim, generator=gen).to(torch.bfloat16)
           for _ in range(args.layers)]
    table = torch.arange(NB, dtype=torch.int32).view(B, nb)
    pos = torch.full((B,), ctx, dtype=torch.int32)
    cos, sin = O.rope_tables(ctx + 1, cfg.head_dim, cfg.rope_theta)
    lm = (torch.randn(cfg.vocab, cfg.hidden, generator=gen) * 0.02).to(torch.bfloat16)
    fn = (1.0 + torch.randn(cfg.hidden, generator=gen) * 0.02).to(torch.bfloat16)
    x = torch.randn(B, cfg.hidden, generator=gen).to(torch.bfloat16)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        O.decode_step(x, [lw], cfg, kcs, vcs, pos, table, cos, sin, fn, lm, "faithful")
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    times, threads = cpu_steps(args, args.warmup, args.steps)
    p50 = statistics.median(times)
    value = args.batch / p50
    sample = (f"oracle (faithful PyTorch CPU restatement of the reference's decode path): {args.steps} whole "
              f"{args.layers}-layer decode steps at B={args.batch} ctx {args.ctx} (layers share one layer's weights, "
              f"distinct KV caches) + final norm + LM head, after {args.warmup} warm-up steps; p50")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
            "p50_ms": p50 * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, KV prefix ~N(0,1))",
            "config": config_of(args, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def print_stage_times(eng, pos_d, table_d, ids_d, args):
    """Per-stage durations from the kernel's globaltimer stamps (CTA 0), averaged over layers."""
    import torch

    names = ["qkv", "attention", "o_proj", "router", "gate_up", "down"]
    acc = {n: [] for n in names}
    for _ in range(3):
        r = eng.decode_step(pos_d, table_d, input_ids=ids_d, stage_times=True)
        torch.cuda.synchronize()
        ts = r["stage_ns"].cpu().tolist()
        d = [(ts[i + 1] - ts[i]) / 1e3 for i in range(len(ts) - 1)]
        # d[0]: kernel start -> first barrier (input copy); then 6 per layer; last: output + LM head
        for l in range(args.layers):
            for k, n in enumerate(names):
                acc[n].append(d[1 + 6 * l + k])
        acc.setdefault("input", []).append(d[0])
        acc.setdefault("lm_head+out", []).append(d[-1])
        acc.setdefault("total", []).append((ts[-1] - ts[0]) / 1e3)
    out = {k: round(statistics.median(v), 2) for k, v in acc.items()}
    per_layer = sum(out[n] for n in names)
    print(json.dumps({"stage_us_median": out, "per_layer_us": round(per_layer, 2)}), file=sys.stderr, flush=True)


# ----------------------------------------------------------------------------- GPU arm
def _nvtx(torch, name):
    try:
        if name is None:
            torch.cuda.nvtx.range_pop()
        else:
            torch.cuda.nvtx.range_push(name)
    except Exception:
        pass


def multi_gpu_parity(rank, world, local, device):
    """Parity of the tensor + expert parallel step, run before the timing at N > 1.

    A small seeded case of the bench model (2 layers, B=4, positions crossing K/V pages, vocab
    4096, every rank building the same full weights from one seed and keeping its shard) runs
    through the sharded engine; rank 0 also runs the single-GPU kernel on the full weights (the
    path the GPU tests pin against the fp32 oracle) and compares hidden states and logits.  Every
    rank hashes its outputs; the hashes are all-gathered to check that the ranks agree bit for
    bit.  Returns the ``parity`` object of the bench line (rank 0) or None."""
    import hashlib

    import torch
    import torch.distributed as dist

    from nki_moe_megakernel_b200.engine import GpuLayer, Qwen3MoeMegakernel, Qwen3MoeShape
    from nki_moe_megakernel_b200.sharding import XchgRegion, plan_shard, shard_attention, shard_experts, xchg_bytes

    L, B, V = 2, 4, 4096
    positions = [600, 33, 1025, 128]
    full = Qwen3MoeShape(num_hidden_layers=L, vocab_size=V)
    H, D, E, I = full.hidden_size, full.head_dim, full.num_experts, full.moe_intermediate_size
    nq, nkv = full.num_attention_heads, full.num_key_value_heads
    g = torch.Generator(device=device).manual_seed(1234)

    def n(*sz):
        return (torch.randn(*sz, generator=g, device=device) * 0.02).to(torch.bfloat16)

    def one(*sz):
        return (1.0 + torch.randn(*sz, generator=g, device=device) * 0.02).to(torch.bfloat16)

    raw = [dict(wq=n(nq * D, H), wk=n(nkv * D, H), wv=n(nkv * D, H), wo=n(H, nq * D), qn=one(D), kn=one(D),
                ln1=one(H), ln2=one(H), router=n(E, H), gu=n(E, 2 * I, H), dn=n(E, H, I)) for _ in range(L)]
    fnorm, lm = one(H), n(V, H)
    embed = torch.randn(V, H, generator=g, device=device).to(torch.bfloat16)
    need = [p // 128 + 1 for p in positions]
    NB = sum(need) + 2
    k0 = torch.randn(L, NB, nkv, 128, D, generator=g, device=device).to(torch.bfloat16)
    v0 = torch.randn(L, NB, nkv, 128, D, generator=g, device=device).to(torch.bfloat16)
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(7)).tolist()
    table = torch.full((B, max(need)), -1, dtype=torch.int32)
    nxt = 0
    for b in range(B):
        for j in range(need[b]):
            table[b, j] = perm[nxt]
            nxt += 1
    tab_d = table.to(device)
    pos_d = torch.tensor(positions, dtype=torch.int32, device=device)
    ids_d = torch.randint(0, V, (B,), generator=torch.Generator().manual_seed(8), dtype=torch.int32).to(device)

    shard = plan_shard(rank, world, nq, nkv, E)
    layers = []
    for r in raw:
        wq, wk, wv, wo = shard_attention(r["wq"], r["wk"], r["wv"], r["wo"], shard, D)
        gu, dn = shard_experts(r["gu"], r["dn"], shard)
        layers.append(GpuLayer(wq, wk, wv, wo, r["qn"], r["kn"], r["ln1"], r["ln2"], r["router"], gu, dn))
    lshape = Qwen3MoeShape(num_hidden_layers=L, vocab_size=V, num_attention_heads=len(shard.q_heads),
                           num_key_value_heads=len(shard.kv_heads))
    xchg = XchgRegion(xchg_bytes(H, B, world, V), rank, world, local)
    eng = Qwen3MoeMegakernel(lshape, layers, max_batch=B, num_blocks=NB, final_norm=fnorm, lm_head=lm, embed=embed,
                             device=device, shard=shard, xchg=xchg)
    eng.k_pool.copy_(k0[:, :, shard.kv_heads])
    eng.v_pool.copy_(v0[:, :, shard.kv_heads])
    dist.barrier()
    res = eng.decode_step(pos_d, tab_d, input_ids=ids_d)
    st = eng.status()
    hid, lg = res["hidden"].cpu(), res["logits"].cpu()
    digest = hashlib.sha256(hid.view(torch.int16).numpy().tobytes() + lg.numpy().tobytes()).hexdigest()
    got = [None] * world
    dist.all_gather_object(got, (digest, st))
    out = None
    if rank == 0:
        ref = Qwen3MoeMegakernel(full, [GpuLayer(r["wq"], r["wk"], r["wv"], r["wo"], r["qn"], r["kn"], r["ln1"],
                                                 r["ln2"], r["router"], r["gu"], r["dn"]) for r in raw],
                                 max_batch=B, num_blocks=NB, final_norm=fnorm, lm_head=lm, embed=embed, device=device)
        ref.k_pool.copy_(k0)
        ref.v_pool.copy_(v0)
        rr = ref.decode_step(pos_d, tab_d, input_ids=ids_d)
        ref_st = ref.status()

        def cmp(a, b):
            a, b = a.float().flatten(), b.float().flatten()
            return (a - b).abs().max().item(), torch.nn.functional.cosine_similarity(a, b, dim=0).item()

        mh, ch = cmp(hid, rr["hidden"].cpu())
        ml, cl = cmp(lg, rr["logits"].cpu())
        ref.close()
        out = {"case": "2 layers, B=4, positions [600, 33, 1025, 128], vocab 4096",
               "against": "single-GPU kernel on the full weights (oracle-pinned by the GPU tests)",
               "hidden": {"max_abs": mh, "cosine": ch}, "logits": {"max_abs": ml, "cosine": cl},
               "max_abs": max(mh, ml), "cosine": min(ch, cl),
               "ranks_identical": len({d for d, _ in got}) == 1,
               "status": [s for _, s in got] + [ref_st],
               "within_tolerance": max(mh, ml) <= 2e-2 and min(ch, cl) >= 0.999}
    dist.barrier()
    eng.close()
    xchg.close()
    del eng, layers, raw
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    shard = xchg = None
    if world > 1:
        import datetime

        from nki_moe_megakernel_b200.engine import Qwen3MoeShape
        from nki_moe_megakernel_b200.sharding import XchgRegion, plan_shard, xchg_bytes

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        full = Qwen3MoeShape(num_hidden_layers=args.layers)
        shard = plan_shard(rank, world, full.num_attention_heads, full.num_key_value_heads, full.num_experts)
        xchg = XchgRegion(xchg_bytes(full.hidden_size, args.batch, world, full.vocab_size), rank, world, local)
        dist.barrier()
    parity = multi_gpu_parity(rank, world, local, device) if world > 1 else None
    eng, shape, table, positions, ids = build_engine(args, device, args.seed, shard, xchg)
    table_d, pos_d, ids_d = table.to(device), positions.to(device), ids.to(device)
    out = {"hidden": torch.empty(args.batch, shape.hidden_size, dtype=torch.bfloat16, device=device),
           "logits": torch.empty(args.batch, shape.vocab_size, dtype=torch.float32, device=device)}
    stream = torch.cuda.current_stream(device)

    def step():
        eng.decode_step(pos_d, table_d, input_ids=ids_d, out=out)

    # routing of the timed step (identical every step: same inputs, the KV slot is rewritten)
    tr = eng.decode_step(pos_d, table_d, input_ids=ids_d, trace=True)
    eng.check_status()
    if shard is None:
        distinct = [len(torch.unique(tr["topk_idx"][l])) for l in range(args.layers)]
    else:  # experts this rank streams
        lo, hi = shard.expert_begin, shard.expert_begin + shard.n_local_experts
        distinct = [int(((u >= lo) & (u < hi)).sum()) for u in (torch.unique(tr["topk_idx"][l]) for l in range(args.layers))]
    del tr
    for _ in range(args.warmup):
        step()
    eng.check_status()
    if args.stage_times:
        print_stage_times(eng, pos_d, table_d, ids_d, args)
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    # the clock sampler starts first: its start-up time differs between ranks, and the ranks must
    # enter the timed region together (a rank that starts late makes the others wait in the
    # step's first exchange)
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        _nvtx(torch, "timed")  # lets `ncu --nvtx --nvtx-include timed/` list exactly the timed launches
        evs[0].record(stream)
        for i in range(args.steps):
            step()
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        _nvtx(torch, None)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    eng.check_status()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    total_ms = evs[0].elapsed_time(evs[-1])
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms = total_ms / args.steps
    # tensor + expert parallel: all ranks serve the same batch (strong scaling)
    value = args.batch / (ms / 1e3)

    # end to end through the public API: pinned host inputs in, logits out, every step
    e2e = None
    if not args.no_e2e:
        ids_h = ids.pin_memory()
        pos_h = positions.pin_memory()
        tab_h = table.pin_memory()
        tokens_d = torch.empty(args.batch, dtype=torch.int32, device=device)
        tokens_h = torch.empty(args.batch, dtype=torch.int32).pin_memory()
        for _ in range(2):
            ids_d.copy_(ids_h, non_blocking=True)
            step()
            eng.sample(out["logits"], pos_d, top_k=1, out=tokens_d)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _nvtx(torch, "e2e")  # `ncu --nvtx --nvtx-include e2e/` lists the end-to-end launches
        e0.record(stream)
        for _ in range(args.steps):
            ids_d.copy_(ids_h, non_blocking=True)
            pos_d.copy_(pos_h, non_blocking=True)
            table_d.copy_(tab_h, non_blocking=True)
            step()
            eng.sample(out["logits"], pos_d, top_k=1, out=tokens_d)  # greedy next token on the device
            tokens_h.copy_(tokens_d, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        _nvtx(torch, None)
        e2e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e2e_ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": args.batch / (e2e_ms / args.steps / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": ids_h.numel() * 4 + pos_h.numel() * 4 + tab_h.numel() * 4,
               "d2h_bytes_per_step": tokens_h.numel() * 4,
               "step": "token ids, positions and block table copied in; decode step; greedy next-token "
                       "selection on the device (nkm_sample_logits); token ids copied out"}
        eng.check_status()

    nbytes = algorithmic_bytes(shape, args, distinct)
    peak, peak_kind = measured_peaks()
    achieved = nbytes / (ms / 1e3) / 1e9
    traffic_path = os.path.join(ROOT, "profiles", "decode_step_dram_traffic.json")
    traffic = None
    if world == 1 and os.path.exists(traffic_path):  # measured on the single-GPU workload
        try:
            traffic = json.load(open(traffic_path)).get("bytes_per_launch")
        except Exception:
            traffic = None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        times, threads = cpu_steps(args, 1, 3)
        step_s = statistics.median(times)
        cpu = {"value": args.batch / step_s, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"oracle (faithful PyTorch CPU restatement): 3 whole {args.layers}-layer decode steps at "
                         f"B={args.batch} ctx {args.ctx} (shared layer weights, distinct KV caches) + final norm + "
                         f"LM head after 1 warm-up step; p50"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "p50_ms": statistics.median(per),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights of the Qwen3-30B-A3B architecture, KV prefix ~N(0,1))",
            "config": config_of(args, world),
            "distinct_experts_per_layer_mean": sum(distinct) / len(distinct),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_step": nbytes,
                         "kernel": "qwen3_decode_kernel (one launch per step)"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "parity": parity,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        eng.close()
        xchg.close()
        dist.destroy_process_group()


def _events_time(torch, stream, fn, steps, warmup, barrier=None):
    """Mean and per-step ms of ``steps`` calls of fn after ``warmup``; ``barrier`` (several ranks)
    lines the ranks up after the warm-up, right before the timed region."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if barrier is not None:
        barrier()
        torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    _nvtx(torch, "timed")  # `ncu --nvtx --nvtx-include timed/` lists exactly the timed launches
    evs[0].record(stream)
    for i in range(steps):
        fn()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    _nvtx(torch, None)
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    return evs[0].elapsed_time(evs[-1]) / steps, per


def run_gpt_oss(args):
    """GPT-OSS-20B decode step (config 4): 24 layers (sliding/full alternating), B=16, context
    4096, MXFP4 experts, vocab 201088, seeded random weights.  Under torchrun (N GPUs) the ranks
    split the KV-head groups and the experts (``sharding.shard_gptoss_layer``) and the LM head
    over the vocabulary, every rank building the same weights from the seed and keeping its part;
    time = max over ranks."""
    import torch
    import torch.distributed as dist

    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssGpuLayer, GptOssMegakernel, GptOssShape

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, ctx = 16, 4096
    shape = GptOssShape(num_hidden_layers=args.gptoss_layers)
    shard = xchg = None
    if world > 1:
        import dataclasses
        import datetime

        from nki_moe_megakernel_b200.sharding import XchgRegion, gptoss_xchg_bytes, plan_shard, shard_gptoss_layer

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        shard = plan_shard(rank, world, shape.num_attention_heads, shape.num_key_value_heads, shape.num_local_experts)
        xchg = XchgRegion(gptoss_xchg_bytes(shape.hidden_size, B, world, shape.vocab_size), rank, world, local)
    H, D, E, I, V = shape.hidden_size, shape.head_dim, shape.num_local_experts, shape.intermediate_size, shape.vocab_size
    nq, nkv, L = shape.num_attention_heads, shape.num_key_value_heads, shape.num_hidden_layers
    g = torch.Generator(device=dev).manual_seed(args.seed)

    def n(*sz, std=0.02):
        return (torch.randn(*sz, generator=g, device=dev) * std).to(torch.bfloat16)

    layers = []
    for l in range(L):
        t = dict(wq=n(nq * D, H), bq=n(nq * D), wk=n(nkv * D, H), bk=n(nkv * D), wv=n(nkv * D, H), bv=n(nkv * D),
                 wo=n(H, nq * D), bo=n(H), sinks=n(nq, std=1.0), ln1=1 + n(H), ln2=1 + n(H), router=n(E, H),
                 router_b=n(E), gu_b=n(E, 2 * I), dn_b=n(E, H),
                 gu_codes=torch.randint(0, 16, (E, 2 * I, H), generator=g, device=dev, dtype=torch.uint8),
                 gu_scales=torch.randint(119, 122, (E, 2 * I, H // 32), generator=g, device=dev, dtype=torch.uint8),
                 dn_codes=torch.randint(0, 16, (E, H, I), generator=g, device=dev, dtype=torch.uint8),
                 dn_scales=torch.randint(119, 122, (E, H, I // 32), generator=g, device=dev, dtype=torch.uint8))
        if shard is not None:
            t = shard_gptoss_layer(t, shard, D)
        layers.append(GptOssGpuLayer(t, shape.is_sliding(l)))
        del t
        torch.cuda.empty_cache()
    nb = ctx // 128 + 1
    NB = B * nb
    eshape = shape if shard is None else dataclasses.replace(shape, num_attention_heads=len(shard.q_heads),
                                                             num_key_value_heads=len(shard.kv_heads))
    eng = GptOssMegakernel(eshape, layers, max_batch=B, num_blocks=NB, max_context=ctx + 128, final_norm=1 + n(H),
                           lm_head=n(V, H), embed=torch.randn(V, H, generator=g, device=dev).to(torch.bfloat16),
                           device=dev, shard=shard, xchg=xchg)
    eng.k_pool.normal_(generator=g)
    eng.v_pool.normal_(generator=g)
    table = torch.randperm(NB, generator=torch.Generator().manual_seed(args.seed)).view(B, nb).to(torch.int32).to(dev)
    pos = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    ids = torch.randint(0, V, (B,), generator=torch.Generator().manual_seed(1), dtype=torch.int32).to(dev)
    out = {"hidden": torch.empty(B, H, dtype=torch.bfloat16, device=dev),
           "logits": torch.empty(B, V, dtype=torch.float32, device=dev)}
    if world > 1:
        dist.barrier()
    tr = eng.decode_step(pos, table, input_ids=ids, trace=True)
    eng.check_status()
    distinct = [len(torch.unique(tr["topk_idx"][l])) for l in range(L)]  # routing is replicated: whole model
    del tr
    if args.stage_times:
        names = ["qkv", "qkv_fin", "attention", "combine", "o_proj", "o_resid", "norm_router", "gate_up", "down",
                 "moe_resid"]
        acc = {}
        for _ in range(5):
            ts = eng.decode_step(pos, table, input_ids=ids, stage_times=True)["stage_ns"].cpu().tolist()
            d = [(ts[i + 1] - ts[i]) / 1e3 for i in range(len(ts) - 1)]
            for l in range(L):
                for k, n in enumerate(names):
                    acc.setdefault(n, []).append(d[1 + 10 * l + k])
            acc.setdefault("lm_head+out", []).append(d[-1])
            acc.setdefault("total", []).append((ts[-1] - ts[0]) / 1e3)
        med = {k: round(statistics.median(v), 2) for k, v in acc.items()}
        print(json.dumps({"stage_us_median": med, "per_layer_us": round(sum(med[n] for n in names), 2)}),
              file=sys.stderr, flush=True)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(local) as clk:
        ms, per = _events_time(torch, stream, lambda: eng.decode_step(pos, table, input_ids=ids, out=out), args.steps,
                               args.warmup, barrier=dist.barrier if world > 1 else None)
    eng.check_status()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    attn_w = ((nq + 2 * nkv) * D * H + H * nq * D) * 2 + ((nq + 2 * nkv) * D + H + nq + 2 * H + E) * 2 + E * H * 2
    expert = (2 * I * H) // 2 + 2 * I * (H // 32) + 2 * I * 2 + (H * I) // 2 + H * (I // 32) + H * 2
    kv = sum(B * (min(ctx, shape.sliding_window - 1) if shape.is_sliding(l) else ctx) * nkv * D * 2 * 2 for l in range(L))
    nbytes = L * attn_w + sum(distinct) * expert + kv + L * B * nkv * D * 2 * 2 + V * H * 2
    peak, peak_kind = measured_peaks()
    achieved = nbytes / (ms / 1e3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "GPT-OSS-20B decode tokens/s at B=16 ctx 4096 (config 4)", "value": B / (ms / 1e3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "p50_ms": statistics.median(per), "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16 activations, MXFP4 experts", "data": "synthetic (seeded random)",
            "config": {"workload": f"gpt-oss-20b decode step ({L} layers + LM head)", "global_batch": B, "ctx": ctx,
                       "distinct_experts_per_layer_mean": sum(distinct) / L,
                       "parallelism": "single GPU" if world == 1 else f"tp{world} (KV-head groups) + ep{world}, "
                                                                      "LM head split over the vocabulary"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak / world, "peak_kind": peak_kind, "algorithmic_bytes_per_step": nbytes,
                         "kernel": "gptoss_decode_kernel (one launch per step per GPU)",
                         "note": "frac against the peak of all the step's GPUs"},
            "gpu_launches": args.steps, "clocks": clk.summary()}), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        eng.close()
        xchg.close()
        dist.destroy_process_group()


def _mx_experts(torch, g, dev, E, rows, cols):
    """Seeded synthetic MXFP8 expert matrices on the device: e4m3 codes of N(0, 32) values
    (clipped to +-448) with the e8m0 scale 2^-11 in every block (weights ~N(0, 0.016))."""
    codes = (torch.randn(E, rows, cols, generator=g, device=dev) * 32).clamp(-448, 448).to(torch.float8_e4m3fn)
    scales = torch.full((E, rows, cols // 32), 127 - 11, dtype=torch.uint8, device=dev)
    return codes.view(torch.uint8), scales


def run_moe_tc(args):
    """The tcgen05 MoE block at config 3's expert stage: 64 tokens, top-8 of 128 Qwen3-30B-A3B
    experts (one layer), seeded random weights."""
    import torch

    from nki_moe_megakernel_b200.engine import MoeTcBlock

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, H, E, K, I = 64, 2048, 128, 8, 768
    g = torch.Generator(device=dev).manual_seed(args.seed)
    n = lambda *sz: (torch.randn(*sz, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    mx = args.weights == "mxfp8"
    if mx:
        blk = MoeTcBlock(1 + n(H), n(E, H), None, None, eps=1e-6, top_k=K, max_tokens=T, device=dev,
                         mxfp8=(*_mx_experts(torch, g, dev, E, 2 * I, H), *_mx_experts(torch, g, dev, E, H, I)))
    else:
        blk = MoeTcBlock(1 + n(H), n(E, H), n(E, 2 * I, H), n(E, H, I), eps=1e-6, top_k=K, max_tokens=T, device=dev)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    _, idx, _ = blk(x)
    assert blk.status() == 0
    distinct = len(torch.unique(idx))
    stream = torch.cuda.current_stream(dev)
    ms, per = _events_time(torch, stream, lambda: blk(x), args.steps, args.warmup)
    assert blk.status() == 0
    wb = (1 + 1 / 32) if mx else 2  # bytes per expert weight
    nbytes = distinct * 3 * I * H * wb + E * H * 2 + 2 * T * H * 2
    flops = 2 * T * K * 3 * I * H
    peak, peak_kind = measured_peaks()
    achieved = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "tcgen05 MoE block (config 3 expert stage) tokens/s", "value": T / (ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_call": ms, "p50_ms": statistics.median(per),
        "dtype": "bf16", "config": {"workload": "qwen3-30b-a3b MoE block, 64 tokens", "distinct_experts": distinct,
                                    "expert_weights": args.weights},
        "tflops": flops / (ms / 1e3) / 1e12,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "algorithmic_bytes_per_call": nbytes}}), flush=True)


def run_wide(args):
    """Config 3 on one GPU: the 48-layer Qwen3-30B-A3B decode step at B=64 with per-sequence
    contexts uniform in [1024, 8192] (``Qwen3MoeWideDecoder``: attention in 32-row decode-kernel
    launches, experts on the tcgen05 grouped GEMMs, final norm + LM head as one GEMM), seeded
    random-init weights (48 distinct layers), K/V ~N(0, 1)."""
    import torch

    from nki_moe_megakernel_b200.engine import Qwen3MoeShape, Qwen3MoeWideDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, L = 64, args.layers
    shape = Qwen3MoeShape(num_hidden_layers=L)
    if world > 1:
        return run_wide_ep(args, rank, world, local, dev, shape)
    H, D, E, I, V = shape.hidden_size, shape.head_dim, shape.num_experts, shape.moe_intermediate_size, shape.vocab_size
    nq, nkv = shape.num_attention_heads, shape.num_key_value_heads
    g = torch.Generator(device=dev).manual_seed(args.seed)
    n = lambda *sz: (torch.randn(*sz, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    one = lambda *sz: (1.0 + torch.randn(*sz, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    mx = args.weights == "mxfp8"
    layers = []
    for _ in range(L):
        lw = {"wq": n(nq * D, H), "wk": n(nkv * D, H), "wv": n(nkv * D, H), "wo": n(H, nq * D), "q_norm": one(D),
              "k_norm": one(D), "ln1": one(H), "ln2": one(H), "router": n(E, H)}
        if mx:
            lw["mxfp8"] = (*_mx_experts(torch, g, dev, E, 2 * I, H), *_mx_experts(torch, g, dev, E, H, I))
        else:
            lw["gate_up"], lw["down"] = n(E, 2 * I, H), n(E, H, I)
        layers.append(lw)
    ctx = torch.randint(1024, 8193, (B,), generator=torch.Generator().manual_seed(args.seed)).tolist()
    need = [c // 128 + 1 for c in ctx]
    NB = sum(need)
    wide = Qwen3MoeWideDecoder(shape, layers, max_batch=B, num_blocks=NB, final_norm=one(H), lm_head=n(V, H),
                               embed=torch.randn(V, H, generator=g, device=dev).to(torch.bfloat16),
                               rope_max_pos=8320, device=dev)
    for lw in layers:  # the tcgen05 blocks hold the expert tensors; the FT copies hold attention
        for k in ("wq", "wk", "wv", "wo", "mxfp8"):
            lw.pop(k, None)
    torch.cuda.empty_cache()
    wide.k_pool.normal_(generator=g)
    wide.v_pool.normal_(generator=g)
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(args.seed + 1))
    maxb = max(need)
    table = torch.full((B, maxb), -1, dtype=torch.int32)
    o = 0
    for b in range(B):
        table[b, :need[b]] = perm[o:o + need[b]].to(torch.int32)
        o += need[b]
    table_d, pos_d = table.to(dev), torch.tensor(ctx, dtype=torch.int32, device=dev)
    ids_d = torch.randint(0, V, (B,), generator=torch.Generator().manual_seed(args.seed + 2), dtype=torch.int32).to(dev)
    tr = wide.decode_step(pos_d, table_d, input_ids=ids_d, trace=True)
    wide.check_status()
    distinct = [len(torch.unique(tr["topk_idx"][li])) for li in range(L)]
    del tr
    stream = torch.cuda.current_stream(dev)
    ms, per = _events_time(torch, stream, lambda: wide.decode_step(pos_d, table_d, input_ids=ids_d), args.steps,
                           args.warmup)
    wide.check_status()
    att_w = (nq * D * H + 2 * nkv * D * H + H * nq * D) * 2
    kv = sum(ctx) * nkv * D * 2 * 2
    wb = (1 + 1 / 32) if mx else 2  # bytes per expert weight
    nbytes = L * (att_w + kv + E * H * 2 + sum(distinct) / L * 3 * I * H * wb) + V * H * 2
    peak, peak_kind = measured_peaks()
    achieved = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "Qwen3-30B-A3B decode tokens/s at B=64, contexts uniform in [1024, 8192] (config 3, 1 GPU)",
        "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "p50_ms": statistics.median(per), "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, 48 distinct layers; K/V ~N(0,1))",
        "config": {"workload": "qwen3-30b-a3b decode step at B=64 (attention 2 x 32-row launches, tcgen05 experts)",
                   "global_batch": B, "ctx_mean": sum(ctx) / B, "layers": L, "expert_weights": args.weights,
                   "distinct_experts_per_layer_mean": sum(distinct) / L},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "algorithmic_bytes_per_step": nbytes}}), flush=True)


def run_wide_ep(args, rank, world, local, dev, shape):
    """Config 3 across the node: B=64 rows split over the ranks for attention, experts split for
    the MoE, NVLink peer-store exchange (``Qwen3MoeWideDecoderEP``); time = max over ranks."""
    import datetime

    import torch
    import torch.distributed as dist

    from nki_moe_megakernel_b200.engine import Qwen3MoeWideDecoderEP
    from nki_moe_megakernel_b200.sharding import XchgRegion

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    B, L = 64, shape.num_hidden_layers
    H, D, E, I, V = shape.hidden_size, shape.head_dim, shape.num_experts, shape.moe_intermediate_size, shape.vocab_size
    nq, nkv = shape.num_attention_heads, shape.num_key_value_heads
    R, e0, nl = B // world, rank * E // world, E // world
    g = torch.Generator(device=dev).manual_seed(args.seed)            # replicated tensors
    gl = torch.Generator(device=dev).manual_seed(args.seed + 1000 + rank)  # this rank's experts
    n = lambda *sz, gen=g: (torch.randn(*sz, generator=gen, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    one = lambda *sz: (1.0 + torch.randn(*sz, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    mx = args.weights == "mxfp8"
    layers = []
    for _ in range(L):
        lw = {"wq": n(nq * D, H), "wk": n(nkv * D, H), "wv": n(nkv * D, H), "wo": n(H, nq * D), "q_norm": one(D),
              "k_norm": one(D), "ln1": one(H), "ln2": one(H), "router": n(E, H)}
        if mx:
            lw["mxfp8"] = (*_mx_experts(torch, gl, dev, nl, 2 * I, H), *_mx_experts(torch, gl, dev, nl, H, I))
        else:
            lw["gate_up"], lw["down"] = n(nl, 2 * I, H, gen=gl), n(nl, H, I, gen=gl)
        layers.append(lw)
    ctx = torch.randint(1024, 8193, (B,), generator=torch.Generator().manual_seed(args.seed)).tolist()
    mine = ctx[rank * R:(rank + 1) * R]
    need = [c // 128 + 1 for c in mine]
    NB = sum(need)
    xchg = XchgRegion(Qwen3MoeWideDecoderEP.exchange_bytes(B, H, world), rank, world, local)
    ep = Qwen3MoeWideDecoderEP(shape, layers, rank=rank, world=world, xchg=xchg, batch=B, expert_begin=e0, n_local=nl,
                               num_blocks=NB, final_norm=one(H), lm_head=n(V, H),
                               embed=torch.randn(V, H, generator=g, device=dev).to(torch.bfloat16),
                               rope_max_pos=8320, device=dev)
    for lw in layers:
        for k in ("wq", "wk", "wv", "wo", "mxfp8"):
            lw.pop(k, None)
    torch.cuda.empty_cache()
    ep.k_pool.normal_(generator=gl)
    ep.v_pool.normal_(generator=gl)
    table = torch.full((R, max(need)), -1, dtype=torch.int32)
    o = 0
    for b in range(R):
        table[b, :need[b]] = torch.arange(o, o + need[b], dtype=torch.int32)
        o += need[b]
    table_d, pos_d = table.to(dev), torch.tensor(mine, dtype=torch.int32, device=dev)
    ids_d = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(args.seed + 2 + rank),
                          dtype=torch.int32).to(dev)
    dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ms, per = _events_time(torch, stream, lambda: ep.decode_step(pos_d, table_d, input_ids=ids_d), args.steps,
                           args.warmup, barrier=dist.barrier)
    ep.check_status()
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({
            "metric": "Qwen3-30B-A3B decode tokens/s at B=64, contexts uniform in [1024, 8192] (config 3)",
            "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (seeded random-init weights; K/V ~N(0,1))",
            "config": {"workload": "qwen3-30b-a3b decode step at B=64, attention rows split over ranks, experts "
                                   "split (expert parallel), NVLink peer-store exchange", "global_batch": B,
                       "ctx_mean": sum(ctx) / B, "layers": L, "expert_weights": args.weights,
                       "parallelism": f"attention dp{world} + ep{world}"}}), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    ep.close()
    xchg.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.workload == "wide":
        run_wide(a)
        raise SystemExit(0)
    if a.workload == "gpt-oss":
        run_gpt_oss(a)
        raise SystemExit(0)
    if a.workload == "moe-tc":
        run_moe_tc(a)
        raise SystemExit(0)
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)
