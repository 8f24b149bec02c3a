"""Driver with the reference ``main.py`` modes (``generate``, ``validate``, ``evaluate_single``).

Same registry convention as the reference (``main.py:927-941``): ``--model qwen3_moe`` with
``--enable-nki`` loads ``megakernels.qwen3_moe.qwen_with_megakernel.NeuronQwen3MoeForCausalLM``
(here: the B200 decode megakernel).  The baseline model of ``validate`` is Hugging Face
``Qwen3MoeForCausalLM`` with the same weights, fp32 (the reference's baseline is the library
model of the same architecture).

Without ``--model-path`` the weights are seeded random-init of the configured shape and the
prompts are turned into token ids deterministically (no tokenizer or checkpoint needed).

Run: ``python -m nki_moe_megakernel_b200.main --mode generate --enable-nki [--num-layers 2]``.
Several GPUs (tensor + expert parallel, reference ``--tp-degree`` / ``--moe-ep-degree``,
``main.py:224-231``): ``torchrun --nproc-per-node 2 -m nki_moe_megakernel_b200.main --mode validate
--enable-nki --tp-degree 2 --moe-ep-degree 2 --num-layers 2``; every rank steps the kernel, rank 0
prints.
"""
from __future__ import annotations

import argparse
import ast
import contextlib
import importlib
import io
import os
import time
from typing import Dict, List, Optional

import torch

_MODEL_REGISTRY = {
    "qwen3_moe": ("nki_moe_megakernel_b200.megakernels.qwen3_moe.qwen_with_megakernel", "NeuronQwen3MoeForCausalLM"),
    "gpt_oss": ("nki_moe_megakernel_b200.megakernels.gpt_oss.gpt_oss_with_megakernel", "NeuronGptOssForCausalLM"),
}
DEFAULT_TOL_MAP = "{None: (1e-5, 0.05), 1000: (1e-5, 0.03), 50: (1e-5, 0.03), 5: (1e-5, 0.03)}"


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--mode", choices=["generate", "validate", "evaluate_single"], default="generate")
    p.add_argument("--model", choices=list(_MODEL_REGISTRY), default="qwen3_moe")
    p.add_argument("--enable-nki", action="store_true",
                   help="accepted for command-line compatibility; the megakernel is the only decode path")
    p.add_argument("--model-path", default=None, help="Hugging Face checkpoint dir (safetensors); random-init if absent")
    p.add_argument("--compiled-model-path", default=None)
    p.add_argument("--prompt", dest="prompts", action="append", default=[])
    p.add_argument("--batch-size", type=int, default=None)
    p.add_argument("--seq-len", type=int, default=640)
    p.add_argument("--max-new-tokens", type=int, default=None)
    p.add_argument("--top-k", type=int, default=1)
    p.add_argument("--do-sample", action="store_true")
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--top-p", type=float, default=1.0)
    p.add_argument("--on-device-sampling", action="store_true",
                   help="accepted for command-line compatibility; tokens are always sampled on the device")
    p.add_argument("--tol-map", default=DEFAULT_TOL_MAP)
    p.add_argument("--num-tokens-to-check", type=int, default=None)
    p.add_argument("--divergence-difference-tol", type=float, default=0.001)
    p.add_argument("--routing-divergence-tol", type=float, default=0.02,
                   help="validate: router-logit gap under which the fp32 baseline takes the megakernel's expert "
                        "set for a token (near ties; the count is printed)")
    p.add_argument("--pa-block-size", type=int, default=128)
    p.add_argument("--pa-num-blocks", type=int, default=None)
    p.add_argument("--num-layers", type=int, default=None, help="override num_hidden_layers (random-init only)")
    p.add_argument("--benchmark-iters", type=int, default=5)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tp-degree", type=int, default=None,
                   help="GPUs of the tensor + expert parallel group (default: WORLD_SIZE, 1 without torchrun)")
    p.add_argument("--moe-ep-degree", type=int, default=None, help="1 or tp-degree (experts split over the TP ranks)")
    p.add_argument("--moe-tp-degree", type=int, default=1)
    return p.parse_args(argv)


def init_distributed(args):
    """One process per GPU under torchrun: NCCL process group, this rank's GPU.  Returns
    (rank, world, device)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    tp = args.tp_degree or world
    if tp != world:
        raise SystemExit(f"--tp-degree {tp} needs {tp} processes (got WORLD_SIZE={world})")
    args.tp_degree = tp
    args.moe_ep_degree = args.moe_ep_degree or tp
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist  # noqa: PLC0415

        if not dist.is_initialized():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    return rank, world, device


# ---------------------------------------------------------------------------
def _tokenizer(model_path: Optional[str]):
    if model_path and os.path.exists(os.path.join(model_path, "tokenizer_config.json")):
        from transformers import AutoTokenizer  # noqa: PLC0415

        return AutoTokenizer.from_pretrained(model_path)
    return None


def encode_prompts(prompts: List[str], tokenizer, vocab: int) -> List[List[int]]:
    if tokenizer is not None:
        return [tokenizer(p)["input_ids"] for p in prompts]
    # no tokenizer: one id per UTF-8 byte, folded into the vocabulary
    return [[(b * 2654435761 + 17) % vocab for b in p.encode()] for p in prompts]


def prepare_inference(model_cls, args):
    """Build config + model, convert weights, create the kernel instance (reference
    ``main.py:382-655``: compile() then load())."""
    ncfg_cls, cfg_cls = model_cls.get_neuron_config_cls(), model_cls.get_config_cls()
    mod = importlib.import_module(model_cls.__module__)
    ncfg = ncfg_cls(batch_size=args.batch_size, max_batch_size=args.batch_size, seq_len=args.seq_len,
                    max_length=args.seq_len, pa_block_size=args.pa_block_size, pa_num_blocks=args.pa_num_blocks,
                    top_k=args.top_k, do_sample=args.do_sample, temperature=args.temperature, top_p=args.top_p,
                    tp_degree=getattr(args, "tp_degree", None) or 1,
                    moe_ep_degree=getattr(args, "moe_ep_degree", None) or 1,
                    moe_tp_degree=getattr(args, "moe_tp_degree", 1))
    overrides = {}
    if args.num_layers is not None and not args.model_path:
        overrides["num_hidden_layers"] = args.num_layers
    cfg = cfg_cls(ncfg, load_config=mod.load_pretrained_config(args.model_path), **overrides)
    model = model_cls(args.model_path, cfg, device=getattr(args, "_device", None), seed=args.seed,
                      state_dict=getattr(args, "_state_dict", None))
    model.compile(args.compiled_model_path)
    model.load(args.compiled_model_path)
    return model, _tokenizer(args.model_path)


def run_generation(model, tokenizer, prompts: List[str], max_new_tokens: int):
    ids = encode_prompts(prompts, tokenizer, model.config.vocab_size)
    outs = model.generate(ids, max_new_tokens)
    for p, o in zip(prompts, outs):
        text = tokenizer.decode(o) if tokenizer is not None else o
        print(f"prompt: {p!r}\n  -> {text}")
    return outs


# ---------------------------------------------------------------------------
def hf_baseline_gpt_oss(model):
    """HF GptOssForCausalLM (fp32) with exactly the megakernel's weights (MXFP4 experts
    dequantised)."""
    from transformers import GptOssConfig, GptOssForCausalLM  # noqa: PLC0415

    from .megakernels.gpt_oss.gpt_oss_with_megakernel import mxfp4_dequant, unpack_mxfp4_blocks  # noqa: PLC0415

    c = model.config
    hc = GptOssConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                      num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                      num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim,
                      num_local_experts=c.num_local_experts, num_experts_per_tok=c.num_experts_per_tok,
                      sliding_window=c.sliding_window, rms_norm_eps=c.rms_norm_eps, tie_word_embeddings=False,
                      max_position_embeddings=c.max_position_embeddings, rope_parameters=dict(c.rope_parameters),
                      layer_types=list(c.layer_types))
    hc._attn_implementation = "eager"
    with torch.device(model.device):
        hf = GptOssForCausalLM(hc).to(torch.float32).eval()
    sd = {}
    raw = model.hf_state_dict()
    for k, v in raw.items():
        if k.endswith("_blocks"):
            base = k[: -len("_blocks")]
            w = mxfp4_dequant(unpack_mxfp4_blocks(v), raw[base + "_scales"])
            sd[base] = w.transpose(-1, -2).float()
        elif not k.endswith("_scales"):
            sd[k] = v.float()
    missing, _ = hf.load_state_dict(sd, strict=False)
    if missing:
        raise RuntimeError(f"baseline weights missing: {missing[:4]}")
    return hf


def hf_baseline(model):
    """HF Qwen3MoeForCausalLM (fp32) with exactly the megakernel's weights (GPT-OSS models:
    ``hf_baseline_gpt_oss``)."""
    if type(model).__name__ == "NeuronGptOssForCausalLM":
        return hf_baseline_gpt_oss(model)
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM  # noqa: PLC0415

    c = model.config
    hf_cfg = Qwen3MoeConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, num_hidden_layers=c.num_hidden_layers,
                            num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                            head_dim=c.head_dim, num_experts=c.num_experts, num_experts_per_tok=c.num_experts_per_tok,
                            moe_intermediate_size=c.moe_intermediate_size, rms_norm_eps=c.rms_norm_eps,
                            max_position_embeddings=c.max_position_embeddings, norm_topk_prob=True,
                            rope_parameters={"rope_theta": c.rope_theta, "rope_type": "default"},
                            tie_word_embeddings=False)
    hf_cfg._attn_implementation = "eager"
    with torch.device(model.device):
        hf = Qwen3MoeForCausalLM(hf_cfg).to(torch.float32).eval()
    sd = model.hf_state_dict()
    missing, unexpected = hf.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    if missing:
        raise RuntimeError(f"baseline weights missing: {missing[:4]}")
    return hf


def _parse_tol_map(s: str) -> Dict:
    return ast.literal_eval(s) if isinstance(s, str) else s


class _FollowNearTies:
    """While active, every MoE router of the Hugging Face baseline (``Qwen3MoeTopKRouter``,
    ``GptOssTopKRouter``) takes the megakernel's expert set for a token wherever that set is a
    top-k of the baseline's own fp32 router logits within ``tol`` (the k-th chosen logit at most
    ``tol`` below the best logit left out); elsewhere the baseline routes by itself.  The
    megakernel's bf16 residual drifts from the fp32 one by ~1e-3 relative, which moves router
    logits by up to ~1e-2: at a near tie the two sides may pick different experts, and one such
    flip changes that token's output by a whole expert's share, far beyond the logit tolerances,
    without either side being wrong.  ``followed`` counts the tokens that took the kernel's set
    and ``max_gap`` is their largest logit gap; a differing set beyond ``tol`` is left alone (and
    then shows up as a logit mismatch)."""

    NAMES = ("Qwen3MoeTopKRouter", "GptOssTopKRouter")

    def __init__(self, hf, routing: torch.Tensor, tol: float):
        self.routers = [m for m in hf.modules() if type(m).__name__ in self.NAMES]
        self.routing, self.tol = routing, tol      # [T, layers, top_k]
        self.followed, self.max_gap = 0, 0.0
        self._saved = []

    def __enter__(self):
        for li, r in enumerate(self.routers):
            self._saved.append((r, r.forward))
            r.forward = self._wrap(r, r.forward, li)
        return self

    def __exit__(self, *exc):
        for r, f in self._saved:
            r.forward = f
        self._saved.clear()

    def _wrap(self, r, orig, li):
        import torch.nn.functional as F  # noqa: PLC0415

        def fwd(hidden_states):
            logits, scores, idx = orig(hidden_states)
            if li >= self.routing.shape[1] or idx.shape[0] != self.routing.shape[0]:
                return logits, scores, idx
            raw = F.linear(hidden_states.reshape(-1, r.hidden_dim).float(), r.weight.float(),
                           None if getattr(r, "bias", None) is None else r.bias.float())
            hint = self.routing[:, li].to(idx.device).long()
            idx, scores = idx.clone(), scores.clone()
            for t in range(idx.shape[0]):
                h = hint[t]
                if set(h.tolist()) == set(idx[t].tolist()):
                    continue
                out = torch.ones(raw.shape[-1], dtype=torch.bool, device=raw.device)
                out[h] = False
                gap = float(raw[t, out].max() - raw[t, h].min())
                if gap > self.tol:
                    continue
                self.followed += 1
                self.max_gap = max(self.max_gap, gap)
                idx[t] = h.to(idx.dtype)
                if type(r).__name__ == "GptOssTopKRouter":
                    scores[t] = torch.softmax(raw[t, h], dim=-1).to(scores.dtype)
                else:
                    pr = torch.softmax(raw[t], dim=-1)[h]
                    scores[t] = (pr / pr.sum() if r.norm_topk_prob else pr).to(scores.dtype)
            return logits, scores, idx

        return fwd


def run_accuracy_check(model, tokenizer, prompts: List[str], tol_map, num_tokens_to_check: int,
                       routing_tol: float = 0.02) -> bool:
    """Greedy-generate with the baseline, teacher-force the megakernel on the same tokens and
    compare every step's logits.  ``tol_map`` = {top-k or None: (atol, rtol)}: over the
    baseline's top-k logits (all logits for None), max |ours - base| <= atol + rtol * max |base|.
    The compared baseline pass follows the megakernel's expert choice at router near ties
    (``_FollowNearTies``, gap ``routing_tol``); the count is printed."""
    tol_map = _parse_tol_map(tol_map)
    hf = hf_baseline(model)
    ids = encode_prompts(prompts, tokenizer, model.config.vocab_size)
    n = num_tokens_to_check
    ok = True
    for b, prompt in enumerate(ids):
        with torch.no_grad():
            seq = torch.tensor([prompt], device=model.device)
            toks = hf.generate(seq, max_new_tokens=n, min_new_tokens=n, do_sample=False, pad_token_id=0)[0].tolist()
        ours, routing = model.teacher_forced_logits(toks[:-1], routing=True)                           # [T-1, V]
        with torch.no_grad(), _FollowNearTies(hf, routing, routing_tol) as follow:
            base_logits = hf(torch.tensor([toks[:-1]], device=model.device)).logits[0]  # [T-1, V]
        if follow.followed:
            print(f"seq {b}: {follow.followed} router decision(s) at near ties follow the megakernel "
                  f"(largest baseline logit gap {follow.max_gap:.3g} <= {routing_tol})")
        check_from = len(prompt) - 1
        for t in range(check_from, len(toks) - 1):
            bl, ol = base_logits[t].float(), ours[t].float()
            for k, (atol, rtol) in tol_map.items():
                idx = torch.arange(bl.numel(), device=bl.device) if k is None else bl.topk(min(k, bl.numel())).indices
                err = (ol[idx] - bl[idx]).abs().max().item()
                lim = atol + rtol * bl[idx].abs().max().item()
                if err > lim:
                    ok = False
                    print(f"seq {b} step {t - check_from}: top-{k} max err {err:.4g} > {lim:.4g}")
            if ol.argmax() != bl.argmax():
                gap = (bl.max() - bl[ol.argmax()]).item()
                print(f"seq {b} step {t - check_from}: greedy token differs (baseline logit gap {gap:.4g})")
    print(f"Validation {'passed' if ok else 'failed'}.")
    return ok


def benchmark_sampling(model, prompts_ids: List[List[int]], max_new_tokens: int, iters: int) -> Dict:
    """End-to-end generation latency (ms, host clock, device synchronised) and throughput
    (generated tokens / s) over ``iters`` runs after one warm-up (reference ``main.py`` report
    keys ``e2e_model.latency_ms_p99`` / ``throughput``)."""
    model.generate(prompts_ids, max_new_tokens)
    lat = []
    for _ in range(iters):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.generate(prompts_ids, max_new_tokens)
        torch.cuda.synchronize()
        lat.append((time.perf_counter() - t0) * 1e3)
    lat.sort()
    p = lambda q: lat[min(len(lat) - 1, int(round(q * (len(lat) - 1))))]  # noqa: E731
    toks = max_new_tokens * len(prompts_ids)
    return {"e2e_model": {"latency_ms_p50": p(0.5), "latency_ms_p99": p(0.99), "latency_ms_avg": sum(lat) / len(lat),
                          "throughput": toks / (sum(lat) / len(lat) / 1e3)}}


def main(argv=None):
    args = parse_args(argv)
    if not args.prompts:
        args.prompts = ["I believe the meaning of life is"]
    args.batch_size = args.batch_size or len(args.prompts)
    if args.batch_size != len(args.prompts):
        raise SystemExit("--batch-size must equal the number of prompts")
    rank, world, args._device = init_distributed(args)
    mod_name, cls_name = _MODEL_REGISTRY[args.model]
    model_cls = getattr(importlib.import_module(mod_name), cls_name)
    torch.manual_seed(args.seed)
    # every rank steps the kernel (the ranks exchange partial sums inside each step); rank 0 prints
    quiet = contextlib.redirect_stdout(io.StringIO()) if rank != 0 else contextlib.nullcontext()
    rc = 0
    with quiet:
        model, tokenizer = prepare_inference(model_cls, args)
        ids = encode_prompts(args.prompts, tokenizer, model.config.vocab_size)
        max_new = args.max_new_tokens or max(1, args.seq_len - max(len(i) for i in ids) - 1)
        n_check = args.num_tokens_to_check or min(max_new, 16)

        if args.mode == "generate":
            run_generation(model, tokenizer, args.prompts, max_new)
        elif args.mode == "validate":
            passed = run_accuracy_check(model, tokenizer, args.prompts, args.tol_map, n_check,
                                       args.routing_divergence_tol)
            rc = 0 if passed else 1
        elif args.mode == "evaluate_single":
            accuracy = 1 if run_accuracy_check(model, tokenizer, args.prompts, args.tol_map, n_check,
                                       args.routing_divergence_tol) else 0
            report = benchmark_sampling(model, ids, max_new, args.benchmark_iters)
            print(f"Prompt: {args.prompts[0]}\n"
                  f"\tAccuracy: {accuracy}\n"
                  f"\tLatency: {report['e2e_model']['latency_ms_p99']}\n"
                  f"\tThroughput: {report['e2e_model']['throughput']}\n"
                  f"\tCustom-kernel FLOPs ratio: 1.0 (every decode-step op runs inside the megakernel)")
    if world > 1:
        import torch.distributed as dist  # noqa: PLC0415

        flag = torch.tensor([rc], device=args._device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)  # a failure on any rank fails every rank
        rc = int(flag.item())
        model.close()
        dist.barrier()
        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
