"""Generate the golden fixtures that pin the CPU oracle.

The reference repository ships no tests, fixtures or known-answer vectors for the decode
path, and its own PyTorch baseline (NxDI ``modeling_qwen3_moe``) cannot be imported here.
The model definition that baseline converts from is Hugging Face ``transformers``
Qwen3-MoE (the reference loads ``Qwen3MoeForCausalLM`` in
``megakernels/qwen3_moe/qwen_with_megakernel.py:606-608``), which is installed
(transformers 5.5.0).  This script runs that implementation on a tiny seeded model and
records:

* per sequence: a prefill of ``P_b`` tokens (which fills HF's KV cache), then one decode
  token; the KV cache after the prefill, the decoder-layer outputs of the decode token and
  its logits;
* a standalone sparse-MoE block call (router logits, top-k indices, top-k weights, output).

Output: ``tests/golden/qwen3_moe_tiny.pt`` (~2.5 MB).  Run from the repo root:
``python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import os

import torch
from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qwen3_moe_tiny.pt")


def build_model(seed: int = 1234):
    cfg = Qwen3MoeConfig(
        vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, num_experts=8,
        num_experts_per_tok=2, moe_intermediate_size=32, norm_topk_prob=True,
        rms_norm_eps=1e-6, rope_parameters={"rope_theta": 1e6, "rope_type": "default"},
        max_position_embeddings=4096, tie_word_embeddings=False, decoder_sparse_step=1,
        mlp_only_layers=[], attention_bias=False,
    )
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = Qwen3MoeForCausalLM(cfg).eval()
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                v = 1.0 + 0.02 * torch.randn(p.shape, generator=gen)
            elif "embed_tokens" in name:
                v = torch.randn(p.shape, generator=gen)
            else:
                v = 0.02 * torch.randn(p.shape, generator=gen)
            # weights are bf16 values; HF runs them in fp32 (the fp32 evaluation)
            p.copy_(v.to(torch.bfloat16).to(torch.float32))
    return cfg, model


def main():
    cfg, model = build_model()
    gen = torch.Generator().manual_seed(99)
    prefix_lens = [5, 130, 141]          # crosses block boundaries of a 128-token page
    seqs = []
    with torch.no_grad():
        for P in prefix_lens:
            ids = torch.randint(0, cfg.vocab_size, (1, P + 1), generator=gen)
            out = model(input_ids=ids[:, :P], use_cache=True)
            cache = out.past_key_values
            keys = [cache.layers[i].keys[0].clone() for i in range(cfg.num_hidden_layers)]
            vals = [cache.layers[i].values[0].clone() for i in range(cfg.num_hidden_layers)]
            layer_outs = []
            hooks = [layer.register_forward_hook(
                lambda m, a, o: layer_outs.append((o[0] if isinstance(o, tuple) else o).clone()))
                for layer in model.model.layers]
            dec = model(input_ids=ids[:, P:P + 1], past_key_values=cache, use_cache=True)
            for h in hooks:
                h.remove()
            seqs.append({
                "prefix_len": P, "new_id": int(ids[0, P]),
                "keys": [k.to(torch.float32) for k in keys],     # [nkv, P, 128] post-norm+RoPE
                "values": [v.to(torch.float32) for v in vals],   # [nkv, P, 128]
                "layer_out": [lo[0, -1].to(torch.float32) for lo in layer_outs],  # [H]
                "logits": dec.logits[0, -1].to(torch.float32),
            })
        # standalone MoE block (router_topk + experts) on T=6 tokens
        moe = model.model.layers[0].mlp
        x = torch.randn(6, cfg.hidden_size, generator=gen).to(torch.bfloat16).to(torch.float32)
        logits_sm, w, idx = moe.gate(x)
        y = moe.experts(x, idx, w)
    state = {k: v.to(torch.bfloat16) for k, v in model.state_dict().items()}
    torch.save({
        "config": cfg.to_dict(),
        "state_dict": state,
        "seqs": seqs,
        "moe": {"x": x, "router_probs": logits_sm, "topk_idx": idx, "topk_w": w, "out": y},
    }, OUT)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
