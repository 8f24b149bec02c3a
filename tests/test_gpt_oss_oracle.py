"""CPU pinning of the GPT-OSS oracle (``oracle/gpt_oss_oracle.py``) against Hugging Face
``transformers`` 5.5.0 ``GptOssForCausalLM`` (the model NxDI's ``modeling_gpt_oss`` restates;
the reference validates its megakernel against it).

A seeded tiny model (hidden 256, 4 query / 2 KV heads of 64, 4 experts top-2, intermediate 128,
one sliding-window layer of window 8 and one full layer, YaRN RoPE, attention sinks, biases)
with MXFP4 expert weights: Hugging Face runs the whole prompt at once, the oracle decodes it one
token per step through a paged K/V cache; every position's logits must agree.  Also: the YaRN
tables against Hugging Face's rotary embedding, MXFP4 dequantisation known answers.
"""
import torch

from oracle import gpt_oss_oracle as G


def _tiny():
    cfg = G.GptOssConfig(hidden=256, n_q_heads=4, n_kv_heads=2, head_dim=64, n_experts=4, top_k=2, inter=128,
                         n_layers=2, vocab=128, sliding_window=8)
    gen = torch.Generator().manual_seed(77)
    layers = [G.random_layer(cfg, gen) for _ in range(cfg.n_layers)]
    embed = torch.randn(cfg.vocab, cfg.hidden, generator=gen).to(torch.bfloat16)
    fnorm = (1 + 0.02 * torch.randn(cfg.hidden, generator=gen)).to(torch.bfloat16)
    lm = (0.02 * torch.randn(cfg.vocab, cfg.hidden, generator=gen)).to(torch.bfloat16)
    return cfg, layers, embed, fnorm, lm


def _hf_model(cfg, layers, embed, fnorm, lm):
    from transformers import GptOssConfig, GptOssForCausalLM

    hc = GptOssConfig(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.inter,
                      num_hidden_layers=cfg.n_layers, num_attention_heads=cfg.n_q_heads,
                      num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, num_local_experts=cfg.n_experts,
                      num_experts_per_tok=cfg.top_k, sliding_window=cfg.sliding_window, rms_norm_eps=cfg.rms_eps,
                      tie_word_embeddings=False, max_position_embeddings=4096,
                      rope_parameters={"rope_type": "yarn", "factor": cfg.rope_factor, "beta_fast": cfg.rope_beta_fast,
                                       "beta_slow": cfg.rope_beta_slow, "truncate": False,
                                       "original_max_position_embeddings": cfg.rope_original_max,
                                       "rope_theta": cfg.rope_theta})
    hc._attn_implementation = "eager"
    m = GptOssForCausalLM(hc).float().eval()
    sd = {"model.embed_tokens.weight": embed, "model.norm.weight": fnorm, "lm_head.weight": lm}
    for i, lw in enumerate(layers):
        p = f"model.layers.{i}."
        sd.update({p + "self_attn.q_proj.weight": lw.wq, p + "self_attn.q_proj.bias": lw.bq,
                   p + "self_attn.k_proj.weight": lw.wk, p + "self_attn.k_proj.bias": lw.bk,
                   p + "self_attn.v_proj.weight": lw.wv, p + "self_attn.v_proj.bias": lw.bv,
                   p + "self_attn.o_proj.weight": lw.wo, p + "self_attn.o_proj.bias": lw.bo,
                   p + "self_attn.sinks": lw.sinks, p + "input_layernorm.weight": lw.ln1,
                   p + "post_attention_layernorm.weight": lw.ln2, p + "mlp.router.weight": lw.router,
                   p + "mlp.router.bias": lw.router_b,
                   p + "mlp.experts.gate_up_proj": G.mx_dequant(lw.gu_codes, lw.gu_scales).transpose(1, 2),
                   p + "mlp.experts.gate_up_proj_bias": lw.gu_b,
                   p + "mlp.experts.down_proj": G.mx_dequant(lw.dn_codes, lw.dn_scales).transpose(1, 2),
                   p + "mlp.experts.down_proj_bias": lw.dn_b})
    missing, unexpected = m.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    assert not missing, missing
    return m


def test_mx_dequant_known_answers():
    codes = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 15, 13] + [2] * 20], dtype=torch.uint8)
    v = G.mx_dequant(codes, torch.tensor([[128]], dtype=torch.uint8))  # scale 2
    assert v[0, :12].tolist() == [0.0, 1.0, 2.0, 3.0, 4.0, 6.0, 8.0, 12.0, 0.0, -1.0, -12.0, -6.0]
    assert G.mx_dequant(codes, torch.tensor([[127]], dtype=torch.uint8))[0, 7] == 6.0


def test_yarn_tables_match_hf():
    from transformers import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssRotaryEmbedding

    cfg = G.GptOssConfig()
    hc = GptOssConfig()
    rot = GptOssRotaryEmbedding(hc)
    pos = torch.arange(0, 5000, 37)[None]
    c_hf, s_hf = rot(torch.zeros(1, dtype=torch.float32), pos)
    c, s = G.rope_tables(cfg, 5000)
    assert torch.allclose(c[pos[0]], c_hf[0], atol=1e-6) and torch.allclose(s[pos[0]], s_hf[0], atol=1e-6)


def test_oracle_decode_matches_hf_prefill():
    cfg, layers, embed, fnorm, lm = _tiny()
    m = _hf_model(cfg, layers, embed, fnorm, lm)
    g = torch.Generator().manual_seed(5)
    toks = torch.randint(0, cfg.vocab, (19,), generator=g)
    with torch.no_grad():
        ref = m(toks[None]).logits[0].float()
    NB = 4
    table = torch.tensor([[2, 0, 3, 1]], dtype=torch.int32)
    kc = [torch.zeros(NB, cfg.n_kv_heads, cfg.block_size, cfg.head_dim) for _ in range(cfg.n_layers)]
    vc = [torch.zeros_like(kc[0]) for _ in range(cfg.n_layers)]
    cos, sin = G.rope_tables(cfg, 64)
    for p in range(len(toks)):
        x = embed[toks[p:p + 1].long()]
        _, lg = G.decode_step(x, layers, cfg, kc, vc, torch.tensor([p]), table, cos, sin, fnorm, lm)
        err = (lg[0] - ref[p]).abs().max().item()
        assert err < 1e-4, (p, err)
