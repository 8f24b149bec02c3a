"""CPU tests of the GPT-OSS host layer: MXFP4 conversion (checkpoint blocks, quantisation) and
the Hugging Face -> kernel converter of the model class."""
import torch

from nki_moe_megakernel_b200.megakernels.gpt_oss import gpt_oss_with_megakernel as gm
from oracle import gpt_oss_oracle as G


def test_unpack_blocks_low_nibble_first():
    blocks = torch.tensor([[[0x21] + [0] * 15]], dtype=torch.uint8)  # codes 1 then 2
    codes = gm.unpack_mxfp4_blocks(blocks)
    assert codes.shape == (1, 32) and codes[0, 0] == 1 and codes[0, 1] == 2


def test_quantize_round_trips_representable_values():
    g = torch.Generator().manual_seed(3)
    codes, scales = G.random_mx((4, 64, 96), g)
    x = G.mx_dequant(codes, scales)
    c2, s2 = gm.quantize_mxfp4(x)
    assert torch.equal(G.mx_dequant(c2, s2), x)
    assert torch.equal(gm.mxfp4_dequant(codes, scales), x)


def test_quantize_rounds_to_nearest_even():
    x = torch.zeros(1, 32)
    x[0, :6] = torch.tensor([6.0, 2.5, 0.25, -1.25, 5.0, 7.0])  # scale 1 (amax 7 -> exp 0)
    c, s = gm.quantize_mxfp4(x)
    v = gm.mxfp4_dequant(c, s)[0, :6].tolist()
    assert int(s[0, 0]) == 127
    assert v == [6.0, 2.0, 0.0, -1.0, 4.0, 6.0]


def test_converter_matches_the_layer_tensors():
    cfg = G.GptOssConfig(hidden=256, n_q_heads=4, n_kv_heads=2, n_experts=4, top_k=2, inter=128, n_layers=2,
                         vocab=128)
    gen = torch.Generator().manual_seed(9)
    lws = [G.random_layer(cfg, gen) for _ in range(2)]
    sd = {"model.embed_tokens.weight": torch.zeros(128, 256), "model.norm.weight": torch.ones(256),
          "lm_head.weight": torch.ones(128, 256)}
    for i, lw in enumerate(lws):
        p = f"model.layers.{i}."
        for name, key in (("q_proj.weight", "wq"), ("q_proj.bias", "bq"), ("k_proj.weight", "wk"),
                          ("k_proj.bias", "bk"), ("v_proj.weight", "wv"), ("v_proj.bias", "bv"),
                          ("o_proj.weight", "wo"), ("o_proj.bias", "bo"), ("sinks", "sinks")):
            sd[p + "self_attn." + name] = getattr(lw, key)
        sd[p + "input_layernorm.weight"], sd[p + "post_attention_layernorm.weight"] = lw.ln1, lw.ln2
        sd[p + "mlp.router.weight"], sd[p + "mlp.router.bias"] = lw.router, lw.router_b
        gu, dn = lw.gu_codes, lw.dn_codes
        sd[p + "mlp.experts.gate_up_proj_blocks"] = (gu[..., 0::2] | (gu[..., 1::2] << 4)).view(4, 256, 8, 16)
        sd[p + "mlp.experts.gate_up_proj_scales"] = lw.gu_scales
        sd[p + "mlp.experts.down_proj_blocks"] = (dn[..., 0::2] | (dn[..., 1::2] << 4)).view(4, 256, 4, 16)
        sd[p + "mlp.experts.down_proj_scales"] = lw.dn_scales
        sd[p + "mlp.experts.gate_up_proj_bias"], sd[p + "mlp.experts.down_proj_bias"] = lw.gu_b, lw.dn_b
    nc = gm.GptOssV1MultilayerNeuronConfig()
    c = gm.GptOssInferenceConfig(nc, hidden_size=256, num_hidden_layers=2)
    out = gm.convert_gpt_oss_hf_to_neuron_state_dict(sd, c)
    for i, lw in enumerate(lws):
        for k in ("wq", "bq", "wo", "sinks", "router_b", "gu_codes", "gu_scales", "dn_codes", "dn_scales", "gu_b"):
            assert torch.equal(out[f"layers.{i}.{k}"], getattr(lw, k)), (i, k)
    # the bf16 route (Hugging Face in-memory gate_up_proj [E, H, 2I]) quantises to the same values
    p = "model.layers.0.mlp.experts."
    sd2 = dict(sd)
    for k in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales"):
        sd2.pop(p + k)
    sd2[p + "gate_up_proj"] = G.mx_dequant(lws[0].gu_codes, lws[0].gu_scales).transpose(1, 2)
    sd2[p + "down_proj"] = G.mx_dequant(lws[0].dn_codes, lws[0].dn_scales).transpose(1, 2)
    out2 = gm.convert_gpt_oss_hf_to_neuron_state_dict(sd2, c)
    assert torch.equal(G.mx_dequant(out2["layers.0.gu_codes"], out2["layers.0.gu_scales"]),
                       G.mx_dequant(lws[0].gu_codes, lws[0].gu_scales))
