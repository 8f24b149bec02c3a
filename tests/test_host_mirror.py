"""CPU tests of the reference-facing host layer (config, checkpoint conversion, CLI plumbing)."""
import json
import os

import pytest
import torch

from nki_moe_megakernel_b200 import main as drv
from nki_moe_megakernel_b200.megakernels.qwen3_moe import qwen_with_megakernel as qm


def _tiny_cfg(**kw):
    nc = qm.Qwen3MoEV3MultilayerNeuronConfig(batch_size=2, seq_len=256)
    args = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, num_experts=8,
                num_experts_per_tok=2, moe_intermediate_size=32, num_hidden_layers=2, vocab_size=128)
    args.update(kw)
    return qm.Qwen3MoeInferenceConfig(nc, **args)


def test_registry_names_match_reference():
    assert qm.NeuronQwen3MoeForCausalLM is qm.NeuronQwen3MoeForCausalLMV3
    assert qm.NeuronQwen3MoeForCausalLM.get_neuron_config_cls() is qm.Qwen3MoEV3MultilayerNeuronConfig
    assert qm.NeuronQwen3MoeForCausalLM.get_config_cls() is qm.Qwen3MoeInferenceConfig
    mod, cls = drv._MODEL_REGISTRY["qwen3_moe"]
    assert mod.endswith("megakernels.qwen3_moe.qwen_with_megakernel") and cls == "NeuronQwen3MoeForCausalLM"


def test_neuron_config_blocks():
    nc = qm.Qwen3MoEV3MultilayerNeuronConfig(batch_size=4, seq_len=300)
    assert nc.max_batch_size == 4 and nc.pa_block_size == 128
    assert nc.pa_num_blocks == 4 * 3
    with pytest.raises(ValueError):
        qm.Qwen3MoEV3MultilayerNeuronConfig(torch_dtype=torch.float16)


def test_inference_config_from_json(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"hidden_size": 512, "num_local_experts": 16,
                                                      "rope_parameters": {"rope_theta": 5e5}}))
    cfg = qm.Qwen3MoeInferenceConfig(qm.Qwen3MoEV3MultilayerNeuronConfig(),
                                     load_config=qm.load_pretrained_config(str(tmp_path)))
    assert cfg.hidden_size == 512 and cfg.num_experts == 16 and cfg.rope_theta == 5e5
    s = cfg.shape()
    assert s.hidden_size == 512 and s.num_experts == 16 and s.block_size == 128
    with pytest.raises(ValueError):
        _tiny_cfg(norm_topk_prob=False)


def test_convert_per_expert_equals_fused():
    cfg = _tiny_cfg()
    fused = torch.load(os.path.join(os.path.dirname(__file__), "golden", "qwen3_moe_tiny.pt"),
                       weights_only=False)["state_dict"]
    per = {k: v for k, v in fused.items() if "mlp.experts" not in k}
    I = cfg.moe_intermediate_size
    for l in range(cfg.num_hidden_layers):
        gu = fused[f"model.layers.{l}.mlp.experts.gate_up_proj"]
        dn = fused[f"model.layers.{l}.mlp.experts.down_proj"]
        for e in range(cfg.num_experts):
            per[f"model.layers.{l}.mlp.experts.{e}.gate_proj.weight"] = gu[e, :I]
            per[f"model.layers.{l}.mlp.experts.{e}.up_proj.weight"] = gu[e, I:]
            per[f"model.layers.{l}.mlp.experts.{e}.down_proj.weight"] = dn[e]
    a = qm.convert_qwen3_moe_hf_to_neuron_state_dict(fused, cfg)
    b = qm.convert_qwen3_moe_hf_to_neuron_state_dict(per, cfg)
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert a["layers.1.wq"].shape == (512, 256) and a["layers.0.gate_up"].shape == (8, 64, 256)
    assert torch.equal(a["lm_head"], fused["lm_head.weight"])


def test_convert_fp8_block_dequant():
    cfg = _tiny_cfg(num_hidden_layers=0, quantization_config={"weight_block_size": [128, 128]})
    w = torch.ones(256, 256)
    scales = torch.tensor([[2.0, 3.0], [4.0, 5.0]])
    sd = {"model.embed_tokens.weight": w.clone(), "model.embed_tokens.weight_scale_inv": scales,
          "model.norm.weight": torch.ones(256)}
    out = qm.convert_qwen3_moe_hf_to_neuron_state_dict(sd, cfg)
    e = out["embed"].float()
    assert e[0, 0] == 2 and e[0, 200] == 3 and e[200, 0] == 4 and e[255, 255] == 5


def test_encode_prompts_and_args():
    ids = drv.encode_prompts(["ab", "hello"], None, 128)
    assert [len(i) for i in ids] == [2, 5] and all(0 <= t < 128 for s in ids for t in s)
    assert ids == drv.encode_prompts(["ab", "hello"], None, 128)
    a = drv.parse_args(["--mode", "validate", "--enable-nki", "--prompt", "x", "--num-layers", "2"])
    assert a.mode == "validate" and a.enable_nki and a.prompts == ["x"] and a.num_layers == 2
    tm = drv._parse_tol_map(drv.DEFAULT_TOL_MAP)
    assert tm[None] == (1e-5, 0.05) and tm[5] == (1e-5, 0.03)


def _save_tiny_checkpoint(path):
    """The golden tiny model written as a Hugging Face checkpoint (config.json + safetensors)."""
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    d = torch.load(os.path.join(os.path.dirname(__file__), "golden", "qwen3_moe_tiny.pt"), weights_only=False)
    cfg = Qwen3MoeConfig(**{k: v for k, v in d["config"].items() if not k.startswith("_")})
    model = Qwen3MoeForCausalLM(cfg)
    missing, _ = model.load_state_dict(d["state_dict"], strict=False)
    assert not missing, missing
    model.save_pretrained(str(path), safe_serialization=True)
    return d


def test_safetensors_checkpoint_loads_like_the_in_memory_state_dict(tmp_path):
    """A Hugging Face checkpoint directory (``save_pretrained``: config.json + *.safetensors, the
    files the reference loads with ``from_pretrained``, ``qwen_with_megakernel.py:606-608``) read
    by the model class gives the same config and, after conversion, the same tensors as the
    in-memory state dict."""
    d = _save_tiny_checkpoint(tmp_path)
    assert list(tmp_path.glob("*.safetensors")), "no safetensors written"
    nc = qm.Qwen3MoEV3MultilayerNeuronConfig(batch_size=1, seq_len=64)
    cfg = qm.Qwen3MoeInferenceConfig(nc, load_config=qm.load_pretrained_config(str(tmp_path)))
    c = d["config"]
    assert (cfg.hidden_size, cfg.num_experts, cfg.num_hidden_layers, cfg.vocab_size) == (
        c["hidden_size"], c.get("num_experts") or c["num_local_experts"], c["num_hidden_layers"], c["vocab_size"])
    model = qm.NeuronQwen3MoeForCausalLM(str(tmp_path), cfg, device="cpu")
    from_disk = qm.convert_qwen3_moe_hf_to_neuron_state_dict(model.hf_state_dict(), cfg)
    in_mem = qm.convert_qwen3_moe_hf_to_neuron_state_dict(d["state_dict"], cfg)
    assert from_disk.keys() == in_mem.keys()
    for k in in_mem:
        assert torch.equal(from_disk[k].to(in_mem[k].dtype), in_mem[k]), k
