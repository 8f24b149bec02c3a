"""GPU tests of the reference-facing model class and driver: the megakernel model against
Hugging Face ``Qwen3MoeForCausalLM`` (fp32) with the same weights."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qwen3_moe_tiny.pt")


def _tiny_model(batch=3, seq_len=300):
    from nki_moe_megakernel_b200.megakernels.qwen3_moe import qwen_with_megakernel as qm

    d = torch.load(GOLDEN, weights_only=False)
    c = d["config"]
    nc = qm.Qwen3MoEV3MultilayerNeuronConfig(batch_size=batch, seq_len=seq_len)
    cfg = qm.Qwen3MoeInferenceConfig(nc, **{k: v for k, v in c.items() if not k.startswith("_")})
    model = qm.NeuronQwen3MoeForCausalLM(None, cfg, device="cuda",
                                         state_dict={k: v.cuda() for k, v in d["state_dict"].items()})
    model.compile()
    model.load()
    return model


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.flatten().double(), b.flatten().double(), dim=0).item()


def test_teacher_forced_logits_vs_hf():
    """Prompt processed one position per decode step (crossing a 128-token K/V block) gives
    the logits of the HF full-sequence forward at every position."""
    from nki_moe_megakernel_b200.main import hf_baseline

    model = _tiny_model()
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, model.config.vocab_size, (140,), generator=g).tolist()
    ours = model.teacher_forced_logits(toks)
    hf = hf_baseline(model)
    with torch.no_grad():
        ref = hf(torch.tensor([toks], device="cuda")).logits[0].float()
    err = (ours - ref).abs().max().item()
    assert err < 2e-2, err
    assert _cos(ours, ref) > 0.999


def test_generate_mixed_prompt_lengths():
    """A batch mixing prompt reading and generation: each generated token is (within the
    tolerance) the HF greedy choice given the same prefix."""
    from nki_moe_megakernel_b200.main import hf_baseline

    model = _tiny_model()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 128, (n,), generator=g).tolist() for n in (1, 7, 130)]
    outs = model.generate(prompts, 12)
    assert [len(o) for o in outs] == [12, 12, 12]
    hf = hf_baseline(model)
    for p, o in zip(prompts, outs):
        seq = p + o
        with torch.no_grad():
            lg = hf(torch.tensor([seq[:-1]], device="cuda")).logits[0].float()
        for t, tok in enumerate(o):
            row = lg[len(p) - 1 + t]
            assert (row.max() - row[tok]).item() <= 2e-2, (t, tok, row.argmax().item())


def test_main_validate_random_init():
    from nki_moe_megakernel_b200 import main as drv

    rc = drv.main(["--mode", "validate", "--enable-nki", "--num-layers", "2", "--seq-len", "96",
                   "--num-tokens-to-check", "8", "--prompt", "I believe the meaning of life is"])
    assert rc == 0


def test_model_from_safetensors_checkpoint_vs_hf_from_pretrained(tmp_path):
    """The checkpoint route of the reference: a Hugging Face directory (config.json +
    safetensors) loaded by the model class from ``model_path``, against the same directory
    loaded with ``Qwen3MoeForCausalLM.from_pretrained`` (fp32), teacher-forced logits."""
    from transformers import Qwen3MoeForCausalLM

    from nki_moe_megakernel_b200.megakernels.qwen3_moe import qwen_with_megakernel as qm
    from tests.test_host_mirror import _save_tiny_checkpoint

    _save_tiny_checkpoint(tmp_path)
    nc = qm.Qwen3MoEV3MultilayerNeuronConfig(batch_size=1, seq_len=200)
    cfg = qm.Qwen3MoeInferenceConfig(nc, load_config=qm.load_pretrained_config(str(tmp_path)))
    model = qm.NeuronQwen3MoeForCausalLM(str(tmp_path), cfg, device="cuda")
    model.compile()
    model.load()
    g = torch.Generator().manual_seed(11)
    toks = torch.randint(0, cfg.vocab_size, (135,), generator=g).tolist()
    ours = model.teacher_forced_logits(toks)
    hf = Qwen3MoeForCausalLM.from_pretrained(str(tmp_path), torch_dtype=torch.float32).cuda().eval()
    with torch.no_grad():
        ref = hf(torch.tensor([toks], device="cuda")).logits[0].float()
    err = (ours - ref).abs().max().item()
    assert err < 2e-2, err
    assert _cos(ours, ref) > 0.999
