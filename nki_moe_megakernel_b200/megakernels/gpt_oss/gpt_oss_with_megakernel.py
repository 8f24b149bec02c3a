"""GPT-OSS model with the B200 decode megakernel (drop-in for the reference module
``megakernels/gpt_oss/gpt_oss_with_megakernel.py``).

Same public names as the reference: ``GptOssV1MultilayerNeuronConfig`` (reference :239),
``convert_gpt_oss_hf_to_neuron_state_dict`` (:290-327), ``NeuronGptOssForCausalLM`` with
``get_neuron_config_cls`` / ``get_config_cls`` / ``convert_hf_to_neuron_state_dict`` (:693-710).

Token generation runs every decoder layer, the final norm and the LM head in ONE persistent
sm_100a kernel per step (``nkm_gptoss_decode_step``), writing each layer's K/V in place into a
paged cache (block 128).  Experts are MXFP4 (e2m1 codes + e8m0 scale per 32 inputs): an MXFP4
checkpoint (``*_blocks`` / ``*_scales``) is used as is, a bf16 one is quantised at load.
Prompts are fed through the decode kernel one position per step.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional, Sequence

import torch

from ...gpt_oss_engine import GptOssGpuLayer, GptOssMegakernel, GptOssShape

BF16 = torch.bfloat16
_E2M1_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


class GptOssV1MultilayerNeuronConfig:
    """Serving configuration (the subset of the reference's GptOssNeuronConfig the decode path
    uses); unknown keyword arguments are kept as attributes."""

    def __init__(self, batch_size: int = 1, max_batch_size: Optional[int] = None, seq_len: int = 640,
                 max_length: Optional[int] = None, tp_degree: int = 1, torch_dtype=BF16, pa_block_size: int = 128,
                 pa_num_blocks: Optional[int] = None, top_k: int = 1, do_sample: bool = False,
                 temperature: float = 1.0, top_p: float = 1.0, is_mxfp4_compute: bool = True, **kwargs):
        self.batch_size = batch_size
        self.max_batch_size = max_batch_size or batch_size
        self.seq_len = seq_len
        self.max_length = max_length or seq_len
        self.tp_degree = tp_degree
        self.torch_dtype = torch_dtype
        self.pa_block_size = pa_block_size
        nb = (self.max_length + pa_block_size) // pa_block_size
        self.pa_num_blocks = pa_num_blocks or self.max_batch_size * nb
        self.top_k, self.do_sample, self.temperature, self.top_p = top_k, do_sample, temperature, top_p
        self.is_mxfp4_compute = is_mxfp4_compute
        for k, v in kwargs.items():
            setattr(self, k, v)
        if tp_degree != 1:
            raise ValueError("the GPT-OSS decode megakernel runs on one GPU (tp_degree=1)")
        if self.max_batch_size > 16:
            raise ValueError("the GPT-OSS decode megakernel handles batches of at most 16")


def load_pretrained_config(model_path: Optional[str]):
    def _load(cfg):
        if model_path and os.path.exists(os.path.join(model_path, "config.json")):
            with open(os.path.join(model_path, "config.json")) as f:
                for k, v in json.load(f).items():
                    setattr(cfg, k, v)
    return _load


class GptOssInferenceConfig:
    """Model hyper-parameters (Hugging Face ``GptOssConfig`` names); defaults GPT-OSS-20B."""

    def __init__(self, neuron_config: GptOssV1MultilayerNeuronConfig, load_config=None, **kwargs):
        self.neuron_config = neuron_config
        self.hidden_size = 2880
        self.num_attention_heads = 64
        self.num_key_value_heads = 8
        self.head_dim = 64
        self.num_local_experts = 32
        self.num_experts_per_tok = 4
        self.intermediate_size = 2880
        self.num_hidden_layers = 24
        self.vocab_size = 201088
        self.rms_norm_eps = 1e-5
        self.sliding_window = 128
        self.swiglu_limit = 7.0
        self.max_position_embeddings = 131072
        self.rope_parameters = {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                "truncate": False, "original_max_position_embeddings": 4096, "rope_theta": 150000.0}
        self.layer_types = None
        if load_config is not None:
            load_config(self)
        for k, v in kwargs.items():
            setattr(self, k, v)
        if getattr(self, "rope_scaling", None) and not kwargs.get("rope_parameters"):
            self.rope_parameters = {**self.rope_parameters, **self.rope_scaling}
            self.rope_parameters.setdefault("rope_theta", getattr(self, "rope_theta", 150000.0))
        if not self.layer_types:
            self.layer_types = ["sliding_attention" if i % 2 == 0 else "full_attention"
                                for i in range(self.num_hidden_layers)]

    def shape(self) -> GptOssShape:
        rp = self.rope_parameters
        return GptOssShape(hidden_size=self.hidden_size, num_attention_heads=self.num_attention_heads,
                           num_key_value_heads=self.num_key_value_heads, head_dim=self.head_dim,
                           num_local_experts=self.num_local_experts, num_experts_per_tok=self.num_experts_per_tok,
                           intermediate_size=self.intermediate_size, num_hidden_layers=self.num_hidden_layers,
                           vocab_size=self.vocab_size, rms_norm_eps=self.rms_norm_eps,
                           sliding_window=self.sliding_window, rope_theta=rp.get("rope_theta", 150000.0),
                           rope_factor=rp.get("factor", 1.0),
                           rope_original_max=rp.get("original_max_position_embeddings", 4096),
                           rope_beta_fast=rp.get("beta_fast", 32.0), rope_beta_slow=rp.get("beta_slow", 1.0),
                           swiglu_limit=self.swiglu_limit, block_size=self.neuron_config.pa_block_size)


# ---------------------------------------------------------------------------
# MXFP4 conversion
# ---------------------------------------------------------------------------
def unpack_mxfp4_blocks(blocks: torch.Tensor) -> torch.Tensor:
    """Hugging Face / OpenAI ``*_blocks [..., K/32, 16]`` (two e2m1 codes per byte, low nibble
    first) -> codes ``[..., K]`` uint8."""
    lo, hi = blocks & 0x0F, blocks >> 4
    return torch.stack([lo, hi], dim=-1).reshape(*blocks.shape[:-2], -1).to(torch.uint8)


def quantize_mxfp4(w: torch.Tensor):
    """fp32/bf16 ``[..., K]`` -> (codes uint8 ``[..., K]``, e8m0 scales ``[..., K/32]``): OCP
    Microscaling conversion, shared exponent floor(log2(amax)) - 2 per 32 elements, elements
    rounded to the nearest e2m1 value (ties to the even code), saturated at 6."""
    x = w.float().reshape(*w.shape[:-1], -1, 32)
    amax = x.abs().amax(-1, keepdim=True)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax)) - 2, torch.full_like(amax, -127.0)).clamp(-127, 127)
    y = (x / torch.pow(2.0, e)).clamp(-6.0, 6.0)
    mag = _E2M1_MAG.to(x.device)
    d = (y.abs()[..., None] - mag).abs()
    best = d.min(-1, keepdim=True).values
    # nearest magnitude; on a tie the even code (mantissa bit 0) scores higher
    score = (d == best).to(torch.int64) * (2 - torch.arange(8, device=x.device) % 2)
    code = score.argmax(-1).to(torch.uint8)
    code = code | (((y < 0) & (code > 0)).to(torch.uint8) << 3)
    return code.reshape(w.shape), (e + 127).to(torch.uint8).squeeze(-1)


def convert_gpt_oss_hf_to_neuron_state_dict(state_dict: Dict[str, torch.Tensor], config) -> Dict[str, torch.Tensor]:
    """Normalise a Hugging Face GPT-OSS state dict to the per-layer tensors the kernel packs
    (reference converter :290-327 pre-bakes the same per-layer operands).  Experts: MXFP4
    checkpoint tensors (``gate_up_proj_blocks`` / ``_scales``, ``down_proj_blocks`` / ``_scales``)
    are unpacked; bf16 ``gate_up_proj [E, H, 2I]`` / ``down_proj [E, I, H]`` are quantised.
    Returned keys ``layers.{l}.{wq,bq,wk,bk,wv,bv,wo,bo,sinks,ln1,ln2,router,router_b,gu_codes,
    gu_scales,gu_b,dn_codes,dn_scales,dn_b}``, ``embed``, ``final_norm``, ``lm_head``."""
    sd = state_dict
    pre = "model." if any(k.startswith("model.") for k in sd) else ""
    out: Dict[str, torch.Tensor] = {}
    for l in range(config.num_hidden_layers):
        p, o = f"{pre}layers.{l}.", f"layers.{l}."
        a = p + "self_attn."
        for dst, src in (("wq", "q_proj.weight"), ("bq", "q_proj.bias"), ("wk", "k_proj.weight"),
                         ("bk", "k_proj.bias"), ("wv", "v_proj.weight"), ("bv", "v_proj.bias"),
                         ("wo", "o_proj.weight"), ("bo", "o_proj.bias"), ("sinks", "sinks")):
            out[o + dst] = sd[a + src]
        out[o + "ln1"] = sd[p + "input_layernorm.weight"]
        out[o + "ln2"] = sd[p + "post_attention_layernorm.weight"]
        out[o + "router"] = sd[p + "mlp.router.weight"]
        out[o + "router_b"] = sd[p + "mlp.router.bias"]
        x = p + "mlp.experts."
        if x + "gate_up_proj_blocks" in sd:
            out[o + "gu_codes"] = unpack_mxfp4_blocks(sd[x + "gate_up_proj_blocks"])
            out[o + "gu_scales"] = sd[x + "gate_up_proj_scales"].to(torch.uint8)
            out[o + "dn_codes"] = unpack_mxfp4_blocks(sd[x + "down_proj_blocks"])
            out[o + "dn_scales"] = sd[x + "down_proj_scales"].to(torch.uint8)
        else:
            out[o + "gu_codes"], out[o + "gu_scales"] = quantize_mxfp4(sd[x + "gate_up_proj"].transpose(1, 2))
            out[o + "dn_codes"], out[o + "dn_scales"] = quantize_mxfp4(sd[x + "down_proj"].transpose(1, 2))
        out[o + "gu_b"] = sd[x + "gate_up_proj_bias"]
        out[o + "dn_b"] = sd[x + "down_proj_bias"]
    out["embed"] = sd[pre + "embed_tokens.weight"]
    out["final_norm"] = sd[pre + "norm.weight"]
    out["lm_head"] = sd.get("lm_head.weight", out["embed"])
    return out


def mxfp4_dequant(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 values of MXFP4 codes ``[..., K]`` with e8m0 scales ``[..., K/32]``."""
    mag = _E2M1_MAG.to(codes.device)
    v = mag[(codes & 7).long()] * torch.where((codes & 8) > 0, -1.0, 1.0)
    s = torch.pow(2.0, scales.float() - 127.0)
    return (v.view(*codes.shape[:-1], -1, 32) * s[..., None]).reshape(codes.shape)


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------
class NeuronGptOssForCausalLM:
    """GPT-OSS CausalLM whose token-generation step is one megakernel launch.
    ``model_path=None`` builds seeded random-init weights (MXFP4 experts) of the configured shape."""

    def __init__(self, model_path: Optional[str], config: GptOssInferenceConfig, device=None, seed: int = 0,
                 state_dict: Optional[Dict[str, torch.Tensor]] = None):
        self.model_path, self.state_dict, self.config = model_path, state_dict, config
        self.neuron_config = config.neuron_config
        self.device = torch.device(device if device is not None else "cuda")
        self.seed = seed
        self._layers: List[GptOssGpuLayer] = []
        self._head: Dict[str, torch.Tensor] = {}
        self.kernel: Optional[GptOssMegakernel] = None

    @classmethod
    def get_neuron_config_cls(cls):
        return GptOssV1MultilayerNeuronConfig

    @classmethod
    def get_config_cls(cls):
        return GptOssInferenceConfig

    @staticmethod
    def convert_hf_to_neuron_state_dict(state_dict: dict, config) -> dict:
        return convert_gpt_oss_hf_to_neuron_state_dict(state_dict, config)

    def _random_hf_state_dict(self) -> Dict[str, torch.Tensor]:
        """Seeded random-init weights in the MXFP4 checkpoint layout (on the model's device)."""
        c, dev = self.config, self.device
        g = torch.Generator(device=dev).manual_seed(self.seed)
        H, D, E, I = c.hidden_size, c.head_dim, c.num_local_experts, c.intermediate_size
        nq, nkv = c.num_attention_heads, c.num_key_value_heads

        def n(*s, std=0.02):
            return (torch.randn(*s, generator=g, device=dev) * std).to(BF16)

        def one(*s):
            return (1.0 + torch.randn(*s, generator=g, device=dev) * 0.02).to(BF16)

        def mx(rows, k):
            codes = torch.randint(0, 16, (E, rows, k), generator=g, device=dev, dtype=torch.uint8)
            blocks = (codes[..., 0::2] | (codes[..., 1::2] << 4)).view(E, rows, k // 32, 16)
            scales = torch.randint(119, 122, (E, rows, k // 32), generator=g, device=dev, dtype=torch.uint8)
            return blocks, scales

        sd = {"model.embed_tokens.weight": torch.randn(c.vocab_size, H, generator=g, device=dev).to(BF16),
              "model.norm.weight": one(H), "lm_head.weight": n(c.vocab_size, H)}
        for l in range(c.num_hidden_layers):
            p = f"model.layers.{l}."
            sd.update({p + "self_attn.q_proj.weight": n(nq * D, H), p + "self_attn.q_proj.bias": n(nq * D),
                       p + "self_attn.k_proj.weight": n(nkv * D, H), p + "self_attn.k_proj.bias": n(nkv * D),
                       p + "self_attn.v_proj.weight": n(nkv * D, H), p + "self_attn.v_proj.bias": n(nkv * D),
                       p + "self_attn.o_proj.weight": n(H, nq * D), p + "self_attn.o_proj.bias": n(H),
                       p + "self_attn.sinks": n(nq, std=1.0), p + "input_layernorm.weight": one(H),
                       p + "post_attention_layernorm.weight": one(H), p + "mlp.router.weight": n(E, H),
                       p + "mlp.router.bias": n(E), p + "mlp.experts.gate_up_proj_bias": n(E, 2 * I),
                       p + "mlp.experts.down_proj_bias": n(E, H)})
            sd[p + "mlp.experts.gate_up_proj_blocks"], sd[p + "mlp.experts.gate_up_proj_scales"] = mx(2 * I, H)
            sd[p + "mlp.experts.down_proj_blocks"], sd[p + "mlp.experts.down_proj_scales"] = mx(H, I)
        return sd

    def hf_state_dict(self) -> Dict[str, torch.Tensor]:
        if self.state_dict is not None:
            return self.state_dict
        if self.model_path:
            from safetensors.torch import load_file  # noqa: PLC0415

            import glob  # noqa: PLC0415

            sd: Dict[str, torch.Tensor] = {}
            for f in sorted(glob.glob(os.path.join(self.model_path, "*.safetensors"))):
                sd.update(load_file(f))
            return sd
        return self._random_hf_state_dict()

    def compile(self, compiled_model_path: Optional[str] = None, debug: bool = False):
        if self._layers:
            return
        sd = self.convert_hf_to_neuron_state_dict(self.hf_state_dict(), self.config)
        keys = ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "sinks", "ln1", "ln2", "router", "router_b",
                "gu_codes", "gu_scales", "gu_b", "dn_codes", "dn_scales", "dn_b")
        for l in range(self.config.num_hidden_layers):
            t = {k: sd.pop(f"layers.{l}.{k}").to(self.device) for k in keys}
            self._layers.append(GptOssGpuLayer(t, self.config.layer_types[l] == "sliding_attention"))
        self._head = {k: sd[k].to(self.device) for k in ("embed", "final_norm", "lm_head")}

    def load(self, compiled_model_path: Optional[str] = None):
        if not self._layers:
            self.compile(compiled_model_path)
        nc = self.neuron_config
        self.kernel = GptOssMegakernel(self.config.shape(), self._layers, max_batch=nc.max_batch_size,
                                       num_blocks=nc.pa_num_blocks, max_context=nc.max_length + 1,
                                       final_norm=self._head["final_norm"], lm_head=self._head["lm_head"],
                                       embed=self._head["embed"], device=self.device)
        self.reset()

    def close(self):
        if self.kernel is not None:
            self.kernel.close()
            self.kernel = None

    def reset(self):
        nc = self.neuron_config
        nb = (nc.max_length + nc.pa_block_size) // nc.pa_block_size
        self.block_table = torch.arange(nc.max_batch_size * nb, dtype=torch.int32, device=self.device).view(
            nc.max_batch_size, nb)

    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
        if self.kernel is None:
            raise RuntimeError("call load() first")
        ids = input_ids.to(self.device, torch.int32).view(-1)
        pos = position_ids.to(self.device, torch.int32).view(-1)
        return self.kernel.decode_step(pos, self.block_table[:ids.shape[0]], input_ids=ids)["logits"]

    def teacher_forced_logits(self, tokens: Sequence[int], routing: bool = False):
        """Every position's logits ``[len(tokens), vocab]`` fp32 (one decode step per position);
        with ``routing`` also the expert indices ``[len(tokens), layers, top_k]``."""
        self.reset()
        out, rt = [], []
        for i, t in enumerate(tokens):
            ids = torch.tensor([t], dtype=torch.int32, device=self.device)
            pos = torch.tensor([i], dtype=torch.int32, device=self.device)
            res = self.kernel.decode_step(pos, self.block_table[:1], input_ids=ids, trace=routing)
            out.append(res["logits"])
            if routing:
                rt.append(res["topk_idx"].transpose(0, 1))
        self.kernel.check_status()
        return (torch.cat(out, 0), torch.cat(rt, 0)) if routing else torch.cat(out, 0)

    def sample(self, logits: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        from ...engine import sample_tokens  # noqa: PLC0415

        nc = self.neuron_config
        greedy = not nc.do_sample or nc.top_k <= 1
        return sample_tokens(logits, positions.to(self.device, torch.int32), top_k=1 if greedy else min(nc.top_k, 64),
                             top_p=float(nc.top_p), temperature=float(nc.temperature), seed=self.seed)

    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int) -> List[List[int]]:
        """Prompt tokens one position per step (each sequence at its own position), then sampled
        tokens."""
        self.reset()
        B = len(prompts)
        lens = [len(p) for p in prompts]
        if min(lens) == 0:
            raise ValueError("empty prompt")
        outs: List[List[int]] = [[] for _ in range(B)]
        cur = [int(p[0]) for p in prompts]
        pos = [0] * B
        while any(len(o) < max_new_tokens for o in outs):
            pt = torch.tensor(pos, dtype=torch.int32)
            nxt = self.sample(self.forward(torch.tensor(cur, dtype=torch.int32), pt), pt).tolist()
            for b in range(B):
                pos[b] += 1
                if pos[b] < lens[b]:
                    cur[b] = int(prompts[b][pos[b]])
                elif len(outs[b]) < max_new_tokens:
                    outs[b].append(int(nxt[b]))
                    cur[b] = int(nxt[b])
        self.kernel.check_status()
        return outs
