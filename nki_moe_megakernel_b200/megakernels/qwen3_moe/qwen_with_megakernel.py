"""Qwen3-MoE model with the B200 decode megakernel (drop-in for the reference module
``megakernels/qwen3_moe/qwen_with_megakernel.py``).

Same public names as the reference: ``Qwen3MoEV3MultilayerNeuronConfig`` (reference
:102-132), ``convert_qwen3_moe_hf_to_neuron_state_dict`` (:171-271),
``NeuronQwen3MoeForCausalLMV3`` with ``get_neuron_config_cls`` / ``get_config_cls`` /
``convert_hf_to_neuron_state_dict`` / ``compile`` / ``load`` (:601-695) and the alias
``NeuronQwen3MoeForCausalLM`` (:728).

Token generation (TKG) runs every decoder layer, the final norm and the LM head in ONE
persistent sm_100a kernel per step (``libnkimoe.so``, C ABI ``include/nkimoe.h``), writing
each layer's K/V in place into a paged cache (block 128).  With ``tp_degree`` = N > 1 (one
process per GPU, ``torch.distributed`` initialised by the caller, e.g. ``torchrun``) every rank
holds its KV-head group and 1/N of the experts and the kernels exchange partial sums over
NVLink inside each step (the reference's TP replica groups, ``qwen_with_megakernel.py:360-362``).  Prompt tokens are fed through the
same decode kernel one position per step (per-sequence positions), so a batch can mix
sequences that are still reading their prompt with sequences that are generating.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Dict, List, Optional, Sequence

import torch

from ...engine import GpuLayer, Qwen3MoeMegakernel, Qwen3MoeShape
from ...sharding import XchgRegion, plan_shard, shard_attention, shard_experts, xchg_bytes

BF16 = torch.bfloat16


# ---------------------------------------------------------------------------
# configs
# ---------------------------------------------------------------------------
class Qwen3MoEV3MultilayerNeuronConfig:
    """Serving configuration (the subset of the reference's MoENeuronConfig that the decode
    path uses).  Unknown keyword arguments are kept as attributes, like NxDI's config."""

    def __init__(self, batch_size: int = 1, max_batch_size: Optional[int] = None, seq_len: int = 640,
                 max_context_length: Optional[int] = None, max_length: Optional[int] = None,
                 tp_degree: int = 1, moe_ep_degree: int = 1, moe_tp_degree: int = 1,
                 torch_dtype=BF16, pa_block_size: int = 128, pa_num_blocks: Optional[int] = None,
                 top_k: int = 1, do_sample: bool = False, temperature: float = 1.0,
                 prefill_chunk_size: int = 32, **kwargs):
        self.batch_size = batch_size
        self.max_batch_size = max_batch_size or batch_size
        self.seq_len = seq_len
        self.max_context_length = max_context_length or seq_len
        self.max_length = max_length or seq_len
        self.tp_degree = tp_degree
        self.moe_ep_degree = moe_ep_degree
        self.moe_tp_degree = moe_tp_degree
        self.torch_dtype = torch_dtype
        self.pa_block_size = pa_block_size
        blocks_per_seq = (self.max_length + pa_block_size) // pa_block_size
        self.pa_num_blocks = pa_num_blocks or self.max_batch_size * blocks_per_seq
        self.top_k = top_k
        self.do_sample = do_sample
        self.temperature = temperature
        # prompt tokens processed per launch (rows of one launch, at most 32): the kernel instance
        # is sized for max(max_batch_size, prefill_chunk_size) rows
        if not 1 <= prefill_chunk_size <= 32:
            raise ValueError("prefill_chunk_size must be in 1..32")
        self.prefill_chunk_size = prefill_chunk_size
        for k, v in kwargs.items():
            setattr(self, k, v)
        if torch_dtype not in (BF16, "bfloat16"):
            raise ValueError("the decode megakernel computes in bf16")
        if tp_degree < 1 or tp_degree > 8:
            raise ValueError("tp_degree must be in 1..8 (GPUs of one node)")
        # experts are always expert-parallel over the tensor-parallel ranks (128/N per GPU); an
        # expert-parallel degree other than 1 or tp_degree has no layout here
        if moe_ep_degree not in (1, tp_degree):
            raise ValueError("moe_ep_degree must be 1 or equal to tp_degree (experts are split over the TP ranks)")
        if moe_tp_degree != 1:
            raise ValueError("expert tensor parallelism is not used: experts are expert-parallel over the TP ranks")


def load_pretrained_config(model_path: Optional[str]):
    """Return a callable that fills a config from ``<model_path>/config.json`` (reference
    ``main.py`` passes ``load_config=load_pretrained_config(model_path)``)."""

    def _load(cfg):
        if model_path and os.path.exists(os.path.join(model_path, "config.json")):
            with open(os.path.join(model_path, "config.json")) as f:
                d = json.load(f)
            for k, v in d.items():
                setattr(cfg, k, v)
    return _load


class Qwen3MoeInferenceConfig:
    """Model hyper-parameters (Hugging Face ``Qwen3MoeConfig`` names).  Defaults are
    Qwen3-30B-A3B.  Router in fp32, softmax, top-k renormalised (reference ``qwen.py:251-277``)."""

    def __init__(self, neuron_config: Qwen3MoEV3MultilayerNeuronConfig, load_config=None, **kwargs):
        self.neuron_config = neuron_config
        self.hidden_size = 2048
        self.num_attention_heads = 32
        self.num_key_value_heads = 4
        self.head_dim = 128
        self.num_experts = 128
        self.num_experts_per_tok = 8
        self.moe_intermediate_size = 768
        self.num_hidden_layers = 48
        self.vocab_size = 151936
        self.rms_norm_eps = 1e-6
        self.rope_theta = 1e6
        self.max_position_embeddings = 40960
        self.norm_topk_prob = True
        self.tie_word_embeddings = False
        if load_config is not None:
            load_config(self)
        for k, v in kwargs.items():
            setattr(self, k, v)
        rp = getattr(self, "rope_parameters", None)
        if isinstance(rp, dict) and "rope_theta" in rp:
            self.rope_theta = rp["rope_theta"]
        if getattr(self, "num_local_experts", None) and not kwargs.get("num_experts"):
            self.num_experts = self.num_local_experts
        if not self.norm_topk_prob:
            raise ValueError("the megakernel implements Qwen3's renormalised top-k (norm_topk_prob=True)")

    def shape(self) -> Qwen3MoeShape:
        return Qwen3MoeShape(hidden_size=self.hidden_size, num_attention_heads=self.num_attention_heads,
                             num_key_value_heads=self.num_key_value_heads, head_dim=self.head_dim,
                             num_experts=self.num_experts, num_experts_per_tok=self.num_experts_per_tok,
                             moe_intermediate_size=self.moe_intermediate_size,
                             num_hidden_layers=self.num_hidden_layers, vocab_size=self.vocab_size,
                             rms_norm_eps=self.rms_norm_eps, rope_theta=self.rope_theta,
                             block_size=self.neuron_config.pa_block_size)


# ---------------------------------------------------------------------------
# checkpoint conversion
# ---------------------------------------------------------------------------
def convert_qwen3_moe_hf_to_neuron_state_dict(state_dict: Dict[str, torch.Tensor], config) -> Dict[str, torch.Tensor]:
    """Normalise a Hugging Face Qwen3-MoE state dict to the per-layer tensors the kernel packs.

    Accepts both checkpoint formats: fused experts (``mlp.experts.gate_up_proj [E, 2I, H]``,
    ``mlp.experts.down_proj [E, H, I]``, transformers >= 5) and per-expert
    ``mlp.experts.{e}.{gate,up,down}_proj.weight`` (original checkpoints), which are stacked
    into the fused form (gate rows then up rows, as the reference's converter builds
    ``gate_up [E, H, 2I]`` at ``qwen_with_megakernel.py:226-253`` before transposing).
    FP8 block-quantised weights with ``*_scale_inv`` are dequantised (reference :146-162).
    Returned keys: ``layers.{l}.{wq,wk,wv,wo,q_norm,k_norm,ln1,ln2,router,gate_up,down}``,
    ``embed``, ``final_norm``, ``lm_head``.
    """
    sd = dict(state_dict)
    pre = "model." if any(k.startswith("model.") for k in sd) else ""
    # fp8 block dequant
    qc = getattr(config, "quantization_config", None)
    for k in [k for k in sd if k.endswith("_scale_inv")]:
        base = k[: -len("_scale_inv")]
        bs = (qc or {}).get("weight_block_size", [128, 128])
        scales = sd.pop(k).to(torch.float32)
        w = sd[base].to(torch.float32)
        s = scales.repeat_interleave(bs[0], 0).repeat_interleave(bs[1], 1)[: w.shape[0], : w.shape[1]]
        sd[base] = (w * s).to(BF16)
    out: Dict[str, torch.Tensor] = {}
    E = config.num_experts
    for l in range(config.num_hidden_layers):
        p = f"{pre}layers.{l}."
        o = f"layers.{l}."
        out[o + "wq"] = sd[p + "self_attn.q_proj.weight"]
        out[o + "wk"] = sd[p + "self_attn.k_proj.weight"]
        out[o + "wv"] = sd[p + "self_attn.v_proj.weight"]
        out[o + "wo"] = sd[p + "self_attn.o_proj.weight"]
        out[o + "q_norm"] = sd[p + "self_attn.q_norm.weight"]
        out[o + "k_norm"] = sd[p + "self_attn.k_norm.weight"]
        out[o + "ln1"] = sd[p + "input_layernorm.weight"]
        out[o + "ln2"] = sd[p + "post_attention_layernorm.weight"]
        out[o + "router"] = sd[p + "mlp.gate.weight"]
        if p + "mlp.experts.gate_up_proj" in sd:
            out[o + "gate_up"] = sd[p + "mlp.experts.gate_up_proj"]
            out[o + "down"] = sd[p + "mlp.experts.down_proj"]
        else:
            out[o + "gate_up"] = torch.stack([torch.cat([sd[p + f"mlp.experts.{e}.gate_proj.weight"],
                                                         sd[p + f"mlp.experts.{e}.up_proj.weight"]], 0)
                                              for e in range(E)])
            out[o + "down"] = torch.stack([sd[p + f"mlp.experts.{e}.down_proj.weight"] for e in range(E)])
    out["embed"] = sd[pre + "embed_tokens.weight"]
    out["final_norm"] = sd[pre + "norm.weight"]
    out["lm_head"] = sd.get("lm_head.weight", out["embed"])
    return out


def _load_safetensors(model_path: str) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file  # noqa: PLC0415  (optional dependency)

    sd: Dict[str, torch.Tensor] = {}
    for f in sorted(glob.glob(os.path.join(model_path, "*.safetensors"))):
        sd.update(load_file(f))
    if not sd:
        raise FileNotFoundError(f"no *.safetensors under {model_path}")
    return sd


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------
class NeuronQwen3MoeForCausalLMV3:
    """Qwen3-MoE CausalLM whose token-generation step is one megakernel launch.

    ``model_path=None`` builds seeded random-init weights of the configured shape (the
    environment has no checkpoints); otherwise Hugging Face safetensors are read.
    """

    def __init__(self, model_path: Optional[str], config: Qwen3MoeInferenceConfig, device=None, seed: int = 0,
                 state_dict: Optional[Dict[str, torch.Tensor]] = None):
        self.model_path = model_path
        self.state_dict = state_dict
        self.config = config
        self.neuron_config = config.neuron_config
        self.device = torch.device(device if device is not None else "cuda")
        self.seed = seed
        self._layers: List[GpuLayer] = []
        self._head: Dict[str, torch.Tensor] = {}
        self.kernel: Optional[Qwen3MoeMegakernel] = None
        self.shard = self._plan_shard()
        self.xchg = None

    def _plan_shard(self):
        """This process's heads and experts when ``tp_degree`` > 1 (None on one GPU)."""
        tp = self.neuron_config.tp_degree
        if tp == 1:
            return None
        import torch.distributed as dist  # noqa: PLC0415

        if not dist.is_initialized() or dist.get_world_size() != tp:
            raise RuntimeError(f"tp_degree={tp} needs torch.distributed initialised with {tp} processes "
                               "(one per GPU, e.g. torchrun --nproc-per-node {tp})")
        c = self.config
        return plan_shard(dist.get_rank(), tp, c.num_attention_heads, c.num_key_value_heads, c.num_experts)

    @classmethod
    def get_neuron_config_cls(cls):
        return Qwen3MoEV3MultilayerNeuronConfig

    @classmethod
    def get_config_cls(cls):
        return Qwen3MoeInferenceConfig

    @staticmethod
    def convert_hf_to_neuron_state_dict(state_dict: dict, config) -> dict:
        return convert_qwen3_moe_hf_to_neuron_state_dict(state_dict, config)

    # -- weights ------------------------------------------------------------
    def _random_hf_state_dict(self) -> Dict[str, torch.Tensor]:
        """Seeded random-init weights in Hugging Face layout (on the model's device)."""
        c, dev = self.config, self.device
        g = torch.Generator(device=dev).manual_seed(self.seed)
        H, D, E, I = c.hidden_size, c.head_dim, c.num_experts, c.moe_intermediate_size

        def n(*s):
            return (torch.randn(*s, generator=g, device=dev) * 0.02).to(BF16)

        def one(*s):
            return (1.0 + torch.randn(*s, generator=g, device=dev) * 0.02).to(BF16)

        sd = {"model.embed_tokens.weight": torch.randn(c.vocab_size, H, generator=g, device=dev).to(BF16),
              "model.norm.weight": one(H), "lm_head.weight": n(c.vocab_size, H)}
        for l in range(c.num_hidden_layers):
            p = f"model.layers.{l}."
            sd[p + "self_attn.q_proj.weight"] = n(c.num_attention_heads * D, H)
            sd[p + "self_attn.k_proj.weight"] = n(c.num_key_value_heads * D, H)
            sd[p + "self_attn.v_proj.weight"] = n(c.num_key_value_heads * D, H)
            sd[p + "self_attn.o_proj.weight"] = n(H, c.num_attention_heads * D)
            sd[p + "self_attn.q_norm.weight"] = one(D)
            sd[p + "self_attn.k_norm.weight"] = one(D)
            sd[p + "input_layernorm.weight"] = one(H)
            sd[p + "post_attention_layernorm.weight"] = one(H)
            sd[p + "mlp.gate.weight"] = n(E, H)
            sd[p + "mlp.experts.gate_up_proj"] = n(E, 2 * I, H)
            sd[p + "mlp.experts.down_proj"] = n(E, H, I)
        return sd

    def hf_state_dict(self) -> Dict[str, torch.Tensor]:
        """The model's weights in Hugging Face layout (re-created or re-read on demand: the
        instance keeps only the kernel layouts)."""
        if self.state_dict is not None:
            return self.state_dict
        if self.model_path:
            return _load_safetensors(self.model_path)
        return self._random_hf_state_dict()

    def _build_layers(self, raw: Dict[str, torch.Tensor]):
        sd = self.convert_hf_to_neuron_state_dict(raw, self.config)
        dev = self.device
        for l in range(self.config.num_hidden_layers):
            t = {k: sd.pop(f"layers.{l}.{k}").to(dev) for k in ("wq", "wk", "wv", "wo", "q_norm", "k_norm", "ln1",
                                                               "ln2", "router", "gate_up", "down")}
            if self.shard is not None:  # this rank's heads and experts
                t["wq"], t["wk"], t["wv"], t["wo"] = shard_attention(t["wq"], t["wk"], t["wv"], t["wo"], self.shard,
                                                                     self.config.head_dim)
                t["gate_up"], t["down"] = shard_experts(t["gate_up"], t["down"], self.shard)
            self._layers.append(GpuLayer(t["wq"], t["wk"], t["wv"], t["wo"], t["q_norm"], t["k_norm"], t["ln1"],
                                         t["ln2"], t["router"], t["gate_up"], t["down"]))
        self._head = {k: sd[k].to(dev) for k in ("embed", "final_norm", "lm_head")}

    def compile(self, compiled_model_path: Optional[str] = None, debug: bool = False):
        """Convert the weights to the kernel layouts on the GPU (the kernel itself is prebuilt)."""
        if self._layers:
            return
        self._build_layers(self.hf_state_dict())

    def load(self, compiled_model_path: Optional[str] = None):
        """Allocate the paged K/V pools and the workspace and create the kernel instance."""
        if not self._layers:
            self.compile(compiled_model_path)
        nc = self.neuron_config
        shape = self.config.shape()
        if self.shard is not None:
            shape.num_attention_heads = len(self.shard.q_heads)
            shape.num_key_value_heads = len(self.shard.kv_heads)
            dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
            self.xchg = XchgRegion(xchg_bytes(shape.hidden_size, self._rows(), self.shard.world,
                                              shape.vocab_size),
                                   self.shard.rank, self.shard.world, dev_index)
        self.kernel = Qwen3MoeMegakernel(shape, self._layers, max_batch=self._rows(),
                                         num_blocks=nc.pa_num_blocks, final_norm=self._head["final_norm"],
                                         lm_head=self._head["lm_head"], embed=self._head["embed"],
                                         rope_max_pos=max(self.config.max_position_embeddings, nc.max_length + 1),
                                         device=self.device, shard=self.shard, xchg=self.xchg)
        self.reset()

    def _rows(self) -> int:
        nc = self.neuron_config
        return max(nc.max_batch_size, nc.prefill_chunk_size)

    def close(self):
        """Release the kernel instance and, on several GPUs, the exchange region (every rank
        calls it, after its last step)."""
        if self.kernel is not None:
            torch.cuda.synchronize(self.device)
            self.kernel.close()
            self.kernel = None
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None

    # -- KV cache bookkeeping ----------------------------------------------
    def reset(self):
        """Fresh block table: sequence b owns blocks [b*nb, (b+1)*nb)."""
        nc = self.neuron_config
        nb = (nc.max_length + nc.pa_block_size) // nc.pa_block_size
        B = nc.max_batch_size
        if B * nb > nc.pa_num_blocks:
            raise ValueError("pa_num_blocks too small for max_batch_size x max_length")
        self.block_table = torch.arange(B * nb, dtype=torch.int32, device=self.device).view(B, nb)

    # -- decode ---------------------------------------------------------------
    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
        """One token-generation step: ``input_ids [B]`` at ``position_ids [B]`` -> logits
        ``[B, vocab]`` fp32.  K/V of every layer are written at ``position_ids``."""
        if self.kernel is None:
            raise RuntimeError("call load() first")
        ids = input_ids.to(self.device, torch.int32).view(-1)
        pos = position_ids.to(self.device, torch.int32).view(-1)
        B = ids.shape[0]
        res = self.kernel.decode_step(pos, self.block_table[:B], input_ids=ids)
        return res["logits"]

    def prefill(self, rows: Sequence[tuple], want_logits: bool = False, routing: Optional[list] = None):
        """Context encoding through the decode kernel: ``rows`` = (sequence, position, token id)
        triples, processed ``prefill_chunk_size`` rows per launch.  Rows of one sequence at
        consecutive positions share a launch: every row's K/V is written before the attention
        reads the cache (``NKM_STAGE_KV_FIRST``), so each row attends causally to the rows
        before it.  Returns the logits of every row ``[len(rows), vocab]`` if ``want_logits``.
        (The reference keeps context encoding on the per-layer NxDI path,
        ``qwen_with_megakernel.py:496-526``.)  ``routing``: a list that receives each row's expert
        indices per layer (``[rows, layers, top_k]`` int32 tensors, one per launch)."""
        if self.kernel is None:
            raise RuntimeError("call load() first")
        n = self.neuron_config.prefill_chunk_size
        out = []
        for c0 in range(0, len(rows), n):
            chunk = rows[c0:c0 + n]
            ids = torch.tensor([r[2] for r in chunk], dtype=torch.int32, device=self.device)
            pos = torch.tensor([r[1] for r in chunk], dtype=torch.int32, device=self.device)
            table = self.block_table[torch.tensor([r[0] for r in chunk], device=self.device)].contiguous()
            res = self.kernel.decode_step(pos, table, input_ids=ids, want_logits=want_logits, kv_first=True,
                                          trace=routing is not None)
            if routing is not None:
                routing.append(res["topk_idx"].transpose(0, 1).contiguous())
            if want_logits:
                out.append(res["logits"])
        return torch.cat(out, 0) if want_logits and out else None

    def teacher_forced_logits(self, tokens: Sequence[int], routing: bool = False):
        """Feed ``tokens`` (sequence 0, positions 0, 1, ...) through the chunked prefill and return
        every position's logits ``[len(tokens), vocab]`` fp32; with ``routing`` also the expert
        indices ``[len(tokens), layers, top_k]``."""
        self.reset()
        rt: Optional[list] = [] if routing else None
        logits = self.prefill([(0, t, tok) for t, tok in enumerate(tokens)], want_logits=True, routing=rt)
        self.kernel.check_status()
        return (logits, torch.cat(rt, 0)) if routing else logits

    def sample(self, logits: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """Next tokens on the device (``nkm_sample_logits``): greedy unless ``do_sample``, else
        top-k (capped to 64, as the reference caps ``global_topk`` to ``top_k``,
        ``qwen_with_megakernel.py:123-127``), temperature and ``top_p``."""
        nc = self.neuron_config
        greedy = not nc.do_sample or nc.top_k <= 1
        return self.kernel.sample(logits, positions.to(self.device, torch.int32),
                                  top_k=1 if greedy else min(nc.top_k, 64), top_p=float(getattr(nc, "top_p", 1.0)),
                                  temperature=float(nc.temperature), seed=self.seed)

    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int) -> List[List[int]]:
        """Greedy (or top-k) generation for a batch of token-id prompts: every prompt but its last
        token through the chunked prefill, then one decode step per new token for the whole
        batch (each sequence at its own position)."""
        self.reset()
        B = len(prompts)
        lens = [len(p) for p in prompts]
        if min(lens) == 0:
            raise ValueError("empty prompt")
        if B > self.neuron_config.max_batch_size:
            raise ValueError("more prompts than max_batch_size")
        total = max(lens) + max_new_tokens
        if total > self.neuron_config.max_length:
            raise ValueError("prompt + new tokens exceed max_length")
        self.prefill([(b, t, int(tok)) for b, p in enumerate(prompts) for t, tok in enumerate(p[:-1])])
        outs: List[List[int]] = [[] for _ in range(B)]
        cur = [int(p[-1]) for p in prompts]
        pos = [n - 1 for n in lens]
        for _ in range(max_new_tokens):
            pos_t = torch.tensor(pos, dtype=torch.int32)
            logits = self.forward(torch.tensor(cur, dtype=torch.int32), pos_t)
            nxt = self.sample(logits, pos_t).tolist()
            for b in range(B):
                outs[b].append(int(nxt[b]))
                cur[b] = int(nxt[b])
                pos[b] += 1
        self.kernel.check_status()
        return outs


# Alias expected by main.py's `NeuronQwen3MoeForCausalLM` convention (reference :728).
NeuronQwen3MoeForCausalLM = NeuronQwen3MoeForCausalLMV3
