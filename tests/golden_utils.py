"""Helpers that turn the Hugging Face golden fixture into oracle inputs."""
import os

import torch

from oracle.qwen3_moe_oracle import LayerWeights, QwenConfig

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qwen3_moe_tiny.pt")


def load_golden():
    return torch.load(GOLDEN, weights_only=False)


def golden_config(d) -> QwenConfig:
    c = d["config"]
    return QwenConfig(hidden=c["hidden_size"], n_q_heads=c["num_attention_heads"],
                      n_kv_heads=c["num_key_value_heads"], head_dim=c["head_dim"],
                      n_experts=c.get("num_experts") or c["num_local_experts"], top_k=c["num_experts_per_tok"],
                      moe_inter=c["moe_intermediate_size"], n_layers=c["num_hidden_layers"],
                      vocab=c["vocab_size"], rms_eps=c["rms_norm_eps"],
                      rope_theta=c["rope_parameters"]["rope_theta"], block_size=128)


def golden_layers(d, cfg: QwenConfig):
    sd = d["state_dict"]
    out = []
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        out.append(LayerWeights(
            wq=sd[p + "self_attn.q_proj.weight"], wk=sd[p + "self_attn.k_proj.weight"],
            wv=sd[p + "self_attn.v_proj.weight"], wo=sd[p + "self_attn.o_proj.weight"],
            q_norm=sd[p + "self_attn.q_norm.weight"], k_norm=sd[p + "self_attn.k_norm.weight"],
            ln1=sd[p + "input_layernorm.weight"], ln2=sd[p + "post_attention_layernorm.weight"],
            router=sd[p + "mlp.gate.weight"], gate_up=sd[p + "mlp.experts.gate_up_proj"],
            down=sd[p + "mlp.experts.down_proj"]))
    return out


def paged_from_contiguous(seqs_kv, n_kv, head_dim, block_size, num_blocks, gen, dtype):
    """Scatter per-sequence contiguous caches ``[n_kv, P, d]`` into a paged pool.

    Blocks are assigned in a shuffled order so that block ids are not monotone.
    Returns ``(pool [num_blocks, n_kv, block_size, d], block_table [B, max_blocks])``.
    """
    B = len(seqs_kv)
    need = [(kv.shape[1] + 1 + block_size - 1) // block_size for kv in seqs_kv]
    maxb = max(need)
    perm = torch.randperm(num_blocks, generator=gen)
    pool = torch.zeros(num_blocks, n_kv, block_size, head_dim, dtype=dtype)
    table = torch.full((B, maxb), -1, dtype=torch.int32)
    nxt = 0
    for b, kv in enumerate(seqs_kv):
        for j in range(need[b]):
            table[b, j] = int(perm[nxt])
            nxt += 1
        P = kv.shape[1]
        for t in range(P):
            pool[table[b, t // block_size], :, t % block_size] = kv[:, t].to(dtype)
    return pool, table
