"""CPU oracle for the GPT-OSS token-generation (decode) step.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA GPT-OSS decode path: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench_gpt_oss.py`` may import it.
The product path never imports, calls or falls back to it.

It restates in plain PyTorch (fp32) the arithmetic of the reference's GPT-OSS megakernel
(``megakernels/gpt_oss/transformer_gpt_oss.py:240-530``) and of the model it is validated
against (Hugging Face ``GptOss*`` modules, which NxDI's ``modeling_gpt_oss`` restates; the CPU
tests pin this file against ``transformers`` 5.5.0):

* layer order ``x -> RMSNorm(ln1) -> attention -> +x -> RMSNorm(ln2) -> MoE -> +x``, RMSNorm
  eps 1e-5 as ``(x * rsqrt(mean(x^2) + eps)) * w`` (``rmsnorm_tkg.py:49-147``);
* q/k/v projections with bias, RoPE on the two halves of each 64-wide head
  (``first' = x1 cos - x2 sin``, ``second' = x2 cos + x1 sin``) with YaRN tables;
* attention with learned per-head sinks: one extra logit per head in the softmax, dropped after
  it (``attention_tkg.py:186-192``); sliding-window layers (even layer index) see the last
  ``W - 1`` positions plus the new token (``transformer_gpt_oss.py:67-205``), full layers every
  prior position plus the new token; O-projection with bias;
* router: linear with bias, top-k on the logits, softmax over the k, no renormalisation
  (``transformer_gpt_oss.py:406-425``, ``router_topk.py:147-188``);
* experts: gate/up rows interleaved (row 2i gate i, 2i+1 up i) plus bias, gate clamped above at
  7, up clamped to [-7, 7], ``glu = gate * sigmoid(1.702 gate)``, ``h = (up + 1) * glu``, down
  projection plus bias, scaled by the routing weight and summed over the k slots
  (``transformer_gpt_oss.py:427-433``; the reference folds the +1 into the up bias and clamps
  up to [-6, 8], which is the same function);
* MXFP4 expert weights: e2m1 codes (sign bit 3, magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6) times an
  e8m0 scale 2^(s - 127) per 32 consecutive input elements (OCP Microscaling format; reference
  ``selective_expert_mx_impl.py:60-531``), dequantised exactly to fp32 here.

Layouts: q/k/v_proj ``[heads*64, H]``, o_proj ``[H, nq*64]``, router ``[E, H]``, expert gate/up
``[E, 2I, H]`` (the transpose of Hugging Face's ``gate_up_proj [E, H, 2I]``), down ``[E, H, I]``
(the transpose of ``down_proj [E, I, H]``).  The paged KV cache per layer is
``[num_blocks, n_kv_heads, 128, 64]``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

F32 = torch.float32
BF16 = torch.bfloat16

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


@dataclass
class GptOssConfig:
    hidden: int = 2880
    n_q_heads: int = 64
    n_kv_heads: int = 8
    head_dim: int = 64
    n_experts: int = 32
    top_k: int = 4
    inter: int = 2880
    n_layers: int = 24
    vocab: int = 201088
    rms_eps: float = 1e-5
    sliding_window: int = 128
    rope_theta: float = 150000.0
    rope_factor: float = 32.0
    rope_original_max: int = 4096
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    block_size: int = 128

    def is_sliding(self, layer: int) -> bool:
        return layer % 2 == 0


@dataclass
class GptOssLayer:
    wq: torch.Tensor
    bq: torch.Tensor
    wk: torch.Tensor
    bk: torch.Tensor
    wv: torch.Tensor
    bv: torch.Tensor
    wo: torch.Tensor
    bo: torch.Tensor
    sinks: torch.Tensor
    ln1: torch.Tensor
    ln2: torch.Tensor
    router: torch.Tensor
    router_b: torch.Tensor
    gu_codes: torch.Tensor   # uint8 [E, 2I, H]  e2m1 codes 0..15
    gu_scales: torch.Tensor  # uint8 [E, 2I, H/32] e8m0
    gu_b: torch.Tensor       # [E, 2I]
    dn_codes: torch.Tensor   # uint8 [E, H, I]
    dn_scales: torch.Tensor  # uint8 [E, H, I/32]
    dn_b: torch.Tensor       # [E, H]


def mx_dequant(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 values of MXFP4 codes ``[..., K]`` with e8m0 scales ``[..., K/32]``."""
    v = E2M1[codes.long()]
    s = torch.pow(2.0, scales.to(F32) - 127.0)
    return (v.view(*codes.shape[:-1], -1, 32) * s[..., None]).reshape(codes.shape)


def random_mx(shape, gen: torch.Generator):
    """Seeded MXFP4 tensor: uniform codes, scales 2^-8 .. 2^-6 (rms ~ 0.02)."""
    codes = torch.randint(0, 16, shape, generator=gen, dtype=torch.uint8)
    scales = torch.randint(119, 122, (*shape[:-1], shape[-1] // 32), generator=gen, dtype=torch.uint8)
    return codes, scales


def random_layer(cfg: GptOssConfig, gen: torch.Generator, std: float = 0.02) -> GptOssLayer:
    H, D, E, I = cfg.hidden, cfg.head_dim, cfg.n_experts, cfg.inter

    def n(*shape, s=std):
        return (torch.randn(*shape, generator=gen) * s).to(BF16)

    def g(*shape):
        return (1.0 + torch.randn(*shape, generator=gen) * std).to(BF16)

    gu_c, gu_s = random_mx((E, 2 * I, H), gen)
    dn_c, dn_s = random_mx((E, H, I), gen)
    return GptOssLayer(
        wq=n(cfg.n_q_heads * D, H), bq=n(cfg.n_q_heads * D), wk=n(cfg.n_kv_heads * D, H), bk=n(cfg.n_kv_heads * D),
        wv=n(cfg.n_kv_heads * D, H), bv=n(cfg.n_kv_heads * D), wo=n(H, cfg.n_q_heads * D), bo=n(H),
        sinks=n(cfg.n_q_heads, s=1.0), ln1=g(H), ln2=g(H), router=n(E, H), router_b=n(E),
        gu_codes=gu_c, gu_scales=gu_s, gu_b=n(E, 2 * I), dn_codes=dn_c, dn_scales=dn_s, dn_b=n(E, H))


# ---------------------------------------------------------------------------
# RoPE (YaRN, Peng et al. 2023, as Hugging Face's _compute_yarn_parameters computes it)
# ---------------------------------------------------------------------------
def yarn_inv_freq(cfg: GptOssConfig):
    dim, base, factor = cfg.head_dim, cfg.rope_theta, cfg.rope_factor

    def corr_dim(rot):
        return (dim * math.log(cfg.rope_original_max / (rot * 2 * math.pi))) / (2 * math.log(base))

    low = max(corr_dim(cfg.rope_beta_fast), 0)
    high = min(corr_dim(cfg.rope_beta_slow), dim - 1)
    if low == high:
        high += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=F32) - low) / (high - low), 0, 1)
    extrap = 1 - ramp
    pos_freqs = base ** (torch.arange(0, dim, 2).to(F32) / dim)
    inv = (1.0 / (factor * pos_freqs)) * (1 - extrap) + (1.0 / pos_freqs) * extrap
    attn_factor = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
    return inv, attn_factor


def rope_tables(cfg: GptOssConfig, max_pos: int):
    """fp32 cos/sin ``[max_pos, head_dim/2]`` (YaRN frequencies, times the attention factor)."""
    inv, af = yarn_inv_freq(cfg)
    freqs = torch.arange(max_pos, dtype=F32)[:, None] * inv[None, :]
    return freqs.cos() * af, freqs.sin() * af


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


# ---------------------------------------------------------------------------
# blocks
# ---------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.to(F32)
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)) * w.to(F32)


def _gather(cache, table, b, h, lo, hi, bs):
    rows = []
    for t0 in range(lo - lo % bs, hi, bs):
        blk = int(table[b, t0 // bs])
        a, z = max(lo, t0) - t0, min(hi, t0 + bs) - t0
        rows.append(cache[blk, h, a:z])
    return torch.cat(rows, 0) if rows else cache.new_zeros(0, cache.shape[-1])


def fp8_qdq(t: torch.Tensor, scale: float) -> torch.Tensor:
    """``e4m3(clip(t * scale, +-240)) / scale`` (round to nearest even): a value as an FP8 K/V
    cache stores and returns it (``attention_block_tkg.py:1694-1737``)."""
    return (t.to(F32) * scale).clamp(-240.0, 240.0).to(torch.float8_e4m3fn).to(F32) / scale


def attention(xn, lw: GptOssLayer, cfg: GptOssConfig, layer: int, k_cache, v_cache, positions, table, cos, sin,
              kv_scales=None, new_kv=None):
    """Attention block on normed rows ``xn [T, H]``; writes the new K/V into the paged cache.

    ``kv_scales = (k_scale, v_scale)``: FP8 K/V cache; the new token's K and V are quantised
    before the attention uses them, as the reference quantises the active K/V it attends to
    (``attention_block_tkg.py:975-986, 1075-1084``).  ``new_kv = (k [T, nkv, D], v [T, nkv, D])``:
    the new tokens' (RoPE'd) K and V as given (e.g. read back from a cache another implementation
    wrote), in place of this function's own projections."""
    T = xn.shape[0]
    D, nq, nkv = cfg.head_dim, cfg.n_q_heads, cfg.n_kv_heads
    grp = nq // nkv
    q = (xn @ lw.wq.to(F32).t() + lw.bq.to(F32)).view(T, nq, D)
    k = (xn @ lw.wk.to(F32).t() + lw.bk.to(F32)).view(T, nkv, D)
    v = (xn @ lw.wv.to(F32).t() + lw.bv.to(F32)).view(T, nkv, D)
    pos = positions.tolist()
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    q, k = apply_rope(q, c, s), apply_rope(k, c, s)
    if kv_scales is not None:
        k, v = fp8_qdq(k, kv_scales[0]), fp8_qdq(v, kv_scales[1])
    if new_kv is not None:
        k, v = new_kv[0].to(F32), new_kv[1].to(F32)
    out = torch.zeros(T, nq, D, dtype=F32)
    sinks = lw.sinks.to(F32)
    for b in range(T):
        p = pos[b]
        lo = max(0, p - (cfg.sliding_window - 1)) if cfg.is_sliding(layer) else 0
        for h in range(nkv):
            keys = torch.cat([_gather(k_cache, table, b, h, lo, p, cfg.block_size).to(F32), k[b, h][None]], 0)
            vals = torch.cat([_gather(v_cache, table, b, h, lo, p, cfg.block_size).to(F32), v[b, h][None]], 0)
            qh = q[b, h * grp:(h + 1) * grp]
            sc = (qh @ keys.t()) / math.sqrt(D)
            sc = torch.cat([sc, sinks[h * grp:(h + 1) * grp, None]], 1)
            pr = torch.softmax(sc, dim=-1)[:, :-1]
            out[b, h * grp:(h + 1) * grp] = pr @ vals
    for b in range(T):
        blk = int(table[b, pos[b] // cfg.block_size])
        if blk < 0:
            continue
        k_cache[blk, :, pos[b] % cfg.block_size] = k[b].to(k_cache.dtype)
        v_cache[blk, :, pos[b] % cfg.block_size] = v[b].to(v_cache.dtype)
    return out.reshape(T, nq * D) @ lw.wo.to(F32).t() + lw.bo.to(F32)


def router(xn, lw: GptOssLayer, cfg: GptOssConfig, topk_hint=None, hint_gap: float = 0.0):
    """Logits, top-k indices and softmax over the top-k.  ``topk_hint [T, k]``: rows whose hinted
    set is a top-k of the logits up to ``hint_gap`` take it (the other side's choice at a near
    tie)."""
    logits = xn @ lw.router.to(F32).t() + lw.router_b.to(F32)
    top, idx = torch.topk(logits, cfg.top_k, dim=-1)
    if topk_hint is not None:
        for r in range(idx.shape[0]):
            h = topk_hint[r].long()
            if set(h.tolist()) == set(idx[r].tolist()):
                continue
            mask = torch.ones(logits.shape[-1], dtype=torch.bool)
            mask[h] = False
            if float(logits[r, mask].max() - logits[r, h].min()) <= hint_gap:
                idx[r] = h
                top[r] = logits[r, h]
    return logits, idx, torch.softmax(top, dim=-1)


def experts(xn, idx, w, lw: GptOssLayer, cfg: GptOssConfig):
    T = xn.shape[0]
    out = torch.zeros(T, cfg.top_k, cfg.hidden, dtype=F32)
    lim, alpha = cfg.swiglu_limit, cfg.swiglu_alpha
    for e in torch.unique(idx).tolist():
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        gu = xn[tok] @ mx_dequant(lw.gu_codes[e], lw.gu_scales[e]).t() + lw.gu_b[e].to(F32)
        gate, up = gu[:, 0::2].clamp(max=lim), gu[:, 1::2].clamp(min=-lim, max=lim)
        h = (up + 1) * (gate * torch.sigmoid(gate * alpha))
        y = h @ mx_dequant(lw.dn_codes[e], lw.dn_scales[e]).t() + lw.dn_b[e].to(F32)
        out[tok, slot] = y * w[tok, slot][:, None]
    acc = torch.zeros(T, cfg.hidden, dtype=F32)
    for kk in range(cfg.top_k):
        acc = acc + out[:, kk]
    return acc


def decoder_layer(x, lw, cfg, layer, k_cache, v_cache, positions, table, cos, sin, trace=None, kv_scales=None,
                  topk_hint=None, hint_gap: float = 0.0, new_kv=None):
    x = x.to(F32)
    mid = x + attention(rmsnorm(x, lw.ln1, cfg.rms_eps), lw, cfg, layer, k_cache, v_cache, positions, table, cos, sin,
                        kv_scales, new_kv)
    xn2 = rmsnorm(mid, lw.ln2, cfg.rms_eps)
    logits, idx, w = router(xn2, lw, cfg, topk_hint, hint_gap)
    out = mid + experts(xn2, idx, w, lw, cfg)
    if trace is not None:
        trace.append({"resid_mid": mid, "router_logits": logits, "topk_idx": idx, "topk_w": w, "resid_out": out})
    return out


def decode_step(x, layers: List[GptOssLayer], cfg: GptOssConfig, k_caches, v_caches, positions, table, cos, sin,
                final_norm=None, lm_head=None, traces: Optional[list] = None):
    """``len(k_caches)`` layers (weights cycle through ``layers``; layer parity picks the attention
    type), then the final RMSNorm and the LM head.  Returns (hidden fp32, logits fp32 or None)."""
    for li in range(len(k_caches)):
        x = decoder_layer(x, layers[li % len(layers)], cfg, li, k_caches[li], v_caches[li], positions, table, cos, sin,
                          traces)
    logits = None
    if lm_head is not None:
        logits = rmsnorm(x, final_norm, cfg.rms_eps) @ lm_head.to(F32).t()
    return x, logits


def compare(a: torch.Tensor, b: torch.Tensor):
    a, b = a.to(F32).flatten(), b.to(F32).flatten()
    return {"max_abs": (a - b).abs().max().item(),
            "cosine": torch.nn.functional.cosine_similarity(a, b, dim=0).item()}
