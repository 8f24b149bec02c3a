"""CPU oracle for the Qwen3-MoE token-generation (decode) step.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA decode path:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``nki_moe_megakernel_b200``) never imports, calls or falls back to it.

It restates, in plain PyTorch on the CPU, the arithmetic of the reference's
decode megakernel and of the baseline decoder forward it is validated against:

* layer order ``x -> RMSNorm(ln1) -> attention -> +x -> RMSNorm(ln2) -> MoE -> +x``
  (reference ``megakernels/qwen3_moe/qwen.py:386-444``,
  ``megakernels/qwen3_moe/transformer_qwen.py:271-378``);
* per-head q/k RMSNorm over head_dim then RoPE with the rotate-half convention
  (``megakernels/qwen3_moe/qwen.py:321-343``,
  ``megakernels/qwen3_moe/attn_fused_nki.py:393-451,494-586``);
* decode attention over prior positions ``t < pos`` plus the active token at ``pos``
  (mask rule ``attn_fused_nki.py:653-677``, active term ``:711-865``);
* fp32 router logits, softmax, top-k selected on the *logits*, softmax values at the
  top-k, bf16 L1 renormalisation (``megakernels/qwen3_moe/moe_fused_nki.py:186-272,404-418``);
* expert SwiGLU with bf16 gate/up, bf16 SiLU(gate)*up, fp32 down projection,
  affinity scaling and fp32 accumulation in top-k slot order
  (``moe_fused_nki.py:486-568,734-757``);
* bf16 residual adds (``transformer_qwen.py:331-333,370-372``).

Two modes:

``mode="fp32"``      every intermediate in fp32 (weights and caches upcast); the
                     tolerance reference (max-abs 2e-2, cosine >= 0.999).
``mode="faithful"``  the reference kernel's bf16 rounding points.  Reductions whose
                     fp32 summation order decides bits that are checked for exact
                     equality (RMSNorm statistics, the router logits, q/k-norm
                     statistics) follow the documented fixed order of the CUDA
                     kernels (see ``lane_sum_hidden`` / ``lane_sum_head``), so that
                     top-k indices and KV-cache slot values can be compared bit for
                     bit when both sides are fed the same bf16 inputs.

Layouts are the Hugging Face ones (transformers ``Qwen3Moe*`` modules):
q/k/v_proj ``[heads*128, H]``, o_proj ``[H, nq*128]``, router ``[E, H]``,
experts gate_up ``[E, 2I, H]`` (gate rows first), down ``[E, H, I]``.
The paged KV cache per layer is ``[num_blocks, n_kv_heads, block_size, head_dim]``
indexed through ``block_table[b, pos // block_size]``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

F32 = torch.float32
BF16 = torch.bfloat16


# ---------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------
def rbf(x: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to bf16 (round-to-nearest-even) and return it as fp32."""
    return x.to(F32).to(BF16).to(F32)


def _butterfly32(s: torch.Tensor) -> torch.Tensor:
    """Xor-butterfly sum over the last dim (32 lanes), offsets 16, 8, 4, 2, 1.

    Mirrors ``__shfl_xor_sync`` reductions in the kernels: after the butterfly every lane
    holds the same value; lane 0's value is returned.
    """
    lanes = torch.arange(32)
    for off in (16, 8, 4, 2, 1):
        s = s + s[..., lanes ^ off]
    return s[..., 0]


def lane_sum_hidden(p: torch.Tensor) -> torch.Tensor:
    """Fixed-order fp32 sum over the last dim (length a multiple of 256).

    Order used by the CUDA kernels for hidden-size reductions: lane ``l`` (0..31) owns
    elements ``k = 256*i + 8*l + j``; it accumulates them sequentially (i outer, j
    inner, starting from 0.0, one rounded add per term), then the 32 lane partials are
    combined by ``_butterfly32``.
    """
    n = p.shape[-1]
    assert n % 256 == 0, n
    v = p.reshape(*p.shape[:-1], n // 256, 32, 8)
    s = torch.zeros(*p.shape[:-1], 32, dtype=F32)
    for i in range(n // 256):
        for j in range(8):
            s = s + v[..., i, :, j]
    return _butterfly32(s)


def lane_sum_head(p: torch.Tensor) -> torch.Tensor:
    """Fixed-order fp32 sum over a 128-long last dim: lane ``l`` owns ``4l..4l+3``."""
    assert p.shape[-1] == 128
    v = p.reshape(*p.shape[:-1], 32, 4)
    s = torch.zeros(*p.shape[:-1], 32, dtype=F32)
    for j in range(4):
        s = s + v[..., :, j]
    return _butterfly32(s)


def rstd_fixed(sumsq: torch.Tensor, n: int, eps: float) -> torch.Tensor:
    """``1 / sqrt(sumsq * fp32(1/n) + eps)`` with IEEE-rounded sqrt and divide.

    The square root and the reciprocal are taken in fp64 and rounded once to fp32, which is the
    correctly rounded fp32 result (fp64 carries more than 2 * 24 + 2 bits); torch's fp32 CPU
    ``sqrt`` is not always correctly rounded (it was 1 ulp low on some inputs here).
    """
    inv_n = torch.tensor(1.0 / n, dtype=F32)
    v = sumsq * inv_n + torch.tensor(eps, dtype=F32)
    s = torch.sqrt(v.to(torch.float64)).to(F32)
    return (1.0 / s.to(torch.float64)).to(F32)


def mxfp8_quantize(w: torch.Tensor):
    """OCP MX (Microscaling Formats v1.0) quantisation of ``w [..., K]`` (K % 32 == 0) to MXFP8:
    per block of 32 along K the shared scale is ``X = 2^(floor(log2(amax)) - 8)`` (8 = the largest
    e4m3 exponent), stored as the e8m0 byte ``127 + floor(log2(amax)) - 8``; elements are
    ``e4m3(clip(w / X, +-448))`` (round to nearest even).  An all-zero block gets the smallest
    scale.  Returns (codes uint8 = e4m3 bits, scales uint8)."""
    shp = w.shape
    b = w.to(F32).reshape(*shp[:-1], shp[-1] // 32, 32)
    amax = b.abs().amax(-1)
    e = torch.floor(torch.log2(amax.clamp_min(2.0 ** -126))) - 8
    e = torch.where(amax > 0, e, torch.full_like(e, -127.0)).clamp(-127, 127)
    q = (b / torch.exp2(e)[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(shp), (e + 127).to(torch.uint8)


def mxfp8_dequant(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 values of MXFP8 codes ``[..., K]`` (e4m3 bits) with e8m0 scales ``[..., K/32]``."""
    v = codes.view(torch.float8_e4m3fn).to(F32)
    shp = v.shape
    s = torch.exp2(scales.to(F32) - 127.0)
    return (v.reshape(*shp[:-1], shp[-1] // 32, 32) * s[..., None]).reshape(shp)


def rstd_fixed_div(sumsq: torch.Tensor, n: int, eps: float) -> torch.Tensor:
    """``1 / sqrt(sumsq / n + eps)`` with an IEEE fp32 divide by ``n`` (for ``n`` whose reciprocal
    is not exact, as the padded-hidden RMSNorm of the GPT-OSS kernel computes it), then the
    correctly rounded sqrt and reciprocal as in ``rstd_fixed``."""
    v = sumsq / torch.tensor(float(n), dtype=F32) + torch.tensor(eps, dtype=F32)
    s = torch.sqrt(v.to(torch.float64)).to(F32)
    return (1.0 / s.to(torch.float64)).to(F32)


# ---------------------------------------------------------------------------
# model description
# ---------------------------------------------------------------------------
@dataclass
class QwenConfig:
    hidden: int = 2048
    n_q_heads: int = 32
    n_kv_heads: int = 4
    head_dim: int = 128
    n_experts: int = 128
    top_k: int = 8
    moe_inter: int = 768
    n_layers: int = 48
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 128


@dataclass
class LayerWeights:
    """One decoder layer in Hugging Face layout (all bf16)."""

    wq: torch.Tensor      # [nq*128, H]
    wk: torch.Tensor      # [nkv*128, H]
    wv: torch.Tensor      # [nkv*128, H]
    wo: torch.Tensor      # [H, nq*128]
    q_norm: torch.Tensor  # [128]
    k_norm: torch.Tensor  # [128]
    ln1: torch.Tensor     # [H]   input_layernorm
    ln2: torch.Tensor     # [H]   post_attention_layernorm
    router: torch.Tensor  # [E, H]
    gate_up: torch.Tensor  # [E, 2I, H]
    down: torch.Tensor    # [E, H, I]
    router_bias: Optional[torch.Tensor] = None  # [E] fp32 added to the logits (router_topk.py:69 bias)


@dataclass
class LayerTrace:
    """Intermediates of one layer (for teacher-forced parity checks)."""

    q_raw: Optional[torch.Tensor] = None
    k_raw: Optional[torch.Tensor] = None
    v_raw: Optional[torch.Tensor] = None
    k_new: Optional[torch.Tensor] = None
    v_new: Optional[torch.Tensor] = None
    attn: Optional[torch.Tensor] = None
    resid_mid: Optional[torch.Tensor] = None
    router_logits: Optional[torch.Tensor] = None
    topk_idx: Optional[torch.Tensor] = None
    # input: a top-k selection [T, k] to follow where the logits make it a top-k within
    # ``hint_gap`` (the other side's choice at a near tie); ``hint_rows`` counts the rows that did
    topk_hint: Optional[torch.Tensor] = None
    hint_gap: float = 0.0
    hint_rows: int = 0
    topk_w: Optional[torch.Tensor] = None
    moe_out: Optional[torch.Tensor] = None
    resid_out: Optional[torch.Tensor] = None


def random_layer(cfg: QwenConfig, gen: torch.Generator, std: float = 0.02) -> LayerWeights:
    """Seeded random layer: weights ~N(0, std), norm weights ~1+N(0, std) (bf16)."""
    H, D, E, I = cfg.hidden, cfg.head_dim, cfg.n_experts, cfg.moe_inter

    def n(*shape):
        return (torch.randn(*shape, generator=gen) * std).to(BF16)

    def g(*shape):
        return (1.0 + torch.randn(*shape, generator=gen) * std).to(BF16)

    return LayerWeights(
        wq=n(cfg.n_q_heads * D, H), wk=n(cfg.n_kv_heads * D, H), wv=n(cfg.n_kv_heads * D, H),
        wo=n(H, cfg.n_q_heads * D), q_norm=g(D), k_norm=g(D), ln1=g(H), ln2=g(H),
        router=n(E, H), gate_up=n(E, 2 * I, H), down=n(E, H, I))


def rope_tables(max_pos: int, head_dim: int, theta: float, dtype=BF16):
    """cos/sin tables ``[max_pos, head_dim]``, Hugging Face default RoPE.

    ``inv_freq = 1 / theta**(arange(0, d, 2)/d)``; ``freqs = pos * inv_freq`` in fp32;
    ``emb = cat(freqs, freqs)``; cast to the model dtype (bf16 for the decode kernels, as the
    reference passes bf16 cos/sin, ``transformer_qwen.py:85-86``; fp32 for an fp32 model)
    (transformers ``Qwen3MoeRotaryEmbedding``).
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(F32) / head_dim))
    pos = torch.arange(max_pos, dtype=F32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


# ---------------------------------------------------------------------------
# primitives
# ---------------------------------------------------------------------------
def rmsnorm_fp32(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.to(F32)
    var = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * w.to(F32)


def rmsnorm_hidden_faithful(x_bf16: torch.Tensor, w: torch.Tensor, eps: float,
                            gamma_first: bool) -> torch.Tensor:
    """RMSNorm of a bf16 ``[T, H]`` row block with the kernel's fixed-order statistics.

    ``gamma_first=False`` is the pre-attention order ``(x*r)*g``
    (``attn_fused_nki.py:306-309``); ``gamma_first=True`` is the MoE order ``(x*g)*r``
    (``moe_fused_nki.py:114-147``).  Returns fp32 (the caller rounds where the reference
    does).
    """
    x = x_bf16.to(F32)
    r = rstd_fixed(lane_sum_hidden(x * x), x.shape[-1], eps)[..., None]
    g = w.to(F32)
    return (x * g) * r if gamma_first else (x * r) * g


def head_norm_rope_faithful(raw_bf16: torch.Tensor, w: torch.Tensor, cos: torch.Tensor,
                            sin: torch.Tensor, eps: float) -> torch.Tensor:
    """q/k head RMSNorm + RoPE exactly at the reference's rounding points.

    ``raw_bf16``: ``[..., 128]`` bf16 projection output; ``cos``/``sin`` ``[..., 128]``
    bf16 broadcastable.  Norm statistics in fp32 (``lane_sum_head`` order), ``(x*r)*w``
    in fp32, rounded to bf16; RoPE as bf16 ops: ``bf16(bf16(x*cos) + bf16(rot(x)*sin))``
    (``attn_fused_nki.py:416-451,494-586``).
    """
    x = raw_bf16.to(F32)
    r = rstd_fixed(lane_sum_head(x * x), 128, eps)[..., None]
    xn = rbf((x * r) * w.to(F32))
    half = xn.shape[-1] // 2
    rot = torch.cat((-xn[..., half:], xn[..., :half]), dim=-1)
    c, s = cos.to(F32), sin.to(F32)
    return rbf(rbf(xn * c) + rbf(rot * s))


def head_norm_rope_fp32(raw: torch.Tensor, w: torch.Tensor, cos, sin, eps: float):
    x = rmsnorm_fp32(raw, w, eps)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos.to(F32) + rot * sin.to(F32)


def router_logits_fixed(xn_f32: torch.Tensor, w_router: torch.Tensor) -> torch.Tensor:
    """fp32 router logits ``[T, E]`` in the kernel's fixed summation order.

    Each product ``W[e,k] * x[t,k]`` is rounded to fp32, then summed by
    ``lane_sum_hidden`` (``moe_fused_nki.py:186-218`` computes the same logits with an
    fp32 router weight copy).
    """
    w = w_router.to(F32)
    prod = w[None, :, :] * xn_f32[:, None, :]
    return lane_sum_hidden(prod)


def topk_select(logits: torch.Tensor, k: int):
    """Top-k on logits, descending, ties broken toward the lower expert index.

    Mirrors ``max8`` + ``nc_find_index8`` on fp32 logits (``moe_fused_nki.py:241-250``).
    """
    # a stable descending sort keeps equal values in ascending index order
    order = torch.sort(logits, dim=-1, descending=True, stable=True).indices
    return order[..., :k]


def follow_hint(logits: torch.Tensor, idx: torch.Tensor, hint: torch.Tensor, gap: float):
    """Rows of ``idx`` replaced by ``hint`` where the hinted set is a top-k of ``logits`` up to
    ``gap`` (its lowest logit is within ``gap`` of the highest logit outside it).  Returns
    (indices, number of rows replaced)."""
    out = idx.clone()
    n = 0
    for r in range(idx.shape[0]):
        a, b = set(idx[r].tolist()), set(hint[r].tolist())
        if a == b:
            continue
        inside = logits[r, hint[r].long()].min()
        mask = torch.ones(logits.shape[-1], dtype=torch.bool)
        mask[hint[r].long()] = False
        if float(logits[r, mask].max() - inside) <= gap:
            out[r] = hint[r].to(out.dtype)
            n += 1
    return out, n


def router_topk(logits: torch.Tensor, k: int, mode: str, hint: Optional[torch.Tensor] = None,
                gap: float = 0.0, counter: Optional[list] = None):
    """Softmax at the top-k and L1 renormalisation.

    faithful: ``v = bf16(exp(l_k - max) * (1/sum))``, ``w = bf16(v * (1/sum_k v))``
    (``moe_fused_nki.py:224-272,404-418``); fp32: plain fp32 softmax + renorm.
    Returns ``(idx [T,k] int64, w [T,k] fp32)``.
    """
    idx = topk_select(logits, k)
    if hint is not None:
        idx, n = follow_hint(logits, idx, hint, gap)
        if counter is not None:
            counter.append(n)
    mx = logits.max(dim=-1, keepdim=True).values
    ex = torch.exp(logits - mx)
    inv = 1.0 / ex.sum(-1, keepdim=True)
    top = torch.gather(ex, -1, idx) * inv
    if mode == "faithful":
        v = rbf(top)
        s = torch.zeros(v.shape[:-1], dtype=F32)
        for j in range(k):
            s = s + v[..., j]
        w = rbf(v * (1.0 / s)[..., None])
    else:
        w = top / top.sum(-1, keepdim=True)
    return idx, w


def experts_forward(xn: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                    gate_up: torch.Tensor, down: torch.Tensor, mode: str) -> torch.Tensor:
    """Selective-expert SwiGLU MLP.  ``xn`` [T,H] (bf16-valued fp32 in faithful mode).

    Output fp32 ``[T, H]`` = sum over k in slot order 0..K-1 of ``w[t,k] * down_e(h)``
    (each expert's GEMVs are evaluated once for all of its tokens).
    """
    T, K = idx.shape
    I = down.shape[-1]
    contrib = torch.zeros(T, K, xn.shape[-1], dtype=F32)
    for e in torch.unique(idx).tolist():
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        gu = xn[tok].to(F32) @ gate_up[e].to(F32).t()
        g, u = gu[:, :I], gu[:, I:]
        if mode == "faithful":
            g, u = rbf(g), rbf(u)
            h = rbf(rbf(torch.nn.functional.silu(g)) * u)
        else:
            h = torch.nn.functional.silu(g) * u
        d = h @ down[e].to(F32).t()
        contrib[tok, slot] = d * w[tok, slot][:, None]
    out = torch.zeros(T, xn.shape[-1], dtype=F32)
    for k in range(K):
        out = out + contrib[:, k]
    return out


def moe_block(x_bf16: torch.Tensor, lw: LayerWeights, cfg: QwenConfig, mode: str,
              trace: Optional[LayerTrace] = None) -> torch.Tensor:
    """RMSNorm(ln2) + router_topk + moe_tkg on ``x`` ``[T, H]`` (bf16).  Returns fp32 MoE out.

    Standalone MoE block of the reference (``moe_fused_nki.py:769-821``, harness
    ``run()`` ``:1000-1043``).
    """
    if mode == "faithful":
        xn32 = rmsnorm_hidden_faithful(x_bf16, lw.ln2, cfg.rms_eps, gamma_first=True)
        logits = router_logits_fixed(xn32, lw.router)
        xn = rbf(xn32)
    else:
        xn = rmsnorm_fp32(x_bf16, lw.ln2, cfg.rms_eps)
        logits = xn @ lw.router.to(F32).t()
    if lw.router_bias is not None:
        logits = logits + lw.router_bias.to(F32)
    used: list = []
    hint = trace.topk_hint if trace is not None else None
    idx, w = router_topk(logits, cfg.top_k, mode, hint, trace.hint_gap if trace is not None else 0.0, used)
    if trace is not None and used:
        trace.hint_rows = used[0]
    out = experts_forward(xn, idx, w, lw.gate_up, lw.down, mode)
    if trace is not None:
        trace.router_logits, trace.topk_idx, trace.topk_w = logits, idx, w
        trace.moe_out = out
    return out


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def kv_slot(block_table: torch.Tensor, b: int, pos: int, block_size: int):
    return int(block_table[b, pos // block_size]), pos % block_size


def gather_context(cache: torch.Tensor, block_table: torch.Tensor, b: int, h: int, n: int,
                   block_size: int) -> torch.Tensor:
    """Tokens ``0..n-1`` of sequence ``b``, kv-head ``h`` from a paged cache -> ``[n, d]``."""
    rows = []
    for start in range(0, n, block_size):
        blk = int(block_table[b, start // block_size])
        m = min(block_size, n - start)
        rows.append(cache[blk, h, :m])
    if not rows:
        return cache.new_zeros(0, cache.shape[-1])
    return torch.cat(rows, 0)


def attention_layer(xn1: torch.Tensor, lw: LayerWeights, cfg: QwenConfig,
                    k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor,
                    block_table: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
                    mode: str, trace: Optional[LayerTrace] = None) -> torch.Tensor:
    """QKV + q/k-norm + RoPE + KV write at ``pos`` + decode attention + O-proj.

    ``xn1`` is the normed input ``[T, H]`` (bf16-valued in faithful mode).  The caches are
    updated in place (the new token's K/V at ``pos``) unless the block id there is negative
    (skip, the reference's ``uint32_max`` convention, ``attention_block_tkg.py:1473-1692``).
    Returns the O-projection output ``[T, H]`` fp32 (bf16-valued in faithful mode).
    """
    T = xn1.shape[0]
    D, nq, nkv = cfg.head_dim, cfg.n_q_heads, cfg.n_kv_heads
    grp = nq // nkv
    q = xn1.to(F32) @ lw.wq.to(F32).t()
    k = xn1.to(F32) @ lw.wk.to(F32).t()
    v = xn1.to(F32) @ lw.wv.to(F32).t()
    if mode == "faithful":
        q, k, v = rbf(q), rbf(k), rbf(v)
    q = q.view(T, nq, D)
    k = k.view(T, nkv, D)
    v = v.view(T, nkv, D)
    pos = positions.tolist()
    cos = cos_tab[pos].to(F32)[:, None, :]
    sin = sin_tab[pos].to(F32)[:, None, :]
    if mode == "faithful":
        qr = head_norm_rope_faithful(q, lw.q_norm, cos, sin, cfg.rms_eps)
        kr = head_norm_rope_faithful(k, lw.k_norm, cos, sin, cfg.rms_eps)
    else:
        qr = head_norm_rope_fp32(q, lw.q_norm, cos, sin, cfg.rms_eps)
        kr = head_norm_rope_fp32(k, lw.k_norm, cos, sin, cfg.rms_eps)
    if trace is not None:
        trace.q_raw, trace.k_raw, trace.v_raw = q.clone(), k.clone(), v.clone()
        trace.k_new, trace.v_new = kr.clone(), v.clone()
    scale = 1.0 / math.sqrt(D)
    out = torch.zeros(T, nq, D, dtype=F32)
    for b in range(T):
        p = pos[b]
        for h in range(nkv):
            kc = gather_context(k_cache, block_table, b, h, p, cfg.block_size).to(F32)
            vc = gather_context(v_cache, block_table, b, h, p, cfg.block_size).to(F32)
            keys = torch.cat([kc, kr[b, h][None]], 0)      # [p+1, D]
            vals = torch.cat([vc, v[b, h][None]], 0)
            qh = qr[b, h * grp:(h + 1) * grp]               # [grp, D]
            s = qh @ keys.t()                              # [grp, p+1]
            if mode == "faithful":
                s = rbf(rbf(s) * scale)
            else:
                s = s * scale
            pr = torch.softmax(s, dim=-1)
            o = pr @ vals
            out[b, h * grp:(h + 1) * grp] = o
    # KV write (after the reads: the reads above use the fresh K/V for the active slot)
    for b in range(T):
        blk, off = kv_slot(block_table, b, pos[b], cfg.block_size)
        if blk < 0:
            continue
        k_cache[blk, :, off] = kr[b].to(k_cache.dtype)
        v_cache[blk, :, off] = v[b].to(v_cache.dtype)
    attn = out.reshape(T, nq * D)
    if mode == "faithful":
        attn = rbf(attn)
    o = attn @ lw.wo.to(F32).t()
    if mode == "faithful":
        o = rbf(o)
    if trace is not None:
        trace.attn = attn
    return o


def decoder_layer(x_bf16: torch.Tensor, lw: LayerWeights, cfg: QwenConfig,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor,
                  block_table: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
                  mode: str, trace: Optional[LayerTrace] = None) -> torch.Tensor:
    """One decoder layer (``qwen.py:386-444``).  Input/outputs ``[T, H]``.

    faithful: the residual stream is bf16 and both adds round to bf16
    (``transformer_qwen.py:331-333,370-372``); returns bf16.
    fp32: residual kept in fp32; returns fp32.
    """
    if mode == "faithful":
        x = x_bf16.to(F32)
        xn1 = rbf(rmsnorm_hidden_faithful(x_bf16.to(BF16), lw.ln1, cfg.rms_eps, gamma_first=False))
    else:
        x = x_bf16.to(F32)
        xn1 = rmsnorm_fp32(x, lw.ln1, cfg.rms_eps)
    o = attention_layer(xn1, lw, cfg, k_cache, v_cache, positions, block_table, cos_tab,
                        sin_tab, mode, trace)
    if mode == "faithful":
        mid = rbf(x + o)
        moe = moe_block(mid.to(BF16), lw, cfg, mode, trace)
        out = rbf(mid + rbf(moe))
    else:
        mid = x + o
        moe = moe_block(mid, lw, cfg, mode, trace)
        out = mid + moe
    if trace is not None:
        trace.resid_mid, trace.resid_out = mid, out
    return out.to(BF16) if mode == "faithful" else out


def decode_step(x_bf16: torch.Tensor, layers: List[LayerWeights], cfg: QwenConfig,
                k_caches: List[torch.Tensor], v_caches: List[torch.Tensor],
                positions: torch.Tensor, block_table: torch.Tensor, cos_tab, sin_tab,
                final_norm: Optional[torch.Tensor], lm_head: Optional[torch.Tensor],
                mode: str, traces: Optional[List[LayerTrace]] = None,
                topk_hints: Optional[List[torch.Tensor]] = None, hint_gap: float = 0.0):
    """Full decode step: ``len(k_caches)`` layers (weights cycle through ``layers``),
    then the final RMSNorm and the LM head (``qwen_with_megakernel.py:20-21,589-594``).

    Returns ``(hidden [T,H] pre-final-norm, logits [T,V] fp32 or None)``.
    """
    x = x_bf16
    for li in range(len(k_caches)):
        tr = LayerTrace() if (traces is not None or topk_hints is not None) else None
        if topk_hints is not None:
            tr.topk_hint, tr.hint_gap = topk_hints[li], hint_gap
        x = decoder_layer(x, layers[li % len(layers)], cfg, k_caches[li], v_caches[li],
                          positions, block_table, cos_tab, sin_tab, mode, tr)
        if traces is not None:
            traces.append(tr)
    logits = None
    if lm_head is not None:
        if mode == "faithful":
            xn = rbf(rmsnorm_hidden_faithful(x.to(BF16), final_norm, cfg.rms_eps, gamma_first=False))
        else:
            xn = rmsnorm_fp32(x, final_norm, cfg.rms_eps)
        logits = xn @ lm_head.to(F32).t()
    return x, logits


def compare(a: torch.Tensor, b: torch.Tensor) -> Dict[str, float]:
    """max-abs difference and cosine similarity of two tensors (flattened, fp32)."""
    a = a.to(F32).flatten()
    b = b.to(F32).flatten()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    return {"max_abs": (a - b).abs().max().item(), "cosine": cos}
