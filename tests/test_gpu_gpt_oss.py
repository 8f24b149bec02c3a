"""GPU parity of the GPT-OSS decode kernel (``nkm_gptoss_*``) against the fp32 oracle
(``oracle/gpt_oss_oracle.py``, pinned against Hugging Face ``GptOssForCausalLM``).

* Two layers at the GPT-OSS-20B shape (hidden 2880, 64/8 heads of 64, 32 MXFP4 experts top-4,
  intermediate 2880; layer 0 sliding window 128, layer 1 full), ragged positions crossing K/V
  blocks and the window edge: every layer's output within max-abs 2e-2 / cosine 0.999 of the
  oracle fed the kernel's own layer input; router logits bit-exact in the kernel's fixed summation
  order and the top-4 experts identical; K and V slots bit-exact given the kernel's own q/k/v
  projections; untouched cache bytes unchanged.
* Config 4 shape, shortened to 4 layers (two distinct weight sets, sliding/full alternating):
  B=16, contexts around 4096, vocabulary 201088, free running against the oracle: hidden and
  logits within max-abs 2e-2 / cosine 0.999.
* Padded hidden size (``hidden_actual``, ``rmsnorm_tkg.py:49-147``): a model whose rows are
  padded with zeros from 256 to 320 gives the logits of the unpadded model.
"""
import pytest
import torch

from oracle import gpt_oss_oracle as G
from oracle import qwen3_moe_oracle as Q
from tests.qwen_cases import BF16, bits_equal, make_kv

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _shape(cfg: G.GptOssConfig, n_layers: int, vocab: int, hidden_actual: int = 0):
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssShape

    return GptOssShape(hidden_size=cfg.hidden, hidden_actual=hidden_actual, num_attention_heads=cfg.n_q_heads,
                       num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, num_local_experts=cfg.n_experts,
                       num_experts_per_tok=cfg.top_k, intermediate_size=cfg.inter, num_hidden_layers=n_layers,
                       vocab_size=vocab, rms_norm_eps=cfg.rms_eps, sliding_window=cfg.sliding_window)


def _gpu_layer(lw: G.GptOssLayer, dev, sliding: bool):
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssGpuLayer

    t = {k: getattr(lw, k).to(dev) for k in ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "sinks", "ln1", "ln2",
                                             "router", "router_b", "gu_codes", "gu_scales", "gu_b", "dn_codes",
                                             "dn_scales", "dn_b")}
    return GptOssGpuLayer(t, sliding)


def _to_vt(v):  # oracle V [.., 128, 64] -> kernel V^T blocks [.., 64, 128]
    return v.transpose(-1, -2).contiguous()


def _fixed_logits(mid: torch.Tensor, lw: G.GptOssLayer, cfg: G.GptOssConfig) -> torch.Tensor:
    """Router logits in the kernel's order: rows zero-padded to a multiple of 256 (adding 0 * 0
    terms changes no fp32 sum), lane-sequential then butterfly sums."""
    H = mid.shape[-1]
    pad = (-H) % 256
    x = torch.nn.functional.pad(mid, (0, pad))
    ss = Q.lane_sum_hidden(x * x)
    r = Q.rstd_fixed_div(ss, H, cfg.rms_eps)
    xn = (x * r[:, None]) * torch.nn.functional.pad(lw.ln2.float(), (0, pad))
    w = torch.nn.functional.pad(lw.router.float(), (0, pad))
    return Q.lane_sum_hidden(w[None] * xn[:, None, :]) + lw.router_b.float()


def test_two_layers_teacher_forced(dev):
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssMegakernel

    cfg = G.GptOssConfig(n_layers=2)
    gen = torch.Generator().manual_seed(901)
    lws = [G.random_layer(cfg, gen) for _ in range(2)]
    positions = [300, 17, 128, 1000]
    B = len(positions)
    NB = sum(p // 128 + 1 for p in positions) + 2
    k0, v0, table = make_kv(cfg, 2, positions, NB, seed=902)
    x = torch.randn(B, cfg.hidden, generator=gen).to(BF16)
    eng = GptOssMegakernel(_shape(cfg, 2, 0), [_gpu_layer(lws[i], dev, cfg.is_sliding(i)) for i in range(2)],
                           max_batch=B, num_blocks=NB, max_context=1152, device=dev)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(_to_vt(v0).to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.decode_step(pos.to(dev), table.to(dev), x=x.to(dev), want_logits=False, trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    cos, sin = eng.rope_cos.cpu(), eng.rope_sin.cpu()
    ocos, osin = G.rope_tables(cfg, eng.rope_max)
    assert torch.allclose(cos, ocos, atol=2e-6) and torch.allclose(sin, osin, atol=2e-6)
    kg, vg = eng.k_pool.cpu(), eng.v_pool.cpu().transpose(-1, -2)
    inp = x.float()
    nq, nkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    for li in range(2):
        lw = lws[li]
        ref = G.decoder_layer(inp, lw, cfg, li, k0[li].clone(), v0[li].clone(), pos, table, cos, sin)
        out = res["resid_out"][li].cpu()
        r = G.compare(out, ref)
        assert r["max_abs"] <= ATOL and r["cosine"] >= COS, (li, r)
        mid = res["resid_mid"][li].cpu()
        lg = _fixed_logits(mid, lw, cfg)
        assert torch.equal(res["router_logits"][li].cpu(), lg), li
        idx = torch.sort(lg, dim=-1, descending=True, stable=True).indices[:, :cfg.top_k]
        assert torch.equal(res["topk_idx"][li].cpu().long(), idx), li
        # K / V slots from the kernel's own projections (fp32 + bias): RoPE in fp32, bf16
        qkv = res["qkv"][li].cpu()
        for b, p in enumerate(positions):
            kraw = qkv[b, nq * D:(nq + nkv) * D].view(nkv, D)
            knew = G.apply_rope(kraw, cos[p], sin[p]).to(BF16)
            vnew = qkv[b, (nq + nkv) * D:].view(nkv, D).to(BF16)
            blk, off = int(table[b, p // 128]), p % 128
            assert bits_equal(kg[li, blk, :, off], knew), (li, b)
            assert bits_equal(vg[li, blk, :, off], vnew), (li, b)
        inp = out
    # every other slot untouched (NaN-filled unused slots stay NaN)
    kexp, vexp = k0.clone(), v0.clone()
    for li in range(2):
        for b, p in enumerate(positions):
            blk, off = int(table[b, p // 128]), p % 128
            kexp[li, blk, :, off] = kg[li, blk, :, off]
            vexp[li, blk, :, off] = vg[li, blk, :, off]
    assert bits_equal(kg, kexp) and bits_equal(vg.contiguous(), vexp)


def test_config4_shape(dev):
    """Config 4's shapes (full width, B=16, contexts near 4096, vocab 201088) over 4 layers: every
    layer within max-abs 2e-2 / cosine 0.999 of the fp32 oracle layer on the kernel's own input
    (near-tie routing follows the kernel), the logits within the same bounds of the fp32 final
    norm + LM head on the kernel's final residual, and the free-running step at cosine >= 0.999
    (its max-abs printed: four bf16 layers run free drift past 2e-2 on |x| ~ 5)."""
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssMegakernel

    L, B = 4, 16
    cfg = G.GptOssConfig(n_layers=L)
    gen = torch.Generator().manual_seed(911)
    distinct = [G.random_layer(cfg, gen) for _ in range(2)]
    positions = [4096 - (b * 37) % 300 for b in range(B)]
    positions[3] = 4095
    positions[7] = 129
    NB = sum(p // 128 + 1 for p in positions) + 2
    k0, v0, table = make_kv(cfg, L, positions, NB, seed=912, nan_fill=False)
    fnorm = (1 + 0.02 * torch.randn(cfg.hidden, generator=gen)).to(BF16)
    lm = (0.02 * torch.randn(cfg.vocab, cfg.hidden, generator=gen)).to(BF16)
    x = torch.randn(B, cfg.hidden, generator=gen).to(BF16)
    gl = [_gpu_layer(distinct[i], dev, cfg.is_sliding(i)) for i in range(2)]
    eng = GptOssMegakernel(_shape(cfg, L, cfg.vocab), [gl[i % 2] for i in range(L)], max_batch=B, num_blocks=NB,
                           max_context=4224, final_norm=fnorm.to(dev), lm_head=lm.to(dev), device=dev)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(_to_vt(v0).to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.decode_step(pos.to(dev), table.to(dev), x=x.to(dev), trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    logits = res["logits"].cpu()
    outs, idx = res["resid_out"].cpu(), res["topk_idx"].cpu()
    cos, sin = eng.rope_cos.cpu(), eng.rope_sin.cpu()
    eng.close()
    del eng, gl, res
    torch.cuda.empty_cache()
    worst = {"max_abs": 0.0, "cosine": 1.0}
    for li in range(L):
        inp = x.float() if li == 0 else outs[li - 1]
        ref = G.decoder_layer(inp, distinct[li % 2], cfg, li, k0[li].clone(), v0[li].clone(), pos, table, cos, sin,
                              topk_hint=idx[li], hint_gap=1e-4)
        r = G.compare(outs[li], ref)
        worst = {"max_abs": max(worst["max_abs"], r["max_abs"]), "cosine": min(worst["cosine"], r["cosine"])}
        assert r["max_abs"] <= ATOL and r["cosine"] >= COS, (li, r)
    ref_l_tf = G.rmsnorm(outs[L - 1], fnorm, cfg.rms_eps) @ lm.float().t()
    rl_tf = G.compare(logits, ref_l_tf)
    ref_h, ref_l = G.decode_step(x.float(), distinct, cfg, [k0[i].clone() for i in range(L)],
                                 [v0[i].clone() for i in range(L)], pos, table, cos, sin, fnorm, lm)
    rh, rl = G.compare(outs[L - 1], ref_h), G.compare(logits, ref_l)
    print(f"[gpt-oss 4 layers B=16 ctx~4096] teacher-forced worst layer {worst}, logits {rl_tf}; "
          f"free-running hidden {rh} logits {rl}", flush=True)
    assert rl_tf["max_abs"] <= ATOL and rl_tf["cosine"] >= COS, rl_tf
    assert rh["cosine"] >= COS and rl["cosine"] >= COS, (rh, rl)


def test_padded_hidden_matches_unpadded(dev):
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssMegakernel

    cfg = G.GptOssConfig(hidden=256, n_q_heads=8, n_kv_heads=2, n_experts=8, top_k=2, inter=128, n_layers=2,
                         vocab=512)
    gen = torch.Generator().manual_seed(921)
    lws = [G.random_layer(cfg, gen) for _ in range(2)]
    positions = [5, 140]
    NB = 6
    k0, v0, table = make_kv(cfg, 2, positions, NB, seed=922, nan_fill=False)
    fnorm = (1 + 0.02 * torch.randn(cfg.hidden, generator=gen)).to(BF16)
    lm = (0.02 * torch.randn(cfg.vocab, cfg.hidden, generator=gen)).to(BF16)
    x = torch.randn(2, cfg.hidden, generator=gen).to(BF16)
    pos = torch.tensor(positions, dtype=torch.int32, device=dev)
    HP = 320

    def padk(t):  # zero columns (input dimension) up to HP
        return torch.nn.functional.pad(t, (0, HP - t.shape[-1]))

    def padr(t, dim):  # zero rows (output dimension) up to HP
        pad = [0, 0] * (t.dim() - dim - 1) + [0, HP - t.shape[dim]]
        return torch.nn.functional.pad(t, pad)

    outs = []
    for padded in (False, True):
        gl = []
        for i, lw in enumerate(lws):
            t = {k: getattr(lw, k) for k in ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "sinks", "ln1", "ln2",
                                             "router", "router_b", "gu_codes", "gu_scales", "gu_b", "dn_codes",
                                             "dn_scales", "dn_b")}
            if padded:
                t.update(wq=padk(t["wq"]), wk=padk(t["wk"]), wv=padk(t["wv"]), wo=padr(t["wo"], 0), bo=padr(t["bo"], 0),
                         ln1=padr(t["ln1"], 0), ln2=padr(t["ln2"], 0), router=padk(t["router"]),
                         gu_codes=padk(t["gu_codes"]), gu_scales=torch.nn.functional.pad(t["gu_scales"], (0, 2)),
                         dn_codes=padr(t["dn_codes"], 1), dn_scales=padr(t["dn_scales"], 1), dn_b=padr(t["dn_b"], 1))
            from nki_moe_megakernel_b200.gpt_oss_engine import GptOssGpuLayer

            gl.append(GptOssGpuLayer({k: v.to(dev) for k, v in t.items()}, cfg.is_sliding(i)))
        c2 = G.GptOssConfig(**{**cfg.__dict__, "hidden": HP}) if padded else cfg
        shape = _shape(c2, 2, cfg.vocab, hidden_actual=256 if padded else 0)
        eng = GptOssMegakernel(shape, gl, max_batch=2, num_blocks=NB, max_context=256,
                               final_norm=(padr(fnorm, 0) if padded else fnorm).to(dev),
                               lm_head=(padk(lm) if padded else lm).to(dev), device=dev)
        eng.k_pool.copy_(k0.to(dev))
        eng.v_pool.copy_(_to_vt(v0).to(dev))
        xx = padk(x) if padded else x
        res = eng.decode_step(pos, table.to(dev), x=xx.to(dev))
        torch.cuda.synchronize()
        assert eng.status() == 0
        outs.append((res["hidden"][:, :256].float().cpu(), res["logits"].cpu()))
        eng.close()
    r = G.compare(outs[1][1], outs[0][1])
    assert r["max_abs"] <= 2e-3 and r["cosine"] >= 0.99999, r
    assert bool((torch.zeros(1) == 0).all())


def test_model_class_validate_against_hf():
    """``main.py --model gpt_oss --mode validate`` on a 2-layer random-init GPT-OSS-20B-shaped
    model (MXFP4 experts): the megakernel's teacher-forced logits pass the reference's tolerance
    map against Hugging Face ``GptOssForCausalLM`` (fp32) with the same weights."""
    from nki_moe_megakernel_b200 import main as drv

    rc = drv.main(["--model", "gpt_oss", "--mode", "validate", "--enable-nki", "--num-layers", "2", "--seq-len", "160",
                   "--num-tokens-to-check", "6", "--prompt", "I believe the meaning of life is"])
    assert rc == 0


def test_two_layers_fp8_kv(dev):
    """FP8 (e4m3) K/V cache (the reference's k_scale / v_scale quantisation,
    attention_block_tkg.py:213-218, 1694): the new K/V bytes equal e4m3(clip(x * scale, +-240)) of
    the kernel's own projections (round to nearest even), and the layer outputs stay within the
    tolerance of the fp32 oracle run on the dequantised cache, the new token's K/V included as the
    kernel quantised them (the reference attends to the quantised active K/V as well)."""
    from nki_moe_megakernel_b200.gpt_oss_engine import GptOssMegakernel

    KS, VS = 16.0, 16.0
    cfg = G.GptOssConfig(n_layers=2)
    gen = torch.Generator().manual_seed(931)
    lws = [G.random_layer(cfg, gen) for _ in range(2)]
    positions = [300, 17, 128, 1000]
    B = len(positions)
    NB = sum(p // 128 + 1 for p in positions) + 2
    k0, v0, table = make_kv(cfg, 2, positions, NB, seed=932, nan_fill=False)
    q8 = lambda t, s: (t.float() * s).clamp(-240, 240).to(torch.float8_e4m3fn)  # noqa: E731
    k8, v8 = q8(k0, KS), q8(v0, VS)
    x = torch.randn(B, cfg.hidden, generator=gen).to(BF16)
    eng = GptOssMegakernel(_shape(cfg, 2, 0), [_gpu_layer(lws[i], dev, cfg.is_sliding(i)) for i in range(2)],
                           max_batch=B, num_blocks=NB, max_context=1152, device=dev, kv_fp8=True, k_scale=KS,
                           v_scale=VS)
    eng.k_pool.copy_(k8.view(torch.uint8).to(dev))
    eng.v_pool.copy_(_to_vt(v8.view(torch.uint8)).to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.decode_step(pos.to(dev), table.to(dev), x=x.to(dev), want_logits=False, trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    cos, sin = eng.rope_cos.cpu(), eng.rope_sin.cpu()
    kg, vg = eng.k_pool.cpu(), eng.v_pool.cpu().transpose(-1, -2)
    nq, nkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    inp = x.float()
    # the new tokens' K/V as the kernel stored them (their bytes are checked below), dequantised
    kg8, vg8 = kg.view(torch.float8_e4m3fn).float() / KS, vg.view(torch.float8_e4m3fn).float() / VS
    for li in range(2):
        newk = torch.stack([kg8[li, int(table[b, p // 128]), :, p % 128] for b, p in enumerate(positions)])
        newv = torch.stack([vg8[li, int(table[b, p // 128]), :, p % 128] for b, p in enumerate(positions)])
        ref = G.decoder_layer(inp, lws[li], cfg, li, k8[li].float() / KS, v8[li].float() / VS, pos, table, cos, sin,
                              new_kv=(newk, newv))
        out = res["resid_out"][li].cpu()
        r = G.compare(out, ref)
        assert r["max_abs"] <= ATOL and r["cosine"] >= COS, (li, r)
        qkv = res["qkv"][li].cpu()
        for b, p in enumerate(positions):
            kraw = qkv[b, nq * D:(nq + nkv) * D].view(nkv, D)
            kexp = q8(G.apply_rope(kraw, cos[p], sin[p]), KS).view(torch.uint8)
            vexp = q8(qkv[b, (nq + nkv) * D:].view(nkv, D), VS).view(torch.uint8)
            blk, off = int(table[b, p // 128]), p % 128
            assert torch.equal(kg[li, blk, :, off], kexp), (li, b)
            assert torch.equal(vg[li, blk, :, off].contiguous(), vexp), (li, b)
        inp = out
