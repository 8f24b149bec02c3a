"""The MoE block on tcgen05/TMEM grouped GEMMs (``nkm_moe_block_tc``) against the oracle.

Config 3's expert stage (64 tokens, top-8 over 128 experts of Qwen3-30B-A3B, ~4 tokens per
expert) and denser batches (256 tokens), uniform and skewed routing: router top-k indices
bit-exact against the oracle's selection on the same input (the kernel's fixed-order fp32
logits), routing weights within one bf16 ulp, block output within max-abs 2e-2 / cosine 0.999
of the fp32 oracle; at 32 tokens the block equals the decode kernel's MoE block within the same
tolerance.
"""
import pytest
import torch

from oracle import qwen3_moe_oracle as O
from tests.qwen_cases import BF16, gpu_layers, make_layers, qwen_cfg, shape_of, skew_bias

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _block(lw, cfg, dev, max_tokens):
    from nki_moe_megakernel_b200.engine import MoeTcBlock

    return MoeTcBlock(lw.ln2, lw.router, lw.gate_up, lw.down, eps=cfg.rms_eps, top_k=cfg.top_k, max_tokens=max_tokens,
                      router_bias=lw.router_bias, device=dev)


@pytest.mark.parametrize("T,skewed", [(64, False), (64, True), (256, False)])
def test_tc_moe_block_vs_oracle(dev, T, skewed):
    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=700 + T)[0]
    if skewed:
        lw.router_bias = skew_bias(cfg)
    x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(T + int(skewed))).to(BF16)
    blk = _block(lw, cfg, dev, max_tokens=T)
    y, idx, w = blk(x.to(dev))
    assert blk.status() == 0
    xn32 = O.rmsnorm_hidden_faithful(x, lw.ln2, cfg.rms_eps, gamma_first=True)
    logits = O.router_logits_fixed(xn32, lw.router)
    if lw.router_bias is not None:
        logits = logits + lw.router_bias
    assert torch.equal(idx.cpu().long(), O.topk_select(logits, cfg.top_k))
    _, w_ref = O.router_topk(logits, cfg.top_k, "faithful")
    torch.testing.assert_close(w.cpu(), w_ref, rtol=8e-3, atol=1e-6)
    ref = O.moe_block(x, lw, cfg, "fp32")
    r = O.compare(y.float().cpu(), ref)
    print(f"[tc moe T={T} skewed={skewed}] {r}", flush=True)
    assert r["max_abs"] <= ATOL and r["cosine"] >= COS, r
    # twice in a row on the same workspace: identical
    y2, _, _ = blk(x.to(dev))
    assert blk.status() == 0 and torch.equal(y2, y)


def test_tc_moe_block_matches_decode_kernel_block(dev):
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=777)[0]
    x = torch.randn(32, cfg.hidden, generator=torch.Generator().manual_seed(8)).to(BF16).to(dev)
    y, idx, _ = _block(lw, cfg, dev, max_tokens=32)(x, residual=True)
    eng = Qwen3MoeMegakernel(shape_of(cfg, 1, 0), gpu_layers([lw], dev, attention=False), max_batch=32, num_blocks=0,
                             kv_pools=False)
    want = eng.moe_block(0, x, residual=True, trace=True)
    assert eng.status() == 0
    assert torch.equal(idx, want["topk_idx"][0])
    r = O.compare(y.float().cpu(), want["hidden"].float().cpu())
    assert r["max_abs"] <= ATOL and r["cosine"] >= COS, r


@pytest.mark.parametrize("T", [64, 256])
def test_tc_moe_block_mxfp8_vs_oracle(dev, T):
    """MXFP8 expert weights (OCP MX: e4m3 values, e8m0 scale per 32 along K): the block equals the
    fp32 oracle run on the dequantised weights (exact in bf16) within max-abs 2e-2 / cosine 0.999,
    routing bit-exact as with bf16 weights, and the same call twice gives the same bytes."""
    from nki_moe_megakernel_b200.engine import MoeTcBlock

    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=900 + T)[0]
    gc, gs = O.mxfp8_quantize(lw.gate_up.float())
    dc, ds = O.mxfp8_quantize(lw.down.float())
    lw.gate_up = O.mxfp8_dequant(gc, gs).to(BF16)
    lw.down = O.mxfp8_dequant(dc, ds).to(BF16)
    assert torch.equal(lw.gate_up.float(), O.mxfp8_dequant(gc, gs))  # the dequantised weights are bf16 values
    x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(T + 5)).to(BF16)
    blk = MoeTcBlock(lw.ln2, lw.router, None, None, eps=cfg.rms_eps, top_k=cfg.top_k, max_tokens=T, device=dev,
                     mxfp8=(gc, gs, dc, ds))
    y, idx, w = blk(x.to(dev))
    assert blk.status() == 0
    logits = O.router_logits_fixed(O.rmsnorm_hidden_faithful(x, lw.ln2, cfg.rms_eps, gamma_first=True), lw.router)
    assert torch.equal(idx.cpu().long(), O.topk_select(logits, cfg.top_k))
    ref = O.moe_block(x, lw, cfg, "fp32")
    r = O.compare(y.float().cpu(), ref)
    print(f"[tc moe MXFP8 T={T}] {r}", flush=True)
    assert r["max_abs"] <= ATOL and r["cosine"] >= COS, r
    # the bf16-weight block on the same (dequantised) weights computes the same products
    yb, _, _ = _block(lw, cfg, dev, max_tokens=T)(x.to(dev))
    rb = O.compare(y.float().cpu(), yb.float().cpu())
    assert rb["max_abs"] <= 1e-2, rb
    y2, _, _ = blk(x.to(dev))
    assert blk.status() == 0 and torch.equal(y2, y)
