"""GPU parity of the decode megakernel against the CPU oracle (through the C ABI).

Checks (tolerances stated at each assert):
* fragment-tiled weight packing equals the documented layout bit for bit;
* router logits and top-k expert indices bit-exact when both sides get the same input;
* KV-cache slot writes bit-exact (placement and values, given the same raw projection) and
  every other byte of the pools untouched (NaN-filled unused slots stay NaN and never leak);
* block / layer outputs within max-abs 2e-2 and cosine >= 0.999 of the fp32 oracle.
"""
import pytest
import torch

from oracle import qwen3_moe_oracle as O
from tests.qwen_cases import (BF16, bits_equal, gpu_layers, make_kv, make_layers, qwen_cfg, shape_of,
                              skew_bias)

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _engine(cfg, gl, n_layers, max_batch, num_blocks, vocab=0, head=None, kv=True):
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    fn, lm = (None, None) if head is None else head
    return Qwen3MoeMegakernel(shape_of(cfg, n_layers, vocab), gl, max_batch=max_batch, num_blocks=num_blocks,
                              final_norm=fn, lm_head=lm, kv_pools=kv)


def _close(a, b, atol=ATOL, cos=COS, what=""):
    r = O.compare(a.float().cpu(), b.float().cpu())
    assert r["max_abs"] <= atol and r["cosine"] >= cos, (what, r)
    return r


# ----------------------------------------------------------------------------- layout
def _ft_reference(w: torch.Tensor, gate_up: bool) -> torch.Tensor:
    R, K = w.shape
    if gate_up:
        I = R // 2
        order = []
        for s in range(I // 8):
            order += list(range(8 * s, 8 * s + 8)) + list(range(I + 8 * s, I + 8 * s + 8))
        w = w[torch.tensor(order)]
    u = w.reshape(R // 16, 2, 8, K // 32, 4, 8)          # rs, h, g, kt, t, j
    return u.permute(0, 3, 1, 2, 4, 5).reshape(R, K)     # rs, kt, h, (g t), j


@pytest.mark.parametrize("gate_up", [False, True])
def test_pack_ft_layout(dev, gate_up):
    from nki_moe_megakernel_b200.engine import pack_ft
    from nki_moe_megakernel_b200 import _lib

    g = torch.Generator().manual_seed(1)
    w = torch.randn(3, 96, 128, generator=g).to(BF16)
    got = pack_ft(w.to(dev), _lib.NKM_PACK_GATE_UP if gate_up else _lib.NKM_PACK_PLAIN).cpu()
    for i in range(3):
        assert bits_equal(got[i].reshape(96, 128), _ft_reference(w[i], gate_up))


# ----------------------------------------------------------------------------- MoE block
@pytest.mark.parametrize("T,skewed", [(32, False), (32, True), (1, False), (5, False), (8, True)])
def test_moe_block(dev, T, skewed):
    """router_topk + moe_tkg (config 1 at T=32, uniform and skewed routing)."""
    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=100 + T)[0]
    if skewed:
        lw.router_bias = skew_bias(cfg)
    x = (torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(5 + T))).to(BF16)
    eng = _engine(cfg, gpu_layers([lw], dev, attention=False, router_bias=lw.router_bias), 1, max(T, 1), 0,
                  kv=False)
    res = eng.moe_block(0, x.to(dev), residual=False, trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    # bit-exact router logits and indices on the identical input
    xn32 = O.rmsnorm_hidden_faithful(x, lw.ln2, cfg.rms_eps, gamma_first=True)
    logits = O.router_logits_fixed(xn32, lw.router)
    if lw.router_bias is not None:
        logits = logits + lw.router_bias
    assert torch.equal(res["router_logits"][0].cpu(), logits)
    idx = O.topk_select(logits, cfg.top_k)
    assert torch.equal(res["topk_idx"][0].cpu().long(), idx)
    _, w_ref = O.router_topk(logits, cfg.top_k, "faithful")
    torch.testing.assert_close(res["topk_w"][0].cpu(), w_ref, rtol=8e-3, atol=1e-6)  # 1 bf16 ulp
    if skewed:
        hot = torch.isin(idx, torch.tensor([3, 17, 64, 101])).float().mean().item()
        assert hot >= 0.45, hot
    ref = O.moe_block(x, lw, cfg, "fp32")
    _close(res["hidden"], ref, what="moe out vs fp32")


# ----------------------------------------------------------------------------- attention
POSITION_SETS = [
    [1024, 1024, 1024, 1024],      # config 0
    [0, 1, 127, 128],              # empty context, page boundaries
    [1000, 33, 257, 5],            # ragged, not multiples of the 32-token tile
]


@pytest.mark.parametrize("positions", POSITION_SETS)
def test_attention_block_kv_and_output(dev, positions):
    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=7)[0]
    B = len(positions)
    NB = sum(p // 128 + 1 for p in positions) + 3
    k0, v0, table = make_kv(cfg, 1, positions, NB, seed=11)
    x = torch.randn(B, cfg.hidden, generator=torch.Generator().manual_seed(3)).to(BF16)
    eng = _engine(cfg, gpu_layers([lw], dev, moe=False), 1, B, NB)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.attention_block(0, x.to(dev), pos.to(dev), table.to(dev), residual=False, trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    kg, vg = eng.k_pool.cpu(), eng.v_pool.cpu()
    qkv = res["qkv"][0].cpu()
    cos, sin = O.rope_tables(4096, cfg.head_dim, cfg.rope_theta)
    nq, nkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    # raw projections vs the oracle's bf16-rounded GEMV (order of fp32 sums differs)
    xn1 = O.rbf(O.rmsnorm_hidden_faithful(x, lw.ln1, cfg.rms_eps, gamma_first=False))
    wqkv = torch.cat([lw.wq, lw.wk, lw.wv], 0).float()
    _close(qkv, O.rbf(xn1 @ wqkv.t()), atol=1e-2, cos=0.9999, what="qkv")
    kexp, vexp = k0.clone(), v0.clone()
    for b, p in enumerate(positions):
        blk, off = int(table[b, p // 128]), p % 128
        kraw = qkv[b, nq * D:(nq + nkv) * D].view(nkv, D)
        vraw = qkv[b, (nq + nkv) * D:].view(nkv, D)
        knew = O.head_norm_rope_faithful(kraw, lw.k_norm, cos[p], sin[p], cfg.rms_eps)
        kexp[0, blk, :, off] = knew.to(BF16)
        vexp[0, blk, :, off] = vraw.to(BF16)
    assert bits_equal(kg, kexp), "K pool differs from the expected in-place write"
    assert bits_equal(vg, vexp), "V pool differs from the expected in-place write"
    # output vs the fp32 oracle
    kc, vc = k0.clone()[0], v0.clone()[0]
    ref = O.attention_layer(O.rmsnorm_fp32(x, lw.ln1, cfg.rms_eps), lw, cfg, kc, vc, pos, table,
                            *O.rope_tables(4096, cfg.head_dim, cfg.rope_theta, torch.float32), "fp32")
    _close(res["hidden"], ref, what="attention out vs fp32")


def test_attention_skip_write_and_bad_block(dev):
    """Block id -1 at the write slot skips the write; an out-of-range id is flagged."""
    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=8)[0]
    positions = [200, 64]
    NB = 8
    k0, v0, table = make_kv(cfg, 1, positions, NB, seed=12)
    table[1, 0] = -1  # sequence 1 writes at slot 64 of block -1: skipped
    x = torch.randn(2, cfg.hidden, generator=torch.Generator().manual_seed(4)).to(BF16)
    eng = _engine(cfg, gpu_layers([lw], dev, moe=False), 1, 2, NB)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    # sequence 1 has no readable context block -> its reads are clamped and flagged
    eng.attention_block(0, x.to(dev), torch.tensor(positions, dtype=torch.int32, device=dev), table.to(dev))
    st = eng.status()
    from nki_moe_megakernel_b200 import _lib

    assert st == _lib.NKM_ERR_INDEX
    kg = eng.k_pool.cpu()
    for blk in range(NB):
        if blk != int(table[0, 1]):
            assert bits_equal(kg[0, blk], k0[0, blk]), blk


def test_out_of_range_token_id_and_position_flagged(dev):
    """A token id >= vocab and a position beyond the block-table row are clamped in bounds and
    reported as NKM_ERR_INDEX; the next valid step reports 0 again."""
    from nki_moe_megakernel_b200 import _lib
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=13)[0]
    positions = [5, 100]
    NB = 4
    k0, v0, table = make_kv(cfg, 1, positions, NB, seed=14, nan_fill=False)   # one block per sequence
    V = 64
    embed = torch.randn(V, cfg.hidden, generator=torch.Generator().manual_seed(15)).to(BF16)
    eng = Qwen3MoeMegakernel(shape_of(cfg, 1, V), gpu_layers([lw], dev), max_batch=2, num_blocks=NB,
                             embed=embed.to(dev))
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    tab = table.to(dev)
    ok_ids = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    ok_pos = torch.tensor(positions, dtype=torch.int32, device=dev)
    eng.decode_step(ok_pos, tab, input_ids=ok_ids)
    assert eng.status() == 0
    eng.decode_step(ok_pos, tab, input_ids=torch.tensor([1, V], dtype=torch.int32, device=dev))
    assert eng.status() == _lib.NKM_ERR_INDEX
    eng.decode_step(torch.tensor([5, 128], dtype=torch.int32, device=dev), tab, input_ids=ok_ids)
    assert eng.status() == _lib.NKM_ERR_INDEX
    eng.decode_step(ok_pos, tab, input_ids=ok_ids)
    assert eng.status() == 0


def test_grid_wait_timeout_reports_status(dev):
    """Failure detection without a fault: the grid barrier counter is set so that the first
    barrier can never be reached; every CTA gives up after the bounded wait (2 s), the step
    ends, the status reads NKM_ERR_TIMEOUT, and the next step on the same handle succeeds."""
    import time

    from nki_moe_megakernel_b200 import _lib

    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=16)[0]
    x = torch.randn(4, cfg.hidden, generator=torch.Generator().manual_seed(17)).to(BF16).to(dev)
    eng = _engine(cfg, gpu_layers([lw], dev, attention=False), 1, 4, 0, kv=False)
    want = eng.moe_block(0, x)["hidden"]
    assert eng.status() == 0
    eng.workspace[0:4].view(torch.int32).fill_(-(1 << 30))  # arrival count far below any target
    t0 = time.time()
    eng.moe_block(0, x)
    st = eng.status()
    elapsed = time.time() - t0
    assert st & _lib.NKM_ERR_TIMEOUT, st
    assert 1.0 < elapsed < 30.0, elapsed
    got = eng.moe_block(0, x)["hidden"]  # status() cleared the control words
    assert eng.status() == 0
    assert torch.equal(got, want)


def test_qkv_in_and_sentinel_wait_timeout(dev):
    """Attention on caller-written q/k/v projections (NKM_STAGE_QKV_IN) equals the projecting
    path bit for bit.  Then the QKV buffer is left as every launch leaves it (each element
    marked unwritten, 0xffff) and nothing writes it: the attention's element waits (the
    barrier-free stage A -> B handoff) run out after the bounded wait (2 s), the launch ends with
    NKM_ERR_TIMEOUT instead of hanging, and the next call with written rows is correct again."""
    import time

    from nki_moe_megakernel_b200 import _lib

    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=18)[0]
    positions = [300, 17, 128, 1000]
    B = len(positions)
    NB = sum(p // 128 + 1 for p in positions) + 1
    k0, v0, table = make_kv(cfg, 1, positions, NB, seed=19)
    x = torch.randn(B, cfg.hidden, generator=torch.Generator().manual_seed(20)).to(BF16).to(dev)
    eng = _engine(cfg, gpu_layers([lw], dev, moe=False), 1, B, NB)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    pos_d = torch.tensor(positions, dtype=torch.int32, device=dev)
    tab_d = table.to(dev)
    want = eng.attention_block(0, x, pos_d, tab_d, trace=True)
    assert eng.status() == 0
    k_want, v_want = eng.k_pool.clone(), eng.v_pool.clone()
    buf = eng.qkv_buffer()
    assert bool((buf[:B].view(torch.int16) == -1).all()), "the launch leaves the buffer marked unwritten"
    buf[:B].copy_(want["qkv"][0])
    got = eng.attention_block(0, x, pos_d, tab_d, qkv_in=True)
    assert eng.status() == 0
    assert bits_equal(got["hidden"].cpu(), want["hidden"].cpu())
    assert bits_equal(eng.k_pool.cpu(), k_want.cpu()) and bits_equal(eng.v_pool.cpu(), v_want.cpu())
    # no producer: the buffer stays marked
    t0 = time.time()
    eng.attention_block(0, x, pos_d, tab_d, qkv_in=True)
    st = eng.status()
    elapsed = time.time() - t0
    assert st & _lib.NKM_ERR_TIMEOUT, st
    assert 1.0 < elapsed < 30.0, elapsed
    buf[:B].copy_(want["qkv"][0])
    got = eng.attention_block(0, x, pos_d, tab_d, qkv_in=True)
    assert eng.status() == 0
    assert bits_equal(got["hidden"].cpu(), want["hidden"].cpu())
    assert bits_equal(eng.k_pool.cpu(), k_want.cpu()) and bits_equal(eng.v_pool.cpu(), v_want.cpu())


# ----------------------------------------------------------------------------- layers / step
def test_decoder_layer_config0(dev):
    """Config 0: one layer, B=4, ctx 1024 (attention + MoE + residuals)."""
    cfg = qwen_cfg(n_layers=1)
    lw = make_layers(cfg, 1, seed=21)[0]
    positions = [1024, 1024, 1024, 1024]
    NB = 40
    k0, v0, table = make_kv(cfg, 1, positions, NB, seed=22)
    x = torch.randn(4, cfg.hidden, generator=torch.Generator().manual_seed(23)).to(BF16)
    eng = _engine(cfg, gpu_layers([lw], dev), 1, 4, NB)
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.decode_step(pos.to(dev), table.to(dev), x=x.to(dev), want_logits=False, trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    ref = O.decoder_layer(x, lw, cfg, k0.clone()[0], v0.clone()[0], pos, table,
                          *O.rope_tables(4096, cfg.head_dim, cfg.rope_theta, torch.float32), "fp32")
    _close(res["hidden"], ref, what="layer out vs fp32")
    assert bits_equal(res["resid_out"][0].to(BF16).cpu(), res["hidden"].cpu()), "trace == output"
    # router on the GPU's own post-attention residual: bit-exact
    mid = res["resid_mid"][0].cpu()
    logits = O.router_logits_fixed(O.rmsnorm_hidden_faithful(mid, lw.ln2, cfg.rms_eps, True), lw.router)
    assert torch.equal(res["router_logits"][0].cpu(), logits)
    assert torch.equal(res["topk_idx"][0].cpu().long(), O.topk_select(logits, cfg.top_k))


@pytest.mark.parametrize("B,ctx,n_layers", [(8, 2048, 4), (16, 512, 2)])
def test_multilayer_step_teacher_forced(dev, B, ctx, n_layers):
    """Full step (layers + final norm + LM head), checked layer by layer against the fp32
    oracle fed the GPU's own input of that layer, plus end-to-end logits."""
    cfg = qwen_cfg(n_layers=n_layers, vocab=4096)
    distinct = make_layers(cfg, 2, seed=31)
    layers = [distinct[i % 2] for i in range(n_layers)]
    g = torch.Generator().manual_seed(32)
    positions = [max(0, ctx - int(torch.randint(0, ctx, (1,), generator=g))) if b % 3 else ctx for b in range(B)]
    positions[-1] = 0
    NB = sum(p // 128 + 1 for p in positions) + 2
    k0, v0, table = make_kv(cfg, n_layers, positions, NB, seed=33)
    final_norm = (1 + 0.02 * torch.randn(cfg.hidden, generator=g)).to(BF16)
    lm_head = (0.02 * torch.randn(cfg.vocab, cfg.hidden, generator=g)).to(BF16)
    x = torch.randn(B, cfg.hidden, generator=g).to(BF16)
    gl = gpu_layers(distinct, dev)
    eng = _engine(cfg, [gl[i % 2] for i in range(n_layers)], n_layers, B, NB, vocab=cfg.vocab,
                  head=(final_norm.to(dev), lm_head.to(dev)))
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    pos = torch.tensor(positions, dtype=torch.int32)
    res = eng.decode_step(pos.to(dev), table.to(dev), x=x.to(dev), trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    cos32, sin32 = O.rope_tables(8192, cfg.head_dim, cfg.rope_theta, torch.float32)
    inp = x
    for li in range(n_layers):
        ref = O.decoder_layer(inp, layers[li], cfg, k0[li].clone(), v0[li].clone(), pos, table, cos32, sin32,
                              "fp32")
        out = res["resid_out"][li].cpu()
        _close(out, ref, what=f"layer {li}")
        mid = res["resid_mid"][li].cpu()
        logits = O.router_logits_fixed(O.rmsnorm_hidden_faithful(mid, layers[li].ln2, cfg.rms_eps, True),
                                       layers[li].router)
        assert torch.equal(res["router_logits"][li].cpu(), logits), li
        assert torch.equal(res["topk_idx"][li].cpu().long(), O.topk_select(logits, cfg.top_k)), li
        inp = out
    xn = O.rmsnorm_fp32(res["hidden"].cpu(), final_norm, cfg.rms_eps)
    _close(res["logits"], xn @ lm_head.float().t(), what="logits (teacher-forced)")
    # end to end (no teacher forcing) against the fp32 oracle
    _, ref_logits = O.decode_step(x, layers, cfg, [k0[i].clone() for i in range(n_layers)],
                                  [v0[i].clone() for i in range(n_layers)], pos, table, cos32, sin32,
                                  final_norm, lm_head, "fp32")
    r = O.compare(res["logits"].cpu(), ref_logits)
    assert r["max_abs"] <= ATOL and r["cosine"] >= COS, r


def test_multi_token_rows_kv_first(dev):
    """Rows of one sequence at consecutive positions in one launch (NKM_STAGE_KV_FIRST: chunked
    prefill / multi-token decode): two sequences with 4 and 3 new tokens.  Every row's logits and
    hidden state match the fp32 oracle run token by token (each token seeing the K/V of the
    earlier ones), and the layer-0 K/V slots of all 7 tokens are bit-exact."""
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    L = 2
    cfg = qwen_cfg(n_layers=L, vocab=4096)
    distinct = make_layers(cfg, 2, seed=61)
    starts, counts = [300, 127], [4, 3]
    NB = sum((s0 + n) // 128 + 1 for s0, n in zip(starts, counts)) + 2
    k0, v0, table = make_kv(cfg, L, [s0 + n for s0, n in zip(starts, counts)], NB, seed=62)
    g = torch.Generator().manual_seed(63)
    final_norm = (1 + 0.02 * torch.randn(cfg.hidden, generator=g)).to(BF16)
    lm_head = (0.02 * torch.randn(cfg.vocab, cfg.hidden, generator=g)).to(BF16)
    rows = [(b, s0 + i) for b, (s0, n) in enumerate(zip(starts, counts)) for i in range(n)]
    B = len(rows)
    x = torch.randn(B, cfg.hidden, generator=g).to(BF16)
    pos = torch.tensor([p for _, p in rows], dtype=torch.int32)
    row_table = torch.stack([table[b] for b, _ in rows]).contiguous()
    eng = Qwen3MoeMegakernel(shape_of(cfg, L, cfg.vocab), gpu_layers(distinct, dev), max_batch=B, num_blocks=NB,
                             final_norm=final_norm.to(dev), lm_head=lm_head.to(dev))
    eng.k_pool.copy_(k0.to(dev))
    eng.v_pool.copy_(v0.to(dev))
    res = eng.decode_step(pos.to(dev), row_table.to(dev), x=x.to(dev), trace=True, kv_first=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    # token by token through the fp32 oracle (its caches are updated in place)
    kc = [k0[i].clone() for i in range(L)]
    vc = [v0[i].clone() for i in range(L)]
    cos32, sin32 = O.rope_tables(4096, cfg.head_dim, cfg.rope_theta, torch.float32)
    order = sorted(range(B), key=lambda r: rows[r][1])
    for r in order:
        b, p_ = rows[r]
        h, lg = O.decode_step(x[r:r + 1], distinct, cfg, kc, vc, pos[r:r + 1], table[b:b + 1], cos32, sin32,
                              final_norm, lm_head, "fp32")
        _close(res["hidden"][r], h[0], what=f"hidden row {r}")
        _close(res["logits"][r], lg[0], what=f"logits row {r}")
    # layer 0 K/V slots: bit-exact from the kernel's own raw projections
    cos, sin = O.rope_tables(4096, cfg.head_dim, cfg.rope_theta)
    nq, nkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    kg, vg = eng.k_pool.cpu(), eng.v_pool.cpu()
    for r, (b, p_) in enumerate(rows):
        qkv = res["qkv"][0, r].cpu()
        knew = O.head_norm_rope_faithful(qkv[nq * D:(nq + nkv) * D].view(nkv, D), distinct[0].k_norm, cos[p_],
                                         sin[p_], cfg.rms_eps).to(BF16)
        blk, off = int(table[b, p_ // 128]), p_ % 128
        assert bits_equal(kg[0, blk, :, off], knew), r
        assert bits_equal(vg[0, blk, :, off], qkv[(nq + nkv) * D:].view(nkv, D)), r
