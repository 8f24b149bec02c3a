"""Pin the CPU oracle against the Hugging Face Qwen3-MoE golden fixture (CPU only).

The fixture (``tests/golden/make_golden.py``) holds a tiny seeded Qwen3-MoE model run by
transformers' own modules in fp32: per sequence a prefill that fills the KV cache, then one
decode token with its per-layer outputs and logits, and a standalone sparse-MoE call.
"""
import torch

from oracle import qwen3_moe_oracle as O
from tests.golden_utils import golden_config, golden_layers, load_golden, paged_from_contiguous


def _decode_all(mode):
    d = load_golden()
    cfg = golden_config(d)
    layers = golden_layers(d, cfg)
    sd = d["state_dict"]
    seqs = d["seqs"]
    gen = torch.Generator().manual_seed(7)
    cache_dtype = torch.float32 if mode == "fp32" else torch.bfloat16
    kc, vc = [], []
    table = None
    for li in range(cfg.n_layers):
        kpool, table = paged_from_contiguous([s["keys"][li] for s in seqs], cfg.n_kv_heads,
                                             cfg.head_dim, cfg.block_size, 16,
                                             torch.Generator().manual_seed(3), cache_dtype)
        vpool, _ = paged_from_contiguous([s["values"][li] for s in seqs], cfg.n_kv_heads,
                                         cfg.head_dim, cfg.block_size, 16,
                                         torch.Generator().manual_seed(3), cache_dtype)
        kc.append(kpool)
        vc.append(vpool)
    del gen
    positions = torch.tensor([s["prefix_len"] for s in seqs], dtype=torch.int32)
    x = sd["model.embed_tokens.weight"][[s["new_id"] for s in seqs]]
    cos, sin = O.rope_tables(4096, cfg.head_dim, cfg.rope_theta,
                             torch.float32 if mode == "fp32" else torch.bfloat16)
    traces = []
    hid, logits = O.decode_step(x, layers, cfg, kc, vc, positions, table, cos, sin,
                                sd["model.norm.weight"], sd["lm_head.weight"], mode, traces)
    return d, cfg, hid, logits, traces, kc, vc, table, positions


def test_oracle_fp32_matches_hf_decode():
    d, cfg, hid, logits, traces, *_ = _decode_all("fp32")
    for b, s in enumerate(d["seqs"]):
        for li in range(cfg.n_layers):
            r = O.compare(traces[li].resid_out[b], s["layer_out"][li])
            assert r["max_abs"] < 1e-4 and r["cosine"] > 0.99999, (b, li, r)
        r = O.compare(logits[b], s["logits"])
        assert r["max_abs"] < 1e-4, (b, r)


def test_oracle_faithful_within_tolerance_of_hf():
    d, cfg, hid, logits, traces, *_ = _decode_all("faithful")
    for b, s in enumerate(d["seqs"]):
        r = O.compare(traces[-1].resid_out[b], s["layer_out"][-1])
        assert r["max_abs"] < 2e-2 and r["cosine"] > 0.999, (b, r)
        r = O.compare(logits[b], s["logits"])
        assert r["max_abs"] < 2e-2 and r["cosine"] > 0.999, (b, r)


def test_oracle_kv_write_placement():
    """The new token's K/V land at (block_table[b][pos//128], pos%128); nothing else moves."""
    d, cfg, hid, logits, traces, kc, vc, table, positions = _decode_all("fp32")
    for li in range(cfg.n_layers):
        for b, s in enumerate(d["seqs"]):
            P = s["prefix_len"]
            blk, off = int(table[b, P // 128]), P % 128
            torch.testing.assert_close(kc[li][blk, :, off], traces[li].k_new[b].to(kc[li].dtype))
            torch.testing.assert_close(vc[li][blk, :, off], traces[li].v_new[b].to(vc[li].dtype))
            # the prefix stays untouched
            for t in range(P):
                torch.testing.assert_close(kc[li][table[b, t // 128], :, t % 128],
                                           s["keys"][li][:, t])


def test_oracle_moe_block_matches_hf():
    d = load_golden()
    cfg = golden_config(d)
    lw = golden_layers(d, cfg)[0]
    m = d["moe"]
    x = m["x"]
    logits = x @ lw.router.to(torch.float32).t()
    idx, w = O.router_topk(logits, cfg.top_k, "fp32")
    assert torch.equal(torch.sort(idx, -1).values, torch.sort(m["topk_idx"], -1).values)
    # HF orders by probability, the oracle by logit: same order without ties
    assert torch.equal(idx, m["topk_idx"])
    torch.testing.assert_close(w, m["topk_w"].to(torch.float32), rtol=1e-5, atol=1e-6)
    y = O.experts_forward(x, idx, w, lw.gate_up, lw.down, "fp32")
    torch.testing.assert_close(y, m["out"].to(torch.float32), rtol=1e-4, atol=1e-5)


def test_kat_rmsnorm_constant_vector():
    """RMSNorm of a constant vector c is sign(c)*g (known answer)."""
    x = torch.full((2, 512), 3.0).to(torch.bfloat16)
    g = torch.ones(512, dtype=torch.bfloat16)
    y = O.rmsnorm_hidden_faithful(x, g, 1e-6, gamma_first=True)
    torch.testing.assert_close(y, torch.ones(2, 512), rtol=1e-5, atol=1e-5)


def test_kat_rope_identity_at_pos0():
    cos, sin = O.rope_tables(8, 128, 1e6)
    raw = torch.randn(3, 128).to(torch.bfloat16)
    w = torch.ones(128, dtype=torch.bfloat16)
    a = O.head_norm_rope_faithful(raw, w, cos[0], sin[0], 1e-6)
    r = O.rstd_fixed(O.lane_sum_head(raw.float() ** 2), 128, 1e-6)[..., None]
    b = O.rbf(raw.float() * r)
    torch.testing.assert_close(a, b)


def test_kat_topk_ties_lower_index_first():
    logits = torch.tensor([[0.5, 2.0, 2.0, 1.0, 2.0, -1.0, 0.0, 1.0]])
    idx = O.topk_select(logits, 4)
    assert idx.tolist() == [[1, 2, 4, 3]]


def test_kat_one_hot_routing_equals_single_swiglu():
    torch.manual_seed(0)
    E, H, I = 4, 256, 32
    gate_up = (torch.randn(E, 2 * I, H) * 0.05).to(torch.bfloat16)
    down = (torch.randn(E, H, I) * 0.05).to(torch.bfloat16)
    x = torch.randn(1, H)
    idx = torch.tensor([[2, 0]])
    w = torch.tensor([[1.0, 0.0]])
    y = O.experts_forward(x, idx, w, gate_up, down, "fp32")
    gu = gate_up[2].float() @ x[0]
    ref = down[2].float() @ (torch.nn.functional.silu(gu[:I]) * gu[I:])
    torch.testing.assert_close(y[0], ref)


def test_lane_sum_fixed_order_is_a_sum():
    x = torch.randn(4, 2048)
    torch.testing.assert_close(O.lane_sum_hidden(x), x.sum(-1), rtol=1e-5, atol=1e-4)
    y = torch.randn(5, 128)
    torch.testing.assert_close(O.lane_sum_head(y), y.sum(-1), rtol=1e-5, atol=1e-5)
