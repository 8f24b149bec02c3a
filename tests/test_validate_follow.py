"""Host logic of ``main.py --mode validate``: the fp32 Hugging Face baseline follows the
megakernel's expert set only at router near ties (``_FollowNearTies``), on tiny CPU models."""
import pytest
import torch

pytestmark = pytest.mark.filterwarnings("ignore")


def _qwen():
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    c = Qwen3MoeConfig(vocab_size=64, hidden_size=64, intermediate_size=64, moe_intermediate_size=32,
                       num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                       num_experts=8, num_experts_per_tok=2, norm_topk_prob=True, max_position_embeddings=64)
    torch.manual_seed(0)
    m = Qwen3MoeForCausalLM(c).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.5)
    return m


def _gptoss():
    from transformers import GptOssConfig, GptOssForCausalLM

    c = GptOssConfig(vocab_size=64, hidden_size=64, intermediate_size=32, num_hidden_layers=2,
                     num_attention_heads=2, num_key_value_heads=1, head_dim=32, num_local_experts=8,
                     num_experts_per_tok=2, sliding_window=4, max_position_embeddings=64,
                     layer_types=["sliding_attention", "full_attention"])
    c._attn_implementation = "eager"
    torch.manual_seed(0)
    m = GptOssForCausalLM(c).eval()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.5)
    return m


def _own_routing(m, ids):
    """The baseline's own top-k per token and layer, and its raw router logits."""
    from nki_moe_megakernel_b200.main import _FollowNearTies

    routers = [x for x in m.modules() if type(x).__name__ in _FollowNearTies.NAMES]
    got = {}
    hooks = [r.register_forward_hook(lambda mod, inp, out, li=li: got.__setitem__(li, (inp[0], out[2])))
             for li, r in enumerate(routers)]
    with torch.no_grad():
        m(ids)
    for h in hooks:
        h.remove()
    idx = torch.stack([got[li][1] for li in range(len(routers))], 1)  # [T, L, k]
    raw = []
    for li, r in enumerate(routers):
        h = got[li][0].reshape(-1, r.hidden_dim)
        raw.append(torch.nn.functional.linear(h, r.weight, getattr(r, "bias", None)))
    return idx, torch.stack(raw, 1)  # [T, L, E]


@pytest.mark.parametrize("make", [_qwen, _gptoss])
def test_follows_only_near_ties(make):
    from nki_moe_megakernel_b200.main import _FollowNearTies

    m = make()
    ids = torch.randint(0, 64, (1, 12), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        base = m(ids).logits[0]
    idx, raw = _own_routing(m, ids)
    # the baseline's own choice: nothing to follow, nothing changes
    with torch.no_grad(), _FollowNearTies(m, idx, 0.02) as f:
        same = m(ids).logits[0]
    assert f.followed == 0 and torch.equal(same, base)
    # token 5, layer 0: swap the k-th choice for the best expert left out
    t, li = 5, 0
    order = torch.sort(raw[t, li], descending=True).indices
    k = idx.shape[-1]
    hint = idx.clone()
    hint[t, li] = torch.cat([order[:k - 1], order[k:k + 1]])
    gap = float(raw[t, li, order[k - 1]] - raw[t, li, order[k]])
    with torch.no_grad(), _FollowNearTies(m, hint, gap / 2) as f:
        out = m(ids).logits[0]
    assert f.followed == 0 and torch.equal(out, base)          # beyond the tolerance: left alone
    with torch.no_grad(), _FollowNearTies(m, hint, gap * 2) as f:
        out = m(ids).logits[0]
    # within it: taken (a later layer of token t may then follow its old set too, also within it)
    assert f.followed >= 1 and gap - 1e-5 <= f.max_gap <= 2 * gap
    # earlier tokens only see the batching of the experts change (rounding); token t changes
    assert torch.allclose(out[:t], base[:t], atol=1e-4) and (out[t] - base[t]).abs().max() > 1e-3
    # the wrapper is removed on exit
    with torch.no_grad():
        assert torch.equal(m(ids).logits[0], base)
