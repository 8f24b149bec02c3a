"""On-device token sampling (``nkm_sample_logits``) against the CPU sampler oracle.

* greedy (top_k = 1): the token is the first maximum of the row, bit-exact, with equal maxima
  and signed zeros planted;
* top-k / temperature / top-p draws at the Qwen3 vocabulary (151936): the token equals the
  oracle's unless the draw sits within 1e-5 (relative) of a CDF boundary or the top-p test
  within 1e-5 of top_p, where fp32 rounding of the softmax may decide (counted, must be rare);
* the draws follow the distribution: 32 rows x 64 seeds of one 4-token distribution, every
  frequency within 5 standard deviations of its probability.
"""
import pytest
import torch

from oracle import sampling_oracle as S

pytestmark = pytest.mark.gpu

V = 151936


@pytest.fixture(scope="module")
def sampler():
    from nki_moe_megakernel_b200.engine import sample_tokens

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sample_tokens


def _logits(B, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, V, generator=g) * 3.0


def test_greedy_first_maximum(sampler):
    B = 8
    l = _logits(B, 1)
    l[0, [1000, 20]] = 50.0             # equal maxima: the lower id wins
    l[1] = -torch.rand(V) - 1.0
    l[1, 77], l[1, 12] = 0.0, -0.0       # +0 and -0 are one value
    l[2, V - 1] = 60.0                   # last entry of the row
    pos = torch.arange(B, dtype=torch.int32)
    got = sampler(l.cuda(), pos.cuda(), top_k=1).cpu()
    want = [S.sample_row(l[b], 1, 1.0, 1.0, 0, b, b)[0] for b in range(B)]
    assert got.tolist() == want
    assert want[0] == 20 and want[1] == 12 and want[2] == V - 1


@pytest.mark.parametrize("top_k,top_p,temp,B", [(50, 0.9, 0.7, 8), (64, 1.0, 1.0, 4), (8, 0.5, 1.3, 32),
                                                (2, 1.0, 0.5, 1)])
def test_sampled_tokens_match_oracle(sampler, top_k, top_p, temp, B):
    close = 0
    for seed in range(3):
        l = _logits(B, 100 + seed)
        pos = torch.randint(0, 4096, (B,), generator=torch.Generator().manual_seed(seed), dtype=torch.int32)
        got = sampler(l.cuda(), pos.cuda(), top_k=top_k, top_p=top_p, temperature=temp, seed=seed).cpu().tolist()
        for b in range(B):
            tok, margin = S.sample_row(l[b], top_k, top_p, temp, seed, int(pos[b]), b)
            if got[b] != tok:
                assert margin < 1e-5, (seed, b, got[b], tok, margin)
                close += 1
            assert got[b] in S.topk_ids(l[b], top_k).tolist()
    assert close <= 1, close


def test_draw_frequencies(sampler):
    B, seeds = 32, 64
    p = torch.tensor([0.4, 0.3, 0.2, 0.1])
    l = torch.full((B, V), -30.0)
    ids = [5, 70000, 123, V - 2]
    l[:, ids] = p.log()
    counts = torch.zeros(4)
    for seed in range(seeds):
        got = sampler(l.cuda(), None, top_k=4, top_p=1.0, temperature=1.0, seed=seed).cpu().tolist()
        for t in got:
            counts[ids.index(t)] += 1
    n = B * seeds
    sd = (n * p * (1 - p)).sqrt()
    assert ((counts - n * p).abs() <= 5 * sd).all(), (counts, n * p)
