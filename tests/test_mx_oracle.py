"""The oracle's OCP MX (MXFP8) quantiser used for the MXFP8 expert weights: known answers."""
import torch

from oracle import qwen3_moe_oracle as O


def test_mxfp8_known_answers():
    w = torch.zeros(3, 32)
    w[0, 0], w[0, 1], w[0, 2] = 1.0, -0.5, 0.25          # amax 1: scale 2^-8 (byte 119), codes exact
    w[1, :] = torch.linspace(-3.0, 3.0, 32)               # amax 3: scale 2^(1-8)
    codes, scales = O.mxfp8_quantize(w)
    assert scales.flatten().tolist() == [119, 120, 0]               # all-zero block: smallest scale
    d = O.mxfp8_dequant(codes, scales)
    assert d[0, :3].tolist() == [1.0, -0.5, 0.25] and torch.equal(d[0, 3:], torch.zeros(29))
    assert d[1].abs().max().item() == 3.0                 # 3 / 2^-7 = 384 is an e4m3 value
    assert torch.equal(d[2], torch.zeros(32))
    # values between e4m3 neighbours round to nearest (even); the largest code saturates at 448
    x = torch.tensor([1.0] + [0.0] * 31)
    x[1] = 1.0 + 1.0 / 16                                 # 272 after scaling: halfway 256 / 288 -> 256 (even)
    c, s = O.mxfp8_quantize(x[None])
    assert O.mxfp8_dequant(c, s)[0, 1].item() == 1.0
    y = torch.tensor([[1.9] + [0.0] * 31])                # 1.9 / 2^-8 = 486.4 > 448: saturates
    c, s = O.mxfp8_quantize(y)
    assert O.mxfp8_dequant(c, s)[0, 0].item() == 448.0 * 2.0 ** -8


def test_mxfp8_error_bound():
    w = torch.randn(8, 256, generator=torch.Generator().manual_seed(3)) * 0.02
    c, s = O.mxfp8_quantize(w)
    d = O.mxfp8_dequant(c, s)
    # every value within an eighth of its block's largest magnitude (e4m3 steps near the top)
    blk = w.reshape(8, 8, 32).abs().amax(-1, keepdim=True)
    assert ((d - w).reshape(8, 8, 32).abs() <= blk * 2.0 ** -3).all()
    assert torch.equal(d.to(torch.bfloat16).float(), d)   # exact in bf16 (the GEMM's operand type)
