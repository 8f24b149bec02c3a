"""CPU checks of the sampler oracle (``oracle/sampling_oracle.py``) and of the sampler's host
entry points (no GPU needed)."""
import ctypes

import torch

from oracle import sampling_oracle as S


def test_splitmix64_known_answer():
    # first output of the SplitMix64 generator seeded with 0 (the published reference sequence)
    assert S.splitmix64(0) == 0xE220A8397B1DCDAF


def test_greedy_is_first_argmax_and_signed_zero_is_one_value():
    g = torch.Generator().manual_seed(0)
    l = torch.randn(1000, generator=g)
    l[[17, 400]] = l.max() + 1.0
    assert S.sample_row(l, 1, 1.0, 1.0, 0, 0, 0)[0] == 17
    z = -torch.rand(50, generator=g) - 0.1
    z[9], z[4] = 0.0, -0.0
    assert S.sample_row(z, 1, 1.0, 1.0, 0, 0, 0)[0] == 4


def test_topk_topp_semantics():
    l = torch.full((100,), -10.0)
    l[[3, 50, 7, 90]] = torch.tensor([4.0, 3.0, 2.0, 1.0])
    assert S.topk_ids(l, 4).tolist() == [3, 50, 7, 90]
    # top_p tiny: only the most likely token survives, whatever the draw
    for seed in range(20):
        assert S.sample_row(l, 4, 1e-6, 1.0, seed, 5, 0)[0] == 3
    # every draw lands in the top-k
    for seed in range(50):
        assert S.sample_row(l, 3, 1.0, 2.0, seed, 9, 1)[0] in (3, 50, 7)


def test_sample_workspace_bytes_host_checks():
    from nki_moe_megakernel_b200 import _lib
    from nki_moe_megakernel_b200.build import build_library

    build_library()
    lib = _lib.lib()
    assert lib.nkm_sample_workspace_bytes(8, 151936, 64) > 0
    assert lib.nkm_sample_workspace_bytes(8, 151936, 65) == 0
    assert lib.nkm_sample_workspace_bytes(0, 151936, 1) == 0
    p = _lib.nkm_sample_params(0, 1.0, 1.0, 0)
    assert lib.nkm_sample_logits(16, 8, 100, ctypes.byref(p), None, 16, 16, 1 << 20, None) == _lib.NKM_ERR_ARG
    assert "top_k" in _lib.last_error()
