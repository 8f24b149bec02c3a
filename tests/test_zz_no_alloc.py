"""The allocation-free MoE block (``nkm_qwen3_moe_block_noalloc``) against the handle-based
``nkm_qwen3_moe_block`` on the same inputs, two calls in a row, through the C ABI.

The allocation-free entry point keeps its scratch in a static device array shared by all
calls, so the second call also checks that nothing left from the first call leaks into it.
"""
import ctypes

import pytest
import torch

from oracle import qwen3_moe_oracle as O
from tests.qwen_cases import BF16, gpu_layers, make_layers, qwen_cfg, shape_of, skew_bias

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


def _close(a, b):
    r = O.compare(a.float().cpu(), b.float().cpu())
    assert r["max_abs"] <= ATOL and r["cosine"] >= COS, r


def test_noalloc_moe_block_matches_handle_entry_point():
    from nki_moe_megakernel_b200 import _lib
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    cfg = qwen_cfg(n_layers=2)
    lws = make_layers(cfg, 2, seed=321)
    lws[1].router_bias = skew_bias(cfg)
    gl = [gpu_layers([lws[0]], dev, attention=False)[0],
          gpu_layers([lws[1]], dev, attention=False, router_bias=lws[1].router_bias)[0]]
    eng = Qwen3MoeMegakernel(shape_of(cfg, 2, 0), gl, max_batch=32, num_blocks=0, kv_pools=False)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    # call 1: layer 0, T=32, block output only; call 2: layer 1 (skewed routing), T=5, residual
    for layer, T, residual in ((0, 32, False), (1, 5, True)):
        x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(40 + T)).to(BF16).to(dev)
        want = eng.moe_block(layer, x, residual=residual, trace=True)
        got = torch.empty(T, cfg.hidden, dtype=BF16, device=dev)
        tr = eng._alloc_traces(T, 1)
        step = eng._step_struct(T, x=x, y=got, residual=int(residual), first_layer=layer, num_layers=1, traces=tr)
        status.fill_(-1)
        rc = lib.nkm_qwen3_moe_block_noalloc(ctypes.byref(eng._desc), layer, ctypes.byref(step), status.data_ptr(),
                                             stream.cuda_stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert eng.status() == 0
        _close(got, want["hidden"])
        assert torch.equal(tr["topk_idx"], want["topk_idx"])


def test_noalloc_rejects_oversized_scratch():
    """A description whose scratch exceeds the static array is refused before any launch
    (here a 12000-entry layer table on top of the T=32 MoE buffers)."""
    from nki_moe_megakernel_b200 import _lib
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    dev = torch.device("cuda:0")
    cfg = qwen_cfg(n_layers=1)
    gl = gpu_layers(make_layers(cfg, 1, seed=1), dev, attention=False)
    eng = Qwen3MoeMegakernel(shape_of(cfg, 1, 0), gl, max_batch=32, num_blocks=0, kv_pools=False)
    n = 12000
    table = (_lib.nkm_qwen3_layer * n)(*([gl[0].c_struct()] * n))
    d = _lib.nkm_qwen3_desc.from_buffer_copy(eng._desc)
    d.n_layers = n
    d.layers = ctypes.cast(table, type(d.layers))
    T = 32
    x = torch.zeros(T, cfg.hidden, dtype=BF16, device=dev)
    y = torch.empty_like(x)
    step = eng._step_struct(T, x=x, y=y, first_layer=0, num_layers=1)
    rc = _lib.lib().nkm_qwen3_moe_block_noalloc(ctypes.byref(d), 0, ctypes.byref(step), None,
                                                torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.NKM_ERR_ARG
    assert "scratch" in _lib.last_error()


def test_handles_and_noalloc_with_different_hidden_sizes():
    """The decode kernel's shared-memory limit is a per-process attribute of the kernel.  A
    handle for hidden 2048 keeps working after a handle for hidden 256 is created and after an
    allocation-free call on that smaller model (neither lowers the limit under the larger
    handle's launches), and the small model's two entry points agree."""
    from nki_moe_megakernel_b200 import _lib
    from nki_moe_megakernel_b200.engine import Qwen3MoeMegakernel

    dev = torch.device("cuda:0")
    big = qwen_cfg(n_layers=1)
    small = qwen_cfg(n_layers=1, hidden=256, n_experts=16, top_k=4, moe_inter=128)
    eb = Qwen3MoeMegakernel(shape_of(big, 1, 0), gpu_layers(make_layers(big, 1, seed=7), dev, attention=False),
                            max_batch=8, num_blocks=0, kv_pools=False)
    es = Qwen3MoeMegakernel(shape_of(small, 1, 0), gpu_layers(make_layers(small, 1, seed=8), dev, attention=False),
                            max_batch=8, num_blocks=0, kv_pools=False)
    xb = torch.randn(8, big.hidden, generator=torch.Generator().manual_seed(9)).to(BF16).to(dev)
    xs = torch.randn(8, small.hidden, generator=torch.Generator().manual_seed(10)).to(BF16).to(dev)
    want_b = eb.moe_block(0, xb)["hidden"]
    assert eb.status() == 0
    want_s = es.moe_block(0, xs)["hidden"]
    assert es.status() == 0
    got_s = torch.empty_like(xs)
    step = es._step_struct(8, x=xs, y=got_s, residual=0, first_layer=0, num_layers=1)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    rc = _lib.lib().nkm_qwen3_moe_block_noalloc(ctypes.byref(es._desc), 0, ctypes.byref(step), status.data_ptr(),
                                                torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _close(got_s, want_s)
    again = eb.moe_block(0, xb)["hidden"]
    assert eb.status() == 0
    assert torch.equal(again, want_b)
