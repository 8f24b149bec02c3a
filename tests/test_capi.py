"""C ABI checks that need no GPU: the library loads, exports every function declared in
include/nkimoe.h, the ctypes structs match the C layout, and host-side argument checks
reject bad descriptions before touching the device."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nkimoe.h")


@pytest.fixture(scope="module")
def L():
    from nki_moe_megakernel_b200.build import build_library
    from nki_moe_megakernel_b200 import _lib

    build_library()
    return _lib


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nkm_\w+)\s*\(", src)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("nkm_qwen3_create", "nkm_qwen3_decode_step", "nkm_qwen3_moe_block", "nkm_qwen3_attention_block",
              "nkm_pack_ft", "nkm_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(L):
    lib = L.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (nkm_\w+)", out.stdout))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():
        assert hasattr(lib, n)
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"


def test_version_string(L):
    assert b"sm_100a" in L.lib().nkm_version()


def test_ctypes_structs_match_c_layout(L):
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "nkimoe.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("nkm_qwen3_layer %zu\n", sizeof(nkm_qwen3_layer));
  printf("nkm_qwen3_desc %zu\n", sizeof(nkm_qwen3_desc));
  printf("nkm_qwen3_step %zu\n", sizeof(nkm_qwen3_step));
  P(nkm_qwen3_desc, layers) P(nkm_qwen3_desc, rope_max_pos) P(nkm_qwen3_desc, max_batch)
  P(nkm_qwen3_desc, n_ranks) P(nkm_qwen3_desc, n_local_experts) P(nkm_qwen3_desc, xchg)
  P(nkm_qwen3_step, max_blocks_per_seq) P(nkm_qwen3_step, trace_resid_out) P(nkm_qwen3_step, trace_stage_ns) P(nkm_qwen3_layer, router_bias)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(line.rsplit(" ", 1) for line in out if line)
    assert int(got["nkm_qwen3_layer"]) == ctypes.sizeof(L.nkm_qwen3_layer)
    assert int(got["nkm_qwen3_desc"]) == ctypes.sizeof(L.nkm_qwen3_desc)
    assert int(got["nkm_qwen3_step"]) == ctypes.sizeof(L.nkm_qwen3_step)
    assert int(got["nkm_qwen3_desc.layers"]) == L.nkm_qwen3_desc.layers.offset
    assert int(got["nkm_qwen3_desc.rope_max_pos"]) == L.nkm_qwen3_desc.rope_max_pos.offset
    assert int(got["nkm_qwen3_desc.max_batch"]) == L.nkm_qwen3_desc.max_batch.offset
    assert int(got["nkm_qwen3_desc.n_ranks"]) == L.nkm_qwen3_desc.n_ranks.offset
    assert int(got["nkm_qwen3_desc.n_local_experts"]) == L.nkm_qwen3_desc.n_local_experts.offset
    assert int(got["nkm_qwen3_desc.xchg"]) == L.nkm_qwen3_desc.xchg.offset
    assert int(got["nkm_qwen3_step.max_blocks_per_seq"]) == L.nkm_qwen3_step.max_blocks_per_seq.offset
    assert int(got["nkm_qwen3_step.trace_resid_out"]) == L.nkm_qwen3_step.trace_resid_out.offset
    assert int(got["nkm_qwen3_step.trace_stage_ns"]) == L.nkm_qwen3_step.trace_stage_ns.offset
    assert int(got["nkm_qwen3_layer.router_bias"]) == L.nkm_qwen3_layer.router_bias.offset


def _desc(L, **kw):
    layer = (L.nkm_qwen3_layer * 1)()
    base = dict(hidden=2048, n_q_heads=32, n_kv_heads=4, head_dim=128, n_experts=128, top_k=8, moe_inter=768,
                n_layers=1, vocab=0, rms_eps=1e-6, max_batch=8, block_size=128, num_blocks=0)
    base.update(kw)
    d = L.nkm_qwen3_desc()
    for k, v in base.items():
        setattr(d, k, v)
    d.layers = layer
    return d, layer


@pytest.mark.parametrize("bad", [dict(head_dim=64), dict(hidden=2000), dict(hidden=4096), dict(top_k=9), dict(max_batch=64),
                                 dict(n_q_heads=30), dict(moe_inter=100), dict(block_size=64),
                                 dict(n_experts=300), dict(vocab=100)])
def test_create_rejects_bad_descriptions(L, bad):
    d, _keep = _desc(L, **bad)
    h = ctypes.c_void_p()
    rc = L.lib().nkm_qwen3_create(ctypes.byref(d), None, 0, ctypes.byref(h))
    assert rc == L.NKM_ERR_ARG
    assert L.last_error()
    assert not h.value


def test_pack_rejects_bad_shapes(L):
    f = L.lib().nkm_pack_ft
    assert f(None, None, 16, 32, 1, 0, None) == L.NKM_ERR_ARG
    assert f(16, 16, 15, 32, 1, 0, None) == L.NKM_ERR_ARG
    assert f(16, 16, 16, 30, 1, 0, None) == L.NKM_ERR_ARG
    assert f(16, 16, 16, 32, 1, 7, None) == L.NKM_ERR_ARG


def test_gptoss_structs_match_c_layout(L):
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "nkimoe.h"
int main(void) {
  printf("layer %zu\n", sizeof(nkm_gptoss_layer));
  printf("desc %zu\n", sizeof(nkm_gptoss_desc));
  printf("step %zu\n", sizeof(nkm_gptoss_step));
  printf("sample %zu\n", sizeof(nkm_sample_params));
  printf("desc.layers %zu\n", offsetof(nkm_gptoss_desc, layers));
  printf("desc.max_context %zu\n", offsetof(nkm_gptoss_desc, max_context));
  printf("desc.n_ranks %zu\n", offsetof(nkm_gptoss_desc, n_ranks));
  printf("desc.xchg %zu\n", offsetof(nkm_gptoss_desc, xchg));
  printf("step.trace_topk_w %zu\n", offsetof(nkm_gptoss_step, trace_topk_w));
  printf("layer.sliding %zu\n", offsetof(nkm_gptoss_layer, sliding));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(line.rsplit(" ", 1) for line in out if line)
    assert int(got["layer"]) == ctypes.sizeof(L.nkm_gptoss_layer)
    assert int(got["desc"]) == ctypes.sizeof(L.nkm_gptoss_desc)
    assert int(got["step"]) == ctypes.sizeof(L.nkm_gptoss_step)
    assert int(got["sample"]) == ctypes.sizeof(L.nkm_sample_params)
    assert int(got["desc.layers"]) == L.nkm_gptoss_desc.layers.offset
    assert int(got["desc.max_context"]) == L.nkm_gptoss_desc.max_context.offset
    assert int(got["desc.n_ranks"]) == L.nkm_gptoss_desc.n_ranks.offset
    assert int(got["desc.xchg"]) == L.nkm_gptoss_desc.xchg.offset
    assert int(got["step.trace_topk_w"]) == L.nkm_gptoss_step.trace_topk_w.offset
    assert int(got["layer.sliding"]) == L.nkm_gptoss_layer.sliding.offset


def test_gptoss_create_rejects_bad_descriptions(L):
    for bad in (dict(head_dim=128), dict(hidden=2000), dict(max_batch=17), dict(top_k=9), dict(inter=100),
                dict(n_ranks=9), dict(n_ranks=2, rank=0, n_local_experts=16),  # no exchange regions
                dict(expert_begin=4), dict(n_ranks=2, rank=2)):
        base = dict(hidden=2880, hidden_actual=0, n_q_heads=64, n_kv_heads=8, head_dim=64, n_experts=32, top_k=4,
                    inter=2880, n_layers=1, vocab=0, rms_eps=1e-5, swiglu_limit=7.0, swiglu_alpha=1.702,
                    sliding_window=128, block_size=128, max_batch=16, max_context=4096)
        base.update(bad)
        d = L.nkm_gptoss_desc()
        for k, v in base.items():
            setattr(d, k, v)
        layer = (L.nkm_gptoss_layer * 1)()
        d.layers = layer
        h = ctypes.c_void_p()
        assert L.lib().nkm_gptoss_create(ctypes.byref(d), None, 0, ctypes.byref(h)) == L.NKM_ERR_ARG, bad
        assert L.lib().nkm_gptoss_workspace_bytes(ctypes.byref(d)) == 0


@pytest.mark.parametrize("world", [1, 2, 8])
def test_xchg_bytes_match_host_sizing(L, world):
    """The exchange region the host allocates (``sharding.xchg_bytes``) is the size the library
    asks for: header, partials and (several ranks) the vocabulary-sharded LM head's logits."""
    from nki_moe_megakernel_b200.sharding import xchg_bytes

    H, B, V = 2048, 8, 151936
    d, _keep = _desc(L, vocab=V, max_batch=B, n_q_heads=32 // world, n_kv_heads=max(1, 4 // world))
    d.n_ranks, d.rank = world, world - 1
    d.expert_begin, d.n_local_experts = 128 // world * (world - 1), 128 // world
    if world > 1:
        for q in range(world):
            d.xchg[q] = 256 * (q + 1)  # only validated for alignment, never dereferenced here
    need = L.lib().nkm_qwen3_xchg_bytes(ctypes.byref(d))
    assert need == xchg_bytes(H, B, world, V)
    if world > 1:
        assert need >= B * V * 4 + 2 * world * B * H * 4


@pytest.mark.parametrize("world", [1, 2, 8])
def test_gptoss_xchg_bytes_match_host_sizing(L, world):
    """GPT-OSS: the host's exchange-region size (``sharding.gptoss_xchg_bytes``) is the library's."""
    from nki_moe_megakernel_b200.sharding import gptoss_xchg_bytes

    H, B, V = 2880, 16, 201088
    base = dict(hidden=H, hidden_actual=0, n_q_heads=64 // world, n_kv_heads=8 // world, head_dim=64, n_experts=32,
                top_k=4, inter=2880, n_layers=1, vocab=V, rms_eps=1e-5, swiglu_limit=7.0, swiglu_alpha=1.702,
                sliding_window=128, block_size=128, max_batch=B, max_context=4096, n_ranks=world, rank=world - 1,
                expert_begin=32 // world * (world - 1), n_local_experts=32 // world)
    d = L.nkm_gptoss_desc()
    for k, v in base.items():
        setattr(d, k, v)
    layer = (L.nkm_gptoss_layer * 1)()
    d.layers = layer
    if world > 1:
        for q in range(world):
            d.xchg[q] = 256 * (q + 1)  # only validated for alignment, never dereferenced here
    need = L.lib().nkm_gptoss_xchg_bytes(ctypes.byref(d))
    assert need == gptoss_xchg_bytes(H, B, world, V)
    if world > 1:
        assert need >= 2 * B * V * 8 + 4 * world * B * H * 8
