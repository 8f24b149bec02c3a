"""Host-side owner of a GPT-OSS decode megakernel instance (``nkm_gptoss_*`` in ``libnkimoe.so``).

Holds the weights in the kernel layouts (bf16 fragment-tiled attention and LM head, MXFP4
experts packed by ``nkm_pack_mxfp4``), the paged K/V pools (V blocks stored transposed), the
YaRN RoPE tables and the workspace.  torch is used for device memory only; every decode step is
one launch of the library's kernel.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import torch

from . import _lib
from ._lib import check, lib
from .engine import pack_ft

BF16 = torch.bfloat16


@dataclass
class GptOssShape:
    """Model dimensions (Hugging Face ``GptOssConfig`` names in comments); defaults GPT-OSS-20B."""

    hidden_size: int = 2880
    hidden_actual: int = 0          # RMSNorm mean over this many elements (0: hidden_size)
    num_attention_heads: int = 64
    num_key_value_heads: int = 8
    head_dim: int = 64
    num_local_experts: int = 32
    num_experts_per_tok: int = 4
    intermediate_size: int = 2880
    num_hidden_layers: int = 24
    vocab_size: int = 201088
    rms_norm_eps: float = 1e-5
    sliding_window: int = 128
    rope_theta: float = 150000.0
    rope_factor: float = 32.0
    rope_original_max: int = 4096
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    block_size: int = 128

    def is_sliding(self, layer: int) -> bool:
        """Even layers use the sliding window (``layer_types`` of the checkpoint)."""
        return layer % 2 == 0


def yarn_tables(shape: GptOssShape, max_pos: int, device) -> tuple:
    """fp32 cos/sin ``[max_pos, head_dim/2]``: YaRN inverse frequencies (Peng et al. 2023; the
    formula of Hugging Face's ``_compute_yarn_parameters`` without truncation of the correction
    range) times the attention factor ``0.1 ln(factor) + 1``."""
    dim, base, factor = shape.head_dim, shape.rope_theta, shape.rope_factor

    def corr(rot):
        return (dim * math.log(shape.rope_original_max / (rot * 2 * math.pi))) / (2 * math.log(base))

    low, high = max(corr(shape.rope_beta_fast), 0), min(corr(shape.rope_beta_slow), dim - 1)
    if low == high:
        high += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low), 0, 1)
    pos_freqs = base ** (torch.arange(0, dim, 2).to(torch.float32) / dim)
    inv = (1.0 / (factor * pos_freqs)) * ramp + (1.0 / pos_freqs) * (1 - ramp)
    af = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
    f = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    return (f.cos() * af).contiguous().to(device), (f.sin() * af).contiguous().to(device)


def pack_mxfp4(codes: torch.Tensor, scales: torch.Tensor, stream=None):
    """Tile MXFP4 codes ``[..., R, K]`` (uint8 0..15) and e8m0 scales ``[..., R, K/32]`` (CUDA) for
    the kernel (``nkm_pack_mxfp4``).  Returns (weights uint8, scales uint8)."""
    assert codes.is_cuda and codes.dtype == torch.uint8 and scales.dtype == torch.uint8
    codes, scales = codes.contiguous(), scales.contiguous()
    R, K = codes.shape[-2], codes.shape[-1]
    count = codes.numel() // (R * K)
    w = torch.empty(codes.numel() // 2, dtype=torch.uint8, device=codes.device)
    s = torch.empty(lib().nkm_mxfp4_scale_bytes(R, K, count), dtype=torch.uint8, device=codes.device)
    st = stream if stream is not None else torch.cuda.current_stream(codes.device)
    check(lib().nkm_pack_mxfp4(codes.data_ptr(), scales.data_ptr(), w.data_ptr(), s.data_ptr(), R, K, count,
                               st.cuda_stream), "nkm_pack_mxfp4")
    return w, s


class GptOssGpuLayer:
    """One GPT-OSS decoder layer in the kernel layouts (device tensors).  Attention weights in
    Hugging Face layout (q/k/v_proj ``[heads*64, H]``, o_proj ``[H, nq*64]``); experts as MXFP4
    codes/scales of gate/up ``[E, 2I, H]`` (rows interleaved gate, up) and down ``[E, H, I]``."""

    def __init__(self, t: Dict[str, torch.Tensor], sliding: bool):
        self.wqkv_ft = pack_ft(torch.cat([t["wq"], t["wk"], t["wv"]], 0).to(BF16))
        self.bqkv = torch.cat([t["bq"], t["bk"], t["bv"]]).to(BF16).contiguous()
        self.wo_ft = pack_ft(t["wo"].to(BF16))
        self.bo = t["bo"].to(BF16).contiguous()
        self.sinks = t["sinks"].to(BF16).contiguous()
        self.ln1 = t["ln1"].to(BF16).contiguous()
        self.ln2 = t["ln2"].to(BF16).contiguous()
        self.router = t["router"].to(BF16).contiguous()
        self.router_b = t["router_b"].to(BF16).contiguous()
        self.w13, self.s13 = pack_mxfp4(t["gu_codes"], t["gu_scales"])
        self.b13 = t["gu_b"].to(BF16).contiguous()
        self.w2, self.s2 = pack_mxfp4(t["dn_codes"], t["dn_scales"])
        self.b2 = t["dn_b"].to(BF16).contiguous()
        self.sliding = bool(sliding)

    def c_struct(self) -> "_lib.nkm_gptoss_layer":
        p = lambda x: x.data_ptr()  # noqa: E731
        return _lib.nkm_gptoss_layer(p(self.wqkv_ft), p(self.bqkv), p(self.wo_ft), p(self.bo), p(self.sinks),
                                     p(self.ln1), p(self.ln2), p(self.router), p(self.router_b), p(self.w13),
                                     p(self.s13), p(self.b13), p(self.w2), p(self.s2), p(self.b2), int(self.sliding))


class GptOssMegakernel:
    """A GPT-OSS decode-megakernel instance on one GPU.  ``layers`` may repeat the same layer
    object (shared weights); each layer still has its own K/V pages."""

    def __init__(self, shape: GptOssShape, layers: Sequence[GptOssGpuLayer], *, max_batch: int, num_blocks: int,
                 max_context: int, final_norm: Optional[torch.Tensor] = None, lm_head: Optional[torch.Tensor] = None,
                 embed: Optional[torch.Tensor] = None, device=None, kv_fp8: bool = False, k_scale: float = 1.0,
                 v_scale: float = 1.0, shard=None, xchg=None):
        """``kv_fp8``: the K/V pools hold e4m3 bytes (``uint8``): stored = e4m3(clip(x * scale,
        +-240)), read = stored / scale.  ``shard`` (``sharding.RankShard``) and ``xchg``
        (``sharding.XchgRegion`` of ``sharding.gptoss_xchg_bytes``) make this instance one rank of
        a tensor + expert parallel group: ``shape`` then carries the rank's head counts and
        ``layers`` its heads and experts (``sharding.shard_gptoss_layer``), while
        ``num_local_experts`` stays the model's expert count."""
        self.shape = shape
        self.device = torch.device(device if device is not None else "cuda")
        self.layers = list(layers)
        L, nkv, D = shape.num_hidden_layers, shape.num_key_value_heads, shape.head_dim
        assert len(self.layers) == L
        self.max_batch, self.num_blocks, self.max_context = max_batch, num_blocks, max_context
        pool_dtype = torch.uint8 if kv_fp8 else BF16
        self.kv_fp8, self.k_scale, self.v_scale = kv_fp8, k_scale, v_scale
        self.k_pool = torch.zeros(L, num_blocks, nkv, shape.block_size, D, dtype=pool_dtype, device=self.device)
        self.v_pool = torch.zeros(L, num_blocks, nkv, D, shape.block_size, dtype=pool_dtype, device=self.device)
        self.rope_max = max_context + shape.block_size
        self.rope_cos, self.rope_sin = yarn_tables(shape, self.rope_max, self.device)
        self.final_norm = None if final_norm is None else final_norm.to(BF16).contiguous()
        self.lm_head_ft = None if lm_head is None else pack_ft(lm_head.to(BF16))
        self.embed = None if embed is None else embed.to(BF16).contiguous()
        self._structs = (_lib.nkm_gptoss_layer * L)(*[l.c_struct() for l in self.layers])
        vocab = shape.vocab_size if (lm_head is not None or embed is not None) else 0
        ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
        self._desc = _lib.nkm_gptoss_desc(
            shape.hidden_size, shape.hidden_actual, shape.num_attention_heads, nkv, D, shape.num_local_experts,
            shape.num_experts_per_tok, shape.intermediate_size, L, vocab, shape.rms_norm_eps, shape.swiglu_limit,
            shape.swiglu_alpha, shape.sliding_window, self._structs, ptr(self.final_norm), ptr(self.lm_head_ft),
            ptr(self.embed), ctypes.cast(self.rope_cos.data_ptr(), ctypes.POINTER(ctypes.c_float)),
            ctypes.cast(self.rope_sin.data_ptr(), ctypes.POINTER(ctypes.c_float)), self.rope_max,
            self.k_pool.data_ptr(), self.v_pool.data_ptr(), num_blocks, shape.block_size, max_batch, max_context,
            int(kv_fp8), k_scale, v_scale)
        self.shard = shard
        if shard is not None and shard.world > 1:
            if xchg is None:
                raise ValueError("a rank of a parallel group needs its exchange region")
            self._desc.n_ranks, self._desc.rank = shard.world, shard.rank
            self._desc.expert_begin, self._desc.n_local_experts = shard.expert_begin, shard.n_local_experts
            for q, ptr_q in enumerate(xchg.ptrs):
                self._desc.xchg[q] = ptr_q
            need = lib().nkm_gptoss_xchg_bytes(ctypes.byref(self._desc))
            if need == 0 or need > xchg.nbytes:
                raise _lib.NkmError(_lib.NKM_ERR_ARG, f"exchange region of {xchg.nbytes} bytes, need {need}")
        else:
            self._desc.n_ranks, self._desc.n_local_experts = 1, shape.num_local_experts
        nbytes = lib().nkm_gptoss_workspace_bytes(ctypes.byref(self._desc))
        if nbytes == 0:
            raise _lib.NkmError(_lib.NKM_ERR_ARG, "nkm_gptoss_workspace_bytes")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        h = ctypes.c_void_p()
        check(lib().nkm_gptoss_create(ctypes.byref(self._desc), self.workspace.data_ptr(), nbytes, ctypes.byref(h)),
              "nkm_gptoss_create")
        self._h = h

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib().nkm_gptoss_destroy(h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode_step(self, positions: torch.Tensor, block_table: torch.Tensor, *, x: Optional[torch.Tensor] = None,
                    input_ids: Optional[torch.Tensor] = None, want_logits: bool = True, trace: bool = False,
                    first_layer: int = 0, num_layers: int = 0, out: Optional[Dict[str, torch.Tensor]] = None,
                    stage_times: bool = False, stream=None) -> Dict[str, torch.Tensor]:
        """One decode step; ``stage_times`` adds ``stage_ns`` (globaltimer of CTA 0 at kernel start,
        after every grid barrier: the input copy, then ten per layer, and at the end)."""
        s, dev = self.shape, self.device
        B = int(positions.shape[0])
        nl = num_layers or (s.num_hidden_layers - first_layer)
        res = out if out is not None else {}
        if "hidden" not in res:
            res["hidden"] = torch.empty(B, s.hidden_size, dtype=BF16, device=dev)
        if want_logits and self.lm_head_ft is not None and "logits" not in res:
            res["logits"] = torch.empty(B, s.vocab_size, dtype=torch.float32, device=dev)
        tr = {}
        if trace:
            R = (s.num_attention_heads + 2 * s.num_key_value_heads) * s.head_dim
            K, E, H = s.num_experts_per_tok, s.num_local_experts, s.hidden_size
            tr = {"qkv": torch.zeros(nl, B, R, device=dev), "resid_mid": torch.zeros(nl, B, H, device=dev),
                  "resid_out": torch.zeros(nl, B, H, device=dev), "router_logits": torch.zeros(nl, B, E, device=dev),
                  "topk_idx": torch.full((nl, B, K), -1, dtype=torch.int32, device=dev),
                  "topk_w": torch.zeros(nl, B, K, device=dev)}
        if stage_times:
            tr["stage_ns"] = torch.zeros(3 + 10 * nl, dtype=torch.int64, device=dev)
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        st = _lib.nkm_gptoss_step(B, p(input_ids), p(x), p(positions), p(block_table), int(block_table.shape[1]),
                                  p(res["hidden"]), p(res.get("logits")) if want_logits else None, first_layer, nl,
                                  p(tr.get("qkv")), p(tr.get("resid_mid")), p(tr.get("resid_out")),
                                  p(tr.get("router_logits")), p(tr.get("topk_idx")), p(tr.get("topk_w")),
                                  p(tr.get("stage_ns")))
        strm = stream if stream is not None else torch.cuda.current_stream(dev)
        check(lib().nkm_gptoss_decode_step(self._h, ctypes.byref(st), strm.cuda_stream), "nkm_gptoss_decode_step")
        res.update(tr)
        return res

    def status(self, stream=None) -> int:
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return lib().nkm_gptoss_status(self._h, s.cuda_stream)

    def check_status(self, stream=None) -> None:
        st = self.status(stream)
        if st != 0:
            raise _lib.NkmError(st, "GPT-OSS decode kernel")
