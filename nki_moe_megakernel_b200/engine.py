"""Host-side owner of a Qwen3-MoE decode megakernel instance.

Holds the weights (converted once to the GPU layouts), the paged K/V pools, the RoPE tables
and the workspace, and calls the C ABI (``libnkimoe.so``) for each decode step.  torch is
used for device memory and streams only; all compute of the step runs in the library's
kernels.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib
from ._lib import check, lib

BF16 = torch.bfloat16


@dataclass
class Qwen3MoeShape:
    """Model dimensions (Hugging Face ``Qwen3MoeConfig`` names) as held by one GPU."""

    hidden_size: int = 2048
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    num_hidden_layers: int = 48
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 128


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def pack_ft(src: torch.Tensor, mode: int = _lib.NKM_PACK_PLAIN, stream=None) -> torch.Tensor:
    """Convert row-major bf16 ``[..., R, K]`` (CUDA) to the fragment-tiled layout."""
    assert src.is_cuda and src.dtype == BF16
    src = src.contiguous()
    R, K = src.shape[-2], src.shape[-1]
    count = src.numel() // (R * K)
    dst = torch.empty_like(src)
    s = stream if stream is not None else torch.cuda.current_stream(src.device)
    check(lib().nkm_pack_ft(src.data_ptr(), dst.data_ptr(), R, K, count, mode, s.cuda_stream), "nkm_pack_ft")
    return dst


def rope_tables(max_pos: int, head_dim: int, theta: float, device) -> tuple:
    """bf16 cos/sin ``[max_pos, head_dim]`` (HF default RoPE, computed in fp32 then cast)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(BF16).to(device), emb.sin().to(BF16).to(device)


def sample_tokens(logits: torch.Tensor, positions: Optional[torch.Tensor] = None, *, top_k: int = 1,
                  top_p: float = 1.0, temperature: float = 1.0, seed: int = 0,
                  workspace: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                  stream=None) -> torch.Tensor:
    """Next tokens ``[B]`` int32 drawn on the device from ``logits [B, V]`` fp32
    (``nkm_sample_logits``): the top_k largest logits, temperature, top_p prefix, a SplitMix64
    uniform per (seed, row, position); ``top_k`` = 1 is greedy."""
    B, V = int(logits.shape[0]), int(logits.shape[1])
    need = lib().nkm_sample_workspace_bytes(B, V, top_k)
    if need == 0:
        raise _lib.NkmError(_lib.NKM_ERR_ARG, "nkm_sample_workspace_bytes")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=logits.device)
    tokens = out if out is not None else torch.empty(B, dtype=torch.int32, device=logits.device)
    params = _lib.nkm_sample_params(top_k, top_p, temperature, seed)
    s = stream if stream is not None else torch.cuda.current_stream(logits.device)
    check(lib().nkm_sample_logits(logits.data_ptr(), B, V, ctypes.byref(params), _ptr(positions), tokens.data_ptr(),
                                  workspace.data_ptr(), workspace.numel(), s.cuda_stream), "nkm_sample_logits")
    return tokens


class GpuLayer:
    """One decoder layer's weights in the kernel layouts (device tensors)."""

    def __init__(self, wq, wk, wv, wo, q_norm, k_norm, ln1, ln2, router, gate_up, down, router_bias=None,
                 attention=True, moe=True):
        if attention:
            self.wqkv_ft = pack_ft(torch.cat([wq, wk, wv], 0).to(BF16))
            self.wo_ft = pack_ft(wo.to(BF16))
            self.q_norm = q_norm.to(BF16).contiguous()
            self.k_norm = k_norm.to(BF16).contiguous()
            self.ln1 = ln1.to(BF16).contiguous()
        else:
            self.wqkv_ft = self.wo_ft = self.q_norm = self.k_norm = self.ln1 = None
        if moe:
            self.ln2 = ln2.to(BF16).contiguous()
            self.router = router.to(BF16).contiguous()
            self.w13_ft = pack_ft(gate_up.to(BF16), _lib.NKM_PACK_GATE_UP)
            self.w2_ft = pack_ft(down.to(BF16))
            self.router_bias = None if router_bias is None else router_bias.to(torch.float32).contiguous()
        else:
            self.ln2 = self.router = self.w13_ft = self.w2_ft = self.router_bias = None

    def c_struct(self) -> _lib.nkm_qwen3_layer:
        return _lib.nkm_qwen3_layer(_ptr(self.wqkv_ft), _ptr(self.wo_ft), _ptr(self.q_norm), _ptr(self.k_norm),
                                    _ptr(self.ln1), _ptr(self.ln2), _ptr(self.router), _ptr(self.w13_ft),
                                    _ptr(self.w2_ft), _ptr(self.router_bias))


class Qwen3MoeMegakernel:
    """A decode-megakernel instance on one GPU.

    ``layers`` may repeat the same ``GpuLayer`` object (weights shared by several layers);
    each layer still has its own K/V pages.
    """

    def __init__(self, shape: Qwen3MoeShape, layers: Sequence[GpuLayer], *, max_batch: int, num_blocks: int,
                 final_norm: Optional[torch.Tensor] = None, lm_head: Optional[torch.Tensor] = None,
                 embed: Optional[torch.Tensor] = None, rope_max_pos: int = 40960, device=None,
                 kv_pools: bool = True, shard=None, xchg=None):
        """``shard`` (``sharding.RankShard``) and ``xchg`` (``sharding.XchgRegion``) make this
        instance one rank of a tensor + expert parallel group: ``shape`` then carries the local
        head counts, ``layers`` the local heads and experts, and ``num_experts`` stays global."""
        self.shape = shape
        self.device = torch.device(device if device is not None else "cuda")
        self.layers = list(layers)
        assert len(self.layers) == shape.num_hidden_layers
        self.max_batch = max_batch
        self.num_blocks = num_blocks
        L, nkv, D = shape.num_hidden_layers, shape.num_key_value_heads, shape.head_dim
        if kv_pools:
            self.k_pool = torch.zeros(L, num_blocks, nkv, shape.block_size, D, dtype=BF16, device=self.device)
            self.v_pool = torch.zeros_like(self.k_pool)
            self.rope_cos, self.rope_sin = rope_tables(rope_max_pos, D, shape.rope_theta, self.device)
        else:
            self.k_pool = self.v_pool = self.rope_cos = self.rope_sin = None
            rope_max_pos = 0
        self.final_norm = None if final_norm is None else final_norm.to(BF16).contiguous()
        self.lm_head_ft = None if lm_head is None else pack_ft(lm_head.to(BF16))
        self.embed = None if embed is None else embed.to(BF16).contiguous()
        self._layer_structs = (_lib.nkm_qwen3_layer * L)(*[l.c_struct() for l in self.layers])
        vocab = shape.vocab_size if (lm_head is not None or embed is not None) else 0
        self._desc = _lib.nkm_qwen3_desc(
            shape.hidden_size, shape.num_attention_heads, nkv, D, shape.num_experts, shape.num_experts_per_tok,
            shape.moe_intermediate_size, L, vocab, shape.rms_norm_eps, self._layer_structs,
            _ptr(self.final_norm), _ptr(self.lm_head_ft), _ptr(self.embed), _ptr(self.rope_cos),
            _ptr(self.rope_sin), rope_max_pos, _ptr(self.k_pool), _ptr(self.v_pool), num_blocks,
            shape.block_size, max_batch)
        self.shard = shard
        if shard is not None and shard.world > 1:
            if xchg is None:
                raise ValueError("a rank of a parallel group needs its exchange region")
            self._desc.n_ranks = shard.world
            self._desc.rank = shard.rank
            self._desc.expert_begin = shard.expert_begin
            self._desc.n_local_experts = shard.n_local_experts
            for q, ptr in enumerate(xchg.ptrs):
                self._desc.xchg[q] = ptr
            need = lib().nkm_qwen3_xchg_bytes(ctypes.byref(self._desc))
            if need == 0 or need > xchg.nbytes:
                raise _lib.NkmError(_lib.NKM_ERR_ARG, f"exchange region of {xchg.nbytes} bytes, need {need}")
        else:
            self._desc.n_ranks = 1
            self._desc.n_local_experts = shape.num_experts
        nbytes = lib().nkm_qwen3_workspace_bytes(ctypes.byref(self._desc))
        if nbytes == 0:
            raise _lib.NkmError(_lib.NKM_ERR_ARG, "nkm_qwen3_workspace_bytes")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        h = ctypes.c_void_p()
        check(lib().nkm_qwen3_create(ctypes.byref(self._desc), self.workspace.data_ptr(), nbytes, ctypes.byref(h)),
              "nkm_qwen3_create")
        self._h = h

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib().nkm_qwen3_destroy(h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ calls
    def _step_struct(self, batch, *, x=None, input_ids=None, positions=None, block_table=None, y=None,
                     logits=None, first_layer=0, num_layers=0, stages=0, residual=1, traces=None):
        tr = traces or {}
        return _lib.nkm_qwen3_step(
            batch, _ptr(input_ids), _ptr(x), _ptr(positions), _ptr(block_table),
            0 if block_table is None else block_table.shape[1], _ptr(y), _ptr(logits), first_layer, num_layers,
            stages, residual, _ptr(tr.get("topk_idx")), _ptr(tr.get("topk_w")), _ptr(tr.get("router_logits")),
            _ptr(tr.get("qkv")), _ptr(tr.get("resid_mid")), _ptr(tr.get("resid_out")), _ptr(tr.get("stage_ns")))

    def _alloc_traces(self, batch, nl) -> Dict[str, torch.Tensor]:
        s, dev = self.shape, self.device
        R = (s.num_attention_heads + 2 * s.num_key_value_heads) * s.head_dim
        return {
            "topk_idx": torch.full((nl, batch, s.num_experts_per_tok), -1, dtype=torch.int32, device=dev),
            "topk_w": torch.zeros(nl, batch, s.num_experts_per_tok, dtype=torch.float32, device=dev),
            "router_logits": torch.zeros(nl, batch, s.num_experts, dtype=torch.float32, device=dev),
            "qkv": torch.zeros(nl, batch, R, dtype=BF16, device=dev),
            "resid_mid": torch.zeros(nl, batch, s.hidden_size, dtype=torch.float32, device=dev),
            "resid_out": torch.zeros(nl, batch, s.hidden_size, dtype=torch.float32, device=dev),
            "stage_ns": torch.zeros(3 + 6 * nl, dtype=torch.int64, device=dev),
        }

    def decode_step(self, positions: torch.Tensor, block_table: torch.Tensor, *, x: Optional[torch.Tensor] = None,
                    input_ids: Optional[torch.Tensor] = None, want_logits: bool = True, trace: bool = False,
                    first_layer: int = 0, num_layers: int = 0, out: Optional[Dict[str, torch.Tensor]] = None,
                    stage_times: bool = False, kv_first: bool = False, stream=None) -> Dict[str, torch.Tensor]:
        """Run one decode step (all layers by default).  K/V pools are updated in place.

        Returns ``{"hidden": [B,H] bf16, "logits": [B,V] fp32 (if requested), traces...}``;
        ``stage_times`` adds ``stage_ns``: globaltimer stamps of CTA 0 at kernel start, after
        every grid barrier and at kernel end.  ``kv_first``: rows may be consecutive positions of
        one sequence (same block-table row); every row's K/V is written before the attention
        reads the cache (``NKM_STAGE_KV_FIRST``: multi-token decode, chunked prefill).
        """
        B = int(positions.shape[0])
        nl = num_layers or (self.shape.num_hidden_layers - first_layer)
        res = out if out is not None else {}
        if "hidden" not in res:
            res["hidden"] = torch.empty(B, self.shape.hidden_size, dtype=BF16, device=self.device)
        if want_logits and self.lm_head_ft is not None and "logits" not in res:
            res["logits"] = torch.empty(B, self.shape.vocab_size, dtype=torch.float32, device=self.device)
        traces = self._alloc_traces(B, nl) if trace else None
        if stage_times and not trace:
            traces = {"stage_ns": torch.zeros(3 + 6 * nl, dtype=torch.int64, device=self.device)}
        if kv_first and traces:
            traces.pop("stage_ns", None)  # the extra barriers of this mode are not stamped
        st = self._step_struct(B, x=x, input_ids=input_ids, positions=positions, block_table=block_table,
                               y=res["hidden"], logits=res.get("logits") if want_logits else None,
                               first_layer=first_layer, num_layers=nl, traces=traces,
                               stages=_lib.NKM_STAGE_KV_FIRST if kv_first else 0)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib().nkm_qwen3_decode_step(self._h, ctypes.byref(st), s.cuda_stream), "nkm_qwen3_decode_step")
        if traces:
            res.update(traces)
        return res

    def attention_block(self, layer: int, x: torch.Tensor, positions: torch.Tensor, block_table: torch.Tensor,
                        residual: bool = False, trace: bool = False, qkv_in: bool = False,
                        stream=None) -> Dict[str, torch.Tensor]:
        """One attention block.  ``qkv_in``: take the q/k/v projections from ``qkv_buffer()``
        (written by the caller) instead of RMSNorm(ln1) + QKV GEMV of ``x``."""
        B = int(x.shape[0])
        y = torch.empty(B, self.shape.hidden_size, dtype=BF16, device=self.device)
        traces = self._alloc_traces(B, 1) if trace else None
        st = self._step_struct(B, x=x, positions=positions, block_table=block_table, y=y, residual=int(residual),
                               first_layer=layer, num_layers=1, traces=traces,
                               stages=_lib.NKM_STAGE_QKV_IN if qkv_in else 0)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib().nkm_qwen3_attention_block(self._h, layer, ctypes.byref(st), s.cuda_stream),
              "nkm_qwen3_attention_block")
        res = {"hidden": y}
        if traces:
            res.update(traces)
        return res

    def sample(self, logits: torch.Tensor, positions: Optional[torch.Tensor] = None, *, top_k: int = 1,
               top_p: float = 1.0, temperature: float = 1.0, seed: int = 0, out: Optional[torch.Tensor] = None,
               stream=None) -> torch.Tensor:
        """Next tokens ``[B]`` int32 drawn on the device from ``logits [B, V]`` fp32 (see
        ``sample_tokens``); the sampler's scratch is kept with the instance."""
        need = lib().nkm_sample_workspace_bytes(int(logits.shape[0]), int(logits.shape[1]), top_k)
        ws = getattr(self, "_sample_ws", None)
        if ws is None or ws.numel() < need:
            ws = self._sample_ws = torch.empty(max(need, 8), dtype=torch.uint8, device=self.device)
        return sample_tokens(logits, positions, top_k=top_k, top_p=top_p, temperature=temperature, seed=seed,
                             workspace=ws, out=out, stream=stream)

    def qkv_buffer(self) -> torch.Tensor:
        """The handle's QKV buffer as a bf16 tensor ``[max_batch, (nq + 2 nkv) * head_dim]`` (a view
        of the workspace): raw q/k/v projections that ``attention_block(..., qkv_in=True)`` consumes
        (``nkm_qwen3_qkv_buffer``)."""
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        check(lib().nkm_qwen3_qkv_buffer(self._h, ctypes.byref(ptr), ctypes.byref(nbytes)), "nkm_qwen3_qkv_buffer")
        off = ptr.value - self.workspace.data_ptr()
        s = self.shape
        R = (s.num_attention_heads + 2 * s.num_key_value_heads) * s.head_dim
        return self.workspace[off:off + nbytes.value].view(BF16).view(self.max_batch, R)

    def moe_block(self, layer: int, x: torch.Tensor, residual: bool = False, trace: bool = False,
                  stream=None) -> Dict[str, torch.Tensor]:
        B = int(x.shape[0])
        y = torch.empty(B, self.shape.hidden_size, dtype=BF16, device=self.device)
        traces = self._alloc_traces(B, 1) if trace else None
        st = self._step_struct(B, x=x, y=y, residual=int(residual), first_layer=layer, num_layers=1, traces=traces)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib().nkm_qwen3_moe_block(self._h, layer, ctypes.byref(st), s.cuda_stream), "nkm_qwen3_moe_block")
        res = {"hidden": y}
        if traces:
            res.update(traces)
        return res

    def status(self, stream=None) -> int:
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return lib().nkm_qwen3_status(self._h, s.cuda_stream)

    def check_status(self, stream=None) -> None:
        st = self.status(stream)
        if st != 0:
            raise _lib.NkmError(st, "decode kernel")


def pack_mxfp8_experts(codes: torch.Tensor, scales: torch.Tensor, gate_up: bool, stream=None) -> torch.Tensor:
    """MXFP8 expert matrices (e4m3 codes ``[E, rows, cols]`` as uint8 or float8_e4m3fn, e8m0
    scales ``[E, rows, cols/32]`` uint8; CUDA) into the units the MXFP8 grouped GEMM streams
    (``nkm_pack_mxfp8_experts``)."""
    codes = codes.contiguous().view(torch.uint8) if codes.dtype != torch.uint8 else codes.contiguous()
    scales = scales.contiguous()
    E, R, K = codes.shape
    n = lib().nkm_mxfp8_experts_bytes(E, R, K)
    if n == 0:
        raise _lib.NkmError(_lib.NKM_ERR_ARG, "nkm_mxfp8_experts_bytes")
    out = torch.empty(n, dtype=torch.uint8, device=codes.device)
    st = stream if stream is not None else torch.cuda.current_stream(codes.device)
    check(lib().nkm_pack_mxfp8_experts(codes.data_ptr(), scales.data_ptr(), out.data_ptr(), E, R, K, int(gate_up),
                                       st.cuda_stream), "nkm_pack_mxfp8_experts")
    return out


class MoeTcBlock:
    """The MoE block on tcgen05/TMEM grouped GEMMs (``nkm_moe_block_tc``) for token counts that
    give the experts several columns each (config 3 and larger batches).  Weights in the plain
    Hugging Face layouts: gate_up ``[E, 2I, H]`` (gate rows then up rows), down ``[E, H, I]``;
    or MXFP8 (``mxfp8=(gate_up codes, gate_up scales, down codes, down scales)``, OCP MX: e4m3
    codes and e8m0 scales per 32 along K, in the same row layouts; ``gate_up``/``down`` then
    unused).  ``expert_begin`` / ``n_local_experts``: the weights hold only that range of experts
    (expert parallel; ``partial`` calls then sum only their contributions)."""

    def __init__(self, ln2: torch.Tensor, router: torch.Tensor, gate_up: Optional[torch.Tensor],
                 down: Optional[torch.Tensor], *, eps: float, top_k: int, max_tokens: int,
                 router_bias: Optional[torch.Tensor] = None, device=None, mxfp8=None, expert_begin: int = 0,
                 n_local_experts: int = 0):
        self.device = torch.device(device if device is not None else "cuda")
        self.ln2 = ln2.to(self.device, BF16).contiguous()
        self.router = router.to(self.device, BF16).contiguous()
        self.router_bias = None if router_bias is None else router_bias.to(self.device, torch.float32).contiguous()
        if mxfp8 is not None:
            gc, gs, dc, ds = (t.to(self.device) for t in mxfp8)
            E, I2, H = gc.shape
            self.w13 = pack_mxfp8_experts(gc, gs, True)
            self.w2 = pack_mxfp8_experts(dc, ds, False)
            fmt = _lib.NKM_MOE_WEIGHTS_MXFP8
        else:
            self.w13 = gate_up.to(self.device, BF16).contiguous()
            self.w2 = down.to(self.device, BF16).contiguous()
            E, I2, H = self.w13.shape
            fmt = _lib.NKM_MOE_WEIGHTS_BF16
        E = int(self.router.shape[0])  # routing covers every expert; the weights may hold a range of them
        self.H, self.E, self.K, self.I = H, E, top_k, I2 // 2
        self._desc = _lib.nkm_moe_tc_desc(H, E, top_k, self.I, eps, self.ln2.data_ptr(), self.router.data_ptr(),
                                          _ptr(self.router_bias), self.w13.data_ptr(), self.w2.data_ptr(), max_tokens,
                                          fmt, expert_begin, n_local_experts)
        n = lib().nkm_moe_tc_workspace_bytes(ctypes.byref(self._desc))
        if n == 0:
            raise _lib.NkmError(_lib.NKM_ERR_ARG, "nkm_moe_tc_workspace_bytes")
        self.workspace = torch.empty(n, dtype=torch.uint8, device=self.device)

    def __call__(self, x: torch.Tensor, residual: bool = False, stream=None):
        T = int(x.shape[0])
        y = torch.empty_like(x)
        idx = torch.empty(T, self.K, dtype=torch.int32, device=self.device)
        w = torch.empty(T, self.K, dtype=torch.float32, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        check(lib().nkm_moe_block_tc(ctypes.byref(self._desc), T, x.data_ptr(), y.data_ptr(), int(residual),
                                     idx.data_ptr(), w.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(),
                                     s.cuda_stream), "nkm_moe_block_tc")
        return y, idx, w

    def status(self, stream=None) -> int:
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return lib().nkm_moe_tc_status(self.workspace.data_ptr(), s.cuda_stream)


class Qwen3MoeWideDecoder:
    """Decode steps at batches beyond one decode-kernel launch (config 3: B = 64, contexts up to
    8192), per layer ``transformer_qwen.py:218-378`` at that batch:

    * the attention block (``nkm_qwen3_attention_block``: RMSNorm, QKV, q/k-norm, RoPE, K/V write,
      GQA decode attention, O-projection, residual) in launches of up to ``row_chunk`` (32) rows;
    * the MoE block on the tcgen05/TMEM grouped GEMMs (``nkm_moe_block_tc``) over all rows at
      once, where 64 tokens give the experts ~4 columns each;
    * the residual between the blocks is bf16 (the reference's bf16 residual adds,
      ``transformer_qwen.py:331-333, 370-372``);
    * final RMSNorm (fp32) and the LM head as one plain GEMM over all rows (cuBLAS through torch:
      one read of the 622 MB head for the whole batch).

    ``layers``: per layer a dict of Hugging Face layout tensors (``wq, wk, wv, wo, q_norm,
    k_norm, ln1, ln2, router, gate_up, down``, optional ``router_bias``; MXFP8 experts as
    ``mxfp8 = (gate_up codes, gate_up scales, down codes, down scales)`` in place of ``gate_up``
    and ``down``); a list may repeat the same dict (weights shared by several layers; each layer
    still has its own K/V pages)."""

    def __init__(self, shape: Qwen3MoeShape, layers: Sequence[Dict[str, torch.Tensor]], *, max_batch: int,
                 num_blocks: int, final_norm: Optional[torch.Tensor] = None, lm_head: Optional[torch.Tensor] = None,
                 embed: Optional[torch.Tensor] = None, rope_max_pos: int = 40960, row_chunk: int = 32,
                 device=None):
        self.shape = shape
        self.device = torch.device(device if device is not None else "cuda")
        self.max_batch = max_batch
        self.row_chunk = min(row_chunk, 32, max_batch)
        att, moe = {}, {}
        for lw in layers:
            if id(lw) in att:
                continue
            att[id(lw)] = GpuLayer(lw["wq"], lw["wk"], lw["wv"], lw["wo"], lw["q_norm"], lw["k_norm"], lw["ln1"],
                                   None, None, None, None, moe=False)
            moe[id(lw)] = MoeTcBlock(lw["ln2"], lw["router"], lw.get("gate_up"), lw.get("down"),
                                     eps=shape.rms_norm_eps, top_k=shape.num_experts_per_tok, max_tokens=max_batch,
                                     router_bias=lw.get("router_bias"), device=self.device, mxfp8=lw.get("mxfp8"))
        self.moe = [moe[id(lw)] for lw in layers]
        self.attn = Qwen3MoeMegakernel(shape, [att[id(lw)] for lw in layers], max_batch=self.row_chunk,
                                       num_blocks=num_blocks, rope_max_pos=rope_max_pos, device=self.device)
        self.k_pool, self.v_pool = self.attn.k_pool, self.attn.v_pool
        self.final_norm = None if final_norm is None else final_norm.to(self.device, torch.float32)
        self.lm_head = None if lm_head is None else lm_head.to(self.device, BF16).contiguous()
        self.embed = None if embed is None else embed.to(self.device, BF16).contiguous()

    def decode_step(self, positions: torch.Tensor, block_table: torch.Tensor, *, x: Optional[torch.Tensor] = None,
                    input_ids: Optional[torch.Tensor] = None, want_logits: bool = True, trace: bool = False,
                    stream=None) -> Dict[str, torch.Tensor]:
        """One decode step for ``B = positions.shape[0]`` rows (``B <= max_batch``).  Returns
        ``{"hidden": [B, H] bf16, "logits": [B, V] fp32}``; ``trace`` adds per layer
        ``resid_mid`` / ``resid_out`` (bf16 as fp32) and the MoE routing ``topk_idx`` / ``topk_w``."""
        B = int(positions.shape[0])
        assert 0 < B <= self.max_batch, B
        if x is None:
            x = self.embed[input_ids.long()]
        h = x.to(BF16).contiguous()
        L = self.shape.num_hidden_layers
        tr = {"resid_mid": [], "resid_out": [], "topk_idx": [], "topk_w": []} if trace else None
        for layer in range(L):
            mid = torch.empty_like(h)
            for r0 in range(0, B, self.row_chunk):
                r1 = min(B, r0 + self.row_chunk)
                mid[r0:r1] = self.attn.attention_block(layer, h[r0:r1], positions[r0:r1], block_table[r0:r1],
                                                       residual=True, stream=stream)["hidden"]
            h, idx, w = self.moe[layer](mid, residual=True, stream=stream)
            if tr is not None:
                tr["resid_mid"].append(mid.float())
                tr["resid_out"].append(h.float())
                tr["topk_idx"].append(idx)
                tr["topk_w"].append(w)
        res = {"hidden": h}
        if want_logits and self.lm_head is not None:
            xf = h.float()
            xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.shape.rms_norm_eps) * self.final_norm
            res["logits"] = torch.mm(xn.to(BF16), self.lm_head.t(), out_dtype=torch.float32)
        if tr is not None:
            res.update({k: torch.stack(v) for k, v in tr.items()})
        return res

    def check_status(self) -> None:
        self.attn.check_status()
        for m in {id(m): m for m in self.moe}.values():
            st = m.status()
            if st != 0:
                raise _lib.NkmError(st, "tcgen05 MoE block")

    def close(self) -> None:
        self.attn.close()


class Qwen3MoeWideDecoderEP:
    """Config 3 across the GPUs of one node (one process per GPU): rank r of N owns the rows
    ``[B r / N, B (r + 1) / N)`` for attention (every rank holds the attention weights; the rows'
    K/V pages live on their rank) and the experts ``[E r / N, E (r + 1) / N)`` (expert parallel).
    Per layer:

    * the attention block on the rank's rows (``nkm_qwen3_attention_block``);
    * the post-attention rows of every rank gathered on every rank over NVLink (``nkm_ep_push``
      into the peers' exchange regions, ``nkm_ep_wait`` on the rank's own counter);
    * the MoE block over all B rows with the rank's experts only (routing over all experts,
      ``nkm_moe_block_tc_partial``), fp32 partial sums;
    * each owner's rows of those partials pushed to the owner, which adds them in rank order to
      its residual (``nkm_ep_reduce``: bf16 residual, as on one GPU).

    ``layers[l]``: dict with the attention tensors (``wq, wk, wv, wo, q_norm, k_norm, ln1``),
    ``ln2``, ``router`` (all experts) and the rank's experts as ``gate_up`` / ``down`` (or
    ``mxfp8``) for experts ``[expert_begin, expert_begin + n_local)``.  ``xchg``: this rank's
    ``sharding.XchgRegion`` of at least ``exchange_bytes(B, H, N)`` bytes."""

    @staticmethod
    def exchange_bytes(batch: int, hidden: int, world: int) -> int:
        rows = batch // world
        return 256 + batch * hidden * 2 + world * rows * hidden * 4

    def __init__(self, shape: Qwen3MoeShape, layers: Sequence[Dict[str, torch.Tensor]], *, rank: int, world: int,
                 xchg, batch: int, expert_begin: int, n_local: int, num_blocks: int,
                 final_norm: Optional[torch.Tensor] = None, lm_head: Optional[torch.Tensor] = None,
                 embed: Optional[torch.Tensor] = None, rope_max_pos: int = 40960, device=None):
        assert batch % world == 0 and batch // world <= 32, (batch, world)
        self.shape, self.rank, self.world, self.xchg = shape, rank, world, xchg
        self.device = torch.device(device if device is not None else "cuda")
        self.B, self.rows, H = batch, batch // world, shape.hidden_size
        att, moe = {}, {}
        for lw in layers:
            if id(lw) in att:
                continue
            att[id(lw)] = GpuLayer(lw["wq"], lw["wk"], lw["wv"], lw["wo"], lw["q_norm"], lw["k_norm"], lw["ln1"],
                                   None, None, None, None, moe=False)
            moe[id(lw)] = MoeTcBlock(lw["ln2"], lw["router"], lw.get("gate_up"), lw.get("down"),
                                     eps=shape.rms_norm_eps, top_k=shape.num_experts_per_tok, max_tokens=batch,
                                     router_bias=lw.get("router_bias"), device=self.device, mxfp8=lw.get("mxfp8"),
                                     expert_begin=expert_begin, n_local_experts=n_local)
        self.moe = [moe[id(lw)] for lw in layers]
        self.attn = Qwen3MoeMegakernel(shape, [att[id(lw)] for lw in layers], max_batch=self.rows,
                                       num_blocks=num_blocks, rope_max_pos=rope_max_pos, device=self.device)
        self.k_pool, self.v_pool = self.attn.k_pool, self.attn.v_pool
        self.final_norm = None if final_norm is None else final_norm.to(self.device, torch.float32)
        self.lm_head = None if lm_head is None else lm_head.to(self.device, BF16).contiguous()
        self.embed = None if embed is None else embed.to(self.device, BF16).contiguous()
        # exchange region: [0] gather counter, [8] scatter counter, [256..) all rows (bf16), then the
        # ranks' partials of this rank's rows (fp32 [N][rows][H])
        self._g_off, self._p_off = 256, 256 + batch * H * 2
        own = xchg.ptrs[rank]
        nbytes = self.exchange_bytes(batch, H, world)
        assert xchg.nbytes >= nbytes, (xchg.nbytes, nbytes)
        self._gather = _device_view(own + self._g_off, batch * H * 2, self.device).view(BF16).view(batch, H)
        self._parts = _device_view(own + self._p_off, world * self.rows * H * 4, self.device).view(
            torch.float32).view(world, self.rows, H)
        self._arr = int(lib().nkm_ep_arrivals_per_push()) * world
        self._targets = [0, 0]
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._part = torch.empty(batch, H, dtype=torch.float32, device=self.device)
        self._dst_g = (ctypes.c_void_p * world)(*[p + self._g_off for p in xchg.ptrs])
        self._flag_g = (ctypes.c_void_p * world)(*[p for p in xchg.ptrs])
        self._flag_s = [(ctypes.c_void_p * 1)(p + 8) for p in xchg.ptrs]
        self._dst_p = [(ctypes.c_void_p * 1)(p + self._p_off) for p in xchg.ptrs]

    def _wait(self, which: int, s) -> None:
        self._targets[which] += self._arr
        check(lib().nkm_ep_wait(self.xchg.ptrs[self.rank] + 8 * which, self._targets[which],
                                self._status.data_ptr(), s.cuda_stream), "nkm_ep_wait")

    def decode_step(self, positions: torch.Tensor, block_table: torch.Tensor, *, x: Optional[torch.Tensor] = None,
                    input_ids: Optional[torch.Tensor] = None, want_logits: bool = True, trace: bool = False,
                    stream=None) -> Dict[str, torch.Tensor]:
        """One decode step for this rank's rows (``positions`` / ``block_table`` / ``x`` or
        ``input_ids`` of those rows).  Every rank must call it for the same step."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        H, R, r = self.shape.hidden_size, self.rows, self.rank
        if x is None:
            x = self.embed[input_ids.long()]
        h = x.to(BF16).contiguous()
        tr = {"resid_mid": [], "resid_out": [], "topk_idx": []} if trace else None
        for layer in range(self.shape.num_hidden_layers):
            mid = self.attn.attention_block(layer, h, positions, block_table, residual=True, stream=s)["hidden"]
            # every rank's rows into every rank's gather area
            check(lib().nkm_ep_push(mid.data_ptr(), R * H * 2, self._dst_g, self.world, r * R * H * 2, self._flag_g,
                                    s.cuda_stream), "nkm_ep_push")
            self._wait(0, s)
            blk = self.moe[layer]
            idx = torch.empty(self.B, blk.K, dtype=torch.int32, device=self.device)
            check(lib().nkm_moe_block_tc_partial(ctypes.byref(blk._desc), self.B, self._gather.data_ptr(),
                                                 self._part.data_ptr(), idx.data_ptr(), None, blk.workspace.data_ptr(),
                                                 blk.workspace.numel(), s.cuda_stream), "nkm_moe_block_tc_partial")
            # each owner's rows of this rank's partials into the owner's slot r
            for q in range(self.world):
                check(lib().nkm_ep_push(self._part[q * R:(q + 1) * R].data_ptr(), R * H * 4, self._dst_p[q], 1,
                                        r * R * H * 4, self._flag_s[q], s.cuda_stream), "nkm_ep_push")
            self._wait(1, s)
            out = torch.empty_like(mid)
            check(lib().nkm_ep_reduce(self._parts.data_ptr(), self.world, R, H, mid.data_ptr(), out.data_ptr(),
                                      s.cuda_stream), "nkm_ep_reduce")
            h = out
            if tr is not None:
                tr["resid_mid"].append(mid.float())
                tr["resid_out"].append(out.float())
                tr["topk_idx"].append(idx[r * R:(r + 1) * R])
        res = {"hidden": h}
        if want_logits and self.lm_head is not None:
            xf = h.float()
            xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.shape.rms_norm_eps) * self.final_norm
            res["logits"] = torch.mm(xn.to(BF16), self.lm_head.t(), out_dtype=torch.float32)
        if tr is not None:
            res.update({k: torch.stack(v) for k, v in tr.items()})
        return res

    def check_status(self) -> None:
        torch.cuda.synchronize(self.device)
        st = int(self._status.item())
        if st:
            raise _lib.NkmError(st, "expert-parallel exchange")
        self.attn.check_status()
        for m in {id(m): m for m in self.moe}.values():
            st = m.status()
            if st != 0:
                raise _lib.NkmError(st, "tcgen05 MoE block")

    def close(self) -> None:
        self.attn.close()


def _device_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor over device memory this process owns (the rank's own exchange region)."""

    class _Mem:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Mem(), device=device)
