/*
 * nkimoe.h — C ABI of the B200 (sm_100a) Qwen3-MoE token-generation megakernel.
 *
 * Plain pointers and sizes only; every pointer named "device" is CUDA device memory owned
 * by the caller.  No entry point allocates device memory: the caller sizes and passes the
 * workspace (nkm_qwen3_workspace_bytes).  All bf16 tensors are row-major unless the name
 * ends in _ft ("fragment-tiled", produced by nkm_pack_ft).
 *
 * Each entry point names the reference interface it replaces (paths inside the reference
 * project KevGomes1403/nki-moe-megakernel).
 */
#ifndef NKIMOE_H_
#define NKIMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (return values and the device status word). */
#define NKM_OK 0
#define NKM_ERR_ARG 1          /* bad argument / unsupported shape (host-side check) */
#define NKM_ERR_CUDA 2         /* a CUDA runtime call failed */
#define NKM_ERR_TIMEOUT 4      /* a grid barrier or copy wait gave up (device) */
#define NKM_ERR_INDEX 8        /* a token id, position or block id was out of range (device;
                                  the access is clamped or skipped) */

typedef struct CUstream_st* nkm_stream_t; /* == cudaStream_t */

/* Per-layer weights (device pointers, bf16).  Replaces the per-layer argument lists
 * Wq/Wk/Wv/Wo/qn/kn/gpre/gpost/router/gate_up/down of
 * megakernels/qwen3_moe/transformer_qwen.py:68-90 (gathered in
 * megakernels/qwen3_moe/qwen_with_megakernel.py:376-408). */
typedef struct nkm_qwen3_layer {
  const void* wqkv_ft;  /* [(nq+2*nkv)*128, H]  rows: q heads, k heads, v heads       */
  const void* wo_ft;    /* [H, nq*128]                                               */
  const void* q_norm;   /* [128]                                                     */
  const void* k_norm;   /* [128]                                                     */
  const void* ln1;      /* [H] input_layernorm                                       */
  const void* ln2;      /* [H] post_attention_layernorm                              */
  const void* router;   /* [E, H] (plain row-major)                                  */
  const void* w13_ft;   /* [E][2I, H]  gate/up, packed with NKM_PACK_GATE_UP          */
  const void* w2_ft;    /* [E][H, I]   down                                          */
  const float* router_bias; /* [E] fp32 added to the router logits, or NULL            */
} nkm_qwen3_layer;

/* Model description.  Replaces the NxDI model + config objects
 * (qwen_with_megakernel.py:102-132, 601-695). */
typedef struct nkm_qwen3_desc {
  int32_t hidden;       /* H (multiple of 256, <= 2048)          2048   */
  int32_t n_q_heads;    /* query heads held by this GPU           32    */
  int32_t n_kv_heads;   /* kv heads held by this GPU              4     */
  int32_t head_dim;     /* must be 128                            128   */
  int32_t n_experts;    /* E (<= 256)                             128   */
  int32_t top_k;        /* K (<= 8)                               8     */
  int32_t moe_inter;    /* I (multiple of 32)                     768   */
  int32_t n_layers;     /* L                                      48    */
  int32_t vocab;        /* V (multiple of 16): rows of embed and lm_head_ft; 0 = neither 151936*/
  float rms_eps;        /*                                        1e-6  */
  const nkm_qwen3_layer* layers; /* host array of n_layers entries      */
  const void* final_norm;        /* [H] bf16 (may be NULL if vocab==0)  */
  const void* lm_head_ft;        /* [V, H] bf16 fragment-tiled          */
  const void* embed;             /* [V, H] bf16 row-major (may be NULL) */
  const void* rope_cos;          /* [rope_max_pos, 128] bf16            */
  const void* rope_sin;          /* [rope_max_pos, 128] bf16            */
  int32_t rope_max_pos;
  void* k_pool;   /* [L][num_blocks][n_kv_heads][block_size][128] bf16, mutated in place */
  void* v_pool;   /* same shape as k_pool                                                */
  int32_t num_blocks;
  int32_t block_size;  /* must be 128 */
  int32_t max_batch;   /* largest batch any step will use (<= 32)                         */
  /* Tensor + expert parallelism across GPUs (one process per GPU).  n_ranks == 1: the whole
   * model on this GPU.  n_ranks > 1: this GPU holds its attention heads (n_q_heads and
   * n_kv_heads above are the local counts) and experts [expert_begin, expert_begin +
   * n_local_experts) of n_experts (router, norms, embedding and LM head replicated); w13_ft /
   * w2_ft point at the local experts.  After the O-projection and after the experts, every
   * rank stores its partial sums into the exchange region of every rank (xchg[q], mapped in
   * this process; nkm_qwen3_xchg_bytes each) and all ranks sum them in rank order, so every
   * rank keeps the same residual stream.  The partials travel as 8-byte words that carry the
   * exchange's sequence number next to the value, so a rank reads them as soon as they land,
   * with no cross-GPU barrier.  The LM head is split over the vocabulary: rank r
   * computes 16-row strips [S r / n_ranks, S (r + 1) / n_ranks) of S = vocab / 16 (lm_head_ft
   * still points at the whole packed head), stores them into every rank's exchange region, and
   * every rank returns the full logits.  Replaces the TP/EP sharding of the NxDI model
   * (qwen_with_megakernel.py:102-132, replica groups at :360-362). */
  int32_t n_ranks;
  int32_t rank;
  int32_t expert_begin;
  int32_t n_local_experts;
  void* xchg[8];
} nkm_qwen3_desc;

typedef struct nkm_qwen3 nkm_qwen3; /* opaque handle (host memory only) */

/* Stage bits for nkm_qwen3_step.stages. */
#define NKM_STAGE_ATTN 1    /* RMSNorm(ln1)+QKV+q/k-norm+RoPE+KV write+attention+O-proj */
#define NKM_STAGE_MOE 2     /* RMSNorm(ln2)+router top-k+expert SwiGLU                  */
#define NKM_STAGE_LMHEAD 4  /* final RMSNorm + LM head (after the last layer run)       */
#define NKM_STAGE_QKV_IN 8  /* with NKM_STAGE_ATTN, one layer: the attention takes the raw q/k/v
                               projections the caller wrote into the QKV buffer
                               (nkm_qwen3_qkv_buffer) instead of RMSNorm(ln1) + QKV GEMV     */
#define NKM_STAGE_KV_FIRST 16 /* with NKM_STAGE_ATTN: every row's new K/V is written to the cache
                               before any row's attention reads it, so rows of ONE sequence at
                               consecutive positions (same block-table row) attend causally to
                               each other: multi-token decode and chunked prefill (reference
                               S_tkg > 1, nki_kernels/attention/attention_block_tkg.py:144-146).
                               Costs two grid barriers per layer.                             */

/* One decode step.  Replaces the kernel call
 *   get_multilayer_kernel_jit(L)[2](X, *W..., *K_caches, *V_caches, cos, sin, position_ids)
 * -> (Y, *K_out, *V_out)   (transformer_qwen.py:420-505, call site
 * qwen_with_megakernel.py:465-473).  K/V are written in place at positions[b]. */
typedef struct nkm_qwen3_step {
  int32_t batch;               /* B (1..max_batch)                                        */
  const int32_t* input_ids;    /* device [B]; if NULL x_in is used                          */
  const void* x_in;            /* device bf16 [B, H] hidden input (embeddings)              */
  const int32_t* positions;    /* device [B]: cache slot of the new token = prior length;
                                  must be < min(rope_max_pos, 128*max_blocks_per_seq)      */
  const int32_t* block_table;  /* device [B, max_blocks_per_seq]; entry < 0 at the write
                                  slot skips the K/V write (reference uint32_max skip)      */
  int32_t max_blocks_per_seq;
  void* y_out;                 /* device bf16 [B, H]: hidden after the last layer run
                                  (pre final norm), or the block output for block calls    */
  float* logits_out;           /* device fp32 [B, V] or NULL (LM head skipped)              */
  int32_t first_layer;         /* layer range to run: [first_layer, first_layer+num_layers) */
  int32_t num_layers;          /* 0 = all layers                                            */
  int32_t stages;              /* NKM_STAGE_* bits; no ATTN/MOE/LMHEAD bit = all three; QKV_IN
                                  and KV_FIRST are added to the selected stages             */
  int32_t residual;            /* 1 = blocks add into the residual stream (decoder layer);
                                  0 = a single-block call returns the block output only    */
  /* optional traces (device, NULL to skip), indexed [layer - first_layer] */
  int32_t* trace_topk_idx;     /* [nl, B, K]                                              */
  float* trace_topk_w;         /* [nl, B, K] renormalised affinities                      */
  float* trace_router_logits;  /* [nl, B, E]                                              */
  void* trace_qkv;             /* bf16 [nl, B, (nq+2nkv)*128] raw projections             */
  float* trace_resid_mid;      /* fp32 [nl, B, H] residual stream after attention         */
  float* trace_resid_out;      /* fp32 [nl, B, H] residual stream after the MoE block     */
  unsigned long long* trace_stage_ns; /* [3 + 6*nl] globaltimer stamps of CTA 0: kernel start,
                                  every grid barrier, kernel end (stage timing)            */
} nkm_qwen3_step;

/* Bytes of device workspace a handle needs (caller allocates, 256-byte aligned). */
size_t nkm_qwen3_workspace_bytes(const nkm_qwen3_desc* desc);

/* Bytes of the exchange region every rank allocates for n_ranks > 1 (zeroed, 256-byte aligned,
 * shared with the other ranks by CUDA IPC).  Replaces the collective buffers of the reference's
 * all-reduce (transformer_qwen.py:331-333, 370-372 with replica_groups). */
size_t nkm_qwen3_xchg_bytes(const nkm_qwen3_desc* desc);

/* Validate the description, lay out the workspace, copy the layer pointer table into it
 * and encode the K/V tensor maps.  Replaces compile()/load() of the NxDI model
 * (qwen_with_megakernel.py:601-695).  The calling thread's current device is used. */
int nkm_qwen3_create(const nkm_qwen3_desc* desc, void* workspace, size_t workspace_bytes,
                     nkm_qwen3** out);
void nkm_qwen3_destroy(nkm_qwen3* h);

/* Enqueue one decode step (exactly one cooperative kernel launch, nothing else) on `stream`.
 * Host-side checks return NKM_ERR_ARG/NKM_ERR_CUDA; device-side errors are reported by
 * nkm_qwen3_status.  Steps on one handle must not overlap (they share the workspace). */
int nkm_qwen3_decode_step(nkm_qwen3* h, const nkm_qwen3_step* step, nkm_stream_t stream);

/* Synchronise `stream` and return the device status word (0 = ok).  Device errors are
 * sticky: they accumulate over steps until this call reads and clears them (a step that
 * starts while a fatal error is recorded returns at its first barrier).  With n_ranks > 1, a
 * non-zero status also clears this rank's exchange region and restarts its exchange sequence:
 * after a failed step every rank calls this once all ranks' launches have ended, and the group
 * synchronises (a host barrier) before its next step. */
int nkm_qwen3_status(nkm_qwen3* h, nkm_stream_t stream);

/* Single fused attention block on layer `layer` (residual=0: returns the O-projection
 * output only).  Replaces attn_fused_qwen (megakernels/qwen3_moe/attn_fused_nki.py:50) and
 * attention_block_tkg (nki_kernels/attention/attention_block_tkg.py:83). */
int nkm_qwen3_attention_block(nkm_qwen3* h, int32_t layer, const nkm_qwen3_step* step,
                              nkm_stream_t stream);

/* The handle's QKV buffer: raw (pre-norm, pre-RoPE) bf16 projections [max_batch][R], R =
 * (n_q_heads + 2 n_kv_heads) * 128, row b = sequence b, columns q heads, k heads, v heads.
 * An attention block called with step->stages containing NKM_STAGE_QKV_IN consumes the rows
 * the caller wrote here instead of projecting the hidden input: the attention core on given
 * projections, as attention_tkg takes projected Q/K/V (nki_kernels/attention/attention_tkg.py:56).
 * At batch <= 8 the attention starts without waiting for the whole buffer: an element still
 * holding 0xffff (the "not written" mark every launch leaves in the buffer after reading it) is
 * re-read until it changes, bounded by the 2 s wait limit (then NKM_ERR_TIMEOUT), so the rows may
 * be produced by work that overlaps the launch.  *ptr receives the device address, *bytes (may
 * be NULL) the size. */
int nkm_qwen3_qkv_buffer(nkm_qwen3* h, void** ptr, size_t* bytes);

/* Single fused MoE block (RMSNorm(ln2) + router top-k + selective-expert SwiGLU) on layer
 * `layer`.  Replaces _qwen3_moe_sbuf_in_sbuf_out_hoisted / qwen3_moe_fused_tkg_sbuf_io
 * (megakernels/qwen3_moe/moe_fused_nki.py:769-997) and the primitive pair router_topk +
 * moe_tkg (nki_kernels/moe/router_topk.py:69, nki_kernels/moe/moe_tkg.py:56). */
int nkm_qwen3_moe_block(nkm_qwen3* h, int32_t layer, const nkm_qwen3_step* step,
                        nkm_stream_t stream);

/* Size of the device scratch array behind nkm_qwen3_moe_block_noalloc: 8 MiB, a static
 * array that every GPU which loads this library holds until the process exits. */
#define NKM_NOALLOC_SCRATCH_BYTES (8u << 20)

/* The MoE block of nkm_qwen3_moe_block (same kernel, same results) for callers that cannot
 * allocate device memory: runtimes whose memory pool owns the whole GPU and forbids library
 * allocations, and latency-critical loops where a cudaMalloc/cudaFree would synchronise the
 * device.  It takes the model description directly (no handle, no workspace) and allocates
 * nothing: its scratch (barrier, counters, residual rows, router logits, expert activations,
 * split-K partials) lives in a static device array of NKM_NOALLOC_SCRATCH_BYTES; a shape
 * whose scratch does not fit (hidden, top_k, moe_inter and batch set the size) is rejected
 * with NKM_ERR_ARG.  The first call on a device looks up that device's array address (again
 * if the device's context was replaced, e.g. after cudaDeviceReset) and must come before any
 * stream capture on that device.  Each call clears the part of the
 * scratch that must start at zero; all calls share the one array per device, so calls that
 * overlap on the GPU (other streams, other host threads) race: serialise them.  K/V pools,
 * RoPE tables and the LM head of `desc` are not used (they may be NULL).  `status_out`
 * (device int32, may be NULL) receives the device status word of this call (0 = ok).
 * No counterpart in the reference. */
int nkm_qwen3_moe_block_noalloc(const nkm_qwen3_desc* desc, int32_t layer, const nkm_qwen3_step* step,
                                int32_t* status_out, nkm_stream_t stream);

/* Weight layout converter (load time).  src: row-major bf16 [R, K]; dst: fragment-tiled
 * bf16 of the same size.  mode NKM_PACK_PLAIN keeps row order; NKM_PACK_GATE_UP takes the
 * Hugging Face experts gate_up [2I, K] (gate rows then up rows) and interleaves 8 gate rows
 * with the matching 8 up rows in every 16-row strip.  `count` matrices of the same shape
 * are converted back to back.  Replaces the HF->kernel converters
 * qwen_with_megakernel.py:171-271. */
#define NKM_PACK_PLAIN 0
#define NKM_PACK_GATE_UP 1
int nkm_pack_ft(const void* src, void* dst, int64_t rows, int64_t cols, int64_t count,
                int32_t mode, nkm_stream_t stream);

/* On-device sampling of the next token from LM-head logits (the on-device sampler the
 * reference configures with OnDeviceSamplingConfig, global_topk capped to top_k:
 * megakernels/qwen3_moe/qwen_with_megakernel.py:123-127, main.py:390-398). */
typedef struct nkm_sample_params {
  int32_t top_k;       /* 1: greedy (argmax; equal logits -> lowest token id); 2..64: sample   */
  float top_p;         /* (0, 1]: keep the shortest prefix of the top-k (by probability, after
                          temperature) whose mass reaches top_p                               */
  float temperature;   /* > 0: logits are multiplied by 1/temperature before the softmax      */
  uint64_t seed;       /* uniform draw u = top 24 bits of SplitMix64(SplitMix64(seed) ^
                          (position << 32 | row))                                              */
} nkm_sample_params;

/* Bytes of device scratch nkm_sample_logits needs (8-byte aligned; 0 for invalid sizes). */
size_t nkm_sample_workspace_bytes(int32_t batch, int32_t vocab, int32_t top_k);

/* tokens_out[b] (device int32) <- a token drawn from row b of logits (device fp32 [batch, vocab]):
 * the top_k largest logits (ties -> lower token id), softmax at temperature, top-p prefix,
 * inverse-CDF draw with the row's uniform (positions: device int32 [batch] or NULL = 0).  Two
 * kernel launches on `stream`; workspace of nkm_sample_workspace_bytes.  Returns NKM_ERR_ARG for
 * bad parameters. */
int nkm_sample_logits(const float* logits, int32_t batch, int32_t vocab, const nkm_sample_params* params,
                      const int32_t* positions, int32_t* tokens_out, void* workspace, size_t workspace_bytes,
                      nkm_stream_t stream);

/* ======================================================================================
 * MoE block on the 5th-generation tensor cores (tcgen05 + TMEM grouped GEMM), for batches
 * whose tokens give the experts several columns each (config 3: 64 tokens x top-8 over 128
 * experts).  Same arithmetic as nkm_qwen3_moe_block (RMSNorm(ln2), fp32 router logits in the
 * same fixed order, top-k on the logits, softmax at the top-k, bf16 renormalisation, bf16
 * SwiGLU, fp32 down projection times the routing weight); the expert outputs of a token are
 * summed in slot order.  Replaces moe_tkg's selective-expert path for dense token counts
 * (nki_kernels/moe/moe_tkg.py:56-293, selective_expert_impl.py:84-520).
 * ====================================================================================== */
typedef struct nkm_moe_tc_desc {
  int32_t hidden;             /* H: multiple of 256 */
  int32_t n_experts;          /* <= 256 */
  int32_t top_k;              /* <= 8 */
  int32_t moe_inter;          /* I: multiple of 64 */
  float rms_eps;
  const void* ln2;            /* bf16 [H] */
  const void* router;         /* bf16 [E, H] */
  const float* router_bias;   /* fp32 [E] or NULL */
  const void* w13;            /* bf16 [E][2I][H] row-major: gate rows then up rows (HF gate_up_proj),
                                 or (MXFP8) nkm_pack_mxfp8_experts(..., rows = 2I, cols = H, gate_up = 1) */
  const void* w2;             /* bf16 [E][H][I] row-major (HF down_proj), or (MXFP8)
                                 nkm_pack_mxfp8_experts(..., rows = H, cols = I, gate_up = 0) */
  int32_t max_tokens;         /* <= 512 */
  int32_t weight_format;      /* NKM_MOE_WEIGHTS_BF16 or NKM_MOE_WEIGHTS_MXFP8 (e4m3 values, e8m0
                                 scale per 32 along K; expanded exactly to bf16 in shared memory) */
  int32_t expert_begin;       /* expert parallel: w13 / w2 hold experts [expert_begin, + n_local_experts) */
  int32_t n_local_experts;    /* 0 = all n_experts (router and routing always cover all experts) */
} nkm_moe_tc_desc;

#define NKM_MOE_WEIGHTS_BF16 0
#define NKM_MOE_WEIGHTS_MXFP8 1

/* Bytes of nkm_pack_mxfp8_experts' output for `count` matrices of [rows, cols] (rows % 128,
 * cols % 64; 0 if invalid). */
size_t nkm_mxfp8_experts_bytes(int32_t count, int32_t rows, int32_t cols);
/* MXFP8 expert matrices (OCP MX: e4m3 codes [count][rows][cols] and e8m0 scales
 * [count][rows][cols/32], device) into the units the MXFP8 grouped GEMM streams.  gate_up = 1
 * for [E][2I][H] gate-then-up matrices.  Replaces the reference's MX weight layout
 * (nki_kernels/moe/down_projection_mx_shard_H.py:43-110, mxfp_x4 [128, n_I512_tile, H]). */
int nkm_pack_mxfp8_experts(const void* codes, const void* scales, void* dst, int32_t count, int32_t rows,
                           int32_t cols, int32_t gate_up, nkm_stream_t stream);

/* Workspace bytes (256-byte aligned; the first 4 bytes are the call's status word). */
size_t nkm_moe_tc_workspace_bytes(const nkm_moe_tc_desc* desc);
/* y_out = MoE(x_in) (+ x_in if residual) for `tokens` rows; topk_idx_out / topk_w_out (device
 * [tokens, top_k], may be NULL) receive the routing.  Six launches on `stream`. */
int nkm_moe_block_tc(const nkm_moe_tc_desc* desc, int32_t tokens, const void* x_in, void* y_out, int32_t residual,
                     int32_t* topk_idx_out, float* topk_w_out, void* workspace, size_t workspace_bytes,
                     nkm_stream_t stream);
/* Expert parallel: y_part (device fp32 [tokens, H]) = the contributions of this call's local experts
 * only (routing weights applied, summed over each token's local slots in slot order; no residual,
 * no rounding): the ranks' partials are then summed (nkm_ep_* below).  Six launches. */
int nkm_moe_block_tc_partial(const nkm_moe_tc_desc* desc, int32_t tokens, const void* x_in, float* y_part,
                             int32_t* topk_idx_out, float* topk_w_out, void* workspace, size_t workspace_bytes,
                             nkm_stream_t stream);
/* Synchronise and return the status word of the last call on this workspace (0 = ok). */
int nkm_moe_tc_status(void* workspace, nkm_stream_t stream);

/* Expert-parallel exchange over NVLink peer memory (the token dispatch / combine of the
 * reference's expert-parallel MoE, selective_expert_impl.py with moe_ep_degree; config 3 across
 * GPUs).  nkm_ep_push: `bytes` (multiple of 16) from src to dst[q] + dst_offset for q < n_dst
 * (<= 8; peer pointers from CUDA IPC), then nkm_ep_arrivals_per_push() arrivals (system-scope
 * release) on each flags[q] (64-bit counters in the receivers' memory).  nkm_ep_wait: polls
 * *flag (acquire, system scope) until it reaches target, bounded by 2 s (then NKM_ERR_TIMEOUT is
 * or-ed into *status).  nkm_ep_reduce: y = bf16(x + bf16(sum over q < n in order of
 * parts[q])) for rows x hidden elements (parts fp32 [n][rows][hidden], x and y bf16). */
int nkm_ep_push(const void* src, int64_t bytes, void* const* dst, int32_t n_dst, int64_t dst_offset,
                unsigned long long* const* flags, nkm_stream_t stream);
int32_t nkm_ep_arrivals_per_push(void);
int nkm_ep_wait(const unsigned long long* flag, unsigned long long target, int32_t* status, nkm_stream_t stream);
int nkm_ep_reduce(const float* parts, int32_t n, int32_t rows, int32_t hidden, const void* x_res, void* y_out,
                  nkm_stream_t stream);

/* ======================================================================================
 * GPT-OSS decode step (the reference's second megakernel,
 * megakernels/gpt_oss/transformer_gpt_oss.py:240-530, model class
 * megakernels/gpt_oss/gpt_oss_with_megakernel.py): sliding-window / full attention with
 * learned sinks, QKV and O-projection biases, YaRN RoPE, top-k softmax router with bias,
 * MXFP4 experts with biases and the clamped SwiGLU.  Head dim 64, batch <= 16.
 * ====================================================================================== */
typedef struct nkm_gptoss_layer {
  const void* wqkv_ft;     /* bf16 FT [(nq+2nkv)*64, H]: q heads, k heads, v heads          */
  const void* bqkv;        /* bf16 [(nq+2nkv)*64]                                           */
  const void* wo_ft;       /* bf16 FT [H, nq*64]                                            */
  const void* bo;          /* bf16 [H]                                                      */
  const void* sinks;       /* bf16 [nq] learned sink logits                                 */
  const void* ln1;         /* bf16 [H]                                                      */
  const void* ln2;         /* bf16 [H]                                                      */
  const void* router;      /* bf16 [E, H] row-major                                         */
  const void* router_bias; /* bf16 [E]                                                      */
  const void* w13_fp4;     /* nkm_pack_mxfp4 weights of gate/up [E][2I, H] (row 2i gate i,
                              row 2i+1 up i: Hugging Face's interleaved gate_up_proj)       */
  const void* s13;         /* nkm_pack_mxfp4 scales of gate/up                              */
  const void* b13;         /* bf16 [E][2I]                                                  */
  const void* w2_fp4;      /* nkm_pack_mxfp4 weights of down [E][H, I]                      */
  const void* s2;          /* nkm_pack_mxfp4 scales of down                                 */
  const void* b2;          /* bf16 [E][H]                                                   */
  int32_t sliding;         /* 1: sliding-window attention (window sliding_window)           */
} nkm_gptoss_layer;

typedef struct nkm_gptoss_desc {
  int32_t hidden;          /* H: multiple of 32, <= 4096 (2880)                              */
  int32_t hidden_actual;   /* RMSNorm mean over this many elements (rows padded with zeros
                              beyond it, rmsnorm_tkg.py:49-147 hidden_actual); 0 = hidden   */
  int32_t n_q_heads;       /* 64 */
  int32_t n_kv_heads;      /* 8  */
  int32_t head_dim;        /* must be 64 */
  int32_t n_experts;       /* <= 128 (32) */
  int32_t top_k;           /* <= 8 (4) */
  int32_t inter;           /* I: multiple of 32, <= 4096 (2880) */
  int32_t n_layers;
  int32_t vocab;           /* multiple of 16 (201088) */
  float rms_eps;           /* 1e-5 */
  float swiglu_limit;      /* 7.0: gate <= limit, up in [-limit, limit] */
  float swiglu_alpha;      /* 1.702 */
  int32_t sliding_window;  /* W (128): a sliding layer sees the last W-1 tokens and the new one */
  const nkm_gptoss_layer* layers;
  const void* final_norm;  /* bf16 [H] */
  const void* lm_head_ft;  /* bf16 FT [V, H] */
  const void* embed;       /* bf16 [V, H] */
  const float* rope_cos;   /* fp32 [rope_max_pos, 32] (YaRN, attention factor applied) */
  const float* rope_sin;
  int32_t rope_max_pos;
  void* k_pool;            /* bf16 [L][num_blocks][nkv][128 tokens][64]                     */
  void* v_pool;            /* bf16 [L][num_blocks][nkv][64][128 tokens] (blocks transposed) */
  int32_t num_blocks;
  int32_t block_size;      /* must be 128 */
  int32_t max_batch;       /* <= 16 */
  int32_t max_context;     /* longest context (tokens) any step will attend to */
  int32_t kv_fp8;          /* 1: K/V pools hold e4m3 bytes (same shapes): stored = e4m3(clip(x * scale,
                              +-240)), read = stored / scale (attention_block_tkg.py:213-218, 1694) */
  float k_scale;           /* used when kv_fp8 */
  float v_scale;
  /* Tensor + expert parallelism across the GPUs of one node (one process per GPU), as in
   * nkm_qwen3_desc.  n_ranks <= 1: the whole model on this GPU.  n_ranks > 1: n_q_heads and
   * n_kv_heads are this rank's heads (its KV-head group with their query heads; the layer's
   * wqkv/bqkv/wo/sinks hold those), and the expert tensors hold its experts [expert_begin,
   * expert_begin + n_local_experts) of n_experts (router, norms, embedding, LM head replicated).
   * After the O-projection and after the experts every rank stores its partial sums as tagged
   * 8-byte words into the exchange region of every rank (xchg[q]: each rank's region mapped in
   * this process, nkm_gptoss_xchg_bytes each, zeroed before the first step) and adds all ranks'
   * partials in rank order, so every rank keeps the same residual.  The LM head is split over
   * the vocabulary (rank r: 16-row strips [S r / n, S (r + 1) / n), S = vocab / 16) and every rank
   * returns the full logits.  Replaces the TP/EP sharding of gpt_oss_with_megakernel.py. */
  int32_t n_ranks;
  int32_t rank;
  int32_t expert_begin;
  int32_t n_local_experts;
  void* xchg[8];
} nkm_gptoss_desc;

typedef struct nkm_gptoss_step {
  int32_t batch;
  const int32_t* input_ids;    /* device [B] or NULL (then x_in) */
  const void* x_in;            /* device bf16 [B, H] */
  const int32_t* positions;    /* device [B] */
  const int32_t* block_table;  /* device [B, max_blocks_per_seq]; -1 at the write slot skips the write */
  int32_t max_blocks_per_seq;
  void* y_out;                 /* device bf16 [B, H] hidden after the last layer (pre final norm) */
  float* logits_out;           /* device fp32 [B, V] or NULL */
  int32_t first_layer;
  int32_t num_layers;          /* 0 = all */
  float* trace_qkv;            /* fp32 [nl, B, (nq+2nkv)*64] projections + bias, before RoPE */
  float* trace_resid_mid;      /* fp32 [nl, B, H] */
  float* trace_resid_out;      /* fp32 [nl, B, H] */
  float* trace_router_logits;  /* fp32 [nl, B, E] */
  int32_t* trace_topk_idx;     /* [nl, B, K] */
  float* trace_topk_w;         /* [nl, B, K] */
  int64_t* trace_stage_ns;     /* [2 + 10 nl + 1] or NULL: globaltimer of CTA 0 at kernel start, after
                                  every grid barrier (the input copy, then ten per layer) and at the end */
} nkm_gptoss_step;

typedef struct nkm_gptoss nkm_gptoss;

/* Workspace bytes of a GPT-OSS handle (caller allocates, 256-byte aligned). */
size_t nkm_gptoss_workspace_bytes(const nkm_gptoss_desc* desc);
/* Bytes of the exchange region each rank allocates when n_ranks > 1 (256-byte aligned, zeroed,
 * shared with the other ranks by CUDA IPC). */
size_t nkm_gptoss_xchg_bytes(const nkm_gptoss_desc* desc);
/* Replaces compile()/load() of the reference's GPT-OSS model (gpt_oss_with_megakernel.py). */
int nkm_gptoss_create(const nkm_gptoss_desc* desc, void* workspace, size_t workspace_bytes, nkm_gptoss** out);
void nkm_gptoss_destroy(nkm_gptoss* h);
/* One decode step, one cooperative launch.  Replaces
 * get_multilayer_kernel_jit(L, mxfp4)(X, Wqkv_*, bqkv_*, Wo_*, bo_*, Sink_*, ..., K_*, V_*, cos, sin,
 * position_ids, position_ids_window) (transformer_gpt_oss.py:540-636). */
int nkm_gptoss_decode_step(nkm_gptoss* h, const nkm_gptoss_step* step, nkm_stream_t stream);
/* Synchronise and return (and clear) the device status word.  With n_ranks > 1 a non-zero status
 * also clears this rank's exchange region and restarts its exchange sequence: after a failed step
 * every rank calls this once all ranks' launches have ended, then the group synchronises. */
int nkm_gptoss_status(nkm_gptoss* h, nkm_stream_t stream);

/* MXFP4 weight packer (load time).  codes: uint8 [count][rows][cols] e2m1 codes 0..15 (bit 3 sign;
 * Hugging Face's *_blocks unpacked low nibble first), scales: uint8 [count][rows][cols/32] e8m0.
 * dst_w receives count*rows*cols/2 bytes, dst_s nkm_mxfp4_scale_bytes(rows, cols, count) bytes
 * (per 16-row strip, groups of 8 k-tiles: 16 rows x 8 scales), in the kernel's tiled order.
 * rows % 16 == 0, cols % 32 == 0.  Replaces the MX layout conversion of
 * gpt_oss_with_megakernel.py:290-327 / selective_expert_mx_impl.py:60. */
int64_t nkm_mxfp4_scale_bytes(int64_t rows, int64_t cols, int64_t count);
int nkm_pack_mxfp4(const void* codes, const void* scales, void* dst_w, void* dst_s, int64_t rows, int64_t cols,
                   int64_t count, nkm_stream_t stream);

/* Message for the last error returned on this thread ("" if none). */
const char* nkm_last_error(void);

/* Library version string. */
const char* nkm_version(void);

#ifdef __cplusplus
}
#endif
#endif /* NKIMOE_H_ */
