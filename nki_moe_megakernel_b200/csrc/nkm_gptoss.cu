// Host side of the GPT-OSS decode path (C ABI in include/nkimoe.h): argument checks, workspace
// layout, the cooperative launch of the decode kernel and the MXFP4 weight packer.  No entry
// point allocates device memory.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "nkimoe.h"
#include "nkm_gptoss_kernel.cuh"

namespace nkm {
void set_last_error(const char* msg);
}

namespace {

int gfail(int code, const char* msg) {
  nkm::set_last_error(msg);
  return code;
}

#define NKG_CUDA(call)                                              \
  do {                                                              \
    cudaError_t e_ = (call);                                        \
    if (e_ != cudaSuccess) return gfail(NKM_ERR_CUDA, cudaGetErrorString(e_)); \
  } while (0)

constexpr size_t kAlign = 256;
size_t al(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

struct GLayout {
  size_t bar, status, xseq, layers, resid, part, qbuf, att_part, attn_out, rlogits, hbuf, ypair, total;
  int max_units;
};

int n_ranks_of(const nkm_gptoss_desc& d) { return d.n_ranks > 1 ? d.n_ranks : 1; }

// Exchange region: header, the partials as tagged words [2 kinds][2 slots][n_ranks][B][H], then
// (several ranks) the logits as tagged words [2 slots][B][V].
size_t xlog_offset(const nkm_gptoss_desc& d) {
  return al(static_cast<size_t>(nkg::kXchgHeader) +
            4 * static_cast<size_t>(n_ranks_of(d)) * d.max_batch * static_cast<size_t>(d.hidden) * 8);
}

int kc_for(int strips, int kt, int warps) {
  int kc = (warps + strips - 1) / strips;
  kc = kc < 1 ? 1 : (kc > nkg::kMaxKC ? nkg::kMaxKC : kc);
  return kc > kt ? kt : kc;
}

GLayout glayout(const nkm_gptoss_desc& d) {
  GLayout w{};
  const size_t B = d.max_batch, H = d.hidden, nq = d.n_q_heads, nkv = d.n_kv_heads;
  const size_t R = (nq + 2 * nkv) * nkg::kHD;
  w.max_units = static_cast<int>(B * nkv * (d.max_context / nkg::kBlk + 2));
  size_t o = 0;
  w.bar = 0;
  w.status = 16;
  w.xseq = 32;  // u32[3]: exchanges of each kind before the next launch (several ranks)
  o = 256;
  w.layers = o;
  o = al(o + sizeof(nkg::Layer) * d.n_layers);
  w.resid = o;
  o = al(o + B * H * 4);
  w.part = o;
  o = al(o + static_cast<size_t>(nkg::kMaxKC) * (R > H ? R : H) * B * 4);
  w.qbuf = o;
  o = al(o + B * nq * nkg::kHD * 2);
  w.att_part = o;
  o = al(o + static_cast<size_t>(w.max_units) * nkg::kMaxGrp * nkg::kPartStride * 4);
  w.attn_out = o;
  o = al(o + B * nq * nkg::kHD * 2);
  w.rlogits = o;
  o = al(o + B * d.n_experts * 4);
  w.hbuf = o;
  o = al(o + B * d.top_k * static_cast<size_t>(d.inter) * 2);
  w.ypair = o;
  o = al(o + B * d.top_k * H * 4);
  w.total = o;
  return w;
}

int gcheck(const nkm_gptoss_desc* d) {
  if (!d) return gfail(NKM_ERR_ARG, "desc is NULL");
  if (d->head_dim != nkg::kHD) return gfail(NKM_ERR_ARG, "head_dim must be 64");
  if (d->hidden <= 0 || d->hidden % 32 || d->hidden > nkg::kMaxHidden)
    return gfail(NKM_ERR_ARG, "hidden must be a positive multiple of 32 and at most 4096");
  if (d->hidden_actual < 0 || d->hidden_actual > d->hidden) return gfail(NKM_ERR_ARG, "hidden_actual outside 0..hidden");
  if (d->n_kv_heads <= 0 || d->n_q_heads <= 0 || d->n_q_heads % d->n_kv_heads ||
      d->n_q_heads / d->n_kv_heads > nkg::kMaxGrp)
    return gfail(NKM_ERR_ARG, "n_q_heads must be a multiple of n_kv_heads with at most 16 query heads per kv head");
  if (d->n_q_heads * nkg::kHD > nkg::kMaxHidden) return gfail(NKM_ERR_ARG, "n_q_heads * 64 must be at most 4096");
  if (d->n_experts <= 0 || d->n_experts > nkg::kMaxE) return gfail(NKM_ERR_ARG, "n_experts must be in 1..128");
  if (d->top_k <= 0 || d->top_k > nkg::kMaxTopK || d->top_k > d->n_experts) return gfail(NKM_ERR_ARG, "top_k must be in 1..8");
  if (d->inter <= 0 || d->inter % 32 || d->inter > nkg::kMaxHidden)
    return gfail(NKM_ERR_ARG, "inter must be a positive multiple of 32 and at most 4096");
  if (d->n_layers <= 0 || !d->layers) return gfail(NKM_ERR_ARG, "n_layers/layers invalid");
  if (d->vocab < 0 || d->vocab % 16) return gfail(NKM_ERR_ARG, "vocab must be a multiple of 16");
  if (d->max_batch <= 0 || d->max_batch > nkg::kMaxB) return gfail(NKM_ERR_ARG, "max_batch must be in 1..16");
  if (d->block_size != nkg::kBlk) return gfail(NKM_ERR_ARG, "block_size must be 128");
  if (d->max_context <= 0) return gfail(NKM_ERR_ARG, "max_context must be positive");
  if (d->sliding_window <= 0) return gfail(NKM_ERR_ARG, "sliding_window must be positive");
  if (d->kv_fp8 && !(d->k_scale > 0.f && d->v_scale > 0.f)) return gfail(NKM_ERR_ARG, "FP8 K/V needs positive scales");
  const int nr = n_ranks_of(*d);
  if (nr > 8) return gfail(NKM_ERR_ARG, "n_ranks must be in 1..8");
  if (d->rank < 0 || d->rank >= nr) return gfail(NKM_ERR_ARG, "rank outside 0..n_ranks-1");
  const int nle = d->n_local_experts > 0 ? d->n_local_experts : d->n_experts;
  if (d->expert_begin < 0 || d->expert_begin + nle > d->n_experts) return gfail(NKM_ERR_ARG, "local experts outside 0..n_experts");
  if (nr == 1 && (d->expert_begin != 0 || nle != d->n_experts)) return gfail(NKM_ERR_ARG, "a single rank holds every expert");
  if (nr > 1)
    for (int q = 0; q < nr; ++q)
      if (!d->xchg[q] || (reinterpret_cast<uintptr_t>(d->xchg[q]) & 255))
        return gfail(NKM_ERR_ARG, "xchg[q] must be a 256-byte aligned device pointer for every rank");
  return NKM_OK;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__global__ void pack_mxfp4_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                  uint8_t* __restrict__ dw, uint8_t* __restrict__ ds, int64_t rows, int64_t cols,
                                  int64_t count) {
  const int64_t KT = cols / 32, S = rows / 16;
  const int64_t nbytes = count * S * KT * 256;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nbytes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t unit = i / 256, byte = i % 256;
    const int64_t c = unit / (S * KT), rem = unit % (S * KT), s = rem / KT, kt = rem % KT;
    const int lane = static_cast<int>(byte / 8), j = static_cast<int>(byte % 8);
    const int64_t row = 16 * s + (lane >> 2) + (j >= 4 ? 8 : 0);
    const int64_t k = 32 * kt + 8 * (lane & 3) + 2 * (j & 3);
    const uint8_t* src = codes + (c * rows + row) * cols + k;
    dw[i] = static_cast<uint8_t>((src[0] & 15u) | ((src[1] & 15u) << 4));
    if (byte < 16 && kt % 8 == 0) {  // the 8 scales of row 16 s + byte for k-tiles kt .. kt + 7
      const int64_t srow = 16 * s + byte, G8 = (KT + 7) / 8;
      uint8_t* d8 = ds + ((c * S + s) * G8 + kt / 8) * 128 + byte * 8;
      for (int u = 0; u < 8; ++u) d8[u] = kt + u < KT ? scales[(c * rows + srow) * KT + kt + u] : 0;
    }
  }
}

}  // namespace

struct nkm_gptoss {
  nkm_gptoss_desc desc;
  std::vector<nkm_gptoss_layer> layers;
  uint8_t* ws;
  size_t ws_bytes;
  GLayout lay;
  int device, num_sms, kc_qkv, kc_o;
  size_t smem;
};

extern "C" {

size_t nkm_gptoss_workspace_bytes(const nkm_gptoss_desc* desc) {
  if (gcheck(desc) != NKM_OK) return 0;
  return glayout(*desc).total;
}

size_t nkm_gptoss_xchg_bytes(const nkm_gptoss_desc* desc) {
  if (gcheck(desc) != NKM_OK) return 0;
  const size_t logits = n_ranks_of(*desc) > 1 ? 2 * static_cast<size_t>(desc->max_batch) * desc->vocab * 8 : 0;
  return al(xlog_offset(*desc) + logits);
}

int nkm_gptoss_create(const nkm_gptoss_desc* desc, void* workspace, size_t workspace_bytes, nkm_gptoss** out) {
  if (!out) return gfail(NKM_ERR_ARG, "out is NULL");
  *out = nullptr;
  int rc = gcheck(desc);
  if (rc) return rc;
  const GLayout lay = glayout(*desc);
  if (!workspace || workspace_bytes < lay.total) return gfail(NKM_ERR_ARG, "workspace too small (nkm_gptoss_workspace_bytes)");
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign) return gfail(NKM_ERR_ARG, "workspace must be 256-byte aligned");
  for (int i = 0; i < desc->n_layers; ++i) {
    const nkm_gptoss_layer& L = desc->layers[i];
    const void* ps[] = {L.wqkv_ft, L.bqkv, L.wo_ft, L.bo, L.sinks, L.ln1, L.ln2, L.router, L.router_bias,
                        L.w13_fp4, L.s13, L.b13, L.w2_fp4, L.s2, L.b2};
    for (const void* q : ps)
      if (!q || !a16(q)) return gfail(NKM_ERR_ARG, "every layer tensor must be a 16-byte aligned device pointer");
  }
  int dev = 0, sms = 0;
  NKG_CUDA(cudaGetDevice(&dev));
  NKG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  nkm_gptoss* h = new (std::nothrow) nkm_gptoss();
  if (!h) return gfail(NKM_ERR_ARG, "out of host memory");
  h->desc = *desc;
  h->layers.assign(desc->layers, desc->layers + desc->n_layers);
  h->desc.layers = h->layers.data();
  h->ws = static_cast<uint8_t*>(workspace);
  h->ws_bytes = workspace_bytes;
  h->lay = lay;
  h->device = dev;
  h->num_sms = sms;
  const int R = (desc->n_q_heads + 2 * desc->n_kv_heads) * nkg::kHD;
  h->kc_qkv = kc_for(R / 16, desc->hidden / 32, sms * nkg::kWarps);
  h->kc_o = kc_for(desc->hidden / 16, desc->n_q_heads * nkg::kHD / 32, sms * nkg::kWarps);
  const int kx = std::max(std::max(desc->hidden, desc->n_q_heads * nkg::kHD), desc->inter);
  h->smem = nkg::Smem(nkg::kMaxB, kx).total;
  std::vector<nkg::Layer> lt(desc->n_layers);
  for (int i = 0; i < desc->n_layers; ++i) {
    const nkm_gptoss_layer& L = desc->layers[i];
    nkg::Layer& o = lt[i];
    o.wqkv = static_cast<const uint8_t*>(L.wqkv_ft);
    o.bqkv = static_cast<const uint16_t*>(L.bqkv);
    o.wo = static_cast<const uint8_t*>(L.wo_ft);
    o.bo = static_cast<const uint16_t*>(L.bo);
    o.sinks = static_cast<const uint16_t*>(L.sinks);
    o.ln1 = static_cast<const uint16_t*>(L.ln1);
    o.ln2 = static_cast<const uint16_t*>(L.ln2);
    o.router = static_cast<const uint16_t*>(L.router);
    o.router_b = static_cast<const uint16_t*>(L.router_bias);
    o.w13 = static_cast<const uint8_t*>(L.w13_fp4);
    o.s13 = static_cast<const uint8_t*>(L.s13);
    o.b13 = static_cast<const uint16_t*>(L.b13);
    o.w2 = static_cast<const uint8_t*>(L.w2_fp4);
    o.s2 = static_cast<const uint8_t*>(L.s2);
    o.b2 = static_cast<const uint16_t*>(L.b2);
    o.sliding = L.sliding ? 1 : 0;
  }
  auto cleanup = [&](int code) {
    delete h;
    return code;
  };
  if (cudaMemcpy(h->ws + lay.layers, lt.data(), sizeof(nkg::Layer) * lt.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(h->ws, 0, 256) != cudaSuccess)
    return cleanup(gfail(NKM_ERR_CUDA, "initialising the workspace failed"));
  if (h->smem > 232448 - 1024) return cleanup(gfail(NKM_ERR_ARG, "shared memory of this shape exceeds the limit"));
  if (cudaFuncSetAttribute(reinterpret_cast<void*>(&nkg::gptoss_decode_kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(nkg::Smem(nkg::kMaxB, nkg::kMaxHidden).total)) != cudaSuccess)
    return cleanup(gfail(NKM_ERR_CUDA, "cudaFuncSetAttribute failed"));
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reinterpret_cast<void*>(&nkg::gptoss_decode_kernel),
                                                    nkg::kThreads, h->smem) != cudaSuccess ||
      occ < 1)
    return cleanup(gfail(NKM_ERR_CUDA, "decode kernel does not fit on an SM"));
  *out = h;
  return NKM_OK;
}

void nkm_gptoss_destroy(nkm_gptoss* h) { delete h; }

int nkm_gptoss_decode_step(nkm_gptoss* h, const nkm_gptoss_step* s, nkm_stream_t stream) {
  if (!h || !s) return gfail(NKM_ERR_ARG, "handle or step is NULL");
  const nkm_gptoss_desc& d = h->desc;
  const int nl = s->num_layers > 0 ? s->num_layers : d.n_layers - s->first_layer;
  if (s->batch <= 0 || s->batch > d.max_batch) return gfail(NKM_ERR_ARG, "batch outside 1..max_batch");
  if (s->first_layer < 0 || nl <= 0 || s->first_layer + nl > d.n_layers) return gfail(NKM_ERR_ARG, "layer range out of bounds");
  if (!s->y_out || !a16(s->y_out)) return gfail(NKM_ERR_ARG, "y_out must be a 16-byte aligned device pointer");
  if (s->input_ids) {
    if (!d.embed || d.vocab <= 0) return gfail(NKM_ERR_ARG, "input_ids given but the model has no embedding table");
  } else if (!s->x_in || !a16(s->x_in)) {
    return gfail(NKM_ERR_ARG, "x_in must be a 16-byte aligned device pointer");
  }
  if (!d.k_pool || !d.v_pool || !d.rope_cos || !d.rope_sin) return gfail(NKM_ERR_ARG, "KV pools and RoPE tables are needed");
  if (!s->positions || !s->block_table || s->max_blocks_per_seq <= 0) return gfail(NKM_ERR_ARG, "positions and a block table are needed");
  if (static_cast<int64_t>(s->max_blocks_per_seq) * nkg::kBlk > static_cast<int64_t>(d.max_context) + nkg::kBlk)
    return gfail(NKM_ERR_ARG, "max_blocks_per_seq exceeds max_context / 128 + 1");
  const bool lm = s->logits_out != nullptr;
  if (lm && (d.vocab <= 0 || !d.lm_head_ft || !d.final_norm)) return gfail(NKM_ERR_ARG, "LM head requested but missing");
  nkg::Params p{};
  p.B = s->batch;
  p.H = d.hidden;
  p.Hact = d.hidden_actual > 0 ? d.hidden_actual : d.hidden;
  p.nq = d.n_q_heads;
  p.nkv = d.n_kv_heads;
  p.grp = d.n_q_heads / d.n_kv_heads;
  p.R = (d.n_q_heads + 2 * d.n_kv_heads) * nkg::kHD;
  p.E = d.n_experts;
  p.K = d.top_k;
  p.I = d.inter;
  p.L = d.n_layers;
  p.V = d.vocab;
  p.window = d.sliding_window;
  p.eps = d.rms_eps;
  p.kv_fp8 = d.kv_fp8 ? 1 : 0;
  p.k_scale = d.k_scale;
  p.v_scale = d.v_scale;
  p.limit = d.swiglu_limit;
  p.alpha = d.swiglu_alpha;
  p.kc_qkv = h->kc_qkv;
  p.kc_o = h->kc_o;
  p.first_layer = s->first_layer;
  p.num_layers = nl;
  p.want_lm = lm ? 1 : 0;
  p.layers = reinterpret_cast<const nkg::Layer*>(h->ws + h->lay.layers) + s->first_layer;
  p.final_norm = static_cast<const uint16_t*>(d.final_norm);
  p.lm_head = static_cast<const uint8_t*>(d.lm_head_ft);
  p.embed = static_cast<const uint16_t*>(d.embed);
  p.rope_cos = d.rope_cos;
  p.rope_sin = d.rope_sin;
  p.rope_max = d.rope_max_pos;
  p.k_pool = static_cast<uint16_t*>(d.k_pool);
  p.v_pool = static_cast<uint16_t*>(d.v_pool);
  p.num_blocks = d.num_blocks;
  p.input_ids = s->input_ids;
  p.x_in = static_cast<const uint16_t*>(s->x_in);
  p.positions = s->positions;
  p.block_table = s->block_table;
  p.max_blocks = s->max_blocks_per_seq;
  p.y_out = static_cast<uint16_t*>(s->y_out);
  p.logits_out = s->logits_out;
  p.tr_qkv = s->trace_qkv;
  p.tr_mid = s->trace_resid_mid;
  p.tr_out = s->trace_resid_out;
  p.tr_rlogits = s->trace_router_logits;
  p.tr_idx = s->trace_topk_idx;
  p.tr_w = s->trace_topk_w;
  p.tr_stage = s->trace_stage_ns;
  uint8_t* ws = h->ws;
  p.bar = reinterpret_cast<unsigned*>(ws + h->lay.bar);
  p.status = reinterpret_cast<int*>(ws + h->lay.status);
  p.resid = reinterpret_cast<float*>(ws + h->lay.resid);
  p.part = reinterpret_cast<float*>(ws + h->lay.part);
  p.qbuf = reinterpret_cast<uint16_t*>(ws + h->lay.qbuf);
  p.att_part = reinterpret_cast<float*>(ws + h->lay.att_part);
  p.attn_out = reinterpret_cast<uint16_t*>(ws + h->lay.attn_out);
  p.rlogits = reinterpret_cast<float*>(ws + h->lay.rlogits);
  p.hbuf = reinterpret_cast<uint16_t*>(ws + h->lay.hbuf);
  p.ypair = reinterpret_cast<float*>(ws + h->lay.ypair);
  p.n_ranks = n_ranks_of(d);
  p.rank = p.n_ranks > 1 ? d.rank : 0;
  p.expert_begin = d.expert_begin;
  p.n_local = d.n_local_experts > 0 ? d.n_local_experts : d.n_experts;
  for (int q = 0; q < 8; ++q) p.xchg[q] = q < p.n_ranks && p.n_ranks > 1 ? static_cast<uint8_t*>(d.xchg[q]) : nullptr;
  p.xseq = reinterpret_cast<unsigned*>(ws + h->lay.xseq);
  p.xlog_off = static_cast<int64_t>(xlog_offset(d));
  {  // the vocabulary's 16-row strips split evenly over the ranks
    const int vs = d.vocab / 16;
    p.lm_s0 = static_cast<int>(static_cast<int64_t>(vs) * p.rank / p.n_ranks);
    p.lm_ns = static_cast<int>(static_cast<int64_t>(vs) * (p.rank + 1) / p.n_ranks) - p.lm_s0;
  }
  void* args[1] = {&p};
  NKG_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(&nkg::gptoss_decode_kernel), dim3(h->num_sms),
                                       dim3(nkg::kThreads), args, h->smem, reinterpret_cast<cudaStream_t>(stream)));
  return NKM_OK;
}

int nkm_gptoss_status(nkm_gptoss* h, nkm_stream_t stream) {
  if (!h) return gfail(NKM_ERR_ARG, "handle is NULL");
  int st = 0;
  NKG_CUDA(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  NKG_CUDA(cudaMemcpy(&st, h->ws + h->lay.status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) {
    gfail(st, (st & NKM_ERR_TIMEOUT) ? "device status: wait timeout" : "device status: index out of range");
    NKG_CUDA(cudaMemset(h->ws, 0, 256));  // barrier, status and the exchange sequence
    if (n_ranks_of(h->desc) > 1) {
      NKG_CUDA(cudaMemset(h->desc.xchg[h->desc.rank], 0, nkm_gptoss_xchg_bytes(&h->desc)));
      NKG_CUDA(cudaDeviceSynchronize());
    }
  }
  return st;
}

int64_t nkm_mxfp4_scale_bytes(int64_t rows, int64_t cols, int64_t count) {
  if (rows <= 0 || rows % 16 || cols <= 0 || cols % 32 || count <= 0) return 0;
  return count * (rows / 16) * ((cols / 32 + 7) / 8) * 128;
}

int nkm_pack_mxfp4(const void* codes, const void* scales, void* dst_w, void* dst_s, int64_t rows, int64_t cols,
                   int64_t count, nkm_stream_t stream) {
  if (!codes || !scales || !dst_w || !dst_s) return gfail(NKM_ERR_ARG, "NULL pointer");
  if (rows <= 0 || rows % 16 || cols <= 0 || cols % 32 || count <= 0)
    return gfail(NKM_ERR_ARG, "rows must be a multiple of 16 and cols a multiple of 32");
  const int64_t n = count * (rows / 16) * (cols / 32) * 256;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8192));
  pack_mxfp4_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(codes), static_cast<const uint8_t*>(scales), static_cast<uint8_t*>(dst_w),
      static_cast<uint8_t*>(dst_s), rows, cols, count);
  NKG_CUDA(cudaGetLastError());
  return NKM_OK;
}

}  // extern "C"
