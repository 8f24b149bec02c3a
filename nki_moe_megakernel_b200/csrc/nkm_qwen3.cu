// Host side of the C ABI declared in include/nkimoe.h: argument checks, workspace layout,
// K/V tensor-map encoding, the cooperative launch of the decode kernel and the weight
// packer.  No entry point allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "nkimoe.h"
#include "nkm_qwen3_kernel.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define NKM_CUDA(call)                                                                         \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) return fail(NKM_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Exchange region of a rank: the barrier counter (kXchgHeader bytes), the O-projection and expert
// partials as tagged 8-byte words [2 kinds][2 slots][n_ranks][max_batch][hidden], then (several
// ranks) the logits [max_batch][vocab] fp32 that the vocabulary-sharded LM head fills on every rank.
size_t xlog_offset(const nkm_qwen3_desc& d) {
  const size_t nr = d.n_ranks > 0 ? static_cast<size_t>(d.n_ranks) : 1;
  return align_up(static_cast<size_t>(nkm::kXchgHeader) +
                  4 * nr * static_cast<size_t>(d.max_batch) * static_cast<size_t>(d.hidden) * 8);
}

// Workspace layout (offsets in bytes from the workspace base).
struct WsLayout {
  size_t ctrl, ctrl_bytes;  // bar, status, strip/attn/row counters (zeroed every step)
  size_t bar, status, gbase, xseq, strip_cnt, attn_cnt, row_cnt;
  size_t layers, resid, qkv, attn_out, att_part, rlogits, hbuf, ypair, gpart;
  size_t total;
};

constexpr int kMaxStrips = 16384;

WsLayout layout_ws(const nkm_qwen3_desc& d, int num_sms) {
  WsLayout w{};
  const size_t Tm = static_cast<size_t>(d.max_batch);
  const size_t NW = static_cast<size_t>(num_sms) * nkm::kWarps;
  const size_t R = static_cast<size_t>(d.n_q_heads + 2 * d.n_kv_heads) * d.head_dim;
  size_t o = 0;
  w.ctrl = o;
  w.bar = o;
  w.status = o + 16;  // bar[0] = barrier arrival count, bar[2] = CTAs that left the launch
  w.gbase = o + 24;   // u64: cross-GPU barrier count before the next launch
  w.xseq = o + 32;    // u32[2]: partial exchanges of each kind before the next launch
  w.strip_cnt = o + 256;
  w.attn_cnt = w.strip_cnt + kMaxStrips * 4;
  w.row_cnt = w.attn_cnt + align_up(Tm * d.n_kv_heads * 4);
  w.ctrl_bytes = align_up(w.row_cnt - o + static_cast<size_t>(d.hidden / 16) * 4);
  o = align_up(o + w.ctrl_bytes);
  w.layers = o;
  o = align_up(o + sizeof(nkm::LayerPtrs) * d.n_layers);
  w.resid = o;
  o = align_up(o + Tm * d.hidden * 4);
  w.qkv = o;
  o = align_up(o + Tm * R * 2);
  w.attn_out = o;
  o = align_up(o + Tm * d.n_q_heads * d.head_dim * 2);
  w.att_part = o;
  o = align_up(o + (NW + Tm * d.n_kv_heads) * nkm::kPartFloats * 4);  // items <= kAttItemsWide per CTA < kWarps
  w.rlogits = o;
  o = align_up(o + Tm * d.n_experts * 4);
  w.hbuf = o;
  o = align_up(o + Tm * d.top_k * d.moe_inter * 2);
  w.ypair = o;
  o = align_up(o + Tm * d.top_k * d.hidden * 4);
  w.gpart = o;
  o = align_up(o + NW * 2 * 4 * 32 * 4 * 4);
  w.total = o;
  return w;
}

int nt_for_batch(int T) { return T <= 8 ? 1 : (T <= 16 ? 2 : 4); }

int check_desc(const nkm_qwen3_desc* d) {
  if (!d) return fail(NKM_ERR_ARG, "desc is NULL");
  if (d->head_dim != nkm::kHeadDim) return fail(NKM_ERR_ARG, "head_dim must be 128 (got %d)", d->head_dim);
  if (d->hidden <= 0 || d->hidden % 256 || d->hidden > nkm::kMaxHidden)
    return fail(NKM_ERR_ARG, "hidden must be a positive multiple of 256 and at most %d", nkm::kMaxHidden);
  if (d->n_kv_heads <= 0 || d->n_q_heads <= 0 || d->n_q_heads % d->n_kv_heads)
    return fail(NKM_ERR_ARG, "n_q_heads must be a positive multiple of n_kv_heads");
  if (d->n_q_heads / d->n_kv_heads > nkm::kAttRows)
    return fail(NKM_ERR_ARG, "at most %d query heads per kv head", nkm::kAttRows);
  if (d->n_experts <= 0 || d->n_experts > nkm::kMaxExperts) return fail(NKM_ERR_ARG, "n_experts must be in 1..256");
  if (d->top_k <= 0 || d->top_k > 8 || d->top_k > d->n_experts) return fail(NKM_ERR_ARG, "top_k must be in 1..8");
  if (d->moe_inter <= 0 || d->moe_inter % 32) return fail(NKM_ERR_ARG, "moe_inter must be a multiple of 32");
  if (d->n_layers <= 0 || !d->layers) return fail(NKM_ERR_ARG, "n_layers/layers invalid");
  if (d->vocab < 0 || d->vocab % 16) return fail(NKM_ERR_ARG, "vocab must be a multiple of 16");
  if (d->max_batch <= 0 || d->max_batch > 32) return fail(NKM_ERR_ARG, "max_batch must be in 1..32");
  if (d->max_batch * d->top_k > nkm::kMaxPairs) return fail(NKM_ERR_ARG, "max_batch*top_k too large");
  if (d->block_size != nkm::kKvBlock) return fail(NKM_ERR_ARG, "block_size must be 128");
  const int nr = d->n_ranks > 0 ? d->n_ranks : 1;
  if (nr > nkm::kMaxRanks) return fail(NKM_ERR_ARG, "n_ranks must be in 1..%d", nkm::kMaxRanks);
  if (d->rank < 0 || d->rank >= nr) return fail(NKM_ERR_ARG, "rank %d outside 0..%d", d->rank, nr - 1);
  const int nle = d->n_local_experts > 0 ? d->n_local_experts : d->n_experts;
  if (d->expert_begin < 0 || d->expert_begin + nle > d->n_experts)
    return fail(NKM_ERR_ARG, "local experts [%d, %d) outside 0..%d", d->expert_begin, d->expert_begin + nle, d->n_experts);
  if (nr == 1 && (d->expert_begin != 0 || nle != d->n_experts))
    return fail(NKM_ERR_ARG, "a single rank holds every expert");
  if (nr > 1)
    for (int q = 0; q < nr; ++q)
      if (!d->xchg[q] || (reinterpret_cast<uintptr_t>(d->xchg[q]) & 255))
        return fail(NKM_ERR_ARG, "xchg[%d] must be a 256-byte aligned device pointer", q);
  // every GEMV stage indexes one split-K counter per 16-row strip
  const int64_t na_max = std::min<int64_t>(d->n_experts, static_cast<int64_t>(d->max_batch) * d->top_k);
  const int64_t strips[] = {na_max * (2 * d->moe_inter / 16), na_max * (d->hidden / 16), d->vocab / 16,
                            static_cast<int64_t>(d->n_q_heads + 2 * d->n_kv_heads) * d->head_dim / 16};
  for (int64_t s : strips)
    if (s > kMaxStrips) return fail(NKM_ERR_ARG, "shape needs %lld split-K counters (max %d)", (long long)s, kMaxStrips);
  return NKM_OK;
}

int current_sms(int* sms, int* dev) {
  NKM_CUDA(cudaGetDevice(dev));
  NKM_CUDA(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, *dev));
  return NKM_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// K or V pool viewed as a 2-D tensor [rows = L*NB*nkv*128, 128] bf16; box 64 x 32 (128-byte
// inner extent, 128-byte swizzle).
int encode_kv_map(CUtensorMap* map, void* pool, const nkm_qwen3_desc& d) {
  memset(map, 0, sizeof(*map));
  if (!pool) return NKM_OK;
  auto enc = tensor_map_encoder();
  if (!enc) return fail(NKM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const uint64_t rows = static_cast<uint64_t>(d.n_layers) * d.num_blocks * d.n_kv_heads * nkm::kKvBlock;
  if (rows >= (1ull << 31)) return fail(NKM_ERR_ARG, "KV pool too large for 32-bit TMA coordinates");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(nkm::kHeadDim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(nkm::kHeadDim * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(nkm::kAttTile)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, pool, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NKM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return NKM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The instantiations of the decode kernel: column tiles NT = 1, 2, 4 for the decode step, and
// NT = 1 and 4 with the caller-q/k/v and K/V-first stage bits (kExt; batches of 9..16 run on the
// NT = 4 one).
constexpr int kNumKernels = 5;
void* decode_kernel_fn(int i) {
  void* kfn[kNumKernels] = {reinterpret_cast<void*>(&nkm::qwen3_decode_kernel<1, false>),
                            reinterpret_cast<void*>(&nkm::qwen3_decode_kernel<2, false>),
                            reinterpret_cast<void*>(&nkm::qwen3_decode_kernel<4, false>),
                            reinterpret_cast<void*>(&nkm::qwen3_decode_kernel<1, true>),
                            reinterpret_cast<void*>(&nkm::qwen3_decode_kernel<4, true>)};
  return kfn[i];
}
constexpr int kNts[kNumKernels] = {1, 2, 4, 1, 4};
constexpr int kMaxDevices = 64;

// Once per device, with that device current: the decode kernel's dynamic shared-memory limit.
// The attribute belongs to the kernel for the whole process, so it is set to what the largest
// accepted hidden size needs (not to one handle's size: a handle with a smaller hidden size would
// otherwise lower it under the launches of a handle with a larger one); every launch still
// requests only its own size.
int ensure_smem_limits() {
  static std::mutex mu;
  static bool done[kMaxDevices] = {};
  int dev = 0;
  NKM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(NKM_ERR_ARG, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return NKM_OK;
  for (int i = 0; i < kNumKernels; ++i) {
    const nkm::SmemLayout sl(nkm::kMaxHidden, kNts[i]);
    if (sl.total > 232448 - 1024) return fail(NKM_ERR_ARG, "decode kernel shared memory exceeds the per-CTA limit");
    NKM_CUDA(cudaFuncSetAttribute(decode_kernel_fn(i), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(sl.total)));
  }
  done[dev] = true;
  return NKM_OK;
}

}  // namespace

namespace nkm {
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace nkm

struct nkm_qwen3 {
  nkm_qwen3_desc desc;
  std::vector<nkm_qwen3_layer> layers;
  uint8_t* ws;
  size_t ws_bytes;
  WsLayout lay;
  CUtensorMap kmap, vmap;
  int device, num_sms;
  size_t smem[kNumKernels];
};

extern "C" {

const char* nkm_last_error(void) { return g_last_error.c_str(); }
const char* nkm_version(void) { return "nkimoe-b200 0.1.0 (sm_100a)"; }

size_t nkm_qwen3_workspace_bytes(const nkm_qwen3_desc* desc) {
  if (check_desc(desc) != NKM_OK) return 0;
  int sms = 0, dev = 0;
  if (current_sms(&sms, &dev) != NKM_OK) return 0;
  return layout_ws(*desc, sms).total;
}

size_t nkm_qwen3_xchg_bytes(const nkm_qwen3_desc* desc) {
  if (check_desc(desc) != NKM_OK) return 0;
  const size_t nr = desc->n_ranks > 0 ? static_cast<size_t>(desc->n_ranks) : 1;
  return align_up(xlog_offset(*desc) +
                  (nr > 1 ? static_cast<size_t>(desc->max_batch) * static_cast<size_t>(desc->vocab) * 4 : 0));
}

int nkm_qwen3_create(const nkm_qwen3_desc* desc, void* workspace, size_t workspace_bytes, nkm_qwen3** out) {
  if (!out) return fail(NKM_ERR_ARG, "out is NULL");
  *out = nullptr;
  int rc = check_desc(desc);
  if (rc) return rc;
  int sms = 0, dev = 0;
  if ((rc = current_sms(&sms, &dev))) return rc;
  WsLayout lay = layout_ws(*desc, sms);
  if (!workspace || workspace_bytes < lay.total)
    return fail(NKM_ERR_ARG, "workspace too small: need %zu bytes", lay.total);
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign) return fail(NKM_ERR_ARG, "workspace must be 256-byte aligned");
  for (int i = 0; i < desc->n_layers; ++i) {
    const nkm_qwen3_layer& L = desc->layers[i];
    const void* ps[] = {L.wqkv_ft, L.wo_ft, L.w13_ft, L.w2_ft, L.router, L.ln1, L.ln2, L.q_norm, L.k_norm};
    for (const void* q : ps)
      if (q && !aligned16(q)) return fail(NKM_ERR_ARG, "layer %d: weight pointers must be 16-byte aligned", i);
  }
  nkm_qwen3* h = new (std::nothrow) nkm_qwen3();
  if (!h) return fail(NKM_ERR_ARG, "out of host memory");
  h->desc = *desc;
  h->layers.assign(desc->layers, desc->layers + desc->n_layers);
  h->desc.layers = h->layers.data();
  h->ws = static_cast<uint8_t*>(workspace);
  h->ws_bytes = workspace_bytes;
  h->lay = lay;
  h->device = dev;
  h->num_sms = sms;
  std::vector<nkm::LayerPtrs> lp(desc->n_layers);
  for (int i = 0; i < desc->n_layers; ++i) {
    const nkm_qwen3_layer& L = desc->layers[i];
    lp[i] = nkm::LayerPtrs{static_cast<const uint8_t*>(L.wqkv_ft), static_cast<const uint8_t*>(L.wo_ft),
                           static_cast<const uint16_t*>(L.q_norm),  static_cast<const uint16_t*>(L.k_norm),
                           static_cast<const uint16_t*>(L.ln1),     static_cast<const uint16_t*>(L.ln2),
                           static_cast<const uint16_t*>(L.router),  static_cast<const uint8_t*>(L.w13_ft),
                           static_cast<const uint8_t*>(L.w2_ft),    L.router_bias};
  }
  auto cleanup = [&](int code) {
    delete h;
    return code;
  };
  if (cudaMemcpy(h->ws + lay.layers, lp.data(), sizeof(nkm::LayerPtrs) * lp.size(), cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return cleanup(fail(NKM_ERR_CUDA, "copying the layer table failed"));
  if (cudaMemset(h->ws + lay.ctrl, 0, lay.ctrl_bytes) != cudaSuccess)
    return cleanup(fail(NKM_ERR_CUDA, "clearing the workspace failed"));
  if ((rc = encode_kv_map(&h->kmap, desc->k_pool, *desc))) return cleanup(rc);
  if ((rc = encode_kv_map(&h->vmap, desc->v_pool, *desc))) return cleanup(rc);
  if ((rc = ensure_smem_limits())) return cleanup(rc);
  for (int i = 0; i < kNumKernels; ++i) {
    nkm::SmemLayout sl(desc->hidden, kNts[i]);
    h->smem[i] = sl.total;
    if (sl.total > 232448 - 1024) return cleanup(fail(NKM_ERR_ARG, "hidden too large for shared memory"));
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel_fn(i), nkm::kThreads, sl.total) !=
            cudaSuccess ||
        occ < 1)
      return cleanup(fail(NKM_ERR_CUDA, "decode kernel does not fit on an SM"));
  }
  *out = h;
  g_last_error.clear();
  return NKM_OK;
}

void nkm_qwen3_destroy(nkm_qwen3* h) { delete h; }

static int launch_step(nkm_qwen3* h, const nkm_qwen3_step* s, int first, int nl, int stages, int residual,
                       cudaStream_t stream) {
  const nkm_qwen3_desc& d = h->desc;
  if (!s) return fail(NKM_ERR_ARG, "step is NULL");
  if (s->batch <= 0 || s->batch > d.max_batch) return fail(NKM_ERR_ARG, "batch %d outside 1..%d", s->batch, d.max_batch);
  if (first < 0 || nl <= 0 || first + nl > d.n_layers) return fail(NKM_ERR_ARG, "layer range out of bounds");
  if (nl > nkm::kMaxLaunchLayers) return fail(NKM_ERR_ARG, "at most %d layers per step", nkm::kMaxLaunchLayers);
  if (!s->y_out || !aligned16(s->y_out)) return fail(NKM_ERR_ARG, "y_out must be a 16-byte aligned device pointer");
  if (s->input_ids) {
    if (!d.embed || d.vocab <= 0) return fail(NKM_ERR_ARG, "input_ids given but the model has no embedding table");
  } else if (!s->x_in || !aligned16(s->x_in)) {
    return fail(NKM_ERR_ARG, "x_in must be a 16-byte aligned device pointer");
  }
  if (stages & NKM_STAGE_ATTN) {
    if (!d.k_pool || !d.v_pool || !d.rope_cos || !d.rope_sin) return fail(NKM_ERR_ARG, "attention needs KV pools and RoPE tables");
    if (!s->positions || !s->block_table || s->max_blocks_per_seq <= 0)
      return fail(NKM_ERR_ARG, "attention needs positions and a block table");
    for (int l = first; l < first + nl; ++l) {
      const nkm_qwen3_layer& L = d.layers[l];
      if (!L.wqkv_ft || !L.wo_ft || !L.q_norm || !L.k_norm || !L.ln1)
        return fail(NKM_ERR_ARG, "layer %d: attention weights missing", l);
    }
  }
  if (stages & NKM_STAGE_MOE) {
    for (int l = first; l < first + nl; ++l) {
      const nkm_qwen3_layer& L = d.layers[l];
      if (!L.router || !L.w13_ft || !L.w2_ft || !L.ln2) return fail(NKM_ERR_ARG, "layer %d: MoE weights missing", l);
    }
  }
  const bool lm = (stages & NKM_STAGE_LMHEAD) && s->logits_out;
  if (lm && (d.vocab <= 0 || !d.lm_head_ft || !d.final_norm)) return fail(NKM_ERR_ARG, "LM head requested but missing");
  if ((stages & NKM_STAGE_QKV_IN) && (!(stages & NKM_STAGE_ATTN) || nl != 1))
    return fail(NKM_ERR_ARG, "NKM_STAGE_QKV_IN needs the attention stage and exactly one layer");
  if ((stages & NKM_STAGE_KV_FIRST) && s->trace_stage_ns)
    return fail(NKM_ERR_ARG, "stage timestamps are not recorded with NKM_STAGE_KV_FIRST");

  nkm::Params p{};
  p.T = s->batch;
  p.H = d.hidden;
  p.nq = d.n_q_heads;
  p.nkv = d.n_kv_heads;
  p.grp = d.n_q_heads / d.n_kv_heads;
  p.R = (d.n_q_heads + 2 * d.n_kv_heads) * d.head_dim;
  p.E = d.n_experts;
  p.K = d.top_k;
  p.I = d.moe_inter;
  p.L = d.n_layers;
  p.V = d.vocab;
  p.eps = d.rms_eps;
  p.n_ranks = d.n_ranks > 0 ? d.n_ranks : 1;
  p.rank = d.rank;
  p.expert_begin = d.expert_begin;
  p.n_local = d.n_local_experts > 0 ? d.n_local_experts : d.n_experts;
  for (int q = 0; q < nkm::kMaxRanks; ++q) p.xchg[q] = q < p.n_ranks ? static_cast<uint8_t*>(d.xchg[q]) : nullptr;
  p.gbase = reinterpret_cast<unsigned long long*>(h->ws + h->lay.gbase);
  p.xseq = reinterpret_cast<unsigned*>(h->ws + h->lay.xseq);
  // the vocabulary's 16-row strips split evenly over the ranks
  const int vs = d.vocab / 16;
  p.lm_s0 = static_cast<int>(static_cast<int64_t>(vs) * p.rank / p.n_ranks);
  p.lm_ns = static_cast<int>(static_cast<int64_t>(vs) * (p.rank + 1) / p.n_ranks) - p.lm_s0;
  p.xlog_off = static_cast<int64_t>(xlog_offset(d));
  p.first_layer = first;
  p.num_layers = nl;
  p.stages = stages & (NKM_STAGE_ATTN | NKM_STAGE_MOE | NKM_STAGE_QKV_IN | NKM_STAGE_KV_FIRST |
                       (lm ? NKM_STAGE_LMHEAD : 0));
  p.residual = residual;
  p.layers = reinterpret_cast<const nkm::LayerPtrs*>(h->ws + h->lay.layers);
  p.final_norm = static_cast<const uint16_t*>(d.final_norm);
  p.lm_head = static_cast<const uint8_t*>(d.lm_head_ft);
  p.embed = static_cast<const uint16_t*>(d.embed);
  p.rope_cos = static_cast<const uint16_t*>(d.rope_cos);
  p.rope_sin = static_cast<const uint16_t*>(d.rope_sin);
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
  p.logits_out = lm ? s->logits_out : nullptr;
  p.tr_topk_idx = s->trace_topk_idx;
  p.tr_topk_w = s->trace_topk_w;
  p.tr_rlogits = s->trace_router_logits;
  p.tr_qkv = static_cast<uint16_t*>(s->trace_qkv);
  p.tr_mid = s->trace_resid_mid;
  p.tr_out = s->trace_resid_out;
  p.tr_stage = s->trace_stage_ns;
  uint8_t* ws = h->ws;
  p.bar = reinterpret_cast<unsigned*>(ws + h->lay.bar);
  p.status = reinterpret_cast<int*>(ws + h->lay.status);
  p.strip_cnt = reinterpret_cast<unsigned*>(ws + h->lay.strip_cnt);
  p.attn_cnt = reinterpret_cast<unsigned*>(ws + h->lay.attn_cnt);
  p.row_cnt = reinterpret_cast<unsigned*>(ws + h->lay.row_cnt);
  p.resid = reinterpret_cast<float*>(ws + h->lay.resid);
  p.qkv = reinterpret_cast<uint16_t*>(ws + h->lay.qkv);
  p.attn_out = reinterpret_cast<uint16_t*>(ws + h->lay.attn_out);
  p.att_part = reinterpret_cast<float*>(ws + h->lay.att_part);
  p.rlogits = reinterpret_cast<float*>(ws + h->lay.rlogits);
  p.hbuf = reinterpret_cast<uint16_t*>(ws + h->lay.hbuf);
  p.ypair = reinterpret_cast<float*>(ws + h->lay.ypair);
  p.gpart = reinterpret_cast<float*>(ws + h->lay.gpart);

  const int nt = nt_for_batch(p.T);
  // the extended kernels also carry the exchange of a group of several ranks: the single-GPU
  // decode kernels stay free of that code
  const bool ext = (stages & (NKM_STAGE_QKV_IN | NKM_STAGE_KV_FIRST)) != 0 || p.n_ranks > 1;
  const int ki = ext ? (nt == 1 ? 3 : 4) : (nt == 1 ? 0 : (nt == 2 ? 1 : 2));
  void* args[3] = {&p, &h->kmap, &h->vmap};
  NKM_CUDA(cudaLaunchCooperativeKernel(decode_kernel_fn(ki), dim3(h->num_sms), dim3(nkm::kThreads), args, h->smem[ki],
                                       stream));
  return NKM_OK;
}

int nkm_qwen3_decode_step(nkm_qwen3* h, const nkm_qwen3_step* s, nkm_stream_t stream) {
  if (!h) return fail(NKM_ERR_ARG, "handle is NULL");
  if (!s) return fail(NKM_ERR_ARG, "step is NULL");
  const int nl = s->num_layers > 0 ? s->num_layers : h->desc.n_layers - s->first_layer;
  // stage bits 1, 2, 4 select stages (none: all three); bits 8, 16 modify the attention stage
  const int sel = s->stages & (NKM_STAGE_ATTN | NKM_STAGE_MOE | NKM_STAGE_LMHEAD);
  const int stages = (sel ? sel : (NKM_STAGE_ATTN | NKM_STAGE_MOE | NKM_STAGE_LMHEAD)) |
                     (s->stages & (NKM_STAGE_QKV_IN | NKM_STAGE_KV_FIRST));
  return launch_step(h, s, s->first_layer, nl, stages, 1, reinterpret_cast<cudaStream_t>(stream));
}

int nkm_qwen3_attention_block(nkm_qwen3* h, int32_t layer, const nkm_qwen3_step* s, nkm_stream_t stream) {
  if (!h) return fail(NKM_ERR_ARG, "handle is NULL");
  if (!s) return fail(NKM_ERR_ARG, "step is NULL");
  return launch_step(h, s, layer, 1, NKM_STAGE_ATTN | (s->stages & (NKM_STAGE_QKV_IN | NKM_STAGE_KV_FIRST)),
                     s->residual ? 1 : 0, reinterpret_cast<cudaStream_t>(stream));
}

int nkm_qwen3_qkv_buffer(nkm_qwen3* h, void** ptr, size_t* bytes) {
  if (!h || !ptr) return fail(NKM_ERR_ARG, "handle or ptr is NULL");
  *ptr = h->ws + h->lay.qkv;
  if (bytes)
    *bytes = static_cast<size_t>(h->desc.max_batch) * (h->desc.n_q_heads + 2 * h->desc.n_kv_heads) * h->desc.head_dim * 2;
  return NKM_OK;
}

int nkm_qwen3_moe_block(nkm_qwen3* h, int32_t layer, const nkm_qwen3_step* s, nkm_stream_t stream) {
  if (!h) return fail(NKM_ERR_ARG, "handle is NULL");
  if (!s) return fail(NKM_ERR_ARG, "step is NULL");
  return launch_step(h, s, layer, 1, NKM_STAGE_MOE, s->residual ? 1 : 0, reinterpret_cast<cudaStream_t>(stream));
}

int nkm_qwen3_status(nkm_qwen3* h, nkm_stream_t stream) {
  if (!h) return fail(NKM_ERR_ARG, "handle is NULL");
  int st = 0;
  NKM_CUDA(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  NKM_CUDA(cudaMemcpy(&st, h->ws + h->lay.status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) {
    fail(st, "device status 0x%x%s%s", st, (st & NKM_ERR_TIMEOUT) ? " (wait timeout)" : "",
         (st & NKM_ERR_INDEX) ? " (index out of range)" : "");
    // the status is sticky until read; after a fault the barrier and counters may be mid-way
    // (with several ranks, every rank calls this before the group continues)
    NKM_CUDA(cudaMemset(h->ws + h->lay.ctrl, 0, h->lay.ctrl_bytes));
    // the exchange sequence restarts with the cleared control words: clear the tagged partials too
    if (h->desc.n_ranks > 1) {
      NKM_CUDA(cudaMemset(h->desc.xchg[h->desc.rank], 0, nkm_qwen3_xchg_bytes(&h->desc)));
      NKM_CUDA(cudaDeviceSynchronize());
    }
  }
  return st;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// MoE block without a handle or workspace, for callers that may not allocate device memory.
// Its scratch is the static array below (one per device that loads the library); the
// address of the calling device's copy is looked up once per device, on the first call.
// ---------------------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[NKM_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxNoAllocDevices = 64;

struct NoAllocDevice {
  uint8_t* scratch;  // device address of this device's g_noalloc_scratch
  int num_sms;
  CUcontext ctx;     // the context the address was looked up in
};

// cuCtxGetCurrent through the runtime's driver entry point (the library links no libcuda).
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  }
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kMaxNoAllocDevices];

// Scratch layout of one MoE-block call of batch T: the control words of the decode
// kernel (barrier, status, split-K strip counters, attention and row counters), the layer
// pointer table, then the MoE block's buffers.  The attention buffers are not needed.
struct NoAllocLayout {
  size_t bar, status, strip_cnt, attn_cnt, row_cnt, ctrl_bytes;
  size_t layers, resid, rlogits, hbuf, ypair, gpart, total;
};

NoAllocLayout layout_noalloc(const nkm_qwen3_desc& d, int T, int num_sms) {
  NoAllocLayout w{};
  const size_t Tm = static_cast<size_t>(T);
  const size_t NW = static_cast<size_t>(num_sms) * nkm::kWarps;
  w.bar = 0;
  w.status = 16;
  w.strip_cnt = 256;
  w.attn_cnt = w.strip_cnt + kMaxStrips * 4;
  w.row_cnt = w.attn_cnt + align_up(Tm * d.n_kv_heads * 4);
  w.ctrl_bytes = align_up(w.row_cnt + static_cast<size_t>(d.hidden / 16) * 4);
  size_t o = w.ctrl_bytes;
  w.layers = o;
  o = align_up(o + sizeof(nkm::LayerPtrs) * d.n_layers);
  w.resid = o;
  o = align_up(o + Tm * d.hidden * 4);
  w.rlogits = o;
  o = align_up(o + Tm * d.n_experts * 4);
  w.hbuf = o;
  o = align_up(o + Tm * d.top_k * d.moe_inter * 2);
  w.ypair = o;
  o = align_up(o + Tm * d.top_k * d.hidden * 4);
  w.gpart = o;
  o = align_up(o + NW * 2 * 4 * 32 * 4 * 4);
  w.total = o;
  return w;
}

// Once per device (and again if the device's context was replaced, e.g. after a device reset),
// with that device current: the address of its scratch array.
int noalloc_device(NoAllocDevice* out) {
  int dev = 0;
  NKM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxNoAllocDevices) return fail(NKM_ERR_ARG, "device %d out of range", dev);
  NKM_CUDA(cudaFree(nullptr));  // makes the device's primary context current (allocates nothing)
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& s = g_noalloc_dev[dev];
  if (!s.scratch || s.ctx != ctx) {
    void* ptr = nullptr;
    NKM_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    int sms = 0;
    NKM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    s.num_sms = sms;
    s.scratch = static_cast<uint8_t*>(ptr);
    s.ctx = ctx;
  }
  *out = s;
  return NKM_OK;
}

// Zero the control words (every call starts from a clean barrier, status and counters) and
// store the layer's pointer table entry; runs on the caller's stream before the MoE kernel.
__global__ void noalloc_prepare_kernel(nkm::LayerPtrs lp, nkm::LayerPtrs* slot, uint4* ctrl, int n16) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x)
    ctrl[i] = make_uint4(0u, 0u, 0u, 0u);
  if (blockIdx.x == 0 && threadIdx.x == 0) *slot = lp;
}

}  // namespace

extern "C" int nkm_qwen3_moe_block_noalloc(const nkm_qwen3_desc* desc, int32_t layer, const nkm_qwen3_step* s,
                                           int32_t* status_out, nkm_stream_t stream_) {
  int rc = check_desc(desc);
  if (rc) return rc;
  const nkm_qwen3_desc& d = *desc;
  if (!s) return fail(NKM_ERR_ARG, "step is NULL");
  if (layer < 0 || layer >= d.n_layers) return fail(NKM_ERR_ARG, "layer %d outside 0..%d", layer, d.n_layers - 1);
  if (s->batch <= 0 || s->batch > d.max_batch) return fail(NKM_ERR_ARG, "batch %d outside 1..%d", s->batch, d.max_batch);
  if (!s->y_out || !aligned16(s->y_out)) return fail(NKM_ERR_ARG, "y_out must be a 16-byte aligned device pointer");
  if (s->input_ids) {
    if (!d.embed || d.vocab <= 0) return fail(NKM_ERR_ARG, "input_ids given but the model has no embedding table");
  } else if (!s->x_in || !aligned16(s->x_in)) {
    return fail(NKM_ERR_ARG, "x_in must be a 16-byte aligned device pointer");
  }
  if (d.n_ranks > 1) return fail(NKM_ERR_ARG, "the allocation-free MoE block runs on one GPU (n_ranks == 1)");
  const nkm_qwen3_layer& L = d.layers[layer];
  if (!L.router || !L.w13_ft || !L.w2_ft || !L.ln2) return fail(NKM_ERR_ARG, "layer %d: MoE weights missing", layer);
  const void* ps[] = {L.w13_ft, L.w2_ft, L.router, L.ln2};
  for (const void* q : ps)
    if (!aligned16(q)) return fail(NKM_ERR_ARG, "layer %d: weight pointers must be 16-byte aligned", layer);

  NoAllocDevice dv{};
  if ((rc = noalloc_device(&dv))) return rc;
  const NoAllocLayout lay = layout_noalloc(d, s->batch, dv.num_sms);
  if (lay.total > NKM_NOALLOC_SCRATCH_BYTES)
    return fail(NKM_ERR_ARG, "this shape and batch need %zu bytes of scratch; the static scratch holds %zu",
                lay.total, static_cast<size_t>(NKM_NOALLOC_SCRATCH_BYTES));

  const int nt = nt_for_batch(s->batch);
  const int ki = nt == 1 ? 0 : (nt == 2 ? 1 : 2);
  const nkm::SmemLayout sl(d.hidden, nt);
  if (sl.total > 232448 - 1024) return fail(NKM_ERR_ARG, "hidden too large for shared memory");
  if ((rc = ensure_smem_limits())) return rc;

  uint8_t* ws = dv.scratch;
  nkm::Params p{};
  p.T = s->batch;
  p.H = d.hidden;
  p.nq = d.n_q_heads;
  p.nkv = d.n_kv_heads;
  p.grp = d.n_q_heads / d.n_kv_heads;
  p.R = (d.n_q_heads + 2 * d.n_kv_heads) * d.head_dim;
  p.E = d.n_experts;
  p.K = d.top_k;
  p.I = d.moe_inter;
  p.L = d.n_layers;
  p.V = d.vocab;
  p.eps = d.rms_eps;
  p.n_ranks = 1;
  p.rank = 0;
  p.expert_begin = 0;
  p.n_local = d.n_experts;
  p.first_layer = layer;
  p.num_layers = 1;
  p.stages = NKM_STAGE_MOE;
  p.residual = s->residual ? 1 : 0;
  p.layers = reinterpret_cast<const nkm::LayerPtrs*>(ws + lay.layers);
  p.embed = static_cast<const uint16_t*>(d.embed);
  p.input_ids = s->input_ids;
  p.x_in = static_cast<const uint16_t*>(s->x_in);
  p.y_out = static_cast<uint16_t*>(s->y_out);
  p.tr_topk_idx = s->trace_topk_idx;
  p.tr_topk_w = s->trace_topk_w;
  p.tr_rlogits = s->trace_router_logits;
  p.tr_mid = s->trace_resid_mid;
  p.tr_out = s->trace_resid_out;
  p.tr_stage = s->trace_stage_ns;
  p.bar = reinterpret_cast<unsigned*>(ws + lay.bar);
  p.status = reinterpret_cast<int*>(ws + lay.status);
  p.strip_cnt = reinterpret_cast<unsigned*>(ws + lay.strip_cnt);
  p.attn_cnt = reinterpret_cast<unsigned*>(ws + lay.attn_cnt);
  p.row_cnt = reinterpret_cast<unsigned*>(ws + lay.row_cnt);
  p.resid = reinterpret_cast<float*>(ws + lay.resid);
  p.rlogits = reinterpret_cast<float*>(ws + lay.rlogits);
  p.hbuf = reinterpret_cast<uint16_t*>(ws + lay.hbuf);
  p.ypair = reinterpret_cast<float*>(ws + lay.ypair);
  p.gpart = reinterpret_cast<float*>(ws + lay.gpart);

  const nkm::LayerPtrs lp{nullptr, nullptr, nullptr, nullptr, nullptr,
                          static_cast<const uint16_t*>(L.ln2), static_cast<const uint16_t*>(L.router),
                          static_cast<const uint8_t*>(L.w13_ft), static_cast<const uint8_t*>(L.w2_ft),
                          L.router_bias};
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  noalloc_prepare_kernel<<<16, 256, 0, stream>>>(lp, reinterpret_cast<nkm::LayerPtrs*>(ws + lay.layers) + layer,
                                                  reinterpret_cast<uint4*>(ws), static_cast<int>(lay.ctrl_bytes / 16));
  NKM_CUDA(cudaGetLastError());
  CUtensorMap nomap;
  memset(&nomap, 0, sizeof(nomap));
  void* args[3] = {&p, &nomap, &nomap};
  NKM_CUDA(cudaLaunchCooperativeKernel(decode_kernel_fn(ki), dim3(dv.num_sms), dim3(nkm::kThreads), args, sl.total,
                                       stream));
  if (status_out)
    NKM_CUDA(cudaMemcpyAsync(status_out, ws + lay.status, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream));
  return NKM_OK;
}
