// Persistent cooperative decode-step kernel for Qwen3-MoE on B200 (sm_100a).
//
// One CTA per SM, 8 warps per CTA.  In the GEMV stages every warp is an independent
// "worker" with a private ring of 4 KB shared-memory slots that its lane 0 fills with TMA
// bulk copies of fragment-tiled weights; the warp consumes the slots with mma.sync.  In the
// attention stage a CTA owns one (sequence, kv head, context chunk) item and its warps stream
// the K/V pages through their rings with 2-D swizzled TMA tensor copies.  Stages of a layer
// are separated by grid-wide barriers with bounded waits.  The residual stream is kept in
// fp32 in a small L2-resident global buffer.
//
// Stages per layer (reference order: megakernels/qwen3_moe/transformer_qwen.py:271-378):
//   A  RMSNorm(ln1) + QKV GEMV                                      -> qkv (raw bf16)
//   B  q/k RMSNorm + RoPE, KV write at pos, split-context attention -> attn_out (bf16)
//   C  O-proj GEMV + residual add                                   -> resid (fp32)
//   D  RMSNorm(ln2) + fp32 router logits                            -> rlogits
//   E  softmax/top-k/renorm (per CTA) + gate/up GEMV + SiLU*up      -> h (bf16)
//   F  down GEMV * affinity + per-token combine + residual add      -> resid (fp32)
#pragma once
#include "nkm_ptx.cuh"

namespace nkm {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kSlotBytes = 4096;           // attention ring slot: one 32-token x 64-dim TMA box
constexpr int kUnitBytes = 1024;           // one fragment tile: 16 rows x 32 k, bf16
constexpr int kMaxBars = 4;                // mbarriers per warp (attention uses up to 4 slots)
constexpr int kHeadDim = 128;
constexpr int kKvBlock = 128;
constexpr int kAttTile = 32;               // tokens per attention tile (rows of one TMA box)
constexpr int kAttItemsWide = 4;           // attention items per CTA at batches above 8 (<= kWarps:
                                           // the partials area holds kWarps items per SM)
constexpr int kMaxExperts = 256;
constexpr int kMaxPairs = 256;             // max batch * top_k
constexpr int kMaxHidden = 2048;           // register-resident row loads: 8 groups of 256
constexpr int kHidGroups = kMaxHidden / 256;
constexpr int kMaxLaunchLayers = 128;       // layer pointer table held in shared memory
constexpr int kMaxRanks = 8;                // GPUs of one tensor/expert-parallel group
constexpr int kXchgHeader = 256;            // exchange region: barrier counter, then partials
constexpr int kAttRows = 16;               // q heads per kv head handled by one mma (<= 16)
constexpr int kAttQStride = kHeadDim + 8;  // bf16 elements per staged q row
constexpr int kAttShared = kAttRows * kAttQStride * 2 + 2 * kHeadDim * 2 + kWarps * 2 * kAttRows * 4 + 16;
constexpr int kPartFloats = 2 * kAttRows + kAttRows * kHeadDim;  // m, l, o of one CTA chunk
constexpr int kStatusFatal = 4;            // NKM_ERR_TIMEOUT
constexpr int kStatusIndex = 8;            // NKM_ERR_INDEX
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any wait
// Router-logit slot not written yet (a NaN bit pattern the arithmetic never produces: results
// that are NaN are stored as the canonical NaN instead).
constexpr uint32_t kLogitEmpty = 0xffffffffu;
// QKV output element not written yet (bf16 NaN pattern never produced by rounding; a computed
// NaN is stored as the canonical 0x7fff).
constexpr uint16_t kBf16Empty = 0xffffu;

struct LayerPtrs {
  const uint8_t* wqkv;
  const uint8_t* wo;
  const uint16_t* qn;
  const uint16_t* kn;
  const uint16_t* ln1;
  const uint16_t* ln2;
  const uint16_t* router;
  const uint8_t* w13;
  const uint8_t* w2;
  const float* router_bias;
};

struct Params {
  int T, H, nq, nkv, grp, R, E, K, I, L, V;
  float eps;
  // tensor + expert parallelism: this rank's experts [expert_begin, expert_begin + n_local)
  int n_ranks, rank, expert_begin, n_local;
  uint8_t* xchg[kMaxRanks];       // exchange region of every rank (kXchgHeader bytes + partials)
  unsigned long long* gbase;      // workspace: cross-GPU barrier count before this launch
  unsigned* xseq;                 // workspace: partial exchanges of each kind before this launch
  // LM head rows of this rank: 16-row strips [lm_s0, lm_s0 + lm_ns) of the vocabulary.  With
  // several ranks every rank stores its logits into every rank's exchange region at byte offset
  // xlog_off ([T][V] fp32), and after a cross-GPU barrier copies the whole of it to logits_out.
  int lm_s0, lm_ns;
  int64_t xlog_off;
  int first_layer, num_layers, stages, residual;
  const LayerPtrs* layers;
  const uint16_t* final_norm;
  const uint8_t* lm_head;
  const uint16_t* embed;
  const uint16_t* rope_cos;
  const uint16_t* rope_sin;
  int rope_max;
  uint16_t* k_pool;
  uint16_t* v_pool;
  int num_blocks;
  const int* input_ids;
  const uint16_t* x_in;
  const int* positions;
  const int* block_table;
  int max_blocks;
  uint16_t* y_out;
  float* logits_out;
  int* tr_topk_idx;
  float* tr_topk_w;
  float* tr_rlogits;
  uint16_t* tr_qkv;
  float* tr_mid;
  float* tr_out;
  unsigned long long* tr_stage;
  unsigned* bar;
  int* status;
  unsigned* strip_cnt;
  unsigned* attn_cnt;
  unsigned* row_cnt;
  float* resid;
  uint16_t* qkv;
  uint16_t* attn_out;
  float* att_part;
  float* rlogits;
  uint16_t* hbuf;
  float* ypair;
  float* gpart;
};

struct Route {
  int nA;
  int act_e[kMaxExperts];
  int act_off[kMaxExperts];
  int act_cnt[kMaxExperts];
  unsigned emask[kMaxExperts];  // tokens that picked each expert (routing scratch)
  int topk_idx[kMaxPairs];
  float topk_w[kMaxPairs];
  int eoff[kMaxExperts];  // pair offset of each expert (routing scratch)
  int pair_tok[kMaxPairs];
  float pair_w[kMaxPairs];
};

// Dense GEMVs with few strips (QKV, O-proj) at batch <= 8 give every CTA whole strips and
// reduce them in shared memory: at most this many strips per CTA.
constexpr int kCtaStripsMax = 3;

// The attention items of one CTA are the same for every layer of a launch (they depend on the
// positions only): planned once per launch.  n < 0: more items than the plan holds (the stage
// then plans on the fly).
constexpr int kMaxAttItems = 2;
struct AttPlan {
  int n, CT;
  int b[kMaxAttItems], h[kMaxAttItems], ch[kMaxAttItems], nch[kMaxAttItems], pos[kMaxAttItems],
      item[kMaxAttItems];
  int blk[kMaxAttItems][32];  // block ids of the item's context chunk (lane j: block tok_beg/128 + j)
};

// Shared-memory layout, identical on host (sizing) and device.  Each warp owns a ring of
// ring_bytes: the GEMV stages use it as 2 slots of (chunk units x 1 KB), the attention stage
// as 4 KB slots.
template <int NT>
struct RingGeom {
  static constexpr int kRingBytes = NT == 4 ? 8192 : 16384;
  static constexpr int kChunk = NT == 4 ? 4 : 8;      // GEMV units per TMA chunk
  static constexpr int kGemvSlots = kRingBytes / (kChunk * kUnitBytes);
  static constexpr int kAttSlots = kRingBytes / kSlotBytes;
  static constexpr int kAccSets = NT == 1 ? 4 : 2;    // independent accumulator chains
};

struct SmemLayout {
  uint32_t ring_bytes;
  uint32_t ring_off, xs_off, bars_off, rstd_off, route_off, lt_off, plan_off, red_off, flag_off, cbar_off, dyn_off, total;
  __host__ __device__ SmemLayout(int H, int NT) {
    ring_bytes = NT == 4 ? 8192u : 16384u;
    ring_off = 0;
    uint32_t ring = static_cast<uint32_t>(kWarps) * ring_bytes;
    xs_off = ring;
    uint32_t xs = static_cast<uint32_t>(8 * NT * (H + 32) * 2);
    uint32_t att = static_cast<uint32_t>(kAttShared);
    uint32_t u = xs > att ? xs : att;
    bars_off = xs_off + ((u + 127u) & ~127u);
    rstd_off = bars_off + static_cast<uint32_t>(kWarps * kMaxBars * 8);
    route_off = rstd_off + 32 * 4;
    lt_off = route_off + static_cast<uint32_t>((sizeof(Route) + 15) & ~size_t(15));
    plan_off = lt_off + static_cast<uint32_t>(kMaxLaunchLayers * sizeof(LayerPtrs));
    red_off = plan_off + static_cast<uint32_t>((sizeof(AttPlan) + 15) & ~size_t(15));
    flag_off = red_off + (NT == 1 ? static_cast<uint32_t>(kCtaStripsMax * kWarps * 32 * 4 * 4) : 0u);
    cbar_off = flag_off + 16;
    dyn_off = cbar_off + 16;
    total = dyn_off + 64 + 1024;  // + alignment slack for the ring base
  }
};

// ------------------------------------------------------------------ per-warp context
struct Ctx {
  uint8_t* ring;       // this warp's ring
  uint8_t* ring_all;   // ring of warp 0 (rings are contiguous, ring_bytes each)
  int ring_bytes;
  uint64_t* bars;
  uint32_t phase;
  int head;
  int nslot;
  int worker, nworkers;
  uint64_t pol;
  uint16_t* xs;
  int xs_stride;  // elements per X row
  uint8_t* att;   // CTA-shared attention staging (aliases xs)
  float* rstd;
  Route* rt;
  const LayerPtrs* lt;  // pointer table of layers first_layer .. first_layer + num_layers - 1
  AttPlan* plan;        // this CTA's attention items
  float* red;           // per-strip partial tiles of the whole-strip GEMV mode (batch <= 8)
  int att_pb;           // K/V boxes of the first attention item already issued (-1: none)
  int* flag;
  int stage_idx;
  unsigned bar_k;  // grid barriers passed in this launch
  unsigned gbar_k;           // cross-GPU barriers passed in this launch
  unsigned long long gbase;  // cross-GPU barrier count before this launch
  int primed;  // ring slots of the next GEMV stage already in flight
  uint64_t* cbar;   // CTA mbarrier of the staged norms' prefetch (thread 0 issues, all wait)
  uint32_t cphase;  // its phase (tracked by every thread)
  int* dyn;         // chunk scheduling words of the expert gate/up stage (shared memory)
  int awaitq;       // attention waits for its q/k/v element by element (no grid barrier before it)
  int npref;        // the next staged norm's prefetch is in flight
};

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ void set_status(const Params& p, int bit) { atomicOr(p.status, bit); }

// Position of sequence b's new token, clamped to what the RoPE tables and the block-table row
// can address; a position outside that range records NKM_ERR_INDEX.
__device__ __forceinline__ int seq_pos(const Params& p, int b) {
  const int raw = __ldg(p.positions + b);
  const int hi = min(p.rope_max, p.max_blocks * kKvBlock) - 1;
  if (raw < 0 || raw > hi) {
    set_status(p, kStatusIndex);
    return max(0, min(raw, hi));
  }
  return raw;
}

__device__ __forceinline__ void stamp(const Params& p, Ctx& c) {
  if (p.tr_stage && blockIdx.x == 0 && threadIdx.x == 0) p.tr_stage[c.stage_idx] = globaltimer_ns();
  ++c.stage_idx;
}

// Bounded wait on a slot's mbarrier.  On timeout the fatal status bit is set and the caller
// continues (the next grid barrier then aborts every CTA).
// Bounded wait for phase `par` of an mbarrier; on timeout the status records a fatal error.
// A wait that has lasted longer than any normal one (kPollAfterNs) also polls the status word:
// once any wait of the launch has given up, every other wait ends at its next poll instead of
// spending its own full bound (the launch then ends at the next grid barrier), so the whole
// launch is bounded by one wait limit plus the polls.  Normal waits never load the status word.
constexpr uint64_t kPollAfterNs = 20000ull;
__device__ __noinline__ void mbar_wait_slow(const Params& p, uint64_t* bar, uint32_t par) {
  // try_wait itself suspends for a while; read the (slow) global timer only every 64 tries
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, par)) break;
    if ((it & 63u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kPollAfterNs) {
        if (ld_volatile_i32(p.status) & kStatusFatal) break;
        if (now - t0 > kWaitLimitNs) {
          if (lane_id() == 0) set_status(p, kStatusFatal);
          break;
        }
      }
    }
  }
}
__device__ __forceinline__ void slot_wait(const Params& p, Ctx& c, int slot) {
  const uint32_t par = (c.phase >> slot) & 1u;
  if (!mbar_try_wait(&c.bars[slot], par)) mbar_wait_slow(p, &c.bars[slot], par);
  c.phase ^= (1u << slot);
}

// Grid-wide barrier (sense reversal): the last CTA to arrive resets the arrival count and
// bumps the generation word the others spin on, so the counter is zero again when the kernel
// ends (no per-launch reset needed).  Co-residency is guaranteed by the cooperative launch.
// Returns false if any CTA recorded a fatal status or the wait timed out.
// Grid barrier on one monotonic arrival counter (bar[0]): barrier k of a launch is passed
// when the counter reaches (k + 1) * gridDim.x, so arrivals need no reply and nothing is reset
// on the way; the last CTA to leave the launch zeroes the counter (launch_exit).  The status
// word is read with every poll: a fatal error anywhere releases every waiter.
// Split form: grid_arrive, then work that does not depend on the other CTAs (issuing the next
// stage's weight copies), then grid_wait.
__device__ __forceinline__ void grid_arrive(const Params& p) {
  __syncthreads();
  if (threadIdx.x == 0) red_release_add_u32(p.bar, 1u);
}
__device__ __noinline__ bool grid_wait(const Params& p, Ctx& c) {
  if (threadIdx.x == 0) {
    unsigned* count = p.bar;
    const unsigned target = (c.bar_k + 1u) * gridDim.x;
    int ok = 1;
    uint64_t t0 = 0;
#pragma unroll 1
    for (unsigned it = 0;; ++it) {
      const unsigned v = ld_acquire_u32(count);
      const int st = ld_volatile_i32(p.status);
      if (st & kStatusFatal) {
        ok = 0;
        break;
      }
      if (static_cast<int>(v - target) >= 0) break;
      if (it == 0) {
        t0 = globaltimer_ns();
      } else if ((it & 15u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(p, kStatusFatal);
        ok = 0;
        break;
      }
      __nanosleep(20);
    }
    *c.flag = ok;
  }
  ++c.bar_k;
  __syncthreads();
  stamp(p, c);
  return *c.flag != 0;
}
__device__ __forceinline__ bool grid_barrier(const Params& p, Ctx& c) {
  grid_arrive(p);
  return grid_wait(p, c);
}

// ------------------------------------------------------------------ ranks (TP + EP)
// Partial sums exchanged between ranks, as tagged words (tag in the high 32 bits, the fp32 value
// in the low 32): exchange number n of kind `which` (0: O-projection, 1: experts) stored by rank
// `src` lands in rank q's region at [which][n % 2][src][T][H] after the header, tagged n + 1.  A
// reader waits until every word it needs carries the tag of the exchange it is in; two slots per
// kind suffice because a rank produces exchange n + 2 only after every rank has read exchange n
// (it needs their exchange n + 1, which each rank produces after reading exchange n).
__device__ __forceinline__ unsigned long long* xchg_ll(const Params& p, int q, int which, unsigned n, int src) {
  return reinterpret_cast<unsigned long long*>(p.xchg[q] + kXchgHeader) +
         static_cast<size_t>((which * 2 + static_cast<int>(n & 1u)) * p.n_ranks + src) * p.T * p.H;
}
// Sequence number of `layer`'s exchange of kind `which`: the exchanges before this launch (written
// by the previous launch's last CTA, constant during this one) plus one per earlier layer.
__device__ __forceinline__ unsigned xseq_of(const Params& p, int which, int layer) {
  return __ldg(p.xseq + which) + static_cast<unsigned>(layer - p.first_layer);
}
__device__ __forceinline__ unsigned long long ll_word(unsigned n, float v) {
  return (static_cast<unsigned long long>(n + 1u) << 32) | __float_as_uint(v);
}
// Store value v of element `off` of this rank's partial of exchange n into every rank's region.
__device__ __forceinline__ void ll_put(const Params& p, int which, unsigned n, size_t off, float v) {
  const unsigned long long w = ll_word(n, v);
#pragma unroll 1
  for (int q = 0; q < p.n_ranks; ++q) st_relaxed_sys_u64(xchg_ll(p, q, which, n, p.rank) + off, w);
}
// Out of line (the single-GPU path never calls them): the elements off + d[i] of `layer`'s
// partial of kind `which`, values v[i].
__device__ __noinline__ void ll_put2(const Params& p, int which, int layer, size_t off, float v0, float v1, int d1) {
  const unsigned n = xseq_of(p, which, layer);
  ll_put(p, which, n, off, v0);
  ll_put(p, which, n, off + d1, v1);
}
__device__ __noinline__ void ll_put4(const Params& p, int which, int layer, size_t off, float4 v) {
  const unsigned n = xseq_of(p, which, layer);
  ll_put(p, which, n, off, v.x);
  ll_put(p, which, n, off + 1, v.y);
  ll_put(p, which, n, off + 2, v.z);
  ll_put(p, which, n, off + 3, v.w);
}

// Vocabulary-sharded LM head: the [T][V] fp32 logits area of rank q's region.
__device__ __forceinline__ float* xchg_logits(const Params& p, int q) {
  return reinterpret_cast<float*>(p.xchg[q] + p.xlog_off);
}

// Barrier over every CTA of every rank: each CTA adds 1 to the counter of every rank (after a
// system-scope fence: its partial stores into the other ranks' regions become visible first) and
// waits until its own rank's counter reaches the launch base + (k + 1) * CTAs * ranks.  The
// counters never reset; every rank adds the same count per launch to its base (launch_exit).
__device__ __noinline__ bool grid_sync_ranks(const Params& p, Ctx& c) {
  __syncthreads();
  // lane q of warp 0 arrives at rank q, after a system-scope fence that orders the CTA's
  // partial stores (made visible to it by the CTA barrier) before the arrival
  if (threadIdx.x < p.n_ranks) {
    fence_acq_rel_sys();
    red_relaxed_sys_add_u64(reinterpret_cast<unsigned long long*>(p.xchg[threadIdx.x]), 1ull);
  }
  if (threadIdx.x == 0) {
    const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(p.xchg[p.rank]);
    const unsigned long long target =
        c.gbase + (static_cast<unsigned long long>(c.gbar_k) + 1ull) * gridDim.x * static_cast<unsigned>(p.n_ranks);
    int ok = 1;
    uint64_t t0 = 0;
#pragma unroll 1
    for (unsigned it = 0;; ++it) {
      const unsigned long long v = ld_acquire_sys_u64(mine);
      const int st = ld_volatile_i32(p.status);
      if (st & kStatusFatal) {
        ok = 0;
        break;
      }
      if (v >= target) break;
      if (it == 0) {
        t0 = globaltimer_ns();
      } else if ((it & 15u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(p, kStatusFatal);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    *c.flag = ok;
  }
  ++c.gbar_k;
  __syncthreads();
  return *c.flag != 0;
}

// resid[t][row] += bf16(sum over ranks, in rank order, of exchange n of kind `which`), for the
// 16-row strips s = blockIdx.x, blockIdx.x + gridDim.x, ...: each element waits (bounded) until
// every rank's word for it carries exchange n's tag.  Every rank computes the same sums, so the
// residual streams stay identical.  Returns false once the launch has failed.
__device__ __noinline__ bool rank_reduce(const Params& p, int which, int layer, unsigned n) {
  const int S = p.H / 16, ne = p.T * 16;
  const unsigned tag = n + 1u;
  float* trace = which == 0 ? p.tr_mid : p.tr_out;
#pragma unroll 1
  for (int s = blockIdx.x; s < S; s += gridDim.x) {
#pragma unroll 1
    for (int e = threadIdx.x; e < ne; e += kThreads) {
      const int t = e >> 4, row = s * 16 + (e & 15);
      const size_t off = static_cast<size_t>(t) * p.H + row;
      unsigned long long w[kMaxRanks];
      unsigned pend = 0u;
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q) {
        w[q] = q < p.n_ranks ? ld_relaxed_sys_u64(xchg_ll(p, p.rank, which, n, q) + off) : 0ull;
        if (q < p.n_ranks && static_cast<unsigned>(w[q] >> 32) != tag) pend |= 1u << q;
      }
      if (pend) {
        uint64_t t0 = 0;
#pragma unroll 1
        for (uint32_t it = 0; pend; ++it) {
          if ((it & 15u) == 0) {
            const uint64_t now = globaltimer_ns();
            if (it == 0) t0 = now;
            if ((ld_volatile_i32(p.status) & kStatusFatal) || now - t0 > kWaitLimitNs) {
              set_status(p, kStatusFatal);
              return false;
            }
          }
          __nanosleep(32);
#pragma unroll
          for (int q = 0; q < kMaxRanks; ++q) {
            if (pend & (1u << q)) {
              w[q] = ld_relaxed_sys_u64(xchg_ll(p, p.rank, which, n, q) + off);
              if (static_cast<unsigned>(w[q] >> 32) == tag) pend &= ~(1u << q);
            }
          }
        }
      }
      float a = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)
        if (q < p.n_ranks) a += __uint_as_float(static_cast<unsigned>(w[q]));
      float* x = p.resid + off;
      const float nv = (p.residual ? *x : 0.f) + rbf(a);
      *x = nv;
      if (trace) trace[static_cast<size_t>(layer - p.first_layer) * p.T * p.H + off] = nv;
    }
  }
  return true;
}

// Rank-partial exchange of `layer`: the rank-order reduction into the residual (it waits for the
// other ranks' tagged words), then a grid barrier (the next stage reads whole residual rows).
__device__ __forceinline__ bool rank_exchange(const Params& p, Ctx& c, int which, int layer) {
  const bool ok = rank_reduce(p, which, layer, xseq_of(p, which, layer));
  // the barrier runs either way: every CTA passes the same barriers, and a failed wait has set
  // the fatal status that ends it early
  const bool ok2 = grid_barrier(p, c);
  return ok && ok2;
}

// End of a launch: the last CTA out zeroes the barrier counter for the next launch on this
// workspace (launches on one workspace are stream-ordered).
// multi: this launch belongs to a group of several ranks (only kernels built with kExt run one)
__device__ __forceinline__ void launch_exit(const Params& p, const Ctx& c, bool multi) {
  if ((ld_volatile_i32(p.status) & kStatusFatal) && lane_id() == 0) {
    // a failed wait ends the launch early: wait for the next phase of each of this warp's
    // mbarriers (and the norm-prefetch barrier for thread 0), each wait bounded by 1 ms.  A copy
    // this warp issued and has not waited for (it writes into this CTA's shared memory) completes
    // that phase when it lands; a slot with no copy in flight spends the 1 ms bound (only on this
    // error path; the hot path carries no per-copy bookkeeping for it).
#pragma unroll 1
    for (int s = 0; s < (threadIdx.x == 0 ? 5 : 4); ++s) {
      uint64_t* bar = s < 4 ? &c.bars[s] : c.cbar;
      const uint32_t par = s < 4 ? ((c.phase >> s) & 1u) : (c.cphase & 1u);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar, par) && globaltimer_ns() - t0 < 1000000ull) {
      }
    }
  }
  __syncthreads();

  if (threadIdx.x == 0) {
    const unsigned old = atom_acqrel_add_u32(p.bar + 2, 1u);
    if (old == gridDim.x - 1) {
      if (multi) {
        *p.gbase = c.gbase + static_cast<unsigned long long>(c.gbar_k) * gridDim.x * static_cast<unsigned>(p.n_ranks);
        // every layer of the launch took one exchange of each kind its stages run (every other
        // CTA has left the launch: nothing reads the counts any more)
        if (p.stages & 1) p.xseq[0] += static_cast<unsigned>(p.num_layers);
        if (p.stages & 2) p.xseq[1] += static_cast<unsigned>(p.num_layers);
      }
      *reinterpret_cast<volatile unsigned*>(p.bar) = 0u;
      *reinterpret_cast<volatile unsigned*>(p.bar + 2) = 0u;
    }
  }
}

// ------------------------------------------------------------------ fixed-order reductions
__device__ __forceinline__ float warp_sum_fixed(float s) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}
__device__ __forceinline__ float warp_max(float s) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}
// Out of line: one copy of the correctly rounded square root and division for every caller.
__device__ __noinline__ float rstd_fixed(float sumsq, int n, float eps) {
  const float v = __fadd_rn(__fmul_rn(sumsq, 1.0f / static_cast<float>(n)), eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(v));
}

// One fp32 hidden row in registers: lane l holds k = 256*i + 8*l + j (i < H/256, j < 8).
struct RowRegs {
  float v[kHidGroups][8];
};
__device__ __forceinline__ void load_row(const float* row, int H, RowRegs& x) {
  const int lane = lane_id();
#pragma unroll
  for (int i = 0; i < kHidGroups; ++i) {
    if (i < H / 256) {
      const float4 a = ldcg_f4(row + 256 * i + 8 * lane);
      const float4 b = ldcg_f4(row + 256 * i + 8 * lane + 4);
      x.v[i][0] = a.x; x.v[i][1] = a.y; x.v[i][2] = a.z; x.v[i][3] = a.w;
      x.v[i][4] = b.x; x.v[i][5] = b.y; x.v[i][6] = b.z; x.v[i][7] = b.w;
    }
  }
}
// Sum of squares in the documented order (lane-sequential i-outer / j-inner, then a xor
// butterfly) — the oracle's lane_sum_hidden.
__device__ __forceinline__ float row_sumsq(const RowRegs& x, int H) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kHidGroups; ++i) {
    if (i < H / 256) {
#pragma unroll
      for (int j = 0; j < 8; ++j) s = __fadd_rn(s, __fmul_rn(x.v[i][j], x.v[i][j]));
    }
  }
  return warp_sum_fixed(s);
}
__device__ __forceinline__ void load_gamma(const uint16_t* g, int H, uint4 (&gv)[kHidGroups]) {
  const int lane = lane_id();
#pragma unroll
  for (int i = 0; i < kHidGroups; ++i)
    if (i < H / 256) gv[i] = ldnc128(g + 256 * i + 8 * lane);
}
__device__ __forceinline__ float gam(const uint4 (&gv)[kHidGroups], int i, int j) {
  const uint32_t w = (j < 2) ? gv[i].x : (j < 4) ? gv[i].y : (j < 6) ? gv[i].z : gv[i].w;
  return (j & 1) ? hi_bf(w) : lo_bf(w);
}

// RMSNorm of the residual rows into X shared memory (bf16), one warp per token; also stores
// the row's rstd.  gamma_first=false: (x*r)*g (attn_fused_nki.py:306-309);
// true: (x*g)*r (moe_fused_nki.py:114-147).
// When x32 is non-null the fp32 normalised rows are also stored there (row stride H).
__device__ __noinline__ void norm_rows_to_smem(const Params& p, Ctx& c, const uint16_t* gamma, bool gamma_first,
                                               float* x32 = nullptr) {
  // every field is read once into a register: stores through the row pointers below could
  // otherwise alias p and c and force reloads on the dependency chain
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const int T = p.T, H = p.H, ng = H / 256;
  const float eps = p.eps;
  const float* __restrict__ resid = p.resid;
  uint16_t* __restrict__ xs = c.xs;
  float* __restrict__ rstd = c.rstd;
  const int stride = c.xs_stride;
  if (warp >= T) return;
  // gamma and the first row are requested together: one memory latency, not one per group
  uint4 gam[kHidGroups];
#pragma unroll
  for (int i = 0; i < kHidGroups; ++i)
    gam[i] = (i < ng) ? ldnc128(gamma + 256 * i + 8 * lane) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll 1
  for (int t = warp; t < T; t += kWarps) {
    RowRegs x;
    load_row(resid + static_cast<size_t>(t) * H, H, x);
    const float r = rstd_fixed(row_sumsq(x, H), H, eps);
    if (lane == 0) rstd[t] = r;
    uint16_t* __restrict__ xr = xs + static_cast<size_t>(t) * stride + 8 * lane;
    float* __restrict__ xf = x32 ? x32 + static_cast<size_t>(t) * H + 8 * lane : nullptr;
#pragma unroll
    for (int i = 0; i < kHidGroups; ++i) {
      if (i < ng) {
        const uint4 gv = gam[i];
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        float y[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float g0 = lo_bf(gw[j]), g1 = hi_bf(gw[j]);
          // (x*r)*g or (x*g)*r without duplicating the code path
          const float a0 = gamma_first ? g0 : r, b0 = gamma_first ? r : g0;
          const float a1 = gamma_first ? g1 : r, b1 = gamma_first ? r : g1;
          y[2 * j] = __fmul_rn(__fmul_rn(x.v[i][2 * j], a0), b0);
          y[2 * j + 1] = __fmul_rn(__fmul_rn(x.v[i][2 * j + 1], a1), b1);
        }
        *reinterpret_cast<uint4*>(xr + 256 * i) =
            make_uint4(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]), pack_bf2(y[4], y[5]), pack_bf2(y[6], y[7]));
        if (xf) {
          *reinterpret_cast<float4*>(xf + 256 * i) = make_float4(y[0], y[1], y[2], y[3]);
          *reinterpret_cast<float4*>(xf + 256 * i + 4) = make_float4(y[4], y[5], y[6], y[7]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ fragment-tiled GEMV
// Code size matters here: the persistent kernel runs every stage once per layer, so each
// stage's instructions are cold in the instruction caches unless the whole per-layer code
// stays small.  The streaming loop below is kept compact; strip flushes (epilogues and the
// split-K fix-up) are out of line.
enum GemvKind { GK_QKV = 0, GK_OPROJ = 1, GK_GATEUP = 2, GK_DOWN = 3, GK_LMHEAD = 4 };

struct GemvGeom {
  const uint8_t* base;   // weights of segment 0 (dense) or of expert 0 (experts)
  uint64_t seg_bytes;    // byte stride between experts
  int nseg;              // segments (1 dense, nA experts)
  int sps;               // strips (16 output rows) per segment
  int kt;                // k-tiles (32) per strip
  int kdim;              // K in elements
  int layer;
};

// LM head rows of this rank (all of them on one GPU)
__device__ __forceinline__ GemvGeom lm_geom(const Params& p, int layer) {
  return GemvGeom{p.lm_head + static_cast<uint64_t>(p.lm_s0) * (p.H / 32) * kUnitBytes, 0, 1, p.lm_ns, p.H / 32, p.H,
                  layer};
}

template <int NT>
struct Acc {
  float v[NT][4];
};

__device__ __forceinline__ bool kind_experts(int kind) { return kind == GK_GATEUP || kind == GK_DOWN; }

__device__ __forceinline__ const uint8_t* seg_base(const GemvGeom& G, const Route* rt, int kind, int seg) {
  return kind_experts(kind) ? G.base + static_cast<uint64_t>(rt->act_e[seg]) * G.seg_bytes : G.base;
}

// number of columns (tokens) of a segment
__device__ __forceinline__ int seg_cols(const Params& p, const Route* rt, int kind, int seg) {
  return kind_experts(kind) ? rt->act_cnt[seg] : p.T;
}

// B fragment (16 bytes: 8 consecutive k of one column) for lane (g,t), n-tile nt.
__device__ __forceinline__ uint4 load_bfrag(const Params& p, const uint16_t* xs, int xs_stride, const Route* rt,
                                            int kind, int seg, int kt, int nt, int ncols) {
  const int lane = lane_id();
  const int col = nt * 8 + (lane >> 2);
  const int k = kt * 32 + 8 * (lane & 3);
  if (col >= ncols) return make_uint4(0, 0, 0, 0);
  if (kind == GK_OPROJ) return ldcg128(p.attn_out + static_cast<size_t>(col) * (p.nq * kHeadDim) + k);
  const int row = kind == GK_GATEUP ? rt->pair_tok[rt->act_off[seg] + col] : col;
  return lds128(smem_addr(xs + static_cast<size_t>(row) * xs_stride + k));
}

__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Final write of one strip's accumulators (all of K reduced): element (row r, column col).
__device__ __forceinline__ void gemv_store(const Params& p, const Route* rt, const GemvGeom& G, int kind, int seg,
                                           int strip, int g, int col, float v0, float v1) {
  if (kind == GK_QKV) {
    const int r0 = strip * 16 + g;
    uint16_t* q = p.qkv + static_cast<size_t>(col) * p.R;
    const uint16_t h0 = f2bf(v0), h1 = f2bf(v1);
    q[r0] = h0 == kBf16Empty ? 0x7fffu : h0;
    q[r0 + 8] = h1 == kBf16Empty ? 0x7fffu : h1;
    if (p.tr_qkv) {
      uint16_t* tq = p.tr_qkv + (static_cast<size_t>(G.layer - p.first_layer) * p.T + col) * p.R;
      tq[r0] = f2bf(v0);
      tq[r0 + 8] = f2bf(v1);
    }
  } else if (kind == GK_OPROJ && p.n_ranks > 1) {
    // tensor parallel: this rank's partial sum over its heads, stored in every rank's region
    ll_put2(p, 0, G.layer, static_cast<size_t>(col) * p.H + strip * 16 + g, v0, v1, 8);
  } else if (kind == GK_OPROJ) {
    const int r0 = strip * 16 + g;
    float* x = p.resid + static_cast<size_t>(col) * p.H;
    const float n0 = (p.residual ? x[r0] : 0.f) + rbf(v0);
    const float n1 = (p.residual ? x[r0 + 8] : 0.f) + rbf(v1);
    x[r0] = n0;
    x[r0 + 8] = n1;
    if (p.tr_mid) {
      float* tm = p.tr_mid + (static_cast<size_t>(G.layer - p.first_layer) * p.T + col) * p.H;
      tm[r0] = n0;
      tm[r0 + 8] = n1;
    }
  } else if (kind == GK_GATEUP) {
    // rows 0-7 of the strip are gate rows 8*strip+g, rows 8-15 the matching up rows
    const int pair = rt->act_off[seg] + col;
    const float h = rbf(rbf(silu_f(rbf(v0))) * rbf(v1));
    p.hbuf[static_cast<size_t>(pair) * p.I + strip * 8 + g] = f2bf(h);
  } else {  // GK_LMHEAD (strip counts from this rank's first vocabulary strip)
    const size_t off = static_cast<size_t>(col) * p.V + (p.lm_s0 + strip) * 16 + g;
    if (p.n_ranks > 1) {
#pragma unroll 1
      for (int q = 0; q < p.n_ranks; ++q) {
        float* lo = xchg_logits(p, q) + off;
        lo[0] = v0;
        lo[8] = v1;
      }
    } else {
      float* lo = p.logits_out + off;
      lo[0] = v0;
      lo[8] = v1;
    }
  }
}

template <int NT, int KIND>
__device__ __noinline__ void gemv_epilogue(const Params& p, const Route* rt, const GemvGeom& G, int seg, int strip,
                                              Acc<NT> acc) {
  constexpr int kind = KIND;
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int ncols = seg_cols(p, rt, kind, seg);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = nt * 8 + 2 * t4 + e;
      if (col < ncols) gemv_store(p, rt, G, kind, seg, strip, g, col, acc.v[nt][e], acc.v[nt][2 + e]);
    }
  }
}

// unit range of worker w among NW workers (NU * NW < 2^31 is checked on the host)
__device__ __forceinline__ int range_lo(int NU, int w, int NW) {
  return static_cast<int>(static_cast<unsigned>(NU) * static_cast<unsigned>(w) / static_cast<unsigned>(NW));
}
__device__ __forceinline__ int worker_of(int u, int NU, int NW) {
  int w = static_cast<int>(static_cast<unsigned>(u) * static_cast<unsigned>(NW) / static_cast<unsigned>(NU));
  while (w + 1 < NW && range_lo(NU, w + 1, NW) <= u) ++w;
  while (w > 0 && range_lo(NU, w, NW) > u) --w;
  return w;
}

// Out-of-line strip flush.  `full`: the worker reduced all of K itself.  Otherwise the
// partial is stored and the last contributor sums all partials in worker order (split-K
// fix-up, deterministic) and runs the epilogue.  Partial slot: 0 if the strip is the
// contributor's first strip, else 1 (only the first contributor can start before it).
template <int NT, int KIND>
__device__ __noinline__ bool gemv_flush(const Params& p, const Route* rt, const GemvGeom& G, int worker, int seg,
                                        int strip, bool full, int u0, int NU, int NWe, Acc<NT> acc) {
  if (full) {
    gemv_epilogue<NT, KIND>(p, rt, G, seg, strip, acc);
    return true;
  }
  const int lane = lane_id();
  const int upseg = G.sps * G.kt;
  const int s0 = seg * upseg + strip * G.kt, s1 = s0 + G.kt;
  const int slot = (u0 >= s0) ? 0 : 1;
  float* dst = p.gpart + ((static_cast<size_t>(worker) * 2 + slot) * NT * 32 + lane) * 4;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    *reinterpret_cast<float4*>(dst + nt * 128) =
        make_float4(acc.v[nt][0], acc.v[nt][1], acc.v[nt][2], acc.v[nt][3]);
  // the warp's partial stores are ordered before lane 0's release by the warp barrier; the
  // acq_rel counter update makes them visible to the last contributor, whose acquire (and
  // the warp barrier of the shuffle) orders its reads of the partials after it
  __syncwarp();
  const int wf = worker_of(s0, NU, NWe), wl = worker_of(s1 - 1, NU, NWe);
  const int gstrip = seg * G.sps + strip;
  unsigned old = 0;
  if (lane == 0) old = atom_acqrel_add_u32(&p.strip_cnt[gstrip], 1u);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != static_cast<unsigned>(wl - wf)) return false;
  const int slot_f = range_lo(NU, wf, NWe) == s0 ? 0 : 1;
  Acc<NT> sum;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) sum.v[nt][0] = sum.v[nt][1] = sum.v[nt][2] = sum.v[nt][3] = 0.f;
#pragma unroll 1
  for (int w0 = wf; w0 <= wl; w0 += 4) {
    float4 v[4][NT];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int w = w0 + u;
      const int sl = (w == wf) ? slot_f : 0;
      const float* src = p.gpart + ((static_cast<size_t>(w) * 2 + sl) * NT * 32 + lane) * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        v[u][nt] = (w <= wl) ? ldcg_f4(src + nt * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sum.v[nt][0] += v[u][nt].x;
        sum.v[nt][1] += v[u][nt].y;
        sum.v[nt][2] += v[u][nt].z;
        sum.v[nt][3] += v[u][nt].w;
      }
    }
  }
  if (lane == 0) p.strip_cnt[gstrip] = 0u;
  gemv_epilogue<NT, KIND>(p, rt, G, seg, strip, sum);
  return true;
}

// One GEMV stage: the unit space (segments x strips x k-tiles, 1 KB each) is split into
// contiguous ranges, one per worker; each worker streams its range through its TMA ring in
// chunks of up to RingGeom::kChunk units that never cross a strip.  Per segment the B-fragment
// row addresses are computed once; consecutive units feed independent accumulator sets so
// that the mma dependency chains stay short.
// Issue the first ring chunks of a GEMV stage early (before the grid barrier that precedes
// it): the weights do not depend on the barrier, so their latency overlaps the barrier.
// Whole-strip mode: strip s of a dense GEMV belongs to CTA s % gridDim.x; warp w of the CTA
// takes K-units [KT w / 8, KT (w + 1) / 8) of each of the CTA's strips.
template <int NT>
__device__ __forceinline__ bool cta_strip_mode(const GemvGeom& G, int kind) {
  return NT == 1 && (kind == GK_QKV || kind == GK_OPROJ) && G.nseg == 1 && G.kt >= kWarps &&
         (G.sps + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x) <= kCtaStripsMax;
}

template <int NT>
__device__ __noinline__ void cta_strips_prime(const Params& p, Ctx& c, const GemvGeom& G, int nprime) {
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots;
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const int Gd = gridDim.x, KT = G.kt;
  const int ns = static_cast<int>(blockIdx.x) < G.sps ? (G.sps - static_cast<int>(blockIdx.x) + Gd - 1) / Gd : 0;
  const int k0 = KT * warp / kWarps, nk = KT * (warp + 1) / kWarps - k0;
  int pj = 0, pk = 0;
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    if (pj >= ns || i >= nprime) break;
    const int n = min(CU, nk - pk);
    if (lane == 0) {
      const int strip = static_cast<int>(blockIdx.x) + pj * Gd;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[i], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + i * (CU * kUnitBytes), G.base + static_cast<uint64_t>(strip * KT + k0 + pk) * kUnitBytes,
               static_cast<uint32_t>(n * kUnitBytes), &c.bars[i], c.pol);
    }
    pk += n;
    if (pk == nk) {
      pk = 0;
      ++pj;
    }
  }
}

// All warps of the CTA call it (one CTA barrier inside).
template <int NT>
__device__ __noinline__ void gemv_cta_strips(const Params& p, Ctx& cref, const GemvGeom& G, int kind) {
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots, NA = RG::kAccSets;
  Ctx c = cref;
  const int primed = c.primed;  // ring slots already filled
  cref.primed = 0;
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3, warp = threadIdx.x >> 5;
  const int Gd = gridDim.x, KT = G.kt;
  const int ns = static_cast<int>(blockIdx.x) < G.sps ? (G.sps - static_cast<int>(blockIdx.x) + Gd - 1) / Gd : 0;
  const int k0 = KT * warp / kWarps, nk = KT * (warp + 1) / kWarps - k0;
  const int ncols = p.T;
  const int ntiles = (ncols + 7) >> 3;
  // B rows of this lane (column g of each n-tile): shared X (QKV) or the attention output (O-proj)
  const bool smem_b = kind == GK_QKV;
  const int col = g;
  const uint4* brow_s = (smem_b && col < ncols)
                            ? reinterpret_cast<const uint4*>(c.xs + static_cast<size_t>(col) * c.xs_stride + 8 * t4)
                            : nullptr;
  const uint16_t* brow_g = (!smem_b && col < ncols)
                               ? p.attn_out + static_cast<size_t>(col) * (p.nq * kHeadDim) + 8 * t4
                               : nullptr;
  int pj = 0, pk = 0;
  auto issue = [&](int slot, bool dry) {
    const int n = min(CU, nk - pk);
    if (lane == 0 && !dry) {
      const int strip = static_cast<int>(blockIdx.x) + pj * Gd;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[slot], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + slot * (CU * kUnitBytes), G.base + static_cast<uint64_t>(strip * KT + k0 + pk) * kUnitBytes,
               static_cast<uint32_t>(n * kUnitBytes), &c.bars[slot], c.pol);
    }
    pk += n;
    if (pk == nk) {
      pk = 0;
      ++pj;
    }
  };
#pragma unroll
  for (int i = 0; i < NS; ++i)
    if (pj < ns) issue(i, i < primed);
  int cs = 0;
#pragma unroll 1
  for (int j = 0; j < ns; ++j) {
    float acc[NA][4];
#pragma unroll
    for (int a = 0; a < NA; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
#pragma unroll 1
    for (int ck = 0; ck < nk; ck += CU) {
      const int n = min(CU, nk - ck);
      uint4 bf[CU];
#pragma unroll
      for (int i = 0; i < CU; ++i) {
        const int kt = k0 + ck + i;
        bf[i] = (i >= n) ? make_uint4(0u, 0u, 0u, 0u)
                         : (brow_s ? brow_s[kt * 4] : (brow_g ? ldcg128(brow_g + kt * 32) : make_uint4(0u, 0u, 0u, 0u)));
      }
      slot_wait(p, c, cs);
      const uint4* sa = reinterpret_cast<const uint4*>(c.ring + cs * (CU * kUnitBytes)) + lane;
#pragma unroll
      for (int i = 0; i < CU; ++i) {
        if (i < n && ntiles > 0) {
          const uint4 a0 = sa[i * (kUnitBytes / 16)];
          const uint4 a1 = sa[i * (kUnitBytes / 16) + 32];
          mma_bf16(acc[i % NA], a0.x, a1.x, a0.y, a1.y, bf[i].x, bf[i].y);
          mma_bf16(acc[i % NA], a0.z, a1.z, a0.w, a1.w, bf[i].z, bf[i].w);
        }
      }
      __syncwarp();
      if (pj < ns) issue(cs, false);
      cs = (cs + 1 == NS) ? 0 : cs + 1;
    }
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      v.x += acc[a][0];
      v.y += acc[a][1];
      v.z += acc[a][2];
      v.w += acc[a][3];
    }
    reinterpret_cast<float4*>(c.red)[(j * kWarps + warp) * 32 + lane] = v;
  }
  cref.phase = c.phase;
  __syncthreads();
  if (warp < ns) {
    // strip `warp` of this CTA: the 8 K-slices summed in warp order
    Acc<NT> sum;
    sum.v[0][0] = sum.v[0][1] = sum.v[0][2] = sum.v[0][3] = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float4 v = reinterpret_cast<const float4*>(c.red)[(warp * kWarps + w) * 32 + lane];
      sum.v[0][0] += v.x;
      sum.v[0][1] += v.y;
      sum.v[0][2] += v.z;
      sum.v[0][3] += v.w;
    }
    if (kind == GK_QKV) gemv_epilogue<NT, GK_QKV>(p, c.rt, G, 0, static_cast<int>(blockIdx.x) + warp * Gd, sum);
    else gemv_epilogue<NT, GK_OPROJ>(p, c.rt, G, 0, static_cast<int>(blockIdx.x) + warp * Gd, sum);
  }
}

// nprime: ring slots to fill (1 when a staged norm uses slot 1 first)
template <int NT, int KIND>
__device__ __noinline__ void gemv_prime(const Params& p, Ctx& c, const GemvGeom& G,
                                        int nprime = RingGeom<NT>::kGemvSlots) {
  constexpr int kind = KIND;
  if (cta_strip_mode<NT>(G, kind)) {
    c.primed = nprime;
    cta_strips_prime<NT>(p, c, G, nprime);
    return;
  }
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots;
  const int lane = lane_id();
  const int KT = G.kt, SPS = G.sps, upseg = SPS * KT, NU = upseg * G.nseg;
  c.primed = nprime;
  if (NU <= 0) return;
  const int NWe = max(1, min(c.nworkers, NU / 2));
  if (c.worker >= NWe) return;
  const int u0 = range_lo(NU, c.worker, NWe), u1 = range_lo(NU, c.worker + 1, NWe);
  int pu = u0, pseg = u0 / upseg, pstrip = (u0 - pseg * upseg) / KT, pkt = u0 - pseg * upseg - pstrip * KT;
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    if (pu >= u1 || i >= nprime) break;
    const int n = min(CU, min(KT - pkt, u1 - pu));
    if (lane == 0) {
      const uint8_t* src = seg_base(G, c.rt, kind, pseg) + static_cast<uint64_t>(pstrip * KT + pkt) * kUnitBytes;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[i], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + i * (CU * kUnitBytes), src, static_cast<uint32_t>(n * kUnitBytes), &c.bars[i], c.pol);
    }
    pu += n;
    pkt += n;
    if (pkt == KT) {
      pkt = 0;
      if (++pstrip == SPS) {
        pstrip = 0;
        ++pseg;
      }
    }
  }
}

// Expert gate/up projection for batches of at most 8 (NT = 1) with the work of each CTA shared
// by its warps.  CTA b owns the contiguous range of whole 16-row strips [NS b / G, NS (b+1) / G)
// of the nA x (2I / 16) strips; a strip's K is split into KB chunks of kChunk units (one ring
// slot).  Warps claim the CTA's chunks in order from a shared-memory counter, so a warp that
// streams faster takes more of them.  Each chunk's partial tile goes to the strip's slot in the
// strip-reduction area; the warp that completes a strip's KB chunks sums the partials in chunk
// order (fixed order: the result does not depend on which warp took which chunk) and writes
// SiLU(gate) * up.  Strips never straddle CTAs, so no partial leaves the SM.  All warps of the CTA
// call it (one CTA barrier at the start).
constexpr int kDynSlots = 3;  // strips in reduction at once (strip s uses slot (s - s0) % kDynSlots)
template <int NT>
__device__ __forceinline__ bool gateup_dyn_ok(const GemvGeom& G) {
  return NT == 1 && G.kt % RingGeom<NT>::kChunk == 0 &&
         (G.kt / RingGeom<NT>::kChunk) * 32 * 16 * kDynSlots <= kCtaStripsMax * kWarps * 32 * 16;
}
template <int NT>
__device__ __noinline__ void gateup_dyn(const Params& p, Ctx& cref, const GemvGeom& G) {
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots, NA = RG::kAccSets;
  Ctx c = cref;
  cref.primed = 0;
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const Route* rt = c.rt;
  const int SPS = G.sps, KT = G.kt, KB = KT / CU, Gd = gridDim.x;
  const int NSt = G.nseg * SPS;
  const int s0 = static_cast<int>(static_cast<long long>(NSt) * blockIdx.x / Gd);
  const int s1 = static_cast<int>(static_cast<long long>(NSt) * (blockIdx.x + 1) / Gd);
  const int c1 = s1 * KB;
  volatile int* next = c.dyn;       // next chunk to claim
  volatile int* gen = c.dyn + 1;    // [kDynSlots] strip each slot currently collects
  int* cnt = c.dyn + 1 + kDynSlots; // [kDynSlots] chunks deposited
  float4* part = reinterpret_cast<float4*>(c.red);  // [kDynSlots][KB][32]
  if (threadIdx.x == 0) {
    *next = s0 * KB;
    for (int j = 0; j < kDynSlots; ++j) {
      gen[j] = s0 + j;
      cnt[j] = 0;
    }
  }
  __syncthreads();
  auto claim = [&]() {
    int id = 0;
    if (lane == 0) id = atomicAdd(const_cast<int*>(next), 1);
    return __shfl_sync(0xffffffffu, id, 0);
  };
  auto issue = [&](int slot, int id) {
    if (lane == 0) {
      const int strip = id / KB, kb = id - strip * KB;
      const int seg = strip / SPS, ss = strip - seg * SPS;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[slot], static_cast<uint32_t>(CU * kUnitBytes));
      bulk_g2s(c.ring + slot * (CU * kUnitBytes),
               G.base + static_cast<uint64_t>(rt->act_e[seg]) * G.seg_bytes +
                   static_cast<uint64_t>(ss * KT + kb * CU) * kUnitBytes,
               static_cast<uint32_t>(CU * kUnitBytes), &c.bars[slot], c.pol);
    }
  };
  int ids[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    ids[i] = claim();
    if (ids[i] < c1) issue(i, ids[i]);
  }
  int cs = 0;
#pragma unroll 1
  while (ids[cs] < c1) {
    const int id = ids[cs];
    const int strip = id / KB, kb = id - strip * KB;
    const int seg = strip / SPS, ss = strip - seg * SPS;
    const int ncols = rt->act_cnt[seg];
    const uint4* brow = g < ncols ? reinterpret_cast<const uint4*>(c.xs + static_cast<size_t>(rt->pair_tok[rt->act_off[seg] + g]) *
                                                                            c.xs_stride + 8 * t4)
                                  : nullptr;
    uint4 bf[CU];
#pragma unroll
    for (int i = 0; i < CU; ++i) bf[i] = brow ? brow[(kb * CU + i) * 4] : make_uint4(0u, 0u, 0u, 0u);
    slot_wait(p, c, cs);
    float acc[NA][4];
#pragma unroll
    for (int a = 0; a < NA; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
    const uint4* sa = reinterpret_cast<const uint4*>(c.ring + cs * (CU * kUnitBytes)) + lane;
#pragma unroll
    for (int i = 0; i < CU; ++i) {
      const uint4 a0 = sa[i * (kUnitBytes / 16)];
      const uint4 a1 = sa[i * (kUnitBytes / 16) + 32];
      mma_bf16(acc[i % NA], a0.x, a1.x, a0.y, a1.y, bf[i].x, bf[i].y);
      mma_bf16(acc[i % NA], a0.z, a1.z, a0.w, a1.w, bf[i].z, bf[i].w);
    }
    __syncwarp();
    ids[cs] = claim();  // the slot's next chunk streams while this one is reduced
    if (ids[cs] < c1) issue(cs, ids[cs]);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      v.x += acc[a][0];
      v.y += acc[a][1];
      v.z += acc[a][2];
      v.w += acc[a][3];
    }
    // deposit the partial into the strip's slot (once the slot's previous strip is reduced)
    const int sl = (strip - s0) % kDynSlots;
    if (gen[sl] != strip) {
      const uint64_t t0 = globaltimer_ns();
      while (gen[sl] != strip) {
        const uint64_t dt = globaltimer_ns() - t0;
        if (dt > kPollAfterNs && ((ld_volatile_i32(p.status) & kStatusFatal) || dt > kWaitLimitNs)) {
          if (lane == 0) set_status(p, kStatusFatal);
          break;
        }
      }
    }
    part[(sl * KB + kb) * 32 + lane] = v;
    __syncwarp();
    int old = 0;
    if (lane == 0) {
      __threadfence_block();
      old = atomicAdd(&cnt[sl], 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == KB - 1) {
      // the strip's last chunk: sum the KB partials in chunk order, release the slot, epilogue
      __threadfence_block();
      Acc<NT> sum;
      sum.v[0][0] = sum.v[0][1] = sum.v[0][2] = sum.v[0][3] = 0.f;
#pragma unroll 1
      for (int k = 0; k < KB; ++k) {
        const float4 u = part[(sl * KB + k) * 32 + lane];
        sum.v[0][0] += u.x;
        sum.v[0][1] += u.y;
        sum.v[0][2] += u.z;
        sum.v[0][3] += u.w;
      }
      __syncwarp();
      if (lane == 0) {
        cnt[sl] = 0;
        __threadfence_block();
        gen[sl] = strip + kDynSlots;
      }
      gemv_epilogue<NT, GK_GATEUP>(p, rt, G, seg, ss, sum);
    }
    cs = (cs + 1 == NS) ? 0 : cs + 1;
  }
  cref.phase = c.phase;
}

template <int NT, int KIND>
__device__ __noinline__ void gemv_stage(const Params& p, Ctx& cref, const GemvGeom& G) {
  constexpr int kind = KIND;
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots, NA = RG::kAccSets;
  Ctx c = cref;  // register-resident copy for the streaming loop
  const int primed = c.primed;  // ring slots already filled
  cref.primed = 0;
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int KT = G.kt, SPS = G.sps;
  const int upseg = SPS * KT;
  const int NU = upseg * G.nseg;
  if (NU <= 0) return;
  const int NWe = max(1, min(c.nworkers, NU / 2));
  if (c.worker >= NWe) return;
  const int u0 = range_lo(NU, c.worker, NWe), u1 = range_lo(NU, c.worker + 1, NWe);
  if (u0 >= u1) return;
  const Route* rt = c.rt;
  const bool smem_b = !(kind == GK_OPROJ || kind == GK_DOWN);
  // producer cursor
  int pu = u0, pseg = u0 / upseg, pstrip = (u0 - pseg * upseg) / KT, pkt = u0 - pseg * upseg - pstrip * KT;
  const uint8_t* pbase = seg_base(G, rt, kind, pseg);
  auto issue = [&](int slot, bool dry) {
    const int n = min(CU, min(KT - pkt, u1 - pu));
    if (lane == 0 && !dry) {
      const uint8_t* src = pbase + static_cast<uint64_t>(pstrip * KT + pkt) * kUnitBytes;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[slot], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + slot * (CU * kUnitBytes), src, static_cast<uint32_t>(n * kUnitBytes), &c.bars[slot], c.pol);
    }
    pu += n;
    pkt += n;
    if (pkt == KT) {
      pkt = 0;
      if (++pstrip == SPS) {
        pstrip = 0;
        ++pseg;
        if (pu < u1) pbase = seg_base(G, rt, kind, pseg);
      }
    }
  };
#pragma unroll
  for (int i = 0; i < NS; ++i)
    if (pu < u1) issue(i, i < primed);
  // consumer cursor and per-segment B-fragment rows
  int cu = u0, cseg = u0 / upseg, cstrip = (u0 - cseg * upseg) / KT, ckt = u0 - cseg * upseg - cstrip * KT;
  const uint4* brow_s[NT];    // this lane's B row in shared memory (smem sources)
  const uint16_t* brow_g[NT]; // global B row (global sources)
  int ntiles = 0;
  auto seg_setup = [&](int seg) {
    const int ncols = seg_cols(p, rt, kind, seg);
    ntiles = (ncols + 7) >> 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + g;
      const bool ok = col < ncols;
      if (smem_b) {
        const int row = (kind == GK_GATEUP && ok) ? rt->pair_tok[rt->act_off[seg] + col] : col;
        brow_s[nt] = ok ? reinterpret_cast<const uint4*>(c.xs + static_cast<size_t>(row) * c.xs_stride + 8 * t4)
                        : nullptr;
        brow_g[nt] = nullptr;
      } else {
        brow_s[nt] = nullptr;
        brow_g[nt] = !ok ? nullptr
                         : (kind == GK_OPROJ ? p.attn_out + static_cast<size_t>(col) * (p.nq * kHeadDim) + 8 * t4
                                             : p.hbuf + static_cast<size_t>(rt->act_off[seg] + col) * p.I + 8 * t4);
      }
    }
  };
  seg_setup(cseg);
  float acc[NA][NT][4];
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
  int strip_kt0 = ckt;
  int cs = 0;
#pragma unroll 1
  while (cu < u1) {
    const int n = min(CU, min(KT - ckt, u1 - cu));
    // B fragments of the whole chunk (before the slot wait, so global loads overlap it)
    uint4 bf[CU][NT];
    if (smem_b) {
#pragma unroll
      for (int i = 0; i < CU; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          bf[i][nt] = (i < n && brow_s[nt]) ? brow_s[nt][(ckt + i) * 4] : make_uint4(0, 0, 0, 0);
    } else {
#pragma unroll
      for (int i = 0; i < CU; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          bf[i][nt] = (i < n && brow_g[nt]) ? ldcg128(brow_g[nt] + (ckt + i) * 32) : make_uint4(0, 0, 0, 0);
    }
    slot_wait(p, c, cs);
    // A fragments: plain shared loads (scheduled by the compiler around the mma chain)
    const uint4* sa = reinterpret_cast<const uint4*>(c.ring + cs * (CU * kUnitBytes)) + lane;
#pragma unroll
    for (int i = 0; i < CU; ++i) {
      if (i < n) {
        const uint4 a0 = sa[i * (kUnitBytes / 16)];
        const uint4 a1 = sa[i * (kUnitBytes / 16) + 32];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt < ntiles) {
            mma_bf16(acc[i % NA][nt], a0.x, a1.x, a0.y, a1.y, bf[i][nt].x, bf[i][nt].y);
            mma_bf16(acc[i % NA][nt], a0.z, a1.z, a0.w, a1.w, bf[i][nt].z, bf[i][nt].w);
          }
        }
      }
    }
    __syncwarp();
    if (pu < u1) issue(cs, false);
    cs = (cs + 1 == NS) ? 0 : cs + 1;
    cu += n;
    ckt += n;
    if (ckt == KT || cu == u1) {
      Acc<NT> sum;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = 0.f;
#pragma unroll
          for (int a = 0; a < NA; ++a) v += acc[a][nt][e];
          sum.v[nt][e] = v;
        }
      gemv_flush<NT, KIND>(p, rt, G, c.worker, cseg, cstrip, strip_kt0 == 0 && ckt == KT, u0, NU, NWe, sum);
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
      if (ckt == KT) {
        ckt = 0;
        if (++cstrip == SPS) {
          cstrip = 0;
          ++cseg;
          if (cu < u1) seg_setup(cseg);
        }
      }
      strip_kt0 = ckt;
    }
  }
  cref.phase = c.phase;
}

// ------------------------------------------------------------------ MoE down projection
// Work items are (16-row output strip s, active expert j) pairs in strip-major order; an item
// is one expert's whole K (= I / 32 units, contiguous in the fragment-tiled w2).  Workers own
// contiguous item ranges, so each worker sees a run of experts for one or two row strips.
// Per item the accumulators are scaled by the routing affinity and added into a per-warp
// shared-memory tile acc[token][16 rows]; when the worker leaves a row strip the tile is
// either final (the worker covered every expert of the strip: it adds the tile into the
// residual) or a partial (stored; the last contributor sums the partials in worker order and
// adds them).  The MoE output of a token is therefore sum_experts(w * down(h)) in fp32,
// rounded to bf16 once before the residual add (moe_fused_nki.py:542-568, 748-757).
__device__ __forceinline__ const uint8_t* down_item_src(const GemvGeom& G, const Route* rt, int item, int kt) {
  const int s = item / G.nseg, j = item - s * G.nseg;
  return G.base + static_cast<uint64_t>(rt->act_e[j]) * G.seg_bytes +
         static_cast<uint64_t>(s * G.kt + kt) * kUnitBytes;
}

template <int NT>
__device__ __noinline__ void down_prime(const Params& p, Ctx& c, const GemvGeom& G) {
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots;
  const int lane = lane_id();
  const int NI = G.sps * G.nseg, KT = G.kt;
  c.primed = NS;
  if (NI <= 0) return;
  const int NWe = max(1, min(c.nworkers, NI));
  if (c.worker >= NWe) return;
  const int i0 = range_lo(NI, c.worker, NWe), i1 = range_lo(NI, c.worker + 1, NWe);
  int pi = i0, pkt = 0;
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    if (pi >= i1) break;
    const int n = min(CU, KT - pkt);
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[k], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + k * (CU * kUnitBytes), down_item_src(G, c.rt, pi, pkt), static_cast<uint32_t>(n * kUnitBytes),
               &c.bars[k], c.pol);
    }
    pkt += n;
    if (pkt == KT) {
      pkt = 0;
      ++pi;
    }
  }
}

// Flush the per-warp row-strip tile `tile` ([T][16] fp32) of strip s.  Lane l handles the
// float4 groups q = l, l + 32, ... of the tile (token q / 4, rows 4 (q % 4) .. + 3); the
// partials of the other contributors are read four workers at a time.
__device__ __noinline__ void down_flush(const Params& p, float* tile, int layer, int s, int worker, int i0, int i1,
                                        int NI, int NWe, int nA) {
  const int lane = lane_id();
  const int n = p.T * 16, n4 = n / 4;
  const int s_lo = s * nA, s_hi = s_lo + nA;  // item range of the strip
  const bool full = (i0 <= s_lo && s_hi <= i1);
  float4* tile4 = reinterpret_cast<float4*>(tile);
  __syncwarp();
  if (!full) {
    const int slot = (i0 >= s_lo) ? 0 : 1;  // 0: the strip is this worker's first
    float4* dst = reinterpret_cast<float4*>(p.gpart + (static_cast<size_t>(worker) * 2 + slot) * n);
#pragma unroll 1
    for (int q = lane; q < n4; q += 32) dst[q] = tile4[q];
    __syncwarp();  // ordered before lane 0's release (as in gemv_flush)
    const int wf = worker_of(s_lo, NI, NWe), wl = worker_of(s_hi - 1, NI, NWe);
    unsigned old = 0;
    if (lane == 0) old = atom_acqrel_add_u32(&p.strip_cnt[s], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != static_cast<unsigned>(wl - wf)) {
#pragma unroll 1
      for (int q = lane; q < n4; q += 32) tile4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncwarp();
      return;
    }
    const int slot_f = (range_lo(NI, wf, NWe) >= s_lo) ? 0 : 1;
#pragma unroll 1
    for (int q = lane; q < n4; q += 32) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
      for (int w0 = wf; w0 <= wl; w0 += 4) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int w = w0 + u;
          v[u] = (w <= wl) ? ldcg_f4(p.gpart + (static_cast<size_t>(w) * 2 + (w == wf ? slot_f : 0)) * n + 4 * q)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          a.x += v[u].x;
          a.y += v[u].y;
          a.z += v[u].z;
          a.w += v[u].w;
        }
      }
      tile4[q] = a;
    }
    if (lane == 0) p.strip_cnt[s] = 0u;
  }
  if (p.n_ranks > 1) {
    // expert parallel: this rank's experts' sum for the strip, stored in every rank's region
#pragma unroll 1
    for (int q = lane; q < n4; q += 32) {
      const int t = q >> 2, row = s * 16 + 4 * (q & 3);
      const size_t off = static_cast<size_t>(t) * p.H + row;
      ll_put4(p, 1, layer, off, tile4[q]);
      tile4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();
    return;
  }
#pragma unroll 1
  for (int q = lane; q < n4; q += 32) {
    const int t = q >> 2, row = s * 16 + 4 * (q & 3);
    float4* x = reinterpret_cast<float4*>(p.resid + static_cast<size_t>(t) * p.H + row);
    const float4 old = p.residual ? *x : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 tv = tile4[q];
    const float4 nv = make_float4(old.x + rbf(tv.x), old.y + rbf(tv.y), old.z + rbf(tv.z), old.w + rbf(tv.w));
    *x = nv;
    if (p.tr_out)
      *reinterpret_cast<float4*>(p.tr_out + (static_cast<size_t>(layer - p.first_layer) * p.T + t) * p.H + row) = nv;
    tile4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncwarp();
}

template <int NT>
__device__ __noinline__ void down_stage(const Params& p, Ctx& cref, const GemvGeom& G) {
  using RG = RingGeom<NT>;
  constexpr int CU = RG::kChunk, NS = RG::kGemvSlots, NA = RG::kAccSets;
  Ctx c = cref;
  const int primed = c.primed;  // ring slots already filled
  cref.primed = 0;
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3, warp = threadIdx.x >> 5;
  const int nA = G.nseg, KT = G.kt, NI = G.sps * nA;
  if (NI <= 0) return;
  const int NWe = max(1, min(c.nworkers, NI));
  if (c.worker >= NWe) return;
  const int i0 = range_lo(NI, c.worker, NWe), i1 = range_lo(NI, c.worker + 1, NWe);
  if (i0 >= i1) return;
  const Route* rt = c.rt;
  float* tile = reinterpret_cast<float*>(c.xs) + warp * (p.T * 16);
#pragma unroll 1
  for (int e = lane; e < p.T * 16; e += 32) tile[e] = 0.f;
  __syncwarp();
  int pi = i0, pkt = 0;
  auto issue = [&](int slot, bool dry) {
    const int n = min(CU, KT - pkt);
    if (lane == 0 && !dry) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&c.bars[slot], static_cast<uint32_t>(n * kUnitBytes));
      bulk_g2s(c.ring + slot * (CU * kUnitBytes), down_item_src(G, rt, pi, pkt), static_cast<uint32_t>(n * kUnitBytes),
               &c.bars[slot], c.pol);
    }
    pkt += n;
    if (pkt == KT) {
      pkt = 0;
      ++pi;
    }
  };
#pragma unroll
  for (int k = 0; k < NS; ++k)
    if (pi < i1) issue(k, k < primed);
  float acc[NA][NT][4];
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
  int ci = i0, ckt = 0, cs = 0;
  int cj = ci % nA, ncols = rt->act_cnt[cj], off = rt->act_off[cj], ntiles = (ncols + 7) >> 3;
  const uint16_t* brow[NT];
  auto item_setup = [&]() {
    cj = ci % nA;
    ncols = rt->act_cnt[cj];
    off = rt->act_off[cj];
    ntiles = (ncols + 7) >> 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + g;
      brow[nt] = col < ncols ? p.hbuf + static_cast<size_t>(off + col) * p.I + 8 * t4 : nullptr;
    }
  };
  item_setup();
#pragma unroll 1
  while (ci < i1) {
    const int n = min(CU, KT - ckt);
    uint4 bf[CU][NT];
#pragma unroll
    for (int i = 0; i < CU; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        bf[i][nt] = (i < n && brow[nt]) ? ldcg128(brow[nt] + (ckt + i) * 32) : make_uint4(0, 0, 0, 0);
    slot_wait(p, c, cs);
    const uint4* sa = reinterpret_cast<const uint4*>(c.ring + cs * (CU * kUnitBytes)) + lane;
#pragma unroll
    for (int i = 0; i < CU; ++i) {
      if (i < n) {
        const uint4 a0 = sa[i * (kUnitBytes / 16)];
        const uint4 a1 = sa[i * (kUnitBytes / 16) + 32];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt < ntiles) {
            mma_bf16(acc[i % NA][nt], a0.x, a1.x, a0.y, a1.y, bf[i][nt].x, bf[i][nt].y);
            mma_bf16(acc[i % NA][nt], a0.z, a1.z, a0.w, a1.w, bf[i][nt].z, bf[i][nt].w);
          }
        }
      }
    }
    __syncwarp();
    if (pi < i1) issue(cs, false);
    cs = (cs + 1 == NS) ? 0 : cs + 1;
    ckt += n;
    if (ckt == KT) {
      // item done: scale by the affinity and add into the warp's row-strip tile
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = nt * 8 + 2 * t4 + e;
          float v0 = 0.f, v1 = 0.f;
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            v0 += acc[a][nt][e];
            v1 += acc[a][nt][2 + e];
          }
          if (col < ncols) {
            const int pair = off + col;
            const float w = rt->pair_w[pair];
            float* trow = tile + rt->pair_tok[pair] * 16;
            trow[g] += v0 * w;
            trow[g + 8] += v1 * w;
          }
        }
      }
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
      const int s_now = ci / nA;
      ++ci;
      ckt = 0;
      if (ci == i1 || ci / nA != s_now) down_flush(p, tile, G.layer, s_now, c.worker, i0, i1, NI, NWe, nA);
      if (ci < i1) item_setup();
    }
  }
  cref.phase = c.phase;
}

// ------------------------------------------------------------------ attention
// q/k head RMSNorm + RoPE for the 4 elements d = 4*lane .. 4*lane+3 of one head
// (rounding points of attn_fused_nki.py:393-451,494-586).
__device__ __forceinline__ void head_norm_rope(float (&x)[4], uint2 wv, uint2 cv, uint2 sv, float eps) {
  const int lane = lane_id();
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) s = __fadd_rn(s, __fmul_rn(x[j], x[j]));
  s = warp_sum_fixed(s);
  const float r = rstd_fixed(s, kHeadDim, eps);
  float xn[4], rot[4];
  const float wf[4] = {lo_bf(wv.x), hi_bf(wv.x), lo_bf(wv.y), hi_bf(wv.y)};
#pragma unroll
  for (int j = 0; j < 4; ++j) xn[j] = rbf(__fmul_rn(__fmul_rn(x[j], r), wf[j]));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float o = __shfl_xor_sync(0xffffffffu, xn[j], 16);
    rot[j] = lane < 16 ? -o : o;
  }
  const float cf[4] = {lo_bf(cv.x), hi_bf(cv.x), lo_bf(cv.y), hi_bf(cv.y)};
  const float sf[4] = {lo_bf(sv.x), hi_bf(sv.x), lo_bf(sv.y), hi_bf(sv.y)};
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = rbf(__fadd_rn(rbf(__fmul_rn(xn[j], cf[j])), rbf(__fmul_rn(rot[j], sf[j]))));
}

__device__ __forceinline__ void unpack4(uint2 v, float (&x)[4]) {
  x[0] = lo_bf(v.x);
  x[1] = hi_bf(v.x);
  x[2] = lo_bf(v.y);
  x[3] = hi_bf(v.y);
}

constexpr float kScoreScale = 0.08838834764831845f;  // 1/sqrt(128)
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float score_round(float acc) { return rbf(rbf(acc) * kScoreScale); }

// One raw bf16 head (4 elements per lane) and its norm weight and RoPE rows: loaded together,
// then normalised + rotated (head_finish) to bf16x4.
struct HeadIn {
  uint2 raw, w, c, s;
};
__device__ __forceinline__ HeadIn head_load(const uint16_t* src, const uint16_t* w, const uint16_t* cs,
                                            const uint16_t* sn) {
  const int lane = lane_id();
  HeadIn in;
  in.raw = ldcg64(src + 4 * lane);
  in.w = *reinterpret_cast<const uint2*>(w + 4 * lane);
  in.c = *reinterpret_cast<const uint2*>(cs + 4 * lane);
  in.s = *reinterpret_cast<const uint2*>(sn + 4 * lane);
  return in;
}
__device__ __noinline__ uint2 head_finish(HeadIn in, float eps) {
  float x[4];
  unpack4(in.raw, x);
  head_norm_rope(x, in.w, in.c, in.s, eps);
  return make_uint2(pack_bf2(x[0], x[1]), pack_bf2(x[2], x[3]));
}

// Per-warp flash-decode over the 32-token tiles tile_first, tile_first+step, ... of
// [tok_beg, tok_end).  Leaves the unnormalised (m, l, o) of rows g and g+8 in registers.
constexpr int kNoBlocks = -2;  // "block ids not preloaded"

// Block ids of the K/V blocks a context chunk [tok_beg, tok_end) touches: lane j holds the
// id of block tok_beg/128 + j (j < 32; -1 past the chunk).  One coalesced load per warp.
__device__ __forceinline__ bool bf16x4_empty(uint2 v) {
  return (v.x & 0xffffu) == kBf16Empty || (v.x >> 16) == kBf16Empty || (v.y & 0xffffu) == kBf16Empty ||
         (v.y >> 16) == kBf16Empty;
}

__device__ __forceinline__ int att_chunk_blocks(const Params& p, int b, int tok_beg, int tok_end) {
  const int j = tok_beg / kKvBlock + lane_id();
  const int jend = tok_end > tok_beg ? (tok_end - 1) / kKvBlock : -1;
  return (j <= jend && j < p.max_blocks) ? __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + j) : -1;
}

// TMA box bi of this warp's tiles (tile bi/4; boxes K d0-63, K d64-127, V d0-63, V d64-127)
// into ring slot `slot`.  All lanes call it (the block id is shuffled from blk_lane); lane 0
// issues the copy.
__device__ __noinline__ void att_issue_box(const Params& p, Ctx& c, int layer, int b, int h, int tok_beg,
                                              int tile_first, int tile_step, int blk_lane, int bi, int slot,
                                              const CUtensorMap* kmap, const CUtensorMap* vmap) {
  const int tile = tile_first + (bi >> 2) * tile_step, kind = bi & 3;
  const int tok0 = tok_beg + tile * kAttTile;
  const int off = tok0 / kKvBlock - tok_beg / kKvBlock;
  int blk = __shfl_sync(0xffffffffu, blk_lane, off & 31);
  if (off >= 32) blk = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + tok0 / kKvBlock);
  if (lane_id() == 0) {
    if (blk < 0 || blk >= p.num_blocks) {
      set_status(p, kStatusIndex);
      blk = 0;
    }
    const size_t head_rows = static_cast<size_t>(layer) * p.num_blocks;
    const int row = static_cast<int>(((head_rows + blk) * p.nkv + h) * kKvBlock + (tok0 % kKvBlock));
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&c.bars[slot], kSlotBytes);
    tma_load_2d(c.ring + slot * kSlotBytes, kind < 2 ? kmap : vmap, (kind & 1) * 64, row, &c.bars[slot]);
  }
}

__device__ __forceinline__ int att_ntile(int tok_beg, int tok_end, int tile_first, int tile_step) {
  const int ntile_all = tok_end > tok_beg ? (tok_end - tok_beg + kAttTile - 1) / kAttTile : 0;
  return ntile_all > tile_first ? (ntile_all - tile_first + tile_step - 1) / tile_step : 0;
}

// Fill the warp's ring with its first boxes (before the q heads are staged, so that the K/V
// copies overlap the staging).  Returns the number of boxes issued.
__device__ __forceinline__ int att_prime(const Params& p, Ctx& c, int layer, int b, int h, int tok_beg, int tok_end,
                                         int tile_first, int tile_step, int blk_lane, const CUtensorMap* kmap,
                                         const CUtensorMap* vmap) {
  const int nbox = 4 * att_ntile(tok_beg, tok_end, tile_first, tile_step);
  int pb = 0, ps = c.head;
  for (; pb < nbox && pb < c.nslot; ++pb) {
    att_issue_box(p, c, layer, b, h, tok_beg, tile_first, tile_step, blk_lane, pb, ps, kmap, vmap);
    ps = (ps + 1 == c.nslot) ? 0 : ps + 1;
  }
  return pb;
}

__device__ __forceinline__ void attention_tiles(const Params& p, Ctx& c, int layer, int b, int h, int tok_beg, int tok_end,
                                int tile_first, int tile_step, int blk_lane, int pb, const uint32_t (&qa)[8][4],
                                float (&m)[2], float (&l)[2], float (&o)[16][4], const CUtensorMap* kmap,
                                const CUtensorMap* vmap) {
  const int lane = lane_id(), t4 = lane & 3;
  const int ntile = att_ntile(tok_beg, tok_end, tile_first, tile_step);
  const int nbox = 4 * ntile;
  auto next_slot = [&](int s) { return (s + 1 == c.nslot) ? 0 : s + 1; };
  auto refill = [&](int slot) {
    __syncwarp();
    if (pb < nbox) {
      att_issue_box(p, c, layer, b, h, tok_beg, tile_first, tile_step, blk_lane, pb, slot, kmap, vmap);
      ++pb;
    }
  };
  int cs = c.head;
#pragma unroll 1
  for (int i = 0; i < ntile; ++i) {
    const int tok0 = tok_beg + (tile_first + i * tile_step) * kAttTile;
    const int nvalid = min(kAttTile, tok_end - tok0);
    // ---- S = Q K^T  (16 rows x 32 tokens)
    const int sk0 = cs, sk1 = next_slot(cs);
    slot_wait(p, c, sk0);
    slot_wait(p, c, sk1);
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
      const uint32_t box = smem_addr(c.ring + (kp < 2 ? sk0 : sk1) * kSlotBytes);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = 8 * j + (lane & 7);
        const int chunk = 4 * (kp & 1) + (lane >> 3);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(box + row * 128 + ((chunk ^ (row & 7)) << 4), r0, r1, r2, r3);
        mma_bf16(sc[j], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], r0, r1);
        mma_bf16(sc[j], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], r2, r3);
      }
    }
    refill(sk0);
    refill(sk1);
    cs = next_slot(sk1);
    // ---- online softmax (rows g and g+8 of this lane)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool valid = (8 * j + 2 * t4 + e) < nvalid;
        sc[j][e] = valid ? score_round(sc[j][e]) : -INFINITY;
        sc[j][2 + e] = valid ? score_round(sc[j][2 + e]) : -INFINITY;
        mx0 = fmaxf(mx0, sc[j][e]);
        mx1 = fmaxf(mx1, sc[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
    const float al0 = exp2f((m[0] - mn0) * kLog2e), al1 = exp2f((m[1] - mn1) * kLog2e);
    m[0] = mn0;
    m[1] = mn1;
    l[0] *= al0;
    l[1] *= al1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
    }
    uint32_t pa[2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p0 = exp2f((sc[j][0] - mn0) * kLog2e), p1 = exp2f((sc[j][1] - mn0) * kLog2e);
      const float p2 = exp2f((sc[j][2] - mn1) * kLog2e), p3 = exp2f((sc[j][3] - mn1) * kLog2e);
      l[0] += p0 + p1;
      l[1] += p2 + p3;
      const int ks = j >> 1;
      if ((j & 1) == 0) {
        pa[ks][0] = pack_bf2(p0, p1);
        pa[ks][1] = pack_bf2(p2, p3);
      } else {
        pa[ks][2] = pack_bf2(p0, p1);
        pa[ks][3] = pack_bf2(p2, p3);
      }
    }
    // ---- O += P V  (two boxes: d 0..63, d 64..127)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int sv = cs;
      slot_wait(p, c, sv);
      uint8_t* vbox = c.ring + sv * kSlotBytes;
      if (nvalid < kAttTile) {  // rows past the end of the context may hold anything
        for (int idx = lane; idx < (kAttTile - nvalid) * 8; idx += 32)
          reinterpret_cast<uint4*>(vbox + nvalid * 128)[idx] = make_uint4(0, 0, 0, 0);
        __syncwarp();
      }
      const uint32_t vb = smem_addr(vbox);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int row = 16 * ks + ((lane >> 3) & 1) * 8 + (lane & 7);
          const int chunk = 2 * np + (lane >> 4);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(vb + row * 128 + ((chunk ^ (row & 7)) << 4), r0, r1, r2, r3);
          const int nt = half * 8 + 2 * np;
          mma_bf16(o[nt], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], r0, r1);
          mma_bf16(o[nt + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], r2, r3);
        }
      }
      refill(sv);
      cs = next_slot(sv);
    }
  }
  c.head = cs;
}

// One (sequence b, kv head h, context chunk ch) item, processed by the whole CTA.
__device__ __forceinline__ void attention_cta_body(const Params& p, Ctx& c, int layer, int b, int h, int ch, int nch,
                                                  int CT, int item, int pos, int blk_pre, const CUtensorMap* kmap,
                                                  const CUtensorMap* vmap) {
  const int warp = threadIdx.x >> 5, lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int tok_beg = ch * CT;
  const int tok_end = min(pos, (ch + 1) * CT);
  const bool last = (ch == nch - 1);
  uint16_t* qs = reinterpret_cast<uint16_t*>(c.att);
  uint16_t* kn = qs + kAttRows * kAttQStride;
  uint16_t* vn = kn + kHeadDim;
  float* wml = reinterpret_cast<float*>(vn + kHeadDim);  // [warp][m 16 | l 16]
  int* cflag = reinterpret_cast<int*>(wml + kWarps * 2 * kAttRows);
  const int prow = min(pos, p.rope_max - 1);
  const uint16_t* cosr = p.rope_cos + static_cast<size_t>(prow) * kHeadDim;
  const uint16_t* sinr = p.rope_sin + static_cast<size_t>(prow) * kHeadDim;
  const LayerPtrs& lw = c.lt[layer - p.first_layer];
  const uint16_t* qkv_b = p.qkv + static_cast<size_t>(b) * p.R;
  const int blk_lane = blk_pre != kNoBlocks ? blk_pre : att_chunk_blocks(p, b, tok_beg, tok_end);
  const int pb = c.att_pb >= 0 ? c.att_pb : att_prime(p, c, layer, b, h, tok_beg, tok_end, warp, kWarps, blk_lane, kmap, vmap);
  c.att_pb = -1;

  // --- stage the q heads (rows warp, warp + 8) and, in the last chunk, the new token's K
  // (warp 7) and V (warp 6); every load is issued before the first one is used
  const bool do_k = last && warp == kWarps - 1, do_v = last && warp == kWarps - 2;
  HeadIn qin[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = warp + i * kWarps;
    qin[i] = r < p.grp ? head_load(qkv_b + static_cast<size_t>(h * p.grp + r) * kHeadDim, lw.qn, cosr, sinr)
                       : HeadIn{};
  }
  HeadIn kin{};
  uint2 vv = make_uint2(0u, 0u);
  int wblk = -1;
  if (do_k) kin = head_load(qkv_b + static_cast<size_t>(p.nq + h) * kHeadDim, lw.kn, cosr, sinr);
  if (do_v) vv = ldcg64(qkv_b + static_cast<size_t>(p.nq + p.nkv + h) * kHeadDim + 4 * lane);
  if (do_k || do_v) wblk = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + pos / kKvBlock);
  if (c.awaitq) {
    // no grid barrier before this stage: re-read the elements still unwritten (bounded wait)
    uint64_t t0 = 0;
#pragma unroll 1
    for (uint32_t it = 0;; ++it) {
      const bool q0 = warp < p.grp && bf16x4_empty(qin[0].raw);
      const bool q1 = warp + kWarps < p.grp && bf16x4_empty(qin[1].raw);
      const bool kk = do_k && bf16x4_empty(kin.raw), vq = do_v && bf16x4_empty(vv);
      if (!__any_sync(0xffffffffu, q0 || q1 || kk || vq)) break;
      if ((it & 15u) == 0) {
        const uint64_t now = globaltimer_ns();
        if (it == 0) t0 = now;
        if ((ld_volatile_i32(p.status) & kStatusFatal) || now - t0 > kWaitLimitNs) {
          if (lane == 0) set_status(p, kStatusFatal);
          break;
        }
      }
      __nanosleep(100);
      if (q0) qin[0].raw = ldcg64(qkv_b + static_cast<size_t>(h * p.grp + warp) * kHeadDim + 4 * lane);
      if (q1) qin[1].raw = ldcg64(qkv_b + static_cast<size_t>(h * p.grp + warp + kWarps) * kHeadDim + 4 * lane);
      if (kk) kin.raw = ldcg64(qkv_b + static_cast<size_t>(p.nq + h) * kHeadDim + 4 * lane);
      if (vq) vv = ldcg64(qkv_b + static_cast<size_t>(p.nq + p.nkv + h) * kHeadDim + 4 * lane);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = warp + i * kWarps;
    const uint2 out = r < p.grp ? head_finish(qin[i], p.eps) : make_uint2(0u, 0u);
    *reinterpret_cast<uint2*>(qs + r * kAttQStride + 4 * lane) = out;
  }
  if (do_k || do_v) {
    const uint2 val = do_k ? head_finish(kin, p.eps) : vv;
    *reinterpret_cast<uint2*>((do_k ? kn : vn) + 4 * lane) = val;
    if (p.stages & 16) {
      // written by kv_prewrite before this stage
    } else if (wblk >= 0 && wblk < p.num_blocks) {
      const size_t off = ((static_cast<size_t>(layer) * p.num_blocks + wblk) * p.nkv + h) * kKvBlock * kHeadDim +
                         static_cast<size_t>(pos % kKvBlock) * kHeadDim + 4 * lane;
      *reinterpret_cast<uint2*>((do_k ? p.k_pool : p.v_pool) + off) = val;
    } else if (wblk >= p.num_blocks && lane == 0) {
      set_status(p, kStatusIndex);
    }
  }
  __syncthreads();
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint16_t* a0 = qs + g * kAttQStride + 16 * ks + 2 * t4;
    const uint16_t* a1 = qs + (g + 8) * kAttQStride + 16 * ks + 2 * t4;
    qa[ks][0] = *reinterpret_cast<const uint32_t*>(a0);
    qa[ks][1] = *reinterpret_cast<const uint32_t*>(a1);
    qa[ks][2] = *reinterpret_cast<const uint32_t*>(a0 + 8);
    qa[ks][3] = *reinterpret_cast<const uint32_t*>(a1 + 8);
  }
  float m[2] = {-1e30f, -1e30f}, l[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  attention_tiles(p, c, layer, b, h, tok_beg, tok_end, warp, kWarps, blk_lane, pb, qa, m, l, o, kmap, vmap);

  // --- the active token (position pos): score with the fresh K, value the fresh V
  if (last && warp == 0) {
    float d0 = 0.f, d1 = 0.f;
    for (int d = 32 * t4; d < 32 * t4 + 32; d += 2) {
      const uint32_t kw = *reinterpret_cast<const uint32_t*>(kn + d);
      const uint32_t q0 = *reinterpret_cast<const uint32_t*>(qs + g * kAttQStride + d);
      const uint32_t q1 = *reinterpret_cast<const uint32_t*>(qs + (g + 8) * kAttQStride + d);
      d0 = fmaf(lo_bf(q0), lo_bf(kw), fmaf(hi_bf(q0), hi_bf(kw), d0));
      d1 = fmaf(lo_bf(q1), lo_bf(kw), fmaf(hi_bf(q1), hi_bf(kw), d1));
    }
    d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
    d0 += __shfl_xor_sync(0xffffffffu, d0, 2);
    d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
    d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
    const float s0 = score_round(d0), s1 = score_round(d1);
    const float mn0 = fmaxf(m[0], s0), mn1 = fmaxf(m[1], s1);
    const float al0 = exp2f((m[0] - mn0) * kLog2e), al1 = exp2f((m[1] - mn1) * kLog2e);
    const float pa0 = exp2f((s0 - mn0) * kLog2e), pa1 = exp2f((s1 - mn1) * kLog2e);
    m[0] = mn0;
    m[1] = mn1;
    l[0] = l[0] * al0 + (t4 == 0 ? pa0 : 0.f);
    l[1] = l[1] * al1 + (t4 == 0 ? pa1 : 0.f);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const uint32_t vw = *reinterpret_cast<const uint32_t*>(vn + 8 * nt + 2 * t4);
      o[nt][0] = o[nt][0] * al0 + pa0 * lo_bf(vw);
      o[nt][1] = o[nt][1] * al0 + pa0 * hi_bf(vw);
      o[nt][2] = o[nt][2] * al1 + pa1 * lo_bf(vw);
      o[nt][3] = o[nt][3] * al1 + pa1 * hi_bf(vw);
    }
  }
  l[0] += __shfl_xor_sync(0xffffffffu, l[0], 1);
  l[0] += __shfl_xor_sync(0xffffffffu, l[0], 2);
  l[1] += __shfl_xor_sync(0xffffffffu, l[1], 1);
  l[1] += __shfl_xor_sync(0xffffffffu, l[1], 2);

  // --- per-warp partials into the warp's own (drained) ring; (m, l) into the shared table
  float* po = reinterpret_cast<float*>(c.ring);  // [16][128]
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = 8 * nt + 2 * t4;
    *reinterpret_cast<float2*>(po + g * kHeadDim + d) = make_float2(o[nt][0], o[nt][1]);
    *reinterpret_cast<float2*>(po + (g + 8) * kHeadDim + d) = make_float2(o[nt][2], o[nt][3]);
  }
  if (t4 == 0) {
    wml[warp * 2 * kAttRows + g] = m[0];
    wml[warp * 2 * kAttRows + g + 8] = m[1];
    wml[warp * 2 * kAttRows + kAttRows + g] = l[0];
    wml[warp * 2 * kAttRows + kAttRows + g + 8] = l[1];
  }
  __syncthreads();
  // --- CTA combine over the 8 warps: warp w owns rows w and w+8
  const size_t out_row = static_cast<size_t>(b) * (p.nq * kHeadDim);
  float* part = p.att_part + static_cast<size_t>(item) * kPartFloats;
  for (int r = warp; r < p.grp; r += kWarps) {
    float M = -1e30f;
#pragma unroll 1
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wml[w * 2 * kAttRows + r]);
    float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int w = 0; w < kWarps; ++w) {
      const float sc = exp2f((wml[w * 2 * kAttRows + r] - M) * kLog2e);
      L += wml[w * 2 * kAttRows + kAttRows + r] * sc;
      const float4 v = *reinterpret_cast<const float4*>(
          reinterpret_cast<const float*>(c.ring_all + w * c.ring_bytes) + r * kHeadDim + 4 * lane);
      acc[0] += v.x * sc;
      acc[1] += v.y * sc;
      acc[2] += v.z * sc;
      acc[3] += v.w * sc;
    }
    if (nch == 1) {
      const float il = 1.f / L;
      *reinterpret_cast<uint2*>(p.attn_out + out_row + static_cast<size_t>(h * p.grp + r) * kHeadDim + 4 * lane) =
          make_uint2(pack_bf2(acc[0] * il, acc[1] * il), pack_bf2(acc[2] * il, acc[3] * il));
    } else {
      if (lane == 0) {
        part[r] = M;
        part[kAttRows + r] = L;
      }
      *reinterpret_cast<float4*>(part + 2 * kAttRows + r * kHeadDim + 4 * lane) =
          make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
  }
  if (nch == 1) {
    __syncthreads();  // the rings are reused by the next item
    return;
  }
  // --- split context: the last CTA of (b, h) combines the chunk partials in chunk order.
  // The CTA barrier orders every thread's partial stores before thread 0's acq_rel update;
  // the second barrier orders the last CTA's partial reads after thread 0's acquire.
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atom_acqrel_add_u32(&p.attn_cnt[b * p.nkv + h], 1u);
    *cflag = (old == static_cast<unsigned>(nch - 1));
  }
  __syncthreads();
  if (!*cflag) return;
  const int item0 = item - ch;  // items of one (b, h) are consecutive, chunk-major
  for (int r = warp; r < p.grp; r += kWarps) {
    // lane k holds chunk k's (m, l) (chunks beyond 32 are folded in a loop)
    float M = -1e30f;
    for (int k0 = 0; k0 < nch; k0 += 32) {
      const int k = k0 + lane;
      if (k < nch) M = fmaxf(M, ldcg_f(p.att_part + static_cast<size_t>(item0 + k) * kPartFloats + r));
    }
    M = warp_max(M);
    float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int k0 = 0; k0 < nch; k0 += 4) {
      float4 v[4];
      float ms[4], ls[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (k0 + u < nch) {
          const float* pk = p.att_part + static_cast<size_t>(item0 + k0 + u) * kPartFloats;
          ms[u] = ldcg_f(pk + r);
          ls[u] = ldcg_f(pk + kAttRows + r);
          v[u] = ldcg_f4(pk + 2 * kAttRows + r * kHeadDim + 4 * lane);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (k0 + u < nch) {
          const float sc = exp2f((ms[u] - M) * kLog2e);
          L += ls[u] * sc;
          acc[0] += v[u].x * sc;
          acc[1] += v[u].y * sc;
          acc[2] += v[u].z * sc;
          acc[3] += v[u].w * sc;
        }
      }
    }
    const float il = 1.f / L;
    *reinterpret_cast<uint2*>(p.attn_out + out_row + static_cast<size_t>(h * p.grp + r) * kHeadDim + 4 * lane) =
        make_uint2(pack_bf2(acc[0] * il, acc[1] * il), pack_bf2(acc[2] * il, acc[3] * il));
  }
  if (threadIdx.x == 0) p.attn_cnt[b * p.nkv + h] = 0u;
  __syncthreads();
}

__device__ __noinline__ void attention_cta_item(const Params& p, Ctx& cref, int layer, int b, int h, int ch, int nch,
                                                int CT, int item, int pos, int blk_pre, const CUtensorMap* kmap,
                                                const CUtensorMap* vmap) {
  Ctx c = cref;  // register-resident copy
  attention_cta_body(p, c, layer, b, h, ch, nch, CT, item, pos, blk_pre, kmap, vmap);
  cref.head = c.head;
  cref.phase = c.phase;
  cref.att_pb = -1;
}

// Chunk length CT (multiple of 32) such that the (b, h, chunk) items fill the grid once, and
// the items of this CTA.  Lane b holds sequence b's position (batch <= 32).  Calls fn(b, h, ch,
// nch, CT, item, pos) for each item of this CTA, in order.
template <class Fn>
__device__ __forceinline__ void att_items(const Params& p, Fn&& fn) {
  const int G = gridDim.x, lane = lane_id();
  const int mypos = lane < p.T ? seq_pos(p, lane) : 0;
  const int mytiles = lane < p.T ? (mypos + kAttTile - 1) / kAttTile : 0;
  int tiles = p.nkv * mytiles, longest = max(1, mytiles);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    tiles += __shfl_xor_sync(0xffffffffu, tiles, off);
    longest = max(longest, __shfl_xor_sync(0xffffffffu, longest, off));
  }
  // Batches of at most 8 rows: at most one item per CTA.  Larger batches (long and unequal contexts
  // at B = 32) take up to kAttItemsWide items per CTA of a smaller chunk, so that the round-robin
  // assignment balances the CTAs' token counts.
  const int cap = p.T > 8 ? kAttItemsWide * G : G;
  int per = max(1, (tiles + cap - 1) / cap);
  int nitems = 0;
  for (;; ++per) {
    int mine = lane < p.T ? p.nkv * max(1, (mypos + kAttTile * per - 1) / (kAttTile * per)) : 0;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, off);
    nitems = mine;
    if (nitems <= cap || per >= longest) break;
  }
  const int CT = kAttTile * per;
  // inclusive prefix of the items of sequences 0..lane
  const int mynch = lane < p.T ? max(1, (mypos + CT - 1) / CT) : 0;
  int incl = p.nkv * mynch;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  for (int it = blockIdx.x; it < nitems; it += G) {
    const unsigned before = __ballot_sync(0xffffffffu, lane < p.T && incl <= it);
    const int b = __popc(before);  // sequences whose items all precede `it`
    const int base = b > 0 ? __shfl_sync(0xffffffffu, incl, b - 1) : 0;
    const int nch = __shfl_sync(0xffffffffu, mynch, b);
    const int pos = __shfl_sync(0xffffffffu, mypos, b);
    const int r = it - base;
    fn(b, r / nch, r % nch, nch, CT, it, pos);
  }
}

// Plan this CTA's attention items for the launch (all threads call it; warp 0 writes).
__device__ __noinline__ void att_plan_build(const Params& p, Ctx& c) {
  AttPlan* pl = c.plan;
  const bool w0 = (threadIdx.x >> 5) == 0;
  int n = 0;
  att_items(p, [&](int b, int h, int ch, int nch, int CT, int item, int pos) {
    if (n < kMaxAttItems && w0) {
      pl->b[n] = b;
      pl->h[n] = h;
      pl->ch[n] = ch;
      pl->nch[n] = nch;
      pl->pos[n] = pos;
      pl->item[n] = item;
      pl->CT = CT;
      pl->blk[n][lane_id()] = att_chunk_blocks(p, b, ch * CT, min(pos, (ch + 1) * CT));
    }
    ++n;
  });
  if (w0 && lane_id() == 0) pl->n = n <= kMaxAttItems ? n : -1;
}

// Issue the first K/V boxes of this CTA's first attention item of `layer` into the warp's
// (drained) ring, so that they stream while the grid barrier before the attention completes.
__device__ __noinline__ void att_prime_layer(const Params& p, Ctx& c, int layer, const CUtensorMap* kmap,
                                             const CUtensorMap* vmap) {
  const AttPlan* pl = c.plan;
  if (pl->n <= 0) return;
  const int warp = threadIdx.x >> 5;
  const int tok_beg = pl->ch[0] * pl->CT, tok_end = min(pl->pos[0], (pl->ch[0] + 1) * pl->CT);
  c.att_pb = att_prime(p, c, layer, pl->b[0], pl->h[0], tok_beg, tok_end, warp, kWarps, pl->blk[0][lane_id()], kmap,
                       vmap);
}

// More items per CTA than the plan holds: plan them again at every layer.
__device__ __noinline__ void attention_unplanned(const Params& p, Ctx& c, int layer, const CUtensorMap* kmap,
                                                 const CUtensorMap* vmap) {
  att_items(p, [&](int b, int h, int ch, int nch, int CT, int item, int pos) {
    attention_cta_item(p, c, layer, b, h, ch, nch, CT, item, pos, kNoBlocks, kmap, vmap);
  });
}

// Rows of one sequence at consecutive positions in one launch (multi-token decode, chunked
// prefill; stages bit 16): every row's new K (q/k-norm + RoPE, the values stage B computes) and V
// are stored into the cache before any attention reads it, so a row's context includes the rows
// at earlier positions.  One warp per (row, kv head, K or V).
__device__ __noinline__ void kv_prewrite(const Params& p, Ctx& c, int layer) {
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const LayerPtrs& lw = c.lt[layer - p.first_layer];
  const int n = p.T * p.nkv;
#pragma unroll 1
  for (int it = blockIdx.x * kWarps + warp; it < 2 * n; it += gridDim.x * kWarps) {
    const int kind = it / n;
    const int r = it - kind * n, b = r / p.nkv, h = r - b * p.nkv;
    const int pos = seq_pos(p, b);
    const int wblk = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + pos / kKvBlock);
    const uint16_t* qkv_b = p.qkv + static_cast<size_t>(b) * p.R;
    uint2 val;
    if (kind == 0) {
      const int prow = min(pos, p.rope_max - 1);
      const HeadIn kin = head_load(qkv_b + static_cast<size_t>(p.nq + h) * kHeadDim, lw.kn,
                                   p.rope_cos + static_cast<size_t>(prow) * kHeadDim,
                                   p.rope_sin + static_cast<size_t>(prow) * kHeadDim);
      val = head_finish(kin, p.eps);
    } else {
      val = ldcg64(qkv_b + static_cast<size_t>(p.nq + p.nkv + h) * kHeadDim + 4 * lane);
    }
    if (wblk >= 0 && wblk < p.num_blocks) {
      const size_t off = ((static_cast<size_t>(layer) * p.num_blocks + wblk) * p.nkv + h) * kKvBlock * kHeadDim +
                         static_cast<size_t>(pos % kKvBlock) * kHeadDim + 4 * lane;
      *reinterpret_cast<uint2*>((kind == 0 ? p.k_pool : p.v_pool) + off) = val;
    } else if (wblk >= p.num_blocks && lane == 0) {
      set_status(p, kStatusIndex);
    }
  }
}

__device__ __noinline__ void attention_stage(const Params& p, Ctx& c, int layer, const CUtensorMap* kmap, const CUtensorMap* vmap) {
  const AttPlan* pl = c.plan;
  if (pl->n < 0) {
    attention_unplanned(p, c, layer, kmap, vmap);
    return;
  }
#pragma unroll 1
  for (int k = 0; k < pl->n; ++k)
    attention_cta_item(p, c, layer, pl->b[k], pl->h[k], pl->ch[k], pl->nch[k], pl->CT, pl->item[k], pl->pos[k],
                       pl->blk[k][lane_id()], kmap, vmap);
}

// ------------------------------------------------------------------ router (stage D)
// fp32 logits of (token, expert) items, one warp per item, fixed summation order
// (moe_fused_nki.py:186-218).
// x32: fp32 normalised rows in shared memory (row stride H), or nullptr to normalise on the
// fly from the residual with the per-CTA rstd (large batches whose rows do not fit).
template <bool kX32>
__device__ __noinline__ void router_stage(const Params& p, Ctx& c, int layer, const float* x32) {
  const int lane = lane_id();
  const LayerPtrs& lw = c.lt[layer - p.first_layer];
  const int nitems = p.T * p.E;
#pragma unroll 1
  for (int it = c.worker; it < nitems; it += c.nworkers) {
    const int t = it / p.E, e = it % p.E;
    const uint16_t* wr = lw.router + static_cast<size_t>(e) * p.H;
    const float r = c.rstd[t];
    // all weight loads of the row first: one memory latency per item, not one per group
    uint4 wv[kHidGroups];
#pragma unroll
    for (int i = 0; i < kHidGroups; ++i)
      wv[i] = (i < p.H / 256) ? ldnc128(wr + 256 * i + 8 * lane) : make_uint4(0u, 0u, 0u, 0u);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kHidGroups; ++i) {
      if (i < p.H / 256) {
        const int k0 = 256 * i + 8 * lane;
        const uint4 w4 = wv[i];
        float xv[8];
        if (kX32) {
          const float4 x0 = *reinterpret_cast<const float4*>(x32 + static_cast<size_t>(t) * p.H + k0);
          const float4 x1 = *reinterpret_cast<const float4*>(x32 + static_cast<size_t>(t) * p.H + k0 + 4);
          xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
          xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
        } else {
          const float4 x0 = ldcg_f4(p.resid + static_cast<size_t>(t) * p.H + k0);
          const float4 x1 = ldcg_f4(p.resid + static_cast<size_t>(t) * p.H + k0 + 4);
          const uint4 g4 = ldnc128(lw.ln2 + k0);
          const float raw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
          for (int j = 0; j < 8; ++j)
            xv[j] = __fmul_rn(__fmul_rn(raw[j], (j & 1) ? hi_bf(gw[j >> 1]) : lo_bf(gw[j >> 1])), r);
        }
        const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float wj = (j & 1) ? hi_bf(ww[j >> 1]) : lo_bf(ww[j >> 1]);
          s = __fadd_rn(s, __fmul_rn(wj, xv[j]));
        }
      }
    }
    s = warp_sum_fixed(s);
    if (lw.router_bias) s = __fadd_rn(s, __ldg(lw.router_bias + e));
    if (lane == 0) {
      p.rlogits[it] = s;
      if (p.tr_rlogits) p.tr_rlogits[static_cast<size_t>(layer - p.first_layer) * nitems + it] = s;
    }
  }
}

// ------------------------------------------------------------------ staged norms (batch <= 8)
// RMSNorm of stage A and fused RMSNorm + router logits of stage D for batches of at most kWarps
// tokens whose residual row fits one GEMV ring slot.  Warp t copies token t's residual row into
// slot 1 of its ring with one bulk copy (when every SM reads the same rows right after a grid
// barrier, one bulk copy per row lands several times sooner than per-thread loads of it),
// normalises it into X and, in stage D, replaces the staged row by its fp32 normalised values
// and scores them against the router rows of this CTA's experts (e = blockIdx.x, blockIdx.x + G,
// ...), so the stage needs no CTA barrier.  The norm's gamma (and in stage D the router row of
// expert blockIdx.x) are copied into the strip-reduction area while the grid barrier before the
// stage completes (norm_prefetch).  Both stages run the same code: it executes cold in the
// instruction cache once per layer, so the loops stay rolled.  Products and summation orders are
// those of norm_rows_to_smem and router_stage: X and the logits are bit-identical to theirs.
template <int NT>
__device__ __forceinline__ bool norm_staged_ok(const Params& p) {
  return NT == 1 && p.T <= kWarps && p.H * 4 <= RingGeom<NT>::kChunk * kUnitBytes;
}
// Call with every thread, after a CTA barrier that ends the strip-reduction area's previous use.
// router: the layer's router weights in stage D (the row of expert blockIdx.x is copied too).
__device__ __noinline__ void norm_prefetch(const Params& p, Ctx& c, const uint16_t* gamma, const uint16_t* router) {
  if (threadIdx.x == 0) {
    const uint32_t hb = static_cast<uint32_t>(p.H) * 2u;
    const bool has_e = router && static_cast<int>(blockIdx.x) < p.E;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(c.cbar, has_e ? 2u * hb : hb);
    bulk_g2s_plain(c.red, gamma, hb, c.cbar);
    if (has_e)
      bulk_g2s_plain(reinterpret_cast<uint8_t*>(c.red) + hb, router + static_cast<size_t>(blockIdx.x) * p.H, hb,
                     c.cbar);
  }
  c.npref = 1;
}

// gamma: the norm's weights (ln1, ln2 or the final norm); d: stage D (router logits of `layer`).
__device__ __noinline__ void norm_staged(const Params& p, Ctx& c, int layer, bool d, const uint16_t* gamma) {
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const int H = p.H, ng = H / 256, E = p.E;
  const LayerPtrs& lw = c.lt[layer - p.first_layer];
  float* stage = reinterpret_cast<float*>(c.ring + RingGeom<1>::kChunk * kUnitBytes);
  const bool mine = warp < p.T;
  if (mine && lane == 0) {
    fence_proxy_async_smem();    // earlier generic accesses of the staging slot
    fence_proxy_async_global();  // the residual was written by other CTAs during this launch
    mbar_arrive_expect_tx(&c.bars[1], static_cast<uint32_t>(H) * 4u);
    bulk_g2s_plain(stage, p.resid + static_cast<size_t>(warp) * H, static_cast<uint32_t>(H) * 4u, &c.bars[1]);
  }
  if (!c.npref) {  // not prefetched during the barrier (a stage launched on its own)
    __syncthreads();
    norm_prefetch(p, c, gamma, d ? lw.router : nullptr);
  }
  c.npref = 0;
  {
    const uint32_t par = c.cphase & 1u;
    if (!mbar_try_wait(c.cbar, par)) mbar_wait_slow(p, c.cbar, par);
    c.cphase ^= 1u;
  }
  if (!mine) return;
  slot_wait(p, c, 1);
  // RMSNorm ((x*r)*g in stage A, (x*g)*r in stage D) into X; in stage D the fp32 normalised row
  // also replaces the staged one
  float* row = stage + 8 * lane;
  float ss = 0.f;
#pragma unroll 2
  for (int i = 0; i < ng; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(row + 256 * i);
    const float4 b = *reinterpret_cast<const float4*>(row + 256 * i + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  }
  const float r = rstd_fixed(warp_sum_fixed(ss), H, p.eps);
  if (lane == 0) c.rstd[warp] = r;
  const uint16_t* gs = reinterpret_cast<const uint16_t*>(c.red) + 8 * lane;
  uint16_t* xr = c.xs + static_cast<size_t>(warp) * c.xs_stride + 8 * lane;
#pragma unroll 2
  for (int i = 0; i < ng; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(row + 256 * i);
    const float4 b = *reinterpret_cast<const float4*>(row + 256 * i + 4);
    const uint4 gv = *reinterpret_cast<const uint4*>(gs + 256 * i);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = (j & 1) ? hi_bf(gw[j >> 1]) : lo_bf(gw[j >> 1]);
      y[j] = __fmul_rn(__fmul_rn(v[j], d ? g : r), d ? r : g);
    }
    *reinterpret_cast<uint4*>(xr + 256 * i) =
        make_uint4(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]), pack_bf2(y[4], y[5]), pack_bf2(y[6], y[7]));
    if (d) {
      *reinterpret_cast<float4*>(row + 256 * i) = make_float4(y[0], y[1], y[2], y[3]);
      *reinterpret_cast<float4*>(row + 256 * i + 4) = make_float4(y[4], y[5], y[6], y[7]);
    }
  }
  if (!d) return;
  // router logits (token warp, expert e); the row of expert blockIdx.x is in shared memory
  const int nitems = p.T * E;
#pragma unroll 1
  for (int e = blockIdx.x; e < E; e += gridDim.x) {
    const bool sm = e == static_cast<int>(blockIdx.x);
    const uint16_t* wr = (sm ? reinterpret_cast<const uint16_t*>(c.red) + H : lw.router + static_cast<size_t>(e) * H) +
                         8 * lane;
    float acc = 0.f;
#pragma unroll 2
    for (int i = 0; i < ng; ++i) {
      const uint4 w4 = sm ? *reinterpret_cast<const uint4*>(wr + 256 * i) : ldnc128(wr + 256 * i);
      const float4 a = *reinterpret_cast<const float4*>(row + 256 * i);
      const float4 b = *reinterpret_cast<const float4*>(row + 256 * i + 4);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn((j & 1) ? hi_bf(ww[j >> 1]) : lo_bf(ww[j >> 1]), v[j]));
    }
    acc = warp_sum_fixed(acc);
    if (lw.router_bias) acc = __fadd_rn(acc, __ldg(lw.router_bias + e));
    if (lane == 0) {
      const int it = warp * E + e;
      if (__float_as_uint(acc) == kLogitEmpty) acc = __uint_as_float(0x7fffffffu);
      p.rlogits[it] = acc;
      if (p.tr_rlogits) p.tr_rlogits[static_cast<size_t>(layer - p.first_layer) * nitems + it] = acc;
    }
  }
}

// Fill a bf16 buffer of n elements (n % 8 == 0) with kBf16Empty, spread over the grid.
__device__ __forceinline__ void bf16_rearm(uint16_t* buf, int n) {
  const uint4 e = make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n / 8; i += gridDim.x * kThreads)
    reinterpret_cast<uint4*>(buf)[i] = e;
}

// Mark this CTA's router-logit slots (tokens x experts blockIdx.x, blockIdx.x + G, ...) as not
// written.  Called at launch start and after the grid barrier that ends stage E, so that the next
// stage D's writes are the only values a reader can see after that barrier.
__device__ __forceinline__ void logits_rearm(const Params& p) {
#pragma unroll 1
  for (int i = threadIdx.x;; i += kThreads) {
    const int ej = i / p.T, t = i - ej * p.T;
    const int e = static_cast<int>(blockIdx.x) + ej * static_cast<int>(gridDim.x);
    if (e >= p.E) break;
    p.rlogits[t * p.E + e] = __uint_as_float(kLogitEmpty);
  }
}

// Softmax / top-k / renorm per token (one warp per token) and the expert tables, in every CTA
// (moe_fused_nki.py:224-272, 404-418).
// Order-preserving key of a float (larger float -> larger key; -0 and +0 map to one key) and
// its inverse.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f == 0.f ? 0.f : f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// wait_logits: stage D published the logits without a grid barrier; every slot is read until it
// no longer holds kLogitEmpty (bounded wait; a fatal status from another CTA ends it).
__device__ __noinline__ void routing_prologue(const Params& p, Ctx& c, int layer, bool wait_logits) {
  const int warp = threadIdx.x >> 5, lane = lane_id();
  Route* rt = c.rt;
  const int E = p.E, K = p.K;
#pragma unroll 1
  for (int t = warp; t < p.T; t += kWarps) {
    // lane l holds experts e = 32 q + l (q < 8); keys order the logits, ties by lower index
    const int per = (E + 31) / 32;
    float v[8];
    uint32_t key[8];
    int qq[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = q * 32 + lane;
      const bool ok = q < per && e < E;
      v[q] = ok ? ldcg_f(p.rlogits + static_cast<size_t>(t) * E + e) : -INFINITY;
    }
    if (wait_logits) {
      uint64_t t0 = 0;
#pragma unroll 1
      for (uint32_t it = 0;; ++it) {
        bool pend = false;
#pragma unroll
        for (int q = 0; q < 8; ++q) pend |= __float_as_uint(v[q]) == kLogitEmpty;
        if (!__any_sync(0xffffffffu, pend)) break;
        if ((it & 15u) == 0) {
          const uint64_t now = globaltimer_ns();
          if (it == 0) t0 = now;
          if ((ld_volatile_i32(p.status) & kStatusFatal) || now - t0 > kWaitLimitNs) {
            if (lane == 0) set_status(p, kStatusFatal);
            break;
          }
        }
        __nanosleep(200);  // back off: the polls share L2 with the last producers
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (__float_as_uint(v[q]) == kLogitEmpty) v[q] = ldcg_f(p.rlogits + static_cast<size_t>(t) * E + q * 32 + lane);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      key[q] = (q < per && q * 32 + lane < E) ? order_key(v[q]) : 0u;
      qq[q] = q;
    }
    // sort the lane's candidates by key, descending: odd-even transposition sort swapping only
    // strictly smaller neighbours, so equal keys keep their (ascending index) order
#pragma unroll
    for (int r = 0; r < 8; ++r) {
#pragma unroll
      for (int a = r & 1; a + 1 < 8; a += 2) {
        const bool sw = key[a + 1] > key[a];
        const uint32_t k0 = key[a], k1 = key[a + 1];
        const int q0 = qq[a], q1 = qq[a + 1];
        key[a] = sw ? k1 : k0;
        key[a + 1] = sw ? k0 : k1;
        qq[a] = sw ? q1 : q0;
        qq[a + 1] = sw ? q0 : q1;
      }
    }
    // top-K picks: the largest head key over the warp, the lowest index among equal ones; its
    // lane pops its head.  Lane k keeps pick k.
    uint32_t wmax0 = 0u, mykey = 0u;
    int mybi = 0;
#pragma unroll 1
    for (int k = 0; k < K; ++k) {
      const uint32_t wmax = __reduce_max_sync(0xffffffffu, key[0]);
      const int bi = static_cast<int>(__reduce_min_sync(
          0xffffffffu, key[0] == wmax ? static_cast<uint32_t>(qq[0] * 32 + lane) : 0xffffffffu));
      const bool own = lane == (bi & 31);
#pragma unroll
      for (int a = 0; a < 7; ++a) {
        key[a] = own ? key[a + 1] : key[a];
        qq[a] = own ? qq[a + 1] : qq[a];
      }
      key[7] = own ? 0u : key[7];
      if (k == 0) wmax0 = wmax;
      if (lane == k) {
        mykey = wmax;
        mybi = bi;
      }
    }
    // softmax over all E logits (lane-sequential over q, then the xor butterfly); its maximum is
    // the first pick
    const float mx = key_value(wmax0);
    float se = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) se += (q < per && q * 32 + lane < E) ? __expf(v[q] - mx) : 0.f;
    se = warp_sum_fixed(se);
    const float inv = 1.f / se;
    const float myval = lane < K ? rbf(__expf(key_value(mykey) - mx) * inv) : 0.f;
    if (lane < K) rt->topk_idx[t * K + lane] = mybi;
    // renormalise in pick order (sum over lanes 0..K-1 sequentially)
    float sk = 0.f;
#pragma unroll 1
    for (int k = 0; k < K; ++k) sk += __shfl_sync(0xffffffffu, myval, k);
    const float inv2 = 1.f / sk;
    if (lane < K) rt->topk_w[t * K + lane] = rbf(myval * inv2);
  }
  __syncthreads();
  // Every (token, slot) entry i = threadIdx.x (NP <= kMaxPairs == kThreads) marks its token in
  // its expert's mask (a token picks an expert at most once).  Counts are popcounts; an
  // entry's rank among the entries of its expert (token order) is the popcount of the lower
  // token bits.
  static_assert(kMaxPairs <= kThreads, "one thread per (token, slot) entry");
  // (batch <= 32, checked on the host: a token mask fits 32 bits)
  // Only this rank's experts [expert_begin, expert_begin + n_local) enter the tables (all of
  // them on one GPU); the tables use local expert indices.
  const int NP = p.T * K;
  const int ie = threadIdx.x;
  const int EL = p.n_local;
  for (int e = threadIdx.x; e < EL; e += kThreads) rt->emask[e] = 0u;
  __syncthreads();
  const int e_i = (ie < NP) ? rt->topk_idx[ie] - p.expert_begin : -1;
  const bool valid = e_i >= 0 && e_i < EL;
  const int t_i = ie / K;
  if (valid) atomicOr(&rt->emask[e_i], 1u << t_i);
  __syncthreads();
  if (warp == 0) {
    // active experts in ascending id order, with pair offsets: lane l takes the contiguous
    // experts [l * pe, (l + 1) * pe); one warp scan of (pairs, active experts) per lane
    const int pe = (EL + 31) / 32;
    const int e0 = lane * pe;
    int cs = 0, ns = 0;
#pragma unroll 1
    for (int a = 0; a < pe; ++a) {
      const int cnt = (e0 + a < EL) ? __popc(rt->emask[e0 + a]) : 0;
      cs += cnt;
      ns += cnt > 0;
    }
    int ci = cs, ni = ns;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, ci, d);
      const int z = __shfl_up_sync(0xffffffffu, ni, d);
      if (lane >= d) {
        ci += y;
        ni += z;
      }
    }
    int off = ci - cs, j = ni - ns;
#pragma unroll 1
    for (int a = 0; a < pe; ++a) {
      const int e = e0 + a;
      const int cnt = (e < EL) ? __popc(rt->emask[e]) : 0;
      if (cnt > 0) {
        rt->act_e[j] = e;
        rt->act_cnt[j] = cnt;
        rt->act_off[j] = off;
        rt->eoff[e] = off;
        ++j;
      }
      off += cnt;
    }
    if (lane == 31) rt->nA = ni;
  }
  __syncthreads();
  if (valid) {
    const int pr = rt->eoff[e_i] + __popc(rt->emask[e_i] & ((1u << t_i) - 1u));
    rt->pair_tok[pr] = t_i;
    rt->pair_w[pr] = rt->topk_w[ie];
  }
  if (blockIdx.x == 0 && p.tr_topk_idx && ie < NP) {
    p.tr_topk_idx[static_cast<size_t>(layer - p.first_layer) * NP + ie] = rt->topk_idx[ie];
    p.tr_topk_w[static_cast<size_t>(layer - p.first_layer) * NP + ie] = rt->topk_w[ie];
  }
  __syncthreads();
}

// ------------------------------------------------------------------ the kernel
// kExt: the instantiation that also serves stages bits 8 (q/k/v from the caller) and 16 (every
// row's K/V before the attention).  The decode step's instantiations (kExt = false) carry none
// of that code: the per-layer path is larger than the SM instruction cache, and code added to it
// costs time even where it never runs.
template <int NT, bool kExt>
__global__ void __launch_bounds__(kThreads, 1)
    qwen3_decode_kernel(const __grid_constant__ Params pk, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ uint8_t smem_raw[];
  // The stage functions read the launch parameters through a reference: a shared-memory copy
  // answers in tens of cycles, the kernel-parameter space behind a generic pointer in
  // hundreds.
  __shared__ __align__(16) Params sp;
  static_assert(sizeof(Params) % 4 == 0 && sizeof(Params) / 4 <= kThreads, "Params copy");
  if (threadIdx.x < sizeof(Params) / 4)
    reinterpret_cast<uint32_t*>(&sp)[threadIdx.x] = reinterpret_cast<const uint32_t*>(&pk)[threadIdx.x];
  __syncthreads();
  const Params& p = sp;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemLayout lay(p.H, NT);
  const int warp = threadIdx.x >> 5, lane = lane_id();
  // several ranks: only the kExt kernels carry the exchange code (the host launches them then)
  const bool multi = kExt && p.n_ranks > 1;
  Ctx c;
  c.ring_bytes = lay.ring_bytes;
  c.nslot = lay.ring_bytes / kSlotBytes;
  c.ring_all = smem + lay.ring_off;
  c.ring = c.ring_all + warp * lay.ring_bytes;
  c.bars = reinterpret_cast<uint64_t*>(smem + lay.bars_off) + warp * kMaxBars;
  c.phase = 0;
  c.head = 0;
  c.worker = blockIdx.x * kWarps + warp;
  c.nworkers = gridDim.x * kWarps;
  c.pol = policy_evict_first();
  c.xs = reinterpret_cast<uint16_t*>(smem + lay.xs_off);
  c.xs_stride = p.H + 32;
  c.att = smem + lay.xs_off;
  c.rstd = reinterpret_cast<float*>(smem + lay.rstd_off);
  c.rt = reinterpret_cast<Route*>(smem + lay.route_off);
  c.flag = reinterpret_cast<int*>(smem + lay.flag_off);
  c.stage_idx = 0;
  c.bar_k = 0;
  c.gbar_k = 0;
  c.gbase = multi ? *p.gbase : 0ull;
  c.plan = reinterpret_cast<AttPlan*>(smem + lay.plan_off);
  c.red = reinterpret_cast<float*>(smem + lay.red_off);
  c.att_pb = -1;
  c.primed = 0;
  c.cbar = reinterpret_cast<uint64_t*>(smem + lay.cbar_off);
  c.dyn = reinterpret_cast<int*>(smem + lay.dyn_off);
  c.awaitq = 0;
  c.cphase = 0;
  c.npref = 0;
  {
    // the layer pointer table, once per launch: every stage reads its pointers from shared memory
    static_assert(sizeof(LayerPtrs) % 16 == 0, "LayerPtrs is copied as uint4");
    LayerPtrs* lt = reinterpret_cast<LayerPtrs*>(smem + lay.lt_off);
    const uint4* src = reinterpret_cast<const uint4*>(p.layers + p.first_layer);
    const int n16 = p.num_layers * static_cast<int>(sizeof(LayerPtrs) / 16);
    for (int i = threadIdx.x; i < n16; i += kThreads) reinterpret_cast<uint4*>(lt)[i] = src[i];
    c.lt = lt;
    if (p.stages & 1) att_plan_build(p, c);
    __syncthreads();
  }
  stamp(p, c);
  if (lane == 0) {
    for (int s = 0; s < kMaxBars; ++s) mbar_init(&c.bars[s], 1);
    if (threadIdx.x == 0) mbar_init(c.cbar, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0 && (p.stages & 1)) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  __syncwarp();

  [&]() {  // the launch body; a fatal error returns from here to launch_exit
  // stages bit 8: the attention takes the q/k/v projections the caller wrote into the QKV buffer
  // (no RMSNorm(ln1) + QKV GEMV; one layer per launch, checked on the host)
  const bool qkv_in = kExt && (p.stages & 8) != 0;
  // stage 0: residual (fp32) <- embeddings / hidden input (bf16); the router-logit slots of the
  // staged path start unwritten
  if (norm_staged_ok<NT>(p) && (p.stages & 2)) logits_rearm(p);
  if (norm_staged_ok<NT>(p) && (p.stages & 1) && !qkv_in) bf16_rearm(p.qkv, p.T * p.R);
  {
    const int nvec = p.T * p.H / 8;
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < nvec; i += gridDim.x * kThreads) {
      const int t = (i * 8) / p.H, k = (i * 8) % p.H;
      const uint16_t* src;
      if (p.input_ids) {
        int id = __ldg(p.input_ids + t);
        if (id < 0 || id >= p.V) {
          set_status(p, kStatusIndex);
          id = 0;
        }
        src = p.embed + static_cast<size_t>(id) * p.H + k;
      } else {
        src = p.x_in + static_cast<size_t>(t) * p.H + k;
      }
      const uint4 v = ldnc128(src);
      float* dst = p.resid + static_cast<size_t>(t) * p.H + k;
      *reinterpret_cast<float4*>(dst) = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y));
      *reinterpret_cast<float4*>(dst + 4) = make_float4(lo_bf(v.z), hi_bf(v.z), lo_bf(v.w), hi_bf(v.w));
    }
  }
  const bool staged = norm_staged_ok<NT>(p);
  grid_arrive(p);
  if ((p.stages & 1) && p.num_layers > 0 && !qkv_in) {  // the first QKV weights stream during the barrier
    const LayerPtrs& l0 = c.lt[0];
    GemvGeom ga{l0.wqkv, 0, 1, p.R / 16, p.H / 32, p.H, p.first_layer};
    gemv_prime<NT, GK_QKV>(p, c, ga, staged ? 1 : RingGeom<NT>::kGemvSlots);
    if (staged) norm_prefetch(p, c, l0.ln1, nullptr);
  }
  if (!grid_wait(p, c)) return;

  const int layer_end = p.first_layer + p.num_layers;

  const bool want_lm = (p.stages & 4) && p.logits_out;
  // prime whatever GEMV follows the last stage of `layer` (next layer's QKV, or the LM head)
  auto prime_after = [&](int layer) {
    if (layer + 1 < layer_end) {
      if (p.stages & 1) {
        const LayerPtrs& nl = c.lt[layer + 1 - p.first_layer];
        GemvGeom ga{nl.wqkv, 0, 1, p.R / 16, p.H / 32, p.H, layer + 1};
        gemv_prime<NT, GK_QKV>(p, c, ga, staged ? 1 : RingGeom<NT>::kGemvSlots);
        if (staged) norm_prefetch(p, c, nl.ln1, nullptr);
      }
    } else if (want_lm) {
      const GemvGeom gl = lm_geom(p, layer);
      gemv_prime<NT, GK_LMHEAD>(p, c, gl, staged ? 1 : RingGeom<NT>::kGemvSlots);
      if (staged) norm_prefetch(p, c, p.final_norm, nullptr);
    }
  };
  for (int layer = p.first_layer; layer < layer_end; ++layer) {
    const LayerPtrs& lw = c.lt[layer - p.first_layer];
    if (p.stages & 1) {
      // A: RMSNorm(ln1) + QKV
      if (!qkv_in) {
        if (staged) norm_staged(p, c, layer, false, lw.ln1);
        else norm_rows_to_smem(p, c, lw.ln1, false);
        __syncthreads();
        GemvGeom ga{lw.wqkv, 0, 1, p.R / 16, p.H / 32, p.H, layer};
        if (cta_strip_mode<NT>(ga, GK_QKV)) gemv_cta_strips<NT>(p, c, ga, GK_QKV);
        else gemv_stage<NT, GK_QKV>(p, c, ga);
      }
      if (kExt && (p.stages & 16)) {
        // K/V of every row first (a grid barrier on each side), then the attention reads them
        if (!grid_barrier(p, c)) return;
        kv_prewrite(p, c, layer);
        grid_arrive(p);
        if (!grid_wait(p, c)) return;
        fence_proxy_async_global();  // this launch's K/V stores, before the TMA reads of them
        att_prime_layer(p, c, layer, &kmap, &vmap);
      } else if (staged) {
        // stage B takes only q/k/v from other CTAs and waits for them element by element
        c.awaitq = 1;
        att_prime_layer(p, c, layer, &kmap, &vmap);
        stamp(p, c);  // (stage-time probes: stage A ends here)
      } else {
        grid_arrive(p);
        att_prime_layer(p, c, layer, &kmap, &vmap);  // this layer's first K/V boxes stream during the barrier
        if (!grid_wait(p, c)) return;
      }
      // B: attention (+ KV write); the O-proj weights start streaming before the barrier
      attention_stage(p, c, layer, &kmap, &vmap);
      GemvGeom gc{lw.wo, 0, 1, p.H / 16, (p.nq * kHeadDim) / 32, p.nq * kHeadDim, layer};
      grid_arrive(p);
      gemv_prime<NT, GK_OPROJ>(p, c, gc);
      if (!grid_wait(p, c)) return;
      // C: O-proj + residual
      if (cta_strip_mode<NT>(gc, GK_OPROJ)) gemv_cta_strips<NT>(p, c, gc, GK_OPROJ);
      else gemv_stage<NT, GK_OPROJ>(p, c, gc);
      // every CTA read this layer's q/k/v before barrier B; with stage D the re-arm waits for it
      // (it then overlaps the router-logit wait instead of delaying this stage's barrier)
      if (staged && !(p.stages & 2)) bf16_rearm(p.qkv, p.T * p.R);
      // stage D's gamma and router row stream during the barrier
      const bool pre_d = (p.stages & 2) && staged;
      if (multi) {
        // tensor parallel: sum the ranks' O-projection partials into the residual
        __syncthreads();  // the rings and the strip-reduction area are free
        if (!(p.stages & 2)) prime_after(layer);
        if (pre_d) norm_prefetch(p, c, lw.ln2, lw.router);
        if (!rank_exchange(p, c, 0, layer)) return;
      } else {
        grid_arrive(p);
        if (!(p.stages & 2)) prime_after(layer);
        if (pre_d) norm_prefetch(p, c, lw.ln2, lw.router);
        if (!grid_wait(p, c)) return;
      }
    }
    if (p.stages & 2) {
      // D: RMSNorm(ln2) once per CTA (fp32 rows into the idle rings, bf16 rows into X for the
      // experts), then the router logits (fp32, fixed order)
      if (staged) {
        norm_staged(p, c, layer, true, lw.ln2);
        if (p.stages & 1) bf16_rearm(p.qkv, p.T * p.R);
      } else {
        float* x32 = (static_cast<uint32_t>(p.T * p.H * 4) <= static_cast<uint32_t>(kWarps * c.ring_bytes))
                         ? reinterpret_cast<float*>(c.ring_all)
                         : nullptr;
        norm_rows_to_smem(p, c, lw.ln2, true, x32);
        __syncthreads();
        if (x32) router_stage<true>(p, c, layer, x32);
        else router_stage<false>(p, c, layer, nullptr);
      }
      // E: routing tables + gate/up (X from stage D); the down weights start streaming early.  On
      // the staged path the logits are the only data stage E takes from other CTAs: routing waits
      // for them slot by slot instead of a grid barrier.
      if (staged) stamp(p, c);  // (stage-time probes: stage D ends here)
      else if (!grid_barrier(p, c)) return;
      routing_prologue(p, c, layer, staged);
      GemvGeom ge{lw.w13, static_cast<uint64_t>(2) * p.I * p.H * 2, c.rt->nA, (2 * p.I) / 16, p.H / 32, p.H, layer};
      if (gateup_dyn_ok<NT>(ge)) gateup_dyn<NT>(p, c, ge);
      else gemv_stage<NT, GK_GATEUP>(p, c, ge);
      GemvGeom gf{lw.w2, static_cast<uint64_t>(p.H) * p.I * 2, c.rt->nA, p.H / 16, p.I / 32, p.I, layer};
      grid_arrive(p);
      down_prime<NT>(p, c, gf);
      if (!grid_wait(p, c)) return;
      // F: down + affinity + combine + residual
      down_stage<NT>(p, c, gf);
      if (staged) logits_rearm(p);  // every CTA read this layer's logits before the last barrier
      if (multi) {
        // expert parallel: sum the ranks' expert partials into the residual (a rank without
        // active experts contributes zeros)
        if (c.rt->nA == 0) {
          const int n = p.T * p.H;
          const unsigned xs = xseq_of(p, 1, layer);
          for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) ll_put(p, 1, xs, i, 0.f);
        }
        prime_after(layer);
        if (!rank_exchange(p, c, 1, layer)) return;
      } else {
        grid_arrive(p);
        prime_after(layer);
        if (!grid_wait(p, c)) return;
      }
    }
  }
  // outputs
  {
    const int nvec = p.T * p.H / 8;
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < nvec; i += gridDim.x * kThreads) {
      const float4 a = ldcg_f4(p.resid + static_cast<size_t>(i) * 8);
      const float4 b = ldcg_f4(p.resid + static_cast<size_t>(i) * 8 + 4);
      reinterpret_cast<uint4*>(p.y_out)[i] =
          make_uint4(pack_bf2(a.x, a.y), pack_bf2(a.z, a.w), pack_bf2(b.x, b.y), pack_bf2(b.z, b.w));
    }
  }
  if (want_lm) {
    if (staged) norm_staged(p, c, max(layer_end - 1, p.first_layer), false, p.final_norm);
    else norm_rows_to_smem(p, c, p.final_norm, false);
    __syncthreads();
    gemv_stage<NT, GK_LMHEAD>(p, c, lm_geom(p, layer_end - 1));
    if (multi) {
      // every rank's strips are in this rank's logits area once all ranks pass the barrier
      if (!grid_sync_ranks(p, c)) return;
      const int n16 = p.T * p.V / 4;
      const float* src = xchg_logits(p, p.rank);
      float4* dst = reinterpret_cast<float4*>(p.logits_out);
      for (int i = blockIdx.x * kThreads + threadIdx.x; i < n16; i += gridDim.x * kThreads) dst[i] = ldcg_f4(src + 4 * i);
    }
  }
  if (p.tr_stage) {
    __syncthreads();
    stamp(p, c);
  }
  }();
  launch_exit(p, c, multi);
}

}  // namespace nkm
