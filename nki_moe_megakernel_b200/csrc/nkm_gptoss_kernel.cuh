// Persistent cooperative decode-step kernel for GPT-OSS on B200 (sm_100a).
//
// One CTA per SM, 8 warps.  Stages are separated by grid barriers (one monotonic arrival counter,
// every wait bounded and polling the status word).  Work inside a stage is split into warp units
// whose weights stream straight from HBM with 16-byte non-allocating loads, several k-tiles in
// flight per lane; activations sit in shared memory.  Per layer (reference order:
// megakernels/gpt_oss/transformer_gpt_oss.py:271-530):
//   A   RMSNorm(ln1) of every row (each CTA) + QKV GEMV (bf16, split-K)      -> partials
//   A2  partials + bias; RoPE (YaRN table) of q and k; K -> cache, V -> transposed cache, q -> qbuf
//   B   attention units (row, kv head, 128-token block of the context): sliding-window or full
//   C0  combine of the block partials with the head's sink logit -> attention output (bf16)
//   C   O-projection GEMV (bf16, split-K)                                    -> partials
//   C2  residual += partials + bias
//   D   RMSNorm(ln2) of every row (each CTA, f16 copy kept for the experts) + router logits
//   E   top-k + softmax over the k (each CTA) + expert gate/up GEMV (MXFP4) + bias + clamped SwiGLU
//   F   expert down GEMV (MXFP4) + bias, times the routing weight           -> per (token, slot)
//   G   residual += slot outputs in slot order
// then the final RMSNorm and the LM head GEMV.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "nkm_ptx.cuh"

namespace nkg {

using nkm::f2bf;
using nkm::globaltimer_ns;
using nkm::hi_bf;
using nkm::lo_bf;
using nkm::mma_bf16;
using nkm::pack_bf2;
using nkm::smem_addr;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kHD = 64;          // head dim
constexpr int kBlk = 128;        // tokens per K/V block
constexpr int kMaxB = 16;        // rows per launch (two 8-column mma tiles)
constexpr int kNT = 2;
constexpr int kMaxE = 128;
constexpr int kMaxTopK = 8;
constexpr int kMaxPairs = kMaxB * kMaxTopK;
constexpr int kMaxHidden = 4096;
constexpr int kMaxRows16 = 4096 + 8;   // shared activation row: K + 8 halves
constexpr int kMaxKC = 4;              // split-K factor of the dense GEMVs
constexpr int kMaxGrp = 16;            // query heads per KV head
constexpr int kPartStride = 2 + kHD;   // m, l, o[64] per head row of an attention unit
constexpr int kStatusFatal = 4;
constexpr int kStatusIndex = 8;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

struct Layer {
  const uint8_t* wqkv;    // FT bf16 [R, H]
  const uint16_t* bqkv;   // [R]
  const uint8_t* wo;      // FT bf16 [H, nq*64]
  const uint16_t* bo;     // [H]
  const uint16_t* sinks;  // [nq]
  const uint16_t* ln1;    // [H]
  const uint16_t* ln2;    // [H]
  const uint16_t* router; // [E, H] row-major
  const uint16_t* router_b;  // [E]
  const uint8_t* w13;     // FT4 [E][2I rows][H]   (row 2i gate i, row 2i+1 up i)
  const uint8_t* s13;     // e8m0 [E][2I/16][H/32][16]
  const uint16_t* b13;    // [E][2I]
  const uint8_t* w2;      // FT4 [E][H rows][I]
  const uint8_t* s2;      // e8m0 [E][H/16][I/32][16]
  const uint16_t* b2;     // [E][H]
  int sliding;            // 1: sliding-window attention
  int pad_[3];
};

struct Params {
  int B, H, Hact, nq, nkv, grp, R, E, K, I, L, V, window;
  float eps, limit, alpha;
  // FP8 K/V cache (e4m3): stored = e4m3(clip(x * k_scale, +-240)), read = stored / k_scale
  // (attention_block_tkg.py:213-218, 1694); 0: bf16 cache
  int kv_fp8;
  float k_scale, v_scale;
  int kc_qkv, kc_o;
  int first_layer, num_layers, want_lm;
  const Layer* layers;
  const uint16_t* final_norm;
  const uint8_t* lm_head;
  const uint16_t* embed;
  const float* rope_cos;  // [rope_max][32]
  const float* rope_sin;
  int rope_max;
  uint16_t* k_pool;       // [L][NB][nkv][128][64]            (bf16, or e4m3 bytes when kv_fp8)
  uint16_t* v_pool;       // [L][NB][nkv][64][128]  transposed blocks (bf16, or e4m3 bytes)
  int num_blocks;
  const int* input_ids;
  const uint16_t* x_in;
  const int* positions;
  const int* block_table;
  int max_blocks;
  uint16_t* y_out;
  float* logits_out;
  float* tr_qkv;
  float* tr_mid;
  float* tr_out;
  float* tr_rlogits;
  int* tr_idx;
  float* tr_w;
  int64_t* tr_stage;
  unsigned* bar;
  int* status;
  float* resid;
  float* part;
  uint16_t* qbuf;
  float* att_part;
  uint16_t* attn_out;
  float* rlogits;
  uint16_t* hbuf;
  float* ypair;
  // tensor + expert parallelism (n_ranks > 1): nq / nkv above are this rank's heads; its experts
  // are [expert_begin, expert_begin + n_local) of E (the layer tensors hold only those); it
  // computes the LM head's vocabulary strips [lm_s0, lm_s0 + lm_ns)
  int n_ranks, rank, expert_begin, n_local, lm_s0, lm_ns;
  uint8_t* xchg[8];     // exchange region of every rank (CUDA IPC mappings)
  unsigned* xseq;       // [3] exchanges of each kind before this launch (workspace)
  int64_t xlog_off;     // byte offset of the logits exchange within a region
};

struct Route {
  int nA;
  int act_e[kMaxE];
  int act_off[kMaxE];
  int act_cnt[kMaxE];
  int cnt[kMaxE];
  int topk_idx[kMaxPairs];
  float topk_w[kMaxPairs];
  int pair_tok[kMaxPairs];
  float pair_w[kMaxPairs];
  int pair_of[kMaxPairs];
};

// Expert weight rings: each warp streams its MXFP4 strips through kRingSlots shared-memory slots
// with 1-D bulk copies; a slot holds kCK k-tiles (256 bytes each: 16 rows x 32 inputs) and their
// grouped scales (128 bytes per 8 k-tiles).
constexpr int kCK = 16;
constexpr int kRingSlots = 2;
constexpr int kSlotW = kCK * 256;
constexpr int kSlotBytes = kSlotW + (kCK / 8) * 128;

// Shared memory: activation rows (bf16 or f16, stride Kx + 8 halves) | rstd | route | flag |
// expert rings | their mbarriers | each warp's ring phase bits.
struct Smem {
  uint32_t xs_off, rstd_off, route_off, flag_off, ring_off, bar_off, phase_off, total;
  __host__ __device__ explicit Smem(int B, int kmax) {
    xs_off = 0;
    uint32_t xs = static_cast<uint32_t>(B) * static_cast<uint32_t>(kmax + 8) * 2u;
    rstd_off = (xs + 15u) & ~15u;
    route_off = rstd_off + kMaxB * 4;
    flag_off = route_off + static_cast<uint32_t>((sizeof(Route) + 15) & ~size_t(15));
    ring_off = (flag_off + 16u + 127u) & ~127u;
    bar_off = ring_off + static_cast<uint32_t>(kWarps * kRingSlots * kSlotBytes);
    phase_off = bar_off + static_cast<uint32_t>(kWarps * kRingSlots * 8);
    total = phase_off + kWarps * 4;
  }
};

// A warp's ring: slots (kRingSlots x kSlotBytes), their mbarriers and the phase bits (kept in
// shared memory between stages).
struct Ring {
  uint8_t* buf;
  uint64_t* bar;
  uint32_t* phase;
};

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ void set_status(const Params& p, int bit) { atomicOr(p.status, bit); }

// ------------------------------------------------------------------ grid barrier
__device__ __noinline__ bool grid_sync(const Params& p, unsigned& bar_k, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    nkm::red_release_add_u32(p.bar, 1u);
    const unsigned target = (bar_k + 1u) * gridDim.x;
    int ok = 1;
    uint64_t t0 = 0;
#pragma unroll 1
    for (unsigned it = 0;; ++it) {
      const unsigned v = nkm::ld_acquire_u32(p.bar);
      if (nkm::ld_volatile_i32(p.status) & kStatusFatal) {
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
    *flag = ok;
    if (p.tr_stage && blockIdx.x == 0) p.tr_stage[bar_k + 1] = static_cast<int64_t>(globaltimer_ns());
  }
  ++bar_k;
  __syncthreads();
  return *flag != 0;
}

// ------------------------------------------------------------------ ranks (TP + EP)
// The ranks exchange tagged 8-byte words: the fp32 value in the low half, the exchange's
// sequence number + 1 in the high half, stored and loaded as one single-copy-atomic access, so a
// reader that sees the tag it expects also sees the value (no fence, flag or barrier).  Kinds:
// 0 the O-projection partials and 1 the expert partials ([kind][n % 2][src rank][B][H] after the
// header), 2 the logits ([n % 2][B][V] from xlog_off; each rank stores its vocabulary strips).
// Two slots per kind: a rank produces exchange n + 2 of a kind only after reading every rank's
// exchange n + 1, which each rank produces only after reading exchange n.
constexpr int kXchgHeader = 256;
__device__ __forceinline__ unsigned long long* xw_part(const Params& p, int q, int kind, unsigned n, int src) {
  return reinterpret_cast<unsigned long long*>(p.xchg[q] + kXchgHeader) +
         static_cast<size_t>((kind * 2 + static_cast<int>(n & 1u)) * p.n_ranks + src) * p.B * p.H;
}
__device__ __forceinline__ unsigned long long* xw_logits(const Params& p, int q, unsigned n) {
  return reinterpret_cast<unsigned long long*>(p.xchg[q] + p.xlog_off) + static_cast<size_t>(n & 1u) * p.B * p.V;
}
// sequence number of `layer`'s exchange of kind 0 or 1, or (kind 2) of this launch's logits
__device__ __forceinline__ unsigned xseq_of(const Params& p, int kind, int layer) {
  return __ldg(p.xseq + kind) + (kind == 2 ? 0u : static_cast<unsigned>(layer - p.first_layer));
}
__device__ __forceinline__ unsigned long long xword(unsigned n, float v) {
  return (static_cast<unsigned long long>(n + 1u) << 32) | __float_as_uint(v);
}
// element i of this rank's partial of exchange n (kind 0 / 1) into every rank's region
__device__ __forceinline__ void put_part(const Params& p, int kind, unsigned n, size_t i, float v) {
  const unsigned long long w = xword(n, v);
#pragma unroll 1
  for (int q = 0; q < p.n_ranks; ++q) nkm::st_relaxed_sys_u64(xw_part(p, q, kind, n, p.rank) + i, w);
}
// The value of a tagged word once it carries exchange n's tag (bounded wait; false once the
// launch has failed).
__device__ __forceinline__ bool take_word(const Params& p, const unsigned long long* a, unsigned n, float& v) {
  unsigned long long w = nkm::ld_relaxed_sys_u64(a);
  if (static_cast<unsigned>(w >> 32) != n + 1u) {
    uint64_t t0 = 0;
#pragma unroll 1
    for (uint32_t it = 0;; ++it) {
      if ((it & 15u) == 0) {
        const uint64_t now = globaltimer_ns();
        if (it == 0) t0 = now;
        if ((nkm::ld_volatile_i32(p.status) & kStatusFatal) || now - t0 > kWaitLimitNs) {
          set_status(p, kStatusFatal);
          return false;
        }
      }
      __nanosleep(32);
      w = nkm::ld_relaxed_sys_u64(a);
      if (static_cast<unsigned>(w >> 32) == n + 1u) break;
    }
  }
  v = __uint_as_float(static_cast<unsigned>(w));
  return true;
}
// Sum over the ranks, in rank order, of element i of exchange n (kind 0 / 1).
__device__ __forceinline__ bool rank_sum(const Params& p, int kind, unsigned n, size_t i, float& s) {
  s = 0.f;
#pragma unroll 1
  for (int q = 0; q < p.n_ranks; ++q) {
    float v;
    if (!take_word(p, xw_part(p, p.rank, kind, n, q) + i, n, v)) return false;
    s += v;
  }
  return true;
}

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}
__device__ __forceinline__ uint2 ldnc64(const void* ptr) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(ptr));
  return v;
}
__device__ __forceinline__ uint32_t ldnc_u8(const uint8_t* ptr) {
  uint16_t v;
  asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(v) : "l"(ptr));
  return v;
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// four e2m1 pairs (one byte each, low nibble -> low half) to f16x2
__device__ __forceinline__ void e2m1x8(uint32_t w, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
}
__device__ __forceinline__ uint32_t ldcg_u32(const void* ptr) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(ptr));
  return v;
}
// two e4m3 bytes (low byte -> low half) to f16x2
__device__ __forceinline__ uint32_t e4m3x2(uint32_t v16) {
  uint32_t d;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(d) : "r"(v16));
  return d;
}
__device__ __forceinline__ uint8_t to_e4m3(float x, float scale) {
  const float y = fminf(fmaxf(x * scale, -240.f), 240.f);
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ uint16_t f2h_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
// e8m0 scale 2^(s - 127) as fp32 (s = 0 gives 0: below any weight this format holds in practice)
__device__ __forceinline__ float e8m0(uint32_t s) { return __uint_as_float(s << 23); }

// Sum over the H (or Hact) elements of a row in a fixed order: lane l owns k = 256 i + 8 l + j.
__device__ __forceinline__ float row_sumsq(const float* row, int H) {
  const int lane = lane_id();
  float s = 0.f;
#pragma unroll 1
  for (int i = 0; i * 256 < H; ++i) {
    const int k = 256 * i + 8 * lane;
    if (k < H) {
      const float4 a = nkm::ldcg_f4(row + k);
      const float4 b = nkm::ldcg_f4(row + k + 4);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) s = __fadd_rn(s, __fmul_rn(v[j], v[j]));
    }
  }
  return warp_sum(s);
}

// RMSNorm of every residual row into shared memory (one warp per row): (x * rstd) * gamma, as
// bf16 (f16 = false) or f16 (f16 = true), row stride H + 8.  The mean uses Hact elements (rows
// padded beyond Hact hold zeros).
__device__ __noinline__ void norm_rows(const Params& p, const uint16_t* gamma, uint16_t* xs, float* rstd, bool f16) {
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const int H = p.H, stride = H + 8;
#pragma unroll 1
  for (int t = warp; t < p.B; t += kWarps) {
    const float* row = p.resid + static_cast<size_t>(t) * H;
    const float ss = row_sumsq(row, H);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.Hact)), p.eps)));
    if (lane == 0) rstd[t] = r;
#pragma unroll 1
    for (int k = 8 * lane; k < H; k += 256) {
      const float4 a = nkm::ldcg_f4(row + k);
      const float4 b = nkm::ldcg_f4(row + k + 4);
      const uint4 g = *reinterpret_cast<const uint4*>(gamma + k);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__fmul_rn(v[j], r), (j & 1) ? hi_bf(gw[j >> 1]) : lo_bf(gw[j >> 1]));
      uint4 o;
      if (f16) {
        const __half2 h0 = __floats2half2_rn(y[0], y[1]), h1 = __floats2half2_rn(y[2], y[3]);
        const __half2 h2 = __floats2half2_rn(y[4], y[5]), h3 = __floats2half2_rn(y[6], y[7]);
        o = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                       *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
      } else {
        o = make_uint4(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]), pack_bf2(y[4], y[5]), pack_bf2(y[6], y[7]));
      }
      *reinterpret_cast<uint4*>(xs + static_cast<size_t>(t) * stride + k) = o;
    }
  }
  // rows B..15 of the two column tiles read zeros
  for (int i = p.B * stride + threadIdx.x * 8; i < kMaxB * stride; i += kThreads * 8)
    if (i + 8 <= kMaxB * stride) *reinterpret_cast<uint4*>(xs + i) = make_uint4(0u, 0u, 0u, 0u);
}

// ------------------------------------------------------------------ GEMV engines
// Weights stream through each warp's shared-memory ring (1-D bulk copies, kRingSlots chunks in
// flight across unit boundaries); the activations are rows in shared memory.
// * bf16 fragment-tiled strips: 1 KB units of 16 rows x 32 k (lane l: row l/4 and l/4 + 8,
//   k 8(l%4)..+7).
// * MXFP4 fragment-tiled strips: 256-byte units of 16 rows x 32 k (lane l: 4 bytes of row l/4 then
//   4 bytes of row l/4 + 8, k 8(l%4)..+7, low nibble first), with the strip's e8m0 scales in groups
//   of 8 k-tiles ([group][16 rows][8], so a lane reads its two rows' 8 scales with two 8-byte
//   loads).  Each unit's product is accumulated from zero and scaled by its rows' scales (exact
//   powers of two).
// Only the 8-column tiles that hold tokens are multiplied (an expert of a 16-row batch usually
// has at most 8 tokens).
__device__ __forceinline__ uint32_t byte_of(const uint2 v, int u) {
  return ((u < 4 ? v.x : v.y) >> (8 * (u & 3))) & 0xffu;
}
// Bytes of one 16-row strip's grouped scales for KT k-tiles.
__device__ __forceinline__ size_t fp4_strip_scale_bytes(int KT) { return static_cast<size_t>((KT + 7) / 8) * 128; }

// ---- expert weight rings (bulk copies into shared memory)
__device__ __forceinline__ uint2 lds64(const void* ptr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_addr(ptr)));
  return v;
}
// Lane 0: nk k-tiles of a strip's weights (w) and their scale groups (sc) into ring slot `slot`.
__device__ __forceinline__ void ring_issue(const Ring& r, int slot, const uint8_t* w, const uint8_t* sc, int nk,
                                           uint64_t pol) {
  const uint32_t wb = static_cast<uint32_t>(nk) * 256u, sb = static_cast<uint32_t>((nk + 7) / 8) * 128u;
  uint8_t* dst = r.buf + slot * kSlotBytes;
  nkm::fence_proxy_async_smem();
  nkm::mbar_arrive_expect_tx(&r.bar[slot], wb + sb);
  nkm::bulk_g2s(dst, w, wb, &r.bar[slot], pol);
  nkm::bulk_g2s(dst + kSlotW, sc, sb, &r.bar[slot], pol);
}
// Bounded wait for phase `par` of slot `slot`; false once the launch has failed (a wait that
// lasts beyond any normal one also polls the status word, so one failure ends every wait).
__device__ __noinline__ bool ring_wait(const Params& p, const Ring& r, int slot, uint32_t par) {
  uint64_t t0 = 0;
#pragma unroll 1
  for (uint32_t it = 0;; ++it) {
    if (nkm::mbar_try_wait(&r.bar[slot], par)) return true;
    if ((it & 63u) == 63u) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > 20000ull) {
        if (nkm::ld_volatile_i32(p.status) & kStatusFatal) return false;
        if (now - t0 > kWaitLimitNs) {
          if (lane_id() == 0) set_status(p, kStatusFatal);
          return false;
        }
      }
    }
  }
}
// After a failed wait: the copies this warp still has in flight land in its slots; wait for
// each (1 ms bound) before the warp leaves the stage.
__device__ __noinline__ void ring_drain(const Ring& r, uint32_t inflight, uint32_t phase) {
#pragma unroll 1
  for (int sl = 0; sl < kRingSlots; ++sl) {
    if (!(inflight & (1u << sl))) continue;
    const uint64_t t0 = globaltimer_ns();
    while (!nkm::mbar_try_wait(&r.bar[sl], (phase >> sl) & 1u) && globaltimer_ns() - t0 < 1000000ull) {
    }
  }
}
// nk k-tiles of one ring slot (k-tile kt of the slot is input block kbase + kt) against the
// activation rows brow[nt] (f16 in shared memory), accumulated into acc.
template <int NTA>  // n-tiles with tokens (1: at most 8 of them)
__device__ __forceinline__ void fp4_slot(const uint8_t* slot, int nk, int kbase, const uint16_t* const (&brow)[kNT],
                                         float (&acc)[kNT][4]) {
  const int lane = lane_id(), g = lane >> 2;
#pragma unroll 1
  for (int k8 = 0; k8 < nk; k8 += 8) {
    const uint8_t* grp = slot + kSlotW + (k8 >> 3) * 128;
    const uint2 sg = lds64(grp + 8 * g), sh = lds64(grp + 8 * (g + 8));
    uint2 w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) w[u] = k8 + u < nk ? lds64(slot + (k8 + u) * 256 + 8 * lane) : make_uint2(0u, 0u);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (k8 + u < nk) {
        uint32_t r0, r1, r2, r3, q0, q1, q2, q3;
        e2m1x8(w[u].x, r0, r1, r2, r3);
        e2m1x8(w[u].y, q0, q1, q2, q3);
        const float s0 = e8m0(byte_of(sg, u)), s1 = e8m0(byte_of(sh, u));
        const int kk = (kbase + k8 + u) * 32;
#pragma unroll
        for (int nt = 0; nt < NTA; ++nt) {
          const uint4 b = brow[nt] ? *reinterpret_cast<const uint4*>(brow[nt] + kk) : make_uint4(0u, 0u, 0u, 0u);
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_f16(d, r0, q0, r1, q1, b.x, b.y);
          mma_f16(d, r2, q2, r3, q3, b.z, b.w);
          acc[nt][0] = fmaf(d[0], s0, acc[nt][0]);
          acc[nt][1] = fmaf(d[1], s0, acc[nt][1]);
          acc[nt][2] = fmaf(d[2], s1, acc[nt][2]);
          acc[nt][3] = fmaf(d[3], s1, acc[nt][3]);
        }
      }
    }
  }
}

// ---- bf16 strips through the same rings (the dense GEMVs and the LM head): 4 k-tiles of 1 KB
// (16 rows x 32 inputs, fragment-tiled) per slot
constexpr int kCKb = kSlotW / 1024;
__device__ __forceinline__ uint4 lds128(const void* ptr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_addr(ptr)));
  return v;
}
template <int NTA>
__device__ __forceinline__ void bf16_slot(const uint8_t* slot, int nk, int kbase, const uint16_t* const (&brow)[kNT],
                                          float (&acc)[kNT][4]) {
  const int lane = lane_id();
#pragma unroll
  for (int k = 0; k < kCKb; ++k) {
    if (k < nk) {
      const uint4 a0 = lds128(slot + k * 1024 + 16 * lane), a1 = lds128(slot + k * 1024 + 512 + 16 * lane);
      const int kk = (kbase + k) * 32;
#pragma unroll
      for (int nt = 0; nt < NTA; ++nt) {
        const uint4 b = brow[nt] ? *reinterpret_cast<const uint4*>(brow[nt] + kk) : make_uint4(0u, 0u, 0u, 0u);
        mma_bf16(acc[nt], a0.x, a1.x, a0.y, a1.y, b.x, b.y);
        mma_bf16(acc[nt], a0.z, a1.z, a0.w, a1.w, b.z, b.w);
      }
    }
  }
}
// This warp's units u = first, first + step, ... < nunits of a bf16 GEMV: unit(u, base, kt0, nk)
// gives the strip's weights and the unit's k-tile range; the weights stream through the ring
// (kRingSlots chunks of kCKb k-tiles in flight, across unit boundaries), and epi(u, acc) takes
// each unit's accumulators.  The activation rows are brow[] (ncols of them).  False once the
// launch has failed.
template <class UnitFn, class EpiFn>
__device__ __forceinline__ bool stream_bf16(const Params& p, const Ring& R, int first, int step, int nunits,
                                            const uint16_t* const (&brow)[kNT], int ncols, UnitFn unit, EpiFn epi) {
  const int lane = lane_id();
  const uint64_t pol = nkm::policy_evict_first();
  uint32_t phase = *R.phase, inflight = 0;
  int pu = first, pk = 0;  // producer: unit and its next k-tile offset
  auto issue = [&](int slot) {
    if (pu >= nunits) return;
    const uint8_t* base;
    int kt0, nk;
    unit(pu, base, kt0, nk);
    const int n = min(kCKb, nk - pk);
    if (lane == 0) {
      nkm::fence_proxy_async_smem();
      nkm::mbar_arrive_expect_tx(&R.bar[slot], static_cast<uint32_t>(n) * 1024u);
      nkm::bulk_g2s(R.buf + slot * kSlotBytes, base + static_cast<size_t>(kt0 + pk) * 1024, static_cast<uint32_t>(n) * 1024u,
                    &R.bar[slot], pol);
    }
    inflight |= 1u << slot;
    pk += n;
    if (pk >= nk) {
      pk = 0;
      pu += step;
    }
  };
#pragma unroll
  for (int sl = 0; sl < kRingSlots; ++sl) issue(sl);
  int cs = 0;
  bool ok = true;
#pragma unroll 1
  for (int u = first; u < nunits && ok; u += step) {
    const uint8_t* base;
    int kt0, nk;
    unit(u, base, kt0, nk);
    float acc[kNT][4] = {};
#pragma unroll 1
    for (int k = 0; k < nk; k += kCKb) {
      if (!ring_wait(p, R, cs, (phase >> cs) & 1u)) {
        ok = false;
        break;
      }
      phase ^= 1u << cs;
      inflight &= ~(1u << cs);
      if (ncols > 8) bf16_slot<2>(R.buf + cs * kSlotBytes, min(kCKb, nk - k), kt0 + k, brow, acc);
      else bf16_slot<1>(R.buf + cs * kSlotBytes, min(kCKb, nk - k), kt0 + k, brow, acc);
      __syncwarp();
      issue(cs);
      cs = cs + 1 == kRingSlots ? 0 : cs + 1;
    }
    if (!ok) break;
    epi(u, acc);
  }
  if (!ok) ring_drain(R, inflight, phase);
  if (lane == 0) *R.phase = phase;
  __syncwarp();
  return ok;
}

// ------------------------------------------------------------------ stages
// Split-K dense GEMV: units (strip, k chunk) over all warps; partial (chunk kc) of row r, column
// c at part[(kc * rows + r) * B + c].
__device__ __noinline__ void dense_splitk(const Params& p, const uint8_t* w, int rows, int KT, int KC,
                                          const uint16_t* xs, int stride, const Ring& R) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int S = rows / 16, nunits = S * KC;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  const uint16_t* brow[kNT];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) brow[nt] = nt * 8 + g < p.B ? xs + static_cast<size_t>(nt * 8 + g) * stride + 8 * t4 : nullptr;
  stream_bf16(
      p, R, gw, nw, nunits, brow, p.B,
      [&](int u, const uint8_t*& base, int& kt0, int& nk) {
        const int s = u / KC, kc = u - s * KC;
        base = w + static_cast<size_t>(s) * KT * 1024;
        kt0 = KT * kc / KC;
        nk = KT * (kc + 1) / KC - kt0;
      },
      [&](int u, float (&acc)[kNT][4]) {
        const int s = u / KC, kc = u - s * KC;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = nt * 8 + 2 * t4 + e;
            if (c < p.B) {
              p.part[(static_cast<size_t>(kc) * rows + s * 16 + g) * p.B + c] = acc[nt][e];
              p.part[(static_cast<size_t>(kc) * rows + s * 16 + g + 8) * p.B + c] = acc[nt][2 + e];
            }
          }
        }
      });
}

__device__ __forceinline__ int seq_pos(const Params& p, int b) {
  const int raw = __ldg(p.positions + b);
  const int hi = min(p.rope_max, p.max_blocks * kBlk) - 1;
  if (raw < 0 || raw > hi) {
    set_status(p, kStatusIndex);
    return max(0, min(raw, hi));
  }
  return raw;
}

// A2: q/k/v = partials + bias; RoPE on q and k (pairs i, i + 32 of a head, fp32 table); q -> qbuf
// (bf16), K -> cache [slot][64], V -> transposed cache [dim][slot].  One thread per (row, head, i).
__device__ __noinline__ void qkv_finalize(const Params& p, const Layer& lw, int layer) {
  const int nh = p.nq + 2 * p.nkv;
  const int n = p.B * nh * 32;
#pragma unroll 1
  for (int it = blockIdx.x * kThreads + threadIdx.x; it < n; it += gridDim.x * kThreads) {
    const int i = it & 31, bh = it >> 5, b = bh / nh, h = bh - b * nh;
    const int r1 = h * kHD + i, r2 = r1 + 32;
    float x1 = __bfloat162float(__ushort_as_bfloat16(lw.bqkv[r1])), x2 = __bfloat162float(__ushort_as_bfloat16(lw.bqkv[r2]));
    float s1 = 0.f, s2 = 0.f;
    for (int kc = 0; kc < p.kc_qkv; ++kc) {
      s1 += nkm::ldcg_f(p.part + (static_cast<size_t>(kc) * p.R + r1) * p.B + b);
      s2 += nkm::ldcg_f(p.part + (static_cast<size_t>(kc) * p.R + r2) * p.B + b);
    }
    x1 = __fadd_rn(s1, x1);
    x2 = __fadd_rn(s2, x2);
    if (p.tr_qkv) {
      float* tq = p.tr_qkv + (static_cast<size_t>(layer - p.first_layer) * p.B + b) * p.R;
      tq[r1] = x1;
      tq[r2] = x2;
    }
    const int pos = seq_pos(p, b);
    if (h < p.nq + p.nkv) {  // RoPE
      const float c = p.rope_cos[static_cast<size_t>(pos) * 32 + i], s = p.rope_sin[static_cast<size_t>(pos) * 32 + i];
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      x1 = y1;
      x2 = y2;
    }
    if (h < p.nq) {  // f16 q for the f16 products of the FP8 cache, bf16 otherwise
      p.qbuf[static_cast<size_t>(b) * p.nq * kHD + r1] = p.kv_fp8 ? f2h_bits(x1) : f2bf(x1);
      p.qbuf[static_cast<size_t>(b) * p.nq * kHD + r2] = p.kv_fp8 ? f2h_bits(x2) : f2bf(x2);
      continue;
    }
    const bool is_k = h < p.nq + p.nkv;
    const int kh = is_k ? h - p.nq : h - p.nq - p.nkv;
    const int blk = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + pos / kBlk);
    if (blk < 0) continue;  // skip-write convention of the reference
    if (blk >= p.num_blocks) {
      set_status(p, kStatusIndex);
      continue;
    }
    const size_t base = ((static_cast<size_t>(layer) * p.num_blocks + blk) * p.nkv + kh) * (kBlk * kHD);
    const int slot = pos % kBlk;
    if (p.kv_fp8) {
      uint8_t* pool = reinterpret_cast<uint8_t*>(is_k ? p.k_pool : p.v_pool) + base;
      const float sc = is_k ? p.k_scale : p.v_scale;
      if (is_k) {
        pool[static_cast<size_t>(slot) * kHD + i] = to_e4m3(x1, sc);
        pool[static_cast<size_t>(slot) * kHD + i + 32] = to_e4m3(x2, sc);
      } else {
        pool[static_cast<size_t>(i) * kBlk + slot] = to_e4m3(x1, sc);
        pool[static_cast<size_t>(i + 32) * kBlk + slot] = to_e4m3(x2, sc);
      }
    } else if (is_k) {
      p.k_pool[base + static_cast<size_t>(slot) * kHD + i] = f2bf(x1);
      p.k_pool[base + static_cast<size_t>(slot) * kHD + i + 32] = f2bf(x2);
    } else {
      p.v_pool[base + static_cast<size_t>(i) * kBlk + slot] = f2bf(x1);
      p.v_pool[base + static_cast<size_t>(i + 32) * kBlk + slot] = f2bf(x2);
    }
  }
}

// Context of row b: [lo, hi) with the new token included (its K/V were written in A2).
__device__ __forceinline__ void att_range(const Params& p, const Layer& lw, int b, int& lo, int& hi) {
  const int pos = seq_pos(p, b);
  hi = pos + 1;
  lo = lw.sliding ? max(0, pos - (p.window - 1)) : 0;
}
__device__ __forceinline__ int att_nblocks(int lo, int hi) { return (hi - 1) / kBlk - lo / kBlk + 1; }

// Unit base of row b (units of rows < b) computed by every lane.
__device__ __forceinline__ int att_base(const Params& p, const Layer& lw, int b) {
  int base = 0;
  for (int r = 0; r < b; ++r) {
    int lo, hi;
    att_range(p, lw, r, lo, hi);
    base += p.nkv * att_nblocks(lo, hi);
  }
  return base;
}

// B: attention of unit (row b, kv head h, block c of the row's context) by one warp.  16 tokens per
// step: S = Q K^T (mma, Q rows = the group's query heads), online softmax, O += P V with V read from
// the transposed cache.  Token order inside a step is permuted (lane t covers tokens 4t..4t+3 of the
// V^T row) so that every lane reads 8 contiguous bytes; S uses the same permutation.
// kFp8: the cache holds e4m3 bytes; q, K, P and V enter f16 products, the 1/scale factors are
// applied to the scores and to the partial output.
template <bool kFp8>
__device__ __noinline__ void attention_unit(const Params& p, const Layer& lw, int layer, int b, int h, int c, int unit) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  int lo, hi;
  att_range(p, lw, b, lo, hi);
  const int blk_idx = lo / kBlk + c;
  const int tb = max(lo, blk_idx * kBlk), te = min(hi, (blk_idx + 1) * kBlk);
  int blk = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + blk_idx);
  if (blk < 0 || blk >= p.num_blocks) {
    if (lane == 0) set_status(p, kStatusIndex);
    blk = 0;
  }
  const size_t base = ((static_cast<size_t>(layer) * p.num_blocks + blk) * p.nkv + h) * (kBlk * kHD);
  const uint16_t* kb = p.k_pool + base;
  const uint16_t* vb = p.v_pool + base;
  const uint8_t* kb8 = reinterpret_cast<const uint8_t*>(p.k_pool) + base;
  const uint8_t* vb8 = reinterpret_cast<const uint8_t*>(p.v_pool) + base;
  // Q fragments: lane (g, t) holds head rows g and g + 8 of the group, dims 16 t .. 16 t + 15 (four k-steps)
  uint32_t qa[4][4];
  {
    const uint16_t* q0 = p.qbuf + static_cast<size_t>(b) * p.nq * kHD + static_cast<size_t>(h * p.grp) * kHD;
    const bool r0 = g < p.grp, r1 = g + 8 < p.grp;
    uint4 x0 = r0 ? nkm::ldcg128(q0 + g * kHD + 16 * t4) : make_uint4(0u, 0u, 0u, 0u);
    uint4 x1 = r0 ? nkm::ldcg128(q0 + g * kHD + 16 * t4 + 8) : make_uint4(0u, 0u, 0u, 0u);
    uint4 y0 = r1 ? nkm::ldcg128(q0 + (g + 8) * kHD + 16 * t4) : make_uint4(0u, 0u, 0u, 0u);
    uint4 y1 = r1 ? nkm::ldcg128(q0 + (g + 8) * kHD + 16 * t4 + 8) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t a[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const uint32_t d[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qa[ks][0] = a[2 * ks];
      qa[ks][1] = d[2 * ks];
      qa[ks][2] = a[2 * ks + 1];
      qa[ks][3] = d[2 * ks + 1];
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[8][4] = {};
  const float kScale = kFp8 ? 0.125f / p.k_scale : 0.125f;  // 1 / sqrt(64) (and the K dequantisation)
  constexpr float kLog2e = 1.4426950408889634f;
  const int s0 = tb - blk_idx * kBlk, s1 = te - blk_idx * kBlk;  // slot range inside the block
#pragma unroll 1
  for (int st = s0 - (s0 & 15); st < s1; st += 16) {
    // tokens of this lane row: n-tile 0 row g -> slot st + tau(g), n-tile 1 -> st + tau(8 + g)
    const int ta = st + 4 * (g >> 1) + (g & 1), tbk = ta + 2;
    float sc[2][4] = {};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int slot = nt ? tbk : ta;
      uint32_t kw[8];
      if (kFp8) {
        const uint4 k8 = nkm::ldcg128(kb8 + static_cast<size_t>(slot) * kHD + 16 * t4);
        const uint32_t w4[4] = {k8.x, k8.y, k8.z, k8.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          kw[2 * j] = e4m3x2(w4[j] & 0xffffu);
          kw[2 * j + 1] = e4m3x2(w4[j] >> 16);
        }
      } else {
        const uint16_t* kr = kb + static_cast<size_t>(slot) * kHD + 16 * t4;
        const uint4 k0 = nkm::ldcg128(kr), k1 = nkm::ldcg128(kr + 8);
        kw[0] = k0.x; kw[1] = k0.y; kw[2] = k0.z; kw[3] = k0.w;
        kw[4] = k1.x; kw[5] = k1.y; kw[6] = k1.z; kw[7] = k1.w;
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        if (kFp8) mma_f16(sc[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kw[2 * ks], kw[2 * ks + 1]);
        else mma_bf16(sc[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kw[2 * ks], kw[2 * ks + 1]);
      }
    }
    // accumulator (row, col 2t + e) of n-tile nt is token st + 4 t + 2 nt + e
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int slot = st + 4 * t4 + 2 * nt + e;
        const bool ok = slot >= s0 && slot < s1;
        sc[nt][e] = ok ? sc[nt][e] * kScale : -INFINITY;
        sc[nt][2 + e] = ok ? sc[nt][2 + e] * kScale : -INFINITY;
        mx0 = fmaxf(mx0, sc[nt][e]);
        mx1 = fmaxf(mx1, sc[nt][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float al0 = n0 == -INFINITY ? 1.f : exp2f((m0 - n0) * kLog2e);
    const float al1 = n1 == -INFINITY ? 1.f : exp2f((m1 - n1) * kLog2e);
    m0 = n0;
    m1 = n1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      o[nd][0] *= al0;
      o[nd][1] *= al0;
      o[nd][2] *= al1;
      o[nd][3] *= al1;
    }
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pr[nt][e] = sc[nt][e] == -INFINITY ? 0.f : exp2f((sc[nt][e] - n0) * kLog2e);
        pr[nt][2 + e] = sc[nt][2 + e] == -INFINITY ? 0.f : exp2f((sc[nt][2 + e] - n1) * kLog2e);
        l0 += pr[nt][e];
        l1 += pr[nt][2 + e];
      }
    // P as the A operand (k = the 16 tokens in the permuted order) and V^T rows (dims) as B
    auto pk = [](float a, float b2) {
      if (kFp8) {
        const __half2 hh = __floats2half2_rn(a, b2);
        return *reinterpret_cast<const uint32_t*>(&hh);
      }
      return pack_bf2(a, b2);
    };
    const uint32_t pa0 = pk(pr[0][0], pr[0][1]), pa1 = pk(pr[0][2], pr[0][3]);
    const uint32_t pa2 = pk(pr[1][0], pr[1][1]), pa3 = pk(pr[1][2], pr[1][3]);
    const int vs = st + 4 * t4;  // this lane's 4 tokens
    const bool vfull = vs >= s0 && vs + 3 < s1;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      uint2 v;
      if (kFp8) {
        const uint32_t v8 = ldcg_u32(vb8 + static_cast<size_t>(nd * 8 + g) * kBlk + vs);
        v = make_uint2(e4m3x2(v8 & 0xffffu), e4m3x2(v8 >> 16));
      } else {
        v = nkm::ldcg64(vb + static_cast<size_t>(nd * 8 + g) * kBlk + vs);
      }
      if (!vfull) {  // slots outside the context may hold anything: zero them
        const uint32_t m[4] = {vs >= s0 && vs < s1 ? 0xffffu : 0u, vs + 1 >= s0 && vs + 1 < s1 ? 0xffffu : 0u,
                               vs + 2 >= s0 && vs + 2 < s1 ? 0xffffu : 0u, vs + 3 >= s0 && vs + 3 < s1 ? 0xffffu : 0u};
        v.x &= m[0] | (m[1] << 16);
        v.y &= m[2] | (m[3] << 16);
      }
      if (kFp8) mma_f16(o[nd], pa0, pa1, pa2, pa3, v.x, v.y);
      else mma_bf16(o[nd], pa0, pa1, pa2, pa3, v.x, v.y);
    }
  }
  if (kFp8) {
    const float iv = 1.f / p.v_scale;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nd][e] *= iv;
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  float* part = p.att_part + static_cast<size_t>(unit) * kMaxGrp * kPartStride;
  if (g < p.grp) {
    float* r = part + g * kPartStride;
    if (t4 == 0) {
      r[0] = m0;
      r[1] = l0;
    }
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      r[2 + nd * 8 + 2 * t4] = o[nd][0];
      r[2 + nd * 8 + 2 * t4 + 1] = o[nd][1];
    }
  }
  if (g + 8 < p.grp) {
    float* r = part + (g + 8) * kPartStride;
    if (t4 == 0) {
      r[0] = m1;
      r[1] = l1;
    }
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      r[2 + nd * 8 + 2 * t4] = o[nd][2];
      r[2 + nd * 8 + 2 * t4 + 1] = o[nd][3];
    }
  }
}

__device__ __noinline__ void attention_stage(const Params& p, const Layer& lw, int layer) {
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  int total = 0;
  for (int b = 0; b < p.B; ++b) {
    int lo, hi;
    att_range(p, lw, b, lo, hi);
    total += p.nkv * att_nblocks(lo, hi);
  }
#pragma unroll 1
  for (int u = gw; u < total; u += nw) {
    int b = 0, base = 0;
    for (;; ++b) {
      int lo, hi;
      att_range(p, lw, b, lo, hi);
      const int n = p.nkv * att_nblocks(lo, hi);
      if (u < base + n || b == p.B - 1) break;
      base += n;
    }
    int lo, hi;
    att_range(p, lw, b, lo, hi);
    const int nb = att_nblocks(lo, hi), r = u - base;
    if (p.kv_fp8) attention_unit<true>(p, lw, layer, b, r / nb, r % nb, u);
    else attention_unit<false>(p, lw, layer, b, r / nb, r % nb, u);
  }
}

// C0: one warp per (row b, query head): blocks combined in order, the sink logit joins the softmax
// as one more term without a value (attention_tkg.py:186-192); bf16 output.
__device__ __noinline__ void attention_combine(const Params& p, const Layer& lw) {
  const int lane = lane_id();
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll 1
  for (int it = gw; it < p.B * p.nq; it += nw) {
    const int b = it / p.nq, qh = it - b * p.nq, h = qh / p.grp, row = qh - h * p.grp;
    int lo, hi;
    att_range(p, lw, b, lo, hi);
    const int nb = att_nblocks(lo, hi);
    const int u0 = att_base(p, lw, b) + h * nb;
    const float sink = __bfloat162float(__ushort_as_bfloat16(lw.sinks[qh]));
    float M = sink;
    for (int c = 0; c < nb; ++c) M = fmaxf(M, nkm::ldcg_f(p.att_part + (static_cast<size_t>(u0 + c) * kMaxGrp + row) * kPartStride));
    float L = exp2f((sink - M) * kLog2e), o0 = 0.f, o1 = 0.f;
    for (int c = 0; c < nb; ++c) {
      const float* r = p.att_part + (static_cast<size_t>(u0 + c) * kMaxGrp + row) * kPartStride;
      const float m = nkm::ldcg_f(r);
      const float sc = m == -INFINITY ? 0.f : exp2f((m - M) * kLog2e);
      L += nkm::ldcg_f(r + 1) * sc;
      o0 += nkm::ldcg_f(r + 2 + 2 * lane) * sc;
      o1 += nkm::ldcg_f(r + 3 + 2 * lane) * sc;
    }
    const float il = 1.f / L;
    reinterpret_cast<uint32_t*>(p.attn_out + static_cast<size_t>(b) * p.nq * kHD + qh * kHD)[lane] =
        pack_bf2(o0 * il, o1 * il);
  }
}

// C2 / G: residual additions over the grid (one thread per element).  With several ranks each
// thread first stores its elements of this rank's partial into every rank's region, then adds
// the ranks' partials in rank order (the O-projection bias once, after the sum).
__device__ __noinline__ void oproj_residual(const Params& p, const Layer& lw, int layer) {
  const int n = p.B * p.H;
  if (p.n_ranks > 1) {
    const unsigned x = xseq_of(p, 0, layer);
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
      const int b = i / p.H, r = i - b * p.H;
      float s = 0.f;
      for (int kc = 0; kc < p.kc_o; ++kc) s += nkm::ldcg_f(p.part + (static_cast<size_t>(kc) * p.H + r) * p.B + b);
      put_part(p, 0, x, i, s);
    }
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
      const int r = i % p.H;
      float s;
      if (!rank_sum(p, 0, x, i, s)) return;
      const float v = nkm::ldcg_f(p.resid + i) + __fadd_rn(s, __bfloat162float(__ushort_as_bfloat16(lw.bo[r])));
      p.resid[i] = v;
      if (p.tr_mid) p.tr_mid[static_cast<size_t>(layer - p.first_layer) * n + i] = v;
    }
    return;
  }
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
    const int b = i / p.H, r = i - b * p.H;
    float s = 0.f;
    for (int kc = 0; kc < p.kc_o; ++kc) s += nkm::ldcg_f(p.part + (static_cast<size_t>(kc) * p.H + r) * p.B + b);
    const float v = nkm::ldcg_f(p.resid + i) + __fadd_rn(s, __bfloat162float(__ushort_as_bfloat16(lw.bo[r])));
    p.resid[i] = v;
    if (p.tr_mid) p.tr_mid[static_cast<size_t>(layer - p.first_layer) * n + i] = v;
  }
}

// D: router logits (fp32 from the fp32 normalised rows, fixed summation order) + bias; one warp
// per (row, expert).  The normalised rows come from the residual and rstd again (fp32).
__device__ __noinline__ void router_logits(const Params& p, const Layer& lw, int layer, const float* rstd) {
  const int lane = lane_id();
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
#pragma unroll 1
  for (int it = gw; it < p.B * p.E; it += nw) {
    const int t = it / p.E, e = it - t * p.E;
    const float* row = p.resid + static_cast<size_t>(t) * p.H;
    const uint16_t* wr = lw.router + static_cast<size_t>(e) * p.H;
    const float r = rstd[t];
    float acc = 0.f;
    // two 256-wide steps per round: their loads are issued together, then summed in k order
#pragma unroll 1
    for (int k0 = 8 * lane; k0 < p.H; k0 += 2 * 256) {
      float4 a[2], bb[2];
      uint4 gv[2], wv[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int k = k0 + 256 * q;
        if (k < p.H) {
          a[q] = nkm::ldcg_f4(row + k);
          bb[q] = nkm::ldcg_f4(row + k + 4);
          gv[q] = *reinterpret_cast<const uint4*>(lw.ln2 + k);
          wv[q] = nkm::ldnc128(wr + k);
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (k0 + 256 * q < p.H) {
          const float v[8] = {a[q].x, a[q].y, a[q].z, a[q].w, bb[q].x, bb[q].y, bb[q].z, bb[q].w};
          const uint32_t gw4[4] = {gv[q].x, gv[q].y, gv[q].z, gv[q].w}, ww[4] = {wv[q].x, wv[q].y, wv[q].z, wv[q].w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xn = __fmul_rn(__fmul_rn(v[j], r), (j & 1) ? hi_bf(gw4[j >> 1]) : lo_bf(gw4[j >> 1]));
            acc = __fadd_rn(acc, __fmul_rn((j & 1) ? hi_bf(ww[j >> 1]) : lo_bf(ww[j >> 1]), xn));
          }
        }
      }
    }
    acc = warp_sum(acc);
    acc = __fadd_rn(acc, __bfloat162float(__ushort_as_bfloat16(lw.router_b[e])));
    if (lane == 0) {
      p.rlogits[it] = acc;
      if (p.tr_rlogits) p.tr_rlogits[static_cast<size_t>(layer - p.first_layer) * p.B * p.E + it] = acc;
    }
  }
}

// E prologue (every CTA): top-k of each row's logits (ties to the lower expert), softmax over the k,
// and the expert tables (active experts ascending, each expert's pairs in token order).
__device__ __noinline__ void routing(const Params& p, Route* rt, int layer) {
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const int E = p.E, K = p.K;
#pragma unroll 1
  for (int t = warp; t < p.B; t += kWarps) {
    float v[kMaxE / 32];
#pragma unroll
    for (int q = 0; q < kMaxE / 32; ++q) {
      const int e = 32 * q + lane;
      v[q] = e < E ? nkm::ldcg_f(p.rlogits + static_cast<size_t>(t) * E + e) : -INFINITY;
    }
    float top[kMaxTopK];
    int idx[kMaxTopK];
#pragma unroll 1
    for (int k = 0; k < K; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < kMaxE / 32; ++q) {
        const int e = 32 * q + lane;
        if (e < E && (v[q] > bv || (v[q] == bv && e < bi))) {
          bv = v[q];
          bi = e;
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      top[k] = bv;
      idx[k] = bi;
#pragma unroll
      for (int q = 0; q < kMaxE / 32; ++q)
        if (32 * q + lane == bi) v[q] = -INFINITY;
    }
    if (lane == 0) {
      float s = 0.f, ex[kMaxTopK];
      for (int k = 0; k < K; ++k) {
        ex[k] = expf(top[k] - top[0]);
        s += ex[k];
      }
      for (int k = 0; k < K; ++k) {
        rt->topk_idx[t * K + k] = idx[k];
        rt->topk_w[t * K + k] = ex[k] / s;
      }
    }
  }
  for (int e = threadIdx.x; e < E; e += kThreads) rt->cnt[e] = 0;
  __syncthreads();
  const int NP = p.B * K, i = threadIdx.x;
  if (i < NP) atomicAdd(&rt->cnt[rt->topk_idx[i]], 1);
  __syncthreads();
  if (threadIdx.x == 0) {  // active experts ascending; cnt[e] becomes the pair offset of expert e
    // (with several ranks only this rank's experts [expert_begin, expert_begin + n_local) enter)
    int off = 0, na = 0;
    const int e_lo = p.expert_begin, e_hi = p.expert_begin + p.n_local;
    for (int e = 0; e < E; ++e) {
      const int n = (e >= e_lo && e < e_hi) ? rt->cnt[e] : 0;
      rt->cnt[e] = off;
      if (n > 0) {
        rt->act_e[na] = e;
        rt->act_off[na] = off;
        rt->act_cnt[na] = n;
        ++na;
        off += n;
      }
    }
    rt->nA = na;
  }
  __syncthreads();
  if (i < NP) {
    const int e = rt->topk_idx[i], t = i / K;
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += rt->topk_idx[j] == e;
    const bool local = e >= p.expert_begin && e < p.expert_begin + p.n_local;
    const int pr = rt->cnt[e] + rank;
    if (local) {
      rt->pair_tok[pr] = t;
      rt->pair_w[pr] = rt->topk_w[i];
    }
    rt->pair_of[i] = local ? pr : -1;
    if (blockIdx.x == 0 && p.tr_idx) {
      p.tr_idx[static_cast<size_t>(layer - p.first_layer) * NP + i] = e;
      p.tr_w[static_cast<size_t>(layer - p.first_layer) * NP + i] = rt->topk_w[i];
    }
  }
  __syncthreads();
}

// E: gate/up units (active expert j, 16-row strip s of the interleaved 2I rows): the expert's
// tokens gathered from the f16 rows in shared memory; bias, clamp, SwiGLU; h (f16) per pair.
// Warp gw takes units gw, gw + nw, ...; their weights and scales stream through the warp's ring
// (kRingSlots chunks of kCK k-tiles in flight, across unit boundaries).
__device__ __noinline__ void expert_gateup(const Params& p, const Layer& lw, const Route* rt, const uint16_t* xs,
                                           const Ring& R) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  const int S = 2 * p.I / 16, KT = p.H / 32, NC = (KT + kCK - 1) / kCK, nunits = rt->nA * S;
  const size_t ebytes = static_cast<size_t>(2 * p.I) * p.H / 2, ssb = fp4_strip_scale_bytes(KT), sbytes = S * ssb;
  const uint64_t pol = nkm::policy_evict_first();
  uint32_t phase = *R.phase, inflight = 0;
  int pu = gw, pc = 0;  // producer: unit and chunk of the next copy
  auto issue = [&](int slot) {
    if (pu >= nunits) return;
    const int j = pu / S, s = pu - j * S, e = rt->act_e[j] - p.expert_begin;  // this rank's expert index
    const int nk = min(kCK, KT - pc * kCK);
    if (lane == 0)
      ring_issue(R, slot, lw.w13 + e * ebytes + static_cast<size_t>(s) * KT * 256 + static_cast<size_t>(pc) * kCK * 256,
                 lw.s13 + e * sbytes + s * ssb + static_cast<size_t>(pc) * (kCK / 8) * 128, nk, pol);
    inflight |= 1u << slot;
    if (++pc == NC) {
      pc = 0;
      pu += nw;
    }
  };
#pragma unroll
  for (int sl = 0; sl < kRingSlots; ++sl) issue(sl);
  int cs = 0;
  bool ok = true;
#pragma unroll 1
  for (int u = gw; u < nunits && ok; u += nw) {
    const int j = u / S, s = u - j * S, e = rt->act_e[j] - p.expert_begin;
    const int* cols = rt->pair_tok + rt->act_off[j];
    const int ncols = rt->act_cnt[j];
    const uint16_t* brow[kNT];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const int c = nt * 8 + g;
      brow[nt] = c < ncols ? xs + static_cast<size_t>(cols[c]) * (p.H + 8) + 8 * t4 : nullptr;
    }
    float acc[kNT][4] = {};
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      if (!ring_wait(p, R, cs, (phase >> cs) & 1u)) {
        ok = false;
        break;
      }
      phase ^= 1u << cs;
      inflight &= ~(1u << cs);
      if (ncols > 8) fp4_slot<2>(R.buf + cs * kSlotBytes, min(kCK, KT - c * kCK), c * kCK, brow, acc);
      else fp4_slot<1>(R.buf + cs * kSlotBytes, min(kCK, KT - c * kCK), c * kCK, brow, acc);
      __syncwarp();
      issue(cs);
      cs = cs + 1 == kRingSlots ? 0 : cs + 1;
    }
    if (!ok) break;
    // rows 16 s + g (even: gate, odd: up) pair up across lanes g, g ^ 1
    const int r0 = 16 * s + g, r1 = r0 + 8;
    const float b0 = __bfloat162float(__ushort_as_bfloat16(lw.b13[static_cast<size_t>(e) * 2 * p.I + r0]));
    const float b1 = __bfloat162float(__ushort_as_bfloat16(lw.b13[static_cast<size_t>(e) * 2 * p.I + r1]));
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
#pragma unroll
      for (int ee = 0; ee < 2; ++ee) {
        const float v0 = acc[nt][ee] + b0, v1 = acc[nt][2 + ee] + b1;
        const float w0 = __shfl_xor_sync(0xffffffffu, v0, 4), w1 = __shfl_xor_sync(0xffffffffu, v1, 4);
        const int c = nt * 8 + 2 * t4 + ee;
        if ((g & 1) == 0 && c < ncols) {
          const int pr = rt->act_off[j] + c;
          // (v0: gate row r0, w0: up row r0 + 1), (v1: gate row r1, w1: up row r1 + 1)
          const float gate0 = fminf(v0, p.limit), up0 = fminf(fmaxf(w0, -p.limit), p.limit);
          const float gate1 = fminf(v1, p.limit), up1 = fminf(fmaxf(w1, -p.limit), p.limit);
          const float h0 = (up0 + 1.f) * (gate0 / (1.f + expf(-gate0 * p.alpha)));
          const float h1 = (up1 + 1.f) * (gate1 / (1.f + expf(-gate1 * p.alpha)));
          __half* hb = reinterpret_cast<__half*>(p.hbuf) + static_cast<size_t>(pr) * p.I;
          hb[r0 >> 1] = __float2half_rn(h0);
          hb[r1 >> 1] = __float2half_rn(h1);
        }
      }
    }
  }
  if (!ok) ring_drain(R, inflight, phase);
  if (lane == 0) *R.phase = phase;
  __syncwarp();
}

// F: down projection.  The nA x H/16 (expert, 16-row strip) units in expert-major order are split
// into contiguous ranges, one per CTA, so a CTA meets at most a few experts: for each it copies the
// expert's h rows (f16, written in stage E by other CTAs) into shared memory once and its warps
// take the expert's strips of its range (warp w: the range's strips w, w + 8, ... of that expert);
// y = acc + bias, times the pair's routing weight -> ypair.  Each warp's weights stream through its
// ring in the order it computes them, across strips and experts (the copies do not depend on h).
__device__ __noinline__ void expert_down(const Params& p, const Layer& lw, const Route* rt, uint16_t* hs,
                                         const Ring& R) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3, warp = threadIdx.x >> 5;
  const int S = p.H / 16, KT = p.I / 32, NC = (KT + kCK - 1) / kCK, NS = rt->nA * S;
  const size_t ebytes = static_cast<size_t>(p.H) * p.I / 2, ssb = fp4_strip_scale_bytes(KT), sbytes = S * ssb;
  const int hstride = p.I + 8;
  const int lo = static_cast<int>((static_cast<long long>(NS) * blockIdx.x) / gridDim.x);
  const int hi = static_cast<int>((static_cast<long long>(NS) * (blockIdx.x + 1)) / gridDim.x);
  // this warp's units in computing order: its first unit in the expert segments from `seg` on,
  // and the unit after st (-1: none)
  auto first_from = [&](int seg) {
#pragma unroll 1
    while (seg < hi) {
      const int e_end = min(hi, (seg / S + 1) * S);
      if (seg + warp < e_end) return seg + warp;
      seg = e_end;
    }
    return -1;
  };
  auto next_unit = [&](int st) {
    const int seg_end = min(hi, (st / S + 1) * S);
    return st + kWarps < seg_end ? st + kWarps : first_from(seg_end);
  };
  const int first = first_from(lo);
  const uint64_t pol = nkm::policy_evict_first();
  uint32_t phase = *R.phase, inflight = 0;
  int pu = first, pc = 0;
  auto issue = [&](int slot) {
    if (pu < 0) return;
    const int j = pu / S, s = pu - j * S, e = rt->act_e[j] - p.expert_begin;
    const int nk = min(kCK, KT - pc * kCK);
    if (lane == 0)
      ring_issue(R, slot, lw.w2 + e * ebytes + static_cast<size_t>(s) * KT * 256 + static_cast<size_t>(pc) * kCK * 256,
                 lw.s2 + e * sbytes + s * ssb + static_cast<size_t>(pc) * (kCK / 8) * 128, nk, pol);
    inflight |= 1u << slot;
    if (++pc == NC) {
      pc = 0;
      pu = next_unit(pu);
    }
  };
#pragma unroll
  for (int sl = 0; sl < kRingSlots; ++sl) issue(sl);
  int cs = 0;
  bool ok = true;
#pragma unroll 1
  for (int seg = lo; seg < hi;) {
    const int j = seg / S, seg_end = min(hi, (j + 1) * S);
    const int e = rt->act_e[j] - p.expert_begin, off = rt->act_off[j], n = rt->act_cnt[j];
    __syncthreads();  // the previous expert's rows are no longer read
    for (int i = threadIdx.x; i < n * (p.I / 8); i += kThreads) {
      const int r = i / (p.I / 8), k = (i - r * (p.I / 8)) * 8;
      *reinterpret_cast<uint4*>(hs + static_cast<size_t>(r) * hstride + k) =
          nkm::ldcg128(p.hbuf + static_cast<size_t>(off + r) * p.I + k);
    }
    __syncthreads();
    const uint16_t* brow[kNT];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const int c = nt * 8 + g;
      brow[nt] = c < n ? hs + static_cast<size_t>(c) * hstride + 8 * t4 : nullptr;
    }
#pragma unroll 1
    for (int st = seg + warp; st < seg_end && ok; st += kWarps) {
      const int s = st - j * S;
      float acc[kNT][4] = {};
#pragma unroll 1
      for (int c = 0; c < NC; ++c) {
        if (!ring_wait(p, R, cs, (phase >> cs) & 1u)) {
          ok = false;
          break;
        }
        phase ^= 1u << cs;
        inflight &= ~(1u << cs);
        if (n > 8) fp4_slot<2>(R.buf + cs * kSlotBytes, min(kCK, KT - c * kCK), c * kCK, brow, acc);
        else fp4_slot<1>(R.buf + cs * kSlotBytes, min(kCK, KT - c * kCK), c * kCK, brow, acc);
        __syncwarp();
        issue(cs);
        cs = cs + 1 == kRingSlots ? 0 : cs + 1;
      }
      if (!ok) break;
      const int r0 = 16 * s + g, r1 = r0 + 8;
      const float b0 = __bfloat162float(__ushort_as_bfloat16(lw.b2[static_cast<size_t>(e) * p.H + r0]));
      const float b1 = __bfloat162float(__ushort_as_bfloat16(lw.b2[static_cast<size_t>(e) * p.H + r1]));
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int ee = 0; ee < 2; ++ee) {
          const int c = nt * 8 + 2 * t4 + ee;
          if (c < n) {
            const float w = rt->pair_w[off + c];
            float* y = p.ypair + static_cast<size_t>(off + c) * p.H;
            y[r0] = (acc[nt][ee] + b0) * w;
            y[r1] = (acc[nt][2 + ee] + b1) * w;
          }
        }
    }
    seg = seg_end;
  }
  if (!ok) ring_drain(R, inflight, phase);
  if (lane == 0) *R.phase = phase;
  __syncwarp();
}

__device__ __noinline__ void moe_residual(const Params& p, const Route* rt, int layer) {
  const int n = p.B * p.H;
  if (p.n_ranks > 1) {
    // this rank's experts' slots (in slot order; the other slots are other ranks') to every rank,
    // then the ranks' sums in rank order
    const unsigned x = xseq_of(p, 1, layer);
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
      const int b = i / p.H, r = i - b * p.H;
      float s = 0.f;
      for (int k = 0; k < p.K; ++k) {
        const int pr = rt->pair_of[b * p.K + k];
        if (pr >= 0) s += nkm::ldcg_f(p.ypair + static_cast<size_t>(pr) * p.H + r);
      }
      put_part(p, 1, x, i, s);
    }
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
      float s;
      if (!rank_sum(p, 1, x, i, s)) return;
      const float v = nkm::ldcg_f(p.resid + i) + s;
      p.resid[i] = v;
      if (p.tr_out) p.tr_out[static_cast<size_t>(layer - p.first_layer) * n + i] = v;
    }
    return;
  }
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
    const int b = i / p.H, r = i - b * p.H;
    float s = 0.f;
    for (int k = 0; k < p.K; ++k) s += nkm::ldcg_f(p.ypair + static_cast<size_t>(rt->pair_of[b * p.K + k]) * p.H + r);
    const float v = nkm::ldcg_f(p.resid + i) + s;
    p.resid[i] = v;
    if (p.tr_out) p.tr_out[static_cast<size_t>(layer - p.first_layer) * n + i] = v;
  }
}

// LM head: one warp per 16-row strip of this rank's part of the vocabulary (whole K).  With
// several ranks the logits go as tagged words into every rank's region (lm_copy gathers them).
__device__ __noinline__ void lm_head(const Params& p, const uint16_t* xs, const Ring& R) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  const int KT = p.H / 32;
  const bool multi = p.n_ranks > 1;
  const unsigned x = multi ? xseq_of(p, 2, 0) : 0u;
  const uint16_t* brow[kNT];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) brow[nt] = nt * 8 + g < p.B ? xs + static_cast<size_t>(nt * 8 + g) * (p.H + 8) + 8 * t4 : nullptr;
  stream_bf16(
      p, R, gw, nw, p.lm_ns, brow, p.B,
      [&](int u, const uint8_t*& base, int& kt0, int& nk) {
        base = p.lm_head + static_cast<size_t>(p.lm_s0 + u) * KT * 1024;
        kt0 = 0;
        nk = KT;
      },
      [&](int u, float (&acc)[kNT][4]) {
        const int s = p.lm_s0 + u;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
          for (int ee = 0; ee < 2; ++ee) {
            const int c = nt * 8 + 2 * t4 + ee;
            if (c < p.B) {
              const size_t i0 = static_cast<size_t>(c) * p.V + 16 * s + g;
              if (multi) {
                const unsigned long long w0 = xword(x, acc[nt][ee]), w1 = xword(x, acc[nt][2 + ee]);
#pragma unroll 1
                for (int q = 0; q < p.n_ranks; ++q) {
                  nkm::st_relaxed_sys_u64(xw_logits(p, q, x) + i0, w0);
                  nkm::st_relaxed_sys_u64(xw_logits(p, q, x) + i0 + 8, w1);
                }
              } else {
                p.logits_out[i0] = acc[nt][ee];
                p.logits_out[i0 + 8] = acc[nt][2 + ee];
              }
            }
          }
      });
}

// Several ranks: every rank's logits, from this rank's region into logits_out (each word waited
// for until it carries this launch's tag).
__device__ __noinline__ void lm_copy(const Params& p) {
  const unsigned x = xseq_of(p, 2, 0);
  const unsigned long long* src = xw_logits(p, p.rank, x);
  const size_t n = static_cast<size_t>(p.B) * p.V, st = static_cast<size_t>(gridDim.x) * kThreads;
  constexpr int U = 8;  // independent loads in flight per thread
  for (size_t i0 = blockIdx.x * static_cast<size_t>(kThreads) + threadIdx.x; i0 < n; i0 += U * st) {
    unsigned long long w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) w[u] = i0 + u * st < n ? nkm::ld_relaxed_sys_u64(src + i0 + u * st) : 0ull;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const size_t i = i0 + u * st;
      if (i >= n) break;
      float v = __uint_as_float(static_cast<unsigned>(w[u]));
      if (static_cast<unsigned>(w[u] >> 32) != x + 1u && !take_word(p, src + i, x, v)) return;
      p.logits_out[i] = v;
    }
  }
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) gptoss_decode_kernel(const __grid_constant__ Params pk) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ __align__(16) Params sp;
  static_assert(sizeof(Params) % 4 == 0 && sizeof(Params) / 4 <= kThreads, "Params copy");
  if (threadIdx.x < sizeof(Params) / 4)
    reinterpret_cast<uint32_t*>(&sp)[threadIdx.x] = reinterpret_cast<const uint32_t*>(&pk)[threadIdx.x];
  __syncthreads();
  const Params& p = sp;
  const int kx = max(max(p.H, p.nq * kHD), p.I);
  const Smem lay(kMaxB, kx);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + lay.xs_off);
  float* rstd = reinterpret_cast<float*>(smem + lay.rstd_off);
  Route* rt = reinterpret_cast<Route*>(smem + lay.route_off);
  int* flag = reinterpret_cast<int*>(smem + lay.flag_off);
  const int warp_i = threadIdx.x >> 5;
  const Ring ring{smem + lay.ring_off + warp_i * kRingSlots * kSlotBytes,
                  reinterpret_cast<uint64_t*>(smem + lay.bar_off) + warp_i * kRingSlots,
                  reinterpret_cast<uint32_t*>(smem + lay.phase_off) + warp_i};
  if (lane_id() == 0) {
    for (int sl = 0; sl < kRingSlots; ++sl) nkm::mbar_init(&ring.bar[sl], 1);
    *ring.phase = 0u;
    nkm::fence_mbar_init();
  }
  __syncthreads();
  unsigned bar_k = 0;
  if (p.tr_stage && blockIdx.x == 0 && threadIdx.x == 0) p.tr_stage[0] = static_cast<int64_t>(globaltimer_ns());

  [&]() {
    // residual (fp32) <- embeddings / hidden input
    const int nvec = p.B * p.H / 8;
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
      const uint4 v = nkm::ldnc128(src);
      float* dst = p.resid + static_cast<size_t>(t) * p.H + k;
      *reinterpret_cast<float4*>(dst) = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y));
      *reinterpret_cast<float4*>(dst + 4) = make_float4(lo_bf(v.z), hi_bf(v.z), lo_bf(v.w), hi_bf(v.w));
    }
    if (!grid_sync(p, bar_k, flag)) return;
    const int layer_end = p.first_layer + p.num_layers;
#pragma unroll 1
    for (int layer = p.first_layer; layer < layer_end; ++layer) {
      const Layer& lw = p.layers[layer - p.first_layer];
      // A
      norm_rows(p, lw.ln1, xs, rstd, false);
      __syncthreads();
      dense_splitk(p, lw.wqkv, p.R, p.H / 32, p.kc_qkv, xs, p.H + 8, ring);
      if (!grid_sync(p, bar_k, flag)) return;
      qkv_finalize(p, lw, layer);  // A2
      if (!grid_sync(p, bar_k, flag)) return;
      attention_stage(p, lw, layer);  // B
      if (!grid_sync(p, bar_k, flag)) return;
      attention_combine(p, lw);  // C0
      if (!grid_sync(p, bar_k, flag)) return;
      {  // C: attention output rows into shared memory, O-projection
        const int Kq = p.nq * kHD, stride = Kq + 8;
        for (int i = threadIdx.x; i < kMaxB * (Kq / 8); i += kThreads) {
          const int t = i / (Kq / 8), k = (i - t * (Kq / 8)) * 8;
          const uint4 v = t < p.B ? nkm::ldcg128(p.attn_out + static_cast<size_t>(t) * Kq + k) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(xs + static_cast<size_t>(t) * stride + k) = v;
        }
        __syncthreads();
        dense_splitk(p, lw.wo, p.H, Kq / 32, p.kc_o, xs, stride, ring);
      }
      if (!grid_sync(p, bar_k, flag)) return;
      oproj_residual(p, lw, layer);  // C2
      if (!grid_sync(p, bar_k, flag)) return;
      norm_rows(p, lw.ln2, xs, rstd, true);  // D (f16 rows stay in shared memory for stage E)
      __syncthreads();  // every row's rstd (written by its warp) before any warp scores it
      router_logits(p, lw, layer, rstd);
      if (!grid_sync(p, bar_k, flag)) return;
      routing(p, rt, layer);  // E
      expert_gateup(p, lw, rt, xs, ring);
      if (!grid_sync(p, bar_k, flag)) return;
      expert_down(p, lw, rt, xs, ring);  // F (the f16 rows of stage D are no longer needed)
      if (!grid_sync(p, bar_k, flag)) return;
      moe_residual(p, rt, layer);  // G
      if (!grid_sync(p, bar_k, flag)) return;
    }
    // outputs
    for (int i = blockIdx.x * kThreads + threadIdx.x; i < p.B * p.H / 8; i += gridDim.x * kThreads) {
      const float4 a = nkm::ldcg_f4(p.resid + static_cast<size_t>(i) * 8);
      const float4 b = nkm::ldcg_f4(p.resid + static_cast<size_t>(i) * 8 + 4);
      reinterpret_cast<uint4*>(p.y_out)[i] =
          make_uint4(pack_bf2(a.x, a.y), pack_bf2(a.z, a.w), pack_bf2(b.x, b.y), pack_bf2(b.z, b.w));
    }
    if (p.want_lm) {
      norm_rows(p, p.final_norm, xs, rstd, false);
      __syncthreads();
      lm_head(p, xs, ring);
      if (p.n_ranks > 1) lm_copy(p);
    }
    __syncthreads();
    if (p.tr_stage && blockIdx.x == 0 && threadIdx.x == 0) p.tr_stage[bar_k + 1] = static_cast<int64_t>(globaltimer_ns());
  }();
  // end of the launch: the last CTA out resets the barrier counter
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = nkm::atom_acqrel_add_u32(p.bar + 2, 1u);
    if (old == gridDim.x - 1) {
      if (p.n_ranks > 1) {  // the exchanges this launch took (every other CTA has left it)
        p.xseq[0] += static_cast<unsigned>(p.num_layers);
        p.xseq[1] += static_cast<unsigned>(p.num_layers);
        if (p.want_lm) p.xseq[2] += 1u;
      }
      *reinterpret_cast<volatile unsigned*>(p.bar) = 0u;
      *reinterpret_cast<volatile unsigned*>(p.bar + 2) = 0u;
    }
  }
}

}  // namespace nkg
