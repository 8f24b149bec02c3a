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

// Shared memory: activation rows (bf16 or f16, stride Kx + 8 halves) | rstd | route | flag.
struct Smem {
  uint32_t xs_off, rstd_off, route_off, flag_off, total;
  __host__ __device__ explicit Smem(int B, int kmax) {
    xs_off = 0;
    uint32_t xs = static_cast<uint32_t>(B) * static_cast<uint32_t>(kmax + 8) * 2u;
    rstd_off = (xs + 15u) & ~15u;
    route_off = rstd_off + kMaxB * 4;
    flag_off = route_off + static_cast<uint32_t>((sizeof(Route) + 15) & ~size_t(15));
    total = flag_off + 16;
  }
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
// bf16 fragment-tiled strip (1 KB units of 16 rows x 32 k; lane l: row l/4 and l/4 + 8, k 8(l%4)..+7)
// times shared-memory columns: acc[nt] += W[strip, kt0 .. kt0+nk) x^T for columns nt*8 + g.
// cols: shared-memory row of each column (nullptr: column c is row c); ncols columns valid.
__device__ __forceinline__ void ft_bf16(const uint8_t* strip, int kt0, int nk, const uint16_t* xs, int stride,
                                        const int* cols, int ncols, float (&acc)[kNT][4]) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const uint16_t* brow[kNT];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) {
    const int c = nt * 8 + g;
    brow[nt] = c < ncols ? xs + static_cast<size_t>(cols ? cols[c] : c) * stride + 8 * t4 : nullptr;
  }
  constexpr int U = 8;
#pragma unroll 1
  for (int k0 = 0; k0 < nk; k0 += U) {
    uint4 a0[U], a1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (k0 + u < nk) {
        const uint8_t* unit = strip + static_cast<size_t>(kt0 + k0 + u) * 1024;
        a0[u] = nkm::ldnc128(unit + 16 * lane);
        a1[u] = nkm::ldnc128(unit + 512 + 16 * lane);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (k0 + u < nk) {
        const int kk = (kt0 + k0 + u) * 32;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
          const uint4 b = brow[nt] ? *reinterpret_cast<const uint4*>(brow[nt] + kk) : make_uint4(0u, 0u, 0u, 0u);
          mma_bf16(acc[nt], a0[u].x, a1[u].x, a0[u].y, a1[u].y, b.x, b.y);
          mma_bf16(acc[nt], a0[u].z, a1[u].z, a0[u].w, a1[u].w, b.z, b.w);
        }
      }
    }
  }
}

// MXFP4 fragment-tiled strip: 256-byte units of 16 rows x 32 k (lane l: 4 bytes of row l/4 then 4
// bytes of row l/4 + 8, k 8(l%4)..+7, low nibble first) and the strip's e8m0 scales in groups of 8
// k-tiles ([group][16 rows][8], so a lane reads its two rows' 8 scales with two 8-byte loads).
// Each unit's product is accumulated from zero and scaled by its rows' scales (exact powers of
// two).  8 k-tiles are in flight per lane; the callers warm L2 with the warp's next unit (one
// bulk prefetch) while this one streams.
__device__ __forceinline__ uint32_t byte_of(const uint2 v, int u) {
  return ((u < 4 ? v.x : v.y) >> (8 * (u & 3))) & 0xffu;
}
__device__ __forceinline__ void ft_fp4(const uint8_t* strip, const uint8_t* scales, int nk, const uint16_t* xs,
                                       int stride, const int* cols, int ncols, float (&acc)[kNT][4]) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const uint16_t* brow[kNT];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt) {
    const int c = nt * 8 + g;
    brow[nt] = c < ncols ? xs + static_cast<size_t>(cols ? cols[c] : c) * stride + 8 * t4 : nullptr;
  }
  constexpr int U = 8;
#pragma unroll 1
  for (int k0 = 0; k0 < nk; k0 += U) {
    uint2 w[U], sg[U / 8], sh[U / 8];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u < nk) w[u] = ldnc64(strip + static_cast<size_t>(k0 + u) * 256 + 8 * lane);
#pragma unroll
    for (int q = 0; q < U / 8; ++q) {
      if (k0 + 8 * q < nk) {
        const uint8_t* grp = scales + static_cast<size_t>(k0 / 8 + q) * 128;
        sg[q] = ldnc64(grp + 8 * g);
        sh[q] = ldnc64(grp + 8 * (g + 8));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (k0 + u < nk) {
        uint32_t r0, r1, r2, r3, q0, q1, q2, q3;
        e2m1x8(w[u].x, r0, r1, r2, r3);
        e2m1x8(w[u].y, q0, q1, q2, q3);
        const float s0 = e8m0(byte_of(sg[u / 8], u & 7)), s1 = e8m0(byte_of(sh[u / 8], u & 7));
        const int kk = (k0 + u) * 32;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
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
// Bytes of one 16-row strip's grouped scales for KT k-tiles.
__device__ __forceinline__ size_t fp4_strip_scale_bytes(int KT) { return static_cast<size_t>((KT + 7) / 8) * 128; }

// ------------------------------------------------------------------ stages
// Split-K dense GEMV: units (strip, k chunk) over all warps; partial (chunk kc) of row r, column
// c at part[(kc * rows + r) * B + c].
__device__ __noinline__ void dense_splitk(const Params& p, const uint8_t* w, int rows, int KT, int KC,
                                          const uint16_t* xs, int stride) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int S = rows / 16, nunits = S * KC;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
#pragma unroll 1
  for (int u = gw; u < nunits; u += nw) {
    const int s = u / KC, kc = u - s * KC;
    const int kt0 = KT * kc / KC, kt1 = KT * (kc + 1) / KC;
    if (lane == 0 && u + nw < nunits) {  // the next unit's weights into L2
      const int s2 = (u + nw) / KC, kc2 = (u + nw) - s2 * KC;
      const int a0 = KT * kc2 / KC, a1 = KT * (kc2 + 1) / KC;
      nkm::prefetch_l2_bulk(w + (static_cast<size_t>(s2) * KT + a0) * 1024, static_cast<uint32_t>(a1 - a0) * 1024u);
    }
    float acc[kNT][4] = {};
    ft_bf16(w + static_cast<size_t>(s) * KT * 1024, kt0, kt1 - kt0, xs, stride, nullptr, p.B, acc);
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
  }
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

// C2 / G: residual additions over the grid (one thread per element).
__device__ __noinline__ void oproj_residual(const Params& p, const Layer& lw, int layer) {
  const int n = p.B * p.H;
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
    int off = 0, na = 0;
    for (int e = 0; e < E; ++e) {
      const int n = rt->cnt[e];
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
    const int pr = rt->cnt[e] + rank;
    rt->pair_tok[pr] = t;
    rt->pair_w[pr] = rt->topk_w[i];
    rt->pair_of[i] = pr;
    if (blockIdx.x == 0 && p.tr_idx) {
      p.tr_idx[static_cast<size_t>(layer - p.first_layer) * NP + i] = e;
      p.tr_w[static_cast<size_t>(layer - p.first_layer) * NP + i] = rt->topk_w[i];
    }
  }
  __syncthreads();
}

// E: gate/up units (active expert j, 16-row strip s of the interleaved 2I rows): the expert's
// tokens gathered from the f16 rows in shared memory; bias, clamp, SwiGLU; h (f16) per pair.
__device__ __noinline__ void expert_gateup(const Params& p, const Layer& lw, const Route* rt, const uint16_t* xs) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  const int S = 2 * p.I / 16, KT = p.H / 32, nunits = rt->nA * S;
  const size_t ebytes = static_cast<size_t>(2 * p.I) * p.H / 2, ssb = fp4_strip_scale_bytes(KT), sbytes = S * ssb;
#pragma unroll 1
  for (int u = gw; u < nunits; u += nw) {
    const int j = u / S, s = u - j * S, e = rt->act_e[j];
    if (lane == 0 && u + nw < nunits) {  // the next unit's weights and scales into L2
      const int j2 = (u + nw) / S, s2 = (u + nw) - j2 * S, e2 = rt->act_e[j2];
      nkm::prefetch_l2_bulk(lw.w13 + e2 * ebytes + static_cast<size_t>(s2) * KT * 256, static_cast<uint32_t>(KT) * 256u);
      nkm::prefetch_l2_bulk(lw.s13 + e2 * sbytes + s2 * ssb, static_cast<uint32_t>(ssb));
    }
    float acc[kNT][4] = {};
    ft_fp4(lw.w13 + e * ebytes + static_cast<size_t>(s) * KT * 256, lw.s13 + e * sbytes + s * ssb, KT, xs, p.H + 8,
           rt->pair_tok + rt->act_off[j], rt->act_cnt[j], acc);
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
        if ((g & 1) == 0 && c < rt->act_cnt[j]) {
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
}

// F: down projection.  The nA x H/16 (expert, 16-row strip) units in expert-major order are split
// into contiguous ranges, one per CTA, so a CTA meets at most a few experts: for each it copies the
// expert's h rows (f16, written in stage E by other CTAs) into shared memory once and its warps
// take the expert's strips of its range; y = acc + bias, times the pair's routing weight -> ypair.
__device__ __noinline__ void expert_down(const Params& p, const Layer& lw, const Route* rt, uint16_t* hs) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3, warp = threadIdx.x >> 5;
  const int S = p.H / 16, KT = p.I / 32, NS = rt->nA * S;
  const size_t ebytes = static_cast<size_t>(p.H) * p.I / 2, ssb = fp4_strip_scale_bytes(KT), sbytes = S * ssb;
  const int hstride = p.I + 8;
  const int lo = static_cast<int>((static_cast<long long>(NS) * blockIdx.x) / gridDim.x);
  const int hi = static_cast<int>((static_cast<long long>(NS) * (blockIdx.x + 1)) / gridDim.x);
#pragma unroll 1
  for (int seg = lo; seg < hi;) {
    const int j = seg / S, seg_end = min(hi, (j + 1) * S);
    const int e = rt->act_e[j], off = rt->act_off[j], n = rt->act_cnt[j];
    __syncthreads();  // the previous expert's rows are no longer read
    for (int i = threadIdx.x; i < n * (p.I / 8); i += kThreads) {
      const int r = i / (p.I / 8), k = (i - r * (p.I / 8)) * 8;
      *reinterpret_cast<uint4*>(hs + static_cast<size_t>(r) * hstride + k) =
          nkm::ldcg128(p.hbuf + static_cast<size_t>(off + r) * p.I + k);
    }
    __syncthreads();
#pragma unroll 1
    for (int st = seg + warp; st < seg_end; st += kWarps) {
      const int s = st - j * S;
      if (lane == 0 && st + kWarps < seg_end) {  // the next strip's weights and scales into L2
        nkm::prefetch_l2_bulk(lw.w2 + e * ebytes + static_cast<size_t>(s + kWarps) * KT * 256,
                              static_cast<uint32_t>(KT) * 256u);
        nkm::prefetch_l2_bulk(lw.s2 + e * sbytes + (s + kWarps) * ssb, static_cast<uint32_t>(ssb));
      }
      float acc[kNT][4] = {};
      ft_fp4(lw.w2 + e * ebytes + static_cast<size_t>(s) * KT * 256, lw.s2 + e * sbytes + s * ssb, KT, hs, hstride,
             nullptr, n, acc);
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
}

__device__ __noinline__ void moe_residual(const Params& p, const Route* rt, int layer) {
  const int n = p.B * p.H;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
    const int b = i / p.H, r = i - b * p.H;
    float s = 0.f;
    for (int k = 0; k < p.K; ++k) s += nkm::ldcg_f(p.ypair + static_cast<size_t>(rt->pair_of[b * p.K + k]) * p.H + r);
    const float v = nkm::ldcg_f(p.resid + i) + s;
    p.resid[i] = v;
    if (p.tr_out) p.tr_out[static_cast<size_t>(layer - p.first_layer) * n + i] = v;
  }
}

// LM head: one warp per 16-row strip of the vocabulary (whole K).
__device__ __noinline__ void lm_head(const Params& p, const uint16_t* xs) {
  const int lane = lane_id(), g = lane >> 2, t4 = lane & 3;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), nw = gridDim.x * kWarps;
  const int S = p.V / 16, KT = p.H / 32;
#pragma unroll 1
  for (int s = gw; s < S; s += nw) {
    float acc[kNT][4] = {};
    ft_bf16(p.lm_head + static_cast<size_t>(s) * KT * 1024, 0, KT, xs, p.H + 8, nullptr, p.B, acc);
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int ee = 0; ee < 2; ++ee) {
        const int c = nt * 8 + 2 * t4 + ee;
        if (c < p.B) {
          p.logits_out[static_cast<size_t>(c) * p.V + 16 * s + g] = acc[nt][ee];
          p.logits_out[static_cast<size_t>(c) * p.V + 16 * s + g + 8] = acc[nt][2 + ee];
        }
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
      dense_splitk(p, lw.wqkv, p.R, p.H / 32, p.kc_qkv, xs, p.H + 8);
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
        dense_splitk(p, lw.wo, p.H, Kq / 32, p.kc_o, xs, stride);
      }
      if (!grid_sync(p, bar_k, flag)) return;
      oproj_residual(p, lw, layer);  // C2
      if (!grid_sync(p, bar_k, flag)) return;
      norm_rows(p, lw.ln2, xs, rstd, true);  // D (f16 rows stay in shared memory for stage E)
      __syncthreads();  // every row's rstd (written by its warp) before any warp scores it
      router_logits(p, lw, layer, rstd);
      if (!grid_sync(p, bar_k, flag)) return;
      routing(p, rt, layer);  // E
      expert_gateup(p, lw, rt, xs);
      if (!grid_sync(p, bar_k, flag)) return;
      expert_down(p, lw, rt, xs);  // F (the f16 rows of stage D are no longer needed)
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
      lm_head(p, xs);
    }
    __syncthreads();
    if (p.tr_stage && blockIdx.x == 0 && threadIdx.x == 0) p.tr_stage[bar_k + 1] = static_cast<int64_t>(globaltimer_ns());
  }();
  // end of the launch: the last CTA out resets the barrier counter
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = nkm::atom_acqrel_add_u32(p.bar + 2, 1u);
    if (old == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned*>(p.bar) = 0u;
      *reinterpret_cast<volatile unsigned*>(p.bar + 2) = 0u;
    }
  }
}

}  // namespace nkg
