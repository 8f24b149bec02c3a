// Qwen3 MoE block for larger batches on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// When the tokens of a step give each expert several columns (config 3: 64 tokens x top-8 over
// 128 experts, and more), the experts' projections are grouped GEMMs: tokens are bucketed per
// expert, and each (expert, 128 output rows) tile is one tcgen05.mma chain with the weights as
// the A operand (M = 128 rows, K-major, 128-byte swizzle, TMA-staged), the expert's gathered
// tokens as B (N = the expert's token count rounded up to 16), the fp32 accumulator in TMEM.
// Launches (caller's stream):
//   route    one CTA per token: RMSNorm(ln2) in the decode kernel's fixed order, fp32 router
//            logits (+ bias), top-k on the logits, softmax at the top-k and bf16 renormalisation
//            (moe_fused_nki.py:186-272, 404-418): the decode kernel's arithmetic, bit for bit
//   plan     one CTA: per-expert counts, 16-row-padded segments, pair slots in token order, tiles
//   gather   normalised bf16 rows into the expert-grouped matrix (padding rows zero)
//   gemm<1>  gate/up: an A tile = 64 gate rows + the 64 matching up rows of one expert, so the
//            epilogue forms h = bf16(bf16(SiLU(bf16 gate)) * bf16 up) (moe_fused_nki.py:506-527)
//   gemm<0>  down: A = 128 rows of W2[e], B = h; y = acc * routing weight (fp32) per pair
//   combine  out[t] = bf16(sum over the token's k slots in slot order) (+ residual)
// Warp roles of the GEMM (192 threads): warp 0 TMA producer (8-stage ring of 128-row weight tiles
// and <= 64-column token tiles), warp 1 TMEM allocation + MMA issue (one elected lane; two 64-column
// accumulators alternate so the next tile's MMAs overlap this tile's epilogue), warps 2-5 epilogue
// (warp w reads TMEM lanes 32 (w % 4) .. + 31).  With MXFP8 weights (736 threads) warp 0 streams
// the packed weight units, warps 6-21 expand them to bf16 tiles (a quarter row per thread), warp
// 22 loads the token tiles.
// Every mbarrier wait is bounded (2 s); on expiry the CTA records NKM_ERR_TIMEOUT, all roles
// leave their loops, outstanding copies and MMAs are waited for (bounded) and TMEM is freed
// before the CTA exits.  No load uses cluster multicast.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "nkimoe.h"
#include "nkm_ptx.cuh"

namespace nkm {
void set_last_error(const char* msg);
}

namespace {

using nkm::smem_addr;

constexpr int kTcThreads = 192;
constexpr int kConvWarps = 16;            // MXFP8: converter warps (thread = a quarter row of a weight unit)
constexpr int kTcThreadsMx = 192 + kConvWarps * 32 + 32;  // + converters and a B-tile producer warp
constexpr int kStages = 8;
constexpr int kStagesMx = 6;              // bf16 operand stages with MXFP8 weights
constexpr int kRawMx = 8;                 // MXFP8 weight units in flight per CTA
constexpr int kMxUnit = 128 * 64 + 128 * 2;  // 128 rows x 64 e4m3 codes, then 128 rows x 2 e8m0 scales
constexpr int kBK = 64;                   // K elements per stage (128 bytes: one swizzle atom row)
constexpr int kMaxN = 64;                 // columns of one tile (an expert with more tokens has several tiles)
constexpr int kAccCols = 64;              // TMEM columns of one accumulator; two accumulators alternate
constexpr int kABytes = 128 * 128;        // A stage: 128 rows x 128 bytes
constexpr int kBBytes = kMaxN * 128;      // B stage: up to 64 rows x 128 bytes
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kXchBytes = 64 * 16 * 4;    // gate/up epilogue exchange (64 rows x 16 columns fp32)
constexpr int kBarBytes = 512;            // mbarriers, TMEM address, abort flag
constexpr int kTcSmem = kStages * kStageBytes + kXchBytes + kBarBytes + 1024;
constexpr int kTcSmemMx = kStagesMx * kStageBytes + kRawMx * kMxUnit + kXchBytes + kBarBytes + 1024;
static_assert(kTcSmem <= 232448, "bf16 GEMM shared memory");
static_assert((3 * kStages + 2 * kRawMx + 4) * 8 + 8 <= kBarBytes, "barrier area");
static_assert(kTcSmemMx <= 232448, "MXFP8 GEMM shared memory");
static_assert(kMxUnit % 16 == 0, "bulk copy size");
constexpr int kMaxTokens = 512;
constexpr int kMaxE = 256;
constexpr int kMaxK = 8;
constexpr uint64_t kWaitNs = 2000000000ull;

struct TcParams {
  int T, H, E, K, I;
  float eps;
  int residual;
  const uint16_t* x;        // [T, H] bf16 input rows
  uint16_t* y;              // [T, H] bf16 output
  const uint16_t* ln2;
  const uint16_t* router;   // [E, H]
  const float* router_bias; // [E] or null
  int* status;
  int* topk_idx;            // [T, K]
  float* topk_w;            // [T, K]
  int* trace_idx;           // optional outputs
  float* trace_w;
  uint16_t* xn;             // [T, H] normalised rows (bf16)
  int* pair_slot;           // [T * K] slot of (token, k)
  int* slot_tok;            // [P] token of a slot (-1: padding)
  float* slot_w;            // [P] routing weight of a slot
  int* tiles;               // [max tiles][3]: expert, first slot, columns (multiple of 16)
  int* ntiles;              // [1]
  uint16_t* xg;             // [P, H] expert-grouped rows
  uint16_t* hbuf;           // [P, I]
  float* ypair;             // [P, H]
  int P;                    // slot capacity
  const uint8_t* w13mx;     // MXFP8 weights (nkm_pack_mxfp8_experts units) or null
  const uint8_t* w2mx;
  int e_lo, e_hi;           // experts whose weights this call holds (expert parallel: a range)
  float* y_part;            // fp32 [T, H] sum of the local experts' contributions (expert parallel), or null
};

// ------------------------------------------------------------------ PTX (tcgen05, TMEM)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// K-major operand tile with 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart):
// start address, leading offset 16 bytes (unused by swizzled K-major layouts), stride offset 1024
// bytes, descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t a = (smem_addr(tile) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, M x N.
__device__ __forceinline__ uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Bounded wait; false (and NKM_ERR_TIMEOUT recorded, abort raised) if it ran out or another
// role aborted.
__device__ __noinline__ bool wait_bar(uint64_t* bar, uint32_t par, const TcParams& p, volatile int* abort_flag) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (nkm::mbar_try_wait(bar, par)) return true;
    if ((it & 255u) == 255u) {
      if (*abort_flag) return false;
      const uint64_t now = nkm::globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitNs) {
        atomicOr(p.status, NKM_ERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ route / plan / gather / combine
__device__ __forceinline__ float warp_sum_fixed(float s) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}
__device__ __forceinline__ float rbf(float f) { return nkm::rbf(f); }

__global__ void __launch_bounds__(256) tc_route_kernel(TcParams p) {
  extern __shared__ float xs32[];  // [H] normalised row
  __shared__ float logits[kMaxE];
  __shared__ float rsh;
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint16_t* xr = p.x + static_cast<size_t>(t) * p.H;
  if (warp == 0) {
    float s = 0.f;
    for (int i = 0; i * 256 < p.H; ++i) {
      const uint4 q = *reinterpret_cast<const uint4*>(xr + 256 * i + 8 * lane);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = (j & 1) ? nkm::hi_bf(w[j >> 1]) : nkm::lo_bf(w[j >> 1]);
        s = __fadd_rn(s, __fmul_rn(v, v));
      }
    }
    s = warp_sum_fixed(s);
    if (lane == 0) {
      const float v = __fadd_rn(__fmul_rn(s, 1.0f / static_cast<float>(p.H)), p.eps);
      rsh = __fdiv_rn(1.0f, __fsqrt_rn(v));
    }
  }
  __syncthreads();
  const float r = rsh;
  for (int k = threadIdx.x; k < p.H; k += 256) {
    const float v = __fmul_rn(__fmul_rn(nkm::bf2f(xr[k]), nkm::bf2f(p.ln2[k])), r);  // (x * g) * r
    xs32[k] = v;
    p.xn[static_cast<size_t>(t) * p.H + k] = nkm::f2bf(v);
  }
  __syncthreads();
  for (int e = warp; e < p.E; e += 8) {
    const uint16_t* wr = p.router + static_cast<size_t>(e) * p.H;
    float acc = 0.f;
    // the row's loads are issued 8 groups at a time, then summed in k order
    for (int i0 = 0; i0 * 256 < p.H; i0 += 8) {
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if ((i0 + u) * 256 < p.H) q[u] = nkm::ldnc128(wr + 256 * (i0 + u) + 8 * lane);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if ((i0 + u) * 256 < p.H) {
          const int k = 256 * (i0 + u) + 8 * lane;
          const float4 a = *reinterpret_cast<const float4*>(xs32 + k), b = *reinterpret_cast<const float4*>(xs32 + k + 4);
          const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
          const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int j = 0; j < 8; ++j)
            acc = __fadd_rn(acc, __fmul_rn((j & 1) ? nkm::hi_bf(w[j >> 1]) : nkm::lo_bf(w[j >> 1]), xv[j]));
        }
      }
    }
    acc = warp_sum_fixed(acc);
    if (p.router_bias) acc = __fadd_rn(acc, p.router_bias[e]);
    if (lane == 0) logits[e] = acc;
  }
  __syncthreads();
  if (warp != 0) return;
  // top-k on the logits (ties: lower expert), softmax over all logits at the picks, bf16 renorm
  float v[kMaxE / 32];
  const int per = (p.E + 31) / 32;
#pragma unroll
  for (int q = 0; q < kMaxE / 32; ++q) v[q] = (q < per && 32 * q + lane < p.E) ? logits[32 * q + lane] : -INFINITY;
  float mx = -INFINITY, myl = -INFINITY;
  int myi = 0;
  for (int k = 0; k < p.K; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < kMaxE / 32; ++q) {
      const int e = 32 * q + lane;
      if (e < p.E && (v[q] > bv || (v[q] == bv && e < bi))) {
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
    if (k == 0) mx = bv;
    if (lane == k) {
      myl = bv;
      myi = bi;
    }
#pragma unroll
    for (int q = 0; q < kMaxE / 32; ++q)
      if (32 * q + lane == bi) v[q] = -INFINITY;
  }
  float se = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxE / 32; ++q) {
    const int e = 32 * q + lane;
    se += (q < per && e < p.E) ? __expf(logits[e] - mx) : 0.f;
  }
  se = warp_sum_fixed(se);
  const float inv = 1.f / se;
  const float myval = lane < p.K ? rbf(__expf(myl - mx) * inv) : 0.f;
  float sk = 0.f;
  for (int k = 0; k < p.K; ++k) sk += __shfl_sync(0xffffffffu, myval, k);
  const float inv2 = 1.f / sk;
  if (lane < p.K) {
    const float w = rbf(myval * inv2);
    p.topk_idx[t * p.K + lane] = myi;
    p.topk_w[t * p.K + lane] = w;
    if (p.trace_idx) p.trace_idx[t * p.K + lane] = myi;
    if (p.trace_w) p.trace_w[t * p.K + lane] = w;
  }
}

__global__ void __launch_bounds__(256) tc_plan_kernel(TcParams p) {
  __shared__ int cnt[kMaxE], seg[kMaxE];
  __shared__ int pidx[kMaxTokens * kMaxK];  // the pairs' experts, in pair order
  for (int e = threadIdx.x; e < p.E; e += 256) cnt[e] = 0;
  const int NP = p.T * p.K;
  for (int i = threadIdx.x; i < NP; i += 256) pidx[i] = p.topk_idx[i];
  __syncthreads();
  for (int i = threadIdx.x; i < NP; i += 256) atomicAdd(&cnt[pidx[i]], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0, nt = 0;
    for (int e = 0; e < p.E; ++e) {
      seg[e] = off;
      const int n = (e >= p.e_lo && e < p.e_hi) ? cnt[e] : 0;  // other ranks' experts: no tiles
      for (int c0 = 0; c0 < n; c0 += kMaxN) {
        const int nc = min(kMaxN, n - c0);
        p.tiles[3 * nt] = e;
        p.tiles[3 * nt + 1] = off + c0;
        p.tiles[3 * nt + 2] = (nc + 15) & ~15;
        ++nt;
      }
      off += (n + 15) & ~15;
    }
    *p.ntiles = nt;
  }
  __syncthreads();
  // slots: padding first (every slot of the capacity), then the pairs in token order per expert
  for (int s = threadIdx.x; s < p.P; s += 256) {
    p.slot_tok[s] = -1;
    p.slot_w[s] = 0.f;
  }
  __syncthreads();
  // warp w places the pairs of experts w, w + 8, ... in pair (token) order: 32 pairs per ballot,
  // a pair's rank among its expert's pairs = the matches before it
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = warp; e < p.E; e += 8) {
    const bool local = e >= p.e_lo && e < p.e_hi;
    int s = seg[e];
    for (int i0 = 0; i0 < NP; i0 += 32) {
      const int i = i0 + lane;
      const bool hit = i < NP && pidx[i] == e;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (hit) {
        const int sl = s + __popc(m & ((1u << lane) - 1u));
        p.pair_slot[i] = local ? sl : -1;  // -1: the pair's expert lives on another rank
        if (local) {
          p.slot_tok[sl] = i / p.K;
          p.slot_w[sl] = p.topk_w[i];
        }
      }
      s += __popc(m);
    }
  }
}

__global__ void tc_gather_kernel(TcParams p) {
  const int s = blockIdx.x;
  const int t = p.slot_tok[s];
  uint4* dst = reinterpret_cast<uint4*>(p.xg + static_cast<size_t>(s) * p.H);
  const uint4* src = t >= 0 ? reinterpret_cast<const uint4*>(p.xn + static_cast<size_t>(t) * p.H) : nullptr;
  for (int i = threadIdx.x; i < p.H / 8; i += blockDim.x) dst[i] = src ? src[i] : make_uint4(0u, 0u, 0u, 0u);
}

__global__ void tc_combine_kernel(TcParams p) {
  const int t = blockIdx.x;
  for (int h = threadIdx.x; h < p.H; h += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < p.K; ++k) {
      const int sl = p.pair_slot[t * p.K + k];
      if (sl >= 0) s += p.ypair[static_cast<size_t>(sl) * p.H + h];
    }
    if (p.y_part) {  // expert parallel: this rank's experts only, summed over the ranks later
      p.y_part[static_cast<size_t>(t) * p.H + h] = s;
      continue;
    }
    const float base = p.residual ? nkm::bf2f(p.x[static_cast<size_t>(t) * p.H + h]) : 0.f;
    p.y[static_cast<size_t>(t) * p.H + h] = nkm::f2bf(base + rbf(s));
  }
}

// ------------------------------------------------------------------ MXFP8 weights
// e8m0 scale byte -> fp32 2^(s - 127) (0 -> 2^-127, 255 -> NaN)
__device__ __forceinline__ float e8m0_f32(uint32_t s) {
  return s == 0u ? __uint_as_float(0x00400000u) : (s == 255u ? __uint_as_float(0x7fc00000u) : __uint_as_float(s << 23));
}
// two e4m3 codes (low byte -> low half) to f16x2 (exact)
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v16) {
  uint32_t d;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(d) : "r"(v16));
  return d;
}
// 4 e4m3 codes times a power-of-two scale -> two bf16x2 words (exact: bf16 has fp32's exponent range)
__device__ __forceinline__ uint2 e4m3x4_bf16(uint32_t w, float sc) {
  const uint32_t lo = e4m3x2_f16x2(w & 0xffffu), hi = e4m3x2_f16x2(w >> 16);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  return make_uint2(nkm::pack_bf2(a.x * sc, a.y * sc), nkm::pack_bf2(b.x * sc, b.y * sc));
}
// Two e4m3 codes with non-zero exponent fields, spread one per 16-bit half (code in the low byte),
// times 2^(s-127), as bf16x2 bits by integer arithmetic: e4m3 s.eeee.mmm is 2^(e-7) (1 + m/8), so
// the bf16 fields are the sign, exponent e + 120 + (s - 127) and mantissa m << 4.  e2 holds
// (120 + s - 127) << 7 in both halves; valid for 7 <= s <= 246 (the exponent stays in 1..254).
__device__ __forceinline__ uint32_t e4m3x2_bf16x2_int(uint32_t x, uint32_t e2) {
  return (x & 0x00800080u) * 256u + (x & 0x007f007fu) * 16u + e2;
}
// 16 codes (one 16-byte load) times 2^(s-127) to 8 bf16x2 words.  Codes whose exponent field is
// zero (zero, subnormal), NaN codes, or a scale outside 7..246 take the conversion instructions.
__device__ __forceinline__ void e4m3x16_bf16(const uint4 c, uint32_t s, float sc, uint32_t (&o)[8]) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
  uint32_t zero_exp = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    zero_exp |= __vcmpeq4(w[i] & 0x78787878u, 0u) | __vcmpeq4(w[i] & 0x7f7f7f7fu, 0x7f7f7f7fu);  // + NaN codes
  if (zero_exp == 0u && s >= 7u && s <= 246u) {
    const uint32_t e = s - 7u;  // 120 + s - 127
    const uint32_t e2 = (e << 7) | (e << 23);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = e4m3x2_bf16x2_int(__byte_perm(w[i], 0u, 0x4140), e2);
      o[2 * i + 1] = e4m3x2_bf16x2_int(__byte_perm(w[i], 0u, 0x4342), e2);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint2 b = e4m3x4_bf16(w[i], sc);
      o[2 * i] = b.x;
      o[2 * i + 1] = b.y;
    }
  }
}
// Quarter q (16 codes) of row `row` of an MXFP8 unit (128 rows x 64 codes, then 128 rows x 2
// scales) into the bf16 K-major tile with the 128-byte swizzle the MMA descriptor expects (16-byte
// chunk c of row r at c ^ (r % 8)).  Consecutive threads take consecutive quarters: the loads and
// the stores of a quarter-warp hit distinct banks.
__device__ __forceinline__ void mx_convert_quarter(const uint8_t* unit, uint8_t* a_tile, int row, int q) {
  const uint4 src = *reinterpret_cast<const uint4*>(unit + row * 64 + q * 16);
  const uint32_t s = unit[128 * 64 + row * 2 + (q >> 1)];
  uint32_t o[8];
  e4m3x16_bf16(src, s, e8m0_f32(s), o);
  uint8_t* dst = a_tile + row * 128;
  const int c0 = 2 * q, c1 = 2 * q + 1;
  *reinterpret_cast<uint4*>(dst + ((c0 ^ (row & 7)) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(dst + ((c1 ^ (row & 7)) * 16)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// ------------------------------------------------------------------ the grouped GEMM
// kGateUp: item = (tile, 64-row block j0 of I): A = gate rows [e*2I + j0, +64) and up rows
// [e*2I + I + j0, +64) of W13, K = H; out h[slot][j0 + r].
// !kGateUp: item = (tile, 128-row block m0 of H): A = W2 rows [e*H + m0, +128), K = I;
// out ypair[slot][m0 + r] = acc * slot_w[slot].
// kMx (MXFP8 weights): the A operand arrives as nkm_pack_mxfp8_experts units (e4m3 codes + e8m0
// scales of the same 128 rows, one 1-D bulk copy each, kRawMx in flight) and warps 6-21 expand
// each unit into the bf16 swizzled A tile (exact: code x power of two); the MMA then runs as for
// bf16 weights.  Warp 22 issues the B (token) tiles of each stage.  Two TMEM accumulators
// alternate, so the MMAs of a tile run while the epilogue reads the previous one.
template <bool kGateUp, bool kMx>
__global__ void __launch_bounds__(kMx ? kTcThreadsMx : kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, TcParams p) {
  constexpr int S = kMx ? kStagesMx : kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint8_t* raw_base = smem + S * kStageBytes;  // kMx: weight units
  float* xch = reinterpret_cast<float*>(raw_base + (kMx ? kRawMx * kMxUnit : 0));
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xch) + kXchBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;       // [2]: accumulator b written
  uint64_t* acc_empty = acc_full + 2;   // [2]: accumulator b read by the epilogue
  uint64_t* bfull = acc_empty + 2;      // kMx: B tiles of a stage landed (S)
  uint64_t* raw_full = bfull + S;       // kMx: weight unit landed (kRawMx)
  uint64_t* raw_empty = raw_full + kRawMx;  // kMx: weight unit converted (kRawMx)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(raw_empty + kRawMx);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = kGateUp ? p.H / kBK : p.I / kBK;      // K chunks
  const int MB = kGateUp ? p.I / 64 : p.H / 128;       // row blocks per tile
  const int nitems = *p.ntiles * MB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      nkm::mbar_init(&full[s], kMx ? kConvWarps : 1);  // kMx: one arrival per converter warp
      nkm::mbar_init(&empty[s], 1);
      nkm::mbar_init(&bfull[s], 1);
    }
    for (int r = 0; r < kRawMx; ++r) {
      nkm::mbar_init(&raw_full[r], 1);
      nkm::mbar_init(&raw_empty[r], kConvWarps);
    }
    for (int b = 0; b < 2; ++b) {
      nkm::mbar_init(&acc_full[b], 1);
      nkm::mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    nkm::fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 2 * kAccCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------- TMA producer (kMx: weight units only)
    if (lane == 0) {
      if (!kMx) nkm::prefetch_tensormap(&amap);
      nkm::prefetch_tensormap(&bmap);
      uint32_t cnt = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        const int tile = item / MB, mb = item - tile * MB;
        const int e = p.tiles[3 * tile], n0 = p.tiles[3 * tile + 1], ncols = p.tiles[3 * tile + 2];
        for (int kc = 0; kc < KT; ++kc, ++cnt) {
          if (kMx) {
            const int r = cnt % kRawMx;
            if (!wait_bar(&raw_empty[r], ((cnt / kRawMx) & 1u) ^ 1u, p, abort_flag)) {
              ok = false;
              break;
            }
            const size_t el = static_cast<size_t>(e - p.e_lo);  // local expert
            const uint8_t* src = kGateUp ? p.w13mx + ((el * MB + mb) * KT + kc) * kMxUnit
                                         : p.w2mx + ((el * MB + mb) * KT + kc) * kMxUnit;
            nkm::mbar_arrive_expect_tx(&raw_full[r], kMxUnit);
            nkm::bulk_g2s_plain(raw_base + r * kMxUnit, src, kMxUnit, &raw_full[r]);
            continue;
          }
          const int s = cnt % S;
          if (!wait_bar(&empty[s], ((cnt / S) & 1u) ^ 1u, p, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* a = stage_base + s * kStageBytes;
          uint8_t* b = a + kABytes;
          const uint32_t bytes = kABytes + static_cast<uint32_t>(ncols) * 128u;
          nkm::mbar_arrive_expect_tx(&full[s], bytes);
          if (kGateUp) {
            nkm::tma_load_2d(a, &amap, kc * kBK, (e - p.e_lo) * 2 * p.I + mb * 64, &full[s]);
            nkm::tma_load_2d(a + 64 * 128, &amap, kc * kBK, (e - p.e_lo) * 2 * p.I + p.I + mb * 64, &full[s]);
          } else {
            nkm::tma_load_2d(a, &amap, kc * kBK, (e - p.e_lo) * p.H + mb * 128, &full[s]);
            nkm::tma_load_2d(a + 64 * 128, &amap, kc * kBK, (e - p.e_lo) * p.H + mb * 128 + 64, &full[s]);
          }
          for (int r = 0; r < ncols; r += 16) nkm::tma_load_2d(b + r * 128, &bmap, kc * kBK, n0 + r, &full[s]);
        }
      }
      if (!ok) {  // copies still in flight land before the CTA leaves (bounded)
        const uint64_t t0 = nkm::globaltimer_ns();
        const uint32_t depth = kMx ? kRawMx : S;
        for (uint32_t c = (cnt >= depth ? cnt - depth : 0); c < cnt; ++c) {
          uint64_t* bar = kMx ? &raw_full[c % kRawMx] : &full[c % S];
          while (!nkm::mbar_try_wait(bar, (c / depth) & 1u) && nkm::globaltimer_ns() - t0 < 1000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      uint32_t cnt = 0, acc_round = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++acc_round) {
        const int tile = item / MB;
        const int ncols = p.tiles[3 * tile + 2];
        const uint32_t idesc = idesc_bf16(128, ncols);
        const uint32_t ab = acc_round & 1u, d_tmem = tmem + ab * kAccCols;
        // the epilogue has read this accumulator's previous tile (two tiles back)
        if (!wait_bar(&acc_empty[ab], ((acc_round >> 1) & 1u) ^ 1u, p, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < KT; ++kc, ++cnt) {
          const int s = cnt % S;
          if (!wait_bar(&full[s], (cnt / S) & 1u, p, abort_flag) ||
              (kMx && !wait_bar(&bfull[s], (cnt / S) & 1u, p, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* a = stage_base + s * kStageBytes;
          const uint8_t* b = a + kABytes;
          const uint64_t ad = sw128_desc(a), bd = sw128_desc(b);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)  // 16 bf16 = 32 bytes per MMA: start address + 2
            tc_mma(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kc | kk) != 0);
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(&acc_full[ab]);
      }
      // every MMA issued has completed before TMEM is released (bounded)
      if (cnt > 0) {
        const uint32_t last = cnt - 1;
        const uint64_t t0 = nkm::globaltimer_ns();
        while (!nkm::mbar_try_wait(&empty[last % S], (last / S) & 1u) &&
               nkm::globaltimer_ns() - t0 < 2000000000ull) {
        }
      }
    }
  } else if (warp < 6) {
    // ---------------- epilogue (warps 2..5; TMEM lanes 32 (warp % 4) .. + 31)
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    uint32_t acc_round = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++acc_round) {
      const uint32_t ab = acc_round & 1u;
      if (!wait_bar(&acc_full[ab], (acc_round >> 1) & 1u, p, abort_flag)) break;
      tc_fence_after();
      const int tile = item / MB, mb = item - tile * MB;
      const int n0 = p.tiles[3 * tile + 1], ncols = p.tiles[3 * tile + 2];
      const int row = 32 * q + lane;  // accumulator row of this thread
      for (int c0 = 0; c0 < ncols; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + lane_base + ab * kAccCols + static_cast<uint32_t>(c0), v);
        if (kGateUp) {
          // rows 0-63: gate j = row; rows 64-127: up j = row - 64 (exchange through shared memory)
          if (row >= 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xch[(row - 64) * 16 + i] = v[i];
          }
          named_sync(1, 128);
          if (row < 64) {
            const int j = mb * 64 + row;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int s = n0 + c0 + i;
              if (p.slot_tok[s] >= 0) {
                const float g = rbf(v[i]), u = rbf(xch[row * 16 + i]);
                const float sl = rbf(__fdividef(g, 1.0f + __expf(-g)));
                p.hbuf[static_cast<size_t>(s) * p.I + j] = nkm::f2bf(rbf(sl * u));
              }
            }
          }
          named_sync(1, 128);
        } else {
          const int m = mb * 128 + row;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int s = n0 + c0 + i;
            if (p.slot_tok[s] >= 0) p.ypair[static_cast<size_t>(s) * p.H + m] = v[i] * p.slot_w[s];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) nkm::mbar_arrive(&acc_empty[ab]);
    }
  } else if (kMx && warp < 6 + kConvWarps) {
    // ---------------- MXFP8 converters (warps 6..21: thread t expands quarter t % 4 of row t / 4)
    const int t = threadIdx.x - 192;
    uint32_t cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
      for (int kc = 0; kc < KT; ++kc, ++cnt) {
        const int s = cnt % S, r = cnt % kRawMx;
        // the stage's previous MMAs are done (its A area is free)
        if (!wait_bar(&empty[s], ((cnt / S) & 1u) ^ 1u, p, abort_flag) ||
            !wait_bar(&raw_full[r], (cnt / kRawMx) & 1u, p, abort_flag)) {
          ok = false;
          break;
        }
        mx_convert_quarter(raw_base + r * kMxUnit, stage_base + s * kStageBytes, t >> 2, t & 3);
        nkm::fence_proxy_async_smem();  // generic writes of the A tile before the MMA reads it
        __syncwarp();
        if (lane == 0) {
          nkm::mbar_arrive(&raw_empty[r]);
          nkm::mbar_arrive(&full[s]);
        }
      }
    }
  } else if (kMx) {
    // ---------------- B-tile producer (warp 6 + kConvWarps): the expert's token tiles of each stage
    if (lane == 0) {
      uint32_t cnt = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        const int tile = item / MB;
        const int n0 = p.tiles[3 * tile + 1], ncols = p.tiles[3 * tile + 2];
        for (int kc = 0; kc < KT; ++kc, ++cnt) {
          const int s = cnt % S;
          if (!wait_bar(&empty[s], ((cnt / S) & 1u) ^ 1u, p, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* b = stage_base + s * kStageBytes + kABytes;
          nkm::mbar_arrive_expect_tx(&bfull[s], static_cast<uint32_t>(ncols) * 128u);
          for (int rr = 0; rr < ncols; rr += 16) nkm::tma_load_2d(b + rr * 128, &bmap, kc * kBK, n0 + rr, &bfull[s]);
        }
      }
      if (!ok) {  // B tiles still in flight land before the CTA leaves (bounded)
        const uint64_t t0 = nkm::globaltimer_ns();
        for (uint32_t c = (cnt >= static_cast<uint32_t>(S) ? cnt - S : 0); c < cnt; ++c)
          while (!nkm::mbar_try_wait(&bfull[c % S], (c / S) & 1u) && nkm::globaltimer_ns() - t0 < 1000000ull) {
          }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 2 * kAccCols);
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// bf16 [rows, cols] row-major, box 64 columns x box_rows rows, 128-byte swizzle, zero fill
int encode(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto enc = encoder();
  if (!enc) {
    nkm::set_last_error("cuTensorMapEncodeTiled unavailable");
    return NKM_ERR_CUDA;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  if (enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    nkm::set_last_error("cuTensorMapEncodeTiled failed");
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}

struct TcLayout {
  size_t status, ntiles, topk_idx, topk_w, xn, pair_slot, slot_tok, slot_w, tiles, xg, hbuf, ypair, total;
  int P, max_tiles;
};

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

TcLayout tc_layout(const nkm_moe_tc_desc& d) {
  TcLayout w{};
  const size_t T = d.max_tokens, K = d.top_k, H = d.hidden, I = d.moe_inter, E = d.n_experts;
  w.P = static_cast<int>(((T * K + 15 * E) + 15) & ~size_t(15));
  w.max_tiles = static_cast<int>(E + (T * K) / kMaxN + 1);
  size_t o = 0;
  w.status = o;
  w.ntiles = o + 4;
  o = 256;
  w.topk_idx = o;
  o = al(o + T * K * 4);
  w.topk_w = o;
  o = al(o + T * K * 4);
  w.xn = o;
  o = al(o + T * H * 2);
  w.pair_slot = o;
  o = al(o + T * K * 4);
  w.slot_tok = o;
  o = al(o + w.P * 4);
  w.slot_w = o;
  o = al(o + w.P * 4);
  w.tiles = o;
  o = al(o + static_cast<size_t>(w.max_tiles) * 12);
  w.xg = o;
  o = al(o + static_cast<size_t>(w.P) * H * 2);
  w.hbuf = o;
  o = al(o + static_cast<size_t>(w.P) * I * 2);
  w.ypair = o;
  o = al(o + static_cast<size_t>(w.P) * H * 4);
  w.total = o;
  return w;
}

int tc_check(const nkm_moe_tc_desc* d) {
  if (!d) return NKM_ERR_ARG;
  if (d->hidden <= 0 || d->hidden % 256 || d->hidden > 8192) return NKM_ERR_ARG;
  if (d->moe_inter <= 0 || d->moe_inter % 64) return NKM_ERR_ARG;
  if (d->n_experts <= 0 || d->n_experts > kMaxE || d->top_k <= 0 || d->top_k > kMaxK || d->top_k > d->n_experts)
    return NKM_ERR_ARG;
  if (d->max_tokens <= 0 || d->max_tokens > kMaxTokens) return NKM_ERR_ARG;
  if (!d->ln2 || !d->router || !d->w13 || !d->w2) return NKM_ERR_ARG;
  if (d->weight_format != NKM_MOE_WEIGHTS_BF16 && d->weight_format != NKM_MOE_WEIGHTS_MXFP8) return NKM_ERR_ARG;
  const int nl = d->n_local_experts > 0 ? d->n_local_experts : d->n_experts;
  if (d->expert_begin < 0 || d->expert_begin + nl > d->n_experts) return NKM_ERR_ARG;
  return NKM_OK;
}

// MXFP8 expert weights, HF-style codes [count][rows][cols] (e4m3) and scales [count][rows][cols/32]
// (e8m0), into the units the MXFP8 GEMM streams: unit (c, mb, kc) = 128 rows x 64 codes of
// columns [64 kc, +64) then the rows' 2 scales.  gate_up (rows = 2I): unit rows 0-63 are gate rows
// [64 mb, +64), rows 64-127 the up rows [I + 64 mb, +64); otherwise unit rows are [128 mb, +128).
__global__ void pack_mxfp8_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                  uint8_t* __restrict__ dst, int64_t count, int64_t rows, int64_t cols, int gate_up) {
  const int64_t KT = cols / 64, MB = gate_up ? rows / 128 : rows / 128, half = rows / 2;
  const int64_t nunits = count * MB * KT;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nunits * kMxUnit;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t u = i / kMxUnit, off = i % kMxUnit;
    const int64_t c = u / (MB * KT), rem = u % (MB * KT), mb = rem / KT, kc = rem % KT;
    const int64_t r = off < 128 * 64 ? off / 64 : (off - 128 * 64) / 2;
    const int64_t src_row = gate_up ? (r < 64 ? 64 * mb + r : half + 64 * mb + (r - 64)) : 128 * mb + r;
    if (off < 128 * 64)
      dst[i] = codes[(c * rows + src_row) * cols + 64 * kc + off % 64];
    else
      dst[i] = scales[(c * rows + src_row) * (cols / 32) + 2 * kc + (off - 128 * 64) % 2];
  }
}

}  // namespace

extern "C" size_t nkm_moe_tc_workspace_bytes(const nkm_moe_tc_desc* desc) {
  if (tc_check(desc) != NKM_OK) return 0;
  return tc_layout(*desc).total;
}

namespace {
int moe_block_tc(const nkm_moe_tc_desc* d, int32_t tokens, const void* x_in, void* y_out, float* y_part,
                 int32_t residual, int32_t* topk_idx_out, float* topk_w_out, void* workspace, size_t workspace_bytes,
                 nkm_stream_t stream_) {
  if (tc_check(d) != NKM_OK) {
    nkm::set_last_error("invalid MoE description: hidden % 256, moe_inter % 64, experts <= 256, top_k <= 8, "
                        "max_tokens <= 512, the local expert range inside the experts and every weight pointer are "
                        "required");
    return NKM_ERR_ARG;
  }
  if (tokens <= 0 || tokens > d->max_tokens) {
    nkm::set_last_error("tokens outside 1..max_tokens");
    return NKM_ERR_ARG;
  }
  void* out = y_part ? static_cast<void*>(y_part) : y_out;
  if (!x_in || !out || (reinterpret_cast<uintptr_t>(x_in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) {
    nkm::set_last_error("x_in and the output must be 16-byte aligned device pointers");
    return NKM_ERR_ARG;
  }
  const TcLayout lay = tc_layout(*d);
  if (!workspace || workspace_bytes < lay.total || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    nkm::set_last_error("workspace missing, too small (nkm_moe_tc_workspace_bytes) or not 256-byte aligned");
    return NKM_ERR_ARG;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  TcParams p{};
  p.T = tokens;
  p.H = d->hidden;
  p.E = d->n_experts;
  p.K = d->top_k;
  p.I = d->moe_inter;
  p.eps = d->rms_eps;
  p.residual = residual ? 1 : 0;
  p.x = static_cast<const uint16_t*>(x_in);
  p.y = static_cast<uint16_t*>(y_out);
  p.ln2 = static_cast<const uint16_t*>(d->ln2);
  p.router = static_cast<const uint16_t*>(d->router);
  p.router_bias = d->router_bias;
  p.status = reinterpret_cast<int*>(ws + lay.status);
  p.ntiles = reinterpret_cast<int*>(ws + lay.ntiles);
  p.topk_idx = reinterpret_cast<int*>(ws + lay.topk_idx);
  p.topk_w = reinterpret_cast<float*>(ws + lay.topk_w);
  p.trace_idx = topk_idx_out;
  p.trace_w = topk_w_out;
  p.xn = reinterpret_cast<uint16_t*>(ws + lay.xn);
  p.pair_slot = reinterpret_cast<int*>(ws + lay.pair_slot);
  p.slot_tok = reinterpret_cast<int*>(ws + lay.slot_tok);
  p.slot_w = reinterpret_cast<float*>(ws + lay.slot_w);
  p.tiles = reinterpret_cast<int*>(ws + lay.tiles);
  p.xg = reinterpret_cast<uint16_t*>(ws + lay.xg);
  p.hbuf = reinterpret_cast<uint16_t*>(ws + lay.hbuf);
  p.ypair = reinterpret_cast<float*>(ws + lay.ypair);
  p.P = lay.P;
  const bool mx = d->weight_format == NKM_MOE_WEIGHTS_MXFP8;
  p.w13mx = mx ? static_cast<const uint8_t*>(d->w13) : nullptr;
  p.w2mx = mx ? static_cast<const uint8_t*>(d->w2) : nullptr;
  const int n_local = d->n_local_experts > 0 ? d->n_local_experts : d->n_experts;
  p.e_lo = d->expert_begin;
  p.e_hi = d->expert_begin + n_local;
  p.y_part = y_part;
  CUtensorMap w13m, w2m, xgm, hm;
  memset(&w13m, 0, sizeof(w13m));
  memset(&w2m, 0, sizeof(w2m));
  int rc;
  if ((!mx && ((rc = encode(&w13m, d->w13, static_cast<uint64_t>(n_local) * 2 * p.I, p.H, 64)) ||
               (rc = encode(&w2m, d->w2, static_cast<uint64_t>(n_local) * p.H, p.I, 64)))) ||
      (rc = encode(&xgm, p.xg, lay.P, p.H, 16)) || (rc = encode(&hm, p.hbuf, lay.P, p.I, 16)))
    return rc;
  if (mx && ((reinterpret_cast<uintptr_t>(d->w13) & 15) || (reinterpret_cast<uintptr_t>(d->w2) & 15))) {
    nkm::set_last_error("MXFP8 weight units must be 16-byte aligned");
    return NKM_ERR_ARG;
  }
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_gemm_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_gemm_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemMx) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_gemm_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemMx) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8192 * 4) != cudaSuccess) {
      nkm::set_last_error("cudaFuncSetAttribute failed");
      return NKM_ERR_CUDA;
    }
    attr_set = true;
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  cudaMemsetAsync(ws, 0, 256, stream);
  tc_route_kernel<<<tokens, 256, p.H * 4, stream>>>(p);
  tc_plan_kernel<<<1, 256, 0, stream>>>(p);
  tc_gather_kernel<<<lay.P, 128, 0, stream>>>(p);
  if (mx) {
    tc_gemm_kernel<true, true><<<sms, kTcThreadsMx, kTcSmemMx, stream>>>(w13m, xgm, p);
    tc_gemm_kernel<false, true><<<sms, kTcThreadsMx, kTcSmemMx, stream>>>(w2m, hm, p);
  } else {
    tc_gemm_kernel<true, false><<<sms, kTcThreads, kTcSmem, stream>>>(w13m, xgm, p);
    tc_gemm_kernel<false, false><<<sms, kTcThreads, kTcSmem, stream>>>(w2m, hm, p);
  }
  tc_combine_kernel<<<tokens, 256, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}
}  // namespace

extern "C" int nkm_moe_block_tc(const nkm_moe_tc_desc* d, int32_t tokens, const void* x_in, void* y_out,
                                int32_t residual, int32_t* topk_idx_out, float* topk_w_out, void* workspace,
                                size_t workspace_bytes, nkm_stream_t stream) {
  return moe_block_tc(d, tokens, x_in, y_out, nullptr, residual, topk_idx_out, topk_w_out, workspace, workspace_bytes,
                      stream);
}

extern "C" int nkm_moe_block_tc_partial(const nkm_moe_tc_desc* d, int32_t tokens, const void* x_in, float* y_part,
                                        int32_t* topk_idx_out, float* topk_w_out, void* workspace,
                                        size_t workspace_bytes, nkm_stream_t stream) {
  return moe_block_tc(d, tokens, x_in, nullptr, y_part, 0, topk_idx_out, topk_w_out, workspace, workspace_bytes,
                      stream);
}

extern "C" int nkm_moe_tc_status(void* workspace, nkm_stream_t stream) {
  if (!workspace) return NKM_ERR_ARG;
  int st = 0;
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess ||
      cudaMemcpy(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return NKM_ERR_CUDA;
  return st;
}

extern "C" size_t nkm_mxfp8_experts_bytes(int32_t count, int32_t rows, int32_t cols) {
  if (count <= 0 || rows <= 0 || cols <= 0 || rows % 128 || cols % 64) return 0;
  return static_cast<size_t>(count) * (rows / 128) * (cols / 64) * kMxUnit;
}

extern "C" int nkm_pack_mxfp8_experts(const void* codes, const void* scales, void* dst, int32_t count, int32_t rows,
                                      int32_t cols, int32_t gate_up, nkm_stream_t stream) {
  if (!codes || !scales || !dst || nkm_mxfp8_experts_bytes(count, rows, cols) == 0 ||
      (reinterpret_cast<uintptr_t>(dst) & 15)) {
    nkm::set_last_error("nkm_pack_mxfp8_experts: rows % 128, cols % 64, 16-byte aligned destination required");
    return NKM_ERR_ARG;
  }
  const int64_t n = static_cast<int64_t>(nkm_mxfp8_experts_bytes(count, rows, cols));
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 65535));
  pack_mxfp8_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(codes), static_cast<const uint8_t*>(scales), static_cast<uint8_t*>(dst), count, rows,
      cols, gate_up ? 1 : 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}
