// On-device sampling of the next token from the LM-head logits (C ABI in include/nkimoe.h).
//
// Two launches on the caller's stream:
//   1. candidates: grid (slices, rows).  Each CTA copies one slice of a row's logits into shared
//      memory as order-preserving keys and selects the slice's K largest entries by an exact
//      radix select over 64-bit composite keys (logit key << 32 | ~index): the composites are
//      distinct, so "the K largest" is unique and ties between equal logits go to the lower
//      vocabulary index.  The K composites go to the scratch buffer.
//   2. pick: one CTA per row selects the K largest of the slices' candidates the same way, sorts
//      them, and one thread applies temperature, softmax over the K, the top-p prefix and an
//      inverse-CDF draw with a counter-based uniform (SplitMix64 of seed, row and position).
// Every array access is bounds-checked on the host (sizes) and by the loop bounds; no wait.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "nkimoe.h"

namespace nkm {
void set_last_error(const char* msg);  // the message nkm_last_error returns (nkm_qwen3.cu)
}

namespace {

constexpr int kThreads = 256;
constexpr int kMaxTopK = 64;
constexpr int kMaxSlices = 64;
constexpr int kSliceSmemBytes = 40960;  // keys of one slice (fp32 logits as 32-bit keys)

// Larger float -> larger key; -0 and +0 map to one key.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f == 0.f ? 0.f : f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ uint64_t composite(uint32_t key, uint32_t idx) {
  return (static_cast<uint64_t>(key) << 32) | static_cast<uint64_t>(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t composite_index(uint64_t c) {
  return 0xffffffffu - static_cast<uint32_t>(c & 0xffffffffull);
}

// SplitMix64 output function (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014).
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// The K-th largest of n distinct 64-bit composites get(i), i < n (K <= n), by an 8-pass radix
// select on 8-bit digits (most significant first).  All threads of the CTA call it.
template <class Get>
__device__ uint64_t radix_kth(int n, int K, Get get, uint32_t* hist, uint32_t* scan, uint64_t* shared_out) {
  uint64_t prefix = 0, mask = 0;
  uint32_t want = static_cast<uint32_t>(K);
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int shift = 56; shift >= 0; shift -= 8) {
    hist[threadIdx.x] = 0u;
    __syncthreads();
#pragma unroll 1
    for (int i0 = 0; i0 < n; i0 += kThreads) {
      const int i = i0 + threadIdx.x;
      bool in = false;
      uint32_t d = 0;
      if (i < n) {
        const uint64_t c = get(i);
        in = (c & mask) == prefix;
        d = static_cast<uint32_t>(c >> shift) & 255u;
      }
      // one shared-memory atomic per distinct digit of the warp
      const uint32_t active = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t same = __match_any_sync(active, d);
        if (lane == __ffs(same) - 1) atomicAdd(&hist[d], static_cast<uint32_t>(__popc(same)));
      }
    }
    __syncthreads();
    // inclusive scan of the counts from the largest digit down: scan[t] = #(digit >= 255 - t)
    scan[threadIdx.x] = hist[255 - threadIdx.x];
    __syncthreads();
#pragma unroll 1
    for (int off = 1; off < 256; off <<= 1) {
      const uint32_t v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0u;
      __syncthreads();
      scan[threadIdx.x] += v;
      __syncthreads();
    }
    const uint32_t below = threadIdx.x > 0 ? scan[threadIdx.x - 1] : 0u;
    if (below < want && want <= scan[threadIdx.x]) {
      shared_out[0] = static_cast<uint64_t>(255 - threadIdx.x);
      shared_out[1] = static_cast<uint64_t>(want - below);
    }
    __syncthreads();
    prefix |= shared_out[0] << shift;
    mask |= 255ull << shift;
    want = static_cast<uint32_t>(shared_out[1]);
    __syncthreads();
  }
  return prefix;
}

// Stage 1: the K largest composites of slice `blockIdx.x` of row `blockIdx.y`.
__global__ void __launch_bounds__(kThreads) sample_candidates_kernel(const float* __restrict__ logits, int vocab,
                                                                     int slice_len, int K,
                                                                     uint64_t* __restrict__ cand) {
  __shared__ uint32_t keys[kSliceSmemBytes / 4];
  __shared__ uint32_t hist[256], scan[256];
  __shared__ uint64_t sel[2];
  __shared__ uint32_t nout;
  const int b = blockIdx.y, s = blockIdx.x, S = gridDim.x;
  const int lo = s * slice_len, hi = min(vocab, lo + slice_len);
  const int n = max(0, hi - lo);
  const float* row = logits + static_cast<size_t>(b) * vocab;
  for (int i = threadIdx.x; i < n; i += kThreads) keys[i] = order_key(row[lo + i]);
  if (threadIdx.x == 0) nout = 0u;
  __syncthreads();
  uint64_t* out = cand + (static_cast<size_t>(b) * S + s) * K;
  auto get = [&](int i) { return composite(keys[i], static_cast<uint32_t>(lo + i)); };
  if (n <= K) {  // the whole slice (and padding that sorts below every real entry)
    for (int j = threadIdx.x; j < K; j += kThreads) out[j] = j < n ? get(j) : 0ull;
    return;
  }
  const uint64_t kth = radix_kth(n, K, get, hist, scan, sel);
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const uint64_t c = get(i);
    if (c >= kth) {  // exactly K entries (the composites are distinct); the guard only bounds the store
      const unsigned j = atomicAdd(&nout, 1u);
      if (j < static_cast<unsigned>(K)) out[j] = c;
    }
  }
}

// Stage 2: the K largest of the S * K candidates of row blockIdx.x, then the draw.
__global__ void __launch_bounds__(kThreads) sample_pick_kernel(const uint64_t* __restrict__ cand, int S, int K,
                                                               int vocab, float temperature, float top_p,
                                                               uint64_t seed, const int32_t* __restrict__ positions,
                                                               int32_t* __restrict__ tokens) {
  __shared__ uint64_t c[kMaxSlices * kMaxTopK];
  __shared__ uint64_t top[kMaxTopK];
  __shared__ uint32_t hist[256], scan[256];
  __shared__ uint64_t sel[2];
  __shared__ uint32_t nout;
  const int b = blockIdx.x, M = S * K;
  for (int i = threadIdx.x; i < M; i += kThreads) c[i] = cand[static_cast<size_t>(b) * M + i];
  if (threadIdx.x == 0) nout = 0u;
  __syncthreads();
  // padding entries (0) never rank above a real logit: every real composite has a key >= 1
  const int kk = min(K, vocab);
  auto get = [&](int i) { return c[i]; };
  const uint64_t kth = radix_kth(M, kk, get, hist, scan, sel);
  for (int i = threadIdx.x; i < M; i += kThreads)
    if (c[i] >= kth && c[i] != 0ull) {
      const unsigned j = atomicAdd(&nout, 1u);
      if (j < static_cast<unsigned>(kk)) top[j] = c[i];
    }
  __syncthreads();
  // rank sort of the kk winners (descending)
  uint64_t mine = 0ull;
  int rank = 0;
  if (threadIdx.x < kk) {
    mine = top[threadIdx.x];
    for (int j = 0; j < kk; ++j) rank += top[j] > mine;
  }
  __syncthreads();
  if (threadIdx.x < kk) top[rank] = mine;
  __syncthreads();
  if (threadIdx.x != 0) return;
  int pick = 0;
  if (kk > 1) {
    // softmax over the kk logits at temperature, in rank order
    float z[kMaxTopK];
    const float inv_t = 1.0f / temperature;
    for (int j = 0; j < kk; ++j) z[j] = key_value(static_cast<uint32_t>(top[j] >> 32)) * inv_t;
    const float zmax = z[0];
    float sum = 0.f;
    for (int j = 0; j < kk; ++j) {
      z[j] = expf(z[j] - zmax);
      sum += z[j];
    }
    // top-p: the shortest prefix whose probability mass reaches top_p
    int keep = kk;
    float acc = 0.f;
    for (int j = 0; j < kk; ++j) {
      acc += z[j] / sum;
      if (acc >= top_p) {
        keep = j + 1;
        break;
      }
    }
    float mass = 0.f;
    for (int j = 0; j < keep; ++j) mass += z[j];
    const int pos = positions ? positions[b] : 0;
    // one stream per seed (SplitMix64 of the seed), one draw per (position, row): the two fields
    // occupy disjoint bits, so no two (seed, position, row) triples share an input
    const uint64_t r = splitmix64(splitmix64(seed) ^ ((static_cast<uint64_t>(static_cast<uint32_t>(pos)) << 32) |
                                                      static_cast<uint64_t>(static_cast<uint32_t>(b))));
    const float u = static_cast<float>(r >> 40) * (1.0f / 16777216.0f);  // [0, 1), 24 bits
    const float target = u * mass;
    float cum = 0.f;
    pick = keep - 1;
    for (int j = 0; j < keep; ++j) {
      cum += z[j];
      if (target < cum) {
        pick = j;
        break;
      }
    }
  }
  tokens[b] = static_cast<int32_t>(composite_index(top[pick]));
}

struct Geometry {
  int S, slice_len;
};

Geometry geometry(int batch, int vocab) {
  Geometry g{};
  int S = (296 + batch - 1) / batch;  // about two CTAs per SM of a B200 over the whole batch
  const int min_s = (vocab * 4 + kSliceSmemBytes - 1) / kSliceSmemBytes;
  S = S < min_s ? min_s : S;
  S = S > kMaxSlices ? kMaxSlices : S;
  S = S < 1 ? 1 : S;
  g.S = S;
  g.slice_len = (vocab + S - 1) / S;
  return g;
}

int sample_fail(const char* msg) {
  nkm::set_last_error(msg);
  return NKM_ERR_ARG;
}

}  // namespace

extern "C" size_t nkm_sample_workspace_bytes(int32_t batch, int32_t vocab, int32_t top_k) {
  if (batch <= 0 || vocab <= 0 || top_k <= 0 || top_k > kMaxTopK) return 0;
  const Geometry g = geometry(batch, vocab);
  return static_cast<size_t>(batch) * g.S * top_k * sizeof(uint64_t);
}

extern "C" int nkm_sample_logits(const float* logits, int32_t batch, int32_t vocab, const nkm_sample_params* sp,
                                 const int32_t* positions, int32_t* tokens_out, void* workspace,
                                 size_t workspace_bytes, nkm_stream_t stream_) {
  if (!logits || !tokens_out || !sp) return sample_fail("logits, tokens_out and params must be given");
  if (batch <= 0 || vocab <= 0) return sample_fail("batch and vocab must be positive");
  const int K = sp->top_k;
  if (K < 1 || K > kMaxTopK) return sample_fail("top_k must be in 1..64");
  if (K > 1 && !(sp->temperature > 0.f)) return sample_fail("temperature must be positive");
  if (K > 1 && !(sp->top_p > 0.f && sp->top_p <= 1.f)) return sample_fail("top_p must be in (0, 1]");
  const Geometry g = geometry(batch, vocab);
  if (static_cast<int64_t>(g.slice_len) * 4 > kSliceSmemBytes) return sample_fail("vocab too large");
  const size_t need = static_cast<size_t>(batch) * g.S * K * sizeof(uint64_t);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 7))
    return sample_fail("workspace missing, too small (nkm_sample_workspace_bytes) or not 8-byte aligned");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  uint64_t* cand = static_cast<uint64_t*>(workspace);
  sample_candidates_kernel<<<dim3(g.S, batch), kThreads, 0, stream>>>(logits, vocab, g.slice_len, K, cand);
  sample_pick_kernel<<<batch, kThreads, 0, stream>>>(cand, g.S, K, vocab, sp->temperature, sp->top_p, sp->seed,
                                                     positions, tokens_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}
