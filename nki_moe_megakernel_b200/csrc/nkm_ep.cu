// Expert-parallel exchange for batches split across GPUs (config 3 across a node): each rank
// owns a contiguous slice of the batch's rows for attention and a contiguous range of experts;
// per layer every rank gathers all rows' post-attention hidden states (its experts may be routed
// any row), runs the MoE block on its experts only (nkm_moe_block_tc_partial), and sends each
// owner the partial sums of the owner's rows, which the owner adds in rank order.
//
// The data crosses NVLink as plain 16-byte stores into the peers' exchange regions (CUDA IPC
// mappings); each sending CTA then releases (system scope) an arrival on the receiver's counter,
// and the receiver's wait kernel polls its own counter with acquire loads, bounded by 2 s
// (NKM_ERR_TIMEOUT in the status word on expiry).  Counters only grow; the caller tracks the
// targets.  No TMA or library kernel ever reads peer memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "nkimoe.h"
#include "nkm_ptx.cuh"

namespace nkm {
void set_last_error(const char* msg);
}

namespace {

constexpr int kPushBlocks = 8;  // CTAs per destination of one push (each adds one arrival)
constexpr uint64_t kWaitNs = 2000000000ull;

struct PushDst {
  uint8_t* dst[8];
  unsigned long long* flag[8];
};

// CTA (i, q): bytes [n * i / kPushBlocks, n * (i + 1) / kPushBlocks) of src to dst[q] + offset
__global__ void __launch_bounds__(256) ep_push_kernel(const uint4* __restrict__ src, int64_t n16, PushDst d,
                                                      int64_t dst_off) {
  const int q = blockIdx.y, i = blockIdx.x;
  const int64_t lo = n16 * i / kPushBlocks, hi = n16 * (i + 1) / kPushBlocks;
  uint4* dst = reinterpret_cast<uint4*>(d.dst[q] + dst_off);
  for (int64_t k = lo + threadIdx.x; k < hi; k += blockDim.x) dst[k] = src[k];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's stores (ordered by the CTA barrier) before the arrival
    atomicAdd_system(d.flag[q], 1ull);
  }
}

__global__ void ep_wait_kernel(const unsigned long long* flag, unsigned long long target, int* status) {
  if (threadIdx.x != 0) return;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= target) return;
    if (it == 0) {
      t0 = nkm::globaltimer_ns();
    } else if ((it & 63u) == 0 && nkm::globaltimer_ns() - t0 > kWaitNs) {
      atomicOr(status, NKM_ERR_TIMEOUT);
      return;
    }
    __nanosleep(100);
  }
}

// y[r] = bf16(x[r] + bf16(sum over the n ranks, in rank order, of parts[q][r]))
__global__ void ep_reduce_kernel(const float* __restrict__ parts, int n, int64_t rows_h, const uint16_t* __restrict__ x,
                                 uint16_t* __restrict__ y) {
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < rows_h;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < n; ++q) s += parts[q * rows_h + k];
    y[k] = nkm::f2bf(nkm::bf2f(x[k]) + nkm::rbf(s));
  }
}

int fail(const char* m) {
  nkm::set_last_error(m);
  return NKM_ERR_ARG;
}

}  // namespace

extern "C" int nkm_ep_push(const void* src, int64_t bytes, void* const* dst, int32_t n_dst, int64_t dst_offset,
                           unsigned long long* const* flags, nkm_stream_t stream) {
  if (!src || !dst || !flags || n_dst <= 0 || n_dst > 8 || bytes <= 0 || bytes % 16 || dst_offset % 16 ||
      (reinterpret_cast<uintptr_t>(src) & 15))
    return fail("nkm_ep_push: 1..8 destinations, 16-byte aligned source, size and offset");
  PushDst d{};
  for (int q = 0; q < n_dst; ++q) {
    if (!dst[q] || !flags[q] || (reinterpret_cast<uintptr_t>(dst[q]) & 15) || (reinterpret_cast<uintptr_t>(flags[q]) & 7))
      return fail("nkm_ep_push: destination or counter missing or misaligned");
    d.dst[q] = static_cast<uint8_t*>(dst[q]);
    d.flag[q] = flags[q];
  }
  ep_push_kernel<<<dim3(kPushBlocks, n_dst), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), bytes / 16, d, dst_offset);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}

extern "C" int32_t nkm_ep_arrivals_per_push(void) { return kPushBlocks; }

extern "C" int nkm_ep_wait(const unsigned long long* flag, unsigned long long target, int32_t* status,
                           nkm_stream_t stream) {
  if (!flag || !status) return fail("nkm_ep_wait: counter and status required");
  ep_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flag, target, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}

extern "C" int nkm_ep_reduce(const float* parts, int32_t n, int32_t rows, int32_t hidden, const void* x_res,
                             void* y_out, nkm_stream_t stream) {
  if (!parts || !x_res || !y_out || n <= 0 || rows <= 0 || hidden <= 0) return fail("nkm_ep_reduce: bad arguments");
  const int64_t rh = static_cast<int64_t>(rows) * hidden;
  const int grid = static_cast<int>((rh + 255) / 256 < 1184 ? (rh + 255) / 256 : 1184);
  ep_reduce_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      parts, n, rh, static_cast<const uint16_t*>(x_res), static_cast<uint16_t*>(y_out));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nkm::set_last_error(cudaGetErrorString(e));
    return NKM_ERR_CUDA;
  }
  return NKM_OK;
}
