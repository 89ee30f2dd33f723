// Shared device/host helpers for the dgfx kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/dgfx.h"

namespace dgfx {

// ---------------------------------------------------------------------------
// Error plumbing. Every C-ABI entry point returns a dgfx_status; the message
// of the last failure on the calling host thread is kept for dgfx_last_error.
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define DGFX_CUDA_TRY(expr)                                                  \
  do {                                                                       \
    cudaError_t _e = (expr);                                                 \
    if (_e != cudaSuccess) {                                                 \
      return ::dgfx::fail(DGFX_ERR_CUDA, std::string(#expr) + ": " +         \
                                             cudaGetErrorString(_e));        \
    }                                                                        \
  } while (0)

#define DGFX_TRY(expr)          \
  do {                          \
    int _s = (expr);            \
    if (_s != DGFX_OK) return _s; \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace. Alignment 256 bytes.
struct Arena {
  char* base;
  size_t cap;
  size_t used = 0;
  bool dry;  // size query only
  Arena(void* b, size_t c) : base(static_cast<char*>(b)), cap(c), dry(b == nullptr) {}
  template <class T>
  T* take(size_t count) {
    const size_t off = align_up(used, 256);
    used = off + align_up(count * sizeof(T), 256);
    if (dry) return nullptr;
    return reinterpret_cast<T*>(base + off);
  }
  bool ok() const { return dry || used <= cap; }
};

// ---------------------------------------------------------------------------
// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC'11). Multipliers and Weyl
// key increments are the published Philox4x32 constants.
// ---------------------------------------------------------------------------
struct U4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ void philox_round(U4& c, uint32_t k0, uint32_t k1) {
  const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c.x;
  const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c.z;
  const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
  const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
  c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
}

__host__ __device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k0, k1);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Uniform integer in [0, range) from a 64-bit uniform word by the
// multiply-high method (Lemire, "Fast random integer generation in an
// interval", 2019); bias <= range / 2^64.
__host__ __device__ __forceinline__ uint64_t bounded64(uint64_t r, uint64_t range) {
#ifdef __CUDA_ARCH__
  return __umul64hi(r, range);
#else
  return static_cast<uint64_t>((static_cast<unsigned __int128>(r) * range) >> 64);
#endif
}

// ---------------------------------------------------------------------------
// Warp / block scan helpers.
// ---------------------------------------------------------------------------
template <class T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

template <class T>
__device__ __forceinline__ T warp_reduce_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide exclusive scan of one value per thread (blockDim.x a multiple
// of 32). `smem` must hold 33 elements. Returns the exclusive prefix; if
// `total` is non-null it receives the block sum. Contains __syncthreads: call
// from every thread of the block.
template <class T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const T inc = warp_inclusive_scan(v);
  if (lane == 31) smem[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const T w = lane < nwarps ? smem[lane] : T(0);
    const T wi = warp_inclusive_scan(w);
    if (lane < nwarps) smem[lane] = wi - w;
    if (lane == 31) smem[32] = wi;
  }
  __syncthreads();
  const T res = smem[warp] + inc - v;
  if (total != nullptr) *total = smem[32];
  __syncthreads();
  return res;
}

}  // namespace dgfx
