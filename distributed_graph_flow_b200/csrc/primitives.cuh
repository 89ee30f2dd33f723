// Device-wide primitives used by the CSR builder, the sampler and the SpMM
// planner: exclusive scan and a stable LSD radix sort of (uint64 key, uint32
// value) pairs. All temporaries come from a caller-provided workspace.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace dgfx {

// ---- exclusive scan -------------------------------------------------------
// out[i] = sum(in[0..i)) for i < n; if write_total, out[n] = sum(in[0..n)).
// `in` and `out` may alias. Tin is widened to int64.
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int64_t kScanTile = kScanThreads * kScanItems;

size_t scan_workspace_bytes(int64_t n);
template <class Tin>
int exclusive_scan(const Tin* d_in, int64_t* d_out, int64_t n, bool write_total,
                   Arena& ws, cudaStream_t stream);
// Two independent exclusive scans with totals (out[n] written). Arrays of at
// most kSmallScanMax elements take one launch of one CTA per array (a batch's
// per-seed counts); longer ones the general scan.
constexpr int kSmallScanThreads = 1024;
constexpr int64_t kSmallScanMax = 16 * kSmallScanThreads;
template <class Tin>
int exclusive_scan_pair(const Tin* d_in0, int64_t* d_out0, int64_t n0, const Tin* d_in1, int64_t* d_out1,
                        int64_t n1, Arena& ws, cudaStream_t stream);

// ---- radix sort -----------------------------------------------------------
// Stable sort of (key, value) pairs by key bits [begin_bit, end_bit).
// Ping-pongs between (k0, v0) and (k1, v1); *result_in_1 tells which pair of
// buffers holds the sorted data.
constexpr int kSortThreads = 256;
constexpr int kSortItemsPerWarp = 512;
constexpr int64_t kSortTile = 8 * kSortItemsPerWarp;  // 4096

size_t radix_sort_workspace_bytes(int64_t n);
int radix_sort_pairs(uint64_t* k0, uint32_t* v0, uint64_t* k1, uint32_t* v1,
                     int64_t n, int begin_bit, int end_bit, bool* result_in_1,
                     Arena& ws, cudaStream_t stream);

inline int bit_length(uint64_t x) {
  int b = 0;
  while (x) {
    ++b;
    x >>= 1;
  }
  return b;
}

}  // namespace dgfx
