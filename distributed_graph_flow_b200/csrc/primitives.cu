// Exclusive scan (reduce-then-scan, recursive over tile sums) and a stable
// LSD radix sort (8-bit digits; per-tile histograms, one scan, then a
// warp-ordered stable scatter using __match_any_sync ranking).
#include "primitives.cuh"

namespace dgfx {

// ===========================================================================
// Scan
// ===========================================================================
template <class Tin>
__global__ void __launch_bounds__(kScanThreads)
scan_reduce_kernel(const Tin* __restrict__ in, int64_t n, int64_t* __restrict__ sums) {
  __shared__ int64_t smem[33];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + static_cast<int64_t>(i) * kScanThreads + threadIdx.x;
    if (idx < n) s += static_cast<int64_t>(in[idx]);
  }
  int64_t total;
  block_exclusive_scan<int64_t>(s, smem, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Each thread owns kScanItems consecutive elements.
template <class Tin>
__global__ void __launch_bounds__(kScanThreads)
scan_tile_kernel(const Tin* in, int64_t* out, int64_t n, const int64_t* __restrict__ tile_offsets,
                 bool write_total) {
  __shared__ int64_t smem[33];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + static_cast<int64_t>(threadIdx.x) * kScanItems;
  int64_t v[kScanItems];
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + i;
    v[i] = idx < n ? static_cast<int64_t>(in[idx]) : 0;
    s += v[i];
  }
  int64_t prefix = block_exclusive_scan<int64_t>(s, smem, nullptr);
  if (tile_offsets != nullptr) prefix += tile_offsets[blockIdx.x];
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const int64_t idx = base + i;
    if (idx < n) out[idx] = prefix;
    if (write_total && idx == n - 1) out[n] = prefix + v[i];
    prefix += v[i];
  }
}

size_t scan_workspace_bytes(int64_t n) {
  size_t bytes = 0;
  int64_t m = n;
  while (m > kScanTile) {
    m = ceil_div(m, kScanTile);
    bytes += align_up(static_cast<size_t>(m) * sizeof(int64_t), 256);
  }
  return bytes + 256;
}

template <class Tin>
int exclusive_scan(const Tin* d_in, int64_t* d_out, int64_t n, bool write_total, Arena& ws,
                   cudaStream_t stream) {
  if (n <= 0) {
    if (write_total && !ws.dry) DGFX_CUDA_TRY(cudaMemsetAsync(d_out, 0, sizeof(int64_t), stream));
    return DGFX_OK;
  }
  const int64_t tiles = ceil_div(n, kScanTile);
  int64_t* tile_offsets = nullptr;
  if (tiles > 1) {
    tile_offsets = ws.take<int64_t>(static_cast<size_t>(tiles));
    if (!ws.ok()) return fail(DGFX_ERR_WORKSPACE, "scan: workspace too small");
    if (!ws.dry) {
      scan_reduce_kernel<Tin><<<static_cast<unsigned>(tiles), kScanThreads, 0, stream>>>(d_in, n, tile_offsets);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
    DGFX_TRY(exclusive_scan<int64_t>(tile_offsets, tile_offsets, tiles, false, ws, stream));
  }
  if (!ws.dry) {
    scan_tile_kernel<Tin><<<static_cast<unsigned>(tiles), kScanThreads, 0, stream>>>(d_in, d_out, n, tile_offsets,
                                                                                      write_total);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  return DGFX_OK;
}

// One CTA per array; thread t owns the contiguous elements [t * per,
// (t + 1) * per).
template <class Tin>
__global__ void __launch_bounds__(kSmallScanThreads)
small_scan_pair_kernel(const Tin* __restrict__ in0, int64_t* __restrict__ out0, int64_t n0,
                       const Tin* __restrict__ in1, int64_t* __restrict__ out1, int64_t n1) {
  __shared__ int64_t smem[33];
  const Tin* in = blockIdx.x == 0 ? in0 : in1;
  int64_t* out = blockIdx.x == 0 ? out0 : out1;
  const int64_t n = blockIdx.x == 0 ? n0 : n1;
  constexpr int kMaxPer = static_cast<int>(kSmallScanMax / kSmallScanThreads);
  const int per = static_cast<int>((n + kSmallScanThreads - 1) / kSmallScanThreads);
  const int64_t lo = static_cast<int64_t>(threadIdx.x) * per;
  Tin v[kMaxPer];  // all loads issued before the scan, kept in registers
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    v[i] = (i < per && lo + i < n) ? in[lo + i] : Tin(0);
    s += static_cast<int64_t>(v[i]);
  }
  int64_t total;
  int64_t prefix = block_exclusive_scan<int64_t>(s, smem, &total);
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    if (i < per && lo + i < n) out[lo + i] = prefix;
    prefix += static_cast<int64_t>(v[i]);
  }
  if (threadIdx.x == 0) out[n] = total;
}

template <class Tin>
int exclusive_scan_pair(const Tin* d_in0, int64_t* d_out0, int64_t n0, const Tin* d_in1, int64_t* d_out1,
                        int64_t n1, Arena& ws, cudaStream_t stream) {
  if (n0 <= kSmallScanMax && n1 <= kSmallScanMax) {
    if (!ws.dry) {
      small_scan_pair_kernel<Tin><<<2, kSmallScanThreads, 0, stream>>>(d_in0, d_out0, n0, d_in1, d_out1, n1);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
    return DGFX_OK;
  }
  const size_t mark = ws.used;
  DGFX_TRY(exclusive_scan<Tin>(d_in0, d_out0, n0, true, ws, stream));
  ws.used = mark;
  return exclusive_scan<Tin>(d_in1, d_out1, n1, true, ws, stream);
}

template int exclusive_scan_pair<int32_t>(const int32_t*, int64_t*, int64_t, const int32_t*, int64_t*, int64_t,
                                          Arena&, cudaStream_t);

template int exclusive_scan<int64_t>(const int64_t*, int64_t*, int64_t, bool, Arena&, cudaStream_t);
template int exclusive_scan<int32_t>(const int32_t*, int64_t*, int64_t, bool, Arena&, cudaStream_t);
template int exclusive_scan<uint32_t>(const uint32_t*, int64_t*, int64_t, bool, Arena&, cudaStream_t);

// ===========================================================================
// Radix sort
// ===========================================================================
__global__ void __launch_bounds__(kSortThreads)
radix_hist_kernel(const uint64_t* __restrict__ keys, int64_t n, int shift, int64_t num_tiles,
                  uint32_t* __restrict__ hist) {
  __shared__ uint32_t cnt[8][256];
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&cnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kSortTile;
  for (int i = threadIdx.x; i < kSortTile; i += blockDim.x) {
    const int64_t idx = base + i;
    if (idx < n) {
      const uint32_t d = static_cast<uint32_t>(keys[idx] >> shift) & 0xFFu;
      atomicAdd(&cnt[warp][d], 1u);
    }
  }
  __syncthreads();
  {
    const int d = threadIdx.x;  // blockDim == 256
    uint32_t s = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += cnt[w][d];
    hist[static_cast<int64_t>(d) * num_tiles + blockIdx.x] = s;
  }
}

// Stable scatter. Warp w of tile t owns items [t*4096 + w*512, +512), visited
// in 16 rounds of 32 consecutive items, so (warp, round, lane) order equals
// input order and equal digits keep their relative order.
__global__ void __launch_bounds__(kSortThreads)
radix_scatter_kernel(const uint64_t* __restrict__ kin, const uint32_t* __restrict__ vin,
                     uint64_t* __restrict__ kout, uint32_t* __restrict__ vout, int64_t n, int shift,
                     int64_t num_tiles, const int64_t* __restrict__ offsets) {
  constexpr int kRounds = kSortItemsPerWarp / 32;
  __shared__ uint32_t wcnt[8][256];
  __shared__ int64_t tile_off[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  tile_off[threadIdx.x] = offsets[static_cast<int64_t>(threadIdx.x) * num_tiles + blockIdx.x];
  __syncthreads();

  const int64_t wbase = static_cast<int64_t>(blockIdx.x) * kSortTile + static_cast<int64_t>(warp) * kSortItemsPerWarp;
  const uint32_t lt_mask = (1u << lane) - 1u;
  uint64_t key[kRounds];
  uint32_t val[kRounds];
  uint32_t rank[kRounds];  // digit in the low 9 bits (256 = empty), rank above
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int64_t idx = wbase + r * 32 + lane;
    const bool valid = idx < n;
    key[r] = valid ? kin[idx] : 0ull;
    val[r] = valid ? vin[idx] : 0u;
    const uint32_t d = valid ? (static_cast<uint32_t>(key[r] >> shift) & 0xFFu) : 256u;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t before = __popc(peers & lt_mask);
    uint32_t base = 0;
    if (valid) base = wcnt[warp][d];
    __syncwarp();
    if (valid && before == 0) wcnt[warp][d] = base + __popc(peers);
    __syncwarp();
    rank[r] = ((base + before) << 9) | d;
  }
  __syncthreads();
  {
    const int d = threadIdx.x;
    uint32_t acc = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t c = wcnt[w][d];
      wcnt[w][d] = acc;
      acc += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const uint32_t d = rank[r] & 0x1FFu;
    if (d < 256u) {
      const int64_t pos = tile_off[d] + wcnt[warp][d] + (rank[r] >> 9);
      kout[pos] = key[r];
      vout[pos] = val[r];
    }
  }
}

size_t radix_sort_workspace_bytes(int64_t n) {
  const int64_t tiles = ceil_div(n, kSortTile);
  const int64_t h = 256 * tiles;
  return align_up(static_cast<size_t>(h) * sizeof(uint32_t), 256) +
         align_up(static_cast<size_t>(h + 1) * sizeof(int64_t), 256) + scan_workspace_bytes(h) + 512;
}

int radix_sort_pairs(uint64_t* k0, uint32_t* v0, uint64_t* k1, uint32_t* v1, int64_t n, int begin_bit,
                     int end_bit, bool* result_in_1, Arena& ws, cudaStream_t stream) {
  *result_in_1 = false;
  if (n <= 1 || end_bit <= begin_bit) return DGFX_OK;
  const int64_t tiles = ceil_div(n, kSortTile);
  const int64_t h = 256 * tiles;
  uint32_t* hist = ws.take<uint32_t>(static_cast<size_t>(h));
  int64_t* offs = ws.take<int64_t>(static_cast<size_t>(h + 1));
  if (!ws.ok()) return fail(DGFX_ERR_WORKSPACE, "radix sort: workspace too small");
  const size_t mark = ws.used;
  bool in1 = false;
  for (int shift = begin_bit; shift < end_bit; shift += 8) {
    uint64_t* ki = in1 ? k1 : k0;
    uint32_t* vi = in1 ? v1 : v0;
    uint64_t* ko = in1 ? k0 : k1;
    uint32_t* vo = in1 ? v0 : v1;
    if (!ws.dry) {
      radix_hist_kernel<<<static_cast<unsigned>(tiles), kSortThreads, 0, stream>>>(ki, n, shift, tiles, hist);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
    ws.used = mark;
    DGFX_TRY(exclusive_scan<uint32_t>(hist, offs, h, false, ws, stream));
    if (!ws.dry) {
      radix_scatter_kernel<<<static_cast<unsigned>(tiles), kSortThreads, 0, stream>>>(ki, vi, ko, vo, n, shift, tiles,
                                                                                     offs);
      DGFX_CUDA_TRY(cudaGetLastError());
    }
    in1 = !in1;
  }
  *result_in_1 = in1;
  return DGFX_OK;
}

}  // namespace dgfx
