// Peer-memory feature gather for node-range-partitioned features.
//
// Every rank's feature partition is a plain cudaMalloc allocation whose CUDA
// IPC handle the other ranks open once (dgfx_ipc_*), so a rank holds device
// pointers to all partitions. dgfx_gather_rows_p2p then fetches each requested
// row from its owner in one kernel: local rows from this GPU's HBM, remote
// rows with ordinary 16-byte loads through NVLink / NVSwitch. No host
// synchronisation, no sort, no all-to-all; it replaces the halo exchange's
// partition + NCCL all-to-all + scatter sequence (driver.HaloFeatures) when
// peer access is available. Loads are plain ld.global (no TMA, no multicast).
#include <algorithm>
#include <cstring>
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {

// out[i] = partition(owner)[row] for ids[*begin + i], owner = id / rows_per_rank.
// Each thread keeps U independent (id load -> row load) chains in flight to
// cover NVLink latency; 16-byte vectors per row = 1 << lvpr (row widths are
// powers of two here; other widths use the division path).
// Small CTAs (64 threads, <= 32 registers) so the gather can run beside a
// resident sampler kernel (it fills shared memory but leaves registers and
// threads for a few such CTAs per SM) when steps are pipelined.
constexpr int kGatherThreads = 64;

template <int U>
__global__ void __launch_bounds__(kGatherThreads, 32) gather_p2p_kernel(const uint4* const* __restrict__ tables, int32_t world,
                                                          uint32_t rows_per_rank, uint32_t num_nodes, int64_t vpr,
                                                          int lvpr, const int64_t* __restrict__ ids,
                                                          const int64_t* __restrict__ begin,
                                                          const int64_t* __restrict__ end, int64_t max_rows,
                                                          uint4* __restrict__ out) {
  const int64_t lo = *begin;
  int64_t n = *end - lo;
  n = n < max_rows ? n : max_rows;
  const int64_t total = n * vpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; base < total;
       base += stride * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = base + u * stride;
      x[u] = make_uint4(0, 0, 0, 0);
      if (v < total) {
        const int64_t i = lvpr >= 0 ? (v >> lvpr) : v / vpr;
        const int64_t c = v - i * vpr;
        const int64_t id = ids[lo + i];
        if (id >= 0 && id < num_nodes) {
          const uint32_t o = static_cast<uint32_t>(id) / rows_per_rank;
          if (o < static_cast<uint32_t>(world)) {
            x[u] = __ldg(tables[o] + (static_cast<int64_t>(static_cast<uint32_t>(id) - o * rows_per_rank) * vpr + c));
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = base + u * stride;
      if (v < total) out[v] = x[u];
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk peer exchange. Random row reads from peer memory are far slower than
// sequential ones on NVSwitch systems with many mapped peers, so this path
// moves only contiguous runs across NVLink: requesters bucket their ids by
// owner in their own buffer; owners read those buckets (sequential peer
// reads), gather the rows from local HBM (random, local) and write them
// into each requester's inbox (sequential peer stores, which outrun peer
// loads here); requesters scatter their inbox rows into request order
// (local). A barrier separates the three launches: exchange_barrier_kernel
// (peer flags, bounded wait) or any group-wide barrier on the same stream.
//
// Exchange buffer layout, identical on every rank (S = slot_rows):
//   [0, 8 * (world + 1))                 int64 request count per owner, then
//                                        per local replica (slot `world`)
//   [kExStatusOff, +4)                   uint32 status: 1 slot overflow, 2 barrier timeout
//   [kExEpochOff, +4)                    uint32 this rank's barrier epoch when barriers take
//                                        their epoch on the device (epoch argument 0)
//   [kExFlagsOff, + 4 * world)           uint32 barrier arrival epoch per rank
//   [kExIdsOff, + 8 * (world + 1) * S)   int64 request ids; slot o = ids owned by
//                                        rank o, slot `world` = replica rows
//   [rows_off, + world * S * row_bytes)  inbox rows; slot o = rows sent by owner o
// Requests whose node has a row in the optional local replica table (a
// read-only copy of frequently requested rows, hot_slot[id] >= 0) never
// cross NVLink: they go to slot `world` and are copied locally by the serve
// launch.
// ---------------------------------------------------------------------------
constexpr int kMaxWorld = 16;
constexpr int64_t kExStatusOff = 256;
constexpr int64_t kExEpochOff = 264;  // uint32 device-side barrier epoch of this rank
constexpr int64_t kExFlagsOff = 320;
constexpr int64_t kExIdsOff = 512;

inline int64_t ex_rows_off(int32_t world, int64_t slot_rows) {
  return (kExIdsOff + 8 * static_cast<int64_t>(world + 1) * slot_rows + 255) / 256 * 256;
}

constexpr int kPartThreads = 256;
constexpr int kPartItems = 8;

// One tile of kPartThreads * kPartItems requests per CTA. Slot offsets come
// from warp-aggregated shared-memory counters and one global atomic per owner
// per CTA (the per-owner counters are the hottest words otherwise).
__global__ void __launch_bounds__(kPartThreads) exchange_partition_kernel(
    char* __restrict__ ex, int32_t world, int64_t slot_rows, uint32_t rows_per_rank, uint32_t num_nodes, int64_t vpr,
    const int64_t* __restrict__ ids, const int64_t* __restrict__ begin, const int64_t* __restrict__ end,
    int64_t max_rows, const int32_t* __restrict__ hot_slot, int32_t* __restrict__ req_pos, uint4* __restrict__ out) {
  __shared__ int s_cnt[kMaxWorld + 1];
  __shared__ unsigned long long s_base[kMaxWorld + 1];
  const int64_t lo = *begin;
  int64_t n = *end - lo;
  n = n < max_rows ? n : max_rows;
  const int64_t tile = static_cast<int64_t>(blockIdx.x) * (kPartThreads * kPartItems);
  if (tile >= n) return;  // uniform over the CTA
  if (threadIdx.x <= kMaxWorld) s_cnt[threadIdx.x] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  int own[kPartItems];
  int off[kPartItems];
  int64_t idv[kPartItems];
#pragma unroll
  for (int k = 0; k < kPartItems; ++k) {
    const int64_t i = tile + k * kPartThreads + threadIdx.x;
    int o = -1;
    int64_t id = -1;
    if (i < n) {
      id = ids[lo + i];
      if (id >= 0 && id < num_nodes) {
        o = static_cast<int>(static_cast<uint32_t>(id) / rows_per_rank);
        if (o >= world) o = -1;
        if (o >= 0 && hot_slot != nullptr) {
          const int32_t h = __ldg(hot_slot + id);
          if (h >= 0) {  // served from the local replica: store its row
            o = world;
            id = h;
          }
        }
      }
      if (o < 0) {
        for (int64_t c = 0; c < vpr; ++c) out[i * vpr + c] = make_uint4(0, 0, 0, 0);
      }
    }
    const unsigned m = __match_any_sync(0xffffffffu, o);
    const int leader = __ffs(m) - 1;
    int b = 0;
    if (o >= 0 && lane == leader) b = atomicAdd(&s_cnt[o], __popc(m));
    b = __shfl_sync(0xffffffffu, b, leader);
    own[k] = o;
    off[k] = b + __popc(m & lt);
    idv[k] = id;
  }
  __syncthreads();
  if (threadIdx.x <= world) {
    s_base[threadIdx.x] = atomicAdd(reinterpret_cast<unsigned long long*>(ex) + threadIdx.x,
                                    static_cast<unsigned long long>(s_cnt[threadIdx.x]));
  }
  __syncthreads();
  int64_t* req_ids = reinterpret_cast<int64_t*>(ex + kExIdsOff);
  bool over = false;
#pragma unroll
  for (int k = 0; k < kPartItems; ++k) {
    if (own[k] < 0) continue;
    const int64_t slot = static_cast<int64_t>(s_base[own[k]]) + off[k];
    if (slot < slot_rows) {
      const int64_t at = static_cast<int64_t>(own[k]) * slot_rows + slot;
      req_ids[at] = idv[k];
      req_pos[at] = static_cast<int32_t>(tile + k * kPartThreads + threadIdx.x);
    } else {
      over = true;
    }
  }
  if (over) atomicOr(reinterpret_cast<unsigned*>(ex + kExStatusOff), 1u);
}

// Small CTAs (2 warps, <= 80 registers) that fit on an SM beside other
// kernels when steps are pipelined; 8 loads in flight per lane.
constexpr int kCopyThreads = 64;
constexpr int kCopyUnroll = 8;
constexpr int kChunk = 32;

// Serve (kServe): segments over requesters p, rows = ids in p's slot for this
// rank; source = local partition row, destination = slot `rank` of p's inbox
// (peer stores), or d_out[req_pos] for p == rank. Scatter: segments over
// owners p != rank, source = slot p of this rank's inbox (contiguous),
// destination = d_out[req_pos]. A warp takes 32 rows: lane l resolves row l's
// source and destination rows, then the warp streams the 32 * vpr vectors
// with U loads in flight per lane. Data other ranks wrote (counts, ids) is
// read with ld.global.cv.
template <bool kServe, int U>
__global__ void __launch_bounds__(kCopyThreads, 8) exchange_copy_kernel(
    const char* const* __restrict__ exs, int32_t world, int32_t rank, int64_t slot_rows, int64_t vpr, int lvpr,
    int64_t rows_off, const uint4* __restrict__ table, int64_t row_base, int64_t local_rows,
    const uint4* __restrict__ replica, int64_t replica_rows, const int32_t* __restrict__ req_pos,
    uint4* __restrict__ out) {
  // Segments: ranks 0..world-1, then (serve only) this rank's replica slot.
  __shared__ int64_t s_cnt[kMaxWorld + 1];
  __shared__ int64_t s_pre[kMaxWorld + 2];
  const int nseg = kServe ? world + 1 : world;
  if (threadIdx.x < nseg) {
    const int p = threadIdx.x;
    int64_t c = 0;
    if (kServe && p < world) {
      c = __ldcv(reinterpret_cast<const long long*>(exs[p]) + rank);
    } else if (kServe) {
      c = reinterpret_cast<const int64_t*>(exs[rank])[world];
    } else if (p != rank) {
      c = reinterpret_cast<const int64_t*>(exs[rank])[p];
    }
    s_cnt[p] = c < slot_rows ? c : slot_rows;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t a = 0;
    for (int p = 0; p < nseg; ++p) {
      s_pre[p] = a;
      a += (s_cnt[p] + kChunk - 1) / kChunk;
    }
    s_pre[nseg] = a;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kCopyThreads / 32);
  const int64_t chunks = s_pre[nseg];
  for (int64_t ch = static_cast<int64_t>(blockIdx.x) * (kCopyThreads / 32) + (threadIdx.x >> 5); ch < chunks;
       ch += warps) {
    int p = 0;
    while (p + 1 < nseg && s_pre[p + 1] <= ch) ++p;
    const int64_t k0 = (ch - s_pre[p]) * kChunk;
    const int64_t left = s_cnt[p] - k0;
    const int rows = left < kChunk ? static_cast<int>(left) : kChunk;
    const bool rep = kServe && p == world;  // replica slot: local copy straight to d_out
    int64_t src = -1, dst = 0;
    if (lane < rows) {
      if (rep) {
        const int64_t h =
            reinterpret_cast<const int64_t*>(exs[rank] + kExIdsOff)[static_cast<int64_t>(world) * slot_rows + k0 + lane];
        src = (h >= 0 && h < replica_rows) ? h : -1;
        dst = req_pos[static_cast<int64_t>(world) * slot_rows + k0 + lane];
      } else if (kServe) {
        const int64_t id =
            __ldcv(reinterpret_cast<const long long*>(exs[p] + kExIdsOff) + static_cast<int64_t>(rank) * slot_rows + k0 + lane);
        const int64_t r = id - row_base;
        src = (r >= 0 && r < local_rows) ? r : -1;
        dst = p == rank ? static_cast<int64_t>(req_pos[static_cast<int64_t>(rank) * slot_rows + k0 + lane])
                        : static_cast<int64_t>(rank) * slot_rows + k0 + lane;
      } else {
        src = static_cast<int64_t>(p) * slot_rows + k0 + lane;
        dst = req_pos[static_cast<int64_t>(p) * slot_rows + k0 + lane];
      }
    }
    const uint4* sbase = rep ? replica : (kServe ? table : reinterpret_cast<const uint4*>(exs[rank] + rows_off));
    uint4* dbase = (kServe && !rep && p != rank) ? reinterpret_cast<uint4*>(const_cast<char*>(exs[p]) + rows_off) : out;
    const int64_t nv = static_cast<int64_t>(rows) * vpr;
    for (int64_t b = 0; b < nv; b += 32 * U) {
      uint4 x[U];
      int64_t d[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = b + u * 32 + lane;
        const int r = v < nv ? static_cast<int>(lvpr >= 0 ? (v >> lvpr) : v / vpr) : 0;
        const int64_t c = v - static_cast<int64_t>(r) * vpr;
        const int64_t s = __shfl_sync(0xffffffffu, src, r);
        const int64_t dd = __shfl_sync(0xffffffffu, dst, r);
        x[u] = make_uint4(0, 0, 0, 0);
        d[u] = -1;
        if (v < nv) {
          d[u] = dd * vpr + c;
          if (s >= 0) x[u] = kServe ? __ldg(sbase + s * vpr + c) : __ldcg(sbase + s * vpr + c);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (d[u] >= 0) dbase[d[u]] = x[u];
      }
    }
  }
}

// Group barrier over the exchange buffers: thread t < world publishes this
// rank's arrival `epoch` in rank t's flag word for this rank (system-scope
// release after a system fence), then waits until rank t's flag in this
// rank's buffer reaches `epoch` (system-scope acquire). The wait is bounded
// by max_wait_ns of %globaltimer; on expiry it sets status bit 2 and returns.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void exchange_barrier_kernel(const char* const* __restrict__ exs, int32_t world, int32_t rank,
                                        uint32_t epoch, uint64_t max_wait_ns) {
  __shared__ uint32_t s_epoch;
  const int t = threadIdx.x;
  if (epoch == 0) {  // the epoch from this rank's device counter (every rank advances its own in step)
    if (t == 0) {
      uint32_t* c = reinterpret_cast<uint32_t*>(const_cast<char*>(exs[rank]) + kExEpochOff);
      uint32_t e = *c + 1;
      if (e > 0x7FFFFFFFu) e = 1;
      *c = e;
      s_epoch = e;
    }
    __syncthreads();
    epoch = s_epoch;
  }
  if (t >= world) return;
  __threadfence_system();
  uint32_t* remote = reinterpret_cast<uint32_t*>(const_cast<char*>(exs[t]) + kExFlagsOff) + rank;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(exs[rank] + kExFlagsOff) + t;
  const uint64_t t0 = global_ns();
  for (uint32_t polls = 0;; ++polls) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (static_cast<int32_t>(v - epoch) >= 0) break;
    if ((polls & 63u) == 63u && (global_ns() - t0 > max_wait_ns || polls > (1u << 28))) {
      atomicOr(reinterpret_cast<unsigned*>(const_cast<char*>(exs[rank]) + kExStatusOff), 2u);
      break;
    }
    __nanosleep(64);
  }
}

int lvpr_of(int64_t vpr) {
  for (int b = 0; b < 31; ++b) {
    if ((int64_t(1) << b) == vpr) return b;
  }
  return -1;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

bool ex_args_ok(int32_t world, int64_t slot_rows, int64_t row_bytes) {
  return world >= 1 && world <= kMaxWorld && slot_rows >= 0 && slot_rows < (int64_t(1) << 31) && row_bytes > 0 &&
         row_bytes % 16 == 0;
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_exchange_buffer_size(int32_t world, int64_t slot_rows, int64_t row_bytes, size_t* bytes) {
  if (bytes == nullptr || !ex_args_ok(world, slot_rows, row_bytes)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_buffer_size: bad arguments");
  }
  *bytes = static_cast<size_t>(ex_rows_off(world, slot_rows) + static_cast<int64_t>(world) * slot_rows * row_bytes);
  return DGFX_OK;
}

extern "C" int dgfx_exchange_partition(void* d_exchange, int32_t world, int64_t slot_rows, int64_t rows_per_rank,
                                       int64_t num_nodes, int64_t row_bytes, const int64_t* d_row_ids,
                                       const int64_t* d_begin, const int64_t* d_end, int64_t max_rows,
                                       const int32_t* d_hot_slot, int32_t* d_req_pos, void* d_out,
                                       dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (d_exchange == nullptr || !ex_args_ok(world, slot_rows, row_bytes) || rows_per_rank < 1 || num_nodes < 0 ||
      num_nodes > rows_per_rank * world || max_rows < 0 || d_begin == nullptr || d_end == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_partition: bad arguments");
  }
  if (num_nodes >= (int64_t(1) << 32) || max_rows >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_exchange_partition: more than 2^32 - 1 nodes or 2^31 - 1 rows");
  }
  DGFX_CUDA_TRY(cudaMemsetAsync(d_exchange, 0, 8 * static_cast<size_t>(world + 1), stream));
  if (max_rows == 0) return DGFX_OK;
  const int64_t blocks = ceil_div(max_rows, static_cast<int64_t>(kPartThreads * kPartItems));
  exchange_partition_kernel<<<static_cast<unsigned>(blocks), kPartThreads, 0, stream>>>(
      static_cast<char*>(d_exchange), world, slot_rows, static_cast<uint32_t>(rows_per_rank),
      static_cast<uint32_t>(num_nodes), row_bytes / 16, d_row_ids, d_begin, d_end, max_rows, d_hot_slot, d_req_pos,
      static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

namespace {
int launch_exchange_copy(bool serve, const void* const* d_exchanges, int32_t world, int32_t rank, int64_t slot_rows,
                         int64_t row_bytes, const void* d_table, int64_t row_base, int64_t local_rows,
                         const void* d_replica, int64_t replica_rows, const int32_t* d_req_pos, void* d_out,
                         cudaStream_t stream) {
  const int64_t vpr = row_bytes / 16;
  const int64_t chunks = static_cast<int64_t>(world + 1) * ceil_div(std::max<int64_t>(slot_rows, 1), int64_t(kChunk));
  // Up to 8 small CTAs (16 warps) per SM: on an idle GPU they keep enough
  // rows in flight for the local gathers and the NVLink stores; beside a
  // resident sampler kernel they start as its CTAs retire (the exchange
  // runs on a high-priority stream).
  const int64_t blocks =
      std::max<int64_t>(1, std::min<int64_t>(ceil_div(chunks, int64_t(kCopyThreads / 32)), int64_t(sm_count()) * 8));
  const auto exs = reinterpret_cast<const char* const*>(d_exchanges);
  const int64_t rows_off = ex_rows_off(world, slot_rows);
  if (serve) {
    exchange_copy_kernel<true, kCopyUnroll><<<static_cast<unsigned>(blocks), kCopyThreads, 0, stream>>>(
        exs, world, rank, slot_rows, vpr, lvpr_of(vpr), rows_off, static_cast<const uint4*>(d_table), row_base,
        local_rows, static_cast<const uint4*>(d_replica), replica_rows, d_req_pos, static_cast<uint4*>(d_out));
  } else {
    exchange_copy_kernel<false, kCopyUnroll><<<static_cast<unsigned>(blocks), kCopyThreads, 0, stream>>>(
        exs, world, rank, slot_rows, vpr, lvpr_of(vpr), rows_off, nullptr, 0, 0, nullptr, 0, d_req_pos,
        static_cast<uint4*>(d_out));
  }
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
}  // namespace

extern "C" int dgfx_exchange_serve(const void* const* d_exchanges, int32_t world, int32_t rank, int64_t slot_rows,
                                   int64_t rows_per_rank, int64_t row_bytes, const void* d_table, int64_t local_rows,
                                   const void* d_replica, int64_t replica_rows, const int32_t* d_req_pos, void* d_out,
                                   dgfx_stream stream_) {
  if (d_exchanges == nullptr || !ex_args_ok(world, slot_rows, row_bytes) || rank < 0 || rank >= world ||
      rows_per_rank < 1 || local_rows < 0 || (local_rows > 0 && d_table == nullptr) || d_req_pos == nullptr ||
      replica_rows < 0 || (replica_rows > 0 && d_replica == nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_serve: bad arguments");
  }
  return launch_exchange_copy(true, d_exchanges, world, rank, slot_rows, row_bytes, d_table,
                              static_cast<int64_t>(rank) * rows_per_rank, local_rows, d_replica, replica_rows,
                              d_req_pos, d_out, reinterpret_cast<cudaStream_t>(stream_));
}

extern "C" int dgfx_exchange_scatter(const void* const* d_exchanges, int32_t world, int32_t rank, int64_t slot_rows,
                                     int64_t row_bytes, const int32_t* d_req_pos, void* d_out, dgfx_stream stream_) {
  if (d_exchanges == nullptr || !ex_args_ok(world, slot_rows, row_bytes) || rank < 0 || rank >= world ||
      d_req_pos == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_scatter: bad arguments");
  }
  if (world == 1) return DGFX_OK;
  return launch_exchange_copy(false, d_exchanges, world, rank, slot_rows, row_bytes, nullptr, 0, 0, nullptr, 0,
                              d_req_pos, d_out, reinterpret_cast<cudaStream_t>(stream_));
}

extern "C" int dgfx_exchange_barrier(const void* const* d_exchanges, int32_t world, int32_t rank, uint32_t epoch,
                                     uint64_t max_wait_ns, dgfx_stream stream_) {
  if (d_exchanges == nullptr || world < 1 || world > kMaxWorld || rank < 0 || rank >= world) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_barrier: bad arguments");
  }
  exchange_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      reinterpret_cast<const char* const*>(d_exchanges), world, rank, epoch, max_wait_ns);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

extern "C" int dgfx_exchange_gather(const void* const* d_exchanges, void* d_exchange, int32_t world, int32_t rank,
                                    int64_t slot_rows, int64_t rows_per_rank, int64_t num_nodes, int64_t row_bytes,
                                    const int64_t* d_row_ids, const int64_t* d_begin, const int64_t* d_end,
                                    int64_t max_rows, const int32_t* d_hot_slot, int32_t* d_req_pos,
                                    const void* d_table, int64_t local_rows, const void* d_replica,
                                    int64_t replica_rows, void* d_out, uint32_t epoch, uint64_t max_wait_ns,
                                    dgfx_stream stream) {
  DGFX_TRY(dgfx_exchange_partition(d_exchange, world, slot_rows, rows_per_rank, num_nodes, row_bytes, d_row_ids,
                                   d_begin, d_end, max_rows, d_hot_slot, d_req_pos, d_out, stream));
  DGFX_TRY(dgfx_exchange_barrier(d_exchanges, world, rank, epoch, max_wait_ns, stream));
  DGFX_TRY(dgfx_exchange_serve(d_exchanges, world, rank, slot_rows, rows_per_rank, row_bytes, d_table, local_rows,
                               d_replica, replica_rows, d_req_pos, d_out, stream));
  uint32_t next = epoch == 0 ? 0 : epoch + 1;  // 0: both barriers take the device epoch
  if (next > 0x7FFFFFFFu) next = 1;
  DGFX_TRY(dgfx_exchange_barrier(d_exchanges, world, rank, next, max_wait_ns, stream));
  return dgfx_exchange_scatter(d_exchanges, world, rank, slot_rows, row_bytes, d_req_pos, d_out, stream);
}

extern "C" int dgfx_exchange_check(const void* d_exchange, int32_t world, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (d_exchange == nullptr || world < 1 || world > kMaxWorld) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_exchange_check: bad arguments");
  }
  uint32_t flag = 0;
  char* status = const_cast<char*>(static_cast<const char*>(d_exchange)) + kExStatusOff;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&flag, status, sizeof(flag), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (flag != 0) {
    DGFX_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(flag), stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
    if (flag & 2u) {
      return fail(DGFX_ERR_FAILED_PRECONDITION,
                  "dgfx_exchange: a barrier wait timed out (a rank did not arrive); rows of that step are invalid");
    }
    return fail(DGFX_ERR_WORKSPACE, "dgfx_exchange: a request slot overflowed (slot_rows too small); rows were dropped");
  }
  return DGFX_OK;
}

extern "C" int dgfx_device_alloc(size_t bytes, void** d_ptr) {
  if (d_ptr == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_device_alloc: null output");
  *d_ptr = nullptr;
  DGFX_CUDA_TRY(cudaMalloc(d_ptr, bytes == 0 ? 256 : bytes));
  return DGFX_OK;
}

extern "C" int dgfx_device_free(void* d_ptr) {
  if (d_ptr != nullptr) DGFX_CUDA_TRY(cudaFree(d_ptr));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_get_handle(const void* d_ptr, void* handle64) {
  if (d_ptr == nullptr || handle64 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_ipc_get_handle: null");
  cudaIpcMemHandle_t h;
  DGFX_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(d_ptr)));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_open(const void* handle64, void** d_ptr) {
  if (d_ptr == nullptr || handle64 == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_ipc_open: null");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  *d_ptr = nullptr;
  DGFX_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return DGFX_OK;
}

extern "C" int dgfx_ipc_close(void* d_ptr) {
  if (d_ptr != nullptr) DGFX_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr));
  return DGFX_OK;
}

extern "C" int dgfx_gather_rows_p2p(const void* const* d_tables, int32_t world, int64_t rows_per_rank,
                                    int64_t num_nodes, int64_t row_bytes, const int64_t* d_row_ids,
                                    const int64_t* d_begin, const int64_t* d_end, int64_t max_rows, void* d_out,
                                    dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (d_tables == nullptr || world < 1 || rows_per_rank < 1 || num_nodes < 0 || row_bytes <= 0 ||
      row_bytes % 16 != 0 || max_rows < 0 || d_begin == nullptr || d_end == nullptr) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_gather_rows_p2p: bad arguments");
  }
  if (max_rows == 0) return DGFX_OK;
  if (num_nodes >= (int64_t(1) << 32) || rows_per_rank >= (int64_t(1) << 32)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_gather_rows_p2p: more than 2^32 - 1 nodes");
  }
  const int64_t vpr = row_bytes / 16;
  int lvpr = -1;
  for (int b = 0; b < 31; ++b) {
    if ((int64_t(1) << b) == vpr) lvpr = b;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int U = 3;
  const int64_t blocks =
      std::min<int64_t>(ceil_div(max_rows * vpr, kGatherThreads * U), static_cast<int64_t>(sms) * 24);
  gather_p2p_kernel<U><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), kGatherThreads, 0, stream>>>(
      reinterpret_cast<const uint4* const*>(d_tables), world, static_cast<uint32_t>(rows_per_rank),
      static_cast<uint32_t>(num_nodes), vpr, lvpr, d_row_ids, d_begin, d_end, max_rows, static_cast<uint4*>(d_out));
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}
