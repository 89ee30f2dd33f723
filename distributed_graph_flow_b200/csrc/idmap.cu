// Raw node id -> node index mapping on the device (sm_100a).
//
// Replaces ByteIdToIdxMapper / PairMapping (dgf/src/io/io_ext.cc:26-170) and
// the integer-id dictionary of _read_node_set (dgf/src/io/graph_in_memory.py:
// 80-125), which turn the raw ids of a GF graph's edge endpoints into 0-based
// node indices when the graph is loaded. Semantics kept: a byte id is its
// bytes without trailing zero bytes (NumpyBytesArray::operator[],
// dgf/src/util/nanobind_util.cc:70-73), so the same id stored with different
// widths or with zero padding matches; when a node set lists an id twice the
// last position wins (the reference's map assignment in index order); an id
// that is not in the index maps to -1, and the reported mismatch is the
// largest position of such an id (the last one, as the single-threaded
// mapper reports).
//
// Design. An open-addressing table of 64-bit words (hash tag << 32 | node
// index), capacity a power of two >= 2n, built by one thread per node id
// (CAS into an empty slot; a slot holding an equal id keeps the larger index
// through atomicMax, since equal ids carry equal tags) and probed by one
// thread per query, comparing tags first and the id bytes only on a tag
// match. Hashes: FNV-1a 64 over the id bytes (Fowler, Noll, Vo), the
// SplitMix64 finaliser for integer ids (Steele, Lea, Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014). Ids are read where they lie:
// int64 arrays, fixed-width byte rows (numpy 'S' arrays) or Arrow binary
// columns (int64 offsets + bytes). Dangling-edge removal is a stable
// compaction (flag, scan, scatter) that also returns the kept edges'
// positions so edge features can be filtered with them.
#include <memory>
#include <string>

#include "common.cuh"
#include "primitives.cuh"

namespace dgfx {
namespace {

constexpr unsigned long long kEmptyWord = ~0ull;
constexpr int kThreads = 256;

struct KeysDev {
  int32_t kind;
  int64_t width;           // DGFX_IDS_FIXED: bytes per id
  const int64_t* ints;     // DGFX_IDS_INT64
  const uint8_t* bytes;    // DGFX_IDS_FIXED / DGFX_IDS_VAR
  const int64_t* offsets;  // DGFX_IDS_VAR: [n + 1]
};

__device__ __forceinline__ void id_bytes(const KeysDev& k, int64_t i, const uint8_t** p, int64_t* len) {
  int64_t b, e;
  if (k.kind == DGFX_IDS_FIXED) {
    b = i * k.width;
    e = b + k.width;
  } else {
    b = k.offsets[i];
    e = k.offsets[i + 1];
  }
  while (e > b && k.bytes[e - 1] == 0) --e;  // trailing zero bytes are not part of the id
  *p = k.bytes + b;
  *len = e - b;
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

__device__ __forceinline__ uint64_t hash_bytes(const uint8_t* p, int64_t len) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (int64_t j = 0; j < len; ++j) {
    h ^= p[j];
    h *= 0x100000001b3ull;
  }
  return mix64(h);  // spread FNV's low bits over the slot index
}

__device__ __forceinline__ uint64_t hash_id(const KeysDev& k, int64_t i) {
  if (k.kind == DGFX_IDS_INT64) return mix64(static_cast<uint64_t>(k.ints[i]));
  const uint8_t* p;
  int64_t len;
  id_bytes(k, i, &p, &len);
  return hash_bytes(p, len);
}

// Id a[i] == id b[j] (both of the same family: integers or bytes).
__device__ __forceinline__ bool same_id(const KeysDev& a, int64_t i, const KeysDev& b, int64_t j) {
  if (a.kind == DGFX_IDS_INT64) return a.ints[i] == b.ints[j];
  const uint8_t *pa, *pb;
  int64_t la, lb;
  id_bytes(a, i, &pa, &la);
  id_bytes(b, j, &pb, &lb);
  if (la != lb) return false;
  for (int64_t t = 0; t < la; ++t) {
    if (pa[t] != pb[t]) return false;
  }
  return true;
}

__global__ void id_index_build_kernel(KeysDev keys, int64_t n, unsigned long long* table, uint64_t mask,
                                      unsigned long long* full) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t h = hash_id(keys, i);
    const unsigned long long word = (static_cast<unsigned long long>(h >> 32) << 32) | static_cast<uint32_t>(i);
    uint64_t s = h & mask;
    bool placed = false;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
      unsigned long long w = *reinterpret_cast<volatile unsigned long long*>(&table[s]);
      if (w == kEmptyWord) {
        const unsigned long long prev = atomicCAS(&table[s], kEmptyWord, word);
        if (prev == kEmptyWord) {
          placed = true;
          break;
        }
        w = prev;
      }
      if ((w >> 32) == (word >> 32) && same_id(keys, static_cast<uint32_t>(w), keys, i)) {
        atomicMax(&table[s], word);  // equal ids: the later position wins
        placed = true;
        break;
      }
      s = (s + 1) & mask;
    }
    if (!placed) atomicAdd(full, 1ull);
  }
}

__global__ void id_index_lookup_kernel(KeysDev keys, const unsigned long long* table, uint64_t mask, KeysDev q,
                                       int64_t n, int64_t* out, unsigned long long* mismatch) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t h = hash_id(q, i);
    const uint32_t tag = static_cast<uint32_t>(h >> 32);
    uint64_t s = h & mask;
    int64_t found = -1;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
      const unsigned long long w = table[s];
      if (w == kEmptyWord) break;
      if (static_cast<uint32_t>(w >> 32) == tag && same_id(keys, static_cast<uint32_t>(w), q, i)) {
        found = static_cast<uint32_t>(w);
        break;
      }
      s = (s + 1) & mask;
    }
    out[i] = found;
    if (found < 0) atomicMax(mismatch, static_cast<unsigned long long>(i + 1));
  }
}

__global__ void pair_keep_kernel(const int64_t* src, const int64_t* dst, int64_t n, int32_t* keep) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    keep[i] = (src[i] >= 0 && dst[i] >= 0) ? 1 : 0;
  }
}

__global__ void pair_scatter_kernel(const int64_t* src, const int64_t* dst, int64_t n, const int64_t* pos,
                                    int64_t* out_src, int64_t* out_dst, int64_t* out_pos) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    if (src[i] >= 0 && dst[i] >= 0) {
      const int64_t o = pos[i];
      out_src[o] = src[i];
      out_dst[o] = dst[i];
      if (out_pos != nullptr) out_pos[o] = i;
    }
  }
}

unsigned grid_for(int64_t n) {
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kThreads), 148 * 16)));
}

int make_keys(int32_t kind, const void* d_ids, const int64_t* d_offsets, int64_t width, int64_t n, KeysDev* k,
              const char* what) {
  k->kind = kind;
  k->width = width;
  k->ints = nullptr;
  k->bytes = nullptr;
  k->offsets = nullptr;
  if (n > 0 && d_ids == nullptr && !(kind == DGFX_IDS_VAR && d_offsets != nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, std::string(what) + ": null ids");
  }
  switch (kind) {
    case DGFX_IDS_INT64:
      k->ints = static_cast<const int64_t*>(d_ids);
      return DGFX_OK;
    case DGFX_IDS_FIXED:
      if (width < 1) return fail(DGFX_ERR_INVALID_ARGUMENT, std::string(what) + ": id width must be >= 1");
      k->bytes = static_cast<const uint8_t*>(d_ids);
      return DGFX_OK;
    case DGFX_IDS_VAR:
      if (d_offsets == nullptr) return fail(DGFX_ERR_INVALID_ARGUMENT, std::string(what) + ": null offsets");
      k->bytes = static_cast<const uint8_t*>(d_ids);
      k->offsets = d_offsets;
      return DGFX_OK;
    default:
      return fail(DGFX_ERR_INVALID_ARGUMENT, std::string(what) + ": unknown id kind");
  }
}

}  // namespace
}  // namespace dgfx

using namespace dgfx;

struct dgfx_id_index {
  KeysDev keys{};
  int64_t n = 0;
  uint64_t mask = 0;
  unsigned long long* table = nullptr;  // [mask + 1] words, then 2 status words
};

extern "C" int dgfx_id_index_create(int32_t kind, const void* d_ids, const int64_t* d_offsets, int64_t width,
                                    int64_t num_ids, dgfx_stream stream_, dgfx_id_index** out) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (out == nullptr || num_ids < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_id_index_create: bad arguments");
  *out = nullptr;
  if (num_ids >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_id_index_create: more than 2^31 - 1 ids in one node set");
  }
  auto ix = std::make_unique<dgfx_id_index>();
  DGFX_TRY(make_keys(kind, d_ids, d_offsets, width, num_ids, &ix->keys, "dgfx_id_index_create"));
  ix->n = num_ids;
  uint64_t cap = 1024;
  while (cap < static_cast<uint64_t>(2 * num_ids)) cap <<= 1;
  ix->mask = cap - 1;
  DGFX_CUDA_TRY(cudaMalloc(&ix->table, (cap + 2) * sizeof(unsigned long long)));
  DGFX_CUDA_TRY(cudaMemsetAsync(ix->table, 0xFF, cap * sizeof(unsigned long long), stream));
  DGFX_CUDA_TRY(cudaMemsetAsync(ix->table + cap, 0, 2 * sizeof(unsigned long long), stream));
  if (num_ids > 0) {
    id_index_build_kernel<<<grid_for(num_ids), kThreads, 0, stream>>>(ix->keys, num_ids, ix->table, ix->mask,
                                                                      ix->table + cap);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  unsigned long long full = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&full, ix->table + cap, sizeof(full), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (full != 0) {
    cudaFree(ix->table);
    ix->table = nullptr;
    return fail(DGFX_ERR_INTERNAL, "dgfx_id_index_create: id table full");
  }
  *out = ix.release();
  return DGFX_OK;
}

extern "C" void dgfx_id_index_destroy(dgfx_id_index* ix) {
  if (ix == nullptr) return;
  if (ix->table != nullptr) cudaFree(ix->table);
  delete ix;
}

extern "C" int dgfx_id_index_lookup(const dgfx_id_index* ix, int32_t kind, const void* d_ids,
                                    const int64_t* d_offsets, int64_t width, int64_t num_ids, int64_t* d_out,
                                    int64_t* mismatch, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (ix == nullptr || num_ids < 0 || (num_ids > 0 && d_out == nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_id_index_lookup: bad arguments");
  }
  KeysDev q;
  DGFX_TRY(make_keys(kind, d_ids, d_offsets, width, num_ids, &q, "dgfx_id_index_lookup"));
  if ((q.kind == DGFX_IDS_INT64) != (ix->keys.kind == DGFX_IDS_INT64)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_id_index_lookup: integer ids against byte ids (or the reverse)");
  }
  unsigned long long* mm = ix->table + ix->mask + 2;
  DGFX_CUDA_TRY(cudaMemsetAsync(mm, 0, sizeof(unsigned long long), stream));
  if (num_ids > 0) {
    id_index_lookup_kernel<<<grid_for(num_ids), kThreads, 0, stream>>>(ix->keys, ix->table, ix->mask, q, num_ids,
                                                                       d_out, mm);
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  if (mismatch != nullptr) {
    unsigned long long m = 0;
    DGFX_CUDA_TRY(cudaMemcpyAsync(&m, mm, sizeof(m), cudaMemcpyDeviceToHost, stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
    *mismatch = static_cast<int64_t>(m) - 1;
  }
  return DGFX_OK;
}

extern "C" int dgfx_compact_pairs_workspace_size(int64_t num_pairs, size_t* bytes) {
  if (bytes == nullptr || num_pairs < 0) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_compact_pairs_workspace_size: bad arguments");
  }
  Arena a(nullptr, 0);
  a.take<int32_t>(static_cast<size_t>(num_pairs) + 1);
  a.take<int64_t>(static_cast<size_t>(num_pairs) + 1);
  *bytes = a.used + scan_workspace_bytes(num_pairs + 1) + 1024;
  return DGFX_OK;
}

extern "C" int dgfx_compact_pairs(const int64_t* d_src, const int64_t* d_dst, int64_t num_pairs, int64_t* d_out_src,
                                  int64_t* d_out_dst, int64_t* d_out_pos, int64_t* num_kept, void* d_workspace,
                                  size_t workspace_bytes, dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (num_pairs < 0 || num_kept == nullptr ||
      (num_pairs > 0 && (d_src == nullptr || d_dst == nullptr || d_out_src == nullptr || d_out_dst == nullptr))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_compact_pairs: bad arguments");
  }
  *num_kept = 0;
  if (num_pairs == 0) return DGFX_OK;
  Arena a(d_workspace, workspace_bytes);
  int32_t* keep = a.take<int32_t>(static_cast<size_t>(num_pairs) + 1);
  int64_t* pos = a.take<int64_t>(static_cast<size_t>(num_pairs) + 1);
  if (!a.ok()) return fail(DGFX_ERR_WORKSPACE, "dgfx_compact_pairs: workspace too small");
  pair_keep_kernel<<<grid_for(num_pairs), kThreads, 0, stream>>>(d_src, d_dst, num_pairs, keep);
  DGFX_CUDA_TRY(cudaGetLastError());
  DGFX_TRY(exclusive_scan<int32_t>(keep, pos, num_pairs, true, a, stream));
  pair_scatter_kernel<<<grid_for(num_pairs), kThreads, 0, stream>>>(d_src, d_dst, num_pairs, pos, d_out_src,
                                                                    d_out_dst, d_out_pos);
  DGFX_CUDA_TRY(cudaGetLastError());
  DGFX_CUDA_TRY(cudaMemcpyAsync(num_kept, pos + num_pairs, sizeof(int64_t), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  return DGFX_OK;
}
