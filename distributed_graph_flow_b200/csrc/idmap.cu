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
// match. A byte id hashes as its little-endian 32-bit words (zero padded)
// folded by multiply-xorshift, then the SplitMix64 finaliser (Steele, Lea,
// Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014),
// which also hashes integer ids. Ids are read where they lie: int64 arrays,
// fixed-width byte rows (numpy 'S' arrays; rows of a multiple of 4 bytes are
// read a word at a time) or Arrow binary columns (int64 offsets + bytes). Dangling-edge removal is a stable
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
  int32_t words;           // fixed-width rows of a multiple of 4 bytes on a 4-byte boundary: read as 32-bit words
  int64_t width;           // DGFX_IDS_FIXED: bytes per id
  const int64_t* ints;     // DGFX_IDS_INT64
  const uint8_t* bytes;    // DGFX_IDS_FIXED / DGFX_IDS_VAR
  const int64_t* offsets;  // DGFX_IDS_VAR: [n + 1]
};

// Byte id i as (first byte, length without trailing zero bytes).
__device__ __forceinline__ void id_span(const KeysDev& k, int64_t i, int64_t* start, int64_t* len) {
  if (k.words) {
    const uint32_t* row = reinterpret_cast<const uint32_t*>(k.bytes + i * k.width);
    int64_t L = 0;
    for (int64_t j = k.width / 4 - 1; j >= 0; --j) {
      const uint32_t w = row[j];
      if (w != 0) {
        L = 4 * j + (39 - __clz(w)) / 8;  // bytes up to the highest non-zero one (little-endian)
        break;
      }
    }
    *start = i * k.width;
    *len = L;
    return;
  }
  int64_t b, e;
  if (k.kind == DGFX_IDS_FIXED) {
    b = i * k.width;
    e = b + k.width;
  } else {
    b = k.offsets[i];
    e = k.offsets[i + 1];
  }
  while (e > b && k.bytes[e - 1] == 0) --e;  // trailing zero bytes are not part of the id
  *start = b;
  *len = e - b;
}

// Little-endian 32-bit word j of an id (bytes past its length read as zero;
// in a fixed-width row they are zero already).
__device__ __forceinline__ uint32_t id_word(const KeysDev& k, int64_t start, int64_t len, int64_t j) {
  if (k.words) return reinterpret_cast<const uint32_t*>(k.bytes + start)[j];
  uint32_t w = 0;
  const int64_t b = 4 * j;
  for (int t = 0; t < 4 && b + t < len; ++t) w |= static_cast<uint32_t>(k.bytes[start + b + t]) << (8 * t);
  return w;
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// Hash of a byte id: its 32-bit words folded by multiply-xorshift, then the
// SplitMix64 finaliser; identical for every storage layout of the same id.
__device__ __forceinline__ uint64_t hash_span(const KeysDev& k, int64_t start, int64_t len) {
  uint64_t h = 0x9E3779B97F4A7C15ull ^ static_cast<uint64_t>(len);
  const int64_t nw = (len + 3) / 4;
  for (int64_t j = 0; j < nw; ++j) {
    h = (h ^ id_word(k, start, len, j)) * 0x9E3779B97F4A7C15ull;
    h ^= h >> 29;
  }
  return mix64(h);
}

__device__ __forceinline__ bool same_span(const KeysDev& a, int64_t sa, int64_t la, const KeysDev& b, int64_t sb,
                                          int64_t lb) {
  if (la != lb) return false;
  const int64_t nw = (la + 3) / 4;
  for (int64_t j = 0; j < nw; ++j) {
    if (id_word(a, sa, la, j) != id_word(b, sb, lb, j)) return false;
  }
  return true;
}

// An id in registers: its hash and, for byte ids, its span.
struct IdRef {
  uint64_t hash;
  int64_t start, len, value;
};

__device__ __forceinline__ IdRef load_id(const KeysDev& k, int64_t i) {
  IdRef r{};
  if (k.kind == DGFX_IDS_INT64) {
    r.value = k.ints[i];
    r.hash = mix64(static_cast<uint64_t>(r.value));
    return r;
  }
  id_span(k, i, &r.start, &r.len);
  r.hash = hash_span(k, r.start, r.len);
  return r;
}

// Index id `idx` equals the id `r` (read from layout `q`).
__device__ __forceinline__ bool matches(const KeysDev& keys, int64_t idx, const KeysDev& q, const IdRef& r) {
  if (keys.kind == DGFX_IDS_INT64) return keys.ints[idx] == r.value;
  int64_t s, l;
  id_span(keys, idx, &s, &l);
  return same_span(keys, s, l, q, r.start, r.len);
}

__global__ void id_index_build_kernel(KeysDev keys, int64_t n, unsigned long long* table, uint64_t mask,
                                      unsigned long long* full) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const IdRef r = load_id(keys, i);
    const uint64_t h = r.hash;
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
      if ((w >> 32) == (word >> 32) && matches(keys, static_cast<uint32_t>(w), keys, r)) {
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
    const IdRef r = load_id(q, i);
    const uint64_t h = r.hash;
    const uint32_t tag = static_cast<uint32_t>(h >> 32);
    uint64_t s = h & mask;
    int64_t found = -1;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
      const unsigned long long w = table[s];
      if (w == kEmptyWord) break;
      if (static_cast<uint32_t>(w >> 32) == tag && matches(keys, static_cast<uint32_t>(w), q, r)) {
        found = static_cast<uint32_t>(w);
        break;
      }
      s = (s + 1) & mask;
    }
    out[i] = found;
    if (found < 0) atomicMax(mismatch, static_cast<unsigned long long>(i + 1));
  }
}

// Fixed-width rows of NW 32-bit words on both sides, the same width: two ids
// are equal exactly when their rows are (both zero padded), so the row stays
// in registers, its length and hash are computed unrolled (the same values as
// id_span / hash_span), and a tag match compares the key row word by word.
constexpr int kMaxRowWords = 8;

template <int NW>
__device__ __forceinline__ void load_row(const uint32_t* __restrict__ base, int64_t i, uint32_t (&w)[NW]) {
  const uint32_t* r = base + i * NW;
#pragma unroll
  for (int j = 0; j < NW; ++j) w[j] = __ldg(r + j);
}

template <int NW>
__device__ __forceinline__ uint64_t hash_row(const uint32_t (&w)[NW]) {
  int len = 0;  // bytes up to the highest non-zero one (little-endian words)
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    if (w[j] != 0) len = 4 * j + (39 - __clz(w[j])) / 8;
  }
  uint64_t h = 0x9E3779B97F4A7C15ull ^ static_cast<uint64_t>(len);
  const int nw = (len + 3) / 4;
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    if (j < nw) {
      h = (h ^ w[j]) * 0x9E3779B97F4A7C15ull;
      h ^= h >> 29;
    }
  }
  return mix64(h);
}

template <int NW>
__device__ __forceinline__ bool row_equals(const uint32_t* __restrict__ keys, uint32_t idx, const uint32_t (&w)[NW]) {
  const uint32_t* k = keys + static_cast<int64_t>(idx) * NW;
  bool eq = true;
#pragma unroll
  for (int j = 0; j < NW; ++j) eq &= __ldg(k + j) == w[j];
  return eq;
}

template <int NW>
__global__ void id_index_build_rows_kernel(const uint32_t* __restrict__ keys, int64_t n, unsigned long long* table,
                                           uint64_t mask, unsigned long long* full) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    uint32_t w[NW];
    load_row<NW>(keys, i, w);
    const uint64_t h = hash_row<NW>(w);
    const unsigned long long word = (static_cast<unsigned long long>(h >> 32) << 32) | static_cast<uint32_t>(i);
    uint64_t s = h & mask;
    bool placed = false;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
      unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(&table[s]);
      if (e == kEmptyWord) {
        const unsigned long long prev = atomicCAS(&table[s], kEmptyWord, word);
        if (prev == kEmptyWord) {
          placed = true;
          break;
        }
        e = prev;
      }
      if ((e >> 32) == (word >> 32) && row_equals<NW>(keys, static_cast<uint32_t>(e), w)) {
        atomicMax(&table[s], word);  // equal ids: the later position wins
        placed = true;
        break;
      }
      s = (s + 1) & mask;
    }
    if (!placed) atomicAdd(full, 1ull);
  }
}

template <int NW>
__global__ void id_index_lookup_rows_kernel(const uint32_t* __restrict__ keys, const unsigned long long* table,
                                            uint64_t mask, const uint32_t* __restrict__ q, int64_t n, int64_t* out,
                                            unsigned long long* mismatch) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    uint32_t w[NW];
    load_row<NW>(q, i, w);
    const uint64_t h = hash_row<NW>(w);
    const uint32_t tag = static_cast<uint32_t>(h >> 32);
    uint64_t s = h & mask;
    int64_t found = -1;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
      const unsigned long long e = table[s];
      if (e == kEmptyWord) break;
      if (static_cast<uint32_t>(e >> 32) == tag && row_equals<NW>(keys, static_cast<uint32_t>(e), w)) {
        found = static_cast<uint32_t>(e);
        break;
      }
      s = (s + 1) & mask;
    }
    out[i] = found;
    if (found < 0) atomicMax(mismatch, static_cast<unsigned long long>(i + 1));
  }
}

// Row words of a fixed-width layout read word by word, 0 otherwise.
int row_words(const KeysDev& k) {
  if (k.kind != DGFX_IDS_FIXED || !k.words) return 0;
  const int64_t nw = k.width / 4;
  return nw >= 1 && nw <= kMaxRowWords ? static_cast<int>(nw) : 0;
}

#define DGFX_ROW_WORDS_CASES(X) X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8)

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
  k->words = 0;
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
      k->words = (width % 4 == 0 && reinterpret_cast<uintptr_t>(d_ids) % 4 == 0) ? 1 : 0;
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
  bool owned = false;                   // allocated here (no caller table)
};

namespace {
uint64_t table_capacity(int64_t num_ids) {
  uint64_t cap = 1024;
  while (cap < static_cast<uint64_t>(2 * num_ids)) cap <<= 1;
  return cap;
}
}  // namespace

extern "C" int dgfx_id_index_table_bytes(int64_t num_ids, size_t* bytes) {
  if (bytes == nullptr || num_ids < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_id_index_table_bytes: bad arguments");
  *bytes = (table_capacity(num_ids) + 2) * sizeof(unsigned long long);
  return DGFX_OK;
}

extern "C" int dgfx_id_index_create(int32_t kind, const void* d_ids, const int64_t* d_offsets, int64_t width,
                                    int64_t num_ids, void* d_table, size_t table_bytes, dgfx_stream stream_,
                                    dgfx_id_index** out) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (out == nullptr || num_ids < 0) return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_id_index_create: bad arguments");
  *out = nullptr;
  if (num_ids >= (int64_t(1) << 31)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_id_index_create: more than 2^31 - 1 ids in one node set");
  }
  auto ix = std::make_unique<dgfx_id_index>();
  DGFX_TRY(make_keys(kind, d_ids, d_offsets, width, num_ids, &ix->keys, "dgfx_id_index_create"));
  ix->n = num_ids;
  const uint64_t cap = table_capacity(num_ids);
  ix->mask = cap - 1;
  const size_t need = (cap + 2) * sizeof(unsigned long long);
  if (d_table != nullptr) {
    if (table_bytes < need || reinterpret_cast<uintptr_t>(d_table) % 8 != 0) {
      return fail(DGFX_ERR_WORKSPACE, "dgfx_id_index_create: table memory too small or not 8-byte aligned");
    }
    ix->table = static_cast<unsigned long long*>(d_table);
  } else {
    DGFX_CUDA_TRY(cudaMalloc(&ix->table, need));
    ix->owned = true;
  }
  DGFX_CUDA_TRY(cudaMemsetAsync(ix->table, 0xFF, cap * sizeof(unsigned long long), stream));
  DGFX_CUDA_TRY(cudaMemsetAsync(ix->table + cap, 0, 2 * sizeof(unsigned long long), stream));
  if (num_ids > 0) {
    const auto* rows = reinterpret_cast<const uint32_t*>(ix->keys.bytes);
    switch (row_words(ix->keys)) {
#define DGFX_BUILD_ROWS(NW)                                                                                   \
  case NW:                                                                                                    \
    id_index_build_rows_kernel<NW><<<grid_for(num_ids), kThreads, 0, stream>>>(rows, num_ids, ix->table,      \
                                                                                ix->mask, ix->table + cap); \
    break;
      DGFX_ROW_WORDS_CASES(DGFX_BUILD_ROWS)
#undef DGFX_BUILD_ROWS
      default:
        id_index_build_kernel<<<grid_for(num_ids), kThreads, 0, stream>>>(ix->keys, num_ids, ix->table, ix->mask,
                                                                          ix->table + cap);
    }
    DGFX_CUDA_TRY(cudaGetLastError());
  }
  unsigned long long full = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&full, ix->table + cap, sizeof(full), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (full != 0) {
    if (ix->owned) cudaFree(ix->table);
    ix->table = nullptr;
    return fail(DGFX_ERR_INTERNAL, "dgfx_id_index_create: id table full");
  }
  *out = ix.release();
  return DGFX_OK;
}

extern "C" void dgfx_id_index_destroy(dgfx_id_index* ix) {
  if (ix == nullptr) return;
  if (ix->owned && ix->table != nullptr) cudaFree(ix->table);
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
    const int nw = row_words(q) == row_words(ix->keys) && q.width == ix->keys.width ? row_words(q) : 0;
    const auto* krows = reinterpret_cast<const uint32_t*>(ix->keys.bytes);
    const auto* qrows = reinterpret_cast<const uint32_t*>(q.bytes);
    switch (nw) {
#define DGFX_LOOKUP_ROWS(NW)                                                                                       \
  case NW:                                                                                                         \
    id_index_lookup_rows_kernel<NW><<<grid_for(num_ids), kThreads, 0, stream>>>(krows, ix->table, ix->mask, qrows, \
                                                                                 num_ids, d_out, mm);              \
    break;
      DGFX_ROW_WORDS_CASES(DGFX_LOOKUP_ROWS)
#undef DGFX_LOOKUP_ROWS
      default:
        id_index_lookup_kernel<<<grid_for(num_ids), kThreads, 0, stream>>>(ix->keys, ix->table, ix->mask, q, num_ids,
                                                                           d_out, mm);
    }
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
