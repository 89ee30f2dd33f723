// ORACLE — test and baseline infrastructure only (see grow.h).
//
// CPU restatement of the library's seeded synthetic generators
// (distributed_graph_flow_b200/csrc/synth.cu), so that the CPU baseline of
// the benchmark builds the same graphs, seeds and features on the host with
// no GPU involved. Every integer output (row pointers, edge endpoints,
// uniform integers) equals the device generator's bit for bit: both run
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) on the same counters,
// draw power-law degrees through the same table of thresholds k^-(alpha-1)
// (computed on the host by the same std::pow), and multiply doubles in the
// same order. Normal features use the Box-Muller transform with the host's
// log / sqrt / cos / sin, which may differ from the device's in the last
// bit of the double before rounding to fp32 / bf16.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace dgf_synth {

struct U4 {
  std::uint32_t x, y, z, w;
};

inline U4 philox4x32_10(U4 c, std::uint32_t k0, std::uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const std::uint64_t p0 = static_cast<std::uint64_t>(0xD2511F53u) * c.x;
    const std::uint64_t p1 = static_cast<std::uint64_t>(0xCD9E8D57u) * c.z;
    c = U4{static_cast<std::uint32_t>(p1 >> 32) ^ c.y ^ k0, static_cast<std::uint32_t>(p1),
           static_cast<std::uint32_t>(p0 >> 32) ^ c.w ^ k1, static_cast<std::uint32_t>(p0)};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

inline double u01(std::uint32_t hi, std::uint32_t lo) {
  const std::uint64_t x = (static_cast<std::uint64_t>(hi) << 32 | lo) >> 11;
  return static_cast<double>(x) * (1.0 / 9007199254740992.0);
}

inline std::uint64_t bounded64(std::uint64_t r, std::uint64_t range) {
  return static_cast<std::uint64_t>((static_cast<unsigned __int128>(r) * range) >> 64);
}

// Runs fn(lo, hi) over [0, n) split into `threads` contiguous blocks.
template <class F>
void parallel_blocks(std::int64_t n, int threads, F&& fn) {
  threads = std::max(1, threads);
  if (threads == 1 || n < 4096) {
    fn(std::int64_t(0), n);
    return;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const std::int64_t lo = n * t / threads, hi = n * (t + 1) / threads;
    pool.emplace_back([&fn, lo, hi]() { fn(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

// thr[k - 1] = k^-(alpha - 1), k = 1 .. max_degree (the device generator
// receives the same table).
inline std::vector<double> degree_thresholds(double alpha, std::int64_t max_degree) {
  std::vector<double> thr(static_cast<std::size_t>(max_degree));
  for (std::int64_t k = 1; k <= max_degree; ++k) thr[k - 1] = std::pow(static_cast<double>(k), -(alpha - 1.0));
  return thr;
}

// Degree of a node with uniform u in (0, 1]: the largest k <= max_degree
// with thr[k - 1] >= u (that is, floor(u^(-1/(alpha-1))) capped).
inline std::int64_t degree_of(const double* thr, std::int64_t max_degree, double u) {
  std::int64_t lo = 1, hi = max_degree;
  while (lo < hi) {
    const std::int64_t mid = (lo + hi + 1) >> 1;
    if (thr[mid - 1] >= u) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Row pointers int64[n_src + 1] of the power-law graph.
inline void graph_rowptr(std::int64_t n_src, std::int64_t num_edges, double alpha, std::int64_t max_degree,
                         std::uint64_t seed, std::int64_t* rowptr, int threads) {
  const std::uint32_t k0 = static_cast<std::uint32_t>(seed), k1 = static_cast<std::uint32_t>(seed >> 32);
  const std::vector<double> thr = degree_thresholds(alpha, max_degree);
  // Raw degrees, then an exclusive prefix (blocked: per-block sums first).
  threads = std::max(1, threads);
  std::vector<std::int64_t> block_sum(threads + 1, 0);
  std::vector<std::thread> pool;
  auto raw = [&](std::int64_t v) {
    const U4 r = philox4x32_10(U4{static_cast<std::uint32_t>(v), static_cast<std::uint32_t>(v >> 32), 0x5eedu, 1u},
                               k0, k1);
    return degree_of(thr.data(), max_degree, 1.0 - u01(r.x, r.y));
  };
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t]() {
      const std::int64_t lo = n_src * t / threads, hi = n_src * (t + 1) / threads;
      std::int64_t s = 0;
      for (std::int64_t v = lo; v < hi; ++v) {
        const std::int64_t d = raw(v);
        rowptr[v] = d;
        s += d;
      }
      block_sum[t + 1] = s;
    });
  }
  for (auto& th : pool) th.join();
  pool.clear();
  for (int t = 0; t < threads; ++t) block_sum[t + 1] += block_sum[t];
  const std::int64_t S = block_sum[threads];
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t]() {
      const std::int64_t lo = n_src * t / threads, hi = n_src * (t + 1) / threads;
      std::int64_t c = block_sum[t];
      for (std::int64_t v = lo; v < hi; ++v) {
        const std::int64_t d = rowptr[v];
        rowptr[v] = S == 0 ? 0
                           : static_cast<std::int64_t>((static_cast<unsigned __int128>(c) *
                                                        static_cast<unsigned __int128>(num_edges)) /
                                                       static_cast<unsigned __int128>(S));
        c += d;
      }
    });
  }
  for (auto& th : pool) th.join();
  rowptr[n_src] = S == 0 ? 0 : num_edges;
}

inline std::uint64_t gcd64(std::uint64_t a, std::uint64_t b) {
  while (b) {
    const std::uint64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

// Affine permutation (a, b) of [0, m) used for target popularity.
inline void target_permutation(std::uint64_t m, std::uint64_t seed, std::uint64_t* a, std::uint64_t* b) {
  std::uint64_t x = (0x9E3779B97F4A7C15ull ^ seed) % m;
  if (x < 2) x = 2;
  while (gcd64(x, m) != 1) ++x;
  *a = x;
  *b = (seed * 0xD1B54A32D192ED03ull) % m;
}

// Target of edge j: popularity rank floor(m * u^3) through the permutation.
inline std::int64_t edge_target(std::int64_t j, std::int64_t m, std::uint64_t pa, std::uint64_t pb, std::uint32_t k0,
                                std::uint32_t k1) {
  const U4 r = philox4x32_10(U4{static_cast<std::uint32_t>(j), static_cast<std::uint32_t>(j >> 32), 0xd57u, 2u}, k0, k1);
  const double u = u01(r.x, r.y);
  std::int64_t rank = static_cast<std::int64_t>(static_cast<double>(m) * u * u * u);
  rank = rank < m ? rank : m - 1;
  const unsigned __int128 t = static_cast<unsigned __int128>(pa) * static_cast<std::uint64_t>(rank) + pb;
  return static_cast<std::int64_t>(t % static_cast<std::uint64_t>(m));
}

// Source-major edge list of the graph whose row pointers are `rowptr`.
inline void graph_edges(const std::int64_t* rowptr, std::int64_t n_src, std::int64_t n_dst, std::uint64_t seed,
                        std::int64_t* src, std::int64_t* dst, int threads) {
  const std::uint32_t k0 = static_cast<std::uint32_t>(seed), k1 = static_cast<std::uint32_t>(seed >> 32);
  std::uint64_t pa = 0, pb = 0;
  target_permutation(static_cast<std::uint64_t>(n_dst), seed, &pa, &pb);
  parallel_blocks(n_src, threads, [&](std::int64_t lo, std::int64_t hi) {
    for (std::int64_t v = lo; v < hi; ++v) {
      for (std::int64_t j = rowptr[v]; j < rowptr[v + 1]; ++j) {
        if (src != nullptr) src[j] = v;
        dst[j] = edge_target(j, n_dst, pa, pb, k0, k1);
      }
    }
  });
}

inline void uniform_int(std::int64_t n, std::int64_t lo, std::int64_t hi, std::uint64_t seed, std::uint32_t stream,
                        std::int64_t* out, int threads) {
  const std::uint32_t k0 = static_cast<std::uint32_t>(seed), k1 = static_cast<std::uint32_t>(seed >> 32);
  const std::uint64_t range = static_cast<std::uint64_t>(hi - lo);
  parallel_blocks(n, threads, [&](std::int64_t a, std::int64_t b) {
    for (std::int64_t i = a; i < b; ++i) {
      const U4 r = philox4x32_10(U4{static_cast<std::uint32_t>(i), static_cast<std::uint32_t>(i >> 32), stream, 3u},
                                 k0, k1);
      out[i] = lo + static_cast<std::int64_t>(bounded64(static_cast<std::uint64_t>(r.y) << 32 | r.x, range));
    }
  });
}

// fp32 -> bf16 bits, round to nearest even (finite inputs).
inline std::uint16_t bf16_bits(float f) {
  std::uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<std::uint16_t>(u >> 16);
}

// Rows [node_begin, node_begin + count) of the N(0, 1) feature table;
// bf16 != 0 writes bf16 bits (uint16), else fp32.
inline void normal_features(std::int64_t node_begin, std::int64_t count, std::int64_t dim, std::uint64_t seed,
                            int bf16, void* out, int threads) {
  const std::uint32_t k0 = static_cast<std::uint32_t>(seed), k1 = static_cast<std::uint32_t>(seed >> 32);
  const std::int64_t pairs = (dim + 1) / 2;
  parallel_blocks(count, threads, [&](std::int64_t a, std::int64_t b) {
    for (std::int64_t row = a; row < b; ++row) {
      const std::int64_t v = node_begin + row;
      for (std::int64_t p = 0; p < pairs; ++p) {
        const U4 r = philox4x32_10(
            U4{static_cast<std::uint32_t>(v), static_cast<std::uint32_t>(v >> 32), static_cast<std::uint32_t>(p), 4u},
            k0, k1);
        const double u1 = 1.0 - u01(r.x, r.y);
        const double u2 = u01(r.z, r.w);
        const double rad = std::sqrt(-2.0 * std::log(u1));
        const double ang = 6.283185307179586 * u2;
        const float f0 = static_cast<float>(rad * std::cos(ang));
        const float f1 = static_cast<float>(rad * std::sin(ang));
        const std::int64_t o = row * dim + 2 * p;
        if (bf16) {
          auto* h = static_cast<std::uint16_t*>(out);
          h[o] = bf16_bits(f0);
          if (2 * p + 1 < dim) h[o + 1] = bf16_bits(f1);
        } else {
          auto* f = static_cast<float*>(out);
          f[o] = f0;
          if (2 * p + 1 < dim) f[o + 1] = f1;
        }
      }
    }
  });
}

}  // namespace dgf_synth
