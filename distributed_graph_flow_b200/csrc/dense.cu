// Dense layer after neighbour aggregation on the 5th-generation tensor cores.
//
// Computes Y = act(concat[X1, X2] @ W^T + b) in bf16 with fp32 accumulation:
// the GraphSAGE / MPNN update "concat[x_dst, agg] -> Dense -> ReLU"
// (dgf/src/learning/jax/layers/hetero_gnn.py:302-312 with GenericBlock's
// nn.Dense, dgf/src/learning/jax/layers/standard.py:238-270). The concat is
// never materialised: the first k1/64 K-blocks of a tile come from X1's
// tensor map, the rest from X2's.
//
// Kernel structure (one persistent CTA per SM, 6 warps):
//   warp 0   TMA producer: per K-block a 128x64 tile of X1|X2 and a BNx64
//            tile of W (both K-major, 128-byte swizzle) into a 4-stage ring;
//   warp 1   owns the TMEM allocation (2 accumulators of BN fp32 columns);
//            one lane issues tcgen05.mma (M=128, N=BN, K=16, bf16 x bf16 ->
//            fp32) and tcgen05.commit to release ring stages and to publish
//            a finished accumulator;
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time from their TMEM
//            lane quarter, + bias, ReLU, round to bf16 into swizzled shared
//            staging boxes, TMA bulk stores to global;
//            double-buffered accumulators let tile i's epilogue overlap
//            tile i+1's MMAs.
// Every mbarrier wait is bounded (%globaltimer); on expiry the CTA raises an
// error flag (dgfx_dense_check), the roles leave their loops, outstanding
// copies and MMAs are drained with bounded waits and TMEM is freed.
// No TMA multicast, no clusters.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"

namespace dgfx {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

__device__ unsigned int g_dense_err;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete; false on timeout or when
// another role already aborted (the abort word is then set).
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (now_ns() - t0 > kWaitNs) {
        *abort_flag = 1;
        atomicOr(&g_dense_err, 1u);
        return false;
      }
    }
    if (i > 32) __nanosleep(20);
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;            // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;            // descriptor version (tcgen05)
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN>
struct DenseSmem {
  static constexpr uint32_t kA = kBM * kBK * 2;  // 16 KB
  static constexpr uint32_t kB = BN * kBK * 2;   // up to 32 KB
  static constexpr uint32_t kStage = kA + kB;
  static constexpr uint32_t kTmemCols = BN * 2 <= 32 ? 32 : BN * 2;  // two accumulators
  // Output staging per epilogue warp: up to two 32-row x 64-column boxes
  // (4 KB each, 128-byte swizzle) handed to TMA stores.
  static constexpr uint32_t kBoxes = BN >= 128 ? 2 : 1;
  static constexpr uint32_t kOutWarp = kBoxes * 4096;
  static constexpr uint32_t kOut = 4 * kOutWarp;
  static constexpr size_t kBytes =
      static_cast<size_t>(kStages) * kStage + kOut + 1024 /* align */ + 256 /* barriers */;
};

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    dense_concat_kernel(const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_x2,
                        const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_y, int64_t m,
                        int32_t n, int32_t kb1, int32_t kb_total, const float* __restrict__ bias, int32_t relu) {
  using L = DenseSmem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte swizzled tiles need 1024-byte aligned shared addresses.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* out_stage = smem + kStages * L::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + L::kOut);
  // bars: full[kStages], empty[kStages], acc_full[2], acc_empty[2], drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages);
  const uint32_t accf0 = smem_u32(bars + 2 * kStages), acce0 = smem_u32(bars + 2 * kStages + 2);
  const uint32_t drain = smem_u32(bars + 2 * kStages + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t m_tiles = (m + kBM - 1) / kBM;
  const int32_t n_tiles = n / BN;
  const int64_t tiles = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;  // stages with a load issued in the current ring pass
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int32_t mb = static_cast<int32_t>(t / n_tiles), nb = static_cast<int32_t>(t % n_tiles);
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = smem_u32(smem + s * L::kStage);
          const uint32_t b_dst = a_dst + L::kA;
          mbar_arrive_expect_tx(full0 + 8 * s, L::kStage);
          if (kb < kb1) {
            tma_load_2d(a_dst, &tm_x1, full0 + 8 * s, kb * kBK, mb * kBM);
          } else {
            tma_load_2d(a_dst, &tm_x2, full0 + 8 * s, (kb - kb1) * kBK, mb * kBM);
          }
          tma_load_2d(b_dst, &tm_w, full0 + 8 * s, kb * kBK, nb * BN);
          issued |= 1u << s;
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
            issued = 0;
          }
        }
      }
      if (!ok) {
        // Drain: every stage loaded in this pass completes its transaction.
        for (int j = 0; j < kStages; ++j) {
          if (issued & (1u << j)) {
            const uint64_t t0 = now_ns();
            while (!mbar_test(full0 + 8 * j, ph) && now_ns() - t0 < kWaitNs) __nanosleep(100);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, BN);
      int s = 0;
      uint32_t ph = 0;
      int b = 0;
      uint32_t aph = 0;
      bool ok = true;
      bool any = false;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(acce0 + 8 * b, aph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * BN);
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::kStage);
          const uint64_t adesc = smem_desc_sw128(a_addr);
          const uint64_t bdesc = smem_desc_sw128(a_addr + L::kA);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K step of 16 bf16 = 32 bytes inside the 128-byte swizzle atom.
            mma_bf16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          any = true;
          mma_commit(empty0 + 8 * s);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(accf0 + 8 * b);
        if (++b == 2) {
          b = 0;
          aph ^= 1u;
        }
      }
      if (any) {
        // All MMAs issued by this thread are complete once `drain` fires.
        mma_commit(drain);
        const uint64_t t0 = now_ns();
        while (!mbar_test(drain, 0) && now_ns() - t0 < kWaitNs) __nanosleep(100);
      }
    }
    __syncwarp();
  } else {
    // Epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (its 32 rows),
    // 32 columns per tcgen05.ld; rounded bf16 rows go to this warp's staging
    // boxes in the 128-byte swizzled layout (16-byte chunk j of row r at
    // chunk j ^ (r % 8)) and leave in 32x64 TMA stores (rows past m are
    // clipped by the tensor map).
    const int q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    uint8_t* my_stage = out_stage + (warp - 2) * L::kOutWarp;
    const uint32_t my_stage_u32 = smem_u32(my_stage);
    constexpr int kGroupCols = L::kBoxes * 64;
    int b = 0;
    uint32_t aph = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      bool ready = true;
      if (lane == 0) ready = mbar_wait(accf0 + 8 * b, aph, abort_flag);
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready) break;
      tc_fence_after();
      const int64_t mb = t / n_tiles;
      const int32_t nb = static_cast<int32_t>(t % n_tiles);
      const int64_t row0 = mb * kBM + 32 * q;
#pragma unroll 1
      for (int g = 0; g < BN / kGroupCols; ++g) {
        // The staging boxes are free once the previous stores read them.
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
#pragma unroll 1
        for (int cc = 0; cc < kGroupCols / 32; ++cc) {
          const int c = g * (kGroupCols / 32) + cc;
          uint32_t v[32];
          float bv[32];
          if (bias != nullptr) {
            const float4* b4 = reinterpret_cast<const float4*>(bias + nb * BN + c * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 f = __ldg(b4 + j);
              bv[4 * j] = f.x;
              bv[4 * j + 1] = f.y;
              bv[4 * j + 2] = f.z;
              bv[4 * j + 3] = f.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) bv[j] = 0.0f;
          }
          tmem_ld32(tmem_base + lane_off + static_cast<uint32_t>(b * BN + c * 32), v);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float x0 = __uint_as_float(v[2 * j]) + bv[2 * j];
            float x1 = __uint_as_float(v[2 * j + 1]) + bv[2 * j + 1];
            if (relu) {
              x0 = fmaxf(x0, 0.0f);
              x1 = fmaxf(x1, 0.0f);
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
            packed[j] = *reinterpret_cast<const uint32_t*>(&h);
          }
          uint8_t* box = my_stage + (cc >> 1) * 4096 + lane * 128;
          const int half = cc & 1;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = (half * 4 + j) ^ (lane & 7);
            *reinterpret_cast<uint4*>(box + chunk * 16) =
                make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && row0 < m) {
#pragma unroll
          for (int bx = 0; bx < static_cast<int>(L::kBoxes); ++bx) {
            tma_store_2d(&tm_y, my_stage_u32 + bx * 4096, nb * BN + g * kGroupCols + bx * 64,
                         static_cast<int32_t>(row0));
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * b);
      if (++b == 2) {
        b = 0;
        aph ^= 1u;
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(L::kTmemCols)
                 : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// Row-major bf16 [rows, cols] matrix, box = box_rows x 64 columns, 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(DGFX_ERR_CUDA, "dgfx_dense: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DGFX_ERR_CUDA, "dgfx_dense: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return DGFX_OK;
}

template <int BN>
int launch_dense(const CUtensorMap& x1, const CUtensorMap& x2, const CUtensorMap& w, const CUtensorMap& ym, int64_t m,
                 int32_t n, int32_t kb1, int32_t kbt, const float* bias, int32_t relu, cudaStream_t stream) {
  using L = DenseSmem<BN>;
  static std::once_flag once[64];
  int dev = 0;
  DGFX_CUDA_TRY(cudaGetDevice(&dev));
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&]() {
    attr_err = cudaFuncSetAttribute(dense_concat_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(L::kBytes));
  });
  DGFX_CUDA_TRY(attr_err);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = ((m + kBM - 1) / kBM) * (n / BN);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms)));
  dense_concat_kernel<BN><<<grid, kThreads, L::kBytes, stream>>>(x1, x2, w, ym, m, n, kb1, kbt, bias, relu);
  DGFX_CUDA_TRY(cudaGetLastError());
  return DGFX_OK;
}

unsigned int* dense_err_word() {
  static std::mutex mu;
  static std::map<int, unsigned int*> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_dense_err) != cudaSuccess) return nullptr;
  cache[dev] = static_cast<unsigned int*>(p);
  return static_cast<unsigned int*>(p);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace dgfx

using namespace dgfx;

extern "C" int dgfx_dense_concat_bf16(const void* d_x1, int64_t k1, const void* d_x2, int64_t k2, int64_t m,
                                      const void* d_w, const float* d_bias, int64_t n, int32_t relu, void* d_y,
                                      dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || k1 < kBK || k1 % kBK != 0 || k2 < 0 || k2 % kBK != 0 || n < 64 || n % 64 != 0 || d_x1 == nullptr ||
      d_w == nullptr || (k2 > 0 && d_x2 == nullptr) || (m > 0 && d_y == nullptr)) {
    return fail(DGFX_ERR_INVALID_ARGUMENT,
                "dgfx_dense_concat_bf16: need k1 >= 64, k1 and k2 multiples of 64, n a multiple of 64, non-null "
                "operands");
  }
  if (!aligned16(d_x1) || !aligned16(d_w) || (d_x2 != nullptr && !aligned16(d_x2)) || !aligned16(d_y) ||
      (d_bias != nullptr && !aligned16(d_bias))) {
    return fail(DGFX_ERR_INVALID_ARGUMENT, "dgfx_dense_concat_bf16: operands must be 16-byte aligned");
  }
  if (m >= (int64_t(1) << 31) || n > (int64_t(1) << 20) || (k1 + k2) / kBK > (1 << 20)) {
    return fail(DGFX_ERR_UNSUPPORTED, "dgfx_dense_concat_bf16: sizes out of range");
  }
  if (m == 0) return DGFX_OK;
  if (dense_err_word() == nullptr) return fail(DGFX_ERR_CUDA, "dgfx_dense: status word unavailable");
  const int bn = n % 256 == 0 ? 256 : (n % 128 == 0 ? 128 : 64);
  CUtensorMap x1, x2, w;
  DGFX_TRY(make_map(&x1, d_x1, m, k1, kBM));
  DGFX_TRY(make_map(&x2, k2 > 0 ? d_x2 : d_x1, m, k2 > 0 ? k2 : k1, kBM));
  DGFX_TRY(make_map(&w, d_w, n, k1 + k2, static_cast<uint32_t>(bn)));
  CUtensorMap ym;
  DGFX_TRY(make_map(&ym, d_y, m, n, 32));
  const int32_t kb1 = static_cast<int32_t>(k1 / kBK), kbt = static_cast<int32_t>((k1 + k2) / kBK);
  const int32_t n32 = static_cast<int32_t>(n);
  switch (bn) {
    case 256:
      return launch_dense<256>(x1, x2, w, ym, m, n32, kb1, kbt, d_bias, relu, stream);
    case 128:
      return launch_dense<128>(x1, x2, w, ym, m, n32, kb1, kbt, d_bias, relu, stream);
    default:
      return launch_dense<64>(x1, x2, w, ym, m, n32, kb1, kbt, d_bias, relu, stream);
  }
}

extern "C" int dgfx_dense_check(dgfx_stream stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  unsigned int* word = dense_err_word();
  if (word == nullptr) return fail(DGFX_ERR_CUDA, "dgfx_dense: status word unavailable");
  unsigned int v = 0;
  DGFX_CUDA_TRY(cudaMemcpyAsync(&v, word, sizeof(v), cudaMemcpyDeviceToHost, stream));
  DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
  if (v != 0) {
    DGFX_CUDA_TRY(cudaMemsetAsync(word, 0, sizeof(v), stream));
    DGFX_CUDA_TRY(cudaStreamSynchronize(stream));
    return fail(DGFX_ERR_INTERNAL, "dgfx_dense: a pipeline wait timed out; the output is invalid");
  }
  return DGFX_OK;
}
