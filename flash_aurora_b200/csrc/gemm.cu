// Linear layer with a fused bias + exact-GELU epilogue on the 5th-generation tensor cores (sm_100a).
//
//   out[m, n] = act(sum_k a[m, k] * w[n, k] + bias[n]),   act = GELU (or identity)
//
// a: (M, K) bf16 row-major, w: (N, K) bf16 (nn.Linear weight layout), bias: (N) bf16, out: (M, N)
// bf16, fp32 accumulation. This is the fc1 -> GELU pair of the Swin3D block MLP (upstream
// swin3d.py:73-109: fc1 in bf16 autocast, then nn.GELU() on its output); fusing the activation
// into the GEMM removes a full read and write of the (tokens x 4D) hidden tensor, and the
// activation's arithmetic runs on the epilogue warps while the tensor cores work on the next tile.
//
// Persistent kernel, one CTA per SM, 128 x 256 output tiles (n fastest, so the CTAs working at the
// same time share their A tiles through L2):
//   warp 0      TMA producer: 64-wide K slices of A (128 x 64) and W (256 x 64), 128-byte swizzle,
//               into a 4-stage ring (48 KB per stage).
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and, from one thread,
//               issues tcgen05.mma kind::f16 (M=128, N=256, K=16) for every slice; commits free the
//               stage and, after the last slice, hand the accumulator to the epilogue.
//   warps 2-9   epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) and half the columns, adds
//               the bias, applies GELU (fitted erfc form, gelu.cuh), rounds to bf16, stages 32 x 64
//               blocks in shared memory and writes them with bulk tensor stores; the accumulator is
//               released for the tile after next.
// Every mbarrier wait is bounded; on expiry the kernel records a code in the status word
// (fa_gemm_status), sets an abort flag, frees TMEM and returns.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "fa_common.cuh"
#include "gelu.cuh"
#include "ptx.cuh"

namespace fa {
namespace gemm {

__device__ int g_status = 0;

using namespace ptx;

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr int kNumBars = 13;
// Epilogue staging: one 32-row x 64-column bf16 tile (128-byte swizzle) per epilogue warp.
constexpr int kStageOutBytes = 32 * 128;
constexpr int kSmem = kStages * kStageBytes + kEpiWarps * kStageOutBytes + kNumBars * 8 + 16 + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
constexpr uint32_t kIdesc = make_idesc(1, kBM, kBN, false, false);
constexpr uint64_t kTimeoutNs = 2000000000ull;
enum { kFull = 0, kEmpty = 4, kAccFull = 8, kAccEmpty = 10, kDone = 12 };

struct Params {
  int M, N, K;
  int tiles_n, num_tiles, k_iters;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;
  int64_t ldo;  // output row stride in elements
  int* status;
};

// Epilogue of one warp: the 32 rows of its TMEM lane quarter (starting at global row `row0`) and
// 128 accumulator columns starting at TMEM address `ta` (global column `col0`): + bias, optional
// GELU (fitted erfc form on the fp32 sum), one bf16 rounding, staged as 32 x 64 blocks (128-byte
// swizzle) and written with bulk tensor stores, which drop rows past M.
template <bool kGelu>
__device__ __forceinline__ void store_tile_half(uint32_t ta, int col0, int row0, uint32_t stage,
                                                const __nv_bfloat16* __restrict__ bias, const CUtensorMap* tmo,
                                                int lane) {
#pragma unroll 1
  for (int c = 0; c < 128; c += 64) {
    uint32_t r0[32], r1[32];
    tmem_ld32(ta + (uint32_t)c, r0);
    tmem_ld32(ta + (uint32_t)c + 32, r1);
    tmem_wait_ld();
    const int col = col0 + c;
    // bias: the same 64 values for every lane of the warp (broadcast loads)
    const uint4* bp = reinterpret_cast<const uint4*>(bias + col);
    uint32_t pk[32];
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const uint4 bw = __ldg(bp + v);
      const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = 8 * v + 2 * e;  // column pair within the 64
        const uint32_t* src = idx < 32 ? r0 : r1;
        const int si = idx & 31;
        const float2 bf = unpack_bf16x2(bb[e]);
        float2 y = make_float2(__uint_as_float(src[si]) + bf.x, __uint_as_float(src[si + 1]) + bf.y);
        if constexpr (kGelu) y = gelu2_bf16out(y);
        pk[4 * v + e] = pack_bf16x2(y.x, y.y);
      }
    }
    // The previous copy must have read the staging tile first.
    if (lane == 0) bulk_wait_group_read0();
    __syncwarp();
    const uint32_t srow = stage + (uint32_t)lane * 128u;
#pragma unroll
    for (int v = 0; v < 8; ++v)
      st_shared_v4(srow + (uint32_t)((v ^ (lane & 7)) << 4), pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmo, stage, col, row0);
      bulk_commit_group();
    }
  }
}

template <bool kGelu>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bias_act_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw,
                     const __grid_constant__ CUtensorMap tmo, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sout = sbase + kStages * kStageBytes;  // epilogue staging, 1024-byte aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kEpiWarps * kStageOutBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int n_local = p.num_tiles > (int)blockIdx.x ? (p.num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(BAR(kFull + s), 1);
      mbar_init(BAR(kEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kAccFull + b), 1);
      mbar_init(BAR(kAccEmpty + b), kEpiWarps);
    }
    mbar_init(BAR(kDone), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmw);
      int it = 0;
      int last_par[kStages] = {-1, -1, -1, -1};
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        const int t = (int)blockIdx.x + j * (int)gridDim.x;
        const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * kBN;
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (uint32_t)((it / kStages) & 1);
          if (!mbar_wait(BAR(kEmpty + s), ph ^ 1u, abort, p.status, 1, kTimeoutNs)) { ok = false; break; }
          const uint32_t sa = sbase + s * kStageBytes;
          mbar_arrive_expect_tx(BAR(kFull + s), (uint32_t)kStageBytes);
          tma_load_2d(sa, &tma, BAR(kFull + s), kb * kBK, m0);
          tma_load_2d(sa + kABytes, &tmw, BAR(kFull + s), kb * kBK, n0);
          last_par[s] = (int)ph;
        }
      }
      // Never leave with bulk copies in flight (bounded, also after an abort).
      int no_abort = 0;
      for (int s = 0; s < kStages; ++s)
        if (last_par[s] >= 0) mbar_wait(BAR(kFull + s), (uint32_t)last_par[s], &no_abort, p.status, 2, kTimeoutNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        const int buf = j & 1;
        if (!mbar_wait(BAR(kAccEmpty + buf), (uint32_t)(((j >> 1) & 1) ^ 1), abort, p.status, 3, kTimeoutNs)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)buf * kBN;
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(BAR(kFull + s), (uint32_t)((it / kStages) & 1), abort, p.status, 4, kTimeoutNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * kStageBytes, sw = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d, desc_sw128(sa + kk * 32, 16, 1024), desc_sw128(sw + kk * 32, 16, 1024), kIdesc,
                     (kb | kk) ? 1u : 0u);
          umma_commit(BAR(kEmpty + s));
        }
        if (ok) umma_commit(BAR(kAccFull + buf));
      }
      umma_commit(BAR(kDone));
      int no_abort = 0;
      mbar_wait(BAR(kDone), 0, &no_abort, p.status, 5, kTimeoutNs);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;      // columns [128 * half, 128 * half + 128)
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const uint32_t stage = sout + (uint32_t)(warp - 2) * kStageOutBytes;
    if (lane == 0) tma_prefetch_desc(&tmo);
    for (int j = 0; j < n_local; ++j) {
      const int buf = j & 1;
      const int t = (int)blockIdx.x + j * (int)gridDim.x;
      const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * kBN;
      if (!mbar_wait(BAR(kAccFull + buf), (uint32_t)((j >> 1) & 1), abort, p.status, 6, kTimeoutNs)) break;
      tc_fence_after();
      store_tile_half<kGelu>(tmem + lane_addr + (uint32_t)buf * kBN + (uint32_t)(half * 128), n0 + half * 128,
                             m0 + q * 32, stage, p.bias, &tmo, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kAccEmpty + buf));
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}


// ------------------------------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): 256 x 256 output tiles per pair.
//
// The even CTA of the pair issues one UMMA of M = 256, N = 256, K = 16 that reads A rows 0..127
// and W rows 0..127 from the even CTA's shared memory and A rows 128..255 / W rows 128..255 from
// the odd CTA's, and accumulates each CTA's 128 rows x 256 columns in its own TMEM. Per CTA a
// K slice brings 32 KB (A half + W half) for the same 128 x 256 x 64 products that cost the
// single-CTA kernel 48 KB: two thirds of the shared-memory fill per FLOP.
//   warp 0 (both CTAs)   TMA producer of its own halves; the bytes of both CTAs are counted on the
//                        even CTA's `full` barrier (cta_group::2 form of the tile load, no multicast).
//   warp 1 (both CTAs)   allocates 512 TMEM columns with cta_group::2; in the even CTA one thread
//                        issues the UMMAs and commits to the `empty` / `acc_full` barriers of both
//                        CTAs (tcgen05.commit with a CTA mask).
//   warps 2-9 (both)     epilogue of the CTA's 128 rows (store_tile_half); each warp releases the
//                        accumulator by arriving on the even CTA's `acc_empty` barrier.
// Every wait is bounded as in the single-CTA kernel; both CTAs meet at cluster barriers after set-up
// (before any remote arrive) and before the TMEM is freed (after every remote access).
// ------------------------------------------------------------------------------------------------
constexpr int kPairStages = 6;
constexpr int kPairHalfBytes = 128 * kBK * 2;            // 16 KB: A half or W half of a K slice
constexpr int kPairStageBytes = 2 * kPairHalfBytes;      // 32 KB per CTA and stage
constexpr int kPairNumBars = 2 * kPairStages + 5;
constexpr int kPairSmem = kPairStages * kPairStageBytes + kEpiWarps * kStageOutBytes + kPairNumBars * 8 + 16 + 1024;
static_assert(kPairSmem <= 227 * 1024, "shared memory budget (pair)");
constexpr uint32_t kPairIdesc = make_idesc(1, 256, kBN, false, false);
enum { kPFull = 0, kPEmpty = kPairStages, kPAccFull = 2 * kPairStages, kPAccEmpty = kPAccFull + 2,
       kPDone = kPAccEmpty + 2 };

template <bool kGelu>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_pair_bias_act_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw,
                          const __grid_constant__ CUtensorMap tmo, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sout = sbase + kPairStages * kPairStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes + kEpiWarps * kStageOutBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kPairNumBars);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the UMMAs; 1: its partner
  const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
  const int n_local = p.num_tiles > pair ? (p.num_tiles - 1 - pair) / npairs + 1 : 0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(BAR(kPFull + s), 1);
      mbar_init(BAR(kPEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kPAccFull + b), 1);
      mbar_init(BAR(kPAccEmpty + b), 2 * kEpiWarps);
    }
    mbar_init(BAR(kPDone), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the partner's barriers exist before any remote arrive or complete_tx
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmw);
      int it = 0;
      int last_par[kPairStages];
      for (int s = 0; s < kPairStages; ++s) last_par[s] = -1;
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        const int t = pair + j * npairs;
        const int m0 = (t / p.tiles_n) * 256 + (int)rank * 128, n0 = (t % p.tiles_n) * kBN + (int)rank * 128;
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kPairStages;
          const uint32_t ph = (uint32_t)((it / kPairStages) & 1);
          if (!mbar_wait(BAR(kPEmpty + s), ph ^ 1u, abort, p.status, 7, kTimeoutNs)) { ok = false; break; }
          const uint32_t sa = sbase + s * kPairStageBytes;
          const uint32_t full0 = map_shared_rank(BAR(kPFull + s), 0);
          if (rank == 0) mbar_arrive_expect_tx(BAR(kPFull + s), (uint32_t)(2 * kPairStageBytes));
          tma_load_2d_pair(sa, &tma, full0, kb * kBK, m0);
          tma_load_2d_pair(sa + kPairHalfBytes, &tmw, full0, kb * kBK, n0);
          last_par[s] = (int)ph;
        }
      }
      // Never leave with bulk copies in flight: the even CTA's `full` barriers count both CTAs'
      // bytes, so it waits for them (bounded); the odd CTA is held by the final cluster barrier.
      if (rank == 0) {
        int no_abort = 0;
        for (int s = 0; s < kPairStages; ++s)
          if (last_par[s] >= 0)
            mbar_wait(BAR(kPFull + s), (uint32_t)last_par[s], &no_abort, p.status, 8, kTimeoutNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        const int buf = j & 1;
        if (!mbar_wait(BAR(kPAccEmpty + buf), (uint32_t)(((j >> 1) & 1) ^ 1), abort, p.status, 9, kTimeoutNs)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)buf * kBN;
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kPairStages;
          if (!mbar_wait(BAR(kPFull + s), (uint32_t)((it / kPairStages) & 1), abort, p.status, 10, kTimeoutNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * kPairStageBytes, sw = sa + kPairHalfBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16_pair(d, desc_sw128(sa + kk * 32, 16, 1024), desc_sw128(sw + kk * 32, 16, 1024), kPairIdesc,
                          (kb | kk) ? 1u : 0u);
          umma_commit_pair(BAR(kPEmpty + s), 0x3);
        }
        if (ok) umma_commit_pair(BAR(kPAccFull + buf), 0x3);
      }
      umma_commit_pair(BAR(kPDone), 0x1);
      int no_abort = 0;
      mbar_wait(BAR(kPDone), 0, &no_abort, p.status, 11, kTimeoutNs);
    }
  } else {
    // ---------------- epilogue (both CTAs: this CTA's 128 rows of the pair's tile) ----------------
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const uint32_t stage = sout + (uint32_t)(warp - 2) * kStageOutBytes;
    if (lane == 0) tma_prefetch_desc(&tmo);
    for (int j = 0; j < n_local; ++j) {
      const int buf = j & 1;
      const int t = pair + j * npairs;
      const int m0 = (t / p.tiles_n) * 256 + (int)rank * 128, n0 = (t % p.tiles_n) * kBN;
      if (!mbar_wait(BAR(kPAccFull + buf), (uint32_t)((j >> 1) & 1), abort, p.status, 12, kTimeoutNs)) break;
      tc_fence_after();
      store_tile_half<kGelu>(tmem + lane_addr + (uint32_t)buf * kBN + (uint32_t)(half * 128), n0 + half * 128,
                             m0 + q * 32, stage, p.bias, &tmo, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(BAR(kPAccEmpty + buf));
        else mbar_arrive_remote(map_shared_rank(BAR(kPAccEmpty + buf), 0));
      }
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote access to the partner's shared memory or TMEM after this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2D map over a row-major (rows, K) bf16 matrix, box (64, box_rows), 128-byte swizzle, rows past
// the end read as zero.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  FA_REQUIRE(fn, FA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t gstr[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, gstr, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FA_REQUIRE(r == CUDA_SUCCESS, FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
}

// 2D map over the (M, N) bf16 output for bulk stores of 32-row x 64-column tiles.
int make_out_map(CUtensorMap* map, void* base, int64_t M, int64_t N, int64_t ld) {
  auto fn = encode_fn();
  FA_REQUIRE(fn, FA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t gstr[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, 32u};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, gstr, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FA_REQUIRE(r == CUDA_SUCCESS, FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
}

// 0: choose by shape; 1: single-CTA kernel; 2: CTA-pair kernel (FA_GEMM_KERNEL=single|pair).
int kernel_choice() {
  const char* e = getenv("FA_GEMM_KERNEL");
  if (!e) return 0;
  if (!strcmp(e, "single")) return 1;
  if (!strcmp(e, "pair")) return 2;
  return 0;
}

int* status_ptr() {
  int* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_status) != cudaSuccess) return nullptr;
  return ptr;
}

}  // namespace gemm
}  // namespace fa

using namespace fa;

extern "C" int fa_linear_bias_act(const void* a, const void* w, const void* bias, void* out, int64_t M,
                                  int64_t N, int64_t K, int64_t lda, int64_t ldw, int64_t ldo, int act,
                                  void* stream) {
  FA_REQUIRE(act == FA_ACT_NONE || act == FA_ACT_GELU, FA_ERR_INVALID, "act must be FA_ACT_NONE or FA_ACT_GELU");
  FA_REQUIRE(M >= 0 && N > 0 && K > 0, FA_ERR_INVALID, "invalid GEMM shape");
  FA_REQUIRE(N % gemm::kBN == 0, FA_ERR_UNSUPPORTED, "N must be a multiple of 256");
  FA_REQUIRE(K % gemm::kBK == 0, FA_ERR_UNSUPPORTED, "K must be a multiple of 64");
  FA_REQUIRE(M < ((int64_t)1 << 31) && N < ((int64_t)1 << 24) && K < ((int64_t)1 << 24), FA_ERR_INVALID,
             "GEMM too large");
  if (M == 0) return FA_OK;
  FA_REQUIRE(a && w && bias && out, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(aligned16(a) && aligned16(w) && aligned16(bias) && aligned16(out), FA_ERR_INVALID,
             "a, w, bias and out must be 16-byte aligned");
  FA_REQUIRE(lda >= K && ldw >= K && ldo >= N && lda % 8 == 0 && ldw % 8 == 0 && ldo % 8 == 0, FA_ERR_INVALID,
             "row strides must cover the rows and be multiples of 8 elements");
  // Kernel: the CTA-pair kernel (256 x 256 tiles, two thirds of the shared-memory fill per FLOP);
  // it measured at least as fast as the single-CTA kernel at every config-4 linear once its
  // accumulator release stopped paying a cluster-scope memory barrier (stage-1 fc1 + GELU 0.47-0.49
  // against 0.48-0.49 ms). FA_GEMM_KERNEL=single|pair forces one (tests).
  const int choice = gemm::kernel_choice();
  const bool use_pair = choice != 1;
  const int64_t tile_m = use_pair ? 256 : gemm::kBM;
  CUtensorMap ma, mw, mo;
  int rc;
  if ((rc = gemm::make_map(&ma, a, M, K, lda, gemm::kBM)) != FA_OK) return rc;
  if ((rc = gemm::make_map(&mw, w, N, K, ldw, use_pair ? 128u : (uint32_t)gemm::kBN)) != FA_OK) return rc;
  if ((rc = gemm::make_out_map(&mo, out, M, N, ldo)) != FA_OK) return rc;
  gemm::Params p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.tiles_n = (int)(N / gemm::kBN);
  const int64_t tiles = ((M + tile_m - 1) / tile_m) * p.tiles_n;
  FA_REQUIRE(tiles < ((int64_t)1 << 31), FA_ERR_INVALID, "too many tiles");
  p.num_tiles = (int)tiles;
  p.k_iters = (int)(K / gemm::kBK);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.status = gemm::status_ptr();
  FA_REQUIRE(p.status, FA_ERR_CUDA, "cannot resolve the GEMM status word");
  if (use_pair) {
    auto kern = act == FA_ACT_GELU ? gemm::gemm_pair_bias_act_kernel<true> : gemm::gemm_pair_bias_act_kernel<false>;
    FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::kPairSmem));
    const int pairs_max = max_resident_pairs((const void*)kern, gemm::kThreads, gemm::kPairSmem);
    const int pairs = p.num_tiles < pairs_max ? p.num_tiles : pairs_max;
    kern<<<2 * pairs, gemm::kThreads, gemm::kPairSmem, (cudaStream_t)stream>>>(ma, mw, mo, p);
    return check_launch("gemm_pair_bias_act_kernel");
  }
  auto kern = act == FA_ACT_GELU ? gemm::gemm_bias_act_kernel<true> : gemm::gemm_bias_act_kernel<false>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::kSmem));
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  kern<<<grid, gemm::kThreads, gemm::kSmem, (cudaStream_t)stream>>>(ma, mw, mo, p);
  return check_launch("gemm_bias_act_kernel");
}

extern "C" int fa_gemm_status(int* status_out) {
  FA_REQUIRE(status_out, FA_ERR_INVALID, "null status pointer");
  int* p = gemm::status_ptr();
  FA_REQUIRE(p, FA_ERR_CUDA, "cannot resolve the GEMM status word");
  FA_CUDA(cudaMemcpy(status_out, p, sizeof(int), cudaMemcpyDeviceToHost));
  return FA_OK;
}

extern "C" int fa_gemm_status_reset(void* stream) {
  int* p = gemm::status_ptr();
  FA_REQUIRE(p, FA_ERR_CUDA, "cannot resolve the GEMM status word");
  FA_CUDA(cudaMemsetAsync(p, 0, sizeof(int), (cudaStream_t)stream));
  return FA_OK;
}
