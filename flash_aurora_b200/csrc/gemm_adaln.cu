// Linear layer fused with the block's AdaLN + residual epilogue, for rows of D = 512 (sm_100a).
//
//   h[m, :] = bf16(a[m, :] . w^T + bias)                       (the bf16 linear output)
//   y[tok]  = residual[tok] + LN(h[m]) * (scale_bias + scale[b]) + shift[b]      (fp32)
//
// Two call sites of the Swin3D block (upstream swin3d.py:706-815, film.py:101-139) each run a
// linear whose every output row is immediately layer-normalised, modulated and added to the fp32
// residual stream:
//   FA_ROWS_WINDOWS  attention proj (rows = window slots) -> crop/un-roll/merge -> norm1: the row
//                    of window slot m lands at its token (pad slots are dropped); a bf16 copy of
//                    y feeds fc1.
//   FA_ROWS_TOKENS   MLP fc2 (rows = tokens) -> norm2; y can also be scattered, in bf16, into the
//                    window layout of the next block (its roll + pad + partition).
// Unfused, the linear writes h (bf16) and the AdaLN kernel reads it back. Here h never leaves the
// SM, and the AdaLN's HBM traffic (residual in, y out) overlaps the next tile's tensor-core work.
//
// CTA pair (cluster of 2, tcgen05 cta_group::2), 256 rows x 512 columns per pair tile: a whole
// row of D = 512 fp32 accumulators sits in one CTA's TMEM (all 512 columns). Per CTA:
//   warp 0      TMA producer, 32-wide K slices (64-byte swizzle) of A (128 rows) and of its two
//               W quarters (rows r*128.. and 256 + r*128..), 4-stage ring; bytes of both CTAs
//               are counted on the even CTA's `full` barrier (no multicast loads).
//   warp 1      TMEM (512 columns, cta_group::2); in the even CTA one thread issues the M = 256,
//               N = 256 UMMAs for both column halves and commits to both CTAs' barriers.
//   warps 2-9   epilogue in two phases per tile:
//               E1  thread = row (TMEM lane): accumulator + bias, rounded to bf16 exactly as the
//                   plain linear rounds its output, written to a 128 x 512 bf16 tile in shared
//                   memory (16-byte chunks XOR-swizzled by row); then the TMEM is released, so
//                   the next tile's UMMAs run during E2.
//                   Each thread also sums its half row.
//               E1b thread = row (four warps): mean from the half-row sums, then the sum of squared
//                   deviations over the bf16 row in shared memory (two-pass variance, fp32).
//               E2  warp = row: y = residual + (h - mean) * rstd * (scale_bias + scale) + shift,
//                   coalesced 16-byte row I/O, four rows' residual loads in flight per warp; the
//                   tile's residual rows are prefetched into L2 when its accumulator is ready.
// The row statistics are summed in another order than the stand-alone AdaLN kernel's warp
// reduction, so results agree with the unfused pair to fp32 rounding, not bit for bit.
// Every mbarrier wait is bounded (status codes 18-23 in the GEMM status word).
#include <cudaTypedefs.h>

#include <string>

#include "fa_common.cuh"
#include "ptx.cuh"

namespace fa {
namespace gemm {
int* status_ptr();
}  // namespace gemm

namespace gemm_adaln {

using namespace ptx;

constexpr int kD = 512;                 // output features = row length of the AdaLN
constexpr int kRows = 128;              // rows per CTA (256 per pair)
constexpr int kBK = 32;                 // K slice (64-byte rows, 64-byte swizzle)
constexpr int kStages = 4;
constexpr int kABytes = kRows * kBK * 2;        // 8 KB
constexpr int kWQBytes = 128 * kBK * 2;         // 8 KB: one W quarter of a K slice
constexpr int kStageBytes = kABytes + 2 * kWQBytes;  // 24 KB
constexpr int kHBytes = kRows * kD * 2;         // 128 KB bf16 row tile
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr int kNumBars = 2 * kStages + 3;
constexpr int kStatBytes = 3 * kRows * 4;  // per row: two half-row sums, then mean and rstd
constexpr int kSmem = kStages * kStageBytes + kHBytes + kStatBytes + kNumBars * 8 + 16 + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
constexpr uint32_t kIdesc = make_idesc(1, 256, 256, false, false);
constexpr uint64_t kTimeoutNs = 2000000000ull;
enum { kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = kAccFull + 1, kDone = kAccEmpty + 1 };
enum { kRowsTokens = 0, kRowsWindows = 1 };

struct Params {
  int M;            // rows of a
  int k_iters;      // K / kBK
  int num_tiles;    // ceil(M / 256)
  const __nv_bfloat16* bias;       // (512)
  const float* scale;              // (B, 512)
  const float* shift;              // (B, 512)
  float scale_bias, eps;
  const float* residual;           // (B * L, 512)
  float* out;                      // (B * L, 512)
  __nv_bfloat16* out_bf16;         // optional (B * L, 512)
  __nv_bfloat16* win_out;          // optional next-block windows (B * nW' * N', 512)
  int64_t L;                       // tokens per batch element
  int64_t slots;                   // window slots per batch element (rows of a, windows mode)
  LayoutParams lp;                 // windows mode: this block's partition (slot -> token)
  LayoutParams wlp;                // tokens mode: next block's partition (token -> slot)
  int* status;
};

// Shared-memory matrix descriptor, K-major, 64-byte swizzle: rows of 64 B (32 bf16 of K), 8-row
// atoms of 512 B (`sbo` apart).
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;  // leading byte offset: unused for swizzled K-major layouts
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

// Barrier of the epilogue warps that also ANDs `ok` over them: every epilogue warp takes the same
// branch after a bounded wait, so none is left alone at a later epilogue barrier.
__device__ __forceinline__ bool epi_all(bool ok) {
  uint32_t r;
  asm volatile("{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, 1, %2, p; selp.u32 %0, 1, 0, q; }"
               : "=r"(r)
               : "r"((uint32_t)ok), "n"(kEpiWarps * 32)
               : "memory");
  return r != 0;
}

// Byte offset of 16-byte chunk j (8 bf16 columns) of row r in the h tile.
__device__ __forceinline__ uint32_t h_off(int r, int j) {
  return (uint32_t)(r * (kD * 2) + ((j ^ (r & 7)) << 4));
}

template <int kMode>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_adaln_pair_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw,
                       const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sh_tile = sbase + kStages * kStageBytes;  // h tile (1024-aligned)
  float* stat = reinterpret_cast<float*>(smem + kStages * kStageBytes + kHBytes);  // [3][kRows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kHBytes + kStatBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
  const int n_local = p.num_tiles > pair ? (p.num_tiles - 1 - pair) / npairs + 1 : 0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(BAR(kFull + s), 1);
      mbar_init(BAR(kEmpty + s), 1);
    }
    mbar_init(BAR(kAccFull), 1);
    mbar_init(BAR(kAccEmpty), 2 * kEpiWarps);
    mbar_init(BAR(kDone), 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmw);
      int it = 0;
      int last_par[kStages];
      for (int s = 0; s < kStages; ++s) last_par[s] = -1;
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        const int t = pair + j * npairs;
        const int m0 = t * 256 + (int)rank * kRows;
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (uint32_t)((it / kStages) & 1);
          if (!mbar_wait(BAR(kEmpty + s), ph ^ 1u, abort, p.status, 18, kTimeoutNs)) { ok = false; break; }
          const uint32_t sa = sbase + s * kStageBytes;
          const uint32_t full0 = map_shared_rank(BAR(kFull + s), 0);
          if (rank == 0) mbar_arrive_expect_tx(BAR(kFull + s), (uint32_t)(2 * kStageBytes));
          tma_load_2d_pair(sa, &tma, full0, kb * kBK, m0);
          tma_load_2d_pair(sa + kABytes, &tmw, full0, kb * kBK, (int)rank * 128);
          tma_load_2d_pair(sa + kABytes + kWQBytes, &tmw, full0, kb * kBK, 256 + (int)rank * 128);
          last_par[s] = (int)ph;
        }
      }
      if (rank == 0) {
        int no_abort = 0;
        for (int s = 0; s < kStages; ++s)
          if (last_par[s] >= 0) mbar_wait(BAR(kFull + s), (uint32_t)last_par[s], &no_abort, p.status, 19, kTimeoutNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < n_local && ok; ++j) {
        if (!mbar_wait(BAR(kAccEmpty), (uint32_t)((j & 1) ^ 1), abort, p.status, 20, kTimeoutNs)) break;
        tc_fence_after();
        for (int kb = 0; kb < p.k_iters; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(BAR(kFull + s), (uint32_t)((it / kStages) & 1), abort, p.status, 21, kTimeoutNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * kStageBytes, sw0 = sa + kABytes, sw1 = sw0 + kWQBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = desc_sw64(sa + kk * 32, 512);
            const uint32_t acc = (kb | kk) ? 1u : 0u;
            umma_f16_pair(tmem, ad, desc_sw64(sw0 + kk * 32, 512), kIdesc, acc);
            umma_f16_pair(tmem + 256, ad, desc_sw64(sw1 + kk * 32, 512), kIdesc, acc);
          }
          umma_commit_pair(BAR(kEmpty + s), 0x3);
        }
        if (ok) umma_commit_pair(BAR(kAccFull), 0x3);
      }
      umma_commit_pair(BAR(kDone), 0x1);
      int no_abort = 0;
      mbar_wait(BAR(kDone), 0, &no_abort, p.status, 22, kTimeoutNs);
    }
  } else {
    // ---------------- epilogue: E1 (thread = row) then E2 (warp = row) ----------------
    const int e = warp - 2;
    const int q = warp & 3;               // TMEM lane quarter (E1 rows q*32 + lane)
    const int half = e >> 2;              // E1 columns [256 * half, 256 * half + 256)
    const int r1 = q * 32 + lane;         // E1 row of this thread
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const float inv_d = 1.0f / (float)kD;

    // Token row (b * L + token) of A row m, or -1 (pad slot / past M).
    auto token_of = [&](int64_t m) -> int64_t {
      if (m >= p.M) return -1;
      if constexpr (kMode == kRowsTokens) return m;
      const int64_t b = m / p.slots;
      const int32_t slot = (int32_t)(m - b * p.slots);
      const int32_t src = partition_source(p.lp, slot / p.lp.N, slot % p.lp.N);
      return src < 0 ? -1 : b * p.L + src;
    };
    auto prefetch_tile = [&](int j) {  // residual rows of tile j of this CTA into L2
      if (j >= n_local || lane != 0) return;
      const int64_t m0 = (int64_t)(pair + j * npairs) * 256 + (int64_t)rank * kRows + e * 16;
      for (int i = 0; i < 16; ++i) {
        const int64_t tok = token_of(m0 + i);
        if (tok >= 0) prefetch_l2_bulk(p.residual + tok * kD, (uint32_t)(kD * 4));
      }
    };
    prefetch_tile(0);
    for (int j = 0; j < n_local; ++j) {
      const int64_t m0 = (int64_t)(pair + j * npairs) * 256 + (int64_t)rank * kRows;
      const bool ready = mbar_wait(BAR(kAccFull), (uint32_t)(j & 1), abort, p.status, 23, kTimeoutNs);
      if (!epi_all(ready)) break;
      tc_fence_after();
      // This tile's residual rows start moving into L2 now, one E1 + E1b ahead of E2. A whole tile
      // ahead was too early: the A stream of the next tile evicted them (ncu: the residual read
      // twice from DRAM).
      if (j > 0) prefetch_tile(j);
      // E1: accumulators + bias -> bf16 row tile, and this thread's half-row sum of the bf16 values.
      float acc4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int c = 0; c < 256; c += 64) {
        uint32_t v0[32], v1[32];
        const uint32_t ta = tmem + lane_addr + (uint32_t)(half * 256 + c);
        tmem_ld32(ta, v0);
        tmem_ld32(ta + 32, v1);
        tmem_wait_ld();
        const int col = half * 256 + c;
        const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const uint4 bw = __ldg(bp + v);
          const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
          uint32_t pk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int idx = 8 * v + 2 * u;
            const uint32_t* src = idx < 32 ? v0 : v1;
            const int si = idx & 31;
            const float2 bf = unpack_bf16x2(bb[u]);
            pk[u] = pack_bf16x2(__uint_as_float(src[si]) + bf.x, __uint_as_float(src[si + 1]) + bf.y);
            const float2 hv = unpack_bf16x2(pk[u]);
            acc4[u] += hv.x + hv.y;
          }
          st_shared_v4(sh_tile + h_off(r1, col / 8 + v), pk[0], pk[1], pk[2], pk[3]);
        }
      }
      stat[half * kRows + r1] = (acc4[0] + acc4[1]) + (acc4[2] + acc4[3]);
      // The accumulator is read: release it (the next tile's UMMAs start during E2).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(BAR(kAccEmpty));
        else mbar_arrive_remote_cluster_release(map_shared_rank(BAR(kAccEmpty), 0));
      }
      epi_bar();  // every row of the h tile and every half-row sum is written
      // E1b (thread = row, the four half-0 warps): mean from the two half-row sums, then the sum
      // of squared deviations over the whole bf16 row from shared memory (two-pass variance).
      if (half == 0) {
        const float mean = (stat[r1] + stat[kRows + r1]) * inv_d;
        float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int jc = 0; jc < kD / 8; ++jc) {
          uint32_t w0, w1, w2, w3;
          ld_shared_v4(sh_tile + h_off(r1, jc), w0, w1, w2, w3);
          const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 f = unpack_bf16x2(ws[u]);
            const float d0 = f.x - mean, d1 = f.y - mean;
            q4[u] = fmaf(d0, d0, q4[u]);
            q4[u] = fmaf(d1, d1, q4[u]);
          }
        }
        stat[2 * kRows + r1] = mean;
        stat[r1] = rsqrtf(((q4[0] + q4[1]) + (q4[2] + q4[3])) * inv_d + p.eps);  // rstd
      }
      epi_bar();
      // E2 (warp = row): y = residual + (h - mean) * rstd * (scale_bias + scale) + shift, 16 rows per
      // warp in groups of 4 whose residual loads are issued together; lane l holds columns
      // 8l..8l+7 and 256+8l..+7. Coalesced 16-byte row I/O, no reductions.
#pragma unroll 1
      for (int i0 = 0; i0 < 16; i0 += 4) {
        int32_t tok[4], bb[4];  // token rows and batch indices fit 32 bits (M < 2^31 is checked)
        float rr[4][16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t m = m0 + e * 16 + i0 + k;
          tok[k] = (int32_t)token_of(m);
          bb[k] = tok[k] < 0 ? 0 : (int32_t)(kMode == kRowsTokens ? tok[k] / p.L : m / p.slots);
          if (tok[k] >= 0) {
            Vec8<float>::load_stream(p.residual + (int64_t)tok[k] * kD + lane * 8, rr[k]);
            Vec8<float>::load_stream(p.residual + (int64_t)tok[k] * kD + 256 + lane * 8, rr[k] + 8);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (tok[k] < 0) continue;
          const int r = e * 16 + i0 + k;
          const float mean = stat[2 * kRows + r], rstd = stat[r];
          int64_t wrow = -1;
          if constexpr (kMode == kRowsTokens) {
            if (p.win_out) {
              const int32_t t = (int32_t)(tok[k] - (int64_t)bb[k] * p.L);
              int32_t cc, hh, w;
              unmerge_token(p.wlp, t, cc, hh, w);
              wrow = bb[k] * (int64_t)p.wlp.nW * p.wlp.N + unmerge_slot(p.wlp, cc, hh, w);
            }
          }
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            const int col = (ch * 32 + lane) * 8;
            uint32_t w0, w1, w2, w3;
            ld_shared_v4(sh_tile + h_off(r, ch * 32 + lane), w0, w1, w2, w3);
            const uint32_t ws[4] = {w0, w1, w2, w3};
            float sc[8], sf[8], y[8];
            Vec8<float>::load(p.scale + (int64_t)bb[k] * kD + col, sc);
            Vec8<float>::load(p.shift + (int64_t)bb[k] * kD + col, sf);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 f = unpack_bf16x2(ws[u]);
              y[2 * u] = (f.x - mean) * rstd * (p.scale_bias + sc[2 * u]) + sf[2 * u];
              y[2 * u + 1] = (f.y - mean) * rstd * (p.scale_bias + sc[2 * u + 1]) + sf[2 * u + 1];
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) y[u] += rr[k][8 * ch + u];
            Vec8<float>::store(p.out + (int64_t)tok[k] * kD + col, y);
            if (p.out_bf16) Vec8<__nv_bfloat16>::store(p.out_bf16 + (int64_t)tok[k] * kD + col, y);
            if (wrow >= 0) Vec8<__nv_bfloat16>::store(p.win_out + wrow * kD + col, y);
          }
        }
      }
      epi_bar();  // the h tile is free for the next E1
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2D map over a row-major (rows, K) bf16 matrix, box (32, 128), 64-byte swizzle, rows past the end
// read as zero.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld) {
  auto fn = encode_fn();
  FA_REQUIRE(fn, FA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t gstr[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, 128u};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, gstr, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FA_REQUIRE(r == CUDA_SUCCESS, FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
}

}  // namespace gemm_adaln
}  // namespace fa

using namespace fa;

extern "C" int fa_linear_adaln_film(const void* a, const void* w, const void* bias, int64_t M, int64_t K,
                                    int64_t lda, int rows_kind, const float* scale, const float* shift,
                                    float scale_bias, float eps, const float* residual, float* out,
                                    void* out_bf16, void* win_out, int64_t B, int64_t C, int64_t H, int64_t W,
                                    const int32_t window_size[3], const int32_t shift_size[3],
                                    const int32_t next_shift_size[3], void* stream) {
  namespace G = gemm_adaln;
  FA_REQUIRE(rows_kind == FA_ROWS_TOKENS || rows_kind == FA_ROWS_WINDOWS, FA_ERR_INVALID,
             "rows_kind must be FA_ROWS_TOKENS or FA_ROWS_WINDOWS");
  FA_REQUIRE(B >= 0 && M >= 0 && K > 0, FA_ERR_INVALID, "invalid shape");
  FA_REQUIRE(K % G::kBK == 0 && K < ((int64_t)1 << 24), FA_ERR_UNSUPPORTED, "K must be a multiple of 32");
  FA_REQUIRE(window_size && shift_size, FA_ERR_INVALID, "null window or shift size");
  Geometry g;
  int rc = make_geometry(C, H, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  const int64_t L = C * H * W;
  const int64_t slots = g.nW * (int64_t)g.N;
  const int64_t want_m = rows_kind == FA_ROWS_TOKENS ? B * L : B * slots;
  FA_REQUIRE(M == want_m, FA_ERR_INVALID,
             "M must be B*C*H*W (tokens) or B*nW*N (window slots) for this geometry");
  FA_REQUIRE(M < ((int64_t)1 << 31), FA_ERR_INVALID, "too many rows");
  FA_REQUIRE(rows_kind == FA_ROWS_TOKENS || !win_out, FA_ERR_INVALID, "window output needs FA_ROWS_TOKENS rows");
  if (M == 0) return FA_OK;
  FA_REQUIRE(a && w && bias && scale && shift && residual && out, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(aligned16(a) && aligned16(w) && aligned16(bias) && aligned16(scale) && aligned16(shift) &&
                 aligned16(residual) && aligned16(out) && (!out_bf16 || aligned16(out_bf16)) &&
                 (!win_out || aligned16(win_out)),
             FA_ERR_INVALID, "every tensor must be 16-byte aligned");
  FA_REQUIRE(lda >= K && lda % 8 == 0, FA_ERR_INVALID, "lda must cover K and be a multiple of 8 elements");
  G::Params p{};
  p.M = (int)M;
  p.k_iters = (int)(K / G::kBK);
  p.num_tiles = (int)((M + 255) / 256);
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.scale = scale;
  p.shift = shift;
  p.scale_bias = scale_bias;
  p.eps = eps;
  p.residual = residual;
  p.out = out;
  p.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  p.win_out = reinterpret_cast<__nv_bfloat16*>(win_out);
  p.L = L;
  p.slots = slots;
  p.lp = layout_params(g);
  if (win_out) {
    FA_REQUIRE(next_shift_size, FA_ERR_INVALID, "null next shift size");
    Geometry gn;
    rc = make_geometry(C, H, W, window_size, next_shift_size, &gn);
    if (rc != FA_OK) return rc;
    p.wlp = layout_params(gn);
  }
  p.status = gemm::status_ptr();
  FA_REQUIRE(p.status, FA_ERR_CUDA, "cannot resolve the GEMM status word");
  CUtensorMap ma, mw;
  if ((rc = G::make_map(&ma, a, M, K, lda)) != FA_OK) return rc;
  if ((rc = G::make_map(&mw, w, G::kD, K, K)) != FA_OK) return rc;
  auto kern = rows_kind == FA_ROWS_TOKENS ? G::gemm_adaln_pair_kernel<G::kRowsTokens>
                                          : G::gemm_adaln_pair_kernel<G::kRowsWindows>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem));
  const int pairs_max = max_resident_pairs((const void*)kern, G::kThreads, G::kSmem);
  const int pairs = p.num_tiles < pairs_max ? p.num_tiles : pairs_max;
  kern<<<2 * pairs, G::kThreads, G::kSmem, (cudaStream_t)stream>>>(ma, mw, p);
  return check_launch("gemm_adaln_pair_kernel");
}
