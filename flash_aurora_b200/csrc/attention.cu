// Shifted-window attention for N <= 144 tokens per window, head_dim 64 (sm_100a).
//
//   out[w, h] = softmax(q k^T * scale + bias) v,   bias = -100 where the mask says "masked"
//
// Persistent kernel, one CTA per SM, one (window, head) tile at a time per CTA:
//   * warp 0 is the TMA producer: Q, K, V of a tile (144 x 64, zero-filled past N) are loaded by
//     cp.async.bulk.tensor into a ring of shared-memory stages with 128-byte swizzle, completion
//     tracked by mbarriers;
//   * the consumer warps each own 16 query rows of the tile and run QK^T, the masked
//     softmax (log2 domain, fp32) and PV on warp-level tensor-core MMAs reading the swizzled
//     tiles with ldmatrix.
// FP32 I/O uses 3xTF32 (hi/lo split of both operands, three products), so it keeps fp32
// accuracy, unlike the upstream 1xTF32 QK^T + BF16 PV kernel (ops/cute/_kernel_fp32.py:142).
//
// Mask semantics follow the upstream SDPA path (swin3d.py:376-384, bias -100 added after the
// scale, window index b % nW) and the CuTe kernel (ops/cute/_kernel_bf16.py:361-365).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "fa_common.cuh"
#include "ptx.cuh"

namespace fa {
namespace attn {

__device__ int g_status = 0;

namespace {

using namespace ptx;

// Swizzled byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-row tile
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------------------------------
// Mask helpers: returns the additive log2-domain bias of (row, key).
// ------------------------------------------------------------------------------------------
template <int kMask>
struct MaskView {
  const uint8_t* base;  // this window's ids (N) or mask rows (N x N)
  int N;
  __device__ __forceinline__ uint32_t row_tag(int r) const {
    if constexpr (kMask == kGroups) return r < N ? __ldg(base + r) : 0u;
    else return (uint32_t)r;
  }
  __device__ __forceinline__ bool masked(uint32_t rtag, int key) const {
    if constexpr (kMask == kGroups) return __ldg(base + key) != rtag;
    else if constexpr (kMask == kMaskU8) return (int)rtag < N && __ldg(base + (int64_t)rtag * N + key) != 0;
    else return false;
  }
  // Key-side data of keys (key, key + 1) for two rows, one load per row pair when aligned.
  __device__ __forceinline__ uint32_t key_pair(int key) const {
    if constexpr (kMask == kGroups) {
      if (key + 1 < N && ((reinterpret_cast<uintptr_t>(base) + key) & 1) == 0)
        return __ldg(reinterpret_cast<const unsigned short*>(base + key));
      const uint32_t lo = key < N ? __ldg(base + key) : 0u;
      const uint32_t hi = key + 1 < N ? __ldg(base + key + 1) : 0u;
      return lo | (hi << 8);
    } else {
      return 0u;
    }
  }
};

// ------------------------------------------------------------------------------------------
// 16 query rows [r0, r0 + 16) of one tile, bf16 operands (mma.sync m16n8k16).
// ------------------------------------------------------------------------------------------
template <int kMask>
__device__ __forceinline__ void rows16_bf16(uint32_t sQ, uint32_t sK, uint32_t sV, int r0, int N,
                                            float scale_log2, const MaskView<kMask>& mv,
                                            __nv_bfloat16* out_rows, int64_t os_n, int lane) {
  const int m = lane >> 3, l8 = lane & 7, q = lane & 3;
  float s[18][4];
#pragma unroll
  for (int j = 0; j < 18; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a0, a1, a2, a3;
    const int qr = r0 + l8 + ((m & 1) << 3);
    ldmatrix_x4(sQ + sw128(qr, 2 * kk + (m >> 1)), a0, a1, a2, a3);
#pragma unroll
    for (int j = 0; j < 18; j += 2) {
      uint32_t b0, b1, b2, b3;
      const int key = 8 * (j + (m >> 1)) + l8;
      ldmatrix_x4(sK + sw128(key, 2 * kk + (m & 1)), b0, b1, b2, b3);
      mma_bf16_16816(s[j], a0, a1, a2, a3, b0, b1);
      mma_bf16_16816(s[j + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  // Scale into the log2 domain, apply the mask, row max.
  const int ra = r0 + (lane >> 2), rb = ra + 8;
  const uint32_t ta = mv.row_tag(ra), tb = mv.row_tag(rb);
  float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
  for (int j = 0; j < 18; ++j) {
    const uint32_t kp = mv.key_pair(8 * j + 2 * q);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * q + e;
      float xa = s[j][e] * scale_log2, xb = s[j][2 + e] * scale_log2;
      if (key >= N) {
        xa = -INFINITY;
        xb = -INFINITY;
      } else if constexpr (kMask == kGroups) {
        const uint32_t kg = (kp >> (8 * e)) & 0xffu;
        if (kg != ta) xa += kMaskedLog2;
        if (kg != tb) xb += kMaskedLog2;
      } else if constexpr (kMask == kMaskU8) {
        if (mv.masked(ta, key)) xa += kMaskedLog2;
        if (mv.masked(tb, key)) xb += kMaskedLog2;
      }
      s[j][e] = xa;
      s[j][2 + e] = xb;
      mxa = fmaxf(mxa, xa);
      mxb = fmaxf(mxb, xb);
    }
  }
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int j = 0; j < 18; ++j) {
    s[j][0] = ex2(s[j][0] - mxa);
    s[j][1] = ex2(s[j][1] - mxa);
    s[j][2] = ex2(s[j][2] - mxb);
    s[j][3] = ex2(s[j][3] - mxb);
    la += s[j][0] + s[j][1];
    lb += s[j][2] + s[j][3];
  }
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);

  float o[8][4];
#pragma unroll
  for (int jd = 0; jd < 8; ++jd) o[jd][0] = o[jd][1] = o[jd][2] = o[jd][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 9; ++kk) {
    const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
    const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
    const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int jd = 0; jd < 8; jd += 2) {
      uint32_t b0, b1, b2, b3;
      const int key = 16 * kk + ((m & 1) << 3) + l8;
      ldmatrix_x4_trans(sV + sw128(key, jd + (m >> 1)), b0, b1, b2, b3);
      mma_bf16_16816(o[jd], a0, a1, a2, a3, b0, b1);
      mma_bf16_16816(o[jd + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  const float ia = 1.f / la, ib = 1.f / lb;
  if (ra < N) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(out_rows + (int64_t)ra * os_n + 2 * q);
#pragma unroll
    for (int jd = 0; jd < 8; ++jd) dst[4 * jd] = pack_bf16x2(o[jd][0] * ia, o[jd][1] * ia);
  }
  if (rb < N) {
    uint32_t* dst = reinterpret_cast<uint32_t*>(out_rows + (int64_t)rb * os_n + 2 * q);
#pragma unroll
    for (int jd = 0; jd < 8; ++jd) dst[4 * jd] = pack_bf16x2(o[jd][2] * ib, o[jd][3] * ib);
  }
}

// ------------------------------------------------------------------------------------------
// 16 query rows, fp32 operands with 3xTF32 products (mma.sync m16n8k8 tf32).
// Each operand tile is two 144 x 32 fp32 halves (d 0-31, d 32-63), 128-byte rows, swizzled.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f32_tile_off(int row, int d) {
  return (uint32_t)((d >> 5) * kTileBytes) + sw128(row, (d & 31) >> 2) + (uint32_t)((d & 3) << 2);
}

__device__ __forceinline__ void mma3_tf32(float c[4], const uint32_t ah[4], const uint32_t al[4],
                                          uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma_tf32_1688(c, al[0], al[1], al[2], al[3], bh0, bh1);
  mma_tf32_1688(c, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
  mma_tf32_1688(c, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
}

template <int kMask>
__device__ __forceinline__ void rows16_tf32x3(uint32_t sQ, uint32_t sK, uint32_t sV, int r0, int N,
                                              float scale_log2, const MaskView<kMask>& mv,
                                              float* out_rows, int64_t os_n, int lane) {
  const int m = lane >> 3, l8 = lane & 7, q = lane & 3;
  float s[18][4];
#pragma unroll
  for (int j = 0; j < 18; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll 1
  for (int kk = 0; kk < 8; ++kk) {
    uint32_t a[4], ah[4], al[4];
    const int qr = r0 + l8 + ((m & 1) << 3);
    ldmatrix_x4(sQ + f32_tile_off(qr, 8 * kk + 4 * (m >> 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) split_tf32(__uint_as_float(a[i]), ah[i], al[i]);
#pragma unroll
    for (int j = 0; j < 18; j += 2) {
      uint32_t b[4], bh[4], bl[4];
      const int key = 8 * (j + (m >> 1)) + l8;
      ldmatrix_x4(sK + f32_tile_off(key, 8 * kk + 4 * (m & 1)), b[0], b[1], b[2], b[3]);
#pragma unroll
      for (int i = 0; i < 4; ++i) split_tf32(__uint_as_float(b[i]), bh[i], bl[i]);
      mma3_tf32(s[j], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3_tf32(s[j + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
  const int ra = r0 + (lane >> 2), rb = ra + 8;
  const uint32_t ta = mv.row_tag(ra), tb = mv.row_tag(rb);
  float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
  for (int j = 0; j < 18; ++j) {
    const uint32_t kp = mv.key_pair(8 * j + 2 * q);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * q + e;
      float xa = s[j][e] * scale_log2, xb = s[j][2 + e] * scale_log2;
      if (key >= N) {
        xa = -INFINITY;
        xb = -INFINITY;
      } else if constexpr (kMask == kGroups) {
        const uint32_t kg = (kp >> (8 * e)) & 0xffu;
        if (kg != ta) xa += kMaskedLog2;
        if (kg != tb) xb += kMaskedLog2;
      } else if constexpr (kMask == kMaskU8) {
        if (mv.masked(ta, key)) xa += kMaskedLog2;
        if (mv.masked(tb, key)) xb += kMaskedLog2;
      }
      s[j][e] = xa;
      s[j][2 + e] = xb;
      mxa = fmaxf(mxa, xa);
      mxb = fmaxf(mxb, xb);
    }
  }
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int j = 0; j < 18; ++j) {
    s[j][0] = ex2(s[j][0] - mxa);
    s[j][1] = ex2(s[j][1] - mxa);
    s[j][2] = ex2(s[j][2] - mxb);
    s[j][3] = ex2(s[j][3] - mxb);
    la += s[j][0] + s[j][1];
    lb += s[j][2] + s[j][3];
  }
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);

  float o[8][4];
#pragma unroll
  for (int jd = 0; jd < 8; ++jd) o[jd][0] = o[jd][1] = o[jd][2] = o[jd][3] = 0.f;
  // Keys are consumed in a permuted order inside each group of 8: logical k = q <-> key 2q,
  // k = q + 4 <-> key 2q + 1, which lets the S accumulator registers serve as the A fragment.
#pragma unroll
  for (int kk = 0; kk < 18; ++kk) {
    uint32_t ah[4], al[4];
    split_tf32(s[kk][0], ah[0], al[0]);
    split_tf32(s[kk][2], ah[1], al[1]);
    split_tf32(s[kk][1], ah[2], al[2]);
    split_tf32(s[kk][3], ah[3], al[3]);
    const int key0 = 8 * kk + 2 * q;
#pragma unroll
    for (int jd = 0; jd < 8; ++jd) {
      const int d = 8 * jd + (lane >> 2);
      const float v0 = __uint_as_float(ld_shared_u32(sV + f32_tile_off(key0, d)));
      const float v1 = __uint_as_float(ld_shared_u32(sV + f32_tile_off(key0 + 1, d)));
      uint32_t bh0, bl0, bh1, bl1;
      split_tf32(v0, bh0, bl0);
      split_tf32(v1, bh1, bl1);
      mma3_tf32(o[jd], ah, al, bh0, bh1, bl0, bl1);
    }
  }
  const float ia = 1.f / la, ib = 1.f / lb;
  if (ra < N) {
    float2* dst = reinterpret_cast<float2*>(out_rows + (int64_t)ra * os_n + 2 * q);
#pragma unroll
    for (int jd = 0; jd < 8; ++jd) dst[4 * jd] = make_float2(o[jd][0] * ia, o[jd][1] * ia);
  }
  if (rb < N) {
    float2* dst = reinterpret_cast<float2*>(out_rows + (int64_t)rb * os_n + 2 * q);
#pragma unroll
    for (int jd = 0; jd < 8; ++jd) dst[4 * jd] = make_float2(o[jd][2] * ib, o[jd][3] * ib);
  }
}

// ------------------------------------------------------------------------------------------
// Kernel
// ------------------------------------------------------------------------------------------
constexpr int kConsumerWarps = kMaxN / 16;  // 9
constexpr int kThreads = 32 * (1 + kConsumerWarps);

template <bool kF32>
struct Cfg {
  static constexpr int kOpBytes = kF32 ? 2 * kTileBytes : kTileBytes;
  static constexpr int kStageBytes = 3 * kOpBytes;
  static constexpr int kStages = kF32 ? 2 : 3;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 128;
};

template <bool kF32, int kMask>
__global__ void __launch_bounds__(kThreads, 1)
attn_sync_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv, const Params p) {
  using C = Cfg<kF32>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + C::kStages);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kConsumerWarps);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      int stage = 0;
      uint32_t phase = 0;
      int filled_parity[4] = {-1, -1, -1, -1};
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, &abort_flag, p.status, 1, kTimeoutNs)) break;
        const int w = t / p.H, h = t - (t / p.H) * p.H;
        const uint32_t full = full0 + 8 * stage;
        const uint32_t dst = sbase + stage * C::kStageBytes;
        mbar_arrive_expect_tx(full, C::kStageBytes);
        if constexpr (kF32) {
          tma_load_4d(dst, &tmq, full, 0, 0, h, w);
          tma_load_4d(dst + kTileBytes, &tmq, full, 32, 0, h, w);
          tma_load_4d(dst + C::kOpBytes, &tmk, full, 0, 0, h, w);
          tma_load_4d(dst + C::kOpBytes + kTileBytes, &tmk, full, 32, 0, h, w);
          tma_load_4d(dst + 2 * C::kOpBytes, &tmv, full, 0, 0, h, w);
          tma_load_4d(dst + 2 * C::kOpBytes + kTileBytes, &tmv, full, 32, 0, h, w);
        } else {
          tma_load_4d(dst, &tmq, full, 0, 0, h, w);
          tma_load_4d(dst + C::kOpBytes, &tmk, full, 0, 0, h, w);
          tma_load_4d(dst + 2 * C::kOpBytes, &tmv, full, 0, 0, h, w);
        }
        filled_parity[stage] = (int)phase;
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      // Never leave the CTA with bulk copies in flight: wait (bounded) for the last fill of
      // every stage, also after an abort.
      int dummy_abort = 0;
      for (int s = 0; s < C::kStages; ++s)
        if (filled_parity[s] >= 0)
          mbar_wait(full0 + 8 * s, (uint32_t)filled_parity[s], &dummy_abort, p.status, 2, kTimeoutNs);
    }
  } else {
    const int r0 = (warp - 1) * 16;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      if (!mbar_wait(full0 + 8 * stage, phase, &abort_flag, p.status, 3, kTimeoutNs)) break;
      const int w = t / p.H, h = t - (t / p.H) * p.H;
      const uint32_t st = sbase + stage * C::kStageBytes;
      if (r0 < p.N) {
        MaskView<kMask> mv;
        mv.N = p.N;
        const int mw = w % p.nW;
        if constexpr (kMask == kGroups) mv.base = p.mask + (int64_t)mw * p.N;
        else if constexpr (kMask == kMaskU8) mv.base = p.mask + (int64_t)mw * p.N * p.N;
        else mv.base = nullptr;
        const int64_t ooff = (int64_t)w * p.os_w + (int64_t)h * p.os_h;
        if constexpr (kF32)
          rows16_tf32x3<kMask>(st, st + C::kOpBytes, st + 2 * C::kOpBytes, r0, p.N, p.scale_log2, mv,
                               reinterpret_cast<float*>(p.out) + ooff, p.os_n, lane);
        else
          rows16_bf16<kMask>(st, st + C::kOpBytes, st + 2 * C::kOpBytes, r0, p.N, p.scale_log2, mv,
                             reinterpret_cast<__nv_bfloat16*>(p.out) + ooff, p.os_n, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * stage);
      if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------
// BF16 kernel on the 5th-generation tensor cores (tcgen05 / UMMA, accumulators in TMEM).
//
// A window has 144 query rows; an M=128 UMMA covers 128. Every tile therefore runs two
// query blocks through the tensor cores: rows 0..127 and rows 16..143 (the second block reuses
// the same shared-memory tiles at a 16-row offset; only its last 16 rows, 128..143, are kept).
//
// Warp roles (256 threads, one CTA per SM, persistent over (window, head) tiles):
//   warp 0      TMA producer: Q, K, V of a tile into a 3-stage ring (128-byte swizzle).
//   warp 1      owns TMEM (512 columns) and, from one thread, issues the UMMAs:
//                 S  = Q[0:128]  K^T, S2 = Q[16:144] K^T   (M=128, N=144, K=64, K-major A and B)
//                 O  = P[0:128]  V,   O2 = P[16:144] V     (M=128, N=64, K=144, V MN-major)
//               and signals completion with tcgen05.commit on mbarriers.
//   warps 4..7  softmax + epilogue of rows 0..127: one TMEM lane (row) per thread; S row from TMEM,
//               scale + mask + exp2 + row sum in fp32, P row (bf16) into shared memory in the UMMA
//               A-operand layout; then O row from TMEM, times 1/sum, bf16, to global memory.
//   warp 3      the same for rows 128..143, read from S2/O2 lanes 112..127 (its TMEM quadrant).
// S is read into registers at the start of the softmax and released at once, so the S UMMAs of
// tile i+1 run under the softmax of tile i; O is double-buffered. Every wait is bounded.
// ------------------------------------------------------------------------------------------
namespace tc {

constexpr int kStages = 3;
constexpr int kStageBytes = 3 * kTileBytes;  // Q, K, V (bf16, 144 x 128 B each)
constexpr int kPChunk = kTileBytes;          // 64 keys x 144 rows of bf16
constexpr int kPBytes = 3 * kPChunk;         // keys 0-63, 64-127, 128-143 (+ unused tail)
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColS2 = 160, kColO0 = 320, kColO1 = 384, kColO2 = 448;
constexpr int kNumBars = 18;
constexpr int kSmem = kStages * kStageBytes + kPBytes + kNumBars * 8 + 16 + 1024;
constexpr uint32_t kIdescS = ptx::make_idesc(1, 128, kMaxN, false, false);
constexpr uint32_t kIdescO = ptx::make_idesc(1, 128, 64, false, true);
constexpr uint32_t kRowOff16 = 16 * 128;  // 16 rows of a 128-byte-row tile (swizzle-atom aligned)

enum { kFull = 0, kEmpty = 3, kSFull = 6, kSFree = 7, kPFull = 8, kPEmpty = 9, kOFull = 10, kOFree = 12,
       kO2Full = 14, kO2Free = 15, kDone = 16 };

// Masked keys of one row as a bit per key (bit j set = masked). Reads the window's region ids
// (or the row of the u8 mask) 16 bytes at a time when N is a multiple of 16.
__device__ __forceinline__ uint32_t nibble_of_bytes(uint32_t ne) {
  return (ne & 1u) | ((ne >> 7) & 2u) | ((ne >> 14) & 4u) | ((ne >> 21) & 8u);
}

template <int kMask>
__device__ __forceinline__ void row_mask_bits(const Params& p, int mw, int row, uint32_t bits[5]) {
#pragma unroll
  for (int i = 0; i < 5; ++i) bits[i] = 0u;
  if constexpr (kMask != kNoMask) {
    const uint8_t* src;
    uint32_t ref = 0;
    if constexpr (kMask == kGroups) {
      src = p.mask + (int64_t)mw * p.N;
      ref = (row < p.N ? (uint32_t)__ldg(src + row) : 0u) * 0x01010101u;
    } else {
      if (row >= p.N) return;
      src = p.mask + ((int64_t)mw * p.N + row) * p.N;
    }
    if ((p.N & 15) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      for (int v = 0; v < p.N / 16; ++v) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + v);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j4 = 4 * v + k;
          bits[j4 >> 3] |= nibble_of_bytes(__vcmpne4(ws[k], ref)) << ((j4 & 7) * 4);
        }
      }
    } else {
      for (int key = 0; key < p.N; ++key) {
        const uint32_t b = __ldg(src + key);
        const bool m = (kMask == kGroups) ? (b != (ref & 0xffu)) : (b != 0u);
        if (m) bits[key >> 5] |= 1u << (key & 31);
      }
    }
  }
}

// One softmax row: S (144 fp32 in registers) -> P (bf16 pairs), returns the row sum. Max and
// sum use 8 independent accumulators so the single warp per scheduler is not latency bound.
template <int kMask>
__device__ __forceinline__ float softmax_row(uint32_t (&sr)[9][16], uint32_t (&pk)[9][8], const uint32_t mbits[5],
                                             float scale_log2, int N) {
  float mx8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
  const uint32_t kMaskBits = __float_as_uint(kMaskedLog2);
#pragma unroll
  for (int c = 0; c < 9; ++c) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int key = 16 * c + e;
      float y;
      if constexpr (kMask != kNoMask) {
        const uint32_t bit = (mbits[key >> 5] >> (key & 31)) & 1u;
        y = fmaf(__uint_as_float(sr[c][e]), scale_log2, __uint_as_float((0u - bit) & kMaskBits));
      } else {
        y = __uint_as_float(sr[c][e]) * scale_log2;
      }
      if (key >= N) y = -INFINITY;
      sr[c][e] = __float_as_uint(y);
      mx8[e & 7] = fmaxf(mx8[e & 7], y);
    }
  }
  const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
  float l8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) l8[e] = 0.f;
#pragma unroll
  for (int c = 0; c < 9; ++c) {
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const float a = ex2(__uint_as_float(sr[c][e]) - mx);
      const float b = ex2(__uint_as_float(sr[c][e + 1]) - mx);
      l8[(e >> 1) & 7] += a + b;
      pk[c][e >> 1] = pack_bf16x2(a, b);
    }
  }
  return ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
}

// P row `prow` (0..143) -> shared memory, UMMA A operand: K-major, 64-key chunks of 144 rows.
__device__ __forceinline__ void store_p_row(uint32_t sP, int prow, const uint32_t (&pk)[9][8]) {
#pragma unroll
  for (int c = 0; c < 9; ++c) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j16 = 2 * c + hh;  // 8-key group 0..17
      const uint32_t addr = sP + (j16 >> 3) * kPChunk + prow * 128 + (((j16 & 7) ^ (prow & 7)) << 4);
      st_shared_v4(addr, pk[c][4 * hh], pk[c][4 * hh + 1], pk[c][4 * hh + 2], pk[c][4 * hh + 3]);
    }
  }
}

// O row (64 fp32 in TMEM) * inv -> bf16 -> 128 contiguous bytes in global memory.
__device__ __forceinline__ void store_o_row(uint32_t taddr, float inv, __nv_bfloat16* dst, bool valid) {
  uint32_t o[4][16];
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_ld16(taddr + 16 * c, o[c]);
  tmem_wait_ld();
  if (!valid) return;
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 a, b;
    a.x = pack_bf16x2(__uint_as_float(o[c][0]) * inv, __uint_as_float(o[c][1]) * inv);
    a.y = pack_bf16x2(__uint_as_float(o[c][2]) * inv, __uint_as_float(o[c][3]) * inv);
    a.z = pack_bf16x2(__uint_as_float(o[c][4]) * inv, __uint_as_float(o[c][5]) * inv);
    a.w = pack_bf16x2(__uint_as_float(o[c][6]) * inv, __uint_as_float(o[c][7]) * inv);
    b.x = pack_bf16x2(__uint_as_float(o[c][8]) * inv, __uint_as_float(o[c][9]) * inv);
    b.y = pack_bf16x2(__uint_as_float(o[c][10]) * inv, __uint_as_float(o[c][11]) * inv);
    b.z = pack_bf16x2(__uint_as_float(o[c][12]) * inv, __uint_as_float(o[c][13]) * inv);
    b.w = pack_bf16x2(__uint_as_float(o[c][14]) * inv, __uint_as_float(o[c][15]) * inv);
    d[2 * c] = a;
    d[2 * c + 1] = b;
  }
}

template <int kMask>
__global__ void __launch_bounds__(kThreads, 1)
attn_tc_bf16_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sP = sbase + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kPBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(BAR(kFull + s), 1);
      mbar_init(BAR(kEmpty + s), 1);
    }
    mbar_init(BAR(kSFull), 1);
    mbar_init(BAR(kSFree), 5);  // 4 softmax warps + the rows-128..143 warp
    mbar_init(BAR(kPFull), 5);
    mbar_init(BAR(kPEmpty), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kOFull + b), 1);
      mbar_init(BAR(kOFree + b), 4);
    }
    mbar_init(BAR(kO2Full), 1);
    mbar_init(BAR(kO2Free), 1);
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
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      int last_par[kStages] = {-1, -1, -1};
      int i = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++i) {
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)((i / kStages) & 1);
        if (!mbar_wait(BAR(kEmpty + s), ph ^ 1u, abort, p.status, 11, kTimeoutNs)) break;
        const int w = t / p.H, h = t - w * p.H;
        const uint32_t dst = sbase + s * kStageBytes;
        mbar_arrive_expect_tx(BAR(kFull + s), kStageBytes);
        tma_load_4d(dst, &tmq, BAR(kFull + s), 0, 0, h, w);
        tma_load_4d(dst + kTileBytes, &tmk, BAR(kFull + s), 0, 0, h, w);
        tma_load_4d(dst + 2 * kTileBytes, &tmv, BAR(kFull + s), 0, 0, h, w);
        last_par[s] = (int)ph;
      }
      int no_abort = 0;
      for (int s = 0; s < kStages; ++s)
        if (last_par[s] >= 0) mbar_wait(BAR(kFull + s), (uint32_t)last_par[s], &no_abort, p.status, 12, kTimeoutNs);
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      auto issue_pv = [&](int j) -> bool {
        const int s = j % kStages, ob = j & 1;
        if (!mbar_wait(BAR(kPFull), (uint32_t)(j & 1), abort, p.status, 13, kTimeoutNs)) return false;
        if (!mbar_wait(BAR(kOFree + ob), (uint32_t)(((j >> 1) & 1) ^ 1), abort, p.status, 14, kTimeoutNs))
          return false;
        if (!mbar_wait(BAR(kO2Free), (uint32_t)((j & 1) ^ 1), abort, p.status, 22, kTimeoutNs)) return false;
        tc_fence_after();
        const uint32_t sV = sbase + s * kStageBytes + 2 * kTileBytes;
        const uint32_t dO = tmem + (ob ? kColO1 : kColO0);
#pragma unroll
        for (int k = 0; k < 9; ++k) {
          const uint32_t pa = sP + (k >> 2) * kPChunk + (k & 3) * 32;
          const uint64_t b = desc_sw128(sV + k * 2048, kTileBytes, 1024);
          umma_f16(dO, desc_sw128(pa, 16, 1024), b, kIdescO, k > 0 ? 1u : 0u);
          umma_f16(tmem + kColO2, desc_sw128(pa + kRowOff16, 16, 1024), b, kIdescO, k > 0 ? 1u : 0u);
        }
        umma_commit(BAR(kOFull + ob));
        umma_commit(BAR(kO2Full));
        umma_commit(BAR(kPEmpty));
        umma_commit(BAR(kEmpty + s));
        return true;
      };
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++i) {
        const int s = i % kStages;
        if (!mbar_wait(BAR(kFull + s), (uint32_t)((i / kStages) & 1), abort, p.status, 15, kTimeoutNs)) { ok = false; break; }
        if (!mbar_wait(BAR(kSFree), (uint32_t)((i & 1) ^ 1), abort, p.status, 16, kTimeoutNs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sQ = sbase + s * kStageBytes, sK = sQ + kTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t b = desc_sw128(sK + k * 32, 16, 1024);
          umma_f16(tmem + kColS, desc_sw128(sQ + k * 32, 16, 1024), b, kIdescS, k > 0 ? 1u : 0u);
          umma_f16(tmem + kColS2, desc_sw128(sQ + kRowOff16 + k * 32, 16, 1024), b, kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(BAR(kSFull));
        if (i > 0 && !issue_pv(i - 1)) { ok = false; break; }
      }
      if (ok && i > 0) issue_pv(i - 1);
      umma_commit(BAR(kDone));
      int no_abort = 0;
      mbar_wait(BAR(kDone), 0, &no_abort, p.status, 17, kTimeoutNs);
    }
  } else if (warp == 3 || warp >= 4) {
    // ---------------- softmax + epilogue ----------------
    // warps 4..7: rows 0..127 from S/O (lane quadrant warp & 3).
    // warp 3:     rows 112..143 from S2/O2 lanes 96..127; only lanes 16..31 (rows 128..143) are kept.
    const bool rem = warp == 3;
    const int q4 = warp & 3;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    const int row = rem ? 112 + lane : q4 * 32 + lane;
    const bool owner = !rem || lane >= 16;  // this thread writes its P/O row
    const uint32_t colS = rem ? kColS2 : kColS;
    float l_prev = 1.f;
    int t_prev = -1, j_prev = -1;

    auto epilogue = [&](int j, int t, float l) -> bool {
      const int ob = j & 1;
      const int fullbar = rem ? kO2Full : kOFull + ob;
      const uint32_t par = rem ? (uint32_t)(j & 1) : (uint32_t)((j >> 1) & 1);
      if (!mbar_wait(BAR(fullbar), par, abort, p.status, 19, kTimeoutNs)) return false;
      tc_fence_after();
      const int w = t / p.H, h = t - w * p.H;
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)w * p.os_w + (int64_t)h * p.os_h +
                           (int64_t)row * p.os_n;
      store_o_row(tmem + lane_addr + (rem ? kColO2 : (ob ? kColO1 : kColO0)), 1.f / l, dst, owner && row < p.N);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(rem ? kO2Free : kOFree + ob));
      return true;
    };

    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++i) {
      const int w = t / p.H;
      uint32_t mbits[5];
      row_mask_bits<kMask>(p, w % p.nW, row, mbits);
      if (!mbar_wait(BAR(kSFull), (uint32_t)(i & 1), abort, p.status, 20, kTimeoutNs)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[9][16];
#pragma unroll
      for (int c = 0; c < 9; ++c) tmem_ld16(tmem + lane_addr + colS + 16 * c, sr[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kSFree));
      if (rem && j_prev >= 0) {  // O2 is single-buffered: drain it before the next PV can start
        if (!epilogue(j_prev, t_prev, l_prev)) { ok = false; break; }
        j_prev = -1;
      }
      uint32_t pk[9][8];
      const float l = softmax_row<kMask>(sr, pk, mbits, p.scale_log2, p.N);
      if (!mbar_wait(BAR(kPEmpty), (uint32_t)((i & 1) ^ 1), abort, p.status, 21, kTimeoutNs)) { ok = false; break; }
      if (owner) store_p_row(sP, rem ? row : row, pk);
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kPFull));
      if (!rem && j_prev >= 0 && !epilogue(j_prev, t_prev, l_prev)) { ok = false; break; }
      j_prev = i;
      t_prev = t;
      l_prev = l;
    }
    if (ok && j_prev >= 0) epilogue(j_prev, t_prev, l_prev);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

// 4D map over (Dh, N, H, Bwin) of one operand, box (inner, 144, 1, 1), 128-byte swizzle,
// out-of-range token rows read as zero.
int make_map(CUtensorMap* map, const void* base, bool f32, int64_t Bwin, int64_t H, int64_t N,
             const int64_t* strides /* window, head, token (elements) */) {
  auto fn = get_encode_fn();
  FA_REQUIRE(fn, FA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t es = f32 ? 4 : 2;
  cuuint64_t dims[4] = {64, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)Bwin};
  cuuint64_t gstr[3] = {(cuuint64_t)(strides[2] * es), (cuuint64_t)(strides[1] * es), (cuuint64_t)(strides[0] * es)};
  cuuint32_t box[4] = {f32 ? 32u : 64u, (cuuint32_t)kMaxN, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                        const_cast<void*>(base), dims, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FA_REQUIRE(r == CUDA_SUCCESS, FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
}

template <int kMask>
int launch_tc_bf16(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                   cudaStream_t s) {
  auto kern = tc::attn_tc_bf16_kernel<kMask>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  kern<<<grid, tc::kThreads, tc::kSmem, s>>>(mq, mk, mv, p);
  return check_launch("attn_tc_bf16_kernel");
}

template <bool kF32, int kMask>
int launch_sync(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                cudaStream_t s) {
  using C = Cfg<kF32>;
  auto kern = attn_sync_kernel<kF32, kMask>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  kern<<<grid, kThreads, C::kSmem, s>>>(mq, mk, mv, p);
  return check_launch("attn_sync_kernel");
}

// FA_ATTN_BF16_KERNEL=mma_sync selects the warp-level kernel for bf16 (kept as a cross-check of
// the tensor-memory kernel); the default is the tcgen05 kernel.
bool use_sync_bf16() {
  const char* e = getenv("FA_ATTN_BF16_KERNEL");
  return e && std::string(e) == "mma_sync";
}

}  // namespace

int* status_ptr() {
  int* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_status) != cudaSuccess) return nullptr;
  return ptr;
}

int run(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh, const void* q, const void* k,
        const void* v, void* out, const int64_t* strides, const uint8_t* mask_u8,
        const uint8_t* group_ids, int64_t nW, float scale, void* stream) {
  FA_REQUIRE(precision == FA_ATTN_BF16 || precision == FA_ATTN_FP32_3XTF32, FA_ERR_INVALID,
             "precision must be FA_ATTN_BF16 or FA_ATTN_FP32_3XTF32");
  FA_REQUIRE(strides, FA_ERR_INVALID, "null stride pointer");
  FA_REQUIRE(Bwin >= 0 && H >= 1 && N >= 1, FA_ERR_INVALID, "invalid attention shape");
  FA_REQUIRE((q && k && v && out) || Bwin == 0, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(Dh == 64, FA_ERR_UNSUPPORTED, "window attention supports head_dim 64");
  FA_REQUIRE(N <= kMaxN, FA_ERR_UNSUPPORTED, "window attention supports N <= 144 tokens");
  FA_REQUIRE(!(mask_u8 && group_ids), FA_ERR_INVALID, "pass at most one of mask_u8 / group_ids");
  FA_REQUIRE(!(mask_u8 || group_ids) || nW >= 1, FA_ERR_INVALID, "nW must be >= 1 with a mask");
  FA_REQUIRE(Bwin * H < ((int64_t)1 << 31), FA_ERR_INVALID, "too many (window, head) tiles");
  if (Bwin == 0) return FA_OK;
  FA_REQUIRE(q && k && v && out, FA_ERR_INVALID, "null tensor pointer");
  const bool f32 = precision == FA_ATTN_FP32_3XTF32;
  const int64_t es = f32 ? 4 : 2;
  const void* ptrs[3] = {q, k, v};
  for (int i = 0; i < 3; ++i) {
    FA_REQUIRE(aligned16(ptrs[i]), FA_ERR_INVALID, "q/k/v must be 16-byte aligned");
    for (int j = 0; j < 3; ++j)
      FA_REQUIRE(strides[3 * i + j] > 0 && (strides[3 * i + j] * es) % 16 == 0, FA_ERR_INVALID,
                 "q/k/v strides must be positive multiples of 16 bytes");
  }
  FA_REQUIRE((reinterpret_cast<uintptr_t>(out) & (f32 ? 7 : 3)) == 0 && strides[11] % 2 == 0, FA_ERR_INVALID,
             "out must be 8-byte (fp32) / 4-byte (bf16) aligned with even token stride");
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, f32, Bwin, H, N, strides + 0)) != FA_OK) return rc;
  if ((rc = make_map(&mk, k, f32, Bwin, H, N, strides + 3)) != FA_OK) return rc;
  if ((rc = make_map(&mv, v, f32, Bwin, H, N, strides + 6)) != FA_OK) return rc;
  Params p{};
  p.Bwin = (int)Bwin; p.H = (int)H; p.N = (int)N; p.nW = (int)(nW > 0 ? nW : 1);
  p.num_tiles = (int)(Bwin * H);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.mask = mask_u8 ? mask_u8 : group_ids;
  p.out = out;
  p.os_w = strides[9]; p.os_h = strides[10]; p.os_n = strides[11];
  p.status = status_ptr();
  FA_REQUIRE(p.status, FA_ERR_CUDA, "cannot resolve the attention status word");
  cudaStream_t s = (cudaStream_t)stream;
  const int kind = mask_u8 ? kMaskU8 : (group_ids ? kGroups : kNoMask);
  if (f32) {
    if (kind == kGroups) return launch_sync<true, kGroups>(mq, mk, mv, p, s);
    if (kind == kMaskU8) return launch_sync<true, kMaskU8>(mq, mk, mv, p, s);
    return launch_sync<true, kNoMask>(mq, mk, mv, p, s);
  }
  // The tensor-memory kernel stores 16-byte output rows: needs 16-byte aligned rows.
  const bool out16 = aligned16(out) && p.os_w % 8 == 0 && p.os_h % 8 == 0 && p.os_n % 8 == 0;
  if (use_sync_bf16() || !out16) {
    if (kind == kGroups) return launch_sync<false, kGroups>(mq, mk, mv, p, s);
    if (kind == kMaskU8) return launch_sync<false, kMaskU8>(mq, mk, mv, p, s);
    return launch_sync<false, kNoMask>(mq, mk, mv, p, s);
  }
  if (kind == kGroups) return launch_tc_bf16<kGroups>(mq, mk, mv, p, s);
  if (kind == kMaskU8) return launch_tc_bf16<kMaskU8>(mq, mk, mv, p, s);
  return launch_tc_bf16<kNoMask>(mq, mk, mv, p, s);
}

}  // namespace attn
}  // namespace fa

using namespace fa;

extern "C" int fa_window_attention(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh,
                                   const void* q, const void* k, const void* v, void* out,
                                   const int64_t strides[12], const uint8_t* mask_u8,
                                   const uint8_t* group_ids, int64_t nW, float scale, void* stream) {
  return attn::run(precision, Bwin, H, N, Dh, q, k, v, out, strides, mask_u8, group_ids, nW, scale, stream);
}

extern "C" int fa_window_attention_qkvpacked(int precision, int64_t Bwin, int64_t N, int64_t H,
                                             int64_t Dh, const void* qkv, void* out, int out_layout,
                                             const uint8_t* mask_u8, const uint8_t* group_ids,
                                             int64_t nW, float scale, void* stream) {
  FA_REQUIRE((qkv && out) || Bwin == 0, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(out_layout == FA_LAYOUT_BHND || out_layout == FA_LAYOUT_BNC, FA_ERR_INVALID,
             "out_layout must be FA_LAYOUT_BHND or FA_LAYOUT_BNC");
  FA_REQUIRE(precision == FA_ATTN_BF16 || precision == FA_ATTN_FP32_3XTF32, FA_ERR_INVALID,
             "precision must be FA_ATTN_BF16 or FA_ATTN_FP32_3XTF32");
  const int64_t es = precision == FA_ATTN_FP32_3XTF32 ? 4 : 2;
  const int64_t C = H * Dh;
  const int64_t row = 3 * C;  // (Bwin, N, 3, H, Dh)
  int64_t st[12] = {N * row, Dh, row, N * row, Dh, row, N * row, Dh, row, 0, 0, 0};
  if (out_layout == FA_LAYOUT_BNC) { st[9] = N * C; st[10] = Dh; st[11] = C; }
  else { st[9] = H * N * Dh; st[10] = N * Dh; st[11] = Dh; }
  const char* base = reinterpret_cast<const char*>(qkv);
  return attn::run(precision, Bwin, H, N, Dh, base, base + C * es, base + 2 * C * es, out, st, mask_u8,
                   group_ids, nW, scale, stream);
}

extern "C" int fa_attention_status(int* status_out) {
  FA_REQUIRE(status_out, FA_ERR_INVALID, "null output pointer");
  FA_CUDA(cudaDeviceSynchronize());
  FA_CUDA(cudaMemcpyFromSymbol(status_out, attn::g_status, sizeof(int)));
  return FA_OK;
}

extern "C" int fa_attention_status_reset(void* stream) {
  int* p = attn::status_ptr();
  FA_REQUIRE(p, FA_ERR_CUDA, "cannot resolve the attention status word");
  FA_CUDA(cudaMemsetAsync(p, 0, sizeof(int), (cudaStream_t)stream));
  return FA_OK;
}
