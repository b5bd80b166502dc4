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
//     tiles with ldmatrix (the mma.sync cross-check kernels; the production kernels below, tc
//     and tc32, issue tcgen05 UMMAs into tensor memory instead).
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
// query blocks through the tensor cores: rows 0..127 (M=128) and rows 80..143 (M=64, reusing the
// same shared-memory tiles at an 80-row offset; only its last 16 rows, 128..143, are kept). An M=64
// accumulator fills half of the TMEM lanes, so two of them (O2 of consecutive tiles) share columns.
//
// Warp roles (384 threads, one CTA per SM, persistent over a contiguous range of
// (window, head) tiles, so consecutive tiles of a CTA are the heads of one window):
//   warps 0, 2   TMA producers: Q and K (warp 0) and V (warp 2) of a tile into 3-slot rings
//                (128-byte swizzle); Q/K slots are freed when the S UMMAs finish, V slots after PV.
//   warp 1       owns TMEM (512 columns) and, from one thread, issues the UMMAs:
//                  S  = Q[0:128]  K^T (M=128), S2 = Q[80:144] K^T (M=64)   (N=144, K=64, K-major)
//                  O  = P[0:128]  V   (M=128), O2 = P[80:144] V   (M=64)   (N=64, K=144, V MN-major)
//                in whatever order their inputs become ready (non-blocking barrier tests),
//                signalling completion with tcgen05.commit on mbarriers.
//   warps 3..11  softmax + epilogue, 16 query rows per warp: warps 4..11 take rows 0..127 of S / O
//                (lanes 32*(w%4) + 16*((w-4)/4) .. +15 of the warp's TMEM quarter), warp 3 rows
//                128..143 of S2 / O2 (lanes 96..111 / 112..127). All use 16x256b TMEM loads: a
//                thread holds two rows x 36 keys, a row's 144 keys sit in four threads of one warp,
//                so the row max and sum take two shuffles and no exchange between warps. P goes to
//                shared memory as bf16 in the UMMA A-operand layout; O rows are scaled by 1/sum,
//                staged in the tile's V slot and stored with one bulk tensor copy per tile.
// The shifted-window mask (region ids) goes through the tensor cores: warp 0 writes, once per
// window, one-hot region operands (32-byte swizzle) and the S UMMAs get one more K=16 step that
// raises every same-region logit by 100/scale, which the softmax cannot tell from upstream's -100
// on the other pairs. Windows with one region skip it; id sets it cannot express (more than 16
// regions, ids >= 32) and byte masks fall back to a bit per key. P keys 128..143 live in a
// 32-byte-swizzled chunk to make room. Every wait is bounded (status word + abort flag).
// ------------------------------------------------------------------------------------------
namespace tc {

constexpr int kStages = 3;
constexpr int kQKBytes = 2 * kTileBytes;  // Q and K of a tile (bf16, 144 x 128 B each)
constexpr int kVBytes = kTileBytes;       // V of a tile
constexpr int kStageBytes = kQKBytes + kVBytes;
constexpr int kPChunk = kTileBytes;          // 64 keys x 144 rows of bf16 (128-byte swizzle)
constexpr int kRow32 = kMaxN * 32;           // 144 rows x 32 bytes (16 bf16, 32-byte swizzle)
// P: keys 0-63 and 64-127 in 128-byte-swizzled chunks, keys 128-143 in a 32-byte-swizzled chunk.
constexpr int kPBytes = 2 * kPChunk + kRow32;
// One-hot region operands of a window's mask UMMA (A: queries, B: keys), two windows in flight.
constexpr int kMaskOpBytes = 2 * kRow32;
constexpr int kMaskBytes = 2 * kMaskOpBytes;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColS2 = 160, kColO0 = 320, kColO1 = 384, kColO2 = 448;
constexpr int kNumBars = 34;
constexpr int kSmem = kStages * kStageBytes + kPBytes + kMaskBytes + kNumBars * 8 + 16 + 16 + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
constexpr uint32_t kIdescS = ptx::make_idesc(1, 128, kMaxN, false, false);
constexpr uint32_t kIdescO = ptx::make_idesc(1, 128, 64, false, true);
// Rows 128..143 go through M=64 UMMAs over rows 80..143: A rows 48..63 land in TMEM lanes 96..111
// (lane offset 0) or 112..127 (lane offset 16), so two M=64 accumulators share the same columns.
constexpr uint32_t kIdescS2 = ptx::make_idesc(1, 64, kMaxN, false, false);
constexpr uint32_t kIdescO2 = ptx::make_idesc(1, 64, 64, false, true);
constexpr uint32_t kRowOff80 = 80 * 128;  // 80 rows of a 128-byte-row tile (swizzle-atom aligned)
constexpr uint32_t kRowOff80_32 = 80 * 32;  // the same in a 32-byte-row tile (256-byte atoms)
constexpr uint32_t kLaneHalf = 16u << 16;

enum { kFullQK = 0, kEmptyQK = 3, kFullV = 6, kEmptyV = 9, kSFull = 12, kSFree = 13, kPFull = 14, kPEmpty = 15,
       kOFull = 16, kOFree = 18, kO2Full = 20, kO2Free = 22, kDone = 24,
       kMaskFull = 27, kMaskEmpty = 29, kOStaged = 31 };

// Byte offset of bf16 element e (0..15) of row r in a 32-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw32_offset(int r, int e) {
  return (uint32_t)(r * 32 + ((((e >> 3) ^ (r >> 2)) & 1) << 4) + (e & 7) * 2);
}

// How a window's region mask is applied. The region ids of a window are ranked among the ids
// present (a 32-bit presence set); with 2..16 distinct ids below 32 the mask is one extra UMMA
// K-step: A[q] = bias * onehot(rank(q)), B[k] = onehot(rank(k)), which adds `bias` (= 100 / scale,
// the upstream -100 after scaling, in the raw logit domain) to every same-region pair. Adding it
// to the same-region pairs instead of subtracting it from the others shifts each row of logits by
// a constant, which the softmax cancels. Other id sets fall back to a per-logit mask.
enum { kModeNone = 0, kModeUmma = 1, kModeBits = 2 };

struct WindowRegions {
  uint32_t present;  // bit i: region id i occurs in the window (ids < 32)
  int mode;
};

// Region-id masks (built into the mask UMMA) and masks with a per-logit path.
template <int kMask> constexpr bool kRegions = kMask == kGroups || kMask == kGroupsFit;
template <int kMask> constexpr bool kBitsPath = kMask == kGroups || kMask == kMaskU8;

// Region ids of the tokens k = lane + 32 m (m < 5) of one window; 0xFF past N.
__device__ __forceinline__ void load_window_ids(const uint8_t* gi, int N, int lane, uint32_t (&ids)[5]) {
#pragma unroll
  for (int m = 0; m < 5; ++m) {
    const int k = lane + 32 * m;
    ids[m] = k < N ? (uint32_t)__ldg(gi + k) : 0xFFu;
  }
}

// Mode of a window from ids held by the 32 lanes (same rule as window_regions).
__device__ __forceinline__ WindowRegions regions_from_ids(const uint32_t (&ids)[5]) {
  uint32_t pres = 0u, over = 0u;
#pragma unroll
  for (int m = 0; m < 5; ++m) {
    if (ids[m] == 0xFFu) continue;
    if (ids[m] < 32u) pres |= 1u << ids[m]; else over = 1u;
  }
  pres = __reduce_or_sync(0xffffffffu, pres);
  over = __reduce_or_sync(0xffffffffu, over);
  const int distinct = __popc(pres);
  WindowRegions r;
  r.present = pres;
  r.mode = over || distinct > 16 ? kModeBits : (distinct > 1 ? kModeUmma : kModeNone);
  return r;
}

__device__ __noinline__ void build_onehot(uint32_t sA, int lane, uint32_t present, uint32_t bias_bits, uint32_t i0,
                                          uint32_t i1, uint32_t i2, uint32_t i3, uint32_t i4);

// One 32-byte row of a one-hot operand: `value` (bf16 bits) at element `slot`, zeros elsewhere;
// slot >= 16 writes a zero row.
__device__ __forceinline__ void store_onehot_row(uint32_t tile, int r, int slot, uint32_t value) {
  const uint32_t swz = (uint32_t)((r >> 2) & 1);
  const uint32_t v = value << (16 * (slot & 1));
  const int wi = (slot >> 1) & 3;
  const uint32_t hot = slot < 16 ? (uint32_t)(slot >> 3) : 2u;  // chunk holding the element
  const uint32_t x0 = wi == 0 ? v : 0u, x1 = wi == 1 ? v : 0u, x2 = wi == 2 ? v : 0u, x3 = wi == 3 ? v : 0u;
  const uint32_t row = tile + (uint32_t)r * 32u;
  if (hot == 0u) {
    st_shared_v4(row + ((0u ^ swz) << 4), x0, x1, x2, x3);
    st_shared_v4(row + ((1u ^ swz) << 4), 0u, 0u, 0u, 0u);
  } else if (hot == 1u) {
    st_shared_v4(row + ((0u ^ swz) << 4), 0u, 0u, 0u, 0u);
    st_shared_v4(row + ((1u ^ swz) << 4), x0, x1, x2, x3);
  } else {
    st_shared_v4(row, 0u, 0u, 0u, 0u);
    st_shared_v4(row + 16u, 0u, 0u, 0u, 0u);
  }
}

// The one-hot A and B operands of one window, out of line so that the producer's loop stays small.
__device__ __noinline__ void build_onehot(uint32_t sA, int lane, uint32_t present, uint32_t bias_bits, uint32_t i0,
                                          uint32_t i1, uint32_t i2, uint32_t i3, uint32_t i4) {
  const uint32_t sB = sA + kRow32;
  const uint32_t ids[5] = {i0, i1, i2, i3, i4};
#pragma unroll 1
  for (int m = 0; m < 5; ++m) {
    const int r = lane + 32 * m;
    if (r < kMaxN) {
      const uint32_t id = m == 0 ? ids[0] : m == 1 ? ids[1] : m == 2 ? ids[2] : m == 3 ? ids[3] : ids[4];
      const int slot = id < 32u ? __popc(present & ((1u << id) - 1u)) : 16;
      store_onehot_row(sA, r, slot, bias_bits);
      store_onehot_row(sB, r, slot, 0x3F80u);
    }
  }
}

__device__ __forceinline__ uint32_t nibble_of_bytes(uint32_t ne) {
  return (ne & 1u) | ((ne >> 7) & 2u) | ((ne >> 14) & 4u) | ((ne >> 21) & 8u);
}

// Masked keys of one row as a bit per key (bit j set = masked), keys 0..143 in 5 words. Reads the
// window's region ids (or the row of the u8 mask) 16 bytes at a time when N is a multiple of 16.
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
#pragma unroll
      for (int v = 0; v < kMaxN / 16; ++v) {
        if (v >= p.N / 16) break;
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

// 72 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld72(uint32_t taddr, uint32_t (&v)[72]) {
  uint32_t a[16], b[16], c[16], d[16], e[8];
  tmem_ld16(taddr, a);
  tmem_ld16(taddr + 16, b);
  tmem_ld16(taddr + 32, c);
  tmem_ld16(taddr + 48, d);
  tmem_ld8(taddr + 64, e);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = a[i];
    v[16 + i] = b[i];
    v[32 + i] = c[i];
    v[48 + i] = d[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[64 + i] = e[i];
}

// Logits of 72 keys in the raw (unscaled) domain: s, plus -100/scale where masked, -inf past N.
template <bool kMasked, bool kFullN>
__device__ __forceinline__ float raw_logits72(uint32_t (&v)[72], const uint32_t rel[3], float braw, int kbase,
                                              int N) {
  float mx[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) mx[e] = -INFINITY;
#pragma unroll
  for (int k = 0; k < 72; k += 2) {
    float y[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      y[e] = __uint_as_float(v[k + e]);
      if constexpr (kMasked) {
        if ((rel[(k + e) >> 5] >> ((k + e) & 31)) & 1u) y[e] += braw;
      }
      if constexpr (!kFullN) {
        if (kbase + k + e >= N) y[e] = -INFINITY;
      }
      v[k + e] = __float_as_uint(y[e]);
    }
    mx[(k >> 1) & 3] = fmax3(mx[(k >> 1) & 3], y[0], y[1]);
  }
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

template <int kMask, bool kFullN>
__global__ void __launch_bounds__(kThreads, 1)
attn_tc_bf16_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sP = sbase + kStages * kStageBytes;
  const uint32_t sMask = sP + kPBytes;  // 256-byte aligned (32-byte-swizzle atoms)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kPBytes + kMaskBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* mask_mode = reinterpret_cast<volatile int*>(tmem_holder + 4);  // per mask buffer
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  __shared__ int abort_flag;

  // Contiguous tile range of this CTA (heads of a window are consecutive tiles).
  const int t_begin = (int)(((int64_t)blockIdx.x * p.num_tiles) / gridDim.x);
  const int t_end = (int)(((int64_t)(blockIdx.x + 1) * p.num_tiles) / gridDim.x);
  const int n_local = t_end - t_begin;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(BAR(kFullQK + s), 1);
      mbar_init(BAR(kEmptyQK + s), 1);
      mbar_init(BAR(kFullV + s), 1);
      mbar_init(BAR(kEmptyV + s), 1);
    }
    mbar_init(BAR(kSFull), 1);
    mbar_init(BAR(kSFree), 9);  // 8 softmax warps + the rows-128..143 warp
    mbar_init(BAR(kPFull), 9);
    mbar_init(BAR(kPEmpty), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kOFull + b), 1);
      mbar_init(BAR(kOFree + b), 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kO2Full + b), 1);
      mbar_init(BAR(kO2Free + b), 1);
    }
    mbar_init(BAR(kDone), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(BAR(kMaskFull + b), 1);
      mbar_init(BAR(kMaskEmpty + b), 1);
    }
    // A tile's output rows are staged in its V slot once PV is done: 8 softmax warps + warp 3.
    for (int s = 0; s < kStages; ++s) mbar_init(BAR(kOStaged + s), 9);
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
  const float braw = kMaskedLog2 / p.scale_log2;  // -100 / scale: the mask bias before scaling

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 loads Q and K, warp 2 loads V ----------------
    // Q/K slots are released as soon as the S UMMAs of their tile complete, V slots after PV, so
    // the Q/K loads of later tiles do not wait for the PV of earlier ones. Warp 0 also builds the
    // one-hot region operands of each window's mask UMMA (all 32 lanes) before its first load.
    const bool qk = warp == 0;
    const int full0 = qk ? kFullQK : kFullV, empty0 = qk ? kEmptyQK : kEmptyV;
    const uint32_t bytes = qk ? (uint32_t)kQKBytes : (uint32_t)kVBytes;
    if (lane == 0) {
      if (qk) {
        tma_prefetch_desc(&tmq);
        tma_prefetch_desc(&tmk);
      } else {
        tma_prefetch_desc(&tmv);
      }
    }
    int last_par[kStages] = {-1, -1, -1};
    int cur_w = -1, wseq = -1;
    // The mask bias of same-region pairs in the raw logit domain, as a bf16 operand value.
    const uint32_t bias_bits = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(-braw));
    // Region ids of the next window, loaded one window ahead so that classifying a window and
    // writing its operands waits on no memory.
    uint32_t nids[5] = {0xFFu, 0xFFu, 0xFFu, 0xFFu, 0xFFu};
    if constexpr (kRegions<kMask>) {
      if (qk && n_local > 0) load_window_ids(p.mask + (int64_t)((t_begin / p.H) % p.nW) * p.N, p.N, lane, nids);
    }
    for (int i = 0; i < n_local; ++i) {
      const int t = t_begin + i;
      const int w = t / p.H, h = t - w * p.H;
      if constexpr (kRegions<kMask>) {
        if (qk && w != cur_w) {
          cur_w = w;
          ++wseq;
          const int mb = wseq & 1;
          const uint32_t u = (uint32_t)(wseq >> 1);
          uint32_t ids[5];
#pragma unroll
          for (int m = 0; m < 5; ++m) ids[m] = nids[m];
          if ((w + 1) * p.H < t_begin + n_local)
            load_window_ids(p.mask + (int64_t)((w + 1) % p.nW) * p.N, p.N, lane, nids);
          WindowRegions wr = regions_from_ids(ids);
          if constexpr (kMask == kGroupsFit) {
            if (wr.mode == kModeBits) {  // the caller's promise does not hold: report, leave unmasked
              if (lane == 0) atomicCAS(p.status, 0, 28);
              wr.mode = kModeNone;
            }
          }
          int okw = 1;
          if (lane == 0) okw = mbar_wait(BAR(kMaskEmpty + mb), (u & 1u) ^ 1u, abort, p.status, 13, kTimeoutNs);
          if (!__shfl_sync(0xffffffffu, okw, 0)) break;
          if (wr.mode == kModeUmma) {
            build_onehot(sMask + (uint32_t)mb * kMaskOpBytes, lane, wr.present, bias_bits, ids[0], ids[1], ids[2],
                         ids[3], ids[4]);
            fence_proxy_async_shared();
          }
          if (lane == 0) mask_mode[mb] = wr.mode;
          __syncwarp();
          if (lane == 0) mbar_arrive(BAR(kMaskFull + mb));
        }
      }
      int ok = 1;
      if (lane == 0) {
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)((i / kStages) & 1);
        bool ready;
        if (qk) {
          ready = mbar_wait(BAR(empty0 + s), ph ^ 1u, abort, p.status, 11, kTimeoutNs);
        } else {
          // The V slot still holds the staged output of tile i - kStages: store it, and wait
          // until the copy has read the slot, before loading V of tile i into it.
          ready = true;
          if (i >= kStages) {
            const int jo = i - kStages, to = t_begin + jo;
            ready = mbar_wait(BAR(kOStaged + s), (uint32_t)((jo / kStages) & 1), abort, p.status, 14, kTimeoutNs);
            if (ready) {
              tma_store_4d(&tmo, sbase + s * kStageBytes + (uint32_t)kQKBytes, 0, 0, to % p.H, to / p.H);
              bulk_commit_group();
              bulk_wait_group_read0();
            }
          }
        }
        if (!ready) {
          ok = 0;
        } else {
          const uint32_t dst = sbase + s * kStageBytes + (qk ? 0u : (uint32_t)kQKBytes);
          mbar_arrive_expect_tx(BAR(full0 + s), bytes);
          if (qk) {
            tma_load_4d(dst, &tmq, BAR(full0 + s), 0, 0, h, w);
            tma_load_4d(dst + kTileBytes, &tmk, BAR(full0 + s), 0, 0, h, w);
          } else {
            tma_load_4d(dst, &tmv, BAR(full0 + s), 0, 0, h, w);
          }
          last_par[s] = (int)ph;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
    if (lane == 0) {
      int no_abort = 0;
      for (int s = 0; s < kStages; ++s)
        if (last_par[s] >= 0) mbar_wait(BAR(full0 + s), (uint32_t)last_par[s], &no_abort, p.status, 12, kTimeoutNs);
      if (!qk) {
        // Outputs of the last tiles (bounded waits; skipped after an abort).
        for (int jo = n_local > kStages ? n_local - kStages : 0; jo < n_local; ++jo) {
          const int s = jo % kStages, to = t_begin + jo;
          if (!mbar_wait(BAR(kOStaged + s), (uint32_t)((jo / kStages) & 1), abort, p.status, 15, kTimeoutNs)) break;
          tma_store_4d(&tmo, sbase + s * kStageBytes + (uint32_t)kQKBytes, 0, 0, to % p.H, to / p.H);
          bulk_commit_group();
        }
        bulk_wait_group0();
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer (event loop) ----------------
    if (lane == 0) {
      int ns = 0, npv = 0;
      uint64_t t_last = cycles();
      uint32_t idle = 0;
      // Window sequence number (within this CTA) of tile ns: selects the mask buffer.
      int s_wseq = 0;
      int s_w = t_begin / p.H;
      while (npv < n_local) {
        bool progressed = false;
        if (ns < n_local) {
          const int s = ns % kStages;
          const int mb = s_wseq & 1;
          bool mask_ready = true;
          if constexpr (kRegions<kMask>)
            mask_ready = mbar_test_wait(BAR(kMaskFull + mb), (uint32_t)((s_wseq >> 1) & 1));
          if (mask_ready && mbar_test_wait(BAR(kFullQK + s), (uint32_t)((ns / kStages) & 1)) &&
              mbar_test_wait(BAR(kSFree), (uint32_t)((ns & 1) ^ 1))) {
            tc_fence_after();
            const uint32_t sQ = sbase + s * kStageBytes, sK = sQ + kTileBytes;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t b = desc_sw128(sK + k * 32, 16, 1024);
              umma_f16(tmem + kColS, desc_sw128(sQ + k * 32, 16, 1024), b, kIdescS, k > 0 ? 1u : 0u);
              umma_f16(tmem + kColS2, desc_sw128(sQ + kRowOff80 + k * 32, 16, 1024), b, kIdescS2, k > 0 ? 1u : 0u);
            }
            const int t_next = t_begin + ns + 1;
            const bool last_of_window = ns + 1 == n_local || t_next / p.H != s_w;
            if constexpr (kRegions<kMask>) {
              if (mask_mode[mb] == kModeUmma) {
                // S += onehot(query region) * bias . onehot(key region)^T (one K=16 step).
                const uint32_t sA = sMask + (uint32_t)mb * kMaskOpBytes, sB = sA + kRow32;
                const uint64_t b = desc_sw32(sB, 256);
                umma_f16(tmem + kColS, desc_sw32(sA, 256), b, kIdescS, 1u);
                umma_f16(tmem + kColS2, desc_sw32(sA + kRowOff80_32, 256), b, kIdescS2, 1u);
              }
            }
            umma_commit(BAR(kSFull));
            umma_commit(BAR(kEmptyQK + s));
            if constexpr (kRegions<kMask>) {
              if (last_of_window) umma_commit(BAR(kMaskEmpty + mb));
            }
            if (last_of_window) {
              ++s_wseq;
              s_w = t_next / p.H;
            }
            ++ns;
            progressed = true;
          }
        }
        if (npv < ns) {
          const int j = npv, s = j % kStages, ob = j & 1;
          if (mbar_test_wait(BAR(kPFull), (uint32_t)(j & 1)) &&
              mbar_test_wait(BAR(kFullV + s), (uint32_t)((j / kStages) & 1)) &&
              mbar_test_wait(BAR(kOFree + ob), (uint32_t)(((j >> 1) & 1) ^ 1)) &&
              mbar_test_wait(BAR(kO2Free + ob), (uint32_t)(((j >> 1) & 1) ^ 1))) {
            tc_fence_after();
            const uint32_t sV = sbase + s * kStageBytes + kQKBytes;
            const uint32_t dO = tmem + (ob ? kColO1 : kColO0);
            const uint32_t dO2 = tmem + kColO2 + (ob ? kLaneHalf : 0u);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t pa = sP + (k >> 2) * kPChunk + (k & 3) * 32;
              const uint64_t b = desc_sw128(sV + k * 2048, kTileBytes, 1024);
              umma_f16(dO, desc_sw128(pa, 16, 1024), b, kIdescO, k > 0 ? 1u : 0u);
              umma_f16(dO2, desc_sw128(pa + kRowOff80, 16, 1024), b, kIdescO2, k > 0 ? 1u : 0u);
            }
            {  // keys 128..143: the 32-byte-swizzled P chunk
              const uint32_t pa = sP + 2 * kPChunk;
              const uint64_t b = desc_sw128(sV + 8 * 2048, kTileBytes, 1024);
              umma_f16(dO, desc_sw32(pa, 256), b, kIdescO, 1u);
              umma_f16(dO2, desc_sw32(pa + kRowOff80_32, 256), b, kIdescO2, 1u);
            }
            umma_commit(BAR(kOFull + ob));
            umma_commit(BAR(kO2Full + ob));
            umma_commit(BAR(kPEmpty));
            ++npv;
            progressed = true;
          }
        }
        if (progressed) {
          idle = 0;
          t_last = cycles();
        } else if ((++idle & 63u) == 0) {
          if (*abort) break;
          if (cycles() - t_last > ns_to_cycles(kTimeoutNs)) {
            atomicCAS(p.status, 0, 16);
            *abort = 1;
            break;
          }
        }
      }
      umma_commit(BAR(kDone));
      int no_abort = 0;
      mbar_wait(BAR(kDone), 0, &no_abort, p.status, 17, kTimeoutNs);
    }
  } else {
    // ---------------- softmax + output rows, 16 rows per warp (16x256b TMEM loads) ----------------
    // Warps 4..11 take rows 0..127 of the M=128 S and O accumulators: warp w reads lanes
    // 32*(w%4) + 16*((w-4)/4) .. +15 of its TMEM quarter. Warp 3 takes rows 128..143 from the M=64
    // S2 / O2 blocks over rows 80..143 (A rows 48..63 land in lanes 96..111). A thread holds rows
    // ra = base + lane/4 and rb = ra + 8, 36 keys each; a row's 144 keys sit in 4 threads of one
    // warp, so its max and sum take two shuffles and no exchange between warps.
    const bool rem = warp == 3;
    const int t0 = lane & 3, t1 = lane >> 2;
    const int rbase = rem ? 128 : 32 * (warp & 3) + 16 * ((warp - 4) >> 2);
    const int ra = rbase + t1, rb = rbase + 8 + t1;
    const uint32_t lane_addr = rem ? (96u << 16) : ((uint32_t)rbase << 16);
    const uint32_t s_col = rem ? kColS2 : kColS;
    int cached_w = -1, wseq = -1;
    uint32_t ta = 0, tb = 0, kp[18];
    bool wmask = false;
#pragma unroll
    for (int j = 0; j < 18; ++j) kp[j] = 0u;
    float la_prev = 1.f, lb_prev = 1.f;
    int t_prev = -1, j_prev = -1;

    auto epilogue_rem = [&](int j, int t, float la, float lb) -> bool {
      const int ob = j & 1;
      if (!mbar_wait(BAR((rem ? kO2Full : kOFull) + ob), (uint32_t)((j >> 1) & 1), abort, p.status, rem ? 23 : 19,
                     kTimeoutNs))
        return false;
      tc_fence_after();
      uint32_t o[32];
      const uint32_t o_col = rem ? kColO2 + (ob ? kLaneHalf : 0u) : (ob ? kColO1 : kColO0);
      tmem_ld_16x256b_r32(tmem + lane_addr + o_col, o);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR((rem ? kO2Free : kOFree) + ob));
      // Rows ra, rb of the tile's output, O / l in bf16, staged in the tile's V slot (128-byte
      // swizzle); warp 2 writes the whole tile with one bulk tensor store (rows past N dropped).
      (void)t;
      const float ia = 1.f / la, ib = 1.f / lb;
      const float2 ia2 = make_float2(ia, ia), ib2 = make_float2(ib, ib);
      const uint32_t stg = sbase + (j % kStages) * kStageBytes + (uint32_t)kQKBytes;
#pragma unroll
      for (int jd = 0; jd < 8; ++jd) {
        const float2 ya = __fmul2_rn(make_float2(__uint_as_float(o[4 * jd]), __uint_as_float(o[4 * jd + 1])), ia2);
        const float2 yb = __fmul2_rn(make_float2(__uint_as_float(o[4 * jd + 2]), __uint_as_float(o[4 * jd + 3])), ib2);
        st_shared_u32(stg + (uint32_t)ra * 128u + (uint32_t)(((jd ^ (ra & 7)) & 7) << 4) + 4u * t0,
                      pack_bf16x2(ya.x, ya.y));
        st_shared_u32(stg + (uint32_t)rb * 128u + (uint32_t)(((jd ^ (rb & 7)) & 7) << 4) + 4u * t0,
                      pack_bf16x2(yb.x, yb.y));
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kOStaged + j % kStages));
      return true;
    };

    bool ok = true;
    for (int i = 0; i < n_local; ++i) {
      const int t = t_begin + i;
      if constexpr (kBitsPath<kMask>) {  // per-logit masks only
        const int w = t / p.H;
        if (w != cached_w) {
          cached_w = w;
          ++wseq;
          const int mw = w % p.nW;
          if constexpr (kMask == kGroupsFit) {
            wmask = false;  // the mask is in S (mask UMMA): nothing to do per window
          } else if constexpr (kMask == kGroups) {
            const uint8_t* gi = p.mask + (int64_t)mw * p.N;
            // Region masks of up to 16 regions are already in S (mask UMMA); the producer
            // classified the window before its first load.
            if (!mbar_wait(BAR(kMaskFull + (wseq & 1)), (uint32_t)((wseq >> 1) & 1), abort, p.status, 27,
                           kTimeoutNs)) { ok = false; break; }
            const int mode = mask_mode[wseq & 1];
            wmask = false;
            if (mode == kModeBits) {
            ta = ra < p.N ? __ldg(gi + ra) : 0u;
            tb = rb < p.N ? __ldg(gi + rb) : 0u;
            uint32_t any = 0;
#pragma unroll
            for (int j = 0; j < 18; ++j) {
              const int key = 8 * j + 2 * t0;
              const uint32_t lo = key < p.N ? __ldg(gi + key) : ta;
              const uint32_t hi = key + 1 < p.N ? __ldg(gi + key + 1) : ta;
              kp[j] = lo | (hi << 8);
              any |= (lo != ta) | (hi != ta) | (lo != tb) | (hi != tb);
            }
            // A window with one region has no masked pair; this is uniform over the window.
            wmask = __any_sync(0xffffffffu, any != 0u);
            }
          } else {
            wmask = true;
          }
        }
      }
      if (!mbar_wait(BAR(kSFull), (uint32_t)(i & 1), abort, p.status, 20, kTimeoutNs)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[72];
      {
        uint32_t a[64], b[8];
        tmem_ld_16x256b_r64(tmem + lane_addr + s_col, a);
        tmem_ld_16x256b_r8(tmem + lane_addr + s_col + 128, b);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = a[k];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[64 + k] = b[k];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kSFree));
      // v[4j + {0,1}] = row ra, keys 8j + 2t0 + {0,1}; v[4j + {2,3}] = row rb, same keys.
      // The per-logit mask runs in its own loop, behind one warp-uniform branch, so windows whose
      // mask is already in S (or that have none) execute none of it.
      float mxa = -INFINITY, mxb = -INFINITY;
      if (kBitsPath<kMask> && wmask) {
#pragma unroll
        for (int j = 0; j < 18; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = 8 * j + 2 * t0 + e;
            float ya = __uint_as_float(v[4 * j + e]), yb = __uint_as_float(v[4 * j + 2 + e]);
            if constexpr (kMask == kGroups) {
              const uint32_t kg = (kp[j] >> (8 * e)) & 0xffu;
              if (kg != ta) ya += braw;
              if (kg != tb) yb += braw;
            } else if constexpr (kMask == kMaskU8) {
              const uint8_t* mr = p.mask + (int64_t)(cached_w % p.nW) * p.N * p.N;
              if (key < p.N && ra < p.N && __ldg(mr + (int64_t)ra * p.N + key)) ya += braw;
              if (key < p.N && rb < p.N && __ldg(mr + (int64_t)rb * p.N + key)) yb += braw;
            }
            if (!kFullN && key >= p.N) {
              ya = -INFINITY;
              yb = -INFINITY;
            }
            v[4 * j + e] = __float_as_uint(ya);
            v[4 * j + 2 + e] = __float_as_uint(yb);
          }
          mxa = fmax3(mxa, __uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]));
          mxb = fmax3(mxb, __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 18; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = 8 * j + 2 * t0 + e;
            float ya = __uint_as_float(v[4 * j + e]), yb = __uint_as_float(v[4 * j + 2 + e]);
            if (!kFullN && key >= p.N) {
              ya = -INFINITY;
              yb = -INFINITY;
            }
            v[4 * j + e] = __float_as_uint(ya);
            v[4 * j + 2 + e] = __float_as_uint(yb);
          }
          mxa = fmax3(mxa, __uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]));
          mxb = fmax3(mxb, __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        }
      }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float c = p.scale_log2, mca = -mxa * c, mcb = -mxb * c;
      const float2 c2 = make_float2(c, c), ma2 = make_float2(mca, mca), mb2 = make_float2(mcb, mcb);
      float2 la2 = make_float2(0.f, 0.f), lb2 = make_float2(0.f, 0.f);
      uint32_t pa[18], pb[18];
#pragma unroll
      for (int j = 0; j < 18; ++j) {
        const float2 ya = __ffma2_rn(make_float2(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1])), c2, ma2);
        const float2 yb =
            __ffma2_rn(make_float2(__uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])), c2, mb2);
        const float a0 = ex2(ya.x), a1 = ex2(ya.y), b0 = ex2(yb.x), b1 = ex2(yb.y);
        la2 = __fadd2_rn(la2, make_float2(a0, a1));
        lb2 = __fadd2_rn(lb2, make_float2(b0, b1));
        pa[j] = pack_bf16x2(a0, a1);
        pb[j] = pack_bf16x2(b0, b1);
      }
      float la = la2.x + la2.y, lb = lb2.x + lb2.y;
      la += __shfl_xor_sync(0xffffffffu, la, 1);
      la += __shfl_xor_sync(0xffffffffu, la, 2);
      lb += __shfl_xor_sync(0xffffffffu, lb, 1);
      lb += __shfl_xor_sync(0xffffffffu, lb, 2);
      if (!mbar_wait(BAR(kPEmpty), (uint32_t)((i & 1) ^ 1), abort, p.status, 21, kTimeoutNs)) { ok = false; break; }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t off = (j >> 3) * kPChunk + (uint32_t)(4 * t0);
        st_shared_u32(sP + off + ra * 128 + (((j & 7) ^ (ra & 7)) << 4), pa[j]);
        st_shared_u32(sP + off + rb * 128 + (((j & 7) ^ (rb & 7)) << 4), pb[j]);
      }
#pragma unroll
      for (int j = 16; j < 18; ++j) {  // keys 128..143: the 32-byte-swizzled chunk
        st_shared_u32(sP + 2 * kPChunk + sw32_offset(ra, (j & 1) * 8 + 2 * t0), pa[j]);
        st_shared_u32(sP + 2 * kPChunk + sw32_offset(rb, (j & 1) * 8 + 2 * t0), pb[j]);
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kPFull));
      if (j_prev >= 0 && !epilogue_rem(j_prev, t_prev, la_prev, lb_prev)) { ok = false; break; }
      j_prev = i;
      t_prev = t;
      la_prev = la;
      lb_prev = lb;
    }
    if (ok && j_prev >= 0) epilogue_rem(j_prev, t_prev, la_prev, lb_prev);
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
// FP32 I/O kernel on the 5th-generation tensor cores: 3xTF32 with tcgen05.mma kind::tf32.
//
// Every operand x is split as x = hi + lo: hi is x with its 13 low mantissa bits cleared, lo = x - hi
// (exact in fp32). kind::tf32 truncates its fp32 inputs to tf32 (measured on B200: 1 + 3*2^-12 is
// taken as 1), so x itself serves as hi and only lo is stored; the tensor core truncates lo too. A product a.b accumulates a_lo.b_hi + a_hi.b_lo + a_hi.b_hi in fp32; the dropped
// a_lo.b_lo term and the rounding of lo leave it within about 2^-21 of the fp32 product, the
// accuracy of the warp-level 3xTF32 kernel above, unlike the upstream 1xTF32 QK^T + BF16 PV
// kernel (ops/cute/_kernel_fp32.py:491-493).
//
// One (window, head) tile at a time per CTA, single-buffered: shared memory holds hi and lo of
// Q and K (144 x 32-float blocks with 128-byte swizzle, as TMA writes them) and of V^T. kind::tf32
// takes K-major operands only (an MN-major tf32 operand yields zeros on B200), so V, which TMA
// lands in the V^T lo slot as soon as the previous tile's PV products are done, is transposed in
// registers by the split warps into 64 x 144 K-major blocks: keys 0..127 with 128-byte swizzle,
// keys 128..143 with 32-byte swizzle.
//   S  = Q K^T  rows 0..127 (M=128) and rows 80..143 (M=64), N=144, 8 K-steps x 3 products, both
//               operands K-major in shared memory;
//   P           the softmax warps write P_hi over S in TMEM (tcgen05.st), then P_lo over P_hi once
//               the two P_hi products have run;
//   O  = P V    M=128, N=64, 18 K-steps x 3 products, A (P) from TMEM, V^T in shared memory.
// A TMEM A operand must sit in the same lanes as its accumulator. The M=64 block (rows 128..143 are
// its rows 48..63) fills half of the lanes: its S and P_hi use the first lane half (lanes 0-15 of
// each 32-lane group) of columns 224..367 with their O accumulator in the first lane half of
// 384..447, and its P_lo uses the second lane half of the same columns with a second O accumulator
// there; the epilogue adds the two. Its products therefore run in one go, while the softmax warps
// write the M=128 block's P_lo. TMEM columns: S / P 0..143, O 160..223, M=64 block 224..447.
// Warp roles (512 threads, one CTA per SM, a contiguous range of tiles per CTA):
//   warp 0       TMA: Q and K of a tile once the previous tile's S products are done, V once its
//                PV products are done;
//   warp 1       TMEM owner and UMMA issuer (one thread, blocking on each input). A tf32 UMMA
//                costs about 74 cycles at N=144 and has a floor near 48 cycles at N=64, so the
//                issue sequence is unrolled with precomputed descriptors, and the M=128 S block is
//                committed before the M=64 one so that the softmax overlaps the latter;
//   warp 3       rows 128..143 (16x256b TMEM shape, two rows per thread, quad reductions);
//   warps 4..11  rows 0..127: two warpgroups of 72 keys per row (row max / sum exchanged through
//                shared memory), then the output rows (32 columns per warpgroup);
//   warps 12..15 write the lo parts of Q and K; transpose V into its hi and lo parts.
// Every wait is bounded (status word + abort flag); warp 2 only takes part in the set-up.
// ------------------------------------------------------------------------------------------
namespace tc32 {

constexpr int kBlk = kTileBytes;  // 144 rows x 32 floats (128 bytes)
constexpr int kMat = 2 * kBlk;    // one 144 x 64 fp32 operand
// Raw / hi blocks of Q and K are adjacent, and so are their lo blocks: one split pass covers both.
// V lands in the V^T lo slot (kOffVl); its transposed hi and lo go to kOffVh / kOffVl.
constexpr int kOffQh = 0, kOffKh = kMat, kOffQl = 2 * kMat, kOffKl = 3 * kMat, kOffVh = 4 * kMat, kOffVl = 5 * kMat;
// V^T (64 rows of head dims): keys 32b..32b+31 in 128-byte-swizzled blocks b = 0..3 (8 KB each),
// keys 128..135 and 136..143 in 32-byte-swizzled blocks (2 KB each); kMat bytes in all.
constexpr int kVtSw32 = 4 * 64 * 128;
constexpr int kXchgBytes = 2 * 2 * 128 * 4;  // {max, sum} x warpgroup x row
constexpr int kThreads = 512;
constexpr int kConvThreads = 128;             // warps 12..15
// Registers per thread after the per-warpgroup split (launched at 128 for 512 threads).
constexpr uint32_t kRegsLaunch = 128, kRegsSoftmax = 136, kRegsConvert = 112;
static_assert(4 * 32 * kRegsLaunch + 8 * 32 * kRegsSoftmax + 4 * 32 * kRegsConvert == kThreads * kRegsLaunch,
              "register split must add up to the launch budget");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 160, kColSR = 224, kColOR = 384;
constexpr uint32_t kLaneHalf = 16u << 16;  // second lane half of an M=64 block
constexpr uint32_t kRowOff80 = 80 * 128;
constexpr uint32_t kHiMask = 0xFFFFE000u;     // sign, exponent and the 10 mantissa bits of tf32
enum { kQKFull = 0, kQKConv, kVFull, kVRead, kVConv, kSFull, kSRemFull, kPFull, kHiDone, kPLoFull, kPRemFull,
       kOFull, kOFree, kORemFull, kORemFree, kPVDone, kXMax, kXSum, kDone, kNumBars };
constexpr int kSmem = 6 * kMat + kXchgBytes + kNumBars * 8 + 16 + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
constexpr uint32_t kIdS = ptx::make_idesc(2, 128, kMaxN, false, false);
constexpr uint32_t kIdSR = ptx::make_idesc(2, 64, kMaxN, false, false);
constexpr uint32_t kIdO = ptx::make_idesc(2, 128, 64, false, false);
constexpr uint32_t kIdOR = ptx::make_idesc(2, 64, 64, false, false);

__device__ __forceinline__ uint32_t hi_of(uint32_t x) { return x & kHiMask; }
__device__ __forceinline__ uint32_t lo_of(uint32_t x) {
  return __float_as_uint(__uint_as_float(x) - __uint_as_float(x & kHiMask));
}

// Byte offset of the 4 keys key..key+3 (key % 4 == 0) of head dim d in the V^T layout.
__device__ __forceinline__ uint32_t vt_off(int d, int key) {
  if (key < 128)
    return (uint32_t)((key >> 5) * 8192 + d * 128 + ((((key & 31) >> 2) ^ (d & 7)) << 4));
  const int k2 = key - 128;
  return (uint32_t)(kVtSw32 + (k2 >> 3) * 2048 + d * 32 + ((((k2 & 7) >> 2) ^ ((d >> 2) & 1)) << 4));
}

// B operand descriptor of PV K-step j (keys 8j..8j+7) of a V^T buffer, from the descriptors of its
// first 128-byte-swizzled block (d128) and first 32-byte-swizzled block (d32): the start address
// field counts 16-byte units, so moving inside the buffer adds offset / 16.
__device__ __forceinline__ uint64_t vt_desc(uint64_t d128, uint64_t d32, int j) {
  return j < 16 ? d128 + (uint64_t)(((j >> 2) * 8192 + (j & 3) * 32) >> 4) : d32 + (uint64_t)(((j - 16) * 2048) >> 4);
}

// lo of `bytes` of landed operand blocks (the landed values are their own hi); 16 bytes per
// thread and step.
__device__ __forceinline__ void split_blocks(uint32_t raw, uint32_t lo, int bytes, int ct) {
#pragma unroll 4
  for (int o = ct * 16; o < bytes; o += kConvThreads * 16) {
    uint32_t a, b, c, d;
    ld_shared_v4(raw + (uint32_t)o, a, b, c, d);
    st_shared_v4(lo + (uint32_t)o, lo_of(a), lo_of(b), lo_of(c), lo_of(d));
  }
}

template <int kMask, bool kFullN>
__global__ void __launch_bounds__(kThreads, 1)
attn_tc_tf32_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  float* xchg = reinterpret_cast<float*>(smem + 6 * kMat);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kMat + kXchgBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int slot) -> uint32_t { return bar0 + 8u * (uint32_t)slot; };
  __shared__ int abort_flag;

  const int t_begin = (int)(((int64_t)blockIdx.x * p.num_tiles) / gridDim.x);
  const int t_end = (int)(((int64_t)(blockIdx.x + 1) * p.num_tiles) / gridDim.x);
  const int n_local = t_end - t_begin;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int b = 0; b < kNumBars; ++b) {
      const uint32_t count = (b == kQKConv || b == kVRead || b == kVConv) ? 4u
                             : (b == kPFull || b == kPLoFull || b == kOFree || b == kXMax || b == kXSum) ? 8u
                                                                                                           : 1u;
      mbar_init(BAR(b), count);
    }
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
  const float braw = kMaskedLog2 / p.scale_log2;  // -100 / scale: the mask bias before scaling

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      int qk_issued = 0, v_issued = 0;
      for (int i = 0; i < n_local; ++i) {
        const int t = t_begin + i, w = t / p.H, h = t - w * p.H;
        const uint32_t prev = (uint32_t)((i & 1) ^ 1);  // completion of tile i-1 (free on tile 0)
        if (!mbar_wait(BAR(kSRemFull), prev, abort, p.status, 41, kTimeoutNs)) break;
        mbar_arrive_expect_tx(BAR(kQKFull), 2 * kMat);
        tma_load_4d(sbase + kOffQh, &tmq, BAR(kQKFull), 0, 0, h, w);
        tma_load_4d(sbase + kOffQh + kBlk, &tmq, BAR(kQKFull), 32, 0, h, w);
        tma_load_4d(sbase + kOffKh, &tmk, BAR(kQKFull), 0, 0, h, w);
        tma_load_4d(sbase + kOffKh + kBlk, &tmk, BAR(kQKFull), 32, 0, h, w);
        ++qk_issued;
        if (!mbar_wait(BAR(kPVDone), prev, abort, p.status, 42, kTimeoutNs)) break;
        mbar_arrive_expect_tx(BAR(kVFull), kMat);
        tma_load_4d(sbase + kOffVl, &tmv, BAR(kVFull), 0, 0, h, w);
        tma_load_4d(sbase + kOffVl + kBlk, &tmv, BAR(kVFull), 32, 0, h, w);
        ++v_issued;
      }
      // Never leave with bulk copies in flight (bounded, also after an abort).
      int no_abort = 0;
      if (qk_issued > 0)
        mbar_wait(BAR(kQKFull), (uint32_t)((qk_issued - 1) & 1), &no_abort, p.status, 43, kTimeoutNs);
      if (v_issued > 0)
        mbar_wait(BAR(kVFull), (uint32_t)((v_issued - 1) & 1), &no_abort, p.status, 43, kTimeoutNs);
    }
  } else if (warp >= 12) {
    // ---------------- hi / lo split of each landed tile ----------------
    // Register split (512 threads launched at 128): warpgroup 0 (TMA, issuer, rows 128..143) keeps
    // 128, the two softmax warpgroups take 136, this one gives up 16:
    // 128*128 + 256*136 + 128*112 = 65536 = 512*128.
    warpgroup_reg_dealloc<kRegsConvert>();
    const int ct = threadIdx.x - 12 * 32;
    for (int i = 0; i < n_local; ++i) {
      const uint32_t par = (uint32_t)(i & 1);
      if (!mbar_wait(BAR(kQKFull), par, abort, p.status, 44, kTimeoutNs)) break;
      split_blocks(sbase + kOffQh, sbase + kOffQl, 2 * kMat, ct);
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kQKConv));
      // V landed in the lo slot after the previous tile's PV products (so both V^T slots are
      // free): read this thread's 4 x 4 blocks (4 keys x 4 dims), wait until every split warp has
      // read, then write them transposed. Blocks run along diagonals, so the eight threads of a
      // quarter warp touch eight different 16-byte columns on both sides.
      if (!mbar_wait(BAR(kVFull), par, abort, p.status, 45, kTimeoutNs)) break;
      uint32_t x[5][4][4];
#pragma unroll
      for (int m = 0; m < 5; ++m) {
        const int n = ct + kConvThreads * m;
        if (n < 36 * 16) {
          const int dc = n & 15, kg = ((n >> 4) + dc) % 36;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int key = 4 * kg + r;
            ld_shared_v4(sbase + kOffVl + (uint32_t)((dc >> 3) * kBlk + key * 128 + (((dc & 7) ^ (key & 7)) << 4)),
                         x[m][r][0], x[m][r][1], x[m][r][2], x[m][r][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kVRead));
      if (!mbar_wait(BAR(kVRead), par, abort, p.status, 64, kTimeoutNs)) break;
#pragma unroll
      for (int m = 0; m < 5; ++m) {
        const int n = ct + kConvThreads * m;
        if (n < 36 * 16) {
          const int dc = n & 15, kg = ((n >> 4) + dc) % 36;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t o = vt_off(4 * dc + c, 4 * kg);
            st_shared_v4(sbase + kOffVh + o, hi_of(x[m][0][c]), hi_of(x[m][1][c]), hi_of(x[m][2][c]), hi_of(x[m][3][c]));
            st_shared_v4(sbase + kOffVl + o, lo_of(x[m][0][c]), lo_of(x[m][1][c]), lo_of(x[m][2][c]), lo_of(x[m][3][c]));
          }
        }
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kVConv));
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      const uint32_t tS = tmem + kColS, tSR = tmem + kColSR, tO = tmem + kColO, tOR = tmem + kColOR;
      const uint64_t dQh = desc_sw128(sbase + kOffQh, 16, 1024), dQl = desc_sw128(sbase + kOffQl, 16, 1024);
      const uint64_t dKh = desc_sw128(sbase + kOffKh, 16, 1024), dKl = desc_sw128(sbase + kOffKl, 16, 1024);
      const uint64_t dVh = desc_sw128(sbase + kOffVh, 16, 1024), dVl = desc_sw128(sbase + kOffVl, 16, 1024);
      const uint64_t dVh32 = desc_sw32(sbase + kOffVh + kVtSw32, 256), dVl32 = desc_sw32(sbase + kOffVl + kVtSw32, 256);
      for (int i = 0; i < n_local; ++i) {
        const uint32_t par = (uint32_t)(i & 1), prev = par ^ 1u;
        // S overwrites the P of the previous tile: wait for all of its PV products.
        if (!mbar_wait(BAR(kQKConv), par, abort, p.status, 46, kTimeoutNs)) break;
        if (!mbar_wait(BAR(kPVDone), prev, abort, p.status, 47, kTimeoutNs)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t off = (uint64_t)(((k >> 2) * kBlk + (k & 3) * 32) >> 4);
          umma_tf32(tS, dQl + off, dKh + off, kIdS, k > 0 ? 1u : 0u);
          umma_tf32(tS, dQh + off, dKl + off, kIdS, 1u);
          umma_tf32(tS, dQh + off, dKh + off, kIdS, 1u);
        }
        umma_commit(BAR(kSFull));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t off = (uint64_t)(((k >> 2) * kBlk + (k & 3) * 32) >> 4), a80 = kRowOff80 >> 4;
          umma_tf32(tSR, dQl + off + a80, dKh + off, kIdSR, k > 0 ? 1u : 0u);
          umma_tf32(tSR, dQh + off + a80, dKl + off, kIdSR, 1u);
          umma_tf32(tSR, dQh + off + a80, dKh + off, kIdSR, 1u);
        }
        umma_commit(BAR(kSRemFull));
        if (!mbar_wait(BAR(kPFull), par, abort, p.status, 48, kTimeoutNs)) break;
        if (!mbar_wait(BAR(kVConv), par, abort, p.status, 49, kTimeoutNs)) break;
        if (!mbar_wait(BAR(kOFree), prev, abort, p.status, 50, kTimeoutNs)) break;
        tc_fence_after();
        // P_hi products first, then P_lo (written over P_hi).
#pragma unroll
        for (int j = 0; j < 18; ++j) {
          const uint64_t vh = vt_desc(dVh, dVh32, j);
          const uint64_t vl = vt_desc(dVl, dVl32, j);
          umma_tf32_ts(tO, tS + 8 * j, vl, kIdO, j > 0 ? 1u : 0u);
          umma_tf32_ts(tO, tS + 8 * j, vh, kIdO, 1u);
        }
        umma_commit(BAR(kHiDone));
        // M=64 block: P_hi (first lane half) and P_lo (second lane half), one O accumulator each.
        if (!mbar_wait(BAR(kPRemFull), par, abort, p.status, 51, kTimeoutNs)) break;
        if (!mbar_wait(BAR(kORemFree), prev, abort, p.status, 52, kTimeoutNs)) break;
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 18; ++j) {
          const uint64_t vh = vt_desc(dVh, dVh32, j);
          const uint64_t vl = vt_desc(dVl, dVl32, j);
          umma_tf32_ts(tOR, tSR + 8 * j, vl, kIdOR, j > 0 ? 1u : 0u);
          umma_tf32_ts(tOR, tSR + 8 * j, vh, kIdOR, 1u);
          umma_tf32_ts(tOR + kLaneHalf, tSR + kLaneHalf + 8 * j, vh, kIdOR, j > 0 ? 1u : 0u);
        }
        umma_commit(BAR(kORemFull));
        if (!mbar_wait(BAR(kPLoFull), par, abort, p.status, 62, kTimeoutNs)) break;
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 18; ++j) {
          const uint64_t vh = vt_desc(dVh, dVh32, j);
          umma_tf32_ts(tO, tS + 8 * j, vh, kIdO, 1u);
        }
        umma_commit(BAR(kOFull));
        umma_commit(BAR(kPVDone));
      }
      umma_commit(BAR(kDone));
      int no_abort = 0;
      mbar_wait(BAR(kDone), 0, &no_abort, p.status, 54, kTimeoutNs);
    }
  } else if (warp >= 4) {
    // ---------------- rows 0..127: softmax, P, output rows ----------------
    warpgroup_reg_alloc<kRegsSoftmax>();
    const int g = (warp - 4) >> 2;  // key columns 72g .. 72g+71, output columns 32g .. 32g+31
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q4 * 32) << 16;
    float* xmax = xchg;        // [2][128]
    float* xsum = xchg + 256;  // [2][128]
    int cached_w = -1;
    uint32_t rel[3] = {0u, 0u, 0u};
    bool wmask = false;
    for (int i = 0; i < n_local; ++i) {
      const int t = t_begin + i, w = t / p.H, h = t - w * p.H;
      const uint32_t par = (uint32_t)(i & 1);
      if constexpr (kMask != kNoMask) {
        if (w != cached_w) {
          cached_w = w;
          uint32_t b[5];
          tc::row_mask_bits<kMask>(p, w % p.nW, row, b);
          wmask = (b[0] | b[1] | b[2] | b[3] | b[4]) != 0u;
          const uint32_t w0 = g ? b[2] : b[0], w1 = g ? b[3] : b[1], w2 = g ? b[4] : b[2];
          const uint32_t w3 = g ? 0u : b[3];
          const uint32_t sh = g ? 8u : 0u;
          rel[0] = __funnelshift_r(w0, w1, sh);
          rel[1] = __funnelshift_r(w1, w2, sh);
          rel[2] = __funnelshift_r(w2, w3, sh) & 0xffu;
        }
      }
      if (!mbar_wait(BAR(kSFull), par, abort, p.status, 55, kTimeoutNs)) break;
      tc_fence_after();
      uint32_t v[72];
      tc::tmem_ld72(tmem + lane_addr + kColS + 72 * g, v);
      float pm;
      if (kMask != kNoMask && wmask) pm = tc::raw_logits72<kMask != kNoMask, kFullN>(v, rel, braw, 72 * g, p.N);
      else pm = tc::raw_logits72<false, kFullN>(v, rel, braw, 72 * g, p.N);
      // Each exchange slot is rewritten only after the partner passed the other exchange barrier
      // of the same tile, so one slot per value suffices.
      xmax[g * 128 + row] = pm;
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kXMax));
      if (!mbar_wait(BAR(kXMax), par, abort, p.status, 56, kTimeoutNs)) break;
      const float m = fmaxf(pm, xmax[(g ^ 1) * 128 + row]);
      const float c = p.scale_log2, mc = -m * c;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 72; ++k) {
        const float e = ex2(fmaf(__uint_as_float(v[k]), c, mc));
        l4[k & 3] += e;
        v[k] = __float_as_uint(e);
      }
#pragma unroll
      for (int c8 = 0; c8 < 9; ++c8) {
        uint32_t hv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) hv[e] = hi_of(v[8 * c8 + e]);
        tmem_st8(tmem + lane_addr + kColS + 72 * g + 8 * c8, hv);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kPFull));
      const float pl = (l4[0] + l4[1]) + (l4[2] + l4[3]);
      xsum[g * 128 + row] = pl;
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kXSum));
      if (!mbar_wait(BAR(kXSum), par, abort, p.status, 57, kTimeoutNs)) break;
      const float l = pl + xsum[(g ^ 1) * 128 + row];
      // P_lo over P_hi once the two P_hi products are done.
      if (!mbar_wait(BAR(kHiDone), par, abort, p.status, 63, kTimeoutNs)) break;
      tc_fence_after();
#pragma unroll
      for (int c8 = 0; c8 < 9; ++c8) {
        uint32_t lv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) lv[e] = lo_of(v[8 * c8 + e]);
        tmem_st8(tmem + lane_addr + kColS + 72 * g + 8 * c8, lv);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kPLoFull));
      if (!mbar_wait(BAR(kOFull), par, abort, p.status, 58, kTimeoutNs)) break;
      tc_fence_after();
      uint32_t o[32];
      tmem_ld32(tmem + lane_addr + kColO + 32 * g, o);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kOFree));
      if (row < p.N) {
        const float inv = 1.f / l;
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (int64_t)w * p.os_w +
                                                (int64_t)h * p.os_h + (int64_t)row * p.os_n + 32 * g);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4)
          dst[c4] = make_float4(__uint_as_float(o[4 * c4]) * inv, __uint_as_float(o[4 * c4 + 1]) * inv,
                                __uint_as_float(o[4 * c4 + 2]) * inv, __uint_as_float(o[4 * c4 + 3]) * inv);
      }
    }
  } else if (warp == 3) {
    // ---------------- rows 128..143: M=64 block rows 48..63 ----------------
    // 16x256b layout: v[4j + {0,1}] = row ra, keys 8j + 2t0 + {0,1}; v[4j + {2,3}] = row rb.
    const int t0 = lane & 3, t1 = lane >> 2;
    const int ra = 128 + t1, rb = 136 + t1;
    const uint32_t lane_s = 96u << 16;
    int cached_w = -1;
    uint32_t ta = 0, tb = 0, kp[18];
    bool wmask = false;
#pragma unroll
    for (int j = 0; j < 18; ++j) kp[j] = 0u;
    for (int i = 0; i < n_local; ++i) {
      const int t = t_begin + i, w = t / p.H, h = t - w * p.H;
      const uint32_t par = (uint32_t)(i & 1);
      if constexpr (kMask != kNoMask) {
        if (w != cached_w) {
          cached_w = w;
          if constexpr (kMask == kGroups) {
            const uint8_t* gi = p.mask + (int64_t)(w % p.nW) * p.N;
            ta = ra < p.N ? __ldg(gi + ra) : 0u;
            tb = rb < p.N ? __ldg(gi + rb) : 0u;
            uint32_t any = 0;
#pragma unroll
            for (int j = 0; j < 18; ++j) {
              const int key = 8 * j + 2 * t0;
              const uint32_t lo = key < p.N ? __ldg(gi + key) : ta;
              const uint32_t hi = key + 1 < p.N ? __ldg(gi + key + 1) : ta;
              kp[j] = lo | (hi << 8);
              any |= (lo != ta) | (hi != ta) | (lo != tb) | (hi != tb);
            }
            wmask = __any_sync(0xffffffffu, any != 0u);
          } else {
            wmask = true;
          }
        }
      }
      if (!mbar_wait(BAR(kSRemFull), par, abort, p.status, 59, kTimeoutNs)) break;
      tc_fence_after();
      uint32_t v[72];
      {
        uint32_t a[64], b[8];
        tmem_ld_16x256b_r64(tmem + lane_s + kColSR, a);
        tmem_ld_16x256b_r8(tmem + lane_s + kColSR + 128, b);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = a[k];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[64 + k] = b[k];
      }
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int j = 0; j < 18; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = 8 * j + 2 * t0 + e;
          float ya = __uint_as_float(v[4 * j + e]), yb = __uint_as_float(v[4 * j + 2 + e]);
          if (kMask != kNoMask && wmask) {
            if constexpr (kMask == kGroups) {
              const uint32_t kg = (kp[j] >> (8 * e)) & 0xffu;
              if (kg != ta) ya += braw;
              if (kg != tb) yb += braw;
            } else if constexpr (kMask == kMaskU8) {
              const uint8_t* mr = p.mask + (int64_t)(w % p.nW) * p.N * p.N;
              if (key < p.N && ra < p.N && __ldg(mr + (int64_t)ra * p.N + key)) ya += braw;
              if (key < p.N && rb < p.N && __ldg(mr + (int64_t)rb * p.N + key)) yb += braw;
            }
          }
          if (!kFullN && key >= p.N) {
            ya = -INFINITY;
            yb = -INFINITY;
          }
          v[4 * j + e] = __float_as_uint(ya);
          v[4 * j + 2 + e] = __float_as_uint(yb);
          mxa = fmaxf(mxa, ya);
          mxb = fmaxf(mxb, yb);
        }
      }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float c = p.scale_log2, mca = -mxa * c, mcb = -mxb * c;
      float la = 0.f, lb = 0.f;
#pragma unroll
      for (int j = 0; j < 18; ++j) {
        const float a0 = ex2(fmaf(__uint_as_float(v[4 * j]), c, mca));
        const float a1 = ex2(fmaf(__uint_as_float(v[4 * j + 1]), c, mca));
        const float b0 = ex2(fmaf(__uint_as_float(v[4 * j + 2]), c, mcb));
        const float b1 = ex2(fmaf(__uint_as_float(v[4 * j + 3]), c, mcb));
        la += a0 + a1;
        lb += b0 + b1;
        v[4 * j] = __float_as_uint(a0);
        v[4 * j + 1] = __float_as_uint(a1);
        v[4 * j + 2] = __float_as_uint(b0);
        v[4 * j + 3] = __float_as_uint(b1);
      }
      la += __shfl_xor_sync(0xffffffffu, la, 1);
      la += __shfl_xor_sync(0xffffffffu, la, 2);
      lb += __shfl_xor_sync(0xffffffffu, lb, 1);
      lb += __shfl_xor_sync(0xffffffffu, lb, 2);
      // P_hi over this block's S (first lane half), P_lo in the second lane half.
#pragma unroll
      for (int q = 0; q < 9; ++q) {
        uint32_t hv[8], lv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hv[e] = hi_of(v[8 * q + e]);
          lv[e] = lo_of(v[8 * q + e]);
        }
        tmem_st_16x256b_r8(tmem + lane_s + kColSR + 16 * q, hv);
        tmem_st_16x256b_r8(tmem + lane_s + kLaneHalf + kColSR + 16 * q, lv);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kPRemFull));
      if (!mbar_wait(BAR(kORemFull), par, abort, p.status, 61, kTimeoutNs)) break;
      tc_fence_after();
      uint32_t o[32], o2[32];
      tmem_ld_16x256b_r32(tmem + lane_s + kColOR, o);
      tmem_ld_16x256b_r32(tmem + lane_s + kLaneHalf + kColOR, o2);
      tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) + __uint_as_float(o2[k]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(kORemFree));
      const float ia = 1.f / la, ib = 1.f / lb;
      float* base = reinterpret_cast<float*>(p.out) + (int64_t)w * p.os_w + (int64_t)h * p.os_h + 2 * t0;
      if (ra < p.N) {
        float2* dst = reinterpret_cast<float2*>(base + (int64_t)ra * p.os_n);
#pragma unroll
        for (int jd = 0; jd < 8; ++jd)
          dst[4 * jd] = make_float2(__uint_as_float(o[4 * jd]) * ia, __uint_as_float(o[4 * jd + 1]) * ia);
      }
      if (rb < p.N) {
        float2* dst = reinterpret_cast<float2*>(base + (int64_t)rb * p.os_n);
#pragma unroll
        for (int jd = 0; jd < 8; ++jd)
          dst[4 * jd] = make_float2(__uint_as_float(o[4 * jd + 2]) * ib, __uint_as_float(o[4 * jd + 3]) * ib);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc32

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
  // Output map: the (Dh, N, H, Bwin) view of `out` with its strides, box of one tile.
  CUtensorMap mo;
  const int64_t ostr[3] = {p.os_w, p.os_h, p.os_n};
  int rc = make_map(&mo, p.out, false, p.Bwin, p.H, p.N, ostr);
  if (rc != FA_OK) return rc;
  auto kern = p.N == kMaxN ? tc::attn_tc_bf16_kernel<kMask, true> : tc::attn_tc_bf16_kernel<kMask, false>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem));
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  kern<<<grid, tc::kThreads, tc::kSmem, s>>>(mq, mk, mv, mo, p);
  return check_launch("attn_tc_bf16_kernel");
}

template <int kMask>
int launch_tc_tf32(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                   cudaStream_t s) {
  auto kern = p.N == kMaxN ? tc32::attn_tc_tf32_kernel<kMask, true> : tc32::attn_tc_tf32_kernel<kMask, false>;
  FA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc32::kSmem));
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  kern<<<grid, tc32::kThreads, tc32::kSmem, s>>>(mq, mk, mv, p);
  return check_launch("attn_tc_tf32_kernel");
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

// FA_ATTN_FP32_KERNEL=mma_sync selects the warp-level 3xTF32 kernel for fp32 I/O (a cross-check of
// the tcgen05 kernel, same accuracy); the default is the tcgen05 kernel.
bool use_sync_fp32() {
  const char* e = getenv("FA_ATTN_FP32_KERNEL");
  return e && std::string(e) == "mma_sync";
}

}  // namespace

int* status_ptr() {
  int* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_status) != cudaSuccess) return nullptr;
  return ptr;
}

int validate(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh, const void* q, const void* k,
             const void* v, const void* out, const int64_t* strides, bool has_mask_u8, bool has_group_ids,
             int64_t nW, unsigned flags) {
  FA_REQUIRE(precision == FA_ATTN_BF16 || precision == FA_ATTN_FP32_3XTF32, FA_ERR_INVALID,
             "precision must be FA_ATTN_BF16 or FA_ATTN_FP32_3XTF32");
  FA_REQUIRE((flags & ~(unsigned)FA_ATTN_FLAG_REGIONS_FIT) == 0, FA_ERR_INVALID, "unknown attention flags");
  FA_REQUIRE(strides, FA_ERR_INVALID, "null stride pointer");
  FA_REQUIRE(Bwin >= 0 && H >= 1 && N >= 1, FA_ERR_INVALID, "invalid attention shape");
  FA_REQUIRE((q && k && v && out) || Bwin == 0, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(Dh == 64, FA_ERR_UNSUPPORTED, "window attention supports head_dim 64");
  FA_REQUIRE(N <= kMaxN, FA_ERR_UNSUPPORTED, "window attention supports N <= 144 tokens");
  FA_REQUIRE(!(has_mask_u8 && has_group_ids), FA_ERR_INVALID, "pass at most one of mask_u8 / group_ids");
  FA_REQUIRE(!(has_mask_u8 || has_group_ids) || nW >= 1, FA_ERR_INVALID, "nW must be >= 1 with a mask");
  FA_REQUIRE(Bwin * H < ((int64_t)1 << 31), FA_ERR_INVALID, "too many (window, head) tiles");
  if (Bwin == 0) return FA_OK;
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
  return FA_OK;
}

int run(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh, const void* q, const void* k,
        const void* v, void* out, const int64_t* strides, const uint8_t* mask_u8,
        const uint8_t* group_ids, int64_t nW, float scale, unsigned flags, void* stream) {
  int rc = validate(precision, Bwin, H, N, Dh, q, k, v, out, strides, mask_u8 != nullptr, group_ids != nullptr,
                    nW, flags);
  if (rc != FA_OK || Bwin == 0) return rc;
  const bool f32 = precision == FA_ATTN_FP32_3XTF32;
  CUtensorMap mq, mk, mv;
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
    // The tcgen05 kernel writes 16-byte output vectors: needs 16-byte aligned rows.
    const bool out16f = aligned16(out) && p.os_w % 4 == 0 && p.os_h % 4 == 0 && p.os_n % 4 == 0;
    if (!use_sync_fp32() && out16f) {
      if (kind == kGroups) return launch_tc_tf32<kGroups>(mq, mk, mv, p, s);
      if (kind == kMaskU8) return launch_tc_tf32<kMaskU8>(mq, mk, mv, p, s);
      return launch_tc_tf32<kNoMask>(mq, mk, mv, p, s);
    }
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
  if (kind == kGroups) {
    if (flags & FA_ATTN_FLAG_REGIONS_FIT) return launch_tc_bf16<kGroupsFit>(mq, mk, mv, p, s);
    return launch_tc_bf16<kGroups>(mq, mk, mv, p, s);
  }
  if (kind == kMaskU8) return launch_tc_bf16<kMaskU8>(mq, mk, mv, p, s);
  return launch_tc_bf16<kNoMask>(mq, mk, mv, p, s);
}

}  // namespace attn
}  // namespace fa

using namespace fa;

extern "C" int fa_window_attention(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh,
                                   const void* q, const void* k, const void* v, void* out,
                                   const int64_t strides[12], const uint8_t* mask_u8,
                                   const uint8_t* group_ids, int64_t nW, float scale, unsigned flags,
                                   void* stream) {
  return attn::run(precision, Bwin, H, N, Dh, q, k, v, out, strides, mask_u8, group_ids, nW, scale, flags,
                   stream);
}

extern "C" int fa_window_attention_qkvpacked(int precision, int64_t Bwin, int64_t N, int64_t H,
                                             int64_t Dh, const void* qkv, void* out, int out_layout,
                                             const uint8_t* mask_u8, const uint8_t* group_ids,
                                             int64_t nW, float scale, unsigned flags, void* stream) {
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
                   group_ids, nW, scale, flags, stream);
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
