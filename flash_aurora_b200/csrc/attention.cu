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

#include <mutex>

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
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * q + e;
      float xa = s[j][e] * scale_log2, xb = s[j][2 + e] * scale_log2;
      if (key >= N) {
        xa = -INFINITY;
        xb = -INFINITY;
      } else if constexpr (kMask != kNoMask) {
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
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * q + e;
      float xa = s[j][e] * scale_log2, xb = s[j][2 + e] * scale_log2;
      if (key >= N) {
        xa = -INFINITY;
        xb = -INFINITY;
      } else if constexpr (kMask != kNoMask) {
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
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  FA_REQUIRE(r == CUDA_SUCCESS, FA_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FA_OK;
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
  if (kind == kGroups) return launch_sync<false, kGroups>(mq, mk, mv, p, s);
  if (kind == kMaskU8) return launch_sync<false, kMaskU8>(mq, mk, mv, p, s);
  return launch_sync<false, kNoMask>(mq, mk, mv, p, s);
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
