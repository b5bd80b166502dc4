// Stage-boundary gathers of the Swin3D U-net fused with their LayerNorm (sm_100a).
//
// PatchMerging3D (upstream swin3d.py:818-861): pad H and W to even at the back, gather each 2 x 2
//   patch into one 4D-channel token (channel (dh * 2 + dw) * D + d), LayerNorm(4D) with affine.
// PatchSplitting3D (upstream swin3d.py:864-919), after its first linear: split every 4D'-channel
//   token into a 2 x 2 patch of D'-channel tokens (sub-token (dh, dw) = channels
//   [(dh * 2 + dw) * D', +D')), crop (C, H, W) at the back, LayerNorm(D') with affine.
// Upstream runs pad + permute + reshape copies and a separate LayerNorm; here every output row is
// gathered straight from the source and normalised in registers: one read, one write. One warp per
// output row, 8-float vectors, two-pass mean and variance in fp32.
#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One output row of `Dout` floats: `src_of(col)` gives the source pointer of the 8 floats at
// output column col (nullptr = zeros). Normalise with weight/bias and store.
template <int kChunks, typename SrcOf>
__device__ __forceinline__ void ln_row(SrcOf src_of, float* out, const float* w, const float* b, int Dout,
                                       float eps, int lane) {
  float v[kChunks][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int col = (i * 32 + lane) * 8;
    const float* p = col < Dout ? src_of(col) : nullptr;
    if (p) {
      Vec8<float>::load_stream(p, v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[i][e];
  }
  const float inv_d = 1.f / (float)Dout;
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int col = (i * 32 + lane) * 8;
    if (col < Dout) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int col = (i * 32 + lane) * 8;
    if (col >= Dout) continue;
    float wv[8], bv[8], y[8];
    Vec8<float>::load(w + col, wv);
    Vec8<float>::load(b + col, bv);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (v[i][e] - mean) * rstd * wv[e] + bv[e];
    Vec8<float>::store(out + col, y);
  }
}

template <int kChunks>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
merge_ln_kernel(const float* __restrict__ x, float* __restrict__ out, const float* __restrict__ w,
                const float* __restrict__ b, int64_t B, int C, int H, int W, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int Ho = (H + 1) / 2, Wo = (W + 1) / 2;
  const int64_t rows = B * (int64_t)C * Ho * Wo;
  const int Dout = 4 * D;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int wo = (int)(row % Wo);
    const int64_t r1 = row / Wo;
    const int ho = (int)(r1 % Ho);
    const int64_t bc = r1 / Ho;  // b * C + c
    auto src_of = [&](int col) -> const float* {
      const int part = col / D, d = col - part * D;
      const int h = 2 * ho + (part >> 1), ww = 2 * wo + (part & 1);
      if (h >= H || ww >= W) return nullptr;  // the zero pad at the back of H / W
      return x + ((bc * H + h) * W + ww) * (int64_t)D + d;
    };
    ln_row<kChunks>(src_of, out + row * Dout, w, b, Dout, eps, lane);
  }
}

template <int kChunks>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
split_ln_kernel(const float* __restrict__ z, float* __restrict__ out, const float* __restrict__ w,
                const float* __restrict__ b, int64_t B, int C, int H, int W, int Dq, int Co, int Ho, int Wo,
                float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = B * (int64_t)Co * Ho * Wo;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int wo = (int)(row % Wo);
    const int64_t r1 = row / Wo;
    const int ho = (int)(r1 % Ho);
    const int64_t r2 = r1 / Ho;
    const int c = (int)(r2 % Co);
    const int64_t bb = r2 / Co;
    const int h = ho >> 1, ww = wo >> 1, part = ((ho & 1) << 1) | (wo & 1);
    const float* base = z + (((bb * C + c) * H + h) * W + ww) * (int64_t)(4 * Dq) + (int64_t)part * Dq;
    auto src_of = [&](int col) -> const float* { return base + col; };
    ln_row<kChunks>(src_of, out + row * Dq, w, b, Dq, eps, lane);
  }
}

int64_t grid_for(int64_t rows) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = (int64_t)num_sms() * 16;
  return blocks < cap ? (blocks > 0 ? blocks : 1) : cap;
}

}  // namespace
}  // namespace fa

using namespace fa;

#define FA_DISPATCH_CHUNKS(KERNEL, DOUT, ROWS, STREAM, ...)                                             \
  do {                                                                                                  \
    const dim3 grid((unsigned)grid_for(ROWS)), block(kWarpsPerBlock * 32);                              \
    if ((DOUT) <= 256) KERNEL<1><<<grid, block, 0, STREAM>>>(__VA_ARGS__);                              \
    else if ((DOUT) <= 512) KERNEL<2><<<grid, block, 0, STREAM>>>(__VA_ARGS__);                         \
    else if ((DOUT) <= 1024) KERNEL<4><<<grid, block, 0, STREAM>>>(__VA_ARGS__);                        \
    else if ((DOUT) <= 2048) KERNEL<8><<<grid, block, 0, STREAM>>>(__VA_ARGS__);                        \
    else KERNEL<16><<<grid, block, 0, STREAM>>>(__VA_ARGS__);                                           \
  } while (0)

extern "C" int fa_patch_merge_ln(const float* x, float* out, const float* weight, const float* bias, int64_t B,
                                 int64_t C, int64_t H, int64_t W, int64_t D, float eps, void* stream) {
  FA_REQUIRE(B >= 0 && C > 0 && H > 1 && W > 1 && D > 0, FA_ERR_INVALID, "invalid merge shape (H, W > 1)");
  FA_REQUIRE(D % 8 == 0 && 4 * D <= 4096, FA_ERR_UNSUPPORTED, "patch merge supports D % 8 == 0 and 4D <= 4096");
  FA_REQUIRE(C < (1 << 20) && H < (1 << 20) && W < (1 << 20), FA_ERR_INVALID, "resolution too large");
  const int64_t rows = B * C * ((H + 1) / 2) * ((W + 1) / 2);
  if (rows == 0) return FA_OK;
  FA_REQUIRE(x && out && weight && bias, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(aligned16(x) && aligned16(out) && aligned16(weight) && aligned16(bias), FA_ERR_INVALID,
             "tensors must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  FA_DISPATCH_CHUNKS(merge_ln_kernel, 4 * D, rows, s, x, out, weight, bias, B, (int)C, (int)H, (int)W, (int)D, eps);
  return check_launch("merge_ln_kernel");
}

extern "C" int fa_patch_split_ln(const float* z, float* out, const float* weight, const float* bias, int64_t B,
                                 int64_t C, int64_t H, int64_t W, int64_t Dq, const int32_t crop[3], float eps,
                                 void* stream) {
  FA_REQUIRE(crop, FA_ERR_INVALID, "null crop pointer");
  FA_REQUIRE(B >= 0 && C > 0 && H > 0 && W > 0 && Dq > 0, FA_ERR_INVALID, "invalid split shape");
  FA_REQUIRE(Dq % 8 == 0 && Dq <= 4096, FA_ERR_UNSUPPORTED, "patch split supports D' % 8 == 0 and D' <= 4096");
  FA_REQUIRE(crop[0] >= 0 && crop[1] >= 0 && crop[2] >= 0 && crop[0] < C && crop[1] < 2 * H && crop[2] < 2 * W,
             FA_ERR_INVALID, "crop out of range");
  FA_REQUIRE(C < (1 << 20) && H < (1 << 20) && W < (1 << 20), FA_ERR_INVALID, "resolution too large");
  const int Co = (int)C - crop[0], Ho = 2 * (int)H - crop[1], Wo = 2 * (int)W - crop[2];
  const int64_t rows = B * (int64_t)Co * Ho * Wo;
  if (rows == 0) return FA_OK;
  FA_REQUIRE(z && out && weight && bias, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(aligned16(z) && aligned16(out) && aligned16(weight) && aligned16(bias), FA_ERR_INVALID,
             "tensors must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  FA_DISPATCH_CHUNKS(split_ln_kernel, Dq, rows, s, z, out, weight, bias, B, (int)C, (int)H, (int)W, (int)Dq, Co, Ho, Wo,
                     eps);
  return check_launch("split_ln_kernel");
}
