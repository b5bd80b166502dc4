// Fused cyclic shift + zero pad + 3D window partition, and its inverse (sm_100a).
//
// Both directions are pure row gathers: each token row of D contiguous elements is copied
// whole (or zero-filled for a pad token), so the kernels work one warp per token row with
// 16-byte vector accesses. The index arithmetic is done once per row, not per element as in
// the upstream Triton kernels (ops/triton_swin3d_layout.py:192-307). Reads of the source use
// the non-allocating streaming path: each source row is read exactly once.
#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kWarpsPerBlock = 8;

template <typename TIn, typename TOut, bool kVec>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
partition_kernel(const TIn* __restrict__ x, TOut* __restrict__ out, LayoutParams p, int64_t B,
                 int32_t D) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = B * (int64_t)p.nW * p.N;
  const int64_t tokens = (int64_t)p.C * p.H * p.W;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int64_t b = row / ((int64_t)p.nW * p.N);
    const int32_t r = (int32_t)(row - b * (int64_t)p.nW * p.N);
    const int32_t win = r / p.N;
    const int32_t n = r - win * p.N;
    const int32_t src = partition_source(p, win, n);
    TOut* dst = out + row * D;
    if constexpr (kVec) {
      if (src < 0) {
        for (int c = lane * 8; c < D; c += 256) Vec8<TOut>::zero(dst + c);
      } else {
        const TIn* s = x + (b * tokens + src) * D;
        for (int c = lane * 8; c < D; c += 256) {
          float v[8];
          Vec8<TIn>::load_stream(s + c, v);
          Vec8<TOut>::store(dst + c, v);
        }
      }
    } else {
      if (src < 0) {
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<TOut>(0.f);
      } else {
        const TIn* s = x + (b * tokens + src) * D;
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<TOut>(to_f32(s[c]));
      }
    }
  }
}

template <typename TIn, typename TOut, bool kVec>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
unmerge_kernel(const TIn* __restrict__ win, TOut* __restrict__ out, LayoutParams p, int64_t B,
               int32_t D) {
  const int lane = threadIdx.x & 31;
  const int64_t tokens = (int64_t)p.C * p.H * p.W;
  const int64_t rows = B * tokens;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int64_t b = row / tokens;
    const int32_t t = (int32_t)(row - b * tokens);
    const int32_t w = t % p.W;
    const int32_t h = (t / p.W) % p.H;
    const int32_t c = t / (p.W * p.H);
    const int64_t slot = b * (int64_t)p.nW * p.N + unmerge_slot(p, c, h, w);
    const TIn* s = win + slot * D;
    TOut* dst = out + row * D;
    if constexpr (kVec) {
      for (int k = lane * 8; k < D; k += 256) {
        float v[8];
        Vec8<TIn>::load_stream(s + k, v);
        Vec8<TOut>::store(dst + k, v);
      }
    } else {
      for (int k = lane; k < D; k += 32) dst[k] = from_f32<TOut>(to_f32(s[k]));
    }
  }
}

int64_t grid_for_rows(int64_t rows) {
  // Enough resident warps to keep ~64 KB of loads in flight per SM; grid-stride beyond that.
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = (int64_t)num_sms() * 32;
  return blocks < cap ? (blocks > 0 ? blocks : 1) : cap;
}

template <typename TIn, typename TOut>
int launch_partition(const void* x, void* out, const LayoutParams& p, int64_t B, int64_t D,
                     cudaStream_t s, bool vec) {
  const int64_t rows = B * (int64_t)p.nW * p.N;
  if (rows == 0 || D == 0) return FA_OK;
  const dim3 grid((unsigned)grid_for_rows(rows)), block(kWarpsPerBlock * 32);
  if (vec)
    partition_kernel<TIn, TOut, true><<<grid, block, 0, s>>>((const TIn*)x, (TOut*)out, p, B, (int32_t)D);
  else
    partition_kernel<TIn, TOut, false><<<grid, block, 0, s>>>((const TIn*)x, (TOut*)out, p, B, (int32_t)D);
  return check_launch("partition_kernel");
}

template <typename TIn, typename TOut>
int launch_unmerge(const void* w, void* out, const LayoutParams& p, int64_t B, int64_t D,
                   cudaStream_t s, bool vec) {
  const int64_t rows = B * (int64_t)p.C * p.H * p.W;
  if (rows == 0 || D == 0) return FA_OK;
  const dim3 grid((unsigned)grid_for_rows(rows)), block(kWarpsPerBlock * 32);
  if (vec)
    unmerge_kernel<TIn, TOut, true><<<grid, block, 0, s>>>((const TIn*)w, (TOut*)out, p, B, (int32_t)D);
  else
    unmerge_kernel<TIn, TOut, false><<<grid, block, 0, s>>>((const TIn*)w, (TOut*)out, p, B, (int32_t)D);
  return check_launch("unmerge_kernel");
}

int check_layout_args(const void* a, int adt, const void* b, int bdt, int64_t B, int64_t C,
                      int64_t H, int64_t W, int64_t D, const int32_t* ws, const int32_t* ss,
                      Geometry* g) {
  FA_REQUIRE(adt == FA_F32 || adt == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(bdt == FA_F32 || bdt == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(B >= 0 && D >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE(D <= (1 << 20), FA_ERR_INVALID, "D too large");
  int rc = make_geometry(C, H, W, ws, ss, g);
  if (rc != FA_OK) return rc;
  // Empty tensors may carry null pointers; only non-empty ones must be valid.
  FA_REQUIRE((a && b) || B == 0 || D == 0, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(B * g->nW * g->N < (int64_t)1 << 40, FA_ERR_INVALID, "tensor too large");
  return FA_OK;
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_roll_pad_partition(const void* x, int x_dtype, void* windows, int windows_dtype,
                                     int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                                     const int32_t window_size[3], const int32_t shift_size[3],
                                     void* stream) {
  Geometry g;
  int rc = check_layout_args(x, x_dtype, windows, windows_dtype, B, C, H, W, D, window_size,
                             shift_size, &g);
  if (rc != FA_OK) return rc;
  const LayoutParams p = layout_params(g);
  const bool vec = (D % 8 == 0) && aligned16(x) && aligned16(windows);
  cudaStream_t s = (cudaStream_t)stream;
  if (x_dtype == FA_F32 && windows_dtype == FA_F32) return launch_partition<float, float>(x, windows, p, B, D, s, vec);
  if (x_dtype == FA_F32) return launch_partition<float, __nv_bfloat16>(x, windows, p, B, D, s, vec);
  if (windows_dtype == FA_F32) return launch_partition<__nv_bfloat16, float>(x, windows, p, B, D, s, vec);
  return launch_partition<__nv_bfloat16, __nv_bfloat16>(x, windows, p, B, D, s, vec);
}

extern "C" int fa_crop_roll_unmerge(const void* windows, int windows_dtype, void* out, int out_dtype,
                                    int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                                    const int32_t window_size[3], const int32_t shift_size[3],
                                    void* stream) {
  Geometry g;
  int rc = check_layout_args(windows, windows_dtype, out, out_dtype, B, C, H, W, D, window_size,
                             shift_size, &g);
  if (rc != FA_OK) return rc;
  const LayoutParams p = layout_params(g);
  const bool vec = (D % 8 == 0) && aligned16(windows) && aligned16(out);
  cudaStream_t s = (cudaStream_t)stream;
  if (windows_dtype == FA_F32 && out_dtype == FA_F32) return launch_unmerge<float, float>(windows, out, p, B, D, s, vec);
  if (windows_dtype == FA_F32) return launch_unmerge<float, __nv_bfloat16>(windows, out, p, B, D, s, vec);
  if (out_dtype == FA_F32) return launch_unmerge<__nv_bfloat16, float>(windows, out, p, B, D, s, vec);
  return launch_unmerge<__nv_bfloat16, __nv_bfloat16>(windows, out, p, B, D, s, vec);
}
