// Fused cyclic shift + zero pad + 3D window partition, and its inverse (sm_100a).
//
// Both directions are pure row gathers: each token row of D contiguous elements is copied
// whole (or zero-filled for a pad token), so the kernels work one warp per token row with
// 16-byte vector accesses. The index arithmetic is done once per row, not per element as in
// the upstream Triton kernels (ops/triton_swin3d_layout.py:192-307). Reads of the source use
// the non-allocating streaming path: each source row is read exactly once.
#include <type_traits>

#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kWarpsPerBlock = 8;

// Blocks per SM the register budget must allow. fp32 -> fp32 rows move two 8-float vectors per
// lane and step; at the 40 registers ptxas picks for them unbounded they spill, so they get 64
// (four blocks). The other type pairs fit in 40 registers (six blocks).
template <typename TIn, typename TOut>
constexpr int min_blocks() {
  return (std::is_same<TIn, float>::value && std::is_same<TOut, float>::value) ? 4 : 6;
}

// THalo: element type of the band-mode halo rows (the input's type, or the output's when the
// neighbour sent its rows already rounded to it: the rounding commutes with the gather).
template <typename TIn, typename TOut, typename THalo, bool kVec>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, min_blocks<TIn, TOut>())
partition_kernel(const TIn* __restrict__ x, const THalo* __restrict__ halo, TOut* __restrict__ out,
                 LayoutParams p, int64_t B, int32_t D) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = B * (int64_t)p.nW * p.N;
  const int64_t tokens = (int64_t)p.C * p.H * p.W;
  const int64_t halo_tokens = (int64_t)p.C * p.band * p.W;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int64_t b = row / ((int64_t)p.nW * p.N);
    const int32_t r = (int32_t)(row - b * (int64_t)p.nW * p.N);
    const int32_t win = r / p.N;
    const int32_t n = r - win * p.N;
    const int32_t src = partition_source(p, win, n);
    TOut* dst = out + row * D;
    // Band mode: sources past the band's own tokens are rows of the halo (a warp-uniform branch).
    const TIn* s = x + (b * tokens + src) * D;
    const THalo* sh = halo + (b * halo_tokens + (src - tokens)) * D;
    if constexpr (kVec) {
      if (src < 0) {
        for (int c = lane * 8; c < D; c += 256) Vec8<TOut>::zero(dst + c);
      } else if (src < tokens) {
        for (int c = lane * 8; c < D; c += 256) {
          float v[8];
          Vec8<TIn>::load_stream(s + c, v);
          Vec8<TOut>::store(dst + c, v);
        }
      } else {
        for (int c = lane * 8; c < D; c += 256) {
          float v[8];
          Vec8<THalo>::load_stream(sh + c, v);
          Vec8<TOut>::store(dst + c, v);
        }
      }
    } else {
      if (src < 0) {
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<TOut>(0.f);
      } else if (src < tokens) {
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<TOut>(to_f32(s[c]));
      } else {
        for (int c = lane; c < D; c += 32) dst[c] = from_f32<TOut>(to_f32(sh[c]));
      }
    }
  }
}

template <typename TIn, typename TOut, bool kVec>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, min_blocks<TIn, TOut>())
unmerge_kernel(const TIn* __restrict__ win, const TIn* __restrict__ halo_in, TOut* __restrict__ out,
               LayoutParams p, int64_t B, int32_t D) {
  const int lane = threadIdx.x & 31;
  const int64_t tokens = (int64_t)p.C * p.Hout * p.W;
  const int64_t rows = B * tokens;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int64_t b = row / tokens;
    const int32_t t = (int32_t)(row - b * tokens);
    int32_t c, h, w;
    unmerge_token(p, t, c, h, w);
    const int32_t slot = unmerge_slot(p, c, h, w);
    // Band mode: the first `band` rows come from the previous band's halo-back rows.
    const TIn* s = slot >= 0 ? win + (b * (int64_t)p.nW * p.N + slot) * D
                             : halo_in + (b * (int64_t)p.C * p.band * p.W + (-1 - slot)) * D;
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

template <typename TIn, typename TOut, typename THalo = TIn>
int launch_partition(const void* x, const void* halo, void* out, const LayoutParams& p, int64_t B,
                     int64_t D, cudaStream_t s, bool vec) {
  const int64_t rows = B * (int64_t)p.nW * p.N;
  if (rows == 0 || D == 0) return FA_OK;
  const dim3 grid((unsigned)grid_for_rows(rows)), block(kWarpsPerBlock * 32);
  if (vec)
    partition_kernel<TIn, TOut, THalo, true><<<grid, block, 0, s>>>((const TIn*)x, (const THalo*)halo,
                                                                    (TOut*)out, p, B, (int32_t)D);
  else
    partition_kernel<TIn, TOut, THalo, false><<<grid, block, 0, s>>>((const TIn*)x, (const THalo*)halo,
                                                                     (TOut*)out, p, B, (int32_t)D);
  return check_launch("partition_kernel");
}

template <typename TIn, typename TOut>
int launch_unmerge(const void* w, const void* halo_in, void* out, const LayoutParams& p, int64_t B,
                   int64_t D, cudaStream_t s, bool vec) {
  const int64_t rows = B * (int64_t)p.C * p.Hout * p.W;
  if (rows == 0 || D == 0) return FA_OK;
  const dim3 grid((unsigned)grid_for_rows(rows)), block(kWarpsPerBlock * 32);
  if (vec)
    unmerge_kernel<TIn, TOut, true><<<grid, block, 0, s>>>((const TIn*)w, (const TIn*)halo_in, (TOut*)out,
                                                           p, B, (int32_t)D);
  else
    unmerge_kernel<TIn, TOut, false><<<grid, block, 0, s>>>((const TIn*)w, (const TIn*)halo_in, (TOut*)out,
                                                            p, B, (int32_t)D);
  return check_launch("unmerge_kernel");
}

template <typename... Args>
int dispatch_partition(int in_dt, int out_dt, Args... a) {
  if (in_dt == FA_F32 && out_dt == FA_F32) return launch_partition<float, float>(a...);
  if (in_dt == FA_F32) return launch_partition<float, __nv_bfloat16>(a...);
  if (out_dt == FA_F32) return launch_partition<__nv_bfloat16, float>(a...);
  return launch_partition<__nv_bfloat16, __nv_bfloat16>(a...);
}

template <typename... Args>
int dispatch_unmerge(int in_dt, int out_dt, Args... a) {
  if (in_dt == FA_F32 && out_dt == FA_F32) return launch_unmerge<float, float>(a...);
  if (in_dt == FA_F32) return launch_unmerge<float, __nv_bfloat16>(a...);
  if (out_dt == FA_F32) return launch_unmerge<__nv_bfloat16, float>(a...);
  return launch_unmerge<__nv_bfloat16, __nv_bfloat16>(a...);
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
  return dispatch_partition(x_dtype, windows_dtype, x, (const void*)nullptr, windows, p, B, D,
                            (cudaStream_t)stream, vec);
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
  return dispatch_unmerge(windows_dtype, out_dtype, windows, (const void*)nullptr, out, p, B, D,
                          (cudaStream_t)stream, vec);
}

// ---------------------------------------------------------------------------------------------
// Latitude-band entry points (one band of a field sharded by window rows across ranks).
// ---------------------------------------------------------------------------------------------

namespace {

int check_band_args(const void* a, int adt, const void* b, int bdt, int64_t B, int64_t C,
                    int64_t H_band, int64_t H_field, int64_t W, int64_t D, const int32_t* ws,
                    const int32_t* ss, Geometry* g) {
  FA_REQUIRE(adt == FA_F32 || adt == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(bdt == FA_F32 || bdt == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(B >= 0 && D >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE(D <= (1 << 20), FA_ERR_INVALID, "D too large");
  int rc = make_band_geometry(C, H_band, H_field, W, ws, ss, g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE((a && b) || B == 0 || D == 0, FA_ERR_INVALID, "null tensor pointer");
  FA_REQUIRE(B * g->nW * g->N < (int64_t)1 << 40, FA_ERR_INVALID, "tensor too large");
  return FA_OK;
}

}  // namespace

extern "C" int fa_roll_pad_partition_band(const void* x, const void* halo, int x_dtype, int halo_dtype,
                                          void* windows, int windows_dtype, int64_t B, int64_t C,
                                          int64_t H_band, int64_t H_field, int64_t W, int64_t D,
                                          const int32_t window_size[3],
                                          const int32_t shift_size[3], void* stream) {
  Geometry g;
  int rc = check_band_args(x, x_dtype, windows, windows_dtype, B, C, H_band, H_field, W, D,
                           window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE(halo_dtype == x_dtype || halo_dtype == windows_dtype, FA_ERR_INVALID,
             "halo_dtype must be x_dtype or windows_dtype");
  const LayoutParams p = band_layout_params(g, false);
  FA_REQUIRE(halo || p.band == 0 || B == 0 || D == 0, FA_ERR_INVALID, "shifted band needs a halo");
  const bool vec = (D % 8 == 0) && aligned16(x) && aligned16(windows) && (!halo || aligned16(halo));
  const cudaStream_t st = (cudaStream_t)stream;
  if (halo_dtype == x_dtype) return dispatch_partition(x_dtype, windows_dtype, x, halo, windows, p, B, D, st, vec);
  // The halo arrives already rounded to the windows' type: only fp32 x -> bf16 windows gains from
  // that (a bf16 x has nothing to round, its fp32 windows are exact).
  FA_REQUIRE(x_dtype == FA_F32 && windows_dtype == FA_BF16, FA_ERR_UNSUPPORTED,
             "a halo in the windows' dtype is supported for fp32 x with bf16 windows");
  return launch_partition<float, __nv_bfloat16, __nv_bfloat16>(x, halo, windows, p, B, D, st, vec);
}

extern "C" int fa_band_halo_extract(const void* windows, int windows_dtype, void* halo_out,
                                    int halo_dtype, int64_t B, int64_t C, int64_t H_band,
                                    int64_t H_field, int64_t W, int64_t D,
                                    const int32_t window_size[3], const int32_t shift_size[3],
                                    void* stream) {
  Geometry g;
  int rc = check_band_args(windows, windows_dtype, halo_out, halo_dtype, B, C, H_band, H_field, W,
                           D, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  const LayoutParams p = band_layout_params(g, true);
  if (p.band == 0) return FA_OK;  // no H shift: nothing crosses the band edge
  const bool vec = (D % 8 == 0) && aligned16(windows) && aligned16(halo_out);
  return dispatch_unmerge(windows_dtype, halo_dtype, windows, (const void*)nullptr, halo_out, p, B,
                          D, (cudaStream_t)stream, vec);
}

extern "C" int fa_crop_roll_unmerge_band(const void* windows, const void* halo_in,
                                         int windows_dtype, void* out, int out_dtype, int64_t B,
                                         int64_t C, int64_t H_band, int64_t H_field, int64_t W,
                                         int64_t D, const int32_t window_size[3],
                                         const int32_t shift_size[3], void* stream) {
  Geometry g;
  int rc = check_band_args(windows, windows_dtype, out, out_dtype, B, C, H_band, H_field, W, D,
                           window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  const LayoutParams p = band_layout_params(g, false);
  FA_REQUIRE(halo_in || p.band == 0 || B == 0 || D == 0, FA_ERR_INVALID,
             "shifted band needs the halo-back rows");
  const bool vec = (D % 8 == 0) && aligned16(windows) && aligned16(out) && (!halo_in || aligned16(halo_in));
  return dispatch_unmerge(windows_dtype, out_dtype, windows, halo_in, out, p, B, D, (cudaStream_t)stream, vec);
}
