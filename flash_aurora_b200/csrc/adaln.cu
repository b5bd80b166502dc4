// Fused AdaLN (LayerNorm without affine + FiLM modulation) + residual add (sm_100a).
//
//   out = [residual +] LN(x) * (scale_bias + scale[b]) + shift[b]
//
// One warp per token row. The row is read from HBM once into registers; mean and variance are
// two-pass (sum, then sum of squared deviations) with warp-shuffle reductions, all in fp32.
// The upstream Triton kernel (ops/triton_adaln.py:148-203) reads x twice and uses
// E[x^2] - mean^2; the two-pass form matches PyTorch's LayerNorm more closely.
//
// The gather variant reads the LN input row of token (c, h, w) directly from the attention
// windows (crop + inverse roll + merge), fusing crop_roll_unmerge into norm1.
#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void load8_any(const T* p, float v[8], bool stream) {
  if (stream) Vec8<T>::load_stream(p, v); else Vec8<T>::load(p, v);
}

__device__ __forceinline__ void load_mod8(const void* p, bool bf16, int64_t off, float v[8]) {
  if (bf16) Vec8<__nv_bfloat16>::load(reinterpret_cast<const __nv_bfloat16*>(p) + off, v);
  else Vec8<float>::load(reinterpret_cast<const float*>(p) + off, v);
}

__device__ __forceinline__ float load_mod1(const void* p, bool bf16, int64_t off) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off])
              : reinterpret_cast<const float*>(p)[off];
}

struct AdaArgs {
  const void* x;
  const void* residual;  // same dtype as out, or null
  const void* scale;
  const void* shift;
  bool mod_bf16;
  float scale_bias, eps;
  void* out;
  __nv_bfloat16* out_bf16;  // optional copy
  int64_t B, L;
  int32_t D;
  bool gather;
  LayoutParams lp;
  const void* halo_in;  // band mode: halo-back rows of the first lp.band band rows (x dtype)
  // Optional scatter of the output rows into the window layout of the next block (its
  // roll + pad + partition); pad slots are left untouched (the caller keeps them zero).
  void* win_out;
  bool win_bf16;
  LayoutParams wlp;
  // Optional row selection: only the token rows (b, c, h, w) with h in [sel_h0, sel_h0 + sel_hn)
  // of the (sel_C, sel_H, sel_W) token grid; sel_hn == 0 selects every row. Lets a caller
  // normalise the rows a halo exchange waits on separately from the others.
  int32_t sel_C, sel_H, sel_W, sel_h0, sel_hn;
  // Divisors (set by run_adaln): L, the selection's run length sel_hn * sel_W, and sel_C. The
  // host keeps B * L below 2^31, so every row index fits 31 bits.
  FastDiv f_L, f_run, f_selC;
};

// Number of rows an AdaArgs launch covers.
__host__ __device__ __forceinline__ int64_t selected_rows(const AdaArgs& a) {
  return a.sel_hn ? a.B * a.sel_C * (int64_t)a.sel_hn * a.sel_W : a.B * a.L;
}

// Token row of one selected row: flat row index, batch element and token index inside it.
struct RowLoc {
  int32_t row, b, t;
};

// The i-th selected row. The selection is B * C runs of sel_hn * sel_W consecutive token rows
// (one per (b, c) slab).
__device__ __forceinline__ RowLoc locate_row(const AdaArgs& a, int32_t i) {
  int32_t r = i;
  if (a.sel_hn) {
    const int32_t seg = fdiv(i, a.f_run);
    const int32_t off = i - seg * (a.sel_hn * a.sel_W);
    const int32_t b = fdiv(seg, a.f_selC);
    const int32_t c = seg - b * a.sel_C;
    r = b * (int32_t)a.L + (c * a.sel_H + a.sel_h0) * a.sel_W + off;
  }
  RowLoc l;
  l.row = r;
  l.b = fdiv(r, a.f_L);
  l.t = r - l.b * (int32_t)a.L;
  return l;
}

// kChunks = number of 8-element (vector path) or 1-element (scalar path) chunks per lane.
// Register bound: vector rows of up to 512 elements are held to 64 registers per thread (four
// 256-thread blocks per SM), everything else to 128 (two blocks).
template <typename TX, typename TO, bool kVec, int kChunks>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, (kVec && kChunks <= 2) ? 4 : 2) adaln_kernel(AdaArgs a) {
  constexpr int kE = kVec ? 8 : 1;  // elements per chunk per lane
  const int lane = threadIdx.x & 31;
  const int D = a.D;
  const int64_t rows = selected_rows(a);
  const TX* const xwin = reinterpret_cast<const TX*>(a.x);
  const TO* __restrict__ rg = reinterpret_cast<const TO*>(a.residual);
  TO* __restrict__ og = reinterpret_cast<TO*>(a.out);
  const float inv_d = 1.0f / (float)D;

  // Address of the LN input row of a token row (window gather in the unmerge form).
  auto x_row = [&](const RowLoc& l) -> const TX* {
    if (!a.gather) return xwin + (int64_t)l.row * D;
    int32_t c, h, w;
    unmerge_token(a.lp, l.t, c, h, w);
    const int32_t slot = unmerge_slot(a.lp, c, h, w);
    if (slot >= 0) return xwin + ((int64_t)l.b * a.lp.nW * a.lp.N + slot) * D;
    // Band mode: row computed by the previous band, received into the halo-back buffer.
    return reinterpret_cast<const TX*>(a.halo_in) + ((int64_t)l.b * a.lp.C * a.lp.band * a.lp.W + (-1 - slot)) * D;
  };
  const int32_t stride = (int32_t)gridDim.x * kWarpsPerBlock;
  int32_t sel = (int32_t)blockIdx.x * kWarpsPerBlock + (int32_t)(threadIdx.x >> 5);
  if (sel >= rows) return;
  // Each iteration locates the next row (index maps, gather address) for its L2 prefetch and
  // carries it over, so every row's map is computed once.
  RowLoc cur = locate_row(a, sel);
  const TX* xr = x_row(cur);
  if (kVec && lane == 0 && rg) prefetch_l2_bulk(rg + (int64_t)cur.row * D, (uint32_t)(D * sizeof(TO)));
  for (; sel < rows; sel += stride) {
    const bool more = (int64_t)sel + stride < rows;
    RowLoc nxt = cur;
    const TX* nxr = xr;
    if (more) {
      nxt = locate_row(a, sel + stride);
      nxr = x_row(nxt);
    }
    if (kVec && lane == 0 && more) {
      // The next row's input and residual stream into L2 while this row is reduced, so that the
      // per-warp chain (load, two reductions, residual load, store) waits less on DRAM.
      prefetch_l2_bulk(nxr, (uint32_t)(D * sizeof(TX)));
      if (rg) prefetch_l2_bulk(rg + (int64_t)nxt.row * D, (uint32_t)(D * sizeof(TO)));
    }
    const int64_t row = cur.row;
    const int64_t b = cur.b;
    int64_t wrow = -1;
    if (a.win_out) {
      int32_t c, h, w;
      unmerge_token(a.wlp, cur.t, c, h, w);
      wrow = b * (int64_t)a.wlp.nW * a.wlp.N + unmerge_slot(a.wlp, c, h, w);
    }
    float v[kChunks][kE];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int col = (i * 32 + lane) * kE;
      if (col < D) {
        if constexpr (kVec) load8_any(xr + col, v[i], true);
        else v[i][0] = to_f32(xr[col]);
      } else {
#pragma unroll
        for (int e = 0; e < kE; ++e) v[i][e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < kE; ++e) s += v[i][e];
    }
    const float mean = warp_sum(s) * inv_d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int col = (i * 32 + lane) * kE;
      if (col < D) {
#pragma unroll
        for (int e = 0; e < kE; ++e) {
          const float d = v[i][e] - mean;
          q += d * d;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(q) * inv_d + a.eps);
    const int64_t mrow = b * D;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int col = (i * 32 + lane) * kE;
      if (col >= D) continue;
      float y[kE];
      if constexpr (kVec) {
        float sc[8], sh[8];
        load_mod8(a.scale, a.mod_bf16, mrow + col, sc);
        load_mod8(a.shift, a.mod_bf16, mrow + col, sh);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = (v[i][e] - mean) * rstd * (a.scale_bias + sc[e]) + sh[e];
        if (rg) {
          float r[8];
          Vec8<TO>::load_stream(rg + row * D + col, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] += r[e];
        }
        Vec8<TO>::store(og + row * D + col, y);
        if (a.out_bf16) Vec8<__nv_bfloat16>::store(a.out_bf16 + row * D + col, y);
        if (wrow >= 0) {
          if (a.win_bf16) Vec8<__nv_bfloat16>::store(reinterpret_cast<__nv_bfloat16*>(a.win_out) + wrow * D + col, y);
          else Vec8<float>::store(reinterpret_cast<float*>(a.win_out) + wrow * D + col, y);
        }
      } else {
        const float sc = load_mod1(a.scale, a.mod_bf16, mrow + col);
        const float sh = load_mod1(a.shift, a.mod_bf16, mrow + col);
        y[0] = (v[i][0] - mean) * rstd * (a.scale_bias + sc) + sh;
        if (rg) y[0] += to_f32(rg[row * D + col]);
        og[row * D + col] = from_f32<TO>(y[0]);
        if (a.out_bf16) a.out_bf16[row * D + col] = __float2bfloat16_rn(y[0]);
        if (wrow >= 0) {
          if (a.win_bf16) reinterpret_cast<__nv_bfloat16*>(a.win_out)[wrow * D + col] = __float2bfloat16_rn(y[0]);
          else reinterpret_cast<float*>(a.win_out)[wrow * D + col] = y[0];
        }
      }
    }
    cur = nxt;
    xr = nxr;
  }
}

template <typename TX, typename TO, bool kVec, int kChunks>
int launch_adaln_chunks(const AdaArgs& a, cudaStream_t s) {
  const int64_t rows = selected_rows(a);
  if (rows == 0 || a.D == 0) return FA_OK;
  int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  adaln_kernel<TX, TO, kVec, kChunks><<<(unsigned)blocks, kWarpsPerBlock * 32, 0, s>>>(a);
  return check_launch("adaln_kernel");
}

template <typename TX, typename TO>
int launch_adaln(const AdaArgs& a, bool vec, cudaStream_t s) {
  if (vec) {
    if (a.D <= 256) return launch_adaln_chunks<TX, TO, true, 1>(a, s);
    if (a.D <= 512) return launch_adaln_chunks<TX, TO, true, 2>(a, s);
    if (a.D <= 1024) return launch_adaln_chunks<TX, TO, true, 4>(a, s);
    return launch_adaln_chunks<TX, TO, true, 8>(a, s);
  }
  if (a.D <= 256) return launch_adaln_chunks<TX, TO, false, 8>(a, s);
  if (a.D <= 1024) return launch_adaln_chunks<TX, TO, false, 32>(a, s);
  return launch_adaln_chunks<TX, TO, false, 64>(a, s);
}

int run_adaln(AdaArgs a, int x_dtype, int residual_dtype, int mod_dtype, int out_dtype,
              cudaStream_t s) {
  FA_REQUIRE((a.x && a.scale && a.shift && a.out) || a.B * a.L == 0 || a.D == 0, FA_ERR_INVALID,
             "null tensor pointer");
  FA_REQUIRE(x_dtype == FA_F32 || x_dtype == FA_BF16, FA_ERR_INVALID, "x dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(out_dtype == FA_F32 || out_dtype == FA_BF16, FA_ERR_INVALID, "out dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(mod_dtype == FA_F32 || mod_dtype == FA_BF16, FA_ERR_INVALID, "scale/shift dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(!a.residual || residual_dtype == out_dtype, FA_ERR_INVALID,
             "residual dtype must equal the output dtype");
  FA_REQUIRE(out_dtype == FA_F32 || x_dtype == FA_BF16, FA_ERR_INVALID,
             "a bf16 output needs a bf16 input (fp32 input writes fp32)");
  FA_REQUIRE(a.B >= 0 && a.L >= 0 && a.D >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE(a.D <= 2048, FA_ERR_UNSUPPORTED, "AdaLN supports D <= 2048");
  FA_REQUIRE(a.B * a.L < (1ll << 31), FA_ERR_UNSUPPORTED, "AdaLN supports fewer than 2^31 rows");
  a.mod_bf16 = mod_dtype == FA_BF16;
  a.f_L = make_fastdiv(a.L);
  a.f_run = make_fastdiv((int64_t)a.sel_hn * a.sel_W);
  a.f_selC = make_fastdiv(a.sel_C);
  const bool vec = (a.D % 8 == 0) && aligned16(a.x) && aligned16(a.scale) && aligned16(a.shift) &&
                   aligned16(a.out) && (!a.residual || aligned16(a.residual)) &&
                   (!a.out_bf16 || aligned16(a.out_bf16)) && (!a.halo_in || aligned16(a.halo_in)) &&
                   (!a.win_out || aligned16(a.win_out));
  if (x_dtype == FA_F32) return launch_adaln<float, float>(a, vec, s);
  if (out_dtype == FA_F32) return launch_adaln<__nv_bfloat16, float>(a, vec, s);
  return launch_adaln<__nv_bfloat16, __nv_bfloat16>(a, vec, s);
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_adaln_film(const void* x, int x_dtype, const void* residual, int residual_dtype,
                             const void* scale, const void* shift, int mod_dtype, float scale_bias,
                             float eps, void* out, int out_dtype, void* out_bf16, int64_t B,
                             int64_t L, int64_t D, void* stream) {
  AdaArgs a{};
  a.x = x; a.residual = residual; a.scale = scale; a.shift = shift;
  a.scale_bias = scale_bias; a.eps = eps; a.out = out;
  a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  a.B = B; a.L = L; a.D = (int32_t)D; a.gather = false;
  FA_REQUIRE(D < (1 << 30), FA_ERR_INVALID, "D too large");
  return run_adaln(a, x_dtype, residual_dtype, mod_dtype, out_dtype, (cudaStream_t)stream);
}

extern "C" int fa_unmerge_adaln_film(const void* windows, int windows_dtype, const void* residual,
                                     int residual_dtype, const void* scale, const void* shift,
                                     int mod_dtype, float scale_bias, float eps, void* out,
                                     int out_dtype, void* out_bf16, int64_t B, int64_t C, int64_t H,
                                     int64_t W, int64_t D, const int32_t window_size[3],
                                     const int32_t shift_size[3], void* stream) {
  Geometry g;
  int rc = make_geometry(C, H, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE(D < (1 << 30), FA_ERR_INVALID, "D too large");
  AdaArgs a{};
  a.x = windows; a.residual = residual; a.scale = scale; a.shift = shift;
  a.scale_bias = scale_bias; a.eps = eps; a.out = out;
  a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  a.B = B; a.L = C * H * W; a.D = (int32_t)D; a.gather = true; a.lp = layout_params(g);
  return run_adaln(a, windows_dtype, residual_dtype, mod_dtype, out_dtype, (cudaStream_t)stream);
}

extern "C" int fa_unmerge_adaln_film_band(const void* windows, const void* halo_in,
                                          int windows_dtype, const void* residual,
                                          int residual_dtype, const void* scale, const void* shift,
                                          int mod_dtype, float scale_bias, float eps, void* out,
                                          int out_dtype, void* out_bf16, int64_t B, int64_t C,
                                          int64_t H_band, int64_t H_field, int64_t W, int64_t D,
                                          const int32_t window_size[3],
                                          const int32_t shift_size[3], int64_t h_begin,
                                          int64_t h_count, void* stream) {
  Geometry g;
  int rc = make_band_geometry(C, H_band, H_field, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE(D < (1 << 30), FA_ERR_INVALID, "D too large");
  FA_REQUIRE(h_begin >= 0 && h_count >= 0 && h_begin + h_count <= H_band, FA_ERR_INVALID,
             "row range outside the band");
  AdaArgs a{};
  a.x = windows; a.residual = residual; a.scale = scale; a.shift = shift;
  a.scale_bias = scale_bias; a.eps = eps; a.out = out;
  a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  a.B = B; a.L = C * H_band * W; a.D = (int32_t)D; a.gather = true;
  a.lp = band_layout_params(g, false);
  a.halo_in = halo_in;
  if (h_count == 0) return FA_OK;
  if (h_begin != 0 || h_count != H_band) {
    a.sel_C = (int32_t)C; a.sel_H = (int32_t)H_band; a.sel_W = (int32_t)W;
    a.sel_h0 = (int32_t)h_begin; a.sel_hn = (int32_t)h_count;
  }
  // Only rows below the band's halo depth read the halo-back buffer.
  FA_REQUIRE(halo_in || a.lp.band == 0 || h_begin >= a.lp.band || B == 0 || D == 0, FA_ERR_INVALID,
             "shifted band needs the halo-back rows");
  return run_adaln(a, windows_dtype, residual_dtype, mod_dtype, out_dtype, (cudaStream_t)stream);
}

extern "C" int fa_adaln_film_rows(const void* x, int x_dtype, const void* residual, int residual_dtype,
                                  const void* scale, const void* shift, int mod_dtype, float scale_bias,
                                  float eps, void* out, int out_dtype, void* out_bf16, int64_t B,
                                  int64_t C, int64_t H, int64_t W, int64_t D, int64_t h_begin,
                                  int64_t h_count, void* stream) {
  FA_REQUIRE(B >= 0 && C >= 0 && H >= 0 && W >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE(C < (1 << 30) && H < (1 << 30) && W < (1 << 30) && C * H * W < (1ll << 31), FA_ERR_INVALID,
             "token grid too large");
  FA_REQUIRE(D < (1 << 30), FA_ERR_INVALID, "D too large");
  FA_REQUIRE(h_begin >= 0 && h_count >= 0 && h_begin + h_count <= H, FA_ERR_INVALID,
             "row range outside the grid");
  AdaArgs a{};
  a.x = x; a.residual = residual; a.scale = scale; a.shift = shift;
  a.scale_bias = scale_bias; a.eps = eps; a.out = out;
  a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  a.B = B; a.L = C * H * W; a.D = (int32_t)D; a.gather = false;
  if (h_count == 0) return FA_OK;
  if (h_begin != 0 || h_count != H) {
    a.sel_C = (int32_t)C; a.sel_H = (int32_t)H; a.sel_W = (int32_t)W;
    a.sel_h0 = (int32_t)h_begin; a.sel_hn = (int32_t)h_count;
  }
  return run_adaln(a, x_dtype, residual_dtype, mod_dtype, out_dtype, (cudaStream_t)stream);
}

extern "C" int fa_adaln_film_partition(const void* x, int x_dtype, const void* residual, int residual_dtype,
                                       const void* scale, const void* shift, int mod_dtype, float scale_bias,
                                       float eps, void* out, int out_dtype, void* windows, int windows_dtype,
                                       int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                                       const int32_t window_size[3], const int32_t shift_size[3],
                                       void* stream) {
  Geometry g;
  int rc = make_geometry(C, H, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE(D < (1 << 30), FA_ERR_INVALID, "D too large");
  FA_REQUIRE(windows_dtype == FA_F32 || windows_dtype == FA_BF16, FA_ERR_INVALID,
             "windows dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(windows || B * C * H * W == 0 || D == 0, FA_ERR_INVALID, "null windows pointer");
  AdaArgs a{};
  a.x = x; a.residual = residual; a.scale = scale; a.shift = shift;
  a.scale_bias = scale_bias; a.eps = eps; a.out = out;
  a.B = B; a.L = C * H * W; a.D = (int32_t)D; a.gather = false;
  a.win_out = windows;
  a.win_bf16 = windows_dtype == FA_BF16;
  a.wlp = layout_params(g);
  return run_adaln(a, x_dtype, residual_dtype, mod_dtype, out_dtype, (cudaStream_t)stream);
}
