// LayerNorm with affine weight / bias over the last dimension, optionally plus a residual: the
// Perceiver decoder's `layer_norm(x) + residual` (upstream ops/triton_perceiver_ln.py:25-145, used by
// aurora/model/perceiver.py:255-276 for the level decoder of decoder.py:100-123).
//
//   out = (x - mean) / sqrt(var + eps) * weight + bias (+ residual),   var over D, biased
//
// computed in fp32 and rounded once to x's dtype, like upstream. Upstream reads every row twice
// and forms the variance as E[x^2] - mean^2 (triton_perceiver_ln.py:122-131); here one warp holds
// its row in registers, so x is read once and the variance is taken about the mean (the form
// nn.LayerNorm uses). Rows whose length is not a multiple of 8, or whose tensors are not 16-byte
// aligned, take a scalar path that reads the row three times (from L1 after the first).
#include <cuda_fp16.h>

#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 8 consecutive elements of a row as fp32, and back (fp16 support beside fa_common's f32 / bf16).
template <typename T> struct Row8;
template <> struct Row8<float> {
  static __device__ __forceinline__ void load(const float* p, float v[8]) { Vec8<float>::load_stream(p, v); }
  static __device__ __forceinline__ void store(float* p, const float v[8]) { Vec8<float>::store(p, v); }
};
template <> struct Row8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float v[8]) {
    Vec8<__nv_bfloat16>::load_stream(p, v);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float v[8]) {
    Vec8<__nv_bfloat16>::store(p, v);
  }
};
template <> struct Row8<__half> {
  static __device__ __forceinline__ void load(const __half* p, float v[8]) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__half* p, const float v[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};

__device__ __forceinline__ float elem_f32(const void* p, int dt, int64_t i) {
  if (dt == FA_F32) return __ldg(reinterpret_cast<const float*>(p) + i);
  if (dt == FA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
template <typename T> __device__ __forceinline__ T store_as(float v);
template <> __device__ __forceinline__ float store_as<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 store_as<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half store_as<__half>(float v) { return __float2half_rn(v); }
template <typename T> __device__ __forceinline__ float load_as(const T* p) { return to_f32(*p); }
template <> __device__ __forceinline__ float load_as<__half>(const __half* p) { return __half2float(*p); }

// weight / bias (any of the three dtypes) at columns col..col+7 (16-byte aligned when vector).
__device__ __forceinline__ void param8(const void* p, int dt, int col, float v[8]) {
  if (dt == FA_F32) {
    Vec8<float>::load(reinterpret_cast<const float*>(p) + col, v);
  } else if (dt == FA_BF16) {
    Vec8<__nv_bfloat16>::load(reinterpret_cast<const __nv_bfloat16*>(p) + col, v);
  } else {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p) + col));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// Memory-bound: the small-row variants are held to at most 64 registers (4 blocks, 32 warps per
// SM) so that enough rows are in flight.
template <typename T, int kChunks, bool kRes>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, kChunks <= 2 ? 3 : (kChunks <= 4 ? 2 : 1))
ln_affine_kernel(const T* x, const T* res, const void* __restrict__ w, const void* __restrict__ b, int wdt, T* out,
                 int64_t rows, int D, float eps) {
  // out may alias x or res: a warp reads its whole row before writing it. Up to D = 2048 the
  // residual row is requested together with x; weight and bias are re-read per row (L1 hits).
  constexpr bool kEarlyRes = kRes && kChunks <= 8;
  const int lane = threadIdx.x & 31;
  const float inv_d = 1.f / (float)D;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* xr = x + row * D;
    float v[kChunks][8], r[kEarlyRes ? kChunks : 1][8];
    float s = 0.f;
    // x and the residual are both requested before the reductions, so their latencies overlap.
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int col = (i * 32 + lane) * 8;
      if (col < D) {
        Row8<T>::load(xr + col, v[i]);
        if constexpr (kEarlyRes) Row8<T>::load(res + row * D + col, r[i]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[i][e];
    }
    const float mean = warp_sum(s) * inv_d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      if ((i * 32 + lane) * 8 < D) {
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
      if (col >= D) continue;
      float y[8], wv[8], bv[8];
      param8(w, wdt, col, wv);
      param8(b, wdt, col, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = (v[i][e] - mean) * rstd * wv[e] + bv[e];
      if constexpr (kEarlyRes) {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] += r[i][e];
      } else if constexpr (kRes) {
        float rl[8];
        Row8<T>::load(res + row * D + col, rl);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] += rl[e];
      }
      Row8<T>::store(out + row * D + col, y);
    }
  }
}

// Any D (<= 4096) and alignment: lane-strided columns, three passes over the row.
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
ln_affine_scalar_kernel(const T* x, const T* res, const void* __restrict__ w, const void* __restrict__ b, int wdt,
                        T* out, int64_t rows, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const float inv_d = 1.f / (float)D;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* xr = x + row * D;
    float s = 0.f;
    for (int c = lane; c < D; c += 32) s += load_as(xr + c);
    const float mean = warp_sum(s) * inv_d;
    float q = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float d = load_as(xr + c) - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
    for (int c = lane; c < D; c += 32) {
      float y = (load_as(xr + c) - mean) * rstd * elem_f32(w, wdt, c) + elem_f32(b, wdt, c);
      if (res) y += load_as(res + row * D + c);
      out[row * D + c] = store_as<T>(y);
    }
  }
}

int64_t grid_for(int64_t rows) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = (int64_t)num_sms() * 16;
  return blocks < cap ? (blocks > 0 ? blocks : 1) : cap;
}

template <typename T, bool kRes>
void dispatch_chunks(dim3 grid, dim3 block, cudaStream_t s, const T* xp, const T* rp, const void* w, const void* b,
                     int wdt, T* op, int64_t rows, int D, float eps) {
  if (D <= 256) ln_affine_kernel<T, 1, kRes><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
  else if (D <= 512) ln_affine_kernel<T, 2, kRes><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
  else if (D <= 1024) ln_affine_kernel<T, 4, kRes><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
  else if (D <= 2048) ln_affine_kernel<T, 8, kRes><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
  else ln_affine_kernel<T, 16, kRes><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
}

template <typename T>
int launch(const void* x, const void* res, const void* w, const void* b, int wdt, void* out, int64_t rows, int D,
           float eps, bool vec, cudaStream_t s) {
  const T* xp = reinterpret_cast<const T*>(x);
  const T* rp = reinterpret_cast<const T*>(res);
  T* op = reinterpret_cast<T*>(out);
  const dim3 grid((unsigned)grid_for(rows)), block(kWarpsPerBlock * 32);
  if (!vec) {
    ln_affine_scalar_kernel<T><<<grid, block, 0, s>>>(xp, rp, w, b, wdt, op, rows, D, eps);
    return check_launch("ln_affine_scalar_kernel");
  }
  if (rp) dispatch_chunks<T, true>(grid, block, s, xp, rp, w, b, wdt, op, rows, D, eps);
  else dispatch_chunks<T, false>(grid, block, s, xp, rp, w, b, wdt, op, rows, D, eps);
  return check_launch("ln_affine_kernel");
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_layernorm_affine(const void* x, int x_dtype, const void* residual, const void* weight,
                                   const void* bias, int wb_dtype, float eps, void* out, int64_t rows, int64_t D,
                                   void* stream) {
  FA_REQUIRE(x_dtype == FA_F32 || x_dtype == FA_BF16 || x_dtype == FA_F16, FA_ERR_INVALID,
             "x dtype must be FA_F32, FA_BF16 or FA_F16");
  FA_REQUIRE(wb_dtype == FA_F32 || wb_dtype == FA_BF16 || wb_dtype == FA_F16, FA_ERR_INVALID,
             "weight / bias dtype must be FA_F32, FA_BF16 or FA_F16");
  FA_REQUIRE(rows >= 0 && D >= 1, FA_ERR_INVALID, "invalid LayerNorm shape");
  FA_REQUIRE(D <= 4096, FA_ERR_UNSUPPORTED, "LayerNorm supports D <= 4096");
  FA_REQUIRE(eps >= 0.f, FA_ERR_INVALID, "eps must be >= 0");
  if (rows == 0) return FA_OK;
  FA_REQUIRE(x && weight && bias && out, FA_ERR_INVALID, "null tensor pointer");
  const bool vec = D % 8 == 0 && aligned16(x) && aligned16(out) && aligned16(weight) && aligned16(bias) &&
                   (!residual || aligned16(residual));
  cudaStream_t s = (cudaStream_t)stream;
  if (x_dtype == FA_F32) return launch<float>(x, residual, weight, bias, wb_dtype, out, rows, (int)D, eps, vec, s);
  if (x_dtype == FA_BF16)
    return launch<__nv_bfloat16>(x, residual, weight, bias, wb_dtype, out, rows, (int)D, eps, vec, s);
  return launch<__half>(x, residual, weight, bias, wb_dtype, out, rows, (int)D, eps, vec, s);
}
