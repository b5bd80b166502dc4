// Exact (erf) GELU over a contiguous bf16 or fp32 tensor, in place or out of place (sm_100a).
//
// The MLP of the Swin3D block applies nn.GELU() (exact erf form, upstream swin3d.py:73-109)
// between fc1 and fc2. This is a streaming kernel (every element read once and written once,
// 16-byte accesses, four vectors per thread in flight) whose cost is the arithmetic: a GELU
// through erff is issue-bound on B200, not bandwidth-bound. Two evaluations:
//
//  FA_GELU_ERFF  x * 0.5 * (1 + erff(x / sqrt(2))) in fp32 in that order, the arithmetic of
//                PyTorch's CUDA GELU (bit-identical to it).
//  FA_GELU_POLY  Phi(x) without the cancellation of 1 + erf: with t = |x| / sqrt(2),
//                h = erfc(t) / 2 = 2^-q(t), where q is a degree-9 polynomial fitted here (numpy,
//                Lawson-reweighted least squares of -log2(erfc(t) / 2) on [0, 4], weight
//                sqrt(erfc)); GELU = x * (1 - h) for x >= 0 and x * h for x < 0, h = 0 past t = 4.
//                The polynomial runs on paired fp32 FMAs (two elements per instruction) and the
//                power of two on the special-function unit. Checked over every finite bf16 input:
//                the bf16 result equals the correctly rounded exact GELU for all |x| < 4; beyond,
//                |GELU| < 1.3e-4 and the result is within 1e-6 of it (PyTorch's 1 + erf form returns
//                0 there).
#include "fa_common.cuh"
#include "gelu.cuh"

namespace fa {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kAlpha = 0.70710678118654752440f;  // 1/sqrt(2)
  return x * 0.5f * (1.0f + erff(x * kAlpha));
}

template <int kMethod>
__device__ __forceinline__ float2 gelu2(float2 x) {
  if constexpr (kMethod == FA_GELU_POLY) return gelu2_poly(x);
  else return make_float2(gelu_erf(x.x), gelu_erf(x.y));
}

// Coherent streaming load (the tensor may be written in place by this kernel).
template <typename T>
__device__ __forceinline__ uint4 ld_cs16(const T* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

template <int kMethod>
__device__ __forceinline__ uint4 gelu16(uint4 a, __nv_bfloat16*) {
  uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 g = gelu2<kMethod>(unpack_bf16x2(w[i]));
    w[i] = pack_bf16x2(g.x, g.y);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int kMethod>
__device__ __forceinline__ uint4 gelu16(uint4 a, float*) {
  const float2 g0 = gelu2<kMethod>(make_float2(__uint_as_float(a.x), __uint_as_float(a.y)));
  const float2 g1 = gelu2<kMethod>(make_float2(__uint_as_float(a.z), __uint_as_float(a.w)));
  return make_uint4(__float_as_uint(g0.x), __float_as_uint(g0.y), __float_as_uint(g1.x), __float_as_uint(g1.y));
}

template <int kMethod>
__device__ __forceinline__ float gelu1(float x) {
  return gelu2<kMethod>(make_float2(x, 0.f)).x;
}

// n16: number of whole 16-byte vectors; the tail (< 16 bytes) is handled by gelu_scalar_kernel.
template <typename T, int kMethod>
__global__ void __launch_bounds__(kThreads) gelu_vec_kernel(const T* x, T* out, int64_t n16) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  constexpr int kPer = 16 / sizeof(T);
  for (; i + (kUnroll - 1) * stride < n16; i += kUnroll * stride) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_cs16(x + (i + u * stride) * kPer);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      *reinterpret_cast<uint4*>(out + (i + u * stride) * kPer) = gelu16<kMethod>(v[u], (T*)nullptr);
  }
  for (; i < n16; i += stride) {
    const uint4 v = ld_cs16(x + i * kPer);
    *reinterpret_cast<uint4*>(out + i * kPer) = gelu16<kMethod>(v, (T*)nullptr);
  }
}

template <typename T, int kMethod>
__global__ void __launch_bounds__(kThreads) gelu_scalar_kernel(const T* x, T* out, int64_t begin,
                                                               int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    out[i] = from_f32<T>(gelu1<kMethod>(to_f32(x[i])));
}

template <typename T, int kMethod>
int launch_gelu(const void* xv, void* ov, int64_t n, cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  T* out = static_cast<T*>(ov);
  if (n == 0) return FA_OK;
  constexpr int kPer = 16 / sizeof(T);
  int64_t done = 0;
  if (aligned16(x) && aligned16(out)) {
    const int64_t n16 = n / kPer;
    if (n16 > 0) {
      int64_t blocks = (n16 + (int64_t)kThreads * kUnroll - 1) / ((int64_t)kThreads * kUnroll);
      const int64_t cap = (int64_t)num_sms() * 8;
      if (blocks > cap) blocks = cap;
      gelu_vec_kernel<T, kMethod><<<(unsigned)blocks, kThreads, 0, s>>>(x, out, n16);
      int rc = check_launch("gelu_vec_kernel");
      if (rc != FA_OK) return rc;
    }
    done = n16 * kPer;
  }
  if (done < n) {
    int64_t blocks = (n - done + kThreads - 1) / kThreads;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    gelu_scalar_kernel<T, kMethod><<<(unsigned)blocks, kThreads, 0, s>>>(x, out, done, n);
    return check_launch("gelu_scalar_kernel");
  }
  return FA_OK;
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_gelu_erf(const void* x, void* out, int dtype, int64_t n, int method, void* stream) {
  FA_REQUIRE(dtype == FA_F32 || dtype == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(method == FA_GELU_ERFF || method == FA_GELU_POLY, FA_ERR_INVALID,
             "method must be FA_GELU_ERFF or FA_GELU_POLY");
  FA_REQUIRE(n >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE((x && out) || n == 0, FA_ERR_INVALID, "null tensor pointer");
  const size_t es = dtype == FA_F32 ? 4 : 2;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x), oa = reinterpret_cast<uintptr_t>(out);
  // In place is allowed; any other overlap would make the result depend on scheduling.
  FA_REQUIRE(xa == oa || xa + (uintptr_t)n * es <= oa || oa + (uintptr_t)n * es <= xa,
             FA_ERR_INVALID, "x and out overlap without being the same tensor");
  cudaStream_t st = (cudaStream_t)stream;
  if (method == FA_GELU_POLY)
    return dtype == FA_F32 ? launch_gelu<float, FA_GELU_POLY>(x, out, n, st)
                           : launch_gelu<__nv_bfloat16, FA_GELU_POLY>(x, out, n, st);
  return dtype == FA_F32 ? launch_gelu<float, FA_GELU_ERFF>(x, out, n, st)
                         : launch_gelu<__nv_bfloat16, FA_GELU_ERFF>(x, out, n, st);
}
