// Exact (erf) GELU over a contiguous bf16 or fp32 tensor, in place or out of place (sm_100a).
//
// The MLP of the Swin3D block applies nn.GELU() (exact erf form, upstream swin3d.py:73-109)
// between fc1 and fc2. This is a pure streaming kernel: every element is read once and written
// once, with 16-byte accesses and four independent vectors per thread in flight. The value is
// x * 0.5 * (1 + erf(x / sqrt(2))) evaluated in fp32 in that order with CUDA's erff, then
// rounded to the tensor's dtype (round to nearest even), the same arithmetic as PyTorch's CUDA
// GELU for bf16/fp32 tensors.
#include "fa_common.cuh"

namespace fa {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kAlpha = 0.70710678118654752440f;  // 1/sqrt(2)
  return x * 0.5f * (1.0f + erff(x * kAlpha));
}

// Coherent streaming load (the tensor may be written in place by this kernel).
template <typename T>
__device__ __forceinline__ uint4 ld_cs16(const T* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint4 gelu16(uint4 a, __nv_bfloat16*) {
  uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    w[i] = pack_bf16x2(gelu_erf(f.x), gelu_erf(f.y));
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 gelu16(uint4 a, float*) {
  return make_uint4(__float_as_uint(gelu_erf(__uint_as_float(a.x))),
                    __float_as_uint(gelu_erf(__uint_as_float(a.y))),
                    __float_as_uint(gelu_erf(__uint_as_float(a.z))),
                    __float_as_uint(gelu_erf(__uint_as_float(a.w))));
}

// n16: number of whole 16-byte vectors; the tail (< 16 bytes) is handled by tail_kernel.
template <typename T>
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
      *reinterpret_cast<uint4*>(out + (i + u * stride) * kPer) = gelu16(v[u], (T*)nullptr);
  }
  for (; i < n16; i += stride) {
    const uint4 v = ld_cs16(x + i * kPer);
    *reinterpret_cast<uint4*>(out + i * kPer) = gelu16(v, (T*)nullptr);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) gelu_scalar_kernel(const T* x, T* out, int64_t begin,
                                                               int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    out[i] = from_f32<T>(gelu_erf(to_f32(x[i])));
}

template <typename T>
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
      gelu_vec_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(x, out, n16);
      int rc = check_launch("gelu_vec_kernel");
      if (rc != FA_OK) return rc;
    }
    done = n16 * kPer;
  }
  if (done < n) {
    int64_t blocks = (n - done + kThreads - 1) / kThreads;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    gelu_scalar_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(x, out, done, n);
    return check_launch("gelu_scalar_kernel");
  }
  return FA_OK;
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_gelu_erf(const void* x, void* out, int dtype, int64_t n, void* stream) {
  FA_REQUIRE(dtype == FA_F32 || dtype == FA_BF16, FA_ERR_INVALID, "dtype must be FA_F32 or FA_BF16");
  FA_REQUIRE(n >= 0, FA_ERR_INVALID, "negative size");
  FA_REQUIRE((x && out) || n == 0, FA_ERR_INVALID, "null tensor pointer");
  const size_t es = dtype == FA_F32 ? 4 : 2;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x), oa = reinterpret_cast<uintptr_t>(out);
  // In place is allowed; any other overlap would make the result depend on scheduling.
  FA_REQUIRE(xa == oa || xa + (uintptr_t)n * es <= oa || oa + (uintptr_t)n * es <= xa,
             FA_ERR_INVALID, "x and out overlap without being the same tensor");
  if (dtype == FA_F32) return launch_gelu<float>(x, out, n, (cudaStream_t)stream);
  return launch_gelu<__nv_bfloat16>(x, out, n, (cudaStream_t)stream);
}
