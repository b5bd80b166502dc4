// Window attention with a float bias for callers that cannot allocate device memory.
//
// The float-bias path normally packs the (nW, N, N) bias into a uint8 mask in a temporary buffer
// before the attention kernel reads it. Here that mask lives in a fixed static device array of
// this library instead, so a call allocates nothing. Callers in this position include code that
// runs inside a memory pool it does not own, plugins whose host forbids allocation on its streams,
// and real-time loops that must not call cudaMalloc after start-up.
#include <mutex>

#include "attention.cuh"
#include "fa_common.cuh"

namespace fa {
namespace {

// Largest packed mask the static scratch holds: nW * N * N bytes (e.g. 202 windows of 144 tokens).
constexpr int64_t kNoAllocMaskBytes = 4 << 20;

// One copy per GPU that loads the library, kept until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_mask[kNoAllocMaskBytes];

__global__ void pack_bias_kernel(const float* __restrict__ bias, uint8_t* __restrict__ mask, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    mask[i] = bias[i] < -50.0f ? 1 : 0;  // the upstream threshold: bias < -50 means masked
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device. The array's name is only a host
// stand-in, so the address is looked up once per device (with that device current) and cached
// for the life of the process. The cache does not survive cudaDeviceReset or a re-created primary
// context: a process that resets a device must not call this entry point on it afterwards.
int scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  FA_CUDA(cudaGetDevice(&dev));
  FA_REQUIRE(dev >= 0 && dev < kMaxDevices, FA_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    uint8_t* ptr = nullptr;
    FA_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_mask));
    FA_REQUIRE(ptr != nullptr, FA_ERR_CUDA, "cudaGetSymbolAddress returned a null scratch address");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return FA_OK;
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" int fa_window_attention_bias_noalloc(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh,
                                                const void* q, const void* k, const void* v, void* out,
                                                const int64_t strides[12], const float* bias, int64_t nW,
                                                float scale, void* stream) {
  // Every argument is checked before the shared scratch is touched, so a rejected call leaves the
  // previous call's packed mask as it was.
  FA_REQUIRE(nW >= 1 && N >= 1, FA_ERR_INVALID, "nW and N must be positive");
  FA_REQUIRE(nW <= kNoAllocMaskBytes, FA_ERR_INVALID, "nW exceeds the static scratch of fa_window_attention_bias_noalloc");
  int rc = attn::validate(precision, Bwin, H, N, Dh, q, k, v, out, strides, true, false, nW, 0u);
  if (rc != FA_OK) return rc;
  // N <= 144 and nW <= 4 MiB here, so the product cannot overflow.
  const int64_t mask_bytes = nW * N * N;
  FA_REQUIRE(mask_bytes <= kNoAllocMaskBytes, FA_ERR_INVALID,
             "the packed mask needs " + std::to_string(mask_bytes) + " bytes; the static scratch of "
             "fa_window_attention_bias_noalloc holds " + std::to_string(kNoAllocMaskBytes) +
             " (nW * N * N must not exceed it)");
  if (Bwin == 0) return FA_OK;
  FA_REQUIRE(bias, FA_ERR_INVALID, "null bias pointer");
  uint8_t* mask = nullptr;
  rc = scratch_for_current_device(&mask);
  if (rc != FA_OK) return rc;
  // Every byte the attention kernel reads (the first nW*N*N) is rewritten here, so no clearing of
  // the previous call's contents is needed.
  const int64_t blocks = (mask_bytes + 255) / 256 < (int64_t)num_sms() * 8 ? (mask_bytes + 255) / 256
                                                                           : (int64_t)num_sms() * 8;
  pack_bias_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(bias, mask, mask_bytes);
  rc = check_launch("pack_bias_kernel");
  if (rc != FA_OK) return rc;
  return attn::run(precision, Bwin, H, N, Dh, q, k, v, out, strides, mask, nullptr, nW, scale, 0u, stream);
}
