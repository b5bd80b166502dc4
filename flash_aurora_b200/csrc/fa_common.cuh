// Shared helpers of the flash_aurora_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "flash_aurora_b200.h"

namespace fa {

// ---------------------------------------------------------------------------------------------
// Error reporting: every C-ABI entry point returns a status and records a thread-local message.
// ---------------------------------------------------------------------------------------------
int set_error(int code, const std::string& msg);
int check_launch(const char* what);  // cudaGetLastError -> FA_ERR_CUDA with the kernel name

#define FA_REQUIRE(cond, code, msg)                      \
  do {                                                   \
    if (!(cond)) return ::fa::set_error((code), (msg));  \
  } while (0)

#define FA_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t e__ = (call);                                                                 \
    if (e__ != cudaSuccess)                                                                   \
      return ::fa::set_error(FA_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e__)); \
  } while (0)

// ---------------------------------------------------------------------------------------------
// Window geometry (upstream util.py:54-72 clamp, swin3d.py:415-432 padding split).
// ---------------------------------------------------------------------------------------------
struct Geometry {
  int64_t C, H, W;
  int32_t ws[3], ss[3], pf[3];  // window, shift (after clamp), front pads (C, H, W)
  int64_t padded[3];
  int64_t grid[3];  // windows per axis
  int64_t nW;
  int32_t N;
};

int make_geometry(int64_t C, int64_t H, int64_t W, const int32_t* window_size,
                  const int32_t* shift_size, Geometry* g);

// Geometry of one latitude band of H_band rows out of a field of H_field rows: window clamping
// and shifts are decided on the whole field (C, H_field, W); the band must hold whole window
// rows, and the field must need no H padding.
int make_band_geometry(int64_t C, int64_t H_band, int64_t H_field, int64_t W,
                       const int32_t* window_size, const int32_t* shift_size, Geometry* g);

// ---------------------------------------------------------------------------------------------
// Division of a non-negative 31-bit integer n by a run-time divisor d (1 <= d < 2^31) with one
// 32 x 32 -> 64-bit multiply and a shift, after Granlund & Montgomery, "Division by invariant
// integers using multiplication" (PLDI 1994): with l = ceil(log2 d), p = 31 + l and
// m = ceil(2^p / d) (< 2^32), m * d = 2^p + e with 0 <= e < d <= 2^l, so
// n * m / 2^p = n / d + n * e / (d * 2^p) and the second term is below 2^-l <= 1 / d: the floor
// is floor(n / d). The index maps of the gathers divide by window and grid extents per row, which
// the hardware's integer division would otherwise spend tens of instructions on each.
// ---------------------------------------------------------------------------------------------
struct FastDiv {
  uint32_t d, m, p;
};

inline FastDiv make_fastdiv(int64_t d) {
  FastDiv f;
  f.d = (uint32_t)(d < 1 ? 1 : d);
  uint32_t l = 0;
  while ((1ull << l) < f.d) ++l;
  f.p = 31 + l;
  f.m = (uint32_t)(((1ull << f.p) + f.d - 1) / f.d);
  return f;
}

// floor(n / f.d) for 0 <= n < 2^31.
__host__ __device__ __forceinline__ int32_t fdiv(int32_t n, const FastDiv& f) {
  return (int32_t)(((uint64_t)(uint32_t)n * f.m) >> f.p);
}

// Device-side copy of the index parameters of a layout gather.
struct LayoutParams {
  int32_t C, H, W;
  int32_t wc, wh, ww;
  int32_t sc, sh, sw;
  int32_t pc, ph, pw;  // front pads
  int32_t W1, HW1;     // windows along W, windows per C slab
  int32_t nW, N;
  // Latitude-band mode (band > 0): the grid is one band of H rows of a larger field and the
  // cyclic H shift is realised by the band offset instead of a wrap. Shifted row s of the band
  // is original band row s + band; rows at or past H come from a halo of `band` rows (the next
  // band's first rows, layout (B, C, band, W, D)). sh is 0 in band mode.
  int32_t band;
  int32_t Hout;  // rows of an unmerge output grid: H, or `band` for the halo extract
  int32_t hs0;   // band mode: shifted row of unmerge output row 0 (-band, or H - band)
  // Divisors of the index maps (see FastDiv).
  FastDiv f_W, f_Hout, f_wc, f_wh, f_ww, f_W1, f_HW1, f_whw;
};

inline void set_divisors(LayoutParams& p) {
  p.f_W = make_fastdiv(p.W);
  p.f_Hout = make_fastdiv(p.Hout);
  p.f_wc = make_fastdiv(p.wc);
  p.f_wh = make_fastdiv(p.wh);
  p.f_ww = make_fastdiv(p.ww);
  p.f_W1 = make_fastdiv(p.W1);
  p.f_HW1 = make_fastdiv(p.HW1);
  p.f_whw = make_fastdiv((int64_t)p.wh * p.ww);
}

inline LayoutParams layout_params(const Geometry& g) {
  LayoutParams p;
  p.C = (int32_t)g.C; p.H = (int32_t)g.H; p.W = (int32_t)g.W;
  p.wc = g.ws[0]; p.wh = g.ws[1]; p.ww = g.ws[2];
  p.sc = g.ss[0]; p.sh = g.ss[1]; p.sw = g.ss[2];
  p.pc = g.pf[0]; p.ph = g.pf[1]; p.pw = g.pf[2];
  p.W1 = (int32_t)g.grid[2];
  p.HW1 = (int32_t)(g.grid[1] * g.grid[2]);
  p.nW = (int32_t)g.nW;
  p.N = g.N;
  p.band = 0;
  p.Hout = p.H;
  p.hs0 = 0;
  set_divisors(p);
  return p;
}

// Band-mode parameters: `g` is the geometry of the band (H = band rows, shifts as for the whole
// field); the H shift becomes the halo depth. `extract` selects the halo-extract unmerge grid
// (the band's last `band` shifted rows, which are the next band's first original rows).
inline LayoutParams band_layout_params(const Geometry& g, bool extract) {
  LayoutParams p = layout_params(g);
  p.band = p.sh;
  p.sh = 0;
  p.Hout = extract ? p.band : p.H;
  p.hs0 = extract ? p.H - p.band : -p.band;
  set_divisors(p);
  return p;
}

// Token (c, h, w) of token index t < C * Hout * W of the unmerge output grid.
__device__ __forceinline__ void unmerge_token(const LayoutParams& p, int32_t t, int32_t& c, int32_t& h,
                                              int32_t& w) {
  const int32_t q = fdiv(t, p.f_W);
  w = t - q * p.W;
  c = fdiv(q, p.f_Hout);
  h = q - c * p.Hout;
}

// Source token (c*H + h)*W + w of window slot (win, n) of one batch element, or -1 for pad.
// Same mapping as ops/triton_swin3d_layout.py:218-246. In band mode a result >= C*H*W is
// halo token (result - C*H*W) of layout (C, band, W).
__device__ __forceinline__ int32_t partition_source(const LayoutParams& p, int32_t win, int32_t n) {
  const int32_t c1 = fdiv(win, p.f_HW1);
  const int32_t r1 = win - c1 * p.HW1;
  const int32_t h1 = fdiv(r1, p.f_W1);
  const int32_t w1 = r1 - h1 * p.W1;
  const int32_t whw = p.wh * p.ww;
  const int32_t wc = fdiv(n, p.f_whw);
  const int32_t r2 = n - wc * whw;
  const int32_t wh = fdiv(r2, p.f_ww);
  const int32_t ww = r2 - wh * p.ww;
  const int32_t cs = c1 * p.wc + wc - p.pc;
  const int32_t hs = h1 * p.wh + wh - p.ph;
  const int32_t wsv = w1 * p.ww + ww - p.pw;
  if (cs < 0 || cs >= p.C || hs < 0 || hs >= p.H || wsv < 0 || wsv >= p.W) return -1;
  int32_t xc = cs + p.sc; if (xc >= p.C) xc -= p.C;
  int32_t xw = wsv + p.sw; if (xw >= p.W) xw -= p.W;
  int32_t xh = hs + p.sh + p.band;
  if (xh >= p.H) {
    if (p.band == 0) {
      xh -= p.H;
    } else {
      // Band mode: rows past the band are halo rows, encoded after the band's C*H*W tokens.
      return p.C * p.H * p.W + (xc * p.band + (xh - p.H)) * p.W + xw;
    }
  }
  return (xc * p.H + xh) * p.W + xw;
}

// Window slot win*N + n holding token (c, h, w) of one batch element (triton_swin3d_layout.py:283-305).
// (c, h, w) indexes the unmerge output grid (C, Hout, W). In band mode a negative result
// -1 - i means halo-back token i.
__device__ __forceinline__ int32_t unmerge_slot(const LayoutParams& p, int32_t c, int32_t h, int32_t w) {
  int32_t cs = c - p.sc; if (cs < 0) cs += p.C;
  int32_t hs = h - p.sh + p.hs0;
  if (p.band == 0) {
    if (hs < 0) hs += p.H;
  } else if (hs < 0) {
    // Band mode: the first `band` original rows were computed by the previous band; they are
    // read from its halo-back buffer (layout (C, band, W)), encoded as -1 - index.
    return -1 - ((c * p.band + h) * p.W + w);
  }
  int32_t wsv = w - p.sw; if (wsv < 0) wsv += p.W;
  const int32_t pc = cs + p.pc, ph = hs + p.ph, pw = wsv + p.pw;
  const int32_t c1 = fdiv(pc, p.f_wc), wc = pc - c1 * p.wc;
  const int32_t h1 = fdiv(ph, p.f_wh), wh = ph - h1 * p.wh;
  const int32_t w1 = fdiv(pw, p.f_ww), ww = pw - w1 * p.ww;
  const int32_t win = c1 * p.HW1 + h1 * p.W1 + w1;
  const int32_t n = (wc * p.wh + wh) * p.ww + ww;
  return win * p.N + n;
}

// ---------------------------------------------------------------------------------------------
// 8-element vector I/O (16 B of bf16, 32 B of fp32) with conversion to/from fp32 registers.
// ---------------------------------------------------------------------------------------------
template <typename T> struct Vec8;

template <> struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float v[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void load_stream(const float* p, float v[8]) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float v[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  static __device__ __forceinline__ void zero(float* p) {
    reinterpret_cast<float4*>(p)[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4*>(p)[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);  // round to nearest even
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Bulk prefetch of `bytes` (a multiple of 16) from a 16-byte-aligned global address into L2. A
// hint: nothing waits for it and it writes no register or shared memory.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Three-input fp32 maximum (one instruction on sm_100; PTX ISA 8.8). NaN handling is that of
// fmaxf: a NaN operand is ignored unless all are NaN.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  // bf16 -> fp32 is exact: the bf16 bits are the top half of the fp32 pattern.
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

template <> struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float v[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    float2 f;
    f = unpack_bf16x2(a.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(a.y); v[2] = f.x; v[3] = f.y;
    f = unpack_bf16x2(a.z); v[4] = f.x; v[5] = f.y;
    f = unpack_bf16x2(a.w); v[6] = f.x; v[7] = f.y;
  }
  static __device__ __forceinline__ void load_stream(const __nv_bfloat16* p, float v[8]) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    float2 f;
    f = unpack_bf16x2(a.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(a.y); v[2] = f.x; v[3] = f.y;
    f = unpack_bf16x2(a.z); v[4] = f.x; v[5] = f.y;
    f = unpack_bf16x2(a.w); v[6] = f.x; v[7] = f.y;
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float v[8]) {
    uint4 a;
    a.x = pack_bf16x2(v[0], v[1]);
    a.y = pack_bf16x2(v[2], v[3]);
    a.z = pack_bf16x2(v[4], v[5]);
    a.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = a;
  }
  static __device__ __forceinline__ void zero(__nv_bfloat16* p) {
    *reinterpret_cast<uint4*>(p) = make_uint4(0u, 0u, 0u, 0u);
  }
};

// Scalar element access for the unaligned fallback paths.
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms();  // SM count of the current device (cached per device)
// CTA pairs (clusters of 2) of `kernel` that fit on the current device at once, for a persistent
// grid of one pair per slot (cached per kernel and device; the GPC layout can leave an SM without a
// partner, so this can be below num_sms() / 2). The kernel's dynamic shared memory attribute must
// already be set.
int max_resident_pairs(const void* kernel, int threads, int smem_bytes);

}  // namespace fa
