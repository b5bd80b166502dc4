// Shared definitions of the window-attention kernels.
#pragma once

#include <stdint.h>

namespace fa {
namespace attn {

constexpr int kMaxN = 144;                   // tokens per window: 2 x 6 x 12
constexpr int kTileBytes = kMaxN * 128;      // one 144-row tile of 128-byte rows
constexpr uint64_t kTimeoutNs = 2000000000;  // bound of every device-side wait (2 s)
constexpr float kMaskedLog2 = -144.26950408889634f;  // -100 * log2(e): masked logit bias

// kGroups: (nW, N) region ids of any form; kGroupsFit: region ids the caller guarantees to have at
// most 16 distinct values below 32 per window (the shifted-window masks do), which lets the bf16
// tensor-core kernel drop its per-logit fallback; kMaskU8: an (nW, N, N) byte mask.
enum MaskKind { kNoMask = 0, kGroups = 1, kMaskU8 = 2, kGroupsFit = 3 };

struct Params {
  int Bwin, H, N, nW;
  int num_tiles;
  float scale_log2;      // softmax scale * log2(e)
  const uint8_t* mask;   // (nW, N, N) u8 or (nW, N) region ids, by MaskKind
  void* out;
  int64_t os_w, os_h, os_n;  // output element strides (window, head, token)
  int* status;               // device status word, first failing wait code
};

int* status_ptr();

// Argument checks of run() (shapes, precision, flags, pointers, strides, alignment), without
// launching anything: FA_OK or the status run() would return for these arguments.
int validate(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh, const void* q, const void* k,
             const void* v, const void* out, const int64_t* strides, bool has_mask_u8, bool has_group_ids,
             int64_t nW, unsigned flags);

// Window attention on (Bwin, H, N, Dh) tensors with element strides {q, k, v, out} x
// {window, head, token}; at most one of mask_u8 (nW, N, N) / group_ids (nW, N). Host entry of the
// kernels in attention.cu; allocates nothing.
int run(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh, const void* q, const void* k,
        const void* v, void* out, const int64_t* strides, const uint8_t* mask_u8, const uint8_t* group_ids,
        int64_t nW, float scale, unsigned flags, void* stream);

}  // namespace attn
}  // namespace fa
