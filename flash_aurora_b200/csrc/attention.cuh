// Shared definitions of the window-attention kernels.
#pragma once

#include <stdint.h>

namespace fa {
namespace attn {

constexpr int kMaxN = 144;                   // tokens per window: 2 x 6 x 12
constexpr int kTileBytes = kMaxN * 128;      // one 144-row tile of 128-byte rows
constexpr uint64_t kTimeoutNs = 2000000000;  // bound of every device-side wait (2 s)
constexpr float kMaskedLog2 = -144.26950408889634f;  // -100 * log2(e): masked logit bias

enum MaskKind { kNoMask = 0, kGroups = 1, kMaskU8 = 2 };

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

}  // namespace attn
}  // namespace fa
