// Host-side helpers of the C ABI: error strings, window geometry, shifted-window region ids.
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "fa_common.cuh"

namespace fa {

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return FA_OK;
}

int max_resident_pairs(const void* kernel, int threads, int smem_bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return num_sms() / 2;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, dev);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(num_sms() & ~1));
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();  // clear the error of the query; fall back to every SM pair
    clusters = num_sms() / 2;
  }
  cache[key] = clusters;
  return clusters;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// util.py:54-72 (clamp) and swin3d.py:415-432 (front = p // 2 of the pad p = (-dim) mod ws).
int make_geometry(int64_t C, int64_t H, int64_t W, const int32_t* window_size,
                  const int32_t* shift_size, Geometry* g) {
  FA_REQUIRE(window_size && shift_size && g, FA_ERR_INVALID, "null window/shift pointer");
  FA_REQUIRE(C > 0 && H > 0 && W > 0, FA_ERR_INVALID, "resolution must be positive");
  FA_REQUIRE(C < (1 << 20) && H < (1 << 20) && W < (1 << 20), FA_ERR_INVALID, "resolution too large");
  const int64_t res[3] = {C, H, W};
  g->C = C; g->H = H; g->W = W;
  int64_t n = 1;
  for (int i = 0; i < 3; ++i) {
    FA_REQUIRE(window_size[i] > 0, FA_ERR_INVALID, "window size must be positive");
    FA_REQUIRE(shift_size[i] >= 0, FA_ERR_INVALID, "shift size must be non-negative");
    int32_t ws = window_size[i], ss = shift_size[i];
    if (res[i] <= ws) {
      ws = (int32_t)res[i];
      ss = 0;
    }
    FA_REQUIRE(ss < ws || ss == 0, FA_ERR_INVALID, "shift must be smaller than the window");
    const int64_t pad = (ws - res[i] % ws) % ws;
    g->ws[i] = ws;
    g->ss[i] = ss;
    g->pf[i] = (int32_t)(pad / 2);
    g->padded[i] = res[i] + pad;
    g->grid[i] = g->padded[i] / ws;
    n *= ws;
  }
  FA_REQUIRE(n <= 4096, FA_ERR_INVALID, "window has too many tokens");
  g->N = (int32_t)n;
  g->nW = g->grid[0] * g->grid[1] * g->grid[2];
  FA_REQUIRE(g->nW < (int64_t)1 << 31, FA_ERR_INVALID, "too many windows");
  return FA_OK;
}

int make_band_geometry(int64_t C, int64_t H_band, int64_t H_field, int64_t W,
                       const int32_t* window_size, const int32_t* shift_size, Geometry* g) {
  int rc = make_geometry(C, H_field, W, window_size, shift_size, g);
  if (rc != FA_OK) return rc;
  const int32_t wh = g->ws[1];
  FA_REQUIRE(g->padded[1] == H_field, FA_ERR_UNSUPPORTED,
             "band sharding needs the field height to be a multiple of the window height");
  FA_REQUIRE(H_band > 0 && H_band <= H_field && H_band % wh == 0, FA_ERR_INVALID,
             "band height must be a positive multiple of the window height, at most the field height");
  FA_REQUIRE(g->ss[1] <= H_band, FA_ERR_INVALID, "halo deeper than the band");
  g->H = H_band;
  g->padded[1] = H_band;
  g->grid[1] = H_band / wh;
  g->nW = g->grid[0] * g->grid[1] * g->grid[2];
  return FA_OK;
}

}  // namespace fa

using namespace fa;

extern "C" const char* fa_last_error(void) { return g_last_error.c_str(); }

extern "C" int fa_version(void) { return 100; }

extern "C" int fa_window_geometry(int64_t C, int64_t H, int64_t W, const int32_t window_size[3],
                                  const int32_t shift_size[3], int32_t ws_out[3], int32_t ss_out[3],
                                  int32_t pad_front_out[3], int64_t padded_out[3],
                                  int64_t* num_windows_out, int32_t* window_tokens_out) {
  Geometry g;
  const int rc = make_geometry(C, H, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  for (int i = 0; i < 3; ++i) {
    if (ws_out) ws_out[i] = g.ws[i];
    if (ss_out) ss_out[i] = g.ss[i];
    if (pad_front_out) pad_front_out[i] = g.pf[i];
    if (padded_out) padded_out[i] = g.padded[i];
  }
  if (num_windows_out) *num_windows_out = g.nW;
  if (window_tokens_out) *window_tokens_out = g.N;
  return FA_OK;
}

namespace {

// Python slice(start, stop) over an axis of length n, with negative indices counted from the
// end and clamped to [0, n]; "none" means the open end. Used to restate the three region
// slices of swin3d.py:567-569 exactly, including their degenerate forms when a shift is 0.
struct Span { int64_t lo, hi; };

int64_t clamp_index(int64_t i, int64_t n) {
  if (i < 0) i += n;
  return std::min<int64_t>(std::max<int64_t>(i, 0), n);
}

void region_spans(int64_t n, int64_t w, int64_t s, Span out[3]) {
  // slice(0, -w), slice(-w, -s), slice(-s, None); "-0" is 0 in Python.
  out[0] = {0, clamp_index(-w, n)};
  out[1] = {clamp_index(-w, n), s == 0 ? 0 : clamp_index(-s, n)};
  out[2] = {s == 0 ? 0 : clamp_index(-s, n), n};
}

}  // namespace

extern "C" int fa_shifted_window_groups(int64_t C, int64_t H, int64_t W,
                                        const int32_t window_size[3], const int32_t shift_size[3],
                                        int warped, uint8_t* groups_out) {
  Geometry g;
  const int rc = make_geometry(C, H, W, window_size, shift_size, &g);
  if (rc != FA_OK) return rc;
  FA_REQUIRE(groups_out, FA_ERR_INVALID, "null output pointer");
  FA_REQUIRE(g.nW * g.N <= ((int64_t)1 << 31), FA_ERR_INVALID, "mask too large");
  std::vector<uint8_t> img((size_t)(C * H * W), 0);
  Span sc[3], sh[3], sw[3];
  region_spans(C, g.ws[0], g.ss[0], sc);
  region_spans(H, g.ws[1], g.ss[1], sh);
  region_spans(W, g.ws[2], g.ss[2], sw);
  int cnt = 0;
  for (int ic = 0; ic < 3; ++ic)
    for (int ih = 0; ih < 3; ++ih)
      for (int iw = 0; iw < 3; ++iw, ++cnt)
        for (int64_t c = sc[ic].lo; c < sc[ic].hi; ++c)
          for (int64_t h = sh[ih].lo; h < sh[ih].hi; ++h)
            for (int64_t w = sw[iw].lo; w < sw[iw].hi; ++w) img[(size_t)((c * H + h) * W + w)] = (uint8_t)cnt;
  if (warped) {
    // swin3d.py:502-514: groups (1,2), (4,5), (7,8) of each C slice (offset 9) are joined.
    static const int pairs[3][2] = {{1, 2}, {4, 5}, {7, 8}};
    for (int i = 0; i < 3; ++i)
      for (int k = 0; k < 3; ++k) {
        const uint8_t a = (uint8_t)(pairs[k][0] + 9 * i), b = (uint8_t)(pairs[k][1] + 9 * i);
        for (auto& v : img)
          if (v == a) v = b;
      }
  }
  // Pad tokens form their own group `cnt` (swin3d.py:589-591); window partition order of
  // swin3d.py:450-451.
  const int64_t Hp = g.padded[1], Wp = g.padded[2];
  const int64_t W1 = g.grid[2], HW1 = g.grid[1] * g.grid[2];
  for (int64_t win = 0; win < g.nW; ++win) {
    const int64_t c1 = win / HW1, h1 = (win % HW1) / W1, w1 = win % W1;
    for (int32_t n = 0; n < g.N; ++n) {
      const int32_t wc = n / (g.ws[1] * g.ws[2]);
      const int32_t wh = (n / g.ws[2]) % g.ws[1];
      const int32_t ww = n % g.ws[2];
      const int64_t c = c1 * g.ws[0] + wc - g.pf[0];
      const int64_t h = h1 * g.ws[1] + wh - g.pf[1];
      const int64_t w = w1 * g.ws[2] + ww - g.pf[2];
      uint8_t v = (uint8_t)cnt;
      if (c >= 0 && c < C && h >= 0 && h < H && w >= 0 && w < W) v = img[(size_t)((c * H + h) * W + w)];
      groups_out[win * g.N + n] = v;
    }
  }
  (void)Hp; (void)Wp;
  return FA_OK;
}
