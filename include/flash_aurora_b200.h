/*
 * flash_aurora_b200 — C ABI of the B200 (sm_100a) Swin3D backbone block hot path.
 *
 * One shared library (libflash_aurora_b200.so) exports these entry points. They take plain
 * device pointers, sizes and a CUDA stream (cudaStream_t passed as void*), launch
 * asynchronously on that stream, never allocate device memory, never synchronise, and return
 * an int status (FA_OK = 0, negative on error; fa_last_error() describes the last failure of
 * the calling thread). Nothing here aborts the process.
 *
 * Each entry point replaces one call site of the upstream Flash-Aurora Python/Triton/CuTe-DSL
 * implementation; the citation is given beside it (paths relative to that project).
 */
#ifndef FLASH_AURORA_B200_H
#define FLASH_AURORA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (FA_F16 only where a function says so). */
enum { FA_F32 = 0, FA_BF16 = 1, FA_F16 = 2 };

/* Status codes. */
enum {
  FA_OK = 0,
  FA_ERR_INVALID = -1,     /* bad argument: null pointer, shape, stride, alignment, dtype */
  FA_ERR_UNSUPPORTED = -2, /* valid but not implemented here (e.g. head_dim != 64) */
  FA_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed; message has the CUDA error */
  FA_ERR_TIMEOUT = -4      /* a bounded device-side wait gave up (see fa_attention_status) */
};

/* Window-attention precision (upstream WinAttnPrecision, ops/cute/window_attn_fwd.py:49-60). */
enum {
  FA_ATTN_BF16 = 0,        /* bf16 in/out, fp32 accumulation and softmax */
  FA_ATTN_FP32_3XTF32 = 1  /* fp32 in/out, 3xTF32 split products, fp32 softmax */
};

enum { FA_ATTN_FLAG_REGIONS_FIT = 1 };

/* Attention output layouts (upstream output_layout "bhnd" / "bnc", window_attn_fwd.py:246-255). */
enum { FA_LAYOUT_BHND = 0, FA_LAYOUT_BNC = 1 };

/* Message for the last failing call on this thread ("" if none). */
const char* fa_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int fa_version(void);

/*
 * Window geometry of one block call: window/shift after the clamp of
 * flash_aurora/aurora/model/util.py:54-72, the front pads (C front, H top, W left) of the
 * symmetric zero padding (swin3d.py:415-432), the padded extents, the window count
 * nW = (Cp/wc)(Hp/wh)(Wp/ww) and the tokens per window N = wc*wh*ww
 * (ops/triton_swin3d_layout.py:78-88). Host-only.
 */
int fa_window_geometry(int64_t C, int64_t H, int64_t W, const int32_t window_size[3],
                       const int32_t shift_size[3], int32_t ws_out[3], int32_t ss_out[3],
                       int32_t pad_front_out[3], int64_t padded_out[3], int64_t* num_windows_out,
                       int32_t* window_tokens_out);

/*
 * Fused cyclic shift (roll by -ss) + zero pad + 3D window partition:
 * x (B, C, H, W, D) -> windows (B*nW, N, D). Replaces roll_pad_partition_windows_triton
 * (ops/triton_swin3d_layout.py:58-121, kernel :192-250). x_dtype/windows_dtype are FA_F32 or
 * FA_BF16 (an f32 -> bf16 store rounds to nearest even; bf16 -> f32 is exact). Bit-exact
 * gather: every output element is an input element or +0.
 */
int fa_roll_pad_partition(const void* x, int x_dtype, void* windows, int windows_dtype,
                          int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                          const int32_t window_size[3], const int32_t shift_size[3], void* stream);

/*
 * Inverse: windows (B*nW, N, D) -> out (B, C, H, W, D), reading only non-pad tokens.
 * Replaces crop_roll_unmerge_windows_triton (ops/triton_swin3d_layout.py:124-189, kernel
 * :253-307).
 */
int fa_crop_roll_unmerge(const void* windows, int windows_dtype, void* out, int out_dtype,
                         int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                         const int32_t window_size[3], const int32_t shift_size[3], void* stream);

/*
 * Fused AdaLN: out = [residual +] LN(x) * (scale_bias + scale) + shift, LN without affine,
 * statistics in fp32 from a single read of x. x: (B, L, D) f32|bf16; residual: (B, L, D) or
 * NULL; scale/shift: (B, D) rows (mod_dtype f32|bf16); out: (B, L, D) in out_dtype; out_bf16:
 * optional second copy of out rounded to bf16 (NULL to skip). D <= 2048. Replaces
 * adaptive_layernorm_film_forward / adaptive_layernorm_film_add_residual_forward
 * (ops/triton_adaln.py:33-145, kernel :148-203; module film.py:72-139).
 */
int fa_adaln_film(const void* x, int x_dtype, const void* residual, int residual_dtype,
                  const void* scale, const void* shift, int mod_dtype, float scale_bias, float eps,
                  void* out, int out_dtype, void* out_bf16, int64_t B, int64_t L, int64_t D,
                  void* stream);

/*
 * fa_adaln_film on the token rows (b, c, h, w) of a (B, C*H*W, D) grid with h in
 * [h_begin, h_begin + h_count) only; every other row of out / out_bf16 is left untouched. Two
 * calls over complementary ranges write what one fa_adaln_film writes, so a caller can finish
 * the rows a neighbour waits on first (the next shifted block's halo rows of a latitude band)
 * and hand them to a transfer while the rest are computed. No reference counterpart.
 */
int fa_adaln_film_rows(const void* x, int x_dtype, const void* residual, int residual_dtype,
                       const void* scale, const void* shift, int mod_dtype, float scale_bias,
                       float eps, void* out, int out_dtype, void* out_bf16, int64_t B, int64_t C,
                       int64_t H, int64_t W, int64_t D, int64_t h_begin, int64_t h_count,
                       void* stream);

/*
 * crop_roll_unmerge fused into the AdaLN above: the AdaLN input row of token (c, h, w) is read
 * straight from the attention windows (B*nW, N, D), so the merged branch tensor is never
 * written. Replaces the pair swin3d.py:751-756 (unmerge) + film.py:101-139 (norm1).
 */
int fa_unmerge_adaln_film(const void* windows, int windows_dtype, const void* residual,
                          int residual_dtype, const void* scale, const void* shift, int mod_dtype,
                          float scale_bias, float eps, void* out, int out_dtype, void* out_bf16,
                          int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                          const int32_t window_size[3], const int32_t shift_size[3], void* stream);

/*
 * fa_adaln_film that also scatters every output row, in windows_dtype, into the window layout
 * (B * nW, N, D) that fa_roll_pad_partition would produce from `out` for (window_size,
 * shift_size): the norm2 of one block fused with the partition of the next. Only token slots are
 * written; the caller keeps the pad slots of `windows` zero (for example one zero-filled buffer
 * reused by every block of a stage). x, residual, out: (B, C*H*W, D). No counterpart in the
 * reference (there, swin3d.py:800-815 is followed by the next block's partition, :742-750).
 */
int fa_adaln_film_partition(const void* x, int x_dtype, const void* residual, int residual_dtype,
                            const void* scale, const void* shift, int mod_dtype, float scale_bias,
                            float eps, void* out, int out_dtype, void* windows, int windows_dtype,
                            int64_t B, int64_t C, int64_t H, int64_t W, int64_t D,
                            const int32_t window_size[3], const int32_t shift_size[3], void* stream);

/*
 * Latitude-band sharding of a field (C, H_field, W) across ranks: each rank holds a band of
 * H_band whole window rows, x (B, C, H_band, W, D). No reference counterpart: the upstream
 * backbone runs one field per device (its only multi-device path is a pipeline placement,
 * engine/distributed/rollout_pipeline.py:137-169). window_size / shift_size are the field's;
 * clamping is decided on the field, which must need no H padding. With an H shift s = ss[1],
 * the band's shifted windows start s rows into the band:
 *
 *  - fa_roll_pad_partition_band: windows of the band; rows past the band are read from `halo`
 *    (B, C, s, W, D), the next band's first s rows (cyclically: the last band takes band 0's).
 *    halo_dtype is x_dtype, or windows_dtype when the neighbour sends its rows already rounded
 *    to the windows' type (bit-identical: the rounding commutes with the gather; half the bytes
 *    for fp32 -> bf16).
 *  - fa_band_halo_extract: halo_out (B, C, s, W, D) = the band's last s shifted rows, unrolled
 *    in C and W; they are the next band's first s original rows (its halo-back buffer).
 *  - fa_crop_roll_unmerge_band / fa_unmerge_adaln_film_band: inverse (plain, or fused with
 *    AdaLN + residual as fa_unmerge_adaln_film); rows 0..s-1 of the band are read from `halo_in`
 *    (B, C, s, W, D, windows dtype), the previous band's halo extract. The AdaLN form writes only
 *    the band rows [h_begin, h_begin + h_count) (0 and H_band for all of them); `halo_in` may be
 *    NULL when h_begin >= s, so the rows that need no halo can run while it is in flight.
 *
 * Window order inside the band is (c1, h1, w1) over the band's own grid, so the band's windows
 * are the rows [h1_begin, h1_end) of the field's window grid; region ids for a mask are sliced
 * from the field's (nW, N) ids in the same way. With s = 0 the halo pointers may be NULL.
 */
int fa_roll_pad_partition_band(const void* x, const void* halo, int x_dtype, int halo_dtype, void* windows,
                               int windows_dtype, int64_t B, int64_t C, int64_t H_band,
                               int64_t H_field, int64_t W, int64_t D, const int32_t window_size[3],
                               const int32_t shift_size[3], void* stream);
int fa_band_halo_extract(const void* windows, int windows_dtype, void* halo_out, int halo_dtype,
                         int64_t B, int64_t C, int64_t H_band, int64_t H_field, int64_t W,
                         int64_t D, const int32_t window_size[3], const int32_t shift_size[3],
                         void* stream);
int fa_crop_roll_unmerge_band(const void* windows, const void* halo_in, int windows_dtype,
                              void* out, int out_dtype, int64_t B, int64_t C, int64_t H_band,
                              int64_t H_field, int64_t W, int64_t D, const int32_t window_size[3],
                              const int32_t shift_size[3], void* stream);
int fa_unmerge_adaln_film_band(const void* windows, const void* halo_in, int windows_dtype,
                               const void* residual, int residual_dtype, const void* scale,
                               const void* shift, int mod_dtype, float scale_bias, float eps,
                               void* out, int out_dtype, void* out_bf16, int64_t B, int64_t C,
                               int64_t H_band, int64_t H_field, int64_t W, int64_t D,
                               const int32_t window_size[3], const int32_t shift_size[3],
                               int64_t h_begin, int64_t h_count, void* stream);

/*
 * Exact GELU, out[i] = x[i] * Phi(x[i]) = x[i] * 0.5 * (1 + erf(x[i] / sqrt(2))) in fp32, rounded to
 * dtype (FA_F32 | FA_BF16); n elements, contiguous; out == x (in place) is allowed, any other
 * overlap is rejected. Replaces the nn.GELU() between fc1 and fc2 of the block MLP
 * (swin3d.py:73-109), which upstream runs as a PyTorch elementwise kernel.
 * method FA_GELU_ERFF: PyTorch's arithmetic (erff), bit-identical to it.
 * method FA_GELU_POLY: Phi from a fitted erfc form without the 1 + erf cancellation, about 1.5x
 * cheaper; bf16 results equal the correctly rounded GELU for |x| < 4.
 */
enum { FA_GELU_ERFF = 0, FA_GELU_POLY = 1 };
int fa_gelu_erf(const void* x, void* out, int dtype, int64_t n, int method, void* stream);

/*
 * Linear layer with a fused bias and activation on the tensor cores (tcgen05, 128 x 256 tiles):
 * out[m, n] = act(sum_k a[m, k] * w[n, k] + bias[n]) for a (M, K), w (N, K) (nn.Linear layout),
 * bias (N), out (M, N), all bf16 and row-major with row strides lda, ldw, ldo (elements), fp32
 * accumulation, act FA_ACT_NONE or FA_ACT_GELU (exact GELU through the fitted erfc form of
 * fa_gelu_erf, applied to the fp32 sum). N % 256 == 0, K % 64 == 0, 16-byte aligned rows.
 * Replaces the fc1 -> nn.GELU() pair of the block MLP (swin3d.py:73-109), where upstream runs a
 * cuBLAS GEMM (bf16 autocast) and then a separate activation kernel.
 * fa_gemm_status reads the kernel's status word (0, or the code of the first wait that timed out);
 * fa_gemm_status_reset clears it (stream-ordered).
 */
enum { FA_ACT_NONE = 0, FA_ACT_GELU = 1 };
int fa_linear_bias_act(const void* a, const void* w, const void* bias, void* out, int64_t M, int64_t N,
                       int64_t K, int64_t lda, int64_t ldw, int64_t ldo, int act, void* stream);
int fa_gemm_status(int* status_out);
int fa_gemm_status_reset(void* stream);

/*
 * Stage-boundary gathers fused with their LayerNorm (affine weight/bias, fp32):
 *  - fa_patch_merge_ln: x (B, C, H, W, D) -> out (B, C*ceil(H/2)*ceil(W/2), 4D), the 2 x 2 patch
 *    of each output token (zero pad at the back of odd H / W; channel (dh*2 + dw)*D + d), then
 *    LayerNorm(4D). Replaces the pad/permute/LayerNorm of PatchMerging3D (swin3d.py:818-861)
 *    before its reduction linear.
 *  - fa_patch_split_ln: z (B, C, H, W, 4*Dq) (the output of PatchSplitting3D's first linear) ->
 *    out (B, (C-crop0)*(2H-crop1)*(2W-crop2), Dq): sub-token (dh, dw) of each token, crop at the
 *    back, then LayerNorm(Dq). Replaces the permute/crop/LayerNorm of PatchSplitting3D
 *    (swin3d.py:864-919) before its second linear.
 * D, Dq multiples of 8; 4D and Dq at most 4096; 16-byte aligned tensors.
 */
int fa_patch_merge_ln(const float* x, float* out, const float* weight, const float* bias, int64_t B, int64_t C,
                      int64_t H, int64_t W, int64_t D, float eps, void* stream);
int fa_patch_split_ln(const float* z, float* out, const float* weight, const float* bias, int64_t B, int64_t C,
                      int64_t H, int64_t W, int64_t Dq, const int32_t crop[3], float eps, void* stream);

/*
 * Shifted-window region ids of every window token, (nW, N) uint8 written to HOST memory.
 * Tokens i, j of a window attend to each other unmasked iff their ids are equal; otherwise the
 * logit gets the upstream -100 (compute_3d_shifted_window_mask, swin3d.py:526-599, with the
 * left/right merge of :502-514 when warped != 0 and pad tokens in their own group :589-591).
 */
int fa_shifted_window_groups(int64_t C, int64_t H, int64_t W, const int32_t window_size[3],
                             const int32_t shift_size[3], int warped, uint8_t* groups_out);

/*
 * Window attention: out = softmax(q k^T * scale + bias) v per (window, head), N tokens.
 * q, k, v, out are (Bwin, H, N, Dh) with element strides strides[0..11] =
 * {q: window, head, token, k: ..., v: ..., out: ...}; head-dim stride 1.
 * Mask (at most one): mask_u8 (nW, N, N) with 1 = masked, or group_ids (nW, N) with masked iff
 * ids differ; window b uses mask index b % nW. A masked logit gets -100 added after scaling
 * (upstream bias semantics, swin3d.py:597; CuTe kernel ops/cute/_kernel_bf16.py:361-365).
 * Supported: Dh == 64, 1 <= N <= 144 for FA_ATTN_BF16 and FA_ATTN_FP32_3XTF32.
 * flags: 0, or FA_ATTN_FLAG_REGIONS_FIT when every window of group_ids has at most 16 distinct ids,
 * all below 32 (true of the shifted-window ids of fa_shifted_window_groups); the bf16 kernel then
 * runs without its per-logit mask path. A window breaking that promise is left unmasked and
 * fa_attention_status reports 28.
 * Replaces window_attn_fwd_cute (ops/cute/window_attn_fwd.py:141-243).
 */
int fa_window_attention(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh,
                        const void* q, const void* k, const void* v, void* out,
                        const int64_t strides[12], const uint8_t* mask_u8,
                        const uint8_t* group_ids, int64_t nW, float scale, unsigned flags,
                        void* stream);

/*
 * Same on the packed output of Linear(D, 3D): qkv (Bwin, N, 3, H, Dh) contiguous; out is
 * (Bwin, H, N, Dh) for FA_LAYOUT_BHND or (Bwin, N, H*Dh) for FA_LAYOUT_BNC.
 * Replaces window_attn_fwd_cute_qkvpacked (ops/cute/window_attn_fwd.py:246-353).
 */
int fa_window_attention_qkvpacked(int precision, int64_t Bwin, int64_t N, int64_t H, int64_t Dh,
                                  const void* qkv, void* out, int out_layout,
                                  const uint8_t* mask_u8, const uint8_t* group_ids, int64_t nW,
                                  float scale, unsigned flags, void* stream);

/*
 * fa_window_attention with a float bias (bias < -50 means masked, as upstream), a contiguous
 * row-major fp32 (nW, N, N) array (there is no stride argument), that allocates no device memory. No counterpart in the reference: it exists for callers that cannot
 * call cudaMalloc (a host that owns the memory pool, a plugin forbidden to allocate, a loop that must
 * not allocate after start-up). The packed mask goes to a static 4 MiB device array of this
 * library, so nW * N * N must be <= 4194304 (larger sizes return FA_ERR_INVALID). The array's
 * device address is looked up on the first call on each device (call it once before any stream
 * capture) and cached for the process; after cudaDeviceReset the cached address is stale, so do
 * not call this entry point on a device that was reset. Every argument is checked before the
 * array is written. All calls share the array: calls that overlap on the GPU (other streams, other host
 * threads) race on it; serialise them. The caller still passes q, k, v, out and bias.
 */
int fa_window_attention_bias_noalloc(int precision, int64_t Bwin, int64_t H, int64_t N, int64_t Dh,
                                     const void* q, const void* k, const void* v, void* out,
                                     const int64_t strides[12], const float* bias, int64_t nW,
                                     float scale, void* stream);

/*
 * Perceiver decoder LayerNorm (+ residual): out = LayerNorm(x) * weight + bias (+ residual) over
 * the last dimension D of `rows` contiguous rows, in fp32, rounded once to x's dtype. Replaces
 * layernorm_affine_forward / layernorm_affine_add_residual_forward (ops/triton_perceiver_ln.py:25-47,
 * kernel :101-145), called by aurora/model/perceiver.py:255-276. x_dtype: FA_F32, FA_BF16 or
 * FA_F16; residual (nullable) and out have x's dtype and shape; weight / bias are (D,) of wb_dtype
 * (any of the three). 1 <= D <= 4096. out may alias x or residual.
 */
int fa_layernorm_affine(const void* x, int x_dtype, const void* residual, const void* weight, const void* bias,
                        int wb_dtype, float eps, void* out, int64_t rows, int64_t D, void* stream);

/*
 * Device status word of the attention kernels: 0 when every bounded wait of every launch since
 * the last reset completed, else the code of the first wait that gave up. Synchronises the
 * device. fa_attention_status_reset clears it (stream-ordered).
 */
int fa_attention_status(int* status_out);
int fa_attention_status_reset(void* stream);

/* Row kinds of fa_linear_adaln_film. */
enum { FA_ROWS_TOKENS = 0, FA_ROWS_WINDOWS = 1 };

/*
 * A bf16 linear with D = 512 output features whose rows are layer-normalised, FiLM-modulated and
 * added to the fp32 residual stream in the same kernel (the output h of the linear never reaches
 * HBM):
 *   h[m]    = bf16(a[m] . w^T + bias)           a (M, K) bf16 (row stride lda), w (512, K), bias (512) bf16
 *   out[t]  = residual[t] + LN(h[m]) * (scale_bias + scale[b]) + shift[b]     (fp32, eps as given)
 * scale / shift are fp32 (B, 512); residual / out fp32 (B * C*H*W, 512) token rows (out must not
 * alias residual). Replaces the linear + AdaLN pairs of the Swin3D block (swin3d.py:706-815,
 * film.py:101-139 / ops/triton_adaln.py:83-145 after ops/triton_swin3d_layout.py:124-189):
 *   FA_ROWS_WINDOWS  rows m are the window slots of this block's geometry (window_size, shift_size),
 *                    M = B * nW * N; token t = the slot's source token (pad slots write nothing):
 *                    attention proj fused with crop/un-roll/unmerge + norm1. out_bf16 (nullable,
 *                    (B * C*H*W, 512) bf16) receives a bf16 copy of out.
 *   FA_ROWS_TOKENS   rows m are tokens, M = B * C*H*W: MLP fc2 + norm2. win_out (nullable, bf16)
 *                    receives out in the window layout of a next block with next_shift_size (same
 *                    window size); its pad slots are left untouched.
 * K must be a multiple of 32; every pointer 16-byte aligned. Equals fa_linear_bias_act followed by
 * fa_unmerge_adaln_film / fa_adaln_film(_partition) up to the summation order of the fp32 row
 * statistics (the linear's bf16 rounding is the same).
 */
int fa_linear_adaln_film(const void* a, const void* w, const void* bias, int64_t M, int64_t K, int64_t lda,
                         int rows_kind, const float* scale, const float* shift, float scale_bias, float eps,
                         const float* residual, float* out, void* out_bf16, void* win_out, int64_t B,
                         int64_t C, int64_t H, int64_t W, const int32_t window_size[3],
                         const int32_t shift_size[3], const int32_t next_shift_size[3], void* stream);

/* Device status codes with a fixed meaning (the other non-zero codes name the bounded wait of a
 * kernel that gave up). */
enum {
  FA_STATUS_REGIONS_BROKEN = 28,      /* region ids tagged FA_ATTN_FLAG_REGIONS_FIT did not fit */
  FA_STATUS_WATCHDOG_SELFTEST = 90    /* written by fa_watchdog_selftest */
};

/*
 * Self-test of the bounded device-side waits (no counterpart in the reference): launches one warp
 * that waits, with a limit of timeout_ns (1 us .. 100 ms), on an mbarrier nothing arrives on. The
 * wait gives up, the kernel writes FA_STATUS_WATCHDOG_SELFTEST into the attention status word and
 * returns; nothing faults and the context stays usable. A host uses it to check that its status
 * polling (fa_attention_status after a sync point) sees a wait that expired.
 */
int fa_watchdog_selftest(int64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_AURORA_B200_H */
