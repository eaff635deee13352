/*
 * fcai_transforms.h -- C ABI of the B200 analysis/synthesis transform layers
 * of a FactorizedPrior (bmshj2018-factorized): 5x5 stride-2 convolutions
 * (g_a) and 5x5 stride-2 transposed convolutions with output padding 1
 * (g_s), each optionally followed by GDN / inverse GDN, computed as
 * implicit GEMMs on the sm_100a tensor cores (tcgen05, bf16 operands, fp32
 * accumulation in tensor memory, TMA tile loads).
 *
 * These layers replace the per-layer modules the reference swaps in for
 * reduced precision (backends/pytorch/bf16_operators.py:13-60:
 * BF16Conv2d, BF16ConvTranspose2d, BF16GDN), whose math is F.conv2d /
 * F.conv_transpose2d in bf16 and x * rsqrt(beta + conv1x1(x^2, gamma)).
 * Here GDN is fused into the convolution's epilogue as a second tensor-core
 * GEMM over the tile's full channel vector.
 *
 * Layouts
 *   activations  bf16 NHWC [B, H, W, C] (C = the layer's padded width), or
 *                fp32 NCHW [B, C, H, W] where stated
 *   weights      packed by the caller:
 *     TMA layers (cin % 64 == 0): bf16 [25][npad][cin], entry [ky*5+kx][n][c]
 *       = conv weight[n][c][ky][kx]  (Conv2d, torch layout [cout, cin, 5, 5])
 *       = deconv weight[c][n][ky][kx] (ConvTranspose2d, [cin, cout, 5, 5]),
 *       zero for n >= cout.
 *     scatter layers: bf16 [npad][cin], entry [(ky*5+kx)*cout + co][c] =
 *       deconv weight[c][co][ky][kx], npad = round16(25 * cout), zero above.
 *     first analysis layer (cin == 3, fp32 NCHW input): bf16 image of the
 *       operand tile, [npad rows][80 k] in 8x8 core matrices:
 *       element (n, k) at (n % 8) * 8 + (n / 8) * 640 + (k / 8) * 64 + k % 8,
 *       k = c * 25 + ky * 5 + kx (< 75, zero above).
 *   gdn_gamma    bf16 [npad][npad]: effective gamma[i][j] (norm_i = beta_i +
 *                sum_j gamma[i][j] x_j^2), zero padded.
 *   bias, gdn_beta  fp32 [cout].
 *
 * All calls are asynchronous on `stream` of the current device; they use no
 * workspace and allocate nothing.  `err` (device int, may be NULL) receives a
 * non-zero code if a pipeline wait timed out (a bug, never expected); the
 * kernel then stops early instead of waiting forever.
 */
#ifndef FCAI_TRANSFORMS_H
#define FCAI_TRANSFORMS_H

#include <stdint.h>

#include "fcai_warp_div.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { FCAI_LAYER_CONV5S2 = 0, FCAI_LAYER_DECONV5S2 = 1 };
enum { FCAI_EPI_NONE = 0, FCAI_EPI_GDN = 1, FCAI_EPI_IGDN = 2 };
enum { FCAI_FMT_NHWC_BF16 = 0, FCAI_FMT_NCHW_F32 = 1 };
/* FCAI_ALGO_IMPLICIT_GEMM: GEMM over output pixels x output channels, one CTA
 *   per tile of 128 output pixels.
 * FCAI_ALGO_IMPLICIT_GEMM_PAIR: the same GEMM on CTA pairs (clusters of 2):
 *   2-SM tensor-core MMAs over 256 output pixels, each SM staging half of the
 *   weight rows.  Layers with bf16 NHWC input and 128 or 192 output channels;
 *   results are identical to FCAI_ALGO_IMPLICIT_GEMM.
 * FCAI_ALGO_SCATTER: transposed convolutions with cout <= 10 (the last
 *   synthesis layer): GEMM over input pixels x (25 taps * cout) columns on
 *   halo tiles, each output pixel summing its taps in the epilogue, so the
 *   input is read about 1.5x instead of once per tap. */
enum { FCAI_ALGO_IMPLICIT_GEMM = 0, FCAI_ALGO_SCATTER = 1, FCAI_ALGO_IMPLICIT_GEMM_PAIR = 2 };
/* Operand precision of the convolution.  FCAI_PREC_FP8_E4M3 follows the
 * reference's FP8 candidates (backends/pytorch/fp8_operators.py: per-tensor
 * symmetric scales amax / 448, e4m3 operands, scaled GEMM, then bias): the
 * input is e4m3 NHWC (fcai_quantize_e4m3) with its scale at act_scale, the
 * weights are e4m3 packed like the bf16 TMA layers with scale weight_scale,
 * the accumulator is multiplied by act_scale * weight_scale before the bias
 * and epilogue.  TMA algorithm only, cin a multiple of 64 (K runs in blocks
 * of 128 channels; the part of the last block past cin reads as zeros);
 * npad 128 (bf16 NHWC output, optionally GDN / IGDN, whose norm GEMM stays
 * bf16), npad 192 with GDN / IGDN, or npad 192 / 160 without epilogue to
 * fp32 NCHW (latent layers). */
enum { FCAI_PREC_BF16 = 0, FCAI_PREC_FP8_E4M3 = 1 };

typedef struct {
    int32_t kind;       /* FCAI_LAYER_CONV5S2 or FCAI_LAYER_DECONV5S2 */
    int32_t cin;        /* input channels (3 with in_format NCHW_F32, else a multiple of 64) */
    int32_t cout;       /* output channels */
    int32_t npad;       /* MMA width: cout rounded up to 16 (<= 256; 128 or 192 with GDN/IGDN) */
    int32_t epilogue;   /* FCAI_EPI_* */
    int32_t in_format;  /* FCAI_FMT_*: NCHW_F32 only for the cin == 3 first analysis layer */
    int32_t out_format; /* FCAI_FMT_*: NHWC_BF16 stores npad channels; NCHW_F32 stores cout */
    int32_t clamp01;    /* clamp outputs to [0, 1] (NCHW_F32 output only) */
    int32_t algorithm;  /* FCAI_ALGO_* */
    int32_t precision;  /* FCAI_PREC_* */
    const void *weight; /* packed, see above */
    const float *bias;
    const float *gdn_beta;
    const void *gdn_gamma;
    const float *act_scale; /* FP8: device float, the input's scale (written by fcai_quantize_e4m3) */
    float weight_scale;     /* FP8: the weights' scale */
    int32_t out_channel_offset; /* NCHW_F32 output: channel of the output tensor this layer's channel 0
                                   lands on (0); a wider layer runs as several launches */
    uint32_t *amax_out;     /* optional (bf16 NHWC outputs): device word the layer raises to the float bits of
                               max |output| over the tensor (caller zeroes it), for an FP8 consumer's scale */
    int32_t out_channels_total; /* NCHW_F32 output: channels per image of the output tensor (0: cout) */
    int32_t reserved;
} fcai_layer;

/* Output spatial size of a layer for an input of h_in x w_in. */
int fcai_layer_out_size(const fcai_layer *layer, int32_t h_in, int32_t w_in, int32_t *h_out, int32_t *w_out);

/* One layer: output = epilogue(conv(input) + bias). */
int fcai_layer_forward(const fcai_layer *layer, int32_t batch, int32_t h_in, int32_t w_in, const void *input,
                       void *output, int32_t *err, fcai_stream_t stream);

/* Per-tensor symmetric e4m3 quantisation of a bf16 tensor of `count`
 * elements (count % 8 == 0, 16-byte aligned buffers), as the reference's
 * _symmetric_scale / _quantize_fp8 (backends/pytorch/fp8_operators.py:44-51):
 * scale = max(amax(|x|) * fl(1 / 448), FLT_MIN) (the reference's amax / 448.0,
 * which PyTorch's CUDA division by a host scalar evaluates this way),
 * out = e4m3(clamp(x / scale, +-448)) rounded to nearest even (NaN inputs give
 * 0x7F of either sign, as torch computes it on the GPU).  Writes the
 * scale to *scale_out (device).  With amax_ready = 0 the call computes the
 * amax into *amax_work (device, 4 bytes, cleared first); with amax_ready != 0,
 * *amax_work already holds it (the producing layer's amax_out) and the call
 * only quantises. */
int fcai_quantize_e4m3(const void *input_bf16, void *output_e4m3, float *scale_out, uint32_t *amax_work,
                       int32_t amax_ready, int64_t count, fcai_stream_t stream);

/* fp32 NCHW [B, C, H, W] -> bf16 NHWC [B, H, W, C] (C % 8 == 0). */
int fcai_nchw_f32_to_nhwc_bf16(const float *input, void *output, int32_t batch, int32_t channels, int32_t h,
                               int32_t w, fcai_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FCAI_TRANSFORMS_H */
