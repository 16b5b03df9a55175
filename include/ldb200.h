/*
 * ldb200.h - C ABI of the B200 (sm_100a) kernels behind the lesiondiffusion
 * denoiser and VQ-decoder hot path.
 *
 * Conventions
 *   - Every entry point is stream-ordered on the `stream` it receives and
 *     returns an int status: LDB_OK (0) or a negative LDB_ERR_* code.  A
 *     human-readable message for the last failure on the calling thread is
 *     available from ldb_last_error().  No C++ exception crosses the ABI.
 *   - Pointers are device pointers unless stated otherwise; memory is owned
 *     by the caller, including any workspace an entry point asks for.
 *   - Activations are NDHWC ("channels last"): element (b, d, h, w, c) of a
 *     tensor with channel stride `ld` sits at ((b*D + d)*H + h)*W + w)*ld + c.
 *     Token matrices (B, L, C) are the same layout with D = H = 1, W = L.
 *   - Kernels never trap: device-side waits are time-bounded and report
 *     through the device status word (ldb_device_status).
 *
 * Reference interfaces (lesiondiffusion-mlx 0.3.0, src/lesiondiffusion_mlx/)
 * each entry point replaces are cited beside it.
 */
#ifndef LDB200_H
#define LDB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LDB_API __attribute__((visibility("default")))
#else
#define LDB_API
#endif

typedef struct CUstream_st* ldb_stream_t; /* binary compatible with cudaStream_t */

#define LDB_ABI_VERSION 4

enum {
  LDB_OK = 0,
  LDB_ERR_INVALID = -1,   /* null pointer or invalid enum value */
  LDB_ERR_SHAPE = -2,     /* unsupported or inconsistent extents */
  LDB_ERR_ALIGNMENT = -3, /* pointer/stride alignment not met (16 bytes for TMA) */
  LDB_ERR_WORKSPACE = -4, /* workspace missing or too small */
  LDB_ERR_CUDA = -5       /* CUDA runtime/driver error (see ldb_last_error) */
};

enum { LDB_F16 = 0, LDB_F32 = 1, LDB_BF16 = 2 };

/* Convolution modes (ldb_conv_desc.mode). */
enum {
  LDB_CONV_3X3X3 = 0,    /* 3x3x3, padding 1, stride 1 */
  LDB_CONV_3X3X3_S2 = 1, /* 3x3x3, padding 1, stride 2 */
  LDB_CONV_UP2 = 2,      /* 3x3x3 of a nearest 2x upsampling, weights folded by ldb_pack_upsample_weight */
  LDB_CONV_1X1 = 3,      /* pointwise conv / dense layer over tokens */
  LDB_CONV_3X3X3_S2_PAD01 = 4 /* 3x3x3, stride 2, zero padding 0 before / 1 after each axis: the VQ
                                 encoder's downsample (lesiondiffusion_mlx/mlx_model.py:735-736) */
};

enum { LDB_ACT_NONE = 0, LDB_ACT_GELU = 1 };

/* Library ABI version (LDB_ABI_VERSION).  Version 2 added
 * ldb_conv_desc.struct_size as the descriptor's first field, version 3
 * ldb_conv_desc.max_ctas, version 4 the step-table row count (`steps`) of
 * ldb_timestep_embedding and ldb_sampler_step[_ex]. */
LDB_API int ldb_version(void);

/* Number of kernels this library has launched (or recorded into a CUDA
 * graph) in this process, for launch accounting in benchmarks. */
LDB_API unsigned long long ldb_launch_count(void);

/* Zero `bytes` bytes of device memory at ptr, ordered on the stream (a
 * memset; in a captured CUDA graph a memset node, not a kernel).  The
 * networks clear their GroupNorm statistics arena (the FP64 sums that
 * ldb_conv3d_fwd_gn_stats adds to) with it before each forward. */
LDB_API int ldb_clear_async(ldb_stream_t stream, void* ptr, size_t bytes);

/* Message describing the last failure on the calling thread. */
LDB_API const char* ldb_last_error(void);

/* Read (and optionally clear) the current device's status word; non-zero
 * bits mean a kernel timed out on a device-side wait (bit 0) or met a shape
 * it could not handle (bit 1).  Synchronizes with the device. */
LDB_API int ldb_device_status(unsigned int* status, int reset);

/* -------------------------------------------------------------------------
 * Convolution: replaces nax_conv3d (_nax_conv.py:451-619), its pack,
 * conv and split reduce kernels (_nax_conv.py:109-289), and the pointwise
 * conv / dense layers of SourceLayers (mlx_model.py:183-220).
 *
 * out[b, o, voxel] = act((sum_k x * w + bias[o] + shift[b, o]) * output_scale
 *                         + residual[b, o, voxel])
 * accumulated in FP32 and rounded once to out_dtype.  x is f16 NDHWC with
 * channel stride x_ld; in exact (FP32) mode x holds per voxel the f16 hi
 * plane then the 2^11-scaled lo plane (ldb_prepare_input), each padded to a
 * multiple of 16 channels.  The residual has the output's dtype and layout
 * (channel stride res_ld).  The input grid is (depth, height, width); the
 * output grid is the same (stride 1, 1x1), halved rounding up (stride 2) or
 * doubled (UP2).
 * ---------------------------------------------------------------------- */
typedef struct {
  /* sizeof(ldb_conv_desc) as the caller compiled it.  Every entry point that
   * takes a descriptor rejects any other value with LDB_ERR_INVALID, so a
   * binding written against another layout of this struct fails cleanly
   * instead of reading past what it passed.  Bindings that mirror the struct
   * (ctypes, cffi) set it to their own structure size. */
  int struct_size;
  int batch, depth, height, width; /* input grid */
  int in_channels;                 /* channels read from x (per plane) */
  int x_ld;                        /* channel stride of x, multiple of 8 */
  int out_channels;
  int out_ld;       /* channel stride of out */
  int res_ld;       /* channel stride of residual */
  int mode;         /* LDB_CONV_* */
  int exact;        /* 1: FP32 via the split-f16 three-product scheme */
  int out_dtype;    /* LDB_F16 or LDB_F32 */
  int act;          /* LDB_ACT_* */
  float output_scale;
  /* Depth halo: the first and last `depth_halo` of x's `depth` slices are a
   * neighbour's slices (or zeros at the volume ends) that the 3x3x3 taps read
   * instead of zero padding; the output covers the depth - 2 * depth_halo
   * interior slices (twice that for LDB_CONV_UP2).  0 or 1; not with stride 2 (modes 1 and 4).
   * Used by the depth-sharded decode, where each GPU holds a slab. */
  int depth_halo;
  /* Upper bound on the CTAs (SMs) the conv occupies; 0: all SMs.  Leaving a
   * few SMs free lets a communication kernel running beside the conv (the
   * halo exchange of the depth-sharded decode) make progress during it. */
  int max_ctas;
  /* Optional device pointer to two 64-bit words (start, end) for timing the
   * launch from the device clock (%globaltimer, ns): the kernel lowers start
   * (atomic min) to the time its first CTA passes its dependency wait and
   * raises end (atomic max) to the time its last CTA, or the split-K reduce,
   * finishes.  The caller sets start high and end to 0 before the launch.
   * Null: no timing. */
  unsigned long long* clock;
} ldb_conv_desc;

/* Workspace bytes ldb_conv3d_fwd needs (split-K partial tiles; 0 if none). */
LDB_API int ldb_conv3d_workspace_size(const ldb_conv_desc* desc, size_t* bytes);

/* ldb_conv3d_fwd that also adds, per (batch, output channel), the sum and the
 * sum of squares of the output values as stored into `stats` (FP64,
 * [batch][out_channels][2]; zero it before the first producer call).  These
 * are the GroupNorm statistics of the output, so the layer that normalizes
 * it (ldb_group_norm_affine_from_stats) needs no statistics pass of its own.  The
 * reference computes them in the GroupNorm call that follows the conv
 * (medmlx-core group_norm_affine at lesiondiffusion_mlx/mlx_model.py:328-335);
 * summation order follows the GPU schedule, so the last bits can differ
 * between runs. */
LDB_API int ldb_conv3d_fwd_gn_stats(ldb_stream_t stream, const ldb_conv_desc* desc, const void* x,
                                    const void* w_packed, const float* bias, const float* shift,
                                    const void* residual, void* out, double* stats, void* workspace,
                                    size_t workspace_bytes);

/* Packed-weight geometry for `desc`: rows per parity (Cout padded to the
 * kernel's column tile) and K elements per row (taps * Cin_pad [* 2]). */
LDB_API int ldb_conv3d_weight_rows(const ldb_conv_desc* desc, int* rows_per_parity, int* k_total);

LDB_API int ldb_conv3d_fwd(ldb_stream_t stream, const ldb_conv_desc* desc, const void* x, const void* w_packed,
                   const float* bias, const float* shift, const void* residual, void* out, void* workspace,
                   size_t workspace_bytes);

/* -------------------------------------------------------------------------
 * Group normalization: replaces medmlx-core's group_norm_affine (called at
 * mlx_model.py:328-335 and _scaled_vq.py:93-100).  The input is the channel
 * concatenation [x1 | x2] (c2 = 0 for a single tensor) of f16 or f32 NDHWC
 * tensors with `voxels` voxels per batch item.  Writes the per-(batch,
 * channel) FP32 affine (scale, offset) of GroupNorm(groups, eps, gamma,
 * beta): affine[(b * C + c) * 2 + {0, 1}].  gamma/beta are f32 (null = 1/0).
 * ---------------------------------------------------------------------- */
LDB_API int ldb_group_norm_workspace_size(int batch, int voxels, int channels, size_t* bytes);
LDB_API int ldb_group_norm_affine(ldb_stream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2,
                                  int ld2, int dtype, int batch, int voxels, int groups, const float* gamma,
                                  const float* beta, float eps, float* affine, void* workspace,
                                  size_t workspace_bytes);

/* Allocation-free variant of ldb_group_norm_affine (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they
 * call -- e.g. an engine that owns every device allocation up front, or a
 * binding without access to a device allocator -- so they cannot provide a
 * workspace.  The partial sums use a fixed 4 MiB device array inside the
 * library (held by every GPU that loads it until exit), so
 * batch * channels must not exceed 524288; larger calls fail with
 * LDB_ERR_SHAPE.  Performs no cudaMalloc / cudaFree.  The first call on a
 * device looks up the array's device address (make it before any stream
 * capture).  Under lazy module loading (the CUDA 12 default) the driver
 * places the array in device memory only at that first call or at the first
 * launch of another GroupNorm kernel of the library: make the first call
 * before reserving all device memory, or set CUDA_MODULE_LOADING=EAGER.  All calls share the array: calls that overlap on the GPU race.
 * Same arguments and results as ldb_group_norm_affine without the workspace. */
LDB_API int ldb_group_norm_affine_noalloc(ldb_stream_t stream, const void* x1, int c1, int ld1, const void* x2,
                                          int c2, int ld2, int dtype, int batch, int voxels, int groups,
                                          const float* gamma, const float* beta, float eps, float* affine);

/* Conv-input preparation: replaces the pack kernel of _nax_conv.py:109-155
 * (and native_group_norm, mlx_model.py:348-358, when used with an affine).
 * out = f16(silu?(x * scale + offset)) over [x1 | x2], or with split = 1 the
 * exact-mode hi / 2^11-scaled lo planes (each padded to 16 channels).
 * Channels are zero padded up to out_ld's plane width. */
LDB_API int ldb_prepare_input(ldb_stream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2,
                              int ld2, int dtype, int batch, int voxels, const float* affine, int silu, int split,
                              void* out, int out_ld);

/* GroupNorm affine (scale, offset per batch and channel, as
 * ldb_group_norm_affine) from producer statistics instead of a pass over the
 * tensor: `stats1` / `stats2` are the FP64 [batch][channels][2] sums and sums
 * of squares of the two channel blocks [x1 | x2] (x2 may be absent, c2 = 0),
 * as ldb_conv3d_fwd_gn_stats accumulates them; `voxels` per batch item.
 * Replaces the statistics half of medmlx-core's group_norm_affine
 * (lesiondiffusion_mlx/mlx_model.py:328-335). */
LDB_API int ldb_group_norm_affine_from_stats(ldb_stream_t stream, const double* stats1, int c1,
                                             const double* stats2, int c2, int batch, int voxels, int groups,
                                             const float* gamma, const float* beta, float eps, float* affine);

/* ldb_group_norm_affine_from_stats followed by ldb_prepare_input in one
 * launch: each block derives the affine of its batch item from the producer
 * statistics (the same values, bit for bit) into shared memory and applies it
 * with SiLU and the f16 rounding or FP32 hi/lo split.  `voxels` per batch
 * item are normalized; `stat_voxels` is the voxel count the statistics cover
 * (0: the same; larger when x is one slab of a volume whose statistics were
 * summed over all slabs).  Replaces the
 * reference's group_norm_affine + conv-prologue pair of a norm_silu_conv
 * (lesiondiffusion_mlx/mlx_model.py:328-342) when the producing convs
 * accumulated statistics. */
LDB_API int ldb_prepare_input_from_stats(ldb_stream_t stream, const void* x1, int c1, int ld1, const void* x2,
                                         int c2, int ld2, int dtype, int batch, int voxels, int stat_voxels,
                                         const double* stats1,
                                         const double* stats2, int groups, const float* gamma, const float* beta,
                                         float eps, int silu, int split, void* out, int out_ld);

/* LayerNorm over the last axis of f16 rows (mlx_model.py:360-367). */
LDB_API int ldb_layer_norm(ldb_stream_t stream, const void* x, int x_ld, const float* gamma, const float* beta,
                           float eps, void* out, int out_ld, int rows, int channels);

/* LayerNorm of f16 or f32 rows (x_dtype LDB_F16 / LDB_F32) in FP32; with
 * split = 1 the f16 output row holds the hi plane then the 2^11-scaled low
 * plane, each padded to a multiple of 16 channels (the FP32-exact conv input,
 * as ldb_prepare_input writes it), for the FP32 network. */
LDB_API int ldb_layer_norm_ex(ldb_stream_t stream, const void* x, int x_dtype, int x_ld, const float* gamma,
                              const float* beta, float eps, void* out, int out_ld, int rows, int channels, int split);

/* -------------------------------------------------------------------------
 * Attention: replaces flash_attention / flash_attention_half
 * (_attention.py:331-375, _attention_half.py:129-147) and the fused SDPA
 * cross-attention (mlx_model.py:477-487).  q (B, lq, q_ld), k/v (B, lk,
 * kv_ld), out (B, lq, out_ld); head h uses columns [h*head_dim, (h+1)*head_dim).
 * head_dim 16, 32 or 64, dtype LDB_F16 or LDB_BF16, any lq / lk.
 * ---------------------------------------------------------------------- */
LDB_API int ldb_flash_attention(ldb_stream_t stream, const void* q, int q_ld, const void* k, const void* v,
                                int kv_ld, void* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim,
                                float scale, int dtype);

/* ldb_flash_attention with a caller workspace that lets the kernel split the
 * keys over several CTAs when (query pairs x heads x batch) would leave SMs
 * idle: each split writes its unnormalised O rows and (max, sum) to the
 * workspace and a second kernel merges them (the online-softmax merge of
 * _attention_half.py:58-113 across key ranges).  With a null or too small
 * workspace it runs unsplit.  Workspace bytes from
 * ldb_flash_attention_workspace_size (0: no split would help). */
/* FP32 attention for 16-, 32- or 64-wide heads (the reference's FP32 flash_attention,
 * _attention.py:148-375): q, k, v, out are f32 projections (B, L, H*32) with
 * row strides q_ld / kv_ld / out_ld (multiples of 4, 16-byte aligned
 * pointers).  Runs the tcgen05 kernel in split-f16 form: Q * scale * log2(e),
 * K and V become f16 hi / low planes in `workspace`
 * (ldb_flash_attention_f32_workspace_size bytes); scores Qh Kh + Qh Kl + Ql Kh
 * and probabilities split the same way (2^11-scaled low planes for P and V),
 * FP32 accumulation and online softmax, output f32. */
LDB_API int ldb_flash_attention_f32_workspace_size(int batch, int lq, int lk, int heads, int head_dim,
                                                   size_t* bytes);
LDB_API int ldb_flash_attention_f32(ldb_stream_t stream, const float* q, int q_ld, const float* k, const float* v,
                                    int kv_ld, float* out, int out_ld, int batch, int lq, int lk, int heads,
                                    int head_dim, float scale, void* workspace, size_t workspace_bytes);

LDB_API int ldb_flash_attention_workspace_size(int batch, int lq, int lk, int heads, int head_dim, size_t* bytes);
/* ldb_flash_attention_ws timed from the device clock: `clock` (device, two
 * 64-bit words set high / 0 by the caller) receives the time the first CTA
 * passes its dependency wait (atomic min) and the time the last CTA or the
 * key-split merge finishes (atomic max), in ns of %globaltimer.  For
 * benchmarks; results are those of ldb_flash_attention_ws. */
LDB_API int ldb_flash_attention_timed(ldb_stream_t stream, const void* q, int q_ld, const void* k, const void* v,
                                      int kv_ld, void* out, int out_ld, int batch, int lq, int lk, int heads,
                                      int head_dim, float scale, int dtype, void* workspace, size_t workspace_bytes,
                                      unsigned long long* clock);
LDB_API int ldb_flash_attention_ws(ldb_stream_t stream, const void* q, int q_ld, const void* k, const void* v,
                                   int kv_ld, void* out, int out_ld, int batch, int lq, int lk, int heads,
                                   int head_dim, float scale, int dtype, void* workspace, size_t workspace_bytes);

/* -------------------------------------------------------------------------
 * Denoise-loop kernels.
 * ---------------------------------------------------------------------- */

/* Device-side step counter.  The denoise-step kernels below can read their
 * per-step inputs (timesteps, sampler coefficients, noise) from device tables
 * indexed by *step, so one captured CUDA graph of a step serves every step;
 * ldb_step_advance increments the counter on the stream.  Those kernels take
 * the tables' row count `steps` (>= 1 when step is given): with *step outside
 * [0, steps) (a step graph replayed past the end of its schedule) they read
 * and write nothing and set status bit 1 (ldb_device_status). */
LDB_API int ldb_step_advance(ldb_stream_t stream, int* step);

/* [cos, sin] timestep embedding (mlx_model.py:609-612); out (batch, channels).
 * timesteps is a device table [steps][batch]; step (device, optional)
 * selects the row (row 0 when null). */
LDB_API int ldb_timestep_embedding(ldb_stream_t stream, const int* timesteps, const int* step, int steps, int batch,
                                   int channels, void* out, int out_dtype);

/* Skinny dense layer for 1..16 rows (time-embedding MLP and the residual
 * blocks' embedding projections, mlx_model.py:434 and :614):
 * out = silu_out?(silu_in?(x) @ w^T + bias), f16 x / w, f32 bias. */
LDB_API int ldb_dense_small(ldb_stream_t stream, const void* x, int x_ld, const void* w, const float* bias, void* out,
                            int out_ld, int rows, int n_out, int k, int in_silu, int out_silu, int out_dtype,
                            int round_f16);

/* Fused sampler step (DdimSampler / Dpmpp2mSampler steps,
 * mlx_sampling.py:172-185, _dpm.py:320-333): kind 0 = compose only,
 * 1 = DDIM update with coefficients (alpha, previous, sigma, sqrt(1 - alpha), 0),
 * 2 = DPM++-2M update with (alpha, sigma, ratio, clean, history).
 * coeff_table is a device table [steps][5], noise a device buffer whose
 * step s starts at s * noise_step_stride; both are indexed by *step (0
 * when step is null).  x is the f32 (B, voxels, channels) state, updated in
 * place; with a mask the known region is re-imposed from `image`; net_in
 * (optional) receives the next f16 network input [x | mask] (or
 * [x | image]) with channel stride in_ld, zero padded. */
LDB_API int ldb_sampler_step(ldb_stream_t stream, int kind, float* x, float* prev, const void* eps, int eps_ld,
                             const float* noise, long long noise_step_stride, const float* mask,
                             const float* image, int image_channels, void* net_in, int in_ld, int batch,
                             int voxels, int channels, const float* coeff_table, const int* step, int steps);

/* ldb_sampler_step for either network: eps_dtype LDB_F16 or LDB_F32 (the
 * FP32 LMNet prediction); with net_split = 1 the next network input is
 * written as the FP32-exact conv input, the f16 hi plane then the 2^11-scaled
 * low plane of the input channels padded to a multiple of 16. */
LDB_API int ldb_sampler_step_ex(ldb_stream_t stream, int kind, float* x, float* prev, const void* eps, int eps_dtype,
                                int eps_ld, const float* noise, long long noise_step_stride, const float* mask,
                                const float* image, int image_channels, void* net_in, int in_ld, int net_split,
                                int batch, int voxels, int channels, const float* coeff_table, const int* step,
                                int steps);

/* Nearest 4-channel codebook search with the straight-through quantize
 * (nearest_codebook4, _vq.py:64-82; VqAutoencoder.quantize,
 * mlx_model.py:742-803).  indices[p] gets the code; `quantized` (optional)
 * gets z + (e - z) in the dtype with channel stride out_ld. */
LDB_API int ldb_vq_nearest4(ldb_stream_t stream, const void* z, int z_ld, long long positions, const void* codebook,
                            int entries, int dtype, int* indices, void* quantized, int out_ld);

/* Nearest resize of NDHWC rows of `row_bytes` bytes (upsample_nearest2 and
 * resize_nearest, _spatial.py:41-69). */
LDB_API int ldb_resize_nearest(ldb_stream_t stream, const void* x, int batch, int in_d, int in_h, int in_w,
                               int row_bytes, int x_row_stride, void* out, int out_d, int out_h, int out_w,
                               int out_row_stride);

/* Inverse CT map to HU of channel 0 of n voxels (piecewise_ct(inverse=True),
 * mlx_pipeline.py:72-96). */
LDB_API int ldb_hu_map(ldb_stream_t stream, const void* x, int dtype, int x_ld, long long n, float* out);

/* Forward CT map of n f32 HU values to the normalized range (piecewise_ct,
 * mlx_pipeline.py:72-96, inverse=False): knots (-1000, -200, 200, 1000) ->
 * (0, 0.2, 0.8, 1) with clipping, FP32 arithmetic, one rounding to out_dtype
 * (LDB_F16 for the VQ encoder input, medmlx.py:1289-1291); element i is
 * written at out + i * out_ld. */
LDB_API int ldb_ct_normalize(ldb_stream_t stream, const float* hu, long long n, void* out, int out_dtype, int out_ld);

/* -------------------------------------------------------------------------
 * Output-region compositing of a generated CT into the input CT
 * (localize_output and apply_lesion_change, medmlx.py:2531-2690).  Volumes
 * are dense float32 (n0, n1, n2) arrays in the reference's axis order.
 * ---------------------------------------------------------------------- */

/* output_region = "box": out = generated inside the box [start, stop) (host
 * arrays of 3), w * generated + (1 - w) * original within margin_mm of it
 * (w = 0.5 (1 + cos(pi d / margin)), d the Euclidean distance in mm between
 * voxel centres with per-axis spacing spacing_mm[3]), original elsewhere.
 * weighted_count (device, optional) gets the number of voxels with
 * d < margin added to it. */
LDB_API int ldb_localize_box(ldb_stream_t stream, const float* original, const float* generated, float* out, int n0,
                             int n1, int n2, const int* start, const int* stop, const double* spacing_mm,
                             double margin_mm, unsigned long long* weighted_count);

/* Lesion extent of a uint8 mask: extent[7] (device) = voxel count, minimum
 * index per axis, maximum index per axis. */
LDB_API int ldb_lesion_extent(ldb_stream_t stream, const uint8_t* lesion, int n0, int n1, int n2, int* extent);

/* output_region = "lesion": out = original + (generated - reconstruction)
 * within `reach` voxels of a lesion voxel along every axis, original
 * elsewhere (f32 arithmetic).  stats[3] (device) = the sum and count of
 * reconstruction - original over the reached non-lesion voxels with
 * |original| < 1000, and the reached count.  workspace >= 2 n0 n1 n2 bytes. */
LDB_API int ldb_apply_lesion_change(ldb_stream_t stream, const float* original, const float* generated,
                                    const float* reconstruction, const uint8_t* lesion, float* out, int n0, int n1,
                                    int n2, int reach, uint8_t* workspace, size_t workspace_bytes, double* stats);

#ifdef __cplusplus
}
#endif

#endif /* LDB200_H */
