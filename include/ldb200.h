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

#define LDB_ABI_VERSION 1

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
  LDB_CONV_1X1 = 3       /* pointwise conv / dense layer over tokens */
};

enum { LDB_ACT_NONE = 0, LDB_ACT_GELU = 1 };

/* Library ABI version (LDB_ABI_VERSION). */
LDB_API int ldb_version(void);

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
} ldb_conv_desc;

/* Workspace bytes ldb_conv3d_fwd needs (split-K partial tiles; 0 if none). */
LDB_API int ldb_conv3d_workspace_size(const ldb_conv_desc* desc, size_t* bytes);

/* Packed-weight geometry for `desc`: rows per parity (Cout padded to the
 * kernel's column tile) and K elements per row (taps * Cin_pad [* 2]). */
LDB_API int ldb_conv3d_weight_rows(const ldb_conv_desc* desc, int* rows_per_parity, int* k_total);

LDB_API int ldb_conv3d_fwd(ldb_stream_t stream, const ldb_conv_desc* desc, const void* x, const void* w_packed,
                   const float* bias, const float* shift, const void* residual, void* out, void* workspace,
                   size_t workspace_bytes);

#ifdef __cplusplus
}
#endif

#endif /* LDB200_H */
