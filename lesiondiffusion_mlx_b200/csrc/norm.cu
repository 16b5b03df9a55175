// GroupNorm statistics, the conv-input "prepare" pass (GN affine + SiLU +
// f16 rounding or FP32 hi/lo split, with optional two-source channel
// concatenation) and LayerNorm.  All are HBM-bound: rows are read with
// 16-byte vector loads, every warp's loads are contiguous, and reductions
// use warp shuffles plus one shared-memory stage.
//
// GroupNorm follows the reference's group_norm_affine / native_group_norm
// (medmlx-core, used at lesiondiffusion_mlx/mlx_model.py:328-358): biased
// variance per (batch, group) over the group's channels and all voxels,
// scale = gamma * rsqrt(var + eps), offset = beta - mean * scale, applied in
// FP32.  Statistics are accumulated per channel as shifted sums (shift =
// the channel's value at the first voxel) in FP32 per block and merged in
// FP64, so large means do not cancel the variance.

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "host_common.h"

namespace ldb {
namespace {

// A virtual NDHWC tensor made of up to two channel blocks [x1 | x2].
struct Src2 {
  const void* x1;
  const void* x2;
  int c1, c2;      // channels in each block
  int ld1, ld2;    // channel strides
  int f32;         // element type: 0 = f16, 1 = f32
};

__device__ __forceinline__ void load8(const Src2& s, long long voxel, int c, float (&v)[8]) {
  const void* base;
  int ld, cc;
  if (c < s.c1) {
    base = s.x1;
    ld = s.ld1;
    cc = c;
  } else {
    base = s.x2;
    ld = s.ld2;
    cc = c - s.c1;
  }
  if (s.f32) {
    const float* p = static_cast<const float*>(base) + voxel * ld + cc;
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const __half* p = static_cast<const __half*>(base) + voxel * ld + cc;
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(h[q]);
      v[2 * q] = f.x;
      v[2 * q + 1] = f.y;
    }
  }
}

// Per-channel shifted partial sums over one chunk of voxels of one batch
// item.  Block (chunk, b); each thread owns 8 consecutive channels of one
// voxel row and strides over rows.  partials[b][chunk][c] = (S1, S2).
__global__ void gn_partial_kernel(Src2 s, int voxels, int chunk_voxels, float2* partials, int nchunks) {
  pdl_begin();
  const int c_total = s.c1 + s.c2;
  const int vecs = c_total / 8;
  const int b = blockIdx.y;
  const int chunk = blockIdx.x;
  const int rows_per_iter = blockDim.x / vecs;  // >= 1 by launch configuration
  const int tid = threadIdx.x;
  const int lane_vec = tid % vecs;
  const int row0 = tid / vecs;
  const bool active = row0 < rows_per_iter;
  const int c = lane_vec * 8;
  float shift[8];
  float s1[8], s2[8];
  const long long batch_base = static_cast<long long>(b) * voxels;
  load8(s, batch_base, c, shift);
#pragma unroll
  for (int j = 0; j < 8; ++j) s1[j] = s2[j] = 0.f;
  const int v0 = chunk * chunk_voxels;
  const int v1 = min(voxels, v0 + chunk_voxels);
  if (active) {
    for (int v = v0 + row0; v < v1; v += rows_per_iter) {
      float x[8];
      load8(s, batch_base + v, c, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = x[j] - shift[j];
        s1[j] += d;
        s2[j] = fmaf(d, d, s2[j]);
      }
    }
  }
  // Reduce the rows_per_iter threads sharing a channel vector through smem.
  extern __shared__ float red[];  // [rows_per_iter][c_total][2]
  if (active) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      red[(row0 * c_total + c + j) * 2] = s1[j];
      red[(row0 * c_total + c + j) * 2 + 1] = s2[j];
    }
  }
  __syncthreads();
  for (int ch = tid; ch < c_total; ch += blockDim.x) {
    float a = 0.f, q = 0.f;
    for (int r = 0; r < rows_per_iter; ++r) {
      a += red[(r * c_total + ch) * 2];
      q += red[(r * c_total + ch) * 2 + 1];
    }
    partials[(static_cast<long long>(b) * nchunks + chunk) * c_total + ch] = make_float2(a, q);
  }
}

// One block per (batch, group): merge the per-channel partials in FP64 and
// write the per-channel affine (scale, offset).  Threads split the
// (chunk, channel) pairs of the group: with cpg <= 256 the block size is a
// multiple of cpg, so each thread keeps one channel and strides over chunks
// (consecutive threads read consecutive channels), then folds its sums into
// shared memory.
__global__ void gn_finalize_kernel(Src2 s, int voxels, const float2* partials, int nchunks, int groups,
                                   const float* gamma, const float* beta, float eps, float* affine) {
  pdl_begin();
  const int c_total = s.c1 + s.c2;
  const int cpg = c_total / groups;
  const int b = blockIdx.x / groups;
  const int g = blockIdx.x % groups;
  __shared__ double sh_a[1024];
  __shared__ double sh_q[1024];
  __shared__ double sh_gmean;
  __shared__ double sh_rstd;
  const double n = static_cast<double>(voxels);
  for (int j = threadIdx.x; j < cpg; j += blockDim.x) {
    sh_a[j] = 0.0;
    sh_q[j] = 0.0;
  }
  __syncthreads();
  const float2* base = partials + static_cast<long long>(b) * nchunks * c_total + g * cpg;
  if (cpg <= static_cast<int>(blockDim.x)) {
    const int lanes = (blockDim.x / cpg) * cpg;  // threads in use, a multiple of cpg
    if (threadIdx.x < lanes) {
      const int j = threadIdx.x % cpg;
      const int k0 = threadIdx.x / cpg;
      const int kstep = lanes / cpg;
      double a = 0.0, q = 0.0;
      for (int k = k0; k < nchunks; k += kstep) {
        const float2 p = base[static_cast<long long>(k) * c_total + j];
        a += p.x;
        q += p.y;
      }
      atomicAdd(&sh_a[j], a);
      atomicAdd(&sh_q[j], q);
    }
  } else {
    for (int j = threadIdx.x; j < cpg; j += blockDim.x) {
      double a = 0.0, q = 0.0;
      for (int k = 0; k < nchunks; ++k) {
        const float2 p = base[static_cast<long long>(k) * c_total + j];
        a += p.x;
        q += p.y;
      }
      sh_a[j] = a;
      sh_q[j] = q;
    }
  }
  __syncthreads();
  // Channel means and centred sums of squares (shift = the channel's value at voxel 0).
  const long long v0 = static_cast<long long>(b) * voxels;
  for (int j = threadIdx.x; j < cpg; j += blockDim.x) {
    const int c = g * cpg + j;
    double shift;
    if (c < s.c1) {
      shift = s.f32 ? static_cast<const float*>(s.x1)[v0 * s.ld1 + c]
                    : __half2float(static_cast<const __half*>(s.x1)[v0 * s.ld1 + c]);
    } else {
      const int cc = c - s.c1;
      shift = s.f32 ? static_cast<const float*>(s.x2)[v0 * s.ld2 + cc]
                    : __half2float(static_cast<const __half*>(s.x2)[v0 * s.ld2 + cc]);
    }
    const double a = sh_a[j];
    const double mean_shifted = a / n;
    const double m2 = fmax(sh_q[j] - a * mean_shifted, 0.0);
    sh_a[j] = shift + mean_shifted;
    sh_q[j] = m2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double gm = 0.0;
    for (int j = 0; j < cpg; ++j) gm += sh_a[j];
    gm /= cpg;
    double m2 = 0.0;
    for (int j = 0; j < cpg; ++j) {
      const double d = sh_a[j] - gm;
      m2 += sh_q[j] + n * d * d;
    }
    const double var = m2 / (n * cpg);
    sh_gmean = gm;
    sh_rstd = 1.0 / sqrt(var + static_cast<double>(eps));
  }
  __syncthreads();
  for (int j = threadIdx.x; j < cpg; j += blockDim.x) {
    const int c = g * cpg + j;
    const float gam = gamma ? gamma[c] : 1.f;
    const float bet = beta ? beta[c] : 0.f;
    const float scale = static_cast<float>(static_cast<double>(gam) * sh_rstd);
    const float offset = static_cast<float>(static_cast<double>(bet) - sh_gmean * static_cast<double>(scale));
    affine[(static_cast<long long>(b) * c_total + c) * 2] = scale;
    affine[(static_cast<long long>(b) * c_total + c) * 2 + 1] = offset;
  }
}

// out = prepare(x): optional affine (scale, offset per channel) and SiLU in
// FP32, then either one f16 rounding or the exact split into hi / 2^11-scaled
// lo planes (_nax_conv.py:109-155).  Channels past C up to the padded plane
// width are written as zeros.
//
// Each thread owns one 8-channel group c of one batch item for the whole
// pass: its 8 (scale, offset) pairs stay in registers and it walks voxels
// with a stride, four voxels' loads in flight before their stores.  Blocks
// are a whole number of channel-group rows (blockDim = rows x cpad / 8).
struct Affine8 {
  float sc[8], of[8];
  bool on;
};

__device__ __forceinline__ Affine8 load_affine8(const float* aff, int c, int c_total) {
  Affine8 a;
  a.on = aff != nullptr && c + 8 <= c_total;
  if (a.on) {
    const float4* a4 = reinterpret_cast<const float4*>(aff);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = a4[q];
      a.sc[2 * q] = t.x;
      a.of[2 * q] = t.y;
      a.sc[2 * q + 1] = t.z;
      a.of[2 * q + 1] = t.w;
    }
  }
  return a;
}

__device__ __forceinline__ void prepare_store(const float (&v)[8], int c, int c_total, const Affine8& a, int silu,
                                              int split, int cpad, __half* o) {
  uint4 hi_raw, lo_raw;
  __half* hi = reinterpret_cast<__half*>(&hi_raw);
  __half* lo = reinterpret_cast<__half*>(&lo_raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float y = 0.f;
    if (c + j < c_total) {
      y = v[j];
      if (a.on) y = fmaf(y, a.sc[j], a.of[j]);
      if (silu) y = silu_f32(y);
    }
    hi[j] = __float2half_rn(y);
    if (split) lo[j] = __float2half_rn((y - __half2float(hi[j])) * 2048.0f);
  }
  *reinterpret_cast<uint4*>(o) = hi_raw;
  if (split) *reinterpret_cast<uint4*>(o + cpad) = lo_raw;
}

// Voxels [0, voxels) of the batch item starting at global voxel v0.  The
// thread's first four loads go out before `get_affine()` is called (they only
// need the input), so deriving the affine overlaps their latency; every
// thread of the block calls get_affine() exactly once.
template <class GetAffine>
__device__ __forceinline__ void prepare_pass(const Src2& s, long long v0, int voxels, GetAffine get_affine, int c,
                                             int silu, int split, int cpad, __half* out, int out_ld) {
  const int c_total = s.c1 + s.c2;
  const int vecs = cpad / 8;
  const int rows = blockDim.x / vecs;
  const long long stride = static_cast<long long>(gridDim.x) * rows;
  const bool live = c + 8 <= c_total;
  long long v = static_cast<long long>(blockIdx.x) * rows + threadIdx.x / vecs;
  Affine8 a;
  {
    float x[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (live && v + u * stride < voxels) {
        load8(s, v0 + v + u * stride, c, x[u]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[u][j] = 0.f;
      }
    }
    a = get_affine();
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v + u * stride < voxels)
        prepare_store(x[u], c, c_total, a, silu, split, cpad, out + (v0 + v + u * stride) * out_ld + c);
    v += 4 * stride;
  }
  for (; v + 3 * stride < voxels; v += 4 * stride) {
    float x[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (live) {
        load8(s, v0 + v + u * stride, c, x[u]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[u][j] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      prepare_store(x[u], c, c_total, a, silu, split, cpad, out + (v0 + v + u * stride) * out_ld + c);
  }
  for (; v < voxels; v += stride) {
    float x[8];
    if (live) {
      load8(s, v0 + v, c, x);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = 0.f;
    }
    prepare_store(x, c, c_total, a, silu, split, cpad, out + (v0 + v) * out_ld + c);
  }
}

// Block (x, b): batch item b; `affine` is (B, C, 2) or null.
__global__ void prepare_kernel(Src2 s, int voxels_per_batch, const float* affine, int silu, int split, int cpad,
                               __half* out, int out_ld) {
  pdl_begin();
  const int c_total = s.c1 + s.c2;
  const int c = (threadIdx.x % (cpad / 8)) * 8;
  const int b = blockIdx.y;
  auto get_affine = [&] {
    return load_affine8(affine ? affine + (static_cast<long long>(b) * c_total + c) * 2 : nullptr, c, c_total);
  };
  prepare_pass(s, static_cast<long long>(b) * voxels_per_batch, voxels_per_batch, get_affine, c, silu, split, cpad,
               out, out_ld);
}

// GroupNorm affine of batch item b from producer statistics (per channel FP64
// sum and sum of squares of each source block, as the convolution epilogue
// adds them up), computed by one thread block in shared memory.  The caller
// has staged gamma / beta in aff[2c], aff[2c + 1] (before its dependency
// wait: they are weights, not the previous kernel's output); this loads the
// statistics with one coalesced sweep, sums each group in channel order on
// one thread (biased variance over the group's channels and voxels, as
// gn_finalize_kernel), and overwrites aff with (scale, offset).  Ends with a
// barrier.  sts holds 2 C doubles, gm 2 * groups doubles.
__device__ __forceinline__ void block_affine_from_stats(const double* st1, int c1, const double* st2, int c2, int b,
                                                        int groups, int voxels, float eps, float* aff, double* sts,
                                                        double* gm) {
  const int C = c1 + c2;
  const int cpg = C / groups;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const double* src = c < c1 ? st1 + (static_cast<long long>(b) * c1 + c) * 2
                               : st2 + (static_cast<long long>(b) * c2 + (c - c1)) * 2;
    const double2 v = *reinterpret_cast<const double2*>(src);
    sts[2 * c] = v.x;
    sts[2 * c + 1] = v.y;
  }
  __syncthreads();
  const double inv_n = 1.0 / (static_cast<double>(voxels) * cpg);
  for (int g = threadIdx.x; g < groups; g += blockDim.x) {
    double a = 0.0, q = 0.0;
    for (int c = g * cpg; c < (g + 1) * cpg; ++c) {
      a += sts[2 * c];
      q += sts[2 * c + 1];
    }
    const double mean = a * inv_n;
    const double var = fmax(q * inv_n - mean * mean, 0.0);
    gm[2 * g] = mean;
    gm[2 * g + 1] = 1.0 / sqrt(var + static_cast<double>(eps));
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int g = c / cpg;
    const double mean = gm[2 * g], rstd = gm[2 * g + 1];
    const float scale = static_cast<float>(static_cast<double>(aff[2 * c]) * rstd);
    const float offset = static_cast<float>(static_cast<double>(aff[2 * c + 1]) - mean * static_cast<double>(scale));
    aff[2 * c] = scale;
    aff[2 * c + 1] = offset;
  }
  __syncthreads();
}

__device__ __forceinline__ void stage_gamma_beta(const float* gamma, const float* beta, int C, float* aff) {
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    aff[2 * c] = gamma ? gamma[c] : 1.f;
    aff[2 * c + 1] = beta ? beta[c] : 0.f;
  }
}

// Shared memory of the two kernels below: aff [C][2] f32, sts [C][2] f64,
// gm [groups][2] f64.
inline size_t stats_smem_bytes(int C, int groups) {
  return static_cast<size_t>(C) * 2 * sizeof(double) + static_cast<size_t>(groups) * 2 * sizeof(double) +
         static_cast<size_t>(C) * 2 * sizeof(float);
}

// The affine alone: one block per batch item into (B, C, 2).
__global__ void gn_stats_affine_kernel(const double* st1, int c1, const double* st2, int c2, int voxels,
                                       int groups, const float* gamma, const float* beta, float eps,
                                       float* affine) {
  extern __shared__ double2 smem2[];
  const int C = c1 + c2;
  double* sts = reinterpret_cast<double*>(smem2);
  double* gm = sts + 2 * C;
  float* aff = reinterpret_cast<float*>(gm + 2 * groups);
  const int b = blockIdx.x;
  stage_gamma_beta(gamma, beta, C, aff);
  pdl_begin();
  block_affine_from_stats(st1, c1, st2, c2, b, groups, voxels, eps, aff, sts, gm);
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) affine[static_cast<long long>(b) * C * 2 + i] = aff[i];
}

// GroupNorm from producer statistics fused with the normalize pass: block
// (x, b) derives the affine of batch item b into shared memory (the same
// arithmetic as gn_stats_affine_kernel, so the same bits), then applies it
// with prepare_pass over a strided range of b's voxels.
__global__ void prepare_stats_kernel(Src2 s, int voxels, int stat_voxels, const double* st1, const double* st2,
                                     int groups, const float* gamma, const float* beta, float eps, int silu,
                                     int split, int cpad, __half* out, int out_ld) {
  extern __shared__ double2 smem2[];
  const int C = s.c1 + s.c2;
  double* sts = reinterpret_cast<double*>(smem2);
  double* gm = sts + 2 * C;
  float* aff = reinterpret_cast<float*>(gm + 2 * groups);
  const int b = blockIdx.y;
  stage_gamma_beta(gamma, beta, C, aff);
  pdl_begin();
  const int c = (threadIdx.x % (cpad / 8)) * 8;
  auto get_affine = [&] {
    block_affine_from_stats(st1, s.c1, st2, s.c2, b, groups, stat_voxels, eps, aff, sts, gm);
    return load_affine8(c < C ? aff + c * 2 : nullptr, c, C);
  };
  prepare_pass(s, static_cast<long long>(b) * voxels, voxels, get_affine, c, silu, split, cpad, out, out_ld);
}

// LayerNorm over the last axis of (rows, C) f16 (mlx_model.py:360-367):
// FP32 statistics, one rounding.  One warp per row; C <= 1024, C % 8 == 0.
template <bool F32_IN, bool SPLIT_OUT>
__global__ void layer_norm_kernel(const void* x_, int x_ld, const float* gamma, const float* beta, float eps,
                                  __half* out, int out_ld, int rows, int C, int cpad) {
  // gamma / beta are weights, not the previous kernel's output: staged in
  // shared memory before the dependency wait, off the rows' critical path.
  __shared__ __align__(16) float s_gamma[1024], s_beta[1024];
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    s_gamma[c] = gamma[c];
    s_beta[c] = beta[c];
  }
  __syncthreads();
  pdl_begin();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float v[32];
  float sum = 0.f;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = (it * 32 + lane) * 8;
    if (c < C) {
      if constexpr (F32_IN) {
        const float* xr = static_cast<const float*>(x_) + static_cast<long long>(warp) * x_ld;
        const float4 a = *reinterpret_cast<const float4*>(xr + c);
        const float4 b = *reinterpret_cast<const float4*>(xr + c + 4);
        const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[it * 8 + j] = f[j];
          sum += f[j];
        }
      } else {
        const __half* xr = static_cast<const __half*>(x_) + static_cast<long long>(warp) * x_ld;
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
        const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(h[q]);
          v[it * 8 + 2 * q] = f.x;
          v[it * 8 + 2 * q + 1] = f.y;
          sum += f.x + f.y;
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / C;
  float sq = 0.f;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = (it * 32 + lane) * 8;
    if (c < C) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[it * 8 + j] - mean;
        sq = fmaf(d, d, sq);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq / C + eps);
  __half* orow = out + static_cast<long long>(warp) * out_ld;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = (it * 32 + lane) * 8;
    if (c < (SPLIT_OUT ? cpad : C)) {
      uint4 raw, lo_raw;
      __half* h = reinterpret_cast<__half*>(&raw);
      __half* lo = reinterpret_cast<__half*>(&lo_raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float y = 0.f;
        if (c < C) y = (v[it * 8 + j] - mean) * rstd * s_gamma[c + j] + s_beta[c + j];
        h[j] = __float2half_rn(y);
        if constexpr (SPLIT_OUT) lo[j] = __float2half_rn((y - __half2float(h[j])) * 2048.0f);
      }
      *reinterpret_cast<uint4*>(orow + c) = raw;
      if constexpr (SPLIT_OUT) *reinterpret_cast<uint4*>(orow + cpad + c) = lo_raw;
    }
  }
}

int make_src(const void* x1, int c1, int ld1, const void* x2, int c2, int ld2, int dtype, Src2* s) {
  if (!x1 || c1 <= 0) return fail(LDB_ERR_INVALID, "first source must be non-null with channels > 0");
  if (c2 > 0 && !x2) return fail(LDB_ERR_INVALID, "second source is null");
  if (dtype != LDB_F16 && dtype != LDB_F32) return fail(LDB_ERR_INVALID, "dtype must be f16 or f32");
  if (c1 % 8 || c2 % 8) return fail(LDB_ERR_SHAPE, "channel blocks must be multiples of 8 (got %d, %d)", c1, c2);
  if (ld1 < c1 || ld1 % 8 || (c2 > 0 && (ld2 < c2 || ld2 % 8)))
    return fail(LDB_ERR_ALIGNMENT, "channel strides must be >= channels and multiples of 8");
  s->x1 = x1;
  s->x2 = c2 > 0 ? x2 : x1;
  s->c1 = c1;
  s->c2 = c2 > 0 ? c2 : 0;
  s->ld1 = ld1;
  s->ld2 = c2 > 0 ? ld2 : ld1;
  s->f32 = dtype == LDB_F32;
  return LDB_OK;
}

// Kernels whose shared memory grows with the channel count may need more
// than the default 48 KB (at most 4096 channels: 97 KB plus the groups).
// Threads per block of the normalize pass: whole rows of cpad / 8 channel
// groups, about 256 threads; and the blocks per batch item (about 2 blocks of
// 256 threads per SM over the batch, at most one row pass per voxel).  Two
// per SM, each thread then looping over several 4-vector batches, measured
// 1.3-2.2x faster than eight: the loop overlaps loads with the SiLU work, and
// the from-statistics pass derives its affine in a quarter as many blocks.
int prepare_threads(int cpad) {
  const int vecs = cpad / 8;
  return vecs >= 256 ? vecs : (256 / vecs) * vecs;
}

int prepare_blocks(int cpad, int voxels, int batch) {
  const int rows = prepare_threads(cpad) / (cpad / 8);
  const long long want = (static_cast<long long>(voxels) + rows - 1) / rows;
  const long long cap = std::max(1, (2 * sm_count() * 256) / (prepare_threads(cpad) * batch));
  return static_cast<int>(std::max<long long>(1, std::min(want, cap)));
}

int stats_smem_attribute(const void* kernel, size_t bytes, unsigned long long* configured) {
  if (bytes <= 48 * 1024) return LDB_OK;
  return ensure_smem_attribute(kernel, 100 * 1024, configured, "stats smem attribute");
}

int gn_chunks(int voxels, int batch) {
  // About 4 blocks per SM overall, at least 32 voxels per block.
  const int target = std::max(1, (4 * sm_count()) / std::max(1, batch));
  return std::max(1, std::min(target, (voxels + 31) / 32));
}

}  // namespace

// Fixed scratch for ldb_group_norm_affine_noalloc: the per-(batch, chunk,
// channel) partial sums live in this file-scope device array instead of a
// caller workspace.  4 MiB (524288 float2 entries); every GPU that loads the
// library holds it until the process exits.
constexpr long long kNoAllocGnEntries = 1LL << 19;
static __device__ __align__(256) float2 g_gn_noalloc_scratch[kNoAllocGnEntries];

namespace {

// Device address of the scratch array for the current device.  Host code
// cannot use the symbol itself (on the host it names a stand-in, not device
// memory), so the address is looked up once per device with that device
// current and cached.
int noalloc_scratch(float2** out) {
  static std::mutex mu;
  static std::vector<float2*> cache;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != LDB_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
  if (!cache[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_gn_noalloc_scratch), "cudaGetSymbolAddress(group-norm scratch)");
    if (rc != LDB_OK) return rc;
    cache[dev] = static_cast<float2*>(p);
  }
  *out = cache[dev];
  return LDB_OK;
}

}  // namespace
}  // namespace ldb

extern "C" {

int ldb_group_norm_workspace_size(int batch, int voxels, int channels, size_t* bytes) {
  if (!bytes) return ldb::fail(LDB_ERR_INVALID, "bytes is null");
  if (batch <= 0 || voxels <= 0 || channels <= 0) return ldb::fail(LDB_ERR_SHAPE, "extents must be positive");
  const int nchunks = ldb::gn_chunks(voxels, batch);
  *bytes = static_cast<size_t>(batch) * nchunks * channels * sizeof(float2);
  return LDB_OK;
}

int ldb_group_norm_affine(cudaStream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2, int ld2,
                          int dtype, int batch, int voxels, int groups, const float* gamma, const float* beta,
                          float eps, float* affine, void* workspace, size_t workspace_bytes) {
  using namespace ldb;
  Src2 s{};
  int rc = make_src(x1, c1, ld1, x2, c2, ld2, dtype, &s);
  if (rc != LDB_OK) return rc;
  const int C = s.c1 + s.c2;
  if (batch <= 0 || voxels <= 0) return fail(LDB_ERR_SHAPE, "batch and voxels must be positive");
  if (groups <= 0 || C % groups) return fail(LDB_ERR_SHAPE, "groups %d must divide channels %d", groups, C);
  if (C / groups > 1024) return fail(LDB_ERR_SHAPE, "at most 1024 channels per group");
  if (C > 8 * 1024) return fail(LDB_ERR_SHAPE, "at most 8192 channels");
  if (!affine) return fail(LDB_ERR_INVALID, "affine output is null");
  const int nchunks = gn_chunks(voxels, batch);
  const size_t need = static_cast<size_t>(batch) * nchunks * C * sizeof(float2);
  if (!workspace || workspace_bytes < need)
    return fail(LDB_ERR_WORKSPACE, "group norm needs %zu workspace bytes, got %zu", need, workspace_bytes);
  const int vecs = C / 8;
  int threads = 256;
  if (vecs > threads) threads = ((vecs + 31) / 32) * 32;
  threads = std::min(threads, 1024);
  if (vecs > threads) return fail(LDB_ERR_SHAPE, "too many channels for one block row");
  const int rows = threads / vecs;
  const size_t smem = static_cast<size_t>(rows) * C * 2 * sizeof(float);
  if (smem > 200 * 1024) return fail(LDB_ERR_SHAPE, "group norm reduction exceeds shared memory");
  if (smem > 48 * 1024) {
    static unsigned long long configured = 0;
    rc = ensure_smem_attribute(reinterpret_cast<const void*>(gn_partial_kernel), 200 * 1024, &configured,
                               "gn smem attribute");
    if (rc != LDB_OK) return rc;
  }
  const int chunk_voxels = (voxels + nchunks - 1) / nchunks;
  float2* partials = static_cast<float2*>(workspace);
  rc = launch_kernel(gn_partial_kernel, dim3(nchunks, batch), dim3(threads), smem, stream, "gn_partial launch", s,
                     voxels, chunk_voxels, partials, nchunks);
  if (rc != LDB_OK) return rc;
  return launch_kernel(gn_finalize_kernel, dim3(batch * groups), dim3(256), 0, stream, "gn_finalize launch", s,
                       voxels, static_cast<const float2*>(partials), nchunks, groups, gamma, beta, eps, affine);
}

int ldb_prepare_input(cudaStream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2, int ld2,
                      int dtype, int batch, int voxels, const float* affine, int silu, int split, void* out,
                      int out_ld) {
  using namespace ldb;
  Src2 s{};
  int rc = make_src(x1, c1, ld1, x2, c2, ld2, dtype, &s);
  if (rc != LDB_OK) return rc;
  if (!out) return fail(LDB_ERR_INVALID, "out is null");
  const int C = s.c1 + s.c2;
  const int cpad = split ? ((C + 15) / 16) * 16 : ((C + 7) / 8) * 8;
  if (out_ld % 8 || out_ld < (split ? 2 * cpad : cpad))
    return fail(LDB_ERR_ALIGNMENT, "out_ld %d too small or not a multiple of 8", out_ld);
  if (batch <= 0 || voxels <= 0) return fail(LDB_ERR_SHAPE, "empty input");
  if (cpad / 8 > 1024) return fail(LDB_ERR_SHAPE, "at most 8192 channels");
  return launch_kernel(prepare_kernel, dim3(static_cast<unsigned>(prepare_blocks(cpad, voxels, batch)), batch),
                       dim3(prepare_threads(cpad)), 0, stream, "prepare launch", s, voxels, affine, silu, split, cpad,
                       static_cast<__half*>(out), out_ld);
}

int ldb_group_norm_affine_from_stats(cudaStream_t stream, const double* stats1, int c1, const double* stats2,
                                     int c2, int batch, int voxels, int groups, const float* gamma,
                                     const float* beta, float eps, float* affine) {
  using namespace ldb;
  if (!stats1 || !affine || (c2 > 0 && !stats2)) return fail(LDB_ERR_INVALID, "gn affine from stats: null pointer");
  if (c1 <= 0 || c2 < 0 || batch <= 0 || voxels <= 0) return fail(LDB_ERR_SHAPE, "extents must be positive");
  const int C = c1 + c2;
  if (groups <= 0 || C % groups) return fail(LDB_ERR_SHAPE, "groups %d must divide channels %d", groups, C);
  if (C > 4096) return fail(LDB_ERR_SHAPE, "at most 4096 channels");
  const size_t smem = stats_smem_bytes(C, groups);
  static unsigned long long configured = 0;
  int rc = stats_smem_attribute(reinterpret_cast<const void*>(gn_stats_affine_kernel), smem, &configured);
  if (rc != LDB_OK) return rc;
  return launch_kernel(gn_stats_affine_kernel, dim3(batch), dim3(256), smem, stream, "gn affine from stats launch",
                       stats1, c1, c2 > 0 ? stats2 : stats1, c2, voxels, groups, gamma, beta, eps, affine);
}

int ldb_prepare_input_from_stats(cudaStream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2,
                                 int ld2, int dtype, int batch, int voxels, int stat_voxels, const double* stats1,
                                 const double* stats2, int groups, const float* gamma, const float* beta, float eps,
                                 int silu, int split, void* out, int out_ld) {
  using namespace ldb;
  Src2 s{};
  int rc = make_src(x1, c1, ld1, x2, c2, ld2, dtype, &s);
  if (rc != LDB_OK) return rc;
  if (!out || !stats1 || (s.c2 > 0 && !stats2)) return fail(LDB_ERR_INVALID, "prepare from stats: null pointer");
  if (batch <= 0 || voxels <= 0 || stat_voxels < 0) return fail(LDB_ERR_SHAPE, "extents must be positive");
  if (stat_voxels == 0) stat_voxels = voxels;
  const int C = s.c1 + s.c2;
  if (groups <= 0 || C % groups) return fail(LDB_ERR_SHAPE, "groups %d must divide channels %d", groups, C);
  if (C > 4096) return fail(LDB_ERR_SHAPE, "at most 4096 channels");
  const int cpad = split ? ((C + 15) / 16) * 16 : ((C + 7) / 8) * 8;
  if (out_ld % 8 || out_ld < (split ? 2 * cpad : cpad))
    return fail(LDB_ERR_ALIGNMENT, "out_ld %d too small or not a multiple of 8", out_ld);
  const size_t smem = stats_smem_bytes(C, groups);
  static unsigned long long configured = 0;
  rc = stats_smem_attribute(reinterpret_cast<const void*>(prepare_stats_kernel), smem, &configured);
  if (rc != LDB_OK) return rc;
  return launch_kernel(prepare_stats_kernel, dim3(static_cast<unsigned>(prepare_blocks(cpad, voxels, batch)), batch),
                       dim3(prepare_threads(cpad)), smem,
                       stream, "prepare from stats launch", s, voxels, stat_voxels, stats1, s.c2 > 0 ? stats2 : stats1, groups,
                       gamma, beta, eps, silu, split, cpad, static_cast<__half*>(out), out_ld);
}

int ldb_layer_norm_ex(cudaStream_t stream, const void* x, int x_dtype, int x_ld, const float* gamma,
                      const float* beta, float eps, void* out, int out_ld, int rows, int channels, int split) {
  using namespace ldb;
  if (!x || !out || !gamma || !beta) return fail(LDB_ERR_INVALID, "layer_norm: null pointer");
  if (x_dtype != LDB_F16 && x_dtype != LDB_F32) return fail(LDB_ERR_INVALID, "layer_norm input must be f16 or f32");
  if (channels <= 0 || channels > 1024 || channels % 8) return fail(LDB_ERR_SHAPE, "channels must be 8..1024, %% 8");
  const int cpad = split ? (channels + 15) / 16 * 16 : channels;
  if (x_ld % 8 || out_ld % 8) return fail(LDB_ERR_ALIGNMENT, "row strides must be multiples of 8");
  if (x_ld < channels) return fail(LDB_ERR_SHAPE, "layer_norm: x_ld %d < %d channels", x_ld, channels);
  if (out_ld < (split ? 2 * cpad : channels)) return fail(LDB_ERR_SHAPE, "out_ld too small");
  if (rows <= 0) return fail(LDB_ERR_SHAPE, "rows must be positive");
  const int threads = 256;
  const long long blocks = (static_cast<long long>(rows) * 32 + threads - 1) / threads;
  auto kernel = x_dtype == LDB_F32 ? (split ? layer_norm_kernel<true, true> : layer_norm_kernel<true, false>)
                                   : (split ? layer_norm_kernel<false, true> : layer_norm_kernel<false, false>);
  return launch_kernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, stream, "layer_norm launch", x,
                       x_ld, gamma, beta, eps, static_cast<__half*>(out), out_ld, rows, channels, cpad);
}

int ldb_layer_norm(cudaStream_t stream, const void* x, int x_ld, const float* gamma, const float* beta, float eps,
                   void* out, int out_ld, int rows, int channels) {
  return ldb_layer_norm_ex(stream, x, LDB_F16, x_ld, gamma, beta, eps, out, out_ld, rows, channels, 0);
}

// GroupNorm affine without any allocation: the same statistics as
// ldb_group_norm_affine, with the partial sums kept in the library's fixed
// device scratch (g_gn_noalloc_scratch) instead of a caller workspace.  For
// callers that cannot allocate device memory at call time.  The first call
// on a device looks up the scratch address (make it before any stream
// capture).  With lazy module loading (the CUDA 12 default) that lookup, or
// the first launch of any kernel of this file, is also when the driver loads
// this file's module and places the 4 MiB array in device memory: make the
// first call before the caller reserves all of the device's memory, or run
// the process with CUDA_MODULE_LOADING=EAGER.  Calls share the scratch, so calls that overlap on the GPU
// (different streams, or different host threads) race; each call fully
// writes every partial it reads, so nothing needs clearing between calls.
int ldb_group_norm_affine_noalloc(cudaStream_t stream, const void* x1, int c1, int ld1, const void* x2, int c2,
                                  int ld2, int dtype, int batch, int voxels, int groups, const float* gamma,
                                  const float* beta, float eps, float* affine) {
  using namespace ldb;
  Src2 s{};
  int rc = make_src(x1, c1, ld1, x2, c2, ld2, dtype, &s);
  if (rc != LDB_OK) return rc;
  const int C = s.c1 + s.c2;
  if (batch <= 0 || voxels <= 0) return fail(LDB_ERR_SHAPE, "batch and voxels must be positive");
  if (groups <= 0 || C % groups) return fail(LDB_ERR_SHAPE, "groups %d must divide channels %d", groups, C);
  if (C / groups > 1024) return fail(LDB_ERR_SHAPE, "at most 1024 channels per group");
  if (C > 8 * 1024) return fail(LDB_ERR_SHAPE, "at most 8192 channels");
  if (!affine) return fail(LDB_ERR_INVALID, "affine output is null");
  const long long per_chunk = static_cast<long long>(batch) * C;
  if (per_chunk > kNoAllocGnEntries)
    return fail(LDB_ERR_SHAPE,
                "group_norm_affine_noalloc: batch * channels = %lld exceeds the fixed scratch of %lld entries",
                per_chunk, kNoAllocGnEntries);
  const int nchunks = static_cast<int>(std::min<long long>(gn_chunks(voxels, batch), kNoAllocGnEntries / per_chunk));
  float2* partials = nullptr;
  rc = noalloc_scratch(&partials);
  if (rc != LDB_OK) return rc;
  const int vecs = C / 8;
  int threads = 256;
  if (vecs > threads) threads = ((vecs + 31) / 32) * 32;
  threads = std::min(threads, 1024);
  if (vecs > threads) return fail(LDB_ERR_SHAPE, "too many channels for one block row");
  const int rows = threads / vecs;
  const size_t smem = static_cast<size_t>(rows) * C * 2 * sizeof(float);
  if (smem > 200 * 1024) return fail(LDB_ERR_SHAPE, "group norm reduction exceeds shared memory");
  if (smem > 48 * 1024) {
    static unsigned long long configured = 0;
    rc = ensure_smem_attribute(reinterpret_cast<const void*>(gn_partial_kernel), 200 * 1024, &configured,
                               "gn smem attribute");
    if (rc != LDB_OK) return rc;
  }
  const int chunk_voxels = (voxels + nchunks - 1) / nchunks;
  rc = launch_kernel(gn_partial_kernel, dim3(nchunks, batch), dim3(threads), smem, stream,
                     "gn_partial (noalloc) launch", s, voxels, chunk_voxels, partials, nchunks);
  if (rc != LDB_OK) return rc;
  return launch_kernel(gn_finalize_kernel, dim3(batch * groups), dim3(256), 0, stream, "gn_finalize (noalloc) launch",
                       s, voxels, static_cast<const float2*>(partials), nchunks, groups, gamma, beta, eps, affine);
}

}  // extern "C"
