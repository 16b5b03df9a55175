// Output-region compositing of a generated CT into the input CT (the
// reference's localize_output and apply_lesion_change,
// lesiondiffusion_mlx/medmlx.py:2531-2690).  Volumes are dense float32
// (n0, n1, n2) arrays in the reference's axis order; every kernel is
// HBM-bound (one read of each input volume, one write of the output).
//
// Box mode: inside the box the generated CT; within margin_mm of the box
// (Euclidean distance between voxel centres in mm, per-axis offsets times the
// spacing) the blend w * generated + (1 - w) * original with
// w = 0.5 (1 + cos(pi d / margin)), evaluated in FP64 in the reference's
// operation order and rounded once to f32; elsewhere the original.
//
// Lesion mode: `reached` = voxels within `reach` voxels of a lesion voxel
// along every axis (a cubic dilation, done as three separable line passes);
// out = original + (generated - reconstruction) there, original elsewhere,
// in f32 as the reference; plus the mean of reconstruction - original over
// the reached non-lesion voxels whose |original| < 1000 HU.

#include <algorithm>
#include <climits>
#include <cmath>

#include "common.cuh"
#include "host_common.h"

namespace ldb {
namespace {

struct BoxGeom {
  int n[3];
  int start[3], stop[3];  // the box [start, stop)
  int low[3], high[3];    // the feathered region [low, high)
  double spacing[3];
  double margin;
};

__global__ void localize_box_kernel(const float* original, const float* generated, float* out, BoxGeom g,
                                    unsigned long long* weighted) {
  pdl_begin();
  const long long total = static_cast<long long>(g.n[0]) * g.n[1] * g.n[2];
  unsigned int affected = 0;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c2 = static_cast<int>(i % g.n[2]);
    const int c1 = static_cast<int>((i / g.n[2]) % g.n[1]);
    const int c0 = static_cast<int>(i / (static_cast<long long>(g.n[2]) * g.n[1]));
    const int c[3] = {c0, c1, c2};
    const float orig = original[i];
    float r = orig;
    bool inside = true, in_region = true;
    double squared = 0.0;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      int off = 0;
      if (c[a] < g.start[a]) off = g.start[a] - c[a];
      if (c[a] >= g.stop[a]) off = c[a] - (g.stop[a] - 1);
      inside = inside && off == 0;
      in_region = in_region && c[a] >= g.low[a] && c[a] < g.high[a];
      const double o = __dmul_rn(static_cast<double>(off), g.spacing[a]);
      squared = __dadd_rn(squared, __dmul_rn(o, o));
    }
    if (inside) {
      r = generated[i];
    } else if (in_region) {
      const double d = __dsqrt_rn(squared);
      if (d < g.margin) {
        affected += 1;
        const double w = __dmul_rn(0.5, __dadd_rn(1.0, cos(__ddiv_rn(__dmul_rn(M_PI, d), g.margin))));
        if (w > 0.0 && w < 1.0) {
          const double blend = __dadd_rn(__dmul_rn(static_cast<double>(generated[i]), w),
                                         __dmul_rn(static_cast<double>(orig), __dsub_rn(1.0, w)));
          r = static_cast<float>(blend);
        }
      }
    }
    if (inside && in_region) affected += 1;  // distance 0 < margin
    out[i] = r;
  }
  if (weighted) {
    for (int o = 16; o > 0; o >>= 1) affected += __shfl_xor_sync(0xffffffffu, affected, o);
    if ((threadIdx.x & 31) == 0 && affected) atomicAdd(weighted, static_cast<unsigned long long>(affected));
  }
}

__global__ void extent_init_kernel(int* extent) {
  pdl_begin();
  if (threadIdx.x < 7) extent[threadIdx.x] = threadIdx.x == 0 ? 0 : (threadIdx.x < 4 ? INT_MAX : -1);
}

// Lesion extent: extent[0] = voxel count, [1..3] = min index per axis,
// [4..6] = max index per axis (initialised to 0, INT_MAX, -1).
__global__ void lesion_extent_kernel(const uint8_t* lesion, int n0, int n1, int n2, int* extent) {
  pdl_begin();
  const long long total = static_cast<long long>(n0) * n1 * n2;
  int cnt = 0, lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (!lesion[i]) continue;
    const int c[3] = {static_cast<int>(i / (static_cast<long long>(n2) * n1)), static_cast<int>((i / n2) % n1),
                      static_cast<int>(i % n2)};
    cnt += 1;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      lo[a] = min(lo[a], c[a]);
      hi[a] = max(hi[a], c[a]);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      lo[a] = min(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
      hi[a] = max(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
    }
  }
  if ((threadIdx.x & 31) == 0 && cnt) {
    atomicAdd(&extent[0], cnt);
    for (int a = 0; a < 3; ++a) {
      atomicMin(&extent[1 + a], lo[a]);
      atomicMax(&extent[4 + a], hi[a]);
    }
  }
}

// One pass of the cubic dilation: out[line] = 1 where an input voxel of the
// same line along `axis` lies within `reach` (a forward and a backward sweep
// tracking the last set index).  One thread per line; adjacent threads take
// adjacent lines along the fastest other axis, so their accesses coalesce
// for axes 0 and 1.
__global__ void dilate_line_kernel(const uint8_t* in, uint8_t* out, int n0, int n1, int n2, int axis, int reach) {
  pdl_begin();
  const int n[3] = {n0, n1, n2};
  const long long stride[3] = {static_cast<long long>(n1) * n2, n2, 1};
  const int len = n[axis];
  const int a1 = axis == 2 ? 1 : 2;        // fastest other axis
  const int a0 = axis == 0 ? 1 : 0;        // remaining axis
  const long long lines = static_cast<long long>(n[a0]) * n[a1];
  const long long line = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (line >= lines) return;
  const int i1 = static_cast<int>(line % n[a1]);
  const int i0 = static_cast<int>(line / n[a1]);
  const long long base = i0 * stride[a0] + i1 * stride[a1];
  const long long step = stride[axis];
  int last = -2 * reach - 2;  // no set voxel seen yet
  for (int k = 0; k < len; ++k) {
    if (in[base + k * step]) last = k;
    out[base + k * step] = (k - last <= reach) ? 1 : 0;
  }
  last = len + 2 * reach + 2;
  for (int k = len - 1; k >= 0; --k) {
    if (in[base + k * step]) last = k;
    if (last - k <= reach) out[base + k * step] = 1;
  }
}

// out = reached ? original + (generated - reconstruction) : original (f32),
// and the reconstruction offset over the surroundings (reached, not lesion,
// |original| < 1000): stats[0] += sum (FP64), stats[1] += count, stats[2] +=
// reached count.
__global__ void lesion_change_kernel(const float* original, const float* generated, const float* reconstruction,
                                     const uint8_t* lesion, const uint8_t* reached, float* out, long long total,
                                     double* stats) {
  pdl_begin();
  double sum = 0.0, cnt = 0.0, nreach = 0.0;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float orig = original[i];
    float r = orig;
    if (reached[i]) {
      const float rec = reconstruction[i];
      r = __fadd_rn(orig, __fsub_rn(generated[i], rec));
      nreach += 1.0;
      if (!lesion[i] && fabsf(orig) < 1000.0f) {
        sum += static_cast<double>(rec) - static_cast<double>(orig);
        cnt += 1.0;
      }
    }
    out[i] = r;
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    nreach += __shfl_xor_sync(0xffffffffu, nreach, o);
  }
  if ((threadIdx.x & 31) == 0 && nreach > 0.0) {
    atomicAdd(&stats[0], sum);
    atomicAdd(&stats[1], cnt);
    atomicAdd(&stats[2], nreach);
  }
}

int grid_for(long long total, int threads) {
  const long long want = (total + threads - 1) / threads;
  return static_cast<int>(std::max(1LL, std::min(want, static_cast<long long>(sm_count()) * 8)));
}

}  // namespace
}  // namespace ldb

extern "C" {

int ldb_localize_box(cudaStream_t stream, const float* original, const float* generated, float* out, int n0, int n1,
                     int n2, const int* start, const int* stop, const double* spacing_mm, double margin_mm,
                     unsigned long long* weighted_count) {
  using namespace ldb;
  if (!original || !generated || !out || !start || !stop || !spacing_mm)
    return fail(LDB_ERR_INVALID, "localize_box: null pointer");
  if (n0 <= 0 || n1 <= 0 || n2 <= 0) return fail(LDB_ERR_SHAPE, "localize_box: extents must be positive");
  if (!(margin_mm > 0.0)) return fail(LDB_ERR_INVALID, "localize_box: margin must be positive");
  BoxGeom g;
  const int n[3] = {n0, n1, n2};
  for (int a = 0; a < 3; ++a) {
    if (!(spacing_mm[a] > 0.0)) return fail(LDB_ERR_INVALID, "localize_box: spacing must be positive");
    if (start[a] < 0 || stop[a] > n[a] || start[a] >= stop[a])
      return fail(LDB_ERR_SHAPE, "localize_box: box [%d, %d) outside axis %d of %d", start[a], stop[a], a, n[a]);
    g.n[a] = n[a];
    g.start[a] = start[a];
    g.stop[a] = stop[a];
    g.spacing[a] = spacing_mm[a];
    // radius = ceil(margin / spacing) voxels (the reference's affected region)
    const int radius = static_cast<int>(std::ceil(margin_mm / spacing_mm[a]));
    g.low[a] = std::max(0, start[a] - radius);
    g.high[a] = std::min(n[a], stop[a] + radius);
  }
  g.margin = margin_mm;
  const long long total = static_cast<long long>(n0) * n1 * n2;
  const int threads = 256;
  return launch_kernel(localize_box_kernel, dim3(grid_for(total, threads)), dim3(threads), 0, stream,
                       "localize_box launch", original, generated, out, g, weighted_count);
}

int ldb_lesion_extent(cudaStream_t stream, const uint8_t* lesion, int n0, int n1, int n2, int* extent) {
  using namespace ldb;
  if (!lesion || !extent) return fail(LDB_ERR_INVALID, "lesion_extent: null pointer");
  if (n0 <= 0 || n1 <= 0 || n2 <= 0) return fail(LDB_ERR_SHAPE, "lesion_extent: extents must be positive");
  int rc = launch_kernel(extent_init_kernel, dim3(1), dim3(32), 0, stream, "lesion_extent init", extent);
  if (rc != LDB_OK) return rc;
  const long long total = static_cast<long long>(n0) * n1 * n2;
  const int threads = 256;
  return launch_kernel(lesion_extent_kernel, dim3(grid_for(total, threads)), dim3(threads), 0, stream,
                       "lesion_extent launch", lesion, n0, n1, n2, extent);
}

int ldb_apply_lesion_change(cudaStream_t stream, const float* original, const float* generated,
                            const float* reconstruction, const uint8_t* lesion, float* out, int n0, int n1, int n2,
                            int reach, uint8_t* workspace, size_t workspace_bytes, double* stats) {
  using namespace ldb;
  if (!original || !generated || !reconstruction || !lesion || !out || !stats)
    return fail(LDB_ERR_INVALID, "apply_lesion_change: null pointer");
  if (n0 <= 0 || n1 <= 0 || n2 <= 0) return fail(LDB_ERR_SHAPE, "apply_lesion_change: extents must be positive");
  if (reach < 0) return fail(LDB_ERR_INVALID, "apply_lesion_change: reach must be >= 0");
  // A reach of the longest axis already covers every line: larger ones dilate
  // the same and would only overflow the sweeps' sentinel arithmetic.
  reach = std::min(reach, std::max(n0, std::max(n1, n2)));
  const long long total = static_cast<long long>(n0) * n1 * n2;
  if (!workspace || workspace_bytes < static_cast<size_t>(2 * total))
    return fail(LDB_ERR_WORKSPACE, "apply_lesion_change needs %lld workspace bytes", 2 * total);
  uint8_t* t0 = workspace;
  uint8_t* t1 = workspace + total;
  int rc = check_cuda(cudaMemsetAsync(stats, 0, 3 * sizeof(double), stream), "lesion stats init");
  if (rc != LDB_OK) return rc;
  const int threads = 256;
  const int n[3] = {n0, n1, n2};
  const uint8_t* src = lesion;
  uint8_t* dst[3] = {t0, t1, t0};
  const int axes[3] = {2, 1, 0};
  for (int p = 0; p < 3; ++p) {
    const int axis = axes[p];
    const long long lines = total / n[axis];
    rc = launch_kernel(dilate_line_kernel, dim3(static_cast<unsigned>((lines + threads - 1) / threads)),
                       dim3(threads), 0, stream, "dilate launch", src, dst[p], n0, n1, n2, axis, reach);
    if (rc != LDB_OK) return rc;
    src = dst[p];
  }
  return launch_kernel(lesion_change_kernel, dim3(grid_for(total, threads)), dim3(threads), 0, stream,
                       "lesion_change launch", original, generated, reconstruction, lesion,
                       static_cast<const uint8_t*>(t0), out, total, stats);
}

}  // extern "C"
