// Small and memory-bound kernels of the denoise loop and the decoder:
// timestep embedding, skinny dense layers (the time-embedding MLP and the
// per-block embedding projections), the fused DDIM and DPM++-2M updates with
// mask composition and the next network-input write, the 4-channel VQ
// nearest-code search with the straight-through quantize, nearest resizes
// and the inverse CT intensity map.

#include <algorithm>

#include "common.cuh"
#include "host_common.h"

namespace ldb {
namespace {

// [cos, sin] sinusoidal embedding (mlx_model.py:609-612): with h = C/2,
// freq_i = exp(-ln(1e4) * i / h) and phase = t * freq_i, all in FP32 and in
// the reference's operation order; out is f16 or f32 (B, C).
__global__ void timestep_embedding_kernel(const int* table, const int* step, int steps, int batch, int channels,
                                          void* out, int out_f32, unsigned int* status) {
  pdl_begin();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int half = channels / 2;
  if (idx >= batch * half) return;
  const int row = step ? *step : 0;
  if (row < 0 || row >= steps) {  // a counter past the table: write nothing, report it
    if (idx == 0) set_bad_shape(status);
    return;
  }
  const int b = idx / half;
  const int i = idx % half;
  const int* t = table + static_cast<long long>(row) * batch;
  const float scaled = __fmul_rn(-9.21034037197618273607f, static_cast<float>(i));
  // Correctly rounded exp of the FP32 argument: the phase t * freq scales
  // any ulp of freq by t (up to 1000), so freq must not carry expf's error.
  const float freq = static_cast<float>(exp(static_cast<double>(__fdiv_rn(scaled, static_cast<float>(half)))));
  const float phase = __fmul_rn(static_cast<float>(t[b]), freq);
  const float c = cosf(phase);
  const float s = sinf(phase);
  if (out_f32) {
    float* o = static_cast<float*>(out) + static_cast<long long>(b) * channels;
    o[i] = c;
    o[half + i] = s;
  } else {
    __half* o = static_cast<__half*>(out) + static_cast<long long>(b) * channels;
    o[i] = __float2half_rn(c);
    o[half + i] = __float2half_rn(s);
  }
}

// out[m][n] = act_out(sum_k act_in(x[m][k]) * w[n][k] + bias[n]) for a few
// rows m (the batch).  One warp per output column n; lanes stride over K
// with 16-byte loads.  act_in = SiLU rounds to f16 first (the UNet's SiLU,
// mlx_model.py:409-413); the f16 store rounds once; `round_f16` makes an f32
// store carry the f16-rounded value (a per-batch conv shift).
constexpr int kDenseMaxRows = 16;

__global__ void dense_small_kernel(const __half* x, int x_ld, const __half* w, const float* bias, void* out,
                                   int out_ld, int rows, int n_out, int k, int in_silu, int out_silu, int out_f32,
                                   int round_f16) {
  pdl_begin();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_out) return;
  const __half* wr = w + static_cast<long long>(warp) * k;
  float acc[kDenseMaxRows];
#pragma unroll
  for (int m = 0; m < kDenseMaxRows; ++m) acc[m] = 0.f;
  for (int c = lane * 8; c < k; c += 32 * 8) {
    const uint4 wraw = *reinterpret_cast<const uint4*>(wr + c);
    const __half2* wh = reinterpret_cast<const __half2*>(&wraw);
    float wf[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(wh[q]);
      wf[2 * q] = f.x;
      wf[2 * q + 1] = f.y;
    }
#pragma unroll
    for (int m = 0; m < kDenseMaxRows; ++m) {
      if (m < rows) {
        const uint4 xraw = *reinterpret_cast<const uint4*>(x + static_cast<long long>(m) * x_ld + c);
        const __half2* xh = reinterpret_cast<const __half2*>(&xraw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 f = __half22float2(xh[q]);
          if (in_silu) {
            f.x = __half2float(__float2half_rn(silu_f32(f.x)));
            f.y = __half2float(__float2half_rn(silu_f32(f.y)));
          }
          acc[m] = fmaf(f.x, wf[2 * q], acc[m]);
          acc[m] = fmaf(f.y, wf[2 * q + 1], acc[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kDenseMaxRows; ++m) {
    if (m < rows) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
  }
  if (lane == 0) {
    const float b = bias ? bias[warp] : 0.f;
    for (int m = 0; m < rows; ++m) {
      float y = acc[m] + b;
      if (out_silu) y = silu_f32(__half2float(__float2half_rn(y)));
      if (out_f32) {
        if (round_f16) y = __half2float(__float2half_rn(y));
        static_cast<float*>(out)[static_cast<long long>(m) * out_ld + warp] = y;
      } else {
        static_cast<__half*>(out)[static_cast<long long>(m) * out_ld + warp] = __float2half_rn(y);
      }
    }
  }
}

// Fused sampler step over (B, V) voxels with C state channels (NDHWC):
//   kind 0 (compose only): x <- x*m + (1-m)*image
//   kind 1 (DDIM, mlx_sampling.py:128-132):
//       pred = (x - s1m*eps) / sqrt(a); dir = sqrt(1 - p - sigma^2) * eps
//       x <- sqrt(p)*pred + dir + sigma*noise, then compose
//   kind 2 (DPM++-2M, _dpm.py:129-133): pred = (x - c1*eps)/c0;
//       x <- c2*x + c3*pred + c4*(pred - prev); prev <- pred; then compose
// With a mask, composition re-imposes the known region (x*m + (1-m)*image,
// mlx_sampling.py:119, :134-135); the next network input
// [x | extra] is written as f16 with channel stride in_ld (zero padded),
// where `extra` is the mask (inpainting) or the conditioning image; for the
// FP32 network (net_cpad > 0) it is written as the f16 hi plane in channels
// [0, net_cpad) and the 2^11-scaled low plane in [net_cpad, 2 net_cpad).
// eps is the network's f16 or f32 prediction.
struct StepArgs {
  const float* coeff;  // [steps][5] f32 coefficient table (device)
  const int* step;     // current step index (device), or null for step 0
  int steps;           // rows of the step tables: a step outside [0, steps) touches nothing
  unsigned int* status;
  long long noise_step_stride;  // elements between the noise of consecutive steps
  float* x;            // (B, V, C) f32 state, updated in place
  float* prev;         // (B, V, C) f32 DPM history
  const void* eps;     // (B, V, eps_ld) f16 or f32 prediction (first C channels used)
  int eps_ld;
  int eps_f32;
  const float* noise;  // (B, V, C) f32
  const float* mask;   // (B, V) f32 or null
  const float* image;  // (B, V, C) f32 known-region latent, or the concatenated image (B, V, extra_c)
  int image_c;         // channels of `image`
  __half* net_in;      // (B, V, in_ld) f16 or null
  int in_ld;
  int net_cpad;        // > 0: split FP32 input planes of net_cpad channels each
  long long voxels;    // B * V
  int channels;
  int kind;
};

__device__ __forceinline__ void put_net_in(const StepArgs& a, long long v, int c, float x) {
  const __half hi = __float2half_rn(x);
  a.net_in[v * a.in_ld + c] = hi;
  if (a.net_cpad > 0) a.net_in[v * a.in_ld + a.net_cpad + c] = __float2half_rn((x - __half2float(hi)) * 2048.0f);
}

__device__ __forceinline__ float load_eps(const StepArgs& a, long long v, int c) {
  return a.eps_f32 ? static_cast<const float*>(a.eps)[v * a.eps_ld + c]
                   : __half2float(static_cast<const __half*>(a.eps)[v * a.eps_ld + c]);
}

__global__ void sampler_step_kernel(StepArgs a) {
  pdl_begin();
  const long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (v >= a.voxels) return;
  const int C = a.channels;
  const int step = a.step ? *a.step : 0;
  if (step < 0 || step >= a.steps) {  // a counter past the tables: write nothing, report it
    if (v == 0) set_bad_shape(a.status);
    return;
  }
  const float m = a.mask ? a.mask[v] : 1.f;
  float k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f, k4 = 0.f;
  if (a.kind != 0) {
    const float* k = a.coeff + 5LL * step;
    k0 = k[0];
    k1 = k[1];
    k2 = k[2];
    k3 = k[3];
    k4 = k[4];
  }
  const float* noise = a.noise ? a.noise + step * a.noise_step_stride : nullptr;
  for (int c = 0; c < C; ++c) {
    const long long i = v * C + c;
    float x = a.x[i];
    if (a.kind == 1) {
      const float e = load_eps(a, v, c);
      // k0 = alpha, k1 = previous, k2 = sigma, k3 = sqrt(1 - alpha)
      const float pred = __fdiv_rn(__fsub_rn(x, __fmul_rn(k3, e)), sqrtf(k0));
      const float dir = __fmul_rn(sqrtf(__fsub_rn(__fsub_rn(1.f, k1), __fmul_rn(k2, k2))), e);
      x = __fadd_rn(__fadd_rn(__fmul_rn(sqrtf(k1), pred), dir), __fmul_rn(k2, noise[i]));
    } else if (a.kind == 2) {
      const float e = load_eps(a, v, c);
      // (alpha, sigma, ratio, clean, history)
      const float pred = __fdiv_rn(__fsub_rn(x, __fmul_rn(k1, e)), k0);
      x = __fadd_rn(__fadd_rn(__fmul_rn(k2, x), __fmul_rn(k3, pred)), __fmul_rn(k4, __fsub_rn(pred, a.prev[i])));
      a.prev[i] = pred;
    }
    if (a.mask) x = __fadd_rn(__fmul_rn(x, m), __fmul_rn(__fsub_rn(1.f, m), a.image[i]));
    a.x[i] = x;
    if (a.net_in) put_net_in(a, v, c, x);
  }
  if (a.net_in) {
    int c = C;
    if (a.mask) {
      put_net_in(a, v, c++, m);
    } else {
      for (int j = 0; j < a.image_c; ++j) put_net_in(a, v, c++, a.image[v * a.image_c + j]);
    }
    for (; c < (a.net_cpad > 0 ? a.net_cpad : a.in_ld); ++c) put_net_in(a, v, c, 0.f);
  }
}

// ---------------------------------------------------------------- VQ search

template <typename T>
struct VqT;
template <>
struct VqT<float> {
  __device__ static float load(const float* p) { return *p; }
  __device__ static float round(float v) { return v; }
  __device__ static void store(float* p, float v) { *p = v; }
};
template <>
struct VqT<__half> {
  __device__ static float load(const __half* p) { return __half2float(*p); }
  __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
  __device__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
};

// Rounded squares summed in FP32 and cast to T (mlx_model.py:763-767, _vq.py:73).
template <typename T>
__device__ __forceinline__ float vq_norm(float a, float b, float c, float d) {
  const float sa = VqT<T>::round(__fmul_rn(a, a));
  const float sb = VqT<T>::round(__fmul_rn(b, b));
  const float sc = VqT<T>::round(__fmul_rn(c, c));
  const float sd = VqT<T>::round(__fmul_rn(d, d));
  return VqT<T>::round(__fadd_rn(__fadd_rn(__fadd_rn(sa, sb), sc), sd));
}

// One thread per latent position.  The codebook (E x 4) and its norms are
// staged in shared memory in tiles.  Distance, tie and NaN rules follow
// _vq.py:20-47: FMA-chained FP32 dot, T(T(|z|^2 + |e|^2) - T(2 T(dot))),
// smallest index on equal distances, NaN first-index priority.  Optionally
// writes the straight-through value z + (e - z) in T (mlx_model.py:780-781)
// to an NDHWC output with channel stride out_ld.
template <typename T>
__global__ void vq_nearest4_kernel(const T* z, int z_ld, long long positions, const T* codebook, int entries,
                                   int* indices, T* quantized, int out_ld) {
  pdl_begin();
  constexpr int kTile = 1024;
  __shared__ float4 cb[kTile];
  __shared__ float cbn[kTile];
  const long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool valid = p < positions;
  float z0 = 0.f, z1 = 0.f, z2 = 0.f, z3 = 0.f;
  if (valid) {
    const T* zp = z + p * z_ld;
    z0 = VqT<T>::load(zp);
    z1 = VqT<T>::load(zp + 1);
    z2 = VqT<T>::load(zp + 2);
    z3 = VqT<T>::load(zp + 3);
  }
  const float zn = vq_norm<T>(z0, z1, z2, z3);
  float best = __int_as_float(0x7f800000);  // +inf
  int best_index = -1;
  for (int base = 0; base < entries; base += kTile) {
    const int n = min(kTile, entries - base);
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += blockDim.x) {
      const T* cp = codebook + static_cast<long long>(base + e) * 4;
      const float c0 = VqT<T>::load(cp), c1 = VqT<T>::load(cp + 1), c2 = VqT<T>::load(cp + 2),
                  c3 = VqT<T>::load(cp + 3);
      cb[e] = make_float4(c0, c1, c2, c3);
      cbn[e] = vq_norm<T>(c0, c1, c2, c3);
    }
    __syncthreads();
    if (valid) {
      for (int e = 0; e < n; ++e) {
        const float4 c = cb[e];
        float dot = __fmul_rn(z0, c.x);
        dot = __fmaf_rn(z1, c.y, dot);
        dot = __fmaf_rn(z2, c.z, dot);
        dot = __fmaf_rn(z3, c.w, dot);
        const float summed = VqT<T>::round(__fadd_rn(zn, cbn[e]));
        const float doubled = VqT<T>::round(__fmul_rn(2.f, VqT<T>::round(dot)));
        const float dist = VqT<T>::round(__fsub_rn(summed, doubled));
        const int code = base + e;
        const bool dnan = isnan(dist), bnan = isnan(best);
        const bool take = best_index < 0 || (dnan && !bnan) || (!bnan && !dnan && dist < best);
        if (take) {
          best = dist;
          best_index = code;
        }
      }
    }
  }
  if (!valid) return;
  indices[p] = best_index;
  if (quantized) {
    const T* cp = codebook + static_cast<long long>(best_index) * 4;
    const float zz[4] = {z0, z1, z2, z3};
    T* q = quantized + p * out_ld;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float e = VqT<T>::load(cp + j);
      VqT<T>::store(q + j, VqT<T>::round(__fadd_rn(zz[j], VqT<T>::round(__fsub_rn(e, zz[j])))));
    }
  }
}

// Nearest resize of an NDHWC tensor with source index floor(i * in / out)
// per axis (_spatial.py:41-69); a 2x resize is the upsample_nearest2 copy.
// One thread per (output voxel, 8-byte channel group).
__global__ void resize_nearest_kernel(const uint8_t* x, int in_d, int in_h, int in_w, uint8_t* out, int od, int oh,
                                      int ow, int batch, int row_bytes, int x_row_stride, int out_row_stride,
                                      float rd, float rh, float rw) {
  pdl_begin();
  const int groups = row_bytes / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(batch) * od * oh * ow * groups;
  if (idx >= total) return;
  const int g = static_cast<int>(idx % groups);
  long long v = idx / groups;
  const int w = static_cast<int>(v % ow);
  v /= ow;
  const int h = static_cast<int>(v % oh);
  v /= oh;
  const int d = static_cast<int>(v % od);
  const int b = static_cast<int>(v / od);
  // floor(f32(i) * f32(in / out)): the reference multiplies an integer
  // range by the Python-float ratio in FP32 (_spatial.py:67-69), which can
  // differ from the exact integer quotient for ratios like 5/3.
  const int sd = min(in_d - 1, static_cast<int>(floorf(__fmul_rn(static_cast<float>(d), rd))));
  const int sh = min(in_h - 1, static_cast<int>(floorf(__fmul_rn(static_cast<float>(h), rh))));
  const int sw = min(in_w - 1, static_cast<int>(floorf(__fmul_rn(static_cast<float>(w), rw))));
  const long long src = ((static_cast<long long>(b) * in_d + sd) * in_h + sh) * in_w + sw;
  const long long dst = ((static_cast<long long>(b) * od + d) * oh + h) * ow + w;
  *reinterpret_cast<uint2*>(out + dst * out_row_stride + g * 8) =
      *reinterpret_cast<const uint2*>(x + src * x_row_stride + g * 8);
}

// Normalized -> HU with knots (0, .2, .8, 1) -> (-1000, -200, 200, 1000) and
// clipping (mlx_pipeline.py:72-96, inverse=True); input f16 or f32 with a
// channel stride (channel 0 is mapped), output dense f32.
__global__ void hu_map_kernel(const void* x, int x_f32, int x_ld, long long n, float* out) {
  pdl_begin();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float a = x_f32 ? static_cast<const float*>(x)[i * x_ld] : __half2float(static_cast<const __half*>(x)[i * x_ld]);
  const float kin[4] = {0.0f, 0.2f, 0.8f, 1.0f};
  const float kout[4] = {-1000.0f, -200.0f, 200.0f, 1000.0f};
  float r = kout[0];
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const float slope = static_cast<float>((static_cast<double>(kout[s + 1]) - kout[s]) /
                                           (static_cast<double>(kin[s + 1]) - kin[s]));
    if (a >= kin[s] && a < kin[s + 1]) r = __fadd_rn(__fmul_rn(slope, __fsub_rn(a, kin[s])), kout[s]);
  }
  if (a >= kin[3]) r = kout[3];
  out[i] = r;
}

// HU -> normalized with knots (-1000, -200, 200, 1000) -> (0, .2, .8, 1) and
// clipping (mlx_pipeline.py:72-96, inverse=False): FP32 arithmetic, one
// rounding to the output dtype (f16 for the encoder input, medmlx.py:1289-1291).
// Output element i at i * out_ld (channel 0 of an NDHWC buffer).
__global__ void ct_normalize_kernel(const float* hu, long long n, void* out, int out_f32, int out_ld) {
  pdl_begin();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float a = hu[i];
  const float kin[4] = {-1000.0f, -200.0f, 200.0f, 1000.0f};
  const float kout[4] = {0.0f, 0.2f, 0.8f, 1.0f};
  float r = kout[0];
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const float slope = static_cast<float>((static_cast<double>(kout[s + 1]) - kout[s]) /
                                           (static_cast<double>(kin[s + 1]) - kin[s]));
    if (a >= kin[s] && a < kin[s + 1]) r = __fadd_rn(__fmul_rn(slope, __fsub_rn(a, kin[s])), kout[s]);
  }
  if (a >= kin[3]) r = kout[3];
  if (out_f32) {
    static_cast<float*>(out)[i * out_ld] = r;
  } else {
    static_cast<__half*>(out)[i * out_ld] = __float2half_rn(r);
  }
}

__global__ void step_advance_kernel(int* step) {
  pdl_begin();
  *step += 1;
}

}  // namespace
}  // namespace ldb

extern "C" {

int ldb_timestep_embedding(cudaStream_t stream, const int* timesteps, const int* step, int steps, int batch,
                           int channels, void* out, int out_dtype) {
  using namespace ldb;
  if (!timesteps || !out) return fail(LDB_ERR_INVALID, "timestep_embedding: null pointer");
  if (batch <= 0 || channels <= 0 || channels % 2) return fail(LDB_ERR_SHAPE, "channels must be even and positive");
  if (step && steps <= 0) return fail(LDB_ERR_SHAPE, "timestep_embedding: the step table needs >= 1 row");
  if (out_dtype != LDB_F16 && out_dtype != LDB_F32)
    return fail(LDB_ERR_INVALID, "timestep_embedding: out dtype f16 or f32");
  unsigned int* status = device_status_ptr();
  if (!status) return fail(LDB_ERR_CUDA, "timestep_embedding: no device status word");
  const int n = batch * (channels / 2);
  return launch_kernel(timestep_embedding_kernel, dim3((n + 255) / 256), dim3(256), 0, stream,
                       "timestep_embedding launch", timesteps, step, step ? steps : 1, batch, channels, out,
                       int(out_dtype == LDB_F32), status);
}

int ldb_dense_small(cudaStream_t stream, const void* x, int x_ld, const void* w, const float* bias, void* out,
                    int out_ld, int rows, int n_out, int k, int in_silu, int out_silu, int out_dtype, int round_f16) {
  using namespace ldb;
  if (!x || !w || !out) return fail(LDB_ERR_INVALID, "dense_small: null pointer");
  if (rows <= 0 || rows > kDenseMaxRows) return fail(LDB_ERR_SHAPE, "dense_small handles 1..%d rows", kDenseMaxRows);
  if (k <= 0 || k % 8 || x_ld % 8) return fail(LDB_ERR_ALIGNMENT, "K and x_ld must be multiples of 8");
  if (n_out <= 0) return fail(LDB_ERR_SHAPE, "n_out must be positive");
  if (rows > 1 && (x_ld < k || out_ld < n_out))
    return fail(LDB_ERR_SHAPE, "dense_small: row strides (%d, %d) must cover K %d and n_out %d", x_ld, out_ld, k, n_out);
  if (out_dtype != LDB_F16 && out_dtype != LDB_F32) return fail(LDB_ERR_INVALID, "dense_small: out dtype f16 or f32");
  const int threads = 256;
  const int blocks = (n_out * 32 + threads - 1) / threads;
  return launch_kernel(dense_small_kernel, dim3(blocks), dim3(threads), 0, stream, "dense_small launch",
                       static_cast<const __half*>(x), x_ld, static_cast<const __half*>(w), bias, out, out_ld, rows,
                       n_out, k, in_silu, out_silu, int(out_dtype == LDB_F32), round_f16);
}

int ldb_sampler_step_ex(cudaStream_t stream, int kind, float* x, float* prev, const void* eps, int eps_dtype,
                        int eps_ld, const float* noise, long long noise_step_stride, const float* mask,
                        const float* image, int image_channels, void* net_in, int in_ld, int net_split, int batch,
                        int voxels, int channels, const float* coeff_table, const int* step, int steps) {
  using namespace ldb;
  if (kind < 0 || kind > 2) return fail(LDB_ERR_INVALID, "sampler step kind %d", kind);
  if (step && steps <= 0) return fail(LDB_ERR_SHAPE, "sampler_step: the step tables need >= 1 row");
  if (!x || channels <= 0 || batch <= 0 || voxels <= 0) return fail(LDB_ERR_SHAPE, "sampler_step: bad extents");
  if (kind >= 1 && (!eps || !coeff_table || eps_ld < channels))
    return fail(LDB_ERR_INVALID, "sampler_step: eps/coeff");
  if (eps_dtype != LDB_F16 && eps_dtype != LDB_F32) return fail(LDB_ERR_INVALID, "sampler_step: eps dtype");
  if (kind == 1 && !noise) return fail(LDB_ERR_INVALID, "DDIM step needs noise");
  if (kind == 2 && !prev) return fail(LDB_ERR_INVALID, "DPM step needs the history buffer");
  if ((mask || net_in) && !image && (mask || image_channels > 0))
    return fail(LDB_ERR_INVALID, "sampler_step: image is required");
  const int need = channels + (mask ? 1 : image_channels);
  const int cpad = net_split ? (need + 15) / 16 * 16 : 0;
  if (net_in && in_ld < (net_split ? 2 * cpad : need))
    return fail(LDB_ERR_SHAPE, "in_ld %d too small for %d network input channels", in_ld, need);
  StepArgs a{};
  a.coeff = coeff_table;
  a.step = step;
  a.steps = step ? steps : 1;
  a.status = device_status_ptr();
  if (!a.status) return fail(LDB_ERR_CUDA, "sampler_step: no device status word");
  a.noise_step_stride = noise_step_stride;
  a.x = x;
  a.prev = prev;
  a.eps = eps;
  a.eps_ld = eps_ld;
  a.eps_f32 = eps_dtype == LDB_F32;
  a.noise = noise;
  a.mask = mask;
  a.image = image;
  a.image_c = mask ? channels : image_channels;
  a.net_in = static_cast<__half*>(net_in);
  a.in_ld = in_ld;
  a.net_cpad = cpad;
  a.voxels = static_cast<long long>(batch) * voxels;
  a.channels = channels;
  a.kind = kind;
  const int threads = 256;
  return launch_kernel(sampler_step_kernel, dim3(static_cast<unsigned>((a.voxels + threads - 1) / threads)),
                       dim3(threads), 0, stream, "sampler_step launch", a);
}

int ldb_sampler_step(cudaStream_t stream, int kind, float* x, float* prev, const void* eps, int eps_ld,
                     const float* noise, long long noise_step_stride, const float* mask, const float* image,
                     int image_channels, void* net_in, int in_ld, int batch, int voxels, int channels,
                     const float* coeff_table, const int* step, int steps) {
  return ldb_sampler_step_ex(stream, kind, x, prev, eps, LDB_F16, eps_ld, noise, noise_step_stride, mask, image,
                             image_channels, net_in, in_ld, 0, batch, voxels, channels, coeff_table, step, steps);
}

int ldb_vq_nearest4(cudaStream_t stream, const void* z, int z_ld, long long positions, const void* codebook,
                    int entries, int dtype, int* indices, void* quantized, int out_ld) {
  using namespace ldb;
  if (!z || !codebook || !indices) return fail(LDB_ERR_INVALID, "vq_nearest4: null pointer");
  if (positions <= 0 || entries <= 0) return fail(LDB_ERR_SHAPE, "positions and entries must be positive");
  if (z_ld < 4 || (quantized && out_ld < 4)) return fail(LDB_ERR_SHAPE, "strides must cover 4 channels");
  const int threads = 128;
  const unsigned blocks = static_cast<unsigned>((positions + threads - 1) / threads);
  if (dtype == LDB_F32)
    return launch_kernel(vq_nearest4_kernel<float>, dim3(blocks), dim3(threads), 0, stream, "vq_nearest4 launch",
                         static_cast<const float*>(z), z_ld, positions, static_cast<const float*>(codebook), entries,
                         indices, static_cast<float*>(quantized), out_ld);
  if (dtype == LDB_F16)
    return launch_kernel(vq_nearest4_kernel<__half>, dim3(blocks), dim3(threads), 0, stream, "vq_nearest4 launch",
                         static_cast<const __half*>(z), z_ld, positions, static_cast<const __half*>(codebook),
                         entries, indices, static_cast<__half*>(quantized), out_ld);
  return fail(LDB_ERR_INVALID, "vq_nearest4: dtype must be f16 or f32");
}

int ldb_resize_nearest(cudaStream_t stream, const void* x, int batch, int in_d, int in_h, int in_w, int row_bytes,
                       int x_row_stride, void* out, int out_d, int out_h, int out_w, int out_row_stride) {
  using namespace ldb;
  if (!x || !out) return fail(LDB_ERR_INVALID, "resize_nearest: null pointer");
  if (row_bytes <= 0 || row_bytes % 8 || x_row_stride % 8 || out_row_stride % 8)
    return fail(LDB_ERR_ALIGNMENT, "row bytes and strides must be multiples of 8 bytes");
  if (x_row_stride < row_bytes || out_row_stride < row_bytes)
    return fail(LDB_ERR_SHAPE, "resize_nearest: row strides (%d, %d) must cover the %d-byte rows", x_row_stride,
                out_row_stride, row_bytes);
  if (batch <= 0 || in_d <= 0 || in_h <= 0 || in_w <= 0 || out_d <= 0 || out_h <= 0 || out_w <= 0)
    return fail(LDB_ERR_SHAPE, "resize_nearest: extents must be positive");
  const long long total = static_cast<long long>(batch) * out_d * out_h * out_w * (row_bytes / 8);
  const int threads = 256;
  return launch_kernel(
      resize_nearest_kernel, dim3(static_cast<unsigned>((total + threads - 1) / threads)), dim3(threads), 0, stream,
      "resize_nearest launch", static_cast<const uint8_t*>(x), in_d, in_h, in_w, static_cast<uint8_t*>(out), out_d,
      out_h, out_w, batch, row_bytes, x_row_stride, out_row_stride,
      static_cast<float>(static_cast<double>(in_d) / out_d), static_cast<float>(static_cast<double>(in_h) / out_h),
      static_cast<float>(static_cast<double>(in_w) / out_w));
}

int ldb_hu_map(cudaStream_t stream, const void* x, int dtype, int x_ld, long long n, float* out) {
  using namespace ldb;
  if (!x || !out || n <= 0) return fail(LDB_ERR_INVALID, "hu_map: bad arguments");
  if (dtype != LDB_F16 && dtype != LDB_F32) return fail(LDB_ERR_INVALID, "hu_map: input dtype f16 or f32");
  if (x_ld < 1) return fail(LDB_ERR_SHAPE, "hu_map: x_ld must be positive");
  const int threads = 256;
  return launch_kernel(hu_map_kernel, dim3(static_cast<unsigned>((n + threads - 1) / threads)), dim3(threads), 0,
                       stream, "hu_map launch", x, int(dtype == LDB_F32), x_ld, n, out);
}

int ldb_ct_normalize(cudaStream_t stream, const float* hu, long long n, void* out, int out_dtype, int out_ld) {
  using namespace ldb;
  if (!hu || !out || n <= 0) return fail(LDB_ERR_INVALID, "ct_normalize: bad arguments");
  if (out_dtype != LDB_F16 && out_dtype != LDB_F32) return fail(LDB_ERR_INVALID, "ct_normalize: out dtype f16 or f32");
  if (out_ld < 1) return fail(LDB_ERR_SHAPE, "ct_normalize: out_ld must be positive");
  const int threads = 256;
  return launch_kernel(ct_normalize_kernel, dim3(static_cast<unsigned>((n + threads - 1) / threads)), dim3(threads), 0,
                       stream, "ct_normalize launch", hu, n, out, int(out_dtype == LDB_F32), out_ld);
}

int ldb_step_advance(cudaStream_t stream, int* step) {
  using namespace ldb;
  if (!step) return fail(LDB_ERR_INVALID, "step pointer is null");
  return launch_kernel(step_advance_kernel, dim3(1), dim3(1), 0, stream, "step_advance launch", step);
}

}  // extern "C"
