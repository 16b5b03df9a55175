// Flash attention on sm_100a tensor cores (tcgen05 + TMEM) for the UNet's
// spatial transformers: self-attention over flattened voxels and
// cross-attention to the projected text context, in the projection layout
// (B, L, H*D) of lesiondiffusion_mlx/_attention*.py (no head transposes).
//
// One CTA owns 128 queries of one (batch, head).  Warp 0 streams Q once and
// K/V blocks of 128 keys by TMA (2 stages); warp 1 issues S = Q K^T into one
// of two TMEM score buffers and O += P V (P from shared memory, V as an
// MN-major operand); warps 2-5 each own 32 query rows (one TMEM lane per
// thread) and run the online softmax: FP32 scores and running max / sum,
// probabilities rounded to the input type for the PV product, the FP32
// output rescaled in TMEM when the running max grows, and the final O / l
// rounded once -- the contract of _attention_half.py:58-113.  Keys past Lk
// get probability 0 (cross-attention to 77 tokens uses one partial block).
// The score buffers are double-buffered, so Q K^T of block j+1 runs on the
// tensor cores while the softmax of block j runs on the CUDA cores.

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace ldb {
namespace {

constexpr int kAttnThreads = 192;
constexpr int kBlockM = 128;
constexpr int kBlockN = 128;

template <int D>
struct AttnCfg {
  static constexpr int kRowBytes = D * 2;
  static constexpr uint32_t kLayout = D == 64 ? kSwizzle128 : (D == 32 ? kSwizzle64 : kSwizzle32);
  static constexpr uint32_t kSbo = 8 * kRowBytes;  // K-major and MN-major 8-row group stride
  static constexpr int kQBytes = kBlockM * kRowBytes;
  static constexpr int kKBytes = kBlockN * kRowBytes;
  static constexpr int kPBytes = kBlockM * kBlockN * 2;  // two 64-key SW128 chunks
  static constexpr int kStages = 2;
  // smem: Q | K0 V0 | K1 V1 | P | barriers
  static constexpr int kOffK = kQBytes;
  static constexpr int kOffP = kQBytes + kStages * 2 * kKBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
  static constexpr int kTmemCols = 512;  // S0: [0,128), S1: [128,256), O: [256, 256 + D)
};

struct AttnParams {
  int batch, heads, lq, lk;
  int out_ld;       // elements between output rows
  float scale_log2;  // softmax scale * log2(e)
  void* out;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const AttnParams p, unsigned int* status) {
  using Cfg = AttnCfg<D>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_ready = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int q0 = blockIdx.x * kBlockM;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nblocks = (p.lk + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(p_ready, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + 256;

  uint8_t* sq = smem;
  uint8_t* sp = smem + Cfg::kOffP;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t armed_mask = 0, armed_parity = 0;
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
      tma_load_3d(sq, &qmap, q_full, h * D, q0, b);
      for (int j = 0; j < nblocks; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag, status)) break;
        uint8_t* sk = smem + Cfg::kOffK + st * 2 * Cfg::kKBytes;
        mbar_arrive_expect_tx(&kv_full[st], 2 * Cfg::kKBytes);
        armed_mask |= 1u << st;
        armed_parity = (armed_parity & ~(1u << st)) | (ph << st);
        tma_load_3d(sk, &kmap, &kv_full[st], h * D, j * kBlockN, b);
        tma_load_3d(sk + Cfg::kKBytes, &vmap, &kv_full[st], h * D, j * kBlockN, b);
      }
      if (*abort_flag) {
        volatile int never = 0;
        mbar_wait(q_full, 0, &never, status);
        for (int s = 0; s < 2; ++s)
          if (armed_mask & (1u << s)) mbar_wait(&kv_full[s], (armed_parity >> s) & 1u, &never, status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBlockM, kBlockN, BF16 ? 1u : 0u, 0u, 0u);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBlockM, D, BF16 ? 1u : 0u, 0u, 1u);
      const uint32_t q_addr = smem_u32(sq);
      const uint32_t p_addr = smem_u32(sp);
      bool ok = mbar_wait(q_full, 0, abort_flag, status);
      for (int j = 0; ok && j <= nblocks; ++j) {
        if (j < nblocks) {
          // S_j = Q K_j^T into score buffer j & 1 once the softmax released it.
          const int st = j & 1;
          if (!mbar_wait(&kv_full[st], (j >> 1) & 1, abort_flag, status)) break;
          if (j >= 2 && !mbar_wait(&s_free[st], ((j >> 1) - 1) & 1, abort_flag, status)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + Cfg::kOffK + st * 2 * Cfg::kKBytes);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ad = make_smem_desc(q_addr + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
            const uint64_t bd = make_smem_desc(k_addr + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
            umma_ss(tmem + st * 128, ad, bd, idesc_qk, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
        }
        if (j > 0) {
          // P_{j-1} is in shared memory: O += P_{j-1} V_{j-1}.
          if (!mbar_wait(p_ready, (j - 1) & 1, abort_flag, status)) break;
          tc_fence_after();
          const int st = (j - 1) & 1;
          const uint32_t v_addr = smem_u32(smem + Cfg::kOffK + st * 2 * Cfg::kKBytes + Cfg::kKBytes);
#pragma unroll
          for (int k = 0; k < kBlockN / 16; ++k) {
            const uint64_t ad = make_smem_desc(p_addr + (k >> 2) * (kBlockM * 128) + (k & 3) * 32, 16, 1024,
                                               kSwizzle128);
            const uint64_t bd = make_smem_desc(v_addr + k * 16 * Cfg::kRowBytes, 16 * Cfg::kRowBytes * 8, Cfg::kSbo,
                                               Cfg::kLayout);
            umma_ss(tmem_o, ad, bd, idesc_pv, (j > 1 || k > 0) ? 1u : 0u);
          }
          umma_commit(pv_done);
          umma_commit(&kv_empty[st]);
        }
      }
      umma_commit(drain);
      volatile int never = 0;
      mbar_wait(drain, 0, &never, status);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.scale_log2;
    float m = -INFINITY;  // running max of raw scores
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblocks; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&s_full[sb], (j >> 1) & 1, abort_flag, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tmem_s = tmem + sb * 128;
      const int valid = min(kBlockN, p.lk - j * kBlockN);
      float mx = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < kBlockN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_s + lane_base + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < valid) mx = fmaxf(mx, __uint_as_float(r[i]));
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = exp2f((m - m_new) * c);
      const float mc = m_new * c;
      if (j > 0) {
        // PV_{j-1} finished: the P buffer is free and O holds blocks < j.
        if (!warp_wait(pv_done, (j - 1) & 1, abort_flag, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale the whole warp's rows
        // when any of them saw a larger maximum (alpha == 1 elsewhere).
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem_o + lane_base + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st16(tmem_o + lane_base + c0, r);
          }
          tmem_wait_st();
        }
      }
      float sum = 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < kBlockN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_s + lane_base + c0, r);
        tmem_wait_ld();
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float e0 = (c0 + i < valid) ? exp2f(fmaf(__uint_as_float(r[i]), c, -mc)) : 0.f;
          const float e1 = (c0 + i + 1 < valid) ? exp2f(fmaf(__uint_as_float(r[i + 1]), c, -mc)) : 0.f;
          sum += e0 + e1;
          if constexpr (BF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(e0, e1);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(e0, e1);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
        // Keys c0..c0+31 of this row: chunk c0/64, 16-byte units u..u+3
        // at the 128-byte-swizzled positions of row `row`.
        uint8_t* chunk = sp + (c0 >> 6) * (kBlockM * 128) + (row >> 3) * 1024 + (row & 7) * 128;
        const int u0 = (c0 & 63) >> 3;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = (u0 + u) ^ (row & 7);
          *reinterpret_cast<uint4*>(chunk + unit * 16) =
              make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
        }
      }
      l = l * alpha + sum;
      m = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[sb]);
        mbar_arrive(p_ready);
      }
    }
    if (ok && warp_wait(pv_done, (nblocks - 1) & 1, abort_flag, status)) {
      tc_fence_after();
      const int qrow = q0 + row;
      const float inv = 1.f / l;
      T* out = static_cast<T*>(p.out) + (static_cast<long long>(b) * p.lq + qrow) * p.out_ld + h * D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_o + lane_base + c0, r);
        tmem_wait_ld();
        if (qrow < p.lq) {
          uint32_t packed[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const float a0 = __uint_as_float(r[i]) * inv;
            const float a1 = __uint_as_float(r[i + 1]) * inv;
            if constexpr (BF16) {
              __nv_bfloat162 v2 = __floats2bfloat162_rn(a0, a1);
              packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
            } else {
              __half2 v2 = __floats2half2_rn(a0, a1);
              packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
            }
          }
          *reinterpret_cast<uint4*>(out + c0) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          *reinterpret_cast<uint4*>(out + c0 + 8) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
    }
    tc_fence_before();
  }

  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int D, bool BF16>
int launch_attn(cudaStream_t stream, const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                const AttnParams& p) {
  using Cfg = AttnCfg<D>;
  auto kernel = flash_attn_kernel<D, BF16>;
  static unsigned long long configured = 0;
  const int rc = ensure_smem_attribute(reinterpret_cast<const void*>(kernel), Cfg::kSmemBytes, &configured,
                                       "attention smem attribute");
  if (rc != LDB_OK) return rc;
  dim3 grid((p.lq + kBlockM - 1) / kBlockM, p.heads, p.batch);
  kernel<<<grid, kAttnThreads, Cfg::kSmemBytes, stream>>>(qm, km, vm, p, device_status_ptr());
  count_launch();
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace
}  // namespace ldb

extern "C" {

int ldb_flash_attention(cudaStream_t stream, const void* q, int q_ld, const void* k, const void* v, int kv_ld,
                        void* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim, float scale,
                        int dtype) {
  using namespace ldb;
  if (!q || !k || !v || !out) return fail(LDB_ERR_INVALID, "flash_attention: null pointer");
  if (head_dim != 16 && head_dim != 32 && head_dim != 64)
    return fail(LDB_ERR_SHAPE, "head_dim must be 16, 32 or 64 (got %d)", head_dim);
  if (dtype != LDB_F16 && dtype != LDB_BF16) return fail(LDB_ERR_INVALID, "dtype must be f16 or bf16");
  if (batch <= 0 || lq <= 0 || lk <= 0 || heads <= 0) return fail(LDB_ERR_SHAPE, "extents must be positive");
  if (q_ld < heads * head_dim || kv_ld < heads * head_dim || out_ld < heads * head_dim)
    return fail(LDB_ERR_SHAPE, "row strides must cover heads * head_dim");
  if (q_ld % 8 || kv_ld % 8 || out_ld % 8) return fail(LDB_ERR_ALIGNMENT, "row strides must be multiples of 8");
  const uint32_t box[3] = {static_cast<uint32_t>(head_dim), 128u, 1u};
  const int sw = head_dim * 2;
  CUtensorMap qm, km, vm;
  const bool bf16 = dtype == LDB_BF16;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(heads) * head_dim, static_cast<uint64_t>(lq),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(q_ld) * 2, static_cast<uint64_t>(lq) * q_ld * 2};
    int rc = encode_tiled_f16(&qm, q, 3, dims, strides, box, sw, bf16);
    if (rc != LDB_OK) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(heads) * head_dim, static_cast<uint64_t>(lk),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kv_ld) * 2, static_cast<uint64_t>(lk) * kv_ld * 2};
    int rc = encode_tiled_f16(&km, k, 3, dims, strides, box, sw, bf16);
    if (rc != LDB_OK) return rc;
    rc = encode_tiled_f16(&vm, v, 3, dims, strides, box, sw, bf16);
    if (rc != LDB_OK) return rc;
  }
  AttnParams p;
  p.batch = batch;
  p.heads = heads;
  p.lq = lq;
  p.lk = lk;
  p.out_ld = out_ld;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  if (head_dim == 64) return bf16 ? launch_attn<64, true>(stream, qm, km, vm, p) : launch_attn<64, false>(stream, qm, km, vm, p);
  if (head_dim == 32) return bf16 ? launch_attn<32, true>(stream, qm, km, vm, p) : launch_attn<32, false>(stream, qm, km, vm, p);
  return bf16 ? launch_attn<16, true>(stream, qm, km, vm, p) : launch_attn<16, false>(stream, qm, km, vm, p);
}

}  // extern "C"
