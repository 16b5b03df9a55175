// Flash attention on sm_100a tensor cores (tcgen05 + TMEM) for the UNet's
// spatial transformers: self-attention over flattened voxels and
// cross-attention to the projected text context, in the projection layout
// (B, L, H*D) of lesiondiffusion_mlx/_attention*.py (no head transposes).
//
// One CTA owns two 128-query tiles of one (batch, head) and streams K/V
// blocks of 128 keys once for both.  Warp 0 issues the TMA loads (Q once,
// K/V in a 3-stage ring); warp 1 issues the MMAs: S_t = Q_t K^T into a TMEM
// score buffer per tile and O_t += P_t V (P from shared memory, V as an
// MN-major operand, P from TMEM).  Warps 4-7 run the online softmax of tile 0 and warps
// 8-11 that of tile 1, one query row per thread: while one warpgroup turns
// its scores into probabilities, the tensor core works on the other tile.
//
// Softmax contract of _attention_half.py:58-113: FP32 scores, running max
// and sum; probabilities rounded to the input type for the PV product; the
// FP32 output divided by the sum and rounded once.  The running output is
// rescaled lazily: a row keeps its reference maximum until a new maximum
// exceeds it by more than 2^8 in probability, so probabilities stay within
// [0, 256] (exact in f16/bf16 range) and most blocks skip the TMEM rescale.
// Keys past Lk get probability 0 (cross-attention to 77 tokens is one
// partial block).

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace ldb {
namespace {

// Three warpgroups: WG0 = producer warp, MMA warp and two idle warps; WG1 and
// WG2 = the softmax of query tiles 0 and 1.  Ten or twelve warps put three
// warps on some SM sub-partitions, which caps a thread at 168 registers at
// launch; WG0 gives registers up (setmaxnreg) so the softmax warps, which
// hold a 128-score row each, get 216.  128 x 72 + 256 x 216 = 384 x 168.
constexpr int kAttnThreads = 384;
constexpr int kAttnLaunchRegs = 168;
constexpr int kAttnRegsWg0 = 72;
constexpr int kAttnRegsSoftmax = 216;
static_assert(128 * kAttnRegsWg0 + 256 * kAttnRegsSoftmax <= kAttnThreads * kAttnLaunchRegs, "register split");
constexpr int kBlockM = 128;       // queries per tile (two tiles per CTA)
constexpr int kBlockN = 128;       // keys per block
constexpr float kRescaleLog2 = 8.0f;

// SPLIT: FP32 attention in the split-f16 form (the reference's FP32 kernel,
// _attention.py:148-280): every operand is two f16 planes, hi = f16(x) and a
// low plane, loaded as separate tiles.  Scores take Qh Kh + Qh Kl + Ql Kh
// into one FP32 accumulator (Q / K low planes unscaled, x - hi, so the three
// products add directly); O keeps Ph Vh and the 2^11-scaled cross terms
// Ph Vl' + Pl' Vh in two accumulators, combined as hi + lo / 2048 at the end.
template <int D, bool SPLIT = false>
struct AttnCfg {
  static constexpr int kPlanes = SPLIT ? 2 : 1;
  static constexpr int kRowBytes = D * 2;
  static constexpr uint32_t kLayout = D == 64 ? kSwizzle128 : (D == 32 ? kSwizzle64 : kSwizzle32);
  static constexpr uint32_t kSbo = 8 * kRowBytes;  // K-major and MN-major 8-row group stride
  static constexpr int kQBytes = kBlockM * kRowBytes;    // one plane of a query tile
  static constexpr int kKBytes = kBlockN * kRowBytes;    // one plane of a K or V block
  static constexpr int kStages = SPLIT ? (D == 64 ? 2 : 3) : 4;
  // smem: Q [tile][plane] | stages x (K planes, V planes) | barriers
  static constexpr int kOffK = 2 * kPlanes * kQBytes;
  static constexpr int kStageBytes = 2 * kPlanes * kKBytes;
  static constexpr int kOffBar = kOffK + kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;  // barriers: 2 kStages + 11 words, then the TMEM slot
  static_assert((2 * kStages + 11) * 8 + 16 <= 256, "attention barrier block");
  // TMEM: S0 [0,128), S1 [128,256), O0 [256, 256 + planes*D), O1 [384, 384 + planes*D).
  // Split form: the probabilities overwrite their scores as packed 16-bit
  // pairs, P_t plane 0 in columns [128t, 128t + 64), plane 1 in [128t + 64,
  // 128t + 128).  16-bit form (one plane, D <= 64): P_t has its own columns
  // [256 + 128t + 64, 256 + 128t + 128) beside O_t, so the next block's
  // scores can be computed into S_t while P_t still feeds the PV product.
  static constexpr bool kSeparateP = !SPLIT;
  static_assert(SPLIT || D <= 64, "O_t and P_t share a 128-column TMEM region");
  static constexpr int kTmemCols = 512;
  static_assert(kSmemBytes <= 232448, "attention shared memory");
};

// Paired FP32 arithmetic (sm_100 f32x2 instructions) and the 3-input max:
// the softmax issues one instruction per pair of scores for the scale and
// the row sum, and one per two scores for the row maximum.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

struct AttnParams {
  int batch, heads, lq, lk;
  int out_ld;        // elements between output rows
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  // Split over keys: blockIdx.x = query pair * kv_splits + split; split s
  // covers key blocks [s * blocks_per_split, ...) and, when kv_splits > 1,
  // writes its unnormalised O rows (f32, [split][b][h][q][D]) and the rows'
  // (reference max, sum) ([split][b][h][q][2]) for attn_combine_kernel.
  int kv_splits, blocks_per_split;
  float* o_part;
  float* ml_part;
  // Device-clock timing of the launch (may be null): [start, end] in ns,
  // lowered / raised atomically by the CTAs (and the merge kernel).
  unsigned long long* clock;
  // Stream-K schedule (sk_ctas > 0; blockIdx.x = CTA, grid 1 x 1 in y, z):
  // the sk_units = pairs x sk_nb (query pair, key block) units are cut into
  // sk_ctas equal ranges; sk_pairs query pairs per (batch, head); a CTA's
  // segment s of a pair it does not cover whole writes its raw O rows and
  // (reference max, sum) to slot blockIdx.x * sk_slots + s of o_part /
  // ml_part (256 rows each) for attn_sk_merge_kernel.
  int sk_ctas, sk_nb, sk_pairs, sk_slots;
  long long sk_units;
};

// One segment of a CTA's work: a query pair (two 128-row tiles of one batch
// item and head) over a range of key blocks.  The plain schedule has one
// segment per CTA (its pair, all keys or one key split); the stream-K
// schedule gives a CTA the end of one pair and the start of the next (or a
// few pairs), each a segment, so every CTA does the same number of blocks.
struct AttnSeg {
  int b, h, q0, jb0, nblocks;
  bool whole;
};

struct AttnSched {
  long long u, u_end;
};

__device__ __forceinline__ long long sk_unit0(const AttnParams& p, long long cta) {
  return cta * p.sk_units / p.sk_ctas;
}

__device__ __forceinline__ AttnSched sched_begin(const AttnParams& p) {
  AttnSched sc;
  if (p.sk_ctas > 0) {
    sc.u = sk_unit0(p, blockIdx.x);
    sc.u_end = sk_unit0(p, blockIdx.x + 1);
  } else {
    sc.u = 0;
    sc.u_end = 1;
  }
  return sc;
}

__device__ __forceinline__ bool sched_next(const AttnParams& p, AttnSched& sc, AttnSeg& g) {
  if (sc.u >= sc.u_end) return false;
  if (p.sk_ctas > 0) {
    const long long pair = sc.u / p.sk_nb;
    const int j0 = static_cast<int>(sc.u - pair * p.sk_nb);
    const int n = static_cast<int>(min(static_cast<long long>(p.sk_nb - j0), sc.u_end - sc.u));
    const long long bh = pair / p.sk_pairs;
    g.q0 = static_cast<int>(pair - bh * p.sk_pairs) * 2 * kBlockM;
    g.h = static_cast<int>(bh % p.heads);
    g.b = static_cast<int>(bh / p.heads);
    g.jb0 = j0;
    g.nblocks = n;
    g.whole = j0 == 0 && n == p.sk_nb;
    sc.u += n;
  } else {
    const int split = blockIdx.x % p.kv_splits;
    g.q0 = (blockIdx.x / p.kv_splits) * 2 * kBlockM;
    g.h = blockIdx.y;
    g.b = blockIdx.z;
    g.jb0 = split * p.blocks_per_split;
    g.nblocks = min((p.lk + kBlockN - 1) / kBlockN - g.jb0, p.blocks_per_split);
    g.whole = p.kv_splits == 1;
    sc.u = sc.u_end;
  }
  return true;
}

template <int D, bool BF16, bool SPLIT>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const AttnParams p, unsigned int* status) {
  using Cfg = AttnCfg<D, SPLIT>;
  constexpr int kPl = Cfg::kPlanes;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  constexpr int kS = Cfg::kStages;
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;             // [kStages]
  uint64_t* kv_empty = kv_full + kS;        // [kStages]
  uint64_t* s_full = kv_empty + kS;         // [2] per query tile
  uint64_t* p_ready = s_full + 2;           // [2]
  uint64_t* pv_done = p_ready + 2;          // [2]
  uint64_t* drain = pv_done + 2;
  uint64_t* q_empty = drain + 1;            // the S MMAs of a segment have read Q
  uint64_t* s_free = q_empty + 1;           // [2] the softmax has read S_t into registers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&pv_done[t], 1);
      mbar_init(&s_free[t], 4);
    }
    mbar_init(drain, 1);
    mbar_init(q_empty, 1);
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
  pdl_begin();
  if (p.clock && threadIdx.x == 0) atomicMin(p.clock, static_cast<unsigned long long>(globaltimer_ns()));

  // The register split sits at the top of each warpgroup's branch (one
  // instruction for all four warps), so every role's code is compiled with
  // its own budget.
  if (warp < 4) {
  regs_dec<kAttnRegsWg0>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t armed_mask = 0, armed_parity = 0;
      AttnSched sc = sched_begin(p);
      AttnSeg g;
      long long blk = 0;  // key blocks loaded so far (the K/V ring position)
      int qloads = 0;
      bool ok = true;
      while (ok && sched_next(p, sc, g)) {
        // the previous segment's S MMAs must have read the Q buffer
        if (qloads > 0 && !mbar_wait(q_empty, (qloads - 1) & 1, abort_flag, status)) break;
        mbar_arrive_expect_tx(q_full, 2 * kPl * Cfg::kQBytes);
        // head h, plane pl starts at column (h * planes + pl) * D of the projection row
        for (int t = 0; t < 2; ++t)
          for (int pl = 0; pl < kPl; ++pl)
            tma_load_3d(smem + (t * kPl + pl) * Cfg::kQBytes, &qmap, q_full, (g.h * kPl + pl) * D,
                        g.q0 + t * kBlockM, g.b);
        ++qloads;
        for (int j = 0; j < g.nblocks; ++j, ++blk) {
          const int st = static_cast<int>(blk % Cfg::kStages);
          const uint32_t ph = static_cast<uint32_t>(blk / Cfg::kStages) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          uint8_t* sk = smem + Cfg::kOffK + st * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&kv_full[st], Cfg::kStageBytes);
          armed_mask |= 1u << st;
          armed_parity = (armed_parity & ~(1u << st)) | (ph << st);
          for (int pl = 0; pl < kPl; ++pl) {
            tma_load_3d(sk + pl * Cfg::kKBytes, &kmap, &kv_full[st], (g.h * kPl + pl) * D, (g.jb0 + j) * kBlockN,
                        g.b);
            tma_load_3d(sk + (kPl + pl) * Cfg::kKBytes, &vmap, &kv_full[st], (g.h * kPl + pl) * D,
                        (g.jb0 + j) * kBlockN, g.b);
          }
        }
      }
      if (*abort_flag) {
        // Let every armed TMA land before the CTA releases its shared memory
        // (earlier Q loads were consumed before the last one was issued).
        volatile int never = 0;
        if (qloads > 0) mbar_wait(q_full, (qloads - 1) & 1, &never, status);
        for (int s = 0; s < Cfg::kStages; ++s)
          if (armed_mask & (1u << s)) mbar_wait(&kv_full[s], (armed_parity >> s) & 1u, &never, status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBlockM, kBlockN, BF16 ? 1u : 0u, 0u, 0u);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBlockM, D, BF16 ? 1u : 0u, 0u, 1u);
      AttnSched sc = sched_begin(p);
      AttnSeg g;
      long long blk = 0;  // key blocks of earlier segments
      int seg = 0;
      bool ok = true;
      while (ok && sched_next(p, sc, g)) {
      ok = mbar_wait(q_full, seg & 1, abort_flag, status);
      if constexpr (Cfg::kSeparateP) {
        // Per key block j: S_t(j) as soon as the softmax has read S_t(j - 1)
        // and K_j has landed, then PV_t(j - 1) when P_t(j - 1) is ready; the
        // score product of the next block runs under the softmax of this one.
        for (int j = 0; ok && j <= g.nblocks; ++j) {
          const long long cur = blk + j;
          const int st = static_cast<int>(cur % Cfg::kStages);
          const int pst = static_cast<int>((cur + Cfg::kStages - 1) % Cfg::kStages);  // stage of block j - 1
          if (j < g.nblocks) {
            if (!mbar_wait(&kv_full[st], static_cast<uint32_t>(cur / Cfg::kStages) & 1u, abort_flag, status)) {
              ok = false;
              break;
            }
            for (int t = 0; t < 2 && ok; ++t) {
              // S_t was last read by the softmax of the previous block (of this or an earlier segment)
              if (cur > 0 && !mbar_wait(&s_free[t], static_cast<uint32_t>(cur - 1) & 1u, abort_flag, status)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t q_addr = smem_u32(smem + t * kPl * Cfg::kQBytes);
              const uint32_t k_addr = smem_u32(smem + Cfg::kOffK + st * Cfg::kStageBytes);
#pragma unroll
              for (int k = 0; k < D / 16; ++k) {
                const uint64_t ad = make_smem_desc(q_addr + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
                const uint64_t bd = make_smem_desc(k_addr + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
                umma_ss(tmem + t * 128, ad, bd, idesc_qk, k > 0 ? 1u : 0u);
              }
              umma_commit(&s_full[t]);
            }
          }
          for (int t = 0; t < 2 && ok && j > 0; ++t) {
            // P_t(j-1) is in its own columns: O_t += P_t V_{j-1}.
            if (!mbar_wait(&p_ready[t], static_cast<uint32_t>(cur - 1) & 1u, abort_flag, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t p_tmem = tmem + 256 + t * 128 + 64;
            const uint32_t v_addr = smem_u32(smem + Cfg::kOffK + pst * Cfg::kStageBytes + kPl * Cfg::kKBytes);
            const uint32_t o_acc = tmem + 256 + t * 128;
#pragma unroll
            for (int k = 0; k < kBlockN / 16; ++k) {
              const uint64_t bd = make_smem_desc(v_addr + k * 16 * Cfg::kRowBytes, 16 * Cfg::kRowBytes * 8,
                                                 Cfg::kSbo, Cfg::kLayout);
              umma_ts(o_acc, p_tmem + k * 8, bd, idesc_pv, (j > 1 || k > 0) ? 1u : 0u);
            }
            umma_commit(&pv_done[t]);
            if (t == 1) umma_commit(&kv_empty[pst]);
          }
        }
      } else
      for (int j = 0; ok && j <= g.nblocks; ++j) {
        const long long cur = blk + j;  // this block's position in the K/V ring and the tile barriers
        const int st = static_cast<int>(cur % Cfg::kStages);
        const int pst = static_cast<int>((cur + Cfg::kStages - 1) % Cfg::kStages);  // stage of block j - 1
        if (j < g.nblocks &&
            !mbar_wait(&kv_full[st], static_cast<uint32_t>(cur / Cfg::kStages) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        for (int t = 0; t < 2 && ok; ++t) {
          if (j > 0) {
            // P_t(j-1) is in TMEM over S_t: O_t += P_t V_{j-1}.
            if (!mbar_wait(&p_ready[t], static_cast<uint32_t>(cur - 1) & 1u, abort_flag, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t p_tmem = tmem + t * 128;  // P_t overwrote S_t
            const uint32_t v_addr = smem_u32(smem + Cfg::kOffK + pst * Cfg::kStageBytes + kPl * Cfg::kKBytes);
            const uint32_t o_hi = tmem + 256 + t * 128;
            // (P plane, V plane, accumulator): Ph Vh -> O_hi; split adds Ph Vl', Pl' Vh -> O_lo
            constexpr int kTerms = SPLIT ? 3 : 1;
#pragma unroll
            for (int term = 0; term < kTerms; ++term) {
              const uint32_t pa = p_tmem + (term == 2 ? 64 : 0);
              const uint32_t va = v_addr + (term == 1 ? Cfg::kKBytes : 0);
              const uint32_t acc = o_hi + (term > 0 ? D : 0);
#pragma unroll
              for (int k = 0; k < kBlockN / 16; ++k) {
                // 16 keys = 8 TMEM columns of packed pairs
                const uint64_t bd = make_smem_desc(va + k * 16 * Cfg::kRowBytes, 16 * Cfg::kRowBytes * 8,
                                                   Cfg::kSbo, Cfg::kLayout);
                umma_ts(acc, pa + k * 8, bd, idesc_pv, (j > 1 || k > 0 || term == 2) ? 1u : 0u);
              }
            }
            umma_commit(&pv_done[t]);
            if (t == 1) umma_commit(&kv_empty[pst]);
          }
          if (j < g.nblocks) {
            // S_t(j) = Q_t K_j^T (split: Qh Kh + Qh Kl + Ql Kh)
            const uint32_t q_addr = smem_u32(smem + t * kPl * Cfg::kQBytes);
            const uint32_t k_addr = smem_u32(smem + Cfg::kOffK + st * Cfg::kStageBytes);
            constexpr int kTerms = SPLIT ? 3 : 1;
#pragma unroll
            for (int term = 0; term < kTerms; ++term) {
              const uint32_t qa = q_addr + (term == 2 ? Cfg::kQBytes : 0);
              const uint32_t ka = k_addr + (term == 1 ? Cfg::kKBytes : 0);
#pragma unroll
              for (int k = 0; k < D / 16; ++k) {
                const uint64_t ad = make_smem_desc(qa + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
                const uint64_t bd = make_smem_desc(ka + k * 32, 16, Cfg::kSbo, Cfg::kLayout);
                umma_ss(tmem + t * 128, ad, bd, idesc_qk, (k > 0 || term > 0) ? 1u : 0u);
              }
            }
            umma_commit(&s_full[t]);
          }
        }
      }
      umma_commit(q_empty);  // arrives when the segment's S MMAs (readers of Q) are done
      blk += g.nblocks;
      ++seg;
      }
      umma_commit(drain);
      volatile int never = 0;
      mbar_wait(drain, 0, &never, status);
    }
  }
  } else {
  regs_inc<kAttnRegsSoftmax>();
  {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;   // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tmem_s = tmem + t * 128 + lane_base;
    const uint32_t tmem_o = tmem + 256 + t * 128 + lane_base;
    // where the packed probabilities go: their own columns, or over the scores
    const uint32_t tmem_p = Cfg::kSeparateP ? tmem_o + 64 : tmem_s;
    const float c = p.scale_log2;
    AttnSched sc = sched_begin(p);
    AttnSeg g;
    long long blk = 0;  // key blocks of earlier segments
    int seg = 0;
    bool ok = true;
    while (ok && sched_next(p, sc, g)) {
    float m_ref = -INFINITY;  // reference maximum (raw scores) of the probabilities in O and l
    float l = 0.f;
    for (int j = 0; j < g.nblocks; ++j) {
      const long long cur = blk + j;
      if (!warp_wait(&s_full[t], static_cast<uint32_t>(cur) & 1u, abort_flag, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = min(kBlockN, p.lk - (g.jb0 + j) * kBlockN);
      uint32_t sr[kBlockN];
#pragma unroll
      for (int c0 = 0; c0 < kBlockN; c0 += 32) {
        uint32_t(&chunk)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[c0]);
        tmem_ld32(tmem_s + c0, chunk);
      }
      tmem_wait_ld();
      if constexpr (Cfg::kSeparateP) {
        // the scores are in registers: S_t may take the next block's product
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);
      }
      const bool full = valid == kBlockN;
      if (!full) {
        // keys past the end never count: -inf scores give zero probability
#pragma unroll
        for (int i = 0; i < kBlockN; ++i)
          if (i >= valid) sr[i] = __float_as_uint(-INFINITY);
      }
      // row maximum: four independent chains of 3-input maxima, folded
      float m4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) m4[k] = fmaxf(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1]));
#pragma unroll
      for (int i = 8; i < kBlockN; i += 8)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          m4[k] = max3(m4[k], __uint_as_float(sr[i + 2 * k]), __uint_as_float(sr[i + 2 * k + 1]));
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      const bool first = j == 0;
      const bool grow = first || (mx - m_ref) * c > kRescaleLog2;
      const float m_new = grow ? fmaxf(m_ref, mx) : m_ref;
      const float alpha = first ? 0.f : exp2f((m_ref - m_new) * c);
      if (j > 0) {
        // PV_t(j-1) finished: the P buffer is free and O holds blocks < j.
        if (!warp_wait(&pv_done[t], static_cast<uint32_t>(cur - 1) & 1u, abort_flag, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale the warp's rows when any grew.
        if (__any_sync(0xffffffffu, grow)) {
          const float scale = grow ? alpha : 1.f;
#pragma unroll
          for (int c0 = 0; c0 < kPl * D; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem_o + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * scale);
            tmem_st16(tmem_o + c0, r);
          }
          tmem_wait_st();
        }
      }
      if (grow) {
        l *= alpha;
        m_ref = m_new;
      }
      const float mc = m_ref * c;
      const uint64_t c2 = pack2(c, c), nmc2 = pack2(-mc, -mc);
      uint64_t sum2[2] = {pack2(0.f, 0.f), pack2(0.f, 0.f)};  // independent paired row sums
#pragma unroll
      for (int c0 = 0; c0 < kBlockN; c0 += 32) {
        uint32_t packed[16];
        uint32_t packed_lo[SPLIT ? 16 : 1];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float x0, x1;
          unpack2(fma2(pack2(__uint_as_float(sr[c0 + i]), __uint_as_float(sr[c0 + i + 1])), c2, nmc2), x0, x1);
          const float e0 = ex2_approx(x0);
          const float e1 = ex2_approx(x1);
          sum2[(i >> 1) & 1] = add2(sum2[(i >> 1) & 1], pack2(e0, e1));
          if constexpr (BF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(e0, e1);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(e0, e1);
            packed[i / 2] = *reinterpret_cast<uint32_t*>(&v2);
            if constexpr (SPLIT) {
              const float2 hf = __half22float2(v2);
              __half2 l2 = __floats2half2_rn((e0 - hf.x) * 2048.0f, (e1 - hf.y) * 2048.0f);
              packed_lo[i / 2] = *reinterpret_cast<uint32_t*>(&l2);
            }
          }
        }
        // Keys c0..c0+31 of this row: 16 packed pairs over its scores (all
        // of which are already in registers).
        tmem_st16(tmem_p + (c0 >> 1), packed);
        if constexpr (SPLIT) tmem_st16(tmem_s + 64 + (c0 >> 1), packed_lo);
      }
      {
        float a0, a1, b0, b1;
        unpack2(sum2[0], a0, a1);
        unpack2(sum2[1], b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t]);
    }
    const bool done = ok && warp_wait(&pv_done[t], static_cast<uint32_t>(blk + g.nblocks - 1) & 1u, abort_flag,
                                      status);
    if (!done) ok = false;
    const int q0 = g.q0, h = g.h, b = g.b;
    if (done && !g.whole) {
      // Partial over this segment's keys: raw O row (hi + lo / 2048 for the
      // split form), reference max and sum.
      tc_fence_after();
      const int qrow = q0 + t * kBlockM + row;
      long long prow;
      if (p.sk_ctas > 0)
        prow = (static_cast<long long>(blockIdx.x) * p.sk_slots + seg) * (2 * kBlockM) + t * kBlockM + row;
      else
        prow = ((static_cast<long long>(blockIdx.x % p.kv_splits) * p.batch + b) * p.heads + h) * p.lq + qrow;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t r[16], lo[16];
        tmem_ld16(tmem_o + c0, r);
        if constexpr (SPLIT) tmem_ld16(tmem_o + D + c0, lo);
        tmem_wait_ld();
        if (qrow < p.lq) {
          float4* o4 = reinterpret_cast<float4*>(p.o_part + prow * D + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4 o = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                   __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
            if constexpr (SPLIT) {
              o.x += __uint_as_float(lo[4 * i]) * (1.0f / 2048.0f);
              o.y += __uint_as_float(lo[4 * i + 1]) * (1.0f / 2048.0f);
              o.z += __uint_as_float(lo[4 * i + 2]) * (1.0f / 2048.0f);
              o.w += __uint_as_float(lo[4 * i + 3]) * (1.0f / 2048.0f);
            }
            o4[i] = o;
          }
        }
      }
      if (qrow < p.lq) *reinterpret_cast<float2*>(p.ml_part + prow * 2) = make_float2(m_ref, l);
    } else if (done && SPLIT) {
      tc_fence_after();
      const int qrow = q0 + t * kBlockM + row;
      const float inv = 1.f / l;
      float* out = static_cast<float*>(p.out) + (static_cast<long long>(b) * p.lq + qrow) * p.out_ld + h * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t r[16], lo[16];
        tmem_ld16(tmem_o + c0, r);
        tmem_ld16(tmem_o + D + c0, lo);
        tmem_wait_ld();
        if (qrow < p.lq) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            float4 o;
            o.x = (__uint_as_float(r[i]) + __uint_as_float(lo[i]) * (1.0f / 2048.0f)) * inv;
            o.y = (__uint_as_float(r[i + 1]) + __uint_as_float(lo[i + 1]) * (1.0f / 2048.0f)) * inv;
            o.z = (__uint_as_float(r[i + 2]) + __uint_as_float(lo[i + 2]) * (1.0f / 2048.0f)) * inv;
            o.w = (__uint_as_float(r[i + 3]) + __uint_as_float(lo[i + 3]) * (1.0f / 2048.0f)) * inv;
            *reinterpret_cast<float4*>(out + c0 + i) = o;
          }
        }
      }
    } else if (done) {
      tc_fence_after();
      const int qrow = q0 + t * kBlockM + row;
      const float inv = 1.f / l;
      T* out = static_cast<T*>(p.out) + (static_cast<long long>(b) * p.lq + qrow) * p.out_ld + h * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_o + c0, r);
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
    // the O reads above come before this warpgroup's next p_ready arrive
    tc_fence_before();
    blk += g.nblocks;
    ++seg;
    }
  }
  }

  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (p.clock && threadIdx.x == 0) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
}

// Merge the key splits of each query row: M = max of the splits' reference
// maxima, out = sum_s 2^((m_s - M) c) O_s / sum_s 2^((m_s - M) c) l_s,
// rounded once.  One warp per (b, h, q) row; lane i holds dims i, i + 32.
template <int D, bool BF16>
__global__ void attn_combine_kernel(const AttnParams p) {
  pdl_begin();
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const long long rows = static_cast<long long>(p.batch) * p.heads * p.lq;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int s = 0; s < p.kv_splits; ++s) mx = fmaxf(mx, p.ml_part[(s * rows + row) * 2]);
  float den = 0.f, a0 = 0.f, a1 = 0.f;
  for (int s = 0; s < p.kv_splits; ++s) {
    const float2 ml = *reinterpret_cast<const float2*>(p.ml_part + (s * rows + row) * 2);
    const float wgt = exp2f((ml.x - mx) * p.scale_log2);
    den = fmaf(wgt, ml.y, den);
    const float* o = p.o_part + (s * rows + row) * D;
    if (lane < D) a0 = fmaf(wgt, o[lane], a0);
    if (lane + 32 < D) a1 = fmaf(wgt, o[lane + 32], a1);
  }
  const float inv = 1.f / den;
  const int q = static_cast<int>(row % p.lq);
  const long long bh = row / p.lq;
  const int h = static_cast<int>(bh % p.heads);
  const int b = static_cast<int>(bh / p.heads);
  T* out = static_cast<T*>(p.out) + (static_cast<long long>(b) * p.lq + q) * p.out_ld + h * D;
  if (lane < D) out[lane] = static_cast<T>(a0 * inv);
  if (lane + 32 < D) out[lane + 32] = static_cast<T>(a1 * inv);
  if (p.clock && lane == 0) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
}

// FP32 projections -> split f16 planes for the SPLIT kernel.  src is
// (rows, H*D) f32 with row stride src_ld; dst is (rows, H*2D) f16 with head
// h at columns [2hD, 2hD + D) (hi) and [2hD + D, 2hD + 2D) (low): hi =
// f16(x * mul), low = f16((x * mul - hi) * lo_scale).  One thread per 8
// elements.
__global__ void attn_split_kernel(const float* src, int src_ld, long long rows, int heads, int d, float mul,
                                  float lo_scale, __half* dst) {
  pdl_begin();
  const int vecs = heads * d / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * vecs) return;
  const long long r = idx / vecs;
  const int col = static_cast<int>(idx - r * vecs) * 8;
  const int hh = col / d, c = col - hh * d;
  const float4 a = *reinterpret_cast<const float4*>(src + r * src_ld + col);
  const float4 b = *reinterpret_cast<const float4*>(src + r * src_ld + col + 4);
  const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint4 hi_raw, lo_raw;
  __half* hi = reinterpret_cast<__half*>(&hi_raw);
  __half* lo = reinterpret_cast<__half*>(&lo_raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = x[j] * mul;
    hi[j] = __float2half_rn(v);
    lo[j] = __float2half_rn((v - __half2float(hi[j])) * lo_scale);
  }
  __half* o = dst + r * (2LL * heads * d) + 2LL * hh * d + c;
  *reinterpret_cast<uint4*>(o) = hi_raw;
  *reinterpret_cast<uint4*>(o + d) = lo_raw;
}

// Merge the stream-K segments of the query rows of each pair that was split
// over several CTAs (a pair one CTA held whole was written by that CTA): M =
// max of the segments' reference maxima, out = sum_s w_s O_s / sum_s w_s l_s
// with w_s = 2^((m_s - M) c), rounded once.  Block (pair, group of 8 rows):
// thread 0 finds the covering CTAs (unit u belongs to CTA ((u + 1) G - 1) / U
// of the even cut) and their slot rows; then one warp per query row, lane i
// on dims i and i + 32, all segments' loads issued together.
constexpr int kMergeMaxCtas = 8;
constexpr int kMergeRows = 8;  // query rows per block (one per warp)

template <int D, typename OutT>
__global__ void attn_sk_merge_kernel(const AttnParams p, unsigned int* status) {
  pdl_begin();
  __shared__ long long slot_row[kMergeMaxCtas];
  __shared__ int ncta;
  constexpr int kGroups = 2 * kBlockM / kMergeRows;
  const long long pair = blockIdx.x / kGroups;
  if (threadIdx.x == 0) {
    const long long u_first = pair * p.sk_nb, u_last = u_first + p.sk_nb - 1;
    const long long c0 = ((u_first + 1) * p.sk_ctas - 1) / p.sk_units;
    const long long c1 = ((u_last + 1) * p.sk_ctas - 1) / p.sk_units;
    int n = 0;
    if (c1 - c0 + 1 > kMergeMaxCtas) {
      n = -1;  // the plan never cuts a pair this finely (at least 8 blocks per CTA)
    } else if (c0 != c1) {
      for (long long cta = c0; cta <= c1; ++cta, ++n)
        slot_row[n] = (cta * p.sk_slots + (pair - sk_unit0(p, cta) / p.sk_nb)) * (2 * kBlockM);
    }
    ncta = n;
  }
  __syncthreads();
  const int n = ncta;
  const long long bh = pair / p.sk_pairs;
  const int r = static_cast<int>(blockIdx.x % kGroups) * kMergeRows + (threadIdx.x >> 5);
  const int q = static_cast<int>(pair - bh * p.sk_pairs) * 2 * kBlockM + r;
  if (n > 0 && q < p.lq) {
    const int lane = threadIdx.x & 31;
    const int h = static_cast<int>(bh % p.heads);
    const int b = static_cast<int>(bh / p.heads);
    float2 ml[kMergeMaxCtas];
    float o0[kMergeMaxCtas], o1[kMergeMaxCtas];
#pragma unroll
    for (int k = 0; k < kMergeMaxCtas; ++k) {
      if (k < n) {
        const long long srow = slot_row[k] + r;
        ml[k] = *reinterpret_cast<const float2*>(p.ml_part + srow * 2);
        const float* o = p.o_part + srow * D;
        o0[k] = lane < D ? o[lane] : 0.f;
        o1[k] = lane + 32 < D ? o[lane + 32] : 0.f;
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMergeMaxCtas; ++k)
      if (k < n) mx = fmaxf(mx, ml[k].x);
    float den = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int k = 0; k < kMergeMaxCtas; ++k) {
      if (k < n) {
        const float wgt = exp2f((ml[k].x - mx) * p.scale_log2);
        den = fmaf(wgt, ml[k].y, den);
        a0 = fmaf(wgt, o0[k], a0);
        a1 = fmaf(wgt, o1[k], a1);
      }
    }
    const float inv = 1.f / den;
    OutT* out = static_cast<OutT*>(p.out) + (static_cast<long long>(b) * p.lq + q) * p.out_ld + h * D;
    if (lane < D) out[lane] = static_cast<OutT>(a0 * inv);
    if (lane + 32 < D) out[lane + 32] = static_cast<OutT>(a1 * inv);
  } else if (n < 0 && threadIdx.x == 0) {
    set_bad_shape(status);
  }
  if (p.clock && threadIdx.x == 0) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
}

// Stream-K plan for a grid of `ctas` CTAs (query pairs x heads x batch) over
// `blocks` key blocks each, when the grid leaves a large share of the SMs
// idle in its last wave (and small grids are not already split over keys):
// every SM takes an equal range of (pair, key block) units, at least 8
// blocks.  Returns the CTAs (0: plain schedule) and the partial slots per CTA.
int choose_stream_k(long long ctas, int blocks, int* slots) {
  const int sms = sm_count();
  *slots = 0;
  if (ctas * 2 <= sms || blocks < 8) return 0;
  const long long waves = (ctas + sms - 1) / sms;
  if (ctas * 10 >= waves * sms * 9) return 0;  // the plain grid already fills 90 % of the waves
  const long long units = ctas * blocks;
  const long long per = (units + sms - 1) / sms;
  if (per < 8) return 0;
  *slots = static_cast<int>((per + blocks - 1) / blocks) + 1;
  return sms;
}

// Key splits for a grid of `ctas` CTAs over `blocks` key blocks.  Splitting
// costs a partial write, a merge launch and per-CTA set-up, which only pays
// when the unsplit grid leaves most SMs idle (measured: 32 CTAs of 800
// queries x 8 heads gain 1.3x with 4 ranges of 2 key blocks, 100 CTAs of
// 6400 x 4 heads lose 1.15x): split only grids of fewer than half the SMs,
// into as many ranges as fill the GPU once.
int choose_kv_splits(long long ctas, int blocks) {
  const int sms = sm_count();
  if (ctas * 2 > sms || blocks < 2) return 1;
  const int want = static_cast<int>(std::min<long long>((sms + ctas - 1) / ctas, 8));
  const int splits = std::max(1, std::min(want, blocks));
  const int bps = (blocks + splits - 1) / splits;
  return (blocks + bps - 1) / bps;  // ranges that get key blocks
}

template <int D, bool BF16, bool SPLIT = false>
int launch_attn(cudaStream_t stream, const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                const AttnParams& p) {
  using Cfg = AttnCfg<D, SPLIT>;
  auto kernel = flash_attn_kernel<D, BF16, SPLIT>;
  static unsigned long long configured = 0;
  int rc = ensure_smem_attribute(reinterpret_cast<const void*>(kernel), Cfg::kSmemBytes, &configured,
                                 "attention smem attribute");
  if (rc != LDB_OK) return rc;
  // The warpgroups' register split must fit the registers the CTA is
  // launched with, or the softmax warps' setmaxnreg.inc would wait forever.
  static int launch_regs = 0;
  if (launch_regs == 0) {
    cudaFuncAttributes attr;
    rc = check_cuda(cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(kernel)), "attention attributes");
    if (rc != LDB_OK) return rc;
    launch_regs = attr.numRegs;
  }
  if (launch_regs * kAttnThreads < 128 * kAttnRegsWg0 + 256 * kAttnRegsSoftmax)
    return fail(LDB_ERR_CUDA, "attention kernel launches with %d registers per thread; the register split needs %d",
                launch_regs, kAttnLaunchRegs);
  dim3 grid(((p.lq + 2 * kBlockM - 1) / (2 * kBlockM)) * p.kv_splits, p.heads, p.batch);
  if (p.sk_ctas > 0) grid = dim3(p.sk_ctas, 1, 1);
  int r = launch_kernel(kernel, grid, dim3(kAttnThreads), Cfg::kSmemBytes, stream, "attention launch", qm, km, vm,
                        p, device_status_ptr());
  if (r != LDB_OK) return r;
  if (p.sk_ctas > 0 && p.sk_nb > 1) {  // (with one key block every unit is whole)
    using OutT = typename std::conditional<SPLIT, float,
                                           typename std::conditional<BF16, __nv_bfloat16, __half>::type>::type;
    const long long blocks = p.sk_units / p.sk_nb * (2 * kBlockM / kMergeRows);
    return launch_kernel(attn_sk_merge_kernel<D, OutT>, dim3(static_cast<unsigned>(blocks)), dim3(32 * kMergeRows),
                         0, stream, "attention merge launch", p, device_status_ptr());
  }
  if (p.kv_splits == 1) return r;
  const long long rows = static_cast<long long>(p.batch) * p.heads * p.lq;
  return launch_kernel(attn_combine_kernel<D, BF16>, dim3(static_cast<unsigned>((rows + 7) / 8)), dim3(256), 0,
                       stream, "attention combine launch", p);
}

}  // namespace
}  // namespace ldb

extern "C" {

static int flash_attention_impl(cudaStream_t stream, const void* q, int q_ld, const void* k, const void* v,
                                int kv_ld, void* out, int out_ld, int batch, int lq, int lk, int heads,
                                int head_dim, float scale, int dtype, void* workspace, size_t workspace_bytes,
                                unsigned long long* clock) {
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
  p.clock = clock;
  const int blocks = (lk + kBlockN - 1) / kBlockN;
  const long long ctas = static_cast<long long>((lq + 2 * kBlockM - 1) / (2 * kBlockM)) * heads * batch;
  p.kv_splits = 1;
  p.blocks_per_split = blocks;
  p.o_part = p.ml_part = nullptr;
  p.sk_ctas = 0;
  p.sk_nb = blocks;
  p.sk_pairs = (lq + 2 * kBlockM - 1) / (2 * kBlockM);
  p.sk_slots = 0;
  p.sk_units = 0;
  if (workspace) {
    const int splits = choose_kv_splits(ctas, blocks);
    const size_t rows = static_cast<size_t>(batch) * heads * lq;
    const size_t need = static_cast<size_t>(splits) * rows * (head_dim + 2) * sizeof(float);
    int slots = 0;
    const int sk = choose_stream_k(ctas, blocks, &slots);
    const size_t sk_rows = static_cast<size_t>(sk) * slots * 2 * kBlockM;
    if (splits > 1 && workspace_bytes >= need) {
      p.kv_splits = splits;
      p.blocks_per_split = (blocks + splits - 1) / splits;
      p.o_part = static_cast<float*>(workspace);
      p.ml_part = p.o_part + static_cast<size_t>(splits) * rows * head_dim;
    } else if (sk > 0 && workspace_bytes >= sk_rows * (head_dim + 2) * sizeof(float)) {
      p.sk_ctas = sk;
      p.sk_slots = slots;
      p.sk_units = ctas * blocks;
      p.o_part = static_cast<float*>(workspace);
      p.ml_part = p.o_part + sk_rows * head_dim;
    }
  }
  // Short keys (one key block) on a grid of more than one wave: a persistent
  // grid of one CTA per SM over the (query pair, head) units, in contiguous
  // ranges, so a CTA's set-up is paid once and its next unit's queries load
  // while it finishes the current one.  Every unit is whole: nothing to merge.
  if (p.sk_ctas == 0 && p.kv_splits == 1 && blocks == 1 && ctas > sm_count()) {
    p.sk_ctas = sm_count();
    p.sk_nb = 1;
    p.sk_units = ctas;
  }
  if (head_dim == 64) return bf16 ? launch_attn<64, true>(stream, qm, km, vm, p) : launch_attn<64, false>(stream, qm, km, vm, p);
  if (head_dim == 32) return bf16 ? launch_attn<32, true>(stream, qm, km, vm, p) : launch_attn<32, false>(stream, qm, km, vm, p);
  return bf16 ? launch_attn<16, true>(stream, qm, km, vm, p) : launch_attn<16, false>(stream, qm, km, vm, p);
}

int ldb_flash_attention(cudaStream_t stream, const void* q, int q_ld, const void* k, const void* v, int kv_ld,
                        void* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim, float scale,
                        int dtype) {
  return flash_attention_impl(stream, q, q_ld, k, v, kv_ld, out, out_ld, batch, lq, lk, heads, head_dim, scale, dtype,
                              nullptr, 0, nullptr);
}

int ldb_flash_attention_workspace_size(int batch, int lq, int lk, int heads, int head_dim, size_t* bytes) {
  using namespace ldb;
  if (!bytes) return fail(LDB_ERR_INVALID, "bytes is null");
  if (batch <= 0 || lq <= 0 || lk <= 0 || heads <= 0 || head_dim <= 0)
    return fail(LDB_ERR_SHAPE, "extents must be positive");
  const int blocks = (lk + kBlockN - 1) / kBlockN;
  const long long ctas = static_cast<long long>((lq + 2 * kBlockM - 1) / (2 * kBlockM)) * heads * batch;
  const int splits = choose_kv_splits(ctas, blocks);
  int slots = 0;
  const int sk = choose_stream_k(ctas, blocks, &slots);
  const size_t split_bytes =
      splits > 1 ? static_cast<size_t>(splits) * batch * heads * lq * (head_dim + 2) * sizeof(float) : 0;
  const size_t sk_bytes = static_cast<size_t>(sk) * slots * 2 * kBlockM * (head_dim + 2) * sizeof(float);
  *bytes = std::max(split_bytes, sk_bytes);
  return LDB_OK;
}

int ldb_flash_attention_ws(cudaStream_t stream, const void* q, int q_ld, const void* k, const void* v, int kv_ld,
                           void* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim, float scale,
                           int dtype, void* workspace, size_t workspace_bytes) {
  return flash_attention_impl(stream, q, q_ld, k, v, kv_ld, out, out_ld, batch, lq, lk, heads, head_dim, scale, dtype,
                              workspace, workspace_bytes, nullptr);
}

int ldb_flash_attention_timed(cudaStream_t stream, const void* q, int q_ld, const void* k, const void* v, int kv_ld,
                              void* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim, float scale,
                              int dtype, void* workspace, size_t workspace_bytes, unsigned long long* clock) {
  return flash_attention_impl(stream, q, q_ld, k, v, kv_ld, out, out_ld, batch, lq, lk, heads, head_dim, scale, dtype,
                              workspace, workspace_bytes, clock);
}

int ldb_flash_attention_f32_workspace_size(int batch, int lq, int lk, int heads, int head_dim, size_t* bytes) {
  using namespace ldb;
  if (!bytes) return fail(LDB_ERR_INVALID, "bytes is null");
  if (batch <= 0 || lq <= 0 || lk <= 0 || heads <= 0 || head_dim <= 0)
    return fail(LDB_ERR_SHAPE, "extents must be positive");
  // split planes of Q, K and V: (rows, heads * 2 * head_dim) f16 each, then
  // the stream-K partial rows (256-byte aligned)
  const size_t planes = static_cast<size_t>(batch) * (static_cast<size_t>(lq) + 2 * lk) * heads * head_dim * 2 * 2;
  const int blocks = (lk + kBlockN - 1) / kBlockN;
  const long long ctas = static_cast<long long>((lq + 2 * kBlockM - 1) / (2 * kBlockM)) * heads * batch;
  int slots = 0;
  const int sk = choose_stream_k(ctas, blocks, &slots);
  *bytes = (planes + 255) / 256 * 256 +
           static_cast<size_t>(sk) * slots * 2 * kBlockM * (head_dim + 2) * sizeof(float);
  return LDB_OK;
}

int ldb_flash_attention_f32(cudaStream_t stream, const float* q, int q_ld, const float* k, const float* v,
                            int kv_ld, float* out, int out_ld, int batch, int lq, int lk, int heads, int head_dim,
                            float scale, void* workspace, size_t workspace_bytes) {
  using namespace ldb;
  if (!q || !k || !v || !out || !workspace) return fail(LDB_ERR_INVALID, "flash_attention_f32: null pointer");
  if (head_dim != 16 && head_dim != 32 && head_dim != 64)
    return fail(LDB_ERR_SHAPE, "FP32 attention takes heads 16, 32 or 64 wide (got %d)", head_dim);
  if (batch <= 0 || lq <= 0 || lk <= 0 || heads <= 0) return fail(LDB_ERR_SHAPE, "extents must be positive");
  if (q_ld < heads * head_dim || kv_ld < heads * head_dim || out_ld < heads * head_dim)
    return fail(LDB_ERR_SHAPE, "row strides must cover heads * head_dim");
  if (q_ld % 4 || kv_ld % 4 || out_ld % 4) return fail(LDB_ERR_ALIGNMENT, "row strides must be multiples of 4");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) % 16)
    return fail(LDB_ERR_ALIGNMENT, "FP32 attention pointers must be 16-byte aligned");
  size_t need = 0;
  int rc = ldb_flash_attention_f32_workspace_size(batch, lq, lk, heads, head_dim, &need);
  if (rc != LDB_OK) return rc;
  if (workspace_bytes < need) return fail(LDB_ERR_WORKSPACE, "FP32 attention needs %zu workspace bytes", need);
  const int width = heads * head_dim * 2;  // split row width in f16
  __half* qs = static_cast<__half*>(workspace);
  __half* ks = qs + static_cast<size_t>(batch) * lq * width;
  __half* vs = ks + static_cast<size_t>(batch) * lk * width;
  const int threads = 256;
  const float log2e = 1.4426950408889634f;
  struct Part {
    const float* src;
    int ld;
    long long rows;
    float mul, lo_scale;
    __half* dst;
  } parts[3] = {{q, q_ld, static_cast<long long>(batch) * lq, scale * log2e, 1.0f, qs},
                {k, kv_ld, static_cast<long long>(batch) * lk, 1.0f, 1.0f, ks},
                {v, kv_ld, static_cast<long long>(batch) * lk, 1.0f, 2048.0f, vs}};
  for (const Part& pt : parts) {
    const long long n = pt.rows * heads * head_dim / 8;
    rc = launch_kernel(attn_split_kernel, dim3(static_cast<unsigned>((n + threads - 1) / threads)), dim3(threads), 0,
                       stream, "attention split launch", pt.src, pt.ld, pt.rows, heads, head_dim, pt.mul, pt.lo_scale,
                       pt.dst);
    if (rc != LDB_OK) return rc;
  }
  const uint32_t box[3] = {static_cast<uint32_t>(head_dim), 128u, 1u};
  CUtensorMap qm, km, vm;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(width), static_cast<uint64_t>(lq), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(width) * 2, static_cast<uint64_t>(lq) * width * 2};
    rc = encode_tiled_f16(&qm, qs, 3, dims, strides, box, head_dim * 2, false);
    if (rc != LDB_OK) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(width), static_cast<uint64_t>(lk), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(width) * 2, static_cast<uint64_t>(lk) * width * 2};
    rc = encode_tiled_f16(&km, ks, 3, dims, strides, box, head_dim * 2, false);
    if (rc != LDB_OK) return rc;
    rc = encode_tiled_f16(&vm, vs, 3, dims, strides, box, head_dim * 2, false);
    if (rc != LDB_OK) return rc;
  }
  AttnParams p;
  p.batch = batch;
  p.heads = heads;
  p.lq = lq;
  p.lk = lk;
  p.out_ld = out_ld;
  p.scale_log2 = 1.0f;  // Q carries scale * log2(e)
  p.out = out;
  p.kv_splits = 1;
  p.blocks_per_split = (lk + kBlockN - 1) / kBlockN;
  p.o_part = p.ml_part = nullptr;
  p.clock = nullptr;
  p.sk_nb = p.blocks_per_split;
  p.sk_pairs = (lq + 2 * kBlockM - 1) / (2 * kBlockM);
  {
    const long long ctas = static_cast<long long>(p.sk_pairs) * heads * batch;
    int slots = 0;
    p.sk_ctas = choose_stream_k(ctas, p.sk_nb, &slots);
    p.sk_slots = slots;
    p.sk_units = ctas * p.sk_nb;
    if (p.sk_ctas > 0) {
      const size_t planes = static_cast<size_t>(batch) * (static_cast<size_t>(lq) + 2 * lk) * width * 2;
      p.o_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + (planes + 255) / 256 * 256);
      p.ml_part = p.o_part + static_cast<size_t>(p.sk_ctas) * slots * 2 * kBlockM * head_dim;
    }
  }
  if (head_dim == 64) return launch_attn<64, false, true>(stream, qm, km, vm, p);
  if (head_dim == 16) return launch_attn<16, false, true>(stream, qm, km, vm, p);
  return launch_attn<32, false, true>(stream, qm, km, vm, p);
}

}  // extern "C"
