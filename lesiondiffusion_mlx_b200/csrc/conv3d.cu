// Implicit-GEMM 3-D convolution on sm_100a tensor cores (tcgen05 + TMEM).
//
// GEMM view: rows M are output voxels (source voxels for the folded 2x
// upsampling conv), columns N are output channels, and K runs over
// (tap, input-channel block).  Nothing is im2col'ed: for each K block a
// producer warp (two or four take the K blocks in turn) issues one 5-D TMA
// load of a bd x bh x bw brick of voxels x KC channels of the NDHWC
// activation, offset by the tap; TMA's out-of-bounds
// zero fill supplies the padding.  Weights are packed K-major
// [parity][Cout][tap][Cin] and loaded as 2-D TMA tiles.  A single thread of
// the MMA warp issues tcgen05.mma (M=128, N=BN, K=16) into a double-buffered
// TMEM accumulator; four epilogue warps drain TMEM (tcgen05.ld) in chunks of
// 128 output bytes per row, add bias + per-batch shift (staged once per
// tile in shared memory), scale, the residual (prefetched by TMA into
// shared memory), optional GELU, round once, write the chunk into a
// swizzled staging buffer and store it with one TMA tensor store (the
// folded upsampling conv stores through 8 output-parity views).  The kernel
// is persistent: CTA i walks tiles i, i+grid, ...
//
// FP32 "exact" mode follows the reference's split (hi = f16(v), lo =
// f16((v - hi) * 2^11)): per K step it issues hi*hi into one accumulator and
// hi*lo + lo*hi into a second, combined as acc0 + acc1 / 2048 in the
// epilogue, as in lesiondiffusion_mlx/_nax_conv.py:26-34 and :224-235.
//
// Split-K: when the output has too few tiles to fill the GPU, K is split
// into ranges computed by different CTAs; each stores raw f32 partial tiles
// and conv_reduce_kernel sums them and applies the epilogue, mirroring the
// reference's SPLIT/reduce kernels (_nax_conv.py:277-289, :556-563).

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "conv3d.cuh"
#include "host_common.h"

namespace ldb {

namespace {

// Warps: 0 and 6 .. 4 + P the P TMA producers, 1 the MMA issuer, 2-5 the epilogue.
constexpr int kTileM = 128;

struct TileCoord {
  int b, td, th, tw, par, nt, ks, out_tile;
};

__device__ __forceinline__ TileCoord decode_tile(const ConvParams& p, int t) {
  TileCoord c;
  c.ks = t % p.k_splits;
  t /= p.k_splits;
  c.out_tile = t;
  c.nt = t % p.n_tiles;
  t /= p.n_tiles;
  c.par = t % p.parities;
  t /= p.parities;
  c.tw = t % p.tiles_w;
  t /= p.tiles_w;
  c.th = t % p.tiles_h;
  t /= p.tiles_h;
  c.td = t % p.tiles_d;
  c.b = t / p.tiles_d;
  return c;
}

// Tile index (as decode_tile reads it) that CTA `rank` of a pair computes for
// work unit u = (pair q, column tile, K range).  A pair shares its weight
// operand, so its two row tiles are two spatial bricks of the same output
// parity (the folded upsampling conv has one weight set per parity): pair q
// = (spatial pair qs, parity) takes bricks 2 qs and 2 qs + 1.  Past the last
// brick the index decodes to batch index p.batch (a placeholder).
__device__ __forceinline__ int pair_tile(const ConvParams& p, int u, int rank) {
  const int ks = u % p.k_splits;
  const int r = u / p.k_splits;
  const int nt = r % p.n_tiles;
  const int q = r / p.n_tiles;
  const int par = q % p.parities;
  const int brick = 2 * (q / p.parities) + rank;
  return ((brick * p.parities + par) * p.n_tiles + nt) * p.k_splits + ks;
}

// Output voxel (linear NDHW index) of GEMM row `r` of a tile, or -1 when
// the row falls outside the brick or the volume.
__device__ __forceinline__ long long row_voxel(const ConvParams& p, const TileCoord& c, int r) {
  const int brick = p.bw * p.bh * p.bd;
  if (r >= brick || c.b >= p.batch) return -1;  // b == batch: a pair's placeholder tile
  const int lw = r % p.bw;
  const int lh = (r / p.bw) % p.bh;
  const int ld = r / (p.bw * p.bh);
  int w = c.tw * p.bw + lw;
  int h = c.th * p.bh + lh;
  int d = c.td * p.bd + ld;
  if (w >= p.grid_w || h >= p.grid_h || d >= p.grid_d) return -1;
  if (p.mode == kConvUp2) {
    d = 2 * d + (c.par >> 2);
    h = 2 * h + ((c.par >> 1) & 1);
    w = 2 * w + (c.par & 1);
  }
  return ((static_cast<long long>(c.b) * p.out_d + d) * p.out_h + h) * p.out_w + w;
}

// Apply the epilogue to `n` consecutive output channels starting at `col`
// of one voxel and store them.  `v` holds the f32 GEMM sums on entry and the
// values as stored (after the output rounding) on return.
template <int N>
__device__ __forceinline__ void store_outputs(const ConvParams& p, int b, long long voxel, int col, float (&v)[N]) {
  const bool full = (col + N <= p.cout);
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const int c = col + j;
    float y = v[j];
    if (c < p.cout) {
      float add = p.bias ? p.bias[c] : 0.0f;
      if (p.shift) add += p.shift[static_cast<long long>(b) * p.cout + c];
      y = (y + add) * p.out_scale;
    }
    v[j] = y;
  }
  if (p.residual) {
    if (p.out_f32) {
      const float* res = static_cast<const float*>(p.residual) + voxel * p.res_ld + col;
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (col + j < p.cout) v[j] += res[j];
    } else {
      const __half* res = static_cast<const __half*>(p.residual) + voxel * p.res_ld + col;
      if (full && (p.res_ld % 8) == 0 && (col % 8) == 0 && (N % 8) == 0) {
#pragma unroll
        for (int j = 0; j < N; j += 8) {
          uint4 raw = *reinterpret_cast<const uint4*>(res + j);
          const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float2 f = __half22float2(h2[q]);
            v[j + 2 * q] += f.x;
            v[j + 2 * q + 1] += f.y;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < N; ++j)
          if (col + j < p.cout) v[j] += __half2float(res[j]);
      }
    }
  }
  if (p.act == kActGelu) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      // The reference rounds the dense output to the activation dtype before
      // its FP32 GELU (mlx_model.py:369-374 after :204-217).
      float y = p.out_f32 ? v[j] : __half2float(__float2half_rn(v[j]));
      v[j] = gelu_erf_f32(y);
    }
  }
  if (p.out_f32) {
    float* o = static_cast<float*>(p.out) + voxel * p.out_ld + col;
    if (full && (p.out_ld % 4) == 0 && (col % 4) == 0 && (N % 4) == 0) {
#pragma unroll
      for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (col + j < p.cout) o[j] = v[j];
    }
  } else {
    __half* o = static_cast<__half*>(p.out) + voxel * p.out_ld + col;
    if (full && (p.out_ld % 8) == 0 && (col % 8) == 0 && (N % 8) == 0) {
#pragma unroll
      for (int j = 0; j < N; j += 8) {
        uint4 raw;
        __half2* h2 = reinterpret_cast<__half2*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          h2[q] = __floats2half2_rn(v[j + 2 * q], v[j + 2 * q + 1]);
          const float2 f = __half22float2(h2[q]);
          v[j + 2 * q] = f.x;
          v[j + 2 * q + 1] = f.y;
        }
        *reinterpret_cast<uint4*>(o + j) = raw;
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const __half h = __float2half_rn(v[j]);
        v[j] = __half2float(h);
        if (col + j < p.cout) o[j] = h;
      }
    }
  }
}

// TRANS: channel-major tile (activation rows are the MMA's N operand, up to
// 256 voxels; the weight tile is the M = 128 operand).
template <int KC, int BN, bool EXACT, bool TRANS = false, bool PAIR = false>
struct ConvCfg {
  static constexpr int kSwizzleBytes = KC * 2;  // one K block row = 32/64/128 B
  static constexpr uint32_t kLayout = KC == 64 ? kSwizzle128 : (KC == 32 ? kSwizzle64 : kSwizzle32);
  static constexpr uint32_t kSbo = 8 * KC * 2;  // bytes between 8-row groups
  static constexpr int kPlanes = EXACT ? 2 : 1;
  static constexpr int kRowsA = TRANS ? 192 : kTileM;  // activation rows per stage (bricks of <= 3 planes)
  static constexpr int kABytes = kRowsA * KC * 2;
  // PAIR: this CTA stages half of the BN weight rows (the peer the other half).
  static constexpr int kBRows = PAIR ? BN / 2 : BN;
  static constexpr int kBBytesRaw = kBRows * KC * 2;
  static constexpr int kBBytes = ((kBBytesRaw + 1023) / 1024) * 1024;
  static constexpr int kStageBytes = kPlanes * (kABytes + kBBytes);
  // Epilogue staging: output + 2 residual buffers of 128 rows x 128 bytes;
  // 2 output buffers in the voxel-major tile.  The channel-major tile keeps
  // one (a tile's few planes of stores drain well within its main loop), so
  // its ring holds a fourth stage: with ~1.2 us per TMA round trip the
  // bytes in flight bound that pipeline.
  static constexpr int kEpiBufBytes = kTileM * 128;
  // (Paired tiles keep two: their grids are mostly one work unit per CTA, so
  // the epilogue is the CTA's tail, not hidden behind a next tile's main loop;
  // one buffer and a fifth ring stage measured 4-8 % slower.)
  static constexpr int kOutBufs = TRANS ? 1 : 2;
  static constexpr int kEpiBytes = (kOutBufs + 2) * kEpiBufBytes;
  // Per-CTA GroupNorm statistics accumulator: [BN][2] FP32 shifted sums
  // (the channel-major tile keeps its sums in registers).
  static constexpr int kStatsBytes = TRANS ? 0 : BN * 8;
  static constexpr int kStagesRaw = (225 * 1024 - kEpiBytes - 2048 - kStatsBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  // Producer warps taking K blocks in turn: four where K blocks are small
  // (16 / 32 channels: the MMA issuer keeps up with more), else two.
  static constexpr int kProducers = KC < 64 && kStages >= 4 ? 4 : 2;
  static constexpr int kThreads = 32 * (5 + kProducers);
  // Two accumulator chains (even / odd K steps, added in the epilogue): the
  // tensor pipe overlaps MMAs into different accumulators but serialises
  // successive MMAs into one, which at N <= 128 leaves it idle about half of
  // the time.  Used where TMEM holds 2 chains x 2 tile buffers.
  static constexpr int kChains = (!EXACT && !TRANS && KC >= 32 && 4 * BN <= 512) ? 2 : 1;
  static constexpr int kAccCols = TRANS ? 256 : BN * kPlanes * kChains;
  static constexpr int kTmemColsRaw = 2 * kAccCols;
  static constexpr int kTmemCols = kTmemColsRaw < 32 ? 32 : kTmemColsRaw;
  // Output element size (f32 in exact mode, f16 otherwise) and the columns
  // per epilogue chunk: one 128-byte row (at most BN).
  static constexpr int kOutBytes = EXACT ? 4 : 2;
  static constexpr int kOutChunk = (128 / kOutBytes) < BN ? (128 / kOutBytes) : BN;
  static constexpr int kPartChunk = 32 < BN ? 32 : BN;  // split-K partials are f32
  static constexpr uint32_t kIdesc = make_idesc_f16(PAIR ? 2 * kTileM : kTileM, BN, 0, 0, 0);
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2], drain, res_full[2]
  static constexpr int kBarrierBytes = (2 * kStages + 7) * 8;
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kEpiBytes + 1024 /*align slack*/ + kBarrierBytes + 64 + BN * 4 + kStatsBytes;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
  static_assert(!TRANS || (BN == 128 && !EXACT), "channel-major tiles are f16 with 128 channel rows");
  static_assert(!PAIR || (BN == 256 && !EXACT && !TRANS), "CTA pairs run the f16 voxel-major 256-column tile");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget exceeded");
};

// Per-thread state of the epilogue warps, carried across tiles.
struct EpiState {
  uint8_t* epi;          // out staging [2] then residual staging [2], 128 rows x 128 B each
  uint64_t* res_full;    // [2]
  float* bsum;           // [BN]
  uint32_t* vmask;       // [2][4] valid-row bits of the current tile (double-buffered by tile)
  float* sacc;           // [BN][2] sums of (x - bsum) and (x - bsum)^2 over the current run of tiles
  int key_b = -1;        // (batch, column tile) of the run: tiles of one run share bsum
  int key_nt = -1;
  int run_rows = 0;      // valid rows (voxels) accumulated in the run
  float run_s1 = 0.f;    // channel-major tile: this thread's channel sums of x - k, (x - k)^2
  float run_s2 = 0.f;
  float run_k = 0.f;
  volatile int* abort_flag;
  unsigned int* status;
  int quarter, row;
  bool leader;
  uint32_t oq = 0;               // output chunks issued (staging buffer parity)
  uint32_t rq = 0;               // residual chunks consumed
  uint32_t res_uses0 = 0;        // completed phases of residual buffer 0
  uint32_t res_uses1 = 0;        // ... and of buffer 1
  uint32_t tiles = 0;            // tiles started (valid-row mask parity)
};

// GroupNorm statistics of one staged output chunk (the values exactly as
// stored).  Each thread owns one 4-byte word of the staged rows (two f16 or
// one f32 column) over its part of the tile's rows, loads 8 rows at a time
// and sums the valid rows' x - k and (x - k)^2 in FP32, k being the column's
// bias + shift (constant over a run of tiles, and close to the column mean,
// so the shifted sums keep the variance from cancelling).  The parts fold
// into the CTA's accumulator with shared-memory FP32 atomics.
template <int CC, int kElem>
__device__ __forceinline__ void chunk_stats(const ConvParams& p, int n0, int c0, const uint8_t* ob,
                                            const uint32_t* vmask, const float* bsum, float* sacc) {
  constexpr uint32_t kRowBytes = CC * kElem;
  constexpr int kThreadsPerRow = kRowBytes / 4;
  constexpr int kColsPer = 4 / kElem;
  constexpr int kParts = 128 / kThreadsPerRow;
  constexpr int kRows = kTileM / kParts;  // 8, 16 or 32
  const int et = threadIdx.x - 64;
  const int w = et % kThreadsPerRow;
  const int part = et / kThreadsPerRow;
  const int jt = c0 + w * kColsPer;  // first column within the tile
  if (n0 + jt >= p.cout) return;
  const int r0 = part * kRows;
  const uint32_t bits = (vmask[r0 >> 5] >> (r0 & 31)) & (kRows == 32 ? 0xffffffffu : ((1u << kRows) - 1u));
  if (bits == 0) return;
  float k[kColsPer], s1[kColsPer], s2[kColsPer];
#pragma unroll
  for (int q = 0; q < kColsPer; ++q) {
    k[q] = bsum[jt + q];
    s1[q] = s2[q] = 0.f;
  }
#pragma unroll 1
  for (int i0 = 0; i0 < kRows; i0 += 8) {
    uint32_t words[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      words[u] = *reinterpret_cast<const uint32_t*>(
          ob + swizzle_offset(static_cast<uint32_t>(r0 + i0 + u) * kRowBytes + w * 4, kRowBytes));
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if ((bits >> (i0 + u)) & 1u) {
        float x[kColsPer];
        if constexpr (kElem == 4) {
          x[0] = __uint_as_float(words[u]);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&words[u]));
          x[0] = f.x;
          x[1] = f.y;
        }
#pragma unroll
        for (int q = 0; q < kColsPer; ++q) {
          const float d = x[q] - k[q];
          s1[q] += d;
          s2[q] = fmaf(d, d, s2[q]);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kColsPer; ++q) {
    if (n0 + jt + q >= p.cout) break;
    atomicAdd(&sacc[(jt + q) * 2], s1[q]);
    atomicAdd(&sacc[(jt + q) * 2 + 1], s2[q]);
  }
}

// Add the CTA's statistics of the finished run (key_b, key_nt) to the global
// FP64 totals, one add pair per column: sum = S1 + n k and sum of squares =
// S2 + 2 k S1 + n k^2 with k the run's bias + shift (still in bsum), then
// optionally clear the accumulator.  Called by the 128 epilogue threads
// after a named barrier.
template <int BN>
__device__ __forceinline__ void flush_stats(const ConvParams& p, const EpiState& st, bool clear) {
  for (int j = threadIdx.x - 64; j < BN; j += 128) {
    if (st.key_b >= 0 && st.run_rows > 0) {
      const int col = st.key_nt * BN + j;
      if (col < p.cout) {
        const double n = st.run_rows;
        const double k = st.bsum[j];
        const double s1 = st.sacc[2 * j], s2 = st.sacc[2 * j + 1];
        double* dst = p.stats + (static_cast<long long>(st.key_b) * p.cout + col) * 2;
        red_add_f64(dst, s1 + n * k);
        red_add_f64(dst + 1, s2 + 2.0 * k * s1 + n * k * k);
      }
    }
    if (clear) {
      st.sacc[2 * j] = 0.f;
      st.sacc[2 * j + 1] = 0.f;
    }
  }
}

// One output tile: wait for its accumulator, then per chunk of CC columns
// TMEM -> registers -> (bias + shift) * scale + residual -> GELU -> round ->
// swizzled staging row -> one TMA store by the leader.  With SPLIT the raw
// f32 partial sums are stored instead (the reduce kernel applies the rest).
template <class Cfg, int BN, bool EXACT, int CC, bool SPLIT>
__device__ __forceinline__ bool epilogue_tile(const ConvParams& p, const ConvMaps& maps, const TileCoord& c,
                                              uint32_t tbase, uint64_t* acc_full_bar, uint32_t acc_parity,
                                              EpiState& st) {
  constexpr int kElem = SPLIT ? 4 : Cfg::kOutBytes;
  constexpr uint32_t kRowBytes = CC * kElem;  // 32, 64 or 128
  constexpr int kPerUnit = 16 / kElem;        // elements per 16-byte unit
  constexpr int kChunks = BN / CC;
  const int et = threadIdx.x - 64;
  const int w0 = c.tw * p.bw, h0 = c.th * p.bh, d0 = c.td * p.bd;
  const int omap = p.mode == kConvUp2 ? c.par : 0;
  const int n0 = c.nt * BN;
  // A pair's placeholder tile (batch index past the end) drains its
  // accumulator like any tile but reads and writes nothing in global memory.
  const bool real = c.b < p.batch;
  const bool has_res = !SPLIT && p.residual != nullptr && real;
  const uint32_t res_bytes = kRowBytes * static_cast<uint32_t>(p.bw * p.bh * p.bd);
  uint8_t* const res_base = st.epi + Cfg::kOutBufs * Cfg::kEpiBufBytes;  // residual buffer rb at res_base + rb * kEpiBufBytes
  if (has_res && st.leader) {
    // prefetch the residual of chunk 0 while the tile's MMAs still run
    const int rb = st.rq & 1;
    mbar_arrive_expect_tx(&st.res_full[rb], res_bytes);
    tma_load_5d(res_base + rb * Cfg::kEpiBufBytes, &maps.r[omap], &st.res_full[rb], n0, w0, h0, d0, c.b);
  }
  // Never leave early: the four epilogue warps must reach the same sequence
  // of named barriers.  After a timeout the waits below fail fast (the abort
  // flag is set) and the tile is written with whatever TMEM holds.
  uint32_t* vmask = st.vmask + (st.tiles & 1) * 4;
  st.tiles += 1;
  if (!SPLIT && p.stats) {
    if (c.b != st.key_b || c.nt != st.key_nt) {
      // a new (batch, column tile): hand the previous run's sums to the totals
      named_barrier(1, 128);
      flush_stats<BN>(p, st, true);
      st.key_b = c.b;
      st.key_nt = c.nt;
      st.run_rows = 0;
    }
    const unsigned int valid = __ballot_sync(0xffffffffu, row_voxel(p, c, st.row) >= 0);
    if ((st.row & 31) == 0) vmask[st.quarter] = valid;
  }
  // bias + shift of the tile's columns, read while the MMAs still run (the
  // previous run's statistics were flushed above with its own values)
  if (!SPLIT) {
    for (int j = et; j < BN; j += 128) {
      const int col = n0 + j;
      float add = 0.f;
      if (col < p.cout && real) {
        if (p.bias) add = p.bias[col];
        if (p.shift) add += p.shift[static_cast<long long>(c.b) * p.cout + col];
      }
      st.bsum[j] = add;
    }
  }
  bool ok = warp_wait(acc_full_bar, acc_parity, st.abort_flag, st.status);
  tc_fence_after();
  named_barrier(1, 128);
  if (!SPLIT && p.stats)  // every thread counts the tile's valid rows (the masks are visible after the barrier)
    st.run_rows += static_cast<int>(__popc(vmask[0]) + __popc(vmask[1]) + __popc(vmask[2]) + __popc(vmask[3]));
  const uint32_t rowoff = static_cast<uint32_t>(st.row) * kRowBytes;
#pragma unroll 1
  for (int q = 0; q < kChunks; ++q) {
    uint8_t* ob = st.epi + (Cfg::kOutBufs == 2 ? (st.oq & 1) * Cfg::kEpiBufBytes : 0);
    if (st.leader) {
      // the store issued kOutBufs chunks ago has read this buffer
      if constexpr (Cfg::kOutBufs == 2) {
        bulk_wait_group_read<1>();
      } else {
        bulk_wait_group_read<0>();
      }
      if (has_res && q + 1 < kChunks) {
        const int rb = (st.rq + 1) & 1;
        mbar_arrive_expect_tx(&st.res_full[rb], res_bytes);
        tma_load_5d(res_base + rb * Cfg::kEpiBufBytes, &maps.r[omap], &st.res_full[rb], n0 + (q + 1) * CC, w0, h0,
                    d0, c.b);
      }
    }
    named_barrier(1, 128);
    const int c0 = q * CC;
    float v[CC];
#pragma unroll
    for (int s16 = 0; s16 < CC / 16; ++s16) {
      uint32_t r[16];
      tmem_ld16(tbase + c0 + s16 * 16, r);
      if constexpr (EXACT) {
        uint32_t lo[16];
        tmem_ld16(tbase + BN + c0 + s16 * 16, lo);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[s16 * 16 + j] = __uint_as_float(r[j]) + __uint_as_float(lo[j]) * (1.0f / 2048.0f);
      } else if constexpr (Cfg::kChains == 2) {
        uint32_t odd[16];
        tmem_ld16(tbase + BN + c0 + s16 * 16, odd);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[s16 * 16 + j] = __uint_as_float(r[j]) + __uint_as_float(odd[j]);
      } else {
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[s16 * 16 + j] = __uint_as_float(r[j]);
      }
    }
    if constexpr (SPLIT) {
#pragma unroll
      for (int u = 0; u < CC / 4; ++u) {
        *reinterpret_cast<float4*>(ob + swizzle_offset(rowoff + u * 16, kRowBytes)) =
            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
      }
    } else {
      const uint8_t* rbuf = nullptr;
      if (has_res) {
        const int rb = st.rq & 1;
        uint32_t& uses = rb ? st.res_uses1 : st.res_uses0;
        if (!mbar_wait(&st.res_full[rb], uses & 1, st.abort_flag, st.status)) ok = false;
        uses += 1;
        st.rq += 1;
        rbuf = res_base + rb * Cfg::kEpiBufBytes;
      }
      // Every shared-memory read of the chunk (bias + shift, the residual)
      // comes before its first staging store: the compiler cannot tell the
      // staging buffer from those arrays, and loads interleaved with stores
      // would run one after another.
#pragma unroll
      for (int j = 0; j < CC; ++j) v[j] = (v[j] + st.bsum[c0 + j]) * p.out_scale;
      if (rbuf) {
#pragma unroll
        for (int u = 0; u < CC / kPerUnit; ++u) {
          const uint32_t off = swizzle_offset(rowoff + u * 16, kRowBytes);
          if constexpr (EXACT) {
            const float4 rr = *reinterpret_cast<const float4*>(rbuf + off);
            v[4 * u] += rr.x;
            v[4 * u + 1] += rr.y;
            v[4 * u + 2] += rr.z;
            v[4 * u + 3] += rr.w;
          } else {
            const uint4 raw = *reinterpret_cast<const uint4*>(rbuf + off);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __half22float2(h2[j]);
              v[8 * u + 2 * j] += f.x;
              v[8 * u + 2 * j + 1] += f.y;
            }
          }
        }
      }
      if (p.act == kActGelu) {
#pragma unroll
        for (int j = 0; j < CC; ++j) {
          // The reference rounds the dense output to the activation dtype
          // before its FP32 GELU (mlx_model.py:369-374 after :204-217).
          const float z = EXACT ? v[j] : __half2float(__float2half_rn(v[j]));
          v[j] = gelu_erf_f32(z);
        }
      }
#pragma unroll
      for (int u = 0; u < CC / kPerUnit; ++u) {
        const uint32_t off = swizzle_offset(rowoff + u * 16, kRowBytes);
        if constexpr (EXACT) {
          *reinterpret_cast<float4*>(ob + off) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        } else {
          uint4 raw;
          __half2* h2 = reinterpret_cast<__half2*>(&raw);
#pragma unroll
          for (int j = 0; j < 4; ++j) h2[j] = __floats2half2_rn(v[8 * u + 2 * j], v[8 * u + 2 * j + 1]);
          *reinterpret_cast<uint4*>(ob + off) = raw;
        }
      }
    }
    fence_proxy_async_smem();
    named_barrier(1, 128);
    if (st.leader && real) {
      if constexpr (SPLIT) {
        const int prow = (c.ks * (p.num_tiles / p.k_splits) + c.out_tile) * kTileM;
        tma_store_2d(&maps.part, ob, c0, prow);
      } else {
        tma_store_5d(&maps.o[omap], ob, n0 + c0, w0, h0, d0, c.b);
      }
      bulk_commit_group();
    }
    if constexpr (!SPLIT) {
      if (p.stats) chunk_stats<CC, kElem>(p, n0, c0, ob, vmask, st.bsum, st.sacc);
    }
    st.oq += 1;
  }
  return ok;
}

// Channel-major tile: TMEM lane = output channel (the warp with quarter q
// owns channels 32q .. 32q + 31), column = voxel of the bd x 8 x 8 brick, so
// each depth plane of the brick is 64 consecutive columns.  Per plane: load
// the plane's 64 sums of this thread's channel, add bias + shift, scale, the
// residual (TMA-prefetched plane, read transposed), optional GELU, round
// once, write each value into the swizzled staging rows [voxel][channel],
// and store the plane with one TMA store per 64 channels.  GroupNorm
// statistics: the thread owns one channel, so it sums x - k and (x - k)^2
// over the run's valid voxels in registers (k = its bias + shift) and adds
// FP64 totals when the batch item changes or the CTA ends.
__device__ __forceinline__ void flush_trans_stats(const ConvParams& p, EpiState& st) {
  if (st.key_b >= 0 && st.run_rows > 0 && st.row < p.cout) {
    const double n = st.run_rows, k = st.run_k, s1 = st.run_s1, s2 = st.run_s2;
    double* dst = p.stats + (static_cast<long long>(st.key_b) * p.cout + st.row) * 2;
    red_add_f64(dst, s1 + n * k);
    red_add_f64(dst + 1, s2 + 2.0 * k * s1 + n * k * k);
  }
  st.run_rows = 0;
  st.run_s1 = st.run_s2 = 0.f;
}

template <class Cfg>
__device__ __forceinline__ bool epilogue_tile_trans(const ConvParams& p, const ConvMaps& maps, const TileCoord& c,
                                                    uint32_t tbase, uint64_t* acc_full_bar, uint32_t acc_parity,
                                                    EpiState& st) {
  const int ch = st.row;  // output channel of this thread (one column tile: n0 = 0)
  const bool live = ch < p.cout;
  const int w0 = c.tw * 8, h0 = c.th * 8, d0 = c.td * p.bd;
  const int omap = p.mode == kConvUp2 ? c.par : 0;
  const int nboxes = (p.cout + 63) / 64;
  constexpr uint32_t kBoxBytes = 64 * 128;  // 64 voxels x 64 channels x 2 B
  const uint32_t res_bytes = static_cast<uint32_t>(nboxes) * kBoxBytes;
  const bool has_res = p.residual != nullptr;
  uint8_t* const res_base = st.epi + Cfg::kOutBufs * Cfg::kEpiBufBytes;
  auto prefetch_res = [&](int pl, int rb) {
    mbar_arrive_expect_tx(&st.res_full[rb], res_bytes);
    for (int bx = 0; bx < nboxes; ++bx)
      tma_load_5d(res_base + rb * Cfg::kEpiBufBytes + bx * kBoxBytes, &maps.r[omap], &st.res_full[rb], bx * 64, w0,
                  h0, d0 + pl, c.b);
  };
  if (has_res && st.leader) prefetch_res(0, st.rq & 1);
  // valid voxels of a plane of this brick: lh < nh and lw < nw
  const int nh = min(8, p.grid_h - h0), nw = min(8, p.grid_w - w0);
  uint64_t plane_mask = 0;
  for (int lh = 0; lh < nh; ++lh) plane_mask |= ((nw >= 8 ? 0xffull : ((1ull << nw) - 1))) << (8 * lh);
  float add = 0.f;
  if (live) {
    if (p.bias) add = p.bias[ch];
    if (p.shift) add += p.shift[static_cast<long long>(c.b) * p.cout + ch];
  }
  if (p.stats && c.b != st.key_b) {
    flush_trans_stats(p, st);
    st.key_b = c.b;
    st.key_nt = 0;
    st.run_k = add;
  }
  bool ok = warp_wait(acc_full_bar, acc_parity, st.abort_flag, st.status);
  tc_fence_after();
  const uint32_t col_off = static_cast<uint32_t>(ch & 63) * 2;
  const uint32_t box_off = static_cast<uint32_t>(ch >> 6) * kBoxBytes;
#pragma unroll 1
  for (int pl = 0; pl < p.bd; ++pl) {
    uint8_t* ob = st.epi;
    if (st.leader) {
      bulk_wait_group_read<0>();  // the previous plane's stores have read the staging buffer
      if (has_res && pl + 1 < p.bd) prefetch_res(pl + 1, (st.rq + 1) & 1);
    }
    named_barrier(1, 128);
    float v[64];
    {
      uint32_t r0[32], r1[32];
      tmem_ld32(tbase + pl * 64, r0);
      tmem_ld32(tbase + pl * 64 + 32, r1);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __uint_as_float(r0[j]);
        v[32 + j] = __uint_as_float(r1[j]);
      }
      if (p.trans_chains == 2) {  // odd K steps accumulated 128 columns further
        tmem_ld32(tbase + 128 + pl * 64, r0);
        tmem_ld32(tbase + 128 + pl * 64 + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] += __uint_as_float(r0[j]);
          v[32 + j] += __uint_as_float(r1[j]);
        }
      }
    }
    const uint8_t* rbuf = nullptr;
    if (has_res) {
      const int rb = st.rq & 1;
      uint32_t& uses = rb ? st.res_uses1 : st.res_uses0;
      if (!mbar_wait(&st.res_full[rb], uses & 1, st.abort_flag, st.status)) ok = false;
      uses += 1;
      st.rq += 1;
      rbuf = res_base + rb * Cfg::kEpiBufBytes;
    }
    const bool dvalid = d0 + pl < p.grid_d;
    // Each step is its own straight loop with the optional parts (residual,
    // GELU, statistics) branched around as a whole: a per-value branch over
    // an inlined GELU spreads the 64 executed iterations over tens of KB of
    // code, and the instruction fetch, not the arithmetic, then sets the
    // per-plane time.
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = (v[j] + add) * p.out_scale;
    if (rbuf) {  // all residual reads before the first staging store (see epilogue_tile)
#pragma unroll
      for (int j = 0; j < 64; ++j)
        v[j] += __half2float(*reinterpret_cast<const __half*>(
            rbuf + box_off + swizzle_offset(static_cast<uint32_t>(j) * 128 + col_off, 128)));
    }
    if (p.act == kActGelu) {
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = gelu_erf_f32(__half2float(__float2half_rn(v[j])));
    }
    if (live) {  // round once; the statistics below read the rounded values
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const __half h = __float2half_rn(v[j]);
        v[j] = __half2float(h);
        *reinterpret_cast<__half*>(ob + box_off + swizzle_offset(static_cast<uint32_t>(j) * 128 + col_off, 128)) = h;
      }
      if (p.stats && dvalid) {
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float d = ((plane_mask >> j) & 1ull) ? v[j] - st.run_k : 0.f;
          s1 += d;
          s2 = fmaf(d, d, s2);
        }
        st.run_s1 += s1;
        st.run_s2 += s2;
        st.run_rows += __popcll(plane_mask);
      }
    }
    fence_proxy_async_smem();
    named_barrier(1, 128);
    if (st.leader) {
      for (int bx = 0; bx < nboxes; ++bx)
        tma_store_5d(&maps.o[omap], ob + bx * kBoxBytes, bx * 64, w0, h0, d0 + pl, c.b);
      bulk_commit_group();
    }
    st.oq += 1;
  }
  return ok;
}

template <int KC, int BN, bool EXACT, bool TRANS, bool PAIR>
__global__ void __launch_bounds__(ConvCfg<KC, BN, EXACT, TRANS, PAIR>::kThreads, 1)
    conv3d_tc_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ CUtensorMap wmap,
                     const ConvParams p, unsigned int* status) {
  using Cfg = ConvCfg<KC, BN, EXACT, TRANS, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = smem + Cfg::kStages * Cfg::kStageBytes;  // out[kOutBufs] | res[2], 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + Cfg::kEpiBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* acc_full = empty + Cfg::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* res_full = drain + 1;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* vmask = tmem_slot + 4;                          // [2][4]
  float* bsum = reinterpret_cast<float*>(tmem_slot + 16);  // [BN] bias + shift of the current tile
  float* sacc = bsum + BN;                                  // [BN][2] GroupNorm statistics

  const int warp = warp_id();
  const int lane = lane_id();
  // Work: without pairs CTA i takes tiles i, i + grid, ...; with pairs the
  // cluster (two CTAs) takes units j, j + grid / 2, ... and CTA `rank` of it
  // computes the unit's row tile 2q + rank.
  const int rank = PAIR ? static_cast<int>(cluster_ctarank()) : 0;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int units = PAIR ? p.num_units : p.num_tiles;
  auto tile_of = [&](int u) { return PAIR ? pair_tile(p, u, rank) : u; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      // with pairs the leader's accumulator is free once both CTAs' epilogues have read it
      mbar_init(&acc_empty[a], PAIR ? 8 : 4);
    }
    mbar_init(drain, 1);
    mbar_init(&res_full[0], 1);
    mbar_init(&res_full[1], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&wmap);
    const int nmaps = (p.mode == kConv3x3x3S2 || p.mode == kConv3x3x3S2Pad01) ? 8 : 1;
    for (int i = 0; i < nmaps; ++i) tma_prefetch_desc(&maps.a[i]);
  }
  if (warp == 2 && lane == 0) {
    const int nout = p.mode == kConvUp2 ? 8 : 1;
    if (p.k_splits > 1) {
      tma_prefetch_desc(&maps.part);
    } else {
      for (int i = 0; i < nout; ++i) tma_prefetch_desc(&maps.o[i]);
      if (p.residual)
        for (int i = 0; i < nout; ++i) tma_prefetch_desc(&maps.r[i]);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or load
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the next kernel may be scheduled at once;
  // each thread that touches global memory the previous kernel may write
  // waits for it first.  The producer waits only right before its first TMA
  // load, so its first tile's arithmetic (and the instruction fetch of that
  // code) overlaps the previous kernel's tail; the MMA warp reads only shared
  // memory and TMEM and never waits.
  pdl_trigger();

  const uint32_t a_box_bytes = static_cast<uint32_t>(KC * 2 * p.bw * p.bh * p.bd);
  const uint32_t tx_bytes = Cfg::kPlanes * (a_box_bytes + static_cast<uint32_t>(Cfg::kBBytesRaw));

  if (warp == 0 || warp >= 6) {
    // ------------------------------------------------------------ producers
    // P producer warps (0, then 6 and up) take the K blocks of the CTA's
    // sequence (flattened over its tiles) in turn: K block j goes to
    // producer j % P and to stage j % kStages.  Per K block one thread waits
    // for the stage, arms it and issues the loads, a path of some hundred
    // cycles of dependent latency that sets the pipeline's rate when it runs
    // on one thread; P run it side by side.
    constexpr int P = Cfg::kProducers;
    static_assert(P <= Cfg::kStages, "a producer's next stage must differ from its current one");
    if (lane == 0) {
      const int pid = warp == 0 ? 0 : warp - 5;
      int stage = pid;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_parity = 0;
      bool waited = false;
      int jt = 0;  // sequence index of the current tile's first K block, mod P
      for (int u = unit0; u < units && !*abort_flag; u += unit_step) {
        const TileCoord c = decode_tile(p, tile_of(u));
        const int kb0 = c.ks * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int w0 = c.tw * p.bw, h0 = c.th * p.bh, d0 = c.td * p.bd;
        const int pd = c.par >> 2, ph = (c.par >> 1) & 1, pw = c.par & 1;
        // (a pair's CTA r stages weight rows [128 r, 128 r + 128) of the column tile)
        const int brow = c.par * p.wrows_per_parity + c.nt * BN + rank * Cfg::kBRows;
        int kb = kb0 + (pid - jt + P) % P;  // this producer's first K block of the tile
        jt = (jt + kb1 - kb0) % P;
        if (kb >= kb1) continue;
        bool ok = true;
        // Tap digits (kd, kh, kw; for the folded up-conv the bits td, th, tw)
        // and channel chunk of kb, then advanced P K blocks at a time by
        // counters (no division per K block).  The weight column of K block kb
        // is kb * KC (tap * cin_pad + chunk * KC).
        int chunk, kd, kh, kw;
        {
          const int tap = kb / p.cin_chunks;
          chunk = kb - tap * p.cin_chunks;
          if (p.mode == kConvUp2) {
            kd = tap >> 2;
            kh = (tap >> 1) & 1;
            kw = tap & 1;
          } else {
            kd = tap / 9;
            kh = (tap / 3) % 3;
            kw = tap % 3;
          }
        }
        const int zb = d0 + p.in_zoff;
        for (; kb < kb1; kb += P) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kPlanes * Cfg::kABytes;
          if (!PAIR || rank == 0) {
            // a pair's leader counts both CTAs' bytes: the loads of both complete on its barrier
            mbar_arrive_expect_tx(&full[stage], PAIR ? 2 * tx_bytes : tx_bytes);
            armed_mask |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          int map = 0, x = w0, y = h0, z = zb;
          if (p.mode == kConv3x3x3) {
            x += kw - 1;
            y += kh - 1;
            z += kd - 1;
          } else if (p.mode == kConv3x3x3S2) {
            // input index 2o + k - 1: k = 1 -> parity 0 at o; k = 0 -> parity 1
            // at o - 1; k = 2 -> parity 1 at o.
            map = (kd != 1) * 4 + (kh != 1) * 2 + (kw != 1);
            x -= (kw == 0);
            y -= (kh == 0);
            z -= (kd == 0);
          } else if (p.mode == kConv3x3x3S2Pad01) {
            // input index 2o + k (no padding before): k = 0 -> parity 0 at o,
            // k = 1 -> parity 1 at o, k = 2 -> parity 0 at o + 1 (past the end:
            // the zero padding after).
            map = (kd == 1) * 4 + (kh == 1) * 2 + (kw == 1);
            x += (kw == 2);
            y += (kh == 2);
            z += (kd == 2);
          } else if (p.mode == kConvUp2) {
            // parity p, folded tap t reads source index m + p + t - 1.
            x += pw + kw - 1;
            y += ph + kh - 1;
            z += pd + kd - 1;
          }
          if (!waited) {
            pdl_wait();
            waited = true;
            if (p.clock) atomicMin(p.clock, static_cast<unsigned long long>(globaltimer_ns()));
          }
          const int chn = chunk * KC;
          if constexpr (PAIR) {
            const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_5d_pair(sa, &maps.a[map], bar, chn, x, y, z, c.b);
            tma_load_2d_pair(sb, &wmap, bar, kb * KC, brow);
          } else {
            tma_load_5d(sa, &maps.a[map], &full[stage], chn, x, y, z, c.b);
            tma_load_2d(sb, &wmap, &full[stage], kb * KC, brow);
          }
          if (EXACT) {
            tma_load_5d(sa + Cfg::kABytes, &maps.a[map], &full[stage], p.cin_pad + chn, x, y, z, c.b);
            tma_load_2d(sb + Cfg::kBBytes, &wmap, &full[stage], p.taps * p.cin_pad + kb * KC, brow);
          }
          for (chunk += P; chunk >= p.cin_chunks;) {  // P K blocks on
            chunk -= p.cin_chunks;
            if (p.mode == kConvUp2) {
              kw ^= 1;
              if (kw == 0) {
                kh ^= 1;
                if (kh == 0) ++kd;
              }
            } else if (++kw == 3) {
              kw = 0;
              if (++kh == 3) {
                kh = 0;
                ++kd;
              }
            }
          }
          stage += P;
          if (stage >= Cfg::kStages) {
            stage -= Cfg::kStages;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        // Let every armed TMA land before the CTA releases its shared memory.
        volatile int never = 0;
        for (int s = 0; s < Cfg::kStages; ++s)
          if (armed_mask & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, &never, status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (with pairs only the leader issues: one M = 256 product per K step)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      const uint32_t smem_base = smem_u32(smem);
      uint32_t stage_addr = smem_base;  // shared address of the current stage
      const uint64_t desc_const = make_smem_desc(0, 16, Cfg::kSbo, Cfg::kLayout);
      const uint32_t trans_idesc = TRANS ? make_idesc_f16(128, p.trans_n, 0, 0, 0) : 0u;
      for (int u = unit0; u < units && !*abort_flag; u += unit_step, ++local) {
        const TileCoord c = decode_tile(p, tile_of(u));
        const int kb0 = c.ks * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int acc = local & 1;
        if (!mbar_wait(&acc_empty[acc], ((local >> 1) & 1) ^ 1u, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t d_hi = tmem_base + acc * Cfg::kAccCols;
        const uint32_t d_lo = d_hi + BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors of the stage's tiles; the K = 16 step k starts 32
          // bytes further, i.e. 2 in the 16-byte address field (which cannot
          // carry: shared addresses are below 256 KB).
          const uint64_t ad0 = desc_const | static_cast<uint64_t>((stage_addr >> 4) & 0x3FFFu);
          const uint64_t bd0 = desc_const | static_cast<uint64_t>(((stage_addr + Cfg::kPlanes * Cfg::kABytes) >> 4) & 0x3FFFu);
#pragma unroll
          for (int k = 0; k < KC / 16; ++k) {
            const uint64_t ad = ad0 + 2 * k;
            const uint64_t bd = bd0 + 2 * k;
            const int step = (kb - kb0) * (KC / 16) + k;  // K step within the tile
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            if constexpr (TRANS) {
              // out^T: the weight tile is the M = 128 operand, the voxels are N
              const int chains = p.trans_chains;
              umma_ss(d_hi + (chains == 2 ? (step & 1) * 128 : 0), bd, ad, trans_idesc, step >= chains ? 1u : 0u);
              continue;
            }
            if constexpr (Cfg::kChains == 2) {
              umma_ss(d_hi + (step & 1) * BN, ad, bd, Cfg::kIdesc, step >= 2 ? 1u : 0u);
              continue;
            }
            if constexpr (PAIR) {
              umma_ss_pair(d_hi, ad, bd, Cfg::kIdesc, accum);
              continue;
            }
            umma_ss(d_hi, ad, bd, Cfg::kIdesc, accum);
            if (EXACT) {
              const uint64_t ad_lo = ad + (Cfg::kABytes >> 4);
              const uint64_t bd_lo = bd + (Cfg::kBBytes >> 4);
              umma_ss(d_lo, ad, bd_lo, Cfg::kIdesc, accum);
              umma_ss(d_lo, ad_lo, bd, Cfg::kIdesc, 1u);
            }
          }
          if constexpr (PAIR) {
            umma_commit_pair(&empty[stage], 3);  // frees the stage in both CTAs
          } else {
            umma_commit(&empty[stage]);
          }
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
            stage_addr = smem_base;
          } else {
            stage_addr += Cfg::kStageBytes;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          umma_commit_pair(&acc_full[acc], 3);  // both CTAs' halves of the accumulator are ready
        } else {
          umma_commit(&acc_full[acc]);
        }
      }
      // All issued MMAs must finish before TMEM is released.
      if constexpr (PAIR) {
        umma_commit_pair(drain, 1);
      } else {
        umma_commit(drain);
      }
      volatile int never = 0;
      mbar_wait(drain, 0, &never, status);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    EpiState st;
    st.epi = epi;
    st.res_full = res_full;
    st.bsum = bsum;
    st.vmask = vmask;
    st.sacc = sacc;
    st.abort_flag = abort_flag;
    st.status = status;
    st.quarter = warp & 3;
    st.row = st.quarter * 32 + lane;
    st.leader = threadIdx.x == 64;
    const bool split = p.k_splits > 1;
    int local = 0;
    for (int u = unit0; u < units; u += unit_step, ++local) {
      const TileCoord c = decode_tile(p, tile_of(u));
      const int acc = local & 1;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(st.quarter * 32) << 16) + acc * Cfg::kAccCols;
      bool ok;
      if constexpr (TRANS) {
        ok = epilogue_tile_trans<Cfg>(p, maps, c, tbase, &acc_full[acc], (local >> 1) & 1, st);
      } else if (split) {
        ok = epilogue_tile<Cfg, BN, EXACT, Cfg::kPartChunk, true>(p, maps, c, tbase, &acc_full[acc], (local >> 1) & 1, st);
      } else {
        ok = epilogue_tile<Cfg, BN, EXACT, Cfg::kOutChunk, false>(p, maps, c, tbase, &acc_full[acc], (local >> 1) & 1, st);
      }
      (void)ok;  // a failed wait already raised the abort flag and the device status
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) {
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));  // the leader's barrier
        } else {
          mbar_arrive(&acc_empty[acc]);
        }
      }
    }
    if constexpr (TRANS) {
      if (p.stats) flush_trans_stats(p, st);
    } else if (p.stats && !split && st.key_b >= 0) {
      named_barrier(1, 128);
      flush_stats<BN>(p, st, false);
    }
    if (st.leader) {
      bulk_wait_group_all();  // stores must finish before the CTA releases its shared memory
      if (p.clock && !split) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
    }
  }

  __syncwarp();
  __syncthreads();
  // With pairs: the leader's MMAs read this CTA's shared memory and write its
  // TMEM, so neither CTA releases either before both have finished (the
  // leader's MMA thread drained all MMAs before reaching this point).
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    } else {
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
  }
}

// Sum split-K partial tiles and apply the epilogue.  Block (slab, row
// block, out_tile) of 256 threads covers up to 64 columns x kRowLanes x
// kRowsPer rows of one output tile; thread (cq, rl) owns 4 columns of rows
// rl + kRowLanes * i and sums their K ranges (all rows' loads of a K range
// issued together).  With GroupNorm statistics requested, the rows' stored
// values are summed around the column's bias + shift in FP32 (lanes sharing
// a column by shuffles, warps by shared atomics) and the block adds one FP64
// pair per column to the totals.
template <int BN, int ROWS>
__global__ void __launch_bounds__(256) conv_reduce_kernel(const ConvParams p) {
  pdl_begin();
  constexpr int kSlab = BN < 64 ? BN : 64;
  constexpr int kQ = kSlab / 4;
  constexpr int kRowLanes = 256 / kQ;
  constexpr int kRowsPer = kTileM / kRowLanes < ROWS ? kTileM / kRowLanes : ROWS;
  __shared__ float red[2][kSlab];
  __shared__ int valid_rows;
  const int out_tiles = p.num_tiles / p.k_splits;
  const int ot = blockIdx.z;
  const int cq = threadIdx.x % kQ;
  const int rl = threadIdx.x / kQ;
  const int row0 = blockIdx.y * kRowLanes * kRowsPer + rl;
  const int col_t = blockIdx.x * kSlab + cq * 4;  // column within the tile
  const TileCoord c = decode_tile(p, ot * p.k_splits);
  const int col = c.nt * BN + col_t;
  const bool stats = p.stats != nullptr;
  if (stats) {
    for (int i = threadIdx.x; i < 2 * kSlab; i += blockDim.x) red[i / kSlab][i % kSlab] = 0.f;
    if (threadIdx.x == 0) valid_rows = 0;
    __syncthreads();
  }
  float v[kRowsPer][4];
#pragma unroll
  for (int i = 0; i < kRowsPer; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) v[i][j] = 0.f;
  if (col < p.cout) {
    const float* src = p.partials + (static_cast<long long>(ot) * kTileM + row0) * BN + col_t;
    const long long split_stride = static_cast<long long>(out_tiles) * kTileM * BN;
#pragma unroll 2
    for (int s = 0; s < p.k_splits; ++s) {
      float4 f[kRowsPer];
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i)
        f[i] = *reinterpret_cast<const float4*>(src + s * split_stride + static_cast<long long>(i) * kRowLanes * BN);
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i) {
        v[i][0] += f[i].x;
        v[i][1] += f[i].y;
        v[i][2] += f[i].z;
        v[i][3] += f[i].w;
      }
    }
  }
  bool live[kRowsPer];
  int nvalid = 0;
#pragma unroll
  for (int i = 0; i < kRowsPer; ++i) {
    const long long voxel = row_voxel(p, c, row0 + i * kRowLanes);
    live[i] = voxel >= 0 && col < p.cout;
    nvalid += voxel >= 0;
    if (live[i]) store_outputs<4>(p, c.b, voxel, col, v[i]);
  }
  if (!stats) {
    if (p.clock && threadIdx.x == 0) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
    return;
  }
  float k[4], d1[4], d2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int cj = col + j;
    k[j] = 0.f;
    if (cj < p.cout) {
      if (p.bias) k[j] = p.bias[cj];
      if (p.shift) k[j] += p.shift[static_cast<long long>(c.b) * p.cout + cj];
    }
    d1[j] = d2[j] = 0.f;
#pragma unroll
    for (int i = 0; i < kRowsPer; ++i) {
      const float d = live[i] ? v[i][j] - k[j] : 0.f;
      d1[j] += d;
      d2[j] = fmaf(d, d, d2[j]);
    }
  }
#pragma unroll
  for (int o = kQ; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      d1[j] += __shfl_xor_sync(0xffffffffu, d1[j], o);
      d2[j] += __shfl_xor_sync(0xffffffffu, d2[j], o);
    }
  }
  if ((threadIdx.x & 31) < kQ) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicAdd(&red[0][cq * 4 + j], d1[j]);
      atomicAdd(&red[1][cq * 4 + j], d2[j]);
    }
  }
  if (cq == 0 && nvalid) atomicAdd(&valid_rows, nvalid);
  __syncthreads();
  const int n = valid_rows;
  for (int j = threadIdx.x; j < kSlab; j += blockDim.x) {
    const int cc = c.nt * BN + blockIdx.x * kSlab + j;
    if (cc < p.cout && n > 0) {
      double kk = 0.0;
      if (p.bias) kk = p.bias[cc];
      if (p.shift) kk += p.shift[static_cast<long long>(c.b) * p.cout + cc];
      kk = static_cast<float>(kk);
      const double s1 = red[0][j], s2 = red[1][j];
      double* dst = p.stats + (static_cast<long long>(c.b) * p.cout + cc) * 2;
      red_add_f64(dst, s1 + n * kk);
      red_add_f64(dst + 1, s2 + 2.0 * kk * s1 + n * kk * kk);
    }
  }
  if (p.clock && threadIdx.x == 0) atomicMax(p.clock + 1, static_cast<unsigned long long>(globaltimer_ns()));
}

// Brick of at most 128 voxels covering a (d, h, w) grid with the fewest
// tiles; ties prefer wider bricks (longer contiguous TMA rows, more
// coalesced stores).
void choose_brick(int d, int h, int w, bool pointwise, int* bd, int* bh, int* bw) {
  long best_tiles = -1;
  int best[3] = {1, 1, 1};
  const int max_w = std::min(w, 128);
  for (int cw = max_w; cw >= 1; --cw) {
    const int max_h = std::min(h, 128 / cw);
    for (int ch = max_h; ch >= 1; --ch) {
      const int cd = std::min(d, 128 / (cw * ch));
      if (cd < 1) continue;
      const long tiles = static_cast<long>((w + cw - 1) / cw) * ((h + ch - 1) / ch) * ((d + cd - 1) / cd);
      if (best_tiles < 0 || tiles < best_tiles) {
        best_tiles = tiles;
        best[0] = cd;
        best[1] = ch;
        best[2] = cw;
      }
    }
    if (pointwise && best_tiles > 0) break;
  }
  *bd = best[0];
  *bh = best[1];
  *bw = best[2];
}

template <int KC, int BN, bool EXACT, bool TRANS = false, bool PAIR = false>
int launch_conv(cudaStream_t stream, const ConvMaps& maps, const CUtensorMap& wmap, const ConvParams& p,
                int grid) {
  using Cfg = ConvCfg<KC, BN, EXACT, TRANS, PAIR>;
  auto kernel = conv3d_tc_kernel<KC, BN, EXACT, TRANS, PAIR>;
  int smem = Cfg::kSmemBytes;
  // Keep one CTA per SM when the accumulators need more than half of TMEM,
  // so co-resident CTAs never queue on tcgen05.alloc.
  if (Cfg::kTmemCols > 256 && smem < 120 * 1024) smem = 120 * 1024;
  static unsigned long long configured = 0;
  {
    const int rc = ensure_smem_attribute(reinterpret_cast<const void*>(kernel), 227 * 1024, &configured,
                                         "conv smem attribute");
    if (rc != LDB_OK) return rc;
  }
  int rc;
  if constexpr (PAIR) {
    rc = launch_kernel_cluster(kernel, dim3(grid), dim3(Cfg::kThreads), smem, stream, "conv3d (CTA pairs) launch", 2u,
                               maps, wmap, p, device_status_ptr());
  } else {
    rc = launch_kernel(kernel, dim3(grid), dim3(Cfg::kThreads), smem, stream, "conv3d launch", maps, wmap, p,
                       device_status_ptr());
  }
  if (rc != LDB_OK) return rc;
  if (p.k_splits > 1) {
    // Many K ranges: one row per thread (more blocks, more loads in flight);
    // few: four rows per thread (fewer blocks, fewer statistics atomics).
    constexpr int kSlab = BN < 64 ? BN : 64;
    constexpr int kRowLanes = 256 / (kSlab / 4);
    constexpr int kRows4 = kTileM / kRowLanes < 4 ? kTileM / kRowLanes : 4;
    const bool deep = p.k_splits >= 6;
    rc = launch_kernel(deep ? conv_reduce_kernel<BN, 1> : conv_reduce_kernel<BN, 4>,
                       dim3(BN / kSlab, kTileM / (kRowLanes * (deep ? 1 : kRows4)), p.num_tiles / p.k_splits),
                       dim3(256), 0, stream, "conv3d split-K reduce launch", p);
  }
  return rc;
}

template <int KC, bool EXACT>
int dispatch_bn(int bn, cudaStream_t stream, const ConvMaps& maps, const CUtensorMap& wmap, const ConvParams& p,
                int grid) {
  switch (bn) {
    case 16: return launch_conv<KC, 16, EXACT>(stream, maps, wmap, p, grid);
    case 32: return launch_conv<KC, 32, EXACT>(stream, maps, wmap, p, grid);
    case 64: return launch_conv<KC, 64, EXACT>(stream, maps, wmap, p, grid);
    case 128: return launch_conv<KC, 128, EXACT>(stream, maps, wmap, p, grid);
    case 256:
      if constexpr (!EXACT) {
        if (p.pair) return launch_conv<KC, 256, false, false, true>(stream, maps, wmap, p, grid);
        return launch_conv<KC, 256, false>(stream, maps, wmap, p, grid);
      }
      break;
  }
  return fail(LDB_ERR_SHAPE, "no conv kernel for BN=%d", bn);
}

struct ConvPlan {
  int kc, bn, taps, cin_pad, grid;
  ConvParams p;
  size_t workspace;
};

// A pointwise conv over whole volumes is a GEMM over their voxels: it is
// planned as a 1 x 1 x (D H W) row of voxels (the voxel stride unchanged),
// so every tile is a run of 128 voxels instead of a box brick whose last
// rows and columns fall past the volume.  Other descriptors (and ones whose
// struct_size the planner will reject) pass through unchanged.
const ldb_conv_desc* flat_pointwise(const ldb_conv_desc* d, ldb_conv_desc* tmp) {
  if (!d || d->struct_size != static_cast<int>(sizeof(ldb_conv_desc))) return d;
  if (d->mode != LDB_CONV_1X1 || d->depth_halo != 0 || d->depth <= 0 || d->height <= 0 || d->width <= 0) return d;
  const long long voxels = static_cast<long long>(d->depth) * d->height * d->width;
  if (voxels > INT_MAX || (d->depth == 1 && d->height == 1)) return d;
  *tmp = *d;
  tmp->depth = 1;
  tmp->height = 1;
  tmp->width = static_cast<int>(voxels);
  return tmp;
}

int plan_conv(const ldb_conv_desc* d, ConvPlan* plan) {
  if (!d) return fail(LDB_ERR_INVALID, "conv descriptor is null");
  if (d->struct_size != static_cast<int>(sizeof(ldb_conv_desc)))
    return fail(LDB_ERR_INVALID,
                "conv descriptor struct_size %d != %d: the caller's ldb_conv_desc layout is not this library's "
                "(ABI version %d)",
                d->struct_size, static_cast<int>(sizeof(ldb_conv_desc)), LDB_ABI_VERSION);
  const int B = d->batch, D = d->depth, H = d->height, W = d->width;
  if (B <= 0 || D <= 0 || H <= 0 || W <= 0) return fail(LDB_ERR_SHAPE, "conv input extents must be positive");
  if (d->in_channels <= 0 || d->out_channels <= 0) return fail(LDB_ERR_SHAPE, "conv channels must be positive");
  if (d->mode < 0 || d->mode > 4) return fail(LDB_ERR_INVALID, "unknown conv mode %d", d->mode);
  const bool exact = d->exact != 0;
  const int cin = d->in_channels;
  const int cin_pad = ((cin + 15) / 16) * 16;
  const int kc = (cin_pad % 64 == 0) ? 64 : ((cin_pad % 32 == 0) ? 32 : 16);
  const int cout = d->out_channels;
  if (cout % 4 != 0 && cout != 1 && cout != 2) {
    // every column count works; the vector paths simply fall back to scalar stores
  }
  const int need_ld = exact ? 2 * cin_pad : cin;
  if (d->x_ld < need_ld) return fail(LDB_ERR_SHAPE, "x_ld %d < %d channels", d->x_ld, need_ld);
  if (d->x_ld % 8 != 0) return fail(LDB_ERR_ALIGNMENT, "x_ld %d must be a multiple of 8", d->x_ld);
  if (d->out_ld < cout) return fail(LDB_ERR_SHAPE, "out_ld %d < out_channels %d", d->out_ld, cout);
  int bn;
  if (cout <= 16) bn = 16;
  else if (cout <= 32) bn = 32;
  else if (cout <= 64) bn = 64;
  else if (cout <= 128 || exact) bn = 128;
  else bn = 256;
  if (d->depth_halo < 0 || d->depth_halo > 1) return fail(LDB_ERR_SHAPE, "depth_halo must be 0 or 1");
  const bool stride2 = d->mode == LDB_CONV_3X3X3_S2 || d->mode == LDB_CONV_3X3X3_S2_PAD01;
  if (d->depth_halo && stride2) return fail(LDB_ERR_SHAPE, "depth_halo with stride 2");
  if (D - 2 * d->depth_halo <= 0) return fail(LDB_ERR_SHAPE, "depth %d leaves no interior slice", D);
  ConvParams& p = plan->p;
  p = ConvParams{};
  p.batch = B;
  p.mode = d->mode;
  p.in_zoff = d->depth_halo;
  int gd = D - 2 * d->depth_halo, gh = H, gw = W;
  if (d->mode == LDB_CONV_3X3X3_S2) {
    gd = (D - 1) / 2 + 1;
    gh = (H - 1) / 2 + 1;
    gw = (W - 1) / 2 + 1;
  } else if (d->mode == LDB_CONV_3X3X3_S2_PAD01) {
    if (D < 2 || H < 2 || W < 2) return fail(LDB_ERR_SHAPE, "padding (0, 1) stride 2 needs extents >= 2");
    gd = (D - 2) / 2 + 1;
    gh = (H - 2) / 2 + 1;
    gw = (W - 2) / 2 + 1;
  }
  p.grid_d = gd;
  p.grid_h = gh;
  p.grid_w = gw;
  choose_brick(gd, gh, gw, d->mode == LDB_CONV_1X1, &p.bd, &p.bh, &p.bw);
  p.tiles_d = (gd + p.bd - 1) / p.bd;
  p.tiles_h = (gh + p.bh - 1) / p.bh;
  p.tiles_w = (gw + p.bw - 1) / p.bw;
  p.parities = d->mode == LDB_CONV_UP2 ? 8 : 1;
  const int taps = d->mode == LDB_CONV_1X1 ? 1 : (d->mode == LDB_CONV_UP2 ? 8 : 27);
  p.taps = taps;
  p.cin_pad = cin_pad;
  p.cin_chunks = cin_pad / kc;
  p.kb_total = taps * p.cin_chunks;
  p.n_tiles = (cout + bn - 1) / bn;
  p.wrows_per_parity = p.n_tiles * bn;
  const long long out_tiles =
      static_cast<long long>(B) * p.tiles_d * p.tiles_h * p.tiles_w * p.parities * p.n_tiles;
  if (out_tiles > (1LL << 30)) return fail(LDB_ERR_SHAPE, "conv has too many tiles");
  if (d->max_ctas < 0) return fail(LDB_ERR_INVALID, "max_ctas must be >= 0");
  const int sms = d->max_ctas > 0 ? std::max(2, std::min(sm_count(), d->max_ctas)) : sm_count();
  if (taps == 1 && !exact && bn == 256 && cout % 256 == 0) {
    // Pointwise: K is a few k-blocks, so split-K would only add a reduce
    // pass; fill the SMs with narrower column tiles instead.  Cost per tile
    // = k-blocks x shared-memory-bound k-block time ((128 + BN) x KC / 32
    // cycles: TMA writes plus MMA operand reads) + ~4000 cycles of set-up and
    // epilogue, times the waves of the persistent grid.
    const long long m_tiles = out_tiles / p.n_tiles;
    long long best = -1;
    for (int cand : {256, 128, 64}) {
      const long long tiles = m_tiles * (cout / cand);
      const long long cost = ((tiles + sms - 1) / sms) * (static_cast<long long>(p.kb_total) * (128 + cand) * kc / 32 + 4000);
      if (best < 0 || cost < best) {
        best = cost;
        bn = cand;
      }
    }
    p.n_tiles = (cout + bn - 1) / bn;
    p.wrows_per_parity = p.n_tiles * bn;
  }
  const long long bricks = static_cast<long long>(B) * p.tiles_d * p.tiles_h * p.tiles_w;
  const long long m_tiles = bricks * p.parities;
  // CTA pairs for the f16 256-column 3x3x3 tile: each CTA of a pair stages
  // its 128-voxel brick and half of the 256 weight rows (32 KB per K block
  // instead of 48), so a stage carries 1.5x the FLOPs per staged byte and the
  // ring keeps more K blocks in flight.
  const bool pair = !exact && bn == 256 && taps > 1 && bricks >= 2;
  // pairs of same-parity bricks (see pair_tile)
  const long long pairs = (bricks + 1) / 2 * p.parities;
  // CTAs one K range of every output tile needs (a pair's placeholder tile counts)
  const long long tiles_now = (pair ? 2 * pairs : m_tiles) * p.n_tiles;
  int splits = 1;
  if (taps > 1 && tiles_now < sms && p.kb_total >= 8) {
    splits = static_cast<int>(std::min<long long>(sms / tiles_now, p.kb_total / 4));
    splits = std::max(1, splits);
  }
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.k_splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.num_tiles = static_cast<int>(m_tiles * p.n_tiles * p.k_splits);
  p.pair = pair ? 1 : 0;
  p.m_tiles = static_cast<int>(m_tiles);
  p.num_units = pair ? static_cast<int>(pairs * p.n_tiles * p.k_splits) : 0;
  p.cout = cout;
  p.out_ld = d->out_ld;
  p.res_ld = d->res_ld;
  p.out_f32 = d->out_dtype == LDB_F32 ? 1 : 0;
  p.out_scale = d->output_scale;
  p.act = d->act;
  const int up = d->mode == LDB_CONV_UP2 ? 2 : 1;
  p.out_d = gd * up;
  p.out_h = gh * up;
  p.out_w = gw * up;
  plan->kc = kc;
  plan->bn = bn;
  plan->taps = taps;
  plan->cin_pad = cin_pad;
  // Channel-major tile for 64 / 128 output channels when the grid needs no
  // split-K: the MMA runs as 128 (channels) x 64*bd (voxels of a bd x 8 x 8
  // brick, bd <= 3: a 192-row stage leaves room for a four-stage ring) where
  // a 128-channel voxel-major tile would run 128 x 128.  bd minimises waves x
  // tile size.
  // (64-channel K blocks only: with 16 / 32 input channels per block the
  // per-block overhead dominates and the voxel-major tile is faster.  3x3x3
  // kernels only: a pointwise conv has too few K blocks per tile to hide the
  // per-plane transposed epilogue, and its voxel-major tile runs ~3x faster.)
  const bool trans_ok = !exact && taps > 1 && p.k_splits == 1 && kc == 64 &&
                        (cout == 128 || (cout == 64 && p.parities == 1));
  if (trans_ok) {
    const long long th = (gh + 7) / 8, tw = (gw + 7) / 8;
    int best_bd = 1;
    long long best_cost = -1;
    for (int cand = 1; cand <= 3; ++cand) {
      const long long tiles = static_cast<long long>(B) * ((gd + cand - 1) / cand) * th * tw * p.parities;
      const long long cost = ((tiles + sms - 1) / sms) * (64LL * cand + 64);
      if (best_cost < 0 || cost <= best_cost) {
        best_cost = cost;
        best_bd = cand;
      }
    }
    p.trans = 1;
    p.pair = 0;
    p.bd = best_bd;
    p.bh = 8;
    p.bw = 8;
    p.trans_n = 64 * best_bd;
    p.trans_chains = p.trans_n <= 128 ? 2 : 1;
    p.tiles_d = (gd + best_bd - 1) / best_bd;
    p.tiles_h = static_cast<int>(th);
    p.tiles_w = static_cast<int>(tw);
    p.n_tiles = 1;  // the weight tile covers all output channels (rows past cout read as zero)
    p.num_tiles = static_cast<int>(static_cast<long long>(B) * p.tiles_d * th * tw * p.parities);
    plan->bn = 128;
  }
  plan->grid = p.pair ? 2 * static_cast<int>(std::min<long long>(p.num_units, sms / 2))
                      : static_cast<int>(std::min<long long>(p.num_tiles, sms));
  plan->workspace = p.k_splits > 1 ? static_cast<size_t>(p.num_tiles) * kTileM * bn * sizeof(float) : 0;
  return LDB_OK;
}

}  // namespace

}  // namespace ldb

extern "C" {

int ldb_conv3d_workspace_size(const ldb_conv_desc* desc, size_t* bytes) {
  if (!bytes) return ldb::fail(LDB_ERR_INVALID, "bytes pointer is null");
  ldb_conv_desc flat;
  desc = ldb::flat_pointwise(desc, &flat);
  ldb::ConvPlan plan;
  int rc = ldb::plan_conv(desc, &plan);
  if (rc != LDB_OK) return rc;
  *bytes = plan.workspace;
  return LDB_OK;
}

int ldb_conv3d_weight_rows(const ldb_conv_desc* desc, int* rows_per_parity, int* k_total) {
  ldb_conv_desc flat;
  desc = ldb::flat_pointwise(desc, &flat);
  ldb::ConvPlan plan;
  int rc = ldb::plan_conv(desc, &plan);
  if (rc != LDB_OK) return rc;
  if (rows_per_parity) *rows_per_parity = plan.p.wrows_per_parity;
  if (k_total) *k_total = plan.taps * plan.cin_pad * (desc->exact ? 2 : 1);
  return LDB_OK;
}

static int conv_forward(cudaStream_t stream, const ldb_conv_desc* desc, const void* x, const void* w_packed,
                        const float* bias, const float* shift, const void* residual, void* out, double* stats,
                        void* workspace, size_t workspace_bytes) {
  using namespace ldb;
  ldb_conv_desc flat;
  desc = flat_pointwise(desc, &flat);
  ConvPlan plan;
  int rc = plan_conv(desc, &plan);
  if (rc != LDB_OK) return rc;
  if (!x || !w_packed || !out) return fail(LDB_ERR_INVALID, "conv3d: x, weights and out must be non-null");
  if (residual && desc->res_ld < desc->out_channels)
    return fail(LDB_ERR_SHAPE, "res_ld %d < out_channels %d", desc->res_ld, desc->out_channels);
  if (plan.workspace > 0 && (!workspace || workspace_bytes < plan.workspace))
    return fail(LDB_ERR_WORKSPACE, "conv3d needs %zu workspace bytes, got %zu", plan.workspace, workspace_bytes);
  if ((desc->exact != 0) != (desc->out_dtype == LDB_F32))
    return fail(LDB_ERR_INVALID, "conv3d output dtype must be f32 in exact mode and f16 otherwise");
  const ldb_conv_desc* d = desc;
  ConvParams& p = plan.p;
  p.bias = bias;
  p.shift = shift;
  p.residual = residual;
  p.out = out;
  p.stats = stats;
  p.clock = desc->clock;
  p.partials = static_cast<float*>(workspace);

  const int B = desc->batch, D = desc->depth, H = desc->height, W = desc->width;
  const bool exact = desc->exact != 0;
  const uint64_t esz = 2;
  const uint64_t ld = static_cast<uint64_t>(desc->x_ld);
  const uint64_t cdim = exact ? 2 * plan.cin_pad : desc->in_channels;
  ConvMaps maps;
  memset(&maps, 0, sizeof(maps));
  const uint32_t abox[5] = {static_cast<uint32_t>(plan.kc), static_cast<uint32_t>(p.bw),
                            static_cast<uint32_t>(p.bh), static_cast<uint32_t>(p.bd), 1u};
  if (desc->mode == LDB_CONV_3X3X3_S2 || desc->mode == LDB_CONV_3X3X3_S2_PAD01) {
    for (int par = 0; par < 8; ++par) {
      const int pd = par >> 2, ph = (par >> 1) & 1, pw = par & 1;
      const uint64_t dims[5] = {cdim, static_cast<uint64_t>((W - pw + 1) / 2), static_cast<uint64_t>((H - ph + 1) / 2),
                                static_cast<uint64_t>((D - pd + 1) / 2), static_cast<uint64_t>(B)};
      const uint64_t strides[4] = {2 * ld * esz, 2 * W * ld * esz, 2 * H * W * ld * esz,
                                   static_cast<uint64_t>(D) * H * W * ld * esz};
      if (dims[1] == 0 || dims[2] == 0 || dims[3] == 0) {
        // A parity view with no voxels (extent 1): alias the even view; every
        // coordinate it would serve is out of range and zero-filled anyway.
        maps.a[par] = maps.a[0];
        continue;
      }
      const uint8_t* base = static_cast<const uint8_t*>(x) +
                            ((static_cast<uint64_t>(pd) * H + ph) * W + pw) * ld * esz;
      rc = encode_tiled_f16(&maps.a[par], base, 5, dims, strides, abox, plan.kc * 2);
      if (rc != LDB_OK) return rc;
    }
  } else {
    const uint64_t dims[5] = {cdim, static_cast<uint64_t>(W), static_cast<uint64_t>(H), static_cast<uint64_t>(D),
                              static_cast<uint64_t>(B)};
    const uint64_t strides[4] = {ld * esz, W * ld * esz, static_cast<uint64_t>(H) * W * ld * esz,
                                 static_cast<uint64_t>(D) * H * W * ld * esz};
    rc = encode_tiled_f16(&maps.a[0], x, 5, dims, strides, abox, plan.kc * 2);
    if (rc != LDB_OK) return rc;
  }
  // Output / residual store-load maps (or the split-K partial map).
  const int out_esz = exact ? 4 : 2;
  if (p.k_splits > 1) {
    const int cc = std::min(plan.bn, 32);
    const uint64_t dims[2] = {static_cast<uint64_t>(plan.bn), static_cast<uint64_t>(p.num_tiles) * kTileM};
    const uint64_t strides[1] = {static_cast<uint64_t>(plan.bn) * 4};
    const uint32_t box[2] = {static_cast<uint32_t>(cc), static_cast<uint32_t>(kTileM)};
    rc = encode_tiled_f32(&maps.part, workspace, 2, dims, strides, box, cc * 4);
    if (rc != LDB_OK) return rc;
  } else {
    const int cc = std::min(plan.bn, 128 / out_esz);
    // channel-major tiles store one depth plane per TMA store
    const uint32_t obox[5] = {static_cast<uint32_t>(cc), static_cast<uint32_t>(p.bw), static_cast<uint32_t>(p.bh),
                              static_cast<uint32_t>(p.trans ? 1 : p.bd), 1u};
    auto encode_out = [&](CUtensorMap* dst, const void* base_ptr, int ld) -> int {
      if ((static_cast<long long>(ld) * out_esz) % 16 != 0)
        return fail(LDB_ERR_ALIGNMENT, "output/residual channel stride %d is not a multiple of 16 bytes", ld);
      const uint64_t lde = static_cast<uint64_t>(ld) * out_esz;
      const int nviews = d->mode == LDB_CONV_UP2 ? 8 : 1;
      for (int v = 0; v < nviews; ++v) {
        uint64_t dims[5], strides[4];
        const uint8_t* base = static_cast<const uint8_t*>(base_ptr);
        if (nviews == 8) {
          const int pd = v >> 2, ph = (v >> 1) & 1, pw = v & 1;
          const uint64_t OW = p.out_w, OH = p.out_h, OD = p.out_d;
          base += ((static_cast<uint64_t>(pd) * OH + ph) * OW + pw) * lde;
          const uint64_t dd[5] = {static_cast<uint64_t>(p.cout), static_cast<uint64_t>(p.grid_w),
                                  static_cast<uint64_t>(p.grid_h), static_cast<uint64_t>(p.grid_d),
                                  static_cast<uint64_t>(p.batch)};
          const uint64_t ss[4] = {2 * lde, 2 * OW * lde, 2 * OH * OW * lde, OD * OH * OW * lde};
          memcpy(dims, dd, sizeof(dd));
          memcpy(strides, ss, sizeof(ss));
        } else {
          const uint64_t OW = p.out_w, OH = p.out_h, OD = p.out_d;
          const uint64_t dd[5] = {static_cast<uint64_t>(p.cout), OW, OH, OD, static_cast<uint64_t>(p.batch)};
          const uint64_t ss[4] = {lde, OW * lde, OH * OW * lde, OD * OH * OW * lde};
          memcpy(dims, dd, sizeof(dd));
          memcpy(strides, ss, sizeof(ss));
        }
        const int r = exact ? encode_tiled_f32(&dst[v], base, 5, dims, strides, obox, cc * out_esz)
                            : encode_tiled_f16(&dst[v], base, 5, dims, strides, obox, cc * out_esz);
        if (r != LDB_OK) return r;
      }
      return LDB_OK;
    };
    rc = encode_out(maps.o, out, desc->out_ld);
    if (rc != LDB_OK) return rc;
    if (residual) {
      rc = encode_out(maps.r, residual, desc->res_ld);
      if (rc != LDB_OK) return rc;
    }
  }

  CUtensorMap wmap;
  const uint64_t ktotal = static_cast<uint64_t>(plan.taps) * plan.cin_pad * (exact ? 2 : 1);
  const uint64_t wrows = static_cast<uint64_t>(p.parities) * p.wrows_per_parity;
  const uint64_t wdims[2] = {ktotal, wrows};
  const uint64_t wstrides[1] = {ktotal * esz};
  // (a pair's CTA stages half of the column tile's weight rows)
  const uint32_t wbox[2] = {static_cast<uint32_t>(plan.kc), static_cast<uint32_t>(p.pair ? plan.bn / 2 : plan.bn)};
  rc = encode_tiled_f16(&wmap, w_packed, 2, wdims, wstrides, wbox, plan.kc * 2);
  if (rc != LDB_OK) return rc;

  if (p.trans) {
    switch (plan.kc) {
      case 16: return launch_conv<16, 128, false, true>(stream, maps, wmap, p, plan.grid);
      case 32: return launch_conv<32, 128, false, true>(stream, maps, wmap, p, plan.grid);
      default: return launch_conv<64, 128, false, true>(stream, maps, wmap, p, plan.grid);
    }
  }
  switch (plan.kc) {
    case 16:
      return exact ? dispatch_bn<16, true>(plan.bn, stream, maps, wmap, p, plan.grid)
                   : dispatch_bn<16, false>(plan.bn, stream, maps, wmap, p, plan.grid);
    case 32:
      return exact ? dispatch_bn<32, true>(plan.bn, stream, maps, wmap, p, plan.grid)
                   : dispatch_bn<32, false>(plan.bn, stream, maps, wmap, p, plan.grid);
    default:
      return exact ? dispatch_bn<64, true>(plan.bn, stream, maps, wmap, p, plan.grid)
                   : dispatch_bn<64, false>(plan.bn, stream, maps, wmap, p, plan.grid);
  }
}

int ldb_conv3d_fwd(cudaStream_t stream, const ldb_conv_desc* desc, const void* x, const void* w_packed,
                   const float* bias, const float* shift, const void* residual, void* out, void* workspace,
                   size_t workspace_bytes) {
  return conv_forward(stream, desc, x, w_packed, bias, shift, residual, out, nullptr, workspace, workspace_bytes);
}

int ldb_conv3d_fwd_gn_stats(cudaStream_t stream, const ldb_conv_desc* desc, const void* x, const void* w_packed,
                            const float* bias, const float* shift, const void* residual, void* out, double* stats,
                            void* workspace, size_t workspace_bytes) {
  if (!stats) return ldb::fail(LDB_ERR_INVALID, "conv3d: stats is null");
  return conv_forward(stream, desc, x, w_packed, bias, shift, residual, out, stats, workspace, workspace_bytes);
}

}  // extern "C"
