// Parameters shared by the implicit-GEMM convolution kernel, its split-K
// reduction and the host launcher.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ldb {

// How GEMM rows (M) and K taps map onto the activation volume.
enum ConvMode : int {
  kConv3x3x3 = 0,    // padding 1, stride 1: 27 taps, rows are output voxels
  kConv3x3x3S2 = 1,  // padding 1, stride 2: 27 taps over 8 parity views of the input
  kConvUp2 = 2,      // conv of a nearest 2x upsampling: 8 parities x 8 folded taps, rows are source voxels
  kConvPointwise = 3, // 1x1x1 (dense over tokens): one tap
  kConv3x3x3S2Pad01 = 4 // stride 2, padding 0 before / 1 after: 27 taps over the 8 parity views
};

enum ConvAct : int { kActNone = 0, kActGelu = 1 };

struct ConvParams {
  // GEMM row space: a (batch, grid_d, grid_h, grid_w) volume tiled by bricks
  // of bd x bh x bw voxels (at most 128), times `parities` output parities.
  int batch, grid_d, grid_h, grid_w;
  int bd, bh, bw;
  int tiles_d, tiles_h, tiles_w;
  int parities;
  int n_tiles;       // output-channel tiles of BN
  int k_splits;      // K ranges computed by separate CTAs (partials reduced later)
  int kb_per_split;  // K blocks per range
  int kb_total;      // taps * cin_chunks
  int cin_chunks;    // K blocks per tap
  int cin_pad;       // weight channels per tap (multiple of the K block)
  int taps;
  int mode;
  // Channel-major tile: the MMA computes out^T (M = output channels, N =
  // trans_n voxels of a bd x 8 x 8 brick); 0 for the voxel-major tile.
  int trans;
  int trans_n;
  int trans_chains;      // channel-major tile: 2 interleaved accumulator chains when trans_n <= 128
  int in_zoff;           // depth index of output slice 0's centre tap in x (the depth halo)
  int wrows_per_parity;  // packed weight rows per parity (Cout padded to BN)
  int num_tiles;         // batch * tiles * parities * n_tiles * k_splits
  // CTA pairs (cta_group::2, voxel-major 256-column tile): two spatial
  // bricks of the same output parity form a pair, computed as one M = 256
  // product by the two CTAs of a cluster; a pair's second brick past the last
  // one is a placeholder whose loads read zeros and whose results are
  // dropped.  Work units are (pair, column tile, K range).  pair = 0: one CTA
  // per tile.
  int pair;
  int m_tiles;    // batch * tiles * parities
  int num_units;  // ceil(bricks / 2) * parities * n_tiles * k_splits when pair
  // Epilogue: out = act((acc + bias + shift[b]) * scale + residual), stored as
  // f16 or f32 in NDHWC with channel stride out_ld; with k_splits > 1 raw f32
  // partial tiles go to `partials` and the reduction kernel applies it.
  int cout;
  const float* bias;   // [cout] f32 (may be null)
  const float* shift;  // [batch][cout] f32 (may be null)
  const void* residual;
  int res_ld;
  void* out;
  int out_ld;
  int out_f32;
  float out_scale;
  int act;
  float* partials;
  // GroupNorm statistics of the stored output (may be null): per (batch,
  // channel) the FP64 sum and sum of squares, added atomically.
  double* stats;
  int out_d, out_h, out_w;
  // Device-clock timing of the launch (may be null): [start, end] in ns.
  unsigned long long* clock;
};

// Tensor maps of one convolution: activation loads (one map, or 8 parity
// views for stride 2), output stores and residual loads (one map, or the 8
// output-parity views of the folded upsampling conv), and the split-K
// partial-tile store.
struct ConvMaps {
  CUtensorMap a[8];
  CUtensorMap o[8];
  CUtensorMap r[8];
  CUtensorMap part;
};

}  // namespace ldb
