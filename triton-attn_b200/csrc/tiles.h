// Tile variants of the fp16 tensor-core kernels: the B200 stand-in for the reference's autotune
// spaces (src/tattn/kernels.py:21-41, chosen per (N bucket, D, causal) at api.py:59-62). Instead of
// timing candidates at run time, each family has a short static list of variants that fit sm_100a's
// TMEM (512 columns) and shared memory, and a fixed default per (D, causal, dtype) chosen from
// measurements on a B200. tile_cfg 0 selects that default; tile_cfg i >= 1 selects variant i - 1 (the
// reference's `_launch(config=...)` bypass, api.py:69-75, which its tests use to check every variant).
#pragma once

namespace tattn {

struct TileVariant {
  int block_m;  // query rows per CTA (forward: two 128-row tiles) or rows of the CTA's own tile (backward)
  int block_n;  // rows of the inner blocks the CTA loops over (keys, or queries for dK/dV)
  int stages;   // depth of the TMA ring of inner blocks
};

// Forward (fwd_f16_kernel): CTA = two 128-row query tiles; key/value blocks of block_n rows through a
// ring of `stages` slots. block_n = 128 at D = 128 writes P over S in TMEM (2 * 128 + 2 * 128 = 512
// columns) and fits shared memory with 2 stages only (2 * 32 KB of Q + 2 * 2 * 32 KB of K and V).
constexpr TileVariant kFwdTiles[] = {
    {256, 128, 4},
    {256, 64, 4},
    {256, 128, 2},
};
// Backward split path (tattn_bwd_dkdv + tattn_bwd_dq): 128-row key tiles whose query blocks have
// block_n rows, and 128-row query tiles whose key blocks have block_n rows. block_n = 128 is D <= 64
// only (TMEM and shared memory).
constexpr TileVariant kBwdTiles[] = {
    {128, 128, 4},
    {128, 64, 4},
};
constexpr int kNumFwdTiles = int(sizeof(kFwdTiles) / sizeof(kFwdTiles[0]));
constexpr int kNumBwdTiles = int(sizeof(kBwdTiles) / sizeof(kBwdTiles[0]));

// Does variant `v` (0-based) of family `kind` (0 forward, 1 backward) exist for head dim D?
constexpr bool tile_supported(int kind, int v, int D) {
  if (kind == 0)
    return v >= 0 && v < kNumFwdTiles && (kFwdTiles[v].block_n == 64 || D <= 64 || kFwdTiles[v].stages <= 2);
  if (kind == 1) return v >= 0 && v < kNumBwdTiles && (kBwdTiles[v].block_n == 64 || D <= 64);
  return false;
}

// The variant (0-based) tile_cfg 0 runs for an fp16 call, by family, head dim (16, 32, 64, 128) and
// causal (no, yes): 128-row inner blocks wherever they fit (at D = 128 the forward's 2-stage variant,
// measured 1-4 % faster than 64-key blocks), 64 rows otherwise. fp32 calls run the SIMT kernels, which
// have no tile choice.
constexpr int kDefaultTile[2][4][2] = {
    {{0, 0}, {0, 0}, {0, 0}, {2, 2}},  // forward
    {{0, 0}, {0, 0}, {0, 0}, {1, 1}},  // backward (split path)
};

constexpr int head_dim_index(int D) { return D == 16 ? 0 : D == 32 ? 1 : D == 64 ? 2 : 3; }

constexpr int tile_default(int kind, int D, bool causal) {
  return kDefaultTile[kind == 0 ? 0 : 1][head_dim_index(D)][causal ? 1 : 0];
}

}  // namespace tattn
