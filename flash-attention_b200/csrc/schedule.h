// Work units and their order.
//
// A work unit is a pair of 128-row query tiles (rows [256 p, 256 p + 256)) of one
// (batch, head) slice.  The reference launches one CTA per 64-row query tile,
// grid (N/64, H, B) (src/forward/forward_v6_mma.cuh:325-412); here persistent CTAs
// take units from an atomic counter in that order:
//  * slices are grouped so that the K/V of the slices in flight stay in L2 while
//    each key block is read by every unit of its slice.  Without a causal mask
//    all units cost the same and a group is one wave of units (about one unit
//    per SM, all reading the same slices' K/V at the same time).  With a causal
//    mask a group is as many slices as fit kL2GroupBytes of K and V, split into
//    groups of equal size (at least one wave each), so that the longest-first
//    order below has many units to balance;
//  * within a group, units go pair-major: for causal attention every slice's
//    pair with the most key blocks (the last one) first, then the next lighter
//    pair, so the group runs longest-first and the lightest units end the launch.
// A CTA claims its next unit only when it reaches that unit's first key block,
// so the order the counter hands out is the order in which CTAs become free.
//
// Plain integer arithmetic, shared by the host (planning, unit tests) and the
// kernel (decoding).
#pragma once

#include "umma_layout.h"  // FA_HD

namespace fa {

constexpr int kUnitRows = 256;  // query rows per work unit (two 128-row tiles)
// K + V bytes of the slices one scheduling group keeps in flight: about half the
// 126 MB L2, leaving the rest to the streamed Q tiles and O stores.
constexpr long long kL2GroupBytes = 64ll << 20;

struct SchedPlan {
  int n_pairs;    // ceil(N / 256): units per slice
  int n_kv;       // ceil(N / key_block): key/value blocks per slice
  int num_tiles;  // batch * heads * n_pairs
  int group_bh;   // slices per scheduling group
  int grid;       // persistent CTAs: min(num_tiles, sms)
};

// Host plan for B x H slices of N rows of head_dim 16-bit elements on a GPU with
// `sms` SMs.
FA_HD SchedPlan plan_schedule(int batch, int heads, int seq_len, int head_dim, int key_block, int sms, bool causal) {
  SchedPlan s;
  s.n_pairs = (seq_len + kUnitRows - 1) / kUnitRows;
  s.n_kv = (seq_len + key_block - 1) / key_block;
  const long long bh = static_cast<long long>(batch) * heads;
  const long long tiles = bh * s.n_pairs;
  s.num_tiles = tiles > (1ll << 30) ? -1 : static_cast<int>(tiles);  // -1: too many
  const long long wave = (sms + s.n_pairs - 1) / s.n_pairs;  // slices that give one unit per SM
  long long g = wave;
  if (causal) {
    // Fewest groups whose K + V fit the budget, then slices spread evenly over them.
    const long long kv_bytes = 4ll * seq_len * head_dim;  // K and V of one slice
    long long groups = (bh * kv_bytes + kL2GroupBytes - 1) / kL2GroupBytes;
    if (groups < 1) groups = 1;
    g = (bh + groups - 1) / groups;
    if (g < wave) g = wave;
  }
  if (g > bh) g = bh;
  if (g < 1) g = 1;
  s.group_bh = static_cast<int>(g);
  s.grid = static_cast<int>(tiles < sms ? tiles : sms);
  return s;
}

struct TileInfo {
  int b, h, pair, n0, n1;  // slice, unit, key blocks of query tile 0 and 1 (0: tile past N)
};

// Unit index -> slice, pair and key-block counts.
FA_HD TileInfo decode_unit(int tile, int batch, int heads, int seq_len, int n_pairs, int n_kv, int group_bh,
                           int key_block, bool causal) {
  const int bh_total = batch * heads;
  const int per_group = group_bh * n_pairs;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int gsize = (group_bh < bh_total - g * group_bh) ? group_bh : bh_total - g * group_bh;
  const int rank = r / gsize;
  const int bh = g * group_bh + (r - rank * gsize);
  TileInfo t;
  t.b = bh / heads;
  t.h = bh - t.b * heads;
  t.pair = causal ? (n_pairs - 1 - rank) : rank;
  const int q1 = t.pair * kUnitRows + 128;
  // causal: key blocks up to the one holding the tile's last row
  const int c0 = (t.pair * kUnitRows + 128 + key_block - 1) / key_block;
  const int c1 = (t.pair * kUnitRows + 256 + key_block - 1) / key_block;
  t.n0 = causal ? (c0 < n_kv ? c0 : n_kv) : n_kv;
  t.n1 = q1 >= seq_len ? 0 : (causal ? (c1 < n_kv ? c1 : n_kv) : n_kv);
  return t;
}

}  // namespace fa
