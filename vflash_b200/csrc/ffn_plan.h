// Work order of the fused FFN kernel (ffn_fused.cu), shared by the kernel and
// the host-side schedule check (tests/ffn_schedule_check.cpp).
//
// The FFN of M token rows runs in row blocks of 256 rows (one CTA-pair tile
// high).  Row block r needs ju "up" tiles (the up projection's output
// columns, 256 per tile, or 128 value + 128 gate columns for SwiGLU) and jd
// "down" tiles (256 output columns each).  A down tile of row block r reads
// the requantised intermediate of the whole row, so it may start only after
// every up tile of row block r has been stored and converted.
//
// Order of the work items (every CTA pair takes the next item from one global
// counter, so an item only ever waits on items that running pairs took
// earlier, whether or not every pair of the grid is resident):
//   * row blocks are taken in groups of `group` blocks; the up tiles of a
//     group run in bands of `band_up` weight tiles (row block by row block
//     inside a band, tile fastest), so one band of the up weight serves the
//     whole group from L2;
//   * the down tiles of group g, in bands of `band_down`, are interleaved
//     with the up tiles of group g + `lag` after a lead of `lead` up items;
//     the lag and the lead give the last up tiles of group g time to finish
//     and convert before its down tiles are taken.  The mix balances the up
//     tiles' heavy epilogues (activation, row maxima, conversion) against the
//     down tiles' long main loops.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define VFB_HD __host__ __device__ __forceinline__
#else
#define VFB_HD inline
#endif

namespace vfb {

struct FfnPlan {
  int rows_blocks;  // R: row blocks of 256 rows
  int ju;           // up tiles per row block
  int jd;           // down tiles per row block
  int group;        // row blocks per group
  int groups;       // ceil(R / group)
  int band_up;      // up weight tiles per band
  int band_down;    // down weight tiles per band
  int lead;         // up items of group g + lag before the first down item of group g
  int lag;          // groups between a group's up tiles and its down tiles (>= 1)
  int total;        // R * (ju + jd)
};

constexpr int kFfnUp = 0;
constexpr int kFfnDown = 1;

VFB_HD int ffn_min(int a, int b) { return a < b ? a : b; }

// Coordinates of item i of a banded grid of `rows` row blocks x `cols` tiles.
VFB_HD void ffn_band_coords(int i, int rows, int cols, int band, int &row, int &col) {
  const int b = i / (rows * band);
  const int rest = i - b * rows * band;
  const int w = ffn_min(band, cols - b * band);
  row = rest / w;
  col = b * band + rest % w;
}

VFB_HD int ffn_group_rows(const FfnPlan &p, int g) { return ffn_min(p.group, p.rows_blocks - g * p.group); }

// Item `s` of the merge of up(g + lag) (n_up items) with down(g) (n_down items).
VFB_HD void ffn_merge_item(const FfnPlan &p, int g, int s, int n_up, int n_down, int &kind, int &r, int &t) {
  const int lead = ffn_min(p.lead, n_up);
  int up_index = -1, down_index = -1;
  if (s < lead) {
    up_index = s;
  } else if (n_down == 0) {
    up_index = s;
  } else {
    // after the lead: n_down cycles, cycle c = one down item followed by
    // a_c up items, a_c spreading the remaining up items evenly
    const int64_t rest = n_up - lead;
    const int64_t u = s - lead;
    int64_t c = u * n_down / (n_down + rest);
    while (c + 1 < n_down && (c + 1) + ((c + 1) * rest) / n_down <= u) ++c;
    while (c > 0 && c + (c * rest) / n_down > u) --c;
    const int64_t start = c + (c * rest) / n_down;
    if (u == start) {
      down_index = static_cast<int>(c);
    } else {
      up_index = lead + static_cast<int>((c * rest) / n_down + (u - start) - 1);
    }
  }
  if (up_index >= 0) {
    const int gr = ffn_group_rows(p, g + p.lag);
    int row, col;
    ffn_band_coords(up_index, gr, p.ju, p.band_up, row, col);
    kind = kFfnUp;
    r = (g + p.lag) * p.group + row;
    t = col;
  } else {
    const int gr = ffn_group_rows(p, g);
    int row, col;
    ffn_band_coords(down_index, gr, p.jd, p.band_down, row, col);
    kind = kFfnDown;
    r = g * p.group + row;
    t = col;
  }
}

// Decodes work item q (0 <= q < total) into its kind, row block and tile.
VFB_HD void ffn_item(const FfnPlan &p, int q, int &kind, int &r, int &t) {
  int s = q;
  // the up tiles of the first `lag` groups come first
  for (int g0 = 0; g0 < p.lag && g0 < p.groups; ++g0) {
    const int gr = ffn_group_rows(p, g0);
    if (s < gr * p.ju) {
      int row, col;
      ffn_band_coords(s, gr, p.ju, p.band_up, row, col);
      kind = kFfnUp;
      r = g0 * p.group + row;
      t = col;
      return;
    }
    s -= gr * p.ju;
  }
  int g = 0;
  // merges 0 .. groups - lag - 2 hold a full group of up items and of down items
  const int full = p.groups - p.lag - 1;
  if (full > 0) {
    const int size = p.group * (p.ju + p.jd);
    if (s < full * size) {
      g = s / size;
      ffn_merge_item(p, g, s - g * size, p.group * p.ju, p.group * p.jd, kind, r, t);
      return;
    }
    s -= full * size;
    g = full;
  }
  for (; g < p.groups; ++g) {
    const int n_up = g + p.lag < p.groups ? ffn_group_rows(p, g + p.lag) * p.ju : 0;
    const int n_down = ffn_group_rows(p, g) * p.jd;
    if (s < n_up + n_down) {
      ffn_merge_item(p, g, s, n_up, n_down, kind, r, t);
      return;
    }
    s -= n_up + n_down;
  }
  kind = -1;  // past the end
  r = t = 0;
}

}  // namespace vfb
