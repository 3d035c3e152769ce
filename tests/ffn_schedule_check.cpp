// Host check of the fused FFN work order (vflash_b200/csrc/ffn_plan.h): for a
// shape given on the command line, every up and down tile appears exactly
// once, and every down tile of a row block comes after all of that row
// block's up tiles.  Prints "ok <items>" or the first violation.
//   usage: ffn_schedule_check R ju jd group band_up band_down lead lag
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "ffn_plan.h"

int main(int argc, char **argv) {
  if (argc != 9) return 2;
  vfb::FfnPlan p{};
  p.rows_blocks = atoi(argv[1]);
  p.ju = atoi(argv[2]);
  p.jd = atoi(argv[3]);
  p.group = atoi(argv[4]);
  p.band_up = atoi(argv[5]);
  p.band_down = atoi(argv[6]);
  p.lead = atoi(argv[7]);
  p.lag = atoi(argv[8]);
  p.groups = (p.rows_blocks + p.group - 1) / p.group;
  p.total = p.rows_blocks * (p.ju + p.jd);
  std::vector<int> seen_up(static_cast<size_t>(p.rows_blocks) * p.ju, -1);
  std::vector<int> seen_down(static_cast<size_t>(p.rows_blocks) * p.jd, -1);
  std::vector<int> ups_done(p.rows_blocks, 0);
  for (int q = 0; q < p.total; ++q) {
    int kind, r, t;
    vfb::ffn_item(p, q, kind, r, t);
    if (r < 0 || r >= p.rows_blocks) { printf("item %d: row block %d out of range\n", q, r); return 1; }
    if (kind == vfb::kFfnUp) {
      if (t < 0 || t >= p.ju) { printf("item %d: up tile %d out of range\n", q, t); return 1; }
      int &slot = seen_up[static_cast<size_t>(r) * p.ju + t];
      if (slot >= 0) { printf("item %d: up (%d,%d) repeats item %d\n", q, r, t, slot); return 1; }
      slot = q;
      ++ups_done[r];
    } else if (kind == vfb::kFfnDown) {
      if (t < 0 || t >= p.jd) { printf("item %d: down tile %d out of range\n", q, t); return 1; }
      int &slot = seen_down[static_cast<size_t>(r) * p.jd + t];
      if (slot >= 0) { printf("item %d: down (%d,%d) repeats item %d\n", q, r, t, slot); return 1; }
      slot = q;
      if (ups_done[r] != p.ju) { printf("item %d: down (%d,%d) before all up tiles\n", q, r, t); return 1; }
    } else {
      printf("item %d: no item\n", q);
      return 1;
    }
  }
  int kind, r, t;
  vfb::ffn_item(p, p.total, kind, r, t);
  if (kind != -1) { printf("item past the end decoded\n"); return 1; }
  printf("ok %d\n", p.total);
  return 0;
}
