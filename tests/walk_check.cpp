// Host check of the hardware walk order (csrc/tb_mapping.h), built and run
// by tests/test_walk_order.py: for every mapping kind and pairing the walk
// must visit each work item exactly once, and a fused item must still cover
// two adjacent tiles (same programs as the reference's pids).
#include <cstdio>
#include <vector>

#include "tb_mapping.h"

using namespace tb;

static int check(int tiles_m, int tiles_n, int group_m, int kind, int fuse) {
  MappingArgs a{};
  a.kind = kind;
  a.tiles_m = tiles_m;
  a.tiles_n = tiles_n;
  a.tiles_k = 4;
  a.split_k = 1;
  if (kind == kMapGroupedTile) {
    a.group_span_m = group_m < tiles_m ? group_m : tiles_m;
    a.programs_per_group = a.group_span_m * tiles_n;
  } else {
    a.group_span_m = 1;
    a.programs_per_group = tiles_n;
  }
  a.total_programs = tiles_m * tiles_n;
  const int items = fuse == 4 ? a.total_programs / 4 : fuse ? a.total_programs / 2 : a.total_programs;
  const int mode = walk_mode(a, fuse);
  std::vector<int> seen(a.total_programs, 0);
  for (int w = 0; w < items; ++w) {
    const int it = walk_item(a, fuse, mode, w);
    if (it < 0 || it >= items) return 1;
    const int p0 = item_first_pid(a, fuse, it);
    const Work x = program_work(a, p0);
    ++seen[p0];
    if (fuse == 4) {
      const int rows = a.tiles_m - (x.tile_m / a.group_span_m) * a.group_span_m < a.group_span_m
                           ? a.tiles_m - (x.tile_m / a.group_span_m) * a.group_span_m
                           : a.group_span_m;
      const int ps[3] = {p0 + 1, p0 + rows, p0 + rows + 1};
      const int dm[3] = {1, 0, 1}, dn[3] = {0, 1, 1};
      if (x.tile_m % 2 != 0 || x.tile_n % 2 != 0) return 5;
      for (int j = 0; j < 3; ++j) {
        const Work y = program_work(a, ps[j]);
        ++seen[ps[j]];
        if (y.tile_m != x.tile_m + dm[j] || y.tile_n != x.tile_n + dn[j]) return 6;
      }
      continue;
    }
    if (fuse) {
      int p1 = p0 + 1;
      if (fuse == 3) {
        const int first = (x.tile_m / a.group_span_m) * a.group_span_m;
        const int left = a.tiles_m - first;
        p1 = p0 + (left < a.group_span_m ? left : a.group_span_m);
      }
      const Work y = program_work(a, p1);
      ++seen[p1];
      if (fuse == 1 && !(y.tile_m == x.tile_m + 1 && y.tile_n == x.tile_n)) return 2;
      if (fuse >= 2 && !(y.tile_n == x.tile_n + 1 && y.tile_m == x.tile_m && x.tile_n % 2 == 0)) return 3;
    }
  }
  for (int v : seen)
    if (v != 1) return 4;
  return 0;
}

int main() {
  int cases = 0;
  for (int tm = 1; tm <= 20; ++tm)
    for (int tn = 1; tn <= 20; ++tn)
      for (int g : {1, 2, 3, 8}) {
        int r;
        if ((r = check(tm, tn, g, kMapGroupedTile, 0))) { printf("FAIL grouped %d %d %d: %d\n", tm, tn, g, r); return 1; }
        const int span = g < tm ? g : tm;
        if (span % 2 == 0 && tm % 2 == 0 && (r = check(tm, tn, g, kMapGroupedTile, 1))) {
          printf("FAIL grouped-vertical %d %d %d: %d\n", tm, tn, g, r);
          return 1;
        }
        if (tn % 2 == 0 && (r = check(tm, tn, g, kMapGroupedTile, 3))) {
          printf("FAIL grouped-horizontal %d %d %d: %d\n", tm, tn, g, r);
          return 1;
        }
        if (span % 2 == 0 && tm % 2 == 0 && tn % 2 == 0 && (r = check(tm, tn, g, kMapGroupedTile, 4))) {
          printf("FAIL grouped-2x2 %d %d %d: %d\n", tm, tn, g, r);
          return 1;
        }
        cases += 3;
      }
  for (int tm = 1; tm <= 30; ++tm)
    for (int tn = 1; tn <= 30; ++tn)
      for (int kind : {(int)kMapTile, (int)kMapPersistentTile}) {
        int r;
        if ((r = check(tm, tn, 1, kind, 0))) { printf("FAIL rowmajor %d %d: %d\n", tm, tn, r); return 1; }
        if (tn % 2 == 0 && (r = check(tm, tn, 1, kind, 2))) { printf("FAIL horizontal %d %d: %d\n", tm, tn, r); return 1; }
        cases += 2;
      }
  printf("OK %d\n", cases);
  return 0;
}
