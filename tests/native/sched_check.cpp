// Exhaustive check of the CTA-pair GEMM's work schedule (csrc/pair_sched.h),
// run by tests/test_sched_cpu.py: for every (tiles, k-blocks, pairs) in the
// given ranges, each (tile, k-block) is computed by exactly one work item; a
// split tile's main pair owns k-blocks [0, kc) and lists exactly the slots its
// helpers write; every slot is written once; the busiest pair's load matches
// busiest(). Prints one summary line per checked shape family and exits 1 on
// the first violation.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <vector>

#include "../../tt-flow_b200/csrc/pair_sched.h"

using namespace tfb200::sched;

static int fail(const char* what, int T, int KB, int P) {
  std::printf("FAIL %s (T=%d KB=%d P=%d)\n", what, T, KB, P);
  return 1;
}

static int check(int T, int KB, int P, int max_slots, int gain, int per_helper) {
  const PairSched s = plan(T, KB, P, max_slots, gain, per_helper);
  if (s.tiles != T || s.kblocks != KB || s.pairs != P) return fail("plan echoes its problem", T, KB, P);
  if (s.rem) {
    if (s.rem != T % P || s.parts < 1 || s.parts > kMaxParts || s.rem * s.parts > max_slots)
      return fail("split parameters", T, KB, P);
    if (s.kc < kMinSegment || s.kc >= KB) return fail("main segment", T, KB, P);
    for (int j = 0; j < s.parts; ++j)
      if (part_lo(s, j + 1) - part_lo(s, j) < kMinSegment) return fail("part length", T, KB, P);
  }
  std::vector<int> cover(static_cast<size_t>(T) * KB, 0);
  std::vector<int> slot_writes(kMaxSlots * kMaxParts + 1, 0);
  std::map<int, int> main_first_slot;  // tile -> first slot
  int64_t busiest_seen = 0;
  std::map<int, int> tile_main;  // split tile -> its main pair
  std::vector<std::pair<int, int>> part_writers;  // (tile, helper pair)
  for (int p = 0; p < P; ++p) {
    const int n = work_count(s, p);
    int64_t load = 0;
    for (int i = 0; i < n; ++i) {
      const Work w = work_item(s, p, i);
      if (w.role == kMain) tile_main[w.tile] = p;
      if (w.role == kPart) part_writers.push_back({w.tile, p});
      if (w.tile < 0 || w.tile >= T || w.k0 < 0 || w.k1 > KB || w.k0 >= w.k1) return fail("item range", T, KB, P);
      for (int k = w.k0; k < w.k1; ++k) ++cover[static_cast<size_t>(w.tile) * KB + k];
      load += w.k1 - w.k0;
      if (w.role == kMain) {
        if (w.k0 != 0 || w.k1 != s.kc) return fail("main item", T, KB, P);
        main_first_slot[w.tile] = w.slot;
      } else if (w.role == kPart) {
        if (w.slot < 0 || w.slot >= s.rem * s.parts) return fail("slot index", T, KB, P);
        ++slot_writes[w.slot];
        // the slot belongs to this tile's main: slots [r * S, r * S + S)
        if (w.slot / s.parts != w.tile - s.waves * s.pairs) return fail("slot/tile", T, KB, P);
        if (w.k0 != part_lo(s, w.slot % s.parts)) return fail("part k range", T, KB, P);
      } else if (w.k0 != 0 || w.k1 != KB) {
        return fail("full item", T, KB, P);
      }
    }
    if (load > busiest_seen) busiest_seen = load;
  }
  for (int v : cover)
    if (v != 1) return fail("coverage", T, KB, P);
  // a main pair waits only on pairs with lower indices
  for (auto& tw : part_writers)
    if (tw.second >= tile_main[tw.first]) return fail("helper index not below its main", T, KB, P);
  for (int g = 0; g < s.rem * s.parts; ++g)
    if (slot_writes[g] != 1) return fail("slot written once", T, KB, P);
  for (int r = 0; r < s.rem; ++r) {
    auto it = main_first_slot.find(s.waves * s.pairs + r);
    if (it == main_first_slot.end() || it->second != r * s.parts) return fail("main slots", T, KB, P);
  }
  if (busiest_seen > busiest(s)) return fail("busiest bound", T, KB, P);
  // never worse than the plain grid stride
  if (busiest(s) > cdiv64(T, P) * KB) return fail("worse than data parallel", T, KB, P);
  return 0;
}

int main(int argc, char** argv) {
  const int tmax = argc > 1 ? std::atoi(argv[1]) : 600;
  long checked = 0;
  const int kbs[] = {1, 2, 7, 8, 9, 16, 17, 63, 64, 65, 128, 256, 448};
  const int pairs[] = {1, 2, 3, 37, 73, 74};
  const int slots[] = {0, 1, 8, 128};
  for (int per_helper : {1, 1 << 20})
    for (int gain : {0, 20})
      for (int P : pairs)
        for (int KB : kbs)
          for (int ms : slots)
            for (int T = 1; T <= tmax; ++T) {
              if (check(T, KB, P, ms, gain, per_helper)) return 1;
              ++checked;
            }
  // The shapes of the benchmark workloads at 1024..8192 rows per GPU on 74 pairs.
  struct { int T, KB; } named[] = {{256, 64}, {64, 256}, {96, 64}, {512, 64}, {128, 256}, {192, 64},
                                   {1024, 64}, {256, 256}, {384, 64}, {2048, 64}, {512, 256}, {768, 64}};
  for (auto& n : named) {
    const PairSched s = plan(n.T, n.KB, 74, static_cast<int>(slot_count(n.T)), argc > 2 ? std::atoi(argv[2]) : 20,
                               argc > 3 ? std::atoi(argv[3]) : 1);
    const double ideal = static_cast<double>(n.T) * n.KB / 74.0;
    std::printf("T=%d KB=%d: rem=%d parts=%d kc=%d busiest=%lld dp=%lld ideal=%.1f balance=%.3f\n", n.T, n.KB, s.rem,
                s.parts, s.kc, static_cast<long long>(busiest(s)), static_cast<long long>(cdiv64(n.T, 74) * n.KB),
                ideal, ideal / static_cast<double>(busiest(s)));
  }
  std::printf("OK %ld schedules\n", checked);
  return 0;
}
