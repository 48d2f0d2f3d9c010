// Work schedule of the persistent CTA-pair GEMM (k_gemm_pair): which output
// tiles and which k-block ranges each CTA pair processes. Shared by the kernel
// (device) and the launcher (host), so that both agree on the split, and
// checked exhaustively on the CPU by tests/native/sched_check.cpp; plain C++
// apart from the qualifiers.
//
// With T output tiles of KB k-blocks on P resident pairs, T / P full waves run
// data parallel (pair p takes tiles p, p + P, ...). When T is not a multiple of
// P the last wave holds only R = T % P tiles, and P - R pairs would idle while
// it runs (at 1024 rows per GPU: 64 down-projection tiles on 74 pairs, 13.5 %
// of the step). The tail split fills that wave:
//   * main pair H + r (r < R, H = P - R) computes k-blocks [0, kc) of
//     remainder tile r and finishes the tile;
//   * the remaining k-blocks [kc, KB) of every remainder tile are cut into S
//     equal parts, and the helper pairs 0 .. H-1 take the R * S parts in
//     contiguous runs. A helper writes each part's fp32 accumulator to its own slot in the
//     caller's workspace and raises a flag; the main pair waits for the S flags
//     of its tile, adds the slots in part order to its own accumulator (a fixed
//     order: the result does not depend on timing) and runs the epilogue.
// A main pair waits only on pairs with lower indices. The hardware dispatches
// a grid's CTAs in index order, so when a main is resident its helpers have
// been dispatched and finish without waiting on anything; this holds however
// many other kernels share the SMs (the rule that decoupled look-back scans
// rely on).
// All main pairs stream the same k rows of the shared weight panels at the same
// time, as the full waves do, so the weights still cross HBM about once; only
// the short tails [kc, KB) are re-read by the helpers, from L2. (A plain
// stream-K split, with contiguous k ranges cut across tile boundaries, lets the
// pairs that share a weight panel read it at different k offsets; with the
// 134 MB down-projection weights that defeats the 126 MB L2.)
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define TFB_SCHED_HD __host__ __device__ __forceinline__
#else
#define TFB_SCHED_HD inline
#endif

namespace tfb200::sched {

// Most helper parts (slots) one launch may use, and most parts per tile.
constexpr int kMaxSlots = 128;
constexpr int kMaxParts = 4;
// Shortest k range (in 64-deep k-blocks) a helper part or a main segment may have.
constexpr int kMinSegment = 4;
// Bytes of one slot: both CTAs' 128 x 256 fp32 accumulators.
constexpr int64_t kSlotBytes = 2 * 128 * 256 * 4;
// Flags of one slot: one counter per (CTA of the pair, epilogue warp, 32-column
// chunk of that warp), counting the rows written.
constexpr int kFlagsPerSlot = 2 * 8 * 4;

struct PairSched {
  int tiles = 0;    // T
  int kblocks = 0;  // KB
  int pairs = 1;    // P
  int waves = 0;    // full data-parallel waves (tail split) / 0 (plain grid stride)
  int rem = 0;      // R: tiles of the last wave (0 = no tail split)
  int parts = 0;    // S: helper parts per remainder tile
  int kc = 0;       // k-blocks [0, kc) of a remainder tile stay with its main pair
};

TFB_SCHED_HD int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// First k-block of tail part j (j = parts gives KB).
TFB_SCHED_HD int part_lo(const PairSched& s, int j) {
  return s.kc + static_cast<int>(static_cast<int64_t>(s.kblocks - s.kc) * j / s.parts);
}

// Helper h (pair h, 0 <= h < P - R) takes parts [part_begin(h), part_begin(h + 1)).
TFB_SCHED_HD int part_begin(const PairSched& s, int h) {
  const int helpers = s.pairs - s.rem;
  return static_cast<int>(static_cast<int64_t>(s.rem) * s.parts * h / helpers);
}

// k-blocks the busiest pair processes under schedule s.
TFB_SCHED_HD int64_t busiest(const PairSched& s) {
  if (s.rem == 0) return cdiv64(s.tiles, s.pairs) * s.kblocks;
  const int helpers = s.pairs - s.rem;
  const int64_t per_helper = cdiv64(static_cast<int64_t>(s.rem) * s.parts, helpers);
  const int64_t part_len = cdiv64(s.kblocks - s.kc, s.parts);
  const int64_t last = s.kc > per_helper * part_len ? s.kc : per_helper * part_len;
  return static_cast<int64_t>(s.waves) * s.kblocks + last;
}

// The schedule for T tiles of KB k-blocks on P pairs. max_slots = 0 (no
// workspace for the slots) gives the plain data-parallel grid stride. A split,
// or more parts per tile, is taken only when it shortens the busiest pair's
// k-block count by at least min_gain_permille of the count it replaces (the
// cost model leaves out the slots' write and read and the extra epilogues),
// and gives no helper more than max_per_helper parts. (Measured on B200 at
// 1024 x 16384 x 4096: helpers that ran 6-7 parts each streamed about 30 %
// slower than the main pairs, and the split launch took 116 us against 107 us
// without it; with one part per helper the splits of the other shapes gained.
// For the 1024-row down-projection, 64 tiles on 74 pairs, seven parts per
// helper would cut the busiest pair from 256 to 224 k-blocks, but the MLP step
// measured 212.5-212.9 us against 206.8-207.2 us without the split; at 2048
// rows four parts per helper gained 1.3-2.7 % (378-383 us against 388 us).)
TFB_SCHED_HD PairSched plan(int T, int KB, int P, int max_slots, int min_gain_permille = 20,
                            int max_per_helper = 1) {
  PairSched dp;
  dp.tiles = T;
  dp.kblocks = KB;
  dp.pairs = P > 0 ? P : 1;
  const int R = T % dp.pairs;
  if (R == 0 || max_slots <= 0 || T <= 0 || KB < 2 * kMinSegment) return dp;
  const int H = dp.pairs - R;
  PairSched best = dp;
  int64_t best_cost = busiest(dp);
  for (int S = 1; S <= kMaxParts; ++S) {
    if (static_cast<int64_t>(R) * S > max_slots || static_cast<int64_t>(R) * S > kMaxSlots) break;
    const int64_t per_helper = cdiv64(static_cast<int64_t>(R) * S, H);
    if (per_helper > max_per_helper) break;
    // Balance the main segment kc against a helper's per_helper parts of
    // (KB - kc) / S k-blocks: kc = per_helper * KB / (S + per_helper).
    const int64_t k0 = per_helper * KB / (S + per_helper);
    PairSched best_s = dp;
    int64_t cost_s = -1;
    for (int64_t kc = k0 - 1; kc <= k0 + 1; ++kc) {
      if (kc < kMinSegment || (KB - kc) / S < kMinSegment) continue;
      PairSched c = dp;
      c.waves = T / dp.pairs;
      c.rem = R;
      c.parts = S;
      c.kc = static_cast<int>(kc);
      const int64_t cost = busiest(c);
      if (cost_s < 0 || cost < cost_s) {
        best_s = c;
        cost_s = cost;
      }
    }
    if (cost_s >= 0 && cost_s < best_cost &&
        (best_cost - cost_s) * 1000 >= static_cast<int64_t>(min_gain_permille) * best_cost) {
      best = best_s;
      best_cost = cost_s;
    }
  }
  return best;
}

// Role of a work item in the epilogue.
enum Role : int { kFull = 0, kMain = 1, kPart = 2 };

struct Work {
  int tile, k0, k1, role, slot;  // slot: first slot of a main tile / the slot of a part
};

// Number of work items of pair p.
TFB_SCHED_HD int work_count(const PairSched& s, int p) {
  if (s.rem == 0) return p < s.tiles ? static_cast<int>((s.tiles - 1 - p) / s.pairs + 1) : 0;
  const int helpers = s.pairs - s.rem;
  if (p >= helpers) return s.waves + 1;
  return s.waves + part_begin(s, p + 1) - part_begin(s, p);
}

// Work item i (0 <= i < work_count(s, p)) of pair p, in the order the pair
// processes them.
TFB_SCHED_HD Work work_item(const PairSched& s, int p, int i) {
  Work w;
  if (s.rem == 0 || i < s.waves) {
    w.tile = p + i * s.pairs;
    w.k0 = 0;
    w.k1 = s.kblocks;
    w.role = kFull;
    w.slot = 0;
    return w;
  }
  const int base = s.waves * s.pairs;
  const int helpers = s.pairs - s.rem;
  if (p >= helpers) {
    const int r = p - helpers;
    w.tile = base + r;
    w.k0 = 0;
    w.k1 = s.kc;
    w.role = kMain;
    w.slot = r * s.parts;
    return w;
  }
  const int g = part_begin(s, p) + (i - s.waves);
  const int r = g / s.parts, j = g - r * s.parts;
  w.tile = base + r;
  w.k0 = part_lo(s, j);
  w.k1 = part_lo(s, j + 1);
  w.role = kPart;
  w.slot = g;
  return w;
}

// Workspace bytes for the slots and flags of one launch with T tiles (an
// upper bound that holds for any P: R * S <= min(kMaxSlots, T * kMaxParts)).
// The flags come first, 256-byte aligned.
TFB_SCHED_HD int64_t flag_bytes() { return (static_cast<int64_t>(kMaxSlots) * kFlagsPerSlot * 4 + 255) / 256 * 256; }
TFB_SCHED_HD int64_t slot_count(int64_t tiles) {
  const int64_t t = tiles * kMaxParts;
  return t < kMaxSlots ? t : kMaxSlots;
}
TFB_SCHED_HD int64_t region_bytes(int64_t tiles) { return flag_bytes() + slot_count(tiles) * kSlotBytes; }

}  // namespace tfb200::sched
