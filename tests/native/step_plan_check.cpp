// Checks the decode-step kernel's work partition (qweninfer_b200/csrc/step_plan.h) on the
// host: every (8-row group, k block) cell of every projection is multiplied by exactly
// one CTA, no ring slot holds more than kSlotKB KB of pieces, no piece straddles a tile,
// layer projections give a CTA at most two tiles (the TMEM budget), K = 896 shares span
// the whole of K and the head has one tile per accumulation unit; the attention and reduce units are each owned by one CTA.
// Prints "ok" or the first violation (exit code 1).
#include <cstdio>
#include <vector>

#include "../../qweninfer_b200/csrc/step_plan.h"

using namespace qi::step;

static int fail(const char* what, int a, int b) {
  std::printf("FAIL %s (%d, %d)\n", what, a, b);
  return 1;
}

int main() {
  const int vocab = 151936;
  for (int op : {kQkv, kO, kGateUp, kDown, kHead}) {
    const int G = op_groups(op, vocab), KB = op_kblocks(op);
    std::vector<int> cover((size_t)G * KB, 0);
    for (int cta = 0; cta < kGrid; ++cta) {
      const Part P = part_of(op, cta, vocab);
      if (P.empty()) continue;
      if (P.g0 < 0 || P.g1 > G || P.kb0 < 0 || P.kb1 > KB) return fail("share out of range", op, cta);
      if (op != kHead && P.ntiles() > kMaxLayerTiles) return fail("more than two tiles", op, cta);
      if (op != kDown && (P.kb0 != 0 || P.kb1 != KB)) return fail("a K = 896 share is not the whole of K", op, cta);
      std::vector<int> slot_kb(4096, 0);
      int units_first = 0, units_last = 0, last_slot = -1;
      const int n = for_each_piece(P, 0, [&](const Piece& pc, int slot, int off, bool first, bool last) {
        const int mt = P.tile0() + pc.u;
        if (pc.lo < 0 || pc.hi > 16 || pc.lo >= pc.hi) throw 1;
        if (slot < last_slot) throw 2;
        last_slot = slot;
        if (off != slot_kb[slot]) throw 3;
        slot_kb[slot] += pc.kbytes();
        for (int g = 16 * mt + pc.lo; g < 16 * mt + pc.hi; ++g) cover[(size_t)g * KB + pc.kb] += 1;
        units_first += first;
        units_last += last;
      });
      for (int s = 0; s < n; ++s)
        if (slot_kb[s] <= 0 || slot_kb[s] > kSlotKB) return fail("slot fill", op, cta);
      if (units_first != units_of(P) || units_last != units_of(P)) return fail("unit boundaries", op, cta);
    }
    for (size_t i = 0; i < cover.size(); ++i)
      if (cover[i] != 1) return fail("cell not covered exactly once", op, (int)i);
  }
  // attention units: each (t, g, split) on exactly one CTA
  for (int M : {1, 7, 22, 32})
    for (int splits : {1, 4, 16}) {
      std::vector<int> seen(splits * 2 * M, 0);
      for (int cta = 0; cta < kGrid; ++cta)
        for (int u = attn_first_unit(cta); u < splits * 2 * M; u += kGrid) {
          if (attn_cta(u) != cta) return fail("attention unit owner", u, cta);
          seen[u] += 1;
        }
      for (int v : seen)
        if (v != 1) return fail("attention unit coverage", M, splits);
    }
  std::printf("ok\n");
  return 0;
}
