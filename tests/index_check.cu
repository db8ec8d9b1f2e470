// Host-side check of the tile-list index arithmetic of the 16-bit kernels:
// list_tile, padding_share and list_padded_role from fst_tc_common.cuh,
// compiled for the host and driven over thousands of random padded batches
// exactly as a launch would (grid = valid_rows / bm + B + pad_ctas CTAs,
// CTA t of g). It checks that every row a padding writer or a NaN fill
// touches lies inside its event's [0, max_len) rows, that every padding row
// is written exactly once, that every live block is computed by exactly one
// CTA, and that a valid_rows too small for the grid turns every valid row
// into NaN instead of leaving rows unwritten. Any violation would be an
// out-of-range store on the GPU. Built and run by tests/test_index_math.py.

#include <algorithm>
#include <cstdio>
#include <random>
#include <vector>

#include "../flash-spacetime_b200/csrc/fst_tc_common.cuh"

namespace {

int fail(int trial, const char* what, int b, int r) {
  std::printf("FAIL trial %d: %s (event %d, row %d)\n", trial, what, b, r);
  return 1;
}

}  // namespace

int main() {
  std::mt19937 rng(2026);
  auto uni = [&](int lo, int hi) { return std::uniform_int_distribution<int>(lo, hi)(rng); };
  int checked = 0, poisoned = 0;
  for (int trial = 0; trial < 6000; ++trial) {
    const int B = uni(1, 48), L = uni(1, 400), bm = uni(0, 1) ? 16 : 32, H = uni(1, 20);
    std::vector<int> lens(B);
    for (int& n : lens) {
      const int kind = uni(0, 3);
      n = kind == 0 ? 0 : (kind == 1 ? L : uni(0, L));
    }
    // Event order: natural, a random permutation, or stable longest first.
    std::vector<int> order(B);
    for (int i = 0; i < B; ++i) order[i] = i;
    const int okind = uni(0, 2);
    if (okind == 1) std::shuffle(order.begin(), order.end(), rng);
    if (okind == 2)
      std::stable_sort(order.begin(), order.end(),
                       [&](int x, int y) { return lens[x] > lens[y]; });
    // The workspace tile_prefix writes: tile prefix [B + 1] in event order,
    // then the padding-row prefix [B + 1] in natural order.
    std::vector<int> ws(2 * (B + 1));
    for (int k = 0; k < B; ++k) ws[k + 1] = ws[k] + (lens[order[k]] + bm - 1) / bm;
    for (int b = 0; b < B; ++b) ws[B + 2 + b] = ws[B + 1 + b] + (L - lens[b]);
    int64_t sum = 0;
    for (int n : lens) sum += n;

    FstProblem p{};
    p.packed = 0;
    p.batch = B;
    p.heads = H;
    p.max_len = L;
    p.head_dim = 32;
    p.channels = 16;
    p.total_rows = (int64_t)B * L;
    p.seqlens = lens.data();
    p.event_order = okind ? order.data() : nullptr;
    // A valid_rows hint: the exact sum or a little above (the normal case),
    // or anything from 1 up (possibly too small for the grid).
    p.valid_rows = uni(0, 4) ? sum + uni(0, 5) : uni(1, (int)(sum > 1 ? sum : 1));
    if (!fst::list_padding(p)) continue;  // the full (L / bm, B) grid: not this path
    ++checked;

    const int writers = fst::pad_ctas(p, 68);
    const int g = (int)((p.valid_rows + bm - 1) / bm + B + writers);
    const int n_tiles = ws[B];
    std::vector<int> zero_hits((size_t)B * L), nan_hits((size_t)B * L), tile_hits(n_tiles);
    int bad = 0, bad_b = -1, bad_r = -1;
    auto fill = [&](int b, int r0, int r1, int nan) {
      if (b < 0 || b >= B || r0 < 0 || r0 > r1 || r1 > L) {
        bad = 1;
        bad_b = b;
        bad_r = r0;
        return;
      }
      for (int r = r0; r < r1; ++r) ++(nan ? nan_hits : zero_hits)[(size_t)b * L + r];
    };
    bool any_poisoned = false;
    for (int t = 0; t < g; ++t) {
      const int role = fst::tc::list_padded_role(p, ws.data(), bm, writers, t, g, fill);
      if (bad) return fail(trial, "fill outside the event's rows", bad_b, bad_r);
      if (role == fst::tc::kRolePoisoned) any_poisoned = true;
      if (role < 0) continue;
      int b = -1, blk = -1;
      if (!fst::tc::list_tile(p, ws.data(), role, b, blk)) continue;  // past the list
      if (b < 0 || b >= B || blk * bm >= lens[b])
        return fail(trial, "tile outside its event", b, blk);
      ++tile_hits[role];
    }
    const bool too_small = n_tiles >= g;  // no CTA left for the padding writers
    if (any_poisoned != too_small)
      return fail(trial, "poisoned iff the grid is too small", -1, -1);
    poisoned += too_small;
    for (int b = 0; b < B; ++b)
      for (int r = 0; r < L; ++r) {
        const int z = zero_hits[(size_t)b * L + r], nn = nan_hits[(size_t)b * L + r];
        if (r >= lens[b] && (z != 1 || nn != 0))
          return fail(trial, "padding row not written once", b, r);
        if (r < lens[b] && z != 0) return fail(trial, "valid row zeroed", b, r);
        if (r < lens[b] && nn != (too_small ? 1 : 0))
          return fail(trial, "valid row NaN count", b, r);
      }
    for (int t = 0; t < n_tiles; ++t)
      if (tile_hits[t] != (too_small ? 0 : 1))
        return fail(trial, "live block not computed once", -1, t);
  }
  std::printf("ok: %d padded tile-list problems checked, %d with a too-small valid_rows\n",
              checked, poisoned);
  return checked > 0 && poisoned > 0 ? 0 : 1;
}
