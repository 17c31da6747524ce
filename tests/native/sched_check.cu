// Host-side check of the persistent GEMM work schedule (WorkSched in
// kernels.cuh) over a sweep of shapes.  Built with nvcc and run on the CPU by
// tests/test_sched_cpu.py; it launches nothing.
//
// For every (token tiles, weight tiles, iterations per unit, workers) it checks
// what the grouped GEMM kernels rely on:
//   * each (unit, iteration) pair is run by exactly one worker, in ascending
//     iteration order inside a worker's share of a unit;
//   * a phase-1 unit (r < 0) is run whole by one worker;
//   * the workers with iterations in a phase-2 unit are exactly
//     first_cta..last_cta, with no empty share among them, so the arrival
//     counter's last contributor is the one that sees old == last - first;
//   * a worker whose share of a unit is not the whole unit publishes it in a
//     slot no other unit of that worker uses;
//   * unit_tile maps units one to one onto (token tile, weight tile).
#include <cstdio>
#include <vector>

#include "kernels.cuh"

using moe::WorkSched;

static int check(int n_mt, int NT, int ITERS, int G) {
  const int units = n_mt * NT;
  std::vector<int> runs((size_t)units * ITERS, 0);
  std::vector<int> first_seen(units, -1), last_seen(units, -1), n_workers(units, 0);
  std::vector<int> whole(units, 0);
  for (int g = 0; g < G; ++g) {
    const WorkSched s = moe::make_work_sched_for(n_mt, NT, ITERS, G, g);
    int prev_u = -1, prev_a = -1, seg_a0 = -1;
    int slot_unit[2] = {-1, -1};
    const int n = s.n_iter();
    if (n < 0) return printf("negative iteration count g=%d\n", g), 1;
    for (int i = 0; i < n; ++i) {
      int u, a, r;
      s.at(i, ITERS, u, a, r);
      if (u < 0 || u >= units || a < 0 || a >= ITERS)
        return printf("out of range u=%d a=%d (g=%d i=%d)\n", u, a, g, i), 1;
      if (s.unit_of(i, ITERS) != u) return printf("unit_of disagrees\n"), 1;
      ++runs[(size_t)u * ITERS + a];
      if (u == prev_u) {
        if (a != prev_a + 1) return printf("iterations out of order u=%d\n", u), 1;
      } else {
        seg_a0 = a;
        if (first_seen[u] < 0) first_seen[u] = g;
        if (last_seen[u] >= 0 && last_seen[u] != g - 1 && last_seen[u] != g)
          return printf("contributors of unit %d not contiguous\n", u), 1;
        last_seen[u] = g;
        ++n_workers[u];
      }
      const bool unit_end = (i + 1 == n) || s.unit_of(i + 1, ITERS) != u;
      if (unit_end) {
        const bool full = seg_a0 == 0 && a == ITERS - 1;
        if (r < 0 && !full) return printf("phase-1 unit %d split\n", u), 1;
        if (full) ++whole[u];
        if (!full) {
          if (r != u - s.Wf * G) return printf("phase-2 index mismatch\n"), 1;
          const int sl = s.slot(g, r, ITERS);
          if (sl < 0 || sl > 1) return printf("bad slot\n"), 1;
          if (slot_unit[sl] >= 0 && slot_unit[sl] != u)
            return printf("slot %d reused by worker %d (units %d, %d)\n", sl, g, slot_unit[sl], u), 1;
          slot_unit[sl] = u;
          if (g < s.first_cta(r, ITERS) || g > s.last_cta(r, ITERS))
            return printf("worker %d outside first..last of unit %d\n", g, u), 1;
        }
      }
      prev_u = u;
      prev_a = a;
    }
  }
  for (size_t k = 0; k < runs.size(); ++k)
    if (runs[k] != 1) return printf("unit %zu iteration %zu run %d times\n", k / ITERS, k % ITERS, runs[k]), 1;
  const WorkSched s0 = moe::make_work_sched_for(n_mt, NT, ITERS, G, 0);
  for (int u = 0; u < units; ++u) {
    if (whole[u]) {
      if (n_workers[u] != 1) return printf("whole unit %d has %d workers\n", u, n_workers[u]), 1;
      continue;
    }
    const int r = u - s0.Wf * G;
    if (r < 0) return printf("phase-1 unit %d not whole\n", u), 1;
    const int lo = s0.first_cta(r, ITERS), hi = s0.last_cta(r, ITERS);
    if (lo != first_seen[u] || hi != last_seen[u] || n_workers[u] != hi - lo + 1)
      return printf("unit %d: contributors %d..%d (%d), schedule says %d..%d\n", u, first_seen[u],
                    last_seen[u], n_workers[u], lo, hi), 1;
  }
  std::vector<int> hit(units, 0);
  for (int u = 0; u < units; ++u) {
    const int2 t = moe::unit_tile(u, n_mt, NT);
    if (t.x < 0 || t.x >= n_mt || t.y < 0 || t.y >= NT) return printf("unit_tile out of range\n"), 1;
    if (hit[t.x * NT + t.y]++) return printf("unit_tile not one to one\n"), 1;
  }
  return 0;
}

int main() {
  // Weight tiles per token tile of the kernels: 16 (GEMM1, 128 feature rows of
  // X1 and X2), 56 (GEMM2, 128 output rows); iterations per unit: K steps or
  // K atoms (7168/128 = 56, 7168/64 = 112, 2048/128 = 16, 2048/64 = 32, ...).
  const int nts[] = {1, 7, 16, 56};
  const int iters[] = {1, 2, 3, 16, 28, 32, 56, 112};
  const int workers[] = {1, 2, 3, 74, 148, 296};
  long cases = 0;
  for (int NT : nts)
    for (int IT : iters)
      for (int G : workers)
        for (int n_mt = 1; n_mt <= 160; n_mt += (n_mt < 24 ? 1 : 17)) {
          if (check(n_mt, NT, IT, G)) {
            printf("FAILED n_mt=%d NT=%d ITERS=%d G=%d\n", n_mt, NT, IT, G);
            return 1;
          }
          ++cases;
        }
  printf("OK %ld schedules\n", cases);
  return 0;
}
