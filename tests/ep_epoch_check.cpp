// Host-side check of the expert-parallel combine epoch arithmetic
// (ep_epoch / ep_reached in strataflow_b200/csrc/sfk_kernels.cuh), built with
// g++ by tests/test_ep_epoch.py.  Walks the step counter across the signed
// and unsigned 32-bit limits at 61 layers (the ~1T shape) and checks that a
// flag holding the previous epoch is never taken for the current one, that the
// current epoch is always taken, and that epochs stay strictly increasing in
// the wrapped order.
#include <cstdio>
#include <climits>
#include "sfk_kernels.cuh"

int main() {
  using sfk::ep_epoch;
  using sfk::ep_reached;
  const int n_layer = 61;
  const unsigned starts[] = {1u, (unsigned)INT_MAX / (2u * n_layer) - 2u, (unsigned)INT_MAX / (2u * n_layer) + 2u,
                             UINT_MAX / (2u * n_layer) - 2u, UINT_MAX / (2u * n_layer) + 2u};
  long checks = 0;
  for (unsigned s0 : starts) {
    unsigned prev = ep_epoch(s0 - 1u, n_layer, n_layer - 1, 1);
    for (unsigned step = s0; step != s0 + 6u; ++step)
      for (int l = 0; l < n_layer; ++l)
        for (int st = 0; st < 2; ++st) {
          const unsigned e = ep_epoch(step, n_layer, l, st);
          if (!ep_reached(e, e)) { printf("FAIL reached(e,e) step=%u l=%d\n", step, l); return 1; }
          if (ep_reached(prev, e)) { printf("FAIL stale flag taken step=%u l=%d\n", step, l); return 1; }
          if (!ep_reached(e, prev)) { printf("FAIL order step=%u l=%d\n", step, l); return 1; }
          if (e - prev != 1u) { printf("FAIL gap step=%u l=%d\n", step, l); return 1; }
          prev = e;
          ++checks;
        }
  }
  // a peer one whole step ahead still counts as having reached this epoch
  const unsigned e = ep_epoch(UINT_MAX / (2u * n_layer), n_layer, 3, 0);
  if (!ep_reached(e + 2u * n_layer, e)) { printf("FAIL ahead\n"); return 1; }
  printf("ok %ld\n", checks);
  return 0;
}
