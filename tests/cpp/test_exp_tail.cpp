// Host check of exp_tail (the exact-tail exponential of the list kernel's
// refinements) against long-double expl: prints the largest relative error
// over a sweep of float arguments in (-700, 0] and exits non-zero above 2^-51.
#include <cmath>
#include <cstdio>
#include <random>

#include "../../mlx-confucius4-tts_b200/csrc/c4s_exp.cuh"

static const double kTab[64] = C4S_EXP2_J64_TABLE;

int main() {
  long double worst = 0.0L;
  float worst_d = 0.0f;
  auto check = [&](float d) {
    const double e = c4s::exp_tail(d, kTab);
    const long double ref = expl((long double)d);
    const long double rel = fabsl(((long double)e - ref) / ref);
    if (rel > worst) { worst = rel; worst_d = d; }
  };
  std::mt19937_64 g(20260101);
  std::uniform_real_distribution<double> wide(-699.99, 0.0), narrow(-2.0, 0.0);
  for (int i = 0; i < 2000000; ++i) check((float)wide(g));
  for (int i = 0; i < 2000000; ++i) check((float)narrow(g));
  // every float in [-1/64, 0] that is a multiple of 2^-30, and around the
  // reduction's half-way points (k + 1/2) ln2/64
  for (int i = 0; i <= (1 << 24); ++i) check(-(float)i * 0x1p-30f);
  for (int k = 0; k < 64 * 40; ++k) {
    const float c = -(float)((k + 0.5) * 0.010830424696249145);
    float lo = c, hi = c;
    for (int s = 0; s < 64; ++s) { check(lo); check(hi); lo = nextafterf(lo, -1e9f); hi = nextafterf(hi, 0.0f); }
  }
  check(0.0f);
  check(-0.0f);
  check(-699.9f);
  printf("max_rel_err %.6Le at d=%a (bound 2^-51 = %.6e)\n", worst, (double)worst_d, std::ldexp(1.0, -51));
  return worst <= 0x1p-51L ? 0 : 1;
}
