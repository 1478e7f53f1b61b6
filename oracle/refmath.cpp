// refmath.cpp -- test infrastructure: evaluates the REFERENCE's pinned
// functions (code/cis2-fp/gpu/cis2_math.h, compiled from where it lies) on
// the sweep of oracle/math_sweep.h under the reference's FTZ/DAZ pin
// (cis2_fpenv.h), and writes one record per point:
//   "CIS2MSW1" (8 bytes), u32 n, then n x (u32 x, u32 exp, sin, cos, ln, silu, rsqrt)
// little-endian, function order as the reference sweep's golden file
// (code/cis2-fp/src/bin/math_dump.rs:254-262).
//
//   refmath OUT.bin
#include "cis2_fpenv.h"
#include "cis2_math.h"
#include "math_sweep.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

static float ref_ln(float x) { return cis2_ln_pinned(x); }
static float ref_exp(float x) { return cis2_exp_pinned(x); }

int main(int argc, char **argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: refmath OUT.bin\n");
    return 2;
  }
  cis2_fpenv_init();
  const size_t n = cis2_math_sweep_inputs(nullptr, ref_ln, ref_exp);
  std::vector<float> x(n);
  cis2_math_sweep_inputs(x.data(), ref_ln, ref_exp);
  FILE *f = fopen(argv[1], "wb");
  if (!f) {
    fprintf(stderr, "cannot write %s\n", argv[1]);
    return 2;
  }
  fwrite("CIS2MSW1", 1, 8, f);
  const uint32_t n32 = (uint32_t)n;
  fwrite(&n32, 4, 1, f);
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float out[7] = {v, cis2_exp_pinned(v), cis2_sin_pinned(v), cis2_cos_pinned(v), cis2_ln_pinned(v),
                          cis2_silu_pinned(v), cis2_rsqrt_cr(v)};
    uint32_t rec[7];
    memcpy(rec, out, sizeof rec);
    fwrite(rec, 4, 7, f);
  }
  fclose(f);
  fprintf(stderr, "refmath: %zu points\n", n);
  return 0;
}
