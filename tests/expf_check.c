/* Exhaustive check of expf_ref (moe.cc_b200/csrc/expf_ref.h, host form)
 * against the C library's expf over every float bit pattern; NaN results
 * compare as equal whatever their payload. Also prints the count of inputs
 * where a double exp rounded once to float differs from the library. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../moe.cc_b200/csrc/expf_ref.h"

int main(void) {
  long long bad = 0, bad_double = 0;
#pragma omp parallel for reduction(+ : bad, bad_double) schedule(dynamic, 65536)
  for (long long u = 0; u < (1LL << 32); ++u) {
    const uint32_t b = (uint32_t)u;
    float x;
    memcpy(&x, &b, 4);
    const float g = expf(x), m = expf_ref(x), d = (float)exp((double)x);
    if (!(isnan(g) && isnan(m)) && memcmp(&g, &m, 4) != 0) ++bad;
    if (!(isnan(g) && isnan(d)) && memcmp(&g, &d, 4) != 0) ++bad_double;
  }
  printf("expf_ref mismatches: %lld\n", bad);
  printf("double exp rounded once, mismatches: %lld\n", bad_double);
  for (int j = 0; j < 32; ++j) printf("t%d=%a\n", j, moe_exp2_32_host[j]);
  return 0;
}
