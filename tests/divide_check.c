// The quantisation epilogues compute (float)dot / S with div_qscale
// (moe.cc_b200/csrc/common.cuh): Markstein's correction of the reciprocal product.
// This checks it against IEEE division for every int32 dot and both divisors.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
static inline uint32_t bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
int main(void) {
  const float Ss[2] = {127.0f, 7.0f};
  for (int si = 0; si < 2; ++si) {
    const float S = Ss[si];
    volatile float one = 1.0f;
    const float r = one / S;
    long long bad = 0;
    #pragma omp parallel for reduction(+:bad) schedule(static)
    for (long long i = -2147483648LL; i <= 2147483647LL; ++i) {
      const float x = (float)(int32_t)i;
      const float q = x / S;
      const float q0 = x * r;
      const float rem = fmaf(-q0, S, x);
      const float q1 = fmaf(rem, r, q0);
      if (bits(q) != bits(q1)) ++bad;
    }
    printf("S=%g: r=%a, mismatches over all int32: %lld\n", S, r, bad);
  }
  return 0;
}
