/*
 * expf_ref.h — expf with the results of the reference's C library, on the
 * GPU and on the host.
 *
 * The reference calls glibc's expf (softmax, test_model_trace.c:485; SiLU,
 * :233). Since glibc 2.28 that function evaluates the published
 * table-and-polynomial method of Szabolcs Nagy (ARM optimized-routines,
 * "expf"): with N = 32,
 *   z  = x * N/ln2 (double),  k = round-to-nearest-even(z),
 *   r  = x * N/ln2 - k, computed as one fused multiply-add of the exact
 *        product (the library is built with contraction on x86-64),
 *   2^(k/N) = 2^(k div N) * 2^((k mod N)/N), the second factor from a table
 *        of the 32 doubles nearest 2^(j/32),
 *   2^(r/N) ~ 1 + c1 r + c2 r^2 + c3 r^3 (a cubic, minimax on |r| <= 1/2,
 *        evaluated in double), result rounded once to float,
 * with the special cases of the C standard outside the finite range.
 * expf_ref restates that method in double arithmetic. It is pinned by an
 * exhaustive comparison with glibc's expf over every finite float input
 * (tests/test_expf_cpu.py: no difference in 2^32 inputs), where a double
 * exp rounded once to float differs from glibc's expf in 170,648 of them.
 *
 * Include from CUDA or C. Device code uses the explicitly rounded
 * intrinsics; host code must be compiled with -ffp-contract=off.
 */
#ifndef MOE_EXPF_REF_H
#define MOE_EXPF_REF_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define MOE_EXPF_FN __host__ __device__ __forceinline__
#else
#define MOE_EXPF_FN static inline
#endif

/* the 32 doubles nearest 2^(j/32), j = 0..31 (tests/test_expf_cpu.py
 * recomputes them in exact rational arithmetic) */
#define MOE_EXP2_32_TABLE                                                       \
  {0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0,            \
   0x1.11301d0125b51p+0, 0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0,            \
   0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0, 0x1.306fe0a31b715p+0,            \
   0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,            \
   0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0,            \
   0x1.6247eb03a5585p+0, 0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0,            \
   0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0, 0x1.8ace5422aa0dbp+0,            \
   0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,            \
   0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0,            \
   0x1.cb720dcef9069p+0, 0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0,            \
   0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0}

#if defined(__CUDACC__)
static __device__ const double moe_exp2_32_dev[32] = MOE_EXP2_32_TABLE;
#endif
static const double moe_exp2_32_host[32] = MOE_EXP2_32_TABLE;

/* N/ln2 rounded to double, and the cubic's coefficients (r^3, r^2, r), each
 * already divided by the matching power of N = 32 (exact) */
#define MOE_EXPF_INVLN2N 0x1.71547652b82fep+5
#define MOE_EXPF_C3 (0x1.c6af84b912394p-5 / 32768.0)
#define MOE_EXPF_C2 (0x1.ebfce50fac4f3p-3 / 1024.0)
#define MOE_EXPF_C1 (0x1.62e42ff0c52d6p-1 / 32.0)

MOE_EXPF_FN float expf_ref(float x) {
#if defined(__CUDA_ARCH__)
  const uint32_t ux = __float_as_uint(x);
#else
  uint32_t ux;
  memcpy(&ux, &x, 4);
#endif
  const uint32_t ax = ux & 0x7fffffffu;
  if (ax >= 0x7f800000u) {                                  /* inf or NaN */
    if (ux == 0xff800000u) return 0.0f;                     /* exp(-inf) = 0 */
    return x + x;                                           /* +inf, NaN */
  }
  if (x > 0x1.62e42ep6f) return (float)INFINITY;            /* overflows */
  if (x < -0x1.9fe368p6f) return 0.0f;                      /* underflows to 0 */
  const double xd = (double)x;
#if defined(__CUDA_ARCH__)
  const double z = __dmul_rn(MOE_EXPF_INVLN2N, xd);
  const double kd = rint(z);
  const double r = __fma_rn(MOE_EXPF_INVLN2N, xd, -kd);
  const long long ki = (long long)kd;
  const int j = (int)(ki & 31);
  const double t = __ldg(moe_exp2_32_dev + j);
  const double p = __fma_rn(__fma_rn(MOE_EXPF_C3, r, MOE_EXPF_C2), __dmul_rn(r, r),
                            __fma_rn(MOE_EXPF_C1, r, 1.0));
  /* 2^((k - j)/32) * t by adding to t's exponent field (no overflow: the
     result's range is that of float) */
  const double s = __longlong_as_double(
      (long long)((unsigned long long)__double_as_longlong(t) + ((unsigned long long)(ki - j) << 47)));
  return __double2float_rn(__dmul_rn(p, s));
#else
  const double z = MOE_EXPF_INVLN2N * xd;
  const double kd = nearbyint(z);
  const double r = fma(MOE_EXPF_INVLN2N, xd, -kd);
  const long long ki = (long long)kd;
  const int j = (int)(ki & 31);
  const double t = moe_exp2_32_host[j];
  const double p = fma(fma(MOE_EXPF_C3, r, MOE_EXPF_C2), r * r, fma(MOE_EXPF_C1, r, 1.0));
  uint64_t tb;
  memcpy(&tb, &t, 8);
  tb += (uint64_t)(ki - j) << 47;   /* 2^((k - j)/32) * t via the exponent field */
  double s;
  memcpy(&s, &tb, 8);
  return (float)(p * s);
#endif
}

#endif /* MOE_EXPF_REF_H */
