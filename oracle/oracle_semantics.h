/* oracle_semantics.h -- CPU definitions of the CUDA math the reference's
 * generated kernels call, for the C oracle.
 *
 * TEST INFRASTRUCTURE ONLY: included by the C that oracle/loom_oracle.py
 * generates; never part of the product path.
 *
 * - fmaf, sqrtf and IEEE division: glibc's are correctly rounded, as are
 *   CUDA's (nvcc defaults -prec-div=true -prec-sqrt=true), so these are used
 *   as is (bit-exact).
 * - fmaxf / fminf: CUDA's return the numeric operand when one is NaN and
 *   order -0.0 below +0.0; glibc's fmaxf(-0.0f, +0.0f) may return either
 *   zero, so both are restated here with CUDA's ordering.
 * - expf / logf: CUDA's implementations are not correctly rounded and differ
 *   from glibc's by up to their documented ulp bounds; bodies that use them
 *   are compared with a ulp tolerance, never bit-exactly.
 */
#ifndef LOOM_ORACLE_SEMANTICS_H
#define LOOM_ORACLE_SEMANTICS_H

#include <math.h>
#include <stdbool.h>
#include <stdint.h>

static inline float oracle_fmaxf(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  if (a == 0.0f && b == 0.0f) return (signbit(a) && signbit(b)) ? -0.0f : 0.0f;
  return a > b ? a : b;
}

static inline float oracle_fminf(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  if (a == 0.0f && b == 0.0f) return (signbit(a) || signbit(b)) ? -0.0f : 0.0f;
  return a < b ? a : b;
}

/* The CUDA fast-divide intrinsic is only rendered under a non-default flag;
 * the oracle evaluates it as IEEE division and such bodies use a tolerance. */
static inline float oracle_fdividef(float a, float b) { return a / b; }

#define fmaxf oracle_fmaxf
#define fminf oracle_fminf
#define __fdividef oracle_fdividef

/* Neumaier-compensated fp64 accumulation: the oracle's "fp64 reference sum". */
typedef struct {
  double sum;
  double comp;
} oracle_acc;

static inline void oracle_acc_add(oracle_acc* a, double v) {
  const double t = a->sum + v;
  if (!isfinite(t)) { /* inf/nan: plain IEEE accumulation, no compensation */
    a->sum = t;
    return;
  }
  if (fabs(a->sum) >= fabs(v))
    a->comp += (a->sum - t) + v;
  else
    a->comp += (v - t) + a->sum;
  a->sum = t;
}

static inline double oracle_acc_value(const oracle_acc* a) {
  return isfinite(a->sum) ? a->sum + a->comp : a->sum;
}

#endif
