/*
 * fw_oracle.c -- C restatement of the FW-loss threshold search.
 * TEST INFRASTRUCTURE ONLY: used by tests/ as a fast checker and by bench.py
 * as the CPU baseline when the reference's own CPU code (oracle/_ref) is not
 * built.  Never linked into the product.
 *
 * Per row (reference_impl.py:11-26, in float64 and in the shifted form of
 * oracle/fw_oracle.py:fw_shifted_fp64):
 *   M = max z;  d = z - M sorted descending;  S_k = d_1 + ... + d_k;
 *   tau = max_k (S_k - 1)/k (first maximal k) = h* - M;  kappa = that k;
 *   loss = 1 + (M - z_y) + tau.
 * Rows with a non-finite maximum: kappa = 1, tau = 0, M = the maximum
 * (NaN if any NaN), loss = 1 - z_y + M in float32 (policy of
 * oracle/fw_oracle.py:nonfinite_policy).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int cmp_desc(const void* a, const void* b) {
  const double x = *(const double*)a, y = *(const double*)b;
  return (x < y) - (x > y);
}

static void solve_row(const float* z, int64_t C, int64_t yr, double* buf, double* tau,
                      int64_t* kappa, double* Mout, double* loss) {
  float M = -INFINITY;
  int has_nan = 0;
  for (int64_t j = 0; j < C; ++j) {
    if (z[j] != z[j]) has_nan = 1;
    else if (z[j] > M) M = z[j];
  }
  const int yok = yr >= 0 && yr < C;
  if (has_nan || !isfinite(M)) {
    const float m = has_nan ? NAN : M;
    *tau = 0.0;
    *kappa = 1;
    *Mout = m;
    *loss = yok ? (double)(1.0f - z[yr] + m) : NAN;
    return;
  }
  for (int64_t j = 0; j < C; ++j) buf[j] = (double)z[j] - (double)M;
  qsort(buf, (size_t)C, sizeof(double), cmp_desc);
  double S = 0.0, best = -INFINITY;
  int64_t bk = 1;
  for (int64_t k = 1; k <= C; ++k) {
    S += buf[k - 1];
    const double h = (S - 1.0) / (double)k;
    if (h > best) { best = h; bk = k; }
  }
  *tau = best;
  *kappa = bk;
  *Mout = M;
  *loss = yok ? 1.0 + ((double)M - (double)z[yr]) + best : NAN;
}

/* Solves rows [0, B) with `threads` OpenMP threads (0 = default). */
void fwo_solve_rows(const float* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                    double* tau, int64_t* kappa, double* M, double* loss, int threads) {
#ifdef _OPENMP
  const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
  const int nt = 1;
  (void)threads;
#endif
#pragma omp parallel num_threads(nt)
  {
    double* buf = (double*)malloc((size_t)(C > 0 ? C : 1) * sizeof(double));
#pragma omp for schedule(dynamic, 1)
    for (int64_t r = 0; r < B; ++r)
      solve_row(z + r * ld, C, y[r], buf, tau + r, kappa + r, M + r, loss + r);
    free(buf);
  }
}
