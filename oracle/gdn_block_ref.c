/* CPU restatement of the reference GDN triangular solve (TEST INFRASTRUCTURE ONLY: the timed
 * CPU baseline and a cross-check, never the product).
 *
 * Algorithm of example/gdn_native/solve_op/gdn_solve_ref.c:16-69 (BL = 16):
 *   1. each BLxBL diagonal block of L = I - A is inverted by forward substitution on int16 codes
 *      of A (scale sA) with int32 accumulation; every row is requantized to int16 codes at sT
 *      (llround, clip to +-32767);
 *   2. off-diagonal blocks are merged in fp64:  T_ij = T_ii @ sum_{k=j}^{i-1} A_ik T_kj  (i > j).
 * Chunks are independent; OpenMP spreads them over the host cores.
 *
 * Exported:  int gdn_block_ref_solve(const int16_t *Aq, const float *sA, float sT,
 *                                    int n_chunks, int C, double *T, int threads)
 *   Aq [n_chunks, C, C] int16 codes (strictly lower), sA per chunk, T [n_chunks, C, C] fp64.
 *   Returns 0, or -1 when C is not a positive multiple of 16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLK 16

static int16_t sat_code(double v) {
  if (v > 32767.0) v = 32767.0;
  if (v < -32767.0) v = -32767.0;
  return (int16_t)llround(v);
}

static void solve_one(const int16_t *A, int C, double sA, double sT, double *T, double *work) {
  const int nb = C / BLK;
  double *Tb = work;                        /* [nb][nb][BLK][BLK] fp64 blocks */
  double *acc = work + (size_t)nb * nb * BLK * BLK;
  int16_t codes[BLK * BLK];
  memset(Tb, 0, sizeof(double) * (size_t)nb * nb * BLK * BLK);
  for (int b = 0; b < nb; ++b) {
    for (int i = 0; i < BLK; ++i) {
      for (int j = 0; j < BLK; ++j) {
        int32_t s = 0;
        for (int k = 0; k < i; ++k)
          s += (int32_t)A[(size_t)(b * BLK + i) * C + b * BLK + k] * (int32_t)codes[k * BLK + j];
        codes[i * BLK + j] = sat_code((i == j ? 1.0 / sT : 0.0) + (double)s * sA);
      }
    }
    double *d = Tb + ((size_t)b * nb + b) * BLK * BLK;
    for (int t = 0; t < BLK * BLK; ++t) d[t] = (double)codes[t] * sT;
  }
  for (int i = 0; i < nb; ++i) {
    for (int j = i - 1; j >= 0; --j) {
      memset(acc, 0, sizeof(double) * BLK * BLK);
      /* per (k, r, c): the BLK-term dot product is summed on its own, then added to acc -- the
       * reference's floating-point order (gdn_solve_ref.c:46-53), so the two agree bit for bit */
      for (int k = j; k < i; ++k) {
        const double *tkj = Tb + ((size_t)k * nb + j) * BLK * BLK;
        for (int r = 0; r < BLK; ++r) {
          double a[BLK];
          for (int m = 0; m < BLK; ++m) a[m] = (double)A[(size_t)(i * BLK + r) * C + k * BLK + m] * sA;
          for (int c = 0; c < BLK; ++c) {
            double s = 0.0;
            for (int m = 0; m < BLK; ++m) s += a[m] * tkj[m * BLK + c];
            acc[r * BLK + c] += s;
          }
        }
      }
      const double *tii = Tb + ((size_t)i * nb + i) * BLK * BLK;
      double *tij = Tb + ((size_t)i * nb + j) * BLK * BLK;
      for (int r = 0; r < BLK; ++r)
        for (int c = 0; c < BLK; ++c) {
          double s = 0.0;
          for (int m = 0; m < BLK; ++m) s += tii[r * BLK + m] * acc[m * BLK + c];
          tij[r * BLK + c] = s;
        }
    }
  }
  for (int r = 0; r < C; ++r)
    for (int c = 0; c < C; ++c) {
      const int i = r / BLK, j = c / BLK;
      T[(size_t)r * C + c] = (j <= i) ? Tb[((size_t)i * nb + j) * BLK * BLK + (r % BLK) * BLK + (c % BLK)] : 0.0;
    }
}

int gdn_block_ref_solve(const int16_t *Aq, const float *sA, float sT, int n_chunks, int C, double *T,
                        int threads) {
  if (C <= 0 || C % BLK) return -1;
  const int nb = C / BLK;
  const size_t wsz = (size_t)nb * nb * BLK * BLK + BLK * BLK;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel
  {
    double *work = (double *)malloc(sizeof(double) * wsz);
#pragma omp for schedule(dynamic, 1)
    for (int h = 0; h < n_chunks; ++h)
      solve_one(Aq + (size_t)h * C * C, C, (double)sA[h], (double)sT, T + (size_t)h * C * C, work);
    free(work);
  }
  return 0;
}
