/*
 * kde_oracle.c -- CPU fp64 oracle for the Gaussian-kernel KDE/MMD sums.
 *
 * TEST INFRASTRUCTURE ONLY.  The CUDA path is compared against this file's
 * results (tests, the smoke check and the CPU-baseline leg of the
 * benchmark).  Nothing in the product package links, loads or calls it.
 *
 * It restates, in plain C and in double precision, the analytic forward and
 * backward of the reference:
 *   rapidalign/kde_gradients.py:32-36   _gaussian_kernel  (direct differences,
 *                                        k = exp(-|u-v|^2 / (2 sigma^2)))
 *   rapidalign/kde_gradients.py:39-73   kde_mmd_forward_cpu (Kxx, Kyy, Kxy)
 *   rapidalign/kde_gradients.py:76-132  kde_mmd_backward_cpu (grads w.r.t.
 *                                        points, raw weights and sigma)
 *   rapidalign/kde_gradients.py:135-193 kde_mmd_backward_ragged_cpu (per pair
 *                                        loop over ptr segments)
 * The reference materialises N x M x D difference tensors; this restatement
 * streams over rows instead, which changes nothing but memory use.
 *
 * Instead of final gradients it returns the per-point "row sums" from which
 * every gradient of the public API is one multiply-add away (the chain rule
 * for centering and weight normalisation is applied by oracle/oracle.py):
 *   s_xx[i]   = sum_j a_j k(x_i, x_j)          G_xx[i] = sum_j a_j k(x_i,x_j)(x_i - x_j)
 *   s_xy[i]   = sum_j b_j k(x_i, y_j)          G_xy[i] = sum_j b_j k(x_i,y_j)(x_i - y_j)
 *   s_yy[j]   = sum_l b_l k(y_j, y_l)          G_yy[j] = sum_l b_l k(y_j,y_l)(y_j - y_l)
 *   s_yx[j]   = sum_i a_i k(y_j, x_i)          G_yx[j] = sum_i a_i k(y_j,x_i)(y_j - x_i)
 * and per pair K = (Kxx, Kyy, Kxy) and S = (Sxx, Syy, Sxy) with
 *   S.. = sum over ordered pairs of w w' k r^2   (so dK/dsigma = S / sigma^3,
 *   kde_gradients.py:115-123).
 * With these, for loss L = Kxx + Kyy - 2 Kxy (kde_gradients.py:98-113):
 *   dL/dx_i = -(2/sigma^2) a_i G_xx[i] + (2/sigma^2) a_i G_xy[i]
 *   dL/da_i = 2 s_xx[i] - 2 s_xy[i]
 *
 * Parallelism: OpenMP over (pair, block, row) tasks; every task writes its own
 * row and its own row partial of K and S, and the per-pair totals are summed
 * sequentially, so results do not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* One row of one block: point u (dim D) against the n points v[0..n) with
 * weights w.  Accumulates s = sum w k, G = sum w k (u - v), S = sum w k r^2. */
static void row_sums(int D, const double *u, const double *v, const double *w, int64_t n,
                     double inv_two_sigma2, double *s_out, double *G_out, double *S_out) {
  double s = 0.0, S = 0.0;
  double G[64];
  double *Gp = G;
  double *Gheap = NULL;
  if (D > 64) {
    Gheap = (double *)calloc((size_t)D, sizeof(double));
    Gp = Gheap;
  } else {
    for (int d = 0; d < D; ++d) G[d] = 0.0;
  }
  for (int64_t j = 0; j < n; ++j) {
    const double *vj = v + j * D;
    double r2 = 0.0;
    for (int d = 0; d < D; ++d) {
      double t = u[d] - vj[d];
      r2 += t * t;
    }
    double k = exp(-r2 * inv_two_sigma2);
    double wk = w[j] * k;
    s += wk;
    S += wk * r2;
    for (int d = 0; d < D; ++d) Gp[d] += wk * (u[d] - vj[d]);
  }
  *s_out = s;
  *S_out = S;
  if (G_out)
    for (int d = 0; d < D; ++d) G_out[d] = Gp[d];
  free(Gheap);
}

/*
 * Ragged batch of P pairs (ptr_x, ptr_y as in rapidalign/kde.py:124-156), raw
 * weights a (for x) and b (for y).  All arrays are host fp64, row-major.
 * Outputs (any of the per-point ones may be NULL to skip them):
 *   K[3*P]  = (Kxx, Kyy, Kxy) per pair     S[3*P] = (Sxx, Syy, Sxy) per pair
 *   s_xx[NX], s_xy[NX], G_xx[NX*D], G_xy[NX*D], s_yy[NY], s_yx[NY],
 *   G_yy[NY*D], G_yx[NY*D]
 * Returns 0, or -1 on invalid arguments.
 */
int ra_oracle_segmented(int64_t P, int D, const double *x, const double *y, const double *a,
                        const double *b, const int64_t *ptr_x, const int64_t *ptr_y,
                        double sigma, int nthreads, double *K, double *S, double *s_xx,
                        double *s_xy, double *G_xx, double *G_xy, double *s_yy, double *s_yx,
                        double *G_yy, double *G_yx) {
  if (P < 0 || D <= 0 || !(sigma > 0.0)) return -1;
  const int64_t NX = P > 0 ? ptr_x[P] : 0;
  const int64_t NY = P > 0 ? ptr_y[P] : 0;
  const double inv_two_sigma2 = 1.0 / (2.0 * sigma * sigma);
  /* per-row partials of K and S: block 0 (xx) and 2 (xy) over x rows,
   * block 1 (yy) over y rows. */
  double *kx_self = (double *)calloc((size_t)(NX > 0 ? NX : 1), sizeof(double));
  double *kx_cross = (double *)calloc((size_t)(NX > 0 ? NX : 1), sizeof(double));
  double *ky_self = (double *)calloc((size_t)(NY > 0 ? NY : 1), sizeof(double));
  double *sx_self = (double *)calloc((size_t)(NX > 0 ? NX : 1), sizeof(double));
  double *sx_cross = (double *)calloc((size_t)(NX > 0 ? NX : 1), sizeof(double));
  double *sy_self = (double *)calloc((size_t)(NY > 0 ? NY : 1), sizeof(double));
  /* pair index of every point, for the flattened task loop */
  int64_t *pair_of_x = (int64_t *)malloc(sizeof(int64_t) * (size_t)(NX > 0 ? NX : 1));
  int64_t *pair_of_y = (int64_t *)malloc(sizeof(int64_t) * (size_t)(NY > 0 ? NY : 1));
  if (!kx_self || !kx_cross || !ky_self || !sx_self || !sx_cross || !sy_self || !pair_of_x ||
      !pair_of_y) {
    free(kx_self); free(kx_cross); free(ky_self); free(sx_self); free(sx_cross); free(sy_self);
    free(pair_of_x); free(pair_of_y);
    return -1;
  }
  for (int64_t p = 0; p < P; ++p) {
    for (int64_t i = ptr_x[p]; i < ptr_x[p + 1]; ++i) pair_of_x[i] = p;
    for (int64_t j = ptr_y[p]; j < ptr_y[p + 1]; ++j) pair_of_y[j] = p;
  }
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  const int64_t ntasks = 2 * NX + 2 * NY;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t t = 0; t < ntasks; ++t) {
    double Gtmp[64];
    double *G = NULL;
    double s_val, S_val;
    if (t < NX) { /* x row i vs x: xx block */
      int64_t i = t, p = pair_of_x[i];
      int64_t x0 = ptr_x[p], nx = ptr_x[p + 1] - x0;
      G = G_xx ? G_xx + i * D : (D <= 64 ? Gtmp : NULL);
      row_sums(D, x + i * D, x + x0 * D, a + x0, nx, inv_two_sigma2, &s_val, G, &S_val);
      if (s_xx) s_xx[i] = s_val;
      kx_self[i] = a[i] * s_val;
      sx_self[i] = a[i] * S_val;
    } else if (t < 2 * NX) { /* x row i vs y: xy block */
      int64_t i = t - NX, p = pair_of_x[i];
      int64_t y0 = ptr_y[p], ny = ptr_y[p + 1] - y0;
      G = G_xy ? G_xy + i * D : (D <= 64 ? Gtmp : NULL);
      row_sums(D, x + i * D, y + y0 * D, b + y0, ny, inv_two_sigma2, &s_val, G, &S_val);
      if (s_xy) s_xy[i] = s_val;
      kx_cross[i] = a[i] * s_val;
      sx_cross[i] = a[i] * S_val;
    } else if (t < 2 * NX + NY) { /* y row j vs y: yy block */
      int64_t j = t - 2 * NX, p = pair_of_y[j];
      int64_t y0 = ptr_y[p], ny = ptr_y[p + 1] - y0;
      G = G_yy ? G_yy + j * D : (D <= 64 ? Gtmp : NULL);
      row_sums(D, y + j * D, y + y0 * D, b + y0, ny, inv_two_sigma2, &s_val, G, &S_val);
      if (s_yy) s_yy[j] = s_val;
      ky_self[j] = b[j] * s_val;
      sy_self[j] = b[j] * S_val;
    } else { /* y row j vs x: the transposed cross block (only its row sums) */
      int64_t j = t - 2 * NX - NY, p = pair_of_y[j];
      int64_t x0 = ptr_x[p], nx = ptr_x[p + 1] - x0;
      G = G_yx ? G_yx + j * D : (D <= 64 ? Gtmp : NULL);
      row_sums(D, y + j * D, x + x0 * D, a + x0, nx, inv_two_sigma2, &s_val, G, &S_val);
      if (s_yx) s_yx[j] = s_val;
    }
  }
  for (int64_t p = 0; p < P; ++p) {
    double kxx = 0.0, kyy = 0.0, kxy = 0.0, sxx = 0.0, syy = 0.0, sxy = 0.0;
    for (int64_t i = ptr_x[p]; i < ptr_x[p + 1]; ++i) {
      kxx += kx_self[i];
      kxy += kx_cross[i];
      sxx += sx_self[i];
      sxy += sx_cross[i];
    }
    for (int64_t j = ptr_y[p]; j < ptr_y[p + 1]; ++j) {
      kyy += ky_self[j];
      syy += sy_self[j];
    }
    if (K) { K[3 * p + 0] = kxx; K[3 * p + 1] = kyy; K[3 * p + 2] = kxy; }
    if (S) { S[3 * p + 0] = sxx; S[3 * p + 1] = syy; S[3 * p + 2] = sxy; }
  }
  free(kx_self); free(kx_cross); free(ky_self); free(sx_self); free(sx_cross); free(sy_self);
  free(pair_of_x); free(pair_of_y);
  return 0;
}

/*
 * Row sums for a chosen subset of rows of ONE pair (spot checks of very large
 * pairs, where the full oracle would take hours).  side = 0: rows are x
 * points (indices into x), returning s_xx, G_xx, s_xy, G_xy for them;
 * side = 1: rows are y points, returning s_yy, G_yy, s_yx, G_yx.
 * out_self_s[R], out_self_G[R*D], out_cross_s[R], out_cross_G[R*D].
 */
int ra_oracle_rows(int side, int D, int64_t n, int64_t m, const double *x, const double *y,
                   const double *a, const double *b, double sigma, int64_t R,
                   const int64_t *rows, int nthreads, double *out_self_s, double *out_self_G,
                   double *out_cross_s, double *out_cross_G) {
  if (D <= 0 || !(sigma > 0.0) || (side != 0 && side != 1)) return -1;
  const double inv_two_sigma2 = 1.0 / (2.0 * sigma * sigma);
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t r = 0; r < 2 * R; ++r) {
    int64_t q = r / 2;
    int cross = (int)(r % 2);
    double Sdummy;
    const double *self_pts = side == 0 ? x : y;
    const double *other_pts = side == 0 ? y : x;
    const double *self_w = side == 0 ? a : b;
    const double *other_w = side == 0 ? b : a;
    int64_t n_self = side == 0 ? n : m, n_other = side == 0 ? m : n;
    const double *u = self_pts + rows[q] * D;
    if (!cross)
      row_sums(D, u, self_pts, self_w, n_self, inv_two_sigma2, out_self_s + q,
               out_self_G + q * D, &Sdummy);
    else
      row_sums(D, u, other_pts, other_w, n_other, inv_two_sigma2, out_cross_s + q,
               out_cross_G + q * D, &Sdummy);
  }
  return 0;
}
