/*
 * CPU oracle for the quaternion linear forward.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * call it to check device results or as the timed CPU baseline; the product never links it.
 *
 * Restates, in double precision, the explicit Hamilton-product definition of
 * the reference:
 *   quaternion/reference.py:31-45   hamilton_product(a, b), a = weight, b = input
 *   quaternion/reference.py:48-86   y[o] = sum_i  W[o,i] (x) X[i]   (no shortcuts)
 *   quaternion/linear.py:120-124    + bias
 *   quaternion/lora.py:60-63        + scale * ((x A^T) B^T)
 * Packing (quaternion/packing.py:5-25): x[m, 4i+q] is component q (r,i,j,k) of
 * input quaternion i; y[m, 4o+a] likewise; W_c[o, i] row-major [N_g, K_g].
 *
 * Inputs are float (bf16/f16 values are exact in float); every product and
 * sum is double.  An optional row list evaluates a subset of tokens, which
 * lets full-size layers be checked on sampled rows.
 */
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Hamilton product w (x) x, both (r,i,j,k); reference.py:31-45. */
static inline void hamilton(const double w[4], const double x[4], double out[4]) {
  out[0] = w[0] * x[0] - w[1] * x[1] - w[2] * x[2] - w[3] * x[3];
  out[1] = w[0] * x[1] + w[1] * x[0] + w[2] * x[3] - w[3] * x[2];
  out[2] = w[0] * x[2] - w[1] * x[3] + w[2] * x[0] + w[3] * x[1];
  out[3] = w[0] * x[3] + w[1] * x[2] - w[2] * x[1] + w[3] * x[0];
}

int qlin_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/*
 * y[r, :] for r in rows (or all M tokens when rows == NULL); y is
 * [n_rows, 4*N_g] double with leading dimension ld_y.  Returns 0, or -1 on
 * bad arguments.  threads <= 0 keeps the OpenMP default.
 */
int qlin_oracle_forward(const float* x, int64_t ld_x,
                        const float* wr, const float* wi, const float* wj, const float* wk,
                        int64_t ld_w,
                        const float* bias,
                        const float* lora_a, const float* lora_b, int rank, double lora_scale,
                        double* y, int64_t ld_y,
                        int64_t M, int64_t K_g, int64_t N_g,
                        const int64_t* rows, int64_t n_rows, int threads) {
  if (!x || !wr || !wi || !wj || !wk || !y) return -1;
  if (M < 0 || K_g < 0 || N_g < 0 || ld_x < 4 * K_g || ld_w < K_g || ld_y < 4 * N_g) return -1;
  if (rank < 0 || (rank > 0 && (!lora_a || !lora_b))) return -1;
  if (!rows) n_rows = M;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  const int64_t K = 4 * K_g;
  /* LoRA down projection once per evaluated token (lora.py:62). */
  double* tbuf = NULL;
  if (rank > 0) {
    tbuf = (double*)malloc((size_t)(n_rows > 0 ? n_rows : 1) * (size_t)rank * sizeof(double));
    if (!tbuf) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t job = 0; job < n_rows * rank; ++job) {
      int64_t rr = job / rank, r = job % rank;
      int64_t m = rows ? rows[rr] : rr;
      double s = 0.0;
      if (m >= 0 && m < M)
        for (int64_t k = 0; k < K; ++k) s += (double)x[m * ld_x + k] * lora_a[r * K + k];
      tbuf[job] = s;
    }
  }
  int64_t total = n_rows * N_g;
#pragma omp parallel for schedule(static)
  for (int64_t job = 0; job < total; ++job) {
    int64_t rr = job / N_g, o = job % N_g;
    int64_t m = rows ? rows[rr] : rr;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    if (m >= 0 && m < M) {
      const float* xm = x + m * ld_x;
      for (int64_t i = 0; i < K_g; ++i) {
        double w[4] = {wr[o * ld_w + i], wi[o * ld_w + i], wj[o * ld_w + i], wk[o * ld_w + i]};
        double xq[4] = {xm[4 * i + 0], xm[4 * i + 1], xm[4 * i + 2], xm[4 * i + 3]};
        double h[4];
        hamilton(w, xq, h);
        acc[0] += h[0]; acc[1] += h[1]; acc[2] += h[2]; acc[3] += h[3];
      }
      for (int a = 0; a < 4; ++a) {
        int64_t n = 4 * o + a;
        double v = acc[a];
        if (bias) v += bias[n];
        if (rank > 0) {
          double l = 0.0;
          for (int r = 0; r < rank; ++r) l += tbuf[rr * rank + r] * lora_b[n * rank + r];
          v += lora_scale * l;
        }
        y[rr * ld_y + n] = v;
      }
    } else {
      for (int a = 0; a < 4; ++a) y[rr * ld_y + 4 * o + a] = 0.0;
    }
  }
  free(tbuf);
  return 0;
}

/*
 * LoRA down projection t[m, r] = sum_k x[m,k] A[r,k] in double, used by the
 * forward above and exposed so the oracle's LoRA term can be formed once per
 * token (lora.py:62).
 */
int qlin_oracle_lora_down(const float* x, int64_t ld_x, const float* lora_a, int rank,
                          double* t, int64_t M, int64_t K) {
  if (!x || !lora_a || !t || rank <= 0 || ld_x < K) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t job = 0; job < M * rank; ++job) {
    int64_t m = job / rank, r = job % rank;
    double s = 0.0;
    for (int64_t k = 0; k < K; ++k) s += (double)x[m * ld_x + k] * lora_a[r * K + k];
    t[m * rank + r] = s;
  }
  return 0;
}
