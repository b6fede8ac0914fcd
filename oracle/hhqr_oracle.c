/*
 * hhqr_oracle.c — CPU oracle for the batched compact-Householder QR path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the GPU library is
 * compared against; it is never linked into, called by, or shipped with the
 * product library (gpumode_qr_b200/libqrb200.so). Only tests/, the smoke
 * check and bench.py's CPU-baseline leg load it.
 *
 * It restates, in plain C, the algorithm of the reference's hot path:
 *   - oracle_geqr2: unblocked Householder QR, step for step as the reference's
 *     fused kernel (src/qrbench/triton_kernels.py:641-720): for column j,
 *     sigma = sum_{i>j} a_ij^2, norm = sqrt(alpha^2 + sigma),
 *     beta = -sign(alpha) norm (alpha >= 0 -> -norm), tau = (beta - alpha)/beta,
 *     v = a(j+1:, j) / (alpha - beta) with v_j = 1, sigma <= 0 -> tau = 0 and
 *     beta = alpha; then every trailing column k > j gets
 *     a_k -= tau * v * (v^T a_k); geqrf packing (R above, beta on, v below the
 *     diagonal). This is also LAPACK sgeqr2 with slarfg/slarf (the algorithm of
 *     torch.geqrf, the reference's own oracle at src/qrbench/reference.py:18-20)
 *     except that slarfg rescales tiny/huge columns and LAPACK's sign of a
 *     negative zero alpha differs.
 *   - oracle_panel: the reference's panel kernel (triton_kernels.py:787-910):
 *     the same column loop on an r x w panel, the explicit unit-lower V, and
 *     the forward LARFT recurrence T[i][i] = tau_i,
 *     T[0:i][i] = -tau_i * T[0:i][0:i] * (V[:,0:i]^T V[:,i]).
 *   - oracle_larfb: the trailing update of _hh_panel_blocked_qr
 *     (src/qrbench/variants.py:800-804): C -= V (T^T (V^T C)).
 *   - oracle_blocked_geqrf: the blocked driver (variants.py:761-805) built
 *     from the three pieces above.
 *   - oracle_larft: the LARFT recurrence alone, from a packed (H, tau) block
 *     (the T factor an apply-Q / form-Q step needs).
 * Every routine takes `f64`: 0 computes in float (the reference's FP32
 * arithmetic, sequential sums), 1 computes in double and rounds the outputs to
 * float (a high-accuracy answer for parity checks).
 *
 * Storage: row-major, element (i, j) of matrix m at m*sb + i*ld + j.
 * The batch loop is parallelised with OpenMP when compiled with -fopenmp.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

typedef double real_d;

/* ------------------------------------------------------------------ */
/* unblocked QR of one rows x cols matrix held as doubles or floats    */
/* ------------------------------------------------------------------ */

#define DEFINE_GEQR2(NAME, T, SQRT)                                            \
  static void NAME(int rows, int cols, T* a, int ld, T* tau) {                 \
    const int steps = rows < cols ? rows : cols;                               \
    for (int j = 0; j < cols; ++j) tau[j] = (T)0;                              \
    for (int j = 0; j < steps; ++j) {                                          \
      T alpha = a[(int64_t)j * ld + j];                                        \
      T sigma = (T)0;                                                          \
      for (int i = j + 1; i < rows; ++i) {                                     \
        const T x = a[(int64_t)i * ld + j];                                    \
        sigma += x * x;                                                        \
      }                                                                        \
      T beta, t, scale;                                                        \
      if (sigma > (T)0) {                                                      \
        const T nrm = SQRT(alpha * alpha + sigma);                             \
        beta = alpha >= (T)0 ? -nrm : nrm;                                     \
        t = (beta - alpha) / beta;                                             \
        scale = (T)1 / (alpha - beta);                                         \
      } else {                                                                 \
        beta = alpha;                                                          \
        t = (T)0;                                                              \
        scale = (T)0;                                                          \
      }                                                                        \
      for (int i = j + 1; i < rows; ++i) a[(int64_t)i * ld + j] *= scale;      \
      for (int k = j + 1; k < cols; ++k) {                                     \
        T d = a[(int64_t)j * ld + k];                                          \
        for (int i = j + 1; i < rows; ++i)                                     \
          d += a[(int64_t)i * ld + j] * a[(int64_t)i * ld + k];                \
        const T f = t * d;                                                     \
        a[(int64_t)j * ld + k] -= f;                                           \
        for (int i = j + 1; i < rows; ++i)                                     \
          a[(int64_t)i * ld + k] -= f * a[(int64_t)i * ld + j];                \
      }                                                                        \
      a[(int64_t)j * ld + j] = beta;                                           \
      tau[j] = t;                                                              \
    }                                                                          \
  }

DEFINE_GEQR2(geqr2_f, float, sqrtf)
DEFINE_GEQR2(geqr2_d, double, sqrt)

/* Forward LARFT: T (w x w, row-major) from explicit unit-lower V (r x w). */
#define DEFINE_LARFT(NAME, T)                                                  \
  static void NAME(int r, int w, const T* v, const T* tau, T* t) {            \
    for (int e = 0; e < w * w; ++e) t[e] = (T)0;                               \
    T* z = (T*)malloc(sizeof(T) * (w > 0 ? w : 1));                            \
    for (int i = 0; i < w; ++i) {                                              \
      for (int k = 0; k < i; ++k) {                                            \
        T s = (T)0;                                                            \
        for (int q = 0; q < r; ++q)                                            \
          s += v[(int64_t)q * w + k] * v[(int64_t)q * w + i];                  \
        z[k] = s;                                                              \
      }                                                                        \
      for (int k = 0; k < i; ++k) {                                            \
        T y = (T)0;                                                            \
        for (int q = 0; q < i; ++q) y += t[k * w + q] * z[q];                  \
        t[k * w + i] = -tau[i] * y;                                            \
      }                                                                        \
      t[i * w + i] = tau[i];                                                   \
    }                                                                          \
    free(z);                                                                   \
  }

DEFINE_LARFT(larft_f, float)
DEFINE_LARFT(larft_d, double)

/* C (r x c, row-major) -= V (T^T (V^T C)); V explicit r x k, T k x k. */
#define DEFINE_LARFB(NAME, T)                                                  \
  static void NAME(int r, int k, int c, const T* v, const T* t, T* cm) {       \
    T* w1 = (T*)calloc((size_t)k * (c > 0 ? c : 1), sizeof(T));                \
    T* w2 = (T*)calloc((size_t)k * (c > 0 ? c : 1), sizeof(T));                \
    for (int a = 0; a < k; ++a)                                                \
      for (int q = 0; q < r; ++q) {                                            \
        const T va = v[(int64_t)q * k + a];                                    \
        if (va == (T)0) continue;                                              \
        for (int j = 0; j < c; ++j) w1[(int64_t)a * c + j] += va * cm[(int64_t)q * c + j]; \
      }                                                                        \
    for (int a = 0; a < k; ++a)                                                \
      for (int q = 0; q < k; ++q) {                                            \
        const T tq = t[q * k + a];                                             \
        if (tq == (T)0) continue;                                              \
        for (int j = 0; j < c; ++j) w2[(int64_t)a * c + j] += tq * w1[(int64_t)q * c + j]; \
      }                                                                        \
    for (int q = 0; q < r; ++q)                                                \
      for (int a = 0; a < k; ++a) {                                            \
        const T va = v[(int64_t)q * k + a];                                    \
        if (va == (T)0) continue;                                              \
        for (int j = 0; j < c; ++j) cm[(int64_t)q * c + j] -= va * w2[(int64_t)a * c + j]; \
      }                                                                        \
    free(w1);                                                                  \
    free(w2);                                                                  \
  }

DEFINE_LARFB(larfb_f, float)
DEFINE_LARFB(larfb_d, double)

/* ------------------------------------------------------------------ */
/* exported batched entry points                                       */
/* ------------------------------------------------------------------ */

ORACLE_API int oracle_version(void) { return 1; }

ORACLE_API void oracle_geqr2(int64_t batch, int rows, int cols, const float* A,
                             int64_t sAb, int64_t sAr, float* H, float* tau,
                             int f64) {
#pragma omp parallel for schedule(dynamic)
  for (int64_t m = 0; m < batch; ++m) {
    const float* src = A + m * sAb;
    float* dst = H + m * (int64_t)rows * cols;
    float* tm = tau + m * (int64_t)cols;
    if (f64) {
      double* a = (double*)malloc(sizeof(double) * (size_t)rows * cols);
      double* t = (double*)malloc(sizeof(double) * (size_t)(cols > 0 ? cols : 1));
      for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) a[(int64_t)i * cols + j] = src[i * sAr + j];
      geqr2_d(rows, cols, a, cols, t);
      for (int64_t e = 0; e < (int64_t)rows * cols; ++e) dst[e] = (float)a[e];
      for (int j = 0; j < cols; ++j) tm[j] = (float)t[j];
      free(a);
      free(t);
    } else {
      for (int i = 0; i < rows; ++i) memcpy(dst + (int64_t)i * cols, src + i * sAr, sizeof(float) * cols);
      geqr2_f(rows, cols, dst, cols, tm);
    }
  }
}

ORACLE_API void oracle_panel(int64_t batch, int r, int w, const float* P,
                             float* H, float* V, float* tau, float* T, int f64) {
#pragma omp parallel for schedule(dynamic)
  for (int64_t m = 0; m < batch; ++m) {
    const float* src = P + m * (int64_t)r * w;
    float* h = H + m * (int64_t)r * w;
    float* vv = V + m * (int64_t)r * w;
    float* tm = tau + m * (int64_t)w;
    float* tt = T + m * (int64_t)w * w;
    if (f64) {
      double* a = (double*)malloc(sizeof(double) * (size_t)r * w);
      double* v = (double*)malloc(sizeof(double) * (size_t)r * w);
      double* t = (double*)malloc(sizeof(double) * (size_t)w);
      double* tf = (double*)malloc(sizeof(double) * (size_t)w * w);
      for (int64_t e = 0; e < (int64_t)r * w; ++e) a[e] = src[e];
      geqr2_d(r, w, a, w, t);
      for (int i = 0; i < r; ++i)
        for (int j = 0; j < w; ++j)
          v[(int64_t)i * w + j] = i > j ? a[(int64_t)i * w + j] : (i == j ? 1.0 : 0.0);
      larft_d(r, w, v, t, tf);
      for (int64_t e = 0; e < (int64_t)r * w; ++e) {
        h[e] = (float)a[e];
        vv[e] = (float)v[e];
      }
      for (int j = 0; j < w; ++j) tm[j] = (float)t[j];
      for (int e = 0; e < w * w; ++e) tt[e] = (float)tf[e];
      free(a);
      free(v);
      free(t);
      free(tf);
    } else {
      memcpy(h, src, sizeof(float) * (size_t)r * w);
      geqr2_f(r, w, h, w, tm);
      for (int i = 0; i < r; ++i)
        for (int j = 0; j < w; ++j)
          vv[(int64_t)i * w + j] = i > j ? h[(int64_t)i * w + j] : (i == j ? 1.f : 0.f);
      larft_f(r, w, vv, tm, tt);
    }
  }
}

ORACLE_API void oracle_larfb(int64_t batch, int r, int k, int c, const float* V,
                             const float* T, float* C, int f64) {
#pragma omp parallel for schedule(dynamic)
  for (int64_t m = 0; m < batch; ++m) {
    const float* v = V + m * (int64_t)r * k;
    const float* t = T + m * (int64_t)k * k;
    float* cm = C + m * (int64_t)r * c;
    if (f64) {
      double* vd = (double*)malloc(sizeof(double) * (size_t)r * k);
      double* td = (double*)malloc(sizeof(double) * (size_t)k * k);
      double* cd = (double*)malloc(sizeof(double) * (size_t)r * c);
      for (int64_t e = 0; e < (int64_t)r * k; ++e) vd[e] = v[e];
      for (int64_t e = 0; e < (int64_t)k * k; ++e) td[e] = t[e];
      for (int64_t e = 0; e < (int64_t)r * c; ++e) cd[e] = cm[e];
      larfb_d(r, k, c, vd, td, cd);
      for (int64_t e = 0; e < (int64_t)r * c; ++e) cm[e] = (float)cd[e];
      free(vd);
      free(td);
      free(cd);
    } else {
      larfb_f(r, k, c, v, t, cm);
    }
  }
}

/* Forward LARFT from a packed block: V is the strictly lower part of the
 * r x k block at H (unit diagonal implied, zero above), tau its k
 * coefficients; T is k x k row-major. Follows the reference panel kernel's
 * recurrence (src/qrbench/triton_kernels.py:886-909). */
ORACLE_API void oracle_larft(int64_t batch, int r, int k, const float* H, int64_t sb, int64_t ld,
                             const float* tau, int64_t tau_sb, float* T, int f64) {
#pragma omp parallel for schedule(dynamic)
  for (int64_t m = 0; m < batch; ++m) {
    const float* h = H + m * sb;
    const float* tm = tau + m * tau_sb;
    float* tt = T + m * (int64_t)k * k;
    if (f64) {
      double* vd = (double*)malloc(sizeof(double) * (size_t)r * k);
      double* td = (double*)malloc(sizeof(double) * (size_t)k);
      double* out = (double*)malloc(sizeof(double) * (size_t)k * k);
      for (int i = 0; i < r; ++i)
        for (int j = 0; j < k; ++j)
          vd[(int64_t)i * k + j] = i > j ? h[(int64_t)i * ld + j] : (i == j ? 1.0 : 0.0);
      for (int j = 0; j < k; ++j) td[j] = tm[j];
      larft_d(r, k, vd, td, out);
      for (int64_t e = 0; e < (int64_t)k * k; ++e) tt[e] = (float)out[e];
      free(vd);
      free(td);
      free(out);
    } else {
      float* vf = (float*)malloc(sizeof(float) * (size_t)r * k);
      for (int i = 0; i < r; ++i)
        for (int j = 0; j < k; ++j)
          vf[(int64_t)i * k + j] = i > j ? h[(int64_t)i * ld + j] : (i == j ? 1.f : 0.f);
      larft_f(r, k, vf, tm, tt);
      free(vf);
    }
  }
}

/* Blocked QR with panel width w (reference _hh_panel_blocked_qr). */
#define DEFINE_BLOCKED(NAME, T, GEQR2, LARFT, LARFB)                           \
  static void NAME(int n, T* a, T* tau, int wpan) {                            \
    T* pan = (T*)malloc(sizeof(T) * (size_t)n * wpan);                         \
    T* v = (T*)malloc(sizeof(T) * (size_t)n * wpan);                           \
    T* tf = (T*)malloc(sizeof(T) * (size_t)wpan * wpan);                       \
    T* cc = (T*)malloc(sizeof(T) * (size_t)n * n);                             \
    for (int j0 = 0; j0 < n; j0 += wpan) {                                     \
      const int w = n - j0 < wpan ? n - j0 : wpan;                             \
      const int r = n - j0;                                                    \
      for (int i = 0; i < r; ++i)                                              \
        for (int j = 0; j < w; ++j) pan[i * w + j] = a[(int64_t)(j0 + i) * n + j0 + j]; \
      GEQR2(r, w, pan, w, tau + j0);                                           \
      for (int i = 0; i < r; ++i)                                              \
        for (int j = 0; j < w; ++j) {                                          \
          a[(int64_t)(j0 + i) * n + j0 + j] = pan[i * w + j];                  \
          v[i * w + j] = i > j ? pan[i * w + j] : (i == j ? (T)1 : (T)0);      \
        }                                                                      \
      const int c = n - j0 - w;                                                \
      if (c <= 0) continue;                                                    \
      LARFT(r, w, v, tau + j0, tf);                                            \
      for (int i = 0; i < r; ++i)                                              \
        for (int j = 0; j < c; ++j) cc[(int64_t)i * c + j] = a[(int64_t)(j0 + i) * n + j0 + w + j]; \
      LARFB(r, w, c, v, tf, cc);                                               \
      for (int i = 0; i < r; ++i)                                              \
        for (int j = 0; j < c; ++j) a[(int64_t)(j0 + i) * n + j0 + w + j] = cc[(int64_t)i * c + j]; \
    }                                                                          \
    free(pan);                                                                 \
    free(v);                                                                   \
    free(tf);                                                                  \
    free(cc);                                                                  \
  }

DEFINE_BLOCKED(blocked_f, float, geqr2_f, larft_f, larfb_f)
DEFINE_BLOCKED(blocked_d, double, geqr2_d, larft_d, larfb_d)

ORACLE_API void oracle_blocked_geqrf(int64_t batch, int n, const float* A,
                                     int64_t sAb, int64_t sAr, float* H,
                                     float* tau, int wpan, int f64) {
  if (wpan < 1) wpan = 32;
#pragma omp parallel for schedule(dynamic)
  for (int64_t m = 0; m < batch; ++m) {
    const float* src = A + m * sAb;
    float* dst = H + m * (int64_t)n * n;
    float* tm = tau + m * (int64_t)n;
    if (f64) {
      double* a = (double*)malloc(sizeof(double) * (size_t)n * n);
      double* t = (double*)malloc(sizeof(double) * (size_t)n);
      for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) a[(int64_t)i * n + j] = src[i * sAr + j];
      blocked_d(n, a, t, wpan);
      for (int64_t e = 0; e < (int64_t)n * n; ++e) dst[e] = (float)a[e];
      for (int j = 0; j < n; ++j) tm[j] = (float)t[j];
      free(a);
      free(t);
    } else {
      for (int i = 0; i < n; ++i) memcpy(dst + (int64_t)i * n, src + i * sAr, sizeof(float) * n);
      blocked_f(n, dst, tm, wpan);
    }
  }
}
