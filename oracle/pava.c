/*
 * TEST INFRASTRUCTURE ONLY - the CPU oracle for torchisotonic_b200's parity tests, smoke check
 * and CPU baseline. Nothing in the product path links or calls this file.
 *
 * A plain-C restatement of torchisotonic's CPU solver and CPU backward:
 *   - pool adjacent violators, a stack of blocks (start, total weight, weighted sum), merging
 *     while the previous block's mean is not below the new one's, so equal means pool
 *     (reference: src/torchisotonic/csrc/pava.h:16-69, merge test at pava.h:46-55);
 *   - a NaN anywhere in a row makes the whole row NaN with one block starting at 0
 *     (pava.h:30-37);
 *   - a decreasing fit is minus the increasing fit of -y (src/torchisotonic/_api.py:131-134);
 *   - results clipped to [y_min, y_max] after the fit, in the accumulation dtype, with the
 *     bounds rounded to that dtype first (_api.py:68-69, torch's clamp on a tensor);
 *   - the gradient of the fit: block sums of the upstream gradient G and the weights W over each
 *     block, d/dy = w G / W and d/dw = (y - fit) G / W (_api.py:92-115), with the clamp's
 *     inclusive mask applied to the upstream gradient first (torch's clamp backward).
 *
 * Two precisions per input dtype:
 *   PREC_REFERENCE: sums in the input dtype, in the reference's operation order, so that the
 *                   result is the reference CPU op's, bit for bit (pava<scalar_t, scalar_t>
 *                   as instantiated at src/torchisotonic/csrc/ops.cpp:34);
 *   PREC_EXTENDED:  sums in long double (float32 input) or __float128 (float64 input): the
 *                   block partition of the exact problem except for ties closer than those
 *                   formats resolve - the partition the GPU kernels must reproduce.
 * Build with -ffp-contract=off so that no multiply-add is fused (the reference is built without
 * FMA instructions).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { PREC_REFERENCE = 0, PREC_EXTENDED = 1 };

typedef __float128 quad;

/* One row of pava.h:16-69, generic over the storage type S and the accumulation type A.
 * start/weight/total: scratch of n entries each. */
#define DEFINE_PAVA(NAME, S, A)                                                              \
  static void NAME(const S* y, const S* w, S* out, uint8_t* starts, int64_t n,              \
                   int64_t* start, A* weight, A* total) {                                    \
    int64_t top = -1;                                                                        \
    for (int64_t i = 0; i < n; ++i) {                                                        \
      A yi = (A)y[i];                                                                        \
      if (yi != yi) {                                                                        \
        for (int64_t j = 0; j < n; ++j) {                                                    \
          out[j] = (S)yi;                                                                    \
          if (starts) starts[j] = (uint8_t)(j == 0);                                         \
        }                                                                                    \
        return;                                                                              \
      }                                                                                      \
      A wi = w ? (A)w[i] : (A)1;                                                             \
      ++top;                                                                                 \
      start[top] = i;                                                                        \
      weight[top] = wi;                                                                      \
      total[top] = wi * yi;                                                                  \
      while (top > 0) {                                                                      \
        A wa = weight[top - 1], ta = total[top - 1];                                         \
        A wb = weight[top], tb = total[top];                                                 \
        if (ta * wb < tb * wa) break;                                                        \
        weight[top - 1] = wa + wb;                                                           \
        total[top - 1] = ta + tb;                                                            \
        --top;                                                                               \
      }                                                                                      \
    }                                                                                        \
    for (int64_t k = top; k >= 0; --k) {                                                     \
      int64_t first = start[k];                                                              \
      int64_t last = k == top ? n : start[k + 1];                                            \
      S mean = (S)(total[k] / weight[k]);                                                    \
      for (int64_t j = first; j < last; ++j) {                                               \
        out[j] = mean;                                                                       \
        if (starts) starts[j] = (uint8_t)(j == first);                                       \
      }                                                                                      \
    }                                                                                        \
  }

DEFINE_PAVA(pava_f32_ref, float, float)
DEFINE_PAVA(pava_f64_ref, double, double)
DEFINE_PAVA(pava_f32_ext, float, long double)
DEFINE_PAVA(pava_f64_ext, double, quad)

/* Rows of [batch, n]: negation for decreasing fits (_api.py:131-134), then the clip. The
 * negated copy and the scratch are per row, so rows run in parallel (ops.cpp:30 parallelises
 * over rows the same way). threads <= 0: all cores. */
#define DEFINE_FIT(NAME, S, A_REF, A_EXT, PAVA_REF, PAVA_EXT)                                 \
  int NAME(const S* y, const S* w, S* out, uint8_t* starts, int64_t batch, int64_t n,         \
           int increasing, int precision, int clip_lo, int clip_hi, double y_min,            \
           double y_max, int threads) {                                                       \
    if (batch < 0 || n < 0) return 1;                                                         \
    const S lo = (S)y_min, hi = (S)y_max;                                                     \
    int nt = threads;                                                                         \
    (void)nt;                                                                                 \
    int err = 0;                                                                              \
    _Pragma("omp parallel num_threads(nt > 0 ? nt : omp_get_max_threads())")                 \
    {                                                                                         \
      S* neg = (S*)malloc(sizeof(S) * (size_t)(n > 0 ? n : 1));                               \
      int64_t* st = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));              \
      void* wt = malloc(sizeof(A_EXT) * (size_t)(n > 0 ? n : 1));                             \
      void* tt = malloc(sizeof(A_EXT) * (size_t)(n > 0 ? n : 1));                             \
      if (!neg || !st || !wt || !tt) {                                                        \
        _Pragma("omp atomic write") err = 2;                                                  \
      } else {                                                                                \
        _Pragma("omp for schedule(dynamic, 16)")                                              \
        for (int64_t b = 0; b < batch; ++b) {                                                 \
          const S* yr = y + b * n;                                                            \
          S* orow = out + b * n;                                                              \
          if (!increasing) {                                                                  \
            for (int64_t i = 0; i < n; ++i) neg[i] = -yr[i];                                  \
            yr = neg;                                                                         \
          }                                                                                   \
          const S* wr = w ? w + b * n : NULL;                                                 \
          uint8_t* sr = starts ? starts + b * n : NULL;                                       \
          if (precision == PREC_REFERENCE)                                                    \
            PAVA_REF(yr, wr, orow, sr, n, st, (A_REF*)wt, (A_REF*)tt);                        \
          else                                                                                \
            PAVA_EXT(yr, wr, orow, sr, n, st, (A_EXT*)wt, (A_EXT*)tt);                        \
          for (int64_t i = 0; i < n; ++i) {                                                   \
            S v = increasing ? orow[i] : -orow[i];                                            \
            /* torch's clamp: NaN stays NaN; min first, then max (max wins if lo > hi) */     \
            if (clip_lo && v < lo) v = lo;                                                    \
            if (clip_hi && v > hi) v = hi;                                                    \
            orow[i] = v;                                                                      \
          }                                                                                   \
        }                                                                                     \
      }                                                                                       \
      free(neg);                                                                              \
      free(st);                                                                               \
      free(wt);                                                                               \
      free(tt);                                                                               \
    }                                                                                         \
    return err;                                                                               \
  }

#ifndef _OPENMP
static int omp_get_max_threads(void) { return 1; }
#endif

DEFINE_FIT(oracle_fit_f32, float, float, long double, pava_f32_ref, pava_f32_ext)
DEFINE_FIT(oracle_fit_f64, double, double, quad, pava_f64_ref, pava_f64_ext)

/* The gradient of a fit with respect to y and w (_api.py:86-115), in extended precision:
 *   fit:    the unclipped fit ([batch, n]);
 *   starts: where its blocks start (a block also starts at every row's first element);
 *   g:      the upstream gradient of the clipped output; where clip_lo/clip_hi are set, it is
 *           zeroed where the fit lies outside [y_min, y_max] (inclusive bounds pass);
 *   w:      weights or NULL (ones);
 *   y:      the data, needed only for grad_w (NULL: grad_w not computed).
 * grad_y: w G / W; grad_w: (y - fit) G / W, G and W the block sums of the masked g and of w. */
#define DEFINE_GRAD(NAME, S, A)                                                                \
  int NAME(const S* fit, const uint8_t* starts, const S* g, const S* w, const S* y,            \
           S* grad_y, S* grad_w, int64_t batch, int64_t n, int clip_lo, int clip_hi,           \
           double y_min, double y_max, int threads) {                                          \
    if (batch < 0 || n < 0) return 1;                                                          \
    const S lo = (S)y_min, hi = (S)y_max;                                                      \
    int nt = threads;                                                                          \
    (void)nt;                                                                                  \
    _Pragma("omp parallel for num_threads(nt > 0 ? nt : omp_get_max_threads()) schedule(dynamic, 16)") \
    for (int64_t b = 0; b < batch; ++b) {                                                      \
      const int64_t base = b * n;                                                              \
      int64_t i = 0;                                                                           \
      while (i < n) {                                                                          \
        int64_t j = i + 1;                                                                     \
        while (j < n && !starts[base + j]) ++j;                                                \
        A gs = 0, ws = 0;                                                                      \
        for (int64_t k = i; k < j; ++k) {                                                      \
          A gk = (A)g[base + k];                                                               \
          const S f = fit[base + k];                                                           \
          if ((clip_lo && !(f >= lo)) || (clip_hi && !(f <= hi))) gk = 0;                      \
          gs += gk;                                                                            \
          ws += w ? (A)w[base + k] : (A)1;                                                     \
        }                                                                                      \
        const A mean = gs / ws;                                                                \
        for (int64_t k = i; k < j; ++k) {                                                      \
          const A wk = w ? (A)w[base + k] : (A)1;                                              \
          if (grad_y) grad_y[base + k] = (S)(wk * mean);                                       \
          if (grad_w && y) grad_w[base + k] = (S)(((A)y[base + k] - (A)fit[base + k]) * mean); \
        }                                                                                      \
        i = j;                                                                                 \
      }                                                                                        \
    }                                                                                          \
    return 0;                                                                                  \
  }

DEFINE_GRAD(oracle_grad_f32, float, long double)
DEFINE_GRAD(oracle_grad_f64, double, quad)
