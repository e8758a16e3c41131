// TEST INFRASTRUCTURE ONLY - builds the reference's own CPU solver into oracle/_ref/ so that
// the parity tests can pin the oracle against it and bench.py can time it as the CPU baseline.
//
// The solver itself is not in this repository: the build includes the reference's header
// src/torchisotonic/csrc/pava.h from the reference checkout (make REF=<checkout>), and this
// file only instantiates it the way the reference's CPU op does (pava<scalar_t, scalar_t,
// int64_t> over rows in parallel, src/torchisotonic/csrc/ops.cpp:26-39) behind a C ABI. A
// decreasing fit negates the data first, as src/torchisotonic/_api.py:131-134 does.
#include <omp.h>

#include <cstdint>
#include <vector>

#include "pava.h"

namespace {

template <typename S>
int fit_rows(const S* y, const S* w, S* out, uint8_t* starts, int64_t batch, int64_t n,
             int increasing, int threads) {
  if (batch < 0 || n < 0) return 1;
  const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt)
  {
    std::vector<int64_t> start(n > 0 ? n : 1);
    std::vector<S> weight(n > 0 ? n : 1), total(n > 0 ? n : 1), ones, neg;
    if (!w) ones.assign(n > 0 ? n : 1, S(1));
    if (!increasing) neg.resize(n > 0 ? n : 1);
#pragma omp for schedule(dynamic, 16)
    for (int64_t b = 0; b < batch; ++b) {
      const S* yr = y + b * n;
      if (!increasing) {
        for (int64_t i = 0; i < n; ++i) neg[i] = -yr[i];
        yr = neg.data();
      }
      S* orow = out + b * n;
      torchisotonic::pava<S, S, int64_t>(yr, w ? w + b * n : ones.data(), orow,
                                         starts ? starts + b * n : nullptr, n, 1, start.data(),
                                         weight.data(), total.data());
      if (!increasing) {
        for (int64_t i = 0; i < n; ++i) orow[i] = -orow[i];
      }
    }
  }
  return 0;
}

}  // namespace

extern "C" {
int ref_fit_f32(const float* y, const float* w, float* out, uint8_t* starts, int64_t batch,
                int64_t n, int increasing, int threads) {
  return fit_rows<float>(y, w, out, starts, batch, n, increasing, threads);
}
int ref_fit_f64(const double* y, const double* w, double* out, uint8_t* starts, int64_t batch,
                int64_t n, int increasing, int threads) {
  return fit_rows<double>(y, w, out, starts, batch, n, increasing, threads);
}
int ref_max_threads(void) { return omp_get_max_threads(); }
}
