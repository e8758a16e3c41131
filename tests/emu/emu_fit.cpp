// TEST INFRASTRUCTURE ONLY - runs the tile kernel's phase logic (torchisotonic_b200/csrc/
// fit_core.cuh, the same source the kernel compiles) on the CPU, one emulated thread after
// another between the kernel's barriers, for whole rows (n <= 16 * 256). The kernel's
// staging and expand, which are device-only code in fit_kernels.cuh, are restated here line for
// line. Lets the CPU test suite check the merge bookkeeping against the oracle without a GPU.
#define TISO_HOST_EMU 1
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include "../../torchisotonic_b200/csrc/fit_core.cuh"

using namespace tiso;

namespace {

constexpr int K = 16;
constexpr int THREADS = 256;

template <typename S, bool kW>
void run_rows(const double* y, const double* w, double* out, uint8_t* starts, int64_t batch,
              int n, int increasing) {
  using Sm = TileSmem<S, kW, K, THREADS>;
  auto sp = std::make_unique<Sm>();
  Sm& s = *sp;
  int g = (n + K - 1) / K;
  int log2g = 0;
  while ((1 << log2g) < g) ++log2g;
  const int G = 1 << log2g;
  const int per = THREADS >> log2g;
  for (int64_t row0 = 0; row0 < batch; row0 += per) {
    const int nseg = static_cast<int>(batch - row0 < per ? batch - row0 : per);
    std::memset(&s, 0, sizeof(Sm));
    for (int t = 0; t < THREADS; ++t) {
      const int q = t >> log2g, r = t & (G - 1);
      int c = 0;
      if (q < nseg) {
        c = n - r * K;
        c = c < 0 ? 0 : (c > K ? K : c);
      }
      s.cnt[t] = static_cast<uint8_t>(c);
    }
    const S sign = increasing ? S(1) : S(-1);
    for (int e = 0; e < nseg * n; ++e) {
      const int q = e / n, elem = e - q * n;
      const int u = (q << log2g) + elem / K;
      const int sl = slot_of(u, elem & (K - 1), K);
      const S yv = static_cast<S>(y[row0 * n + e]);
      if (yv != yv) s.segnan[q] = 1;
      if (kW) {
        const S wv = static_cast<S>(w[row0 * n + e]);
        s.slot_t[sl] = sign * (wv * yv);
        s.slot_w[sl] = wv;
      } else {
        s.slot_t[sl] = sign * yv;
      }
    }
    for (int t = 0; t < THREADS; ++t) thread_pava<S, kW, K>(s, t);
    for (int wd = 0; wd < THREADS / 32; ++wd) {
      uint32_t b = 0;
      for (int l = 0; l < 32; ++l) b |= (s.alive[wd * 32 + l] != 0u ? 1u : 0u) << l;
      s.nz[wd] = b;
    }
    for (int r = 0; r < log2g; ++r) {
      const int gs = 2 << r;
      for (int t = 0; t < THREADS; t += gs) merge_lists<S, kW, K>(s, t, t + (gs >> 1), t + gs);
    }
    // expand, as fit_tile_kernel's 4a
    for (int t = 0; t < THREADS; ++t) {
      const int q = t >> log2g;
      const int c = s.cnt[t];
      if (c == 0) continue;
      for (int j = 0; j < c; ++j) {
        const int64_t gi = (row0 + q) * n + (t & (G - 1)) * K + j;
        double v;
        if (s.segnan[q]) {
          v = NAN;
        } else {
          const int seg_first = q << log2g;
          int vt = t, p = 0;
          // the block covering element j: walk back over this thread's alive bits first
          const uint32_t live = ((s.nz[t >> 5] >> (t & 31)) & 1u) ? s.alive[t] : 0u;
          const uint32_t al = live & bits_upto(j);
          S tt = 0, ww = 1;
          if (al) {
            block_sums<S, kW, K>(s, t, high_bit(al), tt, ww);
          } else {
            vt = last_nz(s, seg_first, t);
            p = vt >= 0 ? high_bit(s.alive[vt]) : 0;
            if (vt >= 0) block_sums<S, kW, K>(s, vt, p, tt, ww);
          }
          v = static_cast<double>(tt / ww);
          if (!increasing) v = -v;
        }
        out[gi] = v;
        const uint32_t live = ((s.nz[t >> 5] >> (t & 31)) & 1u) ? s.alive[t] : 0u;
        starts[gi] = s.segnan[q] ? static_cast<uint8_t>(((t & (G - 1)) * K + j) == 0)
                                 : static_cast<uint8_t>((live >> j) & 1u);
      }
    }
  }
}

}  // namespace

extern "C" {
// exact: sums in double; else in float (the exact=False mode of float32 data).
int emu_fit_rows(const double* y, const double* w, double* out, uint8_t* starts, int64_t batch,
                 int n, int increasing, int exact) {
  if (n < 1 || n > K * THREADS) return 1;
  if (exact) {
    if (w) run_rows<double, true>(y, w, out, starts, batch, n, increasing);
    else run_rows<double, false>(y, w, out, starts, batch, n, increasing);
  } else {
    if (w) run_rows<float, true>(y, w, out, starts, batch, n, increasing);
    else run_rows<float, false>(y, w, out, starts, batch, n, increasing);
  }
  return 0;
}

uint32_t emu_fastdiv(uint32_t n, uint32_t d) { return fastdiv(n, make_fastdiv(d)); }
}
