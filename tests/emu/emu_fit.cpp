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
    for (int e = 0; e < nseg * n; ++e) {
      const int q = e / n, elem = e - q * n;
      const int u = (q << log2g) + elem / K;
      const int sl = tslot(u, elem & (K - 1), K);
      s.slot_t[sl] = static_cast<S>(y[row0 * n + e]);
      if (kW) s.slot_w[sl] = static_cast<S>(w[row0 * n + e]);
    }
    std::vector<S> y0(THREADS, S(0));
    for (int q = 0; q < nseg; ++q) y0[q] = offset_of(s.slot_t[tslot(q << log2g, 0, K)]);
    for (int t = 0; t < THREADS; ++t) {
      bool nan = false, bad = false;
      thread_pava<S, kW, K>(s, t, t & (G - 1), y0[t >> log2g], increasing != 0, nan, bad);
      if (nan) s.segnan[t >> log2g] = 1;
    }
    // merge rounds: each group's walk, then its survivors moved down in increasing order
    for (int r = 0; r < log2g; ++r) {
      const int gs = 2 << r;
      for (int g0 = 0; g0 < THREADS; g0 += gs) {
        const GroupMove mv = merge_groups<S, kW, K>(s, g0, gs >> 1);
        if (mv.src != mv.dst) {
          for (int i = 0; i < mv.cnt; ++i) move_entry<S, kW>(s, mv.src + i, mv.dst + i);
        }
      }
    }
    // expand, as fit_tile_kernel's 4a: values scattered to block starts (entries last to
    // first), carries, then every thread spreads its values
    auto finish_of = [&](int t, S tt, S ww) {
      const S m = tt / ww;
      return static_cast<S>(increasing ? y0[t >> log2g] + m : y0[t >> log2g] - m);
    };
    for (int t = 0; t < THREADS; ++t) s.starts[t] = 0;
    for (int q = 0; q < (THREADS >> log2g); ++q) {
      const int g0 = q << log2g;
      if (s.segnan[q]) continue;
      const int base = tslot(g0, 0, K);
      for (int i = s.len[g0] - 1; i >= 0; --i) {
        const S val = finish_of(g0, s.slot_t[base + i], entry_w<S, kW>(s, base + i));
        const int f = s.st[base + i];
        s.slot_t[tslot(g0 + f / K, f % K, K)] = val;
        s.starts[g0 + f / K] |= 1u << (f % K);
      }
    }
    std::vector<S> carry(THREADS, S(0));
    for (int t = 0; t < THREADS; ++t) {
      const int g0 = t & ~(G - 1);
      for (int v = t - 1; v >= g0; --v) {
        if (s.starts[v]) {
          int hb = 31;
          while (!((s.starts[v] >> hb) & 1u)) --hb;
          carry[t] = s.slot_t[tslot(v, hb, K)];
          break;
        }
      }
    }
    std::vector<uint32_t> starts_mask(THREADS, 0);
    for (int t = 0; t < THREADS; ++t) {
      if (!s.segnan[t >> log2g]) spread_values<S, K>(s, t, carry[t]);
      starts_mask[t] = s.starts[t];
    }
    for (int t = 0; t < THREADS; ++t) {
      const int q = t >> log2g;
      for (int j = 0; j < s.cnt[t]; ++j) {
        const int elem = (t & (G - 1)) * K + j;
        const int64_t gi = (row0 + q) * n + elem;
        out[gi] = s.segnan[q] ? NAN : static_cast<double>(s.slot_t[tslot(t, j, K)]);
        starts[gi] = s.segnan[q] ? static_cast<uint8_t>(elem == 0)
                                 : static_cast<uint8_t>((starts_mask[t] >> j) & 1u);
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
