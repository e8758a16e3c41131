// Short rows (n <= N, N = 16, 32 or 64): one thread fits one whole row.
//
// The row is read with 16-byte vector loads straight into registers (rows of 16-byte multiples;
// else element by element) and moved to a column of shared memory private to the thread:
// element j of thread t at [j][t], so that a warp touching element j of its 32 rows hits
// distinct banks. Pool adjacent violators then runs over the row with the stack of blocks as
// a bit mask of block starts: the top two blocks' bounds and prefix sums live in registers,
// the prefix sums of the row replace its elements in the column (prefix after element j at
// [j]), and a block below the top two is found by the mask's highest bit under the top's start
// and its prefix sum read back from the column. Values fitted are sign * w * (y - y0), y0 the
// row's first element (the offset keeps the pooling decisions and makes float32 data summed in
// double exact where they vary little around a large value).
//
// Expand: blocks last to first, each block's value written at its last element (its own prefix
// sums, at its last element and before its first, are still there when it is reached), then
// one pass down the row spreads the values; 16-byte vector stores of the output and the block
// starts. One launch does the whole fit: one HBM read of y (and w) and one write of the output.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "fit_kernels.cuh"

namespace tiso {

constexpr int kShortThreads = 128;

template <typename M>
TISO_DEV int mask_high(M x) {
  if constexpr (sizeof(M) == 8) {
    return 63 - __clzll(static_cast<long long>(x));
  } else {
    return 31 - __clz(static_cast<int>(x));
  }
}

template <typename In, typename S, bool kW, int N, int THREADS>
__global__ void __launch_bounds__(THREADS) short_rows_kernel(const FitArgs a) {
  using Acc = acc_of<In>;
  using M = std::conditional_t<(N > 32), unsigned long long, uint32_t>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S* col_t = reinterpret_cast<S*>(smem_raw);   // [N][THREADS]
  S* col_w = col_t + N * THREADS;               // weighted only
  const int tid = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * THREADS + tid;
  if (row >= a.batch) return;  // no barriers below: idle threads may leave
  const int n = a.n;
  const In* yr = static_cast<const In*>(a.y) + row * n;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + row * n : nullptr;
#define TISO_CT(j) col_t[(j) * THREADS + tid]
#define TISO_CW(j) col_w[(j) * THREADS + tid]

  // 1. load the row (and its weights) into the thread's column
  {
    constexpr int V = 16 / sizeof(In);
    if ((n % V) == 0 && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
      uint4 r[N / V];
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) r[v] = __ldcs(reinterpret_cast<const uint4*>(yr) + v);
      }
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
          const In* e = reinterpret_cast<const In*>(&r[v]);
#pragma unroll
          for (int i = 0; i < V; ++i) TISO_CT(v * V + i) = to_s<S>(e[i]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j < n) TISO_CT(j) = to_s<S>(yr[j]);
      }
    }
    if constexpr (kW) {
      constexpr int VW = 16 / sizeof(Acc);
      if ((n % VW) == 0 && (reinterpret_cast<uintptr_t>(wr) & 15) == 0) {
        uint4 r[N / VW];
#pragma unroll
        for (int v = 0; v < N / VW; ++v) {
          if (v * VW < n) r[v] = __ldcs(reinterpret_cast<const uint4*>(wr) + v);
        }
#pragma unroll
        for (int v = 0; v < N / VW; ++v) {
          if (v * VW < n) {
            const Acc* e = reinterpret_cast<const Acc*>(&r[v]);
#pragma unroll
            for (int i = 0; i < VW; ++i) TISO_CW(v * VW + i) = static_cast<S>(e[i]);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < N; ++j) {
          if (j < n) TISO_CW(j) = static_cast<S>(wr[j]);
        }
      }
    }
  }

  // 2. PAVA with a bit-mask stack
  const S y0 = TISO_CT(0);
  const bool inc = a.increasing != 0;
  bool nan = false, bad = false;
  M mask = 0;
  S P = 0, PW = 0;            // prefix sums after the elements so far
  int s = 0, p = -1;          // starts of the top block and of the one below (-1: none)
  S ps = 0, pp = 0;           // prefix sums at those starts
  S pws = 0, pwp = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if (j < n) {
      const S x = TISO_CT(j);
      nan |= x != x;
      S v = x - y0, wj = S(1);
      if constexpr (kW) {
        wj = TISO_CW(j);
        bad |= !(wj > S(0));
        v *= wj;
      }
      if (!inc) v = -v;
      if (j > 0) {
        p = s;
        pp = ps;
        pwp = pws;
      }
      s = j;
      ps = P;
      pws = PW;
      mask |= M(1) << j;
      P += v;
      TISO_CT(j) = P;
      if constexpr (kW) {
        PW += wj;
        TISO_CW(j) = PW;
      }
      while (p >= 0) {
        const S tb = ps - pp, tt = P - ps;
        S wb, wt;
        if constexpr (kW) {
          wb = pws - pwp;
          wt = PW - pws;
        } else {
          wb = count_as<S>(s - p);
          wt = count_as<S>(j + 1 - s);
        }
        if (!pool(tb, wb, tt, wt)) break;
        mask &= ~(M(1) << s);
        s = p;
        ps = pp;
        pws = pwp;
        const M below = mask & ((M(1) << s) - 1);
        if (below) {
          p = mask_high(below);
          pp = p > 0 ? TISO_CT(p - 1) : S(0);
          if constexpr (kW) pwp = p > 0 ? TISO_CW(p - 1) : S(0);
        } else {
          p = -1;
        }
      }
    }
  }
  if (kW && bad && a.bad_weight) *a.bad_weight = 1;

  // 3. values: blocks last to first, each at its last element; then spread down the row
  if (nan) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (j < n) TISO_CT(j) = static_cast<S>(nan_of<Acc>());
    }
    mask = 1;
  } else {
    M rest = mask;
    int end = n;
    while (rest) {
      const int st = mask_high(rest);
      rest &= ~(M(1) << st);
      const S t = TISO_CT(end - 1) - (st > 0 ? TISO_CT(st - 1) : S(0));
      S w;
      if constexpr (kW) {
        w = TISO_CW(end - 1) - (st > 0 ? TISO_CW(st - 1) : S(0));
      } else {
        w = count_as<S>(end - st);
      }
      const S m = t / w;
      Acc val = static_cast<Acc>(inc ? y0 + m : y0 - m);
      if (a.clip_lo && val < static_cast<Acc>(a.lo)) val = static_cast<Acc>(a.lo);
      if (a.clip_hi && val > static_cast<Acc>(a.hi)) val = static_cast<Acc>(a.hi);
      TISO_CT(end - 1) = static_cast<S>(val);
      end = st;
    }
    S cur = 0;
#pragma unroll
    for (int j = N - 1; j >= 0; --j) {
      if (j < n) {
        if (j == n - 1 || ((mask >> (j + 1)) & 1u)) cur = TISO_CT(j);
        TISO_CT(j) = cur;
      }
    }
  }

  // 4. store the row (and its block starts)
  In* orow = static_cast<In*>(a.out) + row * n;
  {
    constexpr int V = 16 / sizeof(In);
    if ((n % V) == 0 && (reinterpret_cast<uintptr_t>(orow) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
          union {
            uint4 u;
            In e[V];
          } pk;
#pragma unroll
          for (int i = 0; i < V; ++i) pk.e[i] = from_acc<In>(static_cast<Acc>(TISO_CT(v * V + i)));
          __stcs(reinterpret_cast<uint4*>(orow) + v, pk.u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j < n) orow[j] = from_acc<In>(static_cast<Acc>(TISO_CT(j)));
      }
    }
  }
  if (a.starts) {
    uint8_t* srow = a.starts + row * n;
    if ((n % 16) == 0 && (reinterpret_cast<uintptr_t>(srow) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < N / 16; ++v) {
        if (v * 16 < n) {
          union {
            uint4 u;
            uint8_t e[16];
          } pk;
#pragma unroll
          for (int i = 0; i < 16; ++i) pk.e[i] = static_cast<uint8_t>((mask >> (v * 16 + i)) & 1u);
          __stcs(reinterpret_cast<uint4*>(srow) + v, pk.u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j < n) srow[j] = static_cast<uint8_t>((mask >> j) & 1u);
      }
    }
  }
#undef TISO_CT
#undef TISO_CW
}

}  // namespace tiso
