// Short rows (n <= N, N = 16 or 32): one thread fits one whole row.
//
// The row is read with 16-byte vector loads (rows of 16-byte multiples; else element by
// element) into a column of shared memory private to the thread - element j of thread t at
// [j][t], so that a warp touching element j of its 32 rows hits distinct banks - as the values
// sign * w * (y - y0) in the sum type (offset_of: pooling decisions do not depend on y0,
// exactness of the double sums does). Pool adjacent violators runs over the row as a state
// machine: each step either pools the stack's top block into the current block or pushes the
// current block and takes the next element. Both candidates (the next element, the stack's top)
// are read every step and the new state is picked by selects, so the threads of a warp take the
// same steps and never split; the warp runs max over its rows of (n + pools) steps. The stack
// of blocks lives in the columns: entry k in row k (written only after element k + 1 was read),
// under a sentinel row -1 (T = -inf, W = 0) that never pools, so the top needs no depth test.
//
// Unweighted rows keep a block's weight (its element count) as 32 bits: the high word of the
// double (the low word of a small integer's double is zero) or the float itself; block starts
// follow from the counts, and 1 / count comes from a table, the quotient T / W then being one
// multiplication and one residual correction (Markstein's method: q0 = T r, q = q0 + r (T - q0 W)
// with r = RN(1 / W), both fused multiply-adds; the residual is exact). Weighted rows keep W in
// the sum type, each entry's first element in 16 bits, and divide.
//
// Expand: each block's value (clipped, in the accumulation type) is written at its first
// element's row (a column whose stack entries at and above that row were read already: blocks
// are taken from the top of the stack down and block k starts at or after row k), then one pass
// along the row spreads the values while packing 16-byte vector stores of the output and of the
// block starts. One launch does the whole fit: one HBM read of y (and w), one write of the fit.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "fit_kernels.cuh"

namespace tiso {

constexpr int kShortThreads = 128;

// An element count of an unweighted block held in 32 bits.
template <typename S>
struct CountBits;
template <>
struct CountBits<double> {
  static constexpr uint32_t kOne = 0x3ff00000u;
  static TISO_DEV uint32_t enc(double w) { return static_cast<uint32_t>(__double2hiint(w)); }
  static TISO_DEV double dec(uint32_t b) { return __hiloint2double(static_cast<int>(b), 0); }
};
template <>
struct CountBits<float> {
  static constexpr uint32_t kOne = 0x3f800000u;
  static TISO_DEV uint32_t enc(float w) { return __float_as_uint(w); }
  static TISO_DEV float dec(uint32_t b) { return __uint_as_float(b); }
};

// Shared memory of the kernel: the reciprocal table, then the columns (N + 1 rows each, the
// first the sentinel).
template <typename S, bool kW, int N, int THREADS>
struct ShortLayout {
  static constexpr int kRcp = (N + 16) / 16 * 16;  // 1 / k for k < kRcp (16-byte multiple)
  static constexpr size_t kRows = N + 1;
  static constexpr size_t kBytes =
      kRcp * sizeof(S) + kRows * THREADS * (kW ? 2 * sizeof(S) + sizeof(uint16_t)
                                               : sizeof(S) + sizeof(uint32_t));
  static_assert(N < kRcp, "the reciprocal table covers every count");
};

template <typename In, typename S, bool kW, bool kInc, int N, int THREADS>
__global__ void __launch_bounds__(THREADS) short_rows_kernel(const FitArgs a) {
  static_assert(N <= 64, "block starts are a 64-bit mask at most");  // launched for N <= 32
  using M = std::conditional_t<(N > 32), unsigned long long, uint32_t>;
  using Acc = acc_of<In>;
  using L = ShortLayout<S, kW, N, THREADS>;
  // fitted values go to the 32-bit column when they fit it (unweighted float32 and narrower),
  // else to the values column
  constexpr bool kOutC = !kW && sizeof(Acc) == 4;
  using O = std::conditional_t<kOutC, Acc, S>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S* rcp = reinterpret_cast<S*>(smem_raw);
  S* col_v = rcp + L::kRcp + THREADS;  // row -1 is the sentinel
  S* col_w = col_v + N * THREADS + THREADS;
  uint16_t* col_s = reinterpret_cast<uint16_t*>(col_w + N * THREADS) + THREADS;
  uint32_t* col_c = reinterpret_cast<uint32_t*>(col_v + N * THREADS) + THREADS;
  const int tid = threadIdx.x;
  if constexpr (!kW) {
    for (int i = tid; i < L::kRcp; i += THREADS) rcp[i] = S(1) / static_cast<S>(i > 0 ? i : 1);
    __syncthreads();
  }
  const int64_t row = static_cast<int64_t>(blockIdx.x) * THREADS + tid;
  if (row >= a.batch) return;  // no barriers below: idle threads may leave
  const int n = a.n;
  const In* yr = static_cast<const In*>(a.y) + row * n;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + row * n : nullptr;
#define TISO_C(arr, j) arr[(j) * THREADS + tid]

  // 1. the values sign * w * (y - y0) into the column (weights into theirs), noting a NaN y and
  //    a weight that is not > 0
  bool nan = false, bad = false;
  S y0;
  constexpr int V = 16 / sizeof(In);
  const bool vec = (n % V) == 0 && (reinterpret_cast<uintptr_t>(yr) & 15) == 0;
  if constexpr (!kW) {
    auto put = [&](int k, In x) {
      const S yv = to_s<S>(x);
      nan |= yv != yv;
      TISO_C(col_v, k) = kInc ? yv - y0 : y0 - yv;
    };
    if (vec) {
      uint4 r[N / V];
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) r[v] = __ldcs(reinterpret_cast<const uint4*>(yr) + v);
      }
      y0 = offset_of(to_s<S>(reinterpret_cast<const In*>(&r[0])[0]));
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
#pragma unroll
          for (int i = 0; i < V; ++i) put(v * V + i, reinterpret_cast<const In*>(&r[v])[i]);
        }
      }
    } else {
      y0 = offset_of(to_s<S>(yr[0]));
      for (int k = 0; k < n; ++k) put(k, yr[k]);
    }
  } else {
    if (vec) {
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
          const uint4 r = __ldcs(reinterpret_cast<const uint4*>(yr) + v);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            TISO_C(col_v, v * V + i) = to_s<S>(reinterpret_cast<const In*>(&r)[i]);
          }
        }
      }
    } else {
      for (int k = 0; k < n; ++k) TISO_C(col_v, k) = to_s<S>(yr[k]);
    }
    constexpr int VW = 16 / sizeof(Acc);
    if ((n % VW) == 0 && (reinterpret_cast<uintptr_t>(wr) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < N / VW; ++v) {
        if (v * VW < n) {
          const uint4 r = __ldcs(reinterpret_cast<const uint4*>(wr) + v);
#pragma unroll
          for (int i = 0; i < VW; ++i) {
            TISO_C(col_w, v * VW + i) = static_cast<S>(reinterpret_cast<const Acc*>(&r)[i]);
          }
        }
      }
    } else {
      for (int k = 0; k < n; ++k) TISO_C(col_w, k) = static_cast<S>(wr[k]);
    }
    y0 = offset_of(TISO_C(col_v, 0));
#pragma unroll
    for (int k = 0; k < N; ++k) {
      if (k < n) {
        const S yv = TISO_C(col_v, k);
        const S wk = TISO_C(col_w, k);
        nan |= yv != yv;
        bad |= !(wk > S(0));
        TISO_C(col_v, k) = (kInc ? yv - y0 : y0 - yv) * wk;
      }
    }
  }

  // 2. PAVA as a state machine over the columns; the stack's top is row `top` (-1: sentinel)
  S ct = TISO_C(col_v, 0);
  S cw = kW ? TISO_C(col_w, 0) : S(1);
  uint32_t cs = 0;                    // weighted: the current block's first element
  uint32_t cwb = CountBits<S>::kOne;  // unweighted: the current block's count, as 32 bits
  TISO_C(col_v, -1) = static_cast<S>(-__longlong_as_double(0x7ff0000000000000LL));
  if constexpr (kW) {
    TISO_C(col_w, -1) = S(0);
    TISO_C(col_s, -1) = 0;
  } else {
    TISO_C(col_c, -1) = 0u;
  }
  int top = -1, j = 1;
  for (;;) {
    const S pt = TISO_C(col_v, top);
    S pw;
    uint32_t pb = 0;
    if constexpr (kW) {
      pw = TISO_C(col_w, top);
      pb = TISO_C(col_s, top);
    } else {
      pw = CountBits<S>::dec(TISO_C(col_c, top));
      cw = CountBits<S>::dec(cwb);
    }
    const bool merge = pool_nb(pt, pw, ct, cw);
    if (!merge && j >= n) break;
    const int jj = j < n ? j : n - 1;
    const S v = TISO_C(col_v, jj);
    if (!merge) {
      TISO_C(col_v, top + 1) = ct;
      if constexpr (kW) {
        TISO_C(col_w, top + 1) = cw;
        TISO_C(col_s, top + 1) = static_cast<uint16_t>(cs);
      } else {
        TISO_C(col_c, top + 1) = cwb;
      }
    }
    ct = merge ? pt + ct : v;
    if constexpr (kW) {
      const S x = TISO_C(col_w, jj);
      cw = merge ? pw + cw : x;
      cs = merge ? pb : static_cast<uint32_t>(jj);
    } else {
      cwb = merge ? CountBits<S>::enc(pw + cw) : CountBits<S>::kOne;
    }
    top += merge ? -1 : 1;
    j += merge ? 0 : 1;
  }
  if constexpr (!kW) cw = CountBits<S>::dec(cwb);
  if (kW && bad && a.bad_weight) *a.bad_weight = 1;

  // 3. values: one per block, at its first element's row; block k starts at or after row k
  O* col_o = kOutC ? reinterpret_cast<O*>(col_c) : reinterpret_cast<O*>(col_v);
  M mask = 0;
  if (nan) {
    mask = 1;
    for (int k = 0; k < n; ++k) TISO_C(col_o, k) = static_cast<O>(nan_of<Acc>());
  } else {
    auto value = [&](S t, S w, int cnt) {
      S m;
      if constexpr (kW) {
        m = t / w;
      } else {
        const S r = rcp[cnt];
        const S q0 = t * r;
        m = fma_(fma_(-q0, w, t), r, q0);
      }
      Acc val = static_cast<Acc>(kInc ? y0 + m : y0 - m);
      if (a.clip_lo && val < static_cast<Acc>(a.lo)) val = static_cast<Acc>(a.lo);
      if (a.clip_hi && val > static_cast<Acc>(a.hi)) val = static_cast<Acc>(a.hi);
      return static_cast<O>(val);
    };
    if constexpr (kW) {
      TISO_C(col_o, cs) = value(ct, cw, 0);
      mask |= M(1) << cs;
      for (int k = top; k >= 0; --k) {
        const int st = TISO_C(col_s, k);
        const O val = value(TISO_C(col_v, k), TISO_C(col_w, k), 0);
        TISO_C(col_o, st) = val;
        mask |= M(1) << st;
      }
    } else {
      int cnt = small_int(cw);
      int st = n - cnt;
      TISO_C(col_o, st) = value(ct, cw, cnt);
      mask |= M(1) << st;
      for (int k = top; k >= 0; --k) {
        const S w = CountBits<S>::dec(TISO_C(col_c, k));
        const S t = TISO_C(col_v, k);
        cnt = small_int(w);
        st -= cnt;
        TISO_C(col_o, st) = value(t, w, cnt);
        mask |= M(1) << st;
      }
    }
  }

  // 4. store the row (and its block starts)
  In* orow = static_cast<In*>(a.out) + row * n;
  {
    Acc cur = static_cast<Acc>(TISO_C(col_o, 0));
    if ((n % V) == 0 && (reinterpret_cast<uintptr_t>(orow) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
          union {
            uint4 u;
            In e[V];
          } pk;
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const int k = v * V + i;
            if ((mask >> k) & 1u) cur = static_cast<Acc>(TISO_C(col_o, k));
            pk.e[i] = from_acc<In>(cur);
          }
          __stcs(reinterpret_cast<uint4*>(orow) + v, pk.u);
        }
      }
    } else {
      for (int k = 0; k < n; ++k) {
        if ((mask >> k) & 1u) cur = static_cast<Acc>(TISO_C(col_o, k));
        orow[k] = from_acc<In>(cur);
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
      for (int k = 0; k < n; ++k) srow[k] = static_cast<uint8_t>((mask >> k) & 1u);
    }
  }
#undef TISO_C
}

}  // namespace tiso
