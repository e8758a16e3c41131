// Short rows (n <= N, N = 16, 32 or 64): one thread fits one whole row.
//
// The row is read with 16-byte vector loads (rows of 16-byte multiples; else element by
// element) into a column of shared memory private to the thread - element j of thread t at
// [j][t], so that a warp touching element j of its 32 rows hits distinct banks - in the
// accumulation type. Pool adjacent violators runs over the row as a state machine: each step
// either pools the top two blocks or pushes the next element. Both candidates (the next element,
// the stack entry below) are read every step and the new state is picked by selects, so the
// threads of a warp take the same steps and never split; the warp runs max over its rows of
// (n + pools) steps. The stack of blocks (weighted sum T, weight W, first element) is a second
// set of columns. Values fitted are sign * w * (y - y0) (offset_of: pooling decisions do not
// depend on y0, exactness of the double sums does).
//
// Expand: each block's value (clipped, in the accumulation type) is written at its first
// element's slot of the y column (read already), then one pass along the row spreads the values
// while packing 16-byte vector stores of the output and of the block starts. One launch does
// the whole fit: one HBM read of y (and w) and one write of the output.
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
  // weights of stack entries: the sum type, or an element count
  using WT = std::conditional_t<kW, S, uint16_t>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S* stk_t = reinterpret_cast<S*>(smem_raw);                       // [N][THREADS]
  WT* stk_w = reinterpret_cast<WT*>(stk_t + N * THREADS);          // [N][THREADS]
  Acc* col_y = reinterpret_cast<Acc*>(stk_w + N * THREADS);        // [N][THREADS]: y, then values
  Acc* col_w = col_y + N * THREADS;                                // [N][THREADS]: weights
  uint8_t* stk_s = reinterpret_cast<uint8_t*>(col_w + (kW ? N * THREADS : 0));  // [N][THREADS]
  const int tid = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * THREADS + tid;
  if (row >= a.batch) return;  // no barriers below: idle threads may leave
  const int n = a.n;
  const In* yr = static_cast<const In*>(a.y) + row * n;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + row * n : nullptr;
#define TISO_C(arr, j) arr[(j) * THREADS + tid]

  // 1. load the row (and its weights) into the thread's columns, in the accumulation type
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
          for (int i = 0; i < V; ++i) TISO_C(col_y, v * V + i) = static_cast<Acc>(to_s<S>(e[i]));
        }
      }
    } else {
      for (int j = 0; j < n; ++j) TISO_C(col_y, j) = static_cast<Acc>(to_s<S>(yr[j]));
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
            for (int i = 0; i < VW; ++i) TISO_C(col_w, v * VW + i) = e[i];
          }
        }
      } else {
        for (int j = 0; j < n; ++j) TISO_C(col_w, j) = wr[j];
      }
    }
  }

  // 2. PAVA as a state machine: each step pools the top two blocks or pushes the next element,
  //    so that the threads of a warp take the same steps (n + pools of them at most 2n - 1).
  const S y0 = offset_of(static_cast<S>(TISO_C(col_y, 0)));
  const bool inc = a.increasing != 0;
  bool nan = false, bad = false;
  auto element = [&](int j, S& v, S& x) {
    const S yv = static_cast<S>(TISO_C(col_y, j));
    nan |= yv != yv;
    v = yv - y0;
    x = S(1);
    if constexpr (kW) {
      x = static_cast<S>(TISO_C(col_w, j));
      bad |= !(x > S(0));
      v *= x;
    }
    if (!inc) v = -v;
  };
  S ct, cw, pt = S(0), pw = S(1);  // the top block (cur) and the one below it (prev)
  element(0, ct, cw);
  int cs = 0, ps = 0, depth = 0, j = 1;  // depth: entries below prev
  bool has_prev = false;
  // Each step reads both candidates (the next element, the entry below prev), writes prev to
  // the stack only when it pushes, then picks the new state by selects: no branch but the
  // loop's, so the threads of a warp do not split.
  for (;;) {
    const bool merge = has_prev && pool(pt, pw, ct, cw);
    if (!merge && j >= n) break;
    const int jj = j < n ? j : n - 1;
    S v, x;
    element(jj, v, x);
    const int dd = depth > 0 ? depth - 1 : 0;
    const S bt = TISO_C(stk_t, dd);
    S bw;
    if constexpr (kW) {
      bw = TISO_C(stk_w, dd);
    } else {
      bw = count_as<S>(TISO_C(stk_w, dd));
    }
    const int bs = TISO_C(stk_s, dd);
    if (!merge && has_prev) {
      TISO_C(stk_t, depth) = pt;
      if constexpr (kW) {
        TISO_C(stk_w, depth) = pw;
      } else {
        TISO_C(stk_w, depth) = static_cast<uint16_t>(small_int(pw));
      }
      TISO_C(stk_s, depth) = static_cast<uint8_t>(ps);
    }
    const S ot = ct, ow = cw;
    const int os = cs;
    ct = merge ? ot + pt : v;
    cw = merge ? ow + pw : x;
    cs = merge ? ps : jj;
    pt = merge ? bt : ot;
    pw = merge ? bw : ow;
    ps = merge ? bs : os;
    const bool below = depth > 0;
    depth = merge ? dd : depth + (has_prev ? 1 : 0);
    has_prev = merge ? below : true;
    j += merge ? 0 : 1;
  }
  if (kW && bad && a.bad_weight) *a.bad_weight = 1;

  // 3. values: blocks top down, each at its first element (an element already read); then
  //    spread along the row
  M mask = 0;
  if (nan) {
    mask = 1;
    for (int k = 0; k < n; ++k) TISO_C(col_y, k) = nan_of<Acc>();
  } else {
    auto value = [&](S t, S w) {
      const S m = t / w;
      Acc v = static_cast<Acc>(inc ? y0 + m : y0 - m);
      if (a.clip_lo && v < static_cast<Acc>(a.lo)) v = static_cast<Acc>(a.lo);
      if (a.clip_hi && v > static_cast<Acc>(a.hi)) v = static_cast<Acc>(a.hi);
      return v;
    };
    TISO_C(col_y, cs) = value(ct, cw);
    mask |= M(1) << cs;
    if (has_prev) {
      TISO_C(col_y, ps) = value(pt, pw);
      mask |= M(1) << ps;
    }
    for (int k = depth - 1; k >= 0; --k) {
      S w;
      if constexpr (kW) {
        w = TISO_C(stk_w, k);
      } else {
        w = count_as<S>(TISO_C(stk_w, k));
      }
      const int st = TISO_C(stk_s, k);
      TISO_C(col_y, st) = value(TISO_C(stk_t, k), w);
      mask |= M(1) << st;
    }
  }

  // 4. store the row (and its block starts)
  In* orow = static_cast<In*>(a.out) + row * n;
  {
    constexpr int V = 16 / sizeof(In);
    Acc cur = TISO_C(col_y, 0);
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
            if ((mask >> k) & 1u) cur = TISO_C(col_y, k);
            pk.e[i] = from_acc<In>(cur);
          }
          __stcs(reinterpret_cast<uint4*>(orow) + v, pk.u);
        }
      }
    } else {
      for (int k = 0; k < n; ++k) {
        if ((mask >> k) & 1u) cur = TISO_C(col_y, k);
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
