// Short rows (n <= N, N = 16 or 32): one thread fits one whole row.
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

template <typename In, typename S, bool kW, bool kInc, int N, int THREADS>
__global__ void __launch_bounds__(THREADS) short_rows_kernel(const FitArgs a) {
  using Acc = acc_of<In>;
  using M = std::conditional_t<(N > 32), unsigned long long, uint32_t>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // columns [N][THREADS]: the values v = sign w (y - y0) (then the stack's T), the weights
  // (weighted: then the stack's W), the stack's first elements (and, unweighted, counts)
  S* col_v = reinterpret_cast<S*>(smem_raw);
  S* col_w = col_v + N * THREADS;                                       // weighted only
  uint32_t* col_s = reinterpret_cast<uint32_t*>(col_w + (kW ? N * THREADS : 0));
  Acc* col_o = reinterpret_cast<Acc*>(col_s + N * THREADS);             // output values
  const int tid = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * THREADS + tid;
  if (row >= a.batch) return;  // no barriers below: idle threads may leave
  const int n = a.n;
  const In* yr = static_cast<const In*>(a.y) + row * n;
  const Acc* wr = kW ? static_cast<const Acc*>(a.w) + row * n : nullptr;
#define TISO_C(arr, j) arr[(j) * THREADS + tid]

  // 1. load the row and its weights into the columns (16-byte vector loads where the rows
  //    allow), then turn y into the values sign * w * (y - y0) in place
  bool nan = false, bad = false;
  {
    constexpr int V = 16 / sizeof(In);
    if ((n % V) == 0 && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
#pragma unroll
      for (int v = 0; v < N / V; ++v) {
        if (v * V < n) {
          const uint4 r = __ldcs(reinterpret_cast<const uint4*>(yr) + v);
#pragma unroll
          for (int i = 0; i < V; ++i) TISO_C(col_v, v * V + i) = to_s<S>(reinterpret_cast<const In*>(&r)[i]);
        }
      }
    } else {
      for (int k = 0; k < n; ++k) TISO_C(col_v, k) = to_s<S>(yr[k]);
    }
    if constexpr (kW) {
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
    }
  }
  const S y0 = offset_of(TISO_C(col_v, 0));
#pragma unroll
  for (int k = 0; k < N; ++k) {
    if (k < n) {
      const S yv = TISO_C(col_v, k);
      nan |= yv != yv;
      S v = kInc ? yv - y0 : y0 - yv;
      if constexpr (kW) {
        const S wk = TISO_C(col_w, k);
        bad |= !(wk > S(0));
        v *= wk;
      }
      TISO_C(col_v, k) = v;
    }
  }

  // 2. PAVA as a state machine: each step pools the top of the stack into the current block or
  //    pushes the current block and takes the next element. Only the current block is held in
  //    registers; the stack top is read every step. Both candidates are read and the new state
  //    picked by selects, so the threads of a warp take the same steps. Stack entry k lives in
  //    slot k of the columns (element k has been read by then).
  S ct = TISO_C(col_v, 0), cw = kW ? TISO_C(col_w, 0) : S(1);
  uint32_t ck = kW ? 0u : (1u << 8);  // first element | (unweighted) count << 8
  int depth = 0, j = 1;
  for (;;) {
    const int tt = depth > 0 ? depth - 1 : 0;
    const S pt = TISO_C(col_v, tt);
    const uint32_t pk = TISO_C(col_s, tt);
    S pw;
    if constexpr (kW) {
      pw = TISO_C(col_w, tt);
    } else {
      pw = count_as<S>(static_cast<int>(pk >> 8));
    }
    const bool merge = depth > 0 && pool_nb(pt, pw, ct, cw);
    if (!merge && j >= n) break;
    const int jj = j < n ? j : n - 1;
    const S v = TISO_C(col_v, jj);
    const S x = kW ? TISO_C(col_w, jj) : S(1);
    if (!merge) {
      TISO_C(col_v, depth) = ct;
      if constexpr (kW) TISO_C(col_w, depth) = cw;
      TISO_C(col_s, depth) = ck;
    }
    ct = merge ? pt + ct : v;
    cw = merge ? pw + cw : x;
    if constexpr (kW) {
      ck = merge ? pk : static_cast<uint32_t>(jj);
    } else {
      ck = merge ? pk + (ck & ~0xffu) : (static_cast<uint32_t>(jj) | (1u << 8));
    }
    depth += merge ? -1 : 1;
    j += merge ? 0 : 1;
  }
  if (kW && bad && a.bad_weight) *a.bad_weight = 1;

  // 3. values: one per block, at its first element; then spread along the row
  M mask = 0;
  if (nan) {
    mask = 1;
    for (int k = 0; k < n; ++k) TISO_C(col_o, k) = nan_of<Acc>();
  } else {
    auto value = [&](S t, S w) {
      const S m = t / w;
      Acc val = static_cast<Acc>(kInc ? y0 + m : y0 - m);
      if (a.clip_lo && val < static_cast<Acc>(a.lo)) val = static_cast<Acc>(a.lo);
      if (a.clip_hi && val > static_cast<Acc>(a.hi)) val = static_cast<Acc>(a.hi);
      return val;
    };
    const int c0 = static_cast<int>(ck & 0xffu);
    TISO_C(col_o, c0) = value(ct, cw);
    mask |= M(1) << c0;
    for (int k = depth - 1; k >= 0; --k) {
      const uint32_t sk = TISO_C(col_s, k);
      S w;
      if constexpr (kW) {
        w = TISO_C(col_w, k);
      } else {
        w = count_as<S>(static_cast<int>(sk >> 8));
      }
      const int st = static_cast<int>(sk & 0xffu);
      TISO_C(col_o, st) = value(TISO_C(col_v, k), w);
      mask |= M(1) << st;
    }
  }

  // 4. store the row (and its block starts)
  In* orow = static_cast<In*>(a.out) + row * n;
  {
    constexpr int V = 16 / sizeof(In);
    Acc cur = TISO_C(col_o, 0);
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
            if ((mask >> k) & 1u) cur = TISO_C(col_o, k);
            pk.e[i] = from_acc<In>(cur);
          }
          __stcs(reinterpret_cast<uint4*>(orow) + v, pk.u);
        }
      }
    } else {
      for (int k = 0; k < n; ++k) {
        if ((mask >> k) & 1u) cur = TISO_C(col_o, k);
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
