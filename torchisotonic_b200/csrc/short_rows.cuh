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
    // a negative weight (flagged; the fit is refused) would pool with the sentinel
    const bool merge = (!kW || top >= 0) && pool_nb(pt, pw, ct, cw);
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


// ---------------------------------------------------------------------------------------------
// Unweighted short rows of float32, float16 or bfloat16 data (n <= N, N = 16 or 32): one thread
// fits one whole row, the row held in registers and walked with a static (unrolled) loop over
// its elements.
//
// Memory: persistent warps, each taking groups of 32 consecutive rows (a contiguous span of
// global memory) in turn. A group is read with coalesced 16-byte loads - lane l takes chunks
// l, l + 32, ... of the span - into the warp's region of shared memory (rows padded by 16 bytes,
// so that a lane reading its own row hits distinct banks), and each lane takes its row from
// there; the next group's chunks are loaded into registers while the current one is fitted. The
// fitted rows go back the same way. Rows whose byte length is not a multiple of 16, or spans
// that are not 16-byte aligned, are read and written element by element instead.
//
// The fit: neighbours that do not increase (y[k-1] >= y[k] for an increasing fit, <= for a
// decreasing one) lie in one block of the fit - a boundary between them would need
// y[k-1] <= mean(left block) < mean(right block) <= y[k] - so the walk accumulates maximal runs of
// them in registers (sums of sign * (y - y0) in the sum type, and counts; the comparisons are
// exact and NaN never pools), and only where a run ends does pool adjacent violators act: the run
// pools with the top of the stack of blocks while they violate, then is pushed. The top of the
// stack is kept in registers, the entries below it in the warp's region (entry k of lane l in
// row k, the sentinel T = -inf, W = 0 that never pools in row -1). On trend-plus-noise rows the
// runs take most of the pooling.
//
// Values, as in short_rows_kernel: each block's mean (T times a table's 1 / count, one residual
// correction), clipped, at the block's first element in the 32-bit column (block k starts at or
// after row k, and the entries at and above k were read already), then spread along the row
// from its block starts. A row holding NaN (found from a float sum of the row, checked element
// by element only when that sum is NaN) skips the fit and comes out NaN with one block.

constexpr int kShortUWarps = 4;  // warps per CTA of short_rows_u_kernel

template <typename S, int N>
struct ShortULayout {
  static constexpr int kRcp = (N + 16) / 16 * 16;  // 1 / k for k < kRcp (16-byte multiple)
  // per warp: the sum column and the 32-bit column, N + 1 rows of 32 lanes each (the sentinel
  // row first); the staging of a group (32 rows of at most N * 4 + 16 bytes) reuses it
  static constexpr size_t kWarpBytes = (N + 1) * 32 * (sizeof(S) + sizeof(uint32_t));
  static constexpr size_t kBytes = kRcp * sizeof(S) + kShortUWarps * kWarpBytes;
  static_assert(N < kRcp, "the reciprocal table covers every count");
  static_assert(32 * (N * 4 + 16) <= kWarpBytes, "a staged group fits the warp's region");
};

// kFull: rows of exactly N elements (the row length a compile-time constant); kPlain: no clip
// and no block starts wanted (their tests left out of the code)
template <typename In, typename S, bool kInc, int N, bool kFull, bool kPlain = false>
__global__ void __launch_bounds__(32 * kShortUWarps) short_rows_u_kernel(const FitArgs a) {
  static_assert(N <= 32, "block starts are a 32-bit mask");
  using Acc = acc_of<In>;
  static_assert(std::is_same_v<Acc, float>, "float32, float16 and bfloat16 data");
  using L = ShortULayout<S, N>;
  constexpr int V = 16 / sizeof(In);           // elements per 16-byte chunk
  constexpr int kMaxC = (N + V - 1) / V;       // chunks of a row of N elements
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S* rcp = reinterpret_cast<S*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < L::kRcp; i += 32 * kShortUWarps) {
    rcp[i] = S(1) / static_cast<S>(i > 0 ? i : 1);
  }
  __syncthreads();
  unsigned char* region = smem_raw + L::kRcp * sizeof(S) + warp * L::kWarpBytes;
  S* col_t = reinterpret_cast<S*>(region) + 32 + lane;  // row 0; row -1 is the sentinel
  uint32_t* col_c = reinterpret_cast<uint32_t*>(region + (N + 1) * 32 * sizeof(S)) + 32 + lane;
  float* col_o = reinterpret_cast<float*>(col_c);
#define TISO_T(k) col_t[(k) * 32]
#define TISO_N(k) col_c[(k) * 32]

  const int n = kFull ? N : a.n;
  const int64_t batch = a.batch;
  const int64_t groups = (batch + 31) / 32;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * kShortUWarps;
  const int row_bytes = n * static_cast<int>(sizeof(In));
  const bool staged = (row_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
  const int cpr = row_bytes >> 4;     // chunks per row (staged)
  const int pitch = row_bytes + 16;   // staged row pitch in shared memory
  // this lane's chunks of a group: where they sit in the staging, and their row
  int soff[kMaxC], srow[kMaxC];
#pragma unroll
  for (int it = 0; it < kMaxC; ++it) {
    const int c = it * 32 + lane;
    const int r = staged ? c / cpr : 0;
    srow[it] = r;
    soff[it] = r * pitch + (c - r * (staged ? cpr : 0)) * 16;
  }
  uint4 pre[kMaxC];
  auto fetch = [&](int64_t gg) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.y) +
                                                      gg * 32 * row_bytes);
    const int64_t rows = batch - gg * 32;
#pragma unroll
    for (int it = 0; it < kMaxC; ++it) {
      if (it < cpr && srow[it] < rows) pre[it] = __ldcs(src + it * 32 + lane);
    }
  };

  int64_t g = static_cast<int64_t>(blockIdx.x) * kShortUWarps + warp;
  if (staged && g < groups) fetch(g);
  for (; g < groups; g += gstride) {
    const int64_t row = g * 32 + lane;
    const int64_t rows = batch - g * 32;  // rows of this group (32 but for the last)
    const bool live = lane < rows;

    // 1. the row into registers
    Acc x[N];
#pragma unroll
    for (int k = 0; k < N; ++k) x[k] = Acc(0);
    if (staged) {
#pragma unroll
      for (int it = 0; it < kMaxC; ++it) {
        if (it < cpr && srow[it] < rows) *reinterpret_cast<uint4*>(region + soff[it]) = pre[it];
      }
      __syncwarp();
      if (live) {
#pragma unroll
        for (int p = 0; p < kMaxC; ++p) {
          if (p < cpr) {
            const uint4 r = *reinterpret_cast<const uint4*>(region + lane * pitch + p * 16);
#pragma unroll
            for (int i = 0; i < V; ++i) {
              if (p * V + i < N) x[p * V + i] = to_s<Acc>(reinterpret_cast<const In*>(&r)[i]);
            }
          }
        }
      }
      __syncwarp();  // the staging is read before the columns reuse it
      if (g + gstride < groups) fetch(g + gstride);
    } else if (live) {
      const In* yr = static_cast<const In*>(a.y) + row * n;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if (k < n) x[k] = to_s<Acc>(yr[k]);
      }
    }

    uint32_t mask = 1;
    if (live) {
      Acc sum = x[0];
#pragma unroll
      for (int k = 1; k < N; ++k) sum += x[k];  // elements past n are 0
      bool nan = sum != sum;
      if (nan) {  // NaN, or +inf and -inf together
        nan = false;
#pragma unroll
        for (int k = 0; k < N; ++k) nan |= x[k] != x[k];
      }
      if (nan) {
        col_o[0] = nan_of<float>();
      } else {
        // 2. runs and the stack; (pt, pwb): the top of the stack (the sentinel at first), sp:
        //    the row the top goes to when a run is pushed over it
        const S y0 = offset_of(static_cast<S>(x[0]));
        S pt = static_cast<S>(neg_inf());
        uint32_t pwb = 0u;
        int sp = -1;
        S rt = S(0), rw = S(0);
#pragma unroll
        for (int k = 0; k < N; ++k) {
          if (k < n) {
            const S v = kInc ? static_cast<S>(x[k]) - y0 : y0 - static_cast<S>(x[k]);
            const bool down = k > 0 && (kInc ? x[k - 1] >= x[k] : x[k - 1] <= x[k]);
            rt = down ? rt + v : v;
            rw = down ? rw + S(1) : S(1);
            const bool more = k + 1 < N && k + 1 < n &&
                              (kInc ? x[k] >= x[k + 1] : x[k] <= x[k + 1]);
            if (!more) {  // the run ends here: pool it with the stack while they violate, push
              S ct = rt, cw = rw;
              S pw = CountBits<S>::dec(pwb);
              bool p = pool_nb(pt, pw, ct, cw);
              if (p) {
                ct = pt + ct;
                cw = pw + cw;
                --sp;
                pt = TISO_T(sp);
                pwb = TISO_N(sp);
                pw = CountBits<S>::dec(pwb);
                p = pool_nb(pt, pw, ct, cw);
              }
              while (p) {
                ct = pt + ct;
                cw = pw + cw;
                --sp;
                pt = TISO_T(sp);
                pwb = TISO_N(sp);
                pw = CountBits<S>::dec(pwb);
                p = pool_nb(pt, pw, ct, cw);
              }
              TISO_T(sp) = pt;
              TISO_N(sp) = pwb;
              ++sp;
              pt = ct;
              pwb = CountBits<S>::enc(cw);
            }
          }
        }

        // 3. values: one per block, at its first element's row; blocks: the top, then rows
        //    sp - 1 down to 0 (row -1 holds the sentinel)
        auto value = [&](S t, S w, int cnt) {
          const S rc = rcp[cnt];
          const S q0 = t * rc;
          const S m = fma_(fma_(-q0, w, t), rc, q0);
          float val = static_cast<float>(kInc ? y0 + m : y0 - m);
          if constexpr (!kPlain) {
            if (a.clip_lo && val < static_cast<float>(a.lo)) val = static_cast<float>(a.lo);
            if (a.clip_hi && val > static_cast<float>(a.hi)) val = static_cast<float>(a.hi);
          }
          return val;
        };
        S cw = CountBits<S>::dec(pwb);
        int cnt = small_int(cw);
        int st = n - cnt;
        col_o[st * 32] = value(pt, cw, cnt);
        mask = 1u << st;
        for (int k = sp - 1; k >= 0; --k) {
          const S w = CountBits<S>::dec(TISO_N(k));
          const S t = TISO_T(k);
          cnt = small_int(w);
          st -= cnt;
          col_o[st * 32] = value(t, w, cnt);
          mask |= 1u << st;
        }
      }
    }

    // 4. the fitted row: spread from the block starts, then stored (and the block starts)
    float res[N];
    {
      float cur = col_o[0];
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if (k > 0 && ((mask >> k) & 1u)) cur = col_o[k * 32];
        res[k] = cur;
      }
    }
    if (staged) {
      __syncwarp();  // every lane has its values out of the columns
      if (live) {
#pragma unroll
        for (int p = 0; p < kMaxC; ++p) {
          if (p < cpr) {
            union {
              uint4 u;
              In e[V];
            } pk;
#pragma unroll
            for (int i = 0; i < V; ++i) pk.e[i] = from_acc<In>(p * V + i < N ? res[p * V + i] : 0.f);
            *reinterpret_cast<uint4*>(region + lane * pitch + p * 16) = pk.u;
          }
        }
      }
      __syncwarp();
      uint4* dst = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out) + g * 32 * row_bytes);
#pragma unroll
      for (int it = 0; it < kMaxC; ++it) {
        if (it < cpr && srow[it] < rows) {
          __stcs(dst + it * 32 + lane, *reinterpret_cast<const uint4*>(region + soff[it]));
        }
      }
      __syncwarp();  // the staging is read out before the next group reuses the region
    } else if (live) {
      In* orow = static_cast<In*>(a.out) + row * n;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if (k < n) orow[k] = from_acc<In>(res[k]);
      }
    }
    if (!kPlain && a.starts && live) {
      uint8_t* srow8 = a.starts + row * n;
      if ((n % 16) == 0 && (reinterpret_cast<uintptr_t>(a.starts) & 15) == 0) {
#pragma unroll
        for (int v = 0; v < N / 16; ++v) {
          if (v * 16 < n) {
            union {
              uint4 u;
              uint8_t e[16];
            } pk;
#pragma unroll
            for (int i = 0; i < 16; ++i) pk.e[i] = static_cast<uint8_t>((mask >> (v * 16 + i)) & 1u);
            __stcs(reinterpret_cast<uint4*>(srow8) + v, pk.u);
          }
        }
      } else {
        for (int k = 0; k < n; ++k) srow8[k] = static_cast<uint8_t>((mask >> k) & 1u);
      }
    }
  }
#undef TISO_T
#undef TISO_N
}

}  // namespace tiso
