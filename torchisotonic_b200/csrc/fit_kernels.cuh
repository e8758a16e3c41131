// Forward kernels: the tile kernel (whole short/medium rows in one launch; tiles of long rows),
// the merge rounds over the tiles of long rows, and the expand of long rows.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "fit_core.cuh"

namespace tiso {

constexpr int kK = 16;          // elements per thread
constexpr int kThreads = 32;    // threads per CTA for whole rows: one warp
constexpr int kTile = kK * kThreads;  // longest row fitted whole by one segment of a CTA
constexpr int kLongThreads = 128;     // threads per CTA for the tiles of long rows: four warps
constexpr int kLongTile = kK * kLongThreads;  // elements per tile of a long row

template <typename In>
using acc_of = std::conditional_t<std::is_same_v<In, double>, double, float>;

template <typename S>
TISO_DEV S to_s(float v) { return static_cast<S>(v); }
template <typename S>
TISO_DEV S to_s(double v) { return static_cast<S>(v); }
template <typename S>
TISO_DEV S to_s(__half v) { return static_cast<S>(__half2float(v)); }
template <typename S>
TISO_DEV S to_s(__nv_bfloat16 v) { return static_cast<S>(__bfloat162float(v)); }

template <typename In>
TISO_DEV In from_acc(acc_of<In> v);
template <>
TISO_DEV float from_acc<float>(float v) { return v; }
template <>
TISO_DEV double from_acc<double>(double v) { return v; }
template <>
TISO_DEV __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <>
TISO_DEV __nv_bfloat16 from_acc<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

struct FitArgs {
  const void* y;
  const void* w;
  void* out;
  uint8_t* starts;
  int64_t batch;
  int32_t n;
  int32_t log2g;     // threads per segment = 2^log2g
  int32_t seg_len;   // n (rows fit a segment) or kTile (tiles of long rows)
  int32_t tiles;     // tiles per row; 1 when rows fit a segment
  int32_t words;     // nz words per row (long rows)
  FastDiv div_n;
  int32_t increasing, clip_lo, clip_hi;
  double lo, hi;
  int32_t* bad_weight;
  // long rows: the tiles' block lists (capacity seg_len each), their alive ranges, NaN flags,
  // and a bit per tile with an alive block
  int32_t* l_start;
  void* l_w;
  void* l_t;
  int32_t* l_lo;
  int32_t* l_hi;
  int32_t* l_nan;
  uint32_t* l_nz;
  int32_t* l_cnt;      // per row, per tree node: arrivals at climb_kernel (zeroed before)
  void* l_ct;          // per tile, from merge_rows_kernel (else NULL): the T and W of the block
  void* l_cw;          // reaching into the tile from the left (W = 0: none)
  int32_t cnt_per_row; // tree nodes per row
  int32_t has_y0;      // y0 given (a segment of a row split across devices): use it
  int32_t whole;       // the CTA fits whole rows (else a tile of a long row)
  double y0;
  // ragged rows (else NULL): row r is elements [offsets[r], offsets[r + 1]) of the packed y, w,
  // out and starts, of at most n elements (longer rows are cut to n: no access beyond them)
  const int64_t* offsets;
};

// Ragged rows: the row of segment q (of the CTA's rows starting at row0) into the geometry in
// shared memory, its length clamped to [0, cap].
template <typename VG>
TISO_DEV void load_var_geom(VG& vg, const int64_t* offsets, int64_t row0, int nseg, int cap) {
  for (int q = threadIdx.x; q < nseg; q += blockDim.x) {
    const int64_t o0 = offsets[row0 + q];
    int64_t len = offsets[row0 + q + 1] - o0;
    len = len < 0 ? 0 : (len > cap ? cap : len);
    vg.ofs[q] = o0;
    vg.len[q] = static_cast<int32_t>(len);
  }
}

// A block's value as written, from its sums of sign * w * (y - y0): the mean, clipped
// (src/torchisotonic/_api.py:68-70).
template <typename Acc, typename S>
TISO_DEV Acc finish(S t, S w, S y0, const FitArgs& a) {
  const S m = t / w;
  Acc v = static_cast<Acc>(a.increasing ? y0 + m : y0 - m);
  if (a.clip_lo && v < static_cast<Acc>(a.lo)) v = static_cast<Acc>(a.lo);
  if (a.clip_hi && v > static_cast<Acc>(a.hi)) v = static_cast<Acc>(a.hi);
  return v;
}

template <typename Acc>
TISO_DEV Acc nan_of() {
  return static_cast<Acc>(__longlong_as_double(0x7ff8000000000000LL));
}

// CTA-wide exclusive prefix sum of one int per thread; returns the total in *total.
template <int THREADS>
TISO_DEV int cta_exclusive_scan(int v, int32_t* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < THREADS / 32 ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < THREADS / 32) scratch[lane] = t;  // inclusive warp totals
    if (lane == THREADS / 32 - 1) scratch[THREADS / 32] = t;
  }
  __syncthreads();
  const int before = (warp == 0 ? 0 : scratch[warp - 1]) + x - v;
  *total = scratch[THREADS / 32];
  return before;
}


// ---------------------------------------------------------------------------------------------
// Staging between global memory and the per-thread slots (thread u's element j at
// u (K + 1) + j). The CTA's elements are a contiguous span of global memory: whole rows
// (segment q, element elem of the row) or one tile of a row. Loads are 16-byte vectors, U per
// thread in flight before any is stored to shared memory, so that enough bytes are in flight
// to cover HBM latency; a span whose start is not 16-byte aligned, and its tail, go scalar.

struct SpanMap {
  int32_t n;       // elements per segment (a row, or the tile)
  int32_t log2g;   // threads per segment = 2^log2g
  FastDiv div;     // by n (whole rows)
  bool whole;
  bool dense;      // whole rows of exactly K 2^log2g elements: segment and element by shifts
  int32_t off;     // slot of thread 0's element 0
};

template <int K, bool kLin = false>
struct SlotIter {
  static constexpr int kLog2K = K == 1 ? 0 : K == 2 ? 1 : K == 4 ? 2 : K == 8 ? 3 : K == 16 ? 4 : 5;
  int e, q, elem;  // e: index in the CTA's span; q, elem: segment and element within it
  // kLin: a tile of a long row (one segment, no wrap): the slot follows from e alone
  TISO_DEV void init(int e0, const SpanMap& m) {
    e = e0;
    if (kLin) {
      q = 0;
      elem = e0;
    } else if (m.dense) {
      q = e0 >> (kLog2K + m.log2g);
      elem = e0 - (q << (kLog2K + m.log2g));
    } else if (m.whole) {
      q = static_cast<int>(fastdiv(static_cast<uint32_t>(e0), m.div));
      elem = e0 - q * m.n;
    } else {
      q = 0;
      elem = e0;
    }
  }
  // segments that fill their threads exactly (and tiles): thread u = e / K, so the slot is
  // e + e / K; else from the segment and element
  TISO_DEV int slot(const SpanMap& m) const {
    if (kLin || m.dense || !m.whole) return e + (e >> kLog2K) + m.off;
    return ((q << m.log2g) + (elem >> kLog2K)) * (K + 1) + (elem & (K - 1)) + m.off;
  }
  TISO_DEV void next(const SpanMap& m) {
    ++e;
    ++elem;
    if (!kLin && elem == m.n) {
      elem = 0;
      ++q;
    }
  }
};

template <typename T>
TISO_DEV uint4 ldg_stream(const T* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

// dst[slot(e)] = convert(src[e]) for e in [0, span): up to V - 1 scalar elements before the
// first 16-byte boundary, then vectors, then the scalar tail.
template <int K, int THREADS, int U, bool kLin, typename T, typename D, typename Conv>
TISO_DEV void stage_in_(const T* __restrict__ src, int span, D* dst, const SpanMap& m, Conv conv) {
  constexpr int V = 16 / sizeof(T);
  const int tid = threadIdx.x;
  int head = static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(src) & 15)) & 15) / sizeof(T));
  head = head < span ? head : span;
  const int nvec = (span - head) / V;
  if (tid < head) {
    SlotIter<K, kLin> it;
    it.init(tid, m);
    dst[it.slot(m)] = conv(src[tid]);
  }
  const T* vsrc = src + head;
  for (int v0 = 0; v0 < nvec; v0 += THREADS * U) {
    uint4 r[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int v = v0 + k * THREADS + tid;
      if (v < nvec) r[k] = ldg_stream(vsrc + static_cast<int64_t>(v) * V);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int v = v0 + k * THREADS + tid;
      if (v < nvec) {
        SlotIter<K, kLin> it;
        it.init(head + v * V, m);
        const T* vals = reinterpret_cast<const T*>(&r[k]);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          dst[it.slot(m)] = conv(vals[i]);
          it.next(m);
        }
      }
    }
  }
  for (int e = head + nvec * V + tid; e < span; e += THREADS) {
    SlotIter<K, kLin> it;
    it.init(e, m);
    dst[it.slot(m)] = conv(src[e]);
  }
}

// Tiles of long rows take the branch-free slot arithmetic (kLin).
template <int K, int THREADS, int U, typename T, typename D, typename Conv>
TISO_DEV void stage_in(const T* __restrict__ src, int span, D* dst, const SpanMap& m, Conv conv) {
  if (!m.whole) {
    stage_in_<K, THREADS, U, true>(src, span, dst, m, conv);
  } else {
    stage_in_<K, THREADS, U, false>(src, span, dst, m, conv);
  }
}

// dst[e] = get(iterator at e) for e in [0, span): scalar head to the first 16-byte boundary,
// 16-byte vector stores, scalar tail.
template <int K, int THREADS, bool kLin, typename T, typename Get>
TISO_DEV void stage_out_(T* __restrict__ dst, int span, const SpanMap& m, Get get) {
  constexpr int V = 16 / sizeof(T);
  const int tid = threadIdx.x;
  int head = static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(dst) & 15)) & 15) / sizeof(T));
  head = head < span ? head : span;
  const int nvec = (span - head) / V;
  if (tid < head) {
    SlotIter<K, kLin> it;
    it.init(tid, m);
    dst[tid] = get(it);
  }
  T* vdst = dst + head;
  for (int v = tid; v < nvec; v += THREADS) {
    SlotIter<K, kLin> it;
    it.init(head + v * V, m);
    union {
      uint4 u;
      T t[V];
    } pack;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      pack.t[i] = get(it);
      it.next(m);
    }
    __stcs(reinterpret_cast<uint4*>(vdst + static_cast<int64_t>(v) * V), pack.u);
  }
  for (int e = head + nvec * V + tid; e < span; e += THREADS) {
    SlotIter<K, kLin> it;
    it.init(e, m);
    dst[e] = get(it);
  }
}

template <int K, int THREADS, typename T, typename Get>
TISO_DEV void stage_out(T* __restrict__ dst, int span, const SpanMap& m, Get get) {
  if (!m.whole) {
    stage_out_<K, THREADS, true>(dst, span, m, get);
  } else {
    stage_out_<K, THREADS, false>(dst, span, m, get);
  }
}


// One CTA: stage, thread PAVA, merge rounds; then the fit of whole rows, or a tile's list.
// kVar: ragged rows (a.offsets), whole rows only; each row staged in and out on its own.
template <typename In, typename S, bool kW, int K, int THREADS, bool kVar = false>
__global__ void __launch_bounds__(THREADS) fit_tile_kernel(const FitArgs a) {
  static_assert(THREADS == 32 || THREADS == kLongThreads, "one warp, or a long row's tile");
  static_assert(!kVar || THREADS == 32, "ragged rows: whole rows in one-warp CTAs");
  using Acc = acc_of<In>;
  using Sm = TileSmem<S, kW, K, THREADS, kVar>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Sm& s = *reinterpret_cast<Sm*>(smem_raw);
  const int tid = threadIdx.x;
  const int log2g = a.log2g;
  const int G = 1 << log2g;
  const bool whole = THREADS == 32 && a.whole;  // one-warp CTAs: whole rows, or 512-tiles

  int64_t gbase, row = 0, tile = 0, row0 = 0;
  int nseg, seglen, span;
  if (whole) {
    row0 = static_cast<int64_t>(blockIdx.x) * (THREADS >> log2g);
    const int64_t left = a.batch - row0;
    nseg = static_cast<int>(left < (THREADS >> log2g) ? left : (THREADS >> log2g));
    seglen = a.n;
    gbase = row0 * a.n;
    span = nseg * a.n;
  } else {
    row = blockIdx.x / a.tiles;
    tile = blockIdx.x - row * a.tiles;
    nseg = 1;
    const int64_t t0 = tile * a.seg_len;
    const int64_t rem = a.n - t0;
    seglen = static_cast<int>(rem < a.seg_len ? rem : a.seg_len);
    gbase = row * a.n + t0;
    span = seglen;
  }
  if constexpr (kVar) {
    load_var_geom(s.vg, a.offsets, row0, nseg, K << log2g);
    __syncthreads();
  }
  {
    const int q = tid >> log2g, r = tid & (G - 1);
    int c = 0;
    if (q < nseg) {
      int sl = seglen;
      if constexpr (kVar) sl = s.vg.len[q];
      c = sl - r * K;
      c = c < 0 ? 0 : (c > K ? K : c);
    }
    s.cnt[tid] = static_cast<uint8_t>(c);
    s.segnan[tid] = 0;
  }
  __syncthreads();

  // 1. staging: y (and w) into the slots, in the sum type
  const SpanMap m{seglen, log2g, a.div_n, whole, whole && seglen == (K << log2g), 1};
  if constexpr (kVar) {
    // each row on its own, coalesced along it
    for (int q = 0; q < nseg; ++q) {
      const int64_t o = s.vg.ofs[q];
      const int len = s.vg.len[q];
      const In* src = static_cast<const In*>(a.y) + o;
      for (int e = tid; e < len; e += THREADS) {
        const int sl = tslot((q << log2g) + e / K, e % K, K);
        s.slot_t[sl] = to_s<S>(src[e]);
        if constexpr (kW) s.slot_w[sl] = static_cast<S>(static_cast<const Acc*>(a.w)[o + e]);
      }
    }
  } else {
    stage_in<K, THREADS, 4>(static_cast<const In*>(a.y) + gbase, span, s.slot_t, m,
                            [](In v) { return to_s<S>(v); });
    if (kW) {
      stage_in<K, THREADS, 4>(static_cast<const Acc*>(a.w) + gbase, span, s.slot_w, m,
                              [](Acc v) { return static_cast<S>(v); });
    }
  }
  __syncthreads();

  // 2. each thread's own PAVA
  // the offset y0 of each segment: its row's first element
  if (whole) {
    if ((tid & (G - 1)) == 0) s.seg_y0[tid >> log2g] = offset_of(s.slot_t[tslot(tid, 0, K)]);
  } else if (tid == 0) {
    s.seg_y0[0] = a.has_y0 ? static_cast<S>(a.y0)
                           : offset_of(to_s<S>(static_cast<const In*>(a.y)[row * a.n]));
  }
  __syncthreads();
  const S y0 = s.seg_y0[tid >> log2g];
  {
    bool nan = false, bad = false;
    thread_pava<S, kW, K>(s, tid, tid & (G - 1), y0, a.increasing != 0, nan, bad);
    if (nan) s.segnan[tid >> log2g] = 1;
    if (kW && bad && a.bad_weight) *a.bad_weight = 1;
  }
  __syncwarp();

  // 3. merge rounds within segments: the group's first thread walks the junction, then the
  //    group's threads move the right list's survivors down (reads, then writes, 2^(r+1) at a
  //    time; every destination is at or below its source)
  using WT = typename Sm::WT;
  for (int r = 0; r < log2g; ++r) {
    const int gs = 2 << r;
    const int g0 = tid & ~(gs - 1);
    if (THREADS == 32 || gs <= 32) {
      // groups within a warp: shuffles and warp barriers
      GroupMove mv{0, 0, 0};
      if (tid == g0) mv = merge_groups<S, kW, K>(s, g0, gs >> 1);
      mv.src = __shfl_sync(0xffffffffu, mv.src, g0 & 31);
      mv.dst = __shfl_sync(0xffffffffu, mv.dst, g0 & 31);
      mv.cnt = __shfl_sync(0xffffffffu, mv.cnt, g0 & 31);
      const int moves = mv.src == mv.dst ? 0 : (mv.cnt + gs - 1) >> (r + 1);
      const int rounds = __reduce_max_sync(0xffffffffu, moves);
      for (int c = 0; c < rounds; ++c) {
        const int i = (c << (r + 1)) + (tid - g0);
        const bool act = i < mv.cnt && moves > 0;
        S t = S(0);
        WT w = WT(0);
        uint16_t f = 0;
        if (act) {
          t = s.slot_t[mv.src + i];
          w = s.slot_w[mv.src + i];
          f = s.st[mv.src + i];
        }
        __syncwarp();
        if (act) {
          s.slot_t[mv.dst + i] = t;
          s.slot_w[mv.dst + i] = w;
          s.st[mv.dst + i] = f;
        }
        __syncwarp();
      }
      __syncwarp();
    } else {
      // groups of several warps: the walk's result through shared memory, CTA barriers
      __syncthreads();
      if (tid == g0) s.mv[tid / gs] = merge_groups<S, kW, K>(s, g0, gs >> 1);
      __syncthreads();
      const GroupMove mv = s.mv[tid / gs];
      const int moves = mv.src == mv.dst ? 0 : (mv.cnt + gs - 1) >> (r + 1);
      int rounds = 0;
      for (int q = 0; q < THREADS / gs; ++q) {
        const GroupMove o = s.mv[q];
        const int m = o.src == o.dst ? 0 : (o.cnt + gs - 1) >> (r + 1);
        rounds = m > rounds ? m : rounds;
      }
      for (int c = 0; c < rounds; ++c) {
        const int i = (c << (r + 1)) + (tid - g0);
        const bool act = i < mv.cnt && moves > 0;
        S t = S(0);
        WT w = WT(0);
        uint16_t f = 0;
        if (act) {
          t = s.slot_t[mv.src + i];
          w = s.slot_w[mv.src + i];
          f = s.st[mv.src + i];
        }
        __syncthreads();
        if (act) {
          s.slot_t[mv.dst + i] = t;
          s.slot_w[mv.dst + i] = w;
          s.st[mv.dst + i] = f;
        }
        __syncthreads();
      }
    }
  }
  __syncthreads();

  if constexpr (THREADS != 32) {
    // (long rows only: whole rows are fitted by one-warp CTAs)
  } else if (whole) {
    // 4a. expand: each block's value at its first element's slot (the segment's list taken from
    //     its end down, G entries at a time, all read before any is written), then every thread
    //     spreads the values over its own slots; stored coalesced.
    const int q = tid >> log2g, g0 = tid & ~(G - 1), me = tid & (G - 1);
    s.starts[tid] = 0;
    __syncwarp();
    if (s.segnan[q]) {
      const int b = tslot(tid, 0, K);
#pragma unroll
      for (int j = 0; j < K; ++j) s.slot_t[b + j] = static_cast<S>(nan_of<Acc>());
      s.starts[tid] = me == 0 ? 1u : 0u;
    }
    const int count = s.segnan[q] ? 0 : s.len[g0];
    const int chunks = (count + G - 1) >> log2g;
    const int rounds = __reduce_max_sync(0xffffffffu, chunks);
    const int base = tslot(g0, 0, K);
    for (int c = rounds - 1; c >= 0; --c) {
      const int i = (c << log2g) + me;
      const bool act = i < count;
      S val = S(0);
      int f = 0;
      if (act) {
        val = static_cast<S>(finish<Acc>(s.slot_t[base + i], entry_w<S, kW>(s, base + i), y0, a));
        f = s.st[base + i];
      }
      __syncwarp();
      if (act) {
        s.slot_t[tslot(g0 + f / K, f % K, K)] = val;
        atomicOr(&s.starts[g0 + f / K], 1u << (f % K));
      }
      __syncwarp();
    }
    // the carry into each thread: the value at the last block start before its first element
    const uint32_t with = __ballot_sync(0xffffffffu, s.starts[tid] != 0);
    const uint32_t before = with & bits_below(tid & 31) & ~bits_below(g0 & 31);
    S carry = S(0);
    if (before) {
      const int v = high_bit(before);
      carry = s.slot_t[tslot((tid & ~31) + v, high_bit(s.starts[(tid & ~31) + v]), K)];
    }
    __syncwarp();
    if (!s.segnan[q]) spread_values<S, K>(s, tid, carry);
    __syncthreads();
    if constexpr (kVar) {
      for (int q2 = 0; q2 < nseg; ++q2) {
        const int64_t o = s.vg.ofs[q2];
        const int len = s.vg.len[q2];
        In* dst = static_cast<In*>(a.out) + o;
        for (int e = tid; e < len; e += THREADS) {
          const int u = (q2 << log2g) + e / K, j = e % K;
          dst[e] = from_acc<In>(static_cast<Acc>(s.slot_t[tslot(u, j, K)]));
          if (a.starts) a.starts[o + e] = static_cast<uint8_t>((s.starts[u] >> j) & 1u);
        }
      }
    } else {
      stage_out<K, THREADS>(static_cast<In*>(a.out) + gbase, span, m, [&](const auto& it) {
        return from_acc<In>(static_cast<Acc>(s.slot_t[it.slot(m)]));
      });
      if (a.starts) {
        stage_out<K, THREADS>(a.starts + gbase, span, m, [&](const auto& it) {
          const int u = (it.q << log2g) + it.elem / K;
          return static_cast<uint8_t>((s.starts[u] >> (it.elem & (K - 1))) & 1u);
        });
      }
    }
  }
  if (!whole) {
    // 4b. a tile of a long row: its list, copied to the tile's list in global memory.
    const int count = s.len[0];
    const int64_t id = row * a.tiles + tile;
    const int64_t lbase = id * static_cast<int64_t>(a.seg_len);
    S* lw = static_cast<S*>(a.l_w);
    S* lt = static_cast<S*>(a.l_t);
    const int32_t t0 = static_cast<int32_t>(tile * a.seg_len);
    const int b = tslot(0, 0, K);
    for (int i = tid; i < count; i += THREADS) {
      a.l_start[lbase + i] = t0 + s.st[b + i];
      lw[lbase + i] = entry_w<S, kW>(s, b + i);
      lt[lbase + i] = s.slot_t[b + i];
    }
    if (tid == 0) {
      a.l_lo[id] = 0;
      a.l_hi[id] = count;
      a.l_nan[id] = s.segnan[0];
    }
    // (the list is read by the merge kernels that follow)
  }
}

// ---------------------------------------------------------------------------------------------
// Long rows: merges of the tiles' lists in global memory. The same junction walk as
// merge_groups (fit_core.cuh), over lists whose alive blocks are [l_lo, l_hi) of each tile's
// list (a bit per tile that still has one); the pooled block overwrites the leftmost block it
// absorbed, tiles emptied in between lose their bit.

TISO_DEV void g_clear_nz(uint32_t* nz, int from, int to) {
  while (from < to) {
    const int w = from >> 5;
    const int lo = w << 5;
    uint32_t bits = ~bits_below(from - lo);
    if (to - lo < 32) bits &= bits_below(to - lo);
    atomicAnd(&nz[w], ~bits);
    from = lo + 32;
  }
}

// Merges the lists of tiles [a0, a1) and [a1, a2) of a row (one thread). Lists written by
// other CTAs are read around L1 (__ldcg): they were published with a fence and an atomic.
template <typename S, int LA = 4>
TISO_DEV void merge_tiles(const FitArgs& a, int64_t row, int a0, int a1, int a2) {
  static_assert(LA >= 1 && LA <= 4, "candidates loaded together: 1 to 4");
  const int64_t base = row * a.tiles;
  if (__ldcg(a.l_nan + base + a0) | __ldcg(a.l_nan + base + a1)) {
    a.l_nan[base + a0] = 1;
    return;
  }
  uint32_t* nz = a.l_nz + row * a.words;
  auto last_nz = [&](int from, int to) {
    while (to > from) {
      const int w = (to - 1) >> 5;
      const int lo = w << 5;
      uint32_t bits = __ldcg(nz + w) & bits_below(to - lo);
      if (from > lo) bits &= ~bits_below(from - lo);
      if (bits) return lo + high_bit(bits);
      to = lo;
    }
    return -1;
  };
  auto first_nz = [&](int from, int to) {
    while (from < to) {
      const int w = from >> 5;
      const int lo = w << 5;
      uint32_t bits = __ldcg(nz + w) & ~bits_below(from - lo);
      if (to - lo < 32) bits &= bits_below(to - lo);
      if (bits) return lo + low_bit(bits);
      from = lo + 32;
    }
    return -1;
  };
  const int ul = last_nz(a0, a1), ur = first_nz(a1, a2);
  if (ul < 0 || ur < 0) return;
  const int64_t cap = a.seg_len;
  S* lw = static_cast<S*>(a.l_w);
  S* lt = static_cast<S*>(a.l_t);
  int32_t* llo = a.l_lo + base;
  int32_t* lhi = a.l_hi + base;
  auto at = [&](int u, int i) { return (base + u) * cap + i; };
  int lu = ul, li = __ldcg(lhi + ul) - 1;  // leftmost absorbed block: tile, index
  int ru = ur, ri = __ldcg(llo + ur);      // rightmost absorbed block
  const S at_ = __ldcg(lt + at(lu, li)), aw = __ldcg(lw + at(lu, li));
  const S bt = __ldcg(lt + at(ru, ri)), bw = __ldcg(lw + at(ru, ri));
  if (!pool(at_, aw, bt, bw)) return;
  S ct = at_ + bt, cw = aw + bw;
  int hi_r = __ldcg(lhi + ru);
  // The candidates on either side, up to LA at a time from one tile (loaded together, so a long
  // walk waits for memory once per LA blocks), slot 0 next; a candidate that did not pool stays
  // loaded while the other side is tried.
  S lbt[4], lbw[4], rbt[4], rbw[4];
  int lcu = lu, llo_u = __ldcg(llo + lu), lci = li - 1, ln = 0;  // left: tile, its lo, index
  int rcu = ru, rhi_u = hi_r, rci = ri + 1, rn = 0;             // right: tile, its hi, index
  bool lmore = true, rmore = true;
  auto left_next = [&]() {
    if (ln > 0 || !lmore) return;
    if (lci < llo_u) {  // this tile is used up: the nearest earlier tile with blocks
      const int pu = last_nz(a0, lcu);
      if (pu < 0) {
        lmore = false;
        return;
      }
      lcu = pu;
      lci = __ldcg(lhi + pu) - 1;
      llo_u = __ldcg(llo + pu);
    }
    ln = lci - llo_u + 1 < LA ? lci - llo_u + 1 : LA;
#pragma unroll
    for (int k = 0; k < LA; ++k) {
      if (k < ln) {
        lbt[k] = __ldcg(lt + at(lcu, lci - k));
        lbw[k] = __ldcg(lw + at(lcu, lci - k));
      }
    }
  };
  auto right_next = [&]() {
    if (rn > 0 || !rmore) return;
    if (rci >= rhi_u) {  // the nearest later tile with blocks
      const int nu = first_nz(rcu + 1, a2);
      if (nu < 0) {
        rmore = false;
        return;
      }
      rcu = nu;
      rci = __ldcg(llo + nu);
      rhi_u = __ldcg(lhi + nu);
    }
    rn = rhi_u - rci < LA ? rhi_u - rci : LA;
#pragma unroll
    for (int k = 0; k < LA; ++k) {
      if (k < rn) {
        rbt[k] = __ldcg(lt + at(rcu, rci + k));
        rbw[k] = __ldcg(lw + at(rcu, rci + k));
      }
    }
  };
  for (;;) {
    left_next();
    if (ln > 0 && pool(lbt[0], lbw[0], ct, cw)) {
      ct += lbt[0];
      cw += lbw[0];
      lu = lcu;
      li = lci;
      if constexpr (LA > 1) {
        lbt[0] = lbt[1]; lbt[1] = lbt[2]; lbt[2] = lbt[3];
        lbw[0] = lbw[1]; lbw[1] = lbw[2]; lbw[2] = lbw[3];
      }
      --ln;
      --lci;
      continue;
    }
    right_next();
    if (rn > 0 && pool(ct, cw, rbt[0], rbw[0])) {
      ct += rbt[0];
      cw += rbw[0];
      ru = rcu;
      ri = rci;
      hi_r = rhi_u;
      if constexpr (LA > 1) {
        rbt[0] = rbt[1]; rbt[1] = rbt[2]; rbt[2] = rbt[3];
        rbw[0] = rbw[1]; rbw[1] = rbw[2]; rbw[2] = rbw[3];
      }
      --rn;
      ++rci;
      continue;
    }
    break;
  }
  lt[at(lu, li)] = ct;
  lw[at(lu, li)] = cw;
  lhi[lu] = li + 1;
  g_clear_nz(nz, lu + 1, ru);
  llo[ru] = ri + 1;
  if (ri + 1 >= hi_r) g_clear_nz(nz, ru, ru + 1);
}

// The whole tree of tile merges of each row in one launch: a warp per row, its lanes taking the
// merges of one level at a time (a fence and a warp barrier between levels). Rows proceed in
// parallel; a row's levels one after the other.
template <typename S>
__global__ void merge_rows_kernel(const FitArgs a) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= a.batch) return;  // whole warps leave together
  const int lane = threadIdx.x & 31;
  for (int span = 2; span / 2 < a.tiles; span *= 2) {
    const int groups = (a.tiles + span - 1) / span;
    for (int g = lane; g < groups; g += 32) {
      const int a0 = g * span, a1 = a0 + span / 2;
      if (a1 < a.tiles) {
        merge_tiles<S, 1>(a, row, a0, a1, a0 + span < a.tiles ? a0 + span : a.tiles);
      }
    }
    __threadfence();
    __syncwarp();
  }
  // each tile's carry for the expand: the sums of the last alive block of the nearest earlier
  // tile with one (32 tiles at a time: a ballot of the tiles' bits, the highest below each lane)
  if (!a.l_ct) return;
  const int64_t base = row * a.tiles;
  const uint32_t* nz = a.l_nz + row * a.words;
  const S* lt = static_cast<const S*>(a.l_t);
  const S* lw = static_cast<const S*>(a.l_w);
  S* ct = static_cast<S*>(a.l_ct);
  S* cw = static_cast<S*>(a.l_cw);
  int before = -1;  // the last tile with a block before this chunk
  for (int c0 = 0; c0 < a.tiles; c0 += 32) {
    const int t = c0 + lane;
    const bool has = t < a.tiles && ((__ldcg(nz + (t >> 5)) >> (t & 31)) & 1u);
    const uint32_t bits = __ballot_sync(0xffffffffu, has);
    const uint32_t below = bits & bits_below(lane);
    const int src = below ? c0 + high_bit(below) : before;
    if (t < a.tiles) {
      S st = S(0), sw = S(0);
      if (src >= 0) {
        const int64_t i = (base + src) * static_cast<int64_t>(a.seg_len) + __ldcg(a.l_hi + base + src) - 1;
        st = __ldcg(lt + i);
        sw = __ldcg(lw + i);
      }
      ct[base + t] = st;
      cw[base + t] = sw;
    }
    if (bits) before = c0 + high_bit(bits);
  }
}

// The tree of tile merges of few, long rows: a thread per pair of tiles merges them (level 0;
// both tiles are done when the kernel starts), then climbs - at each level above, the second of
// two sibling groups to arrive (an atomic counter per tree node) merges them and goes on, the
// first leaves. No thread ever waits on another, and the merges of a level overlap.
template <typename S>
__global__ void climb_kernel(const FitArgs a, int64_t pairs_per_row) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = gid / pairs_per_row;
  if (row >= a.batch) return;
  const int tile = static_cast<int>(gid - row * pairs_per_row) * 2;
  if (tile + 1 < a.tiles) merge_tiles<S>(a, row, tile, tile + 1, tile + 2);
  __threadfence();
  int32_t* cnt = a.l_cnt + row * a.cnt_per_row;
  int off = 0;
  for (int level = 1;; ++level) {
    const int span = 2 << level, half = span >> 1;
    if (half >= a.tiles) return;  // the group below covers the row
    off += (a.tiles + (span >> 1) - 1) / (span >> 1);  // the counters of the level below
    const int node = tile / span;
    const int a0 = node * span, a1 = a0 + half;
    if (a1 < a.tiles) {
      const int a2 = a0 + span < a.tiles ? a0 + span : a.tiles;
      if (atomicAdd(cnt + off + node, 1) == 0) return;  // the sibling group goes on
      __threadfence();
      merge_tiles<S>(a, row, a0, a1, a2);
      __threadfence();
    }
  }
}

// Long rows after the last merge level: each tile writes its elements from its own alive blocks
// and the block reaching into it from the left (the last alive block of the nearest tile before
// it with one). The alive blocks' values go to shared memory in list order and their first
// elements to a bitmap of the tile; with each bitmap word's count of starts before it, the block
// of element e is one popcount away (the starts at or before e, less one), so every thread
// writes 16-byte groups of consecutive elements, the warp's stores contiguous. Tiles of one warp
// go four to a CTA (a warp each, warp barriers), so that more of these short latency-bound
// tiles are resident than one-warp CTAs allow.
template <typename In, typename S, int K, int THREADS>
struct ExpandSmem {
  static constexpr int kCap = K * THREADS;
  static constexpr int kWords = kCap / 32;
  acc_of<In> val[kCap];
  uint32_t bits[kWords];
  int32_t pref[kWords];  // starts in the words before
  acc_of<In> carry;
};

template <int THREADS>
constexpr int kExpandTilesPerCta = THREADS >= 128 ? 1 : 128 / THREADS;

template <typename In, typename S, int K, int THREADS>
__global__ void __launch_bounds__(THREADS * kExpandTilesPerCta<THREADS>)
    expand_kernel(const FitArgs a) {
  using Acc = acc_of<In>;
  using Sm = ExpandSmem<In, S, K, THREADS>;
  constexpr int kWords = Sm::kWords;
  constexpr int TP = kExpandTilesPerCta<THREADS>;
  static_assert(kWords <= 64 && kWords % 2 == 0, "a tile's bitmap: at most two words a lane");
  static_assert(TP == 1 || THREADS == 32, "several tiles a CTA: one warp each");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int sub = static_cast<int>(threadIdx.x) / THREADS;
  Sm& s = reinterpret_cast<Sm*>(smem_raw)[sub];
  const int tid = static_cast<int>(threadIdx.x) % THREADS;
  const int64_t id = static_cast<int64_t>(blockIdx.x) * TP + sub;
  if (id >= a.batch * a.tiles) return;  // the whole warp (one tile a warp)
  auto sync = [] {
    if constexpr (TP > 1) {
      __syncwarp();
    } else {
      __syncthreads();
    }
  };
  const int64_t row = id / a.tiles;
  const int tile = static_cast<int>(id - row * a.tiles);
  const int32_t t0 = tile * a.seg_len;
  const int seglen = (a.n - t0) < a.seg_len ? (a.n - t0) : a.seg_len;
  const int64_t gbase = row * a.n + t0;
  In* out = static_cast<In*>(a.out);

  // everything the tile needs that does not depend on anything else, loaded at once
  const uint32_t* nz = a.l_nz + row * a.words;
  const int nan_row = a.l_nan[row * a.tiles];
  const uint32_t word = nz[tile >> 5];
  const int lo_raw = a.l_lo[id], hi_raw = a.l_hi[id];
  const S y0 = a.has_y0 ? static_cast<S>(a.y0)
                        : offset_of(to_s<S>(static_cast<const In*>(a.y)[row * a.n]));
  if (nan_row) {
    for (int e = tid; e < seglen; e += THREADS) {
      out[gbase + e] = from_acc<In>(nan_of<Acc>());
      if (a.starts) a.starts[gbase + e] = static_cast<uint8_t>(t0 + e == 0);
    }
    return;
  }
  for (int w = tid; w < kWords; w += THREADS) s.bits[w] = 0u;
  sync();
  const bool has = (word >> (tile & 31)) & 1u;
  const int lo = has ? lo_raw : 0;
  const int cnt = has ? hi_raw - lo : 0;
  const S* lw = static_cast<const S*>(a.l_w);
  const S* lt = static_cast<const S*>(a.l_t);
  const int64_t lbase = id * static_cast<int64_t>(a.seg_len) + lo;
  for (int i = tid; i < cnt; i += THREADS) {
    const int rel = a.l_start[lbase + i] - t0;
    s.val[i] = finish<Acc>(lt[lbase + i], lw[lbase + i], y0, a);
    atomicOr(&s.bits[rel >> 5], 1u << (rel & 31));
  }
  // the block reaching in from the left: the last alive block of the nearest earlier tile with
  // one, looked for by the tile's first warp 32 bit words (1024 tiles) at a time
  if (a.l_ct) {
    if (tid == 0) {
      const S w = static_cast<const S*>(a.l_cw)[id];
      s.carry = w > S(0) ? finish<Acc>(static_cast<const S*>(a.l_ct)[id], w, y0, a)
                         : nan_of<Acc>();
    }
  } else if (tid < 32) {
    const bool need = cnt == 0 || a.l_start[lbase] > t0;
    Acc carry = nan_of<Acc>();
    if (need) {  // the same on every lane: one tile per warp
      int v = -1;
      for (int top = tile; top > 0 && v < 0;) {  // tiles [0, top) left to search
        const int wtop = (top - 1) >> 5;
        const int w = wtop - tid;
        uint32_t bits = 0;
        if (w >= 0) {
          bits = nz[w];
          if ((w << 5) + 32 > top) bits &= bits_below(top - (w << 5));
        }
        const uint32_t any = __ballot_sync(0xffffffffu, bits != 0);
        if (any) {
          const int l = low_bit(any);
          v = ((wtop - l) << 5) + high_bit(__shfl_sync(0xffffffffu, bits, l));
        }
        top = (wtop - 31) << 5;
      }
      if (v >= 0 && tid == 0) {
        const int64_t vi = (row * a.tiles + v) * static_cast<int64_t>(a.seg_len) +
                           a.l_hi[row * a.tiles + v] - 1;
        carry = finish<Acc>(lt[vi], lw[vi], y0, a);
      }
    }
    if (tid == 0) s.carry = carry;
  }
  sync();
  // each word's count of starts before it: the tile's first warp, two words a lane
  if (tid < 32) {
    const int w0 = 2 * tid;
    const int c0 = w0 < kWords ? __popc(s.bits[w0]) : 0;
    const int c1 = w0 + 1 < kWords ? __popc(s.bits[w0 + 1]) : 0;
    int incl = c0 + c1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, d);
      if (tid >= d) incl += o;
    }
    const int excl = incl - c0 - c1;
    if (w0 < kWords) s.pref[w0] = excl;
    if (w0 + 1 < kWords) s.pref[w0 + 1] = excl + c0;
  }
  sync();
  // groups of V consecutive elements, 16 bytes of output each
  constexpr int V = 16 / sizeof(In);
  const bool vec = ((reinterpret_cast<uintptr_t>(out + gbase)) & 15) == 0;
  const int groups = (seglen + V - 1) / V;
  for (int gi = tid; gi < groups; gi += THREADS) {
    const int e0 = gi * V;
    union {
      uint4 u;
      In e[V];
    } pk;
    uint8_t fl[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int e = e0 + k;
      const int wi = e >> 5;
      const uint32_t bw = e < seglen ? s.bits[wi] : 0u;
      const int idx = e < seglen ? s.pref[wi] + __popc(bw & ((2u << (e & 31)) - 1u)) - 1 : -1;
      const Acc v = idx >= 0 ? s.val[idx] : s.carry;
      pk.e[k] = from_acc<In>(v);
      fl[k] = static_cast<uint8_t>((bw >> (e & 31)) & 1u);
    }
    if (vec && e0 + V <= seglen) {
      *reinterpret_cast<uint4*>(out + gbase + e0) = pk.u;
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (e0 + k < seglen) out[gbase + e0 + k] = pk.e[k];
      }
    }
    if (a.starts) {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (e0 + k < seglen) a.starts[gbase + e0 + k] = fl[k];
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// One long row split into contiguous segments across devices. Each device fits its segment with
// the tile kernel and the climb kernel (the row's offset y0 given) and compacts the segment's alive
// blocks into a list; the lists of all segments are gathered; every device merges them (the
// same junction merges, one list per "tile") and expands its own segment.

// Per tile of the segment: its number of alive blocks.
__global__ void seg_count_kernel(const FitArgs a, int32_t* counts) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= a.tiles) return;
  const bool has = (a.l_nz[t >> 5] >> (t & 31)) & 1u;
  counts[t] = has ? a.l_hi[t] - a.l_lo[t] : 0;
}

// Exclusive prefix sums of counts[0, m) into offs (and the total into offs[m]), in chunks of
// THREADS counts: (1) each chunk's total, one CTA per chunk; (2) one CTA scans the totals;
// (3) each chunk's own scan plus its base.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) seg_chunk_total_kernel(const int32_t* counts,
                                                                   int64_t* chunk, int m) {
  __shared__ int32_t scratch[THREADS / 32 + 1];
  const int i = blockIdx.x * THREADS + threadIdx.x;
  int total;
  cta_exclusive_scan<THREADS>(i < m ? counts[i] : 0, scratch, &total);
  if (threadIdx.x == 0) chunk[blockIdx.x] = total;
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) seg_chunk_scan_kernel(int64_t* chunk, int chunks,
                                                                  int64_t* offs, int m) {
  __shared__ int64_t scratch[THREADS];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < chunks; c0 += THREADS) {
    const int c = c0 + threadIdx.x;
    const int64_t v = c < chunks ? chunk[c] : 0;
    scratch[threadIdx.x] = v;
    __syncthreads();
    for (int d = 1; d < THREADS; d <<= 1) {  // inclusive Hillis-Steele scan of 64-bit totals
      const int64_t add = threadIdx.x >= d ? scratch[threadIdx.x - d] : 0;
      __syncthreads();
      scratch[threadIdx.x] += add;
      __syncthreads();
    }
    if (c < chunks) chunk[c] = carry + scratch[threadIdx.x] - v;  // exclusive, with the carry
    __syncthreads();
    if (threadIdx.x == 0) carry += scratch[THREADS - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) offs[m] = carry;
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) seg_chunk_fill_kernel(const int32_t* counts,
                                                                  const int64_t* chunk,
                                                                  int64_t* offs, int m) {
  __shared__ int32_t scratch[THREADS / 32 + 1];
  const int i = blockIdx.x * THREADS + threadIdx.x;
  int total;
  const int before = cta_exclusive_scan<THREADS>(i < m ? counts[i] : 0, scratch, &total);
  if (i < m) offs[i] = chunk[blockIdx.x] + before;
}

// The segment's alive blocks, in order: global first element, T, W (double).
template <typename S>
__global__ void seg_gather_kernel(const FitArgs a, const int64_t* offs, int64_t seg_start,
                                  int64_t* blk_start, double* blk_t, double* blk_w,
                                  int32_t* count, int32_t* nan) {
  const int t = blockIdx.x;
  if (t >= a.tiles) return;
  const bool has = (a.l_nz[t >> 5] >> (t & 31)) & 1u;
  const int lo = a.l_lo[t], m = has ? a.l_hi[t] - lo : 0;
  const int64_t src = static_cast<int64_t>(t) * a.seg_len + lo, dst = offs[t];
  const S* lw = static_cast<const S*>(a.l_w);
  const S* lt = static_cast<const S*>(a.l_t);
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    blk_start[dst + i] = seg_start + a.l_start[src + i];
    blk_t[dst + i] = static_cast<double>(lt[src + i]);
    blk_w[dst + i] = static_cast<double>(lw[src + i]);
  }
  if (t == 0 && threadIdx.x == 0) {
    *count = static_cast<int32_t>(offs[a.tiles]);
    *nan = a.l_nan[0];
  }
}

// The gathered lists as the tiles of one row: alive ranges [0, count), NaN flags, nz bits.
__global__ void seg_init_kernel(int parts, const int32_t* counts, const int32_t* nans,
                                int32_t* lo, int32_t* hi, int32_t* nan, uint32_t* nz) {
  const int k = threadIdx.x;
  if (k < parts) {
    lo[k] = 0;
    hi[k] = counts[k];
    nan[k] = nans[k];
  }
  const uint32_t b = __ballot_sync(0xffffffffu, k < parts && counts[k] > 0);
  if (k == 0) nz[0] = b;
}

// The fit of this device's segment from the merged lists, a CTA per 512-element tile of the
// segment: the tile's own alive blocks - those of list `me` that start in it, found from the
// tile's offset in the segment's compacted list (tile_offs, from the segment fit's scan) - with
// their values staged in shared memory, and the block reaching in from the left (the alive
// block before them in the list, or the last alive block of the nearest list before it).
// Each element's block by a binary search over the tile's blocks in shared memory.
template <typename In>
__global__ void __launch_bounds__(128) seg_expand_tiles_kernel(const FitArgs a, int me,
                                                               const int64_t* blk_start,
                                                               const int64_t* tile_offs,
                                                               int64_t seg_n, int64_t seg_start) {
  using Acc = acc_of<In>;
  constexpr int E = kTile;
  __shared__ int32_t s_start[E];  // block starts relative to the tile's first element
  __shared__ Acc s_val[E];
  __shared__ Acc s_carry;
  const int64_t t = blockIdx.x;
  const int64_t e0 = t * E;
  if (e0 >= seg_n) return;
  const int len = static_cast<int>(seg_n - e0 < E ? seg_n - e0 : E);
  In* out = static_cast<In*>(a.out) + e0;
  uint8_t* st = a.starts ? a.starts + e0 : nullptr;
  if (a.l_nan[0]) {
    for (int e = threadIdx.x; e < len; e += blockDim.x) {
      out[e] = from_acc<In>(nan_of<Acc>());
      if (st) st[e] = static_cast<uint8_t>(seg_start + e0 + e == 0);
    }
    return;
  }
  const double* lw = static_cast<const double*>(a.l_w);
  const double* lt = static_cast<const double*>(a.l_t);
  const int64_t base = static_cast<int64_t>(me) * a.seg_len;
  const bool has = (a.l_nz[me >> 5] >> (me & 31)) & 1u;
  const int64_t lo = has ? a.l_lo[me] : 0, hi = has ? a.l_hi[me] : 0;
  const int64_t b0 = tile_offs[t] > lo ? tile_offs[t] : lo;
  int64_t b1 = tile_offs[t + 1] < hi ? tile_offs[t + 1] : hi;
  if (b1 < b0) b1 = b0;
  const int nb = static_cast<int>(b1 - b0);  // at most E: the blocks start in the tile
  FitArgs fa = a;
  auto value = [&](int64_t i) { return finish<Acc>(lt[i], lw[i], a.y0, fa); };
  for (int i = threadIdx.x; i < nb; i += blockDim.x) {
    s_start[i] = static_cast<int32_t>(blk_start[base + b0 + i] - (seg_start + e0));
    s_val[i] = value(base + b0 + i);
  }
  if (threadIdx.x == 0) {
    // the last alive block before the tile's own: before b0, and at most the list's last one
    // (tiles whose blocks were all absorbed into it by the merge with the later lists)
    const int64_t c = (b0 < hi ? b0 : hi) - 1;
    Acc carry = nan_of<Acc>();
    if (has && c >= lo) {
      carry = value(base + c);
    } else {
      for (int k = me - 1; k >= 0; --k) {
        if ((a.l_nz[k >> 5] >> (k & 31)) & 1u) {
          carry = value(static_cast<int64_t>(k) * a.seg_len + a.l_hi[k] - 1);
          break;
        }
      }
    }
    s_carry = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < len; e += blockDim.x) {
    int l = 0, r = nb;  // the last block starting at or before e
    while (l < r) {
      const int mid = (l + r) >> 1;
      if (s_start[mid] <= e) l = mid + 1; else r = mid;
    }
    const Acc v = l > 0 ? s_val[l - 1] : s_carry;
    out[e] = from_acc<In>(v);
    if (st) st[e] = static_cast<uint8_t>(l > 0 && s_start[l - 1] == e);
  }
}

// The fit of this device's segment from the merged lists: its own alive blocks (list `me`) and
// the block reaching in from the left (the last alive block of the nearest list before it).
// A thread per 16 elements: a binary search for its first element's block, then a walk.
template <typename In>
__global__ void seg_expand_kernel(const FitArgs a, int me, const int64_t* blk_start,
                                  int64_t seg_n, int64_t seg_start) {
  using Acc = acc_of<In>;
  constexpr int E = 16;
  const int64_t e0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * E;
  if (e0 >= seg_n) return;
  In* out = static_cast<In*>(a.out);
  const double* lw = static_cast<const double*>(a.l_w);
  const double* lt = static_cast<const double*>(a.l_t);
  const int64_t cap = a.seg_len;
  const int64_t end = e0 + E < seg_n ? e0 + E : seg_n;
  if (a.l_nan[0]) {
    for (int64_t e = e0; e < end; ++e) {
      out[e] = from_acc<In>(nan_of<Acc>());
      if (a.starts) a.starts[e] = static_cast<uint8_t>(seg_start + e == 0);
    }
    return;
  }
  const bool has = (a.l_nz[me >> 5] >> (me & 31)) & 1u;
  const int lo = has ? a.l_lo[me] : 0, hi = has ? a.l_hi[me] : 0;
  const int64_t base = static_cast<int64_t>(me) * cap;
  // last own block starting at or before e0 (binary search over [lo, hi))
  int l = lo, r = hi;
  while (l < r) {
    const int mid = (l + r) >> 1;
    if (blk_start[base + mid] <= seg_start + e0) l = mid + 1; else r = mid;
  }
  int idx = l - 1;  // < lo: the block reaching in from the left
  FitArgs fa = a;
  auto value = [&](double t, double w) { return finish<Acc>(t, w, a.y0, fa); };
  Acc cur;
  if (idx >= lo) {
    cur = value(lt[base + idx], lw[base + idx]);
  } else {
    int v = -1;
    for (int k = me - 1; k >= 0; --k) {
      if ((a.l_nz[k >> 5] >> (k & 31)) & 1u) {
        v = k;
        break;
      }
    }
    cur = nan_of<Acc>();
    if (v >= 0) {
      const int64_t vi = static_cast<int64_t>(v) * cap + a.l_hi[v] - 1;
      cur = value(lt[vi], lw[vi]);
    }
  }
  int64_t next = idx + 1 < hi ? blk_start[base + idx + 1] : INT64_MAX;
  for (int64_t e = e0; e < end; ++e) {
    const int64_t g = seg_start + e;
    uint8_t flag = (idx >= lo && blk_start[base + idx] == g) ? 1 : 0;
    while (next <= g) {
      ++idx;
      cur = value(lt[base + idx], lw[base + idx]);
      flag = next == g ? 1 : 0;
      next = idx + 1 < hi ? blk_start[base + idx + 1] : INT64_MAX;
    }
    out[e] = from_acc<In>(cur);
    if (a.starts) a.starts[e] = flag;
  }
}

}  // namespace tiso
