// The forward fit inside one CTA: the phases of the tile kernel, written once for the device and
// for the CPU emulator (tests/emu), which runs each phase for every thread (or group) in turn.
//
// A CTA of THREADS threads holds THREADS / G row segments ("segments") of up to G * K elements:
// whole rows when a row fits (n <= G K), else one tile of a long row (G = THREADS). Thread u of
// the CTA owns elements [(u % G) K, (u % G) K + K) of segment u / G.
//
// 1. Staging: the CTA's elements are read coalesced into shared memory, y and w in the sum type
//    S, thread u's element j at slot tslot(u, j) = u (K + 1) + 1 + j (one spare slot per thread:
//    a warp reading slot j of its 32 threads hits distinct banks; slot 0 is thread 0's spare).
// 2. thread_pava: each thread runs pool adjacent violators over its K elements, fitting
//    sign * w * (y - y0), y0 the row's first element. The offset leaves every pooling decision
//    unchanged and keeps the sums small, so that float32 data summed in double stay exact where
//    the data vary little around a large value. The thread's stack of blocks (weighted sum T,
//    weight W, first element in the segment) lives in its own slots - entry k in slot k, written
//    only once element k + 1 has been read - over a sentinel (T = -inf, W = 0, never pooled) in
//    the spare slot just below them. The loop is a state machine - each step either pools the
//    stack's top into the current block or pushes it and takes the next element - so that the
//    threads of a warp stay in step. The thread's list is its stack: entries [0, len).
// 3. merge_groups: log2(G) rounds of pairwise merges of neighbouring thread groups. A group's
//    list is contiguous from its first thread's slot 0. One thread per merge walks from the
//    junction, pooling the left list's last block and the right list's first block and then
//    whichever neighbour violates, as long as one does (pooling adjacent violators is valid in
//    any order, so the result is PAVA's); the pooled block overwrites the leftmost entry it
//    absorbed. The right list's surviving entries then move down to follow (move_entry, by the
//    group's threads), so that the merged list is contiguous again.
// 4. Then either expand (the segment is a whole row: every element takes its block's value) or
//    a copy of the tile's list to global memory (a tile of a long row).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tiso {

// Where the surviving entries of a merge's right list move.
struct GroupMove {
  int src, dst, cnt;  // entries [src, src + cnt) go to [dst, dst + cnt), dst <= src
};

// Ragged rows (kVar): per segment, where its row starts in the packed array and its length.
template <int THREADS, bool kVar>
struct VarGeom {};
template <int THREADS>
struct VarGeom<THREADS, true> {
  int64_t ofs[THREADS];
  int32_t len[THREADS];
};

template <typename S, bool kW, int K, int THREADS, bool kVar = false>
struct TileSmem {
  static_assert(K >= 1 && K <= 32 && (K & (K - 1)) == 0, "K: a power of two up to 32");
  static_assert(THREADS % 32 == 0, "THREADS: whole warps");
  static constexpr int kSlots = THREADS * (K + 1) + 1;
  // weights: the sum type when weighted; else a block's weight is its element count
  using WT = std::conditional_t<kW, S, uint16_t>;
  S slot_t[kSlots];          // y, then the stacks' and lists' T, then the output values
  WT slot_w[kSlots];         // w (weighted), then W
  uint16_t st[kSlots];       // first element (in the segment) of each entry
  S seg_y0[THREADS];         // per segment: the offset y0
  int32_t segnan[THREADS];   // per segment: a NaN was read
  uint16_t len[THREADS];     // entries of the list of the group that starts at this thread
  uint8_t cnt[THREADS];      // valid elements of the thread (0..K)
  uint32_t starts[THREADS];  // after the expand: bit j, a block starts at the thread's element j
  GroupMove mv[THREADS / 64 + 1];  // merges of groups wider than a warp
  VarGeom<THREADS, kVar> vg;       // ragged rows only
};

// Slot of thread u's element (or stack entry) j; j = -1 is the spare slot below it.
TISO_HD int tslot(int u, int j, int K) { return u * (K + 1) + 1 + j; }

// The same layout without the leading spare slot (the backward and the long-row expand).
TISO_HD int slot_of(int u, int j, int K) { return u * (K + 1) + j; }

template <typename S, bool kW, typename Sm>
TISO_HD S entry_w(const Sm& s, int i) {
  if constexpr (kW) {
    return s.slot_w[i];
  } else {
    return count_as<S>(static_cast<int>(s.slot_w[i]));
  }
}

template <typename S, bool kW, typename Sm>
TISO_HD void put_entry(Sm& s, int i, S t, S w, int first) {
  s.slot_t[i] = t;
  if constexpr (kW) {
    s.slot_w[i] = w;
  } else {
    s.slot_w[i] = static_cast<uint16_t>(small_int(w));
  }
  s.st[i] = static_cast<uint16_t>(first);
}

// Phase 2 for thread u (u_seg: its index within its segment): PAVA over its cnt[u] elements,
// whose slots hold y (and w). First the slots become the values sign * w * (y - y0) (noting a
// NaN y and a weight that is not > 0); then pool adjacent violators as a state machine, the
// current block in registers and the stack's top read every step; both candidates are read and
// the new state picked by selects, so that the threads of a warp take the same steps. Leaves
// the thread's blocks as entries [0, len[u]) of its slots.
template <typename S, bool kW, int K, typename Sm>
TISO_HD void thread_pava(Sm& s, int u, int u_seg, S y0, bool increasing, bool& nan, bool& bad) {
  const int cnt = s.cnt[u];
  const int b = tslot(u, 0, K);
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = 0; j < K; ++j) {
    if (j < cnt) {
      const S yv = s.slot_t[b + j];
      nan |= yv != yv;
      S v = increasing ? yv - y0 : y0 - yv;
      if constexpr (kW) {
        const S x = s.slot_w[b + j];
        bad |= !(x > S(0));
        v *= x;
      }
      s.slot_t[b + j] = v;
    }
  }
  if (cnt == 0) {
    s.len[u] = 0;
    return;
  }
  // the sentinel: -inf never pools with anything (NaN included), nor does W = 0
  s.slot_t[b - 1] = static_cast<S>(neg_inf());
  if constexpr (kW) {
    s.slot_w[b - 1] = S(0);
  } else {
    s.slot_w[b - 1] = 0;
  }
  const int f0 = u_seg * K;
  S ct = s.slot_t[b];
  S cw = S(1);
  if constexpr (kW) cw = s.slot_w[b];
  int cf = f0, top = -1, j = 1;
  for (;;) {
    const S pt = s.slot_t[b + top];
    const S pw = entry_w<S, kW>(s, b + top);
    const int pf = s.st[b + top];
    // a negative weight (flagged; the fit is refused) would pool with the sentinel
    const bool merge = (!kW || top >= 0) && pool_nb(pt, pw, ct, cw);
    if (!merge && j >= cnt) break;
    const int jj = j < cnt ? j : cnt - 1;
    const S v = s.slot_t[b + jj];
    S x = S(1);
    if constexpr (kW) x = s.slot_w[b + jj];
    if (!merge) put_entry<S, kW>(s, b + top + 1, ct, cw, cf);
    ct = merge ? pt + ct : v;
    cw = merge ? pw + cw : x;
    cf = merge ? pf : f0 + jj;
    top += merge ? -1 : 1;
    j += merge ? 0 : 1;
  }
  put_entry<S, kW>(s, b + top + 1, ct, cw, cf);
  s.len[u] = static_cast<uint16_t>(top + 2);
}

// Phase 3, one merge: the lists of the groups of `half` threads starting at threads g0 and
// g0 + half (both contiguous from their first thread's slot 0). Run by one thread. Walks from
// the junction and writes the pooled block; returns where the right list's surviving entries
// are to move (move_entry does it) and sets the merged group's length.

template <typename S, bool kW, int K, typename Sm>
TISO_HD GroupMove merge_groups(Sm& s, int g0, int half) {
  const int l0 = tslot(g0, 0, K), r0 = tslot(g0 + half, 0, K);
  const int nl = s.len[g0], nr = s.len[g0 + half];
  int p = l0 + nl - 1;  // the last entry of the left list kept as it is
  int q = r0;           // the first entry of the right list kept as it is
  if (nl > 0 && nr > 0) {
    const S at = s.slot_t[p], aw = entry_w<S, kW>(s, p);
    const S bt = s.slot_t[q], bw = entry_w<S, kW>(s, q);
    if (pool_nb(at, aw, bt, bw)) {
      S ct = at + bt, cw = aw + bw;
      --p;
      ++q;
      const int r1 = r0 + nr;
      for (;;) {
        if (p >= l0) {
          const S pt = s.slot_t[p], pw = entry_w<S, kW>(s, p);
          if (pool_nb(pt, pw, ct, cw)) {
            ct += pt;
            cw += pw;
            --p;
            continue;
          }
        }
        if (q < r1) {
          const S nt = s.slot_t[q], nw = entry_w<S, kW>(s, q);
          if (pool_nb(ct, cw, nt, nw)) {
            ct += nt;
            cw += nw;
            ++q;
            continue;
          }
        }
        break;
      }
      // the pooled block replaces the leftmost entry it absorbed (keeping its first element)
      ++p;
      put_entry<S, kW>(s, p, ct, cw, s.st[p]);
    }
  }
  GroupMove m{q, p + 1, r0 + nr - q};
  s.len[g0] = static_cast<uint16_t>(p + 1 - l0 + m.cnt);
  return m;
}

template <typename S, bool kW, typename Sm>
TISO_HD void move_entry(Sm& s, int from, int to) {
  s.slot_t[to] = s.slot_t[from];
  s.slot_w[to] = s.slot_w[from];
  s.st[to] = s.st[from];
}

// Phase 4 (whole rows), per list entry i of the segment whose list starts at slot `base`: the
// block's value, written at its first element's slot, and its start bit. Entries are taken
// from the last down (in groups that read before any writes): a block's first element sits at
// or after its entry's slot, so no entry still to be read is overwritten.
template <int K, typename Sm>
TISO_HD int first_slot(const Sm&, int seg_thread0, int first) {
  return tslot(seg_thread0 + first / K, first % K, K);
}

// Phase 4 (whole rows), thread u after the scatter: every element's value in its slot, spread
// from each block start, `carry` below the first one.
template <typename S, int K, typename Sm>
TISO_HD void spread_values(Sm& s, int u, S carry) {
  const int cnt = s.cnt[u];
  const int b = tslot(u, 0, K);
  const uint32_t starts = s.starts[u];
  S cur = carry;
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = 0; j < K; ++j) {
    if (j < cnt) {
      if ((starts >> j) & 1u) cur = s.slot_t[b + j];
      s.slot_t[b + j] = cur;
    }
  }
}

}  // namespace tiso
