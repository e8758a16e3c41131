// The forward fit inside one CTA: the phases of the tile kernel, written once for the device and
// for the CPU emulator (tests/emu), which runs each phase for every thread in turn.
//
// A CTA of THREADS threads holds THREADS / G row segments ("segments") of up to G * K elements:
// whole rows when a row fits (n <= G K), else one tile of a long row (G = THREADS). Thread u of
// the CTA owns elements [(u % G) K, (u % G) K + K) of segment u / G.
//
// 1. Staging: the CTA's elements are read coalesced into shared memory, y and w in the sum type
//    S, thread u's element j at slot u (K + 1) + j (one pad slot per thread: a warp reading
//    slot j of its 32 threads hits distinct banks).
// 2. thread_pava: each thread runs pool adjacent violators over its K elements, fitting
//    sign * w * (y - y0), y0 the row's first element. The offset leaves every pooling decision
//    unchanged and keeps the sums small, so that float32 data summed in double stay exact where
//    the data vary little around a large value. The thread's stack of blocks (weighted sum T,
//    weight W, first element) lives in its own slots: entry k is written only once element k
//    has been read. The loop is a state machine - each step either pools the top two blocks or
//    pushes the next element - so that the threads of a warp stay in step.
// 3. merge_lists: log2(G) rounds of pairwise merges of neighbouring thread groups. Each group is
//    a list of blocks: the concatenation of its threads' alive entries [lo, hi). One thread per
//    merge walks from the junction, pooling the left list's last block and the right list's
//    first block and then whichever neighbour violates, as long as one does (pooling adjacent
//    violators is valid in any order, so the result is PAVA's). The pooled block overwrites the
//    leftmost entry it absorbed; the others drop out of the alive ranges. Nothing is copied, and
//    every alive entry's first element stays within its owner thread's elements.
// 4. Then either expand (the segment is a whole row: every element takes its block's value) or
//    compaction of the alive blocks to a list in global memory (a tile of a long row).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tiso {

template <typename S, bool kW, int K, int THREADS>
struct TileSmem {
  static_assert(K >= 1 && K <= 32 && (K & (K - 1)) == 0, "K: a power of two up to 32");
  static_assert(THREADS % 32 == 0, "THREADS: whole warps");
  static constexpr int kSlots = THREADS * (K + 1);
  // weights: the sum type when weighted; else a block's weight is its element count
  using WT = std::conditional_t<kW, S, uint16_t>;
  S slot_t[kSlots];          // y, then the stack's T, then the output values
  WT slot_w[kSlots];         // w (weighted), then the stack's W
  uint8_t st[kSlots];        // first element (within the thread) of each stack entry
  S seg_y0[THREADS];         // per segment: the offset y0
  uint32_t nz[THREADS / 32]; // bit u: thread u has an alive entry
  int32_t segnan[THREADS];   // per segment: a NaN was read
  uint8_t lo[THREADS];       // alive entries [lo, hi) of each thread's stack
  uint8_t hi[THREADS];
  uint8_t cnt[THREADS];      // valid elements of the thread (0..K)
  uint32_t starts[THREADS];  // after the expand: bit j, a block starts at the thread's element j
  int32_t scan[THREADS / 32 + 1];
};

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
  s.st[i] = static_cast<uint8_t>(first);
}

// Phase 2 for thread u: PAVA over its cnt[u] elements, whose slots hold y (and w). First the
// slots become the values sign * w * (y - y0) (noting a NaN y and a weight that is not > 0);
// then pool adjacent violators as a state machine: each step pools the stack's top entry into
// the current block or pushes the current block and takes the next element. Only the current
// block is held in registers; both candidates are read every step and the new state picked by
// selects, so that the threads of a warp take the same steps. Leaves the thread's blocks as
// stack entries [0, hi) in its slots (entry k is written only once element k has been read).
template <typename S, bool kW, int K, typename Sm>
TISO_HD void thread_pava(Sm& s, int u, S y0, bool increasing, bool& nan, bool& bad) {
  const int cnt = s.cnt[u];
  const int b = slot_of(u, 0, K);
  s.lo[u] = 0;
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
    s.hi[u] = 0;
    return;
  }
  S ct = s.slot_t[b];
  S cw = S(1);
  if constexpr (kW) cw = s.slot_w[b];
  int cf = 0, depth = 0, j = 1;
  for (;;) {
    const int tt = depth > 0 ? depth - 1 : 0;
    const S pt = s.slot_t[b + tt];
    const S pw = entry_w<S, kW>(s, b + tt);
    const int pf = s.st[b + tt];
    const bool merge = depth > 0 && pool_nb(pt, pw, ct, cw);
    if (!merge && j >= cnt) break;
    const int jj = j < cnt ? j : cnt - 1;
    const S v = s.slot_t[b + jj];
    S x = S(1);
    if constexpr (kW) x = s.slot_w[b + jj];
    if (!merge) put_entry<S, kW>(s, b + depth, ct, cw, cf);
    ct = merge ? pt + ct : v;
    cw = merge ? pw + cw : x;
    cf = merge ? pf : jj;
    depth += merge ? -1 : 1;
    j += merge ? 0 : 1;
  }
  put_entry<S, kW>(s, b + depth, ct, cw, cf);
  s.hi[u] = static_cast<uint8_t>(depth + 1);
}

// Bit u of the nz words (threads with an alive entry): last set in [from, to), first set in
// [from, to), or -1.
template <typename Sm>
TISO_HD int last_nz(const Sm& s, int from, int to) {
  while (to > from) {
    const int w = (to - 1) >> 5;
    const int lo = w << 5;
    uint32_t bits = s.nz[w] & bits_below(to - lo);
    if (from > lo) {
      bits &= ~bits_below(from - lo);
    }
    if (bits) {
      return lo + high_bit(bits);
    }
    to = lo;
  }
  return -1;
}

template <typename Sm>
TISO_HD int first_nz(const Sm& s, int from, int to) {
  while (from < to) {
    const int w = from >> 5;
    const int lo = w << 5;
    uint32_t bits = s.nz[w] & ~bits_below(from - lo);
    if (to - lo < 32) {
      bits &= bits_below(to - lo);
    }
    if (bits) {
      return lo + low_bit(bits);
    }
    from = lo + 32;
  }
  return -1;
}

// Clears the nz bits of threads [from, to). Several merges may share a word in the rounds
// within a warp, hence the atomic.
template <typename Sm>
TISO_HD void clear_nz(Sm& s, int from, int to) {
  while (from < to) {
    const int w = from >> 5;
    const int lo = w << 5;
    uint32_t bits = ~bits_below(from - lo);
    if (to - lo < 32) {
      bits &= bits_below(to - lo);
    }
#if defined(__CUDA_ARCH__)
    atomicAnd(&s.nz[w], ~bits);
#else
    s.nz[w] &= ~bits;
#endif
    from = lo + 32;
  }
}

// Phase 3, one merge: the list of threads [a0, a1) with that of [a1, a2). Run by one thread.
template <typename S, bool kW, int K, typename Sm>
TISO_HD void merge_lists(Sm& s, int a0, int a1, int a2) {
  const int ul = last_nz(s, a0, a1), ur = first_nz(s, a1, a2);
  if (ul < 0 || ur < 0) {
    return;
  }
  int lu = ul, li = s.hi[ul] - 1;  // leftmost absorbed entry of the left list: thread, index
  int ru = ur, ri = s.lo[ur];      // rightmost absorbed entry of the right list
  const int ia = slot_of(lu, li, K), ib = slot_of(ru, ri, K);
  S at = s.slot_t[ia], aw = entry_w<S, kW>(s, ia);
  S bt = s.slot_t[ib], bw = entry_w<S, kW>(s, ib);
  if (!pool(at, aw, bt, bw)) {
    return;
  }
  S ct = at + bt, cw = aw + bw;
  for (;;) {
    int pu = lu, pi = li - 1;
    if (pi < s.lo[lu]) {
      pu = last_nz(s, a0, lu);
      pi = pu >= 0 ? s.hi[pu] - 1 : -1;
    }
    if (pu >= 0) {
      const int ip = slot_of(pu, pi, K);
      const S pt = s.slot_t[ip], pw = entry_w<S, kW>(s, ip);
      if (pool(pt, pw, ct, cw)) {
        ct += pt;
        cw += pw;
        lu = pu;
        li = pi;
        continue;
      }
    }
    int nu = ru, ni = ri + 1;
    if (ni >= s.hi[ru]) {
      nu = first_nz(s, ru + 1, a2);
      ni = nu >= 0 ? s.lo[nu] : -1;
    }
    if (nu >= 0) {
      const int in = slot_of(nu, ni, K);
      const S nt = s.slot_t[in], nw = entry_w<S, kW>(s, in);
      if (pool(ct, cw, nt, nw)) {
        ct += nt;
        cw += nw;
        ru = nu;
        ri = ni;
        continue;
      }
    }
    break;
  }
  // the pooled block replaces entry (lu, li); everything after it up to (ru, ri) is gone
  const int ic = slot_of(lu, li, K);
  put_entry<S, kW>(s, ic, ct, cw, s.st[ic]);
  s.hi[lu] = static_cast<uint8_t>(li + 1);
  clear_nz(s, lu + 1, ru);
  s.lo[ru] = static_cast<uint8_t>(ri + 1);
  if (ri + 1 >= s.hi[ru]) {
    clear_nz(s, ru, ru + 1);
  }
}

// ---------------------------------------------------------------------------------------------
// Expand of whole rows, after the last round. A thread emptied by a merge keeps stale lo/hi:
// its nz bit is what counts.

template <typename Sm>
TISO_HD bool has_entries(const Sm& s, int u) {
  return (s.nz[u >> 5] >> (u & 31)) & 1u;
}

// Bit j set: an alive block of thread u starts at its element j.
template <int K, typename Sm>
TISO_HD uint32_t start_mask(const Sm& s, int u) {
  if (!has_entries(s, u)) {
    return 0;
  }
  uint32_t m = 0;
  const int b = slot_of(u, 0, K);
  for (int i = s.lo[u]; i < s.hi[u]; ++i) {
    m |= 1u << s.st[b + i];
  }
  return m;
}

// Step 1, reading other threads' state: the sums of the block reaching into thread u from the
// left (the last alive entry of the nearest thread before it with one). False if thread u's
// first element starts a block of its own (or nothing is found).
template <typename S, bool kW, int K, typename Sm>
TISO_HD bool carry_sums(const Sm& s, int seg_first, int u, S& t, S& w) {
  if (has_entries(s, u) && s.st[slot_of(u, s.lo[u], K)] == 0) {
    return false;
  }
  const int v = last_nz(s, seg_first, u);
  if (v < 0) {
    return false;
  }
  const int i = slot_of(v, s.hi[v] - 1, K);
  t = s.slot_t[i];
  w = entry_w<S, kW>(s, i);
  return true;
}

// Step 2, after a barrier, on thread u's own slots only: every element's output value,
// overwriting its slot, and the thread's block starts (returned). finish(t, w) turns a block's
// sums into its value (of type S). The entries are taken last to first, each value stored at
// its block's first element: that slot is never an entry still to be read (entry k sits at
// slot k, and a block's first element is at or after its entry's index). Then one pass in
// element order spreads the values, the carry below the first block start.
template <typename S, bool kW, int K, typename Sm, typename Finish>
TISO_HD uint32_t thread_values(Sm& s, int u, S carry, Finish finish) {
  const int cnt = s.cnt[u];
  const int b = slot_of(u, 0, K);
  uint32_t starts = 0;
  if (has_entries(s, u)) {
    for (int i = s.hi[u] - 1; i >= s.lo[u]; --i) {
      const S t = s.slot_t[b + i];
      const S w = entry_w<S, kW>(s, b + i);
      const int first = s.st[b + i];
      s.slot_t[b + first] = finish(t, w);
      starts |= 1u << first;
    }
  }
  S cur = carry;
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = 0; j < K; ++j) {
    if (j < cnt) {
      if ((starts >> j) & 1u) {
        cur = s.slot_t[b + j];
      }
      s.slot_t[b + j] = cur;
    }
  }
  return starts;
}

}  // namespace tiso
