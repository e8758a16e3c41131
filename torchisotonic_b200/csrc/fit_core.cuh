// The forward fit inside one CTA: the phases of the tile kernel, written once for the device and
// for the CPU emulator (tests/emu), which runs each phase for every thread in turn.
//
// A CTA of THREADS threads holds THREADS / G row segments ("segments") of up to G * K elements:
// whole rows when a row fits (n <= G K), else one tile of a long row (G = THREADS). Thread u of
// the CTA owns elements [(u % G) K, (u % G) K + K) of segment u / G.
//
// 1. Staging: the CTA's elements are read coalesced into shared memory, as the weighted values
//    w y (negated for a decreasing fit) and weights w in the sum type S, each thread's K
//    elements at u (K + 1) + j (one pad slot per thread: a warp reading element j of its 32
//    threads hits distinct banks).
// 2. thread_pava: each thread runs pool adjacent violators over its K elements, turning its
//    slots into inclusive prefix sums. Its stack of blocks is a bit mask of block starts; the
//    sums of any block are differences of the thread's own prefix sums, so that a block is
//    exact whenever the prefix sums are (float32 input in double: always, but for extreme
//    exponent ranges).
// 3. merge_round: log2(G) rounds of pairwise merges of neighbouring thread groups. Each group
//    is a list of blocks: the concatenation of its threads' alive blocks. One thread per merge
//    walks from the junction, pooling the left list's last block and the right list's first
//    block and then whichever neighbour violates, as long as one does (pooling is valid in any
//    order, so the result is PAVA's). The pooled block is kept in the thread of its leftmost
//    part as an override of that thread's last alive block; the consumed blocks are cleared from
//    the alive masks. Nothing is copied, and every alive block's start stays within its owner
//    thread's elements.
// 4. Then either expand (the segment is a whole row: every element takes its block's mean) or
//    compaction of the alive blocks to a list in global memory (a tile of a long row).
#pragma once

#include "common.cuh"

namespace tiso {

template <typename S, bool kW, int K, int THREADS>
struct TileSmem {
  static_assert(K >= 1 && K <= 32 && (K & (K - 1)) == 0, "K: a power of two up to 32");
  static_assert(THREADS % 32 == 0, "THREADS: whole warps");
  static constexpr int kSlots = THREADS * (K + 1);
  S slot_t[kSlots];            // w y, then prefix sums of it, then the output staging
  S slot_w[kW ? kSlots : 1];   // w, then prefix sums of it
  S ovr_t[THREADS];            // a thread's pooled last block, when ovr is set
  S ovr_w[THREADS];
  uint32_t mask[THREADS];      // block starts of the thread's own PAVA
  uint32_t alive[THREADS];     // those still blocks of the merged lists
  uint32_t nz[THREADS / 32];   // bit u: thread u has an alive block
  uint8_t ovr[THREADS];
  uint8_t cnt[THREADS];        // valid elements of the thread (0..K)
  int32_t segnan[THREADS];     // per segment: a NaN was read
  int32_t scan[THREADS / 32 + 1];
};

TISO_HD int slot_of(int u, int j, int K) { return u * (K + 1) + j; }

// Thread u's prefix sum at element boundary q (0..cnt): the sum of its first q elements.
template <typename Sm, typename S>
TISO_HD S prefix_t(const Sm& s, int u, int q, int K) {
  return q == 0 ? S(0) : s.slot_t[slot_of(u, q - 1, K)];
}

// Sums of thread u's alive block starting at its element p.
template <typename S, bool kW, int K, typename Sm>
TISO_HD void block_sums(const Sm& s, int u, int p, S& t, S& w) {
  const uint32_t al = s.alive[u];
  if (s.ovr[u] && p == high_bit(al)) {
    t = s.ovr_t[u];
    w = s.ovr_w[u];
    return;
  }
  const uint32_t above = s.mask[u] & ~bits_upto(p);
  const int q = above ? low_bit(above) : static_cast<int>(s.cnt[u]);
  const int b = slot_of(u, 0, K);
  t = s.slot_t[b + q - 1] - (p == 0 ? S(0) : s.slot_t[b + p - 1]);
  if (kW) {
    w = s.slot_w[b + q - 1] - (p == 0 ? S(0) : s.slot_w[b + p - 1]);
  } else {
    w = count_as<S>(q - p);
  }
}

// Phase 2 for thread u: PAVA over its cnt[u] elements, whose slots hold y (and w): the values
// fitted are sign * w * y with weights w. Leaves prefix sums of those in its slots and its block
// starts in mask/alive; notes a NaN y and a weight that is not > 0.
template <typename S, bool kW, int K, typename Sm>
TISO_HD void thread_pava(Sm& s, int u, bool increasing, bool& nan, bool& bad) {
  const int cnt = s.cnt[u];
  const int b = slot_of(u, 0, K);
  uint32_t mask = 0;
  S pt = 0, pw = 0;
  S top_t = 0, top_w = 0;
  int top = -1;  // start of the top block; -1: the stack is empty
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = 0; j < K; ++j) {
    if (j < cnt) {
      const S yv = s.slot_t[b + j];
      nan |= yv != yv;
      S v, x;
      if (kW) {
        x = s.slot_w[b + j];
        bad |= !(x > S(0));
        v = x * yv;
        if (!increasing) v = -v;
      } else {
        x = S(1);
        v = increasing ? yv : -yv;
      }
      pt += v;
      s.slot_t[b + j] = pt;
      if (kW) {
        pw += x;
        s.slot_w[b + j] = pw;
      }
      S nt = v, nw = x;
      int ns = j;
      while (top >= 0 && pool(top_t, top_w, nt, nw)) {
        nt += top_t;
        nw += top_w;
        ns = top;
        mask &= ~(1u << top);
        if (mask == 0) {
          top = -1;
          break;
        }
        const int p = high_bit(mask);  // the block below: [p, ns)
        top_t = s.slot_t[b + ns - 1] - (p == 0 ? S(0) : s.slot_t[b + p - 1]);
        if (kW) {
          top_w = s.slot_w[b + ns - 1] - (p == 0 ? S(0) : s.slot_w[b + p - 1]);
        } else {
          top_w = count_as<S>(ns - p);
        }
        top = p;
      }
      mask |= 1u << ns;
      top_t = nt;
      top_w = nw;
      top = ns;
    }
  }
  s.mask[u] = mask;
  s.alive[u] = mask;
  s.ovr[u] = 0;
}

// Bit u of the nz words (threads with an alive block): last set in [from, to), first set in
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
  int lu = ul, lp = high_bit(s.alive[ul]);  // leftmost consumed block of the left list
  int ru = ur, rp = low_bit(s.alive[ur]);   // rightmost consumed block of the right list
  S at, aw, bt, bw;
  block_sums<S, kW, K>(s, lu, lp, at, aw);
  block_sums<S, kW, K>(s, ru, rp, bt, bw);
  if (!pool(at, aw, bt, bw)) {
    return;
  }
  S ct = at + bt, cw = aw + bw;
  for (;;) {
    // the block before the pooled one
    int pu = lu, pp = -1;
    const uint32_t below = s.alive[lu] & bits_below(lp);
    if (below) {
      pp = high_bit(below);
    } else {
      pu = last_nz(s, a0, lu);
      if (pu >= 0) {
        pp = high_bit(s.alive[pu]);
      }
    }
    if (pp >= 0) {
      S pt, pw;
      block_sums<S, kW, K>(s, pu, pp, pt, pw);
      if (pool(pt, pw, ct, cw)) {
        ct += pt;
        cw += pw;
        lu = pu;
        lp = pp;
        continue;
      }
    }
    // the block after it
    int nu = ru, np = -1;
    const uint32_t above = s.alive[ru] & ~bits_upto(rp);
    if (above) {
      np = low_bit(above);
    } else {
      nu = first_nz(s, ru + 1, a2);
      if (nu >= 0) {
        np = low_bit(s.alive[nu]);
      }
    }
    if (np >= 0) {
      S nt, nw;
      block_sums<S, kW, K>(s, nu, np, nt, nw);
      if (pool(ct, cw, nt, nw)) {
        ct += nt;
        cw += nw;
        ru = nu;
        rp = np;
        continue;
      }
    }
    break;
  }
  // The pooled block replaces thread lu's block at lp; everything after it up to (ru, rp) is
  // gone. (ru > lu always: the right list's threads come after the left list's.)
  s.alive[lu] &= bits_upto(lp);
  s.ovr[lu] = 1;
  s.ovr_t[lu] = ct;
  s.ovr_w[lu] = cw;
  clear_nz(s, lu + 1, ru);
  const uint32_t rest = s.alive[ru] & ~bits_upto(rp);
  s.alive[ru] = rest;
  if (!rest) {
    clear_nz(s, ru, ru + 1);
  }
}

// ---------------------------------------------------------------------------------------------
// Expand of whole rows, after the last round. A thread emptied by a merge keeps a stale alive
// mask: its nz bit is what counts.

template <typename Sm>
TISO_HD uint32_t live_mask(const Sm& s, int u) {
  return ((s.nz[u >> 5] >> (u & 31)) & 1u) ? s.alive[u] : 0u;
}

// Step 1, reading other threads' state: the sums of the block reaching into thread u from the
// left (the last alive block of the nearest thread before it with one). False if thread u's
// first element starts a block of its own (or nothing is found).
template <typename S, bool kW, int K, typename Sm>
TISO_HD bool carry_sums(const Sm& s, int seg_first, int u, S& t, S& w) {
  if (live_mask(s, u) & 1u) {
    return false;
  }
  const int v = last_nz(s, seg_first, u);
  if (v < 0) {
    return false;
  }
  block_sums<S, kW, K>(s, v, high_bit(s.alive[v]), t, w);
  return true;
}

// Step 2, after a barrier, on thread u's own slots only: every element's output value,
// overwriting its slot. finish(t, w) turns a block's sums into its value (a value of type S).
// The blocks are taken last to first, each value stored at its last element: the block before
// still finds its prefix sums (at its own last element and before it) untouched. Then one pass
// spreads the values down to the elements, the carry below the first block start.
template <typename S, bool kW, int K, typename Sm, typename Finish>
TISO_HD void thread_values(Sm& s, int u, S carry, Finish finish) {
  const int cnt = s.cnt[u];
  const int b = slot_of(u, 0, K);
  const uint32_t al = live_mask(s, u) & bits_below(cnt);
  uint32_t rest = al;
  int end = cnt;  // one past the last element of the block being done
  while (rest) {
    const int p = high_bit(rest);
    rest &= ~(1u << p);
    S t, w;
    block_sums<S, kW, K>(s, u, p, t, w);
    s.slot_t[b + end - 1] = finish(t, w);
    end = p;
  }
  S cur = carry;
  const int first = al ? low_bit(al) : cnt;
  // downwards: an element is the last of its block if the next one starts a block
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = K - 1; j >= 0; --j) {
    if (j < cnt) {
      if (j >= first) {
        if (j == cnt - 1 || ((al >> (j + 1)) & 1u)) {
          cur = s.slot_t[b + j];
        }
      } else {
        cur = carry;
      }
      s.slot_t[b + j] = cur;
    }
  }
}

}  // namespace tiso
