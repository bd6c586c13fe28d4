// Escape-list cursor shared by the GEMV and the device unpack.
//
// A warp walks the units of one 16-row tile in ascending chunk order.  The tile's escapes for that chunk range
// are a contiguous, chunk-sorted slice of the compressed-sparse list.  The warp keeps a 64-entry window of it
// in two registers per lane (win0 = entries wbase..wbase+31, win1 = the next 32, loaded one window ahead so the
// global load is long finished when it is needed).
//
// Escapes are restored through byte masks, one 1 KB mask per unit laid out like the unit's two low-byte planes:
// byte [v >> 4][lane][v & 15] holds the 7-bit exponent XOR of value v of `lane` (zero for values inside the
// exponent window).  For a group of consecutive chunks (one unrolled consumer pass), every lane holding one of
// their entries stores its byte (positions are unique, so plain stores, lane-parallel, any number of escapes
// per unit); after one __syncwarp each lane loads its two mask words per unit and the decoder XORs them into the
// table-decoded high bytes (decode_unit_m: 8 XOR per unit).  One synchronisation per pass instead of per unit,
// and only lanes that hold an escape touch the masks.  This replaces the reference's capped, sequential
// per-warp list (32 entries, S:46<155-162> sm_patch, S:217 cap) with an unbounded one.
#pragma once
#include "common.cuh"

namespace mbp {

constexpr uint32_t kEscSentinel = 0xFFFFFFFFu;  // chunk field 0x7FFF never matches a real chunk (C <= 32766)
constexpr int kMaskUnitBytes = 1024;            // one unit's XOR bytes: [2 planes][32 lanes][16 values]

// Byte offset of an entry's XOR byte inside its unit mask.
MBP_DEV uint32_t esc_mask_byte(uint32_t e) {
  const uint32_t v = esc_value(e);
  return (v >> 4) * 512u + esc_lane(e) * 16u + (v & 15u);
}

MBP_DEV void sts8(uint32_t addr, uint32_t v) { asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"(v) : "memory"); }

struct EscCursor {
  const uint32_t* esc;
  int ep;      // next unconsumed entry (warp-uniform)
  int eend;    // one past the last entry of the range
  int wbase;   // entry index held by lane 0 of win0
  uint32_t win0, win1;
  uint32_t next_chunk;  // chunk of entry ep (0x7FFF when exhausted)

  MBP_DEV uint32_t load(int i, int lane) const {
    return (i + lane < eend) ? __ldg(esc + i + lane) : kEscSentinel;
  }

  MBP_DEV void init(const uint32_t* e, int begin, int end, int lane) {
    esc = e;
    ep = begin;
    eend = end;
    wbase = begin;
    win0 = load(begin, lane);
    win1 = load(begin + 32, lane);
    next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, 0));
    // The rest of the slice goes to L2 now: a window is loaded only one window (a few units of work) ahead of its
    // use, less than the latency of a cold HBM read while the weights stream.  Only the whole 16-byte blocks
    // inside the slice (a bulk prefetch needs 16-byte alignment), so it never touches memory outside the list.
    const uintptr_t pb = ((uintptr_t)(esc + begin + 64) + 15u) & ~(uintptr_t)15u;
    const uintptr_t pe = (uintptr_t)(esc + end) & ~(uintptr_t)15u;
    if (lane == 0 && end - begin > 64 && pe > pb) prefetch_l2(reinterpret_cast<const void*>(pb), (uint32_t)(pe - pb));
  }

  // Skips the entries of chunks below c (chunks this warp does not process).  Warp-uniform.
  MBP_DEV void seek(uint32_t c, int lane) {
    while (next_chunk < c) {
      const int i = ep - wbase;
      const bool below = lane >= i && esc_chunk(win0) < c;
      ep += __popc(__ballot_sync(0xffffffffu, below));
      if (ep - wbase >= 32) {
        wbase += 32;
        win0 = win1;
        win1 = load(wbase + 32, lane);
      }
      next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, (ep - wbase) & 31));
    }
  }

  // Stores the XOR bytes of every entry with chunk in [cbeg, cend) (cend - cbeg <= NS, cend <= C) into the
  // mask of slot chunk - cbeg at `mask + slot * stride` (masks zero on entry), and ORs into tgt[slot] the lanes
  // that received a byte.  Entries below cbeg must already be consumed.  Warp-uniform.  The caller runs a
  // __syncwarp between this and take_mask.
  template <int NS>
  MBP_DEV void scatter(uint32_t cbeg, uint32_t cend, uint32_t mask, uint32_t stride, int lane,
                       uint32_t (&tgt)[NS]) {
    __syncwarp();  // the previous take_mask re-zeroing (other lanes' regions) is ordered before these stores
    while (true) {
      const int i = ep - wbase;  // 0..31
      const bool m0 = lane >= i && esc_chunk(win0) < cend;
      const bool m1 = esc_chunk(win1) < cend;  // sorted: then every entry of win0 from i on is in range too
      const uint32_t s0 = esc_chunk(win0) - cbeg, s1 = esc_chunk(win1) - cbeg;
      if (m0) sts8(mask + s0 * stride + esc_mask_byte(win0), win0 & 0x7Fu);
      if (m1) sts8(mask + s1 * stride + esc_mask_byte(win1), win1 & 0x7Fu);
      const uint32_t b0 = m0 ? 1u << esc_lane(win0) : 0u, b1 = m1 ? 1u << esc_lane(win1) : 0u;
#pragma unroll
      for (int s = 0; s < NS; ++s)
        tgt[s] |= __reduce_or_sync(0xffffffffu, (s0 == (uint32_t)s ? b0 : 0u) | (s1 == (uint32_t)s ? b1 : 0u));
      ep += __popc(__ballot_sync(0xffffffffu, m0)) + __popc(__ballot_sync(0xffffffffu, m1));
      const int used = ep - wbase;
      if (used >= 64) {  // both windows consumed: refill, and continue if the range goes on
        wbase += 64;
        win0 = load(wbase, lane);
        win1 = load(wbase + 32, lane);
        if (esc_chunk(__shfl_sync(0xffffffffu, win0, 0)) < cend) continue;
      } else if (used >= 32) {
        wbase += 32;
        win0 = win1;
        win1 = load(wbase + 32, lane);
      }
      break;
    }
    next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, (ep - wbase) & 31));
  }
};

// Loads (and re-zeroes) this lane's two mask words of a unit mask when the lane was targeted.
MBP_DEV void take_mask(uint32_t mask, uint32_t tgt, int lane, uint4& m0, uint4& m1) {
  if ((tgt >> lane) & 1u) {
    const uint32_t a = mask + (uint32_t)lane * 16u;
    m0 = lds128(a);
    m1 = lds128(a + 512);
    sts128(a, make_uint4(0, 0, 0, 0));
    sts128(a + 512, make_uint4(0, 0, 0, 0));
  } else {
    m0 = make_uint4(0, 0, 0, 0);
    m1 = make_uint4(0, 0, 0, 0);
  }
}

// Zeroes `bytes` (multiple of 512) of masks starting at `mask`, one warp.
MBP_DEV void mask_clear(uint32_t mask, int bytes, int lane) {
  for (int o = lane * 16; o < bytes; o += 512) sts128(mask + o, make_uint4(0, 0, 0, 0));
  __syncwarp();
}

}  // namespace mbp
