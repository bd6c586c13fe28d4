// Escape-list cursor shared by the GEMV and the device unpack.
//
// A warp walks the units of one 16-row tile in ascending chunk order.  The tile's escapes for that chunk range
// are a contiguous, chunk-sorted slice of the compressed-sparse list.  The warp keeps a 64-entry window of it
// in two registers per lane (win0 = entries wbase..wbase+31, win1 = the next 32, loaded one window ahead so the
// global load is long finished when it is needed).  For a unit with escapes, every lane holding one of that
// unit's entries XORs it into a per-warp shared-memory mask (lane-parallel, any number of escapes per unit);
// each lane then folds its 16 mask words into its decoded registers.  This replaces the reference's capped,
// sequential per-warp list (32 entries, S:46<155-162> sm_patch, S:217 cap) with an unbounded one.
#pragma once
#include "common.cuh"

namespace mbp {

constexpr uint32_t kEscSentinel = 0xFFFFFFFFu;  // chunk field 0x7FFF never matches a real chunk (C <= 32766)
constexpr int kXorPitch = 80;                   // bytes per lane in the XOR mask: 16 words + pad (conflict-free)
constexpr int kXorWarpBytes = 32 * kXorPitch;

struct EscCursor {
  const uint32_t* esc;
  int ep;      // next unconsumed entry (warp-uniform)
  int eend;    // one past the last entry of the range
  int wbase;   // entry index held by lane 0 of win0
  uint32_t win0, win1;
  uint32_t next_chunk;  // chunk of entry ep (0x7FFF when exhausted)

  MBP_DEV void init(const uint32_t* e, int begin, int end, int lane) {
    esc = e;
    ep = begin;
    eend = end;
    wbase = begin;
    win0 = (begin + lane < end) ? __ldg(e + begin + lane) : kEscSentinel;
    win1 = (begin + 32 + lane < end) ? __ldg(e + begin + 32 + lane) : kEscSentinel;
    next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, 0));
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
        win1 = (wbase + 32 + lane < eend) ? __ldg(esc + wbase + 32 + lane) : kEscSentinel;
      }
      next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, (ep - wbase) & 31));
    }
  }

  // Applies the escapes of chunk c to the decoded registers A. Warp-uniform; `xr` = this warp's mask region.
  MBP_DEV void apply(uint32_t c, uint32_t (&A)[16], uint32_t xr, int lane) {
    if (next_chunk != c) return;
    while (true) {
      const int i = ep - wbase;
      const bool mine = lane >= i && esc_chunk(win0) == c;
      if (mine) {
        const uint32_t addr = xr + esc_lane(win0) * kXorPitch + (esc_value(win0) >> 1) * 4;
        asm volatile("red.shared.xor.b32 [%0], %1;" ::"r"(addr), "r"(esc_xor_word(win0)) : "memory");
      }
      ep += __popc(__ballot_sync(0xffffffffu, mine));
      if (ep - wbase < 32) break;
      wbase += 32;
      win0 = win1;
      win1 = (wbase + 32 + lane < eend) ? __ldg(esc + wbase + 32 + lane) : kEscSentinel;
      if (esc_chunk(__shfl_sync(0xffffffffu, win0, 0)) != c) break;
    }
    next_chunk = esc_chunk(__shfl_sync(0xffffffffu, win0, (ep - wbase) & 31));
    __syncwarp();
    const uint32_t mine_addr = xr + lane * kXorPitch;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = lds128(mine_addr + 16 * j);
      A[4 * j + 0] ^= v.x;
      A[4 * j + 1] ^= v.y;
      A[4 * j + 2] ^= v.z;
      A[4 * j + 3] ^= v.w;
      sts128(mine_addr + 16 * j, make_uint4(0, 0, 0, 0));
    }
    __syncwarp();
  }
};

// Zeroes one warp's mask region (call once before the first apply).
MBP_DEV void xor_mask_clear(uint32_t xr, int lane) {
  for (int j = 0; j < kXorPitch / 16; ++j) sts128(xr + lane * kXorPitch + 16 * j, make_uint4(0, 0, 0, 0));
  __syncwarp();
}

}  // namespace mbp
