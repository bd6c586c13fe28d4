// Tensor-core path: out[m, n] = x[m, k] . W[n, k]^T on the 5th-generation tensor cores (tcgen05 + TMEM), the
// weights unpacked from the 12-bit format in shared memory.  Used for the verify shapes (M > 32) and for the
// decode shapes whose token count makes the register-decode GEMV latency-bound.
//
// Replaces the reference's dense BF16 verify GEMMs (submission.py: ss_gemm S:783<17-123>, q_kernel
// S:979<25-170>, qb_kernel S:4576, ol_projection S:1547<18-106>, projection S:2985), its register-A wgmma
// family for 16-32 tokens (m32w_gemm S:2395) and its cuBLASLt routes (S:2309-2376, out of scope); here the
// weights stay packed in HBM.
//
// Work decomposition (stream-K): a TILE is 128 weight rows (8 row tiles) x BN tokens; an ITEM is one 64-column
// chunk of a tile.  The items, tile-major, are cut into gridDim.x equal contiguous ranges, one per CTA (one CTA
// per SM), so every SM streams the same number of packed bytes whatever the tile count (the fused QKV+gate
// matrix has 112 tiles for 148 SMs).  A CTA walks its range as SEGMENTS (its part of one tile).  A segment that
// covers the whole tile is stored directly; the parts of a split tile are written as FP32 partial tiles to the
// caller's workspace, and the contributor that finishes last (an atomic ticket per tile) adds all parts in CTA
// order -- a fixed order, so the result does not depend on timing -- and stores the tile.  No CTA waits for
// another.  Without a workspace every CTA takes one whole tile.
//
// Warp roles (24 warps):
//   warp 0       producer of the weights: a stage holds KC consecutive items, lanes 0-7 each fill their row
//                tile's KC packed units (contiguous) with one TMA bulk copy, PS stages deep;
//   warp 18      TMA producer of x: one 2-D box (BN rows x 128 bytes, 128-byte swizzle) per item;
//   warp 19      MMA scheduler: waits for an item's decoded-A and x stages (and, at a segment start, for the
//                epilogue to release the accumulator) and hands the item to the issuer on a named barrier;
//   warp 1       allocates TMEM (accumulators, and the decoded-A ring); lane 0 issues tcgen05.mma (M=128, N=BN,
//                K=16) x4 per item and commits the stages back to their producers and finished segments to the
//                epilogue;
//   warps 2-17   decoders in two groups of 8 warps taking alternate items; each warp decodes one row tile (12-bit
//                decode and escape restoration in registers, as in the GEMV) and writes it as the MMA's A operand:
//                into TMEM with tcgen05.st (the instances used; A then never touches shared memory, whose
//                bandwidth otherwise bounds the 256-token tiles), or into the canonical SW128 K-major layout of a
//                shared-memory A stage;
//   warps 20-23  epilogue: warp 20+q reads TMEM lanes 32q..32q+31 (tcgen05.ld 32x32b), stores the tile or its
//                partial and releases the accumulator, while the next segment's MMAs run in the other one.
// All waits are bounded (status word, no trap); TMEM is always released.
#include "common.cuh"
#include "escape.cuh"
#include "tmap.h"

#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

using namespace mbp;

namespace {

constexpr int kGroups = 2;                 // decoder groups working on alternate items
constexpr int kDecWarps = 8 * kGroups;
constexpr int kWProdWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kDec0 = 2;
constexpr int kXWarp = kDec0 + kDecWarps;  // 18
constexpr int kSchedWarp = kXWarp + 1;     // 19
constexpr int kEpi0 = kSchedWarp + 1;      // 20 (a multiple of 4: warp kEpi0 + q owns TMEM lane quadrant q)
constexpr int kThreads = 32 * (kEpi0 + 4);
constexpr int kHandBar = 1;                // named barrier: scheduler -> issuer hand-over (64 threads)
constexpr int kEpiBar = 2;                 // named barrier of the 4 epilogue warps (128 threads)
constexpr int kAStage = 128 * 128;                    // 128 rows x 64 bf16
constexpr int kMaxSmem = 227 * 1024;
constexpr int kMaxParts = 8;               // contributors of one split tile (the host's plan keeps to it)
static_assert(kEpi0 % 4 == 0, "epilogue warp kEpi0 + q must own TMEM lane quadrant q");

struct __align__(64) GemmParams {
  CUtensorMap xmap;  // x [m, k] bf16, box {64 columns, bn rows}, 128-byte swizzle
  const uint8_t* units;
  const uint8_t* bases;
  const int32_t* esc_off;
  const uint32_t* esc;
  void* out;
  float* ws_part;  // [2 * gridDim.x][bn][128] FP32 partial tiles (slot 2c: CTA c's first segment, 2c+1: its last)
  int* ws_cnt;     // [tiles] contributor tickets, zero between calls
  long long U;     // items = tiles * C
  int C, Rout, R8, m, ldo, bn, f32out;
  int vec_out;     // out and ldo allow 4-row vector stores (16-byte aligned base, ldo % 8 == 0)
  int tcols;       // TMEM columns allocated
  int acc_cols;    // columns of one accumulator (>= bn, a multiple of 32)
  unsigned long long wait_ns;  // limit of every bounded wait
};

// Layout of one instance: PS weight stages of KC items each (8 row tiles x KC consecutive packed units, filled
// by one bulk copy of KC units per row tile), AS decoded-A stages (TA: in TMEM, 32 columns each after the
// accumulators; else in shared memory), XS x stages of up to BNMAX tokens, NACC TMEM accumulators (2 lets a
// segment's epilogue overlap the next segment's MMAs).
template <int PS, int KC, int AS, int XS, int BNMAX, bool TA, int NACC>
struct Cfg {
  static constexpr int kPS = PS, kKC = KC, kAS = AS, kXS = XS, kBNMax = BNMAX, kNAcc = NACC;
  static constexpr bool kTA = TA;
  static constexpr int kPackedStage = 8 * KC * MBP_C12_UNIT_BYTES;
  static constexpr int kXStage = BNMAX * 128;
  static constexpr int kPacked = 0;
  static constexpr int kA = kPacked + PS * kPackedStage;  // multiples of 1024 (SW128 atoms)
  static constexpr int kX = kA + (TA ? 0 : AS * kAStage);
  static constexpr int kMask = kX + XS * kXStage;
  static constexpr int kBars = kMask + kDecWarps * kMaskUnitBytes;
  // pfull/pempty[PS], afull/aempty[AS], xfull/xempty[XS], accfull/accempty[2]
  static constexpr int kMisc = kBars + 8 * (2 * PS + 2 * AS + 2 * XS + 4);
  static constexpr int kTotal = kMisc + 16;    // TMEM base, abort word, ticket
  static constexpr int kSmem = kTotal + 1024;  // + alignment slack
  // Stage ownership: decoder group g takes items g (mod kGroups).  A ring whose barriers only one group waits on
  // per use must give every stage to a single group (depth a multiple of kGroups): otherwise a group could wait for
  // use k+1 of a stage while use k, owned by the other group and completed out of order by the TMA engine, is
  // still pending, and mbarrier parity waits, which only tell the current phase from the previous one, would
  // return on the stale phase.  The decoded-A ring is such a ring; every decoder warp waits on and releases every
  // use of a weight stage, so that ring may have any depth.
  static_assert(AS % kGroups == 0, "the decoded-A ring depth must be a multiple of the decoder groups");
  static_assert(kSmem <= kMaxSmem, "shared memory");
};

// Instances (ring depths per token-tile class); pick() chooses one per call.
using CfgS0 = Cfg<3, 4, 2, 4, 32, false, 2>;
using CfgS1 = Cfg<3, 4, 4, 4, 32, true, 2>;
using CfgS2 = Cfg<4, 4, 8, 4, 32, true, 2>;
using CfgM0 = Cfg<2, 4, 2, 4, 128, false, 2>;
using CfgM1 = Cfg<3, 4, 4, 4, 128, true, 2>;
using CfgL0 = Cfg<3, 2, 2, 3, 256, false, 2>;
using CfgL1 = Cfg<2, 4, 4, 3, 256, true, 1>;
using CfgL2 = Cfg<3, 2, 8, 3, 256, true, 1>;

MBP_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MBP_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MBP_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte-swizzled operand: rows of 128 bytes, 8-row atoms of 1024 bytes (SBO), LBO unused (1).
MBP_DEV uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: BF16 x BF16 -> FP32, both K-major, M = 128, N = n.
MBP_DEV uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

MBP_DEV void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// A from TMEM (M=128 lanes = rows, 8 columns per K=16: a column holds two consecutive K elements, low half first).
MBP_DEV void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 16 lanes x 32 columns from the mma.sync A-fragment registers of a decoded unit: in the .16x128b shape thread
// 4g + t holds (lane g, column t) and (lane g + 8, column t) of each 4-column block, and .x8 repeats the block
// along the columns with the next register pair -- A[4q], A[4q+1] (k pairs t of step q) then A[4q+2], A[4q+3]
// (k pairs t + 4) -- so the sixteen registers land as 16 rows x 64 K in order.
MBP_DEV void tc_st_a(uint32_t taddr, const uint32_t (&a)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(a[8]), "r"(a[9]),
      "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

MBP_DEV void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

MBP_DEV void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

MBP_DEV void store_elem(const GemmParams& p, int tok, int row, float f) {
  if (p.f32out)
    reinterpret_cast<float*>(p.out)[(size_t)tok * p.ldo + row] = f;
  else
    reinterpret_cast<uint16_t*>(p.out)[(size_t)tok * p.ldo + row] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Stream-K ranges: CTA c owns items [start(c), start(c + 1)), start(c) = floor(c * U / G); owner(u) is the CTA
// whose range holds item u (the largest c with start(c) <= u).
MBP_DEV long long range_start(long long c, long long U, long long G) { return c * U / G; }
MBP_DEV int range_owner(long long u, long long U, long long G) { return (int)(((u + 1) * G + U - 1) / U - 1); }

// The part of CTA range [u0, u1) inside tile `tile`: chunks [cb, ce) of the tile.
struct Seg {
  int tile, cb, ce;
};
MBP_DEV Seg seg_of(int tile, int u0, int u1, int C) {
  const int t0 = tile * C;
  Seg s;
  s.tile = tile;
  s.cb = u0 > t0 ? u0 - t0 : 0;
  s.ce = u1 < t0 + C ? u1 - t0 : C;
  return s;
}

template <class CF>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(const __grid_constant__ GemmParams p) {
  constexpr int PS = CF::kPS, KC = CF::kKC, AS = CF::kAS, XS = CF::kXS, NACC = CF::kNAcc;
  constexpr int kPackedStage = CF::kPackedStage;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bars = base + CF::kBars;
  const uint32_t pfull = bars, pempty = pfull + 8 * PS;
  const uint32_t afull = pempty + 8 * PS, aempty = afull + 8 * AS;
  const uint32_t xfull = aempty + 8 * AS, xempty = xfull + 8 * XS;
  const uint32_t accfull = xempty + 8 * XS, accempty = accfull + 16;
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sm + CF::kMisc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_word = misc + 1;  // set by the scheduler when a wait gave up
  volatile int* ticket_word = reinterpret_cast<volatile int*>(misc + 2);
  const int C = p.C;
  const long long G = gridDim.x;
  const int u0 = (int)range_start(blockIdx.x, p.U, G), u1 = (int)range_start(blockIdx.x + 1, p.U, G);
  const int nit = u1 - u0;
  const int tile_first = u0 / C, tile_last = (u1 - 1) / C;
  const int nseg = tile_last - tile_first + 1;
  const uint32_t acc_cols = (uint32_t)p.acc_cols;
  const uint32_t a_col0 = NACC * acc_cols;  // TMEM-resident A ring (CF::kTA): AS stages of 32 columns

  // Programmatic dependent launch: the packed weights never depend on the previous kernel of the stream, so the
  // first stages' units are pulled into L2 while it drains; every thread waits for it before touching x or out.
  if (warp == kWProdWarp && lane < 8) {  // the first weight stages' units, one contiguous run per row tile
    const Seg sg = seg_of(tile_first, u0, u1, C);
    const int rt = (sg.tile % p.R8) * 8 + lane, n = min(PS * KC, sg.ce - sg.cb);
    if (rt < p.Rout) prefetch_l2(p.units + ((size_t)rt * C + sg.cb) * MBP_C12_UNIT_BYTES, (uint32_t)n * MBP_C12_UNIT_BYTES);
  }
  grid_dep_wait();
  grid_dep_launch();

  if (tid == 0) {
    for (int i = 0; i < PS; ++i) {
      mbar_init(pfull + 8 * i, 1);
      mbar_init(pempty + 8 * i, kDecWarps * 32);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(afull + 8 * i, 8 * 32);
      mbar_init(aempty + 8 * i, 1);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(xfull + 8 * i, 1);
      mbar_init(xempty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accfull + 8 * i, 1);
      mbar_init(accempty + 8 * i, 4);
    }
    *abort_word = 0u;
    fence_mbar_init();
    prefetch_tmap(&p.xmap);
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + CF::kMisc),
                 "r"((uint32_t)p.tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kWProdWarp) {
    // ---------------- weight producer ----------------
    // Stage uses walk the range as groups of up to KC consecutive items of one segment; lanes 0-7 each copy their
    // row tile's KC units (contiguous in the row-tile-major layout) with one bulk copy.  (One 3-D tensor copy of
    // the 8 units of an item per stage measured ~0.45 us per issue on B200, a limit of ~27 GB/s per SM.)
    const uint64_t pol = policy_evict_first();
    int use = 0;
    bool ok = true;
    for (int s = 0; s < nseg && ok; ++s) {
      const Seg sg = seg_of(tile_first + s, u0, u1, C);
      const int rb = sg.tile % p.R8, nr = min(8, p.Rout - rb * 8);
      for (int c0 = sg.cb; c0 < sg.ce; c0 += KC, ++use) {
        const int n = min(KC, sg.ce - c0), ps = use % PS;
        if (use >= PS && !mbar_wait(pempty + 8 * ps, ((use / PS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(pfull + 8 * ps, (uint32_t)(nr * n * MBP_C12_UNIT_BYTES));
        __syncwarp();
        if (lane < nr)
          bulk_g2s_hint(base + CF::kPacked + ps * kPackedStage + lane * KC * MBP_C12_UNIT_BYTES,
                        p.units + ((size_t)(rb * 8 + lane) * C + c0) * MBP_C12_UNIT_BYTES,
                        (uint32_t)n * MBP_C12_UNIT_BYTES, pfull + 8 * ps, pol);
      }
    }
    __syncwarp();
  } else if (warp == kXWarp) {
    // ---------------- x producer ----------------
    if (lane == 0) {
      for (int j = 0; j < nit; ++j) {
        const int u = u0 + j;
        const int tile = u / C, chunk = u - tile * C;
        const int xs = j % XS;
        if (j >= XS && !mbar_wait(xempty + 8 * xs, ((j / XS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) break;
        mbar_arrive_expect_tx(xfull + 8 * xs, (uint32_t)p.bn * 128);
        tma_load_2d(base + CF::kX + xs * CF::kXStage, &p.xmap, chunk * 64, (tile / p.R8) * p.bn, xfull + 8 * xs);
      }
    }
    __syncwarp();
  } else if (warp == kSchedWarp) {
    // ---------------- MMA scheduler ----------------
    // Waits for item j's A and x stages (and, when j starts segment s >= NACC, for the epilogue to have released
    // segment s-NACC's accumulator) while the issuer is still feeding item j-1 to the tensor pipe, then meets it on a
    // named barrier.  Every round is always met, so a timed-out wait ends both warps' loops through the abort word
    // instead of a missing partner.
    bool ok = true;
    int s = 0;
    int seg_end = (tile_first + 1) * C;
    for (int j = 0; j < nit; ++j) {
      const int u = u0 + j;
      if (u == seg_end) {
        ++s;
        seg_end += C;
      }
      if (lane == 0 && ok) {
        if (s >= NACC && u % C == 0)  // segment s reuses accumulator s % NACC: wait for segment s - NACC's epilogue
          ok = mbar_wait(accempty + 8 * (s % NACC), ((s / NACC) - 1) & 1, MBP_DEV_TIMEOUT_MMA, p.wait_ns);
        ok = ok && mbar_wait(afull + 8 * (j % AS), (j / AS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns) &&
             mbar_wait(xfull + 8 * (j % XS), (j / XS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns);
        if (!ok) *abort_word = 1u;
      }
      named_bar_sync(kHandBar, 64);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_bf16(p.bn);
    // descriptors of the first stages; the 14-bit start-address field (bytes >> 4) of a descriptor advances by
    // offset >> 4 without carrying out (shared addresses stay below 256 KB)
    const uint64_t da0 = smem_desc_sw128(base + CF::kA), db0 = smem_desc_sw128(base + CF::kX);
    int s = 0;
    int seg_beg = u0, seg_end = (tile_first + 1) * C;
    for (int j = 0; j < nit; ++j) {
      const int u = u0 + j;
      if (u == seg_end) {
        ++s;
        seg_beg = seg_end;
        seg_end += C;
      }
      named_bar_sync(kHandBar, 64);  // the scheduler saw item j's stages full
      if (lane == 0 && *abort_word == 0u) {
        const int as = j % AS, xs = j % XS;
        tc_fence_after();
        const uint64_t da = da0 + (uint64_t)((as * kAStage) >> 4), db = db0 + (uint64_t)((xs * CF::kXStage) >> 4);
        const uint32_t d = tmem + (uint32_t)(s % NACC) * acc_cols;
        if constexpr (CF::kTA) {
          const uint32_t ta = tmem + a_col0 + (uint32_t)as * 32u;
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma_ts(d, ta + 8 * k, db + 2 * k, idesc, (u != seg_beg || k != 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma(d, da + 2 * k, db + 2 * k, idesc, (u != seg_beg || k != 0) ? 1u : 0u);
        }
        tc_commit(aempty + 8 * as);
        tc_commit(xempty + 8 * xs);
        // the segment's last item: the accumulator is complete once these MMAs are
        if (u + 1 == seg_end || u + 1 == u1) tc_commit(accfull + 8 * (s % NACC));
      }
      __syncwarp();
    }
  } else if (warp < kXWarp) {
    // ---------------- decoders: group gi takes items gi, gi + kGroups, ... ----------------
    // Row tile d of the 128-row tile.  With A in TMEM a warp may only write its lane quadrant (warp % 4), so row tile
    // d (lanes 16d .. 16d+15) goes to a warp of quadrant d / 2: the warps of a group cover quadrants 2, 3, 0, 1 twice.
    const int dw = warp - kDec0, gi = dw >> 3, di = dw & 7;
    const int d = CF::kTA ? 2 * ((di + kDec0) & 3) + (di >> 2) : di;
    const uint32_t xr = base + CF::kMask + dw * kMaskUnitBytes;
    mask_clear(xr, kMaskUnitBytes, lane);
    const int g = lane >> 2, t = lane & 3;
    // shared-memory A: destination rows r = 16 d + 8 rh + g inside the 128-row A tile (SW128 K-major)
    uint32_t dst[2][2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int r = 16 * d + 8 * rh + g;
      const uint32_t row = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
      dst[rh][0] = row + ((uint32_t)((2 * t) ^ (r & 7)) << 4);
      dst[rh][1] = row + ((uint32_t)((2 * t + 1) ^ (r & 7)) << 4);
    }
    // Every decoder warp waits on and releases every stage use; in a use of n items starting at item j0, group gi
    // decodes the items j with j % kGroups == gi.
    bool valid = false, ok = true;
    uint32_t T0 = 0, T1 = 0;
    EscCursor cur;
    int use = 0, j0 = 0;
    for (int s = 0; s < nseg && ok; ++s) {
      const Seg sg = seg_of(tile_first + s, u0, u1, C);
      // a new segment: this warp's row tile, its table and its escape slice
      const int rt = (sg.tile % p.R8) * 8 + d;
      valid = rt < p.Rout;
      T0 = T1 = 0;
      if (valid) {
        const uint32_t b = p.bases[rt];
        T0 = table_lo(b);
        T1 = table_hi(b);
        cur.init(p.esc, p.esc_off[(size_t)rt * C + sg.cb], p.esc_off[(size_t)rt * C + sg.ce], lane);
      } else {
        cur.init(p.esc, 0, 0, lane);
      }
      for (int c0 = sg.cb; c0 < sg.ce && ok; c0 += KC, ++use) {
        const int n = min(KC, sg.ce - c0), ps = use % PS;
        if (!mbar_wait(pfull + 8 * ps, (use / PS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns)) {
          ok = false;
          break;
        }
        uint32_t dep = 0;
        for (int jj = (gi - j0 % kGroups + kGroups) % kGroups; jj < n; jj += kGroups) {
          const int j = j0 + jj, as = j % AS;
          const unsigned char* un =
              sm + CF::kPacked + ps * kPackedStage + (d * KC + jj) * MBP_C12_UNIT_BYTES + lane * 16;
          const uint4 p0 = *reinterpret_cast<const uint4*>(un);
          const uint4 p1 = *reinterpret_cast<const uint4*>(un + 512);
          const uint4 p2 = *reinterpret_cast<const uint4*>(un + 1024);
          uint32_t A[16];
          const uint32_t c = (uint32_t)(c0 + jj);
          if (valid) cur.seek(c, lane);
          if (valid && cur.next_chunk == c) {
            uint32_t tgt[1] = {0u};
            cur.scatter<1>(c, c + 1, xr, kMaskUnitBytes, lane, tgt);
            __syncwarp();
            uint4 m0, m1;
            take_mask(xr, tgt[0], lane, m0, m1);
            decode_unit_m(p0, p1, p2, T0, T1, m0, m1, A);
          } else {
            decode_unit(p0, p1, p2, T0, T1, A);
          }
          dep ^= A[0] ^ A[8];  // A[0] depends on p0 and p2, A[8] on p1
          if (j >= AS && !mbar_wait(aempty + 8 * as, ((j / AS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) {
            ok = false;
            break;
          }
          if constexpr (CF::kTA) {
            tc_st_a(tmem + ((uint32_t)(16 * d) << 16) + a_col0 + (uint32_t)as * 32u, A);
            tc_fence_before();  // the stores are complete (wait::st) and ordered before the arrive
          } else {
            unsigned char* a = sm + CF::kA + as * kAStage;
#pragma unroll
            for (int rh = 0; rh < 2; ++rh) {
              *reinterpret_cast<uint4*>(a + dst[rh][0]) = make_uint4(A[0 + rh], A[2 + rh], A[4 + rh], A[6 + rh]);
              *reinterpret_cast<uint4*>(a + dst[rh][1]) = make_uint4(A[8 + rh], A[10 + rh], A[12 + rh], A[14 + rh]);
            }
            fence_async_smem();
          }
          mbar_arrive(afull + 8 * as);
        }
        // this warp's loads from the stage have returned (dep) before the stage goes back to the producer
        mbar_arrive_dep(pempty + 8 * ps, dep);
        j0 += n;
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> the output, or a partial tile ----------------
    const int q = warp & 3, et = tid - 32 * kEpi0;  // TMEM lane quadrant, thread index among the 128
    const int row_l = q * 32 + lane;                 // row inside the 128-row tile
    const int ncol = p.bn / 16;  // 16-column TMEM loads (bn % 16 == 0)
    const size_t slot_elems = (size_t)p.bn * 128;
    for (int s = 0; s < nseg; ++s) {
      const Seg sg = seg_of(tile_first + s, u0, u1, C);
      const int rb = sg.tile % p.R8, tok0 = (sg.tile / p.R8) * p.bn;
      const int row = rb * 128 + row_l;
      const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(s % NACC) * acc_cols;
      bool ok = mbar_wait(accfull + 8 * (s % NACC), (s / NACC) & 1, MBP_DEV_TIMEOUT_MMA, p.wait_ns);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
      tc_fence_after();
      if (sg.cb == 0 && sg.ce == C) {
        // the whole tile: store
        for (int cc = 0; cc < ncol; ++cc) {
          uint32_t v[16];
          if (ok) tc_ld16(acc + (uint32_t)(cc * 16), v);
          if (ok && row < p.Rout * 16) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int tok = tok0 + cc * 16 + jj;
              if (tok < p.m) store_elem(p, tok, row, __uint_as_float(v[jj]));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accempty + 8 * (s % NACC));
        continue;
      }
      // part of a split tile: the FP32 partial to this CTA's slot (column-major: element (r, col) at col*128 + r)
      float* mine = p.ws_part + (size_t)(2 * blockIdx.x + (s == 0 ? 0 : 1)) * slot_elems;
      for (int cc = 0; cc < ncol; ++cc) {
        uint32_t v[16];
        if (ok) tc_ld16(acc + (uint32_t)(cc * 16), v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
          __stcg(mine + (size_t)(cc * 16 + jj) * 128 + row_l, ok ? __uint_as_float(v[jj]) : 0.f);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty + 8 * (s % NACC));  // a later segment may reuse this accumulator
      // ticket: the contributor that arrives last adds every part, in CTA order
      __threadfence();
      named_bar_sync(kEpiBar, 128);
      const long long t0 = (long long)sg.tile * C;
      const int c_lo = range_owner(t0, p.U, G), c_hi = range_owner(t0 + C - 1, p.U, G);  // its contributors
      if (et == 0) *ticket_word = atomicAdd(p.ws_cnt + sg.tile, 1);
      named_bar_sync(kEpiBar, 128);
      if (*ticket_word == c_hi - c_lo) {
        __threadfence();
        // float4 f = rows 4*(f % 32) .. +3 of column f / 32: a warp reads one column's 128 rows per step.  The
        // contributors are CTAs c_lo..c_hi; the tile is the first segment of each of them but c_lo, whose range may
        // start in an earlier tile (then the tile is its last segment).  Loads of two contributors for two
        // float4s are issued together (L2-resident partials), then added in CTA order.
        const int ncols = min(p.bn, p.m - tok0), nf = ncols * 32;
        const int lo_which = range_start(c_lo, p.U, G) >= t0 ? 0 : 1;
        const float* part0 = p.ws_part + (size_t)(2 * c_lo + lo_which) * slot_elems;  // c_lo's slot
        const float* part1 = p.ws_part + (size_t)(2 * (c_lo + 1)) * slot_elems;       // c_lo + 1 + i: part1 + 2i slots
        for (int f0 = et; f0 < nf; f0 += 2 * 128) {
          float4 sum[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int f = min(f0 + u * 128, nf - 1);
            sum[u] = __ldcg(reinterpret_cast<const float4*>(part0 + (size_t)(f >> 5) * 128 + (f & 31) * 4));
          }
          for (int i0 = 0; i0 < c_hi - c_lo; i0 += 2) {
            float4 v[2][2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int f = min(f0 + u * 128, nf - 1);
#pragma unroll
              for (int i = 0; i < 2; ++i)
                if (i0 + i < c_hi - c_lo)
                  v[u][i] = __ldcg(reinterpret_cast<const float4*>(part1 + (size_t)(2 * (i0 + i)) * slot_elems +
                                                                   (size_t)(f >> 5) * 128 + (f & 31) * 4));
            }
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
              for (int i = 0; i < 2; ++i)
                if (i0 + i < c_hi - c_lo) {
                  sum[u].x += v[u][i].x;
                  sum[u].y += v[u][i].y;
                  sum[u].z += v[u][i].z;
                  sum[u].w += v[u][i].w;
                }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int f = f0 + u * 128;
            if (f >= nf) break;
            const int col = f >> 5, grow = rb * 128 + (f & 31) * 4;
            // Rout * 16 is a multiple of 16: four rows are all in or all out
            if (grow >= p.Rout * 16) continue;
            if (!p.vec_out) {
              store_elem(p, tok0 + col, grow, sum[u].x);
              store_elem(p, tok0 + col, grow + 1, sum[u].y);
              store_elem(p, tok0 + col, grow + 2, sum[u].z);
              store_elem(p, tok0 + col, grow + 3, sum[u].w);
            } else if (p.f32out) {
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)(tok0 + col) * p.ldo + grow) = sum[u];
            } else {
              const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(sum[u].x)) |
                                  (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(sum[u].y)) << 16;
              const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(sum[u].z)) |
                                  (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(sum[u].w)) << 16;
              *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p.out) + (size_t)(tok0 + col) * p.ldo + grow) =
                  make_uint2(lo, hi);
            }
          }
        }
        if (et == 0) p.ws_cnt[sg.tile] = 0;  // ready for the next call (ordered by the kernel boundary)
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)p.tcols)
                 : "memory");
  }
}

using KernelFn = void (*)(GemmParams);

template <class CF>
KernelFn kernel_of() {
  return reinterpret_cast<KernelFn>(&k_gemm<CF>);
}

struct Inst {
  KernelFn fn;
  int smem;
  int nacc, tmem_a;  // accumulators; TMEM columns of the A ring (0: A in shared memory)
};

template <class CF>
Inst inst() {
  return Inst{kernel_of<CF>(), CF::kSmem, CF::kNAcc, CF::kTA ? CF::kAS * 32 : 0};
}

// The instance for a token tile of bn tokens (bn % 16 == 0, <= 256).
// MBP_GEMM_CFG=<i> selects the i-th instance of the class (ring-depth sweeps).
Inst pick(int bn) {
  static const int sel = getenv("MBP_GEMM_CFG") ? atoi(getenv("MBP_GEMM_CFG")) : -1;
  if (bn <= 32) {
    switch (sel) {
      case 0: return inst<CfgS0>();
      case 2: return inst<CfgS2>();
      default: return inst<CfgS1>();
    }
  }
  if (bn <= 128) {
    switch (sel) {
      case 0: return inst<CfgM0>();
      default: return inst<CfgM1>();
    }
  }
  switch (sel) {
    case 0: return inst<CfgL0>();
    case 2: return inst<CfgL2>();
    default: return inst<CfgL1>();
  }
}

std::mutex g_mu;
std::map<std::pair<int, KernelFn>, bool> g_attr_done;

int ensure_attr(KernelFn fn, int smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MBP_ERR_LAUNCH;
  std::lock_guard<std::mutex> lk(g_mu);
  const auto key = std::make_pair(dev, fn);
  if (g_attr_done.count(key)) return MBP_OK;
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return MBP_ERR_SMEM;
  g_attr_done[key] = true;
  return MBP_OK;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// The decomposition of a call: token tile width, tiles, items and the grid.
struct Plan {
  int bn, R8, tiles, G, acc_cols;
  long long U;
};

Plan make_plan(int n_out, int k, int m, int sms, bool streamk) {
  Plan pl;
  pl.bn = m >= 256 ? 256 : ((m + 15) / 16) * 16;
  const int T = (m + pl.bn - 1) / pl.bn;
  pl.R8 = (n_out / 16 + 7) / 8;
  pl.tiles = pl.R8 * T;
  const int C = k / 64;
  pl.U = (long long)pl.tiles * C;
  long long G = pl.tiles;  // whole tiles per CTA
  if (streamk) {
    // One CTA per SM, each with at least C / (parts - 1) items, so that a tile has at most `parts` contributors
    // and the last one's fix-up (it re-reads the others' partial tiles) stays short: FP32 partials of wide token
    // tiles are large, so those get fewer parts.
    static const int parts_env = getenv("MBP_GEMM_PARTS") ? atoi(getenv("MBP_GEMM_PARTS")) : 0;
    const int parts = parts_env >= 2 && parts_env <= kMaxParts ? parts_env : pl.bn <= 64 ? 8 : 4;
    const long long min_items = (C + parts - 2) / (parts - 1);
    G = pl.U / min_items;
    if (G > sms) G = sms;
    if (G < 1) G = 1;
  }
  pl.G = (int)G;
  pl.acc_cols = pl.bn <= 32 ? 32 : ((pl.bn + 31) / 32) * 32;  // accumulator columns
  return pl;
}

// Workspace of a stream-K plan: a fixed region of tickets (one int per tile) that every shape places at the same
// offset -- a workspace shared by calls of different shapes must never see one call's partial tiles land on
// another call's tickets -- then two partial-tile slots per CTA.
constexpr int kMaxTickets = 16384;
constexpr size_t kTicketBytes = (size_t)kMaxTickets * 4;

size_t ws_bytes_for(const Plan& pl) {
  if (pl.G == pl.tiles) return 0;  // every CTA takes exactly one whole tile
  return kTicketBytes + (size_t)2 * pl.G * pl.bn * 128 * 4;
}

int gemm_launch(const mbp_c12* w, const uint16_t* x, int m, int n_out, void* out, int ldo, bool f32, void* ws,
                size_t ws_bytes, cudaStream_t stream) {
  if (!w || !w->units || !w->bases || !w->esc_off || !x || !out) return MBP_ERR_ARG;
  if (w->n_esc > 0 && !w->esc) return MBP_ERR_ARG;
  if (w->n % 16 || w->k % 64 || w->k / 64 > 32766 || n_out > w->n || n_out <= 0 || n_out % 16) return MBP_ERR_SHAPE;
  if (m < 1) return MBP_ERR_M;
  if (ldo < n_out) return MBP_ERR_SHAPE;
  if (((uintptr_t)x & 15u) || ((uintptr_t)w->units & 15u) || ((uintptr_t)ws & 255u)) return MBP_ERR_ALIGN;
  const int sms = sm_count();
  static const bool no_split = getenv("MBP_GEMM_PARTS") && atoi(getenv("MBP_GEMM_PARTS")) == 1;
  Plan pl = make_plan(n_out, w->k, m, sms, !no_split);
  if (pl.U > 0x7fffffffLL / 2) return MBP_ERR_SHAPE;  // items are indexed with 32-bit integers
  // no (or a too small) workspace, or more tiles than tickets: whole tiles per CTA
  if (!ws || ws_bytes < ws_bytes_for(pl) || pl.tiles > kMaxTickets) pl = make_plan(n_out, w->k, m, sms, false);
  const Inst in = pick(pl.bn);
  int tcols = 32;  // TMEM: the accumulators, then the A ring of a TMEM-resident instance
  while (tcols < in.nacc * pl.acc_cols + in.tmem_a) tcols *= 2;
  if (tcols > 512) return MBP_ERR_SMEM;
  int rc = ensure_attr(in.fn, in.smem);
  if (rc) return rc;
  GemmParams p;
  const int C = w->k / 64;
  if (!encode_bf16_2d_cached(&p.xmap, x, (uint64_t)m, (uint64_t)w->k, (uint64_t)w->k, (uint32_t)pl.bn, 64u,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return MBP_ERR_TMAP;
  p.units = w->units;
  p.bases = w->bases;
  p.esc_off = w->esc_off;
  p.esc = w->esc;
  p.out = out;
  const bool split = pl.G != pl.tiles;
  p.ws_cnt = split ? static_cast<int*>(ws) : nullptr;
  p.ws_part = split ? reinterpret_cast<float*>(static_cast<char*>(ws) + kTicketBytes) : nullptr;
  p.U = pl.U;
  p.C = C;
  p.Rout = n_out / 16;
  p.R8 = pl.R8;
  p.m = m;
  p.ldo = ldo;
  p.bn = pl.bn;
  p.f32out = f32 ? 1 : 0;
  p.vec_out = ((uintptr_t)out & 15u) == 0 && ldo % 8 == 0;
  p.tcols = tcols;
  p.acc_cols = pl.acc_cols;
  p.wait_ns = wait_limit_ns();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = in.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  static const bool pdl = getenv("MBP_NO_PDL") == nullptr;  // MBP_NO_PDL set: plain stream serialisation
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, in.fn, p) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

}  // namespace

extern "C" {

size_t mbp_gemm_workspace(int n_out, int k, int m) {
  if (n_out <= 0 || n_out % 16 || k <= 0 || k % 64 || m < 1) return 0;
  return ws_bytes_for(make_plan(n_out, k, m, sm_count(), true));
}

int mbp_gemm_c12(const mbp_c12* w, const uint16_t* x, int m, int n_out, uint16_t* out, int ldo, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream) {
  return gemm_launch(w, x, m, n_out, out, ldo, false, workspace, workspace_bytes, stream);
}

int mbp_gemm_c12_f32(const mbp_c12* w, const uint16_t* x, int m, int n_out, float* out, int ldo, void* workspace,
                     size_t workspace_bytes, cudaStream_t stream) {
  return gemm_launch(w, x, m, n_out, out, ldo, true, workspace, workspace_bytes, stream);
}

}  // extern "C"

int mbp_status_gemm(int* v, int clear) { return read_status_here(v, clear); }
