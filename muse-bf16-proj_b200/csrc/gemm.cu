// Verify-path GEMM for larger token counts (M > 32): out[m, n] = x[m, k] . W[n, k]^T on the 5th-generation
// tensor cores (tcgen05 + TMEM), weights decoded from the 12-bit format in registers and written into TMEM.
// The same kernel runs the FP32 router above 256 tokens (hi/lo units, k_gemm<true>) and, for tensor-parallel
// calls, can store its results as epoch-tagged words into the ranks' exchange buffers (peer pointers) instead of
// `out` (mbp_gemm_c12_multi).
//
// Replaces the reference's dense BF16 verify GEMMs (submission.py: ss_gemm S:783<17-123>, q_kernel
// S:979<25-170>, qb_kernel S:4576, ol_projection S:1547<18-106>, projection S:2985) and its cuBLASLt routes
// (S:2309-2376, out of scope), which read unpacked BF16 weights; here the weights stay packed in HBM.
//
// CTA tile: 128 weight rows (8 row tiles) x BN tokens (<= 256) x a K range; `split` CTAs of a cluster share
// one tile's K range and reduce through distributed shared memory.  The K range advances in stages of two
// 64-column sub-tiles: two consecutive chunks of the 12-bit weights, or one chunk's hi and lo tiles of the FP32
// router (both multiplied by the same x tile into the same accumulator).  Warp roles:
//   warp 0       TMA producer of the weights: per stage one 3-D box of 8 row tiles x 2 sub-tiles;
//   warp 18      TMA producer of x: per stage the stage's x tiles (BN rows x 128 bytes each, 128-byte swizzle);
//                the two rings run independently, so an x stage is refilled as soon as its MMAs are done;
//   warp 19      MMA scheduler: waits for each stage's A and x and hands the stage to the issuer on a named
//                barrier, so the issuing thread never polls an mbarrier behind its own MMAs;
//   warp 1       allocates TMEM (the accumulator, then the decoded-A ring); lane 0 issues tcgen05.mma (M=128,
//                N=BN, K=16, BF16 -> FP32) x8 per stage, A from TMEM and B = x from a K-major SW128 shared-memory
//                descriptor; tcgen05.commit frees the A and x stages and finally signals the accumulator.  Two
//                sub-tiles per stage halve the commits and hand-overs per MMA, the issue gap that bounds the
//                one-chunk stages (the tensor pipe drained while they ran);
//   warps 2-17   decoders, one per (row tile, sub-tile) of every stage: each decodes its unit in registers (same
//                decode and escape cursor as the GEMV; the hi/lo units are copied as they are), transposes its K
//                pairs across its lane quads and writes the tile with tcgen05.st straight into TMEM as the
//                MMA's A operand: the decoded weights never pass through shared memory, whose bandwidth (TMA
//                writes and the MMA's operand reads) otherwise bounds the 256-token tiles.  Afterwards they read
//                the accumulator (tcgen05.ld 32x32b) and store (or cluster-reduce) it.
// All waits are bounded; TMEM is always released.
#include "common.cuh"
#include "escape.cuh"
#include "tmap.h"

#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

using namespace mbp;

namespace {

constexpr int kDecWarps = 16;              // 8 row tiles x 2 sub-tiles per stage
constexpr int kXWarp = 2 + kDecWarps;      // the x producer
constexpr int kSchedWarp = 3 + kDecWarps;  // waits for each stage's operands on behalf of the MMA issuer
constexpr int kThreads = 32 * (4 + kDecWarps);
constexpr int kHandBar = 1;                // named barrier of the scheduler -> issuer hand-over (64 threads)
constexpr int kAS = 2;                     // decoded-A ring depth (stages of 64 TMEM columns)
constexpr int kXS = 2;                     // x ring depth (stages)
constexpr int kMaxSmem = 227 * 1024;
constexpr int kRouterTcMaxChunks = 32;     // most 64-column chunks one CTA accumulates in the FP32 router

// The two weight formats.  A row tile's sub-tile is one 12-bit unit (1.5 KB, decoded in registers; a stage holds
// two consecutive chunks, each with its own x tile) or, for the FP32 router, one BF16 hi or lo unit (2 KB,
// copied as it is: the packer already writes it in the decoder's register layout; a stage is one chunk).
template <bool HILO>
struct WFmt;
template <>
struct WFmt<false> {
  static constexpr int kSub = MBP_C12_UNIT_BYTES;  // bytes of one row tile's sub-tile
  static constexpr int kPS = 3;                    // packed ring depth (stages)
  static constexpr int kXTiles = 2;                // x tiles per stage
};
template <>
struct WFmt<true> {
  static constexpr int kSub = MBP_RAW_UNIT_BYTES;
  static constexpr int kPS = 4;
  static constexpr int kXTiles = 1;
};

struct __align__(64) GemmParams {
  CUtensorMap wmap;  // units as [R][C][192 x u64], box {192, 2, 8}; hi/lo units as [R][2C][256 x u64], box {256, 2, 8}
  CUtensorMap xmap;  // x [m, k] bf16, box {64 columns, BN rows}, 128-byte swizzle
  const uint8_t* units;
  const uint8_t* bases;
  const int32_t* esc_off;
  const uint32_t* esc;
  void* out;
  int C, Rout, m, ldo, bn, split;
  int f32out;
  int wsubs;                   // sub-tiles per weight box: 2 (1 for a 12-bit matrix of a single chunk)
  int nblk;                    // row blocks: block b owns row tiles [b*Rout/nblk, (b+1)*Rout/nblk), at most 8
  // Tensor-parallel column gather (nout > 0): instead of `out`, every result pair (rows 16*tile + g and + 8) goes
  // as one epoch-tagged bf16x2 word (tok, 8*tile + g) into each of the nout exchange buffers (ldo in words; the
  // buffer half of the epoch's parity), epoch = *epoch + 1; the layout mbp_gemv_c12_multi's MBP_OUT_TAGGED_BF16X2
  // writes and mbp_tp_finish's MBP_TP_GATHER_BF16 reads.
  // With tag_f32 set (row-parallel sum), every result goes as its own tagged f32 word (tok, row) instead.
  void* touts[8];
  int nout;
  int tag_f32;
  const int* epoch;
  long long parity_stride;
  unsigned long long wait_ns;  // limit of every bounded wait
};

struct GLayout {
  int packed, a, x, xr, bars, tmem_slot, total;
};

__host__ __device__ inline GLayout gemm_layout(int bn, bool hilo) {
  const int ps = hilo ? WFmt<true>::kPS : WFmt<false>::kPS;
  const int stage = 16 * (hilo ? WFmt<true>::kSub : WFmt<false>::kSub);
  const int xt = hilo ? WFmt<true>::kXTiles : WFmt<false>::kXTiles;
  GLayout L;
  L.packed = 0;
  L.a = L.packed + ps * stage;  // (no shared-memory A: the decoded tiles live in TMEM)
  L.x = L.a;                    // multiple of 1024
  L.xr = L.x + kXS * xt * bn * 128;  // bn multiple of 16 -> multiple of 2048
  L.bars = L.xr + kDecWarps * kMaskUnitBytes;
  L.tmem_slot = L.bars + 8 * (2 * ps + 2 * kAS + 2 * kXS + 1);
  L.total = L.tmem_slot + 16;
  return L;
}

MBP_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

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

// A from TMEM (M=128 lanes = rows, 8 columns per K=16: a column holds two consecutive K elements, low half first).
MBP_DEV void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 4 x 4 transpose across the 4 lanes of a quad (t = lane & 3): afterwards lane t holds, at index a, what lane a
// held at index t.  Two butterfly stages (partners t ^ 2, then t ^ 1), each exchanging the two elements whose
// index differs from t in that stage's bit.
MBP_DEV void quad_transpose(uint32_t& m0, uint32_t& m1, uint32_t& m2, uint32_t& m3, int t) {
  const bool b1 = (t & 2) != 0, b0 = (t & 1) != 0;
  uint32_t s0 = b1 ? m0 : m2, s1 = b1 ? m1 : m3;
  s0 = __shfl_xor_sync(0xffffffffu, s0, 2);
  s1 = __shfl_xor_sync(0xffffffffu, s1, 2);
  if (b1) {
    m0 = s0;
    m1 = s1;
  } else {
    m2 = s0;
    m3 = s1;
  }
  s0 = b0 ? m0 : m1;
  s1 = b0 ? m2 : m3;
  s0 = __shfl_xor_sync(0xffffffffu, s0, 1);
  s1 = __shfl_xor_sync(0xffffffffu, s1, 1);
  if (b0) {
    m0 = s0;
    m2 = s1;
  } else {
    m1 = s0;
    m3 = s1;
  }
}

// A decoded unit into TMEM: 16 lanes (rows) x 32 columns (64 K, two bf16 per column, natural K order).
// The decoder leaves lane 4g + t with the K pairs 8t .. 8t+7 of rows g and g + 8 (register 2s + rh = pair 8t + s
// of row g + 8rh: the unit's lane layout).  The .16x128b.x8 store puts register i of lane 4g + t at row
// g + 8 (i % 2), column 4 (i / 2) + t, i.e. lane t must hold the pairs 4c + t, c = 0..7.  Pair 4c + t lives in lane
// c / 2 at s = 4 (c % 2) + t: for each half h = c % 2 and row rh that is a 4 x 4 transpose across the quad.
MBP_DEV void tc_st_a(uint32_t taddr, const uint32_t (&A)[16], int t) {
  uint32_t a[16];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      uint32_t m0 = A[2 * (4 * h + 0) + rh], m1 = A[2 * (4 * h + 1) + rh], m2 = A[2 * (4 * h + 2) + rh],
               m3 = A[2 * (4 * h + 3) + rh];
      quad_transpose(m0, m1, m2, m3, t);  // now m_j = pair 4(2j + h) + t of row rh (column c = 2j + h)
      a[2 * (2 * 0 + h) + rh] = m0;
      a[2 * (2 * 1 + h) + rh] = m1;
      a[2 * (2 * 2 + h) + rh] = m2;
      a[2 * (2 * 3 + h) + rh] = m3;
    }
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

MBP_DEV void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

MBP_DEV uint32_t bf16_pair(float lo, float hi) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(lo)) | (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16;
}

// One tagged exchange word (rows row and row + 8 of a 16-row tile, row % 16 < 8) into every exchange buffer.
MBP_DEV void store_tagged(const GemmParams& p, int tok, int row, float lo, float hi, uint32_t epoch) {
  const uint64_t w = (uint64_t)epoch << 32 | bf16_pair(lo, hi);
  const long long par = (long long)(epoch & 1u) * p.parity_stride;
  const size_t idx = (size_t)tok * p.ldo + (size_t)(row >> 4) * 8 + (row & 7);
  for (int o = 0; o < p.nout; ++o)
    st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(static_cast<char*>(p.touts[o]) + par) + idx, w);
}

// One tagged f32 word (the row-parallel partial sums) into every exchange buffer.
MBP_DEV void store_tagged_f32(const GemmParams& p, int tok, int row, float f, uint32_t epoch) {
  const uint64_t w = (uint64_t)epoch << 32 | __float_as_uint(f);
  const long long par = (long long)(epoch & 1u) * p.parity_stride;
  const size_t idx = (size_t)tok * p.ldo + row;
  for (int o = 0; o < p.nout; ++o)
    st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(static_cast<char*>(p.touts[o]) + par) + idx, w);
}

MBP_DEV void store_elem(const GemmParams& p, int tok, int row, float f) {
  if (p.f32out)
    reinterpret_cast<float*>(p.out)[(size_t)tok * p.ldo + row] = f;
  else
    reinterpret_cast<uint16_t*>(p.out)[(size_t)tok * p.ldo + row] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

template <bool HILO>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(const __grid_constant__ GemmParams p) {
  using W = WFmt<HILO>;
  constexpr int kPS = W::kPS, kSub = W::kSub, kStage = 16 * W::kSub;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const GLayout L = gemm_layout(p.bn, HILO);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bars = base + L.bars;
  const uint32_t pfull = bars, pempty = pfull + 8 * kPS;
  const uint32_t afull = pempty + 8 * kPS, aempty = afull + 8 * kAS;
  const uint32_t xfull = aempty + 8 * kAS, xempty = xfull + 8 * kXS;
  const uint32_t done = xempty + 8 * kXS;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sm + L.tmem_slot);
  volatile uint32_t* abort_word = tmem_slot + 2;  // set by the scheduler when a wait gave up
  const int C = p.C;
  const int rb0 = (int)((long long)blockIdx.x * p.Rout / p.nblk);  // first row tile
  const int rvalid = (int)((long long)(blockIdx.x + 1) * p.Rout / p.nblk) - rb0;  // its row tiles (<= 8)
  const int tok0 = blockIdx.y * p.bn;
  const int ks = blockIdx.z;       // K split index == cluster rank (cluster dims 1 x 1 x split)
  const int cs = (int)((long long)ks * C / p.split), ce = (int)((long long)(ks + 1) * C / p.split);
  const int nc = ce - cs;                        // chunks of this CTA
  const int nst = HILO ? nc : (nc + 1) / 2;      // stages (the last 12-bit stage may hold one chunk)
  const int xbytes = p.bn * 128;                 // one x tile
  // TMEM: the accumulator (acc_cols >= bn columns), then the decoded-A ring (kAS x 64 columns)
  const uint32_t acc_cols = p.bn <= 32 ? 32 : p.bn <= 64 ? 64 : p.bn <= 128 ? 128 : 256;
  uint32_t tmem_cols = 32;
  while (tmem_cols < acc_cols + 64 * kAS) tmem_cols *= 2;
  const uint32_t a_col0 = acc_cols;

  // Programmatic dependent launch: the packed weights never depend on the previous kernel of the stream, so the
  // first ring's units are pulled into L2 while it drains; every thread waits for it before touching x or out.
  if (warp == 0 && lane < 8 * kPS) {
    const int d = lane & 7, i = lane >> 3;
    if (d < rvalid && i < nst) {
      const size_t unit = HILO ? (size_t)(rb0 + d) * C + cs + i : (size_t)(rb0 + d) * C + cs + 2 * i;
      const int subs = HILO ? 2 : (2 * i + 1 < nc ? 2 : 1);  // stays inside this CTA's chunks
      prefetch_l2(p.units + unit * (HILO ? 2 * kSub : kSub), subs * kSub);
    }
  }
  grid_dep_wait();
  grid_dep_launch();

  if (tid == 0) {
    for (int i = 0; i < kPS; ++i) {
      mbar_init(pfull + 8 * i, 1);
      mbar_init(pempty + 8 * i, kDecWarps * 32);
    }
    for (int i = 0; i < kAS; ++i) {
      mbar_init(afull + 8 * i, kDecWarps * 32);
      mbar_init(aempty + 8 * i, 1);
    }
    for (int i = 0; i < kXS; ++i) {
      mbar_init(xfull + 8 * i, 1);
      mbar_init(xempty + 8 * i, 1);
    }
    mbar_init(done, 1);
    *abort_word = 0u;
    fence_mbar_init();
    prefetch_tmap(&p.wmap);
    prefetch_tmap(&p.xmap);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + L.tmem_slot),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- weight producer ----------------
    // One box per stage: 8 row tiles x 2 sub-tiles.  A last 12-bit stage with one chunk still loads two (the
    // second belongs to the next K range, or lies past the matrix and is zero-filled); its MMAs are skipped.
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int ps = i % kPS;
        if (i >= kPS && !mbar_wait(pempty + 8 * ps, ((i / kPS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) break;
        mbar_arrive_expect_tx(pfull + 8 * ps, (uint32_t)(p.wsubs * 8 * kSub));
        tma_load_3d(base + L.packed + ps * kStage, &p.wmap, 0, HILO ? 2 * (cs + i) : cs + 2 * i, rb0,
                    pfull + 8 * ps);
      }
    }
    __syncwarp();  // lanes 1-31 wait here for the producing lane
  } else if (warp == kXWarp) {
    // ---------------- x producer ----------------
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int xs = i % kXS;
        const int nt = HILO ? 1 : min(2, nc - 2 * i);
        if (i >= kXS && !mbar_wait(xempty + 8 * xs, ((i / kXS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) break;
        mbar_arrive_expect_tx(xfull + 8 * xs, (uint32_t)(nt * xbytes));
        for (int t = 0; t < nt; ++t)
          tma_load_2d(base + L.x + (xs * W::kXTiles + t) * xbytes, &p.xmap, (HILO ? cs + i : cs + 2 * i + t) * 64,
                      tok0, xfull + 8 * xs);
      }
    }
    __syncwarp();
  } else if (warp == kSchedWarp) {
    // ---------------- MMA scheduler ----------------
    // Waits for stage i's A and x while the issuer is still feeding stage i-1 to the tensor pipe, then meets it
    // on a named barrier.  (An mbarrier wait in the issuing thread itself, right behind its MMAs and commits,
    // measured ~300-450 cycles per wait even on phases completed long before.)  Every round is always met, so a
    // timed-out wait ends both warps' loops through the abort word instead of a missing partner.
    bool ok = true;
    for (int i = 0; i < nst; ++i) {
      if (lane == 0 && ok) {
        ok = mbar_wait(afull + 8 * (i % kAS), (i / kAS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns) &&
             mbar_wait(xfull + 8 * (i % kXS), (i / kXS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns);
        if (!ok) *abort_word = 1u;
      }
      named_bar_sync(kHandBar, 64);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_bf16(p.bn);
    // descriptors of the first stages; the 14-bit start-address field (bytes >> 4) of a descriptor advances by
    // offset >> 4 without carrying out (shared addresses stay below 256 KB)
    const uint64_t db0 = smem_desc_sw128(base + L.x);
    for (int i = 0; i < nst; ++i) {
      named_bar_sync(kHandBar, 64);  // the scheduler saw stage i's A and x full
      if (lane == 0 && *abort_word == 0u) {
        const int as = i % kAS, xs = i % kXS;
        tc_fence_after();
        const uint32_t ta = tmem + a_col0 + (uint32_t)(as * 64);
        const uint64_t db = db0 + (uint64_t)((xs * W::kXTiles * xbytes) >> 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma_ts(tmem, ta + 8 * k, db + 2 * k, idesc, (i | k) != 0);
        if (HILO || 2 * i + 1 < nc) {
          // second sub-tile: the lo tile against the same x, or the next chunk against its own x tile
          const uint64_t db1 = HILO ? db : db + (uint64_t)(xbytes >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma_ts(tmem, ta + 32 + 8 * k, db1 + 2 * k, idesc, 1u);
        }
        tc_commit(aempty + 8 * as);
        tc_commit(xempty + 8 * xs);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(done);  // fires when every issued MMA has completed
    __syncwarp();
  } else {
    // ---------------- decoders: warp (d, j) = row tile d, sub-tile j of every stage ----------------
    // A warp may only write its TMEM lane quadrant (warp % 4), so row tile d (lanes 16d .. 16d+15) goes to a warp
    // of quadrant d / 2: the four warps of quadrant q take (2q, 0), (2q + 1, 0), (2q, 1), (2q + 1, 1).
    const int dw = warp - 2, q = (dw + 2) & 3, qi = dw >> 2;
    const int d = 2 * q + (qi & 1), j = qi >> 1;
    const int t = lane & 3;
    const uint32_t ta0 = tmem + ((uint32_t)(16 * d) << 16) + a_col0 + 32u * (uint32_t)j;
    const int rt = rb0 + d;
    const bool valid = d < rvalid;  // the box's other rows belong to the next block or lie past the matrix
    uint32_t T0 = 0, T1 = 0;
    EscCursor cur;
    const uint32_t xr = base + L.xr + dw * kMaskUnitBytes;
    if constexpr (!HILO) {
      mask_clear(xr, kMaskUnitBytes, lane);
      if (valid) {
        const uint32_t b = p.bases[rt];
        T0 = table_lo(b);
        T1 = table_hi(b);
        cur.init(p.esc, p.esc_off[(size_t)rt * C + cs], p.esc_off[(size_t)rt * C + ce], lane);
      } else {
        cur.init(p.esc, 0, 0, lane);
      }
    }
    for (int i = 0; i < nst; ++i) {
      const int ps = i % kPS, as = i % kAS;
      // a last 12-bit stage with one chunk has no sub-tile 1; rows outside the block are neither decoded nor stored
      const bool live = valid && (HILO || 2 * i + j < nc);
      if (!mbar_wait(pfull + 8 * ps, (i / kPS) & 1, MBP_DEV_TIMEOUT_FULL, p.wait_ns)) break;
      const unsigned char* u = sm + L.packed + ps * kStage + (p.wsubs * d + j) * kSub + lane * 16;
      uint32_t A[16];
      uint32_t dep = 0;
      if (!live) {
        // nothing to load: the arrive below hands the stage back at once
      } else if constexpr (HILO) {
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const uint4 v = *reinterpret_cast<const uint4*>(u + qq * 512);
          A[4 * qq] = v.x, A[4 * qq + 1] = v.y, A[4 * qq + 2] = v.z, A[4 * qq + 3] = v.w;
        }
        dep = A[0] ^ A[4] ^ A[8] ^ A[12];  // a value from each load
      } else {
        const uint4 p0 = *reinterpret_cast<const uint4*>(u);
        const uint4 p1 = *reinterpret_cast<const uint4*>(u + 512);
        const uint4 p2 = *reinterpret_cast<const uint4*>(u + 1024);
        const uint32_t c = (uint32_t)(cs + 2 * i + j);
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
        dep = A[0] ^ A[8];  // A[0] depends on p0 and p2, A[8] on p1
      }
      // every load of the stage has returned before it is handed back
      mbar_arrive_dep(pempty + 8 * ps, dep);
      if (i >= kAS && !mbar_wait(aempty + 8 * as, ((i / kAS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY, p.wait_ns)) break;
      if (live) tc_st_a(ta0 + (uint32_t)(as * 64), A, t);
      tc_fence_before();  // the stores are complete (wait::st) and ordered before the arrive
      mbar_arrive(afull + 8 * as);
    }
  }

  // ---------------- epilogue: TMEM -> registers -> global (or a cluster reduction) ----------------
  // Decoder warps own TMEM lane quadrant (warp % 4); the kDecWarps/4 warps of a quadrant split the columns.
  const bool epi = warp >= 2 && warp < 2 + kDecWarps;
  const int q = warp & 3, part = (warp - 2) >> 2, nparts = kDecWarps / 4;
  const int ncol = (p.bn + 31) / 32;
  const int row_l = q * 32 + lane;                 // row inside the 128-row tile
  const int row = rb0 * 16 + row_l;                // global output row
  // the exchange epoch (after this grid's dependency wait: the receive kernel after the previous exchange, which
  // advances the counter, has completed)
  const uint32_t epoch = p.nout > 0 ? (uint32_t)__ldcg(p.epoch) + 1u : 0u;
  bool ok = true;
  if (epi) {
    ok = mbar_wait(done, 0, MBP_DEV_TIMEOUT_MMA, p.wait_ns);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
    tc_fence_after();
  }
  if (p.split == 1) {
    if (epi && ok) {
      for (int cc = part; cc < ncol; cc += nparts) {
        uint32_t v[32];
        tc_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc * 32), v);
        if (p.nout > 0 && p.tag_f32) {
          if (row_l < rvalid * 16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int tok = tok0 + cc * 32 + j;
              if (cc * 32 + j < p.bn && tok < p.m) store_tagged_f32(p, tok, row, __uint_as_float(v[j]), epoch);
            }
          }
        } else if (p.nout > 0) {
          // tagged pairs: row g + 8 of a tile is lane + 8 of the same warp (the shuffle runs on the whole warp)
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float f = __uint_as_float(v[j]);
            const float fh = __shfl_down_sync(0xffffffffu, f, 8);
            const int tok = tok0 + cc * 32 + j;
            if ((lane & 8) == 0 && row_l < rvalid * 16 && cc * 32 + j < p.bn && tok < p.m)
              store_tagged(p, tok, row, f, fh, epoch);
          }
        } else if (row_l < rvalid * 16) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            // columns past the tile's bn tokens (bn % 32 != 0) belong to the next token tile's CTA
            const int tok = tok0 + cc * 32 + j;
            if (cc * 32 + j < p.bn && tok < p.m) store_elem(p, tok, row, __uint_as_float(v[j]));
          }
        }
      }
    }
  } else {
    // Partial tiles go to shared memory column-major (element (r, c) at c*128 + r, conflict-free), the ring
    // area being free once every MMA has completed; rank ks then sums columns [c0, c1) over the cluster.
    float* red = reinterpret_cast<float*>(sm);
    if (epi) {
      for (int cc = part; cc < ncol; cc += nparts) {
        uint32_t v[32];
        if (ok) tc_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc * 32), v);
#pragma unroll
        for (int j = 0; j < 32; ++j) red[(cc * 32 + j) * 128 + row_l] = ok ? __uint_as_float(v[j]) : 0.f;
      }
    }
    __syncthreads();  // every role of this CTA is done before the cluster barrier
    cluster_sync();
    const int per = (ncol * 32 + p.split - 1) / p.split;
    const int c0 = ks * per, c1 = min(ncol * 32, c0 + per);
    const uint32_t raddr = smem_u32(red);
    for (int idx = tid; idx < (c1 - c0) * 128; idx += kThreads) {
      const int c = c0 + idx / 128, r = idx % 128;
      float s = 0.f;
      for (int rk = 0; rk < p.split; ++rk) {
        float f;
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(f)
                     : "r"(mapa(raddr + (uint32_t)(c * 128 + r) * 4, (uint32_t)rk)));
        s += f;
      }
      const int tok = tok0 + c, grow = rb0 * 16 + r;
      if (p.nout > 0 && p.tag_f32) {
        if (c < p.bn && tok < p.m && r < rvalid * 16) store_tagged_f32(p, tok, grow, s, epoch);
      } else if (p.nout > 0) {
        // a warp holds 32 consecutive rows of one column (640 threads, 128 rows per column): row + 8 is lane + 8
        const float sh = __shfl_down_sync(0xffffffffu, s, 8);
        if ((r & 8) == 0 && c < p.bn && tok < p.m && r < rvalid * 16) store_tagged(p, tok, grow, s, sh, epoch);
      } else if (c < p.bn && tok < p.m && r < rvalid * 16) {
        store_elem(p, tok, grow, s);
      }
    }
    cluster_sync();  // keep this CTA's partials alive until every rank has read them
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

// Weight units as a 3-D tensor of u64 with a box of 8 row tiles x 2 sub-tiles per stage:
//   12-bit units [R][C][1536 bytes] -> {192, C, R}, box {192, 2, 8} (chunks c, c + 1; {192, 1, 8} for a matrix of
//   one chunk);
//   hi/lo units  [R][C][2][2048 bytes] -> {256, 2C, R}, box {256, 2, 8} (chunk c = indices 2c, 2c + 1).
// (Measured alternative: 128-byte rows with a 128-byte swizzle and a ring as deep as shared memory allows was
// 10-15 % slower; the decoders' instruction issue, not the copy engine, bounds the small-M calls.)
bool encode_units_3d(CUtensorMap* map, const void* units, int R, int C, bool hilo) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t inner = hilo ? 256 : 192, mid = hilo ? 2 * (cuuint64_t)C : (cuuint64_t)C;
  const cuuint64_t row = (cuuint64_t)C * (hilo ? 2 * MBP_RAW_UNIT_BYTES : MBP_C12_UNIT_BYTES);
  const cuuint64_t dims[3] = {inner, mid, (cuuint64_t)R};
  const cuuint64_t strides[2] = {inner * 8, row};
  const cuuint32_t box[3] = {(cuuint32_t)inner, mid >= 2 ? 2u : 1u, 8};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(units), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

using GemmKernel = void (*)(GemmParams);

GemmKernel kernel_of(bool hilo) { return hilo ? k_gemm<true> : k_gemm<false>; }

std::mutex g_mu;
std::map<std::pair<int, bool>, bool> g_attr_done;
std::map<std::tuple<int, bool, int, int>, int> g_clusters;  // (device, format, split, smem) -> co-resident CTAs

int ensure_attr(bool hilo) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MBP_ERR_LAUNCH;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_attr_done.count({dev, hilo})) return MBP_OK;
  const void* fn = reinterpret_cast<const void*>(kernel_of(hilo));
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
    return MBP_ERR_SMEM;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return MBP_ERR_CLUSTER;
  g_attr_done[{dev, hilo}] = true;
  return MBP_OK;
}

int co_resident_ctas(bool hilo, int split, int smem) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const auto key = std::make_tuple(dev, hilo, split, smem);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_clusters.find(key);
    if (it != g_clusters.end()) return it->second;
  }
  int ctas = sms;
  if (split > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, split);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = split;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    ctas = cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void*>(kernel_of(hilo)), &cfg) ==
                   cudaSuccess
               ? clusters * split
               : 0;
    cudaGetLastError();
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_clusters[key] = ctas;
  return ctas;
}

// K split: the largest cluster (min_split .. max_split, >= 4 chunks per CTA) whose tiles still fit one wave of
// co-resident CTAs, when the tile count alone leaves more than a quarter of the SMs idle; else min_split.
int choose_split(bool hilo, int tiles, int C, int smem, int min_split, int max_split) {
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (tiles * 4 >= sms * 3) return min_split;
  int best = min_split;
  for (int s = min_split < 2 ? 2 : min_split; s <= max_split; ++s) {
    if (C / s < 4) break;
    const int cap = co_resident_ctas(hilo, s, smem);
    if (cap >= tiles * s && tiles * s <= sms) best = s;
  }
  return best;
}

int sm_count_here() {
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// One launch of k_gemm<hilo>: units/bases/escapes describe the weights (bases and escapes unused for hi/lo),
// R16 = row tiles of the weights, rout16 = row tiles written, C = 64-column chunks.  bn: token tile; split: K
// split (cluster size; 0 = choose).
struct GemmTag {  // tagged exchange outputs (tensor-parallel column gather, or row-parallel f32 partials)
  void* const* outs;
  int nout;
  int f32;
  const int* epoch;
  long long parity_stride;
};

int launch_gemm(bool hilo, const uint8_t* units, const uint8_t* bases, const int32_t* esc_off, const uint32_t* esc,
                int R16, int rout16, int C, const uint16_t* x, int m, void* out, int ldo, bool f32, int bn, int split,
                int min_split, int max_split, cudaStream_t stream, const GemmTag* tag = nullptr) {
  const GLayout L = gemm_layout(bn, hilo);
  const int smem = L.total + 1024;
  if (smem > kMaxSmem) return MBP_ERR_SMEM;
  // the cluster reduction reuses the ring area for a 128 x bn FP32 tile
  if (128 * ((bn + 31) / 32) * 32 * 4 > L.xr) return MBP_ERR_SMEM;
  int rc = ensure_attr(hilo);
  if (rc) return rc;
  GemmParams p;
  const TmapKey wkey{units, (uint64_t)R16, (uint64_t)C, 0, 0, 0, hilo ? 0x203u : 0x202u};
  if (!cached_map(&p.wmap, wkey, [&](CUtensorMap* mp) { return encode_units_3d(mp, units, R16, C, hilo); }))
    return MBP_ERR_TMAP;
  if (!encode_bf16_2d_cached(&p.xmap, x, (uint64_t)m, (uint64_t)C * 64, (uint64_t)C * 64, (uint32_t)bn, 64u,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return MBP_ERR_TMAP;
  p.units = units;
  p.bases = bases;
  p.esc_off = esc_off;
  p.esc = esc;
  p.out = out;
  p.C = C;
  p.Rout = rout16;
  p.m = m;
  p.ldo = ldo;
  p.bn = bn;
  p.f32out = f32 ? 1 : 0;
  p.wsubs = (hilo || C >= 2) ? 2 : 1;
  p.nout = tag ? tag->nout : 0;
  p.tag_f32 = tag ? tag->f32 : 0;
  for (int o = 0; o < 8; ++o) p.touts[o] = tag && o < tag->nout ? tag->outs[o] : nullptr;
  p.epoch = tag ? tag->epoch : nullptr;
  p.parity_stride = tag ? tag->parity_stride : 0;
  p.wait_ns = wait_limit_ns();
  const int ntok = (m + bn - 1) / bn;
  p.nblk = (p.Rout + 7) / 8;
  const int tiles = p.nblk * ntok;
  p.split = split > 0 ? split : choose_split(hilo, tiles, C, smem, min_split, max_split);
  if (p.split == 1 && bn <= 128) {
    // No K split and token tiles of <= 128 (decode-bound): spread the row tiles over as many blocks as one wave
    // holds (6-7 tiles each instead of 8 when 8-tile blocks would leave SMs idle, e.g. 148 blocks instead of 112
    // for 896 row tiles); the decoders of a block's unused rows idle, so each CTA decodes fewer units.  Measured
    // 3-8 % faster at 8-128 tokens; at 256 tokens the MMAs (always 128 rows) dominate and 148 blocks were 6 %
    // slower than 112.
    const int wave = sm_count_here() / ntok;
    if (wave > p.nblk) p.nblk = wave < p.Rout ? wave : p.Rout;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nblk, ntok, p.split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  static const bool pdl = getenv("MBP_NO_PDL") == nullptr;  // MBP_NO_PDL set: plain stream serialisation
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = p.split;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel_of(hilo), p) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int gemm_launch(const mbp_c12* w, const uint16_t* x, int m, int n_out, void* out, int ldo, bool f32,
                cudaStream_t stream, const GemmTag* tag = nullptr) {
  if (!w || !w->units || !w->bases || !w->esc_off || !x || (!out && !tag)) return MBP_ERR_ARG;
  if (w->n_esc > 0 && !w->esc) return MBP_ERR_ARG;
  if (w->n % 16 || w->k % 64 || w->k / 64 > 32766 || n_out > w->n || n_out <= 0 || n_out % 16) return MBP_ERR_SHAPE;
  if (m < 1) return MBP_ERR_M;
  if (tag ? ldo < (tag->f32 ? n_out : n_out / 2) : ldo < n_out) return MBP_ERR_SHAPE;  // tagged: ldo in words
  if (((uintptr_t)x & 15u) || ((uintptr_t)w->units & 15u)) return MBP_ERR_ALIGN;
  // Token tile: all tokens up to 256.  Short K (<= 2048): a cluster split-K's reduction costs more than its
  // short main loop saves, so smaller token tiles fill the SMs instead, down to 64 while one wave holds them
  // (measured at M=256: o 8192x1024 11.5 us with 128-token tiles against 16.9 us with a 2-way K split).
  int bn = m >= 256 ? 256 : ((m + 15) / 16) * 16;
  if (w->k / 64 <= 32) {
    const int sms = sm_count_here();
    const int row_blocks = (n_out / 16 + 7) / 8;
    int ntok = (m + bn - 1) / bn;
    for (;;) {  // double the token tiles (balanced, multiples of 16 tokens) while they stay >= 64 and one wave
      const int t2 = 2 * ntok, bn2 = ((m + t2 - 1) / t2 + 15) / 16 * 16;
      if (bn2 < 64 || row_blocks * ((m + bn2 - 1) / bn2) > sms) break;
      ntok = t2;
      bn = bn2;
    }
  }
  return launch_gemm(false, w->units, w->bases, w->esc_off, w->esc, w->n / 16, n_out / 16, w->k / 64, x, m, out,
                     ldo, f32, bn, 0, 1, 8, stream, tag);
}

}  // namespace

extern "C" {

int mbp_gemm_c12(const mbp_c12* w, const uint16_t* x, int m, int n_out, uint16_t* out, int ldo,
                 cudaStream_t stream) {
  return gemm_launch(w, x, m, n_out, out, ldo, false, stream);
}

int mbp_gemm_c12_f32(const mbp_c12* w, const uint16_t* x, int m, int n_out, float* out, int ldo,
                     cudaStream_t stream) {
  return gemm_launch(w, x, m, n_out, out, ldo, true, stream);
}

int mbp_gemm_c12_multi(const mbp_c12* w, const uint16_t* x, int m, int n_out, void* const* outs, int nout, int ldo,
                       int out_kind, const int* epoch, long long parity_stride, cudaStream_t stream) {
  if (out_kind != MBP_OUT_TAGGED_BF16X2 && out_kind != MBP_OUT_TAGGED_F32) return MBP_ERR_ARG;
  const bool f32 = out_kind == MBP_OUT_TAGGED_F32;
  if (!outs || nout < 1 || nout > 8 || !epoch) return MBP_ERR_ARG;
  if (parity_stride < 0 || (parity_stride & 15)) return MBP_ERR_ALIGN;
  for (int o = 0; o < nout; ++o) {
    if (!outs[o]) return MBP_ERR_ARG;
    if ((uintptr_t)outs[o] & 7u) return MBP_ERR_ALIGN;
  }
  if (ldo < (f32 ? n_out : n_out / 2)) return MBP_ERR_SHAPE;
  const GemmTag tag{outs, nout, f32 ? 1 : 0, epoch, parity_stride};
  return gemm_launch(w, x, m, n_out, nullptr, ldo, false, stream, &tag);
}

int mbp_router_hilo_tc(const mbp_hilo* w, const uint16_t* x, int m, float* out, int ldo, int bn, int split,
                       cudaStream_t stream) {
  if (!w || !w->units || !x || !out) return MBP_ERR_ARG;
  const int C = w->k / 64;
  if (w->n % 16 || w->k % 64 || C > kRouterTcMaxChunks * 16) return MBP_ERR_SHAPE;
  if (m < 1) return MBP_ERR_M;
  if (ldo < w->n) return MBP_ERR_SHAPE;
  if (((uintptr_t)x & 15u) || ((uintptr_t)w->units & 15u)) return MBP_ERR_ALIGN;
  // The tensor pipe's FP32 accumulation over one CTA's whole K range measured 1.4e-5 relative error against
  // FP64 at 6144 columns (96 chunks, hi + lo), above the router's 1e-5 bound; with at most 32 chunks per CTA and
  // the cluster's partial sums added in FP32 it stays well inside, so the K split never goes below that.
  const int min_split = (C + kRouterTcMaxChunks - 1) / kRouterTcMaxChunks;
  if (bn < 0 || bn > 128 || bn % 16 || split < 0 || split > 16 || split > C) return MBP_ERR_ARG;
  if (split > 0 && split < min_split) return MBP_ERR_ARG;
  if (bn == 0) {
    // Token tiles of 64 (fewer when M is small), the K split filling the SMs through clusters of up to 16: the
    // router has only two 128-row blocks, so its parallelism comes from the tokens and the K range.
    bn = m >= 64 ? 64 : ((m + 15) / 16) * 16;
  }
  return launch_gemm(true, w->units, nullptr, nullptr, nullptr, w->n / 16, w->n / 16, C, x, m, out, ldo, true, bn,
                     split, min_split, 16, stream);
}

}  // extern "C"

int mbp_status_gemm(int* v, int clear) { return read_status_here(v, clear); }
