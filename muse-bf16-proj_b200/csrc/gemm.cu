// Verify-path GEMM for larger token counts (M > 32): out[m, n] = x[m, k] . W[n, k]^T on the 5th-generation
// tensor cores (tcgen05 + TMEM), weights unpacked from the 12-bit format in shared memory.
//
// Replaces the reference's dense BF16 verify GEMMs (submission.py: ss_gemm S:783<17-123>, q_kernel
// S:979<25-170>, qb_kernel S:4576, ol_projection S:1547<18-106>, projection S:2985) and its cuBLASLt routes
// (S:2309-2376, out of scope), which read unpacked BF16 weights; here the weights stay packed in HBM.
//
// CTA tile: 128 weight rows (8 row tiles) x BN tokens (<= 256), full K.  Warp roles:
//   warp 0      TMA producer: per 64-column chunk, one 3-D box of 8 packed units (12 KB) and one 2-D box of
//               the x tile (BN rows x 128 bytes, 128-byte swizzle), each completing on its ring's mbarrier;
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=16, BF16 -> FP32) x4 per chunk,
//               A = decoded weights and B = x, both K-major SW128 shared-memory descriptors; tcgen05.commit
//               frees the A and x stages and finally signals the accumulator;
//   warps 2-9   decoders: warp d decodes row tile d of each chunk in registers (same decode and escape cursor
//               as the GEMV), stores it into the A stage in the canonical SW128 K-major layout and fences it
//               to the async proxy; afterwards they read the accumulator (tcgen05.ld 32x32b) and store BF16.
// All waits are bounded; TMEM is always released.
#include "common.cuh"
#include "escape.cuh"
#include "tmap.h"

#include <map>
#include <mutex>

using namespace mbp;

namespace {

constexpr int kThreads = 320;  // 10 warps
constexpr int kDecWarps = 8;
constexpr int kPS = 4;         // packed ring depth
constexpr int kAS = 3;         // decoded-A ring depth
constexpr int kXS = 3;         // x ring depth
constexpr int kPackedStage = 8 * MBP_C12_UNIT_BYTES;  // 12 KB
constexpr int kAStage = 128 * 128;                    // 128 rows x 64 bf16

struct __align__(64) GemmParams {
  CUtensorMap wmap;  // units as [R][C][192 x u64], box {192, 1, 8}
  CUtensorMap xmap;  // x [m, k] bf16, box {64 columns, BN rows}, 128-byte swizzle
  const uint8_t* bases;
  const int32_t* esc_off;
  const uint32_t* esc;
  void* out;
  int C, Rout, m, ldo, bn;
  int f32out;
};

struct GLayout {
  int packed, a, x, xr, bars, tmem_slot, total;
};

__host__ __device__ inline GLayout gemm_layout(int bn) {
  GLayout L;
  L.packed = 0;
  L.a = L.packed + kPS * kPackedStage;              // multiple of 1024
  L.x = L.a + kAS * kAStage;                        // multiple of 1024
  L.xr = L.x + kXS * bn * 128;                      // bn multiple of 16 -> multiple of 2048
  L.bars = L.xr + kDecWarps * kXorWarpBytes;
  L.tmem_slot = L.bars + 8 * (2 * kPS + 2 * kAS + 2 * kXS + 1);
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

__global__ void __launch_bounds__(kThreads, 1) k_gemm(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const GLayout L = gemm_layout(p.bn);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bars = base + L.bars;
  const uint32_t pfull = bars, pempty = pfull + 8 * kPS;
  const uint32_t afull = pempty + 8 * kPS, aempty = afull + 8 * kAS;
  const uint32_t xfull = aempty + 8 * kAS, xempty = xfull + 8 * kXS;
  const uint32_t done = xempty + 8 * kXS;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sm + L.tmem_slot);
  const int C = p.C;
  const int rb0 = blockIdx.x * 8;  // first row tile
  const int tok0 = blockIdx.y * p.bn;
  const uint32_t tmem_cols = p.bn <= 32 ? 32 : p.bn <= 64 ? 64 : p.bn <= 128 ? 128 : 256;

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
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int c = 0; c < C; ++c) {
        const int ps = c % kPS, xs = c % kXS;
        if (c >= kPS && !mbar_wait(pempty + 8 * ps, ((c / kPS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY)) break;
        mbar_arrive_expect_tx(pfull + 8 * ps, kPackedStage);
        tma_load_3d(base + L.packed + ps * kPackedStage, &p.wmap, 0, c, rb0, pfull + 8 * ps);
        if (c >= kXS && !mbar_wait(xempty + 8 * xs, ((c / kXS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY)) break;
        mbar_arrive_expect_tx(xfull + 8 * xs, (uint32_t)p.bn * 128);
        tma_load_2d(base + L.x + xs * p.bn * 128, &p.xmap, c * 64, tok0, xfull + 8 * xs);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(p.bn);
      for (int c = 0; c < C; ++c) {
        const int as = c % kAS, xs = c % kXS;
        if (!mbar_wait(afull + 8 * as, (c / kAS) & 1, MBP_DEV_TIMEOUT_FULL)) break;
        if (!mbar_wait(xfull + 8 * xs, (c / kXS) & 1, MBP_DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        const uint32_t a0 = base + L.a + as * kAStage, b0 = base + L.x + xs * p.bn * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma(tmem, smem_desc_sw128(a0 + 32 * k), smem_desc_sw128(b0 + 32 * k), idesc, (c | k) != 0);
        tc_commit(aempty + 8 * as);
        tc_commit(xempty + 8 * xs);
      }
      tc_commit(done);  // fires when every issued MMA has completed
    }
    __syncwarp();
  } else {
    // ---------------- decoders ----------------
    const int d = warp - 2;  // row tile within the block
    const int rt = rb0 + d;
    const bool valid = rt < p.Rout;
    uint32_t T0 = 0, T1 = 0;
    EscCursor cur;
    const uint32_t xr = base + L.xr + d * kXorWarpBytes;
    xor_mask_clear(xr, lane);
    if (valid) {
      const uint32_t b = p.bases[rt];
      T0 = table_lo(b);
      T1 = table_hi(b);
      cur.init(p.esc, p.esc_off[(size_t)rt * C], p.esc_off[(size_t)rt * C + C], lane);
    } else {
      cur.init(p.esc, 0, 0, lane);
    }
    const int g = lane >> 2, t = lane & 3;
    // destination rows r = 16 d + 8 rh + g inside the 128-row A tile (SW128 K-major)
    uint32_t dst[2][2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int r = 16 * d + 8 * rh + g;
      const uint32_t row = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
      dst[rh][0] = row + ((uint32_t)((2 * t) ^ (r & 7)) << 4);
      dst[rh][1] = row + ((uint32_t)((2 * t + 1) ^ (r & 7)) << 4);
    }
    for (int c = 0; c < C; ++c) {
      const int ps = c % kPS, as = c % kAS;
      if (!mbar_wait(pfull + 8 * ps, (c / kPS) & 1, MBP_DEV_TIMEOUT_FULL)) break;
      const unsigned char* u = sm + L.packed + ps * kPackedStage + d * MBP_C12_UNIT_BYTES + lane * 16;
      const uint4 p0 = *reinterpret_cast<const uint4*>(u);
      const uint4 p1 = *reinterpret_cast<const uint4*>(u + 512);
      const uint4 p2 = *reinterpret_cast<const uint4*>(u + 1024);
      mbar_arrive(pempty + 8 * ps);
      uint32_t A[16];
      decode_unit(p0, p1, p2, T0, T1, A);
      if (valid) cur.apply((uint32_t)c, A, xr, lane);
      if (c >= kAS && !mbar_wait(aempty + 8 * as, ((c / kAS) & 1) ^ 1, MBP_DEV_TIMEOUT_EMPTY)) break;
      unsigned char* a = sm + L.a + as * kAStage;
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        *reinterpret_cast<uint4*>(a + dst[rh][0]) = make_uint4(A[0 + rh], A[2 + rh], A[4 + rh], A[6 + rh]);
        *reinterpret_cast<uint4*>(a + dst[rh][1]) = make_uint4(A[8 + rh], A[10 + rh], A[12 + rh], A[14 + rh]);
      }
      fence_async_smem();
      mbar_arrive(afull + 8 * as);
    }
    // ---------------- epilogue: TMEM -> registers -> global ----------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;
    const bool ok = mbar_wait(done, 0, MBP_DEV_TIMEOUT_MMA);
    tc_fence_after();
    if (ok) {
      const int row = rb0 * 16 + q * 32 + lane;
      const int ncol = (p.bn + 31) / 32;
      for (int cc = half; cc < ncol; cc += 2) {
        uint32_t v[32];
        tc_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc * 32), v);
        if (row < p.Rout * 16) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int tok = tok0 + cc * 32 + j;
            if (tok < p.m) {
              const float f = __uint_as_float(v[j]);
              if (p.f32out)
                reinterpret_cast<float*>(p.out)[(size_t)tok * p.ldo + row] = f;
              else
                reinterpret_cast<uint16_t*>(p.out)[(size_t)tok * p.ldo + row] =
                    __bfloat16_as_ushort(__float2bfloat16_rn(f));
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

// units [R][C][1536 bytes] viewed as a 3-D tensor of u64: {192, C, R}, box {192, 1, 8}
bool encode_units_3d(CUtensorMap* map, const void* units, int R, int C) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {192, (cuuint64_t)C, (cuuint64_t)R};
  const cuuint64_t strides[2] = {(cuuint64_t)MBP_C12_UNIT_BYTES, (cuuint64_t)C * MBP_C12_UNIT_BYTES};
  const cuuint32_t box[3] = {192, 1, 8};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(units), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::mutex g_attr_mu;
std::map<int, bool> g_attr_done;

int ensure_attr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MBP_ERR_LAUNCH;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (g_attr_done.count(dev)) return MBP_OK;
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_gemm), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           227 * 1024) != cudaSuccess)
    return MBP_ERR_SMEM;
  g_attr_done[dev] = true;
  return MBP_OK;
}

int gemm_launch(const mbp_c12* w, const uint16_t* x, int m, int n_out, void* out, int ldo, bool f32,
                cudaStream_t stream) {
  if (!w || !w->units || !w->bases || !w->esc_off || !x || !out) return MBP_ERR_ARG;
  if (w->n_esc > 0 && !w->esc) return MBP_ERR_ARG;
  if (w->n % 16 || w->k % 64 || w->k / 64 > 32766 || n_out > w->n || n_out <= 0 || n_out % 16) return MBP_ERR_SHAPE;
  if (m < 1) return MBP_ERR_M;
  if (ldo < n_out) return MBP_ERR_SHAPE;
  if (((uintptr_t)x & 15u) || ((uintptr_t)w->units & 15u)) return MBP_ERR_ALIGN;
  const int bn = m >= 256 ? 256 : ((m + 15) / 16) * 16;
  const GLayout L = gemm_layout(bn);
  if (L.total + 1024 > 227 * 1024) return MBP_ERR_SMEM;
  int rc = ensure_attr();
  if (rc) return rc;
  GemmParams p;
  const int R = w->n / 16, C = w->k / 64;
  if (!encode_units_3d(&p.wmap, w->units, R, C)) return MBP_ERR_TMAP;
  if (!encode_bf16_2d(&p.xmap, x, (uint64_t)m, (uint64_t)w->k, (uint64_t)w->k, (uint32_t)bn, 64u,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return MBP_ERR_TMAP;
  p.bases = w->bases;
  p.esc_off = w->esc_off;
  p.esc = w->esc;
  p.out = out;
  p.C = C;
  p.Rout = n_out / 16;
  p.m = m;
  p.ldo = ldo;
  p.bn = bn;
  p.f32out = f32 ? 1 : 0;
  dim3 grid((p.Rout + 7) / 8, (m + bn - 1) / bn, 1);
  k_gemm<<<grid, kThreads, L.total + 1024, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
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

}  // extern "C"

int mbp_status_gemm(int* v, int clear) { return read_status_here(v, clear); }
