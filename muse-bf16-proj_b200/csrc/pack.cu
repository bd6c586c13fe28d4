// GPU packer for the lossless 12-bit BF16 weight format, its exact inverse, and the FP32 -> BF16 hi/lo
// router split.  Replaces the reference's host-side torch packer (submission.py S:82-227: sm_units,
// sm_c12_bytes, sm_c12_unpack, sm_stream; router split S:876-879), which ran bincount/argsort/nonzero on the
// host at prepare time.
//
// Phases of mbp_pack_c12 (all on the stream):
//   k_hist     one CTA per 16-row tile: 128-bin histogram of the 7 high exponent bits       (S:108-110)
//   k_bases    window argmax, per tile or for the whole matrix                                (S:111-113)
//   k_pack     one warp per 16x64 unit: low bytes + 3-bit offsets + signs, escape count        (S:114-121)
//   k_scan     exclusive scan of per-unit escape counts -> esc_off                              (new: CSR)
// mbp_pack_c12_escapes:
//   k_escapes  one warp per unit: entries chunk<<17 | lane<<12 | value<<7 | xor7 in (lane, value) order
#include <mutex>

#include "common.cuh"
#include "escape.cuh"

using namespace mbp;

namespace {

// Sign bit of value i (0..7) inside a code word: {3, 19, 7, 23, 11, 27, 15, 31}[i] (S:58).
__host__ __device__ constexpr int sign_pos(int i) { return 3 + 2 * i + 14 * (i & 1); }

// Value index v (0..31) of element j (0..15, column 16t + j) of row half rh in a lane's unit slice.
__host__ __device__ constexpr int value_of(int j, int rh) {
  return (j >> 2) * 8 + ((j >> 1) & 1) * 4 + rh * 2 + (j & 1);
}

__global__ void k_hist(const uint16_t* __restrict__ w, int k, int* __restrict__ hist) {
  __shared__ int h[128];
  for (int i = threadIdx.x; i < 128; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int r = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)r * 16 * k);
  const int nvec = 16 * k / 8;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const uint4 v = __ldg(src + i);
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicAdd(&h[(words[j] >> 8) & 0x7F], 1);
      atomicAdd(&h[(words[j] >> 24) & 0x7F], 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 128; i += blockDim.x) hist[r * 128 + i] = h[i];
}

// blockDim.x == 128.  Matrix mode: one CTA sums every tile's histogram; tile mode: one CTA per tile.
__global__ void k_bases(const int* __restrict__ hist, int R, int per_tile, uint8_t* __restrict__ bases) {
  __shared__ long long h[128];
  __shared__ int best;
  const int b = threadIdx.x;
  long long s = 0;
  if (per_tile) {
    s = hist[blockIdx.x * 128 + b];
  } else {
    for (int r = 0; r < R; ++r) s += hist[r * 128 + b];
  }
  h[b] = s;
  __syncthreads();
  if (b == 0) {
    long long bestv = -1;
    int bi = 0;
    for (int i = 0; i < 121; ++i) {  // first maximum of the 8-wide window sums (torch argmax semantics)
      long long ws = 0;
      for (int j = 0; j < 8; ++j) ws += h[i + j];
      if (ws > bestv) {
        bestv = ws;
        bi = i;
      }
    }
    best = bi;
  }
  __syncthreads();
  if (per_tile) {
    if (b == 0) bases[blockIdx.x] = (uint8_t)best;
  } else {
    for (int r = b; r < R; r += 128) bases[r] = (uint8_t)best;
  }
}

// Loads lane (g, t)'s 32 weights of unit (r, c): vals[rh][j] = W[16r + 8rh + g][64c + 16t + j].
__device__ __forceinline__ void load_unit_slice(const uint16_t* __restrict__ w, int k, int r, int c, int lane,
                                                uint16_t (&vals)[2][16]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    const uint4* p = reinterpret_cast<const uint4*>(w + (size_t)(16 * r + 8 * rh + g) * k + 64 * c + 16 * t);
    const uint4 a = __ldg(p), b = __ldg(p + 1);
    const uint32_t words[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      vals[rh][2 * j] = (uint16_t)(words[j] & 0xFFFF);
      vals[rh][2 * j + 1] = (uint16_t)(words[j] >> 16);
    }
  }
}

__global__ void k_pack(const uint16_t* __restrict__ w, int k, int R, int C, const uint8_t* __restrict__ bases,
                       uint8_t* __restrict__ units, int32_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const long long u = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (u >= (long long)R * C) return;
  const int r = (int)(u / C), c = (int)(u % C);
  const int base = bases[r];
  uint16_t vals[2][16];
  load_unit_slice(w, k, r, c, lane, vals);
  uint8_t lo[32];
  uint32_t code[4] = {0, 0, 0, 0};
  int nesc = 0;
#pragma unroll
  for (int rh = 0; rh < 2; ++rh)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int v = value_of(j, rh);
      const uint32_t x = vals[rh][j];
      int d = (int)((x >> 8) & 0x7F) - base;
      if (d < 0 || d >= 8) {
        ++nesc;
        d = 0;
      }
      lo[v] = (uint8_t)(x & 0xFF);
      code[v >> 3] |= ((uint32_t)d << (4 * (v & 7))) | ((x >> 15) << sign_pos(v & 7));
    }
  uint8_t* dst = units + (size_t)u * MBP_C12_UNIT_BYTES + lane * 16;
  uint4 p0, p1;
  p0.x = lo[0] | lo[1] << 8 | lo[2] << 16 | (uint32_t)lo[3] << 24;
  p0.y = lo[4] | lo[5] << 8 | lo[6] << 16 | (uint32_t)lo[7] << 24;
  p0.z = lo[8] | lo[9] << 8 | lo[10] << 16 | (uint32_t)lo[11] << 24;
  p0.w = lo[12] | lo[13] << 8 | lo[14] << 16 | (uint32_t)lo[15] << 24;
  p1.x = lo[16] | lo[17] << 8 | lo[18] << 16 | (uint32_t)lo[19] << 24;
  p1.y = lo[20] | lo[21] << 8 | lo[22] << 16 | (uint32_t)lo[23] << 24;
  p1.z = lo[24] | lo[25] << 8 | lo[26] << 16 | (uint32_t)lo[27] << 24;
  p1.w = lo[28] | lo[29] << 8 | lo[30] << 16 | (uint32_t)lo[31] << 24;
  *reinterpret_cast<uint4*>(dst) = p0;
  *reinterpret_cast<uint4*>(dst + 512) = p1;
  *reinterpret_cast<uint4*>(dst + 1024) = make_uint4(code[0], code[1], code[2], code[3]);
  const int tot = __reduce_add_sync(0xffffffffu, nesc);
  if (lane == 0) counts[u] = tot;
}

// Exclusive scan in place over n counts, writing the total at [n].  One CTA of 1024 threads.
__global__ void k_scan(int32_t* __restrict__ a, long long n) {
  __shared__ int warp_sums[32];
  __shared__ long long carry_s;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  constexpr int PER = 4;
  for (long long base = 0; base < n; base += 1024 * PER) {
    int v[PER];
    int s = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const long long idx = base + (long long)tid * PER + i;
      v[i] = idx < n ? a[idx] : 0;
      s += v[i];
    }
    int inc = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane == 31) warp_sums[wid] = inc;
    __syncthreads();
    if (wid == 0) {
      int ws = warp_sums[lane];
      int wi = ws;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += y;
      }
      warp_sums[lane] = wi - ws;  // exclusive warp offsets
    }
    __syncthreads();
    long long run = carry_s + warp_sums[wid] + (inc - s);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const long long idx = base + (long long)tid * PER + i;
      if (idx < n) a[idx] = (int32_t)run;
      run += v[i];
    }
    __syncthreads();
    if (tid == 1023) carry_s = run;
    __syncthreads();
  }
  if (tid == 0) a[n] = (int32_t)carry_s;
}

__global__ void k_escapes(const uint16_t* __restrict__ w, int k, int R, int C, const uint8_t* __restrict__ bases,
                          const int32_t* __restrict__ esc_off, uint32_t* __restrict__ esc) {
  const int lane = threadIdx.x & 31;
  const long long u = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (u >= (long long)R * C) return;
  const int r = (int)(u / C), c = (int)(u % C);
  const int base = bases[r];
  uint16_t vals[2][16];
  load_unit_slice(w, k, r, c, lane, vals);
  uint32_t mask = 0;  // bit v set when value v escapes
#pragma unroll
  for (int rh = 0; rh < 2; ++rh)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = (int)((vals[rh][j] >> 8) & 0x7F) - base;
      if (d < 0 || d >= 8) mask |= 1u << value_of(j, rh);
    }
  const int cnt = __popc(mask);
  int pre = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, pre, o);
    if (lane >= o) pre += y;
  }
  int pos = esc_off[u] + pre - cnt;
  uint16_t byv[32];  // the lane's values in value order
#pragma unroll
  for (int rh = 0; rh < 2; ++rh)
#pragma unroll
    for (int j = 0; j < 16; ++j) byv[value_of(j, rh)] = vals[rh][j];
#pragma unroll
  for (int v = 0; v < 32; ++v) {
    if (mask >> v & 1u) {
      const uint32_t eh = (byv[v] >> 8) & 0x7F;
      esc[pos++] = ((uint32_t)c << 17) | ((uint32_t)lane << 12) | ((uint32_t)v << 7) | (eh ^ (uint32_t)base);
    }
  }
}

// Device unpack: one warp per unit, through the same decode and escape cursor as the GEMV.
__global__ void k_unpack(const uint8_t* __restrict__ units, const uint8_t* __restrict__ bases,
                         const int32_t* __restrict__ esc_off, const uint32_t* __restrict__ esc, int R, int C, int k,
                         uint16_t* __restrict__ w) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long u = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  const uint32_t xr = smem_u32(smem) + warp * kMaskUnitBytes;
  mask_clear(xr, kMaskUnitBytes, lane);
  if (u >= (long long)R * C) return;
  const int r = (int)(u / C), c = (int)(u % C);
  const uint8_t* src = units + (size_t)u * MBP_C12_UNIT_BYTES + lane * 16;
  const uint4 p0 = *reinterpret_cast<const uint4*>(src);
  const uint4 p1 = *reinterpret_cast<const uint4*>(src + 512);
  const uint4 p2 = *reinterpret_cast<const uint4*>(src + 1024);
  uint32_t A[16];
  EscCursor cur;
  cur.init(esc, esc_off[u], esc_off[u + 1], lane);
  uint32_t tgt[1] = {0u};
  cur.scatter<1>((uint32_t)c, (uint32_t)c + 1, xr, kMaskUnitBytes, lane, tgt);
  __syncwarp();
  uint4 m0, m1;
  take_mask(xr, tgt[0], lane, m0, m1);
  decode_unit_m(p0, p1, p2, table_lo(bases[r]), table_hi(bases[r]), m0, m1, A);
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    uint4* dst = reinterpret_cast<uint4*>(w + (size_t)(16 * r + 8 * rh + g) * k + 64 * c + 16 * t);
    dst[0] = make_uint4(A[0 + rh], A[2 + rh], A[4 + rh], A[6 + rh]);
    dst[1] = make_uint4(A[8 + rh], A[10 + rh], A[12 + rh], A[14 + rh]);
  }
}

// FP32 [n, k] -> hi/lo raw units [R][C][2][2048]: plane q of a unit = 8 values 8q..8q+7 per lane, lane-major.
__global__ void k_pack_hilo(const float* __restrict__ w, int k, int R, int C, uint8_t* __restrict__ units) {
  const int lane = threadIdx.x & 31;
  const long long u = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (u >= (long long)R * C) return;
  const int r = (int)(u / C), c = (int)(u % C);
  const int g = lane >> 2, t = lane & 3;
  uint16_t hi[32], lo[32];
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    const float4* p = reinterpret_cast<const float4*>(w + (size_t)(16 * r + 8 * rh + g) * k + 64 * c + 16 * t);
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const float4 f = __ldg(p + q4);
      const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * q4 + e;
        const int v = value_of(j, rh);
        const __nv_bfloat16 h = __float2bfloat16_rn(fv[e]);
        const __nv_bfloat16 l = __float2bfloat16_rn(fv[e] - __bfloat162float(h));
        hi[v] = __bfloat16_as_ushort(h);
        lo[v] = __bfloat16_as_ushort(l);
      }
    }
  }
  uint8_t* dst = units + (size_t)u * 2 * MBP_RAW_UNIT_BYTES + lane * 16;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 a, b;
    a.x = hi[8 * q + 0] | (uint32_t)hi[8 * q + 1] << 16;
    a.y = hi[8 * q + 2] | (uint32_t)hi[8 * q + 3] << 16;
    a.z = hi[8 * q + 4] | (uint32_t)hi[8 * q + 5] << 16;
    a.w = hi[8 * q + 6] | (uint32_t)hi[8 * q + 7] << 16;
    b.x = lo[8 * q + 0] | (uint32_t)lo[8 * q + 1] << 16;
    b.y = lo[8 * q + 2] | (uint32_t)lo[8 * q + 3] << 16;
    b.z = lo[8 * q + 4] | (uint32_t)lo[8 * q + 5] << 16;
    b.w = lo[8 * q + 6] | (uint32_t)lo[8 * q + 7] << 16;
    *reinterpret_cast<uint4*>(dst + q * 512) = a;
    *reinterpret_cast<uint4*>(dst + MBP_RAW_UNIT_BYTES + q * 512) = b;
  }
}

bool shape_ok(int n, int k) { return n > 0 && k > 0 && n % 16 == 0 && k % 64 == 0 && k / 64 <= 32766; }
bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

constexpr int kWarpsPerCta = 8;

}  // namespace

extern "C" {

size_t mbp_pack_c12_workspace(int n, int k) {
  if (!shape_ok(n, k)) return 0;
  return (size_t)(n / 16) * 128 * sizeof(int);
}

int mbp_pack_c12(const uint16_t* w, int n, int k, int base_mode, uint8_t* units, uint8_t* bases, int32_t* esc_off,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!w || !units || !bases || !esc_off || !workspace) return MBP_ERR_ARG;
  if (base_mode != MBP_BASE_MATRIX && base_mode != MBP_BASE_TILE) return MBP_ERR_ARG;
  if (!shape_ok(n, k)) return MBP_ERR_SHAPE;
  if (!aligned16(w) || !aligned16(units)) return MBP_ERR_ALIGN;
  if (workspace_bytes < mbp_pack_c12_workspace(n, k)) return MBP_ERR_CAP;
  const int R = n / 16, C = k / 64;
  const long long NU = (long long)R * C;
  int* hist = static_cast<int*>(workspace);
  k_hist<<<R, 256, 0, stream>>>(w, k, hist);
  if (base_mode == MBP_BASE_TILE)
    k_bases<<<R, 128, 0, stream>>>(hist, R, 1, bases);
  else
    k_bases<<<1, 128, 0, stream>>>(hist, R, 0, bases);
  const unsigned blocks = (unsigned)((NU + kWarpsPerCta - 1) / kWarpsPerCta);
  k_pack<<<blocks, kWarpsPerCta * 32, 0, stream>>>(w, k, R, C, bases, units, esc_off);
  k_scan<<<1, 1024, 0, stream>>>(esc_off, NU);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_pack_c12_escapes(const uint16_t* w, int n, int k, const uint8_t* bases, const int32_t* esc_off,
                         uint32_t* esc, cudaStream_t stream) {
  if (!w || !bases || !esc_off) return MBP_ERR_ARG;
  if (!shape_ok(n, k)) return MBP_ERR_SHAPE;
  if (!aligned16(w)) return MBP_ERR_ALIGN;
  const int R = n / 16, C = k / 64;
  const long long NU = (long long)R * C;
  if (!esc) return MBP_OK;  // the caller found no escapes
  const unsigned blocks = (unsigned)((NU + kWarpsPerCta - 1) / kWarpsPerCta);
  k_escapes<<<blocks, kWarpsPerCta * 32, 0, stream>>>(w, k, R, C, bases, esc_off, esc);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_unpack_c12(const mbp_c12* p, uint16_t* w_out, cudaStream_t stream) {
  if (!p || !p->units || !p->bases || !p->esc_off || !w_out) return MBP_ERR_ARG;
  if (p->n_esc > 0 && !p->esc) return MBP_ERR_ARG;
  if (!shape_ok(p->n, p->k)) return MBP_ERR_SHAPE;
  if (!aligned16(p->units) || !aligned16(w_out)) return MBP_ERR_ALIGN;
  const int R = p->n / 16, C = p->k / 64;
  const long long NU = (long long)R * C;
  const unsigned blocks = (unsigned)((NU + kWarpsPerCta - 1) / kWarpsPerCta);
  k_unpack<<<blocks, kWarpsPerCta * 32, kWarpsPerCta * kMaskUnitBytes, stream>>>(p->units, p->bases, p->esc_off,
                                                                                 p->esc, R, C, p->k, w_out);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_pack_hilo(const float* w, int n, int k, uint8_t* units, cudaStream_t stream) {
  if (!w || !units) return MBP_ERR_ARG;
  if (!shape_ok(n, k)) return MBP_ERR_SHAPE;
  if (!aligned16(w) || !aligned16(units)) return MBP_ERR_ALIGN;
  const int R = n / 16, C = k / 64;
  const long long NU = (long long)R * C;
  const unsigned blocks = (unsigned)((NU + kWarpsPerCta - 1) / kWarpsPerCta);
  k_pack_hilo<<<blocks, kWarpsPerCta * 32, 0, stream>>>(w, k, R, C, units);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

}  // extern "C"

int mbp_status_pack(int* v, int clear) { return read_status_here(v, clear); }

// ------------------------------------------------------------------------------------------------------------
// Allocation-free packer.  Its scratch -- one 128-bin exponent histogram per 16-row tile -- is this fixed
// device array instead of a caller-provided workspace.  k_hist overwrites every entry it later reads, so
// nothing has to be cleared between calls; concurrent calls on one device would race on it.
// ------------------------------------------------------------------------------------------------------------
namespace {
constexpr int kNoAllocMaxTiles = 1024;  // n <= 16384 rows: 1024 tiles x 128 bins x 4 bytes = 512 KiB
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) int g_pack_scratch[kNoAllocMaxTiles * 128];

namespace {
std::mutex g_scratch_mu;
int* g_scratch_addr[kMaxDevices] = {};

// Device address of g_pack_scratch on the current device, looked up once per device.  In host code the
// array's name is only a host-side stand-in, so kernels must be given this address.
int scratch_on_current_device(int** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MBP_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return MBP_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_pack_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return MBP_ERR_LAUNCH;
    }
    g_scratch_addr[dev] = static_cast<int*>(p);
  }
  *out = g_scratch_addr[dev];
  return MBP_OK;
}
}  // namespace

extern "C" int mbp_pack_c12_noalloc(const uint16_t* w, int n, int k, int base_mode, uint8_t* units,
                                    uint8_t* bases, int32_t* esc_off, cudaStream_t stream) {
  if (!w || !units || !bases || !esc_off) return MBP_ERR_ARG;
  if (base_mode != MBP_BASE_MATRIX && base_mode != MBP_BASE_TILE) return MBP_ERR_ARG;
  if (!shape_ok(n, k)) return MBP_ERR_SHAPE;
  if (n / 16 > kNoAllocMaxTiles) return MBP_ERR_SCRATCH_LIMIT;
  if (!aligned16(w) || !aligned16(units)) return MBP_ERR_ALIGN;
  int* hist = nullptr;
  const int rc = scratch_on_current_device(&hist);
  if (rc != MBP_OK) return rc;
  const int R = n / 16, C = k / 64;
  const long long NU = (long long)R * C;
  k_hist<<<R, 256, 0, stream>>>(w, k, hist);
  if (base_mode == MBP_BASE_TILE)
    k_bases<<<R, 128, 0, stream>>>(hist, R, 1, bases);
  else
    k_bases<<<1, 128, 0, stream>>>(hist, R, 0, bases);
  const unsigned blocks = (unsigned)((NU + kWarpsPerCta - 1) / kWarpsPerCta);
  k_pack<<<blocks, kWarpsPerCta * 32, 0, stream>>>(w, k, R, C, bases, units, esc_off);
  k_scan<<<1, 1024, 0, stream>>>(esc_off, NU);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}
