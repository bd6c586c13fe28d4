// Helpers of the tensor-parallel layer (no counterpart in the reference, which is single-GPU).
//
//   mbp_tp_assemble_columns  all-gathered column shards [P][m][ns] (rank-major, what an NCCL all-gather into
//                            one buffer produces) -> the row-major projection output [m][P*ns]
//   mbp_f32_to_bf16          round-to-nearest-even conversion of the reduced FP32 partial sums of a
//                            row-parallel projection to the BF16 output
//
// Peer-store exchange (one node, NVLink peers mapped through CUDA IPC; plain loads and stores, no multicast):
//   mbp_ipc_alloc / mbp_ipc_open / mbp_ipc_close / mbp_ipc_free   exchange buffers and their cross-process
//                            mappings
//   mbp_tp_finish            the receive step of the two-kernel form (the one-kernel form, mbp_gemv_c12_tp,
//                            does the same inside the GEMV).  The sending GEMVs (mbp_gemv_c12_multi, tagged
//                            outputs) store
//                            64-bit words that carry the exchange's epoch in their upper half into every rank's
//                            buffer; the receive kernel polls its own buffer until each word it needs carries
//                            the epoch, then writes the assembled BF16 columns, or the rank-order sum of the P
//                            FP32 partials of a row-parallel projection (identical on every rank).  No fence or
//                            flag round trip: a system-scope fence costs several microseconds on this part, a
//                            tagged word arrives with its data.  MBP_TP_BARRIER is a plain flag barrier (system
//                            fence + release / acquire).  The epoch counter lives in device memory, so the
//                            exchange replays inside a CUDA graph.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

using namespace mbp;

namespace {

// One thread per 16-byte vector of 8 bf16; ns % 8 == 0.
__global__ void k_assemble(const uint4* __restrict__ src, uint4* __restrict__ dst, int P, int m, int ns8) {
  const long long total = (long long)P * m * ns8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % ns8);
    const long long rest = i / ns8;
    const int row = (int)(rest % m), r = (int)(rest / m);
    dst[(long long)row * P * ns8 + (long long)r * ns8 + j] = src[i];
  }
}

MBP_DEV uint32_t pack_bf16x2(float a, float b) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(a)) | (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16;
}

__global__ void k_f32_to_bf16(const float4* __restrict__ src, uint2* __restrict__ dst, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    dst[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

constexpr int kMaxRanks = 8;
constexpr int kSlots = MBP_TP_COUNTER_SLOTS;  // a receive launch has one block per epoch slot
constexpr int kRecvThreads = 1024;  // the receive of a 256-token exchange has ~400 K items for 64 blocks

struct TPFinish {
  int* flags[kMaxRanks];  // flags[r] = rank r's flag array (kMaxRanks ints), as mapped in this process
  int* counter;           // this rank's epoch slots (all equal between launches)
  const uint8_t* buf;     // this rank's exchange buffers: parity 0 at buf, parity 1 at buf + parity_stride
  long long parity_stride;
  void* out;
  int m, n;               // output [m][n]
  int rank, P, mode;
  unsigned long long wait_ns;  // limit of every bounded wait
};

MBP_DEV int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

MBP_DEV void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Flag barrier (one block; thread i < kSlots advances slot i).  Every rank writes the new epoch into its entry of
// every rank's flag array -- a system-scope release after a system fence, so this rank's earlier stores (stream
// order) are visible to a rank that sees the flag -- and waits, bounded, until its own array holds the epoch from
// every rank.
__global__ void __launch_bounds__(kSlots) k_tp_barrier(const __grid_constant__ TPFinish s) {
  const int l = threadIdx.x;
  const int e = s.counter[l] + 1;
  s.counter[l] = e;
  if (l < s.P) {
    __threadfence_system();
    st_release_sys(s.flags[l] + s.rank, e);
    const int* mine = s.flags[s.rank] + l;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(mine) < e) {
      if (globaltimer() - t0 > s.wait_ns) {
        set_status(MBP_DEV_TIMEOUT_PEER);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// Receive step of a tagged exchange.  Launched as a programmatic dependent of the GEMV that sends this rank's
// share, so it starts while that GEMV drains; it reads nothing the stream's earlier kernels write except the
// tagged words, whose tags it checks.  Block b advances epoch slot b when the GEMV has completed; the epoch's
// parity picks the buffer the GEMVs filled, so back-to-back exchanges and CUDA-graph
// replays alternate buffers on the device: a rank writes a buffer again only two epochs later, after every rank
// has finished reading it (its next receive needs this rank's words of the epoch in between, and a GEMV stores
// its words only after the receive kernel before it has completed).
__global__ void __launch_bounds__(kRecvThreads) k_tp_recv(const __grid_constant__ TPFinish s) {
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) epoch = (uint32_t)s.counter[blockIdx.x] + 1u;
  __syncthreads();
  const uint32_t e = epoch;
  const uint64_t* words = reinterpret_cast<const uint64_t*>(s.buf + (e & 1u) * s.parity_stride);
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  uint64_t t0 = 0;
  bool dead = false;
  if (s.mode == MBP_TP_GATHER_BF16) {
    // item = (token, 16-row tile): 8 words -> 16 bf16
    const int tiles = s.n / 16;
    const long long items = (long long)s.m * tiles;
    for (long long i = i0; i < items; i += stride) {
      const int t = (int)(i / tiles), tile = (int)(i - (long long)t * tiles);
      const uint64_t* w = words + (long long)t * (s.n / 2) + tile * 8;
      uint64_t v[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) v[g] = ld_relaxed_sys_u64(w + g);  // all eight before any check: one round trip
      uint32_t d[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if ((uint32_t)(v[g] >> 32) != e) v[g] = wait_tag(w + g, e, t0, dead, s.wait_ns);
        d[g] = (uint32_t)v[g];
      }
      uint4 lo, hi;
      lo.x = (d[0] & 0xffffu) | d[1] << 16;
      lo.y = (d[2] & 0xffffu) | d[3] << 16;
      lo.z = (d[4] & 0xffffu) | d[5] << 16;
      lo.w = (d[6] & 0xffffu) | d[7] << 16;
      hi.x = (d[0] >> 16) | (d[1] & 0xffff0000u);
      hi.y = (d[2] >> 16) | (d[3] & 0xffff0000u);
      hi.z = (d[4] >> 16) | (d[5] & 0xffff0000u);
      hi.w = (d[6] >> 16) | (d[7] & 0xffff0000u);
      uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(s.out) + (long long)t * s.n + tile * 16);
      o[0] = lo;
      o[1] = hi;
    }
  } else {
    // MBP_TP_SUM_F32: item = (token, 4 columns); P slots of [m][n] words added in rank order
    const int q4 = s.n / 4;
    const long long items = (long long)s.m * q4;
    for (long long i = i0; i < items; i += stride) {
      const int t = (int)(i / q4), c = (int)(i - (long long)t * q4) * 4;
      float a[4];
      const long long rs = (long long)s.m * s.n;
      const uint64_t* w0 = words + (long long)t * s.n + c;
      for (int r0 = 0; r0 < s.P; r0 += 2) {  // two ranks' four words before any check: one round trip per pair
        const int nr = s.P - r0 < 2 ? s.P - r0 : 2;
        uint64_t v[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (h < nr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[h][j] = ld_relaxed_sys_u64(w0 + (r0 + h) * rs + j);
          }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (h < nr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t* wj = w0 + (r0 + h) * rs + j;
              if ((uint32_t)(v[h][j] >> 32) != e) v[h][j] = wait_tag(wj, e, t0, dead, s.wait_ns);
              const float f = __uint_as_float((uint32_t)v[h][j]);
              a[j] = r0 + h == 0 ? f : a[j] + f;
            }
          }
      }
      reinterpret_cast<uint2*>(s.out)[i] = make_uint2(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]));
    }
  }
  // Every word has arrived: let the next kernel launch (a GEMV prefetches its first weights into L2, then waits
  // for this grid to complete before it reads its input, this output or the epoch).  Measured at 4 ranks: 400 us
  // per 16-call step against 405 us when triggered at the start of this kernel and 417 us at its exit.
  grid_dep_launch();
  // Advance this block's epoch slot only once the sending GEMV has completed: it reads slot 0 after its own
  // dependency wait but lets this grid start without ordering that read first.
  grid_dep_wait();
  if (threadIdx.x == 0) s.counter[blockIdx.x] = (int)e;
}

int blocks_for(long long work) {
  long long b = (work + 255) / 256;
  return (int)(b < 1 ? 1 : b > 4096 ? 4096 : b);
}

}  // namespace

extern "C" {

int mbp_tp_assemble_columns(const uint16_t* gathered, uint16_t* out, int P, int m, int ns, cudaStream_t stream) {
  if (!gathered || !out) return MBP_ERR_ARG;
  if (P < 1 || m < 1 || ns < 8 || ns % 8) return MBP_ERR_SHAPE;
  if (((uintptr_t)gathered & 15u) || ((uintptr_t)out & 15u)) return MBP_ERR_ALIGN;
  const int ns8 = ns / 8;
  k_assemble<<<blocks_for((long long)P * m * ns8), 256, 0, stream>>>(reinterpret_cast<const uint4*>(gathered),
                                                                      reinterpret_cast<uint4*>(out), P, m, ns8);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_f32_to_bf16(const float* in, uint16_t* out, long long n, cudaStream_t stream) {
  if (!in || !out) return MBP_ERR_ARG;
  if (n < 0 || n % 4) return MBP_ERR_SHAPE;
  if (((uintptr_t)in & 15u) || ((uintptr_t)out & 7u)) return MBP_ERR_ALIGN;
  if (n == 0) return MBP_OK;
  k_f32_to_bf16<<<blocks_for(n / 4), 256, 0, stream>>>(reinterpret_cast<const float4*>(in),
                                                        reinterpret_cast<uint2*>(out), n / 4);
  return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return MBP_ERR_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MBP_ERR_LAUNCH;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p) != cudaSuccess) {
    cudaFree(p);
    return MBP_ERR_LAUNCH;
  }
  *ptr = p;
  return MBP_OK;
}

int mbp_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return MBP_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_ipc_close(void* ptr) {
  if (!ptr) return MBP_ERR_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_ipc_free(void* ptr) {
  if (!ptr) return MBP_ERR_ARG;
  return cudaFree(ptr) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

int mbp_tp_finish(int* const* flags, int rank, int P, int* counter, const void* buf, long long parity_stride,
                  int mode, int m, int n, void* out, cudaStream_t stream) {
  if (!counter) return MBP_ERR_ARG;
  if (P < 1 || P > kMaxRanks || rank < 0 || rank >= P) return MBP_ERR_SHAPE;
  TPFinish s = {};
  s.counter = counter;
  s.rank = rank;
  s.P = P;
  s.mode = mode;
  s.wait_ns = wait_limit_ns();
  if (mode == MBP_TP_BARRIER) {
    if (!flags) return MBP_ERR_ARG;
    for (int r = 0; r < P; ++r) {
      if (!flags[r]) return MBP_ERR_ARG;
      s.flags[r] = flags[r];
    }
    k_tp_barrier<<<1, kSlots, 0, stream>>>(s);
    return cudaGetLastError() == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
  }
  if (mode != MBP_TP_GATHER_BF16 && mode != MBP_TP_SUM_F32) return MBP_ERR_ARG;
  if (!buf || !out) return MBP_ERR_ARG;
  if (m < 1 || n < 16 || n % 16 || parity_stride < 0) return MBP_ERR_SHAPE;
  if (((uintptr_t)buf & 15u) || (parity_stride & 15) || ((uintptr_t)out & 15u)) return MBP_ERR_ALIGN;
  s.buf = static_cast<const uint8_t*>(buf);
  s.parity_stride = parity_stride;
  s.out = out;
  s.m = m;
  s.n = n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kSlots);
  cfg.blockDim = dim3(kRecvThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  static const bool pdl = getenv("MBP_NO_PDL") == nullptr;  // MBP_NO_PDL set: plain stream serialisation
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k_tp_recv, s) == cudaSuccess ? MBP_OK : MBP_ERR_LAUNCH;
}

}  // extern "C"

int mbp_status_tp(int* v, int clear) { return read_status_here(v, clear); }
