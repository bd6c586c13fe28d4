// Router consumer (no counterpart in the reference, which stops at the FP32 logits): per token, the k largest of
// the router's e logits and their softmax weights -- the expert selection a mixture-of-experts layer makes next.
//
//   mbp_router_topk   weights[t][j], ids[t][j] for j < k: ids in descending logit order (equal logits: the lower
//                     expert index first), weights = softmax over the k selected logits (renorm = 1) or the
//                     full softmax over all e logits, evaluated at the selected ones (renorm = 0).
//
// One warp per token: lane l holds logits l, l+32, ... (e/32 of them, e <= 1024); k rounds of a warp arg-max
// (value, then lower index; NaN ranks below every number), the winner marked as taken after each round.
// Launched as a programmatic dependent of the router GEMV, it waits for that grid before reading the logits.
#include <cfloat>
#include <cstdlib>

#include "common.cuh"

using namespace mbp;

namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kMaxPerLane = 32;  // e <= 1024

template <int PL>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) k_topk(const float* __restrict__ logits, int m, int e, int ld,
                                                               int k, int renorm, float* __restrict__ weights,
                                                               int32_t* __restrict__ ids) {
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= m) return;
  float v[PL];
  const float* row = logits + (size_t)t * ld;
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const int c = lane + 32 * i;
    const float x = c < e ? row[c] : -INFINITY;
    v[i] = x != x ? -INFINITY : x;  // NaN ranks below every number
  }
  uint32_t taken = 0;  // bit i: logit lane + 32*i already selected
  float top = 0.f, sel_v = 0.f;
  int sel_i = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int c = lane + 32 * i;
      if (c < e && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && c < bi))) {
        bv = v[i];
        bi = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (j == 0) top = bv;
    if (lane == j) {  // lane j keeps the j-th selection
      sel_v = bv;
      sel_i = bi;
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);  // the owner marks the winner
  }
  // weights: exp(l - top) normalised over the selection (renorm) or over every logit
  const float ex = lane < k ? expf(sel_v - top) : 0.f;
  float den = ex;
  if (!renorm) {
    den = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i)
      if (lane + 32 * i < e) den += expf(v[i] - top);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  if (lane < k) {
    weights[(size_t)t * k + lane] = ex / den;
    ids[(size_t)t * k + lane] = sel_i;
  }
}

template <int PL>
int launch_topk(const float* logits, int m, int e, int ld, int k, int renorm, float* w, int32_t* ids,
                cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((m + kWarpsPerBlock - 1) / kWarpsPerBlock);
  cfg.blockDim = dim3(32 * kWarpsPerBlock);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  static const bool pdl = getenv("MBP_NO_PDL") == nullptr;  // MBP_NO_PDL set: plain stream serialisation
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k_topk<PL>, logits, m, e, ld, k, renorm, w, ids) == cudaSuccess ? MBP_OK
                                                                                                  : MBP_ERR_LAUNCH;
}

}  // namespace

extern "C" int mbp_router_topk(const float* logits, int m, int e, int ld, int k, int renorm, float* weights,
                               int32_t* ids, cudaStream_t stream) {
  if (!logits || !weights || !ids) return MBP_ERR_ARG;
  if (m < 1) return MBP_ERR_M;
  if (e < 1 || e > 32 * kMaxPerLane || ld < e || k < 1 || k > 32 || k > e) return MBP_ERR_SHAPE;
  if (renorm != 0 && renorm != 1) return MBP_ERR_ARG;
  if (((uintptr_t)logits & 3u) || ((uintptr_t)weights & 3u) || ((uintptr_t)ids & 3u)) return MBP_ERR_ALIGN;
  const int pl = (e + 31) / 32;
  if (pl <= 8) return launch_topk<8>(logits, m, e, ld, k, renorm, weights, ids, stream);
  if (pl <= 16) return launch_topk<16>(logits, m, e, ld, k, renorm, weights, ids, stream);
  return launch_topk<32>(logits, m, e, ld, k, renorm, weights, ids, stream);
}

