// Helpers of the tensor-parallel layer (no counterpart in the reference, which is single-GPU).
//
//   mbp_tp_assemble_columns  all-gathered column shards [P][m][ns] (rank-major, what an NCCL all-gather into
//                            one buffer produces) -> the row-major projection output [m][P*ns]
//   mbp_f32_to_bf16          round-to-nearest-even conversion of the reduced FP32 partial sums of a
//                            row-parallel projection to the BF16 output
#include "common.cuh"

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

__global__ void k_f32_to_bf16(const float4* __restrict__ src, uint2* __restrict__ dst, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(v.x)) | (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v.y)) << 16;
    const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(v.z)) | (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v.w)) << 16;
    dst[i] = make_uint2(a, b);
  }
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

}  // extern "C"
