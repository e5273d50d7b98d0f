// CFG-parallel combine: the elementwise half of _cfg_gather_combine
// (vllm_omni_neuron/diffusion/distributed/cfg_parallel.py:48-71). The two branch outputs arrive from
// the CFG group's all_gather (NCCL over NVLink, a few MB per denoising step); this kernel applies
// negative + scale * (positive - negative) with the rounding torch eager uses for the same
// expression, so the result equals sequential CFG bit for bit.
//
// HBM-bound: 3 streams of n elements, 16-byte vector accesses, a grid of a few CTAs per SM striding
// over the tensor; a scalar tail handles n not divisible by the vector width.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

namespace vomni {
namespace {

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// torch: sub, mul(Tensor, Scalar) and add each compute in fp32 opmath and round to the tensor dtype.
__device__ __forceinline__ float combine_bf16(float p, float n, float s) {
  const float d = bf16_round(__fsub_rn(p, n));
  const float m = bf16_round(__fmul_rn(s, d));
  return __fadd_rn(n, m);  // rounded by the caller's store
}
__device__ __forceinline__ float combine_f32(float p, float n, float s) {
  return __fadd_rn(n, __fmul_rn(s, __fsub_rn(p, n)));
}

__global__ void cfg_combine_bf16_kernel(const __nv_bfloat16* pos, const __nv_bfloat16* neg,
                                        __nv_bfloat16* out, long long n, float s) {
  const long long n8 = n / 8;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const uint4 a = reinterpret_cast<const uint4*>(pos)[i];
    const uint4 b = reinterpret_cast<const uint4*>(neg)[i];
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 r;
    __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 pa = __bfloat1622float2(a2[j]);
      const float2 nb = __bfloat1622float2(b2[j]);
      r2[j] = __floats2bfloat162_rn(combine_bf16(pa.x, nb.x, s), combine_bf16(pa.y, nb.y, s));
    }
    reinterpret_cast<uint4*>(out)[i] = r;
  }
  for (long long i = n8 * 8 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
    out[i] = __float2bfloat16_rn(combine_bf16(__bfloat162float(pos[i]), __bfloat162float(neg[i]), s));
}

__global__ void cfg_combine_f32_kernel(const float* pos, const float* neg, float* out,
                                       long long n, float s) {
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    const float4 a = reinterpret_cast<const float4*>(pos)[i];
    const float4 b = reinterpret_cast<const float4*>(neg)[i];
    reinterpret_cast<float4*>(out)[i] = make_float4(combine_f32(a.x, b.x, s), combine_f32(a.y, b.y, s),
                                                    combine_f32(a.z, b.z, s), combine_f32(a.w, b.w, s));
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
    out[i] = combine_f32(pos[i], neg[i], s);
}

}  // namespace
}  // namespace vomni

extern "C" int vomni_cfg_combine(const void* positive, const void* negative, void* out, long long n, int dtype,
                                 float scale, vomni_stream_t stream) {
  using namespace vomni;
  if (!positive || !negative || !out || n < 0) return VOMNI_EINVAL;
  if (dtype != VOMNI_CFG_F32 && dtype != VOMNI_CFG_BF16) return VOMNI_EINVAL;
  if (n == 0) return VOMNI_OK;
  const uintptr_t al = reinterpret_cast<uintptr_t>(positive) | reinterpret_cast<uintptr_t>(negative) |
                       reinterpret_cast<uintptr_t>(out);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  const int threads = 256;
  const long long vec = dtype == VOMNI_CFG_BF16 ? 8 : 4;
  long long blocks = (n / vec + threads - 1) / threads;
  const long long cap = static_cast<long long>(num_sms()) * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == VOMNI_CFG_BF16)
    cfg_combine_bf16_kernel<<<static_cast<int>(blocks), threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(positive), static_cast<const __nv_bfloat16*>(negative),
        static_cast<__nv_bfloat16*>(out), n, scale);
  else
    cfg_combine_f32_kernel<<<static_cast<int>(blocks), threads, 0, st>>>(
        static_cast<const float*>(positive), static_cast<const float*>(negative), static_cast<float*>(out), n, scale);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}
