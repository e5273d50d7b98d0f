// Fused gated residual + (Layer|RMS|no) norm + modulation + FP8 quantisation, one pass over HBM.
//
// Reference: adaln_quant_kernel (vllm_omni_neuron/kernels/nkilib/experimental/norm/adaln_quant.py:117-810)
// with the semantics of adaln_quant_torch_ref (adaln_quant_torch.py:41-175) and the bridge contract
// adaln_modulate (diffusion/quantization/adaln_kernels.py:87-201):
//     t    = residual + gate * hidden      (fp32 product and sum; t rounded to bf16 = residual_out)
//     xhat = LayerNorm(t) | RMSNorm(t) | t (fp32 statistics, two-pass mean/variance)
//     y    = xhat * mul + add              (mul/add in bf16, arithmetic fp32)
//     out  = bf16(y)                       (quant none)
//          | e4m3fn(y * (1/s)), s = max(amax/range, 1e-6), packed [H codes | 4 bytes fp32 s] (quant row)
//          | e4m3fn(y / 2^(e-127)), e = clip(max biased exponent of 32 values - 7, 0, 255)  (quant mx32)
//
// One 128-thread CTA per row; the row (<= 16384 values) stays in registers, 16-byte vector loads and
// stores, block reductions through shared memory. HBM-bound: every byte is read or written once.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

namespace vomni {
namespace adaln {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;

struct Params {
  const __nv_bfloat16* hidden;
  const __nv_bfloat16* residual;  // optional
  const __nv_bfloat16* mul;       // optional, [n_mod, H]
  const __nv_bfloat16* add;       // optional, [n_mod, H]
  const float* gate;              // optional, [n_mod, H]
  long long rows;
  int H;
  long long rows_per_mod;  // rows sharing one modulation row (the batch's tokens); huge = shared
  float eps;
  int norm;   // 0 layer, 1 rms, 2 none
  int quant;  // 0 none, 1 row, 2 mx32
  float fp8_range;
  int packed;       // row quant: 1 = [H + 4] packed rows, 0 = split codes [H] + scales [rows] fp32
  void* out;        // bf16 [rows, H] | u8 [rows, H+4] | u8 [rows, H]
  void* out_scale;  // row split: fp32 [rows]; mx32: u8 [rows, H/32]
  __nv_bfloat16* residual_out;  // optional
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide reduction; `red` holds kWarps floats. Ends with every thread holding the result.
template <bool kMax>
// One __syncthreads per reduction: each reduction of a row writes its own slot of `red`, and
// consecutive uses of one slot are always separated by another reduction's barrier.
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = kMax ? warp_max(v) : warp_sum(v);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kWarps; ++i) r = kMax ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __bfloat1622float2(p[i]);
    f[2 * i] = a.x;
    f[2 * i + 1] = a.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  return u;
}

VOMNI_DEV void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
VOMNI_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
VOMNI_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// NV = 16-byte chunks (8 values) per thread; a row holds up to NV * 128 * 8 values.
// Persistent: CTA c handles rows c, c + gridDim.x, ...; each thread streams its own chunks of the
// next kS-1 rows (hidden, and residual) into a kS-slot shared-memory ring with cp.async, so
// kS-1 rows per CTA are in flight while one is reduced; the modulation vectors stay in registers
// for as long as consecutive rows share them.
template <int NV, bool kRes, int kS>
__global__ void __launch_bounds__(kThreads, NV <= 6 ? 3 : 1) adaln_kernel(const Params p) {
  extern __shared__ uint4 ring[];  // [kS][H/8] hidden, then [kS][H/8] residual
  // Reduction slots, double-buffered by row parity: a row may take a single barrier, and a slot
  // is rewritten only two rows later, after every thread has passed the next row's barrier.
  __shared__ float red_sq[2][kWarps];       // LayerNorm sum / RMS sum of squares
  __shared__ float red_stat_v[2][kWarps];   // LayerNorm squared deviations
  __shared__ float red_max[2][kWarps];      // absmax for the row quant
  int parity = 0;
  const int H = p.H;
  const int nchunk = H >> 3;
  long long row = blockIdx.x;
  if (row >= p.rows) return;

  const long long G = gridDim.x;
  auto issue = [&](long long r, int slot) {
    if (r < p.rows) {
      const uint4* hp = reinterpret_cast<const uint4*>(p.hidden + static_cast<size_t>(r) * H);
      const uint4* rp = kRes ? reinterpret_cast<const uint4*>(p.residual + static_cast<size_t>(r) * H) : nullptr;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * kThreads;
        if (c < nchunk) {
          cp_async16(ring + slot * nchunk + c, hp + c);
          if (kRes) cp_async16(ring + (kS + slot) * nchunk + c, rp + c);
        }
      }
    }
    cp_async_commit();  // one group per row slot, empty past the end, so wait counts stay uniform
  };
#pragma unroll
  for (int s0 = 0; s0 < kS - 1; ++s0) issue(row + s0 * G, s0);
  int k = 0;
  long long cached_mrow = -1;
  uint4 mul_r[NV], add_r[NV];
  const uint4 one_bf16x8 = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);

  while (row < p.rows) {
    const long long next = row + G;
    const size_t base = static_cast<size_t>(row) * H;
    const long long mrow = row / p.rows_per_mod;
    issue(row + (kS - 1) * G, (k + kS - 1) % kS);  // refill the slot this thread finished with last row
    cp_async_wait<kS - 1>();                        // groups complete in order: this row has landed
    const int slot = k % kS;
    float x[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int cc = threadIdx.x + i * kThreads;
      if (cc < nchunk) unpack8(ring[slot * nchunk + cc], x[i]);
      if (kRes) {
        const int c = cc;
        float r[8];
        if (c < nchunk) unpack8(ring[(kS + slot) * nchunk + c], r);
        if (c < nchunk) {
          if (p.gate) {
            const float4* g = reinterpret_cast<const float4*>(p.gate + static_cast<size_t>(mrow) * H + c * 8);
            const float4 g0 = g[0], g1 = g[1];
            x[i][0] = __fmul_rn(x[i][0], g0.x); x[i][1] = __fmul_rn(x[i][1], g0.y);
            x[i][2] = __fmul_rn(x[i][2], g0.z); x[i][3] = __fmul_rn(x[i][3], g0.w);
            x[i][4] = __fmul_rn(x[i][4], g1.x); x[i][5] = __fmul_rn(x[i][5], g1.y);
            x[i][6] = __fmul_rn(x[i][6], g1.z); x[i][7] = __fmul_rn(x[i][7], g1.w);
          }
          // product and sum rounded separately (no FMA contraction), as the reference computes them
#pragma unroll
          for (int j = 0; j < 8; ++j) x[i][j] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(r[j], x[i][j])));
          reinterpret_cast<uint4*>(p.residual_out + base)[c] = pack8(x[i]);
        }
      }
      if (threadIdx.x + i * kThreads >= nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[i][j] = 0.f;
      }
    }
    if (mrow != cached_mrow) {
      cached_mrow = mrow;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * kThreads;
        mul_r[i] = (p.mul && c < nchunk) ? reinterpret_cast<const uint4*>(p.mul + static_cast<size_t>(mrow) * H)[c] : one_bf16x8;
        add_r[i] = (p.add && c < nchunk) ? reinterpret_cast<const uint4*>(p.add + static_cast<size_t>(mrow) * H)[c] : make_uint4(0, 0, 0, 0);
      }
    }
    // ---- statistics (fp32): per-thread two-pass mean / squared deviations, merged across the row
    const float invH = 1.f / static_cast<float>(H);
    float mean = 0.f, rstd = 1.f;
    if (p.norm == 0) {
      float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sm[j & 3] += x[i][j];
      mean = block_reduce<false>((sm[0] + sm[1]) + (sm[2] + sm[3]), red_sq[parity]) * invH;
      float m2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (threadIdx.x + i * kThreads < nchunk) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = x[i][j] - mean;
            m2[j & 3] = fmaf(d, d, m2[j & 3]);
          }
        }
      }
      rstd = rsqrtf(block_reduce<false>((m2[0] + m2[1]) + (m2[2] + m2[3]), red_stat_v[parity]) * invH + p.eps);
    } else if (p.norm == 1) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j & 3] = fmaf(x[i][j], x[i][j], v[j & 3]);
      rstd = rsqrtf(block_reduce<false>((v[0] + v[1]) + (v[2] + v[3]), red_sq[parity]) * invH + p.eps);
    }
    // ---- normalise + modulate (mul defaults to 1, add to 0)
    float am[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float m[8], a[8];
      unpack8(mul_r[i], m);
      unpack8(add_r[i], a);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float y = p.norm == 2 ? x[i][j] : (x[i][j] - mean) * rstd;
        y = fmaf(y, m[j], a[j]);
        x[i][j] = y;
        am[j & 3] = fmaxf(am[j & 3], fabsf(y));
      }
    }
    float amax = fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3]));
    // ---- quantise + store
    if (p.quant == 0) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * kThreads;
        if (c < nchunk) __stcs(reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + base) + c, pack8(x[i]));
      }
    } else if (p.quant == 1) {
      amax = block_reduce<true>(amax, red_max[parity]);
      const float scale = fmaxf(amax / p.fp8_range, 1e-6f);
      // codes = y * (1 / scale), the reciprocal-multiply of the reference kernel (adaln_quant.py:520-536)
      const float inv = __frcp_rn(scale);
      uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<size_t>(row) * (p.packed ? H + 4 : H);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * kThreads;
        if (c >= nchunk) continue;
        const uint32_t w0 = e4m3x2(x[i][0] * inv, x[i][1] * inv) | (static_cast<uint32_t>(e4m3x2(x[i][2] * inv, x[i][3] * inv)) << 16);
        const uint32_t w1 = e4m3x2(x[i][4] * inv, x[i][5] * inv) | (static_cast<uint32_t>(e4m3x2(x[i][6] * inv, x[i][7] * inv)) << 16);
        if (p.packed) {  // rows are only 4-byte aligned (H + 4 bytes)
          reinterpret_cast<uint32_t*>(orow + c * 8)[0] = w0;
          reinterpret_cast<uint32_t*>(orow + c * 8)[1] = w1;
        } else {
          __stcs(reinterpret_cast<uint2*>(orow) + c, make_uint2(w0, w1));
        }
      }
      if (threadIdx.x == 0) {
        if (p.packed)
          *reinterpret_cast<float*>(orow + H) = scale;
        else
          static_cast<float*>(p.out_scale)[row] = scale;
      }
    } else {  // mx32: a 32-value block = 4 consecutive chunks = 4 consecutive threads of one i
      uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<size_t>(row) * H;
      uint8_t* srow = static_cast<uint8_t*>(p.out_scale) + static_cast<size_t>(row) * (H >> 5);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * kThreads;
        int e = 0;
        if (c < nchunk) {
#pragma unroll
          for (int j = 0; j < 8; ++j) e = max(e, static_cast<int>((__float_as_uint(x[i][j]) >> 23) & 0xFF));
        }
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 1));
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 2));
        if (c >= nchunk) continue;
        const int su = min(max(e - 7, 0), 255);
        // y / 2^(su - 127) as two exact power-of-two multiplies (each factor a normal fp32).
        const int sh = 127 - su;  // in [-128, 127]
        const int sa = sh / 2, sb = sh - sa;
        const float fa = __uint_as_float(static_cast<uint32_t>(sa + 127) << 23);
        const float fb = __uint_as_float(static_cast<uint32_t>(sb + 127) << 23);
        float q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = fminf(fmaxf((x[i][j] * fa) * fb, -448.f), 448.f);
        const uint32_t w0 = e4m3x2(q[0], q[1]) | (static_cast<uint32_t>(e4m3x2(q[2], q[3])) << 16);
        const uint32_t w1 = e4m3x2(q[4], q[5]) | (static_cast<uint32_t>(e4m3x2(q[6], q[7])) << 16);
        reinterpret_cast<uint2*>(orow)[c] = make_uint2(w0, w1);
        if ((c & 3) == 0) srow[c >> 2] = static_cast<uint8_t>(su);
      }
    }
    row = next;
    parity ^= 1;
    ++k;
  }
  cp_async_wait<0>();  // no copy into shared memory may outlive the CTA
}

template <int NV, int kS>
int launch_s(const Params& p, cudaStream_t st) {
  // Persistent grid: as many CTAs as fit on the device at once, each streaming rows through its ring.
  auto kern = p.residual ? adaln_kernel<NV, true, kS> : adaln_kernel<NV, false, kS>;
  const size_t smem = static_cast<size_t>(kS) * p.H * 2 * (p.residual ? 2 : 1);
  int rc = ensure_max_smem(kern, static_cast<int>(smem));
  if (rc) return rc;
  int per_sm = 0;
  VOMNI_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  if (per_sm < 1) per_sm = 1;
  const long long cap = static_cast<long long>(num_sms()) * per_sm;
  const unsigned grid = static_cast<unsigned>(p.rows < cap ? p.rows : cap);
  kern<<<grid, kThreads, smem, st>>>(p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

// Four ring slots while they fit in 80 KB per CTA, else two.
template <int NV>
int launch(const Params& p, cudaStream_t st) {
  const size_t row_bytes = static_cast<size_t>(p.H) * 2 * (p.residual ? 2 : 1);
  return 4 * row_bytes <= 80 * 1024 ? launch_s<NV, 4>(p, st) : launch_s<NV, 2>(p, st);
}

}  // namespace adaln
}  // namespace vomni

using namespace vomni;

extern "C" int vomni_adaln_modulate(const void* hidden, const void* residual, const void* mul, const void* add,
                                    const float* gate, long long rows, int h, long long rows_per_mod, float eps,
                                    int norm_type, int quant, int ocp, int packed, void* out, void* out_scale,
                                    void* residual_out, vomni_stream_t stream) {
  if (!hidden || !out) return VOMNI_EINVAL;
  if (rows <= 0 || h <= 0 || h > 16384 || (h % 8)) return VOMNI_EBADSHAPE;
  if (rows > 0x7fffffffLL) return VOMNI_EBADSHAPE;
  if (norm_type < 0 || norm_type > 2 || quant < 0 || quant > 2) return VOMNI_EINVAL;
  if (quant == 2 && (h % 32)) return VOMNI_EBADSHAPE;
  if ((quant == 2 || (quant == 1 && !packed)) && !out_scale) return VOMNI_EINVAL;
  if (gate && !residual) return VOMNI_EINVAL;  // gate scales the sub-layer output before the residual add
  if (residual && !residual_out) return VOMNI_EINVAL;
  if (rows_per_mod <= 0) rows_per_mod = rows;
  const uintptr_t al = reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(residual) |
                       reinterpret_cast<uintptr_t>(mul) | reinterpret_cast<uintptr_t>(add) |
                       reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(residual_out);
  if (al & 15) return VOMNI_EALIGN;
  if ((reinterpret_cast<uintptr_t>(out) & (quant == 1 && packed ? 3 : 15))) return VOMNI_EALIGN;
  adaln::Params p;
  p.hidden = static_cast<const __nv_bfloat16*>(hidden);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.mul = static_cast<const __nv_bfloat16*>(mul);
  p.add = static_cast<const __nv_bfloat16*>(add);
  p.gate = gate;
  p.rows = rows;
  p.H = h;
  p.rows_per_mod = rows_per_mod;
  p.eps = eps;
  p.norm = norm_type;
  p.quant = quant;
  p.fp8_range = ocp ? 448.f : 240.f;
  p.packed = packed;
  p.out = out;
  p.out_scale = out_scale;
  p.residual_out = static_cast<__nv_bfloat16*>(residual_out);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int nv = (h / 8 + adaln::kThreads - 1) / adaln::kThreads;
  switch (nv) {
    case 1: return adaln::launch<1>(p, st);
    case 2: return adaln::launch<2>(p, st);
    case 3: return adaln::launch<3>(p, st);
    case 4: return adaln::launch<4>(p, st);
    case 5: return adaln::launch<5>(p, st);
    case 6: return adaln::launch<6>(p, st);
    case 7: return adaln::launch<7>(p, st);
    case 8: return adaln::launch<8>(p, st);
    case 9: return adaln::launch<9>(p, st);
    case 10: return adaln::launch<10>(p, st);
    case 11: return adaln::launch<11>(p, st);
    case 12: return adaln::launch<12>(p, st);
    case 13: return adaln::launch<13>(p, st);
    case 14: return adaln::launch<14>(p, st);
    case 15: return adaln::launch<15>(p, st);
    case 16: return adaln::launch<16>(p, st);
    default: return VOMNI_EBADSHAPE;
  }
}
