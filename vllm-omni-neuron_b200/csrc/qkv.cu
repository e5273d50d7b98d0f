// FP8 (e4m3) fused QKV projection with the ROW scale epilogue, plus the across-heads RMS norm and
// rotate-half RoPE apply pass.
//
// Reference: qkv(quantization_type=ROW_MX) -> _qkv_cte_mx_impl
// (vllm_omni_neuron/kernels/nkilib/core/qkv/qkv_cte.py:2725-3993) as called by row_mx_qkv_proj
// (diffusion/quantization/row_mx_kernels.py:48-111):
//   Y = (Xq @ Wq) * row_scale[t] * chan_scale[i] + bias[i]          (_dequant_row_mx, :3996-4021)
//   sumsq_q[t] = sum over the Q segment of Y^2 (stored bf16 values), same for K (:3870-3898)
//   inv = rsqrt(sumsq / (n_heads * d) + eps)
//   Q/K <- rotate-half RoPE(Y * gamma) with inv folded in:
//          out = x*inv*cos + [-x_hi, x_lo]*inv*sin                  (_rope_segment, :4069-4114)
// The MX engine's identity micro-scales (common_types.py:77-78) make the ROW mode a plain FP8 GEMM.
//
// GEMM kernel: persistent, one CTA per SM walking 128 x 256 output tiles; warp 0 TMA producer
// (A [128 x 128 B] and B [256 x 128 B] boxes, 128-byte swizzle, 4-stage ring), warp 1 TMEM owner +
// tcgen05.mma kind::f8f6f4 issuer (M=128, N=256, K=32 per instruction) into one of two 256-column
// accumulators, warps 2-5 epilogue (TMEM -> registers, scales + bias, bf16 stores, per-row partial
// sums of squares) on the other accumulator.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

namespace vomni {
namespace qkv {

constexpr int kBM = 128, kBN = 256, kBK = 128;  // kBK in bytes (= fp8 elements)
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr uint32_t kABytes = kBM * kBK;  // 16 KB
constexpr uint32_t kBBytes = kBN * kBK;  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kSmemBar = kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;
constexpr uint32_t kIdesc = idesc_e4m3(kBM, kBN);

struct Params {
  int T, I, H;
  int m_tiles, n_tiles;
  const float* row_scale;   // [T]
  const float* chan_scale;  // [I]
  const __nv_bfloat16* bias;  // [I] or null
  __nv_bfloat16* y;           // [T, I]
  float* sumsq;               // [T, n_norm_tiles] or null
  int n_norm_tiles;           // output tiles covered by the Q and K segments
  int* status;
};

// Persistent: CTA c processes tiles c, c + gridDim.x, ... (n fastest, so the CTAs in flight share
// the A rows and walk the whole weight, which stays L2-resident). The two 256-column TMEM
// accumulators alternate between tiles, so the epilogue of tile i overlaps the main loop of i+1.
__global__ void __launch_bounds__(kThreads, 1)
    qkv_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.H / kBK;
  const int n_all = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0;  // global k-block counter across this CTA's tiles (stage ring position)
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_all; tile += gridDim.x) {
        const int m0 = (tile / p.n_tiles) * kBM;
        const int n0 = (tile % p.n_tiles) * kBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (it >= kStages && !mbar_wait(&empty[st], ph ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x21)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kStageBytes;
          mbar_expect_tx(&full[st], kStageBytes);
          tma_load_2d(&tmA, &full[st], sa, kb * kBK, m0);
          tma_load_2d(&tmB, &full[st], sa + kABytes, kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint64_t a_desc0 = make_sdesc(smem_u32(smem), 16, 1024, kLayoutSW128);
      uint32_t it = 0;
      int lt = 0;  // local tile index
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_all; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[acc], ((lt >> 1) & 1) ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x24)) break;
        tc_fence_after();
        const uint32_t tacc = tbase + acc * kBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[st], ph, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x22)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Start-address field advanced by integer adds (address >> 4; no carry below 256 KB).
          const uint64_t ad0 = a_desc0 + ((st * kStageBytes) >> 4);
          const uint64_t bd0 = ad0 + (kABytes >> 4);
#pragma unroll
          for (int k4 = 0; k4 < kBK / 32; ++k4)
            mma_f8_ss(tacc, ad0 + k4 * 2, bd0 + k4 * 2, kIdesc, (kb > 0 || k4 > 0) ? 1u : 0u);
          tc_commit(&empty[st]);
        }
        if (ok) tc_commit(&acc_full[acc]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    int lt = 0;
    for (int tile = blockIdx.x; tile < n_all; tile += gridDim.x, ++lt) {
      const int acc = lt & 1;
      if (!mbar_wait(&acc_full[acc], (lt >> 1) & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x23)) break;
      tc_fence_after();
      const int m0 = (tile / p.n_tiles) * kBM;
      const int nt = tile % p.n_tiles;
      const int n0 = nt * kBN;
      const int grow = m0 + row;
      const bool row_ok = grow < p.T;
      const uint32_t tacc = tbase + lane_addr + acc * kBN;
      const float rs = row_ok ? p.row_scale[grow] : 0.f;
      float ss = 0.f;
      __nv_bfloat16* yrow = p.y + static_cast<size_t>(grow) * p.I + n0;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tacc + c * 32, r);
        tmem_ld_wait(r);
        const int col0 = n0 + c * 32;
        const float4* cs4 = reinterpret_cast<const float4*>(p.chan_scale + col0);
        float v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 cs = cs4[i];
          v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) * rs * cs.x;
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) * rs * cs.y;
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) * rs * cs.z;
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) * rs * cs.w;
        }
        if (p.bias) {
          const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 bb = b4[i];
            const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bb);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(b2[j]);
              v[8 * i + 2 * j] += f.x;
              v[8 * i + 2 * j + 1] += f.y;
            }
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
          const float lo = __uint_as_float(pk[i] << 16), hi = __uint_as_float(pk[i] & 0xFFFF0000u);
          ss = fmaf(lo, lo, fmaf(hi, hi, ss));
        }
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(yrow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      // The accumulator has been read: the MMA warp may reuse it for tile lt + 2.
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (row_ok && p.sumsq && nt < p.n_norm_tiles) p.sumsq[static_cast<size_t>(grow) * p.n_norm_tiles + nt] = ss;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 2 * kBN);
  }
}

// [T, H + 4] packed rows (codes then fp32 scale; rows only 4-byte aligned) -> codes [T, H] + scale [T].
__global__ void unpack_rows_kernel(const uint8_t* __restrict__ packed, int T, int H, uint8_t* __restrict__ codes,
                                   float* __restrict__ scales) {
  const int row = blockIdx.x;
  if (row >= T) return;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(packed + static_cast<size_t>(row) * (H + 4));
  uint32_t* dst = reinterpret_cast<uint32_t*>(codes + static_cast<size_t>(row) * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
  if (threadIdx.x == 0) scales[row] = __uint_as_float(src[H / 4]);
}

// Across-heads RMS + gamma + rotate-half RoPE, in place on the Q and K segments of y [T, I].
// One CTA per token; a thread handles 8 consecutive lanes of one head's low half and the matching
// 8 lanes of its high half.
__global__ void qk_norm_rope_kernel(__nv_bfloat16* __restrict__ y, int T, int I, int q_heads, int kv_heads,
                                    const float* __restrict__ sumsq, int n_norm_tiles, int q_tiles, float eps,
                                    const __nv_bfloat16* __restrict__ gamma_q, const __nv_bfloat16* __restrict__ gamma_k,
                                    const float* __restrict__ cos, const float* __restrict__ sin) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ float inv_s[2];
  if (threadIdx.x < 2) {
    const int lo = threadIdx.x == 0 ? 0 : q_tiles;
    const int hi = threadIdx.x == 0 ? q_tiles : n_norm_tiles;
    float s = 0.f;
    for (int i = lo; i < hi; ++i) s += sumsq[static_cast<size_t>(t) * n_norm_tiles + i];
    const int n = threadIdx.x == 0 ? q_heads : kv_heads;
    inv_s[threadIdx.x] = n > 0 ? rsqrtf(s / static_cast<float>(n * 128) + eps) : 1.f;
  }
  __syncthreads();
  const int units = (q_heads + kv_heads) * 8;  // 8 groups of 8 lanes per head half
  __nv_bfloat16* yr = y + static_cast<size_t>(t) * I;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int head = u >> 3;
    const int g = u & 7;
    const bool is_q = head < q_heads;
    const float inv = inv_s[is_q ? 0 : 1];
    const __nv_bfloat16* gamma = is_q ? gamma_q : gamma_k;
    const int hcol = is_q ? head * 128 : (head - q_heads) * 128;  // column within the segment
    __nv_bfloat16* xp = yr + head * 128 + g * 8;
    uint4 lo_u = *reinterpret_cast<const uint4*>(xp);
    uint4 hi_u = *reinterpret_cast<const uint4*>(xp + 64);
    float xl[8], xh[8];
    {
      const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&lo_u);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&hi_u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(a[j]), fb = __bfloat1622float2(b[j]);
        xl[2 * j] = fa.x; xl[2 * j + 1] = fa.y;
        xh[2 * j] = fb.x; xh[2 * j + 1] = fb.y;
      }
    }
    if (gamma) {
      const uint4 gl = *reinterpret_cast<const uint4*>(gamma + hcol + g * 8);
      const uint4 gh = *reinterpret_cast<const uint4*>(gamma + hcol + 64 + g * 8);
      const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&gl);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&gh);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(a[j]), fb = __bfloat1622float2(b[j]);
        xl[2 * j] = __bfloat162float(__float2bfloat16_rn(xl[2 * j] * fa.x));
        xl[2 * j + 1] = __bfloat162float(__float2bfloat16_rn(xl[2 * j + 1] * fa.y));
        xh[2 * j] = __bfloat162float(__float2bfloat16_rn(xh[2 * j] * fb.x));
        xh[2 * j + 1] = __bfloat162float(__float2bfloat16_rn(xh[2 * j + 1] * fb.y));
      }
    }
    float ol[8], oh[8];
    if (cos) {
      const float* cr = cos + static_cast<size_t>(t) * 128;
      const float* sr = sin + static_cast<size_t>(t) * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = g * 8 + j;
        const float s = sr[d] * inv;
        ol[j] = xl[j] * inv * cr[d] - xh[j] * s;
        oh[j] = xh[j] * inv * cr[64 + d] + xl[j] * s;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ol[j] = xl[j] * inv;
        oh[j] = xh[j] * inv;
      }
    }
    uint32_t pl[4], ph[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pl[j] = pack_bf16x2(ol[2 * j], ol[2 * j + 1]);
      ph[j] = pack_bf16x2(oh[2 * j], oh[2 * j + 1]);
    }
    *reinterpret_cast<uint4*>(xp) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    *reinterpret_cast<uint4*>(xp + 64) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
  }
}

}  // namespace qkv
}  // namespace vomni

using namespace vomni;

extern "C" int vomni_qkv_unpack_rows(const void* packed, int t, int h, void* codes, float* scales,
                                     vomni_stream_t stream) {
  if (!packed || !codes || !scales) return VOMNI_EINVAL;
  if (t <= 0 || h <= 0 || (h % 16)) return VOMNI_EBADSHAPE;
  if (reinterpret_cast<uintptr_t>(packed) & 3 || reinterpret_cast<uintptr_t>(codes) & 15) return VOMNI_EALIGN;
  qkv::unpack_rows_kernel<<<t, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(packed), t, h, static_cast<uint8_t*>(codes), scales);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_qkv_fp8_gemm(const void* x_codes, const float* row_scale, const void* w_codes,
                                  const float* chan_scale, const void* bias, int t, int h, int i, int q_dim,
                                  int kv_dim, void* y, float* sumsq, vomni_stream_t stream) {
  if (!x_codes || !row_scale || !w_codes || !chan_scale || !y) return VOMNI_EINVAL;
  if (t <= 0 || h <= 0 || i <= 0 || (h % qkv::kBK) || (i % qkv::kBN)) return VOMNI_EBADSHAPE;
  if (q_dim < 0 || kv_dim < 0 || q_dim + kv_dim > i || (q_dim % qkv::kBN) || (kv_dim % qkv::kBN)) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(x_codes) | reinterpret_cast<uintptr_t>(w_codes) |
                       reinterpret_cast<uintptr_t>(chan_scale) | reinterpret_cast<uintptr_t>(bias) |
                       reinterpret_cast<uintptr_t>(y);
  if (al & 15) return VOMNI_EALIGN;
  if (static_cast<long long>(t + qkv::kBM - 1) / qkv::kBM > 0x7fffffffLL) return VOMNI_EBADSHAPE;
  int rc = require_sm100();
  if (rc) return rc;
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_codes, h, t, h, qkv::kBK, qkv::kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, h, i, h, qkv::kBK, qkv::kBN);
  if (rc) return rc;
  qkv::Params p;
  p.T = t;
  p.I = i;
  p.H = h;
  p.row_scale = row_scale;
  p.chan_scale = chan_scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.sumsq = sumsq;
  p.n_norm_tiles = (q_dim + kv_dim) / qkv::kBN;
  p.m_tiles = (t + qkv::kBM - 1) / qkv::kBM;
  p.n_tiles = i / qkv::kBN;
  p.status = device_status_ptr();
  static bool attr = false;
  if (!attr) {
    VOMNI_CUDA_TRY(cudaFuncSetAttribute(qkv::qkv_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, qkv::kSmemBytes));
    attr = true;
  }
  const int n_all = p.m_tiles * p.n_tiles;
  const int grid = n_all < num_sms() ? n_all : num_sms();
  qkv::qkv_gemm_kernel<<<grid, qkv::kThreads, qkv::kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_qk_norm_rope(void* y, int t, int i, int q_heads, int kv_heads, int head_dim, const float* sumsq,
                                  float eps, const void* gamma_q, const void* gamma_k, const float* cos,
                                  const float* sin, vomni_stream_t stream) {
  if (!y || !sumsq) return VOMNI_EINVAL;
  if (head_dim != 128 || t <= 0 || q_heads < 0 || kv_heads < 0) return VOMNI_EBADSHAPE;
  const int q_dim = q_heads * 128, kv_dim = kv_heads * 128;
  if (q_dim + kv_dim > i || (q_dim % qkv::kBN) || (kv_dim % qkv::kBN)) return VOMNI_EBADSHAPE;
  if ((cos == nullptr) != (sin == nullptr)) return VOMNI_EINVAL;
  const uintptr_t al = reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gamma_q) |
                       reinterpret_cast<uintptr_t>(gamma_k);
  if (al & 15 || (i % 8)) return VOMNI_EALIGN;
  qkv::qk_norm_rope_kernel<<<t, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(y), t, i, q_heads, kv_heads, sumsq, (q_dim + kv_dim) / qkv::kBN, q_dim / qkv::kBN,
      eps, static_cast<const __nv_bfloat16*>(gamma_q), static_cast<const __nv_bfloat16*>(gamma_k), cos, sin);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}
