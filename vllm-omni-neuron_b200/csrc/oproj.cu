// Output projection of the Wan self-attention with the block's norm2 gated residual fused in.
//
// Reference: _wan_o_proj (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:246-254):
//   x = active.reshape(B, N*D, S).transpose(1, 2);  y = x @ W + b      (bf16 tensors, fp32 accumulate)
// consumed by the block's norm2 (:1470-1489):
//   hidden_states, norm_h = adaln_modulate(y, ..., residual=hidden_states, gate=gate_msa)
// whose residual step is t = bf16(residual + gate * y) (fp32 product; adaln_kernels.py:51-84).
// torch rounds the matmul to bf16 before the bias add, and the sum again: y = bf16(bf16(acc) + b).
//
// B200 kernel: the d-major attention output [B, N*D, S] is read in place as an MN-major A operand
// (tokens contiguous) and W [N*D, H] as an MN-major B operand, both by TMA with 128-byte swizzle, so
// neither the reference's transpose nor a weight repack is needed. CTA pairs share each
// tcgen05.mma (cta_group::2, M=256 tokens, N=256 columns, K=16): each CTA stages its 128 tokens and
// its 128 output columns per 64-deep k-block (32 KB per stage, six stages). The epilogue rounds as
// torch does, adds the bias, and with a residual writes t = bf16(residual + gate * y) instead of y,
// so norm2 reads t once (the adaLN kernel then runs without its residual step).
//
// The same kernel with a K-major A operand (token rows, [M, K] row-major) and a GELU-tanh epilogue
// runs the Wan FFN: _wan_mlp (wan2_2_transformer.py:389-410) = GELU_tanh(x @ Wu + bu) @ Wd + bd, each
// step rounded to bf16 as torch does (the GELU in fp32 opmath on the bf16 input).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

namespace vomni {
namespace oproj {

constexpr int kThreads = 192;
constexpr int kStages = 6;
constexpr int kBK = 64;                              // K rows per stage (bf16)
constexpr uint32_t kChunkBytes = kBK * 128;          // 8 KB: 64 K rows x 64 contiguous elements
constexpr uint32_t kABytes = 2 * kChunkBytes;        // this CTA's 128 tokens
constexpr uint32_t kBBytes = 2 * kChunkBytes;        // this CTA's 128 output columns
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // 32 KB
constexpr uint32_t kSmemBar = kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;
constexpr uint32_t kIdescMN = idesc_bf16_mn(256, 256, true, true);   // A MN-major (d-major attention)
constexpr uint32_t kIdescK = idesc_bf16_mn(256, 256, false, true);   // A K-major (token rows)
// Epilogues: bias; bias + gated residual; bias + GELU-tanh; bias + per-head sums of squares of the
// stored bf16 values (the input of the across-heads RMS norm, like the FP8 QKV GEMM's).
enum Epi { EPI_BIAS = 0, EPI_RESIDUAL = 1, EPI_GELU = 2, EPI_SUMSQ = 3 };
constexpr int kGroup = 8;

struct Params {
  int B, S, K, H;
  int m_bands;  // ceil(S / 256) per batch element
  int n_tiles;  // H / 256
  const __nv_bfloat16* bias;      // [H] or null
  const __nv_bfloat16* residual;  // [B, S, H] or null
  const float* gate;              // [B, H] or [H] (gate_per_batch = 0) or null
  int gate_per_batch;
  int gate_rows;  // > 0: gate row = output row / gate_rows (rows of one batch element in a flat [M, H])
  float* sumsq;       // EPI_SUMSQ: [M, n_norm_heads]
  int n_norm_heads;   // 128-column heads covered by sumsq (the Q and K segments)
  __nv_bfloat16* out;  // [B, S, H]
  int* status;
};

struct Tile {
  int b, mb, nb;
};
// Pair tile t -> (batch, 256-token band, 256-column block); column-major inside groups of kGroup
// bands so the pairs in flight share A bands and W column blocks in L2.
VOMNI_DEV Tile tile_of(int t, const Params& p) {
  const int bands = p.B * p.m_bands;
  const int per_group = kGroup * p.n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int rows = min(kGroup, bands - g * kGroup);
  const int band = g * kGroup + r % rows;
  return Tile{band / p.m_bands, band % p.m_bands, r / rows};
}

// GELU-tanh (gelu_tanh in common.cuh): 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3))), fp32.

// kAK: A is K-major ([M, K] rows, one 128-row box of 64 k per stage) instead of MN-major.
template <bool kAK, int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2], in the leader: one arrival per epilogue warp of the pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int nk = p.K / kBK;
  const int n_all = p.B * p.m_bands * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lead_full = mapa_shared(smem_u32(full), 0);
  const uint32_t lead_acc_empty = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < n_all; tile += n_pairs) {
        const Tile tt = tile_of(tile, p);
        const int tok0 = tt.mb * 256 + static_cast<int>(rank) * 128;
        const int n0 = tt.nb * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (it >= kStages && !mbar_wait(&empty[st], ph ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x61)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kStageBytes;
          const uint32_t bar = lead_full + st * 8;
          if (leader) mbar_expect_tx(&full[st], 2 * kStageBytes);
          if (kAK) {
            tma_load_2d_pair(&tmA, bar, sa, kb * kBK, tok0);
          } else {
            tma_load_3d_pair(&tmA, bar, sa, tok0, kb * kBK, tt.b);
            tma_load_3d_pair(&tmA, bar, sa + kChunkBytes, tok0 + 64, kb * kBK, tt.b);
          }
          tma_load_2d_pair(&tmB, bar, sa + kABytes, n0, kb * kBK);
          tma_load_2d_pair(&tmB, bar, sa + kABytes + kChunkBytes, n0 + 64, kb * kBK);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // MN-major SW128 operands: 64-element chunks kChunkBytes apart (LBO), 8-row K groups 1 KB
      // apart (SBO); one K=16 step = 16 rows = +2 KB. K-major A: 128-byte rows of 64 k, 8-row
      // groups 1 KB apart; one K=16 step = +32 B inside the swizzled row.
      const uint64_t a_desc0 = kAK ? make_sdesc(smem_u32(smem), 16, 1024, kLayoutSW128)
                                   : make_sdesc(smem_u32(smem), kChunkBytes, 1024, kLayoutSW128);
      const uint64_t b_desc0 = make_sdesc(smem_u32(smem + kABytes), kChunkBytes, 1024, kLayoutSW128);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < n_all; tile += n_pairs, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[acc], ((lt >> 1) & 1) ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x64)) break;
        tc_fence_after();
        const uint32_t tacc = tbase + acc * 256;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[st], ph, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x62)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad0 = a_desc0 + ((st * kStageBytes) >> 4);
          const uint64_t bd0 = b_desc0 + ((st * kStageBytes) >> 4);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_ss_pair(tacc, ad0 + ((k * (kAK ? 32 : 2048)) >> 4), bd0 + ((k * 2048) >> 4), kAK ? kIdescK : kIdescMN,
                            (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(&empty[st]);
        }
        if (ok) tc_commit_pair(&acc_full[acc]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    int lt = 0;
    for (int tile = pair; tile < n_all; tile += n_pairs, ++lt) {
      const int acc = lt & 1;
      if (!mbar_wait(&acc_full[acc], (lt >> 1) & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x63)) break;
      tc_fence_after();
      const Tile tt = tile_of(tile, p);
      const int tok = tt.mb * 256 + static_cast<int>(rank) * 128 + row;
      const bool row_ok = tok < p.S;
      const int n0 = tt.nb * 256;
      const size_t orow = (static_cast<size_t>(tt.b) * p.S + tok) * p.H;
      const size_t grow_g = p.gate_rows > 0 ? static_cast<size_t>(tok / p.gate_rows) : (p.gate_per_batch ? tt.b : 0);
      const float* gate = p.gate ? p.gate + grow_g * p.H : nullptr;
      const uint32_t tacc = tbase + lane_addr + acc * 256;
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t r[32];
        tmem_ld32(tacc + c * 32, r);
        tmem_ld_wait(r);
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.H) continue;  // rows past S, columns past H (H % 32 == 0)
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[i])));  // torch matmul out
        if (p.bias) {
          const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 bb = b4[i];
            const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bb);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(b2[j]);
              v[8 * i + 2 * j] = __bfloat162float(__float2bfloat16_rn(v[8 * i + 2 * j] + f.x));
              v[8 * i + 2 * j + 1] = __bfloat162float(__float2bfloat16_rn(v[8 * i + 2 * j + 1] + f.y));
            }
          }
        }
        if (kEpi == EPI_GELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
        }
        if (kEpi == EPI_RESIDUAL && p.residual) {
          const uint4* r4 = reinterpret_cast<const uint4*>(p.residual + orow + col0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 rr = r4[i];
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(r2[j]);
              const int e = 8 * i + 2 * j;
              const float g0 = gate ? gate[col0 + e] : 1.f, g1 = gate ? gate[col0 + e + 1] : 1.f;
              v[e] = __fadd_rn(f.x, __fmul_rn(v[e], g0));  // separate roundings, as the reference
              v[e + 1] = __fadd_rn(f.y, __fmul_rn(v[e + 1], g1));
            }
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(p.out + orow + col0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                              pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
        if (kEpi == EPI_SUMSQ) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float q = __bfloat162float(__float2bfloat16_rn(v[i]));  // the stored value
            ss = fmaf(q, q, ss);
          }
          const int head = col0 / 128;
          if ((c & 3) == 3) {  // one 128-column head done
            if (p.sumsq && head < p.n_norm_heads) p.sumsq[static_cast<size_t>(tok) * p.n_norm_heads + head] = ss;
            ss = 0.f;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty + acc * 8);
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
}


// ---------------------------------------------------------------- FP8 (ROW) o-projection input
// row_mx_o_proj (diffusion/quantization/row_mx_kernels.py:114-138) quantises the d-major attention
// output inside its NKI kernel, one scale per token over the token's N*D values (ROW), then runs the
// FP8 GEMM. This kernel does the quantisation with the ROW rule of the in-tree NKI ROW quantiser
// (scale = max(amax / 448, 1e-6), codes = e4m3fn(x * (1 / scale)), adaln_quant.py:520-536) and
// writes token rows, so the FP8 ROW GEMM of the QKV projection consumes them unchanged.
// A cluster of kCR CTAs owns 32 consecutive tokens of one batch element; CTA r of the cluster holds
// rows [r*K/kCR, (r+1)*K/kCR) of those tokens in shared memory (TMA boxes of 32 tokens x up to 256
// rows, 64-byte rows, zero-filled past the sequence end), so the activation crosses HBM once. Each CTA
// reduces its rows' per-token |max|, the cluster merges the kCR partials through distributed shared
// memory, and each CTA converts its rows into 32-byte runs of the tokens' code rows.
constexpr int kRqTok = 32;          // tokens per cluster: one 64-byte box row
constexpr int kRqThreads = 256;     // 8 warps; lane = token
constexpr int kRqWarps = kRqThreads / 32;
constexpr int kRqMaxRows = 2048;    // K rows per CTA (128 KB of shared memory)
constexpr int kSiteRqLoad = 0x40;   // the CTA's tile loads never completed

VOMNI_DEV float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <int kCR>
__global__ void __cluster_dims__(kCR, 1, 1) __launch_bounds__(kRqThreads)
    oproj_rowquant_kernel(const __grid_constant__ CUtensorMap tm, int K, int S, int box_rows, uint8_t* __restrict__ codes,
                          float* __restrict__ scales, int* status) {
  extern __shared__ __align__(128) __nv_bfloat16 tile[];  // [R][32] bf16
  __shared__ __align__(8) uint64_t full;
  __shared__ float red[kRqWarps][kRqTok];
  __shared__ float part[kRqTok];  // this CTA's per-token |max|, read by the whole cluster
  __shared__ float sinv[kRqTok];
  __shared__ int abort_flag;
  const int rank = static_cast<int>(cluster_ctarank());
  const int t0 = (blockIdx.x / kCR) * kRqTok;
  const int b = blockIdx.y;
  const int R = K / kCR;
  const int k0 = rank * R;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(&full, static_cast<uint32_t>(R) * kRqTok * 2u);
    for (int r = 0; r < R; r += box_rows) tma_load_3d(&tm, &full, tile + r * kRqTok, t0, k0 + r, b);
  }
  const bool loaded = mbar_wait(&full, 0, &abort_flag, status, VOMNI_DEV_TIMEOUT_BASE + kSiteRqLoad);
  // pass 1: per-token |max| of this CTA's rows on packed bf16 pairs (max of bf16 values is exact).
  // Half-warp h reads rows 2i + h (32-byte rows of 16 token pairs: the two halves hit disjoint banks),
  // lane l of it the token pair (2l, 2l + 1); warps stride the row pairs.
  {
    const int hw = lane >> 4, pr = lane & 15;
    const __nv_bfloat162* t2 = reinterpret_cast<const __nv_bfloat162*>(tile);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.f);
    for (int r = 2 * warp + hw; r < R; r += 2 * kRqWarps) m2 = __hmax2(m2, __habs2(t2[r * (kRqTok / 2) + pr]));
    float lo = __low2float(m2), hi = __high2float(m2);
    lo = fmaxf(lo, __shfl_xor_sync(0xffffffffu, lo, 16));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, 16));
    if (hw == 0) {
      red[warp][2 * pr] = lo;
      red[warp][2 * pr + 1] = hi;
    }
  }
  __syncthreads();
  if (threadIdx.x < kRqTok) {
    float a = red[0][lane];
#pragma unroll
    for (int w = 1; w < kRqWarps; ++w) a = fmaxf(a, red[w][lane]);
    part[lane] = a;
  }
  cluster_sync();  // every CTA's partials are visible to the cluster
  if (threadIdx.x < kRqTok) {
    float a = 0.f;
#pragma unroll
    for (int q = 0; q < kCR; ++q) a = fmaxf(a, ld_shared_cluster_f32(mapa_shared(smem_u32(&part[lane]), q)));
    const float scale = fmaxf(a / 448.f, 1e-6f);
    sinv[lane] = __frcp_rn(scale);
    if (rank == 0 && t0 + lane < S) scales[static_cast<size_t>(b) * S + t0 + lane] = scale;
  }
  __syncthreads();
  // pass 2: lane = token; a warp turns 32 consecutive rows into one 32-byte run of each token's codes
  const float inv = sinv[lane];
  const bool tok_ok = t0 + lane < S;
  uint8_t* crow = codes + (static_cast<size_t>(b) * S + t0 + lane) * K + k0;
  for (int c = warp; c * 32 < R; c += kRqWarps) {
    const int nrow = min(32, R - c * 32);  // 32, or 16 in a last chunk (K % 64 == 0)
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = c * 32 + 4 * j;
      if (4 * j < nrow) {
        const float x0 = __bfloat162float(tile[(r + 0) * kRqTok + lane]) * inv;
        const float x1 = __bfloat162float(tile[(r + 1) * kRqTok + lane]) * inv;
        const float x2 = __bfloat162float(tile[(r + 2) * kRqTok + lane]) * inv;
        const float x3 = __bfloat162float(tile[(r + 3) * kRqTok + lane]) * inv;
        w[j] = e4m3x2(x0, x1) | (static_cast<uint32_t>(e4m3x2(x2, x3)) << 16);
      } else {
        w[j] = 0;
      }
    }
    if (tok_ok) {
      uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
      __stcs(dst, make_uint4(w[0], w[1], w[2], w[3]));
      if (nrow > 16) __stcs(dst + 1, make_uint4(w[4], w[5], w[6], w[7]));
    }
  }
  // A CTA whose loads gave up waits once more (bounded) so that no copy into its shared memory
  // outlives it; every CTA keeps its partials alive until the whole cluster has read them.
  if (!loaded && threadIdx.x == 0) {
    int ignored = 0;
    mbar_wait(&full, 0, &ignored, status, VOMNI_DEV_TIMEOUT_BASE + kSiteRqLoad);
  }
  cluster_sync();
}

int ensure_smem_attr() {
  // once per kernel and device (ensure_max_smem caches)
  int rc = 0;
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<false, EPI_BIAS>, kSmemBytes);
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<false, EPI_RESIDUAL>, kSmemBytes);
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<true, EPI_BIAS>, kSmemBytes);
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<true, EPI_GELU>, kSmemBytes);
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<true, EPI_RESIDUAL>, kSmemBytes);
  if (!rc) rc = ensure_max_smem(gemm_bf16_pair_kernel<true, EPI_SUMSQ>, kSmemBytes);
  return rc;
}

}  // namespace oproj
}  // namespace vomni

using namespace vomni;

extern "C" int vomni_oproj_gemm(const void* attn, int b, int k, int s, const void* w, const void* bias, int h,
                                const void* residual, const float* gate, int gate_per_batch, void* out,
                                vomni_stream_t stream) {
  if (!attn || !w || !out) return VOMNI_EINVAL;
  if (gate && !residual) return VOMNI_EINVAL;
  if (b <= 0 || s <= 0 || k <= 0 || h <= 0 || (k % oproj::kBK) || (h % 32)) return VOMNI_EBADSHAPE;
  if ((s % 8) || b > 65535) return VOMNI_EBADSHAPE;  // token rows of the d-major input must be 16-byte pitched
  const uintptr_t al = reinterpret_cast<uintptr_t>(attn) | reinterpret_cast<uintptr_t>(w) |
                       reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(residual) |
                       reinterpret_cast<uintptr_t>(out);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  CUtensorMap ta, tb;
  rc = make_tmap_3d_bf16(&ta, attn, static_cast<uint64_t>(s), static_cast<uint64_t>(k), static_cast<uint64_t>(b), 64, 64, 0);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, static_cast<uint64_t>(h), static_cast<uint64_t>(k),
                    static_cast<uint64_t>(h) * 2, 64, 64);
  if (rc) return rc;
  oproj::Params p;
  p.B = b;
  p.S = s;
  p.K = k;
  p.H = h;
  p.m_bands = (s + 255) / 256;
  p.n_tiles = (h + 255) / 256;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.gate = gate;
  p.gate_per_batch = gate_per_batch ? 1 : 0;
  p.gate_rows = 0;
  p.sumsq = nullptr;
  p.n_norm_heads = 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.status = device_status_ptr();
  const long long tiles = static_cast<long long>(b) * p.m_bands * p.n_tiles;
  const int pairs = static_cast<int>(tiles < num_sms() / 2 ? tiles : num_sms() / 2);
  rc = oproj::ensure_smem_attr();
  if (rc) return rc;
  auto kern = residual ? oproj::gemm_bf16_pair_kernel<false, oproj::EPI_RESIDUAL>
                       : oproj::gemm_bf16_pair_kernel<false, oproj::EPI_BIAS>;
  kern<<<2 * pairs, oproj::kThreads, oproj::kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_oproj_rowquant(const void* attn, int b, int k, int s, void* codes, float* scales,
                                    vomni_stream_t stream) {
  if (!attn || !codes || !scales) return VOMNI_EINVAL;
  if (b <= 0 || k <= 0 || s <= 0 || (k % 64) || (s % 8) || b > 65535) return VOMNI_EBADSHAPE;
  if ((reinterpret_cast<uintptr_t>(attn) | reinterpret_cast<uintptr_t>(codes)) & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  // Clusters of 8 CTAs (k / 8 rows each: 40 KB at k = 5120, so several CTAs share an SM and their
  // load and convert phases overlap); 4 when k / 8 would not be a multiple of 16 rows.
  const int cr = (k % 128 == 0) ? 8 : 4;
  if (k / cr > oproj::kRqMaxRows) return VOMNI_EBADSHAPE;
  const int rows = k / cr;  // a multiple of 16
  int box = 256;
  while (rows % box) box >>= 1;
  CUtensorMap tm;
  rc = make_tmap_3d_bf16_plain(&tm, attn, static_cast<uint64_t>(s), static_cast<uint64_t>(k), static_cast<uint64_t>(b),
                               oproj::kRqTok, static_cast<uint32_t>(box));
  if (rc) return rc;
  const int smem = rows * oproj::kRqTok * 2;
  auto kern = cr == 4 ? oproj::oproj_rowquant_kernel<4> : oproj::oproj_rowquant_kernel<8>;
  rc = ensure_max_smem(kern, smem);
  if (rc) return rc;
  const dim3 grid(static_cast<unsigned>((s + oproj::kRqTok - 1) / oproj::kRqTok * cr), static_cast<unsigned>(b));
  kern<<<grid, oproj::kRqThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tm, k, s, box, static_cast<uint8_t*>(codes),
                                                                                  scales, device_status_ptr());
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

static int bf16_linear(const void* x, long long m, int k, const void* w, const void* bias, int n, int act,
                       const void* residual, const float* gate, long long gate_rows, float* sumsq, int n_norm_heads,
                       void* out, vomni_stream_t stream) {
  if (!x || !w || !out) return VOMNI_EINVAL;
  if ((gate && !residual) || (residual && act) || gate_rows < 0 || gate_rows > 0x7fffffffLL) return VOMNI_EINVAL;
  if (m <= 0 || k <= 0 || n <= 0 || (k % oproj::kBK) || (n % 32) || act < 0 || act > 1) return VOMNI_EBADSHAPE;
  if (m > 0x7fffffffLL) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                       reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(residual) |
                       reinterpret_cast<uintptr_t>(out);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, static_cast<uint64_t>(k), static_cast<uint64_t>(m),
                    static_cast<uint64_t>(k) * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, static_cast<uint64_t>(n), static_cast<uint64_t>(k),
                    static_cast<uint64_t>(n) * 2, 64, 64);
  if (rc) return rc;
  oproj::Params p;
  p.B = 1;
  p.S = static_cast<int>(m);
  p.K = k;
  p.H = n;
  p.m_bands = static_cast<int>((m + 255) / 256);
  p.n_tiles = (n + 255) / 256;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.gate = gate;
  p.gate_per_batch = 0;
  p.gate_rows = static_cast<int>(gate_rows);
  p.sumsq = sumsq;
  p.n_norm_heads = n_norm_heads;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.status = device_status_ptr();
  rc = oproj::ensure_smem_attr();
  if (rc) return rc;
  const long long tiles = static_cast<long long>(p.m_bands) * p.n_tiles;
  const int pairs = static_cast<int>(tiles < num_sms() / 2 ? tiles : num_sms() / 2);
  auto kern = act ? oproj::gemm_bf16_pair_kernel<true, oproj::EPI_GELU>
                  : (residual ? oproj::gemm_bf16_pair_kernel<true, oproj::EPI_RESIDUAL>
                              : (sumsq ? oproj::gemm_bf16_pair_kernel<true, oproj::EPI_SUMSQ>
                                       : oproj::gemm_bf16_pair_kernel<true, oproj::EPI_BIAS>));
  kern<<<2 * pairs, oproj::kThreads, oproj::kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_ffn_gemm(const void* x, long long m, int k, const void* w, const void* bias, int n, int act,
                              const void* residual, const float* gate, long long gate_rows, void* out,
                              vomni_stream_t stream) {
  return bf16_linear(x, m, k, w, bias, n, act, residual, gate, gate_rows, nullptr, 0, out, stream);
}

extern "C" int vomni_linear_sumsq(const void* x, long long m, int k, const void* w, const void* bias, int n,
                                  float* sumsq, int n_norm_heads, void* out, vomni_stream_t stream) {
  if (!sumsq || n_norm_heads < 0 || n_norm_heads * 128 > n) return VOMNI_EINVAL;
  return bf16_linear(x, m, k, w, bias, n, 0, nullptr, nullptr, 0, sumsq, n_norm_heads, out, stream);
}
