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
// GEMM kernels: persistent clusters of two CTAs (tcgen05 cta_group::2) walking 256 x 256 output
// tiles; per CTA warp 0 is the TMA producer (its 128 rows of A and 128 rows of W per 128-byte
// k-block, 128-byte swizzle, 6-stage ring), warp 1 the TMEM owner and, in the even CTA, the
// tcgen05.mma issuer (M=256, N=256, K=32 per instruction) into one of two 256-column accumulators,
// and the remaining warps the epilogue (TMEM -> registers, scales + bias, bf16 stores, per-row
// partial sums of squares) on the other accumulator.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

#include <cstdlib>

namespace vomni {
namespace qkv {

constexpr int kBM = 128, kBN = 256, kBK = 128;  // kBK in bytes (= fp8 elements)
constexpr int kThreads = 192;
constexpr uint32_t kSfAtomBytes = 512;  // one tcgen05 scale atom: 128 rows x 4 k-sub-blocks

struct Params {
  int T, I, H;
  int m_tiles, n_tiles;
  int group;  // row bands per tile group (tile_group)
  const float* row_scale;   // [T]
  const float* chan_scale;  // [I]
  const __nv_bfloat16* bias;  // [I] or null
  __nv_bfloat16* y;           // [T, I]
  float* sumsq;               // [T, n_norm_heads] or null
  int n_norm_heads;           // 128-column blocks (heads) of the Q and K segments
  int* status;
  // EPI_MX_GELU (FFN up-projection): MX-32 codes [T, I] and their scales in the tcgen05 atom layout
  // [I/128][sf_row_blocks][512] (the A operand of the block-scaled down-projection)
  uint8_t* codes;
  uint8_t* sf;
  int sf_row_blocks;
};

// Epilogues of the ROW GEMM: bf16 Y + per-head sums of squares (QKV), or bias + GELU-tanh + MX-32
// quantisation of the result (the ROW_MX MLP's up-projection).
enum { EPI_QKV = 0, EPI_MX_GELU = 1 };

// Row bands per tile group for a contraction of k_bytes bytes per row: the largest power of two in
// [8, 32] whose bands (256 rows each) fit in 48 MB, so a group's A bands stay in L2.
inline int tile_group(int k_bytes) {
  int g = 32;
  while (g > 8 && static_cast<long long>(g) * 256 * k_bytes > (48LL << 20)) g >>= 1;
  return g;
}

// ---------------------------------------------------------------- ROW mode on CTA pairs
// The same GEMM on a cluster of two CTAs sharing each MMA (tcgen05 cta_group::2, M=256): a pair
// tile is 256 rows x 256 columns; each CTA loads its 128 rows of A and its 128 rows (half the
// columns) of W per 128-byte k-block (32 KB per stage instead of 48 KB per 128 x 256 tile), so six
// stages fit and W crosses each SM's shared memory half as often. Pair tiles are walked column-major
// in groups of row bands so the pairs in flight share both A bands and W column blocks in L2:
// a group's A bands stay in L2 while W streams through once per group. The group is the largest power
// of two in [8, 32] whose bands of 256 rows x K bytes fit in 48 MB (tile_group): 32 at K = 5120, 8 at
// the FFN down-projection's K = 13824. At the C3 shape 32 bands read 0.90 GB from DRAM per launch
// against 2.09 GB with 8, and run 3 % faster under the power cap.
constexpr int kPairStages = 6;
constexpr uint32_t kPairABytes = kBM * kBK;  // 16 KB
constexpr uint32_t kPairBBytes = 128 * kBK;  // 16 KB: this CTA's half of the 256 columns
constexpr uint32_t kPairStageBytes = kPairABytes + kPairBBytes;
constexpr uint32_t kPairSmemBar = kPairStages * kPairStageBytes;
constexpr uint32_t kPairSmemBytes = kPairSmemBar + 256 + 1024;
constexpr uint32_t kPairIdesc = idesc_e4m3(256, kBN);

struct PairTile {
  int mb, nb;
};
// Pair-tile t -> (row band of 256, column block of 256): column-major inside groups of `group` bands.
VOMNI_DEV PairTile pair_tile(int t, int m_bands, int n_tiles, int group) {
  const int per_group = group * n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int rows = min(group, m_bands - g * group);
  return PairTile{g * group + r % rows, r / rows};
}

template <int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    qkv_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairSmemBar);
  uint64_t* empty = full + kPairStages;
  uint64_t* acc_full = empty + kPairStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2], in the leader: one arrival per epilogue warp of the pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int nk = p.H / kBK;
  const int m_bands = (p.T + 255) / 256;
  const int n_all = m_bands * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPairStages; ++i) {
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
    tmem_alloc_pair(tmem_slot, 2 * kBN);
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
        const PairTile pt = pair_tile(tile, m_bands, p.n_tiles, p.group);
        const int m0 = pt.mb * 256 + static_cast<int>(rank) * kBM;
        const int n0 = pt.nb * kBN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kPairStages;
          const uint32_t ph = (it / kPairStages) & 1;
          if (it >= kPairStages && !mbar_wait(&empty[st], ph ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x51)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kPairStageBytes;
          if (leader) mbar_expect_tx(&full[st], 2 * kPairStageBytes);
          tma_load_2d_pair(&tmA, lead_full + st * 8, sa, kb * kBK, m0);
          tma_load_2d_pair(&tmB, lead_full + st * 8, sa + kPairABytes, kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint64_t a_desc0 = make_sdesc(smem_u32(smem), 16, 1024, kLayoutSW128);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < n_all; tile += n_pairs, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[acc], ((lt >> 1) & 1) ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x54)) break;
        tc_fence_after();
        const uint32_t tacc = tbase + acc * kBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kPairStages;
          const uint32_t ph = (it / kPairStages) & 1;
          if (!mbar_wait(&full[st], ph, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x52)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad0 = a_desc0 + ((st * kPairStageBytes) >> 4);
          const uint64_t bd0 = ad0 + (kPairABytes >> 4);
#pragma unroll
          for (int k4 = 0; k4 < kBK / 32; ++k4)
            mma_f8_ss_pair(tacc, ad0 + k4 * 2, bd0 + k4 * 2, kPairIdesc, (kb > 0 || k4 > 0) ? 1u : 0u);
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
      if (!mbar_wait(&acc_full[acc], (lt >> 1) & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x53)) break;
      tc_fence_after();
      const PairTile pt = pair_tile(tile, m_bands, p.n_tiles, p.group);
      const int nt = pt.nb;
      const int n0 = nt * kBN;
      const int grow = pt.mb * 256 + static_cast<int>(rank) * kBM + row;
      const bool row_ok = grow < p.T;
      const uint32_t tacc = tbase + lane_addr + acc * kBN;
      const float rs = row_ok ? p.row_scale[grow] : 0.f;
      if constexpr (kEpi == EPI_MX_GELU) {
        // One 32-column chunk = one MX block of this thread's row: v = gelu(acc * rs * cs + bias)
        // in fp32, UE8M0 scale = max biased exponent - 7 (clipped to [0, 255]), codes =
        // e4m3fn(clip(v / 2^(scale - 127), +-448)). Rows past T (pad rows of the last 128-row
        // block) get scale 127 and no codes.
        uint8_t* crow = p.codes + static_cast<size_t>(grow) * p.I + n0;
        const bool sf_ok = grow < p.sf_row_blocks * 128;
        const int m = grow & 127;
        uint8_t* sf_row = p.sf + static_cast<size_t>(grow >> 7) * kSfAtomBytes + (m & 31) * 16 + (m >> 5) * 4;
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
          int e = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = gelu_tanh(v[i]);
            e = max(e, static_cast<int>((__float_as_uint(v[i]) >> 23) & 0xFF));
          }
          const int su = min(max(e - 7, 0), 255);
          // v / 2^(su - 127) as two exact power-of-two multiplies (each factor a normal fp32)
          const int sh = 127 - su;
          const int sa = sh / 2, sb = sh - sa;
          const float fa = __uint_as_float(static_cast<uint32_t>(sa + 127) << 23);
          const float fb = __uint_as_float(static_cast<uint32_t>(sb + 127) << 23);
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = fminf(fmaxf((v[4 * i + j] * fa) * fb, -448.f), 448.f);
            w[i] = e4m3x2(q[0], q[1]) | (static_cast<uint32_t>(e4m3x2(q[2], q[3])) << 16);
          }
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
          if (sf_ok)
            sf_row[static_cast<size_t>(col0 >> 7) * p.sf_row_blocks * kSfAtomBytes + ((col0 >> 5) & 3)] =
                static_cast<uint8_t>(row_ok ? su : 127);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead_acc_empty + acc * 8);
      } else {
        float ss = 0.f, ss_lo = 0.f;
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
          if (c == 3) {
            ss_lo = ss;
            ss = 0.f;
          }
        }
        // This warp's rows of the accumulator have been read: tell the leader's MMA warp.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead_acc_empty + acc * 8);
        if (row_ok && p.sumsq && 2 * nt < p.n_norm_heads) {
          float* dst = p.sumsq + static_cast<size_t>(grow) * p.n_norm_heads + 2 * nt;
          dst[0] = ss_lo;
          dst[1] = ss;
        }
      }
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 2 * kBN);
  }
}

// ---------------------------------------------------------------- MX-32 block-scaled mode
// Scale factors (UE8M0, one per 32 contraction elements) are re-tiled once into the tcgen05 scale
// atom: for every 128-element k-block and 128-row block, 512 bytes where the byte for row
// r = 32*m1 + m0 and k-sub-block j (0..3) sits at m0*16 + m1*4 + j. A 32 x 16-byte atom is copied
// to TMEM with tcgen05.cp.32x128b.warpx4, giving lane m0 (in every quadrant) four 32-bit columns,
// column m1 holding the four k-sub-block scales of row 32*m1 + m0; the MMA's sf_id picks the byte.
// Tiled order: [k-block][128-row block][512 B], so the atoms of consecutive row blocks at one
// k-block are adjacent (a 256-column B tile's two atoms are one 1 KB copy).

__global__ void mx_pack_scales_kernel(const uint8_t* __restrict__ sf, int rows, int kblk32, int row_blocks,
                                      uint8_t* __restrict__ out) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one output byte
  const int kb4 = kblk32 / 4;
  const long long total = static_cast<long long>(kb4) * row_blocks * kSfAtomBytes;
  if (idx >= total) return;
  const int within = static_cast<int>(idx % kSfAtomBytes);
  const long long atom = idx / kSfAtomBytes;
  const int rb = static_cast<int>(atom % row_blocks);
  const int kb = static_cast<int>(atom / row_blocks);
  const int m0 = within >> 4, m1 = (within >> 2) & 3, j = within & 3;
  const int r = rb * 128 + m1 * 32 + m0;
  out[idx] = r < rows ? sf[static_cast<size_t>(r) * kblk32 + kb * 4 + j] : static_cast<uint8_t>(127);
}

constexpr uint32_t kMxSfaBytes = kSfAtomBytes;      // 128 rows of A
constexpr uint32_t kMxSfbBytes = 2 * kSfAtomBytes;  // 256 rows of B
constexpr uint32_t kMxColSf = kBN;  // scale columns follow the single accumulator: 12 per stage

struct MxParams {
  int T, I, H;
  int m_tiles, n_tiles;
  int group;  // row bands per tile group (tile_group)
  const uint8_t* sfa;  // tiled [H/128][m_tiles][512]
  const uint8_t* sfb;  // tiled [H/128][I/128][512]
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  float* sumsq;
  int n_norm_heads;
  int* status;
  // MX_EPI_FFN_DOWN: per-column weight scale [I], and the block's closing gated residual
  // y <- bf16(residual + gate * bf16(acc * chan_scale + bias)) (gate fp32 [T / gate_rows, I], NULL = 1)
  const float* chan_scale;
  const __nv_bfloat16* residual;
  const float* gate;
  long long gate_rows;
};

// Epilogues of the MX-32 GEMM: bias + bf16 + per-head sums of squares (QKV), or per-column weight
// scale + bias + bf16 (+ gated residual) (the ROW_MX MLP's down-projection).
enum { MX_EPI_QKV = 0, MX_EPI_FFN_DOWN = 1 };

constexpr int kMxThreads = 320;  // TMA warp, MMA warp, eight epilogue warps

// MX-32 on CTA pairs: 256 x 256 pair tiles, cta_group::2 block-scaled MMA (M=256, N=256, K=32).
// Each CTA stages its 128 rows of X, its 128 rows of W, the scale atom of its X rows and the two
// atoms of all 256 W rows (every SM applies the scales of the full N=256 to its 128 output rows);
// the leader copies both CTAs' atoms into their TMEM with one tcgen05.cp.cta_group::2 per atom.
constexpr int kMxPairStages = 6;
constexpr uint32_t kMxPairABytes = kBM * kBK;  // 16 KB
constexpr uint32_t kMxPairBBytes = 128 * kBK;  // 16 KB
// Stage = A tile, B tile, then the scale atoms, padded to 1 KB so every stage's A/B tiles keep the
// 1024-byte alignment the 128-byte swizzle pattern is defined on.
constexpr uint32_t kMxPairStageBytes =
    (kMxPairABytes + kMxPairBBytes + kMxSfaBytes + kMxSfbBytes + 1023) / 1024 * 1024;  // 34 KB
constexpr uint32_t kMxPairTx = kMxPairABytes + kMxPairBBytes + kMxSfaBytes + kMxSfbBytes;
constexpr uint32_t kMxPairSmemBar = kMxPairStages * kMxPairStageBytes;
constexpr uint32_t kMxPairSmemBytes = kMxPairSmemBar + 256 + 1024;

template <int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kMxThreads, 1)
    qkv_gemm_mx_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmSfa, const __grid_constant__ CUtensorMap tmSfb,
                            const MxParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kMxPairSmemBar);
  uint64_t* empty = full + kMxPairStages;
  uint64_t* acc_full = empty + kMxPairStages;
  uint64_t* acc_empty = acc_full + 1;  // in the leader: one arrival per epilogue warp of the pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int nk = p.H / kBK;
  const int m_bands = (p.T + 255) / 256;
  const int n_all = m_bands * p.n_tiles;
  const int n128 = p.I / 128;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMxPairStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 16);
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
        const PairTile pt = pair_tile(tile, m_bands, p.n_tiles, p.group);
        const int mblk = pt.mb * 2 + static_cast<int>(rank);  // this CTA's 128-row block of X
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kMxPairStages;
          const uint32_t ph = (it / kMxPairStages) & 1;
          if (it >= kMxPairStages && !mbar_wait(&empty[st], ph ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x71)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kMxPairStageBytes;
          const uint32_t bar = lead_full + st * 8;
          if (leader) mbar_expect_tx(&full[st], 2 * kMxPairTx);
          tma_load_2d_pair(&tmA, bar, sa, kb * kBK, mblk * kBM);
          tma_load_2d_pair(&tmB, bar, sa + kMxPairABytes, kb * kBK, pt.nb * kBN + static_cast<int>(rank) * 128);
          // scale atoms as rows of 128 bytes: [H/128][row blocks][4 rows of 128 B]
          tma_load_2d_pair(&tmSfa, bar, sa + kMxPairABytes + kMxPairBBytes, 0, (kb * p.m_tiles + mblk) * 4);
          tma_load_2d_pair(&tmSfb, bar, sa + kMxPairABytes + kMxPairBBytes + kMxSfaBytes, 0, (kb * n128 + pt.nb * 2) * 4);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint64_t a_desc0 = make_sdesc(smem_u32(smem), 16, 1024, kLayoutSW128);
      const uint64_t sf_desc0 = make_sdesc(smem_u32(smem + kMxPairABytes + kMxPairBBytes), 16, 128, 0);
      uint32_t it = 0;
      int lt = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < n_all; tile += n_pairs, ++lt) {
        if (lt >= 1 && !mbar_wait(acc_empty, (lt - 1) & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x74)) break;
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kMxPairStages;
          const uint32_t ph = (it / kMxPairStages) & 1;
          if (!mbar_wait(&full[st], ph, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x72)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t sdesc = sf_desc0 + ((st * kMxPairStageBytes) >> 4);
          const uint32_t t_sfa = tbase + kMxColSf + st * 12;
          const uint32_t t_sfb = t_sfa + 4;
          tmem_cp_32x128b_warpx4_pair(t_sfa, sdesc);
          tmem_cp_32x128b_warpx4_pair(t_sfb, sdesc + (kMxSfaBytes >> 4));
          tmem_cp_32x128b_warpx4_pair(t_sfb + 4, sdesc + ((kMxSfaBytes + kSfAtomBytes) >> 4));
          const uint64_t ad0 = a_desc0 + ((st * kMxPairStageBytes) >> 4);
          const uint64_t bd0 = ad0 + (kMxPairABytes >> 4);
#pragma unroll
          for (int k4 = 0; k4 < kBK / 32; ++k4)
            mma_mxf8_ss_pair(tbase, ad0 + k4 * 2, bd0 + k4 * 2, idesc_mxf8(256, kBN, k4), (kb > 0 || k4 > 0) ? 1u : 0u,
                             t_sfa | (static_cast<uint32_t>(k4) << 30), t_sfb | (static_cast<uint32_t>(k4) << 30));
          tc_commit_pair(&empty[st]);
        }
        if (ok) tc_commit_pair(acc_full);
      }
    }
  } else {
    // Eight epilogue warps per CTA (two per TMEM lane quadrant, 128 columns each): drain the
    // accumulator to registers, release it to the leader's MMA warp, then store.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    int lt = 0;
    for (int tile = pair; tile < n_all; tile += n_pairs, ++lt) {
      if (!mbar_wait(acc_full, lt & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x73)) break;
      tc_fence_after();
      const PairTile pt = pair_tile(tile, m_bands, p.n_tiles, p.group);
      const int nt = pt.nb;
      const int n0 = nt * kBN + half * 128;
      const int grow = pt.mb * 256 + static_cast<int>(rank) * kBM + row;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + lane_addr + half * 128 + c * 32, r);
        tmem_ld_wait(r);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (kEpi == MX_EPI_FFN_DOWN) {
          // v = acc * cs + bias, eight columns at a time (keeps the live set small)
          const float4* cs4 = reinterpret_cast<const float4*>(p.chan_scale + n0 + c * 32);
          const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0 + c * 32);
#pragma unroll
          for (int g8 = 0; g8 < 4; ++g8) {
            const float4 ca = cs4[2 * g8], cb = cs4[2 * g8 + 1];
            const float cs[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
            float bf[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (p.bias) {
              const uint4 bb = b4[g8];
              const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bb);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(b2[j]);
                bf[2 * j] = f.x;
                bf[2 * j + 1] = f.y;
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
              pk[16 * c + 4 * g8 + j] =
                  pack_bf16x2(__fadd_rn(__fmul_rn(v[8 * g8 + 2 * j], cs[2 * j]), bf[2 * j]),
                              __fadd_rn(__fmul_rn(v[8 * g8 + 2 * j + 1], cs[2 * j + 1]), bf[2 * j + 1]));
          }
        } else {
          if (p.bias) {
            const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0 + c * 32);
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
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[16 * c + i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty);
      if constexpr (kEpi == MX_EPI_FFN_DOWN) {
        if (p.residual && grow < p.T) {
          // (residual.float() + y.float() * gate).type_as(residual), product and sum unfused
          const __nv_bfloat16* res = p.residual + static_cast<size_t>(grow) * p.I + n0;
          const float* g = p.gate ? p.gate + static_cast<size_t>(grow / p.gate_rows) * p.I + n0 : nullptr;
#pragma unroll
          for (int i4 = 0; i4 < 16; ++i4) {
            const uint4 rv = reinterpret_cast<const uint4*>(res)[i4];
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int i = 4 * i4 + j;
              const float2 gg = g ? reinterpret_cast<const float2*>(g)[i] : make_float2(1.f, 1.f);
              const float2 rr = __bfloat1622float2(r2[j]);
              const float y0 = __uint_as_float(pk[i] << 16), y1 = __uint_as_float(pk[i] & 0xFFFF0000u);
              pk[i] = pack_bf16x2(__fadd_rn(rr.x, __fmul_rn(y0, gg.x)), __fadd_rn(rr.y, __fmul_rn(y1, gg.y)));
            }
          }
        }
      }
      float ss = 0.f;
      if constexpr (kEpi == MX_EPI_QKV) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float lo = __uint_as_float(pk[i] << 16), hi = __uint_as_float(pk[i] & 0xFFFF0000u);
          ss = fmaf(lo, lo, fmaf(hi, hi, ss));
        }
      }
      if (grow < p.T) {
        uint4* dst = reinterpret_cast<uint4*>(p.y + static_cast<size_t>(grow) * p.I + n0);
#pragma unroll
        for (int i = 0; i < 16; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      if (p.sumsq && grow < p.T && 2 * nt + half < p.n_norm_heads)
        p.sumsq[static_cast<size_t>(grow) * p.n_norm_heads + 2 * nt + half] = ss;
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
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
                                    const float* __restrict__ sumsq, float eps,
                                    const __nv_bfloat16* __restrict__ gamma_q, const __nv_bfloat16* __restrict__ gamma_k,
                                    const float* __restrict__ cos, const float* __restrict__ sin) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ float inv_s[2];
  if (threadIdx.x < 2) {
    const int n_norm = q_heads + kv_heads;  // one partial per head
    const int lo = threadIdx.x == 0 ? 0 : q_heads;
    const int hi = threadIdx.x == 0 ? q_heads : n_norm;
    float s = 0.f;
    for (int i = lo; i < hi; ++i) s += sumsq[static_cast<size_t>(t) * n_norm + i];
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
  // X: [128 B x 128 rows] boxes; W: [128 B x 128 rows] boxes (each CTA of a pair loads half of the
  // 256 output columns).
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_codes, h, t, h, qkv::kBK, qkv::kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, h, i, h, qkv::kBK, 128);
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
  p.n_norm_heads = (q_dim + kv_dim) / 128;
  p.m_tiles = (t + qkv::kBM - 1) / qkv::kBM;
  p.n_tiles = i / qkv::kBN;
  p.group = qkv::tile_group(p.H);
  p.status = device_status_ptr();
  p.codes = nullptr;
  p.sf = nullptr;
  p.sf_row_blocks = 0;
  rc = ensure_max_smem(qkv::qkv_gemm_pair_kernel<qkv::EPI_QKV>, qkv::kPairSmemBytes);
  if (rc) return rc;
  const int pair_tiles = ((t + 255) / 256) * p.n_tiles;
  const int pairs = pair_tiles < num_sms() / 2 ? pair_tiles : num_sms() / 2;
  qkv::qkv_gemm_pair_kernel<qkv::EPI_QKV><<<2 * pairs, qkv::kThreads, qkv::kPairSmemBytes,
                                            reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_qk_norm_rope(void* y, int t, int i, int q_heads, int kv_heads, int head_dim, const float* sumsq,
                                  float eps, const void* gamma_q, const void* gamma_k, const float* cos,
                                  const float* sin, vomni_stream_t stream) {
  if (!y || !sumsq) return VOMNI_EINVAL;
  if (head_dim != 128 || t <= 0 || q_heads < 0 || kv_heads < 0) return VOMNI_EBADSHAPE;
  const int q_dim = q_heads * 128, kv_dim = kv_heads * 128;
  if (q_dim + kv_dim > i) return VOMNI_EBADSHAPE;
  if ((cos == nullptr) != (sin == nullptr)) return VOMNI_EINVAL;
  const uintptr_t al = reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gamma_q) |
                       reinterpret_cast<uintptr_t>(gamma_k);
  if (al & 15 || (i % 8)) return VOMNI_EALIGN;
  qkv::qk_norm_rope_kernel<<<t, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(y), t, i, q_heads, kv_heads, sumsq, eps, static_cast<const __nv_bfloat16*>(gamma_q), static_cast<const __nv_bfloat16*>(gamma_k), cos, sin);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" size_t vomni_mx_packed_scales_bytes(int rows, int k) {
  if (rows <= 0 || k <= 0 || (k % 128)) return 0;
  return static_cast<size_t>(k / 128) * ((rows + 127) / 128) * qkv::kSfAtomBytes;
}

extern "C" int vomni_mx_pack_scales(const void* sf, int rows, int k, void* out, vomni_stream_t stream) {
  if (!sf || !out) return VOMNI_EINVAL;
  const size_t bytes = vomni_mx_packed_scales_bytes(rows, k);
  if (!bytes) return VOMNI_EBADSHAPE;
  if (reinterpret_cast<uintptr_t>(out) & 15) return VOMNI_EALIGN;
  const int threads = 256;
  const long long blocks = (static_cast<long long>(bytes) + threads - 1) / threads;
  qkv::mx_pack_scales_kernel<<<static_cast<unsigned>(blocks), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(sf), rows, k / 32, (rows + 127) / 128, static_cast<uint8_t*>(out));
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_qkv_mx32_gemm(const void* x_codes, const void* x_sf_packed, const void* w_codes,
                                   const void* w_sf_packed, const void* bias, int t, int h, int i, int q_dim, int kv_dim,
                                   void* y, float* sumsq, vomni_stream_t stream) {
  if (!x_codes || !x_sf_packed || !w_codes || !w_sf_packed || !y) return VOMNI_EINVAL;
  if (t <= 0 || h <= 0 || i <= 0 || (h % qkv::kBK) || (i % qkv::kBN)) return VOMNI_EBADSHAPE;
  if (q_dim < 0 || kv_dim < 0 || q_dim + kv_dim > i || (q_dim % qkv::kBN) || (kv_dim % qkv::kBN)) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(x_codes) | reinterpret_cast<uintptr_t>(w_codes) |
                       reinterpret_cast<uintptr_t>(x_sf_packed) | reinterpret_cast<uintptr_t>(w_sf_packed) |
                       reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(y);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_codes, h, t, h, qkv::kBK, qkv::kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, h, i, h, qkv::kBK, 128);
  if (rc) return rc;
  qkv::MxParams p;
  p.T = t;
  p.I = i;
  p.H = h;
  p.m_tiles = (t + qkv::kBM - 1) / qkv::kBM;
  p.n_tiles = i / qkv::kBN;
  p.group = qkv::tile_group(p.H);
  p.sfa = static_cast<const uint8_t*>(x_sf_packed);
  p.sfb = static_cast<const uint8_t*>(w_sf_packed);
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.sumsq = sumsq;
  p.n_norm_heads = (q_dim + kv_dim) / 128;
  p.status = device_status_ptr();
  p.chan_scale = nullptr;
  p.residual = nullptr;
  p.gate = nullptr;
  p.gate_rows = 1;
  rc = ensure_max_smem(qkv::qkv_gemm_mx_pair_kernel<qkv::MX_EPI_QKV>, qkv::kMxPairSmemBytes);
  if (rc) return rc;
  // X scale atoms must exist for every 128-row block a pair tile touches (pair bands are 256 rows)
  CUtensorMap tsa, tsb;
  const uint64_t k128 = static_cast<uint64_t>(h / 128);
  rc = make_tmap_2d_plain(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_sf_packed, 128, k128 * p.m_tiles * 4, 128, 128, 4);
  if (rc) return rc;
  rc = make_tmap_2d_plain(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_sf_packed, 128, k128 * (i / 128) * 4, 128, 128, 8);
  if (rc) return rc;
  const int pair_tiles = ((t + 255) / 256) * p.n_tiles;
  const int pairs = pair_tiles < num_sms() / 2 ? pair_tiles : num_sms() / 2;
  qkv::qkv_gemm_mx_pair_kernel<qkv::MX_EPI_QKV><<<2 * pairs, qkv::kMxThreads, qkv::kMxPairSmemBytes,
                                                  reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, tsa, tsb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

// ---------------------------------------------------------------- ROW_MX MLP (FP8 FFN)
// row_mx_mlp (diffusion/quantization/row_mx_kernels.py:141-198) -> nkilib mlp, ROW_MX, CTE
// (kernels/nkilib/core/mlp/mlp_torch.py:401-600 states its arithmetic):
//   up    = (Xq * row_scale) @ (Wu_q * wu_scale[col]) + bu       fp32
//   inter = gelu_tanh(up), MX-32 quantised along I (_mx_quantize, mlp_torch.py:252-271)
//   out   = (inter_q * mx_scale) @ (Wd_q * wd_scale[col]) + bd   -> bf16
// The up GEMM is the ROW kernel with the GELU + MX epilogue (codes and scale atoms written for the
// down GEMM directly); the down GEMM is the MX-32 block-scaled kernel with identity weight scales
// and the per-column weight scale, bias and optional gated residual in its epilogue.

extern "C" int vomni_ffn_fp8_up(const void* x_codes, const float* row_scale, const void* w_codes,
                                const float* chan_scale, const void* bias, int t, int h, int i, void* inter_codes,
                                void* inter_sf_packed, vomni_stream_t stream) {
  if (!x_codes || !row_scale || !w_codes || !chan_scale || !inter_codes || !inter_sf_packed) return VOMNI_EINVAL;
  if (t <= 0 || h <= 0 || i <= 0 || (h % qkv::kBK) || (i % qkv::kBN)) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(x_codes) | reinterpret_cast<uintptr_t>(w_codes) |
                       reinterpret_cast<uintptr_t>(chan_scale) | reinterpret_cast<uintptr_t>(bias) |
                       reinterpret_cast<uintptr_t>(inter_codes) | reinterpret_cast<uintptr_t>(inter_sf_packed);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_codes, h, t, h, qkv::kBK, qkv::kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, h, i, h, qkv::kBK, 128);
  if (rc) return rc;
  qkv::Params p;
  p.T = t;
  p.I = i;
  p.H = h;
  p.m_tiles = (t + qkv::kBM - 1) / qkv::kBM;
  p.n_tiles = i / qkv::kBN;
  p.group = qkv::tile_group(p.H);
  p.row_scale = row_scale;
  p.chan_scale = chan_scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = nullptr;
  p.sumsq = nullptr;
  p.n_norm_heads = 0;
  p.status = device_status_ptr();
  p.codes = static_cast<uint8_t*>(inter_codes);
  p.sf = static_cast<uint8_t*>(inter_sf_packed);
  p.sf_row_blocks = p.m_tiles;
  rc = ensure_max_smem(qkv::qkv_gemm_pair_kernel<qkv::EPI_MX_GELU>, qkv::kPairSmemBytes);
  if (rc) return rc;
  const int pair_tiles = ((t + 255) / 256) * p.n_tiles;
  const int pairs = pair_tiles < num_sms() / 2 ? pair_tiles : num_sms() / 2;
  qkv::qkv_gemm_pair_kernel<qkv::EPI_MX_GELU><<<2 * pairs, qkv::kThreads, qkv::kPairSmemBytes,
                                                reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_ffn_fp8_down(const void* inter_codes, const void* inter_sf_packed, const void* w_codes,
                                  const void* w_sf_packed, const float* chan_scale, const void* bias, int t, int i,
                                  int h, const void* residual, const float* gate, long long gate_rows, void* out,
                                  vomni_stream_t stream) {
  if (!inter_codes || !inter_sf_packed || !w_codes || !w_sf_packed || !chan_scale || !out) return VOMNI_EINVAL;
  if (t <= 0 || h <= 0 || i <= 0 || (i % qkv::kBK) || (h % qkv::kBN)) return VOMNI_EBADSHAPE;
  if (gate && !residual) return VOMNI_EINVAL;
  if (gate && (gate_rows <= 0 || t % gate_rows)) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(inter_codes) | reinterpret_cast<uintptr_t>(w_codes) |
                       reinterpret_cast<uintptr_t>(inter_sf_packed) | reinterpret_cast<uintptr_t>(w_sf_packed) |
                       reinterpret_cast<uintptr_t>(chan_scale) | reinterpret_cast<uintptr_t>(bias) |
                       reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(gate) |
                       reinterpret_cast<uintptr_t>(out);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;
  // K = i (intermediate), N = h (model dim): MxParams' H is the contraction, I the output width
  CUtensorMap ta, tb, tsa, tsb;
  rc = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, inter_codes, i, t, i, qkv::kBK, qkv::kBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, i, h, i, qkv::kBK, 128);
  if (rc) return rc;
  qkv::MxParams p;
  p.T = t;
  p.I = h;
  p.H = i;
  p.m_tiles = (t + qkv::kBM - 1) / qkv::kBM;
  p.n_tiles = h / qkv::kBN;
  p.group = qkv::tile_group(p.H);
  const uint64_t k128 = static_cast<uint64_t>(i / 128);
  rc = make_tmap_2d_plain(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, inter_sf_packed, 128, k128 * p.m_tiles * 4, 128, 128, 4);
  if (rc) return rc;
  rc = make_tmap_2d_plain(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_sf_packed, 128, k128 * (h / 128) * 4, 128, 128, 8);
  if (rc) return rc;
  p.sfa = static_cast<const uint8_t*>(inter_sf_packed);
  p.sfb = static_cast<const uint8_t*>(w_sf_packed);
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(out);
  p.sumsq = nullptr;
  p.n_norm_heads = 0;
  p.status = device_status_ptr();
  p.chan_scale = chan_scale;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.gate = gate;
  p.gate_rows = gate ? gate_rows : 1;
  rc = ensure_max_smem(qkv::qkv_gemm_mx_pair_kernel<qkv::MX_EPI_FFN_DOWN>, qkv::kMxPairSmemBytes);
  if (rc) return rc;
  const int pair_tiles = ((t + 255) / 256) * p.n_tiles;
  const int pairs = pair_tiles < num_sms() / 2 ? pair_tiles : num_sms() / 2;
  qkv::qkv_gemm_mx_pair_kernel<qkv::MX_EPI_FFN_DOWN><<<2 * pairs, qkv::kMxThreads, qkv::kMxPairSmemBytes,
                                                       reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, tsa, tsb, p);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}
