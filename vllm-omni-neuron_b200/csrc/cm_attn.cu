// Const-max attention for sm_100a: prologue norms + a warp-specialised tcgen05/TMEM attention pass.
//
// Algorithm (reference: vllm_omni_neuron/kernels/nkilib/experimental/attention/
// ring_attention_const_max_fwd.py and attention_const_max.py): every query row i carries a fixed
// softmax bound c_i = scale * ||q_i|| * max_j ||k_j|| (Cauchy-Schwarz, so scale*q_i.k_j - c_i <= 0),
// computed once from a prologue. With a fixed bound there is no running max and no rescaling:
//     O_i += sum_j exp(scale*q_i.k_j - c_i) v_j,   l_i += sum_j exp(...)
// and partial results of different key ranges (ring steps) combine by plain addition; one final
// normalise o_i = O_i / max(l_i, 1e-37).
//
// Kernel layout: a cluster of two CTAs on two SMs (tcgen05 cta_group::2) covers 2 x 256 query rows
// of one (batch, head); query tile t of the pair is 256 rows, 128 in each CTA. Per CTA:
//   warp 0      TMA producer: its halves of both Q tiles once, then K/V 128-key tiles into rings
//               (no multicast)
//   warp 1      TMEM owner; in the even CTA also the MMA issuer (one elected lane):
//               S_t = Q_t K^T (SS form), O_t += P_t V (TS form, P read straight from TMEM)
//   warps 2..9  softmax + epilogue: both warpgroups work on every tile, warpgroup 0 on keys 0-63 and
//               warpgroup 1 on keys 64-127 of each step; one query row per thread (TMEM lane),
//               P = exp2(S*scale*log2e - c*log2e) written back to TMEM as bf16 over S. The tiles
//               ping-pong: while the softmax warps exponentiate one tile, the tensor pipe runs the
//               other tile's PV and next QK.
// TMEM columns: S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "host_util.h"

#include <cstdlib>
#include <mutex>

// Exponentials per 16 consecutive key columns of a row that run on the FMA pipe (the packed
// polynomial of common.cuh) instead of MUFU ex2, counted in column pairs out of 8. A build-time
// constant (nvcc -DVOMNI_CM_POLY_PAIRS=k); the library has exactly one attention kernel.
#ifndef VOMNI_CM_POLY_PAIRS
#define VOMNI_CM_POLY_PAIRS 0
#endif
// Depth of the K/V shared-memory ring (one stage = the K and V halves of one 128-key step,
// 32 KB per CTA of a pair). A stage is released one step after its K was consumed (with its V).
#ifndef VOMNI_CM_KV_STAGES
#define VOMNI_CM_KV_STAGES 3
#endif

namespace vomni {
namespace cm {

constexpr int kTile = 128;  // query rows per tile (per CTA) and keys per tile
constexpr int kD = 128;     // head dim (the reference asserts 128, ring_attention_const_max_fwd.py:1026)
constexpr int kQT = 2;      // query tiles per CTA (two softmax warpgroups ping-pong on the tensor pipe)
constexpr int kThreads = 64 + 128 * kQT;
constexpr uint32_t kTileBytes = kTile * kD * 2;  // 32 KB: one bf16 [128 x 128] tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;  // 16 KB: one [128 x 64] swizzled half
constexpr int kPolyPairs = VOMNI_CM_POLY_PAIRS;
static_assert(kPolyPairs >= 0 && kPolyPairs <= 8, "VOMNI_CM_POLY_PAIRS is a count out of 8 column pairs");
constexpr int kKV = VOMNI_CM_KV_STAGES;
static_assert(kKV >= 2 && kKV <= 5, "K/V ring depth");

// K/V ring barriers: one FULL and one EMPTY per stage (K and V of a step travel together). S_FULL +
// 2t: S of tile t complete. P_FULL + 2t + set: the set-th 32-key chunk of both warpgroups' key
// halves of tile t is in TMEM (one arrival per softmax warp of both CTAs). O_FULL + t: the last PV of
// tile t is complete.
enum Bar : int {
  Q_FULL = 0,
  KV_FULL = 1,
  KV_EMPTY = KV_FULL + kKV,
  S_FULL = KV_EMPTY + kKV,
  P_FULL = S_FULL + 4,
  O_FULL = P_FULL + 4,
  NBAR = O_FULL + kQT
};
constexpr uint32_t kPWarps = 16;  // softmax warps of both CTAs: arrivals per P barrier phase
// P publication granularity: 2 = each tile's P in two chunk sets (the PV MMAs of the first set start
// while the second is exponentiated), 1 = whole tiles (one MMA-thread wait per tile and step).
#ifndef VOMNI_CM_P_SETS
#define VOMNI_CM_P_SETS 2
#endif
constexpr int kPSets = VOMNI_CM_P_SETS;
static_assert(kPSets == 1 || kPSets == 2, "P sets per tile");
static_assert(NBAR * 8 + 8 <= 256, "barriers, TMEM slot and abort flag fit the 256-byte area");

// TMEM columns: tile t owns S_t = [t*128, t*128+128) (P_t, bf16, aliases its first 64 columns) and
// O_t = [256 + t*128, 256 + t*128 + 128).
constexpr uint32_t kColS = 0, kColO = 256;

struct Params {
  int s_q;          // query rows per (batch, head)
  int heads;        // h
  int n_keys;       // keys in this pass
  int k_start;      // first key row in the K/V maps
  float scale_log2;  // softmax_scale * log2(e)
  float scale;      // softmax_scale
  const float* qn2;    // [b*h, s_q]
  const float* kmax2;  // [b*h]
  float* acc_o;        // [b*h, s_q, 128]
  float* acc_l;        // [b*h, s_q]
  void* out;           // bf16
  float* lse;          // [b*h, 128, ceil(s_q/128)]
  int flags;
  int* status;
  const unsigned* ready;  // if set: K/V of this pass are valid once ready[0 .. ready_count) reach ready_epoch
  int ready_count;
  unsigned ready_epoch;
};

// Column pair i (of 16 in a 32-column chunk) takes the FMA-pipe exponential when it is one of the
// kPolyPairs pairs spread evenly over each group of 8.
__host__ __device__ constexpr bool poly_pair(int i) {
  return ((i % 8 + 1) * kPolyPairs) / 8 > ((i % 8) * kPolyPairs) / 8;
}

// One 32-column chunk of one query row: p = 2^(s*scale*log2e - c*log2e), packed to bf16 pairs for
// the PV MMA, and the row sum accumulated from those same bf16 values: the reference sums exactly
// the bf16 P it multiplies, through the ones column of [V|1] (attention_const_max.py:307-311,
// 370-379). The scale-and-shift runs as packed fp32 pairs; the sum adds the bf16 values exactly
// into four independent fp32 accumulators (short add chains). kMask: columns at or past `valid`
// (keys outside this pass) contribute 0.
template <bool kMask>
VOMNI_DEV void softmax_chunk(const uint32_t (&s)[32], uint64_t scale2, uint64_t neg_c2, int valid, float (&acc)[4],
                             uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint64_t x = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), scale2, neg_c2);
    float x0, x1, p0, p1;
    f2_unpack(x, x0, x1);
    if (poly_pair(i)) {
      exp2_poly2(x0, x1, p0, p1);
    } else {
      p0 = ex2_approx(x0);
      p1 = ex2_approx(x1);
    }
    if (kMask) {
      p0 = (2 * i < valid) ? p0 : 0.f;
      p1 = (2 * i + 1 < valid) ? p1 : 0.f;
    }
    pk[i] = pack_bf16x2(p0, p1);
    add_bf16x2_f32(acc[(i & 1) * 2], acc[(i & 1) * 2 + 1], pk[i]);
  }
}


// Signal that this warp's P columns of one (tile, chunk set) are in TMEM, after its stores completed
// (tcgen05.wait::st + fence::before_thread_sync): one arrival per warp on the set's barrier in the
// pair leader (release at cluster scope). `pbar`: shared::cluster address of the leader's P barriers.
VOMNI_DEV void publish_p(uint32_t pbar, int set) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(pbar + 8 * set);
}

// P layout in TMEM: the bf16 probabilities of keys [16kk, 16kk + 16) of query tile t sit in the 8
// columns from S_t + p_col(kk). Warpgroup 0 owns keys 0-63 (S columns 0-63) and writes their P over
// its first 32 S columns; warpgroup 1 owns keys 64-127 (S columns 64-127) and writes their P over
// columns 64-95. Neither overwrites S that the other, or its own not yet loaded chunk, still reads.
__host__ __device__ constexpr uint32_t p_col(int kk) { return kk * 8 + (kk >= 4 ? 32 : 0); }

// Softmax of warpgroup wg's share of one query tile: keys [64wg, 64wg + 64) of this thread's row,
// in two 32-key chunks published separately: chunk A (keys 64wg .. +32) on p_a, chunk B on p_b
// (the caller publishes B after its store completes). Chunk B's S is loaded while chunk A is
// computed; chunk A's P lands on chunk A's own S columns, chunk B's S columns are never written.
template <bool kMask>
VOMNI_DEV void softmax_share(uint32_t col_s, int wg, uint64_t scale2, uint64_t neg_c2, int valid, float (&acc)[4],
                             uint32_t pbar, int set_a) {
  uint32_t sa[32], sb[32], pk[16];
  const uint32_t c0 = col_s + 64 * wg;
  const int v0 = valid - 64 * wg;
  tmem_ld32(c0, sa);
  tmem_ld_wait(sa);
  tmem_ld32(c0 + 32, sb);
  softmax_chunk<kMask>(sa, scale2, neg_c2, v0, acc, pk);
  tmem_st16(col_s + p_col(4 * wg), pk);
  if (kPSets == 2) {
    tmem_st_wait();
    tc_fence_before();
    publish_p(pbar, set_a);
  }
  tmem_ld_wait(sb);
  softmax_chunk<kMask>(sb, scale2, neg_c2, v0 - 32, acc, pk);
  tmem_st16(col_s + p_col(4 * wg + 2), pk);
}

// Stage (j-1) % kKV is free once S of the last query tile for step j is complete: its K was read by
// the QKs of step j-1 and its V by the PVs of step j-1, all issued before that QK (tcgen05 ops of one
// thread complete in order). Replaces a tcgen05.commit per step on the MMA thread.
VOMNI_DEV void release_stage(uint64_t* bars, int j) {
  if (j > 0) mbar_arrive(&bars[KV_EMPTY + (j - 1) % kKV]);
}

// Softmax + epilogue warps (warps 2..9). Both warpgroups work on every query tile, in the order the
// MMA thread produces them (tile 0, tile 1, tile 0, ...): warpgroup wg = (warp-2)/4 takes keys
// [64wg, 64wg + 64) of each 128-key step and, in the epilogue, output columns [64wg, 64wg + 64).
// Two warps per SMSP on the same tile hide each other's TMEM and MUFU latencies. quad = warp % 4
// is the TMEM lane quadrant: thread (quad, lane) owns query row quad*32 + lane of both tiles.
// q_base: first query row of this CTA's tile 0; tile_stride: rows between its tiles. pbar: the
// shared::cluster address of the leader's P barriers. lsum: 2 x 2 x 128 floats of shared memory for
// the row-sum exchange.
VOMNI_DEV void softmax_role(const Params& p, uint64_t* bars, volatile int* abort_flag, uint32_t tbase, int warp, int lane,
                            int q_base, int tile_stride, int bh, int n_tiles, uint32_t pbar, float* lsum) {
  const int wg = (warp - 2) >> 2;
  const int quad = warp & 3;
  const int row = quad * 32 + lane;
  const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
  const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
  int grow[kQT];
  bool row_ok[kQT];
  float c[kQT];
  uint64_t neg_c2[kQT];
#pragma unroll
  for (int t = 0; t < kQT; ++t) {
    grow[t] = q_base + t * tile_stride + row;
    row_ok[t] = grow[t] < p.s_q;
    c[t] = 0.f;
    if (row_ok[t]) {
      // c_i = scale * sqrt(kmax2 * ||q_i||^2), held in bf16 like the reference's c_row
      // (ring_attention_const_max_fwd.py:585-591).
      const float c32 = p.scale * sqrtf(p.kmax2[bh] * p.qn2[static_cast<size_t>(bh) * p.s_q + grow[t]]);
      c[t] = __bfloat162float(__float2bfloat16_rn(c32));
    }
    const float neg_c = -c[t] * 1.4426950408889634f;
    neg_c2[t] = f2_pack(neg_c, neg_c);
  }
  // One thread frees the K/V stages when S of the last tile of step j is complete: every QK of step
  // j (and, issued before it, every PV of step j-1) has then finished reading them.
  const bool releaser = wg == 0 && row == 0;
  float acc[kQT][4] = {};  // per tile: four fp32 partial row sums
  bool ok = true;
  for (int j = 0; j < n_tiles && ok; ++j) {
    const int valid = p.n_keys - j * kTile;  // keys of this step inside the pass's range
#pragma unroll
    for (int t = 0; t < kQT; ++t) {
      if (!mbar_wait_spin(&bars[S_FULL + 2 * t], j & 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 7)) { ok = false; break; }
      tc_fence_after();
      if (releaser && t == kQT - 1) release_stage(bars, j);
      const uint32_t col_s = tbase + lane_addr + kColS + t * 128;
      if (valid >= kTile)
        softmax_share<false>(col_s, wg, scale2, neg_c2[t], valid, acc[t], pbar, 2 * t);
      else
        softmax_share<true>(col_s, wg, scale2, neg_c2[t], valid, acc[t], pbar, 2 * t);
      tmem_st_wait();
      tc_fence_before();
      publish_p(pbar, 2 * t + 1);
    }
  }
  // ---------------------------------------------------------- epilogue
  // Row sums of the two warpgroups' key halves meet in shared memory (added in a fixed order, so
  // results do not depend on scheduling). Every softmax thread reaches the named barrier: all the
  // waits above are bounded, so an aborted CTA gets here too.
#pragma unroll
  for (int t = 0; t < kQT; ++t) {
    lsum[(t * 2 + wg) * 128 + row] = (acc[t][0] + acc[t][1]) + (acc[t][2] + acc[t][3]);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(128 * kQT) : "memory");
  if (!ok) return;
  const bool acc_in = p.flags & VOMNI_CM_ACC_IN;
  const bool final_pass = p.flags & VOMNI_CM_FINAL;
#pragma unroll 1
  for (int t = 0; t < kQT; ++t) {
    if (!mbar_wait_spin(&bars[O_FULL + t], 0, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 9)) return;
    tc_fence_after();
    // A pass launched as a programmatic dependent of the previous pass reads and writes acc / out
    // only from here on, after that pass has completed.
    if (t == 0) pdl_wait();
    const size_t rowidx = static_cast<size_t>(bh) * p.s_q + grow[t];
    float l = lsum[(t * 2) * 128 + row] + lsum[(t * 2 + 1) * 128 + row];
    if (acc_in && row_ok[t]) l += p.acc_l[rowidx];
    const float inv = 1.f / fmaxf(l, 1e-37f);
    float* acc_row = p.acc_o ? p.acc_o + rowidx * kD : nullptr;
    const uint32_t col_o = tbase + lane_addr + kColO + t * 128;
#pragma unroll 1
    for (int ch = 2 * wg; ch < 2 * wg + 2; ++ch) {
      uint32_t o[32];
      tmem_ld32(col_o + ch * 32, o);
      tmem_ld_wait(o);
      if (!row_ok[t]) continue;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]);
      if (acc_in) {
        const float4* src = reinterpret_cast<const float4*>(acc_row + ch * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 a = src[i];
          v[4 * i] += a.x; v[4 * i + 1] += a.y; v[4 * i + 2] += a.z; v[4 * i + 3] += a.w;
        }
      }
      if (!final_pass) {
        float4* dst = reinterpret_cast<float4*>(acc_row + ch * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      } else if (p.flags & VOMNI_CM_OUT_DMAJOR) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(bh) * kD * p.s_q;
#pragma unroll
        for (int i = 0; i < 32; ++i) out[static_cast<size_t>(ch * 32 + i) * p.s_q + grow[t]] = __float2bfloat16_rn(v[i] * inv);
      } else {
        uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + rowidx * kD + ch * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 w;
          w.x = pack_bf16x2(v[8 * i] * inv, v[8 * i + 1] * inv);
          w.y = pack_bf16x2(v[8 * i + 2] * inv, v[8 * i + 3] * inv);
          w.z = pack_bf16x2(v[8 * i + 4] * inv, v[8 * i + 5] * inv);
          w.w = pack_bf16x2(v[8 * i + 6] * inv, v[8 * i + 7] * inv);
          out[i] = w;
        }
      }
    }
    if (wg == 0 && row_ok[t]) {
      if (!final_pass) {
        p.acc_l[rowidx] = l;
      } else if (p.flags & VOMNI_CM_LSE) {
        const int groups = (p.s_q + 127) / 128;
        p.lse[(static_cast<size_t>(bh) * 128 + (grow[t] & 127)) * groups + (grow[t] >> 7)] = c[t] + logf(fmaxf(l, 1e-37f));
      }
    }
  }
}

// ---------------------------------------------------------------- CTA-pair attention
// A cluster of two CTAs (two SMs) shares each MMA (tcgen05 cta_group::2): a pair covers 2 x 256
// query rows of one (batch, head); query tile t of the pair is 256 rows, 128 in each CTA's shared
// memory and TMEM. For QK the pair's 128-key K tile is split by key (64 keys in each CTA); for PV
// the V tile is split by head dimension (64 columns in each CTA). Each CTA therefore streams half
// the K/V bytes through its shared memory per MMA (A 4 KB + B 2 KB per 64 cycles, where a one-CTA
// M=128 MMA would need A 4 KB + B 4 KB and meet the shared-memory operand bandwidth).
// The even CTA issues every MMA; both CTAs run producers and softmax warpgroups. Operand loads
// complete on the leader's barriers (cta_group::2 tile loads, no multicast), MMA completion is
// committed to both CTAs, and the peer's softmax warps arrive on the leader's P barriers.
constexpr uint32_t kPairKBytes = 64 * kD * 2;   // 16 KB: 64 keys x 128 dims
constexpr uint32_t kPairVBytes = kTile * 64 * 2;  // 16 KB: 128 keys x 64 dims
constexpr uint32_t kPairSmemQ = 0;
constexpr uint32_t kPairSmemK = kPairSmemQ + kQT * kTileBytes;
constexpr uint32_t kPairSmemV = kPairSmemK + kKV * kPairKBytes;  // V stage i right after all K stages
constexpr uint32_t kPairSmemBar = kPairSmemV + kKV * kPairVBytes;
constexpr uint32_t kPairSmemLsum = kPairSmemBar + 256;              // [2 tiles][2 warpgroups][128] fp32
constexpr uint32_t kPairSmemBytes = kPairSmemLsum + kQT * 2 * 128 * 4 + 1024;
constexpr uint32_t kIdescQKPair = idesc_bf16(256, 128, false);
constexpr uint32_t kIdescPVPair = idesc_bf16(256, 128, true);

__device__ __forceinline__ void issue_qk_pair(uint32_t d_s, uint64_t q_desc, uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t offa = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
    const uint64_t offb = ((kk >> 2) * (kPairKBytes / 2) + (kk & 3) * 32) >> 4;
    mma_f16_ss_pair(d_s, q_desc + offa, k_desc + offb, kIdescQKPair, kk > 0);
  }
}
// O_t += P_t V over the 16-key groups kk of chunk set `hf`: hf = 0 takes the first 32-key chunk of
// each warpgroup (kk 0, 1, 4, 5), hf = 1 the second (kk 2, 3, 6, 7). P from TMEM (p_col), V as an
// MN-major SW128 operand (16 keys = two 8-row groups = +2048 B).
template <int kSet>
__device__ __forceinline__ void issue_pv_pair_chunks(uint32_t d_o, uint32_t s_tmem, uint64_t v_desc, uint32_t acc_first) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kk = (i & 1) + (i >> 1) * 4 + kSet * 2;
    mma_f16_ts_pair(d_o, s_tmem + p_col(kk), v_desc + ((kk * 2048) >> 4), kIdescPVPair, (kSet > 0 || i > 0) ? 1u : acc_first);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    cm_attend_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairSmemBar);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + kPairSmemBar + NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPairSmemBar + NBAR * 8 + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int q_base = (blockIdx.x >> 1) * (2 * kTile * kQT) + static_cast<int>(rank) * kTile;  // this CTA's tile-0 rows
  const int bh = blockIdx.y;
  const int b = bh / p.heads;
  const int h = bh % p.heads;
  const int n_tiles = (p.n_keys + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    mbar_init(&bars[Q_FULL], 1);
    for (int i = 0; i < kKV; ++i) {
      mbar_init(&bars[KV_FULL + i], 1);
      mbar_init(&bars[KV_EMPTY + i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&bars[P_FULL + i], kPWarps);
    for (int i = 0; i < 4; ++i) mbar_init(&bars[S_FULL + i], 1);
    for (int t = 0; t < kQT; ++t) mbar_init(&bars[O_FULL + t], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tbase = *tmem_base_slot;
  const uint32_t lead_bars = mapa_shared(smem_u32(bars), 0);  // the leader's barrier array

  uint8_t* sQ = smem + kPairSmemQ;
  uint8_t* sK = smem + kPairSmemK;
  uint8_t* sV = smem + kPairSmemV;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int x0 = h * kD;
      if (leader) mbar_expect_tx(&bars[Q_FULL], 2 * kQT * kTileBytes);
      for (int t = 0; t < kQT; ++t) {
        const int qr = q_base + t * 2 * kTile;
        tma_load_3d_pair(&tmQ, lead_bars + Q_FULL * 8, sQ + t * kTileBytes, x0, qr, b);
        tma_load_3d_pair(&tmQ, lead_bars + Q_FULL * 8, sQ + t * kTileBytes + kHalfBytes, x0 + 64, qr, b);
      }
      bool kv_ready = true;
      for (int w = 0; p.ready && kv_ready && w < p.ready_count; ++w)
        kv_ready = ready_wait(p.ready + w, p.ready_epoch, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x20);
      for (int j = 0; kv_ready && j < n_tiles; ++j) {
        const int st = j % kKV;
        const uint32_t ph = (j / kKV) & 1;
        const int k_row = p.k_start + j * kTile;
        if (j >= kKV && !mbar_wait_spin(&bars[KV_EMPTY + st], ph ^ 1, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x21)) break;
        if (leader) mbar_expect_tx(&bars[KV_FULL + st], 2 * (kPairKBytes + kPairVBytes));
        tma_load_3d_pair(&tmK, lead_bars + (KV_FULL + st) * 8, sK + st * kPairKBytes, x0, k_row + rank * 64, b);
        tma_load_3d_pair(&tmK, lead_bars + (KV_FULL + st) * 8, sK + st * kPairKBytes + kPairKBytes / 2, x0 + 64,
                         k_row + rank * 64, b);
        tma_load_3d_pair(&tmV, lead_bars + (KV_FULL + st) * 8, sV + st * kPairVBytes, x0 + rank * 64, k_row, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    // Order per step j and tile t: PV_t(j-1) in its two chunk sets, then QK_t(j), which overwrites
    // S_t / P_t that those PVs read (tcgen05.mma ops of one thread execute in issue order); the tiles
    // alternate so that one tile's MMAs run while the softmax warps work on the other. The tensor
    // pipe queues about one MMA, so every wait here is idle tensor time: K and V share one barrier
    // per stage.
    if (leader && lane == 0) {
      const uint64_t q_desc = make_sdesc(smem_u32(sQ), 16, 1024, kLayoutSW128);
      const uint64_t k_desc = make_sdesc(smem_u32(sK), 16, 1024, kLayoutSW128);
      const uint64_t v_desc = make_sdesc(smem_u32(sV), kPairVBytes, 1024, kLayoutSW128);
      constexpr uint64_t kTileDesc = kTileBytes >> 4;
      bool ok = mbar_wait_spin(&bars[Q_FULL], 0, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x23) &&
                mbar_wait_spin(&bars[KV_FULL], 0, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x24);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < kQT; ++t) {
          issue_qk_pair(tbase + kColS + t * 128, q_desc + t * kTileDesc, k_desc);
          tc_commit_pair(&bars[S_FULL + 2 * t]);
        }
      }
      // stage indices advance with the step instead of being recomputed (vs = (j-1) % kKV, ks = j % kKV)
      int vs = 0, ks = 1 % kKV;
      uint32_t kv_phase = kKV == 1 ? 1u : 0u;  // parity of the KV_FULL phase of step j (stage ks)
      for (int j = 1; ok && j <= n_tiles; ++j) {
        const uint32_t pphase = (j - 1) & 1;
        const uint32_t acc_first = j > 1 ? 1u : 0u;
        const uint64_t vd = v_desc + ((vs * kPairVBytes) >> 4);
        const uint64_t kd = k_desc + ((ks * kPairKBytes) >> 4);
#pragma unroll
        for (int t = 0; t < kQT; ++t) {
          const uint32_t d_o = tbase + kColO + t * 128, d_s = tbase + kColS + t * 128;
          if (kPSets == 2) {
            if (!mbar_wait_spin(&bars[P_FULL + 2 * t], pphase, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x25)) { ok = false; break; }
            tc_fence_after();
            issue_pv_pair_chunks<0>(d_o, d_s, vd, acc_first);
          }
          if (!mbar_wait_spin(&bars[P_FULL + 2 * t + 1], pphase, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x25)) { ok = false; break; }
          tc_fence_after();
          if (kPSets == 1) issue_pv_pair_chunks<0>(d_o, d_s, vd, acc_first);
          issue_pv_pair_chunks<1>(d_o, d_s, vd, acc_first);
          if (j < n_tiles) {
            if (t == 0 && !mbar_wait_spin(&bars[KV_FULL + ks], kv_phase, abort_flag, p.status, VOMNI_DEV_TIMEOUT_BASE + 0x24)) { ok = false; break; }
            tc_fence_after();
            issue_qk_pair(d_s, q_desc + t * kTileDesc, kd);
            tc_commit_pair(&bars[S_FULL + 2 * t]);
          }
        }
        vs = vs + 1 == kKV ? 0 : vs + 1;
        if (++ks == kKV) {
          ks = 0;
          kv_phase ^= 1u;
        }
      }
      for (int t = 0; t < kQT; ++t) tc_commit_pair(&bars[O_FULL + t]);
    }
  } else {
    softmax_role(p, bars, abort_flag, tbase, warp, lane, q_base, 2 * kTile, bh, n_tiles, lead_bars + P_FULL * 8,
                 reinterpret_cast<float*>(smem + kPairSmemLsum));
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair may still touch its barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
  pdl_wait();  // this grid completes only after the pass it overlapped (also on an abort path)
}

// ---------------------------------------------------------------- prologue norms
// One half-warp per (batch, token, head) row of 128 bf16: per-token ||q||^2 to qn2, and the
// per-head max of ||k||^2 folded through shared memory into kmax2 (atomicMax on the float bits,
// valid because sums of squares are non-negative).
__global__ void cm_norms_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, int b, int s,
                                int s_k, int h, long long q_stride, long long k_stride, float* __restrict__ qn2,
                                unsigned int* __restrict__ kmax2_bits) {
  // q rows: b*s*h (per-token ||q||^2); k rows: b*s_k*h (per-head max ||k||^2). s_k != s for
  // cross-attention (keys from another sequence).
  extern __shared__ unsigned int smax[];  // [b*h]
  const int bhn = b * h;
  for (int i = threadIdx.x; i < bhn; i += blockDim.x) smax[i] = 0u;
  __syncthreads();
  const long long rows_q = static_cast<long long>(b) * s * h;
  const long long rows_k = static_cast<long long>(b) * s_k * h;
  const long long rows = rows_q > rows_k ? rows_q : rows_k;
  const int half = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int sub = threadIdx.x & 15;
  const unsigned hmask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
  const int halves = (gridDim.x * blockDim.x) >> 4;
  for (long long r = half; r < rows; r += halves) {
    const long long hd = (r % h) * kD;
    const int hh = static_cast<int>(r % h);
    float sq = 0.f, sk = 0.f;
    if (r < rows_q) {
      const uint4 qv = reinterpret_cast<const uint4*>(q + (r / h) * q_stride + hd)[sub];
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __bfloat1622float2(q2[i]);
        sq = fmaf(a.x, a.x, fmaf(a.y, a.y, sq));
      }
    }
    if (r < rows_k) {
      const uint4 kv = reinterpret_cast<const uint4*>(k + (r / h) * k_stride + hd)[sub];
      const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 c = __bfloat1622float2(k2[i]);
        sk = fmaf(c.x, c.x, fmaf(c.y, c.y, sk));
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(hmask, sq, o);
      sk += __shfl_xor_sync(hmask, sk, o);
    }
    if (sub == 0) {
      if (r < rows_q) {
        const long long tok = r / h;
        qn2[(static_cast<size_t>(tok / s) * h + hh) * s + tok % s] = sq;
      }
      if (r < rows_k) atomicMax(&smax[static_cast<int>((r / h) / s_k) * h + hh], __float_as_uint(sk));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < bhn; i += blockDim.x)
    if (smax[i]) atomicMax(&kmax2_bits[i], smax[i]);
}

}  // namespace cm
}  // namespace vomni

using namespace vomni;

extern "C" size_t vomni_cm_workspace_bytes(int b, int s, int h, int d) {
  (void)d;
  if (b <= 0 || s <= 0 || h <= 0) return 0;
  const size_t qn = static_cast<size_t>(b) * h * s * sizeof(float);
  const size_t km = static_cast<size_t>(b) * h * sizeof(float);
  return align_up(qn, 256) + align_up(km, 256);
}

static int cm_prologue(const void* q, const void* k, int b, int s, int s_k, int h, int d, long long q_stride,
                       long long k_stride, float* qn2, float* kmax2, vomni_stream_t stream) {
  if (!q || !k || !qn2 || !kmax2) return VOMNI_EINVAL;
  if (d != cm::kD || b <= 0 || s <= 0 || s_k <= 0 || h <= 0) return VOMNI_EBADSHAPE;
  if (b * h > 8192) return VOMNI_EBADSHAPE;
  if (q_stride == 0) q_stride = static_cast<long long>(h) * d;
  if (k_stride == 0) k_stride = static_cast<long long>(h) * d;
  if (q_stride < static_cast<long long>(h) * d || k_stride < static_cast<long long>(h) * d) return VOMNI_EBADSHAPE;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & 15) || ((q_stride | k_stride) & 7))
    return VOMNI_EALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  VOMNI_CUDA_TRY(cudaMemsetAsync(kmax2, 0, sizeof(float) * b * h, st));
  const long long rows = static_cast<long long>(b) * (s > s_k ? s : s_k) * h;
  const int threads = 256;
  long long blocks = (rows * 16 + threads - 1) / threads;
  const int max_blocks = num_sms() * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  cm::cm_norms_kernel<<<static_cast<int>(blocks), threads, sizeof(unsigned) * b * h, st>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), b, s, s_k, h, q_stride, k_stride, qn2,
      reinterpret_cast<unsigned int*>(kmax2));
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

extern "C" int vomni_cm_prologue_strided(const void* q, const void* k, int b, int s, int h, int d, long long q_stride,
                                         long long k_stride, float* qn2, float* kmax2, vomni_stream_t stream) {
  return cm_prologue(q, k, b, s, s, h, d, q_stride, k_stride, qn2, kmax2, stream);
}

extern "C" int vomni_cm_prologue(const void* q, const void* k, int b, int s, int h, int d, float* qn2, float* kmax2,
                                 vomni_stream_t stream) {
  return vomni_cm_prologue_strided(q, k, b, s, h, d, 0, 0, qn2, kmax2, stream);
}

extern "C" int vomni_cm_attend_strided(const void* q, const void* k, const void* v, int b, int s_q, int s_kv,
                                       int k_start, int n_keys, int h, int d, long long q_stride, long long kv_stride,
                                       float softmax_scale, const float* qn2, const float* kmax2, float* acc_o,
                                       float* acc_l, int flags, void* out, float* lse, vomni_stream_t stream) {
  return vomni::cm_attend_gated(q, k, v, b, s_q, s_kv, k_start, n_keys, h, d, q_stride, kv_stride, softmax_scale, qn2,
                                kmax2, acc_o, acc_l, flags, out, lse, nullptr, 0, 0u, stream);
}

int vomni::cm_attend_gated(const void* q, const void* k, const void* v, int b, int s_q, int s_kv, int k_start,
                           int n_keys, int h, int d, long long q_stride, long long kv_stride, float softmax_scale,
                           const float* qn2, const float* kmax2, float* acc_o, float* acc_l, int flags, void* out,
                           float* lse, const unsigned* ready, int ready_count, unsigned ready_epoch,
                           vomni_stream_t stream) {
  if (!q || !k || !v || !qn2 || !kmax2) return VOMNI_EINVAL;
  if (d != cm::kD || b <= 0 || s_q <= 0 || h <= 0 || n_keys <= 0 || k_start < 0 || k_start + n_keys > s_kv)
    return VOMNI_EBADSHAPE;
  if (flags & ~(VOMNI_CM_ACC_IN | VOMNI_CM_FINAL | VOMNI_CM_OUT_DMAJOR | VOMNI_CM_LSE | VOMNI_CM_OVERLAP))
    return VOMNI_EINVAL;
  const bool final_pass = flags & VOMNI_CM_FINAL;
  if (final_pass && !out) return VOMNI_EINVAL;
  if ((flags & VOMNI_CM_LSE) && !lse) return VOMNI_EINVAL;
  if ((!final_pass || (flags & VOMNI_CM_ACC_IN)) && (!acc_o || !acc_l)) return VOMNI_EINVAL;
  if (b * h > 65535) return VOMNI_EBADSHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                       reinterpret_cast<uintptr_t>(acc_o) | reinterpret_cast<uintptr_t>(out);
  if (al & 15) return VOMNI_EALIGN;
  int rc = require_sm100();
  if (rc) return rc;

  const uint64_t row_elems = static_cast<uint64_t>(h) * cm::kD;
  if (q_stride == 0) q_stride = static_cast<long long>(row_elems);
  if (kv_stride == 0) kv_stride = static_cast<long long>(row_elems);
  if (q_stride < static_cast<long long>(row_elems) || kv_stride < static_cast<long long>(row_elems)) return VOMNI_EBADSHAPE;
  // Q and V: [64 dims x 128 rows] boxes; K: [64 dims x 64 keys] boxes (each CTA of a pair loads half
  // of a 128-key tile).
  CUtensorMap tq, tk, tv;
  rc = make_tmap_3d_bf16(&tq, q, row_elems, s_q, b, 64, 128, static_cast<uint64_t>(q_stride));
  if (rc) return rc;
  rc = make_tmap_3d_bf16(&tk, k, row_elems, s_kv, b, 64, 64, static_cast<uint64_t>(kv_stride));
  if (rc) return rc;
  rc = make_tmap_3d_bf16(&tv, v, row_elems, s_kv, b, 64, 128, static_cast<uint64_t>(kv_stride));
  if (rc) return rc;

  cm::Params p;
  p.s_q = s_q;
  p.heads = h;
  p.n_keys = n_keys;
  p.k_start = k_start;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.qn2 = qn2;
  p.kmax2 = kmax2;
  p.acc_o = acc_o;
  p.acc_l = acc_l;
  p.out = out;
  p.lse = lse;
  p.flags = flags;
  p.status = device_status_ptr();
  p.ready = ready;
  p.ready_count = ready ? ready_count : 0;
  p.ready_epoch = ready_epoch;

  rc = ensure_max_smem(cm::cm_attend_pair_kernel, cm::kPairSmemBytes);
  if (rc) return rc;
  const int pairs = (s_q + 4 * cm::kTile - 1) / (4 * cm::kTile);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, b * h);
  cfg.blockDim = dim3(cm::kThreads);
  cfg.dynamicSmemBytes = cm::kPairSmemBytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & VOMNI_CM_OVERLAP) ? 1 : 0;
  VOMNI_CUDA_TRY(cudaLaunchKernelEx(&cfg, cm::cm_attend_pair_kernel, tq, tk, tv, p));
  return VOMNI_OK;
}

extern "C" int vomni_cm_attend(const void* q, const void* k, const void* v, int b, int s_q, int s_kv, int k_start,
                               int n_keys, int h, int d, float softmax_scale, const float* qn2, const float* kmax2,
                               float* acc_o, float* acc_l, int flags, void* out, float* lse, vomni_stream_t stream) {
  return vomni_cm_attend_strided(q, k, v, b, s_q, s_kv, k_start, n_keys, h, d, 0, 0, softmax_scale, qn2, kmax2, acc_o,
                                 acc_l, flags, out, lse, stream);
}

extern "C" int vomni_cm_attention_local_strided(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                                int s, int h, int d, long long q_stride, long long kv_stride,
                                                float softmax_scale, int flags, void* workspace, size_t workspace_bytes,
                                                vomni_stream_t stream) {
  if (!workspace) return VOMNI_EINVAL;
  if (flags & ~(VOMNI_CM_OUT_DMAJOR | VOMNI_CM_LSE)) return VOMNI_EINVAL;
  const size_t need = vomni_cm_workspace_bytes(b, s, h, d);
  if (need == 0) return VOMNI_EBADSHAPE;
  if (workspace_bytes < need) return VOMNI_EWORKSPACE;
  float* qn2 = static_cast<float*>(workspace);
  float* kmax2 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                          align_up(static_cast<size_t>(b) * h * s * sizeof(float), 256));
  int rc = vomni_cm_prologue_strided(q, k, b, s, h, d, q_stride, kv_stride, qn2, kmax2, stream);
  if (rc) return rc;
  return vomni_cm_attend_strided(q, k, v, b, s, s, 0, s, h, d, q_stride, kv_stride, softmax_scale, qn2, kmax2, nullptr,
                                 nullptr, flags | VOMNI_CM_FINAL, out, lse, stream);
}

extern "C" int vomni_cm_attention_cross(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                        int s_q, int s_kv, int h, int d, long long q_stride, long long kv_stride,
                                        float softmax_scale, int flags, void* workspace, size_t workspace_bytes,
                                        vomni_stream_t stream) {
  if (!workspace) return VOMNI_EINVAL;
  if (flags & ~(VOMNI_CM_OUT_DMAJOR | VOMNI_CM_LSE)) return VOMNI_EINVAL;
  const size_t need = vomni_cm_workspace_bytes(b, s_q, h, d);
  if (need == 0 || s_kv <= 0) return VOMNI_EBADSHAPE;
  if (workspace_bytes < need) return VOMNI_EWORKSPACE;
  float* qn2 = static_cast<float*>(workspace);
  float* kmax2 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                          align_up(static_cast<size_t>(b) * h * s_q * sizeof(float), 256));
  int rc = cm_prologue(q, k, b, s_q, s_kv, h, d, q_stride, kv_stride, qn2, kmax2, stream);
  if (rc) return rc;
  return vomni_cm_attend_strided(q, k, v, b, s_q, s_kv, 0, s_kv, h, d, q_stride, kv_stride, softmax_scale, qn2, kmax2,
                                 nullptr, nullptr, flags | VOMNI_CM_FINAL, out, lse, stream);
}

extern "C" int vomni_cm_attention_local(const void* q, const void* k, const void* v, void* out, float* lse, int b, int s,
                                        int h, int d, float softmax_scale, int flags, void* workspace,
                                        size_t workspace_bytes, vomni_stream_t stream) {
  return vomni_cm_attention_local_strided(q, k, v, out, lse, b, s, h, d, 0, 0, softmax_scale, flags, workspace,
                                          workspace_bytes, stream);
}

// ---------------------------------------------------------------- exp2 self-test
namespace vomni {
namespace cm {
__global__ void exp2_poly_selftest_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = 2 * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  float p0, p1;
  exp2_poly2(x[i], i + 1 < n ? x[i + 1] : 0.f, p0, p1);
  y[i] = p0;
  if (i + 1 < n) y[i + 1] = p1;
}
}  // namespace cm
}  // namespace vomni

extern "C" int vomni_selftest_exp2_poly(const float* x, float* y, long long n, vomni_stream_t stream) {
  if (!x || !y) return VOMNI_EINVAL;
  if (n <= 0 || n > (1ll << 40)) return VOMNI_EBADSHAPE;
  const int threads = 256;
  const long long blocks = ((n + 1) / 2 + threads - 1) / threads;
  if (blocks > 0x7fffffffll) return VOMNI_EBADSHAPE;
  cm::exp2_poly_selftest_kernel<<<static_cast<unsigned>(blocks), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, y, n);
  VOMNI_CUDA_TRY(cudaGetLastError());
  return VOMNI_OK;
}

// ---------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory: a plugin inside a host runtime that owns the whole
// device heap (an inference server's pool, a C plugin ABI with no allocator hook), or a
// latency-critical path that must not hit cudaMalloc's implicit device synchronisation. For them
// the prologue scratch (per-token ||q||^2 and per-head max ||k||^2) lives in this file-scope array
// instead of a caller workspace: 8 MiB on every device that loads the library, held until exit.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_cm_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlot {
  unsigned long long ctx_id;  // driver context the address belongs to (0: not resolved yet)
  void* ptr;
};
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current driver context (0 if none or unavailable). A device
// reset (cudaDeviceReset) destroys the primary context and the next runtime call creates a new one
// with a new id, so an address cached under the old id is never reused.
unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array on the current device. In host code the array's name is only
// a host-side stand-in, so the address is looked up with cudaGetSymbolAddress, with the device
// current, the first time a device (or a device's new context after a reset) is seen, and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  VOMNI_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return VOMNI_ENOTSUP;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  const unsigned long long id = current_ctx_id();
  if (!slot.ptr || id == 0 || id != slot.ctx_id) {
    void* p = nullptr;
    VOMNI_CUDA_TRY(cudaGetSymbolAddress(&p, g_cm_noalloc_scratch));
    slot.ptr = p;
    slot.ctx_id = current_ctx_id();  // the lookup makes the runtime's context current if it was not
  }
  *out = slot.ptr;
  return VOMNI_OK;
}
}  // namespace

extern "C" int vomni_cm_attention_local_noalloc(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                                int s, int h, int d, float softmax_scale, int flags,
                                                vomni_stream_t stream) {
  const size_t need = vomni_cm_workspace_bytes(b, s, h, d);
  if (need == 0) return VOMNI_EBADSHAPE;
  if (need > kNoAllocScratchBytes) return VOMNI_EWORKSPACE;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // The prologue clears the key-max slots before it max-accumulates; qn2 is fully overwritten.
  return vomni_cm_attention_local(q, k, v, out, lse, b, s, h, d, softmax_scale, flags, scratch, need, stream);
}
