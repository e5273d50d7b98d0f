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
// Persistent 128-thread CTAs stream rows (<= 16384 values) through a shared-memory ring filled by
// bulk async copies; a row's values stay in registers between the passes, block reductions go
// through shared memory. HBM-bound: every byte is read or written once.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_util.h"

namespace vomni {
namespace adaln {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;  // the block reductions read the four warp partials as one float4

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
  int* status;                  // device status word (bounded-wait timeouts)
  int slots;                    // ring slots, 2..kMaxSlots
};

constexpr int kMaxSlots = 4;

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
// Block-wide reduction; `red` holds the kWarps (= 4) warp partials, 16-byte aligned. Ends with every
// thread holding the result (all threads combine the partials in the same order).
// One __syncthreads per reduction: each reduction of a row writes its own slot of `red`, and
// consecutive uses of one slot are always separated by another reduction's barrier.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = kMax ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const float4 r = *reinterpret_cast<const float4*>(red);
  return kMax ? fmaxf(fmaxf(r.x, r.y), fmaxf(r.z, r.w)) : (r.x + r.y) + (r.z + r.w);
}

// sm_100 mixed-precision arithmetic on packed bf16 pairs: the bf16 operand is widened exactly and the
// result rounded once to fp32, so no separate unpacking instructions are needed.
// lo = bf16 lo half of `pk` - c, hi = bf16 hi half - c.
VOMNI_DEV void sub_bf16x2_f32(uint32_t pk, float c, float& lo, float& hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tsub.rn.f32.bf16 %0, l, %3;\n\tsub.rn.f32.bf16 %1, h, %3;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "r"(pk), "f"(c));
}
// Both halves of `pk` widened to fp32 (x + (-0) == x for every x, signed zeros included).
VOMNI_DEV void widen_bf16x2(uint32_t pk, float& lo, float& hi) {
  lo = -0.f;
  hi = -0.f;
  add_bf16x2_f32(lo, hi, pk);
}

constexpr int kSiteRowWait = 0x30;   // a row's bulk copy never completed
constexpr int kSiteRowDrain = 0x31;  // an aborted CTA's copies still in flight at exit
constexpr uint32_t kBf16x2NegZero = 0x80008000u;  // (-0, -0): adding it leaves every value unchanged

// 128 threads per row: thread t owns the 16-byte chunks t, t + 128, ... (NV of them; kFull when they
// tile the row exactly, so no chunk needs a bounds predicate). Persistent: CTA c handles rows c,
// c + gridDim.x, ... One thread moves each row (hidden, and residual) into a p.slots-slot shared-memory
// ring with a single bulk async copy completing on the slot's mbarrier, so p.slots-1 rows per CTA are
// in flight while one is reduced, and the warps spend their issue slots on arithmetic only. Registers
// stay at or under 128 for rows up to 6144 values, so four CTAs (16 warps) share an SM.
// Ring reuse: a slot is refilled at the start of the row after the one that read it; every thread
// finishes its ring reads before the first barrier of its row, which thread 0 has passed by then.
template <int NV, bool kRes, bool kFull>
__global__ void __launch_bounds__(kThreads, NV <= 6 ? 4 : 1) adaln_kernel(const Params p) {
  extern __shared__ __align__(128) uint4 ring[];  // [slots][H/8] hidden, then [slots][H/8] residual
  __shared__ __align__(8) uint64_t full[kMaxSlots];
  __shared__ int abort_flag;
  // Reduction slots, double-buffered by row parity: a row may take a single barrier, and a slot
  // is rewritten only two rows later, after every thread has passed the next row's barrier.
  __shared__ __align__(16) float red_sq[2][kWarps];      // LayerNorm sum / RMS sum of squares
  __shared__ __align__(16) float red_stat_v[2][kWarps];  // LayerNorm squared deviations
  __shared__ __align__(16) float red_max[2][kWarps];     // absmax for the row quant
  if (static_cast<long long>(blockIdx.x) >= p.rows) return;
  const int H = p.H;
  const int nchunk = H >> 3;
  constexpr int nt = kThreads;
  const long long G = gridDim.x;
  const uint32_t row_bytes = static_cast<uint32_t>(H) * 2u;
  volatile int* abort = &abort_flag;
  const int nslot = p.slots;  // ring depth (runtime: 2..kMaxSlots)

  if (threadIdx.x == 0) {
    for (int s = 0; s < nslot; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Thread 0: bring local row kk (global row blockIdx.x + kk * G) into ring slot s (= kk mod nslot).
  auto issue = [&](long long kk, int s) {
    const long long r = blockIdx.x + kk * G;
    if (r >= p.rows) return;
    mbar_expect_tx(&full[s], kRes ? 2u * row_bytes : row_bytes);
    bulk_g2s(ring + s * nchunk, p.hidden + static_cast<size_t>(r) * H, row_bytes, &full[s]);
    if (kRes) bulk_g2s(ring + (nslot + s) * nchunk, p.residual + static_cast<size_t>(r) * H, row_bytes, &full[s]);
  };
  if (threadIdx.x == 0) {
    for (int kk = 0; kk < nslot - 1; ++kk) issue(kk, kk);
  }

  int parity = 0;
  long long cached_mrow = -1;
  // Modulation as packed bf16 pairs, widened where used (it leaves registers for a fourth CTA):
  // multiplier 1 and shift -0 when absent, so the arithmetic below is exact without them.
  uint32_t mulw[NV][4];
  uint32_t addw[NV][4];
  const float invH = 1.f / static_cast<float>(H);
  long long k = 0;
  int slot = 0;        // ring slot of local row k
  uint32_t phase = 0;  // the mbarrier phase parity of that slot's current use
  for (long long row = blockIdx.x; row < p.rows; row += G, ++k) {
    if (threadIdx.x == 0) {
      fence_proxy_async_smem();  // the generic-proxy reads of the refilled slot happen before this copy
      issue(k + nslot - 1, slot == 0 ? nslot - 1 : slot - 1);
    }
    mbar_wait(&full[slot], phase, abort, p.status, VOMNI_DEV_TIMEOUT_BASE + kSiteRowWait);
    const size_t base = static_cast<size_t>(row) * H;
    const long long mrow = p.rows_per_mod >= p.rows ? 0 : row / p.rows_per_mod;

    // ---- this thread's chunks of the row, as packed bf16 pairs (after the gated residual)
    uint32_t xw[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = threadIdx.x + i * nt;
      const bool in = kFull || c < nchunk;
      const uint4 hv = in ? ring[slot * nchunk + c] : make_uint4(0, 0, 0, 0);
      xw[i][0] = hv.x; xw[i][1] = hv.y; xw[i][2] = hv.z; xw[i][3] = hv.w;
      if (kRes && in) {
        const uint4 rv = ring[(nslot + slot) * nchunk + c];
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
        float g[8];
        if (p.gate) {
          const float4* gp = reinterpret_cast<const float4*>(p.gate + static_cast<size_t>(mrow) * H + c * 8);
          const float4 g0 = __ldg(gp), g1 = __ldg(gp + 1);
          g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          float lo, hi;
          widen_bf16x2(xw[i][w], lo, hi);
          if (p.gate) {  // product and sum rounded separately, as the reference computes them
            lo = __fmul_rn(lo, g[2 * w]);
            hi = __fmul_rn(hi, g[2 * w + 1]);
          }
          add_bf16x2_f32(lo, hi, rw[w]);  // residual + gate * hidden, rounded once to fp32
          xw[i][w] = pack_bf16x2(lo, hi);
        }
        reinterpret_cast<uint4*>(p.residual_out + base)[c] = make_uint4(xw[i][0], xw[i][1], xw[i][2], xw[i][3]);
      }
    }
    if (mrow != cached_mrow) {
      cached_mrow = mrow;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * nt;
        const bool in = kFull || c < nchunk;
        uint4 mv = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);  // bf16 (1, 1)
        uint4 av = make_uint4(kBf16x2NegZero, kBf16x2NegZero, kBf16x2NegZero, kBf16x2NegZero);
        if (p.mul && in) mv = __ldg(reinterpret_cast<const uint4*>(p.mul + static_cast<size_t>(mrow) * H) + c);
        if (p.add && in) av = __ldg(reinterpret_cast<const uint4*>(p.add + static_cast<size_t>(mrow) * H) + c);
        mulw[i][0] = mv.x; mulw[i][1] = mv.y; mulw[i][2] = mv.z; mulw[i][3] = mv.w;
        addw[i][0] = av.x; addw[i][1] = av.y; addw[i][2] = av.z; addw[i][3] = av.w;
      }
    }

    // ---- statistics (fp32, two-pass mean / squared deviations) and the centred values d
    float d[NV][8];
    float mean = 0.f, rstd = 1.f;
    if (p.norm == 0) {
      float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        add_bf16x2_f32(sm[0], sm[1], xw[i][0]);
        add_bf16x2_f32(sm[2], sm[3], xw[i][1]);
        add_bf16x2_f32(sm[0], sm[1], xw[i][2]);
        add_bf16x2_f32(sm[2], sm[3], xw[i][3]);
      }
      mean = block_reduce<false>((sm[0] + sm[1]) + (sm[2] + sm[3]), red_sq[parity]) * invH;
      if (*abort) break;  // uniform: every thread has passed the barrier above
      uint64_t m2[2] = {0ull, 0ull};
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const bool in = kFull || threadIdx.x + i * nt < nchunk;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          sub_bf16x2_f32(xw[i][w], mean, d[i][2 * w], d[i][2 * w + 1]);
          if (!in) d[i][2 * w] = d[i][2 * w + 1] = 0.f;
          const uint64_t dd = f2_pack(d[i][2 * w], d[i][2 * w + 1]);
          m2[w & 1] = f2_fma(dd, dd, m2[w & 1]);
        }
      }
      float a0, a1, b0, b1;
      f2_unpack(m2[0], a0, a1);
      f2_unpack(m2[1], b0, b1);
      rstd = rsqrtf(block_reduce<false>((a0 + a1) + (b0 + b1), red_stat_v[parity]) * invH + p.eps);
    } else {
      uint64_t v2[2] = {0ull, 0ull};
#pragma unroll
      for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          widen_bf16x2(xw[i][w], d[i][2 * w], d[i][2 * w + 1]);
          if (p.norm == 1) {
            const uint64_t dd = f2_pack(d[i][2 * w], d[i][2 * w + 1]);
            v2[w & 1] = f2_fma(dd, dd, v2[w & 1]);
          }
        }
      if (p.norm == 1) {
        float a0, a1, b0, b1;
        f2_unpack(v2[0], a0, a1);
        f2_unpack(v2[1], b0, b1);
        rstd = rsqrtf(block_reduce<false>((a0 + a1) + (b0 + b1), red_sq[parity]) * invH + p.eps);
      } else {
        __syncthreads();  // no reduction in this row: the barrier that orders ring reads before refills
      }
      if (*abort) break;
    }

    // ---- normalise, modulate (y * mul, then + add, each rounded, as the reference computes them);
    // rstd is 1 without a norm, so every multiply and add here is exact when its operand is absent.
    const uint64_t rstd2 = f2_pack(rstd, rstd);
    float am[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const bool in = kFull || threadIdx.x + i * nt < nchunk;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float lo, hi;
        float mlo, mhi;
        widen_bf16x2(mulw[i][w], mlo, mhi);
        f2_unpack(f2_mul(f2_mul(f2_pack(d[i][2 * w], d[i][2 * w + 1]), rstd2), f2_pack(mlo, mhi)), lo, hi);
        add_bf16x2_f32(lo, hi, addw[i][w]);
        if (!in) lo = hi = 0.f;
        d[i][2 * w] = lo;
        d[i][2 * w + 1] = hi;
        am[(2 * w) & 3] = fmaxf(am[(2 * w) & 3], fabsf(lo));
        am[(2 * w + 1) & 3] = fmaxf(am[(2 * w + 1) & 3], fabsf(hi));
      }
    }
    // ---- quantise + store
    if (p.quant == 0) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * nt;
        if (!(kFull || c < nchunk)) continue;
        const uint4 o = make_uint4(pack_bf16x2(d[i][0], d[i][1]), pack_bf16x2(d[i][2], d[i][3]),
                                   pack_bf16x2(d[i][4], d[i][5]), pack_bf16x2(d[i][6], d[i][7]));
        __stcs(reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + base) + c, o);
      }
    } else if (p.quant == 1) {
      const float amax = block_reduce<true>(fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3])), red_max[parity]);
      const float scale = fmaxf(amax / p.fp8_range, 1e-6f);
      // codes = y * (1 / scale), the reciprocal-multiply of the reference kernel (adaln_quant.py:520-536)
      const float inv = __frcp_rn(scale);
      const uint64_t inv2 = f2_pack(inv, inv);
      uint8_t* orow = static_cast<uint8_t*>(p.out) + static_cast<size_t>(row) * (p.packed ? H + 4 : H);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = threadIdx.x + i * nt;
        if (!(kFull || c < nchunk)) continue;
        uint32_t q[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          float lo, hi;
          f2_unpack(f2_mul(f2_pack(d[i][2 * w], d[i][2 * w + 1]), inv2), lo, hi);
          q[w] = e4m3x2(lo, hi);
        }
        const uint32_t w0 = q[0] | (q[1] << 16), w1 = q[2] | (q[3] << 16);
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
        const int c = threadIdx.x + i * nt;
        const bool in = kFull || c < nchunk;
        int e = 0;
        if (in) {
#pragma unroll
          for (int j = 0; j < 8; ++j) e = max(e, static_cast<int>((__float_as_uint(d[i][j]) >> 23) & 0xFF));
        }
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 1));
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 2));
        if (!in) continue;
        const int su = min(max(e - 7, 0), 255);
        // y / 2^(su - 127) as two exact power-of-two multiplies (each factor a normal fp32).
        const int sh = 127 - su;  // in [-128, 127]
        const int sa = sh / 2, sb = sh - sa;
        const float fa = __uint_as_float(static_cast<uint32_t>(sa + 127) << 23);
        const float fb = __uint_as_float(static_cast<uint32_t>(sb + 127) << 23);
        float q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = fminf(fmaxf((d[i][j] * fa) * fb, -448.f), 448.f);
        const uint32_t w0 = e4m3x2(q[0], q[1]) | (static_cast<uint32_t>(e4m3x2(q[2], q[3])) << 16);
        const uint32_t w1 = e4m3x2(q[4], q[5]) | (static_cast<uint32_t>(e4m3x2(q[6], q[7])) << 16);
        reinterpret_cast<uint2*>(orow)[c] = make_uint2(w0, w1);
        if ((c & 3) == 0) srow[c >> 2] = static_cast<uint8_t>(su);
      }
    }
    parity ^= 1;
    if (++slot == nslot) {
      slot = 0;
      phase ^= 1;
    }
  }
  // An aborted CTA may still have copies in flight into its ring: rows k .. k + nslot - 1 were issued
  // when it gave up at row k. Wait for them (bounded) before the shared memory is released. A normal
  // exit has consumed every row it issued.
  if (*abort && threadIdx.x == 0) {
    int s = slot;
    uint32_t ph = phase;
    for (long long kk = k; kk < k + nslot; ++kk) {
      if (blockIdx.x + kk * G >= p.rows) break;
      int ignored = 0;
      if (!mbar_wait(&full[s], ph, &ignored, p.status, VOMNI_DEV_TIMEOUT_BASE + kSiteRowDrain)) break;
      if (++s == nslot) {
        s = 0;
        ph ^= 1;
      }
    }
  }
}

// Ring slots: four while four CTAs of them fit on an SM (a slot holds one row of hidden, and one of
// residual), three while three CTAs fit, else two. Persistent grid: as many CTAs as fit on the device
// at once, each streaming rows through its ring.
template <int NV>
int launch_nv(Params p, cudaStream_t st) {
  const bool full = (p.H >> 3) == NV * kThreads;
  const size_t slot_bytes = static_cast<size_t>(p.H) * 2 * (p.residual ? 2 : 1);
  p.slots = 4 * slot_bytes <= 56 * 1024 ? 4 : (3 * slot_bytes <= 72 * 1024 ? 3 : 2);
  auto kern = p.residual ? (full ? adaln_kernel<NV, true, true> : adaln_kernel<NV, true, false>)
                         : (full ? adaln_kernel<NV, false, true> : adaln_kernel<NV, false, false>);
  const size_t smem = static_cast<size_t>(p.slots) * slot_bytes;
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

int launch(const Params& p, cudaStream_t st) {
  switch (((p.H >> 3) + kThreads - 1) / kThreads) {  // NV: chunks per thread, 1..16 for H <= 16384
    case 1: return launch_nv<1>(p, st);
    case 2: return launch_nv<2>(p, st);
    case 3: return launch_nv<3>(p, st);
    case 4: return launch_nv<4>(p, st);
    case 5: return launch_nv<5>(p, st);
    case 6: return launch_nv<6>(p, st);
    case 7: return launch_nv<7>(p, st);
    case 8: return launch_nv<8>(p, st);
    case 9: return launch_nv<9>(p, st);
    case 10: return launch_nv<10>(p, st);
    case 11: return launch_nv<11>(p, st);
    case 12: return launch_nv<12>(p, st);
    case 13: return launch_nv<13>(p, st);
    case 14: return launch_nv<14>(p, st);
    case 15: return launch_nv<15>(p, st);
    case 16: return launch_nv<16>(p, st);
    default: return VOMNI_EBADSHAPE;
  }
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
  p.status = device_status_ptr();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return adaln::launch(p, st);
}
