// Host-side helpers shared by the C-ABI translation units: error mapping, device checks,
// TMA descriptor encoding (driver entry point fetched at run time, so the library does not link
// libcuda directly) and the per-device status word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/vomni_b200.h"

#define VOMNI_CUDA_TRY(expr)                      \
  do {                                            \
    cudaError_t vomni_err_ = (expr);              \
    if (vomni_err_ != cudaSuccess) {              \
      vomni::set_last_cuda_error(vomni_err_);     \
      return VOMNI_ECUDA;                         \
    }                                             \
  } while (0)

namespace vomni {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

void set_last_cuda_error(cudaError_t e);
int num_sms();
// VOMNI_OK on an sm_100 device, VOMNI_ENOTSUP otherwise.
int require_sm100();
// Device address of the library status word on the current device (nullptr if unavailable).
int* device_status_ptr();

// Rank-3 bf16 tensor map over a [dim2][dim1][dim0] tensor whose dim1 rows are row_pitch_elems
// elements apart (0 = dense), box {box0, box1, 1}, 128-byte swizzle, out-of-bounds reads as zero.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2, uint32_t box0,
                      uint32_t box1, uint64_t row_pitch_elems = 0);
// Rank-3 bf16 tensor map over a dense [dim2][dim1][dim0] tensor without swizzle (boxes land in
// shared memory as plain row-major [box1][box0]), OOB reads as zero.
int make_tmap_3d_bf16_plain(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2,
                            uint32_t box0, uint32_t box1);
// Rank-2 tensor map over a [dim1][dim0] row-major tensor of 1- or 2-byte elements with an
// explicit row pitch in bytes, box {box0, box1}, 128-byte swizzle, OOB reads as zero.
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                 uint64_t pitch_bytes, uint32_t box0, uint32_t box1);
// Same without swizzle (plain row-major boxes), e.g. for 512-byte scale-factor atoms.
int make_tmap_2d_plain(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                       uint64_t pitch_bytes, uint32_t box0, uint32_t box1);

// vomni_cm_attend_strided with an optional in-kernel gate: when `ready` is set, every CTA waits
// (bounded) for ready[0 .. ready_count) >= ready_epoch before its first K/V load. Used by the ring, whose copy stream
// posts the word after a block's copies, so that no stream-level wait separates consecutive passes.
int cm_attend_gated(const void* q, const void* k, const void* v, int b, int s_q, int s_kv, int k_start, int n_keys,
                    int h, int d, long long q_stride, long long kv_stride, float softmax_scale, const float* qn2,
                    const float* kmax2, float* acc_o, float* acc_l, int flags, void* out, float* lse,
                    const unsigned* ready, int ready_count, unsigned ready_epoch, vomni_stream_t stream);
// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes) once per (kernel, device, size);
// thread-safe. Kernels above 48 KB of dynamic shared memory need it on every device they run on.
int ensure_max_smem(const void* func, int bytes);
template <typename F>
inline int ensure_max_smem(F* func, int bytes) {
  return ensure_max_smem(reinterpret_cast<const void*>(func), bytes);
}
// cuStreamWriteValue32 (driver entry point fetched at run time); nullptr if unavailable.
typedef CUresult (*StreamWriteValue32Fn)(CUstream stream, CUdeviceptr addr, cuuint32_t value, unsigned int flags);
StreamWriteValue32Fn stream_write_value32();

}  // namespace vomni
