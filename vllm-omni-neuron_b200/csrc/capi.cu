// Library-level C ABI: version, error strings, the device status word, device checks and TMA
// descriptor encoding shared by the kernel translation units.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "host_util.h"

// One status word per device that loads the library; bounded device waits write their error
// code here (first error wins) and vomni_device_status() reads / clears it.
__device__ int g_vomni_status;

namespace vomni {

namespace {
thread_local cudaError_t g_last_cuda_error = cudaSuccess;
constexpr int kMaxDevices = 64;
// Per-device caches, filled on first use by whichever host thread gets there first (every writer
// stores the same value), read lock-free afterwards.
std::atomic<int*> g_status_ptr[kMaxDevices] = {};
std::atomic<int> g_num_sms[kMaxDevices] = {};
std::atomic<int> g_is_sm100[kMaxDevices] = {};  // 0 unknown, 1 yes, -1 no
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}
}  // namespace

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = e; }

int num_sms() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_num_sms[dev].load(std::memory_order_acquire);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_num_sms[dev].store(n, std::memory_order_release);
  }
  return n;
}

int require_sm100() {
  const int dev = current_device();
  if (dev < 0) return VOMNI_ECUDA;
  if (dev < kMaxDevices) {
    const int known = g_is_sm100[dev].load(std::memory_order_acquire);
    if (known) return known > 0 ? VOMNI_OK : VOMNI_ENOTSUP;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return VOMNI_ECUDA;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return VOMNI_ECUDA;
  const bool ok = (major == 10 && minor == 0);
  if (dev < kMaxDevices) g_is_sm100[dev].store(ok ? 1 : -1, std::memory_order_release);
  return ok ? VOMNI_OK : VOMNI_ENOTSUP;
}

int* device_status_ptr() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  int* ptr = g_status_ptr[dev].load(std::memory_order_acquire);
  if (!ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    ptr = g_status_ptr[dev].load(std::memory_order_relaxed);
    if (!ptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_vomni_status) != cudaSuccess) return nullptr;
      ptr = static_cast<int*>(p);
      g_status_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  return ptr;
}

static int get_encoder() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode) return VOMNI_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    return VOMNI_ECUDA;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return VOMNI_OK;
}

int ensure_max_smem(const void* func, int bytes) {
  int dev = -1;
  VOMNI_CUDA_TRY(cudaGetDevice(&dev));
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, int>> done;
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& e : done)
    if (std::get<0>(e) == func && std::get<1>(e) == dev && std::get<2>(e) >= bytes) return VOMNI_OK;
  VOMNI_CUDA_TRY(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.emplace_back(func, dev, bytes);
  return VOMNI_OK;
}

StreamWriteValue32Fn stream_write_value32() {
  static StreamWriteValue32Fn fn_ptr = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn_ptr = reinterpret_cast<StreamWriteValue32Fn>(fn);
  });
  return fn_ptr;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2, uint32_t box0,
                      uint32_t box1, uint64_t row_pitch_elems) {
  int rc = get_encoder();
  if (rc) return rc;
  if (reinterpret_cast<uintptr_t>(base) & 15) return VOMNI_EALIGN;
  if (row_pitch_elems == 0) row_pitch_elems = dim0;
  if (row_pitch_elems < dim0 || (row_pitch_elems * 2) % 16) return VOMNI_EALIGN;
  cuuint64_t dims[3] = {dim0, dim1, dim2};
  cuuint64_t strides[2] = {row_pitch_elems * 2, row_pitch_elems * dim1 * 2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VOMNI_OK : VOMNI_ECUDA;
}

int make_tmap_3d_bf16_plain(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t dim2,
                            uint32_t box0, uint32_t box1) {
  int rc = get_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (dim0 * 2) % 16) return VOMNI_EALIGN;
  cuuint64_t dims[3] = {dim0, dim1, dim2};
  cuuint64_t strides[2] = {dim0 * 2, dim0 * dim1 * 2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VOMNI_OK : VOMNI_ECUDA;
}

int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                 uint64_t pitch_bytes, uint32_t box0, uint32_t box1) {
  int rc = get_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes % 16)) return VOMNI_EALIGN;
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VOMNI_OK : VOMNI_ECUDA;
}

int make_tmap_2d_plain(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                       uint64_t pitch_bytes, uint32_t box0, uint32_t box1) {
  int rc = get_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes % 16)) return VOMNI_EALIGN;
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VOMNI_OK : VOMNI_ECUDA;
}

}  // namespace vomni

extern "C" int vomni_abi_version(void) { return 1; }

extern "C" const char* vomni_strerror(int code) {
  switch (code) {
    case VOMNI_OK: return "ok";
    case VOMNI_EINVAL: return "invalid argument";
    case VOMNI_EBADSHAPE: return "unsupported shape";
    case VOMNI_EALIGN: return "pointer or stride not 16-byte aligned";
    case VOMNI_ECUDA: {
      static thread_local char buf[160];
      snprintf(buf, sizeof(buf), "CUDA error: %s", cudaGetErrorString(vomni::g_last_cuda_error));
      return buf;
    }
    case VOMNI_ENCCL: return "NCCL error";
    case VOMNI_ETIMEOUT: return "bounded wait timed out";
    case VOMNI_ENOTSUP: return "not supported on this device (needs sm_100)";
    case VOMNI_EWORKSPACE: return "workspace too small";
    case VOMNI_ESTATE: return "invalid context state";
    default: return "unknown error";
  }
}

extern "C" int vomni_device_status(int* code, int clear) {
  if (!code) return VOMNI_EINVAL;
  int* p = vomni::device_status_ptr();
  if (!p) return VOMNI_ECUDA;
  VOMNI_CUDA_TRY(cudaDeviceSynchronize());
  VOMNI_CUDA_TRY(cudaMemcpy(code, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) VOMNI_CUDA_TRY(cudaMemset(p, 0, sizeof(int)));
  return VOMNI_OK;
}

// ---------------------------------------------------------------- bounded-wait self-test
// A CTA waits on an mbarrier that nothing ever arrives on, with a short budget. The bounded wait
// must give up, record VOMNI_DEV_TIMEOUT_BASE + 0x7F in the status word and let the kernel end,
// leaving the context usable. This exercises the failure path of every kernel's waits without
// faulting, trapping or hanging the GPU.
__global__ void selftest_wait_kernel(uint64_t budget_ns, int* status, int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    vomni::mbar_init(&bar, 1);
    abort_flag = 0;
    vomni::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = vomni::mbar_wait(&bar, 0, &abort_flag, status, VOMNI_DEV_TIMEOUT_BASE + 0x7F, budget_ns);
  __syncthreads();
  if (threadIdx.x == 0) *result = ok ? 1 : 0;
}

extern "C" int vomni_selftest_bounded_wait(unsigned budget_us, int* result_host, vomni_stream_t stream) {
  if (!result_host || budget_us == 0 || budget_us > 2000000u) return VOMNI_EINVAL;
  int* st = vomni::device_status_ptr();
  if (!st) return VOMNI_ECUDA;
  int* d = nullptr;
  VOMNI_CUDA_TRY(cudaMalloc(&d, sizeof(int)));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 64, 0, s>>>(static_cast<uint64_t>(budget_us) * 1000ull, st, d);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpyAsync(result_host, d, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(d);
  VOMNI_CUDA_TRY(e);
  return VOMNI_OK;
}

__global__ void selftest_ready_kernel(const unsigned* word, uint64_t budget_ns, int* status, int* result) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  if (threadIdx.x == 0)
    *result = vomni::ready_wait(word, 1u, &abort_flag, status, VOMNI_DEV_TIMEOUT_BASE + 0x7E, budget_ns) ? 1 : 0;
}

extern "C" int vomni_selftest_ready_wait(unsigned budget_us, int post, int* result_host, vomni_stream_t stream) {
  if (!result_host || budget_us == 0 || budget_us > 2000000u || (post != 0 && post != 1)) return VOMNI_EINVAL;
  int* st = vomni::device_status_ptr();
  if (!st) return VOMNI_ECUDA;
  const vomni::StreamWriteValue32Fn write_value = vomni::stream_write_value32();
  if (post && !write_value) return VOMNI_ENOTSUP;
  int* d = nullptr;
  VOMNI_CUDA_TRY(cudaMalloc(&d, 2 * sizeof(int)));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned* word = reinterpret_cast<unsigned*>(d + 1);
  cudaError_t e = cudaMemsetAsync(d, 0, 2 * sizeof(int), s);
  if (e == cudaSuccess && post &&
      write_value(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(word), 1u, 0) != CUDA_SUCCESS)
    e = cudaErrorUnknown;
  if (e == cudaSuccess) {
    selftest_ready_kernel<<<1, 32, 0, s>>>(word, static_cast<uint64_t>(budget_us) * 1000ull, st, d);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(result_host, d, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(d);
  VOMNI_CUDA_TRY(e);
  return VOMNI_OK;
}

extern "C" int vomni_memcpy_2d_async(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                                     size_t height, vomni_stream_t stream) {
  if (!dst || !src) return VOMNI_EINVAL;
  if (width > dpitch || width > spitch) return VOMNI_EBADSHAPE;
  if (width == 0 || height == 0) return VOMNI_OK;
  VOMNI_CUDA_TRY(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault,
                                   reinterpret_cast<cudaStream_t>(stream)));
  return VOMNI_OK;
}
