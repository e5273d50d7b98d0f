// Context-parallel ring of the const-max attention over the GPUs of one NVSwitch box.
//
// Reference: the ring driver of ring_attention_const_max_fwd
// (vllm_omni_neuron/kernels/nkilib/experimental/attention/ring_attention_const_max_fwd.py:1287-1398):
// K/V blocks rotate N-1 hops with collective_permute (each rank forwards to the next), the only
// reduction is all_reduce(max) of the per-head key norm (:1196-1205), and partial attention of the
// ring steps combines by plain addition because the softmax bound is static.
//
// B200 design: NVSwitch gives every GPU full bandwidth to every peer, so the store-and-forward ring
// becomes direct pulls: step s copies block (r - s) mod N straight from its owner's registered send
// buffer into a local gather buffer, on copy-engine streams (cudaMemcpyAsync between IPC-mapped
// device memory; no SMs, no TMA on peer memory, no multicast). The steps can be spread round-robin
// over kCopyStreams streams; on 8 B200s one stream (blocks land one after another, in the order the
// passes read them) measured faster than four (2.53 vs 2.91-3.00 ms per C2 layer), so one is built. The attention runs as a few passes
// over ranges of arrived blocks (local block first, then ranges of 1, 2, 4, ... blocks), accumulating
// into an fp32 partial; the last pass normalises. After a block's copies its copy stream posts a
// per-step ready word (cuStreamWriteValue32, executed by the GPU front end, not by a kernel); each
// pass waits for the words of all its blocks inside the kernel (bounded), before its first K/V load, so
// no stream-level wait separates consecutive passes and a pass starts as a programmatic dependent
// of the previous one, filling the SMs its last wave leaves idle.
//
// Ordering guarantees (no device-side cross-GPU waits anywhere):
//  * peers' send buffers are complete before this rank copies them: each rank writes its send
//    buffer, then enters the NCCL all_reduce(max); the all_reduce completing on this rank implies
//    every peer reached it, i.e. finished its earlier stream work;
//  * send buffers are double-buffered by call parity: a rank rewrites send[p] two calls later, after
//    the intervening call's all_reduce, by which time every peer's copies of send[p] have completed
//    (each rank's stream joins its copy streams after the last pass, before it can enter the next
//    all_reduce).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "host_util.h"

namespace vomni {
namespace {

// Copy streams per ring (at most world - 1 are used); a build-time constant.
#ifndef VOMNI_RING_COPY_STREAMS
#define VOMNI_RING_COPY_STREAMS 1
#endif
constexpr int kCopyStreams = VOMNI_RING_COPY_STREAMS;
static_assert(kCopyStreams >= 1 && kCopyStreams <= 8, "copy streams per ring");

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  bool ok = false;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

// NCCL is resolved at run time: the soname lookup returns the copy already loaded by the host
// framework when there is one, else the system library.
const NcclApi* nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.ok) return &g_nccl;
  if (!g_nccl.handle) {
    g_nccl.handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!g_nccl.handle) return nullptr;
  }
  auto sym = [](const char* n) { return dlsym(g_nccl.handle, n); };
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(sym("ncclGetUniqueId"));
  g_nccl.CommInitRank = reinterpret_cast<decltype(g_nccl.CommInitRank)>(sym("ncclCommInitRank"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(sym("ncclCommDestroy"));
  g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(sym("ncclCommAbort"));
  g_nccl.CommGetAsyncError = reinterpret_cast<decltype(g_nccl.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
  g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(sym("ncclAllReduce"));
  g_nccl.AllGather = reinterpret_cast<decltype(g_nccl.AllGather)>(sym("ncclAllGather"));
  g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.CommAbort &&
              g_nccl.CommGetAsyncError && g_nccl.AllReduce && g_nccl.AllGather;
  return g_nccl.ok ? &g_nccl : nullptr;
}

}  // namespace
}  // namespace vomni

using namespace vomni;

struct vomni_ring {
  int rank = 0, world = 1, device = 0;
  int b = 0, s_max = 0, h = 0, d = 0;
  ncclComm_t comm = nullptr;
  cudaStream_t copy_stream = nullptr;  // copy_streams[0]
  std::vector<cudaStream_t> copy_streams;
  cudaEvent_t ev_inputs = nullptr;  // recorded on the caller stream at entry (K/V written)
  cudaEvent_t ev_sent = nullptr;    // recorded on copy stream 0 after the send-buffer copies
  cudaEvent_t ev_ready = nullptr;   // recorded on the caller stream after the all_reduce
  std::vector<cudaEvent_t> ev_block;  // copy of ring step s done
  std::vector<cudaEvent_t> ev_copies_done;  // per copy stream: its last copy done
  unsigned* ready = nullptr;  // [world] device words: ready[s] = call number once step s's block landed
  // Registered send buffer: [parity 2][K|V 2][b, s_max, h, d] bf16 (one allocation, IPC-exported).
  void* send = nullptr;
  size_t block_bytes = 0;  // one K or V block at s_max
  std::vector<void*> peer_send;  // per rank (own entry = send)
  // Gather buffers [b, (world-1)*s_max, h, d] for K and V, and workspace.
  void* gather_k = nullptr;
  void* gather_v = nullptr;
  float* qn2 = nullptr;
  float* kmax2 = nullptr;
  float* acc_o = nullptr;
  float* acc_l = nullptr;
  unsigned long long calls = 0;
  bool broken = false;
};

namespace {

int nccl_check(ncclResult_t r) { return r == ncclSuccess ? VOMNI_OK : VOMNI_ENCCL; }

void ring_free(vomni_ring* R) {
  if (!R) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(R->device);
  for (size_t i = 0; i < R->peer_send.size(); ++i)
    if (R->peer_send[i] && static_cast<int>(i) != R->rank) cudaIpcCloseMemHandle(R->peer_send[i]);
  if (R->send) cudaFree(R->send);
  if (R->gather_k) cudaFree(R->gather_k);
  if (R->gather_v) cudaFree(R->gather_v);
  if (R->qn2) cudaFree(R->qn2);
  if (R->kmax2) cudaFree(R->kmax2);
  if (R->acc_o) cudaFree(R->acc_o);
  if (R->acc_l) cudaFree(R->acc_l);
  if (R->ready) cudaFree(R->ready);
  for (cudaEvent_t e : R->ev_block) cudaEventDestroy(e);
  for (cudaEvent_t e : R->ev_copies_done) cudaEventDestroy(e);
  if (R->ev_ready) cudaEventDestroy(R->ev_ready);
  if (R->ev_inputs) cudaEventDestroy(R->ev_inputs);
  if (R->ev_sent) cudaEventDestroy(R->ev_sent);
  for (cudaStream_t cs : R->copy_streams) cudaStreamDestroy(cs);
  if (R->comm) {
    const NcclApi* n = nccl();
    if (n) (R->broken ? n->CommAbort : n->CommDestroy)(R->comm);
  }
  cudaSetDevice(prev);
  delete R;
}

}  // namespace

extern "C" int vomni_ring_phase_plan(int world, int* first, int* count, int max_phases) {
  // Pass 0 is the local block; passes 1.. cover gather slots [first, first+count) with counts
  // 1, 2, 4, ... (the last pass takes the remainder). Returns the number of passes.
  if (world < 1 || !first || !count || max_phases < 1) return -VOMNI_EINVAL;
  int n = 0;
  first[n] = -1;
  count[n] = 1;
  ++n;
  int slot = 0, size = 1;
  while (slot < world - 1) {
    if (n >= max_phases) return -VOMNI_EINVAL;
    const int c = (slot + size > world - 1) ? world - 1 - slot : size;
    first[n] = slot;
    count[n] = c;
    ++n;
    slot += c;
    size *= 2;
  }
  return n;
}

extern "C" int vomni_ring_source_rank(int rank, int world, int step) {
  // Ring step `step` consumes the block that started on rank (rank - step) mod world
  // (collective_permute to the next rank, ring_attention_const_max_fwd.py:130-144).
  if (world < 1 || rank < 0 || rank >= world) return -1;
  return ((rank - step) % world + world) % world;
}

extern "C" int vomni_nccl_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId)) return VOMNI_EINVAL;
  const NcclApi* n = nccl();
  if (!n) return VOMNI_ENCCL;
  ncclUniqueId id;
  if (n->GetUniqueId(&id) != ncclSuccess) return VOMNI_ENCCL;
  memcpy(out, &id, sizeof(id));
  return VOMNI_OK;
}

extern "C" int vomni_ring_create(vomni_ring** out, int rank, int world, const void* nccl_id, size_t id_bytes, int b,
                                 int s_max, int h, int d) {
  if (!out || !nccl_id || id_bytes < sizeof(ncclUniqueId)) return VOMNI_EINVAL;
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return VOMNI_EINVAL;
  if (b <= 0 || s_max <= 0 || h <= 0 || d != 128) return VOMNI_EBADSHAPE;
  int rc = require_sm100();
  if (rc) return rc;
  const NcclApi* n = nccl();
  if (!n) return VOMNI_ENCCL;
  vomni_ring* R = new vomni_ring();
  R->rank = rank;
  R->world = world;
  R->b = b;
  R->s_max = s_max;
  R->h = h;
  R->d = d;
  cudaGetDevice(&R->device);
#define RING_TRY(expr)               \
  do {                               \
    int rc_ = (expr);                \
    if (rc_) {                       \
      R->broken = true;              \
      ring_free(R);                  \
      return rc_;                    \
    }                                \
  } while (0)
#define RING_CUDA(expr)                                \
  do {                                                 \
    cudaError_t e_ = (expr);                           \
    if (e_ != cudaSuccess) {                           \
      set_last_cuda_error(e_);                         \
      R->broken = true;                                \
      ring_free(R);                                    \
      return VOMNI_ECUDA;                              \
    }                                                  \
  } while (0)
  ncclUniqueId id;
  memcpy(&id, nccl_id, sizeof(id));
  RING_TRY(nccl_check(n->CommInitRank(&R->comm, world, id, rank)));
  const size_t toks = static_cast<size_t>(b) * s_max;
  R->block_bytes = toks * h * d * 2;
  const int ncs = world > 1 ? (world - 1 < kCopyStreams ? world - 1 : kCopyStreams) : 1;
  R->copy_streams.resize(ncs, nullptr);
  R->ev_copies_done.resize(ncs, nullptr);
  for (int i = 0; i < ncs; ++i) {
    RING_CUDA(cudaStreamCreateWithFlags(&R->copy_streams[i], cudaStreamNonBlocking));
    RING_CUDA(cudaEventCreateWithFlags(&R->ev_copies_done[i], cudaEventDisableTiming));
  }
  R->copy_stream = R->copy_streams[0];
  RING_CUDA(cudaEventCreateWithFlags(&R->ev_ready, cudaEventDisableTiming));
  RING_CUDA(cudaEventCreateWithFlags(&R->ev_inputs, cudaEventDisableTiming));
  RING_CUDA(cudaEventCreateWithFlags(&R->ev_sent, cudaEventDisableTiming));
  R->ev_block.resize(world, nullptr);
  for (int i = 0; i < world; ++i) RING_CUDA(cudaEventCreateWithFlags(&R->ev_block[i], cudaEventDisableTiming));
  RING_CUDA(cudaMalloc(&R->qn2, static_cast<size_t>(b) * h * s_max * sizeof(float)));
  RING_CUDA(cudaMalloc(&R->kmax2, static_cast<size_t>(b) * h * sizeof(float)));
  if (world > 1) {
    RING_CUDA(cudaMalloc(&R->send, 4 * R->block_bytes));
    RING_CUDA(cudaMalloc(&R->gather_k, R->block_bytes * (world - 1)));
    RING_CUDA(cudaMalloc(&R->gather_v, R->block_bytes * (world - 1)));
    RING_CUDA(cudaMalloc(&R->acc_o, static_cast<size_t>(b) * h * s_max * d * sizeof(float)));
    RING_CUDA(cudaMalloc(&R->acc_l, static_cast<size_t>(b) * h * s_max * sizeof(float)));
    RING_CUDA(cudaMalloc(&R->ready, sizeof(unsigned) * world));
    RING_CUDA(cudaMemsetAsync(R->ready, 0, sizeof(unsigned) * world, R->copy_stream));  // synchronised below
    // Exchange IPC handles of the send buffers with one all_gather (handles staged through device memory).
    cudaIpcMemHandle_t mine;
    RING_CUDA(cudaIpcGetMemHandle(&mine, R->send));
    void* dh = nullptr;
    RING_CUDA(cudaMalloc(&dh, sizeof(cudaIpcMemHandle_t) * (world + 1)));
    RING_CUDA(cudaMemcpy(dh, &mine, sizeof(mine), cudaMemcpyHostToDevice));
    uint8_t* all_dev = static_cast<uint8_t*>(dh) + sizeof(cudaIpcMemHandle_t);
    ncclResult_t nr = n->AllGather(dh, all_dev, sizeof(cudaIpcMemHandle_t), ncclUint8, R->comm, R->copy_stream);
    if (nr != ncclSuccess) {
      cudaFree(dh);
      RING_TRY(VOMNI_ENCCL);
    }
    std::vector<cudaIpcMemHandle_t> all(world);
    cudaError_t e1 = cudaStreamSynchronize(R->copy_stream);
    cudaError_t e2 = cudaMemcpy(all.data(), all_dev, sizeof(cudaIpcMemHandle_t) * world, cudaMemcpyDeviceToHost);
    cudaFree(dh);
    RING_CUDA(e1);
    RING_CUDA(e2);
    R->peer_send.assign(world, nullptr);
    for (int p = 0; p < world; ++p) {
      if (p == rank) {
        R->peer_send[p] = R->send;
        continue;
      }
      RING_CUDA(cudaIpcOpenMemHandle(&R->peer_send[p], all[p], cudaIpcMemLazyEnablePeerAccess));
    }
    // Everyone has mapped everyone before the first ring call.
    float* one = nullptr;
    RING_CUDA(cudaMalloc(&one, sizeof(float)));
    nr = n->AllReduce(one, one, 1, ncclFloat32, ncclSum, R->comm, R->copy_stream);
    cudaError_t e3 = cudaStreamSynchronize(R->copy_stream);
    cudaFree(one);
    if (nr != ncclSuccess) RING_TRY(VOMNI_ENCCL);
    RING_CUDA(e3);
  }
#undef RING_TRY
#undef RING_CUDA
  *out = R;
  return VOMNI_OK;
}

extern "C" int vomni_ring_destroy(vomni_ring* R) {
  if (!R) return VOMNI_EINVAL;
  cudaSetDevice(R->device);
  cudaDeviceSynchronize();
  ring_free(R);
  return VOMNI_OK;
}

extern "C" int vomni_ring_check(vomni_ring* R) {
  if (!R) return VOMNI_EINVAL;
  if (R->broken) return VOMNI_ESTATE;
  if (!R->comm) return VOMNI_OK;
  const NcclApi* n = nccl();
  if (!n) return VOMNI_ENCCL;
  ncclResult_t ar = ncclSuccess;
  if (n->CommGetAsyncError(R->comm, &ar) != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
    R->broken = true;
    return VOMNI_ENCCL;
  }
  return VOMNI_OK;
}

extern "C" int vomni_ring_attention_strided(vomni_ring* R, const void* q, const void* k, const void* v, void* out,
                                            float* lse, int b, int s_loc, int h, int d, long long q_stride,
                                            long long kv_stride, float softmax_scale, int flags,
                                            vomni_stream_t stream) {
  if (!R || !q || !k || !v || !out) return VOMNI_EINVAL;
  if (R->broken) return VOMNI_ESTATE;
  if (flags & ~(VOMNI_CM_OUT_DMAJOR | VOMNI_CM_LSE)) return VOMNI_EINVAL;
  if (b != R->b || h != R->h || d != R->d || s_loc <= 0 || s_loc > R->s_max) return VOMNI_EBADSHAPE;
  int dev = -1;
  VOMNI_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != R->device) return VOMNI_ESTATE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const NcclApi* n = nccl();
  if (!n) return VOMNI_ENCCL;
  const int N = R->world;
  const size_t blk = static_cast<size_t>(s_loc) * h * d * 2;  // one batch row-block of K or V
  const long long dense = static_cast<long long>(h) * d;
  if (q_stride == 0) q_stride = dense;
  if (kv_stride == 0) kv_stride = dense;
  if (q_stride < dense || kv_stride < dense) return VOMNI_EBADSHAPE;
  if ((q_stride | kv_stride) & 7) return VOMNI_EALIGN;
  int rc;

  if (N == 1) {
    rc = vomni_cm_prologue_strided(q, k, b, s_loc, h, d, q_stride, kv_stride, R->qn2, R->kmax2, stream);
    if (rc) return rc;
    return vomni_cm_attend_strided(q, k, v, b, s_loc, s_loc, 0, s_loc, h, d, q_stride, kv_stride, softmax_scale, R->qn2,
                                   R->kmax2, nullptr, nullptr, flags | VOMNI_CM_FINAL, out, lse, stream);
  }

  const int parity = static_cast<int>(R->calls & 1);
  ++R->calls;
  const unsigned epoch = static_cast<unsigned>(R->calls);
  const StreamWriteValue32Fn write_value = stream_write_value32();
  // Every copy-stream path below ends by joining all copy streams into the caller stream (also on an
  // error), so no later work on the caller stream can overlap this call's copies. A failure after
  // the first copy is queued leaves the ring unusable (peers' copies and ready words no longer match
  // this call), so it also marks the ring broken.
  const int ncs = static_cast<int>(R->copy_streams.size());
  auto join_copies = [&](int status) {
    for (int i = 0; i < ncs; ++i) {
      cudaError_t e = cudaEventRecord(R->ev_copies_done[i], R->copy_streams[i]);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(st, R->ev_copies_done[i], 0);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        cudaStreamSynchronize(R->copy_streams[i]);  // cannot join by event: wait for the queued copies here
        if (status == VOMNI_OK) status = VOMNI_ECUDA;
      }
    }
    return status;
  };
  auto copies_failed = [&](int status) {
    R->broken = true;
    return join_copies(status);
  };
  // 1. publish this rank's K/V block in its registered send buffer (b blocks of s_loc tokens; the
  //    buffer keeps an s_max stride per batch so peers address it with the creation-time geometry),
  //    on copy stream 0 while the caller stream computes the norms.
  uint8_t* my_send = static_cast<uint8_t*>(R->send) + static_cast<size_t>(parity) * 2 * R->block_bytes;
  const size_t bstride = static_cast<size_t>(R->s_max) * h * d * 2;
  const size_t src_bstride = static_cast<size_t>(s_loc) * kv_stride * 2;  // a strided view's batch stride
  const size_t row_bytes = static_cast<size_t>(dense) * 2;
  VOMNI_CUDA_TRY(cudaEventRecord(R->ev_inputs, st));
  if (const cudaError_t e = cudaStreamWaitEvent(R->copy_stream, R->ev_inputs, 0); e != cudaSuccess) {
    set_last_cuda_error(e);
    return VOMNI_ECUDA;
  }
  for (int bi = 0; bi < b; ++bi) {
    cudaError_t e = cudaMemcpy2DAsync(my_send + bi * bstride, row_bytes, static_cast<const uint8_t*>(k) + bi * src_bstride,
                                      static_cast<size_t>(kv_stride) * 2, row_bytes, s_loc, cudaMemcpyDeviceToDevice,
                                      R->copy_stream);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(my_send + R->block_bytes + bi * bstride, row_bytes,
                            static_cast<const uint8_t*>(v) + bi * src_bstride, static_cast<size_t>(kv_stride) * 2, row_bytes,
                            s_loc, cudaMemcpyDeviceToDevice, R->copy_stream);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return copies_failed(VOMNI_ECUDA);
    }
  }
  if (const cudaError_t e = cudaEventRecord(R->ev_sent, R->copy_stream); e != cudaSuccess) {
    set_last_cuda_error(e);
    return copies_failed(VOMNI_ECUDA);
  }
  // 2. local norms, 3. global key max (also the "peers' blocks are published" point: the all_reduce
  //    follows this rank's send-buffer copies on the caller stream)
  rc = vomni_cm_prologue_strided(q, k, b, s_loc, h, d, q_stride, kv_stride, R->qn2, R->kmax2, stream);
  if (rc) return copies_failed(rc);
  if (const cudaError_t e = cudaStreamWaitEvent(st, R->ev_sent, 0); e != cudaSuccess) {
    set_last_cuda_error(e);
    return copies_failed(VOMNI_ECUDA);
  }
  if (n->AllReduce(R->kmax2, R->kmax2, static_cast<size_t>(b) * h, ncclFloat32, ncclMax, R->comm, st) != ncclSuccess)
    return copies_failed(VOMNI_ENCCL);
  if (const cudaError_t e = cudaEventRecord(R->ev_ready, st); e != cudaSuccess) {
    set_last_cuda_error(e);
    return copies_failed(VOMNI_ECUDA);
  }
  // 4. direct pulls, ring step s on copy stream (s - 1) % ncs, each step posting its ready word.
  for (int i = 0; i < ncs; ++i) {
    if (const cudaError_t e = cudaStreamWaitEvent(R->copy_streams[i], R->ev_ready, 0); e != cudaSuccess) {
      set_last_cuda_error(e);
      return copies_failed(VOMNI_ECUDA);
    }
  }
  const size_t gstride = static_cast<size_t>(N - 1) * s_loc * h * d * 2;  // per batch in the gather buffer
  for (int s = 1; s < N; ++s) {
    cudaStream_t cs = R->copy_streams[(s - 1) % ncs];
    const int src = vomni_ring_source_rank(R->rank, N, s);
    const uint8_t* ps = static_cast<const uint8_t*>(R->peer_send[src]) + static_cast<size_t>(parity) * 2 * R->block_bytes;
    for (int bi = 0; bi < b; ++bi) {
      uint8_t* gk = static_cast<uint8_t*>(R->gather_k) + bi * gstride + static_cast<size_t>(s - 1) * blk;
      uint8_t* gv = static_cast<uint8_t*>(R->gather_v) + bi * gstride + static_cast<size_t>(s - 1) * blk;
      cudaError_t e = cudaMemcpyAsync(gk, ps + bi * bstride, blk, cudaMemcpyDeviceToDevice, cs);
      if (e == cudaSuccess) e = cudaMemcpyAsync(gv, ps + R->block_bytes + bi * bstride, blk, cudaMemcpyDeviceToDevice, cs);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return copies_failed(VOMNI_ECUDA);
      }
    }
    if (const cudaError_t e = cudaEventRecord(R->ev_block[s], cs); e != cudaSuccess) {
      set_last_cuda_error(e);
      return copies_failed(VOMNI_ECUDA);
    }
    if (write_value && write_value(reinterpret_cast<CUstream>(cs), reinterpret_cast<CUdeviceptr>(R->ready + s), epoch, 0) !=
                           CUDA_SUCCESS)
      return copies_failed(VOMNI_ECUDA);
  }
  // 5. passes: local block, then ranges of arrived blocks; fp32 partial, normalise on the last.
  int first[64], count[64];
  const int np = vomni_ring_phase_plan(N, first, count, 64);
  if (np < 2) return join_copies(VOMNI_EINVAL);
  rc = vomni_cm_attend_strided(q, k, v, b, s_loc, s_loc, 0, s_loc, h, d, q_stride, kv_stride, softmax_scale, R->qn2,
                               R->kmax2, R->acc_o, R->acc_l, 0, nullptr, nullptr, stream);
  if (rc) return join_copies(rc);
  const int s_kv = (N - 1) * s_loc;
  for (int p = 1; p < np; ++p) {
    // this pass reads gather blocks first[p] .. first[p] + count[p] - 1 = ring steps first[p] + 1 .. + count[p]
    const int step0 = first[p] + 1;
    int fl = VOMNI_CM_ACC_IN | (p == np - 1 ? (VOMNI_CM_FINAL | flags) : 0);
    if (write_value) {
      // In-kernel gate on the blocks' ready words; the pass overlaps the previous pass's last wave
      // and only its epilogue (the accumulator read-modify-write) waits for that pass.
      fl |= VOMNI_CM_OVERLAP;
    } else {
      for (int s = step0; s < step0 + count[p]; ++s) {
        if (const cudaError_t e = cudaStreamWaitEvent(st, R->ev_block[s], 0); e != cudaSuccess) {
          set_last_cuda_error(e);
          return join_copies(VOMNI_ECUDA);
        }
      }
    }
    rc = cm_attend_gated(q, R->gather_k, R->gather_v, b, s_loc, s_kv, first[p] * s_loc, count[p] * s_loc, h, d,
                         q_stride, 0, softmax_scale, R->qn2, R->kmax2, R->acc_o, R->acc_l, fl, out, lse,
                         write_value ? R->ready + step0 : nullptr, count[p], epoch, stream);
    if (rc) return join_copies(rc);
  }
  // Join the copy streams: this rank's copies of its peers' send buffers are complete before any later
  // work on the caller stream (the next call's all_reduce included).
  return join_copies(VOMNI_OK);
}

extern "C" int vomni_ring_attention(vomni_ring* R, const void* q, const void* k, const void* v, void* out, float* lse,
                                    int b, int s_loc, int h, int d, float softmax_scale, int flags,
                                    vomni_stream_t stream) {
  return vomni_ring_attention_strided(R, q, k, v, out, lse, b, s_loc, h, d, 0, 0, softmax_scale, flags, stream);
}
