// The device runtime shim of include/device_cuda.h: device memory, pinned host memory, streams, CUDA graphs, events
// and the NCCL communicator, as plain C functions, so that the C11 engine (engine.c) never includes a CUDA header.
// NCCL is opened with dlopen on first use (libnccl.so.2): the library itself keeps no link-time dependency on it and
// loads on machines without NCCL, where only its symbols are inspected.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/device_cuda.h"
#include "kernels_cuda_internal.h"

namespace {

bool cuda_ok(cudaError_t e, const char *what) {
  if (e == cudaSuccess)
    return true;
  cudaGetLastError();
  return kc_fail("%s: %s", what, cudaGetErrorString(e));
}

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId *);
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  const char *(*error_string)(ncclResult_t);
  bool loaded;
};

const Nccl *nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h)
      h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h)
      return;
    n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
    n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(h, "ncclCommInitRank");
    n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
    n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
    n.comm_destroy = (decltype(n.comm_destroy))dlsym(h, "ncclCommDestroy");
    n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
    n.loaded = n.get_unique_id && n.comm_init_rank && n.all_reduce && n.all_gather && n.comm_destroy && n.error_string;
  });
  if (!n.loaded) {
    kc_fail("NCCL (libnccl.so.2) is not available");
    return nullptr;
  }
  return &n;
}

bool nccl_ok(const Nccl *n, ncclResult_t r, const char *what) {
  if (r == ncclSuccess)
    return true;
  return kc_fail("%s: %s", what, n->error_string(r));
}

}  // namespace

extern "C" {

int kd_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int kd_set_device(int device) { return cuda_ok(cudaSetDevice(device), "kd_set_device") ? 0 : -1; }

int kd_get_device(void) {
  int d = -1;
  return cudaGetDevice(&d) == cudaSuccess ? d : -1;
}

void *kd_malloc(size_t bytes) {
  void *p = nullptr;
  if (!bytes)
    return nullptr;
  if (!cuda_ok(cudaMalloc(&p, bytes), "kd_malloc"))
    return nullptr;
  return p;
}

void kd_free(void *p) {
  if (p)
    cudaFree(p);
}

void *kd_host_alloc(size_t bytes) {
  void *p = nullptr;
  if (!bytes)
    return nullptr;
  if (!cuda_ok(cudaMallocHost(&p, bytes), "kd_host_alloc"))
    return nullptr;
  return p;
}

void kd_host_free(void *p) {
  if (p)
    cudaFreeHost(p);
}

int kd_memset(void *dst, int value, size_t bytes) {
  return cuda_ok(cudaMemsetAsync(dst, value, bytes, kc_stream()), "kd_memset") ? 0 : -1;
}

int kd_copy(void *dst, const void *src, size_t bytes) {
  if (!bytes)
    return 0;
  return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, kc_stream()), "kd_copy") ? 0 : -1;
}

int kd_copy_2d(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t width, size_t height) {
  if (!width || !height)
    return 0;
  return cuda_ok(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, height, cudaMemcpyDefault, kc_stream()),
                 "kd_copy_2d")
             ? 0
             : -1;
}

void *kd_stream_create(void) {
  cudaStream_t s = nullptr;
  if (!cuda_ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "kd_stream_create"))
    return nullptr;
  return s;
}

void kd_stream_free(void *stream) {
  if (stream)
    cudaStreamDestroy(static_cast<cudaStream_t>(stream));
}

int kd_sync(void) { return cuda_ok(cudaStreamSynchronize(kc_stream()), "kd_sync") ? 0 : -1; }

int kd_capture_begin(void) {
  return cuda_ok(cudaStreamBeginCapture(kc_stream(), cudaStreamCaptureModeThreadLocal), "kd_capture_begin") ? 0 : -1;
}

void *kd_capture_end(void) {
  cudaGraph_t g = nullptr;
  if (!cuda_ok(cudaStreamEndCapture(kc_stream(), &g), "kd_capture_end"))
    return nullptr;
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (!cuda_ok(e, "kd_capture_end: instantiate"))
    return nullptr;
  return exec;
}

int kd_graph_launch(void *graph) {
  return cuda_ok(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), kc_stream()), "kd_graph_launch") ? 0 : -1;
}

void kd_graph_free(void *graph) {
  if (graph)
    cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph));
}

void *kd_event_create(void) {
  cudaEvent_t e = nullptr;
  if (!cuda_ok(cudaEventCreate(&e), "kd_event_create"))
    return nullptr;
  return e;
}

int kd_event_record(void *event) {
  return cuda_ok(cudaEventRecord(static_cast<cudaEvent_t>(event), kc_stream()), "kd_event_record") ? 0 : -1;
}

float kd_event_ms(void *start, void *end) {
  float ms = -1.0f;
  if (cudaEventSynchronize(static_cast<cudaEvent_t>(end)) != cudaSuccess ||
      cudaEventElapsedTime(&ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)) != cudaSuccess) {
    cudaGetLastError();
    return -1.0f;
  }
  return ms;
}

void kd_event_free(void *event) {
  if (event)
    cudaEventDestroy(static_cast<cudaEvent_t>(event));
}

// ---- NCCL ---------------------------------------------------------------------------------------------------------

int kd_comm_unique_id(unsigned char id[KD_COMM_ID_BYTES]) {
  static_assert(sizeof(ncclUniqueId) == KD_COMM_ID_BYTES, "ncclUniqueId size");
  const Nccl *n = nccl();
  if (!n)
    return -1;
  ncclUniqueId u;
  if (!nccl_ok(n, n->get_unique_id(&u), "ncclGetUniqueId"))
    return -1;
  memcpy(id, &u, sizeof(u));
  return 0;
}

void *kd_comm_init(int rank, int world, const unsigned char id[KD_COMM_ID_BYTES]) {
  const Nccl *n = nccl();
  if (!n)
    return nullptr;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  if (!nccl_ok(n, n->comm_init_rank(&c, world, u, rank), "ncclCommInitRank"))
    return nullptr;
  return c;
}

int kd_allreduce_sum_f32(void *comm, float *buf, size_t count) {
  const Nccl *n = nccl();
  if (!n)
    return -1;
  return nccl_ok(n, n->all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), kc_stream()),
                 "ncclAllReduce(sum)")
             ? 0
             : -1;
}

int kd_allreduce_max_u64(void *comm, unsigned long long *buf, size_t count) {
  const Nccl *n = nccl();
  if (!n)
    return -1;
  return nccl_ok(n, n->all_reduce(buf, buf, count, ncclUint64, ncclMax, static_cast<ncclComm_t>(comm), kc_stream()),
                 "ncclAllReduce(max)")
             ? 0
             : -1;
}

int kd_allgather_f32(void *comm, const float *send, float *recv, size_t count) {
  const Nccl *n = nccl();
  if (!n)
    return -1;
  return nccl_ok(n, n->all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), kc_stream()),
                 "ncclAllGather")
             ? 0
             : -1;
}

void kd_comm_free(void *comm) {
  const Nccl *n = comm ? nccl() : nullptr;
  if (n)
    n->comm_destroy(static_cast<ncclComm_t>(comm));
}

}  // extern "C"
