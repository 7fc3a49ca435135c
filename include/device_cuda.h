/* Device runtime shim of libllama3x_cuda.so: the CUDA runtime and NCCL calls the C11 engine needs, as plain C
 * functions (no CUDA header in the engine). None of these has a counterpart in the reference, whose engine runs on
 * host memory and worker teams; they replace memory_alloc/memory_free for device buffers (include/runtime.h:48-50),
 * the team exchange (src/workers.c:332-539) for the tensor-parallel reduction, and nothing else.
 *
 * Stream: every call that enqueues work (kd_memset, kd_copy*, kd_capture_*, kd_graph_launch, kd_event_record and the
 * collectives) uses the calling thread's stream, the one kernels_set_stream selected (NULL = the legacy stream).
 * Errors: a failing call returns -1 or NULL and goes through the library's fail() policy (kc_set_fail_mode). */
#ifndef LLAMA3X_DEVICE_CUDA_H
#define LLAMA3X_DEVICE_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

int kd_device_count(void);
int kd_set_device(int device);
int kd_get_device(void);

void *kd_malloc(size_t bytes);
void kd_free(void *p);
void *kd_host_alloc(size_t bytes); /* page-locked host memory */
void kd_host_free(void *p);
int kd_memset(void *dst, int value, size_t bytes);
/* Any direction (unified addressing); asynchronous on the stream for pinned or device memory. */
int kd_copy(void *dst, const void *src, size_t bytes);
int kd_copy_2d(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t width, size_t height);

void *kd_stream_create(void);
void kd_stream_free(void *stream);
int kd_sync(void); /* waits for the calling thread's stream */

/* Stream capture of the calling thread's stream into an instantiated graph. */
int kd_capture_begin(void);
void *kd_capture_end(void);
int kd_graph_launch(void *graph);
void kd_graph_free(void *graph);

void *kd_event_create(void);
int kd_event_record(void *event);
float kd_event_ms(void *start, void *end); /* waits for `end`; -1 on error */
void kd_event_free(void *event);

/* NCCL, one communicator per rank (one process per GPU). */
#define KD_COMM_ID_BYTES 128
int kd_comm_unique_id(unsigned char id[KD_COMM_ID_BYTES]);
void *kd_comm_init(int rank, int world, const unsigned char id[KD_COMM_ID_BYTES]);
int kd_allreduce_sum_f32(void *comm, float *buf, size_t count);
int kd_allreduce_max_u64(void *comm, unsigned long long *buf, size_t count);
int kd_allgather_f32(void *comm, const float *send, float *recv, size_t count); /* recv: count floats per rank */
void kd_comm_free(void *comm);

/* Peer-memory all-reduce for one short vector (the decode step's residual partials), one kernel per call: every rank
 * pushes its partial over NVLink into every rank's receive buffer (CUDA IPC mappings, so all ranks are processes on
 * one node with peer access between every pair of GPUs, as NVSwitch gives) and waits, bounded, for the others'; then
 * x[i] += sum of the partials in rank order, identical on every rank. kd_peer_init is collective over `comm` (it
 * exchanges the IPC handles once); every rank must then make the same kd_peer_allreduce_add calls in the same order.
 * n <= max_floats. A peer that does not arrive within the wait limit raises the kernel error flag (kc_status). */
void *kd_peer_init(void *comm, int rank, int world, size_t max_floats);
int kd_peer_allreduce_add(void *peer, float *x, const float *partial, size_t n);
void kd_peer_free(void *peer);

#ifdef __cplusplus
}
#endif

#endif
