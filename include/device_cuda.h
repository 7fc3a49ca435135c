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
#include <stdint.h>

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
 * n <= max_floats. A peer that does not arrive within the wait limit raises the kernel error flag (kc_status).
 * world 1 (comm may be NULL) is a single rank: no IPC, x += partial, and kd_peer_matmul_q8_add equals
 * k_matmul_q8_add bitwise. */
void *kd_peer_init(void *comm, int rank, int world, size_t max_floats);
int kd_peer_allreduce_add(void *peer, float *x, const float *partial, size_t n);
void kd_peer_free(void *peer);
/* The column-sharded Wo / W2 product and its all-reduce in one kernel, as the reference fuses them into one team job
 * (project_residual / project_reduce_fn, src/tp.c:232-244 and 316-335: a K_PARTIAL share whose rows are flagged to the
 * exchange as they finish, exchange_rows_done / exchange_reduce_add_flags in src/workers.c:476-521, then added into
 * the residual): x[r] += sum over ranks, in rank order, of row r of this rank's slice (wq [d][ld] int8, ws [d][ld / gs]) times its activations (xq [n], xs [n / gs]),
 * each rank's product in the reference's AVX-512 GEMV order. Bitwise equal to k_matmul_q8_ld(..., K_PARTIAL)
 * followed by kd_peer_allreduce_add. d <= max_floats of kd_peer_init; gs 64, 128, ... 1024 dividing n and ld, with
 * (ld / gs) a multiple of 4 and 16-byte aligned activations and scale rows, else rejected (-1). Every rank makes the
 * same calls in the same order, on the same number of SMs. */
int kd_peer_matmul_q8_add(void *peer, float *x, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                          size_t ld, int n, int d, int gs);
/* Test hook, the GPU form of the reference's exchange-fail tests (tests/workers.c:10-11, 603-610): a peer state for
 * rank 0 of `world` whose other ranks never arrive (every rank's slots are this process's own memory and only rank 0
 * writes them). Each kd_peer_allreduce_add / kd_peer_matmul_q8_add call on it gives up after the device wait limit
 * (2 s), raises KC_ERR_TIMEOUT (kc_status) and leaves x unchanged; the context stays usable. Free with kd_peer_free. */
void *kd_peer_test_absent(int world, size_t max_floats);

#ifdef __cplusplus
}
#endif

#endif
