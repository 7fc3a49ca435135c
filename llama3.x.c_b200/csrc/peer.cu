// Peer-memory all-reduce of the decode step's residual partials (include/device_cuda.h: kd_peer_*): the tensor-parallel
// reduction after the column-sharded Wo and W2 products, for one row of `dim` floats. The reference reduces across its
// two NUMA sockets through host memory inside its worker team (src/tp.c: the partial sums of each shard are added by
// the team); here every rank is a GPU of one node and the vector is small (16 KiB for dim 4096), so latency decides,
// not bandwidth: one kernel per reduction, no library collective.
//
// Layout: each rank owns one device allocation, exported with CUDA IPC and mapped by every other rank:
//   recv [2 parities][world sources][stride] 8-byte slots {float bits, call number}   (kd_peer_allreduce_add)
//   gemv [2 parities][world sources][stride] the same, for the reducing GEMV           (kd_peer_matmul_q8_add)
// and private epochs (calls completed per CTA; the same on every rank, as every rank makes the same calls), one
// array per user, so that the two kinds of call can interleave in any order.
// Call number seq = epoch[c] + 1 selects the parity, so a rank can be one call ahead of a peer without overwriting what
// the peer still reads (a rank reaches call seq + 2 only after every peer has pushed call seq + 1, which each does
// only after finishing call seq).
//
// Each value travels with its call number in one 8-byte store, so a slot is complete the moment its number is right:
// no fence and no separate flag between the data and the reader. Thread i of the grid pushes element i of the local
// partial to slot [parity][rank][i] of every rank, then waits (bounded: KC_ERR_TIMEOUT and no sum after KC_WAIT_NS)
// until slot [parity][r][i] of its own memory carries seq for every rank r, and adds the values in rank order to x:
// x[i] + (((p_0 + p_1) + p_2) + ...). Every rank computes the same sum in the same order, so the replicated residual
// stays identical across ranks. Nothing here waits on another CTA of the same GPU.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include "../../include/device_cuda.h"
#include "common.cuh"
#include "kernels_cuda_internal.h"

namespace {

constexpr int kPeerMax = 8;
constexpr int kPeerThreads = 256;
constexpr int kPeerMaxCtas = 128;

struct PeerArgs {
  unsigned long long *recv[kPeerMax];  // every rank's slots, as mapped in this process
  unsigned *epoch;                     // this rank's completed calls per CTA
  long long stride;                    // slots per (parity, source)
  int rank, world, ctas;
};

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_add_kernel(const PeerArgs a, float *x,
                                                                          const float *partial, int n) {
  pdl_wait();  // the partial comes from the previous kernel
  pdl_launch_dependents();
  const int c = blockIdx.x, tid = threadIdx.x;
  const unsigned seq = a.epoch[c] + 1u;
  const long long par = seq & 1u;
  const int per = (n + a.ctas - 1) / a.ctas, lo = c * per, hi = min(n, lo + per);
  for (int i = lo + tid; i < hi; i += kPeerThreads) {
    const unsigned long long v = ((unsigned long long)seq << 32) | __float_as_uint(partial[i]);
#pragma unroll
    for (int p = 0; p < kPeerMax; p++)  // static indices: the pointers stay in parameter space
      if (p < a.world)
        peer_st_slot(a.recv[p] + (par * a.world + a.rank) * a.stride + i, v);
  }
  const unsigned long long *mine = a.recv[0];
#pragma unroll
  for (int p = 1; p < kPeerMax; p++)
    mine = p == a.rank ? a.recv[p] : mine;
  mine += par * a.world * a.stride;
  const uint64_t start = kc_globaltimer();
  bool ok = true;
  for (int i = lo + tid; i < hi; i += kPeerThreads) {
    float s = 0.0f;
    for (int r = 0; r < a.world && ok; r++) {
      unsigned long long v = peer_ld_slot(mine + r * a.stride + i);
      for (unsigned k = 1; (unsigned)(v >> 32) != seq; k++) {
        if ((k & 63u) == 0 && kc_globaltimer() - start > KC_WAIT_NS) {
          kc_raise(KC_ERR_TIMEOUT);
          ok = false;
          break;
        }
        v = peer_ld_slot(mine + r * a.stride + i);
      }
      const float f = __uint_as_float((unsigned)v);
      s = r == 0 ? f : __fadd_rn(s, f);
    }
    if (ok)
      x[i] = __fadd_rn(x[i], s);
  }
  __syncthreads();
  if (tid == 0)
    a.epoch[c] = seq;
}

struct PeerState {
  PeerArgs args;
  KcPeerGemv gemv;           // the reducing GEMV's slots (second half of every rank's allocation) and epochs
  void *base;                // this rank's exported allocation (the slots)
  void *opened[kPeerMax];    // the peers' allocations mapped here
  size_t max_floats;
};

// Set-up failures of the optional peer path (an IPC mapping the node does not allow, say) are reported on stderr
// and leave the caller on NCCL; they do not go through the library's fail() policy.
bool cuda_ok(cudaError_t e, const char *what) {
  if (e == cudaSuccess)
    return true;
  cudaGetLastError();
  fprintf(stderr, "%s: %s (the peer-memory all-reduce is off; NCCL reduces instead)\n", what, cudaGetErrorString(e));
  return false;
}

// A state for `rank` of `world` with this rank's slots (both regions) and call counters allocated and zeroed. *ok is
// false after a CUDA failure (reported on stderr); the state is returned either way, for the caller to free.
PeerState *local_state(int rank, int world, size_t max_floats, size_t *recv_bytes, bool *ok) {
  PeerState *s = new PeerState();
  memset(s, 0, sizeof(*s));
  s->max_floats = max_floats;
  int ctas = (int)((max_floats + kPeerThreads - 1) / kPeerThreads);  // a slot per thread
  ctas = ctas < 1 ? 1 : ctas > kPeerMaxCtas ? kPeerMaxCtas : ctas;
  const long long stride = (long long)((max_floats + 31) / 32 * 32);
  *recv_bytes = (size_t)2 * world * stride * sizeof(unsigned long long);
  s->args.stride = stride;
  s->args.rank = rank;
  s->args.world = world;
  s->args.ctas = ctas;
  s->gemv.stride = stride;
  s->gemv.rank = rank;
  s->gemv.world = world;
  const size_t bytes = 2 * *recv_bytes;
  *ok = cuda_ok(cudaMalloc(&s->base, bytes), "kd_peer_init: cudaMalloc") &&
        cuda_ok(cudaMalloc(&s->args.epoch, kPeerMaxCtas * sizeof(unsigned)), "kd_peer_init: cudaMalloc") &&
        cuda_ok(cudaMalloc(&s->gemv.epoch, kPeerGemvMaxCtas * sizeof(unsigned)), "kd_peer_init: cudaMalloc") &&
        cuda_ok(cudaMemset(s->base, 0, bytes), "kd_peer_init: cudaMemset") &&
        cuda_ok(cudaMemset(s->args.epoch, 0, kPeerMaxCtas * sizeof(unsigned)), "kd_peer_init: cudaMemset") &&
        cuda_ok(cudaMemset(s->gemv.epoch, 0, kPeerGemvMaxCtas * sizeof(unsigned)), "kd_peer_init: cudaMemset") &&
        // Zeroed before any peer can learn the handle: a peer's first store lands after this.
        cuda_ok(cudaDeviceSynchronize(), "kd_peer_init: synchronize");
  return s;
}

// Every rank's slots are this process's own buffer: the single-rank state, and the test hook's absent peers.
void map_local(PeerState *s, size_t recv_bytes) {
  for (int p = 0; p < s->args.world; p++) {
    s->args.recv[p] = reinterpret_cast<unsigned long long *>(s->base);
    s->gemv.slots[p] = reinterpret_cast<unsigned long long *>(static_cast<char *>(s->base) + recv_bytes);
  }
}

}  // namespace

extern "C" {

void kd_peer_free(void *peer) {
  PeerState *s = static_cast<PeerState *>(peer);
  if (!s)
    return;
  for (int p = 0; p < kPeerMax; p++)
    if (s->opened[p])
      cudaIpcCloseMemHandle(s->opened[p]);
  if (s->base)
    cudaFree(s->base);
  if (s->args.epoch)
    cudaFree(s->args.epoch);
  if (s->gemv.epoch)
    cudaFree(s->gemv.epoch);
  delete s;
}

void *kd_peer_init(void *comm, int rank, int world, size_t max_floats) {
  if ((!comm && world > 1) || world < 1 || world > kPeerMax || rank < 0 || rank >= world || max_floats == 0 ||
      max_floats > (1u << 26)) {
    kc_fail("kd_peer_init: invalid arguments (rank %d of %d, %zu floats)", rank, world, max_floats);
    return nullptr;
  }
  size_t recv_bytes = 0;
  bool ok = false;
  PeerState *s = local_state(rank, world, max_floats, &recv_bytes, &ok);
  if (world == 1) {  // one rank: its own slots only, nothing to exchange
    if (!ok) {
      kd_peer_free(s);
      return nullptr;
    }
    map_local(s, recv_bytes);
    return s;
  }
  cudaIpcMemHandle_t mine, all[kPeerMax];
  static_assert(sizeof(cudaIpcMemHandle_t) % sizeof(float) == 0, "IPC handle size");
  constexpr size_t hf = sizeof(cudaIpcMemHandle_t) / sizeof(float);
  memset(&mine, 0, sizeof(mine));
  float *xchg = nullptr;
  if (!cuda_ok(cudaMalloc(&xchg, (world + 1) * sizeof(cudaIpcMemHandle_t)), "kd_peer_init: cudaMalloc")) {
    kd_peer_free(s);
    return nullptr;
  }
  // A local set-up failure still takes part in the exchange below (with an all-zero handle), so that no rank is left
  // waiting in the collective. The engine then agrees on NCCL with the others.
  ok = ok && cuda_ok(cudaIpcGetMemHandle(&mine, s->base), "kd_peer_init: cudaIpcGetMemHandle");
  if (!ok)
    memset(&mine, 0, sizeof(mine));
  // Every rank's handle to every rank, through the NCCL communicator (on the calling thread's stream).
  const bool exchanged =
      cuda_ok(cudaMemcpy(xchg + world * hf, &mine, sizeof(mine), cudaMemcpyHostToDevice), "kd_peer_init: copy") &&
      kd_allgather_f32(comm, xchg + world * hf, xchg, hf) == 0 &&  // NCCL failures do go through fail()
      cuda_ok(cudaStreamSynchronize(kc_stream()), "kd_peer_init: synchronize") &&
      cuda_ok(cudaMemcpy(all, xchg, world * sizeof(cudaIpcMemHandle_t), cudaMemcpyDeviceToHost), "kd_peer_init: copy");
  cudaFree(xchg);
  ok = ok && exchanged;
  static const cudaIpcMemHandle_t none = {};
  for (int p = 0; ok && p < world; p++) {
    char *b = nullptr;
    if (p == rank) {
      b = static_cast<char *>(s->base);
    } else if (!memcmp(&all[p], &none, sizeof(none))) {
      ok = false;  // that rank's set-up failed
    } else {
      void *m = nullptr;
      ok = cuda_ok(cudaIpcOpenMemHandle(&m, all[p], cudaIpcMemLazyEnablePeerAccess), "kd_peer_init: cudaIpcOpenMemHandle");
      s->opened[p] = m;
      b = static_cast<char *>(m);
    }
    s->args.recv[p] = reinterpret_cast<unsigned long long *>(b);
    s->gemv.slots[p] = reinterpret_cast<unsigned long long *>(b ? b + recv_bytes : nullptr);
  }
  if (!ok) {
    kd_peer_free(s);
    return nullptr;
  }
  return s;
}

void *kd_peer_test_absent(int world, size_t max_floats) {
  if (world < 2 || world > kPeerMax || max_floats == 0 || max_floats > (1u << 26)) {
    kc_fail("kd_peer_test_absent: invalid arguments (%d ranks, %zu floats)", world, max_floats);
    return nullptr;
  }
  size_t recv_bytes = 0;
  bool ok = false;
  PeerState *s = local_state(0, world, max_floats, &recv_bytes, &ok);
  if (!ok) {
    kd_peer_free(s);
    return nullptr;
  }
  map_local(s, recv_bytes);
  return s;
}

int kd_peer_allreduce_add(void *peer, float *x, const float *partial, size_t n) {
  const PeerState *s = static_cast<const PeerState *>(peer);
  if (!s || !x || !partial || n == 0 || n > s->max_floats) {
    kc_fail("kd_peer_allreduce_add: invalid arguments (%zu floats)", n);
    return -1;
  }
  const cudaError_t e = kc_launch_pdl(peer_allreduce_add_kernel, dim3(s->args.ctas), kPeerThreads, 0, kc_stream(),
                                      s->args, x, partial, (int)n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    kc_fail("kd_peer_allreduce_add: %s", cudaGetErrorString(e));
    return -1;
  }
  kc_count_launch();
  return 0;
}

int kd_peer_matmul_q8_add(void *peer, float *x, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                          size_t ld, int n, int d, int gs) {
  const PeerState *s = static_cast<const PeerState *>(peer);
  if (!s || !x || !xq || !xs || !wq || !ws || n <= 0 || d <= 0 || (size_t)d > s->max_floats || gs <= 0 ||
      n % gs || ld < (size_t)n || ld % gs || ld > (size_t)INT32_MAX) {
    kc_fail("kd_peer_matmul_q8_add: invalid arguments (ld %zu, n %d, d %d, gs %d)", ld, n, d, gs);
    return -1;
  }
  KcGemvSeg seg = {};
  seg.out = x;
  seg.wq = wq;
  seg.ws = ws;
  seg.d = d;
  const int rc = kc_launch_gemv_reduce(seg, xq, xs, n, (long long)ld, gs, s->gemv, kc_stream());
  if (rc == -1) {
    kc_fail("kd_peer_matmul_q8_add: shape not supported by the reducing GEMV (n %d, gs %d, 16-byte aligned "
            "activations and scale rows needed)", n, gs);
    return -1;
  }
  if (rc != 0) {
    const cudaError_t e = cudaGetLastError();
    kc_fail("kd_peer_matmul_q8_add: %s", cudaGetErrorString(e));
    return -1;
  }
  kc_count_launch();
  return 0;
}

}  // extern "C"
