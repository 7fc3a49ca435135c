// The C-ABI of libllama3x_cuda.so (include/kernels_cuda.h): argument checks with the reference's messages, the
// fail()-style error policy, the per-thread stream, and dispatch to the kernels.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <set>
#include <utility>

#include "../../include/kernels_cuda.h"
#include "common.cuh"
#include "kernels_cuda_internal.h"

__device__ unsigned kc_error_word;

namespace {

thread_local cudaStream_t tl_stream = nullptr;
thread_local char tl_error[512];
int fail_mode = KC_FAIL_EXIT;
bool initialized = false;
bool pdl_on = true;

}  // namespace

bool kc_fail(const char *format, ...) {
  va_list args;
  va_start(args, format);
  vsnprintf(tl_error, sizeof(tl_error), format, args);
  va_end(args);
  if (fail_mode == KC_FAIL_EXIT) {
    fprintf(stderr, "error: %s\n", tl_error);
    exit(EXIT_FAILURE);
  }
  return false;
}

static std::atomic<unsigned long long> launch_counter{0};

void kc_count_launch() { launch_counter.fetch_add(1, std::memory_order_relaxed); }

static bool launched(int rc, const char *what) {
  if (rc == 0) {
    kc_count_launch();
    return true;
  }
  if (rc == -1)
    return kc_fail("%s: shape not supported by the sm_100a kernels", what);
  return kc_fail("%s: CUDA launch failed: %s", what, cudaGetErrorString(cudaGetLastError()));
}

int kc_device_sms() {
  static std::atomic<int> sms[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64)
    return 148;
  int v = sms[dev].load(std::memory_order_relaxed);
  if (!v) {  // a race only repeats the same query
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    v = v > 0 ? v : 148;
    sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

bool kc_pdl_enabled() { return pdl_on; }

cudaError_t kc_allow_smem(const void *kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void *, int>> done;  // (kernel, device) pairs already raised to their limit
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev}))
    return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    done.insert({kernel, dev});
  return e;
}

cudaStream_t kc_stream() { return tl_stream; }

extern "C" {

void kernels_init(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
    kc_fail("kernels_init: no usable CUDA device");
    return;
  }
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, dev);
  if (prop.major != 10) {
    kc_fail("kernels_init: device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, prop.major,
            prop.minor);
    return;
  }
  kc_device_sms();
  initialized = true;
}

const char *kernels_name(void) { return initialized ? "sm_100a" : NULL; }

void kernels_set_stream(void *stream) { tl_stream = static_cast<cudaStream_t>(stream); }

void kernels_set_pdl(int on) { pdl_on = on != 0; }

void kernels_backend_init(void) {}
void kernels_backend_free(void) {}

void kc_set_fail_mode(int mode) { fail_mode = mode == KC_FAIL_RETURN ? KC_FAIL_RETURN : KC_FAIL_EXIT; }

const char *kc_last_error(void) { return tl_error; }

void kc_clear_error(void) { tl_error[0] = 0; }

void kc_fail_message(const char *message) { kc_fail("%s", message); }

unsigned long long kc_launch_count(void) { return launch_counter.load(std::memory_order_relaxed); }

int kc_status(void) {
  cudaError_t e = cudaStreamSynchronize(tl_stream);
  if (e != cudaSuccess) {
    kc_fail("CUDA error: %s", cudaGetErrorString(e));
    return -1;
  }
  unsigned bits = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&bits, kc_error_word, sizeof(bits)) != cudaSuccess) {
    kc_fail("CUDA error reading the device error word");
    return -1;
  }
  if (bits) {
    cudaMemcpyToSymbol(kc_error_word, &zero, sizeof(zero));
    if (bits & KC_ERR_NONFINITE)
      kc_fail("nonfinite activation during INT8 quantization");
    else if (bits & KC_ERR_TIMEOUT)
      kc_fail("a device-side wait timed out");
    else
      kc_fail("a kernel rejected its arguments");
  }
  return (int)bits;
}

// ---- quantizer ----------------------------------------------------------------------------------------------------

void k_quantize_rows(int8_t *q, float *s, const float *x, size_t ldx, int m, int n, int gs) {
  if (gs <= 0 || m < 0 || n < 0 || ldx < (size_t)n) {
    kc_fail("k_quantize_rows: invalid shape m=%d n=%d ldx=%zu gs=%d", m, n, ldx, gs);
    return;
  }
  launched(kc_launch_quantize_rows(q, s, x, (long long)ldx, m, n, gs, tl_stream), "k_quantize_rows");
}

void k_quantize(int8_t *q, float *s, const float *x, int n, int gs) { k_quantize_rows(q, s, x, (size_t)n, 1, n, gs); }

// ---- decode GEMV --------------------------------------------------------------------------------------------------

// W8A8 input (q, s) or, with q NULL, W8A32 (f), as the reference's K8Input (include/kernels.h:101-109).
static bool gemv_input_ok(const char *name, const K8Input *x) {
  if (!x || (x->q ? !x->s : !x->f))
    return kc_fail("%s: the input needs int8 values and scales, or (W8A32) fp32 activations", name);
  return true;
}

static bool gemv_shape_ok(const char *name, const K8Input *x, size_t ld, int n, int gs) {
  if (!gemv_input_ok(name, x))
    return false;
  if (gs <= 0)
    return kc_fail("%s: invalid group size %d", name, gs);
  if (n < 0 || n % gs)
    return kc_fail("%s: %d inputs are not a whole number of %d-groups", name, n, gs);
  if (ld < (size_t)n || ld % (size_t)gs)
    return kc_fail("%s: row stride %zu must be at least %d and a multiple of the group size %d", name, ld, n, gs);
  return true;
}

static bool weight_ok(const char *name, K8Weight w) {
  if (!w.q || !w.s)
    return kc_fail("%s: missing weight values or scales", name);
  return true;
}

// Checks and launches one GEMV; false (the reason recorded) when it did neither.
static bool gemv(const char *name, const KcGemvSeg *segs, int nseg, const K8Input *x, size_t ld, int n, int gs,
                 int kind) {
  if (!gemv_shape_ok(name, x, ld, n, gs))
    return false;
  for (int i = 0; i < nseg; i++) {
    if (segs[i].d < 0)
      return kc_fail("%s: negative row count", name);
    if (segs[i].d > 0 && !segs[i].out)
      return kc_fail("%s: missing output", name);
    if (!weight_ok(name, K8Weight{segs[i].wq, segs[i].ws}) ||
        (kind == KC_SWIGLU && !weight_ok(name, K8Weight{segs[i].w3q, segs[i].w3s})))
      return false;
  }
  if (!x->q)  // W8A32
    return launched(kc_launch_gemv_w8a32(segs, nseg, x->f, n, (long long)ld, gs, kind, tl_stream), name);
  return launched(kc_launch_gemv(segs, nseg, x->q, x->s, n, (long long)ld, gs, kind, tl_stream, 0), name);
}

void k_matmul_q8(float *out, const K8Input *x, K8Weight w, int n, int d, int gs) {
  KcGemvSeg s = {out, w.q, w.s, nullptr, nullptr, d};
  gemv("k_matmul_q8", &s, 1, x, (size_t)n, n, gs, KC_STORE);
}

void k_matmul_q8_add(float *out, const K8Input *x, K8Weight w, int n, int d, int gs) {
  KcGemvSeg s = {out, w.q, w.s, nullptr, nullptr, d};
  gemv("k_matmul_q8_add", &s, 1, x, (size_t)n, n, gs, KC_ADD);
}

void k_matmul_q8_qkv(float *q, float *k, float *v, const K8Input *x, K8Weight wq, K8Weight wk, K8Weight wv, int n,
                     int dq, int dkv, int gs) {
  KcGemvSeg s[3] = {{q, wq.q, wq.s, nullptr, nullptr, dq},
                    {k, wk.q, wk.s, nullptr, nullptr, dkv},
                    {v, wv.q, wv.s, nullptr, nullptr, dkv}};
  gemv("k_matmul_q8_qkv", s, 3, x, (size_t)n, n, gs, KC_STORE);
}

void k_matmul_q8_swiglu(float *out, const K8Input *x, K8Weight w1, K8Weight w3, int n, int d, int gs) {
  KcGemvSeg s = {out, w1.q, w1.s, w3.q, w3.s, d};
  gemv("k_matmul_q8_swiglu", &s, 1, x, (size_t)n, n, gs, KC_SWIGLU);
}

void k_matmul_q8_ld(float *out, const K8Input *x, const K8Weight *w, size_t ld, int n, int d, int gs, int kind) {
  if (kind != K_STORE && kind != K_ADD && kind != K_PARTIAL) {
    kc_fail("k_matmul_q8_ld: invalid epilogue kind %d", kind);
    return;
  }
  KcGemvSeg s = {out, w->q, w->s, nullptr, nullptr, d};
  gemv("k_matmul_q8_ld", &s, 1, x, ld, n, gs, kind);
}

void k_matmul_q8_swiglu_ld(float *out, const K8Input *x, const K8Weight *w1, const K8Weight *w3, size_t ld, int n,
                           int d, int gs) {
  KcGemvSeg s = {out, w1->q, w1->s, w3->q, w3->s, d};
  gemv("k_matmul_q8_swiglu_ld", &s, 1, x, ld, n, gs, KC_SWIGLU);
}

void k_matmul_q8_ld_worker(float *out, const K8Input *x, const K8Weight *w, size_t ld, int n, int d, int gs, int kind,
                           int worker, int workers, kc_atomic_int *claim, RowsDoneFn done, void *done_ctx) {
  (void)claim;
  const char *name = "k_matmul_q8_ld_worker";
  if (kind != K_STORE && kind != K_ADD && kind != K_PARTIAL) {
    kc_fail("%s: invalid epilogue kind %d", name, kind);
    return;
  }
  if (workers < 1 || worker < 0 || worker >= workers || d < 0 || !w || gs <= 0) {
    kc_fail("%s: invalid member %d of %d", name, worker, workers);
    return;
  }
  const int r0 = (int)((long long)d * worker / workers), r1 = (int)((long long)d * (worker + 1) / workers);
  if (r1 <= r0)
    return;
  KcGemvSeg s = {out + r0, w->q + (size_t)r0 * ld, w->s + (size_t)r0 * (ld / (size_t)gs), nullptr, nullptr, r1 - r0};
  gemv(name, &s, 1, x, ld, n, gs, kind);
  if (done && !kc_last_error()[0]) {
    if (cudaStreamSynchronize(tl_stream) != cudaSuccess) {
      kc_fail("%s: %s", name, cudaGetErrorString(cudaGetLastError()));
      return;
    }
    done(done_ctx, r0, r1);
  }
}

// Segments of one kind as KcGemvSeg; false (and fail()) otherwise.
static bool gemv_segments(const char *name, const GemmQ8Segment *segments, int count, KcGemvSeg *segs, int *kind) {
  if (!segments || count < 1 || count > GEMM_MAX_SEGMENTS)
    return kc_fail("%s: needs 1..%d segments, got %d", name, GEMM_MAX_SEGMENTS, segments ? count : 0);
  *kind = -1;
  for (int i = 0; i < count; i++) {
    const GemmQ8Segment &g = segments[i];
    const int k = g.kind == GEMM_STORE ? KC_STORE : g.kind == GEMM_ADD ? KC_ADD : g.kind == GEMM_PARTIAL ? KC_PARTIAL
                  : g.kind == GEMM_SWIGLU ? KC_SWIGLU : -1;
    if (k < 0 || (*kind >= 0 && k != *kind) || (k == KC_SWIGLU && (count != 1 || !g.w3.q || !g.w3.s)) || g.n < 0 ||
        !weight_ok(name, g.w))
      return kc_fail("%s: segments need one kind (a SwiGLU pair alone), weights and non-negative rows", name);
    if (g.n > 0 && !g.c)
      return kc_fail("%s: segment %d is missing its output", name, i);
    *kind = k;
    segs[i] = KcGemvSeg{g.c, g.w.q, g.w.s, g.w3.q, g.w3.s, g.n};
  }
  return true;
}

// The C-ABI tail as the kernel's, checked against the segments; false (kc_fail) when it does not fit them.
static bool tail_from(const char *name, const KernelTail *tail, const GemmQ8Segment *segments, int count, int kind,
                      int gs, KcGemvTail *t) {
  *t = KcGemvTail{};
  if (!tail)
    return true;
  t->kind = tail->kind;
  if (tail->kind == K_TAIL_QUANTIZE || tail->kind == K_TAIL_NORM_QUANTIZE) {
    if (!tail->x || !tail->q || !tail->s || tail->n <= 0 || tail->n % gs ||
        (tail->kind == K_TAIL_NORM_QUANTIZE && !tail->weight))
      return kc_fail("%s: the quantize tail needs x, q, s, a whole number of %d-groups and (to normalize) weights",
                     name, gs);
    t->x = tail->x, t->w = tail->weight, t->eps = tail->epsilon, t->q = tail->q, t->s = tail->s, t->n = tail->n;
  } else if (tail->kind == K_TAIL_ROPE_KV_STORE) {
    if (count != 3 || kind != KC_STORE || !tail->rope_table || !tail->position || !tail->key_cache ||
        !tail->value_cache || tail->head_dim <= 0 || tail->head_dim % 2 || tail->n_kv_heads <= 0 ||
        segments[0].n != tail->n_heads * tail->head_dim || segments[1].n != tail->n_kv_heads * tail->head_dim ||
        segments[2].n != tail->n_kv_heads * tail->head_dim)
      return kc_fail("%s: the RoPE tail needs the q, k, v segments (STORE) of its heads, the table, position and caches",
                     name);
    t->qv = segments[0].c, t->kv = segments[1].c, t->vv = segments[2].c;
    t->kcache = tail->key_cache, t->vcache = tail->value_cache, t->table = tail->rope_table, t->pos = tail->position;
    t->nh = tail->n_heads, t->nkv = tail->n_kv_heads, t->hd = tail->head_dim, t->seq = tail->seq_len;
  } else if (tail->kind == K_TAIL_QUANTIZE_OUTPUT) {
    if (count != 1 || (kind != KC_STORE && kind != KC_SWIGLU) || !tail->q || !tail->s || segments[0].n % gs ||
        segments[0].n / gs > (1 << 16))
      return kc_fail("%s: the output quantizer needs one STORE or SWIGLU segment of whole %d-groups (at most 65536) "
                     "and q, s", name, gs);
    t->q = tail->q, t->s = tail->s, t->n = segments[0].n;
  } else if (tail->kind != K_TAIL_NONE) {
    return kc_fail("%s: invalid tail kind %d", name, (int)tail->kind);
  }
  return true;
}

void k_matmul_q8_fused(const float *x, const float *weight, float epsilon, size_t ld, int n, int gs,
                       const GemmQ8Segment *segments, int count, const KernelTail *tail) {
  const char *name = "k_matmul_q8_fused";
  if (!x) {
    kc_fail("%s: missing activations", name);
    return;
  }
  if (gs <= 0 || n <= 0 || n % gs || ld < (size_t)n || ld % (size_t)gs) {
    kc_fail("%s: invalid shape n=%d ld=%zu gs=%d", name, n, ld, gs);
    return;
  }
  KcGemvSeg segs[GEMM_MAX_SEGMENTS];
  int kind = -1;
  KcGemvTail t;
  if (!gemv_segments(name, segments, count, segs, &kind) || !tail_from(name, tail, segments, count, kind, gs, &t))
    return;
  launched(kc_launch_gemv_f32(segs, count, KcGemvAct{x, weight, epsilon}, n, (long long)ld, gs, kind, tl_stream,
                              t.kind ? &t : nullptr),
           name);
}

void k_matmul_q8_tail(const K8Input *x, size_t ld, int n, int gs, const GemmQ8Segment *segments, int count,
                      const KernelTail *tail) {
  const char *name = "k_matmul_q8_tail";
  KcGemvSeg segs[GEMM_MAX_SEGMENTS];
  int kind = -1;
  if (!gemv_shape_ok(name, x, ld, n, gs) || !gemv_segments(name, segments, count, segs, &kind))
    return;
  if (!x->q) {
    kc_fail("%s: a tail GEMV needs int8 activations (W8A8)", name);
    return;
  }
  if (!tail) {
    kc_fail("%s: missing tail", name);
    return;
  }
  KcGemvTail t;
  if (!tail_from(name, tail, segments, count, kind, gs, &t))
    return;
  if (t.kind == KC_TAIL_NONE) {
    launched(kc_launch_gemv(segs, count, x->q, x->s, n, (long long)ld, gs, kind, tl_stream, 0), name);
    return;
  }
  launched(kc_launch_gemv_tail(segs, count, x->q, x->s, n, (long long)ld, gs, kind, t, tl_stream), name);
}

// ---- batched prefill GEMM -----------------------------------------------------------------------------------------

static int kc_kind_of(GemmKind k) {
  switch (k) {
    case GEMM_STORE: return KC_STORE;
    case GEMM_ADD: return KC_ADD;
    case GEMM_SWIGLU: return KC_SWIGLU;
    case GEMM_PARTIAL: return KC_PARTIAL;
  }
  return -1;
}

static bool gemm_args_ok(const char *name, const int8_t *xq, const float *xs, int m, int k, int gs,
                         const GemmQ8Segment *segments, int count) {
  if (!segments || count < 1 || count > GEMM_MAX_SEGMENTS)
    return kc_fail("GEMM needs 1..%d segments, got %d", GEMM_MAX_SEGMENTS, segments ? count : 0);
  if (gs <= 0 || k % gs)
    return kc_fail("Q8 GEMM: K=%d is not a multiple of the group size %d", k, gs);
  for (int s = 0; s < count; s++) {
    if (kc_kind_of(segments[s].kind) < 0)
      return kc_fail("%s: invalid GEMM kind %d", name, (int)segments[s].kind);
    if (segments[s].kind == GEMM_SWIGLU && !segments[s].w3.q)
      return kc_fail("GEMM_SWIGLU needs a second weight matrix");
    if (segments[s].ldc < segments[s].n)
      return kc_fail("%s: ldc %d is shorter than the %d outputs", name, segments[s].ldc, segments[s].n);
  }
  if (m < 0 || k < 0)
    return kc_fail("%s: negative shape", name);
  // The kernels read every pointer they are given: a missing one is an error here, never an address on the GPU.
  if (m > 0 && k > 0) {
    if (!xq || !xs)
      return kc_fail("%s: missing activations", name);
    for (int s = 0; s < count; s++) {
      const GemmQ8Segment &g = segments[s];
      if (g.n > 0 && (!g.c || !g.w.q || !g.w.s || (g.kind == GEMM_SWIGLU && !g.w3.s)))
        return kc_fail("%s: segment %d is missing its output, weight values or scales", name, s);
    }
  }
  return true;
}

static bool gemm_rows_dp4a(const int8_t *xq, const float *xs, int m, int k, int gs, const GemmQ8Segment *segments,
                           int count) {
  // One row-kernel launch per activation row and segment.
  int groups = k / gs;
  for (int r = 0; r < m; r++) {
    for (int s = 0; s < count; s++) {
      const GemmQ8Segment &g = segments[s];
      KcGemvSeg seg = {g.c + (size_t)r * g.ldc, g.w.q, g.w.s, g.w3.q, g.w3.s, g.n};
      K8Input in = {xq + (size_t)r * k, xs + (size_t)r * groups, nullptr};
      if (!gemv("k_gemm_q8", &seg, 1, &in, (size_t)k, k, gs, kc_kind_of(g.kind)))
        return false;
    }
  }
  return true;
}

static int to_kc_segs(const GemmQ8Segment *segments, int count, KcGemmSeg *out) {
  for (int s = 0; s < count; s++) {
    const GemmQ8Segment &g = segments[s];
    out[s] = KcGemmSeg{g.c, g.ldc, g.w.q, g.w.s, g.w3.q, g.w3.s, g.n, kc_kind_of(g.kind)};
  }
  return count;
}

// Scratch for the transposed activation scales of k_gemm_q8, one buffer per device, grown on demand (the only
// allocation the GEMM entry points make; the engine passes its own transposed scales instead).
static float *gemm_scratch(size_t floats) {
  static std::mutex mu;
  static float *buf[64];
  static size_t cap[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64)
    return nullptr;
  std::lock_guard<std::mutex> hold(mu);
  if (cap[dev] < floats) {
    if (buf[dev])
      cudaFree(buf[dev]);
    buf[dev] = nullptr;
    cap[dev] = 0;
    if (cudaMalloc(&buf[dev], floats * sizeof(float)) != cudaSuccess)
      return nullptr;
    cap[dev] = floats;
  }
  return buf[dev];
}

// The rung k_gemm_q8 takes: the tensor-core GEMM (the reference's AMX-INT8 order, amx_q8_chunk src/gemm.c:554-610)
// for every batch it can describe, whatever the row count, so a row's result never depends on the size of its batch,
// as on the reference's AMX backend; otherwise one decode-GEMV launch per activation row, in the order of the
// reference's AVX-512 rung (q8_micro_body src/gemm.c:862-899, bitwise its GEMV) for gs % 64 == 0 and of its portable
// rung otherwise. The tensor-core GEMM needs gs 64, K % 256 == 0, 16-byte aligned operands and a SwiGLU pair as the
// only segment.
static bool tc_segments_ok(int gs, const KcGemmSeg *segs, int count) {
  if (gs != 64)
    return false;
  for (int s = 0; s < count; s++) {
    if (segs[s].kind == KC_SWIGLU && count != 1)
      return false;
    if (((uintptr_t)segs[s].wq & 15) || ((uintptr_t)segs[s].ws & 15))
      return false;
    if (segs[s].kind == KC_SWIGLU && (((uintptr_t)segs[s].w3q & 15) || ((uintptr_t)segs[s].w3s & 15)))
      return false;
  }
  return true;
}

// What k_gemm_q8 runs for these segments (src/gemm.c:991-1004 reports the same for the CPU backends). The pick sees
// neither K nor the activations: k_gemm_q8 also needs K % 256 == 0 and 16-byte aligned activation rows for the
// tensor-core rung, and takes the row rung when they are not.
Q8GemmBackend k_gemm_q8_pick(int gs, const GemmQ8Segment *segments, int count) {
  if (count < 1 || count > GEMM_MAX_SEGMENTS || !segments)
    return Q8_GEMM_GPU_DP4A;
  KcGemmSeg segs[GEMM_MAX_SEGMENTS];
  to_kc_segs(segments, count, segs);
  return tc_segments_ok(gs, segs, count) ? Q8_GEMM_GPU_TCGEN05 : Q8_GEMM_GPU_DP4A;
}

static Q8GemmBackend pick(const int8_t *xq, int m, int k, int gs, const GemmQ8Segment *segments, int count) {
  KcGemmSeg segs[GEMM_MAX_SEGMENTS];
  to_kc_segs(segments, count, segs);
  if (tc_segments_ok(gs, segs, count) && kc_gemm_tc_supported(segs, count, xq, m, k, gs))
    return Q8_GEMM_GPU_TCGEN05;
  return Q8_GEMM_GPU_DP4A;
}

static bool gemm_run(Q8GemmBackend backend, const int8_t *xq, const float *xs, int m, int k, int gs,
                     const GemmQ8Segment *segments, int count) {
  if (!gemm_args_ok("k_gemm_q8", xq, xs, m, k, gs, segments, count))
    return true;
  if (m == 0 || k == 0)
    return true;
  if (backend == Q8_GEMM_GPU_DP4A) {
    gemm_rows_dp4a(xq, xs, m, k, gs, segments, count);
    return true;
  }
  if (backend == Q8_GEMM_GPU_TCGEN05) {
    KcGemmSeg segs[GEMM_MAX_SEGMENTS];
    to_kc_segs(segments, count, segs);
    for (int s = 0; s < count; s++)
      if (segs[s].kind == KC_SWIGLU && count != 1) {
        kc_fail("k_gemm_q8: the tensor-core GEMM takes a SwiGLU pair as its only segment");
        return true;
      }
    if (!kc_gemm_tc_supported(segs, count, xq, m, k, gs)) {
      kc_fail("k_gemm_q8: shape not supported by the tensor-core GEMM (gs 64, K %% 256 == 0, aligned operands)");
      return true;
    }
    float *xsT = gemm_scratch(kc_gemm_xst_floats(m, k / gs));
    if (!xsT) {
      kc_fail("k_gemm_q8: cannot allocate the transposed-scale scratch");
      return true;
    }
    if (launched(kc_launch_transpose_scales(xsT, xs, m, k / gs, tl_stream), "k_gemm_q8"))
      launched(kc_launch_gemm_tc(segs, count, xq, xsT, m, k, nullptr, tl_stream), "k_gemm_q8");
    return true;
  }
  return false;
}

void k_gemm_q8(const int8_t *xq, const float *xs, int m, int k, int gs, const GemmQ8Segment *segments, int count) {
  // The arguments are checked before the backend is picked: pick() copies the segments into a fixed array.
  if (!gemm_args_ok("k_gemm_q8", xq, xs, m, k, gs, segments, count))
    return;
  gemm_run(pick(xq, m, k, gs, segments, count), xq, xs, m, k, gs, segments, count);
}

int k_gemm_q8_backend_test(Q8GemmBackend backend, const int8_t *xq, const float *xs, int m, int k, int gs,
                           const GemmQ8Segment *segments, int count) {
  if (backend != Q8_GEMM_GPU_DP4A && backend != Q8_GEMM_GPU_TCGEN05)
    return 0;
  return gemm_run(backend, xq, xs, m, k, gs, segments, count) ? 1 : 0;
}

int k_gemm_q8_dots_test(int32_t *dots, const int8_t *xq, int m, int k, int gs, const int8_t *wq, int n) {
  KcGemmSeg seg = {nullptr, n, wq, nullptr, nullptr, nullptr, n, KC_STORE};
  // The dots mode ignores the scales; point the scale operands at valid scratch of the right size.
  const int groups = gs > 0 ? k / gs : 0;
  float *scratch = gemm_scratch(kc_gemm_xst_floats(m, groups) + (size_t)n * groups + 4);
  if (!scratch || gs != 64 || k % 256 || m <= 0 || n <= 0 || ((uintptr_t)xq & 15) || ((uintptr_t)wq & 15))
    return 0;
  seg.ws = scratch + kc_gemm_xst_floats(m, groups);
  seg.ws = reinterpret_cast<const float *>(((uintptr_t)seg.ws + 15) & ~(uintptr_t)15);
  return kc_launch_gemm_tc(&seg, 1, xq, scratch, m, k, dots, tl_stream) == 0 ? 1 : 0;
}

// ---- k_gemm_q8 without device allocation --------------------------------------------------------------------------

// Who needs it: a serving process that hands all of HBM to its weights and KV cache at start-up has no room left for a
// buffer the GEMM would grow on first use, and a caller on a latency-bound path cannot afford the device-wide
// synchronisation cudaMalloc / cudaFree bring. The transposed scales therefore live in this fixed array of the
// library's device image (4 MiB per device); every call overwrites the [K/64][round_up(m, 4)] prefix it reads.
static __device__ __align__(256) float noalloc_scales[K_GEMM_Q8_NOALLOC_MAX_SCALES];

// The array's address on the current device, looked up once per device under a lock (two host threads making their
// first call at once both see one lookup). The cache assumes the device's context lives as long as the process: after
// cudaDeviceReset the module is loaded again at another address, so a process that resets a device must not call this
// entry point afterwards.
static float *noalloc_scales_address() {
  static std::mutex mu;
  static float *addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    kc_fail("k_gemm_q8_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> hold(mu);
  if (!addr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scales);
    if (e != cudaSuccess) {
      kc_fail("k_gemm_q8_noalloc: cannot resolve the scale array on device %d: %s", dev, cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<float *>(p);
  }
  return addr[dev];
}

int k_gemm_q8_noalloc(const int8_t *xq, const float *xs, int m, int k, int gs, const GemmQ8Segment *segments,
                      int count) {
  if (!gemm_args_ok("k_gemm_q8_noalloc", xq, xs, m, k, gs, segments, count))
    return -1;
  if (m == 0 || k == 0)
    return 0;
  const Q8GemmBackend backend = pick(xq, m, k, gs, segments, count);
  if (backend == Q8_GEMM_GPU_DP4A)  // one GEMV launch per row: no scratch at all
    return gemm_rows_dp4a(xq, xs, m, k, gs, segments, count) ? 0 : -1;
  const size_t need = kc_gemm_xst_floats(m, k / gs);
  if (need > (size_t)K_GEMM_Q8_NOALLOC_MAX_SCALES) {
    kc_fail("k_gemm_q8_noalloc: m=%d k=%d needs %zu scale floats, above the fixed %d", m, k, need,
            K_GEMM_Q8_NOALLOC_MAX_SCALES);
    return -1;
  }
  float *xsT = noalloc_scales_address();
  if (!xsT)
    return -1;
  KcGemmSeg segs[GEMM_MAX_SEGMENTS];
  to_kc_segs(segments, count, segs);
  if (!launched(kc_launch_transpose_scales(xsT, xs, m, k / gs, tl_stream), "k_gemm_q8_noalloc") ||
      !launched(kc_launch_gemm_tc(segs, count, xq, xsT, m, k, nullptr, tl_stream), "k_gemm_q8_noalloc"))
    return -1;
  return 0;
}

// ---- supporting kernels -------------------------------------------------------------------------------------------

void k_rmsnorm_rows(float *out, const float *x, const float *weight, int rows, int size, float epsilon) {
  if (rows < 0 || size <= 0) {
    kc_fail("k_rmsnorm_rows: invalid shape rows=%d size=%d", rows, size);
    return;
  }
  launched(kc_launch_rmsnorm(out, nullptr, nullptr, x, weight, rows, size, size, epsilon, 0, tl_stream),
           "k_rmsnorm_rows");
}

void k_rmsnorm(float *out, const float *x, const float *weight, int size, float epsilon) {
  k_rmsnorm_rows(out, x, weight, 1, size, epsilon);
}

void k_rmsnorm_q8_rows(int8_t *q, float *s, float *out, const float *x, size_t ldx, const float *weight, int rows,
                       int size, float epsilon, int gs) {
  if (rows < 0 || size <= 0 || gs <= 0 || size % gs || gs > 256 || ldx < (size_t)size) {
    kc_fail("k_rmsnorm_q8_rows: invalid shape rows=%d size=%d ldx=%zu gs=%d", rows, size, ldx, gs);
    return;
  }
  launched(kc_launch_rmsnorm(out, q, s, x, weight, rows, size, (long long)ldx, epsilon, gs, tl_stream),
           "k_rmsnorm_q8_rows");
}

void k_rope_apply_rows(float *q, size_t q_stride, float *k, size_t k_stride, const float *table, size_t table_stride,
                       int rows, int n_heads, int n_kv_heads, int head_dim) {
  if (rows < 0 || n_heads <= 0 || n_kv_heads <= 0 || n_kv_heads > n_heads || head_dim <= 0 || head_dim % 2) {
    kc_fail("k_rope_apply_rows: invalid shape");
    return;
  }
  launched(kc_launch_rope_rows(q, (long long)q_stride, k, (long long)k_stride, table, (long long)table_stride, rows,
                               n_heads, n_kv_heads, head_dim, tl_stream),
           "k_rope_apply_rows");
}

void k_rope_apply(float *q, float *k, const float *table, int n_heads, int n_kv_heads, int head_dim) {
  k_rope_apply_rows(q, 0, k, 0, table, 0, 1, n_heads, n_kv_heads, head_dim);
}

// ---- AMX packing helpers (host) ------------------------------------------------------------------------------------

size_t s8_vnni_bytes(int rows, int cols) {
  const size_t r = ((size_t)(rows > 0 ? rows : 0) + 15) / 16 * 16, c = ((size_t)(cols > 0 ? cols : 0) + 63) / 64 * 64;
  return r * c;
}

void pack_s8_vnni_tiles(int8_t *dst, const int8_t *w, int rows, int cols, size_t ld, int first, int last) {
  // The reference's layout (pack_s8_vnni_tiles, src/gemm.c:384-394): tile t holds rows [16 t, 16 t + 16); within it,
  // K quad k4 (columns 4 k4 .. 4 k4 + 3) is a run of 16 rows x 4 bytes; rows and columns past the matrix are zeros.
  const size_t kp = ((size_t)cols + 63) / 64 * 64;
  for (int t = first; t < last; t++) {
    int8_t *tile = dst + (size_t)t * 16 * kp;
    for (size_t k4 = 0; k4 < kp / 4; k4++)
      for (int r = 0; r < 16; r++) {
        const size_t row = (size_t)t * 16 + r;
        for (int b = 0; b < 4; b++) {
          const size_t col = 4 * k4 + b;
          tile[(k4 * 16 + r) * 4 + b] = row < (size_t)rows && col < (size_t)cols ? w[row * ld + col] : 0;
        }
      }
  }
}

void pack_s8_vnni(int8_t *dst, const int8_t *w, int rows, int cols, size_t ld) {
  pack_s8_vnni_tiles(dst, w, rows, cols, ld, 0, (rows + 15) / 16);
}

void pack_s8_vnni_many(const PackS8 *jobs, int count) {
  for (int i = 0; i < count; i++)
    pack_s8_vnni(jobs[i].dst, jobs[i].w, jobs[i].rows, jobs[i].cols, jobs[i].ld);
}

}  // extern "C"
