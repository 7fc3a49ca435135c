// Internal interface between the C-ABI layer (abi.cu) and the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// Epilogue kinds, numerically equal to the reference's KernelEpilogue / GemmKind (include/kernels.h:84,
// include/gemm.h:15-20): STORE, ADD, PARTIAL, SWIGLU. KC_REDUCE_ADD (the decode GEMV only) is PARTIAL followed by
// the tensor-parallel sum over ranks, added into the output: out += sum over ranks of this product, in rank order.
enum { KC_STORE = 0, KC_ADD = 1, KC_PARTIAL = 2, KC_SWIGLU = 3, KC_REDUCE_ADD = 4 };

// The reducing GEMV's view of the peer state (peer.cu): every rank's slot region [2 parities][world][stride] of
// 8-byte {float bits, call number} slots as mapped in this process, and this rank's per-CTA call counters. The
// reducing GEMV always launches min(SMs, kPeerGemvMaxCtas) CTAs, whatever the shape, so every counter advances on
// every call and all of them hold the number of calls made.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerGemvMaxCtas = 256;
struct KcPeerGemv {
  unsigned long long *slots[kPeerMaxRanks];
  unsigned *epoch;  // [kPeerGemvMaxCtas]
  long long stride;
  int rank, world;
};

struct KcGemvSeg {
  float *out;
  const int8_t *wq;
  const float *ws;
  const int8_t *w3q;  // SWIGLU only
  const float *w3s;
  int d;
};

int kc_device_sms();
// The calling thread's stream (kernels_set_stream) and the fail() policy of the C-ABI (kc_set_fail_mode): records the
// message, exits under KC_FAIL_EXIT, returns false under KC_FAIL_RETURN.
cudaStream_t kc_stream();
bool kc_fail(const char *format, ...);
// Counts one successful kernel launch for kc_launch_count.
void kc_count_launch();
// Programmatic dependent launch of the kernels that support it (kernels_set_pdl; on by default).
bool kc_pdl_enabled();
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device, once per (kernel, device); safe to
// call from several host threads at once.
cudaError_t kc_allow_smem(const void *kernel, int bytes);

// Launches `kernel` on `stream` with programmatic dependent launch allowed (kernels_set_pdl): it may be scheduled
// while the previous kernel in the stream drains, so every kernel launched this way starts with griddepcontrol.wait
// (pdl_wait) before it touches memory another kernel wrote or reads.
template <typename... KArgs, typename... Args>
cudaError_t kc_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = kc_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Returns 0 on launch, -1 for a shape the kernel does not support, -2 on a launch error.
int kc_launch_gemv(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld, int gs,
                   int kind, cudaStream_t stream, int grid_limit);
// The same with a tail (the TMA kernel only; -1 when the shape does not fit it). Concurrent tail GEMVs on different
// streams of one device race on the kernel's completion counter.
int kc_launch_gemv_tail(const KcGemvSeg *segs, int nseg, const int8_t *xq, const float *xs, int n, long long ld,
                        int gs, int kind, const struct KcGemvTail &tail, cudaStream_t stream);

// Work the last CTA of a decode GEMV does once, after every CTA's outputs are in memory: quantize (or RMS-normalize
// and quantize) an fp32 vector, e.g. the residual the GEMV just added into, for the next GEMV; or rotate the q and k
// rows the three QKV segments produced and store k and v into the K/V cache at *pos. Arithmetic as the separate
// kernels (k_quantize, k_rmsnorm_q8_rows, k_rope_kv_store_rows), bitwise.
// KC_TAIL_QUANTIZE_OUTPUT is not a last-CTA job: the GEMV's own output (one segment) is quantized in gs-groups, each
// by the CTA whose rows complete it.
enum { KC_TAIL_NONE = 0, KC_TAIL_QUANTIZE = 1, KC_TAIL_NORM_QUANTIZE = 2, KC_TAIL_ROPE_KV_STORE = 3,
       KC_TAIL_QUANTIZE_OUTPUT = 4 };
struct KcGemvTail {
  int kind;
  const float *x, *w;  // (NORM_)QUANTIZE: the vector [n] and the RMSNorm weights
  float eps;
  int8_t *q;
  float *s;
  int n;
  float *qv, *kv;      // ROPE_KV_STORE: q [nh * hd] rotated in place, k [nkv * hd], v [nkv * hd]
  const float *vv;
  float *kcache, *vcache;
  const float *table;  // [seq][2 * hd]
  const int *pos;
  int nh, nkv, hd, seq;
};

// fp32 input of the fused GEMV: x (n values), the RMSNorm weights (nullptr: quantize only) and epsilon. Every CTA
// normalizes and quantizes x itself into shared memory, bitwise as kc_launch_rmsnorm / kc_launch_quantize_rows.
struct KcGemvAct {
  const float *x;
  const float *norm;
  float eps;
};
// The reducing decode GEMV: one segment (out, wq, ws, d <= peer.stride), int8 activations; out[r] += the sum over
// ranks, in rank order, of every rank's product row r (0, -1 for a shape the TMA kernel does not take, -2 on a launch
// error). Every rank must make the same calls in the same order.
int kc_launch_gemv_reduce(const KcGemvSeg &seg, const int8_t *xq, const float *xs, int n, long long ld, int gs,
                          const KcPeerGemv &peer, cudaStream_t stream);

// W8A32: fp32 activations against int8 weights, the reference's orders (0, or -2 on a launch error).
int kc_launch_gemv_w8a32(const KcGemvSeg *segs, int nseg, const float *x, int n, long long ld, int gs, int kind,
                         cudaStream_t stream);
int kc_launch_gemv_f32(const KcGemvSeg *segs, int nseg, const KcGemvAct &act, int n, long long ld, int gs, int kind,
                       cudaStream_t stream, const struct KcGemvTail *tail = nullptr);

// One GEMM segment (GemmQ8Segment without the AMX-packed copies), kind in KC_* terms.
struct KcGemmSeg {
  float *c;
  int ldc;
  const int8_t *wq;
  const float *ws;
  const int8_t *w3q;  // SWIGLU only
  const float *w3s;
  int n;
  int kind;
};

// The tcgen05 GEMM (gemm_tc.cu): gs 64, K % 256 == 0, 16-byte aligned operands. It reads the activation scales
// transposed, xsT [K / 64][round_up(M, 4)] (kc_launch_transpose_scales makes them from the row-major xs).
bool kc_gemm_tc_supported(const KcGemmSeg *segs, int nseg, const int8_t *xq, int M, int K, int gs);
size_t kc_gemm_xst_floats(int M, int groups);
int kc_launch_transpose_scales(float *xsT, const float *xs, int M, int groups, cudaStream_t stream);
int kc_launch_gemm_tc(const KcGemmSeg *segs, int nseg, const int8_t *xq, const float *xsT, int M, int K,
                      int32_t *dots, cudaStream_t stream);

int kc_launch_quantize_rows(int8_t *q, float *s, const float *x, long long ldx, int m, int n, int gs,
                            cudaStream_t stream);
int kc_launch_rmsnorm(float *out, int8_t *q, float *s, const float *x, const float *w, int rows, int size,
                      long long ldx, float eps, int gs, cudaStream_t stream);
int kc_launch_rope_rows(float *q, long long q_stride, float *k, long long k_stride, const float *table,
                        long long table_stride, int rows, int n_heads, int n_kv_heads, int head_dim,
                        cudaStream_t stream);
