/* The GPU engine behind include/engine_cuda.h, in C11 like the reference's engine (src/engine.c, src/tp.c). It owns
 * the device copies of this rank's weight shards, the K/V cache and the activations, and calls CUDA only through the
 * C-ABI of libllama3x_cuda.so (include/kernels_cuda.h, include/device_cuda.h).
 *
 * Call order per layer is the reference's forward_q8 (src/tp.c:387-436) for one token and forward_batch
 * (src/tp.c:528-622) for a batch, with the norm+quantize pairs fused (k_rmsnorm_q8_rows) and RoPE fused with the K/V
 * store. With world > 1 the Wo and W2 products write a partial that an NCCL all-reduce sums before the residual add:
 * residual += (p0 + p1 + ...), which at two ranks is the reference's residual[i] += p0[i] + p1[i]
 * (src/workers.c:455-458). */
#define _POSIX_C_SOURCE 200809L
#include <errno.h>
#include <fcntl.h>
#include <limits.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/device_cuda.h"
#include "../../include/engine_cuda.h"
#include "../../include/kernels_cuda.h"

const int engine_q8 = 1;

enum { Q8_MAGIC = 0x616b3432, DEFAULT_PREFILL_BATCH = 2048, DEFAULT_CONTEXT_CAP = 4096 };

typedef struct {
  int8_t *q;
  float *s;
} Q8;

typedef struct {
  float *rms_att, *rms_ffn;
  Q8 wq, wk, wv, wo, w1, w2, w3;
} Layer;

typedef struct {
  Config c;
  int gs, S, rank, device;
  int hl, kl, hd, ql, kvl, hid_l, v0, vl, vmax;
  int context, max_batch, graphs;
  Q8 embed, cls;
  int cls_owned;
  float *rms_final;
  Layer *layers;
  float *key_cache, *value_cache;
  size_t layer_kv;
  float *rope;
  float *x, *q, *k, *v, *att, *hb, *partial;
  int8_t *xq, *aq, *hq;
  float *xs, *as, *hs;
  AttentionWork attn;
  float *logits_dev, *gather_dev, *batch_logits_dev;
  float *logits_host, *batch_logits_host;
  int *tokens_dev, *pos_dev, *step_dev, *gen_dev;
  int gen_capacity;
  unsigned long long *key_dev;
  int *staging; /* pinned: token uploads [max_batch], then the scalar uploads at staging + max_batch */
  void *stream, *comm;
  void *peer; /* peer-memory all-reduce of the decode residual (kd_peer_*), or NULL for NCCL */
  int w8a32;  /* LLAMA_Q8_ACTIVATIONS=fp32: fp32 activations against the int8 weights, one row per forward */
  long batch_env; /* rows per engine_forward_batch the environment asks for, before the context cap */
  int fused;  /* the decode step's fused GEMV modes fit these shapes (fused_shapes) */
  int rope_step; /* the decode step's RoPE + K/V store run inside its attention launch (k_rope_attention_q8_step) */
  int reduce_fused; /* with peer: Wo and W2 reduce inside their GEMV (kd_peer_matmul_q8_add, reduce_shapes) */
  float *xb;  /* W8A32: the normalized row the projections read */
  void *graph_logits, *graph_greedy;
  unsigned long long graph_logits_kernels, graph_greedy_kernels; /* kernels captured in each graph */
  long long captured, replayed; /* launch-count corrections: captured calls do not run, replays bypass the count */
  unsigned long long launches_base;
  void *ev[3];
  EngineStats stats;
} Engine;

static int last_gs;    /* engine_group_size: the group size of the last model set up */
static int last_w8a32; /* engine_precision: whether that model runs W8A32 */

static struct {
  int rank, world, device, set;
  unsigned char id[KD_COMM_ID_BYTES];
} tp_request;

/* ---- errors -------------------------------------------------------------------------------------------------------- */

static int efail(const char *format, ...) {
  char message[512];
  va_list args;
  va_start(args, format);
  vsnprintf(message, sizeof(message), format, args);
  va_end(args);
  kc_fail_message(message); /* exits under KC_FAIL_EXIT, as the reference's fail() */
  return -1;
}

static int failed(void) { return kc_last_error()[0] != 0; }

/* ---- device memory ------------------------------------------------------------------------------------------------- */

static void *dev_alloc(size_t bytes) {
  void *p = kd_malloc(bytes ? bytes : 16);
  if (p)
    kd_memset(p, 0, bytes ? bytes : 16);
  return p;
}

static Q8 q8_alloc(size_t rows, size_t cols, int gs) {
  Q8 w = {dev_alloc(rows * cols), dev_alloc(rows * (cols / (size_t)gs) * sizeof(float))};
  return w;
}

static void q8_free(Q8 *w) {
  kd_free(w->q);
  kd_free(w->s);
  w->q = NULL;
  w->s = NULL;
}

static K8Weight k8(Q8 w) {
  K8Weight r = {w.q, w.s};
  return r;
}

/* ---- RoPE table (k_rope_table / rope_frequency, src/kernels_simd.c:194-201, src/kernels.c:49-60) ---------------- */

/* The Llama 3.1 wavelength-dependent frequency scaling (rope_type 1) over the plain theta^(-j/d) frequencies. */
static float rope_freq(const Config *p, int j) {
  float f = 1.0f / powf(p->rope_theta, (float)j / (float)p->head_dim);
  if (p->rope_type == 1) {
    float wavelength = 6.2831853071795864769f / f;
    if (wavelength > p->rope_original / p->rope_low)
      f /= p->rope_factor;
    else if (wavelength >= p->rope_original / p->rope_high) {
      float smooth = (p->rope_original / wavelength - p->rope_low) / (p->rope_high - p->rope_low);
      f = (1 - smooth) * f / p->rope_factor + smooth * f;
    }
  }
  return f;
}

/* k_rope_table (include/kernels.h:67, src/kernels_simd.c:194-201): one position's row of [2 * head_dim] floats,
 * cosines duplicated per pair, then (-sin, +sin) per pair. */
void k_rope_table(const Config *p, int position, float *table) {
  int hd = p->head_dim;
  for (int j = 0; j < hd; j += 2) {
    float angle = position * rope_freq(p, j), c = cosf(angle), s = sinf(angle);
    table[j] = table[j + 1] = c;
    table[hd + j] = -s;
    table[hd + j + 1] = s;
  }
}

/* Rows [0, positions) of k_rope_table, the device copy's source. */
static float *rope_table_host(const Config *p, int positions) {
  int hd = p->head_dim;
  float *t = malloc((size_t)positions * 2 * hd * sizeof(float));
  if (!t)
    return NULL;
  for (int pos = 0; pos < positions; pos++)
    k_rope_table(p, pos, t + (size_t)pos * 2 * hd);
  return t;
}

/* ---- configuration ------------------------------------------------------------------------------------------------- */

static int validate_config(const Config *p, int gs) {
  /* validate_config (src/runtime.c:148-168) */
  if (p->dim <= 0 || p->hidden_dim <= 0 || p->n_layers <= 0 || p->n_heads <= 0 || p->n_kv_heads <= 0 ||
      p->vocab_size <= 0 || p->seq_len <= 0)
    return efail("invalid checkpoint dimensions: all seven dimensions must be positive");
  if (p->dim % p->n_heads || p->n_heads % p->n_kv_heads || (p->dim / p->n_heads) % 2)
    return efail("unsupported attention dimensions: dim must be divisible by heads, heads must be divisible by KV "
                 "heads, head size must be even");
  if (!isfinite(p->norm_eps) || p->norm_eps <= 0 || !isfinite(p->rope_theta) || p->rope_theta <= 1 ||
      p->head_dim != p->dim / p->n_heads || p->max_seq_len != p->seq_len)
    return efail("invalid RMSNorm, RoPE theta, head dimension or context metadata");
  if (p->rope_type != 0 && p->rope_type != 1)
    return efail("unsupported RoPE scaling type %d", p->rope_type);
  if (!isfinite(p->rope_factor) || !isfinite(p->rope_low) || !isfinite(p->rope_high) || p->rope_factor < 1 ||
      p->rope_low <= 0 || p->rope_high <= p->rope_low || p->rope_original <= 0)
    return efail("invalid RoPE scaling metadata");
  if (p->format == 3 && (p->bos_id < 0 || p->bos_id >= p->vocab_size || p->eos_id < 0 || p->eos_id >= p->vocab_size ||
                         p->eot_id < -1 || p->eot_id >= p->vocab_size || p->eom_id < -1 || p->eom_id >= p->vocab_size))
    return efail("invalid special token metadata");
  if (gs <= 0 || gs > 131071 || p->dim % gs || p->hidden_dim % gs)
    return efail("unsupported INT8 group size %d: must divide dim and hidden_dim and fit int32 accumulation", gs);
  return 0;
}

static void config_defaults(Config *p) {
  /* checkpoint_map's defaults for fields a version 2 header does not carry (src/runtime.c:203-213) */
  p->norm_eps = 1e-5f;
  p->rope_theta = 500000.0f;
  p->rope_factor = 1;
  p->rope_low = 1;
  p->rope_high = 4;
  p->rope_original = 8192;
  p->bos_id = 128000;
  p->eos_id = 128001;
  p->eot_id = 128009;
  p->eom_id = -1;
}

/* The shard plan (src/shards.c:190-272 for two sockets, here any world that divides the heads and groups). */
static int plan(Engine *e) {
  const Config *p = &e->c;
  int S = e->S;
  e->hd = p->head_dim;
  if (p->n_heads % S || p->n_kv_heads % S || (p->dim / S) % e->gs || (p->hidden_dim / S) % e->gs ||
      p->dim % S || p->hidden_dim % S || p->vocab_size < S)
    return efail("tensor parallelism over %d GPUs needs heads, KV heads, dim/%d and hidden/%d divisible (group size "
                 "%d)",
                 S, S, S, e->gs);
  e->hl = p->n_heads / S;
  e->kl = p->n_kv_heads / S;
  e->ql = e->hl * e->hd;
  e->kvl = e->kl * e->hd;
  e->hid_l = p->hidden_dim / S;
  /* split_range (src/shards.c:140-144): equal shares, the last rank takes the remainder */
  int each = p->vocab_size / S;
  e->v0 = e->rank * each;
  e->vl = e->rank == S - 1 ? p->vocab_size - e->v0 : each;
  e->vmax = p->vocab_size - (S - 1) * each;
  return 0;
}

/* The environment the reference's Q8 engine reads before it maps a checkpoint, with its rules and messages:
 * LLAMA_PRECISION (prefill_precision(1), src/prefill.c:9-22), LLAMA_Q8_ACTIVATIONS (src/engine.c:131-135) and
 * prefill_configure's LLAMA_PREFILL_GEMM, LLAMA_PREFILL_BATCH and LLAMA_PREFILL_LOGITS (src/prefill.c:24-50).
 * The GPU's batched GEMM gives the per-row kernel's bits, so LLAMA_PREFILL_GEMM=off only makes the default batch one
 * row. W8A32 always runs one row per forward (src/engine.c:97-104), whatever the batch asked for. */
typedef struct {
  int w8a32;
  long batch;
} Knobs;

static int read_knobs(Knobs *k) {
  const char *precision = getenv("LLAMA_PRECISION");
  if (precision && *precision && strcmp(precision, "fp32") && strcmp(precision, "bf16"))
    return efail("LLAMA_PRECISION must be fp32 or bf16");
  if (precision && !strcmp(precision, "bf16"))
    return efail("LLAMA_PRECISION=bf16 applies to FP32 checkpoints (run); Q8_0 checkpoints keep their int8 semantics "
                 "(runq)");
  const char *a = getenv("LLAMA_Q8_ACTIVATIONS");
  if (a && *a && strcmp(a, "int8") && strcmp(a, "fp32"))
    return efail("LLAMA_Q8_ACTIVATIONS must be int8 or fp32");
  k->w8a32 = a && !strcmp(a, "fp32");
  const char *gemm = getenv("LLAMA_PREFILL_GEMM");
  if (gemm && *gemm && strcmp(gemm, "auto") && strcmp(gemm, "on") && strcmp(gemm, "off"))
    return efail("LLAMA_PREFILL_GEMM must be auto, on or off");
  k->batch = k->w8a32 || (gemm && !strcmp(gemm, "off")) ? 1 : DEFAULT_PREFILL_BATCH;
  const char *b = getenv("LLAMA_PREFILL_BATCH");
  if (b && *b) {
    if (strspn(b, "0123456789") != strlen(b))
      return efail("LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX");
    errno = 0;
    char *end;
    const long count = strtol(b, &end, 10);
    if (errno || *end || count < 1 || count > INT_MAX)
      return efail("LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX");
    k->batch = count;
  }
  const char *logits = getenv("LLAMA_PREFILL_LOGITS");
  if (logits && *logits && strcmp(logits, "last") && strcmp(logits, "all"))
    return efail("LLAMA_PREFILL_LOGITS must be last or all");
  return 0;
}

/* The decode step's fused kernels (RMSNorm and quantize inside the GEMV, the output quantizer) run on the TMA GEMV,
 * which takes group sizes 16..256 that are powers of two and scale rows of whole 16-byte units. Other shapes, such as
 * the reference's gs 2 test fixtures, take the separate kernels (decode_layers_plain). */
static int fused_shapes(const Engine *e) {
  int gs = e->gs, dim = e->c.dim;
  /* The fused GEMVs read dim inputs (QKV, W1/W3, classifier); the output quantizer cuts hid_l outputs into groups. */
  return gs >= 16 && gs <= 256 && !(gs & (gs - 1)) && dim % gs == 0 && (dim / gs) % 4 == 0 && e->hid_l % gs == 0;
}

/* The reducing GEMV is the TMA GEMV on int8 inputs: Wo reads ql of them, W2 hid_l, each a whole number of 4-group
 * units. LLAMA_PEER_GEMV=0 (the same on every rank) keeps the PARTIAL GEMV + kd_peer_allreduce_add pair instead. */
static int reduce_shapes(const Engine *e) {
  int gs = e->gs;
  const char *off = getenv("LLAMA_PEER_GEMV");
  return !(off && !strcmp(off, "0")) && e->fused && e->ql % gs == 0 && (e->ql / gs) % 4 == 0 &&
         (e->hid_l / gs) % 4 == 0;
}

/* Rows per engine_forward_batch: W8A32 never batches (src/engine.c:97-104), else LLAMA_PREFILL_BATCH. Also fixes
 * which decode kernels the shard shapes allow. */
static int max_batch_for(Engine *e) {
  e->fused = fused_shapes(e); /* plan() has set the shard shapes */
  e->rope_step = k_rope_attention_q8_step_ok(e->hl, e->kl, e->hd, e->gs);
  e->reduce_fused = reduce_shapes(e);
  return e->w8a32 ? 1 : e->batch_env < e->context ? (int)e->batch_env : e->context;
}

/* Device buffers sized for the context and the batch. */
static int allocate_state(Engine *e) {
  const Config *p = &e->c;
  size_t B = (size_t)e->max_batch, dim = (size_t)p->dim;
  e->layer_kv = (size_t)e->kl * e->context * e->hd;
  e->key_cache = dev_alloc(e->layer_kv * p->n_layers * sizeof(float));
  e->value_cache = dev_alloc(e->layer_kv * p->n_layers * sizeof(float));
  e->x = dev_alloc(B * dim * sizeof(float));
  e->q = dev_alloc(B * e->ql * sizeof(float));
  e->k = dev_alloc(B * e->kvl * sizeof(float));
  e->v = dev_alloc(B * e->kvl * sizeof(float));
  e->att = dev_alloc(B * e->ql * sizeof(float));
  e->hb = dev_alloc(B * e->hid_l * sizeof(float));
  e->partial = e->S > 1 ? dev_alloc(B * dim * sizeof(float)) : NULL;
  e->xq = dev_alloc(B * dim);
  e->xs = dev_alloc(B * (dim / e->gs) * sizeof(float));
  e->aq = dev_alloc(B * e->ql);
  e->as = dev_alloc(B * (e->ql / e->gs) * sizeof(float));
  e->hq = dev_alloc(B * e->hid_l);
  e->hs = dev_alloc(B * (e->hid_l / e->gs) * sizeof(float));
  e->xb = e->w8a32 ? dev_alloc(B * dim * sizeof(float)) : NULL;
  e->logits_dev = dev_alloc((size_t)e->vmax * sizeof(float));
  e->gather_dev = e->S > 1 ? dev_alloc((size_t)e->vmax * e->S * sizeof(float)) : NULL;
  e->logits_host = kd_host_alloc((size_t)p->vocab_size * sizeof(float));
  e->tokens_dev = dev_alloc(B * sizeof(int));
  e->pos_dev = dev_alloc(sizeof(int));
  e->step_dev = dev_alloc(sizeof(int));
  e->key_dev = dev_alloc(sizeof(unsigned long long));
  e->staging = kd_host_alloc((B + 16) * sizeof(int));
  for (int i = 0; i < 3; i++)
    e->ev[i] = kd_event_create();
  if (failed())
    return -1;
  /* The chunk partials of one row (decode) or of a batch's rows (prefill, in waves when they exceed the work). */
  k_attention_init_rows(&e->attn, e->hl, e->kl, e->hd, e->context, e->max_batch, NULL);
  float *table = rope_table_host(p, e->context);
  if (!table)
    return efail("cannot allocate the RoPE table");
  e->rope = dev_alloc((size_t)e->context * 2 * e->hd * sizeof(float));
  if (e->rope)
    kd_copy(e->rope, table, (size_t)e->context * 2 * e->hd * sizeof(float));
  kd_sync();
  free(table);
  return failed() ? -1 : 0;
}

static Engine *engine_create(Model *model) {
  Engine *e = calloc(1, sizeof(Engine));
  if (!e) {
    efail("cannot allocate the engine");
    return NULL;
  }
  e->S = tp_request.set ? tp_request.world : 1;
  e->rank = tp_request.set ? tp_request.rank : 0;
  e->device = tp_request.set ? tp_request.device : kd_get_device();
  if (e->device < 0 || kd_set_device(e->device)) {
    efail("no usable CUDA device");
    free(e);
    return NULL;
  }
  kernels_init();
  if (!kernels_name()) {
    free(e);
    return NULL;
  }
  e->stream = kd_stream_create();
  kernels_set_stream(e->stream);
  const char *g = getenv("LLAMA_CUDA_GRAPHS");
  e->graphs = !(g && !strcmp(g, "0"));
  model->implementation = e;
  return e;
}

/* 1 on every rank if every rank has its peer path, else 0 everywhere (the others release theirs). A max all-reduce of
 * "this rank lacks it" over NCCL, through the engine's device scratch key. */
static int agree_on_peer(Engine *e) {
  unsigned long long lack = e->peer ? 0 : 1, *d = (unsigned long long *)kd_malloc(sizeof(lack));
  if (!d)
    return -1;
  int rc = kd_copy(d, &lack, sizeof(lack)) || kd_allreduce_max_u64(e->comm, d, 1) || kd_copy(&lack, d, sizeof(lack)) ||
           kd_sync();
  kd_free(d);
  if (rc)
    return -1;
  if (lack && e->peer) {
    kd_peer_free(e->peer);
    e->peer = NULL;
  }
  return 0;
}

static int connect(Engine *e) {
  if (e->S == 1)
    return 0;
  e->comm = kd_comm_init(e->rank, e->S, tp_request.id);
  if (!e->comm)
    return -1;
  /* The decode step's two residual reductions per layer go through peer memory unless LLAMA_PEER_ALLREDUCE=0, or the
   * node does not allow the mapping (kd_peer_init says so on stderr and returns NULL): then NCCL reduces. Every rank
   * takes the same path: a rank whose set-up failed tells the others through one small all-reduce. */
  const char *peer = getenv("LLAMA_PEER_ALLREDUCE");
  if (!(peer && !strcmp(peer, "0")))
    e->peer = kd_peer_init(e->comm, e->rank, e->S, (size_t)e->c.dim);
  return agree_on_peer(e);
}

static void publish(Model *model, Engine *e) {
  last_gs = e->gs;
  last_w8a32 = e->w8a32;
  e->launches_base = kc_launch_count();
  model->config = e->c;
  model->max_batch = e->max_batch;
  const char *logits = getenv("LLAMA_PREFILL_LOGITS");
  model->prefill_logits = logits && !strcmp(logits, "all") ? LOGITS_ALL : LOGITS_LAST;
  model->prefill_gemm = e->max_batch > 1;
  model->prefill_kernel = model->prefill_gemm ? "tcgen05-int8" : NULL;
  model->prefill_bf16 = 0;
}

/* ---- loading a checkpoint (checkpoint_map, src/runtime.c:179-310) ------------------------------------------------ */

typedef struct {
  const unsigned char *base;
  size_t cursor, bytes;
  int gs;
} Reader;

/* A Q8 tensor [rows][cols] at the cursor: values, then fp32 scales (no padding). */
typedef struct {
  const int8_t *q;
  const float *s;
  size_t rows, cols;
} HostQ8;

static HostQ8 next_q8(Reader *r, size_t rows, size_t cols) {
  HostQ8 t = {(const int8_t *)(r->base + r->cursor), (const float *)(r->base + r->cursor + rows * cols), rows, cols};
  r->cursor += rows * cols + rows * cols / (size_t)r->gs * sizeof(float);
  return t;
}

static const float *next_f32(Reader *r, size_t count) {
  const float *p = (const float *)(r->base + r->cursor);
  r->cursor += count * sizeof(float);
  return p;
}

/* Rows [r0, r0 + n) of a host tensor to a new device tensor. */
static Q8 upload_rows(const HostQ8 *t, size_t r0, size_t n, int gs) {
  Q8 w = q8_alloc(n, t->cols, gs);
  if (w.q && w.s) {
    kd_copy(w.q, t->q + r0 * t->cols, n * t->cols);
    kd_copy(w.s, t->s + r0 * (t->cols / gs), n * (t->cols / gs) * sizeof(float));
  }
  return w;
}

/* Columns [c0, c0 + n) of every row (c0 and n multiples of gs). */
static Q8 upload_cols(const HostQ8 *t, size_t c0, size_t n, int gs) {
  Q8 w = q8_alloc(t->rows, n, gs);
  if (w.q && w.s) {
    kd_copy_2d(w.q, n, t->q + c0, t->cols, n, t->rows);
    kd_copy_2d(w.s, n / gs * sizeof(float), t->s + c0 / gs, t->cols / gs * sizeof(float), n / gs * sizeof(float),
               t->rows);
  }
  return w;
}

static float *upload_f32(const float *src, size_t count) {
  float *d = dev_alloc(count * sizeof(float));
  if (d)
    kd_copy(d, src, count * sizeof(float));
  return d;
}

/* checkpoint_map's header rules for the INT8 executable (src/runtime.c:214-275). */
static int read_header(const char *path, const unsigned char *h, size_t bytes, Config *p, int *gs) {
  memset(p, 0, sizeof(*p));
  config_defaults(p);
  uint32_t magic = 0;
  int version, shared = 0;
  if (bytes >= 256)
    memcpy(&magic, h, 4);
  if (magic != Q8_MAGIC)
    return efail("unsupported INT8 checkpoint: expected ak42 version 2 or 3");
  memcpy(&version, h + 4, 4);
  if (version == 3) {
    int precision;
    memcpy(&precision, h + 36, 4);
    if (precision < 0 || precision > 1)
      return efail("unsupported checkpoint precision %d", precision);
    if (precision != 1)
      return efail("checkpoint precision requires run executable");
    memcpy(p, h + 8, 28);
    memcpy(&shared, h + 40, 4);
    memcpy(gs, h + 44, 4);
    memcpy(&p->norm_eps, h + 48, 4);
    memcpy(&p->rope_theta, h + 52, 4);
    memcpy(&p->rope_type, h + 56, 4);
    memcpy(&p->rope_factor, h + 60, 4);
    memcpy(&p->rope_low, h + 64, 4);
    memcpy(&p->rope_high, h + 68, 4);
    memcpy(&p->rope_original, h + 72, 4);
    memcpy(&p->max_seq_len, h + 76, 4);
    memcpy(&p->head_dim, h + 80, 4);
    memcpy(&p->bos_id, h + 84, 4);
    memcpy(&p->eos_id, h + 88, 4);
    memcpy(&p->eot_id, h + 92, 4);
    memcpy(&p->eom_id, h + 96, 4);
    memcpy(p->name, h + 100, 128);
    if (!memchr(p->name, 0, 128))
      return efail("unterminated model name");
    for (int i = 228; i < 256; i++)
      if (h[i])
        return efail("unsupported nonzero reserved checkpoint metadata");
  } else if (version == 2) {
    memcpy(p, h + 8, 28);
    shared = h[36];
    memcpy(gs, h + 37, 4);
  } else {
    return efail("unsupported checkpoint version %d for this executable", version);
  }
  p->format = version;
  if (shared < 0 || shared > 1)
    return efail("invalid classifier flag in '%s'", path);
  p->shared = shared;
  if (version != 3) {
    p->max_seq_len = p->seq_len;
    p->head_dim = p->n_heads > 0 ? p->dim / p->n_heads : 0;
  }
  return validate_config(p, *gs);
}

/* Size arithmetic of a checkpoint the header describes, failing on overflow as checked_mul / checked_add do
 * (src/runtime.c:70-78): a header whose sizes wrap around must not pass the truncation check. *of records the first
 * overflow (which has failed) and makes the rest return 0. */
static size_t mul_checked(size_t a, size_t b, int *of) {
  if (*of)
    return 0;
  if (a && b > SIZE_MAX / a) {
    *of = 1;
    efail("size multiplication overflow: %zu * %zu", a, b);
    return 0;
  }
  return a * b;
}

static size_t add_checked(size_t a, size_t b, int *of) {
  if (*of)
    return 0;
  if (b > SIZE_MAX - a) {
    *of = 1;
    efail("size addition overflow: %zu + %zu", a, b);
    return 0;
  }
  return a + b;
}

/* tensor_bytes (src/runtime.c:170-177): scales follow the bytes unpadded, so a count that is not a multiple of gs and
 * of 4 would leave them unaligned; the reference refuses such a file with this message. */
static size_t q8_bytes(size_t count, int gs, int *of) {
  if (*of)
    return 0;
  if (count % (size_t)gs || count % sizeof(float)) {
    *of = 1;
    efail("unsupported INT8 tensor alignment/group size: %zu elements", count);
    return 0;
  }
  return add_checked(count, mul_checked(count / (size_t)gs, sizeof(float), of), of);
}

/* Bytes of a Q8 checkpoint (src/runtime.c:276-290); 0 after an overflow, which has already failed. */
static size_t checkpoint_bytes(const Config *p, int gs) {
  int of = 0;
  size_t d = p->dim, h = p->hidden_dim, l = p->n_layers, v = p->vocab_size;
  size_t kv = mul_checked((size_t)p->head_dim, (size_t)p->n_kv_heads, &of);
  size_t norms = mul_checked(add_checked(mul_checked(2, l, &of), 1, &of), d, &of);
  size_t embedding = q8_bytes(mul_checked(v, d, &of), gs, &of);
  size_t n = add_checked(256, mul_checked(norms, sizeof(float), &of), &of);
  n = add_checked(n, embedding, &of);
  size_t layer = mul_checked(2, q8_bytes(mul_checked(d, d, &of), gs, &of), &of);
  layer = add_checked(layer, mul_checked(2, q8_bytes(mul_checked(d, kv, &of), gs, &of), &of), &of);
  layer = add_checked(layer, mul_checked(3, q8_bytes(mul_checked(d, h, &of), gs, &of), &of), &of);
  n = add_checked(n, mul_checked(l, layer, &of), &of);
  if (!p->shared)
    n = add_checked(n, embedding, &of);
  return of ? 0 : n;
}

static int load_weights(Engine *e, const unsigned char *base, size_t bytes) {
  const Config *p = &e->c;
  int L = p->n_layers, gs = e->gs;
  size_t d = p->dim, h = p->hidden_dim, kv = (size_t)p->head_dim * p->n_kv_heads, v = p->vocab_size;
  Reader r = {base, 256, bytes, gs};
  e->layers = calloc((size_t)L, sizeof(Layer));
  if (!e->layers)
    return efail("cannot allocate the layer table");
  /* src/shards.c:80-97: norms (rms_att[L], rms_ffn[L], rms_final), embedding, wq..w3 per role, classifier */
  for (int l = 0; l < L; l++)
    e->layers[l].rms_att = upload_f32(next_f32(&r, d), d);
  for (int l = 0; l < L; l++)
    e->layers[l].rms_ffn = upload_f32(next_f32(&r, d), d);
  e->rms_final = upload_f32(next_f32(&r, d), d);
  HostQ8 embed = next_q8(&r, v, d);
  e->embed = upload_rows(&embed, 0, v, gs);
  size_t qrow0 = (size_t)e->rank * e->ql, kvrow0 = (size_t)e->rank * e->kvl, hrow0 = (size_t)e->rank * e->hid_l;
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, d, d);
    e->layers[l].wq = upload_rows(&t, qrow0, e->ql, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, kv, d);
    e->layers[l].wk = upload_rows(&t, kvrow0, e->kvl, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, kv, d);
    e->layers[l].wv = upload_rows(&t, kvrow0, e->kvl, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, d, d);
    e->layers[l].wo = e->S == 1 ? upload_rows(&t, 0, d, gs) : upload_cols(&t, qrow0, e->ql, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, h, d);
    e->layers[l].w1 = upload_rows(&t, hrow0, e->hid_l, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, d, h);
    e->layers[l].w2 = e->S == 1 ? upload_rows(&t, 0, d, gs) : upload_cols(&t, hrow0, e->hid_l, gs);
  }
  for (int l = 0; l < L; l++) {
    HostQ8 t = next_q8(&r, h, d);
    e->layers[l].w3 = upload_rows(&t, hrow0, e->hid_l, gs);
  }
  if (p->shared) {
    e->cls.q = e->embed.q + (size_t)e->v0 * d;
    e->cls.s = e->embed.s + (size_t)e->v0 * (d / gs);
    e->cls_owned = 0;
  } else {
    HostQ8 t = next_q8(&r, v, d);
    e->cls = upload_rows(&t, (size_t)e->v0, (size_t)e->vl, gs);
    e->cls_owned = 1;
  }
  kd_sync();
  return failed() ? -1 : 0;
}

void engine_load(Model *model, const char *path) { engine_load_context(model, path, 0); }

void engine_load_context(Model *model, const char *path, int context) {
  kc_clear_error();
  memset(model, 0, sizeof(*model));
  Knobs knobs;
  if (read_knobs(&knobs))
    return;
  int fd = open(path, O_RDONLY);
  if (fd < 0) {
    efail("cannot open checkpoint '%s': %s", path, strerror(errno));
    return;
  }
  struct stat st;
  if (fstat(fd, &st) || !S_ISREG(st.st_mode) || st.st_size < 256) {
    close(fd);
    efail("invalid/truncated checkpoint '%s': expected a regular file with complete header", path);
    return;
  }
  size_t bytes = (size_t)st.st_size;
  unsigned char *base = mmap(NULL, bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (base == MAP_FAILED) {
    efail("cannot map checkpoint '%s'", path);
    return;
  }
  Config p;
  int gs = 0;
  if (read_header(path, base, bytes, &p, &gs)) {
    munmap(base, bytes);
    return;
  }
  size_t needed = checkpoint_bytes(&p, gs);
  if (!needed) {
    munmap(base, bytes);
    return;
  }
  if (needed > bytes) {
    munmap(base, bytes);
    efail("truncated checkpoint '%s': need %zu bytes, found %zu", path, needed, bytes);
    return;
  }
  if (p.format == 3 && needed != bytes) {
    munmap(base, bytes);
    efail("version 3 checkpoint has unexpected trailing bytes");
    return;
  }
  if (context < 0 || context > p.seq_len) {
    munmap(base, bytes);
    efail("requested context exceeds checkpoint context");
    return;
  }
  Engine *e = engine_create(model);
  if (!e) {
    munmap(base, bytes);
    return;
  }
  e->c = p;
  e->gs = gs;
  e->context = context ? context : (p.seq_len < DEFAULT_CONTEXT_CAP ? p.seq_len : DEFAULT_CONTEXT_CAP);
  e->c.seq_len = e->context;
  model->file_bytes = bytes;
  e->w8a32 = knobs.w8a32;
  e->batch_env = knobs.batch;
  if (plan(e) || (e->max_batch = max_batch_for(e)) < 0 || connect(e) || allocate_state(e) ||
      load_weights(e, base, bytes)) {
    munmap(base, bytes);
    engine_free(model);
    return;
  }
  munmap(base, bytes);
  publish(model, e);
}

void engine_init_random(Model *model, const Config *config, int group_size, unsigned long long seed, int context) {
  kc_clear_error();
  memset(model, 0, sizeof(*model));
  Knobs knobs;
  if (read_knobs(&knobs))
    return;
  Config p;
  memset(&p, 0, sizeof(p));
  memcpy(&p, config, 7 * sizeof(int));
  config_defaults(&p);
  p.format = 2;
  p.shared = config->shared ? 1 : 0;
  p.max_seq_len = p.seq_len;
  p.head_dim = p.n_heads > 0 ? p.dim / p.n_heads : 0;
  if (validate_config(&p, group_size))
    return;
  if (context < 0 || context > p.seq_len) {
    efail("requested context exceeds the model's context");
    return;
  }
  Engine *e = engine_create(model);
  if (!e)
    return;
  e->c = p;
  e->gs = group_size;
  e->context = context ? context : p.seq_len;
  e->c.seq_len = e->context;
  e->w8a32 = knobs.w8a32;
  e->batch_env = knobs.batch;
  if (plan(e) || (e->max_batch = max_batch_for(e)) < 0 || connect(e) || allocate_state(e)) {
    engine_free(model);
    return;
  }
  int L = p.n_layers, gs = group_size;
  size_t d = p.dim, h = p.hidden_dim, v = p.vocab_size;
  const float std = 0.02f;
  e->layers = calloc((size_t)L, sizeof(Layer));
  if (!e->layers) {
    efail("cannot allocate the layer table");
    engine_free(model);
    return;
  }
  /* Tensor numbers: 0 embedding, 1 classifier, 2 + 7 * layer + role (wq wk wv wo w1 w2 w3). */
  e->embed = q8_alloc(v, d, gs);
  k_random_q8(e->embed.q, e->embed.s, (int)v, (int)d, 0, 0, d, seed, 0, std, gs);
  size_t qrow0 = (size_t)e->rank * e->ql, kvrow0 = (size_t)e->rank * e->kvl, hrow0 = (size_t)e->rank * e->hid_l;
  for (int l = 0; l < L && !failed(); l++) {
    Layer *y = &e->layers[l];
    unsigned long long t = 2 + 7ull * l;
    y->rms_att = dev_alloc(d * sizeof(float));
    y->rms_ffn = dev_alloc(d * sizeof(float));
    k_fill(y->rms_att, d, 1.0f);
    k_fill(y->rms_ffn, d, 1.0f);
    y->wq = q8_alloc(e->ql, d, gs);
    k_random_q8(y->wq.q, y->wq.s, e->ql, (int)d, qrow0, 0, d, seed, t + 0, std, gs);
    y->wk = q8_alloc(e->kvl, d, gs);
    k_random_q8(y->wk.q, y->wk.s, e->kvl, (int)d, kvrow0, 0, d, seed, t + 1, std, gs);
    y->wv = q8_alloc(e->kvl, d, gs);
    k_random_q8(y->wv.q, y->wv.s, e->kvl, (int)d, kvrow0, 0, d, seed, t + 2, std, gs);
    y->wo = q8_alloc(d, e->ql, gs);
    k_random_q8(y->wo.q, y->wo.s, (int)d, e->ql, 0, e->S == 1 ? 0 : qrow0, d, seed, t + 3, std, gs);
    y->w1 = q8_alloc(e->hid_l, d, gs);
    k_random_q8(y->w1.q, y->w1.s, e->hid_l, (int)d, hrow0, 0, d, seed, t + 4, std, gs);
    y->w2 = q8_alloc(d, e->hid_l, gs);
    k_random_q8(y->w2.q, y->w2.s, (int)d, e->hid_l, 0, e->S == 1 ? 0 : hrow0, h, seed, t + 5, std, gs);
    y->w3 = q8_alloc(e->hid_l, d, gs);
    k_random_q8(y->w3.q, y->w3.s, e->hid_l, (int)d, hrow0, 0, d, seed, t + 6, std, gs);
  }
  e->rms_final = dev_alloc(d * sizeof(float));
  k_fill(e->rms_final, d, 1.0f);
  if (p.shared) {
    e->cls.q = e->embed.q + (size_t)e->v0 * d;
    e->cls.s = e->embed.s + (size_t)e->v0 * (d / gs);
  } else {
    e->cls = q8_alloc((size_t)e->vl, d, gs);
    e->cls_owned = 1;
    k_random_q8(e->cls.q, e->cls.s, e->vl, (int)d, (size_t)e->v0, 0, d, seed, 1, std, gs);
  }
  kd_sync();
  if (failed()) {
    engine_free(model);
    return;
  }
  publish(model, e);
}

/* ---- forward ------------------------------------------------------------------------------------------------------- */

static void residual_reduce(Engine *e, int rows) {
  size_t n = (size_t)rows * e->c.dim;
  if (rows == 1 && e->peer) {
    kd_peer_allreduce_add(e->peer, e->x, e->partial, n);
    return;
  }
  kd_allreduce_sum_f32(e->comm, e->partial, n);
  k_add(e->x, e->partial, n);
}

static GemmQ8Segment segment(float *c, int ldc, Q8 w, Q8 w3, int n, GemmKind kind) {
  GemmQ8Segment g = {c, ldc, k8(w), k8(w3), NULL, NULL, n, kind};
  return g;
}

/* The W8A32 token (forward_q8 with fp32 activations, src/tp.c:379-436): every projection reads the fp32 vector itself
 * (the normalized row, the attention output, the SwiGLU output), nothing is quantized. */
static void decode_layers_w8a32(Engine *e) {
  const Config *p = &e->c;
  int dim = p->dim, gs = e->gs;
  K8Input xin = {NULL, NULL, e->xb}, ain = {NULL, NULL, e->att}, hin = {NULL, NULL, e->hb};
  k_embed_q8_rows(e->x, e->tokens_dev, k8(e->embed), 1, dim, gs, p->vocab_size);
  for (int l = 0; l < p->n_layers; l++) {
    Layer *y = &e->layers[l];
    float *kc = e->key_cache + (size_t)l * e->layer_kv, *vc = e->value_cache + (size_t)l * e->layer_kv;
    k_rmsnorm(e->xb, e->x, y->rms_att, dim, p->norm_eps);
    k_matmul_q8_qkv(e->q, e->k, e->v, &xin, k8(y->wq), k8(y->wk), k8(y->wv), dim, e->ql, e->kvl, gs);
    k_rope_kv_store_rows(e->q, e->ql, e->k, e->v, e->kvl, kc, vc, e->rope, e->pos_dev, 0, 1, e->hl, e->kl, e->hd,
                         e->context);
    k_attention_q8_rows(e->att, NULL, NULL, e->q, kc, vc, &e->attn, e->hl, e->kl, e->hd, e->context, e->pos_dev, 0,
                        1, gs);
    K8Weight wo = k8(y->wo), w2 = k8(y->w2);
    k_matmul_q8_ld(e->S == 1 ? e->x : e->partial, &ain, &wo, e->ql, e->ql, dim, gs, e->S == 1 ? K_ADD : K_PARTIAL);
    if (e->S > 1)
      residual_reduce(e, 1);
    k_rmsnorm(e->xb, e->x, y->rms_ffn, dim, p->norm_eps);
    k_matmul_q8_swiglu(e->hb, &xin, k8(y->w1), k8(y->w3), dim, e->hid_l, gs);
    k_matmul_q8_ld(e->S == 1 ? e->x : e->partial, &hin, &w2, e->hid_l, e->hid_l, dim, gs,
                   e->S == 1 ? K_ADD : K_PARTIAL);
    if (e->S > 1)
      residual_reduce(e, 1);
  }
  k_rmsnorm(e->xb, e->x, e->rms_final, dim, p->norm_eps);
  k_matmul_q8(e->logits_dev, &xin, k8(e->cls), dim, e->vl, gs);
}

/* The W8A8 token on the separate kernels, for shapes the fused GEMV does not take (fused_shapes): RMSNorm + quantize,
 * the GEMV, the quantize of the attention and SwiGLU outputs as their own launches (forward_q8, src/tp.c:387-436). */
static void decode_layers_plain(Engine *e) {
  const Config *p = &e->c;
  int dim = p->dim, gs = e->gs;
  K8Input in = {e->xq, e->xs, NULL}, att = {e->aq, e->as, NULL}, hid = {e->hq, e->hs, NULL};
  k_embed_q8_rows(e->x, e->tokens_dev, k8(e->embed), 1, dim, gs, p->vocab_size);
  for (int l = 0; l < p->n_layers; l++) {
    Layer *y = &e->layers[l];
    float *kc = e->key_cache + (size_t)l * e->layer_kv, *vc = e->value_cache + (size_t)l * e->layer_kv;
    k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x, dim, y->rms_att, 1, dim, p->norm_eps, gs);
    k_matmul_q8_qkv(e->q, e->k, e->v, &in, k8(y->wq), k8(y->wk), k8(y->wv), dim, e->ql, e->kvl, gs);
    k_rope_kv_store_rows(e->q, e->ql, e->k, e->v, e->kvl, kc, vc, e->rope, e->pos_dev, 0, 1, e->hl, e->kl, e->hd,
                         e->context);
    k_attention_q8_rows(e->att, e->aq, e->as, e->q, kc, vc, &e->attn, e->hl, e->kl, e->hd, e->context, e->pos_dev, 0,
                        1, gs);
    K8Weight wo = k8(y->wo), w2 = k8(y->w2);
    k_matmul_q8_ld(e->S == 1 ? e->x : e->partial, &att, &wo, e->ql, e->ql, dim, gs, e->S == 1 ? K_ADD : K_PARTIAL);
    if (e->S > 1)
      residual_reduce(e, 1);
    k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x, dim, y->rms_ffn, 1, dim, p->norm_eps, gs);
    k_matmul_q8_swiglu(e->hb, &in, k8(y->w1), k8(y->w3), dim, e->hid_l, gs);
    k_quantize(e->hq, e->hs, e->hb, e->hid_l, gs);
    k_matmul_q8_ld(e->S == 1 ? e->x : e->partial, &hid, &w2, e->hid_l, e->hid_l, dim, gs,
                   e->S == 1 ? K_ADD : K_PARTIAL);
    if (e->S > 1)
      residual_reduce(e, 1);
  }
  k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x, dim, e->rms_final, 1, dim, p->norm_eps, gs);
  k_matmul_q8(e->logits_dev, &in, k8(e->cls), dim, e->vl, gs);
}

/* One token at the position in e->pos_dev (device), its id in e->tokens_dev[0]: everything up to the local logits.
 * The RMSNorm + quantize before QKV, W1/W3 and the classifier run inside those GEMVs (k_matmul_q8_fused), and the
 * SwiGLU GEMV quantizes its own output for W2 (K_TAIL_QUANTIZE_OUTPUT): bitwise the separate kernels the batched
 * path uses. */
static void decode_layers(Engine *e) {
  if (e->w8a32) {
    decode_layers_w8a32(e);
    return;
  }
  if (!e->fused) {
    decode_layers_plain(e);
    return;
  }
  const Config *p = &e->c;
  int dim = p->dim, gs = e->gs;
  Q8 none = {NULL, NULL};
  K8Input att = {e->aq, e->as, NULL}, hid = {e->hq, e->hs, NULL};
  /* The SwiGLU GEMV quantizes its output for W2 itself, each group by the CTA that completes it. */
  KernelTail quant_hidden;
  memset(&quant_hidden, 0, sizeof(quant_hidden));
  quant_hidden.kind = K_TAIL_QUANTIZE_OUTPUT;
  quant_hidden.q = e->hq;
  quant_hidden.s = e->hs;
  k_embed_q8_rows(e->x, e->tokens_dev, k8(e->embed), 1, dim, gs, p->vocab_size);
  for (int l = 0; l < p->n_layers; l++) {
    Layer *y = &e->layers[l];
    float *kc = e->key_cache + (size_t)l * e->layer_kv, *vc = e->value_cache + (size_t)l * e->layer_kv;
    GemmQ8Segment qkv[3] = {segment(e->q, e->ql, y->wq, none, e->ql, GEMM_STORE),
                            segment(e->k, e->kvl, y->wk, none, e->kvl, GEMM_STORE),
                            segment(e->v, e->kvl, y->wv, none, e->kvl, GEMM_STORE)};
    k_matmul_q8_fused(e->x, y->rms_att, p->norm_eps, dim, dim, gs, qkv, 3, NULL);
    if (e->rope_step) {
      k_rope_attention_q8_step(e->att, e->aq, e->as, e->q, e->k, e->v, kc, vc, e->rope, &e->attn, e->hl, e->kl, e->hd,
                               e->context, e->pos_dev, gs);
    } else {
      k_rope_kv_store_rows(e->q, e->ql, e->k, e->v, e->kvl, kc, vc, e->rope, e->pos_dev, 0, 1, e->hl, e->kl, e->hd,
                           e->context);
      k_attention_q8_rows(e->att, e->aq, e->as, e->q, kc, vc, &e->attn, e->hl, e->kl, e->hd, e->context, e->pos_dev,
                          0, 1, gs);
    }
    /* Tensor parallel with the peer path: the shard's product and the sum over ranks in one kernel. */
    const int reduce_in_gemv = e->S > 1 && e->peer && e->reduce_fused;
    if (e->S == 1) {
      k_matmul_q8_add(e->x, &att, k8(y->wo), e->ql, dim, gs);
    } else if (reduce_in_gemv) {
      kd_peer_matmul_q8_add(e->peer, e->x, e->aq, e->as, y->wo.q, y->wo.s, (size_t)e->ql, e->ql, dim, gs);
    } else {
      K8Weight wo = k8(y->wo);
      k_matmul_q8_ld(e->partial, &att, &wo, e->ql, e->ql, dim, gs, K_PARTIAL);
      residual_reduce(e, 1);
    }
    GemmQ8Segment up = segment(e->hb, e->hid_l, y->w1, y->w3, e->hid_l, GEMM_SWIGLU);
    k_matmul_q8_fused(e->x, y->rms_ffn, p->norm_eps, dim, dim, gs, &up, 1, &quant_hidden);
    if (reduce_in_gemv) {
      kd_peer_matmul_q8_add(e->peer, e->x, e->hq, e->hs, y->w2.q, y->w2.s, (size_t)e->hid_l, e->hid_l, dim, gs);
    } else {
      K8Weight w2 = k8(y->w2);
      k_matmul_q8_ld(e->S == 1 ? e->x : e->partial, &hid, &w2, e->hid_l, e->hid_l, dim, gs,
                     e->S == 1 ? K_ADD : K_PARTIAL);
      if (e->S > 1)
        residual_reduce(e, 1);
    }
  }
  GemmQ8Segment cls = segment(e->logits_dev, e->vl, e->cls, none, e->vl, GEMM_STORE);
  k_matmul_q8_fused(e->x, e->rms_final, p->norm_eps, dim, dim, gs, &cls, 1, NULL);
}

/* The decode step that hands logits to the host: every rank's shard gathered into gather_dev. */
static void decode_logits_step(Engine *e) {
  decode_layers(e);
  if (e->S > 1)
    kd_allgather_f32(e->comm, e->logits_dev, e->gather_dev, (size_t)e->vmax);
}

/* The greedy decode step: argmax over the shards, then the next token and position on the device. */
static void decode_greedy_step(Engine *e) {
  decode_layers(e);
  k_argmax_key(e->key_dev, e->logits_dev, e->vl, e->v0);
  if (e->S > 1)
    kd_allreduce_max_u64(e->comm, e->key_dev, 1);
  k_greedy_advance(e->gen_dev, e->step_dev, e->tokens_dev, e->pos_dev, e->key_dev);
}

static int run_step(Engine *e, void **graph, unsigned long long *kernels, void (*step)(Engine *)) {
  if (!e->graphs) {
    step(e);
    return failed() ? -1 : 0;
  }
  if (!*graph) {
    unsigned long long before = kc_launch_count();
    if (kd_capture_begin())
      return -1;
    step(e);
    void *g = kd_capture_end();
    if (!g || failed()) {
      kd_graph_free(g);
      return -1;
    }
    *graph = g;
    *kernels = kc_launch_count() - before;
    e->captured += (long long)*kernels;
  }
  e->replayed += (long long)*kernels;
  return kd_graph_launch(*graph);
}

static void copy_logits_host(Engine *e, float *host, const float *local, const float *gathered) {
  if (e->S == 1) {
    kd_copy(host, local, (size_t)e->c.vocab_size * sizeof(float));
    return;
  }
  int each = e->c.vocab_size / e->S;
  for (int r = 0; r < e->S; r++) {
    int n = r == e->S - 1 ? e->c.vocab_size - r * each : each;
    kd_copy(host + (size_t)r * each, gathered + (size_t)r * e->vmax, (size_t)n * sizeof(float));
  }
}

float *engine_forward(Model *model, int token, int position) {
  Engine *e = model->implementation;
  if (!e) {
    efail("engine_forward: no model loaded");
    return NULL;
  }
  if (token < 0 || token >= e->c.vocab_size || position < 0 || position >= e->c.seq_len) {
    efail("forward input out of range: token=%d position=%d", token, position);
    return NULL;
  }
  kc_clear_error();
  kernels_set_stream(e->stream);
  int *scalars = e->staging + e->max_batch; /* the previous call ended with a sync: no copy reads them any more */
  scalars[0] = token;
  scalars[1] = position;
  kd_copy(e->tokens_dev, &scalars[0], sizeof(int));
  kd_copy(e->pos_dev, &scalars[1], sizeof(int));
  if (run_step(e, &e->graph_logits, &e->graph_logits_kernels, decode_logits_step))
    return NULL;
  copy_logits_host(e, e->logits_host, e->logits_dev, e->gather_dev);
  if (kd_sync() || kc_status() || failed())
    return NULL;
  return e->logits_host;
}

/* Classifier over `rows` rows of the final residual starting at row r0, into dst (device, [rows][vl]). */
/* The batch's classifier, per row as the reference's forward_batch does it (src/tp.c:608-621): the final RMSNorm and
 * quantize of each row, then the decode GEMV (k_matmul_q8), so a row's logits are the ones a decode step at that
 * position would give from the same hidden state. */
static void classify_rows(Engine *e, int r0, int rows, float *dst) {
  const Config *p = &e->c;
  int dim = p->dim, gs = e->gs;
  k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x + (size_t)r0 * dim, dim, e->rms_final, rows, dim, p->norm_eps, gs);
  for (int r = 0; r < rows; r++) {
    K8Input in = {e->xq + (size_t)r * dim, e->xs + (size_t)r * (dim / gs), NULL};
    k_matmul_q8(dst + (size_t)r * e->vl, &in, k8(e->cls), dim, e->vl, gs);
  }
}

static void prefill_layers(Engine *e, int m, int pos0) {
  const Config *p = &e->c;
  int dim = p->dim, gs = e->gs;
  k_embed_q8_rows(e->x, e->tokens_dev, k8(e->embed), m, dim, gs, p->vocab_size);
  for (int l = 0; l < p->n_layers; l++) {
    Layer *y = &e->layers[l];
    float *kc = e->key_cache + (size_t)l * e->layer_kv, *vc = e->value_cache + (size_t)l * e->layer_kv;
    k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x, dim, y->rms_att, m, dim, p->norm_eps, gs);
    GemmQ8Segment qkv[3] = {{e->q, e->ql, k8(y->wq), {NULL, NULL}, NULL, NULL, e->ql, GEMM_STORE},
                            {e->k, e->kvl, k8(y->wk), {NULL, NULL}, NULL, NULL, e->kvl, GEMM_STORE},
                            {e->v, e->kvl, k8(y->wv), {NULL, NULL}, NULL, NULL, e->kvl, GEMM_STORE}};
    k_gemm_q8(e->xq, e->xs, m, dim, gs, qkv, 3);
    k_rope_kv_store_rows(e->q, e->ql, e->k, e->v, e->kvl, kc, vc, e->rope, NULL, pos0, m, e->hl, e->kl, e->hd,
                         e->context);
    k_attention_q8_rows(e->att, e->aq, e->as, e->q, kc, vc, &e->attn, e->hl, e->kl, e->hd, e->context, NULL, pos0, m,
                        gs);
    GemmQ8Segment wo = {e->S == 1 ? e->x : e->partial, dim, k8(y->wo), {NULL, NULL}, NULL, NULL, dim,
                        e->S == 1 ? GEMM_ADD : GEMM_PARTIAL};
    k_gemm_q8(e->aq, e->as, m, e->ql, gs, &wo, 1);
    if (e->S > 1)
      residual_reduce(e, m);
    k_rmsnorm_q8_rows(e->xq, e->xs, NULL, e->x, dim, y->rms_ffn, m, dim, p->norm_eps, gs);
    GemmQ8Segment up = {e->hb, e->hid_l, k8(y->w1), k8(y->w3), NULL, NULL, e->hid_l, GEMM_SWIGLU};
    k_gemm_q8(e->xq, e->xs, m, dim, gs, &up, 1);
    k_quantize_rows(e->hq, e->hs, e->hb, e->hid_l, m, e->hid_l, gs);
    GemmQ8Segment down = {e->S == 1 ? e->x : e->partial, dim, k8(y->w2), {NULL, NULL}, NULL, NULL, dim,
                          e->S == 1 ? GEMM_ADD : GEMM_PARTIAL};
    k_gemm_q8(e->hq, e->hs, m, e->hid_l, gs, &down, 1);
    if (e->S > 1)
      residual_reduce(e, m);
  }
}

static int prefill_validate(const Engine *e, const int *tokens, int count, int pos0, LogitsWanted want) {
  /* prefill_validate (src/prefill.c:72-83) */
  if (!tokens || count < 1 || count > e->max_batch || pos0 < 0 || pos0 >= e->c.seq_len ||
      count > e->c.seq_len - pos0)
    return efail("batch input out of range: count=%d position=%d maximum=%d", count, pos0, e->max_batch);
  if (want != LOGITS_NONE && want != LOGITS_LAST && want != LOGITS_ALL)
    return efail("invalid batch logits request: %d", (int)want);
  for (int i = 0; i < count; i++)
    if (tokens[i] < 0 || tokens[i] >= e->c.vocab_size)
      return efail("forward input out of range: token=%d position=%d", tokens[i], pos0 + i);
  return 0;
}

/* The batch through every layer; the last row's local logits in logits_dev when want is LAST (and for generate). */
static int prefill(Engine *e, const int *tokens, int count, int pos0, LogitsWanted want) {
  if (prefill_validate(e, tokens, count, pos0, want))
    return -1;
  kc_clear_error();
  kernels_set_stream(e->stream);
  if (kd_sync()) /* the previous chunk's upload may still be queued on the stream */
    return -1;
  if (e->w8a32) {
    /* W8A32 prefills one row per call (count == 1 == max_batch) through the decode step, as the reference runs it
     * per token; the step leaves that row's logits in logits_dev. Its own staging slots: engine_generate writes
     * staging[max_batch..+1] right after the last of these calls, while the copies below may still be queued. */
    int *scalars = e->staging + e->max_batch + 2;
    scalars[0] = tokens[0];
    scalars[1] = pos0;
    kd_copy(e->tokens_dev, &scalars[0], sizeof(int));
    kd_copy(e->pos_dev, &scalars[1], sizeof(int));
    return run_step(e, &e->graph_logits, &e->graph_logits_kernels, decode_logits_step) || failed() ? -1 : 0;
  }
  memcpy(e->staging, tokens, (size_t)count * sizeof(int));
  kd_copy(e->tokens_dev, e->staging, (size_t)count * sizeof(int));
  prefill_layers(e, count, pos0);
  if (want == LOGITS_LAST)
    classify_rows(e, count - 1, 1, e->logits_dev);
  return failed() ? -1 : 0;
}

float *engine_forward_batch(Model *model, const int *tokens, int count, int pos0, LogitsWanted want) {
  Engine *e = model->implementation;
  if (!e) {
    efail("engine_forward_batch: no model loaded");
    return NULL;
  }
  if (prefill(e, tokens, count, pos0, want))
    return NULL;
  float *result = NULL;
  if (want == LOGITS_LAST) {
    if (e->S > 1)
      kd_allgather_f32(e->comm, e->logits_dev, e->gather_dev, (size_t)e->vmax);
    copy_logits_host(e, e->logits_host, e->logits_dev, e->gather_dev);
    result = e->logits_host;
  } else if (want == LOGITS_ALL) {
    size_t V = (size_t)e->c.vocab_size;
    if (!e->batch_logits_host) {
      e->batch_logits_host = kd_host_alloc((size_t)e->max_batch * V * sizeof(float));
      e->batch_logits_dev = dev_alloc((size_t)e->max_batch * e->vmax * sizeof(float));
      if (!e->batch_logits_host || !e->batch_logits_dev)
        return NULL;
    }
    /* Per row as the reference (src/tp.c:608-621). */
    if (e->w8a32)  /* the one row's local logits, from the decode step */
      kd_copy(e->batch_logits_dev, e->logits_dev, (size_t)e->vl * sizeof(float));
    else
      classify_rows(e, 0, count, e->batch_logits_dev);
    for (int i = 0; i < count; i++) {
      const float *row = e->batch_logits_dev + (size_t)i * e->vl;
      if (e->S > 1) {
        kd_copy(e->logits_dev, row, (size_t)e->vl * sizeof(float));
        kd_allgather_f32(e->comm, e->logits_dev, e->gather_dev, (size_t)e->vmax);
      }
      copy_logits_host(e, e->batch_logits_host + (size_t)i * V, row, e->gather_dev);
    }
    result = e->batch_logits_host;
  }
  if (kd_sync() || kc_status() || failed())
    return NULL;
  return result;
}

int engine_generate(Model *model, const int *prompt, int count, int steps, int *out) {
  Engine *e = model->implementation;
  if (!e)
    return efail("engine_generate: no model loaded");
  if (count < 1 || steps < 1 || count > e->c.seq_len)
    return efail("engine_generate: prompt of %d tokens and %d steps do not fit the context of %d", count, steps,
                 e->c.seq_len);
  /* The probe stops printing at pos == seq_len: at most seq_len - count + 1 tokens, steps - 1 decode forwards. */
  if (steps > e->c.seq_len - count + 1)
    steps = e->c.seq_len - count + 1;
  if (e->gen_capacity < steps) {
    kd_free(e->gen_dev);
    e->gen_dev = dev_alloc((size_t)steps * sizeof(int));
    e->gen_capacity = e->gen_dev ? steps : 0;
    kd_graph_free(e->graph_greedy); /* it wrote the old buffer */
    e->graph_greedy = NULL;
    if (!e->gen_dev)
      return -1;
  }
  kernels_set_stream(e->stream);
  kd_event_record(e->ev[0]);
  for (int i = 0; i < count; i += e->max_batch) {
    int n = count - i < e->max_batch ? count - i : e->max_batch;
    if (prefill(e, prompt + i, n, i, i + n == count ? LOGITS_LAST : LOGITS_NONE))
      return -1;
  }
  /* The first token from the prompt's logits; then each decode step consumes the token it chose. */
  int *scalars = e->staging + e->max_batch;
  scalars[0] = count - 1;
  scalars[1] = 0;
  kd_copy(e->pos_dev, &scalars[0], sizeof(int));
  kd_copy(e->step_dev, &scalars[1], sizeof(int));
  k_argmax_key(e->key_dev, e->logits_dev, e->vl, e->v0);
  if (e->S > 1)
    kd_allreduce_max_u64(e->comm, e->key_dev, 1);
  k_greedy_advance(e->gen_dev, e->step_dev, e->tokens_dev, e->pos_dev, e->key_dev);
  kd_event_record(e->ev[1]);
  for (int i = 1; i < steps; i++)
    if (run_step(e, &e->graph_greedy, &e->graph_greedy_kernels, decode_greedy_step))
      return -1;
  kd_event_record(e->ev[2]);
  int *tokens = malloc((size_t)steps * sizeof(int));
  if (!tokens)
    return efail("engine_generate: out of host memory");
  if (kd_copy(tokens, e->gen_dev, (size_t)steps * sizeof(int)) || kd_sync() || kc_status() || failed()) {
    free(tokens);
    return -1;
  }
  e->stats.prefill_ms += kd_event_ms(e->ev[0], e->ev[1]);
  e->stats.decode_ms += kd_event_ms(e->ev[1], e->ev[2]);
  e->stats.prefill_tokens += count;
  e->stats.decode_tokens += steps - 1;
  int n = 0;
  for (; n < steps; n++) {
    out[n] = tokens[n];
    int t = tokens[n];
    if (t == e->c.eos_id || t == e->c.eot_id || t == e->c.eom_id) {
      n++;
      break;
    }
  }
  free(tokens);
  return n;
}

/* ---- misc ---------------------------------------------------------------------------------------------------------- */

int engine_max_batch(const Model *model) { return model->max_batch; }
const char *engine_precision(void) { return last_w8a32 ? "int8_q8_0_w8a32" : "int8_q8_0"; }
int engine_group_size(void) { return last_gs; }

void engine_stats(Model *model, EngineStats *out) {
  Engine *e = model->implementation;
  memset(out, 0, sizeof(*out));
  if (!e)
    return;
  *out = e->stats;
  out->kernel_launches = (long long)(kc_launch_count() - e->launches_base) - e->captured + e->replayed;
}

/* engine_kv_stats (include/runtime.h:111-113, tp_kv_stats src/tp.c:1147-1160): the K and V caches of every rank, as
 * the reference counts both sockets' caches. They are device memory allocated whole at load, so reserved and resident
 * are the same bytes; there is no host page placement to query (node -1, not verified), whatever `verify` asks. */
void engine_kv_stats(Model *model, int position, int verify, KvStats *out) {
  (void)verify;
  Engine *e = model ? model->implementation : NULL;
  if (!out)
    return;
  memset(out, 0, sizeof(*out));
  out->node = -1;
  if (!e) {
    efail("engine_kv_stats: no model loaded");
    return;
  }
  if (position < 0 || position > e->context) {
    efail("engine_kv_stats: position %d outside the context of %d", position, e->context);
    return;
  }
  size_t per_position = 2 * (size_t)e->c.n_layers * (size_t)e->kvl * sizeof(float) * (size_t)e->S;
  out->reserved_bytes = per_position * (size_t)e->context;
  out->active_bytes = per_position * (size_t)position;
  out->resident_bytes = out->reserved_bytes;
}

void engine_stats_reset(Model *model) {
  Engine *e = model->implementation;
  if (!e)
    return;
  memset(&e->stats, 0, sizeof(e->stats));
  e->launches_base = kc_launch_count();
  e->captured = e->replayed = 0;
}

/* The reduction that joins the Wo and W2 shards in a decode step, the same on every rank (agree_on_peer): "none" on
 * one GPU, "peer_gemv" when it runs inside the GEMV (kd_peer_matmul_q8_add), "peer_kernel" for the separate peer
 * all-reduce kernel, "nccl" for ncclAllReduce + add. The batched prefill always reduces with ncclAllReduce + add. */
const char *engine_reduction(Model *model) {
  Engine *e = model ? model->implementation : NULL;
  if (!e || e->S == 1)
    return "none";
  return e->peer ? (e->reduce_fused ? "peer_gemv" : "peer_kernel") : "nccl";
}

void *engine_stream(Model *model) {
  Engine *e = model->implementation;
  return e ? e->stream : NULL;
}

int engine_set_tp(int rank, int world, int device, const unsigned char *nccl_id) {
  if (world != 1 && world != 2 && world != 4 && world != 8)
    return efail("engine_set_tp: world size %d is not 1, 2, 4 or 8", world);
  if (rank < 0 || rank >= world)
    return efail("engine_set_tp: rank %d outside world %d", rank, world);
  if (world > 1 && !nccl_id)
    return efail("engine_set_tp: a world of %d needs the NCCL id", world);
  tp_request.rank = rank;
  tp_request.world = world;
  tp_request.device = device;
  if (nccl_id)
    memcpy(tp_request.id, nccl_id, KD_COMM_ID_BYTES);
  tp_request.set = 1;
  return 0;
}

static int write_q8(FILE *f, Q8 w, size_t rows, size_t cols, int gs) {
  size_t nq = rows * cols, ns = rows * (cols / gs);
  int8_t *q = malloc(nq);
  float *s = malloc(ns * sizeof(float));
  int ok = q && s && !kd_copy(q, w.q, nq) && !kd_copy(s, w.s, ns * sizeof(float)) && !kd_sync() &&
           fwrite(q, 1, nq, f) == nq && fwrite(s, sizeof(float), ns, f) == ns;
  free(q);
  free(s);
  return ok ? 0 : -1;
}

static int write_f32(FILE *f, const float *d, size_t n) {
  float *h = malloc(n * sizeof(float));
  int ok = h && !kd_copy(h, d, n * sizeof(float)) && !kd_sync() && fwrite(h, sizeof(float), n, f) == n;
  free(h);
  return ok ? 0 : -1;
}

int engine_save(Model *model, const char *path) {
  Engine *e = model->implementation;
  if (!e || e->S != 1)
    return efail("engine_save: needs a model loaded on one GPU");
  kernels_set_stream(e->stream);
  const Config *p = &e->c;
  FILE *f = fopen(path, "wb");
  if (!f)
    return efail("engine_save: cannot create '%s'", path);
  unsigned char h[256];
  memset(h, 0, sizeof(h));
  uint32_t magic = Q8_MAGIC;
  int version = 2, dims[7] = {p->dim, p->hidden_dim, p->n_layers, p->n_heads, p->n_kv_heads, p->vocab_size,
                              p->max_seq_len};
  memcpy(h, &magic, 4);
  memcpy(h + 4, &version, 4);
  memcpy(h + 8, dims, 28);
  h[36] = (unsigned char)p->shared;
  memcpy(h + 37, &e->gs, 4);
  int rc = fwrite(h, 1, 256, f) == 256 ? 0 : -1;
  size_t d = p->dim, hd = p->hidden_dim, kv = (size_t)p->head_dim * p->n_kv_heads, v = p->vocab_size;
  for (int l = 0; l < p->n_layers && !rc; l++)
    rc = write_f32(f, e->layers[l].rms_att, d);
  for (int l = 0; l < p->n_layers && !rc; l++)
    rc = write_f32(f, e->layers[l].rms_ffn, d);
  if (!rc)
    rc = write_f32(f, e->rms_final, d);
  if (!rc)
    rc = write_q8(f, e->embed, v, d, e->gs);
  for (int role = 0; role < 7 && !rc; role++)
    for (int l = 0; l < p->n_layers && !rc; l++) {
      Layer *y = &e->layers[l];
      Q8 w[7] = {y->wq, y->wk, y->wv, y->wo, y->w1, y->w2, y->w3};
      size_t rows[7] = {d, kv, kv, d, hd, d, hd}, cols[7] = {d, d, d, d, d, hd, d};
      rc = write_q8(f, w[role], rows[role], cols[role], e->gs);
    }
  if (!rc && !p->shared)
    rc = write_q8(f, e->cls, v, d, e->gs);
  if (fclose(f) || rc)
    return efail("engine_save: cannot write '%s'", path);
  return 0;
}

void engine_free(Model *model) {
  Engine *e = model->implementation;
  if (!e)
    return;
  kernels_set_stream(e->stream);
  kd_sync();
  kd_graph_free(e->graph_logits);
  kd_graph_free(e->graph_greedy);
  for (int i = 0; i < 3; i++)
    kd_event_free(e->ev[i]);
  if (e->layers)
    for (int l = 0; l < e->c.n_layers; l++) {
      Layer *y = &e->layers[l];
      kd_free(y->rms_att);
      kd_free(y->rms_ffn);
      q8_free(&y->wq);
      q8_free(&y->wk);
      q8_free(&y->wv);
      q8_free(&y->wo);
      q8_free(&y->w1);
      q8_free(&y->w2);
      q8_free(&y->w3);
    }
  free(e->layers);
  q8_free(&e->embed);
  if (e->cls_owned)
    q8_free(&e->cls);
  kd_free(e->rms_final);
  kd_free(e->key_cache);
  kd_free(e->value_cache);
  kd_free(e->rope);
  float *bufs[] = {e->x, e->q, e->k, e->v, e->att, e->hb, e->partial, e->xs, e->as, e->hs, e->logits_dev,
                   e->gather_dev, e->batch_logits_dev, e->xb};
  for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++)
    kd_free(bufs[i]);
  kd_free(e->xq);
  kd_free(e->aq);
  kd_free(e->hq);
  kd_free(e->tokens_dev);
  kd_free(e->pos_dev);
  kd_free(e->step_dev);
  kd_free(e->gen_dev);
  kd_free(e->key_dev);
  k_attention_free(&e->attn);
  kd_host_free(e->logits_host);
  kd_host_free(e->batch_logits_host);
  kd_host_free(e->staging);
  kd_peer_free(e->peer);
  kd_comm_free(e->comm);
  kernels_set_stream(NULL);
  kd_stream_free(e->stream);
  free(e);
  model->implementation = NULL;
}
