/* The GPU engine: the reference's engine API (include/runtime.h:98-116) over device-resident Q8_0 weights, a device
 * K/V cache and the sm_100a kernels, with tensor parallelism over 1/2/4/8 GPUs (one process per GPU, NCCL).
 *
 * A program written against the reference's engine (runq's engine.c: tests/probe.c, src/app.c) links against
 * libllama3x_engine.so instead and runs unchanged: same names, same Config/Model layout, same contracts -- logits
 * belong to the model and are invalidated by the next forward; invalid arguments fail() (kc_set_fail_mode selects
 * exit, the reference's behaviour, or return NULL / -1 with kc_last_error set). The checkpoint is the reference's
 * Q8_0 format, version 2 or 3 (src/runtime.c:179-310, tensor order src/shards.c:80-97).
 *
 * Environment, as in the reference: LLAMA_PREFILL_BATCH (rows per engine_forward_batch call; default 2048 here),
 * LLAMA_PREFILL_LOGITS=last|all. Added: LLAMA_CUDA_GRAPHS=0 runs the decode step eagerly instead of as a CUDA graph. */
#ifndef LLAMA3X_ENGINE_CUDA_H
#define LLAMA3X_ENGINE_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef LLAMA_RUNTIME_H
/* Layout-compatible with the reference's Config, LogitsWanted and Model (include/runtime.h:9-17, 73, 86-97). */
typedef struct {
  int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
  int format, max_seq_len, shared, head_dim;
  float norm_eps, rope_theta, rope_factor, rope_low, rope_high;
  int rope_type, rope_original;
  int bos_id, eos_id, eot_id, eom_id;
  char name[128];
} Config;

typedef enum { LOGITS_NONE, LOGITS_LAST, LOGITS_ALL } LogitsWanted;

/* include/runtime.h:76-85 */
typedef struct {
  size_t reserved_bytes, active_bytes, resident_bytes;
  int node;
  int verified;
  int full;
  size_t pages_queried, pages_wrong_node, pages_missing;
} KvStats;

typedef struct {
  Config config;
  void *implementation;
  size_t file_bytes;
  size_t mapped_bytes;
  int max_batch;
  LogitsWanted prefill_logits;
  int prefill_gemm;
  const char *prefill_kernel;
  int prefill_bf16;
} Model;
#endif

/* ---- the reference's engine API (include/runtime.h:98-116) ------------------------------------------------------- */
extern const int engine_q8; /* 1: this engine reads Q8_0 checkpoints */
void engine_load(Model *model, const char *path);
void engine_load_context(Model *model, const char *path, int context);
float *engine_forward(Model *model, int token, int position);
float *engine_forward_batch(Model *model, const int *tokens, int count, int pos0, LogitsWanted want);
int engine_max_batch(const Model *model);
/* KV cache accounting (include/runtime.h:111-113): reserved and active bytes of the K and V caches of all ranks for
 * positions [0, position). The caches are device memory allocated whole at load: resident equals reserved, node is -1
 * and nothing is verified, as there is no host page placement to query. */
void engine_kv_stats(Model *model, int position, int verify, KvStats *out);
void engine_free(Model *model);
const char *engine_precision(void);
int engine_group_size(void);
/* One position's RoPE table (include/kernels.h:67, src/kernels_simd.c:194-201): 2 * head_dim floats, cosines
 * duplicated per pair, then (-sin, +sin) per pair, with rope_frequency's Llama 3.1 scaling (src/kernels.c:49-60). A
 * host function: it lives in the engine library because it takes the engine's Config. */
void k_rope_table(const Config *p, int position, float *table);

/* ---- GPU additions (no counterpart in the reference) ------------------------------------------------------------- */
/* Tensor parallelism, set before loading: this process is `rank` of `world` (1, 2, 4 or 8) on CUDA device `device`,
 * joined through the NCCL unique id rank 0 made with kd_comm_unique_id (include/device_cuda.h). Shards as the
 * reference's two-socket plan (src/shards.c:190-272) generalised: wq/wk/wv/w1/w3 and the classifier by output rows,
 * wo/w2 by input columns, KV heads n_kv_heads / world per rank. Default: rank 0 of 1 on the current device. */
int engine_set_tp(int rank, int world, int device, const unsigned char *nccl_id);
/* A device-resident random-init model of `config` (the seven dimensions; v2 defaults for the rest): Q8_0 weights
 * drawn N(0, 0.02) by k_random_q8 from `seed`, RMSNorm weights 1, classifier tied when config->shared. Sharded like a
 * loaded checkpoint, and every rank holds exactly its slice of the same model. */
void engine_init_random(Model *model, const Config *config, int group_size, unsigned long long seed, int context);
/* Greedy generation on the device (probe-int8 `generate`, tests/probe.c:110-141): the prompt goes through
 * engine_forward_batch in engine_max_batch chunks, then up to `steps` tokens are chosen by argmax, the first from the
 * prompt's last logits and each next one after a decode step (a CUDA graph replayed with the position and token in
 * device memory, so no host round trip per token). Stops after an EOS/EOT/EOM token or at the end of the context, as
 * the probe does. Writes the tokens to `out` and returns how many, or -1. */
int engine_generate(Model *model, const int *prompt, int count, int steps, int *out);
/* Writes a seeded random-init model of `config`'s architecture (the seven dimensions and `shared`) as a version 2
 * Q8_0 checkpoint both engines load: N(0, 0.02) weights from a counter-based generator (SplitMix64 finalizer,
 * Box-Muller) quantized in group_size groups by k_quantize's rule, RMSNorm weights 1, on every online core. The
 * benchmark's models: the same bytes for the GPU engine and the reference's. Returns 0, or -1 with the fail() policy. */
int engine_write_random(const char *path, const Config *config, int group_size, unsigned long long seed);
/* Writes the model (this rank's copy; world 1 only) as a version 2 Q8_0 checkpoint the reference loads. */
int engine_save(Model *model, const char *path);
/* The decode step's Wo/W2 reduction, agreed by every rank: "none" (one GPU), "peer_gemv" (inside the GEMV over NVLink
 * peer memory), "peer_kernel" (a separate peer all-reduce kernel) or "nccl" (ncclAllReduce + add). */
const char *engine_reduction(Model *model);
/* The engine's CUDA stream (cudaStream_t), for timing with events on it. */
void *engine_stream(Model *model);
/* What engine_generate did since the model was set up or engine_stats_reset: device time of its prefill (the prompt
 * through the last chunk's classifier and the first argmax) and of its decode steps (CUDA events on the engine's
 * stream), the positions each processed, and the kernels of this library it launched (CUDA-graph replays included). */
typedef struct {
  double prefill_ms, decode_ms;
  long long prefill_tokens, decode_tokens;
  long long kernel_launches;
} EngineStats;
void engine_stats(Model *model, EngineStats *out);
void engine_stats_reset(Model *model);

#ifdef __cplusplus
}
#endif

#endif
