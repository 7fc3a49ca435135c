/* TEST INFRASTRUCTURE: the five symbols the reference's src/runtime.c needs besides what tests/probe.c uses, for
 * linking the reference's own probe driver (tests/probe.c + src/runtime.c + src/tokenizer.c + src/sampler.c) against
 * the GPU engine (libllama3x_engine.so) instead of the reference's engine. The reference's kernels, workers and shard
 * files are deliberately not linked: their kernels_init / k_* definitions would interpose on the GPU library's.
 *
 * workers_abort / workers_aborted (include/workers.h:112-113): fail() releases the CPU worker pool's waits; the GPU
 * engine has no pool. The other three belong to reference functions the probe never reaches (checkpoint_map,
 * apply_rope, the CPU softmax); calling one is a build mistake, reported as such. */
#include <stdio.h>
#include <stdlib.h>

#include "runtime.h"
#include "shards.h"
#include "workers.h"

void workers_abort(void) {}

int workers_aborted(void) { return 0; }

static _Noreturn void unreachable(const char *what) {
  fprintf(stderr, "probe-gpu: %s is not part of the GPU engine's drop-in\n", what);
  abort();
}

void manifest_build(TensorManifest *m, const Config *p, int quantized, int gs, size_t header_bytes) {
  (void)m, (void)p, (void)quantized, (void)gs, (void)header_bytes;
  unreachable("manifest_build");
}

float rope_frequency(const Config *p, int j) {
  (void)p, (void)j;
  unreachable("rope_frequency");
}

void softmax(float *x, int size) {
  (void)x, (void)size;
  unreachable("softmax");
}
