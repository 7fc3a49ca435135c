/* TEST INFRASTRUCTURE: the two symbols the reference's CLI (src/app.c, its runq/run front end) needs beyond what
 * tests/probe.c needs, for linking that CLI unchanged against the GPU engine (libllama3x_engine.so) instead of the
 * reference's engine (oracle/Makefile, target runq-gpu). Together with probe_gpu_stubs.c.
 *
 * write_report (include/app.h:13, src/report.c:251): the --json run report describes the CPU run (NUMA topology,
 * worker teams, page placement of host regions), none of which exists on the GPU path, so no report is written; the
 * generated text and LLAMA_TOKENS_OUT are unaffected. placement_active (include/loader.h:44): where the weights live,
 * for the CLI's start-up log line: in device memory. */
#include "app.h"
#include "loader.h"

void write_report(void) {}

const char *placement_active(void) { return "device"; }
