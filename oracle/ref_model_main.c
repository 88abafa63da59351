/*
 * ref_model_main.c — TEST INFRASTRUCTURE ONLY (the model-level checker and
 * the CPU baseline). Driver for a model that nnc-py's own x86 backend
 * generated (model.c / tensors.c / constants_loader.c linked with the
 * reference's runtime/x86/ops.c, all compiled from source by
 * oracle/ref_models.py into oracle/_ref/).
 *
 *   ./model_x86 constants.bin input.bin output.bin [reps] [first] [count]
 *
 * input.bin holds batch-sized samples of the compiled model; samples
 * [first, first + count) are run one compiled batch at a time (count is a
 * multiple of the compiled batch), so a batch-1 model reproduces nnc-py's
 * benchmark definition of "workload batch N = N sequential nnc_run()"
 * (benchmarks/runner_gen.py). The forward is repeated `reps` times and the
 * best wall time per compiled batch is printed as "seconds_per_run=<s>".
 * MODEL_INPUT / MODEL_OUTPUT name the generated input / output tensors.
 */
#define _POSIX_C_SOURCE 199309L
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "model.h"
#include "nnc_types.h"

extern Tensor MODEL_INPUT;
extern Tensor MODEL_OUTPUT;
#ifdef NNC_DEBUG_DUMP
/* nnc-py's x86 debug builds print every intermediate tensor through this
 * stream (declared extern in their model.c); NULL selects stdout. */
FILE* debug_file = NULL;
#endif
int nnc_load_constants(const char* path);

static double now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

int main(int argc, char** argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: %s constants.bin input.bin output.bin [reps] [first] [count]\n", argv[0]);
        return 2;
    }
    const int reps = argc > 4 ? atoi(argv[4]) : 1;
    const long first = argc > 5 ? atol(argv[5]) : 0;
    const size_t in_b = (size_t)MODEL_INPUT.nbytes, out_b = (size_t)MODEL_OUTPUT.nbytes;
    FILE* f = fopen(argv[2], "rb");
    if (!f) return 1;
    fseek(f, 0, SEEK_END);
    const long total = ftell(f) / (long)in_b;
    const long count = argc > 6 ? atol(argv[6]) : total - first;
    if (first < 0 || count <= 0 || first + count > total) {
        fprintf(stderr, "input holds %ld batches, asked for [%ld, %ld)\n", total, first, first + count);
        return 2;
    }
    if (nnc_load_constants(argv[1]) != 0) return 1;
    FILE* o = fopen(argv[3], "wb");
    if (!o) return 1;
    double best = 1e30;
    for (long b = first; b < first + count; ++b) {
        fseek(f, b * (long)in_b, SEEK_SET);
        if (fread(MODEL_INPUT.data, 1, in_b, f) != in_b) return 1;
        for (int r = 0; r < reps; ++r) {
            const double t0 = now();
            nnc_run();
            const double t = now() - t0;
            if (t < best) best = t;
        }
        if (fwrite(MODEL_OUTPUT.data, 1, out_b, o) != out_b) return 1;
    }
    fclose(o);
    fclose(f);
    printf("seconds_per_run=%.6f\n", best);
    return 0;
}
