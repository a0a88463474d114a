/* A C solver calling the engine the way examples/cAPI.c calls roseNNa, with a
 * batch: build with
 *   gcc solver.c -I<repo>/include -L<repo>/rosenna_b200 -lrosenna_b200 -Wl,-rpath,<repo>/rosenna_b200
 * and run it in a directory holding onnxModel.txt, onnxWeights.txt and
 * variables.fpp of a one-input, one-output model.  Prints the status and the
 * outputs of the first sample (all inputs 1, as torch.ones in goldenFiles). */
#include <stdio.h>
#include <stdlib.h>

#include "rosenna.h"

int main(int argc, char **argv) {
    long long n = argc > 1 ? atoll(argv[1]) : 4;
    int rc = rosenna_initialize();
    if (rc) {
        printf("initialize: status %d (%s)\n", rc, rosenna_last_error());
        return 0;
    }
    int64_t dims[8];
    int bdim = 0;
    int r = rosenna_input_shape(0, dims, 8, &bdim);
    long long in_rows = 1, out_rows = 1;
    for (int k = 0; k < r; k++)
        if (k != bdim) in_rows *= dims[k];
    r = rosenna_output_shape(0, dims, 8, &bdim);
    for (int k = 0; k < r; k++)
        if (k != bdim) out_rows *= dims[k];
    float *x = malloc(sizeof(float) * in_rows * n), *y = malloc(sizeof(float) * out_rows * n);
    for (long long i = 0; i < in_rows * n; i++) x[i] = 1.0f; /* like torch.ones in goldenFiles */
    const float *ins[1] = {x};
    float *outs[1] = {y};
    rc = rosenna_use_model_f32(n, ins, outs);
    printf("use_model: status %d launches %lld\n", rc, (long long)rosenna_last_launch_count());
    for (long long i = 0; i < out_rows && !rc; i++) printf("%.9g ", y[i * n]);
    printf("\n");
    free(x);
    free(y);
    return rc;
}
