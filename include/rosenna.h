/*
 * rosenna.h -- C ABI of the B200 batched inference engine behind roseNNa's API.
 *
 * roseNNa's boundary is two bind(c) Fortran symbols:
 *   subroutine initialize() bind(c,name="initialize")          fLibrary/reader.f90:38
 *   SUBROUTINE use_model(i0,..,o0,..) bind(c,name="use_model")  fLibrary/modelCreator.fpp:42
 * which a C solver declares as (examples/cAPI.c:3-4, README.md "C use"):
 *   void use_model(double *i0, double *o0);
 *   void initialize(char *model_file, char *weights_file);
 *
 * This library keeps `initialize` and adds batched entry points.  All arrays use
 * the reference layout: the Fortran (column-major) array of the ONNX shape, with
 * the export batch widened to n.  For every shape roseNNa's golden cases use, the
 * batch index is then the fastest-varying index in memory.
 *
 * Model files: onnxModel.txt, onnxWeights.txt and variables.fpp, as written by
 * fLibrary/modelParserONNX.py (or rosenna_b200.writer).  variables.fpp replaces
 * the fypp expansion of modelCreator.fpp: the engine builds its launch plan from
 * its `architecture` list at initialize time.
 *
 * Threading: one call at a time per process (the reference keeps module
 * globals too).  Every entry point returns a status; none aborts.
 */
#ifndef ROSENNA_H
#define ROSENNA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ROSENNA_OK = 0,
    ROSENNA_ERR_IO = 1,          /* a model file cannot be opened or read */
    ROSENNA_ERR_FORMAT = 2,      /* a model file is malformed */
    ROSENNA_ERR_UNSUPPORTED = 3, /* an op or shape the engine does not run */
    ROSENNA_ERR_SHAPE = 4,       /* arguments do not match the model */
    ROSENNA_ERR_CUDA = 5,        /* a CUDA call failed */
    ROSENNA_ERR_NO_DEVICE = 6,   /* no usable GPU */
    ROSENNA_ERR_STATE = 7,       /* not initialized */
    ROSENNA_ERR_ARG = 8          /* null pointer or negative size */
};

/* Replaces reader.f90:38 initialize(): reads ./onnxModel.txt, ./onnxWeights.txt
 * and ./variables.fpp, builds the launch plan and uploads the weights once to
 * every selected GPU.  Extra arguments passed by C callers that declare
 * initialize(char*, char*) (examples/cAPI.c:4) are ignored, as in the reference.
 * The status is kept for rosenna_last_status()/rosenna_last_error(). */
void initialize(void);

/* initialize() with a status. */
int rosenna_initialize(void);

/* initialize() from explicit paths (variables_fpp may be NULL: then the file
 * variables.fpp beside model_txt is used). */
int rosenna_initialize_from(const char *model_txt, const char *weights_txt, const char *variables_fpp);

/* Reads the model files and builds the launch plan without touching a GPU
 * (variables_fpp may be NULL as above).  The plan is then available from
 * rosenna_plan_description(); initialize state is unchanged. */
int rosenna_check_model(const char *model_txt, const char *weights_txt, const char *variables_fpp);

/* Frees the device weights, buffers, streams and the plan. */
int rosenna_finalize(void);

/* Selects the GPUs that initialize() uploads to and use_model splits over
 * (default: every visible GPU).  Call before initialize. */
int rosenna_set_devices(const int *device_ids, int count);

int rosenna_last_status(void);
const char *rosenna_last_error(void);

/* Model interface, from variables.fpp: trueInputs and outShape (export shapes).
 * *batch_dim receives the index of the batch dimension in that shape. */
int rosenna_num_inputs(void);
int rosenna_num_outputs(void);
int rosenna_input_shape(int i, int64_t *dims, int max_dims, int *batch_dim);
int rosenna_output_shape(int i, int64_t *dims, int max_dims, int *batch_dim);

/* Batched use_model on host arrays (replaces modelCreator.fpp:42 use_model).
 * inputs[i] / outputs[i] hold the export shape with its batch dimension widened
 * to n, Fortran order.  Samples are split contiguously over the selected GPUs;
 * copies are chunked and overlapped with the kernels. */
int rosenna_use_model_f32(int64_t n, const float *const *inputs, float *const *outputs);

/* The same for fp64 host arrays (converted to fp32 on the host). */
int rosenna_use_model_f64(int64_t n, const double *const *inputs, double *const *outputs);

#ifndef ROSENNA_NO_LEGACY_USE_MODEL
/* Replaces modelCreator.fpp:42 use_model(i0,..,o0,..) for fixed-shape callers,
 * which declare it with their model's own argument count (examples/cAPI.c:3:
 * void use_model(double *i0, double *o0)): fp64 arrays of the export shapes,
 * the model's inputs then its outputs, evaluated at the export batch.  Declared
 * here with the largest count the engine accepts (16 arrays); only the model's
 * count is read.  A file that declares its own prototype defines
 * ROSENNA_NO_LEGACY_USE_MODEL before including this header.  The status is kept
 * for rosenna_last_status()/rosenna_last_error(); the reference aborts instead. */
void use_model(double *a0, double *a1, double *a2, double *a3, double *a4, double *a5, double *a6, double *a7, double *a8, double *a9, double *a10, double *a11, double *a12, double *a13, double *a14, double *a15);
#endif

/* Batched use_model on device arrays, on `stream` (a cudaStream_t; NULL = the
 * default stream).  The arrays live on the selected GPU when one is selected,
 * else on the current device.
 * Asynchronous with respect to the host: inputs must stay valid until the
 * stream reaches this work. */
int rosenna_use_model_device_f32(int64_t n, const float *const *inputs, float *const *outputs, void *stream);

/* Allocation-free variant of rosenna_use_model_device_f32.  It has no
 * counterpart in roseNNa.  For callers that cannot let the library allocate
 * device memory during the call: a solver whose own pool allocator holds all
 * free GPU memory, or a time-step loop that cannot absorb the device-wide
 * synchronisation of cudaMalloc/cudaFree.  The plan's intermediate buffers come
 * from one fixed 64 MiB array in device memory that every GPU loading this
 * library holds until exit; n is rejected (ROSENNA_ERR_SHAPE, with the limit in
 * rosenna_last_error()) when the intermediates for n samples do not fit.  The
 * array's address is looked up in initialize(), once per selected GPU with that
 * GPU current (set-up); with lazy module loading that is also when the array is
 * created, so the calls themselves allocate nothing.  All calls share the array and it keeps
 * the last call's contents (no intermediate needs clearing: each is written
 * before it is read), so calls whose work overlaps on the GPU race: order them
 * on one stream.  Arguments and layout as for rosenna_use_model_device_f32. */
int rosenna_use_model_device_noalloc_f32(int64_t n, const float *const *inputs, float *const *outputs, void *stream);

/* Per-step device timing, for benchmarks (no counterpart in roseNNa, whose
 * generated use_model takes CPU_TIME around its body and discards it,
 * fLibrary/modelCreator.fpp:77,168).  After rosenna_step_timing_begin(m), the
 * next use_model calls record a CUDA event pair around every plan step on the
 * stream the step runs on, for up to m steps in total (per GPU).
 * rosenna_step_timing_end waits for those events, writes the summed
 * milliseconds of plan step i to ms[i] and the number of times it ran to
 * runs[i] (i < max_steps), and stops recording. */
int rosenna_step_timing_begin(int64_t max_records);
int rosenna_step_timing_end(double *ms, int64_t *runs, int max_steps);

/* Number of steps of the launch plan, and for step i the kernel that runs it
 * and its algorithmic flops per sample (2 x the multiply-adds of its Gemm, LSTM
 * gate and convolution contractions; 0 for data-movement steps). */
int rosenna_step_count(void);
int rosenna_step_info(int i, char *kernel, int kernel_len, double *flops_per_sample);

/* Number of kernel launches the last use_model call issued (all devices). */
int64_t rosenna_last_launch_count(void);

/* Human-readable launch plan (one line per step), for logs and tests. */
const char *rosenna_plan_description(void);

#ifdef __cplusplus
}
#endif

#endif /* ROSENNA_H */
