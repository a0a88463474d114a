// Tensor-core convolution (implicit GEMM on tcgen05, 3xTF32) fused with ReLU
// and a 2x2 pool: parameter block, weight packing and launcher.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace rosenna {

// B images (floats) of the two MMA forms: per tap, 3 K-chunks x (hi, lo) x
// [16 x 32]; per window, 4 K-chunks x (hi, lo) x [64 x 32].
constexpr int kConvTcBFloatsTap = 3 * 2 * 16 * 32;
constexpr int kConvTcBFloats = 4 * 2 * 64 * 32;

struct ConvTcArgs {
    const float *arena;
    long long bt_off, b_off;  // arena offsets: the B image of `mode`, bias[OC]
    const float *in;          // input element (c, y, x) at row c + C*(y + Hin*x)
    long long ld_in;
    float *out;               // output (oc, qy, qx) at row oc*so_c + qy*so_h + qx*so_w
    long long ld_out, so_c, so_h, so_w;
    long long n;
    int *err;                 // [64] status word shared with the other tensor-core kernels
    int C, Hin, Win, pad, OC, Hq, Wq, pool, relu;  // pool: 1 max, 2 avg (k = s = 2)
    int mode;                 // 0: per tap (N = 16), 1: per window (N = 64)
};

// Whether a conv(+ReLU)+pool step has the shapes conv_tc_kernel covers.
bool conv_tc_shape_ok(int KS, int str_h, int str_w, int pad_h, int pad_w, int C, int OC, int pool, int pk, int pstr_h,
                      int pstr_w, int ppad_h, int ppad_w, int Ho, int Wo);
// Packs 3x3 weights w[oc][ic][kh][kw] (OC <= 16, C <= 8) into the B image of
// `mode` (kConvTcBFloatsTap or kConvTcBFloats floats): tf32 hi and lo parts in
// the 128-byte-swizzled K-major layout the kernel copies to shared memory.
void conv_tc_pack(const float *w, int OC, int C, int mode, float *img);
cudaError_t conv_tc_configure();
cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st);

}  // namespace rosenna
