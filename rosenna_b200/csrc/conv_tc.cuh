// Tensor-core convolution (implicit GEMM on tcgen05, 3xTF32) fused with ReLU
// and a 2x2 pool: parameter block, weight packing and launcher.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace rosenna {

// The B image (floats): up to 4 K-chunks, each tf32 hi then lo parts of
// [64 rows x 32] (rows = pixel*OCp + oc over the block's patch).
constexpr int kConvTcBChunk = 2 * 64 * 32;
constexpr int kConvTcBFloats = 4 * kConvTcBChunk;

// How a conv maps onto the kernel: channels per patch position in K (8, or 1
// for a single-channel input), pooled windows per block (1 with 16 output
// channels, 2 with 8), 32-wide K-chunks per block.
struct ConvTcGeom {
    int cp, bwin, nch;
};
ConvTcGeom conv_tc_geometry(int C, int OC);

struct ConvTcArgs {
    const float *arena;
    long long bt_off, b_off;  // arena offsets: the B image, bias[OC]
    const float *in;          // input element (c, y, x) at row c + C*(y + Hin*x)
    long long ld_in;
    float *out;               // output (oc, qy, qx) at row oc*so_c + qy*so_h + qx*so_w
    long long ld_out, so_c, so_h, so_w;
    long long n;
    int *err;                 // [64] status word shared with the other tensor-core kernels
    int C, Hin, Win, pad, OC, Hq, Wq, pool, relu;  // pool: 1 max, 2 avg (k = s = 2)
    int cp, bwin, nch;        // conv_tc_geometry(C, OC)
};

// Whether a conv(+ReLU)+pool step has the shapes conv_tc_kernel covers.
bool conv_tc_shape_ok(int KS, int str_h, int str_w, int pad_h, int pad_w, int C, int OC, int pool, int pk, int pstr_h,
                      int pstr_w, int ppad_h, int ppad_w, int Ho, int Wo);
// Packs 3x3 weights w[oc][ic][kh][kw] (OC <= 16, C <= 8) into the B image
// (kConvTcBFloats floats): the weights laid out over the block's patch, tf32 hi
// and lo parts, in the 128-byte-swizzled K-major layout the kernel copies to
// shared memory.
void conv_tc_pack(const float *w, int OC, int C, float *img);
cudaError_t conv_tc_configure();
cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st);

}  // namespace rosenna
