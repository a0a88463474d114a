// conv_tc_kernel (conv_tc.cu): a 3x3 stride-1 convolution fused with its ReLU
// and a 2x2 pool: parameter block, weight packing and launcher.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace rosenna {

// The weight image (floats): the sliding-window weight matrix, 288 rows x 32
// K-slots, tf32 hi part then lo part, each in the 128-byte-swizzled K-major
// layout the kernel copies to shared memory as it is.
constexpr int kConvTcRows = 288;
constexpr int kConvTcBFloats = 2 * kConvTcRows * 32;

// How a conv maps onto the kernel.  A block is bh x 4 conv pixels (rows y x
// columns x) times ocp output channels = 128 GEMM columns; its input patch is
// (bh + 2) x 6 positions, loaded as ph rows (>= bh + 2) of cb channels (C
// rounded up to 1, 2, 4 or 8; the extra channels read as zeros) per column,
// cw columns per chunk: rows = cb * ph * cw K-rows (<= 32) per chunk, 6 / cw
// chunks per block.  `slots` chunks are in flight in shared memory.
struct ConvTcGeom {
    int ocp, bh, cb, ph, cw, rows, slots;
    bool ok;
};
ConvTcGeom conv_tc_geometry(int C, int OC);

struct ConvTcArgs {
    CUtensorMap map;          // the input as {samples, cb of C channels, Hin, Win}, box {128, cb, ph, cw}
    CUtensorMap omap;         // the output as {samples, OC, Hq, Wq}, box {128, ocp, bh / 2, 2}
    const float *arena;
    long long bt_off, b_off;  // arena offsets: the weight image, bias[OC]
    float *out;               // output (oc, qy, qx) at row oc*so_c + qy*so_h + qx*so_w
    long long ld_out, so_c, so_h, so_w;
    long long n;
    int *err;                 // [64] status word shared with the other tensor-core kernels
    int C, Hin, Win, pad, OC, Ho, Wo, Hq, Wq, pool, relu;  // pool: 1 max, 2 avg (k = s = 2)
    int ocp, bh, cb, ph, cw, rows, slots;                  // conv_tc_geometry(C, OC)
};

// Whether a conv(+ReLU)+pool step has the shapes conv_tc_kernel covers.
bool conv_tc_shape_ok(int KS, int str_h, int str_w, int pad_h, int pad_w, int C, int OC, int pool, int pk, int pstr_h,
                      int pstr_w, int ppad_h, int ppad_w, int Ho, int Wo);
// Packs 3x3 weights w[oc][ic][kh][kw] (OC <= 16, C <= 8) into the weight image
// (kConvTcBFloats floats).
void conv_tc_pack(const float *w, int OC, int C, float *img);
// Whether an input or output array can be reached by the kernel's tensor maps
// (16-byte aligned base and sample pitch).
bool conv_tc_input_ok(const float *in, long long ld_in);
// Encodes a.map for the input `in` (element (c, y, x) of sample s at
// in[(c + C*(y + Hin*x))*ld_in + s]) from the geometry fields of `a`.
bool conv_tc_encode_input(ConvTcArgs &a, const float *in, long long ld_in, const char **why);
// Encodes a.omap for a.out (output (oc, qy, qx) of sample s at
// out[(oc*so_c + qy*so_h + qx*so_w)*ld_out + s]) from the fields of `a`.
bool conv_tc_encode_output(ConvTcArgs &a, const char **why);
cudaError_t conv_tc_configure();
cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st);

}  // namespace rosenna
