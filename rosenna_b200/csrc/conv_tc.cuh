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
    int group;  // sample tiles that take each block in turn (1..64): the unit order
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

// conv_pair_tc_kernel: a conv(+ReLU)+pool step and the conv(+ReLU)+pool step
// that is the only reader of its output, in one kernel; the first conv's
// pooled output passes through `mid`, two 128-sample columns per CTA (element
// (c, y, x) of column s at mid[(c + C2*(y + Hin2*x))*mid_cols + s]).
struct ConvPairArgs {
    CUtensorMap map1;   // first conv's input, box {128, cb1, ph1, cw1}
    CUtensorMap omap1;  // mid as the first conv's pooled output, box {128, ocp1, bh1 / 2, 2}
    CUtensorMap map2;   // mid as the second conv's input, box {128, cb2, ph2, cw2}
    CUtensorMap omap2;  // the second conv's pooled output, box {128, ocp2, bh2 / 2, 2}
    const float *arena;
    long long s1_off, b1_off, s2_off, b2_off;  // arena offsets: packed first image, bias, second image, bias
    long long n;
    int *err;
    int OC1, Wo1, pad1, relu1, bh1;
    int OC2, Hin2, Wo2, pad2, relu2, bh2, ph2, nb2;
    int slots;
};
// Whether the two steps' shapes have a conv_pair_tc_kernel instantiation
// (first: 1 input channel, <= 8 outputs; second: 5..8 inputs, 9..16 outputs).
bool conv_pair_shape_ok(int C1, int OC1, int pool1, int C2, int OC2, int pool2);
// Packs a first conv's 3x3 weights with each row's tf32 lo part beside its hi
// part (kConvTcBFloats / 2 floats); C <= 2.
void conv_pair_pack1(const float *w, int OC, int C, float *img);
// Samples per mid column group: mid holds 256 columns per CTA.
constexpr int kConvPairMidPerCta = 256;
cudaError_t conv_pair_configure();
// a1/a2: the two steps as launch_conv_tc would take them (maps encoded, a1's
// out unused); mid/mid_cols: the per-CTA buffer (grid = mid_cols / 256 at most).
cudaError_t launch_conv_pair(const ConvTcArgs &a1, long long s1_off, const ConvTcArgs &a2, float *mid,
                             long long mid_cols, int num_sms, cudaStream_t st, const char **why);

}  // namespace rosenna
