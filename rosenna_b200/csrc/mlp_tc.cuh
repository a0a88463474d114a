// Tensor-core (tcgen05, 3xTF32) fused MLP: parameter block and launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace rosenna {

constexpr int kTcMaxLayers = 8;
constexpr int kTcTailMaxN = 16;  // widest last layer run as the CUDA-core tail

// One layer; its packed weights are a [2*Np][Kp] fp32 block (rows 0..Np-1 the
// tf32-rounded high parts W_hi[n][k], rows Np..2Np-1 the rounded remainders).
struct TcLayer {
    int K, N, Kp, Np, nch, act;  // Kp = 32*nch, Np multiple of 16 (<= 256)
    long long w_off, b_off;      // arena offsets (floats): weight block, bias[Np]
};

struct TcArgs {
    CUtensorMap maps[kTcMaxLayers];  // one TMA map per layer over its weight block, box {32, Np}
    const float *arena;
    const float *in;
    long long ld_in;
    float *out;
    long long ld_out;
    long long n;
    int *err;  // [64]: err[0] = non-zero code when a wait times out, err[1..6] where, err[8r..] per role
    int nlayers;  // layers on the tensor cores
    TcLayer L[kTcMaxLayers];
    // A narrow last layer (N <= 16) runs on the CUDA cores after them when
    // tail_n > 0: fp32 W^T [tail_kp][tail_np] at arena offset tail_w_off (the
    // FFMA kernel's layout), bias [tail_np] at tail_b_off.
    int tail_n, tail_np, tail_k, tail_kp, tail_act;
    long long tail_w_off, tail_b_off;
    // every layer's Np <= 128: run mlp_tc_dual_kernel (each column group its
    // own tile) instead of splitting one tile's columns between the groups
    int dual;
    // every layer at most 64 wide with at most 64 inputs and the weights fit in
    // shared memory: run mlp_narrow_tc_kernel (resident weights, A in TMEM)
    int narrow;
    // the same with a first layer of more than 64 inputs: mlp_stream_tc_kernel
    // (that layer's inputs and weights streamed by TMA; xmap set by its launcher)
    int stream;
    CUtensorMap xmap;
};

// One LSTM layer (fLibrary/layers.f90 lstm / lstm_cell) on the tensor cores,
// for 4H <= 256: every time step is a 128-sample x (4H gates) x (Ix + Hh)
// product of [x_t | h_{t-1}] with the packed [2*Np][Kp] block (rows n = 4j+q:
// gate q of unit j, hi then lo), followed by the cell update in registers.
struct TcLstmArgs {
    CUtensorMap map;  // over the block, box {32, Np}
    const float *arena;
    long long b_off, h0_const, c0_const;  // gate bias [Np]; per-unit constant state or -1
    const float *x;
    long long ld_x;  // row t + T*i
    const float *h0;
    long long ld_h0;
    const float *c0;
    long long ld_c0;
    float *y;
    long long ld_y;  // row t + T*j
    float *hn;
    long long ld_hn;
    float *cn;
    long long ld_cn;
    long long n;
    int *err;
    int T, I, H, Np, nx, nh;  // nx / nh: K chunks of 32 of the x / h parts
};

// Two stacked LSTM layers with hidden size 64 (4H = 256) and layer-1 input
// width <= 32, fused in one kernel (lstm2_tc.cu): layer 2 reads layer 1's h_t
// from shared memory.  The blocks are the per-layer tensor-core blocks
// ([2*256][Kp], Kp = 96 and 128), read through maps with boxes of {32, 128}.
struct TcLstm2Args {
    CUtensorMap map1, map2;
    const float *arena;
    long long h0_const[2], c0_const[2];  // per-unit constant initial state or -1
    const float *x;
    long long ld_x;                      // row t + T*i
    const float *h0[2];
    long long ld_h0[2];
    const float *c0[2];
    long long ld_c0[2];
    float *y2;                           // layer 2's output sequence (row t + T*j) or null
    long long ld_y2;
    float *hn[2];
    long long ld_hn[2];
    float *cn[2];
    long long ld_cn[2];
    long long n;
    int *err;
    int T, I;
    float bias1[256], bias2[256];        // b_ih + b_hh per gate column
};

size_t mlp_tc_smem_bytes();
// The tensor-core kernels redistribute their launch registers between roles
// (setmaxnreg) and only run when the compiler gave them exactly the count that
// split assumes.  False when it did not (the plan then uses the FFMA kernels);
// true also when no device can be asked (launches check again).
bool tc_register_split_ok();
cudaError_t mlp_tc_configure();
cudaError_t launch_mlp_tc(const TcArgs &a, int num_sms, cudaStream_t st);
// Narrow chains (mlp_narrow_tc.cu): whether `a` fits the kernel, its
// shared-memory attribute, and its launch (one CTA per SM, two tiles at a time).
bool mlp_narrow_fits(const TcArgs &a);
cudaError_t mlp_narrow_configure();
cudaError_t launch_mlp_narrow(const TcArgs &a, int num_sms, cudaStream_t st);
// Narrow chains with a long first layer (mlp_narrow_tc.cu, mlp_stream_tc_kernel).
// The launch returns cudaErrorNotSupported, launching nothing, when the input
// array cannot be described by a tensor map (16-byte aligned base and pitch).
bool mlp_stream_fits(const TcArgs &a);
cudaError_t mlp_stream_configure();
cudaError_t launch_mlp_stream(const TcArgs &a, int num_sms, cudaStream_t st);
cudaError_t launch_lstm_tc(const TcLstmArgs &a, int num_sms, cudaStream_t st);

// Encodes the TMA map of one layer block at `block` (device pointer), with
// boxes of {32, box_rows} (box_rows 0: Np).  Returns false (with *why set) when
// the driver entry point or encode fails.
bool mlp_tc_encode_map(CUtensorMap *map, const float *block, int Kp, int Np, const char **why, int box_rows = 0);
// Encodes a tiled fp32 TMA map of `rank` dimensions (dims innermost first,
// strides in bytes for dims 1..rank-1), zero fill out of bounds, 128-byte
// swizzle (CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B for an operand the MMA reads
// MN-major).  Returns false (with *why set) when the driver entry point or
// encode fails.
bool tc_encode_f32_map(CUtensorMap *map, int rank, const void *base, const cuuint64_t *dims, const cuuint64_t *strides,
                       const cuuint32_t *box, const char **why,
                       CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// One LSTM layer with I <= 32, H <= 32 (4H <= 128), each column group running
// a tile of its own (lstm_dual_tc.cu); TcLstmArgs as for launch_lstm_tc.
bool lstm_dual_tc_regs_ok();
cudaError_t lstm_dual_tc_configure();
cudaError_t launch_lstm_dual_tc(const TcLstmArgs &a, int num_sms, cudaStream_t st);

// The fused two-layer LSTM kernel.
bool lstm2_tc_regs_ok();
cudaError_t lstm2_tc_configure();
cudaError_t launch_lstm2_tc(const TcLstm2Args &a, int num_sms, cudaStream_t st);

}  // namespace rosenna
