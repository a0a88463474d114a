// Launch plan: what fLibrary/modelCreator.fpp's generated use_model does, as a
// list of fused kernel steps over batched device buffers.
//
// Every tensor lives in a buffer of `rows` x n floats: the per-sample elements
// (the Fortran column-major order of the shape without its batch dimension) are
// rows, samples are contiguous within a row.  That is the reference layout of an
// array whose batch dimension is the first non-unit one, so model inputs and
// outputs are used in place, and every kernel reads and writes whole rows of
// consecutive samples (coalesced, vectorisable).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "model_files.hpp"

namespace rosenna {

enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_TANH = 2, ACT_SIGMOID = 3 };

// One Gemm (+ activation) of a fused chain; weights packed as Wt[Kp][Mp] (zero
// padded) for the FFMA kernel and, when M <= 256, as a [2*tc_Np][tc_Kp] block of
// tf32-rounded high parts and remainders for the tensor-core kernel.
struct MlpLayer {
    int K = 0, M = 0, Kp = 0, Mp = 0, act = ACT_NONE;
    int64_t w_off = 0, b_off = 0;
    int tc_Kp = 0, tc_Np = 0;
    int64_t tc_w_off = -1, tc_b_off = -1;
};

struct Step {
    enum Kind { MLP, LSTM, CONV, GATHER, ACT, COPY, ADD, DEINTERLEAVE } kind = MLP;
    int in = -1, out = -1;  // buffer ids

    // MLP (also the head of an LSTM step); rsub sub-rows per sample (row k of
    // sub-row t is buffer row t + rsub*k)
    std::vector<MlpLayer> layers;
    int rsub = 1;
    bool tc = false;  // run on the tensor-core kernel (decided at initialize)

    // LSTM: one layer, PyTorch gate order, gate columns interleaved per unit
    int T = 0, I = 0, H = 0, Ip = 0, Hp = 0;
    int h0 = -1, c0 = -1;              // buffers of the initial state, or -1
    int64_t h0_const = -1, c0_const = -1;  // arena offsets of a per-unit constant initial state
    int y = -1, hn = -1, cn = -1;      // output buffers (-1 when nothing reads them)
    // tensor-core copy of an LSTM layer with 4H <= 256: [2*Np][Kp] block, rows
    // n = 4j+q (gate q of unit j) hi then lo, columns [x (nx chunks of 32) | h (nh)]
    int64_t lstm_tc_w_off = -1, lstm_tc_b_off = -1;
    int lstm_tc_Np = 0, lstm_tc_Kp = 0, lstm_tc_nx = 0, lstm_tc_nh = 0;
    // this LSTM step and the next one (which reads only its y) run as one fused
    // two-layer kernel, its y never materialised; or this CONV step and the
    // next one (the only reader of its output) run as conv_pair_tc_kernel
    // (decided at initialize)
    bool fuse_next = false;
    // run on the dual-tile tensor-core kernel (I <= 32, H <= 32; decided at initialize)
    bool lstm_dual = false;

    // CONV (+ReLU) (+pool); conv == false means pooling only
    bool conv = true, relu = false;
    int C = 0, Hin = 0, Win = 0, OC = 0, KS = 0, pad_h = 0, pad_w = 0, str_h = 1, str_w = 1, Ho = 0, Wo = 0;
    int pool = 0, pk = 1, ppad_h = 0, ppad_w = 0, pstr_h = 1, pstr_w = 1, Hq = 0, Wq = 0;  // pool: 0 none, 1 max, 2 avg
    int64_t so_c = 1, so_h = 0, so_w = 0;  // output row = oc*so_c + h*so_h + w*so_w
    // tensor-core (implicit GEMM) B image of a 3x3 stride-1 conv with C <= 8
    // and OC <= 16 (conv_tc.cuh); -1 when not packed
    int64_t ctc_off = -1;
    // the same weights with each row's tf32 lo part beside its hi part, for the
    // first conv of a fused pair (one input channel, OC <= 8); -1 when not packed
    int64_t ctc_packed_off = -1;

    // packed weights (MLP: per layer; LSTM/CONV: here)
    int64_t w_off = -1, b_off = -1;

    // GATHER: out row r = in row map[r]; ACT: activation; ADD: out row r =
    // act(in row r + arena[b_off + r])
    int64_t map_off = -1;
    int act = ACT_NONE;

    // DEINTERLEAVE: a model input whose batch index is not the first (shape
    // (p.., n, q..), `pre` = product of the dims in front): out row p + pre*q,
    // sample s = in[q*pre*ld_in + pre*s + p] (the reference layout)
    int64_t pre = 1;
};

struct IoDesc {
    std::vector<int64_t> shape;  // export shape
    int bdim = 0;
    int64_t pre = 1;  // elements in front of the batch index (outputs: > 1 only at n == export batch)
    int64_t rows = 0;
    int buf = -1;
};

struct Plan {
    std::vector<int64_t> buf_rows;
    std::vector<IoDesc> inputs, outputs;
    std::vector<Step> steps;
    std::vector<float> arena;  // packed weights, biases and int32 gather maps
    int64_t export_batch = 1;
    std::string describe() const;
};

Status build_plan(const ModelFiles &mf, Plan *plan);

}  // namespace rosenna
