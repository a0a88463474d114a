// Kernel parameter blocks and launchers (sm_100a).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace rosenna {

constexpr int kMaxMlpLayers = 24;

// one layer of a fused MLP chain; offsets in floats from the weight arena
struct MlpLayerDev {
    int K, M, Kp, Mp, act, pad;
    long long w_off, b_off;
};

struct MlpArgs {
    const float *arena;
    const MlpLayerDev *layers;  // device copy of the layer table (in the arena)
    int nlayers;
    const float *in;
    long long ld_in;
    float *out;
    long long ld_out;
    long long n;
    // per-launch geometry (filled by the launcher)
    int S, max_mp, hid_rows, stage_a_rows, bias_total;
};

struct LstmArgs {
    const float *arena;
    long long w_off, b_off, h0_const, c0_const;  // -1: absent
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
    int T, I, H, Ip, Hp, S;
};

struct ConvArgs {
    const float *arena;
    long long w_off, b_off;
    const float *in;
    long long ld_in;
    float *out;
    long long ld_out;
    long long n;
    int conv, relu, C, Hin, Win, OC, KS, pad_h, pad_w, str_h, str_w, Ho, Wo;
    int pool, pk, ppad_h, ppad_w, pstr_h, pstr_w, Hq, Wq;
    long long so_c, so_h, so_w;
};

// All launchers return cudaSuccess or the launch error.
cudaError_t launch_mlp(MlpArgs a, const MlpLayerDev *host_layers, int num_sms, cudaStream_t st);
cudaError_t launch_lstm(LstmArgs a, int num_sms, cudaStream_t st);
cudaError_t launch_conv(const ConvArgs &a, cudaStream_t st);
// Name of the kernel launch_conv runs for these arguments.
const char *conv_kernel_name(const ConvArgs &a);
cudaError_t launch_gather(const float *in, long long ld_in, float *out, long long ld_out, const int *map, long long rows,
                          long long n, cudaStream_t st);
// rows of a model input whose batch index is not its first (pre = product of
// the dims in front of it): reference layout -> row p + pre*q
cudaError_t launch_deinterleave(const float *in, long long ld_in, float *out, long long ld_out, int pre, long long rows,
                                long long n, cudaStream_t st);
// add: per-row constant added before the activation, or nullptr
cudaError_t launch_act(const float *in, long long ld_in, float *out, long long ld_out, long long rows, long long n,
                       int act, const float *add, cudaStream_t st);

// Opt the kernels into large dynamic shared memory on the current device.
cudaError_t configure_kernels();

// Shared-memory bytes a launch needs (0 if the shape cannot run).
size_t mlp_smem_bytes(const MlpLayerDev *layers, int nlayers, int *S_out);
size_t lstm_smem_bytes(int Ip, int Hp, int *S_out);

}  // namespace rosenna
