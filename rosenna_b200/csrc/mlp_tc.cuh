// Tensor-core (tcgen05, 3xTF32) fused MLP: parameter block and launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace rosenna {

constexpr int kTcMaxLayers = 8;

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
    int nlayers;
    TcLayer L[kTcMaxLayers];
};

size_t mlp_tc_smem_bytes();
cudaError_t mlp_tc_configure();
cudaError_t launch_mlp_tc(const TcArgs &a, int num_sms, cudaStream_t st);

// Encodes the TMA map of one layer block at `block` (device pointer).
// Returns false (with *why set) when the driver entry point or encode fails.
bool mlp_tc_encode_map(CUtensorMap *map, const float *block, int Kp, int Np, const char **why);

}  // namespace rosenna
