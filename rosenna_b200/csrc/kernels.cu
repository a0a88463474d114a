// sm_100a kernels of the launch plan.
//
// Layout (all kernels): a batched tensor is rows x n floats, row r of sample s at
// base[r * ld + s]; consecutive threads own consecutive samples, so every global
// access is a coalesced row segment.
//
// mlp_ffma  : a whole Gemm+bias+activation chain (fLibrary/layers.f90:11-23 and
//             activation_funcs.f90) per tile of S samples.  Activations stay in
//             shared memory between layers; weights stream through a cp.async
//             double buffer in 32-row chunks; each thread owns an 8x8 register
//             tile (8 outputs x 8 samples) of every layer's product.
// lstm_ffma : persistent time loop of one LSTM layer (layers.f90:62-132) per
//             tile of S samples: [W_ih | W_hh] resident in shared memory with
//             each unit's four gates in adjacent columns, so one thread's tile
//             holds all gates of two units and updates their cell state in
//             registers; h_t goes back to shared memory for step t+1.
// conv_pool : direct convolution (layers.f90:183-233) + ReLU + max/avg pool
//             (layers.f90:236-310) with zero padding.  The tiled kernel (stride
//             1, 3x3 kernels, pool windows up to 2x2) gives each lane one sample
//             and each warp a (pooled position, 8 output channels) item:
//             the input patch of the pool window sits in registers, the weights
//             are broadcast from shared memory, and every pool-window conv
//             output of every channel in the group accumulates in registers.
//             Other shapes use one thread per sample and pooled element.
#include "kernels.cuh"

#include <algorithm>
#include <cstdlib>
#include <string>

namespace rosenna {

namespace {

constexpr int kThreads = 256;
constexpr int kKC = 32;  // weight rows per streamed chunk
constexpr size_t kMaxSmem = 226 * 1024;  // dynamic budget; leaves room for static shared memory

// ---- activations -----------------------------------------------------------
// tanh(x) = 1 - 2 / (1 + e^{2x}) and sigmoid(x) = 1 / (1 + e^{-x}), with
// e^y = 2^(y log2 e) from the hardware exp2 unit and a hardware reciprocal.
// Absolute error ~2e-7, far inside the 1e-5 tolerance against the fp64 path.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float act_tanh(float x) {
    return 1.f - 2.f * rcp_approx(1.f + ex2_approx(2.8853900817779268f * x));
}
__device__ __forceinline__ float act_sigmoid(float x) { return rcp_approx(1.f + ex2_approx(-1.4426950408889634f * x)); }
__device__ __forceinline__ float apply_act(float v, int act) {
    switch (act) {
        case 1: return v < 0.f ? 0.f : v;  // relu: `where (x < 0) 0 elsewhere x`
        case 2: return act_tanh(v);
        case 3: return act_sigmoid(v);
        default: return v;
    }
}

// ---- cp.async helpers ------------------------------------------------------
__device__ __forceinline__ unsigned smem_addr(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src));
}
// 4-byte copy; src_bytes == 0 writes zero without reading src
__device__ __forceinline__ void cp_async4(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Copies rows [r0, r0+nr) x samples [0, S) of a batched tensor into shared
// memory (row stride S), zero-filling rows >= rows_valid and samples >= nval.
__device__ __forceinline__ void stage_rows(float *dst, const float *src, long long ld, int r0, int nr, int rows_valid,
                                           int S, int nval, bool vec_ok) {
    const int q4 = S >> 2;
    for (int i = threadIdx.x; i < nr * q4; i += blockDim.x) {
        int r = i / q4, q = (i - r * q4) << 2, row = r0 + r;
        float *d = dst + r * S + q;
        const float *s = src + (long long)row * ld + q;
        if (row < rows_valid && vec_ok && q + 4 <= nval) {
            cp_async16(d, s);
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                bool ok = row < rows_valid && q + e < nval;
                cp_async4(d + e, ok ? (const void *)(s + e) : (const void *)src, ok ? 4 : 0);
            }
        }
    }
}

// ---- fused MLP ---------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) mlp_ffma_kernel(const MlpArgs p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ MlpLayerDev L[kMaxMlpLayers];
    const int tid = threadIdx.x, S = p.S, nl = p.nlayers;
    if (tid < nl) L[tid] = p.layers[tid];
    // double-buffered regions, addressed as offsets from the shared base (an
    // array of pointers would live in local memory and make the loads generic)
    const int act_sz = p.hid_rows * S, stw_sz = kKC * p.max_mp, sta_sz = p.stage_a_rows * S;
    float *const act0 = sm;                  // two [hid_rows][S] activation blocks
    float *const stW0 = act0 + 2 * act_sz;   // two [kKC][max_mp] weight chunks
    float *const stA0 = stW0 + 2 * stw_sz;   // two [stage_a_rows][S] input chunks
    float *bias = stA0 + 2 * sta_sz;
    __syncthreads();
    {
        int bo = 0;
        for (int l = 0; l < nl; l++) {
            for (int i = tid; i < L[l].Mp; i += kThreads) bias[bo + i] = p.arena[L[l].b_off + i];
            bo += L[l].Mp;
        }
    }
    const long long ntiles = (p.n + S - 1) / S;
    long long tile = blockIdx.x;
    if (tile >= ntiles) return;
    const bool in_vec = ((p.ld_in & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.in) & 15) == 0);

    auto issue = [&](long long t, int l, int c, int st) {
        const int k0 = c * kKC, kc = min(kKC, L[l].Kp - k0), mp = L[l].Mp;
        const float *src = p.arena + L[l].w_off + (long long)k0 * mp;
        const int nv = kc * mp / 4;
        for (int i = tid; i < nv; i += kThreads) cp_async16(stW0 + st * stw_sz + 4 * i, src + 4 * i);
        if (l == 0) {
            long long n0 = t * S;
            int nval = (int)min((long long)S, p.n - n0);
            stage_rows(stA0 + st * sta_sz, p.in + n0, p.ld_in, k0, kc, L[0].K, S, nval, in_vec && (n0 & 3) == 0);
        }
        cp_async_commit();
    };

    int st = 0;
    issue(tile, 0, 0, 0);
    for (; tile < ntiles; tile += gridDim.x) {
        const long long n0 = tile * S;
        const int nval = (int)min((long long)S, p.n - n0);
        int bo = 0;
        for (int l = 0; l < nl; l++) {
            const int Mp = L[l].Mp, Kp = L[l].Kp;
            const int mg_n = Mp >> 3, sg_n = S >> 3;
            const bool active = tid < mg_n * sg_n;
            const int mg = tid % mg_n, sg = tid / mg_n;
            const int m0 = mg * 4, s0 = sg * 4, mh = Mp >> 1, sh = S >> 1;
            const float *aprev = act0 + ((l + 1) & 1) * act_sz;
            float acc[8][8];
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
            const int nch = (Kp + kKC - 1) / kKC;
            for (int c = 0; c < nch; c++) {
                cp_async_wait_all();
                __syncthreads();
                // prefetch the next chunk of the cyclic (tile, layer, chunk) sequence
                if (c + 1 < nch) issue(tile, l, c + 1, st ^ 1);
                else if (l + 1 < nl) issue(tile, l + 1, 0, st ^ 1);
                else if (tile + gridDim.x < ntiles) issue(tile + gridDim.x, 0, 0, st ^ 1);
                if (active) {
                    const float *W = stW0 + st * stw_sz;
                    const float *A = (l == 0) ? stA0 + st * sta_sz : aprev + c * kKC * S;
                    const int kc = min(kKC, Kp - c * kKC);
#pragma unroll 4
                    for (int kk = 0; kk < kc; kk++) {
                        const float4 a0 = *reinterpret_cast<const float4 *>(A + kk * S + s0);
                        const float4 a1 = *reinterpret_cast<const float4 *>(A + kk * S + sh + s0);
                        const float4 w0 = *reinterpret_cast<const float4 *>(W + kk * Mp + m0);
                        const float4 w1 = *reinterpret_cast<const float4 *>(W + kk * Mp + mh + m0);
                        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                        for (int i = 0; i < 8; i++)
#pragma unroll
                            for (int j = 0; j < 8; j++) acc[i][j] = fmaf(w[i], a[j], acc[i][j]);
                    }
                }
                st ^= 1;
            }
            if (active) {
                const int actf = L[l].act;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int m = (i < 4 ? m0 + i : mh + m0 + i - 4);
                    const float b = bias[bo + m];
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = apply_act(acc[i][j] + b, actf);
                }
                if (l + 1 < nl) {
                    float *O = act0 + (l & 1) * act_sz;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int m = (i < 4 ? m0 + i : mh + m0 + i - 4);
                        *reinterpret_cast<float4 *>(O + (size_t)m * S + s0) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
                        *reinterpret_cast<float4 *>(O + (size_t)m * S + sh + s0) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
                    }
                } else {
                    const int M = L[l].M;
                    const bool vec = ((p.ld_out & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0) && ((n0 & 3) == 0);
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int m = (i < 4 ? m0 + i : mh + m0 + i - 4);
                        if (m >= M) continue;
                        float *o = p.out + (long long)m * p.ld_out + n0;
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int s = (h ? sh : 0) + s0;
                            if (vec && s + 4 <= nval) {
                                *reinterpret_cast<float4 *>(o + s) =
                                    make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
                            } else {
#pragma unroll
                                for (int e = 0; e < 4; e++)
                                    if (s + e < nval) o[s + e] = acc[i][4 * h + e];
                            }
                        }
                    }
                }
            }
            bo += Mp;
        }
    }
    cp_async_wait_all();
}

// ---- LSTM ----------------------------------------------------------------------
// kPerSm CTAs per SM: with 2 (<= 128 registers a thread, for tiles whose
// shared memory lets two fit) one tile's barrier and gate activations overlap
// the other tile's FMA loop.
// kHp > 0: the padded hidden size and the tile (S = 8 * kThreads / (kHp / 2)
// samples) are compile-time constants, so every operand load is a base register
// plus an immediate offset; kHp = 0 reads both from the arguments.
template <int kHp>
constexpr int lstm_tile_samples() { return kHp ? (8 * kThreads / (kHp / 2) < 256 ? 8 * kThreads / (kHp / 2) : 256) : 0; }
template <int kPerSm, int kHp>
__global__ void __launch_bounds__(kThreads, kPerSm) lstm_ffma_kernel(const LstmArgs p) {
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, S = kHp ? lstm_tile_samples<kHp>() : p.S, Ip = p.Ip, Hp = kHp ? kHp : p.Hp,
              G = 4 * Hp, K = Ip + Hp;
    float *W = sm;                        // [K][G]
    float *bias = W + (size_t)K * G;      // [G]
    // two [K][S] blocks (rows 0..Ip-1 = x_t, Ip.. = h), addressed as offsets from
    // the shared base so every operand load stays a shared-space load
    float *const actb = bias + G;
    const int act_sz = K * S;
    {
        const float4 *src = reinterpret_cast<const float4 *>(p.arena + p.w_off);
        for (int i = tid; i < K * G / 4; i += kThreads) cp_async16(W + 4 * i, src + i);
        for (int i = tid; i < G; i += kThreads) bias[i] = p.arena[p.b_off + i];
        cp_async_commit();
    }
    const int mg_n = Hp >> 1, sg_n = S >> 3;
    const bool active = tid < mg_n * sg_n;
    const int mg = tid % mg_n, sg = tid / mg_n;
    const int s0 = sg * 4, sh = S >> 1;
    const int c0l = mg * 4, c1l = G / 2 + mg * 4;  // gate columns of the two units
    const int u0 = mg, u1 = Hp / 2 + mg;           // the two units
    const bool x_vec = ((p.ld_x & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
    const long long ntiles = (p.n + S - 1) / S;
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long n0 = tile * S;
        const int nval = (int)min((long long)S, p.n - n0);
        const bool vec = x_vec && (n0 & 3) == 0;
        __syncthreads();  // previous tile finished with the activation blocks
        // x_0 into block 0 rows [0, Ip) (rows >= I zero); zero the padding rows of block 1
        stage_rows(actb, p.x + n0, (long long)p.T * p.ld_x, 0, Ip, p.I, S, nval, vec);
        for (int i = tid; i < (Ip - p.I) * S; i += kThreads) actb[act_sz + p.I * S + i] = 0.f;
        // h0 into block 0 rows [Ip, Ip+Hp)
        for (int i = tid; i < Hp * S; i += kThreads) {
            int j = i / S, s = i - j * S;
            float v = 0.f;
            if (j < p.H && s < nval) {
                if (p.h0) v = p.h0[(long long)j * p.ld_h0 + n0 + s];
                else if (p.h0_const >= 0) v = p.arena[p.h0_const + j];
            }
            actb[(Ip + j) * S + s] = v;
        }
        cp_async_commit();
        float c[2][8];
#pragma unroll
        for (int u = 0; u < 2; u++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int unit = u ? u1 : u0, s = (j < 4 ? s0 + j : sh + s0 + j - 4);
                float v = 0.f;
                if (active && unit < p.H && s < nval) {
                    if (p.c0) v = p.c0[(long long)unit * p.ld_c0 + n0 + s];
                    else if (p.c0_const >= 0) v = p.arena[p.c0_const + unit];
                }
                c[u][j] = v;
            }
        cp_async_wait_all();
        __syncthreads();
        for (int t = 0; t < p.T; t++) {
            const float *A = actb + (t & 1) * act_sz;
            float *Nx = actb + ((t + 1) & 1) * act_sz;
            if (t + 1 < p.T) {
                // x_{t+1}: row (t+1) + T*i of the input
                stage_rows(Nx, p.x + (long long)(t + 1) * p.ld_x + n0, (long long)p.T * p.ld_x, 0, p.I, p.I, S, nval,
                           vec && ((p.ld_x * (t + 1)) & 3) == 0);
                cp_async_commit();
            }
            if (active) {
                float acc[8][8];
                {  // k = 0 accumulates onto the gate biases (b_ih + b_hh)
                    const float4 b0 = *reinterpret_cast<const float4 *>(bias + c0l);
                    const float4 b1 = *reinterpret_cast<const float4 *>(bias + c1l);
                    const float4 a0 = *reinterpret_cast<const float4 *>(A + s0);
                    const float4 a1 = *reinterpret_cast<const float4 *>(A + sh + s0);
                    const float4 w0 = *reinterpret_cast<const float4 *>(W + c0l);
                    const float4 w1 = *reinterpret_cast<const float4 *>(W + c1l);
                    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
                    const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(w[i], a[j], bv[i]);
                }
#pragma unroll(kPerSm == 1 ? 4 : 2)
                for (int k = 1; k < K; k++) {
                    const float4 a0 = *reinterpret_cast<const float4 *>(A + k * S + s0);
                    const float4 a1 = *reinterpret_cast<const float4 *>(A + k * S + sh + s0);
                    const float4 w0 = *reinterpret_cast<const float4 *>(W + k * G + c0l);
                    const float4 w1 = *reinterpret_cast<const float4 *>(W + k * G + c1l);
                    const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(w[i], a[j], acc[i][j]);
                }
                // gates of unit u are acc rows 4u..4u+3 (i, f, g, o), layers.f90:88-96
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int unit = u ? u1 : u0;
                    float h[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float ig = act_sigmoid(acc[4 * u][j]);
                        const float fg = act_sigmoid(acc[4 * u + 1][j]);
                        const float gg = act_tanh(acc[4 * u + 2][j]);
                        const float og = act_sigmoid(acc[4 * u + 3][j]);
                        c[u][j] = fg * c[u][j] + ig * gg;
                        h[j] = og * act_tanh(c[u][j]);
                    }
                    float *hr = Nx + (size_t)(Ip + unit) * S;
                    *reinterpret_cast<float4 *>(hr + s0) = make_float4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<float4 *>(hr + sh + s0) = make_float4(h[4], h[5], h[6], h[7]);
                    if (p.y && unit < p.H) {
                        float *yr = p.y + (long long)(t + p.T * unit) * p.ld_y + n0;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const int s = (j < 4 ? s0 + j : sh + s0 + j - 4);
                            if (s < nval) yr[s] = h[j];
                        }
                    }
                }
            }
            cp_async_wait_all();
            __syncthreads();
        }
        if (active) {
            // h_T is the h rows of block T & 1 (the last step's barrier published them)
            const float *hT = actb + (p.T & 1) * act_sz;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int unit = u ? u1 : u0;
                if (unit >= p.H) continue;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int s = (j < 4 ? s0 + j : sh + s0 + j - 4);
                    if (s >= nval) continue;
                    if (p.hn) p.hn[(long long)unit * p.ld_hn + n0 + s] = hT[(size_t)(Ip + unit) * S + s];
                    if (p.cn) p.cn[(long long)unit * p.ld_cn + n0 + s] = c[u][j];
                }
            }
        }
    }
}

// ---- conv + relu + pool --------------------------------------------------------
__device__ __forceinline__ float conv_value(const ConvArgs &p, const float *in, int oc, int ch, int cw) {
    if (!p.conv) return in[(long long)(oc + p.C * (ch + p.Hin * cw)) * p.ld_in];
    const float *w = p.arena + p.w_off + (long long)oc * p.C * p.KS * p.KS;
    float acc = 0.f;
    for (int ic = 0; ic < p.C; ic++)
        for (int kh = 0; kh < p.KS; kh++) {
            const int ih = ch * p.str_h - p.pad_h + kh;
            if (ih < 0 || ih >= p.Hin) continue;
            for (int kw = 0; kw < p.KS; kw++) {
                const int iw = cw * p.str_w - p.pad_w + kw;
                if (iw < 0 || iw >= p.Win) continue;
                acc = fmaf(__ldg(w + (ic * p.KS + kh) * p.KS + kw), in[(long long)(ic + p.C * (ih + p.Hin * iw)) * p.ld_in], acc);
            }
        }
    acc += __ldg(p.arena + p.b_off + oc);
    return p.relu ? (acc < 0.f ? 0.f : acc) : acc;
}

// Lane = sample (32 consecutive samples per warp, coalesced rows), warp = a
// stream of (pooled position, channel group) items.  Shared memory holds the
// weights as [ic][kh][kw][oc] (oc fastest, OCp = OC rounded up to OCB) and the
// bias, so each (ic, kh, kw) step reads OCB weights with OCB/4 broadcast loads.
// Semantics are those of conv_pool_kernel below: conv zero padding by skipping,
// pool-window positions outside the conv output count as 0.
template <int KS, int PK, int OCB>
__global__ void __launch_bounds__(256, (PK - 1 + KS) > 5 || PK == 3 ? 1 : 2) conv_pool_tile_kernel(const ConvArgs p) {
    extern __shared__ float sw[];
    constexpr int P = PK - 1 + KS;  // input patch side of one pool window
    const int OCp = (p.OC + OCB - 1) / OCB * OCB;
    const int nw = p.C * KS * KS * OCp;
    for (int i = threadIdx.x; i < nw; i += blockDim.x) {
        const int oc = i % OCp, r = i / OCp;  // r = (ic*KS + kh)*KS + kw
        sw[i] = oc < p.OC ? p.arena[p.w_off + (long long)oc * p.C * KS * KS + r] : 0.f;
    }
    for (int i = threadIdx.x; i < OCp; i += blockDim.x) sw[nw + i] = i < p.OC ? p.arena[p.b_off + i] : 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const long long s = (long long)blockIdx.x * 32 + lane;
    const bool full = (long long)blockIdx.x * 32 + 32 <= p.n;  // all 32 lanes hold a sample (warp-uniform)
    const bool valid = s < p.n;
    const float *in = p.in + (valid ? s : 0);
    const long long sa = (long long)p.C * p.ld_in, sb = (long long)p.C * p.Hin * p.ld_in;  // +1 in h, +1 in w
    const int ngrp = OCp / OCB, items = p.Hq * p.Wq * ngrp;
    for (int item = warp; item < items; item += nwarps) {
        const int grp = item % ngrp, pos = item / ngrp, ph = pos % p.Hq, pw = pos / p.Hq;
        const int ch0 = PK > 1 ? ph * p.pstr_h - p.ppad_h : ph, cw0 = PK > 1 ? pw * p.pstr_w - p.ppad_w : pw;
        const int ih0 = ch0 - p.pad_h, iw0 = cw0 - p.pad_w;
        // the whole patch inside the input and every lane a sample: no checks
        const bool inner = full && ih0 >= 0 && ih0 + P <= p.Hin && iw0 >= 0 && iw0 + P <= p.Win;
        float acc[PK][PK][OCB];
#pragma unroll
        for (int a = 0; a < PK; a++)
#pragma unroll
            for (int b = 0; b < PK; b++)
#pragma unroll
                for (int o = 0; o < OCB; o++) acc[a][b][o] = 0.f;
        const float *wg = sw + grp * OCB;
        const float *pin = inner ? in + (long long)p.C * (ih0 + p.Hin * iw0) * p.ld_in : in;
#pragma unroll 1
        for (int ic = 0; ic < p.C; ic++) {
            if constexpr (P > 5) {
                // wide patches stream row by row (P registers instead of P*P):
                // patch row ar feeds conv row a = ar - kh of every kernel row kh
#pragma unroll
                for (int ar = 0; ar < P; ar++) {
                    float xr[P];
#pragma unroll
                    for (int b = 0; b < P; b++) {
                        const int ih = ih0 + ar, iw = iw0 + b;
                        xr[b] = inner ? __ldg(pin + (long long)ic * p.ld_in + ar * sa + b * sb)
                                      : (valid && ih >= 0 && ih < p.Hin && iw >= 0 && iw < p.Win)
                                            ? __ldg(in + (long long)(ic + p.C * (ih + p.Hin * iw)) * p.ld_in)
                                            : 0.f;
                    }
#pragma unroll
                    for (int kh = 0; kh < KS; kh++) {
                        const int a = ar - kh;
                        if (a < 0 || a >= PK) continue;
#pragma unroll
                        for (int kw = 0; kw < KS; kw++) {
                            const float4 *w4 = reinterpret_cast<const float4 *>(wg + ((ic * KS + kh) * KS + kw) * OCp);
#pragma unroll
                            for (int o4 = 0; o4 < OCB / 4; o4++) {
                                const float4 w = w4[o4];
#pragma unroll
                                for (int b = 0; b < PK; b++) {
                                    const float xv = xr[b + kw];
                                    acc[a][b][4 * o4 + 0] = fmaf(w.x, xv, acc[a][b][4 * o4 + 0]);
                                    acc[a][b][4 * o4 + 1] = fmaf(w.y, xv, acc[a][b][4 * o4 + 1]);
                                    acc[a][b][4 * o4 + 2] = fmaf(w.z, xv, acc[a][b][4 * o4 + 2]);
                                    acc[a][b][4 * o4 + 3] = fmaf(w.w, xv, acc[a][b][4 * o4 + 3]);
                                }
                            }
                        }
                    }
                }
                continue;
            }
            float x[P][P];
            if (inner) {
                const float *q = pin + (long long)ic * p.ld_in;
#pragma unroll
                for (int b = 0; b < P; b++)
#pragma unroll
                    for (int a = 0; a < P; a++) x[a][b] = __ldg(q + a * sa + b * sb);
            } else {
#pragma unroll
                for (int a = 0; a < P; a++)
#pragma unroll
                    for (int b = 0; b < P; b++) {
                        const int ih = ih0 + a, iw = iw0 + b;
                        x[a][b] = (valid && ih >= 0 && ih < p.Hin && iw >= 0 && iw < p.Win)
                                      ? __ldg(in + (long long)(ic + p.C * (ih + p.Hin * iw)) * p.ld_in)
                                      : 0.f;
                    }
            }
#pragma unroll
            for (int kh = 0; kh < KS; kh++)
#pragma unroll
                for (int kw = 0; kw < KS; kw++) {
                    const float4 *w4 = reinterpret_cast<const float4 *>(wg + ((ic * KS + kh) * KS + kw) * OCp);
#pragma unroll
                    for (int o4 = 0; o4 < OCB / 4; o4++) {
                        const float4 w = w4[o4];
#pragma unroll
                        for (int a = 0; a < PK; a++)
#pragma unroll
                            for (int b = 0; b < PK; b++) {
                                const float xv = x[a + kh][b + kw];
                                acc[a][b][4 * o4 + 0] = fmaf(w.x, xv, acc[a][b][4 * o4 + 0]);
                                acc[a][b][4 * o4 + 1] = fmaf(w.y, xv, acc[a][b][4 * o4 + 1]);
                                acc[a][b][4 * o4 + 2] = fmaf(w.z, xv, acc[a][b][4 * o4 + 2]);
                                acc[a][b][4 * o4 + 3] = fmaf(w.w, xv, acc[a][b][4 * o4 + 3]);
                            }
                    }
                }
        }
        // pool-window positions outside the conv output count as 0 (zero-padded pool input)
        const bool win_inside = ch0 >= 0 && ch0 + PK <= p.Ho && cw0 >= 0 && cw0 + PK <= p.Wo;
        float *po = p.out + (long long)(ph * p.so_h + pw * p.so_w) * p.ld_out + s;
#pragma unroll
        for (int o = 0; o < OCB; o++) {
            const int oc = grp * OCB + o;
            if (oc >= p.OC) break;
            const float bias = sw[nw + oc];
            float best = -INFINITY, sum = 0.f;
#pragma unroll
            for (int a = 0; a < PK; a++)
#pragma unroll
                for (int b = 0; b < PK; b++) {
                    float v = acc[a][b][o] + bias;
                    if (p.relu) v = v < 0.f ? 0.f : v;
                    if (!win_inside && (ch0 + a < 0 || ch0 + a >= p.Ho || cw0 + b < 0 || cw0 + b >= p.Wo)) v = 0.f;
                    best = fmaxf(best, v);
                    sum += v;
                }
            const float y = PK == 1 ? sum : (p.pool == 1 ? best : sum * (1.f / (float)(PK * PK)));
            if (valid) po[(long long)oc * p.so_c * p.ld_out] = y;
        }
    }
}

__global__ void __launch_bounds__(128) conv_pool_kernel(const ConvArgs p) {
    const long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= p.n) return;
    const int e = blockIdx.y;  // pooled output element, oc fastest
    const int oc = e % p.OC, rest = e / p.OC, ph = rest % p.Hq, pw = rest / p.Hq;
    const float *in = p.in + s;
    float v;
    if (!p.pool) {
        v = conv_value(p, in, oc, ph, pw);
    } else {
        float best = -INFINITY, sum = 0.f;
        for (int dw = 0; dw < p.pk; dw++)
            for (int dh = 0; dh < p.pk; dh++) {
                const int ch = ph * p.pstr_h - p.ppad_h + dh, cw = pw * p.pstr_w - p.ppad_w + dw;
                // the reference zero-pads the pooled array (layers.f90:134-181)
                const float x = (ch < 0 || ch >= p.Ho || cw < 0 || cw >= p.Wo) ? 0.f : conv_value(p, in, oc, ch, cw);
                best = fmaxf(best, x);
                sum += x;
            }
        v = p.pool == 1 ? best : sum / (float)(p.pk * p.pk);
    }
    p.out[(long long)(oc * p.so_c + ph * p.so_h + pw * p.so_w) * p.ld_out + s] = v;
}

// ---- data movement / elementwise ------------------------------------------------
// A model input whose batch index is not its first (reference layout: element
// (p, s, q) of shape (pre.., n, post..) at p + pre*s + pre*ld_in*q) into the
// plan's row layout (row p + pre*q, samples contiguous).
__global__ void deinterleave_kernel(const float *in, long long ld_in, float *out, long long ld_out, int pre,
                                    long long n) {
    const long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const int r = blockIdx.y, p = r % pre, q = r / pre;
    out[(long long)r * ld_out + s] = in[(long long)q * pre * ld_in + (long long)pre * s + p];
}

__global__ void gather_kernel(const float *in, long long ld_in, float *out, long long ld_out, const int *map, long long n) {
    const long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const long long r = blockIdx.y;
    const long long src = map ? map[r] : r;
    out[r * ld_out + s] = in[src * ld_in + s];
}

// out row r = act(in row r (+ add[r])): standalone activations and the Add of a
// per-row constant (an ONNX Add whose adder broadcasts over the samples)
__global__ void act_kernel(const float *in, long long ld_in, float *out, long long ld_out, long long n, int act,
                           const float *add) {
    const long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const long long r = blockIdx.y;
    const float x = in[r * ld_in + s];
    out[r * ld_out + s] = apply_act(add ? x + add[r] : x, act);
}

}  // namespace

size_t mlp_smem_bytes(const MlpLayerDev *L, int nl, int *S_out) {
    int max_mp = 8, hid = 8, bias_total = 0;
    for (int l = 0; l < nl; l++) {
        max_mp = std::max(max_mp, L[l].Mp);
        if (l + 1 < nl) hid = std::max(hid, L[l].Mp);
        bias_total += L[l].Mp;
    }
    const int a_rows = std::min(kKC, L[0].Kp);
    // every layer's product must fit one 8x8 tile per thread: (Mp/8)*(S/8) <= 256
    for (int S = std::min(256, (16384 / max_mp) / 8 * 8); S >= 8; S -= 8) {
        size_t bytes = sizeof(float) * ((size_t)2 * hid * S + (size_t)2 * kKC * max_mp + (size_t)2 * a_rows * S + bias_total);
        if (bytes <= kMaxSmem) {
            *S_out = S;
            return bytes;
        }
    }
    return 0;
}

size_t lstm_smem_bytes(int Ip, int Hp, int *S_out) {
    const int K = Ip + Hp, G = 4 * Hp;
    int Smax = std::min(256, (8 * kThreads / (Hp / 2)) / 8 * 8);
    for (int S = Smax; S >= 8; S -= 8) {
        size_t bytes = sizeof(float) * ((size_t)K * G + G + (size_t)2 * K * S);
        if (bytes <= kMaxSmem) {
            *S_out = S;
            return bytes;
        }
    }
    return 0;
}

cudaError_t configure_kernels() {
    cudaError_t e = cudaFuncSetAttribute(mlp_ffma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(lstm_ffma_kernel<1, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(lstm_ffma_kernel<2, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lstm_ffma_kernel<2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
}

cudaError_t launch_mlp(MlpArgs a, const MlpLayerDev *L, int num_sms, cudaStream_t st) {
    int S = 0;
    size_t bytes = mlp_smem_bytes(L, a.nlayers, &S);
    if (!bytes) return cudaErrorInvalidConfiguration;
    a.S = S;
    a.max_mp = 8;
    a.hid_rows = 8;
    a.bias_total = 0;
    for (int l = 0; l < a.nlayers; l++) {
        a.max_mp = std::max(a.max_mp, L[l].Mp);
        if (l + 1 < a.nlayers) a.hid_rows = std::max(a.hid_rows, L[l].Mp);
        a.bias_total += L[l].Mp;
    }
    a.stage_a_rows = std::min(kKC, L[0].Kp);
    const long long tiles = (a.n + S - 1) / S;
    const int grid = (int)std::min<long long>(tiles, num_sms);
    if (grid <= 0) return cudaSuccess;
    mlp_ffma_kernel<<<grid, kThreads, bytes, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_lstm(LstmArgs a, int num_sms, cudaStream_t st) {
    int S = 0;
    size_t bytes = lstm_smem_bytes(a.Ip, a.Hp, &S);
    if (!bytes) return cudaErrorInvalidConfiguration;
    a.S = S;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lstm_ffma_kernel<2, 0>, kThreads, bytes) != cudaSuccess)
        per_sm = 0;
    const bool two = per_sm >= 2;
    const long long tiles = (a.n + S - 1) / S;
    const int grid = (int)std::min<long long>(tiles, (long long)num_sms * (two ? 2 : 1));
    if (grid <= 0) return cudaSuccess;
    if (two && a.Hp == 32 && S == lstm_tile_samples<32>())
        lstm_ffma_kernel<2, 32><<<grid, kThreads, bytes, st>>>(a);
    else if (two)
        lstm_ffma_kernel<2, 0><<<grid, kThreads, bytes, st>>>(a);
    else
        lstm_ffma_kernel<1, 0><<<grid, kThreads, bytes, st>>>(a);
    return cudaGetLastError();
}

template <int KS, int PK, int OCB>
static cudaError_t launch_conv_tile(const ConvArgs &a, cudaStream_t st) {
    const int OCp = (a.OC + OCB - 1) / OCB * OCB;
    const size_t bytes = sizeof(float) * ((size_t)a.C * KS * KS * OCp + OCp);
    const long long tiles = (a.n + 31) / 32;
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    conv_pool_tile_kernel<KS, PK, OCB><<<(unsigned)tiles, 256, bytes, st>>>(a);
    return cudaGetLastError();
}

// Which conv kernel runs a step: the tiled kernel (stride-1 3x3 convolution
// with no pool or a pool window of 2 or 3, 5x5 with no pool or a window of 2;
// 5x5 under a 3-wide window spills even at 255 registers; weights and bias
// within the default 48 KB of dynamic shared memory), else the per-element one.
// ROSENNA_CONV_PATH=direct keeps every convolution on the per-element kernel.
// Returns KS*10 + pool window for the tiled kernel, 0 for the per-element one.
static int conv_tile_variant(const ConvArgs &a) {
    static const bool direct_only = [] {
        const char *e = getenv("ROSENNA_CONV_PATH");
        return e && std::string(e) == "direct";
    }();
    const int pk = a.pool == 0 ? 1 : a.pk;
    const int ocb = pk == 3 ? 4 : 8;  // 3x3 pooled windows of 8 channels would not fit 128 registers
    if (!direct_only && a.conv && (a.KS == 3 || a.KS == 5) && a.str_h == 1 && a.str_w == 1 && pk <= (a.KS == 3 ? 3 : 2) &&
        ((size_t)a.C * a.KS * a.KS + 1) * ((a.OC + ocb - 1) / ocb * ocb) * sizeof(float) <= 48 * 1024)
        return a.KS * 10 + pk;
    return 0;
}

const char *conv_kernel_name(const ConvArgs &a) {
    switch (conv_tile_variant(a)) {
        case 31: return "conv_pool_tile_kernel<3,1,8>";
        case 32: return "conv_pool_tile_kernel<3,2,8>";
        case 33: return "conv_pool_tile_kernel<3,3,4>";
        case 51: return "conv_pool_tile_kernel<5,1,8>";
        case 52: return "conv_pool_tile_kernel<5,2,8>";
        default: return "conv_pool_kernel";
    }
}

cudaError_t launch_conv(const ConvArgs &a, cudaStream_t st) {
    const long long outs = (long long)a.OC * a.Hq * a.Wq;
    if (a.n <= 0 || outs <= 0) return cudaSuccess;
    // 8 output channels per item: two CTAs per SM fit (16 per item spills or halves occupancy)
    switch (conv_tile_variant(a)) {
        case 31: return launch_conv_tile<3, 1, 8>(a, st);
        case 32: return launch_conv_tile<3, 2, 8>(a, st);
        case 33: return launch_conv_tile<3, 3, 4>(a, st);
        case 51: return launch_conv_tile<5, 1, 8>(a, st);
        case 52: return launch_conv_tile<5, 2, 8>(a, st);
        default: break;
    }
    if (outs > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)((a.n + 127) / 128), (unsigned)outs);
    conv_pool_kernel<<<grid, 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_deinterleave(const float *in, long long ld_in, float *out, long long ld_out, int pre, long long rows,
                                long long n, cudaStream_t st) {
    if (n <= 0 || rows <= 0) return cudaSuccess;
    if (rows > 65535 || pre < 1) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)((n + 255) / 256), (unsigned)rows);
    deinterleave_kernel<<<grid, 256, 0, st>>>(in, ld_in, out, ld_out, pre, n);
    return cudaGetLastError();
}

cudaError_t launch_gather(const float *in, long long ld_in, float *out, long long ld_out, const int *map, long long rows,
                          long long n, cudaStream_t st) {
    if (n <= 0 || rows <= 0) return cudaSuccess;
    if (rows > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)((n + 255) / 256), (unsigned)rows);
    gather_kernel<<<grid, 256, 0, st>>>(in, ld_in, out, ld_out, map, n);
    return cudaGetLastError();
}

cudaError_t launch_act(const float *in, long long ld_in, float *out, long long ld_out, long long rows, long long n,
                       int act, const float *add, cudaStream_t st) {
    if (n <= 0 || rows <= 0) return cudaSuccess;
    if (rows > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)((n + 255) / 256), (unsigned)rows);
    act_kernel<<<grid, 256, 0, st>>>(in, ld_in, out, ld_out, n, act, add);
    return cudaGetLastError();
}

}  // namespace rosenna
