// Tensor-core MLP for narrow chains whose weights fit in shared memory (every
// tensor-core layer at most 64 wide, at most 64 inputs), 3xTF32 on tcgen05
// (fLibrary/layers.f90:11-23 linear_layer, activation_funcs.f90 per layer).
//
// Math as in mlp_tc.cu: Y = act(A W^T + b) with A = Ah + Al, W = Wh + Wl taken
// as Al*Wh + Ah*Wl + Ah*Wh, accumulated in fp32 in TMEM.
//
// Per CTA (one per SM, persistent): two 128-sample tiles at a time, one per
// warpgroup (thread = sample = TMEM lane).  Every layer's [Wh | Wl] K-chunks
// are loaded once by TMA and stay in shared memory (the B operand).  The A
// operand lives in TMEM: the warpgroup splits the tile's inputs, and after each
// layer its own activations, into tf32 hi and lo parts and stores them into its
// A region, so activations never pass through shared memory and the
// shared-memory port carries only the weights the MMAs read.  One lane issues
// every MMA, layer by layer, tile 0's then tile 1's, so one tile's epilogue
// (bias, activation, split) runs while the other tile's MMAs do.  A narrow last
// layer (N <= 16) runs on the CUDA cores straight from the registers of the
// layer before.  The next tile's inputs (up to 16) are loaded into registers
// while the current tile runs.  With each layer's K-step loop unrolled (immediate descriptor
// offsets), the MMAs issue back to back.
//
// TMEM per tile (256 columns at 256g): A hi at +0, A lo at +64, the layer's
// accumulator at +128 (up to 64 columns).  A layer's MMAs read A while they
// write the accumulator; the epilogue reads the accumulator (all of it, into
// registers) before it writes the next layer's A, and the MMAs that read the
// old A are complete by then (the accumulator's commit).
//
// Roles (288 threads): warps 0-3 tile group 0, warps 4-7 tile group 1, warp 8
// lane 0 loads the weights and issues the MMAs.  Every wait is bounded; a
// time-out records where in `err`, every role finishes, TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mlp_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kNThreads = 288;
constexpr int kNMaxK = 64;                     // widest A (inputs of a tensor-core layer)
constexpr int kNMaxN = 64;                     // widest tensor-core layer
constexpr uint32_t kNTmemCols = 512;
constexpr uint32_t kNSmemW = 160 * 1024;       // resident weight blocks
constexpr uint32_t kNSmemBias = kTcMaxLayers * kNMaxN * 4;
constexpr uint32_t kNSmemTail = kNMaxK * kTcTailMaxN * 4 + kTcTailMaxN * 4;

enum {
    kNWReady = 0,   // the weights landed (TMA bytes)
    kNAFull = 1,    // [2] the tile's A operand written (128 arrivals)
    kNDFull = 3,    // [2] the tile's layer accumulator complete (commit)
    kNDone = 5,
    kNNumBars = 6
};

size_t mlp_narrow_smem() { return 1024 + kNSmemW + kNSmemBias + kNSmemTail + 8 * kNNumBars + 16; }

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Packed fp32 pairs (sm_100 f32x2, round to nearest: the same results as the
// scalar instructions in half the issue slots; the epilogue shares its
// schedulers with the thread that issues the MMAs).
__device__ __forceinline__ void n_add2(float &a, float &b, float c, float d) {
    asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\tadd.rn.f32x2 x, x, y;\n\t"
        "mov.b64 {%0, %1}, x;\n\t}"
        : "+f"(a), "+f"(b)
        : "f"(c), "f"(d));
}
__device__ __forceinline__ void n_mul2(float &a, float &b, float c, float d) {
    asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\tmul.rn.f32x2 x, x, y;\n\t"
        "mov.b64 {%0, %1}, x;\n\t}"
        : "+f"(a), "+f"(b)
        : "f"(c), "f"(d));
}
// (a, b) = (a, b) * (c, c) + (d, d)
__device__ __forceinline__ void n_fma2(float &a, float &b, float c, float d) {
    asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %2};\n\tmov.b64 z, {%3, %3};\n\t"
        "fma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
        : "+f"(a), "+f"(b)
        : "f"(c), "f"(d));
}
// (a, b) += (h, h) * (c, d)
__device__ __forceinline__ void n_fma2v(float &a, float &b, float h, float c, float d) {
    asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %2};\n\tmov.b64 z, {%3, %4};\n\t"
        "fma.rn.f32x2 x, y, z, x;\n\tmov.b64 {%0, %1}, x;\n\t}"
        : "+f"(a), "+f"(b)
        : "f"(h), "f"(c), "f"(d));
}
// (ra, rb) = (a, b) - (c, d)
__device__ __forceinline__ void n_sub2(float a, float b, float c, float d, float &ra, float &rb) {
    asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tsub.rn.f32x2 x, x, y;\n\t"
        "mov.b64 {%0, %1}, x;\n\t}"
        : "=f"(ra), "=f"(rb)
        : "f"(a), "f"(b), "f"(c), "f"(d));
}
__device__ __forceinline__ float n_ex2(float x) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x));
    return e;
}
__device__ __forceinline__ float n_rcp(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// The activation of a pair, with the same operations as tc_act (tanh(x) =
// 1 - 2/(1 + 2^(2 log2(e) x)), sigmoid(x) = 1/(1 + 2^(-log2(e) x))).
template <int ACT>
__device__ __forceinline__ void n_act2(float &a, float &b) {
    if (ACT == 1) {
        a = a < 0.f ? 0.f : a;
        b = b < 0.f ? 0.f : b;
    } else if (ACT == 2 || ACT == 3) {
        const float k = ACT == 2 ? 2.8853900817779268f : -1.4426950408889634f;
        n_mul2(a, b, k, k);
        a = n_ex2(a);
        b = n_ex2(b);
        n_add2(a, b, 1.f, 1.f);
        a = n_rcp(a);
        b = n_rcp(b);
        if (ACT == 2) n_fma2(a, b, -2.f, 1.f);
    }
}

// Splits 16 values into tf32 hi/lo and stores them at A columns c0.. (hi) and
// 64 + c0.. (lo) of this thread's lane.
__device__ __forceinline__ void n_put_a16(uint32_t lane_a, int c0, const float (&v)[16]) {
    uint32_t h[16], l[16];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        h[e] = tf32_rna(v[e]);
        h[e + 1] = tf32_rna(v[e + 1]);
        float r0, r1;
        n_sub2(v[e], v[e + 1], __uint_as_float(h[e]), __uint_as_float(h[e + 1]), r0, r1);
        l[e] = __float_as_uint(r0);  // left unrounded, as tf32_lo
        l[e + 1] = __float_as_uint(r1);
    }
    tmem_st16u(lane_a + (uint32_t)c0, h);
    tmem_st16u(lane_a + 64u + (uint32_t)c0, l);
}

// Byte offset of layer l's weight chunks in the resident block (hi then lo of
// each 32-wide K-chunk, Np rows of 128 bytes each).
__device__ __forceinline__ uint32_t n_w_off(const TcArgs &p, int l) {
    uint32_t off = 0;
    for (int i = 0; i < l; i++) off += (uint32_t)p.L[i].nch * 2u * (uint32_t)p.L[i].Np * 128u;
    return off;
}

// Layer l of one tile: up to 8 K-steps (K <= 64), three MMAs each, unrolled.
__device__ __forceinline__ void n_issue_layer(uint32_t d, uint32_t a, uint32_t wh, uint32_t np, int ksteps,
                                              uint32_t idesc) {
    const uint32_t lo = (np * 128u) >> 4;  // the lo half of a chunk, in descriptor units
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < ksteps) {
            // chunk j/4 (2*np rows of 128 B), 32 bytes per K-step within it
            const uint32_t bh = wh + (uint32_t)(j >> 2) * ((2u * np * 128u) >> 4) + (uint32_t)((j & 3) * 2);
            umma_tf32_ts(d, a + 64u + 8u * j, bh, idesc, j ? 1u : 0u);
            umma_tf32_ts(d, a + 8u * j, bh + lo, idesc, 1u);
            umma_tf32_ts(d, a + 8u * j, bh, idesc, 1u);
        }
    }
}

// Layer end into the next layer's A: bias, activation, tf32 split, for the
// layer's np (<= 64, a multiple of 16) accumulator columns.  Columns at and
// beyond N hold act(0) and meet zero weight columns in the next layer.
template <int ACT>
__device__ __forceinline__ void n_layer_to_a(uint32_t lane_d, uint32_t lane_a, const float *bias, int np) {
#pragma unroll
    for (int hq = 0; hq < 2; hq++) {  // 32 columns at a time
        if (32 * hq >= np) break;
        uint32_t v[2][16];
        tmem_ld16_nw(lane_d + 32u * hq, v[0]);
        if (32 * hq + 16 < np) tmem_ld16_nw(lane_d + 32u * hq + 16u, v[1]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int c0 = 32 * hq + 16 * q;
            if (c0 >= np) break;
            float y[16];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
                y[e] = __uint_as_float(v[q][e]);
                y[e + 1] = __uint_as_float(v[q][e + 1]);
                n_add2(y[e], y[e + 1], bias[c0 + e], bias[c0 + e + 1]);
                n_act2<ACT>(y[e], y[e + 1]);
            }
            n_put_a16(lane_a, c0, y);
        }
    }
}

// The last tensor-core layer's activations, 16 columns at a time, straight
// into the CUDA-core last layer: o[n] += act(acc[k] + b[k]) W^T[k][n] over the
// zero-padded W^T in shared memory (rows at and beyond np never reached).
template <int ACT, int TNP>
__device__ __forceinline__ void n_layer_tail(uint32_t lane_d, const float *bias, int np, const float *tw,
                                             float (&o)[TNP]) {
#pragma unroll
    for (int n = 0; n < TNP; n++) o[n] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        if (16 * q >= np) break;
        uint32_t v[16];
        tmem_ld16_nw(lane_d + 16u * q, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
            const int k = 16 * q + e;
            float h0 = __uint_as_float(v[e]), h1 = __uint_as_float(v[e + 1]);
            n_add2(h0, h1, bias[k], bias[k + 1]);
            n_act2<ACT>(h0, h1);
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const float h = kk ? h1 : h0;
                const float4 *w = reinterpret_cast<const float4 *>(tw + (k + kk) * kTcTailMaxN);
#pragma unroll
                for (int n4 = 0; n4 < TNP / 4; n4++) {
                    const float4 c = w[n4];
                    n_fma2v(o[4 * n4], o[4 * n4 + 1], h, c.x, c.y);
                    n_fma2v(o[4 * n4 + 2], o[4 * n4 + 3], h, c.z, c.w);
                }
            }
        }
    }
}

// The tail's bias, activation and output row.
template <int TNP, int ACT>
__device__ __forceinline__ void n_tail_out_act(const TcArgs &p, const float (&o)[TNP], const float *tb, long long row) {
#pragma unroll
    for (int n = 0; n < TNP; n++)
        if (n < p.tail_n) p.out[row + (long long)n * p.ld_out] = tc_act<ACT>(o[n] + tb[n]);
}
template <int TNP>
__device__ __forceinline__ void n_tail_out(const TcArgs &p, const float (&o)[TNP], const float *tb, long long row) {
    if (row >= p.n) return;
    switch (p.tail_act) {
        case 1: n_tail_out_act<TNP, 1>(p, o, tb, row); break;
        case 2: n_tail_out_act<TNP, 2>(p, o, tb, row); break;
        case 3: n_tail_out_act<TNP, 3>(p, o, tb, row); break;
        default: n_tail_out_act<TNP, 0>(p, o, tb, row); break;
    }
}

// The last layer on the tensor cores (no CUDA-core tail): its outputs.
template <int ACT>
__device__ __forceinline__ void n_layer_out(const TcArgs &p, uint32_t lane_d, const float *bias, int np, int nout,
                                            long long row) {
    uint32_t v[4][16];
#pragma unroll
    for (int q = 0; q < 4; q++)
        if (16 * q < np) tmem_ld16_nw(lane_d + 16u * q, v[q]);
    tmem_wait_ld();
    if (row >= p.n) return;
#pragma unroll
    for (int q = 0; q < 4; q++)
#pragma unroll
        for (int e = 0; e < 16; e++)
            if (16 * q + e < nout) p.out[row + (long long)(16 * q + e) * p.ld_out] = tc_act<ACT>(__uint_as_float(v[q][e]) + bias[16 * q + e]);
}

// The inputs f = 16q..16q+15 of `row` (zero beyond k0 and past the batch).
__device__ __forceinline__ void n_load_x(const TcArgs &p, int q, int k0, long long row, float (&x)[16]) {
    const bool valid = row < p.n;
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int f = 16 * q + e;
        x[e] = (valid && f < k0) ? __ldg(p.in + (long long)f * p.ld_in + row) : 0.f;
    }
}

// HACT: the activation of every tensor-core layer; TNP: the CUDA-core last
// layer's padded width (8 or 16), 0 when the last layer is on the tensor cores.
template <int HACT, int TNP>
__global__ void __launch_bounds__(kNThreads, 1) mlp_narrow_tc_kernel(const __grid_constant__ TcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *const wsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    float *const sbias = reinterpret_cast<float *>(wsm + kNSmemW);  // [layer][64]
    float *const stw = sbias + kTcMaxLayers * kNMaxN;                // tail W^T [64][16], zero padded
    float *const stb = stw + kNMaxK * kTcTailMaxN;                   // tail bias [16]
    uint64_t *const bars = reinterpret_cast<uint64_t *>(stb + kTcTailMaxN);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kNNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nl = p.nlayers;
    const long long ntiles = (p.n + 127) / 128;

    // biases and the tail's weights (plain loads; every thread)
    for (int i = tid; i < nl * kNMaxN; i += kNThreads) {
        const int l = i / kNMaxN, c = i - l * kNMaxN;
        sbias[i] = c < p.L[l].Np ? p.arena[p.L[l].b_off + c] : 0.f;
    }
    for (int i = tid; i < kNMaxK * kTcTailMaxN; i += kNThreads) {
        const int k = i / kTcTailMaxN, c = i - k * kTcTailMaxN;
        stw[i] = (p.tail_n > 0 && k < p.tail_kp && c < p.tail_np) ? p.arena[p.tail_w_off + (long long)k * p.tail_np + c]
                                                                   : 0.f;
    }
    if (tid < kTcTailMaxN) stb[tid] = (p.tail_n > 0 && tid < p.tail_np) ? p.arena[p.tail_b_off + tid] : 0.f;
    if (tid == 0) {
        mbar_init(bars + kNWReady, 1);
        for (int g = 0; g < 2; g++) {
            mbar_init(bars + kNAFull + g, 128);
            mbar_init(bars + kNDFull + g, 1);
        }
        mbar_init(bars + kNDone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kNTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 8) {
        if (lane == 0) {
            // ---- the weights, then every MMA ----
            uint32_t bytes = 0;
            for (int l = 0; l < nl; l++) bytes += (uint32_t)p.L[l].nch * 2u * (uint32_t)p.L[l].Np * 128u;
            mbar_arrive_expect_tx(bars + kNWReady, bytes);
            for (int l = 0; l < nl; l++) {
                uint8_t *dst = wsm + n_w_off(p, l);
                const uint32_t half = (uint32_t)p.L[l].Np * 128u;
                for (int c = 0; c < p.L[l].nch; c++) {
                    tma_load_2d(dst + c * 2 * half, &p.maps[l], bars + kNWReady, c * 32, 0);
                    tma_load_2d(dst + c * 2 * half + half, &p.maps[l], bars + kNWReady, c * 32, p.L[l].Np);
                }
            }
            bool ok = mbar_wait(bars + kNWReady, 0, p.err, 81);
            const uint32_t wbase = desc_lo(smem_u32(wsm));
            uint32_t acnt0 = 0, acnt1 = 0;
            for (long long k = 0; ok; k++) {
                const long long t0 = blockIdx.x + 2 * k * gridDim.x;
                if (t0 >= ntiles) break;
                const int ng = t0 + gridDim.x < ntiles ? 2 : 1;
                uint32_t woff = 0;
                for (int l = 0; l < nl && ok; l++) {
                    const uint32_t np = (uint32_t)p.L[l].Np, idesc = idesc_tf32((int)np);
                    const int ksteps = (p.L[l].K + 7) / 8;
                    for (int g = 0; g < ng && ok; g++) {
                        const uint32_t ac = g ? acnt1 : acnt0;
                        if (!(ok = mbar_wait(bars + kNAFull + g, ac & 1, p.err, 82, (int)k, l, g))) break;
                        if (g) acnt1++;
                        else acnt0++;
                        tc_fence_after();
                        const uint32_t a = tmem + 256u * g;
                        n_issue_layer(a + 128u, a, wbase + (woff >> 4), np, ksteps, idesc);
                        umma_commit(bars + kNDFull + g);
                    }
                    woff += (uint32_t)p.L[l].nch * 2u * np * 128u;
                }
            }
            umma_commit(bars + kNDone);
            mbar_drain(bars + kNDone, 0);
        }
    } else {
        // ---- tile groups: thread = sample row ----
        const int g = warp >> 2, r = 32 * (warp & 3) + lane;
        const uint32_t lane_a = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 256u * g, lane_d = lane_a + 128u;
        const int k0 = p.L[0].K;
        const bool pre = k0 <= 16;  // the next tile's inputs held in registers while this tile runs
        float xr[16];
        {
            const long long t = blockIdx.x + (long long)g * gridDim.x;
            if (pre && t < ntiles) n_load_x(p, 0, k0, t * 128 + r, xr);
        }
        uint32_t dcnt = 0;
        bool ok = true;
        for (long long k = 0; ok; k++) {
            const long long t = blockIdx.x + (2 * k + g) * gridDim.x;
            if (t >= ntiles) break;
            const long long row = t * 128 + r;
            // layer 0's A: the inputs, zero beyond K (and past the batch)
            if (pre) {
                n_put_a16(lane_a, 0, xr);
                const long long tn = t + 2 * gridDim.x;
                if (tn < ntiles) n_load_x(p, 0, k0, tn * 128 + r, xr);
            } else {
#pragma unroll
                for (int q = 0; q < kNMaxK / 16; q++)
                    if (16 * q < k0) {
                        float x[16];
                        n_load_x(p, q, k0, row, x);
                        n_put_a16(lane_a, 16 * q, x);
                    }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(bars + kNAFull + g);
            for (int l = 0; l < nl; l++) {
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kNDFull + g, dcnt & 1, p.err, 83, (int)k, l));
                dcnt++;
                if (!ok) break;
                tc_fence_after();
                const float *bias = sbias + l * kNMaxN;
                const int np = p.L[l].Np;
                if (l + 1 < nl) {
                    n_layer_to_a<HACT>(lane_d, lane_a, bias, np);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    mbar_arrive(bars + kNAFull + g);
                } else if constexpr (TNP > 0) {
                    float o[TNP];
                    n_layer_tail<HACT, TNP>(lane_d, bias, np, stw, o);
                    n_tail_out<TNP>(p, o, stb, row);
                } else {
                    n_layer_out<HACT>(p, lane_d, bias, np, p.L[l].N, row);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kNTmemCols));
    }
}

// ============================================================================
// mlp_stream_tc_kernel: the same chains with a first layer too long to keep
// (more than 64 inputs, at most 64 outputs; e.g. a CNN's 784-64 head).  That
// layer's inputs and weights are streamed: a producer lane loads, per 32-wide
// K-chunk, the tile's input box {128 samples, 32 features} (the batch is
// sample-fastest, so it lands as rows of 128 samples) into a three-slot ring per
// tile and the weight chunk [Wh | Wl] into a four-slot ring shared by both
// tiles; the tile's threads (thread = sample) split their 32 values into tf32
// hi/lo and store them into one of two 32-column TMEM A slots; the issuer runs
// the chunk's 12 MMAs into one of two 64-column partial buffers, which the
// threads add into fp32 registers (round to nearest: a chain of 25 or more
// truncating accumulations in TMEM would lose accuracy).  Later layers (at most
// 64 wide and 64 deep) keep their weights resident and run as in
// mlp_narrow_tc_kernel, alternating between the two partial buffers.
// Roles (320 threads): warps 0-7 the two tiles, warp 8 lane 0 the MMA issuer,
// warp 9 lane 0 the TMA producer.  Every wait is bounded.
// ============================================================================
constexpr int kSThreads = 320;
constexpr uint32_t kSSmemW = 48 * 1024;      // resident weights of the later layers
constexpr uint32_t kSBSlot = 16384;          // one weight chunk (hi, lo) of <= 64 rows
constexpr int kSBSlots = 4;
constexpr uint32_t kSXSlot = 32 * 128 * 4;   // one input chunk [32 features][128 samples]
constexpr int kSXSlots = 3;

enum {
    kSWReady = 0,                     // the later layers' weights landed
    kSBFull = 1,                      // [4] weight chunk landed (TMA bytes)
    kSBEmpty = kSBFull + kSBSlots,    // [4] both tiles' MMAs done with it (commit)
    kSXFull = kSBEmpty + kSBSlots,    // [2][3] input chunk landed (TMA bytes)
    kSXEmpty = kSXFull + 2 * kSXSlots,  // [2][3] read by the tile's threads (128)
    kSAFull = kSXEmpty + 2 * kSXSlots,  // [2][2] layer-0 A slot written (128)
    kSA1Full = kSAFull + 4,           // [2] a later layer's A written (128)
    kSDFull = kSA1Full + 2,           // [2][2] partial / layer output complete (commit)
    kSDEmpty = kSDFull + 4,           // [2][2] drained (128)
    kSDone = kSDEmpty + 4,
    kSNumBars = kSDone + 1
};

size_t mlp_stream_smem() {
    return 1024 + kSSmemW + kSBSlots * kSBSlot + 2 * kSXSlots * kSXSlot + kNSmemBias + kNSmemTail + 8 * kSNumBars + 16;
}

// The CUDA-core last layer from the layer-0 activations held in registers.
template <int ACT, int TNP>
__device__ __forceinline__ void s_tail_regs(const float (&acc)[64], const float *bias, int np, const float *tw,
                                            float (&o)[TNP]) {
#pragma unroll
    for (int n = 0; n < TNP; n++) o[n] = 0.f;
#pragma unroll
    for (int k = 0; k < 64; k += 2) {
        if (k >= np) break;
        float h0 = acc[k], h1 = acc[k + 1];
        n_add2(h0, h1, bias[k], bias[k + 1]);
        n_act2<ACT>(h0, h1);
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
            const float h = kk ? h1 : h0;
            const float4 *w = reinterpret_cast<const float4 *>(tw + (k + kk) * kTcTailMaxN);
#pragma unroll
            for (int n4 = 0; n4 < TNP / 4; n4++) {
                const float4 c = w[n4];
                n_fma2v(o[4 * n4], o[4 * n4 + 1], h, c.x, c.y);
                n_fma2v(o[4 * n4 + 2], o[4 * n4 + 3], h, c.z, c.w);
            }
        }
    }
}

template <int HACT, int TNP>
__global__ void __launch_bounds__(kSThreads, 1) mlp_stream_tc_kernel(const __grid_constant__ TcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *const wsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const bring = wsm + kSSmemW;
    uint8_t *const xring = bring + kSBSlots * kSBSlot;
    float *const sbias = reinterpret_cast<float *>(xring + 2 * kSXSlots * kSXSlot);  // [layer][64]
    float *const stw = sbias + kTcMaxLayers * kNMaxN;  // tail W^T [64][16], zero padded
    float *const stb = stw + kNMaxK * kTcTailMaxN;     // tail bias [16]
    uint64_t *const bars = reinterpret_cast<uint64_t *>(stb + kTcTailMaxN);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kSNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nl = p.nlayers, nch0 = p.L[0].nch, np0 = p.L[0].Np;
    const long long ntiles = (p.n + 127) / 128;

    for (int i = tid; i < nl * kNMaxN; i += kSThreads) {
        const int l = i / kNMaxN, c = i - l * kNMaxN;
        sbias[i] = c < p.L[l].Np ? p.arena[p.L[l].b_off + c] : 0.f;
    }
    for (int i = tid; i < kNMaxK * kTcTailMaxN; i += kSThreads) {
        const int k = i / kTcTailMaxN, c = i - k * kTcTailMaxN;
        stw[i] = (p.tail_n > 0 && k < p.tail_kp && c < p.tail_np) ? p.arena[p.tail_w_off + (long long)k * p.tail_np + c]
                                                                   : 0.f;
    }
    if (tid < kTcTailMaxN) stb[tid] = (p.tail_n > 0 && tid < p.tail_np) ? p.arena[p.tail_b_off + tid] : 0.f;
    if (tid == 0) {
        mbar_init(bars + kSWReady, 1);
        for (int i = 0; i < kSBSlots; i++) {
            mbar_init(bars + kSBFull + i, 1);
            mbar_init(bars + kSBEmpty + i, 1);
        }
        for (int i = 0; i < 2 * kSXSlots; i++) {
            mbar_init(bars + kSXFull + i, 1);
            mbar_init(bars + kSXEmpty + i, 128);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(bars + kSAFull + i, 128);
            mbar_init(bars + kSDFull + i, 1);
            mbar_init(bars + kSDEmpty + i, 128);
        }
        for (int g = 0; g < 2; g++) mbar_init(bars + kSA1Full + g, 128);
        mbar_init(bars + kSDone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kNTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 9) {
        if (lane == 0) {
            // ---- TMA producer: the later layers' weights once, then per pair of
            // tiles and K-chunk the weight chunk and each tile's input chunk ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.xmap) : "memory");
            uint32_t bytes = 0;
            for (int l = 1; l < nl; l++) bytes += (uint32_t)p.L[l].nch * 2u * (uint32_t)p.L[l].Np * 128u;
            mbar_arrive_expect_tx(bars + kSWReady, bytes);
            {
                uint32_t off = 0;
                for (int l = 1; l < nl; l++) {
                    const uint32_t half = (uint32_t)p.L[l].Np * 128u;
                    for (int c = 0; c < p.L[l].nch; c++) {
                        tma_load_2d(wsm + off + c * 2 * half, &p.maps[l], bars + kSWReady, c * 32, 0);
                        tma_load_2d(wsm + off + c * 2 * half + half, &p.maps[l], bars + kSWReady, c * 32, p.L[l].Np);
                    }
                    off += (uint32_t)p.L[l].nch * 2u * half;
                }
            }
            const uint32_t bhalf = (uint32_t)np0 * 128u;
            uint32_t cb = 0, cx[2] = {0, 0};
            bool ok = true;
            for (long long k = 0; ok; k++) {
                const long long t0 = blockIdx.x + 2 * k * gridDim.x;
                if (t0 >= ntiles) break;
                const int ng = t0 + gridDim.x < ntiles ? 2 : 1;
                for (int c = 0; c < nch0 && ok; c++) {
                    const uint32_t bs = cb % kSBSlots;
                    if (cb >= (uint32_t)kSBSlots &&
                        !(ok = mbar_wait(bars + kSBEmpty + bs, (cb / kSBSlots - 1) & 1, p.err, 91, (int)k, c)))
                        break;
                    mbar_arrive_expect_tx(bars + kSBFull + bs, 2u * bhalf);
                    tma_load_2d(bring + bs * kSBSlot, &p.maps[0], bars + kSBFull + bs, c * 32, 0);
                    tma_load_2d(bring + bs * kSBSlot + bhalf, &p.maps[0], bars + kSBFull + bs, c * 32, np0);
                    cb++;
                    for (int g = 0; g < ng && ok; g++) {
                        const uint32_t xs = cx[g] % kSXSlots, xb = (uint32_t)g * kSXSlots + xs;
                        if (cx[g] >= (uint32_t)kSXSlots &&
                            !(ok = mbar_wait(bars + kSXEmpty + xb, (cx[g] / kSXSlots - 1) & 1, p.err, 92, (int)k, c, g)))
                            break;
                        mbar_arrive_expect_tx(bars + kSXFull + xb, kSXSlot);
                        tma_load_2d(xring + xb * kSXSlot, &p.xmap, bars + kSXFull + xb,
                                    (int)((t0 + (long long)g * gridDim.x) * 128), c * 32);
                        cx[g]++;
                    }
                }
            }
            // copies in flight land before the CTA exits (their consumers waited for
            // every one they needed; after a time-out, some were never consumed)
            for (uint32_t i = cb > (uint32_t)kSBSlots ? cb - kSBSlots : 0; i < cb; i++)
                mbar_drain(bars + kSBFull + i % kSBSlots, (i / kSBSlots) & 1);
            for (int g = 0; g < 2; g++)
                for (uint32_t i = cx[g] > (uint32_t)kSXSlots ? cx[g] - kSXSlots : 0; i < cx[g]; i++)
                    mbar_drain(bars + kSXFull + g * kSXSlots + i % kSXSlots, (i / kSXSlots) & 1);
            mbar_drain(bars + kSWReady, 0);
        }
    } else if (warp == 8) {
        if (lane == 0) {
            // ---- MMA issuer ----
            bool ok = nl <= 1 || mbar_wait(bars + kSWReady, 0, p.err, 93);
            const uint32_t bbase = desc_lo(smem_u32(bring)), wbase = desc_lo(smem_u32(wsm));
            const uint32_t idesc0 = idesc_tf32(np0), blo = ((uint32_t)np0 * 128u) >> 4;
            uint32_t cb = 0, ca[2] = {0, 0}, a1[2] = {0, 0}, cd[2] = {0, 0};
            for (long long k = 0; ok; k++) {
                const long long t0 = blockIdx.x + 2 * k * gridDim.x;
                if (t0 >= ntiles) break;
                const int ng = t0 + gridDim.x < ntiles ? 2 : 1;
                for (int c = 0; c < nch0 && ok; c++) {
                    const uint32_t bs = cb % kSBSlots;
                    if (!(ok = mbar_wait(bars + kSBFull + bs, (cb / kSBSlots) & 1, p.err, 94, (int)k, c))) break;
                    for (int g = 0; g < ng && ok; g++) {
                        const uint32_t as = ca[g] & 1, b = cd[g] & 1, u = cd[g] >> 1;
                        if (!(ok = mbar_wait(bars + kSAFull + 2 * g + as, (ca[g] >> 1) & 1, p.err, 95, (int)k, c, g)))
                            break;
                        if (u > 0 && !(ok = mbar_wait(bars + kSDEmpty + 2 * g + b, (u - 1) & 1, p.err, 96, (int)k, c, g)))
                            break;
                        ca[g]++;
                        tc_fence_after();
                        const uint32_t a = tmem + 256u * g, d = a + 128u + 64u * b;
                        const uint32_t bh = bbase + bs * (kSBSlot >> 4);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            umma_tf32_ts(d, a + 64u + 32u * as + 8u * j, bh + 2u * j, idesc0, j ? 1u : 0u);
                            umma_tf32_ts(d, a + 32u * as + 8u * j, bh + blo + 2u * j, idesc0, 1u);
                            umma_tf32_ts(d, a + 32u * as + 8u * j, bh + 2u * j, idesc0, 1u);
                        }
                        umma_commit(bars + kSDFull + 2 * g + b);
                        cd[g]++;
                    }
                    if (!ok) break;
                    umma_commit(bars + kSBEmpty + bs);
                    cb++;
                }
                uint32_t woff = 0;
                for (int l = 1; l < nl && ok; l++) {
                    const uint32_t np = (uint32_t)p.L[l].Np, idesc = idesc_tf32((int)np);
                    const int ksteps = (p.L[l].K + 7) / 8;
                    for (int g = 0; g < ng && ok; g++) {
                        const uint32_t b = cd[g] & 1, u = cd[g] >> 1;
                        if (!(ok = mbar_wait(bars + kSA1Full + g, a1[g] & 1, p.err, 97, (int)k, l, g))) break;
                        if (u > 0 && !(ok = mbar_wait(bars + kSDEmpty + 2 * g + b, (u - 1) & 1, p.err, 96, (int)k, l, g)))
                            break;
                        a1[g]++;
                        tc_fence_after();
                        const uint32_t a = tmem + 256u * g;
                        n_issue_layer(a + 128u + 64u * b, a, wbase + (woff >> 4), np, ksteps, idesc);
                        umma_commit(bars + kSDFull + 2 * g + b);
                        cd[g]++;
                    }
                    woff += (uint32_t)p.L[l].nch * 2u * np * 128u;
                }
            }
            umma_commit(bars + kSDone);
            mbar_drain(bars + kSDone, 0);
        }
    } else {
        // ---- tile groups: thread = sample row ----
        const int g = warp >> 2, r = 32 * (warp & 3) + lane;
        const uint32_t lane_a = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 256u * g;
        uint32_t cx = 0, ca = 0, cd = 0;
        bool ok = true;
        // layer-0 chunk into A slot ca & 1: this thread's 32 values, split
        auto stage = [&](long long k_, int c_) -> bool {
            const uint32_t xs = cx % kSXSlots, xb = (uint32_t)g * kSXSlots + xs;
            const bool w = __all_sync(0xffffffffu,
                                      mbar_wait(bars + kSXFull + xb, (cx / kSXSlots) & 1, p.err, 98, (int)k_, c_, g));
            if (!w) return false;
            const float *src = reinterpret_cast<const float *>(xring + xb * kSXSlot) + r;
            float v0[16], v1[16];
#pragma unroll
            for (int e = 0; e < 16; e++) {
                v0[e] = src[e * 128];
                v1[e] = src[(16 + e) * 128];
            }
            mbar_arrive(bars + kSXEmpty + xb);
            cx++;
            // slot s: hi columns 32s.., lo 64 + 32s..
            n_put_a16(lane_a, 32 * (int)(ca & 1), v0);
            n_put_a16(lane_a, 32 * (int)(ca & 1) + 16, v1);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(bars + kSAFull + 2 * g + (ca & 1));
            ca++;
            return true;
        };
        for (long long k = 0; ok; k++) {
            const long long t = blockIdx.x + (2 * k + g) * gridDim.x;
            if (t >= ntiles) break;
            const long long row = t * 128 + r;
            float acc[64];
#pragma unroll
            for (int e = 0; e < 64; e++) acc[e] = 0.f;
            ok = stage(k, 0) && (nch0 < 2 || stage(k, 1));
            for (int c = 0; c < nch0 && ok; c++) {
                const uint32_t b = cd & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kSDFull + 2 * g + b, (cd >> 1) & 1, p.err, 99, (int)k, c));
                if (!ok) break;
                tc_fence_after();
                const uint32_t ld = lane_a + 128u + 64u * b;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    if (16 * q >= np0) break;
                    uint32_t v[16];
                    tmem_ld16_nw(ld + 16u * q, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; e += 2) add2(acc[16 * q + e], acc[16 * q + e + 1], v[e], v[e + 1]);
                }
                tc_fence_before();
                mbar_arrive(bars + kSDEmpty + 2 * g + b);
                cd++;
                if (c + 2 < nch0) ok = stage(k, c + 2);
            }
            if (!ok) break;
            const float *bias0 = sbias;
            if (nl == 1) {
                if constexpr (TNP > 0) {
                    float o[TNP];
                    s_tail_regs<HACT, TNP>(acc, bias0, np0, stw, o);
                    n_tail_out<TNP>(p, o, stb, row);
                } else if (row < p.n) {
#pragma unroll
                    for (int e = 0; e < 64; e += 2) {
                        if (e >= p.L[0].N) break;
                        float h0 = acc[e], h1 = acc[e + 1];
                        n_add2(h0, h1, bias0[e], bias0[e + 1]);
                        n_act2<HACT>(h0, h1);
                        p.out[row + (long long)e * p.ld_out] = h0;
                        if (e + 1 < p.L[0].N) p.out[row + (long long)(e + 1) * p.ld_out] = h1;
                    }
                }
                continue;
            }
            // layer 0's activations as layer 1's A (hi 0..63, lo 64..127)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                if (16 * q >= np0) break;
                float y[16];
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                    y[e] = acc[16 * q + e];
                    y[e + 1] = acc[16 * q + e + 1];
                    n_add2(y[e], y[e + 1], bias0[16 * q + e], bias0[16 * q + e + 1]);
                    n_act2<HACT>(y[e], y[e + 1]);
                }
                n_put_a16(lane_a, 16 * q, y);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(bars + kSA1Full + g);
            for (int l = 1; l < nl && ok; l++) {
                const uint32_t b = cd & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kSDFull + 2 * g + b, (cd >> 1) & 1, p.err, 99, (int)k, l));
                if (!ok) break;
                tc_fence_after();
                const uint32_t lane_d = lane_a + 128u + 64u * b;
                const float *bias = sbias + l * kNMaxN;
                const int np = p.L[l].Np;
                if (l + 1 < nl) {
                    n_layer_to_a<HACT>(lane_d, lane_a, bias, np);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    mbar_arrive(bars + kSDEmpty + 2 * g + b);
                    mbar_arrive(bars + kSA1Full + g);
                } else {
                    if constexpr (TNP > 0) {
                        float o[TNP];
                        n_layer_tail<HACT, TNP>(lane_d, bias, np, stw, o);
                        n_tail_out<TNP>(p, o, stb, row);
                    } else {
                        n_layer_out<HACT>(p, lane_d, bias, np, p.L[l].N, row);
                    }
                    tc_fence_before();
                    mbar_arrive(bars + kSDEmpty + 2 * g + b);
                }
                cd++;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kNTmemCols));
    }
}

}  // namespace

bool mlp_narrow_fits(const TcArgs &a) {
    if (a.nlayers < 1 || a.nlayers > kTcMaxLayers) return false;
    uint32_t bytes = 0;
    for (int l = 0; l < a.nlayers; l++) {
        const TcLayer &L = a.L[l];
        if (L.act != a.L[0].act || L.act < 0 || L.act > 3) return false;  // one activation for every layer
        if (L.Np > kNMaxN || L.Np % 16 || L.K > kNMaxK || L.K < 1 || L.nch < 1 || L.nch > 2) return false;
        if (l > 0 && L.K > a.L[l - 1].Np) return false;
        bytes += (uint32_t)L.nch * 2u * (uint32_t)L.Np * 128u;
    }
    if (bytes > kNSmemW) return false;
    if (a.tail_n > 0 && (a.tail_np > kTcTailMaxN || a.tail_kp > kNMaxK || a.tail_k > a.L[a.nlayers - 1].Np))
        return false;
    return true;
}

#define ROSENNA_NARROW_VARIANTS(X) X(0, 0) X(1, 0) X(2, 0) X(3, 0) X(0, 8) X(1, 8) X(2, 8) X(3, 8) X(0, 16) X(1, 16) X(2, 16) X(3, 16)

cudaError_t mlp_narrow_configure() {
    cudaError_t e = cudaSuccess;
#define ROSENNA_NARROW_CFG(A, T)                                                                          \
    if (e == cudaSuccess)                                                                                 \
        e = cudaFuncSetAttribute(mlp_narrow_tc_kernel<A, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)mlp_narrow_smem());
    ROSENNA_NARROW_VARIANTS(ROSENNA_NARROW_CFG)
#undef ROSENNA_NARROW_CFG
    return e;
}

cudaError_t launch_mlp_narrow(const TcArgs &a, int num_sms, cudaStream_t st) {
    if (!mlp_narrow_fits(a)) return cudaErrorInvalidConfiguration;
    const long long tiles = (a.n + 127) / 128, pairs = (tiles + 1) / 2;
    const int grid = (int)(pairs < num_sms ? pairs : num_sms);
    if (grid <= 0) return cudaSuccess;
    const int act = a.L[0].act, tnp = a.tail_n > 0 ? (a.tail_np <= 8 ? 8 : 16) : 0;
    bool launched = false;
#define ROSENNA_NARROW_LAUNCH(A, T)                                                  \
    if (!launched && act == A && tnp == T) {                                        \
        mlp_narrow_tc_kernel<A, T><<<grid, kNThreads, mlp_narrow_smem(), st>>>(a);  \
        launched = true;                                                             \
    }
    ROSENNA_NARROW_VARIANTS(ROSENNA_NARROW_LAUNCH)
#undef ROSENNA_NARROW_LAUNCH
    if (!launched) return cudaErrorInvalidConfiguration;
    return cudaGetLastError();
}

bool mlp_stream_fits(const TcArgs &a) {
    if (a.nlayers < 1 || a.nlayers > kTcMaxLayers) return false;
    const TcLayer &L0 = a.L[0];
    if (L0.K <= kNMaxK || L0.Np > kNMaxN || L0.Np % 16 || L0.nch < 3 || L0.act < 0 || L0.act > 3) return false;
    uint32_t bytes = 0;
    for (int l = 1; l < a.nlayers; l++) {
        const TcLayer &L = a.L[l];
        if (L.act != L0.act) return false;  // one activation for every layer
        if (L.Np > kNMaxN || L.Np % 16 || L.K > kNMaxK || L.K < 1 || L.nch < 1 || L.nch > 2 || L.K > a.L[l - 1].Np)
            return false;
        bytes += (uint32_t)L.nch * 2u * (uint32_t)L.Np * 128u;
    }
    if (bytes > kSSmemW) return false;
    if (a.tail_n > 0 && (a.tail_np > kTcTailMaxN || a.tail_kp > kNMaxK || a.tail_k > a.L[a.nlayers - 1].Np))
        return false;
    return true;
}

cudaError_t mlp_stream_configure() {
    cudaError_t e = cudaSuccess;
#define ROSENNA_STREAM_CFG(A, T)                                                                          \
    if (e == cudaSuccess)                                                                                 \
        e = cudaFuncSetAttribute(mlp_stream_tc_kernel<A, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)mlp_stream_smem());
    ROSENNA_NARROW_VARIANTS(ROSENNA_STREAM_CFG)
#undef ROSENNA_STREAM_CFG
    return e;
}

cudaError_t launch_mlp_stream(const TcArgs &a, int num_sms, cudaStream_t st) {
    if (!mlp_stream_fits(a)) return cudaErrorInvalidConfiguration;
    // the input is read through a tensor map: 16-byte aligned base and sample pitch
    if ((reinterpret_cast<uintptr_t>(a.in) & 15) != 0 || (a.ld_in & 3) != 0 || a.ld_in <= 0) return cudaErrorNotSupported;
    const long long tiles = (a.n + 127) / 128, pairs = (tiles + 1) / 2;
    const int grid = (int)(pairs < num_sms ? pairs : num_sms);
    if (grid <= 0) return cudaSuccess;
    TcArgs b = a;
    const cuuint64_t dims[2] = {(cuuint64_t)a.n, (cuuint64_t)a.L[0].K};
    const cuuint64_t strides[1] = {(cuuint64_t)a.ld_in * sizeof(float)};
    const cuuint32_t box[2] = {128, 32};
    const char *why = nullptr;
    if (!tc_encode_f32_map(&b.xmap, 2, a.in, dims, strides, box, &why, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorNotSupported;
    const int act = a.L[0].act, tnp = a.tail_n > 0 ? (a.tail_np <= 8 ? 8 : 16) : 0;
    bool launched = false;
#define ROSENNA_STREAM_LAUNCH(A, T)                                                  \
    if (!launched && act == A && tnp == T) {                                        \
        mlp_stream_tc_kernel<A, T><<<grid, kSThreads, mlp_stream_smem(), st>>>(b);  \
        launched = true;                                                             \
    }
    ROSENNA_NARROW_VARIANTS(ROSENNA_STREAM_LAUNCH)
#undef ROSENNA_STREAM_LAUNCH
    if (!launched) return cudaErrorInvalidConfiguration;
    return cudaGetLastError();
}

}  // namespace rosenna
