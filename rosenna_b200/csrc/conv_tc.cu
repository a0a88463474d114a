// Convolution as an implicit GEMM on the tensor cores (tcgen05, 3xTF32), fused
// with its ReLU and the following 2x2 pool (fLibrary/layers.f90 conv :183-233,
// relu4d activation_funcs.f90:43-52, max_pool/avgpool :236-310).
//
// Shapes: 3x3 kernel, stride 1, symmetric zero padding, at most 8 input and 16
// output channels, a k=2 s=2 pool without padding over an even conv output.
// One CTA per SM, persistent over tiles of 128 samples (UMMA M = 128: TMEM
// lane = sample row).  A tile's work is its pooled windows; a window's four
// conv pixels read a 4x4 patch of input positions.  The patch is staged as
// four K-chunks (one per patch row) of 4 positions x 8 channels = 32 fp32:
// one 128-byte swizzled K-major row per sample, split into tf32 hi and lo
// parts.  Because a position's 8 channels are exactly one K-step of kind::tf32
// (K = 8), any position of the patch is an A operand: the chunk's descriptor
// advanced by 32 bytes per patch column.  Two ways to multiply (`mode`):
//   0 (per tap):  D[pixel] += A[position(pixel, tap)] x W[tap]^T for the 9
//                 taps of each of the 4 pixels: N = 16 (output channels),
//                 9 K-steps per pixel, no zero products;
//   1 (window):   D[window] += A[patch row] x T[patch row]^T, where T is the
//                 window's weights laid out over its 4x4 patch (row n =
//                 pixel*16 + oc, zero where a position is outside the pixel's
//                 3x3 taps): N = 64, 4 K-chunks, 44 % of the products zero.
// Both accumulate each product as Al*Wh + Ah*Wl first and Ah*Wh last, the
// accumulator starting at zero (bias added in the epilogue).  D (4 pixels x 16
// channels = 64 TMEM columns) is double-buffered over windows.
//
// Roles (288 threads): warps 0-7 stage (warpgroup g: patch columns 2g, 2g+1 of
// each chunk) and drain (warpgroup g: output channels 8g..8g+7: bias, ReLU,
// pool, store); warp 8 lane 0 issues the MMAs.  Every wait is bounded; a
// time-out records where in `err`, every role finishes, TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "conv_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kCtR = 5;                          // A ring slots (patch-row chunks)
constexpr uint32_t kCtATile = 128 * 128;         // one A chunk, hi or lo: 128 rows x 128 B
constexpr uint32_t kCtSlot = 2 * kCtATile;       // hi + lo
constexpr uint32_t kCtSmemA = kCtR * kCtSlot;
constexpr uint32_t kCtBBytes = kConvTcBFloats * 4;  // the larger (window) B image
constexpr uint32_t kCtThreads = 288;
constexpr uint32_t kCtTmemCols = 128;            // two D buffers of 64 columns

size_t conv_tc_smem() { return 1024 + kCtSmemA + kCtBBytes + 64 + 256; }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

struct CtPos {
    int t, qy, qx;  // tile and pooled window of a global window index
};

__device__ __forceinline__ CtPos ct_window(const ConvTcArgs &p, long long j) {
    const int W = p.Hq * p.Wq;
    const long long tw = j / W;  // this CTA's tile number (0, 1, ...)
    const int w = (int)(j - tw * W);
    CtPos c;
    c.t = (int)(blockIdx.x + tw * gridDim.x);
    c.qy = w / p.Wq;
    c.qx = w - c.qy * p.Wq;
    return c;
}

// Stages this thread's half (patch columns 2g, 2g+1) of patch row pr of window
// `wp` into ring slot s: 16 values of sample row r, split into tf32 hi and lo.
__device__ __forceinline__ void ct_stage(const ConvTcArgs &p, uint8_t *a0, int s, int r, int g, const CtPos &wp,
                                         int pr) {
    const long long row = (long long)wp.t * 128 + r;
    const bool valid = row < p.n;
    const int iy = 2 * wp.qy - p.pad + pr;
    float v[16];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int ix = 2 * wp.qx - p.pad + 2 * g + h;
        const bool inside = valid && iy >= 0 && iy < p.Hin && ix >= 0 && ix < p.Win;
        const float *src = p.in + (long long)p.C * (iy + (long long)p.Hin * ix) * p.ld_in + row;
#pragma unroll
        for (int c = 0; c < 8; c++) v[8 * h + c] = (inside && c < p.C) ? __ldg(src + (long long)c * p.ld_in) : 0.f;
    }
    uint8_t *ahi = a0 + (uint32_t)s * kCtSlot;
    put_a16(ahi, ahi + kCtATile, r, 16 * g, v);
}

// Bias, ReLU and the 2x2 pool of this thread's 8 output channels for window
// `wp` from D buffer d (lane_base already holds the warp's lane offset).
__device__ __forceinline__ void ct_drain(const ConvTcArgs &p, const float *sbias, uint32_t dcol, int r, int g,
                                         const CtPos &wp) {
    uint32_t x[4][8];
#pragma unroll
    for (int px = 0; px < 4; px++) tmem_ld8(dcol + (uint32_t)(16 * px + 8 * g), x[px]);
    tmem_wait_ld();
    const long long row = (long long)wp.t * 128 + r;
    if (row >= p.n) return;
    float *o = p.out + (long long)(wp.qy * p.so_h + wp.qx * p.so_w) * p.ld_out + row;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int oc = 8 * g + e;
        const float b = sbias[oc];
        float y[4];
#pragma unroll
        for (int px = 0; px < 4; px++) {
            y[px] = __uint_as_float(x[px][e]) + b;
            if (p.relu) y[px] = y[px] < 0.f ? 0.f : y[px];
        }
        const float v = p.pool == 1 ? fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3])) : ((y[0] + y[1]) + (y[2] + y[3])) * 0.25f;
        if (oc < p.OC) o[(long long)oc * p.so_c * p.ld_out] = v;
    }
}

// MMA issue of mode 0 for conv pixel (a, b) of the window: 9 taps x 3 terms
// into D columns 16*(2a+b).., A from the ring slots of patch rows a+dy.
__device__ __forceinline__ void ct_issue_pixel(const uint32_t (&aslot)[4], uint32_t bs, uint32_t d, int a, int b) {
    const uint32_t idesc = idesc_tf32(16);
    const uint32_t dd = d + (uint32_t)(16 * (2 * a + b));
    // small terms first (Al*Wh, Ah*Wl), then Ah*Wh
#pragma unroll
    for (int t = 0; t < 9; t++) {
        const int dy = t / 3, dx = t - 3 * (t / 3);
        const uint32_t ah = desc_lo(aslot[a + dy]) + (uint32_t)(((b + dx) * 32) >> 4);
        const uint32_t al = ah + (kCtATile >> 4);
        // B image of mode 0: chunk c = t/4 holds taps 4c..4c+3, hi [16 x 128 B] then lo
        const uint32_t bh = desc_lo(bs + (uint32_t)(t >> 2) * 4096u) + (uint32_t)(((t & 3) * 32) >> 4);
        const uint32_t bl = bh + (2048u >> 4);
        umma_tf32_lo(dd, al, bh, idesc, t > 0 ? 1u : 0u);
        umma_tf32_lo(dd, ah, bl, idesc, 1u);
    }
#pragma unroll
    for (int t = 0; t < 9; t++) {
        const int dy = t / 3, dx = t - 3 * (t / 3);
        const uint32_t ah = desc_lo(aslot[a + dy]) + (uint32_t)(((b + dx) * 32) >> 4);
        const uint32_t bh = desc_lo(bs + (uint32_t)(t >> 2) * 4096u) + (uint32_t)(((t & 3) * 32) >> 4);
        umma_tf32_lo(dd, ah, bh, idesc, 1u);
    }
}

// MMA issue of mode 1 for patch row pr: 4 K-steps x 3 terms, N = 64.
__device__ __forceinline__ void ct_issue_row(uint32_t aslot, uint32_t bs, uint32_t d, int pr) {
    const uint32_t idesc = idesc_tf32(64);
    const uint32_t ah0 = desc_lo(aslot), al0 = ah0 + (kCtATile >> 4);
    // B image of mode 1: chunk pr holds hi [64 x 128 B] then lo
    const uint32_t bh0 = desc_lo(bs + (uint32_t)pr * 16384u), bl0 = bh0 + (8192u >> 4);
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, al0 + adv, bh0 + adv, idesc, (pr > 0 || kk > 0) ? 1u : 0u);
        umma_tf32_lo(d, ah0 + adv, bl0 + adv, idesc, 1u);
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, ah0 + adv, bh0 + adv, idesc, 1u);
    }
}

__global__ void __launch_bounds__(kCtThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const a0 = base;
    uint8_t *const b0 = base + kCtSmemA;
    float *const sbias = reinterpret_cast<float *>(base + kCtSmemA + kCtBBytes);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kCtSmemA + kCtBBytes + 64);
    uint64_t *const a_full = bars, *const a_empty = bars + kCtR;
    uint64_t *const d_full = bars + 2 * kCtR, *const d_empty = bars + 2 * kCtR + 2;
    uint64_t *const mma_done = bars + 2 * kCtR + 4;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kCtR + 6);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntiles = (int)((p.n + 127) / 128);
    const long long my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const long long nwin = my_tiles * p.Hq * p.Wq;

    // the B image (pre-swizzled on the host) and the bias
    const uint32_t bfloats = p.mode == 0 ? kConvTcBFloatsTap : kConvTcBFloats;
    for (uint32_t i = tid; i < bfloats / 4; i += kCtThreads)
        reinterpret_cast<float4 *>(b0)[i] = reinterpret_cast<const float4 *>(p.arena + p.bt_off)[i];
    if (tid < 16) sbias[tid] = tid < p.OC ? p.arena[p.b_off + tid] : 0.f;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (tid == 0) {
        for (int s = 0; s < kCtR; s++) {
            mbar_init(&a_full[s], 256);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&d_full[s], 1);
            mbar_init(&d_empty[s], 256);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCtTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 8) {
        if (lane == 0) {
            // ---- MMA issuer ----
            const uint32_t a_s = smem_u32(a0), b_s = smem_u32(b0);
            bool ok = true;
            for (long long j = 0; j < nwin && ok; j++) {
                const uint32_t d = tmem + (uint32_t)((j & 1) * 64);
                ok = mbar_wait(&d_empty[j & 1], (uint32_t)(((j >> 1) & 1) ^ 1), p.err, 11, (int)j, 0, 0, 2);
                uint32_t aslot[4];
                for (int pr = 0; pr < 4 && ok; pr++) {
                    const long long q = 4 * j + pr;
                    aslot[pr] = a_s + (uint32_t)(q % kCtR) * kCtSlot;
                    if (p.mode == 1 || pr < 3) {
                        ok = mbar_wait(&a_full[q % kCtR], (uint32_t)((q / kCtR) & 1), p.err, 12, (int)j, pr, 0, 2);
                        if (!ok) break;
                    }
                    tc_fence_after();
                    if (p.mode == 1) {
                        ct_issue_row(aslot[pr], b_s, d, pr);
                        umma_commit(&a_empty[q % kCtR]);
                    } else if (pr == 2) {  // pixel row 0 reads patch rows 0..2
                        ct_issue_pixel(aslot, b_s, d, 0, 0);
                        ct_issue_pixel(aslot, b_s, d, 0, 1);
                        umma_commit(&a_empty[(4 * j) % kCtR]);
                    } else if (pr == 3) {  // pixel row 1 reads patch rows 1..3
                        ok = mbar_wait(&a_full[q % kCtR], (uint32_t)((q / kCtR) & 1), p.err, 12, (int)j, pr, 0, 2);
                        if (!ok) break;
                        tc_fence_after();
                        ct_issue_pixel(aslot, b_s, d, 1, 0);
                        ct_issue_pixel(aslot, b_s, d, 1, 1);
                        for (int k = 1; k < 4; k++) umma_commit(&a_empty[(4 * j + k) % kCtR]);
                    }
                }
                if (ok) umma_commit(&d_full[j & 1]);
            }
            // nothing may be in flight when TMEM is freed
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, p.err, 0);
        }
    } else {
        // ---- stagers / drainers: warpgroup g, sample row r ----
        const int g = warp >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const int slot = (lane == 0 && quad == 0) ? 3 + g : 0;
        bool ok = true;
        CtPos prev{0, 0, 0};
        for (long long j = 0; j <= nwin && ok; j++) {
            if (j < nwin) {
                const CtPos wp = ct_window(p, j);
                for (int pr = 0; pr < 4 && ok; pr++) {
                    const long long q = 4 * j + pr;
                    const int s = (int)(q % kCtR);
                    if (q >= kCtR) {
                        ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[s], (uint32_t)(((q / kCtR) - 1) & 1), p.err, 13,
                                                               (int)j, pr, 0, slot));
                        if (!ok) break;
                    }
                    ct_stage(p, a0, s, r, g, wp, pr);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_before();
                    mbar_arrive(&a_full[s]);
                }
                if (!ok) break;
            }
            if (j > 0) {
                const long long jd = j - 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&d_full[jd & 1], (uint32_t)((jd >> 1) & 1), p.err, 14, (int)jd, 0, 0, slot));
                if (!ok) break;
                tc_fence_after();
                ct_drain(p, sbias, lane_base + (uint32_t)((jd & 1) * 64), r, g, prev);
                tc_fence_before();
                mbar_arrive(&d_empty[jd & 1]);
            }
            if (j < nwin) prev = ct_window(p, j);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCtTmemCols));
    }
}

}  // namespace

bool conv_tc_shape_ok(int KS, int str_h, int str_w, int pad_h, int pad_w, int C, int OC, int pool, int pk, int pstr_h,
                      int pstr_w, int ppad_h, int ppad_w, int Ho, int Wo) {
    return KS == 3 && str_h == 1 && str_w == 1 && pad_h == pad_w && pad_h >= 0 && pad_h <= 2 && C >= 1 && C <= 8 &&
           OC >= 1 && OC <= 16 && pool != 0 && pk == 2 && pstr_h == 2 && pstr_w == 2 && ppad_h == 0 && ppad_w == 0 &&
           Ho % 2 == 0 && Wo % 2 == 0 && Ho >= 2 && Wo >= 2;
}

// The B images, as 128-byte-swizzled K-major rows (row r of an 8-row atom holds
// 16-byte chunk k at position k ^ (r & 7)) so the kernel copies them linearly.
static void put_swizzled(float *img, int row, int k, float v) {
    const int atom = row >> 3, r = row & 7, chunk = k >> 2, e = k & 3;
    img[atom * 256 + r * 32 + ((chunk ^ r) << 2) + e] = v;
}

static float tf32_hi(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u = (u + 0x1000u) & 0xFFFFE000u;
    float h;
    std::memcpy(&h, &u, 4);
    return h;
}

void conv_tc_pack(const float *w, int OC, int C, int mode, float *img) {
    // w: [oc][ic][kh][kw] (3x3)
    auto W = [&](int oc, int ic, int kh, int kw) {
        return (oc < OC && ic < C) ? w[(((size_t)oc * C + ic) * 3 + kh) * 3 + kw] : 0.f;
    };
    if (mode == 0) {
        // 3 chunks (taps 4c..4c+3; tap t = 3*kh + kw); each hi [16 rows] then lo
        for (int i = 0; i < kConvTcBFloatsTap; i++) img[i] = 0.f;
        for (int c = 0; c < 3; c++)
            for (int oc = 0; oc < 16; oc++)
                for (int kk = 0; kk < 4; kk++) {
                    const int t = 4 * c + kk;
                    if (t >= 9) continue;
                    for (int ic = 0; ic < 8; ic++) {
                        const float x = W(oc, ic, t / 3, t % 3), h = tf32_hi(x), l = tf32_hi(x - h);
                        put_swizzled(img + c * 1024, oc, 8 * kk + ic, h);
                        put_swizzled(img + c * 1024 + 512, oc, 8 * kk + ic, l);
                    }
                }
        return;
    }
    // 4 chunks (patch rows pr); row n = pixel*16 + oc, K = patch column*8 + ic
    for (int i = 0; i < kConvTcBFloats; i++) img[i] = 0.f;
    for (int pr = 0; pr < 4; pr++)
        for (int px = 0; px < 4; px++)
            for (int oc = 0; oc < 16; oc++)
                for (int pc = 0; pc < 4; pc++)
                    for (int ic = 0; ic < 8; ic++) {
                        const int a = px >> 1, b = px & 1, kh = pr - a, kw = pc - b;
                        const float x = (kh >= 0 && kh < 3 && kw >= 0 && kw < 3) ? W(oc, ic, kh, kw) : 0.f;
                        const float h = tf32_hi(x), l = tf32_hi(x - h);
                        put_swizzled(img + pr * 4096, px * 16 + oc, 8 * pc + ic, h);
                        put_swizzled(img + pr * 4096 + 2048, px * 16 + oc, 8 * pc + ic, l);
                    }
}

cudaError_t conv_tc_configure() {
    return cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)conv_tc_smem());
}

cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + 127) / 128;
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    conv_tc_kernel<<<grid, kCtThreads, conv_tc_smem(), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna
