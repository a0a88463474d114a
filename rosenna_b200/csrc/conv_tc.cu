// Convolution as an implicit GEMM on the tensor cores (tcgen05, 3xTF32), fused
// with its ReLU and the following 2x2 pool (fLibrary/layers.f90 conv :183-233,
// relu4d activation_funcs.f90:43-52, max_pool/avgpool :236-310).
//
// Shapes: 3x3 kernel, stride 1, symmetric zero padding, 1 to 8 input and up to
// 16 output channels, a k=2 s=2 pool without padding over an even conv output.
// One CTA per SM, persistent over tiles of 128 samples (UMMA M = 128: TMEM lane
// = sample row).  A tile's work is a sequence of blocks of pooled windows: one
// window (16 output channels) or two stacked vertically (8 output channels).
// A block's conv pixels read a patch of input positions (4x4 for one window,
// 6x4 for two), and its product is one GEMM per sample row:
//     D[pixel*OCp + oc] = sum_k A[k] * T[pixel*OCp + oc][k]
// where A is the patch flattened as k = position*Cp + channel (Cp = 8
// channels per position, or 1 for a single-channel input, so one K-step of
// kind::tf32 -- 8 elements -- is one position's channels or 8 positions) and T
// is the conv weights laid out over the patch: zero where a position is not
// one of the pixel's 3x3 taps.  N = 4 pixels x windows x OCp = 64 always: an
// M = 128 MMA takes the same ~65 cycles for every N up to 128 (measured), so
// the zero products of T cost less than separate dense per-tap MMAs of N = 16
// would.  A is staged per 32-wide K-chunk (128-byte swizzled K-major rows,
// tf32 hi and lo parts); T is the B operand, resident in shared memory for the
// whole kernel.  Each chunk is Al*Th + Ah*Tl (4 K-steps each) then Ah*Th; D
// starts at zero (bias in the epilogue) and is double-buffered over blocks.
//
// Roles (288 threads): warps 0-7 stage (warpgroup g: K elements 16g..16g+15 of
// each chunk) and drain (warpgroup g: one window's 8 output channels: bias,
// ReLU, pool, store); warp 8 lane 0 issues the MMAs.  Every wait is bounded; a
// time-out records where in `err`, every role finishes, TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "conv_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kCtR = 5;                          // A ring slots (K-chunks)
constexpr uint32_t kCtATile = 128 * 128;         // one A chunk, hi or lo: 128 rows x 128 B
constexpr uint32_t kCtSlot = 2 * kCtATile;       // hi + lo
constexpr uint32_t kCtSmemA = kCtR * kCtSlot;
constexpr uint32_t kCtBBytes = kConvTcBFloats * 4;
constexpr uint32_t kCtThreads = 288;
constexpr uint32_t kCtTmemCols = 128;            // two D buffers of 64 columns
constexpr uint32_t kCtBChunk = 2 * 64 * 128;     // one B chunk: hi then lo, 64 rows x 128 B each

size_t conv_tc_smem() { return 1024 + kCtSmemA + kCtBBytes + 64 + 256; }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

struct CtBlock {
    int t, qy, qx;  // tile, and the pooled window at the block's top
};

__device__ __forceinline__ CtBlock ct_block(const ConvTcArgs &p, long long j) {
    const int per_col = p.Hq / p.bwin, nb = per_col * p.Wq;
    const long long tb = j / nb;  // this CTA's tile number (0, 1, ...)
    const int b = (int)(j - tb * nb);
    CtBlock c;
    c.t = (int)(blockIdx.x + tb * gridDim.x);
    c.qx = b / per_col;
    c.qy = (b - c.qx * per_col) * p.bwin;
    return c;
}

// Loads this thread's half (K elements 16g..16g+15) of chunk c of block `bp`
// for sample row r.  CP = 8: the chunk is patch row c (4 positions x 8
// channels), the half its positions 2g, 2g+1; CP = 1: the chunk is patch rows
// 8c..8c+7 (32 single-channel positions), the half rows 8c+4g..8c+4g+3.
template <int CP, int BWIN>
__device__ __forceinline__ void ct_load(const ConvTcArgs &p, int r, int g, const CtBlock &bp, int c, float (&v)[16]) {
    constexpr int PH = 2 * BWIN + 2;  // patch rows (4 columns)
    const long long row = (long long)bp.t * 128 + r;
    const bool valid = row < p.n;
    const int y0 = 2 * bp.qy - p.pad, x0 = 2 * bp.qx - p.pad;
    if constexpr (CP == 8) {
        const int iy = y0 + c;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int ix = x0 + 2 * g + h;
            const bool inside = valid && iy >= 0 && iy < p.Hin && ix >= 0 && ix < p.Win;
            const float *src = p.in + (long long)p.C * (iy + (long long)p.Hin * ix) * p.ld_in + row;
#pragma unroll
            for (int ch = 0; ch < 8; ch++) v[8 * h + ch] = (inside && ch < p.C) ? __ldg(src + (long long)ch * p.ld_in) : 0.f;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const int py = 8 * c + 4 * g + (e >> 2), ix = x0 + (e & 3), iy = y0 + py;
            const bool inside = valid && py < PH && iy >= 0 && iy < p.Hin && ix >= 0 && ix < p.Win;
            v[e] = inside ? __ldg(p.in + (iy + (long long)p.Hin * ix) * p.ld_in + row) : 0.f;
        }
    }
}

// Bias, ReLU and the 2x2 pool of this thread's item (g): window w, output
// channels oc0..oc0+7, from D buffer columns (w*4 + pixel)*OCp + oc.
__device__ __forceinline__ void ct_drain(const ConvTcArgs &p, const float *sbias, uint32_t dcol, int r, int g,
                                         const CtBlock &bp) {
    const int ocp = 16 / p.bwin;  // 16 (one window) or 8 (two)
    const int w = p.bwin == 2 ? g : 0, oc0 = p.bwin == 2 ? 0 : 8 * g;
    uint32_t x[4][8];
#pragma unroll
    for (int px = 0; px < 4; px++) tmem_ld8(dcol + (uint32_t)((w * 4 + px) * ocp + oc0), x[px]);
    tmem_wait_ld();
    const long long row = (long long)bp.t * 128 + r;
    if (row >= p.n) return;
    float *o = p.out + (long long)((bp.qy + w) * p.so_h + bp.qx * p.so_w) * p.ld_out + row;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int oc = oc0 + e;
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

// One K-chunk: 4 K-steps x 3 terms into D (N = 64).
__device__ __forceinline__ void ct_issue_chunk(uint32_t aslot, uint32_t bchunk, uint32_t d, bool first) {
    const uint32_t idesc = idesc_tf32(64);
    const uint32_t ah0 = desc_lo(aslot), al0 = ah0 + (kCtATile >> 4);
    const uint32_t bh0 = desc_lo(bchunk), bl0 = bh0 + ((kCtBChunk / 2) >> 4);
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, al0 + adv, bh0 + adv, idesc, (!first || kk > 0) ? 1u : 0u);
        umma_tf32_lo(d, ah0 + adv, bl0 + adv, idesc, 1u);
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, ah0 + adv, bh0 + adv, idesc, 1u);
    }
}

template <int CP, int BWIN>
__global__ void __launch_bounds__(kCtThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs p) {
    constexpr int NCH = CP == 8 ? 4 : 1;  // K-chunks per block (conv_tc_geometry)
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
    const long long nblk = my_tiles * (p.Hq / BWIN) * p.Wq;
    const int nch = NCH;

    // the weights over the patch (pre-swizzled on the host) and the bias
    for (int i = tid; i < nch * (int)(kCtBChunk / 16); i += kCtThreads)
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
            // ---- MMA issuer: block by block, chunk by chunk ----
            const uint32_t a_s = smem_u32(a0), b_s = smem_u32(b0);
            bool ok = true;
            for (long long j = 0; j < nblk && ok; j++) {
                const uint32_t d = tmem + (uint32_t)((j & 1) * 64);
                ok = mbar_wait(&d_empty[j & 1], (uint32_t)(((j >> 1) & 1) ^ 1), p.err, 11, (int)j, 0, 0, 2);
                for (int c = 0; c < nch && ok; c++) {
                    const long long q = (long long)nch * j + c;
                    ok = mbar_wait(&a_full[q % kCtR], (uint32_t)((q / kCtR) & 1), p.err, 12, (int)j, c, 0, 2);
                    if (!ok) break;
                    tc_fence_after();
                    ct_issue_chunk(a_s + (uint32_t)(q % kCtR) * kCtSlot, b_s + (uint32_t)c * kCtBChunk, d, c == 0);
                    umma_commit(&a_empty[q % kCtR]);
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
        // the chunk stream q = (block, chunk); the loads of chunk q+1 are issued
        // before chunk q is split and stored, so two chunks' loads are in flight
        const long long nq = nblk * NCH;
        float v[16], vn[16];
        if (nq > 0) ct_load<CP, BWIN>(p, r, g, ct_block(p, 0), 0, v);
        for (long long q = 0; q < nq && ok; q++) {
            const long long j = q / NCH;
            const int c = (int)(q - j * NCH);
            if (q + 1 < nq) {
                const long long j1 = (q + 1) / NCH;
                ct_load<CP, BWIN>(p, r, g, ct_block(p, j1), (int)(q + 1 - j1 * NCH), vn);
            }
            const int s = (int)(q % kCtR);
            if (q >= kCtR) {
                ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[s], (uint32_t)(((q / kCtR) - 1) & 1), p.err, 13, (int)j,
                                                       c, 0, slot));
                if (!ok) break;
            }
            uint8_t *ahi = a0 + (uint32_t)s * kCtSlot;
            put_a16(ahi, ahi + kCtATile, r, 16 * g, v);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&a_full[s]);
            if (c == NCH - 1 && j > 0) {  // block j staged: drain block j-1 while its MMAs run
                const long long jd = j - 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&d_full[jd & 1], (uint32_t)((jd >> 1) & 1), p.err, 14, (int)jd, 0, 0, slot));
                if (!ok) break;
                tc_fence_after();
                ct_drain(p, sbias, lane_base + (uint32_t)((jd & 1) * 64), r, g, ct_block(p, jd));
                tc_fence_before();
                mbar_arrive(&d_empty[jd & 1]);
            }
#pragma unroll
            for (int e = 0; e < 16; e++) v[e] = vn[e];
        }
        if (ok && nblk > 0) {  // the last block
            const long long jd = nblk - 1;
            ok = __all_sync(0xffffffffu,
                            mbar_wait(&d_full[jd & 1], (uint32_t)((jd >> 1) & 1), p.err, 14, (int)jd, 0, 0, slot));
            if (ok) {
                tc_fence_after();
                ct_drain(p, sbias, lane_base + (uint32_t)((jd & 1) * 64), r, g, ct_block(p, jd));
                tc_fence_before();
                mbar_arrive(&d_empty[jd & 1]);
            }
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
    if (!(KS == 3 && str_h == 1 && str_w == 1 && pad_h == pad_w && pad_h >= 0 && pad_h <= 2 && C >= 1 && C <= 8 &&
          OC >= 1 && OC <= 16 && pool != 0 && pk == 2 && pstr_h == 2 && pstr_w == 2 && ppad_h == 0 && ppad_w == 0 &&
          Ho % 2 == 0 && Wo % 2 == 0 && Ho >= 2 && Wo >= 2))
        return false;
    ConvTcGeom g = conv_tc_geometry(C, OC);
    return (Ho / 2) % g.bwin == 0;
}

ConvTcGeom conv_tc_geometry(int C, int OC) {
    ConvTcGeom g;
    g.cp = C == 1 ? 1 : 8;
    // a single-channel input with at most 8 output channels: two windows per
    // block (N = 8 pixels x 8 channels); otherwise one (N = 4 x 16)
    g.bwin = (C == 1 && OC <= 8) ? 2 : 1;
    const int positions = (2 * g.bwin + 2) * 4;
    g.nch = (positions * g.cp + 31) / 32;
    return g;
}

// The B image: nch K-chunks, each hi [64 rows x 32] then lo, as
// 128-byte-swizzled K-major rows (row r of an 8-row atom holds 16-byte chunk k
// at position k ^ (r & 7)) so the kernel copies it linearly.
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

void conv_tc_pack(const float *w, int OC, int C, float *img) {
    // w: [oc][ic][kh][kw] (3x3)
    const ConvTcGeom g = conv_tc_geometry(C, OC);
    const int ocp = 16 / g.bwin, PW = 4, PH = 2 * g.bwin + 2;
    for (int i = 0; i < kConvTcBFloats; i++) img[i] = 0.f;
    for (int row = 0; row < 64; row++) {
        const int pix = row / ocp, oc = row - pix * ocp;
        const int win = pix / 4, pa = (pix % 4) / 2, pb = pix % 2;  // pixel (pa, pb) of window win (stacked in y)
        const int cy = 2 * win + pa, cx = pb;  // conv pixel within the block
        for (int k = 0; k < 32 * g.nch; k++) {
            const int pos = k / g.cp, ch = k - pos * g.cp;
            const int py = pos / PW, px = pos - py * PW;
            const int kh = py - cy, kw = px - cx;
            float x = 0.f;
            if (oc < OC && ch < C && pos < PH * PW && kh >= 0 && kh < 3 && kw >= 0 && kw < 3)
                x = w[(((size_t)oc * C + ch) * 3 + kh) * 3 + kw];
            const float h = tf32_hi(x), l = tf32_hi(x - h);
            const int c = k / 32;
            put_swizzled(img + c * kConvTcBChunk, row, k % 32, h);
            put_swizzled(img + c * kConvTcBChunk + kConvTcBChunk / 2, row, k % 32, l);
        }
    }
}

cudaError_t conv_tc_configure() {
    const int smem = (int)conv_tc_smem();
    cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel<8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(conv_tc_kernel<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(conv_tc_kernel<1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    return e;
}

cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + 127) / 128;
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    if (a.Hq % a.bwin) return cudaErrorInvalidConfiguration;
    if (a.cp == 8 && a.bwin == 1 && a.nch == 4)
        conv_tc_kernel<8, 1><<<grid, kCtThreads, conv_tc_smem(), st>>>(a);
    else if (a.cp == 1 && a.bwin == 1 && a.nch == 1)
        conv_tc_kernel<1, 1><<<grid, kCtThreads, conv_tc_smem(), st>>>(a);
    else if (a.cp == 1 && a.bwin == 2 && a.nch == 1)
        conv_tc_kernel<1, 2><<<grid, kCtThreads, conv_tc_smem(), st>>>(a);
    else
        return cudaErrorInvalidConfiguration;
    return cudaGetLastError();
}

}  // namespace rosenna
