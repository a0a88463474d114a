// One LSTM layer with 4H <= 128 gate columns on the tensor cores (tcgen05,
// 3xTF32), each column group running a 128-sample tile of its own
// (fLibrary/layers.f90 lstm :101-132, lstm_cell :62-99).
//
// Shapes: input width I <= 32 and hidden size H <= 32, so a time step is one
// 128-sample x 4H x 64 product of [x_t | h_{t-1}] (two 32-wide K-chunks) with
// the packed gate block (rows n = 4j+q: gate q of unit j; tf32 hi rows, then
// the rounded remainders).  The block is small enough to stay in shared memory
// for the whole kernel (one TMA load).  The CTA runs two tiles at a time, each
// by two warpgroups that split its units (16 each: thread = sample row; its
// units' c and h in registers, their gate columns drained 16 at a time): they stage
// their K halves of [x_t | h_{t-1}] as tf32 hi/lo A chunks, and after the
// step's MMAs drain their half of the gate partial from TMEM and run the cell
// update.  The issuer takes tile 0's step, then tile 1's, so one tile's cell
// update runs while the other's MMAs do; with all 4H columns in one MMA (N =
// 4H), an M = 128 MMA uses the tensor core fully at 4H = 128.  x_{t+1} is
// prefetched by cp.async during step t.  (With one warpgroup per tile holding
// all 32 units, the 192 live registers left the MUFU-bound cell update too few
// warps to hide its latency.)
//
// Roles (544 threads): warps 0-15 the four warpgroups (tile = warpgroup / 2,
// unit half = warpgroup % 2), warp 16 lane 0 issues the MMAs.  Every wait is
// bounded; a time-out records where in `err`, every role finishes, TMEM is
// freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mlp_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kDThreads = 544;

constexpr uint32_t kDTile = 128 * 128;          // one 32-wide K-chunk of 128 rows (hi or lo)
constexpr uint32_t kDOffB = 0;                  // 2 K-chunks x (hi, lo)
constexpr uint32_t kDOffA = 4 * kDTile;         // per group: x slot (hi, lo), h slot (hi, lo)
constexpr uint32_t kDOffX = kDOffA + 8 * kDTile;  // per group: x_{t+1} [32][128] fp32
constexpr uint32_t kDXBuf = 32 * 128 * 4;
constexpr uint32_t kDOffBias = kDOffX + 2 * kDXBuf;
constexpr uint32_t kDOffBars = kDOffBias + 128 * 4;
constexpr uint32_t kDTmemCols = 256;            // group g's gate partial at column 128g

size_t lstm_dual_tc_smem() { return 1024 + kDOffBars + 256; }

enum {
    kDBReady = 0,   // the gate block loaded
    kDAFull = 1,    // [2 tiles][2 chunks] staged (256 arrivals each: both unit halves)
    kDPFull = 5,    // [2] gates of the tile's step complete (commit)
    kDPEmpty = 7,   // [2] drained (256 arrivals)
    kDDone = 9,
    kDNumBars = 10
};

__device__ __forceinline__ void cp_async4(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}

// features 16hf..16hf+15 of x_s, sample row r, into the tile's buffer ([k][row];
// zero beyond I)
__device__ __forceinline__ void d_prefetch_x(const TcLstmArgs &p, float *xbuf, int r, long long row, int s, int hf) {
    const bool valid = row < p.n;
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int k = 16 * hf + e;
        const bool ok = valid && k < p.I;
        cp_async4(xbuf + (size_t)k * 128 + r, ok ? p.x + (long long)(s + (long long)p.T * k) * p.ld_x + row : p.x, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}


__device__ __forceinline__ void d_issue(uint32_t a_s, uint32_t b_s, uint32_t d, uint32_t idesc, bool first) {
    const uint32_t ah = desc_lo(a_s), al = ah + (kDTile >> 4);
    const uint32_t bh = desc_lo(b_s), bl = bh + (kDTile >> 4);
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, al + adv, bh + adv, idesc, (kk > 0 || !first) ? 1u : 0u);
        umma_tf32_lo(d, ah + adv, bl + adv, idesc, 1u);
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, ah + adv, bh + adv, idesc, 1u);
    }
}

__global__ void __launch_bounds__(kDThreads, 1) lstm_dual_tc_kernel(const __grid_constant__ TcLstmArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base + kDOffB;
    float *const sbias = reinterpret_cast<float *>(base + kDOffBias);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kDOffBars);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kDNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = p.T, Np = p.Np;
    const int ntiles = (int)((p.n + 127) / 128);
    // pairs of tiles: pair k of this CTA holds tiles 2*(blockIdx.x + k*gridDim.x) + g
    const int npairs = (ntiles + 1) / 2;
    const int my_pairs = (int)blockIdx.x < npairs ? (npairs - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    for (int i = tid; i < 128; i += kDThreads) sbias[i] = i < Np ? p.arena[p.b_off + i] : 0.f;
    if (tid == 0) {
        mbar_init(bars + kDBReady, 1);
        for (int i = 0; i < 4; i++) mbar_init(bars + kDAFull + i, 256);
        for (int g = 0; g < 2; g++) {
            mbar_init(bars + kDPFull + g, 1);
            mbar_init(bars + kDPEmpty + g, 256);
        }
        mbar_init(bars + kDDone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kDTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 16) {
        if (warp == 16 && lane == 0) {
            // ---- the gate block, once; then the MMA issuer ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map) : "memory");
            mbar_arrive_expect_tx(bars + kDBReady, 4u * (uint32_t)Np * 128u);
            for (int c = 0; c < 2; c++) {
                tma_load_2d(b0 + (uint32_t)c * 2 * kDTile, &p.map, bars + kDBReady, 32 * c, 0);
                tma_load_2d(b0 + (uint32_t)c * 2 * kDTile + kDTile, &p.map, bars + kDBReady, 32 * c, Np);
            }
            bool ok = mbar_wait(bars + kDBReady, 0, p.err, 41, 0, 0, 0, 2);
            const uint32_t sa = smem_u32(base + kDOffA), sb = smem_u32(b0);
            const uint32_t idesc = idesc_tf32(Np);
            uint32_t nst[2] = {0, 0};  // steps issued per group
            for (int k = 0; k < my_pairs && ok; k++) {
                const int t0 = 2 * ((int)blockIdx.x + k * (int)gridDim.x);
                const bool has1 = t0 + 1 < ntiles;
                for (int s = 0; s < T && ok; s++)
                    for (int g = 0; g < 2 && ok; g++) {
                        if (g == 1 && !has1) continue;
                        if (nst[g] > 0)
                            ok = mbar_wait(bars + kDPEmpty + g, (nst[g] - 1) & 1, p.err, 42, s, g, (int)nst[g], 2);
                        for (int c = 0; c < 2 && ok; c++) {
                            ok = mbar_wait(bars + kDAFull + 2 * g + c, nst[g] & 1, p.err, 43, s, g * 2 + c, (int)nst[g], 2);
                            if (!ok) break;
                            tc_fence_after();
                            d_issue(sa + (uint32_t)(2 * g + c) * 2 * kDTile, sb + (uint32_t)c * 2 * kDTile,
                                    tmem + (uint32_t)(128 * g), idesc, c == 0);
                        }
                        if (!ok) break;
                        umma_commit(bars + kDPFull + g);
                        nst[g]++;
                    }
            }
            umma_commit(bars + kDDone);
            mbar_wait(bars + kDDone, 0, p.err, 0);
        }
    } else {
        const int wg = warp >> 2, g = wg >> 1, hf = wg & 1, quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(128 * g + 64 * hf);
        const int slot = (lane == 0 && quad == 2) ? 3 + wg : 0;
        uint8_t *const ax = base + kDOffA + (uint32_t)(2 * g) * 2 * kDTile;  // x slot, then h slot
        uint8_t *const ah = ax + 2 * kDTile;
        float *const xbuf = reinterpret_cast<float *>(base + kDOffX + (uint32_t)g * kDXBuf);
        const float *const bias = sbias + 64 * hf;
        uint32_t nst = 0;
        bool ok = true;
        float c[16], h[16];
        for (int k = 0; k < my_pairs && ok; k++) {
            const int t = 2 * ((int)blockIdx.x + k * (int)gridDim.x) + g;
            if (t >= ntiles) break;  // the last pair may have only tile 0
            const long long row = (long long)t * 128 + r;
            const bool valid = row < p.n;
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int unit = 16 * hf + u;
                float h0 = 0.f, c0 = 0.f;
                if (unit < p.H && valid) {
                    h0 = p.h0 ? p.h0[(long long)unit * p.ld_h0 + row]
                              : (p.h0_const >= 0 ? p.arena[p.h0_const + unit] : 0.f);
                    c0 = p.c0 ? p.c0[(long long)unit * p.ld_c0 + row]
                              : (p.c0_const >= 0 ? p.arena[p.c0_const + unit] : 0.f);
                }
                h[u] = h0;
                c[u] = c0;
            }
            // h_{-1}: the h slot is free (the previous tile's last MMAs completed)
            put_a16(ah, ah + kDTile, r, 16 * hf, h);
            d_prefetch_x(p, xbuf, r, row, 0, hf);
            for (int s = 0; s < T && ok; s++) {
                // x_s (this half's K range) beside h_{s-1}, staged at the end of the step before
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                {
                    float v[16];
#pragma unroll
                    for (int e = 0; e < 16; e++) v[e] = xbuf[(size_t)(16 * hf + e) * 128 + r];
                    put_a16(ax, ax + kDTile, r, 16 * hf, v);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                mbar_arrive(bars + kDAFull + 2 * g);
                mbar_arrive(bars + kDAFull + 2 * g + 1);
                if (s + 1 < T) d_prefetch_x(p, xbuf, r, row, s + 1, hf);
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kDPFull + g, nst & 1, p.err, 44, s, (int)nst, 0, slot));
                if (!ok) break;
                tc_fence_after();
                // gates of this half's units in four rounds of 4 units (16 columns):
                // bias + the partial, then the cell update (layers.f90 lstm_cell)
#pragma unroll
                for (int rd = 0; rd < 4; rd++) {
                    float acc[16];
                    {
                        uint32_t w[16];
                        if (64 * hf + 16 * rd < Np) tmem_ld16_nw(lane_base + (uint32_t)(16 * rd), w);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; e++)
                            acc[e] = 64 * hf + 16 * rd < Np ? __uint_as_float(w[e]) + bias[16 * rd + e] : 0.f;
                    }
                    if (rd == 3) {
                        tc_fence_before();
                        mbar_arrive(bars + kDPEmpty + g);
                    }
#pragma unroll
                    for (int uu = 0; uu < 4; uu++) {
                        const int u = 4 * rd + uu;
                        const float ig = tc_act<3>(acc[4 * uu]), fg = tc_act<3>(acc[4 * uu + 1]);
                        const float gg = tc_act<2>(acc[4 * uu + 2]), og = tc_act<3>(acc[4 * uu + 3]);
                        c[u] = fg * c[u] + ig * gg;
                        h[u] = og * tc_act<2>(c[u]);
                        if (16 * hf + u >= p.H) h[u] = c[u] = 0.f;  // padded units stay zero
                    }
                }
                nst++;
                // h_s into the h slot for the next step (this step's MMAs are complete)
                put_a16(ah, ah + kDTile, r, 16 * hf, h);
                if (valid) {
#pragma unroll
                    for (int u = 0; u < 16; u++) {
                        const int unit = 16 * hf + u;
                        if (unit >= p.H) continue;
                        if (p.y) p.y[(long long)(s + (long long)T * unit) * p.ld_y + row] = h[u];
                        if (s + 1 == T) {
                            if (p.hn) p.hn[(long long)unit * p.ld_hn + row] = h[u];
                            if (p.cn) p.cn[(long long)unit * p.ld_cn + row] = c[u];
                        }
                    }
                }
            }
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDTmemCols));
    }
}

}  // namespace

bool lstm_dual_tc_regs_ok() { return true; }  // no register split between roles

cudaError_t lstm_dual_tc_configure() {
    return cudaFuncSetAttribute(lstm_dual_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)lstm_dual_tc_smem());
}

cudaError_t launch_lstm_dual_tc(const TcLstmArgs &a, int num_sms, cudaStream_t st) {
    const long long pairs = ((a.n + 127) / 128 + 1) / 2;
    const int grid = (int)(pairs < num_sms ? pairs : num_sms);
    if (grid <= 0) return cudaSuccess;
    if (a.nx != 1 || a.nh != 1 || a.Np > 128 || a.H > 32 || a.I > 32) return cudaErrorInvalidConfiguration;
    lstm_dual_tc_kernel<<<grid, kDThreads, lstm_dual_tc_smem(), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna
