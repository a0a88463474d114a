// Two stacked LSTM layers in one persistent tensor-core kernel (tcgen05,
// 3xTF32): fLibrary/layers.f90 lstm (:101-132) run twice, the second layer on
// the first layer's output sequence, as the reference's generated use_model
// does for two LSTM nodes (fLibrary/modelCreator.fpp:92-100).  Layer 1's
// output sequence never leaves shared memory.
//
// Shapes: hidden size 64 in both layers (4H = 256 gate columns), layer-1 input
// width at most 32.  Per CTA (one per SM, persistent over tiles of 128
// samples; TMEM lane = sample row), super-step s = 0..T computes layer-1 step
// s (s < T) and layer-2 step s-1 (s >= 1) as a stream of K-chunks of 32:
//   c0: x_s     x W1[x]          -> P1   (layer-1 gates)
//   c1: h1[0:32]  x W1[h 0:32]   -> P1
//   c2: h1[32:64] x W1[h 32:64]  -> P1     (P1 complete)
//   c3: h1[0:32]  x W2[x 0:32]   -> P2   (layer-2 gates; h1 = h1_{s-1})
//   c4: h1[32:64] x W2[x 32:64]  -> P2     (h1 consumed by both layers)
//   c5: h2[0:32]  x W2[h 0:32]   -> P2
//   c6: h2[32:64] x W2[h 32:64]  -> P2     (P2 complete)
// Each chunk is issued per column group g (gate columns 128g.., units
// 32g..32g+31; N = 128): the small terms (Al*Wh, Ah*Wl) first, Ah*Wh last.
// Group g's warps drain P1 (bias, gates, c1 in registers), write h1_s for
// their 32 units straight into the A tile of h1 (tf32 hi/lo, 128-byte
// swizzled: exactly K-chunk g), then drain P2 and write h2 the same way.
// While the warps run one layer's cell update, the tensor core runs the other
// layer's chunks: after c2 the layer-1 update overlaps c3..c6, after c6 the
// layer-2 update overlaps c0..c4 of the next super-step.  Each layer's gates
// accumulate in one TMEM partial (96 / 128 deep); LSTM gates and weights are
// small, so the tensor core's inexact fp32 accumulation stays far inside the
// tolerance (the per-layer kernel accumulates 64-deep partials the same way).
//
// Roles (384 threads): warps 0-7 the two column groups; warp 8 lane 0 issues
// the MMAs; warp 9 lane 0 streams the weight chunks by TMA (two 32 KB stages:
// one group's 128 rows of a K-chunk, tf32 hi and lo).  setmaxnreg moves
// registers from the producer warpgroup (40) to the groups (232).  Every wait
// is bounded; a time-out records where in `err`, every role finishes, TMEM is
// freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mlp_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kL2Threads = 384;
constexpr int kL2LaunchRegs = 168;
constexpr int kL2ConsumerRegs = 232, kL2ProducerRegs = 40;
static_assert(kL2Threads * kL2LaunchRegs >= 256 * kL2ConsumerRegs + 128 * kL2ProducerRegs, "register split");

constexpr uint32_t kL2Tile = 128 * 128;       // one 32-wide K-chunk of 128 rows: 16 KB
constexpr uint32_t kL2Stage = 2 * kL2Tile;    // hi + lo
constexpr uint32_t kL2OffB = 0;               // 2 weight stages
constexpr uint32_t kL2OffX = 2 * kL2Stage;    // x_s
constexpr uint32_t kL2OffH1 = kL2OffX + kL2Stage;       // h1 chunks 0, 1
constexpr uint32_t kL2OffH2 = kL2OffH1 + 2 * kL2Stage;  // h2 chunks 0, 1
constexpr uint32_t kL2OffBars = kL2OffH2 + 2 * kL2Stage;
constexpr uint32_t kL2TmemCols = 512;         // P1 at 0 (128 per group), P2 at 256

size_t lstm2_tc_smem() { return 1024 + kL2OffBars + 256; }

// Barriers (offsets into the barrier block).
enum {
    kBFull = 0,    // [2] weight stage loaded (TMA bytes)
    kBEmpty = 2,   // [2] weight stage consumed (commit)
    kXFull = 4,    // x_s staged (256 arrivals)
    kXFree = 5,    // x_s consumed (commit)
    kH1Full = 6,   // [2] h1 chunk g written (128 arrivals)
    kH1Free = 8,   // h1 consumed by both layers (commit)
    kH2Full = 9,   // [2] h2 chunk g written (128 arrivals)
    kP1Full = 11,  // [2] layer-1 gates of group g complete (commit)
    kP1Empty = 13, // [2] drained (128 arrivals)
    kP2Full = 15,  // [2]
    kP2Empty = 17, // [2]
    kDone = 19,    // the issuer's last MMAs complete
    kNumBars = 20
};

// One chunk of one column group: 128 samples x 128 gate columns x 32 K, as
// Al*Wh + Ah*Wl (4 K-steps each) then Ah*Wh; `first` starts the partial.
__device__ __forceinline__ void l2_issue(uint32_t a_s, uint32_t b_s, uint32_t d, bool first) {
    const uint32_t ah = desc_lo(a_s), al = ah + (kL2Tile >> 4);
    const uint32_t bh = desc_lo(b_s), bl = bh + (kL2Tile >> 4);
    const uint32_t idesc = idesc_tf32(128);
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

// Weight chunk kc of layer `layer`, rows of group g (hi and lo), into stage st.
__device__ __forceinline__ void l2_load(const TcLstm2Args &p, uint8_t *b0, uint64_t *bars, int layer, int kc, int g,
                                        int st) {
    const CUtensorMap *map = layer == 0 ? &p.map1 : &p.map2;
    uint64_t *full = bars + kBFull + st;
    mbar_arrive_expect_tx(full, kL2Stage);
    tma_load_2d(b0 + (uint32_t)st * kL2Stage, map, full, kc * 32, 128 * g);
    tma_load_2d(b0 + (uint32_t)st * kL2Stage + kL2Tile, map, full, kc * 32, 256 + 128 * g);
}

// Writes this thread's 32 values (units 32g..32g+31) as K-chunk g of an A tile
// (hi at `chunk`, lo 16 KB after it).
__device__ __forceinline__ void l2_put_h(uint8_t *chunk, int r, const float *h) {
    float v[16];
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
#pragma unroll
        for (int e = 0; e < 16; e++) v[e] = h[16 * hf + e];
        put_a16(chunk, chunk + kL2Tile, r, 16 * hf, v);
    }
}

// Stages this thread's K half (features 16g..16g+15) of x_s for sample row r.
__device__ __forceinline__ void l2_stage_x(const TcLstm2Args &p, uint8_t *xa, int r, int g, int t, int s) {
    const long long row = (long long)t * 128 + r;
    const bool valid = row < p.n;
    float v[16];
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int k = 16 * g + e;
        v[e] = (valid && k < p.I) ? __ldg(p.x + (long long)(s + (long long)p.T * k) * p.ld_x + row) : 0.f;
    }
    put_a16(xa, xa + kL2Tile, r, 16 * g, v);
}

// Gates of this group's 32 units from its 128 partial columns (plus bias):
// c <- f*c + i*g, h <- o*tanh(c), with the gates of unit u at columns 4u..4u+3.
__device__ __forceinline__ void l2_cell(float (&acc)[128], float (&c)[32], float (&h)[32]) {
#pragma unroll
    for (int u = 0; u < 32; u++) {
        const float ig = tc_act<3>(acc[4 * u]), fg = tc_act<3>(acc[4 * u + 1]);
        const float gg = tc_act<2>(acc[4 * u + 2]), og = tc_act<3>(acc[4 * u + 3]);
        c[u] = fg * c[u] + ig * gg;
        h[u] = og * tc_act<2>(c[u]);
    }
}

__device__ __forceinline__ void l2_drain(uint32_t taddr, const float *bias, float (&acc)[128]) {
#pragma unroll
    for (int q0 = 0; q0 < 8; q0 += 4) {
        uint32_t v[4][16];
#pragma unroll
        for (int u = 0; u < 4; u++) tmem_ld16_nw(taddr + (uint32_t)(16 * (q0 + u)), v[u]);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int e = 0; e < 16; e++) acc[16 * (q0 + u) + e] = __uint_as_float(v[u][e]) + bias[16 * (q0 + u) + e];
    }
}

__global__ void __launch_bounds__(kL2Threads, 1) lstm2_tc_kernel(const __grid_constant__ TcLstm2Args p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base + kL2OffB;
    uint8_t *const xa = base + kL2OffX;
    uint8_t *const h1a = base + kL2OffH1;
    uint8_t *const h2a = base + kL2OffH2;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kL2OffBars);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = p.T;
    const int ntiles = (int)((p.n + 127) / 128);
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(bars + kBFull + i, 1);
            mbar_init(bars + kBEmpty + i, 1);
            mbar_init(bars + kH1Full + i, 128);
            mbar_init(bars + kH2Full + i, 128);
            mbar_init(bars + kP1Full + i, 1);
            mbar_init(bars + kP1Empty + i, 128);
            mbar_init(bars + kP2Full + i, 1);
            mbar_init(bars + kP2Empty + i, 128);
        }
        mbar_init(bars + kXFull, 256);
        mbar_init(bars + kXFree, 1);
        mbar_init(bars + kH1Free, 1);
        mbar_init(bars + kDone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kL2TmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kL2ProducerRegs));
        if (warp == 8 && lane == 0) {
            // ---- MMA issuer ----
            const uint32_t sb = smem_u32(b0), sx = smem_u32(xa), sh1 = smem_u32(h1a), sh2 = smem_u32(h2a);
            uint32_t bs = 0, nx = 0, np1 = 0, np2 = 0, nh1 = 0;
            bool ok = true;
            for (int tt = 0; tt < my_tiles && ok; tt++) {
                for (int s = 0; s <= T && ok; s++) {
                    const bool l1 = s < T, l2 = s >= 1;
                    if (l1) {
                        for (int kc = 0; kc < 3 && ok; kc++) {
                            if (kc == 0) ok = mbar_wait(bars + kXFull, nx & 1, p.err, 21, s, (int)nx, 0, 2);
                            else ok = mbar_wait(bars + kH1Full + (kc - 1), nh1 & 1, p.err, 22, s, kc, (int)nh1, 2);
                            const uint32_t a_s = kc == 0 ? sx : sh1 + (uint32_t)(kc - 1) * kL2Stage;
                            for (int g = 0; g < 2 && ok; g++) {
                                if (kc == 0 && np1 > 0)
                                    ok = mbar_wait(bars + kP1Empty + g, (np1 - 1) & 1, p.err, 23, s, g, (int)np1, 2);
                                if (ok) ok = mbar_wait(bars + kBFull + (bs & 1), (bs >> 1) & 1, p.err, 24, s, kc, (int)bs, 2);
                                if (!ok) break;
                                tc_fence_after();
                                l2_issue(a_s, sb + (bs & 1) * kL2Stage, tmem + (uint32_t)(128 * g), kc == 0);
                                umma_commit(bars + kBEmpty + (bs & 1));
                                bs++;
                                if (kc == 2) umma_commit(bars + kP1Full + g);
                            }
                            if (kc == 0 && ok) umma_commit(bars + kXFree);
                        }
                        if (!ok) break;
                        nx++;
                        np1++;
                    }
                    if (l2) {
                        for (int kc = 0; kc < 4 && ok; kc++) {
                            if (kc < 2 && !l1)
                                ok = mbar_wait(bars + kH1Full + kc, nh1 & 1, p.err, 25, s, kc, (int)nh1, 2);
                            if (kc >= 2) {
                                // content h2_{s-2}: write number tt*(T+1) + s-1 of its chunk
                                const uint32_t w = (uint32_t)tt * (uint32_t)(T + 1) + (uint32_t)(s - 1);
                                ok = ok && mbar_wait(bars + kH2Full + (kc - 2), w & 1, p.err, 26, s, kc, (int)w, 2);
                            }
                            const uint32_t a_s = kc < 2 ? sh1 + (uint32_t)kc * kL2Stage : sh2 + (uint32_t)(kc - 2) * kL2Stage;
                            for (int g = 0; g < 2 && ok; g++) {
                                if (kc == 0 && np2 > 0)
                                    ok = mbar_wait(bars + kP2Empty + g, (np2 - 1) & 1, p.err, 27, s, g, (int)np2, 2);
                                if (ok) ok = mbar_wait(bars + kBFull + (bs & 1), (bs >> 1) & 1, p.err, 24, s, 3 + kc, (int)bs, 2);
                                if (!ok) break;
                                tc_fence_after();
                                l2_issue(a_s, sb + (bs & 1) * kL2Stage, tmem + 256u + (uint32_t)(128 * g), kc == 0);
                                umma_commit(bars + kBEmpty + (bs & 1));
                                bs++;
                                if (kc == 3) umma_commit(bars + kP2Full + g);
                            }
                            if (kc == 1 && ok) umma_commit(bars + kH1Free);
                        }
                        if (!ok) break;
                        np2++;
                    } else {
                        umma_commit(bars + kH1Free);
                    }
                    nh1++;
                }
            }
            umma_commit(bars + kDone);
            mbar_wait(bars + kDone, 0, p.err, 0);
        } else if (warp == 9 && lane == 0) {
            // ---- weight loader: the issuer's chunk order, one group's rows per stage ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map1) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map2) : "memory");
            uint32_t bs = 0;
            bool ok = true;
            for (int tt = 0; tt < my_tiles && ok; tt++)
                for (int s = 0; s <= T && ok; s++)
                    for (int layer = 0; layer < 2 && ok; layer++) {
                        if ((layer == 0 && s >= T) || (layer == 1 && s < 1)) continue;
                        const int nkc = layer == 0 ? 3 : 4;
                        for (int kc = 0; kc < nkc && ok; kc++)
                            for (int g = 0; g < 2 && ok; g++) {
                                if (bs >= 2)
                                    ok = mbar_wait(bars + kBEmpty + (bs & 1), ((bs >> 1) - 1) & 1, p.err, 28, s, kc,
                                                   (int)bs, 1);
                                if (!ok) break;
                                l2_load(p, b0, bars, layer, kc, g, (int)(bs & 1));
                                bs++;
                            }
                    }
            // the last loads land before the CTA ends
            for (uint32_t k = bs > 2 ? bs - 2 : 0; k < bs; k++) mbar_wait(bars + kBFull + (k & 1), (k >> 1) & 1, p.err, 0);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kL2ConsumerRegs));
        const int g = warp >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const int slot = (lane == 0 && quad == 2) ? 3 + g : 0;
        uint32_t nh1w = 0, nxw = 0, np1 = 0, np2 = 0;
        bool ok = true;
        float acc[128], c1[32], c2[32], h[32];
        for (int tt = 0; tt < my_tiles && ok; tt++) {
            const int t = (int)blockIdx.x + tt * (int)gridDim.x;
            const long long row = (long long)t * 128 + r;
            const bool valid = row < p.n;
            // initial state of both layers for this group's 32 units
            for (int layer = 0; layer < 2; layer++) {
                const float *hp = p.h0[layer], *cp = p.c0[layer];
#pragma unroll
                for (int u = 0; u < 32; u++) {
                    const int unit = 32 * g + u;
                    float hv = 0.f, cv = 0.f;
                    if (valid) {
                        hv = hp ? hp[(long long)unit * p.ld_h0[layer] + row]
                                : (p.h0_const[layer] >= 0 ? p.arena[p.h0_const[layer] + unit] : 0.f);
                        cv = cp ? cp[(long long)unit * p.ld_c0[layer] + row]
                                : (p.c0_const[layer] >= 0 ? p.arena[p.c0_const[layer] + unit] : 0.f);
                    }
                    h[u] = hv;
                    if (layer == 0) c1[u] = cv;
                    else c2[u] = cv;
                }
                if (layer == 0) {
                    if (nh1w > 0) {
                        ok = __all_sync(0xffffffffu, mbar_wait(bars + kH1Free, (nh1w - 1) & 1, p.err, 31, -1, (int)nh1w, 0, slot));
                        if (!ok) break;
                    }
                    l2_put_h(h1a + (uint32_t)g * kL2Stage, r, h);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(bars + kH1Full + g);
                    nh1w++;
                } else {
                    l2_put_h(h2a + (uint32_t)g * kL2Stage, r, h);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(bars + kH2Full + g);
                }
            }
            if (!ok) break;
            // x_0
            if (nxw > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kXFree, (nxw - 1) & 1, p.err, 32, -1, (int)nxw, 0, slot));
                if (!ok) break;
            }
            l2_stage_x(p, xa, r, g, t, 0);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(bars + kXFull);
            nxw++;
            for (int s = 0; s <= T && ok; s++) {
                if (s < T) {
                    // ---- layer 1, step s ----
                    ok = __all_sync(0xffffffffu, mbar_wait(bars + kP1Full + g, np1 & 1, p.err, 33, s, (int)np1, 0, slot));
                    if (!ok) break;
                    tc_fence_after();
                    l2_drain(lane_base + (uint32_t)(128 * g), p.bias1 + 128 * g, acc);
                    tc_fence_before();
                    mbar_arrive(bars + kP1Empty + g);
                    np1++;
                    l2_cell(acc, c1, h);
                    ok = __all_sync(0xffffffffu, mbar_wait(bars + kH1Free, (nh1w - 1) & 1, p.err, 34, s, (int)nh1w, 0, slot));
                    if (!ok) break;
                    l2_put_h(h1a + (uint32_t)g * kL2Stage, r, h);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(bars + kH1Full + g);
                    nh1w++;
                    if (s + 1 == T && valid) {
#pragma unroll
                        for (int u = 0; u < 32; u++) {
                            const int unit = 32 * g + u;
                            if (p.hn[0]) p.hn[0][(long long)unit * p.ld_hn[0] + row] = h[u];
                            if (p.cn[0]) p.cn[0][(long long)unit * p.ld_cn[0] + row] = c1[u];
                        }
                    }
                    if (s + 1 < T) {
                        ok = __all_sync(0xffffffffu, mbar_wait(bars + kXFree, (nxw - 1) & 1, p.err, 32, s, (int)nxw, 0, slot));
                        if (!ok) break;
                        l2_stage_x(p, xa, r, g, t, s + 1);
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        mbar_arrive(bars + kXFull);
                        nxw++;
                    }
                }
                if (s >= 1) {
                    // ---- layer 2, step s-1 ----
                    ok = __all_sync(0xffffffffu, mbar_wait(bars + kP2Full + g, np2 & 1, p.err, 35, s, (int)np2, 0, slot));
                    if (!ok) break;
                    tc_fence_after();
                    l2_drain(lane_base + 256u + (uint32_t)(128 * g), p.bias2 + 128 * g, acc);
                    tc_fence_before();
                    mbar_arrive(bars + kP2Empty + g);
                    np2++;
                    l2_cell(acc, c2, h);
                    // h2_{s-2} was read by c5/c6, complete with P2
                    l2_put_h(h2a + (uint32_t)g * kL2Stage, r, h);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(bars + kH2Full + g);
                    if (valid) {
#pragma unroll
                        for (int u = 0; u < 32; u++) {
                            const int unit = 32 * g + u;
                            if (p.y2) p.y2[(long long)((s - 1) + (long long)T * unit) * p.ld_y2 + row] = h[u];
                            if (s == T) {
                                if (p.hn[1]) p.hn[1][(long long)unit * p.ld_hn[1] + row] = h[u];
                                if (p.cn[1]) p.cn[1][(long long)unit * p.ld_cn[1] + row] = c2[u];
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kL2TmemCols));
    }
}

}  // namespace

bool lstm2_tc_regs_ok() {
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, lstm2_tc_kernel) != cudaSuccess) {
        (void)cudaGetLastError();
        return true;
    }
    return a.numRegs == kL2LaunchRegs;
}

cudaError_t lstm2_tc_configure() {
    return cudaFuncSetAttribute(lstm2_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lstm2_tc_smem());
}

cudaError_t launch_lstm2_tc(const TcLstm2Args &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + 127) / 128;
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    static const int regs = [] {
        cudaFuncAttributes fa{};
        return cudaFuncGetAttributes(&fa, lstm2_tc_kernel) == cudaSuccess ? fa.numRegs : -1;
    }();
    if (regs != kL2LaunchRegs) return cudaErrorInvalidConfiguration;  // the setmaxnreg split needs exactly these
    lstm2_tc_kernel<<<grid, kL2Threads, lstm2_tc_smem(), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna
