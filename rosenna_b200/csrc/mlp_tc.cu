// Tensor-core fused MLP for layers up to 256 wide: tcgen05 (TMEM accumulators)
// with a 3xTF32 split, weights fed by TMA.
//
// Math (fLibrary/layers.f90:11-23 linear_layer + activation_funcs.f90, per
// layer): Y[s][n] = act(sum_k A[s][k] W[n][k] + b[n]).  With A = Ah + Al and
// W = Wh + Wl, where Xh = tf32_round(X) and Xl = tf32_round(X - Xh) (for
// the activations Xl = X - Xh, whose low bits the tensor core drops itself:
// tf32_lo), the product is taken as Al*Wh + Ah*Wl + Ah*Wh (the Al*Wl term is
// below 2^-22 relative), accumulated in fp32 in tensor memory: fp32-level
// accuracy from the TF32 tensor pipe.
//
// Per CTA (one per SM, persistent over tiles of 128 samples): two groups of
// four warps; group g owns output columns [128g, 128g+128) and thread r of a
// group owns sample row r (TMEM lane r); a third warpgroup produces:
//   - one lane issues every tcgen05.mma (M=128 samples, N=128 columns, K=8;
//     three per K-step for the 3xTF32 split), chunk by chunk, group 0's half
//     then group 1's, each into that group's TMEM partial buffer: one 32-deep
//     partial per K-chunk with the small terms first.  A group adds each
//     partial into fp32 registers (round-to-nearest: the tensor core truncates
//     while it accumulates, so long chains inside TMEM lose accuracy) while the
//     other group's MMAs run.  Issuing holds the issuing thread until its MMAs
//     are nearly done (the MMA queue is shallow), which is why it has no other
//     work.
//   - one lane streams [Wh | Wl] K-chunks of 32 (128-byte swizzled rows) by TMA
//     into a 2-stage ring, two chunks ahead of the MMAs.
//   - the A operand of layer 0 is the input tile, of later layers the previous
//     layer's activations (kept in TMEM), split into tf32 hi/lo in a 2-stage
//     smem ring by the group warps (each a 16-wide K half of its rows).
//   - after the last K-chunk a group adds bias, applies the activation and
//     writes its half to TMEM for the next layer (handed over through an
//     mbarrier; group 0 stages the next layer's first two chunks straight from
//     its registers), or to global memory.
// Every wait on an mbarrier is bounded; on time-out the kernel records an error
// code and where it waited in `err`, lets every role finish, frees TMEM and
// returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mlp_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kBM = 128;                 // samples per tile (UMMA M)
constexpr int kKC = 32;                  // K per chunk: 32 fp32 = one 128-byte swizzle row
constexpr int kNMax = 256;               // widest layer (UMMA N)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTCol = 0;             // TMEM cols [0,256): previous layer's activations
constexpr uint32_t kPCol = 256;           // TMEM cols [256,512): partial sums of column half h at 256+128h
constexpr uint32_t kBTile = kNMax * 128;  // bytes of one B tile (hi or lo)
constexpr uint32_t kATile = kBM * 128;    // bytes of one A tile (hi or lo)
constexpr uint32_t kSmemB = 2 * 2 * kBTile;  // 2 stages x (hi, lo)
constexpr uint32_t kSmemA = 2 * 2 * kATile;
constexpr uint32_t kSmemBias = kTcMaxLayers * kNMax * 4;
constexpr uint32_t kSmemTailW = kNMax * kTcTailMaxN * 4;  // tail W^T, rows of 16
constexpr uint32_t kSmemX = kTcTailMaxN * kBM * 4;          // tail K-half exchange [n][row]
constexpr uint32_t kSmemBars = 256;
// Stages the K halves in `halves` (bit h: k = 16h..16h+15) of A chunk c of
// layer l (tile t) into A ring slot j&1 for this thread's row: the input layer
// from global memory, later layers from TMEM (the previous layer's
// activations), split into tf32 hi/lo, 128-byte swizzled.  The slot is known
// free (chunk j-2 was seen consumed); a_full completes when every staging
// thread has arrived.
__device__ __forceinline__ void stage_halves(const TcArgs &p, uint8_t *a0, uint64_t *a_full, uint32_t lane_base, int r,
                                             int halves, int t, int l, int c, uint32_t j) {
    uint8_t *ahi = a0 + (j & 1) * 2 * kATile;
#pragma unroll 1
    for (int h = 0; h < 2; h++) {
        if (!(halves & (1 << h))) continue;
        float v[16];
        const int k0 = c * kKC + 16 * h;
        if (l == 0) {
            const long long row = (long long)t * kBM + r;
            const bool valid = row < p.n;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                const int k = k0 + e;
                v[e] = (valid && k < p.L[0].K) ? __ldg(p.in + (long long)k * p.ld_in + row) : 0.f;
            }
        } else {
            tmem_ld16(lane_base + kTCol + (uint32_t)k0, v);
        }
        put_a16(ahi, ahi + kATile, r, 16 * h, v);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    mbar_arrive(&a_full[j & 1]);
}

// Global chunk after (t, l, c) by `steps` in this CTA's (tile, layer, chunk) order.
__device__ __forceinline__ bool chunk_after(const TcArgs &p, int ntiles, int &t, int &l, int &c, int steps) {
    c += steps;
    while (c >= p.L[l].nch) {
        c -= p.L[l].nch;
        if (++l == p.nlayers) {
            l = 0;
            t += gridDim.x;
            if (t >= ntiles) return false;
        }
    }
    return true;
}

__device__ __forceinline__ void load_b(const TcArgs &p, uint8_t *b0, uint64_t *b_full, int l, int c, uint32_t j) {
    const int s = j & 1;
    mbar_arrive_expect_tx(&b_full[s], 2u * (uint32_t)p.L[l].Np * 128u);
    tma_load_2d(b0 + s * 2 * kBTile, &p.maps[l], &b_full[s], c * kKC, 0);
    tma_load_2d(b0 + s * 2 * kBTile + kBTile, &p.maps[l], &b_full[s], c * kKC, p.L[l].Np);
}

// The MMAs of group g's column half for the A/B ring stage s (layer l): one
// 32-deep product into the group's partial buffer with the small terms (Al*Wh,
// Ah*Wl) first and Ah*Wh last, so the truncating accumulation adds the big
// terms to an accumulator that holds only small ones.
__device__ __forceinline__ void issue_half(uint32_t a_s, uint32_t b_s, uint32_t tmem, int g, int np, int s) {
    // a_s / b_s: shared addresses of the rings; the address fields stay below 2^14
    // (shared memory < 256 KB), so advancing the low word never carries
    const uint32_t ah = desc_lo(a_s + (uint32_t)s * 2 * kATile);
    const uint32_t al = desc_lo(a_s + (uint32_t)s * 2 * kATile + kATile);
    const uint32_t boff = (uint32_t)(g * 128 * 128) >> 4;  // rows 128g.. of the B tiles
    const uint32_t bh = desc_lo(b_s + (uint32_t)s * 2 * kBTile) + boff;
    const uint32_t bl = desc_lo(b_s + (uint32_t)s * 2 * kBTile + kBTile) + boff;
    const uint32_t idesc = idesc_tf32(min(128, np - 128 * g));
    const uint32_t d = tmem + kPCol + (uint32_t)(128 * g);
#pragma unroll
    for (int kk = 0; kk < kKC / 8; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes along K
        umma_tf32_lo(d, al + adv, bh + adv, idesc, kk);
        umma_tf32_lo(d, ah + adv, bl + adv, idesc, 1);
    }
#pragma unroll
    for (int kk = 0; kk < kKC / 8; kk++) {
        const uint32_t adv = (uint32_t)((kk * 32) >> 4);
        umma_tf32_lo(d, ah + adv, bh + adv, idesc, 1);
    }
}

// Layer hand-over by group 0 (which owns columns 0..127): applies the
// activation in place, stages A chunk C0/32 of the next layer (columns
// C0..C0+31) straight from the registers into ring slot j&1, and arrives on
// its a_full (with group 1's empty arrivals: every chunk's a_full counts 256).
template <int ACT>
__device__ __forceinline__ void act_in_place(float (&acc)[128]) {
#pragma unroll
    for (int i = 0; i < 128; i++) acc[i] = tc_act<ACT>(acc[i]);
}
template <int C0>
__device__ __forceinline__ void stage_from_regs(uint8_t *a0, uint64_t *a_full, int r, const float (&acc)[128],
                                                uint32_t j) {
    uint8_t *ahi = a0 + (j & 1) * 2 * kATile;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; e++) v[e] = acc[C0 + 16 * h + e];
        put_a16(ahi, ahi + kATile, r, 16 * h, v);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    mbar_arrive(&a_full[j & 1]);
}

// Applies the activation (the accumulators started at the bias) and writes
// this group's half of the layer output: into TMEM T for the next layer, or to
// global memory.  Columns at and beyond N hold act(0) (their weight rows and
// bias are zero padding) and meet zero weight columns in the next layer, so
// they need no masking.  The code is kept short: it runs once per layer.
template <int ACT>
__device__ __forceinline__ void finalize_half(const TcArgs &p, const float (&acc)[128], int N, int g,
                                              uint32_t lane_base, bool last, int t, int r) {
    if (!last) {
#pragma unroll
        for (int q = 0; q < 8; q++) {
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; e++) v[e] = tc_act<ACT>(acc[16 * q + e]);
            tmem_st16(lane_base + kTCol + (uint32_t)(128 * g + 16 * q), v);
        }
    } else {
        const long long row0 = (long long)t * kBM + r;
        if (row0 < p.n) {
            float *o = p.out + row0 + (long long)(128 * g) * p.ld_out;
#pragma unroll
            for (int q0 = 0; q0 < 128; q0 += 16)
                if (128 * g + q0 < N) {
#pragma unroll
                    for (int q = q0; q < q0 + 16; q++)
                        if (128 * g + q < N) o[(long long)q * p.ld_out] = tc_act<ACT>(acc[q]);
                }
        }
    }
}

// The last layer on the CUDA cores (fp32 FMA), for a narrow output (N <= 16)
// whose MMA chunks would be latency-bound.  tail_dots: this thread's dot
// products over its group's K half, straight from the accumulators of the
// layer before (no TMEM round trip): o[n] = sum over the group's columns
// k < np_prev of act(acc[k]) * W^T[k][n].
template <int ACT, int NP>
__device__ __forceinline__ void tail_dots(float (&o)[NP], const float (&acc)[128], const float *stail, int g,
                                          int np_prev) {
#pragma unroll
    for (int n = 0; n < NP; n++) o[n] = 0.f;
    const uint32_t w_base = smem_u32(stail + 128 * g * kTcTailMaxN);
#pragma unroll
    for (int q = 0; q < 8; q++) {
        if (128 * g + 16 * q >= np_prev) break;
        // RB K-rows at a time (32 weight registers): their weight loads are issued
        // back to back, then their FMAs (one load's latency per RB rows)
        constexpr int RB = NP <= 8 ? 4 : 2;
#pragma unroll
        for (int e0 = 0; e0 < 16; e0 += RB) {
            float4 w4[RB][NP / 4];
#pragma unroll
            for (int e = 0; e < RB; e++) {
                const uint32_t w_row = w_base + (uint32_t)((16 * q + e0 + e) * kTcTailMaxN * 4);
#pragma unroll
                for (int n4 = 0; n4 < NP / 4; n4++)
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(w4[e][n4].x), "=f"(w4[e][n4].y), "=f"(w4[e][n4].z), "=f"(w4[e][n4].w)
                                 : "r"(w_row + 16u * n4));
            }
#pragma unroll
            for (int e = 0; e < RB; e++) {
                const float x = tc_act<ACT>(acc[16 * q + e0 + e]);
#pragma unroll
                for (int n4 = 0; n4 < NP / 4; n4++) {
                    fma2x(o[4 * n4 + 0], o[4 * n4 + 1], x, w4[e][n4].x, w4[e][n4].y);
                    fma2x(o[4 * n4 + 2], o[4 * n4 + 3], x, w4[e][n4].z, w4[e][n4].w);
                }
            }
        }
    }
}

// run_tail: group 1 hands its partial sums to group 0 through shared memory,
// and group 0 adds bias, applies the activation and writes the row.
template <int NP>
__device__ __forceinline__ bool run_tail(const TcArgs &p, uint8_t *base, float (&o)[NP], int g, int r, int t,
                                         uint32_t &xt, int slot) {
    float *sx = reinterpret_cast<float *>(base + kSmemB + kSmemA + kSmemBias + kSmemTailW);
    const float *btail = reinterpret_cast<const float *>(base + kSmemB + kSmemA) + p.nlayers * kNMax;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + kSmemB + kSmemA + kSmemBias + kSmemTailW + kSmemX);
    uint64_t *x_full = bars + 12, *x_empty = bars + 13;
    if (p.tail_k > 128) {  // both groups hold K columns: combine the halves
        if (g == 1) {
            if (!mbar_wait(x_empty, (xt & 1) ^ 1, p.err, 10, t, (int)xt, 0, slot)) return false;
#pragma unroll
            for (int n = 0; n < NP; n++) sx[n * kBM + r] = o[n];
            mbar_arrive(x_full);
        } else {
            if (!mbar_wait(x_full, xt & 1, p.err, 11, t, (int)xt, 0, slot)) return false;
#pragma unroll
            for (int n = 0; n < NP; n++) o[n] += sx[n * kBM + r];
            mbar_arrive(x_empty);
        }
        xt++;
    }
    if (g == 0) {
        const long long row = (long long)t * kBM + r;
        if (row < p.n) {
#pragma unroll
            for (int n = 0; n < NP; n++) {
                if (n >= p.tail_n) break;
                const float y = o[n] + btail[n];
                float z;
                switch (p.tail_act) {
                    case 1: z = tc_act<1>(y); break;
                    case 2: z = tc_act<2>(y); break;
                    case 3: z = tc_act<3>(y); break;
                    default: z = y; break;
                }
                p.out[row + (long long)n * p.ld_out] = z;
            }
        }
    }
    return true;
}

// Warp roles (12 warps, three warpgroups): warps 0-3 and 4-7 are the two
// column groups (drain, stage A, layer ends, tail), at 232 registers; warp 8
// lane 0 issues every MMA of both groups and warp 9 lane 0 streams B, at 40
// registers (setmaxnreg moves registers from the producer warpgroup to the
// groups: 128*40 + 256*232 = 384*168, the launch's registers).  No drain or
// staging waits behind an issuing thread held by the shallow MMA queue.
constexpr int kThreadsWs = 384;
constexpr int kLaunchRegs = 168;  // 65536 / 384 rounded down to 8; setmaxnreg's pool
constexpr int kConsumerRegs = 232, kProducerRegs = 40;
static_assert(kThreadsWs * kLaunchRegs >= 256 * kConsumerRegs + 128 * kProducerRegs, "register split");

__global__ void __launch_bounds__(kThreadsWs, 1) mlp_tc_kernel(const __grid_constant__ TcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base;           // B stage s: hi at b0 + s*2*kBTile, lo + kBTile
    uint8_t *const a0 = base + kSmemB;  // A stage s: hi at a0 + s*2*kATile, lo + kATile
    float *const sbias = reinterpret_cast<float *>(base + kSmemB + kSmemA);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kSmemB + kSmemA + kSmemBias + kSmemTailW + kSmemX);
    uint64_t *const b_full = bars, *const a_full = bars + 2, *const a_empty = bars + 4;
    uint64_t *const p_full = bars + 6, *const p_empty = bars + 8, *const t_ready = bars + 10;
    uint64_t *const mma_done = bars + 11;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nl = p.nlayers;
    const int ntiles = (int)((p.n + kBM - 1) / kBM);

    for (int i = tid; i < nl * kNMax; i += kThreadsWs) {
        const int l = i / kNMax, j = i - l * kNMax;
        sbias[i] = j < p.L[l].Np ? p.arena[p.L[l].b_off + j] : 0.f;
    }
    if (p.tail_n > 0) {  // zero beyond K and tail_np: those activations meet zero weights
        float *stail = reinterpret_cast<float *>(base + kSmemB + kSmemA + kSmemBias);
        for (int i = tid; i < kNMax * kTcTailMaxN; i += kThreadsWs) {
            const int k = i / kTcTailMaxN, n = i - k * kTcTailMaxN;
            stail[i] = (k < p.tail_kp && n < p.tail_np) ? p.arena[p.tail_w_off + (long long)k * p.tail_np + n] : 0.f;
        }
        for (int i = tid; i < kTcTailMaxN; i += kThreadsWs)
            sbias[nl * kNMax + i] = i < p.tail_np ? p.arena[p.tail_b_off + i] : 0.f;
    }
    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&b_full[s], 1);
            mbar_init(&a_full[s], 256);   // every group thread stages a K half of each chunk
            mbar_init(&a_empty[s], 1);    // one tcgen05.commit after both groups' MMAs
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], kBM);  // the group's 128 threads have drained the partial
        }
        mbar_init(t_ready, 256);
        mbar_init(mma_done, 1);
        mbar_init(bars + 12, kBM);  // tail exchange: full, empty
        mbar_init(bars + 13, kBM);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        if (warp == 8 && lane == 0) {
            // ---- MMA issuer: chunk by chunk, group 0's half then group 1's ----
            uint32_t jj = 0, pi0 = 0, pi1 = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x)
                for (int l = 0; l < nl && ok; l++) {
                    const int nch = p.L[l].nch, Np = p.L[l].Np;
                    for (int c = 0; c < nch && ok; c++, jj++) {
                        const int s = jj & 1, where = (l << 8) | c;
                        ok = mbar_wait(&b_full[s], (jj >> 1) & 1, p.err, 2, where, (int)jj, 0, 2) &&
                             mbar_wait(&a_full[s], (jj >> 1) & 1, p.err, 3, where, (int)jj, 0, 2);
                        for (int g = 0; g < 2 && ok; g++) {
                            if (128 * g >= Np) continue;
                            uint32_t &pi = g ? pi1 : pi0;
                            ok = mbar_wait(&p_empty[g], (pi & 1) ^ 1, p.err, 4, where, (int)pi, (int)jj, 2);
                            if (!ok) break;
                            tc_fence_after();
                            issue_half(smem_u32(a0), smem_u32(b0), tmem, g, Np, s);
                            umma_commit(&p_full[g]);
                            pi++;
                        }
                        if (ok) umma_commit(&a_empty[s]);  // the stage is free when these MMAs complete
                    }
                }
            // every MMA issued here has completed before TMEM and shared memory go away
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, p.err, 0);
        } else if (warp == 9 && lane == 0) {
            // ---- B loader: two chunks ahead of the MMAs ----
            for (int l = 0; l < nl; l++) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.maps[l]) : "memory");
            uint32_t issued = 0, jj = 0;
            int t = blockIdx.x, l = 0, c = 0;
            if (t < ntiles) {
                load_b(p, b0, b_full, 0, 0, issued++);
                int t1 = t, l1 = 0, c1 = 0;
                if (chunk_after(p, ntiles, t1, l1, c1, 1)) load_b(p, b0, b_full, l1, c1, issued++);
                bool more = true;
                while (more) {
                    if (!mbar_wait(&a_empty[jj & 1], (jj >> 1) & 1, p.err, 5, (l << 8) | c, (int)jj, (int)issued, 1))
                        break;
                    int t2 = t, l2 = l, c2 = c;
                    if (chunk_after(p, ntiles, t2, l2, c2, 2)) load_b(p, b0, b_full, l2, c2, issued++);
                    jj++;
                    more = chunk_after(p, ntiles, t, l, c, 1);
                }
            }
            // copies issued but not seen consumed (an error path) land first: the
            // last load of each slot completes after the earlier ones
            for (uint32_t k = issued > 2 ? issued - 2 : 0; k < issued; k++)
                mbar_wait(&b_full[k & 1], (k >> 1) & 1, p.err, 0);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
        const int g = warp >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;  // sample row in the tile == TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const int slot = (lane == 0 && quad == 2) ? 3 + g : 0;  // records this group's position on error
        // j: chunks seen consumed; pu: partials of this group drained; tb: T
        // hand-overs between layers seen; xt: tail exchanges seen
        uint32_t j = 0, pu = 0, tb = 0, xt = 0;
        bool ok = true;
        float acc[128];
        if (g == 1) {  // group 1's arrival for chunk 1 when it is a hand-over chunk (no chunk two before)
            int t1 = blockIdx.x, l1 = 0, c1 = 0;
            if (t1 < ntiles && chunk_after(p, ntiles, t1, l1, c1, 1) && l1 > 0 && c1 < 2) mbar_arrive(&a_full[1]);
        }
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            for (int l = 0; l < nl && ok; l++) {
                const int nch = p.L[l].nch, Np = p.L[l].Np;
                const bool has_half = 128 * g < Np;
                if (l == 0) {  // the input layer: chunks 0 and 1 from global memory
                    stage_halves(p, a0, a_full, lane_base, r, 1 << g, t, l, 0, j);
                    if (nch > 1) stage_halves(p, a0, a_full, lane_base, r, 1 << g, t, l, 1, j + 1);
                }
                {  // the accumulators start at the bias (zero beyond Np)
                    const uint32_t b_addr = smem_u32(sbias + l * kNMax + 128 * g);
#pragma unroll
                    for (int q = 0; q < 32; q++)
                        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(acc[4 * q]), "=f"(acc[4 * q + 1]), "=f"(acc[4 * q + 2]), "=f"(acc[4 * q + 3])
                                     : "r"(b_addr + 16u * q));
                }
                for (int c = 0; c < nch && ok; c++) {
                    const uint32_t jj = j + (uint32_t)c;
                    const int s = jj & 1;
                    if (has_half) {
                        // partial of chunk c: add it into acc, four TMEM loads in flight
                        ok = __all_sync(0xffffffffu, mbar_wait(&p_full[g], pu & 1, p.err, 6, (l << 8) | c, (int)pu,
                                                               (int)jj, slot));
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int q0 = 0; q0 < 8; q0 += 4) {
                            if (128 * g + 16 * q0 < Np) {
                                uint32_t v[4][16];
#pragma unroll
                                for (int u = 0; u < 4; u++)
                                    if (128 * g + 16 * (q0 + u) < Np)
                                        tmem_ld16_nw(lane_base + kPCol + (uint32_t)(128 * g + 16 * (q0 + u)), v[u]);
                                tmem_wait_ld();
#pragma unroll
                                for (int u = 0; u < 4; u++)
                                    if (128 * g + 16 * (q0 + u) < Np) {
#pragma unroll
                                        for (int e = 0; e < 16; e += 2)
                                            add2(acc[16 * (q0 + u) + e], acc[16 * (q0 + u) + e + 1], v[u][e],
                                                 v[u][e + 1]);
                                    }
                            }
                        }
                        tc_fence_before();
                        mbar_arrive(&p_empty[g]);
                        pu++;
                    }
                    if (c == 0 && l > 0) {  // T of the previous layer: both halves written (before chunk 2 is staged)
                        ok = __all_sync(0xffffffffu, mbar_wait(t_ready, tb & 1, p.err, 7, l, (int)tb, (int)j, slot));
                        tb++;
                        tc_fence_after();
                        if (!ok) break;
                    }
                    // group 0 takes the last chunk's a_empty at the hand-over to the next layer
                    if (g == 0 && c == nch - 1 && l + 1 < nl) break;
                    // Every thread observes the consumption of every chunk in order, so every
                    // later wait on any ring barrier is at most one phase ahead: no aliasing.
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&a_empty[s], (jj >> 1) & 1, p.err, 5, (l << 8) | c, (int)jj, (int)pu, slot));
                    if (!ok) break;
                    if (c + 2 < nch) {
                        stage_halves(p, a0, a_full, lane_base, r, 1 << g, t, l, c + 2, jj + 2);
                    } else if (g == 1) {
                        // Chunks 0 and 1 of a later layer are staged by group 0 alone at its
                        // hand-over; group 1 arrives for them here, after seeing the chunk two
                        // before consumed, so no chunk can be consumed twice over before group
                        // 1 has seen the one two before it (parity waits stay unambiguous).
                        int t2 = t, l2 = l, c2 = c;
                        if (chunk_after(p, ntiles, t2, l2, c2, 2) && l2 > 0 && c2 < 2) mbar_arrive(&a_full[s]);
                    }
                }
                j += (uint32_t)nch;
                if (!ok) break;
                const bool last = l + 1 == nl;
                const bool to_out = last && p.tail_n == 0;  // else T, for the next layer or the tail
                if (last && !to_out) {  // the CUDA-core tail takes this layer's activations from acc
                    const float *stail = reinterpret_cast<const float *>(base + kSmemB + kSmemA + kSmemBias);
                    const int np_prev = has_half ? Np : 0;
                    if (p.tail_np == 8) {
                        float o[8];
                        switch (p.L[l].act) {
                            case 1: tail_dots<1, 8>(o, acc, stail, g, np_prev); break;
                            case 2: tail_dots<2, 8>(o, acc, stail, g, np_prev); break;
                            case 3: tail_dots<3, 8>(o, acc, stail, g, np_prev); break;
                            default: tail_dots<0, 8>(o, acc, stail, g, np_prev); break;
                        }
                        ok = run_tail<8>(p, base, o, g, r, t, xt, slot);
                    } else {
                        float o[16];
                        switch (p.L[l].act) {
                            case 1: tail_dots<1, 16>(o, acc, stail, g, np_prev); break;
                            case 2: tail_dots<2, 16>(o, acc, stail, g, np_prev); break;
                            case 3: tail_dots<3, 16>(o, acc, stail, g, np_prev); break;
                            default: tail_dots<0, 16>(o, acc, stail, g, np_prev); break;
                        }
                        ok = run_tail<16>(p, base, o, g, r, t, xt, slot);
                    }
                } else if (!last && g == 0) {
                    // Hand-over by group 0: chunk 0 of the next layer straight from the
                    // registers into the slot of chunk j-2 (seen consumed), so the issuer can
                    // queue it behind group 1's last MMAs; columns 64..127 into T for the
                    // other chunks; chunk 1 into the last chunk's slot once it is consumed.
                    switch (p.L[l].act) {
                        case 1: act_in_place<1>(acc); break;
                        case 2: act_in_place<2>(acc); break;
                        case 3: act_in_place<3>(acc); break;
                        default: break;
                    }
                    const int nl1 = l + 1;
                    stage_from_regs<0>(a0, a_full, r, acc, j);
#pragma unroll
                    for (int q = 4; q < 8; q++) {
                        float v[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) v[e] = acc[16 * q + e];
                        tmem_st16(lane_base + kTCol + (uint32_t)(16 * q), v);
                    }
                    const uint32_t jl = j - 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[jl & 1], (jl >> 1) & 1, p.err, 5,
                                                           (l << 8) | (nch - 1), (int)jl, (int)pu, slot));
                    if (!ok) break;
                    if (p.L[nl1].nch > 1) stage_from_regs<32>(a0, a_full, r, acc, j + 1);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    mbar_arrive(t_ready);
                } else if (has_half || !last) {
                    if (has_half) {
                        switch (p.L[l].act) {
                            case 1: finalize_half<1>(p, acc, p.L[l].N, g, lane_base, to_out, t, r); break;
                            case 2: finalize_half<2>(p, acc, p.L[l].N, g, lane_base, to_out, t, r); break;
                            case 3: finalize_half<3>(p, acc, p.L[l].N, g, lane_base, to_out, t, r); break;
                            default: finalize_half<0>(p, acc, p.L[l].N, g, lane_base, to_out, t, r); break;
                        }
                    }
                    if (!last) {  // group 1: its half of T for the next layer
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        tc_fence_before();
                        mbar_arrive(t_ready);
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ============================================================================
// Chains no wider than 128 (every layer's Np <= 128): in mlp_tc_kernel one
// column group would hold all the columns while the other idled, and a tile's
// layer ends and tail would stall the tensor pipe.  Here each group takes a
// tile of its own (group g the tiles blockIdx.x + (2k+g)*gridDim.x) with its
// own 2-slot A ring, its own TMEM partial buffer and T region (columns
// 128g..128g+127); the B ring is shared, one stage per chunk position (the
// same weights serve both tiles).  The issuer takes chunk c of layer l for
// group 0's tile, then for group 1's, so one group's layer end overlaps the
// other group's MMAs.  Each thread stages and reads only its own sample row,
// so the groups never wait for one another (only on the shared B ring).
// ============================================================================
constexpr uint32_t kDualBTile = 128 * 128;            // Np <= 128 rows of 128 bytes
constexpr uint32_t kDualSmemB = 2 * 2 * kDualBTile;  // 2 stages x (hi, lo)
constexpr uint32_t kDualSmemA = 2 * 2 * 2 * kATile;  // 2 groups x 2 slots x (hi, lo)
constexpr uint32_t kDualSmemBias = (kTcMaxLayers + 1) * 128 * 4;  // per layer, then the tail's
constexpr uint32_t kDualSmemTailW = 128 * kTcTailMaxN * 4;
size_t mlp_tc_dual_smem() { return 1024 + kDualSmemB + kDualSmemA + kDualSmemBias + kDualSmemTailW + kSmemBars; }

// (pair k, layer l, chunk c) after `steps` chunk positions in this CTA's order
__device__ __forceinline__ bool pair_after(const TcArgs &p, int npairs, int &k, int &l, int &c, int steps) {
    c += steps;
    while (c >= p.L[l].nch) {
        c -= p.L[l].nch;
        if (++l == p.nlayers) {
            l = 0;
            if (++k >= npairs) return false;
        }
    }
    return true;
}

// One row of the CUDA-core tail: bias, activation, the outputs of `row` (the
// activation switch outside the per-output loop keeps the registers down).
template <int NP, int ACT>
__device__ __forceinline__ void write_tail_row_act(const TcArgs &p, const float (&o)[NP], const float *btail,
                                                   long long row) {
#pragma unroll
    for (int n = 0; n < NP; n++) {
        if (n >= p.tail_n) break;
        p.out[row + (long long)n * p.ld_out] = tc_act<ACT>(o[n] + btail[n]);
    }
}
template <int NP>
__device__ __forceinline__ void write_tail_row(const TcArgs &p, const float (&o)[NP], const float *btail, long long row) {
    if (row >= p.n) return;
    switch (p.tail_act) {
        case 1: write_tail_row_act<NP, 1>(p, o, btail, row); break;
        case 2: write_tail_row_act<NP, 2>(p, o, btail, row); break;
        case 3: write_tail_row_act<NP, 3>(p, o, btail, row); break;
        default: write_tail_row_act<NP, 0>(p, o, btail, row); break;
    }
}

__device__ __forceinline__ void load_b_dual(const TcArgs &p, uint8_t *b0, uint64_t *b_full, int l, int c, uint32_t m) {
    const int s = m & 1;
    mbar_arrive_expect_tx(&b_full[s], 2u * (uint32_t)p.L[l].Np * 128u);
    tma_load_2d(b0 + s * 2 * kDualBTile, &p.maps[l], &b_full[s], c * kKC, 0);
    tma_load_2d(b0 + s * 2 * kDualBTile + kDualBTile, &p.maps[l], &b_full[s], c * kKC, p.L[l].Np);
}

__global__ void __launch_bounds__(kThreadsWs, 1) mlp_tc_dual_kernel(const __grid_constant__ TcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base;               // B stage s: hi at b0 + s*2*kDualBTile, lo + kDualBTile
    uint8_t *const a0 = base + kDualSmemB;  // group g, slot s: hi at a0 + (2g+s)*2*kATile, lo + kATile
    float *const sbias = reinterpret_cast<float *>(base + kDualSmemB + kDualSmemA);  // [l][128], tail at [nl]
    float *const stail = reinterpret_cast<float *>(base + kDualSmemB + kDualSmemA + kDualSmemBias);
    uint64_t *const bars =
        reinterpret_cast<uint64_t *>(base + kDualSmemB + kDualSmemA + kDualSmemBias + kDualSmemTailW);
    uint64_t *const b_full = bars, *const b_empty = bars + 2;
    uint64_t *const a_full = bars + 4, *const a_empty = bars + 8;  // [group][slot]
    uint64_t *const p_full = bars + 12, *const p_empty = bars + 14, *const mma_done = bars + 16;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 18);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nl = p.nlayers;
    const int ntiles = (int)((p.n + kBM - 1) / kBM);
    // tile pairs of this CTA: pair k holds tiles blockIdx.x + (2k + g) * gridDim.x
    const int npairs = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (2 * (int)gridDim.x) + 1 : 0;

    for (int i = tid; i < nl * 128; i += kThreadsWs) {
        const int l = i / 128, j = i - l * 128;
        sbias[i] = j < p.L[l].Np ? p.arena[p.L[l].b_off + j] : 0.f;
    }
    if (p.tail_n > 0) {  // zero beyond K and tail_np: those activations meet zero weights
        for (int i = tid; i < 128 * kTcTailMaxN; i += kThreadsWs) {
            const int k = i / kTcTailMaxN, n = i - k * kTcTailMaxN;
            stail[i] = (k < p.tail_kp && n < p.tail_np) ? p.arena[p.tail_w_off + (long long)k * p.tail_np + n] : 0.f;
        }
        for (int i = tid; i < kTcTailMaxN; i += kThreadsWs)
            sbias[nl * 128 + i] = i < p.tail_np ? p.arena[p.tail_b_off + i] : 0.f;
    }
    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);     // one tcgen05.commit after both tiles' MMAs
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], kBM);   // the group's 128 threads have drained the partial
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(&a_full[i], kBM);    // the group's 128 threads have staged the chunk
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        if (warp == 8 && lane == 0) {
            // ---- MMA issuer: chunk (l, c) for group 0's tile, then for group 1's ----
            uint32_t m = 0, jg0 = 0, jg1 = 0, pi0 = 0, pi1 = 0;
            bool ok = true;
            for (int k = 0; k < npairs && ok; k++) {
                const int ng = (int)blockIdx.x + (2 * k + 1) * (int)gridDim.x < ntiles ? 2 : 1;
                for (int l = 0; l < nl && ok; l++) {
                    const int nch = p.L[l].nch;
                    const uint32_t idesc = idesc_tf32(p.L[l].Np);
                    for (int c = 0; c < nch && ok; c++, m++) {
                        const int sb = m & 1;
                        ok = mbar_wait(&b_full[sb], (m >> 1) & 1, p.err, 2, (l << 8) | c, (int)m, 0, 2);
                        for (int g = 0; g < ng && ok; g++) {
                            uint32_t &jg = g ? jg1 : jg0, &pi = g ? pi1 : pi0;
                            const uint32_t sa = jg & 1;
                            ok = mbar_wait(&a_full[2 * g + sa], (jg >> 1) & 1, p.err, 3, (l << 8) | c, (int)jg, g, 2) &&
                                 mbar_wait(&p_empty[g], (pi & 1) ^ 1, p.err, 4, (l << 8) | c, (int)pi, g, 2);
                            if (!ok) break;
                            tc_fence_after();
                            const uint64_t ah = desc_kmajor_sw128(smem_u32(a0 + (2 * g + sa) * 2 * kATile));
                            const uint64_t al = desc_kmajor_sw128(smem_u32(a0 + (2 * g + sa) * 2 * kATile + kATile));
                            const uint64_t bh = desc_kmajor_sw128(smem_u32(b0 + sb * 2 * kDualBTile));
                            const uint64_t bl = desc_kmajor_sw128(smem_u32(b0 + sb * 2 * kDualBTile + kDualBTile));
                            const uint32_t d = tmem + kPCol + (uint32_t)(128 * g);
#pragma unroll
                            for (int kk = 0; kk < kKC / 8; kk++) {
                                const uint64_t adv = (uint64_t)((kk * 32) >> 4);
                                umma_tf32(d, al + adv, bh + adv, idesc, kk);
                                umma_tf32(d, ah + adv, bl + adv, idesc, 1);
                            }
#pragma unroll
                            for (int kk = 0; kk < kKC / 8; kk++) {
                                const uint64_t adv = (uint64_t)((kk * 32) >> 4);
                                umma_tf32(d, ah + adv, bh + adv, idesc, 1);
                            }
                            umma_commit(&p_full[g]);
                            umma_commit(&a_empty[2 * g + sa]);
                            pi++;
                            jg++;
                        }
                        if (ok) umma_commit(&b_empty[sb]);  // both tiles' MMAs of this B stage
                    }
                }
            }
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, p.err, 0);
        } else if (warp == 9 && lane == 0) {
            // ---- B loader: two chunk positions ahead ----
            for (int l = 0; l < nl; l++) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.maps[l]) : "memory");
            uint32_t issued = 0;
            if (npairs > 0) {
                load_b_dual(p, b0, b_full, 0, 0, issued++);
                int k1 = 0, l1 = 0, c1 = 0;
                if (pair_after(p, npairs, k1, l1, c1, 1)) load_b_dual(p, b0, b_full, l1, c1, issued++);
                int k = 0, l = 0, c = 0;
                uint32_t m = 0;
                bool more = true;
                while (more) {
                    if (!mbar_wait(&b_empty[m & 1], (m >> 1) & 1, p.err, 5, (l << 8) | c, (int)m, (int)issued, 1))
                        break;
                    int k2 = k, l2 = l, c2 = c;
                    if (pair_after(p, npairs, k2, l2, c2, 2)) load_b_dual(p, b0, b_full, l2, c2, issued++);
                    m++;
                    more = pair_after(p, npairs, k, l, c, 1);
                }
            }
            // copies issued but not seen consumed (an error path) land first
            for (uint32_t q = issued > 2 ? issued - 2 : 0; q < issued; q++)
                mbar_wait(&b_full[q & 1], (q >> 1) & 1, p.err, 0);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
        const int g = warp >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;  // sample row in the tile == TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t t_base = lane_base + 128u * g;  // this group's T columns (kTCol + 128g)
        uint8_t *const ag = a0 + 2 * g * 2 * kATile;  // this group's two A slots
        uint64_t *const af = a_full + 2 * g, *const ae = a_empty + 2 * g;
        const int slot = (lane == 0 && quad == 2) ? 3 + g : 0;
        uint32_t j = 0, pu = 0;  // chunks of this group seen consumed; partials drained
        bool ok = true;
        float acc[128];
        for (int k = 0; k < npairs && ok; k++) {
            const int t = (int)blockIdx.x + (2 * k + g) * (int)gridDim.x;
            if (t >= ntiles) break;
            for (int l = 0; l < nl && ok; l++) {
                const int nch = p.L[l].nch, Np = p.L[l].Np;
                if (l == 0) {  // the input layer: chunks 0 and 1 from global memory
                    stage_halves(p, ag, af, t_base, r, 3, t, 0, 0, j);
                    if (nch > 1) stage_halves(p, ag, af, t_base, r, 3, t, 0, 1, j + 1);
                }
                {  // the accumulators start at the bias (zero beyond Np)
                    const uint32_t b_addr = smem_u32(sbias + l * 128);
#pragma unroll
                    for (int q = 0; q < 32; q++)
                        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(acc[4 * q]), "=f"(acc[4 * q + 1]), "=f"(acc[4 * q + 2]), "=f"(acc[4 * q + 3])
                                     : "r"(b_addr + 16u * q));
                }
                for (int c = 0; c < nch && ok; c++) {
                    const uint32_t jj = j + (uint32_t)c;
                    const int s = jj & 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&p_full[g], pu & 1, p.err, 6, (l << 8) | c, (int)pu,
                                                           (int)jj, slot));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int q0 = 0; q0 < 8; q0 += 4) {
                        if (16 * q0 < Np) {
                            uint32_t v[4][16];
#pragma unroll
                            for (int u = 0; u < 4; u++)
                                if (16 * (q0 + u) < Np)
                                    tmem_ld16_nw(lane_base + kPCol + (uint32_t)(128 * g + 16 * (q0 + u)), v[u]);
                            tmem_wait_ld();
#pragma unroll
                            for (int u = 0; u < 4; u++)
                                if (16 * (q0 + u) < Np) {
#pragma unroll
                                    for (int e = 0; e < 16; e += 2)
                                        add2(acc[16 * (q0 + u) + e], acc[16 * (q0 + u) + e + 1], v[u][e], v[u][e + 1]);
                                }
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&p_empty[g]);
                    pu++;
                    // the hand-over takes the last chunk's a_empty
                    if (c == nch - 1 && l + 1 < nl) break;
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&ae[s], (jj >> 1) & 1, p.err, 5, (l << 8) | c, (int)jj, (int)pu, slot));
                    if (!ok) break;
                    if (c + 2 < nch) stage_halves(p, ag, af, t_base, r, 3, t, l, c + 2, jj + 2);
                }
                j += (uint32_t)nch;
                if (!ok) break;
                const bool last = l + 1 == nl;
                if (last && p.tail_n > 0) {  // the CUDA-core tail over all of this tile's columns
                    const long long row = (long long)t * kBM + r;
                    const float *btail = sbias + nl * 128;
                    if (p.tail_np == 8) {
                        float o[8];
                        switch (p.L[l].act) {
                            case 1: tail_dots<1, 8>(o, acc, stail, 0, Np); break;
                            case 2: tail_dots<2, 8>(o, acc, stail, 0, Np); break;
                            case 3: tail_dots<3, 8>(o, acc, stail, 0, Np); break;
                            default: tail_dots<0, 8>(o, acc, stail, 0, Np); break;
                        }
                        write_tail_row<8>(p, o, btail, row);
                    } else {
                        float o[16];
                        switch (p.L[l].act) {
                            case 1: tail_dots<1, 16>(o, acc, stail, 0, Np); break;
                            case 2: tail_dots<2, 16>(o, acc, stail, 0, Np); break;
                            case 3: tail_dots<3, 16>(o, acc, stail, 0, Np); break;
                            default: tail_dots<0, 16>(o, acc, stail, 0, Np); break;
                        }
                        write_tail_row<16>(p, o, btail, row);
                    }
                } else if (last) {  // the last layer to global memory
                    switch (p.L[l].act) {
                        case 1: finalize_half<1>(p, acc, p.L[l].N, 0, lane_base, true, t, r); break;
                        case 2: finalize_half<2>(p, acc, p.L[l].N, 0, lane_base, true, t, r); break;
                        case 3: finalize_half<3>(p, acc, p.L[l].N, 0, lane_base, true, t, r); break;
                        default: finalize_half<0>(p, acc, p.L[l].N, 0, lane_base, true, t, r); break;
                    }
                } else {
                    // Hand-over: chunk 0 of the next layer straight from the registers into
                    // the slot of chunk j-2 (seen consumed), columns 64..127 into this group's
                    // T for the later chunks, chunk 1 once the last chunk's slot is free.
                    switch (p.L[l].act) {
                        case 1: act_in_place<1>(acc); break;
                        case 2: act_in_place<2>(acc); break;
                        case 3: act_in_place<3>(acc); break;
                        default: break;
                    }
                    stage_from_regs<0>(ag, af, r, acc, j);
#pragma unroll
                    for (int q = 4; q < 8; q++) {
                        float v[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) v[e] = acc[16 * q + e];
                        tmem_st16(t_base + kTCol + (uint32_t)(16 * q), v);
                    }
                    const uint32_t jl = j - 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&ae[jl & 1], (jl >> 1) & 1, p.err, 5, (l << 8) | (nch - 1),
                                                           (int)jl, (int)pu, slot));
                    if (!ok) break;
                    if (p.L[l + 1].nch > 1) stage_from_regs<32>(ag, af, r, acc, j + 1);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ============================================================================
// LSTM layer on the tensor cores.  The chunk stream of a tile is T steps of
// nch = nx + nh K-chunks: x_t (from global memory) then h_{t-1} (from TMEM T,
// columns 0..Hh-1, written by the cell update of the step before).  Roles,
// rings, 3xTF32 partials, turn order and bounded waits are those of
// mlp_tc_kernel; the "layer end" is the cell update: each thread holds the
// gates of its row for its group's 32 units (columns 4u+q), keeps c in TMEM T
// (columns 128+32g+u) and writes h to T and, when asked, to y.  The next step's
// x chunks are staged and its first chunk issued before the cell update, so
// those MMAs overlap it.
// ============================================================================

// Shared memory of lstm_tc_kernel: the B and A rings of mlp_tc_kernel, the gate
// bias, and a buffer for the next step's x (up to two chunks, [k][128 rows] fp32)
// filled by cp.async one step ahead.
constexpr uint32_t kLstmBias = 1024, kLstmXBuf = 2 * kKC * kBM * 4;
constexpr int kLstmMaxNxPrefetch = 2;
size_t lstm_tc_smem() { return 1024 + kSmemB + kSmemA + kLstmBias + kLstmXBuf + kSmemBars; }

__device__ __forceinline__ void cp_async4_zfill(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}

// Copies (cp.async) this thread's row of the x chunks of step s into the buffer.
__device__ __forceinline__ void lstm_prefetch_x(const TcLstmArgs &p, float *xbuf, int r, int halves, int t, int s) {
    const long long row = (long long)t * kBM + r;
    const bool valid = row < p.n;
    for (int q = 0; q < p.nx; q++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (!(halves & (1 << h))) continue;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                const int k = q * kKC + 16 * h + e;
                const bool ok = valid && k < p.I;
                cp_async4_zfill(xbuf + (size_t)k * kBM + r, ok ? p.x + (long long)(s + (long long)p.T * k) * p.ld_x + row : p.x,
                                ok);
            }
        }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Stages the K halves in `halves` of chunk q of step s (tile t) into A slot j&1:
// q < nx from x (feature k = 32q + 16h + e, row s + T*k), else from T (h).
__device__ __forceinline__ void lstm_stage(const TcLstmArgs &p, uint8_t *a0, uint64_t *a_full, uint32_t lane_base,
                                           int r, int halves, int t, int s, int q, uint32_t j, const float *xbuf) {
    uint8_t *ahi = a0 + (j & 1) * 2 * kATile;
    if (xbuf && q < p.nx) asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll 1
    for (int h = 0; h < 2; h++) {
        if (!(halves & (1 << h))) continue;
        float v[16];
        if (xbuf && q < p.nx) {  // prefetched by this thread
#pragma unroll
            for (int e = 0; e < 16; e++) v[e] = xbuf[(size_t)(q * kKC + 16 * h + e) * kBM + r];
        } else if (q < p.nx) {
            const long long row = (long long)t * kBM + r;
            const bool valid = row < p.n;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                const int k = q * kKC + 16 * h + e;
                v[e] = (valid && k < p.I) ? __ldg(p.x + (long long)(s + (long long)p.T * k) * p.ld_x + row) : 0.f;
            }
        } else {
            tmem_ld16(lane_base + kTCol + (uint32_t)((q - p.nx) * kKC + 16 * h), v);
        }
        put_a16(ahi, ahi + kATile, r, 16 * h, v);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    mbar_arrive(&a_full[j & 1]);
}

__device__ __forceinline__ void lstm_load_b(const TcLstmArgs &p, uint8_t *b0, uint64_t *b_full, int q, uint32_t j) {
    const int s = j & 1;
    mbar_arrive_expect_tx(&b_full[s], 2u * (uint32_t)p.Np * 128u);
    tma_load_2d(b0 + s * 2 * kBTile, &p.map, &b_full[s], q * kKC, 0);
    tma_load_2d(b0 + s * 2 * kBTile + kBTile, &p.map, &b_full[s], q * kKC, p.Np);
}

// The MMAs of group g's gate columns for the ring stage s, as mlp_tc_kernel's
// issue_half; `first`: the chunk starts its partial (else it accumulates).
__device__ __forceinline__ void lstm_issue_half(const TcLstmArgs &p, uint8_t *a0, uint8_t *b0, uint32_t tmem, int g,
                                                int s, bool first) {
    const uint64_t ah = desc_kmajor_sw128(smem_u32(a0 + s * 2 * kATile));
    const uint64_t al = desc_kmajor_sw128(smem_u32(a0 + s * 2 * kATile + kATile));
    const uint64_t boff = (uint64_t)(g * 128 * 128) >> 4;
    const uint64_t bh = desc_kmajor_sw128(smem_u32(b0 + s * 2 * kBTile)) + boff;
    const uint64_t bl = desc_kmajor_sw128(smem_u32(b0 + s * 2 * kBTile + kBTile)) + boff;
    const uint32_t idesc = idesc_tf32(min(128, p.Np - 128 * g));
    const uint32_t d = tmem + kPCol + (uint32_t)(128 * g);
#pragma unroll
    for (int kk = 0; kk < kKC / 8; kk++) {
        const uint64_t adv = (uint64_t)((kk * 32) >> 4);
        umma_tf32(d, al + adv, bh + adv, idesc, (kk > 0 || !first) ? 1u : 0u);
        umma_tf32(d, ah + adv, bl + adv, idesc, 1);
    }
#pragma unroll
    for (int kk = 0; kk < kKC / 8; kk++) {
        const uint64_t adv = (uint64_t)((kk * 32) >> 4);
        umma_tf32(d, ah + adv, bh + adv, idesc, 1);
    }
}

// Warp roles as in mlp_tc_kernel: warps 0-7 the two column groups (drain,
// stage, cell update), warp 8 lane 0 the MMA issuer, warp 9 lane 0 the B loader.
__global__ void __launch_bounds__(kThreadsWs, 1) lstm_tc_kernel(const __grid_constant__ TcLstmArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base;
    uint8_t *const a0 = base + kSmemB;
    float *const sbias = reinterpret_cast<float *>(base + kSmemB + kSmemA);
    float *const xbuf_all = reinterpret_cast<float *>(base + kSmemB + kSmemA + kLstmBias);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kSmemB + kSmemA + kLstmBias + kLstmXBuf);
    uint64_t *const b_full = bars, *const a_full = bars + 2, *const a_empty = bars + 4;
    uint64_t *const p_full = bars + 6, *const p_empty = bars + 8, *const t_ready = bars + 10;
    uint64_t *const mma_done = bars + 11;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nch = p.nx + p.nh, T = p.T;
    const int ntiles = (int)((p.n + kBM - 1) / kBM);
    // chunks of this CTA: its tiles x T steps x nch
    const long long my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const long long total = my_tiles * T * nch;

    for (int i = tid; i < kNMax; i += kThreadsWs) sbias[i] = i < p.Np ? p.arena[p.b_off + i] : 0.f;
    static_assert(kNMax * 4 <= kLstmBias, "bias area");
    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&b_full[s], 1);
            mbar_init(&a_full[s], 256);  // every group thread stages a K half of each chunk
            mbar_init(&a_empty[s], 1);
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], kBM);
        }
        mbar_init(t_ready, 256);
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        if (warp == 8 && lane == 0) {
            // ---- MMA issuer: chunk by chunk, group 0's gates then group 1's; a
            // step's x chunks accumulate into one partial, its h chunks into another ----
            uint32_t pi0 = 0, pi1 = 0;
            bool ok = true;
            for (long long q = 0; q < total && ok; q++) {
                const uint32_t jj = (uint32_t)q;
                const int s = jj & 1, c = (int)(q % nch);
                const bool first = c == 0 || c == p.nx, part_end = c == p.nx - 1 || c == nch - 1;
                ok = mbar_wait(&b_full[s], (jj >> 1) & 1, p.err, 2, c, (int)jj, 0, 2) &&
                     mbar_wait(&a_full[s], (jj >> 1) & 1, p.err, 3, c, (int)jj, 0, 2);
                for (int g = 0; g < 2 && ok; g++) {
                    if (128 * g >= p.Np) continue;
                    uint32_t &pi = g ? pi1 : pi0;
                    if (first) ok = mbar_wait(&p_empty[g], (pi & 1) ^ 1, p.err, 4, c, (int)pi, (int)jj, 2);
                    if (!ok) break;
                    tc_fence_after();
                    lstm_issue_half(p, a0, b0, tmem, g, s, first);
                    if (part_end) {
                        umma_commit(&p_full[g]);
                        pi++;
                    }
                }
                if (ok) umma_commit(&a_empty[s]);
            }
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, p.err, 0);
        } else if (warp == 9 && lane == 0) {
            // ---- B loader: two chunks ahead ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map) : "memory");
            uint32_t issued = 0;
            for (long long q = 0; q < 2 && q < total; q++) lstm_load_b(p, b0, b_full, (int)(q % nch), issued++);
            for (long long q = 0; q + 2 < total; q++) {
                const uint32_t jj = (uint32_t)q;
                if (!mbar_wait(&a_empty[jj & 1], (jj >> 1) & 1, p.err, 5, (int)(q % nch), (int)jj, (int)issued, 1)) break;
                lstm_load_b(p, b0, b_full, (int)((q + 2) % nch), issued++);
            }
            for (uint32_t k = issued > 2 ? issued - 2 : 0; k < issued; k++)
                mbar_wait(&b_full[k & 1], (k >> 1) & 1, p.err, 0);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
        const int g = warp >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const int halves = 1 << g;
        const int slot = (lane == 0 && quad == 2) ? 3 + g : 0;
        const bool has_half = 128 * g < p.Np;
        // the next step's x through the prefetch buffer (x parts of up to two chunks)
        float *const xbuf = p.nx <= kLstmMaxNxPrefetch ? xbuf_all : nullptr;
        uint32_t j = 0, pu = 0, tb = 0;
        bool ok = true;
        float acc[128];
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const long long row = (long long)t * kBM + r;
            const bool valid = row < p.n;
            // the initial state: h0 into T columns 32g.., c0 into T columns 128+32g..
            if (has_half) {
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    float hv[16], cv[16];
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const int unit = 32 * g + 16 * hf + e;
                        float h0 = 0.f, c0 = 0.f;
                        if (unit < p.H && valid) {
                            h0 = p.h0 ? p.h0[(long long)unit * p.ld_h0 + row]
                                      : (p.h0_const >= 0 ? p.arena[p.h0_const + unit] : 0.f);
                            c0 = p.c0 ? p.c0[(long long)unit * p.ld_c0 + row]
                                      : (p.c0_const >= 0 ? p.arena[p.c0_const + unit] : 0.f);
                        }
                        hv[e] = h0;
                        cv[e] = c0;
                    }
                    tmem_st16(lane_base + kTCol + (uint32_t)(32 * g + 16 * hf), hv);
                    tmem_st16(lane_base + kTCol + (uint32_t)(128 + 32 * g + 16 * hf), cv);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(t_ready);
            ok = __all_sync(0xffffffffu, mbar_wait(t_ready, tb & 1, p.err, 7, 0, (int)tb, (int)j, slot));
            tb++;
            tc_fence_after();
            if (!ok) break;
            // step 0: chunks 0 and 1 staged here; later steps had theirs staged during
            // the step before
            lstm_stage(p, a0, a_full, lane_base, r, halves, t, 0, 0, j, nullptr);
            if (nch > 1) lstm_stage(p, a0, a_full, lane_base, r, halves, t, 0, 1, j + 1, nullptr);
            for (int st = 0; st < T && ok; st++) {
                if (has_half) {
                    const uint32_t b_addr = smem_u32(sbias + 128 * g);
#pragma unroll
                    for (int q = 0; q < 32; q++)
                        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(acc[4 * q]), "=f"(acc[4 * q + 1]), "=f"(acc[4 * q + 2]), "=f"(acc[4 * q + 3])
                                     : "r"(b_addr + 16u * q));
                }
                for (int c = 0; c < nch && ok; c++) {
                    const uint32_t jj = j + (uint32_t)c;
                    const int s = jj & 1;
                    // the x part of the gates is one partial, the h part another (the
                    // truncating TMEM accumulation over 64 K stays ~1e-7 here: small gates)
                    if (has_half && (c == p.nx - 1 || c == nch - 1)) {
                        ok = __all_sync(0xffffffffu, mbar_wait(&p_full[g], pu & 1, p.err, 6, (st << 8) | c, (int)pu,
                                                               (int)jj, slot));
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int q0 = 0; q0 < 8; q0 += 4) {
                            if (128 * g + 16 * q0 < p.Np) {
                                uint32_t v[4][16];
#pragma unroll
                                for (int u = 0; u < 4; u++)
                                    if (128 * g + 16 * (q0 + u) < p.Np)
                                        tmem_ld16_nw(lane_base + kPCol + (uint32_t)(128 * g + 16 * (q0 + u)), v[u]);
                                tmem_wait_ld();
#pragma unroll
                                for (int u = 0; u < 4; u++)
                                    if (128 * g + 16 * (q0 + u) < p.Np) {
#pragma unroll
                                        for (int e = 0; e < 16; e += 2)
                                            add2(acc[16 * (q0 + u) + e], acc[16 * (q0 + u) + e + 1], v[u][e],
                                                 v[u][e + 1]);
                                    }
                            }
                        }
                        tc_fence_before();
                        mbar_arrive(&p_empty[g]);
                        pu++;
                    }
                    ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[s], (jj >> 1) & 1, p.err, 5, (st << 8) | c,
                                                           (int)jj, (int)pu, slot));
                    if (!ok) break;
                    // stage chunk c+2: of this step, or an x chunk of the next step (an h
                    // chunk of the next step waits for this step's cell update).  The next
                    // step's x is prefetched at c = nx-1, after this iteration's staging so
                    // that it runs beside the h MMAs -- unless this iteration already stages
                    // the next step's x (two-chunk steps)
                    const int q2 = c + 2;
                    const bool prefetch = c == p.nx - 1 && xbuf && st + 1 < T;
                    if (prefetch && q2 >= nch) lstm_prefetch_x(p, xbuf, r, halves, t, st + 1);
                    if (q2 < nch) lstm_stage(p, a0, a_full, lane_base, r, halves, t, st, q2, jj + 2, xbuf);
                    else if (st + 1 < T && q2 - nch < p.nx)
                        lstm_stage(p, a0, a_full, lane_base, r, halves, t, st + 1, q2 - nch, jj + 2, xbuf);
                    if (prefetch && q2 < nch) lstm_prefetch_x(p, xbuf, r, halves, t, st + 1);
                }
                j += (uint32_t)nch;
                if (!ok) break;
                // cell update (layers.f90 lstm_cell): gates of unit u at acc[4u..4u+3]
                if (has_half) {
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        float cv[16], hv[16];
                        tmem_ld16(lane_base + kTCol + (uint32_t)(128 + 32 * g + 16 * hf), cv);
#pragma unroll
                        for (int e = 0; e < 16; e++) {
                            const int u = 16 * hf + e;
                            const float ig = tc_act<3>(acc[4 * u]), fg = tc_act<3>(acc[4 * u + 1]);
                            const float gg = tc_act<2>(acc[4 * u + 2]), og = tc_act<3>(acc[4 * u + 3]);
                            cv[e] = fg * cv[e] + ig * gg;
                            hv[e] = og * tc_act<2>(cv[e]);
                        }
                        tmem_st16(lane_base + kTCol + (uint32_t)(128 + 32 * g + 16 * hf), cv);
                        tmem_st16(lane_base + kTCol + (uint32_t)(32 * g + 16 * hf), hv);
                        if (valid) {
#pragma unroll
                            for (int e = 0; e < 16; e++) {
                                const int unit = 32 * g + 16 * hf + e;
                                if (unit < p.H) {
                                    if (p.y) p.y[(long long)(st + (long long)T * unit) * p.ld_y + row] = hv[e];
                                    if (st + 1 == T) {
                                        if (p.hn) p.hn[(long long)unit * p.ld_hn + row] = hv[e];
                                        if (p.cn) p.cn[(long long)unit * p.ld_cn + row] = cv[e];
                                    }
                                }
                            }
                        }
                    }
                }
                // h_t in T for the next step (both groups' units feed both groups' MMAs)
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(t_ready);
                ok = __all_sync(0xffffffffu, mbar_wait(t_ready, tb & 1, p.err, 7, st, (int)tb, (int)j, slot));
                tb++;
                tc_fence_after();
                if (!ok) break;
                // the next step's chunk 1 when it is an h chunk (nx == 1)
                if (st + 1 < T && nch > 1 && p.nx == 1)
                    lstm_stage(p, a0, a_full, lane_base, r, halves, t, st + 1, 1, j + 1, xbuf);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

size_t mlp_tc_smem_bytes() { return 1024 + kSmemB + kSmemA + kSmemBias + kSmemTailW + kSmemX + kSmemBars; }

bool tc_register_split_ok() {
    cudaFuncAttributes a{}, b{}, c{};
    if (cudaFuncGetAttributes(&a, mlp_tc_kernel) != cudaSuccess ||
        cudaFuncGetAttributes(&b, lstm_tc_kernel) != cudaSuccess ||
        cudaFuncGetAttributes(&c, mlp_tc_dual_kernel) != cudaSuccess) {
        (void)cudaGetLastError();
        return true;
    }
    return a.numRegs == kLaunchRegs && b.numRegs == kLaunchRegs && c.numRegs == kLaunchRegs;
}

cudaError_t mlp_tc_configure() {
    cudaError_t e =
        cudaFuncSetAttribute(mlp_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mlp_tc_smem_bytes());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(mlp_tc_dual_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mlp_tc_dual_smem());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(lstm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lstm_tc_smem());
}

cudaError_t launch_lstm_tc(const TcLstmArgs &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + kBM - 1) / kBM;
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    static const int regs = [] {
        cudaFuncAttributes fa{};
        return cudaFuncGetAttributes(&fa, lstm_tc_kernel) == cudaSuccess ? fa.numRegs : -1;
    }();
    if (regs != kLaunchRegs) return cudaErrorInvalidConfiguration;  // the setmaxnreg split needs exactly these
    lstm_tc_kernel<<<grid, kThreadsWs, lstm_tc_smem(), st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_mlp_tc(const TcArgs &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + kBM - 1) / kBM;
    // setmaxnreg redistributes the registers the block was launched with: the
    // split only fits (and only ever completes) at exactly kLaunchRegs a thread
    static const int regs = [] {
        cudaFuncAttributes fa{}, fb{};
        if (cudaFuncGetAttributes(&fa, mlp_tc_kernel) != cudaSuccess ||
            cudaFuncGetAttributes(&fb, mlp_tc_dual_kernel) != cudaSuccess)
            return -1;
        return fa.numRegs == fb.numRegs ? fa.numRegs : -1;
    }();
    if (regs != kLaunchRegs) return cudaErrorInvalidConfiguration;
    if (a.dual) {  // two tiles per CTA at a time, one per column group
        const long long pairs = (tiles + 1) / 2;
        const int grid = (int)(pairs < num_sms ? pairs : num_sms);
        if (grid <= 0) return cudaSuccess;
        mlp_tc_dual_kernel<<<grid, kThreadsWs, mlp_tc_dual_smem(), st>>>(a);
        return cudaGetLastError();
    }
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    mlp_tc_kernel<<<grid, kThreadsWs, mlp_tc_smem_bytes(), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna

namespace rosenna {

bool tc_encode_f32_map(CUtensorMap *map, int rank, const void *base, const cuuint64_t *dims, const cuuint64_t *strides,
                       const cuuint32_t *box, const char **why, CUtensorMapSwizzle swizzle) {
    typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            *why = "cuTensorMapEncodeTiled is not available";
            return false;
        }
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void *>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *why = "cuTensorMapEncodeTiled rejected a tensor map";
        return false;
    }
    return true;
}

bool mlp_tc_encode_map(CUtensorMap *map, const float *block, int Kp, int Np, const char **why, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)(2 * Np)};
    const cuuint64_t strides[1] = {(cuuint64_t)Kp * sizeof(float)};
    const cuuint32_t box[2] = {32, (cuuint32_t)(box_rows > 0 ? box_rows : Np)};
    return tc_encode_f32_map(map, 2, block, dims, strides, box, why);
}

}  // namespace rosenna
