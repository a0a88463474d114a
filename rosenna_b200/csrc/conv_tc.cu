// conv_tc_kernel: a 3x3 stride-1 convolution as an implicit GEMM on tcgen05,
// with its ReLU and the following 2x2 pool (fLibrary/layers.f90 conv :183-233,
// relu4d activation_funcs.f90:43-52, max_pool/avgpool :236-310).
//
// Shapes: 3x3 kernel, stride 1, symmetric zero padding 0..2, 1 to 8 input and
// up to 16 output channels, a k=2 s=2 pool without padding over an even conv
// output.
//
// Samples are the GEMM's M dimension (128 per tile, TMEM lane = sample).  The
// batch is stored sample-fastest (element (c, y, x) of sample s at in[(c +
// C*(y + Hin*x))*ld + s]), so a tile's input patch is one 4-D TMA box {128
// samples, cb channels, ph rows, cw columns} per chunk: it lands in shared
// memory as rows of 128 samples, one row per K element (K = position x
// channel).  The split warps read it there (thread = sample, conflict-free),
// split each value into tf32 hi and lo parts and store both into TMEM, where
// the MMA reads its A operand: the shared-memory port then carries only the
// TMA writes, the split's reads and the weight operand.  The zero padding, and
// channels past C, come from the TMA's out-of-bounds fill.
//
// The N = 128 GEMM columns are a block of bh x 4 conv pixels x ocp output
// channels (bh*ocp = 32), ordered (column q from the right, row, channel):
// column 32q + ocp*i + oc is conv pixel (y0 + i, x0 + 3 - q).  With that order
// the weights for patch column pw are the 128-row window, starting at row
// 32*pw, of one 288-row matrix S whose row 32j + ocp*i + oc holds kernel
// column kw = j - 3 (zero outside 0..2) over the patch rows: K-slot c + cb*r
// holds W[oc][c][r - i][j - 3] (zero outside the kernel).  S (tf32 hi and lo
// parts, 72 KB, K-major) is the B operand, resident in shared memory for the
// whole kernel; each K-step of 8 K-slots is three MMAs, Al*Sh + Ah*Sl + Ah*Sh,
// of M = N = 128.  Columns of pixels outside the image or of padded channels
// are computed and not stored.
//
// Drain: a thread holds its sample's whole accumulator row, so bias, ReLU and
// the 2x2 pool are in-thread; the unit's pooled outputs (128 samples x OC
// channels x bh/2 pooled rows x 2 pooled columns) are staged in shared memory
// and written by one TMA tensor store (plain stores of 128 bytes per warp
// instruction left the drain waiting on the SM's outstanding writes).
//
// Roles (320 threads): warp 0 lane 0 loads chunks by TMA into a ring of
// shared-memory slots; warps 2-5 (thread = sample) split each chunk into a
// ring of four TMEM A slots; warp 1 lane 0 issues the MMAs; warps 6-9 (thread
// = sample) drain the double-buffered TMEM accumulator: bias, ReLU, pool,
// store.  Work is (128-sample tile, block) units, a contiguous range of them
// per CTA.  Every wait is bounded; a time-out records where in `err`, every
// role finishes, copies in flight are waited for, TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "conv_tc.cuh"
#include "mlp_tc.cuh"
#include "tc_common.cuh"

namespace rosenna {
namespace {

constexpr int kCtThreads = 320;
constexpr int kCtMaxSlots = 8;                      // shared-memory chunk slots
constexpr int kCtASlots = 4;                        // TMEM A slots (64 columns: hi at +0, lo at +32)
constexpr uint32_t kCtSBytes = kConvTcBFloats * 4;  // S hi then S lo
constexpr uint32_t kCtSLo = kCtSBytes / 2;
constexpr uint32_t kCtTmemCols = 512;               // A slots 0..255, accumulators 256..511
constexpr uint32_t kCtDCol = 256;
constexpr uint32_t kCtStage = 16384;                // one unit's pooled outputs: 32 x 128 samples x 4 B
constexpr size_t kCtSmemMax = 232448;

enum {
    kCtFull = 0,                          // [slot] chunk landed (TMA bytes)
    kCtFree = kCtFull + kCtMaxSlots,      // [slot] chunk read by the split (128 arrivals)
    kCtAFull = kCtFree + kCtMaxSlots,     // [A slot] written to TMEM (128 arrivals)
    kCtAEmpty = kCtAFull + kCtASlots,     // [A slot] MMAs done with it (commit)
    kCtDFull = kCtAEmpty + kCtASlots,     // [2] accumulator complete (commit)
    kCtDEmpty = kCtDFull + 2,             // [2] accumulator drained (128 arrivals)
    kCtDone = kCtDEmpty + 2,
    kCtNumBars = kCtDone + 1
};

// S, the chunk ring, two output staging buffers, bias, barriers
size_t conv_tc_smem(int rows, int slots) {
    return 1024 + kCtSBytes + (size_t)slots * rows * 512 + 2 * kCtStage + 64 + 8 * kCtNumBars + 16;
}

struct CtUnit {
    long long t;  // sample tile
    int y0, x0;   // the block's first conv row and column
};

// Unit u of ntiles x nblk: tiles in groups of p.group, and within a group
// the same block for consecutive tiles, so consecutive units read and write
// adjacent 512-byte runs of the same rows (the last group may be shorter).
__device__ __forceinline__ CtUnit ct_unit(const ConvTcArgs &p, long long u, int nbw, int nblk, long long ntiles) {
    CtUnit c;
    const int grp = p.group;
    const long long full = ntiles / grp * grp * nblk;  // units in full groups
    int blk;
    if (u < full) {
        const long long per = (long long)nblk * grp, tg = u / per;
        const int r = (int)(u - tg * per);
        blk = r / grp;
        c.t = tg * grp + (r - blk * grp);
    } else {
        const int gt = (int)(ntiles % grp), r = (int)(u - full);
        blk = r / gt;
        c.t = ntiles / grp * grp + (r - blk * gt);
    }
    const int bi = blk / nbw;
    c.y0 = bi * p.bh;
    c.x0 = (blk - bi * nbw) * 4;
    return c;
}

// Bias, ReLU and the 2x2 pool of one output channel from its four conv pixels
// (POOL 1: max, 2: mean); `floor` is 0 with a ReLU, -inf without.
template <int POOL>
__device__ __forceinline__ float ct_pool(float b, float floor, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
    const float v0 = __uint_as_float(a0), v1 = __uint_as_float(a1), v2 = __uint_as_float(a2), v3 = __uint_as_float(a3);
    if (POOL == 1)  // bias and ReLU are monotone: pool first (the same result, bit for bit)
        return fmaxf(fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)) + b, floor);
    const float r0 = fmaxf(v0 + b, floor), r1 = fmaxf(v1 + b, floor), r2 = fmaxf(v2 + b, floor),
                r3 = fmaxf(v3 + b, floor);
    return ((r0 + r1) + (r2 + r3)) * 0.25f;
}

// Writes the pooled outputs of one pair of pixel columns (q = 2h, 2h+1: pooled
// column x0/2 + 1 - h) from that pair's accumulator columns (va: q = 2h, vb:
// q = 2h + 1) into the staging tile [pooled column][pooled row][OCP channels]
// [128 samples] (the output box; channels past OC are not stored by it).
template <int OCP, int POOL>
__device__ __forceinline__ void ct_stage_half(const float (&bias)[OCP], float floor, const uint32_t (&va)[32],
                                              const uint32_t (&vb)[32], float *stage, int h) {
    constexpr int BH = 32 / OCP;
    const int qxl = 1 - h;
#pragma unroll
    for (int a = 0; a < BH / 2; a++)
#pragma unroll
        for (int oc = 0; oc < OCP; oc++) {
            const int r0 = OCP * 2 * a + oc, r1 = r0 + OCP;  // rows y0 + 2a, y0 + 2a + 1
            stage[((qxl * (BH / 2) + a) * OCP + oc) * 128] = ct_pool<POOL>(bias[oc], floor, va[r0], va[r1], vb[r0], vb[r1]);
        }
}

// OCP output channels per pixel column, CW patch columns per chunk, KCOL
// K-steps per patch column (conv_tc_geometry): compile-time, so the issue loop
// unrolls with immediate descriptor offsets (an issue loop that computes its
// descriptors at run time issues an M = N = 128 MMA about every 147 cycles
// instead of every 65).
template <int OCP, int CW, int KCOL, int POOL>
__global__ void __launch_bounds__(kCtThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs p) {
    constexpr int ROWS = CW * KCOL * 8;  // K-rows per chunk (p.rows)
    extern __shared__ uint8_t sm_raw[];
    uint8_t *const base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const ring = base + kCtSBytes;
    constexpr uint32_t slot_bytes = ROWS * 512u;  // ROWS rows of 128 samples x 4 B
    float *const stage0 = reinterpret_cast<float *>(ring + (size_t)p.slots * slot_bytes);
    float *const sbias = stage0 + 2 * kCtStage / 4;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(sbias + 16);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kCtNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nbw = (p.Wo + 3) / 4, nblk = ((p.Ho + p.bh - 1) / p.bh) * nbw;
    const long long ntiles = (p.n + 127) / 128, units = ntiles * nblk;
    const long long u0 = units * blockIdx.x / gridDim.x, u1 = units * (blockIdx.x + 1) / gridDim.x;
    constexpr int nck = 6 / CW;  // chunks per block
    const uint32_t ns = (uint32_t)p.slots;

    {  // the weight matrix S and the bias
        const float4 *src = reinterpret_cast<const float4 *>(p.arena + p.bt_off);
        float4 *dst = reinterpret_cast<float4 *>(base);
        for (int i = tid; i < kConvTcBFloats / 4; i += kCtThreads) dst[i] = __ldg(src + i);
        if (tid < 16) sbias[tid] = tid < p.OC ? p.arena[p.b_off + tid] : 0.f;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < kCtMaxSlots; i++) {
            mbar_init(bars + kCtFull + i, 1);
            mbar_init(bars + kCtFree + i, 128);
        }
        for (int i = 0; i < kCtASlots; i++) {
            mbar_init(bars + kCtAFull + i, 128);
            mbar_init(bars + kCtAEmpty + i, 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bars + kCtDFull + i, 1);
            mbar_init(bars + kCtDEmpty + i, 128);
        }
        mbar_init(bars + kCtDone, 1);
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

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA: each chunk as one box of 128 samples ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map) : "memory");
            uint32_t it = 0;
            bool ok = true;
            for (long long u = u0; u < u1 && ok; u++) {
                const CtUnit c = ct_unit(p, u, nbw, nblk, ntiles);
                for (int ck = 0; ck < nck; ck++, it++) {
                    const uint32_t s = it % ns, k = it / ns;
                    if (k > 0 && !(ok = mbar_wait(bars + kCtFree + s, (k - 1) & 1, p.err, 71, (int)u, ck))) break;
                    uint8_t *dst = ring + s * slot_bytes;
                    mbar_arrive_expect_tx(bars + kCtFull + s, slot_bytes);
                    tma_load_4d(dst, &p.map, bars + kCtFull + s, (int)(c.t * 128), 0, c.y0 - p.pad,
                                c.x0 - p.pad + ck * CW);
                }
            }
            // the last chunks' copies land before the CTA exits
            for (uint32_t i = it > ns ? it - ns : 0; i < it; i++) mbar_drain(bars + kCtFull + i % ns, (i / ns) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: D[sample][column] += A(TMEM) x S window ----
            const uint32_t bh0 = desc_lo(smem_u32(base)), bl0 = bh0 + (kCtSLo >> 4), idesc = idesc_tf32(128);
            uint32_t it = 0, uu = 0;
            bool ok = true;
            for (long long u = u0; u < u1 && ok; u++, uu++) {
                const uint32_t b = uu & 1, m = uu >> 1;
                if (m > 0 && !(ok = mbar_wait(bars + kCtDEmpty + b, (m - 1) & 1, p.err, 72, (int)u))) break;
                tc_fence_after();
                const uint32_t d = tmem + kCtDCol + 128u * b;
                for (int ck = 0; ck < nck && ok; ck++, it++) {
                    const uint32_t a = it % kCtASlots, ka = it / kCtASlots;
                    if (!(ok = mbar_wait(bars + kCtAFull + a, ka & 1, p.err, 73, (int)u, ck))) break;
                    tc_fence_after();
                    const uint32_t ah = tmem + 64u * a, al = ah + 32u;
                    const uint32_t step = (uint32_t)ck * (uint32_t)(CW * 4096 / 16);  // S windows of this chunk
                    const uint32_t bh = bh0 + step, bl = bl0 + step;
                    const uint32_t first = ck ? 1u : 0u;
#pragma unroll
                    for (int pwl = 0; pwl < CW; pwl++)
#pragma unroll
                        for (int g = 0; g < KCOL; g++) {
                            const int j = pwl * KCOL + g;                  // K-step within the chunk
                            const uint32_t off = (uint32_t)((pwl * 4096 + 32 * g) >> 4);  // S window pw, K-step g
                            umma_tf32_ts(d, al + 8u * j, bh + off, idesc, j ? 1u : first);
                            umma_tf32_ts(d, ah + 8u * j, bl + off, idesc, 1u);
                            umma_tf32_ts(d, ah + 8u * j, bh + off, idesc, 1u);
                        }
                    umma_commit(bars + kCtAEmpty + a);
                }
                if (ok) umma_commit(bars + kCtDFull + b);
            }
            umma_commit(bars + kCtDone);
            mbar_drain(bars + kCtDone, 0);
        }
    } else if (warp < 6) {
        // ---- split: thread = sample (lane quadrant warp % 4); K element k of
        // the chunk at row k; hi to A columns [0, rows), lo to [32, 32 + rows) ----
        const int q = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        uint32_t it = 0;
        bool ok = true;
        for (long long u = u0; u < u1 && ok; u++)
            for (int ck = 0; ck < nck; ck++, it++) {
                const uint32_t s = it % ns, k = it / ns, a = it % kCtASlots, ka = it / kCtASlots;
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtFull + s, k & 1, p.err, 74, (int)u, ck));
                if (ok && ka > 0)
                    ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtAEmpty + a, (ka - 1) & 1, p.err, 75, (int)u, ck));
                if (!ok) break;
                tc_fence_after();
                const float *src = reinterpret_cast<const float *>(ring + s * slot_bytes) + 32 * q + lane;
                const uint32_t acol = lane_base + 64u * a;
#pragma unroll
                for (int j = 0; j < ROWS; j += 8) {
                    uint32_t h[8], l[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const float x = src[(j + e) * 128];
                        h[e] = tf32_rna(x);
                        l[e] = tf32_lo(x, h[e]);
                    }
                    tmem_st8(acol + (uint32_t)j, h);
                    tmem_st8(acol + 32u + (uint32_t)j, l);
                }
                mbar_arrive(bars + kCtFree + s);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(bars + kCtAFull + a);
            }
    } else {
        // ---- drain: thread = sample; bias, ReLU, pool into the staging tile,
        // then thread 192 writes the tile with one TMA store ----
        const int q = warp & 3, s = 32 * q + lane;
        const bool leader = tid == 192;
        const float floor = p.relu ? 0.f : -__int_as_float(0x7f800000);
        float bias[OCP];
#pragma unroll
        for (int oc = 0; oc < OCP; oc++) bias[oc] = sbias[oc];
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        if (leader) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.omap) : "memory");
        uint32_t uu = 0;
        bool ok = true;
        for (long long u = u0; u < u1 && ok; u++, uu++) {
            const CtUnit c = ct_unit(p, u, nbw, nblk, ntiles);
            const uint32_t b = uu & 1;
            float *const stage = stage0 + (kCtStage / 4) * b;
            ok = mbar_wait(bars + kCtDFull + b, (uu >> 1) & 1, p.err, 76, (int)u);
            // all four warps agree on `ok`; the leader waited (after its last
            // store) until the store that read this buffer is done
            ok = bar_and(1, 128, ok);
            if (!ok) break;
            tc_fence_after();
            const uint32_t dcol = lane_base + kCtDCol + 128u * b;
            uint32_t va[32], vb[32];
            tmem_ld32_nw(dcol, va);
            tmem_ld32_nw(dcol + 32u, vb);
            tmem_wait_ld();
            ct_stage_half<OCP, POOL>(bias, floor, va, vb, stage + s, 0);
            tmem_ld32_nw(dcol + 64u, va);
            tmem_ld32_nw(dcol + 96u, vb);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(bars + kCtDEmpty + b);
            ct_stage_half<OCP, POOL>(bias, floor, va, vb, stage + s, 1);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (leader) {
                tma_store_4d(&p.omap, stage, (int)(c.t * 128), 0, c.y0 >> 1, c.x0 >> 1);
                bulk_commit();
                bulk_wait_read<1>();  // the other buffer is free for the next unit
            }
        }
        if (leader) bulk_wait<0>();  // every store complete before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCtTmemCols));
    }
}

// ---- two convs in one kernel ----------------------------------------------
//
// conv_pair_tc_kernel runs a conv(+ReLU)+pool step and the conv(+ReLU)+pool
// step that reads its output (fLibrary/layers.f90:183-233 twice, with the pool
// of :236-310 after each).  The first conv's pooled output does not go to a
// batch-sized array: each CTA owns two 128-sample columns of a small buffer
// (`mid`, local tiles alternate between them), which its TMA stores fill and
// its TMA loads read back a few row bands later, while the lines are still in
// L2.  Work is split over the CTAs by (sample tile, second-conv row band); a
// CTA computes the first-conv row bands its own second-conv bands read, so a
// band at each end of its range is computed by both neighbours.  The bands of
// the two convs are interleaved: a second-conv band is taken once the
// first-conv bands it reads were taken at least kPairLag bands earlier (fewer
// when a whole tile has fewer first-conv bands: a local tile's column of mid
// is rewritten two tiles later, after every band that reads it), and
// the loader checks a counter of first-conv bands whose stores have completed
// (published by the drain) before it loads one.  The first conv's weights are
// stored with the tf32 hi and lo parts side by side in each 128-byte row (its
// patch column has at most 16 K-slots), so both weight images fit beside a
// ring of chunk slots.

constexpr int kPairLag = 2;

// The band stream every role of a CTA walks in the same order.
struct PairStream {
    long long tA, tB;  // first and last sample tile of this CTA
    int kaA, kbB;      // first second-conv band of tile tA, end band of tile tB
    int nb2, hq1, bh2, ph2, pad2, hin2;
    int lag;  // kPairLag, or fewer when a whole tile has fewer first-conv bands
    long long t1, pos1;  // first-conv cursor: tile, bands taken so far
    int c1, c1hi;
    long long t2, base1;  // second-conv cursor: tile, position of its first first-conv band
    int k2, k2end, c2lo;

    __device__ __forceinline__ int ka(long long t) const { return t == tA ? kaA : 0; }
    __device__ __forceinline__ int kb(long long t) const { return t == tB ? kbB : nb2; }
    // rows of the first conv's pooled output that second-conv band k reads
    __device__ __forceinline__ int rmin(int k) const { return max(k * bh2 - pad2, 0); }
    __device__ __forceinline__ int rmax(int k) const { return min(k * bh2 - pad2 + ph2 - 1, hin2 - 1); }
    __device__ __forceinline__ int clo(long long t) const { return rmin(ka(t)) / hq1; }
    __device__ __forceinline__ int chi(long long t) const { return rmax(kb(t) - 1) / hq1; }

    __device__ __forceinline__ void init(const ConvPairArgs &p, long long w0, long long w1) {
        nb2 = p.nb2;
        hq1 = p.bh1 / 2;
        bh2 = p.bh2;
        ph2 = p.ph2;
        pad2 = p.pad2;
        hin2 = p.Hin2;
        lag = min(kPairLag, rmax(nb2 - 1) / hq1 + 1);
        if (w1 <= w0) {
            tA = 0;
            tB = -1;
            t1 = t2 = 0;
            return;
        }
        tA = w0 / nb2;
        tB = (w1 - 1) / nb2;
        kaA = (int)(w0 - tA * nb2);
        kbB = (int)(w1 - tB * nb2);
        t1 = t2 = tA;
        c1 = c2lo = clo(tA);
        c1hi = chi(tA);
        pos1 = base1 = 0;
        k2 = ka(tA);
        k2end = kb(tA);
    }
    // The next band: layer (1 or 2), sample tile, band, local-tile parity.  A
    // second-conv band gets `need`, the count of first-conv bands (in this
    // order) that must be stored before it is loaded; a first-conv band its
    // position `pos` and `last`, whether no first-conv band follows.
    __device__ __forceinline__ bool next(int &layer, long long &t, int &band, int &par, long long &need,
                                         long long &pos, bool &last) {
        const bool have1 = t1 <= tB;
        if (t2 <= tB) {
            const long long dep = base1 + (rmax(k2) / hq1 - c2lo);
            if (!have1 || dep + lag < pos1) {
                layer = 2;
                t = t2;
                band = k2;
                par = (int)((t2 - tA) & 1);
                need = dep + 1;
                if (++k2 == k2end) {
                    base1 += chi(t2) - c2lo + 1;
                    if (++t2 <= tB) {
                        k2 = ka(t2);
                        k2end = kb(t2);
                        c2lo = clo(t2);
                    }
                }
                return true;
            }
        }
        if (!have1) return false;
        layer = 1;
        t = t1;
        band = c1;
        par = (int)((t1 - tA) & 1);
        pos = pos1++;
        if (++c1 > c1hi && ++t1 <= tB) {
            c1 = clo(t1);
            c1hi = chi(t1);
        }
        last = t1 > tB;
        return true;
    }
};

// Bounded wait until the shared counter reaches `need`.
__device__ __forceinline__ bool pair_wait_count(const volatile uint32_t *cnt, long long need, int *err, int code,
                                                int where) {
    if ((long long)*cnt >= need) return true;
    const uint64_t t0 = globaltimer();
    bool other = false;
    for (uint32_t i = 0; i < kWaitIters; i++) {
        if ((long long)*cnt >= need) {
            __threadfence_block();
            return true;
        }
        if (*(volatile int *)err) {
            other = true;
            break;
        }
        if ((i & 255) == 255 && globaltimer() - t0 > kWaitNs) break;
        __nanosleep(32);
    }
    if (!other && atomicCAS(err, 0, code) == 0) {
        err[1] = blockIdx.x;
        err[2] = threadIdx.x;
        err[3] = where;
        err[4] = 0;
        err[5] = (int)need;
        err[6] = (int)*cnt;
    }
    __threadfence();
    return false;
}

// Waits until every committed bulk store group but the `newer` most recent
// ones is complete (the group count is an immediate operand).
__device__ __forceinline__ void pair_wait_older(int newer) {
    switch (newer < 7 ? newer : 7) {
        case 0: bulk_wait<0>(); break;
        case 1: bulk_wait<1>(); break;
        case 2: bulk_wait<2>(); break;
        case 3: bulk_wait<3>(); break;
        case 4: bulk_wait<4>(); break;
        case 5: bulk_wait<5>(); break;
        case 6: bulk_wait<6>(); break;
        default: bulk_wait<7>(); break;
    }
}

// The MMAs of one unit: NCK chunks of A slots against the weight windows
// (PACKED: the lo part KCOL K-steps after the hi part in the same rows).
template <int CW, int KCOL, bool PACKED>
__device__ __forceinline__ bool pair_issue_unit(uint64_t *bars, uint32_t tmem, uint32_t d, uint32_t bh0, uint32_t bl0,
                                                uint32_t idesc, uint32_t &it, int *err, int where) {
    constexpr int NCK = 6 / CW;
    for (int ck = 0; ck < NCK; ck++, it++) {
        const uint32_t a = it % kCtASlots, ka = it / kCtASlots;
        if (!mbar_wait(bars + kCtAFull + a, ka & 1, err, 73, where, ck)) return false;
        tc_fence_after();
        const uint32_t ah = tmem + 64u * a, al = ah + 32u;
        const uint32_t step = (uint32_t)ck * (uint32_t)(CW * 4096 / 16);
        const uint32_t bh = bh0 + step;
        const uint32_t bl = PACKED ? bh + (uint32_t)(KCOL * 32 / 16) : bl0 + step;
        const uint32_t first = ck ? 1u : 0u;
#pragma unroll
        for (int pwl = 0; pwl < CW; pwl++)
#pragma unroll
            for (int g = 0; g < KCOL; g++) {
                const int j = pwl * KCOL + g;
                const uint32_t off = (uint32_t)((pwl * 4096 + 32 * g) >> 4);
                umma_tf32_ts(d, al + 8u * j, bh + off, idesc, j ? 1u : first);
                umma_tf32_ts(d, ah + 8u * j, bl + off, idesc, 1u);
                umma_tf32_ts(d, ah + 8u * j, bh + off, idesc, 1u);
            }
        umma_commit(bars + kCtAEmpty + a);
    }
    return true;
}

// The split of one unit's NCK chunks (ROWS K-rows each) into TMEM A slots.
template <int ROWS, int NCK>
__device__ __forceinline__ bool pair_split_unit(uint64_t *bars, const uint8_t *ring, uint32_t slot_bytes, uint32_t ns,
                                                uint32_t lane_base, int q, int lane, uint32_t &it, int *err,
                                                int where) {
    for (int ck = 0; ck < NCK; ck++, it++) {
        const uint32_t s = it % ns, k = it / ns, a = it % kCtASlots, ka = it / kCtASlots;
        bool ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtFull + s, k & 1, err, 74, where, ck));
        if (ok && ka > 0)
            ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtAEmpty + a, (ka - 1) & 1, err, 75, where, ck));
        if (!ok) return false;
        tc_fence_after();
        const float *src = reinterpret_cast<const float *>(ring + s * slot_bytes) + 32 * q + lane;
        const uint32_t acol = lane_base + 64u * a;
#pragma unroll
        for (int j = 0; j < ROWS; j += 8) {
            uint32_t h[8], l[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float x = src[(j + e) * 128];
                h[e] = tf32_rna(x);
                l[e] = tf32_lo(x, h[e]);
            }
            tmem_st8(acol + (uint32_t)j, h);
            tmem_st8(acol + 32u + (uint32_t)j, l);
        }
        mbar_arrive(bars + kCtFree + s);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(bars + kCtAFull + a);
    }
    return true;
}

// S2 (full image), S1 (packed image), the chunk ring, two output staging
// buffers, both biases, barriers, the TMEM address and the band counter
size_t conv_pair_smem(int rows_max, int slots) {
    return 1024 + kCtSBytes + kCtSLo + (size_t)slots * rows_max * 512 + 2 * kCtStage + 128 + 8 * kCtNumBars + 16;
}

template <int OCP1, int CW1, int KCOL1, int POOL1, int OCP2, int CW2, int KCOL2, int POOL2>
__global__ void __launch_bounds__(kCtThreads, 1) conv_pair_tc_kernel(const __grid_constant__ ConvPairArgs p) {
    constexpr int ROWS1 = CW1 * KCOL1 * 8, ROWS2 = CW2 * KCOL2 * 8;
    constexpr uint32_t slot_bytes = (ROWS1 > ROWS2 ? ROWS1 : ROWS2) * 512u;
    constexpr int NCK1 = 6 / CW1, NCK2 = 6 / CW2;
    static_assert(KCOL1 <= 2, "the packed first-conv image holds at most 16 K-slots per row");
    extern __shared__ uint8_t sm_raw[];
    uint8_t *const base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const s1 = base + kCtSBytes;
    uint8_t *const ring = s1 + kCtSLo;
    float *const stage0 = reinterpret_cast<float *>(ring + (size_t)p.slots * slot_bytes);
    float *const sbias = stage0 + 2 * kCtStage / 4;  // [0, 16) first conv, [16, 32) second
    uint64_t *const bars = reinterpret_cast<uint64_t *>(sbias + 32);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kCtNumBars);
    volatile uint32_t *const mid_done = tmem_slot + 1;  // first-conv bands stored and complete

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nbw1 = (p.Wo1 + 3) / 4, nbw2 = (p.Wo2 + 3) / 4;
    const long long ntiles = (p.n + 127) / 128, items = ntiles * p.nb2;
    const long long w0 = items * blockIdx.x / gridDim.x, w1 = items * (blockIdx.x + 1) / gridDim.x;
    const int midc = (int)blockIdx.x * 256;  // this CTA's two 128-sample columns of mid
    const uint32_t ns = (uint32_t)p.slots;

    {  // both weight images and biases
        const float4 *src2 = reinterpret_cast<const float4 *>(p.arena + p.s2_off);
        float4 *dst2 = reinterpret_cast<float4 *>(base);
        for (int i = tid; i < kConvTcBFloats / 4; i += kCtThreads) dst2[i] = __ldg(src2 + i);
        const float4 *src1 = reinterpret_cast<const float4 *>(p.arena + p.s1_off);
        float4 *dst1 = reinterpret_cast<float4 *>(s1);
        for (int i = tid; i < kConvTcBFloats / 8; i += kCtThreads) dst1[i] = __ldg(src1 + i);
        if (tid < 16) sbias[tid] = tid < p.OC1 ? p.arena[p.b1_off + tid] : 0.f;
        else if (tid < 32) sbias[tid] = tid - 16 < p.OC2 ? p.arena[p.b2_off + tid - 16] : 0.f;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < kCtMaxSlots; i++) {
            mbar_init(bars + kCtFull + i, 1);
            mbar_init(bars + kCtFree + i, 128);
        }
        for (int i = 0; i < kCtASlots; i++) {
            mbar_init(bars + kCtAFull + i, 128);
            mbar_init(bars + kCtAEmpty + i, 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bars + kCtDFull + i, 1);
            mbar_init(bars + kCtDEmpty + i, 128);
        }
        mbar_init(bars + kCtDone, 1);
        *mid_done = 0;
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

    PairStream st;
    st.init(p, w0, w1);
    int layer = 0, band = 0, par = 0;
    long long t = 0, need = 0, pos = 0;
    bool last = false;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA: chunks of the first conv's input, or of mid ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map1) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map2) : "memory");
            uint32_t it = 0;
            bool ok = true;
            while (ok && st.next(layer, t, band, par, need, pos, last)) {
                if (layer == 2) {  // the first-conv bands this band reads are in memory
                    if (!(ok = pair_wait_count(mid_done, need, p.err, 77, band))) break;
                    asm volatile("fence.proxy.async;" ::: "memory");
                }
                const int nbw = layer == 1 ? nbw1 : nbw2, nck = layer == 1 ? NCK1 : NCK2;
                const uint32_t bytes = (layer == 1 ? ROWS1 : ROWS2) * 512u;
                const int y0 = band * (layer == 1 ? p.bh1 : p.bh2);
                for (int ub = 0; ub < nbw && ok; ub++)
                    for (int ck = 0; ck < nck; ck++, it++) {
                        const uint32_t s = it % ns, k = it / ns;
                        if (k > 0 && !(ok = mbar_wait(bars + kCtFree + s, (k - 1) & 1, p.err, 71, band, ck))) break;
                        uint8_t *dst = ring + s * slot_bytes;
                        mbar_arrive_expect_tx(bars + kCtFull + s, bytes);
                        if (layer == 1)
                            tma_load_4d(dst, &p.map1, bars + kCtFull + s, (int)(t * 128), 0, y0 - p.pad1,
                                        4 * ub - p.pad1 + ck * CW1);
                        else
                            tma_load_4d(dst, &p.map2, bars + kCtFull + s, midc + 128 * par, 0, y0 - p.pad2,
                                        4 * ub - p.pad2 + ck * CW2);
                    }
            }
            // the last chunks' copies land before the CTA exits
            for (uint32_t i = it > ns ? it - ns : 0; i < it; i++) mbar_drain(bars + kCtFull + i % ns, (i / ns) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            const uint32_t b2h = desc_lo(smem_u32(base)), b2l = b2h + (kCtSLo >> 4), b1h = desc_lo(smem_u32(s1));
            const uint32_t idesc = idesc_tf32(128);
            uint32_t it = 0, uu = 0;
            bool ok = true;
            while (ok && st.next(layer, t, band, par, need, pos, last)) {
                const int nbw = layer == 1 ? nbw1 : nbw2;
                for (int ub = 0; ub < nbw && ok; ub++, uu++) {
                    const uint32_t b = uu & 1, m = uu >> 1;
                    if (m > 0 && !(ok = mbar_wait(bars + kCtDEmpty + b, (m - 1) & 1, p.err, 72, band))) break;
                    tc_fence_after();
                    const uint32_t d = tmem + kCtDCol + 128u * b;
                    if (layer == 1)
                        ok = pair_issue_unit<CW1, KCOL1, true>(bars, tmem, d, b1h, 0u, idesc, it, p.err, band);
                    else
                        ok = pair_issue_unit<CW2, KCOL2, false>(bars, tmem, d, b2h, b2l, idesc, it, p.err, band);
                    if (ok) umma_commit(bars + kCtDFull + b);
                }
            }
            umma_commit(bars + kCtDone);
            mbar_drain(bars + kCtDone, 0);
        }
    } else if (warp < 6) {
        // ---- split: thread = sample ----
        const int q = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        uint32_t it = 0;
        bool ok = true;
        while (ok && st.next(layer, t, band, par, need, pos, last)) {
            const int nbw = layer == 1 ? nbw1 : nbw2;
            for (int ub = 0; ub < nbw && ok; ub++)
                ok = layer == 1 ? pair_split_unit<ROWS1, NCK1>(bars, ring, slot_bytes, ns, lane_base, q, lane, it,
                                                                p.err, band)
                                : pair_split_unit<ROWS2, NCK2>(bars, ring, slot_bytes, ns, lane_base, q, lane, it,
                                                                p.err, band);
        }
    } else {
        // ---- drain: bias, ReLU, pool, staged, one TMA store per unit (to mid
        // for the first conv); thread 192 publishes completed first-conv bands ----
        const int q = warp & 3, s = 32 * q + lane;
        const bool leader = tid == 192;
        const float floor1 = p.relu1 ? 0.f : -__int_as_float(0x7f800000);
        const float floor2 = p.relu2 ? 0.f : -__int_as_float(0x7f800000);
        float bias1[OCP1], bias2[OCP2];
#pragma unroll
        for (int oc = 0; oc < OCP1; oc++) bias1[oc] = sbias[oc];
#pragma unroll
        for (int oc = 0; oc < OCP2; oc++) bias2[oc] = sbias[16 + oc];
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        if (leader) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.omap1) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.omap2) : "memory");
        }
        uint32_t uu = 0;
        // the last first-conv band not yet published, and the stores committed
        // after its last one (it is published at the end of the next
        // first-conv band, when its stores are long complete)
        long long pending = -1;
        int since = 0;
        bool ok = true;
        while (ok && st.next(layer, t, band, par, need, pos, last)) {
            const int nbw = layer == 1 ? nbw1 : nbw2;
            const int y0 = band * (layer == 1 ? p.bh1 : p.bh2);
            for (int ub = 0; ub < nbw && ok; ub++, uu++) {
                const uint32_t b = uu & 1;
                float *const stage = stage0 + (kCtStage / 4) * b;
                ok = mbar_wait(bars + kCtDFull + b, (uu >> 1) & 1, p.err, 76, band);
                ok = bar_and(1, 128, ok);
                if (!ok) break;
                tc_fence_after();
                const uint32_t dcol = lane_base + kCtDCol + 128u * b;
                uint32_t va[32], vb[32];
                tmem_ld32_nw(dcol, va);
                tmem_ld32_nw(dcol + 32u, vb);
                tmem_wait_ld();
                if (layer == 1)
                    ct_stage_half<OCP1, POOL1>(bias1, floor1, va, vb, stage + s, 0);
                else
                    ct_stage_half<OCP2, POOL2>(bias2, floor2, va, vb, stage + s, 0);
                tmem_ld32_nw(dcol + 64u, va);
                tmem_ld32_nw(dcol + 96u, vb);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(bars + kCtDEmpty + b);
                if (layer == 1)
                    ct_stage_half<OCP1, POOL1>(bias1, floor1, va, vb, stage + s, 1);
                else
                    ct_stage_half<OCP2, POOL2>(bias2, floor2, va, vb, stage + s, 1);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (leader) {
                    if (layer == 1)
                        tma_store_4d(&p.omap1, stage, midc + 128 * par, 0, y0 >> 1, 2 * ub);
                    else
                        tma_store_4d(&p.omap2, stage, (int)(t * 128), 0, y0 >> 1, 2 * ub);
                    bulk_commit();
                    if (pending >= 0) since++;
                    const bool band_end = layer == 1 && ub == nbw - 1;
                    long long publish = -1;
                    if (band_end && last) {  // nothing follows that would complete it later
                        bulk_wait<0>();
                        publish = pos + 1;
                        pending = -1;
                    } else {
                        bulk_wait_read<1>();  // the other staging buffer is free for the next unit
                        if (band_end) {
                            if (pending >= 0) {  // its stores are the ones before the last `since`
                                pair_wait_older(since);
                                publish = pending + 1;
                            }
                            pending = pos;
                            since = 0;
                        }
                    }
                    if (publish >= 0) {
                        asm volatile("fence.proxy.async;" ::: "memory");
                        __threadfence_block();
                        *mid_done = (uint32_t)publish;
                    }
                }
            }
        }
        if (leader) bulk_wait<0>();  // every store complete before the CTA exits
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

ConvTcGeom conv_tc_geometry(int C, int OC) {
    ConvTcGeom g{};
    if (C < 1 || C > 8 || OC < 1 || OC > 16) return g;
    g.cb = C == 1 ? 1 : C == 2 ? 2 : C <= 4 ? 4 : 8;
    for (int ocp = OC <= 8 ? 8 : 16; ocp <= 16; ocp *= 2) {
        const int bh = 32 / ocp;
        int ph = bh + 2;
        while ((g.cb * ph) % 8) ph++;
        if (g.cb * ph > 32) continue;  // one patch column's K-slots fit one 128-byte row of S
        g.ocp = ocp;
        g.bh = bh;
        g.ph = ph;
        const int per_col = g.cb * ph;
        g.cw = 6;
        while (g.cw > 1 && (per_col * g.cw > 32 || 6 % g.cw)) g.cw--;  // a chunk fits one 32-column A slot
        g.rows = per_col * g.cw;
        const size_t fixed = conv_tc_smem(g.rows, 0);
        g.slots = (int)((kCtSmemMax - fixed) / ((size_t)g.rows * 512));
        if (g.slots > kCtMaxSlots) g.slots = kCtMaxSlots;
        g.ok = g.slots >= 2;
        return g;
    }
    return g;
}

bool conv_tc_shape_ok(int KS, int str_h, int str_w, int pad_h, int pad_w, int C, int OC, int pool, int pk, int pstr_h,
                      int pstr_w, int ppad_h, int ppad_w, int Ho, int Wo) {
    if (!(KS == 3 && str_h == 1 && str_w == 1 && pad_h == pad_w && pad_h >= 0 && pad_h <= 2 && C >= 1 && C <= 8 &&
          OC >= 1 && OC <= 16 && pool != 0 && pk == 2 && pstr_h == 2 && pstr_w == 2 && ppad_h == 0 && ppad_w == 0 &&
          Ho % 2 == 0 && Wo % 2 == 0 && Ho >= 2 && Wo >= 2))
        return false;
    return conv_tc_geometry(C, OC).ok;
}

// The weight image: S hi then S lo, each 288 rows x 32 K-slots in the
// 128-byte-swizzled K-major layout (row r of an 8-row atom holds 16-byte chunk
// k at position k ^ (r & 7)), so the kernel copies it linearly.
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
    for (int i = 0; i < kConvTcBFloats; i++) img[i] = 0.f;
    const ConvTcGeom g = conv_tc_geometry(C, OC);
    if (!g.ok) return;
    float *lo = img + kConvTcBFloats / 2;
    for (int j = 0; j < kConvTcRows / 32; j++)
        for (int ri = 0; ri < 32; ri++) {
            const int i = ri / g.ocp, oc = ri - i * g.ocp, kw = j - 3;
            for (int r = 0; r < g.ph; r++)
                for (int c = 0; c < g.cb; c++) {
                    const int kh = r - i;
                    float x = 0.f;
                    if (oc < OC && c < C && kw >= 0 && kw < 3 && kh >= 0 && kh < 3)
                        x = w[(((size_t)oc * C + c) * 3 + kh) * 3 + kw];
                    const float h = tf32_hi(x);
                    put_swizzled(img, 32 * j + ri, c + g.cb * r, h);
                    put_swizzled(lo, 32 * j + ri, c + g.cb * r, tf32_hi(x - h));
                }
        }
}

bool conv_tc_input_ok(const float *in, long long ld_in) {
    return (reinterpret_cast<uintptr_t>(in) & 15) == 0 && (ld_in & 3) == 0 && ld_in > 0;
}

bool conv_tc_encode_input(ConvTcArgs &a, const float *in, long long ld_in, const char **why) {
    const cuuint64_t row = (cuuint64_t)ld_in * sizeof(float);
    const cuuint64_t dims[4] = {(cuuint64_t)a.n, (cuuint64_t)a.C, (cuuint64_t)a.Hin, (cuuint64_t)a.Win};
    const cuuint64_t strides[3] = {row, row * (cuuint64_t)a.C, row * (cuuint64_t)a.C * (cuuint64_t)a.Hin};
    const cuuint32_t box[4] = {128, (cuuint32_t)a.cb, (cuuint32_t)a.ph, (cuuint32_t)a.cw};
    return tc_encode_f32_map(&a.map, 4, in, dims, strides, box, why, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool conv_tc_encode_output(ConvTcArgs &a, const char **why) {
    const cuuint64_t row = (cuuint64_t)a.ld_out * sizeof(float);
    const cuuint64_t dims[4] = {(cuuint64_t)a.n, (cuuint64_t)a.OC, (cuuint64_t)a.Hq, (cuuint64_t)a.Wq};
    const cuuint64_t strides[3] = {row * (cuuint64_t)a.so_c, row * (cuuint64_t)a.so_h, row * (cuuint64_t)a.so_w};
    const cuuint32_t box[4] = {128, (cuuint32_t)a.ocp, (cuuint32_t)(a.bh / 2), 2};
    return tc_encode_f32_map(&a.omap, 4, a.out, dims, strides, box, why, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// The (OCP, CW, KCOL) instantiations conv_tc_geometry produces for C = 1..8,
// OC = 1..16, each with max (1) and mean (2) pooling.
#define ROSENNA_CONV_TC_SHAPES(X)                                                                          \
    X(16, 1, 4, 1) X(16, 2, 2, 1) X(16, 3, 1, 1) X(8, 1, 3, 1) X(8, 2, 2, 1) X(8, 3, 1, 1) X(16, 1, 4, 2) \
        X(16, 2, 2, 2) X(16, 3, 1, 2) X(8, 1, 3, 2) X(8, 2, 2, 2) X(8, 3, 1, 2)

cudaError_t conv_tc_configure() {
    cudaError_t e = cudaSuccess;
#define ROSENNA_CONV_TC_CFG(O, W, K, P)                                                                     \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(conv_tc_kernel<O, W, K, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)kCtSmemMax);
    ROSENNA_CONV_TC_SHAPES(ROSENNA_CONV_TC_CFG)
#undef ROSENNA_CONV_TC_CFG
    return e;
}

// ---- conv_pair_tc_kernel host side ----

#define ROSENNA_CONV_PAIR_SHAPES(X) X(1, 1) X(1, 2) X(2, 1) X(2, 2)

bool conv_pair_shape_ok(int C1, int OC1, int pool1, int C2, int OC2, int pool2) {
    const ConvTcGeom g1 = conv_tc_geometry(C1, OC1), g2 = conv_tc_geometry(C2, OC2);
    return g1.ok && g2.ok && C1 == 1 && OC1 <= 8 && OC1 == C2 && C2 >= 5 && OC2 > 8 && g1.ocp == 8 && g1.cw == 3 &&
           g1.cb * g1.ph == 8 && g2.ocp == 16 && g2.cw == 1 && g2.cb * g2.ph == 32 && (pool1 == 1 || pool1 == 2) &&
           (pool2 == 1 || pool2 == 2) && conv_pair_smem(32, 2) <= kCtSmemMax;
}

void conv_pair_pack1(const float *w, int OC, int C, float *img) {
    for (int i = 0; i < kConvTcBFloats / 2; i++) img[i] = 0.f;
    const ConvTcGeom g = conv_tc_geometry(C, OC);
    if (!g.ok || g.cb * g.ph > 16) return;
    const int lo = g.cb * g.ph;  // the lo part's first K-slot
    for (int j = 0; j < kConvTcRows / 32; j++)
        for (int ri = 0; ri < 32; ri++) {
            const int i = ri / g.ocp, oc = ri - i * g.ocp, kw = j - 3;
            for (int r = 0; r < g.ph; r++)
                for (int c = 0; c < g.cb; c++) {
                    const int kh = r - i;
                    float x = 0.f;
                    if (oc < OC && c < C && kw >= 0 && kw < 3 && kh >= 0 && kh < 3)
                        x = w[(((size_t)oc * C + c) * 3 + kh) * 3 + kw];
                    const float h = tf32_hi(x);
                    put_swizzled(img, 32 * j + ri, c + g.cb * r, h);
                    put_swizzled(img, 32 * j + ri, lo + c + g.cb * r, tf32_hi(x - h));
                }
        }
}

cudaError_t conv_pair_configure() {
    cudaError_t e = cudaSuccess;
#define ROSENNA_CONV_PAIR_CFG(P1, P2)                                                                            \
    if (e == cudaSuccess)                                                                                        \
        e = cudaFuncSetAttribute(conv_pair_tc_kernel<8, 3, 1, P1, 16, 1, 4, P2>,                                \
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCtSmemMax);
    ROSENNA_CONV_PAIR_SHAPES(ROSENNA_CONV_PAIR_CFG)
#undef ROSENNA_CONV_PAIR_CFG
    return e;
}

cudaError_t launch_conv_pair(const ConvTcArgs &a1, long long s1_off, const ConvTcArgs &a2, float *mid,
                             long long mid_cols, int num_sms, cudaStream_t st, const char **why) {
    if (!conv_pair_shape_ok(a1.C, a1.OC, a1.pool, a2.C, a2.OC, a2.pool) || a1.Hq != a2.Hin || a1.Wq != a2.Win ||
        a1.n != a2.n || !mid || mid_cols < kConvPairMidPerCta || mid_cols % kConvPairMidPerCta ||
        a1.ocp != 8 || a1.cw != 3 || a2.ocp != 16 || a2.cw != 1) {
        *why = "conv pair: shapes";
        return cudaErrorInvalidConfiguration;
    }
    const long long ntiles = (a1.n + 127) / 128, nb2 = (a2.Ho + a2.bh - 1) / a2.bh, items = ntiles * nb2;
    long long grid = std::min<long long>(num_sms, mid_cols / kConvPairMidPerCta);
    grid = std::min(grid, items);
    if (grid <= 0) return cudaSuccess;
    ConvPairArgs p{};
    p.map1 = a1.map;
    p.omap2 = a2.omap;
    {  // mid, as the first conv's output and as the second conv's input
        const cuuint64_t row = (cuuint64_t)mid_cols * sizeof(float);
        const cuuint64_t C2 = (cuuint64_t)a2.C, H2 = (cuuint64_t)a2.Hin;
        const cuuint64_t dims[4] = {(cuuint64_t)mid_cols, C2, H2, (cuuint64_t)a2.Win};
        const cuuint64_t strides[3] = {row, row * C2, row * C2 * H2};
        const cuuint32_t obox[4] = {128, (cuuint32_t)a1.ocp, (cuuint32_t)(a1.bh / 2), 2};
        if (!tc_encode_f32_map(&p.omap1, 4, mid, dims, strides, obox, why, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
        const cuuint32_t ibox[4] = {128, (cuuint32_t)a2.cb, (cuuint32_t)a2.ph, (cuuint32_t)a2.cw};
        if (!tc_encode_f32_map(&p.map2, 4, mid, dims, strides, ibox, why, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    }
    p.arena = a1.arena;
    p.s1_off = s1_off;
    p.b1_off = a1.b_off;
    p.s2_off = a2.bt_off;
    p.b2_off = a2.b_off;
    p.n = a1.n;
    p.err = a1.err;
    p.OC1 = a1.OC;
    p.Wo1 = a1.Wo;
    p.pad1 = a1.pad;
    p.relu1 = a1.relu;
    p.bh1 = a1.bh;
    p.OC2 = a2.OC;
    p.Hin2 = a2.Hin;
    p.Wo2 = a2.Wo;
    p.pad2 = a2.pad;
    p.relu2 = a2.relu;
    p.bh2 = a2.bh;
    p.ph2 = a2.ph;
    p.nb2 = (int)nb2;
    const int rows_max = std::max(a1.rows, a2.rows);
    const size_t fixed = conv_pair_smem(rows_max, 0);
    p.slots = (int)std::min<size_t>(kCtMaxSlots, (kCtSmemMax - fixed) / ((size_t)rows_max * 512));
    if (p.slots < 2) {
        *why = "conv pair: shared memory";
        return cudaErrorInvalidConfiguration;
    }
    const size_t smem = conv_pair_smem(rows_max, p.slots);
    bool launched = false;
#define ROSENNA_CONV_PAIR_LAUNCH(P1, P2)                                                                 \
    if (!launched && a1.pool == P1 && a2.pool == P2) {                                                   \
        conv_pair_tc_kernel<8, 3, 1, P1, 16, 1, 4, P2><<<(int)grid, kCtThreads, smem, st>>>(p);          \
        launched = true;                                                                                 \
    }
    ROSENNA_CONV_PAIR_SHAPES(ROSENNA_CONV_PAIR_LAUNCH)
#undef ROSENNA_CONV_PAIR_LAUNCH
    if (!launched) return cudaErrorInvalidConfiguration;
    return cudaGetLastError();
}

cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st) {
    const bool geom = (a.ocp == 8 || a.ocp == 16) && a.bh * a.ocp == 32 && a.cw >= 1 && 6 % a.cw == 0 &&
                      (a.cb * a.ph) % 8 == 0 && a.cb * a.ph <= 32 && a.ph >= a.bh + 2 &&
                      a.rows == a.cb * a.ph * a.cw && a.rows <= 32 && a.slots >= 2 && a.slots <= kCtMaxSlots &&
                      a.OC >= 1 && a.OC <= a.ocp && a.C >= 1 && a.C <= a.cb && (a.pool == 1 || a.pool == 2) &&
                      a.group >= 1 && a.group <= 64 &&
                      conv_tc_smem(a.rows, a.slots) <= kCtSmemMax;
    if (!geom) return cudaErrorInvalidConfiguration;
    const long long units = ((a.n + 127) / 128) * (long long)(((a.Ho + a.bh - 1) / a.bh) * ((a.Wo + 3) / 4));
    const int grid = (int)(units < num_sms ? units : num_sms);
    if (grid <= 0) return cudaSuccess;
    const int kc = a.cb * a.ph / 8;
    const size_t smem = conv_tc_smem(a.rows, a.slots);
    bool launched = false;
#define ROSENNA_CONV_TC_LAUNCH(O, W, K, P)                                      \
    if (!launched && a.ocp == O && a.cw == W && kc == K && a.pool == P) {     \
        conv_tc_kernel<O, W, K, P><<<grid, kCtThreads, smem, st>>>(a);        \
        launched = true;                                                      \
    }
    ROSENNA_CONV_TC_SHAPES(ROSENNA_CONV_TC_LAUNCH)
#undef ROSENNA_CONV_TC_LAUNCH
    if (!launched) return cudaErrorInvalidConfiguration;
    return cudaGetLastError();
}

}  // namespace rosenna
