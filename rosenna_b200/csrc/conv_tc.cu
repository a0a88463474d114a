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

// Unit u of ntiles x nblk: tiles in groups of kCtGroup, and within a group
// the same block for consecutive tiles, so consecutive units read and write
// adjacent 512-byte runs of the same rows (the last group may be shorter).
constexpr int kCtGroup = 4;
__device__ __forceinline__ CtUnit ct_unit(const ConvTcArgs &p, long long u, int nbw, int nblk, long long ntiles) {
    CtUnit c;
    const long long full = ntiles / kCtGroup * kCtGroup * nblk;  // units in full groups
    int blk;
    if (u < full) {
        const long long per = (long long)nblk * kCtGroup, tg = u / per;
        const int r = (int)(u - tg * per);
        blk = r / kCtGroup;
        c.t = tg * kCtGroup + (r - blk * kCtGroup);
    } else {
        const int gt = (int)(ntiles % kCtGroup), r = (int)(u - full);
        blk = r / gt;
        c.t = ntiles / kCtGroup * kCtGroup + (r - blk * gt);
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
                        l[e] = tf32_rna(x - __uint_as_float(h[e]));
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

cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st) {
    const bool geom = (a.ocp == 8 || a.ocp == 16) && a.bh * a.ocp == 32 && a.cw >= 1 && 6 % a.cw == 0 &&
                      (a.cb * a.ph) % 8 == 0 && a.cb * a.ph <= 32 && a.ph >= a.bh + 2 &&
                      a.rows == a.cb * a.ph * a.cw && a.rows <= 32 && a.slots >= 2 && a.slots <= kCtMaxSlots &&
                      a.OC >= 1 && a.OC <= a.ocp && a.C >= 1 && a.C <= a.cb && (a.pool == 1 || a.pool == 2) &&
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
