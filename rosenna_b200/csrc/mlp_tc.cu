// Tensor-core fused MLP for layers up to 256 wide: tcgen05 (TMEM accumulators)
// with a 3xTF32 split, weights fed by TMA.
//
// Math (fLibrary/layers.f90:11-23 linear_layer + activation_funcs.f90, per
// layer): Y[s][n] = act(sum_k A[s][k] W[n][k] + b[n]).  With A = Ah + Al and
// W = Wh + Wl, where Xh = tf32_round(X) and Xl = tf32_round(X - Xh), the
// product is taken as Al*Wh + Ah*Wl + Ah*Wh (the Al*Wl term is below 2^-22
// relative), accumulated in fp32 in tensor memory: fp32-level accuracy from
// the TF32 tensor pipe.
//
// Per CTA (one per SM, persistent over tiles of 128 samples):
//   warp 0, one lane : TMA producer — streams each layer's [Wh | Wl] in K-chunks
//                      of 32 (128-byte swizzled rows) into a 2-stage ring
//   warp 1, one lane : MMA issuer — per chunk 4 K-steps x 3 tcgen05.mma
//                      (M=128 samples, N = layer width, K=8), commits free the
//                      ring stages; warp 1 also owns the TMEM allocation
//   warps 4..7       : converters — thread r owns sample r (TMEM lane r): they
//                      stage the input tile, and between layers read the
//                      accumulator (tcgen05.ld), add bias, apply the
//                      activation, split hi/lo and write the next layer's A
//                      chunk (swizzled, K-major) into a 2-stage ring; the last
//                      layer's epilogue writes the outputs to global memory
// Two accumulators of 256 columns alternate between layers (512 TMEM columns).
// Every wait on an mbarrier is bounded; on time-out the kernel records an error
// code in `err`, drains what it issued, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mlp_tc.cuh"

namespace rosenna {
namespace {

constexpr int kBM = 128;                 // samples per tile (UMMA M)
constexpr int kKC = 32;                  // K per chunk: 32 fp32 = one 128-byte swizzle row
constexpr int kNMax = 256;               // widest layer (UMMA N)
constexpr int kThreadsTc = 320;           // warp 0 TMA, warp 1 MMA, warps 2..9 converters
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTCol = 0;             // TMEM cols [0,256): previous layer's activations
constexpr uint32_t kPCol = 256;           // TMEM cols [256,512): partial sums of column half h at 256+128h
constexpr uint32_t kBTile = kNMax * 128;  // bytes of one B tile (hi or lo)
constexpr uint32_t kATile = kBM * 128;    // bytes of one A tile (hi or lo)
constexpr uint32_t kSmemB = 2 * 2 * kBTile;  // 2 stages x (hi, lo)
constexpr uint32_t kSmemA = 2 * 2 * kATile;
constexpr uint32_t kSmemBias = kTcMaxLayers * kNMax * 4;
constexpr uint32_t kSmemBars = 256;
constexpr uint64_t kWaitNs = 2000000000ull;   // 2 s
constexpr uint32_t kWaitIters = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of `parity` to complete.  Gives up (returns false)
// after kWaitNs / kWaitIters, or as soon as another role has recorded an error.
// The first thread to give up records err[0] = code and, in err[1..6], where it
// waited: block, thread, `where` (caller state), parity and two counters.  A
// thread passing `slot` > 0 also records its own state in err[8*slot ..] when
// it gives up for any reason (block 0 only), so every role's position is known.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code, int where = 0,
                                          int c1 = 0, int c2 = 0, int slot = 0) {
    if (mbar_try_wait(bar, parity)) return true;  // fast path
    const uint64_t t0 = globaltimer();
    bool other = false;
    for (uint32_t i = 0; i < kWaitIters; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*(volatile int *)err) {
            other = true;
            break;
        }
        if ((i & 255) == 255 && globaltimer() - t0 > kWaitNs) break;
    }
    if (!other && code != 0 && atomicCAS(err, 0, code) == 0) {
        err[1] = blockIdx.x;
        err[2] = threadIdx.x;
        err[3] = where;
        err[4] = (int)parity;
        err[5] = c1;
        err[6] = c2;
    }
    if (slot > 0 && blockIdx.x == 0) {
        int *e = err + 8 * slot;
        e[0] = code;
        e[1] = where;
        e[2] = (int)parity;
        e[3] = c1;
        e[4] = c2;
        e[5] = (int)(globaltimer() - t0 > kWaitNs);
    }
    __threadfence();
    return false;
}

// ---- TMA -------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// ---- tcgen05 ----------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// K-major operand, 128-byte swizzle: 8-row atoms of 1024 bytes (SBO), rows of
// 128 bytes; LBO unused for swizzled K-major (set to 16 bytes); version 1.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;              // LBO = 16 B
    d |= (uint64_t)(1024 >> 4) << 32;    // SBO = 1024 B
    d |= (uint64_t)1 << 46;              // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;              // SWIZZLE_128B
    return d;
}

// instruction descriptor: D f32, A/B tf32, both K-major, M=128, N
__device__ __forceinline__ uint32_t idesc_tf32(int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ uint32_t tf32_rna(float x) {
    uint32_t y;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float tc_tanh(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(2.8853900817779268f * x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
    return 1.f - 2.f * r;
}
__device__ __forceinline__ float tc_sigmoid(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
    return r;
}
__device__ __forceinline__ float tc_act(float v, int act) {
    switch (act) {
        case 1: return v < 0.f ? 0.f : v;
        case 2: return tc_tanh(v);
        case 3: return tc_sigmoid(v);
        default: return v;
    }
}

// Writes 16 values (k = k0..k0+15 of this chunk) of row r into the hi/lo A
// tiles in the 128-byte-swizzled K-major layout.
__device__ __forceinline__ void put_a16(uint8_t *ahi, uint8_t *alo, int r, int k0, const float (&v)[16]) {
    const uint32_t row = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            h[e] = tf32_rna(v[4 * q + e]);
            l[e] = tf32_rna(v[4 * q + e] - __uint_as_float(h[e]));
        }
        const uint32_t chunk = (uint32_t)((k0 >> 2) + q);
        const uint32_t off = row + ((chunk ^ (uint32_t)(r & 7)) << 4);
        *reinterpret_cast<uint4 *>(ahi + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(alo + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])));
}

// Which converter group (column half) stages A chunk c of layer l: the input
// layer alternates; hidden layers read chunk c from the half holding its columns.
__device__ __forceinline__ int a_owner(int l, int c) { return l == 0 ? (c & 1) : (c >> 2); }

// Stages A chunk c of layer l (tile t) into A ring slot j&1 for this thread's
// row: the input layer from global memory, hidden layers from TMEM (the
// previous layer's activations), split into tf32 hi/lo, 128-byte swizzled.
// The slot is known free (chunk j-2 was seen consumed).
__device__ __forceinline__ void stage_a(const TcArgs &p, uint8_t *a0, uint32_t lane_base, int r, int t, int l, int c,
                                        uint32_t j) {
    uint8_t *ahi = a0 + (j & 1) * 2 * kATile;
#pragma unroll 1
    for (int h = 0; h < 2; h++) {
        float v[16];
        if (l == 0) {
            const long long row = (long long)t * kBM + r;
            const bool valid = row < p.n;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                const int k = c * kKC + h * 16 + e;
                v[e] = (valid && k < p.L[0].K) ? __ldg(p.in + (long long)k * p.ld_in + row) : 0.f;
            }
        } else {
            tmem_ld16(lane_base + kTCol + (uint32_t)(c * kKC + h * 16), v);
        }
        put_a16(ahi, ahi + kATile, r, h * 16, v);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    mbar_arrive(reinterpret_cast<uint64_t *>(a0 + kSmemA + kSmemBias) + 4 + (j & 1));  // a_full[j & 1]
}

__global__ void __launch_bounds__(kThreadsTc, 1) mlp_tc_kernel(const __grid_constant__ TcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const b0 = base;                   // B stage s: hi at b0 + s*2*kBTile, lo + kBTile
    uint8_t *const a0 = base + kSmemB;          // A stage s: hi at a0 + s*2*kATile, lo + kATile
    float *const sbias = reinterpret_cast<float *>(base + kSmemB + kSmemA);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(base + kSmemB + kSmemA + kSmemBias);
    uint64_t *const b_full = bars, *const b_empty = bars + 2, *const a_full = bars + 4, *const a_empty = bars + 6;
    uint64_t *const p_full = bars + 8, *const p_empty = bars + 10, *const drain = bars + 12;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nl = p.nlayers;
    const long long ntiles = (p.n + kBM - 1) / kBM;

    for (int i = tid; i < nl * kNMax; i += kThreadsTc) {
        const int l = i / kNMax, j = i - l * kNMax;
        sbias[i] = j < p.L[l].Np ? p.arena[p.L[l].b_off + j] : 0.f;
    }
    if (tid == 0) {
        for (int s = 0; s < 2; s++) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
            mbar_init(&a_full[s], kBM);
            mbar_init(&a_empty[s], 1);
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], kBM);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        for (int l = 0; l < nl; l++) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.maps[l]) : "memory");
        uint32_t i = 0;  // chunk counter over (tile, layer, chunk)
        bool ok = true;
        for (long long t = blockIdx.x; t < ntiles && ok; t += gridDim.x)
            for (int l = 0; l < nl && ok; l++)
                for (int c = 0; c < p.L[l].nch && ok; c++, i++) {
                    const int s = i & 1;
                    if (!(ok = mbar_wait(&b_empty[s], ((i >> 1) & 1) ^ 1, p.err, 1, (l << 8) | c, (int)i, 0, 1))) break;
                    mbar_arrive_expect_tx(&b_full[s], 2u * (uint32_t)p.L[l].Np * 128u);
                    tma_load_2d(b0 + s * 2 * kBTile, &p.maps[l], &b_full[s], c * kKC, 0);
                    tma_load_2d(b0 + s * 2 * kBTile + kBTile, &p.maps[l], &b_full[s], c * kKC, p.L[l].Np);
                }
        // copies still in flight land before the CTA may exit
        for (uint32_t k = (i > 2 ? i - 2 : 0); k < i; k++) mbar_wait(&b_full[k & 1], (k >> 1) & 1, p.err, 0);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        // per chunk of 32 K: two partials of 16 K per column half, each started fresh
        // (the partials are summed in fp32 registers by the converters)
        uint32_t ib = 0, ia = 0, pu[2] = {0, 0};
        bool ok = true;
        for (long long t = blockIdx.x; t < ntiles && ok; t += gridDim.x)
            for (int l = 0; l < nl && ok; l++) {
                const int Np = p.L[l].Np, nh = (Np + 127) >> 7;
                for (int c = 0; c < p.L[l].nch && ok; c++, ib++, ia++) {
                    const int sb = ib & 1, sa = ia & 1;
                    if (!(ok = mbar_wait(&b_full[sb], (ib >> 1) & 1, p.err, 2, (l << 8) | c, (int)ib, 0, 2))) break;
                    if (!(ok = mbar_wait(&a_full[sa], (ia >> 1) & 1, p.err, 3, (l << 8) | c, (int)ia, 0, 2))) break;
                    tc_fence_after();
                    const uint64_t ah = desc_kmajor_sw128(smem_u32(a0 + sa * 2 * kATile));
                    const uint64_t al = desc_kmajor_sw128(smem_u32(a0 + sa * 2 * kATile + kATile));
                    const uint64_t bh = desc_kmajor_sw128(smem_u32(b0 + sb * 2 * kBTile));
                    const uint64_t bl = desc_kmajor_sw128(smem_u32(b0 + sb * 2 * kBTile + kBTile));
                    for (int sub = 0; sub < 2 && ok; sub++)
                        for (int h = 0; h < nh && ok; h++) {
                            const int Nh = min(128, Np - 128 * h);
                            if (!(ok = mbar_wait(&p_empty[h], (pu[h] & 1) ^ 1, p.err, 4, (l << 16) | (c << 8) | (sub << 4) | h,
                                                 (int)pu[h], (int)ia, 2)))
                                break;
                            tc_fence_after();
                            const uint32_t d = tmem + kPCol + (uint32_t)(128 * h);
                            const uint32_t idesc = idesc_tf32(Nh);
                            const uint64_t boff = (uint64_t)(h * 128 * 128) >> 4;  // rows 128h.. of the B tiles
#pragma unroll
                            for (int kq = 0; kq < 2; kq++) {
                                const int kk = 2 * sub + kq;
                                const uint64_t adv = (uint64_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes along K
                                umma_tf32(d, al + adv, bh + boff + adv, idesc, kq);
                                umma_tf32(d, ah + adv, bl + boff + adv, idesc, 1);
                                umma_tf32(d, ah + adv, bh + boff + adv, idesc, 1);
                            }
                            umma_commit(&p_full[h]);
                            pu[h]++;
                        }
                    if (!ok) break;
                    umma_commit(&a_empty[sa]);
                    umma_commit(&b_empty[sb]);
                }
            }
        // drain: every MMA issued above has completed before TMEM is freed
        umma_commit(drain);
        mbar_wait(drain, 0, p.err, 0);
    } else if (warp >= 2) {
        // ---------------- converters: group g owns output columns [128g, 128g+128) ----------------
        const int g = (warp - 2) >> 2, quad = warp & 3;
        const int r = quad * 32 + lane;  // sample row in the tile == TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const int slot = (lane == 0 && quad == 2) ? 3 + g : 0;  // diagnostics of this group
        uint32_t ia = 0, pu = 0;
        bool ok = true;
        float acc[128];
        for (int t = blockIdx.x; t < (int)ntiles && ok; t += gridDim.x) {
            for (int l = 0; l < nl && ok; l++) {
                const int nch = p.L[l].nch;
                const bool has_half = 128 * g < p.L[l].Np;
#pragma unroll
                for (int q = 0; q < 128; q++) acc[q] = 0.f;
                if (a_owner(l, 0) == g) stage_a(p, a0, lane_base, r, t, l, 0, ia);
                if (nch > 1 && a_owner(l, 1) == g) stage_a(p, a0, lane_base, r, t, l, 1, ia + 1);
                for (int c = 0; c < nch && ok; c++) {
                    if (has_half) {
#pragma unroll 1
                        for (int sub = 0; sub < 2 && ok; sub++) {
                            // one 16-deep partial of this half: add it into acc
                            ok = __all_sync(0xffffffffu, mbar_wait(&p_full[g], pu & 1, p.err, 6, (l << 16) | (c << 8) | sub,
                                                                   (int)pu, (int)ia, slot));
                            if (!ok) break;
                            tc_fence_after();
                            const int Np = p.L[l].Np;
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                if (128 * g + 16 * q < Np) {
                                    float v[16];
                                    tmem_ld16(lane_base + kPCol + (uint32_t)(128 * g + 16 * q), v);
#pragma unroll
                                    for (int e = 0; e < 16; e++) acc[16 * q + e] += v[e];
                                }
                            }
                            tc_fence_before();
                            mbar_arrive(&p_empty[g]);
                            pu++;
                        }
                        if (!ok) break;
                    }
                    // Every converter thread observes the consumption of every A chunk in
                    // order (whichever group staged it), so each a_empty phase is awaited by
                    // a thread that has seen the previous one: the parity test cannot alias.
                    const uint32_t j = ia + (uint32_t)c;
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&a_empty[j & 1], (j >> 1) & 1, p.err, 5, (l << 8) | c, (int)j, (int)pu, slot));
                    if (ok && c + 2 < nch && a_owner(l, c + 2) == g) stage_a(p, a0, lane_base, r, t, l, c + 2, j + 2);
                }
                ia += (uint32_t)nch;
                if (!ok || !has_half) continue;
                // bias + activation of this half; into T for the next layer, or out
                const float *bias = sbias + l * kNMax + 128 * g;
                const int N = p.L[l].N, act = p.L[l].act;
                if (l + 1 < nl) {
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        float v[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) {
                            const int col = 128 * g + 16 * q + e;
                            v[e] = col < N ? tc_act(acc[16 * q + e] + bias[16 * q + e], act) : 0.f;
                        }
                        tmem_st16(lane_base + kTCol + (uint32_t)(128 * g + 16 * q), v);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                } else {
                    const long long row0 = (long long)t * kBM + r;
                    if (row0 < p.n) {
                        float *o = p.out + row0 + (long long)(128 * g) * p.ld_out;
#pragma unroll
                        for (int q = 0; q < 128; q++)
                            if (128 * g + q < N) o[(long long)q * p.ld_out] = tc_act(acc[q] + bias[q], act);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

size_t mlp_tc_smem_bytes() { return 1024 + kSmemB + kSmemA + kSmemBias + kSmemBars; }

cudaError_t mlp_tc_configure() {
    return cudaFuncSetAttribute(mlp_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mlp_tc_smem_bytes());
}

cudaError_t launch_mlp_tc(const TcArgs &a, int num_sms, cudaStream_t st) {
    const long long tiles = (a.n + kBM - 1) / kBM;
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid <= 0) return cudaSuccess;
    mlp_tc_kernel<<<grid, kThreadsTc, mlp_tc_smem_bytes(), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna

namespace rosenna {

bool mlp_tc_encode_map(CUtensorMap *map, const float *block, int Kp, int Np, const char **why) {
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
    const cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)(2 * Np)};
    const cuuint64_t strides[1] = {(cuuint64_t)Kp * sizeof(float)};
    const cuuint32_t box[2] = {32, (cuuint32_t)Np};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(block), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *why = "cuTensorMapEncodeTiled rejected a weight block";
        return false;
    }
    return true;
}

}  // namespace rosenna
