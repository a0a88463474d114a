// Device helpers shared by the tcgen05 kernels (mlp_tc.cu, conv_tc.cu):
// bounded mbarrier waits, TMA loads, tcgen05 MMA / commit / TMEM load-store in
// inline PTX, the K-major 128-byte-swizzle descriptors, tf32 rounding, the
// activations and the hi/lo A-tile writer.  Every function is internal to the
// translation unit that includes this header.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace rosenna {
namespace {

constexpr int kUmmaM = 128;  // rows of every UMMA tile (samples; TMEM lanes)
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
// Bounded wait that does not stop at a recorded error: at exit, for copies a
// role issued that may still be in flight.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0; i < kWaitIters; i++) {
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 255) == 255 && globaltimer() - t0 > kWaitNs) return;
    }
}

// Named barrier `id` over `nthreads` threads that also returns the AND of
// every participant's `v`, so a group of warps leaves a loop together.
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// ---- TMA -------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 4-D tile {c0 innermost, c1, c2, c3}; coordinates past either end of a
// dimension read as zeros
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// 4-D tile store from shared memory (bulk-group completion); parts of the box
// past the end of a dimension are not written.  Coordinates must not be
// negative.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// waits until at most N committed bulk groups still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// waits until at most N committed bulk groups are incomplete
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
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

// the same without the wait: several loads in flight before tmem_wait_ld()
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Two fp32 lanes per instruction (sm_100 packed f32x2, round to nearest):
// (a0, a1) += (bits b0, b1).  Same results as two scalar FADDs in half the
// issue slots.
__device__ __forceinline__ void add2(float &a0, float &a1, uint32_t b0, uint32_t b1) {
    asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\t"
        "add.rn.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(b0), "r"(b1));
}

// (a0, a1) += x * (w0, w1) on one packed f32x2 FMA (round to nearest: the
// results of two scalar FMAs in one issue slot).
__device__ __forceinline__ void fma2x(float &a0, float &a1, float x, float w0, float w1) {
    asm("{\n\t.reg .b64 a, b, c;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %2};\n\tmov.b64 c, {%3, %4};\n\t"
        "fma.rn.f32x2 a, b, c, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(x), "f"(w0), "f"(w1));
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
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kUmmaM >> 4) << 24);
}

// Round to tf32 (10 explicit mantissa bits), to nearest with ties away from
// zero: add half a tf32 ulp to the magnitude bits and clear the 13 low bits.
// Two integer-pipe operations per value; the conversion instruction runs at a
// fraction of that rate, and staging converts 64 values per thread per chunk.
// A carry out of the mantissa rounds up into the exponent, as it should (to
// infinity past the largest float).
__device__ __forceinline__ uint32_t tf32_rna(float x) { return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u; }
// The lo part of an activation's split, x - hi (exact in fp32), left
// unrounded: the tensor core reads a tf32 operand's top 19 bits, so it drops
// lo's low 13 bits itself.  |lo| <= 2^-11 |x| once hi is rounded to nearest,
// so what it drops is below 2^-22 |x|, with the sign of lo (either way, not a
// bias); rounding lo here as well (2^-23) cost three more instructions per
// value on the epilogue and split paths.
__device__ __forceinline__ uint32_t tf32_lo(float x, uint32_t hi) { return __float_as_uint(x - __uint_as_float(hi)); }

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
template <int ACT>
__device__ __forceinline__ float tc_act(float v) {
    if (ACT == 1) return v < 0.f ? 0.f : v;
    if (ACT == 2) return tc_tanh(v);
    if (ACT == 3) return tc_sigmoid(v);
    return v;
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
            l[e] = tf32_lo(v[4 * q + e], h[e]);
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
        "r"(__float_as_uint(v[15]))
        : "memory");
}

// tcgen05.mma kind::tf32 with the descriptors given by their low words (start
// address and LBO) over the common high word of desc_kmajor_sw128 (SBO 1024 B,
// version 1, 128-byte swizzle): one register per descriptor.
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr) { return ((saddr & 0x3FFFFu) >> 4) | (1u << 16); }
__device__ __forceinline__ void umma_tf32_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t idesc,
                                             uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "mov.b64 da, {%1, %5};\n\t"
        "mov.b64 db, {%2, %5};\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], da, db, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(acc), "n"(kDescHi));
}
// The same with A read from TMEM (a_tmem: the column of its first K element,
// lanes 0..127 = the M rows) and B from shared memory (K-major, 128-byte
// swizzle, b_lo from desc_lo).
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t idesc,
                                             uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "mov.b64 db, {%2, %5};\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], db, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(acc), "n"(kDescHi));
}

// 32 lanes x 32 bits, 8 consecutive columns per thread
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
// 32 lanes x 32 bits, 32 consecutive columns per thread (no wait)
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

}  // namespace
}  // namespace rosenna
