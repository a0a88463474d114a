// Convolution as an implicit GEMM on the tensor cores (tcgen05, 3xTF32), fused
// with its ReLU and the following 2x2 pool (fLibrary/layers.f90 conv :183-233,
// relu4d activation_funcs.f90:43-52, max_pool/avgpool :236-310).
//
// Shapes: 3x3 kernel, stride 1, symmetric zero padding 0..2, 1 to 8 input and
// up to 16 output channels, a k=2 s=2 pool without padding over an even conv
// output.
//
// Samples are the GEMM's N dimension (128 per tile).  The batch is stored
// sample-fastest (element (c, y, x) of sample s at in[(c + C*(y + Hin*x))*ld
// + s]), so the input patch of 32 consecutive samples is a 4-D TMA box {32
// samples, cb channels, ph rows, cw columns}: it lands in shared memory as
// 128-byte K-rows of 32 samples, which is the B operand MN-major (K = position
// x channel) in the one layout an MN-major 32-bit operand may take: 128-byte
// swizzle with 32-byte atoms (TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).  The zero padding, and
// channels past C, come from the TMA's out-of-bounds fill.  Threads only split
// the loaded values into tf32 hi and lo parts.
//
// The M = 128 GEMM rows are a block of bh x 4 conv pixels x ocp output channels
// (bh*ocp = 32), ordered (column q from the right, row, channel): row 32q +
// ocp*i + oc is conv pixel (y0 + i, x0 + 3 - q).  With that order the weights
// for patch column pw are the 128-row window, starting at row 32*pw, of one
// 288-row matrix S whose row 32j + ocp*i + oc holds kernel column kw = j - 3
// (zero outside 0..2) over the patch rows: K-slot c + cb*r holds
// W[oc][c][r - i][j - 3] (zero outside the kernel).  S (tf32 hi and lo parts,
// 72 KB) stays in shared memory for the whole kernel, and each K-step of 8
// K-slots is three MMAs, Sl*Bh + Sh*Bl + Sh*Bh, of N = 128 samples (an M = 128
// tf32 MMA takes the same time for every N up to 128, so N = 128 uses the
// tensor core fully).  Rows of pixels outside the image or of padded channels
// are computed and not stored.
//
// Pool: a window's two conv rows are lanes ocp apart in one warp (a shuffle);
// its two columns are TMEM lane quadrants q and q^1, i.e. two warps, which meet
// through shared memory (mbarrier hand-off over two buffers).
//
// Roles (320 threads): warp 0 lane 0 loads chunks by TMA into a ring of slots,
// warps 2-5 split each chunk into hi and lo in place, warp 1 lane 0 issues the
// MMAs, warps 6-9 drain the double-buffered TMEM accumulator (warp w reads lane
// quadrant w % 4): bias, ReLU, pool, store.  Work is (128-sample tile, block)
// units, a contiguous range of them per CTA.  Every wait is bounded; a time-out
// records where in `err`, every role finishes, copies in flight are waited
// for, TMEM is freed.
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
constexpr int kCtMaxSlots = 4;
constexpr uint32_t kCtSBytes = kConvTcBFloats * 4;  // S hi then S lo
constexpr uint32_t kCtSLo = kCtSBytes / 2;
constexpr uint32_t kCtXBytes = 2 * 2 * 16 * 32 * 4;  // pool hand-off [pair][buffer][16 rows][32 samples]
constexpr uint32_t kCtTmemCols = 256;               // two accumulators of 128 columns
constexpr size_t kCtSmemMax = 232448;

enum {
    kCtFull = 0,                        // [slot] chunk landed (TMA bytes)
    kCtSplit = kCtFull + kCtMaxSlots,   // [slot] split into hi and lo (128 arrivals)
    kCtEmpty = kCtSplit + kCtMaxSlots,  // [slot] MMAs done with it (commit)
    kCtDFull = kCtEmpty + kCtMaxSlots,  // [2] accumulator complete (commit)
    kCtDEmpty = kCtDFull + 2,           // [2] accumulator drained (128 arrivals)
    kCtXFull = kCtDEmpty + 2,           // [pair][buffer] hand-off written (32 arrivals)
    kCtXEmpty = kCtXFull + 4,           // [pair][buffer] hand-off read (32 arrivals)
    kCtDone = kCtXEmpty + 4,
    kCtNumBars = kCtDone + 1
};

size_t conv_tc_smem(int rows, int slots) {
    return 1024 + kCtSBytes + (size_t)slots * rows * 1024 + kCtXBytes + 64 + 8 * kCtNumBars + 16;
}

struct CtUnit {
    long long t;  // sample tile
    int y0, x0;   // the block's first conv row and column
};

__device__ __forceinline__ CtUnit ct_unit(const ConvTcArgs &p, long long u, int nbw, int nblk) {
    CtUnit c;
    c.t = u / nblk;
    const int blk = (int)(u - c.t * nblk);
    const int bi = blk / nbw;
    c.y0 = bi * p.bh;
    c.x0 = (blk - bi * nbw) * 4;
    return c;
}

__device__ __forceinline__ void ct_split(float x, float &h, float &l) {
    h = __uint_as_float(tf32_rna(x));
    l = x - h;
}

__device__ __forceinline__ void st_global_v4(float *dst, float a, float b, float c, float d) {
    asm volatile("st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__global__ void __launch_bounds__(kCtThreads, 1) conv_tc_kernel(const __grid_constant__ ConvTcArgs p) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t *const base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *const ring = base + kCtSBytes;
    const uint32_t slot_bytes = (uint32_t)p.rows * 1024u;  // hi part (rows x 128 samples x 4 B), then lo part
    const uint32_t half = slot_bytes / 2;
    float *const xch = reinterpret_cast<float *>(ring + (size_t)p.slots * slot_bytes);
    float *const sbias = xch + kCtXBytes / 4;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(sbias + 16);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + kCtNumBars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nbw = (p.Wo + 3) / 4, nblk = ((p.Ho + p.bh - 1) / p.bh) * nbw;
    const long long units = ((p.n + 127) / 128) * nblk;
    const long long u0 = units * blockIdx.x / gridDim.x, u1 = units * (blockIdx.x + 1) / gridDim.x;
    const int nck = 6 / p.cw, kcol = p.cb * p.ph / 8;  // chunks per block, K-steps per patch column

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
            mbar_init(bars + kCtSplit + i, 128);
            mbar_init(bars + kCtEmpty + i, 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bars + kCtDFull + i, 1);
            mbar_init(bars + kCtDEmpty + i, 128);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(bars + kCtXFull + i, 32);
            mbar_init(bars + kCtXEmpty + i, 32);
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
            // ---- TMA: each chunk as four boxes of 32 samples ----
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.map) : "memory");
            uint32_t it = 0;
            bool ok = true;
            for (long long u = u0; u < u1 && ok; u++) {
                const CtUnit c = ct_unit(p, u, nbw, nblk);
                for (int ck = 0; ck < nck; ck++, it++) {
                    const uint32_t s = it % (uint32_t)p.slots, k = it / (uint32_t)p.slots;
                    if (k > 0 && !(ok = mbar_wait(bars + kCtEmpty + s, (k - 1) & 1, p.err, 71, (int)u, ck))) break;
                    uint8_t *dst = ring + s * slot_bytes;
                    mbar_arrive_expect_tx(bars + kCtFull + s, half);
                    for (int g = 0; g < 4; g++)
                        tma_load_4d(dst + (uint32_t)g * (uint32_t)p.rows * 128u, &p.map, bars + kCtFull + s,
                                    (int)(c.t * 128 + 32 * g), 0, c.y0 - p.pad, c.x0 - p.pad + ck * p.cw);
                }
            }
            // the last chunks' copies land before the CTA exits
            const uint32_t ns = (uint32_t)p.slots;
            for (uint32_t i = it > ns ? it - ns : 0; i < it; i++) mbar_drain(bars + kCtFull + i % ns, (i / ns) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            const uint32_t sh = smem_u32(base), sl = sh + kCtSLo, idesc = idesc_tf32_bmn(128);
            const uint32_t lbo = (uint32_t)p.rows * 128u;  // between the 32-sample groups of a part
            uint32_t it = 0, uu = 0;
            bool ok = true;
            for (long long u = u0; u < u1 && ok; u++, uu++) {
                const uint32_t b = uu & 1, m = uu >> 1;
                if (m > 0 && !(ok = mbar_wait(bars + kCtDEmpty + b, (m - 1) & 1, p.err, 72, (int)u))) break;
                tc_fence_after();
                const uint32_t d = tmem + 128u * b;
                for (int ck = 0; ck < nck && ok; ck++, it++) {
                    const uint32_t s = it % (uint32_t)p.slots, k = it / (uint32_t)p.slots;
                    if (!(ok = mbar_wait(bars + kCtSplit + s, k & 1, p.err, 73, (int)u, ck))) break;
                    tc_fence_after();
                    const uint32_t bh = smem_u32(ring + s * slot_bytes), bl = bh + half;
                    for (int pwl = 0; pwl < p.cw; pwl++)
                        for (int g = 0; g < kcol; g++) {
                            const uint32_t aoff = (uint32_t)(ck * p.cw + pwl) * 4096u + 32u * (uint32_t)g;
                            const uint32_t boff = (uint32_t)(pwl * kcol + g) * 1024u;
                            const uint32_t acc = (ck | pwl | g) ? 1u : 0u;
                            umma_tf32_bmn(d, desc_lo(sl + aoff), desc_mn_lo(bh + boff, lbo), idesc, acc);
                            umma_tf32_bmn(d, desc_lo(sh + aoff), desc_mn_lo(bl + boff, lbo), idesc, 1u);
                            umma_tf32_bmn(d, desc_lo(sh + aoff), desc_mn_lo(bh + boff, lbo), idesc, 1u);
                        }
                    umma_commit(bars + kCtEmpty + s);
                }
                if (ok) umma_commit(bars + kCtDFull + b);
            }
            umma_commit(bars + kCtDone);
            mbar_drain(bars + kCtDone, 0);
        }
    } else if (warp < 6) {
        // ---- split each chunk into tf32 hi (in place) and lo ----
        const int st = tid - 64;
        uint32_t it = 0;
        bool ok = true;
        for (long long u = u0; u < u1 && ok; u++)
            for (int ck = 0; ck < nck; ck++, it++) {
                const uint32_t s = it % (uint32_t)p.slots, k = it / (uint32_t)p.slots;
                ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtFull + s, k & 1, p.err, 74, (int)u, ck));
                if (!ok) break;
                float4 *hi = reinterpret_cast<float4 *>(ring + s * slot_bytes);
                float4 *lo = reinterpret_cast<float4 *>(ring + s * slot_bytes + half);
                const int nv = p.rows * 32;  // float4s per part
                for (int i = st; i < nv; i += 128) {
                    const float4 v = hi[i];
                    float4 h, l;
                    ct_split(v.x, h.x, l.x);
                    ct_split(v.y, h.y, l.y);
                    ct_split(v.z, h.z, l.z);
                    ct_split(v.w, h.w, l.w);
                    hi[i] = h;
                    lo[i] = l;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(bars + kCtSplit + s);
            }
    } else {
        // ---- drain: bias, ReLU, pool over rows (shuffle) and columns (hand-off), store ----
        const int q = warp & 3, pair = q >> 1, odd = q & 1;
        const int ih = lane / p.ocp, oc = lane - ih * p.ocp, iw = 3 - q;
        const bool keep = (ih & 1) == 0;        // the window's upper row holds the row-pooled value
        const int li = (ih >> 1) * p.ocp + oc;  // hand-off row, 0..15
        const float bias = sbias[oc];
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        uint32_t uu = 0, pass = 0;
        bool ok = true;
        for (long long u = u0; u < u1 && ok; u++, uu++) {
            const CtUnit c = ct_unit(p, u, nbw, nblk);
            const uint32_t b = uu & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtDFull + b, (uu >> 1) & 1, p.err, 75, (int)u));
            if (!ok) break;
            tc_fence_after();
            const int qy = (c.y0 + ih) >> 1, qx = (c.x0 + iw) >> 1;
            const bool store = keep && qy < p.Hq && qx < p.Wq && oc < p.OC;
            for (int cc = 0; cc < 4; cc++, pass++) {
                uint32_t w0[16], w1[16];
                tmem_ld16_nw(lane_base + 128u * b + 32u * (uint32_t)cc, w0);
                tmem_ld16_nw(lane_base + 128u * b + 32u * (uint32_t)cc + 16u, w1);
                tmem_wait_ld();
                if (cc == 3) {
                    tc_fence_before();
                    mbar_arrive(bars + kCtDEmpty + b);
                }
                float v[32];
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    v[e] = __uint_as_float(w0[e]) + bias;
                    v[16 + e] = __uint_as_float(w1[e]) + bias;
                }
                if (p.relu) {
#pragma unroll
                    for (int e = 0; e < 32; e++) v[e] = fmaxf(v[e], 0.f);
                }
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    const float o = __shfl_xor_sync(0xffffffffu, v[e], p.ocp);
                    v[e] = p.pool == 1 ? fmaxf(v[e], o) : v[e] + o;
                }
                const uint32_t xb = (uint32_t)pair * 2 + (pass & 1), use = pass >> 1;
                float4 *xv = reinterpret_cast<float4 *>(xch + (xb * 16 + (uint32_t)li) * 32);
                if (odd) {
                    if (use > 0)
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(bars + kCtXEmpty + xb, (use - 1) & 1, p.err, 76, (int)u, cc));
                    if (!ok) break;
                    if (keep) {
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            xv[j ^ (li & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    }
                    mbar_arrive(bars + kCtXFull + xb);
                } else {
                    ok = __all_sync(0xffffffffu, mbar_wait(bars + kCtXFull + xb, use & 1, p.err, 77, (int)u, cc));
                    if (!ok) break;
                    float4 o[8];
                    if (keep) {
#pragma unroll
                        for (int j = 0; j < 8; j++) o[j] = xv[j ^ (li & 7)];
                    }
                    mbar_arrive(bars + kCtXEmpty + xb);
                    if (store) {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            if (p.pool == 1) {
                                v[4 * j] = fmaxf(v[4 * j], o[j].x);
                                v[4 * j + 1] = fmaxf(v[4 * j + 1], o[j].y);
                                v[4 * j + 2] = fmaxf(v[4 * j + 2], o[j].z);
                                v[4 * j + 3] = fmaxf(v[4 * j + 3], o[j].w);
                            } else {
                                v[4 * j] = (v[4 * j] + o[j].x) * 0.25f;
                                v[4 * j + 1] = (v[4 * j + 1] + o[j].y) * 0.25f;
                                v[4 * j + 2] = (v[4 * j + 2] + o[j].z) * 0.25f;
                                v[4 * j + 3] = (v[4 * j + 3] + o[j].w) * 0.25f;
                            }
                        }
                        const long long s0 = c.t * 128 + 32 * cc;
                        float *dst =
                            p.out +
                            ((long long)oc * p.so_c + (long long)qy * p.so_h + (long long)qx * p.so_w) * p.ld_out + s0;
                        if (p.vec_out && s0 + 32 <= p.n) {
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                st_global_v4(dst + 4 * j, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                        } else {
#pragma unroll
                            for (int e = 0; e < 32; e++)
                                if (s0 + e < p.n) dst[e] = v[e];
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
        while (g.cw > 1 && (per_col * g.cw > 48 || 6 % g.cw)) g.cw--;
        g.rows = per_col * g.cw;
        const size_t fixed = conv_tc_smem(g.rows, 0);
        g.slots = (int)((kCtSmemMax - fixed) / ((size_t)g.rows * 1024));
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
    const cuuint32_t box[4] = {32, (cuuint32_t)a.cb, (cuuint32_t)a.ph, (cuuint32_t)a.cw};
    return tc_encode_f32_map(&a.map, 4, in, dims, strides, box, why, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

cudaError_t conv_tc_configure() {
    return cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCtSmemMax);
}

cudaError_t launch_conv_tc(const ConvTcArgs &a, int num_sms, cudaStream_t st) {
    const bool geom = (a.ocp == 8 || a.ocp == 16) && a.bh * a.ocp == 32 && a.cw >= 1 && 6 % a.cw == 0 &&
                      (a.cb * a.ph) % 8 == 0 && a.cb * a.ph <= 32 && a.ph >= a.bh + 2 &&
                      a.rows == a.cb * a.ph * a.cw && a.slots >= 2 && a.slots <= kCtMaxSlots && a.OC >= 1 &&
                      a.OC <= 16 && a.C >= 1 && a.C <= a.cb && (a.pool == 1 || a.pool == 2) &&
                      conv_tc_smem(a.rows, a.slots) <= kCtSmemMax;
    if (!geom) return cudaErrorInvalidConfiguration;
    const long long units = ((a.n + 127) / 128) * (long long)(((a.Ho + a.bh - 1) / a.bh) * ((a.Wo + 3) / 4));
    const int grid = (int)(units < num_sms ? units : num_sms);
    if (grid <= 0) return cudaSuccess;
    conv_tc_kernel<<<grid, kCtThreads, conv_tc_smem(a.rows, a.slots), st>>>(a);
    return cudaGetLastError();
}

}  // namespace rosenna
