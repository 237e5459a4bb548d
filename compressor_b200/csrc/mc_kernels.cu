// mc_kernels.cu -- sm_100a kernels of the FalCom momentum codec.
//
// Memory-bound integer / fp32 work: no tensor cores.  Every float operation
// that feeds a payload byte is written as an explicit round-to-nearest
// intrinsic (__fmaf_rn, __fmul_rn, __fsub_rn, __fadd_rn, __fdiv_rn) in the
// order the reference build uses (momentum_compressor_openmp_simd_final.c,
// compiled -O3 -ffast-math with FMA contraction), and this file is compiled
// with -fmad=false so the compiler adds no contraction of its own.
//
// Encoder, one streaming launch per pass over the batch tile list
// (persistent CTAs, tiles staged in shared memory by bulk copies):
//   pass1  stats sums, min/max, per-kernel sign consistency -> bitmap and
//          dominant-sign words, history copy          (ref :1322-1431, :2040-2062)
//   pass2  squared deviations around the float means   (ref :1384-1416)
//   pass3  memory update, prediction, clamped residual, max|r|, mismatches
//          (ref :2094-2170)
//   pass4  residual codec (q8 / int4 / raw) and dense dominant-sign packing
//          (ref :2196-2214 replaced; :2258-2283)
// zstd frames with Raw / RLE blocks for bitmap, signs and lossless payloads
// are written in place by passes 1 and 4 (ref :2222-2256 framing via libzstd
// replaced).  Every pass writes per-tile partials; a finalize kernel after
// passes 1-3 (one CTA per item) reduces them in tile order, so every result
// is run-to-run deterministic.
//
// Decoder: prefix (predicted-kernel offsets per tile) then reconstruct
// (ref :3186-3474), plus an optional frame-expansion kernel for
// device-resident zstd frames.

#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include <type_traits>

#include "mc_device.h"

#define TPB 256
#define NWARP (TPB / 32)
#define FULL 0xffffffffu
#define ZBLOCK 131072

namespace {

__device__ __forceinline__ float x86max(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ float x86min(float a, float b) { return a < b ? a : b; }

__device__ __forceinline__ uint32_t fdiv32(uint32_t x, mc_fastdiv d) {
    uint32_t hi = __umulhi(x, d.mul);
    return (uint32_t)(((uint64_t)hi + x) >> d.shift);
}

// Programmatic dependent launch.  The kernels of one encode (or decode) are
// launched so that kernel N+1 may start while kernel N is finishing; N+1
// plans its tiles and starts their bulk copies, then waits (pdl_wait) for N
// to complete before it reads N's results or writes anything.  Every kernel
// releases its successor (pdl_release) only after its own wait, so when
// kernel N+1 starts, kernels N-1, N-2, ... have completed: a prologue may
// read their outputs.  Both are no-ops for a kernel launched without the
// attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- deterministic block reductions (result valid in thread 0) ---------
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_min_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float u = __shfl_xor_sync(FULL, v, o);
        v = u < v ? u : v;
    }
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float u = __shfl_xor_sync(FULL, v, o);
        v = u > v ? u : v;
    }
    return v;
}

struct Red {
    double d[4][NWARP];
    float f[3][NWARP];
    long long l[2][NWARP];
};

// Reduce ND doubles, the floats selected by F (bit 0 mn: min, bit 1 mx: max,
// bit 2 mx2: max) and NL integers over the block; the result is valid in
// thread 0.  Only the selected values are exchanged.
#define RF_MN 1
#define RF_MX 2
#define RF_MX2 4
template <int ND, int F, int NL>
__device__ void block_reduce(Red &sh, double (&d)[4], float &mn, float &mx, float &mx2, long long (&l)[2]) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < ND; i++) d[i] = warp_sum_d(d[i]);
    if (F & RF_MN) mn = warp_min_f(mn);
    if (F & RF_MX) mx = warp_max_f(mx);
    if (F & RF_MX2) mx2 = warp_max_f(mx2);
#pragma unroll
    for (int i = 0; i < NL; i++) l[i] = warp_sum_ll(l[i]);
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < ND; i++) sh.d[i][w] = d[i];
        if (F & RF_MN) sh.f[0][w] = mn;
        if (F & RF_MX) sh.f[1][w] = mx;
        if (F & RF_MX2) sh.f[2][w] = mx2;
#pragma unroll
        for (int i = 0; i < NL; i++) sh.l[i][w] = l[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int i = 0; i < ND; i++) {
            double s = 0.0;
            for (int j = 0; j < NWARP; j++) s += sh.d[i][j];
            d[i] = s;
        }
        for (int j = 0; j < NWARP; j++) {
            if (F & RF_MN) mn = sh.f[0][j] < mn ? sh.f[0][j] : mn;
            if (F & RF_MX) mx = sh.f[1][j] > mx ? sh.f[1][j] : mx;
            if (F & RF_MX2) mx2 = sh.f[2][j] > mx2 ? sh.f[2][j] : mx2;
        }
#pragma unroll
        for (int i = 0; i < NL; i++) {
            long long s = 0;
            for (int j = 0; j < NWARP; j++) s += sh.l[i][j];
            l[i] = s;
        }
    }
}

// Exclusive scan of one int per thread over the block; returns the prefix.
__device__ int block_excl_scan(int v, int *sh, int *total) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(FULL, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int j = 0; j < NWARP; j++) {
            int t = sh[j];
            sh[j] = acc;
            acc += t;
        }
        sh[NWARP] = acc;
    }
    __syncthreads();
    if (total) *total = sh[NWARP];
    return sh[w] + x - v;
}

__device__ __forceinline__ int qmax_of(int codec) {
    return (codec == MC_DC_INT4 || codec == MC_DC_INT4_RAW) ? 7 : 127;
}

// Residual code rint(r / scale) clamped to [-qm, qm], with the IEEE quotient
// (ref falcom_cuda_v4_kernels.cu:53-65) but without a division per element:
// y = r * inv, inv = 1/scale rounded to nearest, is within 2^-22 |r / scale|
// (plus 2^-149 below the normal range) of the quotient, so within 2^-15 of it
// wherever |r / scale| < 128, the only range where the code is not clamped.
// There rint(y) equals rint(r / scale) unless y lies within 2^-15 of a
// half-integer; those elements (about 6 in 10^5), and every NaN / Inf case
// (inv = Inf for a subnormal scale), take the exact quotient.
// The product r * (1/scale) rounds like the quotient r / scale except,
// possibly, next to a half-integer: |y - rint(y)| (exact, at most 0.5) of at
// least 0.5 - 2^-15 -- or NaN, when 1/scale overflowed -- takes the exact
// quotient.
#define QUANT_NEAR_HALF 0.499969482421875f
__device__ __forceinline__ int quant1(float r, float scale, float inv, float qm) {
    const float y = __fmul_rn(r, inv);
    float v = rintf(y);
    if (!(fabsf(__fsub_rn(y, v)) < QUANT_NEAR_HALF)) v = rintf(__fdiv_rn(r, scale));
    v = fminf(qm, fmaxf(-qm, v));
    return (int)v;
}

struct TileRange {
    int64_t k0, k1, e0, e1;
};
__device__ __forceinline__ TileRange mom_range(const mc_enc_item &I, int t) {
    TileRange r;
    r.k0 = (int64_t)t * I.tile_kernels;
    r.k1 = min(r.k0 + (int64_t)I.tile_kernels, I.K);
    r.e0 = r.k0 * I.ks;
    r.e1 = r.k1 * I.ks;
    return r;
}

// Residual of one element of a momentum layer from its updated memory, in the
// reference's operation order (ref :2122-2158).
struct MomParams {
    float cm, cs, gmin, gmax;
    bool use_cs;
};
__device__ __forceinline__ float mom_pred_abs(float nm, const MomParams &p) {
    return fabsf(p.use_cs ? __fmaf_rn(nm, p.cs, p.cm) : __fadd_rn(nm, p.cm));
}
__device__ __forceinline__ float mom_residual(float c, float nm, bool pos, const MomParams &p) {
    const float ap = mom_pred_abs(nm, p);
    const float pred = pos ? ap : -ap;
    const float r = __fsub_rn(c, pred);
    return x86min(x86max(r, p.gmin), p.gmax);
}

// ---- quads: 4 consecutive elements, vector access when aligned and whole
__device__ __forceinline__ void ld4(const float *p, int64_t g, int64_t e1, bool vec, float (&o)[4]) {
    if (vec && g + 4 <= e1) {
        const float4 t = *(const float4 *)(p + g);
        o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) o[j] = (g + j < e1) ? p[g + j] : 0.0f;
    }
}
__device__ __forceinline__ void st4(float *p, int64_t g, int64_t e1, bool vec, const float (&v)[4]) {
    if (vec && g + 4 <= e1) {
        *(float4 *)(p + g) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (g + j < e1) p[g + j] = v[j];
    }
}

// Kernel index of element g (first of a quad) and the predicted / dominant
// bits of the quad's 4 elements from bitmap and sign words.
struct QuadBits {
    uint32_t f, pos;   // bit j: element j predicted / dominant sign positive
};
__device__ __forceinline__ QuadBits quad_bits(const uint32_t *bm, const uint32_t *dom, uint32_t wbase,
                                              uint32_t k0, int64_t g, int64_t e0, int64_t e1, int ks,
                                              mc_fastdiv ksdiv) {
    const uint32_t off = (uint32_t)(g - e0);
    const uint32_t q = fdiv32(off, ksdiv);
    uint32_t r = off - q * (uint32_t)ks;
    uint32_t k = k0 + q;
    QuadBits b = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (g + j < e1) {
            const uint32_t sh = k & 31, w = (k >> 5) - wbase;
            b.f |= ((bm[w] >> sh) & 1u) << j;
            if (dom) b.pos |= ((dom[w] >> sh) & 1u) << j;
        }
        if (++r == (uint32_t)ks) {
            r = 0;
            k++;
        }
    }
    return b;
}

// Predicted / dominant bits of the whole quad at tile offset o (the quad's
// elements all lie inside the tile); kernels of one element read the four
// bits straight from the words.
__device__ __forceinline__ QuadBits quad_bits_full(const uint32_t *bm, const uint32_t *dom, uint32_t wbase,
                                                   uint32_t k0, uint32_t o, int ks, mc_fastdiv ksdiv) {
    QuadBits b;
    if (ks == 1) {
        const uint32_t k = k0 + o, w = (k >> 5) - wbase, sh = k & 31;
        b.f = (bm[w] >> sh) & 0xFu;
        b.pos = dom ? (dom[w] >> sh) & 0xFu : 0u;
        return b;
    }
    const uint32_t q = fdiv32(o, ksdiv);
    uint32_t r = o - q * (uint32_t)ks;
    uint32_t k = k0 + q;
    if (ks >= 4) {
        // the quad's elements j < s belong to kernel k, the rest (if any) to
        // kernel k + 1: a quad spans at most two kernels of 4 or more elements
        const uint32_t s = (uint32_t)ks - r;
        const uint32_t lo = s >= 4u ? 0xFu : (1u << s) - 1u;
        const uint32_t k1 = k + (s < 4u ? 1u : 0u);
        const uint32_t wa = (k >> 5) - wbase, sa = k & 31, wb = (k1 >> 5) - wbase, sb = k1 & 31;
        b.f = (lo & (0u - ((bm[wa] >> sa) & 1u))) | (~lo & 0xFu & (0u - ((bm[wb] >> sb) & 1u)));
        b.pos = dom ? (lo & (0u - ((dom[wa] >> sa) & 1u))) | (~lo & 0xFu & (0u - ((dom[wb] >> sb) & 1u))) : 0u;
        return b;
    }
    b.f = b.pos = 0u;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t sh = k & 31, w = (k >> 5) - wbase;
        b.f |= ((bm[w] >> sh) & 1u) << j;
        if (dom) b.pos |= ((dom[w] >> sh) & 1u) << j;
        if (++r == (uint32_t)ks) {
            r = 0;
            k++;
        }
    }
    return b;
}

// Exclusive prefix of the per-tile predicted counts of one item, written to
// out[base .. base+nt); returns the total.  Whole block participates.
__device__ int64_t scan_tile_counts(const int32_t *cnt, int stride_words, int base, int nt,
                                    int64_t *out, int *sh) {
    int64_t carry = 0;
    for (int b0 = 0; b0 < nt; b0 += TPB) {
        const int i = b0 + threadIdx.x;
        const int v = i < nt ? __ldcg(cnt + (size_t)(base + i) * stride_words) : 0;
        int tot;
        const int ex = block_excl_scan(v, sh, &tot);
        if (i < nt) out[base + i] = carry + ex;
        carry += tot;
    }
    return carry;
}


// ------------------------------------------------------------ bulk staging
// A tile's float inputs are brought into shared memory by one thread with
// 1-D bulk async copies (cp.async.bulk, TMA engine, no multicast) completing
// on one mbarrier, so a CTA has its whole tile in flight at once without
// spending registers on it.  Copies need 16-byte aligned addresses and
// sizes: the aligned body of the tile is copied in bulk and the remaining
// (< 4) elements by plain loads.  Every wait on the mbarrier is bounded.
#define STAGE_ELEMS MC_TILE_ELEMS
#define MBAR_SPIN_LIMIT (1u << 24)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// L2 eviction priority of the staged arrays and the large outputs: streamed
// (evict_first).  A round's working set (inputs, previous gradients,
// memories, history copies) is several times the L2; lines kept at a higher
// priority for a later pass only crowd out the lines in use (measured on
// ResNet-50: keeping the inputs and previous gradients, or the inputs alone,
// made the round ~4% slower).  The passes alternate their tile order, so a
// pass still starts on the tiles the previous one touched last.
__device__ __forceinline__ uint64_t l2_stream() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                         uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
// 16-byte store with an L2 eviction priority.
__device__ __forceinline__ void st_f4(float4 *p, float4 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;"
                 ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "l"(pol) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}
// Bounded wait for phase `parity`, polled with a short sleep between tests
// (a polling warp takes issue slots from the other CTAs on the SM): at most
// MBAR_SPIN_LIMIT tests and about two seconds; false when either ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (uint32_t i = 0; i < MBAR_SPIN_LIMIT; i++) {
        __nanosleep(64);
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15) {
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > 2000000000ull) return false;
        }
    }
    return false;
}

// ------------------------------------------------------------ tile CTAs
// The streaming passes run one CTA per tile of the launch's tile list.  A
// tile only writes its outputs and its partials: the per-item reductions run
// in separate finalize kernels, so the passes have no fences or atomics.
#define NSTAGE_ARR 3
// Bitmap words of one tile: at most 4096 kernels (tiles hold at most
// STAGE_ELEMS elements of whole kernels, and start on a word boundary).
#define TILE_WORDS (STAGE_ELEMS / 32)
static_assert(TILE_WORDS <= TPB, "tile kernels handle one bitmap word per thread");

struct StageDesc {
    const float *src[NSTAGE_ARR];   // global source of every staged array (NULL: not staged)
    int64_t e0, e1;                 // element range of the tile
    // optional byte range [x0, x1) staged in the byte region behind the
    // arrays, the byte at address a at offset a - (x0 & ~15)
    const uint8_t *x0, *x1;
    int gt;                         // tile id
    int ii;                         // item index
    int late;                       // bit k: array k is the previous kernel's output, copied after
                                    // the dependent-launch wait (see run_tile)
};

struct TileShared {
    uint64_t bar;
    StageDesc d;
};

__device__ __forceinline__ uint32_t stage_body_bytes(const StageDesc &d) {
    return (uint32_t)(((d.e1 - d.e0) * 4) & ~(int64_t)15);
}
__device__ __forceinline__ uintptr_t up16(const void *p) { return ((uintptr_t)p + 15) & ~(uintptr_t)15; }
__device__ __forceinline__ uintptr_t dn16(const void *p) { return (uintptr_t)p & ~(uintptr_t)15; }

// Thread 0: start the bulk copies of a tile into a stage buffer of NA
// arrays (and the aligned interior of the byte range into the byte region
// xb); a tile with nothing staged still arrives so that the stage's phase
// completes.
template <int NA>
__device__ void pipe_issue(uint32_t bar, float *buf, uint8_t *xb, const StageDesc &d) {
    const uint32_t body = stage_body_bytes(d);
    uint32_t total = 0;
#pragma unroll
    for (int k = 0; k < NA; k++)
        if (d.src[k]) total += body;
    const uintptr_t xa = d.x0 ? up16(d.x0) : 0, xe = d.x0 ? dn16(d.x1) : 0;
    const uint32_t xbytes = xe > xa ? (uint32_t)(xe - xa) : 0u;
    mbar_expect_tx(bar, total + xbytes);
    const uint64_t stream = l2_stream();
    if (body) {
#pragma unroll
        for (int k = 0; k < NA; k++)
            if (d.src[k] && !((d.late >> k) & 1))
                bulk_g2s(smem_u32(buf + k * STAGE_ELEMS), d.src[k] + d.e0, body, bar,
                         stream);
    }
    if (xbytes) bulk_g2s(smem_u32(xb + (xa - dn16(d.x0))), (const void *)xa, xbytes, bar, stream);
}
// Thread 0, after the dependent-launch wait: the copies of the arrays in
// d.late (their bytes were announced with the others by pipe_issue, on the
// same mbarrier phase).
template <int NA>
__device__ void pipe_issue_late(uint32_t bar, float *buf, const StageDesc &d) {
    const uint32_t body = stage_body_bytes(d);
    if (!d.late || !body) return;
    const uint64_t stream = l2_stream();
#pragma unroll
    for (int k = 0; k < NA; k++)
        if (d.src[k] && ((d.late >> k) & 1))
            bulk_g2s(smem_u32(buf + k * STAGE_ELEMS), d.src[k] + d.e0, body, bar, stream);
}

// All threads, while the copies are in flight: what the bulk copies leave
// out -- the (< 4) trailing elements of the staged arrays and the unaligned
// head and tail (< 16 bytes each) of the byte range.
// (visible to the block after the barrier that follows the wait)
template <int NA>
__device__ void pipe_tail(float *buf, uint8_t *xb, const StageDesc &d) {
    const int64_t t0 = d.e0 + stage_body_bytes(d) / 4;
    if (t0 < d.e1) {
#pragma unroll
        for (int k = 0; k < NA; k++) {
            if (!d.src[k]) continue;
            for (int64_t e = t0 + threadIdx.x; e < d.e1; e += TPB) buf[k * STAGE_ELEMS + (e - d.e0)] = d.src[k][e];
        }
    }
    if (d.x0 && threadIdx.x < 32) {
        const int i = threadIdx.x & 15;
        const uintptr_t base = dn16(d.x0), xa = up16(d.x0), xe = dn16(d.x1);
        const uintptr_t a = threadIdx.x < 16 ? (uintptr_t)d.x0 + i : (xe > xa ? xe : xa) + i;
        const uintptr_t lim = threadIdx.x < 16 ? (xa < (uintptr_t)d.x1 ? xa : (uintptr_t)d.x1) : (uintptr_t)d.x1;
        if (a < lim) xb[a - base] = *(const uint8_t *)a;
    }
}

// Staged copy of array k of a tile as a pointer indexed by element number,
// or the global array when it is not staged.
__device__ __forceinline__ const float *staged_or(const StageDesc &d, const float *buf, int k, const float *g) {
    return d.src[k] ? buf + k * STAGE_ELEMS - d.e0 : g;
}

// One CTA per tile: list entry blockIdx.x (counted from the end when
// REVERSE: CTAs start roughly in index order, so a reversed pass first
// touches the tiles the previous pass touched last, still in L2) holds the
// tile id and its item index.  plan(StageDesc&) runs on thread 0 and fills
// the element range, the arrays to stage (src[k] for k < NA) and the byte
// range (x0 / x1, NULL for none; at most the byte region's size less 16);
// thread 0 then starts their bulk copies, all threads copy what the copies
// leave out and wait (bounded) on the mbarrier, and body(const StageDesc&,
// const float *buf) runs with the tile in shared memory (the byte region at
// buf + NA * STAGE_ELEMS); pre(const StageDesc&) runs on all threads between
// the issue and the wait.  A copy that does not complete within the spin
// limit sets the item's error flag and skips the tile.
// Under programmatic dependent launch the plan and the bulk copies run
// before the wait on the previous kernel of the stream, so they may read
// only what was complete before that kernel started: the inputs, the state
// of earlier calls, and the output of kernels two or more launches back
// (pass 4 stages the new memory of pass 3 with the finalize kernel of pass 3
// between them).  Arrays the plan marks in d.late are copied after the wait,
// so they may be the previous kernel's output (the server aggregate, which
// the previous decode on the stream may still be writing).
template <int NA, bool REVERSE, class Plan, class Pre, class Body>
__device__ void run_tile(const int2 *list, float *stage_mem, uint64_t *bar, StageDesc *sd, int32_t *err_of_item,
                         int err_stride_words, Plan plan, Pre pre, Body body) {
    const uint32_t b = smem_u32(bar);
    uint8_t *xb = (uint8_t *)(stage_mem + NA * STAGE_ELEMS);
    if (threadIdx.x == 0) {
        const int2 e = list[REVERSE ? gridDim.x - 1 - blockIdx.x : blockIdx.x];
        StageDesc d;
        d.gt = e.x;
        d.ii = e.y;
        d.x0 = d.x1 = nullptr;
        d.late = 0;
        plan(d);
        *sd = d;
        mbar_init(b, 1);
        pipe_issue<NA>(b, stage_mem, xb, d);
    }
    __syncthreads();
    pdl_wait();
    pdl_release();
    const StageDesc d = *sd;
    if (threadIdx.x == 0) pipe_issue_late<NA>(b, stage_mem, d);
    pipe_tail<NA>(stage_mem, xb, d);
    pre(d);   // the tile's own global reads, while its bulk copies are in flight
    // warp 0 waits for the copies; the other warps wait in the CTA barrier
    // (which issues nothing) and see the staged tile through it
    bool ok = true;
    if (threadIdx.x < 32) {
        ok = mbar_wait(b, 0);
        if (!ok) ok = mbar_wait(b, 0);   // one more bounded wait for the copies in flight
    }
    if (!__syncthreads_and(ok)) {
        if (threadIdx.x == 0) err_of_item[(size_t)d.ii * err_stride_words] = 2;
        return;
    }
    body(d, (const float *)stage_mem);
}

#define STAGE_BYTES(na) ((size_t)(na) * STAGE_ELEMS * sizeof(float))

// ------------------------------------------------------------------ frames
// zstd frames are written in place by the passes: header (magic, descriptor
// 0xA0 = single segment + 4-byte content size), then blocks of at most 2^17
// content bytes behind 3-byte headers (bit 0 last, bits 1-2 type: 0 Raw,
// 1 RLE, bits 3.. size).  Content byte b of an all-Raw frame sits at
// frame + MC_ZHDR + 3 + b + 3 * (b >> 17).
#define MAX_RLE_BLOCKS 64

__device__ __forceinline__ int64_t fpos_raw(int64_t b) {
    return MC_ZHDR + 3 + b + 3 * (b >> MC_ZBLOCK_LOG2);
}
__device__ __forceinline__ int64_t fpos_rle(int64_t b) { return MC_ZHDR + 3 + 4 * (b >> MC_ZBLOCK_LOG2); }
__device__ __forceinline__ int64_t nblocks_of(int64_t c) {
    return c == 0 ? 1 : (c + MC_ZBLOCK - 1) >> MC_ZBLOCK_LOG2;
}

__device__ __forceinline__ void put_frame_header(uint8_t *f, int64_t content) {
    f[0] = 0x28; f[1] = 0xB5; f[2] = 0x2F; f[3] = 0xFD;
    f[4] = 0xA0;
    for (int i = 0; i < 4; i++) f[5 + i] = (uint8_t)((uint64_t)content >> (8 * i));
}
__device__ __forceinline__ void put_block_header(uint8_t *p, bool last, int type, int64_t size) {
    const uint32_t h = (last ? 1u : 0u) | ((uint32_t)type << 1) | ((uint32_t)size << 3);
    p[0] = (uint8_t)h;
    p[1] = (uint8_t)(h >> 8);
    p[2] = (uint8_t)(h >> 16);
}

// Headers of the bitmap frame (one block per 2^20 kernels; a block whose
// kernels are all predicted or all not predicted becomes an RLE block of
// 0xFF / 0x00, decided from the per-tile predicted counts) and of the
// dominant-sign frame (Raw blocks; none when no kernel is predicted).
// Whole block participates; runs in the last CTA of pass 1.
__device__ void write_frame_headers(const mc_enc_item &I, const mc_enc_launch &L, mc_enc_result *R, int64_t P,
                                    int *s_blk) {
    const int64_t c = (I.K + 7) >> 3;
    const int64_t nb = nblocks_of(c);
    const bool plan_rle = nb <= MAX_RLE_BLOCKS;
    if (plan_rle) {
        for (int j = threadIdx.x; j < MAX_RLE_BLOCKS; j += TPB) s_blk[j] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
            const int64_t k0 = (int64_t)i * I.tile_kernels;
            atomicAdd(&s_blk[k0 >> (MC_ZBLOCK_LOG2 + 3)], __ldcg(&L.tiles[I.tile_base + i].P));
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        uint8_t *f = I.bm_frame;
        put_frame_header(f, c);
        int64_t pos = MC_ZHDR;
        for (int64_t j = 0; j < nb; j++) {
            const int64_t b0 = j << MC_ZBLOCK_LOG2;
            const int64_t bytes = c == 0 ? 0 : min((int64_t)MC_ZBLOCK, c - b0);
            const int64_t kern = min(I.K, (b0 + bytes) * 8) - b0 * 8;
            int rle = -1;
            if (plan_rle && bytes > 1) {
                const int pj = s_blk[j];
                if (pj == kern && (kern & 7) == 0) rle = 0xFF;
                else if (pj == 0) rle = 0;
            }
            put_block_header(f + pos, j == nb - 1, rle >= 0 ? 1 : 0, bytes);
            if (rle >= 0) {
                f[pos + 3] = (uint8_t)rle;
                if (j < I.max_blocks) I.blk_pos[j] = 0xFFFFFFFFu;
                pos += 4;
            } else {
                if (j < I.max_blocks) I.blk_pos[j] = (uint32_t)(pos + 3);
                pos += 3 + bytes;
            }
        }
        R->bm_size = pos;
        if (P == 0) {
            R->sg_size = 0;
        } else {
            const int64_t s = (P + 7) >> 3;
            const int64_t ns = nblocks_of(s);
            uint8_t *g = I.sg_frame;
            put_frame_header(g, s);
            for (int64_t j = 0; j < ns; j++) {
                const int64_t bytes = min((int64_t)MC_ZBLOCK, s - (j << MC_ZBLOCK_LOG2));
                put_block_header(g + MC_ZHDR + j * (MC_ZBLOCK + 3), j == ns - 1, 0, bytes);
            }
            R->sg_size = MC_ZHDR + 3 * ns + s;
        }
    }
}

// ------------------------------------------------------------------ pass 1
__device__ void pass1_tile(const mc_enc_launch &L, const StageDesc &d, const float *buf, Red &red) {
    const int ii = d.ii;
    const mc_enc_item I = L.items[ii];
    const int t = d.gt - I.tile_base;
    double dd[4] = {0.0, 0.0, 0.0, 0.0};
    long long l[2] = {0, 0};
    float mn = FLT_MAX, mx = -FLT_MAX, mx2 = 0.0f;

    if (I.kind == MC_K_MOMENTUM) {
        const TileRange tr = mom_range(I, t);
        const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
        const float *prev = staged_or(d, buf, 1, I.prev);
        float *hist = (float *)I.hist_out;
        if (I.vec) {
            // whole quads without range checks (tile-relative 32-bit offsets);
            // the ragged end goes to the thread that owns that quad
            const int len = (int)(tr.e1 - tr.e0), nq = len >> 2;
            const float4 *c4 = (const float4 *)(cur + tr.e0), *p4 = (const float4 *)(prev + tr.e0);
            float4 *h4 = hist ? (float4 *)(hist + tr.e0) : nullptr;
            const uint64_t hpol = l2_stream();   // the history copy is read next round
            // WP: the |prev| sum is computed here (its statistics are not known)
            auto quads = [&](auto wp) {
                constexpr bool WP = decltype(wp)::value;
                for (int q = threadIdx.x; q < nq; q += TPB) {
                    const float4 c = c4[q];
                    dd[0] += (double)fabsf(c.x);
                    dd[0] += (double)fabsf(c.y);
                    dd[0] += (double)fabsf(c.z);
                    dd[0] += (double)fabsf(c.w);
                    if (WP) {
                        const float4 p = p4[q];
                        dd[1] += (double)fabsf(p.x);
                        dd[1] += (double)fabsf(p.y);
                        dd[1] += (double)fabsf(p.z);
                        dd[1] += (double)fabsf(p.w);
                    }
                    mn = c.x < mn ? c.x : mn;
                    mx = c.x > mx ? c.x : mx;
                    mn = c.y < mn ? c.y : mn;
                    mx = c.y > mx ? c.y : mx;
                    mn = c.z < mn ? c.z : mn;
                    mx = c.z > mx ? c.z : mx;
                    mn = c.w < mn ? c.w : mn;
                    mx = c.w > mx ? c.w : mx;
                    if (h4) st_f4(h4 + q, c, hpol);
                }
            };
            if (I.prev_known) quads(std::false_type());
            else quads(std::true_type());
            if ((len & 3) && threadIdx.x == (nq % TPB)) {
                for (int64_t g = tr.e0 + 4 * (int64_t)nq; g < tr.e1; g++) {
                    const float c = cur[g];
                    dd[0] += (double)fabsf(c);
                    if (!I.prev_known) dd[1] += (double)fabsf(prev[g]);
                    mn = c < mn ? c : mn;
                    mx = c > mx ? c : mx;
                    if (hist) hist[g] = c;
                }
            }
        } else {
            for (int64_t g = tr.e0 + 4 * (int64_t)threadIdx.x; g < tr.e1; g += 4 * TPB) {
                float c[4], p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                ld4(cur, g, tr.e1, false, c);
                if (!I.prev_known) ld4(prev, g, tr.e1, false, p);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (g + j < tr.e1) {
                        dd[0] += (double)fabsf(c[j]);
                        dd[1] += (double)fabsf(p[j]);
                        mn = c[j] < mn ? c[j] : mn;
                        mx = c[j] > mx ? c[j] : mx;
                    }
                }
                if (hist) st4(hist, g, tr.e1, false, c);
            }
        }
        {   // this tile's share of zeroing the sign frame slot (pass 4 ORs bits into it)
            const int64_t nq = I.sg_cap >> 4;
            const int64_t per = (nq + I.ntiles - 1) / I.ntiles;
            const int64_t q1 = min(nq, (int64_t)(t + 1) * per);
            for (int64_t q = (int64_t)t * per + threadIdx.x; q < q1; q += TPB)
                ((uint4 *)I.sg_frame)[q] = make_uint4(0u, 0u, 0u, 0u);
        }
        // per-kernel sign consistency: one lane per kernel, 32 kernels per
        // ballot word (reads the staged tile when there is one)
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const float inv_ks = __fdiv_rn(1.0f, (float)I.ks);
        int P = 0;
        if (I.ks == 1 && d.src[0]) {
            // one element per kernel: maj = 1, so every kernel has the same
            // consistency ((1 * 1 - 0.5) * 2) and the dominant sign is "not
            // negative".  A lane takes 4 kernels (one 16-byte load of the
            // staged tile; a quad past the tile's end stays inside the
            // 4096-float stage and its bits are masked off), and each group
            // of 8 lanes ORs its nibbles into one 32-kernel word.
            const float half = __fmaf_rn(1.0f, inv_ks, -0.5f);
            const bool flag = __fadd_rn(half, half) >= I.thr;
            const uint32_t kt = (uint32_t)(tr.k1 - tr.k0);
            const float4 *c4 = (const float4 *)(cur + tr.k0);
            for (uint32_t kb = warp * 128u; kb < kt; kb += NWARP * 128u) {
                const uint32_t k = kb + 4u * lane;
                const float4 v = c4[k >> 2];
                const uint32_t nv = k >= kt ? 0u : (kt - k >= 4u ? 4u : kt - k);
                const uint32_t vm = (1u << nv) - 1u;
                const uint32_t nib = ((v.x < 0.0f ? 0u : 1u) | (v.y < 0.0f ? 0u : 2u) | (v.z < 0.0f ? 0u : 4u) |
                                      (v.w < 0.0f ? 0u : 8u)) & vm;
                const uint32_t sh = 4u * (lane & 7);
                uint32_t dw = nib << sh, bw = (flag ? vm : 0u) << sh;
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    dw |= __shfl_xor_sync(FULL, dw, o);
                    bw |= __shfl_xor_sync(FULL, bw, o);
                }
                const uint32_t kw = kb + 32u * (lane >> 3);
                if ((lane & 7) == 0 && kw < kt) {
                    I.bm_words[(tr.k0 + kw) >> 5] = bw;
                    I.dom_words[(tr.k0 + kw) >> 5] = dw;
                    P += __popc(bw);
                }
            }
        } else if (I.ks == 1) {
            const float half = __fmaf_rn(1.0f, inv_ks, -0.5f);
            const bool flag = __fadd_rn(half, half) >= I.thr;
            for (int64_t kb = tr.k0 + warp * 32; kb < tr.k1; kb += TPB) {
                const int64_t k = kb + lane;
                const bool in = k < tr.k1;
                const uint32_t b = __ballot_sync(FULL, in && flag);
                const uint32_t dw = __ballot_sync(FULL, in && !(cur[in ? k : kb] < 0.0f));
                if (lane == 0) {
                    I.bm_words[kb >> 5] = b;
                    I.dom_words[kb >> 5] = dw;
                    P += __popc(b);
                }
            }
        } else {
            // kernels of KS elements (KS = 0: the item's ks at run time)
            auto kernels = [&](auto ks_c) {
                constexpr int KS = decltype(ks_c)::value;
                const int ks = KS ? KS : I.ks;
                for (int64_t kb = tr.k0 + warp * 32; kb < tr.k1; kb += TPB) {
                    const int64_t k = kb + lane;
                    bool flag = false, dom = false;
                    if (k < tr.k1) {
                        const float *pk = cur + k * ks;
                        int pos = 0, neg = 0;
                        if (KS) {
#pragma unroll
                            for (int j = 0; j < KS; j++) {
                                const float v = pk[j];
                                pos += v > 0.0f;
                                neg += v < 0.0f;
                            }
                        } else {
                            for (int j = 0; j < ks; j++) {
                                const float v = pk[j];
                                pos += v > 0.0f;
                                neg += v < 0.0f;
                            }
                        }
                        const int zero = ks - pos - neg;
                        const int maj = (pos >= neg) ? (pos + zero) : (neg + zero);
                        const float half = __fmaf_rn((float)maj, inv_ks, -0.5f);
                        const float cons = __fadd_rn(half, half);
                        flag = cons >= I.thr;
                        dom = pos >= neg;
                    }
                    const uint32_t b = __ballot_sync(FULL, flag);
                    const uint32_t dw = __ballot_sync(FULL, dom);
                    if (lane == 0) {
                        I.bm_words[kb >> 5] = b;
                        I.dom_words[kb >> 5] = dw;
                        P += __popc(b);
                    }
                }
            };
            if (I.ks == 9) kernels(std::integral_constant<int, 9>());
            else kernels(std::integral_constant<int, 0>());
        }
        l[0] = P;
        block_reduce<2, RF_MN | RF_MX, 1>(red, dd, mn, mx, mx2, l);
        if (threadIdx.x == 0) {
            mc_enc_tile &T = L.tiles[d.gt];
            T.s_cur = dd[0];
            T.s_prev = dd[1];
            T.mn = mn;
            T.mx = mx;
            T.P = (int32_t)l[0];
        }
        return;
    }

    // direct items: element tiles (byte tiles for COPY / FRAME)
    const int64_t e0 = (int64_t)t * I.tile_kernels;
    const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
    if (I.kind == MC_K_FRAME) {
        // lossless payload: history copy plus an all-Raw zstd frame of the
        // input bytes (tiles of at most 2^15 bytes never straddle a 2^17-byte block)
        const uint8_t *src = (const uint8_t *)I.cur;
        uint8_t *hist = (uint8_t *)I.hist_out;
        uint8_t *fr = I.data_out;
        if (t == 0 && threadIdx.x == 0) {
            const int64_t nb = nblocks_of(I.n);
            put_frame_header(fr, I.n);
            for (int64_t j = 0; j < nb; j++)
                put_block_header(fr + MC_ZHDR + j * (MC_ZBLOCK + 3), j == nb - 1, 0,
                                 I.n == 0 ? 0 : min((int64_t)MC_ZBLOCK, I.n - (j << MC_ZBLOCK_LOG2)));
        }
        uint8_t *dst = fr + fpos_raw(e0) - e0;   // frame position of byte e of this tile: dst + e
        if (((((uintptr_t)src | (uintptr_t)hist) & 3) == 0) && (((uintptr_t)(dst + e0)) & 3) == 0) {
            for (int64_t w = (e0 >> 2) + threadIdx.x; w < (e1 >> 2); w += TPB) {
                const uint32_t x = ((const uint32_t *)src)[w];
                if (hist) ((uint32_t *)hist)[w] = x;
                *(uint32_t *)(dst + 4 * w) = x;
            }
            for (int64_t e = (e1 & ~(int64_t)3) + threadIdx.x; e < e1; e += TPB) {
                const uint8_t x = src[e];
                if (hist) hist[e] = x;
                dst[e] = x;
            }
        } else {
            for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
                const uint8_t x = src[e];
                if (hist) hist[e] = x;
                dst[e] = x;
            }
        }
        return;
    }
    if (I.kind == MC_K_COPY) {
        // raw payload ("sz3_memcpy") and history copy of the input bytes
        const uint8_t *src = (const uint8_t *)I.cur;
        uint8_t *hist = (uint8_t *)I.hist_out;
        uint8_t *raw = I.data_out;
        if (I.vec) {   // 16-byte aligned base pointers; tiles are multiples of 16 bytes
            const int64_t v0 = e0 >> 4, v1 = e1 >> 4;
            for (int64_t v = v0 + threadIdx.x; v < v1; v += TPB) {
                const uint4 x = ((const uint4 *)src)[v];
                if (raw) ((uint4 *)raw)[v] = x;
                if (hist) ((uint4 *)hist)[v] = x;
            }
            for (int64_t e = (v1 << 4) + threadIdx.x; e < e1; e += TPB) {
                const uint8_t x = src[e];
                if (raw) raw[e] = x;
                if (hist) hist[e] = x;
            }
        } else {
            for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
                const uint8_t x = src[e];
                if (raw) raw[e] = x;
                if (hist) hist[e] = x;
            }
        }
        return;
    }
    // MC_K_QUANT: max |x| for the scale, history copy
    const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
    float *hist = (float *)I.hist_out;
    for (int64_t g = e0 + 4 * (int64_t)threadIdx.x; g < e1; g += 4 * TPB) {
        float c[4];
        ld4(cur, g, e1, I.vec, c);
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (g + j < e1) mx2 = fmaxf(mx2, fabsf(c[j]));
        if (hist) st4(hist, g, e1, I.vec, c);
    }
    block_reduce<0, RF_MX2, 0>(red, dd, mn, mx, mx2, l);
    if (threadIdx.x == 0) L.tiles[d.gt].maxr = mx2;
}

// Thread 0: tile range of an encoder tile (nothing staged yet).
__device__ __forceinline__ const mc_enc_item &enc_plan_range(const mc_enc_launch &L, StageDesc &d) {
    const mc_enc_item &I = L.items[d.ii];
    const int t = d.gt - I.tile_base;
    if (I.kind == MC_K_MOMENTUM) {
        const TileRange tr = mom_range(I, t);
        d.e0 = tr.e0;
        d.e1 = tr.e1;
    } else {
        d.e0 = (int64_t)t * I.tile_kernels;
        d.e1 = min(d.e0 + (int64_t)I.tile_kernels, I.n);
    }
    d.src[0] = d.src[1] = d.src[2] = nullptr;
    return I;
}
__device__ __forceinline__ bool stageable(int staged, const mc_enc_item &I, const StageDesc &d) {
    // a direct quantised tile stages its input alone, across both arrays of
    // the two-array stages of passes 1 and 4
    const int64_t cap = I.kind == MC_K_QUANT ? 2 * STAGE_ELEMS : STAGE_ELEMS;
    return staged && I.vec && d.e1 - d.e0 <= cap;
}
#define ENC_ERR(L) &(L).results[0].err, (int)(sizeof(mc_enc_result) / 4)

__global__ void __launch_bounds__(TPB, 5) k_enc_pass1(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ TileShared ts;
    extern __shared__ __align__(128) float s_stage[];
    run_tile<2, false>((const int2 *)L.all_tiles, s_stage, &ts.bar, &ts.d, ENC_ERR(L),
                [&](StageDesc &d) {
                    const mc_enc_item &I = enc_plan_range(L, d);
                    if ((I.kind == MC_K_MOMENTUM || I.kind == MC_K_QUANT) && stageable(L.staged, I, d)) {
                        d.src[0] = (const float *)I.cur;
                        if (I.kind == MC_K_MOMENTUM && !I.prev_known) d.src[1] = I.prev;
                    }
                },
                [](const StageDesc &) {},
                [&](const StageDesc &d, const float *buf) { pass1_tile(L, d, buf, red); });
}

// The bitmap and dominant-sign words of a momentum tile, copied to shared
// memory (word wb = k0 / 32 of the layer at index 0).  Called between the
// issue of a tile's bulk copies and the wait; read after the wait.
__device__ __forceinline__ void stage_words(const mc_enc_item &I, int t, uint32_t *s_bw, uint32_t *s_dw) {
    const int64_t k0 = (int64_t)t * I.tile_kernels;
    const int64_t k1 = min(k0 + (int64_t)I.tile_kernels, I.K);
    const int64_t wb = k0 >> 5, we = (k1 + 31) >> 5;
    if (wb + threadIdx.x < we && threadIdx.x < TILE_WORDS) {
        s_bw[threadIdx.x] = I.bm_words[wb + threadIdx.x];
        s_dw[threadIdx.x] = I.dom_words[wb + threadIdx.x];
    }
}

// Per-item results of pass 1 (one CTA per item of the launch, items item0 ..): means and raw
// min / max of a momentum layer, the exclusive scan of its per-tile predicted
// counts, the bitmap / sign frame headers; the scale of a direct quantised
// tensor.  Reductions run over the tiles in order (deterministic).
__global__ void __launch_bounds__(TPB) k_enc_final1(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ int scan_sh[NWARP + 1];
    __shared__ int s_blk[MAX_RLE_BLOCKS + 1];
    pdl_wait();
    pdl_release();
    const int ii = L.item0 + blockIdx.x;
    const mc_enc_item I = L.items[ii];
    if (I.wave != L.wave) return;
    mc_enc_result *R = L.results + ii;
    double a[4] = {0.0, 0.0, 0.0, 0.0};
    long long z[2] = {0, 0};
    if (I.kind == MC_K_MOMENTUM) {
        float tmn = FLT_MAX, tmx = -FLT_MAX, t2 = 0.0f;
        for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
            const mc_enc_tile *T = L.tiles + I.tile_base + i;
            a[0] += T->s_cur;
            a[1] += T->s_prev;
            tmn = T->mn < tmn ? T->mn : tmn;
            tmx = T->mx > tmx ? T->mx : tmx;
        }
        block_reduce<2, RF_MN | RF_MX, 0>(red, a, tmn, tmx, t2, z);
        const int64_t total = scan_tile_counts(&L.tiles[0].P, (int)(sizeof(mc_enc_tile) / 4), I.tile_base,
                                               I.ntiles, L.tile_poff, scan_sh);
        write_frame_headers(I, L, R, total, s_blk);
        if (threadIdx.x == 0) {
            const double dn = (double)I.n;
            R->cm = __double2float_rn(__ddiv_rn(a[0], dn));
            R->pm = I.prev_known ? I.pm_known : __double2float_rn(__ddiv_rn(a[1], dn));
            R->gmin = tmn;
            R->gmax = tmx;
            R->P = total;
        }
    } else if (I.kind == MC_K_QUANT) {
        float m = 0.0f, u0 = FLT_MAX, u1 = -FLT_MAX;
        for (int i = threadIdx.x; i < I.ntiles; i += TPB) m = fmaxf(m, L.tiles[I.tile_base + i].maxr);
        block_reduce<0, RF_MX2, 0>(red, a, u0, u1, m, z);
        if (threadIdx.x == 0) {
            R->maxr = m;
            R->scale = (m == 0.0f) ? 1.0f : __fdiv_rn(m, (float)qmax_of(I.codec));
            if (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) *(float *)I.data_out = R->scale;
        }
    }
}

// ------------------------------------------------------------------ pass 2
__global__ void __launch_bounds__(TPB, 6) k_enc_pass2(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ TileShared ts;
    __shared__ float s_par[2];
    extern __shared__ __align__(128) float s_stage[];
    run_tile<2, true>((const int2 *)L.mom_tiles, s_stage, &ts.bar, &ts.d, ENC_ERR(L),
                    [&](StageDesc &d) {
                        const mc_enc_item &I = enc_plan_range(L, d);
                        if (stageable(L.staged, I, d)) {
                            d.src[0] = (const float *)I.cur;
                            if (!I.prev_known) d.src[1] = I.prev;
                        }
                    },
                    [&](const StageDesc &d) {
                        // the item's means (final1), read while the copies are in flight
                        if (threadIdx.x == 0) {
                            const mc_enc_result *R = L.results + d.ii;
                            s_par[0] = R->cm;
                            s_par[1] = R->pm;
                        }
                    },
                    [&](const StageDesc &d, const float *buf) {
                        const mc_enc_item I = L.items[d.ii];
                        const float cm = s_par[0], pm = s_par[1];
                        const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
                        const float *prev = staged_or(d, buf, 1, I.prev);
                        double dd[4] = {0.0, 0.0, 0.0, 0.0};
                        long long l[2] = {0, 0};
                        float mn = FLT_MAX, mx = -FLT_MAX, mx2 = 0.0f;
                        // with the previous gradient's statistics known only |cur| is summed
                        const bool wp = !I.prev_known;
                        auto accc = [&](float c) {
                            const double dc = (double)__fsub_rn(fabsf(c), cm);
                            dd[0] = __fma_rn(dc, dc, dd[0]);
                        };
                        auto accp = [&](float p) {
                            const double dp = (double)__fsub_rn(fabsf(p), pm);
                            dd[1] = __fma_rn(dp, dp, dd[1]);
                        };
                        const int len = (int)(d.e1 - d.e0), nq = len >> 2;
                        if (I.vec) {
                            const float4 *c4 = (const float4 *)(cur + d.e0), *p4 = (const float4 *)(prev + d.e0);
                            auto quads = [&](auto wpc) {
                                constexpr bool WP = decltype(wpc)::value;
                                for (int q = threadIdx.x; q < nq; q += TPB) {
                                    const float4 c = c4[q];
                                    accc(c.x);
                                    accc(c.y);
                                    accc(c.z);
                                    accc(c.w);
                                    if (WP) {
                                        const float4 p = p4[q];
                                        accp(p.x);
                                        accp(p.y);
                                        accp(p.z);
                                        accp(p.w);
                                    }
                                }
                            };
                            if (wp) quads(std::true_type());
                            else quads(std::false_type());
                            if ((len & 3) && threadIdx.x == (nq % TPB))
                                for (int64_t g = d.e0 + 4 * (int64_t)nq; g < d.e1; g++) {
                                    accc(cur[g]);
                                    if (wp) accp(prev[g]);
                                }
                        } else {
                            for (int64_t g = d.e0 + threadIdx.x * 4; g < d.e1; g += 4 * TPB)
                                for (int64_t e = g; e < g + 4 && e < d.e1; e++) {
                                    accc(cur[e]);
                                    if (wp) accp(prev[e]);
                                }
                        }
                        block_reduce<2, 0, 0>(red, dd, mn, mx, mx2, l);
                        if (threadIdx.x == 0) {
                            L.tiles[d.gt].v_cur = dd[0];
                            L.tiles[d.gt].v_prev = dd[1];
                        }
                    });
}

// Per-item results of pass 2: population std of |cur| and |prev|.
__global__ void __launch_bounds__(TPB) k_enc_final2(mc_enc_launch L) {
    __shared__ Red red;
    pdl_wait();
    pdl_release();
    const int ii = L.item0 + blockIdx.x;
    const mc_enc_item I = L.items[ii];
    if (I.wave != L.wave || I.kind != MC_K_MOMENTUM) return;
    mc_enc_result *R = L.results + ii;
    double a[4] = {0.0, 0.0, 0.0, 0.0};
    long long l[2] = {0, 0};
    float mn = FLT_MAX, mx = -FLT_MAX, mx2 = 0.0f;
    for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
        a[0] += L.tiles[I.tile_base + i].v_cur;
        a[1] += L.tiles[I.tile_base + i].v_prev;
    }
    block_reduce<2, 0, 0>(red, a, mn, mx, mx2, l);
    if (threadIdx.x == 0) {
        const double dn = (double)I.n;
        const float cs = __fsqrt_rn(__double2float_rn(__ddiv_rn(a[0], dn)));
        const float ps = I.prev_known ? I.ps_known : __fsqrt_rn(__double2float_rn(__ddiv_rn(a[1], dn)));
        R->cs = cs;
        R->ps = ps;
        R->inv_ps = (ps > 1e-8f) ? __fdiv_rn(1.0f, ps) : 1.0f;
    }
}

// ------------------------------------------------------------------ pass 3
// The previous gradient is read only for predicted kernels: it is staged
// when most kernels of the layer are predicted, else read directly.
__global__ void __launch_bounds__(TPB, 4) k_enc_pass3(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ TileShared ts;
    __shared__ uint32_t s_bw[TILE_WORDS], s_dw[TILE_WORDS];
    extern __shared__ __align__(128) float s_stage[];
    run_tile<3, false>((const int2 *)L.mom_tiles, s_stage, &ts.bar, &ts.d, ENC_ERR(L),
                    [&](StageDesc &d) {
                        const mc_enc_item &I = enc_plan_range(L, d);
                        if (stageable(L.staged, I, d)) {
                            d.src[0] = (const float *)I.cur;
                            d.src[1] = I.mem_in;
                            if (L.tiles[d.gt].P > 0) d.src[2] = I.prev;
                        }
                    },
                    [&](const StageDesc &d) {
                        const mc_enc_item &I = L.items[d.ii];
                        stage_words(I, d.gt - I.tile_base, s_bw, s_dw);
                    },
                    [&](const StageDesc &d, const float *buf) {
                        const mc_enc_item I = L.items[d.ii];
                        const mc_enc_result *R = L.results + d.ii;
                        const TileRange tr = mom_range(I, d.gt - I.tile_base);
                        const float cm = R->cm, cs = R->cs, pm = R->pm, inv_ps = R->inv_ps;
                        const bool use_ps = R->ps > 1e-8f;
                        const MomParams mp = {cm, cs, R->gmin, R->gmax, cs > 1e-8f};
                        const float lr = I.lr;
                        const float oml = __fsub_rn(1.0f, lr);
                        const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
                        const float *mem_in = staged_or(d, buf, 1, I.mem_in);
                        const float *prev = staged_or(d, buf, 2, I.prev);
                        long long mism = 0;
                        float maxr = 0.0f;
                        const uint32_t k0 = (uint32_t)tr.k0;
                        // one element: memory update and clamped residual of a predicted element
                        auto elem = [&](float c, float m0, float p, bool pos, float &mo) -> float {
                            const float pv = __fsub_rn(fabsf(p), pm);
                            const float pn = use_ps ? __fmul_rn(pv, inv_ps) : pv;
                            const float nm = __fmaf_rn(oml, m0, __fmul_rn(lr, pn));
                            mo = nm;
                            const float ap = mom_pred_abs(nm, mp);
                            const float pred = pos ? ap : -ap;
                            mism += (pred > 0.0f) != (c > 0.0f);
                            return x86min(x86max(__fsub_rn(c, pred), mp.gmin), mp.gmax);
                        };
                        auto quad = [&](int64_t g, const QuadBits &qb, const float (&c)[4], const float (&m0)[4],
                                        const float (&p)[4], float (&mo)[4], int nvalid) {
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                float r = c[j];
                                mo[j] = m0[j];
                                if ((qb.f >> j) & 1u) r = elem(c[j], m0[j], p[j], (qb.pos >> j) & 1u, mo[j]);
                                if (j < nvalid) maxr = fmaxf(maxr, fabsf(r));
                            }
                        };
                        const int len = (int)(tr.e1 - tr.e0), nq = len >> 2;
                        if (I.vec) {
                            const float4 *c4 = (const float4 *)(cur + tr.e0);
                            const float4 *m4 = mem_in ? (const float4 *)(mem_in + tr.e0) : nullptr;
                            const float4 *p4 = (const float4 *)(prev + tr.e0);
                            float4 *o4 = (float4 *)(I.mem_out + tr.e0);
                            const uint64_t spol = l2_stream();
                            for (int q = threadIdx.x; q < nq; q += TPB) {
                                const QuadBits qb = quad_bits_full(s_bw, s_dw, k0 >> 5, k0, 4u * q, I.ks, I.ksdiv);
                                const float4 cv = c4[q];
                                const float4 mv = m4 ? m4[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                                float4 pv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                                if (qb.f) pv = p4[q];
                                const float c[4] = {cv.x, cv.y, cv.z, cv.w}, m0[4] = {mv.x, mv.y, mv.z, mv.w};
                                const float p[4] = {pv.x, pv.y, pv.z, pv.w};
                                float mo[4];
                                quad(tr.e0 + 4 * q, qb, c, m0, p, mo, 4);
                                st_f4(o4 + q, make_float4(mo[0], mo[1], mo[2], mo[3]), spol);
                            }
                        }
                        const int64_t gstart = I.vec ? tr.e0 + 4 * (int64_t)nq : tr.e0;
                        const int owner = I.vec ? nq % TPB : 0;
                        for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < tr.e1;
                             g += 4 * TPB) {
                            const QuadBits qb = quad_bits(s_bw, s_dw, k0 >> 5, k0, g, tr.e0, tr.e1, I.ks, I.ksdiv);
                            float c[4], m0[4], p[4], mo[4];
                            ld4(cur, g, tr.e1, I.vec, c);
                            if (mem_in) ld4(mem_in, g, tr.e1, I.vec, m0);
                            else m0[0] = m0[1] = m0[2] = m0[3] = 0.0f;
                            if (qb.f) ld4(prev, g, tr.e1, I.vec, p);
                            quad(g, qb, c, m0, p, mo, (int)min((int64_t)4, tr.e1 - g));
                            st4(I.mem_out, g, tr.e1, I.vec, mo);
                        }
                        double dd[4];
                        long long l[2] = {mism, 0};
                        float mn = FLT_MAX, mx = -FLT_MAX;
                        block_reduce<0, RF_MX2, 1>(red, dd, mn, mx, maxr, l);
                        if (threadIdx.x == 0) {
                            L.tiles[d.gt].maxr = maxr;
                            L.tiles[d.gt].mism = l[0];
                        }
                    });
}

// Per-item results of pass 3: max |residual| (the codec scale, written into
// the payload header) and sign mismatches.
__global__ void __launch_bounds__(TPB) k_enc_final3(mc_enc_launch L) {
    __shared__ Red red;
    pdl_wait();
    pdl_release();
    const int ii = L.item0 + blockIdx.x;
    const mc_enc_item I = L.items[ii];
    if (I.wave != L.wave || I.kind != MC_K_MOMENTUM) return;
    mc_enc_result *R = L.results + ii;
    double dd[4];
    float m = 0.0f, mn = FLT_MAX, mx = -FLT_MAX;
    long long z[2] = {0, 0};
    for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
        m = fmaxf(m, L.tiles[I.tile_base + i].maxr);
        z[0] += L.tiles[I.tile_base + i].mism;
    }
    block_reduce<0, RF_MX2, 1>(red, dd, mn, mx, m, z);
    if (threadIdx.x == 0) {
        R->maxr = m;
        R->mism = z[0];
        R->scale = (m == 0.0f) ? 1.0f : __fdiv_rn(m, (float)qmax_of(I.codec));
        if (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) *(float *)I.data_out = R->scale;
    }
}

// Parallel bit extract / deposit of the bits of v at the set bits of m, by
// the parallel-suffix method (Hacker's Delight, 2nd ed., 7-4 "compress" and
// 7-5 "expand"): five fixed steps, no data-dependent loop, so the lanes of a
// warp stay converged whatever their masks.
__device__ __forceinline__ uint32_t pext32(uint32_t v, uint32_t m) {
    uint32_t x = v & m, mk = ~m << 1;
#pragma unroll
    for (int i = 0; i < 5; i++) {
        uint32_t mp = mk ^ (mk << 1);
        mp ^= mp << 2;
        mp ^= mp << 4;
        mp ^= mp << 8;
        mp ^= mp << 16;
        const uint32_t mv = mp & m;
        m = (m ^ mv) | (mv >> (1 << i));
        const uint32_t t = x & mv;
        x = (x ^ t) | (t >> (1 << i));
        mk &= ~mp;
    }
    return x;
}
__device__ __forceinline__ uint32_t pdep32(uint32_t v, uint32_t m) {
    const uint32_t m0 = m;
    uint32_t mk = ~m << 1, mvs[5];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        uint32_t mp = mk ^ (mk << 1);
        mp ^= mp << 2;
        mp ^= mp << 4;
        mp ^= mp << 8;
        mp ^= mp << 16;
        mvs[i] = mp & m;
        m = (m ^ mvs[i]) | (mvs[i] >> (1 << i));
        mk &= ~mp;
    }
#pragma unroll
    for (int i = 4; i >= 0; i--) v = (v & ~mvs[i]) | ((v << (1 << i)) & mvs[i]);
    return v & m0;
}

// Writes the residual codes of one quad (4 consecutive elements at g).
__device__ __forceinline__ void put_codes(uint8_t *data_out, int codec, int64_t g, int64_t e1, bool vec,
                                          const float (&r)[4], float scale, float inv, float qm) {
    if (codec == MC_DC_RAW) {
        st4((float *)data_out, g, e1, vec, r);
    } else if (codec == MC_DC_Q8) {
        uint8_t *codes = data_out + 4;   // 4-byte aligned; g is a multiple of 4
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (g + j < e1) word |= ((uint32_t)(uint8_t)(int8_t)quant1(r[j], scale, inv, qm)) << (8 * j);
        if (g + 4 <= e1) *(uint32_t *)(codes + g) = word;
        else
            for (int j = 0; g + j < e1; j++) codes[g + j] = (uint8_t)(word >> (8 * j));
    } else if (codec == MC_DC_INT4) {
        uint8_t *packed = data_out + 4;  // byte g/2, 2-byte aligned
        uint32_t nib[4];
#pragma unroll
        for (int j = 0; j < 4; j++) nib[j] = (g + j < e1) ? (uint32_t)((quant1(r[j], scale, inv, qm) + 8) & 15) : 0u;
        const uint32_t b0 = nib[0] | (nib[1] << 4), b1 = nib[2] | (nib[3] << 4);
        if (g + 4 <= e1) *(uint16_t *)(packed + (g >> 1)) = (uint16_t)(b0 | (b1 << 8));
        else {
            packed[g >> 1] = (uint8_t)b0;
            if (g + 2 < e1) packed[(g >> 1) + 1] = (uint8_t)b1;
        }
    } else {   // Q8_RAW / INT4_RAW: dequantised floats
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = __fmul_rn((float)quant1(r[j], scale, inv, qm), scale);
        st4((float *)data_out, g, e1, vec, v);
    }
}

// Codes of one whole quad (4 consecutive elements at g, all inside the item;
// the item's pointers 16-byte aligned), for codec C.  The exact quotient is
// taken only when a lane of the warp has an element within 2^-15 of a
// half-integer (see quant1).
template <int C>
__device__ __forceinline__ void put_codes_full(uint8_t *data_out, int64_t g, const float (&r)[4], float scale,
                                               float inv, float qm) {
    if (C == MC_DC_RAW) {
        *(float4 *)((float *)data_out + g) = make_float4(r[0], r[1], r[2], r[3]);
        return;
    }
    float v[4];
    bool need = false;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float y = __fmul_rn(r[j], inv);
        v[j] = rintf(y);
        need |= !(fabsf(__fsub_rn(y, v[j])) < QUANT_NEAR_HALF);
    }
    if (__any_sync(__activemask(), need)) {   // the lanes still in the quad loop
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float y = __fmul_rn(r[j], inv);
            if (!(fabsf(__fsub_rn(y, v[j])) < QUANT_NEAR_HALF)) v[j] = rintf(__fdiv_rn(r[j], scale));
        }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) v[j] = fminf(qm, fmaxf(-qm, v[j]));
    if (C == MC_DC_Q8) {
        const uint32_t word = ((uint32_t)(uint8_t)(int8_t)(int)v[0]) | ((uint32_t)(uint8_t)(int8_t)(int)v[1] << 8) |
                              ((uint32_t)(uint8_t)(int8_t)(int)v[2] << 16) |
                              ((uint32_t)(uint8_t)(int8_t)(int)v[3] << 24);
        *(uint32_t *)(data_out + 4 + g) = word;
    } else if (C == MC_DC_INT4) {
        const uint32_t b0 = (uint32_t)(((int)v[0] + 8) & 15) | ((uint32_t)(((int)v[1] + 8) & 15) << 4);
        const uint32_t b1 = (uint32_t)(((int)v[2] + 8) & 15) | ((uint32_t)(((int)v[3] + 8) & 15) << 4);
        *(uint16_t *)(data_out + 4 + (g >> 1)) = (uint16_t)(b0 | (b1 << 8));
    } else {   // Q8_RAW / INT4_RAW: dequantised floats (through the integer code, so a code of -0.0 gives +0.0)
        *(float4 *)((float *)data_out + g) =
            make_float4(__fmul_rn((float)(int)v[0], scale), __fmul_rn((float)(int)v[1], scale),
                        __fmul_rn((float)(int)v[2], scale), __fmul_rn((float)(int)v[3], scale));
    }
}

// ------------------------------------------------------------------ pass 4
// Side inputs of a pass-4 tile, read while its bulk copies are in flight:
// the offset of its first predicted kernel in the dense signs and the
// position of its block in the bitmap frame.
struct P4Side {
    int64_t poff;
    uint32_t blkpos;
};

// The frames of a momentum tile in pass 4, from its bitmap and dominant-sign
// words alone (no staged input), so it runs while the tile's bulk copies are
// in flight: the tile's bitmap content into its block of the bitmap frame,
// and its dense dominant signs into the sign frame.
__device__ void pass4_frames(const mc_enc_launch &L, const StageDesc &d, int *scan_sh, uint32_t *s_sg,
                             const uint32_t *s_bw, const uint32_t *s_dw, const P4Side &S) {
    const mc_enc_item &I = L.items[d.ii];
    const int t = d.gt - I.tile_base;
    const TileRange tr = mom_range(I, t);
    // bitmap content of this tile into its block of the bitmap frame
    // (ref :2222-2253; RLE blocks were written whole by pass 1)
    {
        const int64_t c = (I.K + 7) >> 3;
        const int64_t cb0 = tr.k0 >> 3, cb1 = min((tr.k1 + 7) >> 3, c);
        const uint32_t pos = S.blkpos;
        if (pos != 0xFFFFFFFFu) {
            uint8_t *dst = I.bm_frame + pos - ((cb0 >> MC_ZBLOCK_LOG2) << MC_ZBLOCK_LOG2);  // + cb
            // content byte b is byte b & 3 of the staged word (b >> 2) - wb0
            const int64_t wb0 = tr.k0 >> 5;
            if ((((uintptr_t)(dst + cb0)) & 3) == 0) {
                for (int64_t w = (cb0 >> 2) + threadIdx.x; 4 * w < cb1; w += TPB) {
                    const uint32_t v = s_bw[w - wb0];
                    if (4 * w + 4 <= cb1) *(uint32_t *)(dst + 4 * w) = v;
                    else
                        for (int64_t b = 4 * w; b < cb1; b++) dst[b] = (uint8_t)(v >> (8 * (b & 3)));
                }
            } else {
                for (int64_t b = cb0 + threadIdx.x; b < cb1; b += TPB)
                    dst[b] = (uint8_t)(s_bw[(b >> 2) - wb0] >> (8 * (b & 3)));
            }
        }
    }
    // dense dominant signs of predicted kernels (ref :2258-2283): the
    // tile's bits are assembled in shared memory, then written into the
    // sign frame; the two edge bytes shared with neighbour tiles are ORed
    const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
    const int i = threadIdx.x;
    s_sg[i] = 0u;
    if (i < 2) s_sg[TPB + i] = 0u;
    uint32_t mw = 0, dv = 0;
    if (wb + i < we && i < TILE_WORDS) {
        mw = s_bw[i];
        dv = s_dw[i];
    }
    const int pc = __popc(mw);
    int tot;
    const int off_l = block_excl_scan(pc, scan_sh, &tot);   // also orders the zeroing above
    const int64_t poff = S.poff;
    if (pc) {
        const uint32_t bits = pext32(dv, mw);
        const int lb = (int)(poff & 7) + off_l;
        const int sh = lb & 31;
        atomicOr(&s_sg[lb >> 5], bits << sh);
        if (sh + pc > 32) atomicOr(&s_sg[(lb >> 5) + 1], bits >> (32 - sh));
    }
    __syncthreads();
    if (tot > 0) {
        const int64_t cb0 = poff >> 3;
        const int64_t nbytes = ((poff + tot - 1) >> 3) - cb0 + 1;
        for (int64_t j = threadIdx.x; j < nbytes; j += TPB) {
            const uint32_t v = (s_sg[j >> 2] >> (8 * (j & 3))) & 0xFFu;
            const int64_t fb = fpos_raw(cb0 + j);
            if (j == 0 || j == nbytes - 1) {
                if (v) atomicOr((uint32_t *)(I.sg_frame + (fb & ~(int64_t)3)), v << (8 * (fb & 3)));
            } else {
                I.sg_frame[fb] = (uint8_t)v;
            }
        }
    }
}

__device__ void pass4_tile(const mc_enc_launch &L, const StageDesc &d, const float *buf, const uint32_t *s_bw,
                           const uint32_t *s_dw) {
    const int gt = d.gt;
    const int ii = d.ii;
    const mc_enc_item I = L.items[ii];
    const int t = gt - I.tile_base;
    const mc_enc_result *R = L.results + ii;
    if (I.kind == MC_K_MOMENTUM) {
        const TileRange tr = mom_range(I, t);
        const MomParams mp = {R->cm, R->cs, R->gmin, R->gmax, R->cs > 1e-8f};
        const float scale = R->scale;
        const float inv = __fdiv_rn(1.0f, scale);
        const float qm = (float)qmax_of(I.codec);
        const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
        const float *mem = staged_or(d, buf, 1, I.mem_out);
        const uint32_t k0 = (uint32_t)tr.k0;
        const int len = (int)(tr.e1 - tr.e0), nq = len >> 2;
        if (I.vec) {   // whole quads, no range checks
            const float4 *c4 = (const float4 *)(cur + tr.e0), *m4 = (const float4 *)(mem + tr.e0);
            auto quads = [&](auto codec) {
                for (int q = threadIdx.x; q < nq; q += TPB) {
                    const QuadBits qb = quad_bits_full(s_bw, s_dw, k0 >> 5, k0, 4u * q, I.ks, I.ksdiv);
                    const float4 cv = c4[q];
                    float4 mv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (qb.f) mv = m4[q];
                    const float c[4] = {cv.x, cv.y, cv.z, cv.w}, m[4] = {mv.x, mv.y, mv.z, mv.w};
                    float r[4];
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        r[j] = ((qb.f >> j) & 1u) ? mom_residual(c[j], m[j], (qb.pos >> j) & 1u, mp) : c[j];
                    put_codes_full<decltype(codec)::value>(I.data_out, tr.e0 + 4 * q, r, scale, inv, qm);
                }
            };
            switch (I.codec) {
                case MC_DC_Q8: quads(std::integral_constant<int, MC_DC_Q8>()); break;
                case MC_DC_INT4: quads(std::integral_constant<int, MC_DC_INT4>()); break;
                case MC_DC_RAW: quads(std::integral_constant<int, MC_DC_RAW>()); break;
                case MC_DC_Q8_RAW: quads(std::integral_constant<int, MC_DC_Q8_RAW>()); break;
                default: quads(std::integral_constant<int, MC_DC_INT4_RAW>()); break;
            }
        }
        const int64_t gstart = I.vec ? tr.e0 + 4 * (int64_t)nq : tr.e0;
        const int owner = I.vec ? nq % TPB : 0;
        for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < tr.e1; g += 4 * TPB) {
            const QuadBits qb = quad_bits(s_bw, s_dw, k0 >> 5, k0, g, tr.e0, tr.e1, I.ks, I.ksdiv);
            float c[4], m[4], r[4];
            ld4(cur, g, tr.e1, I.vec, c);
            if (qb.f) ld4(mem, g, tr.e1, I.vec, m);
#pragma unroll
            for (int j = 0; j < 4; j++)
                r[j] = ((qb.f >> j) & 1u) ? mom_residual(c[j], m[j], (qb.pos >> j) & 1u, mp) : c[j];
            put_codes(I.data_out, I.codec, g, tr.e1, I.vec, r, scale, inv, qm);
        }
        return;
    }
    if (I.kind == MC_K_QUANT) {
        const int64_t e0 = (int64_t)t * I.tile_kernels;
        const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
        const float scale = R->scale;
        const float inv = __fdiv_rn(1.0f, scale);
        const float qm = (float)qmax_of(I.codec);
        const float *cur = staged_or(d, buf, 0, (const float *)I.cur);
        int64_t gstart = e0;
        int owner = 0;
        if (I.vec) {   // whole quads, no range checks, the codec a template argument
            const int nq = (int)((e1 - e0) >> 2);
            const float4 *c4 = (const float4 *)(cur + e0);
            auto quads = [&](auto codec) {
                for (int q = threadIdx.x; q < nq; q += TPB) {
                    const float4 cv = c4[q];
                    const float c[4] = {cv.x, cv.y, cv.z, cv.w};
                    put_codes_full<decltype(codec)::value>(I.data_out, e0 + 4 * q, c, scale, inv, qm);
                }
            };
            switch (I.codec) {
                case MC_DC_Q8: quads(std::integral_constant<int, MC_DC_Q8>()); break;
                case MC_DC_INT4: quads(std::integral_constant<int, MC_DC_INT4>()); break;
                case MC_DC_RAW: quads(std::integral_constant<int, MC_DC_RAW>()); break;
                case MC_DC_Q8_RAW: quads(std::integral_constant<int, MC_DC_Q8_RAW>()); break;
                default: quads(std::integral_constant<int, MC_DC_INT4_RAW>()); break;
            }
            gstart = e0 + 4 * (int64_t)nq;
            owner = nq % TPB;
        }
        // the ragged end (or every quad of an unaligned item)
        for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < e1; g += 4 * TPB) {
            float c[4];
            ld4(cur, g, e1, I.vec, c);
            put_codes(I.data_out, I.codec, g, e1, I.vec, c, scale, inv, qm);
        }
    }
}

__global__ void __launch_bounds__(TPB, 5) k_enc_pass4(mc_enc_launch L) {
    __shared__ int scan_sh[NWARP + 1];
    __shared__ uint32_t s_sg[TPB + 2];
    __shared__ uint32_t s_bw[TILE_WORDS], s_dw[TILE_WORDS];
    __shared__ P4Side side;
    __shared__ TileShared ts;
    extern __shared__ __align__(128) float s_stage[];
    run_tile<2, true>((const int2 *)L.all_tiles, s_stage, &ts.bar, &ts.d, ENC_ERR(L),
                    [&](StageDesc &d) {
                        const mc_enc_item &I = enc_plan_range(L, d);
                        if ((I.kind == MC_K_MOMENTUM || I.kind == MC_K_QUANT) && stageable(L.staged, I, d)) {
                            d.src[0] = (const float *)I.cur;
                            if (I.kind == MC_K_MOMENTUM && L.tiles[d.gt].P > 0) d.src[1] = I.mem_out;
                        }
                    },
                    [&](const StageDesc &d) {
                        const mc_enc_item &I = L.items[d.ii];
                        if (I.kind != MC_K_MOMENTUM) return;
                        const int t = d.gt - I.tile_base;
                        stage_words(I, t, s_bw, s_dw);
                        if (threadIdx.x == 0) {
                            side.poff = L.tile_poff[d.gt];
                            side.blkpos = I.blk_pos[((int64_t)t * I.tile_kernels) >> (MC_ZBLOCK_LOG2 + 3)];
                        }
                        __syncthreads();
                        pass4_frames(L, d, scan_sh, s_sg, s_bw, s_dw, side);
                    },
                    [&](const StageDesc &d, const float *buf) { pass4_tile(L, d, buf, s_bw, s_dw); });
}

// ------------------------------------------------------------------ frames
// Copies n bytes; 4-byte words when both ends are 4-byte aligned.
__device__ __forceinline__ void copy_bytes(uint8_t *dst, const uint8_t *src, int64_t n) {
    if ((((uintptr_t)dst | (uintptr_t)src) & 3) == 0) {
        const int64_t nw = n >> 2;
        for (int64_t i = threadIdx.x; i < nw; i += TPB) ((uint32_t *)dst)[i] = ((const uint32_t *)src)[i];
        for (int64_t i = (nw << 2) + threadIdx.x; i < n; i += TPB) dst[i] = src[i];
    } else {
        for (int64_t i = threadIdx.x; i < n; i += TPB) dst[i] = src[i];
    }
}

// ------------------------------------------------------------------ unframe
#define MAX_SEGS 64
__global__ void __launch_bounds__(TPB) k_unframe(const mc_unframe_job *jobs) {
    const mc_unframe_job &J = jobs[blockIdx.x];
    __shared__ int64_t s_src[MAX_SEGS], s_dst[MAX_SEGS], s_len[MAX_SEGS];
    __shared__ int s_type[MAX_SEGS];
    __shared__ int s_nseg, s_err;
    __shared__ int64_t s_total;
    if (threadIdx.x == 0) {
        const uint8_t *f = J.frame;
        const int64_t fs = J.frame_size;
        int err = 0, nseg = 0;
        int64_t p = 0, outp = 0;
        unsigned long long csize = 0;
        if (fs < 6 || f[0] != 0x28 || f[1] != 0xB5 || f[2] != 0x2F || f[3] != 0xFD) err = 1;
        if (!err) {
            const uint8_t fhd = f[4];
            const int fcs_flag = fhd >> 6, ss = (fhd >> 5) & 1, ck = (fhd >> 2) & 1, did = fhd & 3;
            if (fhd & 0x08) err = 1;
            p = 5 + (ss ? 0 : 1);
            const int did_bytes = did == 0 ? 0 : (did == 1 ? 1 : (did == 2 ? 2 : 4));
            p += did_bytes;
            const int fcs_bytes = fcs_flag == 0 ? (ss ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
            if (fcs_bytes == 0 || p + fcs_bytes > fs) err = 1;
            if (!err) {
                for (int i = 0; i < fcs_bytes; i++) csize |= (unsigned long long)f[p + i] << (8 * i);
                if (fcs_bytes == 2) csize += 256;
                p += fcs_bytes;
            }
            while (!err) {
                if (p + 3 > fs) { err = 1; break; }
                const uint32_t h = f[p] | ((uint32_t)f[p + 1] << 8) | ((uint32_t)f[p + 2] << 16);
                p += 3;
                const int last = h & 1, type = (h >> 1) & 3;
                const int64_t bsz = h >> 3;
                if (nseg >= MAX_SEGS || type > 1) { err = 1; break; }
                if (type == 0) {
                    if (p + bsz > fs) { err = 1; break; }
                    s_src[nseg] = p;
                    p += bsz;
                } else {
                    if (p + 1 > fs) { err = 1; break; }
                    s_src[nseg] = p;
                    p += 1;
                }
                s_type[nseg] = type;
                s_dst[nseg] = outp;
                s_len[nseg] = bsz;
                outp += bsz;
                nseg++;
                if (last) break;
            }
            if (!err && ck) p += 4;
            if (!err && (p > fs || (unsigned long long)outp != csize || outp > J.cap)) err = 1;
        }
        s_err = err;
        s_nseg = nseg;
        s_total = outp;
        if (err) *J.content_out = -1;
        else *J.content_out = outp;
    }
    __syncthreads();
    if (s_err) return;
    for (int s = 0; s < s_nseg; s++) {
        uint8_t *o = J.dst + s_dst[s];
        const uint8_t *src = J.frame + s_src[s];
        if (s_type[s] == 0) {
            copy_bytes(o, src, s_len[s]);
        } else {
            const uint8_t v = src[0];
            for (int64_t i = threadIdx.x; i < s_len[s]; i += TPB) o[i] = v;
        }
    }
    // zero padding up to the next 4-byte word so word readers see clean bits
    const int64_t pad_end = min(J.cap, (s_total + 3) & ~(int64_t)3);
    for (int64_t i = s_total + threadIdx.x; i < pad_end; i += TPB) J.dst[i] = 0;
}

// ------------------------------------------------------------------ decode
__device__ __forceinline__ uint32_t word_mask(int64_t w, int64_t nbits) {
    const int64_t lo = w * 32;
    if (lo + 32 <= nbits) return FULL;
    if (lo >= nbits) return 0u;
    return (1u << (uint32_t)(nbits - lo)) - 1u;
}

struct DecTile {
    int64_t k0, k1, e0, e1;
};
__device__ __forceinline__ DecTile dec_range(const mc_dec_item &I, int t) {
    DecTile r;
    r.k0 = (int64_t)t * I.tile_kernels;
    r.k1 = min(r.k0 + (int64_t)I.tile_kernels, I.K);
    r.e0 = r.k0 * I.ks;
    r.e1 = r.k1 * I.ks;
    return r;
}

// Usable bitmap bits: min(content bytes * 8, K); content expanded on the
// device reports its length (or -1 when the frame could not be read).
__device__ __forceinline__ int64_t dec_bm_bits(const mc_dec_item &I) {
    if (!I.bm_len_ptr) return I.bm_bits;
    const int64_t len = *I.bm_len_ptr;
    if (len < 0) return 0;
    return min(len * 8, I.K);
}

// Content byte b of a payload read in place (Raw / RLE frames) or from
// contiguous content.
__device__ __forceinline__ uint32_t src_byte(const uint8_t *p, int mode, int64_t b) {
    if (mode == MC_BM_RAW) return p[fpos_raw(b)];
    if (mode == MC_BM_RLE) return p[fpos_rle(b)];
    return p[b];
}

// Bitmap word w (unmasked).  The 4 bytes of a word never straddle a block.
__device__ __forceinline__ uint32_t dec_bm_word(const mc_dec_item &I, int64_t w) {
    if (I.bm_mode == MC_BM_RLE) return src_byte(I.bm_frame, MC_BM_RLE, 4 * w) * 0x01010101u;
    if (I.bm_mode == MC_BM_RAW) {
        const uint8_t *q = I.bm_frame + fpos_raw(4 * w);
        if ((((uintptr_t)q) & 3) == 0) return *(const uint32_t *)q;
        return (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16) | ((uint32_t)q[3] << 24);
    }
    return I.bm_words[w];
}

__device__ __forceinline__ uint32_t le32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Checks that a frame read in place is what the host assumed: descriptor
// 0xA0 with a 4-byte content size (equal to `want` when want >= 0), then
// blocks of 2^17 bytes (the last one shorter), all of one type, the last
// one flagged.  Returns the content size or -1.  One thread.
__device__ int64_t check_frame(const uint8_t *f, int mode, int64_t want) {
    if (f[0] != 0x28 || f[1] != 0xB5 || f[2] != 0x2F || f[3] != 0xFD || f[4] != 0xA0) return -1;
    const int64_t cs = le32(f + 5);
    if (want >= 0 && cs != want) return -1;
    const int64_t nb = nblocks_of(cs);
    const int type = mode == MC_BM_RAW ? 0 : 1;
    for (int64_t j = 0; j < nb; j++) {
        const uint8_t *p = f + MC_ZHDR + j * (mode == MC_BM_RAW ? (int64_t)MC_ZBLOCK + 3 : 4);
        const uint32_t h = p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16);
        const int64_t bytes = cs == 0 ? 0 : min((int64_t)MC_ZBLOCK, cs - (j << MC_ZBLOCK_LOG2));
        if ((int)(h & 1u) != (j == nb - 1) || (int)((h >> 1) & 3u) != type || (int64_t)(h >> 3) != bytes)
            return -1;
    }
    return cs;
}

// Decoder, first launch (one warp per momentum tile): predicted kernels of
// the tile from its bitmap words; the first tile of an item also checks the
// headers of the frames read in place.
__global__ void __launch_bounds__(TPB) k_dec_prefix(mc_dec_launch L) {
    pdl_wait();
    pdl_release();
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * NWARP + (threadIdx.x >> 5);
    if (j >= L.nmom_tiles) return;
    const int2 e = ((const int2 *)L.mom_tiles)[j];
    const int gt = e.x, ii = e.y;
    const mc_dec_item &I = L.items[ii];
    const int t = gt - I.tile_base;
    if (t == 0 && lane == 0) {
        int bad = 0;
        if (I.bm_mode != MC_BM_WORDS) bad |= check_frame(I.bm_frame, I.bm_mode, (I.bm_bits + 7) >> 3) < 0;
        if (I.sg_mode != MC_BM_WORDS && I.sg_frame) bad |= check_frame(I.sg_frame, I.sg_mode, I.sg_len) < 0;
        if (bad) L.results[ii].err = 1;
    }
    const DecTile tr = dec_range(I, t);
    const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
    const int64_t bm_bits = dec_bm_bits(I);
    long long c = 0;
    for (int64_t w = wb + lane; w < we; w += 32) c += __popc(dec_bm_word(I, w) & word_mask(w, bm_bits));
    c = warp_sum_ll(c);
    if (lane == 0) L.tile_count[gt] = (int32_t)c;
}

// Decoder, second launch (one CTA per item): offset of each momentum tile's
// first predicted kernel in the dense signs (exclusive scan of the tile
// counts, in tile order) and the item's predicted total.
__global__ void __launch_bounds__(TPB) k_dec_scan(mc_dec_launch L) {
    __shared__ int scan_sh[NWARP + 1];
    pdl_wait();
    pdl_release();
    const int ii = L.item0 + blockIdx.x;
    const mc_dec_item &I = L.items[ii];
    if (I.kind != MC_D_MOMENTUM) return;
    const int64_t P = scan_tile_counts(L.tile_count, 1, I.tile_base, I.ntiles, L.tile_poff, scan_sh);
    if (threadIdx.x == 0) L.results[ii].P = P;
}

// Residual values of one quad from the payload (codes * scale or raw floats);
// `data` is the payload's data pointer or its staged copy (same indexing).
__device__ __forceinline__ void dec_resid4(const mc_dec_item &I, const uint8_t *data, int64_t g, int64_t e1,
                                           float scale, float (&r)[4]) {
    if (I.codec == MC_DC_Q8) {
        uint32_t w;
        if (I.vec && g + 4 <= e1) {
            w = *(const uint32_t *)(data + g);
        } else {
            w = 0;
            for (int j = 0; j < 4; j++)
                if (g + j < e1) w |= (uint32_t)data[g + j] << (8 * j);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) r[j] = __fmul_rn((float)(int8_t)(uint8_t)(w >> (8 * j)), scale);
    } else if (I.codec == MC_DC_INT4) {
        uint32_t w;
        if (I.vec && g + 4 <= e1) {
            w = *(const uint16_t *)(data + (g >> 1));
        } else {
            w = data[g >> 1];
            if (g + 2 < e1) w |= (uint32_t)data[(g >> 1) + 1] << 8;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) r[j] = __fmul_rn((float)((int)((w >> (4 * j)) & 15u) - 8), scale);
    } else {
        ld4((const float *)data, g, e1, I.vec, r);
    }
}

// Fused server-side aggregate of a decoded quad at element g (I.agg != NULL):
// agg = fma(w, decoded, agg), or fma(w, decoded, +0) in store mode (the old
// value not read).  One rounding per element and client, the same bits as a
// separate accumulate pass over the decoded tensor.
// Landing buffer of rank r (a select over the kernel-parameter array, so it
// is not copied to local memory for a dynamic index).
__device__ __forceinline__ float *landing_of(const mc_agg_shards &S, int r) {
    float *p = nullptr;
#pragma unroll
    for (int k = 0; k < MC_MAX_RANKS; k++)
        if (k == r) p = S.landing[k];
    return p;
}

// With a sharded aggregate (the SHARD instantiation of the decoder) the
// value, this rank's partial sum (the local aggregate, not read in store
// mode, plus weight * decoded), goes to the owner's landing slot for this
// rank instead (peer memory).
// `agg_in`: the aggregate's old values, element-indexed like I.agg (its
// staged copy, or I.agg itself).
template <bool SHARD>
__device__ __forceinline__ void agg_quad(const mc_dec_launch &L, const mc_dec_item &I, int64_t g, int64_t e1,
                                         const float (&v)[4], const float *agg_in) {
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (!I.agg_store) ld4(agg_in, g, e1, I.agg_vec != 0, a);
#pragma unroll
    for (int j = 0; j < 4; j++) a[j] = __fmaf_rn(I.agg_w, v[j], a[j]);
    if constexpr (!SHARD) {
        st4(I.agg, g, e1, I.agg_vec != 0, a);
    } else {
        const int64_t S = L.shards.shard;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (g + j >= e1) break;
            const int64_t x = I.agg_off + g + j;
            const int64_t sh = x / S;
            landing_of(L.shards, (int)sh)[(int64_t)L.shards.rank * S + (x - sh * S)] = a[j];
        }
    }
}

// Sign bytes a reconstruct tile needs: its predicted kernels' bits start at
// bit (tile_poff & 7) of the window; up to STAGE_ELEMS kernels per tile, plus
// the read-ahead of the 5-byte gather.
#define SIGN_WIN (STAGE_ELEMS / 8 + 16)
// Byte region of a reconstruct stage: the tile's q8 / int4 codes (at most
// STAGE_ELEMS bytes, plus the 15-byte misalignment of their start).
#define RC_XB (STAGE_ELEMS + 32)

// Momentum tiles of the decoder, before the wait on the tile's bulk copies:
// the tile's bitmap words, the offset of its first predicted kernel in the
// dense signs (from the scan kernel) and the deposited dominant-sign words,
// into shared memory (s_m, s_d; word wb = k0 / 32 at index 0); every tile
// also reads the payload's scale header into *s_scale.
__device__ void recon_pre(const mc_dec_launch &L, const StageDesc &d, uint32_t *s_m, uint32_t *s_d, int *scan_sh,
                          uint8_t *s_sb, float *s_scale) {
    const int ii = d.ii;
    const mc_dec_item &I = L.items[ii];
    const int t = d.gt - I.tile_base;
    // the scale header may sit at any byte address (payloads from the caller)
    if (threadIdx.x == 0)
        *s_scale = (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) ? __uint_as_float(le32((const uint8_t *)I.scale_ptr))
                                                                  : 1.0f;
    if (I.kind == MC_D_MOMENTUM) {
        const DecTile tr = dec_range(I, t);
        const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
        const int i = threadIdx.x;
        const int64_t bm_bits = dec_bm_bits(I);
        // sign source: expanded content, or a frame read in place
        const uint8_t *sg = I.sg_mode == MC_BM_WORDS ? I.sg_bytes : I.sg_frame;
        int64_t sg_len = I.sg_len;
        if (I.sg_len_ptr) {
            sg_len = *I.sg_len_ptr;
            if (sg_len < 0) sg = nullptr;
        }
        const int64_t poff = L.tile_poff[d.gt];
        uint32_t m = 0;
        if (wb + i < we && i < TILE_WORDS) m = dec_bm_word(I, wb + i) & word_mask(wb + i, bm_bits);
        const int pc = __popc(m);
        int tot;
        const int off_l = block_excl_scan(pc, scan_sh, &tot);
        // the tile's sign bits, staged as bytes; bytes past the sign content
        // read as 0xFF: missing signs default to +1 (ref :3296-3302)
        const int64_t b0 = poff >> 3;
        const int nb = tot > 0 ? (int)(((poff + tot + 7) >> 3) - b0) : 0;
        for (int j = threadIdx.x; j < nb + 8 && j < SIGN_WIN; j += TPB) {
            const int64_t b = b0 + j;
            uint32_t v = 0xFFu;
            if (sg && j < nb && b < sg_len) v = src_byte(sg, I.sg_mode, b);
            s_sb[j] = (uint8_t)v;
        }
        __syncthreads();
        uint32_t dm = 0;
        if (pc) {
            const int o = (int)(poff & 7) + off_l;
            const int ob = o >> 3;
            uint64_t w = 0;
#pragma unroll
            for (int k = 0; k < 5; k++) w |= (uint64_t)s_sb[ob + k] << (8 * k);
            dm = pdep32((uint32_t)(w >> (o & 7)), m);   // the pc sign bits at the set bits of m
        }
        if (i < TILE_WORDS) {
            s_m[i] = m;
            s_d[i] = dm;
        }
    }
}

// `codes`: the tile's payload bytes, staged or in place, indexed like
// I.data; `scale`: the payload's scale header (1 without one).
template <bool SHARD>
__device__ void recon_tile(const mc_dec_launch &L, const StageDesc &d, const float *buf, const uint32_t *s_m,
                           const uint32_t *s_d, const uint8_t *codes, float scale) {
    const int gt = d.gt;
    const int ii = d.ii;
    const mc_dec_item I = L.items[ii];
    const int t = gt - I.tile_base;
    float *hist = (float *)I.hist_out;
    float *out = (float *)I.out;
    if (I.kind == MC_D_MOMENTUM) {
        const DecTile tr = dec_range(I, t);
        const int64_t wb = tr.k0 >> 5;
        const MomParams mp = {I.cm, I.cs, 0.0f, 0.0f, I.cs > 1e-8f};
        const float pm = I.pm, lr = I.lr;
        const bool use_ps = I.ps > 1e-8f;
        const float inv_ps = use_ps ? __fdiv_rn(1.0f, I.ps) : 1.0f;
        const float oml = __fsub_rn(1.0f, lr);
        const uint32_t k0 = (uint32_t)tr.k0;
        const float *mem_in = staged_or(d, buf, 0, I.mem_in);
        const float *prev = staged_or(d, buf, 1, I.prev);
        // reconstruction of a quad: memory update and prediction on predicted elements
        auto quad = [&](const QuadBits &qb, const float (&r)[4], const float (&m0)[4], const float (&p)[4],
                        float (&mo)[4], float (&rec)[4]) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                rec[j] = r[j];
                mo[j] = m0[j];
                if ((qb.f >> j) & 1u) {
                    const float pv = __fsub_rn(fabsf(p[j]), pm);
                    const float pn = use_ps ? __fmul_rn(pv, inv_ps) : pv;
                    const float nm = __fmaf_rn(oml, m0[j], __fmul_rn(lr, pn));
                    mo[j] = nm;
                    const float ap = mom_pred_abs(nm, mp);
                    rec[j] = __fadd_rn(r[j], ((qb.pos >> j) & 1u) ? ap : -ap);
                }
            }
        };
        // bitmap / sign words of the tile are in shared memory from word wb on
        const int len = (int)(tr.e1 - tr.e0), nq = len >> 2;
        if (I.vec) {   // whole quads, no range checks
            const float4 *m4 = mem_in ? (const float4 *)(mem_in + tr.e0) : nullptr;
            const float4 *p4 = (const float4 *)(prev + tr.e0);
            float4 *mo4 = (float4 *)(I.mem_out + tr.e0), *h4 = (float4 *)(hist + tr.e0);
            const uint64_t spol = l2_stream();   // read again next round only
            // one loop per destination set, so each keeps only the pointers it
            // writes live: 0 output copy (or none), 1 aggregate, 2 both (or a
            // sharded aggregate through agg_quad), 3 sharded aggregate alone
            auto quads = [&](auto dst) {
                constexpr int M = decltype(dst)::value;
                float4 *o4 = (M == 0 || M == 2) && out ? (float4 *)(out + tr.e0) : nullptr;
                float4 *a4 = M != 0 ? (float4 *)(I.agg + tr.e0) : nullptr;
                const float aw = I.agg_w;
                const bool astore = I.agg_store != 0, avec = I.agg_vec != 0;
                // sharded: the tile's elements lie in at most two shards (a
                // shard holds at least a tile); x < sb1 goes to sp0 + x, the
                // rest to sp1 + x
                float *sp0 = nullptr, *sp1 = nullptr;
                int64_t sb1 = 0;
                if (M == 3) {
                    const int64_t S = L.shards.shard, x0 = I.agg_off + tr.e0;
                    const int s0 = (int)(x0 / S);
                    sb1 = (int64_t)(s0 + 1) * S;
                    sp0 = landing_of(L.shards, s0) + (int64_t)L.shards.rank * S - (int64_t)s0 * S;
                    if (s0 + 1 < L.shards.nranks)
                        sp1 = landing_of(L.shards, s0 + 1) + (int64_t)L.shards.rank * S - (int64_t)(s0 + 1) * S;
                }
                for (int q = threadIdx.x; q < nq; q += TPB) {
                    const QuadBits qb = quad_bits_full(s_m, s_d, (uint32_t)wb, k0, 4u * q, I.ks, I.ksdiv);
                    float r[4];
                    dec_resid4(I, codes, tr.e0 + 4 * q, tr.e1, scale, r);
                    const float4 mv = m4 ? m4[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    float4 pv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (qb.f) pv = p4[q];
                    const float m0[4] = {mv.x, mv.y, mv.z, mv.w}, p[4] = {pv.x, pv.y, pv.z, pv.w};
                    float mo[4], rec[4];
                    quad(qb, r, m0, p, mo, rec);
                    st_f4(mo4 + q, make_float4(mo[0], mo[1], mo[2], mo[3]), spol);
                    const float4 rv = make_float4(rec[0], rec[1], rec[2], rec[3]);
                    st_f4(h4 + q, rv, spol);
                    if ((M == 0 || M == 2) && o4) st_f4(o4 + q, rv, spol);
                    if (M == 3) {
                        // this rank's partial sum into the owner's landing slot
                        float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        if (!astore) a = a4[q];
                        const int64_t x = I.agg_off + tr.e0 + 4 * q;
                        *(float4 *)((x < sb1 ? sp0 : sp1) + x) =
                            make_float4(__fmaf_rn(aw, rec[0], a.x), __fmaf_rn(aw, rec[1], a.y),
                                        __fmaf_rn(aw, rec[2], a.z), __fmaf_rn(aw, rec[3], a.w));
                    } else if (M != 0) {
                        if (avec && !SHARD) {
                            // streamed like the other outputs: the aggregate is
                            // read again only by the next client's decode
                            float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                            if (!astore) a = a4[q];
                            st_f4(a4 + q, make_float4(__fmaf_rn(aw, rec[0], a.x), __fmaf_rn(aw, rec[1], a.y),
                                                      __fmaf_rn(aw, rec[2], a.z), __fmaf_rn(aw, rec[3], a.w)), spol);
                        } else {
                            agg_quad<SHARD>(L, I, tr.e0 + 4 * q, tr.e1, rec, I.agg);
                        }
                    }
                }
            };
            if (!I.agg) quads(std::integral_constant<int, 0>());
            else if constexpr (SHARD) {
                if (!out && I.agg_vec) quads(std::integral_constant<int, 3>());
                else quads(std::integral_constant<int, 2>());
            } else {
                if (!out) quads(std::integral_constant<int, 1>());
                else quads(std::integral_constant<int, 2>());
            }
        }
        const int64_t gstart = I.vec ? tr.e0 + 4 * (int64_t)nq : tr.e0;
        const int owner = I.vec ? nq % TPB : 0;
        for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < tr.e1; g += 4 * TPB) {
            const QuadBits qb = quad_bits(s_m, s_d, (uint32_t)wb, k0, g, tr.e0, tr.e1, I.ks, I.ksdiv);
            float r[4], m0[4], p[4], mo[4], rec[4];
            dec_resid4(I, codes, g, tr.e1, scale, r);
            if (mem_in) ld4(mem_in, g, tr.e1, I.vec, m0);
            else m0[0] = m0[1] = m0[2] = m0[3] = 0.0f;
            if (qb.f) ld4(prev, g, tr.e1, I.vec, p);
            quad(qb, r, m0, p, mo, rec);
            st4(I.mem_out, g, tr.e1, I.vec, mo);
            st4(hist, g, tr.e1, I.vec, rec);
            if (out) st4(out, g, tr.e1, I.vec, rec);
        }
        if (I.agg) {
            // the aggregate of the same quads, from this thread's own history
            // writes (kept out of the loop above, which holds more live values)
            for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < tr.e1; g += 4 * TPB) {
                float rec[4];
                ld4(hist, g, tr.e1, I.vec, rec);
                agg_quad<SHARD>(L, I, g, tr.e1, rec, I.agg);
            }
        }
        return;
    }
    const int64_t e0 = (int64_t)t * I.tile_kernels;
    const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
    if (I.kind == MC_D_RESIDUAL || I.kind == MC_D_QUANT) {
        // sharded: the tile's (at most 4096) elements lie in at most two
        // shards; whole aligned quads go to sp0 + x or sp1 + x
        float *sp0 = nullptr, *sp1 = nullptr;
        int64_t sb1 = 0;
        bool sfast = false;
        if constexpr (SHARD) {
            if (I.agg) {
                const int64_t S = L.shards.shard, x0 = I.agg_off + e0;
                const int s0 = (int)(x0 / S);
                sb1 = (int64_t)(s0 + 1) * S;
                sp0 = landing_of(L.shards, s0) + (int64_t)L.shards.rank * S - (int64_t)s0 * S;
                if (s0 + 1 < L.shards.nranks)
                    sp1 = landing_of(L.shards, s0 + 1) + (int64_t)L.shards.rank * S - (int64_t)(s0 + 1) * S;
                sfast = I.agg_vec && (I.agg_off & 3) == 0;
            }
        }
        // the old aggregate, staged as array 0 when the plan staged it
        const float *agg_in = staged_or(d, buf, 0, I.agg);
        int64_t gstart = e0;
        int owner = 0;
        if (!SHARD && I.vec && (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) && (!I.agg || I.agg_vec)) {
            // whole quads, no range checks; codec and aggregate mode as template arguments
            const int nq = (int)((e1 - e0) >> 2);
            auto quads = [&](auto codec, auto store) {
                constexpr int C = decltype(codec)::value;
                constexpr bool ST = decltype(store)::value;
                for (int q = threadIdx.x; q < nq; q += TPB) {
                    const int64_t g = e0 + 4 * (int64_t)q;
                    float r[4];
                    if (C == MC_DC_Q8) {
                        const uint32_t w = *(const uint32_t *)(codes + g);
#pragma unroll
                        for (int j = 0; j < 4; j++) r[j] = __fmul_rn((float)(int8_t)(uint8_t)(w >> (8 * j)), scale);
                    } else {
                        const uint32_t w = *(const uint16_t *)(codes + (g >> 1));
#pragma unroll
                        for (int j = 0; j < 4; j++) r[j] = __fmul_rn((float)((int)((w >> (4 * j)) & 15u) - 8), scale);
                    }
                    const float4 rv = make_float4(r[0], r[1], r[2], r[3]);
                    *(float4 *)(hist + g) = rv;
                    if (out) *(float4 *)(out + g) = rv;
                    if (I.agg) {
                        float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                        if (!ST) a = *(const float4 *)(agg_in + g);
                        *(float4 *)(I.agg + g) = make_float4(__fmaf_rn(I.agg_w, r[0], a.x), __fmaf_rn(I.agg_w, r[1], a.y),
                                                             __fmaf_rn(I.agg_w, r[2], a.z), __fmaf_rn(I.agg_w, r[3], a.w));
                    }
                }
            };
            const bool st = I.agg_store != 0;
            if (I.codec == MC_DC_Q8) {
                if (st) quads(std::integral_constant<int, MC_DC_Q8>(), std::true_type());
                else quads(std::integral_constant<int, MC_DC_Q8>(), std::false_type());
            } else {
                if (st) quads(std::integral_constant<int, MC_DC_INT4>(), std::true_type());
                else quads(std::integral_constant<int, MC_DC_INT4>(), std::false_type());
            }
            gstart = e0 + 4 * (int64_t)nq;
            owner = nq % TPB;
        }
        // the ragged end (or every quad, where the fast loop does not apply)
        for (int64_t g = gstart + 4 * (int64_t)((threadIdx.x - owner + TPB) % TPB); g < e1; g += 4 * TPB) {
            float r[4];
            dec_resid4(I, codes, g, e1, scale, r);
            st4(hist, g, e1, I.vec, r);
            if (out) st4(out, g, e1, I.vec, r);
            if (!I.agg) continue;
            if (SHARD && sfast && g + 4 <= e1) {
                float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (!I.agg_store) a = *(const float4 *)(agg_in + g);
                const int64_t x = I.agg_off + g;
                *(float4 *)((x < sb1 ? sp0 : sp1) + x) =
                    make_float4(__fmaf_rn(I.agg_w, r[0], a.x), __fmaf_rn(I.agg_w, r[1], a.y),
                                __fmaf_rn(I.agg_w, r[2], a.z), __fmaf_rn(I.agg_w, r[3], a.w));
            } else {
                agg_quad<SHARD>(L, I, g, e1, r, agg_in);
            }
        }
        return;
    }
    // MC_D_COPY: bytes (tile in bytes)
    auto copy_tile = [&]() {
        const uint8_t *src = I.data;
        uint8_t *h8 = (uint8_t *)I.hist_out, *o8 = (uint8_t *)I.out;
        if (I.data_mode != MC_BM_WORDS) {
            // lossless frame read in place: check the header the host assumed;
            // a tile (at most 2^15 bytes) lies inside one block of the frame
            if (t == 0 && threadIdx.x == 0 && check_frame(I.data_frame, I.data_mode, I.n) < 0)
                L.results[ii].err = 1;
            if (I.data_mode == MC_BM_RLE) {
                const uint8_t v = (uint8_t)src_byte(I.data_frame, MC_BM_RLE, e0);
                for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
                    h8[e] = v;
                    if (o8) o8[e] = v;
                }
                return;
            }
            src = I.data_frame + fpos_raw(e0) - e0;   // byte e of this tile at src[e]
        }
        if (!I.vec && ((((uintptr_t)src | (uintptr_t)h8 | (uintptr_t)o8) & 3) == 0)) {
            // 4-byte words (tiles are multiples of 16 bytes)
            const int64_t w0 = e0 >> 2, w1 = e1 >> 2;
            for (int64_t w = w0 + threadIdx.x; w < w1; w += TPB) {
                const uint32_t x = ((const uint32_t *)src)[w];
                ((uint32_t *)h8)[w] = x;
                if (o8) ((uint32_t *)o8)[w] = x;
            }
            for (int64_t e = (w1 << 2) + threadIdx.x; e < e1; e += TPB) {
                h8[e] = src[e];
                if (o8) o8[e] = src[e];
            }
            return;
        }
        if (I.vec) {
            const int64_t v0 = e0 >> 4, v1 = e1 >> 4;
            for (int64_t v = v0 + threadIdx.x; v < v1; v += TPB) {
                const uint4 x = ((const uint4 *)src)[v];
                ((uint4 *)h8)[v] = x;
                if (o8) ((uint4 *)o8)[v] = x;
            }
            for (int64_t e = (v1 << 4) + threadIdx.x; e < e1; e += TPB) {
                h8[e] = src[e];
                if (o8) o8[e] = src[e];
            }
        } else {
            for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
                const uint8_t v = src[e];
                h8[e] = v;
                if (o8) o8[e] = v;
            }
        }
    };
    copy_tile();
    if (I.agg) {
        // float32 item: the aggregate from the history copy this CTA just
        // wrote (visible to the whole CTA after the barrier); byte tiles
        // of a float32 item start and end on element boundaries
        __syncthreads();
        const float *hf = (const float *)I.hist_out;
        const int64_t f0 = e0 >> 2, f1 = e1 >> 2;
        for (int64_t g = f0 + 4 * (int64_t)threadIdx.x; g < f1; g += 4 * TPB) {
            float v[4];
            ld4(hf, g, f1, true, v);
            agg_quad<SHARD>(L, I, g, f1, v, I.agg);
        }
    }
}

template <bool SHARD>
__global__ void __launch_bounds__(TPB, SHARD ? 3 : 4) k_dec_recon(mc_dec_launch L) {
    __shared__ uint32_t s_m[TILE_WORDS], s_d[TILE_WORDS];
    __shared__ int scan_sh[NWARP + 1];
    __shared__ uint8_t s_sb[SIGN_WIN];
    __shared__ float s_scale;
    __shared__ TileShared ts;
    extern __shared__ __align__(128) float s_stage[];
    run_tile<2, false>((const int2 *)L.all_tiles, s_stage, &ts.bar, &ts.d, &L.results[0].err,
                (int)(sizeof(mc_dec_result) / 4),
                    [&](StageDesc &d) {
                        const mc_dec_item &I = L.items[d.ii];
                        const int t = d.gt - I.tile_base;
                        d.src[0] = d.src[1] = d.src[2] = nullptr;
                        if (I.kind == MC_D_MOMENTUM) {
                            const DecTile tr = dec_range(I, t);
                            d.e0 = tr.e0;
                            d.e1 = tr.e1;
                            if (L.staged && I.vec && d.e1 - d.e0 <= STAGE_ELEMS) {
                                d.src[0] = I.mem_in;
                                if (L.tile_count[d.gt] > 0) d.src[1] = I.prev;
                                // the codes, staged behind the arrays
                                if (I.codec == MC_DC_Q8) {
                                    d.x0 = I.data + d.e0;
                                    d.x1 = I.data + d.e1;
                                } else if (I.codec == MC_DC_INT4) {
                                    d.x0 = I.data + (d.e0 >> 1);
                                    d.x1 = I.data + ((d.e1 + 1) >> 1);
                                }
                            }
                        } else {
                            d.e0 = (int64_t)t * I.tile_kernels;
                            d.e1 = min(d.e0 + (int64_t)I.tile_kernels, I.n);
                            // direct codes: staged like a momentum tile's; the old
                            // aggregate (add mode) too, after the dependent-launch
                            // wait: the previous decode on the stream may write it
                            if (I.kind == MC_D_QUANT && L.staged && I.vec && d.e1 - d.e0 <= STAGE_ELEMS &&
                                (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4)) {
                                if (I.codec == MC_DC_Q8) {
                                    d.x0 = I.data + d.e0;
                                    d.x1 = I.data + d.e1;
                                } else {
                                    d.x0 = I.data + (d.e0 >> 1);
                                    d.x1 = I.data + ((d.e1 + 1) >> 1);
                                }
                                if (I.agg && !I.agg_store && I.agg_vec) {
                                    d.src[0] = I.agg;
                                    d.late = 1;
                                }
                            }
                        }
                    },
                    [&](const StageDesc &d) { recon_pre(L, d, s_m, s_d, scan_sh, s_sb, &s_scale); },
                    [&](const StageDesc &d, const float *buf) {
                        const uint8_t *data = L.items[d.ii].data;
                        const uint8_t *xb = (const uint8_t *)(buf + 2 * STAGE_ELEMS);
                        const uint8_t *codes = d.x0 ? xb + ((intptr_t)data - (intptr_t)dn16(d.x0)) : data;
                        recon_tile<SHARD>(L, d, buf, s_m, s_d, codes, s_scale);
                    });
}

// ------------------------------------------------------- sharded aggregate
// Second half of the sharded aggregate (the first is the decoder's stores
// into the owners' landing slots): this rank sums its shard over the nranks
// slots of its own landing buffer, in rank order, and stores the sum into
// every rank's aggregate (an all-gather by peer stores over NVLink).  Quads
// of 16-byte loads and stores: landing and aggregate bases are 16-byte
// aligned and the shard a multiple of 64 elements.
struct ShardDst {
    float *agg[MC_MAX_RANKS];
};
__global__ void __launch_bounds__(TPB) k_shard_reduce(const float *__restrict__ land, int nranks, int rank,
                                                     int64_t shard, int64_t total, ShardDst dst) {
    const int64_t base = (int64_t)rank * shard;
    const int64_t nq = shard >> 2;
    for (int64_t q = blockIdx.x * (int64_t)TPB + threadIdx.x; q < nq; q += (int64_t)gridDim.x * TPB) {
        const int64_t x = base + 4 * q;
        if (x >= total) break;
        float4 v = __ldcg((const float4 *)(land + 4 * q));
#pragma unroll
        for (int j = 1; j < MC_MAX_RANKS; j++) {
            if (j >= nranks) break;
            const float4 u = __ldcg((const float4 *)(land + (int64_t)j * shard + 4 * q));
            v.x = __fadd_rn(v.x, u.x);
            v.y = __fadd_rn(v.y, u.y);
            v.z = __fadd_rn(v.z, u.z);
            v.w = __fadd_rn(v.w, u.w);
        }
        if (x + 4 <= total) {
#pragma unroll
            for (int r = 0; r < MC_MAX_RANKS; r++)
                if (r < nranks) *(float4 *)(dst.agg[r] + x) = v;
        } else {
            const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int r = 0; r < MC_MAX_RANKS; r++) {
                if (r >= nranks) break;
                for (int k = 0; k < 4 && x + k < total; k++) dst.agg[r][x + k] = w[k];
            }
        }
    }
}

// One-shot in-place sum all-reduce of the ranks' aggregates over NVLink peer
// memory: this rank owns elements [lo, hi); it loads them from every rank's
// aggregate (peer loads, fetched again from the owner: ld.global.cv, so no
// line of an earlier round is reused), sums them in rank order and stores the
// sum into every rank's aggregate.  The ranks' ranges are disjoint, so no
// element is touched by two ranks, and each thread loads all of an element's
// values before it stores any.  Loads and stores go both ways over NVLink at
// once: the reduce-scatter (ingress) and the all-gather (egress) overlap.
struct PeerAggs {
    float *agg[MC_MAX_RANKS];
};
__global__ void __launch_bounds__(TPB) k_peer_allreduce(PeerAggs a, int nranks, int64_t lo, int64_t hi) {
    const int64_t nq = (hi - lo) >> 2;
    for (int64_t q = blockIdx.x * (int64_t)TPB + threadIdx.x; q < nq; q += (int64_t)gridDim.x * TPB) {
        const int64_t x = lo + 4 * q;
        float4 u[MC_MAX_RANKS];
#pragma unroll
        for (int r = 0; r < MC_MAX_RANKS; r++)
            if (r < nranks) u[r] = __ldcv((const float4 *)(a.agg[r] + x));
        float4 v = u[0];
#pragma unroll
        for (int r = 1; r < MC_MAX_RANKS; r++) {
            if (r >= nranks) break;
            v.x = __fadd_rn(v.x, u[r].x);
            v.y = __fadd_rn(v.y, u[r].y);
            v.z = __fadd_rn(v.z, u[r].z);
            v.w = __fadd_rn(v.w, u[r].w);
        }
#pragma unroll
        for (int r = 0; r < MC_MAX_RANKS; r++)
            if (r < nranks) *(float4 *)(a.agg[r] + x) = v;
    }
    // the last 0-3 elements of the range
    const int64_t x = lo + 4 * nq;
    if (blockIdx.x == 0 && x + threadIdx.x < hi) {
        const int64_t e = x + threadIdx.x;
        float v = __ldcv(a.agg[0] + e);
        for (int r = 1; r < nranks; r++) v = __fadd_rn(v, __ldcv(a.agg[r] + e));
        for (int r = 0; r < nranks; r++) a.agg[r][e] = v;
    }
}

// The one-shot all-reduce with its two barriers in the kernel itself, over
// flag words in every rank's memory (block f of rank r, mapped into every
// rank: words [0, 8) arrival of rank q, [8, 16) completion of rank q, word
// 16 this launch's CTA count, word 17 an error flag).  Each launch carries a
// round number `epoch`, larger than the last one; a flag is set when it
// holds epoch (compared modulo 2^32).
//  * arrival: block 0 of every rank, once its kernel starts (so its decodes,
//    earlier on its stream, are complete), stores epoch into word `rank` of
//    every rank's block (system-scope release after a system fence); every
//    CTA waits until its own block shows all ranks arrived, then sums its
//    share of the rank's shard as k_peer_allreduce does;
//  * completion: every CTA fences its peer stores and counts itself in word
//    16; the last one stores epoch into word 8 + rank of every rank's block
//    and waits until all ranks completed, so no kernel after this one on the
//    stream (the next round's decodes into the aggregate) starts while a
//    peer still reads or writes this rank's aggregate.
// Every wait is bounded (about a second); one that runs out sets word 17
// and the CTA stops, so a missing rank ends in an error flag, not a hang.
struct PeerFlags {
    uint32_t *blk[MC_MAX_RANKS];
};
#define PF_ARRIVE 0
#define PF_DONE 8
#define PF_COUNT 16
#define PF_ERR 17
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// true once p[k] has reached `epoch` for every k < n; false after about a second
__device__ bool wait_flags(const uint32_t *p, int n, uint32_t epoch) {
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (int k = 0; k < n; k++) {
        for (uint32_t i = 0;; i++) {
            if ((int32_t)(ld_acquire_sys(p + k) - epoch) >= 0) break;
            if (i >= (1u << 22)) return false;
            __nanosleep(128);
            if ((i & 63) == 63) {
                uint64_t t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > 1000000000ull) return false;
            }
        }
    }
    return true;
}
__global__ void __launch_bounds__(TPB) k_peer_allreduce_sync(PeerAggs a, PeerFlags f, int nranks, int rank,
                                                             int64_t lo, int64_t hi, uint32_t epoch) {
    __shared__ int s_ok;
    uint32_t *mine = f.blk[rank];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        __threadfence_system();
        for (int r = 0; r < nranks; r++) st_release_sys(f.blk[r] + PF_ARRIVE + rank, epoch);
    }
    if (threadIdx.x == 0) {
        s_ok = wait_flags(mine + PF_ARRIVE, nranks, epoch);
        if (!s_ok) atomicExch(mine + PF_ERR, 1u);
    }
    __syncthreads();
    // a CTA whose wait ran out skips the sum but still counts itself, so the
    // count resets and every rank is released; the error flag reports it
    const int64_t nq = s_ok ? (hi - lo) >> 2 : 0;
    for (int64_t q = blockIdx.x * (int64_t)TPB + threadIdx.x; q < nq; q += (int64_t)gridDim.x * TPB) {
        const int64_t x = lo + 4 * q;
        float4 u[MC_MAX_RANKS];
#pragma unroll
        for (int r = 0; r < MC_MAX_RANKS; r++)
            if (r < nranks) u[r] = __ldcv((const float4 *)(a.agg[r] + x));
        float4 v = u[0];
#pragma unroll
        for (int r = 1; r < MC_MAX_RANKS; r++) {
            if (r >= nranks) break;
            v.x = __fadd_rn(v.x, u[r].x);
            v.y = __fadd_rn(v.y, u[r].y);
            v.z = __fadd_rn(v.z, u[r].z);
            v.w = __fadd_rn(v.w, u[r].w);
        }
#pragma unroll
        for (int r = 0; r < MC_MAX_RANKS; r++)
            if (r < nranks) *(float4 *)(a.agg[r] + x) = v;
    }
    const int64_t xt = lo + 4 * nq;
    if (s_ok && blockIdx.x == 0 && xt + threadIdx.x < hi) {
        const int64_t e = xt + threadIdx.x;
        float v = __ldcv(a.agg[0] + e);
        for (int r = 1; r < nranks; r++) v = __fadd_rn(v, __ldcv(a.agg[r] + e));
        for (int r = 0; r < nranks; r++) a.agg[r][e] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(mine + PF_COUNT, 1u) == gridDim.x - 1) {
            __threadfence_system();
            mine[PF_COUNT] = 0;   // the next launch comes after this one on the stream
            for (int r = 0; r < nranks; r++) st_release_sys(f.blk[r] + PF_DONE + rank, epoch);
            if (!wait_flags(mine + PF_DONE, nranks, epoch)) atomicExch(mine + PF_ERR, 1u);
        }
    }
}

// Copy of `bytes` bytes by the SMs: a transfer between pinned host memory
// (mapped into the device address space) and device memory that occupies
// no copy engine, so the copies the codec queues on the copy engines never
// wait behind it.  When source and destination are congruent modulo 16 the
// body moves in 16-byte loads and stores (up to four in flight per thread)
// and block 0 copies the ragged head and tail bytewise; otherwise every byte
// is copied on its own.
__global__ void __launch_bounds__(TPB) k_copy(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                              int64_t bytes, int64_t head, int64_t nq) {
    if (nq < 0) {   // incongruent ends
        for (int64_t i = blockIdx.x * (int64_t)TPB + threadIdx.x; i < bytes; i += (int64_t)gridDim.x * TPB)
            dst[i] = src[i];
        return;
    }
    const uint4 *s4 = (const uint4 *)(src + head);
    uint4 *d4 = (uint4 *)(dst + head);
    const int64_t stride = (int64_t)gridDim.x * TPB;
    for (int64_t q0 = blockIdx.x * (int64_t)TPB + threadIdx.x; q0 < nq; q0 += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (q0 + k * stride < nq) v[k] = __ldcs(s4 + q0 + k * stride);
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (q0 + k * stride < nq) __stcs(d4 + q0 + k * stride, v[k]);
    }
    if (blockIdx.x == 0) {
        for (int64_t i = threadIdx.x; i < head; i += TPB) dst[i] = src[i];
        for (int64_t i = head + 16 * nq + threadIdx.x; i < bytes; i += TPB) dst[i] = src[i];
    }
}

}  // namespace

// ---------------------------------------------------------------- launchers
static inline void tr_begin(mc_ktrace *tr, int kid, cudaStream_t s) {
    if (tr && tr->n < MC_KTRACE_MAX) {
        cudaEventRecord((cudaEvent_t)tr->ev[2 * tr->n], s);
        tr->kid[tr->n] = kid;
    }
}
static inline void tr_end(mc_ktrace *tr, cudaStream_t s) {
    if (tr && tr->n < MC_KTRACE_MAX) {
        cudaEventRecord((cudaEvent_t)tr->ev[2 * tr->n + 1], s);
        tr->n++;
    }
}

// Launch of a kernel that may start while the previous kernel on the stream
// is finishing (programmatic dependent launch; see pdl_wait).
template <typename... P, typename... A>
static void launch_pdl(void (*kern)(P...), int grid, size_t smem, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(TPB);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, args...);
}

// Dynamic shared memory of the staged kernels (one stage of NA arrays),
// opted in above the 48 KiB default once per kernel and device.
enum { KF_P1 = 0, KF_P2, KF_P3, KF_P4, KF_RECON, KF_RECON_SHARD, KF_N };
#define MAX_DEVICES 64
static int g_smem_set[KF_N][MAX_DEVICES];

static void smem_opt_in(int kf, const void *fn, size_t smem) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) dev = 0;
    if (!g_smem_set[kf][dev]) {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        g_smem_set[kf][dev] = 1;
    }
}

#define P1_SMEM STAGE_BYTES(2)
#define P2_SMEM STAGE_BYTES(2)
#define P3_SMEM STAGE_BYTES(3)
#define P4_SMEM STAGE_BYTES(2)
#define RECON_SMEM (STAGE_BYTES(2) + RC_XB)

extern "C" int mc_launch_encode(const mc_enc_launch *L, void *stream, mc_ktrace *tr) {
    cudaStream_t s = (cudaStream_t)stream;
    int n = 0;
    if (L->nall_tiles > 0) {
        smem_opt_in(KF_P1, (const void *)k_enc_pass1, P1_SMEM);
        tr_begin(tr, MC_KT_ENC_PASS1, s);
        k_enc_pass1<<<L->nall_tiles, TPB, P1_SMEM, s>>>(*L);
        tr_end(tr, s);
        tr_begin(tr, MC_KT_ENC_FINAL, s);
        launch_pdl(k_enc_final1, L->nitems, 0, s, *L);
        tr_end(tr, s);
        n += 2;
    }
    if (L->nmom_tiles > 0) {
        smem_opt_in(KF_P2, (const void *)k_enc_pass2, P2_SMEM);
        tr_begin(tr, MC_KT_ENC_PASS2, s);
        launch_pdl(k_enc_pass2, L->nmom_tiles, P2_SMEM, s, *L);
        tr_end(tr, s);
        tr_begin(tr, MC_KT_ENC_FINAL, s);
        launch_pdl(k_enc_final2, L->nitems, 0, s, *L);
        tr_end(tr, s);
        smem_opt_in(KF_P3, (const void *)k_enc_pass3, P3_SMEM);
        tr_begin(tr, MC_KT_ENC_PASS3, s);
        launch_pdl(k_enc_pass3, L->nmom_tiles, P3_SMEM, s, *L);
        tr_end(tr, s);
        tr_begin(tr, MC_KT_ENC_FINAL, s);
        launch_pdl(k_enc_final3, L->nitems, 0, s, *L);
        tr_end(tr, s);
        n += 4;
    }
    if (L->nall_tiles > 0) {
        smem_opt_in(KF_P4, (const void *)k_enc_pass4, P4_SMEM);
        tr_begin(tr, MC_KT_ENC_PASS4, s);
        launch_pdl(k_enc_pass4, L->nall_tiles, P4_SMEM, s, *L);
        tr_end(tr, s);
        n++;
    }
    if (cudaGetLastError() != cudaSuccess) return -1;
    return n;
}

extern "C" int mc_launch_decode(const mc_dec_launch *L, void *stream, mc_ktrace *tr) {
    cudaStream_t s = (cudaStream_t)stream;
    int n = 0;
    if (L->nmom_tiles > 0) {
        tr_begin(tr, MC_KT_DEC_PREFIX, s);
        k_dec_prefix<<<(L->nmom_tiles + NWARP - 1) / NWARP, TPB, 0, s>>>(*L);
        launch_pdl(k_dec_scan, L->item1 - L->item0, 0, s, *L);
        tr_end(tr, s);
        n += 2;
    }
    if (L->nall_tiles > 0) {
        tr_begin(tr, MC_KT_DEC_RECON, s);
        if (L->shards.nranks > 0) {   // the sharded-aggregate instantiation
            smem_opt_in(KF_RECON_SHARD, (const void *)k_dec_recon<true>, RECON_SMEM);
            launch_pdl(k_dec_recon<true>, L->nall_tiles, RECON_SMEM, s, *L);
        } else {
            smem_opt_in(KF_RECON, (const void *)k_dec_recon<false>, RECON_SMEM);
            launch_pdl(k_dec_recon<false>, L->nall_tiles, RECON_SMEM, s, *L);
        }
        tr_end(tr, s);
        n++;
    }
    if (cudaGetLastError() != cudaSuccess) return -1;
    return n;
}

extern "C" int mc_launch_unframe(const mc_unframe_job *jobs, int njobs, void *stream, mc_ktrace *tr) {
    if (njobs <= 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    tr_begin(tr, MC_KT_UNFRAME, s);
    k_unframe<<<njobs, TPB, 0, s>>>(jobs);
    tr_end(tr, s);
    if (cudaGetLastError() != cudaSuccess) return -1;
    return 1;
}

extern "C" int mc_launch_shard_reduce(const float *landing, int nranks, int rank, int64_t shard, int64_t total,
                                      float *const *aggregates, void *stream) {
    if (nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks || shard <= 0) return -1;
    ShardDst d;
    for (int r = 0; r < MC_MAX_RANKS; r++) d.agg[r] = r < nranks ? aggregates[r] : nullptr;
    const int64_t nq = shard >> 2;
    int blocks = (int)((nq + TPB - 1) / TPB);
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    cudaStream_t s = (cudaStream_t)stream;
    k_shard_reduce<<<blocks, TPB, 0, s>>>(landing, nranks, rank, shard, total, d);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}

extern "C" int mc_launch_copy(void *dst, const void *src, int64_t bytes, int nblocks, void *stream) {
    if (bytes <= 0) return 0;
    if (!dst || !src) return -1;
    const uintptr_t d = (uintptr_t)dst, s = (uintptr_t)src;
    int64_t head = 0, nq = -1;
    if (((d - s) & 15) == 0) {
        head = (int64_t)((16 - (d & 15)) & 15);
        if (head > bytes) head = bytes;
        nq = (bytes - head) >> 4;
    }
    if (nblocks < 1) nblocks = 1;
    if (nblocks > 148 * 8) nblocks = 148 * 8;
    cudaStream_t st = (cudaStream_t)stream;
    k_copy<<<nblocks, TPB, 0, st>>>((const uint8_t *)src, (uint8_t *)dst, bytes, head, nq);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}

extern "C" int mc_launch_peer_allreduce_sync(float *const *aggregates, uint32_t *const *flags, int nranks, int rank,
                                             int64_t shard, int64_t total, uint32_t epoch, void *stream) {
    if (nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks || shard <= 0 || (shard & 3) != 0)
        return -1;
    PeerAggs a;
    PeerFlags f;
    for (int r = 0; r < MC_MAX_RANKS; r++) {
        a.agg[r] = r < nranks ? aggregates[r] : nullptr;
        f.blk[r] = r < nranks ? flags[r] : nullptr;
    }
    const int64_t lo = (int64_t)rank * shard;
    int64_t hi = lo + shard < total ? lo + shard : total;
    if (hi < lo) hi = lo;   // an empty shard still takes part in both barriers
    const int64_t nq = (hi - lo) >> 2;
    int blocks = (int)((nq + TPB - 1) / TPB);
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    cudaStream_t s = (cudaStream_t)stream;
    k_peer_allreduce_sync<<<blocks, TPB, 0, s>>>(a, f, nranks, rank, lo, hi, epoch);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}

extern "C" int mc_launch_peer_allreduce(float *const *aggregates, int nranks, int rank, int64_t shard, int64_t total,
                                        void *stream) {
    if (nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks || shard <= 0 || (shard & 3) != 0)
        return -1;
    PeerAggs a;
    for (int r = 0; r < MC_MAX_RANKS; r++) a.agg[r] = r < nranks ? aggregates[r] : nullptr;
    const int64_t lo = (int64_t)rank * shard;
    const int64_t hi = lo + shard < total ? lo + shard : total;
    if (hi <= lo) return 0;
    const int64_t nq = (hi - lo) >> 2;
    int blocks = (int)((nq + TPB - 1) / TPB);
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    cudaStream_t s = (cudaStream_t)stream;
    k_peer_allreduce<<<blocks, TPB, 0, s>>>(a, nranks, lo, hi);
    return cudaGetLastError() == cudaSuccess ? 1 : -1;
}
