// mc_kernels.cu -- sm_100a kernels of the FalCom momentum codec.
//
// Memory-bound integer / fp32 work: no tensor cores.  Every float operation
// that feeds a payload byte is written as an explicit round-to-nearest
// intrinsic (__fmaf_rn, __fmul_rn, __fsub_rn, __fadd_rn, __fdiv_rn) in the
// order the reference build uses (momentum_compressor_openmp_simd_final.c,
// compiled -O3 -ffast-math with FMA contraction), and this file is compiled
// with -fmad=false so the compiler adds no contraction of its own.
//
// Encoder, one launch per pass over the batch tile list (one CTA per tile):
//   pass1  stats sums, min/max, per-kernel sign consistency -> bitmap and
//          dominant-sign words, history copy          (ref :1322-1431, :2040-2062)
//   pass2  squared deviations around the float means   (ref :1384-1416)
//   pass3  memory update, prediction, clamped residual, max|r|, mismatches
//          (ref :2094-2170)
//   pass4  residual codec (q8 / int4 / raw) and dense dominant-sign packing
//          (ref :2196-2214 replaced; :2258-2283)
//   frames zstd frames with Raw / RLE blocks for bitmap, signs and lossless
//          payloads (ref :2222-2256 framing via libzstd replaced)
// The last CTA of an item in each pass (atomic ticket) reduces the per-tile
// partials in a fixed order, so every result is run-to-run deterministic.
//
// Decoder: prefix (predicted-kernel offsets per tile) then reconstruct
// (ref :3186-3474), plus an optional frame-expansion kernel for
// device-resident zstd frames.

#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

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

// Reduce up to 4 doubles, 1 min, 2 max floats and 2 integers over the block.
__device__ void block_reduce(Red &sh, double (&d)[4], int nd, float &mn, float &mx, float &mx2,
                             long long (&l)[2], int nl) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = 0; i < nd; i++) d[i] = warp_sum_d(d[i]);
    mn = warp_min_f(mn);
    mx = warp_max_f(mx);
    mx2 = warp_max_f(mx2);
    for (int i = 0; i < nl; i++) l[i] = warp_sum_ll(l[i]);
    __syncthreads();
    if (lane == 0) {
        for (int i = 0; i < nd; i++) sh.d[i][w] = d[i];
        sh.f[0][w] = mn;
        sh.f[1][w] = mx;
        sh.f[2][w] = mx2;
        for (int i = 0; i < nl; i++) sh.l[i][w] = l[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 0; i < nd; i++) {
            double s = 0.0;
            for (int j = 0; j < NWARP; j++) s += sh.d[i][j];
            d[i] = s;
        }
        for (int j = 0; j < NWARP; j++) {
            mn = sh.f[0][j] < mn ? sh.f[0][j] : mn;
            mx = sh.f[1][j] > mx ? sh.f[1][j] : mx;
            mx2 = sh.f[2][j] > mx2 ? sh.f[2][j] : mx2;
        }
        for (int i = 0; i < nl; i++) {
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

// Elect the last CTA of an item for pass `phase` (all threads get the answer).
__device__ bool last_cta(uint32_t *ticket, int ntiles, int *flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *flag = (atomicAdd(ticket, 1u) == (uint32_t)(ntiles - 1));
    __syncthreads();
    if (*flag) __threadfence();
    return *flag != 0;
}

__device__ __forceinline__ int qmax_of(int codec) {
    return (codec == MC_DC_INT4 || codec == MC_DC_INT4_RAW) ? 7 : 127;
}

__device__ __forceinline__ int quant1(float r, float scale, float qm) {
    float v = rintf(__fdiv_rn(r, scale));
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

// Residual of one element of a momentum layer, recomputed from the updated
// memory (pass 4).  Same operation order as pass 3.
struct MomParams {
    float cm, cs, gmin, gmax;
    bool use_cs;
};
__device__ __forceinline__ float mom_residual(float c, float nm, bool pos, const MomParams &p) {
    float ap = p.use_cs ? __fmaf_rn(nm, p.cs, p.cm) : __fadd_rn(nm, p.cm);
    ap = fabsf(ap);
    float pred = pos ? ap : -ap;
    float r = __fsub_rn(c, pred);
    return x86min(x86max(r, p.gmin), p.gmax);
}

// ------------------------------------------------------------------ pass 1
__global__ void __launch_bounds__(TPB) k_enc_pass1(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ int s_flag;
    const int gt = L.all_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_enc_item I = L.items[ii];
    const int t = gt - I.tile_base;
    mc_enc_result *R = L.results + ii;
    double d[4] = {0.0, 0.0, 0.0, 0.0};
    long long l[2] = {0, 0};
    float mn = FLT_MAX, mx = -FLT_MAX, mx2 = 0.0f;

    if (I.kind == MC_K_MOMENTUM) {
        const TileRange tr = mom_range(I, t);
        const float *cur = (const float *)I.cur;
        const float *prev = I.prev;
        float *hist = (float *)I.hist_out;
        for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB) {
            const float c = cur[e];
            const float p = prev[e];
            d[0] += (double)fabsf(c);
            d[1] += (double)fabsf(p);
            mn = c < mn ? c : mn;
            mx = c > mx ? c : mx;
            if (hist) hist[e] = c;
        }
        // per-kernel sign consistency: one lane per kernel, 32 kernels per ballot word
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const float inv_ks = __fdiv_rn(1.0f, (float)I.ks);
        int P = 0;
        for (int64_t kb = tr.k0 + warp * 32; kb < tr.k1; kb += TPB) {
            const int64_t k = kb + lane;
            bool flag = false, dom = false;
            if (k < tr.k1) {
                const float *p = cur + k * I.ks;
                int pos = 0, neg = 0;
                for (int j = 0; j < I.ks; j++) {
                    const float v = p[j];
                    pos += v > 0.0f;
                    neg += v < 0.0f;
                }
                const int zero = I.ks - pos - neg;
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
        l[0] = P;
        block_reduce(red, d, 2, mn, mx, mx2, l, 1);
        if (threadIdx.x == 0) {
            mc_enc_tile &T = L.tiles[gt];
            T.s_cur = d[0];
            T.s_prev = d[1];
            T.mn = mn;
            T.mx = mx;
            T.P = (int32_t)l[0];
        }
        if (last_cta(&R->ticket[0], I.ntiles, &s_flag)) {
            double a[4] = {0.0, 0.0, 0.0, 0.0};
            long long z[2] = {0, 0};
            float tmn = FLT_MAX, tmx = -FLT_MAX, t2 = 0.0f;
            for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
                const mc_enc_tile *T = L.tiles + I.tile_base + i;
                a[0] += __ldcg(&T->s_cur);
                a[1] += __ldcg(&T->s_prev);
                const float tm = __ldcg(&T->mn), tx = __ldcg(&T->mx);
                tmn = tm < tmn ? tm : tmn;
                tmx = tx > tmx ? tx : tmx;
            }
            block_reduce(red, a, 2, tmn, tmx, t2, z, 0);
            if (threadIdx.x == 0) {
                const double dn = (double)I.n;
                R->cm = __double2float_rn(__ddiv_rn(a[0], dn));
                R->pm = __double2float_rn(__ddiv_rn(a[1], dn));
                R->gmin = tmn;
                R->gmax = tmx;
                long long off = 0;
                for (int i = 0; i < I.ntiles; i++) {
                    L.tile_poff[I.tile_base + i] = off;
                    off += __ldcg(&L.tiles[I.tile_base + i].P);
                }
                R->P = off;
            }
        }
        return;
    }

    // direct items: element tiles
    const int64_t e0 = (int64_t)t * I.tile_kernels;
    const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
    if (I.kind == MC_K_COPY) {
        // raw payload ("sz3_memcpy") and history copy; tiles count bytes
        const uint8_t *src = (const uint8_t *)I.cur;
        uint8_t *hist = (uint8_t *)I.hist_out;
        uint8_t *raw = I.data_out;
        for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
            const uint8_t v = src[e];
            raw[e] = v;
            if (hist) hist[e] = v;
        }
        return;
    }
    if (I.kind == MC_K_QUANT) {
        const float *cur = (const float *)I.cur;
        float *hist = (float *)I.hist_out;
        for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
            const float c = cur[e];
            mx2 = fmaxf(mx2, fabsf(c));
            if (hist) hist[e] = c;
        }
        block_reduce(red, d, 0, mn, mx, mx2, l, 0);
        if (threadIdx.x == 0) L.tiles[gt].maxr = mx2;
        if (last_cta(&R->ticket[0], I.ntiles, &s_flag)) {
            float m = 0.0f, u0 = FLT_MAX, u1 = -FLT_MAX;
            for (int i = threadIdx.x; i < I.ntiles; i += TPB)
                m = fmaxf(m, __ldcg(&L.tiles[I.tile_base + i].maxr));
            block_reduce(red, d, 0, u0, u1, m, l, 0);
            if (threadIdx.x == 0) {
                R->maxr = m;
                R->scale = (m == 0.0f) ? 1.0f : __fdiv_rn(m, (float)qmax_of(I.codec));
                if (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) {
                    *(float *)I.data_out = R->scale;
                }
            }
        }
        return;
    }
    if (I.kind == MC_K_FRAME && I.hist_out) {
        // element tiles in bytes for lossless payloads
        const uint8_t *src = (const uint8_t *)I.cur;
        uint8_t *dst = (uint8_t *)I.hist_out;
        for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) dst[e] = src[e];
    }
}

// ------------------------------------------------------------------ pass 2
__global__ void __launch_bounds__(TPB) k_enc_pass2(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ int s_flag;
    const int gt = L.mom_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_enc_item I = L.items[ii];
    const int t = gt - I.tile_base;
    mc_enc_result *R = L.results + ii;
    const TileRange tr = mom_range(I, t);
    const float cm = R->cm, pm = R->pm;
    const float *cur = (const float *)I.cur;
    const float *prev = I.prev;
    double d[4] = {0.0, 0.0, 0.0, 0.0};
    long long l[2] = {0, 0};
    float mn = FLT_MAX, mx = -FLT_MAX, mx2 = 0.0f;
    for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB) {
        const double dc = (double)__fsub_rn(fabsf(cur[e]), cm);
        const double dp = (double)__fsub_rn(fabsf(prev[e]), pm);
        d[0] = __fma_rn(dc, dc, d[0]);
        d[1] = __fma_rn(dp, dp, d[1]);
    }
    block_reduce(red, d, 2, mn, mx, mx2, l, 0);
    if (threadIdx.x == 0) {
        L.tiles[gt].v_cur = d[0];
        L.tiles[gt].v_prev = d[1];
    }
    if (last_cta(&R->ticket[1], I.ntiles, &s_flag)) {
        double a[4] = {0.0, 0.0, 0.0, 0.0};
        for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
            a[0] += __ldcg(&L.tiles[I.tile_base + i].v_cur);
            a[1] += __ldcg(&L.tiles[I.tile_base + i].v_prev);
        }
        block_reduce(red, a, 2, mn, mx, mx2, l, 0);
        if (threadIdx.x == 0) {
            const double dn = (double)I.n;
            const float cs = __fsqrt_rn(__double2float_rn(__ddiv_rn(a[0], dn)));
            const float ps = __fsqrt_rn(__double2float_rn(__ddiv_rn(a[1], dn)));
            R->cs = cs;
            R->ps = ps;
            R->inv_ps = (ps > 1e-8f) ? __fdiv_rn(1.0f, ps) : 1.0f;
        }
    }
}

// ------------------------------------------------------------------ pass 3
__global__ void __launch_bounds__(TPB) k_enc_pass3(mc_enc_launch L) {
    __shared__ Red red;
    __shared__ int s_flag;
    const int gt = L.mom_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_enc_item I = L.items[ii];
    const int t = gt - I.tile_base;
    mc_enc_result *R = L.results + ii;
    const TileRange tr = mom_range(I, t);
    const float cm = R->cm, cs = R->cs, pm = R->pm, inv_ps = R->inv_ps;
    const bool use_ps = R->ps > 1e-8f;
    const MomParams mp = {cm, cs, R->gmin, R->gmax, cs > 1e-8f};
    const float lr = I.lr;
    const float oml = __fsub_rn(1.0f, lr);
    const float *cur = (const float *)I.cur;
    const float *prev = I.prev;
    const float *mem_in = I.mem_in;
    float *mem_out = I.mem_out;
    long long mism = 0;
    float maxr = 0.0f;
    const uint32_t k0 = (uint32_t)tr.k0;
    for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB) {
        const uint32_t k = k0 + fdiv32((uint32_t)(e - tr.e0), I.ksdiv);
        const bool f = (I.bm_words[k >> 5] >> (k & 31)) & 1u;
        const float c = cur[e];
        const float m0 = mem_in ? mem_in[e] : 0.0f;
        float r;
        if (f) {
            const bool pos = (I.dom_words[k >> 5] >> (k & 31)) & 1u;
            const float pv = __fsub_rn(fabsf(prev[e]), pm);
            const float pn = use_ps ? __fmul_rn(pv, inv_ps) : pv;
            const float nm = __fmaf_rn(oml, m0, __fmul_rn(lr, pn));
            mem_out[e] = nm;
            r = mom_residual(c, nm, pos, mp);
            const float ap = fabsf(mp.use_cs ? __fmaf_rn(nm, cs, cm) : __fadd_rn(nm, cm));
            const float pred = pos ? ap : -ap;
            mism += (pred > 0.0f) != (c > 0.0f);
        } else {
            mem_out[e] = m0;
            r = c;
        }
        maxr = fmaxf(maxr, fabsf(r));
    }
    double d[4];
    long long l[2] = {mism, 0};
    float mn = FLT_MAX, mx = -FLT_MAX;
    block_reduce(red, d, 0, mn, mx, maxr, l, 1);
    if (threadIdx.x == 0) {
        L.tiles[gt].maxr = maxr;
        L.tiles[gt].mism = l[0];
    }
    if (last_cta(&R->ticket[2], I.ntiles, &s_flag)) {
        float m = 0.0f;
        long long z[2] = {0, 0};
        for (int i = threadIdx.x; i < I.ntiles; i += TPB) {
            m = fmaxf(m, __ldcg(&L.tiles[I.tile_base + i].maxr));
            z[0] += __ldcg(&L.tiles[I.tile_base + i].mism);
        }
        block_reduce(red, d, 0, mn, mx, m, z, 1);
        if (threadIdx.x == 0) {
            R->maxr = m;
            R->mism = z[0];
            R->scale = (m == 0.0f) ? 1.0f : __fdiv_rn(m, (float)qmax_of(I.codec));
            if (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) *(float *)I.data_out = R->scale;
        }
    }
}

// Software parallel-bit-extract: the bits of `v` at the set positions of
// `m`, packed towards bit 0 in ascending position order.
__device__ __forceinline__ uint32_t pext32(uint32_t v, uint32_t m) {
    uint32_t out = 0;
    int j = 0;
    while (m) {
        const int b = __ffs(m) - 1;
        out |= ((v >> b) & 1u) << j;
        j++;
        m &= m - 1;
    }
    return out;
}

// ------------------------------------------------------------------ pass 4
__global__ void __launch_bounds__(TPB) k_enc_pass4(mc_enc_launch L) {
    __shared__ int scan_sh[NWARP + 1];
    const int gt = L.all_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_enc_item I = L.items[ii];
    const int t = gt - I.tile_base;
    const mc_enc_result *R = L.results + ii;
    if (I.kind == MC_K_MOMENTUM) {
        const TileRange tr = mom_range(I, t);
        const MomParams mp = {R->cm, R->cs, R->gmin, R->gmax, R->cs > 1e-8f};
        const float scale = R->scale;
        const float qm = (float)qmax_of(I.codec);
        const float *cur = (const float *)I.cur;
        const float *mem = I.mem_out;
        const uint32_t k0 = (uint32_t)tr.k0;
        auto resid = [&](int64_t e) -> float {
            const uint32_t k = k0 + fdiv32((uint32_t)(e - tr.e0), I.ksdiv);
            const uint32_t bw = I.bm_words[k >> 5];
            const float c = cur[e];
            if (!((bw >> (k & 31)) & 1u)) return c;
            const bool pos = (I.dom_words[k >> 5] >> (k & 31)) & 1u;
            return mom_residual(c, mem[e], pos, mp);
        };
        if (I.codec == MC_DC_RAW) {
            float *out = (float *)I.data_out;
            for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB) out[e] = resid(e);
        } else if (I.codec == MC_DC_Q8) {
            // four codes per 32-bit store; tiles start at multiples of 4 elements
            uint8_t *codes = I.data_out + 4;
            for (int64_t g = tr.e0 + 4 * (int64_t)threadIdx.x; g < tr.e1; g += 4 * TPB) {
                uint32_t word = 0;
                for (int j = 0; j < 4; j++) {
                    if (g + j < tr.e1) {
                        const int q = quant1(resid(g + j), scale, qm);
                        word |= ((uint32_t)(uint8_t)(int8_t)q) << (8 * j);
                    }
                }
                if (g + 3 < tr.e1) {
                    *(uint32_t *)(codes + g) = word;
                } else {
                    for (int j = 0; g + j < tr.e1; j++) codes[g + j] = (uint8_t)(word >> (8 * j));
                }
            }
        } else if (I.codec == MC_DC_INT4) {
            uint8_t *packed = I.data_out + 4;
            for (int64_t p = (tr.e0 >> 1) + threadIdx.x; 2 * p < tr.e1; p += TPB) {
                const int lo = quant1(resid(2 * p), scale, qm) + 8;
                const int hi = (2 * p + 1 < tr.e1) ? quant1(resid(2 * p + 1), scale, qm) + 8 : 0;
                packed[p] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            }
        } else {  // Q8_RAW / INT4_RAW: dequantised floats
            float *out = (float *)I.data_out;
            for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB)
                out[e] = __fmul_rn((float)quant1(resid(e), scale, qm), scale);
        }
        // dense dominant signs of predicted kernels (ref :2258-2283)
        const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
        const int i = threadIdx.x;
        uint32_t m = 0, dv = 0;
        if (wb + i < we) {
            m = I.bm_words[wb + i];
            dv = I.dom_words[wb + i];
        }
        const int pc = __popc(m);
        const int off_l = block_excl_scan(pc, scan_sh, nullptr);
        if (pc) {
            const int64_t off = L.tile_poff[gt] + off_l;
            const uint32_t bits = pext32(dv, m);
            const int64_t w0 = off >> 5;
            const int sh = (int)(off & 31);
            atomicOr(&I.sign_words[w0], bits << sh);
            if (sh + pc > 32) atomicOr(&I.sign_words[w0 + 1], bits >> (32 - sh));
        }
        return;
    }
    if (I.kind == MC_K_QUANT) {
        const int64_t e0 = (int64_t)t * I.tile_kernels;
        const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
        const float *cur = (const float *)I.cur;
        const float scale = R->scale;
        const float qm = (float)qmax_of(I.codec);
        if (I.codec == MC_DC_Q8) {
            int8_t *codes = (int8_t *)(I.data_out + 4);
            for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) codes[e] = (int8_t)quant1(cur[e], scale, qm);
        } else if (I.codec == MC_DC_INT4) {
            uint8_t *packed = I.data_out + 4;
            for (int64_t p = (e0 >> 1) + threadIdx.x; 2 * p < e1; p += TPB) {
                const int lo = quant1(cur[2 * p], scale, qm) + 8;
                const int hi = (2 * p + 1 < e1) ? quant1(cur[2 * p + 1], scale, qm) + 8 : 0;
                packed[p] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            }
        } else {
            float *out = (float *)I.data_out;
            for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB)
                out[e] = __fmul_rn((float)quant1(cur[e], scale, qm), scale);
        }
    }
}

// ------------------------------------------------------------------ frames
// zstd frame (RFC 8878) with a single-segment header, 4- or 8-byte content
// size, and Raw / RLE blocks of at most 128 KiB.
__global__ void __launch_bounds__(TPB) k_frames(const mc_frame_job *jobs) {
    const mc_frame_job &J = jobs[blockIdx.x];
    int64_t size = J.size;
    if (size < 0) {
        const int64_t P = *J.P_src;
        if (P == 0) {
            if (threadIdx.x == 0) *J.size_out = 0;
            return;
        }
        size = (P + 7) >> 3;
    }
    uint8_t *dst = J.dst;
    const bool big = size >= (int64_t)0xFFFFFFFFll;
    int64_t pos = big ? 13 : 9;
    if (threadIdx.x == 0) {
        dst[0] = 0x28; dst[1] = 0xB5; dst[2] = 0x2F; dst[3] = 0xFD;
        dst[4] = big ? 0xE0 : 0xA0;   // FCS flag 3/2, single segment
        const int nb = big ? 8 : 4;
        for (int i = 0; i < nb; i++) dst[5 + i] = (uint8_t)((uint64_t)size >> (8 * i));
    }
    const int64_t nblk = size == 0 ? 1 : (size + ZBLOCK - 1) / ZBLOCK;
    for (int64_t b = 0; b < nblk; b++) {
        const int64_t bs = min((int64_t)ZBLOCK, size - b * ZBLOCK);
        const uint8_t *src = J.src + b * ZBLOCK;
        int eq = 1;
        if (bs > 1) {
            const uint8_t first = src[0];
            for (int64_t i = threadIdx.x; i < bs; i += TPB) eq &= (src[i] == first);
        }
        const int rle = (bs > 1) && __syncthreads_and(eq);
        const uint32_t last = (b == nblk - 1) ? 1u : 0u;
        const uint32_t hdr = last | ((uint32_t)(rle ? 1 : 0) << 1) | ((uint32_t)bs << 3);
        if (threadIdx.x == 0) {
            dst[pos] = (uint8_t)hdr;
            dst[pos + 1] = (uint8_t)(hdr >> 8);
            dst[pos + 2] = (uint8_t)(hdr >> 16);
            if (rle) dst[pos + 3] = src[0];
        }
        if (!rle) {
            uint8_t *o = dst + pos + 3;
            for (int64_t i = threadIdx.x; i < bs; i += TPB) o[i] = src[i];
            pos += 3 + bs;
        } else {
            pos += 4;
        }
    }
    if (threadIdx.x == 0) *J.size_out = pos;
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
            for (int64_t i = threadIdx.x; i < s_len[s]; i += TPB) o[i] = src[i];
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

__global__ void __launch_bounds__(TPB) k_dec_prefix(mc_dec_launch L) {
    __shared__ long long sh[NWARP];
    __shared__ int s_flag;
    const int gt = L.mom_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_dec_item I = L.items[ii];
    const int t = gt - I.tile_base;
    mc_dec_result *R = L.results + ii;
    const DecTile tr = dec_range(I, t);
    const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
    const int64_t bm_bits = dec_bm_bits(I);
    int c = 0;
    for (int64_t w = wb + threadIdx.x; w < we; w += TPB) c += __popc(I.bm_words[w] & word_mask(w, bm_bits));
    long long v = warp_sum_ll(c);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long s = 0;
        for (int j = 0; j < NWARP; j++) s += sh[j];
        L.tile_count[gt] = (int32_t)s;
    }
    if (last_cta(&R->ticket, I.ntiles, &s_flag) && threadIdx.x == 0) {
        long long off = 0;
        for (int i = 0; i < I.ntiles; i++) {
            L.tile_poff[I.tile_base + i] = off;
            off += __ldcg(&L.tile_count[I.tile_base + i]);
        }
        R->P = off;
    }
}

__device__ __forceinline__ float dec_resid(const mc_dec_item &I, int64_t e, float scale) {
    if (I.codec == MC_DC_Q8) return __fmul_rn((float)(int8_t)I.data[e], scale);
    if (I.codec == MC_DC_INT4) {
        const uint8_t b = I.data[e >> 1];
        const int q = (int)((e & 1) ? (b >> 4) : (b & 15)) - 8;
        return __fmul_rn((float)q, scale);
    }
    return ((const float *)I.data)[e];
}

__global__ void __launch_bounds__(TPB) k_dec_recon(mc_dec_launch L) {
    __shared__ uint32_t s_m[TPB], s_d[TPB];
    __shared__ int scan_sh[NWARP + 1];
    const int gt = L.all_tiles[blockIdx.x];
    const int ii = L.tile_item[gt];
    const mc_dec_item I = L.items[ii];
    const int t = gt - I.tile_base;
    const float scale = (I.codec == MC_DC_Q8 || I.codec == MC_DC_INT4) ? *I.scale_ptr : 1.0f;
    float *hist = (float *)I.hist_out;
    float *out = (float *)I.out;
    if (I.kind == MC_D_MOMENTUM) {
        const DecTile tr = dec_range(I, t);
        const int64_t wb = tr.k0 >> 5, we = (tr.k1 + 31) >> 5;
        const int i = threadIdx.x;
        const int64_t bm_bits = dec_bm_bits(I);
        const uint8_t *sg = I.sg_bytes;
        int64_t sg_len = I.sg_len;
        if (I.sg_len_ptr) {
            sg_len = *I.sg_len_ptr;
            if (sg_len < 0) sg = nullptr;
        }
        uint32_t m = 0;
        if (wb + i < we) m = I.bm_words[wb + i] & word_mask(wb + i, bm_bits);
        const int pc = __popc(m);
        const int off_l = block_excl_scan(pc, scan_sh, nullptr);
        uint32_t dm = 0;
        if (pc) {
            int64_t idx = L.tile_poff[gt] + off_l;
            uint32_t mm = m;
            while (mm) {
                const int b = __ffs(mm) - 1;
                int bit = 1;
                if (sg && (idx >> 3) < sg_len) bit = (sg[idx >> 3] >> (idx & 7)) & 1;
                dm |= (uint32_t)bit << b;
                idx++;
                mm &= mm - 1;
            }
        }
        s_m[i] = m;
        s_d[i] = dm;
        __syncthreads();
        const float cm = I.cm, cs = I.cs, pm = I.pm, lr = I.lr;
        const bool use_cs = cs > 1e-8f, use_ps = I.ps > 1e-8f;
        const float inv_ps = use_ps ? __fdiv_rn(1.0f, I.ps) : 1.0f;
        const float oml = __fsub_rn(1.0f, lr);
        const uint32_t k0 = (uint32_t)tr.k0;
        for (int64_t e = tr.e0 + threadIdx.x; e < tr.e1; e += TPB) {
            const uint32_t k = k0 + fdiv32((uint32_t)(e - tr.e0), I.ksdiv);
            const uint32_t lw = (k >> 5) - (uint32_t)wb;
            const bool f = (s_m[lw] >> (k & 31)) & 1u;
            const float r = dec_resid(I, e, scale);
            const float m0 = I.mem_in ? I.mem_in[e] : 0.0f;
            float rec;
            if (f) {
                const bool pos = (s_d[lw] >> (k & 31)) & 1u;
                const float pv = __fsub_rn(fabsf(I.prev[e]), pm);
                const float pn = use_ps ? __fmul_rn(pv, inv_ps) : pv;
                const float nm = __fmaf_rn(oml, m0, __fmul_rn(lr, pn));
                I.mem_out[e] = nm;
                float ap = use_cs ? __fmaf_rn(nm, cs, cm) : __fadd_rn(nm, cm);
                ap = fabsf(ap);
                rec = __fadd_rn(r, pos ? ap : -ap);
            } else {
                I.mem_out[e] = m0;
                rec = r;
            }
            hist[e] = rec;
            if (out) out[e] = rec;
        }
        return;
    }
    const int64_t e0 = (int64_t)t * I.tile_kernels;
    const int64_t e1 = min(e0 + (int64_t)I.tile_kernels, I.n);
    if (I.kind == MC_D_RESIDUAL || I.kind == MC_D_QUANT) {
        for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
            const float r = dec_resid(I, e, scale);
            hist[e] = r;
            if (out) out[e] = r;
        }
        return;
    }
    // MC_D_COPY: bytes (tile in bytes)
    const uint8_t *src = I.data;
    uint8_t *h8 = (uint8_t *)I.hist_out, *o8 = (uint8_t *)I.out;
    for (int64_t e = e0 + threadIdx.x; e < e1; e += TPB) {
        const uint8_t v = src[e];
        h8[e] = v;
        if (o8) o8[e] = v;
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

extern "C" int mc_launch_encode(const mc_enc_launch *L, void *stream, mc_ktrace *tr) {
    cudaStream_t s = (cudaStream_t)stream;
    int n = 0;
    if (L->nall_tiles > 0) {
        tr_begin(tr, MC_KT_ENC_PASS1, s);
        k_enc_pass1<<<L->nall_tiles, TPB, 0, s>>>(*L);
        tr_end(tr, s);
        n++;
    }
    if (L->nmom_tiles > 0) {
        tr_begin(tr, MC_KT_ENC_PASS2, s);
        k_enc_pass2<<<L->nmom_tiles, TPB, 0, s>>>(*L);
        tr_end(tr, s);
        tr_begin(tr, MC_KT_ENC_PASS3, s);
        k_enc_pass3<<<L->nmom_tiles, TPB, 0, s>>>(*L);
        tr_end(tr, s);
        n += 2;
    }
    if (L->nall_tiles > 0) {
        tr_begin(tr, MC_KT_ENC_PASS4, s);
        k_enc_pass4<<<L->nall_tiles, TPB, 0, s>>>(*L);
        tr_end(tr, s);
        n++;
    }
    if (L->nframes > 0) {
        tr_begin(tr, MC_KT_FRAMES, s);
        k_frames<<<L->nframes, TPB, 0, s>>>(L->frames);
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
        k_dec_prefix<<<L->nmom_tiles, TPB, 0, s>>>(*L);
        tr_end(tr, s);
        n++;
    }
    if (L->nall_tiles > 0) {
        tr_begin(tr, MC_KT_DEC_RECON, s);
        k_dec_recon<<<L->nall_tiles, TPB, 0, s>>>(*L);
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
