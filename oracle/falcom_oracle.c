/*
 * falcom_oracle.c -- CPU restatement of the FalCom momentum codec numerics.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and the CPU
 * baseline.  The shipped library never links or calls this file.
 *
 * Built with -ffp-contract=off; every fused multiply-add that the reference
 * build contracts is written here as an explicit fmaf()/fma(), and every
 * separate multiply/add stays separate, so each float result has the same
 * rounding as the reference build of momentum_compressor_openmp_simd_final.c
 * (-O3 -ffast-math; the contraction choices were read from the x86-64
 * assembly of that file compiled here from source).
 */
#include "falcom_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* x86 maxss/minss semantics, which the reference's fmaxf/fminf compile to
 * under -ffast-math: the second operand is returned unless the first one is
 * strictly larger (smaller). */
static inline float x86_max(float a, float b) { return a > b ? a : b; }
static inline float x86_min(float a, float b) { return a < b ? a : b; }

/* momentum_compressor_openmp_simd_final.c:1322-1431
 * Pass 1: double sums of |cur| and |prev|, raw min/max of cur.
 * Pass 2: double sum of squares of the float difference |x| - mean. */
void fo_triple_stats(const float *cur, const float *prev, int64_t n, fo_layer_stats *st) {
    double sc = 0.0, sp = 0.0;
    float mn = FLT_MAX, mx = -FLT_MAX;
    for (int64_t i = 0; i < n; i++) {
        float c = cur[i];
        sc += (double)fabsf(c);
        sp += (double)fabsf(prev[i]);
        if (c < mn) mn = c;
        if (c > mx) mx = c;
    }
    double dn = (double)n;
    float cm = (float)(sc / dn);
    float pm = (float)(sp / dn);
    double vc = 0.0, vp = 0.0;
    for (int64_t i = 0; i < n; i++) {
        double dc = (double)(fabsf(cur[i]) - cm);   /* float subtraction, then widen */
        double dp = (double)(fabsf(prev[i]) - pm);
        vc = fma(dc, dc, vc);
        vp = fma(dp, dp, vp);
    }
    st->cur_mean = cm;
    st->prev_mean = pm;
    st->cur_std = sqrtf((float)(vc / dn));
    st->prev_std = sqrtf((float)(vp / dn));
    st->gmin = mn;
    st->gmax = mx;
}

/* :1438-1476 compute_sign_info_fused, called per kernel from :2046-2060.
 * consistency = ((float)majority * (1/ks) - 0.5) * 2 with the multiply-add
 * fused, 1/ks computed once per layer (reciprocal hoisting under
 * -ffast-math); predicted iff consistency >= threshold; zeros count toward
 * the majority; dominant sign +1 on ties. */
int64_t fo_sign_consistency(const float *cur, int64_t n_kernels, int64_t ks, float threshold,
                            uint8_t *flags, int8_t *dom) {
    int64_t predicted = 0;
    float inv_ks = 1.0f / (float)ks;
    for (int64_t k = 0; k < n_kernels; k++) {
        const float *p = cur + k * ks;
        int64_t pos = 0, neg = 0, zero = 0;
        for (int64_t j = 0; j < ks; j++) {
            if (p[j] > 0.0f) pos++;
            else if (p[j] < 0.0f) neg++;
            else zero++;
        }
        int64_t maj = (pos >= neg) ? (pos + zero) : (neg + zero);
        float half = fmaf((float)maj, inv_ks, -0.5f);
        float cons = half + half;
        flags[k] = (cons >= threshold) ? 1 : 0;
        dom[k] = (pos >= neg) ? 1 : -1;
        predicted += flags[k];
    }
    return predicted;
}

void fo_pack_bits(const uint8_t *flags, int64_t n, uint8_t *out) {
    int64_t nbytes = (n + 7) / 8;
    memset(out, 0, (size_t)nbytes);
    for (int64_t i = 0; i < n; i++) {
        if (flags[i]) out[i >> 3] |= (uint8_t)(1u << (i & 7));
    }
}

/* :1859-2318 compress_conv_layer_momentum (everything except the residual
 * codec and the zstd framing of bitmap / signs). */
int64_t fo_encode_momentum(const float *cur, const float *prev, float *mem,
                           int64_t out_ch, int64_t in_ch, int64_t ks, int step,
                           float lr, float threshold,
                           float *residual, uint8_t *bitmap, uint8_t *signs,
                           fo_layer_stats *st) {
    const int64_t K = out_ch * in_ch;
    const int64_t n = K * ks;
    fo_triple_stats(cur, prev, n, st);

    /* :1937-1955 normalisation of |prev| (reciprocal of the std, then multiply) */
    const float pm = st->prev_mean;
    const int prev_use_std = st->prev_std > 1e-8f;
    const float inv_ps = prev_use_std ? (1.0f / st->prev_std) : 1.0f;

    /* :2040-2062 sign consistency: per-kernel flags and dominant signs */
    uint8_t *f = (uint8_t *)malloc((size_t)(K > 0 ? K : 1));
    int8_t *d = (int8_t *)malloc((size_t)(K > 0 ? K : 1));
    int64_t P = fo_sign_consistency(cur, K, ks, threshold, f, d);
    st->predicted = P;
    st->prediction_ratio = (float)P / (float)K;

    /* :2088 residual defaults to the input; :2094-2170 prediction loop */
    memcpy(residual, cur, (size_t)n * sizeof(float));
    int64_t mism = 0, pelems = 0;
    if (P > 0 && step > 0) {
        const float one_minus_lr = 1.0f - lr;
        const float cs = st->cur_std, cm = st->cur_mean;
        const int cur_use_std = cs > 1e-8f;
        for (int64_t k = 0; k < K; k++) {
            if (!f[k]) continue;
            const float sign = (float)d[k];
            for (int64_t j = 0; j < ks; j++) {
                const int64_t i = k * ks + j;
                float pv = fabsf(prev[i]) - pm;
                float pn = prev_use_std ? pv * inv_ps : pv;
                float nm = fmaf(one_minus_lr, mem[i], lr * pn);
                mem[i] = nm;
                float ap = cur_use_std ? fmaf(nm, cs, cm) : (nm + cm);
                ap = fabsf(ap);
                float pred = sign * ap;
                if ((pred > 0.0f) != (cur[i] > 0.0f)) mism++;
                pelems++;
                float r = cur[i] - pred;
                r = x86_min(x86_max(r, st->gmin), st->gmax);
                residual[i] = r;
            }
        }
    }
    st->mismatches = mism;
    st->predicted_elems = pelems;
    st->sign_mismatch_ratio = pelems > 0 ? (float)mism / (float)pelems : 0.0f;

    /* :2222-2253 bitmap, :2258-2283 dominant signs of predicted kernels */
    fo_pack_bits(f, K, bitmap);
    int64_t sign_bytes = 0;
    if (P > 0) {
        sign_bytes = (P + 7) / 8;
        memset(signs, 0, (size_t)sign_bytes);
        int64_t pi = 0;
        for (int64_t k = 0; k < K; k++) {
            if (!f[k]) continue;
            if (d[k] > 0) signs[pi >> 3] |= (uint8_t)(1u << (pi & 7));
            pi++;
        }
    }
    free(f);
    free(d);
    return sign_bytes;
}

/* :3186-3474 decompress_momentum_predicted_layer */
int fo_decode_momentum(const float *residual, const uint8_t *bitmap, int64_t bitmap_bytes,
                       const uint8_t *signs, int64_t sign_bytes,
                       const float *prev_dec, float *mem,
                       int64_t out_ch, int64_t in_ch, int64_t ks,
                       float cur_mean, float cur_std, float prev_mean, float prev_std,
                       float lr, float *recon) {
    const int64_t K = out_ch * in_ch;
    const int64_t n = K * ks;
    memcpy(recon, residual, (size_t)n * sizeof(float));
    if (!bitmap || bitmap_bytes == 0) return 1;                  /* :3227-3230 */
    int64_t safe_bits = bitmap_bytes * 8 < K ? bitmap_bytes * 8 : K;
    int64_t P = 0;
    for (int64_t k = 0; k < safe_bits; k++) P += (bitmap[k >> 3] >> (k & 7)) & 1;
    if (P == 0) return 1;                                         /* :3266-3269 */
    int8_t *dom = NULL;
    if (signs && sign_bytes > 0) {                                /* :3272-3310 */
        dom = (int8_t *)malloc((size_t)K);
        memset(dom, 0, (size_t)K);
        int64_t pi = 0;
        for (int64_t k = 0; k < safe_bits; k++) {
            if (!((bitmap[k >> 3] >> (k & 7)) & 1)) continue;
            if ((pi >> 3) < sign_bytes) dom[k] = ((signs[pi >> 3] >> (pi & 7)) & 1) ? 1 : -1;
            else dom[k] = 1;
            pi++;
        }
    }
    if (!prev_dec) { free(dom); return 1; }                       /* :3320-3329 */
    /* :3351-3356 decoder-side normalisation: reciprocal hoisted, multiply */
    const int prev_use_std = prev_std > 1e-8f;
    const float inv_ps = prev_use_std ? (1.0f / prev_std) : 1.0f;
    const float one_minus_lr = 1.0f - lr;
    const int cur_use_std = cur_std > 1e-8f;
    for (int64_t k = 0; k < safe_bits; k++) {                     /* :3394-3434 */
        if (!((bitmap[k >> 3] >> (k & 7)) & 1)) continue;
        for (int64_t j = 0; j < ks; j++) {
            const int64_t i = k * ks + j;
            float pv = fabsf(prev_dec[i]) - prev_mean;
            float pn = prev_use_std ? pv * inv_ps : pv;
            float nm = fmaf(one_minus_lr, mem[i], lr * pn);
            mem[i] = nm;
            float ap = cur_use_std ? fmaf(nm, cur_std, cur_mean) : (nm + cur_mean);
            ap = fabsf(ap);
            if (dom) recon[i] = fmaf((float)dom[k], ap, residual[i]);
            else recon[i] = ap + residual[i];
        }
    }
    free(dom);
    return 0;
}

/* falcom_cuda_v4_kernels.cu:53-65 (+ scale rule :178-182) for qmax = 127;
 * falcom_cuda_v3_wrapper.py:133-149 for qmax = 7.  IEEE division and
 * round-half-to-even. */
float fo_quantize(const float *x, int64_t n, int qmax, int8_t *codes) {
    float mx = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        float a = fabsf(x[i]);
        if (a > mx) mx = a;
    }
    float scale = (mx == 0.0f) ? 1.0f : mx / (float)qmax;
    const float q = (float)qmax;
    for (int64_t i = 0; i < n; i++) {
        float v = rintf(x[i] / scale);
        v = fminf(q, fmaxf(-q, v));
        codes[i] = (int8_t)v;
    }
    return scale;
}

void fo_dequantize(const int8_t *codes, int64_t n, float scale, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = (float)codes[i] * scale;
}

void fo_pack_int4(const int8_t *codes, int64_t n, uint8_t *out) {
    for (int64_t i = 0; i < (n + 1) / 2; i++) {
        uint8_t lo = (uint8_t)(codes[2 * i] + 8) & 0x0F;
        uint8_t hi = (2 * i + 1 < n) ? ((uint8_t)(codes[2 * i + 1] + 8) & 0x0F) : 0;
        out[i] = (uint8_t)(lo | (hi << 4));
    }
}

void fo_unpack_int4(const uint8_t *packed, int64_t n, int8_t *codes) {
    for (int64_t i = 0; i < n; i++) {
        uint8_t b = packed[i >> 1];
        uint8_t nib = (i & 1) ? (b >> 4) : (b & 0x0F);
        codes[i] = (int8_t)((int)nib - 8);
    }
}
