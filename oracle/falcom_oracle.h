/*
 * falcom_oracle.h -- CPU restatement of the FalCom momentum codec numerics.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker used by tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline leg.  The product
 * (compressor_b200/libmomentum_compressor.so) never links, loads or calls it.
 *
 * Every routine restates one step of the reference grouped OpenMP/SIMD codec
 * (momentum_compressor_openmp_simd_final.c) or of the reference GPU
 * quantisers (cuda_feasibility/falcom_cuda_v4, falcom_cuda_v3), with the same
 * floating-point operation order that the reference build
 * (-O3 -ffast-math, FMA contraction on) produces.  Parity of this restatement
 * is pinned against the reference library built from its own sources
 * (oracle/_ref) and against the golden vectors in tests/golden/.
 */
#ifndef FALCOM_ORACLE_H
#define FALCOM_ORACLE_H
#include <stdint.h>
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float cur_mean, cur_std;     /* mean / population std of |cur|  */
    float prev_mean, prev_std;   /* mean / population std of |prev| */
    float gmin, gmax;            /* raw min / max of cur            */
    int64_t predicted;           /* kernels whose bitmap bit is set */
    int64_t mismatches;          /* sign mismatches over predicted elements */
    int64_t predicted_elems;     /* elements inside predicted kernels       */
    float prediction_ratio;
    float sign_mismatch_ratio;
} fo_layer_stats;

/* Triple statistics: momentum_compressor_openmp_simd_final.c:1322-1431. */
void fo_triple_stats(const float *cur, const float *prev, int64_t n, fo_layer_stats *st);

/* Per-kernel sign consistency: :1438-1476 (+ loop :2040-2062).
 * Writes one flag byte (0/1) and one dominant sign (+1/-1) per kernel. */
int64_t fo_sign_consistency(const float *cur, int64_t n_kernels, int64_t ks, float threshold,
                            uint8_t *flags, int8_t *dom);

/* Full encoder step for one 4-D momentum layer: :1859-2318.
 *   mem        in/out prediction memory (n floats; zeros when newly created)
 *   residual   out, n floats (the payload before the residual codec)
 *   bitmap     out, ceil(K/8) bytes, LSB-first (:2222-2253)
 *   signs      out, ceil(K/8) bytes capacity; ceil(P/8) bytes used (:2258-2283)
 * Returns ceil(P/8), the number of sign bytes written (0 when P == 0). */
int64_t fo_encode_momentum(const float *cur, const float *prev, float *mem,
                           int64_t out_ch, int64_t in_ch, int64_t ks, int step,
                           float lr, float threshold,
                           float *residual, uint8_t *bitmap, uint8_t *signs,
                           fo_layer_stats *st);

/* Decoder step for one momentum_predicted layer: :3186-3474.
 *   residual      n floats (already decoded from the residual codec)
 *   bitmap/signs  packed content (zstd already removed)
 *   prev_dec      decoder-side history head (NULL when missing)
 *   mem           in/out decoder prediction memory
 *   recon         out, n floats
 * Return value mirrors the reference's early exits:
 *   0 = full reconstruction (caller appends recon to history),
 *   1 = residual returned as-is, history NOT appended (no bitmap, P == 0,
 *       or no history), memory untouched. */
int fo_decode_momentum(const float *residual, const uint8_t *bitmap, int64_t bitmap_bytes,
                       const uint8_t *signs, int64_t sign_bytes,
                       const float *prev_dec, float *mem,
                       int64_t out_ch, int64_t in_ch, int64_t ks,
                       float cur_mean, float cur_std, float prev_mean, float prev_std,
                       float lr, float *recon);

/* Symmetric residual quantiser (q8: falcom_cuda_v4_kernels.cu:53-65,182;
 * int4: falcom_cuda_v3_wrapper.py:133-149).  qmax = 127 or 7.
 * Returns the scale (max|x| / qmax, or 1 when max|x| == 0). */
float fo_quantize(const float *x, int64_t n, int qmax, int8_t *codes);
/* out[i] = (float)codes[i] * scale   (falcom_cuda_v4_kernels.cu:67-77) */
void fo_dequantize(const int8_t *codes, int64_t n, float scale, float *out);
/* int4 packing: (q+8) nibbles, element 2i in the low nibble
 * (falcom_cuda_v3_wrapper.py:159-166 / 169-177). */
void fo_pack_int4(const int8_t *codes, int64_t n, uint8_t *out);
void fo_unpack_int4(const uint8_t *packed, int64_t n, int8_t *codes);

/* LSB-first bit packing of 0/1 flags (:2240-2242). */
void fo_pack_bits(const uint8_t *flags, int64_t n, uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif
