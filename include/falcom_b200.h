/*
 * falcom_b200.h -- extension entry points of the B200 FalCom codec.
 *
 * None of these exist in the reference interface; a caller that only uses
 * momentum_compressor.h (for example EB-FaLCom's FalComC.py) gets the
 * defaults listed here, which can also be set through environment variables
 * read at momentum_compressor_create():
 *
 *   FALCOM_RESIDUAL_CODEC = q8 | int4 | raw | q8_raw | int4_raw   (default q8)
 *   FALCOM_FRAME_MODE     = gpu | libzstd                          (default gpu)
 */
#ifndef FALCOM_B200_H
#define FALCOM_B200_H

#include "momentum_compressor.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Residual codec: where the reference runs SZ3 (momentum residual with an ABS
 * bound, direct lossy tensors with a REL bound), this codec runs a symmetric
 * quantiser.
 *   "q8"       codec tag "q8":   [f32 scale][int8 code x n]
 *   "int4"     codec tag "int4": [f32 scale][(q+8) nibbles, element 2i low]
 *   "raw"      codec tag "sz3_memcpy": raw fp32 (what the reference emits
 *              when SZ3 is unavailable); bit-comparable with the reference
 *   "q8_raw" / "int4_raw"  quantise, then store the dequantised fp32 values
 *              with codec tag "sz3_memcpy" so an unmodified reference decoder
 *              reads them.
 * Returns 0, or ERROR_INVALID_PARAM for an unknown name. */
int falcom_set_residual_codec(MomentumCompressor *mc, const char *codec);

/* zstd framing of bitmap / dominant-sign / lossless payloads.
 *   "gpu"      frames written on the GPU with Raw and RLE blocks only
 *              (RFC 8878); every zstd decoder, the reference's included,
 *              reads them.
 *   "libzstd"  host libzstd level 10, byte-identical to the reference's
 *              frames (reference momentum_compressor_openmp_simd_final.c:647). */
int falcom_set_frame_mode(MomentumCompressor *mc, const char *mode);

/* Where returned payloads / decoded arrays live.
 *   FALCOM_LOC_AUTO    same memory kind as the inputs of the call
 *   FALCOM_LOC_HOST    host memory (pinned, owned by the library)
 *   FALCOM_LOC_DEVICE  device memory of the instance's GPU
 * Device-resident CompressedLayerData / NDArray are released with the same
 * compressed_layer_data_free() / ndarray_destroy(). */
enum { FALCOM_LOC_AUTO = 0, FALCOM_LOC_HOST = 1, FALCOM_LOC_DEVICE = 2 };
int falcom_set_payload_location(MomentumCompressor *mc, int loc);
int falcom_set_output_location(MomentumCompressor *mc, int loc);

/* CUDA stream (cudaStream_t) the instance issues its work on; NULL selects
 * the instance's own stream.  Calls remain synchronous with the host. */
int falcom_set_stream(MomentumCompressor *mc, void *stream);

/* Device ordinal the instance was created on. */
int falcom_get_device(const MomentumCompressor *mc);

/* Last error message of the instance ("" when none). */
const char *falcom_last_error(const MomentumCompressor *mc);

/* Kernel launches issued by the last compress / decompress call, and the
 * number issued since the instance was created. */
int falcom_last_launches(const MomentumCompressor *mc);
long long falcom_total_launches(const MomentumCompressor *mc);

/* 1 when this pointer is device memory that the library can read directly. */
int falcom_is_device_pointer(const void *ptr);

/* Per-kernel device time.  When enabled, every kernel launch of the instance
 * is bracketed by CUDA events on the instance's stream; after each call the
 * elapsed times are added to per-kernel totals.  falcom_kernel_times fills
 * up to n totals (milliseconds) and launch counts, indexed by kernel id, and
 * returns the number of kernel ids; falcom_kernel_name names an id.
 * Enabling resets the totals. */
int falcom_set_kernel_timing(MomentumCompressor *mc, int on);

/* Releases, in one call, every CompressedLayerData held by items[0..n) and
 * every array in outs[0..n) (either pointer may be NULL); entries are reset
 * to NULL. */
void falcom_free_batch(BatchItem *items, size_t n, NDArray **outs);
int falcom_kernel_times(const MomentumCompressor *mc, double *ms, long long *counts, int n);
const char *falcom_kernel_name(int id);

#ifdef __cplusplus
}
#endif

#endif /* FALCOM_B200_H */
