/*
 * Stub of the SZ3 C API (szcompressor/SZ3, unpinned upstream version) used by
 * the reference at momentum_compressor_openmp_simd_final.c:1040-1211.  SZ3 is
 * not installed in this container.  SZ_compress_args returns NULL, so the
 * reference takes its own raw-copy fallback and tags payloads "sz3_memcpy"
 * (momentum_compressor_openmp_simd_final.c:1262-1275).  Test infrastructure only.
 */
#ifndef ORACLE_SHIM_SZ3C_H
#define ORACLE_SHIM_SZ3C_H
#include <stddef.h>
#define SZ_FLOAT 0
#define SZ_DOUBLE 1
#define ABS 0
#define REL 1
unsigned char *SZ_compress_args(int dataType, void *data, size_t *outSize, int errBoundMode,
                                double absErrBound, double relBoundRatio, double pwrBoundRatio,
                                size_t r5, size_t r4, size_t r3, size_t r2, size_t r1);
void *SZ_decompress(int dataType, unsigned char *bytes, size_t byteLength,
                    size_t r5, size_t r4, size_t r3, size_t r2, size_t r1);
void free_buf(void *buf);
#endif
