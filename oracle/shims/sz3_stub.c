/* Link-time stub for the SZ3 C API; see SZ3c/sz3c.h.  Test infrastructure only. */
#include <stdlib.h>
#include "SZ3c/sz3c.h"
unsigned char *SZ_compress_args(int dataType, void *data, size_t *outSize, int errBoundMode,
                                double absErrBound, double relBoundRatio, double pwrBoundRatio,
                                size_t r5, size_t r4, size_t r3, size_t r2, size_t r1) {
    (void)dataType; (void)data; (void)errBoundMode; (void)absErrBound; (void)relBoundRatio;
    (void)pwrBoundRatio; (void)r5; (void)r4; (void)r3; (void)r2; (void)r1;
    if (outSize) *outSize = 0;
    return NULL;
}
void *SZ_decompress(int dataType, unsigned char *bytes, size_t byteLength,
                    size_t r5, size_t r4, size_t r3, size_t r2, size_t r1) {
    (void)dataType; (void)bytes; (void)byteLength; (void)r5; (void)r4; (void)r3; (void)r2; (void)r1;
    return NULL;
}
void free_buf(void *buf) { free(buf); }
