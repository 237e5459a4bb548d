/*
 * mc_wire.c -- zstd frame handling on the host.
 *
 * The codec's bitmap, dominant-sign and lossless payloads are zstd frames
 * (reference momentum_compressor_openmp_simd_final.c:635-705, level 10 at
 * :647).  Frames written by this library on the GPU hold only Raw and RLE
 * blocks (RFC 8878 sections 3.1.1.2); any zstd decoder reads them.  Frames
 * with compressed blocks (written by the reference or in "libzstd" frame
 * mode) are decoded through the system libzstd, loaded at run time.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

#include "mc_internal.h"

#define ZBLOCK 131072

size_t zf_max_frame_size(size_t content) {
    size_t nb = content == 0 ? 1 : (content + ZBLOCK - 1) / ZBLOCK;
    return 13 + 3 * nb + content;
}

/* Host writer of a Raw/RLE frame (same layout as the GPU writer). */
size_t zf_write_raw_host(uint8_t *dst, const uint8_t *src, size_t n) {
    int big = n >= 0xFFFFFFFFull;
    size_t pos = big ? 13 : 9;
    dst[0] = 0x28; dst[1] = 0xB5; dst[2] = 0x2F; dst[3] = 0xFD;
    dst[4] = big ? 0xE0 : 0xA0;
    for (int i = 0; i < (big ? 8 : 4); i++) dst[5 + i] = (uint8_t)((uint64_t)n >> (8 * i));
    size_t nb = n == 0 ? 1 : (n + ZBLOCK - 1) / ZBLOCK;
    for (size_t b = 0; b < nb; b++) {
        size_t bs = n - b * ZBLOCK < ZBLOCK ? n - b * ZBLOCK : ZBLOCK;
        const uint8_t *s = src + b * ZBLOCK;
        int rle = bs > 1;
        for (size_t i = 1; rle && i < bs; i++) rle = s[i] == s[0];
        uint32_t h = (b == nb - 1 ? 1u : 0u) | ((uint32_t)(rle ? 1 : 0) << 1) | ((uint32_t)bs << 3);
        dst[pos] = (uint8_t)h;
        dst[pos + 1] = (uint8_t)(h >> 8);
        dst[pos + 2] = (uint8_t)(h >> 16);
        if (rle) {
            dst[pos + 3] = s[0];
            pos += 4;
        } else {
            memcpy(dst + pos + 3, s, bs);
            pos += 3 + bs;
        }
    }
    return pos;
}

/* Parses the frame header.  Returns the header length, or -1. */
static int zf_header(const uint8_t *f, size_t n, unsigned long long *csize, int *checksum) {
    if (n < 6 || f[0] != 0x28 || f[1] != 0xB5 || f[2] != 0x2F || f[3] != 0xFD) return -1;
    uint8_t fhd = f[4];
    int fcs_flag = fhd >> 6, ss = (fhd >> 5) & 1, did = fhd & 3;
    if (fhd & 0x08) return -1;
    size_t p = 5 + (ss ? 0 : 1);
    p += did == 0 ? 0 : (did == 1 ? 1 : (did == 2 ? 2 : 4));
    int fcs = fcs_flag == 0 ? (ss ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
    if (fcs == 0 || p + (size_t)fcs > n) return -1;
    unsigned long long v = 0;
    for (int i = 0; i < fcs; i++) v |= (unsigned long long)f[p + i] << (8 * i);
    if (fcs == 2) v += 256;
    *csize = v;
    *checksum = (fhd >> 2) & 1;
    return (int)(p + (size_t)fcs);
}

int zf_content_size(const uint8_t *frame, size_t n, unsigned long long *out) {
    int ck;
    return zf_header(frame, n, out, &ck) < 0 ? -1 : 0;
}

int zf_is_simple(const uint8_t *f, size_t n) {
    unsigned long long cs;
    int ck;
    int h = zf_header(f, n, &cs, &ck);
    if (h < 0) return 0;
    size_t p = (size_t)h;
    for (;;) {
        if (p + 3 > n) return 0;
        uint32_t bh = f[p] | ((uint32_t)f[p + 1] << 8) | ((uint32_t)f[p + 2] << 16);
        p += 3;
        int last = bh & 1, type = (bh >> 1) & 3;
        size_t bs = bh >> 3;
        if (type == 0) p += bs;
        else if (type == 1) p += 1;
        else return 0;
        if (p > n) return 0;
        if (last) break;
    }
    return 1;
}

/* ------------------------------------------------------------- libzstd */
typedef size_t (*fn_decompress)(void *, size_t, const void *, size_t);
typedef size_t (*fn_compress)(void *, size_t, const void *, size_t, int);
typedef unsigned (*fn_iserror)(size_t);
static fn_decompress p_decompress;
static fn_compress p_compress;
static fn_iserror p_iserror;
static int z_state = 0;  /* 0 unknown, 1 ok, -1 missing */
static pthread_mutex_t z_mu = PTHREAD_MUTEX_INITIALIZER;

int zf_libzstd_available(void) {
    pthread_mutex_lock(&z_mu);
    if (z_state == 0) {
        void *h = dlopen("libzstd.so.1", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libzstd.so", RTLD_NOW | RTLD_LOCAL);
        if (h) {
            p_decompress = (fn_decompress)dlsym(h, "ZSTD_decompress");
            p_compress = (fn_compress)dlsym(h, "ZSTD_compress");
            p_iserror = (fn_iserror)dlsym(h, "ZSTD_isError");
        }
        z_state = (h && p_decompress && p_compress && p_iserror) ? 1 : -1;
    }
    int ok = z_state == 1;
    pthread_mutex_unlock(&z_mu);
    return ok;
}

size_t zf_libzstd_compress(uint8_t *dst, size_t cap, const uint8_t *src, size_t n, int level) {
    if (!zf_libzstd_available()) return 0;
    size_t rc = p_compress(dst, cap, src, n, level);
    return p_iserror(rc) ? 0 : rc;
}

/* Decodes a frame into dst (cap bytes).  Returns 0 and the content length. */
int zf_decode_host(const uint8_t *f, size_t n, uint8_t *dst, size_t cap, size_t *out) {
    unsigned long long cs;
    int ck;
    int h = zf_header(f, n, &cs, &ck);
    if (h < 0 || cs > cap) return -1;
    if (!zf_is_simple(f, n)) {
        if (!zf_libzstd_available()) return -1;
        size_t rc = p_decompress(dst, cap, f, n);
        if (p_iserror(rc)) return -1;
        *out = rc;
        return 0;
    }
    size_t p = (size_t)h, o = 0;
    for (;;) {
        uint32_t bh = f[p] | ((uint32_t)f[p + 1] << 8) | ((uint32_t)f[p + 2] << 16);
        p += 3;
        int last = bh & 1, type = (bh >> 1) & 3;
        size_t bs = bh >> 3;
        if (o + bs > cap) return -1;
        if (type == 0) {
            memcpy(dst + o, f + p, bs);
            p += bs;
        } else {
            memset(dst + o, f[p], bs);
            p += 1;
        }
        o += bs;
        if (last) break;
    }
    if (o != cs) return -1;
    *out = o;
    return 0;
}
