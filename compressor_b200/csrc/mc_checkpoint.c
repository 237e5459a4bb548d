/*
 * mc_checkpoint.c -- export and import of an instance's codec state.
 *
 * The reference keeps its state (step counts, gradient histories,
 * prediction memories; momentum_compressor_openmp_simd_final.c:420-471) in
 * process memory only.  Here the whole state of an instance -- every
 * "client:layer" record (step count, committed history head) and every
 * prediction memory -- can be written to a file and read back into any
 * instance, so an encoder or decoder resumes where it stopped after a
 * restart or moves to another GPU.
 *
 * File layout (little-endian):
 *   char magic[8] "FCSTATE1" | u32 version (1) | u32 zero |
 *   u64 layers | u64 memories | u64 memory clients
 *   layer:   u32 key bytes | key | i32 step | u32 has_tensor | [tensor]
 *   memory:  u32 key bytes | key | u32 has_tensor | [tensor]
 *   client:  u32 bytes | client id
 *   tensor:  u32 dtype | u32 ndim | u64 shape[ndim] | u64 bytes | bytes
 * Keys are the instance's own ("client:layer"; client, 0x1f, then
 * "layer|dtype|conv_(shape)").
 */
#define _FILE_OFFSET_BITS 64
#define _GNU_SOURCE
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "mc_internal.h"

static const char CK_MAGIC[8] = {'F', 'C', 'S', 'T', 'A', 'T', 'E', '1'};
#define CK_MAX_KEY (1u << 16)

typedef struct {
    uint8_t *buf;
    size_t cap;
} bounce_t;

static uint8_t *bounce(bounce_t *b, size_t n) {
    if (n <= b->cap) return b->buf;
    uint8_t *p = (uint8_t *)realloc(b->buf, n);
    if (!p) return NULL;
    b->buf = p;
    b->cap = n;
    return p;
}

static int wr(FILE *f, const void *p, size_t n) { return n == 0 || fwrite(p, 1, n, f) == n; }
static int rd(FILE *f, void *p, size_t n) { return n == 0 || fread(p, 1, n, f) == n; }

static int put_key(FILE *f, const char *k) {
    const uint32_t n = (uint32_t)strlen(k);
    return wr(f, &n, 4) && wr(f, k, n);
}

static int put_tensor(FILE *f, const mc_tensor *t, bounce_t *b) {
    const uint32_t has = t != NULL;
    if (!wr(f, &has, 4)) return 0;
    if (!t) return 1;
    const uint32_t dt = (uint32_t)t->dtype, nd = (uint32_t)t->ndim;
    uint64_t shape[MAX_NDIM];
    for (size_t d = 0; d < t->ndim; d++) shape[d] = t->shape[d];
    const uint64_t bytes = t->bytes;
    uint8_t *h = bounce(b, t->bytes ? t->bytes : 1);
    if (!h) return 0;
    if (t->bytes && cudaMemcpy(h, t->dev, t->bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return wr(f, &dt, 4) && wr(f, &nd, 4) && wr(f, shape, nd * 8) && wr(f, &bytes, 8) && wr(f, h, t->bytes);
}

MC_EXPORT int falcom_state_save(MomentumCompressor *mc, const char *path) {
    if (!mc || !path) return ERROR_INVALID_PARAM;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(mc->device);
    cudaStreamSynchronize(mc->stream);
    FILE *f = fopen(path, "wb");
    if (!f) {
        if (prev >= 0) cudaSetDevice(prev);
        return ERROR_INVALID_PARAM;
    }
    bounce_t b = {NULL, 0};
    const uint32_t ver = 1, zero = 0;
    const uint64_t nl = mc->layers->len, nm = mc->memory->len, nc = mc->mem_clients->len;
    int ok = wr(f, CK_MAGIC, 8) && wr(f, &ver, 4) && wr(f, &zero, 4) && wr(f, &nl, 8) && wr(f, &nm, 8) &&
             wr(f, &nc, 8);
    for (size_t i = 0; ok && i < mc->layers->cap; i++) {
        if (!MAP_LIVE(mc->layers, i)) continue;
        const mc_layer_rec *r = (const mc_layer_rec *)mc->layers->vals[i];
        const int32_t step = r->step;
        ok = put_key(f, mc->layers->keys[i]) && wr(f, &step, 4) && put_tensor(f, r->hist, &b);
    }
    for (size_t i = 0; ok && i < mc->memory->cap; i++) {
        if (!MAP_LIVE(mc->memory, i)) continue;
        const mc_mem_rec *r = (const mc_mem_rec *)mc->memory->vals[i];
        ok = put_key(f, mc->memory->keys[i]) && put_tensor(f, r->t, &b);
    }
    for (size_t i = 0; ok && i < mc->mem_clients->cap; i++) {
        if (!MAP_LIVE(mc->mem_clients, i)) continue;
        ok = put_key(f, mc->mem_clients->keys[i]);
    }
    free(b.buf);
    if (fclose(f) != 0) ok = 0;
    if (prev >= 0) cudaSetDevice(prev);
    if (!ok) {
        snprintf(mc->last_error, sizeof(mc->last_error), "state save to %s failed", path);
        return ERROR_ALLOCATION;
    }
    return ERROR_NONE;
}

static char *get_key(FILE *f) {
    uint32_t n;
    if (!rd(f, &n, 4) || n == 0 || n >= CK_MAX_KEY) return NULL;
    char *k = (char *)malloc(n + 1);
    if (!k) return NULL;
    if (!rd(f, k, n) || memchr(k, 0, n)) {
        free(k);
        return NULL;
    }
    k[n] = 0;
    return k;
}

/* Reads a tensor into a new device tensor (*out NULL when the record has
 * none); 0 on a format or allocation error. */
static int get_tensor(FILE *f, int device, bounce_t *b, mc_tensor **out) {
    *out = NULL;
    uint32_t has;
    if (!rd(f, &has, 4) || has > 1) return 0;
    if (!has) return 1;
    uint32_t dt, nd;
    uint64_t shape[MAX_NDIM], bytes;
    if (!rd(f, &dt, 4) || !rd(f, &nd, 4) || dt >= DTYPE_UNKNOWN || nd < 1 || nd > MAX_NDIM) return 0;
    if (!rd(f, shape, (size_t)nd * 8) || !rd(f, &bytes, 8)) return 0;
    size_t sh[MAX_NDIM];
    uint64_t n = 1;
    for (uint32_t d = 0; d < nd; d++) {
        if (shape[d] && n > (UINT64_MAX >> 4) / shape[d]) return 0;
        n *= shape[d];
        sh[d] = (size_t)shape[d];
    }
    if (n * mc_dtype_size((DataType)dt) != bytes) return 0;
    uint8_t *h = bounce(b, bytes ? (size_t)bytes : 1);
    if (!h || !rd(f, h, (size_t)bytes)) return 0;
    mc_tensor *t = tensor_new((DataType)dt, nd, sh, device);
    if (!t) return 0;
    if (bytes && cudaMemcpy(t->dev, h, (size_t)bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        (void)cudaGetLastError();
        tensor_drop(t);
        return 0;
    }
    *out = t;
    return 1;
}

MC_EXPORT int falcom_state_load(MomentumCompressor *mc, const char *path) {
    if (!mc || !path) return ERROR_INVALID_PARAM;
    FILE *f = fopen(path, "rb");
    if (!f) return ERROR_NOT_FOUND;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(mc->device);
    cudaStreamSynchronize(mc->stream);
    mc_map *layers = map_new(), *memory = map_new(), *clients = map_new();
    bounce_t b = {NULL, 0};
    char magic[8];
    uint32_t ver, zero;
    uint64_t nl, nm, nc;
    int ok = layers && memory && clients && rd(f, magic, 8) && memcmp(magic, CK_MAGIC, 8) == 0 &&
             rd(f, &ver, 4) && ver == 1 && rd(f, &zero, 4) && rd(f, &nl, 8) && rd(f, &nm, 8) && rd(f, &nc, 8);
    for (uint64_t i = 0; ok && i < nl; i++) {
        char *k = get_key(f);
        int32_t step;
        mc_layer_rec *r = (mc_layer_rec *)calloc(1, sizeof(mc_layer_rec));
        ok = k && r && rd(f, &step, 4) && step >= 0 && get_tensor(f, mc->device, &b, &r->hist) &&
             !map_get(layers, k);
        if (ok) {
            r->step = step;
            ok = map_put(layers, k, r) == 0;
        }
        if (!ok) layer_rec_drop(r);
        free(k);
    }
    for (uint64_t i = 0; ok && i < nm; i++) {
        char *k = get_key(f);
        mc_mem_rec *r = (mc_mem_rec *)calloc(1, sizeof(mc_mem_rec));
        ok = k && r && get_tensor(f, mc->device, &b, &r->t) && !map_get(memory, k) && strchr(k, '\x1f');
        if (ok) ok = map_put(memory, k, r) == 0;
        if (!ok) mem_rec_drop(r);
        free(k);
    }
    for (uint64_t i = 0; ok && i < nc; i++) {
        char *k = get_key(f);
        ok = k && map_put(clients, k, (void *)1) == 0;
        free(k);
    }
    if (ok) {   /* nothing may follow */
        char extra;
        ok = fread(&extra, 1, 1, f) == 0;
    }
    fclose(f);
    free(b.buf);
    if (!ok) {
        map_free(layers, layer_rec_drop);
        map_free(memory, mem_rec_drop);
        map_free(clients, NULL);
        if (prev >= 0) cudaSetDevice(prev);
        snprintf(mc->last_error, sizeof(mc->last_error), "state load from %s failed: not a state file", path);
        return ERROR_INVALID_PARAM;
    }
    map_free(mc->layers, layer_rec_drop);
    map_free(mc->memory, mem_rec_drop);
    map_free(mc->mem_clients, NULL);
    mc->layers = layers;
    mc->memory = memory;
    mc->mem_clients = clients;
    mc->state_gen++;   /* key caches hold pointers into the old records */
    if (prev >= 0) cudaSetDevice(prev);
    return ERROR_NONE;
}
