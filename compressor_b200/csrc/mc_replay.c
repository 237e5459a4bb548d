/*
 * mc_replay.c -- replay rounds: captured client updates read from disk and
 * handed to the batch codec as ready-made BatchItems.
 *
 * File layout (little-endian), as written by the reference's capture tools
 * and read by benchmark_real.c:30-89 (load_test_data) and
 * cuda_feasibility/profile_appfl_hot_rounds.py:47-72 (read_round):
 *
 *   u32 round | char client_id[64] | u64 layer_count
 *   per layer: char name[256] | u64 shape[8] | u64 ndim | u32 dtype |
 *              u64 data_size | data_size bytes
 *
 * dtype codes are the DataType enum (0 float32, 1 float64, 2 int32, 3 int64,
 * 4 uint8); ndim 0 is a scalar (one element).  The reference loader trusts
 * data_size; this one also requires data_size == prod(shape[:ndim]) *
 * element size, ndim <= 8 and a known dtype, so that the NDArrays it returns
 * are consistent.
 *
 * Device residency: the headers are read first (the data blocks are skipped
 * with fseeko), one device block holds every tensor (256-byte aligned), and
 * the data streams through two pinned staging buffers: while one chunk is
 * copied to the device, the next one is read from the file.
 */
#define _FILE_OFFSET_BITS 64
#define _GNU_SOURCE
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include <cuda_runtime_api.h>

#include "mc_internal.h"

#define RP_NAME 256
#define RP_CLIENT 64
#define RP_MAXDIM 8
#define RP_ALIGN 256
#define RP_CHUNK ((size_t)16 << 20)

struct falcom_replay {
    uint32_t round;
    char client[RP_CLIENT + 1];
    size_t n;
    int location;   /* FALCOM_LOC_HOST or FALCOM_LOC_DEVICE */
    int device;
    char (*names)[RP_NAME + 1];
    size_t (*shapes)[RP_MAXDIM];
    NDArray *arrays;
    BatchItem *items;
    void *block;    /* every tensor: aligned host memory or one cudaMalloc */
    size_t block_bytes;
    size_t data_bytes;
};

static size_t dtype_bytes(uint32_t code) {
    switch (code) {
    case DTYPE_FLOAT32: return 4;
    case DTYPE_FLOAT64: return 8;
    case DTYPE_INT32: return 4;
    case DTYPE_INT64: return 8;
    case DTYPE_UINT8: return 1;
    default: return 0;
    }
}

static int rd(FILE *f, void *p, size_t n) { return fread(p, 1, n, f) == n; }

static void replay_free(falcom_replay *r) {
    if (!r) return;
    if (r->block) {
        if (r->location == FALCOM_LOC_DEVICE) {
            int cur = 0;
            cudaGetDevice(&cur);
            cudaSetDevice(r->device);
            cudaFree(r->block);
            cudaSetDevice(cur);
        } else {
            free(r->block);
        }
    }
    free(r->names);
    free(r->shapes);
    free(r->arrays);
    free(r->items);
    free(r);
}

/* Streams `len` bytes at file offset `off` to device address `dst` through
 * the two pinned staging buffers (ev[b] marks the last copy out of buffer b). */
static int stream_to_device(FILE *f, off_t off, size_t len, uint8_t *dst, uint8_t *pin[2], cudaEvent_t ev[2],
                            int *turn, cudaStream_t st) {
    if (fseeko(f, off, SEEK_SET) != 0) return -1;
    while (len) {
        const int b = *turn;
        *turn ^= 1;
        if (cudaEventSynchronize(ev[b]) != cudaSuccess) return -1;
        const size_t k = len < RP_CHUNK ? len : RP_CHUNK;
        if (!rd(f, pin[b], k)) return -1;
        if (cudaMemcpyAsync(dst, pin[b], k, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaEventRecord(ev[b], st) != cudaSuccess)
            return -1;
        dst += k;
        len -= k;
    }
    return 0;
}

MC_EXPORT falcom_replay *falcom_replay_open(const char *path, int location, int device) {
    if (!path || (location != FALCOM_LOC_HOST && location != FALCOM_LOC_DEVICE)) return NULL;
    FILE *f = fopen(path, "rb");
    if (!f) {
        fprintf(stderr, "Failed to open %s\n", path);
        return NULL;
    }
    falcom_replay *r = (falcom_replay *)calloc(1, sizeof(falcom_replay));
    off_t *offs = NULL;
    uint8_t *pin[2] = {NULL, NULL};
    cudaEvent_t ev[2] = {NULL, NULL};
    cudaStream_t st = NULL;
    int cur_dev = -1;
    struct stat sb;
    if (!r || fstat(fileno(f), &sb) != 0) goto fail;
    r->location = location;
    r->device = device;
    uint64_t count;
    char client[RP_CLIENT];
    if (!rd(f, &r->round, 4) || !rd(f, client, RP_CLIENT) || !rd(f, &count, 8)) goto fail;
    memcpy(r->client, client, RP_CLIENT);
    r->client[RP_CLIENT] = 0;
    /* every layer takes at least its 340-byte header */
    if (count > (uint64_t)sb.st_size / 340) goto fail;
    r->n = (size_t)count;
    const size_t n1 = r->n ? r->n : 1;
    r->names = calloc(n1, sizeof(*r->names));
    r->shapes = calloc(n1, sizeof(*r->shapes));
    r->arrays = (NDArray *)calloc(n1, sizeof(NDArray));
    r->items = (BatchItem *)calloc(n1, sizeof(BatchItem));
    offs = (off_t *)calloc(n1, sizeof(off_t));
    if (!r->names || !r->shapes || !r->arrays || !r->items || !offs) goto fail;

    /* headers; data blocks skipped */
    size_t total = 0;
    for (size_t i = 0; i < r->n; i++) {
        char name[RP_NAME];
        uint64_t shape[RP_MAXDIM], ndim, size;
        uint32_t dtype;
        if (!rd(f, name, RP_NAME) || !rd(f, shape, sizeof(shape)) || !rd(f, &ndim, 8) || !rd(f, &dtype, 4) ||
            !rd(f, &size, 8))
            goto fail;
        const size_t eb = dtype_bytes(dtype);
        if (ndim > RP_MAXDIM || eb == 0) goto fail;
        uint64_t elems = 1;
        for (uint64_t d = 0; d < ndim; d++) {
            if (shape[d] && elems > UINT64_MAX / shape[d]) goto fail;
            elems *= shape[d];
        }
        if (elems > UINT64_MAX / eb || elems * eb != size) goto fail;
        const off_t at = ftello(f);
        if (at < 0 || (uint64_t)at + size > (uint64_t)sb.st_size || fseeko(f, (off_t)size, SEEK_CUR) != 0) goto fail;
        offs[i] = at;
        memcpy(r->names[i], name, RP_NAME);
        r->names[i][RP_NAME] = 0;
        for (uint64_t d = 0; d < ndim; d++) r->shapes[i][d] = (size_t)shape[d];
        NDArray *a = &r->arrays[i];
        a->shape = r->shapes[i];
        a->ndim = (size_t)ndim;
        a->total_size = (size_t)elems;
        a->dtype = (DataType)dtype;
        a->data = (void *)(uintptr_t)total;   /* offset in the block for now */
        total += ((size_t)size + RP_ALIGN - 1) & ~(size_t)(RP_ALIGN - 1);
        r->data_bytes += (size_t)size;
    }
    r->block_bytes = total;

    /* data */
    if (location == FALCOM_LOC_HOST) {
        r->block = aligned_alloc(RP_ALIGN, total ? total : RP_ALIGN);   /* total: a multiple of RP_ALIGN */
        if (!r->block) goto fail;
        for (size_t i = 0; i < r->n; i++) {
            uint8_t *dst = (uint8_t *)r->block + (uintptr_t)r->arrays[i].data;
            const size_t len = r->arrays[i].total_size * dtype_bytes((uint32_t)r->arrays[i].dtype);
            if (fseeko(f, offs[i], SEEK_SET) != 0 || (len && !rd(f, dst, len))) goto fail;
        }
    } else {
        if (cudaGetDevice(&cur_dev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) goto fail_cuda;
        if (cudaMalloc(&r->block, total ? total : RP_ALIGN) != cudaSuccess) {
            r->block = NULL;
            goto fail_cuda;
        }
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
            cudaHostAlloc((void **)&pin[0], RP_CHUNK, cudaHostAllocDefault) != cudaSuccess ||
            cudaHostAlloc((void **)&pin[1], RP_CHUNK, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming) != cudaSuccess)
            goto fail_cuda;
        int turn = 0;
        for (size_t i = 0; i < r->n; i++) {
            uint8_t *dst = (uint8_t *)r->block + (uintptr_t)r->arrays[i].data;
            const size_t len = r->arrays[i].total_size * dtype_bytes((uint32_t)r->arrays[i].dtype);
            if (stream_to_device(f, offs[i], len, dst, pin, ev, &turn, st) != 0) goto fail_cuda;
        }
        if (cudaStreamSynchronize(st) != cudaSuccess) goto fail_cuda;
    }
    for (size_t i = 0; i < r->n; i++) {
        r->arrays[i].data = (uint8_t *)r->block + (uintptr_t)r->arrays[i].data;
        r->items[i].layer_name = r->names[i];
        r->items[i].gradient = &r->arrays[i];
        r->items[i].compressed = NULL;
        r->items[i].error = ERROR_NONE;
    }
    goto done;

fail_cuda:
    (void)cudaGetLastError();
fail:
    if (r) {
        /* the host / device block is released by replay_free */
        replay_free(r);
        r = NULL;
    }
done:
    if (st) {
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    for (int b = 0; b < 2; b++) {
        if (ev[b]) cudaEventDestroy(ev[b]);
        if (pin[b]) cudaFreeHost(pin[b]);
    }
    if (cur_dev >= 0) cudaSetDevice(cur_dev);
    free(offs);
    fclose(f);
    if (!r) fprintf(stderr, "[ERROR] replay round %s: unreadable or inconsistent file\n", path);
    return r;
}

MC_EXPORT size_t falcom_replay_count(const falcom_replay *r) { return r ? r->n : 0; }
MC_EXPORT uint32_t falcom_replay_round(const falcom_replay *r) { return r ? r->round : 0; }
MC_EXPORT const char *falcom_replay_client(const falcom_replay *r) { return r ? r->client : ""; }
MC_EXPORT size_t falcom_replay_bytes(const falcom_replay *r) { return r ? r->data_bytes : 0; }
MC_EXPORT BatchItem *falcom_replay_items(falcom_replay *r) { return r ? r->items : NULL; }
MC_EXPORT void falcom_replay_close(falcom_replay *r) { replay_free(r); }

MC_EXPORT int falcom_replay_write(const char *path, uint32_t round, const char *client_id, const BatchItem *items,
                                  size_t n) {
    if (!path || (n && !items)) return ERROR_INVALID_PARAM;
    for (size_t i = 0; i < n; i++) {
        const NDArray *a = items[i].gradient;
        if (!items[i].layer_name || !a || !a->data || (!a->shape && a->ndim) || a->ndim > RP_MAXDIM ||
            dtype_bytes((uint32_t)a->dtype) == 0 || strlen(items[i].layer_name) >= RP_NAME)
            return ERROR_INVALID_PARAM;
    }
    FILE *f = fopen(path, "wb");
    if (!f) return ERROR_INVALID_PARAM;
    int rc = ERROR_NONE;
    char client[RP_CLIENT];
    memset(client, 0, sizeof(client));
    if (client_id) strncpy(client, client_id, RP_CLIENT - 1);
    const uint64_t count = n;
    uint8_t *bounce = NULL;
    size_t bounce_cap = 0;
    mc_ptrcache pc;
    pc.n = 0;
    if (fwrite(&round, 4, 1, f) != 1 || fwrite(client, RP_CLIENT, 1, f) != 1 || fwrite(&count, 8, 1, f) != 1)
        rc = ERROR_ALLOCATION;
    for (size_t i = 0; i < n && rc == ERROR_NONE; i++) {
        const NDArray *a = items[i].gradient;
        char name[RP_NAME];
        memset(name, 0, sizeof(name));
        strncpy(name, items[i].layer_name, RP_NAME - 1);
        uint64_t shape[RP_MAXDIM], ndim = a->ndim, size;
        uint32_t dtype = (uint32_t)a->dtype;
        memset(shape, 0, sizeof(shape));
        uint64_t elems = 1;
        for (size_t d = 0; d < a->ndim; d++) {
            shape[d] = a->shape[d];
            elems *= a->shape[d];
        }
        size = elems * dtype_bytes(dtype);
        if (fwrite(name, RP_NAME, 1, f) != 1 || fwrite(shape, sizeof(shape), 1, f) != 1 ||
            fwrite(&ndim, 8, 1, f) != 1 || fwrite(&dtype, 4, 1, f) != 1 || fwrite(&size, 8, 1, f) != 1) {
            rc = ERROR_ALLOCATION;
            break;
        }
        if (!size) continue;
        const void *src = a->data;
        int dev = -1;
        if (mc_classify(&pc, a->data, &dev)) {   /* device tensor: copied out first */
            if (size > bounce_cap) {
                free(bounce);
                bounce = (uint8_t *)malloc((size_t)size);
                bounce_cap = bounce ? (size_t)size : 0;
                if (!bounce) {
                    rc = ERROR_ALLOCATION;
                    break;
                }
            }
            if (cudaMemcpy(bounce, a->data, (size_t)size, cudaMemcpyDeviceToHost) != cudaSuccess) {
                (void)cudaGetLastError();
                rc = ERROR_INVALID_PARAM;
                break;
            }
            src = bounce;
        }
        if (fwrite(src, 1, (size_t)size, f) != (size_t)size) rc = ERROR_ALLOCATION;
    }
    free(bounce);
    if (fclose(f) != 0 && rc == ERROR_NONE) rc = ERROR_ALLOCATION;
    return rc;
}
