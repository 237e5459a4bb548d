/*
 * mc_batch.c -- grouped batch compress and batch decompress engines.
 *
 * Compress follows the reference grouped path
 * (momentum_compressor_openmp_simd_final.c build_batch_pipeline :2566-2675,
 * process_batch_group :2710-2814, commit_grouped_batch_results :2869-2952):
 * the host plans every item (group key, local step chain, direct / momentum /
 * generic mode, which earlier input is its previous gradient), the GPU runs
 * the numeric passes for the whole batch, and the state maps are updated only
 * after every device step succeeded (all-or-nothing).
 *
 * Decompress follows decompress_batch (:4707-4838) -> decompress_layer
 * (:3476-3598) -> decompress_momentum_predicted_layer (:3186-3474), with the
 * per-item early exits of the reference decided on the host before launch
 * (or, for device-resident bitmaps, from the device-computed predicted count
 * before commit).
 */
#define _GNU_SOURCE
#include <stdlib.h>
#include <string.h>

#include "mc_internal.h"

#define ALIGN_UP(x, a) (((x) + ((a)-1)) & ~((size_t)(a)-1))

/* Host phase profile, printed to stderr when FALCOM_PROFILE is set. */
#include <time.h>
static double prof_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e6 + (double)ts.tv_nsec * 1e-3;
}
typedef struct {
    int on;
    int n;
    double t[24];
    const char *what[24];
} prof_t;
static void prof_mark(prof_t *p, const char *what) {
    if (!p->on || p->n >= 24) return;
    p->t[p->n] = prof_now();
    p->what[p->n] = what;
    p->n++;
}
static void prof_print(prof_t *p, const char *tag) {
    if (!p->on || p->n < 2) return;
    fprintf(stderr, "[falcom-profile] %s total %.1f us:", tag, p->t[p->n - 1] - p->t[0]);
    for (int i = 1; i < p->n; i++) fprintf(stderr, " %s=%.1f", p->what[i], p->t[i] - p->t[i - 1]);
    fprintf(stderr, "\n");
}
/* The pinned table buffer (scratch slot SH_TABLES) is rewritten by every
 * call; event k (k = 0) marks the last upload out of it, so a call waits
 * for that copy only, not for other work the caller queued on the stream. */
void mc_tables_wait(MomentumCompressor *mc, int k) {
    if (mc->tab_ev_live[k] && cudaEventSynchronize(mc->tab_ev[k]) != cudaSuccess) {
        (void)cudaGetLastError();
        cudaDeviceSynchronize();
    }
}
int mc_tables_mark(MomentumCompressor *mc, int k, cudaStream_t st) {
    if (!mc->tab_ev[k] && cudaEventCreateWithFlags(&mc->tab_ev[k], cudaEventDisableTiming) != cudaSuccess) {
        mc->tab_ev[k] = NULL;
        return -1;
    }
    if (cudaEventRecord(mc->tab_ev[k], st) != cudaSuccess) return -1;
    mc->tab_ev_live[k] = 1;
    return 0;
}

#define SLOT_ALIGN 256
#define TILE_ELEMS MC_TILE_ELEMS

enum { MODE_DIRECT = 0, MODE_MOMENTUM = 1, MODE_GENERIC = 2 };

/* device scratch slots of an instance */
enum {
    SD_TABLES = 0,   /* item tables, tile lists, frame jobs */
    SD_RESULTS,      /* per-item results */
    SD_TILES,        /* per-tile partials */
    SD_POFF,         /* per-tile predicted offsets */
    SD_WORDS,        /* bitmap / dominant / dense-sign words */
    SD_INPUT,        /* staged host inputs */
    SD_PAYLOAD,      /* payload arena when payloads return to the host */
    SD_FSIZE,        /* frame sizes written by the device */
    SD_DSTAGE,       /* decoder: staged payload bytes */
    SD_DOUT,         /* decoder: contiguous decoded output before the host copy */
    SD_DCONTENT,     /* decoder: frame contents expanded on the device */
};
enum { SH_TABLES = 0, SH_RESULTS, SH_STAGE };

/* ------------------------------------------------------------ list cache */
static uint64_t sig_mix(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    return h * 1099511628211ull;
}

void listcache_free(MomentumCompressor *mc, mc_listcache *set) {
    for (int i = 0; i < MC_LIST_CACHE; i++) {
        if (set[i].dev) dbuf_put(mc->device, set[i].dev, set[i].bytes);
        free(set[i].counts);
        memset(&set[i], 0, sizeof(set[i]));
    }
}

/* The cached lists of signature `sig` (*hit = 1), or a slot prepared for
 * them: `bytes` of device memory and `nlists` counts (*hit = 0).  NULL when
 * memory is short. */
static mc_listcache *lists_get(MomentumCompressor *mc, mc_listcache *set, uint64_t sig, int nlists, size_t bytes,
                               int *hit) {
    mc_listcache *v = &set[0];
    for (int i = 0; i < MC_LIST_CACHE; i++) {
        if (set[i].sig == sig && set[i].nlists == nlists && set[i].bytes == bytes && set[i].dev) {
            set[i].used = ++mc->lc_tick;
            *hit = 1;
            return &set[i];
        }
        if (set[i].used < v->used) v = &set[i];
    }
    *hit = 0;
    if (v->dev && v->bytes != bytes) {
        dbuf_put(mc->device, v->dev, v->bytes);
        v->dev = NULL;
    }
    if (!v->dev) v->dev = dbuf_get(mc->device, bytes);
    int *c = (int *)realloc(v->counts, (size_t)nlists * sizeof(int));
    if (!v->dev || !c) {
        if (c) v->counts = c;
        v->sig = 0;
        return NULL;
    }
    v->counts = c;
    v->bytes = bytes;
    v->nlists = nlists;
    v->sig = 0;   /* set by the caller once the lists are uploaded */
    v->used = ++mc->lc_tick;
    return v;
}

/* ---------------------------------------------------- chunked pipelines */
/* A call with host buffers moves every byte over PCIe; splitting its items
 * into chunks lets the upload of chunk c+1 run under the kernels of chunk c
 * and the download of chunk c under the kernels of chunk c+1 (two copy
 * streams, one per direction, ordered against the compute stream by
 * events). */
#define CHUNK_MIN_BYTES ((size_t)12 << 20)

int mc_pipeline_init(MomentumCompressor *mc) {
    if (mc->copy_in && mc->copy_out && mc->ev_done[MC_MAX_CHUNKS - 1]) return 0;
    if (!mc->copy_in && cudaStreamCreateWithFlags(&mc->copy_in, cudaStreamNonBlocking) != cudaSuccess) return -1;
    if (!mc->copy_out && cudaStreamCreateWithFlags(&mc->copy_out, cudaStreamNonBlocking) != cudaSuccess) return -1;
    for (int i = 0; i < MC_MAX_CHUNKS; i++) {
        if (!mc->ev_in[i] && cudaEventCreateWithFlags(&mc->ev_in[i], cudaEventDisableTiming) != cudaSuccess) return -1;
        if (!mc->ev_done[i] && cudaEventCreateWithFlags(&mc->ev_done[i], cudaEventDisableTiming) != cudaSuccess)
            return -1;
    }
    return 0;
}

/* Splits items [0, n) into at most MC_MAX_CHUNKS consecutive ranges of about
 * equal bytes (bytes[i] per item), each at least CHUNK_MIN_BYTES; starts[c]
 * is the first item of chunk c, starts[nc] = n.  Returns nc. */
static int chunk_items(const size_t *bytes, size_t n, size_t *starts) {
    size_t total = 0;
    for (size_t i = 0; i < n; i++) total += bytes[i];
    int nc = (int)(total / CHUNK_MIN_BYTES);
    if (nc > MC_MAX_CHUNKS) nc = MC_MAX_CHUNKS;
    if (nc < 1) nc = 1;
    size_t acc = 0;
    int c = 0;
    starts[0] = 0;
    for (size_t i = 0; i < n && c + 1 < nc; i++) {
        acc += bytes[i];
        if (acc * (size_t)nc >= total * (size_t)(c + 1)) starts[++c] = i + 1;
    }
    nc = c + 1;
    starts[nc] = n;
    return nc;
}



/* Call-local string -> int table (keys are borrowed, not copied). */
typedef struct {
    const char **keys;
    int *vals;
    size_t cap;
} strtab;

static uint64_t st_hash(const char *s) {
    uint64_t h = 1469598103934665603ull;
    while (*s) {
        h ^= (unsigned char)*s++;
        h *= 1099511628211ull;
    }
    return h;
}

static int strtab_init(strtab *t, size_t n) {
    t->cap = 16;
    while (t->cap < 4 * n) t->cap <<= 1;
    t->keys = (const char **)calloc(t->cap, sizeof(char *));
    t->vals = (int *)calloc(t->cap, sizeof(int));
    return t->keys && t->vals ? 0 : -1;
}

static void strtab_free(strtab *t) {
    free(t->keys);
    free(t->vals);
}

/* Returns the value slot of `key`, inserting it with value `init` if absent. */
static int *strtab_slot(strtab *t, const char *key, int init) {
    size_t i = (size_t)st_hash(key) & (t->cap - 1);
    while (t->keys[i]) {
        if (strcmp(t->keys[i], key) == 0) return &t->vals[i];
        i = (i + 1) & (t->cap - 1);
    }
    t->keys[i] = key;
    t->vals[i] = init;
    return &t->vals[i];
}

/* ================================================================ compress */
typedef struct {
    mc_layer_rec *lrec;
    mc_mem_rec *mrec;
    int group;
    int mode;
    int local_step;
    int kind;
    int dcodec;
    const char *codec_tag;
    int wave;
    int prev_item;
    mc_tensor *prev_t;
    int use_lossy;
    int candidate;
    DataType dt;
    size_t n, bytes, K, ks;
    const NDArray *g;
    int src_dev;
    const void *dev_in;
    mc_tensor *hist;
    size_t off_data, cap_data, off_bm, cap_bm, off_sg, cap_sg;
    size_t words_off;    /* in SD_WORDS, units of uint32 */
    size_t kwords;
    int tile_base, ntiles, tile_param;
    size_t nblk;                     /* MOMENTUM: bitmap frame blocks */
    size_t fs_bm, fs_sg, fs_data;    /* frame sizes in libzstd frame mode */
} cplan;

typedef struct {
    mc_mem_rec *mrec;          /* memory record of a layer-key group */
    mc_tensor *mem_committed;
    mc_tensor *mem_new;
    int n_mom;
    int last;   /* last item of the group in batch order, -1 before the first */
} cgroup;

static int layout_equal(const NDArray *a, DataType dt, size_t ndim, const size_t *shape, size_t n) {
    if (a->dtype != dt || a->ndim != ndim || a->total_size != n) return 0;
    for (size_t i = 0; i < ndim; i++)
        if (a->shape[i] != shape[i]) return 0;
    return 1;
}

static int dcodec_of(int codec) {
    switch (codec) {
        case MC_CODEC_INT4: return MC_DC_INT4;
        case MC_CODEC_RAW: return MC_DC_RAW;
        case MC_CODEC_Q8_RAW: return MC_DC_Q8_RAW;
        case MC_CODEC_INT4_RAW: return MC_DC_INT4_RAW;
        default: return MC_DC_Q8;
    }
}

static size_t residual_bytes(int dcodec, size_t n) {
    switch (dcodec) {
        case MC_DC_Q8: return 4 + n;
        case MC_DC_INT4: return 4 + (n + 1) / 2;
        default: return 4 * n;
    }
}

static const char *codec_tag_of(int dcodec) {
    switch (dcodec) {
        case MC_DC_Q8: return "q8";
        case MC_DC_INT4: return "int4";
        default: return "sz3_memcpy";
    }
}

/* Kernels per momentum tile of a layer of K kernels of ks elements: at
 * least 32 (one ballot word), a multiple of 32 (tiles start on bitmap
 * words), at most TILE_ELEMS elements where that allows more than 32.
 * A layer whose bitmap frame has one block (K <= 2^20) takes the largest
 * such multiple (ks = 9: 448 kernels, 4032 elements, 98 % of a stage);
 * a longer bitmap takes the largest power of two, so that every 2^20-kernel
 * block of the frame is a union of whole tiles. */
static int tile_kernels_for(size_t ks, size_t K) {
    const size_t e = ks ? ks : 1;
    if (K <= ((size_t)MC_ZBLOCK << 3)) {
        const size_t tk = (TILE_ELEMS / e) & ~(size_t)31;
        return (int)(tk >= 32 ? tk : 32);
    }
    size_t tk = TILE_ELEMS;
    while (tk > 32 && tk * e > TILE_ELEMS) tk >>= 1;
    return (int)tk;
}

static size_t frame_blocks(size_t content) {
    return content == 0 ? 1 : (content + MC_ZBLOCK - 1) / MC_ZBLOCK;
}

/* Returns the batch's new tensors to their records' spare slots (or the pool). */
static void free_plan_tensors(MomentumCompressor *mc, cplan *P, size_t n, cgroup *G, size_t ng) {
    for (size_t i = 0; i < n; i++) {
        if (P[i].hist) {
            if (P[i].lrec && !P[i].lrec->spare) P[i].lrec->spare = P[i].hist;
            else tensor_drop(P[i].hist);
        }
        P[i].hist = NULL;
    }
    for (size_t g = 0; g < ng; g++) {
        if (G[g].mem_new) {
            if (G[g].mrec && !G[g].mrec->spare) G[g].mrec->spare = G[g].mem_new;
            else tensor_drop(G[g].mem_new);
        }
        G[g].mem_new = NULL;
    }
    (void)mc;
}

/* one host-to-device copy of adjacent host inputs */
typedef struct {
    uintptr_t base, end;
    size_t off;   /* in the staging buffer */
    int chunk;
} in_run;

int mc_compress_grouped(MomentumCompressor *mc, BatchItem *items, size_t n, const char *client,
                        int payload_loc, int allow_fault) {
    /* chunked pipeline state (declared first: every exit path frees it) */
    int nchunks = 1;
    size_t cstart[MC_MAX_CHUNKS + 1];
    in_run *runs = NULL;
    size_t nruns = 0;
    uint8_t *stage = NULL;
    int rc = ERROR_NONE;
    CompressedLayerData **outs = NULL, *blk = NULL;   /* result structs (filled while the GPU works) */
    cplan *P = (cplan *)calloc(n, sizeof(cplan));
    cgroup *G = (cgroup *)calloc(n, sizeof(cgroup));
    if (!P || !G) {
        free(P);
        free(G);
        return ERROR_ALLOCATION;
    }
    size_t ng = 0;
    prof_t prof = {0};
    prof.on = mc_env_flag("FALCOM_PROFILE");
    prof_mark(&prof, "start");

    /* ---------------------------------------------------- validation / meta */
    for (size_t i = 0; i < n; i++) {
        items[i].compressed = NULL;
        items[i].error = ERROR_NONE;
    }
    mc_keyreq *req = (mc_keyreq *)malloc(n * sizeof(mc_keyreq));
    int *gid = (int *)malloc(3 * n * sizeof(int));
    if (!req || !gid) {
        free(req);
        free(gid);
        rc = ERROR_ALLOCATION;
        goto out;
    }
    for (size_t i = 0; i < n; i++) {
        const NDArray *g = items[i].gradient;
        if (!g || !items[i].layer_name) {
            items[i].error = ERROR_INVALID_PARAM;
            mc_set_error(mc, "Batch compress: item[%zu] has NULL gradient or layer_name", i);
            rc = ERROR_INVALID_PARAM;
            break;
        }
        size_t elem = mc_dtype_size(g->dtype);
        size_t prod = 1;
        int bad = g->ndim < MIN_NDIM || g->ndim > MAX_NDIM || !g->shape || !g->data || elem == 0;
        for (size_t d = 0; !bad && d < g->ndim; d++) prod *= g->shape[d];
        if (bad || prod == 0 || prod != g->total_size) {
            items[i].error = ERROR_INVALID_PARAM;
            mc_set_error(mc, "Batch compress: item[%zu] '%s' has an invalid array descriptor", i,
                         items[i].layer_name);
            rc = ERROR_INVALID_PARAM;
            break;
        }
        cplan *p = &P[i];
        p->g = g;
        p->dt = g->dtype;
        p->n = g->total_size;
        p->bytes = p->n * elem;
        p->prev_item = -1;
        p->fs_bm = p->fs_sg = p->fs_data = 0;
        req[i].name = items[i].layer_name;
        req[i].dt = g->dtype;
        req[i].ndim = g->ndim;
        req[i].shape = g->shape;
    }
    const mc_keycache *kc = NULL;
    if (rc == ERROR_NONE) kc = keycache_get(mc, mc->enc_kc, client, req, n, &rc);
    free(req);
    if (rc != ERROR_NONE) {
        free(gid);
        goto out;
    }
    for (size_t i = 0; i < n; i++) {
        P[i].lrec = kc->lrec[i];
        P[i].mrec = kc->mrec[i];
        P[i].use_lossy = kc->lossy[i];
        P[i].candidate = P[i].g->ndim == 4 && P[i].dt == DTYPE_FLOAT32 && P[i].use_lossy;
    }

    /* ------------------------------------------------ fault injection hook */
    {
        const char *fault = allow_fault ? getenv("FALCOM_FAULT_INJECT_COMPRESS_FAIL_AT") : NULL;
        if (fault && *fault && (size_t)strtoull(fault, NULL, 10) < n) {
            mc_set_error(mc, "fault injection requested for item[%zu]",
                         (size_t)strtoull(fault, NULL, 10));
            for (size_t i = 0; i < n; i++) items[i].error = ERROR_COMPRESSION;
            rc = ERROR_COMPRESSION;
            free(gid);
            goto out;
        }
    }

    prof_mark(&prof, "validate");
    /* --------------------------------------------- group keys (:2627-2645)
     * layer-key groups are identified by the first item with that layer
     * key, history-key groups by the first item with that history key. */
    for (size_t i = 0; i < 3 * n; i++) gid[i] = -1;
    for (size_t i = 0; i < n; i++) {
        const int same = kc->same[i];
        P[i].prev_t = P[i].lrec->hist;
        int slot;
        if (P[i].candidate && (P[i].prev_t != NULL || same > 1)) slot = kc->first_l[i];
        else if (same > 1) slot = (int)n + kc->first_h[i];
        else slot = 2 * (int)n + (int)i;
        if (gid[slot] < 0) {
            gid[slot] = (int)ng;
            G[ng].mrec = slot < (int)n ? P[i].mrec : NULL;
            G[ng].mem_committed = G[ng].mrec ? G[ng].mrec->t : NULL;
            G[ng].last = -1;
            ng++;
        }
        P[i].group = gid[slot];
    }
    free(gid);

    /* ------------------------ per-group step chains (:2710-2814, in order)
     * Every item of a group has the same history key (the group key is the
     * layer key, which contains the layer name, or the history key itself),
     * so the group's chain state is its last processed item. */
    for (size_t i = 0; i < n; i++) {
        cgroup *grp = &G[P[i].group];
        const int last = grp->last;
        int step0 = last >= 0 ? P[last].local_step : P[i].lrec->step;
        P[i].local_step = step0 + 1;
        const NDArray *g_i = P[i].g;
        int has_prev = 0, prev_match = 0;
        if (last >= 0) {
            has_prev = 1;
            const NDArray *pg = P[last].g;
            prev_match = layout_equal(g_i, pg->dtype, pg->ndim, pg->shape, pg->total_size);
            P[i].prev_item = last;
            P[i].prev_t = NULL;
        } else if (P[i].prev_t) {
            mc_tensor *h = P[i].prev_t;
            has_prev = 1;
            prev_match = layout_equal(g_i, h->dtype, h->ndim, h->shape, h->n);
        }
        if (P[i].local_step == 1) P[i].mode = MODE_DIRECT;
        else if (has_prev && prev_match && P[i].candidate) P[i].mode = MODE_MOMENTUM;
        else P[i].mode = MODE_GENERIC;
        if (P[i].mode == MODE_MOMENTUM) {
            P[i].wave = grp->n_mom;
            grp->n_mom++;
        }
        grp->last = (int)i;
    }

    prof_mark(&prof, "plan");
    /* --------------------------------------------- kinds, codecs, tiling */
    const int dcodec = dcodec_of(mc->residual_codec);
    int nwaves = 1;
    int ntiles_total = 0, nmom = 0;
    size_t words_total = 0;
    for (size_t i = 0; i < n; i++) {
        cplan *p = &P[i];
        if (p->mode == MODE_MOMENTUM) {
            p->kind = MC_K_MOMENTUM;
            p->dcodec = dcodec;
            p->codec_tag = codec_tag_of(dcodec);
            p->K = p->g->shape[0] * p->g->shape[1];
            p->ks = p->g->shape[2] * p->g->shape[3];
            p->tile_param = tile_kernels_for(p->ks, p->K);
            p->ntiles = (int)((p->K + (size_t)p->tile_param - 1) / (size_t)p->tile_param);
            p->kwords = (p->K + 31) / 32 + 1;
            p->nblk = frame_blocks((p->K + 7) / 8);
            p->words_off = words_total;
            words_total += 2 * ALIGN_UP(p->kwords, 64) + ALIGN_UP(p->nblk, 64);
            if (p->wave + 1 > nwaves) nwaves = p->wave + 1;
            nmom++;
        } else if (p->use_lossy && p->dt == DTYPE_FLOAT32 && dcodec != MC_DC_RAW) {
            p->dcodec = dcodec;
            p->codec_tag = codec_tag_of(dcodec);
            p->kind = MC_K_QUANT;
            /* the encoder stages only the input of a direct quantised tile,
             * so its tile fills both arrays of the two-array stage */
            p->tile_param = 2 * TILE_ELEMS;
            p->ntiles = (int)((p->n + 2 * TILE_ELEMS - 1) / (2 * TILE_ELEMS));
        } else if (p->use_lossy) {
            /* raw residual codec, and float64 lossy tensors: raw copy (the
             * reference's result when SZ3 is unavailable) */
            p->kind = MC_K_COPY;
            p->dcodec = MC_DC_RAW;
            p->codec_tag = "sz3_memcpy";
            p->tile_param = TILE_ELEMS * 4;
            p->ntiles = (int)((p->bytes + (size_t)p->tile_param - 1) / (size_t)p->tile_param);
        } else {
            p->kind = MC_K_FRAME;
            p->codec_tag = "zstd";
            p->tile_param = TILE_ELEMS * 4;
            p->ntiles = (int)((p->bytes + (size_t)p->tile_param - 1) / (size_t)p->tile_param);
        }
        p->tile_base = ntiles_total;
        ntiles_total += p->ntiles;
    }
    if (mc->frame_mode == MC_FRAME_LIBZSTD) payload_loc = FALCOM_LOC_HOST;

    /* --------------------------------------------------- payload layout */
    size_t arena_bytes = 0;
    for (size_t i = 0; i < n; i++) {
        cplan *p = &P[i];
        size_t cap;
        if (p->kind == MC_K_MOMENTUM || p->kind == MC_K_QUANT) cap = residual_bytes(p->dcodec, p->n);
        else if (p->kind == MC_K_COPY) cap = p->bytes;
        else cap = zf_max_frame_size(p->bytes) + (mc->frame_mode == MC_FRAME_LIBZSTD ? p->bytes / 64 + 1024 : 0);
        p->off_data = arena_bytes;
        p->cap_data = cap;
        arena_bytes = ALIGN_UP(arena_bytes + cap, SLOT_ALIGN);
        if (p->kind == MC_K_MOMENTUM) {
            size_t c = (p->K + 7) / 8;
            size_t fc = ALIGN_UP(zf_max_frame_size(c) + (mc->frame_mode == MC_FRAME_LIBZSTD ? c / 64 + 1024 : 0), 16);
            p->off_bm = arena_bytes;
            p->cap_bm = fc;
            arena_bytes = ALIGN_UP(arena_bytes + fc, SLOT_ALIGN);
            p->off_sg = arena_bytes;
            p->cap_sg = fc;
            arena_bytes = ALIGN_UP(arena_bytes + fc, SLOT_ALIGN);
        }
    }

    /* --------------------------------------- device memory for this batch */
    cudaStream_t st = mc->stream;
    const int dev = mc->device;
    mc_arena *dev_arena = NULL, *host_arena = NULL;
    uint8_t *payload_dev;
    if (payload_loc == FALCOM_LOC_DEVICE) {
        dev_arena = arena_acquire(arena_bytes, dev);
        payload_dev = dev_arena ? (uint8_t *)dev_arena->ptr : NULL;
    } else {
        payload_dev = (uint8_t *)scratch_dev(&mc->scratch, SD_PAYLOAD, arena_bytes);
        host_arena = arena_acquire(arena_bytes, -1);
    }
    if (!payload_dev || (payload_loc != FALCOM_LOC_DEVICE && !host_arena)) {
        mc_set_error(mc, "Batch compress: payload allocation failed (%zu bytes)", arena_bytes);
        rc = ERROR_ALLOCATION;
        goto fail;
    }

    prof_mark(&prof, "layout");
    /* history tensors, group memories */
    for (size_t i = 0; i < n; i++) {
        /* an item that is not the last of its history key in this batch
         * never becomes the committed head: take a pooled buffer for it */
        int last_of_key = G[P[i].group].last == (int)i;
        P[i].hist = rec_take(last_of_key ? &P[i].lrec->spare : NULL, P[i].dt, P[i].g->ndim, P[i].g->shape, dev);
        if (!P[i].hist) {
            rc = ERROR_ALLOCATION;
            mc_set_error(mc, "Batch compress: device allocation failed for history");
            goto fail;
        }
    }
    for (size_t i = 0; i < n; i++) {
        cgroup *grp = &G[P[i].group];
        if (P[i].mode != MODE_MOMENTUM || grp->mem_new) continue;
        /* every momentum item of a group has the group's shape */
        grp->mem_new = rec_take(grp->mrec ? &grp->mrec->spare : NULL, DTYPE_FLOAT32, 4, P[i].g->shape, dev);
        if (!grp->mem_new) {
            rc = ERROR_ALLOCATION;
            mc_set_error(mc, "Batch compress: device allocation failed for prediction memory");
            goto fail;
        }
    }

    prof_mark(&prof, "alloc");
    /* ----------------------------------------------- stage host inputs */
    /* host inputs are copied into one device staging buffer, adjacent
     * inputs (16-byte aligned) as one copy; with enough host bytes and one
     * wave the copies are split by item chunk and issued later, interleaved
     * with the chunk launches (chunked pipeline) */
    cstart[0] = 0;
    cstart[1] = n;
    {
        size_t stage_bytes = 0, host_bytes = 0;
        int any_host = 0;
        mc_ptrcache pc;
        pc.n = 0;
        for (size_t i = 0; i < n; i++) {
            int d = -1;
            P[i].src_dev = mc_classify(&pc, P[i].g->data, &d);
            if (P[i].src_dev && d != dev) P[i].src_dev = 0;   /* another GPU: copy */
            if (!P[i].src_dev) {
                any_host = 1;
                host_bytes += P[i].bytes;
            }
        }
        if (any_host && nwaves == 1 && host_bytes >= 2 * CHUNK_MIN_BYTES && mc_pipeline_init(mc) == 0) {
            size_t *hb = (size_t *)malloc(n * sizeof(size_t));
            if (hb) {
                for (size_t i = 0; i < n; i++) hb[i] = P[i].src_dev ? 0 : P[i].bytes;
                nchunks = chunk_items(hb, n, cstart);
                free(hb);
            }
        }
        if (any_host) {
            size_t *order = (size_t *)malloc(n * sizeof(size_t));
            int *chunk_of = (int *)malloc(n * sizeof(int));
            runs = (in_run *)malloc(n * sizeof(in_run));
            if (!order || !chunk_of || !runs) {
                free(order);
                free(chunk_of);
                rc = ERROR_ALLOCATION;
                goto fail;
            }
            for (int c = 0; c < nchunks; c++)
                for (size_t i = cstart[c]; i < cstart[c + 1]; i++) chunk_of[i] = c;
            size_t no = 0;
            for (size_t i = 0; i < n; i++)
                if (!P[i].src_dev) order[no++] = i;
            for (size_t a = 1; a < no; a++) { /* insertion sort by (chunk, address) */
                size_t v = order[a], b = a;
                while (b > 0 && (chunk_of[order[b - 1]] > chunk_of[v] ||
                                 (chunk_of[order[b - 1]] == chunk_of[v] &&
                                  (uintptr_t)P[order[b - 1]].g->data > (uintptr_t)P[v].g->data))) {
                    order[b] = order[b - 1];
                    b--;
                }
                order[b] = v;
            }
            for (size_t a = 0; a < no;) {
                size_t i0 = order[a];
                uintptr_t base = (uintptr_t)P[i0].g->data, end = base + P[i0].bytes;
                size_t b = a + 1;
                while (b < no && chunk_of[order[b]] == chunk_of[i0]) {
                    uintptr_t s2 = (uintptr_t)P[order[b]].g->data;
                    if (s2 != end || (s2 & 15) || (base & 15)) break;
                    end = s2 + P[order[b]].bytes;
                    b++;
                }
                runs[nruns].base = base;
                runs[nruns].end = end;
                runs[nruns].off = stage_bytes;
                runs[nruns].chunk = chunk_of[i0];
                for (size_t c = a; c < b; c++)
                    P[order[c]].dev_in = (const void *)(stage_bytes + ((uintptr_t)P[order[c]].g->data - base));
                stage_bytes = ALIGN_UP(stage_bytes + (end - base), SLOT_ALIGN);
                nruns++;
                a = b;
            }
            free(order);
            free(chunk_of);
            stage = (uint8_t *)scratch_dev(&mc->scratch, SD_INPUT, stage_bytes);
            if (!stage) {
                rc = ERROR_ALLOCATION;
                mc_set_error(mc, "Batch compress: input staging allocation failed");
                goto fail;
            }
            for (size_t i = 0; i < n; i++)
                if (!P[i].src_dev) P[i].dev_in = stage + (uintptr_t)P[i].dev_in;
            if (nchunks == 1) {   /* one chunk: all copies now, in stream order before the kernels */
                for (size_t r = 0; r < nruns; r++) {
                    if (cudaMemcpyAsync(stage + runs[r].off, (const void *)runs[r].base, runs[r].end - runs[r].base,
                                        cudaMemcpyHostToDevice, st) != cudaSuccess) {
                        rc = ERROR_COMPRESSION;
                        mc_set_error(mc, "Batch compress: host-to-device copy failed");
                        goto fail;
                    }
                }
            }
        }
        for (size_t i = 0; i < n; i++)
            if (P[i].src_dev) P[i].dev_in = P[i].g->data;
    }

    prof_mark(&prof, "stage");
    /* ------------------------------------------------------ scratch sizes */
    uint32_t *words = NULL;
    if (words_total) {
        words = (uint32_t *)scratch_dev(&mc->scratch, SD_WORDS, words_total * 4);
        if (!words) {
            rc = ERROR_ALLOCATION;
            goto fail;
        }
    }
    mc_enc_result *results = (mc_enc_result *)scratch_dev(&mc->scratch, SD_RESULTS,
                                                          n * sizeof(mc_enc_result));
    mc_enc_tile *tiles = (mc_enc_tile *)scratch_dev(&mc->scratch, SD_TILES,
                                                    (size_t)(ntiles_total + 1) * sizeof(mc_enc_tile));
    int64_t *poff = (int64_t *)scratch_dev(&mc->scratch, SD_POFF, (size_t)(ntiles_total + 1) * 8);
    if (!results || !tiles || !poff) {
        rc = ERROR_ALLOCATION;
        goto fail;
    }

    /* ------------------------------------------------ build device tables */
    /* the item table is uploaded every call; the per-wave tile lists (all
     * tiles, momentum tiles) come from the list cache when this batch has the
     * structure of a recent one */
    size_t tab_items = ALIGN_UP(n * sizeof(mc_enc_item), 256);
    size_t tab_list = ALIGN_UP((size_t)(ntiles_total + 1) * sizeof(mc_tile_ref), 256);
    uint64_t sig = sig_mix(0x6A09E667F3BCC908ull, (uint64_t)n);
    sig = sig_mix(sig, (uint64_t)nwaves);
    for (size_t i = 0; i < n; i++)
        sig = sig_mix(sig, ((uint64_t)P[i].kind << 56) ^ ((uint64_t)(uint32_t)P[i].wave << 32) ^
                               (uint64_t)(uint32_t)P[i].ntiles);
    int lhit = 0;
    mc_listcache *lc = lists_get(mc, mc->enc_lists, sig, 2 * nwaves, 2 * tab_list * (size_t)nwaves, &lhit);
    size_t tab_total = tab_items + (lhit ? 0 : 2 * tab_list * (size_t)nwaves);
    uint8_t *htab = (uint8_t *)scratch_host(&mc->scratch, SH_TABLES, tab_total);
    uint8_t *dtab = (uint8_t *)scratch_dev(&mc->scratch, SD_TABLES, tab_items);
    if (!htab || !dtab || !lc) {
        rc = ERROR_ALLOCATION;
        goto fail;
    }
    /* the pinned table buffer is reused by every call: wait for the previous
     * upload from it to finish before rewriting it */
    mc_tables_wait(mc, 0);
    prof_mark(&prof, "t_sync");
    mc_enc_item *hit = (mc_enc_item *)htab;
    for (size_t i = 0; i < n; i++) {
        cplan *p = &P[i];
        mc_enc_item *I = &hit[i];
        memset(I, 0, sizeof(*I));
        I->cur = p->dev_in;
        I->hist_out = p->hist->dev;
        I->data_out = payload_dev + p->off_data;
        I->n = (int64_t)p->n;
        I->kind = p->kind;
        I->codec = p->dcodec;
        I->tile_kernels = p->tile_param;
        I->ntiles = p->ntiles;
        I->tile_base = p->tile_base;
        I->elem_bytes = (int32_t)mc_dtype_size(p->dt);
        I->step = p->local_step;
        I->wave = p->kind == MC_K_MOMENTUM ? p->wave : 0;
        I->vec = (((uintptr_t)I->cur | (uintptr_t)I->hist_out | (uintptr_t)I->data_out) & 15) == 0;
        I->lr = mc->config.momentum_lr;
        I->thr = mc->config.consistency_threshold;
        if (p->kind == MC_K_MOMENTUM) {
            cgroup *grp = &G[p->group];
            if (p->prev_item >= 0) I->prev = (const float *)P[p->prev_item].dev_in;
            else I->prev = (const float *)p->prev_t->dev;
            if (p->prev_item < 0 && p->prev_t->st_valid) {
                I->prev_known = 1;
                I->pm_known = p->prev_t->st_mean;
                I->ps_known = p->prev_t->st_std;
            }
            /* the first momentum item of a group reads the committed memory;
             * later ones continue in the group's new buffer */
            I->mem_in = p->wave == 0 ? (grp->mem_committed ? (const float *)grp->mem_committed->dev
                                                           : NULL)
                                     : (const float *)grp->mem_new->dev;
            I->mem_out = (float *)grp->mem_new->dev;
            I->vec = I->vec && (((uintptr_t)I->prev | (uintptr_t)I->mem_in | (uintptr_t)I->mem_out) & 15) == 0;
            I->K = (int64_t)p->K;
            I->ks = (int32_t)p->ks;
            I->ksdiv = mc_fastdiv_make((uint32_t)p->ks);
            size_t stride = ALIGN_UP(p->kwords, 64);
            I->bm_words = words + p->words_off;
            I->dom_words = words + p->words_off + stride;
            I->blk_pos = words + p->words_off + 2 * stride;
            I->max_blocks = (int32_t)p->nblk;
            I->bm_frame = payload_dev + p->off_bm;
            I->sg_frame = payload_dev + p->off_sg;
            I->sg_cap = (int64_t)p->cap_sg;
        } else if (p->kind == MC_K_FRAME || p->kind == MC_K_COPY) {
            I->n = (int64_t)p->bytes;   /* byte tiles */
        }
    }
    prof_mark(&prof, "t_items");
    if (!lhit) {
        /* per-wave tile lists: direct items run in wave 0, momentum items in
         * the wave of their position in the group's memory chain */
        for (int w = 0; w < nwaves; w++) {
            mc_tile_ref *la = (mc_tile_ref *)(htab + tab_items + 2 * tab_list * (size_t)w);
            mc_tile_ref *lm = (mc_tile_ref *)((uint8_t *)la + tab_list);
            int na = 0, nm = 0;
            for (size_t i = 0; i < n; i++) {
                cplan *p = &P[i];
                int in_wave = p->kind == MC_K_MOMENTUM ? p->wave == w : w == 0;
                if (!in_wave) continue;
                for (int t = 0; t < p->ntiles; t++) {
                    la[na].tile = p->tile_base + t;
                    la[na++].item = (int32_t)i;
                    if (p->kind == MC_K_MOMENTUM) {
                        lm[nm].tile = p->tile_base + t;
                        lm[nm++].item = (int32_t)i;
                    }
                }
            }
            lc->counts[2 * w] = na;
            lc->counts[2 * w + 1] = nm;
        }
        if (cudaMemcpyAsync(lc->dev, htab + tab_items, 2 * tab_list * (size_t)nwaves, cudaMemcpyHostToDevice,
                            st) != cudaSuccess) {
            rc = ERROR_COMPRESSION;
            goto fail;
        }
        lc->sig = sig;
    }
    prof_mark(&prof, "t_lists");
    if (cudaMemcpyAsync(dtab, htab, tab_items, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        mc_tables_mark(mc, 0, st) != 0 ||
        cudaMemsetAsync(results, 0, n * sizeof(mc_enc_result), st) != cudaSuccess) {
        rc = ERROR_COMPRESSION;
        goto fail;
    }

    prof_mark(&prof, "tables");
    /* ---------------------------------------------------------- launch */
    mc->last_launches = 0;
    mc_ktrace *tr = mc_trace_begin(mc);
    const int staged = !mc_env_off("FALCOM_STAGE");
    if (nchunks > 1) {
        /* chunked pipeline (one wave): per chunk, its input copies on the
         * upload stream, its kernels on the compute stream after them, its
         * payload download on the download stream after the kernels */
        int all0 = 0, mom0 = 0;
        for (int c = 0; c < nchunks; c++) {
            for (size_t r = 0; r < nruns; r++) {
                if (runs[r].chunk != c) continue;
                if (cudaMemcpyAsync(stage + runs[r].off, (const void *)runs[r].base, runs[r].end - runs[r].base,
                                    cudaMemcpyHostToDevice, mc->copy_in) != cudaSuccess) {
                    rc = ERROR_COMPRESSION;
                    mc_set_error(mc, "Batch compress: host-to-device copy failed");
                    goto fail;
                }
            }
            int na = 0, nm = 0;
            for (size_t i = cstart[c]; i < cstart[c + 1]; i++) {
                na += P[i].ntiles;
                if (P[i].kind == MC_K_MOMENTUM) nm += P[i].ntiles;
            }
            mc_enc_launch L;
            memset(&L, 0, sizeof(L));
            L.items = (const mc_enc_item *)dtab;
            L.results = results;
            L.item0 = (int32_t)cstart[c];
            L.nitems = (int32_t)(cstart[c + 1] - cstart[c]);
            L.all_tiles = (const uint8_t *)lc->dev + (size_t)all0 * sizeof(mc_tile_ref);
            L.nall_tiles = na;
            L.mom_tiles = (const uint8_t *)lc->dev + tab_list + (size_t)mom0 * sizeof(mc_tile_ref);
            L.nmom_tiles = nm;
            L.tiles = tiles;
            L.tile_poff = poff;
            L.staged = staged;
            L.wave = 0;
            all0 += na;
            mom0 += nm;
            if (cudaEventRecord(mc->ev_in[c], mc->copy_in) != cudaSuccess ||
                cudaStreamWaitEvent(st, mc->ev_in[c], 0) != cudaSuccess) {
                rc = ERROR_COMPRESSION;
                goto fail;
            }
            int k = L.nitems > 0 ? mc_launch_encode(&L, st, tr) : 0;
            if (k < 0) {
                rc = ERROR_COMPRESSION;
                mc_set_error(mc, "Batch compress: kernel launch failed: %s",
                             cudaGetErrorString(cudaGetLastError()));
                goto fail;
            }
            mc->last_launches += k;
            if (host_arena) {
                const size_t o0 = P[cstart[c]].off_data;
                const size_t o1 = c + 1 < nchunks ? P[cstart[c + 1]].off_data : arena_bytes;
                if (cudaEventRecord(mc->ev_done[c], st) != cudaSuccess ||
                    cudaStreamWaitEvent(mc->copy_out, mc->ev_done[c], 0) != cudaSuccess ||
                    cudaMemcpyAsync((uint8_t *)host_arena->ptr + o0, payload_dev + o0, o1 - o0,
                                    cudaMemcpyDeviceToHost, mc->copy_out) != cudaSuccess) {
                    rc = ERROR_COMPRESSION;
                    goto fail;
                }
            }
        }
    }
    for (int w = 0; nchunks == 1 && w < nwaves; w++) {
        uint8_t *dl = (uint8_t *)lc->dev + 2 * tab_list * (size_t)w;
        mc_enc_launch L;
        memset(&L, 0, sizeof(L));
        L.items = (const mc_enc_item *)dtab;
        L.results = results;
        L.item0 = 0;
        L.nitems = (int32_t)n;
        L.all_tiles = dl;
        L.nall_tiles = lc->counts[2 * w];
        L.mom_tiles = dl + tab_list;
        L.nmom_tiles = lc->counts[2 * w + 1];
        L.tiles = tiles;
        L.tile_poff = poff;
        L.staged = staged;
        L.wave = w;
        int k = mc_launch_encode(&L, st, tr);
        if (k < 0) {
            rc = ERROR_COMPRESSION;
            mc_set_error(mc, "Batch compress: kernel launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
            goto fail;
        }
        mc->last_launches += k;
    }
    mc->total_launches += mc->last_launches;

    /* ------------------------------------------------- results to host */
    mc_enc_result *hres = (mc_enc_result *)scratch_host(&mc->scratch, SH_RESULTS, n * sizeof(mc_enc_result));
    cudaMemcpyAsync(hres, results, n * sizeof(mc_enc_result), cudaMemcpyDeviceToHost, st);
    if (host_arena && nchunks == 1)
        cudaMemcpyAsync(host_arena->ptr, payload_dev, arena_bytes, cudaMemcpyDeviceToHost, st);
    prof_mark(&prof, "launch");
    /* while the GPU works: the result structs and every field that does not
     * depend on the device results (they live in one block owned by the
     * payload arena, released with it once the caller has freed every item) */
    {
        mc_arena *arena = dev_arena ? dev_arena : host_arena;
        uint8_t *base = (uint8_t *)arena->ptr;
        outs = (CompressedLayerData **)malloc((n ? n : 1) * sizeof(*outs));
        blk = (CompressedLayerData *)calloc(n ? n : 1, sizeof(CompressedLayerData));
        if (!outs || !blk) {
            rc = ERROR_ALLOCATION;
            goto fail;
        }
        for (size_t i = 0; i < n; i++) {
            cplan *p = &P[i];
            CompressedLayerData *c = outs[i] = &blk[i];
            /* fixed strings, all shorter than their fields */
            strcpy(c->type, p->mode == MODE_DIRECT ? "direct"
                                                   : (p->mode == MODE_MOMENTUM ? "momentum_predicted"
                                                                               : "direct_generic"));
            strcpy(c->codec, p->codec_tag);
            c->ndim = p->g->ndim;
            memcpy(c->shape, p->g->shape, p->g->ndim * sizeof(size_t));
            strcpy(c->original_dtype, mc_dtype_name(p->dt));
            strcpy(c->stored_dtype, c->original_dtype);
            c->step = p->local_step;
            c->data = base + p->off_data;
            if (p->kind == MC_K_MOMENTUM || p->kind == MC_K_QUANT) c->data_size = residual_bytes(p->dcodec, p->n);
            else if (p->kind == MC_K_COPY) c->data_size = p->bytes;
            else c->data_size = MC_ZHDR + 3 * frame_blocks(p->bytes) + p->bytes;
            if (p->kind == MC_K_MOMENTUM) c->bitmap = base + p->off_bm;
        }
    }
    prof_mark(&prof, "prefill");
    cudaError_t e = cudaStreamSynchronize(st);
    if (nchunks > 1) {
        const cudaError_t e2 = cudaStreamSynchronize(mc->copy_out);
        const cudaError_t e3 = cudaStreamSynchronize(mc->copy_in);
        if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3;
    }
    prof_mark(&prof, "sync");
    mc_trace_end(mc);
    if (e != cudaSuccess) {
        rc = ERROR_COMPRESSION;
        mc_set_error(mc, "Batch compress: device execution failed: %s", cudaGetErrorString(e));
        goto fail;
    }
    for (size_t i = 0; i < n; i++) {
        if (hres[i].err) {   /* a tile's bulk copies did not complete in time */
            rc = ERROR_COMPRESSION;
            mc_set_error(mc, "Batch compress: device tile staging timed out (item %zu)", i);
            goto fail;
        }
    }

    /* libzstd frame mode: the GPU frames (now in the host arena) are
     * decoded and written again by libzstd level 10, byte-identical to the
     * reference's frames */
    if (mc->frame_mode == MC_FRAME_LIBZSTD) {
        if (!zf_libzstd_available()) {
            rc = ERROR_COMPRESSION;
            mc_set_error(mc, "Batch compress: libzstd frame mode requested but libzstd.so.1 is missing");
            goto fail;
        }
        uint8_t *ha = (uint8_t *)host_arena->ptr;
        size_t tmp_cap = 0;
        for (size_t i = 0; i < n; i++) {
            size_t need = P[i].kind == MC_K_MOMENTUM ? (P[i].K + 7) / 8 : (P[i].kind == MC_K_FRAME ? P[i].bytes : 0);
            if (need > tmp_cap) tmp_cap = need;
        }
        uint8_t *tmp = (uint8_t *)malloc(tmp_cap + 16);
        if (!tmp) {
            rc = ERROR_ALLOCATION;
            goto fail;
        }
        int bad = 0;
        for (size_t i = 0; i < n && !bad; i++) {
            cplan *p = &P[i];
            size_t got = 0;
            if (p->kind == MC_K_MOMENTUM) {
                bad |= zf_decode_host(ha + p->off_bm, (size_t)hres[i].bm_size, tmp, tmp_cap + 16, &got) != 0;
                p->fs_bm = bad ? 0 : zf_libzstd_compress(ha + p->off_bm, p->cap_bm, tmp, got, 10);
                bad |= p->fs_bm == 0;
                if (!bad && hres[i].sg_size) {
                    bad |= zf_decode_host(ha + p->off_sg, (size_t)hres[i].sg_size, tmp, tmp_cap + 16, &got) != 0;
                    p->fs_sg = bad ? 0 : zf_libzstd_compress(ha + p->off_sg, p->cap_sg, tmp, got, 10);
                    bad |= p->fs_sg == 0;
                }
            } else if (p->kind == MC_K_FRAME) {
                size_t fsz = MC_ZHDR + 3 * frame_blocks(p->bytes) + p->bytes;
                bad |= zf_decode_host(ha + p->off_data, fsz, tmp, tmp_cap + 16, &got) != 0;
                p->fs_data = bad ? 0 : zf_libzstd_compress(ha + p->off_data, p->cap_data, tmp, got, 10);
                bad |= p->fs_data == 0;
            }
        }
        free(tmp);
        if (bad) {
            rc = ERROR_COMPRESSION;
            mc_set_error(mc, "Batch compress: libzstd framing failed");
            goto fail;
        }
    }

    /* -------------------------------------------- CompressedLayerData out */
    {
        mc_arena *arena = dev_arena ? dev_arena : host_arena;
        uint8_t *base = (uint8_t *)arena->ptr;
        arena->objs = blk;
        blk = NULL;
        const int libz = mc->frame_mode == MC_FRAME_LIBZSTD;
        for (size_t i = 0; i < n; i++) {
            cplan *p = &P[i];
            CompressedLayerData *c = outs[i];
            const mc_enc_result *r = &hres[i];
            if (libz && p->kind == MC_K_FRAME) c->data_size = p->fs_data;
            if (p->kind == MC_K_MOMENTUM) {
                c->bitmap_size = libz ? p->fs_bm : (size_t)r->bm_size;
                size_t sgs = libz ? p->fs_sg : (size_t)r->sg_size;
                c->dominant_signs = sgs ? base + p->off_sg : NULL;
                c->dominant_signs_size = sgs;
                c->num_predicted_kernels = (int)r->P;
                c->prediction_ratio = (float)r->P / (float)p->K;
                int64_t pel = r->P * (int64_t)p->ks;
                c->sign_mismatch_ratio = pel > 0 ? (float)r->mism / (float)pel : 0.0f;
                c->current_mean = r->cm;
                c->current_std = r->cs;
                c->prev_mean = r->pm;
                c->prev_std = r->ps;
                c->global_min = r->gmin;
                c->global_max = r->gmax;
            }
        }
        /* ------------------------------------------------------- commit */
        for (size_t g = 0; g < ng; g++) {
            if (!G[g].mem_new) continue;
            rec_commit(&G[g].mrec->t, &G[g].mrec->spare, G[g].mem_new);
            G[g].mem_new = NULL;
            map_put(mc->mem_clients, client, (void *)1);
        }
        for (size_t i = 0; i < n; i++) {
            mc_layer_rec *r = P[i].lrec;
            r->step++;
            /* a momentum item's history is an exact copy of its input, whose
             * |x| statistics the item just computed: the next round's
             * encode of this layer takes them instead of recomputing */
            if (P[i].hist) {
                P[i].hist->st_valid = P[i].kind == MC_K_MOMENTUM;
                P[i].hist->st_mean = hres[i].cm;
                P[i].hist->st_std = hres[i].cs;
            }
            /* the last item of a history key becomes the head (ref :2902) */
            rec_commit(&r->hist, &r->spare, P[i].hist);
            P[i].hist = NULL;
            mc_record_stats(mc, outs[i]);
            items[i].compressed = outs[i];
            items[i].error = ERROR_NONE;
        }
        registry_add_many((const void **)outs, n, arena);
        arena_retain(arena, (int)n - 1);
        free(outs);
        outs = NULL;
        if (n == 0) arena_release(arena);
    }
    prof_mark(&prof, "commit");
    prof_print(&prof, "compress");
    rc = ERROR_NONE;
    goto out;

fail:
    /* nothing may still be writing into memory that goes back to the pools */
    cudaStreamSynchronize(mc->stream);
    if (mc->copy_in) cudaStreamSynchronize(mc->copy_in);
    if (mc->copy_out) cudaStreamSynchronize(mc->copy_out);
    (void)cudaGetLastError();
    free_plan_tensors(mc, P, n, G, ng);
    if (dev_arena) arena_release(dev_arena);
    if (host_arena) arena_release(host_arena);
    for (size_t i = 0; i < n; i++) {
        items[i].compressed = NULL;
        if (items[i].error == ERROR_NONE) items[i].error = rc;
    }
out:
    free(outs);
    free(blk);
    free(runs);
    free(P);
    free(G);
    return rc;
}

/* ============================================================== decompress */
typedef struct {
    int ok;               /* planned successfully */
    int kind;             /* MC_D_* */
    int dcodec;
    DataType dt;
    size_t ndim, shape[MAX_NDIM], n, bytes, K, ks;
    mc_layer_rec *lrec;       /* "client:layer" record (history) */
    mc_mem_rec *mrec;         /* decoder prediction memory record */
    mc_tensor *prev;          /* decoder history head (MOMENTUM) */
    mc_tensor *mem_in;
    mc_tensor *mem_new;
    mc_tensor *hist;
    /* payload sources */
    const uint8_t *data;      /* data bytes as passed (host or device) */
    size_t data_size;
    const uint8_t *bm;
    size_t bm_size;
    const uint8_t *sg;
    size_t sg_size;
    int data_frame;           /* data is a zstd frame (lossless content) */
    /* device addresses after staging */
    const uint8_t *d_data, *d_bm, *d_sg;
    /* content buffers (device) */
    size_t c_data_off, c_bm_off, c_sg_off;
    int j_data, j_bm, j_sg;   /* unframe job indices, -1 when none */
    size_t out_off;
    int tile_base, ntiles, tile_param;
    int bm_mode, sg_mode;     /* MC_BM_* */
    int data_mode;            /* lossless frame: MC_BM_* */
    size_t sg_len;            /* sign content bytes of a Raw-block sign frame */
    int foreign;              /* a frame lives in device memory the library does not own */
    float *agg;               /* fused aggregate region of this item (float32 items), NULL */
    size_t agg_off;           /* its element offset in the aggregate */
    int agg_only;             /* decoded into the aggregate only: no output array */
    const char *why;
} dplan;

typedef struct {
    const uint8_t *src;
    size_t len;
    const uint8_t **dst;      /* where the device address is written */
    int chunk;                /* pipeline chunk of the item */
} hrange;

/* one host-to-device copy of staged payload bytes */
typedef struct {
    uintptr_t base;
    size_t len;
    uint8_t *dst;
    int chunk;
} dec_run;

/* Plans one item (reference decompress_layer :3476-3598 validation order). */
static void dplan_item(MomentumCompressor *mc, dplan *d, const BatchItem *it, const mc_keycache *kc,
                       size_t idx) {
    const CompressedLayerData *c = it->compressed;
    d->ok = 0;
    d->j_data = d->j_bm = d->j_sg = -1;
    if (!c || !it->layer_name || !*it->layer_name) { d->why = "NULL compressed data or layer name"; return; }
    if (!c->type[0]) { d->why = "compressed type is empty"; return; }
    if (c->ndim < MIN_NDIM || c->ndim > MAX_NDIM) { d->why = "invalid ndim"; return; }
    if (!c->data || c->data_size == 0) { d->why = "compressed data is empty"; return; }
    if (mc_dtype_parse(c->original_dtype, &d->dt) != 0) { d->why = "unknown original dtype"; return; }
    d->ndim = c->ndim;
    d->n = 1;
    for (size_t i = 0; i < c->ndim; i++) {
        d->shape[i] = c->shape[i];
        d->n *= c->shape[i];
    }
    if (d->n == 0) { d->why = "empty shape"; return; }
    d->bytes = d->n * mc_dtype_size(d->dt);
    d->lrec = kc->lrec[idx];
    d->mrec = kc->mrec[idx];
    d->data = c->data;
    d->data_size = c->data_size;
    const char *codec = c->codec;
    int is_direct = strcmp(c->type, "direct") == 0 || strcmp(c->type, "direct_generic") == 0;
    int is_mom = strcmp(c->type, "momentum_predicted") == 0;
    if (!is_direct && !is_mom) { d->why = "unknown compression type"; return; }

    /* residual / data codec */
    if (strcmp(codec, "q8") == 0 || strcmp(codec, "int4") == 0) {
        if (d->dt != DTYPE_FLOAT32) { d->why = "quantised payload for a non-float32 tensor"; return; }
        d->dcodec = codec[0] == 'q' ? MC_DC_Q8 : MC_DC_INT4;
        if (c->data_size != residual_bytes(d->dcodec, d->n)) { d->why = "size mismatch"; return; }
        d->kind = MC_D_QUANT;
    } else if (strcmp(codec, "sz3_memcpy") == 0) {
        if (c->data_size != d->bytes) { d->why = "size mismatch"; return; }
        d->dcodec = MC_DC_RAW;
        d->kind = MC_D_COPY;
    } else if (strcmp(codec, "zstd") == 0 || strcmp(codec, "blosc") == 0) {
        /* blosc is decoded as zstd, as the reference does without USE_BLOSC */
        d->data_frame = 1;
        d->dcodec = MC_DC_RAW;
        d->kind = MC_D_COPY;
    } else if (strcmp(codec, "pickle") == 0) {
        /* "PICKLE\0\0" + u64 size + bytes (reference :714-745) */
        if (c->data_size < 16 || memcmp(c->data, "PICKLE\0\0", 8) != 0) { d->why = "invalid pickle header"; return; }
        uint64_t sz;
        memcpy(&sz, c->data + 8, 8);
        if (sz + 16 != c->data_size || sz != d->bytes) { d->why = "size mismatch"; return; }
        d->data = c->data + 16;
        d->data_size = sz;
        d->dcodec = MC_DC_RAW;
        d->kind = MC_D_COPY;
    } else {
        d->why = "unsupported codec";
        return;
    }

    if (is_mom) {
        if (d->dt != DTYPE_FLOAT32 || d->ndim != 4) { d->why = "momentum layer must be 4-D float32"; return; }
        d->K = d->shape[0] * d->shape[1];
        d->ks = d->shape[2] * d->shape[3];
        if (d->kind == MC_D_COPY && !d->data_frame) d->kind = MC_D_RESIDUAL;  /* raw floats */
        if (d->kind == MC_D_QUANT) d->kind = MC_D_RESIDUAL;
        if (d->data_frame) { d->why = "zstd-coded momentum residual is not supported"; return; }
        d->bm = c->bitmap;
        d->bm_size = c->bitmap ? c->bitmap_size : 0;
        d->sg = c->dominant_signs;
        d->sg_size = c->dominant_signs ? c->dominant_signs_size : 0;
        mc_tensor *h = d->lrec->hist;
        int hist_ok = h && h->dtype == DTYPE_FLOAT32 && h->ndim == 4 && h->n == d->n;
        for (size_t i = 0; hist_ok && i < 4; i++) hist_ok = h->shape[i] == d->shape[i];
        if (d->bm_size > 0 && hist_ok) {
            d->kind = MC_D_MOMENTUM;
            d->prev = h;
            d->mem_in = d->mrec->t;
        }
    } else if (d->kind == MC_D_QUANT) {
        /* direct tensor through the quantiser */
    }
    d->ok = 1;
}

/* In-place reading mode of a frame of `size` bytes whose content is known to
 * be `content` bytes: all Raw blocks, all RLE blocks, or neither. */
static int frame_mode_for(size_t size, size_t content, int inplace) {
    if (!inplace) return MC_BM_WORDS;
    const size_t nb = frame_blocks(content);
    if (size == MC_ZHDR + 3 * nb + content) return MC_BM_RAW;
    if (content >= 2 && size == MC_ZHDR + 4 * nb) return MC_BM_RLE;
    return MC_BM_WORDS;
}

/* Content bytes of an all-Raw frame of `size` bytes, or 0 when no content
 * length fits that size. */
static size_t sign_content_len(size_t size) {
    if (size <= MC_ZHDR + 3) return 0;
    const size_t nb = (size - MC_ZHDR + MC_ZBLOCK + 2) / (MC_ZBLOCK + 3);
    if (nb == 0 || size < MC_ZHDR + 3 * nb) return 0;
    const size_t s = size - MC_ZHDR - 3 * nb;
    return (s > 0 && frame_blocks(s) == nb) ? s : 0;
}


#define DEC_RETRY_EXPAND 1
static int dec_segment(MomentumCompressor *mc, const BatchItem *items, size_t n, const char *client,
                       NDArray **out, int out_loc, size_t *n_ok, int force_expand, size_t base) {
    cudaStream_t st = mc->stream;
    const int dev = mc->device;
    int nch = 1;
    size_t dstart[MC_MAX_CHUNKS + 1];
    dstart[0] = 0;
    dstart[1] = n;
    dec_run *runs = NULL;
    size_t nruns = 0;
    dplan *D = (dplan *)calloc(n, sizeof(dplan));
    if (!D) return ERROR_ALLOCATION;
    int rc = ERROR_NONE;
    prof_t prof = {0};
    prof.on = mc_env_flag("FALCOM_PROFILE");
    prof_mark(&prof, "start");
    /* keys and state records of every item (cached across rounds) */
    const mc_keycache *dkc = NULL;
    {
        mc_keyreq *req = (mc_keyreq *)malloc(n * sizeof(mc_keyreq));
        static const size_t one = 1;
        if (!req) { free(D); return ERROR_ALLOCATION; }
        for (size_t i = 0; i < n; i++) {
            const CompressedLayerData *c = items[i].compressed;
            DataType dt = DTYPE_FLOAT32;
            if (c) mc_dtype_parse(c->original_dtype, &dt);
            int ok = c && items[i].layer_name && c->ndim >= MIN_NDIM && c->ndim <= MAX_NDIM;
            req[i].name = items[i].layer_name ? items[i].layer_name : "";
            req[i].dt = dt;
            req[i].ndim = ok ? c->ndim : 1;
            req[i].shape = ok ? c->shape : &one;
        }
        dkc = keycache_get(mc, mc->dec_kc, client, req, n, &rc);
        free(req);
        if (rc != ERROR_NONE) { free(D); return rc; }
    }
    for (size_t i = 0; i < n; i++) {
        out[i] = NULL;
        dplan_item(mc, &D[i], &items[i], dkc, i);
        if (!D[i].ok)
            fprintf(stderr, "[ERROR] Batch decompress: item '%s': %s\n",
                    items[i].layer_name ? items[i].layer_name : "(null)", D[i].why);
    }

    prof_mark(&prof, "plan");
    /* ---------------------------------------------- payload residency */
    /* host payload ranges are copied to the device (adjacent ranges merged);
     * frames with compressed blocks are decoded on the host first */
    /* chunked pipeline: items split by decoded bytes when the call moves
     * payloads or outputs between host and device */
    if (!force_expand && mc_pipeline_init(mc) == 0) {
        size_t *ob = (size_t *)malloc(n * sizeof(size_t));
        if (ob) {
            for (size_t i = 0; i < n; i++) ob[i] = D[i].ok ? D[i].bytes : 0;
            nch = chunk_items(ob, n, dstart);
            free(ob);
        }
    }
    size_t nr = 0;
    hrange *R = (hrange *)calloc(3 * n + 1, sizeof(hrange));
    uint8_t **host_dec = (uint8_t **)calloc(3 * n + 1, sizeof(uint8_t *));
    size_t nhd = 0;
    if (!R || !host_dec) { rc = ERROR_ALLOCATION; goto done; }
    mc_ptrcache pc;
    pc.n = 0;
    for (size_t i = 0; i < n; i++) {
        dplan *d = &D[i];
        if (!d->ok) continue;
        const uint8_t *srcs[3] = {d->data, d->kind == MC_D_MOMENTUM ? d->bm : NULL,
                                  d->kind == MC_D_MOMENTUM ? d->sg : NULL};
        size_t lens[3] = {d->data_size, d->bm_size, d->sg_size};
        const uint8_t **dsts[3] = {&d->d_data, &d->d_bm, &d->d_sg};
        int is_frame[3] = {d->data_frame, 1, 1};
        for (int k = 0; k < 3; k++) {
            if (!srcs[k] || lens[k] == 0) continue;
            int pd = -1, in_arena = 0;
            if (mc_classify2(&pc, srcs[k], &pd, &in_arena) && pd == dev) {
                *dsts[k] = srcs[k];
                if (!in_arena) d->foreign = 1;
                continue;
            }
            const uint8_t *src = srcs[k];
            size_t len = lens[k];
            if (is_frame[k] && !zf_is_simple(src, len)) {
                /* compressed blocks: decode with libzstd on the host */
                unsigned long long cs = 0;
                if (zf_content_size(src, len, &cs) != 0 || cs > (1ull << 40)) {
                    if (k == 0) { d->ok = 0; d->why = "zstd decompression failed"; }
                    else if (k == 1) d->kind = MC_D_RESIDUAL;
                    else d->sg = NULL, d->sg_size = 0;
                    continue;
                }
                size_t cap = (size_t)cs + 16;
                uint8_t *buf = (uint8_t *)malloc(cap);
                size_t got = 0;
                if (!buf || zf_decode_host(src, len, buf, cap, &got) != 0) {
                    free(buf);
                    if (k == 0) { d->ok = 0; d->why = "zstd decompression failed"; }
                    else if (k == 1) d->kind = MC_D_RESIDUAL;
                    else d->sg = NULL, d->sg_size = 0;
                    continue;
                }
                /* re-frame as a raw frame so the device path reads it */
                uint8_t *fr = (uint8_t *)malloc(zf_max_frame_size(got));
                if (!fr) { free(buf); rc = ERROR_ALLOCATION; goto done; }
                size_t fl = zf_write_raw_host(fr, buf, got);
                free(buf);
                host_dec[nhd++] = fr;
                src = fr;
                len = fl;
                if (k == 0) d->data_size = fl;
                else if (k == 1) d->bm_size = fl;
                else d->sg_size = fl;
            }
            R[nr].src = src;
            R[nr].len = len;
            R[nr].dst = dsts[k];
            R[nr].chunk = 0;
            while (R[nr].chunk + 1 < nch && i >= dstart[R[nr].chunk + 1]) R[nr].chunk++;
            nr++;
        }
    }
    /* momentum items whose bitmap turned out unusable fall back to residual only */
    /* stage host ranges: sorted by (chunk, address), ranges with gaps below
     * 64 KiB merged within a chunk; the copies are recorded and issued at
     * launch time (per chunk when the call is pipelined) */
    if (nr) {
        for (size_t a = 1; a < nr; a++) {
            hrange v = R[a];
            size_t b = a;
            while (b > 0 && (R[b - 1].chunk > v.chunk ||
                             (R[b - 1].chunk == v.chunk && (uintptr_t)R[b - 1].src > (uintptr_t)v.src))) {
                R[b] = R[b - 1];
                b--;
            }
            R[b] = v;
        }
        size_t total = 0;
        for (size_t a = 0; a < nr;) {
            uintptr_t base = (uintptr_t)R[a].src, end = base + R[a].len;
            size_t b = a + 1;
            while (b < nr && R[b].chunk == R[a].chunk && (uintptr_t)R[b].src <= end + 65536) {
                uintptr_t e2 = (uintptr_t)R[b].src + R[b].len;
                if (e2 > end) end = e2;
                b++;
            }
            total = ALIGN_UP(total + (base & 15) + (end - base), SLOT_ALIGN);
            a = b;
        }
        uint8_t *stage = (uint8_t *)scratch_dev(&mc->scratch, SD_DSTAGE, total + 256);
        runs = (dec_run *)malloc(nr * sizeof(dec_run));
        if (!stage || !runs) { rc = ERROR_ALLOCATION; goto done; }
        size_t off = 0;
        for (size_t a = 0; a < nr;) {
            uintptr_t base = (uintptr_t)R[a].src, end = base + R[a].len;
            size_t b = a + 1;
            while (b < nr && R[b].chunk == R[a].chunk && (uintptr_t)R[b].src <= end + 65536) {
                uintptr_t e2 = (uintptr_t)R[b].src + R[b].len;
                if (e2 > end) end = e2;
                b++;
            }
            /* keep the source's 16-byte phase so 4-byte fields stay aligned */
            size_t phase = base & 15;
            uint8_t *dst = stage + off + phase;
            runs[nruns].base = base;
            runs[nruns].len = end - base;
            runs[nruns].dst = dst;
            runs[nruns].chunk = R[a].chunk;
            nruns++;
            for (size_t c = a; c < b; c++) *R[c].dst = dst + ((uintptr_t)R[c].src - base);
            off = ALIGN_UP(off + phase + (end - base), SLOT_ALIGN);
            a = b;
        }
    }

    prof_mark(&prof, "stage");
    /* ------------------------------------------ tiles, contents, outputs */
    int ntiles = 0, nmom_tiles = 0, njobs = 0;
    size_t content_bytes = 0, out_bytes = 0;
    for (size_t i = 0; i < n; i++) {
        dplan *d = &D[i];
        if (!d->ok) continue;
        if (d->kind == MC_D_MOMENTUM) {
            d->tile_param = tile_kernels_for(d->ks, d->K);
            d->ntiles = (int)((d->K + (size_t)d->tile_param - 1) / (size_t)d->tile_param);
            nmom_tiles += d->ntiles;
            size_t wb = ALIGN_UP(((d->K + 31) / 32 + 1) * 4 + 4096, 256);
            /* Frames made only of Raw blocks, or only of RLE blocks, are read
             * in place (the kernel checks every header it relies on; a
             * mismatch re-runs the segment with expansion); anything else is
             * expanded first.  In place only inside library-owned or staged
             * memory: a word read may touch up to 3 bytes past the frame. */
            const size_t c = (d->K + 7) / 8;
            const int inplace = !force_expand && !d->foreign;
            d->bm_mode = frame_mode_for(d->bm_size, c, inplace);
            if (d->bm_mode == MC_BM_WORDS) {
                d->c_bm_off = content_bytes;
                content_bytes += wb;
                d->j_bm = njobs++;
            }
            d->sg_mode = MC_BM_WORDS;
            if (d->d_sg) {
                d->sg_len = sign_content_len(d->sg_size);
                if (inplace && d->sg_len > 0) d->sg_mode = MC_BM_RAW;
                if (d->sg_mode == MC_BM_WORDS) {
                    d->c_sg_off = content_bytes;
                    content_bytes += wb;
                    d->j_sg = njobs++;
                }
            }
        } else if (d->kind == MC_D_COPY) {
            d->tile_param = TILE_ELEMS * 4;
            d->ntiles = (int)((d->bytes + (size_t)d->tile_param - 1) / (size_t)d->tile_param);
            d->data_mode = MC_BM_WORDS;
            if (d->data_frame) {
                d->data_mode = frame_mode_for(d->data_size, d->bytes, !force_expand && !d->foreign);
                if (d->data_mode == MC_BM_WORDS) {
                    d->c_data_off = content_bytes;
                    content_bytes += ALIGN_UP(d->bytes + 16, 256);
                    d->j_data = njobs++;
                }
            }
        } else {
            d->tile_param = TILE_ELEMS;
            d->ntiles = (int)((d->n + TILE_ELEMS - 1) / TILE_ELEMS);
        }
        d->tile_base = ntiles;
        ntiles += d->ntiles;
        /* float32 items with an aggregate offset are added into the fused
         * aggregate by the reconstruct kernel; without decode outputs they
         * get no output slot */
        if (mc->agg && d->dt == DTYPE_FLOAT32 && base + i < mc->agg_n) {
            d->agg = mc->agg + mc->agg_off[base + i];
            d->agg_off = mc->agg_off[base + i];
            d->agg_only = mc->agg_no_output;
            /* sharded: every element must fall in a shard, quads must not
             * straddle two (offsets and shards are multiples of 4) */
            if (mc->agg_shards.nranks > 0 &&
                (d->agg_off % 4 != 0 ||
                 d->agg_off + d->n > (size_t)mc->agg_shards.nranks * (size_t)mc->agg_shards.shard)) {
                mc_set_error(mc, "Batch decompress: item %zu's aggregate region [%zu, %zu) does not fit the %d "
                                 "shards of %lld elements (offsets must be multiples of 4)", base + i,
                             d->agg_off, d->agg_off + d->n, mc->agg_shards.nranks,
                             (long long)mc->agg_shards.shard);
                rc = ERROR_INVALID_PARAM;
                goto done;
            }
        }
        d->out_off = out_bytes;
        if (!d->agg_only) out_bytes = ALIGN_UP(out_bytes + d->bytes, SLOT_ALIGN);
    }
    uint8_t *content = content_bytes ? (uint8_t *)scratch_dev(&mc->scratch, SD_DCONTENT, content_bytes) : NULL;
    mc_arena *oarena = NULL;
    uint8_t *dout;
    if (out_loc == FALCOM_LOC_DEVICE) {
        oarena = arena_acquire(out_bytes, dev);
        dout = oarena ? (uint8_t *)oarena->ptr : NULL;
    } else {
        dout = (uint8_t *)scratch_dev(&mc->scratch, SD_DOUT, out_bytes + 256);
        oarena = arena_acquire(out_bytes, -1);
    }
    if ((content_bytes && !content) || !dout || !oarena) { rc = ERROR_ALLOCATION; goto fail_arena; }
    for (size_t i = 0; i < n; i++) {
        dplan *d = &D[i];
        if (!d->ok) continue;
        d->hist = rec_take(&d->lrec->spare, d->dt, d->ndim, d->shape, dev);
        if (!d->hist) { rc = ERROR_ALLOCATION; goto fail_arena; }
        if (d->kind == MC_D_MOMENTUM) {
            d->mem_new = rec_take(&d->mrec->spare, DTYPE_FLOAT32, 4, d->shape, dev);
            if (!d->mem_new) { rc = ERROR_ALLOCATION; goto fail_arena; }
        }
    }

    prof_mark(&prof, "alloc");
    /* ------------------------------------------------------- tables */
    /* host upload: [items][frame jobs]; device: the same, then job lengths,
     * results, per-tile counts and offsets; the tile lists (all tiles,
     * momentum tiles) come from the list cache for a recent structure */
    size_t t_items = ALIGN_UP(n * sizeof(mc_dec_item), 256);
    size_t t_tiles = ALIGN_UP((size_t)(ntiles + 1) * sizeof(mc_tile_ref), 256);
    size_t t_jobs = ALIGN_UP((size_t)(njobs + 1) * sizeof(mc_unframe_job), 256);
    size_t t_lens = ALIGN_UP((size_t)(njobs + 1) * 8, 256);
    size_t t_res = ALIGN_UP(n * sizeof(mc_dec_result), 256);
    size_t t_count = ALIGN_UP((size_t)(ntiles + 1) * 4, 256);
    size_t t_poff = ALIGN_UP((size_t)(ntiles + 1) * 8, 256);
    size_t tab = t_items + t_jobs;
    size_t dyn = t_lens + t_res + t_count + t_poff;
    uint64_t sig = sig_mix(0xBB67AE8584CAA73Bull, (uint64_t)n);
    for (size_t i = 0; i < n; i++)
        sig = sig_mix(sig, D[i].ok ? (((uint64_t)D[i].kind << 40) ^ (uint64_t)(uint32_t)D[i].ntiles) : ~0ull);
    int lhit = 0;
    mc_listcache *lc = lists_get(mc, mc->dec_lists, sig, 2, 2 * t_tiles, &lhit);
    uint8_t *ht = (uint8_t *)scratch_host(&mc->scratch, SH_TABLES, tab + t_lens + t_res + (lhit ? 0 : 2 * t_tiles));
    uint8_t *dt = (uint8_t *)scratch_dev(&mc->scratch, SD_TABLES, tab + dyn);
    if (!ht || !dt || !lc) { rc = ERROR_ALLOCATION; goto fail_arena; }
    prof_mark(&prof, "t_scratch");
    mc_tables_wait(mc, 0);
    prof_mark(&prof, "t_sync");
    if (njobs) memset(ht + t_items, 0, t_jobs);
    mc_dec_item *hi = (mc_dec_item *)ht;
    mc_unframe_job *h_jobs = (mc_unframe_job *)(ht + t_items);
    mc_tile_ref *h_all = (mc_tile_ref *)(ht + tab + t_lens + t_res);
    mc_tile_ref *h_mom = (mc_tile_ref *)(ht + tab + t_lens + t_res + t_tiles);
    int64_t *d_lens = (int64_t *)(dt + tab);
    mc_dec_result *d_res = (mc_dec_result *)(dt + tab + t_lens);
    int32_t *d_count = (int32_t *)(dt + tab + t_lens + t_res);
    int64_t *d_poff = (int64_t *)(dt + tab + t_lens + t_res + t_count);
    int na = 0, nm = 0;
    for (size_t i = 0; i < n; i++) {
        dplan *d = &D[i];
        mc_dec_item *I = &hi[i];
        memset(I, 0, sizeof(*I));
        if (!d->ok) continue;
        I->kind = d->kind;
        I->codec = d->dcodec;
        I->n = (int64_t)(d->kind == MC_D_COPY ? d->bytes : d->n);
        I->tile_kernels = d->tile_param;
        I->ntiles = d->ntiles;
        I->tile_base = d->tile_base;
        I->elem_bytes = (int32_t)mc_dtype_size(d->dt);
        I->hist_out = d->hist->dev;
        I->out = d->agg_only ? NULL : dout + d->out_off;
        if (d->agg) {
            I->agg = d->agg;
            I->agg_w = mc->agg_w;
            I->agg_store = mc->agg_store;
            I->agg_vec = (((uintptr_t)d->agg) & 15) == 0;
            I->agg_shard = mc->agg_shards.nranks > 0;
            I->agg_off = (int64_t)d->agg_off;
        }
        if (d->dcodec == MC_DC_Q8 || d->dcodec == MC_DC_INT4) {
            I->scale_ptr = (const float *)d->d_data;
            I->data = d->d_data + 4;
        } else {
            I->data = d->d_data;
        }
        if (d->data_frame && d->data_mode != MC_BM_WORDS) {
            I->data_mode = d->data_mode;
            I->data_frame = d->d_data;
            I->data = d->d_data + MC_ZHDR + 3;
        }
        if (d->j_data >= 0) {
            mc_unframe_job *J = &h_jobs[d->j_data];
            J->frame = d->d_data;
            J->frame_size = (int64_t)d->data_size;
            J->dst = content + d->c_data_off;
            J->cap = (int64_t)d->bytes;
            J->content_out = d_lens + d->j_data;
            I->data = content + d->c_data_off;
        }
        if (d->kind == MC_D_MOMENTUM) {
            const CompressedLayerData *c = items[i].compressed;
            I->K = (int64_t)d->K;
            I->ks = (int32_t)d->ks;
            I->ksdiv = mc_fastdiv_make((uint32_t)d->ks);
            I->prev = (const float *)d->prev->dev;
            I->mem_in = d->mem_in ? (const float *)d->mem_in->dev : NULL;
            I->mem_out = (float *)d->mem_new->dev;
            I->cm = c->current_mean;
            I->cs = c->current_std;
            I->pm = c->prev_mean;
            I->ps = c->prev_std;
            I->lr = mc->config.momentum_lr;
            I->bm_mode = d->bm_mode;
            I->sg_mode = d->sg_mode;
            I->bm_bits = (int64_t)d->K;
            if (d->bm_mode == MC_BM_WORDS) {
                mc_unframe_job *J = &h_jobs[d->j_bm];
                J->frame = d->d_bm;
                J->frame_size = (int64_t)d->bm_size;
                J->dst = content + d->c_bm_off;
                J->cap = (int64_t)(((d->K + 31) / 32 + 1) * 4 + 4096);
                J->content_out = d_lens + d->j_bm;
                I->bm_words = (const uint32_t *)(content + d->c_bm_off);
                I->bm_len_ptr = d_lens + d->j_bm;
            } else {
                I->bm_frame = d->d_bm;
            }
            if (d->j_sg >= 0) {
                mc_unframe_job *J = &h_jobs[d->j_sg];
                J->frame = d->d_sg;
                J->frame_size = (int64_t)d->sg_size;
                J->dst = content + d->c_sg_off;
                J->cap = (int64_t)(((d->K + 31) / 32 + 1) * 4 + 4096);
                J->content_out = d_lens + d->j_sg;
                I->sg_bytes = content + d->c_sg_off;
                I->sg_len_ptr = d_lens + d->j_sg;
            } else if (d->sg_mode == MC_BM_RAW) {
                I->sg_frame = d->d_sg;
                I->sg_len = (int64_t)d->sg_len;
            }
        }
        {
            uintptr_t need = (d->kind == MC_D_COPY || I->codec == MC_DC_RAW || I->codec == MC_DC_Q8_RAW ||
                              I->codec == MC_DC_INT4_RAW) ? 15 : (I->codec == MC_DC_Q8 ? 3 : 1);
            uintptr_t al = (uintptr_t)I->hist_out | (uintptr_t)I->out | (uintptr_t)I->mem_in |
                           (uintptr_t)I->mem_out | (uintptr_t)I->prev;
            I->vec = ((al & 15) == 0) && (((uintptr_t)I->data & need) == 0);
        }
        if (!lhit) {
            for (int t = 0; t < d->ntiles; t++) {
                h_all[na].tile = d->tile_base + t;
                h_all[na++].item = (int32_t)i;
                if (d->kind == MC_D_MOMENTUM) {
                    h_mom[nm].tile = d->tile_base + t;
                    h_mom[nm++].item = (int32_t)i;
                }
            }
        }
    }
    prof_mark(&prof, "t_fill");
    if (!lhit) {
        lc->counts[0] = na;
        lc->counts[1] = nm;
        if (cudaMemcpyAsync(lc->dev, ht + tab + t_lens + t_res, 2 * t_tiles, cudaMemcpyHostToDevice, st) !=
            cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
        lc->sig = sig;
    }
    if (cudaMemcpyAsync(dt, ht, tab, cudaMemcpyHostToDevice, st) != cudaSuccess || mc_tables_mark(mc, 0, st) != 0 ||
        cudaMemsetAsync(d_res, 0, t_res, st) != cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }

    prof_mark(&prof, "tables");
    /* ------------------------------------------------------- launch */
    mc->last_launches = 0;
    mc_ktrace *tr = mc_trace_begin(mc);
    /* pipelined only without frame expansion jobs and with bytes to move */
    const int pipelined = nch > 1 && njobs == 0 && (nruns > 0 || out_loc != FALCOM_LOC_DEVICE);
    const int dstaged = !mc_env_off("FALCOM_STAGE");
    if (!pipelined) {
        for (size_t r = 0; r < nruns; r++)
            if (cudaMemcpyAsync(runs[r].dst, (const void *)runs[r].base, runs[r].len, cudaMemcpyHostToDevice, st) !=
                cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
        if (njobs) {
            /* bitmaps must decode into clean zero-padded words */
            if (content_bytes) cudaMemsetAsync(content, 0, content_bytes, st);
            int k = mc_launch_unframe((const mc_unframe_job *)(dt + t_items), njobs, st, tr);
            if (k < 0) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
            mc->last_launches += k;
        }
        mc_dec_launch L;
        memset(&L, 0, sizeof(L));
        L.items = (const mc_dec_item *)dt;
        L.results = d_res;
        L.nitems = (int32_t)n;
        L.all_tiles = lc->dev;
        L.nall_tiles = lc->counts[0];
        L.mom_tiles = (uint8_t *)lc->dev + t_tiles;
        L.nmom_tiles = lc->counts[1];
        L.tile_count = d_count;
        L.tile_poff = d_poff;
        L.staged = dstaged;
        L.shards = mc->agg_shards;
        L.item0 = 0;
        L.item1 = (int32_t)n;
        int k = mc_launch_decode(&L, st, tr);
        if (k < 0) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
        mc->last_launches += k;
    } else {
        /* per chunk: its payload copies on the upload stream, its kernels on
         * the compute stream after them, its decoded outputs downloaded on
         * the download stream after the kernels */
        int all0 = 0, mom0 = 0;
        for (int c = 0; c < nch; c++) {
            for (size_t r = 0; r < nruns; r++) {
                if (runs[r].chunk != c) continue;
                if (cudaMemcpyAsync(runs[r].dst, (const void *)runs[r].base, runs[r].len, cudaMemcpyHostToDevice,
                                    mc->copy_in) != cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
            }
            int na = 0, nm = 0;
            size_t o0 = (size_t)-1, o1 = 0;
            for (size_t i = dstart[c]; i < dstart[c + 1]; i++) {
                if (!D[i].ok) continue;
                na += D[i].ntiles;
                if (D[i].kind == MC_D_MOMENTUM) nm += D[i].ntiles;
                if (D[i].agg_only) continue;
                if (o0 == (size_t)-1) o0 = D[i].out_off;
                o1 = D[i].out_off + D[i].bytes;
            }
            if (cudaEventRecord(mc->ev_in[c], mc->copy_in) != cudaSuccess ||
                cudaStreamWaitEvent(st, mc->ev_in[c], 0) != cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
            mc_dec_launch L;
            memset(&L, 0, sizeof(L));
            L.items = (const mc_dec_item *)dt;
            L.results = d_res;
            L.nitems = (int32_t)n;
            L.all_tiles = (const uint8_t *)lc->dev + (size_t)all0 * sizeof(mc_tile_ref);
            L.nall_tiles = na;
            L.mom_tiles = (const uint8_t *)lc->dev + t_tiles + (size_t)mom0 * sizeof(mc_tile_ref);
            L.nmom_tiles = nm;
            L.tile_count = d_count;
            L.tile_poff = d_poff;
            L.staged = dstaged;
            L.shards = mc->agg_shards;
            L.item0 = (int32_t)dstart[c];
            L.item1 = (int32_t)dstart[c + 1];
            all0 += na;
            mom0 += nm;
            int k = mc_launch_decode(&L, st, tr);
            if (k < 0) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
            mc->last_launches += k;
            if (out_loc != FALCOM_LOC_DEVICE && o0 != (size_t)-1) {
                if (cudaEventRecord(mc->ev_done[c], st) != cudaSuccess ||
                    cudaStreamWaitEvent(mc->copy_out, mc->ev_done[c], 0) != cudaSuccess ||
                    cudaMemcpyAsync((uint8_t *)oarena->ptr + o0, dout + o0, o1 - o0, cudaMemcpyDeviceToHost,
                                    mc->copy_out) != cudaSuccess) { rc = ERROR_DECOMPRESSION; goto fail_arena; }
            }
        }
    }
    mc->total_launches += mc->last_launches;

    /* ------------------------------------------------- back to the host */
    int64_t *h_lens = (int64_t *)(ht + tab);
    mc_dec_result *h_res = (mc_dec_result *)(ht + tab + t_lens);
    if (njobs) cudaMemcpyAsync(h_lens, d_lens, (size_t)njobs * 8, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(h_res, d_res, n * sizeof(mc_dec_result), cudaMemcpyDeviceToHost, st);
    if (out_loc != FALCOM_LOC_DEVICE && out_bytes && !pipelined)
        cudaMemcpyAsync(oarena->ptr, dout, out_bytes, cudaMemcpyDeviceToHost, st);
    prof_mark(&prof, "launch");
    cudaError_t e = cudaStreamSynchronize(st);
    if (pipelined) {
        const cudaError_t e2 = cudaStreamSynchronize(mc->copy_out);
        const cudaError_t e3 = cudaStreamSynchronize(mc->copy_in);
        if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3;
    }
    prof_mark(&prof, "sync");
    mc_trace_end(mc);
    if (e != cudaSuccess) {
        mc_set_error(mc, "Batch decompress: device execution failed: %s", cudaGetErrorString(e));
        rc = ERROR_DECOMPRESSION;
        goto fail_arena;
    }

    /* an in-place frame that was not what its size suggested: redo the
     * segment with every frame expanded (nothing is committed yet) */
    for (size_t i = 0; i < n; i++) {
        if (D[i].ok && h_res[i].err >= 2) {   /* a tile's bulk copies did not complete in time */
            mc_set_error(mc, "Batch decompress: device tile staging timed out (item %zu)", i);
            rc = ERROR_DECOMPRESSION;
            goto fail_arena;
        }
    }
    for (size_t i = 0; i < n; i++) {
        if (D[i].ok && h_res[i].err) {
            if (prof.on)
                fprintf(stderr, "[falcom-profile] decompress: in-place frame check failed for item %zu "
                                "(kind %d bm %d sg %d data %d, sizes %zu/%zu/%zu); expanding\n", i, D[i].kind,
                        D[i].bm_mode, D[i].sg_mode, D[i].data_mode, D[i].data_size, D[i].bm_size, D[i].sg_size);
            rc = DEC_RETRY_EXPAND;
            goto fail_arena;
        }
    }

    /* ------------------------------------------------------- commit */
    int handed = 0;
    for (size_t i = 0; i < n; i++) {
        dplan *d = &D[i];
        if (!d->ok) continue;
        if (d->j_data >= 0 && h_lens[d->j_data] != (int64_t)d->bytes) {
            fprintf(stderr, "[ERROR] Size mismatch: got %lld, expected %zu\n",
                    (long long)h_lens[d->j_data], d->bytes);
            d->ok = 0;
            continue;
        }
        if (d->agg_only) {
            /* decoded into the aggregate only: no array, the state commits */
            (*n_ok)++;
        } else {
        if (!oarena->objs) {   /* arrays and shapes: one block owned by the output arena */
            oarena->objs = calloc(n, sizeof(NDArray) + MAX_NDIM * sizeof(size_t));
            if (!oarena->objs) { rc = ERROR_ALLOCATION; goto fail_arena; }
        }
        NDArray *a = (NDArray *)oarena->objs + i;
        size_t *shp = (size_t *)((NDArray *)oarena->objs + n) + i * MAX_NDIM;
        memcpy(shp, d->shape, d->ndim * sizeof(size_t));
        a->data = (uint8_t *)oarena->ptr + d->out_off;
        a->shape = shp;
        a->ndim = d->ndim;
        a->total_size = d->n;
        a->dtype = d->dt;
        out[i] = a;
        handed++;
        (*n_ok)++;
        }
        int commit_hist = 1;
        if (d->kind == MC_D_MOMENTUM) {
            /* reference :3266-3269: no predicted kernel -> residual returned,
             * neither memory nor history touched */
            if (h_res[i].P == 0) commit_hist = 0;
            else {
                rec_commit(&d->mrec->t, &d->mrec->spare, d->mem_new);
                d->mem_new = NULL;
                map_put(mc->mem_clients, client, (void *)1);
            }
        } else if (d->kind == MC_D_RESIDUAL) {
            commit_hist = 0;
        }
        if (commit_hist) {
            rec_commit(&d->lrec->hist, &d->lrec->spare, d->hist);
            d->hist = NULL;
        }
    }
    {
        const void **objs = (const void **)malloc(n * sizeof(void *));
        size_t no = 0;
        for (size_t i = 0; objs && i < n; i++)
            if (out[i]) objs[no++] = out[i];
        if (objs) registry_add_many(objs, no, oarena);
        else
            for (size_t i = 0; i < n; i++)
                if (out[i]) registry_add(out[i], oarena);
        free(objs);
    }
    if (handed > 0) arena_retain(oarena, handed - 1);
    else arena_release(oarena);
    oarena = NULL;
    prof_mark(&prof, "commit");
    prof_print(&prof, "decompress");
    if (prof.on) {
        int nb[3] = {0, 0, 0}, ns[3] = {0, 0, 0}, nd[3] = {0, 0, 0};
        for (size_t i = 0; i < n; i++) {
            if (!D[i].ok) continue;
            if (D[i].kind == MC_D_MOMENTUM) {
                nb[D[i].bm_mode]++;
                if (D[i].d_sg) ns[D[i].sg_mode]++;
            }
            if (D[i].data_frame) nd[D[i].data_mode]++;
        }
        int nf = 0;
        for (size_t i = 0; i < n; i++) nf += D[i].foreign;
        fprintf(stderr, "[falcom-profile] decompress frames: force_expand=%d foreign=%d jobs=%d bitmap "
                        "words/raw/rle=%d/%d/%d signs=%d/%d/%d data=%d/%d/%d\n", force_expand, nf, njobs,
                nb[0], nb[1], nb[2], ns[0], ns[1], ns[2], nd[0], nd[1], nd[2]);
    }

fail_arena:
    if (rc != ERROR_NONE) {   /* nothing may still write into memory going back to the pools */
        cudaStreamSynchronize(st);
        if (mc->copy_in) cudaStreamSynchronize(mc->copy_in);
        if (mc->copy_out) cudaStreamSynchronize(mc->copy_out);
        (void)cudaGetLastError();
    }
    if (oarena) arena_release(oarena);
    for (size_t i = 0; i < n; i++) {
        if (D[i].hist) {
            if (D[i].lrec && !D[i].lrec->spare) D[i].lrec->spare = D[i].hist;
            else tensor_drop(D[i].hist);
        }
        if (D[i].mem_new) {
            if (D[i].mrec && !D[i].mrec->spare) D[i].mrec->spare = D[i].mem_new;
            else tensor_drop(D[i].mem_new);
        }
    }
done:
    for (size_t i = 0; i < nhd; i++) free(host_dec[i]);
    free(host_dec);
    free(runs);
    free(R);
    free(D);
    return rc;
}

int mc_decompress_items(MomentumCompressor *mc, const BatchItem *items, size_t n,
                        const char *client, NDArray **out, int out_loc) {
    /* Items that share a history key with an earlier item of the call run in
     * a later segment, after the earlier one's state is committed, so the
     * serial semantics of the reference decoder hold. */
    size_t ok = 0;
    size_t a = 0;
    int rc = ERROR_NONE;
    strtab seen;
    if (strtab_init(&seen, n)) return ERROR_ALLOCATION;
    while (a < n) {
        size_t b = a;
        /* a segment ends before the first repeated layer name */
        for (; b < n; b++) {
            const char *nm = items[b].layer_name ? items[b].layer_name : "";
            int *s = strtab_slot(&seen, nm, (int)a - 1);
            if (*s == (int)a) break;   /* already in this segment */
            *s = (int)a;
        }
        if (b == a) b = a + 1;
        int r = dec_segment(mc, items + a, b - a, client, out + a, out_loc, &ok, 0, a);
        if (r == DEC_RETRY_EXPAND) {
            /* the first attempt's reconstruct kernel already added into the
             * aggregate: in add mode the retry cannot undo that, so the
             * call reports the aggregate as invalid (store mode rewrites
             * the same values) */
            if (mc->agg && !mc->agg_store) {
                mc_set_error(mc, "Batch decompress: aggregate invalid (frames re-read after a failed check)");
                mc->agg_failed = 1;
            }
            r = dec_segment(mc, items + a, b - a, client, out + a, out_loc, &ok, 1, a);
        }
        if (r != ERROR_NONE) {
            rc = r;
            for (size_t j = a; j < b; j++) {
                if (out[j]) { ndarray_destroy(out[j]); out[j] = NULL; }
            }
        }
        a = b;
    }
    strtab_free(&seen);
    (void)rc;
    if (mc->agg_failed) {
        mc->agg_failed = 0;
        return ERROR_DECOMPRESSION;
    }
    if (ok == 0) return ERROR_DECOMPRESSION;
    if (ok < n) return -((int)n - (int)ok);
    return ERROR_NONE;
}
