/*
 * mc_internal.h -- shared types of the host side of libmomentum_compressor.so.
 *
 * Host code is C11; device work is issued through the launchers declared at
 * the end of this file (implemented in mc_kernels.cu).
 */
#ifndef MC_INTERNAL_H
#define MC_INTERNAL_H

#include <pthread.h>
#include <stdint.h>
#include <stdio.h>

#include <cuda_runtime_api.h>

#include "falcom_b200.h"
#include "momentum_compressor.h"
#include "mc_device.h"

#define MC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ maps */
/* Open-addressing string-keyed hash map (keys are copied). */
typedef struct mc_map {
    char **keys;
    void **vals;
    size_t cap;   /* power of two */
    size_t len;
    size_t tomb;
} mc_map;

mc_map *map_new(void);
void map_free(mc_map *m, void (*drop)(void *));
void *map_get(const mc_map *m, const char *key);
int map_put(mc_map *m, const char *key, void *val);   /* 0 ok, -1 OOM; replaces */
void *map_del(mc_map *m, const char *key);            /* returns removed value */
#define MAP_TOMB ((char *)1)
#define MAP_LIVE(m, i) ((m)->keys[i] && (m)->keys[i] != MAP_TOMB)

/* ------------------------------------------------------------- buffers */
/* Arena of library-owned output memory (pinned host or device), reference
 * counted by the CompressedLayerData / NDArray objects that point into it. */
typedef struct mc_arena {
    void *ptr;
    size_t bytes;
    int device;      /* -1 for pinned host memory */
    int refs;
    void *objs;      /* malloc'd block holding the objects themselves, freed with the arena */
} mc_arena;

mc_arena *arena_acquire(size_t bytes, int device);   /* refs = 1 */
void arena_release(mc_arena *a);
void arena_release_n(mc_arena *a, int k);                      /* refs--, pooled at 0 */
void arena_retain(mc_arena *a, int n);

/* Ownership registry of returned objects. */
void registry_add(const void *obj, mc_arena *a);
void registry_add_many(const void **objs, size_t n, mc_arena *a);
mc_arena *registry_take(const void *obj, int *found);
void registry_take_many(const void *const *objs, size_t n, mc_arena **arenas);

/* Device buffers held by state entries (pooled per device by byte size). */
void *dbuf_get(int device, size_t bytes);
void dbuf_put(int device, void *ptr, size_t bytes);

/* ------------------------------------------------------------- state */
typedef struct {
    DataType dtype;
    size_t ndim;
    size_t shape[MAX_NDIM];
    size_t n;          /* elements */
    size_t bytes;
    int device;
    void *dev;         /* device copy */
    /* mean and population std of |x| of exactly these values as a momentum
     * encode computed them (st_valid 1), set when the encode commits the
     * tensor as a layer's history head; 0 for any other writer */
    int st_valid;
    float st_mean, st_std;
} mc_tensor;

mc_tensor *tensor_new(DataType dt, size_t ndim, const size_t *shape, int device);
void tensor_drop(void *t);   /* for map_free; NULL is ignored */

/* Step count and latest history tensor of one "client:layer". */
typedef struct {
    int step;
    mc_tensor *hist;     /* committed history head, NULL when none */
    mc_tensor *spare;    /* previous head, reused by the next round */
} mc_layer_rec;

/* One prediction memory ("client" + "layer|dtype|conv_(shape)"). */
typedef struct {
    mc_tensor *t;        /* committed memory, NULL when none */
    mc_tensor *spare;
} mc_mem_rec;

/* Keys and records of every item of one batch an engine saw.  An engine
 * keeps MC_KC_SLOTS of them (one per recent client, least recently used
 * replaced), so a server decoding many clients in turn hits as well. */
#define MC_KC_SLOTS 64
typedef struct {
    int valid;
    unsigned gen;
    unsigned long long used;        /* tick of the last hit */
    char client[256];
    size_t n;
    char **names;
    DataType *dt;
    size_t *ndim;
    size_t *shape;                  /* n x MAX_NDIM */
    char (*hkey)[MAX_KEY_LENGTH];   /* "client:layer" */
    char (*lkey)[MAX_KEY_LENGTH];   /* "layer|dtype|conv_(...)" */
    mc_layer_rec **lrec;
    mc_mem_rec **mrec;              /* memory record of (client, lkey) */
    int *same;                      /* items sharing the history key */
    int *first_l, *first_h;         /* first item with the same layer / history key */
    int *lossy;                     /* reference :399-415 routing */
} mc_keycache;

typedef struct {
    const char *name;
    DataType dt;
    size_t ndim;
    const size_t *shape;
} mc_keyreq;

/* Device-resident tile lists of a recent batch structure: a call whose
 * per-item plan (kinds, tile counts, waves) hashes to `sig` reuses them. */
#define MC_LIST_CACHE 8
typedef struct {
    uint64_t sig;             /* 0: empty */
    unsigned long long used;
    void *dev;                /* nlists lists of list_bytes each */
    size_t bytes;
    int nlists;
    int *counts;              /* entries of every list */
} mc_listcache;

struct MomentumCompressor {
    CompressorConfig config;
    char current_client_id[256];
    int log_level;
    int device;
    cudaStream_t stream;
    cudaStream_t own_stream;
    /* chunked host<->device pipelines: copy streams and per-chunk events
     * (created on first use) */
#define MC_MAX_CHUNKS 8
    cudaStream_t copy_in, copy_out;
    cudaEvent_t ev_in[MC_MAX_CHUNKS], ev_done[MC_MAX_CHUNKS];
    /* recorded after the last upload from the pinned table buffer: a call
     * waits on it (not on the whole stream) before rewriting the buffer */
    cudaEvent_t tab_ev[1];
    int tab_ev_live[1];
    int residual_codec;      /* MC_CODEC_* */
    int frame_mode;          /* MC_FRAME_GPU / MC_FRAME_LIBZSTD */
    int payload_loc;
    int output_loc;

    mc_map *layers;          /* "client:layer" -> mc_layer_rec* */
    mc_map *memory;          /* "client\x1f<layer|dtype|conv_(...)>" -> mc_mem_rec* */
    mc_map *mem_clients;     /* clients that own a prediction-memory table */
    unsigned state_gen;      /* bumped when records are deleted (resets) */
    mc_keycache enc_kc[MC_KC_SLOTS], dec_kc[MC_KC_SLOTS];
    unsigned long long kc_tick;
    mc_listcache enc_lists[MC_LIST_CACHE], dec_lists[MC_LIST_CACHE];
    unsigned long long lc_tick;

    struct {
        size_t total_compressions;
        float *prediction_ratios;
        size_t pr_count, pr_cap;
        float *sign_mismatch_ratios;
        size_t sm_count, sm_cap;
    } stats;

    char last_error[256];
    int last_launches;
    long long total_launches;

    /* reusable scratch (grown on demand) */
    mc_scratch scratch;

    /* server-side aggregate (falcom_set_aggregate): decoded float32 item i
     * of every batch decompress is added, times agg_w, at agg + agg_off[i],
     * by the reconstruct kernel itself */
    float *agg;
    size_t *agg_off;
    size_t agg_n;
    float agg_w;
    int agg_store;      /* 1: the next batches store weight * decoded instead of adding */
    int agg_no_output;  /* 1: items added into the aggregate get no decoded array */
    mc_agg_shards agg_shards;   /* nranks > 0: sharded aggregate (falcom_set_aggregate_shards) */
    int agg_failed;

    /* per-kernel device time (falcom_set_kernel_timing) */
    int ktiming;
    mc_ktrace ktrace;
    double ktime_ms[MC_NKERN];
    long long kcount[MC_NKERN];
};

/* pinned table buffer k: wait for / mark the last upload from it */
void mc_tables_wait(MomentumCompressor *mc, int k);
int mc_tables_mark(MomentumCompressor *mc, int k, cudaStream_t st);

/* kernel timing: start a trace for one call / fold it into the totals after
 * the call's stream synchronisation */
mc_ktrace *mc_trace_begin(MomentumCompressor *mc);
void mc_trace_end(MomentumCompressor *mc);

enum { MC_CODEC_Q8 = 0, MC_CODEC_INT4, MC_CODEC_RAW, MC_CODEC_Q8_RAW, MC_CODEC_INT4_RAW };
enum { MC_FRAME_GPU = 0, MC_FRAME_LIBZSTD = 1 };

/* ------------------------------------------------------------- helpers */
size_t mc_dtype_size(DataType dt);
const char *mc_dtype_name(DataType dt);
int mc_dtype_parse(const char *s, DataType *out);
void mc_history_key(char *out, const char *client, const char *layer);
void mc_layer_key(char *out, size_t cap, const char *layer, const size_t *shape, size_t ndim,
                  DataType dt);
void mc_memory_key(char *out, size_t cap, const char *client, const char *layer_key);
int mc_should_lossy(const char *name, size_t n, DataType dt, size_t threshold);
int mc_env_flag(const char *name);
int mc_env_off(const char *name);
void mc_set_error(MomentumCompressor *mc, const char *fmt, ...);
void mc_log(const MomentumCompressor *mc, int level, const char *fmt, ...);
int mc_ptr_is_device(const void *p, int *device);
#define MC_PTRCACHE 32
typedef struct {
    struct {
        uintptr_t lo, hi;
        int device;
        int arena;   /* 1: memory the library allocated for outputs */
    } r[MC_PTRCACHE];
    int n;
} mc_ptrcache;
int mc_classify(mc_ptrcache *pc, const void *p, int *device);
/* as mc_classify; *in_arena = 1 when p lies in library-owned output memory */
int mc_classify2(mc_ptrcache *pc, const void *p, int *device, int *in_arena);
int mc_is_arena_ptr(const void *p);   /* inside memory the library allocated for outputs */
void mc_record_stats(MomentumCompressor *mc, const CompressedLayerData *c);

/* zstd frames (mc_wire.c) */
size_t zf_max_frame_size(size_t content);
size_t zf_write_raw_host(uint8_t *dst, const uint8_t *src, size_t n);  /* raw/RLE */
int zf_content_size(const uint8_t *frame, size_t n, unsigned long long *out);
int zf_decode_host(const uint8_t *frame, size_t n, uint8_t *dst, size_t cap, size_t *out);
int zf_is_simple(const uint8_t *frame, size_t n);   /* raw/RLE blocks only */
int zf_libzstd_available(void);
size_t zf_libzstd_compress(uint8_t *dst, size_t cap, const uint8_t *src, size_t n, int level);

/* state records and key cache (mc_state.c) */
mc_layer_rec *state_layer(MomentumCompressor *mc, const char *hkey, int create);
mc_mem_rec *state_mem(MomentumCompressor *mc, const char *mkey, int create);
void layer_rec_drop(void *r);
void mem_rec_drop(void *r);
mc_tensor *rec_take(mc_tensor **spare, DataType dt, size_t ndim, const size_t *shape, int device);
void rec_commit(mc_tensor **slot, mc_tensor **spare, mc_tensor *t);
void keycache_free(mc_keycache *kc);
mc_keycache *keycache_get(MomentumCompressor *mc, mc_keycache *set, const char *client, const mc_keyreq *req,
                          size_t n, int *rc);

/* copy streams and events of the chunked pipelines; 0 on success */
int mc_pipeline_init(MomentumCompressor *mc);

/* tile-list cache (mc_batch.c) */
void listcache_free(MomentumCompressor *mc, mc_listcache *set);

/* batch engines (mc_batch.c) */
int mc_compress_grouped(MomentumCompressor *mc, BatchItem *items, size_t n, const char *client,
                        int payload_loc, int allow_fault);
int mc_decompress_items(MomentumCompressor *mc, const BatchItem *items, size_t n,
                        const char *client, NDArray **out, int out_loc);

#endif
