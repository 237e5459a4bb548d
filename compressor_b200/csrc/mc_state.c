/*
 * mc_state.c -- per-client keyed state of one compressor instance.
 *
 * The reference keeps three uthash tables (momentum_compressor_openmp_simd_final.c
 * :420-471): step counts and gradient histories keyed "client:layer", and
 * prediction memories keyed by client then "layer|dtype|conv_(shape)".  Here
 * the step count and the latest history tensor of a "client:layer" live in one
 * stable record (mc_layer_rec), and every prediction memory in another
 * (mc_mem_rec); both hold device tensors plus one spare buffer that the next
 * round reuses, so a steady-state round allocates nothing.  Only the latest
 * history entry is kept: it is the only one any code path reads.
 *
 * A batch key cache remembers, for the last batch seen by an engine, the
 * keys and records of every item; a round with the same tensor list (names,
 * dtypes, shapes, client) skips key formatting and hashing entirely.
 */
#define _GNU_SOURCE
#include <stdlib.h>
#include <string.h>

#include "mc_internal.h"

mc_layer_rec *state_layer(MomentumCompressor *mc, const char *hkey, int create) {
    mc_layer_rec *r = (mc_layer_rec *)map_get(mc->layers, hkey);
    if (r || !create) return r;
    r = (mc_layer_rec *)calloc(1, sizeof(mc_layer_rec));
    if (!r) return NULL;
    if (map_put(mc->layers, hkey, r) != 0) {
        free(r);
        return NULL;
    }
    return r;
}

mc_mem_rec *state_mem(MomentumCompressor *mc, const char *mkey, int create) {
    mc_mem_rec *r = (mc_mem_rec *)map_get(mc->memory, mkey);
    if (r || !create) return r;
    r = (mc_mem_rec *)calloc(1, sizeof(mc_mem_rec));
    if (!r) return NULL;
    if (map_put(mc->memory, mkey, r) != 0) {
        free(r);
        return NULL;
    }
    return r;
}

void layer_rec_drop(void *p) {
    mc_layer_rec *r = (mc_layer_rec *)p;
    if (!r) return;
    tensor_drop(r->hist);
    tensor_drop(r->spare);
    free(r);
}

void mem_rec_drop(void *p) {
    mc_mem_rec *r = (mc_mem_rec *)p;
    if (!r) return;
    tensor_drop(r->t);
    tensor_drop(r->spare);
    free(r);
}

static int same_layout(const mc_tensor *t, DataType dt, size_t ndim, const size_t *shape) {
    if (t->dtype != dt || t->ndim != ndim) return 0;
    for (size_t i = 0; i < ndim; i++)
        if (t->shape[i] != shape[i]) return 0;
    return 1;
}

/* A device tensor of the given layout: the record's spare buffer when it
 * fits, a pooled buffer otherwise. */
mc_tensor *rec_take(mc_tensor **spare, DataType dt, size_t ndim, const size_t *shape, int device) {
    if (spare && *spare) {
        mc_tensor *s = *spare;
        s->st_valid = 0;   /* about to be rewritten */
        if (same_layout(s, dt, ndim, shape)) {
            *spare = NULL;
            return s;
        }
        size_t n = 1;
        for (size_t i = 0; i < ndim; i++) n *= shape[i];
        if (n * mc_dtype_size(dt) == s->bytes) {   /* same bytes: relabel */
            *spare = NULL;
            s->dtype = dt;
            s->ndim = ndim;
            s->n = n;
            memcpy(s->shape, shape, ndim * sizeof(size_t));
            return s;
        }
    }
    return tensor_new(dt, ndim, shape, device);
}

/* Installs t as the committed tensor; the previous one becomes the spare. */
void rec_commit(mc_tensor **slot, mc_tensor **spare, mc_tensor *t) {
    mc_tensor *old = *slot;
    *slot = t;
    if (old) {
        tensor_drop(*spare);
        *spare = old;
    }
}

/* ------------------------------------------------------------ key cache */
void keycache_free(mc_keycache *kc) {
    if (kc->names)
        for (size_t i = 0; i < kc->n; i++) free(kc->names[i]);
    free(kc->names);
    free(kc->dt);
    free(kc->ndim);
    free(kc->shape);
    free(kc->hkey);
    free(kc->lkey);
    free(kc->lrec);
    free(kc->mrec);
    free(kc->same);
    free(kc->first_l);
    free(kc->first_h);
    free(kc->lossy);
    memset(kc, 0, sizeof(*kc));
}

static int keycache_hit(const MomentumCompressor *mc, const mc_keycache *kc, const char *client,
                        const mc_keyreq *req, size_t n) {
    if (!kc->valid || kc->gen != mc->state_gen || kc->n != n || strcmp(kc->client, client) != 0) return 0;
    for (size_t i = 0; i < n; i++) {
        if (kc->dt[i] != req[i].dt || kc->ndim[i] != req[i].ndim) return 0;
        const size_t *s = kc->shape + i * MAX_NDIM;
        for (size_t d = 0; d < req[i].ndim; d++)
            if (s[d] != req[i].shape[d]) return 0;
        if (strcmp(kc->names[i], req[i].name) != 0) return 0;
    }
    return 1;
}

static int keycache_resolve(MomentumCompressor *mc, mc_keycache *kc, const char *client, const mc_keyreq *req,
                            size_t n) {
    keycache_free(kc);
    kc->names = (char **)calloc(n, sizeof(char *));
    kc->dt = (DataType *)calloc(n, sizeof(DataType));
    kc->ndim = (size_t *)calloc(n, sizeof(size_t));
    kc->shape = (size_t *)calloc(n * MAX_NDIM, sizeof(size_t));
    kc->hkey = (char(*)[MAX_KEY_LENGTH])calloc(n, MAX_KEY_LENGTH);
    kc->lkey = (char(*)[MAX_KEY_LENGTH])calloc(n, MAX_KEY_LENGTH);
    kc->lrec = (mc_layer_rec **)calloc(n, sizeof(void *));
    kc->mrec = (mc_mem_rec **)calloc(n, sizeof(void *));
    kc->same = (int *)calloc(n, sizeof(int));
    kc->first_l = (int *)calloc(n, sizeof(int));
    kc->first_h = (int *)calloc(n, sizeof(int));
    kc->lossy = (int *)calloc(n, sizeof(int));
    kc->n = n;
    if (!kc->names || !kc->dt || !kc->ndim || !kc->shape || !kc->hkey || !kc->lkey || !kc->lrec ||
        !kc->mrec || !kc->same || !kc->first_l || !kc->first_h || !kc->lossy) {
        keycache_free(kc);
        return ERROR_ALLOCATION;
    }
    snprintf(kc->client, sizeof(kc->client), "%s", client);
    mc_map *hmap = map_new(), *lmap = map_new();
    if (!hmap || !lmap) {
        map_free(hmap, NULL);
        map_free(lmap, NULL);
        keycache_free(kc);
        return ERROR_ALLOCATION;
    }
    int rc = ERROR_NONE;
    for (size_t i = 0; i < n && rc == ERROR_NONE; i++) {
        kc->names[i] = strdup(req[i].name);
        kc->dt[i] = req[i].dt;
        kc->ndim[i] = req[i].ndim;
        memcpy(kc->shape + i * MAX_NDIM, req[i].shape, req[i].ndim * sizeof(size_t));
        mc_history_key(kc->hkey[i], client, req[i].name);
        mc_layer_key(kc->lkey[i], MAX_KEY_LENGTH, req[i].name, req[i].shape, req[i].ndim, req[i].dt);
        char mk[2 * MAX_KEY_LENGTH];
        mc_memory_key(mk, sizeof(mk), client, kc->lkey[i]);
        kc->lrec[i] = state_layer(mc, kc->hkey[i], 1);
        kc->mrec[i] = state_mem(mc, mk, 1);
        size_t elems = 1;
        for (size_t d = 0; d < req[i].ndim; d++) elems *= req[i].shape[d];
        kc->lossy[i] = mc_should_lossy(req[i].name, elems, req[i].dt, mc->config.param_count_threshold);
        /* first item with the same history key / layer key (1-based in the maps) */
        intptr_t fh = (intptr_t)map_get(hmap, kc->hkey[i]);
        if (!fh) {
            map_put(hmap, kc->hkey[i], (void *)(intptr_t)(i + 1));
            fh = (intptr_t)(i + 1);
        }
        kc->first_h[i] = (int)fh - 1;
        intptr_t fl = (intptr_t)map_get(lmap, kc->lkey[i]);
        if (!fl) {
            map_put(lmap, kc->lkey[i], (void *)(intptr_t)(i + 1));
            fl = (intptr_t)(i + 1);
        }
        kc->first_l[i] = (int)fl - 1;
        if (!kc->names[i] || !kc->lrec[i] || !kc->mrec[i]) rc = ERROR_ALLOCATION;
    }
    for (size_t i = 0; i < n && rc == ERROR_NONE; i++) kc->same[kc->first_h[i]]++;
    for (size_t i = 0; i < n && rc == ERROR_NONE; i++) kc->same[i] = kc->same[kc->first_h[i]];
    map_free(hmap, NULL);
    map_free(lmap, NULL);
    if (rc != ERROR_NONE) {
        keycache_free(kc);
        return rc;
    }
    kc->gen = mc->state_gen;
    kc->valid = 1;
    return ERROR_NONE;
}

/* The cache of this batch: a slot that matches it, else the least recently
 * used slot rebuilt.  NULL with *rc set when rebuilding fails. */
mc_keycache *keycache_get(MomentumCompressor *mc, mc_keycache *set, const char *client, const mc_keyreq *req,
                          size_t n, int *rc) {
    mc_keycache *victim = &set[0];
    for (int i = 0; i < MC_KC_SLOTS; i++) {
        mc_keycache *kc = &set[i];
        if (keycache_hit(mc, kc, client, req, n)) {
            kc->used = ++mc->kc_tick;
            *rc = ERROR_NONE;
            return kc;
        }
        if (!kc->valid) {
            if (victim->valid) victim = kc;
        } else if (victim->valid && kc->used < victim->used) {
            victim = kc;
        }
    }
    *rc = keycache_resolve(mc, victim, client, req, n);
    if (*rc != ERROR_NONE) return NULL;
    victim->used = ++mc->kc_tick;
    return victim;
}
