/*
 * mc_util.c -- containers, memory pools, ownership registry and small helpers
 * of the host side.
 */
#define _GNU_SOURCE
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include "mc_internal.h"

/* ===================================================================== maps */
static uint64_t hash_str(const char *s) {
    /* FNV-1a 64 */
    uint64_t h = 1469598103934665603ull;
    while (*s) {
        h ^= (unsigned char)*s++;
        h *= 1099511628211ull;
    }
    return h;
}

mc_map *map_new(void) {
    mc_map *m = (mc_map *)calloc(1, sizeof(mc_map));
    if (!m) return NULL;
    m->cap = 64;
    m->keys = (char **)calloc(m->cap, sizeof(char *));
    m->vals = (void **)calloc(m->cap, sizeof(void *));
    if (!m->keys || !m->vals) {
        free(m->keys);
        free(m->vals);
        free(m);
        return NULL;
    }
    return m;
}

void map_free(mc_map *m, void (*drop)(void *)) {
    if (!m) return;
    for (size_t i = 0; i < m->cap; i++) {
        if (MAP_LIVE(m, i)) {
            if (drop) drop(m->vals[i]);
            free(m->keys[i]);
        }
    }
    free(m->keys);
    free(m->vals);
    free(m);
}

static size_t map_find(const mc_map *m, const char *key) {
    size_t mask = m->cap - 1, i = (size_t)hash_str(key) & mask;
    for (;;) {
        char *k = m->keys[i];
        if (!k) return (size_t)-1;
        if (k != MAP_TOMB && strcmp(k, key) == 0) return i;
        i = (i + 1) & mask;
    }
}

void *map_get(const mc_map *m, const char *key) {
    size_t i = map_find(m, key);
    return i == (size_t)-1 ? NULL : m->vals[i];
}

static int map_grow(mc_map *m) {
    size_t ncap = m->cap * 2;
    char **nk = (char **)calloc(ncap, sizeof(char *));
    void **nv = (void **)calloc(ncap, sizeof(void *));
    if (!nk || !nv) {
        free(nk);
        free(nv);
        return -1;
    }
    for (size_t i = 0; i < m->cap; i++) {
        if (!MAP_LIVE(m, i)) continue;
        size_t j = (size_t)hash_str(m->keys[i]) & (ncap - 1);
        while (nk[j]) j = (j + 1) & (ncap - 1);
        nk[j] = m->keys[i];
        nv[j] = m->vals[i];
    }
    free(m->keys);
    free(m->vals);
    m->keys = nk;
    m->vals = nv;
    m->cap = ncap;
    m->tomb = 0;
    return 0;
}

int map_put(mc_map *m, const char *key, void *val) {
    size_t i = map_find(m, key);
    if (i != (size_t)-1) {
        m->vals[i] = val;
        return 0;
    }
    if ((m->len + m->tomb + 1) * 4 >= m->cap * 3 && map_grow(m) != 0) return -1;
    char *k = strdup(key);
    if (!k) return -1;
    size_t mask = m->cap - 1;
    i = (size_t)hash_str(key) & mask;
    while (MAP_LIVE(m, i)) i = (i + 1) & mask;
    if (m->keys[i] == MAP_TOMB) m->tomb--;
    m->keys[i] = k;
    m->vals[i] = val;
    m->len++;
    return 0;
}

void *map_del(mc_map *m, const char *key) {
    size_t i = map_find(m, key);
    if (i == (size_t)-1) return NULL;
    void *v = m->vals[i];
    free(m->keys[i]);
    m->keys[i] = MAP_TOMB;
    m->vals[i] = NULL;
    m->len--;
    m->tomb++;
    return v;
}

/* ============================================================ fast divide */
mc_fastdiv mc_fastdiv_make(uint32_t d) {
    mc_fastdiv f;
    uint32_t s = 0;
    while (((uint64_t)1 << s) < d) s++;
    f.shift = s;
    f.mul = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << s) - d)) / d + 1);
    if (d == 1) f.mul = 0;
    return f;
}

/* ====================================================== device buffer pool */
typedef struct pool_ent {
    void *ptr;
    size_t bytes;
    int device;
    struct pool_ent *next;
} pool_ent;

static pthread_mutex_t g_pool_mu = PTHREAD_MUTEX_INITIALIZER;
#define DPOOL_BUCKETS 1024
static pool_ent *g_dpool[DPOOL_BUCKETS];   /* free device buffers, by exact size */
static pool_ent *g_hpool = NULL;           /* free pinned / device arenas */

static size_t dpool_bucket(int device, size_t bytes) {
    uint64_t x = (uint64_t)bytes * 0x9E3779B97F4A7C15ull ^ (uint64_t)(device + 7);
    return (size_t)(x >> 54) & (DPOOL_BUCKETS - 1);
}

void *dbuf_get(int device, size_t bytes) {
    if (bytes == 0) bytes = 16;
    size_t b = dpool_bucket(device, bytes);
    pthread_mutex_lock(&g_pool_mu);
    for (pool_ent **pp = &g_dpool[b]; *pp; pp = &(*pp)->next) {
        if ((*pp)->device == device && (*pp)->bytes == bytes) {
            pool_ent *e = *pp;
            *pp = e->next;
            pthread_mutex_unlock(&g_pool_mu);
            void *p = e->ptr;
            free(e);
            return p;
        }
    }
    pthread_mutex_unlock(&g_pool_mu);
    void *p = NULL;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        /* release cached buffers of this device and retry once */
        (void)cudaGetLastError();
        pthread_mutex_lock(&g_pool_mu);
        for (size_t k = 0; k < DPOOL_BUCKETS; k++) {
            pool_ent **q = &g_dpool[k];
            while (*q) {
                if ((*q)->device == device) {
                    pool_ent *e = *q;
                    *q = e->next;
                    cudaFree(e->ptr);
                    free(e);
                } else {
                    q = &(*q)->next;
                }
            }
        }
        pthread_mutex_unlock(&g_pool_mu);
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            (void)cudaGetLastError();
            return NULL;
        }
    }
    return p;
}

void dbuf_put(int device, void *ptr, size_t bytes) {
    if (!ptr) return;
    if (bytes == 0) bytes = 16;
    pool_ent *e = (pool_ent *)malloc(sizeof(pool_ent));
    if (!e) {
        cudaFree(ptr);
        return;
    }
    e->ptr = ptr;
    e->bytes = bytes;
    e->device = device;
    size_t b = dpool_bucket(device, bytes);
    pthread_mutex_lock(&g_pool_mu);
    e->next = g_dpool[b];
    g_dpool[b] = e;
    pthread_mutex_unlock(&g_pool_mu);
}

/* ================================================================ arenas */
/* Every arena allocation ever made (arenas are pooled, never freed), so that
 * pointers into library-owned memory are classified without a driver query. */
typedef struct {
    uintptr_t lo, hi;
    int device;
} arena_range;
static arena_range *g_arena_ranges = NULL;
static size_t g_arena_nranges = 0, g_arena_cap = 0;

static void arena_note_range(void *p, size_t bytes, int device) {
    pthread_mutex_lock(&g_pool_mu);
    if (g_arena_nranges == g_arena_cap) {
        size_t nc = g_arena_cap ? 2 * g_arena_cap : 64;
        arena_range *n = (arena_range *)realloc(g_arena_ranges, nc * sizeof(arena_range));
        if (!n) {
            pthread_mutex_unlock(&g_pool_mu);
            return;
        }
        g_arena_ranges = n;
        g_arena_cap = nc;
    }
    g_arena_ranges[g_arena_nranges].lo = (uintptr_t)p;
    g_arena_ranges[g_arena_nranges].hi = (uintptr_t)p + bytes;
    g_arena_ranges[g_arena_nranges].device = device;
    g_arena_nranges++;
    pthread_mutex_unlock(&g_pool_mu);
}

static int arena_lookup(uintptr_t a, uintptr_t *lo, uintptr_t *hi, int *device) {
    int found = 0;
    pthread_mutex_lock(&g_pool_mu);
    for (size_t i = 0; i < g_arena_nranges; i++) {
        if (a >= g_arena_ranges[i].lo && a < g_arena_ranges[i].hi) {
            *lo = g_arena_ranges[i].lo;
            *hi = g_arena_ranges[i].hi;
            *device = g_arena_ranges[i].device;
            found = 1;
            break;
        }
    }
    pthread_mutex_unlock(&g_pool_mu);
    return found;
}
mc_arena *arena_acquire(size_t bytes, int device) {
    if (bytes == 0) bytes = 64;
    mc_arena *a = (mc_arena *)calloc(1, sizeof(mc_arena));
    if (!a) return NULL;
    /* best fit among pooled arenas of the same kind, at most 2x oversized */
    pthread_mutex_lock(&g_pool_mu);
    pool_ent **best = NULL;
    for (pool_ent **pp = &g_hpool; *pp; pp = &(*pp)->next) {
        pool_ent *e = *pp;
        if (e->device == device && e->bytes >= bytes && e->bytes <= 2 * bytes + (1u << 20)) {
            if (!best || e->bytes < (*best)->bytes) best = pp;
        }
    }
    if (best) {
        pool_ent *e = *best;
        *best = e->next;
        pthread_mutex_unlock(&g_pool_mu);
        a->ptr = e->ptr;
        a->bytes = e->bytes;
        free(e);
    } else {
        pthread_mutex_unlock(&g_pool_mu);
        void *p = NULL;
        cudaError_t rc = device < 0 ? cudaHostAlloc(&p, bytes, cudaHostAllocPortable)
                                    : cudaMalloc(&p, bytes);
        if (rc != cudaSuccess) {
            (void)cudaGetLastError();
            free(a);
            return NULL;
        }
        a->ptr = p;
        a->bytes = bytes;
        arena_note_range(p, bytes, device);
    }
    a->device = device;
    a->refs = 1;
    a->objs = NULL;
    return a;
}

void arena_retain(mc_arena *a, int n) {
    pthread_mutex_lock(&g_pool_mu);
    a->refs += n;
    pthread_mutex_unlock(&g_pool_mu);
}

void arena_release(mc_arena *a) { arena_release_n(a, 1); }

void arena_release_n(mc_arena *a, int k) {
    if (!a || k <= 0) return;
    pthread_mutex_lock(&g_pool_mu);
    a->refs -= k;
    int left = a->refs;
    if (left > 0) {
        pthread_mutex_unlock(&g_pool_mu);
        return;
    }
    pool_ent *e = (pool_ent *)malloc(sizeof(pool_ent));
    if (e) {
        e->ptr = a->ptr;
        e->bytes = a->bytes;
        e->device = a->device;
        e->next = g_hpool;
        g_hpool = e;
    }
    pthread_mutex_unlock(&g_pool_mu);
    if (!e) {
        if (a->device < 0) cudaFreeHost(a->ptr);
        else cudaFree(a->ptr);
    }
    free(a->objs);
    free(a);
}

/* ============================================================== registry */
typedef struct reg_ent {
    const void *obj;
    mc_arena *arena;
} reg_ent;
static reg_ent *g_reg = NULL;
static size_t g_reg_cap = 0, g_reg_len = 0, g_reg_tomb = 0;
static pthread_mutex_t g_reg_mu = PTHREAD_MUTEX_INITIALIZER;
#define REG_TOMB ((const void *)1)

static size_t reg_hash(const void *p, size_t cap) {
    uint64_t x = (uint64_t)(uintptr_t)p;
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 33;
    return (size_t)x & (cap - 1);
}

/* Rebuilds the table without tombstones, doubling it when it is more than a
 * quarter full of live entries. */
static int reg_rehash(void) {
    size_t ncap = g_reg_cap ? g_reg_cap : 1024;
    if ((g_reg_len + 1) * 4 >= ncap) ncap *= 2;
    reg_ent *n = (reg_ent *)calloc(ncap, sizeof(reg_ent));
    if (!n) return -1;
    for (size_t i = 0; i < g_reg_cap; i++) {
        if (!g_reg[i].obj || g_reg[i].obj == REG_TOMB) continue;
        size_t j = reg_hash(g_reg[i].obj, ncap);
        while (n[j].obj) j = (j + 1) & (ncap - 1);
        n[j] = g_reg[i];
    }
    free(g_reg);
    g_reg = n;
    g_reg_cap = ncap;
    g_reg_tomb = 0;
    return 0;
}

/* caller holds g_reg_mu */
static int reg_insert(const void *obj, mc_arena *a) {
    if ((g_reg_len + g_reg_tomb + 1) * 2 >= g_reg_cap && reg_rehash() != 0) return -1;
    size_t j = reg_hash(obj, g_reg_cap);
    while (g_reg[j].obj && g_reg[j].obj != REG_TOMB) j = (j + 1) & (g_reg_cap - 1);
    if (g_reg[j].obj == REG_TOMB) g_reg_tomb--;
    g_reg[j].obj = obj;
    g_reg[j].arena = a;
    g_reg_len++;
    return 0;
}

void registry_add(const void *obj, mc_arena *a) {
    pthread_mutex_lock(&g_reg_mu);
    reg_insert(obj, a);
    pthread_mutex_unlock(&g_reg_mu);
}

void registry_add_many(const void **objs, size_t n, mc_arena *a) {
    pthread_mutex_lock(&g_reg_mu);
    for (size_t k = 0; k < n; k++)
        if (reg_insert(objs[k], a) != 0) break;
    pthread_mutex_unlock(&g_reg_mu);
}

mc_arena *registry_take(const void *obj, int *found) {
    *found = 0;
    pthread_mutex_lock(&g_reg_mu);
    if (g_reg_cap == 0) {
        pthread_mutex_unlock(&g_reg_mu);
        return NULL;
    }
    size_t j = reg_hash(obj, g_reg_cap);
    while (g_reg[j].obj) {
        if (g_reg[j].obj == obj) {
            mc_arena *a = g_reg[j].arena;
            g_reg[j].obj = REG_TOMB;
            g_reg[j].arena = NULL;
            g_reg_len--;
            g_reg_tomb++;
            *found = 1;
            pthread_mutex_unlock(&g_reg_mu);
            return a;
        }
        j = (j + 1) & (g_reg_cap - 1);
    }
    pthread_mutex_unlock(&g_reg_mu);
    return NULL;
}

/* Takes the registry entries of objs[0..n) under one lock: arenas[i] is the
 * owning arena, or NULL for an object the registry does not hold. */
void registry_take_many(const void *const *objs, size_t n, mc_arena **arenas) {
    pthread_mutex_lock(&g_reg_mu);
    for (size_t k = 0; k < n; k++) {
        arenas[k] = NULL;
        if (!objs[k] || g_reg_cap == 0) continue;
        size_t j = reg_hash(objs[k], g_reg_cap);
        while (g_reg[j].obj) {
            if (g_reg[j].obj == objs[k]) {
                arenas[k] = g_reg[j].arena;
                g_reg[j].obj = REG_TOMB;
                g_reg[j].arena = NULL;
                g_reg_len--;
                g_reg_tomb++;
                break;
            }
            j = (j + 1) & (g_reg_cap - 1);
        }
    }
    pthread_mutex_unlock(&g_reg_mu);
}

/* =============================================================== scratch */
void *scratch_dev(mc_scratch *s, int slot, size_t bytes) {
    mc_sbuf *b = &s->dev[slot];
    if (b->bytes >= bytes && b->ptr) return b->ptr;
    size_t nb = bytes + bytes / 4 + 4096;
    if (b->ptr) {
        cudaDeviceSynchronize();
        cudaFree(b->ptr);
        b->ptr = NULL;
        b->bytes = 0;
    }
    if (cudaMalloc(&b->ptr, nb) != cudaSuccess) {
        (void)cudaGetLastError();
        b->ptr = NULL;
        return NULL;
    }
    b->bytes = nb;
    return b->ptr;
}

void *scratch_host(mc_scratch *s, int slot, size_t bytes) {
    mc_sbuf *b = &s->host[slot];
    if (b->bytes >= bytes && b->ptr) return b->ptr;
    size_t nb = bytes + bytes / 4 + 4096;
    if (b->ptr) {
        cudaDeviceSynchronize();
        cudaFreeHost(b->ptr);
        b->ptr = NULL;
        b->bytes = 0;
    }
    if (cudaHostAlloc(&b->ptr, nb, cudaHostAllocPortable) != cudaSuccess) {
        (void)cudaGetLastError();
        b->ptr = NULL;
        return NULL;
    }
    b->bytes = nb;
    return b->ptr;
}

void scratch_free(mc_scratch *s) {
    for (int i = 0; i < 16; i++)
        if (s->dev[i].ptr) cudaFree(s->dev[i].ptr);
    for (int i = 0; i < 8; i++)
        if (s->host[i].ptr) cudaFreeHost(s->host[i].ptr);
    memset(s, 0, sizeof(*s));
}

/* =============================================================== tensors */
mc_tensor *tensor_new(DataType dt, size_t ndim, const size_t *shape, int device) {
    mc_tensor *t = (mc_tensor *)calloc(1, sizeof(mc_tensor));
    if (!t) return NULL;
    t->dtype = dt;
    t->ndim = ndim;
    t->n = 1;
    for (size_t i = 0; i < ndim; i++) {
        t->shape[i] = shape[i];
        t->n *= shape[i];
    }
    t->bytes = t->n * mc_dtype_size(dt);
    t->device = device;
    t->dev = dbuf_get(device, t->bytes);
    if (!t->dev) {
        free(t);
        return NULL;
    }
    return t;
}

/* Returns a tensor's buffer to the pool of its device. */
void tensor_drop(void *p) {
    mc_tensor *t = (mc_tensor *)p;
    if (!t) return;
    dbuf_put(t->device, t->dev, t->bytes);
    free(t);
}

/* =============================================================== helpers */
size_t mc_dtype_size(DataType dt) {
    switch (dt) {
        case DTYPE_FLOAT32: return 4;
        case DTYPE_FLOAT64: return 8;
        case DTYPE_INT32: return 4;
        case DTYPE_INT64: return 8;
        case DTYPE_UINT8: return 1;
        default: return 0;
    }
}

const char *mc_dtype_name(DataType dt) {
    switch (dt) {
        case DTYPE_FLOAT32: return "float32";
        case DTYPE_FLOAT64: return "float64";
        case DTYPE_INT32: return "int32";
        case DTYPE_INT64: return "int64";
        case DTYPE_UINT8: return "uint8";
        default: return "unknown";
    }
}

int mc_dtype_parse(const char *s, DataType *out) {
    static const char *names[] = {"float32", "float64", "int32", "int64", "uint8"};
    for (int i = 0; i < 5; i++) {
        if (strcmp(s, names[i]) == 0) {
            *out = (DataType)i;
            return 0;
        }
    }
    return -1;
}

/* reference :1478-1480 */
void mc_history_key(char *out, const char *client, const char *layer) {
    snprintf(out, MAX_KEY_LENGTH, "%s:%s", client, layer);
}

/* reference :1482-1506: "<layer>|<dtype>|conv_(d0, d1, ...)" */
void mc_layer_key(char *out, size_t cap, const char *layer, const size_t *shape, size_t ndim,
                  DataType dt) {
    size_t off = (size_t)snprintf(out, cap, "%s|%s|conv_(", layer ? layer : "<unknown>",
                                  mc_dtype_name(dt));
    for (size_t i = 0; i < ndim && off + 1 < cap; i++) {
        int w = snprintf(out + off, cap - off, "%zu%s", shape[i], (i + 1 < ndim) ? ", " : "");
        if (w < 0) break;
        off += (size_t)w;
    }
    if (off + 1 < cap) snprintf(out + off, cap - off, ")");
    else if (cap > 0) out[cap - 1] = '\0';
}

void mc_memory_key(char *out, size_t cap, const char *client, const char *layer_key) {
    snprintf(out, cap, "%s\x1f%s", client, layer_key);
}

/* reference :399-415 */
int mc_should_lossy(const char *name, size_t n, DataType dt, size_t threshold) {
    return strstr(name, "weight") != NULL && n > threshold &&
           (dt == DTYPE_FLOAT32 || dt == DTYPE_FLOAT64);
}

/* reference :2414-2422 */
int mc_env_flag(const char *name) {
    const char *v = getenv(name);
    if (!v || !*v) return 0;
    return strcmp(v, "0") != 0 && strcmp(v, "false") != 0 && strcmp(v, "FALSE") != 0 &&
           strcmp(v, "off") != 0 && strcmp(v, "OFF") != 0;
}

/* 1 when the variable is set to an off value ("0", "false", "off") */
int mc_env_off(const char *name) {
    const char *v = getenv(name);
    return v && *v && !mc_env_flag(name);
}

void mc_set_error(MomentumCompressor *mc, const char *fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (mc) snprintf(mc->last_error, sizeof(mc->last_error), "%s", buf);
    fprintf(stderr, "[ERROR] %s\n", buf);
}

void mc_log(const MomentumCompressor *mc, int level, const char *fmt, ...) {
    if (mc && level < mc->log_level) return;
    va_list ap;
    va_start(ap, fmt);
    vfprintf(level >= LOG_LEVEL_WARNING ? stderr : stdout, fmt, ap);
    va_end(ap);
}

int mc_is_arena_ptr(const void *p) {
    uintptr_t lo, hi;
    int d;
    return arena_lookup((uintptr_t)p, &lo, &hi, &d);
}

int mc_ptr_is_device(const void *p, int *device) {
    mc_ptrcache pc;
    pc.n = 0;
    return mc_classify(&pc, p, device);
}

typedef int (*fn_getrange)(unsigned long long *, size_t *, unsigned long long);
static fn_getrange p_getrange = NULL;
static int g_getrange_state = 0;

static int driver_range(const void *p, uintptr_t *lo, uintptr_t *hi) {
    if (g_getrange_state == 0) {
        void *fp = NULL;
        enum cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess && fp) {
            p_getrange = (fn_getrange)fp;
            g_getrange_state = 1;
        } else {
            (void)cudaGetLastError();
            g_getrange_state = -1;
        }
    }
    if (g_getrange_state != 1) return 0;
    unsigned long long base = 0;
    size_t size = 0;
    if (p_getrange(&base, &size, (unsigned long long)(uintptr_t)p) != 0 || size == 0) return 0;
    *lo = (uintptr_t)base;
    *hi = (uintptr_t)base + size;
    return 1;
}

/* Classifies a pointer as device memory (1, *device set) or host memory (0).
 * Ranges seen during one call are remembered in `pc`, so a batch whose
 * tensors live in one allocation costs one driver query. */
int mc_classify(mc_ptrcache *pc, const void *p, int *device) {
    int in_arena;
    return mc_classify2(pc, p, device, &in_arena);
}

int mc_classify2(mc_ptrcache *pc, const void *p, int *device, int *in_arena) {
    *in_arena = 0;
    if (!p) return 0;
    uintptr_t a = (uintptr_t)p;
    for (int i = 0; i < pc->n; i++) {
        if (a >= pc->r[i].lo && a < pc->r[i].hi) {
            if (device) *device = pc->r[i].device;
            *in_arena = pc->r[i].arena;
            return pc->r[i].device >= 0;
        }
    }
    uintptr_t lo, hi;
    int d;
    if (arena_lookup(a, &lo, &hi, &d)) {
        if (pc->n < MC_PTRCACHE) {
            pc->r[pc->n].lo = lo;
            pc->r[pc->n].hi = hi;
            pc->r[pc->n].device = d;
            pc->r[pc->n].arena = 1;
            pc->n++;
        }
        if (device) *device = d;
        *in_arena = 1;
        return d >= 0;
    }
    struct cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    int is_dev = at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
    if (at.type != cudaMemoryTypeUnregistered && pc->n < MC_PTRCACHE && driver_range(p, &lo, &hi)) {
        pc->r[pc->n].lo = lo;
        pc->r[pc->n].hi = hi;
        pc->r[pc->n].device = is_dev ? at.device : -1;
        pc->r[pc->n].arena = 0;
        pc->n++;
    }
    if (is_dev && device) *device = at.device;
    return is_dev;
}

/* reference :2844-2867 */
void mc_record_stats(MomentumCompressor *mc, const CompressedLayerData *c) {
    mc->stats.total_compressions++;
    if (!c || strcmp(c->type, "momentum_predicted") != 0) return;
    if (mc->stats.pr_count >= mc->stats.pr_cap) {
        size_t nc = mc->stats.pr_cap ? mc->stats.pr_cap * 2 : 16;
        float *p = (float *)realloc(mc->stats.prediction_ratios, nc * sizeof(float));
        if (!p) return;
        mc->stats.prediction_ratios = p;
        mc->stats.pr_cap = nc;
    }
    mc->stats.prediction_ratios[mc->stats.pr_count++] = c->prediction_ratio;
    if (mc->stats.sm_count >= mc->stats.sm_cap) {
        size_t nc = mc->stats.sm_cap ? mc->stats.sm_cap * 2 : 16;
        float *p = (float *)realloc(mc->stats.sign_mismatch_ratios, nc * sizeof(float));
        if (!p) return;
        mc->stats.sign_mismatch_ratios = p;
        mc->stats.sm_cap = nc;
    }
    mc->stats.sign_mismatch_ratios[mc->stats.sm_count++] = c->sign_mismatch_ratio;
}
