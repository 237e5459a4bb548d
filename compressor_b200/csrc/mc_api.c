/*
 * mc_api.c -- exported C ABI (momentum_compressor.h) and extensions
 * (falcom_b200.h).
 *
 * Each entry point keeps the argument meaning, return values and error
 * behaviour of the reference entry point it replaces
 * (momentum_compressor_openmp_simd_final.c, cited per function).  All numeric
 * work runs on the GPU through mc_batch.c; when no CUDA device is usable the
 * library fails loudly (NULL / error code and an [ERROR] line) instead of
 * computing anything on the host.
 */
#define _GNU_SOURCE
#include <ctype.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "mc_internal.h"

/* ----------------------------------------------------------- device scope */
static int dev_enter(const MomentumCompressor *mc) {
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) {
        (void)cudaGetLastError();
        prev = -1;
    }
    if (mc && prev != mc->device) cudaSetDevice(mc->device);
    return prev;
}
static void dev_leave(const MomentumCompressor *mc, int prev) {
    if (mc && prev >= 0 && prev != mc->device) cudaSetDevice(prev);
}

/* --------------------------------------------------------- breakdown state */
typedef struct {
    double batch_total_time;
    double plan_time;
    double device_time;
    size_t num_layers;
    size_t total_elements;
    int launches;
} mc_breakdown;
static int g_breakdown = 0;
static mc_breakdown g_last_breakdown;

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* reference :160-166 */
MC_EXPORT void momentum_compressor_enable_breakdown(int enable) { g_breakdown = enable ? 1 : 0; }

/* reference :197-199 */
MC_EXPORT const void *momentum_compressor_get_last_breakdown(void) { return &g_last_breakdown; }

/* reference :241-340 */
MC_EXPORT void momentum_compressor_print_breakdown(void) {
    if (!g_breakdown) {
        printf("[INFO] Breakdown is disabled. Call momentum_compressor_enable_breakdown(1) first.\n");
        return;
    }
    if (g_last_breakdown.num_layers == 0) {
        printf("[INFO] No breakdown data available.\n");
        return;
    }
    const mc_breakdown *b = &g_last_breakdown;
    printf("\nBatch Summary (GPU codec):\n");
    printf("  Total layers:      %zu\n", b->num_layers);
    printf("  Total elements:    %zu (%.2f MB)\n", b->total_elements, b->total_elements * 4.0 / 1048576.0);
    printf("  Batch total time:  %.3f ms\n", b->batch_total_time * 1e3);
    printf("  Kernel launches:   %d\n", b->launches);
    if (b->batch_total_time > 0)
        printf("  Throughput:        %.2f MB/s\n", (b->total_elements * 4.0 / 1048576.0) / b->batch_total_time);
}

/* ------------------------------------------------------------------ config */
/* reference :1699-1716 */
MC_EXPORT CompressorConfig momentum_compressor_default_config(void) {
    CompressorConfig c;
    memset(&c, 0, sizeof(c));
    c.momentum_lr = DEFAULT_MOMENTUM_LR;
    c.consistency_threshold = DEFAULT_CONSISTENCY_THRESHOLD;
    snprintf(c.lossless_compressor, sizeof(c.lossless_compressor), "zstd");
    snprintf(c.error_bounding_mode, sizeof(c.error_bounding_mode), "REL");
    c.error_bound = DEFAULT_ERROR_BOUND;
    c.param_count_threshold = DEFAULT_PARAM_COUNT_THRESHOLD;
    c.max_history_length = DEFAULT_MAX_HISTORY_LENGTH;
    return c;
}

static int log_level_parse(const char *s, int fallback) {
    if (!s || !*s) return fallback;
    if (!strcmp(s, "DEBUG") || !strcmp(s, "debug")) return LOG_LEVEL_DEBUG;
    if (!strcmp(s, "INFO") || !strcmp(s, "info")) return LOG_LEVEL_INFO;
    if (!strcmp(s, "WARNING") || !strcmp(s, "warning") || !strcmp(s, "WARN") || !strcmp(s, "warn"))
        return LOG_LEVEL_WARNING;
    if (!strcmp(s, "ERROR") || !strcmp(s, "error")) return LOG_LEVEL_ERROR;
    return fallback;
}

static int codec_parse(const char *s) {
    if (!s) return -1;
    if (!strcmp(s, "q8")) return MC_CODEC_Q8;
    if (!strcmp(s, "int4")) return MC_CODEC_INT4;
    if (!strcmp(s, "raw") || !strcmp(s, "sz3_memcpy")) return MC_CODEC_RAW;
    if (!strcmp(s, "q8_raw")) return MC_CODEC_Q8_RAW;
    if (!strcmp(s, "int4_raw")) return MC_CODEC_INT4_RAW;
    return -1;
}

/* reference :1722-1767 */
MC_EXPORT MomentumCompressor *momentum_compressor_create(const CompressorConfig *config) {
    if (!config) {
        fprintf(stderr, "[ERROR] momentum_compressor_create: config is NULL\n");
        return NULL;
    }
    int dev = -1, ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0 || cudaGetDevice(&dev) != cudaSuccess) {
        (void)cudaGetLastError();
        fprintf(stderr, "[ERROR] momentum_compressor_create: no CUDA device is available; "
                        "this codec runs on the GPU only\n");
        return NULL;
    }
    MomentumCompressor *mc = (MomentumCompressor *)calloc(1, sizeof(MomentumCompressor));
    if (!mc) return NULL;
    memcpy(&mc->config, config, sizeof(CompressorConfig));
    mc->device = dev;
    mc->log_level = log_level_parse(getenv("FALCOM_LOG_LEVEL"), LOG_LEVEL_WARNING);
    mc->layers = map_new();
    mc->memory = map_new();
    mc->mem_clients = map_new();
    int codec = codec_parse(getenv("FALCOM_RESIDUAL_CODEC"));
    mc->residual_codec = codec < 0 ? MC_CODEC_Q8 : codec;
    const char *fm = getenv("FALCOM_FRAME_MODE");
    mc->frame_mode = (fm && !strcmp(fm, "libzstd")) ? MC_FRAME_LIBZSTD : MC_FRAME_GPU;
    if (cudaStreamCreateWithFlags(&mc->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        !mc->layers || !mc->memory || !mc->mem_clients) {
        (void)cudaGetLastError();
        fprintf(stderr, "[ERROR] momentum_compressor_create: initialisation failed\n");
        map_free(mc->layers, NULL);
        map_free(mc->memory, NULL);
        map_free(mc->mem_clients, NULL);
        free(mc);
        return NULL;
    }
    mc->stream = mc->own_stream;
    mc->scratch.device = dev;
    if (mc->log_level <= LOG_LEVEL_INFO) {
        struct cudaDeviceProp prop;
        cudaGetDeviceProperties(&prop, dev);
        printf("PASS MomentumCompressor (B200 GPU codec) created on device %d (%s)\n", dev, prop.name);
        printf("  - momentum_lr: %.3f\n", config->momentum_lr);
        printf("  - consistency_threshold: %.3f\n", config->consistency_threshold);
        printf("  - param_count_threshold: %zu\n", config->param_count_threshold);
        printf("  - lossless_compressor: %s\n", config->lossless_compressor);
    }
    return mc;
}

/* reference :1769-1811 */
MC_EXPORT void momentum_compressor_destroy(MomentumCompressor *mc) {
    if (!mc) return;
    int prev = dev_enter(mc);
    cudaStreamSynchronize(mc->stream);
    map_free(mc->layers, layer_rec_drop);
    map_free(mc->memory, mem_rec_drop);
    map_free(mc->mem_clients, NULL);
    for (int i = 0; i < MC_KC_SLOTS; i++) {
        keycache_free(&mc->enc_kc[i]);
        keycache_free(&mc->dec_kc[i]);
    }
    listcache_free(mc, mc->enc_lists);
    listcache_free(mc, mc->dec_lists);
    scratch_free(&mc->scratch);
    if (mc->own_stream) cudaStreamDestroy(mc->own_stream);
    if (mc->copy_in) cudaStreamDestroy(mc->copy_in);
    if (mc->copy_out) cudaStreamDestroy(mc->copy_out);
    for (int i = 0; i < MC_MAX_CHUNKS; i++) {
        if (mc->ev_in[i]) cudaEventDestroy(mc->ev_in[i]);
        if (mc->ev_done[i]) cudaEventDestroy(mc->ev_done[i]);
    }
    if (mc->tab_ev[0]) cudaEventDestroy(mc->tab_ev[0]);
    for (int i = 0; i < 2 * MC_KTRACE_MAX; i++)
        if (mc->ktrace.ev[i]) cudaEventDestroy((cudaEvent_t)mc->ktrace.ev[i]);
    free(mc->stats.prediction_ratios);
    free(mc->stats.sign_mismatch_ratios);
    free(mc->agg_off);
    int lvl = mc->log_level;
    dev_leave(mc, prev);
    free(mc);
    if (lvl <= LOG_LEVEL_INFO) printf("PASS MomentumCompressor destroyed\n");
}

/* reference :1813-1817 */
MC_EXPORT void momentum_compressor_set_client(MomentumCompressor *mc, const char *client_id) {
    if (!mc || !client_id) return;
    strncpy(mc->current_client_id, client_id, 255);
    mc->current_client_id[255] = '\0';
}

/* ------------------------------------------------------------ compression */
static int payload_loc_for(const MomentumCompressor *mc, const BatchItem *items, size_t n) {
    if (mc->payload_loc != FALCOM_LOC_AUTO) return mc->payload_loc;
    for (size_t i = 0; i < n; i++) {
        if (items[i].gradient && items[i].gradient->data) {
            int d = -1;
            return mc_ptr_is_device(items[i].gradient->data, &d) ? FALCOM_LOC_DEVICE : FALCOM_LOC_HOST;
        }
    }
    return FALCOM_LOC_HOST;
}

static void note_breakdown(const BatchItem *items, size_t n, double t0, int launches) {
    if (!g_breakdown) return;
    g_last_breakdown.batch_total_time = now_s() - t0;
    g_last_breakdown.num_layers = n;
    g_last_breakdown.total_elements = 0;
    for (size_t i = 0; i < n; i++)
        if (items[i].gradient) g_last_breakdown.total_elements += items[i].gradient->total_size;
    g_last_breakdown.launches = launches;
}

/* reference :2954-3149 (per-layer API; a one-item batch has the same
 * semantics as the grouped path) */
MC_EXPORT CompressedLayerData *momentum_compressor_compress_layer(MomentumCompressor *mc,
                                                                  const char *layer_name,
                                                                  const NDArray *gradient) {
    if (!mc) {
        fprintf(stderr, "[ERROR] compress_layer: compressor is NULL\n");
        return NULL;
    }
    if (!layer_name || !*layer_name) {
        fprintf(stderr, "[ERROR] compress_layer: invalid layer_name\n");
        return NULL;
    }
    if (!gradient) {
        fprintf(stderr, "[ERROR] compress_layer: gradient is NULL\n");
        return NULL;
    }
    if (!mc->current_client_id[0]) {
        fprintf(stderr, "[ERROR] compress_layer: client_id not set (call set_client first)\n");
        return NULL;
    }
    if (strlen(layer_name) >= MAX_LAYER_NAME_LENGTH) {
        fprintf(stderr, "[ERROR] compress_layer: layer_name too long (%zu >= %d)\n", strlen(layer_name),
                MAX_LAYER_NAME_LENGTH);
        return NULL;
    }
    BatchItem it = {layer_name, gradient, NULL, ERROR_NONE};
    int prev = dev_enter(mc);
    char client[256];
    snprintf(client, sizeof(client), "%s", mc->current_client_id);
    int rc = mc_compress_grouped(mc, &it, 1, client, payload_loc_for(mc, &it, 1), 0);
    dev_leave(mc, prev);
    return rc == ERROR_NONE ? it.compressed : NULL;
}

static int validate_batch(const MomentumCompressor *mc, const void *items, size_t n, const char *client,
                          const char *what) {
    if (!mc) {
        fprintf(stderr, "[ERROR] Batch %s: compressor is NULL\n", what);
        return ERROR_INVALID_PARAM;
    }
    if (!items || n == 0) {
        fprintf(stderr, "[ERROR] Batch %s: invalid items (ptr=%p, count=%zu)\n", what, items, n);
        return ERROR_INVALID_PARAM;
    }
    if (!client || !*client) {
        fprintf(stderr, "[ERROR] Batch %s: invalid client_id\n", what);
        return ERROR_INVALID_PARAM;
    }
    if (n > MAX_BATCH_SIZE) {
        fprintf(stderr, "[ERROR] Batch %s: num_items (%zu) exceeds MAX_BATCH_SIZE (%d)\n", what, n,
                MAX_BATCH_SIZE);
        return ERROR_INVALID_PARAM;
    }
    return ERROR_NONE;
}

/* reference :4322-4493 (serial batch: the per-layer API in order) */
static int compress_batch_serial(MomentumCompressor *mc, BatchItem *items, size_t n, const char *client) {
    size_t ok = 0;
    for (size_t i = 0; i < n; i++) {
        items[i].compressed = NULL;
        items[i].error = ERROR_NONE;
        if (!items[i].gradient || !items[i].layer_name) {
            fprintf(stderr, "[ERROR] Batch compress: item[%zu] has NULL gradient or layer_name\n", i);
            items[i].error = ERROR_INVALID_PARAM;
            continue;
        }
        BatchItem one = {items[i].layer_name, items[i].gradient, NULL, ERROR_NONE};
        int rc = mc_compress_grouped(mc, &one, 1, client, payload_loc_for(mc, &one, 1), 0);
        if (rc != ERROR_NONE) {
            fprintf(stderr, "[ERROR] Batch compress: safe path failed for item[%zu] layer='%s'\n", i,
                    items[i].layer_name);
            items[i].error = ERROR_COMPRESSION;
            continue;
        }
        items[i].compressed = one.compressed;
        ok++;
    }
    if (ok == 0) return ERROR_COMPRESSION;
    if (ok < n) return -((int)n - (int)ok);
    return 0;
}

/* reference :4495-4705 */
MC_EXPORT int momentum_compressor_compress_batch(MomentumCompressor *mc, BatchItem *items,
                                                 size_t num_items, const char *client_id) {
    int v = validate_batch(mc, items, num_items, client_id, "compress");
    if (v != ERROR_NONE) return v;
    double t0 = g_breakdown ? now_s() : 0.0;
    mc_log(mc, LOG_LEVEL_INFO, "[INFO] Batch compress: processing %zu layers for client '%s'\n",
           num_items, client_id);
    momentum_compressor_set_client(mc, client_id);
    int prev = dev_enter(mc);
    char client[256];
    snprintf(client, sizeof(client), "%s", client_id);
    int rc;
    const char *par = getenv("FALCOM_BATCH_PARALLEL");
    if (mc_env_flag("FALCOM_BATCH_SERIAL") || (par && !mc_env_flag("FALCOM_BATCH_PARALLEL")) ||
        num_items == 1) {
        rc = compress_batch_serial(mc, items, num_items, client);
    } else {
        rc = mc_compress_grouped(mc, items, num_items, client, payload_loc_for(mc, items, num_items), 1);
    }
    dev_leave(mc, prev);
    note_breakdown(items, num_items, t0, mc->last_launches);
    if (rc == ERROR_NONE && mc->log_level <= LOG_LEVEL_INFO) {
        size_t comp = 0, orig = 0;
        for (size_t i = 0; i < num_items; i++) {
            const CompressedLayerData *c = items[i].compressed;
            if (!c) continue;
            comp += c->data_size + c->bitmap_size + c->dominant_signs_size;
            orig += items[i].gradient->total_size * (items[i].gradient->dtype == DTYPE_FLOAT32 ? 4 : 8);
        }
        printf("[INFO] Batch compress: %zu/%zu layers succeeded, compression ratio: %.2f%% (%.2f KB -> %.2f KB)\n",
               num_items, num_items, orig ? 100.0f * (float)comp / (float)orig : 0.0f, orig / 1024.0f,
               comp / 1024.0f);
    }
    return rc;
}

/* ---------------------------------------------------------- decompression */
static int out_loc_for(const MomentumCompressor *mc, const BatchItem *items, size_t n) {
    if (mc->output_loc != FALCOM_LOC_AUTO) return mc->output_loc;
    for (size_t i = 0; i < n; i++) {
        if (items[i].compressed && items[i].compressed->data) {
            int d = -1;
            return mc_ptr_is_device(items[i].compressed->data, &d) ? FALCOM_LOC_DEVICE : FALCOM_LOC_HOST;
        }
    }
    return FALCOM_LOC_HOST;
}

/* reference :3476-3598 */
MC_EXPORT NDArray *momentum_compressor_decompress_layer(MomentumCompressor *mc,
                                                        const CompressedLayerData *compressed,
                                                        const char *client_id, const char *layer_name) {
    if (!mc) {
        fprintf(stderr, "[ERROR] decompress_layer: compressor is NULL\n");
        return NULL;
    }
    if (!compressed) {
        fprintf(stderr, "[ERROR] decompress_layer: compressed data is NULL\n");
        return NULL;
    }
    if (!client_id || !*client_id) {
        fprintf(stderr, "[ERROR] decompress_layer: invalid client_id\n");
        return NULL;
    }
    if (!layer_name || !*layer_name) {
        fprintf(stderr, "[ERROR] decompress_layer: invalid layer_name\n");
        return NULL;
    }
    BatchItem it = {layer_name, NULL, (CompressedLayerData *)compressed, ERROR_NONE};
    NDArray *out = NULL;
    int prev = dev_enter(mc);
    mc_decompress_items(mc, &it, 1, client_id, &out, out_loc_for(mc, &it, 1));
    dev_leave(mc, prev);
    return out;
}

/* reference :4707-4838 */
MC_EXPORT int momentum_compressor_decompress_batch(MomentumCompressor *mc, const BatchItem *items,
                                                   size_t num_items, const char *client_id,
                                                   NDArray **out_gradients) {
    int v = validate_batch(mc, items, num_items, client_id, "decompress");
    if (v != ERROR_NONE) return v;
    if (!out_gradients) {
        fprintf(stderr, "[ERROR] Batch decompress: out_gradients is NULL\n");
        return ERROR_INVALID_PARAM;
    }
    double t0 = g_breakdown ? now_s() : 0.0;
    mc_log(mc, LOG_LEVEL_INFO, "[INFO] Batch decompress: processing %zu layers for client '%s'\n",
           num_items, client_id);
    momentum_compressor_set_client(mc, client_id);
    int prev = dev_enter(mc);
    char client[256];
    snprintf(client, sizeof(client), "%s", client_id);
    int rc = mc_decompress_items(mc, items, num_items, client, out_gradients,
                                 out_loc_for(mc, items, num_items));
    dev_leave(mc, prev);
    (void)t0;
    if (mc->log_level <= LOG_LEVEL_INFO) {
        size_t ok = 0;
        for (size_t i = 0; i < num_items; i++) ok += out_gradients[i] != NULL;
        printf("[INFO] Batch decompress: %zu/%zu layers succeeded\n", ok, num_items);
    }
    return rc;
}

/* ---------------------------------------------------------------- resets */

/* reference :3941-4000: histories and step counts of "client:*", and the
 * client's prediction-memory table */
MC_EXPORT void momentum_compressor_reset_client(MomentumCompressor *mc, const char *client_id) {
    if (!mc || !client_id) return;
    if (mc->log_level <= LOG_LEVEL_INFO) printf("[INFO] Resetting state for client: %s\n", client_id);
    int prev = dev_enter(mc);
    cudaStreamSynchronize(mc->stream);
    size_t len = strlen(client_id);
    int count = 0;
    for (size_t i = 0; i < mc->layers->cap; i++) {
        if (!MAP_LIVE(mc->layers, i)) continue;
        const char *k = mc->layers->keys[i];
        if (strncmp(k, client_id, len) == 0 && k[len] == ':') {
            mc_layer_rec *r = (mc_layer_rec *)mc->layers->vals[i];
            count += (r->hist != NULL) + (r->step > 0);
            char *key = strdup(k);
            layer_rec_drop(map_del(mc->layers, key));
            free(key);
        }
    }
    for (size_t i = 0; i < mc->memory->cap; i++) {
        if (!MAP_LIVE(mc->memory, i)) continue;
        const char *k = mc->memory->keys[i];
        if (strncmp(k, client_id, len) == 0 && k[len] == '\x1f') {
            char *key = strdup(k);
            mem_rec_drop(map_del(mc->memory, key));
            free(key);
        }
    }
    if (map_del(mc->mem_clients, client_id)) count++;
    mc->state_gen++;
    dev_leave(mc, prev);
    if (mc->log_level <= LOG_LEVEL_INFO) printf("PASS Deleted %d entries for client %s\n", count, client_id);
}

/* reference :4002-4052 */
MC_EXPORT void momentum_compressor_reset_all(MomentumCompressor *mc) {
    if (!mc) return;
    int prev = dev_enter(mc);
    cudaStreamSynchronize(mc->stream);
    map_free(mc->layers, layer_rec_drop);
    map_free(mc->memory, mem_rec_drop);
    map_free(mc->mem_clients, NULL);
    mc->layers = map_new();
    mc->memory = map_new();
    mc->mem_clients = map_new();
    mc->state_gen++;
    dev_leave(mc, prev);
    if (mc->log_level <= LOG_LEVEL_INFO) printf("PASS All states reset\n");
}

/* ----------------------------------------------------------------- stats */
/* reference :4058-4091 */
MC_EXPORT void momentum_compressor_print_stats(const MomentumCompressor *mc) {
    if (!mc) return;
    printf("\n+--------------------------------------------------------------+\n");
    printf("| Compression Statistics                                       |\n");
    printf("+--------------------------------------------------------------+\n");
    printf("| Total compressions: %-41zu|\n", mc->stats.total_compressions);
    size_t nh = 0, ns = 0;
    for (size_t i = 0; i < mc->layers->cap; i++) {
        if (!MAP_LIVE(mc->layers, i)) continue;
        const mc_layer_rec *r = (const mc_layer_rec *)mc->layers->vals[i];
        nh += r->hist != NULL;
        ns += r->step > 0;
    }
    printf("| History entries: %-44zu|\n", nh);
    printf("| Prediction memories: %-40zu|\n", mc->mem_clients->len);
    printf("| Step counters: %-46zu|\n", ns);
    if (mc->stats.pr_count > 0) {
        float s = 0.0f;
        for (size_t i = 0; i < mc->stats.pr_count; i++) s += mc->stats.prediction_ratios[i];
        printf("| Avg prediction ratio: %.2f%% (from %zu predictions)\n", s / mc->stats.pr_count * 100,
               mc->stats.pr_count);
    }
    if (mc->stats.sm_count > 0) {
        float s = 0.0f;
        for (size_t i = 0; i < mc->stats.sm_count; i++) s += mc->stats.sign_mismatch_ratios[i];
        printf("| Avg sign mismatch: %.2f%%\n", s / mc->stats.sm_count * 100);
    }
    printf("+--------------------------------------------------------------+\n\n");
}

/* reference :4097-4139 */
MC_EXPORT CompressionStats *momentum_compressor_get_stats(const MomentumCompressor *mc) {
    if (!mc) return NULL;
    CompressionStats *s = (CompressionStats *)malloc(sizeof(CompressionStats));
    if (!s) return NULL;
    s->total_compressions = mc->stats.total_compressions;
    s->num_predictions = mc->stats.pr_count;
    if (mc->stats.pr_count > 0) {
        float sum = 0.0f, sq = 0.0f;
        for (size_t i = 0; i < mc->stats.pr_count; i++) {
            float v = mc->stats.prediction_ratios[i];
            sum += v;
            sq += v * v;
        }
        s->avg_prediction_ratio = sum / mc->stats.pr_count;
        float var = sq / mc->stats.pr_count - s->avg_prediction_ratio * s->avg_prediction_ratio;
        s->std_prediction_ratio = sqrtf(var > 0 ? var : 0);
    } else {
        s->avg_prediction_ratio = 0.0f;
        s->std_prediction_ratio = 0.0f;
    }
    if (mc->stats.sm_count > 0) {
        float sum = 0.0f;
        for (size_t i = 0; i < mc->stats.sm_count; i++) sum += mc->stats.sign_mismatch_ratios[i];
        s->avg_sign_mismatch_ratio = sum / mc->stats.sm_count;
    } else {
        s->avg_sign_mismatch_ratio = 0.0f;
    }
    return s;
}

/* reference :4141-4236 */
MC_EXPORT DetailedStats *momentum_compressor_get_detailed_stats(const MomentumCompressor *mc) {
    if (!mc) return NULL;
    DetailedStats *d = (DetailedStats *)calloc(1, sizeof(DetailedStats));
    if (!d) return NULL;
    CompressionStats *cs = momentum_compressor_get_stats(mc);
    if (!cs) {
        free(d);
        return NULL;
    }
    d->compression = *cs;
    free(cs);
    /* unique client ids from the step counters ("client:layer") */
    char(*ids)[256] = (char(*)[256])calloc(256, 256);
    size_t nu = 0;
    for (size_t i = 0; ids && i < mc->layers->cap; i++) {
        if (!MAP_LIVE(mc->layers, i)) continue;
        if (((const mc_layer_rec *)mc->layers->vals[i])->step <= 0) continue;
        const char *k = mc->layers->keys[i];
        const char *colon = strchr(k, ':');
        if (!colon) continue;
        size_t len = (size_t)(colon - k);
        if (len == 0 || len >= 256) continue;
        int found = 0;
        for (size_t j = 0; j < nu && !found; j++) found = strncmp(ids[j], k, len) == 0 && ids[j][len] == 0;
        if (!found && nu < 256) {
            memcpy(ids[nu], k, len);
            ids[nu][len] = 0;
            nu++;
        }
    }
    d->num_clients = nu;
    if (nu) {
        d->clients = (ClientStats *)calloc(nu, sizeof(ClientStats));
        if (!d->clients) {
            free(ids);
            free(d);
            return NULL;
        }
    }
    for (size_t c = 0; c < nu; c++) {
        ClientStats *s = &d->clients[c];
        size_t len = strlen(ids[c]);
        memcpy(s->client_id, ids[c], len + 1);
        for (size_t i = 0; i < mc->layers->cap; i++) {
            if (!MAP_LIVE(mc->layers, i)) continue;
            const char *k = mc->layers->keys[i];
            if (strncmp(k, ids[c], len) != 0 || k[len] != ':') continue;
            const mc_layer_rec *r = (const mc_layer_rec *)mc->layers->vals[i];
            if (r->step > s->step_count) s->step_count = r->step;
            s->history_length += r->hist != NULL;
        }
        for (size_t i = 0; i < mc->memory->cap; i++) {
            if (!MAP_LIVE(mc->memory, i)) continue;
            const char *k = mc->memory->keys[i];
            if (strncmp(k, ids[c], len) == 0 && k[len] == '\x1f' &&
                ((const mc_mem_rec *)mc->memory->vals[i])->t)
                s->num_memory_layers++;
        }
    }
    free(ids);
    return d;
}

MC_EXPORT void compression_stats_free(CompressionStats *s) { free(s); }

MC_EXPORT void detailed_stats_free(DetailedStats *s) {
    if (!s) return;
    free(s->clients);
    free(s);
}

/* reference :4250-4261 */
MC_EXPORT void momentum_compressor_set_log_level(MomentumCompressor *mc, const char *level) {
    if (!mc || !level) return;
    int p = log_level_parse(level, -1);
    if (p >= 0) {
        mc->log_level = p;
    } else {
        fprintf(stderr, "Unknown log level: %s (using WARNING)\n", level);
        mc->log_level = LOG_LEVEL_WARNING;
    }
}

/* reference :4263-4291 */
MC_EXPORT void momentum_compressor_set_client_context(MomentumCompressor *mc, const char *client_id) {
    if (!mc || !client_id) return;
    if (strncmp(client_id, "Client", 6) == 0 && isdigit((unsigned char)client_id[6])) {
        snprintf(mc->current_client_id, sizeof(mc->current_client_id), "%s", client_id);
    } else {
        const char *p = client_id;
        while (*p && !isdigit((unsigned char)*p)) p++;
        if (*p) snprintf(mc->current_client_id, sizeof(mc->current_client_id), "Client%d", atoi(p));
        else snprintf(mc->current_client_id, sizeof(mc->current_client_id), "%s", client_id);
    }
    if (mc->log_level <= LOG_LEVEL_INFO) printf("[INFO] Client context set to: %s\n", mc->current_client_id);
}

MC_EXPORT int momentum_compressor_get_log_level(const MomentumCompressor *mc) { return mc ? mc->log_level : -1; }

MC_EXPORT const char *momentum_compressor_get_current_client_id(const MomentumCompressor *mc) {
    return mc ? mc->current_client_id : NULL;
}

/* ----------------------------------------------------------------- arrays */
/* reference :517-575 */
MC_EXPORT NDArray *ndarray_create(const size_t *shape, size_t ndim, DataType dtype) {
    if (!shape) {
        fprintf(stderr, "[ERROR] ndarray_create: shape is NULL\n");
        return NULL;
    }
    if (ndim < MIN_NDIM || ndim > MAX_NDIM) {
        fprintf(stderr, "[ERROR] ndarray_create: invalid ndim=%zu (valid range: %d-%d)\n", ndim, MIN_NDIM,
                MAX_NDIM);
        return NULL;
    }
    for (size_t i = 0; i < ndim; i++) {
        if (shape[i] == 0) {
            fprintf(stderr, "[ERROR] ndarray_create: shape[%zu]=0 is invalid\n", i);
            return NULL;
        }
    }
    if (dtype == DTYPE_UNKNOWN || mc_dtype_size(dtype) == 0) {
        fprintf(stderr, "[ERROR] ndarray_create: unknown dtype\n");
        return NULL;
    }
    NDArray *a = (NDArray *)malloc(sizeof(NDArray));
    if (!a) return NULL;
    a->ndim = ndim;
    a->dtype = dtype;
    a->shape = (size_t *)malloc(ndim * sizeof(size_t));
    if (!a->shape) {
        free(a);
        return NULL;
    }
    memcpy(a->shape, shape, ndim * sizeof(size_t));
    a->total_size = 1;
    for (size_t i = 0; i < ndim; i++) a->total_size *= shape[i];
    a->data = calloc(a->total_size, mc_dtype_size(dtype));
    if (!a->data) {
        free(a->shape);
        free(a);
        return NULL;
    }
    return a;
}

/* reference :577-582; library-owned arrays return their arena */
MC_EXPORT void ndarray_destroy(NDArray *a) {
    if (!a) return;
    int found = 0;
    mc_arena *ar = registry_take(a, &found);
    if (found) {   /* the array, its shape and its data belong to the arena */
        arena_release(ar);
        return;
    }
    free(a->data);
    free(a->shape);
    free(a);
}

/* reference :584-592; a device-resident array is copied on its device */
MC_EXPORT NDArray *ndarray_copy(const NDArray *src) {
    if (!src) return NULL;
    int d = -1;
    if (src->data && mc_ptr_is_device(src->data, &d)) {
        size_t bytes = src->total_size * mc_dtype_size(src->dtype);
        mc_arena *a = arena_acquire(bytes, d);
        NDArray *o = (NDArray *)calloc(1, sizeof(NDArray));
        size_t *shp = (size_t *)malloc(src->ndim * sizeof(size_t));
        if (!a || !o || !shp || cudaMemcpy(a->ptr, src->data, bytes, cudaMemcpyDeviceToDevice) != cudaSuccess) {
            (void)cudaGetLastError();
            if (a) arena_release(a);
            free(o);
            free(shp);
            return NULL;
        }
        memcpy(shp, src->shape, src->ndim * sizeof(size_t));
        *o = *src;
        o->shape = shp;
        o->data = a->ptr;
        registry_add(o, a);
        return o;
    }
    NDArray *o = ndarray_create(src->shape, src->ndim, src->dtype);
    if (!o) return NULL;
    memcpy(o->data, src->data, src->total_size * mc_dtype_size(src->dtype));
    return o;
}

/* reference :594-600; library-owned results return their arena */
MC_EXPORT void compressed_layer_data_free(CompressedLayerData *c) {
    if (!c) return;
    int found = 0;
    mc_arena *a = registry_take(c, &found);
    if (found) {   /* the struct and its payloads belong to the arena */
        arena_release(a);
        return;
    }
    free(c->data);
    free(c->bitmap);
    free(c->dominant_signs);
    free(c);
}

/* -------------------------------------------------------------- MOMC model */
static void put32(uint8_t **p, uint32_t v) { memcpy(*p, &v, 4); *p += 4; }
static void put64(uint8_t **p, uint64_t v) { memcpy(*p, &v, 8); *p += 8; }
static void putb(uint8_t **p, const void *s, size_t n) { if (n) memcpy(*p, s, n); *p += n; }

/* reference :3600-3754 */
MC_EXPORT uint8_t *momentum_compressor_compress_model(MomentumCompressor *mc, const NDArray **gradients,
                                                      const char **layer_names, size_t num_layers,
                                                      const char *client_id, size_t *out_size) {
    if (out_size) *out_size = 0;
    if (!mc || !gradients || !layer_names || !out_size) return NULL;
    if (mc->log_level <= LOG_LEVEL_INFO)
        printf("[INFO] Compressing model with %zu layers for client %s\n", num_layers, client_id ? client_id : "");
    if (client_id && *client_id) momentum_compressor_set_client(mc, client_id);
    CompressedLayerData **L = (CompressedLayerData **)calloc(num_layers ? num_layers : 1, sizeof(*L));
    if (!L) return NULL;
    int save_loc = mc->payload_loc;
    mc->payload_loc = FALCOM_LOC_HOST;
    for (size_t i = 0; i < num_layers; i++) {
        L[i] = momentum_compressor_compress_layer(mc, layer_names[i], gradients[i]);
        if (!L[i]) {
            fprintf(stderr, "[ERROR] Failed to compress layer %zu: %s\n", i, layer_names[i]);
            for (size_t j = 0; j < i; j++) compressed_layer_data_free(L[j]);
            free(L);
            mc->payload_loc = save_loc;
            return NULL;
        }
    }
    mc->payload_loc = save_loc;
    char meta[1024];
    snprintf(meta, sizeof(meta),
             "{\"compressor_type\":\"MomentumPredictorCompressor\",\"client_id\":\"%s\",\"layer_count\":%zu,"
             "\"momentum_lr\":%.6f,\"param_cutoff\":%zu}",
             client_id ? client_id : "", num_layers, mc->config.momentum_lr, mc->config.param_count_threshold);
    size_t ml = strlen(meta);
    size_t total = 12 + ml;
    for (size_t i = 0; i < num_layers; i++) {
        const CompressedLayerData *c = L[i];
        total += 4 + strlen(layer_names[i]) + 4 + strlen(c->type) + 4 + strlen(c->codec) + 4 +
                 strlen(c->original_dtype) + 4 + c->ndim * sizeof(size_t) + 8 + c->data_size + 8 +
                 c->bitmap_size + 8 + c->dominant_signs_size + 16 + 8;
    }
    uint8_t *buf = (uint8_t *)malloc(total);
    if (!buf) {
        for (size_t i = 0; i < num_layers; i++) compressed_layer_data_free(L[i]);
        free(L);
        return NULL;
    }
    uint8_t *p = buf;
    put32(&p, 0x4D4F4D43u);
    put32(&p, (uint32_t)num_layers);
    put32(&p, (uint32_t)ml);
    putb(&p, meta, ml);
    for (size_t i = 0; i < num_layers; i++) {
        const CompressedLayerData *c = L[i];
        size_t l;
        l = strlen(layer_names[i]); put32(&p, (uint32_t)l); putb(&p, layer_names[i], l);
        l = strlen(c->type); put32(&p, (uint32_t)l); putb(&p, c->type, l);
        l = strlen(c->codec); put32(&p, (uint32_t)l); putb(&p, c->codec, l);
        l = strlen(c->original_dtype); put32(&p, (uint32_t)l); putb(&p, c->original_dtype, l);
        put32(&p, (uint32_t)c->ndim);
        putb(&p, c->shape, c->ndim * sizeof(size_t));
        put64(&p, c->data_size); putb(&p, c->data, c->data_size);
        put64(&p, c->bitmap_size); putb(&p, c->bitmap, c->bitmap_size);
        put64(&p, c->dominant_signs_size); putb(&p, c->dominant_signs, c->dominant_signs_size);
        putb(&p, &c->current_mean, 4);
        putb(&p, &c->current_std, 4);
        putb(&p, &c->prev_mean, 4);
        putb(&p, &c->prev_std, 4);
        put64(&p, (uint64_t)c->num_predicted_kernels);
    }
    *out_size = (size_t)(p - buf);
    for (size_t i = 0; i < num_layers; i++) compressed_layer_data_free(L[i]);
    free(L);
    return buf;
}

static int get_bytes(const uint8_t **p, const uint8_t *end, void *dst, size_t n) {
    if ((size_t)(end - *p) < n) return -1;
    memcpy(dst, *p, n);
    *p += n;
    return 0;
}

/* reference :3756-3939 (with bounds checks on every field) */
MC_EXPORT NDArray **momentum_compressor_decompress_model(MomentumCompressor *mc, const uint8_t *data,
                                                         size_t size, char ***layer_names_out,
                                                         size_t *num_layers_out) {
    if (!mc || !data || size < 12 || !layer_names_out || !num_layers_out) {
        fprintf(stderr, "[ERROR] Invalid input to decompress_model\n");
        return NULL;
    }
    const uint8_t *p = data, *end = data + size;
    uint32_t magic, nl, ml;
    get_bytes(&p, end, &magic, 4);
    if (magic != 0x4D4F4D43u) {
        fprintf(stderr, "[ERROR] Invalid magic number: 0x%X\n", magic);
        return NULL;
    }
    get_bytes(&p, end, &nl, 4);
    get_bytes(&p, end, &ml, 4);
    if ((size_t)(end - p) < ml) {
        fprintf(stderr, "[ERROR] Truncated model container\n");
        return NULL;
    }
    char *meta = (char *)malloc((size_t)ml + 1);
    if (!meta) return NULL;
    memcpy(meta, p, ml);
    meta[ml] = 0;
    p += ml;
    if (mc->log_level <= LOG_LEVEL_INFO) {
        printf("[INFO] Decompressing model: %u layers\n", nl);
        printf("[INFO] Metadata: %s\n", meta);
    }
    char client[256] = "unknown";
    const char *cs = strstr(meta, "\"client_id\":\"");
    if (cs) {
        cs += 13;
        const char *ce = strchr(cs, '"');
        if (ce && (size_t)(ce - cs) < sizeof(client)) {
            memcpy(client, cs, (size_t)(ce - cs));
            client[ce - cs] = 0;
        }
    }
    free(meta);
    NDArray **grads = (NDArray **)calloc(nl ? nl : 1, sizeof(NDArray *));
    char **names = (char **)calloc(nl ? nl : 1, sizeof(char *));
    CompressedLayerData *C = (CompressedLayerData *)calloc(nl ? nl : 1, sizeof(CompressedLayerData));
    BatchItem *items = (BatchItem *)calloc(nl ? nl : 1, sizeof(BatchItem));
    if (!grads || !names || !C || !items) {
        free(grads); free(names); free(C); free(items);
        return NULL;
    }
    size_t parsed = 0;
    for (uint32_t i = 0; i < nl; i++) {
        uint32_t len;
        char tmp[64];
        CompressedLayerData *c = &C[i];
        if (get_bytes(&p, end, &len, 4) || (size_t)(end - p) < len) break;
        names[i] = (char *)malloc((size_t)len + 1);
        if (!names[i]) break;
        memcpy(names[i], p, len);
        names[i][len] = 0;
        p += len;
        char *fields[3] = {c->type, c->codec, c->original_dtype};
        size_t caps[3] = {sizeof(c->type), sizeof(c->codec), sizeof(c->original_dtype)};
        int bad = 0;
        for (int f = 0; f < 3 && !bad; f++) {
            if (get_bytes(&p, end, &len, 4) || (size_t)(end - p) < len) { bad = 1; break; }
            size_t k = len < caps[f] - 1 ? len : caps[f] - 1;
            memcpy(fields[f], p, k);
            fields[f][k] = 0;
            p += len;
        }
        (void)tmp;
        if (bad) break;
        snprintf(c->stored_dtype, sizeof(c->stored_dtype), "%s", c->original_dtype);
        uint32_t nd;
        if (get_bytes(&p, end, &nd, 4) || nd > MAX_NDIM) break;
        c->ndim = nd;
        if (get_bytes(&p, end, c->shape, nd * sizeof(size_t))) break;
        uint64_t sz;
        if (get_bytes(&p, end, &sz, 8) || (uint64_t)(end - p) < sz) break;
        c->data = (uint8_t *)p; c->data_size = (size_t)sz; p += sz;
        if (get_bytes(&p, end, &sz, 8) || (uint64_t)(end - p) < sz) break;
        c->bitmap = sz ? (uint8_t *)p : NULL; c->bitmap_size = (size_t)sz; p += sz;
        if (get_bytes(&p, end, &sz, 8) || (uint64_t)(end - p) < sz) break;
        c->dominant_signs = sz ? (uint8_t *)p : NULL; c->dominant_signs_size = (size_t)sz; p += sz;
        if (get_bytes(&p, end, &c->current_mean, 4) || get_bytes(&p, end, &c->current_std, 4) ||
            get_bytes(&p, end, &c->prev_mean, 4) || get_bytes(&p, end, &c->prev_std, 4))
            break;
        uint64_t np;
        if (get_bytes(&p, end, &np, 8)) break;
        c->num_predicted_kernels = (int)np;
        items[i].layer_name = names[i];
        items[i].compressed = c;
        parsed++;
    }
    if (parsed) {
        int prev = dev_enter(mc);
        mc_decompress_items(mc, items, parsed, client, grads, FALCOM_LOC_HOST);
        dev_leave(mc, prev);
    }
    for (size_t i = 0; i < parsed; i++)
        if (!grads[i]) fprintf(stderr, "[ERROR] Failed to decompress layer %zu: %s\n", i, names[i]);
    free(C);
    free(items);
    *layer_names_out = names;
    *num_layers_out = nl;
    return grads;
}

/* ------------------------------------------------------------- extensions */
MC_EXPORT int falcom_set_residual_codec(MomentumCompressor *mc, const char *codec) {
    int c = codec_parse(codec);
    if (!mc || c < 0) return ERROR_INVALID_PARAM;
    mc->residual_codec = c;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_frame_mode(MomentumCompressor *mc, const char *mode) {
    if (!mc || !mode) return ERROR_INVALID_PARAM;
    if (!strcmp(mode, "gpu")) mc->frame_mode = MC_FRAME_GPU;
    else if (!strcmp(mode, "libzstd")) {
        if (!zf_libzstd_available()) return ERROR_NOT_FOUND;
        mc->frame_mode = MC_FRAME_LIBZSTD;
    } else return ERROR_INVALID_PARAM;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_payload_location(MomentumCompressor *mc, int loc) {
    if (!mc || loc < FALCOM_LOC_AUTO || loc > FALCOM_LOC_DEVICE) return ERROR_INVALID_PARAM;
    mc->payload_loc = loc;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_output_location(MomentumCompressor *mc, int loc) {
    if (!mc || loc < FALCOM_LOC_AUTO || loc > FALCOM_LOC_DEVICE) return ERROR_INVALID_PARAM;
    mc->output_loc = loc;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_stream(MomentumCompressor *mc, void *stream) {
    if (!mc) return ERROR_INVALID_PARAM;
    mc->stream = stream ? (cudaStream_t)stream : mc->own_stream;
    return ERROR_NONE;
}

MC_EXPORT int falcom_get_device(const MomentumCompressor *mc) { return mc ? mc->device : -1; }

MC_EXPORT const char *falcom_last_error(const MomentumCompressor *mc) { return mc ? mc->last_error : ""; }

MC_EXPORT int falcom_last_launches(const MomentumCompressor *mc) { return mc ? mc->last_launches : 0; }

MC_EXPORT long long falcom_total_launches(const MomentumCompressor *mc) { return mc ? mc->total_launches : 0; }

MC_EXPORT int falcom_is_device_pointer(const void *ptr) {
    int d = -1;
    return mc_ptr_is_device(ptr, &d);
}

/* ----------------------------------------------------------- aggregate */
MC_EXPORT int falcom_set_aggregate(MomentumCompressor *mc, float *aggregate, const size_t *offsets, size_t n,
                                   float weight) {
    if (!mc) return ERROR_INVALID_PARAM;
    if (!aggregate) {
        free(mc->agg_off);
        mc->agg_off = NULL;
        mc->agg = NULL;
        mc->agg_n = 0;
        mc->agg_store = 0;
        mc->agg_no_output = 0;
        memset(&mc->agg_shards, 0, sizeof(mc->agg_shards));
        return ERROR_NONE;
    }
    int d = -1;
    if (!offsets || n == 0 || !mc_ptr_is_device(aggregate, &d) || d != mc->device) {
        mc_set_error(mc, "falcom_set_aggregate: aggregate must be device memory of device %d, with offsets",
                     mc->device);
        return ERROR_INVALID_PARAM;
    }
    size_t *o = (size_t *)malloc(n * sizeof(size_t));
    if (!o) return ERROR_ALLOCATION;
    memcpy(o, offsets, n * sizeof(size_t));
    free(mc->agg_off);
    mc->agg_off = o;
    mc->agg = aggregate;
    mc->agg_n = n;
    mc->agg_w = weight;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_aggregate_store(MomentumCompressor *mc, int store) {
    if (!mc || (store != 0 && store != 1)) return ERROR_INVALID_PARAM;
    mc->agg_store = store;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_aggregate_only(MomentumCompressor *mc, int on) {
    if (!mc || (on != 0 && on != 1)) return ERROR_INVALID_PARAM;
    mc->agg_no_output = on;
    return ERROR_NONE;
}

MC_EXPORT int falcom_set_aggregate_shards(MomentumCompressor *mc, float *const *landing, int nranks, int rank,
                                          size_t shard_elems) {
    if (!mc) return ERROR_INVALID_PARAM;
    if (!landing || nranks == 0) {
        memset(&mc->agg_shards, 0, sizeof(mc->agg_shards));
        return ERROR_NONE;
    }
    if (nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks || shard_elems % 64 != 0 ||
        shard_elems < MC_TILE_ELEMS) {
        mc_set_error(mc, "falcom_set_aggregate_shards: need 1..%d ranks, 0 <= rank < nranks and a shard of a "
                         "multiple of 64 elements, at least %d", MC_MAX_RANKS, MC_TILE_ELEMS);
        return ERROR_INVALID_PARAM;
    }
    for (int r = 0; r < nranks; r++) {
        if (!landing[r] || ((uintptr_t)landing[r] & 15) != 0) {
            mc_set_error(mc, "falcom_set_aggregate_shards: landing buffer %d is NULL or not 16-byte aligned", r);
            return ERROR_INVALID_PARAM;
        }
    }
    memset(&mc->agg_shards, 0, sizeof(mc->agg_shards));
    for (int r = 0; r < nranks; r++) mc->agg_shards.landing[r] = landing[r];
    mc->agg_shards.shard = (int64_t)shard_elems;
    mc->agg_shards.nranks = nranks;
    mc->agg_shards.rank = rank;
    return ERROR_NONE;
}

MC_EXPORT int falcom_shard_reduce(const float *landing, int nranks, int rank, size_t shard_elems,
                                  size_t total_elems, float *const *aggregates, void *stream) {
    if (!landing || !aggregates || nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks ||
        shard_elems % 64 != 0 || shard_elems == 0 || total_elems > (size_t)nranks * shard_elems ||
        ((uintptr_t)landing & 15) != 0) {
        fprintf(stderr, "[ERROR] falcom_shard_reduce: invalid arguments\n");
        return ERROR_INVALID_PARAM;
    }
    for (int r = 0; r < nranks; r++) {
        if (!aggregates[r] || ((uintptr_t)aggregates[r] & 15) != 0) {
            fprintf(stderr, "[ERROR] falcom_shard_reduce: aggregate %d is NULL or not 16-byte aligned\n", r);
            return ERROR_INVALID_PARAM;
        }
    }
    return mc_launch_shard_reduce(landing, nranks, rank, (int64_t)shard_elems, (int64_t)total_elems, aggregates,
                                  stream) == 1 ? ERROR_NONE : ERROR_DECOMPRESSION;
}

MC_EXPORT int falcom_peer_allreduce(float *const *aggregates, int nranks, int rank, size_t shard_elems,
                                    size_t total_elems, void *stream) {
    if (!aggregates || nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks ||
        shard_elems % 64 != 0 || shard_elems == 0 || total_elems > (size_t)nranks * shard_elems) {
        fprintf(stderr, "[ERROR] falcom_peer_allreduce: invalid arguments\n");
        return ERROR_INVALID_PARAM;
    }
    for (int r = 0; r < nranks; r++) {
        if (!aggregates[r] || ((uintptr_t)aggregates[r] & 15) != 0) {
            fprintf(stderr, "[ERROR] falcom_peer_allreduce: aggregate %d is NULL or not 16-byte aligned\n", r);
            return ERROR_INVALID_PARAM;
        }
    }
    return mc_launch_peer_allreduce(aggregates, nranks, rank, (int64_t)shard_elems, (int64_t)total_elems,
                                    stream) >= 0 ? ERROR_NONE : ERROR_DECOMPRESSION;
}

MC_EXPORT int falcom_peer_allreduce_sync(float *const *aggregates, uint32_t *const *flags, int nranks, int rank,
                                         size_t shard_elems, size_t total_elems, uint32_t epoch, void *stream) {
    if (!aggregates || !flags || nranks < 1 || nranks > MC_MAX_RANKS || rank < 0 || rank >= nranks ||
        shard_elems % 64 != 0 || shard_elems == 0 || total_elems > (size_t)nranks * shard_elems) {
        fprintf(stderr, "[ERROR] falcom_peer_allreduce_sync: invalid arguments\n");
        return ERROR_INVALID_PARAM;
    }
    for (int r = 0; r < nranks; r++) {
        if (!aggregates[r] || ((uintptr_t)aggregates[r] & 15) != 0 || !flags[r] || ((uintptr_t)flags[r] & 3) != 0) {
            fprintf(stderr, "[ERROR] falcom_peer_allreduce_sync: aggregate or flag block %d is NULL or misaligned\n",
                    r);
            return ERROR_INVALID_PARAM;
        }
    }
    return mc_launch_peer_allreduce_sync(aggregates, flags, nranks, rank, (int64_t)shard_elems, (int64_t)total_elems,
                                         epoch, stream) >= 0 ? ERROR_NONE : ERROR_DECOMPRESSION;
}

/* Device address of [p, p + bytes) for a kernel of the current device:
 * device memory of that device as is, pinned host memory through its mapped
 * device pointer; NULL (with a message) for anything else. */
static void *sm_copy_addr(const void *p, size_t bytes, const char *what) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) {
        (void)cudaGetLastError();
        return NULL;
    }
    void *res = NULL;
    for (int end = 0; end < 2; end++) {
        const void *q = end ? (const void *)((const uint8_t *)p + bytes - 1) : p;
        struct cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, q) != cudaSuccess) {
            (void)cudaGetLastError();
            at.type = cudaMemoryTypeUnregistered;
        }
        void *a = NULL;
        if ((at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) && at.device == cur)
            a = (void *)q;
        else if (at.type == cudaMemoryTypeHost && at.devicePointer)
            a = at.devicePointer;
        if (!a) {
            fprintf(stderr, "[ERROR] falcom_copy_sm: %s is neither device memory of the current device nor pinned "
                            "host memory\n", what);
            return NULL;
        }
        if (!end) res = a;
        else if ((uint8_t *)a != (uint8_t *)res + bytes - 1) {
            fprintf(stderr, "[ERROR] falcom_copy_sm: %s range is not contiguous in the device address space\n", what);
            return NULL;
        }
    }
    return res;
}

MC_EXPORT int falcom_copy_sm(void *dst, const void *src, size_t bytes, int nblocks, void *stream) {
    if (bytes == 0) return ERROR_NONE;
    if (!dst || !src) {
        fprintf(stderr, "[ERROR] falcom_copy_sm: NULL pointer\n");
        return ERROR_INVALID_PARAM;
    }
    void *d = sm_copy_addr(dst, bytes, "destination");
    const void *s = d ? sm_copy_addr(src, bytes, "source") : NULL;
    if (!d || !s) return ERROR_INVALID_PARAM;
    return mc_launch_copy(d, s, (int64_t)bytes, nblocks > 0 ? nblocks : 32, stream) >= 0 ? ERROR_NONE
                                                                                          : ERROR_COMPRESSION;
}

/* ----------------------------------------------------------- kernel timing */
static const char *k_names[MC_NKERN] = {"enc_pass1_stats_sign", "enc_pass2_variance", "enc_pass3_predict",
                                        "enc_pass4_quantize_pack", "frames_expand",
                                        "dec_prefix", "dec_reconstruct", "enc_finalize"};

mc_ktrace *mc_trace_begin(MomentumCompressor *mc) {
    if (!mc->ktiming) return NULL;
    if (!mc->ktrace.ev[0]) {
        for (int i = 0; i < 2 * MC_KTRACE_MAX; i++) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return NULL;
            mc->ktrace.ev[i] = (void *)e;
        }
    }
    mc->ktrace.n = 0;
    return &mc->ktrace;
}

void mc_trace_end(MomentumCompressor *mc) {
    if (!mc->ktiming || !mc->ktrace.ev[0]) return;
    for (int i = 0; i < mc->ktrace.n; i++) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, (cudaEvent_t)mc->ktrace.ev[2 * i], (cudaEvent_t)mc->ktrace.ev[2 * i + 1]) ==
            cudaSuccess) {
            mc->ktime_ms[mc->ktrace.kid[i]] += ms;
            mc->kcount[mc->ktrace.kid[i]] += 1;
        }
    }
    (void)cudaGetLastError();
    mc->ktrace.n = 0;
}

MC_EXPORT int falcom_set_kernel_timing(MomentumCompressor *mc, int on) {
    if (!mc) return ERROR_INVALID_PARAM;
    mc->ktiming = on ? 1 : 0;
    memset(mc->ktime_ms, 0, sizeof(mc->ktime_ms));
    memset(mc->kcount, 0, sizeof(mc->kcount));
    return ERROR_NONE;
}

MC_EXPORT int falcom_kernel_times(const MomentumCompressor *mc, double *ms, long long *counts, int n) {
    if (!mc) return 0;
    for (int i = 0; i < n && i < MC_NKERN; i++) {
        if (ms) ms[i] = mc->ktime_ms[i];
        if (counts) counts[i] = mc->kcount[i];
    }
    return MC_NKERN;
}

MC_EXPORT const char *falcom_kernel_name(int id) {
    return (id >= 0 && id < MC_NKERN) ? k_names[id] : "";
}

MC_EXPORT void falcom_free_batch(BatchItem *items, size_t n, NDArray **outs) {
    /* one registry pass for all objects; arena references dropped per run of
     * objects that share an arena */
    const void **objs = (const void **)malloc(2 * n * sizeof(void *));
    mc_arena **ar = (mc_arena **)malloc(2 * n * sizeof(mc_arena *));
    if (!objs || !ar) {
        free(objs);
        free(ar);
        for (size_t i = 0; i < n; i++) {
            if (items && items[i].compressed) compressed_layer_data_free(items[i].compressed);
            if (items) items[i].compressed = NULL;
            if (outs && outs[i]) ndarray_destroy(outs[i]);
            if (outs) outs[i] = NULL;
        }
        return;
    }
    for (size_t i = 0; i < n; i++) {
        objs[i] = items ? items[i].compressed : NULL;
        objs[n + i] = outs ? outs[i] : NULL;
    }
    registry_take_many(objs, 2 * n, ar);
    mc_arena *run = NULL;
    int cnt = 0;
    for (size_t k = 0; k < 2 * n; k++) {
        if (!objs[k]) continue;
        if (!ar[k]) {   /* not library-owned: free it field by field */
            if (k < n) {
                CompressedLayerData *c = (CompressedLayerData *)objs[k];
                free(c->data);
                free(c->bitmap);
                free(c->dominant_signs);
                free(c);
            } else {
                NDArray *a = (NDArray *)objs[k];
                free(a->data);
                free(a->shape);
                free(a);
            }
            continue;
        }
        if (ar[k] != run) {
            arena_release_n(run, cnt);
            run = ar[k];
            cnt = 0;
        }
        cnt++;
    }
    arena_release_n(run, cnt);
    for (size_t i = 0; i < n; i++) {
        if (items) items[i].compressed = NULL;
        if (outs) outs[i] = NULL;
    }
    free(objs);
    free(ar);
}
