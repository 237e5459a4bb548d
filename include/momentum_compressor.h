/*
 * momentum_compressor.h -- C ABI of the B200 FalCom momentum-prediction codec.
 *
 * This header declares the same types and entry points, with the same struct
 * layouts, as the reference interface Gonglz/Compressor momentum_compressor.h,
 * so a program (or EB-FaLCom's FalComC.py over ctypes) built against the
 * reference links and runs against libmomentum_compressor.so from this
 * package unchanged.  Each declaration names the reference line it replaces.
 *
 * Memory rules (reference momentum_compressor.h:114-152, FalComC.py:287-319):
 *   - inputs are borrowed; NDArray.data may be host memory (pageable or
 *     pinned) or, as an extension, CUDA device memory of the current device;
 *   - every CompressedLayerData / NDArray returned by the library is owned by
 *     the caller and released with compressed_layer_data_free() /
 *     ndarray_destroy() from this library (never with free()).
 */
#ifndef MOMENTUM_COMPRESSOR_H
#define MOMENTUM_COMPRESSOR_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Limits: reference momentum_compressor.h:31-58 */
#define MAX_KEY_LENGTH 512
#define MAX_CLIENT_ID_LENGTH 256
#define MAX_LAYER_NAME_LENGTH 256
#define MAX_COMPRESSOR_NAME_LENGTH 64
#define MAX_PATH_LENGTH 512
#define MAX_ERROR_MESSAGE_LENGTH 256
#define MAX_NDIM 8
#define MIN_NDIM 1
#define DEFAULT_MOMENTUM_LR 0.07f
#define DEFAULT_CONSISTENCY_THRESHOLD 0.5f
#define DEFAULT_PARAM_COUNT_THRESHOLD 1024
#define DEFAULT_MAX_HISTORY_LENGTH 3
#define DEFAULT_ERROR_BOUND 1.0f
#define MIN_COMPRESSION_SIZE 1024
#define MAX_BATCH_SIZE 1024
#define STATS_INITIAL_CAPACITY 100
#define LOG_LEVEL_DEBUG 0
#define LOG_LEVEL_INFO 1
#define LOG_LEVEL_WARNING 2
#define LOG_LEVEL_ERROR 3

/* reference momentum_compressor.h:64-71 */
typedef enum {
    DTYPE_FLOAT32,
    DTYPE_FLOAT64,
    DTYPE_INT32,
    DTYPE_INT64,
    DTYPE_UINT8,
    DTYPE_UNKNOWN
} DataType;

/* reference momentum_compressor.h:73-81 */
typedef enum {
    ERROR_NONE = 0,
    ERROR_ALLOCATION = -1,
    ERROR_COMPRESSION = -2,
    ERROR_DECOMPRESSION = -3,
    ERROR_INVALID_PARAM = -4,
    ERROR_NOT_FOUND = -5,
    ERROR_SZ3_FAILED = -6
} ErrorCode;

/* reference momentum_compressor.h:84-90 (layout frozen: FalComC.py:47-55) */
typedef struct {
    void *data;          /* element buffer (host or device memory) */
    size_t *shape;       /* ndim extents */
    size_t ndim;
    size_t total_size;   /* product of the extents */
    DataType dtype;
} NDArray;

/* reference momentum_compressor.h:96-108 (layout frozen: FalComC.py:58-69) */
typedef struct {
    float momentum_lr;
    float consistency_threshold;
    char lossless_compressor[32];
    char error_bounding_mode[16];
    float error_bound;
    char sz3_lib_path[512];
    size_t param_count_threshold;
    int max_history_length;
} CompressorConfig;

/* reference momentum_compressor.h:114-152 (layout frozen: FalComC.py:72-105).
 * type:  "direct" | "direct_generic" | "momentum_predicted"
 * codec: "q8" | "int4" | "sz3_memcpy" | "sz3" | "zstd" | "blosc" | "pickle" */
typedef struct {
    char type[32];
    char codec[16];
    uint8_t *data;
    size_t data_size;
    uint8_t *bitmap;             /* zstd frame, momentum_predicted only */
    size_t bitmap_size;
    uint8_t *dominant_signs;     /* zstd frame, momentum_predicted only */
    size_t dominant_signs_size;
    size_t shape[MAX_NDIM];
    size_t ndim;
    char original_dtype[16];
    char stored_dtype[16];
    int step;
    int num_predicted_kernels;
    float prediction_ratio;
    float sign_mismatch_ratio;
    float current_mean, current_std;
    float prev_mean, prev_std;
    float global_min, global_max;
    double breakdown_stats_time;
    double breakdown_normalize_time;
    double breakdown_consistency_time;
    double breakdown_prediction_time;
    double breakdown_residual_compress_time;
    double breakdown_bitmap_compress_time;
    double breakdown_metadata_time;
    double breakdown_total_time;
} CompressedLayerData;

typedef struct MomentumCompressor MomentumCompressor;

/* reference momentum_compressor.h:169 */
MomentumCompressor *momentum_compressor_create(const CompressorConfig *config);
/* reference momentum_compressor.h:175 */
void momentum_compressor_destroy(MomentumCompressor *compressor);
/* reference momentum_compressor.h:182 */
void momentum_compressor_set_client(MomentumCompressor *compressor, const char *client_id);
/* reference momentum_compressor.h:192-196 */
CompressedLayerData *momentum_compressor_compress_layer(MomentumCompressor *compressor,
                                                        const char *layer_name,
                                                        const NDArray *gradient);
/* reference momentum_compressor.h:206-211 */
NDArray *momentum_compressor_decompress_layer(MomentumCompressor *compressor,
                                              const CompressedLayerData *compressed,
                                              const char *client_id, const char *layer_name);

/* reference momentum_compressor.h:220-225 */
typedef struct {
    const char *layer_name;
    const NDArray *gradient;
    CompressedLayerData *compressed;
    ErrorCode error;
} BatchItem;

/* reference momentum_compressor.h:247-252 (grouped path :4495-4705) */
int momentum_compressor_compress_batch(MomentumCompressor *compressor, BatchItem *items,
                                       size_t num_items, const char *client_id);
/* reference momentum_compressor.h:276-282 (:4707-4838) */
int momentum_compressor_decompress_batch(MomentumCompressor *compressor, const BatchItem *items,
                                         size_t num_items, const char *client_id,
                                         NDArray **out_gradients);
/* reference momentum_compressor.h:289 */
void momentum_compressor_reset_client(MomentumCompressor *compressor, const char *client_id);
/* reference momentum_compressor.h:295 */
void momentum_compressor_reset_all(MomentumCompressor *compressor);
/* reference momentum_compressor.h:301 */
void momentum_compressor_print_stats(const MomentumCompressor *compressor);

/* reference momentum_compressor.h:310-316 */
typedef struct {
    size_t total_compressions;
    float avg_prediction_ratio;
    float std_prediction_ratio;
    float avg_sign_mismatch_ratio;
    size_t num_predictions;
} CompressionStats;

/* reference momentum_compressor.h:321-326 */
typedef struct {
    char client_id[256];
    size_t history_length;
    int step_count;
    size_t num_memory_layers;
} ClientStats;

/* reference momentum_compressor.h:331-335 */
typedef struct {
    CompressionStats compression;
    ClientStats *clients;
    size_t num_clients;
} DetailedStats;

/* reference momentum_compressor.h:342 */
CompressionStats *momentum_compressor_get_stats(const MomentumCompressor *compressor);
/* reference momentum_compressor.h:349 */
DetailedStats *momentum_compressor_get_detailed_stats(const MomentumCompressor *compressor);
/* reference momentum_compressor.h:354-355 */
void compression_stats_free(CompressionStats *stats);
void detailed_stats_free(DetailedStats *stats);
/* reference momentum_compressor.h:362 */
void momentum_compressor_set_log_level(MomentumCompressor *compressor, const char *level);
/* reference momentum_compressor.h:369 */
void momentum_compressor_set_client_context(MomentumCompressor *compressor,
                                            const char *client_id);
/* reference momentum_compressor.h:374 */
int momentum_compressor_get_log_level(const MomentumCompressor *compressor);
/* reference momentum_compressor.h:379 */
const char *momentum_compressor_get_current_client_id(const MomentumCompressor *compressor);

/* reference momentum_compressor.h:391-398 (MOMC container :3600-3754) */
uint8_t *momentum_compressor_compress_model(MomentumCompressor *compressor,
                                            const NDArray **gradients, const char **layer_names,
                                            size_t num_layers, const char *client_id,
                                            size_t *out_size);
/* reference momentum_compressor.h:409-415 (:3756-3939) */
NDArray **momentum_compressor_decompress_model(MomentumCompressor *compressor,
                                               const uint8_t *compressed_data,
                                               size_t compressed_size, char ***layer_names,
                                               size_t *num_layers);

/* reference momentum_compressor.h:424 */
NDArray *ndarray_create(const size_t *shape, size_t ndim, DataType dtype);
/* reference momentum_compressor.h:429 */
void ndarray_destroy(NDArray *array);
/* reference momentum_compressor.h:434 */
NDArray *ndarray_copy(const NDArray *src);
/* reference momentum_compressor.h:439 */
void compressed_layer_data_free(CompressedLayerData *data);
/* reference momentum_compressor.h:444 */
CompressorConfig momentum_compressor_default_config(void);
/* reference momentum_compressor.h:454 */
void momentum_compressor_enable_breakdown(int enable);
/* reference momentum_compressor.h:460 */
void momentum_compressor_print_breakdown(void);
/* reference momentum_compressor_openmp_simd_final.c:197 (exported, not in the
 * reference header): pointer to the last grouped-batch timing record. */
const void *momentum_compressor_get_last_breakdown(void);

#ifdef __cplusplus
}
#endif

#endif /* MOMENTUM_COMPRESSOR_H */
