/*
 * mc_device.h -- plain-C descriptors shared by the host code and the sm_100a
 * kernels (mc_kernels.cu), plus the extern "C" launchers.
 *
 * Work is described per batch as a table of items (one per tensor) cut into
 * tiles; one CTA processes one tile.  Momentum tiles always hold whole conv
 * kernels (a multiple of 32 kernels except at the end of a layer), so every
 * per-kernel decision and every 32-bit word of the bitmap belongs to exactly
 * one tile.
 */
#ifndef MC_DEVICE_H
#define MC_DEVICE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* q = floor(x / d) for 32-bit x as ((umulhi(x, mul) + x) >> shift). */
typedef struct {
    uint32_t mul;
    uint32_t shift;
} mc_fastdiv;
mc_fastdiv mc_fastdiv_make(uint32_t d);

/* item kinds of the encoder table */
enum {
    MC_K_MOMENTUM = 0,  /* 4-D momentum layer: stats, bitmap, signs, memory, residual codec */
    MC_K_QUANT = 1,     /* direct lossy tensor through the residual codec */
    MC_K_COPY = 2,      /* direct lossy tensor stored raw ("sz3_memcpy") */
    MC_K_FRAME = 3      /* direct lossless tensor: zstd frame of its bytes */
};

/* residual codecs on the device */
enum { MC_DC_Q8 = 0, MC_DC_INT4 = 1, MC_DC_RAW = 2, MC_DC_Q8_RAW = 3, MC_DC_INT4_RAW = 4 };

typedef struct {
    const void *cur;        /* input (fp32 for MOMENTUM/QUANT/COPY, bytes for FRAME) */
    const float *prev;      /* MOMENTUM: encoder history head */
    const float *mem_in;    /* MOMENTUM: committed prediction memory, NULL = zeros */
    float *mem_out;         /* MOMENTUM: new prediction memory */
    void *hist_out;         /* copy of the input for the new history head, or NULL */
    uint8_t *data_out;      /* payload data slot (FRAME: the zstd frame) */
    uint8_t *bm_frame;      /* MOMENTUM: bitmap zstd frame slot */
    uint8_t *sg_frame;      /* MOMENTUM: dominant-sign zstd frame slot */
    int64_t sg_cap;         /* bytes of the sign frame slot */
    uint32_t *bm_words;     /* MOMENTUM: bitmap content, ceil(K/32) words */
    uint32_t *dom_words;    /* MOMENTUM: dominant sign per kernel, ceil(K/32) words */
    uint32_t *blk_pos;      /* MOMENTUM: frame offset of each bitmap block's content (~0 = RLE) */
    int32_t max_blocks;     /* MOMENTUM: capacity of blk_pos */
    int32_t wave;           /* launch wave the item runs in */
    int64_t n;              /* elements */
    int64_t K;              /* kernels (MOMENTUM) */
    int32_t ks;             /* kernel size h*w (MOMENTUM) */
    int32_t kind;
    int32_t codec;          /* MC_DC_* */
    int32_t tile_kernels;   /* MOMENTUM: kernels per tile; others: elements per tile */
    int32_t ntiles;
    int32_t tile_base;      /* index of the first tile in the batch tile list */
    int32_t elem_bytes;     /* bytes per element of the input */
    int32_t step;
    int32_t vec;            /* 1: every fp32 pointer of the item is 16-byte aligned */
    mc_fastdiv ksdiv;
    float lr;
    float thr;
    /* MOMENTUM: 1 when the history head `prev` is an exact copy of an input
     * whose mean and population std of |x| an earlier momentum encode of the
     * same layer computed (pm_known, ps_known): the passes then take them
     * instead of reading prev for them.  Same values, same reduction order:
     * the history has the input's shape and so its tiling. */
    int32_t prev_known;
    float pm_known, ps_known;
} mc_enc_item;

typedef struct {
    double s_cur, s_prev;   /* sums of |cur|, |prev| */
    double v_cur, v_prev;   /* sums of squared deviations */
    float mn, mx, maxr;
    int32_t P;
    int64_t mism;
} mc_enc_tile;

typedef struct {
    float cm, cs, pm, ps, gmin, gmax;
    float inv_ps;           /* 1/prev_std when prev_std > 1e-8, else 1 */
    float scale;            /* residual codec scale */
    float maxr;
    float pad0;
    int64_t P;              /* predicted kernels */
    int64_t mism;           /* sign mismatches over predicted elements */
    int64_t bm_size;        /* bitmap frame bytes */
    int64_t sg_size;        /* sign frame bytes (0 when no kernel is predicted) */
    uint32_t ticket[4];     /* last-CTA election per pass; zeroed before launch */
    int32_t err;
    int32_t pad1;
} mc_enc_result;


typedef struct {
    const mc_enc_item *items;   /* device */
    mc_enc_result *results;     /* device, zeroed by the caller before the first wave */
    int32_t nitems;             /* items covered by the finalize kernels of this launch */
    const void *all_tiles;      /* device mc_tile_ref[]: tiles processed by passes 1 and 4 */
    int32_t nall_tiles;
    const void *mom_tiles;      /* device mc_tile_ref[]: tiles of momentum items (passes 2, 3) */
    int32_t nmom_tiles;
    mc_enc_tile *tiles;         /* device scratch, one per tile id */
    int64_t *tile_poff;         /* device scratch, ntiles */
    int32_t staged;             /* 1: stage tiles of aligned items in shared memory (bulk copies) */
    int32_t wave;               /* wave of this launch (finalize kernels skip other items) */
    int32_t item0;              /* finalize kernels: items item0 .. item0 + nitems - 1 */
    int32_t pad;
} mc_enc_launch;

/* One entry of a launch's tile list: tile id and the item it belongs to. */
typedef struct {
    int32_t tile;
    int32_t item;
} mc_tile_ref;

/* ---------------------------------------------------------------- decode */
enum {
    MC_D_MOMENTUM = 0,      /* full reconstruction with memory update */
    MC_D_RESIDUAL = 1,      /* residual only (no usable history / bitmap) */
    MC_D_QUANT = 2,         /* direct, codes * scale */
    MC_D_COPY = 3           /* direct, bytes copied (raw floats or lossless content) */
};

/* Elements of one tile: the unit of work of one CTA of the streaming
 * kernels and the capacity of one array of its shared-memory stage.  A
 * momentum tile holds a multiple of 32 whole kernels (at least 32; a power
 * of two when the layer's bitmap frame has more than one block) with at
 * most MC_TILE_ELEMS elements; other tiles hold MC_TILE_ELEMS elements (2x
 * that for the encoder's direct quantised tiles, whose input fills a
 * two-array stage; 4x for byte copies). */
#define MC_TILE_ELEMS 4096

/* zstd framing shared by encoder and decoder: single-segment frame header
 * (magic, descriptor 0xA0 and a 4-byte content size: 9 bytes), then blocks of
 * at most 2^17 content bytes, each behind a 3-byte block header. */
#define MC_ZBLOCK_LOG2 17
#define MC_ZBLOCK (1 << MC_ZBLOCK_LOG2)
#define MC_ZHDR 9

/* Sharded server aggregate over peer memory (a reduce-scatter fused into
 * the decoder).  The aggregate's elements are split into nranks shards of
 * `shard` elements; rank s owns shard s.  Every rank has a landing buffer of
 * nranks * shard floats, slot r (elements [r * shard, (r + 1) * shard)) for
 * rank r's contribution; landing[s] is rank s's buffer as addressed from
 * this device (peer memory).  The decoder of rank `rank` writes the value of
 * aggregate element x to landing[x / shard][rank * shard + x % shard]. */
#define MC_MAX_RANKS 8
typedef struct {
    float *landing[MC_MAX_RANKS];
    int64_t shard;              /* elements per shard: a multiple of 64, at least MC_TILE_ELEMS */
    int32_t nranks;
    int32_t rank;
} mc_agg_shards;

/* How the decoder reads a bitmap / sign / lossless payload. */
enum {
    MC_BM_WORDS = 0,        /* contiguous content (expanded, or staged content) */
    MC_BM_RAW = 1,          /* zstd frame of Raw blocks, read in place */
    MC_BM_RLE = 2           /* zstd frame of RLE blocks, read in place */
};

typedef struct {
    const uint8_t *data;        /* codes (after the scale header), raw floats or content bytes */
    const uint32_t *bm_words;   /* MOMENTUM: bitmap content words (WORDS / RAW1) */
    const uint8_t *bm_frame;    /* MOMENTUM: the bitmap frame (RAW1 / RLE1) */
    const uint8_t *sg_bytes;    /* MOMENTUM: sign content (WORDS / RAW1), NULL when absent */
    const uint8_t *sg_frame;    /* MOMENTUM: the sign frame (RAW1 / RLE1) */
    int64_t sg_len;             /* sign content bytes (when sg_len_ptr is NULL) */
    const int64_t *sg_len_ptr;  /* device-expanded sign content length, -1 = failed */
    const int64_t *bm_len_ptr;  /* device-expanded bitmap content length, -1 = failed */
    const float *prev;          /* MOMENTUM: decoder history head */
    const float *mem_in;        /* MOMENTUM: decoder memory, NULL = zeros */
    float *mem_out;
    void *hist_out;             /* decoded tensor (becomes the history head) */
    void *out;                  /* optional second copy (device output), NULL */
    /* fused server-side weighted aggregate of a float32 item (NULL: none):
     * agg[e] = fma(agg_w, decoded[e], agg[e]), or with agg_store set
     * fma(agg_w, decoded[e], +0) (agg not read: the bits of clearing to +0
     * and adding) */
    float *agg;
    float agg_w;
    int32_t agg_store;
    int32_t agg_vec;            /* 1: agg is 16-byte aligned */
    int32_t agg_shard;          /* 1: the aggregate value goes to its owner's landing slot (mc_agg_shards) */
    int64_t agg_off;            /* element offset of the item in the aggregate */
    int64_t n;
    int64_t K;
    int64_t bm_bits;            /* min(bitmap content bytes*8, K) */
    int32_t ks;
    int32_t kind;
    int32_t codec;              /* MC_DC_* for the residual / QUANT data */
    int32_t tile_kernels;
    int32_t ntiles;
    int32_t tile_base;
    int32_t elem_bytes;
    int32_t vec;                /* 1: float4 / packed-code access is aligned */
    int32_t bm_mode;            /* MC_BM_* */
    int32_t sg_mode;            /* MC_BM_* */
    int32_t data_mode;          /* COPY from a frame: MC_BM_WORDS (content), RAW1 or RLE1 */
    int32_t pad2;
    const uint8_t *data_frame;  /* COPY: the lossless zstd frame read in place */
    const float *scale_ptr;     /* device pointer to the f32 scale header (any alignment) */
    mc_fastdiv ksdiv;
    float cm, cs, pm, ps, lr;
} mc_dec_item;

typedef struct {
    int64_t P;
    uint32_t ticket;
    int32_t err;
} mc_dec_result;

/* One device-resident zstd frame to expand into contiguous content. */
typedef struct {
    const uint8_t *frame;
    int64_t frame_size;
    uint8_t *dst;
    int64_t cap;                /* bytes available at dst */
    int64_t *content_out;       /* content bytes produced, -1 on a format error */
} mc_unframe_job;

typedef struct {
    const mc_dec_item *items;
    mc_dec_result *results;     /* zeroed by the caller */
    int32_t nitems;
    const void *all_tiles;      /* mc_tile_ref[] for the reconstruct kernel */
    int32_t nall_tiles;
    const void *mom_tiles;      /* mc_tile_ref[] of momentum items (prefix kernel) */
    int32_t nmom_tiles;
    int32_t *tile_count;        /* scratch: predicted kernels per momentum tile */
    int64_t *tile_poff;         /* scratch: first predicted kernel of each momentum tile in the dense signs */
    int32_t staged;             /* 1: stage tiles of aligned items in shared memory (bulk copies) */
    int32_t item0, item1;       /* items [item0, item1) own this launch's tiles */
    int32_t pad;
    mc_agg_shards shards;       /* sharded aggregate (items with agg_shard set) */
} mc_dec_launch;


/* Optional per-kernel event trace (events created by the host). */
enum {
    MC_KT_ENC_PASS1 = 0, MC_KT_ENC_PASS2, MC_KT_ENC_PASS3, MC_KT_ENC_PASS4,
    MC_KT_UNFRAME, MC_KT_DEC_PREFIX, MC_KT_DEC_RECON, MC_KT_ENC_FINAL, MC_NKERN
};
#define MC_KTRACE_MAX 64
typedef struct {
    void *ev[2 * MC_KTRACE_MAX];   /* cudaEvent_t pairs */
    int kid[MC_KTRACE_MAX];
    int n;
} mc_ktrace;

/* Second half of the sharded aggregate: rank `rank` sums its shard over the
 * nranks slots of its own landing buffer, in rank order, and stores the sum
 * into aggregates[r][rank * shard + i] for every rank r (an all-gather by
 * peer stores); elements at or beyond `total` are not written.  Returns 1,
 * or a negative value when the launch failed. */
int mc_launch_shard_reduce(const float *landing, int nranks, int rank, int64_t shard, int64_t total,
                           float *const *aggregates, void *stream);
/* one-shot in-place sum all-reduce of elements [rank*shard, min((rank+1)*shard, total)) over the ranks'
 * aggregates (peer loads and stores); 1 launched, 0 nothing to do, -1 error */
/* copy of `bytes` bytes by a kernel of `nblocks` CTAs (device addresses; pinned host memory mapped into the
 * device address space included); 1 launched, 0 nothing to do, -1 error */
int mc_launch_copy(void *dst, const void *src, int64_t bytes, int nblocks, void *stream);
int mc_launch_peer_allreduce(float *const *aggregates, int nranks, int rank, int64_t shard, int64_t total,
                             void *stream);
/* the same with the barriers before and after it done by the kernel over the ranks' flag blocks (18 words each,
 * zeroed before the first round); 1 launched, -1 error */
int mc_launch_peer_allreduce_sync(float *const *aggregates, uint32_t *const *flags, int nranks, int rank,
                                  int64_t shard, int64_t total, uint32_t epoch, void *stream);

/* Launchers: return the number of kernels launched, or a negative value
 * when a launch failed.  `tr` may be NULL. */
int mc_launch_encode(const mc_enc_launch *L, void *stream, mc_ktrace *tr);
int mc_launch_decode(const mc_dec_launch *L, void *stream, mc_ktrace *tr);
int mc_launch_unframe(const mc_unframe_job *jobs, int njobs, void *stream, mc_ktrace *tr);

/* Reusable device / pinned scratch owned by one compressor instance. */
typedef struct {
    void *ptr;
    size_t bytes;
} mc_sbuf;
typedef struct {
    mc_sbuf dev[16];
    mc_sbuf host[8];
    int device;
} mc_scratch;
void *scratch_dev(mc_scratch *s, int slot, size_t bytes);
void *scratch_host(mc_scratch *s, int slot, size_t bytes);
void scratch_free(mc_scratch *s);

#ifdef __cplusplus
}
#endif
#endif
