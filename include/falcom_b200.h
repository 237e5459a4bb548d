/*
 * falcom_b200.h -- extension entry points of the B200 FalCom codec.
 *
 * None of these exist in the reference interface; a caller that only uses
 * momentum_compressor.h (for example EB-FaLCom's FalComC.py) gets the
 * defaults listed here, which can also be set through environment variables
 * read at momentum_compressor_create():
 *
 *   FALCOM_RESIDUAL_CODEC = q8 | int4 | raw | q8_raw | int4_raw   (default q8)
 *   FALCOM_FRAME_MODE     = gpu | libzstd                          (default gpu)
 */
#ifndef FALCOM_B200_H
#define FALCOM_B200_H

#include "momentum_compressor.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Residual codec: where the reference runs SZ3 (momentum residual with an ABS
 * bound, direct lossy tensors with a REL bound), this codec runs a symmetric
 * quantiser.
 *   "q8"       codec tag "q8":   [f32 scale][int8 code x n]
 *   "int4"     codec tag "int4": [f32 scale][(q+8) nibbles, element 2i low]
 *   "raw"      codec tag "sz3_memcpy": raw fp32 (what the reference emits
 *              when SZ3 is unavailable); bit-comparable with the reference
 *   "q8_raw" / "int4_raw"  quantise, then store the dequantised fp32 values
 *              with codec tag "sz3_memcpy" so an unmodified reference decoder
 *              reads them.
 * Returns 0, or ERROR_INVALID_PARAM for an unknown name. */
int falcom_set_residual_codec(MomentumCompressor *mc, const char *codec);

/* zstd framing of bitmap / dominant-sign / lossless payloads.
 *   "gpu"      frames written on the GPU with Raw and RLE blocks only
 *              (RFC 8878); every zstd decoder, the reference's included,
 *              reads them.
 *   "libzstd"  host libzstd level 10, byte-identical to the reference's
 *              frames (reference momentum_compressor_openmp_simd_final.c:647). */
int falcom_set_frame_mode(MomentumCompressor *mc, const char *mode);

/* Where returned payloads / decoded arrays live.
 *   FALCOM_LOC_AUTO    same memory kind as the inputs of the call
 *   FALCOM_LOC_HOST    host memory (pinned, owned by the library)
 *   FALCOM_LOC_DEVICE  device memory of the instance's GPU
 * Device-resident CompressedLayerData / NDArray are released with the same
 * compressed_layer_data_free() / ndarray_destroy(). */
enum { FALCOM_LOC_AUTO = 0, FALCOM_LOC_HOST = 1, FALCOM_LOC_DEVICE = 2 };
int falcom_set_payload_location(MomentumCompressor *mc, int loc);
int falcom_set_output_location(MomentumCompressor *mc, int loc);

/* CUDA stream (cudaStream_t) the instance issues its work on; NULL selects
 * the instance's own stream.  Calls remain synchronous with the host. */
int falcom_set_stream(MomentumCompressor *mc, void *stream);

/* Device ordinal the instance was created on. */
int falcom_get_device(const MomentumCompressor *mc);

/* Last error message of the instance ("" when none). */
const char *falcom_last_error(const MomentumCompressor *mc);

/* Kernel launches issued by the last compress / decompress call, and the
 * number issued since the instance was created. */
int falcom_last_launches(const MomentumCompressor *mc);
long long falcom_total_launches(const MomentumCompressor *mc);

/* 1 when this pointer is device memory that the library can read directly. */
int falcom_is_device_pointer(const void *ptr);

/* Per-kernel device time.  When enabled, every kernel launch of the instance
 * is bracketed by CUDA events on the instance's stream; after each call the
 * elapsed times are added to per-kernel totals.  falcom_kernel_times fills
 * up to n totals (milliseconds) and launch counts, indexed by kernel id, and
 * returns the number of kernel ids; falcom_kernel_name names an id.
 * Enabling resets the totals. */
int falcom_set_kernel_timing(MomentumCompressor *mc, int on);

/* Releases, in one call, every CompressedLayerData held by items[0..n) and
 * every array in outs[0..n) (either pointer may be NULL); entries are reset
 * to NULL. */
void falcom_free_batch(BatchItem *items, size_t n, NDArray **outs);
int falcom_kernel_times(const MomentumCompressor *mc, double *ms, long long *counts, int n);
const char *falcom_kernel_name(int id);

/* Server-side weighted aggregate.  No counterpart in the reference
 * interface (the federated server sums the decoded client updates itself).
 *
 * While set, every momentum_compressor_decompress_batch call on `mc` also
 * adds weight * (decoded item i) into aggregate[offsets[i] ...
 * offsets[i] + numel_i) for every item i < n that is float32 (other dtypes
 * are not added).  The addition (one fma per element) is done by the
 * decoder's reconstruct kernel as it writes each decoded element, so the
 * aggregate costs no pass of its own and is complete when the call
 * returns.  `aggregate` is float32 device memory of the instance's device,
 * `offsets` element offsets (copied); items must not overlap in the
 * aggregate; a region 16-byte aligned is written with vector stores.  Set it
 * again to change the weight (one call per client); aggregate = NULL stops
 * it.  The aggregate is valid when the call returns 0: an item that fails
 * after its reconstruction ran may already have written its region, and the
 * call then reports the failure.  Returns 0, or ERROR_INVALID_PARAM when
 * aggregate is not device memory of the instance's device. */
int falcom_set_aggregate(MomentumCompressor *mc, float *aggregate, const size_t *offsets, size_t n,
                         float weight);

/* Store mode of the weighted aggregate.  No counterpart in the reference.
 *   store = 0  (default) aggregate[...] += weight * decoded
 *   store = 1  aggregate[...] = weight * decoded, computed as
 *              fma(weight, decoded, +0): the same bits as clearing the region
 *              to +0 and adding, without the clear or the read of the old
 *              value.  For the first client of a round.
 * Applies to the following decompress_batch calls until changed;
 * falcom_set_aggregate(mc, NULL, ...) resets it to 0.  Items that are not
 * float32 leave their region as it was.
 * Returns 0, or ERROR_INVALID_PARAM for mc NULL or store not 0 / 1. */
int falcom_set_aggregate_store(MomentumCompressor *mc, int store);

/* Aggregate-only decoding.  No counterpart in the reference.
 *   on = 1  items that go into the aggregate (float32 items with an offset)
 *           get no decoded array: decompress_batch sets out[i] = NULL for
 *           them, writes neither a device nor a host copy of the decoded
 *           tensor, and still updates the instance's history and memory
 *           (the next round decodes against them).  A server that only needs
 *           the aggregate saves one 4-byte write (and, for host outputs, the
 *           device-to-host copy) per element and client.  The call's return
 *           code reports success as before; items not added keep their
 *           arrays.
 *   on = 0  (default) every decoded item is returned.
 * falcom_set_aggregate(mc, NULL, ...) resets it to 0.  Returns 0, or
 * ERROR_INVALID_PARAM for mc NULL or on not 0 / 1. */
int falcom_set_aggregate_only(MomentumCompressor *mc, int on);

/* Sharded aggregate over several GPUs: the reduce-scatter of the
 * aggregate's cross-GPU sum fused into the decoder.  No counterpart in the
 * reference.
 *
 * The aggregate's elements are split into nranks shards of shard_elems
 * elements (a multiple of 64, at least 4096); rank s owns shard s.  Every
 * rank has a landing buffer of nranks * shard_elems floats; its slot r
 * (elements [r * shard_elems, (r + 1) * shard_elems)) receives rank r's
 * contribution to shard s.  landing[s] is rank s's landing buffer as
 * addressed from this instance's device (peer memory mapped with CUDA IPC,
 * 16-byte aligned; landing[rank] is this rank's own).  While set, the value
 * each decode computes for aggregate element x -- this rank's partial sum,
 * the local aggregate (not read in store mode) plus weight * decoded -- is
 * written to landing[x / shard_elems][rank * shard_elems + x % shard_elems]
 * over NVLink, by the reconstruct kernel as it decodes, instead of to the
 * local aggregate.  Use it for a rank's last client of a round (its earlier
 * clients go to the local aggregate as usual), then, once every rank's
 * decodes are done (a barrier on the stream, for example a one-element
 * all-reduce), falcom_shard_reduce on every rank, then a barrier again.
 * Aggregate offsets must be multiples of 4 and every item must lie inside
 * the nranks shards, else the decompress call fails with
 * ERROR_INVALID_PARAM.  landing = NULL or nranks = 0 switches it off, as
 * does falcom_set_aggregate(mc, NULL, ...).  Returns 0, or
 * ERROR_INVALID_PARAM. */
int falcom_set_aggregate_shards(MomentumCompressor *mc, float *const *landing, int nranks, int rank,
                                size_t shard_elems);

/* Second half of the sharded aggregate, on each rank after every rank's
 * decodes have landed: sums shard `rank` over the nranks slots of this
 * rank's own landing buffer, in rank order, and stores the sum into
 * aggregates[r][rank * shard_elems + i] for every rank r (peer stores over
 * NVLink, an all-gather), for elements below total_elems.  Every rank's
 * aggregate then holds the whole sum once all ranks' calls have completed
 * (a barrier on the stream).  aggregates[r] as addressed from the current
 * device, 16-byte aligned.  Queued on `stream` (cudaStream_t) without
 * waiting.  Returns 0, ERROR_INVALID_PARAM, or ERROR_DECOMPRESSION when the
 * launch fails. */
int falcom_shard_reduce(const float *landing, int nranks, int rank, size_t shard_elems, size_t total_elems,
                        float *const *aggregates, void *stream);

/* One-shot in-place sum all-reduce of float32 aggregates over NVLink peer
 * memory, the alternative to the sharded aggregate when the decodes write
 * local aggregates (plain falcom_set_aggregate): after every rank's decodes
 * are done (a barrier on the stream), each rank calls it once; rank `rank`
 * loads elements [rank * shard_elems, (rank + 1) * shard_elems) below
 * total_elems from every rank's aggregate, sums them in rank order and
 * stores the sum into every rank's aggregate, so every aggregate holds the
 * whole sum once all ranks' calls have completed (a barrier again, which
 * also keeps any rank from overwriting its aggregate while a peer still
 * reads it).  aggregates[r] as addressed from the current device (CUDA IPC
 * mappings of the peers' buffers), 16-byte aligned; shard_elems a multiple
 * of 64.  Queued on `stream` (cudaStream_t) without waiting.  Returns 0,
 * ERROR_INVALID_PARAM, or ERROR_DECOMPRESSION when the launch fails. */
int falcom_peer_allreduce(float *const *aggregates, int nranks, int rank, size_t shard_elems,
                          size_t total_elems, void *stream);

/* falcom_peer_allreduce with its two barriers done by the kernel itself over
 * flag words in peer memory, without the caller's barriers: flags[r] is
 * rank r's block of 18 uint32 (as addressed from the current device, 4-byte
 * aligned, zeroed before the first call), `epoch` the round number, larger
 * on every call (1, 2, ...; compared modulo 2^32), the same on every rank.
 * The kernel announces the rank's arrival to every rank when it starts (the
 * caller's decodes earlier on `stream` are then complete), waits for every
 * rank's arrival, sums the rank's shard in rank order into every rank's
 * aggregate, and returns once every rank has finished, so work queued after
 * it on `stream` sees the whole sum and cannot overwrite the aggregate
 * while a peer still uses it.  Every wait is bounded (about one second): a
 * rank that never arrives sets word 17 of the waiting ranks' blocks, and
 * their aggregates are then incomplete.  Queued on `stream` without
 * waiting.  Returns 0, ERROR_INVALID_PARAM, or ERROR_DECOMPRESSION when the
 * launch fails. */
int falcom_peer_allreduce_sync(float *const *aggregates, uint32_t *const *flags, int nranks, int rank,
                               size_t shard_elems, size_t total_elems, uint32_t epoch, void *stream);

/* Copies `bytes` bytes from src to dst with a kernel of `nblocks` CTAs (0:
 * 32) on `stream` (cudaStream_t) instead of a copy engine, returning without
 * waiting.  Each side is device memory of the current device or pinned host
 * memory (cudaHostAlloc / cudaHostRegister, read and written through its
 * mapped device address); pageable host memory is refused.  For callers
 * that pipeline host transfers around the codec calls: a large upload of the
 * next inputs or download of the aggregate issued as a copy-engine copy can
 * hold up the small table uploads and payload copies a compress or
 * decompress call queues on the copy engines behind it, while this copy
 * leaves the copy engines to them (at about 51 GB/s over PCIe 5 x16 on a
 * B200, against 55 for a copy engine).  Returns 0, ERROR_INVALID_PARAM, or
 * ERROR_COMPRESSION when the launch fails. */
int falcom_copy_sm(void *dst, const void *src, size_t bytes, int nblocks, void *stream);

/* Residual quantiser that allocates no memory.  No counterpart in the
 * reference interface.
 *
 * Writes the quantised payload of a float32 residual -- the same bytes the
 * codec stores in CompressedLayerData.data under codec tag "q8" (bits = 8:
 * [f32 scale][int8 code x n], 4 + n bytes) or "int4" (bits = 4: [f32 scale]
 * [(q + 8) nibbles, element 2i low], 4 + (n + 1) / 2 bytes) -- with
 * scale = max|r| / qmax (1 when max|r| == 0) and q = clamp(rint(r / scale)).
 * `residual` and `out` are device memory of the current CUDA device; the
 * work is queued on `stream` (cudaStream_t, NULL = the legacy default
 * stream) and the function returns without waiting for it.
 *
 * Who needs it: callers that cannot allocate device memory -- a training
 * step whose GPU memory belongs to another allocator (e.g. a framework's
 * caching allocator, which must account for every byte), and
 * latency-critical paths, where cudaMalloc / cudaFree would stall the GPU
 * (cudaFree synchronises the device).  The batch entry points above grow
 * device pools of their own on demand; this one only launches three kernels.
 *
 * Scratch is a fixed 65,792-byte __device__ array inside the library, one per
 * device (every GPU that loads the library holds it until exit), which bounds
 * n at FALCOM_NOALLOC_MAX_ELEMS (8192-element tiles x 16384 tiles).  Each call
 * writes every scratch word it reads before reading it, so no word has to
 * start at zero, and a call cut short leaves nothing a later call depends on.
 * The first call on each device (and in each CUDA context) does a one-time
 * set-up: it looks up the array's device address with cudaGetSymbolAddress;
 * make that call before any stream capture begins -- n = 0 does the set-up
 * only.  cudaDeviceReset destroys the array with its context; a call after a
 * reset in the same process is not supported.
 *
 * Calls share the scratch of their device, so calls on one device must not
 * overlap: issue them on one stream, or order them with events.  Two calls
 * running at once on different streams race and give wrong results.
 *
 * Returns 0; ERROR_INVALID_PARAM (message on stderr) when bits is not 8 or
 * 4, n > FALCOM_NOALLOC_MAX_ELEMS, or a pointer is NULL with n > 0;
 * ERROR_COMPRESSION when set-up or a launch fails, or when a CUDA error from
 * the caller's earlier work is already pending on the calling thread (then
 * nothing is launched and that error is left pending for its owner). */
#define FALCOM_NOALLOC_MAX_ELEMS 134217728LL
int falcom_quantize_residual_noalloc(const float *residual, size_t n, int bits, void *out, void *stream);

/* Replay rounds: one captured client update per file, in the layout the
 * reference's replay tools read (benchmark_real.c:30-89 load_test_data,
 * cuda_feasibility/profile_appfl_hot_rounds.py:47-72 read_round):
 *   u32 round | char client_id[64] | u64 layer_count, then per layer
 *   char name[256] | u64 shape[8] | u64 ndim | u32 dtype | u64 data_size |
 *   data_size bytes  (little-endian; dtype = DataType code).
 *
 * falcom_replay_open reads a file into one block of host memory
 * (FALCOM_LOC_HOST, malloc'd) or of device memory of `device`
 * (FALCOM_LOC_DEVICE; the data streams through pinned staging buffers while
 * the file is read) and returns the round, or NULL when the file cannot be
 * opened or is inconsistent (truncated, ndim above 8, unknown dtype,
 * data_size != numel * element size), as the reference loader returns NULL;
 * ndim 0 is a scalar.
 * falcom_replay_items returns falcom_replay_count items whose layer_name and
 * gradient are set (compressed NULL): ready for
 * momentum_compressor_compress_batch, valid until falcom_replay_close.
 * falcom_replay_bytes is the sum of the data sizes.
 *
 * falcom_replay_write writes items[0..n) (host or device gradients) as one
 * round file.  Returns 0, or ERROR_INVALID_PARAM (bad item, file not
 * writable), ERROR_ALLOCATION (write failed). */
typedef struct falcom_replay falcom_replay;
falcom_replay *falcom_replay_open(const char *path, int location, int device);
size_t falcom_replay_count(const falcom_replay *r);
uint32_t falcom_replay_round(const falcom_replay *r);
const char *falcom_replay_client(const falcom_replay *r);
size_t falcom_replay_bytes(const falcom_replay *r);
BatchItem *falcom_replay_items(falcom_replay *r);
void falcom_replay_close(falcom_replay *r);
int falcom_replay_write(const char *path, uint32_t round, const char *client_id, const BatchItem *items,
                        size_t n);

/* State checkpoint.  No counterpart in the reference, whose state
 * (momentum_compressor_openmp_simd_final.c:420-471) lives in process memory
 * only.
 *
 * falcom_state_save writes the instance's whole codec state -- for every
 * "client:layer" its step count and history head, every prediction memory,
 * the clients that own memories -- to `path`.  falcom_state_load replaces the
 * instance's state with a file's contents (on any instance and device), so
 * the next compress / decompress continues exactly where the saved instance
 * would; when loading fails the state is left unchanged.  Both wait for the
 * instance's stream.  Returns 0, or ERROR_NOT_FOUND (no such file),
 * ERROR_INVALID_PARAM (not a state file / not writable), ERROR_ALLOCATION. */
int falcom_state_save(MomentumCompressor *mc, const char *path);
int falcom_state_load(MomentumCompressor *mc, const char *path);

#ifdef __cplusplus
}
#endif

#endif /* FALCOM_B200_H */
