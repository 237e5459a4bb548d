// mc_noalloc.cu -- residual quantiser that never allocates device memory.
//
// falcom_quantize_residual_noalloc() produces, from a float32 residual in
// device memory, the exact bytes that the codec stores in a quantised
// payload (CompressedLayerData.data for codec tags "q8" / "int4"):
//   q8    [f32 scale][int8 code x n]
//   int4  [f32 scale][(q + 8) nibbles, element 2i in the low nibble]
// with scale = max|r| / qmax (1 when max|r| is 0) and
// q = clamp(rint(r / scale), -qmax, qmax), qmax 127 or 7.
//
// It is for callers that must not allocate: a training step whose device
// memory is owned by another allocator (a framework caching allocator that
// must see every byte), and latency-critical paths where cudaMalloc /
// cudaFree would stall, since cudaFree synchronises the whole device.  The
// batch entry points keep device pools of their own and may grow them on any
// call; this entry point only launches kernels on the caller's stream.
//
// Scratch lives in a file-scope __device__ array (g_quant_scratch, 65,792
// bytes per device): one max|r| slot per 8192-element tile and the scale.
// Its size bounds n at FALCOM_NOALLOC_MAX_ELEMS.  Every call writes each slot
// it reads before reading it, so nothing has to start at zero and a call
// that was cut short leaves nothing behind that a later call depends on.
//
// Three kernels, all on the caller's stream:
//   k_na_tiles   per-tile max|r| into the tile's slot
//   k_na_scale   one CTA: max over the tile slots, the scale into out[0..4)
//                and into the scale slot
//   k_na_codes   codes from the scale
// HBM-bound: 4 bytes read twice and 1 (q8) or 1/2 (int4) byte written per
// element; the second read of a residual under the 126 MB L2 hits in L2.

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "falcom_b200.h"

#define NA_TPB 256
#define NA_TILE 8192
#define NA_MAX_TILES 16384
#define NA_MAX_ELEMS ((int64_t)NA_TILE * NA_MAX_TILES)
#define NA_MAX_DEVICES 64

static_assert(NA_MAX_ELEMS == FALCOM_NOALLOC_MAX_ELEMS, "scratch bound and public limit differ");

// Words [0, NA_MAX_TILES): per-tile max|r| (float bits), written by
// k_na_tiles for the call's tiles before k_na_scale reads them.  Word
// NA_SCALE: the scale of the current call, written by k_na_scale before
// k_na_codes reads it.  The rest is padding.
#define NA_SCALE NA_MAX_TILES
#define NA_SCRATCH_WORDS (NA_MAX_TILES + 64)
static __device__ __align__(256) uint32_t g_quant_scratch[NA_SCRATCH_WORDS];

namespace {

__device__ __forceinline__ float na_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// max over the block of one float per thread; result valid in every thread
__device__ float na_block_max(float v, float *sh) {
    v = na_warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = sh[0];
    for (int j = 1; j < NA_TPB / 32; j++) m = fmaxf(m, sh[j]);
    return m;
}

__device__ __forceinline__ int na_quant(float r, float scale, float qm) {
    float v = rintf(__fdiv_rn(r, scale));
    v = fminf(qm, fmaxf(-qm, v));
    return (int)v;
}

__global__ void __launch_bounds__(NA_TPB) k_na_tiles(const float *__restrict__ x, int64_t n, int vec,
                                                     uint32_t *__restrict__ scratch) {
    __shared__ float sh[NA_TPB / 32];
    const int t = blockIdx.x;
    const int64_t e0 = (int64_t)t * NA_TILE;
    const int64_t e1 = min(e0 + (int64_t)NA_TILE, n);
    float m = 0.0f;
    if (vec) {   // x 16-byte aligned; tiles start at multiples of 8192 elements
        for (int64_t g = e0 + 4 * (int64_t)threadIdx.x; g < e1; g += 4 * NA_TPB) {
            if (g + 4 <= e1) {
                const float4 v = *(const float4 *)(x + g);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            } else {
                for (int64_t j = g; j < e1; j++) m = fmaxf(m, fabsf(x[j]));
            }
        }
    } else {
        for (int64_t g = e0 + threadIdx.x; g < e1; g += NA_TPB) m = fmaxf(m, fabsf(x[g]));
    }
    m = na_block_max(m, sh);
    if (threadIdx.x == 0) scratch[t] = __float_as_uint(m);
}

// One CTA: max over the ntiles tile slots, then the scale.
__global__ void __launch_bounds__(NA_TPB) k_na_scale(int ntiles, int qmax, uint8_t *__restrict__ out,
                                                     uint32_t *__restrict__ scratch) {
    __shared__ float sh[NA_TPB / 32];
    float a = 0.0f;
    for (int i = threadIdx.x; i < ntiles; i += NA_TPB) a = fmaxf(a, __uint_as_float(__ldcg(&scratch[i])));
    a = na_block_max(a, sh);
    if (threadIdx.x == 0) {
        const float scale = (a == 0.0f) ? 1.0f : __fdiv_rn(a, (float)qmax);
        const uint32_t b = __float_as_uint(scale);
        out[0] = (uint8_t)b;
        out[1] = (uint8_t)(b >> 8);
        out[2] = (uint8_t)(b >> 16);
        out[3] = (uint8_t)(b >> 24);
        scratch[NA_SCALE] = b;
    }
}

__global__ void __launch_bounds__(NA_TPB) k_na_codes(const float *__restrict__ x, int64_t n, int vec, int qmax,
                                                     uint8_t *__restrict__ out, const uint32_t *__restrict__ scratch) {
    const float scale = __uint_as_float(__ldcg(&scratch[NA_SCALE]));
    const float qm = (float)qmax;
    const int64_t e0 = (int64_t)blockIdx.x * NA_TILE;
    const int64_t e1 = min(e0 + (int64_t)NA_TILE, n);
    uint8_t *codes = out + 4;
    if (qmax == 127) {
        if (vec) {   // x 16-byte aligned, codes 4-byte aligned
            for (int64_t g = e0 + 4 * (int64_t)threadIdx.x; g < e1; g += 4 * NA_TPB) {
                if (g + 4 <= e1) {
                    const float4 v = *(const float4 *)(x + g);
                    const uint32_t w = (uint32_t)(uint8_t)na_quant(v.x, scale, qm) |
                                       ((uint32_t)(uint8_t)na_quant(v.y, scale, qm) << 8) |
                                       ((uint32_t)(uint8_t)na_quant(v.z, scale, qm) << 16) |
                                       ((uint32_t)(uint8_t)na_quant(v.w, scale, qm) << 24);
                    *(uint32_t *)(codes + g) = w;
                } else {
                    for (int64_t j = g; j < e1; j++) codes[j] = (uint8_t)(int8_t)na_quant(x[j], scale, qm);
                }
            }
        } else {
            for (int64_t g = e0 + threadIdx.x; g < e1; g += NA_TPB)
                codes[g] = (uint8_t)(int8_t)na_quant(x[g], scale, qm);
        }
    } else {
        // one output byte per thread step: elements 2b (low nibble) and 2b+1
        for (int64_t b = (e0 >> 1) + threadIdx.x; 2 * b < e1; b += NA_TPB) {
            const int64_t g = 2 * b;
            const uint32_t lo = (uint32_t)((na_quant(x[g], scale, qm) + 8) & 15);
            const uint32_t hi = g + 1 < e1 ? (uint32_t)((na_quant(x[g + 1], scale, qm) + 8) & 15) : 0u;
            codes[b] = (uint8_t)(lo | (hi << 4));
        }
    }
}

std::mutex g_setup_mu;
struct ScratchSlot {
    void *ctx;            // CUDA context the address belongs to
    uint32_t *ptr;        // device address of g_quant_scratch in it
};
ScratchSlot g_scratch[NA_MAX_DEVICES];

// CUcontext of the calling thread through the driver entry point (the
// library links the static runtime only); NULL when it cannot be had, and
// the cache is then kept per device alone.
void *current_context() {
    typedef int (*ctx_get_fn)(void **);
    static ctx_get_fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *fp = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fp, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (ctx_get_fn)fp;
        else
            (void)cudaGetLastError();
    });
    void *ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

// Device address of g_quant_scratch on the current device, looked up once
// per device and context (cudaGetSymbolAddress, with that device current);
// a call from another context (a context the caller created, or a primary
// context created again) looks it up anew.  NULL on failure (message on
// stderr).
uint32_t *scratch_of_current_device() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: no usable current CUDA device (%s)\n",
                e != cudaSuccess ? cudaGetErrorString(e) : "ordinal out of range");
        return nullptr;
    }
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_setup_mu);
    ScratchSlot &slot = g_scratch[dev];
    if (slot.ptr && slot.ctx == ctx) return slot.ptr;
    uint32_t *p = nullptr;
    e = cudaGetSymbolAddress((void **)&p, g_quant_scratch);
    if (e != cudaSuccess || !p) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: scratch set-up failed on device %d: %s\n", dev,
                cudaGetErrorString(e));
        return nullptr;
    }
    slot.ctx = ctx;
    slot.ptr = p;
    return p;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int falcom_quantize_residual_noalloc(const float *residual,
                                                                                      size_t n, int bits,
                                                                                      void *out, void *stream) {
    if (bits != 8 && bits != 4) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: bits must be 8 or 4, got %d\n", bits);
        return ERROR_INVALID_PARAM;
    }
    if (n > (size_t)NA_MAX_ELEMS) {
        fprintf(stderr,
                "[ERROR] falcom_quantize_residual_noalloc: n = %zu exceeds the maximum of %lld elements "
                "(scratch of %d tiles x %d elements)\n",
                n, (long long)NA_MAX_ELEMS, NA_MAX_TILES, NA_TILE);
        return ERROR_INVALID_PARAM;
    }
    uint32_t *scratch = scratch_of_current_device();
    if (!scratch) return ERROR_COMPRESSION;
    if (n == 0) return ERROR_NONE;   // set-up only
    if (!residual || !out) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: NULL residual or output pointer\n");
        return ERROR_INVALID_PARAM;
    }
    const int qmax = bits == 8 ? 127 : 7;
    const int ntiles = (int)((n + NA_TILE - 1) / NA_TILE);
    const uintptr_t xa = (uintptr_t)residual, oa = (uintptr_t)out + 4;
    const int vec = (xa & 15) == 0 && (bits == 4 || (oa & 3) == 0);
    cudaStream_t s = (cudaStream_t)stream;
    // an error left pending by the caller's earlier work stays the caller's:
    // nothing is launched, and it is not cleared
    cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: a CUDA error is already pending (%s); "
                        "nothing launched\n", cudaGetErrorString(e));
        return ERROR_COMPRESSION;
    }
    k_na_tiles<<<ntiles, NA_TPB, 0, s>>>(residual, (int64_t)n, vec, scratch);
    if ((e = cudaGetLastError()) == cudaSuccess) {
        k_na_scale<<<1, NA_TPB, 0, s>>>(ntiles, qmax, (uint8_t *)out, scratch);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        k_na_codes<<<ntiles, NA_TPB, 0, s>>>(residual, (int64_t)n, vec, qmax, (uint8_t *)out, scratch);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        fprintf(stderr, "[ERROR] falcom_quantize_residual_noalloc: launch failed: %s\n", cudaGetErrorString(e));
        return ERROR_COMPRESSION;
    }
    return ERROR_NONE;
}
