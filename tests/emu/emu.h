// emu.h -- host emulation of the CUDA device features that
// compressor_b200/csrc/mc_kernels.cu uses, for CPU tests of the kernel
// source (tests/emu/build.py compiles a copy of the kernels against this
// header into a test-only library; the product library never uses it).
//
// Model: one CTA at a time; its 256 threads are a persistent pool of host
// threads; __syncthreads is a barrier over the pool; warp shuffles and
// ballots go through per-warp exchange slots and 32-thread barriers; bulk
// async copies are checked (16-byte alignment, inside the CTA's dynamic
// shared memory) and done as memcpy at issue, so an mbarrier wait always
// finds its phase complete; IEEE round-to-nearest float intrinsics map to the
// host's IEEE operations (the build disables contraction).  Shared-window
// addresses are 32-bit offsets from a base inside this library's own data,
// which holds every emulated shared variable.
#pragma once
#include <cuda_runtime.h>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>

#define EMU_TPB 256

struct EmuBarrier {
    std::mutex m;
    std::condition_variable cv;
    int n, count = 0;
    unsigned long gen = 0;
    int acc_and = 1, result = 1;
    explicit EmuBarrier(int n_) : n(n_) {}
    int wait(int v = 1) {
        std::unique_lock<std::mutex> lk(m);
        const unsigned long g = gen;
        acc_and &= (v != 0);
        if (++count == n) {
            result = acc_and;
            acc_and = 1;
            count = 0;
            gen++;
            cv.notify_all();
            return result;
        }
        cv.wait(lk, [&] { return gen != g; });
        return result;
    }
};

struct EmuUint3 {
    unsigned x, y, z;
};
extern thread_local EmuUint3 emu_tid;
extern EmuUint3 emu_bid, emu_gdim;
#define threadIdx emu_tid
#define blockIdx emu_bid
#define gridDim emu_gdim

struct EmuCta {
    EmuBarrier cta{EMU_TPB};
    EmuBarrier *warp[EMU_TPB / 32];
    unsigned long long slot[EMU_TPB];
    float *lo = nullptr, *hi = nullptr;   // dynamic shared memory of the running kernel
    EmuCta() {
        for (auto &w : warp) w = new EmuBarrier(32);
    }
    ~EmuCta() {
        for (auto &w : warp) delete w;
    }
};
extern EmuCta *emu_cta;

inline void __syncthreads() { emu_cta->cta.wait(); }
inline int __syncthreads_and(int v) { return emu_cta->cta.wait(v); }
inline void __syncwarp(unsigned = 0xffffffffu) { emu_cta->warp[threadIdx.x >> 5]->wait(); }
inline void __threadfence() { __atomic_thread_fence(__ATOMIC_SEQ_CST); }
inline void __threadfence_system() { __atomic_thread_fence(__ATOMIC_SEQ_CST); }
inline void __nanosleep(unsigned) { std::this_thread::yield(); }
// Callers vote only to skip work that each lane guards by its own predicate,
// so a per-lane answer gives the same result.
inline unsigned __activemask() { return 0xffffffffu; }
inline bool __any_sync(unsigned, bool p) { return p; }

template <class T>
inline T emu_shfl(T v, bool up, int arg) {
    static_assert(sizeof(T) <= 8, "shuffle of a value wider than 8 bytes");
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long bits = 0;
    memcpy(&bits, &v, sizeof(T));
    emu_cta->slot[threadIdx.x] = bits;
    emu_cta->warp[w]->wait();
    const int src = up ? (lane >= arg ? lane - arg : lane) : (lane ^ arg);
    const unsigned long long got = emu_cta->slot[(w << 5) + src];
    emu_cta->warp[w]->wait();
    T out;
    memcpy(&out, &got, sizeof(T));
    return out;
}
template <class T>
inline T __shfl_xor_sync(unsigned, T v, int o) { return emu_shfl(v, false, o); }
template <class T>
inline T __shfl_up_sync(unsigned, T v, int o) { return emu_shfl(v, true, o); }
inline unsigned __ballot_sync(unsigned, int p) {
    const int w = threadIdx.x >> 5;
    emu_cta->slot[threadIdx.x] = p ? 1 : 0;
    emu_cta->warp[w]->wait();
    unsigned m = 0;
    for (int j = 0; j < 32; j++) m |= (unsigned)(emu_cta->slot[(w << 5) + j] & 1) << j;
    emu_cta->warp[w]->wait();
    return m;
}
inline int __popc(unsigned x) { return __builtin_popcount(x); }
inline int __ffs(unsigned x) { return __builtin_ffs((int)x); }
inline int __ffs(int x) { return __builtin_ffs(x); }
inline unsigned __umulhi(unsigned a, unsigned b) { return (unsigned)(((unsigned long long)a * b) >> 32); }

template <class T>
inline T atomicAdd(T *p, T v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }
template <class T>
inline T atomicOr(T *p, T v) { return __atomic_fetch_or(p, v, __ATOMIC_SEQ_CST); }
template <class T>
inline T atomicExch(T *p, T v) { return __atomic_exchange_n(p, v, __ATOMIC_SEQ_CST); }
inline int atomicAdd(int *p, int32_t v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }

template <class T>
inline T __ldcg(const T *p) { return *(const volatile T *)p; }
inline float4 __ldcg(const float4 *p) {
    if (((uintptr_t)p) & 15) {
        fprintf(stderr, "emu: misaligned 16-byte load %p\n", (const void *)p);
        abort();
    }
    return *p;
}

template <class T>
inline T __ldcv(const T *p) { return __ldcg(p); }
template <class T>
inline T __ldcs(const T *p) {
    if (sizeof(T) == 16 && (((uintptr_t)p) & 15)) {
        fprintf(stderr, "emu: misaligned 16-byte load %p\n", (const void *)p);
        abort();
    }
    return *p;
}
template <class T>
inline void __stcs(T *p, T v) {
    if (sizeof(T) == 16 && (((uintptr_t)p) & 15)) {
        fprintf(stderr, "emu: misaligned 16-byte store %p\n", (void *)p);
        abort();
    }
    *p = v;
}

inline float __fmaf_rn(float a, float b, float c) { return fmaf(a, b, c); }
inline float __fmul_rn(float a, float b) { volatile float r = a * b; return r; }
inline float __fadd_rn(float a, float b) { volatile float r = a + b; return r; }
inline float __fsub_rn(float a, float b) { volatile float r = a - b; return r; }
inline float __fdiv_rn(float a, float b) { volatile float r = a / b; return r; }
inline float __fsqrt_rn(float a) { return sqrtf(a); }
inline double __fma_rn(double a, double b, double c) { return fma(a, b, c); }
inline double __ddiv_rn(double a, double b) { volatile double r = a / b; return r; }
inline float __double2float_rn(double a) { return (float)a; }
inline float __uint_as_float(unsigned u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
inline unsigned __float_as_uint(float f) {
    unsigned u;
    memcpy(&u, &f, 4);
    return u;
}

template <class A, class B>
inline auto min(A a, B b) -> decltype(a < b ? a : b) { return a < b ? a : b; }
template <class A, class B>
inline auto max(A a, B b) -> decltype(a < b ? a : b) { return a < b ? b : a; }

// 32-bit shared-window addresses: offsets from emu_smem_base
extern uintptr_t emu_smem_base;
inline uint32_t emu_smem_u32(const void *p) {
    const uintptr_t off = (uintptr_t)p - emu_smem_base;
    if ((uintptr_t)p < emu_smem_base || off >> 32) {
        fprintf(stderr, "emu: %p is outside the emulated shared window\n", p);
        abort();
    }
    return (uint32_t)off;
}
inline void *emu_smem_ptr(uint32_t a) { return (void *)(emu_smem_base + a); }

extern float s_stage[];
// Runs `grid` CTAs of the kernel body f one after another on the thread pool,
// with dyn_smem bytes of dynamic shared memory at s_stage.
void emu_run(int grid, size_t dyn_smem, const std::function<void()> &f);
