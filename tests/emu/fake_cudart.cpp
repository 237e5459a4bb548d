// fake_cudart.cpp -- the CUDA runtime calls the library makes, on host
// memory, for the kernel emulator (test infrastructure only).  "Device"
// memory is host memory filled with a poison pattern at allocation, every
// copy is a memmove, kernels run to completion at launch (so streams and
// events are no-ops), and CTAs run one at a time on a persistent pool of
// EMU_TPB host threads.
#include <cuda_runtime_api.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>

#include "emu.h"

thread_local EmuUint3 emu_tid;
EmuUint3 emu_bid, emu_gdim;
EmuCta *emu_cta;
uintptr_t emu_smem_base;

// Dynamic shared memory of the running CTA.  Shared-window handles are
// offsets from emu_smem_base, placed 2 GiB below this array so that every
// static of this library (the emulated __shared__ variables) is in reach.
#define EMU_DYN_FLOATS (64 * 1024)
alignas(128) float s_stage[EMU_DYN_FLOATS];

namespace {

std::map<uintptr_t, size_t> g_dev, g_host;
std::mutex g_mu;

bool inside(const std::map<uintptr_t, size_t> &m, const void *p) {
    const uintptr_t a = (uintptr_t)p;
    auto it = m.upper_bound(a);
    if (it == m.begin()) return false;
    --it;
    return a < it->first + (it->second ? it->second : 1);
}

void *poisoned_alloc(size_t n) {
    void *p = aligned_alloc(256, (n + 255) & ~(size_t)255);
    if (p) memset(p, 0xA5, n);   // device memory starts as garbage
    return p;
}

// Persistent pool: worker t runs thread t of every CTA.
struct Pool {
    std::mutex m;
    std::condition_variable start, done;
    unsigned long job = 0;
    int finished = 0;
    const std::function<void()> *fn = nullptr;

    Pool() {
        emu_cta = new EmuCta;
        for (int t = 0; t < EMU_TPB; t++) std::thread([this, t] { work(t); }).detach();
    }
    void work(int t) {
        emu_tid = {(unsigned)t, 0, 0};
        unsigned long seen = 0;
        for (;;) {
            const std::function<void()> *f;
            {
                std::unique_lock<std::mutex> lk(m);
                start.wait(lk, [&] { return job != seen; });
                seen = job;
                f = fn;
            }
            (*f)();
            std::lock_guard<std::mutex> lk(m);
            if (++finished == EMU_TPB) done.notify_one();
        }
    }
    void run_cta(const std::function<void()> &f) {
        std::unique_lock<std::mutex> lk(m);
        fn = &f;
        finished = 0;
        job++;
        start.notify_all();
        done.wait(lk, [&] { return finished == EMU_TPB; });
    }
};

Pool *pool() {
    static Pool *p = new Pool;   // never destroyed: the workers outlive static destructors
    return p;
}

std::mutex g_launch_mu;

}  // namespace

void emu_run(int grid, size_t dyn, const std::function<void()> &f) {
    if (dyn > sizeof(s_stage)) {
        fprintf(stderr, "emu: %zu bytes of dynamic shared memory requested, %zu emulated\n", dyn,
                sizeof(s_stage));
        abort();
    }
    std::lock_guard<std::mutex> lk(g_launch_mu);
    Pool *p = pool();
    emu_gdim = {(unsigned)grid, 1, 1};
    emu_cta->lo = s_stage;
    emu_cta->hi = s_stage + dyn / sizeof(float);
    for (int b = 0; b < grid; b++) {
        memset(s_stage, 0xCD, dyn);   // shared memory starts as garbage
        emu_bid = {(unsigned)b, 0, 0};
        p->run_cta(f);
    }
}

__attribute__((constructor)) static void emu_init_base() {
    const uintptr_t a = (uintptr_t)s_stage;
    emu_smem_base = a > (uintptr_t)1 << 31 ? a - ((uintptr_t)1 << 31) : 0;
}

extern "C" {

cudaError_t cudaMalloc(void **p, size_t n) {
    *p = poisoned_alloc(n);
    if (!*p) return cudaErrorMemoryAllocation;
    std::lock_guard<std::mutex> lk(g_mu);
    g_dev[(uintptr_t)*p] = n;
    return cudaSuccess;
}
cudaError_t cudaFree(void *p) {
    if (!p) return cudaSuccess;
    std::lock_guard<std::mutex> lk(g_mu);
    g_dev.erase((uintptr_t)p);
    free(p);
    return cudaSuccess;
}
cudaError_t cudaHostAlloc(void **p, size_t n, unsigned int) {
    *p = poisoned_alloc(n);
    if (!*p) return cudaErrorMemoryAllocation;
    std::lock_guard<std::mutex> lk(g_mu);
    g_host[(uintptr_t)*p] = n;
    return cudaSuccess;
}
cudaError_t cudaFreeHost(void *p) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_host.erase((uintptr_t)p);
    free(p);
    return cudaSuccess;
}
cudaError_t cudaPointerGetAttributes(cudaPointerAttributes *a, const void *p) {
    memset(a, 0, sizeof(*a));
    std::lock_guard<std::mutex> lk(g_mu);
    if (inside(g_dev, p)) {
        a->type = cudaMemoryTypeDevice;
        a->devicePointer = (void *)p;
    } else if (inside(g_host, p)) {
        a->type = cudaMemoryTypeHost;
        a->hostPointer = (void *)p;
        a->devicePointer = (void *)p;   // mapped at the same address (unified addressing)
    } else {
        a->type = cudaMemoryTypeUnregistered;
    }
    return cudaSuccess;
}
cudaError_t cudaMemcpy(void *d, const void *s, size_t n, cudaMemcpyKind) {
    memmove(d, s, n);
    return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void *d, const void *s, size_t n, cudaMemcpyKind, cudaStream_t) {
    memmove(d, s, n);
    return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void *d, int v, size_t n, cudaStream_t) {
    memset(d, v, n);
    return cudaSuccess;
}
cudaError_t cudaMemset(void *d, int v, size_t n) {
    memset(d, v, n);
    return cudaSuccess;
}
static std::atomic<int> g_handles;
cudaError_t cudaStreamCreateWithFlags(cudaStream_t *s, unsigned int) {
    *s = (cudaStream_t)(uintptr_t)(0x1000 + ++g_handles);
    return cudaSuccess;
}
cudaError_t cudaStreamDestroy(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t, unsigned int) { return cudaSuccess; }
cudaError_t cudaEventCreate(cudaEvent_t *e) {
    *e = (cudaEvent_t)(uintptr_t)(0x100000 + ++g_handles);
    return cudaSuccess;
}
cudaError_t cudaEventCreateWithFlags(cudaEvent_t *e, unsigned int) { return cudaEventCreate(e); }
cudaError_t cudaEventDestroy(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t) { return cudaSuccess; }
cudaError_t cudaEventSynchronize(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaEventElapsedTime(float *ms, cudaEvent_t, cudaEvent_t) {
    *ms = 0.0f;
    return cudaSuccess;
}
cudaError_t cudaSetDevice(int) { return cudaSuccess; }
cudaError_t cudaGetDevice(int *d) {
    *d = 0;
    return cudaSuccess;
}
cudaError_t cudaGetDeviceCount(int *n) {
    *n = 1;
    return cudaSuccess;
}
cudaError_t cudaDeviceSynchronize(void) { return cudaSuccess; }
cudaError_t cudaGetLastError(void) { return cudaSuccess; }
cudaError_t cudaPeekAtLastError(void) { return cudaSuccess; }
const char *cudaGetErrorString(cudaError_t) { return "emulated CUDA error"; }
cudaError_t cudaGetDeviceProperties_v2(cudaDeviceProp *p, int) {
    memset(p, 0, sizeof(*p));
    strcpy(p->name, "kernel emulator");
    p->multiProcessorCount = 148;
    return cudaSuccess;
}
cudaError_t cudaFuncSetAttribute(const void *, cudaFuncAttribute, int) { return cudaSuccess; }
cudaError_t cudaGetSymbolAddress(void **p, const void *symbol) {
    *p = (void *)symbol;
    return cudaSuccess;
}
cudaError_t cudaGetDriverEntryPoint(const char *, void **fp, unsigned long long,
                                    cudaDriverEntryPointQueryResult *q) {
    *fp = nullptr;
    if (q) *q = cudaDriverEntryPointSymbolNotFound;
    return cudaErrorUnknown;
}

}  // extern "C"

// Test hooks of the emulation library: "device" memory for arguments that
// the library checks to be device memory (the fused aggregate), and pinned
// "host" memory.
extern "C" __attribute__((visibility("default"))) void *emu_device_alloc(size_t n) {
    void *p = nullptr;
    return cudaMalloc(&p, n) == cudaSuccess ? p : nullptr;
}
extern "C" __attribute__((visibility("default"))) void emu_device_free(void *p) { cudaFree(p); }
extern "C" __attribute__((visibility("default"))) void *emu_host_alloc(size_t n) {
    void *p = nullptr;
    return cudaHostAlloc(&p, n, 0) == cudaSuccess ? p : nullptr;
}
extern "C" __attribute__((visibility("default"))) void emu_host_free(void *p) { cudaFreeHost(p); }
