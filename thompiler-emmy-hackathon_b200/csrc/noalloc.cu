// An allocation-free f32 array sum: the variant of the two-pass grid
// reduction (grid-stride float4 stream, one partial per CTA, the last CTA to
// arrive folds the partials in CTA order) whose scratch is a file-scope
// device array instead of memory the caller or the runner allocates.
//
// Why: some callers cannot call cudaMalloc.  A framework that hands all
// device memory to its own caching allocator or to a pool sized at start-up
// has none left for a library to take, and cudaMalloc / cudaFree can block
// or synchronise the device on a latency-critical path.  Such a caller
// passes its input and output buffers, and this entry point takes nothing
// else: its scratch is `g_sum_scratch` below, which every GPU that loads the
// library holds (16,640 bytes) until the process exits.
//
// Set-up: the first call on each device (with that device current) asks the
// runtime for the device address of the array with cudaGetSymbolAddress and
// caches it with the current context's ID; in host code the array's name is
// only a host-side stand-in, so the kernel always receives the looked-up
// address.  A call that finds another context current (the first call after
// a cudaDeviceReset, which destroys the context and the module that held the
// array) looks the address up again.  Make the first call on a device, and
// the first after a reset, before any stream capture.
//
// Sharing: every call uses the same array and leaves its contents behind.
// The arrival counter, which must start at zero, is cleared on the stream
// before each launch; the partials are fully rewritten by each launch.
// Calls whose kernels overlap on the GPU (other streams, other threads)
// race on the array and give wrong sums: issue them in order on one stream.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/thompiler_runner.h"

extern "C" int thr_noalloc_set_error(const char *msg);

namespace {

constexpr unsigned kMaxCtas = THR_NOALLOC_MAX_CTAS;
constexpr unsigned kThreads = 256;
constexpr int kMaxDevices = 64;

struct SumScratch {
    float partials[kMaxCtas];   // one per CTA
    unsigned arrivals;          // CTAs that have stored their partial
    unsigned pad[63];
};

static __device__ __align__(256) SumScratch g_sum_scratch;

struct ScratchAddr {
    SumScratch *ptr = nullptr;
    unsigned long long ctx_id = 0;    // the context the address belongs to
};
ScratchAddr g_scratch[kMaxDevices];
std::mutex g_setup_mu;

typedef CUresult (*PFN_CtxGetCurrent)(CUcontext *);
typedef CUresult (*PFN_CtxGetId)(CUcontext, unsigned long long *);

// The current context's unique ID (0 when there is none or the driver lacks cuCtxGetId).
unsigned long long current_ctx_id() {
    static PFN_CtxGetCurrent get_current = nullptr;
    static PFN_CtxGetId get_id = nullptr;
    static bool looked = false;
    if (!looked) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_CtxGetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_CtxGetId>(f);
        looked = true;
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

__device__ __forceinline__ float block_sum(float v, float *slots) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) slots[warp] = v;
    __syncthreads();
    v = lane < (kThreads / 32) ? slots[lane] : 0.0f;
    for (int o = (kThreads / 64); o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return __shfl_sync(0xffffffffu, v, 0);
}

__global__ void __launch_bounds__(kThreads)
sum_f32_noalloc_kernel(const float *__restrict__ x, unsigned long long n, float *out, SumScratch *s) {
    __shared__ float slots[kThreads / 32];
    __shared__ unsigned is_last;
    const unsigned long long chunks = n / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    const unsigned long long stride = (unsigned long long)gridDim.x * kThreads;
    float acc = 0.0f;
    unsigned long long c = (unsigned long long)blockIdx.x * kThreads + threadIdx.x;
    for (; c + 3 * stride < chunks; c += 4 * stride) {
        float4 a = __ldg(x4 + c), b = __ldg(x4 + c + stride), d = __ldg(x4 + c + 2 * stride),
               e = __ldg(x4 + c + 3 * stride);
        acc += (a.x + a.y) + (a.z + a.w);
        acc += (b.x + b.y) + (b.z + b.w);
        acc += (d.x + d.y) + (d.z + d.w);
        acc += (e.x + e.y) + (e.z + e.w);
    }
    for (; c < chunks; c += stride) {
        float4 a = __ldg(x4 + c);
        acc += (a.x + a.y) + (a.z + a.w);
    }
    if (blockIdx.x == 0)  // the n % 4 tail elements
        for (unsigned long long i = chunks * 4 + threadIdx.x; i < n; i += kThreads) acc += x[i];
    float total = block_sum(acc, slots);
    if (threadIdx.x == 0) {
        s->partials[blockIdx.x] = total;
        __threadfence();
        unsigned prev = atomicAdd(&s->arrivals, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    __syncthreads();   // the block_sum slots are reused below
    float v = 0.0f;
    for (unsigned i = threadIdx.x; i < gridDim.x; i += kThreads)
        v += __ldcg(&s->partials[i]);
    v = block_sum(v, slots);
    if (threadIdx.x == 0) {
        out[0] = v;
        s->arrivals = 0;
    }
}

}  // namespace

extern "C" int thr_sum_f32_noalloc(uint64_t x, uint64_t n, uint64_t out, uint32_t ctas, uint64_t stream) {
    if (ctas > kMaxCtas) {
        char msg[160];
        snprintf(msg, sizeof msg, "thr_sum_f32_noalloc: %u CTAs asked, the static scratch holds at most %u",
                 ctas, kMaxCtas);
        thr_noalloc_set_error(msg);
        return THR_ERR_REQUEST;
    }
    if (!x || !out || (x & 15) || (out & 3)) {
        thr_noalloc_set_error(
            "thr_sum_f32_noalloc: x and out must be device pointers, x 16-byte and out 4-byte aligned");
        return THR_ERR_REQUEST;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        thr_noalloc_set_error("thr_sum_f32_noalloc: no usable current device");
        return THR_ERR_CUDA;
    }
    SumScratch *s = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_setup_mu);
        ScratchAddr &a = g_scratch[dev];
        unsigned long long ctx = current_ctx_id();
        if (!a.ptr || !ctx || ctx != a.ctx_id) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_sum_scratch);
            if (e != cudaSuccess || !p) {
                std::string m = std::string("thr_sum_f32_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
                thr_noalloc_set_error(m.c_str());
                return THR_ERR_CUDA;
            }
            a.ptr = static_cast<SumScratch *>(p);
            a.ctx_id = current_ctx_id();      // the lookup made the device's context current
        }
        s = a.ptr;
    }
    if (ctas == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        ctas = (unsigned)sms * 4u;
        unsigned long long need = (n / 4 + kThreads * 4 - 1) / (kThreads * 4);
        if (need < ctas) ctas = need ? (unsigned)need : 1u;
        if (ctas > kMaxCtas) ctas = kMaxCtas;
    }
    cudaStream_t st = (cudaStream_t)(uintptr_t)stream;
    e = cudaMemsetAsync(&s->arrivals, 0, sizeof(unsigned), st);
    if (e == cudaSuccess) {
        sum_f32_noalloc_kernel<<<ctas, kThreads, 0, st>>>(reinterpret_cast<const float *>(x), n,
                                                          reinterpret_cast<float *>(out), s);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        std::string m = std::string("thr_sum_f32_noalloc: launch failed: ") + cudaGetErrorString(e);
        thr_noalloc_set_error(m.c_str());
        return THR_ERR_RUN;
    }
    return THR_OK;
}
