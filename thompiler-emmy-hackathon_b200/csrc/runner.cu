// thompiler runner: loads compile.py's PTX with the CUDA driver's JIT and
// launches it (the C ABI of include/thompiler_runner.h).
//
// The library links the CUDA runtime statically and reaches the driver API
// through cudaGetDriverEntryPointByVersion, so it loads on a machine
// without a GPU driver (the build host) and only needs libcuda at thr_init.
// The kernels it runs are PTX text from the compiler; the one kernel it
// holds itself is the allocation-free sum (noalloc.cu).

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <deque>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/thompiler_runner.h"

namespace {

thread_local std::string g_err;

int fail(int status, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(THR_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ---- driver entry points ------------------------------------------------

typedef CUresult (*PFN_LoadDataEx)(CUmodule *, const void *, unsigned, CUjit_option *, void **);
typedef CUresult (*PFN_Unload)(CUmodule);
typedef CUresult (*PFN_GetFunction)(CUfunction *, CUmodule, const char *);
typedef CUresult (*PFN_GetGlobal)(CUdeviceptr *, size_t *, CUmodule, const char *);
typedef CUresult (*PFN_FuncGetAttribute)(int *, CUfunction_attribute, CUfunction);
typedef CUresult (*PFN_FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
typedef CUresult (*PFN_LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                                     unsigned, unsigned, CUstream, void **, void **);
typedef CUresult (*PFN_LaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **, void **);
typedef CUresult (*PFN_TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                             const cuuint64_t *, const cuuint64_t *,
                                             const cuuint32_t *, const cuuint32_t *,
                                             CUtensorMapInterleave, CUtensorMapSwizzle,
                                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
typedef CUresult (*PFN_GetErrorString)(CUresult, const char **);

struct Driver {
    bool ok = false;
    PFN_LoadDataEx load = nullptr;
    PFN_Unload unload = nullptr;
    PFN_GetFunction get_function = nullptr;
    PFN_GetGlobal get_global = nullptr;
    PFN_FuncGetAttribute func_get = nullptr;
    PFN_FuncSetAttribute func_set = nullptr;
    PFN_LaunchKernel launch = nullptr;
    PFN_LaunchKernelEx launch_ex = nullptr;
    PFN_TensorMapEncodeTiled tmap = nullptr;
    PFN_GetErrorString err_string = nullptr;
};

Driver g_drv;
std::mutex g_mu;

template <typename T>
bool entry(const char *name, T *out) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) return false;
    *out = reinterpret_cast<T>(fn);
    return true;
}

const char *cu_name(CUresult r) {
    const char *s = nullptr;
    if (g_drv.err_string && g_drv.err_string(r, &s) == CUDA_SUCCESS && s) return s;
    return "unknown CUDA driver error";
}

int drv_fail(CUresult r, const char *what) {
    return fail(r == CUDA_ERROR_NOT_FOUND ? THR_ERR_LOOKUP : THR_ERR_CUDA, "%s: %s (CUresult %d)",
                what, cu_name(r), (int)r);
}

int ensure_driver() {
    if (g_drv.ok) return THR_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_drv.ok) return THR_OK;
    cudaError_t e = cudaFree(nullptr);  // creates / binds the primary context
    if (e != cudaSuccess) return cuda_fail(e, "CUDA runtime initialisation");
    Driver d;
    bool all = entry("cuModuleLoadDataEx", &d.load) && entry("cuModuleUnload", &d.unload) &&
               entry("cuModuleGetFunction", &d.get_function) &&
               entry("cuModuleGetGlobal", &d.get_global) &&
               entry("cuFuncGetAttribute", &d.func_get) && entry("cuFuncSetAttribute", &d.func_set) &&
               entry("cuLaunchKernel", &d.launch) && entry("cuGetErrorString", &d.err_string);
    entry("cuTensorMapEncodeTiled", &d.tmap);  // optional: only TMA kernels need it
    entry("cuLaunchKernelEx", &d.launch_ex);   // optional: launches that overlap the previous kernel
    if (!all) return fail(THR_ERR_CUDA, "the CUDA driver does not export the required entry points");
    d.ok = true;
    g_drv = d;
    return THR_OK;
}

// ---- the runner's device buffers -----------------------------------------

struct Slot {
    void *ptr = nullptr;
    uint64_t cap = 0;
};
std::vector<Slot> g_slots;

int slot_buffer(size_t i, uint64_t nbytes, void **out) {
    if (g_slots.size() <= i) g_slots.resize(i + 1);
    Slot &s = g_slots[i];
    if (s.cap < nbytes || s.ptr == nullptr) {
        if (s.ptr) cudaFree(s.ptr);
        s.ptr = nullptr;
        s.cap = 0;
        uint64_t want = std::max<uint64_t>(nbytes, 256);
        cudaError_t e = cudaMalloc(&s.ptr, want);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc of a run buffer");
        s.cap = want;
    }
    *out = s.ptr;
    return THR_OK;
}

// thr_run_batch's copy-in, compute and copy-out streams and its events, per device, created on
// first use and kept (a serving loop calls the batch repeatedly); every batch waits for all of its
// work before returning, so the next one can reuse them
struct BatchRes {
    cudaStream_t s[3] = {nullptr, nullptr, nullptr};
    std::vector<cudaEvent_t> events;
};
std::vector<BatchRes> g_batch;

int batch_resources(BatchRes **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if ((int)g_batch.size() <= dev) g_batch.resize(dev + 1);
    BatchRes &b = g_batch[dev];
    for (auto &st : b.s)
        if (!st && (e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_fail(e, "thr_run_batch: creating streams");
    *out = &b;
    return THR_OK;
}

int batch_event(BatchRes &b, size_t i, cudaEvent_t *ev) {
    while (b.events.size() <= i) {
        cudaEvent_t e = nullptr;
        cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        if (r != cudaSuccess) return cuda_fail(r, "cudaEventCreate");
        b.events.push_back(e);
    }
    *ev = b.events[i];
    return THR_OK;
}

void release_batch_resources() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || (int)g_batch.size() <= dev) return;
    BatchRes &b = g_batch[dev];
    for (auto &st : b.s)
        if (st) {
            cudaStreamSynchronize(st);
            cudaStreamDestroy(st);
            st = nullptr;
        }
    for (auto e : b.events) cudaEventDestroy(e);
    b.events.clear();
}

// ---- tensor-map sets ------------------------------------------------------------
//
// A tuned module reads its tensor maps from module globals.  Those laid out as a ring -- every map
// spec naming one global of `sets` x `ntmaps` maps of 128 bytes, and a pointer table of `sets` x
// `ntmaps` buffer addresses -- hold several sets at once: the kernel uses the set whose recorded
// addresses equal its parameters, so launches of one module on different buffers can be in flight
// together (on several streams, or one thr_run_batch).  Per module the runner keeps, for each set,
// the addresses it is encoded for, an event after the last launch that read it and an event after
// its last upload.  A launch binds the set already encoded for its buffers, else re-encodes the
// least recently used one: the upload, from the set's own pinned staging, waits on the stream for
// the set's last reader.  A set read by a launch captured into a CUDA graph is never re-encoded
// (the graph may replay at any time), and a capture only binds sets uploaded before it: the
// capturing stream makes no event queries or uploads (both would invalidate a global-mode
// capture), so an upload's completion is also published to the host by a host function.  Maps
// in separate globals (one per spec) form one set.

struct TmapSet {
    std::vector<uint64_t> ptrs;           // the buffers this set is encoded for; empty: unused
    uint64_t stamp = 0;                   // last use (least recently used is re-encoded first)
    cudaEvent_t read = nullptr;           // after the last launch that read the set
    bool read_pending = false;
    cudaEvent_t uploaded = nullptr;       // after the set's last upload
    bool upload_pending = false;
    unsigned char *staging = nullptr;     // pinned host copy of the maps, then the addresses
    std::atomic<int> *upload_done = nullptr;  // set by a host function once the last upload ran
    bool pinned = false;                  // read by a captured launch
};

std::deque<std::atomic<int>> g_upload_flags;  // never freed: a host function may still write one

void CUDART_CB mark_uploaded(void *flag) { static_cast<std::atomic<int> *>(flag)->store(1); }

struct TmapRing {
    int sets = 0, nmaps = 0;
    bool ring = false;                    // one global of sets x nmaps maps (else one global per map)
    std::vector<uint64_t> globals;        // per map (ring: the ring global, repeated)
    uint64_t table = 0;                   // the pointer table, 0 if none
    uint64_t clock = 0;
    std::vector<TmapSet> s;
};

std::map<uint64_t, TmapRing> g_rings;     // by module handle
std::mutex g_ring_mu;

bool stream_capturing(cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
}

int ring_of(uint64_t module, const thr_tmap_spec *tmaps, int ntmaps, const char *ptr_table, TmapRing **out) {
    auto it = g_rings.find(module);
    if (it != g_rings.end()) {
        if (it->second.nmaps != ntmaps) return fail(THR_ERR_REQUEST, "tensor maps: %d specs for a module of %d",
                                                    ntmaps, it->second.nmaps);
        *out = &it->second;
        return THR_OK;
    }
    TmapRing r;
    r.nmaps = ntmaps;
    bool one = true;
    for (int i = 1; i < ntmaps; ++i) one = one && !strcmp(tmaps[i].global, tmaps[0].global);
    uint64_t g = 0, n = 0;
    int s;
    // every spec naming one global: a ring of sets x ntmaps maps (one set fits exactly)
    r.ring = one && ntmaps > 0;
    if (r.ring) {
        if ((s = thr_module_global(module, tmaps[0].global, &g, &n))) return s;
        r.sets = (int)(n / (128 * (uint64_t)ntmaps));
        if (r.sets < 1)
            return fail(THR_ERR_LOOKUP, "tensor-map global %s holds %llu bytes, %d maps need %d", tmaps[0].global,
                        (unsigned long long)n, ntmaps, 128 * ntmaps);
        r.globals.assign(ntmaps, g);
    } else {
        r.sets = 1;
        for (int i = 0; i < ntmaps; ++i) {
            for (int j = 0; j < i; ++j)
                if (!strcmp(tmaps[i].global, tmaps[j].global))
                    return fail(THR_ERR_REQUEST, "tensor maps %d and %d share the global %s", j, i, tmaps[i].global);
            if ((s = thr_module_global(module, tmaps[i].global, &g, &n))) return s;
            if (n < 128) return fail(THR_ERR_LOOKUP, "tensor-map global %s is %llu bytes", tmaps[i].global,
                                     (unsigned long long)n);
            r.globals.push_back(g);
        }
    }
    if (ptr_table) {
        if ((s = thr_module_global(module, ptr_table, &g, &n))) return s;
        if (n < 8 * (uint64_t)ntmaps * r.sets)
            return fail(THR_ERR_LOOKUP, "pointer table %s holds %llu bytes, %d sets of %d maps need %d", ptr_table,
                        (unsigned long long)n, r.sets, ntmaps, 8 * ntmaps * r.sets);
        r.table = g;
    }
    r.s.resize(r.sets);
    *out = &g_rings.emplace(module, std::move(r)).first->second;
    return THR_OK;
}

// Make the set encoded for the mapped buffers (args[tmaps[i].arg]) current for a launch on `st`.
int tmap_bind(uint64_t module, const thr_tmap_spec *tmaps, int ntmaps, const char *ptr_table,
              const uint64_t *args, int nargs, cudaStream_t st, int *set_out) {
    std::lock_guard<std::mutex> lk(g_ring_mu);
    TmapRing *r = nullptr;
    int s = ring_of(module, tmaps, ntmaps, ptr_table, &r);
    if (s) return s;
    std::vector<uint64_t> want(ntmaps);
    for (int i = 0; i < ntmaps; ++i) {
        if (tmaps[i].arg < 0 || tmaps[i].arg >= nargs) return fail(THR_ERR_REQUEST, "tensor map %d: bad argument", i);
        want[i] = args[tmaps[i].arg];
    }
    bool capturing = stream_capturing(st);
    auto settle = [&](cudaEvent_t ev, bool &pending, const char *what) -> int {
        // order `st` after ev (not capturing)
        if (!pending) return THR_OK;
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) {
            pending = false;
            return THR_OK;
        }
        if (q != cudaErrorNotReady) return cuda_fail(q, what);
        cudaError_t e = cudaStreamWaitEvent(st, ev, 0);
        return e == cudaSuccess ? THR_OK : cuda_fail(e, what);
    };
    for (int k = 0; k < r->sets; ++k) {
        TmapSet &t = r->s[k];
        if (t.ptrs == want) {
            if (!capturing) {
                if ((s = settle(t.uploaded, t.upload_pending, "the set's upload"))) return s;
            } else if (t.upload_pending) {
                if (!t.upload_done || !t.upload_done->load())
                    return fail(THR_ERR_REQUEST, "tensor maps: the set for these buffers is still being uploaded "
                                                 "while the stream is captured (synchronise before capturing)");
                t.upload_pending = false;
            }
            t.stamp = ++r->clock;
            *set_out = k;
            return THR_OK;
        }
    }
    if (capturing)
        return fail(THR_ERR_REQUEST, "tensor maps: no set of the module is encoded for these buffers, and a "
                                     "captured stream cannot upload one (launch on them once before capturing)");
    // A kernel picks the lowest set whose addresses equal its parameters, reading the table while
    // another stream may rewrite a set.  A launch in flight on buffers T could then match a set
    // caught half-way from its old addresses O to the new ones N if every T[i] is O[i] or N[i]:
    // such a set is not re-encoded while that launch may run.
    auto in_flight = [&](TmapSet &o) -> bool {
        if (!o.read_pending) return false;
        cudaError_t q = cudaEventQuery(o.read);
        if (q == cudaSuccess) o.read_pending = false;
        return o.read_pending || o.pinned;
    };
    auto confusable = [&](int v) -> int {         // a set in flight that v's rewrite could alias, or -1
        const std::vector<uint64_t> &old_ = r->s[v].ptrs;
        if (old_.empty()) return -1;
        for (int k = 0; k < r->sets; ++k) {
            TmapSet &o = r->s[k];
            if (k == v || o.ptrs.empty() || !in_flight(o)) continue;
            bool mix = true;
            for (int i = 0; i < ntmaps && mix; ++i) mix = o.ptrs[i] == old_[i] || o.ptrs[i] == want[i];
            if (mix) return k;
        }
        return -1;
    };
    int victim = -1;
    for (int k = 0; k < r->sets; ++k)
        if (!r->s[k].pinned && confusable(k) < 0 && (victim < 0 || r->s[k].stamp < r->s[victim].stamp)) victim = k;
    if (victim < 0) {                             // every free set could be aliased: wait for the reader
        for (int k = 0; k < r->sets; ++k)
            if (!r->s[k].pinned && (victim < 0 || r->s[k].stamp < r->s[victim].stamp)) victim = k;
        if (victim < 0)
            return fail(THR_ERR_REQUEST, "tensor maps: all %d sets of the module are read by captured graphs", r->sets);
        for (int c; (c = confusable(victim)) >= 0;) {
            if (r->s[c].pinned)
                return fail(THR_ERR_REQUEST, "tensor maps: re-encoding a set could alias one a captured graph reads");
            cudaError_t e = cudaEventSynchronize(r->s[c].read);
            if (e != cudaSuccess) return cuda_fail(e, "waiting for a tensor-map reader");
            r->s[c].read_pending = false;
        }
    }
    TmapSet &t = r->s[victim];
    if ((s = settle(t.read, t.read_pending, "the set's last reader"))) return s;
    cudaError_t e;
    if (t.upload_pending) {                 // its staging is rewritten below
        if ((e = cudaEventSynchronize(t.uploaded)) != cudaSuccess) return cuda_fail(e, "tensor-map staging");
        t.upload_pending = false;
    }
    size_t mbytes = 128 * (size_t)ntmaps, pbytes = 8 * (size_t)ntmaps;
    if (!t.staging && (e = cudaHostAlloc((void **)&t.staging, mbytes + pbytes, cudaHostAllocDefault)) != cudaSuccess)
        return cuda_fail(e, "tensor-map staging");
    for (int i = 0; i < ntmaps; ++i) {
        const thr_tmap_spec &m = tmaps[i];
        if ((s = thr_tensor_map(t.staging + 128 * i, m.dtype_code, m.rank, want[i], m.dims, m.strides, m.box,
                                m.swizzle)))
            return s;
    }
    memcpy(t.staging + mbytes, want.data(), pbytes);
    if (!t.uploaded && (e = cudaEventCreateWithFlags(&t.uploaded, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "cudaEventCreate");
    if (r->ring) {
        e = cudaMemcpyAsync((void *)(uintptr_t)(r->globals[0] + victim * mbytes), t.staging, mbytes,
                            cudaMemcpyHostToDevice, st);
    } else {
        e = cudaSuccess;
        for (int i = 0; i < ntmaps && e == cudaSuccess; ++i)
            e = cudaMemcpyAsync((void *)(uintptr_t)r->globals[i], t.staging + 128 * i, 128, cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess && r->table)
        e = cudaMemcpyAsync((void *)(uintptr_t)(r->table + victim * pbytes), t.staging + mbytes, pbytes,
                            cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaEventRecord(t.uploaded, st);
    if (e == cudaSuccess) {
        if (!t.upload_done) t.upload_done = &g_upload_flags.emplace_back(0);
        t.upload_done->store(0);
        e = cudaLaunchHostFunc(st, mark_uploaded, t.upload_done);
    }
    if (e != cudaSuccess) {
        t.ptrs.clear();
        return cuda_fail(e, "uploading tensor maps");
    }
    t.upload_pending = true;
    t.ptrs = want;
    t.stamp = ++r->clock;
    *set_out = victim;
    return THR_OK;
}

// A launch that reads set `k` was just issued on `st`.
int tmap_launched(uint64_t module, int k, cudaStream_t st) {
    std::lock_guard<std::mutex> lk(g_ring_mu);
    auto it = g_rings.find(module);
    if (it == g_rings.end() || k < 0 || k >= it->second.sets) return fail(THR_ERR_REQUEST, "tensor maps: set %d", k);
    TmapSet &t = it->second.s[k];
    if (stream_capturing(st)) {
        t.pinned = true;
        return THR_OK;
    }
    cudaError_t e;
    if (!t.read && (e = cudaEventCreateWithFlags(&t.read, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "cudaEventCreate");
    if ((e = cudaEventRecord(t.read, st)) != cudaSuccess) return cuda_fail(e, "recording a tensor-map reader");
    t.read_pending = true;
    return THR_OK;
}

void drop_ring(uint64_t module) {
    std::lock_guard<std::mutex> lk(g_ring_mu);
    auto it = g_rings.find(module);
    if (it == g_rings.end()) return;
    for (TmapSet &t : it->second.s) {
        if (t.uploaded) {
            cudaEventSynchronize(t.uploaded);
            cudaEventDestroy(t.uploaded);
        }
        if (t.read) cudaEventDestroy(t.read);
        if (t.staging) cudaFreeHost(t.staging);
    }
    g_rings.erase(it);
}

// Wait for `ev` at most timeout_s seconds.  A request's work often ends within a millisecond
// (a few MiB over PCIe and a short kernel), so the first 2 ms poll back to back (yielding the
// core), then every 20 us, and after 50 ms every 200 us: the answer is seen a few microseconds
// after the work ends instead of up to one sleep later.
int wait_event(cudaEvent_t ev, double timeout_s) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return THR_OK;
        if (e != cudaErrorNotReady) return fail(THR_ERR_RUN, "launch failed: %s", cudaGetErrorString(e));
        double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (timeout_s > 0 && el > timeout_s)
            return fail(THR_ERR_TIMEOUT, "the launch did not finish within %.1f s", timeout_s);
        if (el < 2e-3)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(el < 0.05 ? 20 : 200));
    }
}

}  // namespace

extern "C" {

int thr_version(void) { return 2; }

int thr_init(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(THR_ERR_REQUEST, "device %d of %d", device, n);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    return ensure_driver();
}

int thr_device_info(int device, int *sm_count, int *cc_major, int *cc_minor, char *name, size_t name_len) {
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    if (name && name_len) {
        strncpy(name, p.name, name_len - 1);
        name[name_len - 1] = 0;
    }
    return THR_OK;
}

int thr_module_load(const char *ptx, uint64_t *module, char *log, size_t log_len) {
    if (!ptx || !module) return fail(THR_ERR_REQUEST, "thr_module_load: null argument");
    int s = ensure_driver();
    if (s) return s;
    std::vector<char> info(16384, 0), error(16384, 0);
    CUjit_option opts[5] = {CU_JIT_INFO_LOG_BUFFER, CU_JIT_INFO_LOG_BUFFER_SIZE_BYTES,
                            CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES,
                            CU_JIT_LOG_VERBOSE};
    void *vals[5] = {info.data(), (void *)(uintptr_t)info.size(), error.data(),
                     (void *)(uintptr_t)error.size(), (void *)(uintptr_t)1};
    CUmodule m = nullptr;
    CUresult r = g_drv.load(&m, ptx, 5, opts, vals);
    if (log && log_len) {
        strncpy(log, info.data(), log_len - 1);
        log[log_len - 1] = 0;
    }
    if (r != CUDA_SUCCESS)
        return fail(THR_ERR_PTXAS, "PTX JIT failed (%s): %s", cu_name(r), error.data());
    *module = (uint64_t)(uintptr_t)m;
    return THR_OK;
}

int thr_module_unload(uint64_t module) {
    int s = ensure_driver();
    if (s) return s;
    drop_ring(module);
    CUresult r = g_drv.unload((CUmodule)(uintptr_t)module);
    return r == CUDA_SUCCESS ? THR_OK : drv_fail(r, "cuModuleUnload");
}

int thr_get_function(uint64_t module, const char *entry_name, uint64_t *function) {
    int s = ensure_driver();
    if (s) return s;
    CUfunction f = nullptr;
    CUresult r = g_drv.get_function(&f, (CUmodule)(uintptr_t)module, entry_name);
    if (r != CUDA_SUCCESS) return fail(THR_ERR_LOOKUP, "no entry %s in the module (%s)", entry_name, cu_name(r));
    *function = (uint64_t)(uintptr_t)f;
    return THR_OK;
}

int thr_function_attrs(uint64_t function, int *num_regs, int *max_threads, int *static_smem, int *local_bytes) {
    int s = ensure_driver();
    if (s) return s;
    CUfunction f = (CUfunction)(uintptr_t)function;
    int v = 0;
    if (num_regs && g_drv.func_get(&v, CU_FUNC_ATTRIBUTE_NUM_REGS, f) == CUDA_SUCCESS) *num_regs = v;
    if (max_threads && g_drv.func_get(&v, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, f) == CUDA_SUCCESS) *max_threads = v;
    if (static_smem && g_drv.func_get(&v, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, f) == CUDA_SUCCESS) *static_smem = v;
    if (local_bytes && g_drv.func_get(&v, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f) == CUDA_SUCCESS) *local_bytes = v;
    return THR_OK;
}

int thr_module_global(uint64_t module, const char *name, uint64_t *dptr, uint64_t *nbytes) {
    int s = ensure_driver();
    if (s) return s;
    CUdeviceptr p = 0;
    size_t n = 0;
    CUresult r = g_drv.get_global(&p, &n, (CUmodule)(uintptr_t)module, name);
    if (r != CUDA_SUCCESS) return fail(THR_ERR_LOOKUP, "no global %s in the module (%s)", name, cu_name(r));
    if (dptr) *dptr = (uint64_t)p;
    if (nbytes) *nbytes = (uint64_t)n;
    return THR_OK;
}

int thr_launch(uint64_t function, const uint32_t grid[3], const uint32_t block[3], uint32_t smem_bytes,
               const uint64_t *args, int nargs, uint64_t stream) {
    return thr_launch_ex(function, grid, block, smem_bytes, args, nargs, stream, 0);
}

int thr_launch_ex(uint64_t function, const uint32_t grid[3], const uint32_t block[3], uint32_t smem_bytes,
                  const uint64_t *args, int nargs, uint64_t stream, uint32_t flags) {
    int s = ensure_driver();
    if (s) return s;
    if (!grid || !block || nargs < 0 || (nargs > 0 && !args) || (flags & ~THR_LAUNCH_OVERLAP_PREVIOUS))
        return fail(THR_ERR_REQUEST, "thr_launch: bad arguments");
    CUfunction f = (CUfunction)(uintptr_t)function;
    if (smem_bytes > 48 * 1024) {
        CUresult r = g_drv.func_set(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem_bytes);
        if (r != CUDA_SUCCESS) return drv_fail(r, "raising the dynamic shared memory limit");
    }
    std::vector<uint64_t> vals(args, args + nargs);
    std::vector<void *> params(nargs);
    for (int i = 0; i < nargs; ++i) params[i] = &vals[i];
    if ((flags & THR_LAUNCH_OVERLAP_PREVIOUS) && g_drv.launch_ex) {
        // programmatic stream serialisation: the launch may begin while the stream's previous
        // kernel is still running (once that kernel's CTAs signal griddepcontrol.launch_dependents);
        // the kernel itself waits (griddepcontrol.wait) before it touches global data
        CUlaunchAttribute attr;
        memset(&attr, 0, sizeof attr);
        attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attr.value.programmaticStreamSerializationAllowed = 1;
        CUlaunchConfig cfg;
        memset(&cfg, 0, sizeof cfg);
        cfg.gridDimX = grid[0];
        cfg.gridDimY = grid[1];
        cfg.gridDimZ = grid[2];
        cfg.blockDimX = block[0];
        cfg.blockDimY = block[1];
        cfg.blockDimZ = block[2];
        cfg.sharedMemBytes = smem_bytes;
        cfg.hStream = (CUstream)(uintptr_t)stream;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        CUresult r = g_drv.launch_ex(&cfg, f, nargs ? params.data() : nullptr, nullptr);
        return r == CUDA_SUCCESS ? THR_OK : fail(THR_ERR_RUN, "cuLaunchKernelEx: %s", cu_name(r));
    }
    CUresult r = g_drv.launch(f, grid[0], grid[1], grid[2], block[0], block[1], block[2], smem_bytes,
                              (CUstream)(uintptr_t)stream, nargs ? params.data() : nullptr, nullptr);
    return r == CUDA_SUCCESS ? THR_OK : fail(THR_ERR_RUN, "cuLaunchKernel: %s", cu_name(r));
}

int thr_run(uint64_t function, const uint32_t grid[3], const uint32_t block[3], uint32_t smem_bytes,
            const thr_arg *args, int nargs, int warmup, int iters, double timeout_s, float *median_us,
            uint64_t stream) {
    return thr_run_ex(0, function, grid, block, smem_bytes, args, nargs, nullptr, 0, nullptr, warmup, iters,
                      timeout_s, median_us, stream);
}

int thr_run_ex(uint64_t module, uint64_t function, const uint32_t grid[3], const uint32_t block[3],
               uint32_t smem_bytes, const thr_arg *args, int nargs, const thr_tmap_spec *tmaps, int ntmaps,
               const char *ptr_table, int warmup, int iters, double timeout_s, float *median_us,
               uint64_t stream) {
    int s = ensure_driver();
    if (s) return s;
    if (nargs < 0 || (nargs && !args) || warmup < 0 || iters < 0 || ntmaps < 0 || (ntmaps && (!tmaps || !module)))
        return fail(THR_ERR_REQUEST, "thr_run: bad arguments");
    cudaStream_t st = (cudaStream_t)(uintptr_t)stream;
    std::vector<uint64_t> dev(nargs);
    for (int i = 0; i < nargs; ++i) {
        void *p = nullptr;
        if ((s = slot_buffer(i, args[i].nbytes, &p))) return s;
        dev[i] = (uint64_t)(uintptr_t)p;
        cudaError_t e = args[i].kind == THR_ARG_INPUT
                            ? cudaMemcpyAsync(p, args[i].host, args[i].nbytes, cudaMemcpyHostToDevice, st)
                            : cudaMemsetAsync(p, 0, args[i].nbytes, st);
        if (e != cudaSuccess) return cuda_fail(e, "staging a run argument");
    }
    int set = -1;
    if (ntmaps && (s = tmap_bind(module, tmaps, ntmaps, ptr_table, dev.data(), nargs, st, &set))) return s;
    auto rezero = [&]() -> int {
        for (int i = 0; i < nargs; ++i)
            if (args[i].zero_each) {
                cudaError_t e = cudaMemsetAsync((void *)(uintptr_t)dev[i], 0, args[i].nbytes, st);
                if (e != cudaSuccess) return cuda_fail(e, "zeroing an output");
            }
        return THR_OK;
    };
    int total = warmup + std::max(iters, 1);
    std::vector<cudaEvent_t> ev(2 * total, nullptr);
    for (auto &e : ev)
        if (cudaEventCreate(&e) != cudaSuccess) return fail(THR_ERR_CUDA, "cudaEventCreate");
    int rc = THR_OK;
    for (int k = 0; k < total && rc == THR_OK; ++k) {
        if ((rc = rezero())) break;
        cudaEventRecord(ev[2 * k], st);
        rc = thr_launch(function, grid, block, smem_bytes, dev.data(), nargs, stream);
        if (rc == THR_OK && ntmaps) rc = tmap_launched(module, set, st);
        cudaEventRecord(ev[2 * k + 1], st);
    }
    if (rc == THR_OK) rc = wait_event(ev[2 * total - 1], timeout_s);
    if (rc == THR_OK) {
        std::vector<float> t;
        for (int k = warmup; k < total; ++k) {
            float ms = 0;
            cudaEventElapsedTime(&ms, ev[2 * k], ev[2 * k + 1]);
            t.push_back(ms * 1000.0f);
        }
        std::sort(t.begin(), t.end());
        if (median_us) *median_us = t.empty() ? 0.0f : t[t.size() / 2];
        for (int i = 0; i < nargs && rc == THR_OK; ++i)
            if (args[i].kind == THR_ARG_OUTPUT) {
                cudaError_t e = cudaMemcpyAsync(args[i].host, (void *)(uintptr_t)dev[i], args[i].nbytes,
                                                cudaMemcpyDeviceToHost, st);
                if (e != cudaSuccess) rc = cuda_fail(e, "copying an output back");
            }
        if (rc == THR_OK) {
            cudaError_t e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) rc = fail(THR_ERR_RUN, "run failed: %s", cudaGetErrorString(e));
        }
    }
    for (auto &e : ev) cudaEventDestroy(e);  // deferred by CUDA if still pending
    return rc;
}

int thr_run_batch(const thr_run_desc *runs, int nruns, double timeout_s) {
    int s = ensure_driver();
    if (s) return s;
    if (nruns < 0 || (nruns && !runs)) return fail(THR_ERR_REQUEST, "thr_run_batch: bad arguments");
    for (int r = 0; r < nruns; ++r) {
        const thr_run_desc &d = runs[r];
        if (d.nargs < 0 || (d.nargs && !d.args) || d.ntmaps < 0 || (d.ntmaps && (!d.tmaps || !d.module)))
            return fail(THR_ERR_REQUEST, "thr_run_batch: request %d has bad arguments", r);
    }
    BatchRes *res = nullptr;
    int rc = batch_resources(&res);
    if (rc) return rc;
    cudaStream_t sin = res->s[0], scmp = res->s[1], sout = res->s[2];
    size_t nev = 0;
    auto event = [&](cudaEvent_t *e) -> bool { return batch_event(*res, nev++, e) == THR_OK; };
    // the batch's buffers sit after the slots thr_run uses for one request's arguments
    size_t slot = 4096;
    for (int r = 0; r < nruns && rc == THR_OK; ++r) {
        const thr_run_desc &d = runs[r];
        std::vector<uint64_t> dev(d.nargs);
        for (int i = 0; i < d.nargs && rc == THR_OK; ++i) {
            void *p = nullptr;
            if ((rc = slot_buffer(slot++, d.args[i].nbytes, &p))) break;
            dev[i] = (uint64_t)(uintptr_t)p;
            cudaError_t e = d.args[i].kind == THR_ARG_INPUT
                                ? cudaMemcpyAsync(p, d.args[i].host, d.args[i].nbytes, cudaMemcpyHostToDevice, sin)
                                : cudaMemsetAsync(p, 0, d.args[i].nbytes, sin);
            if (e != cudaSuccess) rc = cuda_fail(e, "staging a batch argument");
        }
        if (rc) break;
        int set = -1;
        if (d.ntmaps && (rc = tmap_bind(d.module, d.tmaps, d.ntmaps, d.ptr_table, dev.data(), d.nargs, sin, &set)))
            break;
        cudaEvent_t staged, ran;
        if (!event(&staged) || !event(&ran)) {
            rc = fail(THR_ERR_CUDA, "cudaEventCreate");
            break;
        }
        cudaEventRecord(staged, sin);
        cudaStreamWaitEvent(scmp, staged, 0);
        if ((rc = thr_launch(d.function, d.grid, d.block, d.smem_bytes, dev.data(), d.nargs,
                             (uint64_t)(uintptr_t)scmp)))
            break;
        if (d.ntmaps && (rc = tmap_launched(d.module, set, scmp))) break;
        cudaEventRecord(ran, scmp);
        cudaStreamWaitEvent(sout, ran, 0);
        for (int i = 0; i < d.nargs && rc == THR_OK; ++i)
            if (d.args[i].kind == THR_ARG_OUTPUT) {
                cudaError_t e = cudaMemcpyAsync(d.args[i].host, (void *)(uintptr_t)dev[i], d.args[i].nbytes,
                                                cudaMemcpyDeviceToHost, sout);
                if (e != cudaSuccess) rc = cuda_fail(e, "copying an output back");
            }
    }
    if (sout) {
        // every request's copies and launch are ordered before this point of the copy-out stream
        cudaEvent_t done;
        if (event(&done)) {
            cudaEventRecord(done, sout);
            int w = wait_event(done, timeout_s);
            if (rc == THR_OK) rc = w;
        } else if (rc == THR_OK) {
            rc = fail(THR_ERR_CUDA, "cudaEventCreate");
        }
    }
    if (rc != THR_OK) {
        // leave nothing in flight that reads the caller's host buffers (or the reused events)
        cudaStreamSynchronize(sin);
        cudaStreamSynchronize(scmp);
        cudaStreamSynchronize(sout);
    }
    return rc;
}

int thr_tmap_bind(uint64_t module, const thr_tmap_spec *tmaps, int ntmaps, const char *ptr_table,
                  const uint64_t *args, int nargs, uint64_t stream, int *set) {
    int s = ensure_driver();
    if (s) return s;
    if (!module || ntmaps <= 0 || !tmaps || !args || nargs <= 0 || !set)
        return fail(THR_ERR_REQUEST, "thr_tmap_bind: bad arguments");
    for (int i = 0; i < ntmaps; ++i)
        if (!tmaps[i].global) return fail(THR_ERR_REQUEST, "thr_tmap_bind: tensor map %d names no global", i);
    return tmap_bind(module, tmaps, ntmaps, ptr_table, args, nargs, (cudaStream_t)(uintptr_t)stream, set);
}

int thr_tmap_launched(uint64_t module, int set, uint64_t stream) {
    return tmap_launched(module, set, (cudaStream_t)(uintptr_t)stream);
}

int thr_tensor_map(void *out128, int dtype_code, int rank, uint64_t base, const uint64_t *dims,
                   const uint64_t *strides_bytes, const uint32_t *box, int swizzle) {
    int s = ensure_driver();
    if (s) return s;
    if (!g_drv.tmap) return fail(THR_ERR_CUDA, "the driver has no cuTensorMapEncodeTiled");
    if (!out128 || rank < 1 || rank > 5 || !dims || !box) return fail(THR_ERR_REQUEST, "thr_tensor_map: bad arguments");
    CUtensorMapDataType dt = dtype_code == 0   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                             : dtype_code == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    CUtensorMapSwizzle sw = swizzle == 3   ? CU_TENSOR_MAP_SWIZZLE_128B
                            : swizzle == 2 ? CU_TENSOR_MAP_SWIZZLE_64B
                            : swizzle == 1 ? CU_TENSOR_MAP_SWIZZLE_32B
                                           : CU_TENSOR_MAP_SWIZZLE_NONE;
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        gd[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) gs[i] = strides_bytes[i];
    }
    CUresult r = g_drv.tmap((CUtensorMap *)out128, dt, (cuuint32_t)rank, (void *)(uintptr_t)base, gd, gs, bx, es,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? THR_OK : drv_fail(r, "cuTensorMapEncodeTiled");
}

int thr_memcpy_htod(uint64_t dst, const void *src, uint64_t nbytes, uint64_t stream) {
    cudaError_t e = cudaMemcpyAsync((void *)(uintptr_t)dst, src, nbytes, cudaMemcpyHostToDevice,
                                    (cudaStream_t)(uintptr_t)stream);
    return e == cudaSuccess ? THR_OK : cuda_fail(e, "host to device copy");
}

int thr_memcpy_dtoh(void *dst, uint64_t src, uint64_t nbytes) {
    cudaError_t e = cudaMemcpy(dst, (const void *)(uintptr_t)src, nbytes, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? THR_OK : cuda_fail(e, "device to host copy");
}

int thr_synchronize(void) {
    cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? THR_OK : fail(THR_ERR_RUN, "device synchronise: %s", cudaGetErrorString(e));
}

int thr_release_buffers(void) {
    release_batch_resources();
    for (auto &s : g_slots)
        if (s.ptr) cudaFree(s.ptr);
    g_slots.clear();
    return THR_OK;
}

// ---- peer mailboxes (CUDA IPC, plain device memory) -----------------------------------

int thr_peer_alloc(uint64_t bytes, uint64_t *dptr, unsigned char handle[THR_IPC_HANDLE_BYTES]) {
    if (!dptr || !handle || bytes == 0) return fail(THR_ERR_REQUEST, "thr_peer_alloc: bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == THR_IPC_HANDLE_BYTES, "IPC handle size");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "peer mailbox cudaMalloc");
    e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "peer mailbox handle");
    }
    memcpy(handle, &h, sizeof h);
    *dptr = (uint64_t)(uintptr_t)p;
    return THR_OK;
}

int thr_peer_open(const unsigned char handle[THR_IPC_HANDLE_BYTES], uint64_t *dptr) {
    if (!dptr || !handle) return fail(THR_ERR_REQUEST, "thr_peer_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *dptr = (uint64_t)(uintptr_t)p;
    return THR_OK;
}

int thr_peer_close(uint64_t dptr) {
    cudaError_t e = cudaIpcCloseMemHandle((void *)(uintptr_t)dptr);
    return e == cudaSuccess ? THR_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int thr_peer_free(uint64_t dptr) {
    cudaError_t e = cudaFree((void *)(uintptr_t)dptr);
    return e == cudaSuccess ? THR_OK : cuda_fail(e, "peer mailbox cudaFree");
}

// Lets the allocation-free entry points (noalloc.cu) report through thr_last_error.
int thr_noalloc_set_error(const char *msg) {
    g_err = msg ? msg : "";
    return THR_OK;
}

int thr_last_error(char *buf, size_t n) {
    if (!buf || !n) return THR_ERR_REQUEST;
    strncpy(buf, g_err.c_str(), n - 1);
    buf[n - 1] = 0;
    return THR_OK;
}

}  // extern "C"
