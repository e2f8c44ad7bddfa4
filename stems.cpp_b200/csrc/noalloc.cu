// noalloc.cu -- a RoFormer separation that allocates no device memory.
//
// Some hosts cannot call cudaMalloc: plug-ins that run inside an audio application whose
// device memory is handed out by the host (a DAW or a game engine owns the CUDA context and
// forbids allocations from its plug-ins), and real-time callers that must not block on the
// allocator. stg_separate_roformer_noalloc serves them: the caller passes the mix, the masks
// and the output buffer; the tables and the scratch of the fused kernel live in one static
// device array of 64 MiB, reserved on every GPU that loads this library until the process
// exits. The kernels are the same as stg_separate's.
//
// Contexts. The call runs in `device`'s primary context, the one the CUDA runtime and the
// applications built on it use: when another device's primary context (or none) is current
// on the calling thread, it makes `device`'s current for the call and puts the caller's back
// afterwards. A context the caller created with the driver API (cuCtxCreate) is refused with
// STG_UNSUPPORTED before any GPU work: the runtime resolves the array's address, and loads the
// library's kernels, for primary contexts. The address is looked up (cudaGetSymbolAddress)
// once per context, on its first call, and kept by the driver's unique context ID.
#include "../../include/stems_gpu_v1.h"
#include "kernels.h"
#include "plan.h"

#include <cuda.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

namespace {

using namespace stg;

constexpr size_t kArenaBytes = (size_t)64 << 20;

// The scratch arena. In host code this name is a host-side stand-in, not a device address:
// kernels get the address that cudaGetSymbolAddress returns for the current context.
static __device__ __align__(256) unsigned char g_arena[kArenaBytes];

// Driver entry points through the runtime, so that the library needs no link to libcuda.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxSetCurrentFn = CUresult (*)(CUcontext);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
using CtxGetDeviceFn = CUresult (*)(CUdevice*);
using PrimaryRetainFn = CUresult (*)(CUcontext*, CUdevice);
using PrimaryReleaseFn = CUresult (*)(CUdevice);
struct Driver {
    CtxGetCurrentFn get = nullptr;
    CtxSetCurrentFn set = nullptr;
    CtxGetIdFn id = nullptr;
    CtxGetDeviceFn device = nullptr;
    PrimaryRetainFn retain = nullptr;
    PrimaryReleaseFn release = nullptr;
    bool ok() const { return get && set && id && device && retain && release; }
};
template <class F> F entry_point(const char* name) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<F>(p);
}
const Driver& driver() {
    static const Driver d{entry_point<CtxGetCurrentFn>("cuCtxGetCurrent"), entry_point<CtxSetCurrentFn>("cuCtxSetCurrent"),
                          entry_point<CtxGetIdFn>("cuCtxGetId"), entry_point<CtxGetDeviceFn>("cuCtxGetDevice"),
                          entry_point<PrimaryRetainFn>("cuDevicePrimaryCtxRetain"),
                          entry_point<PrimaryReleaseFn>("cuDevicePrimaryCtxRelease")};
    return d;
}

// Per context (by the driver's unique context ID, which a later context never reuses): the
// arena's device address, and the host copy of the tables the last call uploaded, kept for the
// life of the library so that no copy reads host memory a return has freed.
struct ContextState {
    unsigned char* arena = nullptr;
    std::vector<unsigned char> staging;
    size_t uploaded = 0;   // bytes of staging the arena holds (0: none)
};
std::mutex g_mutex;
std::map<unsigned long long, ContextState> g_contexts;

// Carves 256-byte aligned regions out of the arena, in order.
struct Carver {
    size_t used = 0;
    size_t take(size_t bytes) {
        const size_t at = (used + 255) & ~(size_t)255;
        used = at + bytes;
        return at;
    }
};

template <class T>
void stage(std::vector<unsigned char>& host, size_t at, const std::vector<T>& v) {
    if (!v.empty()) std::memcpy(host.data() + at, v.data(), v.size() * sizeof(T));
}

void write_message(char* msg, size_t cap, const char* text) {
    if (msg && cap) std::snprintf(msg, cap, "%s", text);
}

// Makes `device`'s primary context current for the call (refusing a caller-created context);
// the destructor puts the caller's context back.
struct ContextScope {
    bool switched = false;
    CUcontext previous = nullptr;
    explicit ContextScope(int device) {
        const Driver& d = driver();
        if (!d.ok()) fail(STG_INTERNAL_ERROR, "the CUDA driver's context entry points are unavailable");
        if (d.get(&previous) != CUDA_SUCCESS) fail(STG_INTERNAL_ERROR, "cuCtxGetCurrent failed");
        bool ours = false;   // previous is `device`'s primary context
        if (previous) {
            CUdevice dev = 0;
            CUcontext primary = nullptr;
            if (d.device(&dev) != CUDA_SUCCESS || d.retain(&primary, dev) != CUDA_SUCCESS)
                fail(STG_INTERNAL_ERROR, "cannot query the current context");
            d.release(dev);
            if (primary != previous)
                fail(STG_UNSUPPORTED, "the current CUDA context is not a primary context: this entry point runs in "
                                      "the device's primary context (the CUDA runtime's)");
            int current = -1;
            cuda_check(cudaGetDevice(&current), "cudaGetDevice");
            ours = current == device;
        }
        if (!ours) {
            cuda_check(cudaSetDevice(device), "cudaSetDevice");
            switched = true;
        }
    }
    ~ContextScope() {
        if (switched) driver().set(previous);
    }
    static unsigned long long current_id() {
        CUcontext c = nullptr;
        unsigned long long id = 0;
        if (driver().get(&c) != CUDA_SUCCESS || !c || driver().id(c, &id) != CUDA_SUCCESS)
            fail(STG_INTERNAL_ERROR, "no current CUDA context");
        return id;
    }
};

} // namespace

extern "C" STG_API stg_status stg_separate_roformer_noalloc(int device, const stg_roformer_config* config,
                                                            int64_t n_samples, const float* d_mix,
                                                            const float* d_mask, float* d_out, void* stream,
                                                            char* message, size_t message_size) {
    write_message(message, message_size, "");
    stg_status status = STG_OK;
    try {
        if (!config || config->size < sizeof(stg_roformer_config))
            fail(STG_INVALID_ARGUMENT, "config is NULL or config.size is too small");
        if (!d_mix || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        if (reinterpret_cast<uintptr_t>(d_mask) % 16) fail(STG_INVALID_ARGUMENT, "mask must be 16-byte aligned");
        if (n_samples <= 0) fail(STG_INVALID_ARGUMENT, "empty input");
        if (n_samples > (int64_t)INT32_MAX / 4) fail(STG_INVALID_ARGUMENT, "input is too long");
        int n_dev = 0;
        cuda_check(cudaGetDeviceCount(&n_dev), "cudaGetDeviceCount");
        if (device < 0 || device >= n_dev) fail(STG_INVALID_ARGUMENT, "no such device");
        // the plan's tile size asks the current device for its resident CTAs: the context first
        ContextScope scope(device);

        HostPlan H;
        H.len = n_samples;
        build_roformer(H, *config, n_samples);
        std::vector<float> win;
        std::vector<float2> tw;
        fft_tables(H.g.n_fft, win, tw);

        Carver c;
        const size_t o_chunks = c.take(H.chunks.size() * sizeof(ChunkDesc));
        const size_t o_groups = c.take(H.groups.size() * sizeof(ChunkGroup));
        const size_t o_w = c.take(H.W.size() * sizeof(float));
        const size_t o_env = c.take(H.env.size() * sizeof(float));
        const size_t o_envp = c.take(std::max<size_t>(1, H.env_period.size()) * sizeof(float));
        const size_t o_btab = c.take(H.btab.size() * sizeof(int2));
        const size_t o_ebeg = c.take(H.ebeg.size() * sizeof(int));
        const size_t o_ent = c.take(std::max<size_t>(1, H.ent.size()) * sizeof(int2));
        const size_t o_binv = c.take(H.binv.size() * sizeof(float));
        const size_t o_win = c.take(win.size() * sizeof(float));
        const size_t o_tw = c.take(tw.size() * sizeof(float2));
        const size_t tables = c.used;
        const size_t o_y = c.take(H.y_bytes());
        const size_t o_tr = c.take(std::max<size_t>(16, H.tr_bytes()));
        if (c.used > kArenaBytes) {
            char text[256];
            std::snprintf(text, sizeof(text),
                          "this separation needs %.1f MiB of scratch; the no-allocation entry point has %zu MiB "
                          "(use stg_plan_roformer + stg_separate)", (double)c.used / (1 << 20), kArenaBytes >> 20);
            fail(STG_INVALID_ARGUMENT, text);
        }

        // the tables as one block, laid out as in the arena
        std::vector<unsigned char> next(tables, 0);
        stage(next, o_chunks, H.chunks);
        stage(next, o_groups, H.groups);
        stage(next, o_w, H.W);
        stage(next, o_env, H.env);
        stage(next, o_envp, H.env_period);
        stage(next, o_btab, H.btab);
        stage(next, o_ebeg, H.ebeg);
        stage(next, o_ent, H.ent);
        stage(next, o_binv, H.binv);
        stage(next, o_win, win);
        stage(next, o_tw, tw);

        std::lock_guard<std::mutex> lock(g_mutex);
        ContextState& cs = g_contexts[ContextScope::current_id()];
        if (!cs.arena) {   // once per context: the arena's address in it
            void* p = nullptr;
            cuda_check(cudaGetSymbolAddress(&p, g_arena), "cudaGetSymbolAddress(arena)");
            cs.arena = static_cast<unsigned char*>(p);
        }
        unsigned char* arena = cs.arena;
        // The previous call's tables are still in the arena when they are these very bytes (its
        // scratch lies after them); otherwise one copy from the library's host staging.
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (cs.uploaded != tables || cs.staging != next) {
            cs.uploaded = 0;
            cs.staging.swap(next);
            cuda_check(cudaMemcpyAsync(arena, cs.staging.data(), tables, cudaMemcpyHostToDevice, st),
                       "copy the tables into the arena");
            cs.uploaded = tables;
        }

        // Every Y and Tr element the combine reads is written by the fused kernel of the same
        // call, so the arena needs no clearing between calls.
        PlanDevice D;
        D.chunks = reinterpret_cast<const ChunkDesc*>(arena + o_chunks);
        D.groups = reinterpret_cast<const ChunkGroup*>(arena + o_groups);
        D.W = reinterpret_cast<const float*>(arena + o_w);
        D.env = reinterpret_cast<const float*>(arena + o_env);
        D.env_period = H.env_period.empty() ? nullptr : reinterpret_cast<const float*>(arena + o_envp);
        D.btab = reinterpret_cast<const int2*>(arena + o_btab);
        D.ebeg = reinterpret_cast<const int*>(arena + o_ebeg);
        D.ent = reinterpret_cast<const int2*>(arena + o_ent);
        D.binv = reinterpret_cast<const float*>(arena + o_binv);
        D.win = reinterpret_cast<const float*>(arena + o_win);
        D.tw = reinterpret_cast<const float2*>(arena + o_tw);
        D.Y = reinterpret_cast<float*>(arena + o_y);
        D.Tr = reinterpret_cast<float*>(arena + o_tr);
        launch_plan(H, D, d_mix, d_mask, d_out, st, nullptr, nullptr);
    } catch (const Failure& f) {
        status = f.code;
        write_message(message, message_size, f.what());
    } catch (const std::bad_alloc&) {
        status = STG_OUT_OF_MEMORY;
        write_message(message, message_size, "out of host memory");
    } catch (const std::exception& x) {
        status = STG_INTERNAL_ERROR;
        write_message(message, message_size, x.what());
    }
    return status;
}
