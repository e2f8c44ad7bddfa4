// noalloc.cu -- a RoFormer separation that allocates no device memory.
//
// Some hosts cannot call cudaMalloc: plug-ins that run inside an audio application whose
// device memory is handed out by the host (a DAW or a game engine owns the CUDA context and
// forbids allocations from its plug-ins), and real-time callers that must not block on the
// allocator. stg_separate_roformer_noalloc serves them: the caller passes the mix, the masks
// and the output buffer; the tables and the scratch of the fused kernel live in one static
// device array of 64 MiB, reserved on every GPU that loads this library until the process
// exits. The kernels are the same as stg_separate's.
#include "../../include/stems_gpu_v1.h"
#include "kernels.h"
#include "plan.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

using namespace stg;

constexpr size_t kArenaBytes = (size_t)64 << 20;
constexpr int kMaxDevices = 64;

// The scratch arena. In host code this name is a host-side stand-in, not a device address:
// kernels get the address that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_arena[kArenaBytes];

std::mutex g_mutex;
void* g_arena_address[kMaxDevices];   // per device, set by the first call on that device

// The arena's device address on `device` (the current device), looked up once.
void* arena_on(int device) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_arena_address[device]) {
        void* p = nullptr;
        cuda_check(cudaGetSymbolAddress(&p, g_arena), "cudaGetSymbolAddress(arena)");
        g_arena_address[device] = p;
    }
    return g_arena_address[device];
}

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
void put(unsigned char* base, size_t at, const std::vector<T>& v, cudaStream_t st) {
    if (!v.empty())
        cuda_check(cudaMemcpyAsync(base + at, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st),
                   "copy a table into the arena");
}

void write_message(char* msg, size_t cap, const char* text) {
    if (msg && cap) std::snprintf(msg, cap, "%s", text);
}

} // namespace

extern "C" STG_API stg_status stg_separate_roformer_noalloc(int device, const stg_roformer_config* config,
                                                            int64_t n_samples, const float* d_mix,
                                                            const float* d_mask, float* d_out, void* stream,
                                                            char* message, size_t message_size) {
    write_message(message, message_size, "");
    int previous = -1;
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
        if (device < 0 || device >= n_dev || device >= kMaxDevices) fail(STG_INVALID_ARGUMENT, "no such device");
        cuda_check(cudaGetDevice(&previous), "cudaGetDevice");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        unsigned char* arena = static_cast<unsigned char*>(arena_on(device));

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
        const size_t o_btab = c.take(H.btab.size() * sizeof(int2));
        const size_t o_ebeg = c.take(H.ebeg.size() * sizeof(int));
        const size_t o_ent = c.take(std::max<size_t>(1, H.ent.size()) * sizeof(int2));
        const size_t o_binv = c.take(H.binv.size() * sizeof(float));
        const size_t o_win = c.take(win.size() * sizeof(float));
        const size_t o_tw = c.take(tw.size() * sizeof(float2));
        const size_t o_y = c.take(H.y_bytes());
        const size_t o_tr = c.take(std::max<size_t>(16, H.tr_bytes()));
        if (c.used > kArenaBytes) {
            char text[256];
            std::snprintf(text, sizeof(text),
                          "this separation needs %.1f MiB of scratch; the no-allocation entry point has %zu MiB "
                          "(use stg_plan_roformer + stg_separate)", (double)c.used / (1 << 20), kArenaBytes >> 20);
            fail(STG_INVALID_ARGUMENT, text);
        }

        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        put(arena, o_chunks, H.chunks, st);
        put(arena, o_groups, H.groups, st);
        put(arena, o_w, H.W, st);
        put(arena, o_env, H.env, st);
        put(arena, o_btab, H.btab, st);
        put(arena, o_ebeg, H.ebeg, st);
        put(arena, o_ent, H.ent, st);
        put(arena, o_binv, H.binv, st);
        put(arena, o_win, win, st);
        put(arena, o_tw, tw, st);

        // Every Y and Tr element the combine reads is written by the fused kernel of the same
        // call, so the arena needs no clearing between calls.
        PlanDevice D;
        D.chunks = reinterpret_cast<const ChunkDesc*>(arena + o_chunks);
        D.groups = reinterpret_cast<const ChunkGroup*>(arena + o_groups);
        D.W = reinterpret_cast<const float*>(arena + o_w);
        D.env = reinterpret_cast<const float*>(arena + o_env);
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
    if (previous >= 0) cudaSetDevice(previous);
    return status;
}
