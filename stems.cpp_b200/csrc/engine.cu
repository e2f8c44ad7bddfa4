// engine.cu -- engines, plans with device-resident tables, and the C ABI declared in
// include/stems_gpu_v1.h. The schedule itself is built by plan.cu.
#include "../../include/stems_gpu_v1.h"
#include "kernels.h"
#include "plan.h"

#include <algorithm>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <new>
#include <string>
#include <tuple>
#include <vector>

#define STG_VERSION_STRING "stems-b200 spectral 0.1 (stems_gpu abi 1)"

namespace {

using namespace stg;

// A device buffer that frees itself.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { if (p) cudaFree(p); }
    void reserve(size_t n, const char* what) {
        if (n <= bytes) return;
        if (p) { cudaFree(p); p = nullptr; bytes = 0; }
        if (n == 0) return;
        cuda_check(cudaMalloc(&p, n), what);
        bytes = n;
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

template <class T>
void upload(DevBuf& d, const std::vector<T>& v, const char* what) {
    d.reserve(std::max<size_t>(v.size() * sizeof(T), 16), what);
    if (!v.empty()) cuda_check(cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), what);
}

struct FftTables {
    DevBuf win, tw;
};

} // namespace

// ---- engine -------------------------------------------------------------------------------
struct stg_engine {
    int device = 0;
    bool profiling = false;
    std::string last_error;
    std::map<int, std::unique_ptr<FftTables>> tables;
    // single-chunk plans of the DSP primitives, by (kind, n_fft, hop, normalized, C, length)
    std::map<std::tuple<int, int, int, int, int, int64_t>, std::unique_ptr<stg_plan>> primitives;
    // Kaiser kernel tables of the resampler, by (source rate, destination rate)
    struct Kaiser {
        DevBuf table;
        double half = 0, ratio = 1;
    };
    std::map<std::pair<int, int>, std::unique_ptr<Kaiser>> kaiser;

    const Kaiser& kaiser_for(int src, int dst) {
        auto& k = kaiser[{src, dst}];
        if (!k) {
            auto nk = std::make_unique<Kaiser>();
            std::vector<double> t;
            kaiser_table(src, dst, t, nk->half, nk->ratio);
            upload(nk->table, t, "resampling table");
            k = std::move(nk);
        }
        return *k;
    }

    const FftTables& fft_tables_for(int n) {
        auto& t = tables[n];
        if (!t) {
            auto nt = std::make_unique<FftTables>();
            std::vector<float> win;
            std::vector<float2> tw;
            fft_tables(n, win, tw);
            upload(nt->win, win, "window table");
            upload(nt->tw, tw, "twiddle table");
            t = std::move(nt);
        }
        return *t;
    }
};

struct stg_plan {
    stg_engine* engine = nullptr;
    HostPlan H;
    PlanDevice D;
    DevBuf d_chunks, d_groups, d_w, d_env, d_btab, d_ebeg, d_ent, d_binv;
    DevBuf d_y, d_tr;
    DevBuf d_mixn, d_mono, d_cac_part, d_cac_stats;   // scratch of the HTDemucs normalisations
    DevBuf d_mask_t;                                  // t-major masks (HTDemucs, TFC-TDF)
    const float* mono_src = nullptr;                  // the track d_mixn was normalised from
    DevBuf s_mix, s_mask, s_out;   // device staging for stg_separate_host
    DevBuf n_in, n_out;            // one batch of network input and output (stg_separate_network)
    RunTiming timing;

    ~stg_plan() {
        for (cudaEvent_t& e : timing.ev)
            if (e) cudaEventDestroy(e);
    }

    // Device copies of the tables, and the scratch the fused kernel writes.
    void upload_all() {
        const FftTables& t = engine->fft_tables_for(H.g.n_fft);
        upload(d_chunks, H.chunks, "chunk table");
        upload(d_groups, H.groups, "chunk groups");
        upload(d_w, H.W, "weight table");
        upload(d_env, H.env, "envelope table");
        upload(d_btab, H.btab, "band table");
        upload(d_ebeg, H.ebeg, "band table");
        upload(d_ent, H.ent, "band table");
        upload(d_binv, H.binv, "band table");
        d_y.reserve(std::max<size_t>(16, H.y_bytes()), "chunk outputs");
        d_tr.reserve(std::max<size_t>(16, H.tr_bytes()), "tile partials");
        if (H.mono_norm) {
            d_mixn.reserve(H.mixn_bytes(), "normalised mix");
            d_mono.reserve(H.mono_bytes(), "mono statistics");
            D.mixn = d_mixn.as<float>();
            D.mono = reinterpret_cast<double*>(d_mono.p);
        }
        if (H.mask_planes) {
            d_mask_t.reserve(H.mask_t_bytes(), "t-major masks");
            D.mask_t = reinterpret_cast<float4*>(d_mask_t.p);
        }
        if (H.cac_norm) {
            d_cac_part.reserve(H.cac_part_bytes(), "CaC partial sums");
            d_cac_stats.reserve(H.cac_stats_bytes(), "CaC statistics");
            D.cac_part = reinterpret_cast<double2*>(d_cac_part.p);
            D.cac_stats = reinterpret_cast<double2*>(d_cac_stats.p);
        }
        D.chunks = d_chunks.as<ChunkDesc>();
        D.groups = d_groups.as<ChunkGroup>();
        D.W = d_w.as<float>();
        D.env = d_env.as<float>();
        D.btab = d_btab.as<int2>();
        D.ebeg = d_ebeg.as<int>();
        D.ent = d_ent.as<int2>();
        D.binv = d_binv.as<float>();
        D.win = t.win.as<float>();
        D.tw = t.tw.as<float2>();
        D.Y = d_y.as<float>();
        D.Tr = d_tr.as<float>();
    }

    void run(const float* d_mix, const float* d_mask, float* d_out, cudaStream_t st, const stg_run_options* opt) {
        if (!d_mix || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        if (reinterpret_cast<uintptr_t>(d_mask) % 16) fail(STG_INVALID_ARGUMENT, "mask must be 16-byte aligned");
        cuda_check(cudaSetDevice(engine->device), "cudaSetDevice");
        timing.timed = engine->profiling;
        if (timing.timed)
            for (cudaEvent_t& e : timing.ev)
                if (!e) cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        launch_plan(H, D, d_mix, d_mask, d_out, st, opt, &timing);
    }

    // The mix the front half reads: with the mono normalisation, chunk 0's call normalises
    // the track into d_mixn and later calls of the same track read it.
    const float* front_mix(const float* d_mix, int first, cudaStream_t st) {
        if (!H.mono_norm) return d_mix;
        if (!d_mix) fail(STG_INVALID_ARGUMENT, "null buffer");
        if (first == 0) {
            normalise_mix(H, D, d_mix, st);
            mono_src = d_mix;
        } else if (mono_src != d_mix) {
            fail(STG_INVALID_ARGUMENT, "with the mono normalisation, the first batch must start at chunk 0");
        }
        return D.mixn;
    }
};

namespace {

template <class T> bool sized(const T* p) { return p && p->size >= sizeof(uint32_t) * 2; }

stg_status guard(stg_engine* e, const std::function<void()>& fn) {
    try {
        fn();
        if (e) e->last_error.clear();
        return STG_OK;
    } catch (const Failure& f) {
        if (e) e->last_error = f.what();
        return f.code;
    } catch (const std::bad_alloc&) {
        if (e) e->last_error = "out of memory";
        return STG_OUT_OF_MEMORY;
    } catch (const std::exception& x) {
        if (e) e->last_error = x.what();
        return STG_INTERNAL_ERROR;
    }
}

template <class Cfg, class Fn>
stg_status make_plan(stg_engine* e, const Cfg* cfg, int64_t n, stg_plan** out, Fn build) {
    if (!out) return STG_INVALID_ARGUMENT;
    *out = nullptr;
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        if (!sized(cfg) || cfg->size < sizeof(Cfg)) fail(STG_INVALID_ARGUMENT, "config is NULL or config.size is too small");
        if (n <= 0) fail(STG_INVALID_ARGUMENT, "empty input");
        if (n > (int64_t)INT32_MAX / 4) fail(STG_INVALID_ARGUMENT, "input is too long");   // libstems.cpp:148
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        auto p = std::make_unique<stg_plan>();
        p->engine = e;
        p->H.len = n;
        build(p->H, *cfg, n);
        p->upload_all();
        *out = p.release();
    });
}

// The engine's cached single-chunk plan of a DSP primitive (kind 0: torch.stft geometry,
// 1: torch.istft, 2: HTDemucs _spec/_ispec).
stg_plan& primitive_plan(stg_engine* e, int kind, int n_fft, int hop, int normalized, int C, int64_t len) {
    const auto key = std::make_tuple(kind, n_fft, hop, normalized, C, len);
    auto it = e->primitives.find(key);
    if (it != e->primitives.end()) return *it->second;
    auto p = std::make_unique<stg_plan>();
    p->engine = e;
    if (kind == 2) build_htdemucs_spec(p->H, C, len);
    else build_torch_stft(p->H, n_fft, hop, normalized != 0, C, len, kind == 1);
    p->upload_all();
    if (e->primitives.size() >= 64) e->primitives.clear();   // keep the cache bounded
    return *(e->primitives[key] = std::move(p));
}

} // namespace

// ---- C ABI -----------------------------------------------------------------------------------
extern "C" {

STG_API const char* stg_version(void) { return STG_VERSION_STRING; }

STG_API int stg_device_count(void) {
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) { cudaGetLastError(); return e == cudaErrorNoDevice ? 0 : -1; }
    return n;
}

STG_API stg_status stg_engine_create(int device, stg_engine** out) {
    if (!out) return STG_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return STG_INTERNAL_ERROR; }
    if (device < 0 || device >= n) return STG_INVALID_ARGUMENT;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) { cudaGetLastError(); return STG_INTERNAL_ERROR; }
    if (prop.major < 10) return STG_UNSUPPORTED;   // built for sm_100a only
    if (cudaSetDevice(device) != cudaSuccess) { cudaGetLastError(); return STG_INTERNAL_ERROR; }
    stg_engine* e = new (std::nothrow) stg_engine;
    if (!e) return STG_OUT_OF_MEMORY;
    e->device = device;
    *out = e;
    return STG_OK;
}

STG_API void stg_engine_destroy(stg_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    delete e;
}

STG_API const char* stg_engine_last_error(const stg_engine* e) { return e ? e->last_error.c_str() : ""; }

STG_API stg_status stg_engine_set_profiling(stg_engine* e, int32_t enabled) {
    if (!e) return STG_INVALID_ARGUMENT;
    e->profiling = enabled != 0;
    return STG_OK;
}

STG_API stg_status stg_plan_last_timing(stg_plan* p, float* fused_ms, float* combine_ms, int32_t* launches) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (!p->timing.timed) fail(STG_INVALID_ARGUMENT, "the last run was not timed (stg_engine_set_profiling)");
        cuda_check(cudaEventSynchronize(p->timing.ev[3]), "cudaEventSynchronize");
        float a = 0.0f, b = 0.0f;
        cuda_check(cudaEventElapsedTime(&a, p->timing.ev[0], p->timing.ev[2]), "cudaEventElapsedTime");
        cuda_check(cudaEventElapsedTime(&b, p->timing.ev[2], p->timing.ev[3]), "cudaEventElapsedTime");
        if (fused_ms) *fused_ms = a;
        if (combine_ms) *combine_ms = b;
        if (launches) *launches = p->timing.launches;
    });
}

STG_API stg_status stg_plan_last_timing_detail(stg_plan* p, float* prep_ms, float* fused_ms, float* combine_ms,
                                               int32_t* launches) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (!p->timing.timed) fail(STG_INVALID_ARGUMENT, "the last run was not timed (stg_engine_set_profiling)");
        cuda_check(cudaEventSynchronize(p->timing.ev[3]), "cudaEventSynchronize");
        float t[3] = {0.0f, 0.0f, 0.0f};
        for (int k = 0; k < 3; k++)
            cuda_check(cudaEventElapsedTime(&t[k], p->timing.ev[k], p->timing.ev[k + 1]), "cudaEventElapsedTime");
        if (prep_ms) *prep_ms = t[0];
        if (fused_ms) *fused_ms = t[1];
        if (combine_ms) *combine_ms = t[2];
        if (launches) *launches = p->timing.launches;
    });
}

STG_API stg_status stg_plan_htdemucs(stg_engine* e, const stg_htdemucs_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, build_htdemucs);
}
STG_API stg_status stg_plan_roformer(stg_engine* e, const stg_roformer_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, build_roformer);
}
STG_API stg_status stg_plan_tfc(stg_engine* e, const stg_tfc_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, build_tfc);
}

STG_API void stg_plan_destroy(stg_plan* p) {
    if (!p) return;
    cudaSetDevice(p->engine->device);
    delete p;
}

STG_API stg_status stg_plan_get_info(const stg_plan* p, stg_plan_info* info) {
    if (!p || !info || info->size < sizeof(stg_plan_info)) return STG_INVALID_ARGUMENT;
    const HostPlan& H = p->H;
    info->arch = H.arch;
    info->n_samples = H.len;
    info->n_channels = H.C;
    info->n_out_sources = H.S_out;
    info->n_chunks = H.n_chunks();
    info->n_frames = H.g.T;
    info->mask_floats_per_chunk = H.mask_per_chunk;
    info->out_floats = H.out_floats();
    info->scratch_bytes = (int64_t)(p->d_y.bytes + p->d_tr.bytes + p->d_mixn.bytes + p->d_mono.bytes +
                                    p->d_cac_part.bytes + p->d_cac_stats.bytes + p->d_mask_t.bytes);
    return STG_OK;
}

STG_API stg_status stg_separate_ex(stg_plan* p, const float* d_mix, const float* d_mask, float* d_out,
                                   void* stream, const stg_run_options* opt) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (opt && opt->size < sizeof(stg_run_options)) fail(STG_INVALID_ARGUMENT, "options.size is too small");
        p->run(d_mix, d_mask, d_out, static_cast<cudaStream_t>(stream), opt);
    });
}

STG_API stg_status stg_separate(stg_plan* p, const float* d_mix, const float* d_mask, float* d_out, void* stream) {
    return stg_separate_ex(p, d_mix, d_mask, d_out, stream, nullptr);
}

STG_API stg_status stg_separate_host(stg_plan* p, const float* h_mix, const float* h_mask, float* h_out,
                                     void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (!h_mix || !h_mask || !h_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        const HostPlan& H = p->H;
        const size_t mix_b = sizeof(float) * (size_t)H.C * H.len;
        const size_t mask_b = sizeof(float) * (size_t)H.mask_per_chunk * H.chunks.size();
        const size_t out_b = sizeof(float) * (size_t)H.out_floats();
        p->s_mix.reserve(mix_b, "staging");
        p->s_mask.reserve(mask_b, "staging");
        p->s_out.reserve(out_b, "staging");
        cuda_check(cudaMemcpyAsync(p->s_mix.p, h_mix, mix_b, cudaMemcpyHostToDevice, st), "copy mix in");
        cuda_check(cudaMemcpyAsync(p->s_mask.p, h_mask, mask_b, cudaMemcpyHostToDevice, st), "copy masks in");
        p->run(p->s_mix.as<float>(), p->s_mask.as<float>(), p->s_out.as<float>(), st, nullptr);
        cuda_check(cudaMemcpyAsync(h_out, p->s_out.p, out_b, cudaMemcpyDeviceToHost, st), "copy result out");
        cuda_check(cudaStreamSynchronize(st), "separation");
    });
}

// ---- the halves around a real network ----------------------------------------------------
STG_API stg_status stg_plan_network_info(const stg_plan* p, stg_network_info* info) {
    if (!p || !info || info->size < sizeof(stg_network_info)) return STG_INVALID_ARGUMENT;
    info->net_in_floats_per_chunk = p->H.net_in_per_chunk;
    info->net_out_floats_per_chunk = p->H.net_out_per_chunk;
    return STG_OK;
}

STG_API stg_status stg_front(stg_plan* p, const float* d_mix, int32_t first, int32_t n, float* d_net_in, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch_front(p->H, p->D, p->front_mix(d_mix, first, st), first, n, d_net_in, st);
    });
}

STG_API stg_status stg_back(stg_plan* p, const float* d_mix, const float* d_net_out, int32_t first, int32_t n,
                            void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        launch_back(p->H, p->D, d_mix, d_net_out, first, n, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_finish(stg_plan* p, const float* d_mix, float* d_out, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        launch_finish(p->H, p->D, d_mix, d_out, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_separate_network(stg_plan* p, const float* d_mix, float* d_out, int32_t per_batch,
                                        stg_network_fn network, void* user, const stg_run_options* opt,
                                        void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (!network || !d_mix || !d_out) fail(STG_INVALID_ARGUMENT, "null argument");
        if (opt && opt->size < sizeof(stg_run_options)) fail(STG_INVALID_ARGUMENT, "options.size is too small");
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        const HostPlan& H = p->H;
        const int G = (int)H.chunks.size();
        const int per = per_batch > 0 ? std::min(per_batch, G) : G;
        p->n_in.reserve(std::max<size_t>(16, sizeof(float) * (size_t)H.net_in_per_chunk * per), "network input");
        p->n_out.reserve(std::max<size_t>(16, sizeof(float) * (size_t)H.net_out_per_chunk * per), "network output");
        for (int b0 = 0; b0 < G; b0 += per) {
            if (opt && opt->should_cancel && opt->should_cancel(opt->user)) fail(STG_CANCELLED, "cancelled");
            const int nb = std::min(per, G - b0);
            launch_front(H, p->D, p->front_mix(d_mix, b0, st), b0, nb, p->n_in.as<float>(), st);
            if (network(user, b0, nb, p->n_in.as<float>(), p->n_out.as<float>(), stream) != 0)
                fail(STG_MODEL_ERROR, "the network callback failed");
            launch_back(H, p->D, d_mix, p->n_out.as<float>(), b0, nb, st);
            if (opt && opt->on_progress) {
                cuda_check(cudaStreamSynchronize(st), "spectral kernels");
                opt->on_progress(opt->user, b0 + nb, G);
            }
        }
        launch_finish(H, p->D, d_mix, d_out, st);
    });
}

// ---- the request's audio in and the stems out ------------------------------------------------
namespace {
void resample_rows(stg_engine* e, const float* d_in, int interleaved, int64_t n, int in_ch, int to_channels,
                   int rows, int src_rate, int dst_rate, int64_t out_pin, float* d_out, cudaStream_t st) {
    if (!d_in || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
    if (n <= 0 || n > (int64_t)INT32_MAX) fail(STG_INVALID_ARGUMENT, "bad length");
    if (in_ch < 1 || rows < 1 || rows > 4096) fail(STG_INVALID_ARGUMENT, "bad channel count");
    if (src_rate <= 0 || dst_rate <= 0) fail(STG_INVALID_ARGUMENT, "sample rates must be positive");
    cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
    ResampleParams p{};
    p.in = d_in;
    p.in_n = n;
    p.in_ch = in_ch;
    p.interleaved = interleaved;
    p.to_channels = to_channels;
    p.rows = rows;
    p.out_n = resampled_length(n, src_rate, dst_rate);
    p.out_pin = out_pin < 0 ? p.out_n : out_pin;
    p.out_n = std::min(p.out_n, p.out_pin);
    if (src_rate != dst_rate) {
        const auto& k = e->kaiser_for(src_rate, dst_rate);
        p.table = k.table.as<double>();
        p.half = k.half;
        p.ratio = k.ratio;
    }
    p.out = d_out;
    cuda_check(launch_resample(p, st), "resampling kernel launch");
}
} // namespace

STG_API int64_t stg_resampled_length(int64_t n, int32_t src_rate, int32_t dst_rate) {
    if (n < 0 || src_rate <= 0 || dst_rate <= 0) return -1;
    return resampled_length(n, src_rate, dst_rate);
}

STG_API stg_status stg_prepare_input(stg_engine* e, const float* d_in, int32_t interleaved, int64_t n,
                                     int32_t n_channels, int32_t sample_rate, int32_t model_channels,
                                     int32_t model_rate, float* d_out, void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        resample_rows(e, d_in, interleaved != 0, n, n_channels, 1, model_channels, sample_rate, model_rate, -1,
                      d_out, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_restore_output(stg_engine* e, const float* d_stems, int32_t rows, int64_t len,
                                      int32_t model_rate, int32_t sample_rate, int64_t n_samples, float* d_out,
                                      void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        if (n_samples <= 0) fail(STG_INVALID_ARGUMENT, "bad length");
        resample_rows(e, d_stems, 0, len, rows, 0, rows, model_rate, sample_rate, n_samples, d_out,
                      static_cast<cudaStream_t>(stream));
    });
}

// ---- the DSP primitives of src/stft.h --------------------------------------------------
STG_API stg_status stg_torch_stft(stg_engine* e, int32_t n_fft, int32_t hop, int32_t normalized, const float* d_x,
                                  int32_t C, int64_t n, float* d_spec, void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        stg_plan& p = primitive_plan(e, 0, n_fft, hop, normalized, C, n);
        launch_front(p.H, p.D, d_x, 0, 1, d_spec, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_torch_istft(stg_engine* e, int32_t n_fft, int32_t hop, int32_t normalized,
                                   const float* d_spec, int32_t C, int32_t n_frames, float* d_y, void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        if (n_frames < 2 || hop < 1) fail(STG_INVALID_ARGUMENT, "need at least two frames");
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        stg_plan& p = primitive_plan(e, 1, n_fft, hop, normalized, C, (int64_t)hop * (n_frames - 1));
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch_back(p.H, p.D, nullptr, d_spec, 0, 1, st);
        launch_finish(p.H, p.D, nullptr, d_y, st);
    });
}

STG_API stg_status stg_htdemucs_spec(stg_engine* e, const float* d_x, int32_t C, int64_t n, float* d_spec,
                                     void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        stg_plan& p = primitive_plan(e, 2, 4096, 1024, 1, C, n);
        launch_front(p.H, p.D, d_x, 0, 1, d_spec, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_htdemucs_ispec(stg_engine* e, const float* d_spec, int32_t C, int32_t n_frames, int64_t length,
                                      float* d_y, void* stream) {
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        if (length < 1 || n_frames != (int)((length + 1023) / 1024))
            fail(STG_INVALID_ARGUMENT, "n_frames must be ceil(length / 1024)");
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        stg_plan& p = primitive_plan(e, 2, 4096, 1024, 1, C, length);
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch_back(p.H, p.D, nullptr, d_spec, 0, 1, st);
        launch_finish(p.H, p.D, nullptr, d_y, st);
    });
}

} // extern "C"
