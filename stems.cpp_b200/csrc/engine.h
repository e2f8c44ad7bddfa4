// engine.h -- engines and plans with device-resident tables: the objects behind the C ABI
// handles (engine.cu, vr.cu). The schedule itself is built by plan.cu.
#pragma once
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


namespace stg {

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
inline void upload(DevBuf& d, const std::vector<T>& v, const char* what) {
    d.reserve(std::max<size_t>(v.size() * sizeof(T), 16), what);
    if (!v.empty()) cuda_check(cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), what);
}

struct FftTables {
    DevBuf win, tw;
};

} // namespace stg

// the handles of the C ABI live in the global namespace, as the header declares them
using namespace stg;

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
            // entry t and its successor side by side: one 16-byte load per tap
            std::vector<double2> pairs(t.size() - 1);
            for (size_t i = 0; i + 1 < t.size(); i++) pairs[i] = make_double2(t[i], t[i + 1]);
            upload(nk->table, pairs, "resampling table");
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
    DevBuf d_chunks, d_groups, d_w, d_env, d_envp, d_btab, d_ebeg, d_ent, d_binv, d_bag, d_bag_tot;
    DevBuf d_y, d_tr;
    DevBuf d_mixn, d_mono, d_cac_part, d_cac_stats;   // scratch of the HTDemucs normalisations
    DevBuf d_mask_t;                                  // t-major masks (HTDemucs, TFC-TDF)
    DevBuf d_zspec;                                   // HTDemucs spectra
    const float* mono_src = nullptr;                  // the track d_mixn was normalised from
    DevBuf s_mix, s_mask, s_out;   // device staging for stg_separate_host
    // stg_separate_host: a copy stream that brings the masks in batch by batch, and the events
    // the batches' kernels wait for
    cudaStream_t copy_st = nullptr;
    cudaEvent_t copy_fork = nullptr;
    std::vector<cudaEvent_t> copy_ev;
    std::vector<cudaEvent_t> side_ev;   // HTDemucs: per batch, its masks transposed (PlanDevice::side_ev)
    DevBuf dm_out;                 // one channel's result (stg_separate_dual_mono)
    cudaStream_t multi_st = nullptr;   // stg_separate_multi_host: this plan's device's stream
    DevBuf n_in, n_out;            // one batch of network input and output (stg_separate_network)
    RunTiming timing;

    ~stg_plan() {
        for (cudaEvent_t& e : timing.ev)
            if (e) cudaEventDestroy(e);
        if (D.fork) cudaEventDestroy(D.fork);
        if (D.join) cudaEventDestroy(D.join);
        if (D.side) cudaStreamDestroy(D.side);
        for (cudaEvent_t e : copy_ev)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : side_ev)
            if (e) cudaEventDestroy(e);
        if (copy_fork) cudaEventDestroy(copy_fork);
        if (copy_st) cudaStreamDestroy(copy_st);
        if (multi_st) cudaStreamDestroy(multi_st);
    }

    // Device copies of the tables, and the scratch the fused kernel writes.
    void upload_all() {
        const FftTables& t = engine->fft_tables_for(H.g.n_fft);
        upload(d_chunks, H.chunks, "chunk table");
        upload(d_groups, H.groups, "chunk groups");
        upload(d_w, H.W, "weight table");
        upload(d_env, H.env, "envelope table");
        upload(d_envp, H.env_period, "envelope period");
        upload(d_btab, H.btab, "band table");
        upload(d_ebeg, H.ebeg, "band table");
        upload(d_ent, H.ent, "band table");
        upload(d_binv, H.binv, "band table");
        if (!H.bag.empty()) {
            upload(d_bag, H.bag, "bag weights");
            upload(d_bag_tot, H.bag_tot, "bag weights");
            D.bag = d_bag.as<float>();
            D.bag_tot = d_bag_tot.as<float>();
        }
        d_y.reserve(std::max<size_t>(16, H.y_bytes()), "chunk outputs");
        d_tr.reserve(std::max<size_t>(16, H.tr_bytes()), "tile partials");
        if (H.mono_norm) {
            d_mixn.reserve(H.mixn_bytes(), "normalised mix");
            d_mono.reserve(H.mono_bytes(), "mono statistics");
            D.mixn = d_mixn.as<float>();
            D.mono = reinterpret_cast<double*>(d_mono.p);
        }
        if (H.z_per_chunk()) {
            d_zspec.reserve(H.z_bytes(), "segment spectra");
            D.zspec = reinterpret_cast<float4*>(d_zspec.p);
        }
        if (H.mask_planes) {
            d_mask_t.reserve(H.mask_t_bytes(), "t-major masks");
            D.mask_t = reinterpret_cast<float4*>(d_mask_t.p);
            if (H.z_per_chunk() && !D.side) {
                cuda_check(cudaStreamCreateWithFlags(&D.side, cudaStreamNonBlocking), "cudaStreamCreate");
                cuda_check(cudaEventCreateWithFlags(&D.fork, cudaEventDisableTiming), "cudaEventCreate");
                cuda_check(cudaEventCreateWithFlags(&D.join, cudaEventDisableTiming), "cudaEventCreate");
                D.side_ev = &side_ev;
            }
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
        D.env_period = H.env_period.empty() ? nullptr : d_envp.as<float>();
        D.btab = d_btab.as<int2>();
        D.ebeg = d_ebeg.as<int>();
        D.ent = d_ent.as<int2>();
        D.binv = d_binv.as<float>();
        D.win = t.win.as<float>();
        D.tw = t.tw.as<float2>();
        D.Y = d_y.as<float>();
        D.Tr = d_tr.as<float>();
    }

    void run(const float* d_mix, const float* d_mask, float* d_out, cudaStream_t st, const stg_run_options* opt,
             int64_t sample_begin = 0, int64_t sample_end = -1, const std::vector<cudaEvent_t>* ready = nullptr) {
        if (!d_mix || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        H.check_mask(d_mask);
        cuda_check(cudaSetDevice(engine->device), "cudaSetDevice");
        timing.timed = engine->profiling;
        if (timing.timed)
            for (cudaEvent_t& e : timing.ev)
                if (!e) cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        launch_plan(H, D, d_mix, d_mask, d_out, st, opt, &timing, sample_begin, sample_end, ready);
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

namespace stg {

template <class T> bool sized(const T* p) { return p && p->size >= sizeof(uint32_t) * 2; }

inline stg_status guard(stg_engine* e, const std::function<void()>& fn) {
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
// kind: 0 torch.stft, 1 torch.istft, 2 HTDemucs _spec/_ispec, 3 VR's zero-centred stft
inline stg_plan& primitive_plan(stg_engine* e, int kind, int n_fft, int hop, int normalized, int C, int64_t len) {
    const auto key = std::make_tuple(kind, n_fft, hop, normalized, C, len);
    auto it = e->primitives.find(key);
    if (it != e->primitives.end()) return *it->second;
    auto p = std::make_unique<stg_plan>();
    p->engine = e;
    if (kind == 2) build_htdemucs_spec(p->H, C, len);
    else build_torch_stft(p->H, n_fft, hop, normalized != 0, C, len, kind == 1, kind == 3);
    p->upload_all();
    if (e->primitives.size() >= 64) e->primitives.clear();   // keep the cache bounded
    return *(e->primitives[key] = std::move(p));
}

} // namespace stg
