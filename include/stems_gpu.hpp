// stems_gpu.hpp -- a C++ face of stems_gpu_v1.h shaped like stems.cpp's Separator.
//
// Header only, over the C ABI. stems.cpp's separators implement
//     std::vector<float> Separator::separate(const float* mix, int len, const SeparateOptions&)
// (src/separator.h:50-53) with the network inside; here the network is the caller's, so each
// architecture's separate() takes the network's output for the whole track (the plan's mask
// layout, include/stems_gpu_v1.h) beside the same arguments, and returns the same planar
// [sources][channels][len] floats. SeparateOptions carries the reference's fields (shifts,
// overlap, seed, progress, should_cancel; src/separator.h:19-31); a cancelled run throws
// Cancelled and a failure throws Error with the library's status and message, as the
// reference's exceptions map to libstems statuses (src/libstems.cpp:210-218).
//
// Buffers are host memory (the call copies them in batch by batch and the result out,
// stg_separate_host_ex); a plan is built per (length, run options) and kept for the next call
// with the same ones.
#ifndef STEMS_GPU_HPP
#define STEMS_GPU_HPP

#include "stems_gpu_v1.h"

#include <cmath>
#include <cstdint>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace stems_gpu {

class Error : public std::runtime_error {
public:
    Error(stg_status code, const std::string& what) : std::runtime_error(what), code_(code) {}
    stg_status code() const { return code_; }

private:
    stg_status code_;
};

class Cancelled : public Error {
public:
    explicit Cancelled(const std::string& what) : Error(STG_CANCELLED, what) {}
};

// src/separator.h:19-31, plus the batch size the progress and cancellation run at
struct SeparateOptions {
    int shifts = 0;
    float overlap = -1.0f;
    uint32_t seed = 0;
    std::function<void(int, int)> progress;
    std::function<bool()> should_cancel;
    int chunks_per_batch = 1;   // 1: a report and a cancellation point per chunk, as the reference
};

// One CUDA device (stg_engine_create); separators share it.
class Engine {
public:
    explicit Engine(int device = 0) {
        const stg_status st = stg_engine_create(device, &e_);
        if (st != STG_OK) throw Error(st, "stg_engine_create(" + std::to_string(device) + ") failed");
    }
    ~Engine() { stg_engine_destroy(e_); }
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;
    stg_engine* get() const { return e_; }
    std::string last_error() const { return stg_engine_last_error(e_); }

private:
    stg_engine* e_ = nullptr;
};

namespace detail {
inline void check(const Engine& eng, stg_status st, const char* what) {
    if (st == STG_OK) return;
    const std::string msg = std::string(what) + ": " + eng.last_error();
    if (st == STG_CANCELLED) throw Cancelled(msg);
    throw Error(st, msg);
}

// A plan per (length, shifts, overlap, seed), the last one kept.
class PlanCache {
public:
    ~PlanCache() { stg_plan_destroy(plan_); }
    template <class Make> stg_plan* get(int len, const SeparateOptions& o, Make&& make) {
        const auto key = std::make_tuple(len, o.shifts, o.overlap, o.seed);
        if (!plan_ || key != key_) {
            stg_plan_destroy(plan_);
            plan_ = nullptr;
            plan_ = make();
            key_ = key;
        }
        return plan_;
    }

private:
    stg_plan* plan_ = nullptr;
    std::tuple<int, int, float, uint32_t> key_{};
};

inline void trampoline_progress(void* user, int32_t done, int32_t total) {
    const auto* o = static_cast<const SeparateOptions*>(user);
    if (o->progress) o->progress(done, total);
}
inline int32_t trampoline_cancel(void* user) {
    const auto* o = static_cast<const SeparateOptions*>(user);
    return o->should_cancel && o->should_cancel() ? 1 : 0;
}

// The whole separation from host buffers, with the options' callbacks.
inline std::vector<float> run(const Engine& eng, stg_plan* plan, const float* mix, const float* masks,
                              const SeparateOptions& o) {
    stg_plan_info info{};
    info.size = sizeof info;
    check(eng, stg_plan_get_info(plan, &info), "stg_plan_get_info");
    std::vector<float> out((size_t)info.out_floats);
    stg_run_options ro{};
    ro.size = sizeof ro;
    ro.chunks_per_batch = o.chunks_per_batch;
    ro.on_progress = o.progress ? trampoline_progress : nullptr;
    ro.should_cancel = o.should_cancel ? trampoline_cancel : nullptr;
    ro.user = const_cast<SeparateOptions*>(&o);
    check(eng, stg_separate_host_ex(plan, mix, masks, out.data(), nullptr, &ro), "stg_separate_host_ex");
    return out;
}

inline int64_t mask_floats(const Engine& eng, stg_plan* plan) {
    stg_plan_info info{};
    info.size = sizeof info;
    check(eng, stg_plan_get_info(plan, &info), "stg_plan_get_info");
    return info.mask_floats_per_chunk * info.n_chunks;
}
} // namespace detail

// Mel-Band / BS-RoFormer (src/roformer.cpp:436-486). `model` holds the GGUF's values (band
// tables, chunk, n_fft, ...); its overlap, shifts and seed are taken from the options.
class RoFormer {
public:
    RoFormer(Engine& eng, const stg_roformer_config& model)
        : eng_(eng), cfg_(model), sizes_(model.band_sizes, model.band_sizes + model.n_bands) {
        int64_t n = 0;
        for (int32_t s : sizes_) n += s;
        freqs_.assign(model.band_freqs, model.band_freqs + n);
        cfg_.band_sizes = sizes_.data();
        cfg_.band_freqs = freqs_.data();
    }
    // masks: the network's per-band masks of every chunk (stg_plan_info mask floats)
    std::vector<float> separate(const float* mix, int len, const SeparateOptions& opt, const float* masks) {
        return detail::run(eng_, plan(len, opt), mix, masks, opt);
    }
    int64_t mask_floats(int len, const SeparateOptions& opt) { return detail::mask_floats(eng_, plan(len, opt)); }

private:
    stg_plan* plan(int len, const SeparateOptions& opt) {
        return plans_.get(len, opt, [&] {
            stg_roformer_config c = cfg_;
            c.size = sizeof c;
            c.overlap = opt.overlap;
            c.shifts = opt.shifts;
            c.seed = opt.seed;
            stg_plan* p = nullptr;
            detail::check(eng_, stg_plan_roformer(eng_.get(), &c, len, &p), "stg_plan_roformer");
            return p;
        });
    }
    Engine& eng_;
    stg_roformer_config cfg_;
    std::vector<int32_t> sizes_, freqs_;
    detail::PlanCache plans_;
};

// HTDemucs, a single model or a bag (src/htdemucs.cpp:534-644).
class HTDemucs {
public:
    HTDemucs(Engine& eng, const stg_htdemucs_config& model) : eng_(eng), cfg_(model) {
        if (model.bag_weights && model.n_models > 0)
            bag_.assign(model.bag_weights, model.bag_weights + (size_t)model.n_models * model.n_sources);
        cfg_.bag_weights = bag_.empty() ? nullptr : bag_.data();
    }
    // masks: ox = Z * M per segment, every model's after the previous one's
    std::vector<float> separate(const float* mix, int len, const SeparateOptions& opt, const float* masks) {
        return detail::run(eng_, plan(len, opt), mix, masks, opt);
    }
    int64_t mask_floats(int len, const SeparateOptions& opt) { return detail::mask_floats(eng_, plan(len, opt)); }

private:
    stg_plan* plan(int len, const SeparateOptions& opt) {
        return plans_.get(len, opt, [&] {
            stg_htdemucs_config c = cfg_;
            c.size = sizeof c;
            c.overlap = opt.overlap;
            c.shifts = opt.shifts;
            c.seed = opt.seed;
            stg_plan* p = nullptr;
            detail::check(eng_, stg_plan_htdemucs(eng_.get(), &c, len, &p), "stg_plan_htdemucs");
            return p;
        });
    }
    Engine& eng_;
    stg_htdemucs_config cfg_;
    std::vector<float> bag_;
    detail::PlanCache plans_;
};

// TFC-TDF / MDX (src/tfc_tdf.cpp:570-598); the reference refuses shifts for this architecture.
class TFCTDF {
public:
    TFCTDF(Engine& eng, const stg_tfc_config& model) : eng_(eng), cfg_(model) {}
    std::vector<float> separate(const float* mix, int len, const SeparateOptions& opt, const float* masks) {
        if (opt.shifts != 0) throw Error(STG_INTERNAL_ERROR, "tfc_tdf: shifts are unsupported");     // :574
        for (size_t k = 0; k < (size_t)2 * (size_t)(len > 0 ? len : 0); k++)                           // :572-573
            if (!std::isfinite(mix[k])) throw Error(STG_INTERNAL_ERROR, "tfc_tdf: non-finite input");
        return detail::run(eng_, plan(len, opt), mix, masks, opt);
    }
    int64_t mask_floats(int len, const SeparateOptions& opt) { return detail::mask_floats(eng_, plan(len, opt)); }

private:
    stg_plan* plan(int len, const SeparateOptions& opt) {
        return plans_.get(len, opt, [&] {
            stg_tfc_config c = cfg_;
            c.size = sizeof c;
            c.overlap = opt.overlap;
            stg_plan* p = nullptr;
            detail::check(eng_, stg_plan_tfc(eng_.get(), &c, len, &p), "stg_plan_tfc");
            return p;
        });
    }
    Engine& eng_;
    stg_tfc_config cfg_;
    detail::PlanCache plans_;
};

} // namespace stems_gpu

#endif // STEMS_GPU_HPP
