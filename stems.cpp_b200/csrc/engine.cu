// engine.cu -- the C ABI declared in include/stems_gpu_v1.h over the engines and plans of
// engine.h.
#include "engine.h"

#include <cstring>
#include <thread>

#define STG_VERSION_STRING "stems-b200 spectral 0.1 (stems_gpu abi 1)"

using namespace stg;

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
    // a config without the bag-of-models fields is a single model: read it into a full one
    stg_htdemucs_config full{};
    if (c && c->size >= STG_HTDEMUCS_CONFIG_V1_SIZE && c->size < sizeof(full)) {
        std::memcpy(&full, c, c->size);
        full.size = sizeof(full);
        c = &full;
    }
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
    if (!p || !info || info->size < STG_PLAN_INFO_V1_SIZE) return STG_INVALID_ARGUMENT;
    const HostPlan& H = p->H;
    info->arch = H.arch;
    info->n_samples = H.len;
    info->n_channels = H.C;
    info->n_out_sources = H.S_out;
    info->n_chunks = H.n_mask_chunks();
    if (info->size >= sizeof(stg_plan_info)) info->n_models = H.n_models;
    info->n_frames = H.g.T;
    info->mask_floats_per_chunk = H.mask_per_chunk;
    info->out_floats = H.out_floats();
    info->scratch_bytes = (int64_t)(p->d_y.bytes + p->d_tr.bytes + p->d_mixn.bytes + p->d_mono.bytes +
                                    p->d_cac_part.bytes + p->d_cac_stats.bytes + p->d_mask_t.bytes +
                                    p->d_zspec.bytes);
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

STG_API stg_status stg_separate_part(stg_plan* p, const float* d_mix, const float* d_mask, int64_t sample_begin,
                                     int64_t sample_end, float* d_out, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        p->run(d_mix, d_mask, d_out, static_cast<cudaStream_t>(stream), nullptr, sample_begin, sample_end);
    });
}

STG_API stg_status stg_separate_dual_mono(stg_plan* p, const float* d_mix, const float* d_mask, float* d_out,
                                          void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        const HostPlan& H = p->H;
        if (H.C != 1) fail(STG_INVALID_ARGUMENT, "dual mono needs a plan of a one-channel model");
        if (!d_mix || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        const size_t row = sizeof(float) * (size_t)H.len;
        p->dm_out.reserve(row * H.S_out, "dual-mono scratch");
        const int64_t mask_per_channel = H.mask_floats();
        for (int c = 0; c < 2; c++) {                                  // separator.cpp:36-43
            p->run(d_mix + (size_t)c * H.len, d_mask + c * mask_per_channel, p->dm_out.as<float>(), st, nullptr);
            // stem s of this channel to row s * 2 + c of the stereo result
            cuda_check(cudaMemcpy2DAsync(d_out + (size_t)c * H.len, 2 * row, p->dm_out.p, row, row, H.S_out,
                                         cudaMemcpyDeviceToDevice, st), "interleave the channels");
        }
    });
}

// mask batches of stg_separate_host (per bag member)
constexpr int kHostBatches = 8;

namespace {
void separate_host(stg_plan* p, const float* h_mix, const float* h_mask, float* h_out, cudaStream_t st,
                   const stg_run_options* user_opt) {
    if (!h_mix || !h_mask || !h_out) fail(STG_INVALID_ARGUMENT, "null buffer");
    if (user_opt && user_opt->size < sizeof(stg_run_options)) fail(STG_INVALID_ARGUMENT, "options.size is too small");
    cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
    const HostPlan& H = p->H;
    const size_t mix_b = sizeof(float) * (size_t)H.C * H.len;
    const size_t mask_b = sizeof(float) * (size_t)H.mask_floats();
    const size_t out_b = sizeof(float) * (size_t)H.out_floats();
    p->s_mix.reserve(mix_b, "staging");
    p->s_mask.reserve(mask_b, "staging");
    p->s_out.reserve(out_b, "staging");
    // on a failure or a cancellation, no copy may still read or write the caller's host buffers
    // after the return
    try {
        cuda_check(cudaMemcpyAsync(p->s_mix.p, h_mix, mix_b, cudaMemcpyHostToDevice, st), "copy mix in");
        // The masks are most of the bytes (RoFormer cfg1: 934 MB against 21 MB of audio) and
        // the PCIe copy takes some 30 times the kernels. They come in batch by batch on a copy
        // stream, and each batch's kernels (HTDemucs: its transposition, then its back kernel)
        // wait only for their own masks, so the kernels run under the next batches' copies.
        // The batches are launch_plan's: per bag member, runs of `per` chunks.
        const int n = (int)H.chunks.size(), M = H.bag.empty() ? 1 : H.n_models;
        const int per = (user_opt && user_opt->chunks_per_batch > 0) ? std::min(user_opt->chunks_per_batch, n)
                                                                      : (n + std::min(n, kHostBatches) - 1) / std::min(n, kHostBatches);
        const int per_model = (n + per - 1) / per;
        stg_run_options o{};
        if (user_opt) o = *user_opt;
        o.size = sizeof(o);
        o.chunks_per_batch = per;
        if (M * per_model <= 1) {
            cuda_check(cudaMemcpyAsync(p->s_mask.p, h_mask, mask_b, cudaMemcpyHostToDevice, st), "copy masks in");
            p->run(p->s_mix.as<float>(), p->s_mask.as<float>(), p->s_out.as<float>(), st, &o);
        } else {
            if (!p->copy_st) {
                cuda_check(cudaStreamCreateWithFlags(&p->copy_st, cudaStreamNonBlocking), "cudaStreamCreate");
                cuda_check(cudaEventCreateWithFlags(&p->copy_fork, cudaEventDisableTiming), "cudaEventCreate");
            }
            while ((int)p->copy_ev.size() < M * per_model) {
                cudaEvent_t e = nullptr;
                cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
                p->copy_ev.push_back(e);
            }
            const size_t chunk_b = sizeof(float) * (size_t)H.mask_per_chunk;
            // the copies overwrite the staging that the caller's earlier work on st may still read
            cuda_check(cudaEventRecord(p->copy_fork, st), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(p->copy_st, p->copy_fork, 0), "cudaStreamWaitEvent");
            int b = 0;
            for (int m = 0; m < M; m++)
                for (int c0 = 0; c0 < n; c0 += per, b++) {
                    const size_t first = (size_t)m * n + c0, nb = (size_t)std::min(per, n - c0);
                    cuda_check(cudaMemcpyAsync(static_cast<char*>(p->s_mask.p) + chunk_b * first,
                                               reinterpret_cast<const char*>(h_mask) + chunk_b * first, chunk_b * nb,
                                               cudaMemcpyHostToDevice, p->copy_st),
                               "copy masks in");
                    cuda_check(cudaEventRecord(p->copy_ev[b], p->copy_st), "cudaEventRecord");
                }
            p->run(p->s_mix.as<float>(), p->s_mask.as<float>(), p->s_out.as<float>(), st, &o, 0, -1, &p->copy_ev);
        }
        cuda_check(cudaMemcpyAsync(h_out, p->s_out.p, out_b, cudaMemcpyDeviceToHost, st), "copy result out");
        cuda_check(cudaStreamSynchronize(st), "separation");
    } catch (...) {
        cudaStreamSynchronize(st);
        if (p->copy_st) cudaStreamSynchronize(p->copy_st);
        throw;
    }
}
} // namespace

STG_API stg_status stg_separate_host(stg_plan* p, const float* h_mix, const float* h_mask, float* h_out,
                                     void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] { separate_host(p, h_mix, h_mask, h_out, static_cast<cudaStream_t>(stream), nullptr); });
}

STG_API stg_status stg_separate_host_ex(stg_plan* p, const float* h_mix, const float* h_mask, float* h_out,
                                        void* stream, const stg_run_options* opt) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] { separate_host(p, h_mix, h_mask, h_out, static_cast<cudaStream_t>(stream), opt); });
}

// ---- one track over several devices -----------------------------------------------------------
namespace {
// Device d's share of a multi-device separation: output samples [b, e) of every row.
void separate_range(stg_plan* p, const float* h_mix, const float* h_mask, float* h_out, int64_t b, int64_t e) {
    cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
    const HostPlan& H = p->H;
    if (!p->multi_st) cuda_check(cudaStreamCreateWithFlags(&p->multi_st, cudaStreamNonBlocking), "cudaStreamCreate");
    const cudaStream_t st = p->multi_st;
    const size_t mix_b = sizeof(float) * (size_t)H.C * H.len;
    const size_t chunk_b = sizeof(float) * (size_t)H.mask_per_chunk;
    const size_t out_b = sizeof(float) * (size_t)H.out_floats();
    p->s_mix.reserve(mix_b, "staging");
    p->s_mask.reserve(sizeof(float) * (size_t)H.mask_floats(), "staging");
    p->s_out.reserve(out_b, "staging");
    try {
        cuda_check(cudaMemcpyAsync(p->s_mix.p, h_mix, mix_b, cudaMemcpyHostToDevice, st), "copy mix in");
        // the masks of the chunks that reach [b, e), every bag member's, at their own offsets
        const int n = (int)H.chunks.size(), M = H.bag.empty() ? 1 : H.n_models;
        for (const auto& rg : chunks_for(H, b, e))
            for (int m = 0; m < M; m++) {
                const size_t first = (size_t)m * n + rg.first, count = (size_t)(rg.second - rg.first);
                cuda_check(cudaMemcpyAsync(static_cast<char*>(p->s_mask.p) + chunk_b * first,
                                           reinterpret_cast<const char*>(h_mask) + chunk_b * first, chunk_b * count,
                                           cudaMemcpyHostToDevice, st),
                           "copy masks in");
            }
        p->run(p->s_mix.as<float>(), p->s_mask.as<float>(), p->s_out.as<float>(), st, nullptr, b, e);
        // samples [b, e) of every output row
        const size_t row = sizeof(float) * (size_t)H.len;
        cuda_check(cudaMemcpy2DAsync(h_out + b, row, p->s_out.as<float>() + b, row, sizeof(float) * (size_t)(e - b),
                                     (size_t)H.S_out * H.C, cudaMemcpyDeviceToHost, st),
                   "copy the result out");
        cuda_check(cudaStreamSynchronize(st), "separation");
    } catch (...) {
        cudaStreamSynchronize(st);
        throw;
    }
}
} // namespace

STG_API stg_status stg_separate_multi_host(stg_plan* const* plans, int32_t n_plans, const float* h_mix,
                                           const float* h_mask, float* h_out) {
    if (!plans || n_plans < 1 || !plans[0]) return STG_INVALID_ARGUMENT;
    return guard(plans[0]->engine, [&] {
        if (!h_mix || !h_mask || !h_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        const HostPlan& H0 = plans[0]->H;
        for (int d = 0; d < n_plans; d++) {
            if (!plans[d]) fail(STG_INVALID_ARGUMENT, "null plan");
            const HostPlan& H = plans[d]->H;
            if (H.arch != H0.arch || H.len != H0.len || H.C != H0.C || H.S_out != H0.S_out ||
                H.chunks.size() != H0.chunks.size() || H.mask_per_chunk != H0.mask_per_chunk ||
                H.n_models != H0.n_models)
                fail(STG_INVALID_ARGUMENT, "the plans differ: they must share the model configuration and length");
            for (int k = 0; k < d; k++)
                if (plans[k] == plans[d] || plans[k]->engine == plans[d]->engine)
                    fail(STG_INVALID_ARGUMENT, "every plan needs an engine of its own");
        }
        const int64_t len = H0.len;
        std::vector<std::string> errors(n_plans);
        std::vector<stg_status> codes(n_plans, STG_OK);
        std::vector<std::thread> workers;
        workers.reserve(n_plans);
        for (int d = 0; d < n_plans; d++) {
            const int64_t b = len * d / n_plans, e = len * (d + 1) / n_plans;
            if (b >= e) continue;
            workers.emplace_back([&, d, b, e] {
                codes[d] = guard(plans[d]->engine, [&] { separate_range(plans[d], h_mix, h_mask, h_out, b, e); });
                if (codes[d] != STG_OK) errors[d] = plans[d]->engine->last_error;
            });
        }
        for (std::thread& t : workers) t.join();
        for (int d = 0; d < n_plans; d++)
            if (codes[d] != STG_OK) fail(codes[d], "device part " + std::to_string(d) + ": " + errors[d]);
    });
}

// ---- the halves around a real network ----------------------------------------------------
STG_API stg_status stg_plan_network_info(const stg_plan* p, stg_network_info* info) {
    if (!p || !info || info->size < sizeof(stg_network_info)) return STG_INVALID_ARGUMENT;
    info->net_in_floats_per_chunk = p->H.net_in_per_chunk;
    info->net_out_floats_per_chunk = p->H.net_out_per_chunk;
    return STG_OK;
}

namespace {
void no_bag(const HostPlan& H) {
    if (!H.bag.empty())
        fail(STG_UNSUPPORTED, "a bag of models runs through stg_separate or stg_separate_network, not the halves");
}
} // namespace

STG_API stg_status stg_front(stg_plan* p, const float* d_mix, int32_t first, int32_t n, float* d_net_in, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        no_bag(p->H);
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch_front(p->H, p->D, p->front_mix(d_mix, first, st), first, n, d_net_in, st);
    });
}

STG_API stg_status stg_back(stg_plan* p, const float* d_mix, const float* d_net_out, int32_t first, int32_t n,
                            void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        no_bag(p->H);
        cuda_check(cudaSetDevice(p->engine->device), "cudaSetDevice");
        launch_back(p->H, p->D, d_mix, d_net_out, first, n, static_cast<cudaStream_t>(stream));
    });
}

STG_API stg_status stg_finish(stg_plan* p, const float* d_mix, float* d_out, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        no_bag(p->H);
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
        const int G = (int)H.chunks.size(), M = H.bag.empty() ? 1 : H.n_models;
        const int per = per_batch > 0 ? std::min(per_batch, G) : G;
        p->n_in.reserve(std::max<size_t>(16, sizeof(float) * (size_t)H.net_in_per_chunk * per), "network input");
        p->n_out.reserve(std::max<size_t>(16, sizeof(float) * (size_t)H.net_out_per_chunk * per), "network output");
        const auto cancelled = [&] { return opt && opt->should_cancel && opt->should_cancel(opt->user); };
        const int total = H.progress_total > 0 ? H.progress_total : M * G;
        // a bag of models: member m sees chunk indices m * G + k, every member's chunks through
        // the network and the back half before its combine adds its weighted stems
        for (int m = 0; m < M; m++) {
            for (int b0 = 0; b0 < G; b0 += per) {
                if (cancelled()) fail(STG_CANCELLED, "cancelled");
                const int nb = std::min(per, G - b0);
                launch_front(H, p->D, p->front_mix(d_mix, m == 0 ? b0 : 1, st), b0, nb, p->n_in.as<float>(), st);
                if (network(user, m * G + b0, nb, p->n_in.as<float>(), p->n_out.as<float>(), stream) != 0)
                    fail(STG_MODEL_ERROR, "the network callback failed");
                launch_back(H, p->D, d_mix, p->n_out.as<float>(), b0, nb, st);
                if (opt && opt->on_progress) {
                    cuda_check(cudaStreamSynchronize(st), "spectral kernels");
                    const int done = m * G + b0 + nb;
                    const bool final_batch = m == M - 1 && b0 + nb >= G;
                    opt->on_progress(opt->user, final_batch && H.progress_final_total ? total : done, total);
                }
            }
            if (m == M - 1 && H.cancel_after_last && cancelled()) fail(STG_CANCELLED, "cancelled");
            launch_finish(H, p->D, d_mix, d_out, st, m);
        }
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
        p.table = k.table.as<double2>();
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
