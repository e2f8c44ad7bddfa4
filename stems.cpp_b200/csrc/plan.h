// plan.h -- host-side schedule of one separation, independent of where its tables live.
//
// build_* restate, for one model configuration and one track length, what each reference
// separator computes on the host before and around its chunk loop:
//   HTDemucs   src/htdemucs.cpp:534-606  (segments, centre padding, triangular weight)
//   RoFormer   src/roformer.cpp:286-357  (reflect-padded borders, linear fades, tails)
//   TFC-TDF    src/tfc_tdf.cpp:398-495   (UVR trim + np.hanning, or MSST fades)
// into a HostPlan (chunk table, weight tables, window-sum envelope, band tables). The caller
// copies the tables to device memory it owns (engine.cu: buffers per plan; noalloc.cu: a
// static arena) and launch_plan runs the kernels on those copies.
#pragma once
#include "../../include/stems_gpu_v1.h"
#include "kernels.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace stg {

// Errors thrown by the host code and mapped to a stg_status at the C ABI.
struct Failure : std::runtime_error {
    stg_status code;
    Failure(stg_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] void fail(stg_status code, const std::string& msg);
void cuda_check(cudaError_t e, const char* what);

struct HostPlan {
    int arch = 0;
    int64_t len = 0;
    int C = 2, S = 1, S_out = 1;
    int64_t mask_per_chunk = 0;
    std::vector<ChunkDesc> chunks;
    std::vector<ChunkGroup> groups;   // the passes of the shift average (finish_plan: one)
    int shift_mean = 0;               // CombineParams::shift_mean
    FrameGeom g{};
    int K = 16, n_tiles = 0;
    float fwd_scale = 1.0f, inv_scale = 1.0f;
    int reflect_global = 0;        // the default of ChunkDesc::reflect
    int64_t step_out = 1, out_shift = 0, max_out_len = 0;   // out_shift: the default group's
    int nan_to_zero = 0, complement = 0;
    float compensate = 1.0f;
    int zero_dc = 0, dim_f = 0, zero_bins = 0, bin_multi = 0;
    int mono_norm = 0, cac_norm = 0;   // HTDemucs: mono-mix and CaC normalisation
    // HTDemucs bag of models (src/htdemucs.cpp:585-642): every model runs the chunk list on its
    // own masks (model m's after model m - 1's); bag [n_models][S] weights and bag_tot [S] their
    // sums. Empty bag: one model of weight 1 (no accumulation pass).
    int n_models = 1;
    std::vector<float> bag, bag_tot;
    // progress as the reference separator counts it (stg_separate_ex): the total it reports,
    // whether its last report is (total, total) (RoFormer) and whether it polls should_cancel
    // once more after the last chunk (TFC-TDF)
    int progress_total = 0;
    bool progress_final_total = false, cancel_after_last = false;
    // f-major masks (HTDemucs, TFC-TDF): planes and bins per stem; the fused kernel reads
    // them after launch_mask_transpose, 0 planes for the other layouts
    int mask_planes = 0, mask_bins = 0;
    int64_t stem_stride = 0;
    int64_t y_chunk_stride = 0, tr_chunk_stride = 0;
    std::vector<float> W;          // crossfade weight tables (ChunkDesc::w_off)
    std::vector<float> env;        // inverse window-sum envelope of a chunk's output
    std::vector<float> env_period; // env over [env_lo, env_hi), one hop of it (FusedParams)
    int env_lo = 0, env_hi = 0;
    std::vector<int2> btab;        // RoFormer bin table (kernels.h: FusedParams::bin_tab)
    std::vector<int> ebeg;         // RoFormer CSR over bins
    std::vector<int2> ent;
    std::vector<float> binv;
    // the network between the halves: layouts and floats per chunk of its input and output
    int front_layout = FRONT_COMPLEX, back_layout = BACK_COMPLEX;
    int front_bins = 0, back_bins = 0;
    int64_t net_in_per_chunk = 0, net_out_per_chunk = 0;
    bool back_is_fused = false;    // RoFormer: the network outputs a mask; the fused kernel applies it

    bool primitive = false;        // a single-chunk DSP primitive: the output is the chunk's
    int64_t arch_out_len() const { return primitive ? g.Lout : len; }
    // the alignment the masks need: RoFormer's kernel reads a bin's entries as one vector of
    // 2C floats; the other layouts go through the transposition, which reads floats
    int mask_align() const { return arch == ARCH_ROFORMER ? 8 * C : 4; }
    void check_mask(const void* m) const {
        if (reinterpret_cast<uintptr_t>(m) % mask_align())
            fail(STG_INVALID_ARGUMENT, "mask must be " + std::to_string(mask_align()) + "-byte aligned");
    }
    int64_t n_chunks() const { return (int64_t)chunks.size(); }
    // chunks whose masks the caller passes: every model's (the mask buffer's chunks)
    int64_t n_mask_chunks() const { return (int64_t)n_models * (int64_t)chunks.size(); }
    int64_t mask_floats() const { return mask_per_chunk * n_mask_chunks(); }
    int64_t out_floats() const { return (int64_t)S_out * C * len; }
    size_t y_bytes() const { return sizeof(float) * (size_t)y_chunk_stride * chunks.size(); }
    size_t tr_bytes() const { return sizeof(float) * (size_t)tr_chunk_stride * chunks.size(); }
    // scratch of the normalisations: the normalised mix, the mono statistics, the CaC partial
    // sums ([chunk][tile]) and the CaC statistics ([chunk])
    size_t mixn_bytes() const { return mono_norm ? sizeof(float) * (size_t)C * len : 0; }
    size_t mono_bytes() const { return mono_norm ? sizeof(double) * mono_scratch_doubles() : 0; }
    size_t cac_part_bytes() const { return cac_norm ? sizeof(double2) * (size_t)n_tiles * chunks.size() : 0; }
    size_t cac_stats_bytes() const { return cac_norm ? sizeof(double2) * chunks.size() : 0; }
    int64_t mask_t_per_chunk() const { return mask_planes ? (int64_t)S * g.T * mask_bins : 0; }   // float4
    // HTDemucs: each segment's spectra once, t-major (FRONT_ZSPEC), for the back kernel
    int64_t z_per_chunk() const { return arch == ARCH_HTDEMUCS && !primitive ? (int64_t)g.T * (g.n_fft / 2) : 0; }
    size_t z_bytes() const { return sizeof(float4) * (size_t)z_per_chunk() * chunks.size(); }
    size_t mask_t_bytes() const { return sizeof(float4) * (size_t)mask_t_per_chunk() * chunks.size(); }
};

// Where the device copies of a plan's tables and scratch live.
struct PlanDevice {
    const ChunkDesc* chunks = nullptr;
    const ChunkGroup* groups = nullptr;
    const float* W = nullptr;
    const float* env = nullptr;
    const float* env_period = nullptr;
    const int2* btab = nullptr;
    const int* ebeg = nullptr;
    const int2* ent = nullptr;
    const float* binv = nullptr;
    const float* win = nullptr;    // periodic Hann [n_fft]
    const float2* tw = nullptr;    // FFT twiddles (fft_tables)
    float* Y = nullptr;            // scratch: chunk outputs
    float* Tr = nullptr;           // scratch: tile-boundary partials
    float* mixn = nullptr;         // scratch: the mono-normalised mix (HostPlan::mono_norm)
    double* mono = nullptr;        // scratch: mono statistics, mean and std at [0], [1]
    double2* cac_part = nullptr;   // scratch: CaC partial sums (HostPlan::cac_norm)
    double2* cac_stats = nullptr;  // scratch: per-chunk CaC (mean, std)
    float4* mask_t = nullptr;      // scratch: t-major masks (HostPlan::mask_planes)
    float4* zspec = nullptr;       // scratch: HTDemucs spectra (HostPlan::z_per_chunk)
    const float* bag = nullptr;    // HostPlan::bag and bag_tot (null without a bag)
    const float* bag_tot = nullptr;
    // HTDemucs: a second stream on which every segment's mask transposition runs beside the
    // normalisation and the front kernel, joined before the first back kernel (null: the
    // transpositions run in order on the caller's stream)
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    std::vector<cudaEvent_t>* side_ev = nullptr;   // one per batch: its transposition done
};

void build_htdemucs(HostPlan& P, const stg_htdemucs_config& c, int64_t len);
// Single-chunk plans of the DSP primitives: torch.stft / torch.istft (src/stft.h:146-197) of
// `len` samples (the istft's output length), HTDemucs _spec/_ispec (src/stft.h:79-140).
// For the inverse, len = hop * (frames - 1), the istft's output length. zero_pad: VR's
// zero-centred forward STFT (src/vr_dsp.h:43-62) instead of torch's reflect padding; VR's
// inverse (src/vr_dsp.h:64-88) is torch's.
void build_torch_stft(HostPlan& P, int n_fft, int hop, bool normalized, int n_channels, int64_t len,
                      bool inverse, bool zero_pad = false);
void build_htdemucs_spec(HostPlan& P, int n_channels, int64_t len);
void build_roformer(HostPlan& P, const stg_roformer_config& c, int64_t len);
void build_tfc(HostPlan& P, const stg_tfc_config& c, int64_t len);

// The window and twiddle tables the fused kernel reads for n_fft (host copies).
void fft_tables(int n_fft, std::vector<float>& win, std::vector<float2>& tw);
// The per-pass twiddles of a radix plan of n_fft points (fft.cuh: twiddle_index).
void fft_twiddles(int n_fft, const std::vector<int>& radices, std::vector<float2>& tw);

// Optional timing of one run: events recorded on the run's stream around the kernels.
struct RunTiming {
    // run start, first fused launch, combine start, combine end
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    bool timed = false;
    int launches = 0;
};

// The chunks whose outputs reach output samples [b, e), as index ranges of the plan's chunk
// list (one per chunk group, adjacent ones merged).
std::vector<std::pair<int, int>> chunks_for(const HostPlan& P, int64_t b, int64_t e);

// Run a separation on device buffers with the plan's device tables: the fused kernel over
// chunk batches (progress and cancellation between batches), then the combine.
// With a sample range, only the chunks reaching output samples [sample_begin, sample_end) run
// and only those samples of every output row are written (end < 0: the whole track).
// ready, when given, streams the masks in: batch k of the run (the batches of
// opt->chunks_per_batch, in order) reads its masks only after (*ready)[k] has completed.
void launch_plan(const HostPlan& P, const PlanDevice& D, const float* d_mix, const float* d_mask,
                 float* d_out, cudaStream_t st, const stg_run_options* opt, RunTiming* timing,
                 int64_t sample_begin = 0, int64_t sample_end = -1,
                 const std::vector<cudaEvent_t>* ready = nullptr);

// The halves around a real network, on chunks [first, first + n): the front writes the
// network's input (net_in_per_chunk floats per chunk) into d_net_in; the back reads its
// output (net_out_per_chunk floats per chunk) and leaves the chunks' results in the scratch;
// finish (the combine) produces the separation once every chunk went through the back.
// With HostPlan::mono_norm, d_mix of launch_front and launch_back is the normalised mix that
// normalise_mix left in D.mixn; normalise_mix returns the mix the kernels read.
const float* normalise_mix(const HostPlan& P, const PlanDevice& D, const float* d_mix, cudaStream_t st);
void launch_front(const HostPlan& P, const PlanDevice& D, const float* d_mix, int first, int n,
                  float* d_net_in, cudaStream_t st);
void launch_back(const HostPlan& P, const PlanDevice& D, const float* d_mix, const float* d_net_out, int first,
                 int n, cudaStream_t st);
// model: the bag member whose chunk outputs the scratch holds (its weights accumulate into d_out,
// the last one divides and maps back); ignored without a bag.
void launch_finish(const HostPlan& P, const PlanDevice& D, const float* d_mix, float* d_out, cudaStream_t st,
                   int model = 0);

} // namespace stg
