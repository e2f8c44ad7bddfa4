/* stems_gpu_v1.h -- C ABI of the B200 spectral front/back end of stems.cpp.
 *
 * This library replaces the host-side spectral path of stems.cpp's separators with CUDA
 * kernels for sm_100a. It sits under the reference's unchanged outer contract
 * (src/libstems_v1.h: stems_get_api(1)->separate) and behind the internal seam
 * Separator::separate(const float* mix, int len, const SeparateOptions&)
 * (src/separator.h:53), where each architecture's separate() runs
 *
 *     chunk scheduler -> STFT -> [network] -> mask / unpack -> iSTFT -> overlap-add
 *
 * The network is out of scope: a caller-supplied mask buffer stands in for its output, in
 * exactly the layout the reference's network produces (see each plan's mask layout).
 *
 * Conventions (same as libstems_v1.h):
 *   - every function returns a stg_status; the codes are stems_status_v1's (0 = OK);
 *   - audio is planar float: samples[channel * n_samples + sample];
 *   - results are planar [source][channel][sample];
 *   - an engine is bound to one CUDA device and is not reentrant (one per host thread);
 *   - "d_" pointers are device memory owned by the caller, "h_" pointers host memory;
 *     `stream` is a cudaStream_t (NULL = the legacy default stream);
 *   - size-tagged structs: zero them, set .size = sizeof(struct), fill the fields.
 */
#ifndef STEMS_GPU_V1_H
#define STEMS_GPU_V1_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#  define STG_API __attribute__((visibility("default")))
#else
#  define STG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t stg_status;
enum {
    STG_OK               = 0,   /* STEMS_STATUS_OK_V1 */
    STG_INVALID_ARGUMENT = 1,   /* STEMS_STATUS_INVALID_ARGUMENT_V1 */
    STG_UNSUPPORTED      = 2,   /* a configuration the kernels do not implement */
    STG_CANCELLED        = 3,   /* STEMS_STATUS_CANCELLED_V1 */
    STG_MODEL_ERROR      = 4,   /* STEMS_STATUS_MODEL_ERROR_V1: inconsistent model configuration */
    STG_IO_ERROR         = 5,
    STG_OUT_OF_MEMORY    = 6,   /* STEMS_STATUS_OUT_OF_MEMORY_V1 */
    STG_INTERNAL_ERROR   = 7    /* STEMS_STATUS_INTERNAL_ERROR_V1: CUDA errors and the rest */
};

typedef struct stg_engine stg_engine;
typedef struct stg_plan stg_plan;

/* ---- library and engine ------------------------------------------------------------------ */

/* Version string, like libstems' runtime_version (src/libstems.cpp:16, 39). */
STG_API const char* stg_version(void);

/* Number of CUDA devices visible, or a negative value when the CUDA runtime fails. */
STG_API int stg_device_count(void);

/* One engine per device and host thread. Replaces the per-model backend handle that
 * HTDemucs/RoFormer/TFCTDF::Impl hold (src/htdemucs.cpp:309, src/roformer.cpp:65,
 * src/tfc_tdf.cpp:75) for the spectral path. */
STG_API stg_status stg_engine_create(int device, stg_engine** out_engine);
STG_API void stg_engine_destroy(stg_engine* engine);
/* The message of the engine's last failure ("" after success). Borrowed. */
STG_API const char* stg_engine_last_error(const stg_engine* engine);

/* Kernel timing, the counterpart of the reference's wall-clock timers
 * (tools/stems-split.cpp:94-97): when enabled, every run records CUDA events around its
 * kernels on the run's stream; stg_plan_last_timing waits for the last run and returns the
 * milliseconds of the kernels before the combine (the fused spectral kernels and their
 * preparation) and of the combine kernel. */
STG_API stg_status stg_engine_set_profiling(stg_engine* engine, int32_t enabled);
STG_API stg_status stg_plan_last_timing(stg_plan* plan, float* fused_ms, float* combine_ms,
                                        int32_t* kernel_launches);
/* The same run split three ways: prep_ms = the kernels before the first fused launch (HTDemucs
 * normalisations, the first batch's mask transposition), fused_ms = from the first fused launch
 * to the combine (later batches' transpositions included), combine_ms = the combine. No
 * reference counterpart beyond the timers of stg_plan_last_timing. */
STG_API stg_status stg_plan_last_timing_detail(stg_plan* plan, float* prep_ms, float* fused_ms,
                                               float* combine_ms, int32_t* kernel_launches);

/* ---- model configurations (the GGUF metadata the reference reads) ------------------------ */

/* HTDemucs (src/htdemucs.cpp:478-500; n_fft 4096 and hop 1024 are fixed, :35-36).
 * The reference always applies both normalisations; 0 turns one off (the stand-in network
 * then sees the raw spectrogram, or the raw mix). */
typedef struct {
    uint32_t size;
    int32_t n_channels;      /* stems.audio_channels (2) */
    int32_t n_sources;       /* len(stems.sources) (4 or 6) */
    int32_t segment;         /* segment_samples() = seg_num * sr / seg_den (343980) */
    float overlap;           /* SeparateOptions.overlap; < 0 = 0.25 */
    int32_t mono_norm;       /* 1: the mix / mono std normalisation and the stems' inverse
                                (src/htdemucs.cpp:539-549, 638-642) */
    int32_t cac_norm;        /* 1: per-segment mean / std of the CaC spectrogram around the
                                network (src/htdemucs.cpp:434-436, 466-469) */
    int32_t shifts;          /* SeparateOptions.shifts: random time shifts averaged, 0 = one pass
                                (src/htdemucs.cpp:610-626); every shift's segments are chunks of
                                the plan, shift by shift */
    uint32_t seed;           /* SeparateOptions.seed: std::mt19937 seed of the shift offsets */
    int32_t sample_rate;     /* the model's sample rate (max shift = sample_rate / 2); 0 = 44100 */
    /* Bag of models (stems.n_models, stems.bag_weights; src/htdemucs.cpp:585-642): every model
     * runs the whole separation (shifts included) on the same normalised mix with its own masks;
     * stem s of the result is sum_m bag_weights[m][s] * (model m's stem s), summed in model
     * order, divided by sum_m bag_weights[m][s], then mapped back by the mono statistics once.
     * The masks of model m follow those of model m - 1. n_models <= 0 with bag_weights NULL:
     * one model of weight 1, the plain path. These two fields are optional: a config whose
     * size is STG_HTDEMUCS_CONFIG_V1_SIZE (without them) is a single model. */
    int32_t n_models;
    const float* bag_weights;  /* [n_models][n_sources], or NULL for all 1 */
} stg_htdemucs_config;
/* The size of stg_htdemucs_config without the bag-of-models fields (older callers). */
#define STG_HTDEMUCS_CONFIG_V1_SIZE ((uint32_t)offsetof(stg_htdemucs_config, n_models))

/* Mel-Band / BS-RoFormer (src/roformer.cpp:360-412). */
typedef struct {
    uint32_t size;
    int32_t n_channels;      /* 2 */
    int32_t n_stems;         /* the model's own stems */
    int32_t n_fft;           /* roformer.stft_n_fft (2048) */
    int32_t hop;             /* roformer.stft_hop_length (441) */
    int32_t normalized;      /* roformer.stft_normalized */
    int32_t zero_dc;         /* roformer.zero_dc */
    int32_t chunk;           /* roformer.chunk_size (352800) */
    int32_t num_overlap;     /* roformer.num_overlap */
    float overlap;           /* SeparateOptions.overlap; < 0 = chunk / num_overlap */
    int32_t n_bands;
    const int32_t* band_sizes;   /* roformer.band_sizes [n_bands] */
    const int32_t* band_freqs;   /* roformer.band_freqs [sum band_sizes] */
    int32_t complement;      /* stems.complement present: append mix - first stem */
    int32_t shifts;          /* SeparateOptions.shifts (src/roformer.cpp:456-478); every shift's
                                chunks are chunks of the plan, shift by shift */
    uint32_t seed;           /* SeparateOptions.seed: std::mt19937 seed of the shift offsets */
    int32_t sample_rate;     /* the model's sample rate (max shift = sample_rate / 2); 0 = 44100 */
} stg_roformer_config;

/* TFC-TDF / MDX (src/tfc_tdf.cpp:498-553). */
typedef struct {
    uint32_t size;
    int32_t n_stems;
    int32_t n_fft;           /* tfc_tdf.n_fft (7680 for Kim_Vocal_2) */
    int32_t hop;             /* tfc_tdf.hop */
    int32_t dim_f;           /* tfc_tdf.dim_f */
    int32_t dim_t;           /* tfc_tdf.dim_t */
    int32_t zero_bins;       /* tfc_tdf.zero_bins (uvr_mdx) */
    int32_t chunking;        /* 0 = "uvr_mdx", 1 = "msst" (tfc_tdf.chunking) */
    int32_t num_overlap;     /* tfc_tdf.num_overlap (msst) */
    float overlap;           /* SeparateOptions.overlap; < 0 = the model default */
    float compensate;        /* tfc_tdf.compensate */
    int32_t complement;      /* stems.complement present: append mix - sum of stems */
} stg_tfc_config;

/* ---- plans: one model configuration and one track length ---------------------------------- */

/* Build the chunk schedule and every table of one separation. Replaces the set-up half of
 * HTDemucs::separate (src/htdemucs.cpp:534-583), RoFormer::Impl::demix (src/roformer.cpp:
 * 286-316) and TFCTDF::Impl::demix_uvr / demix_msst (src/tfc_tdf.cpp:398-410, 434-460).
 * Fails with STG_INVALID_ARGUMENT for the inputs the reference rejects (empty input,
 * overlap >= 1, reflect pads longer than the signal) and STG_UNSUPPORTED for an n_fft the
 * kernels do not implement (2048 and 4096; 7680 for TFC-TDF). */
STG_API stg_status stg_plan_htdemucs(stg_engine* engine, const stg_htdemucs_config* config,
                                     int64_t n_samples, stg_plan** out_plan);
STG_API stg_status stg_plan_roformer(stg_engine* engine, const stg_roformer_config* config,
                                     int64_t n_samples, stg_plan** out_plan);
STG_API stg_status stg_plan_tfc(stg_engine* engine, const stg_tfc_config* config,
                                int64_t n_samples, stg_plan** out_plan);
STG_API void stg_plan_destroy(stg_plan* plan);

typedef struct {
    uint32_t size;
    int32_t arch;                  /* 0 RoFormer, 1 HTDemucs, 2 TFC-TDF */
    int64_t n_samples;             /* per channel, in and out */
    int32_t n_channels;
    int32_t n_out_sources;         /* stems in the result, complement included */
    int64_t n_chunks;              /* segments (HTDemucs) or chunks: the reference's passes
                                      (a bag of models: every model's, n_models x per model) */
    int64_t n_frames;              /* STFT frames per chunk */
    int64_t mask_floats_per_chunk; /* the stand-in network output of one chunk */
    int64_t out_floats;            /* n_out_sources * n_channels * n_samples */
    int64_t scratch_bytes;         /* device scratch the plan holds */
    int32_t n_models;              /* models of an HTDemucs bag (1 otherwise); optional field */
} stg_plan_info;
/* The size of stg_plan_info without n_models (older callers). */
#define STG_PLAN_INFO_V1_SIZE ((uint32_t)offsetof(stg_plan_info, n_models))
STG_API stg_status stg_plan_get_info(const stg_plan* plan, stg_plan_info* info);

/* Layout of one chunk's mask (the network output the plan consumes):
 *   HTDemucs  [S][2C][F = 2048][T] float: plane 2c = real, 2c+1 = imaginary part of a
 *             complex multiplier of the CaC spectrogram (the network's `ox`,
 *             src/htdemucs.cpp:450-452 and 463-469, with ox = Z * M);
 *   RoFormer  [S][sum_b din_b * T] float, band-major: band b is a [T][din_b] block,
 *             din_b = size_b * C * 2, entry (j*C + c)*2 + {re, im}: the network's per-band
 *             masks (src/roformer.cpp:251-269);
 *   TFC-TDF   [4S][dim_f][T] float: a real multiplier of the CaC input (the network's
 *             output y = in * mask, src/tfc_tdf.cpp:377-387).
 * Chunks follow each other. */

/* Run the whole separation on device buffers: d_mix [C][n], d_mask [n_chunks][mask per
 * chunk], d_out [n_out_sources][C][n]. Asynchronous on `stream`. Replaces the scheduler
 * loops and the spectral glue of HTDemucs::separate (src/htdemucs.cpp:589-606, with
 * Impl::run :419-475), RoFormer::Impl::demix (src/roformer.cpp:317-350, with Impl::run
 * :217-283) and TFCTDF demix_uvr / demix_msst (src/tfc_tdf.cpp:411-428, 461-494, with
 * run_chunk :362-391), plus the complement and compensation epilogues
 * (src/roformer.cpp:481-485, src/tfc_tdf.cpp:586-596). d_mask must be 16-byte aligned. */
STG_API stg_status stg_separate(stg_plan* plan, const float* d_mix, const float* d_mask,
                                float* d_out, void* stream);

/* The same on host buffers: copies the mix and the masks in, runs, copies the result out,
 * and returns when the result is in h_out. This is the end-to-end call a host such as
 * libstems' separate (src/libstems.cpp:135-219) makes. The masks come in up to eight batches
 * of chunks on a stream of the plan's own, each batch's kernels running as soon as its masks
 * have arrived; pinned host buffers let the copies run at full PCIe speed. */
STG_API stg_status stg_separate_host(stg_plan* plan, const float* h_mix, const float* h_mask,
                                     float* h_out, void* stream);

/* Progress and cancellation between chunk batches, like SeparateOptions.progress /
 * should_cancel (src/separator.h:28-31): on_progress(user, done, total) after each batch,
 * should_cancel(user) before each batch (non-zero abandons the job with STG_CANCELLED). */
typedef void (*stg_progress_fn)(void* user, int32_t done, int32_t total);
typedef int32_t (*stg_cancel_fn)(void* user);
typedef struct {
    uint32_t size;
    int32_t chunks_per_batch;      /* <= 0: everything in one batch */
    stg_progress_fn on_progress;
    stg_cancel_fn should_cancel;
    void* user;
} stg_run_options;
STG_API stg_status stg_separate_ex(stg_plan* plan, const float* d_mix, const float* d_mask,
                                   float* d_out, void* stream, const stg_run_options* options);

/* The (done, total) pairs follow each reference separator's own counting, so a caller's
 * progress bar moves as it does with the reference (with chunks_per_batch = 1, pair for pair):
 *   HTDemucs  total = n_models * max(1, shifts) * ceil(n_samples / stride); after every batch
 *             (done chunks, total) (src/htdemucs.cpp:576-577, 602); with shifts the views are
 *             longer than the track, so done can pass total, as in the reference;
 *   RoFormer  total = max(1, shifts) * the chunks of one pass over n_samples; after every batch
 *             but the last (done chunks, total), after the last (total, total)
 *             (src/roformer.cpp:444-451, 479);
 *   TFC-TDF   total = the chunks; after every batch (done chunks, total) (src/tfc_tdf.cpp:
 *             411, 425, 577-579), and should_cancel is polled once more after the last batch,
 *             as the reference's tick after its last chunk does.
 * should_cancel is polled before every batch. A cancelled run returns STG_CANCELLED having
 * enqueued no further kernel; d_out is then incomplete. */

/* stg_separate_host with progress and cancellation (options may be NULL). On STG_CANCELLED
 * (and on any failure) it returns only after every copy it enqueued from h_mix / h_mask has
 * finished; the result is not copied, so h_out is left as it was. */
STG_API stg_status stg_separate_host_ex(stg_plan* plan, const float* h_mix, const float* h_mask,
                                        float* h_out, void* stream, const stg_run_options* options);

/* Output samples [sample_begin, sample_end) of every output row of the separation, running only
 * the chunks that reach them: the same floats stg_separate writes there (each sample sums the
 * same chunks in the same order). d_mix, d_mask and d_out are the whole track's buffers; other
 * samples of d_out are left as they are. One track split over several GPUs by sample ranges
 * needs no exchange between them; the chunks at a range's edges run on both neighbours. No
 * reference counterpart: the reference separates a track in one call. */
STG_API stg_status stg_separate_part(stg_plan* plan, const float* d_mix, const float* d_mask,
                                     int64_t sample_begin, int64_t sample_end, float* d_out, void* stream);

/* One track over several GPUs of this node, from host buffers, in one call: plans[d] (one per
 * device, each from an engine of its own, all of the same model configuration and length)
 * writes output samples [n * d / n_plans, n * (d + 1) / n_plans) of every output row, running
 * only the chunks that reach them (stg_separate_part); the chunks at a range's edge run on
 * both neighbours, so nothing is exchanged and every sample is the float one GPU writes. One
 * host thread and one stream per device; each copies in the mix and the masks of its own
 * chunks and copies its range of h_out back. Returns when h_out holds the whole result, or the
 * first failure's status after every device has stopped. Pinned host buffers let the devices'
 * copies run side by side. No reference counterpart: libstems separates a track on one device
 * (src/libstems.cpp:188); this is the node-wide form of that call. */
STG_API stg_status stg_separate_multi_host(stg_plan* const* plans, int32_t n_plans, const float* h_mix,
                                           const float* h_mask, float* h_out);

/* DualMono (src/separator.cpp:15-47): a plan of a one-channel model (n_channels 1) run on
 * each channel of a stereo mix on its own, the results interleaved into planar stereo.
 * d_mix [2][n_samples]; d_mask holds the left channel's masks (stg_plan_info's
 * mask_floats_per_chunk x n_chunks floats), then the right channel's; d_out
 * [n_out_sources][2][n_samples]. The plan keeps one channel's result as scratch. */
STG_API stg_status stg_separate_dual_mono(stg_plan* plan, const float* d_mix, const float* d_mask,
                                          float* d_out, void* stream);

/* ---- the halves around a real network --------------------------------------------------- */

/* The same separation with the network between the halves, as the reference runs it: for
 * each batch of chunks, the front half writes the network's input, the network runs, the
 * back half reads the network's output; once every chunk went through the back half,
 * stg_finish overlap-adds the chunks into the result.
 *   HTDemucs  input  in_x  [2C][2048][T] float CaC planes (src/htdemucs.cpp:423-433), with
 *                    cac_norm normalised by the segment's mean / std (:434-436);
 *             output ox    [S][2C][2048][T] (:463-469), with cac_norm mapped back by the
 *                    segment's std and mean (:469) in the back half.
 *             With mono_norm, the call with first_chunk 0 normalises the whole track into
 *             the plan's scratch (:539-549) and later calls read that copy: batches start at
 *             chunk 0 with the same d_mix; stg_finish maps the stems back (:638-642).
 *   RoFormer  input  feat  [sum_b din_b * T] band-major (src/roformer.cpp:226-241);
 *             output the per-band masks, the plan's mask layout (:251-269).
 *   TFC-TDF   input  in    [4][dim_f][T], bins below zero_bins 0 (src/tfc_tdf.cpp:366-376);
 *             output y     [4S][dim_f][T] (:381-387).
 * Chunk k of a batch starting at first_chunk sits at k * (floats per chunk) in the buffers. */
typedef struct {
    uint32_t size;
    int64_t net_in_floats_per_chunk;
    int64_t net_out_floats_per_chunk;
} stg_network_info;
STG_API stg_status stg_plan_network_info(const stg_plan* plan, stg_network_info* info);
STG_API stg_status stg_front(stg_plan* plan, const float* d_mix, int32_t first_chunk, int32_t n_chunks,
                             float* d_net_in, void* stream);
STG_API stg_status stg_back(stg_plan* plan, const float* d_mix, const float* d_net_out,
                            int32_t first_chunk, int32_t n_chunks, void* stream);
STG_API stg_status stg_finish(stg_plan* plan, const float* d_mix, float* d_out, void* stream);

/* The whole loop with the network as a callback, run on the calling thread between the
 * halves: network(user, first_chunk, n_chunks, d_net_in, d_net_out, stream) enqueues the
 * network on `stream` and returns 0, or non-zero to fail the separation with
 * STG_MODEL_ERROR. The batch buffers belong to the plan. Progress and cancellation as in
 * stg_separate_ex (options may be NULL). Replaces the chunk loops of the separators with the
 * graph call in the middle (src/htdemucs.cpp:589-606, src/roformer.cpp:317-341,
 * src/tfc_tdf.cpp:411-424). */
typedef int32_t (*stg_network_fn)(void* user, int32_t first_chunk, int32_t n_chunks, const float* d_net_in,
                                  float* d_net_out, void* stream);
STG_API stg_status stg_separate_network(stg_plan* plan, const float* d_mix, float* d_out,
                                        int32_t chunks_per_batch, stg_network_fn network, void* user,
                                        const stg_run_options* options, void* stream);

/* ---- the request's audio in and the stems out (src/libstems.cpp:160-199) ------------------ */

/* Samples per channel after resampling n samples from src_rate to dst_rate:
 * llround(n * dst_rate / src_rate), or n at the same rate (src/audio.h:20-21). */
STG_API int64_t stg_resampled_length(int64_t n_samples, int32_t src_rate, int32_t dst_rate);

/* The request's audio in the model's format, as libstems.cpp:160-169 makes it: d_in holds
 * n_samples frames of n_channels channels, interleaved (interleaved = 1) or planar; d_out
 * receives planar [model_channels][stg_resampled_length(n_samples, sample_rate, model_rate)]:
 * channels converted by to_channels (mono duplicated, extra channels dropped,
 * src/audio.h:59-68), then resampled to model_rate by the Kaiser-windowed sinc of
 * resample_planar (src/audio.h:17-56) when the rates differ. Sample for sample the floats
 * the reference computes. Asynchronous on `stream`. */
STG_API stg_status stg_prepare_input(stg_engine* engine, const float* d_in, int32_t interleaved,
                                     int64_t n_samples, int32_t n_channels, int32_t sample_rate,
                                     int32_t model_channels, int32_t model_rate, float* d_out,
                                     void* stream);

/* The stems back at the request's rate (libstems.cpp:189-199): d_stems planar [rows][len] at
 * model_rate -> d_out planar [rows][n_samples] at sample_rate, resampled when the rates
 * differ and then pinned to n_samples (cut, or zero-filled past the resampled end). */
STG_API stg_status stg_restore_output(stg_engine* engine, const float* d_stems, int32_t rows,
                                      int64_t len, int32_t model_rate, int32_t sample_rate,
                                      int64_t n_samples, float* d_out, void* stream);

/* ---- VR (src/vr.cpp:215-269, 349-377; src/vr_dsp.h:43-125) -------------------------------- */

/* One band of a VR model (vr.band.<i>.* of the GGUF, src/vr.cpp:306-318), lowest rate first.
 * -1 in hpf_start / lpf_start: no filter. */
typedef struct {
    int32_t sample_rate, hop, n_fft, crop_start, crop_stop;
    int32_t hpf_start, hpf_stop, lpf_start, lpf_stop;
} stg_vr_band;
/* A resampling FIR of the model (resample.<src>.<dst>, src/vr.cpp:320-327). */
typedef struct {
    int32_t src_rate, dst_rate, n_taps;
    const float* taps;
} stg_vr_fir;
typedef struct {
    uint32_t size;
    int32_t sample_rate;        /* stems.samplerate: the last band's rate */
    int32_t bins;               /* vr.bins */
    int32_t pre_filter_start;   /* vr.pre_filter_start / stop */
    int32_t pre_filter_stop;
    int32_t n_bands;            /* 1..16 */
    const stg_vr_band* bands;
    int32_t n_firs;             /* every rate pair the chain crosses, both directions */
    const stg_vr_fir* firs;
} stg_vr_config;
typedef struct stg_vr_plan stg_vr_plan;

/* A VR separation of n_samples stereo samples at sample_rate, checked as src/vr.cpp:296-327
 * checks a model (STG_MODEL_ERROR) and as synthesize() checks the band lengths. Band n_fft
 * 320, 512, 640, 960, 1024 or 2048 with hop <= n_fft / 2 (else STG_UNSUPPORTED). */
STG_API stg_status stg_plan_vr(stg_engine* engine, const stg_vr_config* config, int64_t n_samples,
                               stg_vr_plan** out_plan);
STG_API void stg_vr_plan_destroy(stg_vr_plan* plan);
/* T, the frames of the spectrum; the network's input and mask are [2][bins + 1][T]. */
STG_API stg_status stg_vr_plan_frames(const stg_vr_plan* plan, int64_t* n_frames);
/* spectrum() (src/vr.cpp:215-239) of d_mix [2][n_samples]: kept in the plan for stg_vr_back;
 * |spec| into d_mag [2][bins+1][T] and its peak into d_peak (one float) when not NULL, the
 * network's input before the patching (vr.cpp:357-366). */
STG_API stg_status stg_vr_front(stg_vr_plan* plan, const float* d_mix, float* d_mag, float* d_peak,
                                void* stream);
/* The two stems from the last front's spectrum and the network's mask [2][bins+1][T]:
 * spec x mask and spec x (1 - mask), each synthesised (vr.cpp:241-269, 368-377) into
 * d_out [2 stems][2][n_samples]. */
STG_API stg_status stg_vr_back(stg_vr_plan* plan, const float* d_mask, float* d_out, void* stream);
/* stg_vr_front without outputs, then stg_vr_back: the whole separation with the mask as the
 * stand-in for the network. */
STG_API stg_status stg_separate_vr(stg_vr_plan* plan, const float* d_mix, const float* d_mask,
                                   float* d_out, void* stream);

/* ---- model configurations from GGUF files ----------------------------------------------- */

/* A model file's metadata, read without ggml and without its weights: what the separators'
 * constructors read (src/htdemucs.cpp:478-500, src/roformer.cpp:360-412,
 * src/tfc_tdf.cpp:498-553, src/vr.cpp:296-327) and VR's resampling FIRs. Host only; needs
 * no GPU. `message` (optional) receives the reason for a failure: STG_IO_ERROR when the file
 * cannot be opened, STG_MODEL_ERROR for a file that is not GGUF or lacks a key. */
typedef struct stg_model stg_model;
STG_API stg_status stg_model_open(const char* gguf_path, stg_model** out_model, char* message,
                                  size_t message_size);
STG_API void stg_model_close(stg_model* model);
/* general.architecture: "htdemucs", "mel_band_roformer", "bs_roformer", "tfc_tdf" or
 * "vr_cascaded". Borrowed until stg_model_close. */
STG_API const char* stg_model_architecture(const stg_model* model);
/* stems.samplerate, or 0 when absent. */
STG_API int32_t stg_model_sample_rate(const stg_model* model);
/* The configuration of the model's architecture, with the reference's defaults for the run
 * options (overlap < 0, no shifts, HTDemucs' normalisations on); set config->size first.
 * Arrays the configs point to (band tables, VR bands and FIRs) belong to the model. */
STG_API stg_status stg_model_htdemucs_config(const stg_model* model, stg_htdemucs_config* config,
                                             char* message, size_t message_size);
STG_API stg_status stg_model_roformer_config(const stg_model* model, stg_roformer_config* config,
                                             char* message, size_t message_size);
STG_API stg_status stg_model_tfc_config(const stg_model* model, stg_tfc_config* config, char* message,
                                        size_t message_size);
STG_API stg_status stg_model_vr_config(const stg_model* model, stg_vr_config* config, char* message,
                                       size_t message_size);

/* ---- the DSP primitives of src/stft.h on the device -------------------------------------- */

/* torch.stft (src/stft.h:146-164) of each channel: periodic Hann, centre reflect pad,
 * onesided, 1/sqrt(n_fft) when normalized. d_x [C][n_samples]; d_spec complex (interleaved
 * float re, im) [C][n_fft/2 + 1][T], T = n_samples / hop + 1. n_fft 2048, 4096 or 7680. */
STG_API stg_status stg_torch_stft(stg_engine* engine, int32_t n_fft, int32_t hop, int32_t normalized,
                                  const float* d_x, int32_t n_channels, int64_t n_samples, float* d_spec,
                                  void* stream);
/* torch.istft (src/stft.h:167-197): d_spec complex [C][n_fft/2 + 1][n_frames] ->
 * d_y [C][hop * (n_frames - 1)], window-sum normalised. */
STG_API stg_status stg_torch_istft(stg_engine* engine, int32_t n_fft, int32_t hop, int32_t normalized,
                                   const float* d_spec, int32_t n_channels, int32_t n_frames, float* d_y,
                                   void* stream);
/* HTDemucs _spec (src/stft.h:79-103): d_x [C][n_samples] -> complex [C][2048][T],
 * T = ceil(n_samples / 1024). */
STG_API stg_status stg_htdemucs_spec(stg_engine* engine, const float* d_x, int32_t n_channels, int64_t n_samples,
                                     float* d_spec, void* stream);
/* HTDemucs _ispec (src/stft.h:106-140): complex [C][2048][n_frames] -> d_y [C][length];
 * n_frames must be ceil(length / 1024), as the model calls it. */
STG_API stg_status stg_htdemucs_ispec(stg_engine* engine, const float* d_spec, int32_t n_channels,
                                      int32_t n_frames, int64_t length, float* d_y, void* stream);

/* ---- a separation that allocates no device memory ---------------------------------------- */

/* No counterpart in the reference: the reference runs this path on the host.
 *
 * For callers that cannot call cudaMalloc: plug-ins hosted inside an audio application that
 * owns the CUDA context and hands out all device memory itself, and real-time code that must
 * not block on the device allocator. The caller passes the mix, the masks and the output
 * (device buffers, same layouts as stg_separate with a RoFormer plan); everything else the
 * separation needs, its tables and the fused kernel's scratch, lives in one static device
 * array of 64 MiB that every GPU loading this library reserves until the process exits.
 * With 352800-sample chunks of a stereo one-stem model that is 17 chunks (61.8 MiB): a track of
 * up to 22 s at num_overlap 4, 60 s at num_overlap 2. Longer inputs are rejected with
 * STG_INVALID_ARGUMENT and a message saying how much they need.
 *
 * Contexts: the call runs in `device`'s primary context, the one the CUDA runtime (and an
 * application built on it) uses. When the calling thread has no current context, or another
 * device's primary context, it makes `device`'s current for the call and afterwards makes the
 * caller's (or none) current again. A context the caller created with the driver API
 * (cuCtxCreate) is refused with STG_UNSUPPORTED before any GPU work; the buffers and the stream
 * must belong to the primary context. The first call in a context looks up the array's device
 * address there (cudaGetSymbolAddress); make that first call before any stream capture begins.
 * Each call copies its tables (chunk schedule, weights, window, twiddles) from host memory the
 * library keeps into the array with one cudaMemcpyAsync on `stream`, which may wait for the
 * stream's earlier work; a call with the same configuration and length as the previous call
 * in the same context skips the copy. Every call writes the same array (the fused kernel
 * writes all the scratch a call reads, so nothing needs clearing), so calls that overlap on
 * the GPU, for instance on two streams of the same device, race: serialise them.
 * Asynchronous on `stream`; `message` (optional, message_size bytes) receives the reason for
 * a failure. */
STG_API stg_status stg_separate_roformer_noalloc(int device, const stg_roformer_config* config,
                                                 int64_t n_samples, const float* d_mix,
                                                 const float* d_mask, float* d_out, void* stream,
                                                 char* message, size_t message_size);

#ifdef __cplusplus
}
#endif

#endif /* STEMS_GPU_V1_H */
