/* oracle.h -- CPU checker for the spectral front/back end of stems.cpp.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product links, loads or calls this library:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
 * use it, and only as the checker or as the timed CPU baseline.
 *
 * It restates, in plain C and double precision, the reference's host path:
 *   - the DSP primitives of src/stft.h and src/vr_dsp.h (radix-2 FFT, Bluestein FFT,
 *     reflect pad, periodic Hann, HTDemucs _spec/_ispec, torch.stft/istft);
 *   - the per-architecture glue and chunk schedulers of src/htdemucs.cpp,
 *     src/roformer.cpp and src/tfc_tdf.cpp, with the network replaced by a synthetic
 *     stand-in that multiplies the spectrogram by a caller-supplied mask.
 * Each function names the reference lines it follows. The primitives can be swapped for
 * the reference's own compiled stft.h/vr_dsp.h (oracle/_ref/libstems_ref.so, built from the
 * reference sources by oracle/build_ref.sh) with or_use_reference(), which is how the
 * restatement is pinned and how the "reference" CPU baseline is timed.
 *
 * Complex arrays are interleaved doubles (re, im), i.e. numpy complex128.
 * Every function returns 0 on success and a negative code on bad arguments.
 */
#ifndef STEMS_ORACLE_H
#define STEMS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- DSP primitives (src/stft.h, src/vr_dsp.h) ---------------------------------------- */
int or_fft(int n, double* a, int inverse);                 /* stft.h:19-55, n a power of two */
int or_vrfft(int n, double* a, int inverse);               /* vr_dsp.h:11-37 (Bluestein) */
int or_torch_stft(int n_fft, const float* x, int len, int hop, int normalized,
                  double* out, int* n_frames);             /* stft.h:146-164 */
int or_torch_istft(int n_fft, const double* spec, int n_frames, int hop, int normalized,
                   float* out);                            /* stft.h:167-197 */
int or_htdemucs_spec(int n_fft, const float* x, int len, double* out, int* n_frames);  /* stft.h:79-103 */
int or_htdemucs_ispec(int n_fft, const double* spec, int n_frames, int length, float* out); /* stft.h:106-140 */

/* The random-shift offsets the separators draw: std::mt19937(seed), then `shifts` draws of
 * std::uniform_int_distribution<int>(0, hi) (src/htdemucs.cpp:578, 617-619, hi = max_shift;
 * src/roformer.cpp:461-465, hi = max_shift - 1). oracle/shifts.cpp, C++ for the same
 * standard-library sequence. */
int or_shift_offsets(unsigned seed, int shifts, int hi, int* out);

/* ---- the request's audio in and the stems out (src/audio.h:17-56) ---------------------- */
/* resample_planar: Kaiser-windowed sinc (32 zero crossings, cutoff 0.95 of the lower Nyquist,
 * beta 8.6, 2^15-entry table interpolated linearly), planar in [ch][n] -> out [ch][out_n],
 * out_n = llround(n * dst / src). out must hold ch * or_resampled_length(...) floats. */
long long or_resampled_length(long long n, int src_rate, int dst_rate);
int or_resample_planar(const float* in, int n, int ch, int src_rate, int dst_rate, float* out, int* out_n);

/* ---- VR (src/vr_dsp.h:43-125, src/vr.cpp:215-269, 349-377) ----------------------------- */
/* Stereo only, as the reference. Spectra are [2][nfft/2+1][frames] complex (interleaved
 * double pairs holding complex64 values). */
int or_vr_stft(const float* wave, int n, int nfft, int hop, double* out, int* n_frames);
int or_vr_istft(const double* spec, int frames, int nfft, int hop, float* out);   /* out [2][hop*(frames-1)] */
int or_vr_resampled_length(int n, int src_rate, int dst_rate);
int or_vr_resample(const float* x, int n, int src_rate, int dst_rate, const float* fir, int n_taps, float* y);
float or_vr_lowpass(int f, int start, int stop);
float or_vr_highpass(int f, int start, int stop);
typedef struct { int sr, hop, nfft, start, stop, hp_start, hp_stop, lp_start, lp_stop; } or_vr_band;
typedef struct { int src, dst, n_taps; const float* taps; } or_vr_fir;
typedef struct {
    int sample_rate, bins, pre_start, pre_stop;
    int n_bands;
    const or_vr_band* bands;   /* lowest rate first, as vr.band.0 .. */
    int n_firs;
    const or_vr_fir* firs;     /* the model's resample.<src>.<dst> FIRs */
} or_vr_params;
int or_vr_n_frames(const or_vr_params* p, int len);
/* mask [2][bins+1][T] (the network's output, the stand-in); out [2 stems][2][len]:
 * spectrum x mask, spectrum x (1 - mask), each synthesised. */
int or_vr_separate(const or_vr_params* p, const float* mix, int len, const float* mask, float* out);

/* Swap the primitives above (as used by the glue below) for the reference's own compiled
 * code. path = NULL restores the restatement. Returns 0 on success. */
int or_use_reference(const char* path);
int or_using_reference(void);

/* ---- glue: HTDemucs (src/htdemucs.cpp:419-475, 534-644) ------------------------------ */
typedef struct {
    int n_channels;      /* C */
    int n_sources;       /* S */
    int segment;         /* samples per segment (343980 for the published models) */
    float overlap;       /* < 0: 0.25 */
    int cac_norm;        /* 1: mean/std normalise the CaC spectrogram around the stand-in */
    int mono_norm;       /* 1: demucs' mono-mix normalisation around the whole separation */
    int sample_first;    /* timing only: process segments [first, first+count) */
    int sample_count;    /* <= 0: all segments (the window applies without shifts only) */
    int threads;         /* worker threads for the per-segment work (<= 1: serial) */
    int shifts;          /* random shifts averaged (:610-626); 0 = one pass */
    unsigned seed;       /* std::mt19937 seed of the shift offsets */
    int sample_rate;     /* max shift = sample_rate / 2; 0 = 44100 */
    int n_models;        /* bag of models (:585-642); <= 1 with bag NULL: one model */
    const float* bag;    /* [n_models][S] weights, or NULL for all 1 */
} or_ht_params;
/* mask: per segment [S][2C][F = n_fft/2][T] float (re plane 2c, im plane 2c+1), segments
 * back to back (with shifts: every shift's segments, shift by shift; with a bag, every
 * model's masks, model by model). out: [S][C][len]. */
int or_ht_n_segments(const or_ht_params* p, int len);
int or_ht_n_frames(const or_ht_params* p);
int or_ht_separate(const or_ht_params* p, const float* mix, int len, const float* mask, float* out);

/* ---- glue: RoFormer (src/roformer.cpp:217-357, 436-486) ------------------------------ */
typedef struct {
    int n_channels, n_stems;
    int n_fft, hop, normalized, zero_dc;
    int chunk, step;
    int n_bands;
    const int* band_sizes;  /* [n_bands] */
    const int* band_freqs;  /* [sum band_sizes] */
    int complement;         /* append mix - est as one more stem */
    int sample_first, sample_count, threads;
    int shifts;             /* random shifts averaged (:456-478); 0 = one pass */
    unsigned seed;          /* std::mt19937 seed of the shift offsets */
    int sample_rate;        /* max shift = sample_rate / 2; 0 = 44100 */
} or_rf_params;
/* mask: per chunk [S][sum_b din_b * T] band-major, block b = [T][din_b], din_b = size_b*C*2,
 * entries (j*C + c)*2 + {re, im}. out: [S(+1)][C][len]. */
int or_rf_n_chunks(const or_rf_params* p, int len);
int or_rf_separate(const or_rf_params* p, const float* mix, int len, const float* mask, float* out);
/* The band gather of one chunk (roformer.cpp:226-241): z [C][F][T] complex -> feat. */
int or_rf_band_gather(const or_rf_params* p, const double* z, int n_frames, float* feat);

/* ---- glue: TFC-TDF / MDX (src/tfc_tdf.cpp:55-70, 354-495, 570-598) ------------------- */
typedef struct {
    int n_stems;
    int n_fft, hop, dim_f, dim_t, zero_bins;
    int chunking;           /* 0 = uvr_mdx, 1 = msst */
    float overlap;          /* < 0: the model default */
    int num_overlap;        /* msst default step = chunk / num_overlap */
    float compensate;
    int complement;
    int sample_first, sample_count, threads;
} or_tfc_params;
/* mask: per chunk real [4S][dim_f][dim_t]; the stand-in network is y = in * mask. */
int or_tfc_n_chunks(const or_tfc_params* p, int len);
int or_tfc_separate(const or_tfc_params* p, const float* mix, int len, const float* mask, float* out);

#ifdef __cplusplus
}
#endif
#endif
