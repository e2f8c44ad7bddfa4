// kernels.h -- device data structures and kernel launchers of the spectral path.
//
// Everything here is plain data: the host scheduler (engine.cu) builds these structs from a
// model configuration and a track length, and the launchers in kernels.cu run them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace stg {

enum Arch : int { ARCH_ROFORMER = 0, ARCH_HTDEMUCS = 1, ARCH_TFC = 2 };

// One chunk (RoFormer/TFC-TDF) or segment (HTDemucs) of a track.
//
// Input side: chunk-local sample p in [0, Lc) reads the chunk's virtual track at src0 + p
// when p < valid; past valid it reads the mirror 2*(valid-1) - p (tail_reflect) or zero.
// Virtual-track coordinates outside [0, vlen) are reflected (reflect) or read as zero; the
// virtual track's sample x is the mix's sample x + vshift, zero outside the mix. (The
// virtual track is the mix itself, or one pass of the random-shift average: the mix behind
// max_shift - offset zeros, src/roformer.cpp:464-472.)
// Output side: the chunk contributes out_len samples starting at output coordinate out0 of
// its group; sample u of them is the chunk's own output at y_off + u, weighted by
// W[w_off + u].
struct ChunkDesc {
    int64_t src0;
    int64_t out0;
    int64_t vlen;
    int64_t vshift;
    int32_t valid;
    int32_t tail_reflect;
    int32_t reflect;
    int32_t out_len;
    int32_t y_off;
    int32_t w_off;
    int32_t _pad[2];
};

// Chunks [c0, c1) overlap-added into one normalised estimate (a pass of the shift average);
// output sample i of the track is the group's output coordinate i + out_shift.
struct ChunkGroup {
    int32_t c0, c1;
    int32_t out_shift;
    int32_t _pad;
};

// STFT geometry of one chunk. Frame t covers padded positions [first_pos + t*hop, +n_fft).
// A padded position q maps to chunk-local sample reflect(q - n_fft/2, Lc) (torch.stft's
// centre pad), or, for HTDemucs' _spec, reflect(reflect(q - n_fft/2, ht_lxf) - ht_pad, Lc).
// The chunk's output sample j (iSTFT with window-sum normalisation) sits at q = j + out_offset.
// zero_pad: chunk-local sample q - n_fft/2, zero outside [0, Lc) (VR's zero-centred STFT).
struct FrameGeom {
    int n_fft, hop;
    int Lc;
    int T;
    int first_pos;
    int ht_pad;
    int ht_lxf;
    int out_offset;
    int Lout;
    int zero_pad;
};

struct FusedParams {
    const float* mix;          // planar [C][len]
    int64_t len;
    int n_channels;            // 1 or 2
    const ChunkDesc* chunks;
    int n_chunks;
    FrameGeom g;
    int K;                     // frames per tile
    int n_tiles;
    int S;                     // stems
    const float* win;          // periodic Hann [n_fft]
    const float2* tw;          // the FFT plan's per-pass twiddles (fft.cuh: twiddle_index)
    const float* inv_env;      // [Lout]: 1 / sum of squared windows, 0 where it vanishes
    const float* env_period;   // [hop]: inv_env over [env_lo, env_hi), where it repeats every hop
    int env_lo, env_hi;        // (empty when env_period is null)
    float fwd_scale, inv_scale;
    // mask (the stand-in for the network's output), one block per chunk; TFC-TDF masks in the
    // t-major layout of launch_mask_transpose
    const float* mask;
    int64_t mask_chunk_stride;
    // RoFormer: bin -> (band entry) inverse table. bin_tab[f] holds the first two bands holding
    // f as (offset without the frame term) / (2C) in bits 0-21 and the band size (bins) in bits
    // 22-31, 0 when absent; bin_ebeg/bin_ent list every entry (CSR over bins) for the bins that
    // more than two bands hold (bin_multi).
    const int2* bin_tab;       // [F] compact entries, see kernels.cu (RoFormer MaskOp)
    int bin_multi;             // 1 when some bin is held by more than two bands
    const int* bin_ebeg;       // [F + 1]
    const int2* bin_ent;       // (offset of the entry in a stem's mask block without t, din_b)
    const float* bin_inv;      // [F] 1 / max(bands_per_freq, 1)
    int zero_dc;
    int64_t stem_stride;       // floats per stem within a chunk's mask block
    // TFC-TDF
    int dim_f, zero_bins;
    // outputs
    float* Y;                  // [chunk][S][Lout][C]: the channels of a sample side by side
    int64_t y_chunk_stride;
    float* Tr;                 // [chunk][tile][S][n_fft - hop][C]
    int64_t tr_chunk_stride;
};

struct CombineParams {
    const float* Y;
    int64_t y_chunk_stride;
    const float* Tr;
    int64_t tr_chunk_stride;
    const ChunkDesc* chunks;
    int n_chunks;
    const ChunkGroup* groups;  // the passes of the shift average (one group without shifts)
    int n_groups;
    int shift_mean;            // 1: sum the groups, then divide (src/htdemucs.cpp:618-626);
                               // 2: add each group divided by n_groups (src/roformer.cpp:474-477)
    int64_t step_out;          // regular chunk step in output coordinates
    int64_t max_out_len;       // longest out_len of any chunk
    FrameGeom g;
    int K, n_tiles;
    const float* W;            // weight tables
    int S, C;
    int64_t len;               // output samples per row
    int64_t i_begin, i_end;    // the output samples this launch writes
    int mode;                  // ARCH_*
    int nan_to_zero;
    float compensate;          // multiplies the stems (1 = off)
    int complement;            // 1: first stem; 2: all stems (TFC-TDF) subtracted from the mix
    const float* mix;          // for the complement
    const double* mono_stats;  // HTDemucs mono-mix normalisation (mean, std), or null
    // HTDemucs bag of models (src/htdemucs.cpp:628-642), or bag == null: out accumulates
    // bag[model][s] * (this model's stem s) (the first model starts from zero), and the last
    // model divides by bag_tot[s] and then applies mono_stats
    const float* bag;          // [n_models][S]
    const float* bag_tot;      // [S]
    int bag_model, bag_last;
    float* out;                // [S(+1)][C][len]
};

// The two halves of the path around a real network (split.cu). The front half computes the
// STFT of every chunk and writes it in the network's input layout; the back half reads a
// spectrogram in the network's output layout and runs the iSTFT and the overlap-add into
// the same Y / Tr scratch as the fused kernel (the combine then finishes the separation).
enum FrontLayout : int {
    FRONT_COMPLEX = 0,   // complex [C][F][T], F = n_bins (torch_stft, htdemucs_spec)
    FRONT_CAC = 1,       // float planes [2C][F][T]: re = 2c, im = 2c + 1 (HTDemucs input)
    FRONT_BANDS = 2,     // RoFormer band-major features [sum_b din_b * T]
    FRONT_TFC = 3,       // float planes [4][dim_f][T], bins below zero_bins 0 (TFC-TDF input)
    FRONT_STATS = 4,     // no output: (sum, sum of squares) of the CaC values per (chunk, tile)
    FRONT_ZSPEC = 5      // the spectra t-major, zspec [chunk][T][n_bins] float4 (L re, L im, R re, R im)
};
enum BackLayout : int {
    BACK_COMPLEX = 0,    // complex [C][F][T] (torch_istft, htdemucs_ispec)
    BACK_CAC = 1,        // float planes [S][2C][F][T] (HTDemucs output)
    BACK_TFC = 2,        // float planes [4S][dim_f][T] (TFC-TDF output)
    BACK_ZMASK = 3       // HTDemucs with the stand-in network: zspec times the t-major masks
                         // [S][T][n_bins] float4 in net (launch_mask_transpose), CaC-normalised
};

struct SplitParams {
    const float* mix;          // front: the track
    int64_t len;
    int n_channels;
    const ChunkDesc* chunks;
    int n_chunks;
    FrameGeom g;
    int K, n_tiles;
    int S;                     // back: stems in the network output
    const float* win;
    const float2* tw;
    float fwd_scale, inv_scale;
    const float* inv_env;
    const float* env_period;   // as FusedParams
    int env_lo, env_hi;
    int layout;                // FrontLayout or BackLayout
    int n_bins;                // bins the layout holds
    int zero_bins;             // FRONT_TFC
    const int2* bin_tab;       // FRONT_BANDS (FusedParams::bin_tab)
    int bin_multi;
    const int* bin_ebeg;
    const int2* bin_ent;
    float* net;                // front: written; back: read
    int64_t net_chunk_stride;
    const double2* cac_stats;  // FRONT_CAC / BACK_CAC / BACK_ZMASK: per-chunk (mean, std), or null
    double2* stats_out;        // front: [chunk][tile] partial sums of the CaC values, or null
    float4* zspec;             // FRONT_ZSPEC: written; BACK_ZMASK: read
    int64_t z_chunk_stride;    // float4 per chunk
    float* Y;                  // back
    int64_t y_chunk_stride;
    float* Tr;
    int64_t tr_chunk_stride;
};

// Launchers. Return a cudaError_t from the launch (kernel errors surface on sync).
cudaError_t launch_fused(int arch, const FusedParams& p, cudaStream_t st);
cudaError_t launch_front(const SplitParams& p, cudaStream_t st);
cudaError_t launch_back(const SplitParams& p, cudaStream_t st);
cudaError_t launch_combine(const CombineParams& p, cudaStream_t st);
// f-major mask planes [S][P][F][T] per chunk (in_chunk_stride floats apart) -> t-major
// [S][T][F] float4 per chunk (out_chunk_stride float4 apart), plane p in component p.
// max_ctas > 0 caps the grid (the CTAs stride over the tiles), leaving room on the SMs for
// a kernel that runs beside it.
cudaError_t launch_mask_transpose(const float* in, int64_t in_chunk_stride, int n_chunks, int S, int P, int F,
                                  int T, float4* out, int64_t out_chunk_stride, cudaStream_t st, int max_ctas = 0);
size_t fused_smem_bytes(int arch, int n_fft);
int fused_threads(int n_fft);
int fused_max_hop(int n_fft);      // the largest hop the fused kernel takes at this n_fft
// CTAs of the fused kernel resident at once on the current device (0 when unknown).
int fused_resident_ctas(int arch, int n_fft);
// The radices of the FFT plan at this n_fft, in pass order (fft.cuh: twiddle_index).
std::vector<int> fused_radices(int n_fft);
// The radices of the forward transform's own plan where it differs from fused_radices (empty
// otherwise); its twiddles follow that plan's n_fft entries in the table.
std::vector<int> fused_fwd_radices(int n_fft);
bool fused_supported(int n_fft);
// TFC-TDF at n_fft 7680 with an even hop runs on CTA pairs (pair.cu): whether it does, the
// pair plan's radices (its twiddles follow the n_fft table: the 3840-point plan's, then
// W_7680^k for k < 3840), the clusters resident at once, and the launch
bool fused_pair(int arch, int n_fft, int hop);
std::vector<int> fused_pair_radices(int n_fft);
int fused_pair_slots();
cudaError_t launch_fused_pair(const FusedParams& p, cudaStream_t st);
bool split_supported(int n_fft);   // n_fft the front and back kernels take
int back_resident_ctas(int n_fft); // CTAs of the back kernel resident at once (0 when unknown)
int split_resident_ctas(int n_fft, bool front);   // the same for the front (generic) or back kernel
int split_max_hop(int n_fft);

// convert.cu. Resampling (and layout / channel conversion) of planar or interleaved audio:
// output row k, sample i < out_n, is the resampled input channel src(k) (to_channels: 0 for
// a mono input, else min(k, in_ch - 1); otherwise k); samples [out_n, out_pin) are zero.
// table == nullptr copies instead of resampling (same rate).
struct ResampleParams {
    const float* in;
    int64_t in_n;              // samples per input channel
    int in_ch;
    int interleaved;           // 1: in[i * in_ch + c]; 0: in[c * in_n + i]
    int to_channels;
    int rows;
    const double2* table;      // kaiser_table's entries t and t + 1 side by side, or null
    double half, ratio;
    int64_t out_n;             // resampled length
    int64_t out_pin;           // row stride of the output (pinned length)
    float* out;                // [rows][out_pin]
};
int64_t resampled_length(int64_t n, int src_rate, int dst_rate);
void kaiser_table(int src_rate, int dst_rate, std::vector<double>& table, double& half, double& ratio);
cudaError_t launch_resample(const ResampleParams& p, cudaStream_t st);

// norm.cu. Mono-mix normalisation of mix [C][len] into out, with scratch of
// mono_scratch_doubles() doubles (scratch[0] = mean, scratch[1] = std afterwards).
size_t mono_scratch_doubles();
cudaError_t launch_mono_norm(const float* mix, int64_t len, int C, double* scratch, float* out, cudaStream_t st);
// Per-chunk (mean, std) of the CaC values from the FRONT_STATS partials ([chunk][tile]).
cudaError_t launch_cac_finish(const double2* partial, int n_chunks, int n_tiles, double count, double2* stats,
                              cudaStream_t st);

} // namespace stg
