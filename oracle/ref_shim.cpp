// ref_shim.cpp -- C entry points over the reference's own DSP headers. TEST INFRASTRUCTURE.
//
// Compiled by oracle/build.sh against the reference sources where they lie
// (REF_SRC, the reference project's src/ directory) into oracle/_ref/libstems_ref.so. Nothing
// from the reference is copied here: this file only forwards to st::FFT, st::VRFFT,
// st::torch_stft/istft and st::htdemucs_spec/ispec (src/stft.h, src/vr_dsp.h) so the C
// restatement in oracle.c can be pinned against them, golden vectors can be generated from
// them, and the CPU baseline can time them. ref_resample_planar forwards to
// st::resample_planar (src/audio.h).
#include "audio.h"
#include "stft.h"
#include "vr_dsp.h"

#include <cstring>
#include <map>
#include <memory>

namespace {

// One transform object per size and thread, built once like the models build theirs
// (src/htdemucs.cpp:315, src/roformer.cpp:398, src/tfc_tdf.cpp:551-552).
const st::FFT& fft_for(int n) {
    thread_local std::map<int, std::unique_ptr<st::FFT>> cache;
    auto& p = cache[n];
    if (!p) p = std::make_unique<st::FFT>(n);
    return *p;
}
const st::VRFFT& vrfft_for(int n) {
    thread_local std::map<int, std::unique_ptr<st::VRFFT>> cache;
    auto& p = cache[n];
    if (!p) p = std::make_unique<st::VRFFT>(n);
    return *p;
}
bool pow2(int n) { return n >= 2 && !(n & (n - 1)); }

void put(const std::vector<st::cplx>& v, double* out) {
    std::memcpy(out, v.data(), v.size() * sizeof(st::cplx));
}
std::vector<st::cplx> get(const double* in, size_t n) {
    std::vector<st::cplx> v(n);
    std::memcpy(v.data(), in, n * sizeof(st::cplx));
    return v;
}

} // namespace

extern "C" {

int ref_fft(int n, double* a, int inverse) {
    try {
        std::vector<st::cplx> v = get(a, (size_t)n);
        fft_for(n).run(v, inverse != 0);
        put(v, a);
        return 0;
    } catch (...) { return -1; }
}

int ref_vrfft(int n, double* a, int inverse) {
    try {
        std::vector<st::cplx> v = get(a, (size_t)n);
        vrfft_for(n).run(v, inverse != 0);
        put(v, a);
        return 0;
    } catch (...) { return -1; }
}

int ref_torch_stft(int n_fft, const float* x, int len, int hop, int normalized, double* out, int* n_frames) {
    try {
        int T = 0;
        const std::vector<st::cplx> s = pow2(n_fft)
            ? st::torch_stft(fft_for(n_fft), x, len, hop, normalized != 0, T)
            : st::torch_stft(vrfft_for(n_fft), x, len, hop, normalized != 0, T);
        put(s, out);
        if (n_frames) *n_frames = T;
        return 0;
    } catch (...) { return -3; }
}

int ref_torch_istft(int n_fft, const double* spec, int n_frames, int hop, int normalized, float* out) {
    try {
        const std::vector<st::cplx> s = get(spec, (size_t)(n_fft / 2 + 1) * n_frames);
        const std::vector<float> y = pow2(n_fft)
            ? st::torch_istft(fft_for(n_fft), s, n_frames, hop, normalized != 0)
            : st::torch_istft(vrfft_for(n_fft), s, n_frames, hop, normalized != 0);
        std::memcpy(out, y.data(), y.size() * sizeof(float));
        return 0;
    } catch (...) { return -3; }
}

int ref_htdemucs_spec(int n_fft, const float* x, int len, double* out, int* n_frames) {
    try {
        int T = 0;
        put(st::htdemucs_spec(fft_for(n_fft), x, len, T), out);
        if (n_frames) *n_frames = T;
        return 0;
    } catch (...) { return -3; }
}

int ref_htdemucs_ispec(int n_fft, const double* spec, int n_frames, int length, float* out) {
    try {
        const std::vector<st::cplx> s = get(spec, (size_t)(n_fft / 2) * n_frames);
        const std::vector<float> y = st::htdemucs_ispec(fft_for(n_fft), s, n_frames, length);
        std::memcpy(out, y.data(), y.size() * sizeof(float));
        return 0;
    } catch (...) { return -3; }
}

int ref_resample_planar(const float* in, int n, int ch, int src_rate, int dst_rate, float* out, int* out_n) {
    try {
        const std::vector<float> x(in, in + (size_t)n * ch);
        int m = 0;
        const std::vector<float> y = st::resample_planar(x, n, ch, src_rate, dst_rate, m);
        std::memcpy(out, y.data(), y.size() * sizeof(float));
        *out_n = m;
        return 0;
    } catch (...) { return -3; }
}

int ref_vr_stft(const float* wave, int n, int nfft, int hop, double* out, int* n_frames) {
    try {
        const std::vector<float> w(wave, wave + 2 * (size_t)n);
        const st::VRBand b = {0, hop, nfft, 0, nfft / 2 + 1, -1, -1, -1, -1};
        int frames = 0;
        put(st::vr_stft(w, n, b, frames), out);
        *n_frames = frames;
        return 0;
    } catch (...) { return -3; }
}

int ref_vr_istft(const double* spec, int frames, int nfft, int hop, float* out) {
    try {
        const st::VRBand b = {0, hop, nfft, 0, nfft / 2 + 1, -1, -1, -1, -1};
        const std::vector<float> y = st::vr_istft(get(spec, (size_t)2 * (nfft / 2 + 1) * frames), frames, b);
        std::memcpy(out, y.data(), y.size() * sizeof(float));
        return 0;
    } catch (...) { return -3; }
}

int ref_vr_resample(const float* x, int n, int src, int dst, const float* fir, int n_taps, float* y) {
    try {
        const std::vector<float> in(x, x + 2 * (size_t)n), h(fir, fir + n_taps);
        int m = 0;
        const std::vector<float> out = st::vr_resample(in, n, src, dst, h, m);
        std::memcpy(y, out.data(), out.size() * sizeof(float));
        return 0;
    } catch (...) { return -3; }
}

} // extern "C"
