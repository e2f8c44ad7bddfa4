// vr.cu -- the VR architecture's spectral path on the device (src/vr.cpp:215-269, 349-377;
// src/vr_dsp.h:43-125), with the network between the halves:
//
//   front  the mix resampled band by band, from the model rate down (rational polyphase FIR,
//          src/vr_dsp.h:92-111), each band's zero-centred STFT (43-62), the bands' crops
//          concatenated into one spectrum [2][bins+1][T] with the pre-filter applied
//          (vr.cpp:219-239); |spec| and its peak, the network's input
//   back   for each of the two stems, the spectrum times mask (or 1 - mask), split back into
//          the bands with their high/low-pass gains, each band's iSTFT (64-88), and the
//          bands summed from the lowest rate up, resampled between them (vr.cpp:241-269)
//
// The STFTs and iSTFTs are the single-chunk front/back kernels of split.cu at the band's
// n_fft (320 to 2048); the resampler, the crop/concat and the band split are kernels here.
// The resampler accumulates the float taps in double in the reference's order, so it
// returns the reference's floats for the same input.
#include "engine.h"

#include <numeric>

namespace stg {

namespace {

constexpr int kMaxBands = 16;
constexpr size_t kResampleSmemMax = 96 * 1024;   // larger stretches use the kernel without staging

// scipy-style centred upfirdn of stereo x [2][n] (src/vr_dsp.h:92-111)
__global__ void __launch_bounds__(256) vr_resample_kernel(const float* __restrict__ x, int n, int up, int down,
                                                         const float* __restrict__ fir, int n_taps,
                                                         float* __restrict__ y, int out_n) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= out_n) return;
    const int64_t pos = (int64_t)j * down + n_taps / 2;
    const int lo = (int)max((int64_t)0, (pos - n_taps + up) / up);
    const int hi = (int)min((int64_t)n - 1, pos / up);
    double s0 = 0.0, s1 = 0.0;
    for (int i = lo; i <= hi; i++) {
        const double h = (double)__ldg(fir + (pos - (int64_t)i * up));
        s0 = __dadd_rn(s0, __dmul_rn((double)__ldg(x + i), h));
        s1 = __dadd_rn(s1, __dmul_rn((double)__ldg(x + n + i), h));
    }
    y[j] = (float)s0;
    y[out_n + j] = (float)s1;
}

// The same sums, with the block's input stretch of both channels and the FIR converted to
// double once into shared memory (each input sample feeds about n_taps / up outputs). The
// loads and products are the same doubles in the same order, so the outputs are the same.
__global__ void __launch_bounds__(256) vr_resample_smem_kernel(const float* __restrict__ x, int n, int up, int down,
                                                              const float* __restrict__ fir, int n_taps,
                                                              float* __restrict__ y, int out_n, int cap) {
    extern __shared__ double sm[];
    const int j0 = blockIdx.x * blockDim.x;
    const int jl = min(out_n - 1, j0 + (int)blockDim.x - 1);
    const auto lo_of = [&](int j) {
        return (int)max((int64_t)0, ((int64_t)j * down + n_taps / 2 - n_taps + up) / up);
    };
    const auto hi_of = [&](int j) { return (int)min((int64_t)n - 1, ((int64_t)j * down + n_taps / 2) / up); };
    const int base = lo_of(j0), span = hi_of(jl) - base + 1;   // lo and hi grow with j
    if (span > cap) {   // more than the launch allocated (the host bound makes this unreachable)
        const int j = j0 + threadIdx.x;
        if (j <= jl) {
            const int64_t pos = (int64_t)j * down + n_taps / 2;
            double s0 = 0.0, s1 = 0.0;
            for (int i = lo_of(j); i <= hi_of(j); i++) {
                const double h = (double)__ldg(fir + (pos - (int64_t)i * up));
                s0 = __dadd_rn(s0, __dmul_rn((double)__ldg(x + i), h));
                s1 = __dadd_rn(s1, __dmul_rn((double)__ldg(x + n + i), h));
            }
            y[j] = (float)s0;
            y[out_n + j] = (float)s1;
        }
        return;
    }
    double* xs = sm;             // [2][cap]
    double* hs = sm + 2 * cap;   // [n_taps]
    for (int k = threadIdx.x; k < span; k += blockDim.x) {
        xs[k] = (double)__ldg(x + base + k);
        xs[cap + k] = (double)__ldg(x + n + base + k);
    }
    for (int k = threadIdx.x; k < n_taps; k += blockDim.x) hs[k] = (double)__ldg(fir + k);
    __syncthreads();
    const int j = j0 + threadIdx.x;
    if (j > jl) return;
    const int64_t pos = (int64_t)j * down + n_taps / 2;
    const int lo = lo_of(j), hi = hi_of(j);
    double s0 = 0.0, s1 = 0.0;
    for (int i = lo; i <= hi; i++) {
        const double h = hs[pos - (int64_t)i * up];
        s0 = __dadd_rn(s0, __dmul_rn(xs[i - base], h));
        s1 = __dadd_rn(s1, __dmul_rn(xs[cap + i - base], h));
    }
    y[j] = (float)s0;
    y[out_n + j] = (float)s1;
}

struct AssembleParams {
    const float2* band_spec[kMaxBands];   // [2][F_i][frames_i]
    int F[kMaxBands], frames[kMaxBands], start[kMaxBands], off[kMaxBands], count[kMaxBands];
    int n_bands, F1, T;
    int pre_start, pre_stop;
    float2* spec;                         // [2][F1][T]
    float* mag;                           // [2][F1][T] or null
};

__device__ __forceinline__ float vr_lowpass(int f, int start, int stop) {    // src/vr_dsp.h:113-118
    if (start < 0) return 1.0f;
    if (f < start - 1) return 1.0f;
    if (f >= stop) return 0.0f;
    return 1.0f - (float)(f - start + 1) / (stop - start);
}
__device__ __forceinline__ float vr_highpass(int f, int start, int stop) {   // src/vr_dsp.h:119-125
    if (start <= 0) return 1.0f;
    if (f <= stop + 1) return 0.0f;
    if (f >= start + 1) return 1.0f;
    return (float)(f - stop - 1) / (start - stop);
}

// the bands' crops side by side, the pre-filter, |spec| and its peak (vr.cpp:226-239, 357-360)
__global__ void __launch_bounds__(256) vr_assemble_kernel(const AssembleParams p) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t per_c = (int64_t)p.F1 * p.T;
    if (e >= 2 * per_c) return;
    const int c = (int)(e / per_c);
    const int f = (int)((e - c * per_c) / p.T);
    const int t = (int)(e - c * per_c - (int64_t)f * p.T);
    float2 v = make_float2(0.0f, 0.0f);
    for (int i = 0; i < p.n_bands; i++)
        if (f >= p.off[i] && f < p.off[i] + p.count[i]) {
            v = p.band_spec[i][((int64_t)c * p.F[i] + p.start[i] + f - p.off[i]) * p.frames[i] + t];
            break;
        }
    if (p.pre_start > 0) {
        const float g = vr_lowpass(f, p.pre_start, p.pre_stop);
        v = make_float2(v.x * g, v.y * g);
    }
    p.spec[e] = v;
    if (p.mag) p.mag[e] = hypotf(v.x, v.y);
}

// max of |spec| over the whole spectrum: a grid-stride pass, one atomic per block (the
// maximum does not depend on the order)
__global__ void __launch_bounds__(256) vr_peak_kernel(const float* __restrict__ mag, int64_t n, unsigned int* peak) {
    __shared__ float red[8];
    float mx = 0.0f;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        mx = fmaxf(mx, mag[e]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_down_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
        atomicMax(peak, __float_as_uint(mx));   // non-negative floats order as their bits
    }
}

struct PartParams {
    const float2* spec;   // [2][F1][T]
    const float* mask;    // [2][F1][T]
    int stem;             // 0: spec * mask, 1: spec * (1 - mask)
    int F1, T;
    int F, start, stop, off;
    int hp_start, hp_stop, lp_start, lp_stop, last;
    float2* part;         // [2][F][T]
};

// one band's share of one stem's spectrum, with the band's gains (vr.cpp:244-253, 372-373)
__global__ void __launch_bounds__(256) vr_part_kernel(const PartParams p) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t per_c = (int64_t)p.F * p.T;
    if (e >= 2 * per_c) return;
    const int c = (int)(e / per_c);
    const int f = (int)((e - c * per_c) / p.T);
    const int t = (int)(e - c * per_c - (int64_t)f * p.T);
    float2 v = make_float2(0.0f, 0.0f);
    if (f >= p.start && f < p.stop) {
        const int64_t k = ((int64_t)c * p.F1 + p.off + f - p.start) * p.T + t;
        const float mk = __ldg(p.mask + k);
        const float m = p.stem == 0 ? mk : 1.0f - mk;
        const float2 z = p.spec[k];
        const float gain = vr_highpass(f, p.hp_start, p.hp_stop - 1) *
                           (p.last ? 1.0f : vr_lowpass(f, p.lp_start, p.lp_stop));
        v = make_float2(z.x * m * gain, z.y * m * gain);
    }
    p.part[e] = v;
}

__global__ void vr_add_kernel(float* __restrict__ w, const float* __restrict__ a, int64_t n) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n) w[e] += a[e];
}

// the synthesised wave [2][n] into a stem's [2][len] (vr.cpp:265-267)
__global__ void vr_crop_kernel(const float* __restrict__ w, int n, float* __restrict__ out, int len) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= 2 * (int64_t)len) return;
    const int c = (int)(e / len), j = (int)(e - (int64_t)c * len);
    out[e] = j < n ? w[(int64_t)c * n + j] : 0.0f;
}

unsigned blocks_for(int64_t n, int threads = 256) { return (unsigned)((n + threads - 1) / threads); }

int resampled(int n, int src, int dst) {   // src/vr_dsp.h:96
    if (src == dst) return n;
    const int g = std::gcd(src, dst), up = dst / g, down = src / g;
    return (int)(((int64_t)n * up + down - 1) / down);
}

} // namespace
} // namespace stg

struct stg_vr_plan {
    stg_engine* engine = nullptr;
    std::vector<stg_vr_band> bands;
    int sr = 0, bins = 0, pre_start = 0, pre_stop = 0;
    int len = 0, T = 0;
    std::map<std::pair<int, int>, std::pair<DevBuf, int>> firs;   // (src, dst) -> (taps, count)
    std::vector<int> n_in, frames;                                 // per band: input samples, frames
    std::vector<std::unique_ptr<stg_plan>> stft, istft;
    std::vector<std::unique_ptr<DevBuf>> wave, spec_b;
    DevBuf spec, part, add, syn, tmp, peak;
    int n_syn_max = 0;

    const std::pair<DevBuf, int>& fir(int src, int dst) const {
        auto it = firs.find({src, dst});
        if (it == firs.end()) fail(STG_MODEL_ERROR, "vr: no resampling FIR for this rate pair");
        return it->second;
    }

    void resample(const float* x, int n, int src, int dst, float* y, cudaStream_t st) const {
        const int m = resampled(n, src, dst);
        if (src == dst) {
            cuda_check(cudaMemcpyAsync(y, x, sizeof(float) * 2 * (size_t)n, cudaMemcpyDeviceToDevice, st), "copy");
            return;
        }
        const int g = std::gcd(src, dst);
        const auto& h = fir(src, dst);
        const int up = dst / g, down = src / g, taps = h.second;
        // a block's input stretch: at most 255 output steps of down/up inputs plus the FIR's
        // reach, with a margin for the roundings of both ends
        const int64_t span = (int64_t)255 * down / up + taps / up + 4;
        const size_t smem = sizeof(double) * (size_t)(2 * span + taps);
        if (smem <= kResampleSmemMax) {
            cuda_check(cudaFuncSetAttribute(vr_resample_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)kResampleSmemMax),
                       "vr resampling kernel attribute");
            vr_resample_smem_kernel<<<blocks_for(m), 256, smem, st>>>(x, n, up, down, h.first.as<float>(), taps, y, m,
                                                                      (int)span);
        } else {
            vr_resample_kernel<<<blocks_for(m), 256, 0, st>>>(x, n, up, down, h.first.as<float>(), taps, y, m);
        }
        cuda_check(cudaGetLastError(), "vr resampling kernel launch");
    }

    // spectrum() and the network input (|spec| into d_mag and its peak into d_peak when given)
    void front(const float* d_mix, float* d_mag, float* d_peak, cudaStream_t st) {
        if (!d_mix) fail(STG_INVALID_ARGUMENT, "null buffer");
        cuda_check(cudaSetDevice(engine->device), "cudaSetDevice");
        const int B = (int)bands.size();
        const float* src = d_mix;
        int n = len, rate = sr;
        for (int i = B - 1; i >= 0; i--) {                                // vr.cpp:221-225
            const float* w = src;
            if (bands[i].sample_rate != rate) {
                resample(src, n, rate, bands[i].sample_rate, wave[i]->as<float>(), st);
                w = wave[i]->as<float>();
                n = resampled(n, rate, bands[i].sample_rate);
                rate = bands[i].sample_rate;
            }
            launch_front(stft[i]->H, stft[i]->D, w, 0, 1, spec_b[i]->as<float>(), st);
            src = w;
        }
        AssembleParams a{};
        int off = 0;
        for (int i = 0; i < B; i++) {
            a.band_spec[i] = spec_b[i]->as<float2>();
            a.F[i] = bands[i].n_fft / 2 + 1;
            a.frames[i] = frames[i];
            a.start[i] = bands[i].crop_start;
            a.off[i] = off;
            a.count[i] = bands[i].crop_stop - bands[i].crop_start;
            off += a.count[i];
        }
        a.n_bands = B;
        a.F1 = bins + 1;
        a.T = T;
        a.pre_start = pre_start;
        a.pre_stop = pre_stop;
        a.spec = spec.as<float2>();
        a.mag = d_mag;
        const int64_t K = (int64_t)2 * (bins + 1) * T;
        vr_assemble_kernel<<<blocks_for(K), 256, 0, st>>>(a);
        cuda_check(cudaGetLastError(), "vr assemble kernel launch");
        if (d_peak) {
            if (!d_mag) fail(STG_INVALID_ARGUMENT, "the peak needs the magnitude buffer");
            cuda_check(cudaMemsetAsync(d_peak, 0, sizeof(float), st), "clear the peak");
            vr_peak_kernel<<<std::min<unsigned>(blocks_for(K), 1184), 256, 0, st>>>(
                d_mag, K, reinterpret_cast<unsigned int*>(d_peak));
            cuda_check(cudaGetLastError(), "vr peak kernel launch");
        }
    }

    // the two stems from the spectrum the last front() left, synthesised (vr.cpp:368-377)
    void back(const float* d_mask, float* d_out, cudaStream_t st) {
        if (!d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
        cuda_check(cudaSetDevice(engine->device), "cudaSetDevice");
        const int B = (int)bands.size();
        for (int s = 0; s < 2; s++) {
            int off = 0, n = 0;
            float* wave = syn.as<float>();     // the running sum, and the buffer it moves to
            float* other = tmp.as<float>();
            for (int i = 0; i < B; i++) {                                 // vr.cpp:241-262
                const stg_vr_band& b = bands[i];
                PartParams q{};
                q.spec = spec.as<float2>();
                q.mask = d_mask;
                q.stem = s;
                q.F1 = bins + 1;
                q.T = T;
                q.F = b.n_fft / 2 + 1;
                q.start = b.crop_start;
                q.stop = b.crop_stop;
                q.off = off;
                q.hp_start = b.hpf_start;
                q.hp_stop = b.hpf_stop;
                q.lp_start = b.lpf_start;
                q.lp_stop = b.lpf_stop;
                q.last = i + 1 == B;
                q.part = part.as<float2>();
                off += b.crop_stop - b.crop_start;
                vr_part_kernel<<<blocks_for((int64_t)2 * q.F * T), 256, 0, st>>>(q);
                cuda_check(cudaGetLastError(), "vr part kernel launch");
                const int bn = b.hop * (T - 1);
                float* dst = i == 0 ? wave : add.as<float>();
                launch_back(istft[i]->H, istft[i]->D, nullptr, part.as<float>(), 0, 1, st);
                launch_finish(istft[i]->H, istft[i]->D, nullptr, dst, st);
                if (i > 0) {
                    vr_add_kernel<<<blocks_for(2 * (int64_t)n), 256, 0, st>>>(wave, add.as<float>(), 2 * (int64_t)n);
                    cuda_check(cudaGetLastError(), "vr add kernel launch");
                } else {
                    n = bn;
                }
                if (i + 1 < B) {
                    resample(wave, n, b.sample_rate, bands[i + 1].sample_rate, other, st);
                    n = resampled(n, b.sample_rate, bands[i + 1].sample_rate);
                    std::swap(wave, other);
                }
            }
            vr_crop_kernel<<<blocks_for(2 * (int64_t)len), 256, 0, st>>>(wave, n, d_out + (size_t)s * 2 * len, len);
            cuda_check(cudaGetLastError(), "vr crop kernel launch");
        }
    }
};

namespace {

void build_vr(stg_vr_plan& P, const stg_vr_config& c, int64_t n_samples) {
    // the reference's configuration checks (src/vr.cpp:296-327)
    if (c.sample_rate <= 0 || c.bins < 32 || c.bins > 8192 || c.bins % 32 || c.pre_filter_start < 0 ||
        c.pre_filter_stop > c.bins || c.pre_filter_stop <= c.pre_filter_start)
        fail(STG_MODEL_ERROR, "vr: invalid configuration");
    if (c.n_bands < 1 || c.n_bands > kMaxBands || !c.bands) fail(STG_MODEL_ERROR, "vr: invalid band count");
    if (n_samples <= 0 || n_samples > INT32_MAX / 8) fail(STG_INVALID_ARGUMENT, "empty or too long input");
    int total = 0;
    for (int i = 0; i < c.n_bands; i++) {
        const stg_vr_band& b = c.bands[i];
        if (b.sample_rate <= 0 || b.hop <= 0 || b.n_fft < 2 || b.n_fft > 16384 || b.n_fft % 2 || b.crop_start < 0 ||
            b.crop_stop <= b.crop_start || b.crop_stop > b.n_fft / 2 + 1)
            fail(STG_MODEL_ERROR, "vr: invalid frequency band");
        if ((b.hpf_start >= 0 && (b.hpf_start < 1 || b.hpf_stop < 0 || b.hpf_stop >= b.hpf_start ||
                                  b.hpf_start > b.n_fft / 2)) ||
            (b.lpf_start >= 0 && (b.lpf_start < 1 || b.lpf_stop <= b.lpf_start || b.lpf_stop > b.n_fft / 2)))
            fail(STG_MODEL_ERROR, "vr: invalid band filter");
        if (!split_supported(b.n_fft) || b.hop > split_max_hop(b.n_fft))
            fail(STG_UNSUPPORTED, "vr: n_fft " + std::to_string(b.n_fft) + " / hop " + std::to_string(b.hop) +
                                      " is not implemented");
        total += b.crop_stop - b.crop_start;
        P.bands.push_back(b);
    }
    const stg_vr_band& last = P.bands.back();
    if (total > c.bins || last.sample_rate != c.sample_rate) fail(STG_MODEL_ERROR, "vr: band layout mismatch");
    for (const auto& b : P.bands)
        if ((int64_t)b.sample_rate * last.hop != (int64_t)c.sample_rate * b.hop)
            fail(STG_MODEL_ERROR, "vr: frame duration mismatch");
    P.sr = c.sample_rate;
    P.bins = c.bins;
    P.pre_start = c.pre_filter_start;
    P.pre_stop = c.pre_filter_stop;
    P.len = (int)n_samples;
    for (int k = 0; k < c.n_firs; k++) {
        const stg_vr_fir& f = c.firs[k];
        if (!f.taps || f.n_taps < 1) fail(STG_MODEL_ERROR, "vr: invalid resampling FIR");
        auto& slot = P.firs[{f.src_rate, f.dst_rate}];
        upload(slot.first, std::vector<float>(f.taps, f.taps + f.n_taps), "vr FIR");
        slot.second = f.n_taps;
    }
    // lengths: the analysis chain from the model rate down (vr.cpp:219-225)
    const int B = c.n_bands;
    P.n_in.assign(B, 0);
    P.frames.assign(B, 0);
    int n = P.len, rate = P.sr;
    P.T = INT32_MAX;
    for (int i = B - 1; i >= 0; i--) {
        if (P.bands[i].sample_rate != rate) {
            P.fir(rate, P.bands[i].sample_rate);
            n = resampled(n, rate, P.bands[i].sample_rate);
            rate = P.bands[i].sample_rate;
        }
        P.n_in[i] = n;
        P.frames[i] = n / P.bands[i].hop + 1;
        P.T = std::min(P.T, P.frames[i]);
    }
    if (P.T < 2) fail(STG_INVALID_ARGUMENT, "vr: input shorter than two frames");
    // the synthesis chain from the lowest rate up must land on each band's length (vr.cpp:257-261)
    int ns = P.bands[0].hop * (P.T - 1);
    P.n_syn_max = ns;
    for (int i = 0; i + 1 < B; i++) {
        P.fir(P.bands[i].sample_rate, P.bands[i + 1].sample_rate);
        ns = resampled(ns, P.bands[i].sample_rate, P.bands[i + 1].sample_rate);
        P.n_syn_max = std::max(P.n_syn_max, ns);
        if (ns != P.bands[i + 1].hop * (P.T - 1)) fail(STG_MODEL_ERROR, "vr: synthesis bands do not align");
    }
    // sub-plans and buffers
    int f_max = 0;
    for (int i = 0; i < B; i++) {
        const stg_vr_band& b = P.bands[i];
        auto fw = std::make_unique<stg_plan>();
        fw->engine = P.engine;
        build_torch_stft(fw->H, b.n_fft, b.hop, false, 2, P.n_in[i], false, true);   // vr_stft
        fw->upload_all();
        auto iv = std::make_unique<stg_plan>();
        iv->engine = P.engine;
        build_torch_stft(iv->H, b.n_fft, b.hop, false, 2, (int64_t)b.hop * (P.T - 1), true);   // vr_istft
        iv->upload_all();
        P.stft.push_back(std::move(fw));
        P.istft.push_back(std::move(iv));
        auto w = std::make_unique<DevBuf>();
        if (b.sample_rate != P.sr || i != B - 1) w->reserve(sizeof(float) * 2 * (size_t)P.n_in[i], "vr band input");
        P.wave.push_back(std::move(w));
        auto sb = std::make_unique<DevBuf>();
        sb->reserve(sizeof(float2) * 2 * (size_t)(b.n_fft / 2 + 1) * P.frames[i], "vr band spectrum");
        P.spec_b.push_back(std::move(sb));
        f_max = std::max(f_max, b.n_fft / 2 + 1);
    }
    P.spec.reserve(sizeof(float2) * 2 * (size_t)(P.bins + 1) * P.T, "vr spectrum");
    P.part.reserve(sizeof(float2) * 2 * (size_t)f_max * P.T, "vr band part");
    P.add.reserve(sizeof(float) * 2 * (size_t)P.n_syn_max + 16, "vr band wave");
    P.syn.reserve(sizeof(float) * 2 * (size_t)P.n_syn_max + 16, "vr synthesis");
    P.tmp.reserve(sizeof(float) * 2 * (size_t)P.n_syn_max + 16, "vr synthesis");
}

} // namespace

extern "C" {

STG_API stg_status stg_plan_vr(stg_engine* e, const stg_vr_config* c, int64_t n_samples, stg_vr_plan** out) {
    if (!out) return STG_INVALID_ARGUMENT;
    *out = nullptr;
    if (!e) return STG_INVALID_ARGUMENT;
    return guard(e, [&] {
        if (!c || c->size < sizeof(stg_vr_config)) fail(STG_INVALID_ARGUMENT, "config is NULL or config.size is too small");
        cuda_check(cudaSetDevice(e->device), "cudaSetDevice");
        auto p = std::make_unique<stg_vr_plan>();
        p->engine = e;
        build_vr(*p, *c, n_samples);
        *out = p.release();
    });
}

STG_API void stg_vr_plan_destroy(stg_vr_plan* p) {
    if (!p) return;
    cudaSetDevice(p->engine->device);
    delete p;
}

STG_API stg_status stg_vr_plan_frames(const stg_vr_plan* p, int64_t* n_frames) {
    if (!p || !n_frames) return STG_INVALID_ARGUMENT;
    *n_frames = p->T;
    return STG_OK;
}

STG_API stg_status stg_vr_front(stg_vr_plan* p, const float* d_mix, float* d_mag, float* d_peak, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] { p->front(d_mix, d_mag, d_peak, static_cast<cudaStream_t>(stream)); });
}

STG_API stg_status stg_vr_back(stg_vr_plan* p, const float* d_mask, float* d_out, void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] { p->back(d_mask, d_out, static_cast<cudaStream_t>(stream)); });
}

STG_API stg_status stg_separate_vr(stg_vr_plan* p, const float* d_mix, const float* d_mask, float* d_out,
                                   void* stream) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        p->front(d_mix, nullptr, nullptr, st);
        p->back(d_mask, d_out, st);
    });
}

} // extern "C"
