// engine.cu -- host side of the spectral path: engines, plans (chunk schedules and tables)
// and the C ABI declared in include/stems_gpu_v1.h.
//
// A plan restates, for one model configuration and one track length, what each reference
// separator computes on the host before and around its chunk loop:
//   HTDemucs   src/htdemucs.cpp:534-606  (segments, centre padding, triangular weight)
//   RoFormer   src/roformer.cpp:286-357  (reflect-padded borders, linear fades, tails)
//   TFC-TDF    src/tfc_tdf.cpp:398-495   (UVR trim + np.hanning, or MSST fades)
// and the STFT tables every chunk shares (window, twiddles, the window-sum envelope of
// src/stft.h:130-137 and 185-194). Windows, envelopes and twiddles are computed in double
// with the C library's cos/sin and rounded once to float.
#include "../../include/stems_gpu_v1.h"
#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#define STG_VERSION_STRING "stems-b200 spectral 0.1 (stems_gpu abi 1)"

namespace {

using namespace stg;

struct Failure : std::runtime_error {
    stg_status code;
    Failure(stg_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(stg_status code, const std::string& msg) { throw Failure(code, msg); }

void cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    cudaGetLastError();   // clear a non-sticky launch error so the next call starts clean
    fail(e == cudaErrorMemoryAllocation ? STG_OUT_OF_MEMORY : STG_INTERNAL_ERROR,
         std::string(what) + ": " + cudaGetErrorString(e));
}

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

// ---- STFT tables ----------------------------------------------------------------------------
std::vector<double> hann_periodic(int n) {                        // src/stft.h:70-74
    std::vector<double> w(n);
    for (int i = 0; i < n; i++) w[i] = 0.5 - 0.5 * std::cos(2.0 * M_PI * i / n);
    return w;
}

// 1 / sum_t w^2(q - t*hop) over env_frames frames, for the chunk's output samples j
// (q = j + out_offset); 0 where the sum is not above 1e-11 (src/stft.h:137, 194).
std::vector<float> inv_envelope(int n_fft, int hop, int env_frames, int out_offset, int Lout) {
    const std::vector<double> w = hann_periodic(n_fft);
    std::vector<float> out(Lout);
    for (int j = 0; j < Lout; j++) {
        const int64_t q = (int64_t)j + out_offset;
        int64_t t = (q - n_fft) / hop;
        if (t < 0) t = 0;
        double env = 0.0;
        for (; t < env_frames && t * hop <= q; t++) {
            const int64_t k = q - t * hop;
            if (k < n_fft) env += w[k] * w[k];
        }
        out[j] = env > 1e-11 ? (float)(1.0 / env) : 0.0f;
    }
    return out;
}

// torch.linspace(a, b, n) in float32 from both ends (src/tfc_tdf.cpp:55-62,
// src/roformer.cpp:303-309).
std::vector<float> torch_linspace(float a, float b, int n) {
    std::vector<float> v(std::max(n, 0));
    if (n == 1) v[0] = a;
    if (n < 2) return v;
    const float step = (b - a) / (float)(n - 1);
    for (int i = 0; i < n; i++) v[i] = i < n / 2 ? a + step * (float)i : b - step * (float)(n - 1 - i);
    return v;
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

    const FftTables& fft_tables(int n) {
        auto& t = tables[n];
        if (!t) {
            auto nt = std::make_unique<FftTables>();
            const std::vector<double> w = hann_periodic(n);
            std::vector<float> wf(w.begin(), w.end());
            // per-pass tables of the kernel's radix plan: the pass at stride NS (radix R)
            // holds W_{NS*R}^{k*r} at (NS - 1) + (r - 1)*NS + k
            std::vector<float2> tw(n, make_float2(1.0f, 0.0f));
            int ns = 1;
            for (int R : fused_radices(n)) {
                for (int r = 1; r < R; r++)
                    for (int k = 0; k < ns; k++) {
                        const double th = -2.0 * M_PI * (double)k * r / ((double)ns * R);
                        tw[(ns - 1) + (r - 1) * ns + k] = make_float2((float)std::cos(th), (float)std::sin(th));
                    }
                ns *= R;
            }
            if (ns != n) fail(STG_INTERNAL_ERROR, "radix plan does not multiply to n_fft");
            upload(nt->win, wf, "window table");
            upload(nt->tw, tw, "twiddle table");
            t = std::move(nt);
        }
        return *t;
    }
};

struct stg_plan {
    stg_engine* engine = nullptr;
    int arch = 0;
    int64_t len = 0;
    int C = 2, S = 1, S_out = 1;
    int64_t mask_per_chunk = 0;
    std::vector<ChunkDesc> chunks;
    FrameGeom g{};
    int K = 16, n_tiles = 0;
    float fwd_scale = 1.0f, inv_scale = 1.0f;
    int reflect_global = 0;
    int64_t step_out = 1, out_shift = 0, max_out_len = 0;
    int nan_to_zero = 0, complement = 0;
    float compensate = 1.0f;
    int zero_dc = 0, dim_f = 0, zero_bins = 0, bin_multi = 0;
    int64_t stem_stride = 0;
    DevBuf d_chunks, d_w, d_env, d_btab, d_ebeg, d_ent, d_binv;
    DevBuf d_y, d_tr;
    DevBuf s_mix, s_mask, s_out;   // device staging for stg_separate_host
    int64_t y_chunk_stride = 0, tr_chunk_stride = 0;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};   // fused start, fused end, combine end
    bool timed = false;
    int launches = 0;

    ~stg_plan() {
        for (cudaEvent_t& e : ev)
            if (e) cudaEventDestroy(e);
    }

    int64_t n_chunks() const { return (int64_t)chunks.size(); }
    int64_t out_floats() const { return (int64_t)S_out * C * len; }
    size_t scratch_bytes() const { return d_y.bytes + d_tr.bytes; }
};

namespace {

// Tables shared by every arch, and the scratch the fused kernel writes.
void finish_plan(stg_plan& P, const std::vector<float>& W, int env_frames) {
    const int N = P.g.n_fft, hop = P.g.hop;
    if (!fused_supported(N)) fail(STG_UNSUPPORTED, "n_fft " + std::to_string(N) + " is not implemented");
    if (hop > fused_max_hop(N) || hop > N)
        fail(STG_UNSUPPORTED, "hop " + std::to_string(hop) + " is too large for n_fft " + std::to_string(N));
    if (P.K * hop < N - hop) P.K = (N - hop + hop - 1) / hop;   // one tile boundary per sample at most
    P.n_tiles = (P.g.T + P.K - 1) / P.K;
    P.y_chunk_stride = (int64_t)P.S * P.C * P.g.Lout;
    P.tr_chunk_stride = (int64_t)P.n_tiles * P.S * P.C * (N - hop);
    P.max_out_len = 0;
    for (const ChunkDesc& c : P.chunks) P.max_out_len = std::max<int64_t>(P.max_out_len, c.out_len);
    P.engine->fft_tables(N);
    upload(P.d_chunks, P.chunks, "chunk table");
    upload(P.d_w, W, "weight table");
    upload(P.d_env, inv_envelope(N, hop, env_frames, P.g.out_offset, P.g.Lout), "envelope table");
    P.d_y.reserve(sizeof(float) * (size_t)P.y_chunk_stride * P.chunks.size(), "chunk outputs");
    P.d_tr.reserve(std::max<size_t>(16, sizeof(float) * (size_t)P.tr_chunk_stride * P.chunks.size()),
                   "tile partials");
}

template <class T> bool sized(const T* p) { return p && p->size >= sizeof(uint32_t) * 2; }

// ---- HTDemucs: src/htdemucs.cpp:534-606 ---------------------------------------------------
void plan_htdemucs(stg_plan& P, const stg_htdemucs_config& c, int64_t len) {
    const int N = 4096, hl = N / 4;                                   // htdemucs.cpp:35-36
    if (c.n_channels < 1 || c.n_channels > 2 || c.n_sources < 1 || c.n_sources > 8)
        fail(STG_INVALID_ARGUMENT, "htdemucs: n_channels must be 1..2 and n_sources 1..8");
    const int seg = c.segment;
    const int pad = hl / 2 * 3;
    const int T = (seg + hl - 1) / hl;                                // :320
    if (seg <= pad || seg <= pad + T * hl - seg)                      // stft.h:59 (reflect_pad)
        fail(STG_INVALID_ARGUMENT, "htdemucs: segment too short for the reflect pads");
    const double overlap = c.overlap < 0.0f ? 0.25 : (double)c.overlap;
    if (!(c.overlap < 1.0f)) fail(STG_INVALID_ARGUMENT, "overlap must be < 1");
    const int stride = (int)((1.0 - overlap) * seg);                  // :563-565
    if (stride <= 0) fail(STG_INVALID_ARGUMENT, "overlap must be < 1");
    P.arch = ARCH_HTDEMUCS;
    P.C = c.n_channels; P.S = c.n_sources; P.S_out = P.S;
    P.g = FrameGeom{N, hl, seg, T, 2 * hl, pad, 2 * pad + T * hl, N / 2 + pad, seg};
    P.fwd_scale = (float)(1.0 / std::sqrt((double)N));                // stft.h:91
    P.inv_scale = (float)(std::sqrt((double)N) / N);                  // stft.h:116
    P.reflect_global = 0;                                             // padded(): zeros outside
    P.mask_per_chunk = (int64_t)P.S * 2 * P.C * (N / 2) * T;
    for (int64_t off = 0; off < len; off += stride) {                 // :592
        const int length = (int)std::min<int64_t>(seg, len - off);
        ChunkDesc d{};
        d.src0 = off - (seg - length) / 2;                            // :553-554
        d.valid = seg;
        d.tail_reflect = 0;
        d.out0 = off;
        d.out_len = length;
        d.y_off = (seg - length) / 2;                                 // center_trim (:597)
        d.w_off = 0;
        P.chunks.push_back(d);
    }
    std::vector<float> weight(seg);                                   // :566-573
    const int half = seg / 2;
    for (int i = 0; i < half; i++) weight[i] = (float)(i + 1);
    for (int i = half; i < seg; i++) weight[i] = (float)(seg - i);
    const float mx = *std::max_element(weight.begin(), weight.end());
    for (float& w : weight) w /= mx;
    P.step_out = stride;
    P.out_shift = 0;
    P.nan_to_zero = 0;
    finish_plan(P, weight, T + 4);                                    // 2 zero frames per side
}

// ---- RoFormer: src/roformer.cpp:286-357, 394-411, 436-486 -------------------------------
void plan_roformer(stg_plan& P, const stg_roformer_config& c, int64_t len) {
    if (c.n_channels < 1 || c.n_channels > 2 || c.n_stems < 1 || c.n_stems > 8)
        fail(STG_INVALID_ARGUMENT, "roformer: n_channels must be 1..2 and n_stems 1..8");
    if (c.hop < 1 || c.chunk < 1 || c.chunk % c.hop)
        fail(STG_MODEL_ERROR, "roformer: chunk_size is not a multiple of the hop");   // :396
    if (c.n_bands < 1 || !c.band_sizes || !c.band_freqs) fail(STG_MODEL_ERROR, "roformer: no band table");
    if (!(c.overlap < 1.0f)) fail(STG_INVALID_ARGUMENT, "overlap must be < 1");           // :440
    if (c.overlap < 0.0f && c.num_overlap < 1) fail(STG_MODEL_ERROR, "roformer: num_overlap < 1");
    const int N = c.n_fft, hop = c.hop, Cc = c.chunk, F = N / 2 + 1;
    const int step = c.overlap < 0.0f ? Cc / c.num_overlap
                                      : std::max(1, (int)std::lround(Cc * (1.0 - c.overlap)));   // :442-443
    if (step < 1) fail(STG_INVALID_ARGUMENT, "roformer: step < 1");
    if (Cc <= N / 2) fail(STG_INVALID_ARGUMENT, "roformer: chunk shorter than the STFT reflect pad");
    P.arch = ARCH_ROFORMER;
    P.C = c.n_channels; P.S = c.n_stems; P.S_out = P.S + (c.complement ? 1 : 0);
    const int T = Cc / hop + 1;                                       // :83
    P.g = FrameGeom{N, hop, Cc, T, 0, 0, 0, N / 2, hop * (T - 1)};
    P.fwd_scale = c.normalized ? (float)(1.0 / std::sqrt((double)N)) : 1.0f;
    P.inv_scale = (float)((c.normalized ? std::sqrt((double)N) : 1.0) / N);
    P.zero_dc = c.zero_dc != 0;
    // band table (:394-411) -> per-bin inverse table
    std::vector<int> bpf(F, 0);
    std::vector<std::vector<int2>> per_bin(F);
    int64_t off = 0, foff = 0;
    for (int b = 0; b < c.n_bands; b++) {
        const int sz = c.band_sizes[b];
        if (sz < 1) fail(STG_MODEL_ERROR, "roformer: empty band");
        const int din = sz * P.C * 2;                                 // :85
        if (din > 0xffff) fail(STG_UNSUPPORTED, "roformer: band too wide");
        for (int j = 0; j < sz; j++) {
            const int f = c.band_freqs[foff + j];
            if (f < 0 || f >= F) fail(STG_MODEL_ERROR, "roformer: band frequency out of range");
            bpf[f]++;
            per_bin[f].push_back(make_int2((int)(off * T + (int64_t)j * P.C * 2), din));
        }
        foff += sz;
        off += din;
    }
    if (off * T > INT32_MAX) fail(STG_UNSUPPORTED, "roformer: band table too large");
    P.stem_stride = off * T;
    P.mask_per_chunk = (int64_t)P.S * P.stem_stride;
    std::vector<int> ebeg(F + 1, 0);
    std::vector<int2> ent;
    std::vector<float> binv(F);
    // bin_tab[f]: the first two bands holding f, each as (entry offset without the frame term)
    // / (2C) in bits 0-21 | band size in bits 22-31; 0 when absent. A bin no band holds gets
    // weight 0: its mask average is 0 / 1 (src/roformer.cpp:272).
    std::vector<int2> btab(F, make_int2(0, 0));
    int multi = 0;
    for (int f = 0; f < F; f++) {
        ebeg[f] = (int)ent.size();
        ent.insert(ent.end(), per_bin[f].begin(), per_bin[f].end());
        binv[f] = per_bin[f].empty() ? 0.0f : (float)(1.0 / bpf[f]);
        const size_t n = per_bin[f].size();
        int v[2] = {0, 0};
        for (size_t k = 0; k < n && k < 2; k++) {
            const int units = per_bin[f][k].x / (P.C * 2), size = per_bin[f][k].y / (P.C * 2);
            if (units >= (1 << 22) || size >= (1 << 10)) fail(STG_UNSUPPORTED, "roformer: band table too large");
            v[k] = (int)((unsigned)units | ((unsigned)size << 22));
        }
        btab[f] = make_int2(v[0], v[1]);
        if (n > 2) multi = 1;
    }
    P.bin_multi = multi;
    ebeg[F] = (int)ent.size();
    upload(P.d_btab, btab, "band table");
    upload(P.d_ebeg, ebeg, "band table");
    upload(P.d_ent, ent, "band table");
    upload(P.d_binv, binv, "band table");
    // chunking (:288-341)
    const int fade = Cc / 10, border = Cc - step;
    const bool pad = len > 2 * (int64_t)border && border > 0;
    const int64_t Lp = pad ? len + 2 * (int64_t)border : len;
    std::vector<float> fade_in(std::max(fade, 0), 0.0f);
    if (fade > 1) {
        const float stp = 1.0f / (float)(fade - 1);
        for (int i = 0; i < fade; i++) fade_in[i] = i < fade / 2 ? (float)i * stp : 1.0f - (float)(fade - 1 - i) * stp;
    }
    std::vector<float> window(Cc, 1.0f);
    for (int i = 0; i < fade; i++) { window[i] *= fade_in[i]; window[Cc - 1 - i] *= fade_in[i]; }
    // weight tables: [normal][first][last]
    std::vector<float> W((size_t)3 * Cc);
    for (int v = 0; v < 3; v++) {
        float* w = &W[(size_t)v * Cc];
        std::copy(window.begin(), window.end(), w);
        if (v == 1) std::fill(w, w + fade, 1.0f);                     // :335
        if (v == 2) std::fill(w + Cc - fade, w + Cc, 1.0f);           // :336
    }
    for (int64_t i = 0; i < Lp; i += step) {                          // :317
        const int length = (int)std::min<int64_t>(Cc, Lp - i);
        ChunkDesc d{};
        d.src0 = i - (pad ? border : 0);
        d.valid = length;
        d.tail_reflect = length < Cc && length > Cc / 2 + 1;          // :323-330
        d.out0 = i;
        d.out_len = length;
        d.y_off = 0;
        d.w_off = i == 0 ? Cc : (i + Cc >= Lp ? 2 * Cc : 0);
        P.chunks.push_back(d);
    }
    P.reflect_global = pad;
    P.step_out = step;
    P.out_shift = pad ? border : 0;                                   // :344
    P.nan_to_zero = 1;                                                // :348
    P.complement = c.complement ? 1 : 0;                              // :481-485
    P.K = 16;
    finish_plan(P, W, T);
}

// ---- TFC-TDF: src/tfc_tdf.cpp:398-495, 570-598 -------------------------------------------
void plan_tfc(stg_plan& P, const stg_tfc_config& c, int64_t len) {
    if (c.n_stems < 1 || c.n_stems > 7) fail(STG_INVALID_ARGUMENT, "tfc_tdf: n_stems must be 1..7");
    const int N = c.n_fft, hop = c.hop;
    if (N < 16 || N % 2 || hop < 1 || hop > N || c.dim_f < 1 || c.dim_f > N / 2 + 1 || c.dim_t < 2 ||
        c.zero_bins < 0 || c.zero_bins > c.dim_f || (c.chunking != 0 && c.chunking != 1) ||
        (c.chunking == 1 && c.num_overlap < 1) || !std::isfinite(c.compensate) || c.compensate <= 0)
        fail(STG_MODEL_ERROR, "tfc_tdf: invalid configuration");      // :537-549
    if (!(c.overlap < 1.0f)) fail(STG_INVALID_ARGUMENT, "overlap must be < 1");
    const int Cc = hop * (c.dim_t - 1);                               // :94
    if (Cc <= N / 2) fail(STG_MODEL_ERROR, "tfc_tdf: chunk shorter than the FFT");
    P.arch = ARCH_TFC;
    P.C = 2; P.S = c.n_stems; P.S_out = P.S + (c.complement ? 1 : 0);
    P.g = FrameGeom{N, hop, Cc, c.dim_t, 0, 0, 0, N / 2, Cc};
    P.fwd_scale = 1.0f;
    P.inv_scale = (float)(1.0 / N);
    P.dim_f = c.dim_f;
    P.zero_bins = c.chunking == 0 ? c.zero_bins : 0;                  // :532
    P.mask_per_chunk = (int64_t)4 * P.S * c.dim_f * c.dim_t;
    std::vector<float> W;
    if (c.chunking == 0) {                                            // demix_uvr :398-429
        const int trim = N / 2, gen = Cc - 2 * trim;
        if (gen <= 0) fail(STG_MODEL_ERROR, "tfc_tdf: chunk shorter than the FFT");
        const int64_t M = (int64_t)trim + len + gen + trim - len % gen;
        const int64_t step = c.overlap < 0 ? Cc - N : (int64_t)((1.0 - (double)c.overlap) * Cc);
        if (step <= 0) fail(STG_INVALID_ARGUMENT, "overlap too large for this model");
        std::map<int, int> table_of;   // chunk length -> offset of its np.hanning table
        for (int64_t i = 0; i < M; i += step) {
            const int actual = (int)std::min<int64_t>(Cc, M - i);
            auto it = table_of.find(actual);
            if (it == table_of.end()) {
                const int o = (int)W.size();
                for (int k = 0; k < actual; k++)                      // np.hanning (:65-70), or ones
                    W.push_back(c.overlap == 0 || actual == 1 ? 1.0f
                                : (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * k / (actual - 1))));
                it = table_of.emplace(actual, o).first;
            }
            ChunkDesc d{};
            d.src0 = i - trim;
            d.valid = actual;
            d.tail_reflect = 0;
            d.out0 = i;
            d.out_len = actual;
            d.y_off = 0;
            d.w_off = it->second;
            P.chunks.push_back(d);
        }
        P.reflect_global = 0;
        P.step_out = step;
        P.out_shift = trim;
        P.nan_to_zero = 0;
    } else {                                                          // demix_msst :434-495
        const int step = c.overlap < 0 ? Cc / c.num_overlap
                                       : std::max(1, (int)std::lround(Cc * (1.0 - c.overlap)));
        const int fade = Cc / 10, border = Cc - step;
        const bool pad = len > 2 * (int64_t)border && border > 0;
        const int64_t Lp = pad ? len + 2 * (int64_t)border : len;
        std::vector<float> window(Cc, 1.0f);
        if (fade > 0) {
            const std::vector<float> in = torch_linspace(0, 1, fade), out = torch_linspace(1, 0, fade);
            std::copy(out.begin(), out.end(), window.end() - fade);
            std::copy(in.begin(), in.end(), window.begin());
        }
        W.resize((size_t)3 * Cc);
        for (int v = 0; v < 3; v++) {
            float* w = &W[(size_t)v * Cc];
            std::copy(window.begin(), window.end(), w);
            if (v == 1) std::fill(w, w + fade, 1.0f);                 // :480
            if (v == 2) std::fill(w + Cc - fade, w + Cc, 1.0f);       // :481
        }
        for (int64_t i = 0; i < Lp; i += step) {
            const int n = (int)std::min<int64_t>(Cc, Lp - i);
            ChunkDesc d{};
            d.src0 = i - (pad ? border : 0);
            d.valid = n;
            d.tail_reflect = n < Cc && n > Cc / 2;                    // :467-474
            d.out0 = i;
            d.out_len = n;
            d.y_off = 0;
            d.w_off = i == 0 ? Cc : (i + step >= Lp ? 2 * Cc : 0);
            P.chunks.push_back(d);
        }
        P.reflect_global = pad;
        P.step_out = step;
        P.out_shift = pad ? border : 0;
        P.nan_to_zero = 1;
    }
    P.compensate = c.compensate;                                      // :586-587
    P.complement = c.complement ? 2 : 0;                              // :588-596
    P.K = 16;
    finish_plan(P, W, c.dim_t);
}

void run_plan(stg_plan& P, const float* d_mix, const float* d_mask, float* d_out, cudaStream_t st,
              const stg_run_options* opt) {
    if (!d_mix || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
    if (reinterpret_cast<uintptr_t>(d_mask) % 16) fail(STG_INVALID_ARGUMENT, "mask must be 16-byte aligned");
    cuda_check(cudaSetDevice(P.engine->device), "cudaSetDevice");
    const FftTables& tabs = P.engine->fft_tables(P.g.n_fft);
    FusedParams f{};
    f.mix = d_mix; f.len = P.len; f.n_channels = P.C; f.reflect_global = P.reflect_global;
    f.g = P.g; f.K = P.K; f.n_tiles = P.n_tiles; f.S = P.S;
    f.win = tabs.win.as<float>(); f.tw = tabs.tw.as<float2>(); f.inv_env = P.d_env.as<float>();
    f.fwd_scale = P.fwd_scale; f.inv_scale = P.inv_scale;
    f.mask_chunk_stride = P.mask_per_chunk;
    f.bin_tab = P.d_btab.as<int2>();
    f.bin_multi = P.bin_multi;
    f.bin_ebeg = P.d_ebeg.as<int>(); f.bin_ent = P.d_ent.as<int2>(); f.bin_inv = P.d_binv.as<float>();
    f.zero_dc = P.zero_dc; f.stem_stride = P.stem_stride;
    f.dim_f = P.dim_f; f.zero_bins = P.zero_bins;
    f.y_chunk_stride = P.y_chunk_stride; f.tr_chunk_stride = P.tr_chunk_stride;
    const int G = (int)P.chunks.size();
    const int per = (opt && opt->chunks_per_batch > 0) ? opt->chunks_per_batch : G;
    P.timed = P.engine->profiling;
    P.launches = 0;
    if (P.timed) {
        for (cudaEvent_t& e : P.ev)
            if (!e) cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        cuda_check(cudaEventRecord(P.ev[0], st), "cudaEventRecord");
    }
    for (int b0 = 0; b0 < G; b0 += per) {
        if (opt && opt->should_cancel && opt->should_cancel(opt->user)) fail(STG_CANCELLED, "cancelled");
        const int nb = std::min(per, G - b0);
        f.chunks = P.d_chunks.as<ChunkDesc>() + b0;
        f.n_chunks = nb;
        f.mask = d_mask + (int64_t)b0 * P.mask_per_chunk;
        f.Y = P.d_y.as<float>() + (int64_t)b0 * P.y_chunk_stride;
        f.Tr = P.d_tr.as<float>() + (int64_t)b0 * P.tr_chunk_stride;
        cuda_check(launch_fused(P.arch, f, st), "fused spectral kernel launch");
        P.launches++;
        if (opt && opt->on_progress) {
            cuda_check(cudaStreamSynchronize(st), "fused spectral kernel");
            opt->on_progress(opt->user, b0 + nb, G);
        }
    }
    CombineParams c{};
    c.Y = P.d_y.as<float>(); c.y_chunk_stride = P.y_chunk_stride;
    c.Tr = P.d_tr.as<float>(); c.tr_chunk_stride = P.tr_chunk_stride;
    c.chunks = P.d_chunks.as<ChunkDesc>(); c.n_chunks = G;
    c.step_out = P.step_out; c.max_out_len = P.max_out_len;
    c.g = P.g; c.K = P.K; c.n_tiles = P.n_tiles;
    c.W = P.d_w.as<float>();
    c.S = P.S; c.C = P.C; c.len = P.len; c.out_shift = P.out_shift;
    c.mode = P.arch; c.nan_to_zero = P.nan_to_zero; c.compensate = P.compensate;
    c.complement = P.complement; c.mix = d_mix; c.out = d_out;
    if (P.timed) cuda_check(cudaEventRecord(P.ev[1], st), "cudaEventRecord");
    cuda_check(launch_combine(c, st), "combine kernel launch");
    P.launches++;
    if (P.timed) cuda_check(cudaEventRecord(P.ev[2], st), "cudaEventRecord");
}

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
        p->len = n;
        build(*p, *cfg, n);
        *out = p.release();
    });
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
        if (!p->timed) fail(STG_INVALID_ARGUMENT, "the last run was not timed (stg_engine_set_profiling)");
        cuda_check(cudaEventSynchronize(p->ev[2]), "cudaEventSynchronize");
        float a = 0.0f, b = 0.0f;
        cuda_check(cudaEventElapsedTime(&a, p->ev[0], p->ev[1]), "cudaEventElapsedTime");
        cuda_check(cudaEventElapsedTime(&b, p->ev[1], p->ev[2]), "cudaEventElapsedTime");
        if (fused_ms) *fused_ms = a;
        if (combine_ms) *combine_ms = b;
        if (launches) *launches = p->launches;
    });
}

STG_API stg_status stg_plan_htdemucs(stg_engine* e, const stg_htdemucs_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, plan_htdemucs);
}
STG_API stg_status stg_plan_roformer(stg_engine* e, const stg_roformer_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, plan_roformer);
}
STG_API stg_status stg_plan_tfc(stg_engine* e, const stg_tfc_config* c, int64_t n, stg_plan** out) {
    return make_plan(e, c, n, out, plan_tfc);
}

STG_API void stg_plan_destroy(stg_plan* p) {
    if (!p) return;
    cudaSetDevice(p->engine->device);
    delete p;
}

STG_API stg_status stg_plan_get_info(const stg_plan* p, stg_plan_info* info) {
    if (!p || !info || info->size < sizeof(stg_plan_info)) return STG_INVALID_ARGUMENT;
    info->arch = p->arch;
    info->n_samples = p->len;
    info->n_channels = p->C;
    info->n_out_sources = p->S_out;
    info->n_chunks = p->n_chunks();
    info->n_frames = p->g.T;
    info->mask_floats_per_chunk = p->mask_per_chunk;
    info->out_floats = p->out_floats();
    info->scratch_bytes = (int64_t)p->scratch_bytes();
    return STG_OK;
}

STG_API stg_status stg_separate_ex(stg_plan* p, const float* d_mix, const float* d_mask, float* d_out,
                                   void* stream, const stg_run_options* opt) {
    if (!p) return STG_INVALID_ARGUMENT;
    return guard(p->engine, [&] {
        if (opt && opt->size < sizeof(stg_run_options)) fail(STG_INVALID_ARGUMENT, "options.size is too small");
        run_plan(*p, d_mix, d_mask, d_out, static_cast<cudaStream_t>(stream), opt);
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
        const size_t mix_b = sizeof(float) * (size_t)p->C * p->len;
        const size_t mask_b = sizeof(float) * (size_t)p->mask_per_chunk * p->chunks.size();
        const size_t out_b = sizeof(float) * (size_t)p->out_floats();
        p->s_mix.reserve(mix_b, "staging");
        p->s_mask.reserve(mask_b, "staging");
        p->s_out.reserve(out_b, "staging");
        cuda_check(cudaMemcpyAsync(p->s_mix.p, h_mix, mix_b, cudaMemcpyHostToDevice, st), "copy mix in");
        cuda_check(cudaMemcpyAsync(p->s_mask.p, h_mask, mask_b, cudaMemcpyHostToDevice, st), "copy masks in");
        run_plan(*p, p->s_mix.as<float>(), p->s_mask.as<float>(), p->s_out.as<float>(), st, nullptr);
        cuda_check(cudaMemcpyAsync(h_out, p->s_out.p, out_b, cudaMemcpyDeviceToHost, st), "copy result out");
        cuda_check(cudaStreamSynchronize(st), "separation");
    });
}

} // extern "C"
