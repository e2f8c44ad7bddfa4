// plan.cu -- see plan.h. Windows, envelopes and twiddles are computed in double with the C
// library's cos/sin and rounded once to float.
#include "plan.h"

#include <random>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>

namespace stg {

void fail(stg_status code, const std::string& msg) { throw Failure(code, msg); }

void cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    cudaGetLastError();   // clear a non-sticky launch error so the next call starts clean
    fail(e == cudaErrorMemoryAllocation ? STG_OUT_OF_MEMORY : STG_INTERNAL_ERROR,
         std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {

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

// Sizes shared by every arch, and the window-sum envelope of a chunk's output.
void finish_plan(HostPlan& P, int env_frames) {
    const int N = P.g.n_fft, hop = P.g.hop;
    // single-chunk primitives run the front and back kernels only; plans also the fused one
    if (P.primitive ? !split_supported(N) : !fused_supported(N))
        fail(STG_UNSUPPORTED, "n_fft " + std::to_string(N) + " is not implemented");
    if (hop > (P.primitive ? split_max_hop(N) : fused_max_hop(N)) || hop > N)
        fail(STG_UNSUPPORTED, "hop " + std::to_string(hop) + " is too large for n_fft " + std::to_string(N));
    // Frames per tile. The persistent CTAs take work items (chunk, tile) round-robin, so a
    // launch lasts ceil(items / resident CTAs) rounds of one tile each; a tile costs its K
    // frames plus about one frame of prologue (the first window) and flush. K is the one in
    // [K_min, 16] with the shortest critical path, the larger on ties. K_min keeps every
    // sample within one tile boundary (K * hop >= n_fft - hop).
    // (HTDemucs separations run the back kernel over the chunks, the others the fused one)
    // (single-chunk primitives run the front and back kernels: the fewer resident of the two)
    // (TFC-TDF at n_fft 7680 runs on CTA pairs: a work slot is a cluster)
    const int64_t slots = std::max(1, P.primitive ? std::min(split_resident_ctas(N, true), split_resident_ctas(N, false))
                                      : P.arch == ARCH_HTDEMUCS ? back_resident_ctas(N)
                                      : fused_pair(P.arch, N, hop) ? fused_pair_slots()
                                                                   : fused_resident_ctas(P.arch, N));
    const int k_min = std::max(1, (N - hop + hop - 1) / hop);
    P.K = std::max(16, k_min);
    int64_t best = INT64_MAX;
    // HTDemucs separations: the front kernel's items are (chunk, tile), the back kernel's
    // (chunk, tile, stem); a frame costs about the same in both, so their rounds add up
    const bool ht = P.arch == ARCH_HTDEMUCS && !P.primitive;
    const int64_t front_slots = ht ? std::max(1, split_resident_ctas(N, true)) : 1;
    for (int K = std::max(16, k_min); K >= k_min; K--) {
        const int64_t items = (int64_t)P.chunks.size() * ((P.g.T + K - 1) / K);
        const int64_t cost = ht ? ((items * P.S + slots - 1) / slots + (items + front_slots - 1) / front_slots) * (K + 1)
                                : (items + slots - 1) / slots * (K + 1);
        if (cost < best) { best = cost; P.K = K; }
    }
    P.n_tiles = (P.g.T + P.K - 1) / P.K;
    // chunks of the plain track (no shift pass): the mix itself, reflected as the plan says
    for (ChunkDesc& d : P.chunks)
        if (d.vlen == 0) {
            d.vlen = P.len;
            d.vshift = 0;
            d.reflect = P.reflect_global;
        }
    if (P.groups.empty()) {
        if (P.out_shift > INT32_MAX) fail(STG_INVALID_ARGUMENT, "input is too long");
        P.groups.push_back(ChunkGroup{0, (int32_t)P.chunks.size(), (int32_t)P.out_shift, 0});
    }
    P.y_chunk_stride = (int64_t)P.S * P.C * P.g.Lout;
    P.tr_chunk_stride = (int64_t)P.n_tiles * P.S * P.C * (N - hop);
    P.max_out_len = 0;
    for (const ChunkDesc& c : P.chunks) P.max_out_len = std::max<int64_t>(P.max_out_len, c.out_len);
    P.env = inv_envelope(N, hop, env_frames, P.g.out_offset, P.g.Lout);
    // Where every frame overlapping a sample exists, the window sum repeats every hop, bit for
    // bit (the same squares summed in the same order): the kernels read that stretch from a
    // hop-long table in shared memory instead of the envelope in global memory.
    P.env_lo = P.env_hi = 0;
    P.env_period.clear();
    {
        const int lo = std::max(0, N - P.g.out_offset);
        const int hi = std::min(P.g.Lout, env_frames * hop - P.g.out_offset);
        bool periodic = hi - lo >= hop;
        for (int j = lo + hop; periodic && j < hi; j++) periodic = P.env[j] == P.env[j - hop];
        if (periodic) {
            P.env_lo = lo;
            P.env_hi = hi;
            P.env_period.assign(P.env.begin() + lo, P.env.begin() + lo + hop);
        }
    }
}

} // namespace

void fft_twiddles(int n, const std::vector<int>& radices, std::vector<float2>& tw) {
    // per-pass tables of a radix plan: the pass at stride NS (radix R) holds W_{NS*R}^{k*r} at
    // (NS - 1) + (r - 1)*NS + k (fft.cuh: twiddle_index)
    tw.assign(n, make_float2(1.0f, 0.0f));
    int ns = 1;
    for (int R : radices) {
        for (int r = 1; r < R; r++)
            for (int k = 0; k < ns; k++) {
                const double th = -2.0 * M_PI * (double)k * r / ((double)ns * R);
                tw[(ns - 1) + (r - 1) * ns + k] = make_float2((float)std::cos(th), (float)std::sin(th));
            }
        ns *= R;
    }
    if (ns != n) fail(STG_INTERNAL_ERROR, "radix plan does not multiply to n_fft");
}

void fft_tables(int n, std::vector<float>& win, std::vector<float2>& tw) {
    const std::vector<double> w = hann_periodic(n);
    win.assign(w.begin(), w.end());
    fft_twiddles(n, fused_radices(n), tw);
    // a forward plan of its own (n_fft 2048): its table right after
    const std::vector<int> fr = fused_fwd_radices(n);
    if (!fr.empty()) {
        std::vector<float2> f;
        fft_twiddles(n, fr, f);
        tw.insert(tw.end(), f.begin(), f.end());
    }
    // the CTA-pair kernel's tables after them: its half-length plan, then W_n^k for k < n/2
    const std::vector<int> pr = fused_pair_radices(n);
    if (!pr.empty()) {
        std::vector<float2> h;
        fft_twiddles(n / 2, pr, h);
        tw.insert(tw.end(), h.begin(), h.end());
        for (int k = 0; k < n / 2; k++) {
            const double th = -2.0 * M_PI * (double)k / (double)n;
            tw.push_back(make_float2((float)std::cos(th), (float)std::sin(th)));
        }
    }
}

// The offsets of the random-shift passes: std::mt19937 seeded with `seed`, one draw of
// std::uniform_int_distribution<int>(0, hi) per pass, as the separators draw them
// (src/htdemucs.cpp:578, 617-619; src/roformer.cpp:461-465). The same standard library
// produces the same sequence.
static std::vector<int> shift_offsets(uint32_t seed, int shifts, int hi) {
    std::mt19937 rng(seed);
    std::uniform_int_distribution<int> dist(0, hi);
    std::vector<int> v(shifts);
    for (int& o : v) o = dist(rng);
    return v;
}

// ---- HTDemucs: src/htdemucs.cpp:534-626 ---------------------------------------------------
void build_htdemucs(HostPlan& P, const stg_htdemucs_config& c, int64_t len) {
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
    P.mono_norm = c.mono_norm != 0;                                   // :539-549, 638-642
    P.cac_norm = c.cac_norm != 0;                                     // :434-436, 466-469
    P.g = FrameGeom{N, hl, seg, T, 2 * hl, pad, 2 * pad + T * hl, N / 2 + pad, seg};
    P.fwd_scale = (float)(1.0 / std::sqrt((double)N));                // stft.h:91
    P.inv_scale = (float)(std::sqrt((double)N) / N);                  // stft.h:116
    P.reflect_global = 0;                                             // padded(): zeros outside
    P.mask_per_chunk = (int64_t)P.S * 2 * P.C * (N / 2) * T;
    P.mask_planes = 2 * P.C;
    P.mask_bins = N / 2;
    // split() over one view of the (zero-padded) mix: segments of the view, each read with
    // real samples around it where the buffer has them (:552-561, 588-606). view0 is the mix
    // coordinate of the view's sample 0; output sample i of the track is view sample
    // i + out_shift.
    auto split_view = [&](int64_t view0, int64_t view_len, int out_shift) {
        const int c0 = (int)P.chunks.size();
        for (int64_t off = 0; off < view_len; off += stride) {        // :592
            const int length = (int)std::min<int64_t>(seg, view_len - off);
            ChunkDesc d{};
            d.src0 = view0 + off - (seg - length) / 2;                // :553-554
            d.vlen = len;
            d.vshift = 0;
            d.reflect = 0;                                            // padded(): zeros outside
            d.valid = seg;
            d.tail_reflect = 0;
            d.out0 = off;
            d.out_len = length;
            d.y_off = (seg - length) / 2;                             // center_trim (:597)
            d.w_off = 0;
            P.chunks.push_back(d);
        }
        P.groups.push_back(ChunkGroup{c0, (int32_t)P.chunks.size(), out_shift, 0});
    };
    const int shifts = std::max(0, c.shifts);                         // :575
    if (shifts == 0) {
        split_view(0, len, 0);                                        // :610-611
    } else {
        // views [offset, offset + len + max_shift - offset) of the mix padded by max_shift
        // zeros per side; offset uniform in [0, max_shift] (:612-626)
        const int max_shift = (c.sample_rate > 0 ? c.sample_rate : 44100) / 2;
        for (int offset : shift_offsets(c.seed, shifts, max_shift))
            split_view((int64_t)offset - max_shift, len + max_shift - offset, max_shift - offset);
        P.shift_mean = 1;                                             // sum, then / shifts (:626)
    }
    std::vector<float>& weight = P.W;                                 // :566-573
    weight.assign(seg, 0.0f);
    const int half = seg / 2;
    for (int i = 0; i < half; i++) weight[i] = (float)(i + 1);
    for (int i = half; i < seg; i++) weight[i] = (float)(seg - i);
    const float mx = *std::max_element(weight.begin(), weight.end());
    for (float& w : weight) w /= mx;
    P.step_out = stride;
    P.out_shift = 0;
    P.nan_to_zero = 0;
    P.front_layout = FRONT_CAC;                                       // in_x (:423-433)
    P.back_layout = BACK_CAC;                                         // ox (:463-469)
    P.front_bins = P.back_bins = N / 2;
    P.net_in_per_chunk = (int64_t)2 * P.C * (N / 2) * T;
    P.net_out_per_chunk = P.mask_per_chunk;
    // bag of models (:585-642): weights [n_models][S], their sums per stem
    P.n_models = std::max(1, c.n_models);
    if (c.n_models > 64) fail(STG_INVALID_ARGUMENT, "htdemucs: at most 64 models in a bag");
    if (c.n_models > 1 || c.bag_weights) {
        P.bag.assign((size_t)P.n_models * P.S, 1.0f);
        if (c.bag_weights) std::copy(c.bag_weights, c.bag_weights + P.bag.size(), P.bag.begin());
        P.bag_tot.assign(P.S, 0.0f);
        for (int m = 0; m < P.n_models; m++)
            for (int s = 0; s < P.S; s++) {
                const float w = P.bag[(size_t)m * P.S + s];
                if (!std::isfinite(w)) fail(STG_MODEL_ERROR, "htdemucs: bag weight is not finite");
                P.bag_tot[s] += w;                                    // float sums in model order (:631)
            }
    }
    // progress (:576-577): models x passes x ceil(len / stride) segment passes
    P.progress_total = (int)std::min<int64_t>(INT32_MAX, (int64_t)P.n_models * std::max(1, shifts) *
                                                             ((len + stride - 1) / stride));
    finish_plan(P, T + 4);                                            // 2 zero frames per side
}

// ---- RoFormer: src/roformer.cpp:286-357, 394-411, 436-486 -------------------------------
void build_roformer(HostPlan& P, const stg_roformer_config& c, int64_t len) {
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
    std::vector<int>& ebeg = P.ebeg;
    std::vector<int2>& ent = P.ent;
    std::vector<float>& binv = P.binv;
    ebeg.assign(F + 1, 0);
    binv.assign(F, 0.0f);
    // bin_tab[f]: the first two bands holding f, each as (entry offset without the frame term)
    // / (2C) in bits 0-21 | band size in bits 22-31; 0 when absent. A bin no band holds gets
    // weight 0: its mask average is 0 / 1 (src/roformer.cpp:272).
    std::vector<int2>& btab = P.btab;
    btab.assign(F, make_int2(0, 0));
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
    // chunking (:288-341)
    const int fade = Cc / 10, border = Cc - step;
    const bool pad = len > 2 * (int64_t)border && border > 0;
    std::vector<float> fade_in(std::max(fade, 0), 0.0f);
    if (fade > 1) {
        const float stp = 1.0f / (float)(fade - 1);
        for (int i = 0; i < fade; i++) fade_in[i] = i < fade / 2 ? (float)i * stp : 1.0f - (float)(fade - 1 - i) * stp;
    }
    std::vector<float> window(Cc, 1.0f);
    for (int i = 0; i < fade; i++) { window[i] *= fade_in[i]; window[Cc - 1 - i] *= fade_in[i]; }
    // weight tables: [normal][first][last]
    std::vector<float>& W = P.W;
    W.assign((size_t)3 * Cc, 0.0f);
    for (int v = 0; v < 3; v++) {
        float* w = &W[(size_t)v * Cc];
        std::copy(window.begin(), window.end(), w);
        if (v == 1) std::fill(w, w + fade, 1.0f);                     // :335
        if (v == 2) std::fill(w + Cc - fade, w + Cc, 1.0f);           // :336
    }
    // demix() of one track of n samples, the mix's sample x + vshift at its sample x (zero
    // outside the mix); output sample i of the separation is the track's sample i + out_extra.
    auto demix = [&](int64_t n, int64_t vshift, int out_extra) {
        const bool pad_n = n > 2 * (int64_t)border && border > 0;      // :290-299
        const int64_t Lp_n = pad_n ? n + 2 * (int64_t)border : n;
        const int c0 = (int)P.chunks.size();
        for (int64_t i = 0; i < Lp_n; i += step) {                    // :317
            const int length = (int)std::min<int64_t>(Cc, Lp_n - i);
            ChunkDesc d{};
            d.src0 = i - (pad_n ? border : 0);
            d.vlen = n;
            d.vshift = vshift;
            d.reflect = pad_n;
            d.valid = length;
            d.tail_reflect = length < Cc && length > Cc / 2 + 1;      // :323-330
            d.out0 = i;
            d.out_len = length;
            d.y_off = 0;
            d.w_off = i == 0 ? Cc : (i + Cc >= Lp_n ? 2 * Cc : 0);
            P.chunks.push_back(d);
        }
        P.groups.push_back(ChunkGroup{c0, (int32_t)P.chunks.size(), (pad_n ? border : 0) + out_extra, 0});   // :344
    };
    if (c.shifts <= 0) {
        demix(len, 0, 0);                                             // :456-457
    } else {
        // tracks of len + max_shift - offset samples, the mix behind max_shift - offset zeros;
        // offset uniform in [0, max_shift - 1] (:458-478)
        const int max_shift = (c.sample_rate > 0 ? c.sample_rate : 44100) / 2;
        for (int offset : shift_offsets(c.seed, c.shifts, max_shift - 1))
            demix(len + max_shift - offset, (int64_t)offset - max_shift, max_shift - offset);
        P.shift_mean = 2;                                             // y / shifts, summed (:476)
    }
    P.reflect_global = pad;
    P.step_out = step;
    P.out_shift = pad ? border : 0;
    P.nan_to_zero = 1;                                                // :348
    P.complement = c.complement ? 1 : 0;                              // :481-485
    P.front_layout = FRONT_BANDS;                                     // feat (:226-241)
    P.front_bins = F;
    P.net_in_per_chunk = P.stem_stride;
    P.net_out_per_chunk = P.mask_per_chunk;                           // masks (:251-269)
    P.back_is_fused = true;
    // progress (:444-451, 479): passes x the chunks of one pass over the track itself, the last
    // report (total, total)
    {
        const int64_t Lp = pad ? len + 2 * (int64_t)border : len;
        P.progress_total = (int)std::min<int64_t>(INT32_MAX, (int64_t)std::max(1, c.shifts) * ((Lp + step - 1) / step));
        P.progress_final_total = true;
    }
    finish_plan(P, T);
}

// ---- TFC-TDF: src/tfc_tdf.cpp:398-495, 570-598 -------------------------------------------
void build_tfc(HostPlan& P, const stg_tfc_config& c, int64_t len) {
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
    P.mask_planes = 4;
    P.mask_bins = c.dim_f;
    std::vector<float>& W = P.W;
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
    P.front_layout = FRONT_TFC;                                       // in (:366-376)
    P.back_layout = BACK_TFC;                                         // y (:381-387)
    P.front_bins = P.back_bins = c.dim_f;
    P.net_in_per_chunk = (int64_t)4 * c.dim_f * c.dim_t;
    P.net_out_per_chunk = P.mask_per_chunk;
    // progress (:411-425, 461-494, 577-579): one report per chunk; cancellation is polled once
    // more after the last chunk
    P.progress_total = (int)P.chunks.size();
    P.cancel_after_last = true;
    finish_plan(P, c.dim_t);
}

// ---- the DSP primitives as single-chunk plans -----------------------------------------------
namespace {
void single_chunk(HostPlan& P, int64_t len) {
    ChunkDesc d{};
    d.src0 = 0;
    d.valid = (int32_t)len;
    d.tail_reflect = 0;
    d.out0 = 0;
    d.out_len = P.g.Lout;
    d.y_off = 0;
    d.w_off = 0;
    P.chunks.assign(1, d);
    P.W.assign(std::max(P.g.Lout, 1), 1.0f);
    P.reflect_global = 0;
    P.step_out = std::max(P.g.Lout, 1);
    P.out_shift = 0;
    P.nan_to_zero = 0;
    P.S = P.S_out = 1;
    P.primitive = true;
}
} // namespace

void build_torch_stft(HostPlan& P, int n_fft, int hop, bool normalized, int n_channels, int64_t len,
                      bool inverse, bool zero_pad) {
    if (n_channels < 1 || n_channels > 2) fail(STG_INVALID_ARGUMENT, "n_channels must be 1 or 2");
    if (hop < 1 || len < 1 || len > INT32_MAX / 4) fail(STG_INVALID_ARGUMENT, "bad hop or length");
    if (!inverse && !zero_pad && len <= n_fft / 2)
        fail(STG_INVALID_ARGUMENT, "reflect pad larger than the signal");   // stft.h:59
    P.arch = ARCH_TFC;                                                // plain CaC-free spectra
    P.len = len;
    P.C = n_channels;
    const int T = (int)(len / hop) + 1;                               // stft.h:153
    P.g = FrameGeom{n_fft, hop, (int)len, T, 0, 0, 0, n_fft / 2, hop * (T - 1), zero_pad ? 1 : 0};
    P.fwd_scale = normalized ? (float)(1.0 / std::sqrt((double)n_fft)) : 1.0f;
    P.inv_scale = (float)((normalized ? std::sqrt((double)n_fft) : 1.0) / n_fft);
    single_chunk(P, len);
    P.front_layout = FRONT_COMPLEX;
    P.back_layout = BACK_COMPLEX;
    P.front_bins = P.back_bins = n_fft / 2 + 1;
    P.net_in_per_chunk = P.net_out_per_chunk = (int64_t)2 * n_channels * (n_fft / 2 + 1) * T;
    finish_plan(P, T);
}

void build_htdemucs_spec(HostPlan& P, int n_channels, int64_t len) {
    const int N = 4096, hl = N / 4, pad = hl / 2 * 3;
    if (n_channels < 1 || n_channels > 2) fail(STG_INVALID_ARGUMENT, "n_channels must be 1 or 2");
    if (len < 1 || len > INT32_MAX / 4) fail(STG_INVALID_ARGUMENT, "bad length");
    const int L = (int)len, T = (L + hl - 1) / hl;                   // stft.h:81
    if (L <= pad || L <= pad + T * hl - L) fail(STG_INVALID_ARGUMENT, "reflect pad larger than the signal");
    P.arch = ARCH_HTDEMUCS;
    P.len = len;
    P.C = n_channels;
    P.g = FrameGeom{N, hl, L, T, 2 * hl, pad, 2 * pad + T * hl, N / 2 + pad, L};
    P.fwd_scale = (float)(1.0 / std::sqrt((double)N));
    P.inv_scale = (float)(std::sqrt((double)N) / N);
    single_chunk(P, len);
    P.front_layout = FRONT_COMPLEX;
    P.back_layout = BACK_COMPLEX;
    P.front_bins = P.back_bins = N / 2;
    P.net_in_per_chunk = P.net_out_per_chunk = (int64_t)2 * n_channels * (N / 2) * T;
    finish_plan(P, T + 4);
}

namespace {
SplitParams split_params(const HostPlan& P, const PlanDevice& D, const float* d_mix, int first, int n);

// The (mean, std) of every chunk of [first, first + n) over its 2C x F x T CaC values
// (src/htdemucs.cpp:434-435): a front pass that only sums, then the per-chunk finish.
int cac_statistics(const HostPlan& P, const PlanDevice& D, const float* mix, int first, int n, cudaStream_t st) {
    if (!D.cac_part || !D.cac_stats) fail(STG_INTERNAL_ERROR, "no scratch for the CaC normalisation");
    SplitParams s = split_params(P, D, mix, first, n);
    s.layout = FRONT_STATS;
    s.n_bins = P.front_bins;
    s.stats_out = D.cac_part + (int64_t)first * P.n_tiles;
    cuda_check(stg::launch_front(s, st), "CaC statistics launch");
    const double count = 2.0 * P.C * P.front_bins * P.g.T;
    cuda_check(launch_cac_finish(s.stats_out, n, P.n_tiles, count, D.cac_stats + first, st), "CaC statistics launch");
    return 2;
}
} // namespace

const float* normalise_mix(const HostPlan& P, const PlanDevice& D, const float* d_mix, cudaStream_t st) {
    if (!P.mono_norm) return d_mix;
    if (!D.mixn || !D.mono) fail(STG_INTERNAL_ERROR, "no scratch for the mono normalisation");
    cuda_check(launch_mono_norm(d_mix, P.len, P.C, D.mono, D.mixn, st), "mono normalisation launch");
    return D.mixn;
}

// The chunks whose outputs reach output samples [b, e), as index ranges (one per chunk group,
// adjacent ones merged). Chunks of a group are in output order.
std::vector<std::pair<int, int>> chunks_for(const HostPlan& P, int64_t b, int64_t e) {
    std::vector<std::pair<int, int>> r;
    for (const ChunkGroup& g : P.groups) {
        int lo = -1, hi = -1;
        for (int k = g.c0; k < g.c1; k++) {
            const ChunkDesc& d = P.chunks[k];
            if (d.out0 < e + g.out_shift && d.out0 + d.out_len > b + g.out_shift) {
                if (lo < 0) lo = k;
                hi = k + 1;
            }
        }
        if (lo < 0) continue;
        if (!r.empty() && r.back().second == lo) r.back().second = hi;
        else r.emplace_back(lo, hi);
    }
    return r;
}

namespace {
// The fused kernel's parameters apart from the chunk range and the mask.
FusedParams fused_params(const HostPlan& P, const PlanDevice& D, const float* d_mix) {
    FusedParams f{};
    f.mix = d_mix; f.len = P.len; f.n_channels = P.C;
    f.g = P.g; f.K = P.K; f.n_tiles = P.n_tiles; f.S = P.S;
    f.win = D.win; f.tw = D.tw; f.inv_env = D.env;
    f.env_period = D.env_period; f.env_lo = P.env_lo; f.env_hi = P.env_hi;
    f.fwd_scale = P.fwd_scale; f.inv_scale = P.inv_scale;
    f.bin_tab = D.btab;
    f.bin_multi = P.bin_multi;
    f.bin_ebeg = D.ebeg; f.bin_ent = D.ent; f.bin_inv = D.binv;
    f.zero_dc = P.zero_dc; f.stem_stride = P.stem_stride;
    f.dim_f = P.dim_f; f.zero_bins = P.zero_bins;
    f.y_chunk_stride = P.y_chunk_stride; f.tr_chunk_stride = P.tr_chunk_stride;
    return f;
}

// The combine of one run (or of one bag member's run) over output samples [b, e).
CombineParams combine_params(const HostPlan& P, const PlanDevice& D, const float* d_mix, float* d_out, int64_t b,
                             int64_t e, int model) {
    CombineParams c{};
    c.Y = D.Y; c.y_chunk_stride = P.y_chunk_stride;
    c.Tr = D.Tr; c.tr_chunk_stride = P.tr_chunk_stride;
    c.chunks = D.chunks; c.n_chunks = (int)P.chunks.size();
    c.groups = D.groups; c.n_groups = (int)P.groups.size(); c.shift_mean = P.shift_mean;
    c.step_out = P.step_out; c.max_out_len = P.max_out_len;
    c.g = P.g; c.K = P.K; c.n_tiles = P.n_tiles;
    c.W = D.W;
    c.S = P.S; c.C = P.C; c.len = P.arch_out_len();
    c.i_begin = b; c.i_end = e;
    c.mode = P.arch; c.nan_to_zero = P.nan_to_zero; c.compensate = P.compensate;
    c.complement = P.complement; c.mix = d_mix; c.out = d_out;
    c.mono_stats = P.mono_norm ? D.mono : nullptr;
    if (!P.bag.empty()) {
        if (!D.bag || !D.bag_tot) fail(STG_INTERNAL_ERROR, "no device copy of the bag weights");
        c.bag = D.bag;
        c.bag_tot = D.bag_tot;
        c.bag_model = model;
        c.bag_last = model == P.n_models - 1;
    }
    return c;
}
} // namespace

void launch_plan(const HostPlan& P, const PlanDevice& D, const float* d_mix_in, const float* d_mask,
                 float* d_out, cudaStream_t st, const stg_run_options* opt, RunTiming* timing,
                 int64_t sample_begin, int64_t sample_end, const std::vector<cudaEvent_t>* ready) {
    if (!d_mix_in || !d_mask || !d_out) fail(STG_INVALID_ARGUMENT, "null buffer");
    P.check_mask(d_mask);
    if (sample_end < 0) sample_end = P.len;
    if (sample_begin < 0 || sample_begin >= sample_end || sample_end > P.len)
        fail(STG_INVALID_ARGUMENT, "sample range outside the track");
    const bool whole = sample_begin == 0 && sample_end == P.len;
    const std::vector<std::pair<int, int>> ranges =
        whole ? std::vector<std::pair<int, int>>{{0, (int)P.chunks.size()}} : chunks_for(P, sample_begin, sample_end);
    int total = 0;
    for (const auto& rg : ranges) total += rg.second - rg.first;
    // bag of models: every member runs the chunk list on its own masks, then its combine adds
    // its weighted stems to d_out (src/htdemucs.cpp:585-636)
    const int M = P.bag.empty() ? 1 : P.n_models;
    const int64_t mask_per_model = P.mask_per_chunk * (int64_t)P.chunks.size();
    const bool timed = timing && timing->timed;
    if (timing) timing->launches = 0;
    if (timed) cuda_check(cudaEventRecord(timing->ev[0], st), "cudaEventRecord");
    const bool zpath = P.z_per_chunk() > 0;   // HTDemucs: spectra once, then the back kernel per stem
    // HTDemucs: the masks' transposition (HBM-bound) on the side stream, beside the
    // normalisation and the front kernel (latency-bound); every segment has its own slot of
    // the scratch. The fork orders it after the caller's earlier work, including the previous
    // separation's back kernels, which read the same scratch. (A bag's members transpose
    // batch by batch on the caller's stream: they share the scratch.)
    const bool side_t = zpath && P.mask_planes && D.side && D.side_ev && M == 1;
    const int per = std::max(1, (opt && opt->chunks_per_batch > 0) ? opt->chunks_per_batch : total);
    int n_batches = 0;
    for (const auto& rg : ranges) n_batches += (rg.second - rg.first + per - 1) / per;
    if (ready && (int)ready->size() < M * n_batches) fail(STG_INTERNAL_ERROR, "fewer mask events than batches");
    // the caller's stream waits for the side stream before anything after this point,
    // the back kernels, or a failure, can hand the masks back to the caller
    struct Join {
        cudaStream_t st = nullptr;
        cudaEvent_t ev = nullptr;
        void now() {
            if (ev) cudaStreamWaitEvent(st, ev, 0);
            ev = nullptr;
        }
        ~Join() { now(); }
    } join;
    const float* d_mix = normalise_mix(P, D, d_mix_in, st);
    if (timing && P.mono_norm) timing->launches += 3;
    if (side_t) cuda_check(cudaEventRecord(D.fork, st), "cudaEventRecord");
    for (const auto& rg : ranges) {
        const int c0 = rg.first, G = rg.second - rg.first;
        if (zpath) {
            if (!D.zspec || !D.mask_t) fail(STG_INTERNAL_ERROR, "no scratch for the segment spectra");
            SplitParams z = split_params(P, D, d_mix, c0, G);
            z.layout = FRONT_ZSPEC;
            z.n_bins = P.front_bins;
            z.zspec = D.zspec + (int64_t)c0 * P.z_per_chunk();
            z.z_chunk_stride = P.z_per_chunk();
            if (P.cac_norm) {
                if (!D.cac_part || !D.cac_stats) fail(STG_INTERNAL_ERROR, "no scratch for the CaC normalisation");
                z.stats_out = D.cac_part + (int64_t)c0 * P.n_tiles;
            }
            cuda_check(stg::launch_front(z, st), "segment spectra launch");
            if (timing) timing->launches++;
            if (P.cac_norm) {
                const double count = 2.0 * P.C * P.front_bins * P.g.T;
                cuda_check(launch_cac_finish(D.cac_part + (int64_t)c0 * P.n_tiles, G, P.n_tiles, count,
                                             D.cac_stats + c0, st),
                           "CaC statistics launch");
                if (timing) timing->launches++;
            }
        } else if (P.cac_norm) {
            const int k = cac_statistics(P, D, d_mix, c0, G, st);
            if (timing) timing->launches += k;
        }
    }
    if (side_t) {   // batch by batch, each after its masks (when streamed in)
        if (!D.mask_t) fail(STG_INTERNAL_ERROR, "no scratch for the mask transposition");
        while ((int)D.side_ev->size() < n_batches) {
            cudaEvent_t e = nullptr;
            cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
            D.side_ev->push_back(e);
        }
        cuda_check(cudaStreamWaitEvent(D.side, D.fork, 0), "cudaStreamWaitEvent");
        int k = 0;
        for (const auto& rg : ranges)
            for (int b0 = rg.first; b0 < rg.second; b0 += per, k++) {
                const int nb = std::min(per, rg.second - b0);
                if (ready) cuda_check(cudaStreamWaitEvent(D.side, (*ready)[k], 0), "cudaStreamWaitEvent");
                cuda_check(launch_mask_transpose(d_mask + (int64_t)b0 * P.mask_per_chunk, P.mask_per_chunk, nb, P.S,
                                                 P.mask_planes, P.mask_bins, P.g.T,
                                                 D.mask_t + (int64_t)b0 * P.mask_t_per_chunk(),
                                                 P.mask_t_per_chunk(), D.side),
                           "mask transposition launch");
                if (timing) timing->launches++;
                cuda_check(cudaEventRecord((*D.side_ev)[k], D.side), "cudaEventRecord");
            }
        cuda_check(cudaEventRecord(D.join, D.side), "cudaEventRecord");
        join.st = st;
        join.ev = D.join;
    }
    FusedParams f = fused_params(P, D, d_mix);
    const auto cancelled = [&] { return opt && opt->should_cancel && opt->should_cancel(opt->user); };
    int done = 0, k = 0;
    bool first_batch = true;
    for (int m = 0; m < M; m++) {
        const float* mask_m = d_mask + (int64_t)m * mask_per_model;
        int kb = 0;   // batch of this model (the side stream's events are the first model's)
        for (const auto& rg : ranges) {
            for (int b0 = rg.first; b0 < rg.second; b0 += per, k++, kb++) {
                if (cancelled()) fail(STG_CANCELLED, "cancelled");
                const int nb = std::min(per, rg.second - b0);
                // the batch's masks: transposed on the side stream, or streamed in by the caller
                if (side_t) cuda_check(cudaStreamWaitEvent(st, (*D.side_ev)[kb], 0), "cudaStreamWaitEvent");
                else if (ready) cuda_check(cudaStreamWaitEvent(st, (*ready)[k], 0), "cudaStreamWaitEvent");
                f.chunks = D.chunks + b0;
                f.n_chunks = nb;
                f.mask = mask_m + (int64_t)b0 * P.mask_per_chunk;
                f.mask_chunk_stride = P.mask_per_chunk;
                f.Y = D.Y + (int64_t)b0 * P.y_chunk_stride;
                f.Tr = D.Tr + (int64_t)b0 * P.tr_chunk_stride;
                if (side_t) {   // transposed on the side stream
                    f.mask = reinterpret_cast<const float*>(D.mask_t + (int64_t)b0 * P.mask_t_per_chunk());
                    f.mask_chunk_stride = 4 * P.mask_t_per_chunk();
                } else if (P.mask_planes) {   // the batch's masks t-major, into the scratch the kernel reads
                    if (!D.mask_t) fail(STG_INTERNAL_ERROR, "no scratch for the mask transposition");
                    cuda_check(launch_mask_transpose(f.mask, P.mask_per_chunk, nb, P.S, P.mask_planes, P.mask_bins,
                                                     P.g.T, D.mask_t, P.mask_t_per_chunk(), st),
                               "mask transposition launch");
                    if (timing) timing->launches++;
                    f.mask = reinterpret_cast<const float*>(D.mask_t);
                    f.mask_chunk_stride = 4 * P.mask_t_per_chunk();
                }
                if (timed && first_batch) cuda_check(cudaEventRecord(timing->ev[1], st), "cudaEventRecord");
                first_batch = false;
                if (zpath) {   // every stem's ox = Z * M (CaC-normalised), iSTFT and overlap-add
                    SplitParams b = split_params(P, D, d_mix, b0, nb);
                    b.layout = BACK_ZMASK;
                    b.n_bins = P.back_bins;
                    b.net = const_cast<float*>(f.mask);
                    b.net_chunk_stride = f.mask_chunk_stride;
                    b.zspec = D.zspec + (int64_t)b0 * P.z_per_chunk();
                    b.z_chunk_stride = P.z_per_chunk();
                    b.cac_stats = P.cac_norm ? D.cac_stats + b0 : nullptr;
                    cuda_check(stg::launch_back(b, st), "back kernel launch");
                } else {
                    cuda_check(launch_fused(P.arch, f, st), "fused spectral kernel launch");
                }
                if (timing) timing->launches++;
                done += nb;
                if (opt && opt->on_progress) {
                    cuda_check(cudaStreamSynchronize(st), "fused spectral kernel");
                    const bool final_batch = m == M - 1 && b0 + nb >= rg.second && &rg == &ranges.back();
                    opt->on_progress(opt->user, final_batch && P.progress_final_total ? P.progress_total : done,
                                     P.progress_total > 0 ? P.progress_total : total * M);
                }
            }
        }
        if (m == M - 1) {
            join.now();
            if (P.cancel_after_last && cancelled()) fail(STG_CANCELLED, "cancelled");
            if (timed) cuda_check(cudaEventRecord(timing->ev[2], st), "cudaEventRecord");
        }
        cuda_check(launch_combine(combine_params(P, D, d_mix, d_out, sample_begin, sample_end, m), st),
                   "combine kernel launch");
        if (timing) timing->launches++;
    }
    if (timed) cuda_check(cudaEventRecord(timing->ev[3], st), "cudaEventRecord");
}

// ---- the halves around a real network ----------------------------------------------------------
namespace {
SplitParams split_params(const HostPlan& P, const PlanDevice& D, const float* d_mix, int first, int n) {
    SplitParams s{};
    s.mix = d_mix;
    s.len = P.len;
    s.n_channels = P.C;
    s.chunks = D.chunks + first;
    s.n_chunks = n;
    s.g = P.g;
    s.K = P.K;
    s.n_tiles = P.n_tiles;
    s.S = P.S;
    s.win = D.win;
    s.tw = D.tw;
    s.fwd_scale = P.fwd_scale;
    s.inv_scale = P.inv_scale;
    s.inv_env = D.env;
    s.env_period = D.env_period;
    s.env_lo = P.env_lo;
    s.env_hi = P.env_hi;
    s.bin_tab = D.btab;
    s.bin_multi = P.bin_multi;
    s.bin_ebeg = D.ebeg;
    s.bin_ent = D.ent;
    s.zero_bins = P.zero_bins;
    s.Y = D.Y + (int64_t)first * P.y_chunk_stride;
    s.y_chunk_stride = P.y_chunk_stride;
    s.Tr = D.Tr + (int64_t)first * P.tr_chunk_stride;
    s.tr_chunk_stride = P.tr_chunk_stride;
    return s;
}

void check_range(const HostPlan& P, int first, int n) {
    if (first < 0 || n < 1 || (int64_t)first + n > (int64_t)P.chunks.size())
        fail(STG_INVALID_ARGUMENT, "chunk range outside the plan");
}
} // namespace

void launch_front(const HostPlan& P, const PlanDevice& D, const float* d_mix, int first, int n, float* d_net_in,
                  cudaStream_t st) {
    if (!d_mix || !d_net_in) fail(STG_INVALID_ARGUMENT, "null buffer");
    check_range(P, first, n);
    if (P.front_layout == FRONT_BANDS && reinterpret_cast<uintptr_t>(d_net_in) % 16)
        fail(STG_INVALID_ARGUMENT, "the feature buffer must be 16-byte aligned");
    SplitParams s = split_params(P, D, d_mix, first, n);
    if (P.cac_norm) cac_statistics(P, D, d_mix, first, n, st);
    s.layout = P.front_layout;
    s.n_bins = P.front_bins;
    s.net = d_net_in;
    s.net_chunk_stride = P.net_in_per_chunk;
    s.cac_stats = P.cac_norm ? D.cac_stats + first : nullptr;
    cuda_check(stg::launch_front(s, st), "front kernel launch");
}

void launch_back(const HostPlan& P, const PlanDevice& D, const float* d_mix, const float* d_net_out, int first,
                 int n, cudaStream_t st) {
    if (!d_net_out || (P.back_is_fused && !d_mix)) fail(STG_INVALID_ARGUMENT, "null buffer");
    check_range(P, first, n);
    if (P.back_is_fused) {
        // RoFormer: the network's masks are exactly the fused kernel's mask input
        P.check_mask(d_net_out);
        FusedParams f = fused_params(P, D, d_mix);
        f.chunks = D.chunks + first; f.n_chunks = n;
        f.mask = d_net_out; f.mask_chunk_stride = P.mask_per_chunk;
        f.Y = D.Y + (int64_t)first * P.y_chunk_stride;
        f.Tr = D.Tr + (int64_t)first * P.tr_chunk_stride;
        cuda_check(launch_fused(P.arch, f, st), "fused spectral kernel launch");
        return;
    }
    SplitParams s = split_params(P, D, d_mix, first, n);
    s.layout = P.back_layout;
    s.n_bins = P.back_bins;
    s.net = const_cast<float*>(d_net_out);
    s.net_chunk_stride = P.net_out_per_chunk;
    s.cac_stats = P.cac_norm ? D.cac_stats + first : nullptr;
    cuda_check(stg::launch_back(s, st), "back kernel launch");
}

void launch_finish(const HostPlan& P, const PlanDevice& D, const float* d_mix, float* d_out, cudaStream_t st,
                   int model) {
    if (!d_out || (P.complement && !d_mix)) fail(STG_INVALID_ARGUMENT, "null buffer");
    if (model < 0 || model >= P.n_models) fail(STG_INVALID_ARGUMENT, "no such model in the bag");
    cuda_check(launch_combine(combine_params(P, D, d_mix, d_out, 0, P.arch_out_len(), model), st),
               "combine kernel launch");
}

} // namespace stg
