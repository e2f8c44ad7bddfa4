// kernels.cu -- the fused spectral kernel and the chunk combine for sm_100a.
//
// Fused kernel, persistent CTAs taking (chunk, frame tile) items. For every stem and every
// frame of a tile:
//   1. load the frame's new samples of both channels from the track into an input ring, a
//      frame ahead (reflect / zero padding of the chunk, the track and the STFT evaluated per
//      sample where a rule applies), window the frame, and pack the two real channels as one
//      complex frame L + iR;
//   2. forward FFT in shared memory (fft.cuh);
//   3. split the two channels' spectra, apply the architecture's spectral op (the stand-in
//      for the network: RoFormer's band-averaged mask or TFC-TDF's CaC real mask), drop what
//      the reference's c2r drops, and repack the two masked spectra as one Hermitian pair;
//   4. inverse FFT, window, and overlap-add into a ring buffer of n_fft samples per channel;
//   5. flush the hop of samples that no later frame of the tile touches, scaled by the
//      inverse window-sum envelope, to the chunk output Y. The last frame of a tile sends
//      its n_fft - hop trailing samples to Tr instead; the combine adds them to the next
//      tile's leading samples, so every sum is formed in a fixed order (no atomics).
// (HTDemucs, whose four or six stems share one spectrum, runs the front kernel once per frame
// and the back kernel per stem instead: split.cu, FRONT_ZSPEC / BACK_ZMASK.)
// Combine kernel: one thread per output sample (four for one or two stereo stems); it sums
// the chunks that cover the sample with their crossfade weights (reading Y and the
// tile-boundary partials Tr), divides by the summed weight, and applies the architecture's
// epilogue (nan_to_num, compensation, complement).
#include <algorithm>
#include <type_traits>
#include <vector>

#include "fft.cuh"
#include "frame.cuh"
#include "kernels.h"

namespace stg {

// ---- the stand-in network ---------------------------------------------------------------
// Each thread owns the bins bin(tid, i) (i < BPT); prefetch() issues every mask load of its
// bins for one (stem, frame) before apply() consumes them, so the loads overlap one another.
template <int ARCH, int N, int T> struct MaskOp {
    static constexpr int NBIN = N / 2 + 1;
    static constexpr int BPT = (NBIN + T - 1) / T;
    // RoFormer at n_fft 2048 (the mirror step of fused_kernel): thread tid holds the radix-8
    // butterflies g0 = tid and g1 = 256 - tid (128 for thread 0), i.e. the points g + 256r, so its
    // bins are g0 + 256i (i < 4), g1 + 256(i - 4) (i < 8) and, for thread 0, the Nyquist bin.
    // Elsewhere bins are dealt round-robin: tid + i*T.
    static constexpr bool MIR = ARCH == ARCH_ROFORMER && N == 2048;
    static_assert(!MIR || (T == 128 && BPT == 9), "the mirror step deals 2048 points to 128 threads");
    __device__ __forceinline__ static int bin(int tid, int i) {
        if constexpr (MIR) {
            if (i < 4) return tid + 256 * i;
            if (i < 8) return (tid ? 256 - tid : 128) + 256 * (i - 4);
            return tid ? NBIN : N / 2;
        } else {
            return tid + i * T;
        }
    }
    float4 a[BPT];
    float4 b[BPT];   // RoFormer: the second band holding the bin
    float inv[BPT];  // RoFormer: 1 / bands holding the bin, times scale
    float scale = 1.0f;   // RoFormer: folded into inv (the split's factor)

    const int2* btab;   // RoFormer: the bin table's copy in shared memory

    // Issue the mask loads of every bin slot of the thread.
    __device__ __forceinline__ void prefetch(const FusedParams& p, int ci, int s, int t, int tid) {
        const float* __restrict__ m = p.mask + (int64_t)ci * p.mask_chunk_stride;
        if constexpr (ARCH == ARCH_ROFORMER) {
            // src/roformer.cpp:256-269: band b's mask for frame t is the row
            // [off_b*T + t*din_b, +din_b) of the stem's block; entry (j*C + c)*2 + {re, im}.
            const float* ms = m + (int64_t)s * p.stem_stride;
#pragma unroll
            for (int i = 0; i < BPT; i++) {
                const int f = bin(tid, i);
                a[i] = b[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                inv[i] = 0.0f;
                if (f < NBIN) {
                    // (offset / 2C) in bits 0-21, band size in bits 22-31; the band's row for
                    // frame t starts size * t entries further on
                    const int2 e = btab[f];
                    const unsigned s0 = (unsigned)e.x >> 22, s1 = (unsigned)e.y >> 22;
                    const int u0 = (e.x & 0x3fffff) + t * (int)s0, u1 = (e.y & 0x3fffff) + t * (int)s1;
                    inv[i] = p.bin_multi ? __ldg(p.bin_inv + f) * scale : (s1 ? 0.5f * scale : (s0 ? scale : 0.0f));
                    if (p.n_channels == 2) {
                        a[i] = ld_stream4(ms + 4 * u0);
                        if (s1) b[i] = ld_stream4(ms + 4 * u1);
                    } else {
                        const float2 u = ld_stream2(ms + 2 * u0);
                        a[i] = make_float4(u.x, u.y, 0.f, 0.f);
                        if (s1) {
                            const float2 v = ld_stream2(ms + 2 * u1);
                            b[i] = make_float4(v.x, v.y, 0.f, 0.f);
                        }
                    }
                }
            }
        } else {
            // TFC-TDF y planes [4S][dim_f][T] (src/tfc_tdf.cpp:370-387), rewritten t-major by
            // mask_transpose: [S][T][dim_f] float4 (L re, L im, R re, R im), so frame t's bins
            // are contiguous.
            const int F = p.dim_f;
            const int f_lo = p.zero_bins;
            const float* ms = m + ((int64_t)s * p.g.T + t) * F * 4;
#pragma unroll
            for (int i = 0; i < BPT; i++) {
                const int f = tid + i * T;
                a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (f >= f_lo && f < F) a[i] = ld_stream4(ms + 4 * f);
            }
        }
    }

    // Bin f = bin(tid, i) of the two channels' spectra zl, zr -> the spectra the iSTFT consumes.
    __device__ __forceinline__ void apply(const FusedParams& p, int ci, int s, int t, int f, int i,
                                          float2 zl, float2 zr, float2& yl, float2& yr) const {
        if constexpr (ARCH == ARCH_ROFORMER) {
            // masks of every band holding f, averaged (src/roformer.cpp:270-276), times z
            float2 al = make_float2(a[i].x + b[i].x, a[i].y + b[i].y);
            float2 ar = make_float2(a[i].z + b[i].z, a[i].w + b[i].w);
            if (p.bin_multi) {   // bins in more than two bands: the rest straight from memory
                const int e0 = __ldg(p.bin_ebeg + f), e1 = __ldg(p.bin_ebeg + f + 1);
                const float* ms = p.mask + (int64_t)ci * p.mask_chunk_stride + (int64_t)s * p.stem_stride;
                for (int k = e0 + 2; k < e1; k++) {
                    const int2 en = __ldg(p.bin_ent + k);
                    const float* q = ms + en.x + (int64_t)t * en.y;
                    al.x += ld_stream(q); al.y += ld_stream(q + 1);
                    if (p.n_channels == 2) { ar.x += ld_stream(q + 2); ar.y += ld_stream(q + 3); }
                }
            }
            yl = cmul(zl, al);   // the band average's weight came with zl, zr
            yr = cmul(zr, ar);
            if (p.zero_dc && f == 0) { yl = make_float2(0.f, 0.f); yr = yl; }      // :278
        } else {
            // y = in * mask per CaC plane; zero below zero_bins and from dim_f up (the loads
            // left a[i] at zero there)
            yl = make_float2(zl.x * a[i].x, zl.y * a[i].y);
            yr = make_float2(zr.x * a[i].z, zr.y * a[i].w);
        }
    }
};

// The forward transform's radix plan: FftCfg::FwdPlan for the mirror step, else the common one.
template <class Cfg, bool OWN> struct FwdPlanOf { using type = typename Cfg::Plan; };
template <class Cfg> struct FwdPlanOf<Cfg, true> { using type = typename Cfg::FwdPlan; };

template <int ARCH, int N>
__global__ void __launch_bounds__(FftCfg<N>::T, FftCfg<N>::MINB) fused_kernel(const FusedParams p) {
    constexpr int T = FftCfg<N>::T;
    using Plan = typename FftCfg<N>::Plan;
    constexpr int R1 = Head<Plan>::first;                 // first forward pass
    using FwdRest = typename Head<Plan>::tail;
    using InvInit = typename Init<Plan>::type;            // inverse passes but the last
    constexpr int RL = Init<Plan>::last, NSL = Init<Plan>::prod;
    constexpr bool SWIN = FftCfg<N>::SMEM_WIN;
    // the RoFormer instance at n_fft 2048 has the registers to load each pass's twiddles early
    constexpr bool TW_EARLY = ARCH == ARCH_ROFORMER && N == 2048;
    // and its codelets' complex additions in f32x2 instructions (fft.cuh: PF2)
    using CV = std::conditional_t<ARCH == ARCH_ROFORMER && N == 2048, PF2, float2>;
    // and its loads of the next frame's new samples issued after the frame's mask loads
    constexpr bool LATE_NX = ARCH == ARCH_ROFORMER && N == 2048;
    // and the mirror step: the forward plan ends in radix 8 (FftCfg::FwdPlan), and each thread's
    // two last butterflies g and 256 - g hold the bins k and N - k that the split pairs, which are
    // also the points of the inverse's first radix-8 butterflies. So the forward's last pass, the
    // spectral op and the inverse's first pass run in registers between one load and one store
    // of the frame.
    constexpr bool MIR = MaskOp<ARCH, N, T>::MIR;
    using FwdPlan = typename FwdPlanOf<FftCfg<N>, MIR>::type;
    constexpr int R1F = Head<FwdPlan>::first;
    using FwdMid = typename Init<typename Head<FwdPlan>::tail>::type;   // [MIR] passes before the step
    using InvMid = typename Head<InvInit>::tail;                         // [MIR] passes after it
    static_assert(!MIR || (Init<FwdPlan>::last == 8 && Head<Plan>::first == 8), "mirror step: radix 8 both sides");
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);    // padded frame
    float2* in_ring = buf + padded_size(N);               // input samples (L, R) by position mod N
    float2* out_ring = in_ring + N;                       // overlap-add sums (L, R) by position mod N
    float* win_s = reinterpret_cast<float*>(out_ring + N);   // [SWIN] window copy
    int2* btab_s = reinterpret_cast<int2*>(win_s + (SWIN ? N : 0));   // [RoFormer] bin table copy
    float* env_s = reinterpret_cast<float*>(btab_s + (ARCH == ARCH_ROFORMER ? N / 2 + 2 : 0));   // envelope period
    const TwGlobal tw{p.tw};
    const TwGlobal twf{p.tw + (MIR ? N : 0)};   // the forward plan's table (plan.cu: fft_tables)
    const float* win = SWIN ? win_s : p.win;

    const int tid = threadIdx.x;
    const FrameGeom& G = p.g;
    const int hop = G.hop;
    const int C = p.n_channels;
    const float* chL = p.mix;
    const float* chR = p.mix + (C > 1 ? p.len : 0);
    const int lxf = G.ht_pad ? G.ht_lxf : G.Lc;
    const float half_fwd = 0.5f * p.fwd_scale;

    // every stem pass flushes the whole output ring at its last frame, so one zeroing lasts
    for (int i = tid; i < N; i += T) out_ring[i] = make_float2(0.f, 0.f);
    if constexpr (SWIN)
        for (int i = tid; i < N; i += T) win_s[i] = __ldg(p.win + i);
    const bool env_on = p.env_period != nullptr;
    if (env_on)
        for (int i = tid; i < hop; i += T) env_s[i] = __ldg(p.env_period + i);

    // The mirror instance keeps the window in registers: its forward's first pass and its
    // overlap-add both give a thread one butterfly, on the samples tid + r*T, so the same 16
    // values serve both (12 bytes of spills at the 168-register cap, and still 1 % faster on a
    // 60 s track than 32 window loads through L1 per frame)
    float wr[MIR ? 16 : 1];
    if constexpr (MIR) {
        static_assert(N / R1F == T && N / RL == T && NSL == T, "one butterfly per thread at both ends");
#pragma unroll
        for (int r = 0; r < 16; r++) wr[r] = __ldg(p.win + tid + r * T);
    }
    MaskOp<ARCH, N, T> mk;
    // RoFormer: the inverse transform's scale goes in with the mask too (the transform is
    // linear), so the overlap-add multiplies by the window alone
    mk.scale = ARCH == ARCH_ROFORMER ? half_fwd * p.inv_scale : half_fwd;
    InPrefetch<T, FftCfg<N>::HOPMAX> nx;
    if constexpr (ARCH == ARCH_ROFORMER) {
        for (int i = tid; i < N / 2 + 1; i += T) btab_s[i] = __ldg(p.bin_tab + i);
        mk.btab = btab_s;
    }

    // persistent CTAs: work items are (chunk, tile) pairs, tiles of a chunk adjacent
    for (int item = blockIdx.x; item < p.n_tiles * p.n_chunks; item += gridDim.x) {
    const int tile = item % p.n_tiles, ci = item / p.n_tiles;
    const ChunkDesc cd = p.chunks[ci];
    const int t_begin = tile * p.K;
    const int t_end = min(G.T, t_begin + p.K);
    const bool last_tile = t_end == G.T;
    const int lin = linear_offset(p, cd, t_begin, t_end);

    for (int s = 0; s < p.S; s++) {
        float* Ys = p.Y + (int64_t)ci * p.y_chunk_stride + (int64_t)s * C * G.Lout;
        float* Trs = p.Tr + (int64_t)ci * p.tr_chunk_stride + ((int64_t)tile * p.S + s) * C * (N - hop);
        // prologue of a stem pass: the first frame's window and the next frame's new samples
        {
            const int q0 = G.first_pos + t_begin * hop;
            if constexpr (N == 2048) {   // every load in flight before the first store
                float2 pv[N / T];
#pragma unroll
                for (int k = 0; k < N / T; k++) pv[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + tid + k * T);
#pragma unroll
                for (int k = 0; k < N / T; k++) in_ring[ring_slot<N>(q0 + tid + k * T)] = pv[k];
            } else {
                for (int n = tid; n < N; n += T) in_ring[ring_slot<N>(q0 + n)] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + n);
            }
#pragma unroll
            for (int k = 0; k < nx.K; k++) {
                const int u = tid + k * T;
                if (u < hop && t_begin + 1 < t_end) nx.v[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + N + u);
            }
        }
        __syncthreads();
        // TFC-TDF: frame t's mask row (dim_f float4, 16-byte aligned) requested from L2 a frame
        // before its loads
        const auto mask_row_to_l2 = [&](int t) {
            if constexpr (ARCH == ARCH_TFC && FftCfg<N>::MASK_L2)
                if (tid == 0 && t < t_end)
                    prefetch_l2(p.mask + (int64_t)ci * p.mask_chunk_stride + ((int64_t)s * G.T + t) * p.dim_f * 4,
                                (unsigned)p.dim_f * 16u);
        };
        mask_row_to_l2(t_begin);
        for (int t = t_begin; t < t_end; t++) {
            const int q0 = G.first_pos + t * hop;
            mask_row_to_l2(t + 1);
            // forward pass 1: windowed frame straight from the input ring
            pass_io<N, R1F, 1, T, false, false, false, CV>(
                twf, tid,
                [&](int j, int r) {
                    const int n = j + r * (N / R1F);
                    const float2 x = in_ring[ring_slot<N>(q0 + n)];
                    float w;
                    if constexpr (MIR) w = wr[r];
                    else w = SWIN ? win[n] : __ldg(win + n);
                    return make_float2(x.x * w, x.y * w);
                },
                [&](int base, int r, float2 v) { buf[pad_store<R1F, 1>(base, r)] = v; });
            __syncthreads();
            // the next frame's new samples replace the ones this frame was the last to use
            if (t + 1 < t_end) {
#pragma unroll
                for (int k = 0; k < nx.K; k++) {
                    const int u = tid + k * T;
                    if (u < hop) in_ring[ring_slot<N>(q0 + N + u)] = nx.v[k];
                }
                if (!LATE_NX && t + 2 < t_end) {   // (RoFormer at n_fft 2048: after the mask loads, below)
#pragma unroll
                    for (int k = 0; k < nx.K; k++) {
                        const int u = tid + k * T;
                        if (u < hop) nx.v[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + hop + N + u);
                    }
                }
            }
            // all of this frame's mask loads in flight at once (at n_fft 2048 before the rest of
            // the forward transform, whose work hides their latency, and before the next frame's
            // new samples), then the spectral op: split the channels, apply the stand-in network,
            // repack as one Hermitian pair
            constexpr int BPT = MaskOp<ARCH, N, T>::BPT;
            if constexpr (N == 2048) {
                mk.prefetch(p, ci, s, t, tid);
                if (LATE_NX && t + 2 < t_end) {
#pragma unroll
                    for (int k = 0; k < nx.K; k++) {
                        const int u = tid + k * T;
                        if (u < hop) nx.v[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + hop + N + u);
                    }
                }
                if constexpr (MIR) passes<N, T, false, R1F, TW_EARLY, CV>(buf, twf, tid, FwdMid{});
                else passes<N, T, false, R1, TW_EARLY, CV>(buf, tw, tid, FwdRest{});
            } else {
                passes<N, T, false, R1>(buf, tw, tid, FwdRest{});
                mk.prefetch(p, ci, s, t, tid);
            }
            // (n_fft 2048: the frame's loads batched ahead of its stores here and in the flush)
            constexpr bool BATCH = N == 2048;
            if constexpr (MIR) {
                // the mirror step. Thread tid takes the forward's last radix-8 butterflies g0 = tid
                // and g1 = 256 - tid (thread 0: 0 and 128), whose outputs are the bins g + 256r
                // (fft.cuh: a last pass writes j + r*N/R). Bin k's mirror N - k is then
                // g1 + 256(7 - r) for k = g0 + 256r and the other way round, except on thread 0,
                // whose two butterflies each hold their own mirrors (and bins 0 and N/2).
                constexpr int NB = N / 8;
                const int g0 = tid, g1 = tid ? NB - tid : NB / 2;
                const bool t0 = tid == 0;
                CV z[16];
                float2 w[16];
#pragma unroll
                for (int r = 1; r < 8; r++) {
                    w[r] = twf(twiddle_index<NB>(r, g0));
                    w[8 + r] = twf(twiddle_index<NB>(r, g1));
                }
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    z[r] = buf[pad_load<N, 8>(g0, r)];
                    z[8 + r] = buf[pad_load<N, 8>(g1, r)];
                }
                __syncthreads();   // every point read before the inverse's first pass writes
#pragma unroll
                for (int r = 1; r < 8; r++) {
                    z[r] = cmul(z[r], w[r]);
                    z[8 + r] = cmul(z[8 + r], w[8 + r]);
                }
                Dft<8, false>::template run<1>(z);
                Dft<8, false>::template run<1>(z + 8);
                // slot i: bin bin(tid, i) at z[i] (i < 4), z[i + 4] (i < 8) or z[4] (thread 0's
                // Nyquist bin); gx the inverse's input at the bin, gm at its mirror
                float2 gx[BPT], gm[BPT];
                gx[8] = make_float2(0.f, 0.f);   // (read, and not used, by the other threads)
#pragma unroll
                for (int i = 0; i < BPT; i++) {
                    const int f = MaskOp<ARCH, N, T>::bin(tid, i);
                    if (i < 8 || t0) {
                        const float2 X = i < 4 ? z[i] : (i < 8 ? z[i + 4] : z[4]);
                        const float2 Xm = i < 4 ? (t0 ? z[(8 - i) & 7] : z[15 - i])
                                                : (i < 8 ? (t0 ? z[19 - i] : z[11 - i]) : z[4]);
                        const float sc = mk.inv[i];   // with the band weight
                        const float2 zl = make_float2(sc * (X.x + Xm.x), sc * (X.y - Xm.y));
                        const float2 zr = make_float2(sc * (X.y + Xm.y), -sc * (X.x - Xm.x));
                        float2 yl, yr;
                        mk.apply(p, ci, s, t, f, i, zl, zr, yl, yr);
                        if ((i == 0 && t0) || i == 8) { yl.y = 0.0f; yr.y = 0.0f; }   // c2r ignores these
                        gx[i] = make_float2(yl.x - yr.y, yl.y + yr.x);
                        gm[i] = make_float2(yl.x + yr.y, yr.x - yl.y);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    z[i] = gx[i];
                    z[i + 8] = gx[i + 4];
                    z[12 + i] = t0 ? gm[7 - i] : gm[3 - i];
                }
                z[4] = t0 ? gx[8] : gm[7];
#pragma unroll
                for (int m = 1; m < 4; m++) z[4 + m] = t0 ? gm[4 - m] : gm[7 - m];
                // the inverse's first pass (radix 8 at stride 1): butterfly g writes 8g + r
                Dft<8, true>::template run<1>(z);
                Dft<8, true>::template run<1>(z + 8);
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    buf[pad_store<8, 1>(8 * g0, r)] = z[r];
                    buf[pad_store<8, 1>(8 * g1, r)] = z[8 + r];
                }
                __syncthreads();
                passes<N, T, true, 8, TW_EARLY, CV>(buf, tw, tid, InvMid{});
            } else {
                // at n_fft 2048 every bin's two spectrum points are loaded before the arithmetic
                // and the stores (the stores could alias later loads as far as the compiler
                // knows); at 4096 the 128-register cap leaves no room for it
                float2 Xa[BATCH ? BPT : 1], Xb[BATCH ? BPT : 1];
                if constexpr (BATCH) {
    #pragma unroll
                    for (int i = 0; i < BPT; i++) {
                        const int f = tid + i * T;
                        if (f <= N / 2) {
                            Xa[i] = buf[pad_idx(f)];
                            Xb[i] = buf[pad_idx(f == 0 ? 0 : N - f)];
                        }
                    }
                }
    #pragma unroll
                for (int i = 0; i < BPT; i++) {
                    const int f = tid + i * T;
                    if (f <= N / 2) {
                        const int fm = f == 0 ? 0 : N - f;
                        const float2 X = BATCH ? Xa[BATCH ? i : 0] : buf[pad_idx(f)];
                        const float2 Xm = BATCH ? Xb[BATCH ? i : 0] : buf[pad_idx(fm)];
                        const float sc = ARCH == ARCH_ROFORMER ? mk.inv[i] : half_fwd;   // RoFormer: with the band weight
                        const float2 zl = make_float2(sc * (X.x + Xm.x), sc * (X.y - Xm.y));
                        const float2 zr = make_float2(sc * (X.y + Xm.y), -sc * (X.x - Xm.x));
                        float2 yl, yr;
                        mk.apply(p, ci, s, t, f, i, zl, zr, yl, yr);
                        if (f == 0 || f == N / 2) { yl.y = 0.0f; yr.y = 0.0f; }   // c2r ignores these
                        buf[pad_idx(f)] = make_float2(yl.x - yr.y, yl.y + yr.x);
                        if (f != 0 && f != N / 2) buf[pad_idx(fm)] = make_float2(yl.x + yr.y, yr.x - yl.y);
                    }
                }
                __syncthreads();
                passes<N, T, true, 1, TW_EARLY, CV>(buf, tw, tid, InvInit{});
            }
            // inverse last pass: window and overlap-add straight into the output ring. Butterfly
            // j < NSL writes the positions j + r*NSL, so a thread adds into the ring positions
            // q0 + n with n = tid mod T, the very ones it flushes below: the pass's barrier goes
            // between its loads and its stores (the next frame's first pass rewrites buf), and the
            // flush needs none before it.
            static_assert(NSL % T == 0, "the overlap-add and the flush give a thread the same positions");
            pass_io<N, RL, NSL, T, true, true, false, CV>(
                tw, tid, [&](int j, int r) { return buf[pad_load<N, RL>(j, r)]; },
                [&](int base, int r, float2 v) {
                    const int n = base + r * NSL;
                    float w;
                    if constexpr (MIR) w = wr[r];
                    else w = ARCH == ARCH_ROFORMER ? (SWIN ? win[n] : __ldg(win + n))
                                                   : (SWIN ? win[n] : __ldg(win + n)) * p.inv_scale;
                    float2& o = out_ring[ring_slot<N>(q0 + n)];
                    o = make_float2(fmaf(v.x, w, o.x), fmaf(v.y, w, o.y));
                });
            // flush what no later frame of this tile touches
            const bool last = t == t_end - 1;
            const int ny = (last && last_tile) ? N : hop;
            const int nflush = last ? N : hop;
            // the envelope from the shared-memory period where it repeats (r: the period slot
            // of this thread's sample, advanced by T per iteration)
            int r = 0;
            if (env_on) {
                r = (q0 - G.out_offset + tid - p.env_lo) % hop;
                if (r < 0) r += hop;
            }
            if (BATCH && !last && env_on) {
                // a frame inside the tile: hop samples to Y, every ring and envelope load of the
                // thread issued before its first store
                constexpr int KF = (FftCfg<N>::HOPMAX + T - 1) / T;
                float2 fv[KF];
                float fe[KF];
#pragma unroll
                for (int k = 0; k < KF; k++) {
                    const int u = tid + k * T;
                    fe[k] = 0.0f;
                    if (u < hop) {
                        const int q = q0 + u;
                        fv[k] = out_ring[ring_slot<N>(q)];
                        const int j = q - G.out_offset;
                        if (j >= 0 && j < G.Lout) fe[k] = j >= p.env_lo && j < p.env_hi ? env_s[r] : ld_stream(p.inv_env + j);
                    }
                    r += T;
                    while (r >= hop) r -= hop;
                }
#pragma unroll
                for (int k = 0; k < KF; k++) {
                    const int u = tid + k * T;
                    if (u < hop) {
                        const int q = q0 + u;
                        out_ring[ring_slot<N>(q)] = make_float2(0.f, 0.f);
                        const int j = q - G.out_offset;
                        if (j >= 0 && j < G.Lout) {
                            if (C > 1) reinterpret_cast<float2*>(Ys)[j] = make_float2(fv[k].x * fe[k], fv[k].y * fe[k]);
                            else Ys[j] = fv[k].x * fe[k];
                        }
                    }
                }
            } else {
                for (int u = tid; u < nflush; u += T) {
                    const int q = q0 + u;
                    float2& o = out_ring[ring_slot<N>(q)];
                    const float2 v = o;
                    o = make_float2(0.f, 0.f);
                    const int j = q - G.out_offset;
                    const bool in = j >= 0 && j < G.Lout;
                    float ie = 0.0f;
                    if (in) ie = env_on && j >= p.env_lo && j < p.env_hi ? env_s[r] : ld_stream(p.inv_env + j);
                    if (env_on) {
                        r += T;
                        while (r >= hop) r -= hop;
                    }
                    if (u < ny) {
                        if (in) {
                            if (C > 1) reinterpret_cast<float2*>(Ys)[j] = make_float2(v.x * ie, v.y * ie);
                            else Ys[j] = v.x * ie;
                        }
                    } else {
                        if (C > 1) reinterpret_cast<float2*>(Trs)[u - hop] = make_float2(v.x * ie, v.y * ie);
                        else Trs[u - hop] = v.x * ie;
                    }
                }
            }
            // the next iteration's first barrier (after forward pass 1) orders these ring
            // writes before any later read of the same slots
        }
        __syncthreads();
    }
    }
}

// ---- combine ------------------------------------------------------------------------------
// One thread per output sample and SC = stems x channels rows. Per group (a pass of the shift
// average; one group without shifts): sum the chunks covering the sample in ascending chunk
// order (src/roformer.cpp:337-340, src/tfc_tdf.cpp:420-422, src/htdemucs.cpp:598-601), each
// value the chunk output Y plus, on a tile boundary, the previous tile's trailing partial Tr,
// and divide by the summed weight; then average the groups and finish (epilogue).
// The value the separator returns for row k (stem k / C) at output sample i, from this launch's
// estimate v: the shift average's division, compensation, then either the mono-mix inverse
// (src/htdemucs.cpp:641; finish_plain) or, for a bag of models (finish_bag), this model's
// weighted term added to the previous models' sum in out (float products and sums in model
// order, :628-635) and, after the last model, the division by the weights' sum and the mono
// inverse (:638-642).
__device__ __forceinline__ float finish_plain(const CombineParams& p, float v) {
    v = p.shift_mean == 1 ? v / (float)p.n_groups : v;
    v *= p.compensate;
    if (p.mono_stats) v = (float)((double)v * p.mono_stats[1] + p.mono_stats[0]);   // htdemucs.cpp:641
    return v;
}
__device__ __forceinline__ float finish_bag(const CombineParams& p, int k, int64_t i, float v) {
    if (p.shift_mean == 1) v = v / (float)p.n_groups;
    v *= p.compensate;
    const int s = k / p.C;
    const float w = __ldg(p.bag + p.bag_model * p.S + s);
    float acc = p.bag_model == 0 ? 0.0f : p.out[(int64_t)k * p.len + i];
    if (w != 0.0f) acc = __fadd_rn(acc, __fmul_rn(w, v));
    if (!p.bag_last) return acc;
    v = __fdiv_rn(acc, __ldg(p.bag_tot + s));
    if (p.mono_stats) v = (float)((double)v * p.mono_stats[1] + p.mono_stats[0]);
    return v;
}

template <int SC>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
    const int i = (int)(p.i_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= p.i_end) return;
    const FrameGeom& G = p.g;
    const int step = (int)p.step_out;
    const int span = p.K * G.hop, ov = G.n_fft - G.hop;
    float res[SC];
#pragma unroll
    for (int k = 0; k < SC; k++) res[k] = 0.0f;
    for (int gi = 0; gi < p.n_groups; gi++) {
        const ChunkGroup grp = p.groups[gi];
        const int P = i + grp.out_shift;
        const int out00 = (int)p.chunks[grp.c0].out0;
        const int n = grp.c1 - grp.c0;
        int ghi = (P - out00) / step;
        ghi = min(ghi, n - 1);
        int glo = (P - out00 - (int)p.max_out_len) / step;
        glo = max(glo, 0);
        float acc[SC];
#pragma unroll
        for (int k = 0; k < SC; k++) acc[k] = 0.0f;
        float wsum = 0.0f;
        for (int gl = glo; gl <= ghi + 1 && gl < n; gl++) {
            const int g = grp.c0 + gl;
            const ChunkDesc& d = p.chunks[g];
            const int u = P - (int)d.out0;
            if (u < 0 || u >= d.out_len) continue;
            const float w = __ldg(p.W + d.w_off + u);
            wsum += w;
            const int j = d.y_off + u;
            const float* y = p.Y + (int64_t)g * p.y_chunk_stride + (int64_t)j * p.C;
            // the tile boundary region j falls in, if any
            const int q = j + G.out_offset - G.first_pos;
            const int tau = q / span;
            const int uu = q - tau * span;
            const float* tr = nullptr;
            if (tau >= 1 && tau < p.n_tiles && uu < ov)
                tr = p.Tr + (int64_t)g * p.tr_chunk_stride + (int64_t)(tau - 1) * SC * ov + uu * p.C;
            if (p.C == 2) {   // the stems' (L, R) pairs as one 8-byte load each
#pragma unroll
                for (int s = 0; s < SC / 2; s++) {
                    float2 v = __ldg(reinterpret_cast<const float2*>(y + (int64_t)s * 2 * G.Lout));
                    if (tr) {
                        const float2 r = __ldg(reinterpret_cast<const float2*>(tr + s * 2 * ov));
                        v = make_float2(v.x + r.x, v.y + r.y);
                    }
                    acc[2 * s] = fmaf(w, v.x, acc[2 * s]);
                    acc[2 * s + 1] = fmaf(w, v.y, acc[2 * s + 1]);
                }
            } else {
#pragma unroll
                for (int k = 0; k < SC; k++) {
                    float v = __ldg(y + (int64_t)k * G.Lout);
                    if (tr) v += __ldg(tr + k * ov);
                    acc[k] = fmaf(w, v, acc[k]);
                }
            }
        }
        const float inv = 1.0f / wsum;
#pragma unroll
        for (int k = 0; k < SC; k++) {
            float v = acc[k] * inv;
            if (p.nan_to_zero && !isfinite(v)) v = 0.0f;
            res[k] += p.shift_mean == 2 ? v / (float)p.n_groups : v;
        }
    }
    float outv[SC];
    if (!p.bag) {
#pragma unroll
        for (int k = 0; k < SC; k++) outv[k] = finish_plain(p, res[k]);
    } else {   // a bag member's pass reads the previous members' sums in out
#pragma unroll
        for (int k = 0; k < SC; k++) outv[k] = finish_bag(p, k, i, res[k]);
    }
#pragma unroll
    for (int k = 0; k < SC; k++) p.out[(int64_t)k * p.len + i] = outv[k];
    if (p.complement) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (c < p.C) {
                float v = __ldg(p.mix + (int64_t)c * p.len + i);
#pragma unroll
                for (int k = 0; k < SC; k++)
                    if (k % p.C == c && (p.complement == 2 || k < p.C)) v -= outv[k];
                p.out[(int64_t)(SC + c) * p.len + i] = v;
            }
        }
    }
}

// Stereo rows, V = 4 consecutive output samples per thread: the same sums in the same order as
// combine_kernel (so the same floats), with the group and chunk bookkeeping (the divisions
// by the chunk step, the chunk table loads, the tile of each sample) done once per four
// samples; the tile of the next sample is the previous one's advanced by one. Every load
// address is clamped into its table or buffer; the host replay of this arithmetic
// (tests/combine_index) shows each clamp leaves its index unchanged wherever the loaded value
// is used. 128 threads a block (measured against 256 and 512: cfg1 45 -> 43 us).
constexpr int kCombineV = 4;
constexpr int kCombineThreads = 128;

template <int SC>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel4(const CombineParams p) {
    constexpr int V = kCombineV;
    const int64_t il = p.i_begin + ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * V;
    if (il >= p.i_end) return;
    const int i0 = (int)il;
    const int nv = (int)min((int64_t)V, p.i_end - il);
    const FrameGeom& G = p.g;
    const int step = (int)p.step_out;
    const int span = p.K * G.hop, ov = G.n_fft - G.hop;
    float res[V][SC];
#pragma unroll
    for (int s = 0; s < V; s++)
#pragma unroll
        for (int k = 0; k < SC; k++) res[s][k] = 0.0f;
    for (int gi = 0; gi < p.n_groups; gi++) {
        const ChunkGroup grp = p.groups[gi];
        const int P0 = i0 + grp.out_shift;
        const int out00 = (int)p.chunks[grp.c0].out0;
        const int n = grp.c1 - grp.c0;
        // the union of the four samples' chunk ranges of combine_kernel
        const int ghi = min((P0 + V - 1 - out00) / step, n - 1);
        const int glo = max((P0 - out00 - (int)p.max_out_len) / step, 0);
        float acc[V][SC];
        float wsum[V];
#pragma unroll
        for (int s = 0; s < V; s++) {
            wsum[s] = 0.0f;
#pragma unroll
            for (int k = 0; k < SC; k++) acc[s][k] = 0.0f;
        }
        for (int gl = glo; gl <= ghi + 1 && gl < n; gl++) {
            const int g = grp.c0 + gl;
            const ChunkDesc& d = p.chunks[g];
            const int u0 = P0 - (int)d.out0, olen = d.out_len;
            if (olen <= 0 || u0 + V <= 0 || u0 >= olen) continue;
            const float* Wg = p.W + d.w_off;
            const float* yg = p.Y + (int64_t)g * p.y_chunk_stride;
            const float* tg = p.Tr + (int64_t)g * p.tr_chunk_stride;
            const int j0 = d.y_off + u0;
            const int q0 = j0 + G.out_offset - G.first_pos;
            const int tau0 = q0 / span, uu0 = q0 - tau0 * span;
            // all four samples inside the chunk, none on a tile boundary's partial sums, and
            // 16-byte aligned rows: the weights as one vector and each row's samples as two
            // (the same sums in the same order as the per-sample loop below)
            const bool no_tr = q0 >= 0 && (tau0 < 1 || uu0 >= ov) && uu0 + V <= span;
            if (nv == V && u0 >= 0 && u0 + V <= olen && no_tr && ((d.w_off + u0) & 3) == 0 && (j0 & 1) == 0 &&
                (G.Lout & 1) == 0) {
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(Wg + u0));
                const float wv[V] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int s = 0; s < V; s++) wsum[s] += wv[s];
#pragma unroll
                for (int st = 0; st < SC / 2; st++) {
                    const float4* y4 = reinterpret_cast<const float4*>(yg + 2 * ((int64_t)st * G.Lout + j0));
                    const float4 a = __ldg(y4), b = __ldg(y4 + 1);
                    const float2 v[V] = {make_float2(a.x, a.y), make_float2(a.z, a.w), make_float2(b.x, b.y),
                                         make_float2(b.z, b.w)};
#pragma unroll
                    for (int s = 0; s < V; s++) {
                        acc[s][2 * st] = fmaf(wv[s], v[s].x, acc[s][2 * st]);
                        acc[s][2 * st + 1] = fmaf(wv[s], v[s].y, acc[s][2 * st + 1]);
                    }
                }
                continue;
            }
#pragma unroll
            for (int s = 0; s < V; s++) {
                const int u = u0 + s;
                if (s >= nv || u < 0 || u >= olen) continue;
                // the tile boundary region of sample s (q0 + s), as q / span would give it
                int tau, uu;
                if (q0 >= 0) {
                    tau = tau0;
                    uu = uu0 + s;
                    if (uu >= span) { uu -= span; tau++; }
                } else {
                    tau = (q0 + s) / span;
                    uu = q0 + s - tau * span;
                }
                const int uc = min(max(u, 0), olen - 1);   // = u here; clamped for the address
                const float w = __ldg(Wg + uc);
                wsum[s] += w;
                const float2* y = reinterpret_cast<const float2*>(yg) + (d.y_off + uc);
                const bool has_tr = tau >= 1 && tau < p.n_tiles && uu < ov;
                const int tc = min(max(tau, 1), p.n_tiles) - 1, uc2 = min(max(uu, 0), ov - 1);
                const float2* tr = reinterpret_cast<const float2*>(tg + (int64_t)tc * SC * ov) + uc2;
#pragma unroll
                for (int st = 0; st < SC / 2; st++) {
                    float2 v = __ldg(y + (int64_t)st * G.Lout);
                    if (has_tr) {
                        const float2 r = __ldg(tr + st * ov);
                        v = make_float2(v.x + r.x, v.y + r.y);
                    }
                    acc[s][2 * st] = fmaf(w, v.x, acc[s][2 * st]);
                    acc[s][2 * st + 1] = fmaf(w, v.y, acc[s][2 * st + 1]);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < V; s++) {
            const float inv = 1.0f / wsum[s];
#pragma unroll
            for (int k = 0; k < SC; k++) {
                float v = acc[s][k] * inv;
                if (p.nan_to_zero && !isfinite(v)) v = 0.0f;
                res[s][k] += p.shift_mean == 2 ? v / (float)p.n_groups : v;
            }
        }
    }
    float outv[V][SC];
    if (!p.bag) {
#pragma unroll
        for (int s = 0; s < V; s++)
#pragma unroll
            for (int k = 0; k < SC; k++) outv[s][k] = finish_plain(p, res[s][k]);
    } else {   // a bag member's pass reads the previous members' sums in out
#pragma unroll
        for (int s = 0; s < V; s++)
#pragma unroll
            for (int k = 0; k < SC; k++) outv[s][k] = s < nv ? finish_bag(p, k, i0 + s, res[s][k]) : 0.0f;
    }
    // rows of 4 samples as one 16-byte store where the row offset allows it
    const bool vec = nv == V && (p.len % V) == 0 && (i0 % V) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.out) % (sizeof(float) * V)) == 0;
    const auto put = [&](int row, const float (&v)[V]) {
        float* o = p.out + (int64_t)row * p.len + i0;
        if (vec) {
            *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int s = 0; s < V; s++)
                if (s < nv) o[s] = v[s];
        }
    };
#pragma unroll
    for (int k = 0; k < SC; k++) {
        float v[V];
#pragma unroll
        for (int s = 0; s < V; s++) v[s] = outv[s][k];
        put(k, v);
    }
    if (p.complement) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            float v[V];
#pragma unroll
            for (int s = 0; s < V; s++) {
                const float m = __ldg(p.mix + (int64_t)c * p.len + i0 + min(s, nv - 1));
                v[s] = s < nv ? m : 0.0f;
#pragma unroll
                for (int k = 0; k < SC; k++)
                    if (k % 2 == c && (p.complement == 2 || k < 2)) v[s] -= outv[s][k];
            }
            put(SC + c, v);
        }
    }
}

// ---- launchers ----------------------------------------------------------------------------
bool fused_supported(int n) { return n == 2048 || n == 4096 || n == 7680; }

int fused_threads(int n) {
    switch (n) {
        case 2048: return FftCfg<2048>::T;
        case 4096: return FftCfg<4096>::T;
        case 7680: return FftCfg<7680>::T;
        default: return 0;
    }
}

template <int ARCH, int N> static size_t smem_bytes_t() {
    return sizeof(float2) * ((size_t)padded_size(N) + 2 * (size_t)N) +
           (FftCfg<N>::SMEM_WIN ? sizeof(float) * (size_t)N : 0) +
           (ARCH == ARCH_ROFORMER ? sizeof(int2) * (size_t)(N / 2 + 2) : 0) +
           sizeof(float) * (size_t)FftCfg<N>::HOPMAX;   // the envelope period
}

size_t fused_smem_bytes(int arch, int n) {
    switch (n) {
        case 2048: return arch == ARCH_ROFORMER ? smem_bytes_t<ARCH_ROFORMER, 2048>() : smem_bytes_t<ARCH_TFC, 2048>();
        case 4096: return arch == ARCH_ROFORMER ? smem_bytes_t<ARCH_ROFORMER, 4096>() : smem_bytes_t<ARCH_TFC, 4096>();
        case 7680: return smem_bytes_t<ARCH_TFC, 7680>();
        default: return 0;
    }
}

template <int... Rs> static std::vector<int> radix_vec(RadixList<Rs...>) { return {Rs...}; }

std::vector<int> fused_radices(int n) {
    switch (n) {
        case 320: return radix_vec(FftCfg<320>::Plan{});
        case 512: return radix_vec(FftCfg<512>::Plan{});
        case 640: return radix_vec(FftCfg<640>::Plan{});
        case 960: return radix_vec(FftCfg<960>::Plan{});
        case 1024: return radix_vec(FftCfg<1024>::Plan{});
        case 2048: return radix_vec(FftCfg<2048>::Plan{});
        case 4096: return radix_vec(FftCfg<4096>::Plan{});
        case 7680: return radix_vec(FftCfg<7680>::Plan{});
        default: return {};
    }
}

std::vector<int> fused_fwd_radices(int n) {
    if (n == 2048) return radix_vec(FftCfg<2048>::FwdPlan{});
    return {};
}

template <int ARCH, int N> static int resident_t() {
    int per_sm = 0, n_sm = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaFuncSetAttribute(fused_kernel<ARCH, N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes_t<ARCH, N>()) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_kernel<ARCH, N>, FftCfg<N>::T,
                                                      smem_bytes_t<ARCH, N>()) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm * n_sm;
}

int fused_resident_ctas(int arch, int n) {
    switch (arch) {
        case ARCH_ROFORMER:
            if (n == 2048) return resident_t<ARCH_ROFORMER, 2048>();
            if (n == 4096) return resident_t<ARCH_ROFORMER, 4096>();
            break;
        case ARCH_TFC:
            if (n == 7680) return resident_t<ARCH_TFC, 7680>();
            if (n == 4096) return resident_t<ARCH_TFC, 4096>();
            if (n == 2048) return resident_t<ARCH_TFC, 2048>();
            break;
    }
    return 0;
}

int fused_max_hop(int n) {
    switch (n) {
        case 2048: return FftCfg<2048>::HOPMAX;
        case 4096: return FftCfg<4096>::HOPMAX;
        case 7680: return FftCfg<7680>::HOPMAX;
        default: return 0;
    }
}

template <int ARCH, int N>
static cudaError_t launch_fused_t(const FusedParams& p, cudaStream_t st) {
    const size_t smem = smem_bytes_t<ARCH, N>();
    cudaError_t e = cudaFuncSetAttribute(fused_kernel<ARCH, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    static int per_sm = 0, n_sm = 0;
    if (!per_sm) {
        int dev = 0;
        e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_kernel<ARCH, N>, FftCfg<N>::T, smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
    }
    const int64_t items = (int64_t)p.n_tiles * p.n_chunks;
    const int grid = (int)std::min<int64_t>(items, (int64_t)per_sm * n_sm);
    fused_kernel<ARCH, N><<<grid, FftCfg<N>::T, smem, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_fused(int arch, const FusedParams& p, cudaStream_t st) {
    if (p.n_chunks <= 0 || p.n_tiles <= 0) return cudaSuccess;
    if (fused_pair(arch, p.g.n_fft, p.g.hop)) return launch_fused_pair(p, st);
    switch (arch) {
        case ARCH_ROFORMER:
            if (p.g.n_fft == 2048) return launch_fused_t<ARCH_ROFORMER, 2048>(p, st);
            if (p.g.n_fft == 4096) return launch_fused_t<ARCH_ROFORMER, 4096>(p, st);
            break;
        case ARCH_TFC:
            if (p.g.n_fft == 7680) return launch_fused_t<ARCH_TFC, 7680>(p, st);
            if (p.g.n_fft == 4096) return launch_fused_t<ARCH_TFC, 4096>(p, st);
            if (p.g.n_fft == 2048) return launch_fused_t<ARCH_TFC, 2048>(p, st);
            break;
    }
    return cudaErrorInvalidValue;
}

// ---- mask transposition -------------------------------------------------------------------
// f-major planes [S][P][F][T] per chunk (t fastest) -> t-major [S][T][F] float4 per chunk,
// component p = plane p (zero from P up). A CTA moves 32 x 32 (f, t) tiles of every plane,
// work item w = ((chunk * S + stem) * f tiles + f tile) * t tiles + t tile, striding by the grid:
// rows read 32 consecutive t (128 bytes), rows written 32 consecutive f (512 bytes of float4).
constexpr int kTile = 32;

__global__ void __launch_bounds__(256) mask_transpose(const float* __restrict__ in, int64_t in_chunk_stride,
                                                      int n_cs, int S, int P, int F, int T,
                                                      float4* __restrict__ out, int64_t out_chunk_stride) {
    __shared__ float tile[4][kTile][kTile + 1];
    const int lx = threadIdx.x & 31, ly = threadIdx.x >> 5;
    const int ntx = (T + kTile - 1) / kTile, nty = (F + kTile - 1) / kTile;
    const int64_t n_work = (int64_t)ntx * nty * n_cs;
    for (int64_t w = blockIdx.x; w < n_work; w += gridDim.x) {
        const int tx = (int)(w % ntx);
        const int64_t rest = w / ntx;
        const int ty = (int)(rest % nty), cs = (int)(rest / nty);
        const int f0 = ty * kTile, t0 = tx * kTile;
        const int ci = cs / S, s = cs - ci * S;
        const float* src = in + ci * in_chunk_stride + (int64_t)s * P * F * T;
        // all 16 loads of a thread in flight before the first shared-memory store
        float v[4][kTile / 8];
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int k = 0; k < kTile / 8; k++) {
                const int f = f0 + ly + 8 * k, t = t0 + lx;
                v[p][k] = (p < P && f < F && t < T) ? ld_stream(src + ((int64_t)p * F + f) * T + t) : 0.0f;
            }
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int k = 0; k < kTile / 8; k++) tile[p][ly + 8 * k][lx] = v[p][k];
        __syncthreads();
        float4* dst = out + ci * out_chunk_stride + (int64_t)s * T * F;
        for (int r = ly; r < kTile; r += 8) {
            const int t = t0 + r, f = f0 + lx;
            if (t < T && f < F)
                dst[(int64_t)t * F + f] = make_float4(tile[0][lx][r], tile[1][lx][r], tile[2][lx][r], tile[3][lx][r]);
        }
        __syncthreads();
    }
}

cudaError_t launch_mask_transpose(const float* in, int64_t in_chunk_stride, int n_chunks, int S, int P, int F,
                                  int T, float4* out, int64_t out_chunk_stride, cudaStream_t st, int max_ctas) {
    if (n_chunks <= 0) return cudaSuccess;
    if (P < 1 || P > 4 || F < 1 || T < 1 || S < 1) return cudaErrorInvalidValue;
    const int n_cs = n_chunks * S;
    const int64_t n_work = (int64_t)((T + kTile - 1) / kTile) * ((F + kTile - 1) / kTile) * n_cs;
    int64_t blocks = std::min<int64_t>(n_work, INT32_MAX);
    if (max_ctas > 0) blocks = std::min<int64_t>(blocks, max_ctas);
    mask_transpose<<<(unsigned)blocks, 256, 0, st>>>(in, in_chunk_stride, n_cs, S, P, F, T, out, out_chunk_stride);
    return cudaGetLastError();
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t st) {
    if (p.i_end <= p.i_begin) return cudaSuccess;
    const int threads = 256;
    if (p.C == 2 && p.S <= 2) {   // one or two stereo stems: four samples per thread (from
        // three stems up, its registers cost more occupancy than the shared bookkeeping saves)
        const int64_t per = (int64_t)kCombineThreads * kCombineV;
        const unsigned b4 = (unsigned)((p.i_end - p.i_begin + per - 1) / per);
        if (p.S == 1) combine_kernel4<2><<<b4, kCombineThreads, 0, st>>>(p);
        else combine_kernel4<4><<<b4, kCombineThreads, 0, st>>>(p);
        return cudaGetLastError();
    }
    const unsigned blocks = (unsigned)((p.i_end - p.i_begin + threads - 1) / threads);
    switch (p.S * p.C) {
        case 1: combine_kernel<1><<<blocks, threads, 0, st>>>(p); break;
        case 2: combine_kernel<2><<<blocks, threads, 0, st>>>(p); break;
        case 3: combine_kernel<3><<<blocks, threads, 0, st>>>(p); break;
        case 4: combine_kernel<4><<<blocks, threads, 0, st>>>(p); break;
        case 5: combine_kernel<5><<<blocks, threads, 0, st>>>(p); break;
        case 6: combine_kernel<6><<<blocks, threads, 0, st>>>(p); break;
        case 7: combine_kernel<7><<<blocks, threads, 0, st>>>(p); break;
        case 8: combine_kernel<8><<<blocks, threads, 0, st>>>(p); break;
        case 10: combine_kernel<10><<<blocks, threads, 0, st>>>(p); break;
        case 12: combine_kernel<12><<<blocks, threads, 0, st>>>(p); break;
        case 14: combine_kernel<14><<<blocks, threads, 0, st>>>(p); break;
        case 16: combine_kernel<16><<<blocks, threads, 0, st>>>(p); break;
        default: return cudaErrorInvalidValue;   // S <= 8 and C <= 2 never get here
    }
    return cudaGetLastError();
}

} // namespace stg
