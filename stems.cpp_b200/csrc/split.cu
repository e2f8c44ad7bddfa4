// split.cu -- the front and back halves of the path, for a real network between them.
//
// front_kernel: for every frame of every chunk, the same padded load and stereo-packed
// forward FFT as the fused kernel, then the two channels' spectra written in the network's
// input layout: complex [C][F][T] (src/stft.h:146-164 torch_stft, 79-103 htdemucs_spec),
// HTDemucs CaC planes (src/htdemucs.cpp:423-433), RoFormer band-major features
// (src/roformer.cpp:226-241) or TFC-TDF CaC planes with the low bins zero
// (src/tfc_tdf.cpp:366-376).
// back_kernel: for every stem and frame, a spectrogram read from the network's output layout
// (src/htdemucs.cpp:463-469, src/tfc_tdf.cpp:381-387, or complex for torch_istft /
// htdemucs_ispec), the c2r conventions (DC and Nyquist imaginary parts dropped, the HTDemucs
// Nyquist bin zero), the inverse FFT, the window, and the overlap-add into the fused kernel's
// Y / Tr scratch.
#include <type_traits>

#include <algorithm>

#include "fft.cuh"
#include "frame.cuh"
#include "kernels.h"

namespace stg {

namespace {

// The spectra of bin f (zl, zr) to the front layout, frame t of chunk ci. L: the layout, or
// -1 to read it from p.layout.
template <int N, int L>
__device__ __forceinline__ void front_store(const SplitParams& p, const int2* btab, int ci, int t, int f,
                                            float2 zl, float2 zr) {
    const int T = p.g.T, C = p.n_channels;
    float* out = p.net + (int64_t)ci * p.net_chunk_stride;
    const int64_t plane = (int64_t)p.n_bins * T, idx = (int64_t)f * T + t;
    switch (L >= 0 ? L : p.layout) {
        case FRONT_COMPLEX:
            if (f < p.n_bins) {
                reinterpret_cast<float2*>(out)[idx] = zl;
                if (C > 1) reinterpret_cast<float2*>(out)[plane + idx] = zr;
            }
            break;
        case FRONT_CAC:
            if (f < p.n_bins) {
                if (p.cac_stats) {   // (v - mean) / (1e-5 + std) (src/htdemucs.cpp:436)
                    const double2 st = p.cac_stats[ci];
                    const float mean = (float)st.x, inv = (float)(1.0 / (1e-5 + st.y));
                    zl = make_float2((zl.x - mean) * inv, (zl.y - mean) * inv);
                    zr = make_float2((zr.x - mean) * inv, (zr.y - mean) * inv);
                }
                out[idx] = zl.x;
                out[plane + idx] = zl.y;
                if (C > 1) {
                    out[2 * plane + idx] = zr.x;
                    out[3 * plane + idx] = zr.y;
                }
            }
            break;
        case FRONT_ZSPEC:
            if (f < p.n_bins)
                p.zspec[(int64_t)ci * p.z_chunk_stride + (int64_t)t * p.n_bins + f] = make_float4(zl.x, zl.y, zr.x, zr.y);
            break;
        case FRONT_TFC:
            if (f < p.n_bins) {
                const bool z = f < p.zero_bins;
                out[idx] = z ? 0.0f : zl.x;
                out[plane + idx] = z ? 0.0f : zl.y;
                out[2 * plane + idx] = z ? 0.0f : zr.x;
                out[3 * plane + idx] = z ? 0.0f : zr.y;
            }
            break;
        default: {   // FRONT_BANDS: every band holding f gets the bin's entry (j*C + c)*2 + {re, im}
            if (f >= p.n_bins) break;
            const int2 e = btab[f];
            const int v[2] = {e.x, e.y};
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const unsigned size = (unsigned)v[k] >> 22;
                if (!size) continue;
                float* q = out + (int64_t)((v[k] & 0x3fffff) + t * (int)size) * (2 * C);
                if (C > 1) *reinterpret_cast<float4*>(q) = make_float4(zl.x, zl.y, zr.x, zr.y);
                else *reinterpret_cast<float2*>(q) = zl;
            }
            if (p.bin_multi) {
                const int e1 = __ldg(p.bin_ebeg + f + 1);
                for (int k = __ldg(p.bin_ebeg + f) + 2; k < e1; k++) {
                    const int2 en = __ldg(p.bin_ent + k);
                    float* q = out + en.x + (int64_t)t * en.y;
                    q[0] = zl.x; q[1] = zl.y;
                    if (C > 1) { q[2] = zr.x; q[3] = zr.y; }
                }
            }
        }
    }
}

// Bin f of stem s, frame t, from the back layout: the two channels' spectra.
__device__ __forceinline__ void back_load(const SplitParams& p, int ci, int s, int t, int f, float2& yl, float2& yr) {
    const int T = p.g.T, C = p.n_channels;
    const float* in = p.net + (int64_t)ci * p.net_chunk_stride;
    yl = yr = make_float2(0.f, 0.f);
    if (f >= p.n_bins) return;   // the HTDemucs Nyquist bin, TFC-TDF bins from dim_f up
    const int64_t plane = (int64_t)p.n_bins * T, idx = (int64_t)f * T + t;
    switch (p.layout) {
        case BACK_COMPLEX: {
            const float2* z = reinterpret_cast<const float2*>(in);
            yl = z[idx];
            if (C > 1) yr = z[plane + idx];
            break;
        }
        case BACK_CAC: {
            const float* q = in + (int64_t)s * 2 * C * plane + idx;
            yl = make_float2(q[0], q[plane]);
            if (C > 1) yr = make_float2(q[2 * plane], q[3 * plane]);
            if (p.cac_stats) {   // v * std + mean (src/htdemucs.cpp:469)
                const double2 st = p.cac_stats[ci];
                const float mean = (float)st.x, sd = (float)st.y;
                yl = make_float2(fmaf(yl.x, sd, mean), fmaf(yl.y, sd, mean));
                yr = make_float2(fmaf(yr.x, sd, mean), fmaf(yr.y, sd, mean));
                if (C == 1) yr = make_float2(0.f, 0.f);
            }
            break;
        }
        default: {   // BACK_TFC (BACK_ZMASK has its own batched path in back_kernel)
            const float* q = in + (int64_t)s * 4 * plane + idx;
            yl = make_float2(q[0], q[plane]);
            yr = make_float2(q[2 * plane], q[3 * plane]);
        }
    }
}

// BACK_ZMASK: ox = Z * M for bin f, with the CaC normalisation around the stand-in
// (src/htdemucs.cpp:434-436, 469); z and m were loaded by the caller (zero past n_bins).
__device__ __forceinline__ void zmask_apply(const SplitParams& p, int ci, float4 z, float4 m, float2& yl,
                                            float2& yr) {
    float2 zl = make_float2(z.x, z.y), zr = make_float2(z.z, z.w);
    if (p.cac_stats) {
        const double2 st = p.cac_stats[ci];
        const float mean = (float)st.x, sd = (float)st.y, inv = (float)(1.0 / (1e-5 + st.y));
        zl = make_float2((zl.x - mean) * inv, (zl.y - mean) * inv);
        zr = make_float2((zr.x - mean) * inv, (zr.y - mean) * inv);
        yl = cmul(zl, make_float2(m.x, m.y));
        yr = cmul(zr, make_float2(m.z, m.w));
        yl = make_float2(fmaf(yl.x, sd, mean), fmaf(yl.y, sd, mean));
        yr = p.n_channels > 1 ? make_float2(fmaf(yr.x, sd, mean), fmaf(yr.y, sd, mean)) : make_float2(0.f, 0.f);
    } else {
        yl = cmul(zl, make_float2(m.x, m.y));
        yr = cmul(zr, make_float2(m.z, m.w));
    }
}

// The codelets' complex type: at n_fft 4096 (HTDemucs) their additions run in f32x2
// instructions (fft.cuh: PF2)
template <int N> using SplitCV = std::conditional_t<N == 4096, PF2, float2>;

// The CTAs per SM the HTDemucs segment-spectra instance (FRONT_ZSPEC) aims its registers at
// (two: at three, the 80-register cap spills and the separation is slower); 0 leaves the
// other instances to the compiler's default, which an explicit 1 would raise by 30-70 registers.
template <int N, int L> constexpr int front_minb() { return L == FRONT_ZSPEC && N == 4096 ? 2 : 0; }

// L: the layout (the HTDemucs FRONT_ZSPEC instance), or -1 to read it from p.layout.
template <int N, int L>
__global__ void __launch_bounds__(FftCfg<N>::T, (front_minb<N, L>())) front_kernel(const SplitParams p) {
    constexpr int T = FftCfg<N>::T;
    using Plan = typename FftCfg<N>::Plan;
    constexpr int R1 = Head<Plan>::first;
    using FwdRest = typename Head<Plan>::tail;
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* in_ring = buf + padded_size(N);
    int2* btab = reinterpret_cast<int2*>(in_ring + N);
    const TwGlobal tw{p.tw};
    const int tid = threadIdx.x;
    const FrameGeom& G = p.g;
    const int hop = G.hop, C = p.n_channels;
    const float* chL = p.mix;
    const float* chR = p.mix + (C > 1 ? p.len : 0);
    const int lxf = G.ht_pad ? G.ht_lxf : G.Lc;
    const float half_fwd = 0.5f * p.fwd_scale;
    if (p.layout == FRONT_BANDS)
        for (int i = tid; i < p.n_bins; i += T) btab[i] = __ldg(p.bin_tab + i);
    InPrefetch<T, split_hopmax<N>()> nx;
    __shared__ double red[2 * (T / 32)];

    for (int item = blockIdx.x; item < p.n_tiles * p.n_chunks; item += gridDim.x) {
        const int tile = item % p.n_tiles, ci = item / p.n_tiles;
        const ChunkDesc cd = p.chunks[ci];
        const int t_begin = tile * p.K, t_end = min(G.T, t_begin + p.K);
        const int lin = linear_offset(p, cd, t_begin, t_end);
        double acc_s = 0.0, acc_q = 0.0;   // FRONT_STATS
        {
            const int q0 = G.first_pos + t_begin * hop;
            for (int n = tid; n < N; n += T) in_ring[ring_slot<N>(q0 + n)] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + n);
#pragma unroll
            for (int k = 0; k < nx.K; k++) {
                const int u = tid + k * T;
                if (u < hop && t_begin + 1 < t_end) nx.v[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + N + u);
            }
        }
        __syncthreads();
        for (int t = t_begin; t < t_end; t++) {
            const int q0 = G.first_pos + t * hop;
            pass_io<N, R1, 1, T, false, false, false, SplitCV<N>>(
                tw, tid,
                [&](int j, int r) {
                    const int n = j + r * (N / R1);
                    const float2 x = in_ring[ring_slot<N>(q0 + n)];
                    const float w = __ldg(p.win + n);
                    return make_float2(x.x * w, x.y * w);
                },
                [&](int base, int r, float2 v) { buf[pad_store<R1, 1>(base, r)] = v; });
            __syncthreads();
            if (t + 1 < t_end) {
#pragma unroll
                for (int k = 0; k < nx.K; k++) {
                    const int u = tid + k * T;
                    if (u < hop) in_ring[ring_slot<N>(q0 + N + u)] = nx.v[k];
                }
                if (t + 2 < t_end) {
#pragma unroll
                    for (int k = 0; k < nx.K; k++) {
                        const int u = tid + k * T;
                        if (u < hop) nx.v[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + hop + N + u);
                    }
                }
            }
            passes<N, T, false, R1, false, SplitCV<N>>(buf, tw, tid, FwdRest{});
            // the thread's bins f = tid + i*T (the FRONT_ZSPEC instance unrolls over its slots)
            constexpr int BPT = L == FRONT_ZSPEC ? (N / 2 + T) / T : 1;
#pragma unroll
            for (int i = 0; i < BPT; i++) {
                for (int f = tid + i * T; f < p.n_bins && f <= N / 2; f += BPT * T) {
                    const int fm = f == 0 ? 0 : N - f;
                    const float2 X = buf[pad_idx(f)], Xm = buf[pad_idx(fm)];
                    const float2 zl = make_float2(half_fwd * (X.x + Xm.x), half_fwd * (X.y - Xm.y));
                    const float2 zr = make_float2(half_fwd * (X.y + Xm.y), -half_fwd * (X.x - Xm.x));
                    if (p.stats_out && f < p.n_bins) {
                        acc_s += (double)zl.x + (double)zl.y;
                        acc_q += (double)zl.x * zl.x + (double)zl.y * zl.y;
                        if (C > 1) {
                            acc_s += (double)zr.x + (double)zr.y;
                            acc_q += (double)zr.x * zr.x + (double)zr.y * zr.y;
                        }
                    }
                    if (L == FRONT_ZSPEC || (L < 0 && p.layout != FRONT_STATS)) front_store<N, L>(p, btab, ci, t, f, zl, zr);
                    if constexpr (L == FRONT_ZSPEC) break;
                }
            }
            __syncthreads();
        }
        if (p.stats_out) {   // block sums in a fixed order, one partial per item
            for (int o = 16; o > 0; o >>= 1) {
                acc_s += __shfl_down_sync(0xffffffffu, acc_s, o);
                acc_q += __shfl_down_sync(0xffffffffu, acc_q, o);
            }
            if ((tid & 31) == 0) { red[2 * (tid >> 5)] = acc_s; red[2 * (tid >> 5) + 1] = acc_q; }
            __syncthreads();
            if (tid == 0) {
                double s = 0.0, q = 0.0;
                for (int w = 0; w < T / 32; w++) { s += red[2 * w]; q += red[2 * w + 1]; }
                p.stats_out[(int64_t)ci * p.n_tiles + tile] = make_double2(s, q);
            }
            __syncthreads();
        }
    }
}

// n_fft 4096 (HTDemucs): registers capped for three CTAs per SM, which its shared memory allows
template <int N>
__global__ void __launch_bounds__(FftCfg<N>::T, (N == 4096 ? 3 : 0)) back_kernel(const SplitParams p) {
    constexpr int T = FftCfg<N>::T;
    using Plan = typename FftCfg<N>::Plan;
    using InvInit = typename Init<Plan>::type;
    constexpr int RL = Init<Plan>::last, NSL = Init<Plan>::prod;
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* out_ring = buf + padded_size(N);
    float* env_s = reinterpret_cast<float*>(out_ring + N);   // the envelope period
    const TwGlobal tw{p.tw};
    const int tid = threadIdx.x;
    const FrameGeom& G = p.g;
    const int hop = G.hop, C = p.n_channels;
    for (int i = tid; i < N; i += T) out_ring[i] = make_float2(0.f, 0.f);
    // the window (times the inverse scale) at the samples this thread overlap-adds, tid + r*NSL,
    // in registers when the last pass has one butterfly per thread
    constexpr bool RW = N / RL == T;
    float wreg[RW ? RL : 1];
#pragma unroll
    for (int r = 0; r < (RW ? RL : 1); r++) wreg[r] = RW ? __ldg(p.win + tid + r * NSL) * p.inv_scale : 0.0f;
    const bool env_on = p.env_period != nullptr;
    if (env_on)
        for (int i = tid; i < hop; i += T) env_s[i] = __ldg(p.env_period + i);

    // work items are (chunk, tile, stem), the stems of a tile adjacent: a stem's frames are a
    // CTA's work, and the tile's other stems, on other SMs at about the same time, read the same
    // Z rows from L2
    const int n_items = p.n_tiles * p.n_chunks * p.S;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int s = item % p.S, ct = item / p.S;
        const int tile = ct % p.n_tiles, ci = ct / p.n_tiles;
        const int t_begin = tile * p.K, t_end = min(G.T, t_begin + p.K);
        const bool last_tile = t_end == G.T;
        {
            float* Ys = p.Y + (int64_t)ci * p.y_chunk_stride + (int64_t)s * C * G.Lout;
            float* Trs = p.Tr + (int64_t)ci * p.tr_chunk_stride + ((int64_t)tile * p.S + s) * C * (N - hop);
            for (int t = t_begin; t < t_end; t++) {
                const int q0 = G.first_pos + t * hop;
                // BACK_ZMASK: the next frame's Z and mask rows (contiguous, 16-byte aligned) asked
                // of L2 a frame ahead (cfg4's back kernel 1.41 -> 1.28 ms)
                if (p.layout == BACK_ZMASK && tid == 0 && t + 1 < t_end) {
                    const unsigned bytes = (unsigned)p.n_bins * 16u;
                    prefetch_l2(p.zspec + (int64_t)ci * p.z_chunk_stride + (int64_t)(t + 1) * p.n_bins, bytes);
                    prefetch_l2(p.net + (int64_t)ci * p.net_chunk_stride + 4 * ((int64_t)s * G.T + t + 1) * p.n_bins, bytes);
                }
                auto pack = [&](int f, float2 yl, float2 yr) {
                    if (f == 0 || f == N / 2) { yl.y = 0.0f; yr.y = 0.0f; }   // c2r ignores these
                    const int fm = f == 0 ? 0 : N - f;
                    buf[pad_idx(f)] = make_float2(yl.x - yr.y, yl.y + yr.x);
                    if (f != 0 && f != N / 2) buf[pad_idx(fm)] = make_float2(yl.x + yr.y, yr.x - yl.y);
                };
                bool paired = false;
                if constexpr (N == 4096) {
                    if (p.layout == BACK_ZMASK) {
                        // lane pairs: threads 2m and 2m + 1 take the inverse's first butterflies
                        // j = m and 256 - m (thread 1: 128). Butterfly j reads the points j + 256r,
                        // and bin k's mirror point N - k lies in the partner's butterfly, so each
                        // thread repacks its own bins j + 256r (r < 8; thread 0 also N/2) into both
                        // points, keeps the one at its own position and hands the partner the other
                        // (one shuffle per point); the first pass then runs in registers.
                        // (groups of three bins' loads in flight: five spilled 48 bytes at the
                        // 128-register cap and ran 11 % slower)
                        paired = true;
                        constexpr int NB = N / 16, GRP = 3;
                        static_assert(NB == T && Head<InvInit>::first == 16, "one first-pass butterfly per thread");
                        const int m2 = tid >> 1;
                        const int j = (tid & 1) ? (m2 ? NB - m2 : NB / 2) : m2;
                        const float4* zs = p.zspec + (int64_t)ci * p.z_chunk_stride + (int64_t)t * p.n_bins;
                        const float* ms = p.net + (int64_t)ci * p.net_chunk_stride + 4 * ((int64_t)s * G.T + t) * p.n_bins;
                        SplitCV<N> v[16];
                        float2 gm[9];
                        float2 g8 = make_float2(0.f, 0.f);
#pragma unroll
                        for (int g0 = 0; g0 < 9; g0 += GRP) {
                            float4 z[GRP], m[GRP];
#pragma unroll
                            for (int k = 0; k < GRP; k++) {
                                const int r = g0 + k, f = j + NB * r;
                                z[k] = m[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                                if (r < 9 && (r < 8 || tid == 0) && f < p.n_bins) {
                                    z[k] = zs[f];
                                    m[k] = ld_stream4(ms + 4 * f);
                                }
                            }
#pragma unroll
                            for (int k = 0; k < GRP; k++) {
                                const int r = g0 + k;
                                if (r >= 9) continue;
                                float2 yl, yr;
                                zmask_apply(p, ci, z[k], m[k], yl, yr);
                                if (r == 8 || (r == 0 && tid == 0)) { yl.y = 0.0f; yr.y = 0.0f; }   // c2r ignores these
                                const float2 gx = make_float2(yl.x - yr.y, yl.y + yr.x);
                                if (r < 8) {
                                    v[r] = gx;
                                    gm[r] = make_float2(yl.x + yr.y, yr.x - yl.y);
                                } else {
                                    g8 = gx;
                                }
                            }
                        }
#pragma unroll
                        for (int r = 8; r < 16; r++) {
                            const float2 q = gm[15 - r];
                            const float2 t2 = make_float2(__shfl_xor_sync(0xffffffffu, q.x, 1),
                                                          __shfl_xor_sync(0xffffffffu, q.y, 1));
                            // the butterflies 0 and 128 hold their own mirrors
                            const float2 own = tid == 1 ? gm[15 - r] : (r == 8 ? g8 : gm[(16 - r) & 7]);
                            v[r] = tid > 1 ? t2 : own;
                        }
                        Dft<16, true>::template run<1>(v);
                        // (the previous frame's overlap-add barrier ordered its reads of buf first)
#pragma unroll
                        for (int r = 0; r < 16; r++) buf[pad_store<16, 1>(16 * j, r)] = v[r];
                        __syncthreads();
                        passes<N, T, true, 16, false, SplitCV<N>>(buf, tw, tid, typename Head<InvInit>::tail{});
                    }
                }
                if (!paired) {
                    if (p.layout == BACK_ZMASK) {
                        // the bins' Z and mask vectors in groups of GRP slots, every load of a group in
                        // flight before the first is used
                        constexpr int BPT = (N / 2 + T) / T, GRP = 5;
                        const float4* zs = p.zspec + (int64_t)ci * p.z_chunk_stride + (int64_t)t * p.n_bins;
                        const float* ms = p.net + (int64_t)ci * p.net_chunk_stride + 4 * ((int64_t)s * G.T + t) * p.n_bins;
#pragma unroll
                        for (int g0 = 0; g0 < BPT; g0 += GRP) {
                            float4 z[GRP], m[GRP];
#pragma unroll
                            for (int k = 0; k < GRP; k++) {
                                const int f = tid + (g0 + k) * T;
                                z[k] = m[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                                if (g0 + k < BPT && f < p.n_bins) {
                                    z[k] = zs[f];
                                    m[k] = ld_stream4(ms + 4 * f);
                                }
                            }
#pragma unroll
                            for (int k = 0; k < GRP; k++) {
                                const int f = tid + (g0 + k) * T;
                                if (g0 + k >= BPT || f > N / 2) continue;
                                float2 yl, yr;
                                zmask_apply(p, ci, z[k], m[k], yl, yr);
                                pack(f, yl, yr);
                            }
                        }
                    } else {
                        for (int f = tid; f <= N / 2; f += T) {
                            float2 yl, yr;
                            back_load(p, ci, s, t, f, yl, yr);
                            pack(f, yl, yr);
                        }
                    }
                    __syncthreads();
                    passes<N, T, true, 1, false, SplitCV<N>>(buf, tw, tid, InvInit{});
                }
                // the overlap-add: a thread adds into the ring positions q0 + n, n = tid mod T, the
                // ones it flushes below, so the barrier goes between the pass's loads and stores
                // (the next frame's packing rewrites buf) and the flush needs none
                static_assert(NSL % T == 0, "the overlap-add and the flush give a thread the same positions");
                pass_io<N, RL, NSL, T, true, true, false, SplitCV<N>>(
                    tw, tid, [&](int j, int r) { return buf[pad_load<N, RL>(j, r)]; },
                    [&](int base, int r, float2 v) {
                        const int n = base + r * NSL;
                        const float w = RW ? wreg[r] : __ldg(p.win + n) * p.inv_scale;
                        float2& o = out_ring[ring_slot<N>(q0 + n)];
                        o = make_float2(fmaf(v.x, w, o.x), fmaf(v.y, w, o.y));
                    });
                const bool last = t == t_end - 1;
                const int ny = (last && last_tile) ? N : hop;
                const int nflush = last ? N : hop;
                int r = 0;   // the envelope period slot of this thread's sample (kernels.cu)
                if (env_on) {
                    r = (q0 - G.out_offset + tid - p.env_lo) % hop;
                    if (r < 0) r += hop;
                }
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
                // the next frame's first barrier orders these ring writes before later reads
            }
            __syncthreads();
        }
    }
}

template <class K>
cudaError_t launch_persistent(K kernel, int threads, size_t smem, int64_t items, cudaStream_t st,
                              const SplitParams& p) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0, n_sm = 0, dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem)) != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = (int)std::min<int64_t>(items, (int64_t)per_sm * n_sm);
    kernel<<<grid, threads, smem, st>>>(p);
    return cudaGetLastError();
}

template <int N> cudaError_t front_t(const SplitParams& p, cudaStream_t st) {
    const size_t smem = sizeof(float2) * ((size_t)padded_size(N) + N);   // frame and input ring
    const int64_t items = (int64_t)p.n_tiles * p.n_chunks;
    if constexpr (N == 4096)
        if (p.layout == FRONT_ZSPEC)
            return launch_persistent(front_kernel<N, FRONT_ZSPEC>, FftCfg<N>::T, smem, items, st, p);
    return launch_persistent(front_kernel<N, -1>, FftCfg<N>::T, smem + sizeof(int2) * (size_t)(N / 2 + 2), items, st, p);
}
template <int N> cudaError_t back_t(const SplitParams& p, cudaStream_t st) {
    const size_t smem = sizeof(float2) * ((size_t)padded_size(N) + N) + sizeof(float) * (size_t)(N / 2);
    return launch_persistent(back_kernel<N>, FftCfg<N>::T, smem, (int64_t)p.n_tiles * p.n_chunks * p.S, st, p);
}

} // namespace

bool split_supported(int n) {
    switch (n) {
        case 320: case 512: case 640: case 960: case 1024: case 2048: case 4096: case 7680: return true;
    }
    return false;
}

int split_max_hop(int n) { return split_supported(n) ? n / 2 : 0; }

namespace {
template <class K> int resident_of(K kernel, int threads, size_t smem) {
    int per_sm = 0, n_sm = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm * n_sm;
}
// the resident CTAs of the front (generic layouts) or the back kernel at size N
template <int N> int split_resident_t(bool front) {
    const size_t ring = sizeof(float2) * ((size_t)padded_size(N) + N);
    return front ? resident_of(front_kernel<N, -1>, FftCfg<N>::T, ring + sizeof(int2) * (size_t)(N / 2 + 2))
                 : resident_of(back_kernel<N>, FftCfg<N>::T, ring + sizeof(float) * (size_t)(N / 2));
}
} // namespace

int split_resident_ctas(int n, bool front) {
    switch (n) {
        case 320: return split_resident_t<320>(front);
        case 512: return split_resident_t<512>(front);
        case 640: return split_resident_t<640>(front);
        case 960: return split_resident_t<960>(front);
        case 1024: return split_resident_t<1024>(front);
        case 2048: return split_resident_t<2048>(front);
        case 4096: return split_resident_t<4096>(front);
        case 7680: return split_resident_t<7680>(front);
    }
    return 0;
}

int back_resident_ctas(int n) { return split_resident_ctas(n, false); }

cudaError_t launch_front(const SplitParams& p, cudaStream_t st) {
    if (p.n_chunks <= 0 || p.n_tiles <= 0) return cudaSuccess;
    if (p.g.hop > split_max_hop(p.g.n_fft)) return cudaErrorInvalidValue;
    switch (p.g.n_fft) {
        case 320: return front_t<320>(p, st);
        case 512: return front_t<512>(p, st);
        case 640: return front_t<640>(p, st);
        case 960: return front_t<960>(p, st);
        case 1024: return front_t<1024>(p, st);
        case 2048: return front_t<2048>(p, st);
        case 4096: return front_t<4096>(p, st);
        case 7680: return front_t<7680>(p, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_back(const SplitParams& p, cudaStream_t st) {
    if (p.n_chunks <= 0 || p.n_tiles <= 0) return cudaSuccess;
    switch (p.g.n_fft) {
        case 320: return back_t<320>(p, st);
        case 512: return back_t<512>(p, st);
        case 640: return back_t<640>(p, st);
        case 960: return back_t<960>(p, st);
        case 1024: return back_t<1024>(p, st);
        case 2048: return back_t<2048>(p, st);
        case 4096: return back_t<4096>(p, st);
        case 7680: return back_t<7680>(p, st);
    }
    return cudaErrorInvalidValue;
}

} // namespace stg
