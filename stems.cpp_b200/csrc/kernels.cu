// kernels.cu -- the fused spectral kernel and the chunk combine for sm_100a.
//
// Fused kernel, one CTA per (frame tile, chunk). For every stem and every frame of its tile:
//   1. load the frame of both channels straight from the track (reflect / zero padding of
//      the chunk, the track and the STFT evaluated per sample), window it, and pack the two
//      real channels as one complex frame L + iR;
//   2. forward FFT in shared memory (fft.cuh);
//   3. split the two channels' spectra, apply the architecture's spectral op (the stand-in
//      for the network: complex mask, band-averaged mask, or CaC real mask), drop what the
//      reference's c2r drops, and repack the two masked spectra as one Hermitian pair;
//   4. inverse FFT, window, and overlap-add into a ring buffer of n_fft samples per channel;
//   5. flush the hop of samples that no later frame of the tile touches, scaled by the
//      inverse window-sum envelope, to the chunk output Y. The last frame of a tile sends
//      its n_fft - hop trailing samples to Tr instead; the combine adds them to the next
//      tile's leading samples, so every sum is formed in a fixed order (no atomics).
// Combine kernel: one thread per output sample; it sums the chunks that cover the sample
// with their crossfade weights (reading Y and the tile-boundary partials Tr), divides by the
// summed weight, and applies the architecture's epilogue (nan_to_num, compensation,
// complement).
#include "fft.cuh"
#include "kernels.h"

namespace stg {

template <int N> struct FftCfg;
template <> struct FftCfg<2048> { static constexpr int T = 128; using Plan = RadixList<8, 16, 16>; };
template <> struct FftCfg<4096> { static constexpr int T = 256; using Plan = RadixList<16, 16, 16>; };
template <> struct FftCfg<7680> { static constexpr int T = 512; using Plan = RadixList<15, 8, 8, 8>; };

__device__ __forceinline__ int64_t reflect1(int64_t j, int64_t n) {
    if (j < 0) j = -j;
    if (j >= n) j = 2 * (n - 1) - j;
    return j;
}

__device__ __forceinline__ float chunk_sample(const FusedParams& p, const ChunkDesc& cd,
                                              const float* __restrict__ chan, int64_t pl) {
    if (pl >= cd.valid) {
        if (!cd.tail_reflect) return 0.0f;
        pl = 2 * (int64_t)(cd.valid - 1) - pl;
    }
    int64_t x = cd.src0 + pl;
    if (p.reflect_global) x = reflect1(x, p.len);
    else if (x < 0 || x >= p.len) return 0.0f;
    return __ldg(chan + x);
}

// The stand-in network: turn the two channels' spectra at bin f of frame t into the
// spectra the iSTFT consumes for stem s.
template <int ARCH, int N>
__device__ __forceinline__ void spectral_op(const FusedParams& p, int ci, int s, int t, int f,
                                            float2 zl, float2 zr, float2& yl, float2& yr) {
    const float* __restrict__ m = p.mask + (int64_t)ci * p.mask_chunk_stride;
    if constexpr (ARCH == ARCH_ROFORMER) {
        // src/roformer.cpp:251-278: masks of every band holding f, averaged, times z.
        float2 al = make_float2(0.f, 0.f), ar = make_float2(0.f, 0.f);
        const float* ms = m + (int64_t)s * p.stem_stride;
        const int e1 = __ldg(p.bin_ebeg + f + 1);
        for (int e = __ldg(p.bin_ebeg + f); e < e1; e++) {
            const int2 en = __ldg(p.bin_ent + e);
            const float* q = ms + en.x + (int64_t)t * en.y;
            if (p.n_channels == 2) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(q));
                al.x += v.x; al.y += v.y; ar.x += v.z; ar.y += v.w;
            } else {
                const float2 v = __ldg(reinterpret_cast<const float2*>(q));
                al.x += v.x; al.y += v.y;
            }
        }
        const float inv = __ldg(p.bin_inv + f);
        yl = cmul(zl, cscale(al, inv));
        yr = cmul(zr, cscale(ar, inv));
        if (p.zero_dc && f == 0) { yl = make_float2(0.f, 0.f); yr = yl; }
    } else if constexpr (ARCH == ARCH_HTDEMUCS) {
        // src/htdemucs.cpp:463-470 with the network output ox = Z * M; Nyquist dropped.
        if (f >= N / 2) { yl = make_float2(0.f, 0.f); yr = yl; return; }
        const int T = p.g.T, F = N / 2;
        const int64_t plane = (int64_t)F * T, idx = (int64_t)f * T + t;
        const float* ms = m + (int64_t)s * 2 * p.n_channels * plane;
        const float2 ml = make_float2(__ldg(ms + idx), __ldg(ms + plane + idx));
        yl = cmul(zl, ml);
        if (p.n_channels == 2) {
            const float2 mr = make_float2(__ldg(ms + 2 * plane + idx), __ldg(ms + 3 * plane + idx));
            yr = cmul(zr, mr);
        } else {
            yr = make_float2(0.f, 0.f);
        }
    } else {
        // src/tfc_tdf.cpp:370-387: CaC planes [4][dim_f][T], bins below zero_bins and at or
        // above dim_f zero, network output y = in * mask.
        if (f < p.zero_bins || f >= p.dim_f) { yl = make_float2(0.f, 0.f); yr = yl; return; }
        const int T = p.g.T;
        const int64_t plane = (int64_t)p.dim_f * T, idx = (int64_t)f * T + t;
        const float* ms = m + (int64_t)s * 4 * plane;
        yl = make_float2(zl.x * __ldg(ms + idx), zl.y * __ldg(ms + plane + idx));
        yr = make_float2(zr.x * __ldg(ms + 2 * plane + idx), zr.y * __ldg(ms + 3 * plane + idx));
    }
}

template <int ARCH, int N>
__global__ void __launch_bounds__(FftCfg<N>::T) fused_kernel(const FusedParams p) {
    constexpr int T = FftCfg<N>::T;
    using Plan = typename FftCfg<N>::Plan;
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float* ring = reinterpret_cast<float*>(buf + padded_size(N));   // [2][N]

    const int tid = threadIdx.x;
    const int tile = blockIdx.x, ci = blockIdx.y;
    const ChunkDesc cd = p.chunks[ci];
    const FrameGeom G = p.g;
    const int hop = G.hop;
    const int t_begin = tile * p.K;
    const int t_end = min(G.T, t_begin + p.K);
    const int C = p.n_channels;
    const float* chL = p.mix;
    const float* chR = p.mix + (C > 1 ? p.len : 0);
    const int lxf = G.ht_pad ? G.ht_lxf : G.Lc;
    const bool last_tile = t_end == G.T;

    for (int i = tid; i < 2 * N; i += T) ring[i] = 0.0f;

    for (int s = 0; s < p.S; s++) {
        float* Ys = p.Y + (int64_t)ci * p.y_chunk_stride + (int64_t)s * C * G.Lout;
        float* Trs = p.Tr + (int64_t)ci * p.tr_chunk_stride + ((int64_t)tile * p.S + s) * C * (N - hop);
        for (int t = t_begin; t < t_end; t++) {
            const int64_t q0 = (int64_t)G.first_pos + (int64_t)t * hop;
            // 1. frame load + window + stereo pack
            for (int n = tid; n < N; n += T) {
                int64_t r = reflect1(q0 + n - N / 2, lxf);
                if (G.ht_pad) r = reflect1(r - G.ht_pad, G.Lc);
                const float w = __ldg(p.win + n);
                const float a = chunk_sample(p, cd, chL, r);
                const float b = C > 1 ? chunk_sample(p, cd, chR, r) : 0.0f;
                buf[pad_idx(n)] = make_float2(a * w, b * w);
            }
            __syncthreads();
            fft<N, T, false>(buf, p.tw, tid, Plan{});
            // 3. split channels, spectral op, repack as one Hermitian pair
            for (int f = tid; f <= N / 2; f += T) {
                const int fm = f == 0 ? 0 : N - f;
                const float2 X = buf[pad_idx(f)], Xm = buf[pad_idx(fm)];
                const float2 zl = make_float2(0.5f * p.fwd_scale * (X.x + Xm.x), 0.5f * p.fwd_scale * (X.y - Xm.y));
                const float2 zr = make_float2(0.5f * p.fwd_scale * (X.y + Xm.y), -0.5f * p.fwd_scale * (X.x - Xm.x));
                float2 yl, yr;
                spectral_op<ARCH, N>(p, ci, s, t, f, zl, zr, yl, yr);
                if (f == 0 || f == N / 2) { yl.y = 0.0f; yr.y = 0.0f; }   // c2r ignores these
                buf[pad_idx(f)] = make_float2(yl.x - yr.y, yl.y + yr.x);
                if (f != 0 && f != N / 2) buf[pad_idx(fm)] = make_float2(yl.x + yr.y, yr.x - yl.y);
            }
            __syncthreads();
            fft<N, T, true>(buf, p.tw, tid, Plan{});
            // 4. window + overlap-add into the ring
            for (int n = tid; n < N; n += T) {
                const float2 v = buf[pad_idx(n)];
                const float w = __ldg(p.win + n) * p.inv_scale;
                const int slot = (int)((q0 + n) % N);
                ring[slot] += v.x * w;
                ring[N + slot] += v.y * w;
            }
            __syncthreads();
            // 5. flush what no later frame of this tile touches
            const bool last = t == t_end - 1;
            const int ny = (last && last_tile) ? N : hop;
            for (int u = tid; u < N; u += T) {
                if (u >= ny && !last) break;
                const int64_t q = q0 + u;
                const int slot = (int)(q % N);
                const float v0 = ring[slot], v1 = ring[N + slot];
                ring[slot] = 0.0f;
                ring[N + slot] = 0.0f;
                const int64_t j = q - G.out_offset;
                const float ie = (j >= 0 && j < G.Lout) ? __ldg(p.inv_env + j) : 0.0f;
                if (u < ny) {
                    if (j >= 0 && j < G.Lout) {
                        Ys[j] = v0 * ie;
                        if (C > 1) Ys[G.Lout + j] = v1 * ie;
                    }
                } else {
                    Trs[u - hop] = v0 * ie;
                    if (C > 1) Trs[(N - hop) + u - hop] = v1 * ie;
                }
            }
            __syncthreads();
        }
    }
}

// ---- combine ------------------------------------------------------------------------------
__device__ __forceinline__ float chunk_value(const CombineParams& p, int g, int k, int64_t j) {
    const FrameGeom& G = p.g;
    float v = __ldg(p.Y + (int64_t)g * p.y_chunk_stride + (int64_t)k * G.Lout + j);
    const int64_t q = j + G.out_offset - G.first_pos;
    const int64_t span = (int64_t)p.K * G.hop;
    const int64_t tau = q / span;
    const int64_t u = q - tau * span;
    if (tau >= 1 && tau < p.n_tiles && u < G.n_fft - G.hop) {
        const int s = k / p.C, c = k % p.C;
        v += __ldg(p.Tr + (int64_t)g * p.tr_chunk_stride +
                   (((tau - 1) * p.S + s) * p.C + c) * (int64_t)(G.n_fft - G.hop) + u);
    }
    return v;
}

__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.len) return;
    const int64_t P = i + p.out_shift;
    const ChunkDesc c0 = p.chunks[0];
    int64_t ghi = (P - c0.out0) / p.step_out;
    if (ghi > p.n_chunks - 1) ghi = p.n_chunks - 1;
    if (ghi < 0) ghi = 0;
    const int SC = p.S * p.C;
    constexpr int MAXK = 16;
    float acc[MAXK];
#pragma unroll
    for (int k = 0; k < MAXK; k++) acc[k] = 0.0f;
    float wsum = 0.0f;
    // chunks are ordered by out0; accumulate in ascending chunk order like the reference
    int64_t glo = (P - c0.out0 - p.max_out_len) / p.step_out;
    if (glo < 0) glo = 0;
    for (int g = (int)glo; g <= (int)ghi + 1 && g < p.n_chunks; g++) {
        const ChunkDesc d = p.chunks[g];
        const int64_t u = P - d.out0;
        if (u < 0 || u >= d.out_len) continue;
        const float w = __ldg(p.W + d.w_off + u);
        wsum += w;
#pragma unroll
        for (int k = 0; k < MAXK; k++)
            if (k < SC) acc[k] += w * chunk_value(p, g, k, d.y_off + u);
    }
    float outv[MAXK];
#pragma unroll
    for (int k = 0; k < MAXK; k++) {
        if (k < SC) {
            float v = acc[k] / wsum;
            if (p.nan_to_zero && !isfinite(v)) v = 0.0f;
            v *= p.compensate;
            outv[k] = v;
            p.out[(int64_t)k * p.len + i] = v;
        }
    }
    if (p.complement) {
        for (int c = 0; c < p.C; c++) {
            float v = __ldg(p.mix + (int64_t)c * p.len + i);
            if (p.complement == 1) {
                v -= outv[c];
            } else {
#pragma unroll
                for (int k = 0; k < MAXK; k++)
                    if (k < SC && k % p.C == c) v -= outv[k];
            }
            p.out[(int64_t)(SC + c) * p.len + i] = v;
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

size_t fused_smem_bytes(int n) {
    return sizeof(float2) * (size_t)padded_size(n) + sizeof(float) * 2 * (size_t)n;
}

template <int ARCH, int N>
static cudaError_t launch_fused_t(const FusedParams& p, cudaStream_t st) {
    const size_t smem = fused_smem_bytes(N);
    cudaError_t e = cudaFuncSetAttribute(fused_kernel<ARCH, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.n_tiles, p.n_chunks);
    fused_kernel<ARCH, N><<<grid, FftCfg<N>::T, smem, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_fused(int arch, const FusedParams& p, cudaStream_t st) {
    if (p.n_chunks <= 0 || p.n_tiles <= 0) return cudaSuccess;
    switch (arch) {
        case ARCH_ROFORMER:
            if (p.g.n_fft == 2048) return launch_fused_t<ARCH_ROFORMER, 2048>(p, st);
            if (p.g.n_fft == 4096) return launch_fused_t<ARCH_ROFORMER, 4096>(p, st);
            break;
        case ARCH_HTDEMUCS:
            if (p.g.n_fft == 4096) return launch_fused_t<ARCH_HTDEMUCS, 4096>(p, st);
            break;
        case ARCH_TFC:
            if (p.g.n_fft == 7680) return launch_fused_t<ARCH_TFC, 7680>(p, st);
            if (p.g.n_fft == 4096) return launch_fused_t<ARCH_TFC, 4096>(p, st);
            if (p.g.n_fft == 2048) return launch_fused_t<ARCH_TFC, 2048>(p, st);
            break;
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t st) {
    if (p.len <= 0) return cudaSuccess;
    if (p.S * p.C > 16) return cudaErrorInvalidValue;
    const int threads = 256;
    const int64_t blocks = (p.len + threads - 1) / threads;
    combine_kernel<<<(unsigned)blocks, threads, 0, st>>>(p);
    return cudaGetLastError();
}

} // namespace stg
