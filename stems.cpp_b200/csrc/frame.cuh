// frame.cuh -- what the spectral kernels share: the FFT configuration per n_fft, the padded
// frame loader, streaming loads and the ring-buffer index. Included by kernels.cu (fused
// separation) and split.cu (front and back halves around a network).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "fft.cuh"
#include "kernels.h"

namespace stg {

// Threads per CTA, radix plan, the CTAs per SM the register budget aims at, and the largest
// hop the input prefetch registers cover.
template <int N> struct FftCfg;
template <> struct FftCfg<2048> {
    static constexpr int T = 128, MINB = 3, HOPMAX = 512;
    static constexpr bool MASK_L2 = false;  // TFC-TDF: the next frame's mask row prefetched into L2
    static constexpr bool SMEM_WIN = false;   // the window copied into shared memory
    using Plan = RadixList<8, 16, 16>;
    // The RoFormer kernel's forward transform runs the radices in the opposite order, so its
    // last pass and the inverse's first are both radix 8 on the same butterflies (kernels.cu:
    // the mirror step); its twiddles follow Plan's in the table.
    using FwdPlan = RadixList<16, 16, 8>;
};
template <> struct FftCfg<4096> {
    static constexpr int T = 256, MINB = 2, HOPMAX = 1024;
    static constexpr bool MASK_L2 = false;
    static constexpr bool SMEM_WIN = false;
    using Plan = RadixList<16, 16, 16>;
};
// 7680: radix 15 last, because a first radix-15 pass stores at stride 15, which the padding
// of pad_idx cancels into 16-way bank conflicts; 256 threads let a thread keep its ~200 live
// values in registers (at 512 threads the 128-register cap spilled). One CTA per SM: its
// window goes in shared memory (30 KB, beside the 188 KB of frame and rings), and with only
// 8 warps per SM to hide the masks' DRAM latency, each frame's mask row is prefetched into L2
// a frame ahead (both measured: 1.59 -> 1.42 ms on a 180 s track).
template <> struct FftCfg<7680> {
    static constexpr int T = 256, MINB = 1, HOPMAX = 1024;
    static constexpr bool MASK_L2 = true;
    static constexpr bool SMEM_WIN = true;
    using Plan = RadixList<8, 8, 8, 15>;
};
// The VR bands' sizes (src/vr_dsp.h, 320 to 2048 points): front and back kernels only.
template <int N, int TT, class P> struct SmallFft {
    static constexpr int T = TT, MINB = 1, HOPMAX = N / 2;
    static constexpr bool MASK_L2 = false;
    static constexpr bool SMEM_WIN = false;
    using Plan = P;
};
template <> struct FftCfg<320> : SmallFft<320, 64, RadixList<8, 8, 5>> {};
template <> struct FftCfg<512> : SmallFft<512, 64, RadixList<8, 8, 8>> {};
template <> struct FftCfg<640> : SmallFft<640, 64, RadixList<8, 8, 10>> {};
template <> struct FftCfg<960> : SmallFft<960, 64, RadixList<8, 8, 15>> {};
template <> struct FftCfg<1024> : SmallFft<1024, 64, RadixList<8, 8, 16>> {};

// The largest hop of the front kernel's input prefetch: half the frame, which covers every
// STFT the reference runs (the fused kernel's own limit is FftCfg::HOPMAX).
template <int N> __host__ __device__ constexpr int split_hopmax() { return N / 2; }

__device__ __forceinline__ int reflect1(int j, int n) {
    if (j < 0) j = -j;
    if (j >= n) j = 2 * (n - 1) - j;
    return j;
}

// Loads for data read once per kernel (the masks): bypass L1 so the tables stay resident.
__device__ __forceinline__ float ld_stream(const float* p) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float4 ld_stream4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
// Bring [p, p + bytes) into L2 ahead of its loads (p 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ float2 ld_stream2(const float* p) {
    float2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
    return v;
}

// The track sample chunk-local sample pl reads, or -1 for a zero. 32-bit arithmetic: plans
// are limited to INT32_MAX / 4 samples.
template <class Params>
__device__ __forceinline__ int chunk_index(const Params& p, const ChunkDesc& cd, int pl) {
    if (pl >= cd.valid) {
        if (!cd.tail_reflect) return -1;
        pl = 2 * (cd.valid - 1) - pl;
    }
    int x = (int)cd.src0 + pl;
    if (cd.reflect) x = reflect1(x, (int)cd.vlen);
    else if ((unsigned)x >= (unsigned)cd.vlen) return -1;
    x += (int)cd.vshift;
    if ((unsigned)x >= (unsigned)p.len) return -1;
    return x;
}

// New input samples [q, q + hop) a frame needs beyond the previous one, per thread.
template <int T, int HOPMAX> struct InPrefetch {
    static constexpr int K = (HOPMAX + T - 1) / T;
    float2 v[K];
};

template <class Params>
__device__ __forceinline__ float2 frame_sample(const Params& p, const ChunkDesc& cd, const float* chL,
                                               const float* chR, int lxf, int q) {
    int r;
    if (p.g.zero_pad) {   // zeros around the signal instead of its mirror (src/vr_dsp.h:50-53)
        r = q - p.g.n_fft / 2;
        if (r < 0 || r >= p.g.Lc) return make_float2(0.0f, 0.0f);
    } else {
        r = reflect1(q - p.g.n_fft / 2, lxf);
        if (p.g.ht_pad) r = reflect1(r - p.g.ht_pad, p.g.Lc);
    }
    const int x = chunk_index(p, cd, r);   // one index for both channels
    if (x < 0) return make_float2(0.0f, 0.0f);
    return make_float2(ld_stream(chL + x), p.n_channels > 1 ? ld_stream(chR + x) : 0.0f);
}

// When no padding rule touches any sample frames [t_begin, t_end) of the chunk read, the tile
// reads one linear stretch of the track: sample x = q + offset for padded position q. Returns
// that offset, or INT_MIN when some sample needs the general rule (chunk and track edges).
constexpr int kNoLinear = -2147483647 - 1;
template <class Params>
__device__ __forceinline__ int linear_offset(const Params& p, const ChunkDesc& cd, int t_begin, int t_end) {
    const FrameGeom& G = p.g;
    const int qa = G.first_pos + t_begin * G.hop, qb = G.first_pos + (t_end - 1) * G.hop + G.n_fft;
    const int shift = G.n_fft / 2 + G.ht_pad;                       // chunk-local r = q - shift
    const int ra = qa - shift, rb = qb - shift;
    if (ra < 0 || rb > G.Lc || rb > cd.valid) return kNoLinear;
    if (G.ht_pad && qb - G.n_fft / 2 > G.ht_lxf) return kNoLinear;  // HTDemucs' first reflect
    const int xa = (int)cd.src0 + ra, xb = (int)cd.src0 + rb;
    if (xa < 0 || xb > (int)cd.vlen) return kNoLinear;
    if (xa + (int)cd.vshift < 0 || xb + (int)cd.vshift > (int)p.len) return kNoLinear;
    return (int)cd.src0 + (int)cd.vshift - shift;
}

// frame_sample through the tile's linear offset when it has one
template <class Params>
__device__ __forceinline__ float2 tile_sample(const Params& p, const ChunkDesc& cd, const float* chL,
                                              const float* chR, int lxf, int lin, int q) {
    if (lin == kNoLinear) return frame_sample(p, cd, chL, chR, lxf, q);
    const int x = lin + q;
    return make_float2(ld_stream(chL + x), p.n_channels > 1 ? ld_stream(chR + x) : 0.0f);
}

template <int N> __device__ __forceinline__ int ring_slot(int q) {
    if constexpr ((N & (N - 1)) == 0) return q & (N - 1);
    else return q % N;
}

} // namespace stg
