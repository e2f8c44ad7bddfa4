// pair.cu -- the fused spectral kernel of TFC-TDF at n_fft 7680 on CTA pairs (sm_100a clusters).
//
// One CTA of the single-CTA kernel (kernels.cu: fused_kernel<ARCH_TFC, 7680>) holds a whole
// 7680-point frame, its two rings and its window: 223 KB of shared memory, one CTA of 8 warps
// per SM. Here a cluster of two CTAs shares each frame, split by sample parity:
//   * CTA r owns the frame's samples n = 2m + r. Frames advance by an even hop, so a track
//     position keeps its owner from frame to frame: each CTA keeps the input ring, the output
//     ring and the window entries of its parity (3840 of each), all local.
//   * Forward: CTA r transforms its half, F^r = FFT_3840(z_{2m+r} w_{2m+r}); then
//     X_f = E_{f mod 3840} + W^f O_{f mod 3840} (E = F^0, O = F^1, W = e^{-2 pi i/7680}).
//   * Spectral op: bins a and 3840 - a need the same four values (E and O at a and 3840 - a),
//     and with their mirrors 7680 - a and 3840 + a they also give everything the inverse's
//     split needs at those two indices. One thread takes such a pair of bins: it reads E from
//     CTA 0's frame buffer and O from CTA 1's (one of them through distributed shared memory),
//     masks both bins' channels as the single-CTA kernel does, repacks, and writes
//       G^s_k = (Y_k + (-1)^s Y_{k+3840}) conj(W)^{s k}
//     to CTA s's buffer for its two indices k. The pairs are split between the two CTAs; every
//     buffer entry is read and then written by one thread, so the phase needs no barrier inside.
//   * Inverse: CTA s transforms G^s, whose output is x_{2m+s}, the frame's samples of its own
//     parity: window and overlap-add into the local output ring, flush as the single-CTA kernel.
// Two cluster barriers per frame: both halves' spectra complete before the pairs read them,
// and every G written before either inverse reads it. Shared memory per CTA is 113.5 KB, so two
// CTAs (16 warps) fit on an SM. The sums and the flush order are those of the single-CTA
// kernel; the FFT's own rounding differs (a 3840-point plan and one split stage).
#include <algorithm>
#include <vector>

#include <cooperative_groups.h>

#include "fft.cuh"
#include "frame.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace stg {

namespace {
constexpr int kN = 7680, kH = kN / 2, kT = 256, kHop = 1024;
// 3840 = 16 * 4 * 4 * 15, radix 15 last (see FftCfg<7680>). Measured on a 180 s track against
// 8*4*8*15, 16*8*2*15 and 16*15*16 (all without spills under the 128 registers that two CTAs
// of 256 threads per SM leave; 16*16*15 spilled): 1.342 ms against 1.381, 1.354 and 1.369.
using PairPlan = RadixList<16, 4, 4, 15>;
constexpr int kR1 = Head<PairPlan>::first;
using PairFwdRest = typename Head<PairPlan>::tail;
using PairInvInit = typename Init<PairPlan>::type;
constexpr int kRL = Init<PairPlan>::last, kNSL = Init<PairPlan>::prod;
constexpr int kA1 = (kH / 2 + 2) / 2;           // pairs a in [0, kA1) on CTA 0, [kA1, kH/2] on CTA 1
constexpr int kPR = (kA1 + kT - 1) / kT;        // pair rounds per thread (CTA 0's share, the larger)
static_assert(kA1 >= kH / 2 + 1 - kA1, "CTA 0 takes the larger share of the pairs");

size_t pair_smem_bytes() {
    return sizeof(float2) * ((size_t)padded_size(kH) + 2 * (size_t)kH) + sizeof(float) * ((size_t)kH + kHop);
}

// Distributed shared memory through 32-bit shared::cluster addresses: the address of this
// CTA's shared variable p in CTA `rank` of the cluster, and loads and stores there.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ float2 ld_cluster(uint32_t a) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster(uint32_t a, float2 v) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v.x), "f"(v.y) : "memory");
}

// The cluster barrier in two halves, so that loads can be issued between them (after the
// release, which would wait for them).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Ring slot of this parity's sample i of a frame whose first sample of the parity sits at slot
// h0: positions q0 + 2i + rank map to ((q0 + rank) mod N) / 2 + i, modulo N / 2.
__device__ __forceinline__ int hslot(int h0, int i) {
    const int s = h0 + i;
    return s >= kH ? s - kH : s;
}

// Split bin f's two channels from X_f, X_{N-f}, mask them (CaC planes; zero outside
// [zero_bins, dim_f), as the loads leave m), and return the repacked Y_f and Y_{N-f}.
__device__ __forceinline__ void tfc_bin(float2 X, float2 Xm, float4 m, bool edge, float half_fwd, float2& y, float2& ym) {
    const float2 zl = make_float2(half_fwd * (X.x + Xm.x), half_fwd * (X.y - Xm.y));
    const float2 zr = make_float2(half_fwd * (X.y + Xm.y), -half_fwd * (X.x - Xm.x));
    float2 yl = make_float2(zl.x * m.x, zl.y * m.y);
    float2 yr = make_float2(zr.x * m.z, zr.y * m.w);
    if (edge) { yl.y = 0.0f; yr.y = 0.0f; }   // bins 0 and N/2: c2r ignores these
    y = make_float2(yl.x - yr.y, yl.y + yr.x);
    ym = make_float2(yl.x + yr.y, yr.x - yl.y);
}
} // namespace

__global__ void __launch_bounds__(kT, 2) fused_pair_kernel(const FusedParams p) {
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);   // padded half frame
    float2* in_ring = buf + padded_size(kH);               // (L, R) of this parity, by (position mod N) / 2
    float2* out_ring = in_ring + kH;
    float* win_s = reinterpret_cast<float*>(out_ring + kH);   // w[2m + rank]
    float* env_s = win_s + kH;                               // envelope period
    // the two frame buffers in the cluster's window: CTA 0's holds E, then G^0; CTA 1's O, then G^1
    const uint32_t buf0 = cluster_addr(buf, 0), buf1 = cluster_addr(buf, 1);
    const TwGlobal tw{p.tw + kN};         // the 3840-point plan's twiddles
    const float2* __restrict__ tws = p.tw + kN + kH;   // W_N^k, k < 3840

    const int tid = threadIdx.x;
    const FrameGeom& G = p.g;
    const int hop = G.hop;
    const float* chL = p.mix;
    const float* chR = p.mix + p.len;
    const int lxf = G.ht_pad ? G.ht_lxf : G.Lc;
    const float half_fwd = 0.5f * p.fwd_scale;
    const int F = p.dim_f, f_lo = p.zero_bins;

    for (int i = tid; i < kH; i += kT) {
        out_ring[i] = make_float2(0.f, 0.f);
        win_s[i] = __ldg(p.win + 2 * i + rank);
    }
    const bool env_on = p.env_period != nullptr;
    if (env_on)
        for (int i = tid; i < hop; i += kT) env_s[i] = __ldg(p.env_period + i);
    constexpr int KX = (kHop / 2 + kT - 1) / kT;   // new samples of this parity per thread and frame
    float2 nx[KX];
    // the peer's shared memory is live from here on
    cl.sync();

    const int n_items = p.n_tiles * p.n_chunks;
    const int n_clusters = (int)(gridDim.x / 2);
    for (int item = (int)(blockIdx.x / 2); item < n_items; item += n_clusters) {
    const int tile = item % p.n_tiles, ci = item / p.n_tiles;
    const ChunkDesc cd = p.chunks[ci];
    const int t_begin = tile * p.K;
    const int t_end = min(G.T, t_begin + p.K);
    const bool last_tile = t_end == G.T;
    const int lin = linear_offset(p, cd, t_begin, t_end);

    for (int s = 0; s < p.S; s++) {
        float* Ys = p.Y + (int64_t)ci * p.y_chunk_stride + (int64_t)s * 2 * G.Lout;
        float* Trs = p.Tr + (int64_t)ci * p.tr_chunk_stride + ((int64_t)tile * p.S + s) * 2 * (kN - hop);
        {   // the first frame's samples of this parity, and the next frame's new ones
            const int q0 = G.first_pos + t_begin * hop;
            const int h0 = ring_slot<kN>(q0 + rank) >> 1;
            for (int i = tid; i < kH; i += kT)
                in_ring[hslot(h0, i)] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + 2 * i + rank);
#pragma unroll
            for (int k = 0; k < KX; k++) {
                const int u = 2 * (tid + k * kT) + rank;
                if (u < hop && t_begin + 1 < t_end) nx[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + kN + u);
            }
        }
        __syncthreads();
        const float* mrow0 = p.mask + (int64_t)ci * p.mask_chunk_stride + (int64_t)s * G.T * F * 4;
        for (int t = t_begin; t < t_end; t++) {
            const int q0 = G.first_pos + t * hop;
            const int h0 = ring_slot<kN>(q0 + rank) >> 1;
            // forward pass 1 over this parity's windowed samples, straight from the ring
            pass_io<kH, kR1, 1, kT, false, false>(
                tw, tid,
                [&](int j, int r) {
                    const int m = j + r * (kH / kR1);
                    const float2 x = in_ring[hslot(h0, m)];
                    const float w = win_s[m];
                    return make_float2(x.x * w, x.y * w);
                },
                [&](int base, int r, float2 v) { buf[pad_store<kR1, 1>(base, r)] = v; });
            __syncthreads();
            if (t + 1 < t_end) {
#pragma unroll
                for (int k = 0; k < KX; k++) {
                    const int i = tid + k * kT;
                    if (2 * i + rank < hop) in_ring[hslot(h0, i)] = nx[k];   // position q0 + N + 2i + rank
                }
            }
            // this frame's mask row (t-major, mask_transpose), the bins of this CTA's pairs, into
            // L2 while the transforms run: CTA 0 a in [0, kA1) and 3840 - a in (2880, 3840], CTA 1
            // the bins between
            const float* mrow = mrow0 + (int64_t)t * F * 4;
            if (tid == 0) {
                const int lo0 = rank ? kA1 : 0, hi0 = rank ? kH - kA1 + 1 : kA1;
                if (min(hi0, F) > lo0) prefetch_l2(mrow + 4 * lo0, 16u * (unsigned)(min(hi0, F) - lo0));
                if (rank == 0 && F > kH - kA1 + 1) prefetch_l2(mrow + 4 * (kH - kA1 + 1), 16u * (unsigned)(min(kH + 1, F) - (kH - kA1 + 1)));
            }
            passes<kH, kT, false, kR1>(buf, tw, tid, PairFwdRest{});
            // both halves' spectra complete
            cluster_arrive();
            cluster_wait();
            // the thread's bin pairs, two at a time (each with its two mask entries, from L2)
#pragma unroll 2
            for (int i = 0; i < kPR; i++) {
                const int a = (rank ? kA1 : 0) + tid + i * kT;
                if (a < (rank ? kH / 2 + 1 : kA1)) {
                    const int b = kH - a, bi = a == 0 ? 0 : b;
                    const float4 mai = a >= f_lo && a < F ? ld_stream4(mrow + 4 * a) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float4 mbi = b >= f_lo && b < F ? ld_stream4(mrow + 4 * b) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const uint32_t oa = 8u * (uint32_t)pad_idx(a), ob = 8u * (uint32_t)pad_idx(bi);
                    const float2 Ea = ld_cluster(buf0 + oa), Oa = ld_cluster(buf1 + oa);
                    const float2 Eb = ld_cluster(buf0 + ob), Ob = ld_cluster(buf1 + ob);
                    const float2 Wa = __ldg(tws + a);
                    const float2 Wb = a == 0 ? make_float2(-1.0f, 0.0f) : __ldg(tws + b);
                    const float2 ta = cmul(Wa, Oa), tb = cmul(Wb, Ob);
                    const float2 Xa = cadd(Ea, ta), XaH = csub(Ea, ta);   // X_a, X_{a+H}
                    const float2 Xb = cadd(Eb, tb), XbH = csub(Eb, tb);   // X_b, X_{b+H} = X_{N-a}
                    float2 Ya, YNa, Yb, YNb;
                    tfc_bin(Xa, XbH, mai, a == 0, half_fwd, Ya, YNa);       // bin a and its mirror N - a
                    if (a == 0) {
                        // bins 0 and N/2 = H: X_0 = E_0 + O_0, X_H = E_0 - O_0, each its own mirror
                        tfc_bin(Xb, Xb, mbi, true, half_fwd, Yb, YNb);
                        st_cluster(buf0 + oa, cadd(Ya, Yb));
                        st_cluster(buf1 + oa, csub(Ya, Yb));
                    } else if (a == b) {
                        // a = H/2: its mirror N - a is a + H
                        st_cluster(buf0 + oa, cadd(Ya, YNa));
                        st_cluster(buf1 + oa, cmul(csub(Ya, YNa), cconj(Wa)));
                    } else {
                        tfc_bin(Xb, XaH, mbi, false, half_fwd, Yb, YNb);    // bin b and N - b = a + H
                        st_cluster(buf0 + oa, cadd(Ya, YNb));
                        st_cluster(buf1 + oa, cmul(csub(Ya, YNb), cconj(Wa)));
                        st_cluster(buf0 + ob, cadd(Yb, YNa));
                        st_cluster(buf1 + ob, cmul(csub(Yb, YNa), cconj(Wb)));
                    }
                }
            }
            // every G in place before either inverse reads it; the new samples of frame t + 2 are
            // requested between the barrier's halves (the release would wait for them) and stay in
            // flight through the inverse transform
            cluster_arrive();
            if (t + 2 < t_end) {
#pragma unroll
                for (int k = 0; k < KX; k++) {
                    const int u = 2 * (tid + k * kT) + rank;
                    if (u < hop) nx[k] = tile_sample(p, cd, chL, chR, lxf, lin, q0 + hop + kN + u);
                }
            }
            cluster_wait();
            passes<kH, kT, true, 1>(buf, tw, tid, PairInvInit{});
            // inverse last pass: x_{2m + rank}, windowed, into the local output ring
            pass_io<kH, kRL, kNSL, kT, true, false>(
                tw, tid, [&](int j, int r) { return buf[pad_load<kH, kRL>(j, r)]; },
                [&](int base, int r, float2 v) {
                    const int m = base + r * kNSL;
                    const float w = win_s[m] * p.inv_scale;
                    float2& o = out_ring[hslot(h0, m)];
                    o = make_float2(fmaf(v.x, w, o.x), fmaf(v.y, w, o.y));
                });
            __syncthreads();
            // flush this parity's samples that no later frame of the tile touches
            const bool last = t == t_end - 1;
            const int ny = (last && last_tile) ? kN : hop;
            const int nflush = last ? kN : hop;
            int r = 0;
            if (env_on) {
                r = (q0 - G.out_offset + 2 * tid + rank - p.env_lo) % hop;
                if (r < 0) r += hop;
            }
            for (int i = tid; 2 * i + rank < nflush; i += kT) {
                const int u = 2 * i + rank, q = q0 + u;
                float2& o = out_ring[hslot(h0, i)];
                const float2 v = o;
                o = make_float2(0.f, 0.f);
                const int j = q - G.out_offset;
                const bool in = j >= 0 && j < G.Lout;
                float ie = 0.0f;
                if (in) ie = env_on && j >= p.env_lo && j < p.env_hi ? env_s[r] : ld_stream(p.inv_env + j);
                if (env_on) {
                    r += 2 * kT;
                    while (r >= hop) r -= hop;
                }
                if (u < ny) {
                    if (in) reinterpret_cast<float2*>(Ys)[j] = make_float2(v.x * ie, v.y * ie);
                } else {
                    reinterpret_cast<float2*>(Trs)[u - hop] = make_float2(v.x * ie, v.y * ie);
                }
            }
            // the next frame's barrier after forward pass 1 orders these ring writes before any
            // later read of the same slots
        }
        __syncthreads();
    }
    }
    // neither CTA leaves while the other may still write its frame buffer
    cl.sync();
}

bool fused_pair(int arch, int n_fft, int hop) {
    return arch == ARCH_TFC && n_fft == kN && hop > 0 && hop <= kHop && hop % 2 == 0;
}

template <int... Rs> static std::vector<int> radices_of(RadixList<Rs...>) { return {Rs...}; }

std::vector<int> fused_pair_radices(int n_fft) {
    if (n_fft != kN) return {};
    return radices_of(PairPlan{});
}

static cudaLaunchConfig_t pair_config(int grid, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(kT, 1, 1);
    cfg.dynamicSmemBytes = pair_smem_bytes();
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

static cudaError_t pair_prepare() {
    return cudaFuncSetAttribute(fused_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pair_smem_bytes());
}

// Clusters of the pair kernel resident at once on the current device (0 when unknown).
int fused_pair_slots() {
    if (pair_prepare() != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pair_config(2, nullptr, attr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fused_pair_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_fused_pair(const FusedParams& p, cudaStream_t st) {
    if (p.n_chunks <= 0 || p.n_tiles <= 0) return cudaSuccess;
    if (p.n_channels != 2 || !fused_pair(ARCH_TFC, p.g.n_fft, p.g.hop)) return cudaErrorInvalidValue;
    cudaError_t e = pair_prepare();
    if (e != cudaSuccess) return e;
    static int slots = 0;
    if (!slots) {
        slots = fused_pair_slots();
        if (slots < 1) return cudaErrorInvalidConfiguration;
    }
    const int64_t items = (int64_t)p.n_tiles * p.n_chunks;
    const int clusters = (int)std::min<int64_t>(items, slots);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pair_config(2 * clusters, st, attr);
    return cudaLaunchKernelEx(&cfg, fused_pair_kernel, p);
}

} // namespace stg
