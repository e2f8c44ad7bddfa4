// norm.cu -- the normalisations HTDemucs wraps around its network, as deterministic
// reductions: every sum runs over a fixed launch shape and combines partial sums in a fixed
// order, so a result is the same bits on every run.
//
//   mono-mix normalisation (src/htdemucs.cpp:539-549, 638-642): mono = mean over channels
//     (rounded to float), mean and unbiased std over the track in double, std at least 1e-8;
//     the mix becomes (x - mean) / std and every stem v / 1 * std + mean.
//   CaC normalisation (src/htdemucs.cpp:434-436, 466-469): mean and unbiased std over all
//     2C x F x T spectrogram values of a segment; the network sees (v - mean) / (1e-5 + std)
//     and its output is mapped back by v * std + mean.
#include "kernels.h"

namespace stg {

namespace {

constexpr int kThreads = 256;
constexpr int kBlocks = 512;

__device__ __forceinline__ double block_sum(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
    __syncthreads();
    return s;   // valid in thread 0
}

__device__ __forceinline__ float mono_at(const float* mix, int64_t len, int C, int64_t i) {
    double s = 0.0;
    for (int c = 0; c < C; c++) s += mix[(int64_t)c * len + i];
    return (float)(s / C);
}

// pass 0: partial sums of mono; pass 1: partial sums of (mono - mean)^2 (mean from stats[0]).
__global__ void __launch_bounds__(kThreads) mono_partials(const float* __restrict__ mix, int64_t len, int C,
                                                          int pass, const double* __restrict__ stats,
                                                          double* __restrict__ partial) {
    __shared__ double red[kThreads / 32];
    const double mean = pass ? stats[0] : 0.0;
    double acc = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (int64_t)gridDim.x * blockDim.x) {
        const double m = mono_at(mix, len, C, i);
        acc += pass ? (m - mean) * (m - mean) : m;
    }
    const double s = block_sum(acc, red);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

// Sums the kBlocks partials by a fixed tree (one block of kBlocks threads): pass 0 writes the
// mean, pass 1 the std (at least 1e-8).
__global__ void __launch_bounds__(kBlocks) mono_finish(const double* __restrict__ partial, int64_t len, int pass,
                                                       double* stats) {
    __shared__ double s[kBlocks];
    s[threadIdx.x] = partial[threadIdx.x];
    __syncthreads();
    for (int o = kBlocks / 2; o > 0; o >>= 1) {
        if ((int)threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x != 0) return;
    if (pass == 0) stats[0] = s[0] / (double)len;
    else stats[1] = fmax(sqrt(s[0] / (double)(len - 1)), 1e-8);
}

__global__ void __launch_bounds__(kThreads) mono_apply(const float* __restrict__ mix, int64_t n,
                                                       const double* __restrict__ stats, float* __restrict__ out) {
    const double mean = stats[0], sd = stats[1];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (float)(((double)mix[i] - mean) / sd);
}

// One warp per segment: lane l adds tiles l, l + 32, ... in order, then the lanes' sums meet
// in a fixed shuffle tree.
__global__ void __launch_bounds__(128) cac_finish(const double2* __restrict__ partial, int n_chunks, int n_tiles,
                                                  double count, double2* __restrict__ stats) {
    const int ci = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (ci >= n_chunks) return;
    double s = 0.0, q = 0.0;
    for (int t = lane; t < n_tiles; t += 32) {
        const double2 v = partial[(int64_t)ci * n_tiles + t];
        s += v.x;
        q += v.y;
    }
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_down_sync(0xffffffffu, s, o);
        q += __shfl_down_sync(0xffffffffu, q, o);
    }
    if (lane != 0) return;
    const double mean = s / count;
    const double var = (q - s * mean) / (count - 1.0);
    stats[ci] = make_double2(mean, sqrt(fmax(var, 0.0)));
}

} // namespace

size_t mono_scratch_doubles() { return kBlocks + 2; }

cudaError_t launch_mono_norm(const float* mix, int64_t len, int C, double* scratch, float* out, cudaStream_t st) {
    double* partial = scratch + 2;
    double* stats = scratch;
    for (int pass = 0; pass < 2; pass++) {
        mono_partials<<<kBlocks, kThreads, 0, st>>>(mix, len, C, pass, stats, partial);
        mono_finish<<<1, kBlocks, 0, st>>>(partial, len, pass, stats);
    }
    mono_apply<<<kBlocks, kThreads, 0, st>>>(mix, (int64_t)C * len, stats, out);
    return cudaGetLastError();
}

cudaError_t launch_cac_finish(const double2* partial, int n_chunks, int n_tiles, double count, double2* stats,
                              cudaStream_t st) {
    cac_finish<<<(n_chunks + 3) / 4, 128, 0, st>>>(partial, n_chunks, n_tiles, count, stats);
    return cudaGetLastError();
}

} // namespace stg
