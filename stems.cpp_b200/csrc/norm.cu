// norm.cu -- the normalisations HTDemucs wraps around its network, as deterministic
// reductions: every sum runs over a fixed launch shape and combines partial sums in a fixed
// order, so a result is the same bits on every run.
//
//   mono-mix normalisation (src/htdemucs.cpp:539-549, 638-642): mono = mean over channels
//     (rounded to float), mean and unbiased std over the track in double, std at least 1e-8;
//     the mix becomes (x - mean) / std and every stem v / 1 * std + mean. One pass sums mono
//     and mono^2 in double; the variance is (sum sq - sum * mean) / (n - 1), which for audio
//     (|mono| <= 1, n < 2^29) agrees with the reference's second pass to about 1e-15.
//   CaC normalisation (src/htdemucs.cpp:434-436, 466-469): mean and unbiased std over all
//     2C x F x T spectrogram values of a segment; the network sees (v - mean) / (1e-5 + std)
//     and its output is mapped back by v * std + mean.
#include "kernels.h"

namespace stg {

namespace {

constexpr int kThreads = 256;
constexpr int kBlocks = 512;

__device__ __forceinline__ double2 block_sum2(double2 v, double2* red) {
    for (int o = 16; o > 0; o >>= 1) {
        v.x += __shfl_down_sync(0xffffffffu, v.x, o);
        v.y += __shfl_down_sync(0xffffffffu, v.y, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double2 s = make_double2(0.0, 0.0);
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) { s.x += red[w].x; s.y += red[w].y; }
    __syncthreads();
    return s;   // valid in thread 0
}

__device__ __forceinline__ float mono_at(const float* mix, int64_t len, int C, int64_t i) {
    double s = 0.0;
    for (int c = 0; c < C; c++) s += mix[(int64_t)c * len + i];
    return (float)(s / C);
}

// Per block: the partial sums of mono and of mono^2.
__global__ void __launch_bounds__(kThreads) mono_partials(const float* __restrict__ mix, int64_t len, int C,
                                                          double2* __restrict__ partial) {
    __shared__ double2 red[kThreads / 32];
    double2 acc = make_double2(0.0, 0.0);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (int64_t)gridDim.x * blockDim.x) {
        const double m = mono_at(mix, len, C, i);
        acc.x += m;
        acc.y = fma(m, m, acc.y);
    }
    const double2 s = block_sum2(acc, red);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

// Sums the kBlocks partials by a fixed tree (one block of kBlocks threads) and writes the mean
// and the std (at least 1e-8).
__global__ void __launch_bounds__(kBlocks) mono_finish(const double2* __restrict__ partial, int64_t len,
                                                       double* stats) {
    __shared__ double2 s[kBlocks];
    s[threadIdx.x] = partial[threadIdx.x];
    __syncthreads();
    for (int o = kBlocks / 2; o > 0; o >>= 1) {
        if ((int)threadIdx.x < o) {
            s[threadIdx.x].x += s[threadIdx.x + o].x;
            s[threadIdx.x].y += s[threadIdx.x + o].y;
        }
        __syncthreads();
    }
    if (threadIdx.x != 0) return;
    const double mean = s[0].x / (double)len;
    stats[0] = mean;
    stats[1] = fmax(sqrt(fmax(s[0].y - s[0].x * mean, 0.0) / (double)(len - 1)), 1e-8);
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

size_t mono_scratch_doubles() { return 2 * kBlocks + 2; }

cudaError_t launch_mono_norm(const float* mix, int64_t len, int C, double* scratch, float* out, cudaStream_t st) {
    double2* partial = reinterpret_cast<double2*>(scratch + 2);   // scratch is 16-byte aligned
    double* stats = scratch;
    mono_partials<<<kBlocks, kThreads, 0, st>>>(mix, len, C, partial);
    mono_finish<<<1, kBlocks, 0, st>>>(partial, len, stats);
    mono_apply<<<kBlocks, kThreads, 0, st>>>(mix, (int64_t)C * len, stats, out);
    return cudaGetLastError();
}

cudaError_t launch_cac_finish(const double2* partial, int n_chunks, int n_tiles, double count, double2* stats,
                              cudaStream_t st) {
    cac_finish<<<(n_chunks + 3) / 4, 128, 0, st>>>(partial, n_chunks, n_tiles, count, stats);
    return cudaGetLastError();
}

} // namespace stg
