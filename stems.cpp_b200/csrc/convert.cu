// convert.cu -- the request's audio into the model's format and the stems back out, on the
// device: the conversions src/libstems.cpp:160-199 runs around every separate() call.
//
//   layout    interleaved or planar input -> planar (libstems.cpp:162-167)
//   channels  to_channels: mono duplicated, extra channels dropped (src/audio.h:59-68)
//   rate      resample_planar: Kaiser-windowed sinc, 32 zero crossings, cutoff 0.95 of the
//             lower Nyquist, beta 8.6, a 2^15-entry kernel table interpolated linearly,
//             double accumulation (src/audio.h:17-56)
//   length    the stems resampled back and pinned to the input's length (libstems.cpp:190-199)
//
// One thread computes one output sample of up to ROWS rows (2, 4 or 8, the smallest that
// covers the rows, so that the stems' 8 rows share one weight computation): the tap weights
// are computed once per sample and shared by the rows, as the reference shares them across
// channels. The weight interpolation and the accumulation use explicitly rounded double
// operations (__dmul_rn, __dadd_rn) in the reference's order, so no multiply-add is fused and
// every output sample is the same float the reference computes.
#include <cmath>

#include "kernels.h"

namespace stg {

namespace {

constexpr int kTableN = 1 << 15;

template <int kRows>
__global__ void __launch_bounds__(256) resample_kernel(const ResampleParams p) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int row0 = blockIdx.y * kRows;
    if (i >= p.out_pin) return;
    double acc[kRows];
#pragma unroll
    for (int k = 0; k < kRows; k++) acc[k] = 0.0;
    int src[kRows];
#pragma unroll
    for (int k = 0; k < kRows; k++) {
        const int r = min(row0 + k, p.rows - 1);
        src[k] = p.to_channels ? (p.in_ch == 1 ? 0 : min(r, p.in_ch - 1)) : r;
    }
    const int64_t cs = p.interleaved ? 1 : p.in_n;    // channel stride of the input
    const int64_t ss = p.interleaved ? p.in_ch : 1;   // sample stride of the input
    if (i < p.out_n) {
        if (!p.table) {   // same rate: a copy
#pragma unroll
            for (int k = 0; k < kRows; k++) acc[k] = (double)p.in[src[k] * cs + i * ss];
        } else {
            const double c = (double)i / p.ratio;
            const int64_t lo = max((int64_t)0, (int64_t)ceil(c - p.half));
            const int64_t hi = min(p.in_n - 1, (int64_t)floor(c + p.half));
            for (int64_t j = lo; j <= hi; j++) {
                const double pos = fabs((double)j - c) / p.half * (double)kTableN;
                const int t = (int)pos;
                if (t >= kTableN) continue;
                const double fr = pos - t;
                const double2 ab = __ldg(p.table + t);
                const double a = ab.x, b = ab.y;
                const double w = __dadd_rn(a, __dmul_rn(__dadd_rn(b, -a), fr));
#pragma unroll
                for (int k = 0; k < kRows; k++)
                    acc[k] = __dadd_rn(acc[k], __dmul_rn(w, (double)__ldg(p.in + src[k] * cs + j * ss)));
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kRows; k++)
        if (row0 + k < p.rows) p.out[(int64_t)(row0 + k) * p.out_pin + i] = (float)acc[k];
}

double bessel_i0(double x) {   // the reference's 30-term series (src/audio.h:27-31)
    double s = 1, t = 1;
    for (int k = 1; k < 30; k++) {
        t *= (x / (2 * k)) * (x / (2 * k));
        s += t;
    }
    return s;
}

} // namespace

int64_t resampled_length(int64_t n, int src_rate, int dst_rate) {
    if (src_rate == dst_rate) return n;
    return std::llround(n * ((double)dst_rate / src_rate));              // audio.h:21
}

void kaiser_table(int src_rate, int dst_rate, std::vector<double>& table, double& half, double& ratio) {
    ratio = (double)dst_rate / src_rate;                                  // audio.h:20
    const double cutoff = 0.95 * std::min(1.0, ratio);
    const int zc = 32;
    half = zc / cutoff;
    const double beta = 8.6;
    const double i0b = bessel_i0(beta);
    table.assign(kTableN + 2, 0.0);
    for (int t = 0; t <= kTableN + 1; t++) {                             // audio.h:35-42
        const double x = std::min((double)t / kTableN, 1.0) * half;
        const double r = x / half;
        const double arg = M_PI * x * cutoff;
        const double sinc = arg < 1e-12 ? 1.0 : std::sin(arg) / arg;
        table[t] = r >= 1 ? 0.0 : sinc * bessel_i0(beta * std::sqrt(1 - r * r)) / i0b * cutoff;
    }
}

template <int kRows> cudaError_t launch_rows(const ResampleParams& p, cudaStream_t st) {
    if (p.rows > 65535 * kRows) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((p.out_pin + 255) / 256), (unsigned)((p.rows + kRows - 1) / kRows));
    resample_kernel<kRows><<<grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_resample(const ResampleParams& p, cudaStream_t st) {
    if (p.out_pin <= 0 || p.rows <= 0) return cudaSuccess;
    if (p.rows <= 2) return launch_rows<2>(p, st);
    if (p.rows <= 4) return launch_rows<4>(p, st);
    return launch_rows<8>(p, st);
}

} // namespace stg
