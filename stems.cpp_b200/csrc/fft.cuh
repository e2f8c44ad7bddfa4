// fft.cuh -- shared-memory mixed-radix Stockham FFT for sm_100a.
//
// One thread group (a whole CTA here) transforms one complex frame of N points held in
// shared memory. Each pass of radix R gives every thread N/R/T butterflies: it loads R
// points with stride N/R (unit stride across threads, so conflict-free), applies the
// inter-pass twiddles, runs a fully unrolled radix-R codelet in registers and stores the
// outputs with stride Ns (the Stockham autosort, so no bit reversal). Passes are in place:
// every thread loads all its points, the group synchronises, then every thread stores.
//
// Shared memory is indexed through PAD(i) = i + i/16 (one spare complex per 16), which
// makes the radix-16 scatter of the first pass conflict-free for 64-bit accesses.
//
// Twiddles: the codelets' internal twiddles W_R^m are compile-time constants derived from
// the DFT definition (constexpr Taylor series in double, rounded once to float); the
// inter-pass twiddles come from per-pass tables computed on the host in double precision
// (twiddle_index). No device trigonometry is used anywhere.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace stg {

// ---- complex helpers ----------------------------------------------------------------------
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
// multiply by -i (forward) or +i (inverse)
template <bool INV> __device__ __forceinline__ float2 mul_mi(float2 a) {
    return INV ? make_float2(-a.y, a.x) : make_float2(a.y, -a.x);
}

// A complex value whose additions and subtractions run as one sm_100 f32x2 instruction
// (add/sub.rn.f32x2: the real and imaginary parts in the two halves of a register pair, each
// rounded as the scalar operation rounds it), which halves the issue slots the codelets spend
// on them. Everything else (twiddle products, multiplications by -i) is the float2 code.
struct PF2 : float2 {
    PF2() = default;
    __device__ __forceinline__ PF2(float2 v) : float2(v) {}
};
__device__ __forceinline__ PF2 cadd(PF2 a, PF2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ PF2 csub(PF2 a, PF2 b) {
    float2 r;
    asm("{.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\t"
        "mov.b64 pb, {%4, %5};\n\t"
        "sub.rn.f32x2 pd, pa, pb;\n\t"
        "mov.b64 {%0, %1}, pd;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
template <bool INV> __device__ __forceinline__ PF2 mul_mi(PF2 a) { return mul_mi<INV>(static_cast<float2>(a)); }

__host__ __device__ constexpr int pad_idx(int i) { return i + (i >> 4); }
__host__ __device__ constexpr int padded_size(int n) { return n + (n >> 4) + 1; }

// ---- compile-time trigonometry (Taylor series on a reduced argument) ----------------------
namespace ct {
constexpr double kPi = 3.14159265358979323846264338327950288;
__host__ __device__ constexpr double sin_poly(double x) {   // |x| <= pi/4
    double term = x, sum = x;
    for (int k = 1; k < 14; k++) { term *= -x * x / ((2.0 * k) * (2.0 * k + 1.0)); sum += term; }
    return sum;
}
__host__ __device__ constexpr double cos_poly(double x) {
    double term = 1.0, sum = 1.0;
    for (int k = 1; k < 14; k++) { term *= -x * x / ((2.0 * k - 1.0) * (2.0 * k)); sum += term; }
    return sum;
}
// cos and sin of 2*pi*m/n, exact symmetry handling by octant.
__host__ __device__ constexpr double cos2pi(long m, long n) {
    m %= n; if (m < 0) m += n;
    // angle = 2 pi m / n in [0, 2pi); reduce with 8 * m / n
    const long e = 8 * m;               // octant numerator
    const long oct = e / n;             // 0..7
    const double r = 2.0 * kPi * (double)(e - oct * n) / (8.0 * (double)n);   // [0, pi/4)
    switch (oct) {
        case 0: return cos_poly(r);
        case 1: return sin_poly(kPi / 4 - r);
        case 2: return -sin_poly(r);
        case 3: return -cos_poly(kPi / 4 - r);
        case 4: return -cos_poly(r);
        case 5: return -sin_poly(kPi / 4 - r);
        case 6: return sin_poly(r);
        default: return cos_poly(kPi / 4 - r);
    }
}
__host__ __device__ constexpr double sin2pi(long m, long n) { return cos2pi(m * 4 - n, 4 * n); }   // sin x = cos(x - pi/2)
} // namespace ct

// Multiply v by W_n^m = exp(-+ 2 pi i m / n) (sign by INV), with the trivial angles exact.
template <long M, long Nn, bool INV>
__device__ __forceinline__ float2 twc(float2 v) {
    constexpr long m = ((M % Nn) + Nn) % Nn;
    if constexpr (m == 0) {
        return v;
    } else if constexpr ((4 * m) % Nn == 0) {
        constexpr long q = (4 * m) / Nn;   // quarter turns (clockwise for forward)
        if constexpr (q == 2) return make_float2(-v.x, -v.y);
        else if constexpr (q == 1) return mul_mi<INV>(v);
        else return mul_mi<!INV>(v);
    } else if constexpr ((8 * m) % Nn == 0) {
        constexpr float h = 0.70710678118654752440f;
        constexpr long o = (8 * m) / Nn;   // odd octant 1,3,5,7
        // forward: W = cos(o pi/4) - i sin(o pi/4)
        constexpr float c = (o == 1 || o == 7) ? h : -h;
        constexpr float s0 = (o == 1 || o == 3) ? h : -h;
        constexpr float s = INV ? -s0 : s0;   // W = c - i s
        return make_float2(c * v.x + s * v.y, c * v.y - s * v.x);
    } else {
        constexpr float c = (float)ct::cos2pi(m, Nn);
        constexpr float s0 = (float)ct::sin2pi(m, Nn);
        constexpr float s = INV ? -s0 : s0;   // W = c - i s
        return make_float2(fmaf(c, v.x, s * v.y), fmaf(c, v.y, -s * v.x));
    }
}
template <long M, long Nn, bool INV>
__device__ __forceinline__ PF2 twc(PF2 v) { return twc<M, Nn, INV>(static_cast<float2>(v)); }

// ---- radix-R codelets, in place on a register array ------------------------------------
template <int R, bool INV> struct Dft;

template <bool INV> struct Dft<2, INV> {
    template <int S, class V> __device__ __forceinline__ static void run(V* a) {
        const V t = a[0];
        a[0] = cadd(t, a[S]);
        a[S] = csub(t, a[S]);
    }
};

template <bool INV> struct Dft<3, INV> {
    template <int S> __device__ __forceinline__ static void run(float2* a) {
        constexpr float s3 = 0.86602540378443864676f;   // sin(2 pi / 3)
        const float2 t = cadd(a[S], a[2 * S]);
        const float2 u = csub(a[S], a[2 * S]);
        const float2 m = make_float2(a[0].x - 0.5f * t.x, a[0].y - 0.5f * t.y);
        a[0] = cadd(a[0], t);
        const float2 ju = mul_mi<INV>(cscale(u, s3));   // -i s u (forward)
        a[S] = cadd(m, ju);
        a[2 * S] = csub(m, ju);
    }
};

template <bool INV> struct Dft<4, INV> {
    template <int S, class V> __device__ __forceinline__ static void run(V* a) {
        const V t0 = cadd(a[0], a[2 * S]), t1 = csub(a[0], a[2 * S]);
        const V t2 = cadd(a[S], a[3 * S]), t3 = mul_mi<INV>(csub(a[S], a[3 * S]));
        a[0] = cadd(t0, t2);
        a[2 * S] = csub(t0, t2);
        a[S] = cadd(t1, t3);
        a[3 * S] = csub(t1, t3);
    }
};

template <bool INV> struct Dft<5, INV> {
    template <int S> __device__ __forceinline__ static void run(float2* a) {
        constexpr float c1 = 0.30901699437494742410f, c2 = -0.80901699437494742410f;   // cos 2pi/5, 4pi/5
        constexpr float s1 = 0.95105651629515357212f, s2 = 0.58778525229247312917f;    // sin 2pi/5, 4pi/5
        const float2 t1 = cadd(a[S], a[4 * S]), t2 = cadd(a[2 * S], a[3 * S]);
        const float2 t3 = csub(a[S], a[4 * S]), t4 = csub(a[2 * S], a[3 * S]);
        const float2 x0 = a[0];
        a[0] = cadd(x0, cadd(t1, t2));
        const float2 b1 = make_float2(fmaf(c2, t2.x, fmaf(c1, t1.x, x0.x)), fmaf(c2, t2.y, fmaf(c1, t1.y, x0.y)));
        const float2 b2 = make_float2(fmaf(c1, t2.x, fmaf(c2, t1.x, x0.x)), fmaf(c1, t2.y, fmaf(c2, t1.y, x0.y)));
        const float2 d1 = mul_mi<INV>(make_float2(fmaf(s1, t3.x, s2 * t4.x), fmaf(s1, t3.y, s2 * t4.y)));
        const float2 d2 = mul_mi<INV>(make_float2(fmaf(s2, t3.x, -s1 * t4.x), fmaf(s2, t3.y, -s1 * t4.y)));
        a[S] = cadd(b1, d1);
        a[4 * S] = csub(b1, d1);
        a[2 * S] = cadd(b2, d2);
        a[3 * S] = csub(b2, d2);
    }
};

// Composite radix R = R1 * R2 (Cooley-Tukey in registers). Input a[n*S], n = R2*n1 + n2;
// output X[k*S] with k = k1 + R1*k2 (natural order).
template <int R1, int R2, bool INV> struct DftCT {
    static constexpr int R = R1 * R2;
    template <int S, class V> __device__ __forceinline__ static void run(V* a) {
        // inner DFTs of length R1 over n1 (stride R2) for each n2
        inner<S, 0>(a);
        // twiddles W_R^{n2 k1}: element (n2, k1) sits at index R2*k1 + n2
        twiddle<S, 0>(a);
        // outer DFTs of length R2 over n2 (stride 1) for each k1: results land at
        // R2*k1 + k2, but natural order wants k1 + R1*k2 -> transpose the R1 x R2 block.
        outer<S, 0>(a);
        V tmp[R];
#pragma unroll
        for (int k1 = 0; k1 < R1; k1++)
#pragma unroll
            for (int k2 = 0; k2 < R2; k2++) tmp[k1 + R1 * k2] = a[(R2 * k1 + k2) * S];
#pragma unroll
        for (int k = 0; k < R; k++) a[k * S] = tmp[k];
    }
    template <int S, int N2, class V> __device__ __forceinline__ static void inner(V* a) {
        if constexpr (N2 < R2) {
            Dft<R1, INV>::template run<S * R2>(a + N2 * S);
            inner<S, N2 + 1>(a);
        }
    }
    template <int S, int I, class V> __device__ __forceinline__ static void twiddle(V* a) {
        if constexpr (I < R) {
            constexpr int k1 = I / R2, n2 = I % R2;
            a[I * S] = twc<(long)n2 * k1, R, INV>(a[I * S]);
            twiddle<S, I + 1>(a);
        }
    }
    template <int S, int K1, class V> __device__ __forceinline__ static void outer(V* a) {
        if constexpr (K1 < R1) {
            Dft<R2, INV>::template run<S>(a + K1 * R2 * S);
            outer<S, K1 + 1>(a);
        }
    }
};

template <bool INV> struct Dft<8, INV> : DftCT<2, 4, INV> {};
template <bool INV> struct Dft<16, INV> : DftCT<4, 4, INV> {};
template <bool INV> struct Dft<15, INV> : DftCT<3, 5, INV> {};
template <bool INV> struct Dft<6, INV> : DftCT<2, 3, INV> {};
template <bool INV> struct Dft<10, INV> : DftCT<2, 5, INV> {};
template <bool INV> struct Dft<32, INV> : DftCT<2, 16, INV> {};

// ---- one Stockham pass and a whole transform ---------------------------------------------
// Twiddle table of a radix plan: the pass at stride NS (radix R) multiplies point r of its
// butterfly k (k = j mod NS) by W_{NS*R}^{k*r}. Its (R-1)*NS values sit at
// (NS - 1) + (r - 1)*NS + k, so the passes' tables tile [0, N - 1) (the sizes (R-1)*NS
// telescope) and the lanes of a warp, which hold consecutive k, read consecutive entries.
template <int NS> __host__ __device__ constexpr int twiddle_index(int r, int k) { return (NS - 1) + (r - 1) * NS + k; }

// The twiddle table in global memory, read through L1.
struct TwGlobal {
    const float2* __restrict__ p;
    __device__ __forceinline__ float2 operator()(int i) const { return __ldg(p + i); }
};

// One pass with caller-supplied input and output. Butterfly j reads the points
// j + r*NB (NB = N/R) through ld(j, r) and writes the points base + r*NS through
// st(base, r, v); r is a compile-time constant after unrolling, so callers fold it into
// immediate offsets. MID_SYNC puts a barrier between the loads and the stores, which an
// in-place pass needs; a pass that reads one buffer and writes another does not.
// TW_EARLY: load the pass's twiddles with the points, ahead of the barrier (a kernel that has
// the registers for them).
// V: the codelets' complex type (float2, or PF2 for packed additions).
template <int N, int R, int NS, int T, bool INV, bool MID_SYNC, bool TW_EARLY = false, class V = float2, class Tw,
          class Ld, class St>
__device__ __forceinline__ void pass_io(const Tw& tw, int tid, Ld&& ld, St&& st) {
    constexpr int NB = N / R;
    constexpr int ROUNDS = (NB + T - 1) / T;
    constexpr bool EXACT = (NB % T) == 0;
    V v[ROUNDS][R];
    constexpr bool HOIST = TW_EARLY && NS > 1 && ROUNDS * (R - 1) <= 16;
    float2 wv[HOIST ? ROUNDS : 1][HOIST ? R : 1];
#pragma unroll
    for (int rd = 0; rd < ROUNDS; rd++) {
        const int j = tid + rd * T;
        if (EXACT || j < NB) {
            if constexpr (HOIST) {
#pragma unroll
                for (int r = 1; r < R; r++) wv[rd][r] = tw(twiddle_index<NS>(r, j % NS));
            }
#pragma unroll
            for (int r = 0; r < R; r++) v[rd][r] = ld(j, r);
        }
    }
    if constexpr (MID_SYNC) __syncthreads();
#pragma unroll
    for (int rd = 0; rd < ROUNDS; rd++) {
        const int j = tid + rd * T;
        if (EXACT || j < NB) {
            const int k = j % NS;
            if constexpr (NS > 1) {
#pragma unroll
                for (int r = 1; r < R; r++) {
                    float2 w;
                    if constexpr (HOIST) w = wv[rd][r];
                    else w = tw(twiddle_index<NS>(r, k));
                    if (INV) w.y = -w.y;
                    v[rd][r] = cmul(v[rd][r], w);
                }
            }
            Dft<R, INV>::template run<1>(v[rd]);
            const int base = (j / NS) * NS * R + k;
#pragma unroll
            for (int r = 0; r < R; r++) st(base, r, v[rd][r]);
        }
    }
}

// Padded addresses of a pass's points. pad_idx(x + c) = pad_idx(x) + c + c/16 whenever c is
// a multiple of 16, and pad_idx(x + r) = pad_idx(x) + r whenever x mod 16 + r < 16.
template <int N, int R> __device__ __forceinline__ int pad_load(int j, int r) {
    constexpr int NB = N / R;
    if constexpr (NB % 16 == 0) return pad_idx(j) + r * (NB + NB / 16);
    else return pad_idx(j + r * NB);
}
template <int R, int NS> __device__ __forceinline__ int pad_store(int base, int r) {
    if constexpr (NS % 16 == 0) return pad_idx(base) + r * (NS + NS / 16);
    else if constexpr (NS == 1 && 16 % R == 0) return pad_idx(base) + r;   // base = j*R
    // NS divides 16 and NS*R is a multiple of 16: base mod 16 = k < NS and (r*NS) mod 16 is a
    // multiple of NS below 16, so the pair never crosses a 16-boundary beyond r*NS's own
    else if constexpr (16 % NS == 0 && (NS * R) % 16 == 0) return pad_idx(base) + r * NS + (r * NS) / 16;
    else return pad_idx(base + r * NS);
}

// In-place pass on the padded shared-memory frame buf, ending with a barrier.
template <int N, int R, int NS, int T, bool INV, bool TW_EARLY = false, class V = float2, class Tw>
__device__ __forceinline__ void stockham_pass(float2* buf, const Tw& tw, int tid) {
    pass_io<N, R, NS, T, INV, true, TW_EARLY, V>(
        tw, tid, [&](int j, int r) { return buf[pad_load<N, R>(j, r)]; },
        [&](int base, int r, float2 v) { buf[pad_store<R, NS>(base, r)] = v; });
    __syncthreads();
}

template <int... Rs> struct RadixList {};

// Split a radix list: Init<L>::type drops the last radix, ::last is it, ::prod multiplies the rest.
template <class A, class B> struct Concat;
template <int... A, int... B> struct Concat<RadixList<A...>, RadixList<B...>> { using type = RadixList<A..., B...>; };
template <class L> struct Init;
template <int R> struct Init<RadixList<R>> {
    using type = RadixList<>;
    static constexpr int last = R, prod = 1;
};
template <int R, int R2, int... Rest> struct Init<RadixList<R, R2, Rest...>> {
    using sub = Init<RadixList<R2, Rest...>>;
    using type = typename Concat<RadixList<R>, typename sub::type>::type;
    static constexpr int last = sub::last, prod = R * sub::prod;
};
template <class L> struct Head;
template <int R, int... Rest> struct Head<RadixList<R, Rest...>> {
    static constexpr int first = R;
    using tail = RadixList<Rest...>;
};

// In-place passes for the radices of a list, the first of them at stride NS.
template <int N, int T, bool INV, int NS, bool TW_EARLY = false, class V = float2, class Tw>
__device__ __forceinline__ void passes(float2*, const Tw&, int, RadixList<>) {}
template <int N, int T, bool INV, int NS, bool TW_EARLY = false, class V = float2, class Tw, int R, int... Rest>
__device__ __forceinline__ void passes(float2* buf, const Tw& tw, int tid, RadixList<R, Rest...>) {
    stockham_pass<N, R, NS, T, INV, TW_EARLY, V>(buf, tw, tid);
    passes<N, T, INV, NS * R, TW_EARLY, V>(buf, tw, tid, RadixList<Rest...>{});
}

// Transform the frame in buf (padded layout) in place: X[k] = sum_n x[n] W_N^{nk}, W = e^{-2 pi i/N}
// (forward) or e^{+2 pi i/N} (inverse, unnormalised). Callers synchronise before the first
// pass reads what they wrote; the last pass ends with a barrier.
template <int N, int T, bool INV, class Tw, int... Rs>
__device__ __forceinline__ void fft(float2* buf, const Tw& tw, int tid, RadixList<Rs...>) {
    passes<N, T, INV, 1>(buf, tw, tid, RadixList<Rs...>{});
}

} // namespace stg
