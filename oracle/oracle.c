/* oracle.c -- CPU restatement of stems.cpp's spectral path. TEST INFRASTRUCTURE ONLY.
 * See oracle.h for what this is and who may call it. All citations are paths inside the
 * reference project (betweentwomidnights/stems.cpp). */
#define _GNU_SOURCE
#include "oracle.h"

#include <complex.h>
#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef double complex cplx;

#define ERR_ARG (-1)
#define ERR_MEM (-2)
#define ERR_PAD (-3)

/* ===================================================================================== */
/* radix-2 FFT: src/stft.h:19-55                                                           */
/* ===================================================================================== */
typedef struct { int n; int* rev; cplx* tw; } fft_plan;
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static fft_plan* g_fft[31];

static const fft_plan* fft_plan_for(int n) {
    if (n < 2 || (n & (n - 1))) return NULL;               /* stft.h:22 */
    int bits = 0;
    while ((1 << bits) < n) bits++;
    pthread_mutex_lock(&g_mu);
    if (!g_fft[bits]) {
        fft_plan* p = (fft_plan*)calloc(1, sizeof(fft_plan));
        p->n = n;
        p->rev = (int*)malloc(sizeof(int) * n);
        p->tw = (cplx*)malloc(sizeof(cplx) * (n / 2));
        for (int i = 0; i < n; i++) {                       /* stft.h:25-29 */
            int r = 0;
            for (int b = 0; b < bits; b++) r |= ((i >> b) & 1) << (bits - 1 - b);
            p->rev[i] = r;
        }
        for (int i = 0; i < n / 2; i++) {                   /* stft.h:30, std::polar(1, th) */
            const double th = -2.0 * M_PI * i / n;
            p->tw[i] = cos(th) + I * sin(th);
        }
        g_fft[bits] = p;
    }
    pthread_mutex_unlock(&g_mu);
    return g_fft[bits];
}

/* In place, unnormalised; inverse uses conjugate twiddles (stft.h:35-49). */
static void fft_run(const fft_plan* p, cplx* a, int inverse) {
    const int n = p->n;
    for (int i = 0; i < n; i++)
        if (i < p->rev[i]) { cplx t = a[i]; a[i] = a[p->rev[i]]; a[p->rev[i]] = t; }
    for (int len = 2; len <= n; len <<= 1) {
        const int step = n / len, h = len / 2;
        for (int i = 0; i < n; i += len)
            for (int j = 0; j < h; j++) {
                cplx w = p->tw[j * step];
                if (inverse) w = conj(w);
                const cplx u = a[i + j], v = a[i + j + h] * w;
                a[i + j] = u + v;
                a[i + j + h] = u - v;
            }
    }
}

int or_fft(int n, double* a, int inverse) {
    const fft_plan* p = fft_plan_for(n);
    if (!p || !a) return ERR_ARG;
    fft_run(p, (cplx*)a, inverse);
    return 0;
}

/* ===================================================================================== */
/* Bluestein FFT for any n: src/vr_dsp.h:11-37                                             */
/* ===================================================================================== */
typedef struct { int n, m; const fft_plan* fft; cplx* chirp; cplx* kernel; } blue_plan;
static blue_plan* g_blue[16];

static const blue_plan* blue_plan_for(int n) {
    if (n < 1) return NULL;
    pthread_mutex_lock(&g_mu);
    blue_plan* found = NULL;
    int slot = -1;
    for (int i = 0; i < 16; i++) {
        if (g_blue[i] && g_blue[i]->n == n) { found = g_blue[i]; break; }
        if (!g_blue[i] && slot < 0) slot = i;
    }
    pthread_mutex_unlock(&g_mu);
    if (found) return found;
    if (slot < 0) return NULL;
    int m = 1;
    while (m < 2 * n - 1) m *= 2;                           /* vr_dsp.h:16 */
    const fft_plan* f = fft_plan_for(m);
    blue_plan* p = (blue_plan*)calloc(1, sizeof(blue_plan));
    p->n = n; p->m = m; p->fft = f;
    p->chirp = (cplx*)calloc((size_t)n, sizeof(cplx));
    p->kernel = (cplx*)calloc((size_t)m, sizeof(cplx));
    for (int i = 0; i < n; i++) {                           /* vr_dsp.h:18-22 */
        const double th = -M_PI * (double)i * i / n;
        p->chirp[i] = cos(th) + I * sin(th);
        p->kernel[i] = conj(p->chirp[i]);
        if (i) p->kernel[m - i] = p->kernel[i];
    }
    fft_run(f, p->kernel, 0);                               /* vr_dsp.h:23 */
    pthread_mutex_lock(&g_mu);
    for (int i = 0; i < 16; i++)
        if (g_blue[i] && g_blue[i]->n == n) { found = g_blue[i]; break; }
    if (!found) { g_blue[slot] = p; found = p; }
    pthread_mutex_unlock(&g_mu);
    return found;
}

static void blue_run(const blue_plan* p, cplx* x, int inverse) {   /* vr_dsp.h:26-36 */
    const int n = p->n, m = p->m;
    cplx* a = (cplx*)calloc((size_t)m, sizeof(cplx));
    for (int i = 0; i < n; i++) a[i] = (inverse ? conj(x[i]) : x[i]) * p->chirp[i];
    fft_run(p->fft, a, 0);
    for (int i = 0; i < m; i++) a[i] *= p->kernel[i];
    fft_run(p->fft, a, 1);
    for (int i = 0; i < n; i++) {
        const cplx v = a[i] * p->chirp[i] / (double)m;
        x[i] = inverse ? conj(v) : v;
    }
    free(a);
}

int or_vrfft(int n, double* a, int inverse) {
    const blue_plan* p = blue_plan_for(n);
    if (!p || !a) return ERR_ARG;
    blue_run(p, (cplx*)a, inverse);
    return 0;
}

/* The transform torch_stft/istft is given: st::FFT for powers of two, st::VRFFT otherwise
 * (src/tfc_tdf.cpp:551-552). */
static int dft(int n, cplx* a, int inverse) {
    if (n >= 2 && !(n & (n - 1))) { fft_run(fft_plan_for(n), a, inverse); return 0; }
    const blue_plan* p = blue_plan_for(n);
    if (!p) return ERR_ARG;
    blue_run(p, a, inverse);
    return 0;
}

/* ===================================================================================== */
/* reflect pad, Hann, STFT / iSTFT: src/stft.h:57-197                                      */
/* ===================================================================================== */
static double* reflect_pad(const float* x, int n, int left, int right) {  /* stft.h:58-68 */
    if (n <= left || n <= right) return NULL;
    const size_t sz = (size_t)n + left + right;
    double* y = (double*)malloc(sizeof(double) * sz);
    for (int i = 0; i < (int)sz; i++) {
        int j = i - left;
        if (j < 0) j = -j;
        if (j >= n) j = 2 * (n - 1) - j;
        y[i] = x[j];
    }
    return y;
}

static double* hann_periodic(int n) {                                    /* stft.h:70-74 */
    double* w = (double*)malloc(sizeof(double) * n);
    for (int i = 0; i < n; i++) w[i] = 0.5 - 0.5 * cos(2.0 * M_PI * i / n);
    return w;
}

int or_torch_stft(int nfft, const float* x, int len, int hop, int normalized, double* outd,
                  int* n_frames) {                                       /* stft.h:146-164 */
    if (nfft < 2 || hop < 1 || !x || !outd || len < 1) return ERR_ARG;
    const int F = nfft / 2 + 1;
    double* xp = reflect_pad(x, len, nfft / 2, nfft / 2);
    if (!xp) return ERR_PAD;
    double* win = hann_periodic(nfft);
    const double norm = normalized ? 1.0 / sqrt((double)nfft) : 1.0;
    const int T = len / hop + 1;
    if (n_frames) *n_frames = T;
    cplx* out = (cplx*)outd;
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    int rc = 0;
    for (int t = 0; t < T && !rc; t++) {
        const size_t start = (size_t)t * hop;
        for (int i = 0; i < nfft; i++) buf[i] = xp[start + i] * win[i];
        rc = dft(nfft, buf, 0);
        for (int f = 0; f < F; f++) out[(size_t)f * T + t] = buf[f] * norm;
    }
    free(buf); free(win); free(xp);
    return rc;
}

int or_torch_istft(int nfft, const double* specd, int n_frames, int hop, int normalized,
                   float* out) {                                         /* stft.h:167-197 */
    if (nfft < 2 || hop < 1 || n_frames < 1 || !specd || !out) return ERR_ARG;
    const cplx* spec = (const cplx*)specd;
    const int F = nfft / 2 + 1;
    double* win = hann_periodic(nfft);
    const size_t full = (size_t)nfft + (size_t)hop * (n_frames - 1);
    double* y = (double*)calloc(full, sizeof(double));
    double* env = (double*)calloc(full, sizeof(double));
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    const double norm = (normalized ? sqrt((double)nfft) : 1.0) / nfft;
    int rc = 0;
    for (int t = 0; t < n_frames && !rc; t++) {
        buf[0] = creal(spec[t]);                     /* c2r ignores the DC and Nyquist imag */
        for (int f = 1; f < F - 1; f++) {
            buf[f] = spec[(size_t)f * n_frames + t];
            buf[nfft - f] = conj(buf[f]);
        }
        buf[F - 1] = creal(spec[(size_t)(F - 1) * n_frames + t]);
        rc = dft(nfft, buf, 1);
        const size_t off = (size_t)t * hop;
        for (int i = 0; i < nfft; i++) {
            y[off + i] += creal(buf[i]) * norm * win[i];
            env[off + i] += win[i] * win[i];
        }
    }
    const int length = hop * (n_frames - 1);
    for (int i = 0; i < length; i++) {
        const size_t j = (size_t)nfft / 2 + i;
        out[i] = env[j] > 1e-11 ? (float)(y[j] / env[j]) : 0.0f;
    }
    free(buf); free(env); free(y); free(win);
    return rc;
}

int or_htdemucs_spec(int nfft, const float* x, int len, double* outd, int* n_frames) {
    /* stft.h:79-103 */
    if (nfft < 8 || (nfft & (nfft - 1)) || !x || !outd || len < 1) return ERR_ARG;
    const int hl = nfft / 4;
    const int le = (len + hl - 1) / hl;
    const int pad = hl / 2 * 3;
    double* p = reflect_pad(x, len, pad, pad + le * hl - len);
    if (!p) return ERR_PAD;
    const int nxf = len + pad + pad + le * hl - len;
    float* xf = (float*)malloc(sizeof(float) * nxf);
    for (int i = 0; i < nxf; i++) xf[i] = (float)p[i];
    free(p);
    double* xp = reflect_pad(xf, nxf, nfft / 2, nfft / 2);
    free(xf);
    if (!xp) return ERR_PAD;
    double* win = hann_periodic(nfft);
    const double norm = 1.0 / sqrt((double)nfft);
    const int F = nfft / 2;
    if (n_frames) *n_frames = le;
    cplx* out = (cplx*)outd;
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    for (int t = 0; t < le; t++) {
        const size_t start = (size_t)(t + 2) * hl;          /* skip the first two frames */
        for (int i = 0; i < nfft; i++) buf[i] = xp[start + i] * win[i];
        fft_run(fft_plan_for(nfft), buf, 0);
        for (int f = 0; f < F; f++) out[(size_t)f * le + t] = buf[f] * norm;
    }
    free(buf); free(win); free(xp);
    return 0;
}

int or_htdemucs_ispec(int nfft, const double* specd, int n_frames, int length, float* out) {
    /* stft.h:106-140 */
    if (nfft < 8 || (nfft & (nfft - 1)) || !specd || !out || n_frames < 1 || length < 0)
        return ERR_ARG;
    const cplx* spec = (const cplx*)specd;
    const int hl = nfft / 4, F = nfft / 2;
    const int pad = hl / 2 * 3;
    const int le_out = hl * ((length + hl - 1) / hl) + 2 * pad;
    const int frames = n_frames + 4;
    double* win = hann_periodic(nfft);
    const size_t full = (size_t)nfft + (size_t)hl * (frames - 1);
    double* y = (double*)calloc(full, sizeof(double));
    double* env = (double*)calloc(full, sizeof(double));
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    const double norm = sqrt((double)nfft) / nfft;
    for (int t = 0; t < frames; t++) {
        const int st = t - 2;
        const size_t off = (size_t)t * hl;
        if (st >= 0 && st < n_frames) {
            buf[0] = creal(spec[st]);
            for (int f = 1; f < F; f++) {
                buf[f] = spec[(size_t)f * n_frames + st];
                buf[nfft - f] = conj(buf[f]);
            }
            buf[F] = 0.0;
            fft_run(fft_plan_for(nfft), buf, 1);
            for (int i = 0; i < nfft; i++) y[off + i] += creal(buf[i]) * norm * win[i];
        }
        for (int i = 0; i < nfft; i++) env[off + i] += win[i] * win[i];
    }
    for (int i = 0; i < length; i++) {
        const size_t j = (size_t)nfft / 2 + pad + i;
        if ((int)(j - nfft / 2) >= le_out || j >= full) { out[i] = 0.0f; continue; }
        out[i] = env[j] > 1e-11 ? (float)(y[j] / env[j]) : 0.0f;
    }
    free(buf); free(env); free(y); free(win);
    return 0;
}

/* ===================================================================================== */
/* primitive table: the restatement above, or the reference's own compiled code            */
/* ===================================================================================== */
typedef int (*stft_fn)(int, const float*, int, int, int, double*, int*);
typedef int (*istft_fn)(int, const double*, int, int, int, float*);
typedef int (*hspec_fn)(int, const float*, int, double*, int*);
typedef int (*hispec_fn)(int, const double*, int, int, float*);
static struct { stft_fn stft; istft_fn istft; hspec_fn hspec; hispec_fn hispec; void* so; } g_dsp = {
    or_torch_stft, or_torch_istft, or_htdemucs_spec, or_htdemucs_ispec, NULL};

int or_use_reference(const char* path) {
    if (!path) {
        g_dsp.stft = or_torch_stft; g_dsp.istft = or_torch_istft;
        g_dsp.hspec = or_htdemucs_spec; g_dsp.hispec = or_htdemucs_ispec;
        return 0;
    }
    void* so = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!so) return ERR_ARG;
    stft_fn a = (stft_fn)dlsym(so, "ref_torch_stft");
    istft_fn b = (istft_fn)dlsym(so, "ref_torch_istft");
    hspec_fn c = (hspec_fn)dlsym(so, "ref_htdemucs_spec");
    hispec_fn d = (hispec_fn)dlsym(so, "ref_htdemucs_ispec");
    if (!a || !b || !c || !d) { dlclose(so); return ERR_ARG; }
    g_dsp.stft = a; g_dsp.istft = b; g_dsp.hspec = c; g_dsp.hispec = d; g_dsp.so = so;
    return 0;
}

int or_using_reference(void) { return g_dsp.stft != or_torch_stft; }

/* ===================================================================================== */
/* a tiny parallel-for over chunk indices (the per-chunk work is independent; the          */
/* accumulation afterwards runs in chunk order, exactly as the reference's serial loop)    */
/* ===================================================================================== */
typedef struct {
    int (*fn)(void* ctx, int i);
    void* ctx;
    int first, end;
    int next;
    int rc;
    pthread_mutex_t mu;
} pfor_t;

static void* pfor_worker(void* arg) {
    pfor_t* pf = (pfor_t*)arg;
    for (;;) {
        pthread_mutex_lock(&pf->mu);
        const int i = pf->next++;
        const int stop = pf->rc != 0;
        pthread_mutex_unlock(&pf->mu);
        if (i >= pf->end || stop) break;
        const int rc = pf->fn(pf->ctx, i);
        if (rc) { pthread_mutex_lock(&pf->mu); if (!pf->rc) pf->rc = rc; pthread_mutex_unlock(&pf->mu); }
    }
    return NULL;
}

static int parallel_for(int first, int end, int threads, int (*fn)(void*, int), void* ctx) {
    if (threads <= 1 || end - first <= 1) {
        for (int i = first; i < end; i++) { const int rc = fn(ctx, i); if (rc) return rc; }
        return 0;
    }
    pfor_t pf = {fn, ctx, first, end, first, 0, PTHREAD_MUTEX_INITIALIZER};
    if (threads > end - first) threads = end - first;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    for (int k = 0; k < threads; k++) pthread_create(&th[k], NULL, pfor_worker, &pf);
    for (int k = 0; k < threads; k++) pthread_join(th[k], NULL);
    free(th);
    return pf.rc;
}

static void sample_window(int n, int first, int count, int* lo, int* hi) {
    *lo = 0; *hi = n;
    if (count > 0) {
        *lo = first < 0 ? 0 : (first > n ? n : first);
        *hi = *lo + count > n ? n : *lo + count;
    }
}

/* ===================================================================================== */
/* HTDemucs: Impl::run spectral part (htdemucs.cpp:419-475) + separate (534-644)           */
/* ===================================================================================== */
enum { HT_NFFT = 4096, HT_HOP = 1024 };   /* htdemucs.cpp:35-36 */

int or_ht_n_frames(const or_ht_params* p) { return (p->segment + HT_HOP - 1) / HT_HOP; }  /* :320 */

static int ht_stride(const or_ht_params* p) {                            /* htdemucs.cpp:563-564 */
    const double overlap = p->overlap < 0.0f ? 0.25 : (double)p->overlap;
    return (int)((1.0 - overlap) * p->segment);
}

static int ht_view_segments(const or_ht_params* p, int view_len) {
    const int stride = ht_stride(p);
    if (stride <= 0 || view_len <= 0) return 0;
    return (view_len + stride - 1) / stride;                              /* :576, 592 */
}

static int max_shift_of(int sample_rate);

/* All segments the separation runs, every shift's view included (:575-577). */
int or_ht_n_segments(const or_ht_params* p, int len) {
    if (p->shifts <= 0) return ht_view_segments(p, len);
    const int ms = max_shift_of(p->sample_rate);
    int* off = (int*)malloc(sizeof(int) * p->shifts);
    or_shift_offsets(p->seed, p->shifts, ms, off);                          /* :617-619 */
    int n = 0;
    for (int k = 0; k < p->shifts; k++) n += ht_view_segments(p, len + ms - off[k]);
    free(off);
    return n;
}

static double mean_of(const float* x, size_t n) {                        /* htdemucs.cpp:293-297 */
    double s = 0;
    for (size_t i = 0; i < n; i++) s += x[i];
    return s / n;
}
static double std_of(const float* x, size_t n, double mean) {            /* :298-302 */
    double s = 0;
    for (size_t i = 0; i < n; i++) { const double d = x[i] - mean; s += d * d; }
    return sqrt(s / (n - 1));
}

typedef struct {
    const or_ht_params* p;
    const float* buf;      /* the buffer the view looks into [C][total] */
    int total;
    int view0, view_len;   /* the view: buffer samples [view0, view0 + view_len) */
    int stride, seg, T;
    const float* mask;     /* the view's first segment's mask */
    float* seg_out;        /* [G][S][C][seg] */
} ht_job;

/* One segment: padded view (htdemucs.cpp:552-561, 594-595) -> run (419-475) with the
 * network replaced by ox = Z * M (complex, per stem and channel). */
static int ht_segment(void* vctx, int g) {
    ht_job* J = (ht_job*)vctx;
    const or_ht_params* p = J->p;
    const int C = p->n_channels, S = p->n_sources, L = J->seg, T = J->T, F = HT_NFFT / 2;
    const int off = g * J->stride;
    const int length = J->view_len - off < L ? J->view_len - off : L;
    const int start = J->view0 + off - (L - length) / 2;
    float* seg_in = (float*)calloc((size_t)C * L, sizeof(float));
    for (int c = 0; c < C; c++)
        for (int i = 0; i < L; i++) {
            const int j = start + i;
            if (j >= 0 && j < J->total) seg_in[(size_t)c * L + i] = J->buf[(size_t)c * J->total + j];
        }
    const size_t FT = (size_t)F * T;
    float* mag = (float*)malloc(sizeof(float) * 2 * C * FT);
    cplx* z = (cplx*)malloc(sizeof(cplx) * FT);
    int rc = 0;
    for (int c = 0; c < C && !rc; c++) {
        int frames = 0;
        rc = g_dsp.hspec(HT_NFFT, seg_in + (size_t)c * L, L, (double*)z, &frames);
        if (!rc && frames != T) rc = ERR_ARG;
        for (size_t i = 0; i < FT && !rc; i++) {
            mag[(size_t)(2 * c) * FT + i] = (float)creal(z[i]);
            mag[(size_t)(2 * c + 1) * FT + i] = (float)cimag(z[i]);
        }
    }
    double mean = 0.0, sd = 1.0;
    if (!rc && p->cac_norm) {                                             /* :434-436 */
        mean = mean_of(mag, 2 * C * FT);
        sd = std_of(mag, 2 * C * FT, mean);
        for (size_t i = 0; i < 2 * C * FT; i++) mag[i] = (float)((mag[i] - mean) / (1e-5 + sd));
    }
    cplx* spec = z;
    float* y = (float*)malloc(sizeof(float) * L);
    const float* M = J->mask + (size_t)g * S * 2 * C * FT;
    for (int s = 0; s < S && !rc; s++)
        for (int c = 0; c < C && !rc; c++) {
            const float* zr = mag + (size_t)(2 * c) * FT;
            const float* zi = mag + (size_t)(2 * c + 1) * FT;
            const float* mr = M + (size_t)(s * 2 * C + 2 * c) * FT;
            const float* mi = M + (size_t)(s * 2 * C + 2 * c + 1) * FT;
            for (size_t i = 0; i < FT; i++) {
                /* stand-in network output, a float tensor like ox (htdemucs.cpp:450-452) */
                const float re = (float)((double)zr[i] * mr[i] - (double)zi[i] * mi[i]);
                const float im = (float)((double)zr[i] * mi[i] + (double)zi[i] * mr[i]);
                spec[i] = p->cac_norm ? (re * sd + mean) + I * (im * sd + mean)   /* :469 */
                                      : (double)re + I * (double)im;
            }
            rc = g_dsp.hispec(HT_NFFT, (const double*)spec, T, L, y);     /* :470 */
            float* o = J->seg_out + (((size_t)g * S + s) * C + c) * L;
            memcpy(o, y, sizeof(float) * L);                              /* time branch dropped */
        }
    free(y); free(z); free(mag); free(seg_in);
    return rc;
}

/* split() over one view (htdemucs.cpp:588-606): the view's segments, weighted overlap-add,
 * centre trim, divided by the summed weight. out [S][C][view_len]. sampled: honour the
 * params' sample window (timing only). */
static int ht_split(const or_ht_params* p, const float* buf, int total, int view0, int view_len,
                    const float* mask, const float* weight, int sampled, float* out) {
    const int S = p->n_sources, C = p->n_channels, seg = p->segment, stride = ht_stride(p);
    const int G = ht_view_segments(p, view_len);
    int lo = 0, hi = G;
    if (sampled) sample_window(G, p->sample_first, p->sample_count, &lo, &hi);
    ht_job J = {p, buf, total, view0, view_len, stride, seg, or_ht_n_frames(p), mask, NULL};
    J.seg_out = (float*)malloc(sizeof(float) * (size_t)G * S * C * seg);
    if (!J.seg_out) return ERR_MEM;
    int rc = parallel_for(lo, hi, p->threads, ht_segment, &J);
    float* sum_w = (float*)calloc((size_t)view_len, sizeof(float));
    memset(out, 0, sizeof(float) * (size_t)S * C * view_len);
    for (int g = lo; g < hi && !rc; g++) {
        const int off = g * stride;
        const int length = view_len - off < seg ? view_len - off : seg;
        const int trim = (seg - length) / 2;                              /* center_trim */
        for (int sc = 0; sc < S * C; sc++) {
            const float* so = J.seg_out + ((size_t)g * S * C + sc) * seg;
            for (int i = 0; i < length; i++)
                out[(size_t)sc * view_len + off + i] += weight[i] * so[trim + i];
        }
        for (int i = 0; i < length; i++) sum_w[off + i] += weight[i];
    }
    for (int sc = 0; sc < S * C && !rc; sc++)
        for (int i = 0; i < view_len; i++) out[(size_t)sc * view_len + i] /= sum_w[i];
    free(sum_w); free(J.seg_out);
    return rc;
}

/* One model's estimate on the normalised mix (htdemucs.cpp:609-627): split() over the mix, or
 * the shifts' views averaged; res [S][C][len]. */
static int ht_model(const or_ht_params* p, const float* mix, int len, const float* mask, const float* weight,
                    float* res) {
    const int S = p->n_sources, C = p->n_channels;
    int rc = 0;
    if (p->shifts <= 0) {
        rc = ht_split(p, mix, len, 0, len, mask, weight, 1, res);         /* :610-611 */
    } else {
        /* views of the mix padded by max_shift zeros per side; offset uniform in
         * [0, max_shift], the views' estimates summed then divided (:612-626) */
        const int ms = max_shift_of(p->sample_rate), total = len + 2 * ms;
        float* pm = (float*)calloc((size_t)C * total, sizeof(float));
        for (int c = 0; c < C; c++) memcpy(pm + (size_t)c * total + ms, mix + (size_t)c * len, sizeof(float) * len);
        int* off = (int*)malloc(sizeof(int) * p->shifts);
        or_shift_offsets(p->seed, p->shifts, ms, off);
        memset(res, 0, sizeof(float) * (size_t)S * C * len);
        const size_t mask_per_seg = (size_t)S * 2 * C * (HT_NFFT / 2) * or_ht_n_frames(p);
        const float* m = mask;
        for (int k = 0; k < p->shifts && !rc; k++) {
            const int vl = len + ms - off[k];
            float* o = (float*)malloc(sizeof(float) * (size_t)S * C * vl);
            rc = ht_split(p, pm, total, off[k], vl, m, weight, 0, o);
            for (int sc = 0; sc < S * C && !rc; sc++)
                for (int i = 0; i < len; i++) res[(size_t)sc * len + i] += o[(size_t)sc * vl + ms - off[k] + i];
            m += (size_t)ht_view_segments(p, vl) * mask_per_seg;
            free(o);
        }
        for (size_t i = 0; i < (size_t)S * C * len && !rc; i++) res[i] /= p->shifts;
        free(off); free(pm);
    }
    return rc;
}

int or_ht_separate(const or_ht_params* p, const float* mix_in, int len, const float* mask,
                   float* est) {
    if (!p || !mix_in || !mask || !est || len <= 0 || p->n_channels < 1 || p->n_sources < 1 ||
        p->segment < 4 * HT_HOP)
        return ERR_ARG;
    const int S = p->n_sources, C = p->n_channels, seg = p->segment;
    const int stride = ht_stride(p);
    if (stride <= 0) return ERR_ARG;
    /* mono-mix normalisation (htdemucs.cpp:539-549), optional here */
    float* mix = (float*)malloc(sizeof(float) * C * len);
    double ref_mean = 0.0, ref_std = 1.0;
    if (p->mono_norm) {
        float* mono = (float*)malloc(sizeof(float) * len);
        for (int i = 0; i < len; i++) {
            double s = 0;
            for (int c = 0; c < C; c++) s += mix_in[(size_t)c * len + i];
            mono[i] = (float)(s / C);
        }
        ref_mean = mean_of(mono, len);
        ref_std = std_of(mono, len, ref_mean);
        if (ref_std < 1e-8) ref_std = 1e-8;
        for (size_t i = 0; i < (size_t)C * len; i++) mix[i] = (float)((mix_in[i] - ref_mean) / ref_std);
        free(mono);
    } else {
        memcpy(mix, mix_in, sizeof(float) * C * len);
    }
    /* triangular weight (htdemucs.cpp:566-573) */
    float* weight = (float*)malloc(sizeof(float) * seg);
    {
        const int half = seg / 2;
        for (int i = 0; i < half; i++) weight[i] = (float)(i + 1);
        for (int i = half; i < seg; i++) weight[i] = (float)(seg - i);
        float mx = weight[0];
        for (int i = 1; i < seg; i++) if (weight[i] > mx) mx = weight[i];
        for (int i = 0; i < seg; i++) weight[i] /= mx;
    }
    int rc = 0;
    const size_t n_out = (size_t)S * C * len;
    if (p->n_models <= 1 && !p->bag) {
        rc = ht_model(p, mix, len, mask, weight, est);
        /* one model, weight 1: v / 1 * ref_std + ref_mean (:629-642) */
        if (p->mono_norm && !rc)
            for (size_t i = 0; i < n_out; i++) est[i] = (float)(est[i] * ref_std + ref_mean);
    } else {
        /* the bag (:585-642): each model's estimate weighted per stem and summed in model order
         * (float), then divided by the weights' sum and mapped back by the mono statistics */
        const int M = p->n_models > 1 ? p->n_models : 1;
        const size_t mask_per_model = (size_t)or_ht_n_segments(p, len) * S * 2 * C * (HT_NFFT / 2) * or_ht_n_frames(p);
        float* res = (float*)malloc(sizeof(float) * n_out);
        float* totals = (float*)calloc((size_t)S, sizeof(float));
        memset(est, 0, sizeof(float) * n_out);
        for (int mi = 0; mi < M && !rc; mi++) {
            rc = ht_model(p, mix, len, mask + (size_t)mi * mask_per_model, weight, res);
            for (int s = 0; s < S && !rc; s++) {
                const float w = p->bag ? p->bag[(size_t)mi * S + s] : 1.0f;     /* :630 */
                totals[s] += w;
                if (w == 0.0f) continue;
                for (size_t i = 0; i < (size_t)C * len; i++) est[(size_t)s * C * len + i] += w * res[(size_t)s * C * len + i];
            }
        }
        for (int s = 0; s < S && !rc; s++)                                   /* :638-642 */
            for (size_t i = 0; i < (size_t)C * len; i++) {
                float* v = &est[(size_t)s * C * len + i];
                *v = (float)(*v / totals[s] * ref_std + ref_mean);
            }
        free(totals); free(res);
    }
    free(weight); free(mix);
    return rc;
}

/* ===================================================================================== */
/* RoFormer: Impl::run (roformer.cpp:217-283), demix (286-351), separate (436-486)         */
/* ===================================================================================== */
static int rf_check(const or_rf_params* p) {
    if (!p || p->n_channels < 1 || p->n_stems < 1 || p->n_fft < 2 || p->hop < 1 ||
        p->chunk < 1 || p->step < 1 || p->chunk % p->hop || p->n_bands < 1 || !p->band_sizes ||
        !p->band_freqs)
        return ERR_ARG;
    const int F = p->n_fft / 2 + 1;
    size_t nf = 0;
    for (int b = 0; b < p->n_bands; b++) nf += p->band_sizes[b];
    for (size_t k = 0; k < nf; k++)
        if (p->band_freqs[k] < 0 || p->band_freqs[k] >= F) return ERR_ARG;  /* :408-411 */
    return 0;
}

static int rf_demix_chunks(const or_rf_params* p, int len) {            /* roformer.cpp:353-357 */
    const int border = p->chunk - p->step;
    const int Lp = (len > 2 * border && border > 0) ? len + 2 * border : len;
    return (Lp + p->step - 1) / p->step;
}

static int max_shift_of(int sample_rate) { return (sample_rate > 0 ? sample_rate : 44100) / 2; }

int or_rf_n_chunks(const or_rf_params* p, int len) {
    if (p->shifts <= 0) return rf_demix_chunks(p, len);
    const int ms = max_shift_of(p->sample_rate);                           /* :460 */
    int* off = (int*)malloc(sizeof(int) * p->shifts);
    or_shift_offsets(p->seed, p->shifts, ms - 1, off);                      /* :461-465 */
    int n = 0;
    for (int k = 0; k < p->shifts; k++) n += rf_demix_chunks(p, len + ms - off[k]);
    free(off);
    return n;
}

int or_rf_band_gather(const or_rf_params* p, const double* zd, int T, float* feat) {
    /* roformer.cpp:226-241: 'b (f s) t c' by the band lists, then 'b f t c -> b t (f c)' */
    if (rf_check(p) || !zd || !feat) return ERR_ARG;
    const cplx* z = (const cplx*)zd;
    const int C = p->n_channels, F = p->n_fft / 2 + 1;
    size_t foff = 0, off = 0;
    for (int b = 0; b < p->n_bands; b++) {
        const int din = p->band_sizes[b] * C * 2;
        float* blk = feat + off * T;
        for (int j = 0; j < p->band_sizes[b]; j++) {
            const int f = p->band_freqs[foff + j];
            for (int c = 0; c < C; c++)
                for (int t = 0; t < T; t++) {
                    const cplx v = z[((size_t)c * F + f) * T + t];
                    float* q = &blk[(size_t)t * din + (j * C + c) * 2];
                    q[0] = (float)creal(v);
                    q[1] = (float)cimag(v);
                }
        }
        foff += p->band_sizes[b];
        off += din;
    }
    return 0;
}

typedef struct {
    const or_rf_params* p;
    const float* x;       /* padded mix [C][Lp] */
    int Lp;
    const float* mask;
    size_t mask_per_chunk;
    float* y;             /* [G][S][C][chunk] */
    const int* bpf;       /* bands_per_freq [F] */
} rf_job;

static int rf_chunk(void* vctx, int g) {
    rf_job* J = (rf_job*)vctx;
    const or_rf_params* p = J->p;
    const int C = p->n_channels, S = p->n_stems, Cc = p->chunk, F = p->n_fft / 2 + 1;
    const int T = Cc / p->hop + 1;                                        /* :83 */
    const int i0 = g * p->step;
    const int length = J->Lp - i0 < Cc ? J->Lp - i0 : Cc;
    /* chunk copy with the short-tail rule (roformer.cpp:318-331) */
    float* part = (float*)calloc((size_t)C * Cc, sizeof(float));
    int rc = 0;
    for (int c = 0; c < C && !rc; c++) {
        const float* src = &J->x[(size_t)c * J->Lp + i0];
        float* dst = &part[(size_t)c * Cc];
        memcpy(dst, src, sizeof(float) * length);
        if (length < Cc) {
            if (length > Cc / 2 + 1) {
                double* q = reflect_pad(src, length, 0, Cc - length);
                if (!q) { rc = ERR_PAD; break; }
                for (int k = 0; k < Cc; k++) dst[k] = (float)q[k];
                free(q);
            }
        }
    }
    const size_t FT = (size_t)F * T;
    cplx* z = (cplx*)malloc(sizeof(cplx) * C * FT);
    for (int c = 0; c < C && !rc; c++) {                                  /* :220-224 */
        int frames = 0;
        rc = g_dsp.stft(p->n_fft, part + (size_t)c * Cc, Cc, p->hop, p->normalized,
                        (double*)(z + (size_t)c * FT), &frames);
        if (!rc && frames != T) rc = ERR_ARG;
    }
    /* masks averaged where bands overlap, applied, inverted (:251-282) */
    cplx* acc = (cplx*)malloc(sizeof(cplx) * C * FT);
    cplx* spec = (cplx*)malloc(sizeof(cplx) * FT);
    float* yt = (float*)malloc(sizeof(float) * ((size_t)p->hop * (T - 1)));
    for (int s = 0; s < S && !rc; s++) {
        memset(acc, 0, sizeof(cplx) * C * FT);
        const float* m = J->mask + (size_t)g * J->mask_per_chunk + (size_t)s * (J->mask_per_chunk / S);
        size_t foff = 0, off = 0;
        for (int b = 0; b < p->n_bands; b++) {
            const int din = p->band_sizes[b] * C * 2;
            const float* mb = m + off * T;
            for (int j = 0; j < p->band_sizes[b]; j++) {
                const int f = p->band_freqs[foff + j];
                for (int c = 0; c < C; c++)
                    for (int t = 0; t < T; t++) {
                        const float* q = &mb[(size_t)t * din + (j * C + c) * 2];
                        acc[((size_t)c * F + f) * T + t] += q[0] + I * (double)q[1];
                    }
            }
            foff += p->band_sizes[b];
            off += din;
        }
        for (int c = 0; c < C && !rc; c++) {
            for (int f = 0; f < F; f++) {
                const double denom = J->bpf[f] > 1 ? J->bpf[f] : 1;
                for (int t = 0; t < T; t++) {
                    const size_t i = (size_t)f * T + t;
                    spec[i] = z[(size_t)c * FT + i] * (acc[(size_t)c * FT + i] / denom);
                }
            }
            if (p->zero_dc) for (int t = 0; t < T; t++) spec[t] = 0.0;        /* :278 */
            rc = g_dsp.istft(p->n_fft, (const double*)spec, T, p->hop, p->normalized, yt);
            memcpy(J->y + (((size_t)g * S + s) * C + c) * Cc, yt, sizeof(float) * Cc);  /* :280 */
        }
    }
    free(yt); free(spec); free(acc); free(z); free(part);
    return rc;
}

/* demix() of one track (roformer.cpp:286-351): out [S][C][len]. */
static int rf_demix(const or_rf_params* p, const float* mix, int len, const float* mask, float* out) {
    const int C = p->n_channels, S = p->n_stems, Cc = p->chunk, step = p->step, F = p->n_fft / 2 + 1;
    const int T = Cc / p->hop + 1;
    const int fade = Cc / 10, border = Cc - step;                         /* :288-291 */
    const int pad = len > 2 * border && border > 0;
    const int Lp = pad ? len + 2 * border : len;
    float* x = (float*)malloc(sizeof(float) * C * Lp);
    for (int c = 0; c < C; c++) {
        const float* src = &mix[(size_t)c * len];
        if (pad) {
            double* q = reflect_pad(src, len, border, border);
            if (!q) { free(x); return ERR_PAD; }
            for (int k = 0; k < Lp; k++) x[(size_t)c * Lp + k] = (float)q[k];
            free(q);
        } else {
            memcpy(&x[(size_t)c * Lp], src, sizeof(float) * len);
        }
    }
    /* torch.linspace(0, 1, fade) from both ends; fade-in and fade-out window (:303-313) */
    float* fade_in = (float*)calloc((size_t)(fade > 0 ? fade : 1), sizeof(float));
    float* window = (float*)malloc(sizeof(float) * Cc);
    for (int i = 0; i < Cc; i++) window[i] = 1.0f;
    if (fade > 1) {
        const float stp = 1.0f / (float)(fade - 1);
        for (int i = 0; i < fade; i++)
            fade_in[i] = i < fade / 2 ? (float)i * stp : 1.0f - (float)(fade - 1 - i) * stp;
    }
    for (int i = 0; i < fade; i++) { window[i] *= fade_in[i]; window[Cc - 1 - i] *= fade_in[i]; }
    /* bands per frequency (:399-411) and the per-chunk mask size */
    int* bpf = (int*)calloc((size_t)F, sizeof(int));
    size_t nf = 0, din_total = 0;
    for (int b = 0; b < p->n_bands; b++) { nf += p->band_sizes[b]; din_total += (size_t)p->band_sizes[b] * C * 2; }
    for (size_t k = 0; k < nf; k++) bpf[p->band_freqs[k]]++;
    const int G = (Lp + step - 1) / step;
    int lo, hi;
    sample_window(G, p->sample_first, p->sample_count, &lo, &hi);
    rf_job J = {p, x, Lp, mask, (size_t)S * din_total * T, NULL, bpf};
    J.y = (float*)malloc(sizeof(float) * (size_t)G * S * C * Cc);
    int rc = J.y ? parallel_for(lo, hi, p->threads, rf_chunk, &J) : ERR_MEM;
    double* result = (double*)calloc((size_t)S * C * Lp, sizeof(double));
    double* counter = (double*)calloc((size_t)Lp, sizeof(double));
    float* w = (float*)malloc(sizeof(float) * Cc);
    for (int g = lo; g < hi && !rc; g++) {                                /* :317-341 */
        const int i0 = g * step;
        const int length = Lp - i0 < Cc ? Lp - i0 : Cc;
        memcpy(w, window, sizeof(float) * Cc);
        if (i0 == 0) for (int k = 0; k < fade; k++) w[k] = 1.0f;
        else if (i0 + Cc >= Lp) for (int k = Cc - fade; k < Cc; k++) w[k] = 1.0f;
        for (int k = 0; k < S * C; k++)
            for (int t = 0; t < length; t++)
                result[(size_t)k * Lp + i0 + t] += (double)J.y[((size_t)g * S * C + k) * Cc + t] * w[t];
        for (int t = 0; t < length; t++) counter[i0 + t] += w[t];
    }
    const int off = pad ? border : 0;                                     /* :343-349 */
    for (int k = 0; k < S * C && !rc; k++)
        for (int t = 0; t < len; t++) {
            const double v = result[(size_t)k * Lp + off + t] / counter[off + t];
            out[(size_t)k * len + t] = isfinite(v) ? (float)v : 0.0f;
        }
    free(w); free(counter); free(result); free(J.y); free(bpf); free(window); free(fade_in); free(x);
    return rc;
}

/* separate() (roformer.cpp:436-486): one demix, or the average over random shifts, then the
 * complement. */
int or_rf_separate(const or_rf_params* p, const float* mix, int len, const float* mask, float* out) {
    if (rf_check(p) || !mix || !mask || !out || len <= 0) return ERR_ARG;
    const int C = p->n_channels, S = p->n_stems;
    int rc = 0;
    if (p->shifts <= 0) {
        rc = rf_demix(p, mix, len, mask, out);                            /* :456-457 */
    } else {
        const int ms = max_shift_of(p->sample_rate), T = p->chunk / p->hop + 1;
        size_t din_total = 0;
        for (int b = 0; b < p->n_bands; b++) din_total += (size_t)p->band_sizes[b] * C * 2;
        const size_t mask_per_chunk = (size_t)S * din_total * T;
        int* off = (int*)malloc(sizeof(int) * p->shifts);
        or_shift_offsets(p->seed, p->shifts, ms - 1, off);                  /* :461-465 */
        memset(out, 0, sizeof(float) * (size_t)S * C * len);
        const float* m = mask;
        for (int k = 0; k < p->shifts && !rc; k++) {
            const int n = len + ms - off[k];                              /* :466 */
            float* shifted = (float*)calloc((size_t)C * n, sizeof(float));
            float* y = (float*)malloc(sizeof(float) * (size_t)S * C * n);
            for (int c = 0; c < C; c++)                                   /* :467-472 */
                for (int t = 0; t < n; t++) {
                    const int src = t + off[k] - ms;
                    if (src >= 0 && src < len) shifted[(size_t)c * n + t] = mix[(size_t)c * len + src];
                }
            rc = rf_demix(p, shifted, n, m, y);
            for (int i = 0; i < S * C && !rc; i++)                        /* :474-477 */
                for (int t = 0; t < len; t++)
                    out[(size_t)i * len + t] += y[(size_t)i * n + ms - off[k] + t] / p->shifts;
            m += (size_t)rf_demix_chunks(p, n) * mask_per_chunk;
            free(y); free(shifted);
        }
        free(off);
    }
    if (p->complement && !rc)                                             /* :481-485 */
        for (size_t i = 0; i < (size_t)C * len; i++) out[(size_t)S * C * len + i] = mix[i] - out[i];
    return rc;
}

/* ===================================================================================== */
/* TFC-TDF: run_chunk (tfc_tdf.cpp:362-391), demix_uvr (398-429), demix_msst (434-495),    */
/* separate (570-598)                                                                      */
/* ===================================================================================== */
static int tfc_chunk_len(const or_tfc_params* p) { return p->hop * (p->dim_t - 1); }   /* :94 */

static int64_t tfc_step(const or_tfc_params* p) {
    const int C = tfc_chunk_len(p);
    if (p->chunking == 0)                                                 /* :403 */
        return p->overlap < 0 ? C - p->n_fft : (int64_t)((1.0 - (double)p->overlap) * C);
    if (p->overlap < 0) return C / p->num_overlap;                        /* :437 */
    const long s = lround(C * (1.0 - p->overlap));
    return s > 1 ? s : 1;
}

static int tfc_check(const or_tfc_params* p) {
    if (!p || p->n_stems < 1 || p->n_fft < 16 || p->hop < 1 || p->dim_f < 1 ||
        p->dim_f > p->n_fft / 2 + 1 || p->dim_t < 2 || p->zero_bins < 0 || p->zero_bins > p->dim_f ||
        (p->chunking != 0 && p->chunking != 1) || (p->chunking == 1 && p->num_overlap < 1))
        return ERR_ARG;
    if (tfc_chunk_len(p) <= p->n_fft / 2) return ERR_ARG;
    if (p->chunking == 0 && tfc_chunk_len(p) - p->n_fft <= 0) return ERR_ARG;
    if (tfc_step(p) <= 0) return ERR_ARG;
    return 0;
}

/* Length of the padded signal the chunks walk over, and where the track starts in it. */
static int64_t tfc_padded(const or_tfc_params* p, int len, int* start) {
    const int C = tfc_chunk_len(p);
    if (p->chunking == 0) {
        const int trim = p->n_fft / 2, gen = C - 2 * trim;                /* :400-402 */
        *start = trim;
        return (int64_t)trim + len + gen + trim - len % gen;
    }
    const int border = C - (int)tfc_step(p);                              /* :438-440 */
    const int pad = len > 2 * border && border > 0;
    *start = pad ? border : 0;
    return pad ? (int64_t)len + 2 * border : len;
}

int or_tfc_n_chunks(const or_tfc_params* p, int len) {
    if (tfc_check(p) || len <= 0) return 0;
    int start;
    const int64_t M = tfc_padded(p, len, &start);
    const int64_t step = tfc_step(p);
    return (int)((M + step - 1) / step);
}

typedef struct {
    const or_tfc_params* p;
    const float* x;     /* padded [2][M] */
    int64_t M, step;
    const float* mask;
    float* y;           /* [G][S][2][chunk] */
} tfc_job;

static int tfc_chunk(void* vctx, int g) {
    tfc_job* J = (tfc_job*)vctx;
    const or_tfc_params* p = J->p;
    const int C = tfc_chunk_len(p), S = p->n_stems, Fn = p->n_fft / 2 + 1, dim_f = p->dim_f,
              dim_t = p->dim_t;
    const int64_t i0 = (int64_t)g * J->step;
    const int n = (int)(J->M - i0 < C ? J->M - i0 : C);
    float* part = (float*)calloc((size_t)2 * C, sizeof(float));
    int rc = 0;
    for (int c = 0; c < 2; c++) {
        const float* src = &J->x[(size_t)c * J->M + i0];
        float* dst = &part[(size_t)c * C];
        memcpy(dst, src, sizeof(float) * n);                              /* uvr: zero tail (:413-416) */
        if (p->chunking == 1 && n < C && n > C / 2) {                     /* msst (:467-474) */
            double* q = reflect_pad(src, n, 0, C - n);
            if (!q) { rc = ERR_PAD; break; }
            for (int k = 0; k < C; k++) dst[k] = (float)q[k];
            free(q);
        }
    }
    const size_t plane = (size_t)dim_f * dim_t;
    float* in = (float*)calloc(4 * plane, sizeof(float));
    cplx* s = (cplx*)malloc(sizeof(cplx) * (size_t)Fn * dim_t);
    /* zero_bins is read only for uvr_mdx models; msst ones keep every bin (:532) */
    const int zero_bins = p->chunking == 0 ? p->zero_bins : 0;
    for (int c = 0; c < 2 && !rc; c++) {                                  /* :366-376 */
        int T = 0;
        rc = g_dsp.stft(p->n_fft, part + (size_t)c * C, C, p->hop, 0, (double*)s, &T);
        if (!rc && T != dim_t) rc = ERR_ARG;
        for (int f = zero_bins; f < dim_f && !rc; f++)
            for (int t = 0; t < T; t++) {
                const cplx v = s[(size_t)f * T + t];
                in[(2 * c) * plane + (size_t)f * T + t] = (float)creal(v);
                in[(2 * c + 1) * plane + (size_t)f * T + t] = (float)cimag(v);
            }
    }
    float* w = (float*)malloc(sizeof(float) * C);
    const float* m = J->mask + (size_t)g * 4 * S * plane;
    for (int k = 0; k < S && !rc; k++)                                    /* :381-390 */
        for (int c = 0; c < 2 && !rc; c++) {
            const float* mr = m + (size_t)(4 * k + 2 * c) * plane;
            const float* mi = mr + plane;
            const float* re = in + (size_t)(2 * c) * plane;
            const float* im = re + plane;
            for (size_t i = 0; i < (size_t)Fn * dim_t; i++) s[i] = 0.0;
            for (size_t i = 0; i < plane; i++) s[i] = (double)(re[i] * mr[i]) + I * (double)(im[i] * mi[i]);
            rc = g_dsp.istft(p->n_fft, (const double*)s, dim_t, p->hop, 0, w);
            memcpy(J->y + (((size_t)g * S + k) * 2 + c) * C, w, sizeof(float) * C);
        }
    free(w); free(s); free(in); free(part);
    return rc;
}

static void np_hanning(int n, double* w) {                                /* tfc_tdf.cpp:65-70 */
    for (int i = 0; i < n; i++) w[i] = 1.0;
    if (n > 1) for (int i = 0; i < n; i++) w[i] = 0.5 - 0.5 * cos(2.0 * M_PI * i / (n - 1));
}

static void torch_linspace(float a, float b, int n, float* v) {           /* tfc_tdf.cpp:55-62 */
    if (n == 1) v[0] = a;
    if (n < 2) return;
    const float step = (b - a) / (float)(n - 1);
    for (int i = 0; i < n; i++) v[i] = i < n / 2 ? a + step * (float)i : b - step * (float)(n - 1 - i);
}

int or_tfc_separate(const or_tfc_params* p, const float* mix, int len, const float* mask, float* out) {
    if (tfc_check(p) || !mix || !mask || !out || len <= 0) return ERR_ARG;
    for (size_t k = 0; k < (size_t)2 * len; k++) if (!isfinite(mix[k])) return ERR_ARG;   /* :573-574 */
    const int C = tfc_chunk_len(p), S = p->n_stems;
    int start = 0;
    const int64_t M = tfc_padded(p, len, &start);
    const int64_t step = tfc_step(p);
    float* x = (float*)calloc((size_t)2 * M, sizeof(float));
    for (int c = 0; c < 2; c++) {
        const float* src = mix + (size_t)c * len;
        if (p->chunking == 0 || start == 0) {
            memcpy(&x[(size_t)c * M + start], src, sizeof(float) * len);  /* :405-406 */
        } else {
            double* q = reflect_pad(src, len, start, start);              /* :442-450 */
            if (!q) { free(x); return ERR_PAD; }
            for (int64_t k = 0; k < M; k++) x[(size_t)c * M + k] = (float)q[k];
            free(q);
        }
    }
    const int G = (int)((M + step - 1) / step);
    int lo, hi;
    sample_window(G, p->sample_first, p->sample_count, &lo, &hi);
    tfc_job J = {p, x, M, step, mask, NULL};
    J.y = (float*)malloc(sizeof(float) * (size_t)G * S * 2 * C);
    int rc = J.y ? parallel_for(lo, hi, p->threads, tfc_chunk, &J) : ERR_MEM;
    double* result = (double*)calloc((size_t)S * 2 * M, sizeof(double));
    double* divider = (double*)calloc((size_t)M, sizeof(double));
    double* w = (double*)malloc(sizeof(double) * C);
    const int fade = C / 10;
    float* window = (float*)malloc(sizeof(float) * C);
    if (p->chunking == 1) {                                               /* :451-456 */
        for (int i = 0; i < C; i++) window[i] = 1.0f;
        if (fade > 0) {
            float* a = (float*)malloc(sizeof(float) * fade);
            torch_linspace(1, 0, fade, a);
            memcpy(window + C - fade, a, sizeof(float) * fade);
            torch_linspace(0, 1, fade, a);
            memcpy(window, a, sizeof(float) * fade);
            free(a);
        }
    }
    for (int g = lo; g < hi && !rc; g++) {
        const int64_t i0 = (int64_t)g * step;
        const int n = (int)(M - i0 < C ? M - i0 : C);
        if (p->chunking == 0) {                                           /* :419-422 */
            if (p->overlap == 0) for (int t = 0; t < n; t++) w[t] = 1.0;
            else np_hanning(n, w);
        } else {                                                          /* :479-484 */
            for (int t = 0; t < C; t++) w[t] = window[t];
            if (i0 == 0) for (int t = 0; t < fade; t++) w[t] = 1.0f;
            else if (i0 + step >= M) for (int t = C - fade; t < C; t++) w[t] = 1.0f;
        }
        for (int k = 0; k < S * 2; k++)
            for (int t = 0; t < n; t++)
                result[(size_t)k * M + i0 + t] += (double)J.y[((size_t)g * S * 2 + k) * C + t] * w[t];
        for (int t = 0; t < n; t++) divider[i0 + t] += w[t];
    }
    for (int k = 0; k < S * 2 && !rc; k++)
        for (int t = 0; t < len; t++) {
            const double v = result[(size_t)k * M + start + t] / divider[start + t];
            out[(size_t)k * len + t] = p->chunking == 0 ? (float)v : (isfinite(v) ? (float)v : 0.0f);
        }
    if (!rc && p->compensate != 1.0f)                                     /* :586-587 */
        for (size_t i = 0; i < (size_t)S * 2 * len; i++) out[i] *= p->compensate;
    if (!rc && p->complement) {                                           /* :588-596 */
        const size_t n = (size_t)2 * len;
        float* rest = out + (size_t)S * n;
        for (size_t i = 0; i < n; i++) {
            float v = mix[i];
            for (int k = 0; k < S; k++) v -= out[(size_t)k * n + i];
            rest[i] = v;
        }
    }
    free(window); free(w); free(divider); free(result); free(J.y); free(x);
    return rc;
}

/* ===================================================================================== */
/* Input conversion: resample_planar (audio.h:17-56)                                      */
/* ===================================================================================== */
long long or_resampled_length(long long n, int src_rate, int dst_rate) {
    if (src_rate == dst_rate) return n;
    return llround((double)n * ((double)dst_rate / src_rate));           /* :20-21 */
}

static double kaiser_i0(double x) {                                       /* :27-31 */
    double s = 1, t = 1;
    for (int k = 1; k < 30; k++) { t *= (x / (2 * k)) * (x / (2 * k)); s += t; }
    return s;
}

int or_resample_planar(const float* in, int n, int ch, int src_rate, int dst_rate, float* out, int* out_n) {
    if (!in || !out || !out_n || n <= 0 || ch < 1 || src_rate <= 0 || dst_rate <= 0) return ERR_ARG;
    if (src_rate == dst_rate) {
        memcpy(out, in, sizeof(float) * (size_t)n * ch);
        *out_n = n;
        return 0;
    }
    const double ratio = (double)dst_rate / src_rate;
    const int m = (int)llround(n * ratio);
    const double cutoff = 0.95 * (ratio < 1.0 ? ratio : 1.0);             /* :22 */
    const int zc = 32;
    const double half = zc / cutoff;
    const double beta = 8.6;
    const double i0b = kaiser_i0(beta);
    const int table_n = 1 << 15;                                          /* :33-42 */
    double* table = (double*)malloc(sizeof(double) * (table_n + 2));
    double* acc = (double*)malloc(sizeof(double) * ch);
    if (!table || !acc) { free(table); free(acc); return ERR_MEM; }
    for (int t = 0; t <= table_n + 1; t++) {
        const double q = (double)t / table_n;
        const double x = (q < 1.0 ? q : 1.0) * half;
        const double r = x / half;
        const double arg = M_PI * x * cutoff;
        const double sinc = arg < 1e-12 ? 1.0 : sin(arg) / arg;
        table[t] = r >= 1 ? 0.0 : sinc * kaiser_i0(beta * sqrt(1 - r * r)) / i0b * cutoff;
    }
    for (int i = 0; i < m; i++) {                                         /* :45-54 */
        const double c = i / ratio;
        const int lo0 = (int)ceil(c - half), hi0 = (int)floor(c + half);
        const int lo = lo0 > 0 ? lo0 : 0, hi = hi0 < n - 1 ? hi0 : n - 1;
        for (int k = 0; k < ch; k++) acc[k] = 0.0;
        for (int j = lo; j <= hi; j++) {
            const double pos = fabs(j - c) / half * table_n;
            const int t = (int)pos;
            if (t >= table_n) continue;
            const double fr = pos - t;
            const double w = table[t] + (table[t + 1] - table[t]) * fr;
            for (int k = 0; k < ch; k++) acc[k] += w * in[(size_t)k * n + j];
        }
        for (int k = 0; k < ch; k++) out[(size_t)k * m + i] = (float)acc[k];
    }
    *out_n = m;
    free(acc); free(table);
    return 0;
}

/* ===================================================================================== */
/* VR: vr_stft / vr_istft / vr_resample / band filters (vr_dsp.h:43-125), spectrum and     */
/* synthesize (vr.cpp:215-269), separate with the network replaced by a given mask          */
/* (vr.cpp:349-377)                                                                         */
/* ===================================================================================== */
int or_vr_stft(const float* wave, int n, int nfft, int hop, double* outd, int* n_frames) {
    if (!wave || !outd || !n_frames || n < 1 || nfft < 2 || hop < 1) return ERR_ARG;
    const int frames = n / hop + 1, F = nfft / 2 + 1;                     /* :44-45 */
    cplx* out = (cplx*)outd;
    double* win = hann_periodic(nfft);
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    int rc = 0;
    for (int c = 0; c < 2 && !rc; c++)
        for (int t = 0; t < frames && !rc; t++) {
            for (int j = 0; j < nfft; j++) {                              /* :50-53 */
                const int k = t * hop + j - nfft / 2;
                buf[j] = k >= 0 && k < n ? wave[(size_t)c * n + k] * win[j] : 0.0;
            }
            rc = or_vrfft(nfft, (double*)buf, 0);
            for (int f = 0; f < F; f++)                                   /* :55-59: complex64 */
                out[((size_t)c * F + f) * frames + t] = (double)(float)creal(buf[f]) + I * (double)(float)cimag(buf[f]);
        }
    *n_frames = frames;
    free(buf); free(win);
    return rc;
}

int or_vr_istft(const double* specd, int frames, int nfft, int hop, float* out) {
    if (!specd || !out || frames < 1 || nfft < 2 || hop < 1) return ERR_ARG;
    const cplx* spec = (const cplx*)specd;
    const int F = nfft / 2 + 1, n = hop * (frames - 1);                    /* :65 */
    const size_t full = (size_t)nfft + n;
    double* win = hann_periodic(nfft);
    double* env = (double*)calloc(full, sizeof(double));
    double* y = (double*)malloc(sizeof(double) * full);
    cplx* buf = (cplx*)malloc(sizeof(cplx) * nfft);
    for (int t = 0; t < frames; t++)                                      /* :69-70 */
        for (int j = 0; j < nfft; j++) env[(size_t)t * hop + j] += win[j] * win[j];
    int rc = 0;
    for (int c = 0; c < 2 && !rc; c++) {
        memset(y, 0, sizeof(double) * full);
        for (int t = 0; t < frames && !rc; t++) {
            for (int f = 0; f < F; f++) buf[f] = spec[((size_t)c * F + f) * frames + t];
            buf[0] = creal(buf[0]);                                       /* :77-79 */
            buf[F - 1] = creal(buf[F - 1]);
            for (int f = 1; f < F - 1; f++) buf[nfft - f] = conj(buf[f]);
            rc = or_vrfft(nfft, (double*)buf, 1);
            for (int j = 0; j < nfft; j++) y[(size_t)t * hop + j] += creal(buf[j]) / nfft * win[j];
        }
        for (int j = 0; j < n; j++) {                                     /* :83-86 */
            const size_t k = (size_t)j + nfft / 2;
            out[(size_t)c * n + j] = env[k] > 1e-11 ? (float)(y[k] / env[k]) : 0.0f;
        }
    }
    free(buf); free(y); free(env); free(win);
    return rc;
}

static int gcd_int(int a, int b) { while (b) { const int t = a % b; a = b; b = t; } return a; }

int or_vr_resampled_length(int n, int src, int dst) {
    if (src == dst) return n;
    const int g = gcd_int(src, dst), up = dst / g, down = src / g;
    return (int)(((int64_t)n * up + down - 1) / down);                    /* :96 */
}

int or_vr_resample(const float* x, int n, int src, int dst, const float* fir, int n_taps, float* y) {
    if (!x || !y || n < 1 || src <= 0 || dst <= 0) return ERR_ARG;
    if (src == dst) { memcpy(y, x, sizeof(float) * 2 * (size_t)n); return 0; }
    if (!fir || n_taps < 1) return ERR_ARG;
    const int g = gcd_int(src, dst), up = dst / g, down = src / g;
    const int out_n = or_vr_resampled_length(n, src, dst);
    const int half = n_taps / 2;
    for (int c = 0; c < 2; c++)                                           /* :99-108 */
        for (int j = 0; j < out_n; j++) {
            const int64_t pos = (int64_t)j * down + half;
            const int64_t lo0 = (pos - n_taps + up) / up;
            const int lo = (int)(lo0 > 0 ? lo0 : 0);
            const int64_t hi0 = pos / up;
            const int hi = (int)(hi0 < n - 1 ? hi0 : n - 1);
            double sum = 0;
            for (int i = lo; i <= hi; i++) sum += (double)x[(size_t)c * n + i] * fir[(size_t)(pos - (int64_t)i * up)];
            y[(size_t)c * out_n + j] = (float)sum;
        }
    return 0;
}

float or_vr_lowpass(int f, int start, int stop) {                       /* :113-118 */
    if (start < 0) return 1;
    if (f < start - 1) return 1;
    if (f >= stop) return 0;
    return 1.0f - (float)(f - start + 1) / (stop - start);
}
float or_vr_highpass(int f, int start, int stop) {                      /* :119-125 */
    if (start <= 0) return 1;
    if (f <= stop + 1) return 0;
    if (f >= start + 1) return 1;
    return (float)(f - stop - 1) / (start - stop);
}

static const or_vr_fir* vr_fir(const or_vr_params* p, int src, int dst) {
    for (int k = 0; k < p->n_firs; k++)
        if (p->firs[k].src == src && p->firs[k].dst == dst) return &p->firs[k];
    return NULL;
}

/* Resample [2][n] from src to dst with the model's FIR (vr.cpp:211-214); *out is malloc'd. */
static int vr_resample_model(const or_vr_params* p, const float* x, int n, int src, int dst, float** out, int* out_n) {
    const int m = or_vr_resampled_length(n, src, dst);
    *out = (float*)malloc(sizeof(float) * 2 * (size_t)m);
    *out_n = m;
    if (src == dst) { memcpy(*out, x, sizeof(float) * 2 * (size_t)n); return 0; }
    const or_vr_fir* f = vr_fir(p, src, dst);
    if (!f) return ERR_ARG;
    return or_vr_resample(x, n, src, dst, f->taps, f->n_taps, *out);
}

int or_vr_n_frames(const or_vr_params* p, int len) {                     /* vr.cpp:219-225 */
    int n = len, rate = p->sample_rate, T = INT32_MAX;
    for (int i = p->n_bands - 1; i >= 0; i--) {
        n = or_vr_resampled_length(n, rate, p->bands[i].sr);
        rate = p->bands[i].sr;
        const int frames = n / p->bands[i].hop + 1;
        if (frames < T) T = frames;
    }
    return T;
}

/* spectrum() (vr.cpp:215-236): spec [2][bins+1][T] complex. */
static int vr_spectrum(const or_vr_params* p, const float* mix, int len, cplx* spec, int T) {
    const int B = p->n_bands, F1 = p->bins + 1;
    cplx** specs = (cplx**)calloc(B, sizeof(cplx*));
    int* frames = (int*)calloc(B, sizeof(int));
    float* wave = (float*)malloc(sizeof(float) * 2 * (size_t)len);
    memcpy(wave, mix, sizeof(float) * 2 * (size_t)len);
    int n = len, rate = p->sample_rate, rc = 0;
    for (int i = B - 1; i >= 0 && !rc; i--) {
        float* w2 = NULL;
        int n2 = 0;
        rc = vr_resample_model(p, wave, n, rate, p->bands[i].sr, &w2, &n2);
        free(wave);
        wave = w2; n = n2; rate = p->bands[i].sr;
        const int F = p->bands[i].nfft / 2 + 1;
        specs[i] = (cplx*)malloc(sizeof(cplx) * 2 * (size_t)F * (n / p->bands[i].hop + 1));
        if (!rc) rc = or_vr_stft(wave, n, p->bands[i].nfft, p->bands[i].hop, (double*)specs[i], &frames[i]);
    }
    memset(spec, 0, sizeof(cplx) * 2 * (size_t)F1 * T);
    int off = 0;
    for (int i = 0; i < B && !rc; i++) {                                  /* :228-235 */
        const or_vr_band* b = &p->bands[i];
        const int F = b->nfft / 2 + 1;
        for (int c = 0; c < 2; c++)
            for (int f = b->start; f < b->stop; f++)
                for (int t = 0; t < T; t++)
                    spec[((size_t)c * F1 + off + f - b->start) * T + t] = specs[i][((size_t)c * F + f) * frames[i] + t];
        off += b->stop - b->start;
    }
    if (p->pre_start > 0 && !rc)                                          /* :236-239 */
        for (int c = 0; c < 2; c++)
            for (int f = 0; f <= p->bins; f++)
                for (int t = 0; t < T; t++) spec[((size_t)c * F1 + f) * T + t] *= or_vr_lowpass(f, p->pre_start, p->pre_stop);
    for (int i = 0; i < B; i++) free(specs[i]);
    free(specs); free(frames); free(wave);
    return rc;
}

/* synthesize() (vr.cpp:241-269): out [2][len]. */
static int vr_synthesize(const or_vr_params* p, const cplx* spec, int T, int len, float* out) {
    const int B = p->n_bands, F1 = p->bins + 1;
    float* wave = NULL;
    int off = 0, n = 0, rc = 0;
    for (int i = 0; i < B && !rc; i++) {
        const or_vr_band* b = &p->bands[i];
        const int F = b->nfft / 2 + 1;
        cplx* part = (cplx*)calloc((size_t)2 * F * T, sizeof(cplx));
        for (int c = 0; c < 2; c++)
            for (int f = b->start; f < b->stop; f++) {
                const float gain = or_vr_highpass(f, b->hp_start, b->hp_stop - 1) *
                                   (i + 1 == B ? 1 : or_vr_lowpass(f, b->lp_start, b->lp_stop));
                for (int t = 0; t < T; t++)
                    part[((size_t)c * F + f) * T + t] = spec[((size_t)c * F1 + off + f - b->start) * T + t] * (double)gain;
            }
        off += b->stop - b->start;
        const int bn = b->hop * (T - 1);
        float* add = (float*)malloc(sizeof(float) * 2 * (size_t)bn);
        rc = or_vr_istft((const double*)part, T, b->nfft, b->hop, add);
        free(part);
        if (!wave) { wave = add; n = bn; }
        else {
            if (n != bn) rc = ERR_ARG;                                    /* "bands do not align" */
            for (size_t k = 0; k < 2 * (size_t)n && !rc; k++) wave[k] += add[k];
            free(add);
        }
        if (i + 1 < B && !rc) {
            float* w2 = NULL;
            int n2 = 0;
            rc = vr_resample_model(p, wave, n, b->sr, p->bands[i + 1].sr, &w2, &n2);
            free(wave);
            wave = w2; n = n2;
        }
    }
    for (int c = 0; c < 2 && !rc; c++)
        for (int j = 0; j < len; j++) out[(size_t)c * len + j] = j < n ? wave[(size_t)c * n + j] : 0.0f;
    free(wave);
    return rc;
}

int or_vr_separate(const or_vr_params* p, const float* mix, int len, const float* mask, float* out) {
    if (!p || !mix || !mask || !out || len <= 0 || p->n_bands < 1) return ERR_ARG;
    const int T = or_vr_n_frames(p, len), F1 = p->bins + 1;
    const size_t K = (size_t)2 * F1 * T;
    cplx* spec = (cplx*)malloc(sizeof(cplx) * K);
    cplx* z = (cplx*)malloc(sizeof(cplx) * K);
    int rc = vr_spectrum(p, mix, len, spec, T);
    float peak = 0;                                                       /* :357-360 */
    for (size_t k = 0; k < K && !rc; k++) {
        const float m = (float)cabs(spec[k]);
        if (m > peak) peak = m;
    }
    if (!rc && peak == 0) {
        memset(out, 0, sizeof(float) * 4 * (size_t)len);
    } else {
        for (int s = 0; s < 2 && !rc; s++) {                              /* :370-376 */
            for (size_t k = 0; k < K; k++) z[k] = spec[k] * (s == 0 ? mask[k] : 1 - mask[k]);
            rc = vr_synthesize(p, z, T, len, out + (size_t)s * 2 * len);
        }
    }
    free(z); free(spec);
    return rc;
}

