// emulate.cpp -- TEST INFRASTRUCTURE: a host replay of the combine kernels' index arithmetic.
//
// Builds with the library's own host scheduler (stems.cpp_b200/csrc/plan.cu, compiled for the
// host) and stubs for everything that would touch a GPU. launch_plan runs unchanged; the
// launch_combine stub receives exactly the CombineParams a GPU launch would, with the plan's
// tables (chunks, groups, weights) in host memory, and replays the index arithmetic of
// kernels.cu's combine_kernel4 (one or two stereo stems) or combine_kernel (the rest) for every
// output sample the launch writes. It checks:
//   1. every chunk whose output reaches a sample is visited by the kernel's chunk range, and
//      every visited chunk that passes the sample's guard does reach it;
//   2. wherever a loaded value is used, each clamp of combine_kernel4 (uc, tc, uc2, and the
//      complement's min(s, nv - 1)) leaves its index unchanged, and every address lies in its
//      buffer (weights, Y, Tr, mix, out);
//   3. for the loads whose value the guard discards, the address an unguarded load would have
//      used, and whether it leaves its buffer: the candidates for the fault of the first,
//      unclamped combine_kernel4.
// Output: one line per plan, "name violations=N oob_unguarded_W=.. Y=.. Tr=.. mix=.. first=..."
#include "plan.h"
#include "kernels.h"

#include <cstdio>
#include <cstdlib>
#include <functional>
#include <string>
#include <vector>

namespace stg {

// ---- stubs for the device side (values as kernels.cu and split.cu give them) ------------
static int g_slots = 444;
bool fused_supported(int n) { return n == 2048 || n == 4096 || n == 7680; }
bool fused_pair(int, int, int) { return false; }
std::vector<int> fused_pair_radices(int) { return {}; }
int fused_pair_slots() { return g_slots; }
int fused_max_hop(int n) { return n == 2048 ? 512 : (n == 4096 || n == 7680) ? 1024 : 0; }
bool split_supported(int n) {
    return n == 320 || n == 512 || n == 640 || n == 960 || n == 1024 || n == 2048 || n == 4096 || n == 7680;
}
int split_max_hop(int n) { return split_supported(n) ? n / 2 : 0; }
int fused_resident_ctas(int, int) { return g_slots; }
int back_resident_ctas(int) { return g_slots; }
int split_resident_ctas(int, bool) { return g_slots; }
std::vector<int> fused_radices(int) { return {}; }
std::vector<int> fused_fwd_radices(int) { return {}; }
size_t mono_scratch_doubles() { return 1026; }
cudaError_t launch_fused(int, const FusedParams&, cudaStream_t) { return cudaSuccess; }
cudaError_t launch_front(const SplitParams&, cudaStream_t) { return cudaSuccess; }
cudaError_t launch_back(const SplitParams&, cudaStream_t) { return cudaSuccess; }
cudaError_t launch_mask_transpose(const float*, int64_t, int, int, int, int, int, float4*, int64_t, cudaStream_t, int) {
    return cudaSuccess;
}
cudaError_t launch_mono_norm(const float*, int64_t, int, double*, float*, cudaStream_t) { return cudaSuccess; }
cudaError_t launch_cac_finish(const double2*, int, int, double, double2*, cudaStream_t) { return cudaSuccess; }

// ---- the replay ---------------------------------------------------------------------------
struct Sizes {
    int64_t W = 0, Y = 0, Tr = 0, mix = 0, out = 0;   // floats
};
static Sizes g_sz;
// base addresses of the buffers the replay pretends the launch got (never dereferenced)
static float* const kY = reinterpret_cast<float*>(0x100000000000ull);
static float* const kTr = reinterpret_cast<float*>(0x200000000000ull);
static float* const kMix = reinterpret_cast<float*>(0x300000000000ull);
static float* const kOut = reinterpret_cast<float*>(0x400000000000ull);

struct Report {
    long violations = 0, oob_w = 0, oob_y = 0, oob_tr = 0, oob_mix = 0, launches = 0, vec = 0;
    std::string first;
    void bad(const std::string& what) {
        if (violations++ == 0) first = what;
    }
};
static Report g_rep;

static bool in(int64_t i, int64_t n) { return i >= 0 && i < n; }

// combine_kernel4: V = 4 samples per thread, stereo rows (SC = 2 or 4)
static void replay4(const CombineParams& p) {
    const int V = 4, SC = p.S * p.C;
    const FrameGeom& G = p.g;
    const int step = (int)p.step_out, span = p.K * G.hop, ov = G.n_fft - G.hop;
    for (int64_t il = p.i_begin; il < p.i_end; il += V) {
        const int i0 = (int)il;
        const int nv = (int)std::min<int64_t>(V, p.i_end - il);
        for (int gi = 0; gi < p.n_groups; gi++) {
            const ChunkGroup grp = p.groups[gi];
            const int P0 = i0 + grp.out_shift;
            const int out00 = (int)p.chunks[grp.c0].out0;
            const int n = grp.c1 - grp.c0;
            const int ghi = std::min((P0 + V - 1 - out00) / step, n - 1);
            const int glo = std::max((P0 - out00 - (int)p.max_out_len) / step, 0);
            // 1. completeness: the chunks that reach each sample, against the visited range
            for (int s = 0; s < nv; s++)
                for (int g = grp.c0; g < grp.c1; g++) {
                    const ChunkDesc& d = p.chunks[g];
                    const int u = P0 + s - (int)d.out0;
                    const bool reaches = u >= 0 && u < d.out_len;
                    const int gl = g - grp.c0;
                    const bool visited = gl >= glo && gl <= ghi + 1 && gl < n;
                    if (reaches && !visited) g_rep.bad("chunk " + std::to_string(g) + " reaches sample " +
                                                       std::to_string(i0 + s) + " but is not visited");
                }
            for (int gl = glo; gl <= ghi + 1 && gl < n; gl++) {
                const int g = grp.c0 + gl;
                const ChunkDesc& d = p.chunks[g];
                const int u0 = P0 - (int)d.out0, olen = d.out_len;
                if (olen <= 0 || u0 + V <= 0 || u0 >= olen) continue;
                const int64_t ybase = (int64_t)g * p.y_chunk_stride, tbase = (int64_t)g * p.tr_chunk_stride;
                const int j0 = d.y_off + u0;
                const int q0 = j0 + G.out_offset - G.first_pos;
                const int tau0 = q0 / span, uu0 = q0 - tau0 * span;
                // the vector path: when the kernel takes it, its four samples must be exactly the
                // ones the per-sample loop would use (all inside the chunk, none with a Tr
                // partial), and its 16-byte loads aligned and inside the weight table and Y
                const bool no_tr = q0 >= 0 && (tau0 < 1 || uu0 >= ov) && uu0 + V <= span;
                if (nv == V && u0 >= 0 && u0 + V <= olen && no_tr && ((d.w_off + u0) & 3) == 0 && (j0 & 1) == 0 &&
                    (G.Lout & 1) == 0) {
                    g_rep.vec++;
                    for (int s = 0; s < V; s++) {
                        const int tau = tau0, uu = uu0 + s;
                        if (tau >= 1 && tau < p.n_tiles && uu < ov) g_rep.bad("vector path over a Tr partial");
                    }
                    const int64_t w0 = d.w_off + (int64_t)u0;
                    if ((w0 & 3) || !in(w0, g_sz.W) || !in(w0 + 3, g_sz.W)) g_rep.bad("vector weight load outside the table");
                    for (int st = 0; st < SC / 2; st++) {
                        const int64_t y0 = ybase + 2 * ((int64_t)st * G.Lout + j0);
                        if ((y0 & 3) || !in(y0, g_sz.Y) || !in(y0 + 7, g_sz.Y)) g_rep.bad("vector Y load misaligned or outside");
                    }
                    continue;
                }
                for (int s = 0; s < V; s++) {
                    const int u = u0 + s;
                    int tau, uu;
                    if (q0 >= 0) {
                        tau = tau0;
                        uu = uu0 + s;
                        if (uu >= span) { uu -= span; tau++; }
                    } else {
                        tau = (q0 + s) / span;
                        uu = q0 + s - tau * span;
                    }
                    const bool used = !(s >= nv || u < 0 || u >= olen);
                    const int uc = std::min(std::max(u, 0), olen - 1);
                    const bool has_tr = tau >= 1 && tau < p.n_tiles && uu < ov;
                    const int tc = std::min(std::max(tau, 1), p.n_tiles) - 1, uc2 = std::min(std::max(uu, 0), ov - 1);
                    if (used) {
                        if (uc != u) g_rep.bad("uc clamps a used index");
                        if (!in(d.w_off + (int64_t)u, g_sz.W)) g_rep.bad("weight index outside the table");
                        for (int st = 0; st < SC / 2; st++) {
                            const int64_t yi = ybase + 2 * ((int64_t)d.y_off + uc + (int64_t)st * G.Lout);
                            if (!in(yi, g_sz.Y) || !in(yi + 1, g_sz.Y)) g_rep.bad("Y index outside the buffer");
                            if (has_tr) {
                                if (tc != tau - 1 || uc2 != uu) g_rep.bad("tc / uc2 clamp a used index");
                                const int64_t ti = tbase + (int64_t)tc * SC * ov + 2 * ((int64_t)uc2 + (int64_t)st * ov);
                                if (!in(ti, g_sz.Tr) || !in(ti + 1, g_sz.Tr)) g_rep.bad("Tr index outside the buffer");
                            }
                        }
                    } else {
                        // the addresses an unguarded load would have read
                        if (!in(d.w_off + (int64_t)u, g_sz.W)) g_rep.oob_w++;
                        const int64_t yi = ybase + 2 * ((int64_t)d.y_off + u);
                        if (!in(yi, g_sz.Y)) g_rep.oob_y++;
                        if (tau >= 1 && tau < p.n_tiles && uu < ov) {
                            const int64_t ti = tbase + (int64_t)(tau - 1) * SC * ov + 2 * (int64_t)uu;
                            if (!in(ti, g_sz.Tr)) g_rep.oob_tr++;
                        }
                    }
                }
            }
        }
        for (int s = 0; s < V; s++) {
            for (int k = 0; k < SC + (p.complement ? 2 : 0); k++)
                if (s < nv && !in((int64_t)k * p.len + i0 + s, g_sz.out)) g_rep.bad("out index outside the buffer");
            if (p.complement)
                for (int c = 0; c < 2; c++) {
                    const int64_t mi = (int64_t)c * p.len + i0 + std::min(s, nv - 1);
                    if (s < nv && std::min(s, nv - 1) != s) g_rep.bad("complement clamp changes a used index");
                    if (!in(mi, g_sz.mix)) g_rep.bad("mix index outside the buffer");
                    const int64_t raw = (int64_t)c * p.len + i0 + s;   // unguarded
                    if (s >= nv && !in(raw, g_sz.mix)) g_rep.oob_mix++;
                }
        }
    }
}

// combine_kernel: one sample per thread, any S * C
static void replay1(const CombineParams& p) {
    const int SC = p.S * p.C;
    const FrameGeom& G = p.g;
    const int step = (int)p.step_out, span = p.K * G.hop, ov = G.n_fft - G.hop;
    for (int64_t i = p.i_begin; i < p.i_end; i++) {
        for (int gi = 0; gi < p.n_groups; gi++) {
            const ChunkGroup grp = p.groups[gi];
            const int P = (int)i + grp.out_shift;
            const int out00 = (int)p.chunks[grp.c0].out0;
            const int n = grp.c1 - grp.c0;
            const int ghi = std::min((P - out00) / step, n - 1);
            const int glo = std::max((P - out00 - (int)p.max_out_len) / step, 0);
            for (int g = grp.c0; g < grp.c1; g++) {
                const ChunkDesc& d = p.chunks[g];
                const int u = P - (int)d.out0;
                const int gl = g - grp.c0;
                if (u >= 0 && u < d.out_len && !(gl >= glo && gl <= ghi + 1))
                    g_rep.bad("chunk " + std::to_string(g) + " reaches sample " + std::to_string(i) + " but is not visited");
            }
            for (int gl = glo; gl <= ghi + 1 && gl < n; gl++) {
                const int g = grp.c0 + gl;
                const ChunkDesc& d = p.chunks[g];
                const int u = P - (int)d.out0;
                if (u < 0 || u >= d.out_len) continue;
                if (!in(d.w_off + (int64_t)u, g_sz.W)) g_rep.bad("weight index outside the table");
                const int j = d.y_off + u;
                const int64_t yb = (int64_t)g * p.y_chunk_stride + (int64_t)j * p.C;
                const int q = j + G.out_offset - G.first_pos;
                const int tau = q / span, uu = q - tau * span;
                for (int k = 0; k < SC; k++) {
                    const int64_t yi = yb + (int64_t)(k / p.C) * p.C * G.Lout + k % p.C;
                    if (!in(yi, g_sz.Y)) g_rep.bad("Y index outside the buffer");
                    if (tau >= 1 && tau < p.n_tiles && uu < ov) {
                        const int64_t ti = (int64_t)g * p.tr_chunk_stride + (int64_t)(tau - 1) * SC * ov +
                                           (int64_t)uu * p.C + (int64_t)(k / p.C) * p.C * ov + k % p.C;
                        if (!in(ti, g_sz.Tr)) g_rep.bad("Tr index outside the buffer");
                    }
                }
            }
        }
        for (int k = 0; k < SC + (p.complement ? p.C : 0); k++)
            if (!in((int64_t)k * p.len + i, g_sz.out)) g_rep.bad("out index outside the buffer");
    }
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t) {
    g_rep.launches++;
    if (p.Y != kY || p.Tr != kTr || p.mix == nullptr || p.out != kOut) g_rep.bad("unexpected buffer bases");
    if (p.C == 2 && p.S <= 2) replay4(p);
    else replay1(p);
    return cudaSuccess;
}

} // namespace stg

using namespace stg;

// One plan: build it with the library's scheduler, point its tables at host copies, run
// launch_plan over [b, e) (e < 0: the whole track), replay every combine launch.
static void run(const std::string& name, const std::function<void(HostPlan&)>& build, int64_t b = 0, int64_t e = -1) {
    for (int slots : {148, 296, 444, 1184}) {
        g_slots = slots;
        HostPlan H;
        build(H);
        PlanDevice D;
        D.chunks = H.chunks.data();
        D.groups = H.groups.data();
        D.W = H.W.data();
        D.env = H.env.data();
        D.Y = kY;
        D.Tr = kTr;
        static double mono[2048];
        static double2 cac[1 << 16];
        static float4 mt[16];
        D.mono = mono;
        D.mixn = kMix;
        D.cac_part = cac;
        D.cac_stats = cac;
        D.mask_t = mt;
        D.zspec = mt;
        if (!H.bag.empty()) { D.bag = H.bag.data(); D.bag_tot = H.bag_tot.data(); }
        g_sz.W = (int64_t)H.W.size();
        g_sz.Y = H.y_chunk_stride * (int64_t)H.chunks.size();
        g_sz.Tr = H.tr_chunk_stride * (int64_t)H.chunks.size();
        g_sz.mix = (int64_t)H.C * H.len;
        g_sz.out = H.out_floats();
        g_rep = Report{};
        static float fake_mask[4];
        try {
            launch_plan(H, D, kMix, fake_mask, kOut, nullptr, nullptr, nullptr, b, e);
        } catch (const std::exception& x) {
            g_rep.bad(std::string("launch_plan: ") + x.what());
        }
        std::printf("%s slots=%d K=%d chunks=%zu launches=%ld violations=%ld oob_unguarded_W=%ld Y=%ld Tr=%ld mix=%ld vec=%ld first=%s\n",
                    name.c_str(), slots, H.K, H.chunks.size(), g_rep.launches, g_rep.violations, g_rep.oob_w,
                    g_rep.oob_y, g_rep.oob_tr, g_rep.oob_mix, g_rep.vec, g_rep.first.empty() ? "-" : g_rep.first.c_str());
    }
}

// The band tables of the benchmark's Mel and BS RoFormers come from the test driver (argv).
static std::vector<int32_t> read_ints(const char* path) {
    std::vector<int32_t> v;
    FILE* f = std::fopen(path, "rb");
    if (!f) { std::perror(path); std::exit(2); }
    int32_t x;
    while (std::fread(&x, sizeof x, 1, f) == 1) v.push_back(x);
    std::fclose(f);
    return v;
}

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: emulate mel_sizes mel_freqs bs_sizes bs_freqs\n");
        return 2;
    }
    const std::vector<int32_t> ms = read_ints(argv[1]), mf = read_ints(argv[2]), bs = read_ints(argv[3]),
                               bf = read_ints(argv[4]);
    auto rf = [&](bool mel, int chunk, int nov, int64_t len, bool zdc, bool comp, int shifts, int C = 2) {
        return [=, &ms, &mf, &bs, &bf](HostPlan& H) {
            stg_roformer_config c{};
            c.size = sizeof c;
            c.n_channels = C; c.n_stems = 1; c.n_fft = 2048; c.hop = 441; c.zero_dc = zdc; c.chunk = chunk;
            c.num_overlap = nov; c.overlap = -1.0f;
            c.n_bands = (int)(mel ? ms.size() : bs.size());
            c.band_sizes = mel ? ms.data() : bs.data();
            c.band_freqs = mel ? mf.data() : bf.data();
            c.complement = comp; c.shifts = shifts; c.seed = 9; c.sample_rate = 44100;
            H.len = len;
            build_roformer(H, c, len);
        };
    };
    auto ht = [&](int seg, int64_t len, int S, float ov, int C, int shifts, int models) {
        return [=](HostPlan& H) {
            stg_htdemucs_config c{};
            c.size = sizeof c;
            c.n_channels = C; c.n_sources = S; c.segment = seg; c.overlap = ov; c.mono_norm = 1; c.cac_norm = 1;
            c.shifts = shifts; c.seed = 5; c.sample_rate = 44100; c.n_models = models;
            H.len = len;
            build_htdemucs(H, c, len);
        };
    };
    auto tfc = [&](int dim_t, int chunking, float ov, int64_t len, bool comp, int S = 1) {
        return [=](HostPlan& H) {
            stg_tfc_config c{};
            c.size = sizeof c;
            c.n_stems = S; c.n_fft = 7680; c.hop = 1024; c.dim_f = 3072; c.dim_t = dim_t; c.zero_bins = 3;
            c.chunking = chunking; c.num_overlap = 4; c.overlap = ov; c.compensate = 1.009f; c.complement = comp;
            H.len = len;
            build_tfc(H, c, len);
        };
    };
    // the GPU parity tests' plans (tests/test_gpu_parity.py, test_gpu_contracts.py)
    run("rf_mel_ov4_pad", rf(true, 441 * 40, 4, 441 * 80 + 1234, true, false, 0));
    run("rf_bs_ov2_complement", rf(false, 441 * 40, 2, 441 * 100 + 17, true, true, 0));
    run("rf_mel_short_reflect_tail", rf(true, 441 * 40, 2, 441 * 31, false, false, 0));
    run("rf_bs_short_zero_tail", rf(false, 441 * 40, 2, 441 * 15, false, false, 0));
    run("rf_mel_no_border_pad", rf(true, 441 * 40, 4, 441 * 50, true, false, 0));
    run("rf_shifts_long", rf(false, 441 * 40, 2, 441 * 100 + 33, true, true, 2));
    run("rf_shifts_15000", rf(false, 441 * 40, 2, 15000, true, true, 2));
    run("rf_mono_complement", rf(true, 441 * 40, 2, 441 * 60 + 5, true, true, 0, 1));
    run("rf_part_mid", rf(false, 441 * 40, 2, 441 * 100 + 17, true, true, 0), 1001, 30003);
    run("rf_part_odd", rf(true, 441 * 40, 4, 441 * 80 + 1234, true, false, 0), 3, 441 * 80 + 1233);
    run("ht_seg24k_4src", ht(1024 * 24, 60000, 4, -1.0f, 2, 0, 1));
    run("ht_seg24k_short", ht(1024 * 24, 9000, 2, -1.0f, 2, 0, 1));
    run("ht_seg_odd_ov05", ht(1024 * 20 + 333, 51001, 4, 0.5f, 2, 0, 1));
    run("ht_six_src", ht(1024 * 24, 70001, 6, -1.0f, 2, 0, 1));
    run("ht_one_channel", ht(1024 * 24, 60000, 4, -1.0f, 1, 0, 1));
    run("ht_two_src_stereo", ht(1024 * 24, 60000, 2, -1.0f, 2, 0, 1));
    run("ht_shifts3", ht(1024 * 24, 60000, 4, -1.0f, 2, 3, 1));
    run("ht_bag3_shifts2", ht(1024 * 24, 60000, 4, -1.0f, 2, 2, 3));
    run("tfc_uvr_dt32_ov05", tfc(32, 0, 0.5f, 70000, true));
    run("tfc_uvr_dt32_default", tfc(32, 0, -1.0f, 50000, false));
    run("tfc_msst_dt32", tfc(32, 1, -1.0f, 90001, true));
    run("tfc_two_stems", tfc(32, 0, 0.5f, 70000, true, 2));
    // the five BASELINE configurations
    run("cfg0_htdemucs_20s", ht(343980, 20 * 44100, 4, -1.0f, 2, 0, 1));
    run("cfg1_mel_roformer_60s", rf(true, 352800, 4, 60 * 44100, false, false, 0));
    run("cfg2_bs_roformer_180s", rf(false, 352800, 2, 180 * 44100, true, false, 0));
    run("cfg3_tfc_180s", tfc(256, 0, 0.5f, 180 * 44100, false));
    run("cfg4_htdemucs_240s", ht(343980, 240 * 44100, 4, -1.0f, 2, 0, 1));
    return 0;
}
