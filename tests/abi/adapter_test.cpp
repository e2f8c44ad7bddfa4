// adapter_test.cpp -- include/stems_gpu.hpp from a C++ host (TEST INFRASTRUCTURE).
//
//   adapter_test            no GPU: the header compiles C++17-clean, errors map to exceptions
//   adapter_test CASE_DIR   one RoFormer separation through stems_gpu::RoFormer::separate,
//                           compared with CASE_DIR/want.f32, then a cancelled one
//
// The separation part is the code INTEGRATION.md shows for RoFormer::separate.
#include "stems_gpu.hpp"

#include <cmath>
#include <cstdio>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

static int failures = 0;
static void check(bool ok, const char* what) {
    std::printf("  %-66s %s\n", what, ok ? "ok" : "FAIL");
    if (!ok) failures++;
}

template <class T> static std::vector<T> read(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> b((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<T> v(b.size() / sizeof(T));
    std::copy(b.begin(), b.begin() + v.size() * sizeof(T), reinterpret_cast<char*>(v.data()));
    return v;
}

int main(int argc, char** argv) {
    std::printf("exceptions\n");
    try {
        throw stems_gpu::Cancelled("cancelled");
    } catch (const stems_gpu::Error& e) {
        check(e.code() == STG_CANCELLED, "Cancelled is an Error with STG_CANCELLED");
    }
    if (argc < 2) {
        if (stg_device_count() <= 0) {
            try {
                stems_gpu::Engine eng(0);
                check(false, "Engine(0) without a GPU throws");
            } catch (const stems_gpu::Error& e) {
                check(e.code() != STG_OK, "Engine(0) without a GPU throws Error with its status");
            }
        }
        std::printf("%s\n", failures ? "FAILED" : "all passed");
        return failures ? 1 : 0;
    }
    const std::string dir = argv[1];
    std::ifstream cf(dir + "/case.txt");
    long long n = 0;
    int chunk = 0, nov = 0, n_bands = 0;
    cf >> n >> chunk >> nov >> n_bands;
    const std::vector<int32_t> sizes = read<int32_t>(dir + "/sizes.i32"), freqs = read<int32_t>(dir + "/freqs.i32");
    const std::vector<float> mix = read<float>(dir + "/mix.f32"), masks = read<float>(dir + "/mask.f32"),
                             want = read<float>(dir + "/want.f32");

    std::printf("RoFormer::separate through the adapter\n");
    // -- as INTEGRATION.md: once per model, the configuration the GGUF gives --
    stems_gpu::Engine eng(0);
    stg_roformer_config model{};
    model.size = sizeof model;
    model.n_channels = 2;  model.n_stems = 1;
    model.n_fft = 2048;    model.hop = 441;
    model.chunk = chunk;   model.num_overlap = nov;
    model.n_bands = n_bands;
    model.band_sizes = sizes.data();  model.band_freqs = freqs.data();
    model.sample_rate = 44100;
    stems_gpu::RoFormer roformer(eng, model);
    // -- per request: the reference's SeparateOptions --
    stems_gpu::SeparateOptions opt;
    int reports = 0, last_done = 0, last_total = 0;
    opt.progress = [&](int done, int total) { reports++; last_done = done; last_total = total; };
    check(roformer.mask_floats((int)n, opt) == (int64_t)masks.size(), "mask_floats matches the network output size");
    const std::vector<float> out = roformer.separate(mix.data(), (int)n, opt, masks.data());
    // -- end of the INTEGRATION.md code --
    check(out.size() == want.size(), "the result is [1][2][n]");
    double worst = 0, scale = 0;
    for (size_t i = 0; i < out.size() && i < want.size(); i++) {
        worst = std::fmax(worst, std::fabs((double)out[i] - (double)want[i]));
        scale = std::fmax(scale, std::fabs((double)want[i]));
    }
    std::printf("  max |got - oracle| / max |oracle| = %.3e\n", worst / scale);
    check(worst / scale <= 1e-5, "the result matches the oracle within 1e-5");
    check(reports > 1 && last_done == last_total, "progress per chunk, ending at (total, total)");
    stems_gpu::SeparateOptions stop;
    int polls = 0;
    stop.should_cancel = [&] { return ++polls > 1; };
    bool cancelled = false;
    try {
        roformer.separate(mix.data(), (int)n, stop, masks.data());
    } catch (const stems_gpu::Cancelled&) {
        cancelled = true;
    }
    check(cancelled && polls == 2, "should_cancel true before the second chunk throws Cancelled");
    std::printf("%s\n", failures ? "FAILED" : "all passed");
    return failures ? 1 : 0;
}
