/* abi_test.c -- the stems_gpu_v1.h contract as a C host sees it (TEST INFRASTRUCTURE).
 *
 *   abi_test LIBRARY                    no GPU: symbols, statuses, argument checks
 *   abi_test LIBRARY CASE_DIR           also one RoFormer separation from host buffers,
 *                                       compared with CASE_DIR/want.f32 (the CPU oracle's)
 *
 * Like the reference's tests/abi_test.c, the library is loaded at run time with dlopen and
 * every entry point is resolved with dlsym, as a plug-in loads it; nothing links against it.
 * Pure C, so the public header has to stay C-clean. CASE_DIR holds case.txt (n_samples chunk
 * num_overlap n_bands), sizes.i32, freqs.i32, mix.f32 [2][n], mask.f32 and want.f32 [1][2][n].
 */
#include "stems_gpu_v1.h"

#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int failures = 0;

static void check(int ok, const char* what) {
    printf("  %-66s %s\n", what, ok ? "ok" : "FAIL");
    if (!ok) failures++;
}

static void* lib;
static void* sym(const char* name) {
    void* p = dlsym(lib, name);
    if (!p) {
        printf("  missing symbol %s\n", name);
        failures++;
    }
    return p;
}

static void* read_file(const char* dir, const char* name, size_t* bytes) {
    char path[4096];
    snprintf(path, sizeof path, "%s/%s", dir, name);
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void* p = malloc((size_t)n);
    if (p && fread(p, 1, (size_t)n, f) != (size_t)n) { free(p); p = NULL; }
    fclose(f);
    if (bytes) *bytes = (size_t)n;
    return p;
}

typedef const char* (*version_fn)(void);
typedef int (*device_count_fn)(void);
typedef stg_status (*engine_create_fn)(int, stg_engine**);
typedef void (*engine_destroy_fn)(stg_engine*);
typedef const char* (*last_error_fn)(const stg_engine*);
typedef stg_status (*plan_roformer_fn)(stg_engine*, const stg_roformer_config*, int64_t, stg_plan**);
typedef stg_status (*plan_htdemucs_fn)(stg_engine*, const stg_htdemucs_config*, int64_t, stg_plan**);
typedef void (*plan_destroy_fn)(stg_plan*);
typedef stg_status (*plan_info_fn)(const stg_plan*, stg_plan_info*);
typedef stg_status (*separate_fn)(stg_plan*, const float*, const float*, float*, void*);
typedef stg_status (*separate_host_ex_fn)(stg_plan*, const float*, const float*, float*, void*, const stg_run_options*);
typedef stg_status (*model_open_fn)(const char*, stg_model**, char*, size_t);
typedef int64_t (*resampled_length_fn)(int64_t, int32_t, int32_t);
typedef stg_status (*noalloc_fn)(int, const stg_roformer_config*, int64_t, const float*, const float*, float*, void*,
                                 char*, size_t);

static int progress_calls = 0, last_done = 0, last_total = 0;
static void on_progress(void* user, int32_t done, int32_t total) {
    (void)user;
    progress_calls++;
    last_done = done;
    last_total = total;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: abi_test LIBRARY [CASE_DIR]\n");
        return 2;
    }
    lib = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        printf("FAIL: dlopen(%s): %s\n", argv[1], dlerror());
        return 1;
    }
    const char* case_dir = argc > 2 ? argv[2] : NULL;

    printf("entry points\n");
    version_fn version = (version_fn)sym("stg_version");
    device_count_fn device_count = (device_count_fn)sym("stg_device_count");
    engine_create_fn engine_create = (engine_create_fn)sym("stg_engine_create");
    engine_destroy_fn engine_destroy = (engine_destroy_fn)sym("stg_engine_destroy");
    last_error_fn last_error = (last_error_fn)sym("stg_engine_last_error");
    plan_roformer_fn plan_roformer = (plan_roformer_fn)sym("stg_plan_roformer");
    plan_htdemucs_fn plan_htdemucs = (plan_htdemucs_fn)sym("stg_plan_htdemucs");
    plan_destroy_fn plan_destroy = (plan_destroy_fn)sym("stg_plan_destroy");
    plan_info_fn plan_info = (plan_info_fn)sym("stg_plan_get_info");
    separate_fn separate = (separate_fn)sym("stg_separate");
    separate_host_ex_fn separate_host_ex = (separate_host_ex_fn)sym("stg_separate_host_ex");
    model_open_fn model_open = (model_open_fn)sym("stg_model_open");
    resampled_length_fn resampled_length = (resampled_length_fn)sym("stg_resampled_length");
    noalloc_fn noalloc = (noalloc_fn)sym("stg_separate_roformer_noalloc");
    if (failures) return 1;

    const char* v = version();
    printf("  version: %s\n", v ? v : "(null)");
    check(v && strstr(v, "abi 1") != NULL, "stg_version names ABI 1");

    printf("argument checks (no GPU work)\n");
    check(engine_create(0, NULL) == STG_INVALID_ARGUMENT, "engine_create(NULL out) is INVALID_ARGUMENT");
    stg_plan* plan = (stg_plan*)1;
    check(plan_roformer(NULL, NULL, 1000, &plan) == STG_INVALID_ARGUMENT && plan == NULL,
          "plan_roformer(NULL engine) is INVALID_ARGUMENT, *out cleared");
    check(plan_htdemucs(NULL, NULL, 1000, NULL) == STG_INVALID_ARGUMENT, "plan_htdemucs(NULL out) is INVALID_ARGUMENT");
    check(plan_info(NULL, NULL) == STG_INVALID_ARGUMENT, "plan_get_info(NULL) is INVALID_ARGUMENT");
    check(separate(NULL, NULL, NULL, NULL, NULL) == STG_INVALID_ARGUMENT, "separate(NULL plan) is INVALID_ARGUMENT");
    check(separate_host_ex(NULL, NULL, NULL, NULL, NULL, NULL) == STG_INVALID_ARGUMENT,
          "separate_host_ex(NULL plan) is INVALID_ARGUMENT");
    plan_destroy(NULL);
    engine_destroy(NULL);
    check(1, "destroy(NULL) is a no-op");
    check(strcmp(last_error(NULL), "") == 0, "last_error(NULL) is an empty string");
    check(resampled_length(48000, 48000, 44100) == 44100 && resampled_length(-1, 1, 1) == -1,
          "resampled_length (llround, negative length rejected)");
    char msg[512] = "";
    stg_model* model = NULL;
    check(model_open("/nonexistent/model.gguf", &model, msg, sizeof msg) == STG_IO_ERROR && model == NULL && msg[0],
          "model_open of a missing file is IO_ERROR with a message");
    stg_roformer_config small;
    memset(&small, 0, sizeof small);
    small.size = 4;
    check(noalloc(0, &small, 1000, (const float*)16, (const float*)16, (float*)16, NULL, msg, sizeof msg) ==
              STG_INVALID_ARGUMENT,
          "a config whose size is too small is INVALID_ARGUMENT");
    const int n_dev = device_count();
    printf("  devices: %d\n", n_dev);
    check(n_dev >= -1, "device_count: a count, or -1 when the CUDA runtime has no driver");
    if (case_dir) check(n_dev >= 1, "a GPU is visible for the separation");

    if (case_dir) {
        printf("one separation from host buffers (%s)\n", case_dir);
        size_t nb = 0;
        char* text = (char*)read_file(case_dir, "case.txt", &nb);
        int32_t* sizes = (int32_t*)read_file(case_dir, "sizes.i32", NULL);
        int32_t* freqs = (int32_t*)read_file(case_dir, "freqs.i32", NULL);
        float* mix = (float*)read_file(case_dir, "mix.f32", NULL);
        float* mask = (float*)read_file(case_dir, "mask.f32", NULL);
        float* want = (float*)read_file(case_dir, "want.f32", NULL);
        if (!text || !sizes || !freqs || !mix || !mask || !want) {
            printf("FAIL: incomplete case directory\n");
            return 1;
        }
        long long n = 0;
        int chunk = 0, nov = 0, n_bands = 0;
        text = (char*)realloc(text, nb + 1);
        text[nb] = 0;
        sscanf(text, "%lld %d %d %d", &n, &chunk, &nov, &n_bands);
        stg_engine* eng = NULL;
        check(engine_create(0, &eng) == STG_OK && eng, "engine_create(0)");
        if (!eng) return 1;
        stg_roformer_config cfg;
        memset(&cfg, 0, sizeof cfg);
        cfg.size = sizeof cfg;
        cfg.n_channels = 2; cfg.n_stems = 1; cfg.n_fft = 2048; cfg.hop = 441; cfg.chunk = chunk;
        cfg.num_overlap = nov; cfg.overlap = -1.0f; cfg.n_bands = n_bands;
        cfg.band_sizes = sizes; cfg.band_freqs = freqs; cfg.sample_rate = 44100;
        stg_roformer_config truncated = cfg;
        truncated.size = 8;
        check(plan_roformer(eng, &truncated, n, &plan) == STG_INVALID_ARGUMENT && plan == NULL && last_error(eng)[0],
              "plan_roformer with a too-small config.size: INVALID_ARGUMENT, message");
        check(plan_roformer(eng, &cfg, 0, &plan) == STG_INVALID_ARGUMENT, "plan_roformer of an empty input");
        check(plan_roformer(eng, &cfg, n, &plan) == STG_OK && plan, "plan_roformer");
        stg_plan_info info;
        memset(&info, 0, sizeof info);
        info.size = sizeof info;
        check(plan_info(plan, &info) == STG_OK && info.n_samples == n && info.n_out_sources == 1 && info.n_models == 1,
              "plan_get_info");
        stg_plan_info old;
        memset(&old, 0, sizeof old);
        old.size = STG_PLAN_INFO_V1_SIZE;
        check(plan_info(plan, &old) == STG_OK && old.n_chunks == info.n_chunks,
              "plan_get_info with the size before n_models");
        float* out = (float*)malloc(sizeof(float) * 2 * (size_t)n);
        stg_run_options opt;
        memset(&opt, 0, sizeof opt);
        opt.size = sizeof opt;
        opt.chunks_per_batch = 1;
        opt.on_progress = on_progress;
        const stg_status st = separate_host_ex(plan, mix, mask, out, NULL, &opt);
        check(st == STG_OK, "separate_host_ex");
        check(progress_calls == (int)info.n_chunks && last_done == last_total && last_total == (int)info.n_chunks,
              "progress once per chunk, ending at (total, total)");
        double worst = 0.0, scale = 0.0;
        for (long long i = 0; i < 2 * n; i++) {
            const double d = fabs((double)out[i] - (double)want[i]);
            if (d > worst) worst = d;
            if (fabs((double)want[i]) > scale) scale = fabs((double)want[i]);
        }
        printf("  max |got - oracle| / max |oracle| = %.3e\n", worst / scale);
        check(worst / scale <= 1e-5, "the result matches the oracle within 1e-5");
        plan_destroy(plan);
        engine_destroy(eng);
        free(out);
    }
    printf("%s\n", failures ? "FAILED" : "all passed");
    return failures ? 1 : 0;
}
