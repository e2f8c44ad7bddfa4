// gguf.cu -- a model's spectral-path configuration read straight from its GGUF file, without
// ggml: the metadata the separators' constructors read (src/htdemucs.cpp:478-500,
// src/roformer.cpp:360-412, src/tfc_tdf.cpp:498-553, src/vr.cpp:296-327) and, for VR, the
// resampling FIR tensors. Weights are never read.
//
// The file format is GGUF version 2 or 3 as published: the magic "GGUF", a version, the tensor
// and key/value counts, the key/value pairs (a string key, a type tag, a value; arrays carry
// an element type and a count), the tensor infos (name, dimensions, ggml type, offset), and the
// data section at the next multiple of general.alignment (32 when absent).
#include "../../include/stems_gpu_v1.h"
#include "plan.h"

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

using stg::fail;

enum : uint32_t {
    T_U8 = 0, T_I8 = 1, T_U16 = 2, T_I16 = 3, T_U32 = 4, T_I32 = 5, T_F32 = 6, T_BOOL = 7,
    T_STRING = 8, T_ARRAY = 9, T_U64 = 10, T_I64 = 11, T_F64 = 12
};

// One metadata value: scalars as double (every integer the separators read fits), strings,
// and arrays of either.
struct Value {
    uint32_t type = 0, elem = 0;
    double num = 0;
    std::string str;
    std::vector<double> nums;
    std::vector<std::string> strs;
};

struct TensorInfo {
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
};

class Reader {
public:
    explicit Reader(const char* path) : f_(std::fopen(path, "rb")) {
        if (!f_) fail(STG_IO_ERROR, std::string("cannot open ") + path);
    }
    ~Reader() { if (f_) std::fclose(f_); }
    void raw(void* p, size_t n) {
        if (n && std::fread(p, 1, n, f_) != n) fail(STG_MODEL_ERROR, "gguf: truncated file");
    }
    template <class T> T get() { T v; raw(&v, sizeof v); return v; }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > (1u << 26)) fail(STG_MODEL_ERROR, "gguf: implausible string length");
        std::string s(n, '\0');
        raw(&s[0], n);
        return s;
    }
    double scalar(uint32_t t) {
        switch (t) {
            case T_U8: return get<uint8_t>();
            case T_I8: return get<int8_t>();
            case T_U16: return get<uint16_t>();
            case T_I16: return get<int16_t>();
            case T_U32: return get<uint32_t>();
            case T_I32: return get<int32_t>();
            case T_F32: return get<float>();
            case T_BOOL: return get<uint8_t>() != 0;
            case T_U64: return (double)get<uint64_t>();
            case T_I64: return (double)get<int64_t>();
            case T_F64: return get<double>();
        }
        fail(STG_MODEL_ERROR, "gguf: unknown value type");
    }
    Value value(uint32_t t) {
        Value v;
        v.type = t;
        if (t == T_STRING) {
            v.str = str();
        } else if (t == T_ARRAY) {
            v.elem = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            if (n > (1u << 28)) fail(STG_MODEL_ERROR, "gguf: implausible array length");
            for (uint64_t i = 0; i < n; i++) {
                if (v.elem == T_STRING) v.strs.push_back(str());
                else if (v.elem == T_ARRAY) fail(STG_MODEL_ERROR, "gguf: nested arrays are not read");
                else v.nums.push_back(scalar(v.elem));
            }
        } else {
            v.num = scalar(t);
        }
        return v;
    }
    uint64_t tell() { return (uint64_t)std::ftell(f_); }
    void seek(uint64_t off) {
        if (std::fseek(f_, (long)off, SEEK_SET) != 0) fail(STG_MODEL_ERROR, "gguf: seek failed");
    }

private:
    FILE* f_;
};

} // namespace

struct stg_model {
    std::string path, arch;
    std::map<std::string, Value> kv;
    std::map<std::string, TensorInfo> tensors;
    uint64_t data_start = 0;
    // the configurations, and the arrays their pointers borrow
    std::vector<int32_t> band_sizes, band_freqs;
    std::vector<float> bag;
    std::vector<stg_vr_band> vr_bands;
    std::vector<stg_vr_fir> vr_firs;
    std::vector<std::vector<float>> fir_taps;

    const Value& at(const std::string& k) const {
        auto it = kv.find(k);
        if (it == kv.end()) fail(STG_MODEL_ERROR, path + ": missing key " + k);
        return it->second;
    }
    bool has(const std::string& k) const { return kv.count(k) != 0; }
    int64_t integer(const std::string& k) const {
        const Value& v = at(k);
        if (v.type == T_STRING || v.type == T_ARRAY || v.type == T_F32 || v.type == T_F64)
            fail(STG_MODEL_ERROR, path + ": key " + k + " is not an integer");
        return (int64_t)v.num;
    }
    double real(const std::string& k) const {
        const Value& v = at(k);
        if (v.type == T_STRING || v.type == T_ARRAY) fail(STG_MODEL_ERROR, path + ": key " + k + " is not a number");
        return v.num;
    }
    bool boolean(const std::string& k) const {
        const Value& v = at(k);
        if (v.type != T_BOOL) fail(STG_MODEL_ERROR, path + ": key " + k + " is not bool");
        return v.num != 0;
    }
    const std::string& string(const std::string& k) const {
        const Value& v = at(k);
        if (v.type != T_STRING) fail(STG_MODEL_ERROR, path + ": key " + k + " is not a string");
        return v.str;
    }
    size_t n_sources() const {
        const Value& v = at("stems.sources");
        if (v.type != T_ARRAY || v.elem != T_STRING) fail(STG_MODEL_ERROR, path + ": bad stems.sources");
        return v.strs.size();
    }
    std::vector<float> floats(const std::string& k) const {
        const Value& v = at(k);
        if (v.type != T_ARRAY || v.elem != T_F32) fail(STG_MODEL_ERROR, path + ": bad " + k);
        return std::vector<float>(v.nums.begin(), v.nums.end());
    }
    std::vector<int32_t> ints(const std::string& k) const {
        const Value& v = at(k);
        if (v.type != T_ARRAY || (v.elem != T_I32 && v.elem != T_U32)) fail(STG_MODEL_ERROR, path + ": bad " + k);
        return std::vector<int32_t>(v.nums.begin(), v.nums.end());
    }

    void load(const char* p) {
        path = p;
        Reader r(p);
        char magic[4];
        r.raw(magic, 4);
        if (std::memcmp(magic, "GGUF", 4) != 0) fail(STG_MODEL_ERROR, path + ": not a GGUF file");
        const uint32_t version = r.get<uint32_t>();
        if (version != 2 && version != 3) fail(STG_MODEL_ERROR, path + ": unsupported GGUF version");
        const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
        if (n_tensors > (1u << 24) || n_kv > (1u << 20)) fail(STG_MODEL_ERROR, path + ": implausible counts");
        for (uint64_t i = 0; i < n_kv; i++) {
            std::string k = r.str();
            const uint32_t t = r.get<uint32_t>();
            kv[k] = r.value(t);
        }
        for (uint64_t i = 0; i < n_tensors; i++) {
            std::string name = r.str();
            TensorInfo ti;
            const uint32_t nd = r.get<uint32_t>();
            if (nd > 8) fail(STG_MODEL_ERROR, path + ": tensor with more than 8 dimensions");
            for (uint32_t d = 0; d < nd; d++) ti.dims.push_back(r.get<uint64_t>());
            ti.type = r.get<uint32_t>();
            ti.offset = r.get<uint64_t>();
            tensors[name] = ti;
        }
        const uint64_t align = has("general.alignment") ? (uint64_t)integer("general.alignment") : 32;
        if (align == 0 || (align & (align - 1))) fail(STG_MODEL_ERROR, path + ": bad general.alignment");
        data_start = (r.tell() + align - 1) / align * align;
        arch = string("general.architecture");
    }

    // an F32 vector tensor's values (the VR FIRs)
    std::vector<float> f32_vector(const std::string& name) const {
        auto it = tensors.find(name);
        if (it == tensors.end()) fail(STG_MODEL_ERROR, path + ": missing tensor " + name);
        const TensorInfo& t = it->second;
        uint64_t n = 1;
        for (uint64_t d : t.dims) n *= d;
        if (t.type != 0 || n == 0 || n > (1u << 24)) fail(STG_MODEL_ERROR, path + ": bad tensor " + name);
        std::vector<float> v(n);
        Reader r(path.c_str());
        r.seek(data_start + t.offset);
        r.raw(v.data(), n * sizeof(float));
        return v;
    }
};

namespace {

void write_message(char* msg, size_t cap, const char* text) {
    if (msg && cap) std::snprintf(msg, cap, "%s", text);
}

template <class Fn> stg_status run(char* msg, size_t cap, Fn fn) {
    write_message(msg, cap, "");
    try {
        fn();
        return STG_OK;
    } catch (const stg::Failure& f) {
        write_message(msg, cap, f.what());
        return f.code;
    } catch (const std::bad_alloc&) {
        write_message(msg, cap, "out of host memory");
        return STG_OUT_OF_MEMORY;
    } catch (const std::exception& x) {
        write_message(msg, cap, x.what());
        return STG_INTERNAL_ERROR;
    }
}

} // namespace

extern "C" {

STG_API stg_status stg_model_open(const char* gguf_path, stg_model** out, char* message, size_t message_size) {
    if (!out || !gguf_path) return STG_INVALID_ARGUMENT;
    *out = nullptr;
    return run(message, message_size, [&] {
        auto m = std::make_unique<stg_model>();
        m->load(gguf_path);
        *out = m.release();
    });
}

STG_API void stg_model_close(stg_model* m) { delete m; }

STG_API const char* stg_model_architecture(const stg_model* m) { return m ? m->arch.c_str() : ""; }

STG_API int32_t stg_model_sample_rate(const stg_model* m) {
    if (!m || !m->has("stems.samplerate")) return 0;
    return (int32_t)m->real("stems.samplerate");
}

STG_API stg_status stg_model_htdemucs_config(const stg_model* m, stg_htdemucs_config* c, char* message,
                                             size_t message_size) {
    if (!m || !c || c->size < STG_HTDEMUCS_CONFIG_V1_SIZE) return STG_INVALID_ARGUMENT;
    return run(message, message_size, [&] {
        if (m->arch != "htdemucs") fail(STG_MODEL_ERROR, m->path + ": not an htdemucs GGUF");   // :483
        const int64_t sr = m->integer("stems.samplerate"), num = m->integer("stems.segment_num"),
                      den = m->integer("stems.segment_den");
        if (den <= 0) fail(STG_MODEL_ERROR, m->path + ": bad stems.segment_den");
        const uint32_t size = c->size;
        std::memset(c, 0, sizeof(*c));
        c->size = size;
        c->n_channels = (int32_t)m->integer("stems.audio_channels");
        c->n_sources = (int32_t)m->n_sources();
        c->segment = (int32_t)(num * sr / den);                         // segment_samples() :317
        c->overlap = -1.0f;
        c->mono_norm = 1;
        c->cac_norm = 1;
        c->sample_rate = (int32_t)sr;
        // the bag (:493-499): stems.n_models and stems.bag_weights [n_models][sources]; a file
        // without them is one model
        if (m->has("stems.n_models") || m->has("stems.bag_weights")) {
            const int64_t n_models = m->integer("stems.n_models");
            std::vector<float> w = m->floats("stems.bag_weights");
            if (n_models < 1 || n_models > 64 || w.size() != (size_t)n_models * (size_t)c->n_sources)
                fail(STG_MODEL_ERROR, m->path + ": stems.bag_weights has the wrong size");
            if (size >= sizeof(stg_htdemucs_config)) {
                auto* mm = const_cast<stg_model*>(m);
                mm->bag = std::move(w);
                c->n_models = (int32_t)n_models;
                c->bag_weights = mm->bag.data();
            } else if (n_models > 1) {
                fail(STG_INVALID_ARGUMENT, "a bag of models needs the full stg_htdemucs_config (n_models, bag_weights)");
            }
        }
    });
}

STG_API stg_status stg_model_roformer_config(const stg_model* m, stg_roformer_config* c, char* message,
                                             size_t message_size) {
    if (!m || !c || c->size < sizeof(stg_roformer_config)) return STG_INVALID_ARGUMENT;
    return run(message, message_size, [&] {
        if (m->arch != "mel_band_roformer" && m->arch != "bs_roformer")            // :366-368
            fail(STG_MODEL_ERROR, m->path + ": not a roformer GGUF");
        auto* mm = const_cast<stg_model*>(m);
        mm->band_sizes = m->ints("roformer.band_sizes");                             // :394-395
        mm->band_freqs = m->ints("roformer.band_freqs");
        const uint32_t size = c->size;
        std::memset(c, 0, sizeof(*c));
        c->size = size;
        c->n_channels = (int32_t)m->integer("stems.audio_channels");
        c->n_stems = (int32_t)m->n_sources();
        c->n_fft = (int32_t)m->integer("roformer.stft_n_fft");
        c->hop = (int32_t)m->integer("roformer.stft_hop_length");
        c->normalized = m->boolean("roformer.stft_normalized");
        c->zero_dc = m->boolean("roformer.zero_dc");
        c->chunk = (int32_t)m->integer("roformer.chunk_size");
        c->num_overlap = (int32_t)m->integer("roformer.num_overlap");
        c->overlap = -1.0f;
        c->n_bands = (int32_t)mm->band_sizes.size();
        c->band_sizes = mm->band_sizes.data();
        c->band_freqs = mm->band_freqs.data();
        c->complement = m->has("stems.complement");                                  // :374-377
        c->sample_rate = (int32_t)m->integer("stems.samplerate");
    });
}

STG_API stg_status stg_model_tfc_config(const stg_model* m, stg_tfc_config* c, char* message, size_t message_size) {
    if (!m || !c || c->size < sizeof(stg_tfc_config)) return STG_INVALID_ARGUMENT;
    return run(message, message_size, [&] {
        if (m->arch != "tfc_tdf" || m->integer("tfc_tdf.schema_version") != 1)   // :504
            fail(STG_MODEL_ERROR, m->path + ": not a tfc_tdf GGUF (schema 1)");
        const std::string& chunking = m->string("tfc_tdf.chunking");
        const uint32_t size = c->size;
        std::memset(c, 0, sizeof(*c));
        c->size = size;
        c->n_stems = (int32_t)m->n_sources();
        c->n_fft = (int32_t)m->integer("tfc_tdf.n_fft");
        c->hop = (int32_t)m->integer("tfc_tdf.hop");
        c->dim_f = (int32_t)m->integer("tfc_tdf.dim_f");
        c->dim_t = (int32_t)m->integer("tfc_tdf.dim_t");
        if (chunking == "uvr_mdx") {                                                  // :532-534
            c->chunking = 0;
            c->zero_bins = (int32_t)m->integer("tfc_tdf.zero_bins");
        } else if (chunking == "msst") {
            c->chunking = 1;
            c->num_overlap = (int32_t)m->integer("tfc_tdf.num_overlap");
        } else {
            fail(STG_MODEL_ERROR, m->path + ": unknown tfc_tdf.chunking '" + chunking + "'");
        }
        c->overlap = -1.0f;
        c->compensate = (float)m->real("tfc_tdf.compensate");
        c->complement = m->has("stems.complement");
    });
}

STG_API stg_status stg_model_vr_config(const stg_model* m, stg_vr_config* c, char* message, size_t message_size) {
    if (!m || !c || c->size < sizeof(stg_vr_config)) return STG_INVALID_ARGUMENT;
    return run(message, message_size, [&] {
        if (m->arch != "vr_cascaded" || m->integer("vr.schema_version") != 1)        // vr.cpp:300-301
            fail(STG_MODEL_ERROR, m->path + ": not a vr GGUF (schema 1)");
        if (m->string("vr.resampling") != "polyphase") fail(STG_MODEL_ERROR, m->path + ": vr.resampling is not polyphase");
        auto* mm = const_cast<stg_model*>(m);
        const int64_t count = m->integer("vr.band_count");
        if (count < 1 || count > 16) fail(STG_MODEL_ERROR, m->path + ": invalid band count");
        mm->vr_bands.clear();
        for (int64_t i = 0; i < count; i++) {                                        // vr.cpp:311-318
            auto key = [&](const char* k) {
                const std::string n = "vr.band." + std::to_string(i) + "." + k;
                const Value& v = m->at(n);
                if (v.type != T_I32) fail(STG_MODEL_ERROR, m->path + ": " + n + " is not int32");
                return (int32_t)v.num;
            };
            mm->vr_bands.push_back(stg_vr_band{key("sr"), key("hl"), key("n_fft"), key("crop_start"), key("crop_stop"),
                                               key("hpf_start"), key("hpf_stop"), key("lpf_start"), key("lpf_stop")});
        }
        mm->vr_firs.clear();
        mm->fir_taps.clear();
        for (const auto& a : mm->vr_bands)                                            // vr.cpp:320-327
            for (const auto& b : mm->vr_bands) {
                if (a.sample_rate == b.sample_rate) continue;
                bool seen = false;
                for (const auto& f : mm->vr_firs) seen |= f.src_rate == a.sample_rate && f.dst_rate == b.sample_rate;
                if (seen) continue;
                mm->fir_taps.push_back(m->f32_vector("resample." + std::to_string(a.sample_rate) + "." +
                                                     std::to_string(b.sample_rate)));
                mm->vr_firs.push_back(stg_vr_fir{a.sample_rate, b.sample_rate, 0, nullptr});
            }
        for (size_t k = 0; k < mm->vr_firs.size(); k++) {   // pointers once the vectors stop moving
            mm->vr_firs[k].n_taps = (int32_t)mm->fir_taps[k].size();
            mm->vr_firs[k].taps = mm->fir_taps[k].data();
        }
        const uint32_t size = c->size;
        std::memset(c, 0, sizeof(*c));
        c->size = size;
        c->sample_rate = (int32_t)m->integer("stems.samplerate");
        c->bins = (int32_t)m->integer("vr.bins");
        c->pre_filter_start = (int32_t)m->integer("vr.pre_filter_start");
        c->pre_filter_stop = (int32_t)m->integer("vr.pre_filter_stop");
        c->n_bands = (int32_t)mm->vr_bands.size();
        c->bands = mm->vr_bands.data();
        c->n_firs = (int32_t)mm->vr_firs.size();
        c->firs = mm->vr_firs.data();
    });
}

} // extern "C"
