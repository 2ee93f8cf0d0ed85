// lc_gguf.cpp -- GGUF v3 reader for lc_model_load_gguf.
//
// Follows GGUFReader.readMetadata (GGUFReader.java:57-123): magic 0x46554747,
// version, tensor count, KV count, typed metadata values, tensor infos
// (name, n_dims, shape, type, offset), data start aligned to
// general.alignment (default 32).  Validation follows LlamaModel
// (LlamaModel.java:74-86): general.architecture must be "llama".  The file is
// memory-mapped and every tensor is uploaded to the device once, straight
// from the mapping (no intermediate host copy).
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/llamacuda.h"

extern "C" int lc_gguf_set_error(int code, const char* msg);

namespace {

struct Reader {
    const uint8_t* base;
    size_t size;
    size_t off = 0;
    bool bad = false;

    bool need(size_t n) {
        if (off + n > size) {
            bad = true;
            return false;
        }
        return true;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, base + off, sizeof(T));
            off += sizeof(T);
        }
        return v;
    }
    std::string str() {
        uint64_t n = get<uint64_t>();
        if (bad || !need(n)) return std::string();
        std::string s((const char*)base + off, (size_t)n);
        off += n;
        return s;
    }
};

struct Value {
    int type = -1;
    double num = 0;
    std::string s;
};

// Size in bytes of one scalar of a GGUF value type, 0 for string/array.
size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;     // u8, i8, bool
        case 2: case 3: return 2;             // u16, i16
        case 4: case 5: case 6: return 4;     // u32, i32, f32
        case 10: case 11: case 12: return 8;  // u64, i64, f64
        default: return 0;
    }
}

double read_scalar(Reader& r, uint32_t t) {
    switch (t) {
        case 0: return r.get<uint8_t>();
        case 1: return r.get<int8_t>();
        case 2: return r.get<uint16_t>();
        case 3: return r.get<int16_t>();
        case 4: return r.get<uint32_t>();
        case 5: return r.get<int32_t>();
        case 6: return r.get<float>();
        case 7: return r.get<uint8_t>();
        case 10: return (double)r.get<uint64_t>();
        case 11: return (double)r.get<int64_t>();
        case 12: return r.get<double>();
        default: r.bad = true; return 0;
    }
}

bool read_value(Reader& r, uint32_t t, Value* v) {
    v->type = (int)t;
    if (t == 8) {
        v->s = r.str();
    } else if (t == 9) {
        uint32_t et = r.get<uint32_t>();
        uint64_t n = r.get<uint64_t>();
        if (et == 8) {
            for (uint64_t i = 0; i < n && !r.bad; ++i) r.str();
        } else {
            size_t es = scalar_size(et);
            if (!es || !r.need(es * n)) return false;
            r.off += es * n;
        }
    } else {
        if (!scalar_size(t)) return false;
        v->num = read_scalar(r, t);
    }
    return !r.bad;
}

struct TensorInfo {
    std::vector<uint64_t> shape;
    uint32_t type;
    uint64_t offset;
    uint64_t elems() const {
        uint64_t n = 1;
        for (uint64_t d : shape) n *= d;
        return n;
    }
};

}  // namespace

extern "C" int lc_model_load_gguf(lc_context* ctx, const char* path, int32_t max_seq, lc_model** out) {
    return lc_model_load_gguf_mode(ctx, path, max_seq, LC_WEIGHTS_F16, out);
}

extern "C" int lc_model_load_gguf_mode(lc_context* ctx, const char* path, int32_t max_seq, int32_t weight_mode,
                                       lc_model** out) {
    if (!ctx || !path || !out) return lc_gguf_set_error(LC_ERR_INVALID_ARG, "NULL argument");
    if (weight_mode != LC_WEIGHTS_F16 && weight_mode != LC_WEIGHTS_F32)
        return lc_gguf_set_error(LC_ERR_INVALID_ARG, "Unknown weight storage mode (F16 = 0, F32 = 1)");
    int fd = open(path, O_RDONLY);
    if (fd < 0) return lc_gguf_set_error(LC_ERR_IO, "cannot open GGUF file");
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return lc_gguf_set_error(LC_ERR_IO, "GGUF file too small");
    }
    const size_t size = (size_t)st.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return lc_gguf_set_error(LC_ERR_IO, "mmap failed");
    int rc = LC_OK;
    lc_model* m = nullptr;
    do {
        Reader r{(const uint8_t*)map, size};
        uint32_t magic = r.get<uint32_t>();
        if (magic != 0x46554747u) {
            rc = lc_gguf_set_error(LC_ERR_IO, "Not a GGUF file or wrong magic");
            break;
        }
        r.get<uint32_t>();  // version
        uint64_t n_tensors = r.get<uint64_t>();
        uint64_t n_kv = r.get<uint64_t>();
        std::map<std::string, Value> meta;
        for (uint64_t i = 0; i < n_kv && !r.bad; ++i) {
            std::string key = r.str();
            uint32_t t = r.get<uint32_t>();
            Value v;
            if (!read_value(r, t, &v)) {
                r.bad = true;
                break;
            }
            meta[key] = v;
        }
        std::map<std::string, TensorInfo> tensors;
        for (uint64_t i = 0; i < n_tensors && !r.bad; ++i) {
            std::string name = r.str();
            uint32_t nd = r.get<uint32_t>();
            TensorInfo ti;
            for (uint32_t d = 0; d < nd && !r.bad; ++d) ti.shape.push_back(r.get<uint64_t>());
            ti.type = r.get<uint32_t>();
            ti.offset = r.get<uint64_t>();
            tensors[name] = ti;
        }
        if (r.bad) {
            rc = lc_gguf_set_error(LC_ERR_IO, "truncated or malformed GGUF header");
            break;
        }
        uint64_t alignment = 32;
        auto ai = meta.find("general.alignment");
        if (ai != meta.end() && ai->second.type != 8 && ai->second.num > 0) alignment = (uint64_t)ai->second.num;
        const uint64_t data_start = (r.off + alignment - 1) / alignment * alignment;

        auto arch = meta.find("general.architecture");
        if (arch == meta.end() || arch->second.s != "llama") {
            rc = lc_gguf_set_error(LC_ERR_INVALID_ARG, "Expected 'llama' architecture");
            break;
        }
        // Architecture: Llama-3.2-1B constants, overridden by llama.* metadata
        // when present; vocab from the embedding shape.
        lc_config cfg;
        lc_config_llama32_1b(&cfg);
        auto num = [&](const char* k, double* v) {
            auto it = meta.find(k);
            if (it == meta.end() || it->second.type == 8 || it->second.type == 9) return false;
            *v = it->second.num;
            return true;
        };
        double v;
        if (num("llama.embedding_length", &v)) cfg.dim = (int32_t)v;
        if (num("llama.feed_forward_length", &v)) cfg.hidden = (int32_t)v;
        if (num("llama.block_count", &v)) cfg.n_layers = (int32_t)v;
        if (num("llama.attention.head_count", &v)) cfg.n_heads = (int32_t)v;
        if (num("llama.attention.head_count_kv", &v)) cfg.n_kv_heads = (int32_t)v;
        if (num("llama.rope.freq_base", &v)) cfg.rope_theta = (float)v;
        if (num("llama.attention.layer_norm_rms_epsilon", &v)) cfg.rms_eps = (float)v;
        cfg.head_dim = cfg.n_heads > 0 ? cfg.dim / cfg.n_heads : 0;
        auto emb = tensors.find("token_embd.weight");
        if (emb == tensors.end()) {
            rc = lc_gguf_set_error(LC_ERR_NOT_FOUND, "Tensor not found: token_embd.weight");
            break;
        }
        if (cfg.dim > 0) cfg.vocab = (int32_t)(emb->second.elems() / (uint64_t)cfg.dim);
        if (max_seq > 0) cfg.max_seq = max_seq;
        cfg.weight_mode = weight_mode;
        if ((rc = lc_model_create(ctx, &cfg, &m)) != LC_OK) break;
        for (auto& kv : tensors) {
            const TensorInfo& ti = kv.second;
            if (ti.type != 0 && ti.type != 1) {
                rc = lc_gguf_set_error(LC_ERR_INVALID_ARG, "Unsupported tensor type (only F32 and F16)");
                break;
            }
            const uint64_t bytes = ti.elems() * (ti.type == 0 ? 4 : 2);
            if (data_start + ti.offset + bytes > size) {
                rc = lc_gguf_set_error(LC_ERR_IO, "tensor data past end of file");
                break;
            }
            rc = lc_model_upload_tensor(m, kv.first.c_str(), (const uint8_t*)map + data_start + ti.offset,
                                        (int64_t)ti.elems(), (int32_t)ti.type);
            if (rc == LC_ERR_NOT_FOUND) rc = LC_OK;  // tensors outside the decode path are ignored
            if (rc != LC_OK) break;
        }
        if (rc != LC_OK) break;
        rc = lc_model_finalize(m);
    } while (0);
    munmap(map, size);
    if (rc != LC_OK) {
        if (m) lc_model_destroy(m);
        return rc;
    }
    *out = m;
    return LC_OK;
}
