// gguf.cu -- GGUF package reader and the talker step built from a package
// (include/b200q8_gguf.h).  Host code only.
//
// Format (GGUF v2/v3, little-endian): "GGUF", u32 version, u64 tensor count,
// u64 metadata count; metadata entries {string key, u32 type, value}; tensor
// infos {string name, u32 n_dims, u64 ne[n_dims], u32 type, u64 offset}; the
// data section starts at the next multiple of general.alignment (32 when
// absent).  A string is {u64 length, bytes}.  The reference reads packages
// through ggml's gguf reader (src/gguf-metadata.cpp:12-46); this is a
// separate reader with every read bounds-checked against the mapped file.
#include "../../include/b200q8_gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);
}  // namespace b200q8

using namespace b200q8;

namespace {

enum GgufValueType : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kStr = 8, kArr = 9, kU64 = 10,
    kI64 = 11, kF64 = 12,
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// Bytes of a tensor of this ggml type and element count; 0 when unknown.
uint64_t tensor_bytes(int32_t type, uint64_t n) {
    switch (type) {
        case 0: return n * 4;                                  // F32
        case 1: case 30: return n * 2;                         // F16, BF16
        case 8: return n % 32 ? 0 : n / 32 * kBlockBytes;      // Q8_0
        case 24: return n;                                     // I8
        case 25: return n * 2;                                 // I16
        case 26: return n * 4;                                 // I32
        case 27: case 28: return n * 8;                        // I64, F64
        default: return 0;
    }
}

struct Reader {
    const uint8_t * p;
    size_t          size;
    size_t          pos = 0;
    bool            ok  = true;
    bool need(size_t n) {
        if (!ok || n > size - pos) {
            ok = false;
        }
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p + pos, sizeof(T));
            pos += sizeof(T);
        }
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || !need(n)) {
            ok = false;
            return std::string();
        }
        std::string s(reinterpret_cast<const char *>(p + pos), n);
        pos += n;
        return s;
    }
    // skips one value of type t (arrays of any depth, strings)
    void skip(uint32_t t, int depth = 0) {
        if (t == kStr) {
            str();
        } else if (t == kArr) {
            const uint32_t et = get<uint32_t>();
            const uint64_t n  = get<uint64_t>();
            if (!ok || depth > 4) {
                ok = false;
                return;
            }
            const size_t es = scalar_size(et);
            if (es != 0) {
                if (n > (size - pos) / es) {
                    ok = false;
                    return;
                }
                pos += n * es;
            } else {
                for (uint64_t i = 0; i < n && ok; ++i) {
                    skip(et, depth + 1);
                }
            }
        } else {
            const size_t es = scalar_size(t);
            if (es == 0) {
                ok = false;
            } else if (need(es)) {
                pos += es;
            }
        }
    }
};

struct Kv {
    std::string key;
    uint32_t    type;
    size_t      value_pos;  // file offset of the value
};

struct Tensor {
    std::string name;
    int32_t     type;
    int32_t     n_dims;
    int64_t     ne[4];
    uint64_t    offset;
    uint64_t    nbytes;
};

}  // namespace

struct b200q8_gguf {
    int                 fd   = -1;
    const uint8_t *     map  = nullptr;
    size_t              size = 0;
    uint32_t            version = 0;
    std::vector<Kv>     kv;
    std::vector<Tensor> tensors;
    size_t              data_start = 0;

    const Kv * find_kv(const char * key) const {
        for (const Kv & e : kv) {
            if (e.key == key) {
                return &e;
            }
        }
        return nullptr;
    }
};

extern "C" {

void b200q8_gguf_close(b200q8_gguf * g) {
    if (g == nullptr) {
        return;
    }
    if (g->map != nullptr) {
        munmap(const_cast<uint8_t *>(g->map), g->size);
    }
    if (g->fd >= 0) {
        close(g->fd);
    }
    delete g;
}

b200q8_status_t b200q8_gguf_open(const char * path, b200q8_gguf ** out) {
    if (path == nullptr || out == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: null argument");
    }
    *out             = nullptr;
    b200q8_gguf * g  = new b200q8_gguf();
    g->fd            = open(path, O_RDONLY);
    struct stat st   = {};
    if (g->fd < 0 || fstat(g->fd, &st) != 0 || st.st_size < 24) {
        b200q8_gguf_close(g);
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: cannot read %s", path);
    }
    g->size = (size_t) st.st_size;
    void * m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        b200q8_gguf_close(g);
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: cannot map %s", path);
    }
    g->map   = static_cast<const uint8_t *>(m);
    Reader r = { g->map, g->size };
    if (memcmp(g->map, "GGUF", 4) != 0) {
        b200q8_gguf_close(g);
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: %s is not a GGUF file", path);
    }
    r.pos              = 4;
    g->version         = r.get<uint32_t>();
    const uint64_t n_t = r.get<uint64_t>();
    const uint64_t n_k = r.get<uint64_t>();
    if (!r.ok || g->version < 2 || g->version > 3 || n_t > g->size / 24 || n_k > g->size / 12) {
        b200q8_gguf_close(g);
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: unsupported version or bad counts in %s", path);
    }
    uint32_t alignment = 32;
    for (uint64_t i = 0; i < n_k && r.ok; ++i) {
        Kv e;
        e.key       = r.str();
        e.type      = r.get<uint32_t>();
        e.value_pos = r.pos;
        if (e.key == "general.alignment" && e.type == kU32) {
            alignment = r.get<uint32_t>();
        } else {
            r.skip(e.type);
        }
        g->kv.push_back(std::move(e));
    }
    for (uint64_t i = 0; i < n_t && r.ok; ++i) {
        Tensor t;
        t.name   = r.str();
        t.n_dims = (int32_t) r.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) {
            r.ok = false;
            break;
        }
        uint64_t n = 1;
        for (int d = 0; d < 4; ++d) {
            t.ne[d] = 1;
        }
        for (int d = 0; d < t.n_dims; ++d) {
            const uint64_t v = r.get<uint64_t>();
            if (v == 0 || v > ((uint64_t) 1 << 40) || n > ((uint64_t) 1 << 62) / v) {
                r.ok = false;
            }
            t.ne[d] = (int64_t) v;
            n *= v;
        }
        t.type   = (int32_t) r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        t.nbytes = tensor_bytes(t.type, n);
        g->tensors.push_back(std::move(t));
    }
    if (!r.ok || alignment == 0 || (alignment & (alignment - 1)) != 0) {
        b200q8_gguf_close(g);
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: truncated or malformed header in %s", path);
    }
    g->data_start = (r.pos + alignment - 1) / alignment * alignment;
    for (const Tensor & t : g->tensors) {
        if (g->data_start > g->size || t.offset > g->size - g->data_start ||
            t.nbytes > g->size - g->data_start - t.offset) {
            const std::string name = t.name;
            b200q8_gguf_close(g);
            return set_error(B200Q8_ERR_INVALID_ARG, "gguf_open: tensor %s extends past the end of %s", name.c_str(),
                             path);
        }
    }
    *out = g;
    return B200Q8_OK;
}

int64_t b200q8_gguf_tensor_count(const b200q8_gguf * g) {
    return g == nullptr ? 0 : (int64_t) g->tensors.size();
}

int64_t b200q8_gguf_find_tensor(const b200q8_gguf * g, const char * name) {
    if (g == nullptr || name == nullptr) {
        return -1;
    }
    for (size_t i = 0; i < g->tensors.size(); ++i) {
        if (g->tensors[i].name == name) {
            return (int64_t) i;
        }
    }
    return -1;
}

b200q8_status_t b200q8_gguf_tensor(const b200q8_gguf * g, int64_t index, b200q8_gguf_tensor_info * out) {
    if (g == nullptr || out == nullptr || index < 0 || index >= (int64_t) g->tensors.size()) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_tensor: bad handle or index %lld", (long long) index);
    }
    const Tensor & t = g->tensors[(size_t) index];
    out->name        = t.name.c_str();
    out->type        = t.type;
    out->n_dims      = t.n_dims;
    for (int d = 0; d < 4; ++d) {
        out->ne[d] = t.ne[d];
    }
    out->offset = t.offset;
    out->nbytes = t.nbytes;
    out->data   = g->map + g->data_start + t.offset;
    return B200Q8_OK;
}

static b200q8_status_t get_scalar(const b200q8_gguf * g, const char * key, uint32_t type, void * out, size_t n) {
    if (g == nullptr || key == nullptr || out == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_get: null argument");
    }
    const Kv * e = g->find_kv(key);
    if (e == nullptr || e->type != type) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_get: %s is missing or has another type", key);
    }
    memcpy(out, g->map + e->value_pos, n);
    return B200Q8_OK;
}

b200q8_status_t b200q8_gguf_get_u32(const b200q8_gguf * g, const char * key, uint32_t * out) {
    return get_scalar(g, key, kU32, out, 4);
}

b200q8_status_t b200q8_gguf_get_f32(const b200q8_gguf * g, const char * key, float * out) {
    return get_scalar(g, key, kF32, out, 4);
}

b200q8_status_t b200q8_gguf_get_str(const b200q8_gguf * g, const char * key, char * buf, size_t buf_size) {
    if (g == nullptr || key == nullptr || buf == nullptr || buf_size == 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_get_str: null argument");
    }
    const Kv * e = g->find_kv(key);
    if (e == nullptr || e->type != kStr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_get_str: %s is missing or not a string", key);
    }
    uint64_t n;
    memcpy(&n, g->map + e->value_pos, 8);  // bounds checked at open
    const size_t c = (size_t) std::min<uint64_t>(n, buf_size - 1);
    memcpy(buf, g->map + e->value_pos + 8, c);
    buf[c] = '\0';
    return B200Q8_OK;
}

}  // extern "C"

namespace {

struct Need {
    std::string name;
    int32_t     type;  // ggml type id: 0 F32, 8 Q8_0
    int64_t     ne0, ne1;
};

// Finds every tensor of `need` (shape and type checked; host only).
b200q8_status_t find_tensors(const b200q8_gguf * g, const std::vector<Need> & need, const char * who,
                             std::vector<const Tensor *> & found) {
    found.clear();
    for (const Need & n : need) {
        const int64_t i = b200q8_gguf_find_tensor(g, n.name.c_str());
        if (i < 0) {
            return set_error(B200Q8_ERR_INVALID_ARG, "%s: tensor %s is missing", who, n.name.c_str());
        }
        const Tensor & t = g->tensors[(size_t) i];
        if (t.ne[0] != n.ne0 || t.ne[1] != n.ne1 || t.ne[2] != 1 || t.ne[3] != 1) {
            return set_error(B200Q8_ERR_INVALID_ARG, "%s: %s has shape [%lld, %lld], expected [%lld, %lld]", who,
                             n.name.c_str(), (long long) t.ne[0], (long long) t.ne[1], (long long) n.ne0,
                             (long long) n.ne1);
        }
        if (t.type != n.type) {
            return set_error(B200Q8_ERR_UNSUPPORTED, "%s: %s is ggml type %d, the step needs %s", who,
                             n.name.c_str(), t.type, n.type == 8 ? "Q8_0" : "F32");
        }
        found.push_back(&t);
    }
    return B200Q8_OK;
}

// Uploads the found tensors into one device buffer (current device) at
// 16-byte steps, so q|k|v and gate|up stay adjacent and the chain uses them in
// place; returns their device pointers.
b200q8_status_t upload_tensors(const b200q8_gguf * g, const std::vector<const Tensor *> & found, uint8_t ** buf,
                               std::vector<const void *> & ptr) {
    size_t total = 0;
    for (const Tensor * t : found) {
        total += (t->nbytes + 15) & ~(size_t) 15;
    }
    uint8_t *   dev = nullptr;
    cudaError_t e   = cudaMalloc(&dev, std::max<size_t>(total, 16));
    if (e != cudaSuccess) {
        return cuda_error(e, "gguf: weight buffer");
    }
    ptr.assign(found.size(), nullptr);
    size_t off = 0;
    for (size_t i = 0; i < found.size() && e == cudaSuccess; ++i) {
        ptr[i] = dev + off;
        e      = cudaMemcpy(dev + off, g->map + g->data_start + found[i]->offset, found[i]->nbytes,
                            cudaMemcpyHostToDevice);
        off += (found[i]->nbytes + 15) & ~(size_t) 15;
    }
    if (e != cudaSuccess) {
        cudaFree(dev);
        return cuda_error(e, "gguf: weight upload");
    }
    *buf = dev;
    return B200Q8_OK;
}

// One decoder stack of the package (the talker's or the code predictor's: the
// same block, src/arch/qwen3-tts/catalog.cpp:234-262).
struct StackSpec {
    std::string              prefix;  // "talker.model.layers." or "talker.code_predictor.model.layers."
    uint32_t                 layers = 0, hidden = 0, heads = 0, kv = 0, head_dim = 0, inter = 0;
    float                    eps = 0.0f, rope_theta = 0.0f;
    bool                     attention = false;
    int64_t                  n_ctx = 0, n_slots = 0;
    std::vector<std::string> tables;  // Q8_0 [table_hidden, table_rows]; the first is the chain's table
    uint32_t                 table_hidden = 0;
    int64_t                  table_rows   = 0;
    std::string              norm;    // final norm; empty: no output stage
    std::vector<std::string> head_names;
    int64_t                  vocab = 0;
};

b200q8_status_t build_stack(const b200q8_gguf * g, const StackSpec & s, int32_t device, int64_t max_m,
                            int32_t mode, const char * who, b200q8_chain ** out, std::vector<const void *> * tables) {
    const int64_t     Q = (int64_t) s.heads * s.head_dim, KV = (int64_t) s.kv * s.head_dim;
    const int         per_layer = s.attention ? 11 : 9;
    std::vector<Need> need;
    for (uint32_t l = 0; l < s.layers; ++l) {
        const std::string b = s.prefix + std::to_string(l) + ".";
        need.push_back({ b + "self_attn.q_proj.weight", 8, s.hidden, Q });
        need.push_back({ b + "self_attn.k_proj.weight", 8, s.hidden, KV });
        need.push_back({ b + "self_attn.v_proj.weight", 8, s.hidden, KV });
        need.push_back({ b + "self_attn.o_proj.weight", 8, Q, s.hidden });
        need.push_back({ b + "mlp.gate_proj.weight", 8, s.hidden, s.inter });
        need.push_back({ b + "mlp.up_proj.weight", 8, s.hidden, s.inter });
        need.push_back({ b + "mlp.down_proj.weight", 8, s.inter, s.hidden });
        need.push_back({ b + "input_layernorm.weight", 0, s.hidden, 1 });
        need.push_back({ b + "post_attn_norm.weight", 0, s.hidden, 1 });
        if (s.attention) {
            need.push_back({ b + "self_attn.q_norm.weight", 0, s.head_dim, 1 });
            need.push_back({ b + "self_attn.k_norm.weight", 0, s.head_dim, 1 });
        }
    }
    const size_t t0 = need.size();
    for (const std::string & t : s.tables) {
        need.push_back({ t, 8, s.table_hidden, s.table_rows });
    }
    const size_t n0 = need.size();
    if (!s.norm.empty()) {
        need.push_back({ s.norm, 0, s.hidden, 1 });
        for (const std::string & h : s.head_names) {
            need.push_back({ h, 8, s.hidden, s.vocab });
        }
    }
    std::vector<const Tensor *> found;
    b200q8_status_t             st = find_tensors(g, need, who, found);
    if (st != B200Q8_OK) {
        return st;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        return cuda_error(e, "gguf: cudaSetDevice");
    }
    uint8_t *                 dev = nullptr;
    std::vector<const void *> ptr;
    st = upload_tensors(g, found, &dev, ptr);
    if (st != B200Q8_OK) {
        cudaSetDevice(prev);
        return st;
    }
    std::vector<b200q8_layer>  ls(s.layers);
    std::vector<const float *> qn(s.layers), kn(s.layers);
    for (uint32_t l = 0; l < s.layers; ++l) {
        const void * const * q = &ptr[(size_t) l * per_layer];
        ls[l] = { q[0], q[1], q[2], q[3], q[4], q[5], q[6], static_cast<const float *>(q[7]),
                  static_cast<const float *>(q[8]) };
        if (s.attention) {
            qn[l] = static_cast<const float *>(q[9]);
            kn[l] = static_cast<const float *>(q[10]);
        }
    }
    b200q8_attention_desc ad = { s.rope_theta, s.n_ctx, s.n_slots, qn.data(), kn.data() };
    std::vector<const void *> heads(ptr.begin() + (std::ptrdiff_t) std::min(n0 + 1, ptr.size()), ptr.end());
    b200q8_output_desc        od = { s.norm.empty() ? nullptr : static_cast<const float *>(ptr[n0]), heads.data(),
                                     (int32_t) heads.size(), s.vocab };
    b200q8_chain_desc d = {};
    d.n_layers          = (int32_t) s.layers;
    d.hidden            = s.hidden;
    d.n_head            = s.heads;
    d.n_kv              = s.kv;
    d.head_dim          = s.head_dim;
    d.inter             = s.inter;
    d.eps               = s.eps;
    d.max_m             = max_m;
    d.mode              = mode;
    d.layers            = ls.data();
    d.table             = ptr[t0];
    d.table_rows        = s.table_rows;
    d.attention         = s.attention ? &ad : nullptr;
    d.output            = s.norm.empty() ? nullptr : &od;
    b200q8_chain * c    = nullptr;
    st                  = b200q8_chain_create(&d, device, &c);
    if (st != B200Q8_OK) {
        cudaFree(dev);
        cudaSetDevice(prev);
        return st;
    }
    c->owned.push_back(dev);  // the chain frees the weights with its own buffers
    if (tables != nullptr) {
        tables->assign(ptr.begin() + (std::ptrdiff_t) t0, ptr.begin() + (std::ptrdiff_t) n0);
    }
    cudaSetDevice(prev);
    *out = c;
    return B200Q8_OK;
}

// The decoder block's hyperparameters under `p` (weights.cpp:128-138 for the
// talker, 168-212 for the code predictor).
b200q8_status_t read_block(const b200q8_gguf * g, const std::string & p, const char * vocab_key, StackSpec & s,
                           uint32_t & vocab, const char * who) {
    const struct {
        const char * k;
        uint32_t *   v;
    } u32s[] = { { "layer_count", &s.layers }, { "hidden_size", &s.hidden }, { "attention_head_count", &s.heads },
                 { "key_value_head_count", &s.kv }, { "head_dim", &s.head_dim }, { vocab_key, &vocab } };
    for (const auto & e : u32s) {
        if (b200q8_gguf_get_u32(g, (p + e.k).c_str(), e.v) != B200Q8_OK) {
            return B200Q8_ERR_INVALID_ARG;
        }
    }
    if (s.layers == 0 || s.hidden == 0 || s.heads == 0 || s.kv == 0 || s.head_dim == 0 || vocab == 0 ||
        s.heads % s.kv != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "%s: zero hyperparameter or heads not a multiple of kv heads", who);
    }
    return B200Q8_OK;
}

}  // namespace

extern "C" {

b200q8_status_t b200q8_gguf_talker_chain(const b200q8_gguf * g, int32_t device, int64_t max_m, int32_t mode,
                                         b200q8_chain ** out) {
    if (g == nullptr || out == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_talker_chain: null argument");
    }
    *out = nullptr;
    const std::string p = "synthesize.qwen3-tts.talker.";
    StackSpec         s;
    uint32_t          vocab = 0;
    b200q8_status_t   st    = read_block(g, p, "codec_vocab_size", s, vocab, "gguf_talker_chain");
    if (st == B200Q8_OK) st = b200q8_gguf_get_u32(g, (p + "intermediate_size").c_str(), &s.inter);
    if (st == B200Q8_OK) st = b200q8_gguf_get_f32(g, (p + "rms_norm_eps").c_str(), &s.eps);
    if (st != B200Q8_OK) {
        return st;
    }
    if (s.inter == 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_talker_chain: zero hyperparameter");
    }
    s.prefix       = "talker.model.layers.";
    s.tables       = { "talker.model.codec_embedding.weight" };
    s.table_hidden = s.hidden;
    s.table_rows   = vocab;
    return build_stack(g, s, device, max_m, mode, "gguf_talker_chain", out, nullptr);
}

b200q8_status_t b200q8_gguf_decoder(const b200q8_gguf * g, int32_t device, int64_t max_m, int32_t mode,
                                    int64_t n_ctx, int64_t n_slots, b200q8_chain ** talker,
                                    b200q8_chain ** predictor, b200q8_frame ** frame) {
    if (g == nullptr || talker == nullptr || predictor == nullptr || max_m < 1 || n_ctx < 1 || n_slots < 1) {
        return set_error(B200Q8_ERR_INVALID_ARG, "gguf_decoder: null argument or non-positive size");
    }
    *talker    = nullptr;
    *predictor = nullptr;
    if (frame != nullptr) {
        *frame = nullptr;
    }
    const char *      who = "gguf_decoder";
    const std::string tp = "synthesize.qwen3-tts.talker.", pp = "synthesize.qwen3-tts.code_predictor.";
    StackSpec         ts, ps;
    uint32_t          t_vocab = 0, p_vocab = 0, t_groups = 0, p_groups = 0;
    b200q8_status_t   st = read_block(g, tp, "codec_vocab_size", ts, t_vocab, who);
    if (st == B200Q8_OK) st = read_block(g, pp, "vocab_size", ps, p_vocab, who);
    if (st == B200Q8_OK) st = b200q8_gguf_get_u32(g, (tp + "intermediate_size").c_str(), &ts.inter);
    if (st == B200Q8_OK) st = b200q8_gguf_get_f32(g, (tp + "rms_norm_eps").c_str(), &ts.eps);
    if (st == B200Q8_OK) st = b200q8_gguf_get_f32(g, (tp + "rope_theta").c_str(), &ts.rope_theta);
    if (st == B200Q8_OK) st = b200q8_gguf_get_u32(g, (tp + "code_group_count").c_str(), &t_groups);
    if (st == B200Q8_OK) st = b200q8_gguf_get_u32(g, (pp + "code_group_count").c_str(), &p_groups);
    if (st != B200Q8_OK) {
        return st;
    }
    // optional: packages converted before the key carry the talker's width (weights.cpp:178-193)
    if (b200q8_gguf_get_u32(g, (pp + "intermediate_size").c_str(), &ps.inter) != B200Q8_OK) {
        ps.inter = ts.inter;
    }
    char rope_type[16] = {};
    if (b200q8_gguf_get_str(g, (tp + "rope_type").c_str(), rope_type, sizeof(rope_type)) == B200Q8_OK &&
        std::strcmp(rope_type, "1d") != 0) {
        return set_error(B200Q8_ERR_UNSUPPORTED, "%s: rope type %s (only 1d is defined)", who, rope_type);
    }
    float penalty = 1.0f;
    if (b200q8_gguf_get_f32(g, "synthesize.qwen3-tts.sampling.repetition_penalty", &penalty) != B200Q8_OK) {
        penalty = 1.0f;
    }
    if (ts.inter == 0 || ps.inter == 0 || !(ts.eps > 0.0f) || !(ts.rope_theta > 0.0f) || t_groups < 2 ||
        t_groups != p_groups) {
        return set_error(B200Q8_ERR_INVALID_ARG, "%s: bad hyperparameters (intermediate sizes, eps, rope_theta, "
                                                 "code groups >= 2 and equal for both heads)", who);
    }
    // a predictor of another width than the talker reads its input through
    // small_to_mtp_projection (catalog.cpp:322-340): weight and bias
    const bool              proj = ps.hidden != ts.hidden;
    std::vector<const Tensor *> proj_found;
    if (proj) {
        const std::vector<Need> pn = {
            { "talker.code_predictor.small_to_mtp_projection.weight", 8, ts.hidden, ps.hidden },
            { "talker.code_predictor.small_to_mtp_projection.bias", 0, ps.hidden, 1 },
        };
        st = find_tensors(g, pn, who, proj_found);
        if (st != B200Q8_OK) {
            return st;
        }
    }
    // the talker's text side (build_text_projection, talker.cpp:37-50; tensors
    // as catalog.cpp:271-275 resolves them), when the package carries it
    const bool                  txt = b200q8_gguf_find_tensor(g, "talker.model.text_embedding.weight") >= 0;
    uint32_t                    t_text_hidden = 0, t_text_vocab = 0;
    std::vector<const Tensor *> txt_found;
    if (txt) {
        if (b200q8_gguf_get_u32(g, (tp + "text_hidden_size").c_str(), &t_text_hidden) != B200Q8_OK ||
            b200q8_gguf_get_u32(g, (tp + "text_vocab_size").c_str(), &t_text_vocab) != B200Q8_OK ||
            t_text_hidden == 0 || t_text_vocab == 0) {
            return set_error(B200Q8_ERR_INVALID_ARG, "%s: text_embedding without text_hidden_size / text_vocab_size",
                             who);
        }
        const std::vector<Need> tn = {
            { "talker.model.text_embedding.weight", 8, t_text_hidden, t_text_vocab },
            { "talker.text_projection.linear_fc1.weight", 8, t_text_hidden, t_text_hidden },
            { "talker.text_projection.linear_fc1.bias", 0, t_text_hidden, 1 },
            { "talker.text_projection.linear_fc2.weight", 8, t_text_hidden, ts.hidden },
            { "talker.text_projection.linear_fc2.bias", 0, ts.hidden, 1 },
        };
        st = find_tensors(g, tn, who, txt_found);
        if (st != B200Q8_OK) {
            return st;
        }
    }
    ts.prefix       = "talker.model.layers.";
    ts.attention    = true;
    ts.n_ctx        = n_ctx;
    ts.n_slots      = n_slots;
    ts.tables       = { "talker.model.codec_embedding.weight" };
    ts.table_hidden = ts.hidden;
    ts.table_rows   = t_vocab;
    ts.norm         = "talker.model.norm.weight";
    ts.head_names   = { "talker.codec_head.weight" };
    ts.vocab        = t_vocab;
    ps.prefix       = "talker.code_predictor.model.layers.";
    ps.eps          = ts.eps;  // the predictor shares the talker's eps and rope (model.cpp:315-322)
    ps.rope_theta   = ts.rope_theta;
    ps.attention    = true;
    ps.n_ctx        = t_groups;
    ps.n_slots      = n_slots;
    for (uint32_t k = 0; k + 1 < t_groups; ++k) {
        ps.tables.push_back("talker.code_predictor.model.codec_embedding." + std::to_string(k) + ".weight");
        ps.head_names.push_back("talker.code_predictor.lm_head." + std::to_string(k) + ".weight");
    }
    ps.table_hidden = ts.hidden;  // the predictor's tables are at the talker's width (catalog.cpp:297-321)
    ps.table_rows   = p_vocab;
    ps.norm         = "talker.code_predictor.model.norm.weight";
    ps.vocab        = p_vocab;
    b200q8_chain *            tc = nullptr, *pc = nullptr;
    std::vector<const void *> ptables;
    st = build_stack(g, ts, device, max_m, mode, who, &tc, nullptr);
    if (st == B200Q8_OK) st = build_stack(g, ps, device, std::max<int64_t>(8, 2 * max_m), mode, who, &pc, &ptables);
    std::vector<const void *> proj_ptr(2, nullptr);
    if (st == B200Q8_OK && proj) {  // uploaded into a buffer the predictor chain owns
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(device);
        uint8_t *   buf = nullptr;
        st = e == cudaSuccess ? upload_tensors(g, proj_found, &buf, proj_ptr) : cuda_error(e, "gguf: cudaSetDevice");
        if (st == B200Q8_OK) {
            pc->owned.push_back(buf);
        }
        cudaSetDevice(prev);
    }
    std::vector<const void *> txt_ptr(5, nullptr);
    if (st == B200Q8_OK && txt) {  // uploaded into a buffer the talker chain owns
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(device);
        uint8_t *   buf = nullptr;
        st = e == cudaSuccess ? upload_tensors(g, txt_found, &buf, txt_ptr) : cuda_error(e, "gguf: cudaSetDevice");
        if (st == B200Q8_OK) {
            tc->owned.push_back(buf);
        }
        cudaSetDevice(prev);
    }
    if (st == B200Q8_OK && frame != nullptr) {
        b200q8_frame_desc fd     = {};
        fd.talker                = tc;
        fd.predictor             = pc;
        fd.groups                = (int32_t) t_groups;
        fd.tables                = ptables.data();
        fd.table_rows            = p_vocab;
        fd.repetition_penalty    = penalty;
        fd.input_projection      = proj_ptr[0];
        fd.input_projection_bias = static_cast<const float *>(proj_ptr[1]);
        if (txt) {
            fd.text_embedding = txt_ptr[0];
            fd.text_rows      = t_text_vocab;
            fd.text_hidden    = t_text_hidden;
            fd.text_fc1       = txt_ptr[1];
            fd.text_fc1_bias  = static_cast<const float *>(txt_ptr[2]);
            fd.text_fc2       = txt_ptr[3];
            fd.text_fc2_bias  = static_cast<const float *>(txt_ptr[4]);
        }
        st = b200q8_frame_create(&fd, frame);
    }
    if (st != B200Q8_OK) {
        b200q8_chain_destroy(tc);
        b200q8_chain_destroy(pc);
        return st;
    }
    *talker    = tc;
    *predictor = pc;
    return B200Q8_OK;
}

}  // extern "C"
