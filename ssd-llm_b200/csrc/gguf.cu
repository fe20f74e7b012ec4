// gguf.cu — GGUF reader and HBM weight loader (host code).
//
// Replaces GgufFile::open and its accessors (src/model/gguf.rs:233-441) and the tensor
// lookups of the layer step (transformer.rs:171-180, :557, :644-700): the file's header,
// metadata and tensor infos are parsed with the reference's rules (magic "GGUF", version
// 2 or 3, strings of at most 1 MiB, tensor size = ceil(n_elements / block) * block bytes,
// data section at the next multiple of general.alignment, default 32), tensors are read in
// the reference's own block formats and uploaded HBM-resident through the model's shard
// logic (ssd_model_set_tensor), and a Llama-shaped model config is derived from the
// "{arch}.*" metadata keys.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint64_t kMaxString = 1024 * 1024;  // read_gguf_string's limit (gguf.rs:442-447)

enum MetaType {
    M_U8 = 0, M_I8 = 1, M_U16 = 2, M_I16 = 3, M_U32 = 4, M_I32 = 5, M_F32 = 6, M_BOOL = 7,
    M_STR = 8, M_ARR = 9, M_U64 = 10, M_I64 = 11, M_F64 = 12
};

struct Meta {
    std::string key;
    uint32_t type = 0;
    uint64_t u = 0;  // unsigned / bool value (and the raw bits of signed ones)
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    uint32_t arr_type = 0;
    uint64_t arr_len = 0;
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0, size = 0;
};

// GgmlType::block_size / type_size (gguf.rs:87-135), including the fallbacks for types
// the reference does not list (block 32, size 2).
uint64_t block_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 24: case 25: case 26: case 27: case 28: case 30: return 1;
        case 10: case 11: case 12: case 13: case 14: case 15: return 256;
        case 16: case 17: case 18: case 21: case 22: case 23: return 256;
        default: return 32;
    }
}
uint64_t type_size(uint32_t t) {
    switch (t) {
        case 0: case 26: return 4;
        case 1: case 30: case 25: return 2;
        case 24: return 1;
        case 2: return 18;
        case 3: return 20;
        case 6: return 22;
        case 7: return 24;
        case 8: return 34;
        case 9: return 40;
        case 10: return 84;
        case 11: return 256 / 8 * 3 + 256 / 4 + 12 + 2;
        case 12: return 2 + 2 + 12 + 256 / 2;
        case 13: return 2 + 2 + 12 + 256 / 8 + 256 / 2;
        case 14: return 256 / 2 + 256 / 4 + 256 / 16 + 2;
        case 15: return 292;
        case 20: return 18;
        case 23: return 148;
        case 18: return 98;
        case 21: return 110;
        case 16: return 66;
        case 17: return 74;
        case 22: return 82;
        case 27: case 28: return 8;
        default: return 2;
    }
}

struct Reader {
    FILE* f;
    bool ok = true;
    bool read(void* dst, size_t n) {
        if (ok && n && fread(dst, 1, n, f) != n) ok = false;
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        read(&v, sizeof v);
        return v;
    }
    bool str(std::string& out) {
        const uint64_t n = get<uint64_t>();
        if (!ok) return false;
        if (n > kMaxString) {
            ok = false;
            return false;
        }
        out.resize(n);
        return read(out.data(), n);
    }
};

}  // namespace

struct ssd_gguf {
    std::string path;
    uint32_t version = 0;
    uint64_t n_tensors = 0, n_kv = 0, data_offset = 0, file_size = 0;
    std::vector<Meta> meta;
    std::vector<Tensor> tensors;
    const Meta* find(const char* key) const {
        for (const Meta& m : meta)
            if (m.key == key) return &m;
        return nullptr;
    }
};

using namespace ssd;

namespace {

// read_metadata_value_typed (gguf.rs:454-483); arrays keep their element type and length
// (their elements are read and skipped)
bool read_value(Reader& r, uint32_t type, Meta& m, int depth) {
    m.type = type;
    switch (type) {
        case M_U8: m.u = r.get<uint8_t>(); break;
        case M_I8: m.i = r.get<int8_t>(); m.u = (uint64_t)m.i; break;
        case M_U16: m.u = r.get<uint16_t>(); break;
        case M_I16: m.i = r.get<int16_t>(); m.u = (uint64_t)m.i; break;
        case M_U32: m.u = r.get<uint32_t>(); break;
        case M_I32: m.i = r.get<int32_t>(); m.u = (uint64_t)m.i; break;
        case M_F32: m.f = r.get<float>(); break;
        case M_BOOL: m.u = r.get<uint8_t>() != 0; break;
        case M_STR: r.str(m.s); break;
        case M_ARR: {
            if (depth > 8) return false;
            m.arr_type = r.get<uint32_t>();
            m.arr_len = r.get<uint64_t>();
            for (uint64_t k = 0; k < m.arr_len && r.ok; k++) {
                Meta e;
                if (!read_value(r, m.arr_type, e, depth + 1)) return false;
            }
            break;
        }
        case M_U64: m.u = r.get<uint64_t>(); break;
        case M_I64: m.i = r.get<int64_t>(); m.u = (uint64_t)m.i; break;
        case M_F64: m.f = r.get<double>(); break;
        default: return false;  // "Unknown metadata value type"
    }
    return r.ok;
}

// MetadataValue::as_u32 (gguf.rs:183-190): u32, i32 and u64 values
bool as_u32(const Meta* m, uint32_t* out) {
    if (!m || (m->type != M_U32 && m->type != M_I32 && m->type != M_U64)) return false;
    *out = (uint32_t)m->u;
    return true;
}

}  // namespace

extern "C" int ssd_gguf_open(const char* path, ssd_gguf** out) {
    SSD_REQ(path && out, SSD_ERR_ARG, "null argument");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    SSD_REQ(f != nullptr, SSD_ERR_ARG, "Failed to open GGUF file %s", path);
    ssd_gguf* g = new ssd_gguf();
    g->path = path;
    Reader r{f};
    int st = SSD_OK;
    do {
        fseek(f, 0, SEEK_END);
        g->file_size = (uint64_t)ftell(f);
        fseek(f, 0, SEEK_SET);
        const uint32_t magic = r.get<uint32_t>();
        if (!r.ok || magic != kGgufMagic) {
            set_error("Not a GGUF file (magic: %#x, expected %#x)", magic, kGgufMagic);
            st = SSD_ERR_ARG;
            break;
        }
        g->version = r.get<uint32_t>();
        if (!r.ok || g->version < 2 || g->version > 3) {
            set_error("Unsupported GGUF version: %u (supported: 2-3)", g->version);
            st = SSD_ERR_ARG;
            break;
        }
        g->n_tensors = r.get<uint64_t>();
        g->n_kv = r.get<uint64_t>();
        for (uint64_t k = 0; k < g->n_kv && r.ok; k++) {
            Meta m;
            if (!r.str(m.key)) break;
            const uint32_t t = r.get<uint32_t>();
            if (!r.ok || !read_value(r, t, m, 0)) {
                r.ok = false;
                break;
            }
            g->meta.push_back(std::move(m));
        }
        for (uint64_t k = 0; k < g->n_tensors && r.ok; k++) {
            Tensor t;
            if (!r.str(t.name)) break;
            const uint32_t nd = r.get<uint32_t>();
            if (!r.ok || nd > 8) {
                r.ok = false;
                break;
            }
            uint64_t n = 1;
            for (uint32_t d = 0; d < nd; d++) {
                t.dims.push_back(r.get<uint64_t>());
                n *= t.dims.back();
            }
            t.type = r.get<uint32_t>();
            t.offset = r.get<uint64_t>();
            const uint64_t bs = block_size(t.type);
            t.size = (n + bs - 1) / bs * type_size(t.type);
            g->tensors.push_back(std::move(t));
        }
        if (!r.ok) {
            set_error("GGUF file %s is truncated or malformed", path);
            st = SSD_ERR_ARG;
            break;
        }
        uint32_t align = 32;
        as_u32(g->find("general.alignment"), &align);
        if (align == 0) align = 32;
        const uint64_t pos = (uint64_t)ftell(f);
        g->data_offset = (pos + align - 1) / align * align;
    } while (false);
    fclose(f);
    if (st != SSD_OK) {
        delete g;
        return st;
    }
    *out = g;
    return SSD_OK;
}

extern "C" int ssd_gguf_close(ssd_gguf* g) {
    delete g;
    return SSD_OK;
}

extern "C" int ssd_gguf_info(const ssd_gguf* g, uint32_t* version, uint64_t* n_tensors,
                             uint64_t* n_kv, uint64_t* data_offset) {
    SSD_REQ(g, SSD_ERR_ARG, "null file");
    if (version) *version = g->version;
    if (n_tensors) *n_tensors = g->n_tensors;
    if (n_kv) *n_kv = g->n_kv;
    if (data_offset) *data_offset = g->data_offset;
    return SSD_OK;
}

extern "C" int ssd_gguf_tensor(const ssd_gguf* g, uint64_t i, char* name, size_t cap,
                               uint32_t* n_dims, uint64_t dims[8], uint32_t* type,
                               uint64_t* offset, uint64_t* size_bytes) {
    SSD_REQ(g && i < g->tensors.size(), SSD_ERR_ARG, "tensor index out of range");
    const Tensor& t = g->tensors[i];
    if (name && cap) {
        const size_t n = t.name.size() < cap - 1 ? t.name.size() : cap - 1;
        memcpy(name, t.name.data(), n);
        name[n] = '\0';
    }
    if (n_dims) *n_dims = (uint32_t)t.dims.size();
    if (dims)
        for (size_t d = 0; d < t.dims.size(); d++) dims[d] = t.dims[d];
    if (type) *type = t.type;
    if (offset) *offset = t.offset;
    if (size_bytes) *size_bytes = t.size;
    return SSD_OK;
}

extern "C" int ssd_gguf_find(const ssd_gguf* g, const char* name, int64_t* index) {
    SSD_REQ(g && name && index, SSD_ERR_ARG, "null argument");
    *index = -1;
    for (size_t i = 0; i < g->tensors.size(); i++)
        if (g->tensors[i].name == name) {
            *index = (int64_t)i;
            break;
        }
    return SSD_OK;
}

// Metadata lookups: *found = 0 when the key is absent or of another type (the
// reference's Option::None), else the value.
extern "C" int ssd_gguf_get_u32(const ssd_gguf* g, const char* key, int* found, uint32_t* v) {
    SSD_REQ(g && key && found && v, SSD_ERR_ARG, "null argument");
    *found = as_u32(g->find(key), v) ? 1 : 0;
    return SSD_OK;
}
extern "C" int ssd_gguf_get_f32(const ssd_gguf* g, const char* key, int* found, float* v) {
    SSD_REQ(g && key && found && v, SSD_ERR_ARG, "null argument");
    const Meta* m = g->find(key);  // MetadataValue::as_f32: Float32 only (gguf.rs:200-205)
    *found = m && m->type == M_F32;
    if (*found) *v = (float)m->f;
    return SSD_OK;
}
extern "C" int ssd_gguf_get_str(const ssd_gguf* g, const char* key, int* found, char* out,
                                size_t cap) {
    SSD_REQ(g && key && found && out && cap, SSD_ERR_ARG, "null argument");
    const Meta* m = g->find(key);
    *found = m && m->type == M_STR;
    out[0] = '\0';
    if (*found) {
        const size_t n = m->s.size() < cap - 1 ? m->s.size() : cap - 1;
        memcpy(out, m->s.data(), n);
        out[n] = '\0';
    }
    return SSD_OK;
}
extern "C" int ssd_gguf_array_len(const ssd_gguf* g, const char* key, int* found, uint64_t* n) {
    SSD_REQ(g && key && found && n, SSD_ERR_ARG, "null argument");
    const Meta* m = g->find(key);
    *found = m && m->type == M_ARR;
    *n = *found ? m->arr_len : 0;
    return SSD_OK;
}

extern "C" int ssd_gguf_read(const ssd_gguf* g, uint64_t i, void* dst, size_t bytes) {
    SSD_REQ(g && dst && i < g->tensors.size(), SSD_ERR_ARG, "bad tensor read");
    const Tensor& t = g->tensors[i];
    SSD_REQ(bytes == t.size, SSD_ERR_SHAPE, "%s: %zu bytes asked, tensor has %llu", t.name.c_str(),
            bytes, (unsigned long long)t.size);
    SSD_REQ(g->data_offset + t.offset + t.size <= g->file_size, SSD_ERR_ARG,
            "%s lies past the end of the file", t.name.c_str());
    FILE* f = fopen(g->path.c_str(), "rb");
    SSD_REQ(f != nullptr, SSD_ERR_ARG, "cannot reopen %s", g->path.c_str());
    const bool ok = fseeko(f, (off_t)(g->data_offset + t.offset), SEEK_SET) == 0 &&
                    fread(dst, 1, bytes, f) == bytes;
    fclose(f);
    SSD_REQ(ok, SSD_ERR_ARG, "short read of %s", t.name.c_str());
    return SSD_OK;
}

namespace {
const Tensor* tensor_named(const ssd_gguf* g, const std::string& name) {
    for (const Tensor& t : g->tensors)
        if (t.name == name) return &t;
    return nullptr;
}
}  // namespace

// The decode engine's config from the file: GgufFile::{n_layers, n_embd, n_head,
// n_head_kv, vocab_size} (gguf.rs:326-379) with their defaults, head_dim = n_embd /
// n_head, n_ff from the ffn_gate tensor, RoPE base {arch}.rope.freq_base (default
// DEFAULT_ROPE_THETA = 10000, transformer.rs:20-21), RMSNorm eps
// {arch}.attention.layer_norm_rms_epsilon (default 1e-5, the reference's constant), the
// weight types of blk.0.attn_q / output / token_embd (output falls back to token_embd,
// transformer.rs:690-700).
extern "C" int ssd_gguf_model_config(const ssd_gguf* g, int kv_capacity, int tp_rank,
                                     int tp_size, ssd_model_config* cfg) {
    SSD_REQ(g && cfg, SSD_ERR_ARG, "null argument");
    const Meta* am = g->find("general.architecture");
    const std::string arch = am && am->type == M_STR ? am->s : "unknown";
    auto u32 = [&](const char* suffix, uint32_t dflt) {
        uint32_t v = dflt;
        if (!as_u32(g->find((arch + suffix).c_str()), &v)) v = dflt;
        return v;
    };
    auto f32 = [&](const char* suffix, float dflt) {
        const Meta* m = g->find((arch + suffix).c_str());
        return m && m->type == M_F32 ? (float)m->f : dflt;
    };
    ssd_model_config c = {};
    c.n_layers = (int)u32(".block_count", 0);
    c.n_embd = (int)u32(".embedding_length", 0);
    c.n_head = (int)u32(".attention.head_count", 0);
    c.n_head_kv = (int)u32(".attention.head_count_kv", (uint32_t)c.n_head);
    SSD_REQ(c.n_layers > 0 && c.n_embd > 0 && c.n_head > 0 && c.n_embd % c.n_head == 0,
            SSD_ERR_SHAPE, "GGUF: missing or inconsistent %s.* dimensions", arch.c_str());
    c.head_dim = c.n_embd / c.n_head;
    const Tensor* q = tensor_named(g, "blk.0.attn_q.weight");
    const Tensor* gate = tensor_named(g, "blk.0.ffn_gate.weight");
    const Tensor* emb = tensor_named(g, "token_embd.weight");
    const Tensor* out = tensor_named(g, "output.weight");
    SSD_REQ(q && gate && emb, SSD_ERR_ARG, "GGUF: blk.0.attn_q / ffn_gate or token_embd missing");
    SSD_REQ(gate->dims.size() == 2, SSD_ERR_SHAPE, "GGUF: ffn_gate is not a matrix");
    c.n_ff = (int)gate->dims[1];
    uint64_t nv = 0;
    const Meta* tok = g->find("tokenizer.ggml.tokens");
    if (tok && tok->type == M_ARR) nv = tok->arr_len;
    if (nv == 0 && emb->dims.size() == 2) nv = emb->dims[1];
    c.vocab = (int)nv;
    c.wtype = (int)q->type;
    c.out_type = (int)(out ? out->type : emb->type);
    c.embd_type = (int)emb->type;
    c.kv_capacity = kv_capacity;
    c.theta = f32(".rope.freq_base", 10000.0f);
    c.eps = f32(".attention.layer_norm_rms_epsilon", 1e-5f);
    c.tp_rank = tp_rank;
    c.tp_size = tp_size;
    *cfg = c;
    return SSD_OK;
}

// Streams every tensor the decode engine holds from the file into the model (this rank's
// shard, HBM-resident): blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm,
// ffn_gate, ffn_up, ffn_down}.weight, token_embd, output_norm, and output (token_embd
// when the file has none). One tensor is in host memory at a time.
extern "C" int ssd_model_load_gguf(ssd_model* m, const ssd_gguf* g, int n_layers) {
    SSD_REQ(m && g && n_layers > 0, SSD_ERR_ARG, "bad argument");
    static const char* kLayer[] = {"attn_norm", "attn_q",   "attn_k", "attn_v", "attn_output",
                                   "ffn_norm",  "ffn_gate", "ffn_up", "ffn_down"};
    std::vector<uint8_t> buf;
    auto load = [&](const std::string& file_name, const char* model_name, int layer) {
        const Tensor* t = tensor_named(g, file_name);
        SSD_REQ(t != nullptr, SSD_ERR_ARG, "GGUF: tensor %s missing", file_name.c_str());
        buf.resize(t->size);
        SSD_TRY(ssd_gguf_read(g, (uint64_t)(t - g->tensors.data()), buf.data(), buf.size()));
        return ssd_model_set_tensor_typed(m, model_name, layer, buf.data(), buf.size(),
                                          (int)t->type);  // each tensor's own type
    };
    for (int l = 0; l < n_layers; l++)
        for (const char* nm : kLayer)
            SSD_TRY(load("blk." + std::to_string(l) + "." + nm + ".weight", nm, l));
    SSD_TRY(load("token_embd.weight", "token_embd", -1));
    SSD_TRY(load("output_norm.weight", "output_norm", -1));
    SSD_TRY(load(tensor_named(g, "output.weight") ? "output.weight" : "token_embd.weight",
                 "output", -1));
    return SSD_OK;
}
