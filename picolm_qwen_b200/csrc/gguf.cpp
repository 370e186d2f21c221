// gguf.cpp -- GGUF model files to the device: the C++ engine's loader
// (Model::parse_gguf, cpp/model.hpp:705-902) restated on the host, and an
// upload of every tensor the forward uses into one caller-allocated device
// arena, so that picoattn_decode_block / picoattn_logits run a real model file.
//
// Parsing follows the reference exactly where it decides what a file means:
// the metadata keys it reads (by substring, cpp/gguf_metadata.hpp:241-275; only
// 32-bit integer and float values), the way it steps over every other value and
// over the tokenizer arrays (cpp/model.hpp:737-815), its defaults (RoPE base
// 1e4, context 2048, head_dim = n_embd / n_heads), the context cap (the
// override when smaller, else at most 2048), the tensor type's +1 shift
// (cpp/model.hpp:848), the data base rounded up to general.alignment (32 by
// default), the names it keeps (token_embd, output_norm, output, and
// blk.<l>.<key> with ".weight" removed: a bias stored as "blk.<l>.attn_q.bias"
// keeps that key and is not the engine's "attn_q_b"), the tied output matrix
// (output = token_embd when the file has none) and the vocabulary size from the
// embedding's shape.  The file is mapped read-only; nothing is written to it.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "picoattn.h"
#include "picoattn_internal.h"

using namespace picoattn;

struct picoattn_gguf {
    int fd = -1;
    const uint8_t* data = nullptr;
    size_t size = 0;
    picoattn_gguf_config_t cfg{};
    struct Tensor {
        size_t offset = 0;  // from the file's start
        size_t bytes = 0;
        int32_t type = 0;   // PICOATTN_WT_* numbering (the engine's GGUFType)
        int64_t n0 = 0;     // elements per row (dims[0])
        size_t arena = 0;   // offset of its bytes in the device arena
        size_t arena_f32 = SIZE_MAX;  // norms and biases: offset of the fp32 copy
    };
    std::map<std::string, Tensor> output;                 // token_embd, output_norm, output
    std::vector<std::map<std::string, Tensor>> layers;    // per layer, by the engine's keys
    size_t arena_bytes = 0;
};

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF"

// Block elements and bytes per block of a type (the engine's gguf_type_block_size
// / gguf_type_quant_size, cpp/quant.hpp:137-169), 0 for an unknown type.
void type_block(int32_t t, int* elems, int* bytes) {
    static const int tab[][3] = {{1, 1, 4},   {2, 1, 2},   {3, 32, 18},  {4, 32, 20},  {7, 32, 22},
                                 {8, 32, 24}, {9, 32, 34}, {10, 32, 40}, {11, 256, 84}, {12, 256, 110},
                                 {13, 256, 144}, {14, 256, 176}, {15, 256, 210}};
    *elems = *bytes = 0;
    for (const auto& r : tab)
        if (r[0] == t) *elems = r[1], *bytes = r[2];
}

// Keys whose tensors the engine dequantises into fp32 arrays once at load
// (norms and biases, cpp/model.hpp:924-1000): the arena holds an fp32 copy.
bool state_key(const std::string& k) {
    return k == "attn_norm" || k == "ffn_norm" || k == "output_norm" || k == "attn_q_norm" || k == "attn_k_norm" ||
           (k.size() > 2 && k.compare(k.size() - 2, 2, "_b") == 0);
}

struct Reader {
    const uint8_t* d;
    size_t n, pos = 0;
    bool ok = true;
    bool need(size_t k) {
        if (!ok || pos + k > n) ok = false;
        return ok;
    }
    uint32_t u32() {
        uint32_t v = 0;
        if (need(4)) std::memcpy(&v, d + pos, 4);
        pos += 4;
        return v;
    }
    uint64_t u64() {
        uint64_t v = 0;
        if (need(8)) std::memcpy(&v, d + pos, 8);
        pos += 8;
        return v;
    }
    float f32() {
        float v = 0;
        if (need(4)) std::memcpy(&v, d + pos, 4);
        pos += 4;
        return v;
    }
    std::string str(uint64_t len) {
        std::string s;
        if (len > n || !need((size_t)len)) return s;
        s.assign(reinterpret_cast<const char*>(d + pos), (size_t)len);
        pos += (size_t)len;
        return s;
    }
    void skip(uint64_t k) {
        if (k > n || !need((size_t)k)) return;
        pos += (size_t)k;
    }
};

// Steps over one value of a metadata type, as the engine's skip_value does
// (cpp/model.hpp:741-774).
void skip_value(Reader& r, uint32_t vtype) {
    auto scalar = [&](uint32_t t) {
        switch (t) {
            case 0: case 1: case 7: r.skip(1); break;
            case 2: case 3: r.skip(2); break;
            case 4: case 5: case 6: r.skip(4); break;
            case 10: case 11: case 12: r.skip(8); break;
            case 8: r.skip(r.u64()); break;
            default: break;
        }
    };
    if (vtype == 9) {
        const uint32_t et = r.u32();
        const uint64_t len = r.u64();
        for (uint64_t k = 0; k < len && r.ok; k++) scalar(et);
    } else {
        scalar(vtype);
    }
}

int32_t parse(picoattn_gguf* g, int32_t max_seq_override) {
    Reader r{g->data, g->size};
    if (r.u32() != kGgufMagic) return PICOATTN_EFORMAT;
    const uint32_t version = r.u32();
    if (version < 2 || version > 3) return PICOATTN_EFORMAT;
    const uint64_t n_tensors = r.u64(), n_meta = r.u64();
    if (!r.ok) return PICOATTN_EFORMAT;
    picoattn_gguf_config_t& c = g->cfg;
    c = picoattn_gguf_config_t{};
    c.rope_freq_base = 10000.0f;
    c.max_seq_len = 2048;
    c.head_dim = -1;
    c.alignment = 0;
    uint64_t n_tok_strings = 0;
    for (uint64_t i = 0; i < n_meta && r.ok; i++) {
        const std::string key = r.str(r.u64());
        const uint32_t vtype = r.u32();
        auto has = [&](const char* s) { return key.find(s) != std::string::npos; };
        if (has("tokenizer.ggml.bos_token_id") || has("tokenizer.ggml.eos_token_id")) {
            r.u32();  // read as 4 bytes whatever the stored type
        } else if (has("tokenizer.ggml.tokens")) {
            r.u32();
            const uint64_t len = r.u64();
            n_tok_strings = len;
            for (uint64_t k = 0; k < len && r.ok; k++) r.skip(r.u64());
        } else if (has("tokenizer.ggml.scores") || has("tokenizer.ggml.token_type")) {
            r.u32();
            r.skip(r.u64() * 4);
        } else if (has("tokenizer.ggml.pre")) {
            skip_value(r, vtype);
        } else if (vtype == 4 || vtype == 5) {
            const int32_t v = (int32_t)r.u32();
            // cpp/gguf_metadata.hpp:241-268
            if (has("embedding_length")) c.n_embd = v;
            else if (has("feed_forward_length")) c.n_ffn = v;
            else if (has("attention.head_count") && !has("_kv")) c.n_heads = v;
            else if (has("attention.head_count_kv")) c.n_kv_heads = v;
            else if (has("block_count")) c.n_layers = v;
            else if (has("context_length")) c.max_seq_len = v;
            else if (has("general.alignment")) c.alignment = v;
            else if (has("attention.key_length")) c.head_dim = v;
        } else if (vtype == 6) {
            const float v = r.f32();
            if (has("rope.freq_base")) c.rope_freq_base = v;
        } else {
            skip_value(r, vtype);
        }
    }
    if (!r.ok) return PICOATTN_EFORMAT;
    if (max_seq_override > 0 && max_seq_override < c.max_seq_len) c.max_seq_len = max_seq_override;
    else if (c.max_seq_len > 2048) c.max_seq_len = 2048;
    if (c.head_dim < 1 && c.n_heads > 0) c.head_dim = c.n_embd / c.n_heads;
    if (c.n_layers <= 0 || c.n_layers > 64 || c.n_embd <= 0 || c.n_heads <= 0) return PICOATTN_EFORMAT;
    if (c.n_kv_heads <= 0) c.n_kv_heads = c.n_heads;

    struct Info {
        std::string name;
        uint32_t n_dims;
        uint64_t dims[4];
        int32_t type;
        uint64_t offset;
    };
    std::vector<Info> infos((size_t)std::min<uint64_t>(n_tensors, 1u << 20));
    if (infos.size() != n_tensors) return PICOATTN_EFORMAT;
    for (auto& ti : infos) {
        ti.name = r.str(r.u64());
        ti.n_dims = r.u32();
        if (ti.n_dims > 4) return PICOATTN_EFORMAT;
        for (uint32_t d = 0; d < ti.n_dims; d++) ti.dims[d] = r.u64();
        ti.type = (int32_t)r.u32() + 1;  // the engine's numbering (cpp/model.hpp:848)
        ti.offset = r.u64();
        if (!r.ok) return PICOATTN_EFORMAT;
    }
    const size_t align = c.alignment > 0 ? (size_t)c.alignment : 32;
    const size_t base = (r.pos + align - 1) / align * align;
    g->layers.assign((size_t)c.n_layers, {});
    for (const auto& ti : infos) {
        picoattn_gguf::Tensor t;
        t.offset = base + ti.offset;
        t.type = ti.type;
        t.n0 = ti.n_dims > 0 ? (int64_t)ti.dims[0] : 1;
        int be, bb;
        type_block(t.type, &be, &bb);
        uint64_t rows = 1;
        for (uint32_t d = 1; d < ti.n_dims; d++) rows *= ti.dims[d];
        t.bytes = be ? (size_t)(t.n0 / be) * bb * rows : 0;
        if (t.bytes == 0 || t.offset + t.bytes > g->size || t.offset < base) return PICOATTN_EFORMAT;
        std::string nm = ti.name;
        const std::string wsfx = ".weight";
        if (nm.size() >= 6 && nm.compare(0, 4, "blk.") == 0) {
            const size_t dot = nm.find('.', 4);
            if (dot == std::string::npos) continue;
            int layer = -1;
            try {
                layer = std::stoi(nm.substr(4, dot - 4));
            } catch (...) {
                continue;
            }
            std::string key = nm.substr(dot + 1);
            if (key.size() > wsfx.size() && key.compare(key.size() - wsfx.size(), wsfx.size(), wsfx) == 0)
                key = key.substr(0, key.size() - wsfx.size());
            if (layer >= 0 && layer < c.n_layers) g->layers[(size_t)layer][key] = t;
        } else {
            std::string b = nm;
            if (b.size() >= wsfx.size() && b.compare(b.size() - wsfx.size(), wsfx.size(), wsfx) == 0)
                b = b.substr(0, b.size() - wsfx.size());
            if (b == "token_embd" || b == "output_norm" || b == "output") g->output[b] = t;
        }
    }
    if (!g->output.count("token_embd")) return PICOATTN_EFORMAT;
    if (!g->output.count("output")) g->output["output"] = g->output["token_embd"];
    c.vocab_size = 0;
    for (const auto& ti : infos) {
        if (ti.name == "token_embd.weight" && ti.n_dims >= 2) {
            c.vocab_size = ti.dims[0] == (uint64_t)c.n_embd ? (int32_t)ti.dims[1] : (int32_t)ti.dims[0];
            break;
        }
    }
    if (c.vocab_size == 0 && n_tok_strings > 0) c.vocab_size = (int32_t)n_tok_strings;
    // the device arena: every tensor's bytes, then fp32 copies of the norms and biases
    size_t off = 0;
    auto place = [&](picoattn_gguf::Tensor& t, const std::string& key) {
        t.arena = off;
        off = align_up(off + t.bytes, 256);
        if (state_key(key)) {
            t.arena_f32 = off;
            off = align_up(off + (size_t)t.n0 * 4, 256);
        }
    };
    for (auto& kv : g->output) place(kv.second, kv.first);
    for (auto& lm : g->layers)
        for (auto& kv : lm) place(kv.second, kv.first);
    g->arena_bytes = off;
    return PICOATTN_OK;
}

const picoattn_gguf::Tensor* find(const picoattn_gguf* g, int32_t layer, const char* key) {
    if (!g || !key) return nullptr;
    if (layer < 0) {
        auto it = g->output.find(key);
        return it == g->output.end() ? nullptr : &it->second;
    }
    if (layer >= (int32_t)g->layers.size()) return nullptr;
    auto it = g->layers[(size_t)layer].find(key);
    return it == g->layers[(size_t)layer].end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int32_t picoattn_gguf_open(const char* path, int32_t max_seq_len_override, picoattn_gguf_t** out) {
    if (!path || !out) return PICOATTN_EINVAL;
    *out = nullptr;
    auto* g = new picoattn_gguf();
    g->fd = open(path, O_RDONLY);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0 || st.st_size < 24) {
        if (g->fd >= 0) close(g->fd);
        delete g;
        return PICOATTN_EIO;
    }
    g->size = (size_t)st.st_size;
    void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
        close(g->fd);
        delete g;
        return PICOATTN_EIO;
    }
    g->data = static_cast<const uint8_t*>(m);
    const int32_t s = parse(g, max_seq_len_override);
    if (s != PICOATTN_OK) {
        picoattn_gguf_close(g);
        return s;
    }
    *out = g;
    return PICOATTN_OK;
}

int32_t picoattn_gguf_close(picoattn_gguf_t* g) {
    if (!g) return PICOATTN_EINVAL;
    if (g->data) munmap(const_cast<uint8_t*>(g->data), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return PICOATTN_OK;
}

int32_t picoattn_gguf_get_config(const picoattn_gguf_t* g, picoattn_gguf_config_t* cfg) {
    if (!g || !cfg) return PICOATTN_EINVAL;
    *cfg = g->cfg;
    return PICOATTN_OK;
}

int32_t picoattn_gguf_find(const picoattn_gguf_t* g, int32_t layer, const char* key, int32_t* type, size_t* bytes,
                           size_t* file_offset) {
    const picoattn_gguf::Tensor* t = find(g, layer, key);
    if (!t) return PICOATTN_ENOENT;
    if (type) *type = t->type;
    if (bytes) *bytes = t->bytes;
    if (file_offset) *file_offset = t->offset;
    return PICOATTN_OK;
}

size_t picoattn_gguf_arena_bytes(const picoattn_gguf_t* g) { return g ? g->arena_bytes : 0; }

int32_t picoattn_gguf_upload(const picoattn_gguf_t* g, void* arena, size_t arena_bytes, picoattn_stream_t stream) {
    if (!g || !arena || ((uintptr_t)arena & 255u)) return PICOATTN_EINVAL;
    if (arena_bytes < g->arena_bytes) return PICOATTN_ENOSPACE;
    uint8_t* dst = static_cast<uint8_t*>(arena);
    const cudaStream_t s = (cudaStream_t)stream;
    std::vector<float> f32;
    auto put = [&](const picoattn_gguf::Tensor& t) -> int32_t {
        int32_t st = cuda_status(cudaMemcpyAsync(dst + t.arena, g->data + t.offset, t.bytes, cudaMemcpyHostToDevice, s));
        if (st != PICOATTN_OK || t.arena_f32 == SIZE_MAX) return st;
        // the engine's dequantize_row into an fp32 array (norms and biases: F32 or F16)
        f32.resize((size_t)t.n0);
        if (t.type == PICOATTN_WT_F32) {
            std::memcpy(f32.data(), g->data + t.offset, (size_t)t.n0 * 4);
        } else if (t.type == PICOATTN_WT_F16) {
            for (int64_t i = 0; i < t.n0; i++) {
                uint16_t h;
                std::memcpy(&h, g->data + t.offset + 2 * i, 2);
                f32[(size_t)i] = __half2float(__ushort_as_half(h));
            }
        } else {
            return PICOATTN_EUNSUPPORTED;
        }
        st = cuda_status(cudaMemcpyAsync(dst + t.arena_f32, f32.data(), f32.size() * 4, cudaMemcpyHostToDevice, s));
        if (st == PICOATTN_OK) st = cuda_status(cudaStreamSynchronize(s));  // f32 is reused
        return st;
    };
    for (const auto& kv : g->output) {
        const int32_t st = put(kv.second);
        if (st != PICOATTN_OK) return st;
    }
    for (const auto& lm : g->layers)
        for (const auto& kv : lm) {
            const int32_t st = put(kv.second);
            if (st != PICOATTN_OK) return st;
        }
    return cuda_status(cudaStreamSynchronize(s));  // the mapped file is read by the copies
}

int32_t picoattn_gguf_arena_tensor(const picoattn_gguf_t* g, const void* arena, int32_t layer, const char* key,
                                   const void** dev_ptr, int32_t* type) {
    const picoattn_gguf::Tensor* t = find(g, layer, key);
    if (!t) return PICOATTN_ENOENT;
    if (!arena || !dev_ptr) return PICOATTN_EINVAL;
    const bool f32 = t->arena_f32 != SIZE_MAX;
    *dev_ptr = static_cast<const uint8_t*>(arena) + (f32 ? t->arena_f32 : t->arena);
    if (type) *type = f32 ? PICOATTN_WT_F32 : t->type;
    return PICOATTN_OK;
}

}  // extern "C"
