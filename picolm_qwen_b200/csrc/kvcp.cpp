// kvcp.cpp -- KV-cache persistence in the C engine's KVCP file format
// (picolm/model.c:870-983: kvcache_save / kvcache_load), read from and written
// to a device cache in the library's layout.
//
// The layout on the device is the reference's ([n_layers][max_seq_len][kv_dim]
// fp16 per sequence), so the K rows 0..n_pos-1 of one layer are one contiguous
// range and the file's K section is a strided 2-D copy (height n_layers, row
// n_pos*kv_dim*2 bytes, pitch max_seq_len*kv_dim*2 bytes); the same for V.
// Files go through two pinned staging buffers, so the device copy of one chunk
// overlaps the file I/O of the other.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "picoattn.h"
#include "picoattn_internal.h"

namespace {

constexpr size_t kStageBytes = 32u << 20;  // per staging buffer

struct Shape {
    size_t kvd, row_bytes, layer_pitch;  // kv_dim, bytes per row, bytes per layer slab
    int n_layers, max_seq;
};

Shape shape_of(const picoattn_config_t& c) {
    Shape s{};
    s.kvd = (size_t)c.n_kv_heads * c.head_dim;
    s.row_bytes = s.kvd * 2;
    s.layer_pitch = (size_t)c.max_seq_len * s.row_bytes;
    s.n_layers = c.n_layers;
    s.max_seq = c.max_seq_len;
    return s;
}

// Two pinned buffers and an event each: chunk i goes through buffer i % 2.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool ok = false;
    Staging() {
        ok = cudaHostAlloc(&buf[0], kStageBytes, cudaHostAllocDefault) == cudaSuccess &&
             cudaHostAlloc(&buf[1], kStageBytes, cudaHostAllocDefault) == cudaSuccess &&
             cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming) == cudaSuccess;
    }
    ~Staging() {
        for (int i = 0; i < 2; i++) {
            if (ev[i]) cudaEventDestroy(ev[i]);
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
};

// The file's two sections as a list of (device address, bytes) pieces no
// larger than a staging buffer, in file order.
struct Piece {
    size_t dev_off;  // byte offset from the cache base
    size_t bytes;
    int kv;          // 0: K, 1: V
};

std::vector<Piece> pieces_of(const Shape& s, int n_pos) {
    std::vector<Piece> out;
    const size_t rows_per = std::max<size_t>(1, kStageBytes / s.row_bytes);
    for (int kv = 0; kv < 2; kv++)
        for (int l = 0; l < s.n_layers; l++)
            for (size_t r = 0; r < (size_t)n_pos; r += rows_per) {
                const size_t n = std::min(rows_per, (size_t)n_pos - r);
                out.push_back({(size_t)l * s.layer_pitch + r * s.row_bytes, n * s.row_bytes, kv});
            }
    return out;
}

int32_t check_cfg(const picoattn_config_t* cfg) {
    if (!cfg) return PICOATTN_EINVAL;
    return picoattn_config_check(cfg);
}

}  // namespace

extern "C" {

size_t picoattn_kvcp_bytes(const picoattn_config_t* cfg, int32_t n_pos) {
    if (check_cfg(cfg) != PICOATTN_OK || n_pos < 0) return 0;
    const Shape s = shape_of(*cfg);
    return 16 + 2 * (size_t)s.n_layers * (size_t)n_pos * s.row_bytes;
}

int32_t picoattn_kvcp_pack(const picoattn_config_t* cfg, int32_t n_pos, const uint16_t* k_cache,
                           const uint16_t* v_cache, void* dst, size_t dst_bytes, picoattn_stream_t stream) {
    int32_t st = check_cfg(cfg);
    if (st != PICOATTN_OK) return st;
    if (!k_cache || !v_cache || !dst) return PICOATTN_EINVAL;
    if (n_pos <= 0 || n_pos > cfg->max_seq_len) return PICOATTN_ERANGE;
    if (dst_bytes < picoattn_kvcp_bytes(cfg, n_pos)) return PICOATTN_ENOSPACE;
    const Shape s = shape_of(*cfg);
    auto* sm = static_cast<cudaStream_t>(stream);
    const uint32_t header[4] = {PICOATTN_KVCP_MAGIC, (uint32_t)n_pos, (uint32_t)s.n_layers, (uint32_t)s.kvd};
    uint8_t* d = static_cast<uint8_t*>(dst);
    const size_t sec = (size_t)s.n_layers * n_pos * s.row_bytes;
    cudaError_t e = cudaMemcpyAsync(d, header, sizeof header, cudaMemcpyDefault, sm);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(d + 16, (size_t)n_pos * s.row_bytes, k_cache, s.layer_pitch, (size_t)n_pos * s.row_bytes,
                              (size_t)s.n_layers, cudaMemcpyDefault, sm);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(d + 16 + sec, (size_t)n_pos * s.row_bytes, v_cache, s.layer_pitch,
                              (size_t)n_pos * s.row_bytes, (size_t)s.n_layers, cudaMemcpyDefault, sm);
    // the header came from the stack: it must have been read before returning
    if (e == cudaSuccess) e = cudaStreamSynchronize(sm);
    return e == cudaSuccess ? PICOATTN_OK : PICOATTN_ECUDA;
}

int32_t picoattn_kvcp_unpack(const picoattn_config_t* cfg, const void* src, size_t src_bytes, uint16_t* k_cache,
                             uint16_t* v_cache, int32_t* n_pos_out, picoattn_stream_t stream) {
    if (n_pos_out) *n_pos_out = 0;
    int32_t st = check_cfg(cfg);
    if (st != PICOATTN_OK) return st;
    if (!src || !k_cache || !v_cache || !n_pos_out) return PICOATTN_EINVAL;
    if (src_bytes < 16) return PICOATTN_EFORMAT;
    const Shape s = shape_of(*cfg);
    auto* sm = static_cast<cudaStream_t>(stream);
    uint32_t h[4];
    if (cudaMemcpyAsync(h, src, sizeof h, cudaMemcpyDefault, sm) != cudaSuccess || cudaStreamSynchronize(sm) != cudaSuccess)
        return PICOATTN_ECUDA;
    if (h[0] != PICOATTN_KVCP_MAGIC || h[2] != (uint32_t)s.n_layers || h[3] != (uint32_t)s.kvd ||
        h[1] > (uint32_t)s.max_seq)
        return PICOATTN_EFORMAT;
    const int n_pos = (int)h[1];
    if (src_bytes < picoattn_kvcp_bytes(cfg, n_pos)) return PICOATTN_EFORMAT;
    if (n_pos > 0) {
        const uint8_t* p = static_cast<const uint8_t*>(src) + 16;
        const size_t w = (size_t)n_pos * s.row_bytes, sec = (size_t)s.n_layers * w;
        cudaError_t e = cudaMemcpy2DAsync(k_cache, s.layer_pitch, p, w, w, (size_t)s.n_layers, cudaMemcpyDefault, sm);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(v_cache, s.layer_pitch, p + sec, w, w, (size_t)s.n_layers, cudaMemcpyDefault, sm);
        if (e != cudaSuccess) return PICOATTN_ECUDA;
    }
    *n_pos_out = n_pos;
    return PICOATTN_OK;
}

int32_t picoattn_kvcp_save(const picoattn_config_t* cfg, int32_t n_pos, const uint16_t* k_cache,
                           const uint16_t* v_cache, const char* path, picoattn_stream_t stream) {
    int32_t st = check_cfg(cfg);
    if (st != PICOATTN_OK) return st;
    if (!k_cache || !v_cache || !path) return PICOATTN_EINVAL;
    if (n_pos <= 0 || n_pos > cfg->max_seq_len) return PICOATTN_ERANGE;
    const Shape s = shape_of(*cfg);
    auto* sm = static_cast<cudaStream_t>(stream);
    Staging sg;
    if (!sg.ok) return PICOATTN_ECUDA;
    FILE* f = std::fopen(path, "wb");
    if (!f) return PICOATTN_EIO;
    const uint32_t header[4] = {PICOATTN_KVCP_MAGIC, (uint32_t)n_pos, (uint32_t)s.n_layers, (uint32_t)s.kvd};
    bool io_ok = std::fwrite(header, sizeof(uint32_t), 4, f) == 4;
    const std::vector<Piece> ps = pieces_of(s, n_pos);
    const uint8_t* base[2] = {reinterpret_cast<const uint8_t*>(k_cache), reinterpret_cast<const uint8_t*>(v_cache)};
    cudaError_t e = cudaSuccess;
    // piece i is copied into buffer i % 2 while piece i - 1 is written out
    auto issue = [&](size_t i) {
        const Piece& p = ps[i];
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(sg.buf[i & 1], base[p.kv] + p.dev_off, p.bytes, cudaMemcpyDeviceToHost, sm);
        if (e == cudaSuccess) e = cudaEventRecord(sg.ev[i & 1], sm);
    };
    if (!ps.empty()) issue(0);
    for (size_t i = 0; i < ps.size() && e == cudaSuccess && io_ok; i++) {
        if (i + 1 < ps.size()) issue(i + 1);
        if (e == cudaSuccess) e = cudaEventSynchronize(sg.ev[i & 1]);
        if (e == cudaSuccess) io_ok = std::fwrite(sg.buf[i & 1], 1, ps[i].bytes, f) == ps[i].bytes;
    }
    if (e != cudaSuccess) cudaStreamSynchronize(sm);  // no copy into the staging may outlive it
    if (std::fclose(f) != 0) io_ok = false;
    if (e != cudaSuccess) return PICOATTN_ECUDA;
    return io_ok ? PICOATTN_OK : PICOATTN_EIO;
}

int32_t picoattn_kvcp_load(const picoattn_config_t* cfg, const char* path, uint16_t* k_cache, uint16_t* v_cache,
                           int32_t* n_pos_out, picoattn_stream_t stream) {
    if (n_pos_out) *n_pos_out = 0;
    int32_t st = check_cfg(cfg);
    if (st != PICOATTN_OK) return st;
    if (!path || !k_cache || !v_cache || !n_pos_out) return PICOATTN_EINVAL;
    const Shape s = shape_of(*cfg);
    FILE* f = std::fopen(path, "rb");
    if (!f) return PICOATTN_EIO;
    uint32_t h[4];
    if (std::fread(h, sizeof(uint32_t), 4, f) != 4) {
        std::fclose(f);
        return PICOATTN_EFORMAT;
    }
    if (h[0] != PICOATTN_KVCP_MAGIC || h[2] != (uint32_t)s.n_layers || h[3] != (uint32_t)s.kvd ||
        h[1] > (uint32_t)s.max_seq) {
        std::fclose(f);
        return PICOATTN_EFORMAT;
    }
    const int n_pos = (int)h[1];
    auto* sm = static_cast<cudaStream_t>(stream);
    Staging sg;
    if (!sg.ok) {
        std::fclose(f);
        return PICOATTN_ECUDA;
    }
    const std::vector<Piece> ps = pieces_of(s, n_pos);
    uint8_t* base[2] = {reinterpret_cast<uint8_t*>(k_cache), reinterpret_cast<uint8_t*>(v_cache)};
    cudaError_t e = cudaSuccess;
    bool io_ok = true;
    // piece i is read into buffer i % 2 once the upload of piece i - 2 has left it
    for (size_t i = 0; i < ps.size() && e == cudaSuccess && io_ok; i++) {
        if (i >= 2) e = cudaEventSynchronize(sg.ev[i & 1]);
        if (e != cudaSuccess) break;
        io_ok = std::fread(sg.buf[i & 1], 1, ps[i].bytes, f) == ps[i].bytes;
        if (!io_ok) break;
        e = cudaMemcpyAsync(base[ps[i].kv] + ps[i].dev_off, sg.buf[i & 1], ps[i].bytes, cudaMemcpyHostToDevice, sm);
        if (e == cudaSuccess) e = cudaEventRecord(sg.ev[i & 1], sm);
    }
    std::fclose(f);
    // the staging buffers are freed on return: every upload from them must be done
    const cudaError_t e2 = cudaStreamSynchronize(sm);
    if (e != cudaSuccess || e2 != cudaSuccess) return PICOATTN_ECUDA;
    if (!io_ok) return PICOATTN_EFORMAT;  // a short file
    *n_pos_out = n_pos;
    return PICOATTN_OK;
}

}  // extern "C"
