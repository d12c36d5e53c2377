// gguf.cu -- GGUF loader (host code): the file memory-mapped and parsed as
// the reference's GgufParser parses it (crates/parser/src/gguf.rs:239-592,
// crates/parser/src/mmap.rs:29-70 in SugarFreeDoNoSo/bml), and tensors
// copied into device memory through pinned staging buffers.
//
// Parsing keeps the reference's rules: a file of at least 24 bytes, magic
// 0x46554747, version <= 3; metadata value types 0-12 with arrays nesting;
// tensor types from GgufDataType::from_u32 (an unknown id fails the open);
// the data section starts at the end of the tensor infos rounded up to 32.
// Every read is bounds-checked against the mapping (the reference's
// "offset fuera de rango" errors).
//
// Upload.  A model's tensors are gigabytes read once: each of `threads`
// host threads (8 by default) owns one pinned staging buffer and one
// stream, copies a 32 MiB piece of the mapping into its buffer (the CPU
// read from the page cache, ~4-8 GB/s per thread) and queues its DMA to
// the device, so the pieces' page-in and memcpy run side by side and
// overlap the transfers of the others.  One cudaMemcpyAsync per piece.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/bml_gguf.h"
#include "common.cuh"

#define BML_API extern "C" __attribute__((visibility("default")))

namespace bml {
bml_status api_fail(bml_status st, const char *fmt, ...);
bml_status api_ok();
bml_status api_cuda_fail(cudaError_t e, const char *where);
}  // namespace bml

#define CUDA_TRY_API(call, what)                                    \
    do {                                                            \
        cudaError_t e_ = (call);                                    \
        if (e_ != cudaSuccess) return bml::api_cuda_fail(e_, what); \
    } while (0)

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;
constexpr uint32_t kGgufMaxVersion = 3;
constexpr uint64_t kAlign = 32;
constexpr size_t kPiece = 32u << 20;  // staging buffer size

struct Value {
    uint32_t type = 0, elem_type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    std::vector<Value> items;
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
};

// GgufDataType::from_u32 (gguf.rs:77-108): the tensor type ids the
// reference accepts.
bool tensor_type_known(uint32_t t) { return t <= 3 || (t >= 6 && t <= 29); }

// Fixed per-element size (GgufDataType::element_size, gguf.rs:132-143); 0
// for block-quantized types.
uint64_t element_size(uint32_t t) {
    switch (t) {
        case 0: case 26: return 4;   // F32, I32
        case 1: case 25: case 29: return 2;  // F16, I16, BF16
        case 24: return 1;           // I8
        case 27: case 28: return 8;  // I64, F64
        default: return 0;
    }
}

// GgufDataType::is_quantized (gguf.rs:145-170): the block types 2-23, and
// F16 / BF16 (which element_size catches first).
bool is_quantized(uint32_t t) { return (t >= 2 && t <= 23) || t == 1 || t == 29; }

// ggml block layouts: (values per block, bytes per block); (0, 0) where
// this library does not know the layout.
void block_layout(uint32_t t, uint64_t *vals, uint64_t *bytes) {
    static const struct { uint32_t t; uint64_t v, b; } tab[] = {
        {2, 32, 18}, {3, 32, 20}, {6, 32, 22}, {7, 32, 24}, {8, 32, 34}, {9, 32, 36},
        {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292},
    };
    *vals = 0;
    *bytes = 0;
    for (const auto &e : tab)
        if (e.t == t) {
            *vals = e.v;
            *bytes = e.b;
        }
}

struct Reader {
    const uint8_t *b;
    uint64_t n;
    std::string err;
    bool need(uint64_t off, uint64_t len, const char *what) {
        if (off > n || len > n - off) {
            err = std::string("offset out of range reading ") + what;
            return false;
        }
        return true;
    }
    template <typename T>
    T get(uint64_t off) const {
        T v;
        memcpy(&v, b + off, sizeof(T));
        return v;
    }
    bool str(uint64_t &off, std::string &out, const char *what) {  // decode_string
        if (!need(off, 8, what)) return false;
        const uint64_t len = get<uint64_t>(off);
        if (!need(off + 8, len, what)) return false;
        out.assign(reinterpret_cast<const char *>(b + off + 8), len);
        off += 8 + len;
        return true;
    }
    // decode_metadata_value (gguf.rs:415-545)
    bool value(uint64_t &off, uint32_t type, Value &v, int depth) {
        if (depth > 64) {  // (the reference recurses without a limit)
            err = "metadata arrays nested too deeply";
            return false;
        }
        v.type = type;
        switch (type) {
            case 0: if (!need(off, 1, "U8")) return false; v.u = b[off]; off += 1; return true;
            case 1: if (!need(off, 1, "I8")) return false; v.i = (int8_t)b[off]; off += 1; return true;
            case 2: if (!need(off, 2, "U16")) return false; v.u = get<uint16_t>(off); off += 2; return true;
            case 3: if (!need(off, 2, "I16")) return false; v.i = get<int16_t>(off); off += 2; return true;
            case 4: if (!need(off, 4, "U32")) return false; v.u = get<uint32_t>(off); off += 4; return true;
            case 5: if (!need(off, 4, "I32")) return false; v.i = get<int32_t>(off); off += 4; return true;
            case 6: if (!need(off, 4, "F32")) return false; v.f = get<float>(off); off += 4; return true;
            case 7: if (!need(off, 1, "Bool")) return false; v.u = b[off] != 0; off += 1; return true;
            case 8: return str(off, v.s, "string");
            case 10: if (!need(off, 8, "U64")) return false; v.u = get<uint64_t>(off); off += 8; return true;
            case 11: if (!need(off, 8, "I64")) return false; v.i = get<int64_t>(off); off += 8; return true;
            case 12: if (!need(off, 8, "F64")) return false; v.f = get<double>(off); off += 8; return true;
            case 9: {
                if (!need(off, 12, "array header")) return false;
                v.elem_type = get<uint32_t>(off);
                const uint64_t count = get<uint64_t>(off + 4);
                off += 12;
                // every element takes at least one byte: a count beyond the
                // file cannot be satisfied (and must not size a vector)
                if (count > n - off + 1 && count > 0) {
                    if (v.elem_type > 12) {
                        err = "unknown metadata type " + std::to_string(v.elem_type);
                        return false;
                    }
                    err = "offset out of range reading array element";
                    return false;
                }
                v.items.reserve(count < 4096 ? count : 4096);  // grows as elements parse
                for (uint64_t k = 0; k < count; ++k) {
                    v.items.emplace_back();
                    if (!value(off, v.elem_type, v.items.back(), depth + 1)) return false;
                }
                // the element type is checked after the elements, as the
                // reference does (an empty array of an unknown type fails too)
                if (v.elem_type > 12) {
                    err = "unknown array type " + std::to_string(v.elem_type);
                    return false;
                }
                return true;
            }
            default: err = "unknown metadata type " + std::to_string(type); return false;
        }
    }
};

}  // namespace

struct bml_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t size = 0;
    bml_gguf_header header{};
    std::vector<std::pair<std::string, Value>> meta;
    std::vector<Tensor> tensors;
    // upload staging
    std::vector<void *> staging;
    std::vector<cudaStream_t> streams;
    std::vector<cudaEvent_t> events;
    int staging_device = -1;
};

namespace {

void release(bml_gguf *g) {
    for (auto e : g->events) cudaEventDestroy(e);
    for (auto s : g->streams) cudaStreamDestroy(s);
    for (auto p : g->staging) cudaFreeHost(p);
    if (g->map && g->size) munmap(const_cast<uint8_t *>(g->map), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

uint64_t tensor_elems(const Tensor &t) {
    uint64_t n = 1;
    for (uint64_t d : t.dims) {
        if (d && n > UINT64_MAX / d) return UINT64_MAX;
        n *= d;
    }
    return n;
}

void describe(const bml_gguf *g, const Tensor &t, bml_gguf_tensor *o) {
    o->name = t.name.c_str();
    o->name_len = t.name.size();
    o->n_dims = (uint32_t)t.dims.size();
    o->dims = t.dims.data();
    o->type = t.type;
    o->offset = t.offset;
    o->present = 0;
    o->data_offset = 0;
    o->view_len = 0;
    o->nbytes = 0;
    const uint64_t n = tensor_elems(t);
    const uint64_t es = element_size(t.type);
    if (es) {
        o->nbytes = n > UINT64_MAX / es ? 0 : n * es;
    } else {
        uint64_t bv, bb;
        block_layout(t.type, &bv, &bb);
        if (bv && n % bv == 0 && n / bv <= UINT64_MAX / bb) o->nbytes = n / bv * bb;
    }
    // tensor_data (gguf.rs:339-364)
    const uint64_t start = g->header.data_offset + t.offset;
    if (t.offset > UINT64_MAX - g->header.data_offset || start > g->size) return;
    if (es) {
        if (o->nbytes == 0 && n != 0) return;
        if (o->nbytes > g->size - start) return;
        o->present = 1;
        o->data_offset = start;
        o->view_len = o->nbytes;
    } else if (is_quantized(t.type)) {
        o->present = 1;
        o->data_offset = start;
        o->view_len = g->size - start;
    }
}

const Value *walk(const Value &root, const uint64_t *path, uint32_t depth) {
    const Value *v = &root;
    for (uint32_t k = 0; k < depth; ++k) {
        if (v->type != BML_GGUF_META_ARRAY || path[k] >= v->items.size()) return nullptr;
        v = &v->items[path[k]];
    }
    return v;
}

}  // namespace

BML_API bml_status bml_gguf_open(const char *path, bml_gguf **out) {
    const char *fn = "bml_gguf_open";
    if (!path || !out) return bml::api_fail(BML_E_INVALID, "%s: null argument", fn);
    std::unique_ptr<bml_gguf, void (*)(bml_gguf *)> g(new bml_gguf, release);
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) return bml::api_fail(BML_E_INVALID, "%s: cannot open %s: %s", fn, path, strerror(errno));
    struct stat st;
    if (fstat(g->fd, &st) != 0) return bml::api_fail(BML_E_INVALID, "%s: fstat: %s", fn, strerror(errno));
    g->size = (uint64_t)st.st_size;
    if (g->size < 24) return bml::api_fail(BML_E_INVALID, "%s: file too small (%llu bytes)", fn, (unsigned long long)g->size);
    void *m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) return bml::api_fail(BML_E_INVALID, "%s: mmap: %s", fn, strerror(errno));
    g->map = static_cast<const uint8_t *>(m);
    Reader r{g->map, g->size, {}};
    g->header.magic = r.get<uint32_t>(0);
    g->header.version = r.get<uint32_t>(4);
    g->header.tensor_count = r.get<uint64_t>(8);
    g->header.metadata_kv_count = r.get<uint64_t>(16);
    g->header.file_size = g->size;
    if (g->header.magic != kGgufMagic)
        return bml::api_fail(BML_E_INVALID, "%s: bad magic 0x%08X", fn, g->header.magic);
    if (g->header.version > kGgufMaxVersion)
        return bml::api_fail(BML_E_INVALID, "%s: unsupported version %u", fn, g->header.version);
    uint64_t off = 24;
    // each KV and each tensor info takes at least 12 bytes: larger counts
    // cannot be satisfied and must not size a vector
    if (g->header.metadata_kv_count > g->size / 12 || g->header.tensor_count > g->size / 12)
        return bml::api_fail(BML_E_INVALID, "%s: offset out of range (counts beyond the file)", fn);
    g->meta.reserve(g->header.metadata_kv_count);
    for (uint64_t k = 0; k < g->header.metadata_kv_count; ++k) {
        std::string key;
        if (!r.str(off, key, "metadata key")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        if (!r.need(off, 4, "value type")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        const uint32_t type = r.get<uint32_t>(off);
        off += 4;
        Value v;
        if (!r.value(off, type, v, 0)) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        g->meta.emplace_back(std::move(key), std::move(v));
    }
    g->tensors.reserve(g->header.tensor_count);
    for (uint64_t k = 0; k < g->header.tensor_count; ++k) {  // decode_tensor_info
        Tensor t;
        if (!r.str(off, t.name, "tensor name")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        if (!r.need(off, 4, "n_dims")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        const uint32_t nd = r.get<uint32_t>(off);
        off += 4;
        if ((uint64_t)nd * 8 > g->size - off)
            return bml::api_fail(BML_E_INVALID, "%s: offset out of range reading dim", fn);
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; ++d, off += 8) t.dims[d] = r.get<uint64_t>(off);
        if (!r.need(off, 4, "data_type")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        t.type = r.get<uint32_t>(off);
        off += 4;
        if (!tensor_type_known(t.type)) return bml::api_fail(BML_E_INVALID, "%s: unknown tensor type %u", fn, t.type);
        if (!r.need(off, 8, "tensor offset")) return bml::api_fail(BML_E_INVALID, "%s: %s", fn, r.err.c_str());
        t.offset = r.get<uint64_t>(off);
        off += 8;
        g->tensors.push_back(std::move(t));
    }
    g->header.data_offset = (off + kAlign - 1) / kAlign * kAlign;
    *out = g.release();
    return bml::api_ok();
}

BML_API bml_status bml_gguf_close(bml_gguf *g) {
    if (!g) return bml::api_fail(BML_E_INVALID, "bml_gguf_close: null handle");
    if (g->staging_device >= 0) cudaSetDevice(g->staging_device);
    release(g);
    return bml::api_ok();
}

BML_API bml_status bml_gguf_get_header(const bml_gguf *g, bml_gguf_header *out) {
    if (!g || !out) return bml::api_fail(BML_E_INVALID, "bml_gguf_get_header: null argument");
    *out = g->header;
    return bml::api_ok();
}

BML_API bml_status bml_gguf_tensor_info(const bml_gguf *g, uint64_t index, bml_gguf_tensor *out) {
    if (!g || !out) return bml::api_fail(BML_E_INVALID, "bml_gguf_tensor_info: null argument");
    if (index >= g->tensors.size())
        return bml::api_fail(BML_E_INVALID, "bml_gguf_tensor_info: index %llu of %zu", (unsigned long long)index,
                             g->tensors.size());
    describe(g, g->tensors[index], out);
    return bml::api_ok();
}

BML_API bml_status bml_gguf_find_tensor(const bml_gguf *g, const char *name, uint64_t *index) {
    if (!g || !name || !index) return bml::api_fail(BML_E_INVALID, "bml_gguf_find_tensor: null argument");
    *index = UINT64_MAX;
    for (size_t k = 0; k < g->tensors.size(); ++k)
        if (g->tensors[k].name == name) {
            *index = k;
            break;
        }
    return bml::api_ok();
}

BML_API bml_status bml_gguf_tensor_view(const bml_gguf *g, uint64_t index, const void **ptr, uint64_t *len) {
    if (!g || !ptr || !len) return bml::api_fail(BML_E_INVALID, "bml_gguf_tensor_view: null argument");
    if (index >= g->tensors.size()) return bml::api_fail(BML_E_INVALID, "bml_gguf_tensor_view: bad index");
    bml_gguf_tensor t;
    describe(g, g->tensors[index], &t);
    *ptr = t.present ? g->map + t.data_offset : nullptr;
    *len = t.present ? t.view_len : 0;
    return bml::api_ok();
}

BML_API bml_status bml_gguf_meta_key(const bml_gguf *g, uint64_t index, const char **key, uint64_t *key_len) {
    if (!g || !key || !key_len) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_key: null argument");
    if (index >= g->meta.size()) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_key: bad index");
    *key = g->meta[index].first.c_str();
    *key_len = g->meta[index].first.size();
    return bml::api_ok();
}

BML_API bml_status bml_gguf_meta_find(const bml_gguf *g, const char *key, uint64_t *index) {
    if (!g || !key || !index) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_find: null argument");
    *index = UINT64_MAX;
    for (size_t k = 0; k < g->meta.size(); ++k)
        if (g->meta[k].first == key) *index = k;  // the last one wins, as in a HashMap
    return bml::api_ok();
}

BML_API bml_status bml_gguf_meta_value(const bml_gguf *g, uint64_t index, const uint64_t *path, uint32_t depth,
                                       bml_gguf_value *out) {
    if (!g || !out || (depth && !path)) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_value: null argument");
    if (index >= g->meta.size()) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_value: bad index");
    const Value *v = walk(g->meta[index].second, path, depth);
    if (!v) return bml::api_fail(BML_E_INVALID, "bml_gguf_meta_value: path does not address an element");
    out->type = v->type;
    out->elem_type = v->elem_type;
    out->len = v->type == BML_GGUF_META_ARRAY ? v->items.size() : v->s.size();
    out->u = v->u;
    out->i = v->i;
    out->f = v->f;
    out->str = v->type == BML_GGUF_META_STRING ? v->s.data() : nullptr;
    return bml::api_ok();
}

BML_API bml_status bml_gguf_upload(bml_gguf *g, const uint64_t *indices, uint32_t n, void *const *dev_dst,
                                   uint32_t threads) {
    const char *fn = "bml_gguf_upload";
    if (!g || (n && (!indices || !dev_dst))) return bml::api_fail(BML_E_INVALID, "%s: null argument", fn);
    // validate everything before copying anything
    struct Job {
        const uint8_t *src;
        uint8_t *dst;
        uint64_t len;
    };
    std::vector<Job> pieces;
    for (uint32_t k = 0; k < n; ++k) {
        if (indices[k] >= g->tensors.size()) return bml::api_fail(BML_E_INVALID, "%s: bad tensor index", fn);
        bml_gguf_tensor t;
        describe(g, g->tensors[indices[k]], &t);
        if (t.nbytes == 0 && tensor_elems(g->tensors[indices[k]]) != 0)
            return bml::api_fail(BML_E_UNSUPPORTED, "%s: %s: no known byte layout for type %u", fn, t.name, t.type);
        const uint64_t start = g->header.data_offset + g->tensors[indices[k]].offset;
        if (start > g->size || t.nbytes > g->size - start)
            return bml::api_fail(BML_E_INVALID, "%s: %s runs past the end of the file", fn, t.name);
        if (!dev_dst[k] && t.nbytes) return bml::api_fail(BML_E_INVALID, "%s: null destination", fn);
        for (uint64_t o = 0; o < t.nbytes; o += kPiece)
            pieces.push_back({g->map + start + o, static_cast<uint8_t *>(dev_dst[k]) + o,
                              std::min<uint64_t>(kPiece, t.nbytes - o)});
    }
    if (pieces.empty()) return bml::api_ok();
    int dev = 0;
    CUDA_TRY_API(cudaGetDevice(&dev), fn);
    const uint32_t nt = threads ? std::min<uint32_t>(threads, 16) : 8;
    if (g->staging_device != dev || g->staging.size() < nt) {  // (re)create the staging set on this device
        if (g->staging_device >= 0) {
            cudaSetDevice(g->staging_device);
            for (auto e : g->events) cudaEventDestroy(e);
            for (auto s : g->streams) cudaStreamDestroy(s);
            for (auto p : g->staging) cudaFreeHost(p);
            g->events.clear();
            g->streams.clear();
            g->staging.clear();
            cudaSetDevice(dev);
        }
        g->staging_device = dev;
        for (uint32_t t = 0; t < nt; ++t) {
            void *p = nullptr;
            cudaStream_t s;
            cudaEvent_t e;
            CUDA_TRY_API(cudaHostAlloc(&p, kPiece, cudaHostAllocDefault), fn);
            g->staging.push_back(p);
            CUDA_TRY_API(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), fn);
            g->streams.push_back(s);
            CUDA_TRY_API(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), fn);
            g->events.push_back(e);
        }
    }
    madvise(const_cast<uint8_t *>(g->map), g->size, MADV_SEQUENTIAL);
    std::atomic<cudaError_t> first_err{cudaSuccess};
    auto worker = [&](uint32_t t) {
        cudaError_t e = cudaSetDevice(dev);
        bool used = false;
        for (size_t k = t; k < pieces.size() && e == cudaSuccess; k += nt) {
            if (used) e = cudaEventSynchronize(g->events[t]);  // the buffer's previous DMA is done
            if (e != cudaSuccess) break;
            memcpy(g->staging[t], pieces[k].src, pieces[k].len);
            e = cudaMemcpyAsync(pieces[k].dst, g->staging[t], pieces[k].len, cudaMemcpyHostToDevice, g->streams[t]);
            if (e == cudaSuccess) e = cudaEventRecord(g->events[t], g->streams[t]);
            used = true;
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(g->streams[t]);
        cudaError_t expect = cudaSuccess;
        if (e != cudaSuccess) first_err.compare_exchange_strong(expect, e);
    };
    std::vector<std::thread> pool;
    for (uint32_t t = 1; t < nt; ++t) pool.emplace_back(worker, t);
    worker(0);
    for (auto &th : pool) th.join();
    if (first_err.load() != cudaSuccess) return bml::api_cuda_fail(first_err.load(), fn);
    return bml::api_ok();
}
