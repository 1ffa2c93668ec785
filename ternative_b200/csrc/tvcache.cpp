// The merged-weight cache file (.tvcache) written straight from device memory
// and read back into it.
//
// File layout (the reference's ModelCache format, include/ternative/cache.h:
// 28-62, writer src/cache.cpp:263-375, reader :378-470), kept byte-for-byte so
// either side reads the other's files:
//
//   [0, 256)          header: "TVCACHE\0", version, dtype, key (SHA-256 of the
//                     base and LoRA GGUF files, LoRA alpha and rank), tensor
//                     count, table offset (256), data offset, file size
//   [256, ...)        one 192-byte entry per tensor: name, ggml type, dims,
//                     shape (ggml order), offset in the data section, bytes
//   [data, ...)       tensor bytes, each tensor starting on a 64-byte boundary;
//                     the data section starts on a 4096-byte boundary
//
// Extension: per-row INT8 weights (the codes as ggml type 24, I8, plus an F32
// entry "<name>.row_scale") are written as version 2, which the reference's
// reader refuses instead of misreading; files without them are version 1.
//
// Device tensors are staged through two pinned buffers: the copy of chunk
// i + 1 runs while chunk i is written to (or read from) the file.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

#pragma pack(push, 1)
struct FileHeader {
    char magic[8];
    uint32_t version;
    uint32_t dtype;
    uint64_t base_size;
    uint8_t base_sha256[32];
    uint64_t lora_size;
    uint8_t lora_sha256[32];
    float lora_alpha;
    uint32_t lora_rank;
    uint32_t num_tensors;
    uint64_t table_offset;
    uint64_t data_offset;
    uint64_t total_size;
    uint8_t reserved[124];
};
struct FileTensor {
    char name[128];
    uint32_t dtype;
    uint32_t n_dims;
    uint64_t shape[4];
    uint64_t data_offset;
    uint64_t nbytes;
    uint8_t pad[8];
};
#pragma pack(pop)
static_assert(sizeof(FileHeader) == 256, "header is 256 bytes");
static_assert(sizeof(FileTensor) == 192, "table entry is 192 bytes");

constexpr uint32_t kTypeF32 = 0, kTypeF16 = 1, kTypeI8 = 24;
constexpr size_t kChunk = 32u << 20;   // staging chunk

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Whether p is device memory the runtime knows (host memory, or no GPU, is not).
bool on_device(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

// Two pinned staging buffers and a stream for device <-> file transfers.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    tvb_status init() {
        if (st) return TVB_OK;
        for (int i = 0; i < 2; ++i) {
            TVB_CUDA(cudaHostAlloc(&buf[i], kChunk, cudaHostAllocDefault));
            TVB_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
        }
        TVB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        return TVB_OK;
    }
    ~Staging() {
        if (st) cudaStreamSynchronize(st);
        for (int i = 0; i < 2; ++i) {
            if (buf[i]) cudaFreeHost(buf[i]);
            if (ev[i]) cudaEventDestroy(ev[i]);
        }
        if (st) cudaStreamDestroy(st);
    }
};

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

tvb_status write_bytes(FILE* f, const void* p, size_t n, const char* what) {
    if (n && fwrite(p, 1, n, f) != n) return tvb::set_error(TVB_ERR_INVALID, "tvcache: short write (%s)", what);
    return TVB_OK;
}

// One tensor's bytes to the file, from host memory or through the staging.
tvb_status write_tensor(FILE* f, const void* src, size_t n, Staging& sg) {
    if (!on_device(src)) return write_bytes(f, src, n, "tensor data");
    TVB_TRY(sg.init());
    const char* s = static_cast<const char*>(src);
    size_t done = 0;
    int cur = 0;
    size_t len = n < kChunk ? n : kChunk;
    TVB_CUDA(cudaMemcpyAsync(sg.buf[cur], s, len, cudaMemcpyDeviceToHost, sg.st));
    TVB_CUDA(cudaEventRecord(sg.ev[cur], sg.st));
    while (done < n) {
        const size_t next = done + len;
        size_t nlen = 0;
        if (next < n) {   // the next chunk's copy overlaps this chunk's write
            nlen = n - next < kChunk ? n - next : kChunk;
            TVB_CUDA(cudaMemcpyAsync(sg.buf[cur ^ 1], s + next, nlen, cudaMemcpyDeviceToHost, sg.st));
            TVB_CUDA(cudaEventRecord(sg.ev[cur ^ 1], sg.st));
        }
        TVB_CUDA(cudaEventSynchronize(sg.ev[cur]));
        TVB_TRY(write_bytes(f, sg.buf[cur], len, "tensor data"));
        done = next;
        len = nlen;
        cur ^= 1;
    }
    return TVB_OK;
}

// n bytes from the file's position into dst: host memory directly, device
// memory through the staging (the upload of chunk i overlaps the read of
// chunk i + 1).  The staging belongs to the open file and is pinned once, on
// its first device read.
tvb_status read_into(FILE* f, void* dst, uint64_t n, const char* name, Staging& sg) {
    if (!on_device(dst)) {
        if (std::fread(dst, 1, n, f) != n) return tvb::set_error(TVB_ERR_INVALID, "short read of '%s'", name);
        return TVB_OK;
    }
    TVB_TRY(sg.init());
    char* d = static_cast<char*>(dst);
    size_t done = 0;
    int cur = 0;
    while (done < n) {
        const size_t len = n - done < kChunk ? n - done : kChunk;
        TVB_CUDA(cudaEventSynchronize(sg.ev[cur]));   // the buffer's previous upload is done
        if (std::fread(sg.buf[cur], 1, len, f) != len)
            return tvb::set_error(TVB_ERR_INVALID, "short read of '%s'", name);
        TVB_CUDA(cudaMemcpyAsync(d + done, sg.buf[cur], len, cudaMemcpyHostToDevice, sg.st));
        TVB_CUDA(cudaEventRecord(sg.ev[cur], sg.st));
        done += len;
        cur ^= 1;
    }
    TVB_CUDA(cudaStreamSynchronize(sg.st));
    return TVB_OK;
}

}  // namespace

struct tvb_cache {
    Staging sg;   // destroyed after the file: declared first
    File file;
    FileHeader hdr;
    std::vector<FileTensor> table;
    std::string path;
};

extern "C" {

tvb_status tvb_cache_write(const char* path, const tvb_cache_key* key, const tvb_cache_tensor* tensors, int n) {
    TVB_REQUIRE(path && key && (tensors || n == 0) && n >= 0, "cache_write: bad arguments");
    // table: every tensor, and a row-scale entry after each per-row INT8 one
    std::vector<FileTensor> table;
    std::vector<const void*> src;
    bool int8 = false;
    uint64_t off = 0;
    auto add = [&](const char* name, uint32_t type, int n_dims, const int64_t* shape, uint64_t nbytes,
                   const void* data) -> tvb_status {
        FileTensor e;
        std::memset(&e, 0, sizeof(e));
        TVB_REQUIRE(std::strlen(name) < sizeof(e.name), "cache_write: tensor name '%s' too long", name);
        std::strncpy(e.name, name, sizeof(e.name) - 1);
        e.dtype = type;
        e.n_dims = (uint32_t)n_dims;
        for (int d = 0; d < n_dims; ++d) e.shape[d] = (uint64_t)shape[d];
        e.data_offset = off;
        e.nbytes = nbytes;
        off = align_up(off + nbytes, 64);
        table.push_back(e);
        src.push_back(data);
        return TVB_OK;
    };
    for (int i = 0; i < n; ++i) {
        const tvb_cache_tensor& t = tensors[i];
        TVB_REQUIRE(t.name && t.n_dims >= 1 && t.n_dims <= 4 && t.data, "cache_write: tensor %d incomplete", i);
        uint64_t count = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            TVB_REQUIRE(t.shape[d] > 0, "cache_write: tensor '%s' dim %d is %lld", t.name, d, (long long)t.shape[d]);
            count *= (uint64_t)t.shape[d];
        }
        if (t.ggml_type == (int)kTypeI8) {
            TVB_REQUIRE(t.n_dims == 2 && t.row_scales, "cache_write: INT8 tensor '%s' needs 2 dims and row scales",
                        t.name);
            TVB_TRY(add(t.name, kTypeI8, 2, t.shape, count, t.data));
            const std::string sname = std::string(t.name) + ".row_scale";
            const int64_t rows[1] = {t.shape[1]};
            TVB_TRY(add(sname.c_str(), kTypeF32, 1, rows, (uint64_t)t.shape[1] * 4, t.row_scales));
            int8 = true;
        } else {
            TVB_REQUIRE(t.ggml_type == (int)kTypeF16 || t.ggml_type == (int)kTypeF32,
                        "cache_write: tensor '%s' type %d (F32, F16 or I8)", t.name, t.ggml_type);
            TVB_TRY(add(t.name, (uint32_t)t.ggml_type, t.n_dims, t.shape,
                        count * (t.ggml_type == (int)kTypeF16 ? 2 : 4), t.data));
        }
    }
    FileHeader h;
    std::memset(&h, 0, sizeof(h));
    std::memcpy(h.magic, "TVCACHE\0", 8);
    h.version = int8 ? 2u : 1u;
    h.dtype = int8 ? 2u : 1u;
    h.base_size = key->base_size;
    std::memcpy(h.base_sha256, key->base_sha256, 32);
    h.lora_size = key->lora_size;
    std::memcpy(h.lora_sha256, key->lora_sha256, 32);
    h.lora_alpha = key->lora_alpha;
    h.lora_rank = key->lora_rank;
    h.num_tensors = (uint32_t)table.size();
    h.table_offset = sizeof(FileHeader);
    h.data_offset = align_up(sizeof(FileHeader) + table.size() * sizeof(FileTensor), 4096);
    h.total_size = h.data_offset + off;

    // written to <path>.tmp, renamed over <path> once complete
    const std::string tmp = std::string(path) + ".tmp";
    Staging sg;
    {
        File f;
        f.f = std::fopen(tmp.c_str(), "wb");
        TVB_REQUIRE(f.f, "cache_write: cannot create %s", tmp.c_str());
        TVB_TRY(write_bytes(f.f, &h, sizeof(h), "header"));
        TVB_TRY(write_bytes(f.f, table.data(), table.size() * sizeof(FileTensor), "table"));
        static const char zeros[4096] = {};
        TVB_TRY(write_bytes(f.f, zeros, h.data_offset - sizeof(h) - table.size() * sizeof(FileTensor), "padding"));
        for (size_t i = 0; i < table.size(); ++i) {
            TVB_TRY(write_tensor(f.f, src[i], table[i].nbytes, sg));
            TVB_TRY(write_bytes(f.f, zeros, align_up(table[i].nbytes, 64) - table[i].nbytes, "padding"));
        }
        const bool ok = std::fflush(f.f) == 0;
        std::fclose(f.f);
        f.f = nullptr;
        if (!ok) {
            std::remove(tmp.c_str());
            return tvb::set_error(TVB_ERR_INVALID, "cache_write: flush of %s failed", tmp.c_str());
        }
    }
    std::remove(path);
    if (std::rename(tmp.c_str(), path) != 0) {
        std::remove(tmp.c_str());
        return tvb::set_error(TVB_ERR_INVALID, "cache_write: rename to %s failed", path);
    }
    return TVB_OK;
}

tvb_status tvb_cache_open(const char* path, tvb_cache** out) {
    TVB_REQUIRE(path && out, "cache_open: null argument");
    *out = nullptr;
    auto* c = new (std::nothrow) tvb_cache();
    if (!c) return tvb::set_error(TVB_ERR_OOM, "cache_open: host allocation");
    c->path = path;
    c->file.f = std::fopen(path, "rb");
    auto fail = [&](tvb_status s) {
        delete c;
        return s;
    };
    if (!c->file.f) return fail(tvb::set_error(TVB_ERR_INVALID, "cache_open: cannot open %s", path));
    if (std::fread(&c->hdr, 1, sizeof(c->hdr), c->file.f) != sizeof(c->hdr) ||
        std::memcmp(c->hdr.magic, "TVCACHE\0", 8) != 0)
        return fail(tvb::set_error(TVB_ERR_INVALID, "cache_open: %s is not a .tvcache file", path));
    if (c->hdr.version != 1 && c->hdr.version != 2)
        return fail(tvb::set_error(TVB_ERR_INVALID, "cache_open: version %u", c->hdr.version));
    c->table.resize(c->hdr.num_tensors);
    if (std::fseek(c->file.f, (long)c->hdr.table_offset, SEEK_SET) != 0 ||
        std::fread(c->table.data(), sizeof(FileTensor), c->table.size(), c->file.f) != c->table.size())
        return fail(tvb::set_error(TVB_ERR_INVALID, "cache_open: truncated tensor table in %s", path));
    for (auto& e : c->table) {
        e.name[sizeof(e.name) - 1] = 0;
        // bounds written so that no file-supplied sum can wrap around
        const uint64_t size = c->hdr.total_size, base = c->hdr.data_offset;
        if (e.n_dims > 4 || base > size || e.data_offset > size - base || e.nbytes > size - base - e.data_offset)
            return fail(tvb::set_error(TVB_ERR_INVALID, "cache_open: entry '%s' out of range", e.name));
    }
    *out = c;
    return TVB_OK;
}

int tvb_cache_count(const tvb_cache* c) { return c ? (int)c->table.size() : 0; }

tvb_status tvb_cache_info(const tvb_cache* c, tvb_cache_key* key, int* version) {
    TVB_REQUIRE(c, "cache_info: null cache");
    if (key) {
        key->base_size = c->hdr.base_size;
        std::memcpy(key->base_sha256, c->hdr.base_sha256, 32);
        key->lora_size = c->hdr.lora_size;
        std::memcpy(key->lora_sha256, c->hdr.lora_sha256, 32);
        key->lora_alpha = c->hdr.lora_alpha;
        key->lora_rank = c->hdr.lora_rank;
    }
    if (version) *version = (int)c->hdr.version;
    return TVB_OK;
}

tvb_status tvb_cache_entry(const tvb_cache* c, int i, tvb_cache_tensor* info, uint64_t* nbytes) {
    TVB_REQUIRE(c && info && i >= 0 && i < (int)c->table.size(), "cache_entry: bad arguments");
    const FileTensor& e = c->table[i];
    std::memset(info, 0, sizeof(*info));
    info->name = e.name;
    info->ggml_type = (int)e.dtype;
    info->n_dims = (int)e.n_dims;
    for (uint32_t d = 0; d < e.n_dims; ++d) info->shape[d] = (int64_t)e.shape[d];
    if (nbytes) *nbytes = e.nbytes;
    return TVB_OK;
}

tvb_status tvb_cache_read(tvb_cache* c, const char* name, void* dst, uint64_t capacity) {
    TVB_REQUIRE(c && name && dst, "cache_read: null argument");
    const FileTensor* e = nullptr;
    for (const auto& t : c->table)
        if (std::strcmp(t.name, name) == 0) e = &t;
    TVB_REQUIRE(e, "cache_read: no tensor '%s' in %s", name, c->path.c_str());
    TVB_REQUIRE(capacity >= e->nbytes, "cache_read: '%s' needs %llu bytes, destination has %llu", name,
                (unsigned long long)e->nbytes, (unsigned long long)capacity);
    if (std::fseek(c->file.f, (long)(c->hdr.data_offset + e->data_offset), SEEK_SET) != 0)
        return tvb::set_error(TVB_ERR_INVALID, "cache_read: seek failed for '%s'", name);
    return read_into(c->file.f, dst, e->nbytes, name, c->sg);
}

tvb_status tvb_cache_close(tvb_cache* c) {
    delete c;
    return TVB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// GGUF ingest: the tensor table of a GGUF v3 file (gguf.cpp's
// gguf_parse_buffer: header, metadata key/values, tensor infos, the data
// section at general.alignment) read without loading the file, and single
// tensors streamed from the file into device (or host) memory through the
// same pinned staging -- instead of gguf_load's copy of the whole file into
// host memory before anything reaches the GPU.  Byte sizes follow the
// reference's Tensor (tensor.cpp:108-121): F32 4, F16 / BF16 2 bytes per
// element, I2_S 32 bytes per 128 weights plus the F32 scale.
// ---------------------------------------------------------------------------
struct tvb_gguf {
    Staging sg;
    File file;
    std::string path;
    struct Info {
        std::string name;
        uint32_t type;
        std::vector<uint64_t> shape;
        uint64_t offset, nbytes;
    };
    std::vector<Info> tensors;
    uint64_t data_offset = 0;
    uint64_t file_size = 0;
};

namespace {

bool rd(FILE* f, void* p, size_t n) { return std::fread(p, 1, n, f) == n; }

bool rd_string(FILE* f, std::string* out) {
    uint64_t n = 0;
    if (!rd(f, &n, 8) || n > (1ull << 30)) return false;
    if (!out) return std::fseek(f, (long)n, SEEK_CUR) == 0;
    out->resize(n);
    return n == 0 || rd(f, &(*out)[0], n);
}

// Skip (or read, for the one key the layout needs) one metadata value of type t.
bool skip_value(FILE* f, uint32_t t, int depth, uint64_t* u32_out) {
    static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t > 12 || depth > 4) return false;
    if (t == 8) return rd_string(f, nullptr);
    if (t == 9) {
        uint32_t et = 0;
        uint64_t n = 0;
        if (!rd(f, &et, 4) || !rd(f, &n, 8) || et > 12) return false;
        if (et != 8 && et != 9) return std::fseek(f, (long)(n * (uint64_t)sizes[et]), SEEK_CUR) == 0;
        for (uint64_t i = 0; i < n; ++i)
            if (!skip_value(f, et, depth + 1, nullptr)) return false;
        return true;
    }
    if (u32_out && t == 4) {
        uint32_t v = 0;
        if (!rd(f, &v, 4)) return false;
        *u32_out = v;
        return true;
    }
    return std::fseek(f, sizes[t], SEEK_CUR) == 0;
}

// Byte size of n elements of a ggml type; false for a type this reader does
// not size, or for a count whose size does not fit 64 bits.
bool gguf_bytes(uint32_t type, uint64_t n, uint64_t* out) {
    switch (type) {
        case 0: if (n > UINT64_MAX / 4) return false; *out = n * 4; return true;              // F32
        case 1: case 30: if (n > UINT64_MAX / 2) return false; *out = n * 2; return true;     // F16, BF16
        case 36: *out = (n / 128 + (n % 128 != 0)) * 32 + 4; return n <= UINT64_MAX / 2;     // I2_S + F32 scale
        default: return false;
    }
}

}  // namespace

extern "C" {

tvb_status tvb_gguf_open(const char* path, tvb_gguf** out) {
    TVB_REQUIRE(path && out, "gguf_open: null argument");
    *out = nullptr;
    auto* g = new (std::nothrow) tvb_gguf();
    if (!g) return tvb::set_error(TVB_ERR_OOM, "gguf_open: host allocation");
    auto fail = [&](const char* why) {
        delete g;
        return tvb::set_error(TVB_ERR_INVALID, "gguf_open: %s: %s", path, why);
    };
    g->path = path;
    g->file.f = std::fopen(path, "rb");
    if (!g->file.f) return fail("cannot open");
    FILE* f = g->file.f;
    std::fseek(f, 0, SEEK_END);
    g->file_size = (uint64_t)std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    uint32_t magic = 0, version = 0;
    uint64_t n_tensors = 0, n_kv = 0;
    if (!rd(f, &magic, 4) || magic != 0x46554747u) return fail("not a GGUF file");
    if (!rd(f, &version, 4) || version != 3) return fail("GGUF version is not 3");
    if (!rd(f, &n_tensors, 8) || !rd(f, &n_kv, 8) || n_tensors > 1000000) return fail("bad header");
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        uint32_t t = 0;
        if (!rd_string(f, &key) || !rd(f, &t, 4)) return fail("truncated metadata");
        uint64_t v = 0;
        const bool want = key == "general.alignment";
        if (!skip_value(f, t, 0, want ? &v : nullptr)) return fail("bad metadata value");
        if (want && t == 4 && v > 0) {
            // the reference rounds with any alignment (gguf.cpp:299-304); a cap of
            // 1 MiB keeps the rounding from wrapping
            if (v > (1u << 20)) return fail("general.alignment above 1 MiB");
            alignment = v;
        }
    }
    g->tensors.resize(n_tensors);
    for (auto& ti : g->tensors) {
        uint32_t nd = 0;
        // up to 8 dimensions, the reference parser's cap (gguf.cpp:286-287)
        if (!rd_string(f, &ti.name) || !rd(f, &nd, 4) || nd > 8) return fail("bad tensor info");
        ti.shape.resize(nd);
        uint64_t n = 1;
        for (auto& d : ti.shape) {
            if (!rd(f, &d, 8)) return fail("bad tensor info");
            if (d != 0 && n > UINT64_MAX / d) return fail("tensor element count overflows");
            n *= d;
        }
        if (!rd(f, &ti.type, 4) || !rd(f, &ti.offset, 8)) return fail("bad tensor info");
        if (!gguf_bytes(ti.type, n, &ti.nbytes)) ti.nbytes = 0;   // a type this reader does not size
    }
    const uint64_t pos = (uint64_t)std::ftell(f);
    g->data_offset = (pos + alignment - 1) / alignment * alignment;
    *out = g;
    return TVB_OK;
}

int tvb_gguf_count(const tvb_gguf* g) { return g ? (int)g->tensors.size() : 0; }

tvb_status tvb_gguf_tensor(const tvb_gguf* g, int i, tvb_cache_tensor* info, uint64_t* nbytes) {
    TVB_REQUIRE(g && info && i >= 0 && i < (int)g->tensors.size(), "gguf_tensor: bad arguments");
    const auto& t = g->tensors[i];
    std::memset(info, 0, sizeof(*info));
    info->name = t.name.c_str();
    info->ggml_type = (int)t.type;
    if (t.shape.size() > 4)
        return tvb::set_error(TVB_ERR_UNSUPPORTED, "gguf_tensor: '%s' has %d dimensions (tvb_cache_tensor holds 4)",
                              t.name.c_str(), (int)t.shape.size());
    info->n_dims = (int)t.shape.size();
    for (int d = 0; d < info->n_dims; ++d) info->shape[d] = (int64_t)t.shape[d];
    if (nbytes) *nbytes = t.nbytes;
    return TVB_OK;
}

tvb_status tvb_gguf_read(tvb_gguf* g, const char* name, void* dst, uint64_t capacity) {
    TVB_REQUIRE(g && name && dst, "gguf_read: null argument");
    const tvb_gguf::Info* t = nullptr;
    for (const auto& x : g->tensors)
        if (x.name == name) t = &x;
    TVB_REQUIRE(t, "gguf_read: no tensor '%s' in %s", name, g->path.c_str());
    TVB_REQUIRE(t->nbytes > 0, "gguf_read: '%s' has ggml type %u (F32, F16, BF16 and I2_S are read)", name,
                t->type);
    TVB_REQUIRE(capacity >= t->nbytes, "gguf_read: '%s' needs %llu bytes, destination has %llu", name,
                (unsigned long long)t->nbytes, (unsigned long long)capacity);
    TVB_REQUIRE(g->data_offset <= g->file_size && t->offset <= g->file_size - g->data_offset &&
                    t->nbytes <= g->file_size - g->data_offset - t->offset,
                "gguf_read: '%s' runs past the file end", name);
    if (std::fseek(g->file.f, (long)(g->data_offset + t->offset), SEEK_SET) != 0)
        return tvb::set_error(TVB_ERR_INVALID, "gguf_read: seek failed for '%s'", name);
    return read_into(g->file.f, dst, t->nbytes, name, g->sg);
}

tvb_status tvb_gguf_close(tvb_gguf* g) {
    delete g;
    return TVB_OK;
}

}  // extern "C"
