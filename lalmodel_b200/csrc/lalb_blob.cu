// lalb_blob.cu -- the weight-blob file: writer (converter) and loader.
//
// The reference ships real weights as one pre-converted file
// (prebuilt/qwen7b_q4k_weights.bin, made by scripts/convert_qwen7b_q4k.py
// from BF16 safetensors; README.md:18-20,154) and loads its seed models from
// GPW2 files (tensor_load_all, runtime/lal_runtime.c:2798-2822: magic, count,
// then per tensor a key, shape and fp32 data, read with fread into malloc'd
// host memory).  Neither the Q4_K file's format nor its converter is in the
// reference snapshot, so this format is our own, versioned, and laid out for
// loading straight into device memory:
//
//   offset 0     header, 64 bytes: "LQ4K", u32 version (1), u32 n_tensors,
//                u32 alignment (4096), u64 table offset, u64 table bytes,
//                u64 file bytes, 24 reserved zero bytes
//   4096 ...     tensor data, each tensor starting on a 4096-byte boundary
//   table        n_tensors entries of 128 bytes: key[72] (NUL-terminated),
//                u32 dtype, u32 ndim, u64 dims[3], u64 offset, u64 bytes,
//                u64 FNV-1a-64 checksum of the tensor's bytes
//
// All integers little-endian.  dtypes: F32, Q4K (dims [rows, K]: rows *
// K/256 * 144 bytes in the layout of include/lalb.h), I8, F16, BF16.  A 2-D
// tensor's rows are contiguous, so a tensor-parallel rank loads its row
// shard as one byte range.
//
// The loader streams a byte range through two pinned staging buffers: the
// file read of chunk i+1 overlaps the host-to-device copy of chunk i on the
// caller's stream.  The writer quantizes fp32 or bf16 weights with the
// library's own GPU quantizers (lalb_q4k_quantize, lalb_q8_quantize_rows),
// so a blob holds exactly the bytes the kernels would have made in memory.
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "lalb_internal.cuh"

namespace {

constexpr char kMagic[4] = {'L', 'Q', '4', 'K'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kAlign = 4096;
constexpr size_t kHeaderBytes = 64;
constexpr size_t kEntryBytes = 128;
constexpr size_t kKeyBytes = 72;
constexpr size_t kStageBytes = 32u << 20;   // per staging buffer

struct Entry {
    char key[kKeyBytes];
    uint32_t dtype, ndim;
    uint64_t dims[3];
    uint64_t offset, bytes, fnv;
};
static_assert(sizeof(Entry) == kEntryBytes, "table entry layout");

uint64_t fnv1a(uint64_t h, const unsigned char *p, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 0x100000001b3ull;
    }
    return h;
}
constexpr uint64_t kFnvInit = 0xcbf29ce484222325ull;

void put_u32(unsigned char *p, uint32_t v) { memcpy(p, &v, 4); }
void put_u64(unsigned char *p, uint64_t v) { memcpy(p, &v, 8); }
uint32_t get_u32(const unsigned char *p) { uint32_t v; memcpy(&v, p, 4); return v; }
uint64_t get_u64(const unsigned char *p) { uint64_t v; memcpy(&v, p, 8); return v; }

bool full_pwrite(int fd, const void *buf, size_t n, uint64_t off) {
    const unsigned char *p = static_cast<const unsigned char *>(buf);
    while (n) {
        const ssize_t w = pwrite(fd, p, n, (off_t)off);
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) return false;
        p += w;
        n -= (size_t)w;
        off += (uint64_t)w;
    }
    return true;
}

bool full_pread(int fd, void *buf, size_t n, uint64_t off) {
    unsigned char *p = static_cast<unsigned char *>(buf);
    while (n) {
        const ssize_t r = pread(fd, p, n, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        n -= (size_t)r;
        off += (uint64_t)r;
    }
    return true;
}

// Bytes of a tensor of dtype with dims, 0 when the shape is not valid.
uint64_t tensor_bytes(uint32_t dtype, uint32_t ndim, const uint64_t *dims) {
    if (ndim < 1 || ndim > 3) return 0;
    uint64_t n = 1;
    for (uint32_t i = 0; i < ndim; ++i) {
        if (dims[i] == 0 || dims[i] > (1ull << 40)) return 0;
        n *= dims[i];
    }
    switch (dtype) {
        case LALB_DT_F32: return 4 * n;
        case LALB_DT_I8: return n;
        case LALB_DT_F16:
        case LALB_DT_BF16: return 2 * n;
        case LALB_DT_Q4K:
            if (ndim != 2 || dims[1] % 256) return 0;
            return dims[0] * (dims[1] / 256) * 144;
        default: return 0;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// writer
// ---------------------------------------------------------------------------
struct lalb_blob_writer {
    int fd = -1;
    uint64_t end = kAlign;        // next free data byte
    std::vector<Entry> table;
    std::string path;
    bool failed = false;
};

extern "C" int lalb_blob_writer_open(const char *path, lalb_blob_writer **out) {
    if (!path || !out) return LALB_ERR_INVALID;
    *out = nullptr;
    const int fd = open(path, O_CREAT | O_TRUNC | O_WRONLY, 0644);
    if (fd < 0) return LALB_ERR_INVALID;
    lalb_blob_writer *w = new (std::nothrow) lalb_blob_writer();
    if (!w) {
        close(fd);
        return LALB_ERR_NOMEM;
    }
    w->fd = fd;
    w->path = path;
    *out = w;
    return LALB_OK;
}

extern "C" int lalb_blob_writer_add(lalb_blob_writer *w, const char *key, int dtype, int ndim,
                                    const uint64_t *dims, const void *data) {
    if (!w || w->failed || !key || !dims || !data) return LALB_ERR_INVALID;
    const size_t klen = strlen(key);
    if (klen == 0 || klen >= kKeyBytes) return LALB_ERR_INVALID;
    for (const Entry &e : w->table)
        if (strcmp(e.key, key) == 0) return LALB_ERR_INVALID;   // keys are unique
    if (ndim < 1 || ndim > 3) return LALB_ERR_INVALID;
    Entry e = {};
    memcpy(e.key, key, klen);
    e.dtype = (uint32_t)dtype;
    e.ndim = (uint32_t)ndim;
    for (int i = 0; i < ndim; ++i) e.dims[i] = dims[i];
    e.bytes = tensor_bytes(e.dtype, e.ndim, e.dims);
    if (!e.bytes) return LALB_ERR_INVALID;
    e.offset = w->end;
    e.fnv = fnv1a(kFnvInit, static_cast<const unsigned char *>(data), e.bytes);
    if (!full_pwrite(w->fd, data, e.bytes, e.offset)) {
        w->failed = true;
        return LALB_ERR_INVALID;
    }
    w->end = (e.offset + e.bytes + kAlign - 1) / kAlign * kAlign;
    w->table.push_back(e);
    return LALB_OK;
}

// Quantizes fp32 rows on the GPU with the library's quantizer and adds the
// result.  Q4K: rows x K (K % 256 == 0); I8: rows x K int8 under key plus
// the per-row scales under scale_key.
static int add_quantized(lalb_ctx *ctx, lalb_blob_writer *w, const char *key,
                         const char *scale_key, int dtype, const float *host, int rows, int K) {
    float *dw = nullptr;
    void *dq = nullptr;
    float *ds = nullptr;
    const uint64_t dims[2] = {(uint64_t)rows, (uint64_t)K};
    const size_t nq = tensor_bytes((uint32_t)dtype, 2, dims);
    if (!nq) return lalb_fail(ctx, LALB_ERR_INVALID, "blob: shape %d x %d for dtype %d", rows, K, dtype);
    int st = LALB_OK;
    std::vector<unsigned char> hq(nq);
    std::vector<float> hs(dtype == LALB_DT_I8 ? rows : 0);
    if (cudaMalloc(&dw, sizeof(float) * (size_t)rows * K) != cudaSuccess ||
        cudaMalloc(&dq, nq) != cudaSuccess ||
        (dtype == LALB_DT_I8 && cudaMalloc(&ds, sizeof(float) * rows) != cudaSuccess)) {
        cudaGetLastError();
        st = lalb_fail(ctx, LALB_ERR_NOMEM, "blob: device staging for %s", key);
    }
    if (!st && cudaMemcpy(dw, host, sizeof(float) * (size_t)rows * K, cudaMemcpyHostToDevice) !=
                   cudaSuccess)
        st = lalb_fail(ctx, LALB_ERR_CUDA, "blob: upload of %s", key);
    if (!st)
        st = dtype == LALB_DT_Q4K ? lalb_q4k_quantize(ctx, dw, rows, K, dq, nullptr)
                                  : lalb_q8_quantize_rows(ctx, dw, rows, K, (int8_t *)dq, ds, nullptr);
    if (!st && (cudaMemcpy(hq.data(), dq, nq, cudaMemcpyDeviceToHost) != cudaSuccess ||
                (ds && cudaMemcpy(hs.data(), ds, sizeof(float) * rows, cudaMemcpyDeviceToHost) !=
                           cudaSuccess)))
        st = lalb_fail(ctx, LALB_ERR_CUDA, "blob: download of %s", key);
    cudaFree(dw);
    cudaFree(dq);
    cudaFree(ds);
    if (!st && (st = lalb_blob_writer_add(w, key, dtype, 2, dims, hq.data())))
        lalb_fail(ctx, st, "blob: writing %s", key);
    if (!st && ds) {
        const uint64_t sd[1] = {(uint64_t)rows};
        if ((st = lalb_blob_writer_add(w, scale_key, LALB_DT_F32, 1, sd, hs.data())))
            lalb_fail(ctx, st, "blob: writing %s", scale_key);
    }
    return st;
}

static bool bf16_rows_to_f32(const uint16_t *src, size_t n, std::vector<float> &dst) {
    dst.resize(n);
    for (size_t i = 0; i < n; ++i) {
        const uint32_t u = (uint32_t)src[i] << 16;   // bf16 is the top half of fp32: exact
        memcpy(&dst[i], &u, 4);
    }
    return true;
}

extern "C" int lalb_blob_writer_add_quantized(lalb_ctx *ctx, lalb_blob_writer *w, const char *key,
                                              const char *scale_key, int dtype, int src_dtype,
                                              const void *host, int rows, int K) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!w || !key || !host || rows <= 0 || K <= 0 ||
        (dtype != LALB_DT_Q4K && dtype != LALB_DT_I8) ||
        (dtype == LALB_DT_I8 && !scale_key) || (src_dtype != LALB_DT_F32 && src_dtype != LALB_DT_BF16))
        return lalb_fail(ctx, LALB_ERR_INVALID, "blob_writer_add_quantized: bad arguments");
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (src_dtype == LALB_DT_F32)
        return add_quantized(ctx, w, key, scale_key, dtype, static_cast<const float *>(host), rows, K);
    std::vector<float> f;
    bf16_rows_to_f32(static_cast<const uint16_t *>(host), (size_t)rows * K, f);
    return add_quantized(ctx, w, key, scale_key, dtype, f.data(), rows, K);
}

extern "C" int lalb_blob_writer_close(lalb_blob_writer *w) {
    if (!w) return LALB_ERR_INVALID;
    int st = w->failed ? LALB_ERR_INVALID : LALB_OK;
    if (!st) {
        const uint64_t table_off = w->end;
        const uint64_t table_bytes = w->table.size() * kEntryBytes;
        unsigned char hdr[kHeaderBytes] = {};
        memcpy(hdr, kMagic, 4);
        put_u32(hdr + 4, kVersion);
        put_u32(hdr + 8, (uint32_t)w->table.size());
        put_u32(hdr + 12, (uint32_t)kAlign);
        put_u64(hdr + 16, table_off);
        put_u64(hdr + 24, table_bytes);
        put_u64(hdr + 32, table_off + table_bytes);
        if ((table_bytes && !full_pwrite(w->fd, w->table.data(), table_bytes, table_off)) ||
            !full_pwrite(w->fd, hdr, kHeaderBytes, 0) || ftruncate(w->fd, (off_t)(table_off + table_bytes)))
            st = LALB_ERR_INVALID;
    }
    close(w->fd);
    delete w;
    return st;
}

// ---------------------------------------------------------------------------
// reader / loader
// ---------------------------------------------------------------------------
struct lalb_blob {
    int fd = -1;
    uint64_t file_bytes = 0;
    std::vector<Entry> table;
    void *stage[2] = {nullptr, nullptr};   // pinned, allocated on the first device load
    cudaEvent_t done[2] = {nullptr, nullptr};
    int stage_device = -1;
};

extern "C" int lalb_blob_open(const char *path, lalb_blob **out) {
    if (!path || !out) return LALB_ERR_INVALID;
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return LALB_ERR_INVALID;
    struct stat sb;
    unsigned char hdr[kHeaderBytes];
    int st = LALB_OK;
    lalb_blob *b = nullptr;
    if (fstat(fd, &sb) || (uint64_t)sb.st_size < kHeaderBytes || !full_pread(fd, hdr, kHeaderBytes, 0) ||
        memcmp(hdr, kMagic, 4) != 0 || get_u32(hdr + 4) != kVersion || get_u32(hdr + 12) != kAlign)
        st = LALB_ERR_INVALID;
    const uint32_t n = st ? 0 : get_u32(hdr + 8);
    const uint64_t toff = st ? 0 : get_u64(hdr + 16), tbytes = st ? 0 : get_u64(hdr + 24);
    if (!st && (tbytes != (uint64_t)n * kEntryBytes || toff < kAlign || toff + tbytes != (uint64_t)sb.st_size ||
                get_u64(hdr + 32) != (uint64_t)sb.st_size))
        st = LALB_ERR_INVALID;
    if (!st) {
        b = new (std::nothrow) lalb_blob();
        if (!b) st = LALB_ERR_NOMEM;
    }
    if (!st) {
        b->fd = fd;
        b->file_bytes = (uint64_t)sb.st_size;
        b->table.resize(n);
        if (n && !full_pread(fd, b->table.data(), tbytes, toff)) st = LALB_ERR_INVALID;
        for (uint32_t i = 0; !st && i < n; ++i) {
            const Entry &e = b->table[i];
            if (memchr(e.key, 0, kKeyBytes) == nullptr || e.key[0] == 0 ||
                tensor_bytes(e.dtype, e.ndim, e.dims) != e.bytes || e.offset % kAlign ||
                e.offset < kAlign || e.offset + e.bytes > toff)
                st = LALB_ERR_INVALID;
        }
    }
    if (st) {
        if (b) {
            b->fd = -1;
            delete b;
        }
        close(fd);
        return st;
    }
    *out = b;
    return LALB_OK;
}

extern "C" int lalb_blob_close(lalb_blob *b) {
    if (!b) return LALB_ERR_INVALID;
    if (b->stage_device >= 0) cudaSetDevice(b->stage_device);
    for (int i = 0; i < 2; ++i) {
        if (b->done[i]) cudaEventDestroy(b->done[i]);
        if (b->stage[i]) cudaFreeHost(b->stage[i]);
    }
    close(b->fd);
    delete b;
    return LALB_OK;
}

extern "C" int lalb_blob_count(const lalb_blob *b) {
    return b ? (int)b->table.size() : LALB_ERR_INVALID;
}

extern "C" int lalb_blob_find(const lalb_blob *b, const char *key) {
    if (!b || !key) return LALB_ERR_INVALID;
    for (size_t i = 0; i < b->table.size(); ++i)
        if (strncmp(b->table[i].key, key, kKeyBytes) == 0) return (int)i;
    return LALB_ERR_INVALID;
}

extern "C" int lalb_blob_info(const lalb_blob *b, int index, lalb_blob_tensor *info) {
    if (!b || !info || index < 0 || index >= (int)b->table.size()) return LALB_ERR_INVALID;
    const Entry &e = b->table[index];
    memset(info, 0, sizeof(*info));
    memcpy(info->key, e.key, kKeyBytes);
    info->dtype = (int)e.dtype;
    info->ndim = (int)e.ndim;
    for (int i = 0; i < 3; ++i) info->dims[i] = e.dims[i];
    info->bytes = e.bytes;
    info->row_bytes = e.bytes / e.dims[0];
    return LALB_OK;
}

extern "C" int lalb_blob_read_host(const lalb_blob *b, int index, uint64_t row0, uint64_t row1,
                                   void *dst) {
    if (!b || !dst || index < 0 || index >= (int)b->table.size()) return LALB_ERR_INVALID;
    const Entry &e = b->table[index];
    const uint64_t rb = e.bytes / e.dims[0];
    if (row0 > row1 || row1 > e.dims[0]) return LALB_ERR_INVALID;
    return full_pread(b->fd, dst, (row1 - row0) * rb, e.offset + row0 * rb) ? LALB_OK
                                                                          : LALB_ERR_INVALID;
}

extern "C" int lalb_blob_verify(const lalb_blob *b, int index) {
    if (!b || index < 0 || index >= (int)b->table.size()) return LALB_ERR_INVALID;
    const Entry &e = b->table[index];
    std::vector<unsigned char> buf(1u << 22);
    uint64_t h = kFnvInit;
    for (uint64_t off = 0; off < e.bytes;) {
        const size_t n = (size_t)std::min<uint64_t>(buf.size(), e.bytes - off);
        if (!full_pread(b->fd, buf.data(), n, e.offset + off)) return LALB_ERR_INVALID;
        h = fnv1a(h, buf.data(), n);
        off += n;
    }
    return h == e.fnv ? LALB_OK : LALB_ERR_INVALID;
}

extern "C" int lalb_blob_load(lalb_ctx *ctx, lalb_blob *b, int index, uint64_t row0, uint64_t row1,
                              void *dst, lalb_stream stream) {
    if (!ctx) return LALB_ERR_INVALID;
    if (!b || !dst || index < 0 || index >= (int)b->table.size())
        return lalb_fail(ctx, LALB_ERR_INVALID, "blob_load: bad arguments");
    const Entry &e = b->table[index];
    const uint64_t rb = e.bytes / e.dims[0];
    if (row0 > row1 || row1 > e.dims[0])
        return lalb_fail(ctx, LALB_ERR_INVALID, "blob_load: rows [%llu, %llu) of %llu",
                         (unsigned long long)row0, (unsigned long long)row1,
                         (unsigned long long)e.dims[0]);
    LALB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (b->stage_device != ctx->device) {
        if (b->stage_device >= 0)
            return lalb_fail(ctx, LALB_ERR_INVALID, "blob_load: a blob loads onto one device");
        for (int i = 0; i < 2; ++i) {
            LALB_CUDA_TRY(ctx, cudaMallocHost(&b->stage[i], kStageBytes));
            LALB_CUDA_TRY(ctx, cudaEventCreateWithFlags(&b->done[i], cudaEventDisableTiming));
        }
        b->stage_device = ctx->device;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const uint64_t total = (row1 - row0) * rb, base = e.offset + row0 * rb;
    unsigned char *out = static_cast<unsigned char *>(dst);
    int k = 0;
    for (uint64_t off = 0; off < total; off += kStageBytes, k ^= 1) {
        const size_t n = (size_t)std::min<uint64_t>(kStageBytes, total - off);
        // the copy that last used this staging buffer must be done with it
        LALB_CUDA_TRY(ctx, cudaEventSynchronize(b->done[k]));
        if (!full_pread(b->fd, b->stage[k], n, base + off))
            return lalb_fail(ctx, LALB_ERR_INVALID, "blob_load: read of %s failed", e.key);
        LALB_CUDA_TRY(ctx, cudaMemcpyAsync(out + off, b->stage[k], n, cudaMemcpyHostToDevice, s));
        LALB_CUDA_TRY(ctx, cudaEventRecord(b->done[k], s));
    }
    // the staging buffers are reused by the next call
    LALB_CUDA_TRY(ctx, cudaEventSynchronize(b->done[0]));
    LALB_CUDA_TRY(ctx, cudaEventSynchronize(b->done[1]));
    return LALB_OK;
}
