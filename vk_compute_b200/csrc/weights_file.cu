// On-disk weights: named matrices in exactly the layout the kernels read.
//
// vk-compute keeps no weight files (its model/ directory is not part of the
// project); it builds its matrices in memory with src/data.c's quantisers and
// transpose_block16.  This file format stores those arrays as they are:
//
//   header (64 bytes)   "VKCWGT01", u32 version (1), u32 count,
//                       u64 directory offset, zero padding
//   directory           count entries of 128 bytes: char name[64] (NUL
//                       terminated), u32 bits, u32 K, u32 N, u32 reserved,
//                       u64 data offset, u64 data bytes (K*N*bits/8),
//                       u64 scale offset, u64 zero offset, u64 bytes of each
//                       of scale and zero (K*(N/256)*4; 0 for 16/32-bit),
//                       zero padding
//   sections            packed chunks (transpose_block16, src/data.c:198-222),
//                       then block-major fp32 scale and zero
//                       (src/data.c:122-124), each at a 256-byte boundary
//
// All integers little-endian.  Loading reads each section into pinned host
// memory and copies it to the device, so a matrix goes from disk to HBM
// without any repacking.
#include "vkc_common.cuh"
#include "vk_compute_b200.h"

#include <cstring>
#include <string>
#include <vector>

namespace vkc {
namespace {

constexpr char kMagic[8] = {'V', 'K', 'C', 'W', 'G', 'T', '0', '1'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kAlign = 256;
constexpr size_t kHeaderBytes = 64;
constexpr size_t kEntryBytes = 128;

struct Entry {
    char name[64];
    uint32_t bits, K, N, reserved;
    uint64_t data_off, data_bytes, scale_off, zero_off, sz_bytes;
};
static_assert(sizeof(Entry) <= kEntryBytes, "directory entry");

uint64_t align_up(uint64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

bool valid_shape(uint32_t bits, uint32_t K, uint32_t N) {
    if (bits != 32 && bits != 16 && bits != 8 && bits != 4) return false;
    if (K == 0 || N == 0 || K % (128 / bits) != 0) return false;
    if (bits <= 8 && N % 256 != 0) return false;
    return true;
}

uint64_t data_bytes_of(uint32_t bits, uint32_t K, uint32_t N) {
    return static_cast<uint64_t>(K) * N * bits / 8;
}
uint64_t sz_bytes_of(uint32_t bits, uint32_t K, uint32_t N) {
    return bits <= 8 ? static_cast<uint64_t>(K) * (N / 256) * 4 : 0;
}

}  // namespace
}  // namespace vkc

using namespace vkc;

struct vkc_weight_file {
    FILE* fp = nullptr;
    uint64_t size = 0;
    std::vector<Entry> entries;
};

extern "C" {

int vkc_weights_write(const char* path, const vkc_weight_entry* entries, int count) {
    if (!path || (count > 0 && !entries) || count < 0) return set_error(kErrArg, "null path or entries");
    std::vector<Entry> dir(static_cast<size_t>(count));
    uint64_t at = align_up(kHeaderBytes + static_cast<uint64_t>(count) * kEntryBytes);
    for (int i = 0; i < count; ++i) {
        const vkc_weight_entry& e = entries[i];
        if (!valid_shape(static_cast<uint32_t>(e.bits), static_cast<uint32_t>(e.K), static_cast<uint32_t>(e.N)) ||
            e.K <= 0 || e.N <= 0)
            return set_error(kErrArg, "matrix %d (%s): unsupported bits=%d K=%d N=%d", i, e.name, e.bits, e.K, e.N);
        if (!e.data || (e.bits <= 8 && (!e.scale || !e.zero)))
            return set_error(kErrArg, "matrix %d (%s): missing data, scale or zero", i, e.name);
        if (memchr(e.name, '\0', sizeof e.name) == nullptr)
            return set_error(kErrArg, "matrix %d: name is not NUL-terminated within 64 bytes", i);
        Entry& d = dir[static_cast<size_t>(i)];
        memset(&d, 0, sizeof d);
        memcpy(d.name, e.name, sizeof d.name);
        d.bits = static_cast<uint32_t>(e.bits);
        d.K = static_cast<uint32_t>(e.K);
        d.N = static_cast<uint32_t>(e.N);
        d.data_bytes = data_bytes_of(d.bits, d.K, d.N);
        d.sz_bytes = sz_bytes_of(d.bits, d.K, d.N);
        d.data_off = at;
        at = align_up(at + d.data_bytes);
        if (d.sz_bytes) {
            d.scale_off = at;
            at = align_up(at + d.sz_bytes);
            d.zero_off = at;
            at = align_up(at + d.sz_bytes);
        }
    }
    FILE* fp = fopen(path, "wb");
    if (!fp) return set_error(kErrArg, "cannot create %s", path);
    bool ok = true;
    auto put = [&](const void* p, size_t n) {
        if (ok && n && fwrite(p, 1, n, fp) != n) ok = false;
    };
    auto pad_to = [&](uint64_t off) {
        static const char zeros[kAlign] = {};
        long cur = ftell(fp);
        if (cur < 0) {
            ok = false;
            return;
        }
        while (ok && static_cast<uint64_t>(cur) < off) {
            const size_t n = static_cast<size_t>(off - static_cast<uint64_t>(cur) < kAlign ? off - cur : kAlign);
            put(zeros, n);
            cur += static_cast<long>(n);
        }
    };
    unsigned char header[kHeaderBytes] = {};
    memcpy(header, kMagic, 8);
    const uint32_t ver = kVersion, cnt = static_cast<uint32_t>(count);
    const uint64_t dir_off = kHeaderBytes;
    memcpy(header + 8, &ver, 4);
    memcpy(header + 12, &cnt, 4);
    memcpy(header + 16, &dir_off, 8);
    put(header, sizeof header);
    for (const Entry& d : dir) {
        unsigned char rec[kEntryBytes] = {};
        memcpy(rec, &d, sizeof d);
        put(rec, sizeof rec);
    }
    for (int i = 0; i < count && ok; ++i) {
        const Entry& d = dir[static_cast<size_t>(i)];
        pad_to(d.data_off);
        put(entries[i].data, d.data_bytes);
        if (d.sz_bytes) {
            pad_to(d.scale_off);
            put(entries[i].scale, d.sz_bytes);
            pad_to(d.zero_off);
            put(entries[i].zero, d.sz_bytes);
        }
    }
    if (fclose(fp) != 0) ok = false;
    if (!ok) return set_error(kErrArg, "writing %s failed", path);
    return kOk;
}

int vkc_weights_open(const char* path, vkc_weight_file** out) {
    if (!path || !out) return set_error(kErrArg, "null path or output");
    *out = nullptr;
    FILE* fp = fopen(path, "rb");
    if (!fp) return set_error(kErrArg, "cannot open %s", path);
    auto fail = [&](const char* why) {
        fclose(fp);
        return set_error(kErrArg, "%s: %s", path, why);
    };
    if (fseek(fp, 0, SEEK_END) != 0) return fail("cannot seek");
    const long end = ftell(fp);
    if (end < 0) return fail("cannot size");
    const uint64_t size = static_cast<uint64_t>(end);
    rewind(fp);
    unsigned char header[kHeaderBytes];
    if (size < kHeaderBytes || fread(header, 1, kHeaderBytes, fp) != kHeaderBytes) return fail("truncated header");
    if (memcmp(header, kMagic, 8) != 0) return fail("not a weights file (bad magic)");
    uint32_t ver = 0, cnt = 0;
    uint64_t dir_off = 0;
    memcpy(&ver, header + 8, 4);
    memcpy(&cnt, header + 12, 4);
    memcpy(&dir_off, header + 16, 8);
    if (ver != kVersion) return fail("unsupported version");
    if (cnt > (1u << 20) || dir_off < kHeaderBytes || dir_off + static_cast<uint64_t>(cnt) * kEntryBytes > size)
        return fail("directory outside the file");
    std::vector<Entry> dir(cnt);
    if (fseek(fp, static_cast<long>(dir_off), SEEK_SET) != 0) return fail("cannot seek to the directory");
    for (uint32_t i = 0; i < cnt; ++i) {
        unsigned char rec[kEntryBytes];
        if (fread(rec, 1, kEntryBytes, fp) != kEntryBytes) return fail("truncated directory");
        Entry& d = dir[i];
        memcpy(&d, rec, sizeof d);
        if (memchr(d.name, '\0', sizeof d.name) == nullptr) return fail("unterminated matrix name");
        if (!valid_shape(d.bits, d.K, d.N)) return fail("unsupported matrix shape");
        if (d.data_bytes != data_bytes_of(d.bits, d.K, d.N) || d.sz_bytes != sz_bytes_of(d.bits, d.K, d.N))
            return fail("section sizes do not match the shape");
        auto inside = [&](uint64_t off, uint64_t n) { return off % kAlign == 0 && off <= size && n <= size - off; };
        if (!inside(d.data_off, d.data_bytes)) return fail("data section outside the file");
        if (d.sz_bytes && (!inside(d.scale_off, d.sz_bytes) || !inside(d.zero_off, d.sz_bytes)))
            return fail("scale or zero section outside the file");
    }
    vkc_weight_file* f = new vkc_weight_file;
    f->fp = fp;
    f->size = size;
    f->entries = std::move(dir);
    *out = f;
    return kOk;
}

int vkc_weights_count(const vkc_weight_file* f) { return f ? static_cast<int>(f->entries.size()) : -1; }

int vkc_weights_find(const vkc_weight_file* f, const char* name) {
    if (!f || !name) return -1;
    for (size_t i = 0; i < f->entries.size(); ++i)
        if (strncmp(f->entries[i].name, name, sizeof f->entries[i].name) == 0) return static_cast<int>(i);
    return -1;
}

int vkc_weights_info(const vkc_weight_file* f, int index, vkc_weight_entry* info) {
    if (!f || !info) return set_error(kErrArg, "null file or output");
    if (index < 0 || index >= static_cast<int>(f->entries.size()))
        return set_error(kErrArg, "matrix index %d of %zu", index, f->entries.size());
    const Entry& d = f->entries[static_cast<size_t>(index)];
    memset(info, 0, sizeof *info);
    memcpy(info->name, d.name, sizeof info->name);
    info->bits = static_cast<int>(d.bits);
    info->K = static_cast<int>(d.K);
    info->N = static_cast<int>(d.N);
    return kOk;
}

static int read_section(vkc_weight_file* f, uint64_t off, uint64_t n, void* host) {
    if (fseek(f->fp, static_cast<long>(off), SEEK_SET) != 0) return set_error(kErrArg, "seek failed");
    if (fread(host, 1, n, f->fp) != n) return set_error(kErrArg, "short read");
    return kOk;
}

int vkc_weights_read_host(vkc_weight_file* f, int index, void* data, float* scale, float* zero) {
    if (!f || !data) return set_error(kErrArg, "null file or data");
    if (index < 0 || index >= static_cast<int>(f->entries.size()))
        return set_error(kErrArg, "matrix index %d of %zu", index, f->entries.size());
    const Entry& d = f->entries[static_cast<size_t>(index)];
    if (d.sz_bytes && (!scale || !zero)) return set_error(kErrArg, "%s: quantised matrix needs scale and zero", d.name);
    if (int e = read_section(f, d.data_off, d.data_bytes, data)) return e;
    if (d.sz_bytes) {
        if (int e = read_section(f, d.scale_off, d.sz_bytes, scale)) return e;
        if (int e = read_section(f, d.zero_off, d.sz_bytes, zero)) return e;
    }
    return kOk;
}

int vkc_weights_read(vkc_weight_file* f, int index, void* data, float* scale, float* zero, void* stream) {
    if (!f || !data) return set_error(kErrArg, "null file or data");
    if (index < 0 || index >= static_cast<int>(f->entries.size()))
        return set_error(kErrArg, "matrix index %d of %zu", index, f->entries.size());
    const Entry& d = f->entries[static_cast<size_t>(index)];
    if (d.sz_bytes && (!scale || !zero)) return set_error(kErrArg, "%s: quantised matrix needs scale and zero", d.name);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t total = d.data_bytes + 2 * d.sz_bytes;
    void* pinned = nullptr;
    VKC_CUDA_TRY(cudaHostAlloc(&pinned, total, cudaHostAllocDefault));
    char* h = static_cast<char*>(pinned);
    int rc = read_section(f, d.data_off, d.data_bytes, h);
    if (rc == 0 && d.sz_bytes) rc = read_section(f, d.scale_off, d.sz_bytes, h + d.data_bytes);
    if (rc == 0 && d.sz_bytes) rc = read_section(f, d.zero_off, d.sz_bytes, h + d.data_bytes + d.sz_bytes);
    cudaError_t ce = cudaSuccess;
    if (rc == 0) {
        ce = cudaMemcpyAsync(data, h, d.data_bytes, cudaMemcpyHostToDevice, s);
        if (ce == cudaSuccess && d.sz_bytes)
            ce = cudaMemcpyAsync(scale, h + d.data_bytes, d.sz_bytes, cudaMemcpyHostToDevice, s);
        if (ce == cudaSuccess && d.sz_bytes)
            ce = cudaMemcpyAsync(zero, h + d.data_bytes + d.sz_bytes, d.sz_bytes, cudaMemcpyHostToDevice, s);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);  // the pinned copy is freed below
    }
    cudaFreeHost(pinned);
    if (rc) return rc;
    if (ce != cudaSuccess) return set_error(kErrCuda, "copying %s to the device: %s", d.name, cudaGetErrorString(ce));
    return kOk;
}

void vkc_weights_close(vkc_weight_file* f) {
    if (!f) return;
    if (f->fp) fclose(f->fp);
    delete f;
}

}  // extern "C"
