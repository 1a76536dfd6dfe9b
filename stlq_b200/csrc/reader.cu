// Vector-file reader feeding the encoder: the reference's BvecsReader / FvecsReader / FbinReader
// (include/stlq/io/{bvecs,fvecs,fbin}_reader.h) and its block prefetcher
// (AsyncBasicBlockPrefetcher, src/quantizer/encode_base_streaming.cpp:72-230), rebuilt around the
// device.
//
// File formats (the reference's, restated):
//   .bvecs / .siftbin   records of int32 d + d uint8 (n = file size / (4 + d))
//   .fvecs              records of int32 d + d float32 (n = file size / (4 + 4d))
//   .fbin               int32 n, int32 d, then n x d float32 row-major (file at least that long)
// Vector i of a block is row i of a row-major n x d array, which is the reference's column-major
// d x n ColMajorMatrix: the same bytes.
//
// Pipeline: a prefetch thread reads the raw bytes of block after block (the records with their
// dimension prefixes, io_threads positional reads in parallel) into `depth` pinned slots, in
// order.  stlq_b200_reader_next copies the next slot to the device with one contiguous copy on the
// caller's stream, then a kernel strips the 4-byte prefix of every record (an .fbin block needs no
// unpacking: it is copied straight into the destination) and checks each prefix against d.  A slot
// is refilled once the copy that read it has completed.  With device < 0 the reader is host-only:
// next() unpacks into host memory.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/stlq_b200.h"

namespace stlq_b200 {
int SetError(int code, const char* msg);
}  // namespace stlq_b200

namespace {

using stlq_b200::SetError;

int Fail(int code, const std::string& msg) { return SetError(code, ("stlq_b200 reader: " + msg).c_str()); }

bool HasSuffix(const std::string& s, const char* suf) {
    const size_t n = std::strlen(suf);
    if (s.size() < n) return false;
    for (size_t i = 0; i < n; ++i)
        if (std::tolower(static_cast<unsigned char>(s[s.size() - n + i])) != suf[i]) return false;
    return true;
}

// Each record's prefix must equal d; the payload words follow it.  W is the copy width (4 bytes
// when records, payloads and the destination allow it, else 1).
template <typename W>
__global__ void UnpackRecords(const uint8_t* __restrict__ raw, uint64_t rec_bytes, int64_t count, int words, int d,
                              W* __restrict__ out, unsigned int* bad) {
    const int64_t total = count * words;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = idx / words;
        const int j = static_cast<int>(idx - i * words);
        const uint8_t* r = raw + static_cast<uint64_t>(i) * rec_bytes;
        out[idx] = reinterpret_cast<const W*>(r + 4)[j];
        if (j == 0) {
            int32_t dim;
            if constexpr (sizeof(W) == 4) {
                dim = *reinterpret_cast<const int32_t*>(r);
            } else {
                dim = static_cast<int32_t>(r[0] | (r[1] << 8) | (r[2] << 16) | (static_cast<uint32_t>(r[3]) << 24));
            }
            if (dim != d) atomicOr(bad, 1u);
        }
    }
}

struct Slot {
    uint8_t* raw = nullptr;  // pinned (device reader) or heap (host-only)
    std::vector<uint8_t> raw_host;
    uint64_t start = 0;
    int64_t count = 0;
    cudaEvent_t consumed = nullptr;  // recorded after the copy that reads the slot
    bool pending = false;            // `consumed` recorded and not yet waited for
};

}  // namespace

struct stlq_b200_reader {
    std::string path;
    int fd = -1;
    int format = 0;
    int d = 0, elem = 1, prefix = 4;
    uint64_t n = 0, rec = 0, header = 0;
    uint64_t begin = 0, end = 0;
    int64_t block = 0;
    int io_threads = 1;
    int device = -1;
    // Prefetch.
    std::vector<Slot> slots;
    std::deque<int> filled;  // slot ids in file order
    int free_slots = 0;
    int next_fill = 0;  // slots are filled and consumed round robin
    std::mutex mu;
    std::condition_variable cv;
    std::thread worker;
    bool stop = false, done = false;
    std::string error;
    // Device staging.
    uint8_t* d_raw = nullptr;
    cudaEvent_t staged_free = nullptr;
    unsigned int* bad = nullptr;  // mapped pinned: set by the unpack kernel on a dimension mismatch
    unsigned int* bad_dev = nullptr;
};

namespace {

// Positional read of [off, off+len) into dst with up to `threads` parallel reads.
bool ReadRange(int fd, uint64_t off, uint64_t len, uint8_t* dst, int threads, std::string* err) {
    auto one = [&](uint64_t o, uint64_t l, uint8_t* p) {
        while (l > 0) {
            const ssize_t r = ::pread(fd, p, static_cast<size_t>(std::min<uint64_t>(l, 1ull << 30)),
                                      static_cast<off_t>(o));
            if (r <= 0) return false;
            o += static_cast<uint64_t>(r);
            p += r;
            l -= static_cast<uint64_t>(r);
        }
        return true;
    };
    const uint64_t min_chunk = 4ull << 20;
    const int t = static_cast<int>(std::max<uint64_t>(1, std::min<uint64_t>(threads, len / min_chunk)));
    bool ok = true;
    if (t == 1) {
        ok = one(off, len, dst);
    } else {
        const uint64_t chunk = (len + t - 1) / t;
        std::vector<std::thread> th;
        std::vector<char> res(t, 1);
        for (int i = 0; i < t; ++i) {
            const uint64_t o = std::min(len, i * chunk), l = std::min(len, o + chunk) - o;
            th.emplace_back([&, i, o, l] { res[i] = one(off + o, l, dst + o); });
        }
        for (auto& x : th) x.join();
        for (char r : res) ok = ok && r;
    }
    if (!ok) *err = "read failed";
    return ok;
}

// Host unpack of `count` raw records into dst (row-major count x d); false on a dimension mismatch.
bool UnpackHost(const stlq_b200_reader* rd, const uint8_t* raw, int64_t count, uint8_t* dst) {
    const size_t payload = static_cast<size_t>(rd->d) * rd->elem;
    if (rd->prefix == 0) {
        std::memcpy(dst, raw, payload * count);
        return true;
    }
    for (int64_t i = 0; i < count; ++i) {
        const uint8_t* r = raw + static_cast<uint64_t>(i) * rd->rec;
        int32_t dim;
        std::memcpy(&dim, r, 4);
        if (dim != rd->d) return false;
        std::memcpy(dst + static_cast<size_t>(i) * payload, r + 4, payload);
    }
    return true;
}

void WorkerLoop(stlq_b200_reader* rd) {
    uint64_t s = rd->begin;
    while (s < rd->end) {
        const int64_t cnt = static_cast<int64_t>(std::min<uint64_t>(rd->block, rd->end - s));
        int id;
        {
            std::unique_lock<std::mutex> lock(rd->mu);
            rd->cv.wait(lock, [&] { return rd->stop || rd->free_slots > 0; });
            if (rd->stop) return;
            id = rd->next_fill;
            rd->next_fill = (rd->next_fill + 1) % static_cast<int>(rd->slots.size());
            --rd->free_slots;
        }
        Slot& sl = rd->slots[id];
        std::string err;
        bool ok = true;
        if (sl.pending) {  // the copy that read this slot last time must be complete
            cudaSetDevice(rd->device);
            const cudaError_t e = cudaEventSynchronize(sl.consumed);
            sl.pending = false;
            if (e != cudaSuccess) {
                ok = false;
                err = std::string("staging copy: ") + cudaGetErrorString(e);
            }
        }
        if (ok) ok = ReadRange(rd->fd, rd->header + s * rd->rec, static_cast<uint64_t>(cnt) * rd->rec, sl.raw,
                               rd->io_threads, &err);
        std::lock_guard<std::mutex> lock(rd->mu);
        if (!ok) {
            if (rd->error.empty()) rd->error = err + " at vector " + std::to_string(s) + " of " + rd->path;
            rd->done = true;
            rd->cv.notify_all();
            return;
        }
        sl.start = s;
        sl.count = cnt;
        rd->filled.push_back(id);
        rd->cv.notify_all();
        s += static_cast<uint64_t>(cnt);
    }
    std::lock_guard<std::mutex> lock(rd->mu);
    rd->done = true;
    rd->cv.notify_all();
}

int OpenFile(stlq_b200_reader* rd, const char* path, int format) {
    rd->path = path;
    if (format == STLQ_B200_FMT_AUTO) {
        // The reference's suffix detection (src/io/dataset_reader_factory.cpp:81-91).
        if (HasSuffix(rd->path, ".bvecs") || HasSuffix(rd->path, ".siftbin")) format = STLQ_B200_FMT_BVECS;
        else if (HasSuffix(rd->path, ".fbin")) format = STLQ_B200_FMT_FBIN;
        else if (HasSuffix(rd->path, ".fvecs")) format = STLQ_B200_FMT_FVECS;
        else return Fail(STLQ_B200_EINVAL, "cannot tell the format of " + rd->path + " from its suffix");
    }
    if (format != STLQ_B200_FMT_BVECS && format != STLQ_B200_FMT_FVECS && format != STLQ_B200_FMT_FBIN)
        return Fail(STLQ_B200_EINVAL, "unknown format");
    rd->format = format;
    rd->fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (rd->fd < 0) return Fail(STLQ_B200_EINVAL, "failed to open " + rd->path);
    struct stat stt;
    if (::fstat(rd->fd, &stt) != 0) return Fail(STLQ_B200_EINVAL, "failed to stat " + rd->path);
    const uint64_t size = static_cast<uint64_t>(stt.st_size);
    int32_t hdr[2] = {0, 0};
    const ssize_t got = ::pread(rd->fd, hdr, format == STLQ_B200_FMT_FBIN ? 8 : 4, 0);
    if (format == STLQ_B200_FMT_FBIN) {
        if (got != 8 || hdr[0] <= 0 || hdr[1] <= 0) return Fail(STLQ_B200_EINVAL, "invalid header in " + rd->path);
        rd->d = hdr[1];
        rd->elem = 4;
        rd->prefix = 0;
        rd->header = 8;
        rd->rec = 4ull * rd->d;
        const uint64_t expected = 8 + static_cast<uint64_t>(hdr[0]) * rd->rec;
        if (size < expected)
            return Fail(STLQ_B200_EINVAL, "file too small (expected " + std::to_string(expected) + " bytes, got " +
                                              std::to_string(size) + ") for " + rd->path);
        rd->n = static_cast<uint64_t>(hdr[0]);
    } else {
        if (got != 4 || hdr[0] <= 0) return Fail(STLQ_B200_EINVAL, "invalid dimension header in " + rd->path);
        rd->d = hdr[0];
        rd->elem = format == STLQ_B200_FMT_BVECS ? 1 : 4;
        rd->prefix = 4;
        rd->rec = 4ull + static_cast<uint64_t>(rd->d) * rd->elem;
        rd->n = size / rd->rec;
        if (rd->n == 0 && format == STLQ_B200_FMT_BVECS) return Fail(STLQ_B200_EINVAL, "empty file: " + rd->path);
    }
    return 0;
}

void Destroy(stlq_b200_reader* rd) {
    if (rd->worker.joinable()) {
        {
            std::lock_guard<std::mutex> lock(rd->mu);
            rd->stop = true;
            rd->cv.notify_all();
        }
        rd->worker.join();
    }
    if (rd->device >= 0) {
        cudaSetDevice(rd->device);
        for (auto& s : rd->slots) {
            if (s.consumed) {
                cudaEventSynchronize(s.consumed);
                cudaEventDestroy(s.consumed);
            }
            if (s.raw) cudaFreeHost(s.raw);
        }
        if (rd->staged_free) {
            cudaEventSynchronize(rd->staged_free);
            cudaEventDestroy(rd->staged_free);
        }
        if (rd->d_raw) cudaFree(rd->d_raw);
        if (rd->bad) cudaFreeHost(rd->bad);
    }
    if (rd->fd >= 0) ::close(rd->fd);
    delete rd;
}

}  // namespace

namespace stlq_b200 {

// For the block loop (pipeline.cpp).
void ReaderShape(const stlq_b200_reader* rd, int* device, int* d, int* x_dtype, int64_t* block, uint64_t* begin,
                 uint64_t* end) {
    *device = rd->device;
    *d = rd->d;
    *x_dtype = rd->elem == 1 ? STLQ_B200_U8 : STLQ_B200_F32;
    *block = rd->block;
    *begin = rd->begin;
    *end = rd->end;
}

}  // namespace stlq_b200

extern "C" {

int stlq_b200_reader_open(const char* path, int format, uint64_t begin, uint64_t end, int64_t block, int depth,
                          int io_threads, int device, stlq_b200_reader** out) {
    if (!out) return Fail(STLQ_B200_EINVAL, "out is null");
    *out = nullptr;
    if (!path || !*path || block < 1) return Fail(STLQ_B200_EINVAL, "path and block >= 1 are required");
    auto* rd = new stlq_b200_reader();
    if (int rc = OpenFile(rd, path, format)) {
        Destroy(rd);
        return rc;
    }
    rd->begin = std::min(begin, rd->n);
    rd->end = end == 0 ? rd->n : std::min(end, rd->n);
    rd->end = std::max(rd->end, rd->begin);
    rd->block = block;
    rd->io_threads = std::max(1, io_threads);
    rd->device = device;
    const int nslot = std::max(2, depth);
    rd->slots.resize(nslot);
    rd->free_slots = nslot;
    const size_t raw_bytes = static_cast<size_t>(block) * rd->rec;
    if (device < 0) {
        for (auto& s : rd->slots) {
            s.raw_host.resize(raw_bytes);
            s.raw = s.raw_host.data();
        }
    } else {
        cudaError_t e = cudaSetDevice(device);
        for (auto& s : rd->slots) {
            if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&s.raw), raw_bytes);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.consumed, cudaEventDisableTiming);
        }
        if (e == cudaSuccess && rd->prefix) e = cudaMalloc(reinterpret_cast<void**>(&rd->d_raw), raw_bytes);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&rd->staged_free, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&rd->bad), sizeof(unsigned int),
                                                cudaHostAllocMapped);
        if (e == cudaSuccess) {
            *rd->bad = 0;
            e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&rd->bad_dev), rd->bad, 0);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            Destroy(rd);
            return Fail(e == cudaErrorMemoryAllocation ? STLQ_B200_ENOMEM : STLQ_B200_ECUDA,
                        std::string("staging buffers: ") + cudaGetErrorString(e));
        }
    }
    rd->worker = std::thread(WorkerLoop, rd);
    *out = rd;
    return 0;
}

int stlq_b200_reader_info(const stlq_b200_reader* rd, int* d, uint64_t* n, int* x_dtype) {
    if (!rd) return Fail(STLQ_B200_EINVAL, "reader handle is null");
    if (d) *d = rd->d;
    if (n) *n = rd->n;
    if (x_dtype) *x_dtype = rd->elem == 1 ? STLQ_B200_U8 : STLQ_B200_F32;
    return 0;
}

int stlq_b200_reader_next(stlq_b200_reader* rd, void* dst, size_t dst_bytes, void* stream, uint64_t* start,
                          int64_t* count) {
    if (!rd || !count) return Fail(STLQ_B200_EINVAL, "reader handle and count are required");
    *count = 0;
    if (start) *start = rd->end;
    int id;
    {
        std::unique_lock<std::mutex> lock(rd->mu);
        rd->cv.wait(lock, [&] { return !rd->filled.empty() || rd->done || !rd->error.empty(); });
        if (!rd->error.empty()) return Fail(STLQ_B200_EINVAL, rd->error);
        if (rd->filled.empty()) return 0;  // end of the range
        id = rd->filled.front();
    }
    Slot& sl = rd->slots[id];
    const size_t payload = static_cast<size_t>(rd->d) * rd->elem;
    const size_t need = payload * static_cast<size_t>(sl.count);
    if (!dst || dst_bytes < need) return Fail(STLQ_B200_EINVAL, "destination missing or smaller than a block");
    if (rd->device < 0) {
        if (!UnpackHost(rd, sl.raw, sl.count, static_cast<uint8_t*>(dst)))
            return Fail(STLQ_B200_EINVAL, "dimension mismatch in a record of " + rd->path);
    } else {
        if (*reinterpret_cast<volatile unsigned int*>(rd->bad))
            return Fail(STLQ_B200_EINVAL, "dimension mismatch in a record of " + rd->path);
        auto s = static_cast<cudaStream_t>(stream);
        cudaSetDevice(rd->device);
        cudaError_t e;
        if (rd->prefix == 0) {
            e = cudaMemcpyAsync(dst, sl.raw, need, cudaMemcpyHostToDevice, s);
        } else {
            e = cudaStreamWaitEvent(s, rd->staged_free, 0);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(rd->d_raw, sl.raw, static_cast<size_t>(sl.count) * rd->rec,
                                    cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) {
                const bool wide = rd->rec % 4 == 0 && payload % 4 == 0 && reinterpret_cast<uintptr_t>(dst) % 4 == 0;
                const int words = static_cast<int>(wide ? payload / 4 : payload);
                const int64_t total = sl.count * words;
                const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 8));
                if (wide)
                    UnpackRecords<uint32_t><<<grid, 256, 0, s>>>(rd->d_raw, rd->rec, sl.count, words, rd->d,
                                                                 static_cast<uint32_t*>(dst), rd->bad_dev);
                else
                    UnpackRecords<uint8_t><<<grid, 256, 0, s>>>(rd->d_raw, rd->rec, sl.count, words, rd->d,
                                                                static_cast<uint8_t*>(dst), rd->bad_dev);
                e = cudaGetLastError();
            }
            if (e == cudaSuccess) e = cudaEventRecord(rd->staged_free, s);
        }
        if (e == cudaSuccess) e = cudaEventRecord(sl.consumed, s);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return Fail(STLQ_B200_ECUDA, std::string("block copy: ") + cudaGetErrorString(e));
        }
        sl.pending = true;
    }
    if (start) *start = sl.start;
    *count = sl.count;
    std::lock_guard<std::mutex> lock(rd->mu);
    rd->filled.pop_front();
    ++rd->free_slots;
    rd->cv.notify_all();
    return 0;
}

int stlq_b200_reader_read(stlq_b200_reader* rd, uint64_t start, int64_t count, void* dst, size_t dst_bytes,
                          int64_t* nread) {
    if (!rd || !nread) return Fail(STLQ_B200_EINVAL, "reader handle and nread are required");
    *nread = 0;
    if (count <= 0 || start >= rd->n) return 0;
    const int64_t cnt = static_cast<int64_t>(std::min<uint64_t>(rd->n - start, static_cast<uint64_t>(count)));
    const size_t need = static_cast<size_t>(rd->d) * rd->elem * static_cast<size_t>(cnt);
    if (!dst || dst_bytes < need) return Fail(STLQ_B200_EINVAL, "dst_bytes too small");
    std::vector<uint8_t> raw(static_cast<size_t>(cnt) * rd->rec);
    std::string err;
    if (!ReadRange(rd->fd, rd->header + start * rd->rec, raw.size(), raw.data(), rd->io_threads, &err))
        return Fail(STLQ_B200_EINVAL, err + " in " + rd->path);
    if (!UnpackHost(rd, raw.data(), cnt, static_cast<uint8_t*>(dst)))
        return Fail(STLQ_B200_EINVAL, "dimension mismatch in a record of " + rd->path);
    *nread = cnt;
    return 0;
}

int stlq_b200_reader_close(stlq_b200_reader* rd) {
    if (!rd) return 0;
    int rc = 0;
    if (rd->device >= 0 && rd->staged_free) {
        cudaSetDevice(rd->device);
        cudaEventSynchronize(rd->staged_free);
        if (rd->bad && *reinterpret_cast<volatile unsigned int*>(rd->bad))
            rc = Fail(STLQ_B200_EINVAL, "dimension mismatch in a record of " + rd->path);
    }
    Destroy(rd);
    return rc;
}

}  // extern "C"
