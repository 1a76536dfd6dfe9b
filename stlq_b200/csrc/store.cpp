// Base-store writer fed from device (or host) buffers: the files of the reference's
// BaseBasicWriter (include/stlq/io/base_store.h:29-97, src/io/base_store.cpp), byte for byte.
//
// Layout written (the reference's, restated):
//   meta.json, meta.bin           store parameters (meta.bin: ten 32-bit header fields, then h_vec)
//   cluster_id.u32                every vector's root code, in order
//   codes_shard_NNNN.bin          the (m-1) small codes of each vector, by shard of shard_size ids;
//   coeffs_shard_NNNN.bin         the m coefficients; a block goes whole to its first id's shard
//   bucket_NNNN.bin               per bucket of bucket_size root codes (all truncated at open), a
//                                 record per vector: uint32 id, uint32 root code, [raw vector],
//                                 [small codes, coefficients]
// Blocks are written in the order of the append calls.  An append copies the block into a pinned
// staging slot on the store's copy stream, after the work already enqueued on the caller's stream
// (so device outputs can be appended right after the kernels that produce them), and one writer
// thread writes the slots in order once their copies are complete.  With device < 0 the store is
// host-only: appends copy host buffers into the slot and no CUDA call is made.
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <filesystem>
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

std::string Tag(int v) {
    char b[16];
    std::snprintf(b, sizeof(b), "%04d", v);
    return b;
}

// One block in a staging slot.
struct Slot {
    std::vector<uint32_t> cluster_host;  // host-only stores
    std::vector<uint8_t> codes_host, x_host;
    std::vector<float> a_host;
    uint32_t* cluster = nullptr;  // pinned (device stores) or the host vectors' data
    uint8_t* codes = nullptr;
    float* a = nullptr;
    uint8_t* x = nullptr;
    int64_t cap = 0;
    cudaEvent_t copied = nullptr;
    // The job.
    uint64_t start_id = 0;
    int64_t n = 0;
    bool busy = false;
};

}  // namespace

struct stlq_b200_store {
    // Parameters (the reference's BaseBasicStoreConfig after its normalisation).
    std::string dir;
    int d = 0, m = 0, shard_size = 0, bucket_size = 0, raw_bytes = 0;
    bool vec_bucket = false, basic_bucket = false;
    size_t flush_bytes = 0;
    std::vector<int> h_vec;
    int device = -1;
    // Files.
    FILE* cluster_f = nullptr;
    FILE* codes_f = nullptr;
    FILE* coeffs_f = nullptr;
    int shard = -1;
    std::vector<FILE*> bucket_f;
    std::vector<std::vector<uint8_t>> bucket_buf;
    // Staging and the writer thread.
    std::vector<Slot> slots;
    std::deque<int> queue;  // slot ids in append order
    cudaStream_t copy = nullptr;
    std::mutex mu;
    std::condition_variable cv;
    std::thread writer;
    bool stop = false;
    std::string error;  // the first failure of the writer thread
};

namespace {

bool WriteAll(FILE* f, const void* p, size_t bytes) { return bytes == 0 || std::fwrite(p, 1, bytes, f) == bytes; }

bool OpenShard(stlq_b200_store* st, uint64_t start_id, std::string* err) {
    const int shard = static_cast<int>(start_id / static_cast<uint64_t>(std::max(1, st->shard_size)));
    if (shard == st->shard) return true;
    if (st->codes_f) std::fclose(st->codes_f);
    if (st->coeffs_f) std::fclose(st->coeffs_f);
    st->codes_f = std::fopen((st->dir + "/codes_shard_" + Tag(shard) + ".bin").c_str(), "wb");
    st->coeffs_f = std::fopen((st->dir + "/coeffs_shard_" + Tag(shard) + ".bin").c_str(), "wb");
    st->shard = shard;
    if (!st->codes_f || !st->coeffs_f) {
        *err = "failed to open shard outputs in " + st->dir;
        return false;
    }
    return true;
}

bool FlushBucket(stlq_b200_store* st, size_t b, std::string* err) {
    auto& buf = st->bucket_buf[b];
    if (buf.empty()) return true;
    if (!WriteAll(st->bucket_f[b], buf.data(), buf.size())) {
        *err = "bucket write failed";
        return false;
    }
    buf.clear();
    return true;
}

bool OpenBucket(stlq_b200_store* st, size_t b, std::string* err) {
    if (b >= st->bucket_f.size()) {
        st->bucket_f.resize(b + 1, nullptr);
        st->bucket_buf.resize(b + 1);
    }
    if (st->bucket_f[b]) return true;
    st->bucket_f[b] = std::fopen((st->dir + "/bucket_" + Tag(static_cast<int>(b)) + ".bin").c_str(), "wb");
    if (!st->bucket_f[b]) {
        *err = "failed to open bucket file " + Tag(static_cast<int>(b));
        return false;
    }
    return true;
}

// Writes one block (the writer thread, or the caller of a host-only store).
bool WriteBlock(stlq_b200_store* st, const Slot& s, std::string* err) {
    const int64_t n = s.n;
    const int mc = std::max(0, st->m - 1);
    if (!WriteAll(st->cluster_f, s.cluster, sizeof(uint32_t) * n)) {
        *err = "failed to write cluster_id.u32";
        return false;
    }
    if (!OpenShard(st, s.start_id, err)) return false;
    if (!WriteAll(st->codes_f, s.codes, static_cast<size_t>(mc) * n) ||
        !WriteAll(st->coeffs_f, s.a, sizeof(float) * st->m * n)) {
        *err = "failed to write shard outputs";
        return false;
    }
    if (!st->vec_bucket && !st->basic_bucket) return true;
    const int bsize = std::max(1, st->bucket_size);
    const size_t xb = st->vec_bucket ? static_cast<size_t>(st->raw_bytes) : 0;
    const size_t cb = st->basic_bucket ? static_cast<size_t>(mc) : 0;
    const size_t ab = st->basic_bucket ? sizeof(float) * st->m : 0;
    const size_t rec = 8 + xb + cb + ab;
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t gid = static_cast<uint32_t>(s.start_id + static_cast<uint64_t>(i));
        const uint32_t cid = s.cluster[i];
        const size_t b = cid / static_cast<uint32_t>(bsize);
        if (b > static_cast<size_t>(INT32_MAX)) {  // the reference's int bucket id would be negative
            *err = "invalid bucket id (cluster id " + std::to_string(cid) + ")";
            return false;
        }
        if (!OpenBucket(st, b, err)) return false;
        auto& buf = st->bucket_buf[b];
        // One record: id, root code, [raw vector], [small codes, coefficients].
        if (buf.capacity() - buf.size() < rec)
            buf.reserve(std::max(buf.size() + rec, std::max<size_t>(buf.capacity() * 3 / 2, 1u << 20)));
        const size_t at = buf.size();
        buf.resize(at + rec);
        uint8_t* p = buf.data() + at;
        std::memcpy(p, &gid, 4);
        std::memcpy(p + 4, &cid, 4);
        p += 8;
        if (xb) std::memcpy(p, s.x + static_cast<size_t>(i) * xb, xb);
        p += xb;
        if (cb) std::memcpy(p, s.codes + static_cast<size_t>(i) * mc, cb);
        p += cb;
        if (ab) std::memcpy(p, s.a + static_cast<size_t>(i) * st->m, ab);
        if (buf.size() >= st->flush_bytes && !FlushBucket(st, b, err)) return false;
    }
    return true;
}

void WriterLoop(stlq_b200_store* st) {
    for (;;) {
        int id;
        {
            std::unique_lock<std::mutex> lock(st->mu);
            st->cv.wait(lock, [&] { return st->stop || !st->queue.empty(); });
            if (st->queue.empty()) return;  // stop requested and nothing left
            id = st->queue.front();
        }
        Slot& s = st->slots[id];
        std::string err;
        bool ok = true;
        if (s.copied) {
            cudaSetDevice(st->device);
            const cudaError_t e = cudaEventSynchronize(s.copied);
            if (e != cudaSuccess) {
                ok = false;
                err = std::string("staging copy: ") + cudaGetErrorString(e);
            }
        }
        if (ok && st->error.empty()) ok = WriteBlock(st, s, &err);
        std::lock_guard<std::mutex> lock(st->mu);
        if (!ok && st->error.empty()) st->error = err;
        s.busy = false;
        st->queue.pop_front();
        st->cv.notify_all();
    }
}

int Fail(int code, const std::string& msg) { return SetError(code, ("stlq_b200 store: " + msg).c_str()); }

int AllocSlot(stlq_b200_store* st, Slot& s, int64_t cap) {
    const int mc = std::max(0, st->m - 1);
    s.cap = cap;
    if (st->device < 0) {
        s.cluster_host.resize(cap);
        s.codes_host.resize(static_cast<size_t>(mc) * cap);
        s.a_host.resize(static_cast<size_t>(st->m) * cap);
        s.x_host.resize(st->vec_bucket ? static_cast<size_t>(st->raw_bytes) * cap : 0);
        s.cluster = s.cluster_host.data();
        s.codes = s.codes_host.data();
        s.a = s.a_host.data();
        s.x = s.x_host.data();
        return 0;
    }
    const size_t xb = st->vec_bucket ? static_cast<size_t>(st->raw_bytes) * cap : 0;
    if (cudaMallocHost(reinterpret_cast<void**>(&s.cluster), sizeof(uint32_t) * cap) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&s.codes), std::max<size_t>(1, static_cast<size_t>(mc) * cap)) !=
            cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&s.a), sizeof(float) * st->m * cap) != cudaSuccess ||
        (xb && cudaMallocHost(reinterpret_cast<void**>(&s.x), xb) != cudaSuccess) ||
        cudaEventCreateWithFlags(&s.copied, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return Fail(STLQ_B200_ENOMEM, "pinned staging buffers");
    }
    return 0;
}

void FreeSlot(stlq_b200_store* st, Slot& s) {
    if (st->device < 0) return;
    if (s.cluster) cudaFreeHost(s.cluster);
    if (s.codes) cudaFreeHost(s.codes);
    if (s.a) cudaFreeHost(s.a);
    if (s.x) cudaFreeHost(s.x);
    if (s.copied) cudaEventDestroy(s.copied);
    s = Slot{};
}

// Waits until the writer has drained every queued block; returns its first error, if any.
int Drain(stlq_b200_store* st) {
    std::unique_lock<std::mutex> lock(st->mu);
    st->cv.wait(lock, [&] { return st->queue.empty(); });
    if (!st->error.empty()) return Fail(STLQ_B200_EDEVICE, st->error);
    return 0;
}

}  // namespace

namespace stlq_b200 {

// For the block loop (pipeline.cpp).
void StoreShape(const stlq_b200_store* st, int* device, int* d, int* m, int* raw_bytes, int64_t* max_block) {
    *device = st->device;
    *d = st->d;
    *m = st->m;
    *raw_bytes = st->raw_bytes;
    *max_block = st->slots.empty() ? 0 : st->slots[0].cap;
}

}  // namespace stlq_b200

extern "C" {

int stlq_b200_store_open(const char* dir, int d, int m, const int* h_vec, int shard_size, int bucket_size,
                         int bucket_flush_mb, int write_vector_bucket, int write_basic_to_bucket, int raw_bytes_per_vec,
                         int device, int64_t max_block, stlq_b200_store** out) {
    if (!out) return Fail(STLQ_B200_EINVAL, "out is null");
    *out = nullptr;
    if (!dir || !*dir || d <= 0 || m <= 0 || !h_vec || max_block < 1)
        return Fail(STLQ_B200_EINVAL, "dir, d > 0, m > 0, h_vec and max_block >= 1 are required");
    auto* st = new stlq_b200_store();
    st->dir = dir;
    st->d = d;
    st->m = m;
    st->h_vec.assign(h_vec, h_vec + m);
    st->shard_size = shard_size;
    st->vec_bucket = write_vector_bucket != 0;
    st->basic_bucket = write_basic_to_bucket != 0;
    st->raw_bytes = st->vec_bucket ? (raw_bytes_per_vec > 0 ? raw_bytes_per_vec : d) : 0;
    st->flush_bytes = static_cast<size_t>(std::max(1, bucket_flush_mb)) * 1024ull * 1024ull;
    st->device = device;
    auto fail = [&](int rc) {
        stlq_b200_store_close(st);
        return rc;
    };
    std::error_code ec;
    std::filesystem::create_directories(st->dir, ec);
    if (ec) return fail(Fail(STLQ_B200_EINVAL, "cannot create " + st->dir));
    // Every bucket the root can address is truncated now, so no earlier run's records remain.
    const int h0 = h_vec[0];
    const int nbucket = h0 > 0 ? (h0 + std::max(1, bucket_size) - 1) / std::max(1, bucket_size) : 0;
    for (int b = 0; b < nbucket; ++b) {
        FILE* f = std::fopen((st->dir + "/bucket_" + Tag(b) + ".bin").c_str(), "wb");
        if (f) std::fclose(f);
    }
    FILE* meta = std::fopen((st->dir + "/meta.json").c_str(), "wb");
    if (!meta) return fail(Fail(STLQ_B200_EINVAL, "cannot write meta.json"));
    std::string js = "{\n  \"d\": " + std::to_string(d) + ",\n  \"m\": " + std::to_string(m) +
                     ",\n  \"m_codes\": " + std::to_string(std::max(0, m - 1)) + ",\n  \"shard_size\": " +
                     std::to_string(shard_size) + ",\n  \"bucket_size\": " + std::to_string(bucket_size) +
                     ",\n  \"write_vector_bucket\": " + (st->vec_bucket ? "true" : "false") +
                     ",\n  \"write_basic_to_bucket\": " + (st->basic_bucket ? "true" : "false") +
                     ",\n  \"raw_bytes_per_vec\": " + std::to_string(st->raw_bytes) + ",\n  \"h_vec\": [";
    for (int i = 0; i < m; ++i) js += (i ? ", " : "") + std::to_string(h_vec[i]);
    js += "]\n}\n";
    const bool meta_ok = WriteAll(meta, js.data(), js.size());
    std::fclose(meta);
    // meta.bin: magic "CBAS", version 2, d, m, m_codes, shard_size, bucket_size, flags, h_len,
    // raw_bytes_per_vec (32-bit little-endian), then h_vec.
    const int32_t hdr[10] = {0x53414243, 2, d, m, std::max(0, m - 1), shard_size, bucket_size,
                             (st->vec_bucket ? 1 : 0) | (st->basic_bucket ? 2 : 0), m, st->raw_bytes};
    FILE* mb = std::fopen((st->dir + "/meta.bin").c_str(), "wb");
    const bool mb_ok = mb && WriteAll(mb, hdr, sizeof(hdr)) && WriteAll(mb, h_vec, sizeof(int) * m);
    if (mb) std::fclose(mb);
    if (!meta_ok || !mb_ok) return fail(Fail(STLQ_B200_EINVAL, "cannot write meta.bin"));
    st->bucket_size = bucket_size > 0 ? bucket_size : 256;
    st->cluster_f = std::fopen((st->dir + "/cluster_id.u32").c_str(), "wb");
    if (!st->cluster_f) return fail(Fail(STLQ_B200_EINVAL, "cannot open cluster_id.u32"));
    // Three staging slots: one being filled while two are written.
    st->slots.resize(st->device < 0 ? 1 : 3);
    if (st->device >= 0) {
        if (cudaSetDevice(st->device) != cudaSuccess ||
            cudaStreamCreateWithFlags(&st->copy, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            return fail(Fail(STLQ_B200_ECUDA, "copy stream"));
        }
    }
    for (auto& s : st->slots)
        if (int rc = AllocSlot(st, s, max_block)) return fail(rc);
    st->writer = std::thread(WriterLoop, st);
    *out = st;
    return 0;
}

int stlq_b200_store_append(stlq_b200_store* st, uint64_t start_id, int64_t n, const uint32_t* cluster,
                           const uint8_t* B_small, const float* a, const void* x_raw, int64_t ld_x_bytes,
                           void* stream) {
    if (!st) return Fail(STLQ_B200_EINVAL, "store handle is null");
    if (n <= 0) return 0;
    if (n > st->slots[0].cap) return Fail(STLQ_B200_EINVAL, "block larger than the store's max_block");
    if (!cluster || !a || (st->m > 1 && !B_small) || (st->vec_bucket && (!x_raw || ld_x_bytes < st->raw_bytes)))
        return Fail(STLQ_B200_EINVAL, "null block buffer (or raw vectors missing for write_vector_bucket)");
    int id = -1;
    {
        std::unique_lock<std::mutex> lock(st->mu);
        if (!st->error.empty()) return Fail(STLQ_B200_EDEVICE, st->error);
        st->cv.wait(lock, [&] {
            for (size_t i = 0; i < st->slots.size(); ++i)
                if (!st->slots[i].busy) return true;
            return false;
        });
        for (size_t i = 0; i < st->slots.size(); ++i)
            if (!st->slots[i].busy) {
                id = static_cast<int>(i);
                break;
            }
        st->slots[id].busy = true;
    }
    Slot& s = st->slots[id];
    s.start_id = start_id;
    s.n = n;
    const int mc = std::max(0, st->m - 1);
    const size_t xrow = static_cast<size_t>(st->raw_bytes);
    if (st->device < 0) {
        std::memcpy(s.cluster, cluster, sizeof(uint32_t) * n);
        if (mc) std::memcpy(s.codes, B_small, static_cast<size_t>(mc) * n);
        std::memcpy(s.a, a, sizeof(float) * st->m * n);
        if (st->vec_bucket)
            for (int64_t i = 0; i < n; ++i)
                std::memcpy(s.x + i * xrow, static_cast<const uint8_t*>(x_raw) + i * ld_x_bytes, xrow);
    } else {
        // After the producer's work on `stream`, on the copy stream.
        cudaSetDevice(st->device);
        cudaEvent_t ready = nullptr;
        cudaError_t e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventRecord(ready, static_cast<cudaStream_t>(stream));
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st->copy, ready, 0);
        if (ready) cudaEventDestroy(ready);
        if (e == cudaSuccess) e = cudaMemcpyAsync(s.cluster, cluster, sizeof(uint32_t) * n, cudaMemcpyDefault, st->copy);
        if (e == cudaSuccess && mc)
            e = cudaMemcpyAsync(s.codes, B_small, static_cast<size_t>(mc) * n, cudaMemcpyDefault, st->copy);
        if (e == cudaSuccess) e = cudaMemcpyAsync(s.a, a, sizeof(float) * st->m * n, cudaMemcpyDefault, st->copy);
        if (e == cudaSuccess && st->vec_bucket)
            e = cudaMemcpy2DAsync(s.x, xrow, x_raw, static_cast<size_t>(ld_x_bytes), xrow, static_cast<size_t>(n),
                                  cudaMemcpyDefault, st->copy);
        if (e == cudaSuccess) e = cudaEventRecord(s.copied, st->copy);
        // Later work on the caller's stream (which may reuse or free the block's buffers) waits
        // for the staging copy.
        if (e == cudaSuccess) e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), s.copied, 0);
        if (e != cudaSuccess) {
            cudaGetLastError();
            std::lock_guard<std::mutex> lock(st->mu);
            s.busy = false;
            st->cv.notify_all();
            return Fail(STLQ_B200_ECUDA, std::string("staging copy: ") + cudaGetErrorString(e));
        }
    }
    std::lock_guard<std::mutex> lock(st->mu);
    st->queue.push_back(id);
    st->cv.notify_all();
    return 0;
}

int stlq_b200_store_flush(stlq_b200_store* st) {
    if (!st) return Fail(STLQ_B200_EINVAL, "store handle is null");
    if (int rc = Drain(st)) return rc;
    std::string err;
    for (size_t b = 0; b < st->bucket_f.size(); ++b)
        if (st->bucket_f[b] && (!FlushBucket(st, b, &err) || std::fflush(st->bucket_f[b]) != 0))
            return Fail(STLQ_B200_EDEVICE, err.empty() ? "bucket flush failed" : err);
    for (FILE* f : {st->cluster_f, st->codes_f, st->coeffs_f})
        if (f && std::fflush(f) != 0) return Fail(STLQ_B200_EDEVICE, "flush failed");
    return 0;
}

int stlq_b200_store_close(stlq_b200_store* st) {
    if (!st) return 0;
    int rc = 0;
    if (st->writer.joinable()) {
        rc = stlq_b200_store_flush(st);
        {
            std::lock_guard<std::mutex> lock(st->mu);
            st->stop = true;
            st->cv.notify_all();
        }
        st->writer.join();
    }
    for (FILE* f : st->bucket_f)
        if (f) std::fclose(f);
    for (FILE* f : {st->cluster_f, st->codes_f, st->coeffs_f})
        if (f) std::fclose(f);
    if (st->device >= 0) {
        cudaSetDevice(st->device);
        if (st->copy) cudaStreamSynchronize(st->copy);
        for (auto& s : st->slots) FreeSlot(st, s);
        if (st->copy) cudaStreamDestroy(st->copy);
    }
    delete st;
    return rc;
}

}  // extern "C"
