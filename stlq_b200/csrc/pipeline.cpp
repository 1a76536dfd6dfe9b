// The large pipeline's block loop on one GPU (reference: src/quantizer/encode_base_streaming.cpp,
// the basic-encode branch of the large pipeline, 640-1310): read a block of base vectors, encode it
// with the large-root encoder (sample ids from the block's first global id), append the block's
// root codes, small codes, coefficients and raw vectors to the basic store, and accumulate the
// block MSEs as the reference does (mse_sum += float(mean cost of the block) x block size,
// 1303-1304).
//
// Three streams carry the blocks: `cs` copies block k+1 into one of two device input buffers
// while `s` encodes block k from the other, and `h` hands block k's outputs to the store (whose
// staging copies then run on its own stream).  Events order buffer reuse: block k+2 is neither
// read into nor encoded into its buffers before block k's store copies are complete.
#include <algorithm>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/stlq_b200.h"

namespace stlq_b200 {
int SetError(int code, const char* msg);
void EncoderShape(const stlq_b200_encoder* enc, int* device, int* d, int* m, int* large_root);
void ReaderShape(const stlq_b200_reader* rd, int* device, int* d, int* x_dtype, int64_t* block, uint64_t* begin,
                 uint64_t* end);
void StoreShape(const stlq_b200_store* st, int* device, int* d, int* m, int* raw_bytes, int64_t* max_block);
}  // namespace stlq_b200

namespace {

using stlq_b200::SetError;

int Fail(int code, const std::string& msg) { return SetError(code, ("stlq_b200 block loop: " + msg).c_str()); }

struct DevMem {
    void* p = nullptr;
    ~DevMem() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

// Streams and events of one call; the destructor waits for all their work before releasing them.
struct Lanes {
    cudaStream_t cs = nullptr, s = nullptr, h = nullptr;
    cudaEvent_t in[2] = {}, enc[2] = {}, stored[2] = {};
    cudaError_t Create() {
        cudaError_t e = cudaSuccess;
        for (cudaStream_t* x : {&cs, &s, &h})
            if (e == cudaSuccess) e = cudaStreamCreateWithFlags(x, cudaStreamNonBlocking);
        for (int b = 0; b < 2; ++b)
            for (cudaEvent_t* x : {&in[b], &enc[b], &stored[b]})
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(x, cudaEventDisableTiming);
        return e;
    }
    ~Lanes() {
        for (cudaStream_t x : {cs, s, h})
            if (x) cudaStreamSynchronize(x);
        for (int b = 0; b < 2; ++b)
            for (cudaEvent_t x : {in[b], enc[b], stored[b]})
                if (x) cudaEventDestroy(x);
        for (cudaStream_t x : {cs, s, h})
            if (x) cudaStreamDestroy(x);
    }
};

}  // namespace

extern "C" int stlq_b200_encode_file_large_root(stlq_b200_encoder* enc, stlq_b200_reader* rd, stlq_b200_store* st,
                                                int beam, int icm_iters, int ils_iters, int perturb_k, int use_abs,
                                                uint32_t seed, double* mse_sums_out, int64_t* vectors_out) {
    if (!enc || !rd) return Fail(STLQ_B200_EINVAL, "encoder and reader are required");
    int dev = 0, d = 0, m = 0, large_root = 0;
    stlq_b200::EncoderShape(enc, &dev, &d, &m, &large_root);
    int rdev = 0, rd_d = 0, x_dtype = 0;
    int64_t block = 0;
    uint64_t begin = 0, end = 0;
    stlq_b200::ReaderShape(rd, &rdev, &rd_d, &x_dtype, &block, &begin, &end);
    if (!large_root) return Fail(STLQ_B200_EINVAL, "the encoder must be a large-root encoder");
    if (rdev != dev) return Fail(STLQ_B200_EINVAL, "the reader must copy to the encoder's device");
    if (rd_d != d) return Fail(STLQ_B200_EINVAL, "the file's dimension differs from the encoder's");
    const size_t elem = x_dtype == STLQ_B200_U8 ? 1 : 4;
    const size_t row = static_cast<size_t>(d) * elem;
    if (st) {
        int sdev = 0, sd = 0, sm = 0, raw = 0;
        int64_t smax = 0;
        stlq_b200::StoreShape(st, &sdev, &sd, &sm, &raw, &smax);
        if (sdev != dev) return Fail(STLQ_B200_EINVAL, "the store must stage from the encoder's device");
        if (sd != d || sm != m) return Fail(STLQ_B200_EINVAL, "the store's d and m differ from the encoder's");
        if (smax < block) return Fail(STLQ_B200_EINVAL, "the store's max_block is below the reader's block");
        if (static_cast<size_t>(raw) > row) return Fail(STLQ_B200_EINVAL, "the store's raw_bytes_per_vec exceeds a vector");
    }
    const int64_t nblocks = end > begin ? static_cast<int64_t>((end - begin + block - 1) / block) : 0;
    if (cudaSetDevice(dev) != cudaSuccess) return Fail(STLQ_B200_ECUDA, "cudaSetDevice");
    DevMem X[2], cl[2], Bs[2], a[2], cost[2], sums;
    const size_t nb = static_cast<size_t>(block);
    cudaError_t e = cudaSuccess;
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        e = cudaMalloc(&X[b].p, nb * row);
        if (e == cudaSuccess) e = cudaMalloc(&cl[b].p, nb * 4);
        if (e == cudaSuccess) e = cudaMalloc(&Bs[b].p, std::max<size_t>(1, nb * (m - 1)));
        if (e == cudaSuccess) e = cudaMalloc(&a[b].p, nb * m * 4);
        if (e == cudaSuccess) e = cudaMalloc(&cost[b].p, nb * 4);
    }
    if (e == cudaSuccess) e = cudaMalloc(&sums.p, sizeof(double) * 2 * std::max<int64_t>(1, nblocks));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return Fail(STLQ_B200_ENOMEM, std::string("block buffers: ") + cudaGetErrorString(e));
    }
    Lanes L;
    if ((e = L.Create()) != cudaSuccess) {
        cudaGetLastError();
        return Fail(STLQ_B200_ECUDA, std::string("streams: ") + cudaGetErrorString(e));
    }
    std::vector<int64_t> counts;
    uint64_t start = 0;
    int64_t cnt = 0;
    if (int rc = stlq_b200_reader_next(rd, X[0].p, nb * row, L.cs, &start, &cnt)) return rc;
    if ((e = cudaEventRecord(L.in[0], L.cs)) != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
    for (int64_t k = 0; cnt > 0; ++k) {
        if (k >= nblocks) return Fail(STLQ_B200_EINVAL, "the reader returned more blocks than its range holds");
        const int b = static_cast<int>(k & 1), o = b ^ 1;
        // Block k+1 into the other buffer once block k-1 is encoded and stored.
        uint64_t start2 = 0;
        int64_t cnt2 = 0;
        e = cudaStreamWaitEvent(L.cs, L.stored[o], 0);
        if (e != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        if (int rc = stlq_b200_reader_next(rd, X[o].p, nb * row, L.cs, &start2, &cnt2)) return rc;
        if (cnt2 > 0 && (e = cudaEventRecord(L.in[o], L.cs)) != cudaSuccess)
            return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        // Encode block k once it is on the device and block k-2's outputs are stored.
        e = cudaStreamWaitEvent(L.s, L.in[b], 0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(L.s, L.stored[b], 0);
        if (e != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        if (int rc = stlq_b200_encode_base_large_root_device(
                enc, X[b].p, x_dtype, cnt, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, start,
                cl[b].as<uint32_t>(), Bs[b].as<uint8_t>(), a[b].as<float>(), cost[b].as<float>(),
                sums.as<double>() + 2 * k, L.s))
            return rc;
        if ((e = cudaEventRecord(L.enc[b], L.s)) != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        // Hand block k to the store.
        if ((e = cudaStreamWaitEvent(L.h, L.enc[b], 0)) != cudaSuccess)
            return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        if (st) {
            if (int rc = stlq_b200_store_append(st, start, cnt, cl[b].as<uint32_t>(), Bs[b].as<uint8_t>(),
                                                a[b].as<float>(), X[b].p, static_cast<int64_t>(row), L.h))
                return rc;
        }
        if ((e = cudaEventRecord(L.stored[b], L.h)) != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
        counts.push_back(cnt);
        start = start2;
        cnt = cnt2;
    }
    for (cudaStream_t x : {L.cs, L.s, L.h})
        if ((e = cudaStreamSynchronize(x)) != cudaSuccess) return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
    if (int rc = stlq_b200_sync(enc, L.s)) return rc;
    std::vector<double> hs(2 * counts.size());
    if (!hs.empty() && (e = cudaMemcpy(hs.data(), sums.p, sizeof(double) * hs.size(), cudaMemcpyDeviceToHost)) !=
                           cudaSuccess)
        return Fail(STLQ_B200_ECUDA, cudaGetErrorString(e));
    double mse[2] = {0.0, 0.0};
    int64_t total = 0;
    for (size_t k = 0; k < counts.size(); ++k) {
        const double nk = static_cast<double>(counts[k]);
        for (int j = 0; j < 2; ++j) mse[j] += static_cast<double>(static_cast<float>(hs[2 * k + j] / nk)) * nk;
        total += counts[k];
    }
    if (mse_sums_out) {
        mse_sums_out[0] = mse[0];
        mse_sums_out[1] = mse[1];
    }
    if (vectors_out) *vectors_out = total;
    return 0;
}
