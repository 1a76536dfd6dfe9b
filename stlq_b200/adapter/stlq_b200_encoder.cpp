// Drop-in C++ adapter: the reference's encode-stage signatures on top of the stlq_b200 C-ABI.
// See stlq_b200_encoder.h for the mapping to the reference's functions.
#include "stlq_b200_encoder.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "stlq_b200.h"

namespace stlq {
namespace b200 {

namespace {

struct CachedEncoder {
    int device;
    std::uint64_t build_tag;
    const float* c_all;
    int H, d;
    stlq_b200_encoder* handle;
};

struct ThreadEncoders {
    std::vector<CachedEncoder> items;
    ~ThreadEncoders() {
        for (auto& e : items) stlq_b200_destroy(e.handle);
    }
};

ThreadEncoders& Cache() {
    static thread_local ThreadEncoders c;
    return c;
}

[[noreturn]] void Throw(const char* what) {
    throw std::runtime_error(std::string("stlq_b200: ") + what + ": " + stlq_b200_last_error());
}

void Check(int rc, const char* what) {
    if (rc != 0) Throw(what);
}

void CheckCuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("stlq_b200 adapter: ") + what + ": " + cudaGetErrorString(e));
}

// The encoder for this Precomp on `device`, created on first use: C_all, G and invnorm_flat are
// handed over as the reference computed them (BuildPrecomp), so the device never re-derives them.
stlq_b200_encoder* EncoderFor(const Precomp& pre, int device) {
    auto& items = Cache().items;
    for (auto& e : items) {
        if (e.device == device && e.build_tag == pre.build_tag && e.c_all == pre.C_all.data.data() && e.H == pre.H &&
            e.d == pre.d)
            return e.handle;
    }
    stlq_b200_encoder* h = nullptr;
    Check(stlq_b200_create(device, pre.d, pre.m, pre.h_vec.data(), pre.C_all.data.data(), pre.G.data.data(),
                           pre.invnorm_flat.data(), STLQ_B200_GEMM_EXACT, &h),
          "stlq_b200_create");
    items.push_back({device, pre.build_tag, pre.C_all.data.data(), pre.H, pre.d, h});
    return h;
}

// The large-root encoder for this PrecompLargeRoot: C_all = [C0 | C_small] (root codewords first);
// G, norm0 and invnorm are derived on the device in the reference's orders.
stlq_b200_encoder* LargeRootEncoderFor(const PrecompLargeRoot& pre, int device) {
    auto& items = Cache().items;
    const int H = pre.h_vec.empty() ? 0 : pre.h_vec[0] + pre.H_small;
    for (auto& e : items) {
        if (e.device == device && e.build_tag == pre.build_tag && e.c_all == pre.C0.data.data() && e.H == H &&
            e.d == pre.d)
            return e.handle;
    }
    std::vector<float> c_all(static_cast<size_t>(pre.d) * H);
    std::memcpy(c_all.data(), pre.C0.data.data(), sizeof(float) * pre.C0.data.size());
    std::memcpy(c_all.data() + pre.C0.data.size(), pre.C_small.data.data(), sizeof(float) * pre.C_small.data.size());
    stlq_b200_encoder* h = nullptr;
    Check(stlq_b200_create_large_root(device, pre.d, pre.m, pre.h_vec.data(), c_all.data(), STLQ_B200_GEMM_EXACT, &h),
          "stlq_b200_create_large_root");
    items.push_back({device, pre.build_tag, pre.C0.data.data(), H, pre.d, h});
    return h;
}

// Device scratch for the host-buffer stage adapters.
struct DeviceBuffer {
    void* p = nullptr;
    explicit DeviceBuffer(size_t bytes) { CheckCuda(cudaMalloc(&p, std::max<size_t>(bytes, 1)), "cudaMalloc"); }
    ~DeviceBuffer() { cudaFree(p); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

void Upload(void* dst, const void* src, size_t bytes) {
    CheckCuda(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
}

void Download(void* dst, const void* src, size_t bytes) {
    CheckCuda(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
}

void IcmCommon(const ColMajorMatrix<float>& X, const Precomp& precomp, const ColMajorMatrix<float>& xC, int icm_iters,
               int ils_iters, int perturb_k, std::uint32_t seed, ColMajorMatrix<FullCode>* B, ColMajorMatrix<float>* a,
               std::vector<float>* X_norm2, std::vector<float>* cost, std::uint64_t sample_id_offset, int device,
               int use_abs) {
    if (!B || !a) return;
    const int n = B->cols, m = precomp.m, H = precomp.H, d = X.rows;
    stlq_b200_encoder* enc = EncoderFor(precomp, device);
    CheckCuda(cudaSetDevice(device), "cudaSetDevice");
    DeviceBuffer dxc(sizeof(float) * static_cast<size_t>(H) * n), dn(sizeof(float) * n), dB(static_cast<size_t>(m) * n),
        da(sizeof(float) * static_cast<size_t>(m) * n), dc(sizeof(float) * n);
    Upload(dxc.p, xC.data.data(), sizeof(float) * static_cast<size_t>(H) * n);
    Upload(dB.p, B->data.data(), static_cast<size_t>(m) * n);
    if (X_norm2 && X_norm2->size() == static_cast<size_t>(n)) {
        Upload(dn.p, X_norm2->data(), sizeof(float) * n);
    } else {
        DeviceBuffer dX(sizeof(float) * static_cast<size_t>(d) * n);
        Upload(dX.p, X.data.data(), sizeof(float) * static_cast<size_t>(d) * n);
        Check(stlq_b200_xnorm2(enc, dX.p, STLQ_B200_F32, n, dn.as<float>(), nullptr), "stlq_b200_xnorm2");
        Check(stlq_b200_sync(enc, nullptr), "stlq_b200_sync");
    }
    Check(stlq_b200_icm(enc, dxc.as<float>(), dn.as<float>(), n, icm_iters, ils_iters, perturb_k, use_abs, seed,
                        sample_id_offset, dB.as<std::uint8_t>(), da.as<float>(), dc.as<float>(), nullptr),
          "stlq_b200_icm");
    Check(stlq_b200_sync(enc, nullptr), "stlq_b200_sync");
    Download(B->data.data(), dB.p, static_cast<size_t>(m) * n);
    a->rows = m;
    a->cols = n;
    a->data.resize(static_cast<size_t>(m) * n);
    Download(a->data.data(), da.p, sizeof(float) * static_cast<size_t>(m) * n);
    if (X_norm2 && X_norm2->size() != static_cast<size_t>(n)) {
        X_norm2->resize(n);
        Download(X_norm2->data(), dn.p, sizeof(float) * n);
    }
    if (cost) {
        cost->resize(n);
        Download(cost->data(), dc.p, sizeof(float) * n);
    }
}

}  // namespace

bool EncodeBase(const Config& config, const Dataset& dataset, const CodebookPack& codebooks, const Precomp& precomp,
                KernelProvider* kernels, BaseEncoding* base, float* out_beam_mse, float* out_final_mse,
                std::string* error) {
    (void)kernels;
    if (!base) {
        if (error) *error = "BaseEncoding output is null.";
        return false;
    }
    const int d = dataset.Xb.rows, n = dataset.Xb.cols;
    if (d <= 0 || n <= 0) {
        if (error) *error = "Empty base dataset.";
        return false;
    }
    if (precomp.d != d || precomp.m != static_cast<int>(codebooks.books.size())) {
        if (error) *error = "Precomp dimensions do not match codebooks or dataset.";
        return false;
    }
    try {
        stlq_b200_encoder* enc = EncoderFor(precomp, config.runtime.cuda_device);
        const auto& e = config.base.encode;
        const int m = precomp.m;
        base->B = ColMajorMatrix<FullCode>(m, n);
        base->a = ColMajorMatrix<float>(m, n);
        double sse[2] = {0.0, 0.0};
        Check(stlq_b200_encode_base(enc, dataset.Xb.data.data(), STLQ_B200_F32, n, std::max(1, e.H_beam), e.icm_iters,
                                    e.ils_iters, e.perturb_k, e.use_abs ? 1 : 0, static_cast<std::uint32_t>(e.seed), 0,
                                    base->B.data.data(), base->a.data.data(), nullptr, sse),
              "stlq_b200_encode_base");
        if (out_beam_mse) *out_beam_mse = static_cast<float>(sse[0] / n);
        if (out_final_mse) *out_final_mse = static_cast<float>(sse[1] / n);
    } catch (const std::exception& ex) {
        if (error) *error = ex.what();
        return false;
    }
    return true;
}

namespace {

// Sharded encoders cached per (thread, device list, Precomp), like the single-device ones.
struct CachedSharded {
    std::vector<int> devices;
    std::uint64_t build_tag;
    const float* c_all;
    int H, d;
    stlq_b200_sharded* handle;
};
struct ThreadSharded {
    std::vector<CachedSharded> items;
    ~ThreadSharded() {
        for (auto& e : items) stlq_b200_sharded_destroy(e.handle);
    }
};

stlq_b200_sharded* ShardedFor(const Precomp& pre, const std::vector<int>& devices) {
    static thread_local ThreadSharded cache;
    for (auto& e : cache.items)
        if (e.devices == devices && e.build_tag == pre.build_tag && e.c_all == pre.C_all.data.data() && e.H == pre.H &&
            e.d == pre.d)
            return e.handle;
    stlq_b200_sharded* h = nullptr;
    Check(stlq_b200_sharded_create(static_cast<int>(devices.size()), devices.data(), pre.d, pre.m, pre.h_vec.data(),
                                   pre.C_all.data.data(), pre.G.data.data(), pre.invnorm_flat.data(),
                                   STLQ_B200_GEMM_EXACT, &h),
          "stlq_b200_sharded_create");
    cache.items.push_back({devices, pre.build_tag, pre.C_all.data.data(), pre.H, pre.d, h});
    return h;
}

}  // namespace

bool EncodeBaseSharded(const Config& config, const Dataset& dataset, const CodebookPack& codebooks,
                       const Precomp& precomp, const std::vector<int>& devices, BaseEncoding* base,
                       float* out_beam_mse, float* out_final_mse, std::string* error) {
    if (!base) {
        if (error) *error = "BaseEncoding output is null.";
        return false;
    }
    const int d = dataset.Xb.rows, n = dataset.Xb.cols;
    if (d <= 0 || n <= 0) {
        if (error) *error = "Empty base dataset.";
        return false;
    }
    if (precomp.d != d || precomp.m != static_cast<int>(codebooks.books.size())) {
        if (error) *error = "Precomp dimensions do not match codebooks or dataset.";
        return false;
    }
    try {
        const std::vector<int> devs = devices.empty() ? std::vector<int>{config.runtime.cuda_device} : devices;
        stlq_b200_sharded* sh = ShardedFor(precomp, devs);
        const auto& e = config.base.encode;
        const int m = precomp.m;
        base->B = ColMajorMatrix<FullCode>(m, n);
        base->a = ColMajorMatrix<float>(m, n);
        double sse[2] = {0.0, 0.0};
        Check(stlq_b200_encode_sharded(sh, dataset.Xb.data.data(), STLQ_B200_F32, n, std::max(1, e.H_beam), e.icm_iters,
                                       e.ils_iters, e.perturb_k, e.use_abs ? 1 : 0, static_cast<std::uint32_t>(e.seed),
                                       0, base->B.data.data(), base->a.data.data(), nullptr, sse),
              "stlq_b200_encode_sharded");
        if (out_beam_mse) *out_beam_mse = static_cast<float>(sse[0] / n);
        if (out_final_mse) *out_final_mse = static_cast<float>(sse[1] / n);
    } catch (const std::exception& ex) {
        if (error) *error = ex.what();
        return false;
    }
    return true;
}

void BeamSearchPrefixLS(const ColMajorMatrix<float>& X, const Precomp& precomp, const ColMajorMatrix<float>& xC,
                        int H_beam, ColMajorMatrix<FullCode>* B, int device) {
    const int n = X.cols, d = X.rows, m = precomp.m, H = precomp.H;
    stlq_b200_encoder* enc = EncoderFor(precomp, device);
    CheckCuda(cudaSetDevice(device), "cudaSetDevice");
    DeviceBuffer dX(sizeof(float) * static_cast<size_t>(d) * n), dxc(sizeof(float) * static_cast<size_t>(H) * n),
        dn(sizeof(float) * n), dB(static_cast<size_t>(m) * n);
    Upload(dX.p, X.data.data(), sizeof(float) * static_cast<size_t>(d) * n);
    Upload(dxc.p, xC.data.data(), sizeof(float) * static_cast<size_t>(H) * n);
    Check(stlq_b200_xnorm2(enc, dX.p, STLQ_B200_F32, n, dn.as<float>(), nullptr), "stlq_b200_xnorm2");
    Check(stlq_b200_beam_search(enc, dn.as<float>(), dxc.as<float>(), n, std::max(1, H_beam), dB.as<std::uint8_t>(),
                                nullptr),
          "stlq_b200_beam_search");
    Check(stlq_b200_sync(enc, nullptr), "stlq_b200_sync");
    B->rows = m;
    B->cols = n;
    B->data.resize(static_cast<size_t>(m) * n);
    Download(B->data.data(), dB.p, static_cast<size_t>(m) * n);
}

void SolveLeastSquaresAll(const Precomp& precomp, const ColMajorMatrix<float>& xC, const ColMajorMatrix<FullCode>& B,
                          ColMajorMatrix<float>* a, int device) {
    const int n = B.cols, m = precomp.m, H = precomp.H;
    stlq_b200_encoder* enc = EncoderFor(precomp, device);
    CheckCuda(cudaSetDevice(device), "cudaSetDevice");
    DeviceBuffer dxc(sizeof(float) * static_cast<size_t>(H) * n), dB(static_cast<size_t>(m) * n),
        da(sizeof(float) * static_cast<size_t>(m) * n);
    Upload(dxc.p, xC.data.data(), sizeof(float) * static_cast<size_t>(H) * n);
    Upload(dB.p, B.data.data(), static_cast<size_t>(m) * n);
    Check(stlq_b200_solve_ls(enc, dxc.as<float>(), dB.as<std::uint8_t>(), n, da.as<float>(), nullptr),
          "stlq_b200_solve_ls");
    Check(stlq_b200_sync(enc, nullptr), "stlq_b200_sync");
    a->rows = m;
    a->cols = n;
    a->data.resize(static_cast<size_t>(m) * n);
    Download(a->data.data(), da.p, sizeof(float) * static_cast<size_t>(m) * n);
}

void DynamicIcmWithIlsAbsNoNormalCuda(const ColMajorMatrix<float>& X, const Precomp& precomp,
                                      const ColMajorMatrix<float>& xC, int icm_iters, int ils_iters, int perturb_k,
                                      std::uint32_t seed, ColMajorMatrix<FullCode>* B, ColMajorMatrix<float>* a,
                                      std::vector<float>* X_norm2, std::vector<float>* cost, bool print_progress,
                                      std::uint64_t sample_id_offset, int device) {
    (void)print_progress;
    IcmCommon(X, precomp, xC, icm_iters, ils_iters, perturb_k, seed, B, a, X_norm2, cost, sample_id_offset, device, 1);
}

void DynamicIcmWithIlsNoAbsNoNormalCuda(const ColMajorMatrix<float>& X, const Precomp& precomp,
                                        const ColMajorMatrix<float>& xC, int icm_iters, int ils_iters, int perturb_k,
                                        std::uint32_t seed, ColMajorMatrix<FullCode>* B, ColMajorMatrix<float>* a,
                                        std::vector<float>* X_norm2, std::vector<float>* cost, bool print_progress,
                                        std::uint64_t sample_id_offset, int device) {
    (void)print_progress;
    IcmCommon(X, precomp, xC, icm_iters, ils_iters, perturb_k, seed, B, a, X_norm2, cost, sample_id_offset, device, 0);
}

void EncodeBaseLargeRoot(const PrecompLargeRoot& pre, const ColMajorMatrix<float>& Xblk, int H_beam, int icm_iters,
                         int ils_iters, int perturb_k, bool use_abs, std::uint32_t seed,
                         std::uint64_t sample_id_offset, std::vector<std::uint32_t>* cluster_id,
                         ColMajorMatrix<Code>* B_small, ColMajorMatrix<float>* a, std::vector<float>* cost,
                         float* out_beam_mse, float* out_final_mse, int device) {
    if (!cluster_id || !B_small || !a) return;
    const int n = Xblk.cols, m = pre.m;
    cluster_id->resize(static_cast<size_t>(n));
    B_small->rows = std::max(0, m - 1);
    B_small->cols = n;
    B_small->data.resize(static_cast<size_t>(B_small->rows) * n);
    a->rows = m;
    a->cols = n;
    a->data.resize(static_cast<size_t>(m) * n);
    std::vector<float> c(static_cast<size_t>(n));
    if (n <= 0) return;
    stlq_b200_encoder* enc = LargeRootEncoderFor(pre, device);
    double sums[2] = {0.0, 0.0};
    Check(stlq_b200_encode_base_large_root(enc, Xblk.data.data(), STLQ_B200_F32, n, std::max(1, H_beam), icm_iters,
                                           ils_iters, perturb_k, use_abs ? 1 : 0, seed, sample_id_offset,
                                           cluster_id->data(), B_small->data.data(), a->data.data(), c.data(), sums),
          "stlq_b200_encode_base_large_root");
    if (cost) *cost = std::move(c);
    if (out_beam_mse) *out_beam_mse = static_cast<float>(sums[0] / n);
    if (out_final_mse) *out_final_mse = static_cast<float>(sums[1] / n);
}

void ReleaseThreadEncoders() {
    auto& items = Cache().items;
    for (auto& e : items) stlq_b200_destroy(e.handle);
    items.clear();
}

}  // namespace b200
}  // namespace stlq
