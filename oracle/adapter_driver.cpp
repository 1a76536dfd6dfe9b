// Test infrastructure only: drives the drop-in adapter (stlq_b200/adapter) with the reference's own
// types, so a GPU test can compare stlq::b200::EncodeBase & co. against the reference's functions
// on the same Precomp object (created by ref_precomp_create in ref_driver.cpp).
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "stlq/common/config.h"
#include "stlq/common/types.h"
#include "stlq_b200_encoder.h"

extern "C" int adapter_encode_base(void* pre_h, const float* X, int n, int beam, int icm, int ils, int perturb,
                                   int use_abs, int seed, int device, std::uint8_t* B_out, float* a_out,
                                   float* mse_out, char* err, int errlen) {
    const auto* pre = static_cast<const stlq::Precomp*>(pre_h);
    stlq::Config cfg;
    cfg.base.encode.H_beam = beam;
    cfg.base.encode.icm_iters = icm;
    cfg.base.encode.ils_iters = ils;
    cfg.base.encode.perturb_k = perturb;
    cfg.base.encode.use_abs = use_abs != 0;
    cfg.base.encode.seed = seed;
    cfg.runtime.use_cuda = true;
    cfg.runtime.cuda_device = device;
    stlq::Dataset ds;
    ds.Xb = stlq::ColMajorMatrix<float>(pre->d, n);
    std::memcpy(ds.Xb.data.data(), X, sizeof(float) * static_cast<size_t>(pre->d) * n);
    stlq::CodebookPack books;
    books.d = pre->d;
    books.h_vec = pre->h_vec;
    books.books.resize(pre->m);
    stlq::BaseEncoding base;
    std::string e;
    float bm = 0.0f, fm = 0.0f;
    const bool ok = stlq::b200::EncodeBase(cfg, ds, books, *pre, nullptr, &base, &bm, &fm, &e);
    if (!ok) {
        std::strncpy(err, e.c_str(), static_cast<size_t>(errlen) - 1);
        err[errlen - 1] = 0;
        return 1;
    }
    std::memcpy(B_out, base.B.data.data(), base.B.data.size());
    std::memcpy(a_out, base.a.data.data(), sizeof(float) * base.a.data.size());
    mse_out[0] = bm;
    mse_out[1] = fm;
    return 0;
}

extern "C" int adapter_stages(void* pre_h, const float* X, int n, const float* xC, int beam, int icm, int ils,
                              int perturb, int use_abs, unsigned seed, int device, std::uint8_t* B_beam,
                              float* a_beam, std::uint8_t* B_icm, float* a_icm, float* cost, char* err, int errlen) {
    const auto* pre = static_cast<const stlq::Precomp*>(pre_h);
    try {
        stlq::ColMajorMatrix<float> Xm(pre->d, n), xCm(pre->H, n);
        std::memcpy(Xm.data.data(), X, sizeof(float) * static_cast<size_t>(pre->d) * n);
        std::memcpy(xCm.data.data(), xC, sizeof(float) * static_cast<size_t>(pre->H) * n);
        stlq::ColMajorMatrix<stlq::FullCode> B;
        stlq::b200::BeamSearchPrefixLS(Xm, *pre, xCm, beam, &B, device);
        std::memcpy(B_beam, B.data.data(), B.data.size());
        stlq::ColMajorMatrix<float> a;
        stlq::b200::SolveLeastSquaresAll(*pre, xCm, B, &a, device);
        std::memcpy(a_beam, a.data.data(), sizeof(float) * a.data.size());
        std::vector<float> xn, c;
        if (use_abs)
            stlq::b200::DynamicIcmWithIlsAbsNoNormalCuda(Xm, *pre, xCm, icm, ils, perturb, seed, &B, &a, &xn, &c,
                                                         false, 0, device);
        else
            stlq::b200::DynamicIcmWithIlsNoAbsNoNormalCuda(Xm, *pre, xCm, icm, ils, perturb, seed, &B, &a, &xn, &c,
                                                           false, 0, device);
        std::memcpy(B_icm, B.data.data(), B.data.size());
        std::memcpy(a_icm, a.data.data(), sizeof(float) * a.data.size());
        std::memcpy(cost, c.data(), sizeof(float) * c.size());
    } catch (const std::exception& ex) {
        std::strncpy(err, ex.what(), static_cast<size_t>(errlen) - 1);
        err[errlen - 1] = 0;
        return 1;
    }
    return 0;
}

extern "C" void adapter_release(void) { stlq::b200::ReleaseThreadEncoders(); }

// The large-root drop-in (stlq::b200::EncodeBaseLargeRoot) on a PrecompLargeRoot built by the
// reference's BuildPrecompLargeRoot from C_all (d x H, root codewords first).
extern "C" int adapter_large_root_encode(int d, int m, const int* h_vec, const float* C_all, const float* X, int n,
                                         int beam, int icm, int ils, int perturb, int use_abs, unsigned seed,
                                         int device, std::uint32_t* cluster_out, std::uint8_t* B_small_out,
                                         float* a_out, float* cost_out, float* mse_out, char* err, int errlen) {
    try {
        stlq::CodebookPack pack;
        pack.d = d;
        int off = 0;
        for (int l = 0; l < m; ++l) {
            stlq::ColMajorMatrix<float> book(d, h_vec[l]);
            std::memcpy(book.data.data(), C_all + static_cast<size_t>(off) * d, sizeof(float) * book.data.size());
            pack.h_vec.push_back(h_vec[l]);
            pack.books.push_back(std::move(book));
            off += h_vec[l];
        }
        stlq::PrecompLargeRoot pre;
        stlq::PrecompLargeRootBuildOptions opts;
        std::string e;
        if (!stlq::BuildPrecompLargeRoot(pack, nullptr, opts, &pre, &e)) throw std::runtime_error(e);
        stlq::ColMajorMatrix<float> Xm(d, n);
        std::memcpy(Xm.data.data(), X, sizeof(float) * static_cast<size_t>(d) * n);
        std::vector<std::uint32_t> cluster;
        stlq::ColMajorMatrix<stlq::Code> B_small;
        stlq::ColMajorMatrix<float> a;
        std::vector<float> cost;
        stlq::b200::EncodeBaseLargeRoot(pre, Xm, beam, icm, ils, perturb, use_abs != 0, seed, 0, &cluster, &B_small,
                                        &a, &cost, &mse_out[0], &mse_out[1], device);
        std::memcpy(cluster_out, cluster.data(), sizeof(std::uint32_t) * n);
        std::memcpy(B_small_out, B_small.data.data(), B_small.data.size());
        std::memcpy(a_out, a.data.data(), sizeof(float) * a.data.size());
        std::memcpy(cost_out, cost.data(), sizeof(float) * n);
    } catch (const std::exception& ex) {
        std::strncpy(err, ex.what(), static_cast<size_t>(errlen) - 1);
        err[errlen - 1] = 0;
        return 1;
    }
    return 0;
}
