// Test infrastructure only: drives the drop-in adapter (stlq_b200/adapter) with the reference's own
// types, so a GPU test can compare stlq::b200::EncodeBase & co. against the reference's functions
// on the same Precomp object (created by ref_precomp_create in ref_driver.cpp).
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "stlq/common/config.h"
#include "stlq/common/types.h"
#include "stlq_b200_encoder.h"

// n_devices > 0: stlq::b200::EncodeBaseSharded on devices 0 .. n_devices-1 instead of EncodeBase.
extern "C" int adapter_encode_base_on(void* pre_h, const float* X, int n, int beam, int icm, int ils, int perturb,
                                      int use_abs, int seed, int device, int n_devices, std::uint8_t* B_out,
                                      float* a_out, float* mse_out, char* err, int errlen);

extern "C" int adapter_encode_base(void* pre_h, const float* X, int n, int beam, int icm, int ils, int perturb,
                                   int use_abs, int seed, int device, std::uint8_t* B_out, float* a_out,
                                   float* mse_out, char* err, int errlen) {
    return adapter_encode_base_on(pre_h, X, n, beam, icm, ils, perturb, use_abs, seed, device, 0, B_out, a_out,
                                  mse_out, err, errlen);
}

extern "C" int adapter_encode_base_on(void* pre_h, const float* X, int n, int beam, int icm, int ils, int perturb,
                                      int use_abs, int seed, int device, int n_devices, std::uint8_t* B_out,
                                      float* a_out, float* mse_out, char* err, int errlen) {
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
    std::vector<int> devices;
    for (int i = 0; i < n_devices; ++i) devices.push_back(i);
    const bool ok = n_devices > 0
                        ? stlq::b200::EncodeBaseSharded(cfg, ds, books, *pre, devices, &base, &bm, &fm, &e)
                        : stlq::b200::EncodeBase(cfg, ds, books, *pre, nullptr, &base, &bm, &fm, &e);
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

// ---- Kernel provider: stlq::b200::B200StreamKernels next to the reference's CpuStreamKernels ----
#include "stlq/core/kernel_provider_cpu.h"
#include "stlq_b200_kernels.h"

namespace {

template <typename T>
stlq::ColMajorMatrix<T> MatOf(const T* p, int rows, int cols) {
    stlq::ColMajorMatrix<T> m(rows, cols);
    if (p && rows > 0 && cols > 0) std::memcpy(m.data.data(), p, sizeof(T) * static_cast<size_t>(rows) * cols);
    return m;
}

void CopyErr(const std::exception& e, char* err, int errlen) {
    std::strncpy(err, e.what(), static_cast<size_t>(errlen) - 1);
    err[errlen - 1] = 0;
}

}  // namespace

extern "C" void* prov_create(int device, char* err, int errlen) {
    try {
        return new stlq::b200::B200StreamKernels(device);
    } catch (const std::exception& e) {
        CopyErr(e, err, errlen);
        return nullptr;
    }
}

extern "C" void prov_destroy(void* p) { delete static_cast<stlq::b200::B200StreamKernels*>(p); }

// C (cr x cc, in/out) through one of the provider's GEMM entries (B200 when p is non-null, else the
// reference's CpuStreamKernels::Gemm): 0 Gemm, 1 GemmDevice, 2 GemmDeviceHostPtrB,
// 3 EnsureDeviceF32(B) then GemmDeviceDevicePtrB; 1-3 read the result back with DownloadF32.
extern "C" int prov_gemm(void* p, int which, int ta, int tb, float alpha, const float* A, int ar, int ac,
                         const float* B, int br, int bc, float beta, float* C, int cr, int cc, char* err, int errlen) {
    try {
        const auto Am = MatOf(A, ar, ac), Bm = MatOf(B, br, bc);
        auto Cm = MatOf(C, cr, cc);
        if (!p) {
            stlq::CpuStreamKernels cpu;
            cpu.Gemm(ta != 0, tb != 0, alpha, Am, Bm, beta, &Cm);
        } else {
            auto* k = static_cast<stlq::b200::B200StreamKernels*>(p);
            stlq::DeviceMatF32View v;
            if (which == 0) {
                k->Gemm(ta != 0, tb != 0, alpha, Am, Bm, beta, &Cm);
            } else {
                if (which == 1) {
                    k->GemmDevice(ta != 0, tb != 0, alpha, Am, Bm, beta, &v);
                } else if (which == 2) {
                    k->GemmDeviceHostPtrB(ta != 0, tb != 0, alpha, Am, Bm.data.data(), br, br, bc, beta, &v);
                } else {
                    stlq::DeviceMatF32View dB;
                    if (!k->EnsureDeviceF32(Bm, &dB)) throw std::runtime_error("EnsureDeviceF32 failed");
                    k->GemmDeviceDevicePtrB(ta != 0, tb != 0, alpha, Am, dB.ptr, dB.ld, br, bc, beta, &v);
                }
                k->DownloadF32(v, &Cm);
            }
        }
        if (Cm.rows != cr || Cm.cols != cc) throw std::runtime_error("result shape differs");
        std::memcpy(C, Cm.data.data(), sizeof(float) * static_cast<size_t>(cr) * cc);
        return 0;
    } catch (const std::exception& e) {
        CopyErr(e, err, errlen);
        return 1;
    }
}

// ConvertU8ToF32 (mode 0), ConvertU8ToF32AndRotate (1) or ConvertU8ToF32AndRotatePtr (2, `in` with
// leading dimension ld_in) on the B200 provider (p non-null) or the CPU one.  out: (R rows or
// rows) x cols.  cached: TryGetCachedDeviceF32 of the result, then 1 if a GemmDevice of
// C_small^T with it equals Gemm on the host copy (-1 when not asked: C_small null).
extern "C" int prov_convert(void* p, int mode, const std::uint8_t* in, int ld_in, int rows, int cols, const float* R,
                            int rr, int rc, float* out, const float* C_small, int hs, int* cached, char* err,
                            int errlen) {
    try {
        std::unique_ptr<stlq::StreamKernelProvider> own;
        stlq::StreamKernelProvider* k = static_cast<stlq::b200::B200StreamKernels*>(p);
        if (!k) {
            own = std::make_unique<stlq::CpuStreamKernels>();
            k = own.get();
        }
        const auto Rm = MatOf(R, rr, rc);
        stlq::ColMajorMatrix<float> X;
        if (mode == 0 || mode == 1) {
            stlq::ColMajorMatrix<std::uint8_t> U(rows, cols);
            for (int j = 0; j < cols; ++j)
                std::memcpy(U.Col(j), in + static_cast<size_t>(j) * ld_in, static_cast<size_t>(rows));
            if (mode == 0) k->ConvertU8ToF32(U, &X);
            else k->ConvertU8ToF32AndRotate(U, Rm, &X);
        } else {
            k->ConvertU8ToF32AndRotatePtr(in, ld_in, rows, cols, Rm, &X);
        }
        std::memcpy(out, X.data.data(), sizeof(float) * X.data.size());
        if (cached) {
            stlq::DeviceMatF32View v;
            cached[0] = k->TryGetCachedDeviceF32(X, &v) ? 1 : 0;
            cached[1] = -1;
            if (C_small && hs > 0) {
                const auto Cs = MatOf(C_small, X.rows, hs);
                stlq::ColMajorMatrix<float> host_xc(hs, X.cols), dev_xc;
                k->Gemm(true, false, 1.0f, Cs, X, 0.0f, &host_xc);
                stlq::DeviceMatF32View xv;
                k->GemmDevice(true, false, 1.0f, Cs, X, 0.0f, &xv);
                k->DownloadF32(xv, &dev_xc);
                cached[1] = dev_xc.data == host_xc.data ? 1 : 0;
            }
        }
        return 0;
    } catch (const std::exception& e) {
        CopyErr(e, err, errlen);
        return 1;
    }
}

// ArgmaxColsF32 of a host score matrix (rows x cols) uploaded with EnsureDeviceF32.
extern "C" int prov_argmax(void* p, const float* S, int rows, int cols, int* idx, float* val, char* err, int errlen) {
    try {
        auto* k = static_cast<stlq::b200::B200StreamKernels*>(p);
        const auto Sm = MatOf(S, rows, cols);
        stlq::DeviceMatF32View v;
        if (!k->EnsureDeviceF32(Sm, &v)) throw std::runtime_error("EnsureDeviceF32 failed");
        std::vector<int> a;
        std::vector<float> b;
        k->ArgmaxColsF32(v, &a, &b);
        std::memcpy(idx, a.data(), sizeof(int) * a.size());
        std::memcpy(val, b.data(), sizeof(float) * b.size());
        return 0;
    } catch (const std::exception& e) {
        CopyErr(e, err, errlen);
        return 1;
    }
}
