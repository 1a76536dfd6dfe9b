// B200StreamKernels: StreamKernelProvider on the stlq_b200 kernel-provider C-ABI (see the header).
#include "stlq_b200_kernels.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

#include <cuda_runtime.h>

#include "stlq_b200.h"

namespace stlq {
namespace b200 {

namespace {

[[noreturn]] void ThrowAbi(const char* what) {
    throw std::runtime_error(std::string("B200StreamKernels::") + what + ": " + stlq_b200_last_error());
}

void CheckAbi(int rc, const char* what) {
    if (rc != 0) ThrowAbi(what);
}

void CheckCuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("B200StreamKernels::") + what + ": " + cudaGetErrorString(e));
}

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    void Ensure(size_t need) {
        if (need <= bytes) return;
        Release();
        CheckCuda(cudaMalloc(&p, std::max<size_t>(need, 16)), "cudaMalloc");
        bytes = need;
    }
    void Release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

// Identity of a host matrix whose contents are on the device: pointer, shape and a content stamp
// over 256 evenly spaced elements.
struct HostKey {
    const void* ptr = nullptr;
    int rows = 0, cols = 0;
    std::uint64_t stamp = 0;
    bool valid = false;
};

std::uint64_t Stamp(const ColMajorMatrix<float>& h) {
    std::uint64_t x = 0xcbf29ce484222325ull;
    auto mix = [&](std::uint64_t v) {
        x ^= v;
        x *= 0x100000001b3ull;
    };
    mix(static_cast<std::uint64_t>(h.rows));
    mix(static_cast<std::uint64_t>(h.cols));
    const size_t n = h.data.size();
    mix(n);
    if (n == 0) return x;
    const size_t samples = std::min<size_t>(256, n);
    for (size_t i = 0; i < samples; ++i) {
        const size_t idx = (n - 1) * i / std::max<size_t>(samples - 1, 1);
        std::uint32_t bits = 0;
        std::memcpy(&bits, &h.data[idx], sizeof(bits));
        mix(bits);
    }
    return x;
}

HostKey KeyOf(const ColMajorMatrix<float>& h) {
    return HostKey{h.data.data(), h.rows, h.cols, Stamp(h), true};
}

bool Same(const HostKey& k, const ColMajorMatrix<float>& h) {
    return k.valid && k.ptr == h.data.data() && k.rows == h.rows && k.cols == h.cols && !h.data.empty() &&
           k.stamp == Stamp(h);
}

void ClearView(DeviceMatF32View* v) {
    if (v) *v = DeviceMatF32View{};
}

struct GemmShape {
    int m, n, k;
};

GemmShape ShapeOf(bool transA, bool transB, int a_rows, int a_cols, int b_rows, int b_cols, const char* who) {
    const int m = transA ? a_cols : a_rows;
    const int k = transA ? a_rows : a_cols;
    const int kb = transB ? b_cols : b_rows;
    const int n = transB ? b_rows : b_cols;
    if (k != kb) throw std::runtime_error(std::string("B200StreamKernels::") + who + ": inner dimensions differ");
    return {m, n, k};
}

}  // namespace

struct B200StreamKernels::Impl {
    int device = 0;
    cudaStream_t stream = nullptr;
    stlq_b200_kernels* k = nullptr;
    DevBuf u8, tmp;            // uploaded uint8 tile, its float conversion before rotation
    DevBuf xtile;              // the last tile ConvertU8ToF32* produced (equal to the host output)
    HostKey xkey;
    DevBuf A;                  // the last A operand (codebooks, rotations): reused while unchanged
    HostKey akey;
    DevBuf R;                  // the rotation of ConvertU8ToF32AndRotate*
    HostKey rkey;
    DevBuf B, C;               // per-call operand and result scratch of Gemm
    DevBuf pub;                // GemmDevice* results
    DevBuf ens;                // EnsureDeviceF32's copy
    HostKey ekey;
    DevBuf aidx, aval;         // argmax results

    struct Scope {
        int prev = -1;
        explicit Scope(int dev) {
            if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
            CheckCuda(cudaSetDevice(dev), "cudaSetDevice");
        }
        ~Scope() {
            if (prev >= 0) cudaSetDevice(prev);
        }
    };

    void Upload(DevBuf& buf, HostKey& key, const ColMajorMatrix<float>& h) {
        if (Same(key, h)) return;
        buf.Ensure(sizeof(float) * h.data.size());
        CheckCuda(cudaMemcpyAsync(buf.p, h.data.data(), sizeof(float) * h.data.size(), cudaMemcpyHostToDevice, stream),
                  "upload");
        key = KeyOf(h);
    }

    // Device pointer of a B operand: the tile or EnsureDeviceF32 copy already on the device, else
    // uploaded to the per-call scratch.
    const float* DeviceB(const ColMajorMatrix<float>& h) {
        if (Same(xkey, h)) return xtile.as<const float>();
        if (Same(ekey, h)) return ens.as<const float>();
        B.Ensure(sizeof(float) * h.data.size());
        CheckCuda(cudaMemcpyAsync(B.p, h.data.data(), sizeof(float) * h.data.size(), cudaMemcpyHostToDevice, stream),
                  "upload B");
        return B.as<const float>();
    }

    void Download(float* host, const float* dev, size_t count) {
        CheckCuda(cudaMemcpyAsync(host, dev, sizeof(float) * count, cudaMemcpyDeviceToHost, stream), "download");
        CheckCuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    }

    // in: `cols` columns of `rows` bytes at stride ld_in (host) -> xtile = R * float(in) (or float(in)).
    void ConvertTile(const std::uint8_t* in, int ld_in, int rows, int cols, const ColMajorMatrix<float>* Rm,
                     ColMajorMatrix<float>* out) {
        const size_t span = static_cast<size_t>(ld_in) * (cols - 1) + rows;
        u8.Ensure(span);
        CheckCuda(cudaMemcpyAsync(u8.p, in, span, cudaMemcpyHostToDevice, stream), "upload u8 tile");
        const int out_rows = Rm ? Rm->rows : rows;
        xtile.Ensure(sizeof(float) * static_cast<size_t>(out_rows) * cols);
        if (Rm) {
            tmp.Ensure(sizeof(float) * static_cast<size_t>(rows) * cols);
            CheckAbi(stlq_b200_u8_to_f32(k, u8.as<std::uint8_t>(), ld_in, rows, cols, tmp.as<float>(), stream),
                     "ConvertU8ToF32AndRotate");
            Upload(R, rkey, *Rm);
            CheckAbi(stlq_b200_sgemm(k, 0, 0, Rm->rows, cols, rows, 1.0f, R.as<float>(), Rm->rows, tmp.as<float>(),
                                     rows, 0.0f, xtile.as<float>(), Rm->rows, stream),
                     "ConvertU8ToF32AndRotate");
        } else {
            CheckAbi(stlq_b200_u8_to_f32(k, u8.as<std::uint8_t>(), ld_in, rows, cols, xtile.as<float>(), stream),
                     "ConvertU8ToF32");
        }
        out->rows = out_rows;
        out->cols = cols;
        out->data.resize(static_cast<size_t>(out_rows) * cols);
        Download(out->data.data(), xtile.as<float>(), out->data.size());
        xkey = KeyOf(*out);
    }

    // op(A) (cached) times a device B into `dst` (m x n, ld m), C = alpha op(A) op(B) + beta * dst.
    void GemmInto(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& Am, const float* dB, int ldb,
                  const GemmShape& g, float beta, float* dst) {
        Upload(A, akey, Am);
        CheckAbi(stlq_b200_sgemm(k, transA, transB, g.m, g.n, g.k, alpha, A.as<float>(), std::max(1, Am.rows), dB,
                                 std::max(1, ldb), beta, dst, std::max(1, g.m), stream),
                 "Gemm");
    }

    // A GemmDevice* result published in `pub` (C starts at 0: the device variants have no input C).
    void Publish(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& Am, const float* dB, int ldb,
                 const GemmShape& g, float beta, DeviceMatF32View* out) {
        pub.Ensure(sizeof(float) * static_cast<size_t>(g.m) * g.n);
        if (beta != 0.0f)
            CheckCuda(cudaMemsetAsync(pub.p, 0, sizeof(float) * static_cast<size_t>(g.m) * g.n, stream), "memset");
        GemmInto(transA, transB, alpha, Am, dB, ldb, g, beta, pub.as<float>());
        // A view may be read on any stream: it is complete when returned.
        CheckCuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        out->ptr = pub.as<const float>();
        out->rows = g.m;
        out->cols = g.n;
        out->ld = g.m;
    }
};

B200StreamKernels::B200StreamKernels(int device) : impl_(new Impl()) {
    impl_->device = device;
    Impl::Scope scope(device);
    CheckAbi(stlq_b200_kernels_create(device, &impl_->k), "stlq_b200_kernels_create");
    CheckCuda(cudaStreamCreateWithFlags(&impl_->stream, cudaStreamNonBlocking), "cudaStreamCreate");
}

B200StreamKernels::~B200StreamKernels() {
    if (!impl_) return;
    {
        int prev = -1;
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(impl_->device);
        if (impl_->stream) cudaStreamSynchronize(impl_->stream);
        for (DevBuf* b : {&impl_->u8, &impl_->tmp, &impl_->xtile, &impl_->A, &impl_->R, &impl_->B, &impl_->C,
                          &impl_->pub, &impl_->ens, &impl_->aidx, &impl_->aval})
            b->Release();
        if (impl_->stream) cudaStreamDestroy(impl_->stream);
        stlq_b200_kernels_destroy(impl_->k);
        if (prev >= 0) cudaSetDevice(prev);
    }
    delete impl_;
}

void B200StreamKernels::ResetState() {
    Impl::Scope scope(impl_->device);
    CheckCuda(cudaStreamSynchronize(impl_->stream), "cudaStreamSynchronize");
    for (DevBuf* b : {&impl_->u8, &impl_->tmp, &impl_->xtile, &impl_->A, &impl_->R, &impl_->B, &impl_->C, &impl_->pub,
                      &impl_->ens, &impl_->aidx, &impl_->aval})
        b->Release();
    impl_->xkey = impl_->akey = impl_->rkey = impl_->ekey = HostKey{};
}

void B200StreamKernels::ConvertU8ToF32(const ColMajorMatrix<std::uint8_t>& in, ColMajorMatrix<float>* out) {
    if (!out) throw std::runtime_error("B200StreamKernels::ConvertU8ToF32: output is null");
    if (in.rows <= 0 || in.cols <= 0) {
        out->rows = in.rows > 0 ? in.rows : 0;
        out->cols = 0;
        out->data.clear();
        return;
    }
    Impl::Scope scope(impl_->device);
    impl_->ConvertTile(in.data.data(), in.rows, in.rows, in.cols, nullptr, out);
}

void B200StreamKernels::ConvertU8ToF32AndRotate(const ColMajorMatrix<std::uint8_t>& in, const ColMajorMatrix<float>& R,
                                                ColMajorMatrix<float>* out) {
    if (!out) throw std::runtime_error("B200StreamKernels::ConvertU8ToF32AndRotate: output is null");
    if (R.cols != in.rows) throw std::runtime_error("B200StreamKernels::ConvertU8ToF32AndRotate: R.cols != rows");
    if (in.rows <= 0 || in.cols <= 0) {
        out->rows = R.rows;
        out->cols = 0;
        out->data.clear();
        return;
    }
    Impl::Scope scope(impl_->device);
    impl_->ConvertTile(in.data.data(), in.rows, in.rows, in.cols, &R, out);
}

void B200StreamKernels::ConvertU8ToF32AndRotatePtr(const std::uint8_t* in, int ld_in, int rows, int cols,
                                                   const ColMajorMatrix<float>& R, ColMajorMatrix<float>* out) {
    if (!out) return;
    if (!in || rows <= 0 || cols <= 0) {
        out->rows = 0;
        out->cols = 0;
        out->data.clear();
        return;
    }
    if (R.cols != rows)
        throw std::runtime_error("B200StreamKernels::ConvertU8ToF32AndRotatePtr: dim mismatch (R.cols != rows).");
    if (ld_in < rows) throw std::runtime_error("B200StreamKernels::ConvertU8ToF32AndRotatePtr: ld_in < rows");
    Impl::Scope scope(impl_->device);
    impl_->ConvertTile(in, ld_in, rows, cols, &R, out);
}

void B200StreamKernels::Gemm(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A,
                             const ColMajorMatrix<float>& B, float beta, ColMajorMatrix<float>* C) {
    if (!C) throw std::runtime_error("B200StreamKernels::Gemm: output is null");
    const GemmShape g = ShapeOf(transA, transB, A.rows, A.cols, B.rows, B.cols, "Gemm");
    const size_t mn = static_cast<size_t>(std::max(g.m, 0)) * std::max(g.n, 0);
    if (C->rows != g.m || C->cols != g.n || C->data.size() < mn) {
        if (beta != 0.0f) throw std::runtime_error("B200StreamKernels::Gemm: C must be m x n when beta != 0");
        C->rows = g.m;
        C->cols = g.n;
        C->data.resize(mn);
    }
    if (mn == 0) return;
    Impl::Scope scope(impl_->device);
    Impl& I = *impl_;
    const float* dB = g.k > 0 ? I.DeviceB(B) : nullptr;
    I.C.Ensure(sizeof(float) * mn);
    if (beta != 0.0f)
        CheckCuda(cudaMemcpyAsync(I.C.p, C->data.data(), sizeof(float) * mn, cudaMemcpyHostToDevice, I.stream),
                  "upload C");
    if (g.k > 0) {
        I.GemmInto(transA, transB, alpha, A, dB, B.rows, g, beta, I.C.as<float>());
    } else {
        CheckAbi(stlq_b200_sgemm(I.k, transA, transB, g.m, g.n, 0, alpha, nullptr, std::max(1, A.rows), nullptr,
                                 std::max(1, B.rows), beta, I.C.as<float>(), std::max(1, g.m), I.stream),
                 "Gemm");
    }
    I.Download(C->data.data(), I.C.as<float>(), mn);
}

void B200StreamKernels::GemmDevice(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A,
                                   const ColMajorMatrix<float>& B, float beta, DeviceMatF32View* out) {
    if (!out) throw std::runtime_error("B200StreamKernels::GemmDevice: output view is null");
    ClearView(out);
    const GemmShape g = ShapeOf(transA, transB, A.rows, A.cols, B.rows, B.cols, "GemmDevice");
    if (g.m <= 0 || g.n <= 0 || g.k <= 0) return;
    Impl::Scope scope(impl_->device);
    impl_->Publish(transA, transB, alpha, A, impl_->DeviceB(B), B.rows, g, beta, out);
}

void B200StreamKernels::GemmDeviceHostPtrB(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A,
                                           const float* B, int ldB, int rowsB, int colsB, float beta,
                                           DeviceMatF32View* out) {
    ClearView(out);
    if (!out || !B || rowsB <= 0 || colsB <= 0 || ldB < rowsB) return;
    const GemmShape g = ShapeOf(transA, transB, A.rows, A.cols, rowsB, colsB, "GemmDeviceHostPtrB");
    if (g.m <= 0 || g.n <= 0 || g.k <= 0) return;
    Impl::Scope scope(impl_->device);
    Impl& I = *impl_;
    const size_t span = static_cast<size_t>(ldB) * (colsB - 1) + rowsB;
    I.B.Ensure(sizeof(float) * span);
    CheckCuda(cudaMemcpyAsync(I.B.p, B, sizeof(float) * span, cudaMemcpyHostToDevice, I.stream), "upload B");
    I.Publish(transA, transB, alpha, A, I.B.as<const float>(), ldB, g, beta, out);
}

bool B200StreamKernels::EnsureDeviceF32(const ColMajorMatrix<float>& host, DeviceMatF32View* out) {
    ClearView(out);
    if (host.rows <= 0 || host.cols <= 0 || host.data.empty()) return false;
    try {
        Impl::Scope scope(impl_->device);
        impl_->Upload(impl_->ens, impl_->ekey, host);
        CheckCuda(cudaStreamSynchronize(impl_->stream), "cudaStreamSynchronize");
    } catch (const std::exception&) {
        return false;  // no persistent copy (out of memory): the caller tiles its uploads instead
    }
    if (out) {
        out->ptr = impl_->ens.as<const float>();
        out->rows = host.rows;
        out->cols = host.cols;
        out->ld = host.rows;
    }
    return true;
}

void B200StreamKernels::GemmDeviceDevicePtrB(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A,
                                             const float* dB, int ldB, int rowsB, int colsB, float beta,
                                             DeviceMatF32View* out) {
    if (!out) throw std::runtime_error("B200StreamKernels::GemmDeviceDevicePtrB: output view is null.");
    ClearView(out);
    if (A.rows <= 0 || A.cols <= 0 || !dB || rowsB <= 0 || colsB <= 0) return;
    if (ldB < rowsB) throw std::runtime_error("B200StreamKernels::GemmDeviceDevicePtrB: invalid ldB.");
    const GemmShape g = ShapeOf(transA, transB, A.rows, A.cols, rowsB, colsB, "GemmDeviceDevicePtrB");
    Impl::Scope scope(impl_->device);
    impl_->Publish(transA, transB, alpha, A, dB, ldB, g, beta, out);
}

void B200StreamKernels::DownloadF32(const DeviceMatF32View& view, ColMajorMatrix<float>* out) {
    if (!out) throw std::runtime_error("B200StreamKernels::DownloadF32: output is null.");
    if (!view.ptr || view.rows <= 0 || view.cols <= 0 || view.ld < view.rows) {
        out->rows = 0;
        out->cols = 0;
        out->data.clear();
        return;
    }
    Impl::Scope scope(impl_->device);
    out->rows = view.rows;
    out->cols = view.cols;
    out->data.resize(static_cast<size_t>(view.rows) * view.cols);
    CheckCuda(cudaMemcpy2DAsync(out->data.data(), sizeof(float) * view.rows, view.ptr, sizeof(float) * view.ld,
                                sizeof(float) * view.rows, view.cols, cudaMemcpyDeviceToHost, impl_->stream),
              "DownloadF32");
    CheckCuda(cudaStreamSynchronize(impl_->stream), "cudaStreamSynchronize (DownloadF32)");
}

bool B200StreamKernels::TryGetCachedDeviceF32(const ColMajorMatrix<float>& host, DeviceMatF32View* out) {
    ClearView(out);
    const float* p = nullptr;
    if (Same(impl_->xkey, host)) p = impl_->xtile.as<const float>();
    else if (Same(impl_->ekey, host)) p = impl_->ens.as<const float>();
    if (!p) return false;
    if (out) {
        out->ptr = p;
        out->rows = host.rows;
        out->cols = host.cols;
        out->ld = host.rows;
    }
    return true;
}

void B200StreamKernels::ArgmaxColsF32(const DeviceMatF32View& scores, std::vector<int>* assignments,
                                      std::vector<float>* best_values) {
    if (!assignments || !best_values)
        throw std::runtime_error("B200StreamKernels::ArgmaxColsF32: output vectors must be non-null.");
    DeviceVecI32View di;
    DeviceVecF32View dv;
    ArgmaxColsF32Device(scores, &di, &dv);
    const int cols = std::max(scores.cols, 0);
    assignments->resize(cols);
    best_values->resize(cols);
    if (cols == 0 || !di.ptr) return;
    Impl::Scope scope(impl_->device);
    CheckCuda(cudaMemcpyAsync(assignments->data(), di.ptr, sizeof(int) * cols, cudaMemcpyDeviceToHost, impl_->stream),
              "ArgmaxColsF32");
    CheckCuda(cudaMemcpyAsync(best_values->data(), dv.ptr, sizeof(float) * cols, cudaMemcpyDeviceToHost,
                              impl_->stream),
              "ArgmaxColsF32");
    CheckCuda(cudaStreamSynchronize(impl_->stream), "cudaStreamSynchronize (ArgmaxColsF32)");
}

void B200StreamKernels::ArgmaxColsF32Device(const DeviceMatF32View& scores, DeviceVecI32View* d_assign,
                                            DeviceVecF32View* d_best) {
    if (d_assign) *d_assign = DeviceVecI32View{};
    if (d_best) *d_best = DeviceVecF32View{};
    if (scores.cols <= 0) return;
    if (!scores.ptr || scores.ld < std::max(scores.rows, 1))
        throw std::runtime_error("B200StreamKernels::ArgmaxColsF32Device: invalid scores view");
    Impl::Scope scope(impl_->device);
    Impl& I = *impl_;
    I.aidx.Ensure(sizeof(int) * scores.cols);
    I.aval.Ensure(sizeof(float) * scores.cols);
    CheckAbi(stlq_b200_argmax_cols(I.k, scores.ptr, scores.ld, scores.rows, scores.cols, I.aidx.as<int>(),
                                   I.aval.as<float>(), I.stream),
             "ArgmaxColsF32Device");
    CheckCuda(cudaStreamSynchronize(I.stream), "cudaStreamSynchronize (ArgmaxColsF32Device)");
    if (d_assign) {
        d_assign->ptr = I.aidx.as<const int>();
        d_assign->n = scores.cols;
    }
    if (d_best) {
        d_best->ptr = I.aval.as<const float>();
        d_best->n = scores.cols;
    }
}

void B200StreamKernels::Sync() {
    Impl::Scope scope(impl_->device);
    CheckCuda(cudaStreamSynchronize(impl_->stream), "Sync");
}

void B200StreamKernels::SyncCompute() { Sync(); }

}  // namespace b200
}  // namespace stlq
