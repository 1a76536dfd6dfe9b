// B200 implementation of the reference's GPU backend seam, StreamKernelProvider
// (include/stlq/core/kernel_provider.h:28-221), on the stlq_b200 kernel-provider C-ABI
// (stlq_b200_sgemm, stlq_b200_u8_to_f32, stlq_b200_argmax_cols).
//
// It replaces CudaStreamKernels (include/stlq/core/kernel_provider_cuda_stream.h:18, cuBLAS) where
// PrepareKernelRuntimeStage selects the provider (src/pipeline/stlq_entry_stages.cpp:59-76).
// Differences from the reference's CUDA provider, all in its favour:
//  * every GEMM (Gemm, GemmDevice*, the rotation of ConvertU8ToF32AndRotate*) is bit-identical to
//    the reference's CPU provider (CpuStreamKernels: OpenBLAS 0.3.15 sgemm with one BLAS thread;
//    with several threads OpenBLAS splits K differently when K is in (448, 896) and not one of the
//    sizes where both rules agree, such as 512, 768, 896), instead of cuBLAS's order;
//  * DownloadF32 honours the view's leading dimension.
// Device views it returns stay valid until the next call that rewrites the same buffer: the
// rotated X tile (ConvertU8ToF32*), EnsureDeviceF32's copy, the GemmDevice* output and the argmax
// results each have their own buffer.  Host matrices are recognised as already on the device by
// pointer, shape and a 256-sample content stamp (the reference samples 32).  Errors throw
// std::runtime_error, as the reference's CUDA provider does.
#pragma once

#include <cstdint>
#include <vector>

#include "stlq/core/kernel_provider.h"

namespace stlq {
namespace b200 {

class B200StreamKernels final : public StreamKernelProvider {
public:
    explicit B200StreamKernels(int device = 0);
    ~B200StreamKernels() override;
    B200StreamKernels(const B200StreamKernels&) = delete;
    B200StreamKernels& operator=(const B200StreamKernels&) = delete;

    bool IsGpu() const override { return true; }

    void ConvertU8ToF32(const ColMajorMatrix<std::uint8_t>& in, ColMajorMatrix<float>* out) override;
    void ConvertU8ToF32AndRotate(const ColMajorMatrix<std::uint8_t>& in, const ColMajorMatrix<float>& R,
                                 ColMajorMatrix<float>* out) override;
    void ConvertU8ToF32AndRotatePtr(const std::uint8_t* in, int ld_in, int rows, int cols,
                                    const ColMajorMatrix<float>& R, ColMajorMatrix<float>* out) override;

    void Gemm(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A, const ColMajorMatrix<float>& B,
              float beta, ColMajorMatrix<float>* C) override;
    void GemmDevice(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A,
                    const ColMajorMatrix<float>& B, float beta, DeviceMatF32View* out) override;
    void GemmDeviceHostPtrB(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A, const float* B,
                            int ldB, int rowsB, int colsB, float beta, DeviceMatF32View* out) override;
    bool EnsureDeviceF32(const ColMajorMatrix<float>& host, DeviceMatF32View* out) override;
    void GemmDeviceDevicePtrB(bool transA, bool transB, float alpha, const ColMajorMatrix<float>& A, const float* dB,
                              int ldB, int rowsB, int colsB, float beta, DeviceMatF32View* out) override;
    void DownloadF32(const DeviceMatF32View& view, ColMajorMatrix<float>* out) override;
    bool TryGetCachedDeviceF32(const ColMajorMatrix<float>& host, DeviceMatF32View* out) override;
    void ArgmaxColsF32(const DeviceMatF32View& scores, std::vector<int>* assignments,
                       std::vector<float>* best_values) override;
    void ArgmaxColsF32Device(const DeviceMatF32View& scores, DeviceVecI32View* d_assign,
                             DeviceVecF32View* d_best) override;
    void Sync() override;
    void SyncCompute() override;

    // Frees every device buffer and cache (CudaStreamKernels::ResetCudaState); the provider stays
    // usable.
    void ResetState();

    struct Impl;

private:
    Impl* impl_;
};

}  // namespace b200
}  // namespace stlq
