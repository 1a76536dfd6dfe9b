// Test infrastructure only: an extern "C" driver around the REFERENCE's own CUDA ICM
// (src/quantizer/icm_cuda.cu, DynamicIcmWithIls{Abs,NoAbs}NoNormalCuda, compiled for sm_100a from its
// sources by oracle/Makefile), the GPU kernel the reference runs for this stage.  Used to compare
// the B200 refinement kernel with it on the same inputs; never part of the product.
#include <cstdint>
#include <cstring>
#include <vector>

#include "stlq/common/types.h"
#include "stlq/quantizer/icm_cuda.h"

extern "C" {

// X: d x n, xC: H x n (column-major, host), B_io: m x n codes in (beam) and out.  timing_out (7
// doubles, seconds, device-timed by the reference): uploads of xC/norms, upload of B, initial ICM,
// ILS copy+perturb, ILS ICM, ILS accept, downloads.  Returns 0 on success.
int ref_icm_cuda(void* pre_h, const float* X, int n, const float* xC, int icm_iters, int ils_iters, int perturb_k,
                 int use_abs, std::uint32_t seed, std::uint64_t sample_id_offset, std::uint8_t* B_io, float* a_out,
                 float* cost_out, double* timing_out) {
    const auto* pre = static_cast<const stlq::Precomp*>(pre_h);
    if (!pre || n <= 0) return 1;
    stlq::ColMajorMatrix<float> Xm(pre->d, n), xCm(pre->H, n);
    std::memcpy(Xm.data.data(), X, sizeof(float) * Xm.data.size());
    std::memcpy(xCm.data.data(), xC, sizeof(float) * xCm.data.size());
    stlq::ColMajorMatrix<stlq::FullCode> B(pre->m, n);
    std::memcpy(B.data.data(), B_io, B.data.size());
    stlq::ColMajorMatrix<float> a;
    std::vector<float> xn, cost;
    stlq::CudaIcmTiming t;
    if (use_abs)
        stlq::DynamicIcmWithIlsAbsNoNormalCuda(Xm, *pre, xCm, icm_iters, ils_iters, perturb_k, seed, &B, &a, &xn, &cost,
                                               false, sample_id_offset, &t);
    else
        stlq::DynamicIcmWithIlsNoAbsNoNormalCuda(Xm, *pre, xCm, icm_iters, ils_iters, perturb_k, seed, &B, &a, &xn,
                                                 &cost, false, sample_id_offset, &t);
    std::memcpy(B_io, B.data.data(), B.data.size());
    if (a_out && a.data.size() == static_cast<size_t>(pre->m) * n) std::memcpy(a_out, a.data.data(), sizeof(float) * a.data.size());
    if (cost_out && cost.size() == static_cast<size_t>(n)) std::memcpy(cost_out, cost.data(), sizeof(float) * n);
    if (timing_out) {
        const double v[7] = {t.upload_fixed, t.upload_B, t.icm_init, t.ils_copy_perturb, t.ils_icm, t.ils_accept,
                             t.download};
        std::memcpy(timing_out, v, sizeof(v));
    }
    return 0;
}

}  // extern "C"
