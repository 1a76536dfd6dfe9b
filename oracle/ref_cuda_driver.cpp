// Test infrastructure only: an extern "C" driver around the REFERENCE's own CUDA code paths,
// compiled for sm_100a from its sources by oracle/Makefile: the CUDA ICM
// (src/quantizer/icm_cuda.cu, DynamicIcmWithIls{Abs,NoAbs}NoNormalCuda) and the large-root CUDA
// beam search (src/quantizer/beam_search_cuda.cu, BeamSearchPrefixLSLargeRootCudaH2/H4), the GPU
// kernels the reference runs for these stages.  Used to compare the B200 kernels with them on the
// same inputs; never part of the product.
#include <cstdint>
#include <cstring>
#include <vector>

#include "stlq/common/types.h"
#include "stlq/quantizer/beam_search.h"
#include "stlq/quantizer/icm_cuda.h"
#include "stlq/quantizer/precomp_large_root.h"

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

// Large-root beam search on the reference's CUDA path for H_beam 2 or 4: BuildPrecompLargeRoot
// and ComputeXcSmall on the host (as the reference's large pipeline does before the call), then
// BeamSearchPrefixLSLargeRootCudaH2/H4.  C_all: d x H column-major, root codewords first; X: d x n.
// Outputs: cluster (n), B_small ((m-1) x n); timing_out (4 doubles, seconds, the reference's own
// BeamSearchLargeRootTiming): norms, root GEMM, root top-H update, expansion of layers 1..m-1.
// Returns 0 on success.
int ref_beam_large_root_cuda(int d, int m, const int* h_vec, const float* C_all, const float* X, int n, int beam,
                             int allow_tf32, std::uint32_t* cluster_out, std::uint8_t* B_small_out,
                             double* timing_out) {
    if (n <= 0 || d <= 0 || m <= 1 || (beam != 2 && beam != 4)) return 1;
    stlq::CodebookPack pack;
    pack.d = d;
    int off = 0;
    for (int l = 0; l < m; ++l) {
        pack.h_vec.push_back(h_vec[l]);
        stlq::ColMajorMatrix<float> book(d, h_vec[l]);
        std::memcpy(book.data.data(), C_all + static_cast<std::size_t>(off) * d, sizeof(float) * d * h_vec[l]);
        pack.books.push_back(std::move(book));
        off += h_vec[l];
    }
    stlq::PrecompLargeRoot pre;
    stlq::PrecompLargeRootBuildOptions opts;
    std::string err;
    if (!stlq::BuildPrecompLargeRoot(pack, nullptr, opts, &pre, &err)) return 2;
    stlq::ColMajorMatrix<float> Xm(d, n);
    std::memcpy(Xm.data.data(), X, sizeof(float) * Xm.data.size());
    stlq::ColMajorMatrix<float> xC_small;
    stlq::ComputeXcSmall(pre, Xm, nullptr, &xC_small);
    std::vector<std::uint32_t> cluster;
    stlq::ColMajorMatrix<stlq::Code> B_small;
    stlq::BeamSearchLargeRootTiming t;
    if (beam == 2)
        stlq::BeamSearchPrefixLSLargeRootCudaH2(Xm, pre, xC_small, allow_tf32 != 0, &cluster, &B_small, &t);
    else
        stlq::BeamSearchPrefixLSLargeRootCudaH4(Xm, pre, xC_small, allow_tf32 != 0, &cluster, &B_small, &t);
    if (cluster.size() != static_cast<std::size_t>(n)) return 3;
    std::memcpy(cluster_out, cluster.data(), sizeof(std::uint32_t) * n);
    std::memcpy(B_small_out, B_small.data.data(), B_small.data.size());
    if (timing_out) {
        timing_out[0] = t.norm_x2;
        timing_out[1] = t.root_gemm;
        timing_out[2] = t.root_update;
        timing_out[3] = t.expand;
    }
    return 0;
}

}  // extern "C"
