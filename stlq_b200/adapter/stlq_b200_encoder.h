// Drop-in C++ adapter: the reference's encode-stage signatures on top of the stlq_b200 C-ABI.
//
// Compiled inside the reference tree (it includes the reference's headers), it gives a maintainer
// B200 replacements with the exact signatures EncodeBase calls:
//   stlq::b200::EncodeBase                     <- stlq::EncodeBase            (include/stlq/quantizer/encoder.h:66-74)
//   stlq::b200::BeamSearchPrefixLS             <- stlq::BeamSearchPrefixLS    (include/stlq/quantizer/beam_search.h:18-22)
//   stlq::b200::SolveLeastSquaresAll           <- stlq::SolveLeastSquaresAll  (include/stlq/quantizer/least_squares.h)
//   stlq::b200::DynamicIcmWithIls{Abs,NoAbs}NoNormalCuda
//                                              <- stlq::DynamicIcmWithIls*NoNormalCuda (include/stlq/quantizer/icm_cuda.h:31-68)
// Semantics: the same inputs, outputs and ownership as the reference (callers own the matrices;
// outputs are resized here).  Errors: EncodeBase returns false and fills *error; the others throw
// std::runtime_error, like the reference's CUDA helpers (icm_cuda_kernels.inc:10-15).
//
// One encoder handle per (host thread, device, Precomp::build_tag) is cached thread-locally, the
// way the reference caches its CUDA sessions by build_tag (icm_cuda_kernels.inc:2110-2118).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "stlq/common/config.h"
#include "stlq/common/types.h"
#include "stlq/quantizer/precomp_large_root.h"

namespace stlq {

class KernelProvider;

namespace b200 {

bool EncodeBase(const Config& config, const Dataset& dataset, const CodebookPack& codebooks, const Precomp& precomp,
                KernelProvider* kernels, BaseEncoding* base, float* out_beam_mse, float* out_final_mse,
                std::string* error);

// EncodeBase on several GPUs of this process (stlq_b200_encode_sharded): the base vectors split into
// contiguous shards, one per device, with the codebooks replicated by one NCCL broadcast and the MSE
// sums combined by one NCCL reduce.  Same inputs and outputs as EncodeBase, bit for bit; `devices`
// lists the GPUs (empty: config.runtime.cuda_device alone).  No counterpart in the reference, whose
// EncodeBase runs on one device.
bool EncodeBaseSharded(const Config& config, const Dataset& dataset, const CodebookPack& codebooks,
                       const Precomp& precomp, const std::vector<int>& devices, BaseEncoding* base,
                       float* out_beam_mse, float* out_final_mse, std::string* error);

void BeamSearchPrefixLS(const ColMajorMatrix<float>& X, const Precomp& precomp, const ColMajorMatrix<float>& xC,
                        int H_beam, ColMajorMatrix<FullCode>* B, int device = 0);

void SolveLeastSquaresAll(const Precomp& precomp, const ColMajorMatrix<float>& xC, const ColMajorMatrix<FullCode>& B,
                          ColMajorMatrix<float>* a, int device = 0);

void DynamicIcmWithIlsAbsNoNormalCuda(const ColMajorMatrix<float>& X, const Precomp& precomp,
                                      const ColMajorMatrix<float>& xC, int icm_iters, int ils_iters, int perturb_k,
                                      std::uint32_t seed, ColMajorMatrix<FullCode>* B, ColMajorMatrix<float>* a,
                                      std::vector<float>* X_norm2, std::vector<float>* cost,
                                      bool print_progress = true, std::uint64_t sample_id_offset = 0, int device = 0);

void DynamicIcmWithIlsNoAbsNoNormalCuda(const ColMajorMatrix<float>& X, const Precomp& precomp,
                                        const ColMajorMatrix<float>& xC, int icm_iters, int ils_iters, int perturb_k,
                                        std::uint32_t seed, ColMajorMatrix<FullCode>* B, ColMajorMatrix<float>* a,
                                        std::vector<float>* X_norm2, std::vector<float>* cost,
                                        bool print_progress = true, std::uint64_t sample_id_offset = 0,
                                        int device = 0);

// The large pipeline's basic encode of one block (encode_base_streaming.cpp:1040-1300, CPU
// branch): BeamSearchPrefixLSLargeRoot (beam_search.h:26-32) + SolveLeastSquaresAllLargeRoot +
// ComputeCostsLargeRoot + DynamicIcmWithIls{Abs,NoAbs}NoNormalLargeRoot, on the GPU from the block's
// vectors.  Outputs are resized as the reference resizes them; out_beam_mse / out_final_mse (may be
// null) are the means of the beam-stage and final costs (MeanMseFromCosts).  The root (h_vec[0])
// may hold up to STLQ_B200_MAX_ROOT (65,536) codewords; codebooks 1..m-1 up to 256.
// Throws std::runtime_error on failure.
void EncodeBaseLargeRoot(const PrecompLargeRoot& pre, const ColMajorMatrix<float>& Xblk, int H_beam, int icm_iters,
                         int ils_iters, int perturb_k, bool use_abs, std::uint32_t seed,
                         std::uint64_t sample_id_offset, std::vector<std::uint32_t>* cluster_id,
                         ColMajorMatrix<Code>* B_small, ColMajorMatrix<float>* a, std::vector<float>* cost,
                         float* out_beam_mse, float* out_final_mse, int device = 0);

// Drops this thread's cached encoder handles (e.g. before the device is reset).
void ReleaseThreadEncoders();

}  // namespace b200
}  // namespace stlq
