// Test infrastructure only.  Runs the reference's own pipeline (stlq::RunStlq, compiled from its
// sources by oracle/Makefile's `full` objects) with the B200 drop-in bound where INTEGRATION.md
// binds it: every call of stlq::EncodeBase (made by RunNonLargePipelineFlow,
// src/pipeline/stlq_non_large_pipeline_flow.cpp:73) reaches this wrapper through the linker's
// --wrap, which stands for the one-line `#if defined(STLQ_WITH_B200)` binding at the top of the
// reference's EncodeBase without editing its sources.
//
// STLQ_B200_DROPIN selects what the wrapper does:
//   unset   the reference's EncodeBase (the CPU encode), unchanged;
//   "b200"  stlq::b200::EncodeBase only (what a maintainer's build would run);
//   "both"  both on the same arguments; the B200 result is returned to the pipeline, and
//           STLQ_B200_DROPIN_REPORT (a file path) receives a comparison of the two (one JSON
//           line per call, appended).
// STLQ_B200_DROPIN_BOOKS (a file path), when set, receives the codebooks the pipeline passed in
// (the reference trainer's C_root): int32 m, int32 d, m x int32 h, then each book d x h float32.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "stlq/quantizer/encoder.h"
#include "stlq/stlq.h"
#include "stlq_b200_encoder.h"

#define STLQ_ENCODE_BASE_SYM _ZN4stlq10EncodeBaseERKNS_6ConfigERKNS_7DatasetERKNS_12CodebookPackERKNS_7PrecompEPNS_14KernelProviderEPNS_12BaseEncodingEPfSG_PNSt7__cxx1112basic_stringIcSt11char_traitsIcESaIcEEE
#define STLQ_CAT2(a, b) a##b
#define STLQ_CAT(a, b) STLQ_CAT2(a, b)

extern "C" bool STLQ_CAT(__real_, STLQ_ENCODE_BASE_SYM)(const stlq::Config& config, const stlq::Dataset& dataset,
                                                         const stlq::CodebookPack& codebooks,
                                                         const stlq::Precomp& precomp, stlq::KernelProvider* kernels,
                                                         stlq::BaseEncoding* base, float* out_beam_mse,
                                                         float* out_final_mse, std::string* error);

namespace {

void DumpBooks(const char* path, const stlq::CodebookPack& cb) {
    FILE* f = std::fopen(path, "wb");
    if (!f) return;
    const int32_t m = static_cast<int32_t>(cb.books.size()), d = cb.d;
    std::fwrite(&m, 4, 1, f);
    std::fwrite(&d, 4, 1, f);
    for (int l = 0; l < m; ++l) {
        const int32_t h = cb.h_vec[static_cast<size_t>(l)];
        std::fwrite(&h, 4, 1, f);
    }
    for (const auto& b : cb.books) std::fwrite(b.data.data(), sizeof(float), b.data.size(), f);
    std::fclose(f);
}

}  // namespace

extern "C" bool STLQ_CAT(__wrap_, STLQ_ENCODE_BASE_SYM)(const stlq::Config& config, const stlq::Dataset& dataset,
                                                         const stlq::CodebookPack& codebooks,
                                                         const stlq::Precomp& precomp, stlq::KernelProvider* kernels,
                                                         stlq::BaseEncoding* base, float* out_beam_mse,
                                                         float* out_final_mse, std::string* error) {
    if (const char* books = std::getenv("STLQ_B200_DROPIN_BOOKS")) DumpBooks(books, codebooks);
    const char* mode = std::getenv("STLQ_B200_DROPIN");
    if (!mode || !*mode)
        return STLQ_CAT(__real_, STLQ_ENCODE_BASE_SYM)(config, dataset, codebooks, precomp, kernels, base,
                                                        out_beam_mse, out_final_mse, error);
    if (std::strcmp(mode, "both") != 0)
        return stlq::b200::EncodeBase(config, dataset, codebooks, precomp, kernels, base, out_beam_mse,
                                      out_final_mse, error);
    stlq::BaseEncoding ref;
    float ref_beam = 0.0f, ref_final = 0.0f;
    std::string ref_err;
    const bool ok_ref = STLQ_CAT(__real_, STLQ_ENCODE_BASE_SYM)(config, dataset, codebooks, precomp, kernels, &ref,
                                                                 &ref_beam, &ref_final, &ref_err);
    const bool ok = stlq::b200::EncodeBase(config, dataset, codebooks, precomp, kernels, base, out_beam_mse,
                                           out_final_mse, error);
    if (const char* rep = std::getenv("STLQ_B200_DROPIN_REPORT")) {
        long n = 0, codes_equal = 0, coeffs_equal = 0;
        if (ok && ok_ref && ref.B.cols == base->B.cols && ref.B.rows == base->B.rows) {
            n = base->B.cols;
            const int m = base->B.rows;
            for (long j = 0; j < n; ++j) {
                codes_equal += std::memcmp(ref.B.Col(static_cast<int>(j)), base->B.Col(static_cast<int>(j)),
                                           sizeof(stlq::FullCode) * static_cast<size_t>(m)) == 0;
                coeffs_equal += std::memcmp(ref.a.Col(static_cast<int>(j)), base->a.Col(static_cast<int>(j)),
                                            sizeof(float) * static_cast<size_t>(m)) == 0;
            }
        }
        if (FILE* f = std::fopen(rep, "a")) {
            std::fprintf(f,
                         "{\"ok_reference\": %d, \"ok_b200\": %d, \"vectors\": %ld, \"m\": %d, \"d\": %d, "
                         "\"codes_equal\": %ld, \"coeffs_equal\": %ld, \"beam_mse_reference\": %.9g, "
                         "\"beam_mse_b200\": %.9g, \"final_mse_reference\": %.9g, \"final_mse_b200\": %.9g, "
                         "\"H_beam\": %d, \"icm_iters\": %d, \"ils_iters\": %d, \"error\": \"%s\"}\n",
                         ok_ref ? 1 : 0, ok ? 1 : 0, n, base->B.rows, codebooks.d, codes_equal, coeffs_equal,
                         ref_beam, out_beam_mse ? *out_beam_mse : 0.0f, ref_final,
                         out_final_mse ? *out_final_mse : 0.0f, config.base.encode.H_beam, config.base.encode.icm_iters,
                         config.base.encode.ils_iters, ok ? "" : (error ? error->c_str() : ""));
            std::fclose(f);
        }
    }
    return ok;
}

// RunStlq with a stage request (include/stlq/stlq.h: kTrainOnly = 2, kBuildBaseOnly = 3) on the
// configuration file `cfg_path`, loaded over the reference's defaults as its own loader does.
extern "C" int dropin_run_mode(const char* cfg_path, int mode) {
    stlq::StlqRunRequest request;
    request.config = stlq::DefaultConfig(false);
    std::string error;
    if (!stlq::LoadConfigFile(cfg_path, &request.config, &error)) {
        std::fprintf(stderr, "LoadConfigFile: %s\n", error.c_str());
        return 1;
    }
    stlq::ApplyDatasetDefaults(&request.config);
    stlq::NormalizeModelHVec(&request.config);
    request.mode = static_cast<stlq::StlqRunMode>(mode);
    stlq::StlqRunResult result;
    const int rc = stlq::RunStlq(request, &result);
    if (rc != 0 && !result.error.empty()) std::fprintf(stderr, "RunStlq: %s\n", result.error.c_str());
    return rc;
}

// RunStlq(argc, argv) exactly as the reference's stlq_main calls it (--config / --set).
extern "C" int dropin_run(int argc, char** argv) {
    stlq::StlqRunResult result;
    const int rc = stlq::RunStlq(argc, argv, &result);
    if (rc != 0 && !result.error.empty()) std::fprintf(stderr, "RunStlq: %s\n", result.error.c_str());
    return rc;
}
