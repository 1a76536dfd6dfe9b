// Host-side launchers of the stlq_b200 kernels (defined in the .cu files of this directory).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "types.h"

namespace stlq_b200 {

cudaError_t LaunchXcGemmExact(const float* C, int rows, int d, const void* X, int x_dtype, int64_t n, float* out,
                              int ldo, float* xnorm2, double* xnorm2_d, cudaStream_t stream);
int MaxGemmSliceVectors();

// Tensor-core (tcgen05) GEMM of the STRICT (split = true, 3xTF32) and FAST (1xTF32) modes.
// A = rows x d and B = n x d row-major fp32 (hi parts; lo parts used when split); d % 4 == 0 and
// 16-byte aligned bases (TMA); n <= 65535 * 128.  Bounded waits raise kErrWaitTimeout in *err.
cudaError_t LaunchXcGemmTc(const float* a_hi, const float* a_lo, int rows, const float* b_hi, const float* b_lo,
                           int64_t n, int d, float* out, int ldo, bool split, unsigned int* err, cudaStream_t stream);
// hi = x rounded to TF32, lo = (x - hi) rounded to TF32 (lo may be null); x is F32 or U8.
cudaError_t LaunchSplitTf32(const void* x, int x_dtype, int64_t count, float* hi, float* lo, cudaStream_t stream);
// ||x||^2 per vector in float (the reference's 4-lane SIMD order) and in double; either may be null.
cudaError_t LaunchNorms(const void* X, int x_dtype, int64_t n, int d, float* xn, double* xnd, cudaStream_t stream);

// Dynamic shared memory of the fast beam kernel (the larger of the two beam kernels); strict: its
// STRICT-mode instantiation.
size_t BeamFastSmemBytes(const Dims& dims, int beam, bool strict = false);
// ea (null, or ea->X null: xC is exact): STRICT mode's inputs for exact xC entries on demand.
cudaError_t LaunchBeamSearch(const Dims& dims, const float* Grow, const float* Gdiag, const float* xnorm2,
                             const float* xC, int64_t n, int beam, void* Bout, int* redo, int check,
                             unsigned int* err_flag, int num_sms, cudaStream_t stream,
                             const ExactDotArgs* ea = nullptr);

struct RefineArgs {
    Dims dims;
    const float* Gcol;   // Gram array of the refinement (layout: Dims::ldg, Dims::c0)
    const float* Gdiag;  // G(h, h) for every flat index h
    const float* invnorm;
    const float* xC;
    const float* xnorm2;
    const double* xnorm2_d;
    int64_t n;
    int mode;  // 0 = LS only, 1 = full (LS, ICM, ILS, cost)
    int icm_iters;
    int n_ils;
    int perturb_k;
    int use_abs;
    uint32_t seed;
    uint64_t sample_id_offset;
    const int* orders;  // [(n_ils + 1)][icm_iters][m]
    void* B;  // m x n codes, uint8 or (dims.wide) uint16
    float* a;
    float* cost;
    double* partials;  // [grid][2] (beam SSE, final SSE) or null
    // STRICT mode (ex.X non-null, mode 1): xC holds tensor-core entries; the kernel writes the exact
    // entry of every codeword an LS solve or a cost reads into xC (which must be writable) before
    // reading it, and resolves ICM choices from bounds plus exact scores (see refine.cu).
    ExactDotArgs ex;
    unsigned int* err_flag;  // STRICT: kErrTcBound is raised here
};

cudaError_t LaunchRefine(const RefineArgs& args, int grid, cudaStream_t stream);
cudaError_t LaunchReducePartials(const double* partials, int nblocks, double* out, cudaStream_t stream);
cudaError_t LaunchSse(const Dims& dims, const float* Gcol, const float* Gdiag, const float* xC, const double* xnorm2_d,
                      const void* B, const float* a, int64_t n, double* partials, int grid, cudaStream_t stream);
int RefineWarpsPerBlock();
int RefineBlocksPerSm();

// Loads both beam kernels and sets their shared-memory attributes (no launch).
cudaError_t PrepareBeamKernels(const Dims& dims, int beam);
// Loads every instantiation of the beam kernels on the current device (no launch).
cudaError_t LoadAllBeamKernels();

// What the beam-search launch needs from an encoder handle (api.cpp).
struct BeamInputs {
    Dims dims;
    const float* Grow;
    const float* Gdiag;
    unsigned int* err_flag;
    int check_filter;
    int num_sms;
    int device;
};

cudaError_t LaunchTranspose(const float* in, float* out, int rows, int cols, cudaStream_t stream);
cudaError_t LaunchDiag(const float* Gcol, float* diag, int H, cudaStream_t stream);
cudaError_t LaunchInvnorm(const float* C, int H, int d, float* invnorm, cudaStream_t stream);
// The beam's diagonal: Gdiag with -0.0f for codewords of codebooks 1..m-1 whose Gram column is
// exactly zero (skipped by the reference in every slot) and +0.0f for any other zero.
cudaError_t LaunchBeamDiag(const Dims& dims, const float* Gcol, const float* Gdiag, float* Bdiag,
                           cudaStream_t stream);
cudaError_t LaunchU8ToF32(const uint8_t* x, int64_t count, float* out, cudaStream_t stream);
// cn[h] >= ||c_h|| for the H codewords of C (H x d): STRICT mode's tensor-core error bounds.
cudaError_t LaunchNormBounds(const float* C, int H, int d, float* cn, cudaStream_t stream);
// Large-root precompute: invnorm from the SIMD-order norms; Gdiag = norm0 for the h0 root codewords
// and the compact Gram's diagonal (G[h * Hs + h - h0]) for the others.
cudaError_t LaunchLargeRootPrecomp(const float* norms, int h0, int H, const float* G, float* Gdiag, float* invnorm,
                                   cudaStream_t stream);
// Large-root mode: xC[vec][root] = the reference's SIMD-order dot of the chosen root codeword with
// x (Dot, least_squares.cpp:35-42), which its LS, cost and ICM use for the root term.
cudaError_t LaunchRootDot(const Dims& dims, const float* C, const void* X, int x_dtype, const void* B, int64_t n,
                          float* xC, cudaStream_t stream);
cudaError_t LaunchSplitRootCodes(int m, const void* B, int wide, int64_t n, uint32_t* cluster, uint8_t* B_small,
                                 cudaStream_t stream);

}  // namespace stlq_b200
