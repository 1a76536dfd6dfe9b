// Plain types shared by the host launchers and the kernels of stlq_b200.
#pragma once

#include <cstdint>

namespace stlq_b200 {

constexpr int kMaxM = 16;
constexpr int kMaxK = 256;
constexpr int kMaxBeam = 32;
constexpr int kMaxKWide = 1024;  // codewords per codebook with uint16 codes
constexpr float kIcmEps = 1e-6f;  // icm.cpp:29, least_squares.cpp:19

// Device-side error flags (bit set by a kernel that met a state it cannot handle; read by the
// host after the stream synchronises).  Kernels never trap.
enum DeviceError : unsigned int {
    kErrNone = 0,
    kErrSurvivorOverflow = 1u << 0,
    kErrBadShape = 1u << 1,
    kErrFilterMiss = 1u << 2,  // self-check: a candidate the beam pre-filter dropped would have entered
    kErrWaitTimeout = 1u << 3,  // a bounded barrier wait of the tensor-core GEMM ran out
    kErrTcBound = 1u << 4,      // STRICT: a tensor-core xC entry was outside its error bound
};

// STRICT mode inputs of the exact xC entries computed on demand (see ExactCtx in common.cuh).
// X == nullptr: the kernels take xC as exact (EXACT and FAST modes, the stage entry points).
struct ExactDotArgs {
    const float* C;      // C_all, codeword h at C + h * d
    const void* X;       // the slice's vectors as encoded (rotated when a rotation is set)
    int x_dtype;         // 0 float32, 1 uint8
    const float* cn;     // upper bounds of ||c_h||
    float kappa;         // |xC_tensor - xC_exact| <= kappa ||c_h|| ||x||
};

// Encoder constants shared by every kernel, passed by value.
struct Dims {
    int d;        // vector dimension
    int m;        // codebooks
    int H;        // sum of h_vec
    int maxK;     // max of h_vec
    int maxKs;    // max of h_vec[1..m-1] (1 when m == 1): candidates per beam slot and layer
    int h_vec[kMaxM];
    int off[kMaxM];
    // Gram storage.  The beam reads G(r, c), c >= c0, at Grow[r * ldg + (c - c0)]; the refinement
    // reads G(r, c), r >= c0, at Gcol[c * ldg + (r - c0)].  Regular encoders hold all of G in both
    // orientations (ldg = H, c0 = 0).  Large-root encoders hold one array for both (G is computed
    // on the device and symmetric) with only the columns of codebooks 1..m-1 (ldg = H - h0,
    // c0 = h0): the reference's G0S and G_small blocks.  The root codewords' own diagonal is in
    // the diagonal array; no other root-root entry is ever needed.
    int ldg;
    int c0;
    // Large-root encoder (PrecompLargeRoot, reference include/stlq/quantizer/precomp_large_root.h):
    // codebook 0 is the root; the beam's triangular solves multiply by 1/R_ii
    // (beam_search.cpp:517-575) and costs follow SampleCostLargeRoot (cost_utils.cpp:160-209).
    int large_root;
    // Codes are uint16 (some codebook has more than 256 codewords) instead of uint8.
    int wide;
};

}  // namespace stlq_b200
