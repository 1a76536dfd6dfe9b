// Device-side parts of BuildPrecomp (reference src/quantizer/encoder_precomp.inc:1-53) that the
// encoder derives from C_all and G: the row-major copy of G used by the beam kernel's coalesced
// cross-term gathers, the diagonal alpha = G(h, h), and 1/||c_h||.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

// out[c * rows + r] = in[r * cols + c] through 32x32 shared-memory tiles.
__global__ void TransposeKernel(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = in[static_cast<size_t>(r) * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = bx + j, r = by + threadIdx.x;
        if (r < rows && c < cols) out[static_cast<size_t>(c) * rows + r] = tile[threadIdx.x][j];
    }
}

__global__ void DiagKernel(const float* __restrict__ Gcol, float* __restrict__ diag, int H) {
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h < H) diag[h] = Gcol[static_cast<size_t>(h) * H + h];
}

// The beam's copy of the Gram diagonal: -0.0f marks a codeword of codebooks 1..m-1 whose Gram
// column G(., c) is exactly zero (it can never enter a beam); a diagonal 0 of any other codeword
// is written as +0.0f, and every other value is copied.  One warp per codeword; the column is read
// through the refinement's layout (Gcol[c * ldg + r - c0] = G(r, c) for r >= c0; a large-root
// encoder's root rows G(r, c), r < c0, at Gcol[r * ldg + c - c0]).
__global__ void BeamDiagKernel(Dims dims, const float* __restrict__ Gcol, const float* __restrict__ Gdiag,
                               float* __restrict__ Bdiag) {
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= dims.H) return;
    const float g = Gdiag[c];
    bool zero = dims.m > 1 && c >= dims.off[1] && g == 0.0f;
    if (zero) {  // warp-uniform: c is the warp's, and `zero` only changes through __all_sync
        const size_t ld = static_cast<size_t>(dims.ldg);
        for (int r0 = 0; r0 < dims.H; r0 += 32) {
            const int r = r0 + lane;
            float v = 0.0f;
            if (r < dims.H) v = r >= dims.c0 ? Gcol[c * ld + (r - dims.c0)] : Gcol[r * ld + (c - dims.c0)];
            zero = __all_sync(0xffffffffu, v == 0.0f);
            if (!zero) break;
        }
    }
    if (lane == 0) Bdiag[c] = zero ? -0.0f : (g == 0.0f ? 0.0f : g);
}

// invnorm_flat[h] = 1/sqrt(sum_r c_r^2) with the reference's sequential float sum
// (encoder_precomp.inc:31-39); 0 for a zero codeword.
__global__ void InvnormKernel(const float* __restrict__ C, int H, int d, float* __restrict__ invnorm) {
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= H) return;
    const float* c = C + static_cast<size_t>(h) * d;
    float s = 0.0f;
    for (int r = 0; r < d; ++r) s = __fadd_rn(s, __fmul_rn(c[r], c[r]));
    invnorm[h] = s > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(s)) : 0.0f;
}

// Large-root precompute from the codewords' norms in the reference's SIMD order (Norm2,
// precomp_large_root.cpp:15-23): invnorm = 1/sqrt(norm) (0 for a zero codeword); the diagonal is
// norm0 for the h0 root codewords (BuildPrecompLargeRoot :85-91) and G_small's for the others (the
// compact Gram G[h * (H - h0) + (h - h0)]).
__global__ void LargeRootPrecompKernel(const float* __restrict__ norms, int h0, int H, const float* __restrict__ G,
                                       float* Gdiag, float* invnorm) {
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= H) return;
    const float n2 = norms[h];
    invnorm[h] = n2 > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(n2)) : 0.0f;
    Gdiag[h] = h < h0 ? n2 : G[static_cast<size_t>(h) * (H - h0) + (h - h0)];
}

__global__ void U8ToF32Kernel(const uint8_t* __restrict__ x, int64_t count, float* __restrict__ out) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = static_cast<float>(x[i]);
}

// Upper bounds of ||c_h||: the norm in double, rounded to float and raised by 2^-20 (far above
// the roundings), one warp per codeword.
__global__ void NormBoundKernel(const float* __restrict__ C, int H, int d, float* __restrict__ cn) {
    const int h = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (h >= H) return;
    double s = 0.0;
    for (int i = lane; i < d; i += 32) {
        const double v = C[static_cast<size_t>(h) * d + i];
        s += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) cn[h] = static_cast<float>(sqrt(s)) * (1.0f + 0x1p-20f);
}

}  // namespace

cudaError_t LaunchNormBounds(const float* C, int H, int d, float* cn, cudaStream_t stream) {
    NormBoundKernel<<<(H + 7) / 8, 256, 0, stream>>>(C, H, d, cn);
    return cudaGetLastError();
}

cudaError_t LaunchU8ToF32(const uint8_t* x, int64_t count, float* out, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 32));
    U8ToF32Kernel<<<grid, 256, 0, stream>>>(x, count, out);
    return cudaGetLastError();
}

cudaError_t LaunchLargeRootPrecomp(const float* norms, int h0, int H, const float* G, float* Gdiag, float* invnorm,
                                   cudaStream_t stream) {
    LargeRootPrecompKernel<<<(H + 255) / 256, 256, 0, stream>>>(norms, h0, H, G, Gdiag, invnorm);
    return cudaGetLastError();
}

cudaError_t LaunchTranspose(const float* in, float* out, int rows, int cols, cudaStream_t stream) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    TransposeKernel<<<grid, block, 0, stream>>>(in, out, rows, cols);
    return cudaGetLastError();
}

cudaError_t LaunchDiag(const float* Gcol, float* diag, int H, cudaStream_t stream) {
    DiagKernel<<<(H + 255) / 256, 256, 0, stream>>>(Gcol, diag, H);
    return cudaGetLastError();
}

cudaError_t LaunchBeamDiag(const Dims& dims, const float* Gcol, const float* Gdiag, float* Bdiag,
                           cudaStream_t stream) {
    BeamDiagKernel<<<(dims.H + 7) / 8, 256, 0, stream>>>(dims, Gcol, Gdiag, Bdiag);
    return cudaGetLastError();
}

cudaError_t LaunchInvnorm(const float* C, int H, int d, float* invnorm, cudaStream_t stream) {
    InvnormKernel<<<(H + 127) / 128, 128, 0, stream>>>(C, H, d, invnorm);
    return cudaGetLastError();
}

}  // namespace stlq_b200
