// xC = C_all^T X with FP32 FMA chains in the summation order of the reference's CPU BLAS
// backend (call site: reference src/quantizer/encoder_encode_base.inc:33-37 -> src/core/blas.cpp).
//
// The reference build links OpenBLAS (or MKL); in this image that is OpenBLAS 0.3.15, whose
// SkylakeX SGEMM computes each output as one FMA chain per K block, with K split into blocks of
// 448 (the remainder halved and rounded up to 16 when between 448 and 896) and the block results
// summed in order.  Reproducing that order makes xC, and therefore every later decision of the
// encoder, bit-identical to the reference's.
//
// Tiling: a CTA computes 128 codewords x 128 vectors with 256 threads, each an 8 x 8 register tile
// (rows tx*4..+3 and 64+tx*4..+3, vectors ty*4..+3 and 64+ty*4..+3, so that every shared-memory
// read is a 128-bit broadcast or a conflict-free row).  K advances 16 at a time through two
// shared-memory buffers: the next step's global loads are in flight while the current one is
// multiplied, with one barrier per step.  Every K block boundary (a multiple of 16) falls between
// steps; a partial last step runs only its kn terms, so no output gets an extra (+0) term.
// Output layout: xC[vec * ldo + codeword].  ||x||^2 comes from LaunchNorms (same order as the
// reference's SIMD loop).
//
// The same kernel is the general sgemm of the kernel-provider seam (LaunchSgemmExact): with row
// strides lda / ldb and OpenBLAS's alpha / beta epilogue, C starts at fl(beta * C) (0 when beta is 0)
// and each K block's chain is folded as C = fma(alpha, chain, C), in block order (the single-thread
// OpenBLAS 0.3.15 result for every transpose, checked against the reference's GemmRaw).  With
// alpha = 1 and beta = 0 that is exactly the xC product above.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kTM = 128, kTN = 128, kBK = 16, kGemmThreads = 256;

// Loads rows [row0, row0 + 128) x k [k0, k0 + 16) of a row-major matrix with `d` columns into
// registers: thread t holds rows t/4 and t/4 + 64, columns 4*(t%4)..+3 (zero outside).
template <typename T>
struct TileLoader {
    float v[2][4];
    __device__ __forceinline__ void Load(const T* __restrict__ M, int64_t nrows, int64_t ld, int d, int64_t row0,
                                         int k0, bool vec4) {  // row r at M + r * ld; vec4: aligned 4-loads
        const int tid = threadIdx.x;
        const int kq = 4 * (tid & 3);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t r = row0 + (tid >> 2) + 64 * h;
            const int k = k0 + kq;
            if (r < nrows && vec4 && k + 3 < d) {
                const T* p = M + r * ld + k;
                if constexpr (sizeof(T) == 4) {
                    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
                    v[h][0] = q.x, v[h][1] = q.y, v[h][2] = q.z, v[h][3] = q.w;
                } else {
                    const uchar4 q = *reinterpret_cast<const uchar4*>(p);
                    v[h][0] = q.x, v[h][1] = q.y, v[h][2] = q.z, v[h][3] = q.w;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    v[h][c] = (r < nrows && k + c < d) ? static_cast<float>(M[r * ld + k + c]) : 0.0f;
            }
        }
    }
    // Transposed into S[k][row].
    __device__ __forceinline__ void Store(float (*S)[kTM]) const {
        const int tid = threadIdx.x;
        const int kq = 4 * (tid & 3);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 4; ++c) S[kq + c][(tid >> 2) + 64 * h] = v[h][c];
    }
};

// Output element (row i, vector j) of this thread's 8 x 8 tile before the product: fl(beta * C),
// or 0 when beta is 0 (C not read).
__device__ __forceinline__ float InitialC(const float* out, int ldo, int r0, int64_t j0, int i, int j, int rows,
                                         int64_t n, float beta, int tx, int ty) {
    if (beta == 0.0f) return 0.0f;
    const int r = r0 + (i < 4 ? tx * 4 + i : 64 + tx * 4 + (i - 4));
    const int64_t gj = j0 + (j < 4 ? ty * 4 + j : 64 + ty * 4 + (j - 4));
    return (r < rows && gj < n) ? __fmul_rn(beta, out[gj * ldo + r]) : 0.0f;
}

template <typename T, bool kMulti>
__global__ void __launch_bounds__(kGemmThreads, kMulti ? 1 : 2)
    XcGemmExactKernel(const float* __restrict__ C, int rows, int d, const T* __restrict__ X, int64_t n,
                      float* __restrict__ out, int ldo, bool cvec, bool xvec, bool ovec, int64_t ldc_in,
                      int64_t ldx, float alpha, float beta) {
    __shared__ __align__(16) float Cs[2][kBK][kTM];
    __shared__ __align__(16) float Xs[2][kBK][kTN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int r0 = blockIdx.x * kTM;
    const int64_t j0 = static_cast<int64_t>(blockIdx.y) * kTN;

    float part[8][8];
    float tot[kMulti ? 8 : 1][kMulti ? 8 : 1];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) part[i][j] = 0.0f;
    bool first = true;
    int kb_end = NextKBlock(d);  // end of the current K block

    TileLoader<float> lc;
    TileLoader<T> lx;
    lc.Load(C, rows, ldc_in, d, r0, 0, cvec);
    lx.Load(X, n, ldx, d, j0, 0, xvec);
    lc.Store(Cs[0]);
    lx.Store(Xs[0]);
    __syncthreads();
    const int steps = (d + kBK - 1) / kBK;
    for (int s = 0; s < steps; ++s) {
        const int k0 = s * kBK, buf = s & 1;
        if (s + 1 < steps) {
            lc.Load(C, rows, ldc_in, d, r0, k0 + kBK, cvec);
            lx.Load(X, n, ldx, d, j0, k0 + kBK, xvec);
        }
        if (kMulti && k0 == kb_end) {  // a new K block: fold the finished block's chains
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if constexpr (kMulti) {
                        if (first) tot[i][j] = InitialC(out, ldo, r0, j0, i, j, rows, n, beta, tx, ty);
                        tot[i][j] = __fmaf_rn(alpha, part[i][j], tot[i][j]);
                    }
                    part[i][j] = 0.0f;
                }
            first = false;
            kb_end += NextKBlock(d - k0);
        }
        const int kn = min(kBK, d - k0);
        auto step = [&](int kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&Cs[buf][kk][tx * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&Cs[buf][kk][64 + tx * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Xs[buf][kk][ty * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Xs[buf][kk][64 + ty * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) part[i][j] = __fmaf_rn(a[i], b[j], part[i][j]);
        };
        if (kn == kBK) {
#pragma unroll
            for (int kk = 0; kk < kBK; ++kk) step(kk);
        } else {
            for (int kk = 0; kk < kn; ++kk) step(kk);
        }
        if (s + 1 < steps) {
            lc.Store(Cs[buf ^ 1]);
            lx.Store(Xs[buf ^ 1]);
        }
        __syncthreads();
    }

#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int64_t gj = j0 + (j < 4 ? ty * 4 + j : 64 + ty * 4 + (j - 4));
        if (gj >= n) continue;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float c;
            if constexpr (kMulti) c = first ? InitialC(out, ldo, r0, j0, i, j, rows, n, beta, tx, ty) : tot[i][j];
            else c = InitialC(out, ldo, r0, j0, i, j, rows, n, beta, tx, ty);
            v[i] = __fmaf_rn(alpha, part[i][j], c);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = r0 + 64 * h + tx * 4;
            float* o = out + gj * ldo + r;
            if (r + 4 <= rows && ovec) {
                *reinterpret_cast<float4*>(o) = make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (r + i < rows) o[i] = v[4 * h + i];
            }
        }
    }
}

// C rows at C + r * ldc_in, X rows at X + j * ldx (both contiguous over the d products).
template <typename T>
cudaError_t LaunchT(const float* C, int rows, int d, const T* X, int64_t n, float* out, int ldo, cudaStream_t stream,
                    int64_t ldc_in, int64_t ldx, float alpha = 1.0f, float beta = 0.0f) {
    const int64_t gy = (n + kTN - 1) / kTN;
    if (gy > 65535) return cudaErrorInvalidValue;  // callers slice n
    dim3 grid((rows + kTM - 1) / kTM, static_cast<unsigned>(gy));
    // Vector loads need every row to start aligned: d and the row stride multiples of 4, an aligned base.
    const bool cvec = d % 4 == 0 && ldc_in % 4 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0;
    const bool xvec = d % 4 == 0 && ldx % 4 == 0 && reinterpret_cast<uintptr_t>(X) % (4 * sizeof(T)) == 0;
    const bool ovec = ldo % 4 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
    if (d > 448)
        XcGemmExactKernel<T, true><<<grid, kGemmThreads, 0, stream>>>(C, rows, d, X, n, out, ldo, cvec, xvec, ovec,
                                                                      ldc_in, ldx, alpha, beta);
    else
        XcGemmExactKernel<T, false><<<grid, kGemmThreads, 0, stream>>>(C, rows, d, X, n, out, ldo, cvec, xvec, ovec,
                                                                       ldc_in, ldx, alpha, beta);
    return cudaGetLastError();
}

}  // namespace

// out (ldo-strided per vector) = C^T X for `rows` codewords; optional norms (LaunchNorms).
cudaError_t LaunchXcGemmExact(const float* C, int rows, int d, const void* X, int x_dtype, int64_t n, float* out,
                              int ldo, float* xnorm2, double* xnorm2_d, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    cudaError_t e = x_dtype == 0 ? LaunchT(C, rows, d, static_cast<const float*>(X), n, out, ldo, stream, d, d)
                                 : LaunchT(C, rows, d, static_cast<const uint8_t*>(X), n, out, ldo, stream, d, d);
    if (e != cudaSuccess) return e;
    if (xnorm2 || xnorm2_d) return LaunchNorms(X, x_dtype, n, d, xnorm2, xnorm2_d, stream);
    return cudaSuccess;
}

int MaxGemmSliceVectors() { return 65535 * 64; }

// out(rows x n, ldo) = alpha * A B + beta * out with A's rows at A + i * lda and B's columns at
// B + j * ldb, both contiguous over the k products (an op(A) of a transposed A, an op(B) of a
// plain B); n is sliced to the grid limit here.
cudaError_t LaunchSgemmExact(const float* A, int64_t lda, int rows, int k, const float* B, int64_t ldb, int64_t n,
                             float alpha, float beta, float* out, int ldo, cudaStream_t stream) {
    const int64_t S = int64_t{65535} * kTN;
    for (int64_t j0 = 0; j0 < n; j0 += S) {
        const int64_t nj = std::min<int64_t>(S, n - j0);
        cudaError_t e = LaunchT(A, rows, k, B + j0 * ldb, nj, out + j0 * ldo, ldo, stream, lda, ldb, alpha, beta);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace stlq_b200
