// xC = C_all^T X with FP32 FMA chains in the summation order of the reference's CPU BLAS
// backend (call site: reference src/quantizer/encoder_encode_base.inc:33-37 -> src/core/blas.cpp).
//
// The reference build links OpenBLAS (or MKL); in this image that is OpenBLAS 0.3.15, whose
// SkylakeX SGEMM computes each output as one FMA chain per K block, with K split into blocks of
// 448 (the remainder halved and rounded up to 16 when between 448 and 896) and the block results
// summed in order.  Reproducing that order makes xC, and therefore every later decision of the
// encoder, bit-identical to the reference's.
//
// The same kernel fuses ||x||^2 per vector in the order GCC gives the reference's
// `#pragma omp simd reduction` (4 lanes, tail into lane 0, lanes summed in order;
// cost_utils.cpp:99-109, beam_search.cpp:218-223) plus the double-precision norm used by the MSE
// (linkage_tools.cpp:187-191): the CTAs of the first codeword tile write them.
//
// Tiling: a CTA computes 128 codewords x 64 vectors; 256 threads, each an 8 x 4 register tile;
// K advances 16 at a time through shared memory.  Output layout: xC[vec * H + codeword].
#include <cstdint>

#include "common.cuh"
#include "launch.h"

namespace stlq_b200 {

namespace {

constexpr int kBR = 128, kBJ = 64, kBK = 16, kTR = 8, kTJ = 4, kGemmThreads = 256;

__host__ __device__ __forceinline__ int NextKBlock(int rem) {
    const int Q = 448, U = 16;
    if (rem >= 2 * Q) return Q;
    if (rem > Q) return ((rem / 2) + U - 1) & ~(U - 1);
    return rem;
}

template <typename T>
__device__ __forceinline__ float ToF(T v) { return static_cast<float>(v); }

template <typename T, bool kNorms>
__global__ void __launch_bounds__(kGemmThreads) XcGemmExactKernel(const float* __restrict__ C, int rows, int d,
                                                                  const T* __restrict__ X, int64_t n,
                                                                  float* __restrict__ out, int ldo,
                                                                  float* __restrict__ xnorm2,
                                                                  double* __restrict__ xnorm2_d) {
    __shared__ __align__(16) float Cs[kBK][kBR + 4];
    __shared__ __align__(16) float Xs[kBK][kBJ + 4];
    const int tid = threadIdx.x;
    const int tr = tid % 16, tj = tid / 16;
    const int r0 = blockIdx.x * kBR;
    const int64_t j0 = static_cast<int64_t>(blockIdx.y) * kBJ;

    float tot[kTR][kTJ], part[kTR][kTJ];
#pragma unroll
    for (int i = 0; i < kTR; ++i)
#pragma unroll
        for (int j = 0; j < kTJ; ++j) tot[i][j] = 0.0f;

    // Norm lanes: thread (nj = tid / 4, lane = tid % 4) owns vector j0+nj, lane `lane`.
    const bool do_norm = kNorms && blockIdx.x == 0;
    float lane_sum = 0.0f;
    double dsum = 0.0;
    const int body = (d / 4) * 4;

    bool first_block = true;
    for (int kb0 = 0; kb0 < d;) {
        const int kblk = NextKBlock(d - kb0);
#pragma unroll
        for (int i = 0; i < kTR; ++i)
#pragma unroll
            for (int j = 0; j < kTJ; ++j) part[i][j] = 0.0f;
        for (int k0 = kb0; k0 < kb0 + kblk; k0 += kBK) {
            const int kn = min(kBK, kb0 + kblk - k0);
            // Stage C (128 x kn) and X (64 x kn), transposed to [k][row].
            for (int e = tid; e < kBR * kBK; e += kGemmThreads) {
                const int r = e / kBK, kk = e % kBK;
                const int gr = r0 + r;
                Cs[kk][r] = (kk < kn && gr < rows) ? __ldg(C + static_cast<size_t>(gr) * d + k0 + kk) : 0.0f;
            }
            for (int e = tid; e < kBJ * kBK; e += kGemmThreads) {
                const int j = e / kBK, kk = e % kBK;
                const int64_t gj = j0 + j;
                Xs[kk][j] = (kk < kn && gj < n) ? ToF(X[gj * d + k0 + kk]) : 0.0f;
            }
            __syncthreads();
            for (int kk = 0; kk < kn; ++kk) {
                float a[kTR], b[kTJ];
#pragma unroll
                for (int i = 0; i < kTR; ++i) a[i] = Cs[kk][tr * kTR + i];
#pragma unroll
                for (int j = 0; j < kTJ; ++j) b[j] = Xs[kk][tj * kTJ + j];
#pragma unroll
                for (int i = 0; i < kTR; ++i)
#pragma unroll
                    for (int j = 0; j < kTJ; ++j) part[i][j] = __fmaf_rn(a[i], b[j], part[i][j]);
            }
            if (do_norm) {
                const int nj = tid / 4, lane = tid % 4;
                for (int kk = 0; kk < kn; ++kk) {
                    const int k = k0 + kk;
                    const float x = Xs[kk][nj];
                    const bool mine = (k < body) ? ((k & 3) == lane) : (lane == 0);
                    if (mine) {
                        lane_sum = __fadd_rn(lane_sum, __fmul_rn(x, x));
                        dsum = __dadd_rn(dsum, __dmul_rn(static_cast<double>(x), static_cast<double>(x)));
                    }
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < kTR; ++i)
#pragma unroll
            for (int j = 0; j < kTJ; ++j) tot[i][j] = first_block ? part[i][j] : __fadd_rn(tot[i][j], part[i][j]);
        first_block = false;
        kb0 += kblk;
    }

#pragma unroll
    for (int j = 0; j < kTJ; ++j) {
        const int64_t gj = j0 + tj * kTJ + j;
        if (gj >= n) continue;
        float* o = out + gj * ldo + r0 + tr * kTR;
        if (r0 + tr * kTR + kTR <= rows && (ldo % 4) == 0) {
            reinterpret_cast<float4*>(o)[0] = make_float4(tot[0][j], tot[1][j], tot[2][j], tot[3][j]);
            reinterpret_cast<float4*>(o)[1] = make_float4(tot[4][j], tot[5][j], tot[6][j], tot[7][j]);
        } else {
#pragma unroll
            for (int i = 0; i < kTR; ++i)
                if (r0 + tr * kTR + i < rows) o[i] = tot[i][j];
        }
    }

    if (do_norm) {
        // Combine the 4 lanes of each vector in order: ((l0 + l1) + l2) + l3.
        __shared__ float lanes[kBJ][4];
        __shared__ double dl[kBJ][4];
        const int nj = tid / 4, lane = tid % 4;
        lanes[nj][lane] = lane_sum;
        dl[nj][lane] = dsum;
        __syncthreads();
        if (tid < kBJ && j0 + tid < n) {
            float s = __fadd_rn(lanes[tid][0], lanes[tid][1]);
            s = __fadd_rn(s, lanes[tid][2]);
            s = __fadd_rn(s, lanes[tid][3]);
            if (xnorm2) xnorm2[j0 + tid] = s;
            if (xnorm2_d) xnorm2_d[j0 + tid] = (dl[tid][0] + dl[tid][1]) + (dl[tid][2] + dl[tid][3]);
        }
    }
}

}  // namespace

// out (ldo-strided per vector) = C^T X for `rows` codewords; optional norms.
cudaError_t LaunchXcGemmExact(const float* C, int rows, int d, const void* X, int x_dtype, int64_t n, float* out,
                              int ldo, float* xnorm2, double* xnorm2_d, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int64_t gy = (n + kBJ - 1) / kBJ;
    if (gy > 65535) return cudaErrorInvalidValue;  // callers slice n
    dim3 grid((rows + kBR - 1) / kBR, static_cast<unsigned>(gy));
    const bool norms = xnorm2 || xnorm2_d;
    if (x_dtype == 0) {
        if (norms)
            XcGemmExactKernel<float, true><<<grid, kGemmThreads, 0, stream>>>(C, rows, d, static_cast<const float*>(X),
                                                                             n, out, ldo, xnorm2, xnorm2_d);
        else
            XcGemmExactKernel<float, false><<<grid, kGemmThreads, 0, stream>>>(C, rows, d, static_cast<const float*>(X),
                                                                              n, out, ldo, nullptr, nullptr);
    } else {
        if (norms)
            XcGemmExactKernel<uint8_t, true><<<grid, kGemmThreads, 0, stream>>>(
                C, rows, d, static_cast<const uint8_t*>(X), n, out, ldo, xnorm2, xnorm2_d);
        else
            XcGemmExactKernel<uint8_t, false><<<grid, kGemmThreads, 0, stream>>>(
                C, rows, d, static_cast<const uint8_t*>(X), n, out, ldo, nullptr, nullptr);
    }
    return cudaGetLastError();
}

int MaxGemmSliceVectors() { return 65535 * kBJ; }

}  // namespace stlq_b200
