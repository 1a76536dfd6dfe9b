// xC = C_all^T X on the 5th-generation tensor cores (tcgen05, TMEM accumulator, TMA operand loads):
// the STLQ_B200_GEMM_STRICT (3xTF32) and STLQ_B200_GEMM_FAST (1xTF32) modes.
//
// Reference call site: src/quantizer/encoder_encode_base.inc:33-37 (CPU SGEMM) and the cuBLAS
// GEMM of the CUDA kernel provider (src/core/kernel_provider_cuda_stream_impl.inc:407-463, TF32
// in "fast" mode).  These modes are FP32-accurate (3xTF32) or TF32-accurate, not bit-identical to
// the reference's BLAS; STLQ_B200_GEMM_EXACT (xc_gemm_exact.cu) is the bit-identical mode.
//
// 3xTF32: each operand is split once into hi = the value rounded to the nearest TF32 number and
// lo = (value - hi) rounded to TF32 (|lo| <= 2^-11 |value|); the tile then accumulates
// hi*hi + hi*lo + lo*hi in FP32 in TMEM, so a product carries ~2^-21 relative error (the dropped
// lo*lo term and the rounding of lo) before the FP32 accumulation.  1xTF32 uses hi alone.
//
// One CTA computes a 128-codeword x 128-vector tile: warp 0 issues TMA loads (128-byte swizzle,
// 32 K-elements = one swizzle row per stage) into a 2-stage ring, warp 1 allocates 128 TMEM
// columns and one thread issues the MMAs (4 K-steps of 8 per stage), warps 2-5 read the
// accumulator back with tcgen05.ld (one TMEM lane quarter each) and store it coalesced along the
// codeword axis.  Every barrier wait is bounded in time; on expiry the kernel raises a flag,
// releases its TMEM and returns.
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "launch.h"
#include "tc_ptx.cuh"

namespace stlq_b200 {

namespace {

constexpr int kTile = 128;                          // M = N = 128
constexpr int kTileK = 32;                          // fp32 elements per 128-byte swizzle row
constexpr uint32_t kTileBytes = kTile * kTileK * 4;  // 16 KB per operand tile
// One shared-memory stage (64 KB of operand tiles) so that three CTAs fit on an SM: a CTA's
// epilogue (TMEM -> registers -> 64 KB of stores) then overlaps the others' loads and MMAs.  With
// two stages (128 KB) one CTA fit and the tile's work ran serially: 1.42 ms against 0.97 ms per
// 262,144 x 2,048 x 128 STRICT GEMM.
constexpr int kStages = 1;
constexpr int kCtasPerSm = 3;
constexpr int kTcThreads = 192;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per barrier wait

template <bool kSplit>
__global__ void __launch_bounds__(kTcThreads, kCtasPerSm)
    XcGemmTcKernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo, int rows,
                   int64_t n, int d, float* __restrict__ out, int ldo, unsigned int* err) {
    extern __shared__ unsigned char smem_raw[];
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023);
    float* tiles = reinterpret_cast<float*>(base);  // [kStages][4 operands][kTile * kTileK]
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * 4 * kTileBytes);
    uint64_t* empty = full + kStages;
    uint64_t* accum = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    auto tile = [&](int s, int op) { return tiles + (s * 4 + op) * (kTile * kTileK); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTile;
    const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kTile;
    const int nk = (d + kTileK - 1) / kTileK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::MbarInit(&full[s], 1);
            tc::MbarInit(&empty[s], 1);
        }
        tc::MbarInit(accum, 1);
        tc::FenceBarrierInit();
    }
    if (warp == 1) tc::TmemAlloc(tmem_slot, kTile);
    tc::FenceBeforeSync();
    __syncthreads();
    tc::FenceAfterSync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // Producer: TMA loads of the A (codeword) and B (vector) tiles for each K stage.
        const uint32_t bytes = (kSplit ? 4u : 2u) * kTileBytes;
        int issued = 0;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStages;
            if (kb >= kStages && !tc::MbarWait(&empty[s], ((kb / kStages) - 1) & 1, err, kWaitNs)) break;
            tc::MbarArriveExpectTx(&full[s], bytes);
            tc::TmaLoad2d(tile(s, 0), &ta_hi, &full[s], kb * kTileK, m0);
            tc::TmaLoad2d(tile(s, 2), &tb_hi, &full[s], kb * kTileK, static_cast<int>(n0));
            if (kSplit) {
                tc::TmaLoad2d(tile(s, 1), &ta_lo, &full[s], kb * kTileK, m0);
                tc::TmaLoad2d(tile(s, 3), &tb_lo, &full[s], kb * kTileK, static_cast<int>(n0));
            }
            ++issued;
        }
        // Copies still in flight complete before the CTA may exit (bounded: they always land).
        for (int kb = issued - 1; kb >= 0 && kb >= issued - kStages; --kb)
            tc::MbarWait(&full[kb % kStages], (kb / kStages) & 1, err, kWaitNs, false);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: one thread drives the tensor core.
        const uint32_t idesc = tc::InstrDescTf32(kTile, kTile);
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStages;
            if (!tc::MbarWait(&full[s], (kb / kStages) & 1, err, kWaitNs)) break;
            tc::FenceAfterSync();
            const uint32_t a_hi = tc::SmemAddr(tile(s, 0)), a_lo = tc::SmemAddr(tile(s, 1));
            const uint32_t b_hi = tc::SmemAddr(tile(s, 2)), b_lo = tc::SmemAddr(tile(s, 3));
#pragma unroll
            for (int k = 0; k < kTileK / 8; ++k) {
                const uint32_t off = k * 32;  // 8 tf32 = 32 bytes along the swizzled row
                const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                tc::UmmaTf32(tmem, tc::SmemDescSw128(a_hi + off), tc::SmemDescSw128(b_hi + off), idesc, acc);
                if (kSplit) {
                    tc::UmmaTf32(tmem, tc::SmemDescSw128(a_hi + off), tc::SmemDescSw128(b_lo + off), idesc, 1u);
                    tc::UmmaTf32(tmem, tc::SmemDescSw128(a_lo + off), tc::SmemDescSw128(b_hi + off), idesc, 1u);
                }
            }
            tc::UmmaCommit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        tc::UmmaCommit(accum);
    } else if (warp >= 2) {
        // Epilogue: TMEM lane quarter q (fixed by warp % 4) holds codewords m0 + 32q .. + 31.
        // The warp takes one decision so that the .sync.aligned TMEM loads stay convergent.
        const bool ok = __all_sync(0xffffffffu, tc::MbarWait(accum, 0, err, kWaitNs, false));
        if (ok) {
            tc::FenceAfterSync();
            const int q = warp & 3;
            const int r = m0 + q * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < kTile; c0 += 32) {
                float v[32];
                tc::TmemLoad32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
                if (r < rows) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int64_t col = n0 + c0 + j;
                        if (col < n) out[col * ldo + r] = v[j];
                    }
                }
            }
        }
    }
    tc::FenceBeforeSync();
    __syncthreads();
    if (warp == 1) tc::TmemDealloc(tmem, kTile);
}

__device__ __forceinline__ float RoundTf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// hi = x rounded to TF32, lo = (x - hi) rounded to TF32 (x - hi itself is exact in FP32).
template <typename T>
__global__ void SplitTf32Kernel(const T* __restrict__ x, int64_t count, float* __restrict__ hi, float* __restrict__ lo) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = static_cast<float>(x[i]);
        const float h = RoundTf32(v);
        hi[i] = h;
        if (lo) lo[i] = RoundTf32(__fsub_rn(v, h));
    }
}

// ||x||^2 in the reference's SIMD order (4 lanes, tail into lane 0, lanes summed in order) and in
// double, for the tensor-core modes (the exact GEMM produces both itself).
template <typename T>
__global__ void NormsKernel(const T* __restrict__ X, int64_t n, int d, float* __restrict__ xn, double* __restrict__ xnd) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t vec = t >> 2;
    const int l = static_cast<int>(t & 3);
    const bool ok = vec < n;
    float s = 0.0f;
    double sd = 0.0;
    if (ok) {
        const T* x = X + vec * d;
        const int body = (d / 4) * 4;
        for (int k = l; k < body; k += 4) {
            const float v = static_cast<float>(x[k]);
            s = __fadd_rn(s, __fmul_rn(v, v));
            sd = __dadd_rn(sd, __dmul_rn(static_cast<double>(v), static_cast<double>(v)));
        }
        if (l == 0)
            for (int k = body; k < d; ++k) {
                const float v = static_cast<float>(x[k]);
                s = __fadd_rn(s, __fmul_rn(v, v));
                sd = __dadd_rn(sd, __dmul_rn(static_cast<double>(v), static_cast<double>(v)));
            }
    }
    const float s1 = __shfl_sync(0xffffffffu, s, (threadIdx.x & 31 & ~3) + 1);
    const float s2 = __shfl_sync(0xffffffffu, s, (threadIdx.x & 31 & ~3) + 2);
    const float s3 = __shfl_sync(0xffffffffu, s, (threadIdx.x & 31 & ~3) + 3);
    const double d1 = __shfl_sync(0xffffffffu, sd, (threadIdx.x & 31 & ~3) + 1);
    const double d2 = __shfl_sync(0xffffffffu, sd, (threadIdx.x & 31 & ~3) + 2);
    const double d3 = __shfl_sync(0xffffffffu, sd, (threadIdx.x & 31 & ~3) + 3);
    if (ok && l == 0) {
        if (xn) xn[vec] = __fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3);
        if (xnd) xnd[vec] = (sd + d1) + (d2 + d3);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 EncodeFn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Row-major rows x d fp32 matrix, 128 x 32 boxes, 128-byte swizzle, zero fill out of bounds.
bool MakeMap(CUtensorMap* map, const float* ptr, int64_t rows, int d) {
    auto fn = EncodeFn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d) * sizeof(float)};
    const cuuint32_t box[2] = {kTileK, kTile};
    const cuuint32_t estride[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t TcSmemBytes() { return kStages * 4 * kTileBytes + 1024 + 256; }

cudaError_t LaunchSplitTf32(const void* x, int x_dtype, int64_t count, float* hi, float* lo, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 16));
    if (x_dtype == 0) SplitTf32Kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), count, hi, lo);
    else SplitTf32Kernel<uint8_t><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(x), count, hi, lo);
    return cudaGetLastError();
}

cudaError_t LaunchNorms(const void* X, int x_dtype, int64_t n, int d, float* xn, double* xnd, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int64_t threads = n * 4;
    const int grid = static_cast<int>((threads + 255) / 256);
    if (x_dtype == 0) NormsKernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(X), n, d, xn, xnd);
    else NormsKernel<uint8_t><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(X), n, d, xn, xnd);
    return cudaGetLastError();
}

// out (ldo-strided per vector) = A^T B for A = rows x d (hi/lo) and B = n x d (hi/lo), both
// row-major fp32; split == false uses only the hi parts (1xTF32).
cudaError_t LaunchXcGemmTc(const float* a_hi, const float* a_lo, int rows, const float* b_hi, const float* b_lo,
                           int64_t n, int d, float* out, int ldo, bool split, unsigned int* err, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if ((d % 4) != 0 || (reinterpret_cast<uintptr_t>(a_hi) | reinterpret_cast<uintptr_t>(b_hi)) % 16 != 0)
        return cudaErrorInvalidValue;  // TMA needs 16-byte aligned rows
    if ((n + kTile - 1) / kTile > 65535) return cudaErrorInvalidValue;
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;
    if (!MakeMap(&ta_hi, a_hi, rows, d) || !MakeMap(&tb_hi, b_hi, n, d)) return cudaErrorInvalidValue;
    if (split) {
        if (!MakeMap(&ta_lo, a_lo, rows, d) || !MakeMap(&tb_lo, b_lo, n, d)) return cudaErrorInvalidValue;
    } else {
        ta_lo = ta_hi;
        tb_lo = tb_hi;
    }
    const size_t smem = TcSmemBytes();
    dim3 grid((rows + kTile - 1) / kTile, static_cast<unsigned>((n + kTile - 1) / kTile));
    cudaError_t e;
    if (split) {
        e = cudaFuncSetAttribute(XcGemmTcKernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        XcGemmTcKernel<true><<<grid, kTcThreads, smem, stream>>>(ta_hi, ta_lo, tb_hi, tb_lo, rows, n, d, out, ldo, err);
    } else {
        e = cudaFuncSetAttribute(XcGemmTcKernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        XcGemmTcKernel<false><<<grid, kTcThreads, smem, stream>>>(ta_hi, ta_lo, tb_hi, tb_lo, rows, n, d, out, ldo, err);
    }
    return cudaGetLastError();
}

}  // namespace stlq_b200
