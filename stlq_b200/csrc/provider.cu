// Device primitives of the kernel-provider seam (the reference's StreamKernelProvider,
// include/stlq/core/kernel_provider.h:28-221): a general column-major sgemm with the reference
// BLAS's summation order, uint8 -> float conversion of a strided tile, and per-column argmax.
// The C++ provider class (stlq_b200/adapter/stlq_b200_kernels.cpp) builds the host-matrix interface
// on top of these.
#include <algorithm>
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "../../include/stlq_b200.h"
#include "launch.h"

namespace stlq_b200 {
int SetError(int code, const char* msg);
cudaError_t LaunchSgemmExact(const float* A, int64_t lda, int rows, int k, const float* B, int64_t ldb, int64_t n,
                             float alpha, float beta, float* out, int ldo, cudaStream_t stream);
}  // namespace stlq_b200

namespace {

// out[i * k + kk] = in[i + kk * ld]: the rows of a column-major (rows x k) matrix made contiguous.
__global__ void RowsContiguousKernel(const float* __restrict__ in, int64_t ld, int rows, int k,
                                     float* __restrict__ out) {
    __shared__ float tile[32][33];
    const int i0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int kk = k0 + j, i = i0 + threadIdx.x;
        if (i < rows && kk < k) tile[j][threadIdx.x] = in[i + static_cast<int64_t>(kk) * ld];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int i = i0 + j, kk = k0 + threadIdx.x;
        if (i < rows && kk < k) out[static_cast<int64_t>(i) * k + kk] = tile[threadIdx.x][j];
    }
}

// C = beta * C (C not read when beta is 0): BLAS's result when k is 0 or alpha is 0.
__global__ void ScaleKernel(float* C, int64_t ldc, int m, int64_t n, float beta) {
    const int64_t total = static_cast<int64_t>(m) * n;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = t / m;
        const int i = static_cast<int>(t - j * m);
        float* p = C + j * ldc + i;
        *p = beta == 0.0f ? 0.0f : __fmul_rn(beta, *p);
    }
}

__global__ void U8ToF32StridedKernel(const uint8_t* __restrict__ in, int64_t ld_in, int rows, int64_t cols,
                                     float* __restrict__ out) {
    const int64_t total = static_cast<int64_t>(rows) * cols;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = t / rows;
        const int r = static_cast<int>(t - c * rows);
        out[t] = static_cast<float>(in[c * ld_in + r]);
    }
}

// One warp per column: the first row holding the column's maximum (ties to the smaller row; NaN
// never wins; a column with no value above -inf gives row 0 and -inf), as ArgmaxColsF32 defines it.
__global__ void ArgmaxColsKernel(const float* __restrict__ scores, int64_t ld, int rows, int64_t cols,
                                 int* __restrict__ idx, float* __restrict__ val) {
    const int lane = threadIdx.x & 31;
    const int64_t c = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= cols) return;
    const float* col = scores + c * ld;
    float best = -__int_as_float(0x7f800000);
    int bi = 0;
    for (int r = lane; r < rows; r += 32) {
        const float v = col[r];
        if (v > best) {  // rows increase along a lane: the first maximum stays
            best = v;
            bi = r;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_down_sync(0xffffffffu, best, o);
        const int oi = __shfl_down_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
            best = ob;
            bi = oi;
        }
    }
    if (lane == 0) {
        if (idx) idx[c] = bi;
        if (val) val[c] = best;
    }
}

int Ck(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    cudaGetLastError();
    return stlq_b200::SetError(e == cudaErrorMemoryAllocation ? STLQ_B200_ENOMEM : STLQ_B200_ECUDA,
                               (std::string(what) + ": " + cudaGetErrorString(e)).c_str());
}

struct Scratch {
    void* p = nullptr;
    size_t bytes = 0;
    int Ensure(size_t need) {
        if (need <= bytes) return 0;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        if (int rc = Ck(cudaMalloc(&p, need), "cudaMalloc (kernel-provider scratch)")) return rc;
        bytes = need;
        return 0;
    }
    void Release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
};

class DeviceScope {
public:
    explicit DeviceScope(int device) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        ok_ = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceScope() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }
    bool ok() const { return ok_; }

private:
    int prev_ = -1;
    bool ok_ = false;
};

int GridFor(int64_t total) { return static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 32)); }

}  // namespace

struct stlq_b200_kernels {
    int device = 0;
    Scratch At, Bt;  // op(A) rows / op(B) columns made contiguous when the operand layout needs it
};

extern "C" {

int stlq_b200_kernels_create(int device, stlq_b200_kernels** out) {
    if (!out) return stlq_b200::SetError(STLQ_B200_EINVAL, "out is null");
    *out = nullptr;
    int ndev = 0;
    if (int rc = Ck(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount")) return rc;
    if (device < 0 || device >= ndev) return stlq_b200::SetError(STLQ_B200_EINVAL, "device ordinal out of range");
    auto* k = new stlq_b200_kernels();
    k->device = device;
    *out = k;
    return 0;
}

int stlq_b200_kernels_destroy(stlq_b200_kernels* k) {
    if (!k) return 0;
    DeviceScope scope(k->device);
    k->At.Release();
    k->Bt.Release();
    delete k;
    return 0;
}

int stlq_b200_sgemm(stlq_b200_kernels* kp, int trans_a, int trans_b, int m, int n, int k, float alpha, const float* A,
                    int lda, const float* B, int ldb, float beta, float* C, int ldc, void* stream) {
    if (!kp) return stlq_b200::SetError(STLQ_B200_EINVAL, "kernel-provider handle is null");
    if (m < 0 || n < 0 || k < 0) return stlq_b200::SetError(STLQ_B200_EINVAL, "m, n and k must be >= 0");
    const int a_rows = trans_a ? k : m, b_rows = trans_b ? n : k;
    if (lda < std::max(1, a_rows) || ldb < std::max(1, b_rows) || ldc < std::max(1, m))
        return stlq_b200::SetError(STLQ_B200_EINVAL, "lda, ldb or ldc below the operand's row count");
    if (m == 0 || n == 0) return 0;
    if (!C || (k > 0 && alpha != 0.0f && (!A || !B)))
        return stlq_b200::SetError(STLQ_B200_EINVAL, "null matrix pointer");
    DeviceScope scope(kp->device);
    if (!scope.ok()) return stlq_b200::SetError(STLQ_B200_ECUDA, "cudaSetDevice failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (k == 0 || alpha == 0.0f) {
        ScaleKernel<<<GridFor(static_cast<int64_t>(m) * n), 256, 0, s>>>(C, ldc, m, n, beta);
        return Ck(cudaGetLastError(), "sgemm scale");
    }
    // The GEMM kernel reads op(A) by rows and op(B) by columns, each contiguous over k.
    const float* Ar = A;
    int64_t ar_ld = lda;
    if (!trans_a) {  // op(A) = A (m x k): its rows are strided; make them contiguous
        if (int rc = kp->At.Ensure(sizeof(float) * static_cast<size_t>(m) * k)) return rc;
        dim3 grid((m + 31) / 32, (k + 31) / 32), block(32, 8);
        RowsContiguousKernel<<<grid, block, 0, s>>>(A, lda, m, k, static_cast<float*>(kp->At.p));
        if (int rc = Ck(cudaGetLastError(), "sgemm op(A)")) return rc;
        Ar = static_cast<const float*>(kp->At.p);
        ar_ld = k;
    }
    const float* Bc = B;
    int64_t bc_ld = ldb;
    if (trans_b) {  // op(B) = B^T (k x n) with B (n x k): B's rows are op(B)'s columns
        if (int rc = kp->Bt.Ensure(sizeof(float) * static_cast<size_t>(n) * k)) return rc;
        dim3 grid((n + 31) / 32, (k + 31) / 32), block(32, 8);
        RowsContiguousKernel<<<grid, block, 0, s>>>(B, ldb, n, k, static_cast<float*>(kp->Bt.p));
        if (int rc = Ck(cudaGetLastError(), "sgemm op(B)")) return rc;
        Bc = static_cast<const float*>(kp->Bt.p);
        bc_ld = k;
    }
    return Ck(stlq_b200::LaunchSgemmExact(Ar, ar_ld, m, k, Bc, bc_ld, n, alpha, beta, C, ldc, s), "sgemm");
}

int stlq_b200_u8_to_f32(stlq_b200_kernels* kp, const uint8_t* in, int ld_in, int rows, int64_t cols, float* out,
                        void* stream) {
    if (!kp) return stlq_b200::SetError(STLQ_B200_EINVAL, "kernel-provider handle is null");
    if (rows < 0 || cols < 0 || ld_in < std::max(1, rows))
        return stlq_b200::SetError(STLQ_B200_EINVAL, "rows, cols >= 0 and ld_in >= rows required");
    if (rows == 0 || cols == 0) return 0;
    if (!in || !out) return stlq_b200::SetError(STLQ_B200_EINVAL, "null pointer");
    DeviceScope scope(kp->device);
    U8ToF32StridedKernel<<<GridFor(static_cast<int64_t>(rows) * cols), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        in, ld_in, rows, cols, out);
    return Ck(cudaGetLastError(), "u8_to_f32");
}

int stlq_b200_argmax_cols(stlq_b200_kernels* kp, const float* scores, int ld, int rows, int64_t cols, int* idx,
                          float* val, void* stream) {
    if (!kp) return stlq_b200::SetError(STLQ_B200_EINVAL, "kernel-provider handle is null");
    if (rows < 0 || cols < 0 || ld < std::max(1, rows))
        return stlq_b200::SetError(STLQ_B200_EINVAL, "rows, cols >= 0 and ld >= rows required");
    if (cols == 0) return 0;
    if (!scores && rows > 0) return stlq_b200::SetError(STLQ_B200_EINVAL, "null scores");
    DeviceScope scope(kp->device);
    const int per_block = 8;  // warps
    const int64_t blocks = (cols + per_block - 1) / per_block;
    if (blocks > 0x7fffffff) return stlq_b200::SetError(STLQ_B200_EINVAL, "too many columns");
    ArgmaxColsKernel<<<static_cast<unsigned>(blocks), 32 * per_block, 0, static_cast<cudaStream_t>(stream)>>>(
        scores, ld, rows, cols, idx, val);
    return Ck(cudaGetLastError(), "argmax_cols");
}

}  // extern "C"
