// C-ABI of stlq_b200 (include/stlq_b200.h): encoder handles, device scratch, the slice loop of
// the encode stage, and the pinned double-buffered host path.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/stlq_b200.h"
#include "launch.h"

using stlq_b200::Dims;

namespace {

thread_local std::string g_last_error;

int Fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

#define STLQ_CK(expr)                                                                                \
    do {                                                                                             \
        const cudaError_t e_ = (expr);                                                               \
        if (e_ != cudaSuccess)                                                                       \
            return Fail(e_ == cudaErrorMemoryAllocation ? STLQ_B200_ENOMEM : STLQ_B200_ECUDA,        \
                        std::string(#expr) + ": " + cudaGetErrorString(e_));                         \
    } while (0)

#define STLQ_TRY(expr)              \
    do {                            \
        const int rc_ = (expr);     \
        if (rc_ != 0) return rc_;   \
    } while (0)

// Makes `device` current for the scope and restores the caller's device afterwards.
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

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    int Ensure(size_t need) {
        if (need <= bytes) return 0;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        const cudaError_t e = cudaMalloc(&p, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return Fail(STLQ_B200_ENOMEM, "cudaMalloc(" + std::to_string(need) + " bytes) failed: " +
                                              cudaGetErrorString(e));
        }
        bytes = need;
        return 0;
    }
    void Release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

struct PinBuf {
    void* p = nullptr;
    size_t bytes = 0;
    int Ensure(size_t need) {
        if (need <= bytes) return 0;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        const cudaError_t e = cudaMallocHost(&p, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return Fail(STLQ_B200_ENOMEM, "cudaMallocHost(" + std::to_string(need) + " bytes) failed");
        }
        bytes = need;
        return 0;
    }
    void Release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
    }
};

bool IsPinnedHost(const void* p) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

size_t ElemSize(int x_dtype) { return x_dtype == STLQ_B200_U8 ? 1 : 4; }

// Device flag word (kernels OR error bits into it) followed, at byte 16, by four 64-bit beam
// counters: survivors evaluated exactly, layers, vectors, vectors handed to the replay kernel.
constexpr size_t kFlagBytes = 64;

}  // namespace

struct stlq_b200_encoder {
    int device = 0;
    int num_sms = 148;
    size_t max_block_smem = 232448;  // opt-in dynamic shared memory per block (B200: 227 KB)
    int gemm_mode = STLQ_B200_GEMM_EXACT;
    // Self-check of the beam pre-filter (environment STLQ_B200_CHECK_FILTER=1 at create time):
    // every candidate is also evaluated exactly and a wrongly dropped one raises EDEVICE.
    int check_filter = 0;
    Dims dims{};
    DevBuf C, Gcol, Grow, Gdiag, invnorm, err_flag;
    DevBuf Bdiag;  // the beam's diagonal (LaunchBeamDiag)
    // Tensor-core modes: C_all split into TF32 hi / lo parts once at create; STRICT mode also keeps
    // upper bounds of the codeword norms (its tensor-core error bound is kappa ||c|| ||x||).
    DevBuf Chi, Clo, cn;
    // Input rotation X <- R X (ApplyRotationInPlace), R stored by rows; off when R is the identity.
    DevBuf Rrow;
    bool rotate = false;
    // Per-call scratch, grown on demand and kept for the handle's lifetime.
    DevBuf xC, xn, xnd, partials, orders, redo, Xhi, Xlo, Bfull, Xrot;
    std::vector<int> orders_host;
    int64_t orders_key[4] = {-1, -1, -1, -1};
    // Host path.
    cudaStream_t compute = nullptr, copy = nullptr;
    cudaEvent_t ev_h2d[2] = {}, ev_comp[2] = {}, ev_d2h[2] = {};
    DevBuf xin[2], Bd[2], ad[2], costd[2], sse_d;
    PinBuf pin_in[2], pin_B[2], pin_a[2], pin_cost[2], pin_sse;
};

namespace {

size_t CodeBytes(const stlq_b200_encoder* enc) { return enc->dims.wide ? 2 : 1; }

// The beam's Gram array: the row-major copy, or the large-root encoder's one symmetric array.
const float* BeamGram(const stlq_b200_encoder* enc) {
    return enc->Grow.p ? enc->Grow.as<float>() : enc->Gcol.as<float>();
}

// Vectors per encode slice: bounds the xC scratch (H floats per vector) to ~2 GiB.
int64_t SliceVectors(const stlq_b200_encoder* enc) {
    const int64_t by_mem = (int64_t{1} << 31) / (static_cast<int64_t>(enc->dims.H) * 4);
    return std::max<int64_t>(1024, std::min<int64_t>(by_mem, stlq_b200::MaxGemmSliceVectors()));
}

// One resident wave of refinement CTAs (each warp loops over its vectors), fewer for small n.
int RefineGrid(const stlq_b200_encoder* enc, int64_t n) {
    const int64_t per_block = stlq_b200::RefineWarpsPerBlock();
    const int64_t want = (n + per_block - 1) / per_block;
    const int64_t wave = int64_t{enc->num_sms} * stlq_b200::RefineBlocksPerSm();
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, wave)));
}

int CheckEnc(const stlq_b200_encoder* enc) {
    if (!enc) return Fail(STLQ_B200_EINVAL, "encoder handle is null");
    return 0;
}

int CheckEncodeArgs(const stlq_b200_encoder* enc, int x_dtype, int64_t n, int beam, int icm_iters, int ils_iters,
                    int perturb_k) {
    STLQ_TRY(CheckEnc(enc));
    if (x_dtype != STLQ_B200_F32 && x_dtype != STLQ_B200_U8) return Fail(STLQ_B200_EINVAL, "x_dtype must be F32 or U8");
    if (n < 0) return Fail(STLQ_B200_EINVAL, "n must be >= 0");
    if (beam < 1 || beam > STLQ_B200_MAX_BEAM)
        return Fail(STLQ_B200_EINVAL, "beam must be in [1, " + std::to_string(STLQ_B200_MAX_BEAM) + "]");
    if (icm_iters < 0 || ils_iters < 0 || perturb_k < 0)
        return Fail(STLQ_B200_EINVAL, "icm_iters, ils_iters and perturb_k must be >= 0");
    // The beam kernels keep one float per candidate of a layer (beam x codebook size) in shared
    // memory; every beam <= 32 with codebooks <= 1024 fits a B200's 227 KB.
    if (BeamFastSmemBytes(enc->dims, beam, enc->gemm_mode == STLQ_B200_GEMM_STRICT) > enc->max_block_smem)
        return Fail(STLQ_B200_EINVAL, "beam x (largest codebook) needs more shared memory than a block of this "
                                      "device has");
    return 0;
}

// Entry points with uint8 codes serve encoders whose codebooks have at most 256 codewords; the
// _u16 ones the others.
int CheckCodeWidth(const stlq_b200_encoder* enc, bool wide) {
    STLQ_TRY(CheckEnc(enc));
    if (enc->dims.wide != static_cast<int>(wide))
        return Fail(STLQ_B200_EINVAL, wide ? "this encoder has uint8 codes (codebooks of at most 256 codewords); use "
                                             "the uint8 entry points"
                                           : "this encoder has codebooks above 256 codewords (uint16 codes); use the "
                                             "_u16 entry points");
    return 0;
}

// ICM layer orders exactly as the reference draws them: one std::mt19937(seed) for the whole
// call, `order` reset to iota at each RunIcm call and std::shuffle'd once per ICM iteration
// (icm.cpp:119-122, 239-243, 890-895, 974-975).  Uploaded only when they change.
int UploadOrders(stlq_b200_encoder* enc, int icm_iters, int n_ils, uint32_t seed, cudaStream_t stream) {
    const int m = enc->dims.m;
    const int64_t key[4] = {m, icm_iters, n_ils, static_cast<int64_t>(seed)};
    if (std::equal(key, key + 4, enc->orders_key)) return 0;
    const size_t count = static_cast<size_t>(n_ils + 1) * icm_iters * m;
    enc->orders_host.assign(std::max<size_t>(count, 1), 0);
    std::mt19937 rng(static_cast<std::mt19937::result_type>(seed));
    std::vector<int> order(m);
    size_t w = 0;
    for (int call = 0; call <= n_ils; ++call) {
        std::iota(order.begin(), order.end(), 0);
        for (int it = 0; it < icm_iters; ++it) {
            std::shuffle(order.begin(), order.end(), rng);
            for (int l = 0; l < m; ++l) enc->orders_host[w++] = order[l];
        }
    }
    STLQ_TRY(enc->orders.Ensure(enc->orders_host.size() * sizeof(int)));
    STLQ_CK(cudaMemcpyAsync(enc->orders.p, enc->orders_host.data(), enc->orders_host.size() * sizeof(int),
                            cudaMemcpyHostToDevice, stream));
    STLQ_CK(cudaStreamSynchronize(stream));  // orders_host may change on the next call
    std::copy(key, key + 4, enc->orders_key);
    return 0;
}

bool TensorCoreMode(const stlq_b200_encoder* enc) { return enc->gemm_mode != STLQ_B200_GEMM_EXACT; }

// STRICT mode's bound on |xC_tensor - xC_exact| / (||c|| ||x||): (0.4 d + 16) 2^-24.  Measured on
// B200 at the benchmark shapes (134M entries at d = 128, 67M at d = 96 and d = 960): at most
// 1.3e-6 (d = 128), 7.3e-7 (d = 96), 7.2e-6 (d = 960), i.e. 3.1x, 4.4x and 3.3x below this bound.
// The kernels check the bound on every entry they compute exactly and report kErrTcBound
// (STLQ_B200_EDEVICE) if it is ever exceeded.
float StrictKappa(int d) { return (0.4f * static_cast<float>(d) + 16.0f) * 0x1p-24f; }

// xC (rows x n, ldo-strided per vector) and optional norms for n <= MaxGemmSliceVectors() vectors
// in the encoder's GEMM mode.
int LaunchXc(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int rows, float* out, int ldo, float* xn,
             double* xnd, cudaStream_t stream) {
    const int d = enc->dims.d;
    if (!TensorCoreMode(enc)) {
        STLQ_CK(stlq_b200::LaunchXcGemmExact(enc->C.as<float>(), rows, d, X, x_dtype, n, out, ldo, xn, xnd, stream));
        return 0;
    }
    if (n <= 0) return 0;
    const bool strict = enc->gemm_mode == STLQ_B200_GEMM_STRICT;
    const size_t count = static_cast<size_t>(n) * d;
    STLQ_TRY(enc->Xhi.Ensure(count * sizeof(float)));
    if (strict) STLQ_TRY(enc->Xlo.Ensure(count * sizeof(float)));
    float* xlo = strict ? enc->Xlo.as<float>() : nullptr;
    STLQ_CK(stlq_b200::LaunchSplitTf32(X, x_dtype, static_cast<int64_t>(count), enc->Xhi.as<float>(), xlo, stream));
    STLQ_CK(stlq_b200::LaunchXcGemmTc(enc->Chi.as<float>(), strict ? enc->Clo.as<float>() : nullptr, rows,
                                      enc->Xhi.as<float>(), xlo, n, d, out, ldo, strict, enc->err_flag.as<unsigned int>(),
                                      stream));
    if (xn || xnd) STLQ_CK(stlq_b200::LaunchNorms(X, x_dtype, n, d, xn, xnd, stream));
    return 0;
}

int EnsureScratch(stlq_b200_encoder* enc, int64_t slice) {
    STLQ_TRY(enc->xC.Ensure(static_cast<size_t>(slice) * enc->dims.H * sizeof(float)));
    STLQ_TRY(enc->xn.Ensure(static_cast<size_t>(slice) * sizeof(float)));
    STLQ_TRY(enc->xnd.Ensure(static_cast<size_t>(slice) * sizeof(double)));
    STLQ_TRY(enc->partials.Ensure(static_cast<size_t>(RefineGrid(enc, slice)) * 2 * sizeof(double)));
    STLQ_TRY(enc->redo.Ensure(static_cast<size_t>(slice + 1) * sizeof(int)));
    return 0;
}

// The encode stage on device buffers for n vectors, sliced; sse_dev (2 doubles) accumulates.
int EncodeDevice(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters, int ils_iters,
                 int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset, void* Bv, float* a,
                 float* cost, double* sse_dev, cudaStream_t stream) {
    const Dims& dims = enc->dims;
    char* B = static_cast<char*>(Bv);  // codes of CodeBytes(enc) bytes each
    const size_t cb = CodeBytes(enc);
    const int n_ils = (ils_iters <= 0 || perturb_k <= 0 || dims.m <= 1) ? 0 : ils_iters;
    if (icm_iters > 0) STLQ_TRY(UploadOrders(enc, icm_iters, n_ils, seed, stream));
    const int64_t S = std::min<int64_t>(std::max<int64_t>(n, 1), SliceVectors(enc));
    STLQ_TRY(EnsureScratch(enc, S));
    const size_t esz = ElemSize(x_dtype);
    if (enc->rotate) STLQ_TRY(enc->Xrot.Ensure(static_cast<size_t>(S) * dims.d * sizeof(float)));
    for (int64_t s0 = 0; s0 < n; s0 += S) {
        const int64_t ns = std::min(S, n - s0);
        const void* Xs = static_cast<const char*>(X) + static_cast<size_t>(s0) * dims.d * esz;
        int xt = x_dtype;
        if (enc->rotate) {  // X <- R X as the reference's GemmRaw computes it, then encode the result
            STLQ_CK(stlq_b200::LaunchXcGemmExact(enc->Rrow.as<float>(), dims.d, dims.d, Xs, x_dtype, ns,
                                                 enc->Xrot.as<float>(), dims.d, nullptr, nullptr, stream));
            Xs = enc->Xrot.p;
            xt = STLQ_B200_F32;
        }
        STLQ_TRY(LaunchXc(enc, Xs, xt, ns, dims.H, enc->xC.as<float>(), dims.H, enc->xn.as<float>(),
                          enc->xnd.as<double>(), stream));
        // STRICT: xC is the tensor cores'; the beam and refinement kernels recompute, in the exact
        // GEMM's order, every entry a decision or an output depends on.
        stlq_b200::ExactDotArgs ea{};
        if (enc->gemm_mode == STLQ_B200_GEMM_STRICT)
            ea = stlq_b200::ExactDotArgs{enc->C.as<float>(), Xs, xt, enc->cn.as<float>(), StrictKappa(dims.d)};
        STLQ_CK(stlq_b200::LaunchBeamSearch(dims, BeamGram(enc), enc->Bdiag.as<float>(), enc->xn.as<float>(),
                                            enc->xC.as<float>(), ns, beam, B + s0 * dims.m * cb, enc->redo.as<int>(),
                                            enc->check_filter,
                                            enc->err_flag.as<unsigned int>(), enc->num_sms, stream, &ea));
        if (dims.large_root)  // LS, cost and ICM take the root term from the SIMD-order dot
            STLQ_CK(stlq_b200::LaunchRootDot(dims, enc->C.as<float>(), Xs, xt, B + s0 * dims.m * cb, ns,
                                             enc->xC.as<float>(), stream));
        stlq_b200::RefineArgs ra{};
        ra.dims = dims;
        ra.Gcol = enc->Gcol.as<float>();
        ra.Gdiag = enc->Gdiag.as<float>();
        ra.invnorm = enc->invnorm.as<float>();
        ra.xC = enc->xC.as<float>();
        ra.xnorm2 = enc->xn.as<float>();
        ra.xnorm2_d = enc->xnd.as<double>();
        ra.n = ns;
        ra.mode = 1;
        ra.icm_iters = icm_iters;
        ra.n_ils = n_ils;
        ra.perturb_k = perturb_k;
        ra.use_abs = use_abs;
        ra.seed = seed;
        ra.sample_id_offset = sample_id_offset + static_cast<uint64_t>(s0);
        ra.orders = icm_iters > 0 ? enc->orders.as<int>() : nullptr;
        ra.B = B + s0 * dims.m * cb;
        ra.a = a ? a + s0 * dims.m : nullptr;
        ra.cost = cost ? cost + s0 : nullptr;
        ra.partials = sse_dev ? enc->partials.as<double>() : nullptr;
        ra.ex = ea;
        ra.err_flag = enc->err_flag.as<unsigned int>();
        const int grid = RefineGrid(enc, ns);
        STLQ_CK(stlq_b200::LaunchRefine(ra, grid, stream));
        if (sse_dev) STLQ_CK(stlq_b200::LaunchReducePartials(enc->partials.as<double>(), grid, sse_dev, stream));
    }
    return 0;
}

}  // namespace

namespace stlq_b200 {

// Internal accessors for entry points defined in other translation units.
int GetBeamInputs(const stlq_b200_encoder* enc, BeamInputs* out) {
    if (!enc) return Fail(STLQ_B200_EINVAL, "encoder handle is null");
    out->dims = enc->dims;
    out->Grow = BeamGram(enc);
    out->Gdiag = enc->Bdiag.as<float>();
    out->err_flag = enc->err_flag.as<unsigned int>();
    out->check_filter = enc->check_filter;
    out->num_sms = enc->num_sms;
    out->device = enc->device;
    return 0;
}

int SetError(int code, const char* msg) { return Fail(code, msg); }

// The argument checks of stlq_b200_beam_search (uint8 codes, n, beam, and the beam kernels'
// shared memory for this encoder's codebooks), for entry points in other translation units.
int CheckBeamCall(const stlq_b200_encoder* enc, int64_t n, int beam) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    return CheckEncodeArgs(enc, STLQ_B200_F32, n, beam, 0, 0, 0);
}

}  // namespace stlq_b200

extern "C" {

const char* stlq_b200_last_error(void) { return g_last_error.c_str(); }

const char* stlq_b200_version(void) { return "stlq_b200 0.1.0 sm_100a"; }

}  // extern "C"

namespace {

// Both encoder kinds.  Regular: the full Gram G = C_all^T C_all in both orientations (or the
// caller's G).  Large root (BuildPrecompLargeRoot): only the columns of codebooks 1..m-1, one
// symmetric array, with the root codewords' norms as their diagonal.
int CreateImpl(int device, int d, int m, const int* h_vec, const float* C_all, const float* G, const float* invnorm,
               int gemm_mode, bool large_root, stlq_b200_encoder** out) {
    if (!out) return Fail(STLQ_B200_EINVAL, "out is null");
    *out = nullptr;
    if (!h_vec || !C_all) return Fail(STLQ_B200_EINVAL, "h_vec and C_all must be non-null");
    if (d < 1) return Fail(STLQ_B200_EINVAL, "d must be >= 1");
    if (m < 1 || m > STLQ_B200_MAX_M) return Fail(STLQ_B200_EINVAL, "m must be in [1, 16]");
    if (gemm_mode != STLQ_B200_GEMM_EXACT && gemm_mode != STLQ_B200_GEMM_STRICT && gemm_mode != STLQ_B200_GEMM_FAST)
        return Fail(STLQ_B200_EINVAL, "gemm_mode must be STLQ_B200_GEMM_EXACT, _STRICT or _FAST");
    if (gemm_mode != STLQ_B200_GEMM_EXACT && d % 4 != 0)
        return Fail(STLQ_B200_EINVAL, "gemm_mode STRICT/FAST needs d to be a multiple of 4 (16-byte TMA rows)");
    Dims dims{};
    dims.d = d;
    dims.m = m;
    if (large_root && m < 2)
        return Fail(STLQ_B200_EINVAL, "a large-root encoder needs m >= 2 (a root and at least one small codebook)");
    int H = 0, maxK = 0, maxKs = 1;
    for (int l = 0; l < m; ++l) {
        if (large_root) {
            const int lim = l == 0 ? STLQ_B200_MAX_ROOT : STLQ_B200_MAX_K;
            if (h_vec[l] < 1 || h_vec[l] > lim)
                return Fail(STLQ_B200_EINVAL, "h_vec[" + std::to_string(l) + "] must be in [1, " + std::to_string(lim) +
                                                  "] for a large-root encoder");
        } else if (h_vec[l] < 1 || h_vec[l] > STLQ_B200_MAX_K_WIDE) {
            return Fail(STLQ_B200_EINVAL, "h_vec[" + std::to_string(l) +
                                              "] must be in [1, 1024] (uint8 codes up to 256, uint16 above)");
        }
        dims.h_vec[l] = h_vec[l];
        dims.off[l] = H;
        H += h_vec[l];
        maxK = std::max(maxK, h_vec[l]);
        if (l > 0) maxKs = std::max(maxKs, h_vec[l]);
    }
    dims.H = H;
    dims.maxK = maxK;
    dims.maxKs = maxKs;
    dims.large_root = large_root ? 1 : 0;
    dims.wide = maxK > STLQ_B200_MAX_K;  // large root: only the root can exceed 256
    dims.c0 = large_root ? h_vec[0] : 0;
    dims.ldg = H - dims.c0;
    const int Hs = dims.ldg;
    int ndev = 0;
    STLQ_CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return Fail(STLQ_B200_EINVAL, "device ordinal out of range");
    DeviceScope scope(device);
    if (!scope.ok()) return Fail(STLQ_B200_ECUDA, "cudaSetDevice failed");
    auto* enc = new stlq_b200_encoder();
    enc->device = device;
    enc->dims = dims;
    enc->gemm_mode = gemm_mode;
    if (const char* cf = std::getenv("STLQ_B200_CHECK_FILTER")) enc->check_filter = std::atoi(cf) != 0;
    auto fail = [&](int rc) {
        stlq_b200_destroy(enc);
        return rc;
    };
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) {
        enc->num_sms = prop.multiProcessorCount;
        enc->max_block_smem = prop.sharedMemPerBlockOptin;
    }
    const size_t HH = static_cast<size_t>(H) * Hs;  // Gram entries held
    int rc = 0;
    if ((rc = enc->C.Ensure(sizeof(float) * H * d)) || (rc = enc->Gcol.Ensure(sizeof(float) * HH)) ||
        (!large_root && (rc = enc->Grow.Ensure(sizeof(float) * HH))) || (rc = enc->Gdiag.Ensure(sizeof(float) * H)) ||
        (rc = enc->Bdiag.Ensure(sizeof(float) * H)) || (rc = enc->invnorm.Ensure(sizeof(float) * H)) ||
        (rc = enc->err_flag.Ensure(kFlagBytes)))
        return fail(rc);
    if (cudaStreamCreateWithFlags(&enc->compute, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&enc->copy, cudaStreamNonBlocking) != cudaSuccess)
        return fail(Fail(STLQ_B200_ECUDA, "cudaStreamCreate failed"));
    for (int b = 0; b < 2; ++b) {
        if (cudaEventCreateWithFlags(&enc->ev_h2d[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&enc->ev_comp[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&enc->ev_d2h[b], cudaEventDisableTiming) != cudaSuccess)
            return fail(Fail(STLQ_B200_ECUDA, "cudaEventCreate failed"));
    }
    cudaStream_t s = enc->compute;
    auto ck = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return 0;
        return Fail(STLQ_B200_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
    };
    if ((rc = ck(cudaMemcpyAsync(enc->C.p, C_all, sizeof(float) * H * d, cudaMemcpyDefault, s), "upload C_all")))
        return fail(rc);
    if (large_root) {
        // G(r, h0 + j) = C_all[r] . C_small[j] at Gcol[r * Hs + j], the GEMM's summation order
        // (BuildPrecompLargeRoot's G0S and G_small GEMMs; the products commute).
        rc = ck(stlq_b200::LaunchXcGemmExact(enc->C.as<float>() + static_cast<size_t>(dims.c0) * d, Hs, d, enc->C.p,
                                             STLQ_B200_F32, H, enc->Gcol.as<float>(), Hs, nullptr, nullptr, s),
                "G0S / G_small gemm");
    } else if (G) {
        rc = ck(cudaMemcpyAsync(enc->Gcol.p, G, sizeof(float) * HH, cudaMemcpyDefault, s), "upload G");
    } else {
        // G = C_all^T C_all in the same summation order as xC (BuildPrecomp calls the same Gemm).
        rc = ck(stlq_b200::LaunchXcGemmExact(enc->C.as<float>(), H, d, enc->C.p, STLQ_B200_F32, H, enc->Gcol.as<float>(),
                                             H, nullptr, nullptr, s),
                "G gemm");
    }
    if (rc) return fail(rc);
    if (gemm_mode != STLQ_B200_GEMM_EXACT) {
        const bool strict = gemm_mode == STLQ_B200_GEMM_STRICT;
        if ((rc = enc->Chi.Ensure(sizeof(float) * H * d)) || (strict && (rc = enc->Clo.Ensure(sizeof(float) * H * d))))
            return fail(rc);
        rc = ck(stlq_b200::LaunchSplitTf32(enc->C.p, STLQ_B200_F32, static_cast<int64_t>(H) * d, enc->Chi.as<float>(),
                                           strict ? enc->Clo.as<float>() : nullptr, s),
                "split C_all");
        if (rc) return fail(rc);
        if (strict) {
            if ((rc = enc->cn.Ensure(sizeof(float) * H))) return fail(rc);
            rc = ck(stlq_b200::LaunchNormBounds(enc->C.as<float>(), H, d, enc->cn.as<float>(), s), "codeword norm bounds");
            if (rc) return fail(rc);
        }
    }
    if (large_root) {
        // invnorm and the root norms from the reference's SIMD-order Norm2.
        DevBuf norms;
        if ((rc = norms.Ensure(sizeof(float) * H))) return fail(rc);
        rc = ck(stlq_b200::LaunchNorms(enc->C.p, STLQ_B200_F32, H, d, norms.as<float>(), nullptr, s), "codeword norms");
        if (!rc)
            rc = ck(stlq_b200::LaunchLargeRootPrecomp(norms.as<float>(), dims.c0, H, enc->Gcol.as<float>(),
                                                      enc->Gdiag.as<float>(), enc->invnorm.as<float>(), s),
                    "large-root precompute");
        if (!rc) rc = ck(cudaStreamSynchronize(s), "create sync");
        norms.Release();
        if (rc) return fail(rc);
    } else {
        if (invnorm) {
            rc = ck(cudaMemcpyAsync(enc->invnorm.p, invnorm, sizeof(float) * H, cudaMemcpyDefault, s),
                    "upload invnorm");
        } else {
            rc = ck(stlq_b200::LaunchInvnorm(enc->C.as<float>(), H, d, enc->invnorm.as<float>(), s), "invnorm");
        }
        if (rc) return fail(rc);
        if ((rc = ck(stlq_b200::LaunchTranspose(enc->Gcol.as<float>(), enc->Grow.as<float>(), H, H, s), "transpose G")) ||
            (rc = ck(stlq_b200::LaunchDiag(enc->Gcol.as<float>(), enc->Gdiag.as<float>(), H, s), "diag G")))
            return fail(rc);
    }
    if ((rc = ck(stlq_b200::LaunchBeamDiag(dims, enc->Gcol.as<float>(), enc->Gdiag.as<float>(), enc->Bdiag.as<float>(),
                                           s),
                 "beam diagonal")) ||
        (rc = ck(cudaMemsetAsync(enc->err_flag.p, 0, kFlagBytes, s), "memset")) ||
        (rc = ck(cudaStreamSynchronize(s), "create sync")))
        return fail(rc);
    *out = enc;
    return 0;
}

}  // namespace

extern "C" {

int stlq_b200_create(int device, int d, int m, const int* h_vec, const float* C_all, const float* G,
                     const float* invnorm, int gemm_mode, stlq_b200_encoder** out) {
    return CreateImpl(device, d, m, h_vec, C_all, G, invnorm, gemm_mode, false, out);
}

int stlq_b200_destroy(stlq_b200_encoder* enc) {
    if (!enc) return 0;
    DeviceScope scope(enc->device);
    if (enc->compute) cudaStreamSynchronize(enc->compute);
    if (enc->copy) cudaStreamSynchronize(enc->copy);
    for (DevBuf* b : {&enc->C, &enc->Gcol, &enc->Grow, &enc->Gdiag, &enc->Bdiag, &enc->invnorm, &enc->err_flag, &enc->xC, &enc->xn,
                      &enc->Chi, &enc->Clo, &enc->cn, &enc->Xhi, &enc->Xlo, &enc->Bfull, &enc->Xrot, &enc->Rrow, &enc->xnd, &enc->partials, &enc->orders, &enc->redo, &enc->sse_d})
        b->Release();
    for (int i = 0; i < 2; ++i) {
        enc->xin[i].Release();
        enc->Bd[i].Release();
        enc->ad[i].Release();
        enc->costd[i].Release();
        enc->pin_in[i].Release();
        enc->pin_B[i].Release();
        enc->pin_a[i].Release();
        enc->pin_cost[i].Release();
        if (enc->ev_h2d[i]) cudaEventDestroy(enc->ev_h2d[i]);
        if (enc->ev_comp[i]) cudaEventDestroy(enc->ev_comp[i]);
        if (enc->ev_d2h[i]) cudaEventDestroy(enc->ev_d2h[i]);
    }
    enc->pin_sse.Release();
    if (enc->compute) cudaStreamDestroy(enc->compute);
    if (enc->copy) cudaStreamDestroy(enc->copy);
    delete enc;
    return 0;
}

int stlq_b200_beam_stats(stlq_b200_encoder* enc, uint64_t out[4], int reset) {
    STLQ_TRY(CheckEnc(enc));
    if (!out) return Fail(STLQ_B200_EINVAL, "out is null");
    DeviceScope scope(enc->device);
    STLQ_CK(cudaDeviceSynchronize());
    STLQ_CK(cudaMemcpy(out, static_cast<char*>(enc->err_flag.p) + 16, 4 * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    if (reset) STLQ_CK(cudaMemset(static_cast<char*>(enc->err_flag.p) + 16, 0, 4 * sizeof(uint64_t)));
    return 0;
}

int stlq_b200_dims(const stlq_b200_encoder* enc, int* d, int* m, int* H) {
    STLQ_TRY(CheckEnc(enc));
    if (d) *d = enc->dims.d;
    if (m) *m = enc->dims.m;
    if (H) *H = enc->dims.H;
    return 0;
}

int stlq_b200_sync(stlq_b200_encoder* enc, void* stream) {
    STLQ_TRY(CheckEnc(enc));
    DeviceScope scope(enc->device);
    STLQ_CK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    unsigned int flag = 0;
    STLQ_CK(cudaMemcpy(&flag, enc->err_flag.p, sizeof(flag), cudaMemcpyDeviceToHost));
    if (flag) {
        cudaMemset(enc->err_flag.p, 0, sizeof(flag));
        std::string what;
        if (flag & stlq_b200::kErrSurvivorOverflow) what += " beam-survivor-overflow";
        if (flag & stlq_b200::kErrBadShape) what += " bad-shape";
        if (flag & stlq_b200::kErrFilterMiss) what += " beam-filter-miss";
        if (flag & stlq_b200::kErrWaitTimeout) what += " tensor-core-gemm-wait-timeout";
        if (flag & stlq_b200::kErrTcBound) what += " tensor-core-xc-outside-its-error-bound";
        return Fail(STLQ_B200_EDEVICE, "a kernel reported internal errors:" + what);
    }
    return 0;
}

int stlq_b200_encode_base_device(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, int beam,
                                 int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                 uint64_t sample_id_offset, uint8_t* B_dev, float* a_dev, float* cost_dev,
                                 double* sse_out_dev, void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    STLQ_TRY(CheckEncodeArgs(enc, x_dtype, n, beam, icm_iters, ils_iters, perturb_k));
    if (n > 0 && (!X_dev || !B_dev)) return Fail(STLQ_B200_EINVAL, "X_dev and B_dev must be non-null");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (sse_out_dev) STLQ_CK(cudaMemsetAsync(sse_out_dev, 0, 2 * sizeof(double), s));
    return EncodeDevice(enc, X_dev, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset,
                        B_dev, a_dev, cost_dev, sse_out_dev, s);
}

int stlq_b200_encode_base_device_u16(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, int beam,
                                 int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                 uint64_t sample_id_offset, uint16_t* B_dev, float* a_dev, float* cost_dev,
                                 double* sse_out_dev, void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, true));
    STLQ_TRY(CheckEncodeArgs(enc, x_dtype, n, beam, icm_iters, ils_iters, perturb_k));
    if (n > 0 && (!X_dev || !B_dev)) return Fail(STLQ_B200_EINVAL, "X_dev and B_dev must be non-null");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (sse_out_dev) STLQ_CK(cudaMemsetAsync(sse_out_dev, 0, 2 * sizeof(double), s));
    return EncodeDevice(enc, X_dev, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset,
                        B_dev, a_dev, cost_dev, sse_out_dev, s);
}

}  // extern "C"

namespace {

// The host-buffer stage for codes of CodeBytes(enc) bytes.  Slices of up to `kHostSlice` vectors
// go through two pinned/device buffer pairs: the copy stream carries H2D of slice s+1 and D2H of
// slice s-1 while the compute stream encodes slice s; host staging into pinned memory is skipped
// when the caller's buffers are pinned.
int EncodeHost(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters, int ils_iters,
               int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset, void* B_outv, float* a_out,
               float* cost_out, double* sse_out) {
    STLQ_TRY(CheckEncodeArgs(enc, x_dtype, n, beam, icm_iters, ils_iters, perturb_k));
    char* B_out = static_cast<char*>(B_outv);
    const size_t cb = CodeBytes(enc);
    if (n > 0 && (!X || !B_out)) return Fail(STLQ_B200_EINVAL, "X and B_out must be non-null");
    DeviceScope scope(enc->device);
    const Dims& dims = enc->dims;
    const int64_t kHostSlice = 262144;
    const int64_t S = std::min<int64_t>(std::max<int64_t>(n, 1), kHostSlice);
    const size_t esz = ElemSize(x_dtype);
    const size_t in_bytes = static_cast<size_t>(S) * dims.d * esz;
    const bool pin_x = IsPinnedHost(X);
    const bool pin_B = IsPinnedHost(B_out);
    const bool pin_a = !a_out || IsPinnedHost(a_out);
    const bool pin_c = !cost_out || IsPinnedHost(cost_out);
    for (int b = 0; b < 2; ++b) {
        STLQ_TRY(enc->xin[b].Ensure(in_bytes));
        STLQ_TRY(enc->Bd[b].Ensure(static_cast<size_t>(S) * dims.m * cb));
        STLQ_TRY(enc->ad[b].Ensure(static_cast<size_t>(S) * dims.m * sizeof(float)));
        STLQ_TRY(enc->costd[b].Ensure(static_cast<size_t>(S) * sizeof(float)));
        if (!pin_x) STLQ_TRY(enc->pin_in[b].Ensure(in_bytes));
        if (!pin_B) STLQ_TRY(enc->pin_B[b].Ensure(static_cast<size_t>(S) * dims.m * cb));
        if (!pin_a) STLQ_TRY(enc->pin_a[b].Ensure(static_cast<size_t>(S) * dims.m * sizeof(float)));
        if (!pin_c) STLQ_TRY(enc->pin_cost[b].Ensure(static_cast<size_t>(S) * sizeof(float)));
    }
    STLQ_TRY(enc->sse_d.Ensure(2 * sizeof(double)));
    STLQ_TRY(enc->pin_sse.Ensure(2 * sizeof(double)));
    cudaStream_t cs = enc->compute, ps = enc->copy;
    STLQ_CK(cudaMemsetAsync(enc->sse_d.p, 0, 2 * sizeof(double), cs));
    const int64_t nslices = (n + S - 1) / S;
    std::vector<int64_t> pending;  // slice ids whose outputs still sit in the pinned buffers
    auto drain = [&](int64_t s) -> int {
        const int b = static_cast<int>(s % 2);
        const int64_t s0 = s * S, ns = std::min(S, n - s0);
        STLQ_CK(cudaEventSynchronize(enc->ev_d2h[b]));
        if (!pin_B) std::memcpy(B_out + s0 * dims.m * cb, enc->pin_B[b].p, static_cast<size_t>(ns) * dims.m * cb);
        if (!pin_a) std::memcpy(a_out + s0 * dims.m, enc->pin_a[b].p, static_cast<size_t>(ns) * dims.m * sizeof(float));
        if (!pin_c) std::memcpy(cost_out + s0, enc->pin_cost[b].p, static_cast<size_t>(ns) * sizeof(float));
        return 0;
    };
    for (int64_t s = 0; s < nslices; ++s) {
        const int b = static_cast<int>(s % 2);
        const int64_t s0 = s * S, ns = std::min(S, n - s0);
        if (s >= 2) STLQ_TRY(drain(s - 2));
        const char* src = static_cast<const char*>(X) + static_cast<size_t>(s0) * dims.d * esz;
        const size_t nbytes = static_cast<size_t>(ns) * dims.d * esz;
        if (!pin_x) {
            std::memcpy(enc->pin_in[b].p, src, nbytes);
            src = static_cast<const char*>(enc->pin_in[b].p);
        }
        STLQ_CK(cudaMemcpyAsync(enc->xin[b].p, src, nbytes, cudaMemcpyHostToDevice, ps));
        STLQ_CK(cudaEventRecord(enc->ev_h2d[b], ps));
        STLQ_CK(cudaStreamWaitEvent(cs, enc->ev_h2d[b], 0));
        STLQ_TRY(EncodeDevice(enc, enc->xin[b].p, x_dtype, ns, beam, icm_iters, ils_iters, perturb_k, use_abs, seed,
                              sample_id_offset + static_cast<uint64_t>(s0), enc->Bd[b].p,
                              a_out ? enc->ad[b].as<float>() : nullptr, cost_out ? enc->costd[b].as<float>() : nullptr,
                              sse_out ? enc->sse_d.as<double>() : nullptr, cs));
        STLQ_CK(cudaEventRecord(enc->ev_comp[b], cs));
        STLQ_CK(cudaStreamWaitEvent(ps, enc->ev_comp[b], 0));
        void* dB = pin_B ? static_cast<void*>(B_out + s0 * dims.m * cb) : enc->pin_B[b].p;
        STLQ_CK(cudaMemcpyAsync(dB, enc->Bd[b].p, static_cast<size_t>(ns) * dims.m * cb, cudaMemcpyDeviceToHost, ps));
        if (a_out) {
            void* da = pin_a ? static_cast<void*>(a_out + s0 * dims.m) : enc->pin_a[b].p;
            STLQ_CK(cudaMemcpyAsync(da, enc->ad[b].p, static_cast<size_t>(ns) * dims.m * sizeof(float),
                                    cudaMemcpyDeviceToHost, ps));
        }
        if (cost_out) {
            void* dc = pin_c ? static_cast<void*>(cost_out + s0) : enc->pin_cost[b].p;
            STLQ_CK(cudaMemcpyAsync(dc, enc->costd[b].p, static_cast<size_t>(ns) * sizeof(float), cudaMemcpyDeviceToHost,
                                    ps));
        }
        STLQ_CK(cudaEventRecord(enc->ev_d2h[b], ps));
    }
    for (int64_t s = std::max<int64_t>(0, nslices - 2); s < nslices; ++s) STLQ_TRY(drain(s));
    if (sse_out) {
        STLQ_CK(cudaMemcpyAsync(enc->pin_sse.p, enc->sse_d.p, 2 * sizeof(double), cudaMemcpyDeviceToHost, cs));
        STLQ_CK(cudaStreamSynchronize(cs));
        std::memcpy(sse_out, enc->pin_sse.p, 2 * sizeof(double));
    }
    return stlq_b200_sync(enc, cs);
}

}  // namespace

extern "C" {

int stlq_b200_encode_base(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                          int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                          uint8_t* B_out, float* a_out, float* cost_out, double* sse_out) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    return EncodeHost(enc, X, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset, B_out,
                      a_out, cost_out, sse_out);
}

int stlq_b200_encode_base_u16(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                              int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                              uint16_t* B_out, float* a_out, float* cost_out, double* sse_out) {
    STLQ_TRY(CheckCodeWidth(enc, true));
    return EncodeHost(enc, X, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset, B_out,
                      a_out, cost_out, sse_out);
}

int stlq_b200_create_large_root(int device, int d, int m, const int* h_vec, const float* C_all, int gemm_mode,
                                stlq_b200_encoder** out) {
    return CreateImpl(device, d, m, h_vec, C_all, nullptr, nullptr, gemm_mode, true, out);
}

int stlq_b200_encode_base_large_root(stlq_b200_encoder* enc, const void* X, int x_dtype, int64_t n, int beam,
                                     int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                     uint64_t sample_id_offset, uint32_t* cluster_out, uint8_t* B_small_out,
                                     float* a_out, float* cost_out, double* cost_sums_out) {
    STLQ_TRY(CheckEnc(enc));
    if (!enc->dims.large_root) return Fail(STLQ_B200_EINVAL, "encoder was not created by stlq_b200_create_large_root");
    if (n > 0 && (!cluster_out || !B_small_out)) return Fail(STLQ_B200_EINVAL, "cluster_out and B_small_out must be non-null");
    const int m = enc->dims.m;
    const bool wide = enc->dims.wide != 0;  // root codes above 255 are held as uint16
    std::vector<uint8_t> B(static_cast<size_t>(std::max<int64_t>(n, 0)) * m * CodeBytes(enc));
    STLQ_TRY(EncodeHost(enc, X, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset,
                        B.data(), a_out, cost_out, cost_sums_out));
    const uint16_t* B16 = reinterpret_cast<const uint16_t*>(B.data());
    for (int64_t v = 0; v < n; ++v) {
        const size_t o = static_cast<size_t>(v) * m;
        cluster_out[v] = wide ? B16[o] : B[o];
        for (int l = 1; l < m; ++l)
            B_small_out[v * (m - 1) + l - 1] = static_cast<uint8_t>(wide ? B16[o + l] : B[o + l]);
    }
    return 0;
}

int stlq_b200_encode_base_large_root_device(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n,
                                            int beam, int icm_iters, int ils_iters, int perturb_k, int use_abs,
                                            uint32_t seed, uint64_t sample_id_offset, uint32_t* cluster_dev,
                                            uint8_t* B_small_dev, float* a_dev, float* cost_dev,
                                            double* cost_sums_dev, void* stream) {
    STLQ_TRY(CheckEncodeArgs(enc, x_dtype, n, beam, icm_iters, ils_iters, perturb_k));
    if (!enc->dims.large_root) return Fail(STLQ_B200_EINVAL, "encoder was not created by stlq_b200_create_large_root");
    if (n > 0 && (!X_dev || !cluster_dev || !B_small_dev))
        return Fail(STLQ_B200_EINVAL, "X_dev, cluster_dev and B_small_dev must be non-null");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n <= 0) return 0;
    STLQ_TRY(enc->Bfull.Ensure(static_cast<size_t>(n) * enc->dims.m * CodeBytes(enc)));
    if (cost_sums_dev) STLQ_CK(cudaMemsetAsync(cost_sums_dev, 0, 2 * sizeof(double), s));
    STLQ_TRY(EncodeDevice(enc, X_dev, x_dtype, n, beam, icm_iters, ils_iters, perturb_k, use_abs, seed,
                          sample_id_offset, enc->Bfull.p, a_dev, cost_dev, cost_sums_dev, s));
    STLQ_CK(stlq_b200::LaunchSplitRootCodes(enc->dims.m, enc->Bfull.p, enc->dims.wide, n, cluster_dev, B_small_dev, s));
    return 0;
}

int stlq_b200_set_rotation(stlq_b200_encoder* enc, const float* R) {
    STLQ_TRY(CheckEnc(enc));
    const int d = enc->dims.d;
    bool identity = true;
    if (R) {
        for (int c = 0; c < d && identity; ++c)
            for (int r = 0; r < d; ++r)
                if (R[static_cast<size_t>(c) * d + r] != (r == c ? 1.0f : 0.0f)) {
                    identity = false;
                    break;
                }
    }
    DeviceScope scope(enc->device);
    STLQ_CK(cudaStreamSynchronize(enc->compute));
    enc->rotate = false;
    if (!R || identity) return 0;  // IsIdentityRotation: the reference skips the product
    std::vector<float> rows(static_cast<size_t>(d) * d);
    for (int i = 0; i < d; ++i)
        for (int k = 0; k < d; ++k) rows[static_cast<size_t>(i) * d + k] = R[static_cast<size_t>(k) * d + i];
    STLQ_TRY(enc->Rrow.Ensure(rows.size() * sizeof(float)));
    STLQ_CK(cudaMemcpy(enc->Rrow.p, rows.data(), rows.size() * sizeof(float), cudaMemcpyHostToDevice));
    enc->rotate = true;
    return 0;
}

int stlq_b200_rotate(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* out_dev, void* stream) {
    STLQ_TRY(CheckEnc(enc));
    if (x_dtype != STLQ_B200_F32 && x_dtype != STLQ_B200_U8) return Fail(STLQ_B200_EINVAL, "x_dtype must be F32 or U8");
    if (n > 0 && (!X_dev || !out_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int d = enc->dims.d;
    const size_t esz = ElemSize(x_dtype);
    const int64_t S = stlq_b200::MaxGemmSliceVectors();
    for (int64_t s0 = 0; s0 < n; s0 += S) {
        const int64_t ns = std::min(S, n - s0);
        const void* Xs = static_cast<const char*>(X_dev) + static_cast<size_t>(s0) * d * esz;
        if (enc->rotate) {
            STLQ_CK(stlq_b200::LaunchXcGemmExact(enc->Rrow.as<float>(), d, d, Xs, x_dtype, ns, out_dev + s0 * d, d,
                                                 nullptr, nullptr, s));
        } else if (x_dtype == STLQ_B200_F32) {
            STLQ_CK(cudaMemcpyAsync(out_dev + s0 * d, Xs, sizeof(float) * ns * d, cudaMemcpyDeviceToDevice, s));
        } else {  // identity: the u8 -> f32 conversion alone
            STLQ_CK(stlq_b200::LaunchU8ToF32(static_cast<const uint8_t*>(Xs), ns * d, out_dev + s0 * d, s));
        }
    }
    return 0;
}

int stlq_b200_xc_gemm(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* xC_dev, void* stream) {
    STLQ_TRY(CheckEnc(enc));
    if (n > 0 && (!X_dev || !xC_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    const int64_t S = stlq_b200::MaxGemmSliceVectors();
    const size_t esz = ElemSize(x_dtype);
    for (int64_t s0 = 0; s0 < n; s0 += S) {
        const int64_t ns = std::min(S, n - s0);
        STLQ_TRY(LaunchXc(enc, static_cast<const char*>(X_dev) + static_cast<size_t>(s0) * enc->dims.d * esz, x_dtype,
                          ns, enc->dims.H, xC_dev + s0 * enc->dims.H, enc->dims.H, nullptr, nullptr,
                          static_cast<cudaStream_t>(stream)));
    }
    return 0;
}

int stlq_b200_xnorm2(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, int64_t n, float* xnorm2_dev,
                     void* stream) {
    STLQ_TRY(CheckEnc(enc));
    if (n > 0 && (!X_dev || !xnorm2_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    STLQ_CK(stlq_b200::LaunchNorms(X_dev, x_dtype, n, enc->dims.d, xnorm2_dev, nullptr,
                                   static_cast<cudaStream_t>(stream)));
    return 0;
}

int stlq_b200_beam_search(stlq_b200_encoder* enc, const float* xnorm2_dev, const float* xC_dev, int64_t n, int beam,
                          uint8_t* B_dev, void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    STLQ_TRY(CheckEncodeArgs(enc, STLQ_B200_F32, n, beam, 0, 0, 0));
    if (n > 0 && (!xnorm2_dev || !xC_dev || !B_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    STLQ_TRY(enc->redo.Ensure(static_cast<size_t>(n + 1) * sizeof(int)));
    STLQ_CK(stlq_b200::LaunchBeamSearch(enc->dims, BeamGram(enc), enc->Bdiag.as<float>(), xnorm2_dev, xC_dev, n,
                                        beam, B_dev, enc->redo.as<int>(), enc->check_filter, enc->err_flag.as<unsigned int>(), enc->num_sms,
                                        static_cast<cudaStream_t>(stream)));
    return 0;
}

int stlq_b200_solve_ls(stlq_b200_encoder* enc, const float* xC_dev, const uint8_t* B_dev, int64_t n, float* a_dev,
                       void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    STLQ_TRY(CheckEnc(enc));
    if (n > 0 && (!xC_dev || !B_dev || !a_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    stlq_b200::RefineArgs ra{};
    ra.dims = enc->dims;
    ra.Gcol = enc->Gcol.as<float>();
    ra.Gdiag = enc->Gdiag.as<float>();
    ra.invnorm = enc->invnorm.as<float>();
    ra.xC = xC_dev;
    ra.n = n;
    ra.mode = 0;
    ra.B = const_cast<uint8_t*>(B_dev);  // read only in mode 0
    ra.a = a_dev;
    STLQ_CK(stlq_b200::LaunchRefine(ra, RefineGrid(enc, n), static_cast<cudaStream_t>(stream)));
    return 0;
}

int stlq_b200_icm(stlq_b200_encoder* enc, const float* xC_dev, const float* xnorm2_dev, int64_t n, int icm_iters,
                  int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset, uint8_t* B_dev,
                  float* a_dev, float* cost_dev, void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    STLQ_TRY(CheckEncodeArgs(enc, STLQ_B200_F32, n, 1, icm_iters, ils_iters, perturb_k));
    if (n > 0 && (!xC_dev || !xnorm2_dev || !B_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int n_ils = (ils_iters <= 0 || perturb_k <= 0 || enc->dims.m <= 1) ? 0 : ils_iters;
    if (icm_iters > 0) STLQ_TRY(UploadOrders(enc, icm_iters, n_ils, seed, s));
    stlq_b200::RefineArgs ra{};
    ra.dims = enc->dims;
    ra.Gcol = enc->Gcol.as<float>();
    ra.Gdiag = enc->Gdiag.as<float>();
    ra.invnorm = enc->invnorm.as<float>();
    ra.xC = xC_dev;
    ra.xnorm2 = xnorm2_dev;
    ra.n = n;
    ra.mode = 1;
    ra.icm_iters = icm_iters;
    ra.n_ils = n_ils;
    ra.perturb_k = perturb_k;
    ra.use_abs = use_abs;
    ra.seed = seed;
    ra.sample_id_offset = sample_id_offset;
    ra.orders = icm_iters > 0 ? enc->orders.as<int>() : nullptr;
    ra.B = B_dev;
    ra.a = a_dev;
    ra.cost = cost_dev;
    STLQ_CK(stlq_b200::LaunchRefine(ra, RefineGrid(enc, n), s));
    return 0;
}

int stlq_b200_sse(stlq_b200_encoder* enc, const void* X_dev, int x_dtype, const float* xC_dev, const uint8_t* B_dev,
                  const float* a_dev, int64_t n, double* sse_dev, void* stream) {
    STLQ_TRY(CheckCodeWidth(enc, false));
    STLQ_TRY(CheckEnc(enc));
    if (n > 0 && (!X_dev || !xC_dev || !B_dev || !a_dev || !sse_dev)) return Fail(STLQ_B200_EINVAL, "null buffer");
    DeviceScope scope(enc->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t S = std::min<int64_t>(std::max<int64_t>(n, 1), stlq_b200::MaxGemmSliceVectors());
    STLQ_TRY(enc->xnd.Ensure(static_cast<size_t>(S) * sizeof(double)));
    const int grid = static_cast<int>(std::min<int64_t>((S + 255) / 256, int64_t{enc->num_sms} * 8));
    STLQ_TRY(enc->partials.Ensure(static_cast<size_t>(grid) * 2 * sizeof(double)));
    const size_t esz = ElemSize(x_dtype);
    for (int64_t s0 = 0; s0 < n; s0 += S) {
        const int64_t ns = std::min(S, n - s0);
        STLQ_CK(stlq_b200::LaunchNorms(static_cast<const char*>(X_dev) + static_cast<size_t>(s0) * enc->dims.d * esz,
                                       x_dtype, ns, enc->dims.d, nullptr, enc->xnd.as<double>(), s));
        const int g = static_cast<int>(std::min<int64_t>((ns + 255) / 256, grid));
        STLQ_CK(stlq_b200::LaunchSse(enc->dims, enc->Gcol.as<float>(), enc->Gdiag.as<float>(), xC_dev + s0 * enc->dims.H, enc->xnd.as<double>(),
                                     B_dev + s0 * enc->dims.m, a_dev + s0 * enc->dims.m, ns, enc->partials.as<double>(),
                                     g, s));
        STLQ_CK(stlq_b200::LaunchReducePartials(enc->partials.as<double>(), g, sse_dev, s));
    }
    return 0;
}

}  // extern "C"

namespace stlq_b200 {

// For the multi-GPU entry points (sharded.cpp): the encoder's device-side sums of the last
// host-buffer encode (2 doubles, written on its compute stream) and that stream.
double* EncoderSseDevice(stlq_b200_encoder* enc) { return enc ? enc->sse_d.as<double>() : nullptr; }
cudaStream_t EncoderStream(stlq_b200_encoder* enc) { return enc ? enc->compute : nullptr; }

// For the block loop (pipeline.cpp): the encoder's device, dimension, codebooks and kind.
void EncoderShape(const stlq_b200_encoder* enc, int* device, int* d, int* m, int* large_root) {
    *device = enc->device;
    *d = enc->dims.d;
    *m = enc->dims.m;
    *large_root = enc->dims.large_root;
}

}  // namespace stlq_b200
