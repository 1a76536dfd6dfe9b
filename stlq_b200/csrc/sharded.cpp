// Single-process multi-GPU encode: one encoder per device, contiguous shards of the base vectors,
// one host thread per device.  The reference encodes on one GPU; here base vectors are independent,
// so the only data that crosses GPUs are the frozen codebooks (one NCCL broadcast from the first
// device, over NVLink) and the per-shard MSE sums (one NCCL reduce onto the first device).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2) by the first sharded call: the library has
// no link-time NCCL dependency, and in a process that already holds an NCCL (torch's, say) that
// same copy is used.  Every wait on a collective is bounded; on expiry the communicators are
// aborted and the call returns STLQ_B200_EDEVICE.
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/stlq_b200.h"

namespace stlq_b200 {
int SetError(int code, const char* msg);
double* EncoderSseDevice(stlq_b200_encoder* enc);
cudaStream_t EncoderStream(stlq_b200_encoder* enc);
}  // namespace stlq_b200

namespace {

using stlq_b200::SetError;

// The NCCL entry points used here, resolved from the loaded library.
struct NcclApi {
    decltype(&ncclCommInitAll) CommInitAll = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclCommAbort) CommAbort = nullptr;
    decltype(&ncclBroadcast) Broadcast = nullptr;
    decltype(&ncclReduce) Reduce = nullptr;
    decltype(&ncclGroupStart) GroupStart = nullptr;
    decltype(&ncclGroupEnd) GroupEnd = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    std::string error;  // why NCCL could not be loaded ("" when it was)
};

const NcclApi& Nccl() {
    static const NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            a.error = std::string("cannot load NCCL (libnccl.so.2): ") + (e ? e : "unknown error");
            return a;
        }
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p && a.error.empty()) a.error = std::string("NCCL lacks ") + name;
            return p;
        };
        a.CommInitAll = reinterpret_cast<decltype(a.CommInitAll)>(sym("ncclCommInitAll"));
        a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
        a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(sym("ncclCommAbort"));
        a.Broadcast = reinterpret_cast<decltype(a.Broadcast)>(sym("ncclBroadcast"));
        a.Reduce = reinterpret_cast<decltype(a.Reduce)>(sym("ncclReduce"));
        a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(sym("ncclGroupStart"));
        a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(sym("ncclGroupEnd"));
        a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
        return a;
    }();
    return api;
}

int NcclFail(ncclResult_t r, const char* what) {
    return SetError(STLQ_B200_ECUDA, (std::string(what) + ": " + Nccl().GetErrorString(r)).c_str());
}

// Collectives on these streams must finish within this many seconds (they move at most the
// codebooks, a few hundred MB at the largest shapes, between GPUs of one node).
constexpr double kCollectiveTimeoutS = 120.0;

// Waits for every stream (streams[i] on devices[i]) with a deadline; on expiry the communicators
// are aborted (which ends the stuck collectives) and EDEVICE is returned.
int WaitStreams(const std::vector<int>& devices, const std::vector<cudaStream_t>& streams,
                std::vector<ncclComm_t>& comms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (size_t i = 0; i < streams.size(); ++i) {
        cudaSetDevice(devices[i]);
        for (;;) {
            const cudaError_t q = cudaStreamQuery(streams[i]);
            if (q == cudaSuccess) break;
            if (q != cudaErrorNotReady)
                return SetError(STLQ_B200_ECUDA, (std::string("collective stream: ") + cudaGetErrorString(q)).c_str());
            const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            if (s > kCollectiveTimeoutS) {
                for (auto& c : comms)
                    if (c) Nccl().CommAbort(c);
                comms.assign(comms.size(), nullptr);
                return SetError(STLQ_B200_EDEVICE, "an NCCL collective did not finish within its time limit; the "
                                                   "communicators were aborted");
            }
            std::this_thread::sleep_for(std::chrono::microseconds(200));
        }
    }
    return 0;
}

// Runs fn(i) on one host thread per device; returns the first failure with its message (the
// message lives in the failing thread's last-error slot and is carried over here).
template <class Fn>
int OnEachDevice(int n, Fn fn) {
    std::vector<int> rc(n, 0);
    std::vector<std::string> msg(n);
    std::vector<std::thread> th;
    th.reserve(n);
    for (int i = 0; i < n; ++i)
        th.emplace_back([&, i] {
            rc[i] = fn(i);
            if (rc[i]) msg[i] = stlq_b200_last_error();
        });
    for (auto& t : th) t.join();
    for (int i = 0; i < n; ++i)
        if (rc[i]) return SetError(rc[i], ("device " + std::to_string(i) + ": " + msg[i]).c_str());
    return 0;
}

}  // namespace

struct stlq_b200_sharded {
    std::vector<int> devices;
    std::vector<stlq_b200_encoder*> enc;
    std::vector<ncclComm_t> comms;
    double* sse_root = nullptr;  // the reduced sums, on devices[0]
    int d = 0, m = 0;
    bool large_root = false;
};

namespace {

int CheckSharded(const stlq_b200_sharded* sh) {
    if (!sh) return SetError(STLQ_B200_EINVAL, "sharded encoder handle is null");
    if (sh->comms.empty() || !sh->comms[0]) return SetError(STLQ_B200_EDEVICE, "the sharded encoder's communicators were aborted");
    return 0;
}

// Shard i of n vectors over k devices: contiguous, the first n % k shards one vector larger.
void ShardRange(int64_t n, int k, int i, int64_t* start, int64_t* count) {
    const int64_t base = n / k, extra = n % k;
    *start = i * base + std::min<int64_t>(i, extra);
    *count = base + (i < extra ? 1 : 0);
}

int CreateSharded(int n_devices, const int* devices, int d, int m, const int* h_vec, const float* C_all,
                  const float* G, const float* invnorm, int gemm_mode, bool large_root, stlq_b200_sharded** out) {
    if (!out) return SetError(STLQ_B200_EINVAL, "out is null");
    *out = nullptr;
    if (n_devices < 1 || !devices) return SetError(STLQ_B200_EINVAL, "n_devices must be >= 1 with a device list");
    if (!h_vec || !C_all || d < 1 || m < 1 || m > STLQ_B200_MAX_M)
        return SetError(STLQ_B200_EINVAL, "d, m, h_vec and C_all must describe a codebook set");
    for (int i = 0; i < n_devices; ++i)
        for (int j = 0; j < i; ++j)
            if (devices[j] == devices[i]) return SetError(STLQ_B200_EINVAL, "devices must be distinct");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess) {
        cudaGetLastError();
        return SetError(STLQ_B200_ECUDA, "no CUDA device");
    }
    for (int i = 0; i < n_devices; ++i)
        if (devices[i] < 0 || devices[i] >= ndev) return SetError(STLQ_B200_EINVAL, "device ordinal out of range");
    const NcclApi& nc = Nccl();
    if (!nc.error.empty()) return SetError(STLQ_B200_ECUDA, nc.error.c_str());
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    auto* sh = new stlq_b200_sharded();
    sh->devices.assign(devices, devices + n_devices);
    sh->d = d;
    sh->m = m;
    sh->large_root = large_root;
    sh->enc.assign(n_devices, nullptr);
    sh->comms.assign(n_devices, nullptr);
    auto fail = [&](int rc) {
        stlq_b200_sharded_destroy(sh);
        if (prev >= 0) cudaSetDevice(prev);
        return rc;
    };
    ncclResult_t r = nc.CommInitAll(sh->comms.data(), n_devices, sh->devices.data());
    if (r != ncclSuccess) {
        sh->comms.assign(n_devices, nullptr);
        return fail(NcclFail(r, "ncclCommInitAll"));
    }
    // The codebook set (C_all, then G and invnorm when given) in one buffer per device, filled on
    // devices[0] from the host and broadcast to the others.
    int64_t H = 0;
    for (int l = 0; l < m; ++l) H += h_vec[l];
    const bool with_g = G && !large_root, with_inv = invnorm && !large_root;
    const size_t nc_all = static_cast<size_t>(H) * d, ng = with_g ? static_cast<size_t>(H) * H : 0,
                 ninv = with_inv ? static_cast<size_t>(H) : 0, count = nc_all + ng + ninv;
    std::vector<float*> buf(n_devices, nullptr);
    std::vector<cudaStream_t> st(n_devices, nullptr);
    auto release = [&] {
        for (int i = 0; i < n_devices; ++i) {
            cudaSetDevice(sh->devices[i]);
            if (st[i]) cudaStreamDestroy(st[i]);
            if (buf[i]) cudaFree(buf[i]);
        }
    };
    for (int i = 0; i < n_devices; ++i) {
        cudaSetDevice(sh->devices[i]);
        if (cudaMalloc(&buf[i], count * sizeof(float)) != cudaSuccess ||
            cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            release();
            return fail(SetError(STLQ_B200_ENOMEM, "codebook broadcast buffers"));
        }
    }
    cudaSetDevice(sh->devices[0]);
    cudaError_t ce = cudaMemcpy(buf[0], C_all, nc_all * sizeof(float), cudaMemcpyDefault);
    if (ce == cudaSuccess && with_g) ce = cudaMemcpy(buf[0] + nc_all, G, ng * sizeof(float), cudaMemcpyDefault);
    if (ce == cudaSuccess && with_inv)
        ce = cudaMemcpy(buf[0] + nc_all + ng, invnorm, ninv * sizeof(float), cudaMemcpyDefault);
    if (ce != cudaSuccess) {
        cudaGetLastError();
        release();
        return fail(SetError(STLQ_B200_ECUDA, (std::string("codebook upload: ") + cudaGetErrorString(ce)).c_str()));
    }
    nc.GroupStart();
    for (int i = 0; i < n_devices && r == ncclSuccess; ++i)
        r = nc.Broadcast(buf[0], buf[i], count, ncclFloat32, 0, sh->comms[i], st[i]);
    const ncclResult_t rg = nc.GroupEnd();
    if (r != ncclSuccess || rg != ncclSuccess) {
        release();
        return fail(NcclFail(r != ncclSuccess ? r : rg, "ncclBroadcast of the codebooks"));
    }
    if (int rc = WaitStreams(sh->devices, st, sh->comms)) {
        release();
        return fail(rc);
    }
    // Every device builds its encoder (Gram matrix and all) from its replica, in parallel.
    int rc = OnEachDevice(n_devices, [&](int i) {
        const float* Cd = buf[i];
        if (large_root) return stlq_b200_create_large_root(sh->devices[i], d, m, h_vec, Cd, gemm_mode, &sh->enc[i]);
        return stlq_b200_create(sh->devices[i], d, m, h_vec, Cd, with_g ? Cd + nc_all : nullptr,
                                with_inv ? Cd + nc_all + ng : nullptr, gemm_mode, &sh->enc[i]);
    });
    release();
    if (rc) return fail(rc);
    cudaSetDevice(sh->devices[0]);
    if (cudaMalloc(&sh->sse_root, 2 * sizeof(double)) != cudaSuccess) {
        cudaGetLastError();
        return fail(SetError(STLQ_B200_ENOMEM, "reduce buffer"));
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = sh;
    return 0;
}

// The per-shard sums (each encoder's device-side pair, left by its last host-buffer encode) summed
// onto devices[0] by one NCCL reduce, then copied to sse_out.
int ReduceSums(stlq_b200_sharded* sh, double* sse_out) {
    const NcclApi& nc = Nccl();
    const int k = static_cast<int>(sh->devices.size());
    std::vector<cudaStream_t> st(k);
    ncclResult_t r = ncclSuccess;
    nc.GroupStart();
    for (int i = 0; i < k && r == ncclSuccess; ++i) {
        st[i] = stlq_b200::EncoderStream(sh->enc[i]);
        r = nc.Reduce(stlq_b200::EncoderSseDevice(sh->enc[i]), sh->sse_root, 2, ncclFloat64, ncclSum, 0, sh->comms[i],
                      st[i]);
    }
    const ncclResult_t rg = nc.GroupEnd();
    if (r != ncclSuccess || rg != ncclSuccess) return NcclFail(r != ncclSuccess ? r : rg, "ncclReduce of the MSE sums");
    if (int rc = WaitStreams(sh->devices, st, sh->comms)) return rc;
    cudaSetDevice(sh->devices[0]);
    const cudaError_t e = cudaMemcpy(sse_out, sh->sse_root, 2 * sizeof(double), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return SetError(STLQ_B200_ECUDA, cudaGetErrorString(e));
    return 0;
}

// Shared by the regular, uint16 and large-root entry points: `encode(i, start, count, sums)` encodes
// shard i on device i (its host thread) into the caller's outputs at `start`.
template <class Encode>
int EncodeShards(stlq_b200_sharded* sh, int64_t n, double* sse_out, Encode encode) {
    if (int rc = CheckSharded(sh)) return rc;
    if (n < 0) return SetError(STLQ_B200_EINVAL, "n must be >= 0");
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    const int k = static_cast<int>(sh->devices.size());
    int rc = OnEachDevice(k, [&](int i) {
        int64_t start = 0, count = 0;
        ShardRange(n, k, i, &start, &count);
        double sums[2] = {0.0, 0.0};  // also makes the encoder accumulate its device-side sums
        return encode(i, start, count, sums);
    });
    if (!rc && sse_out) rc = ReduceSums(sh, sse_out);
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

size_t ElemBytes(int x_dtype) { return x_dtype == STLQ_B200_U8 ? 1 : 4; }

}  // namespace

extern "C" {

int stlq_b200_sharded_create(int n_devices, const int* devices, int d, int m, const int* h_vec, const float* C_all,
                             const float* G, const float* invnorm, int gemm_mode, stlq_b200_sharded** out) {
    return CreateSharded(n_devices, devices, d, m, h_vec, C_all, G, invnorm, gemm_mode, false, out);
}

int stlq_b200_sharded_create_large_root(int n_devices, const int* devices, int d, int m, const int* h_vec,
                                        const float* C_all, int gemm_mode, stlq_b200_sharded** out) {
    return CreateSharded(n_devices, devices, d, m, h_vec, C_all, nullptr, nullptr, gemm_mode, true, out);
}

int stlq_b200_sharded_destroy(stlq_b200_sharded* sh) {
    if (!sh) return 0;
    for (auto* e : sh->enc)
        if (e) stlq_b200_destroy(e);
    for (auto& c : sh->comms)
        if (c) Nccl().CommDestroy(c);
    if (sh->sse_root) {
        cudaSetDevice(sh->devices[0]);
        cudaFree(sh->sse_root);
    }
    delete sh;
    return 0;
}

int stlq_b200_sharded_encoder(stlq_b200_sharded* sh, int i, stlq_b200_encoder** out) {
    if (!sh || !out || i < 0 || i >= static_cast<int>(sh->enc.size()))
        return SetError(STLQ_B200_EINVAL, "sharded encoder handle, index or out invalid");
    *out = sh->enc[i];
    return 0;
}

int stlq_b200_encode_sharded(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam, int icm_iters,
                             int ils_iters, int perturb_k, int use_abs, uint32_t seed, uint64_t sample_id_offset,
                             uint8_t* B_out, float* a_out, float* cost_out, double* sse_out) {
    if (sh && n > 0 && (!X || !B_out)) return SetError(STLQ_B200_EINVAL, "X and B_out must be non-null");
    return EncodeShards(sh, n, sse_out, [&](int i, int64_t s0, int64_t ns, double* sums) {
        const size_t m = sh->m;
        return stlq_b200_encode_base(sh->enc[i], static_cast<const char*>(X) + s0 * sh->d * ElemBytes(x_dtype), x_dtype,
                                     ns, beam, icm_iters, ils_iters, perturb_k, use_abs, seed, sample_id_offset + s0,
                                     B_out + s0 * m, a_out ? a_out + s0 * m : nullptr, cost_out ? cost_out + s0 : nullptr,
                                     sums);
    });
}

int stlq_b200_encode_sharded_u16(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam,
                                 int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                 uint64_t sample_id_offset, uint16_t* B_out, float* a_out, float* cost_out,
                                 double* sse_out) {
    if (sh && n > 0 && (!X || !B_out)) return SetError(STLQ_B200_EINVAL, "X and B_out must be non-null");
    return EncodeShards(sh, n, sse_out, [&](int i, int64_t s0, int64_t ns, double* sums) {
        const size_t m = sh->m;
        return stlq_b200_encode_base_u16(sh->enc[i], static_cast<const char*>(X) + s0 * sh->d * ElemBytes(x_dtype),
                                         x_dtype, ns, beam, icm_iters, ils_iters, perturb_k, use_abs, seed,
                                         sample_id_offset + s0, B_out + s0 * m, a_out ? a_out + s0 * m : nullptr,
                                         cost_out ? cost_out + s0 : nullptr, sums);
    });
}

int stlq_b200_encode_sharded_large_root(stlq_b200_sharded* sh, const void* X, int x_dtype, int64_t n, int beam,
                                        int icm_iters, int ils_iters, int perturb_k, int use_abs, uint32_t seed,
                                        uint64_t sample_id_offset, uint32_t* cluster_out, uint8_t* B_small_out,
                                        float* a_out, float* cost_out, double* cost_sums_out) {
    if (sh && !sh->large_root)
        return SetError(STLQ_B200_EINVAL, "sharded encoder was not created by stlq_b200_sharded_create_large_root");
    if (sh && n > 0 && (!X || !cluster_out || !B_small_out))
        return SetError(STLQ_B200_EINVAL, "X, cluster_out and B_small_out must be non-null");
    return EncodeShards(sh, n, cost_sums_out, [&](int i, int64_t s0, int64_t ns, double* sums) {
        const size_t m = sh->m;
        return stlq_b200_encode_base_large_root(
            sh->enc[i], static_cast<const char*>(X) + s0 * sh->d * ElemBytes(x_dtype), x_dtype, ns, beam, icm_iters,
            ils_iters, perturb_k, use_abs, seed, sample_id_offset + s0, cluster_out + s0, B_small_out + s0 * (m - 1),
            a_out ? a_out + s0 * m : nullptr, cost_out ? cost_out + s0 : nullptr, sums);
    });
}

}  // extern "C"
