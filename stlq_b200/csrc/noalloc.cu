// stlq_b200_beam_search_noalloc: the beam-search stage without any device allocation.
//
// The beam search hands vectors whose exact errors tie at a selection boundary from its fast
// kernel to its slot-replay kernel through a scratch list (a count followed by vector ids).  The
// regular entry point keeps that list in memory the encoder allocates on demand.  This variant
// keeps it in a file-scope device array of fixed size instead, so a call allocates nothing.
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../../include/stlq_b200.h"
#include "launch.h"

namespace stlq_b200 {
int GetBeamInputs(const stlq_b200_encoder* enc, BeamInputs* out);
int SetError(int code, const char* msg);
int CheckBeamCall(const stlq_b200_encoder* enc, int64_t n, int beam);
}  // namespace stlq_b200

namespace {

constexpr int kMaxDevices = 64;

// The hand-off list: element 0 is the count, then up to STLQ_B200_NOALLOC_MAX_VECTORS vector ids.
// Every GPU that loads the library holds these 4 MiB until the process exits.  All calls share
// it: each call clears the count before use, and calls whose work overlaps on the GPU race.
static __device__ __align__(256) int g_handoff[STLQ_B200_NOALLOC_MAX_VECTORS + 1];

std::mutex g_setup_mutex;
// The array's device address per device, looked up once.  It stays valid for the process's CUDA
// context on that device: the library does not support resetting a device (cudaDeviceReset) while
// it is loaded, which would leave this address stale.
int* g_handoff_addr[kMaxDevices] = {};

// Once per device, with that device current: the device address of g_handoff (the host-side
// name of the array is only a stand-in, never a device pointer), and every beam kernel variant
// loaded, so that no later call on this device, for any encoder shape, does first-use work.
int SetupDevice(int device) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_handoff_addr[device]) return 0;
    int* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_handoff);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return stlq_b200::SetError(STLQ_B200_ECUDA,
                                   (std::string("cudaGetSymbolAddress(hand-off scratch): ") + cudaGetErrorString(e)).c_str());
    }
    const cudaError_t e2 = stlq_b200::LoadAllBeamKernels();
    if (e2 != cudaSuccess) {
        cudaGetLastError();
        return stlq_b200::SetError(STLQ_B200_ECUDA,
                                   (std::string("loading the beam kernels: ") + cudaGetErrorString(e2)).c_str());
    }
    g_handoff_addr[device] = p;
    return 0;
}

}  // namespace

extern "C" int stlq_b200_beam_search_noalloc(stlq_b200_encoder* enc, const float* xnorm2_dev, const float* xC_dev,
                                             int64_t n, int beam, uint8_t* B_dev, void* stream) {
    stlq_b200::BeamInputs in{};
    if (int rc = stlq_b200::GetBeamInputs(enc, &in)) return rc;
    if (in.dims.wide)
        return stlq_b200::SetError(STLQ_B200_EINVAL,
                                   "stlq_b200_beam_search_noalloc writes uint8 codes; this encoder has a codebook above "
                                   "256 codewords");
    if (n > STLQ_B200_NOALLOC_MAX_VECTORS) {
        const std::string msg = "stlq_b200_beam_search_noalloc: n = " + std::to_string(n) + " exceeds " +
                                std::to_string(STLQ_B200_NOALLOC_MAX_VECTORS) +
                                " vectors, the size of its static scratch; split the call";
        return stlq_b200::SetError(STLQ_B200_EINVAL, msg.c_str());
    }
    // The same checks as stlq_b200_beam_search (n, beam, shared memory for this beam width and
    // these codebooks), with the same EINVAL results.
    if (int rc = stlq_b200::CheckBeamCall(enc, n, beam)) return rc;
    if (n > 0 && (!xnorm2_dev || !xC_dev || !B_dev)) return stlq_b200::SetError(STLQ_B200_EINVAL, "null buffer");
    if (in.device < 0 || in.device >= kMaxDevices) return stlq_b200::SetError(STLQ_B200_EINVAL, "device ordinal too large");
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (cudaSetDevice(in.device) != cudaSuccess) return stlq_b200::SetError(STLQ_B200_ECUDA, "cudaSetDevice failed");
    int rc = SetupDevice(in.device);
    if (rc == 0 && n > 0) {
        const cudaError_t e = stlq_b200::LaunchBeamSearch(in.dims, in.Grow, in.Gdiag, xnorm2_dev, xC_dev, n, beam, B_dev,
                                                          g_handoff_addr[in.device], in.check_filter, in.err_flag,
                                                          in.num_sms, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess)
            rc = stlq_b200::SetError(STLQ_B200_ECUDA, (std::string("beam search launch: ") + cudaGetErrorString(e)).c_str());
    }
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}
