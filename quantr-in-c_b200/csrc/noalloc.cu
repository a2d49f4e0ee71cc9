// noalloc.cu -- quantr_gemv_noalloc_dev: the quantized GEMV without any
// device allocation.
//
// Some callers cannot call cudaMalloc: embedders whose own memory manager owns
// every device allocation, plugin hosts that hand a plugin nothing but its
// input and output buffers, and latency-critical paths that cannot afford the
// implicit device synchronisation and unbounded latency of cudaMalloc/cudaFree.
// quantr_gemv_dev needs a caller-provided workspace for the quantized
// activations; this variant instead uses one fixed scratch array compiled into
// the library (a file-scope __device__ array of QUANTR_NOALLOC_SCRATCH_BYTES),
// which every GPU that loads the library holds until the process exits.
#include "quantr_cuda.h"

#include "formats.cuh"
#include "kernels.cuh"

#include <mutex>

namespace {

using namespace qr;

// Bytes [0, 256) hold the device error word; the quantized activations of the
// current call start at byte 256.
constexpr size_t kErrBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[QUANTR_NOALLOC_SCRATCH_BYTES];

std::mutex g_addr_mu;
void* g_addr[64] = {};

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the real address is looked
// up once per device (with that device current) and cached.
int scratch_address(void** out)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return QUANTR_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return QUANTR_ERR_CUDA;
        }
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return QUANTR_OK;
}

int code_of(cudaError_t e)
{
    if (e == cudaSuccess) return QUANTR_OK;
    cudaGetLastError();
    return e == cudaErrorInvalidConfiguration ? QUANTR_ERR_TOO_LARGE : QUANTR_ERR_CUDA;
}

} // namespace

// Error word of the allocation-free path on the current device, read (and
// optionally cleared) by quantr_gpu_device_status.  Returns DEV_OK when no
// allocation-free call has run on this device yet (the word was never looked
// up, and the array starts zeroed).  Allocates nothing.
int qr::noalloc_device_error(int reset)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return DEV_OK;
    }
    void* p = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_addr_mu);
        p = g_addr[dev];
    }
    if (!p) return DEV_OK;
    int v = DEV_OK;
    if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return DEV_OK;
    }
    if (reset && v != DEV_OK) {
        const int zero = DEV_OK;
        if (cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) cudaGetLastError();
    }
    return v;
}

extern "C" int quantr_gemv_noalloc_dev(float* out, long long ldo, const float* x, long long ldx, const void* w,
                                       uint32_t type, int n, int d, int B, void* stream)
{
    if (n <= 0 || B <= 0) return QUANTR_OK;
    if (!out || !x || !w || d < 0 || ldo < n || ldx < d) return QUANTR_ERR_BAD_ARG;
    if (!type_supported(type)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    if (kErrBytes + actq_bytes(d, B) > QUANTR_NOALLOC_SCRATCH_BYTES) return QUANTR_ERR_TOO_LARGE;
    void* base = nullptr;
    int rc = scratch_address(&base);
    if (rc) return rc;
    int* err = static_cast<int*>(base);
    ActQ a = actq_carve(static_cast<unsigned char*>(base) + kErrBytes, d, B);
    LaunchCfg c;
    c.stream = static_cast<cudaStream_t>(stream);
    // The quantizer overwrites every activation byte the GEMV reads, so
    // nothing left by an earlier call leaks in.  The error word is NOT cleared
    // here: a bounded wait that gave up stays recorded until
    // quantr_gpu_device_status(stream, 1) reads and clears it.
    rc = code_of(launch_quantize(x, ldx, d, B, a, nullptr, nullptr, c));
    if (rc) return rc;
    GemvArgs g;
    g.w = static_cast<const uint8_t*>(w);
    g.type = type;
    g.n = n;
    g.d = d;
    g.x = a;
    g.out = out;
    g.ldo = ldo;
    g.B = B;
    g.err = err;
    return code_of(launch_gemv(g, c));
}
