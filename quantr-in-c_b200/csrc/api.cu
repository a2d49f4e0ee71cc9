// api.cu -- C ABI of libquantr_cuda.so (declared in include/quantr_cuda.h).
//
// Part 1 (reference-compatible, host pointers, synchronous) keeps the
// reference's contracts (src/quant.c:441-523): NULL weights or any failure give
// a zero-filled `out`, nothing aborts, and the first failure is kept as a
// sticky code.  Part 2 is the stream-ordered device API.
#include "quantr_cuda.h"

#include "formats.cuh"
#include "kernels.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

namespace {

using namespace qr;

struct Region {
    size_t bytes;
    uint8_t* dev;
};

// One context serves the Part 1 calls (the reference calls them from one host
// thread; the mutex only makes concurrent misuse safe, not parallel).
struct Ctx {
    bool ready = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    void* ws = nullptr;  // quantized-activation workspace
    size_t ws_bytes = 0;
    uint8_t* dbuf = nullptr;  // device staging: x | out+err | blocks | unregistered weights
    size_t dbuf_bytes = 0;
    uint8_t* hbuf = nullptr;      // pinned, device-mapped host staging (x | out | err | blocks)
    uint8_t* hbuf_dev = nullptr;  // the same memory as seen by kernels
    size_t hbuf_bytes = 0;
    std::map<uintptr_t, Region> regions;  // keyed by host start address
};

std::recursive_mutex g_mu;
Ctx g;
int g_err = QUANTR_OK;
bool g_warned = false;

// Per-device error word for the device API.
int* g_dev_err[64] = {};

void set_err(int code)
{
    if (code == QUANTR_OK) return;
    if (g_err == QUANTR_OK) g_err = code;
    if (!g_warned) {
        g_warned = true;
        std::fprintf(stderr, "[quantr_cuda] error %d: %s\n", code, quantr_gpu_error_string(code));
    }
}

int code_of(cudaError_t e)
{
    if (e == cudaSuccess) return QUANTR_OK;
    if (e == cudaErrorMemoryAllocation) return QUANTR_ERR_OOM;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || e == cudaErrorInvalidDevice)
        return QUANTR_ERR_NO_DEVICE;
    if (e == cudaErrorInvalidConfiguration) return QUANTR_ERR_TOO_LARGE;
    return QUANTR_ERR_CUDA;
}

// Device error word value -> QUANTR_* code.
int dev_code(int v)
{
    if (v == DEV_OK) return QUANTR_OK;
    if (v == DEV_ERR_ROUTING) return QUANTR_ERR_ROUTING;
    return QUANTR_ERR_DEVICE_TIMEOUT;
}

size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

int ensure_ready()
{
    if (g.ready) return QUANTR_OK;
    int dev = 0;
    if (const char* s = std::getenv("QUANTR_DEVICE")) dev = std::atoi(s);
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        cudaGetLastError();
        return QUANTR_ERR_NO_DEVICE;
    }
    if (dev < 0 || dev >= count) return QUANTR_ERR_NO_DEVICE;
    cudaError_t e = cudaSetDevice(dev);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return code_of(e);
    g.device = dev;
    g.ready = true;
    return QUANTR_OK;
}

int grow_dev(void** p, size_t* cap, size_t need)
{
    if (*cap >= need) return QUANTR_OK;
    if (*p) {
        cudaStreamSynchronize(g.stream);
        cudaFree(*p);
        *p = nullptr;
        *cap = 0;
    }
    size_t sz = std::max(need, (size_t)1 << 20);
    if (cudaMalloc(p, sz) != cudaSuccess) {
        cudaGetLastError();
        return QUANTR_ERR_OOM;
    }
    *cap = sz;
    return QUANTR_OK;
}

// Pinned, device-mapped host staging: kernels read x and write out and the
// error word through it directly (zero-copy), so a Part 1 call issues no
// copy operations of its own - only its kernels and one synchronisation.
int grow_host(size_t need)
{
    if (g.hbuf_bytes >= need) return QUANTR_OK;
    if (g.hbuf) {
        cudaStreamSynchronize(g.stream);
        cudaFreeHost(g.hbuf);
        g.hbuf = nullptr;
        g.hbuf_dev = nullptr;
        g.hbuf_bytes = 0;
    }
    size_t sz = std::max(need, (size_t)1 << 20);
    if (cudaHostAlloc((void**)&g.hbuf, sz, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        g.hbuf = nullptr;
        return QUANTR_ERR_OOM;
    }
    if (cudaHostGetDevicePointer((void**)&g.hbuf_dev, g.hbuf, 0) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(g.hbuf);
        g.hbuf = nullptr;
        return QUANTR_ERR_CUDA;
    }
    g.hbuf_bytes = sz;
    return QUANTR_OK;
}

// Host-side read of a word the device wrote into mapped staging.
int read_mapped_int(const uint8_t* p) { return *reinterpret_cast<const volatile int*>(p); }
void write_mapped_int(uint8_t* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// Device copy of [host, host+len) if a registered region covers it.
const uint8_t* lookup(const void* host, size_t len)
{
    const uintptr_t h = (uintptr_t)host;
    auto it = g.regions.upper_bound(h);
    if (it == g.regions.begin()) return nullptr;
    --it;
    if (h + len > it->first + it->second.bytes) return nullptr;
    return it->second.dev + (h - it->first);
}

// Device layout of one Part 1 call's staging buffer.
struct Stage {
    size_t x_off, out_off, err_off, blk_off, w_off, total;
};

Stage plan(size_t xbytes, size_t obytes, size_t blkbytes, size_t wbytes)
{
    Stage s{};
    s.x_off = 0;
    s.out_off = a256(xbytes);
    s.err_off = s.out_off + ((obytes + 15) & ~size_t(15));
    s.blk_off = a256(s.err_off + 16);
    s.w_off = a256(s.blk_off + blkbytes);
    s.total = s.w_off + a256(wbytes);
    return s;
}

void zero_out(float* out, size_t count)
{
    if (out && count) std::memset(out, 0, count * sizeof(float));
}

// Shared body of matmul_q_fused / matmul_q_fused_batch.
int fused_host(float* out, const float* x, const void* w, uint32_t type, int n, int d, int B)
{
    if (n <= 0 || B <= 0) return QUANTR_OK;
    if (!out || !x || d < 0) return QUANTR_ERR_BAD_ARG;
    if (type != T_F32 && !type_supported(type)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    int rc = ensure_ready();
    if (rc) return rc;
    const size_t xbytes = (size_t)B * d * 4, obytes = (size_t)B * n * 4;
    const size_t wbytes = (size_t)n * (size_t)row_bytes(type, d);
    const uint8_t* wdev = lookup(w, wbytes);
    Stage st = plan(xbytes, obytes, 0, 0);
    if (!wdev && (rc = grow_dev((void**)&g.dbuf, &g.dbuf_bytes, a256(wbytes)))) return rc;
    if ((rc = grow_host(st.err_off + 16))) return rc;
    const size_t need_ws = quantr_gemv_workspace_bytes(d, B);
    if (type != T_F32 && (rc = grow_dev(&g.ws, &g.ws_bytes, need_ws))) return rc;

    // x, out and the error word live in mapped pinned staging.
    const float* dx = (const float*)(g.hbuf_dev + st.x_off);
    float* dout = (float*)(g.hbuf_dev + st.out_off);
    int* derr = (int*)(g.hbuf_dev + st.err_off);
    std::memcpy(g.hbuf + st.x_off, x, xbytes);
    write_mapped_int(g.hbuf + st.err_off, 0);
    cudaError_t e = cudaSuccess;
    if (!wdev) {  // unregistered weights: copy this call's rows up
        wdev = g.dbuf;
        e = cudaMemcpyAsync((void*)wdev, w, wbytes, cudaMemcpyHostToDevice, g.stream);
    }
    LaunchCfg c;
    c.stream = g.stream;
    if (e == cudaSuccess) {
        if (type == T_F32) {
            e = launch_gemv_f32((const float*)wdev, dx, d, dout, n, n, d, B, c);
        } else {
            e = launch_gemv_tc(wdev, type, n, d, B, dx, d, dout, n, derr, g.stream);  // 2+ tokens
            if (e == cudaErrorNotSupported)
                e = launch_gemv_engine(wdev, type, n, d, B, dx, d, dout, n, g.ws, g.ws_bytes, derr, g.stream);
            if (e == cudaErrorNotSupported) {  // shapes the engine does not take
                ActQ a = actq_carve(g.ws, d, B);
                e = launch_quantize(dx, d, d, B, a, nullptr, derr, c);
                GemvArgs ga;
                ga.w = wdev;
                ga.type = type;
                ga.n = n;
                ga.d = d;
                ga.x = a;
                ga.out = dout;
                ga.ldo = n;
                ga.B = B;
                ga.err = derr;
                if (e == cudaSuccess) e = launch_gemv(ga, c);
            }
        }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return code_of(e);
    }
    if (read_mapped_int(g.hbuf + st.err_off)) return QUANTR_ERR_DEVICE_TIMEOUT;
    std::memcpy(out, g.hbuf + st.out_off, obytes);
    return QUANTR_OK;
}

// Runs one GEMV row against pre-quantized activation blocks (vec_dot_*).
float vec_dot_host(const void* a, const void* b, int k, uint32_t type)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (k <= 0 || row_bytes(type, k) == 0) return 0.0f;
    if (!a || !b) {
        set_err(QUANTR_ERR_BAD_ARG);
        return 0.0f;
    }
    int rc = ensure_ready();
    const size_t wbytes = (size_t)row_bytes(type, k);
    const int nbx = k / 32;
    const size_t blkbytes = (size_t)nbx * 34;
    Stage st = plan(0, 4, blkbytes, 0);
    if (!rc) rc = grow_dev((void**)&g.dbuf, &g.dbuf_bytes, a256(wbytes));
    if (!rc) rc = grow_host(st.total);
    if (!rc) rc = grow_dev(&g.ws, &g.ws_bytes, actq_bytes(k, 1));
    if (rc) {
        set_err(rc);
        return 0.0f;
    }
    // Activation blocks, result and error word in mapped staging; the weight
    // row goes to device memory (the GEMV streams weights with bulk copies).
    const uint8_t* dblk = g.hbuf_dev + st.blk_off;
    uint8_t* dw = g.dbuf;
    float* dout = (float*)(g.hbuf_dev + st.out_off);
    int* derr = (int*)(g.hbuf_dev + st.err_off);
    std::memcpy(g.hbuf + st.blk_off, b, blkbytes);
    write_mapped_int(g.hbuf + st.err_off, 0);
    cudaError_t e = cudaMemcpyAsync(dw, a, wbytes, cudaMemcpyHostToDevice, g.stream);
    LaunchCfg c;
    c.stream = g.stream;
    ActQ act = actq_carve(g.ws, k, 1);
    if (e == cudaSuccess) e = launch_repack(dblk, nbx, 1, act, c);
    GemvArgs ga;
    ga.w = dw;
    ga.type = type;
    ga.n = 1;
    ga.d = k;
    ga.x = act;
    ga.out = dout;
    ga.ldo = 1;
    ga.B = 1;
    ga.err = derr;
    if (e == cudaSuccess) e = launch_gemv(ga, c);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_err(code_of(e));
        return 0.0f;
    }
    if (read_mapped_int(g.hbuf + st.err_off)) {
        set_err(QUANTR_ERR_DEVICE_TIMEOUT);
        return 0.0f;
    }
    float r;
    std::memcpy(&r, g.hbuf + st.out_off, 4);
    return r;
}

} // namespace

int* qr::device_error_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!g_dev_err[dev]) {
        int* p = nullptr;
        if (cudaMalloc(&p, 16) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        cudaMemset(p, 0, 16);
        g_dev_err[dev] = p;
    }
    return g_dev_err[dev];
}

extern "C" {

// ------------------------------------------------------------------ errors --

int quantr_gpu_last_error(void) { return g_err; }

void quantr_gpu_clear_error(void)
{
    g_err = QUANTR_OK;
    g_warned = false;
}

const char* quantr_gpu_error_string(int code)
{
    switch (code) {
    case QUANTR_OK: return "ok";
    case QUANTR_ERR_CUDA: return "CUDA runtime call failed";
    case QUANTR_ERR_NO_DEVICE: return "no usable CUDA device";
    case QUANTR_ERR_BAD_ARG: return "invalid argument";
    case QUANTR_ERR_UNSUPPORTED_TYPE: return "unsupported quantization type";
    case QUANTR_ERR_OOM: return "allocation failed";
    case QUANTR_ERR_DEVICE_TIMEOUT: return "bounded in-kernel wait timed out";
    case QUANTR_ERR_TOO_LARGE: return "shape exceeds a kernel limit";
    case QUANTR_ERR_WORKSPACE: return "workspace too small";
    case QUANTR_ERR_ROUTING: return "router probabilities not finite for some token";
    case QUANTR_ERR_UNREGISTERED: return "weights not registered with quantr_gpu_register_weights";
    default: return "unknown error";
    }
}

// ------------------------------------------------------------- lifecycle --

int quantr_gpu_init(int device)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (g.ready) return g.device == device ? QUANTR_OK : QUANTR_ERR_BAD_ARG;
    char buf[16];
    std::snprintf(buf, sizeof buf, "%d", device);
    setenv("QUANTR_DEVICE", buf, 1);
    int rc = ensure_ready();
    if (rc) set_err(rc);
    return rc;
}

void quantr_gpu_shutdown(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!g.ready) return;
    cudaStreamSynchronize(g.stream);
    for (auto& kv : g.regions) cudaFree(kv.second.dev);
    g.regions.clear();
    if (g.ws) cudaFree(g.ws);
    if (g.dbuf) cudaFree(g.dbuf);
    if (g.hbuf) cudaFreeHost(g.hbuf);
    cudaStreamDestroy(g.stream);
    g = Ctx{};
}

uint64_t quantr_gpu_launch_count(void) { return (uint64_t)launch_count(); }

// --------------------------------------------------------------- registry --

int quantr_gpu_register_weights(const void* host, size_t bytes)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!host || bytes == 0) return QUANTR_ERR_BAD_ARG;
    int rc = ensure_ready();
    if (rc) return rc;
    const uintptr_t h = (uintptr_t)host;
    auto it = g.regions.lower_bound(h);
    if (it != g.regions.end() && it->first < h + bytes) return QUANTR_ERR_BAD_ARG;
    if (it != g.regions.begin()) {
        auto pv = std::prev(it);
        if (pv->first + pv->second.bytes > h) return QUANTR_ERR_BAD_ARG;
    }
    uint8_t* dev = nullptr;
    // 16 spare bytes keep every bulk-copy window of the last row in bounds.
    if (cudaMalloc((void**)&dev, bytes + 16) != cudaSuccess) {
        cudaGetLastError();
        return QUANTR_ERR_OOM;
    }
    cudaError_t e = cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(dev);
        cudaGetLastError();
        return code_of(e);
    }
    g.regions[h] = Region{bytes, dev};
    return QUANTR_OK;
}

int quantr_gpu_unregister_weights(const void* host)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    auto it = g.regions.find((uintptr_t)host);
    if (it == g.regions.end()) return QUANTR_ERR_BAD_ARG;
    cudaStreamSynchronize(g.stream);
    cudaFree(it->second.dev);
    g.regions.erase(it);
    return QUANTR_OK;
}

void* quantr_gpu_device_ptr(const void* host)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    return (void*)lookup(host, 1);
}

// ------------------------------------------------- reference entry points --

void matmul_q_fused(float* out, const float* x, const void* w, uint32_t type, int n, int d, int threads)
{
    (void)threads;
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (n <= 0) return;
    if (!w) {  // src/quant.c:443-446
        zero_out(out, (size_t)n);
        return;
    }
    int rc = fused_host(out, x, w, type, n, d, 1);
    if (rc) {
        set_err(rc);
        zero_out(out, (size_t)n);
    }
}

void matmul_q_fused_batch(float* out, const float* x, const void* w, uint32_t type, int n, int d, int B)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (n <= 0 || B <= 0) return;
    if (!w) {
        zero_out(out, (size_t)n * B);
        return;
    }
    int rc = fused_host(out, x, w, type, n, d, B);
    if (rc) {
        set_err(rc);
        zero_out(out, (size_t)n * B);
    }
}

void quantize_row_q8_0(const float* x, block_q8_0* y, int k)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    const int nbx = k / 32;
    if (nbx <= 0) return;
    if (!x || !y) {
        set_err(QUANTR_ERR_BAD_ARG);
        return;
    }
    const size_t xbytes = (size_t)nbx * 32 * 4, blkbytes = (size_t)nbx * 34;
    Stage st = plan(xbytes, 0, blkbytes, 0);
    int rc = ensure_ready();
    if (!rc) rc = grow_host(st.total);
    if (rc) {
        set_err(rc);
        std::memset(y, 0, blkbytes);
        return;
    }
    // Zero-copy: the quantizer reads x from and writes the packed blocks to
    // mapped pinned staging (no activation workspace needed: blocks only).
    std::memcpy(g.hbuf + st.x_off, x, xbytes);
    LaunchCfg c;
    c.stream = g.stream;
    ActQ none{};
    cudaError_t e = launch_quantize((const float*)(g.hbuf_dev + st.x_off), k, k, 1, none, g.hbuf_dev + st.blk_off,
                                    nullptr, c);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_err(code_of(e));
        std::memset(y, 0, blkbytes);
        return;
    }
    std::memcpy(y, g.hbuf + st.blk_off, blkbytes);
}

void dequantize_row(float* out, const void* src, uint32_t type, int n)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (n <= 0) return;
    if (!src) {  // src/quant.c:161-164
        zero_out(out, (size_t)n);
        return;
    }
    if (type == T_F32) {  // src/quant.c:165-168: a plain copy, no arithmetic
        std::memcpy(out, src, (size_t)n * 4);
        return;
    }
    if (!type_supported(type)) {  // src/quant.c:239
        zero_out(out, (size_t)n);
        return;
    }
    // The reference decodes whole blocks only and leaves out[] past the last
    // block untouched (src/quant.c:171-177, :182-194): so does this call.
    const int done = (n / block_elems(type)) * block_elems(type);
    if (done == 0) return;
    const size_t sbytes = (size_t)row_bytes(type, n), obytes = (size_t)done * 4;
    Stage st = plan(0, obytes, 0, sbytes);
    int rc = ensure_ready();
    if (!rc) rc = grow_host(st.w_off + sbytes);
    if (rc) {
        set_err(rc);
        zero_out(out, (size_t)done);
        return;
    }
    // Zero-copy: the kernel reads the packed row from and writes the floats
    // to mapped pinned staging.
    std::memcpy(g.hbuf + st.w_off, src, sbytes);
    LaunchCfg c;
    c.stream = g.stream;
    cudaError_t e = launch_dequantize((float*)(g.hbuf_dev + st.out_off), g.hbuf_dev + st.w_off, type, n, c);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_err(code_of(e));
        zero_out(out, (size_t)done);
        return;
    }
    std::memcpy(out, g.hbuf + st.out_off, obytes);
}

float vec_dot_q8_0_q8_0(const block_q8_0* a, const block_q8_0* b, int k) { return vec_dot_host(a, b, k, T_Q8_0); }
float vec_dot_q4K_q8_0(const block_q4_K* a, const block_q8_0* b, int k) { return vec_dot_host(a, b, k, T_Q4_K); }
float vec_dot_q5K_q8_0(const block_q5_K* a, const block_q8_0* b, int k) { return vec_dot_host(a, b, k, T_Q5_K); }
float vec_dot_q6K_q8_0(const void* a, const block_q8_0* b, int k) { return vec_dot_host(a, b, k, T_Q6_K); }

// ------------------------------------------------------------- device API --

// Covers both the general kernel's layout (actq_bytes) and the engine's
// compact one, which pads each token's scale rows to 4 entries.
size_t quantr_gemv_workspace_bytes(int d, int B)
{
    B = B > 0 ? B : 1;
    return actq_bytes(d, B) + 256 + 32 * (size_t)B;
}

static int gemv_dev_common(float* out, long long ldo, const float* x, long long ldx, const uint8_t* xblocks,
                           const void* w, uint32_t type, int n, int d, int B, void* ws, size_t ws_bytes,
                           void* stream, int32_t* isum, int32_t* bsum)
{
    if (n <= 0 || B <= 0) return QUANTR_OK;
    if (!out || !w || (!x && !xblocks) || d < 0 || ldo < n) return QUANTR_ERR_BAD_ARG;
    if (x && ldx < d) return QUANTR_ERR_BAD_ARG;
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    cudaError_t e;
    if (type == T_F32) {
        if (!x || isum) return QUANTR_ERR_BAD_ARG;
        e = launch_gemv_f32((const float*)w, x, ldx, out, ldo, n, d, B, c);
        return code_of(e);
    }
    if (!type_supported(type)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    if (!ws || ws_bytes < actq_bytes(d, B)) return QUANTR_ERR_WORKSPACE;
    int* err = device_error_word();
    if (x && !isum && B >= 2) {
        // 2+ tokens: the tensor-core kernel (16-byte aligned weights).
        e = launch_gemv_tc((const uint8_t*)w, type, n, d, B, x, ldx, out, ldo, err, c.stream);
        if (e != cudaErrorNotSupported) return code_of(e);
    }
    if (x && !isum && ((uintptr_t)ws & 15) == 0) {
        // Fast path: the persistent engine (16-byte aligned weights, B <= 16).
        e = launch_gemv_engine((const uint8_t*)w, type, n, d, B, x, ldx, out, ldo, ws, ws_bytes, err, c.stream);
        if (e != cudaErrorNotSupported) return code_of(e);
    }
    ActQ a = actq_carve(ws, d, B);
    if (x)
        e = launch_quantize(x, ldx, d, B, a, nullptr, nullptr, c);
    else
        e = launch_repack(xblocks, d / 32, B, a, c);
    if (e != cudaSuccess) return code_of(e);
    GemvArgs ga;
    ga.w = (const uint8_t*)w;
    ga.type = type;
    ga.n = n;
    ga.d = d;
    ga.x = a;
    ga.out = out;
    ga.ldo = ldo;
    ga.B = B;
    ga.dbg_isum = isum;
    ga.dbg_bsum = bsum;
    ga.err = err;
    return code_of(launch_gemv(ga, c));
}

int quantr_gemv_dev(float* out, long long ldo, const float* x, long long ldx, const void* w, uint32_t type, int n,
                    int d, int B, void* workspace, size_t workspace_bytes, void* stream)
{
    return gemv_dev_common(out, ldo, x, ldx, nullptr, w, type, n, d, B, workspace, workspace_bytes, stream, nullptr,
                           nullptr);
}

int quantr_gemv_q8act_dev(float* out, long long ldo, const block_q8_0* xq, const void* w, uint32_t type, int n, int d,
                          int B, void* workspace, size_t workspace_bytes, void* stream)
{
    if (type == T_F32) return QUANTR_ERR_UNSUPPORTED_TYPE;
    return gemv_dev_common(out, ldo, nullptr, 0, (const uint8_t*)xq, w, type, n, d, B, workspace, workspace_bytes,
                           stream, nullptr, nullptr);
}

int quantr_gemv_partials_dev(float* out, int32_t* isum, int32_t* bsum, const float* x, const void* w, uint32_t type,
                             int n, int d, int B, void* workspace, size_t workspace_bytes, void* stream)
{
    if (!isum || !bsum || type == T_F32) return QUANTR_ERR_BAD_ARG;
    return gemv_dev_common(out, n, x, d, nullptr, w, type, n, d, B, workspace, workspace_bytes, stream, isum, bsum);
}

int quantr_quantize_q8_0_dev(block_q8_0* y, const float* x, long long ldx, int k, int B, void* stream)
{
    if (k / 32 <= 0 || B <= 0) return QUANTR_OK;
    if (!y || !x || ldx < k) return QUANTR_ERR_BAD_ARG;
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    ActQ none{};  // packed blocks only
    return code_of(launch_quantize(x, ldx, k, B, none, (uint8_t*)y, nullptr, c));
}

// ------------------------------------------------------------------- MoE --

// Public MoE workspace: the stage layout, then o (P x dim), sel and wts (P each)
// for quantr_moe_dev's internal use.
struct MoePublicWs {
    size_t o, sel, wts, total;
};

static MoePublicWs moe_public(int T, int E, int k, int dim, int hidden)
{
    const size_t P = (size_t)std::max(T, 1) * std::max(k, 1);
    MoePublicWs w;
    w.o = a256(moe_workspace_bytes(T, E, k, dim, hidden));
    w.sel = w.o + a256(P * std::max(dim, 1) * 4);
    w.wts = w.sel + a256(P * 4);
    w.total = w.wts + a256(P * 4);
    return w;
}

size_t quantr_moe_workspace_bytes(int T, int E, int k, int dim, int hidden)
{
    return moe_public(T, E, k, dim, hidden).total;
}

static bool expert_ok(const quantr_expert_weights* w)
{
    return w && (w->base || w->table) && type_supported(w->type) && w->type != T_F32;
}

static int experts_check(const quantr_expert_weights* w1, const quantr_expert_weights* w3,
                         const quantr_expert_weights* w2)
{
    if (!w1 || !w3 || !w2) return QUANTR_ERR_BAD_ARG;
    if (!(w1->base || w1->table) || !(w3->base || w3->table) || !(w2->base || w2->table)) return QUANTR_ERR_BAD_ARG;
    if (!expert_ok(w1) || !expert_ok(w3) || !expert_ok(w2)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    return QUANTR_OK;
}

static int route_check(const float* xb, long long ldx, int T, const float* router, const float* logits,
                       long long ldl, int E, int k, int dim)
{
    if (T < 0 || dim <= 0) return QUANTR_ERR_BAD_ARG;
    if (E <= 0 || E > kMoeMaxExperts || k <= 0 || k > kMoeMaxK || k > E) return QUANTR_ERR_BAD_ARG;
    if (router && (!xb || ldx < dim)) return QUANTR_ERR_BAD_ARG;
    if (!router && (!logits || ldl < E)) return QUANTR_ERR_BAD_ARG;
    return QUANTR_OK;
}

static bool ws_ok(const void* ws, size_t have, size_t need)
{
    return ws && have >= need && ((uintptr_t)ws & 255) == 0;
}

static ExpertMats mats_of(const quantr_expert_weights* w)
{
    ExpertMats m;
    m.base = (const uint8_t*)w->base;
    m.stride = w->stride;
    m.table = (const uint8_t* const*)w->table;
    m.type = w->type;
    return m;
}

int quantr_moe_route_dev(int* sel, float* wts, const float* xb, long long ldx, int T, const float* router,
                         const float* logits, long long ldl, int E, int k, int dim, void* workspace,
                         size_t workspace_bytes, void* stream)
{
    int rc = route_check(xb, ldx, T, router, logits, ldl, E, k, dim);
    if (rc || T == 0) return rc;
    if (!sel || !wts) return QUANTR_ERR_BAD_ARG;
    if (!ws_ok(workspace, workspace_bytes, moe_workspace_bytes(T, E, k, dim, 1))) return QUANTR_ERR_WORKSPACE;
    MoeRoute r;
    r.sel = sel;
    r.wts = wts;
    r.xb = xb;
    r.ldx = ldx;
    r.T = T;
    r.router = router;
    r.logits = logits;
    r.ldl = ldl;
    r.E = E;
    r.k = k;
    r.dim = dim;
    r.ws = workspace;
    r.ws_bytes = workspace_bytes;
    r.err = device_error_word();
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    return code_of(launch_moe_route(r, c));
}

int quantr_moe_experts_dev(float* o, const float* xb, long long ldx, int T, const int* sel, int k, int e0, int E_local,
                           const quantr_expert_weights* w1, const quantr_expert_weights* w3,
                           const quantr_expert_weights* w2, int dim, int hidden, void* workspace,
                           size_t workspace_bytes, void* stream)
{
    if (T < 0 || !o || !xb || !sel || dim <= 0 || hidden <= 0 || ldx < dim || k <= 0 || k > kMoeMaxK || e0 < 0 ||
        E_local <= 0 || E_local > kMoeMaxExperts)
        return QUANTR_ERR_BAD_ARG;
    int rc = experts_check(w1, w3, w2);
    if (rc || T == 0) return rc;
    if (!ws_ok(workspace, workspace_bytes, moe_workspace_bytes(T, E_local, k, dim, hidden)))
        return QUANTR_ERR_WORKSPACE;
    MoeExperts a;
    a.o = o;
    a.xb = xb;
    a.ldx = ldx;
    a.T = T;
    a.sel = sel;
    a.k = k;
    a.e0 = e0;
    a.El = E_local;
    a.dim = dim;
    a.hidden = hidden;
    a.w1 = mats_of(w1);
    a.w3 = mats_of(w3);
    a.w2 = mats_of(w2);
    a.ws = workspace;
    a.ws_bytes = workspace_bytes;
    a.err = device_error_word();
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    return code_of(launch_moe_experts(a, c));
}

int quantr_moe_combine_dev(float* out, long long ldo, const float* o, const int* sel, const float* wts, int T, int k,
                           int dim, void* stream)
{
    if (T < 0 || !out || !o || !sel || !wts || dim <= 0 || ldo < dim || k <= 0 || k > kMoeMaxK)
        return QUANTR_ERR_BAD_ARG;
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    return code_of(launch_moe_combine(out, ldo, o, sel, wts, T, k, dim, c));
}

// route -> experts (all E local) -> combine; o, and sel/wts when the caller
// passes none, live in the workspace.
static cudaError_t moe_full(float* out, long long ldo, const float* xb, long long ldx, int T, const float* router,
                            const float* logits, long long ldl, int E, int k, const ExpertMats& w1,
                            const ExpertMats& w3, const ExpertMats& w2, int dim, int hidden, int* sel, float* wts,
                            void* ws, size_t ws_bytes, int* err, const LaunchCfg& c)
{
    const MoePublicWs L = moe_public(T, E, k, dim, hidden);
    uint8_t* base = static_cast<uint8_t*>(ws);
    float* o = reinterpret_cast<float*>(base + L.o);
    if (!sel) sel = reinterpret_cast<int*>(base + L.sel);
    if (!wts) wts = reinterpret_cast<float*>(base + L.wts);
    MoeRoute r;
    r.sel = sel;
    r.wts = wts;
    r.xb = xb;
    r.ldx = ldx;
    r.T = T;
    r.router = router;
    r.logits = logits;
    r.ldl = ldl;
    r.E = E;
    r.k = k;
    r.dim = dim;
    r.ws = ws;
    r.ws_bytes = L.o;
    r.err = err;
    cudaError_t e = launch_moe_route(r, c);
    MoeExperts a;
    a.o = o;
    a.xb = xb;
    a.ldx = ldx;
    a.T = T;
    a.sel = sel;
    a.k = k;
    a.e0 = 0;
    a.El = E;
    a.dim = dim;
    a.hidden = hidden;
    a.w1 = w1;
    a.w3 = w3;
    a.w2 = w2;
    a.ws = ws;
    a.ws_bytes = L.o;
    a.err = err;
    if (e == cudaSuccess) e = launch_moe_experts(a, c);
    if (e == cudaSuccess) e = launch_moe_combine(out, ldo, o, sel, wts, T, k, dim, c);
    return e;
}

int quantr_moe_dev(float* out, long long ldo, const float* xb, long long ldx, int T, const float* router,
                   const float* logits, long long ldl, int E, int k, const quantr_expert_weights* w1,
                   const quantr_expert_weights* w3, const quantr_expert_weights* w2, int dim, int hidden, int* sel,
                   float* wts, void* workspace, size_t workspace_bytes, void* stream)
{
    int rc = route_check(xb, ldx, T, router, logits, ldl, E, k, dim);
    if (!rc && (!out || !xb || hidden <= 0 || ldx < dim || ldo < dim)) rc = QUANTR_ERR_BAD_ARG;
    if (!rc) rc = experts_check(w1, w3, w2);
    if (rc || T == 0) return rc;
    if (!ws_ok(workspace, workspace_bytes, quantr_moe_workspace_bytes(T, E, k, dim, hidden)))
        return QUANTR_ERR_WORKSPACE;
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    return code_of(moe_full(out, ldo, xb, ldx, T, router, logits, ldl, E, k, mats_of(w1), mats_of(w3), mats_of(w2),
                            dim, hidden, sel, wts, workspace, workspace_bytes, device_error_word(), c));
}

// Resolves an array of E host expert pointers to device memory: a uniform
// stride when the experts are evenly spaced (returns QUANTR_OK), else the
// caller needs a pointer table (returns -1).
static int resolve_experts(const void* const* host, int E, size_t mat_bytes, uint32_t type,
                           quantr_expert_weights* w, const uint8_t** devs)
{
    if (!host) return QUANTR_ERR_BAD_ARG;
    for (int e = 0; e < E; ++e) {
        if (!host[e]) return QUANTR_ERR_BAD_ARG;
        devs[e] = lookup(host[e], mat_bytes);
        if (!devs[e]) return QUANTR_ERR_UNREGISTERED;
    }
    const long long stride = E > 1 ? (long long)(devs[1] - devs[0]) : 0;
    bool uniform = true;
    for (int e = 1; e < E && uniform; ++e) uniform = (long long)(devs[e] - devs[0]) == (long long)e * stride;
    w->base = devs[0];
    w->stride = uniform ? stride : 0;
    w->table = nullptr;
    w->type = type;
    return uniform ? QUANTR_OK : -1;
}

int quantr_moe_layer(float* out, const float* xb, int T, const float* router, const float* logits, int E, int k,
                     const void* const* w1, uint32_t t1, const void* const* w3, uint32_t t3, const void* const* w2,
                     uint32_t t2, int dim, int hidden, int* sel, float* wts)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    auto fail = [&](int rc) {
        if (out && T > 0 && dim > 0) zero_out(out, (size_t)T * dim);
        set_err(rc);
        return rc;
    };
    if (T == 0) return QUANTR_OK;
    int rc = route_check(xb, dim, T, router, logits, E, E, k, dim);
    if (!rc && (!out || !xb || hidden <= 0 || !w1 || !w3 || !w2)) rc = QUANTR_ERR_BAD_ARG;
    if (!rc) {
        const quantr_expert_weights v1{(const void*)1, 0, nullptr, t1}, v3{(const void*)1, 0, nullptr, t3},
            v2{(const void*)1, 0, nullptr, t2};
        rc = experts_check(&v1, &v3, &v2);
    }
    if (rc) return fail(rc);
    if ((rc = ensure_ready())) return fail(rc);

    // Expert matrices: W1/W3 are hidden x dim, W2 dim x hidden
    // (ggml_type_row_size slices, src/model.c:20-30, 412-414).
    quantr_expert_weights w[3];
    const void* const* hosts[3] = {w1, w3, w2};
    const uint32_t types[3] = {t1, t3, t2};
    const size_t mats[3] = {(size_t)hidden * row_bytes(t1, dim), (size_t)hidden * row_bytes(t3, dim),
                            (size_t)dim * row_bytes(t2, hidden)};
    std::vector<const uint8_t*> devs((size_t)3 * E);
    bool need_table[3] = {false, false, false};
    for (int m = 0; m < 3; ++m) {
        rc = resolve_experts(hosts[m], E, std::max(mats[m], (size_t)1), types[m], &w[m], &devs[(size_t)m * E]);
        if (rc == -1) need_table[m] = true;
        else if (rc) return fail(rc);
    }

    // Host staging (mapped): x | logits | tables | out | sel | wts | err; the
    // first three are copied to device memory with one copy.
    const size_t xbytes = (size_t)T * dim * 4, lbytes = router ? 0 : (size_t)T * E * 4;
    const size_t tbytes = (size_t)3 * E * sizeof(void*), rbytes = (size_t)E * dim * 4;
    const size_t x_off = 0, l_off = a256(xbytes), t_off = l_off + a256(lbytes), in_end = t_off + a256(tbytes);
    const size_t o_off = in_end, s_off = o_off + a256(xbytes), w_off = s_off + a256((size_t)T * k * 4);
    const size_t e_off = w_off + a256((size_t)T * k * 4), h_total = e_off + 256;
    const uint8_t* rdev = router ? lookup(router, rbytes) : nullptr;
    const size_t r_off = in_end, d_total = in_end + (router && !rdev ? a256(rbytes) : 0);
    if ((rc = grow_host(h_total))) return fail(rc);
    if ((rc = grow_dev((void**)&g.dbuf, &g.dbuf_bytes, d_total))) return fail(rc);
    const size_t wsb = quantr_moe_workspace_bytes(T, E, k, dim, hidden);
    if ((rc = grow_dev(&g.ws, &g.ws_bytes, wsb))) return fail(rc);

    std::memcpy(g.hbuf + x_off, xb, xbytes);
    if (!router) std::memcpy(g.hbuf + l_off, logits, lbytes);
    const uint8_t** tab = reinterpret_cast<const uint8_t**>(g.hbuf + t_off);
    for (size_t i = 0; i < (size_t)3 * E; ++i) tab[i] = devs[i];
    for (int m = 0; m < 3; ++m)
        if (need_table[m]) w[m].table = (const void* const*)(g.dbuf + t_off + (size_t)m * E * sizeof(void*));
    write_mapped_int(g.hbuf + e_off, 0);
    cudaError_t e = cudaMemcpyAsync(g.dbuf, g.hbuf, in_end, cudaMemcpyHostToDevice, g.stream);
    if (e == cudaSuccess && router && !rdev) {
        e = cudaMemcpyAsync(g.dbuf + r_off, router, rbytes, cudaMemcpyHostToDevice, g.stream);
        rdev = g.dbuf + r_off;
    }
    LaunchCfg c;
    c.stream = g.stream;
    if (e == cudaSuccess)
        e = moe_full((float*)(g.hbuf_dev + o_off), dim, (const float*)(g.dbuf + x_off), dim, T,
                     router ? (const float*)rdev : nullptr, router ? nullptr : (const float*)(g.dbuf + l_off), E, E,
                     k, mats_of(&w[0]), mats_of(&w[1]), mats_of(&w[2]), dim, hidden, (int*)(g.hbuf_dev + s_off),
                     (float*)(g.hbuf_dev + w_off), g.ws, g.ws_bytes, (int*)(g.hbuf_dev + e_off), c);
    if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(code_of(e));
    }
    const int dv = read_mapped_int(g.hbuf + e_off);
    if (dv != DEV_OK && dv != DEV_ERR_ROUTING) return fail(dev_code(dv));
    std::memcpy(out, g.hbuf + o_off, xbytes);
    if (sel) std::memcpy(sel, g.hbuf + s_off, (size_t)T * k * 4);
    if (wts) std::memcpy(wts, g.hbuf + w_off, (size_t)T * k * 4);
    if (dv == DEV_ERR_ROUTING) {
        set_err(QUANTR_ERR_ROUTING);
        return QUANTR_ERR_ROUTING;
    }
    return QUANTR_OK;
}

int quantr_dequantize_rows_dev(float* out, long long ldo, const void* src, long long src_stride, uint32_t type, int n,
                               int rows, void* stream)
{
    if (n <= 0 || rows <= 0) return QUANTR_OK;
    if (!out || !src || ldo < n || src_stride < row_bytes(type, n)) return QUANTR_ERR_BAD_ARG;
    if (!type_supported(type)) return QUANTR_ERR_UNSUPPORTED_TYPE;
    LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    return code_of(launch_dequantize_rows(out, ldo, (const uint8_t*)src, src_stride, type, n, rows, c));
}

int quantr_gpu_device_status(void* stream, int reset)
{
    int* w = device_error_word();
    if (!w) return QUANTR_ERR_CUDA;
    int v = 0;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) {
        cudaGetLastError();
        return QUANTR_ERR_CUDA;
    }
    if (cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return QUANTR_ERR_CUDA;
    if (reset) cudaMemset(w, 0, 4);
    // The allocation-free GEMV keeps its own word in the library's static
    // scratch array; a timeout recorded there is reported here too.
    const int na = noalloc_device_error(reset);
    if (v == DEV_OK) v = na;
    return dev_code(v);
}

} // extern "C"
