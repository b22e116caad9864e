// kx_linear_i8_noalloc: the int8 LINEAR step (kx_linear_i8) for callers that must not allocate device memory.
//
// Who needs it: code on a latency-critical path, where cudaMalloc's implicit device-wide synchronisation and
// unbounded latency are not acceptable, and hosts whose device memory is owned by a framework allocator that does
// not allow extra allocations. kx_linear_i8 needs two scratch buffers (the int8 activations and the per-row
// scales); this variant takes them from one fixed array compiled into the library instead of from the caller.
//
// The array below is a file-scope __device__ object of KX_NOALLOC_SCRATCH_BYTES. With CUDA's default lazy module
// loading it comes into existence on a device the first time this file's module is needed there: the first call
// of this entry point on each device (in its CUDA context) loads the module, which reserves the array, and looks
// the array's device address up with cudaGetSymbolAddress, with that device current. So that first call is the
// one that may take device memory and synchronise; make it in initialisation code, before any stream capture.
// Later calls in the same context reuse the cached address and allocate nothing; the array then stays reserved
// until the process exits (or the context is destroyed). Host code cannot use the array's name as a device
// address, which is why the address is looked up rather than taken. Nothing here calls cudaMalloc or cudaFree.
//
// The cached address belongs to one CUDA context: it is keyed by device and by the context current at the call,
// so after cudaDeviceReset (a new primary context) or under a different driver context it is looked up again.
//
// All calls in a context share the one array. Every byte a call reads is written earlier in the same call (the
// quantiser writes all rows, including the zero padding up to the 16-byte row pitch, and every row scale), so no
// state carries over between calls and nothing needs clearing. Two calls whose work overlaps on the GPU (different
// streams, or other threads) race on the array and corrupt each other's results: order them on one stream.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "kx_kernels.h"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[KX_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
struct Cached {
    CUcontext ctx;
    uint8_t* ptr;
};
Cached g_cache[kMaxDevices] = {};
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library links no libcuda stub)
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<CtxGetCurrentFn>(nullptr);
        }
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

// device address of the array in the current context, looked up once per (device, context)
uint8_t* scratch_in_current_context() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    CUcontext ctx = nullptr;
    CtxGetCurrentFn get = ctx_get_current();
    if (get != nullptr) get(&ctx);  // NULL before the runtime made its context current: then the lookup below does
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    Cached& c = g_cache[dev];
    if (c.ptr == nullptr || ctx == nullptr || c.ctx != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();  // leave no error behind for the next, unrelated launch check
            std::fprintf(stderr, "kx_linear_i8_noalloc: cannot locate the scratch array on device %d: %s\n", dev,
                         cudaGetErrorString(e));
            c.ptr = nullptr;
            return nullptr;
        }
        if (ctx == nullptr && get != nullptr) get(&ctx);  // the lookup made the primary context current
        c.ctx = ctx;
        c.ptr = static_cast<uint8_t*>(p);
    }
    return c.ptr;
}

}  // namespace

extern "C" int kx_linear_i8_noalloc(const float* x, int ldx, int rows, int k, const int8_t* wq, int ldw, const float* scale,
                                    const float* bias, float* y, int ldy, int n, int act, float alpha, int* status,
                                    void* stream) {
    if (rows <= 0 || n <= 0) return 0;
    if (k <= 0) return -1;
    // scratch layout: int8 activations rows x ldq, then the row scales at the next 256-byte boundary
    const size_t ldq = (static_cast<size_t>(k) + 15) / 16 * 16;
    const size_t sx_off = (static_cast<size_t>(rows) * ldq + 255) / 256 * 256;
    const size_t need = sx_off + static_cast<size_t>(rows) * sizeof(float);
    if (need > KX_NOALLOC_SCRATCH_BYTES) {
        std::fprintf(stderr,
                     "kx_linear_i8_noalloc: %d rows x %d inputs need %zu bytes of scratch, more than the %d-byte built-in "
                     "array; split the rows or call kx_linear_i8 with caller scratch\n",
                     rows, k, need, KX_NOALLOC_SCRATCH_BYTES);
        return -1;
    }
    uint8_t* base = scratch_in_current_context();
    if (base == nullptr) return -1;
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* sx = reinterpret_cast<float*>(base + sx_off);
    if (kx_quant_rows(x, ldx, rows, k, xq, static_cast<int>(ldq), sx, stream) != 0) return -1;
    return kx_gemm_i8(xq, static_cast<int>(ldq), sx, wq, ldw, scale, bias, y, ldy, rows, n, k, act, alpha, status, stream);
}
