// kx_linear_i8_noalloc: the int8 LINEAR step (kx_linear_i8) for callers that must not allocate device memory.
//
// Who needs it: code on a latency-critical path, where cudaMalloc's implicit device-wide synchronisation and
// unbounded latency are not acceptable, and hosts whose device memory is owned by a framework allocator that does
// not allow extra allocations. kx_linear_i8 needs two scratch buffers (the int8 activations and the per-row
// scales); this variant takes them from one fixed array compiled into the library instead of from the caller.
//
// The array below is a file-scope __device__ object: every GPU that loads the library holds its
// KX_NOALLOC_SCRATCH_BYTES until the process exits. Host code cannot use the array's name as a device address, so
// the first call on each device looks the address up with cudaGetSymbolAddress (with that device current) and
// caches it; make that first call before any stream capture. Nothing here calls cudaMalloc or cudaFree.
//
// All calls on a device share the one array. Every byte a call reads is written earlier in the same call (the
// quantiser writes all rows, including the zero padding up to the 16-byte row pitch, and every row scale), so no
// state carries over between calls and nothing needs clearing. Two calls whose work overlaps on the GPU (different
// streams, or other threads) race on the array and corrupt each other's results: order them on one stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "kx_kernels.h"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[KX_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
uint8_t* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// device address of the array on the current device, looked up once per device
uint8_t* scratch_on_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "kx_linear_i8_noalloc: cannot locate the scratch array on device %d: %s\n", dev,
                         cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_ptr[dev] = static_cast<uint8_t*>(p);
    }
    return g_scratch_ptr[dev];
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
    uint8_t* base = scratch_on_current_device();
    if (base == nullptr) return -1;
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* sx = reinterpret_cast<float*>(base + sx_off);
    if (kx_quant_rows(x, ldx, rows, k, xq, static_cast<int>(ldq), sx, stream) != 0) return -1;
    return kx_gemm_i8(xq, static_cast<int>(ldq), sx, wq, ldw, scale, bias, y, ldy, rows, n, k, act, alpha, status, stream);
}
