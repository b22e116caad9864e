// KERNIX-B200 GPU backend of the reference's 2-D tensor library: the functions include/kernix.h calls when built
// with its GPU backend (include/kernix_gpu.h lists them with the reference lines they replace; the reference's
// implementation is src/kernix_metal.m). Storage of >= 64 KB tensors is page-locked host memory mapped into the device
// address space, so the library's CPU code and these kernels work on the same bytes: kernels stream them over PCIe,
// one read of each input and one write of the output. Element-wise and row kernels are grid-stride, float4 where the
// shapes allow; all calls complete before they return (the reference waits for its command buffers too).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <vector>

#include "kernix_gpu.h"
#include "kx_kernels.h"

namespace {

constexpr size_t TB_GPU_MIN = size_t(1) << 22;      // elements below which the caller's CPU code is used
constexpr size_t TB_CACHE_MAX = size_t(256) << 20;  // bytes of freed storage kept for reuse
constexpr size_t TB_PAGE = 16384;                   // the reference's tensor page (include/kernix.h:28)

std::mutex g_mu;
std::unordered_map<const void*, size_t> g_live;  // backend storage -> bytes
std::vector<std::pair<void*, size_t>> g_cache;   // freed storage, oldest first
size_t g_cache_bytes = 0;

// scratch of kernix_matmul_ep_into: one buffer per device, grown to the largest product seen, released by
// kernix_metal_release_cache; callers hold g_mm_mu for the whole product
constexpr int TB_MAX_DEVICES = 64;
std::mutex g_mm_mu;
struct MmScratch {
    void* p;
    size_t cap;
};
MmScratch g_mm[TB_MAX_DEVICES] = {};

uint8_t* mm_scratch(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= TB_MAX_DEVICES) {
        cudaGetLastError();
        return nullptr;
    }
    MmScratch& s = g_mm[dev];
    if (s.cap < bytes) {
        if (s.p != nullptr) cudaFree(s.p);
        s.p = nullptr;
        s.cap = 0;
        if (cudaMalloc(&s.p, bytes) != cudaSuccess) {
            cudaGetLastError();
            s.p = nullptr;
            return nullptr;
        }
        s.cap = bytes;
    }
    return static_cast<uint8_t*>(s.p);
}

bool is_backend(const void* p, size_t bytes) {
    std::lock_guard<std::mutex> g(g_mu);
    const auto it = g_live.find(p);
    return it != g_live.end() && it->second >= bytes;
}

// Device-readable view of `bytes` of host data: backend storage as is, anything else copied into *tmp (device
// memory the caller frees). nullptr on failure.
const float* device_view(const float* p, size_t bytes, void** tmp) {
    *tmp = nullptr;
    if (p == nullptr) return nullptr;
    if (is_backend(p, bytes)) {
        void* d = nullptr;
        return cudaHostGetDevicePointer(&d, const_cast<float*>(p), 0) == cudaSuccess ? static_cast<const float*>(d) : nullptr;
    }
    if (cudaMalloc(tmp, bytes) != cudaSuccess) {
        cudaGetLastError();
        *tmp = nullptr;
        return nullptr;
    }
    if (cudaMemcpy(*tmp, p, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(*tmp);
        *tmp = nullptr;
        return nullptr;
    }
    return static_cast<const float*>(*tmp);
}

float* device_out(float* p) {
    void* d = nullptr;
    return cudaHostGetDevicePointer(&d, p, 0) == cudaSuccess ? static_cast<float*>(d) : nullptr;
}

int grid_for(size_t work, int block) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t want = (work + block - 1) / block, cap = static_cast<size_t>(sms) * 8;
    return static_cast<int>(want < cap ? (want ? want : 1) : cap);
}

// GELU with the Abramowitz-Stegun 7.1.26 erf (the reference's CPU and GPU formula, include/kernix.h:485-496)
__device__ __forceinline__ float gelu_as_exact(float x) {
    const float z = __fmul_rn(fabsf(x), 0.70710678f);
    const float k = __fdiv_rn(1.0f, __fmaf_rn(0.3275911f, z, 1.0f));
    const float p =
        k * (0.254829592f + k * (-0.284496736f + k * (1.421413741f + k * (-1.453152027f + k * 1.061405429f))));
    return 0.5f * x * (1.0f + copysignf(1.0f - p * expf(-z * z), x));
}

__device__ __forceinline__ float map_op(int op, float v, float w, float p0, float p1) {
    switch (op) {
    case KERNIX_GPU_NEG: return -v;
    case KERNIX_GPU_ABS: return fabsf(v);
    case KERNIX_GPU_EXP: return expf(v);
    case KERNIX_GPU_LOG: return logf(v);
    case KERNIX_GPU_SQRT: return __fsqrt_rn(v);
    case KERNIX_GPU_TANH: return tanhf(v);
    case KERNIX_GPU_RELU: return fmaxf(v, 0.0f);
    case KERNIX_GPU_SIGMOID: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
    case KERNIX_GPU_SILU: return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    case KERNIX_GPU_GELU: return gelu_as_exact(v);
    case KERNIX_GPU_ADD_SCALAR: return __fadd_rn(v, p0);
    case KERNIX_GPU_MUL_SCALAR: return __fmul_rn(v, p0);
    case KERNIX_GPU_CLAMP: return fminf(fmaxf(v, p0), p1);
    case KERNIX_GPU_ADD: return __fadd_rn(v, w);
    case KERNIX_GPU_SUB: return __fsub_rn(v, w);
    case KERNIX_GPU_MUL: return __fmul_rn(v, w);
    default: return __fdiv_rn(v, w);  // KERNIX_GPU_DIV
    }
}

// y[i] = op(x[i], b[i] or b[i % bcols]) over n4 float4s; b4cols = bcols / 4 (0: b has x's shape)
__global__ void k_tb_map(int op, const float4* __restrict__ x, const float4* __restrict__ b, size_t b4cols,
                         float4* __restrict__ y, size_t n4, float p0, float p1) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float4 v = x[i];
        const float4 w = b ? b[b4cols ? i % b4cols : i] : v;
        y[i] = make_float4(map_op(op, v.x, w.x, p0, p1), map_op(op, v.y, w.y, p0, p1), map_op(op, v.z, w.z, p0, p1),
                           map_op(op, v.w, w.w, p0, p1));
    }
}

// block-wide reduction of one float (max or sum) over blockDim.x <= 1024 threads
__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, u) : __fadd_rn(v, u);
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();  // sh is free (the previous reduction's readers are done)
    if (lane == 0) sh[w] = v;
    __syncthreads();
    v = lane < nw ? sh[lane] : (is_max ? -INFINITY : 0.0f);
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, u) : __fadd_rn(v, u);
    }
    return v;
}

// one block per row: softmax (mode 0), log_softmax (1), layer_norm with optional gamma / beta (2), as the reference's
// row kernel and CPU loops compute them (include/kernix.h:640-666, src/kernix_metal.m rows_op)
__global__ void k_tb_rows(int mode, const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ bt,
                          float eps, float* __restrict__ y, size_t rows, size_t cols) {
    __shared__ float sh[32];
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* xr = x + r * cols;
        float* yr = y + r * cols;
        if (mode < 2) {
            float m = -INFINITY;
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, xr[c]);
            m = block_reduce(m, true, sh);
            float s = 0.0f;
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, expf(__fsub_rn(xr[c], m)));
            s = block_reduce(s, false, sh);
            if (mode == 0) {
                const float inv = __fdiv_rn(1.0f, s);
                for (size_t c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = __fmul_rn(expf(__fsub_rn(xr[c], m)), inv);
            } else {
                const float k = __fadd_rn(m, logf(s));
                for (size_t c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = __fsub_rn(xr[c], k);
            }
        } else {
            float s = 0.0f;
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, xr[c]);
            const float mean = __fdiv_rn(block_reduce(s, false, sh), static_cast<float>(cols));
            float v = 0.0f;
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) {
                const float d = __fsub_rn(xr[c], mean);
                v = __fmaf_rn(d, d, v);
            }
            const float var = __fdiv_rn(block_reduce(v, false, sh), static_cast<float>(cols));
            const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
            for (size_t c = threadIdx.x; c < cols; c += blockDim.x) {
                float o = __fmul_rn(__fsub_rn(xr[c], mean), rstd);
                if (g) o = __fmul_rn(o, g[c]);
                if (bt) o = __fadd_rn(o, bt[c]);
                yr[c] = o;
            }
        }
    }
}

// 32 x 32 tiles (+1 column of padding): coalesced reads of x and writes of y
__global__ void k_tb_transpose(const float* __restrict__ x, float* __restrict__ y, size_t R, size_t C) {
    __shared__ float tile[32][33];
    const size_t c = blockIdx.x * 32ull + threadIdx.x, r = blockIdx.y * 32ull + threadIdx.y;
    for (int k = 0; k < 32; k += 8)
        if (r + k < R && c < C) tile[threadIdx.y + k][threadIdx.x] = x[(r + k) * C + c];
    __syncthreads();
    const size_t oc = blockIdx.y * 32ull + threadIdx.x, orow = blockIdx.x * 32ull + threadIdx.y;
    for (int k = 0; k < 32; k += 8)
        if (orow + k < C && oc < R) y[(orow + k) * R + oc] = tile[threadIdx.x][threadIdx.y + k];
}

int finish(void* t0, void* t1, void* t2) {
    const bool ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    cudaFree(t0);
    cudaFree(t1);
    cudaFree(t2);
    return ok ? 1 : 0;
}

// a new tensor with the reference's allocation rule (include/kernix.h:148-174): >= 64 KB in backend storage
float_tensor* tensor_new(int rows, int cols) {
    if (rows < 0 || cols < 0) return nullptr;
    float_tensor* t = static_cast<float_tensor*>(std::malloc(sizeof(float_tensor)));
    if (t == nullptr) return nullptr;
    t->row = rows;
    t->col = cols;
    const size_t bytes = (sizeof(float) * static_cast<size_t>(rows) * cols + TB_PAGE - 1) / TB_PAGE * TB_PAGE;
    void* mem = bytes >= (1u << 16) ? kernix_metal_alloc(bytes) : nullptr;
    if (mem == nullptr && posix_memalign(&mem, TB_PAGE, bytes ? bytes : TB_PAGE) != 0) mem = nullptr;
    t->tensor = static_cast<float*>(mem);
    if (t->tensor == nullptr) {
        std::free(t);
        return nullptr;
    }
    return t;
}

}  // namespace

extern "C" {

void* kernix_metal_alloc(size_t bytes) {
    if (bytes == 0) return nullptr;
    {
        std::lock_guard<std::mutex> g(g_mu);
        for (size_t i = 0; i < g_cache.size(); i++)
            if (g_cache[i].second == bytes) {
                void* p = g_cache[i].first;
                g_cache.erase(g_cache.begin() + static_cast<long>(i));
                g_cache_bytes -= bytes;
                g_live[p] = bytes;
                return p;
            }
    }
    void* p = nullptr;
    if (cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_mu);
    g_live[p] = bytes;
    return p;
}

int kernix_metal_free(void* p) {
    if (p == nullptr) return 0;
    std::vector<void*> drop;
    {
        std::lock_guard<std::mutex> g(g_mu);
        const auto it = g_live.find(p);
        if (it == g_live.end()) return 0;
        const size_t bytes = it->second;
        g_live.erase(it);
        if (bytes <= TB_CACHE_MAX) {
            while (g_cache_bytes + bytes > TB_CACHE_MAX && !g_cache.empty()) {
                g_cache_bytes -= g_cache.front().second;
                drop.push_back(g_cache.front().first);
                g_cache.erase(g_cache.begin());
            }
            g_cache.emplace_back(p, bytes);
            g_cache_bytes += bytes;
        } else {
            drop.push_back(p);
        }
    }
    for (void* q : drop) cudaFreeHost(q);
    return 1;
}

void kernix_metal_release_cache(void) {
    std::vector<std::pair<void*, size_t>> drop;
    {
        std::lock_guard<std::mutex> g(g_mu);
        drop.swap(g_cache);
        g_cache_bytes = 0;
    }
    for (auto& e : drop) cudaFreeHost(e.first);
    std::lock_guard<std::mutex> lock(g_mm_mu);
    int cur = 0;
    cudaGetDevice(&cur);
    for (int d = 0; d < TB_MAX_DEVICES; ++d) {
        if (g_mm[d].p == nullptr) continue;
        cudaSetDevice(d);
        cudaFree(g_mm[d].p);
        g_mm[d] = MmScratch{};
    }
    cudaSetDevice(cur);
    cudaGetLastError();
}

size_t kernix_metal_map(int op, const float* x, const float* b, size_t bcols, float* y, size_t n, float p0, float p1) {
    const size_t n4 = n / 4;
    if (n < TB_GPU_MIN || bcols % 4 != 0 || op < KERNIX_GPU_NEG || op > KERNIX_GPU_DIV || x == nullptr ||
        !is_backend(y, n * sizeof(float)))
        return 0;
    const bool binary = op >= KERNIX_GPU_ADD;
    if (binary && b == nullptr) return 0;
    void *tx = nullptr, *tb = nullptr;
    const float* dx = device_view(x, n * sizeof(float), &tx);
    const float* db = binary ? device_view(b, (bcols ? bcols : n) * sizeof(float), &tb) : nullptr;
    float* dy = device_out(y);
    if (dx == nullptr || dy == nullptr || (binary && db == nullptr)) {
        finish(tx, tb, nullptr);
        return 0;
    }
    k_tb_map<<<grid_for(n4, 256), 256>>>(op, reinterpret_cast<const float4*>(dx), reinterpret_cast<const float4*>(db),
                                         bcols / 4, reinterpret_cast<float4*>(dy), n4, p0, p1);
    return finish(tx, tb, nullptr) ? n4 * 4 : 0;
}

int kernix_metal_rows(int mode, const float* x, const float* g, const float* b, float eps, float* y, size_t rows,
                      size_t cols) {
    if (rows * cols < TB_GPU_MIN || cols == 0 || mode < 0 || mode > 2 || x == nullptr || x == y ||
        !is_backend(y, rows * cols * sizeof(float)))
        return 0;
    void *tx = nullptr, *tg = nullptr, *tbt = nullptr;
    const float* dx = device_view(x, rows * cols * sizeof(float), &tx);
    const float* dg = (mode == 2 && g) ? device_view(g, cols * sizeof(float), &tg) : nullptr;
    const float* dbt = (mode == 2 && b) ? device_view(b, cols * sizeof(float), &tbt) : nullptr;
    float* dy = device_out(y);
    if (dx == nullptr || dy == nullptr || (mode == 2 && g && dg == nullptr) || (mode == 2 && b && dbt == nullptr)) {
        finish(tx, tg, tbt);
        return 0;
    }
    int threads = static_cast<int>(((cols + 3) / 4 + 31) / 32 * 32);
    if (threads > 1024) threads = 1024;
    const size_t blocks = rows < 65535ull * 16 ? rows : 65535ull * 16;
    k_tb_rows<<<static_cast<unsigned>(blocks), threads>>>(mode, dx, dg, dbt, eps, dy, rows, cols);
    return finish(tx, tg, tbt);
}

int kernix_metal_transpose(const float* x, float* y, size_t rows, size_t cols) {
    if (rows * cols < TB_GPU_MIN || x == nullptr || x == y || !is_backend(y, rows * cols * sizeof(float)) ||
        (cols + 31) / 32 > 0x7fffffffull || (rows + 31) / 32 > 65535)
        return 0;
    void* tx = nullptr;
    const float* dx = device_view(x, rows * cols * sizeof(float), &tx);
    float* dy = device_out(y);
    if (dx == nullptr || dy == nullptr) {
        finish(tx, nullptr, nullptr);
        return 0;
    }
    k_tb_transpose<<<dim3(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32)), dim3(32, 8)>>>(
        dx, dy, rows, cols);
    return finish(tx, nullptr, nullptr);
}

int kernix_matmul_ep_into(const float_tensor* a, const float_tensor* b, float_tensor* c, const float* bias, int act,
                          float alpha, kernix_rows_fn cpu_ep) {
    if (a == nullptr || b == nullptr || c == nullptr || a->tensor == nullptr || b->tensor == nullptr || c->tensor == nullptr)
        return -1;
    if (a->col != b->row) {
        std::fprintf(stderr, "matmul: dimension mismatch A(%dx%d) x B(%dx%d)\n", a->row, a->col, b->row, b->col);
        return -1;
    }
    if (c->row != a->row || c->col != b->col) return -1;
    const int m = a->row, k = a->col, n = b->col;
    if (m == 0 || n == 0) return 0;
    if (k == 0) {  // inner dimension 0: the product is all zeros, the post-processing runs on the CPU
        std::memset(c->tensor, 0, sizeof(float) * static_cast<size_t>(m) * n);
        if (cpu_ep != nullptr) cpu_ep(0, static_cast<size_t>(m));
        return 0;
    }
    // device copies: A (m x k), B (k x n) split into the tf32 planes (n x ldw), bias, C, status word; all carved
    // from one per-device scratch buffer that only grows, so repeated products allocate nothing
    const int ldw = (k + 31) / 32 * 32;
    const size_t sa = static_cast<size_t>(m) * k, sw = static_cast<size_t>(k) * n, sp = static_cast<size_t>(n) * ldw,
                 sc = static_cast<size_t>(m) * n;
    const size_t parts[7] = {sa * 4, sw * 4, sp * 4, sp * 4, sc * 4, static_cast<size_t>(n) * 4, sizeof(int)};
    size_t offs[7], total = 0;
    for (int i = 0; i < 7; ++i) {
        offs[i] = total;
        total += (parts[i] + 255) / 256 * 256;
    }
    std::lock_guard<std::mutex> lock(g_mm_mu);
    uint8_t* base = mm_scratch(total);
    if (base == nullptr) {
        std::fprintf(stderr, "matmul: no device memory for a %dx%dx%d product\n", m, k, n);
        return -1;
    }
    float* da = reinterpret_cast<float*>(base + offs[0]);
    float* dw = reinterpret_cast<float*>(base + offs[1]);
    float* dhi = reinterpret_cast<float*>(base + offs[2]);
    float* dlo = reinterpret_cast<float*>(base + offs[3]);
    float* dc = reinterpret_cast<float*>(base + offs[4]);
    float* dbias = bias ? reinterpret_cast<float*>(base + offs[5]) : nullptr;
    int* dst = reinterpret_cast<int*>(base + offs[6]);
    bool ok = cudaMemsetAsync(dst, 0, sizeof(int), nullptr) == cudaSuccess &&
              cudaMemcpy(da, a->tensor, sa * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(dw, b->tensor, sw * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              (bias == nullptr || cudaMemcpy(dbias, bias, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice) == cudaSuccess);
    ok = ok && kx_prep_f32_weight(dw, k, n, dhi, dlo, ldw, nullptr) == 0 &&
         kx_gemm_f32(da, k, dhi, dlo, ldw, dbias, dc, n, m, n, k, act, alpha, dst, nullptr) == 0 &&
         cudaDeviceSynchronize() == cudaSuccess;
    int status = 1;
    ok = ok && cudaMemcpy(&status, dst, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && status == 0 &&
         cudaMemcpy(c->tensor, dc, sc * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        std::fprintf(stderr, "matmul: the GPU product failed\n");
        return -1;
    }
    return 0;
}

float_tensor* float_matmul_metal(const float_tensor* a, const float_tensor* b) {
    if (a == nullptr || b == nullptr) return nullptr;
    float_tensor* c = tensor_new(a->row, b->col);
    if (c != nullptr && kernix_matmul_ep_into(a, b, c, nullptr, KERNIX_ACT_NONE, 0.0f, nullptr) != 0) {
        float_free(c);
        c = nullptr;
    }
    return c;
}

float_tensor* floats_fma_relu_metal(const float_tensor* a, const float_tensor* x, const float_tensor* b) {
    if (a == nullptr || x == nullptr || b == nullptr || a->tensor == nullptr || x->tensor == nullptr || b->tensor == nullptr ||
        a->row != x->row || a->col != x->col || b->row != x->row || b->col != x->col)
        return nullptr;
    float_tensor* y = tensor_new(x->row, x->col);
    if (y == nullptr) return nullptr;
    const size_t n = static_cast<size_t>(x->row) * x->col;
    if (n == 0) return y;
    // every size on the GPU: inputs and a non-backend output go through device copies
    void *ta = nullptr, *tx = nullptr, *tb = nullptr, *ty = nullptr;
    const float* da = device_view(a->tensor, n * 4, &ta);
    const float* dx = device_view(x->tensor, n * 4, &tx);
    const float* db = device_view(b->tensor, n * 4, &tb);
    const bool direct = is_backend(y->tensor, n * 4);
    float* dy = direct ? device_out(y->tensor) : nullptr;
    if (!direct && cudaMalloc(&ty, n * 4) == cudaSuccess) dy = static_cast<float*>(ty);
    bool ok = da && dx && db && dy && kx_fma_relu(da, dx, db, dy, n, nullptr) == 0 && cudaDeviceSynchronize() == cudaSuccess;
    if (ok && !direct) ok = cudaMemcpy(y->tensor, dy, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    ok = finish(ta, tx, tb) && ok;
    cudaFree(ty);
    if (!ok) {
        float_free(y);
        return nullptr;
    }
    return y;
}

}  // extern "C"
