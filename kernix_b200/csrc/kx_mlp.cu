// Fused small fp32 MLP: a chain of dense layers y = act(x . W + b) (kernix_dense :544-550, each layer reading only
// the previous one's output) and an optional trailing row softmax (floats_softmax_into include/kernix.h:652-657), run
// as ONE cooperative launch for batches small enough that the per-launch fixed costs of the tensor-core GEMMs
// (launch, set-up, pipeline fill, an epilogue nothing overlaps) dominate: configuration c1 (784-512-256-10 + softmax,
// 256 rows) is four launches of a few microseconds of work each otherwise.
//
// Each layer but a narrow last one is a phase. Its output is cut into 64 x 64 tiles and its reduction into `split`
// contiguous K ranges; the (tile, range) items are dealt round robin to the CTAs, each computing a 64 x 64 partial
// product on the CUDA cores in fp32 fused multiply-adds (4 x 4 outputs per thread, 32-deep K chunks staged in shared
// memory). The first layer reads a plain matrix, so its chunks are copied straight into an 8-deep cp.async ring: a
// whole K range is in flight at once and the multiply never waits on more than one memory round trip. Later layers
// form each input element as act(P[0] + P[1] + ... + b) from the previous layer's partial sums P[range][row][col] (in
// that fixed order; all ranges' loads issued before the first add) while staging their tiles through registers, one
// chunk ahead. A grid barrier ends each phase. The weights of the later layers are prefetched into L2 when the kernel
// starts, so that their first chunks do not wait on HBM.
//
// A narrow last layer (at most 64 outputs, at most 1024 inputs and 8192 weights: a classifier head) is no phase of
// its own: its weights are copied into shared memory at the start, and after the last barrier one warp per row forms
// the row's inputs from the partial sums, multiplies them by the weights (each output a dot product over K in four
// interleaved fp32 sums, added pairwise) and applies bias, activation and the softmax (max, exp(x - max), sum, times
// 1/sum: the reference's steps). Otherwise a final phase adds the last layer's partial sums the same way. Every
// order of additions is fixed and a function of the layer shapes only, so results do not depend on scheduling or on
// how the batch is cut. fp32 accumulation over K <= 8192 stays within ~1e-6 of the exact product, inside the
// dense-MLP bound of 1e-5.
//
// The grid barrier counts arrivals in bar[0]; the last arriver resets it and advances the generation bar[1], on which
// the others wait (bounded: a timeout writes KX_STATUS_TIMEOUT and the CTA leaves; the runtime then zeroes both
// words), so the words need no clearing between launches. Each CTA reads the generation once when it starts: it
// advances only when every CTA has arrived, so even a CTA that starts after the others have reached the first barrier
// reads the value from before it (an arrival count read at the start would not be: a late CTA would see the others'
// arrivals). A cooperative launch makes every CTA resident at once.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kx_act.cuh"
#include "kx_kernels.h"
#include "kx_sm100.cuh"

namespace {

constexpr int MT = 64, NT = 64, KC = 32, THREADS = 256, WARPS = THREADS / 32;
constexpr int NSTAGE = 8;                                    // first-layer chunks in flight
constexpr int AS_LD = KC + 4;                                // ring A stage: row-major, 144-byte rows
constexpr int STAGE_FLOATS = MT * AS_LD + KC * NT;           // one ring stage: A then W
constexpr int RING_FLOATS = NSTAGE * STAGE_FLOATS;           // also holds the register path's double buffers
constexpr int REG_FLOATS = 2 * KC * (MT + 4) + 2 * KC * NT;
constexpr int FUSE_MAX_K = 1024, FUSE_MAX_W = 8192, FUSE_MAX_N = 64;  // a last layer run per row by the final phase
constexpr size_t SMEM_BYTES = sizeof(float) * (RING_FLOATS + FUSE_MAX_W + WARPS * FUSE_MAX_K);
static_assert(REG_FLOATS <= RING_FLOATS, "the register path's buffers live in the ring");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");

struct MlpLayer {
    const float* w;  // k x n, row-major (in x out)
    const float* b;  // n, or nullptr
    float* part;     // split x M x n partial sums (nullptr for a last layer run by the final phase)
    int k, n, split, act;
    float alpha;
};

struct MlpChain {
    MlpLayer L[KX_MLP_MAX_LAYERS];
    int n_layers;
    int ring;  // the first layer streams through the cp.async ring
    int fuse;  // the last layer runs per row in the final phase
    const float* x;
    int ldx;
    float* y;
    int M;
    int softmax;
    uint32_t* bar;  // [0] arrivals at the current barrier, [1] generation
    int* status;
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(kx::smem_u32(dst)), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(kx::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ float f4(const float4& v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// bounded grid barrier over gridDim.x CTAs, passed when the generation reaches `target`; false (status set) if it
// gave up
__device__ bool grid_barrier(uint32_t* bar, uint32_t target, int* status, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        bool ok = true;
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const uint64_t t0 = kx::globaltimer();
            for (uint32_t spin = 0; static_cast<int>(kx::ld_acquire_gpu(bar + 1) - target) < 0; spin++) {
                if ((spin & 15) == 15) {
                    if (kx::globaltimer() - t0 > KX_WAIT_NS) {
                        if (status) atomicExch(status, KX_STATUS_TIMEOUT);
                        ok = false;
                        break;
                    }
                    __nanosleep(32);
                }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// the sum over the K ranges of a layer's partial sums at element offset `off` (four floats when v4), added in range
// order; every range's load is issued before the first add
__device__ __forceinline__ float4 sum_parts4(const MlpLayer& p, size_t plane, size_t off, bool v4, int valid) {
    float4 t[KX_MLP_MAX_SPLIT];
#pragma unroll
    for (int q = 0; q < KX_MLP_MAX_SPLIT; q++) {
        if (q >= p.split) break;
        const float* src = p.part + q * plane + off;
        if (v4) {
            t[q] = __ldcg(reinterpret_cast<const float4*>(src));
        } else {
            t[q].x = valid > 0 ? __ldcg(src) : 0.f;
            t[q].y = valid > 1 ? __ldcg(src + 1) : 0.f;
            t[q].z = valid > 2 ? __ldcg(src + 2) : 0.f;
            t[q].w = valid > 3 ? __ldcg(src + 3) : 0.f;
        }
    }
    float4 s = t[0];
#pragma unroll
    for (int q = 1; q < KX_MLP_MAX_SPLIT; q++) {
        if (q >= p.split) break;
        s = make_float4(__fadd_rn(s.x, t[q].x), __fadd_rn(s.y, t[q].y), __fadd_rn(s.z, t[q].z), __fadd_rn(s.w, t[q].w));
    }
    return s;
}

// the activations other than ReLU and identity, out of line (the loops that call them stay small in the
// instruction cache)
__device__ __noinline__ float act_slow(int act, float v, float alpha) { return kx::act_apply(act, v, alpha); }

// act(sum + bias) of a layer's output element c (the value the next layer reads)
__device__ __forceinline__ float finish1(const MlpLayer& p, float sum, int c) {
    const float t = p.b ? __fadd_rn(sum, __ldg(p.b + c)) : sum;
    if (p.act == kx::ACT_RELU) return t < 0.0f ? 0.0f : t;
    if (p.act == kx::ACT_NONE) return t;
    return act_slow(p.act, t, p.alpha);
}

// four input elements (row r, columns k..k+3) of layer l: the chain input, or the previous layer's finished output
__device__ __forceinline__ float4 load_a4(const MlpChain& c, int l, int r, int k, int kend) {
    if (r >= c.M || k >= kend) return make_float4(0.f, 0.f, 0.f, 0.f);
    const int valid = kend - k < 4 ? kend - k : 4;
    if (l == 0) {
        const float* src = c.x + static_cast<size_t>(r) * c.ldx + k;
        if (valid == 4) return __ldg(reinterpret_cast<const float4*>(src));
        return make_float4(__ldg(src), valid > 1 ? __ldg(src + 1) : 0.f, valid > 2 ? __ldg(src + 2) : 0.f, 0.f);
    }
    const MlpLayer& p = c.L[l - 1];
    const float4 s = sum_parts4(p, static_cast<size_t>(c.M) * p.n, static_cast<size_t>(r) * p.n + k, valid == 4, valid);
    return make_float4(finish1(p, s.x, k), valid > 1 ? finish1(p, s.y, k + 1) : 0.f, valid > 2 ? finish1(p, s.z, k + 2) : 0.f,
                       valid > 3 ? finish1(p, s.w, k + 3) : 0.f);
}

// four weights (row k, columns n..n+3) of layer l, zero outside
__device__ __forceinline__ float4 load_w4(const MlpLayer& L, int k, int kend, int n) {
    if (k >= kend) return make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = L.w + static_cast<size_t>(k) * L.n + n;
    if (n + 3 < L.n && (L.n & 3) == 0) return __ldg(reinterpret_cast<const float4*>(src));
    float v[4];
    for (int j = 0; j < 4; j++) v[j] = n + j < L.n ? __ldg(src + j) : 0.f;
    return make_float4(v[0], v[1], v[2], v[3]);
}

// one 64 x 64 item of the first layer over K range [k0, k1) through the cp.async ring (x and the weights 16-byte
// aligned, k and n multiples of 4: every 16-byte copy lies wholly inside or wholly outside, the latter zero-filled).
// Per output the products are added in increasing k, as on the register path.
__device__ __forceinline__ void item_ring(const MlpChain& c, const MlpLayer& L, int m0, int n0, int k0, int k1, float* ring,
                                          float (&acc)[4][4]) {
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int nch = (k1 - k0 + KC - 1) / KC;
    auto issue = [&](int ch) {
        float* sa = ring + (ch % NSTAGE) * STAGE_FLOATS;
        float* sw = sa + MT * AS_LD;
        const int kb = k0 + ch * KC;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int idx = tid + j * THREADS;
            const int row = idx >> 3, kq = (idx & 7) * 4;  // A: 64 rows x 8 float4
            const bool oka = m0 + row < c.M && kb + kq < k1;
            cp_async16(sa + row * AS_LD + kq, oka ? c.x + static_cast<size_t>(m0 + row) * c.ldx + kb + kq : c.x, oka ? 16 : 0);
            const int kr = idx >> 4, nq = (idx & 15) * 4;  // W: 32 k rows x 16 float4
            const bool okw = kb + kr < k1 && n0 + nq < L.n;
            cp_async16(sw + kr * NT + nq, okw ? L.w + static_cast<size_t>(kb + kr) * L.n + n0 + nq : L.w, okw ? 16 : 0);
        }
    };
    for (int s = 0; s < NSTAGE; s++) {
        if (s < nch) issue(s);
        cp_async_commit();
    }
    for (int ch = 0; ch < nch; ch++) {
        cp_async_wait<NSTAGE - 1>();  // NSTAGE + ch groups committed: chunk ch's has landed
        __syncthreads();
        const float* sa = ring + (ch % NSTAGE) * STAGE_FLOATS;
        const float* sw = sa + MT * AS_LD;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 4) {
            float4 a[4], w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = *reinterpret_cast<const float4*>(sa + (4 * ty + i) * AS_LD + kk);
#pragma unroll
            for (int j = 0; j < 4; j++) w[j] = *reinterpret_cast<const float4*>(sw + (kk + j) * NT + 4 * tx);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float wv[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float av = f4(a[i], j);
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) acc[i][jj] = fmaf(av, wv[jj], acc[i][jj]);
                }
            }
        }
        if (ch + NSTAGE < nch) {  // the stage just read takes chunk ch + NSTAGE
            __syncthreads();
            issue(ch + NSTAGE);
        }
        cp_async_commit();
    }
}

// row softmax of a warp's row (lane holds columns lane and lane + 32, -inf outside the n columns) into row
__device__ __forceinline__ void softmax_row(float (&o)[2], int n, int lane, float* row) {
    float mx = o[0] > o[1] ? o[0] : o[1];
    for (int off = 16; off > 0; off >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, mx, off);
        mx = t > mx ? t : mx;
    }
    float sum = 0.f;
    for (int h = 0; h < 2; h++) {
        const int col = lane + 32 * h;
        o[h] = col < n ? expf(__fsub_rn(o[h], mx)) : 0.f;
        sum = __fadd_rn(sum, o[h]);
    }
    for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
    const float inv = __fdiv_rn(1.0f, sum);
    for (int h = 0; h < 2; h++) {
        const int col = lane + 32 * h;
        if (col < n) row[col] = __fmul_rn(o[h], inv);
    }
}

__global__ void __launch_bounds__(THREADS) k_mlp_chain(const MlpChain c) {
    extern __shared__ __align__(16) float smem[];
    __shared__ int s_ok;
    float(*As)[KC][MT + 4] = reinterpret_cast<float(*)[KC][MT + 4]>(smem);  // register path: k-major A, padded
    float(*Ws)[KC][NT] = reinterpret_cast<float(*)[KC][NT]>(smem + 2 * KC * (MT + 4));
    float* const wf = smem + RING_FLOATS;  // the last layer's weights when the final phase runs it
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int ar = tid >> 2, akq = (tid & 3) * 4;  // A staging: row, first k of the thread's four (+16 for the second)
    const int wk = tid >> 4, wn = (tid & 15) * 4;  // W staging: k row (+16 for the second), first of four columns
    const int n_gemm = c.n_layers - c.fuse;
    uint32_t gen = 0;  // the generation before this launch's first barrier (thread 0 waits on it)
    if (tid == 0) gen = kx::ld_acquire_gpu(c.bar + 1);
    // in flight while the first layer runs: the last layer's weights into shared memory, later layers' towards L2
    if (c.fuse) {
        const MlpLayer& F = c.L[c.n_layers - 1];
        for (int i = tid; i < F.k * F.n; i += THREADS) cp_async4(wf + i, F.w + i);
        cp_async_commit();
    }
    for (int l = 1; l < n_gemm; l++) {
        const char* w = reinterpret_cast<const char*>(c.L[l].w);
        const size_t lines = (static_cast<size_t>(c.L[l].k) * c.L[l].n * sizeof(float) + 127) / 128;
        for (size_t i = static_cast<size_t>(blockIdx.x) * THREADS + tid; i < lines; i += static_cast<size_t>(gridDim.x) * THREADS)
            prefetch_l2(w + i * 128);
    }
    for (int l = 0; l < n_gemm; l++) {
        const MlpLayer& L = c.L[l];
        const int m_tiles = (c.M + MT - 1) / MT, n_tiles = (L.n + NT - 1) / NT;
        const int items = m_tiles * n_tiles * L.split;
        const int kc = (L.k + L.split - 1) / L.split, kcr = (kc + KC - 1) / KC * KC;  // K per range, rounded to chunks
        for (int it = blockIdx.x; it < items; it += gridDim.x) {
            const int s = it % L.split, tile = it / L.split;
            const int mt = tile % m_tiles, nt = tile / m_tiles;
            const int m0 = mt * MT, n0 = nt * NT;
            const int k0 = s * kcr, k1 = min(L.k, k0 + kcr);
            float acc[4][4] = {};
            if (l == 0 && c.ring) {
                item_ring(c, L, m0, n0, k0, k1, smem, acc);
            } else {
                float4 ra0 = load_a4(c, l, m0 + ar, k0 + akq, k1), ra1 = load_a4(c, l, m0 + ar, k0 + 16 + akq, k1);
                float4 rw0 = load_w4(L, k0 + wk, k1, n0 + wn), rw1 = load_w4(L, k0 + 16 + wk, k1, n0 + wn);
                int buf = 0;
                for (int kb = k0; kb < k1; kb += KC) {
                    const float a0[4] = {ra0.x, ra0.y, ra0.z, ra0.w}, a1[4] = {ra1.x, ra1.y, ra1.z, ra1.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        As[buf][akq + j][ar] = a0[j];
                        As[buf][16 + akq + j][ar] = a1[j];
                    }
                    *reinterpret_cast<float4*>(&Ws[buf][wk][wn]) = rw0;
                    *reinterpret_cast<float4*>(&Ws[buf][16 + wk][wn]) = rw1;
                    __syncthreads();
                    if (kb + KC < k1) {  // the next chunk's loads fly while this one is multiplied
                        ra0 = load_a4(c, l, m0 + ar, kb + KC + akq, k1);
                        ra1 = load_a4(c, l, m0 + ar, kb + KC + 16 + akq, k1);
                        rw0 = load_w4(L, kb + KC + wk, k1, n0 + wn);
                        rw1 = load_w4(L, kb + KC + 16 + wk, k1, n0 + wn);
                    }
#pragma unroll
                    for (int kk = 0; kk < KC; kk++) {
                        const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk][4 * ty]);
                        const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][kk][4 * tx]);
                        const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int i = 0; i < 4; i++)
#pragma unroll
                            for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
                    }
                    buf ^= 1;  // the other buffer is free: every thread passed the barrier above after reading it
                }
            }
            const int nc = n0 + 4 * tx;  // partial sums of this K range
            float* dst = L.part + static_cast<size_t>(s) * c.M * L.n;
            for (int i = 0; i < 4; i++) {
                const int r = m0 + 4 * ty + i;
                if (r >= c.M) continue;
                float* row = dst + static_cast<size_t>(r) * L.n;
                if (nc + 3 < L.n && (L.n & 3) == 0) {
                    __stcg(reinterpret_cast<float4*>(row + nc), make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]));
                } else {
                    for (int j = 0; j < 4; j++)
                        if (nc + j < L.n) __stcg(row + nc + j, acc[i][j]);
                }
            }
            __syncthreads();  // the staging buffers are reused by the next item
        }
        if (!grid_barrier(c.bar, gen + l + 1, c.status, &s_ok)) {
            cp_async_wait<0>();
            return;
        }
    }
    const int warp = tid >> 5, lane = tid & 31;
    if (c.fuse) {
        // final phase, narrow last layer F: one warp per row forms the row's inputs (F's k = the previous layer's n, a
        // multiple of 4) into shared memory, then lane o computes output o (and o + 32)
        cp_async_wait<0>();
        __syncthreads();
        const MlpLayer& P = c.L[c.n_layers - 2];
        const MlpLayer& F = c.L[c.n_layers - 1];
        const size_t plane = static_cast<size_t>(c.M) * P.n;
        float* h = smem + RING_FLOATS + FUSE_MAX_W + warp * FUSE_MAX_K;
        for (int r = blockIdx.x * WARPS + warp; r < c.M; r += gridDim.x * WARPS) {
            for (int k4 = 4 * lane; k4 < F.k; k4 += 128) {
                const float4 sm = sum_parts4(P, plane, static_cast<size_t>(r) * P.n + k4, true, 4);
                *reinterpret_cast<float4*>(h + k4) = make_float4(finish1(P, sm.x, k4), finish1(P, sm.y, k4 + 1),
                                                                 finish1(P, sm.z, k4 + 2), finish1(P, sm.w, k4 + 3));
            }
            __syncwarp();
            float o[2];
            for (int hh = 0; hh < 2; hh++) {
                const int col = lane + 32 * hh;
                o[hh] = -INFINITY;
                if (col < F.n) {
                    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                    const float* wc = wf + col;
                    for (int k = 0; k < F.k; k += 4) {
                        const float4 hv = *reinterpret_cast<const float4*>(h + k);
                        a0 = fmaf(hv.x, wc[k * F.n], a0);
                        a1 = fmaf(hv.y, wc[(k + 1) * F.n], a1);
                        a2 = fmaf(hv.z, wc[(k + 2) * F.n], a2);
                        a3 = fmaf(hv.w, wc[(k + 3) * F.n], a3);
                    }
                    o[hh] = finish1(F, __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), col);
                }
            }
            __syncwarp();  // the row's inputs are rewritten for the warp's next row
            float* row = c.y + static_cast<size_t>(r) * F.n;
            if (c.softmax) {
                softmax_row(o, F.n, lane, row);
            } else {
                for (int hh = 0; hh < 2; hh++)
                    if (lane + 32 * hh < F.n) row[lane + 32 * hh] = o[hh];
            }
        }
        return;
    }
    // final phase: the last layer's sums, bias and activation (and the row softmax), one warp per row at a time
    const MlpLayer& L = c.L[c.n_layers - 1];
    const size_t plane = static_cast<size_t>(c.M) * L.n;
    for (int r = blockIdx.x * WARPS + warp; r < c.M; r += gridDim.x * WARPS) {
        float* row = c.y + static_cast<size_t>(r) * L.n;
        if (!c.softmax) {
            for (int col = 4 * lane; col < L.n; col += 128) {
                const int valid = L.n - col < 4 ? L.n - col : 4;
                const float4 sm = sum_parts4(L, plane, static_cast<size_t>(r) * L.n + col, valid == 4 && (L.n & 3) == 0, valid);
                const float v[4] = {sm.x, sm.y, sm.z, sm.w};
                for (int j = 0; j < valid; j++) row[col + j] = finish1(L, v[j], col + j);
            }
            continue;
        }
        // softmax rows have at most 64 columns: lane holds columns lane and lane + 32
        float o[2];
        for (int h = 0; h < 2; h++) {
            const int col = lane + 32 * h;
            o[h] = -INFINITY;
            if (col < L.n) {
                const float4 sm = sum_parts4(L, plane, static_cast<size_t>(r) * L.n + col, false, 1);
                o[h] = finish1(L, sm.x, col);
            }
        }
        softmax_row(o, L.n, lane, row);
    }
}

int g_mlp_grid = 0, g_mlp_dev = -1;

int mlp_grid() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_mlp_dev != dev) {
        int per_sm = 0, sms = 0;
        if (cudaFuncSetAttribute(k_mlp_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM_BYTES)) !=
                cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_mlp_chain, THREADS, SMEM_BYTES) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        g_mlp_grid = per_sm * sms;
        g_mlp_dev = dev;
    }
    return g_mlp_grid;
}

// K ranges of a layer with k inputs and n outputs: as many as keep a 256-row batch (4 row tiles) within one item per
// SM, at most one range per K chunk, none empty. A function of (k, n) only, so a row's sums never depend on the
// batch size.
int k_ranges(int k, int n) {
    const int tiles = 4 * ((n + NT - 1) / NT);
    int split = 148 / tiles;
    if (split < 1) split = 1;
    if (split > KX_MLP_MAX_SPLIT) split = KX_MLP_MAX_SPLIT;
    const int kmax = (k + KC - 1) / KC;
    if (split > kmax) split = kmax;
    while (split > 1 && (split - 1) * (((k + split - 1) / split + KC - 1) / KC * KC) >= k) split--;
    return split;
}

// 1 if the final phase runs the last layer per row (a narrow head after at least one other layer)
int fuse_last(const int* k, const int* n, int n_layers) {
    const int kl = k[n_layers - 1], nl = n[n_layers - 1];
    return n_layers >= 2 && nl <= FUSE_MAX_N && kl <= FUSE_MAX_K && kl * nl <= FUSE_MAX_W && kl % 4 == 0;
}

}  // namespace

extern "C" {

size_t kx_mlp_chain_scratch_floats(int m, const int* k, const int* n, int n_layers) {
    size_t total = 0;
    const int n_gemm = n_layers - fuse_last(k, n, n_layers);
    for (int l = 0; l < n_gemm; l++) total += static_cast<size_t>(k_ranges(k[l], n[l])) * m * n[l];
    return total;
}

int kx_mlp_chain(const float* x, int ldx, int m, int n_layers, const float* const* w, const float* const* bias, const int* k,
                 const int* n, const int* act, const float* alpha, int softmax, float* y, float* scratch, uint32_t* bar,
                 int* status, void* stream) {
    if (m <= 0) return 0;
    if (n_layers < 1 || n_layers > KX_MLP_MAX_LAYERS || x == nullptr || y == nullptr || bar == nullptr || ldx < k[0] ||
        (ldx & 3) || (reinterpret_cast<uintptr_t>(x) & 15) || (softmax && n[n_layers - 1] > 64) || scratch == nullptr ||
        (reinterpret_cast<uintptr_t>(scratch) & 15))
        return -1;
    for (int l = 0; l < n_layers; l++)
        if ((n[l] & 3) && l + 1 < n_layers) return -1;  // a layer's output is read four at a time by the next
    const int grid_max = mlp_grid();
    if (grid_max <= 0) return -1;
    MlpChain c{};
    c.n_layers = n_layers;
    c.fuse = fuse_last(k, n, n_layers);
    c.ring = k[0] % 4 == 0 && n[0] % 4 == 0 && (reinterpret_cast<uintptr_t>(w[0]) & 15) == 0;
    c.x = x;
    c.ldx = ldx;
    c.y = y;
    c.M = m;
    c.softmax = softmax;
    c.bar = bar;
    c.status = status;
    int items_max = 1;
    float* part = scratch;
    for (int l = 0; l < n_layers; l++) {
        if (k[l] <= 0 || n[l] <= 0 || (l > 0 && k[l] != n[l - 1]) || w[l] == nullptr) return -1;
        const bool gemm = l < n_layers - c.fuse;
        const int split = gemm ? k_ranges(k[l], n[l]) : 1;
        c.L[l] = MlpLayer{w[l], bias[l], gemm ? part : nullptr, k[l], n[l], split, act[l], alpha[l]};
        if (!gemm) continue;
        part += static_cast<size_t>(split) * m * n[l];
        const int tiles = ((m + MT - 1) / MT) * ((n[l] + NT - 1) / NT);
        if (tiles * split > items_max) items_max = tiles * split;
    }
    const int grid = items_max < grid_max ? items_max : grid_max;
    void* args[] = {&c};
    if (cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(k_mlp_chain), dim3(grid), dim3(THREADS), args, SMEM_BYTES,
                                    static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return 0;
}

}  // extern "C"
