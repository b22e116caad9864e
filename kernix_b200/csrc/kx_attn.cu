// KERNIX-B200 attention core on the 5th-generation tensor cores, for the short sequences of the reference's
// ATTENTION step (kernix_attention_run, include/kernix_model.h:1005-1048): per (sample, head)
//   S = scale * (Q . K^T)   (optional causal mask: key j > query row -> -inf)
//   P = row softmax(S)      (max, e = exp(s - max), sum, p = e * (1 / sum))
//   ctx = P . V
// with at most 128 queries, 128 keys and head dims of at most 64 (the c4 encoder: 128 / 128 / 64).
//
// One CTA of 512 threads (16 warps) per (sample, head). Warp w works on TMEM lane quarter q = w % 4 (rows
// 32 q .. 32 q + 31) and column group g = w / 4. Both products run in 3xTF32 (a.b = ah.bh + (al.bh + ah.bl), the
// split of kx::tf32_split) as single-CTA tcgen05.mma with M = 128, the large ah.bh sums and the small cross terms in
// separate TMEM accumulators (the truncating accumulation of tcgen05 then costs ~1e-7 at these K <= 128):
//   1. all threads load Q, K (row = query / key, K index = head dim) and V with every load in flight at once, split
//      every value into hi / lo and store Q and K in the canonical K-major 128-byte-swizzle layout as 128-row tiles of
//      32 floats of K;
//   2. thread 0 issues S = Q . K^T (N = 128 keys) into TMEM columns [0, 128) (ah.bh) and [128, 256) (cross terms),
//      while the threads store V transposed (rows = head dim, K index = key), the B operand of P . V;
//   3. row r's scores are shared by the four warps of its quarter, 32 keys each (tcgen05.ld of 32 columns): each
//      finds its partial max, the four meet through shared memory (max; then the sum of e = exp(s - max), added in
//      key-group order), and p = e * (1 / sum) is split into hi / lo and written as the A operand tiles of P . V over
//      the Q / K tiles, whose MMAs have completed;
//   4. thread 0 issues ctx = P . V (N = 64) into TMEM columns [256, 320) and [320, 384);
//   5. warp (q, g) adds the two accumulators of rows 32 q .. 32 q + 31, head-dim columns 16 g .. 16 g + 15, and
//      stores them.
// Every wait is bounded; a timeout records KX_STATUS_TIMEOUT in the status word and the CTA stores nothing.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kx_kernels.h"
#include "kx_sm100.cuh"

namespace {

constexpr int AT_MAX = 128;                 // queries and keys per (sample, head), at most
constexpr int AT_THREADS = 512;
constexpr int AT_DMAX = 64;                 // head dims, at most
constexpr int AT_TILE = AT_MAX * 128;       // a 128-row x 128-byte tile (32 floats of K): 16 KB
constexpr int AT_VTILE = AT_DMAX * 128;     // a 64-row x 128-byte tile of V^T: 8 KB
constexpr int AT_QK_BYTES = 8 * AT_TILE;    // Q hi/lo and K hi/lo (2 tiles each), later P hi/lo (4 tiles each)
constexpr int AT_V_BYTES = 8 * AT_VTILE;    // V^T hi/lo, 4 tiles each
struct AtCtl {
    uint64_t bar;
    uint32_t tmem;
    int abort;
    float red[4][AT_MAX];  // per key group g and row: partial max, then partial sum
};
constexpr int AT_SMEM = AT_QK_BYTES + AT_V_BYTES + 1024 + static_cast<int>(sizeof(AtCtl));
constexpr uint32_t AT_S_MAIN = 0, AT_S_CROSS = 128, AT_O_MAIN = 256, AT_O_CROSS = 320, AT_TMEM_COLS = 512;

// byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ float4 load_row4(const float* src, int d, int dmax, bool vec) {
    if (d >= dmax) return make_float4(0.f, 0.f, 0.f, 0.f);
    if (vec && d + 3 < dmax) return __ldg(reinterpret_cast<const float4*>(src + d));
    return make_float4(__ldg(src + d), d + 1 < dmax ? __ldg(src + d + 1) : 0.f, d + 2 < dmax ? __ldg(src + d + 2) : 0.f,
                       d + 3 < dmax ? __ldg(src + d + 3) : 0.f);
}

__device__ __forceinline__ void split4(const float4& v, float4& h, float4& l) {
    kx::tf32_split(v.x, h.x, l.x);
    kx::tf32_split(v.y, h.y, l.y);
    kx::tf32_split(v.z, h.z, l.z);
    kx::tf32_split(v.w, h.w, l.w);
}

// bounded wait for phase `parity` of the CTA's barrier; false after a timeout (recorded in *status)
__device__ __forceinline__ bool at_wait(AtCtl* ctl, uint32_t parity, int* status) {
    return kx::mbar_wait(&ctl->bar, parity, &ctl->abort, status);
}

__global__ void __launch_bounds__(AT_THREADS, 1)
k_attention_tc(const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk, const float* __restrict__ v,
               int ldv, float* __restrict__ ctx, int ldc, int Rq, int S, int dk, int dv, int causal, float scale,
               int ahead, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    AtCtl* ctl = reinterpret_cast<AtCtl*>(smem + AT_QK_BYTES + AT_V_BYTES);
    uint8_t* qk = smem;                   // Q hi t0,t1 | Q lo t0,t1 | K hi t0,t1 | K lo t0,t1; then P hi t0..3 | P lo t0..3
    uint8_t* vt = smem + AT_QK_BYTES;     // V^T hi t0..3 | V^T lo t0..3
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, grp = warp >> 2;
    const int h = blockIdx.x, b = blockIdx.y;
    const float* qb = q + static_cast<long>(b) * Rq * ldq + h * dk;
    const float* kb = k + static_cast<long>(b) * S * ldk + h * dk;
    const float* vb = v + static_cast<long>(b) * S * ldv + h * dv;
    const bool vq = ((ldq | dk) & 3) == 0 && (reinterpret_cast<uintptr_t>(qb) & 15) == 0;
    const bool vk = ((ldk | dk) & 3) == 0 && (reinterpret_cast<uintptr_t>(kb) & 15) == 0;
    const bool vv = ((ldv | dv) & 3) == 0 && (reinterpret_cast<uintptr_t>(vb) & 15) == 0;

    if (tid == 0) {
        kx::mbar_init(&ctl->bar, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
    }
    if (warp == 0) {
        kx::tmem_alloc(&ctl->tmem, AT_TMEM_COLS);
        kx::tmem_relinquish();
    }

    // 1. operands, every load issued before the first store. Q and K: thread t handles the float4s
    // (row, d4) = (i / 16, i % 16), i = t + 512 u (a half-warp reads one row's 256 contiguous bytes). V: warp w takes
    // keys 32 (w % 4) + lane and head dims 16 (w / 4) .. +15, so each scalar store into a row of V^T covers 32
    // consecutive keys (one 128-byte row of a tile: conflict-free).
    constexpr int NQ = AT_MAX * 16 / AT_THREADS;  // float4s of Q (and of K) per thread
    float4 xq[NQ], xk[NQ], xv[4];
#pragma unroll
    for (int u = 0; u < NQ; u++) {
        const int i = u * AT_THREADS + tid, row = i >> 4, d = (i & 15) * 4;
        xq[u] = row < Rq ? load_row4(qb + static_cast<long>(row) * ldq, d, dk, vq) : make_float4(0.f, 0.f, 0.f, 0.f);
        xk[u] = row < S ? load_row4(kb + static_cast<long>(row) * ldk, d, dk, vk) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int vj = quarter * 32 + lane, vd0 = grp * 16;
#pragma unroll
    for (int u = 0; u < 4; u++)
        xv[u] = vj < S ? load_row4(vb + static_cast<long>(vj) * ldv, vd0 + 4 * u, dv, vv) : make_float4(0.f, 0.f, 0.f, 0.f);
    // While these loads are in flight, ask L2 for the rows of the (sample, head) that will most likely run on this
    // SM next (`ahead` CTAs later in launch order: one CTA per SM at a time), so that its loads hit L2 instead of
    // paying a full DRAM round trip at its start. One 128-byte line per thread and row segment, rows of Q, K, V.
    if (ahead > 0) {
        const long nxt = static_cast<long>(b) * gridDim.x + h + ahead;
        if (nxt < static_cast<long>(gridDim.x) * gridDim.y) {
            const int hn = static_cast<int>(nxt % gridDim.x), bn = static_cast<int>(nxt / gridDim.x);
            const int lq = (dk * 4 + 127) / 128, lv = (dv * 4 + 127) / 128;  // lines per row segment
            for (int i = tid; i < Rq * lq + S * lq + S * lv; i += AT_THREADS) {
                const float* p;
                if (i < Rq * lq) p = q + (static_cast<long>(bn) * Rq + i / lq) * ldq + hn * dk + 32 * (i % lq);
                else if (i < Rq * lq + S * lq) {
                    const int j = i - Rq * lq;
                    p = k + (static_cast<long>(bn) * S + j / lq) * ldk + hn * dk + 32 * (j % lq);
                } else {
                    const int j = i - Rq * lq - S * lq;
                    p = v + (static_cast<long>(bn) * S + j / lv) * ldv + hn * dv + 32 * (j % lv);
                }
                kx::prefetch_l2(p);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < NQ; u++) {
        const int i = u * AT_THREADS + tid, row = i >> 4, d4 = i & 15;
        const uint32_t off = (d4 >> 3) * AT_TILE + swz(row, d4 & 7);
        float4 hv, lv;
        split4(xq[u], hv, lv);
        *reinterpret_cast<float4*>(qk + off) = hv;
        *reinterpret_cast<float4*>(qk + 2 * AT_TILE + off) = lv;
        split4(xk[u], hv, lv);
        *reinterpret_cast<float4*>(qk + 4 * AT_TILE + off) = hv;
        *reinterpret_cast<float4*>(qk + 6 * AT_TILE + off) = lv;
    }
    kx::fence_proxy_async_smem();
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    const uint32_t base = kx::smem_u32(smem);

    // 2. S = Q . K^T
    if (tid == 0) {
        constexpr uint32_t idesc = kx::idesc_tf32(AT_MAX, AT_MAX);
        const int nks = (dk + 7) / 8;
        for (int ks = 0; ks < nks; ks++) {
            const uint32_t o = (ks >> 2) * AT_TILE + (ks & 3) * 32;
            const uint32_t ah = base + o, al = base + 2 * AT_TILE + o, bh = base + 4 * AT_TILE + o, bl = base + 6 * AT_TILE + o;
            kx::mma_tf32(tmem + AT_S_CROSS, kx::desc_sw128_kmajor(al), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
            kx::mma_tf32(tmem + AT_S_CROSS, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bl), idesc, 1);
            kx::mma_tf32(tmem + AT_S_MAIN, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
        }
        kx::mma_commit(&ctl->bar);
    }
    __syncwarp();
    // V^T while the S MMAs run (made visible to them by the barrier before P . V)
    {
        uint8_t* hi = vt + quarter * AT_VTILE;
        uint8_t* lo = vt + (4 + quarter) * AT_VTILE;
        const int c = lane >> 2, e4 = (lane & 3) * 4;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            float4 hv, lv;
            split4(xv[u], hv, lv);
            const float hh[4] = {hv.x, hv.y, hv.z, hv.w}, ll[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t off = swz(vd0 + 4 * u + e, c) + e4;
                *reinterpret_cast<float*>(hi + off) = hh[e];
                *reinterpret_cast<float*>(lo + off) = ll[e];
            }
        }
    }
    // the warps read TMEM with warp-collective loads: agree on the outcome first
    bool ok = __syncthreads_and(at_wait(ctl, 0, status)) != 0;
    int pending = ok ? -1 : 0;  // barrier phase a timed-out wait left behind
    kx::tc_fence_after();

    // 3. softmax: row r = 32 quarter + lane, keys 32 grp .. 32 grp + 31
    const int r = quarter * 32 + lane, key0 = grp * 32;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    float e[32];
    float m = -INFINITY;
    if (ok) {
        uint32_t mv[32], xv2[32];
        kx::tmem_ld32(tmem + lanes + AT_S_MAIN + key0, mv);
        kx::tmem_ld32(tmem + lanes + AT_S_CROSS + key0, xv2);
        kx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int key = key0 + j;
            const float t = __fmul_rn(__fadd_rn(__uint_as_float(mv[j]), __uint_as_float(xv2[j])), scale);
            e[j] = (key >= S || (causal && key > r)) ? -INFINITY : t;
            m = fmaxf(m, e[j]);
        }
        ctl->red[grp][r] = m;
    }
    __syncthreads();
    if (ok) {
        m = fmaxf(fmaxf(ctl->red[0][r], ctl->red[1][r]), fmaxf(ctl->red[2][r], ctl->red[3][r]));
#pragma unroll
        for (int j = 0; j < 32; j++) e[j] = expf(__fsub_rn(e[j], m));
    }
    __syncthreads();  // every partial max has been read before the partial sums overwrite them
    if (ok) {
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) part = __fadd_rn(part, e[j]);
        ctl->red[grp][r] = part;
    }
    __syncthreads();
    if (ok) {
        const float sum = __fadd_rn(__fadd_rn(__fadd_rn(ctl->red[0][r], ctl->red[1][r]), ctl->red[2][r]), ctl->red[3][r]);
        const float inv = __fdiv_rn(1.0f, sum);
        // P tile grp (keys 32 grp ..) over the Q / K tiles (every MMA that read them has completed); keys past S
        // have e = 0
        uint8_t* ph = qk + grp * AT_TILE;
        uint8_t* pl = qk + (4 + grp) * AT_TILE;
#pragma unroll
        for (int j4 = 0; j4 < 8; j4++) {
            const float4 p = make_float4(__fmul_rn(e[4 * j4], inv), __fmul_rn(e[4 * j4 + 1], inv), __fmul_rn(e[4 * j4 + 2], inv),
                                         __fmul_rn(e[4 * j4 + 3], inv));
            float4 hv, lv;
            split4(p, hv, lv);
            *reinterpret_cast<float4*>(ph + swz(r, j4)) = hv;
            *reinterpret_cast<float4*>(pl + swz(r, j4)) = lv;
        }
    }
    kx::fence_proxy_async_smem();
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();

    // 4. ctx = P . V (N = 64 head-dim columns, K = keys)
    if (tid == 0 && ok) {
        constexpr uint32_t idesc = kx::idesc_tf32(AT_MAX, AT_DMAX);
        const int nks = (S + 7) / 8;
        for (int ks = 0; ks < nks; ks++) {
            const uint32_t o = (ks >> 2) * AT_TILE + (ks & 3) * 32, ov = (ks >> 2) * AT_VTILE + (ks & 3) * 32;
            const uint32_t ah = base + o, al = base + 4 * AT_TILE + o;
            const uint32_t bh = base + AT_QK_BYTES + ov, bl = base + AT_QK_BYTES + 4 * AT_VTILE + ov;
            kx::mma_tf32(tmem + AT_O_CROSS, kx::desc_sw128_kmajor(al), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
            kx::mma_tf32(tmem + AT_O_CROSS, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bl), idesc, 1);
            kx::mma_tf32(tmem + AT_O_MAIN, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
        }
        kx::mma_commit(&ctl->bar);
    }
    __syncwarp();
    if (ok) {
        ok = __syncthreads_and(at_wait(ctl, 1, status)) != 0;
        if (!ok) pending = 1;
    }
    kx::tc_fence_after();

    // 5. ctx rows 32 quarter .. +31, head-dim columns 16 grp .. 16 grp + 15
    if (ok) {
        const int c0 = grp * 16;
        uint32_t mv[16], xv2[16];
        kx::tmem_ld16(tmem + lanes + AT_O_MAIN + c0, mv);
        kx::tmem_ld16(tmem + lanes + AT_O_CROSS + c0, xv2);
        kx::tmem_ld_wait();
        if (r < Rq && c0 < dv) {
            float* dst = ctx + (static_cast<long>(b) * Rq + r) * ldc + h * dv + c0;
            const int nv = dv - c0;
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; j++) o[j] = __fadd_rn(__uint_as_float(mv[j]), __uint_as_float(xv2[j]));
            if (nv >= 16 && ((ldc | dv) & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                for (int j4 = 0; j4 < 4; j4++)
                    reinterpret_cast<float4*>(dst)[j4] = make_float4(o[4 * j4], o[4 * j4 + 1], o[4 * j4 + 2], o[4 * j4 + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (j < nv) dst[j] = o[j];
            }
        }
    } else if (pending >= 0) {
        // the MMAs of the timed-out phase may still be running: give them time to finish (bounded) before the TMEM
        // and the shared memory go away
        const uint64_t t0 = kx::globaltimer();
        while (!kx::mbar_try_wait(&ctl->bar, static_cast<uint32_t>(pending)) && kx::globaltimer() - t0 < KX_WAIT_NS)
            __nanosleep(256);
    }
    kx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        kx::tc_fence_after();
        kx::tmem_dealloc(tmem, AT_TMEM_COLS);
    }
}

}  // namespace

// The tensor-core path of kx_attention (kx_ops.cu): 0 on success, 1 when the shape is not covered (the caller
// then runs its CUDA-core kernels), -1 on a launch error.
int kx_attention_tc(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* ctx, int ldc, int B,
                    int Rq, int S, int H, int dk, int dv, int causal, float scale, int* status, cudaStream_t st) {
    if (Rq > AT_MAX || S > AT_MAX || dk > AT_DMAX || dv > AT_DMAX || B > 65535) return 1;
    static unsigned long long devs_set = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(__atomic_load_n(&devs_set, __ATOMIC_ACQUIRE) & bit)) {
        if (cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM) != cudaSuccess)
            return -1;
        __atomic_fetch_or(&devs_set, bit, __ATOMIC_RELEASE);
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 0;
    dim3 grid(H, B);
    k_attention_tc<<<grid, AT_THREADS, AT_SMEM, st>>>(q, ldq, k, ldk, v, ldv, ctx, ldc, Rq, S, dk, dv, causal, scale, sms,
                                                      status);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
