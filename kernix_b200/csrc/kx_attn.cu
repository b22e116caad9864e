// KERNIX-B200 attention core on the 5th-generation tensor cores, for the short sequences of the reference's
// ATTENTION step (kernix_attention_run, include/kernix_model.h:1005-1048): per (sample, head)
//   S = scale * (Q . K^T)   (optional causal mask: key j > query row -> -inf)
//   P = row softmax(S)      (max, e = exp(s - max), sum, p = e * (1 / sum))
//   ctx = P . V
// with at most 128 queries, 128 keys and head dims of at most 64 (the c4 encoder: 128 / 128 / 64).
//
// A persistent kernel: one CTA of 512 threads (16 warps) per SM walks the (sample, head) pairs p = blockIdx.x,
// + gridDim.x, ... Warp w works on TMEM lane quarter q = w % 4 (rows 32 q .. 32 q + 31) and column group g = w / 4.
// Both products run in 3xTF32 (a.b = ah.bh + al.bh + ah.bl, the split of kx::tf32_split) as single-CTA tcgen05.mma
// with M = 128, the three products of a pair summed in one TMEM accumulator (<= 48 accumulated MMAs: ~1e-6 of the
// truncating accumulation). Per pair, with the pair's Q, K, V rows already in registers:
//   1. every thread splits its Q and K values into hi / lo and stores them in the canonical K-major 128-byte-swizzle
//      layout as 128-row tiles of 32 floats of K;
//   2. thread 0 issues S = Q . K^T (N = 128 keys) into TMEM columns [0, 128), while the threads store V transposed
//      (rows = head dim, K index = key), the B operand of P . V; the NEXT pair's rows are then loaded into the same
//      registers in three parts (Q here, K after the softmax's partial maxima, V after the P . V MMAs are issued), so
//      that no part stalls its warps on the load queue and the loads complete behind this pair's MMAs and softmax;
//   3. row r's scores are shared by the four warps of its quarter, 32 keys each (one tcgen05.ld of 32 columns): each
//      finds its partial max, the four meet through shared memory (max; then the sum of e = exp(s - max), added in
//      key-group order; the scores are kept in base-2 units, s log2(e), so e is one ex2.approx, ~2 ulp), and
//      p = e * (1 / sum) is split into hi / lo and written as the A operand tiles of P . V over the Q / K tiles,
//      whose MMAs have completed;
//   4. thread 0 issues ctx = P . V (N = 64) into TMEM columns [128, 192);
//   5. warp (q, g) takes rows 32 q .. 32 q + 31, head-dim columns 16 g .. 16 g + 15 of ctx out of TMEM and stages
//      them in the V^T tiles (free once P . V has completed); when the quarter's rows are staged, whole rows go to
//      global memory by bulk copies (cp.async.bulk) that run while the next pair starts (plain stores where rows are
//      not 16-byte aligned). The softmax's exchanges between the four warps of a quarter use a barrier per quarter.
// Every wait is bounded; a timeout records KX_STATUS_TIMEOUT in the status word and the CTA stops.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kx_act.cuh"
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
constexpr uint32_t AT_S = 0, AT_O = 128, AT_TMEM_COLS = 256;
constexpr int AT_CROW = 272;  // bytes per staged ctx row (64 floats + 16: 16-byte aligned, fewer bank conflicts)
static_assert(AT_MAX * AT_CROW <= AT_V_BYTES, "the staged ctx rows fit in the V^T tiles");
constexpr int AT_NQ = AT_MAX * 16 / AT_THREADS;  // float4s of Q (and of K) per thread

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

struct AtArgs {
    const float* q;
    const float* k;
    const float* v;
    float* ctx;
    int ldq, ldk, ldv, ldc, Rq, S, H, dk, dv, causal, pairs;
    float scale;
};

// The rows of pair p into registers, in three calls (Q, K, V: 32 KB per CTA each) made at different points of the
// previous pair, so that no call puts more loads in flight than the load queue takes without stalling its warps.
// Q and K as float4s (row, d4) = (i / 16, i % 16), i = t + 512 u (a half-warp reads one row's 256 contiguous bytes);
// V as keys 32 (w % 4) + lane, head dims 16 (w / 4) .. +15.
__device__ __forceinline__ void at_load_qk(const float* base, int ld, int rows, int d, int p, int H, int tid,
                                           float4 (&x)[AT_NQ]) {
    const int b = p / H, h = p - b * H;
    const float* xb = base + static_cast<long>(b) * rows * ld + h * d;
    const bool vec = ((ld | d) & 3) == 0 && (reinterpret_cast<uintptr_t>(xb) & 15) == 0;
#pragma unroll
    for (int u = 0; u < AT_NQ; u++) {
        const int i = u * AT_THREADS + tid, row = i >> 4, c = (i & 15) * 4;
        x[u] = row < rows ? load_row4(xb + static_cast<long>(row) * ld, c, d, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
__device__ __forceinline__ void at_load_v(const AtArgs& A, int p, int quarter, int grp, int lane, float4 (&xv)[4]) {
    const int b = p / A.H, h = p - b * A.H;
    const float* vb = A.v + static_cast<long>(b) * A.S * A.ldv + h * A.dv;
    const bool vv = ((A.ldv | A.dv) & 3) == 0 && (reinterpret_cast<uintptr_t>(vb) & 15) == 0;
    const int vj = quarter * 32 + lane, vd0 = grp * 16;
#pragma unroll
    for (int u = 0; u < 4; u++)
        xv[u] = vj < A.S ? load_row4(vb + static_cast<long>(vj) * A.ldv, vd0 + 4 * u, A.dv, vv) : make_float4(0.f, 0.f, 0.f, 0.f);
}

__global__ void __launch_bounds__(AT_THREADS, 1) k_attention_tc(const AtArgs A, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    AtCtl* ctl = reinterpret_cast<AtCtl*>(smem + AT_QK_BYTES + AT_V_BYTES);
    uint8_t* qk = smem;                   // Q hi t0,t1 | Q lo t0,t1 | K hi t0,t1 | K lo t0,t1; then P hi t0..3 | P lo t0..3
    uint8_t* vt = smem + AT_QK_BYTES;     // V^T hi t0..3 | V^T lo t0..3
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, grp = warp >> 2;
    const int r = quarter * 32 + lane, key0 = grp * 32, vd0 = grp * 16;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;

    if (tid == 0) {
        kx::mbar_init(&ctl->bar, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
    }
    if (warp == 0) {
        kx::tmem_alloc(&ctl->tmem, AT_TMEM_COLS);
        kx::tmem_relinquish();
    }
    float4 xq[AT_NQ], xk[AT_NQ], xv[4];
    int p = blockIdx.x;
    if (p < A.pairs) {
        at_load_qk(A.q, A.ldq, A.Rq, A.dk, p, A.H, tid, xq);
        at_load_qk(A.k, A.ldk, A.S, A.dk, p, A.H, tid, xk);
        at_load_v(A, p, quarter, grp, lane, xv);
    }
    // the scores in base-2 units: exp(s - m) = 2^(s log2(e) - m log2(e)), one ex2.approx per score (~2 ulp)
    const float scale2 = A.scale * 1.4426950408889634f;
    // whole ctx rows by bulk copy: every row start 16-byte aligned and the row a multiple of 16 bytes
    const bool bulk_out = ((A.ldc | A.dv) & 3) == 0 && (reinterpret_cast<uintptr_t>(A.ctx) & 15) == 0;
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    const uint32_t base = kx::smem_u32(smem);
    int pending = -1;  // barrier phase a timed-out wait left behind

    for (; p < A.pairs; p += gridDim.x) {
        const int b = p / A.H, h = p - b * A.H;
        if (bulk_out && lane < 8) kx::bulk_wait_read();  // the previous pair's staged rows (in the V^T tiles) are read
        // 1. Q and K of this pair into the operand tiles (the previous pair's MMAs have completed)
#pragma unroll
        for (int u = 0; u < AT_NQ; u++) {
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

        // 2. S = Q . K^T; meanwhile V^T, then the next pair's loads
        if (tid == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(AT_MAX, AT_MAX);
            const int nks = (A.dk + 7) / 8;
            for (int ks = 0; ks < nks; ks++) {
                const uint32_t o = (ks >> 2) * AT_TILE + (ks & 3) * 32;
                const uint32_t ah = base + o, al = base + 2 * AT_TILE + o, bh = base + 4 * AT_TILE + o, bl = base + 6 * AT_TILE + o;
                kx::mma_tf32(tmem + AT_S, kx::desc_sw128_kmajor(al), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
                kx::mma_tf32(tmem + AT_S, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bl), idesc, 1);
                kx::mma_tf32(tmem + AT_S, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bh), idesc, 1);
            }
            kx::mma_commit(&ctl->bar);
        }
        __syncwarp();
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
        const int pn = p + static_cast<int>(gridDim.x);  // the next pair: Q now, K after the softmax's max, V later
        if (pn < A.pairs) at_load_qk(A.q, A.ldq, A.Rq, A.dk, pn, A.H, tid, xq);
        // the warps read TMEM with warp-collective loads: agree on the outcome first
        if (!__syncthreads_and(kx::mbar_wait(&ctl->bar, 0, &ctl->abort, status))) {
            pending = 0;
            break;
        }
        kx::tc_fence_after();

        // 3. softmax: row r, keys key0 .. key0 + 31
        float e[32];
        {
            uint32_t sv[32];
            kx::tmem_ld32(tmem + lanes + AT_S + key0, sv);
            kx::tmem_ld_wait();
            float m = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int key = key0 + j;
                const float t = __fmul_rn(__uint_as_float(sv[j]), scale2);
                e[j] = (key >= A.S || (A.causal && key > r)) ? -INFINITY : t;
                m = fmaxf(m, e[j]);
            }
            ctl->red[grp][r] = m;
        }
        if (pn < A.pairs) at_load_qk(A.k, A.ldk, A.S, A.dk, pn, A.H, tid, xk);
        kx::named_bar(1 + quarter, 128);  // the four warps of this lane quarter (the rows they share)
        {
            const float m = fmaxf(fmaxf(ctl->red[0][r], ctl->red[1][r]), fmaxf(ctl->red[2][r], ctl->red[3][r]));
#pragma unroll
            for (int j = 0; j < 32; j++) e[j] = kx::ex2_approx(__fsub_rn(e[j], m));
        }
        kx::named_bar(1 + quarter, 128);  // every partial max has been read before the partial sums overwrite them
        {
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) part = __fadd_rn(part, e[j]);
            ctl->red[grp][r] = part;
        }
        kx::named_bar(1 + quarter, 128);
        {
            const float sum = __fadd_rn(__fadd_rn(__fadd_rn(ctl->red[0][r], ctl->red[1][r]), ctl->red[2][r]), ctl->red[3][r]);
            const float inv = __fdiv_rn(1.0f, sum);
            // P tile grp (keys 32 grp ..) over the Q / K tiles (every MMA that read them has completed); keys past S
            // have e = 0
            uint8_t* ph = qk + grp * AT_TILE;
            uint8_t* pl = qk + (4 + grp) * AT_TILE;
#pragma unroll
            for (int j4 = 0; j4 < 8; j4++) {
                const float4 pv = make_float4(__fmul_rn(e[4 * j4], inv), __fmul_rn(e[4 * j4 + 1], inv),
                                              __fmul_rn(e[4 * j4 + 2], inv), __fmul_rn(e[4 * j4 + 3], inv));
                float4 hv, lv;
                split4(pv, hv, lv);
                *reinterpret_cast<float4*>(ph + swz(r, j4)) = hv;
                *reinterpret_cast<float4*>(pl + swz(r, j4)) = lv;
            }
        }
        kx::fence_proxy_async_smem();
        kx::tc_fence_before();
        __syncthreads();
        kx::tc_fence_after();

        // 4. ctx = P . V (N = 64 head-dim columns, K = keys)
        if (tid == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(AT_MAX, AT_DMAX);
            const int nks = (A.S + 7) / 8;
            for (int ks = 0; ks < nks; ks++) {
                const uint32_t o = (ks >> 2) * AT_TILE + (ks & 3) * 32, ov = (ks >> 2) * AT_VTILE + (ks & 3) * 32;
                const uint32_t ah = base + o, al = base + 4 * AT_TILE + o;
                const uint32_t bh = base + AT_QK_BYTES + ov, bl = base + AT_QK_BYTES + 4 * AT_VTILE + ov;
                kx::mma_tf32(tmem + AT_O, kx::desc_sw128_kmajor(al), kx::desc_sw128_kmajor(bh), idesc, ks != 0);
                kx::mma_tf32(tmem + AT_O, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bl), idesc, 1);
                kx::mma_tf32(tmem + AT_O, kx::desc_sw128_kmajor(ah), kx::desc_sw128_kmajor(bh), idesc, 1);
            }
            kx::mma_commit(&ctl->bar);
        }
        __syncwarp();
        if (pn < A.pairs) at_load_v(A, pn, quarter, grp, lane, xv);
        if (!__syncthreads_and(kx::mbar_wait(&ctl->bar, 1, &ctl->abort, status))) {
            pending = 1;
            break;
        }
        kx::tc_fence_after();

        // 5. ctx rows 32 quarter .. +31, head-dim columns 16 grp .. 16 grp + 15: staged in the V^T tiles (free once
        // P . V has completed), then written by bulk copies of whole rows that run while the next pair starts; plain
        // stores where the rows are not 16-byte aligned
        {
            uint32_t ov[16];
            kx::tmem_ld16(tmem + lanes + AT_O + vd0, ov);
            kx::tmem_ld_wait();
            if (bulk_out) {
                if (vd0 < A.dv) {
                    float4* srow = reinterpret_cast<float4*>(vt + r * AT_CROW + vd0 * 4);
#pragma unroll
                    for (int j4 = 0; j4 < 4; j4++)
                        srow[j4] = make_float4(__uint_as_float(ov[4 * j4]), __uint_as_float(ov[4 * j4 + 1]),
                                               __uint_as_float(ov[4 * j4 + 2]), __uint_as_float(ov[4 * j4 + 3]));
                }
                kx::fence_proxy_async_smem();
                kx::named_bar(1 + quarter, 128);  // the quarter's 32 rows are staged
                if (lane < 8) {  // warp (quarter, grp) copies rows 32 quarter + 8 grp .. + 7
                    const int rr = quarter * 32 + grp * 8 + lane;
                    if (rr < A.Rq) {
                        kx::bulk_store(A.ctx + (static_cast<long>(b) * A.Rq + rr) * A.ldc + h * A.dv, vt + rr * AT_CROW,
                                       static_cast<uint32_t>(A.dv) * 4);
                        kx::bulk_commit();
                    }
                }
            } else if (r < A.Rq && vd0 < A.dv) {
                float* dst = A.ctx + (static_cast<long>(b) * A.Rq + r) * A.ldc + h * A.dv + vd0;
                const int nv = A.dv - vd0;
                if (nv >= 16 && ((A.ldc | A.dv) & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                    for (int j4 = 0; j4 < 4; j4++)
                        reinterpret_cast<float4*>(dst)[j4] = make_float4(__uint_as_float(ov[4 * j4]), __uint_as_float(ov[4 * j4 + 1]),
                                                                         __uint_as_float(ov[4 * j4 + 2]), __uint_as_float(ov[4 * j4 + 3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < nv) dst[j] = __uint_as_float(ov[j]);
                }
            }
        }
        kx::tc_fence_before();
        __syncthreads();  // every warp has read this pair's ctx before the next pair's MMAs write TMEM
        kx::tc_fence_after();
    }
    if (bulk_out && lane < 8) kx::bulk_wait_all();  // the last pair's rows are written before the CTA ends
    if (pending >= 0) {
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
    if (Rq > AT_MAX || S > AT_MAX || dk > AT_DMAX || dv > AT_DMAX) return 1;
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
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    const long pairs = static_cast<long>(B) * H;
    if (pairs <= 0) return 0;
    if (pairs > INT32_MAX) return 1;
    const AtArgs A{q, k, v, ctx, ldq, ldk, ldv, ldc, Rq, S, H, dk, dv, causal, static_cast<int>(pairs), scale};
    const int grid = pairs < sms ? static_cast<int>(pairs) : sms;  // persistent: one CTA per SM walks the pairs
    k_attention_tc<<<grid, AT_THREADS, AT_SMEM, st>>>(A, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
