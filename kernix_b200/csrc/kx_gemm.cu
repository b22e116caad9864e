// KERNIX-B200 dense GEMMs on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
//  * kx_gemm_i8   : int8 x int8 -> int32 (kind::i8) with the dequant / bias / activation epilogue of the
//                   reference's kernix_qmatmul (include/kernix_model.h:143-177) and the LINEAR step's
//                   activation (:1854-1856). Operands: A = per-row quantised activations [M][lda] int8,
//                   B = weights [N][ldb] int8 (K-major, transposed from the file's in x out q at load).
//  * kx_gemm_f32  : fp32 GEMM in 3xTF32 split precision with fused bias + activation, replacing
//                   kernix_dense -> kernix_matmul_ep_into (include/kernix_model.h:544-550,
//                   include/kernix.h:955-976, src/kernix_metal.m:161-265). A is read from global memory by
//                   converter warps that split every value into a tf32 "hi" part (rounded to 10 mantissa
//                   bits) and the exact remainder "lo", written into swizzled shared memory; B arrives
//                   pre-split (hi/lo planes, [N][ldb] K-major) by TMA. Each K step issues
//                   hi*hi + hi*lo + lo*hi into one fp32 TMEM accumulator.
//
// CTA layout (one 128 x BN output tile per CTA):
//   warp 0      TMA producer (elected lane)
//   warp 1      TMEM allocator + MMA issuer (elected lane)
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31), then
//               dequant/bias/act and global stores
//   warps 6-13  (3xTF32 only) A converters
// Shared memory holds STAGES operand stages in the canonical K-major 128-byte-swizzle layout; full/empty
// mbarriers form the ring. Every wait is bounded (kx_sm100.cuh); a timeout sets the status word, the CTA
// drains its in-flight copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <climits>
#include <mutex>

#include "kx_act.cuh"
#include "kx_kernels.h"
#include "kx_pdl.cuh"
#include "kx_sm100.cuh"

namespace {

constexpr int BM = 128;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// bounded wait that ignores the abort flag: used to drain work already issued before leaving the CTA
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = kx::globaltimer();
    while (!kx::mbar_try_wait(bar, parity)) {
        if (kx::globaltimer() - t0 > KX_WAIT_NS) return;
        __nanosleep(128);
    }
}

// Epilogue activation: the configurations' activations (none, ReLU, GELU) are compiled into the kernel; the
// other thirteen go through one out-of-line call, which keeps the unrolled epilogue small enough for the
// instruction cache.
constexpr int ACT_GENERIC = 99;
__device__ __noinline__ float act_outline(int act, float v, float alpha) { return kx::act_apply(act, v, alpha); }
template <int ACTC>
__device__ __forceinline__ float epi_act(float v, int act, float alpha) {
    if constexpr (ACTC == ACT_GENERIC) return act_outline(act, v, alpha);
    else return kx::act_apply(ACTC, v, alpha);
}
// the epilogue activation on two values (packed f32x2 arithmetic for GELU; per component otherwise)
template <int ACTC>
__device__ __forceinline__ float2 epi_act2(float2 v, int act, float alpha) {
    if constexpr (ACTC == 1) return kx::gelu_as2(v);
    else return make_float2(epi_act<ACTC>(v.x, act, alpha), epi_act<ACTC>(v.y, act, alpha));
}
inline int act_class(int act) { return act == -1 || act == 0 || act == 1 ? act : ACT_GENERIC; }

struct SmemCtl {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t accf;
    uint32_t tmem;
    int abort;
};

// ------------------------------------------------------------------------------------------ int8
// Persistent kernel: each CTA walks output tiles t = blockIdx.x, +gridDim.x, ... (M-tile fastest so the CTAs
// running at once share B tiles in L2). TMEM holds two 128 x BN int32 accumulators; the MMA warp fills one
// while the 16 epilogue warps drain the other, so the epilogue of tile i overlaps the mainloop of tile i+1.
// Epilogue (4 warps per TMEM lane quarter, each owning a quarter of the tile's columns -- four warps per
// scheduler hide the latency of the activation math): thread-per-row tcgen05.ld of 16 columns (the next
// chunk's load is in flight while this one is processed) -> 64-byte-row swizzled per-warp staging tile -> each
// lane then owns 4 columns of 4 rows, applies ((float)acc*sx)*scale + bias and the activation, and the warp
// writes eight full 64-byte row segments per store instruction.
template <int BN, int STAGES>
struct I8Cfg {
    static constexpr int BK = 128;  // bytes of K per stage (one 128-byte swizzle row)
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int EPI_COLS = BN / 4;                     // columns of the tile per epilogue warp
    static constexpr int STAGE_EPI = EPI_WARPS * 32 * 16 * 4;  // per-warp 32 x 16 x 4-byte staging tiles
    static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + STAGE_EPI + 1024 + static_cast<int>(sizeof(SmemCtl));
    static constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator
};

struct TileMap {  // tile t -> (m-tile, n-tile): M-tile fastest, or N-tile fastest (row blocks in order) if n_fast
    int m_tiles, n_tiles;
    bool n_fast;
    __device__ __forceinline__ void at(int t, int& mt, int& nt) const {
        if (n_fast) {
            mt = t / n_tiles;
            nt = t - mt * n_tiles;
        } else {
            nt = t / m_tiles;
            mt = t - nt * m_tiles;
        }
    }
};

// Per-warp dequantisation factors of one tile, loaded one tile ahead so that their global-load latency hides
// behind the wait for the accumulator: sx of the thread's four rows (r0 + 16h + 8e + lane/4 -> sx[2h + e]) and,
// spread over the warp (two columns per lane), scale and bias of the warp's 64 columns starting at col0.
struct EpiPre {
    float sx[4];
    float2 sc, bi;
};
__device__ __forceinline__ void epi_prefetch(EpiPre& p, int r0, int col0, int lane, int M, int N, const float* __restrict__ sx,
                                             const float* __restrict__ scale, const float* __restrict__ bias) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int gr = r0 + 16 * (i >> 1) + 8 * (i & 1) + (lane >> 2);
        p.sx[i] = gr < M ? __ldg(sx + gr) : 0.0f;
    }
    const int c = col0 + 2 * lane;
    p.sc.x = c < N ? __ldg(scale + c) : 0.0f;
    p.sc.y = c + 1 < N ? __ldg(scale + c + 1) : 0.0f;
    p.bi.x = bias && c < N ? __ldg(bias + c) : 0.0f;
    p.bi.y = bias && c + 1 < N ? __ldg(bias + c + 1) : 0.0f;
}

// Raw int32 sums of one 16x256b.x4 block (rows ra and ra + 8, columns gc0 + 8k, +1): the accumulator test path.
__device__ __forceinline__ void epi_block_acc(const uint32_t (&r)[16], int ra, int gc0, int32_t* __restrict__ acc_out, int ldy,
                                              int M, int N) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int gc = gc0 + 8 * k;
        if (gc >= N) continue;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int gr = ra + 8 * e;
            if (gr >= M) continue;
            int32_t* dst = acc_out + static_cast<size_t>(gr) * ldy + gc;
            dst[0] = static_cast<int32_t>(r[4 * k + 2 * e]);
            if (gc + 1 < N) dst[1] = static_cast<int32_t>(r[4 * k + 2 * e + 1]);
        }
    }
}

// Dequantise and activate one 16x256b.x4 block: o[2k + e] = the thread's two values in row ra + 8e at columns
// gc0 + 8k, +1. ((float)acc * sx) * scale + bias keeps the reference's IEEE step order: the two products are packed
// (mul.rn.f32x2) and the add is scalar, so no product is contracted into an fma with the add. All 16 values are
// dequantised, then all activated, before anything is stored, so the eight independent chains interleave.
// cf[4k] = (scale, scale, bias, bias) of the thread's two columns in block k.
template <int ACTC>
__device__ __forceinline__ void epi_math(const uint32_t (&r)[16], float sxa, float sxb, const float4* __restrict__ cf,
                                         float2 (&o)[8], int act, float alpha) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float4 f = cf[4 * k];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float2 a = make_float2(static_cast<float>(static_cast<int32_t>(r[4 * k + 2 * e])),
                                         static_cast<float>(static_cast<int32_t>(r[4 * k + 2 * e + 1])));
            const float2 p = kx::mul2(kx::mul2(a, kx::f2(e ? sxb : sxa)), make_float2(f.x, f.y));
            o[2 * k + e] = make_float2(__fadd_rn(p.x, f.z), __fadd_rn(p.y, f.w));
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) o[i] = epi_act2<ACTC>(o[i], act, alpha);
}

// store a block's values: rows ra (o[2k]) and ra + 8 (o[2k + 1]), columns gc0 + 8k, +1
__device__ __forceinline__ void epi_store_full(const float2 (&o)[8], float* __restrict__ rowa, float* __restrict__ rowb) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        *reinterpret_cast<float2*>(rowa + 8 * k) = o[2 * k];
        *reinterpret_cast<float2*>(rowb + 8 * k) = o[2 * k + 1];
    }
}
__device__ __forceinline__ void epi_store_checked(const float2 (&o)[8], float* __restrict__ y, int ra, int gc0, int ldy, int M,
                                                  int N, bool vec) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int gc = gc0 + 8 * k;
        if (gc >= N) continue;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int gr = ra + 8 * e;
            if (gr >= M) continue;
            float* dst = y + static_cast<size_t>(gr) * ldy + gc;
            const float2 v = o[2 * k + e];
            if (vec && gc + 1 < N) {
                *reinterpret_cast<float2*>(dst) = v;
            } else {
                dst[0] = v.x;
                if (gc + 1 < N) dst[1] = v.y;
            }
        }
    }
}

// Epilogue of one 128 x BN accumulator tile for one warp: its 32 TMEM lanes (tile rows r0 .. r0+31, TMEM address
// tbase = lane quarter base) and columns [c_lo, c_lo + BN/4) of the tile, whose first global column is n0.
// tcgen05.ld 16x256b: four consecutive threads hold 8 consecutive columns of one row, so every store writes
// whole 32-byte sectors straight from registers (no shared-memory transpose); the loads are double-buffered so
// each block's load is in flight while the previous block is processed. The warp's column factors sit in
// its shared-memory slot (written from the prefetched registers) as (scale, scale, bias, bias) per column pair
// and are read as broadcasts. Tiles entirely inside the output store without bounds checks. ACC_ONLY writes the
// raw int32 sums.
template <int BN, bool ACC_ONLY, int ACTC>
__device__ __forceinline__ void epi_tile_i8(uint32_t tbase, int r0, int n0, int c_lo, float* slot, int lane, const EpiPre& f,
                                            float* __restrict__ y, int32_t* __restrict__ acc_out, int ldy, int M, int N,
                                            int act, float alpha) {
    constexpr int EPI_COLS = BN / 4;  // 64 or 32 columns: 2 or 1 column halves of 32
    constexpr int NB = 2 * (EPI_COLS / 32);  // 16x256b.x4 blocks per warp: (row half, column half)
    float4* cf = reinterpret_cast<float4*>(slot);
    if (!ACC_ONLY) {
        __syncwarp();
        cf[lane] = make_float4(f.sc.x, f.sc.y, f.bi.x, f.bi.y);  // columns c_lo + 2 lane, +1
        __syncwarp();
    }
    const int t4 = lane & 3, row = lane >> 2;
    const bool vec = (ldy & 1) == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0;
    const bool full = vec && r0 + 32 <= M && n0 + c_lo + EPI_COLS <= N;
    uint32_t ra[16], rb[16];
    // block i: row half h = i % 2, column half cc = i / 2
    auto taddr = [&](int i) { return tbase + (static_cast<uint32_t>(16 * (i & 1)) << 16) + c_lo + 32 * (i >> 1); };
    auto run = [&](const uint32_t (&r)[16], int i) {
        const int h = i & 1, cc = i >> 1;
        const int gr = r0 + 16 * h + row, gc = n0 + c_lo + 32 * cc + 2 * t4;
        if (ACC_ONLY) {
            epi_block_acc(r, gr, gc, acc_out, ldy, M, N);
        } else {
            float2 o[8];
            epi_math<ACTC>(r, f.sx[2 * h], f.sx[2 * h + 1], cf + 16 * cc + t4, o, act, alpha);
            if (full) {
                float* rowa = y + static_cast<size_t>(gr) * ldy + gc;
                epi_store_full(o, rowa, rowa + 8 * static_cast<size_t>(ldy));
            } else {
                epi_store_checked(o, y, gr, gc, ldy, M, N, vec);
            }
        }
    };
    kx::tmem_ld16x256b_x4(taddr(0), ra);
    kx::tmem_ld16_wait(ra);
    kx::tmem_ld16x256b_x4(taddr(1), rb);
    run(ra, 0);
    kx::tmem_ld16_wait(rb);
    if (NB > 2) kx::tmem_ld16x256b_x4(taddr(2), ra);
    run(rb, 1);
    if (NB > 2) {
        kx::tmem_ld16_wait(ra);
        kx::tmem_ld16x256b_x4(taddr(3), rb);
        run(ra, 2);
        kx::tmem_ld16_wait(rb);
        run(rb, 3);
    }
}

// ------------------------------------------------------------------ int8 with a quantised output (QOUT)
// The output of a hidden int8 layer is read only by the next int8 layer, and only quantised: row by row as
// q = clamp(rint(y * (1 / sx)), +-127) with sx = max|y| / 127 over the whole row (kernix_qmatmul :110-142, the
// next step's quantisation). A QOUT launch of the CTA-pair kernel writes q and sx instead of y, so there is no fp32
// intermediate and no separate quantiser pass. Tiles are walked row-block-major, so the CTA tiles of one 128-row
// group run at the same time on different clusters. Per CTA tile, once its accumulator is complete:
//   pass 1: dequantise and activate exactly as the fp32 epilogue, write the fp32 values back over the accumulator
//           in TMEM, and publish each row's max|y| (atomicMax on the IEEE bits of |y|, so NaN wins, as the
//           quantiser's max) into rowmax; after a barrier of the CTA's 16 epilogue warps one thread counts the tile
//           in the row group's counter;
//   wait:   until every N-tile of the row group has been counted (bounded; a timeout sets the status word);
//   pass 2: read the values back (one thread per row), scale by 1 / sx in the quantiser's IEEE steps, round to
//           nearest even with the 1.5 * 2^23 addition (exact for |v| < 2^22; here |v| <= 127.0001), clamp, and store
//           32 bytes of a row per 16-byte pair of stores; rows whose max is inf or NaN get sx = NaN and q = 0, as
//           the quantiser gives them.
// The same values, the same max and the same IEEE steps as the quantiser kernel on the fp32 output: q and sx are
// bit for bit what kx_quant_rows would produce from y. The grid is a whole number of row groups' worth of clusters,
// so a round of the round-robin walk covers whole row groups and a tile's wait is only for the tiles of the same
// round (no deadlock either way: a tile's wait depends only on pass 1 of the tiles of its row group, which sit at
// the same or the next round, and pass 1 of a round needs only the accumulator buffer freed two rounds earlier).
struct QOut {
    int8_t* q;         // M x ldq, the next layer's A operand; columns N .. ldq-1 are written as 0
    float* sx;         // M row scales
    uint32_t* rowmax;  // M, zero at launch
    uint32_t* cnt;     // ceil(M / 128), zero at launch
    uint32_t* zero;    // words this launch clears after its dependency wait (the next QOUT launch's rowmax and cnt)
    int ldq, zero_words;
};

// pass 1 of one warp's part of a CTA tile (32 rows x 64 columns): rows r0 + 16h + lane/4 + 8e -> mx[2h + e]
template <int ACTC>
__device__ __forceinline__ void q_pass1(uint32_t tbase, int c_lo, const float4* __restrict__ cf, int lane, const EpiPre& f,
                                        int act, float alpha, uint32_t (&mx)[4]) {
    const int t4 = lane & 3;
    uint32_t ra[16], rb[16];
    auto taddr = [&](int i) { return tbase + (static_cast<uint32_t>(16 * (i & 1)) << 16) + c_lo + 32 * (i >> 1); };
    auto run = [&](uint32_t (&r)[16], int i) {
        const int h = i & 1, cc = i >> 1;
        float2 o[8];
        epi_math<ACTC>(r, f.sx[2 * h], f.sx[2 * h + 1], cf + 16 * cc + t4, o, act, alpha);
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                mx[2 * h + e] = kx::absmax_nan(kx::absmax_nan(mx[2 * h + e], o[2 * k + e].x), o[2 * k + e].y);
                r[4 * k + 2 * e] = __float_as_uint(o[2 * k + e].x);
                r[4 * k + 2 * e + 1] = __float_as_uint(o[2 * k + e].y);
            }
        kx::tmem_st16x256b_x4(taddr(i), r);
    };
    kx::tmem_ld16x256b_x4(taddr(0), ra);
    kx::tmem_ld16_wait(ra);
    kx::tmem_ld16x256b_x4(taddr(1), rb);
    run(ra, 0);
    kx::tmem_ld16_wait(rb);
    kx::tmem_ld16x256b_x4(taddr(2), ra);
    run(rb, 1);
    kx::tmem_ld16_wait(ra);
    kx::tmem_ld16x256b_x4(taddr(3), rb);
    run(ra, 2);
    kx::tmem_ld16_wait(rb);
    run(rb, 3);
    kx::tmem_st_wait();
}

// four quantised bytes of v[0..3] (the quantiser's steps: rint(v * inv), clamped to +-127), inv finite. t = v inv
// rounded, plus 1.5 2^23, is the integer q = rint(v inv) in the last bits of 0x4B400000 + q, so q's byte is t's low
// byte; |v inv| <= 127 (1 + 2^-22) since |v| <= the row's maximum, so the clamp never acts and is not applied
__device__ __forceinline__ uint32_t q_word(const uint32_t* v, float inv) {
    uint32_t t[4];
#pragma unroll
    for (int e = 0; e < 4; e++) t[e] = __float_as_uint(__fadd_rn(__fmul_rn(__uint_as_float(v[e]), inv), 12582912.0f));
    return __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
}

// pass 2 of one warp: thread = row r0 + lane (TMEM lane quarter), columns c_lo .. c_lo + 63 of the tile; both
// 32-column loads are in flight before the first is used
__device__ __forceinline__ void q_pass2(uint32_t tbase, int c_lo, int lane, float inv, bool nan_row, int gr, int gc0,
                                        const QOut& qo, int M, int N) {
    uint32_t v[2][32];
    kx::tmem_ld32(tbase + c_lo, v[0]);
    kx::tmem_ld32(tbase + c_lo + 32, v[1]);
    kx::tmem_ld_wait();
    if (gr >= M) return;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = nan_row ? 0u : q_word(&v[half][4 * j], inv);
        const int gc = gc0 + 32 * half;
        if (gc >= qo.ldq) continue;
        if (gc + 32 > N) {  // the last columns: bytes at N and beyond are the zero padding up to ldq
#pragma unroll
            for (int j = 0; j < 8; j++)
#pragma unroll
                for (int b = 0; b < 4; b++)
                    if (gc + 4 * j + b >= N) w[j] &= ~(0xFFu << (8 * b));
        }
        uint4* dst = reinterpret_cast<uint4*>(qo.q + static_cast<size_t>(gr) * qo.ldq + gc);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        if (gc + 16 < qo.ldq) dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// wait (bounded) until the counter reaches target; false on a timeout (status set, abort raised) or abort
__device__ __forceinline__ bool q_wait_count(const uint32_t* cnt, uint32_t target, volatile int* abort, int* status) {
    const uint64_t t0 = kx::globaltimer();
    for (uint32_t spin = 0;; spin++) {  // polled without sleeping: the other tiles of a row group finish together
        if (kx::ld_acquire_gpu(cnt) >= target) return true;
        if (*abort) return false;
        if ((spin & 63) == 63 && kx::globaltimer() - t0 > KX_WAIT_NS) {
            *abort = 1;
            if (status) atomicExch(status, KX_STATUS_TIMEOUT);
            return false;
        }
    }
}

template <int BN, int STAGES, bool ACC_ONLY, int ACTC>
__global__ void __launch_bounds__(I8Cfg<BN, STAGES>::THREADS, 1)
k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
          const float* __restrict__ sx, const float* __restrict__ scale, const float* __restrict__ bias,
          float* __restrict__ y, int32_t* __restrict__ acc_out, int ldy, int M, int N, int K, int act, float alpha,
          int* status, int kbs) {
    using C = I8Cfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sE = sB + STAGES * C::B_BYTES;
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(sE + C::STAGE_EPI);
    volatile int* abort_flag = &ctl->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // split-K (ACC_ONLY, kbs > 0): the reduction is cut into ranges of kbs K blocks; tile t covers output tile
    // t % (m_tiles n_tiles) over range t / (m_tiles n_tiles) and writes its int32 sums into plane z of acc_out (M x
    // ldy each). kbs <= 0: one range.
    const int nk_all = (K + C::BK - 1) / C::BK;
    const int kpr = kbs > 0 ? kbs : nk_all;
    const TileMap tm{(M + BM - 1) / BM, (N + BN - 1) / BN, false};
    const int mn_tiles = tm.m_tiles * tm.n_tiles;
    const int n_tiles = mn_tiles * ((nk_all + kpr - 1) / kpr);
    auto at = [&](int t, int& mt, int& nt, int& kb0, int& nk) {  // tile t: output tile and its K blocks
        const int z = t / mn_tiles;
        tm.at(t - z * mn_tiles, mt, nt);
        kb0 = z * kpr;
        nk = min(nk_all - kb0, kpr);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1);
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], C::EPI_WARPS);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {
        kx::tmem_alloc(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish();
    }
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    kx::griddep_wait();  // a programmatic dependent (the split-K form) reads the kernel before's rows after this
    kx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmA);
            kx::tma_prefetch_desc(&tmB);
            int it = 0;
            for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
                int mt, nt, kb0, nk;
                at(t, mt, nt, kb0, nk);
                for (int kb = kb0; kb < kb0 + nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) break;
                    kx::mbar_arrive_expect_tx(&ctl->full[s], C::A_BYTES + C::B_BYTES);
                    kx::tma_load_2d(sA + s * C::A_BYTES, &tmA, kb * C::BK, mt * BM, &ctl->full[s]);
                    kx::tma_load_2d(sB + s * C::B_BYTES, &tmB, kb * C::BK, nt * BN, &ctl->full[s]);
                }
            }
            if (*abort_flag)  // let copies already in flight land before the CTA's shared memory goes away
                for (int i = it > STAGES ? it - STAGES : 0; i < it; i++) drain_wait(&ctl->full[i % STAGES], (i / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = kx::idesc_i8(BM, BN);
            int it = 0, j = 0;
            for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x, j++) {
                const int b = j & 1;
                int mt, nt, kb0, nk;
                at(t, mt, nt, kb0, nk);
                (void)mt;
                (void)nt;
                if (!kx::mbar_wait(&ctl->acc_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->full[s], (it / STAGES) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    kx::tc_fence_after();
                    const uint32_t a0 = kx::smem_u32(sA + s * C::A_BYTES), b0 = kx::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < C::BK / 32; kk++)
                        kx::mma_i8(d, kx::desc_sw128_kmajor(a0 + kk * 32), kx::desc_sw128_kmajor(b0 + kk * 32), idesc,
                                   (kb | kk) != 0);
                    kx::mma_commit(&ctl->empty[s]);
                }
                if (!ok) break;
                kx::mma_commit(&ctl->acc_full[b]);
            }
            kx::mma_commit(&ctl->accf);  // completes once every MMA issued above has finished
            drain_wait(&ctl->accf, 0);
        }
        __syncwarp();
    } else {
        const int ew = warp - 2;                    // 0..15
        const int q = warp & 3;                     // TMEM lane quarter this warp may read
        const int c_lo = (ew >> 2) * C::EPI_COLS;   // this warp's quarter of the tile's columns
        float* stg = reinterpret_cast<float*>(sE + ew * 2048);
        EpiPre cur{}, nxt{};
        if (!ACC_ONLY && blockIdx.x < n_tiles) {
            int mt, nt, kb0, nk;
            at(blockIdx.x, mt, nt, kb0, nk);
            epi_prefetch(cur, mt * BM + q * 32, nt * BN + c_lo, lane, M, N, sx, scale, bias);
        }
        int j = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, j++) {
            int mt, nt, kb0, nk;
            at(t, mt, nt, kb0, nk);
            const int b = j & 1;
            if (!ACC_ONLY && t + static_cast<int>(gridDim.x) < n_tiles) {
                int mt2, nt2, kb2, nk2;
                at(t + gridDim.x, mt2, nt2, kb2, nk2);
                epi_prefetch(nxt, mt2 * BM + q * 32, nt2 * BN + c_lo, lane, M, N, sx, scale, bias);
            }
            if (!kx::mbar_wait(&ctl->acc_full[b], (j >> 1) & 1, abort_flag, status)) break;
            kx::tc_fence_after();
            int32_t* plane = ACC_ONLY ? acc_out + static_cast<size_t>(kb0 / kpr) * M * ldy : acc_out;
            epi_tile_i8<BN, ACC_ONLY, ACTC>(tmem + b * BN + (static_cast<uint32_t>(q * 32) << 16), mt * BM + q * 32, nt * BN,
                                            c_lo, stg, lane, cur, y, plane, ldy, M, N, act, alpha);
            cur = nxt;
            kx::tc_fence_before();
            __syncwarp();
            if (lane == 0) kx::mbar_arrive(&ctl->acc_empty[b]);
        }
    }
    kx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------ int8, CTA pairs
// The same persistent GEMM on 256 x 256 output tiles computed by a cluster of two CTAs with one M = 256
// tcgen05.mma (cta_group::2). CTA rank r of the pair stages A rows [m0 + 128 r, +128) and B rows
// [n0 + 128 r, +128) of each K block in its own shared memory; the MMA, issued by rank 0, reads both CTAs'
// halves and leaves rows [m0 + 128 r, +128) x 256 columns in rank r's TMEM, which rank r's 16 epilogue warps
// drain exactly as in the one-CTA kernel. Per SM a K block moves 32 KB of operands for 128 x 256 x 128 MACs
// (the one-CTA 128 x 256 tile moves 48 KB), so six stages fit where the one-CTA kernel holds four.
// Synchronisation: both CTAs' TMA loads complete on rank 0's full[s] (rank 0 alone arms it with the bytes of
// both); rank 0's MMA thread commits every stage to empty[s] and every tile to acc_full[b] of BOTH CTAs (one
// commit per CTA, no multicast); each epilogue warp of either CTA arrives on rank 0's acc_empty[b] (32 arrivals).
// Every wait is bounded. On a timeout rank 0 waits (bounded) for the stages it armed, which cover the peer's
// copies of the same stages; the peer's producer can run at most STAGES K blocks ahead of rank 0's MMA, and
// those copies land within microseconds, long before any timeout expires.
template <int STAGES>
struct I8PairCfg {
    static constexpr int BN = 256;                 // columns per tile (the MMA's N)
    static constexpr int BK = 128;                 // bytes of K per stage
    static constexpr int A_BYTES = BM * BK;        // this CTA's 128 rows of A
    static constexpr int B_BYTES = (BN / 2) * BK;  // this CTA's 128 rows of B
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int STAGE_EPI = EPI_WARPS * 32 * 16 * 4;
    static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + STAGE_EPI + 1024 + static_cast<int>(sizeof(SmemCtl));
    static constexpr uint32_t TMEM_COLS = 2 * BN;
};

template <int STAGES, bool ACC_ONLY, int ACTC, bool QOUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(I8PairCfg<STAGES>::THREADS, 1)
k_gemm_i8_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const float* __restrict__ sx, const float* __restrict__ scale, const float* __restrict__ bias,
               float* __restrict__ y, int32_t* __restrict__ acc_out, int ldy, int M, int N, int K, int act, float alpha,
               int* status, const QOut qo) {
    using C = I8PairCfg<STAGES>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);  // the same offset in both CTAs (same kernel, same static layout)
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sE = sB + STAGES * C::B_BYTES;
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(sE + C::STAGE_EPI);
    volatile int* abort_flag = &ctl->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kx::cluster_ctarank();
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const int nk = (K + C::BK - 1) / C::BK;
    const TileMap tm{(M + 2 * BM - 1) / (2 * BM), (N + BN - 1) / BN, QOUT};  // pair tiles: 256 rows x 256 columns
    const int n_tiles = tm.m_tiles * tm.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1);
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], 2 * C::EPI_WARPS);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {  // warp 1 of both CTAs, same destination offset
        kx::tmem_alloc_pair(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish_pair();
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    kx::griddep_wait();  // launched as a dependent of the row quantiser: A and sx are its output
    kx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmA);
            kx::tma_prefetch_desc(&tmB);
            int it = 0;
            for (int t = cluster; t < n_tiles && !*abort_flag; t += n_clusters) {
                int mt, nt;
                tm.at(t, mt, nt);
                const int arow = mt * 2 * BM + static_cast<int>(rank) * BM, brow = nt * BN + static_cast<int>(rank) * (BN / 2);
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) break;
                    if (rank == 0) kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * (C::A_BYTES + C::B_BYTES));
                    const uint32_t full0 = kx::mapa(kx::smem_u32(&ctl->full[s]), 0);
                    kx::tma_load_2d_pair(sA + s * C::A_BYTES, &tmA, kb * C::BK, arow, full0);
                    kx::tma_load_2d_pair(sB + s * C::B_BYTES, &tmB, kb * C::BK, brow, full0);
                }
            }
            if (*abort_flag && rank == 0)  // the stages armed here also carry the peer's copies
                for (int i = it > STAGES ? it - STAGES : 0; i < it; i++) drain_wait(&ctl->full[i % STAGES], (i / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = kx::idesc_i8(2 * BM, BN);
            int it = 0, j = 0;
            for (int t = cluster; t < n_tiles && !*abort_flag; t += n_clusters, j++) {
                const int b = j & 1;
                if (!kx::mbar_wait(&ctl->acc_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->full[s], (it / STAGES) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    kx::tc_fence_after();
                    const uint32_t a0 = kx::smem_u32(sA + s * C::A_BYTES), b0 = kx::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < C::BK / 32; kk++)
                        kx::mma_i8_pair(d, kx::desc_sw128_kmajor(a0 + kk * 32), kx::desc_sw128_kmajor(b0 + kk * 32), idesc,
                                        (kb | kk) != 0);
                    const uint32_t e = kx::smem_u32(&ctl->empty[s]);
                    kx::mma_commit_pair(e);
                    kx::mma_commit_pair(kx::mapa(e, 1));
                }
                if (!ok) break;
                const uint32_t f = kx::smem_u32(&ctl->acc_full[b]);
                kx::mma_commit_pair(f);
                kx::mma_commit_pair(kx::mapa(f, 1));
            }
            kx::mma_commit_pair(kx::smem_u32(&ctl->accf));  // completes once every MMA issued above has finished
            drain_wait(&ctl->accf, 0);
        }
        __syncwarp();
    } else {
        const int ew = warp - 2;                 // 0..15
        const int q = warp & 3;                  // TMEM lane quarter this warp may read
        const int c_lo = (ew >> 2) * (BN / 4);   // this warp's quarter of the tile's columns
        float* stg = reinterpret_cast<float*>(sE + ew * 2048);
        const int row_off = static_cast<int>(rank) * BM + q * 32;  // this warp's rows within a pair tile
        EpiPre cur{}, nxt{};
        if (!ACC_ONLY && cluster < n_tiles) {
            int mt, nt;
            tm.at(cluster, mt, nt);
            epi_prefetch(cur, mt * 2 * BM + row_off, nt * BN + c_lo, lane, M, N, sx, scale, bias);
        }
        const uint32_t acc_empty0 = kx::mapa(kx::smem_u32(&ctl->acc_empty[0]), 0);
        if constexpr (QOUT) {  // clear the next QOUT launch's row maxima and counters (this launch's dependency is met)
            const int et = ew * 32 + lane, estride = static_cast<int>(gridDim.x) * C::EPI_WARPS * 32;
            for (int i = static_cast<int>(blockIdx.x) * C::EPI_WARPS * 32 + et; i < qo.zero_words; i += estride) qo.zero[i] = 0;
        }
        int j = 0;
        for (int t = cluster; t < n_tiles; t += n_clusters, j++) {
            int mt, nt;
            tm.at(t, mt, nt);
            const int b = j & 1;
            if (!ACC_ONLY && t + n_clusters < n_tiles) {
                int mt2, nt2;
                tm.at(t + n_clusters, mt2, nt2);
                epi_prefetch(nxt, mt2 * 2 * BM + row_off, nt2 * BN + c_lo, lane, M, N, sx, scale, bias);
            }
            const bool full_ok = __all_sync(0xffffffffu, kx::mbar_wait(&ctl->acc_full[b], (j >> 1) & 1, abort_flag, status));
            if constexpr (!QOUT) {
                if (!full_ok) break;
                kx::tc_fence_after();
                epi_tile_i8<BN, ACC_ONLY, ACTC>(tmem + b * BN + (static_cast<uint32_t>(q * 32) << 16), mt * 2 * BM + row_off,
                                                nt * BN, c_lo, stg, lane, cur, y, acc_out, ldy, M, N, act, alpha);
            } else {
                // every epilogue warp of the CTA passes the same two barriers per tile, whatever happens, and leaves
                // only on the OR of their abort states taken at the second one
                const uint32_t tb = tmem + b * BN + (static_cast<uint32_t>(q * 32) << 16);
                const int r0 = mt * 2 * BM + row_off;       // this warp's first row
                const int rg = mt * 2 + static_cast<int>(rank);  // this CTA's 128-row group
                const bool live = rg * BM < M;              // the CTA has rows in the output
                bool ok = full_ok;
                if (ok) {
                    kx::tc_fence_after();
                    float4* cf = reinterpret_cast<float4*>(stg);
                    __syncwarp();
                    cf[lane] = make_float4(cur.sc.x, cur.sc.y, cur.bi.x, cur.bi.y);
                    __syncwarp();
                    uint32_t mx[4] = {0u, 0u, 0u, 0u};
                    q_pass1<ACTC>(tb, c_lo, cf, lane, cur, act, alpha, mx);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
                        mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
                    }
                    if ((lane & 3) == 0)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int gr = r0 + 16 * (i >> 1) + (lane >> 2) + 8 * (i & 1);
                            if (gr < M) atomicMax(qo.rowmax + gr, mx[i]);
                        }
                    __threadfence();
                }
                kx::named_bar(1, C::EPI_WARPS * 32);  // every warp of this CTA tile has published its rows
                if (ok && live && ew == 0 && lane == 0) atomicAdd(qo.cnt + rg, 1u);
                if (ok && live) {
                    if (lane == 0) ok = q_wait_count(qo.cnt + rg, static_cast<uint32_t>(tm.n_tiles), abort_flag, status);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                }
                if (ok) {
                    const int gr = r0 + lane;
                    const uint32_t m = gr < M ? kx::ld_relaxed_gpu(qo.rowmax + gr) : 0u;
                    const bool nan_row = m >= 0x7F800000u;  // inf or NaN in the row: sx = NaN, q = 0
                    float sxv = 1.0f, inv = 1.0f;
                    if (nan_row) {
                        sxv = __uint_as_float(0x7FC00000u);
                    } else if (m != 0u) {
                        sxv = __fdiv_rn(__uint_as_float(m), 127.0f);
                        inv = __fdiv_rn(1.0f, sxv);
                    }
                    if (nt == 0 && c_lo == 0 && gr < M) qo.sx[gr] = sxv;
                    q_pass2(tb, c_lo, lane, inv, nan_row, gr, nt * BN + c_lo, qo, M, N);
                }
                if (kx::named_bar_or(1, C::EPI_WARPS * 32, !ok || *abort_flag)) break;
            }
            cur = nxt;
            kx::tc_fence_before();
            __syncwarp();
            if (lane == 0) kx::mbar_arrive_remote(acc_empty0 + b * static_cast<uint32_t>(sizeof(uint64_t)));
        }
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // no CTA leaves while its peer may still signal it or read its shared memory
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ int8 layer chains in one launch
// A chain of int8 LINEAR steps (kernix_qmatmul :99-182 and the activation :1854-1856 per step, each layer's output
// quantised as the next layer's input) as ONE persistent launch of the CTA-pair GEMM: the launch, set-up and pipeline
// fill are paid once, and a layer's first tiles start while the previous layer's last tiles finish. Tiles of every
// layer are walked in one round-robin order (layer by layer, row-block-major inside a layer). Hidden layers use the
// quantised-output epilogue (QOUT above); after a CTA tile's int8 rows are stored it counts the tile in its row
// group's `ready` word. The producer of a tile of layer l > 0 waits (bounded) until its CTA's 128-row group of layer
// l - 1 is complete -- every N-tile counted -- then issues its TMA loads of those rows. The last layer writes fp32.
// Waits only ever point to tiles earlier in the walk, whose progress needs nothing later: no deadlock (all clusters
// are resident; a wait that runs out sets the status word).
constexpr int KX_I8C_MAX = 4;
struct I8CLayer {
    const float* sx;     // row scales of the layer's int8 input (layer 0: the quantiser's; else the previous layer's)
    const float* scale;  // per-output-channel weight scales
    const float* bias;
    float* y;            // the last layer's fp32 output (n columns per row)
    QOut qo;             // hidden layers: the next layer's int8 rows and row scales
    uint32_t* ready;     // hidden layers: per 128-row group, CTA tiles whose int8 rows are stored
    int n, k, act, n_tiles_n, tile0;
    float alpha;
};
struct I8Chain {
    I8CLayer L[KX_I8C_MAX];
    int n_layers, total_tiles;
};

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// bounded wait until *w >= target (acquire), then order the async proxy (TMA) after it
__device__ __forceinline__ bool wait_ready(const uint32_t* w, uint32_t target, volatile int* abort, int* status) {
    if (!q_wait_count(w, target, abort, status)) return false;
    fence_proxy_async_global();
    return true;
}

template <int STAGES, int ACTH, int ACTL>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(I8PairCfg<STAGES>::THREADS, 1)
k_i8_chain(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
           const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmA3,
           const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1,
           const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmB3, const I8Chain ch, int M,
           int* status) {
    using C = I8PairCfg<STAGES>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sE = sB + STAGES * C::B_BYTES;
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(sE + C::STAGE_EPI);
    volatile int* abort_flag = &ctl->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kx::cluster_ctarank();
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const int m_tiles = (M + 2 * BM - 1) / (2 * BM);
    const int last = ch.n_layers - 1;
    // global tile t -> layer l, m-tile, n-tile (row-block-major inside a layer)
    auto decode = [&](int t, int& l, int& mt, int& nt) {
        l = 0;
        while (l < last && t >= ch.L[l + 1].tile0) l++;
        const int u = t - ch.L[l].tile0;
        mt = u / ch.L[l].n_tiles_n;
        nt = u - mt * ch.L[l].n_tiles_n;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1);
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], 2 * C::EPI_WARPS);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {
        kx::tmem_alloc_pair(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish_pair();
    }
    kx::tc_fence_before();
    kx::cluster_sync();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    kx::griddep_wait();  // launched as a dependent of the quantiser of the chain's input
    kx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            const CUtensorMap* mA[KX_I8C_MAX] = {&tmA0, &tmA1, &tmA2, &tmA3};
            const CUtensorMap* mB[KX_I8C_MAX] = {&tmB0, &tmB1, &tmB2, &tmB3};
            for (int l = 0; l < ch.n_layers; l++) {
                kx::tma_prefetch_desc(mA[l]);
                kx::tma_prefetch_desc(mB[l]);
            }
            int it = 0;
            for (int t = cluster; t < ch.total_tiles && !*abort_flag; t += n_clusters) {
                int l, mt, nt;
                decode(t, l, mt, nt);
                const int rg = mt * 2 + static_cast<int>(rank);
                if (l > 0 && rg * BM < M &&
                    !wait_ready(ch.L[l - 1].ready + rg, static_cast<uint32_t>(ch.L[l - 1].n_tiles_n), abort_flag, status))
                    break;
                const int arow = mt * 2 * BM + static_cast<int>(rank) * BM, brow = nt * BN + static_cast<int>(rank) * (BN / 2);
                const int nk = (ch.L[l].k + C::BK - 1) / C::BK;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) break;
                    if (rank == 0) kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * (C::A_BYTES + C::B_BYTES));
                    const uint32_t full0 = kx::mapa(kx::smem_u32(&ctl->full[s]), 0);
                    kx::tma_load_2d_pair(sA + s * C::A_BYTES, mA[l], kb * C::BK, arow, full0);
                    kx::tma_load_2d_pair(sB + s * C::B_BYTES, mB[l], kb * C::BK, brow, full0);
                }
            }
            if (*abort_flag && rank == 0)
                for (int i = it > STAGES ? it - STAGES : 0; i < it; i++) drain_wait(&ctl->full[i % STAGES], (i / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = kx::idesc_i8(2 * BM, BN);
            int it = 0, j = 0;
            for (int t = cluster; t < ch.total_tiles && !*abort_flag; t += n_clusters, j++) {
                int l, mt, nt;
                decode(t, l, mt, nt);
                const int b = j & 1;
                if (!kx::mbar_wait(&ctl->acc_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t d = tmem + b * BN;
                const int nk = (ch.L[l].k + C::BK - 1) / C::BK;
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->full[s], (it / STAGES) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    kx::tc_fence_after();
                    const uint32_t a0 = kx::smem_u32(sA + s * C::A_BYTES), b0 = kx::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < C::BK / 32; kk++)
                        kx::mma_i8_pair(d, kx::desc_sw128_kmajor(a0 + kk * 32), kx::desc_sw128_kmajor(b0 + kk * 32), idesc,
                                        (kb | kk) != 0);
                    const uint32_t e = kx::smem_u32(&ctl->empty[s]);
                    kx::mma_commit_pair(e);
                    kx::mma_commit_pair(kx::mapa(e, 1));
                }
                if (!ok) break;
                const uint32_t f = kx::smem_u32(&ctl->acc_full[b]);
                kx::mma_commit_pair(f);
                kx::mma_commit_pair(kx::mapa(f, 1));
            }
            kx::mma_commit_pair(kx::smem_u32(&ctl->accf));
            drain_wait(&ctl->accf, 0);
        }
        __syncwarp();
    } else {
        const int ew = warp - 2;
        const int q = warp & 3;
        const int c_lo = (ew >> 2) * (BN / 4);
        float* stg = reinterpret_cast<float*>(sE + ew * 2048);
        const int row_off = static_cast<int>(rank) * BM + q * 32;
        const uint32_t acc_empty0 = kx::mapa(kx::smem_u32(&ctl->acc_empty[0]), 0);
        int j = 0;
        for (int t = cluster; t < ch.total_tiles; t += n_clusters, j++) {
            int l, mt, nt;
            decode(t, l, mt, nt);
            const I8CLayer& L = ch.L[l];
            const int b = j & 1;
            const bool full_ok = __all_sync(0xffffffffu, kx::mbar_wait(&ctl->acc_full[b], (j >> 1) & 1, abort_flag, status));
            // the dequantisation factors after the accumulator: a layer's row scales are written by the previous one
            EpiPre f{};
            {
                const int r0 = mt * 2 * BM + row_off;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int gr = r0 + 16 * (i >> 1) + 8 * (i & 1) + (lane >> 2);
                    f.sx[i] = gr < M ? __ldcg(L.sx + gr) : 0.0f;
                }
                const int c = nt * BN + c_lo + 2 * lane;
                f.sc.x = c < L.n ? __ldg(L.scale + c) : 0.0f;
                f.sc.y = c + 1 < L.n ? __ldg(L.scale + c + 1) : 0.0f;
                f.bi.x = L.bias && c < L.n ? __ldg(L.bias + c) : 0.0f;
                f.bi.y = L.bias && c + 1 < L.n ? __ldg(L.bias + c + 1) : 0.0f;
            }
            const uint32_t tb = tmem + b * BN + (static_cast<uint32_t>(q * 32) << 16);
            if (l == last) {  // fp32 output; no barriers from here on (the last layer's tiles come last)
                if (!full_ok) break;
                kx::tc_fence_after();
                epi_tile_i8<BN, false, ACTL>(tb, mt * 2 * BM + row_off, nt * BN, c_lo, stg, lane, f, L.y, nullptr, L.n, M, L.n,
                                             L.act, L.alpha);
            } else {  // the quantised-output epilogue of the QOUT kernel, then the tile counts as ready
                const int r0 = mt * 2 * BM + row_off;
                const int rg = mt * 2 + static_cast<int>(rank);
                const bool live = rg * BM < M;
                bool ok = full_ok;
                if (ok) {
                    kx::tc_fence_after();
                    float4* cf = reinterpret_cast<float4*>(stg);
                    __syncwarp();
                    cf[lane] = make_float4(f.sc.x, f.sc.y, f.bi.x, f.bi.y);
                    __syncwarp();
                    uint32_t mx[4] = {0u, 0u, 0u, 0u};
                    q_pass1<ACTH>(tb, c_lo, cf, lane, f, L.act, L.alpha, mx);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
                        mx[i] = max(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
                    }
                    if ((lane & 3) == 0)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int gr = r0 + 16 * (i >> 1) + (lane >> 2) + 8 * (i & 1);
                            if (gr < M) atomicMax(L.qo.rowmax + gr, mx[i]);
                        }
                    __threadfence();
                }
                kx::named_bar(1, C::EPI_WARPS * 32);
                if (ok && live && ew == 0 && lane == 0) atomicAdd(L.qo.cnt + rg, 1u);
                if (ok && live) {
                    if (lane == 0) ok = q_wait_count(L.qo.cnt + rg, static_cast<uint32_t>(L.n_tiles_n), abort_flag, status);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                }
                if (ok) {
                    const int gr = r0 + lane;
                    const uint32_t m = gr < M ? kx::ld_relaxed_gpu(L.qo.rowmax + gr) : 0u;
                    const bool nan_row = m >= 0x7F800000u;
                    float sxv = 1.0f, inv = 1.0f;
                    if (nan_row) {
                        sxv = __uint_as_float(0x7FC00000u);
                    } else if (m != 0u) {
                        sxv = __fdiv_rn(__uint_as_float(m), 127.0f);
                        inv = __fdiv_rn(1.0f, sxv);
                    }
                    if (nt == 0 && c_lo == 0 && gr < M) L.qo.sx[gr] = sxv;
                    q_pass2(tb, c_lo, lane, inv, nan_row, gr, nt * BN + c_lo, L.qo, M, L.n);
                    fence_proxy_async_global();  // the next layer reads these rows with TMA (the async proxy)
                }
                // the barrier orders every warp's stores before one thread's gpu-scope fence and count (the pattern of
                // a grid barrier): the other warps go on to the next tile instead of each waiting for its stores
                const bool stop = kx::named_bar_or(1, C::EPI_WARPS * 32, !ok || *abort_flag);
                if (!stop && live && ew == 0 && lane == 0) {
                    __threadfence();
                    atomicAdd(L.ready + rg, 1u);
                }
                if (stop) break;
            }
            kx::tc_fence_before();
            __syncwarp();
            if (lane == 0) kx::mbar_arrive_remote(acc_empty0 + b * static_cast<uint32_t>(sizeof(uint64_t)));
        }
    }
    kx::tc_fence_before();
    kx::cluster_sync();
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------------ 3xTF32
// Accuracy of the 3xTF32 product A.B = Ah.Bh + (Al.Bh + Ah.Bl): the tensor core adds each MMA's result into the
// fp32 accumulator with truncation, which shrinks the sum's magnitude by about 1.6e-8 per accumulated MMA
// (measured). So the two small cross terms accumulate in their own TMEM region (their truncation is 2^-11
// smaller), and the large Ah.Bh sum sees one MMA per 8 K. DRAIN, for long reductions: Ah.Bh accumulates chunks of
// KC_BLOCKS K blocks (256 K) into two alternating TMEM buffers, and the epilogue warps add every chunk into an fp32
// running sum in a third region with round-to-nearest adds (((P0 + P1) + P2) + ..., a fixed order), which bounds
// the truncated accumulation length by 32 MMAs: about 5e-7 per layer at any K. The result is running sum (or
// Ah.Bh sum) + cross terms, rounded to nearest. The persistent kernel (k_gemm_tf32x3_pp) alone sums all three
// products in one accumulator (no TMEM left for a separate one): ~6e-6 of the output scale at K = 1024.
// shared-memory bytes of the control block; the tile's bias (BN floats) follows it
constexpr int F32_CTL_BYTES = (static_cast<int>(sizeof(SmemCtl)) + 15) & ~15;
// warps per TMEM lane quarter in the final epilogue: the epilogue warp and the two converter warps of that quarter
constexpr int F32_EPI_PARTS = 3;

constexpr int KC_BLOCKS = 8;
// reductions longer than this drain: up to 2048 the undrained sum stays within ~5.5e-6 of the output scale (the
// 1e-5 per-product bound), and 256-column tiles run ~1.8x faster than the drained 128-column ones
constexpr int DRAIN_MIN_K = 2048;
template <int BN, int STAGES, bool DRAIN = false>
struct F32Cfg {
    static constexpr int BK = 32;  // fp32 elements of K per stage (128 bytes per row)
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // A hi, A lo, B hi, B lo
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + F32_CTL_BYTES + BN * 4;  // + the tile's bias
    // TMEM: [Ah.Bh | cross] or, draining, [Ah.Bh chunk 0 | Ah.Bh chunk 1 | cross | running sum]
    static constexpr uint32_t MAIN0 = 0, CROSS = DRAIN ? 2 * BN : BN, RUN = 3 * BN;
    static constexpr uint32_t TMEM_COLS = DRAIN ? 512 : 2 * BN;
    static_assert((DRAIN ? 4 : 2) * BN <= 512, "accumulator regions exceed TMEM");
};

using kx::tf32_split;

// Implicit-GEMM convolution geometry: output row m = (b, oy, ox), reduction index k = (ky, kx, ci) with ci
// fastest, matching the file's weight row order (tools/knx3.py:93-104). Group g = blockIdx.z reads input
// channels [g*cg, (g+1)*cg) and writes output channels [g*cog, (g+1)*cog).
struct ConvGeom {
    int H, W, C, Ho, Wo, kh, kw, sh, sw, dh, dw, pt, pl, cg, cog;
};

// ---- pieces shared by the one-CTA and the CTA-pair 3xTF32 kernels
// Thread roles (448 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue, warps 6-13 A converters.
// Converter warp cw (0..7) covers tile rows 4 P cw .. 4 P cw + 4 P - 1 (P = rows per thread: A_PASSES, or
// CM_PASSES for the 256-pixel tiles of the channel-major convolution); per pass, lanes 8i..8i+7 read one row's 128
// contiguous bytes (coalesced), split them, and write the 16-byte chunks to their swizzled places. For a
// convolution each thread's rows have their output-pixel geometry computed once per tile.
constexpr int F32_THREADS = 448;
constexpr int A_CONV_WARPS = 8;
constexpr int A_ROWS_PER_WARP = BM / A_CONV_WARPS;  // 16
constexpr int A_PASSES = A_ROWS_PER_WARP / 4;       // rows of one thread
template <int P>
struct ARowsT {
    long rbase[P];
    int iy0[P], ix0[P];
};

template <bool CONV>
__device__ __forceinline__ bool a_vec_ok(const float* A, int lda, const ConvGeom& cv) {
    return CONV ? ((cv.cg & 3) == 0 && (cv.C & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0)
                : (((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0));
}

template <bool CONV, int P>
__device__ __forceinline__ void a_rows_setup(ARowsT<P>& g, const ConvGeom& cv, int m0, int cw, int lane) {
    if constexpr (CONV) {
#pragma unroll
        for (int it = 0; it < P; it++) {
            const int gm = m0 + cw * 4 * P + it * 4 + (lane >> 3);
            const int hw = cv.Ho * cv.Wo;
            const int b = gm / hw, rem = gm - b * hw, oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
            g.rbase[it] = static_cast<long>(b) * cv.H;
            g.iy0[it] = oy * cv.sh - cv.pt;
            g.ix0[it] = ox * cv.sw - cv.pl;
        }
    }
}

// K block [k0, k0 + 32) of this warp's 32 rows (tile origin m0): load into registers (zero outside A)
template <bool CONV, int P>
__device__ __forceinline__ void a_load_block(const float* __restrict__ A, int lda, bool vec, const ConvGeom& cv,
                                             const ARowsT<P>& g, int M, int K, int m0, int cw, int lane, int k0,
                                             float4 (&v)[P]) {
    const int gk = k0 + (lane & 7) * 4;
    int ky = 0, kx2 = 0, ci = 0;
    if (CONV && gk < K) {
        const int tap = gk / cv.cg;
        ci = gk - tap * cv.cg;
        ky = tap / cv.kw;
        kx2 = tap - ky * cv.kw;
    }
#pragma unroll
    for (int it = 0; it < P; it++) {
        const int gm = m0 + cw * 4 * P + it * 4 + (lane >> 3);
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gm < M && gk < K) {
            if (!CONV) {
                const float* src = A + static_cast<size_t>(gm) * lda + gk;
                if (vec && gk + 3 < K) {
                    t = __ldg(reinterpret_cast<const float4*>(src));
                } else {
                    t.x = __ldg(src);
                    if (gk + 1 < K) t.y = __ldg(src + 1);
                    if (gk + 2 < K) t.z = __ldg(src + 2);
                    if (gk + 3 < K) t.w = __ldg(src + 3);
                }
            } else if (vec) {  // 4 consecutive channels of one tap
                const int iy = g.iy0[it] + ky * cv.dh, ix = g.ix0[it] + kx2 * cv.dw;
                if (iy >= 0 && iy < cv.H && ix >= 0 && ix < cv.W)
                    t = __ldg(reinterpret_cast<const float4*>(A + ((g.rbase[it] + iy) * cv.W + ix) * cv.C + ci));
            } else {  // channels per group not a multiple of 4: element by element
                float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int kq = gk + q;
                    if (kq >= K) break;
                    const int tap = kq / cv.cg, c = kq - tap * cv.cg, yy = tap / cv.kw, xx = tap - yy * cv.kw;
                    const int iy = g.iy0[it] + yy * cv.dh, ix = g.ix0[it] + xx * cv.dw;
                    if (iy >= 0 && iy < cv.H && ix >= 0 && ix < cv.W)
                        e[q] = __ldg(A + ((g.rbase[it] + iy) * cv.W + ix) * cv.C + c);
                }
                t = make_float4(e[0], e[1], e[2], e[3]);
            }
        }
        v[it] = t;
    }
}

// split the loaded block into hi / lo and store both into the stage's swizzled A tiles
template <int P>
__device__ __forceinline__ void a_store_block(const float4 (&v)[P], int cw, int lane, uint8_t* hi, uint8_t* lo) {
#pragma unroll
    for (int it = 0; it < P; it++) {
        const int r = cw * 4 * P + it * 4 + (lane >> 3);
        const int j = lane & 7;
        const int off = r * 128 + ((j ^ (r & 7)) << 4);
        float4 h, l;
        tf32_split(v[it].x, h.x, l.x);
        tf32_split(v[it].y, h.y, l.y);
        tf32_split(v[it].z, h.z, l.z);
        tf32_split(v[it].w, h.w, l.w);
        *reinterpret_cast<float4*>(hi + off) = h;
        *reinterpret_cast<float4*>(lo + off) = l;
    }
}

// Dense A: converter warp cw asks L2 for the 128-byte segments of its rows in the K block at k0; lane l takes row
// A_ROWS_PER_WARP cw + l % 16, the first float (lanes 0-15) or the last (lanes 16-31), so a segment that
// straddles two lines brings both.
__device__ __forceinline__ void a_prefetch_block(const float* __restrict__ A, int lda, int M, int K, int m0, int cw,
                                                 int lane, int k0) {
    static_assert(A_ROWS_PER_WARP == 16, "two prefetching lanes per row");
    const int gm = m0 + cw * A_ROWS_PER_WARP + (lane & 15);
    if (gm >= M || k0 >= K) return;
    const int off = lane < 16 ? 0 : (K - k0 < 32 ? K - k0 : 32) - 1;
    kx::prefetch_l2(A + static_cast<size_t>(gm) * lda + k0 + off);
}
constexpr int A_L2_AHEAD = 5;  // K blocks between the L2 prefetch of a block and its register load

// The converter warps' loop. Blocks kb + 1 and kb + 2 are in flight into registers (three rotating buffers, no
// register copies) while block kb waits for its stage and is split and stored, and (dense A) block
// kb + A_L2_AHEAD is requested into L2, so the load latency of A is hidden behind two stages. `arrive(s)` signals
// that stage s holds this warp's rows. P: rows per thread (the tile has 32 P rows). it0: the stage-ring position
// of block 0 (a persistent kernel's earlier tiles' blocks). False on a timeout.
template <bool CONV, int BK, int STAGES, int P = A_PASSES, class StageA, class Arrive>
__device__ __forceinline__ bool a_convert_loop(const float* __restrict__ A, int lda, const ConvGeom& cv, int M, int K,
                                               int m0, int cw, int lane, int nk, int it0, SmemCtl* ctl,
                                               volatile int* abort_flag, int* status, StageA stage_a, Arrive arrive) {
    const bool vec = a_vec_ok<CONV>(A, lda, cv);
    static_assert(CONV || P == A_PASSES, "the L2 prefetch of dense A covers A_PASSES rows per thread");
    ARowsT<P> g;
    a_rows_setup<CONV, P>(g, cv, m0, cw, lane);
    if constexpr (!CONV)
        for (int j = 2; j < A_L2_AHEAD; j++) a_prefetch_block(A, lda, M, K, m0, cw, lane, j * BK);
    float4 va[P], vb[P], vc[P];
    a_load_block<CONV, P>(A, lda, vec, cv, g, M, K, m0, cw, lane, 0, va);
    if (nk > 1) a_load_block<CONV, P>(A, lda, vec, cv, g, M, K, m0, cw, lane, BK, vb);
    // block kb from `cur`; block kb + 2 into `ahead`; false on a timeout
    auto step = [&](int kb, float4 (&cur)[P], float4 (&ahead)[P]) {
        const int it = it0 + kb, s = it % STAGES;
        if constexpr (!CONV) a_prefetch_block(A, lda, M, K, m0, cw, lane, (kb + A_L2_AHEAD) * BK);
        if (kb + 2 < nk) a_load_block<CONV, P>(A, lda, vec, cv, g, M, K, m0, cw, lane, (kb + 2) * BK, ahead);
        if (!kx::mbar_wait(&ctl->empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) return false;
        a_store_block<P>(cur, cw, lane, stage_a(s), stage_a(s) + 4 * P * A_CONV_WARPS * BK * 4);
        kx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive(s);
        return true;
    };
    for (int kb = 0; kb < nk; kb += 3) {
        if (!step(kb, va, vc)) return false;
        if (kb + 1 >= nk) break;
        if (!step(kb + 1, vb, va)) return false;
        if (kb + 2 >= nk) break;
        if (!step(kb + 2, vc, vb)) return false;
    }
    return true;
}

// DRAIN: add the finished Ah.Bh chunk at TMEM address t_chunk into the running sum at t_run (BN columns of this
// warp's 32 lanes; the first chunk is copied)
template <int BN>
__device__ __forceinline__ void f32_add_chunk(uint32_t t_chunk, uint32_t t_run, bool first) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t p[32], t[32];
        kx::tmem_ld32(t_chunk + c0, p);
        if (!first) kx::tmem_ld32(t_run + c0, t);
        kx::tmem_ld_wait();
        if (!first) {
#pragma unroll
            for (int j = 0; j < 32; j++) p[j] = __float_as_uint(__fadd_rn(__uint_as_float(t[j]), __uint_as_float(p[j])));
        }
        kx::tmem_st32(t_run + c0, p);
    }
    kx::tmem_st_wait();
}

// The epilogue warps copy the tile's bias columns [n0, n0 + BN) into shared memory while the mainloop runs (zero
// past N), then meet on named barrier 1 (the four epilogue warps only).
template <int BN>
__device__ __forceinline__ void f32_stage_bias(float* sbias, const float* __restrict__ bias, int n0, int N, int ew,
                                               int lane) {
    for (int i = ew * 32 + lane; i < BN; i += 128) sbias[i] = (bias && n0 + i < N) ? __ldg(bias + n0 + i) : 0.0f;
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// The residual values of one 32 x 32 output block as the store loops below write it (lane: rows 4 p + lane / 8,
// columns col0 + 4 (lane % 8) .. + 3), all eight loads issued at once so that their latency overlaps the block's
// TMEM loads and activation math; zero where the block leaves the output.
__device__ __forceinline__ void load_residual(const float* __restrict__ res, int ldr, bool rvec, int row0, int col0, int lane,
                                              int M, int N, float4 (&rv)[8]) {
    const int gcol = col0 + 4 * (lane & 7);
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const int grow = row0 + 4 * p + (lane >> 3);
        rv[p] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (grow >= M || gcol >= N) continue;
        const float* rp = res + static_cast<size_t>(grow) * ldr + gcol;
        if (rvec && gcol + 3 < N) {
            rv[p] = __ldg(reinterpret_cast<const float4*>(rp));
        } else {
            rv[p].x = __ldg(rp);
            if (gcol + 1 < N) rv[p].y = __ldg(rp + 1);
            if (gcol + 2 < N) rv[p].z = __ldg(rp + 2);
            if (gcol + 3 < N) rv[p].w = __ldg(rp + 3);
        }
    }
}
// y = (activation output) + res with round-to-nearest adds (the separate ADD step's arithmetic)
__device__ __forceinline__ float4 add4(float4 w, float4 r) {
    return make_float4(__fadd_rn(w.x, r.x), __fadd_rn(w.y, r.y), __fadd_rn(w.z, r.z), __fadd_rn(w.w, r.w));
}

// Final epilogue of one warp's 32 rows (TMEM lanes; thread = row row0 + lane), 32-column blocks part, part + 3, ...
// (the three warps of a TMEM lane quarter share a tile's blocks): (Ah.Bh sum + cross terms) rounded
// to nearest, bias (from the shared-memory copy), activation. Each 32-column block is staged through one of the
// warp's two 4 KB shared-memory buffers `stg` (row r's float4 j at r * 8 + (j ^ (r & 7)), conflict-free both ways;
// the two alternate, so the next block's staging never waits for this block's reads) and written with lanes
// 8i..8i+7 covering one row's 128 contiguous bytes, four full rows per store instruction. `ok` must be the same in
// the whole warp.
template <int BN, int ACTC>
__device__ __forceinline__ void f32_store_tile(uint32_t t_sum, uint32_t t_cross, bool ok, int row0, int lane, int n0,
                                               const float* sbias, bool has_bias, float* __restrict__ y, int ldy,
                                               int M, int N, int act, float alpha, float4* stg, int part,
                                               const float* __restrict__ res, int ldr) {
    const bool vec = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
    const bool rvec = ((ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(res) & 15) == 0);
#pragma unroll 1
    for (int c0 = 32 * part; c0 < BN; c0 += 32 * F32_EPI_PARTS) {
        uint32_t r[32], x[32];
        kx::tmem_ld32(t_sum + c0, r);
        kx::tmem_ld32(t_cross + c0, x);
        const int col0 = n0 + c0;
        float4 rv[8];
        if (res && ok) load_residual(res, ldr, rvec, row0, col0, lane, M, N, rv);
        kx::tmem_ld_wait();
        if (!ok || col0 >= N) continue;
        float4* buf = stg + ((c0 >> 5) & 1) * 256;
#pragma unroll
        for (int j4 = 0; j4 < 8; j4++) {
            const float4 b4 = reinterpret_cast<const float4*>(sbias)[(c0 >> 2) + j4];
            const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float t = __fadd_rn(__uint_as_float(r[4 * j4 + e]), __uint_as_float(x[4 * j4 + e]));
                if (has_bias) t = __fadd_rn(t, bb[e]);
                v[e] = epi_act<ACTC>(t, act, alpha);
            }
            buf[lane * 8 + (j4 ^ (lane & 7))] = make_float4(v[0], v[1], v[2], v[3]);
        }
        __syncwarp();
        const int q = lane & 7, gcol = col0 + 4 * q;
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const int rr = 4 * p + (lane >> 3), grow = row0 + rr;
            float4 w = buf[rr * 8 + (q ^ (rr & 7))];
            if (grow >= M || gcol >= N) continue;
            if (res) w = add4(w, rv[p]);
            float* dst = y + static_cast<size_t>(grow) * ldy + gcol;
            if (vec && gcol + 3 < N) {
                *reinterpret_cast<float4*>(dst) = w;
            } else {
                dst[0] = w.x;
                if (gcol + 1 < N) dst[1] = w.y;
                if (gcol + 2 < N) dst[2] = w.z;
                if (gcol + 3 < N) dst[3] = w.w;
            }
        }
    }
}

template <int BN, int STAGES, bool CONV, int ACTC, bool DRAIN>
__global__ void __launch_bounds__(F32_THREADS, 1)
k_gemm_tf32x3(const float* __restrict__ A, int lda, const __grid_constant__ CUtensorMap tmBhi,
              const __grid_constant__ CUtensorMap tmBlo, const float* __restrict__ bias, float* __restrict__ y, int ldy,
              int M, int N, int K, int act, float alpha, int* status, const ConvGeom cv, const float* __restrict__ res,
              int ldr, int ksl) {
    using C = F32Cfg<BN, STAGES, DRAIN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + STAGES * C::STAGE_BYTES);
    // dense split-K (ksl > 0): CTA z of the grid's third dimension takes K range [z ksl, (z + 1) ksl) (ksl a multiple of
    // 256, whole drain chunks) and writes its raw sums into plane z of y (M x ldy each); the caller adds the planes
    const int kz = !CONV && ksl > 0 ? static_cast<int>(blockIdx.z) * ksl : 0;
    if (!CONV && ksl > 0) {
        A += kz;
        K = min(K - kz, ksl);
        y += static_cast<size_t>(blockIdx.z) * M * ldy;
    }
    volatile int* abort_flag = &ctl->abort;
    auto sAhi = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto sAlo = [&](int s) { return smem + s * C::STAGE_BYTES + C::A_BYTES; };
    auto sBhi = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES; };
    auto sBlo = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nk = (K + C::BK - 1) / C::BK;
    const int grp = CONV ? static_cast<int>(blockIdx.z) : 0;
    const int brow0 = grp * (CONV ? cv.cog : 0);  // first weight row / output column of this group
    if (CONV) {
        A += grp * cv.cg;
        y += brow0;
        if (bias) bias += brow0;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1 + A_CONV_WARPS);  // TMA producer + the converter warps
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {  // DRAIN: chunk buffer b holds a finished chunk / has been added in
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], 4);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {
        kx::tmem_alloc(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish();
    }
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmBhi);
            kx::tma_prefetch_desc(&tmBlo);
            int issued = 0;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % STAGES;
                if (!kx::mbar_wait(&ctl->empty[s], ((kb / STAGES) & 1) ^ 1, abort_flag, status)) break;
                kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * C::B_BYTES);
                kx::tma_load_2d(sBhi(s), &tmBhi, kz + kb * C::BK, brow0 + n0, &ctl->full[s]);
                kx::tma_load_2d(sBlo(s), &tmBlo, kz + kb * C::BK, brow0 + n0, &ctl->full[s]);
                issued = kb + 1;
            }
            if (*abort_flag)
                for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++)
                    drain_wait(&ctl->full[kb % STAGES], (kb / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(BM, BN);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % STAGES;
                const int c = DRAIN ? kb / KC_BLOCKS : 0, kc = DRAIN ? kb % KC_BLOCKS : kb;  // chunk, block in chunk
                const uint32_t d = tmem + (DRAIN ? (c & 1) * BN : C::MAIN0), dx = tmem + C::CROSS;
                if (DRAIN && kc == 0) {  // chunk buffer free: the epilogue has added chunk c - 2 in
                    if (!kx::mbar_wait(&ctl->acc_empty[c & 1], ((c >> 1) & 1) ^ 1, abort_flag, status)) break;
                    kx::tc_fence_after();
                }
                if (!kx::mbar_wait(&ctl->full[s], (kb / STAGES) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t ah = kx::smem_u32(sAhi(s)), al = kx::smem_u32(sAlo(s));
                const uint32_t bh = kx::smem_u32(sBhi(s)), bl = kx::smem_u32(sBlo(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 8; kk++) {
                    const uint32_t o = kk * 32;  // 8 tf32 = 32 bytes of K per MMA
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(al + o), kx::desc_sw128_kmajor(bh + o), idesc, (kb | kk) != 0);
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bl + o), idesc, 1);
                    kx::mma_tf32(d, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bh + o), idesc, (kc | kk) != 0);
                }
                kx::mma_commit(&ctl->empty[s]);
                if (DRAIN && (kc == KC_BLOCKS - 1 || kb == nk - 1)) kx::mma_commit(&ctl->acc_full[c & 1]);
            }
            kx::mma_commit(&ctl->accf);
        }
        __syncwarp();
    } else if (warp < 6) {
        const int q = warp & 3;
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        float* sbias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + F32_CTL_BYTES);
        f32_stage_bias<BN>(sbias, bias, n0, N, warp - 2, lane);
        if (DRAIN) {  // add each chunk into the running sum
            const int nchunks = (nk + KC_BLOCKS - 1) / KC_BLOCKS;
            for (int c = 0; c < nchunks; c++) {
                if (!kx::mbar_wait(&ctl->acc_full[c & 1], (c >> 1) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                f32_add_chunk<BN>(tmem + lanes + (c & 1) * BN, tmem + lanes + C::RUN, c == 0);
                kx::tc_fence_before();
                __syncwarp();
                if (lane == 0) kx::mbar_arrive(&ctl->acc_empty[c & 1]);
            }
        }
    } else {
        a_convert_loop<CONV, C::BK, STAGES>(A, lda, cv, M, K, m0, warp - 6, lane, nk, 0, ctl, abort_flag, status, sAhi,
                                            [&](int s) { kx::mbar_arrive(&ctl->full[s]); });
    }
    if (warp >= 2) {
        // Final epilogue on twelve warps: per TMEM lane quarter the epilogue warp and the two converter warps of that
        // quarter share the tile's 32-column blocks. Every MMA has completed (accf): the operand stages are free and
        // warp w stages its stores in 8 KB of them; named barrier 2 (these twelve warps) makes the bias copy visible.
        drain_wait(&ctl->accf, 0);
        kx::tc_fence_after();
        asm volatile("bar.sync 2, 384;" ::: "memory");
        const int q = warp & 3, part = warp < 6 ? 0 : (warp < 10 ? 1 : 2);
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        const float* sbias = reinterpret_cast<const float*>(reinterpret_cast<uint8_t*>(ctl) + F32_CTL_BYTES);
        const bool ok = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
        f32_store_tile<BN, ACTC>(tmem + lanes + (DRAIN ? C::RUN : C::MAIN0), tmem + lanes + C::CROSS, ok, m0 + q * 32, lane,
                                 n0, sbias, bias != nullptr, y, ldy, M, N, act, alpha,
                                 reinterpret_cast<float4*>(smem + (warp - 2) * 8192), part, res, ldr);
    }
    kx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ 3xTF32, persistent CTA pairs
// For dense layers with K <= PP_MAX_K and more 256 x 256 tiles than resident clusters: the CTA-pair kernel above,
// made persistent so that a tile's epilogue overlaps the next tile's mainloop. A cluster walks tiles t = cluster,
// + clusters, ... (M-tile fastest: the clusters running at once share B tiles in L2); the TMA producer and the
// converters run ahead through the 3-stage ring across tile boundaries, and TMEM holds two 256-column accumulators
// (one per tile in flight), so the three products of a tile (Ah.Bh, Al.Bh, Ah.Bl) share one accumulator instead of
// keeping the cross terms apart: with the truncating accumulation of tcgen05 that costs ~6e-6 of the output scale
// at K = 1024 (~3e-6 at K = 512), inside the 1e-5 bound of the other 3xTF32 paths. The four epilogue warps of each
// CTA drain a tile (the next tile's bias columns fetched into registers a tile ahead, then copied into the warp's own
// shared-memory buffer, so that no barrier joins the warps; 32x32 blocks staged through a 4 KB per-warp buffer;
// full-row stores) and free its accumulator on rank 0's acc_empty.
constexpr int PP_MAX_K = 1024;
struct PpCfg {
    static constexpr int BN = 256;
    static constexpr int BK = 32;
    static constexpr int STAGES = 3;
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = (BN / 2) * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STG_BYTES = 4096;  // per epilogue warp
    static constexpr int BIAS_BYTES = 2 * BN * 4;  // per epilogue warp: two tiles' bias columns
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + F32_CTL_BYTES + 4 * BIAS_BYTES + 4 * STG_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
};

// one warp's 32 rows of a finished tile (thread = row row0 + lane): accumulator + bias, activation, 32-column blocks
// staged through the warp's 4 KB buffer `stg` and written as full 128-byte row segments
template <int ACTC>
__device__ __forceinline__ void pp_store_tile(uint32_t t_acc, int row0, int lane, int n0, const float* sbias, bool has_bias,
                                              float* __restrict__ y, int ldy, int M, int N, int act, float alpha, float4* stg,
                                              const float* __restrict__ res, int ldr) {
    constexpr int BN = PpCfg::BN;
    const bool vec = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
    const bool rvec = ((ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(res) & 15) == 0);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        kx::tmem_ld32(t_acc + c0, r);
        const int col0 = n0 + c0;
        float4 rv[8];
        if (res) load_residual(res, ldr, rvec, row0, col0, lane, M, N, rv);
        kx::tmem_ld_wait();
        if (col0 >= N) break;
        __syncwarp();  // the previous block's reads of stg are done
#pragma unroll
        for (int j4 = 0; j4 < 8; j4++) {
            const float4 b4 = reinterpret_cast<const float4*>(sbias)[(c0 >> 2) + j4];
            const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float t = __uint_as_float(r[4 * j4 + e]);
                if (has_bias) t = __fadd_rn(t, bb[e]);
                v[e] = epi_act<ACTC>(t, act, alpha);
            }
            stg[lane * 8 + (j4 ^ (lane & 7))] = make_float4(v[0], v[1], v[2], v[3]);
        }
        __syncwarp();
        const int q = lane & 7, gcol = col0 + 4 * q;
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const int rr = 4 * p + (lane >> 3), grow = row0 + rr;
            float4 w = stg[rr * 8 + (q ^ (rr & 7))];
            if (grow >= M || gcol >= N) continue;
            if (res) w = add4(w, rv[p]);
            float* dst = y + static_cast<size_t>(grow) * ldy + gcol;
            if (vec && gcol + 3 < N) {
                *reinterpret_cast<float4*>(dst) = w;
            } else {
                dst[0] = w.x;
                if (gcol + 1 < N) dst[1] = w.y;
                if (gcol + 2 < N) dst[2] = w.z;
                if (gcol + 3 < N) dst[3] = w.w;
            }
        }
    }
}

template <int ACTC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(F32_THREADS, 1)
k_gemm_tf32x3_pp(const float* __restrict__ A, int lda, const __grid_constant__ CUtensorMap tmBhi,
                 const __grid_constant__ CUtensorMap tmBlo, const float* __restrict__ bias, float* __restrict__ y, int ldy,
                 int M, int N, int K, int act, float alpha, int* status, const float* __restrict__ res, int ldr) {
    using C = PpCfg;
    constexpr int BN = C::BN, STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);  // the same offset in both CTAs (same kernel, same static layout)
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + STAGES * C::STAGE_BYTES);
    float* sbias_all = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + F32_CTL_BYTES);  // 4 warps x 2 x BN
    float4* stg_all = reinterpret_cast<float4*>(sbias_all + 4 * 2 * BN);                           // 4 warps x 4 KB
    volatile int* abort_flag = &ctl->abort;
    auto sAhi = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto sAlo = [&](int s) { return smem + s * C::STAGE_BYTES + C::A_BYTES; };
    auto sBhi = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES; };
    auto sBlo = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kx::cluster_ctarank();
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const int nk = (K + C::BK - 1) / C::BK;
    const TileMap tm{(M + 2 * BM - 1) / (2 * BM), (N + BN - 1) / BN};
    const int n_tiles = tm.m_tiles * tm.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1 + 2 * A_CONV_WARPS);  // rank 0's producer + the converter warps of both CTAs
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], 8);  // the epilogue warps of both CTAs
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {  // warp 1 of both CTAs, same destination offset
        kx::tmem_alloc_pair(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish_pair();
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    const uint32_t full0 = kx::mapa(kx::smem_u32(&ctl->full[0]), 0);  // rank 0's full[0]; full[s] = + 8 s

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmBhi);
            kx::tma_prefetch_desc(&tmBlo);
            int it = 0;
            for (int t = cluster; t < n_tiles && !*abort_flag; t += n_clusters) {
                int mt, nt;
                tm.at(t, mt, nt);
                const int brow = nt * BN + static_cast<int>(rank) * (BN / 2);
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, status)) break;
                    if (rank == 0) kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * 2 * C::B_BYTES);
                    const uint32_t bar = full0 + 8u * static_cast<uint32_t>(s);
                    kx::tma_load_2d_pair(sBhi(s), &tmBhi, kb * C::BK, brow, bar);
                    kx::tma_load_2d_pair(sBlo(s), &tmBlo, kb * C::BK, brow, bar);
                }
            }
            if (*abort_flag && rank == 0)  // the stages armed here also carry the peer's copies
                for (int i = it > STAGES ? it - STAGES : 0; i < it; i++) drain_wait(&ctl->full[i % STAGES], (i / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(2 * BM, BN);
            int it = 0, j = 0;
            for (int t = cluster; t < n_tiles && !*abort_flag; t += n_clusters, j++) {
                const int b = j & 1;
                if (!kx::mbar_wait(&ctl->acc_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!kx::mbar_wait(&ctl->full[s], (it / STAGES) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    kx::tc_fence_after();
                    const uint32_t ah = kx::smem_u32(sAhi(s)), al = kx::smem_u32(sAlo(s));
                    const uint32_t bh = kx::smem_u32(sBhi(s)), bl = kx::smem_u32(sBlo(s));
#pragma unroll
                    for (int kk = 0; kk < C::BK / 8; kk++) {
                        const uint32_t o = kk * 32;
                        kx::mma_tf32_pair(d, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bh + o), idesc, (kb | kk) != 0);
                        kx::mma_tf32_pair(d, kx::desc_sw128_kmajor(al + o), kx::desc_sw128_kmajor(bh + o), idesc, 1);
                        kx::mma_tf32_pair(d, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bl + o), idesc, 1);
                    }
                    const uint32_t e = kx::smem_u32(&ctl->empty[s]);
                    kx::mma_commit_pair(e);
                    kx::mma_commit_pair(kx::mapa(e, 1));
                }
                if (!ok) break;
                const uint32_t f = kx::smem_u32(&ctl->acc_full[b]);
                kx::mma_commit_pair(f);
                kx::mma_commit_pair(kx::mapa(f, 1));
            }
            kx::mma_commit_pair(kx::smem_u32(&ctl->accf));  // completes once every MMA issued above has finished
            drain_wait(&ctl->accf, 0);
        }
        __syncwarp();
    } else if (warp < 6) {
        const int ew = warp - 2, q = warp & 3;
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        float4* stg = stg_all + ew * (C::STG_BYTES / 16);
        float* sbias = sbias_all + ew * 2 * BN;
        const uint32_t acc_empty0 = kx::mapa(kx::smem_u32(&ctl->acc_empty[0]), 0);
        const int bc = 8 * lane;  // the eight bias columns this lane fetches
        auto fetch_bias = [&](int t, float (&v)[8]) {
            int mt, nt;
            tm.at(t, mt, nt);
            const int c = nt * BN + bc;
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = (bias && c + e < N) ? __ldg(bias + c + e) : 0.0f;
        };
        float bcur[8], bnext[8];
#pragma unroll
        for (int e = 0; e < 8; e++) bcur[e] = bnext[e] = 0.0f;
        if (cluster < n_tiles) fetch_bias(cluster, bcur);
        int j = 0;
        for (int t = cluster; t < n_tiles; t += n_clusters, j++) {
            int mt, nt;
            tm.at(t, mt, nt);
            const int b = j & 1;
            if (t + n_clusters < n_tiles) fetch_bias(t + n_clusters, bnext);
            float* sb = sbias + b * BN;
            reinterpret_cast<float4*>(sb + bc)[0] = make_float4(bcur[0], bcur[1], bcur[2], bcur[3]);
            reinterpret_cast<float4*>(sb + bc)[1] = make_float4(bcur[4], bcur[5], bcur[6], bcur[7]);
            __syncwarp();  // the tile's bias columns are in this warp's buffer
            if (!kx::mbar_wait(&ctl->acc_full[b], (j >> 1) & 1, abort_flag, status)) break;
            kx::tc_fence_after();
            pp_store_tile<ACTC>(tmem + lanes + b * BN, mt * 2 * BM + static_cast<int>(rank) * BM + q * 32, lane, nt * BN, sb,
                                bias != nullptr, y, ldy, M, N, act, alpha, stg, res, ldr);
#pragma unroll
            for (int e = 0; e < 8; e++) bcur[e] = bnext[e];
            kx::tc_fence_before();
            __syncwarp();
            if (lane == 0) kx::mbar_arrive_remote(acc_empty0 + 8u * static_cast<uint32_t>(b));
        }
    } else {
        const int cw = warp - 6;
        int j = 0;
        for (int t = cluster; t < n_tiles && !*abort_flag; t += n_clusters, j++) {
            int mt, nt;
            tm.at(t, mt, nt);
            const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
            if (!a_convert_loop<false, C::BK, STAGES>(A, lda, ConvGeom{}, M, K, m0, cw, lane, nk, j * nk, ctl, abort_flag,
                                                      status, sAhi,
                                                      [&](int s) { kx::mbar_arrive_remote(full0 + 8u * static_cast<uint32_t>(s)); }))
                break;
        }
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // no CTA leaves while its peer may still signal it or read its shared memory
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ 3xTF32 convolution, channel-major tiles
// For at most 128 output channels per group the row-major tiles above leave most of each MMA's columns empty (a
// 64-channel layer fills 64 of a 128-column tile) while a tcgen05.mma costs about the same time at N = 128 as at
// N = 256 (measured), so here the operands swap roles: D^T = W . X^T, the group's weight rows (output channels,
// padded to 128 by the TMA's zero fill) are the A operand and 256 gathered output pixels the B operand, one
// M = 128 x N = 256 MMA per 8 K and product. TMEM lane c holds channel c, column p pixel p: Ah.Bh in columns
// [0, 256), the cross terms in [256, 512). 320 threads: warp 0 TMA (weights), warp 1 MMA, warps 2-9 convert 32
// pixel rows each (no separate epilogue warps, which leaves each converter thread the registers for its 8 rows);
// after the last MMA the converter warps are the epilogue, two per TMEM lane quarter sharing its 32-pixel column
// blocks, and lane c stores channel c of each pixel, so every store instruction writes a pixel's 32 consecutive
// channels (128 bytes). Reductions of at most DRAIN_MIN_K only (no chunk draining).
constexpr int CM_NP = 256;                              // output pixels per tile
constexpr int CM_THREADS = 64 + 32 * A_CONV_WARPS;
constexpr int CM_PASSES = CM_NP / A_CONV_WARPS / 4;      // pixel rows per converter thread
struct CmCfg {
    static constexpr int BK = 32;
    static constexpr int STAGES = 2;
    static constexpr int W_BYTES = BM * BK * 4;         // 128 weight rows of one plane
    static constexpr int X_BYTES = CM_NP * BK * 4;      // 256 pixel rows of one plane
    static constexpr int STAGE_BYTES = 2 * W_BYTES + 2 * X_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + F32_CTL_BYTES;
    static constexpr uint32_t MAIN0 = 0, CROSS = CM_NP, TMEM_COLS = 2 * CM_NP;
};

template <int ACTC>
__global__ void __launch_bounds__(CM_THREADS, 1)
k_conv_tf32x3_cm(const float* __restrict__ X, const __grid_constant__ CUtensorMap tmWhi,
                 const __grid_constant__ CUtensorMap tmWlo, const float* __restrict__ bias, float* __restrict__ y, int ldy,
                 int M, int K, int act, float alpha, int* status, const ConvGeom cv) {
    using C = CmCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + C::STAGES * C::STAGE_BYTES);
    volatile int* abort_flag = &ctl->abort;
    auto sWhi = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto sWlo = [&](int s) { return smem + s * C::STAGE_BYTES + C::W_BYTES; };
    auto sXhi = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::W_BYTES; };
    auto sXlo = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::W_BYTES + C::X_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * CM_NP;
    const int nk = (K + C::BK - 1) / C::BK;
    const int grp = static_cast<int>(blockIdx.y);
    const int wrow0 = grp * cv.cog;  // first weight row / output channel of this group
    X += grp * cv.cg;
    y += wrow0;
    if (bias) bias += wrow0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1 + A_CONV_WARPS);  // TMA producer + the converter warps
            kx::mbar_init(&ctl->empty[s], 1);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {
        kx::tmem_alloc(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish();
    }
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmWhi);
            kx::tma_prefetch_desc(&tmWlo);
            int issued = 0;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % C::STAGES;
                if (!kx::mbar_wait(&ctl->empty[s], ((kb / C::STAGES) & 1) ^ 1, abort_flag, status)) break;
                kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * C::W_BYTES);
                kx::tma_load_2d(sWhi(s), &tmWhi, kb * C::BK, wrow0, &ctl->full[s]);
                kx::tma_load_2d(sWlo(s), &tmWlo, kb * C::BK, wrow0, &ctl->full[s]);
                issued = kb + 1;
            }
            if (*abort_flag)
                for (int kb = issued > C::STAGES ? issued - C::STAGES : 0; kb < issued; kb++)
                    drain_wait(&ctl->full[kb % C::STAGES], (kb / C::STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(BM, CM_NP);
            const uint32_t d = tmem + C::MAIN0, dx = tmem + C::CROSS;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % C::STAGES;
                if (!kx::mbar_wait(&ctl->full[s], (kb / C::STAGES) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t wh = kx::smem_u32(sWhi(s)), wl = kx::smem_u32(sWlo(s));
                const uint32_t xh = kx::smem_u32(sXhi(s)), xl = kx::smem_u32(sXlo(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 8; kk++) {
                    const uint32_t o = kk * 32;  // 8 tf32 = 32 bytes of K per MMA
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(wl + o), kx::desc_sw128_kmajor(xh + o), idesc, (kb | kk) != 0);
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(wh + o), kx::desc_sw128_kmajor(xl + o), idesc, 1);
                    kx::mma_tf32(d, kx::desc_sw128_kmajor(wh + o), kx::desc_sw128_kmajor(xh + o), idesc, (kb | kk) != 0);
                }
                kx::mma_commit(&ctl->empty[s]);
            }
            kx::mma_commit(&ctl->accf);
        }
        __syncwarp();
    } else {
        a_convert_loop<true, C::BK, C::STAGES, CM_PASSES>(X, 0, cv, M, K, m0, warp - 2, lane, nk, 0, ctl, abort_flag, status,
                                                          sXhi, [&](int s) { kx::mbar_arrive(&ctl->full[s]); });
        // Final epilogue: warp w reads TMEM lane quarter q = w % 4 (channels 32 q .. 32 q + 31, thread = channel) and
        // takes the quarter's 32-pixel column blocks part, part + 2, ...: (Ah.Bh + cross terms) rounded to nearest,
        // bias, activation, then per pixel one 128-byte store of its 32 channels.
        drain_wait(&ctl->accf, 0);
        kx::tc_fence_after();
        const int q = warp & 3, part = (warp - 2) >> 2;
        const int ch = q * 32 + lane;
        const bool ok = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
        if (ok && q * 32 < cv.cog) {
            const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
            const bool live = ch < cv.cog;
            const float bch = (bias && live) ? __ldg(bias + ch) : 0.0f;
#pragma unroll 1
            for (int c0 = 32 * part; c0 < CM_NP; c0 += 64) {
                if (m0 + c0 >= M) break;
                uint32_t r[32], x[32];
                kx::tmem_ld32(tmem + lanes + C::MAIN0 + c0, r);
                kx::tmem_ld32(tmem + lanes + C::CROSS + c0, x);
                kx::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    float t = __fadd_rn(__uint_as_float(r[j]), __uint_as_float(x[j]));
                    if (bias) t = __fadd_rn(t, bch);
                    const int pix = m0 + c0 + j;
                    if (live && pix < M) y[static_cast<size_t>(pix) * ldy + ch] = epi_act<ACTC>(t, act, alpha);
                }
            }
        }
    }
    kx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------- 3xTF32 convolution, channel-major tiles fed by TMA
// The channel-major convolution with its pixel operand loaded by the TMA instead of gathered by converter warps
// (whose ~13 GB/s of gathered rows per SM bound the kernel above at ~2.4 us per K block against ~1.1 us of MMAs).
// The activations are first split once into tf32 hi / lo planes (k_split_planes, into caller-provided scratch); a
// K block is one tap (ky, kx) and 32 channels, and its 256 output pixels (whole output rows of one image, or whole
// images) read a 4-D box {32 channels, Wo columns, rows, images} of each plane at (c0, kx dw - pl, oy0 + ky dh - pt,
// b0): stride 1 makes the box's pixels the tile's pixels in order, and the TMA's zero fill outside the tensor is the
// convolution's zero padding. The box lands in the canonical K-major 128-byte-swizzle layout of the B operand. 320
// threads: warp 0 TMA (weights and both planes), warp 1 MMA, warps 2-9 the epilogue of the kernel above after the
// last MMA. Conditions (checked by the host): stride 1, channels per group a multiple of 32, at most 128 output
// channels per group, K <= DRAIN_MIN_K, and 256 a multiple of the image's output pixels or of its output width.
struct CmtGeom {
    int cg, kw, dh, dw, pt, pl;  // channels per group, kernel width, dilation, padding (top, left)
    int Ho, Wo, rows, imgs;      // output size; output rows and images per 256-pixel tile
};

__global__ void __launch_bounds__(256) k_split_planes(const float* __restrict__ x, float* __restrict__ hi,
                                                      float* __restrict__ lo, long n) {
    const long n4 = n >> 2;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
        float4 h, l;
        tf32_split(v.x, h.x, l.x);
        tf32_split(v.y, h.y, l.y);
        tf32_split(v.z, h.z, l.z);
        tf32_split(v.w, h.w, l.w);
        reinterpret_cast<float4*>(hi)[i] = h;
        reinterpret_cast<float4*>(lo)[i] = l;
    }
    for (long i = 4 * n4 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long>(gridDim.x) * blockDim.x)
        tf32_split(x[i], hi[i], lo[i]);
}

template <int ACTC>
__global__ void __launch_bounds__(CM_THREADS, 1)
k_conv_tf32x3_cmt(const __grid_constant__ CUtensorMap tmXhi, const __grid_constant__ CUtensorMap tmXlo,
                  const __grid_constant__ CUtensorMap tmWhi, const __grid_constant__ CUtensorMap tmWlo,
                  const float* __restrict__ bias, float* __restrict__ y, int ldy, int cog, int M, int K, int act,
                  float alpha, int* status, const CmtGeom gm) {
    using C = CmCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + C::STAGES * C::STAGE_BYTES);
    volatile int* abort_flag = &ctl->abort;
    auto sWhi = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto sWlo = [&](int s) { return smem + s * C::STAGE_BYTES + C::W_BYTES; };
    auto sXhi = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::W_BYTES; };
    auto sXlo = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::W_BYTES + C::X_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * CM_NP;
    const int nk = (K + C::BK - 1) / C::BK;
    const int grp = static_cast<int>(blockIdx.y);
    const int wrow0 = grp * cog;
    y += wrow0;
    if (bias) bias += wrow0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1);
            kx::mbar_init(&ctl->empty[s], 1);
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {
        kx::tmem_alloc(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish();
    }
    kx::tc_fence_before();
    __syncthreads();
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmXhi);
            kx::tma_prefetch_desc(&tmXlo);
            kx::tma_prefetch_desc(&tmWhi);
            kx::tma_prefetch_desc(&tmWlo);
            const int hw = gm.Ho * gm.Wo;
            const int b0 = m0 / hw, oy0 = (m0 - b0 * hw) / gm.Wo;  // the tile's first image and output row
            int issued = 0;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % C::STAGES;
                if (!kx::mbar_wait(&ctl->empty[s], ((kb / C::STAGES) & 1) ^ 1, abort_flag, status)) break;
                kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * C::W_BYTES + 2 * C::X_BYTES);
                const int k0 = kb * C::BK, tap = k0 / gm.cg, ky = tap / gm.kw, kxx = tap - ky * gm.kw;
                const int c0 = grp * gm.cg + (k0 - tap * gm.cg);
                const int ix = kxx * gm.dw - gm.pl, iy = oy0 + ky * gm.dh - gm.pt;
                kx::tma_load_2d(sWhi(s), &tmWhi, k0, wrow0, &ctl->full[s]);
                kx::tma_load_2d(sWlo(s), &tmWlo, k0, wrow0, &ctl->full[s]);
                kx::tma_load_4d(sXhi(s), &tmXhi, c0, ix, iy, b0, &ctl->full[s]);
                kx::tma_load_4d(sXlo(s), &tmXlo, c0, ix, iy, b0, &ctl->full[s]);
                issued = kb + 1;
            }
            if (*abort_flag)
                for (int kb = issued > C::STAGES ? issued - C::STAGES : 0; kb < issued; kb++)
                    drain_wait(&ctl->full[kb % C::STAGES], (kb / C::STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(BM, CM_NP);
            const uint32_t d = tmem + C::MAIN0, dx = tmem + C::CROSS;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % C::STAGES;
                if (!kx::mbar_wait(&ctl->full[s], (kb / C::STAGES) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t wh = kx::smem_u32(sWhi(s)), wl = kx::smem_u32(sWlo(s));
                const uint32_t xh = kx::smem_u32(sXhi(s)), xl = kx::smem_u32(sXlo(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 8; kk++) {
                    const uint32_t o = kk * 32;
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(wl + o), kx::desc_sw128_kmajor(xh + o), idesc, (kb | kk) != 0);
                    kx::mma_tf32(dx, kx::desc_sw128_kmajor(wh + o), kx::desc_sw128_kmajor(xl + o), idesc, 1);
                    kx::mma_tf32(d, kx::desc_sw128_kmajor(wh + o), kx::desc_sw128_kmajor(xh + o), idesc, (kb | kk) != 0);
                }
                kx::mma_commit(&ctl->empty[s]);
            }
            kx::mma_commit(&ctl->accf);
        }
        __syncwarp();
    } else {
        drain_wait(&ctl->accf, 0);
        kx::tc_fence_after();
        const int q = warp & 3, part = (warp - 2) >> 2;
        const int ch = q * 32 + lane;
        const bool ok = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
        if (ok && q * 32 < cog) {
            const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
            const bool live = ch < cog;
            const float bch = (bias && live) ? __ldg(bias + ch) : 0.0f;
#pragma unroll 1
            for (int c0 = 32 * part; c0 < CM_NP; c0 += 64) {
                if (m0 + c0 >= M) break;
                uint32_t r[32], x[32];
                kx::tmem_ld32(tmem + lanes + C::MAIN0 + c0, r);
                kx::tmem_ld32(tmem + lanes + C::CROSS + c0, x);
                kx::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    float t = __fadd_rn(__uint_as_float(r[j]), __uint_as_float(x[j]));
                    if (bias) t = __fadd_rn(t, bch);
                    const int pix = m0 + c0 + j;
                    if (live && pix < M) y[static_cast<size_t>(pix) * ldy + ch] = epi_act<ACTC>(t, act, alpha);
                }
            }
        }
    }
    kx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------ 3xTF32, CTA pairs
// The same GEMM on 256 x BN output tiles computed by a cluster of two CTAs with M = 256 tcgen05.mma
// (cta_group::2). CTA rank r converts A rows [m0 + 128 r, +128) of each K block into its own shared memory and
// TMA-loads the hi / lo planes of B rows [n0 + (BN/2) r, +BN/2); the MMAs, issued by rank 0, read both CTAs'
// halves and leave rows [m0 + 128 r, +128) x BN columns in rank r's TMEM, which rank r's epilogue warps drain.
// Per SM a K block moves (BN/2) x 32 x 8 bytes of B instead of BN x 32 x 8 for the same MMA work, which halves
// the L2 -> SM traffic of B and frees shared memory for more stages (BN = 256: 3 stages of 64 KB where the
// one-CTA kernel holds 2 of 96 KB).
// Synchronisation: rank 0's full[s] completes on its producer's arrive (armed with both CTAs' B bytes), the
// arrivals of the sixteen converter warps of both CTAs (each after fence.proxy.async, which makes its shared-memory
// stores visible to the tensor core's async proxy; the same default-semantics remote arrive CUTLASS's sm100
// transform pipelines use to hand a converted stage to the 2-SM MMA) and both CTAs' TMA bytes. Rank 0's MMA thread
// commits each stage to empty[s] of both CTAs, each DRAIN chunk to acc_full of both and its last MMAs to accf of
// both (one commit per CTA, no multicast); the DRAIN epilogue warps of both CTAs arrive on rank 0's acc_empty.
// Every wait is bounded; neither CTA leaves before the closing cluster barrier.
template <int BN, bool DRAIN>
struct F32PairCfg {
    static constexpr int BK = 32;
    static constexpr int STAGES = BN == 256 ? 3 : 4;
    static constexpr int A_BYTES = BM * BK * 4;        // this CTA's 128 rows of one plane
    static constexpr int B_BYTES = (BN / 2) * BK * 4;  // this CTA's BN / 2 rows of one plane
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + F32_CTL_BYTES + BN * 4;  // + the tile's bias
    static constexpr uint32_t MAIN0 = 0, CROSS = DRAIN ? 2 * BN : BN, RUN = 3 * BN;
    static constexpr uint32_t TMEM_COLS = DRAIN ? 512 : 2 * BN;
    static_assert((DRAIN ? 4 : 2) * BN <= 512, "accumulator regions exceed TMEM");
};

template <int BN, bool CONV, int ACTC, bool DRAIN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(F32_THREADS, 1)
k_gemm_tf32x3_pair(const float* __restrict__ A, int lda, const __grid_constant__ CUtensorMap tmBhi,
                   const __grid_constant__ CUtensorMap tmBlo, const float* __restrict__ bias, float* __restrict__ y,
                   int ldy, int M, int N, int K, int act, float alpha, int* status, const ConvGeom cv,
                   const float* __restrict__ res, int ldr) {
    using C = F32PairCfg<BN, DRAIN>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);  // the same offset in both CTAs (same kernel, same static layout)
    SmemCtl* ctl = reinterpret_cast<SmemCtl*>(smem + STAGES * C::STAGE_BYTES);
    volatile int* abort_flag = &ctl->abort;
    auto sAhi = [&](int s) { return smem + s * C::STAGE_BYTES; };
    auto sAlo = [&](int s) { return smem + s * C::STAGE_BYTES + C::A_BYTES; };
    auto sBhi = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES; };
    auto sBlo = [&](int s) { return smem + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kx::cluster_ctarank();
    const int n0 = static_cast<int>(blockIdx.x >> 1) * BN, m0 = blockIdx.y * (2 * BM) + static_cast<int>(rank) * BM;
    const int nk = (K + C::BK - 1) / C::BK;
    const int grp = CONV ? static_cast<int>(blockIdx.z) : 0;
    const int brow0 = grp * (CONV ? cv.cog : 0);
    if (CONV) {
        A += grp * cv.cg;
        y += brow0;
        if (bias) bias += brow0;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            kx::mbar_init(&ctl->full[s], 1 + 2 * A_CONV_WARPS);  // rank 0's producer + the converter warps of both CTAs
            kx::mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            kx::mbar_init(&ctl->acc_full[b], 1);
            kx::mbar_init(&ctl->acc_empty[b], 8);  // the epilogue warps of both CTAs
        }
        kx::mbar_init(&ctl->accf, 1);
        ctl->abort = 0;
        kx::fence_mbar_init();
        kx::fence_proxy_async_smem();
    }
    if (warp == 1) {  // warp 1 of both CTAs, same destination offset
        kx::tmem_alloc_pair(&ctl->tmem, C::TMEM_COLS);
        kx::tmem_relinquish_pair();
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    kx::tc_fence_after();
    const uint32_t tmem = ctl->tmem;
    const uint32_t full0 = kx::mapa(kx::smem_u32(&ctl->full[0]), 0);  // rank 0's full[0]; full[s] = + 8 s

    if (warp == 0) {
        if (lane == 0) {
            kx::tma_prefetch_desc(&tmBhi);
            kx::tma_prefetch_desc(&tmBlo);
            const int brow = brow0 + n0 + static_cast<int>(rank) * (BN / 2);
            int issued = 0;
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % STAGES;
                if (!kx::mbar_wait(&ctl->empty[s], ((kb / STAGES) & 1) ^ 1, abort_flag, status)) break;
                if (rank == 0) kx::mbar_arrive_expect_tx(&ctl->full[s], 2 * 2 * C::B_BYTES);
                const uint32_t bar = full0 + 8u * static_cast<uint32_t>(s);
                kx::tma_load_2d_pair(sBhi(s), &tmBhi, kb * C::BK, brow, bar);
                kx::tma_load_2d_pair(sBlo(s), &tmBlo, kb * C::BK, brow, bar);
                issued = kb + 1;
            }
            if (*abort_flag && rank == 0)  // the stages armed here also carry the peer's copies
                for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++)
                    drain_wait(&ctl->full[kb % STAGES], (kb / STAGES) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = kx::idesc_tf32(2 * BM, BN);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % STAGES;
                const int c = DRAIN ? kb / KC_BLOCKS : 0, kc = DRAIN ? kb % KC_BLOCKS : kb;
                const uint32_t d = tmem + (DRAIN ? (c & 1) * BN : C::MAIN0), dx = tmem + C::CROSS;
                if (DRAIN && kc == 0) {
                    if (!kx::mbar_wait(&ctl->acc_empty[c & 1], ((c >> 1) & 1) ^ 1, abort_flag, status)) break;
                    kx::tc_fence_after();
                }
                if (!kx::mbar_wait(&ctl->full[s], (kb / STAGES) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                const uint32_t ah = kx::smem_u32(sAhi(s)), al = kx::smem_u32(sAlo(s));
                const uint32_t bh = kx::smem_u32(sBhi(s)), bl = kx::smem_u32(sBlo(s));
#pragma unroll
                for (int kk = 0; kk < C::BK / 8; kk++) {
                    const uint32_t o = kk * 32;
                    kx::mma_tf32_pair(dx, kx::desc_sw128_kmajor(al + o), kx::desc_sw128_kmajor(bh + o), idesc, (kb | kk) != 0);
                    kx::mma_tf32_pair(dx, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bl + o), idesc, 1);
                    kx::mma_tf32_pair(d, kx::desc_sw128_kmajor(ah + o), kx::desc_sw128_kmajor(bh + o), idesc, (kc | kk) != 0);
                }
                const uint32_t e = kx::smem_u32(&ctl->empty[s]);
                kx::mma_commit_pair(e);
                kx::mma_commit_pair(kx::mapa(e, 1));
                if (DRAIN && (kc == KC_BLOCKS - 1 || kb == nk - 1)) {
                    const uint32_t f = kx::smem_u32(&ctl->acc_full[c & 1]);
                    kx::mma_commit_pair(f);
                    kx::mma_commit_pair(kx::mapa(f, 1));
                }
            }
            const uint32_t f = kx::smem_u32(&ctl->accf);
            kx::mma_commit_pair(f);
            kx::mma_commit_pair(kx::mapa(f, 1));
        }
        __syncwarp();
    } else if (warp < 6) {
        const int q = warp & 3;
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        float* sbias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + F32_CTL_BYTES);
        f32_stage_bias<BN>(sbias, bias, n0, N, warp - 2, lane);
        if (DRAIN) {
            const uint32_t acc_empty0 = kx::mapa(kx::smem_u32(&ctl->acc_empty[0]), 0);
            const int nchunks = (nk + KC_BLOCKS - 1) / KC_BLOCKS;
            for (int c = 0; c < nchunks; c++) {
                if (!kx::mbar_wait(&ctl->acc_full[c & 1], (c >> 1) & 1, abort_flag, status)) break;
                kx::tc_fence_after();
                f32_add_chunk<BN>(tmem + lanes + (c & 1) * BN, tmem + lanes + C::RUN, c == 0);
                kx::tc_fence_before();
                __syncwarp();
                if (lane == 0) kx::mbar_arrive_remote(acc_empty0 + 8u * static_cast<uint32_t>(c & 1));
            }
        }
    } else {
        a_convert_loop<CONV, C::BK, STAGES>(A, lda, cv, M, K, m0, warp - 6, lane, nk, 0, ctl, abort_flag, status, sAhi,
                                            [&](int s) { kx::mbar_arrive_remote(full0 + 8u * static_cast<uint32_t>(s)); });
    }
    if (warp >= 2) {
        // Final epilogue on twelve warps: per TMEM lane quarter the epilogue warp and the two converter warps of that
        // quarter share the tile's 32-column blocks. Every MMA has completed (accf): the operand stages are free and
        // warp w stages its stores in 8 KB of them; named barrier 2 (these twelve warps) makes the bias copy visible.
        drain_wait(&ctl->accf, 0);
        kx::tc_fence_after();
        asm volatile("bar.sync 2, 384;" ::: "memory");
        const int q = warp & 3, part = warp < 6 ? 0 : (warp < 10 ? 1 : 2);
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        const float* sbias = reinterpret_cast<const float*>(reinterpret_cast<uint8_t*>(ctl) + F32_CTL_BYTES);
        const bool ok = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
        f32_store_tile<BN, ACTC>(tmem + lanes + (DRAIN ? C::RUN : C::MAIN0), tmem + lanes + C::CROSS, ok, m0 + q * 32, lane,
                                 n0, sbias, bias != nullptr, y, ldy, M, N, act, alpha,
                                 reinterpret_cast<float4*>(smem + (warp - 2) * 8192), part, res, ldr);
    }
    kx::tc_fence_before();
    kx::cluster_sync();  // no CTA leaves while its peer may still signal it or read its shared memory
    if (warp == 1) {
        kx::tc_fence_after();
        kx::tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t encode_fn() {
    static PFN_encodeTiled_t fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled_t>(p);
    });
    return fn;
}

// 2-D row-major tensor [outer][inner] with row pitch row_bytes; box box_inner x box_outer; 128-byte swizzle
struct MapKey {
    const void* base;
    uint64_t inner, outer, row_bytes;
    uint32_t box_inner, box_outer;
    int dt, swz;
};

struct MapEntry {
    MapKey key;
    CUtensorMap map;
    bool used;
};

thread_local MapEntry t_maps[64];

bool same_key(const MapKey& a, const MapKey& b) { return std::memcmp(&a, &b, sizeof(MapKey)) == 0; }

int make_map_2d(CUtensorMap* out, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    MapKey k;
    std::memset(&k, 0, sizeof k);
    k.base = base; k.inner = inner; k.outer = outer; k.row_bytes = row_bytes;
    k.box_inner = box_inner; k.box_outer = box_outer; k.dt = static_cast<int>(dt); k.swz = static_cast<int>(swz);
    const size_t h = (reinterpret_cast<uintptr_t>(base) >> 8 ^ inner * 31 ^ outer * 131 ^ box_outer) & 63;
    if (t_maps[h].used && same_key(t_maps[h].key, k)) {
        *out = t_maps[h].map;
        return 0;
    }
    PFN_encodeTiled_t enc = encode_fn();
    if (enc == nullptr) return -1;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return -1;  // TMA alignment rules
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    if (enc(out, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1;
    t_maps[h].key = k;
    t_maps[h].map = *out;
    t_maps[h].used = true;
    return 0;
}

// raise the dynamic shared-memory limit of a kernel once per (kernel, device); the attribute is per device context
int set_smem_once(const void* kern, int bytes) {
    struct Done {
        const void* k;
        uint64_t devs;
    };
    static Done done[32];
    static int n_done = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    std::lock_guard<std::mutex> g(mu);
    int i = 0;
    while (i < n_done && done[i].k != kern) i++;
    if (i < n_done && dev < 64 && ((done[i].devs >> dev) & 1)) return 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
    if (i == n_done && n_done < 32) done[n_done++] = Done{kern, 0};
    if (i < n_done && dev < 64) done[i].devs |= uint64_t(1) << dev;
    return 0;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 64 && cached[dev]) return cached[dev];
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev < 64) cached[dev] = n;
    return n;
}

template <int BN, bool ACC_ONLY, int ACTC>
int launch_i8(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale,
              const float* bias, float* y, int32_t* acc, int ldy, int m, int n, int k, int act, float alpha, int* status,
              cudaStream_t st, int kbs = 0) {
    constexpr int STAGES = 4;
    using C = I8Cfg<BN, STAGES>;
    CUtensorMap ta, tb;
    if (make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, static_cast<uint64_t>(ldq), static_cast<uint64_t>(m),
                    static_cast<uint64_t>(ldq), C::BK, BM) != 0 ||
        make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, static_cast<uint64_t>(ldw), static_cast<uint64_t>(n),
                    static_cast<uint64_t>(ldw), C::BK, BN) != 0)
        return -1;
    auto kern = k_gemm_i8<BN, STAGES, ACC_ONLY, ACTC>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    const int nk = (k + C::BK - 1) / C::BK;
    const int ranges = kbs > 0 ? (nk + kbs - 1) / kbs : 1;
    const int tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN) * ranges;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    if (kbs > 0)  // split-K: a dependent of the quantiser or row kernel before it
        return kx::launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM, st, ta, tb, sx, scale, bias, y, acc, ldy, m, n, k,
                              act, alpha, status, kbs);
    kern<<<grid, C::THREADS, C::SMEM, st>>>(ta, tb, sx, scale, bias, y, acc, ldy, m, n, k, act, alpha, status, kbs);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// The rows of a split-K int8 layer (kx_gemm_i8_split_acc's int32 planes [z][row][column]): one block of 1024 threads
// per row adds the planes (exact: int32 sums modulo 2^32 do not depend on the order; four columns per thread group read
// as one 16-byte load per plane, four planes' loads in flight at once; a row of fewer than 512 four-column groups gives
// each group G = 2..8 adjacent threads, which take every G-th plane and then add their sums by shuffles), then applies the epilogue's steps in its order --
// ((float)acc * sx) * scale + bias (0 without one), the activation on pairs of columns -- and either stores the fp32
// row or (QOUT) quantises it as the quantised-output epilogue does: the row's maximum |y| (NaN wins), sx = m / 127,
// inv = 1 / sx, q = rint(y inv) as the low byte of y inv + 1.5 2^23; columns N .. ldq - 1 are written as 0.
constexpr int I8R_THREADS = 1024, I8R_QUADS = 2, I8R_MAXN = 4 * I8R_THREADS * I8R_QUADS;
template <int ACTC, bool QOUT>
__global__ void __launch_bounds__(I8R_THREADS) k_i8_rows(const int32_t* __restrict__ part, int planes, int M, int N,
                                                          const float* __restrict__ sx, const float* __restrict__ scale,
                                                          const float* __restrict__ bias, int act, float alpha,
                                                          float* __restrict__ y, int ldy, int8_t* __restrict__ q, int ldq,
                                                          float* __restrict__ sx_out) {
    __shared__ uint32_t red[I8R_THREADS / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    kx::griddep_wait();  // launched as a dependent of the split-K GEMM that writes the planes
    kx::griddep_launch_dependents();
    const float sxr = __ldg(sx + row);
    const size_t plane = static_cast<size_t>(M) * N;
    const bool vec = (N & 3) == 0 && (reinterpret_cast<uintptr_t>(part) & 15) == 0;
    const bool yvec = !QOUT && ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
    const int quads = (N + 3) / 4;
    int G = 1;  // threads per four-column group
    while (G < 8 && quads * G * 2 <= I8R_THREADS) G *= 2;
    const int g = tid % G, per_pass = I8R_THREADS / G;
    float v[I8R_QUADS][4];
    uint32_t mx = 0u;
#pragma unroll
    for (int j = 0; j < I8R_QUADS; j++) {
        const int c = 4 * (tid / G + j * per_pass);
#pragma unroll
        for (int e = 0; e < 4; e++) v[j][e] = 0.0f;
        uint32_t acc[4] = {0u, 0u, 0u, 0u};  // modulo 2^32, as the MMA's int32 accumulator
        if (c < N) {
            const int32_t* src = part + static_cast<size_t>(row) * N + c;
            if (vec) {
                int z = g;
                for (; z + 3 * G < planes; z += 4 * G) {
                    int4 t[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) t[u] = __ldg(reinterpret_cast<const int4*>(src + (z + u * G) * plane));
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        acc[0] += static_cast<uint32_t>(t[u].x);
                        acc[1] += static_cast<uint32_t>(t[u].y);
                        acc[2] += static_cast<uint32_t>(t[u].z);
                        acc[3] += static_cast<uint32_t>(t[u].w);
                    }
                }
                for (; z < planes; z += G) {
                    const int4 t = __ldg(reinterpret_cast<const int4*>(src + z * plane));
                    acc[0] += static_cast<uint32_t>(t.x);
                    acc[1] += static_cast<uint32_t>(t.y);
                    acc[2] += static_cast<uint32_t>(t.z);
                    acc[3] += static_cast<uint32_t>(t.w);
                }
            } else {
                for (int z = g; z < planes; z += G)
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (c + e < N) acc[e] += static_cast<uint32_t>(__ldg(src + z * plane + e));
            }
        }
        // the group's lanes are adjacent within a warp (G divides 32); every lane takes part in the shuffles
        for (int o = 1; o < G; o <<= 1)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
        if (c >= N || g != 0) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {  // column pairs (c, c + 1) and (c + 2, c + 3), as the epilogue pairs them
            const int c0 = c + 2 * h;
            const bool has0 = c0 < N, has1 = c0 + 1 < N;
            const float2 f = kx::mul2(kx::mul2(make_float2(static_cast<float>(static_cast<int32_t>(acc[2 * h])),
                                                           static_cast<float>(static_cast<int32_t>(acc[2 * h + 1]))),
                                               kx::f2(sxr)),
                                      make_float2(has0 ? __ldg(scale + c0) : 0.0f, has1 ? __ldg(scale + c0 + 1) : 0.0f));
            const float2 b = make_float2(bias && has0 ? __ldg(bias + c0) : 0.0f, bias && has1 ? __ldg(bias + c0 + 1) : 0.0f);
            const float2 o = epi_act2<ACTC>(make_float2(__fadd_rn(f.x, b.x), __fadd_rn(f.y, b.y)), act, alpha);
            v[j][2 * h] = o.x;
            v[j][2 * h + 1] = o.y;
            if constexpr (QOUT) {
                if (has0) mx = kx::absmax_nan(mx, o.x);
                if (has1) mx = kx::absmax_nan(mx, o.y);
            }
        }
        if constexpr (!QOUT) {
            float* dst = y + static_cast<size_t>(row) * ldy + c;
            if (yvec && c + 3 < N) {
                *reinterpret_cast<float4*>(dst) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if (c + e < N) dst[e] = v[j][e];
            }
        }
    }
    if constexpr (QOUT) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((tid & 31) == 0) red[tid >> 5] = mx;
        __syncthreads();
        mx = red[0];
#pragma unroll
        for (int w = 1; w < I8R_THREADS / 32; w++) mx = max(mx, red[w]);
        const bool nan_row = mx >= 0x7F800000u;
        float sxv = 1.0f, inv = 1.0f;
        if (nan_row) {
            sxv = __uint_as_float(0x7FC00000u);
        } else if (mx != 0u) {
            sxv = __fdiv_rn(__uint_as_float(mx), 127.0f);
            inv = __fdiv_rn(1.0f, sxv);
        }
        if (tid == 0) sx_out[row] = sxv;
        uint32_t* qrow = reinterpret_cast<uint32_t*>(q + static_cast<size_t>(row) * ldq);
#pragma unroll
        for (int j = 0; j < I8R_QUADS; j++) {
            const int c = 4 * (tid / G + j * per_pass);
            if (c >= ldq || g != 0) continue;
            uint32_t w = 0u;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (!nan_row && c + e < N)
                    w |= (__float_as_uint(__fadd_rn(__fmul_rn(v[j][e], inv), 12582912.0f)) & 0xFFu) << (8 * e);
            qrow[c >> 2] = w;
        }
    }
}

// clusters of the pair kernel that can be resident at once (per kernel and device; 0 if the query fails)
int max_pair_clusters(const void* kern, int threads, int smem) {
    static std::mutex mu;
    static const void* keys[64];
    static int devs[64], vals[64], n = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < n; i++)
        if (keys[i] == kern && devs[i] == dev) return vals[i];
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * 148, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        c = 0;
    }
    if (n < 64) {
        keys[n] = kern;
        devs[n] = dev;
        vals[n] = c;
        n++;
    }
    return c;
}

template <bool ACC_ONLY, int ACTC, bool QOUT = false>
int launch_i8_pair(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale,
                   const float* bias, float* y, int32_t* acc, int ldy, int m, int n, int k, int act, float alpha, int* status,
                   cudaStream_t st, const QOut& qo = QOut{}) {
    constexpr int STAGES = 6;
    using C = I8PairCfg<STAGES>;
    CUtensorMap ta, tb;
    if (make_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, static_cast<uint64_t>(ldq), static_cast<uint64_t>(m),
                    static_cast<uint64_t>(ldq), C::BK, BM) != 0 ||
        make_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, static_cast<uint64_t>(ldw), static_cast<uint64_t>(n),
                    static_cast<uint64_t>(ldw), C::BK, C::BN / 2) != 0)
        return -1;
    auto kern = k_gemm_i8_pair<STAGES, ACC_ONLY, ACTC, QOUT>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    const int n_tiles_n = (n + C::BN - 1) / C::BN;
    const int tiles = ((m + 2 * BM - 1) / (2 * BM)) * n_tiles_n;
    int clusters = max_pair_clusters(reinterpret_cast<const void*>(kern), C::THREADS, C::SMEM);
    if (clusters <= 0) clusters = sm_count() / 2;
    // QOUT: a tile's pass 2 waits for every tile of its row group (consecutive in the walk) to finish pass 1, and a
    // cluster takes tile t + clusters only after finishing tile t; with at least n_tiles_n clusters every wait points
    // to tiles earlier in the walk, so the waits always end, whatever the cluster count
    if (QOUT && n_tiles_n > clusters) return -1;
    if (clusters > tiles) clusters = tiles;
    return kx::launch_pdl(kern, dim3(2 * clusters), dim3(C::THREADS), C::SMEM, st, ta, tb, sx, scale, bias, y, acc, ldy, m, n,
                          k, act, alpha, status, qo);
}

template <int BN, bool CONV, int ACTC, bool DRAIN>
int launch_f32(const float* x, int ldx, const float* whi, const float* wlo, int ldw, int wrows, const float* bias, float* y,
               int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st, const ConvGeom& cv,
               int groups, const float* res, int ldr, int splits = 1, int ksl = 0) {
    constexpr int STAGES = BN == 256 ? 2 : 3;
    using C = F32Cfg<BN, STAGES, DRAIN>;
    CUtensorMap th, tl;
    if (make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, whi, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BN) != 0 ||
        make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wlo, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BN) != 0)
        return -1;
    auto kern = k_gemm_tf32x3<BN, STAGES, CONV, ACTC, DRAIN>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM, CONV ? groups : splits);
    kern<<<grid, F32_THREADS, C::SMEM, st>>>(x, ldx, th, tl, bias, y, ldy, m, n, k, act, alpha, status, cv, res, ldr, ksl);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <int BN, bool CONV, int ACTC, bool DRAIN>
int launch_f32_pair(const float* x, int ldx, const float* whi, const float* wlo, int ldw, int wrows, const float* bias,
                    float* y, int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st,
                    const ConvGeom& cv, int groups, const float* res, int ldr) {
    using C = F32PairCfg<BN, DRAIN>;
    CUtensorMap th, tl;
    if (make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, whi, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BN / 2) != 0 ||
        make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wlo, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BN / 2) != 0)
        return -1;
    auto kern = k_gemm_tf32x3_pair<BN, CONV, ACTC, DRAIN>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    dim3 grid(2 * ((n + BN - 1) / BN), (m + 2 * BM - 1) / (2 * BM), groups);
    kern<<<grid, F32_THREADS, C::SMEM, st>>>(x, ldx, th, tl, bias, y, ldy, m, n, k, act, alpha, status, cv, res, ldr);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// persistent CTA-pair 3xTF32 launch: 1 (nothing launched) when the tiles fit in one wave of clusters, where the
// one-tile-per-cluster kernel (with its separate cross-term accumulator) costs the same
template <int ACTC>
int launch_f32_pp(const float* x, int ldx, const float* whi, const float* wlo, int ldw, int wrows, const float* bias, float* y,
                  int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st, const float* res, int ldr) {
    using C = PpCfg;
    auto kern = k_gemm_tf32x3_pp<ACTC>;
    const int tiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + C::BN - 1) / C::BN);
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    int clusters = max_pair_clusters(reinterpret_cast<const void*>(kern), F32_THREADS, C::SMEM);
    if (clusters <= 0) clusters = sm_count() / 2;
    if (tiles <= clusters) return 1;
    CUtensorMap th, tl;
    if (make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, whi, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, C::BN / 2) != 0 ||
        make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wlo, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, C::BN / 2) != 0)
        return -1;
    kern<<<2 * clusters, F32_THREADS, C::SMEM, st>>>(x, ldx, th, tl, bias, y, ldy, m, n, k, act, alpha, status, res, ldr);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <int ACTC>
int launch_conv_cm(const float* x, const float* whi, const float* wlo, int ldw, int wrows, const float* bias, float* y,
                   int ldy, int m, int k, int act, float alpha, int* status, cudaStream_t st, const ConvGeom& cv, int groups) {
    using C = CmCfg;
    CUtensorMap th, tl;
    if (make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, whi, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BM) != 0 ||
        make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wlo, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BM) != 0)
        return -1;
    auto kern = k_conv_tf32x3_cm<ACTC>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    dim3 grid((m + CM_NP - 1) / CM_NP, groups);
    kern<<<grid, CM_THREADS, C::SMEM, st>>>(x, th, tl, bias, y, ldy, m, k, act, alpha, status, cv);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// 4-D map of an NHWC fp32 activation tensor {C, W, H, B} (C innermost) with box {32, bw, bh, bn}, 128-byte swizzle
int make_map_nhwc(CUtensorMap* out, const float* base, int B, int H, int W, int C, uint32_t bw, uint32_t bh, uint32_t bn) {
    PFN_encodeTiled_t enc = encode_fn();
    if (enc == nullptr) return -1;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (C & 3)) return -1;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                          static_cast<cuuint64_t>(B)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 4, static_cast<cuuint64_t>(W) * C * 4,
                             static_cast<cuuint64_t>(H) * W * C * 4};
    cuuint32_t box[4] = {32, bw, bh, bn};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -1;
}

// tile shape of the TMA-fed channel-major convolution: 0 and (rows, images) per 256-pixel tile, or -1 if the
// output's geometry does not cut into whole rows / images
int cmt_tiling(int Ho, int Wo, int& rows, int& imgs) {
    const long P = static_cast<long>(Ho) * Wo;
    if (P <= 0 || Wo > 256) return -1;
    if (P <= CM_NP) {
        if (CM_NP % P) return -1;
        rows = Ho;
        imgs = static_cast<int>(CM_NP / P);
        return 0;
    }
    if (P % CM_NP || CM_NP % Wo) return -1;
    rows = CM_NP / Wo;
    imgs = 1;
    return 0;
}

template <int ACTC>
int launch_conv_cmt(const CUtensorMap& xh, const CUtensorMap& xl, const float* whi, const float* wlo, int ldw, int wrows,
                    const float* bias, float* y, int ldy, int cog, int m, int k, int act, float alpha, int* status,
                    cudaStream_t st, const CmtGeom& gm, int groups) {
    using C = CmCfg;
    CUtensorMap th, tl;
    if (make_map_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, whi, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BM) != 0 ||
        make_map_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wlo, static_cast<uint64_t>(ldw), static_cast<uint64_t>(wrows),
                    static_cast<uint64_t>(ldw) * 4, C::BK, BM) != 0)
        return -1;
    auto kern = k_conv_tf32x3_cmt<ACTC>;
    if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
    dim3 grid((m + CM_NP - 1) / CM_NP, groups);
    kern<<<grid, CM_THREADS, C::SMEM, st>>>(xh, xl, th, tl, bias, y, ldy, cog, m, k, act, alpha, status, gm);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ------------------------------------------------------------------- direct convolution, tiny K
// For reductions of at most DC_MAXK with at most 64 output channels per group (the first 3x3 layer over RGB: K = 27,
// 64 channels) a tensor-core tile spends its time on pipeline set-up and a whole epilogue per 32 K, so these layers run
// on the CUDA cores. Persistent blocks of 256 threads: lane l of every warp owns output channels l and l + 32 (their
// K weights in registers, w = hi + lo of the split planes, exact); per tile of DC_PIX consecutive output pixels the
// block gathers their K inputs into shared memory (zero outside the image, the file's (ky, kx, ci) order, through
// per-pixel and per-k offset tables), then warp w computes pixels w, w + 8, ...: fp32 fmas over the reduction in
// order, bias, activation, and two coalesced 128-byte stores per pixel.
constexpr int DC_MAXK = 32, DC_MAXCO = 64, DC_PIX = 64;
template <int ACTC>
__global__ void __launch_bounds__(256) k_conv_direct(const float* __restrict__ x, const float* __restrict__ whi,
                                                      const float* __restrict__ wlo, int ldw, const float* __restrict__ bias,
                                                      float* __restrict__ y, int M, int Co, int K, const ConvGeom cv,
                                                      int act, float alpha) {
    __shared__ __align__(16) float xs[DC_PIX][DC_MAXK];
    __shared__ int kdy[DC_MAXK], kdx[DC_MAXK], kci[DC_MAXK];  // per reduction index: input row / column offset, channel
    __shared__ int pb[2][DC_PIX], py[2][DC_PIX], px[2][DC_PIX];  // per pixel of a tile: image, top row, left column
    const int g = blockIdx.y, cog = cv.cog, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hw = cv.Ho * cv.Wo;
    if (threadIdx.x < DC_MAXK) {
        const int k = threadIdx.x, tap = k / cv.cg, ci = k - tap * cv.cg, ky = tap / cv.kw, kx2 = tap - ky * cv.kw;
        kdy[k] = ky * cv.dh;
        kdx[k] = kx2 * cv.dw;
        kci[k] = g * cv.cg + ci;
    }
    float w0[DC_MAXK], w1[DC_MAXK];
    const int c0 = lane, c1 = lane + 32;
#pragma unroll
    for (int k = 0; k < DC_MAXK; k++) {
        w0[k] = 0.0f;
        w1[k] = 0.0f;
        if (k < K) {
            if (c0 < cog) {
                const size_t src = static_cast<size_t>(g * cog + c0) * ldw + k;
                w0[k] = __fadd_rn(__ldg(whi + src), __ldg(wlo + src));
            }
            if (c1 < cog) {
                const size_t src = static_cast<size_t>(g * cog + c1) * ldw + k;
                w1[k] = __fadd_rn(__ldg(whi + src), __ldg(wlo + src));
            }
        }
    }
    const float b0 = (bias && c0 < cog) ? __ldg(bias + g * cog + c0) : 0.0f;
    const float b1 = (bias && c1 < cog) ? __ldg(bias + g * cog + c1) : 0.0f;
    // Tiles of DC_PIX pixels, software-pipelined: the next tile's inputs are requested into registers right after
    // this tile's are stored to shared memory, so their latency hides behind this tile's fmas.
    constexpr int PER = DC_PIX * DC_MAXK / 256;  // inputs gathered per thread
    auto geom = [&](int buf, int t0) {  // pixel geometry of the tile at t0 (threads 0 .. DC_PIX - 1)
        if (threadIdx.x < DC_PIX) {
            const int m = t0 + threadIdx.x;
            const int b = m / hw, rem = m - b * hw, oy = rem / cv.Wo, ox = rem - oy * cv.Wo;
            pb[buf][threadIdx.x] = b * cv.H;
            py[buf][threadIdx.x] = oy * cv.sh - cv.pt;
            px[buf][threadIdx.x] = ox * cv.sw - cv.pl;
        }
    };
    auto gather = [&](int buf, int t0, float (&v)[PER]) {  // all loads issued before any use
#pragma unroll
        for (int u = 0; u < PER; u++) {
            const int i = u * 256 + threadIdx.x, p = i / DC_MAXK, k = i % DC_MAXK;
            v[u] = 0.0f;
            if (k < K && t0 + p < M) {
                const int iy = py[buf][p] + kdy[k], ix = px[buf][p] + kdx[k];
                if (iy >= 0 && iy < cv.H && ix >= 0 && ix < cv.W)
                    v[u] = __ldg(x + ((static_cast<size_t>(pb[buf][p]) + iy) * cv.W + ix) * cv.C + kci[k]);
            }
        }
    };
    const int stride = gridDim.x * DC_PIX;
    float v[PER];
    int p0 = blockIdx.x * DC_PIX, buf = 0;
    if (p0 < M) {
        geom(0, p0);
        __syncthreads();  // also publishes kdy / kdx / kci
        gather(0, p0, v);
    }
    for (; p0 < M; p0 += stride, buf ^= 1) {
        __syncthreads();  // the previous tile's inputs and the other geometry buffer are no longer read
#pragma unroll
        for (int u = 0; u < PER; u++) {
            const int i = u * 256 + threadIdx.x;
            xs[i / DC_MAXK][i % DC_MAXK] = v[u];
        }
        const int pn = p0 + stride;
        if (pn < M) geom(buf ^ 1, pn);
        __syncthreads();
        if (pn < M) gather(buf ^ 1, pn, v);
        // four pixels per warp at a time: eight independent fma chains per lane (each still sums k in order, so the
        // same bits as one pixel at a time), the pixels' inputs broadcast from shared memory as float4s
        for (int p = warp * 4; p < DC_PIX; p += 32) {
            if (p0 + p >= M) break;
            float a0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, a1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k4 = 0; k4 < DC_MAXK / 4; k4++) {
                if (4 * k4 >= K) break;
                float4 xv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) xv[i] = *reinterpret_cast<const float4*>(&xs[p + i][4 * k4]);
#pragma unroll
                for (int e = 0; e < 4; e++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float xk = e == 0 ? xv[i].x : (e == 1 ? xv[i].y : (e == 2 ? xv[i].z : xv[i].w));
                        a0[i] = __fmaf_rn(xk, w0[4 * k4 + e], a0[i]);
                        a1[i] = __fmaf_rn(xk, w1[4 * k4 + e], a1[i]);
                    }
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = p0 + p + i;
                if (m >= M) break;
                float* yr = y + static_cast<size_t>(m) * Co + g * cog;
                if (c0 < cog) yr[c0] = epi_act<ACTC>(bias ? __fadd_rn(a0[i], b0) : a0[i], act, alpha);
                if (c1 < cog) yr[c1] = epi_act<ACTC>(bias ? __fadd_rn(a1[i], b1) : a1[i], act, alpha);
            }
        }
    }
}

int launch_conv_direct(const float* x, const float* whi, const float* wlo, int ldw, const float* bias, float* y, int m,
                       int Co, int k, const ConvGeom& cv, int groups, int act, float alpha, cudaStream_t st) {
    const int tiles = (m + DC_PIX - 1) / DC_PIX, cap = sm_count() * 4;  // 4 blocks of 256 threads per SM
    dim3 grid(tiles < cap ? tiles : cap, groups);
    switch (act_class(act)) {
    case -1: k_conv_direct<-1><<<grid, 256, 0, st>>>(x, whi, wlo, ldw, bias, y, m, Co, k, cv, act, alpha); break;
    case 0: k_conv_direct<0><<<grid, 256, 0, st>>>(x, whi, wlo, ldw, bias, y, m, Co, k, cv, act, alpha); break;
    case 1: k_conv_direct<1><<<grid, 256, 0, st>>>(x, whi, wlo, ldw, bias, y, m, Co, k, cv, act, alpha); break;
    default: k_conv_direct<ACT_GENERIC><<<grid, 256, 0, st>>>(x, whi, wlo, ldw, bias, y, m, Co, k, cv, act, alpha); break;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------- weight preparation
// q_kn: k x n int8 row-major (in x out, the file's order) -> wq: n x ldw (K-major), zero padded
__global__ void k_prep_i8(const int8_t* __restrict__ q, int k, int n, int8_t* __restrict__ wq, int ldw) {
    __shared__ int8_t tile[32][33];
    const int kb = blockIdx.x * 32, nb = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int kk = kb + i, nn = nb + threadIdx.x;
        tile[i][threadIdx.x] = (kk < k && nn < n) ? q[static_cast<size_t>(kk) * n + nn] : 0;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int nn = nb + i, kk = kb + threadIdx.x;
        if (nn < n && kk < ldw) wq[static_cast<size_t>(nn) * ldw + kk] = tile[threadIdx.x][i];
    }
}

// w_kn: k x n fp32 -> hi, lo: n x ldw (K-major) tf32 split planes, zero padded
__global__ void k_prep_f32(const float* __restrict__ w, int k, int n, float* __restrict__ hi, float* __restrict__ lo,
                           int ldw) {
    __shared__ float tile[32][33];
    const int kb = blockIdx.x * 32, nb = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int kk = kb + i, nn = nb + threadIdx.x;
        tile[i][threadIdx.x] = (kk < k && nn < n) ? w[static_cast<size_t>(kk) * n + nn] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int nn = nb + i, kk = kb + threadIdx.x;
        if (nn < n && kk < ldw) {
            float h, l;
            tf32_split(tile[threadIdx.x][i], h, l);
            hi[static_cast<size_t>(nn) * ldw + kk] = h;
            lo[static_cast<size_t>(nn) * ldw + kk] = l;
        }
    }
}

template <int BN>
int dispatch_i8(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale, const float* bias,
                float* y, int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st) {
    if (BN == 256) {  // 256 x 256 tiles on CTA pairs
        switch (act_class(act)) {
        case -1: return launch_i8_pair<false, -1>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
        case 0: return launch_i8_pair<false, 0>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
        case 1: return launch_i8_pair<false, 1>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
        default:
            return launch_i8_pair<false, ACT_GENERIC>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha,
                                                      status, st);
        }
    }
    switch (act_class(act)) {
    case -1: return launch_i8<BN, false, -1>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
    case 0: return launch_i8<BN, false, 0>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
    case 1: return launch_i8<BN, false, 1>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
    default:
        return launch_i8<BN, false, ACT_GENERIC>(xq, ldq, sx, wq, ldw, scale, bias, y, nullptr, ldy, m, n, k, act, alpha, status, st);
    }
}

#define KX_F32_ARGS x, ldx, whi, wlo, ldw, wrows, bias, y, ldy, m, n, k, act, alpha, status, st, cv, groups, res, ldr
template <int BN, bool CONV, bool DRAIN, bool PAIR>
int launch_f32_act(const float* x, int ldx, const float* whi, const float* wlo, int ldw, int wrows, const float* bias,
                   float* y, int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st,
                   const ConvGeom& cv, int groups, const float* res, int ldr) {
    if constexpr (PAIR) {
        switch (act_class(act)) {
        case -1: return launch_f32_pair<BN, CONV, -1, DRAIN>(KX_F32_ARGS);
        case 0: return launch_f32_pair<BN, CONV, 0, DRAIN>(KX_F32_ARGS);
        case 1: return launch_f32_pair<BN, CONV, 1, DRAIN>(KX_F32_ARGS);
        default: return launch_f32_pair<BN, CONV, ACT_GENERIC, DRAIN>(KX_F32_ARGS);
        }
    } else {
        switch (act_class(act)) {
        case -1: return launch_f32<BN, CONV, -1, DRAIN>(KX_F32_ARGS);
        case 0: return launch_f32<BN, CONV, 0, DRAIN>(KX_F32_ARGS);
        case 1: return launch_f32<BN, CONV, 1, DRAIN>(KX_F32_ARGS);
        default: return launch_f32<BN, CONV, ACT_GENERIC, DRAIN>(KX_F32_ARGS);
        }
    }
}

// Tile choice: more than 128 rows -> CTA pairs (256-row tiles); reductions longer than DRAIN_MIN_K -> 128-column
// tiles with chunk draining; otherwise BN (128 for at most 128 output columns, else 256).
template <int BN, bool CONV>
int dispatch_f32(const float* x, int ldx, const float* whi, const float* wlo, int ldw, int wrows, const float* bias, float* y,
                 int ldy, int m, int n, int k, int act, float alpha, int* status, cudaStream_t st, const ConvGeom& cv,
                 int groups, const float* res = nullptr, int ldr = 0) {
    const bool pair = m > BM;
    if (!CONV && BN == 256 && pair && k <= PP_MAX_K) {  // persistent CTA pairs when there is more than one wave
        int r;
        switch (act_class(act)) {
        case -1: r = launch_f32_pp<-1>(x, ldx, whi, wlo, ldw, wrows, bias, y, ldy, m, n, k, act, alpha, status, st, res, ldr); break;
        case 0: r = launch_f32_pp<0>(x, ldx, whi, wlo, ldw, wrows, bias, y, ldy, m, n, k, act, alpha, status, st, res, ldr); break;
        case 1: r = launch_f32_pp<1>(x, ldx, whi, wlo, ldw, wrows, bias, y, ldy, m, n, k, act, alpha, status, st, res, ldr); break;
        default: r = launch_f32_pp<ACT_GENERIC>(x, ldx, whi, wlo, ldw, wrows, bias, y, ldy, m, n, k, act, alpha, status, st, res, ldr);
        }
        if (r <= 0) return r;
    }
    if (k > DRAIN_MIN_K)
        return pair ? launch_f32_act<128, CONV, true, true>(KX_F32_ARGS) : launch_f32_act<128, CONV, true, false>(KX_F32_ARGS);
    return pair ? launch_f32_act<BN, CONV, false, true>(KX_F32_ARGS) : launch_f32_act<BN, CONV, false, false>(KX_F32_ARGS);
}
#undef KX_F32_ARGS

// One warp waits, with the library's bounded wait (mbar_wait_for), on an mbarrier of arrival count 1. With
// arrive = 1 lane 0 arrives first and the wait completes; with arrive = 0 nothing ever arrives, so the wait gives
// up after limit_ns and records KX_STATUS_TIMEOUT in *status. Nothing asynchronous (TMA, MMA) is in flight.
// waited[0] receives the nanoseconds lane 0 spent in the wait.
__global__ void k_probe_wait(int arrive, uint64_t limit_ns, int* status, unsigned long long* waited) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        kx::mbar_init(&bar, 1);
        abort_flag = 0;
        kx::fence_mbar_init();
    }
    __syncwarp();
    if (arrive && threadIdx.x == 0) kx::mbar_arrive(&bar);
    __syncwarp();
    const uint64_t t0 = kx::globaltimer();
    kx::mbar_wait_for(&bar, 0, &abort_flag, status, limit_ns);
    if (threadIdx.x == 0) waited[0] = kx::globaltimer() - t0;
}

}  // namespace

extern "C" {

int kx_probe_bounded_wait(int arrive, unsigned long long limit_ns, int* status, unsigned long long* waited_ns, void* stream) {
    if (status == nullptr || waited_ns == nullptr || limit_ns > 2000000000ull) return -1;
    k_probe_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(arrive, limit_ns, status, waited_ns);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kx_gemm_i8(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale,
               const float* bias, float* y, int ldy, int m, int n, int k, int act, float alpha, int* status,
               void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldq || k > ldw || (ldq & 15) || (ldw & 15)) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n <= 128) return dispatch_i8<128>(xq, ldq, sx, wq, ldw, scale, bias, y, ldy, m, n, k, act, alpha, status, st);
    return dispatch_i8<256>(xq, ldq, sx, wq, ldw, scale, bias, y, ldy, m, n, k, act, alpha, status, st);
}

int kx_i8_chain(int n_layers, int m, const int8_t* const* a, const int* lda, const float* const* sx, const int8_t* const* wq,
                const int* ldw, const float* const* scale, const float* const* bias, const int* k, const int* n, const int* act,
                const float* alpha, float* const* sx_out, uint32_t* ctl, float* y, int* status, void* stream) {
    if (m <= 0) return 0;
    if (n_layers < 2 || n_layers > KX_I8C_MAX || ctl == nullptr || y == nullptr) return -1;
    using C = I8PairCfg<6>;
    const int rgs = (m + BM - 1) / BM;
    I8Chain ch{};
    ch.n_layers = n_layers;
    CUtensorMap ta[KX_I8C_MAX], tb[KX_I8C_MAX];
    std::memset(ta, 0, sizeof ta);
    std::memset(tb, 0, sizeof tb);
    const int m_tiles = (m + 2 * BM - 1) / (2 * BM);
    int tiles = 0, max_nt = 1;
    for (int l = 0; l < n_layers; l++) {
        if (k[l] <= 0 || n[l] <= 128 || k[l] > lda[l] || k[l] > ldw[l] || (lda[l] & 15) || (ldw[l] & 15) ||
            (l > 0 && k[l] != n[l - 1]) || (reinterpret_cast<uintptr_t>(a[l]) & 15))
            return -1;
        if (make_map_2d(&ta[l], CU_TENSOR_MAP_DATA_TYPE_UINT8, a[l], static_cast<uint64_t>(lda[l]), static_cast<uint64_t>(m),
                        static_cast<uint64_t>(lda[l]), C::BK, BM) != 0 ||
            make_map_2d(&tb[l], CU_TENSOR_MAP_DATA_TYPE_UINT8, wq[l], static_cast<uint64_t>(ldw[l]), static_cast<uint64_t>(n[l]),
                        static_cast<uint64_t>(ldw[l]), C::BK, C::BN / 2) != 0)
            return -1;
        I8CLayer& L = ch.L[l];
        L.sx = sx[l];
        L.scale = scale[l];
        L.bias = bias[l];
        L.n = n[l];
        L.k = k[l];
        L.act = act[l];
        L.alpha = alpha[l];
        L.n_tiles_n = (n[l] + C::BN - 1) / C::BN;
        L.tile0 = tiles;
        tiles += m_tiles * L.n_tiles_n;
        if (l + 1 < n_layers) {  // the next layer's int8 rows, row scales and this layer's control words
            uint32_t* w = ctl + static_cast<size_t>(l) * (m + 2 * rgs);
            L.qo = QOut{const_cast<int8_t*>(a[l + 1]), sx_out[l], w, w + m, nullptr, lda[l + 1], 0};
            L.ready = w + m + rgs;
            if (lda[l + 1] < n[l]) return -1;
            if (L.n_tiles_n > max_nt) max_nt = L.n_tiles_n;  // clusters: at least every hidden layer's tiles per row group
        } else {
            L.y = y;
        }
    }
    ch.total_tiles = tiles;
    const int ah = act_class(act[0]), al = act_class(act[n_layers - 1]);
    for (int l = 1; l + 1 < n_layers; l++)
        if (act_class(act[l]) != ah) return -1;  // hidden layers share one activation class (compiled in)
    auto pick = [&](auto kern) -> int {
        if (set_smem_once(reinterpret_cast<const void*>(kern), C::SMEM) != 0) return -1;
        int clusters = max_pair_clusters(reinterpret_cast<const void*>(kern), C::THREADS, C::SMEM);
        if (clusters <= 0) clusters = sm_count() / 2;
        if (max_nt > clusters) return -1;
        if (clusters > tiles) clusters = tiles;
        return kx::launch_pdl(kern, dim3(2 * clusters), dim3(C::THREADS), C::SMEM, static_cast<cudaStream_t>(stream), ta[0],
                              ta[1], ta[2], ta[3], tb[0], tb[1], tb[2], tb[3], ch, m, status);
    };
    if (ah == 1 && al == -1) return pick(k_i8_chain<6, 1, -1>);
    if (ah == 1 && al == 1) return pick(k_i8_chain<6, 1, 1>);
    if (ah == 0 && al == -1) return pick(k_i8_chain<6, 0, -1>);
    if (ah == 0 && al == 0) return pick(k_i8_chain<6, 0, 0>);
    if (ah == -1 && al == -1) return pick(k_i8_chain<6, -1, -1>);
    return pick(k_i8_chain<6, ACT_GENERIC, ACT_GENERIC>);
}

int kx_gemm_i8_q(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale, const float* bias,
                 int m, int n, int k, int act, float alpha, int8_t* q_out, int ldq_out, float* sx_out, uint32_t* ctl,
                 uint32_t* zero_next, int zero_words, int* status, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldq || k > ldw || (ldq & 15) || (ldw & 15) || n <= 128 || ldq_out < n || (ldq_out & 15) ||
        q_out == nullptr || sx_out == nullptr || ctl == nullptr || (reinterpret_cast<uintptr_t>(q_out) & 15) ||
        (zero_words > 0 && zero_next == nullptr))
        return -1;
    const QOut qo{q_out, sx_out, ctl, ctl + m, zero_next, ldq_out, zero_words};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (act_class(act)) {
    case -1: return launch_i8_pair<false, -1, true>(xq, ldq, sx, wq, ldw, scale, bias, nullptr, nullptr, n, m, n, k, act, alpha, status, st, qo);
    case 0: return launch_i8_pair<false, 0, true>(xq, ldq, sx, wq, ldw, scale, bias, nullptr, nullptr, n, m, n, k, act, alpha, status, st, qo);
    case 1: return launch_i8_pair<false, 1, true>(xq, ldq, sx, wq, ldw, scale, bias, nullptr, nullptr, n, m, n, k, act, alpha, status, st, qo);
    default:
        return launch_i8_pair<false, ACT_GENERIC, true>(xq, ldq, sx, wq, ldw, scale, bias, nullptr, nullptr, n, m, n, k, act, alpha,
                                                        status, st, qo);
    }
}

int kx_linear_i8(const float* x, int ldx, int rows, int k, const int8_t* wq, int ldw, const float* scale, const float* bias,
                 float* y, int ldy, int n, int act, float alpha, int8_t* xq_scratch, float* sx_scratch, int* status,
                 void* stream) {
    if (rows <= 0 || n <= 0) return 0;
    if (xq_scratch == nullptr || sx_scratch == nullptr) return -1;
    const int ldq = (k + 15) / 16 * 16;
    if (kx_quant_rows(x, ldx, rows, k, xq_scratch, ldq, sx_scratch, stream) != 0) return -1;
    return kx_gemm_i8(xq_scratch, ldq, sx_scratch, wq, ldw, scale, bias, y, ldy, rows, n, k, act, alpha, status, stream);
}

int kx_i8_split_blocks(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 1;
    const int bn = n <= 128 ? 128 : 256, nk = (k + 127) / 128;
    const int tiles = ((m + BM - 1) / BM) * ((n + bn - 1) / bn);
    int ranges = sm_count() / tiles;
    if (ranges < 1) ranges = 1;
    if (ranges > nk) ranges = nk;
    if (ranges > KX_I8_SPLIT_MAX) ranges = KX_I8_SPLIT_MAX;
    return (nk + ranges - 1) / ranges;
}

int kx_gemm_i8_split_acc(const int8_t* xq, int ldq, const int8_t* wq, int ldw, int m, int n, int k, int kbs, int32_t* part,
                         int* status, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldq || k > ldw || (ldq & 15) || (ldw & 15) || kbs <= 0 || part == nullptr) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n <= 128)
        return launch_i8<128, true, -1>(xq, ldq, nullptr, wq, ldw, nullptr, nullptr, nullptr, part, n, m, n, k, -1, 0.0f, status,
                                        st, kbs);
    return launch_i8<256, true, -1>(xq, ldq, nullptr, wq, ldw, nullptr, nullptr, nullptr, part, n, m, n, k, -1, 0.0f, status,
                                    st, kbs);
}

int kx_i8_rows(const int32_t* part, int planes, int m, int n, const float* sx, const float* scale, const float* bias, int act,
               float alpha, float* y, int ldy, int8_t* q, int ldq, float* sx_out, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (planes < 1 || part == nullptr || sx == nullptr || scale == nullptr || n > I8R_MAXN) return -1;
    if (q == nullptr ? (y == nullptr || ldy < n) : (sx_out == nullptr || ldq < n || ldq > I8R_MAXN || (ldq & 15)))
        return -1;  // (the blocks' column pairs cover I8R_MAXN columns: every byte up to ldq is written)
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(m));
    int rc = -1;
#define KX_I8R_LAUNCH(A, Q)                                                                                     \
    rc = kx::launch_pdl(k_i8_rows<A, Q>, grid, dim3(I8R_THREADS), 0, st, part, planes, m, n, sx, scale, bias, act, alpha, y, \
                        ldy, q, ldq, sx_out)
    if (q != nullptr) {
        switch (act_class(act)) {
        case -1: KX_I8R_LAUNCH(-1, true); break;
        case 0: KX_I8R_LAUNCH(0, true); break;
        case 1: KX_I8R_LAUNCH(1, true); break;
        default: KX_I8R_LAUNCH(ACT_GENERIC, true);
        }
    } else {
        switch (act_class(act)) {
        case -1: KX_I8R_LAUNCH(-1, false); break;
        case 0: KX_I8R_LAUNCH(0, false); break;
        case 1: KX_I8R_LAUNCH(1, false); break;
        default: KX_I8R_LAUNCH(ACT_GENERIC, false);
        }
    }
#undef KX_I8R_LAUNCH
    return rc;
}

int kx_gemm_i8_acc(const int8_t* xq, int ldq, const int8_t* wq, int ldw, int32_t* acc, int ldacc, int m, int n, int k,
                   int* status, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldq || k > ldw || (ldq & 15) || (ldw & 15)) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n <= 128)
        return launch_i8<128, true, -1>(xq, ldq, nullptr, wq, ldw, nullptr, nullptr, nullptr, acc, ldacc, m, n, k, -1, 0.0f, status, st);
    return launch_i8_pair<true, -1>(xq, ldq, nullptr, wq, ldw, nullptr, nullptr, nullptr, acc, ldacc, m, n, k, -1, 0.0f, status, st);
}

int kx_gemm_f32(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y,
                int ldy, int m, int n, int k, int act, float alpha, int* status, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldx || k > ldw || (ldw & 3)) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const ConvGeom cv{};
    if (n <= 128) return dispatch_f32<128, false>(x, ldx, w_hi, w_lo, ldw, n, bias, y, ldy, m, n, k, act, alpha, status, st, cv, 1);
    return dispatch_f32<256, false>(x, ldx, w_hi, w_lo, ldw, n, bias, y, ldy, m, n, k, act, alpha, status, st, cv, 1);
}

int kx_gemm_f32_splits(int m, int n, int k) {
    if (m <= 0 || m > BM || n <= 0 || k < 2048) return 1;
    const int bn = k > DRAIN_MIN_K || n <= 128 ? 128 : 256;
    const int tiles = (n + bn - 1) / bn;
    int s = sm_count() / tiles;
    if (s > KX_SPLITK_MAX) s = KX_SPLITK_MAX;
    if (s > k / 1024) s = k / 1024;
    return s < 2 ? 1 : s;
}

int kx_gemm_f32_split(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y,
                      int ldy, int m, int n, int k, int act, float alpha, int splits, float* part, int* status, void* stream) {
    if (splits == 1) return kx_gemm_f32(x, ldx, w_hi, w_lo, ldw, bias, y, ldy, m, n, k, act, alpha, status, stream);
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldx || k > ldw || (ldw & 3) || m > BM || splits < 1 || splits > KX_SPLITK_MAX || part == nullptr)
        return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const ConvGeom cv{};
    const int ksl = ((k + splits - 1) / splits + 255) / 256 * 256;  // whole drain chunks per range
    const int used = (k + ksl - 1) / ksl;                           // ranges that hold any K
    int r;
    if (k > DRAIN_MIN_K)
        r = launch_f32<128, false, -1, true>(x, ldx, w_hi, w_lo, ldw, n, nullptr, part, n, m, n, k, -1, 0.0f, status, st, cv, 1,
                                             nullptr, 0, used, ksl);
    else if (n > 128)
        r = launch_f32<256, false, -1, false>(x, ldx, w_hi, w_lo, ldw, n, nullptr, part, n, m, n, k, -1, 0.0f, status, st, cv, 1,
                                              nullptr, 0, used, ksl);
    else
        r = launch_f32<128, false, -1, false>(x, ldx, w_hi, w_lo, ldw, n, nullptr, part, n, m, n, k, -1, 0.0f, status, st, cv, 1,
                                              nullptr, 0, used, ksl);
    if (r != 0) return r;
    return kx_add_planes(part, used, m, n, bias, act, alpha, y, ldy, stream);
}

int kx_gemm_f32_res(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y,
                    int ldy, int m, int n, int k, int act, float alpha, const float* res, int ldr, int* status, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (k <= 0 || k > ldx || k > ldw || (ldw & 3) || res == nullptr || ldr < n) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const ConvGeom cv{};
    if (n <= 128)
        return dispatch_f32<128, false>(x, ldx, w_hi, w_lo, ldw, n, bias, y, ldy, m, n, k, act, alpha, status, st, cv, 1, res, ldr);
    return dispatch_f32<256, false>(x, ldx, w_hi, w_lo, ldw, n, bias, y, ldy, m, n, k, act, alpha, status, st, cv, 1, res, ldr);
}

int kx_conv_f32(const float* x, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y, int B, int H,
                int W, int C, int Co, int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl,
                int groups, int act, float alpha, int* status, void* stream) {
    if (B <= 0) return 0;
    if (groups < 1 || C % groups || Co % groups || (ldw & 3)) return -1;
    const long m = static_cast<long>(B) * Ho * Wo;
    const int cg = C / groups, cog = Co / groups, k = kh * kw * cg;
    if (m > INT32_MAX || k > ldw) return -1;
    const ConvGeom cv{H, W, C, Ho, Wo, kh, kw, sh, sw, dh, dw, pt, pl, cg, cog};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (k <= DC_MAXK && cog <= DC_MAXCO && groups <= 65535)
        return launch_conv_direct(x, w_hi, w_lo, ldw, bias, y, static_cast<int>(m), Co, k, cv, groups, act, alpha, st);
    if (cog <= 128 && m > BM && k <= DRAIN_MIN_K && groups <= 65535) {  // channel-major tiles
        const int mi = static_cast<int>(m);
        switch (act_class(act)) {
        case -1: return launch_conv_cm<-1>(x, w_hi, w_lo, ldw, Co, bias, y, Co, mi, k, act, alpha, status, st, cv, groups);
        case 0: return launch_conv_cm<0>(x, w_hi, w_lo, ldw, Co, bias, y, Co, mi, k, act, alpha, status, st, cv, groups);
        case 1: return launch_conv_cm<1>(x, w_hi, w_lo, ldw, Co, bias, y, Co, mi, k, act, alpha, status, st, cv, groups);
        default: return launch_conv_cm<ACT_GENERIC>(x, w_hi, w_lo, ldw, Co, bias, y, Co, mi, k, act, alpha, status, st, cv, groups);
        }
    }
    if (cog <= 128)
        return dispatch_f32<128, true>(x, C, w_hi, w_lo, ldw, Co, bias, y, Co, static_cast<int>(m), cog, k, act, alpha, status,
                                       st, cv, groups);
    return dispatch_f32<256, true>(x, C, w_hi, w_lo, ldw, Co, bias, y, Co, static_cast<int>(m), cog, k, act, alpha, status, st,
                                   cv, groups);
}

int kx_conv_f32_ws(const float* x, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y, int B, int H,
                   int W, int C, int Co, int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl,
                   int groups, int act, float alpha, float* ws, size_t ws_floats, int* status, void* stream) {
    if (B <= 0) return 0;
    if (groups < 1 || C % groups || Co % groups || (ldw & 3)) return -1;
    const long m = static_cast<long>(B) * Ho * Wo, n = static_cast<long>(B) * H * W * C;
    const int cg = C / groups, cog = Co / groups, k = kh * kw * cg;
    int rows = 0, imgs = 0;
    const bool tma = sh == 1 && sw == 1 && cg % 32 == 0 && cog <= 128 && m > BM && m <= INT32_MAX && k <= DRAIN_MIN_K &&
                     k <= ldw && groups <= 65535 && cmt_tiling(Ho, Wo, rows, imgs) == 0 && ws != nullptr &&
                     ws_floats >= static_cast<size_t>(2 * n) && (reinterpret_cast<uintptr_t>(ws) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (!tma)
        return kx_conv_f32(x, w_hi, w_lo, ldw, bias, y, B, H, W, C, Co, Ho, Wo, kh, kw, sh, sw, dh, dw, pt, pl, groups, act,
                           alpha, status, stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* xh = ws;
    float* xl = ws + n;  // n is a multiple of 4: 16-byte aligned
    const long blocks = (n / 4 + 255) / 256;
    k_split_planes<<<static_cast<unsigned>(blocks < 4L * sm_count() ? (blocks > 0 ? blocks : 1) : 4L * sm_count()), 256, 0, st>>>(
        x, xh, xl, n);
    if (cudaGetLastError() != cudaSuccess) return -1;
    CUtensorMap mh, ml;
    if (make_map_nhwc(&mh, xh, B, H, W, C, static_cast<uint32_t>(Wo), static_cast<uint32_t>(rows), static_cast<uint32_t>(imgs)) != 0 ||
        make_map_nhwc(&ml, xl, B, H, W, C, static_cast<uint32_t>(Wo), static_cast<uint32_t>(rows), static_cast<uint32_t>(imgs)) != 0)
        return -1;
    const CmtGeom gm{cg, kw, dh, dw, pt, pl, Ho, Wo, rows, imgs};
    const int mi = static_cast<int>(m);
    switch (act_class(act)) {
    case -1: return launch_conv_cmt<-1>(mh, ml, w_hi, w_lo, ldw, Co, bias, y, Co, cog, mi, k, act, alpha, status, st, gm, groups);
    case 0: return launch_conv_cmt<0>(mh, ml, w_hi, w_lo, ldw, Co, bias, y, Co, cog, mi, k, act, alpha, status, st, gm, groups);
    case 1: return launch_conv_cmt<1>(mh, ml, w_hi, w_lo, ldw, Co, bias, y, Co, cog, mi, k, act, alpha, status, st, gm, groups);
    default:
        return launch_conv_cmt<ACT_GENERIC>(mh, ml, w_hi, w_lo, ldw, Co, bias, y, Co, cog, mi, k, act, alpha, status, st, gm,
                                            groups);
    }
}

int kx_prep_i8_weight(const int8_t* q_kn, int k, int n, int8_t* wq, int ldw, void* stream) {
    if (k <= 0 || n <= 0 || ldw < k) return -1;
    dim3 grid((ldw + 31) / 32, (n + 31) / 32), block(32, 8);
    k_prep_i8<<<grid, block, 0, static_cast<cudaStream_t>(stream)>>>(q_kn, k, n, wq, ldw);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kx_prep_f32_weight(const float* w_kn, int k, int n, float* w_hi, float* w_lo, int ldw, void* stream) {
    if (k <= 0 || n <= 0 || ldw < k) return -1;
    dim3 grid((ldw + 31) / 32, (n + 31) / 32), block(32, 8);
    k_prep_f32<<<grid, block, 0, static_cast<cudaStream_t>(stream)>>>(w_kn, k, n, w_hi, w_lo, ldw);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
