/* KERNIX-B200 kernel-level C ABI: the sm_100a CUDA kernels behind the model runtime.
 *
 * Plain device pointers, sizes and a cudaStream_t passed as void*; no CUDA or torch types. All matrices
 * are row-major with an explicit leading dimension (elements). Every function returns 0 when the launch
 * was accepted and -1 on bad arguments or a launch error. Kernels whose waits are bounded write
 * KX_STATUS_TIMEOUT into *status (device memory, may be NULL) instead of hanging.
 * Each entry names the reference computation it replaces (KERNIX reference file:line).
 */
#ifndef KX_KERNELS_H
#define KX_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#include "kernix.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KX_STATUS_OK 0
#define KX_STATUS_TIMEOUT 1

/* ---- int8 path (include/kernix_model.h:99-182 kernix_qmatmul) ---- */

/* Per-row dynamic int8 quantisation (kernix_qmatmul :110-142): m = max|x| over the row (NaN wins),
 * sx = m > 0 ? m / 127 : 1, xq = clamp(rint(x * (1/sx)), -127, 127); rows whose m is NaN/inf get sx = NaN
 * (their GEMM output becomes NaN, as the reference's NaN rows). xq columns k..ldq-1 are zeroed. */
KERNIX_API int kx_quant_rows(const float* x, int ldx, int rows, int k, int8_t* xq, int ldq, float* sx, void* stream);

/* kx_quant_rows that also clears zero[0 .. zero_words) once the kernel before it has completed: the row maxima
 * and counters of the kx_gemm_i8_q launch that follows (an internal step of the model runtime). */
KERNIX_API int kx_quant_rows_z(const float* x, int ldx, int rows, int k, int8_t* xq, int ldq, float* sx, uint32_t* zero,
                               int zero_words, void* stream);

/* y = act(((float)acc * sx[row]) * scale[col] + bias[col]) with acc = sum_t xq[row][t] * wq[col][t] in int32
 * on tcgen05 kind::i8 (kernix_qmatmul :143-177 and the step's activation :1854-1856). wq: n x ldw int8,
 * K-major (see kx_prep_i8_weight). ldq, ldw multiples of 16. bias may be NULL (adds 0). */
KERNIX_API int kx_gemm_i8(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale,
               const float* bias, float* y, int ldy, int m, int n, int k, int act, float alpha, int* status, void* stream);

/* A hidden int8 layer whose output feeds only the next int8 layer (kernix_qmatmul :99-182 twice, :1854-1856):
 * the int8 GEMM of kx_gemm_i8 whose epilogue quantises its own output rows for the next layer, as kx_quant_rows
 * would from y, and writes q_out (m x ldq_out int8; ldq_out >= n, a multiple of 16; columns n .. ldq_out-1 zero;
 * 16-byte aligned) and sx_out (m floats) instead of y: bit for bit the kx_quant_rows result of y. ctl: m + ceil(m/128)
 * words of device memory that must be zero at launch (row maxima and row-group counters); the launch clears
 * zero_next[0 .. zero_words) for the next one. n > 128 (CTA-pair tiles) and at most as many 256-column tiles as
 * CTA pairs resident at once, else -1. */
KERNIX_API int kx_gemm_i8_q(const int8_t* xq, int ldq, const float* sx, const int8_t* wq, int ldw, const float* scale,
                            const float* bias, int m, int n, int k, int act, float alpha, int8_t* q_out, int ldq_out,
                            float* sx_out, uint32_t* ctl, uint32_t* zero_next, int zero_words, int* status, void* stream);

/* A chain of n_layers (2..4) int8 LINEAR steps (kernix_qmatmul :99-182 plus the activation :1854-1856, step after
 * step, each hidden output quantised as the next step's input as kx_quant_rows would) in ONE persistent launch of the
 * CTA-pair int8 GEMM, every layer's tiles in one walk: a tile of layer l > 0 starts once the rows it reads are
 * quantised. a[0] / sx[0]: the chain input quantised (kx_quant_rows_z); a[l] / sx[l] = sx_out[l-1] for l > 0: the
 * buffers layer l-1 writes (m x lda[l] int8, 16-byte aligned; m floats). y: m x n[last] fp32. ctl: (n_layers - 1) x
 * (m + 2 * ceil(m / 128)) words, zero at launch (clear them with the quantiser before). Every n[l] > 128, at most 64
 * tiles of 256 columns per layer, hidden layers of one activation class (ReLU, GELU, none or another); else -1.
 * Bit for bit the results of running the steps one by one. */
KERNIX_API int kx_i8_chain(int n_layers, int m, const int8_t* const* a, const int* lda, const float* const* sx,
                           const int8_t* const* wq, const int* ldw, const float* const* scale, const float* const* bias,
                           const int* k, const int* n, const int* act, const float* alpha, float* const* sx_out,
                           uint32_t* ctl, float* y, int* status, void* stream);

/* One int8 LINEAR step from fp32 activations, the whole of kernix_qmatmul plus the step's activation
 * (include/kernix_model.h:99-182, :1854-1856): quantise x's rows into xq_scratch (rows x ldq int8, ldq =
 * k rounded up to 16) and sx_scratch (rows floats), then y = act(((float)acc * sx) * scale + bias) with the
 * int8 tcgen05 GEMM. The two scratch buffers are device memory supplied by the caller. */
KERNIX_API int kx_linear_i8(const float* x, int ldx, int rows, int k, const int8_t* wq, int ldw, const float* scale,
                            const float* bias, float* y, int ldy, int n, int act, float alpha, int8_t* xq_scratch,
                            float* sx_scratch, int* status, void* stream);

/* kx_linear_i8 for callers that cannot allocate device memory (latency-critical code that cannot take cudaMalloc's
 * device-wide synchronisation, or hosts whose allocator forbids extra device allocations). No counterpart in the
 * reference. Same arguments and result as kx_linear_i8 minus the two scratch buffers: they come from one
 * KX_NOALLOC_SCRATCH_BYTES array compiled into the library (held on every GPU that loads it until exit), so
 * rows * (k rounded up to 16) + 4 * rows (+ alignment) must fit, else it returns -1 with a message. The first call on
 * a device (per CUDA context) loads the module that holds the array, which reserves its 16 MiB there, and looks
 * the array up (cudaGetSymbolAddress): make that call in initialisation code, before any stream capture. Later
 * calls in the same context allocate nothing; after cudaDeviceReset the next call looks the array up again.
 * Calls share the array: calls whose work overlaps on the GPU race, so order them on one stream. */
#define KX_NOALLOC_SCRATCH_BYTES (16 << 20)
KERNIX_API int kx_linear_i8_noalloc(const float* x, int ldx, int rows, int k, const int8_t* wq, int ldw, const float* scale,
                                    const float* bias, float* y, int ldy, int n, int act, float alpha, int* status,
                                    void* stream);

/* Failure-detection check of the bounded waits every tcgen05 kernel here uses (the counterpart of the reference's
 * command-buffer error handling, src/kernix_metal.m:259-263, which turns a failed GPU command into -1): one warp
 * waits on an mbarrier with the library's wait helper and a limit of limit_ns (at most 2 s). arrive = 1: the
 * barrier completes and *status is left as it was; arrive = 0: nothing arrives, the wait gives up after limit_ns
 * and writes KX_STATUS_TIMEOUT (1) to *status, and the launch ends normally. *waited_ns: time spent waiting.
 * Device pointers; returns -1 on bad arguments or a launch error. */
KERNIX_API int kx_probe_bounded_wait(int arrive, unsigned long long limit_ns, int* status, unsigned long long* waited_ns,
                                     void* stream);

/* Small-batch int8 layers with the reduction split over the SMs. kx_i8_split_blocks: K blocks (of 128) per range for an
 * m x n x k layer so that its output tiles times its ranges about fill the SMs (at most KX_I8_SPLIT_MAX ranges).
 * kx_gemm_i8_split_acc: the int32 sums of each K range into plane z of part (ceil(ceil(k / 128) / kbs) planes of
 * m x n int32). kx_i8_rows: one row per block adds the planes (exactly), then ((float)acc * sx) * scale + bias and the
 * activation as the int8 GEMM epilogue does, and stores the fp32 row (q == NULL) or quantises it for the next int8
 * layer exactly as the quantised-output epilogue does (q: m x ldq int8, columns n .. ldq - 1 written 0; sx_out: row
 * scales). n, ldq <= 8192. Bit for bit the results of kx_gemm_i8 / kx_gemm_i8_q (the per-step kernels the
 * reference's kernix_qmatmul :99-182 maps to). */
#define KX_I8_SPLIT_MAX 64
KERNIX_API int kx_i8_split_blocks(int m, int n, int k);
KERNIX_API int kx_gemm_i8_split_acc(const int8_t* xq, int ldq, const int8_t* wq, int ldw, int m, int n, int k, int kbs,
                                   int32_t* part, int* status, void* stream);
KERNIX_API int kx_i8_rows(const int32_t* part, int planes, int m, int n, const float* sx, const float* scale, const float* bias,
                          int act, float alpha, float* y, int ldy, int8_t* q, int ldq, float* sx_out, void* stream);

/* int32 accumulators only (acc[row][col], leading dimension ldacc): exposes the integer result for tests. */
KERNIX_API int kx_gemm_i8_acc(const int8_t* xq, int ldq, const int8_t* wq, int ldw, int32_t* acc, int ldacc, int m, int n, int k,
                   int* status, void* stream);

/* Load-time repack of an I8_COL weight block (the file's k x n, in x out) into n x ldw K-major, zero padded
 * (replaces kernix_qweight_pack :62-81, whose layout served NEON sdot). */
KERNIX_API int kx_prep_i8_weight(const int8_t* q_kn, int k, int n, int8_t* wq, int ldw, void* stream);

/* ---- fp32 dense path (kernix_dense :544-550 -> kernix_matmul_ep_into include/kernix.h:955-976,
 *      src/kernix_metal.m:161-265 MPS+AMX split with the bias_act epilogue :269-299) ---- */

/* y = act(x . W + bias) in 3xTF32 on tcgen05 kind::tf32, fp32 accumulation in TMEM. W is given as the
 * tf32 split planes w_hi, w_lo (n x ldw, K-major, ldw % 4 == 0; see kx_prep_f32_weight). bias may be NULL. */
KERNIX_API int kx_gemm_f32(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y,
                int ldy, int m, int n, int k, int act, float alpha, int* status, void* stream);

/* y = act(x . W + bias) + res (ldr >= n): a LINEAR step and the elementwise ADD that consumes it in one kernel
 * (kernix_dense :544-550 followed by kernix_binary_run :877-906), each output written once. The add is the ADD
 * step's round-to-nearest fp32 add on the activation's output, so results are bitwise those of the two steps run
 * apart. y may be res (in place); neither may overlap x. */
KERNIX_API int kx_gemm_f32_res(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y,
                    int ldy, int m, int n, int k, int act, float alpha, const float* res, int ldr, int* status, void* stream);

/* kx_gemm_f32 for at most 128 rows with the reduction split into `splits` (<= KX_SPLITK_MAX) ranges of K (multiples
 * of 256) run by separate CTAs -- for layers whose few output tiles would leave most SMs idle (a column-sharded wide
 * layer at small batch) -- then y = act(P[0] + ... + P[splits-1] + bias) added in range order (kx_add_planes).
 * part: splits x m x n floats of device scratch. splits = 1 is kx_gemm_f32 (any m; part unused). */
#define KX_SPLITK_MAX 4
KERNIX_API int kx_gemm_f32_split(const float* x, int ldx, const float* w_hi, const float* w_lo, int ldw, const float* bias,
                                 float* y, int ldy, int m, int n, int k, int act, float alpha, int splits, float* part,
                                 int* status, void* stream);
/* the split count kx_gemm_f32_split should be given for an m x n x k layer: 1 (no split) unless m <= 128, k >= 2048 and
 * the layer's output tiles fill fewer than half the SMs; at most KX_SPLITK_MAX, ranges of at least 1024 */
KERNIX_API int kx_gemm_f32_splits(int m, int n, int k);
KERNIX_API int kx_add_planes(const float* part, int planes, int m, int n, const float* bias, int act, float alpha, float* y,
                             int ldy, void* stream);

/* Load-time transpose + split of a float weight (k x n, in x out) into n x ldw K-major planes
 * hi = tf32(w), lo = w - hi (exact), zero padded. */
KERNIX_API int kx_prep_f32_weight(const float* w_kn, int k, int n, float* w_hi, float* w_lo, int ldw, void* stream);

/* A chain of small fp32 dense layers y_l = act_l(y_{l-1} . W_l + b_l) (kernix_dense :544-550 step after step, each
 * reading only the previous output) and, if softmax, a row softmax of the last (floats_softmax_into
 * include/kernix.h:652-657; then the last layer has at most 64 outputs), in ONE cooperative launch: each layer a phase
 * of CUDA-core tiles over K ranges, partial sums in scratch, added in a fixed order by the next layer (the last
 * layer's by a final phase, which also runs a narrow last layer per row), a bounded grid barrier after each phase;
 * each layer's K ranges depend on its k and n only, so a row's result does not depend on the batch it is in. For batches whose tensor-core GEMMs are dominated by per-launch costs (rows <=
 * KX_MLP_MAX_ROWS). w[l]: k[l] x n[l] row-major fp32; bias[l] may be NULL; ldx and every n[l] but the last multiples of
 * 4, x and scratch 16-byte aligned; scratch: kx_mlp_chain_scratch_floats(m, k, n, n_layers) floats; bar: two words
 * (arrivals at the current grid barrier, barrier generation), zero before the first launch, kept between launches
 * (reset them after a timeout). */
#define KX_MLP_MAX_LAYERS 8
#define KX_MLP_MAX_SPLIT 8
#define KX_MLP_MAX_ROWS 512
KERNIX_API int kx_mlp_chain(const float* x, int ldx, int m, int n_layers, const float* const* w, const float* const* bias,
                            const int* k, const int* n, const int* act, const float* alpha, int softmax, float* y,
                            float* scratch, uint32_t* bar, int* status, void* stream);
KERNIX_API size_t kx_mlp_chain_scratch_floats(int m, const int* k, const int* n, int n_layers);

/* ---- elementwise / row ops (memory-bound) ---- */

/* y[r][c] = act(x[r][c] + bias[c]) (kernix_bias_act :528-541; ACT step :1864-1866). x == y allowed; bias may be NULL. */
KERNIX_API int kx_bias_act(const float* x, float* y, long rows, int cols, const float* bias, int act, float alpha, void* stream);

/* row softmax (floats_softmax_into include/kernix.h:652-657); x == y allowed */
KERNIX_API int kx_softmax_rows(const float* x, float* y, long rows, int cols, void* stream);

/* row layer norm, biased variance, (x-mean)*rstd*gamma + beta (kernix_layer_norm_rows_into include/kernix.h:667-677);
 * gamma/beta may be NULL; x == y allowed */
KERNIX_API int kx_layernorm_rows(const float* x, float* y, long rows, int cols, const float* gamma, const float* beta, float eps,
                      void* stream);

/* y = x * g[c] + b[c] per row (AFFINE step :1882-1890); x == y allowed */
KERNIX_API int kx_affine_rows(const float* x, float* y, long rows, int cols, const float* g, const float* b, void* stream);

/* y[s][i] = x[s][i] + cst[i] per sample of `per` floats (ADD_CONST step :1891-1895); x == y allowed */
KERNIX_API int kx_add_const(const float* x, float* y, long samples, long per, const float* cst, void* stream);

/* elementwise op with size-1 row/column broadcast inside each sample (kernix_binary_run :877-906).
 * a: samples x ra x ca, b: samples x rb x cb, y: samples x R x C; y may alias a or b when shapes match. */
KERNIX_API int kx_binary(const float* a, int ra, int ca, const float* b, int rb, int cb, float* y, long samples, int R, int C, int op,
              void* stream);

/* max / avg k x k pooling, NHWC (kernix_pooling_run :773-807) */
KERNIX_API int kx_pool2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int kh, int kw, int sh, int sw, int pt,
              int pl, int type, int count_pad, void* stream);

/* per-sample max / mean over R rows (kernix_global_pool_run :810-830) */
KERNIX_API int kx_global_pool(const float* x, float* y, long B, int R, int C, int type, void* stream);

/* per-sample axis permutation, output axis k = input axis perm[k] (kernix_permute_run :833-862) */
KERNIX_API int kx_permute(const float* x, float* y, long B, int nd, const int* dims, const int* perm, void* stream);

/* copy `cols` columns of each row from x (leading dimension ldx) into y at column offset yoff (leading dimension ldy):
 * CONCAT on the channel axis (:908-921) and SELECT on the last axis (:944-947) */
KERNIX_API int kx_copy_cols(const float* x, long ldx, float* y, long ldy, long yoff, long rows, long cols, void* stream);

/* zero-pad H and W of an NHWC image (kernix_pad_run :949-966) */
KERNIX_API int kx_pad2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int pt, int pl, void* stream);

/* nearest upsampling (kernix_upsample_run :968-983) */
KERNIX_API int kx_upsample2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int sh, int sw, void* stream);

/* table rows for float ids, NaN rows for ids out of range or not integral (kernix_embedding_run :986-1000) */
KERNIX_API int kx_embedding(const float* ids, long n, const float* table, int vocab, int dim, float* y, void* stream);

/* depthwise conv (groups == cin): out = bias, += x * w per in-range tap, then act (kernix_conv_run :724-752) */
KERNIX_API int kx_conv_depthwise(const float* x, const float* w, const float* bias, float* y, int B, int H, int W, int C, int Co,
                      int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl, int act, float alpha,
                      void* stream);

/* Implicit-GEMM convolution (NHWC, weights (ky,kx,ci) x cout as the file stores them) on tcgen05 3xTF32 with
 * fused bias + act; the im2col rows are gathered straight into shared memory, never materialised
 * (replaces kernix_conv_run's im2col + sgemm tiles :662-771). w_hi/w_lo: cout x ldw split planes of the
 * weight (kx_prep_f32_weight), ldw >= kh*kw*cin/groups. Output group g writes channels [g*cog, (g+1)*cog). */
KERNIX_API int kx_conv_f32(const float* x, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y, int B, int H,
                int W, int C, int Co, int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl,
                int groups, int act, float alpha, int* status, void* stream);

/* kx_conv_f32 with caller scratch ws of ws_floats floats (16-byte aligned): when the convolution has stride 1, a
 * multiple of 32 input channels and at most 128 output channels per group, K <= 2048, and output images whose
 * pixels cut into 256-pixel tiles of whole rows or whole images, x is split once into tf32 hi / lo planes in ws
 * (2 * B*H*W*C floats) and the pixel operand is loaded by the TMA as 4-D boxes (zero fill = padding) instead of
 * being gathered by threads; otherwise, or with too little scratch, it is kx_conv_f32. Same results within the
 * 3xTF32 bound (the same products in another order). Same role as kx_conv_f32 (kernix_conv_run :662-771). */
KERNIX_API int kx_conv_f32_ws(const float* x, const float* w_hi, const float* w_lo, int ldw, const float* bias, float* y, int B,
                   int H, int W, int C, int Co, int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl,
                   int groups, int act, float alpha, float* ws, size_t ws_floats, int* status, void* stream);

/* scaled dot-product attention per (sample, head): ctx = softmax(scale * Q K^T [+ causal -inf]) V with
 * scale = 1/sqrt(dk) (kernix_attention_run :1015-1046). q: (B*Rq) rows of H*dk at leading dim ldq, k: (B*S) rows
 * of H*dk (ldk), v: (B*S) rows of H*dv (ldv), ctx: (B*Rq) rows of H*dv (ldc). Rq, S <= 128 with head dims <= 64
 * run on the tensor cores (3xTF32), the rest on the CUDA cores. status: device word that receives
 * KX_STATUS_TIMEOUT if a bounded wait gives up (may be NULL). */
KERNIX_API int kx_attention(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* ctx, int ldc, int B,
                 int Rq, int S, int H, int dk, int dv, int causal, int* status, void* stream);

/* y = max(a*x + b, 0), fused multiply-add then max (src/kernix_metal.m:331-338; include/kernix.h:990) */
KERNIX_API int kx_fma_relu(const float* a, const float* x, const float* b, float* y, size_t n, void* stream);

/* Re-interleave an all-gathered column-sharded output: src = [world][rows][slice] -> y rows x (world * slice)
 * with row pitch ldy: y[r][g * slice + j] = src[(g * rows + r) * slice + j]. (Extension; the reference has no
 * sharding.) */
KERNIX_API int kx_unshard_cols(const float* src, int world, long rows, int slice, float* y, int ldy, void* stream);

/* One time step of one direction of an LSTM (kind 0), GRU (1) or SimpleRNN (2) (kernix_rnn_dir,
 * include/kernix_model.h:560-634). zx: (B*T) x G*u input projections x.W + b of all steps (G = 4, 3, 1); U: u x G*u
 * recurrent weights (row-major as in the file); brec: GRU recurrent bias (G*u); h_prev / h_next: B x u states
 * (h_prev unused when first); c: B x u LSTM cell state; the state at time t goes to out + (b*T + t)*stride when
 * ret_seq, else (when last) to out + b*stride. u <= 12288. */
KERNIX_API int kx_rnn_step(int kind, const float* zx, const float* U, const float* brec, const float* h_prev, float* h_next,
                           float* c, float* out, long stride, int B, int T, int t, int u, int first, int ret_seq, int last,
                           int act, float alpha, void* stream);
/* Merge of a bidirectional RNN's directions in place (kernix_rnn_run :641-646): merge 1 sum, 2 product, 3 average. */
KERNIX_API int kx_rnn_merge(float* y, const float* bw, long n, int merge, void* stream);

/* Dense layer for at most KX_SKINNY_MAX_ROWS rows (weight streaming) on the CUDA cores in fp32:
 * y = act(x . W + bias) with W the k x n row-major fp32 weight as in the file; K is split into kx_skinny_slices(n, k)
 * slices whose partial sums (part: slices x m x n floats) are added in slice order. (Extension; the reference runs
 * every dense layer through one sgemm.) */
#define KX_SKINNY_MAX_ROWS 16
KERNIX_API int kx_skinny_slices(int n, int k);
KERNIX_API int kx_gemm_f32_skinny(const float* x, int ldx, const float* w, const float* bias, float* y, int ldy, int m, int n,
                                  int k, int act, float alpha, float* part, size_t part_floats, void* stream);

#ifdef __cplusplus
}
#endif
#endif
