/* KERNIX-B200 device-memory forward (extension; no counterpart in the reference, whose forward only takes
 * host memory: include/kernix_model.h:2023, src/kernix_capi.c:24-32).
 *
 * For callers whose input rows already live in GPU memory (e.g. produced by other kernels): runs the same
 * forward as kernix_capi_forward but reads x and writes out on the device, ordered on the caller's stream,
 * without host copies and without synchronising. The workspace is chunked by the model's workspace limit as
 * in the host-memory forward.
 */
#ifndef KERNIX_CUDA_H
#define KERNIX_CUDA_H

#include "kernix_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* d_x: rows x in_dim device floats (rows a positive multiple of seq_len), d_out: (rows/seq_len) x out_dim device
 * floats, stream: cudaStream_t the work is ordered on (0 = the legacy default stream). Both buffers must be on the model's device.
 * Returns 0 when all work was enqueued, -1 on bad arguments or a launch failure. Wait on the stream, then call
 * kernix_model_check to learn whether a kernel reported a failure. */
KERNIX_API int kernix_model_forward_device(kernix_model* m, const float* d_x, int rows, float* d_out, void* stream);

/* After the work of kernix_model_forward_device has completed (stream synchronised): 0 if every kernel
 * finished normally, -1 if one gave up on a bounded wait (the output is then invalid). Resets the flag. */
KERNIX_API int kernix_model_check(kernix_model* m);

/* ------------------------------------------------------------------ output-column sharding across GPUs
 * (extension; no counterpart in the reference, whose GPU/CPU row split of one sgemm, src/kernix_metal.m:161-265,
 * becomes a split of wide dense layers across the GPUs of one node).
 *
 * One process per GPU loads the same .knx with its rank. Every fp32 LINEAR step with at least
 * KERNIX_SHARD_MIN_COLS outputs, divisible by world, keeps only its slice of weight and bias columns
 * [out * rank / world, out * (rank + 1) / world); the forward computes that slice of the layer's output, then the
 * caller-supplied all-gather assembles every rank's slice (rank-major: [world][rows][out / world]) and a kernel
 * re-interleaves it into the full rows for the next step. All other steps run whole on every rank, so every rank
 * returns the full output. The collective order is the step order, the same on every rank; the host-memory
 * forward of a sharded model runs each chunk in one piece for that reason. */
#define KERNIX_SHARD_MIN_COLS 1024

/* All-gather of `count` floats per rank: every rank's `send` (device) lands in `recv` (device, world * count
 * floats, rank r at offset r * count), ordered on `stream` (a cudaStream_t) after the work already on it, and
 * later work on the stream waits for it. Returns 0 on success. */
typedef int (*kernix_allgather_fn)(void* ctx, const float* send, float* recv, size_t count, void* stream);

/* kernix_model_load for rank `rank` of `world` processes (0 <= rank < world); `gather` is called with `ctx` at
 * every sharded step. world = 1 loads the whole model (gather unused). NULL on failure, as kernix_model_load. */
KERNIX_API kernix_model* kernix_model_load_sharded(const char* path, int rank, int world, kernix_allgather_fn gather,
                                                   void* ctx);

/* The same sharded load with the all-gather done by the runtime itself: every rank calls it with the same 128-byte
 * NCCL unique id (kernix_nccl_unique_id on one rank, then shared by the host program), the model creates its NCCL
 * communicator on its device (collective: all ranks must call concurrently) and each sharded step calls
 * ncclAllGather on the model's stream -- no host callback, so a C program can shard. NCCL (libnccl.so.2) is
 * loaded on first use. The communicator is destroyed by kernix_model_free. world = 1 loads the whole model. */
KERNIX_API kernix_model* kernix_model_load_sharded_nccl(const char* path, int rank, int world, const void* nccl_id);

/* A new NCCL unique id (128 bytes into id) for kernix_model_load_sharded_nccl. 0, or -1 if NCCL is unavailable. */
KERNIX_API int kernix_nccl_unique_id(void* id);

/* ------------------------------------------------------------------ batch sharding across GPUs
 * (extension; the reference's chunk loop over one batch, include/kernix_model.h:2036-2063, spread over devices).
 * With $KERNIX_GPUS naming two or more devices ("0,1,2,3" or "all") when kernix_model_load runs, the model is
 * loaded whole onto each of them; every host-memory forward (kernix_model_forward, kernix_capi_forward) then gives
 * each device a contiguous share of the samples, run concurrently (one host thread per extra device), each
 * share's rows read from and written to the caller's buffers at their offsets -- the same rows as one device
 * computes. kernix_model_forward_device runs on the first device only. Unset or one device: one device. */

#ifdef __cplusplus
}
#endif
#endif
