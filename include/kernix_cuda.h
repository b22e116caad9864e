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

#ifdef __cplusplus
}
#endif
#endif
