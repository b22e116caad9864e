/* KERNIX-B200 shared-library ABI for FFI callers (the numpy/ctypes binding python/kernix.py).
 *
 * Exactly the ten symbols of the reference's src/kernix_capi.c, same arguments and return codes, so the
 * unchanged reference binding runs against libkernix.so (KERNIX_LIB=/path/to/libkernix.so). The model
 * handle is a kernix_model* passed as void*.
 */
#ifndef KERNIX_CAPI_H
#define KERNIX_CAPI_H

#include <stddef.h>
#include "kernix.h"

#ifdef __cplusplus
extern "C" {
#endif

/* src/kernix_capi.c:7 — NULL on failure (reason on stderr) */
KERNIX_API void* kernix_capi_load(const char* path);
/* src/kernix_capi.c:9 */
KERNIX_API void kernix_capi_free(void* m);
/* src/kernix_capi.c:12 — release the workspace, keep weights */
KERNIX_API void kernix_capi_trim(void* m);
/* src/kernix_capi.c:15 — workspace bound in bytes, 0 = unlimited */
KERNIX_API void kernix_capi_set_workspace_limit(void* m, size_t bytes);
/* src/kernix_capi.c:17-20 */
KERNIX_API void kernix_capi_dims(const void* m, int* in_dim, int* out_dim, int* seq_len);
/* src/kernix_capi.c:24-32 — x: rows x in_dim host floats (rows a positive multiple of seq_len); writes
 * (rows / seq_len) x out_dim floats to out. 0 = success, -1 = failure. Page-locked x / out are copied
 * asynchronously at full PCIe speed; pageable buffers work too. */
KERNIX_API int kernix_capi_forward(void* m, const float* x, int rows, float* out);
/* src/kernix_capi.c:35 — -1 for on = 1 (no Neural Engine), 0 for on = 0 */
KERNIX_API int kernix_capi_set_ane(void* m, int on);
/* src/kernix_capi.c:38-43 — out[4] = segments, compiles, ane_runs, failures (all 0) */
KERNIX_API void kernix_capi_ane_info(const void* m, int* out);
/* src/kernix_capi.c:46-54 — always -1 (no Core ML) */
KERNIX_API int kernix_capi_ane_dump(const void* m, int seg, int batch, const char* path);
/* src/kernix_capi.c:57-61 */
KERNIX_API void kernix_capi_shapes(const void* m, int* in_nd, int* in_shape, int* out_nd, int* out_shape, int* layout);

#ifdef __cplusplus
}
#endif
#endif
