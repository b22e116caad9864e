/* NCCL data plane of the column-sharded forward (include/kernix_cuda.h kernix_model_load_sharded_nccl): the
 * all-gather of every sharded step is called by the runtime itself, on the model's stream, with no host callback,
 * so a C program can shard a model across the GPUs of a node. This is the multi-GPU form of the reference's
 * per-call device split of one sgemm (src/kernix_metal.m:161-265), with the exchange over NVLink.
 *
 * libnccl.so.2 is loaded on first use (dlopen; whichever copy the process already has, else the system's), so the
 * library itself neither links NCCL nor needs it unless this plane is used. */
#define _GNU_SOURCE
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "kernix_cuda.h"
#include "kx_internal.h"

static struct {
    void* h;
    ncclResult_t (*get_id)(ncclUniqueId*);
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*destroy)(ncclComm_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char* (*error)(ncclResult_t);
} nccl;
static pthread_once_t nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == NULL) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h == NULL) {
        fprintf(stderr, "kernix: NCCL is not available (%s)\n", dlerror());
        return;
    }
    *(void**)&nccl.get_id = dlsym(h, "ncclGetUniqueId");
    *(void**)&nccl.init_rank = dlsym(h, "ncclCommInitRank");
    *(void**)&nccl.destroy = dlsym(h, "ncclCommDestroy");
    *(void**)&nccl.all_gather = dlsym(h, "ncclAllGather");
    *(void**)&nccl.error = dlsym(h, "ncclGetErrorString");
    if (!nccl.get_id || !nccl.init_rank || !nccl.destroy || !nccl.all_gather || !nccl.error) {
        fprintf(stderr, "kernix: libnccl lacks an entry point this runtime uses\n");
        return;
    }
    nccl.h = h;
}

static int nccl_ready(void) {
    pthread_once(&nccl_once, nccl_load);
    return nccl.h != NULL;
}

KERNIX_API int kernix_nccl_unique_id(void* id) {
    if (id == NULL || !nccl_ready()) return -1;
    ncclUniqueId u;
    const ncclResult_t r = nccl.get_id(&u);
    if (r != ncclSuccess) {
        fprintf(stderr, "kernix: ncclGetUniqueId failed: %s\n", nccl.error(r));
        return -1;
    }
    memcpy(id, &u, sizeof u);
    return 0;
}

/* a communicator of `world` ranks on the current device (collective: every rank calls it with the same id) */
void* kx_nccl_comm_init(int rank, int world, const void* id) {
    if (id == NULL || !nccl_ready()) return NULL;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclComm_t comm = NULL;
    const ncclResult_t r = nccl.init_rank(&comm, world, u, rank);
    if (r != ncclSuccess) {
        fprintf(stderr, "kernix: ncclCommInitRank (rank %d of %d) failed: %s\n", rank, world, nccl.error(r));
        return NULL;
    }
    return comm;
}

void kx_nccl_comm_free(void* comm) {
    if (comm != NULL && nccl.h != NULL) nccl.destroy((ncclComm_t)comm);
}

/* kernix_allgather_fn over a communicator: count floats per rank, rank-major into recv, on the model's stream */
int kx_nccl_gather(void* ctx, const float* send, float* recv, size_t count, void* stream) {
    const ncclResult_t r = nccl.all_gather(send, recv, count, ncclFloat32, (ncclComm_t)ctx, (cudaStream_t)stream);
    if (r != ncclSuccess) {
        fprintf(stderr, "kernix: ncclAllGather failed: %s\n", nccl.error(r));
        return -1;
    }
    return 0;
}
