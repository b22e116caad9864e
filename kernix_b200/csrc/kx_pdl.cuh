// Programmatic dependent launch between consecutive kernels of one stream (the row quantiser and the int8 GEMM of
// the int8 dense steps). A kernel launched with launch_pdl may be scheduled while the kernel before it in the stream
// is still running: its CTAs do their set-up (barrier initialisation, tensor-memory allocation, descriptor
// prefetch), then griddep_wait() holds them until that kernel has completed and its writes are visible, so they
// touch no global memory before it. Each such kernel calls griddep_launch_dependents() once it has passed its own
// wait, which lets the next kernel in the stream start launching as soon as every CTA of this one has started;
// those CTAs take SM space only as this kernel's CTAs leave it. A kernel that was not launched this way returns
// from griddep_wait() at once, and a kernel launched normally after these still waits for them to complete.
#pragma once
#include <cuda_runtime.h>

namespace kx {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// <<<grid, block, smem, st>>> with programmatic stream serialisation on a non-default stream (the legacy default
// stream launches normally); 0 on success, -1 on a launch error
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = st != nullptr ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...) == cudaSuccess ? 0 : -1;
}

}  // namespace kx
