/* GCD dispatch_apply stand-in for compiling the KERNIX reference on Linux.
 * TEST INFRASTRUCTURE ONLY (oracle/ref/Makefile). dispatch_apply(n, queue, fn) runs fn(0..n-1) and returns
 * when all have finished, as GCD does; here the iterations are an OpenMP dynamic loop. The block argument
 * arrives as a function pointer because deblock.py rewrote every block literal into a nested function. */
#ifndef KX_DISPATCH_SHIM_H
#define KX_DISPATCH_SHIM_H
#include <stddef.h>
#define DISPATCH_APPLY_AUTO 0
static inline void dispatch_apply(size_t n, int queue, void (*fn)(size_t))
{
    (void)queue;
#pragma omp parallel for schedule(dynamic, 1)
    for (long i = 0; i < (long)n; i++) fn((size_t)i);
}
#endif
