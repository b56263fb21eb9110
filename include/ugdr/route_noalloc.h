/* MoE routing without any allocation.  This entry point has no counterpart in the reference.
 *
 * ugdr_x_moe_route (include/ugdr/collective.h) needs caller-provided scratch device memory for
 * its per-block expert histograms.  Some callers cannot allocate device memory at all: code that
 * runs where cudaMalloc / cudaFree are not allowed (inside a framework's memory-pool hooks or
 * allocator callbacks, in a process whose allocator is owned by someone else, or with a strict
 * "no allocation after start-up" rule on a serving path).  This variant keeps that scratch in a
 * fixed array compiled into libugdr instead:
 *
 *  - Capacity: UGDR_X_ROUTE_NOALLOC_MAX_ENTRIES 32-bit entries (256 KiB).  A call needs
 *    ceil(rows / 4096) * nexp entries; larger calls are rejected with cudaErrorInvalidValue and
 *    nothing is launched.  Every GPU that loads libugdr holds this 256 KiB until the process exits.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
 *    that device current) and keeps it for the life of the process; make that first call before
 *    any stream capture.  cudaDeviceReset (or any other teardown of the device's primary
 *    context) unloads the module and makes the kept address stale: after one, call
 *    ugdr_x_moe_route_noalloc_reset() on that device before the next call.
 *  - Every call on a device shares the same array.  Calls that overlap on the GPU (different
 *    streams, or different host threads) race and corrupt each other's results; serialise them.
 *    Nothing is read before being written within a call, so the previous call's leftovers do not
 *    matter.
 *  - No cudaMalloc, cudaFree or other allocating routine is called.
 *
 * Inputs, outputs and the return value are those of ugdr_x_moe_route. */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UGDR_X_ROUTE_NOALLOC_MAX_ENTRIES (64u * 1024u)

int ugdr_x_moe_route_noalloc(const int32_t *expert_ids, uint64_t rows, int nexp, int32_t *counts,
                             int32_t *positions, void *stream);

/* Forget the kept scratch address of the current device, so the next call looks it up again.
 * Needed only after cudaDeviceReset or another teardown of the primary context.  Returns a
 * cudaError_t value. */
int ugdr_x_moe_route_noalloc_reset(void);

#ifdef __cplusplus
}
#endif
