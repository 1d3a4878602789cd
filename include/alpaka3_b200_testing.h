/* alpaka3_b200 -- test hooks exported by libalpaka3_b200.so. Not part of the product interface
 * (include/alpaka3_b200.h): they exist so the test suite can drive failure paths and host-side bookkeeping without a
 * GPU fault. No counterpart in alpaka3. */
#ifndef ALPAKA3_B200_TESTING_H
#define ALPAKA3_B200_TESTING_H

#include "alpaka3_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Failure detection: runs a3b_scan (no caller buffer) with tile `stall_tile` never publishing its aggregate, so every
 * later tile's bounded wait for it gives up after the configured timeout, raises bit 0 of the device error word and
 * returns. The output is undefined; the context stays usable. */
A3B_API int a3b_scan_debug_stall(a3b_stream_t stream, int dtype, void const* in, void* out, uint64_t n, uint64_t stall_tile);

/* a3b_set_early_start for an explicit device ordinal, without touching the CUDA runtime (host bookkeeping only). */
A3B_API int a3b_debug_early_start_enable(int device, a3b_stream_t stream, int enable);

/* The reductions' early-start guard on its own (host only, launches nothing): whether a reduction of the `in_bytes`
 * bytes at in0 / in1 (either may be null) writing `out` would be launched with the early start on (device, stream),
 * after which `out` joins the stream's history exactly as in a real launch. *early receives 1 or 0. */
A3B_API int a3b_debug_early_start_probe(int device, a3b_stream_t stream, void const* in0, void const* in1,
                                        uint64_t in_bytes, void* out, int* early);

#ifdef __cplusplus
}
#endif

#endif /* ALPAKA3_B200_TESTING_H */
