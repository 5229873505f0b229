/*
 * pkv_trace.h -- NVTX ranges around the library's entry points.
 *
 * Each public call (append, decode, prefill, the dense SDPA, the step
 * transaction, the decoder entry point) opens a range named after itself,
 * so a profiler timeline (nsys, ncu's NVTX filter) shows which host call
 * issued which kernels.  This is the tracing counterpart of the SDK's
 * phase timers (include/timing.h, compiled in with TENSOR_TIMING_ENABLE).
 * NVTX v3 is header-only: until a tool injects itself (NVTX_INJECTION64_PATH
 * or a profiler), a range costs one indirect call to an empty function.
 * Define PKV_NO_NVTX to compile the ranges out.
 */
#ifndef PKV_TRACE_H
#define PKV_TRACE_H

#ifndef PKV_NO_NVTX
#include <nvtx3/nvToolsExt.h>
#define PKV_RANGE_PUSH(name) ((void)nvtxRangePushA(name))
#define PKV_RANGE_POP() ((void)nvtxRangePop())
#else
#define PKV_RANGE_PUSH(name) ((void)(name))
#define PKV_RANGE_POP() ((void)0)
#endif

#ifdef __cplusplus
/* Scoped range: pushed here, popped on every return path. */
struct PkvTraceRange {
    explicit PkvTraceRange(const char *name) { PKV_RANGE_PUSH(name); }
    ~PkvTraceRange() { PKV_RANGE_POP(); }
    PkvTraceRange(const PkvTraceRange &) = delete;
    PkvTraceRange &operator=(const PkvTraceRange &) = delete;
};
#define PKV_RANGE(name) PkvTraceRange pkv_trace_range_(name)
#endif

#endif
