/* fmha_fwd_trace.h -- entry points of the trace build of the kernel
 * (libfmha_b200_trace.so: the same source compiled with -DFMHA_TRACE).
 *
 * No counterpart in the reference: it exposes the per-role pipeline timeline
 * of the sm_100a kernel (clock64 stamps of pass 0 for a window of CTAs),
 * which is how the kernel's limiter is measured.  The product library
 * (libfmha_b200.so) exports none of these.  The launch entry points of
 * include/fmha_fwd.h are exported by the trace library too; stamping costs a
 * few instructions per event and changes no result.
 */
#ifndef FMHA_FWD_TRACE_H
#define FMHA_FWD_TRACE_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Buffer geometry: *ctas consecutive CTAs x *steps KV steps x *slots events
 * of 64-bit clock64 values. */
int fmha_fwd_d64_trace_shape(int* ctas, int* steps, int* slots);

/* Trace CTAs [first_cta, first_cta + ctas) of the following launches and
 * clear the buffer (synchronous; current device). */
int fmha_fwd_d64_trace_configure(int first_cta);

/* Copy the first `count` 64-bit entries of the buffer to host memory
 * (synchronous). */
int fmha_fwd_d64_trace_read(unsigned long long* dst, size_t count);

#ifdef __cplusplus
}
#endif

#endif /* FMHA_FWD_TRACE_H */
