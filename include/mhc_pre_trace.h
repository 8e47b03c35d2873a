/*
 * mhc_pre_trace.h -- stage stamps of the trace build (libmhcpre_b200_trace.so).
 *
 * The trace build is the operator library compiled with -DMHC_TRACE: the same
 * entry points (include/mhc_pre.h) and the same results, plus, in the kernels of
 * the split-K path (0), the one-pass path (5) and the fused post step
 * (mhcPostPreRun), %globaltimer stamps of their
 * stages, recorded by every 8th CTA into a device array of 4 Mi records.  The
 * default library exports none of this and records nothing.  No reference
 * counterpart (the reference's own notes propose GetSystemCycle stage markers,
 * docs/MhcPre_组化路线性能分析.md:64-86, which it never implemented).
 *
 * Record layout (24 bytes, little endian):
 *   uint64 t_ns   %globaltimer at the event
 *   uint32 cta    blockIdx.x
 *   uint16 warp   warp index within the CTA
 *   uint16 event  1 producer item taken, 2 item's first chunk issued, 3 item's
 *                 records published (a = tile, b = split); 4 hIn row taken,
 *                 5 row's tile complete, 6 row's records summed, 7 row's hIn
 *                 written (one-pass path), 8 / 9 split-K epilogue row begin / end
 *                 (a = row low 32 bits, b = row high 32 bits); 10 / 11 CTA begin /
 *                 end (a = path).  In the fused post + MhcPre kernel (mhcPostPreRun):
 *                 2 a stage's loads issued, 5 its data landed, 6 its xNext formed,
 *                 7 its xNext stores have read it (a = the CTA's stage count, b = tile)
 *   uint32 a, b   event arguments
 */
#ifndef MHC_PRE_TRACE_H
#define MHC_PRE_TRACE_H

#include <stddef.h>
#include <stdint.h>

#include "mhc_pre.h"

#ifdef __cplusplus
extern "C" {
#endif

#define MHC_PRE_TRACE_RECORD_BYTES 24

/* Copies up to maxRecords trace records (synchronizing the current device first)
 * into host memory at dst, stores how many the kernels recorded since the last call
 * in *recorded (it may exceed maxRecords or the device capacity: the excess is
 * lost) and clears the trace. */
MHC_API int mhcPreTraceRead(void* dst, size_t maxRecords, size_t* recorded);

#ifdef __cplusplus
}
#endif
#endif /* MHC_PRE_TRACE_H */
