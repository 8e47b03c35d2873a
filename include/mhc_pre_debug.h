/*
 * mhc_pre_debug.h -- extra entry points of the debug build (libmhcpre_b200_debug.so).
 *
 * The debug build is the operator library compiled with -DMHC_DEBUG: the same entry
 * points (include/mhc_pre.h) and the same results, plus bounds checks in the
 * kernels on every partial-record index (the workspace buffer the kernels index
 * with computed offsets).  A failed check skips the access it guards, sets the
 * device status word to MHC_STATUS_INTERNAL_CHECK (read it with
 * mhcPreGetDeviceStatus) and records the source line.  It stands in for a memory
 * checker, which is not available on every machine.  The default library exports
 * none of this and checks nothing.  No reference counterpart.
 */
#ifndef MHC_PRE_DEBUG_H
#define MHC_PRE_DEBUG_H

#include <stdint.h>

#include "mhc_pre.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Tells the kernels of later calls that the records buffer holds at most
 * maxFloats floats (0: its real size).  With a cap below the real size, the
 * checks fail on the first record beyond it -- on purpose, and without any
 * access outside a buffer -- which is how the tests exercise them.  Process-wide;
 * not for concurrent use. */
MHC_API int mhcPreDebugSetRecordCap(int64_t maxFloats);

/* Source line (in mhc_pre_kernels.cu and the headers it includes) of the first
 * check that failed since the last call, or 0; clears it.  Synchronizes the
 * current device. */
MHC_API int mhcPreDebugLastCheckLine(int32_t* line);

#ifdef __cplusplus
}
#endif
#endif /* MHC_PRE_DEBUG_H */
