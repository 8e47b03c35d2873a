// Stage stamps for the trace build (compile flag MHC_TRACE; libmhcpre_b200_trace.so).
//
// A traced kernel records events {%globaltimer ns, CTA, warp, event, a, b} into a
// device array: every CTA whose index is a multiple of kTraceCtaStride records, the
// others do not, so the trace stays small and the traced CTAs stay representative.
// The host reads and clears it with mhcPreTraceRead (include/mhc_pre_trace.h).  In
// the default build MHC_TRACE_EV expands to nothing and no array exists.
#pragma once

#include <cstdint>

namespace mhc {

// Event codes (the a/b arguments in brackets).
enum TraceEvent : uint32_t {
    kTrGemmItemBegin = 1,  // split-K / one-pass producer: item taken [tile, split]
    kTrGemmItemIssue = 2,  // producer: first chunk of the item issued [tile, split]
    kTrGemmRecord = 3,     // square-sum warp: item's records published [tile, split]
    kTrRowWait = 4,        // hIn warp: row taken, waiting for its tile [row lo, row hi]
    kTrRowReady = 5,       // hIn warp: the tile's records are complete [row lo, row hi]
    kTrRowReduced = 6,     // hIn warp: records summed, slot row freed [row lo, row hi]
    kTrRowDone = 7,        // hIn warp: hIn of the row written [row lo, row hi]
    kTrEpiRowBegin = 8,    // split-K epilogue: row begins (after its dependency wait) [row lo, row hi]
    kTrEpiRowDone = 9,     // split-K epilogue: row done [row lo, row hi]
    kTrKernelBegin = 10,   // any traced kernel: CTA start [path, 0]
    kTrKernelEnd = 11,     // any traced kernel: CTA end [path, 0]
};

struct TraceRecord {
    uint64_t t_ns;
    uint32_t cta;
    uint16_t warp;
    uint16_t event;
    uint32_t a;
    uint32_t b;
};
static_assert(sizeof(TraceRecord) == 24, "trace records are 24 bytes");

constexpr int kTraceCtaStride = 8;
constexpr unsigned kTraceCapacity = 4u << 20;  // records (96 MiB)

#ifdef MHC_TRACE
// Defined here: the header is included by the one translation unit that holds all
// device code (mhc_pre_kernels.cu).
__device__ TraceRecord g_trace[kTraceCapacity];
__device__ unsigned g_trace_count = 0;

__device__ __forceinline__ void trace_event(uint32_t ev, uint32_t a, uint32_t b) {
    if (blockIdx.x % kTraceCtaStride != 0) return;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const unsigned i = atomicAdd(&g_trace_count, 1u);
    if (i < kTraceCapacity) {
        TraceRecord r;
        r.t_ns = t;
        r.cta = blockIdx.x;
        r.warp = static_cast<uint16_t>(threadIdx.x >> 5);
        r.event = static_cast<uint16_t>(ev);
        r.a = a;
        r.b = b;
        g_trace[i] = r;
    }
}
#define MHC_TRACE_EV(ev, a, b) ::mhc::trace_event((ev), static_cast<uint32_t>(a), static_cast<uint32_t>(b))
#else
#define MHC_TRACE_EV(ev, a, b) ((void)0)
#endif

}  // namespace mhc
