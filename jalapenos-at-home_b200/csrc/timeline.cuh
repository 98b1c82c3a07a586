// Kernel phase timeline: a diagnostic build of the library (-DJL_TIMELINE,
// `make timeline` -> lib/libjalapeno_timeline.so) in which the decode-pass
// kernels write %globaltimer stamps at fixed points of their critical path,
// one row of TL_POINTS per (launch, CTA), into a device table that
// jl_timeline_read copies out.  Launch ids are handed out in recording order
// and restart with every recorded pass, so a captured pass replayed any
// number of times rewrites the same rows: the table holds the last replay of
// the last pass recorded (time_pass and time_pass_draft record one pass and
// replay it).  In the normal build every stamp compiles to nothing, the
// table is never allocated and kernels receive a null slot.
//
// Points (unused points stay 0):
//   k_mx_gemv      0 entry, 1 loader past the grid-dependency wait, 2 first
//                  ring slot full (MMA warp), 3 first accumulator complete
//                  (epilogue), 4 split-K partials of the first tile in (leader),
//                  5 outputs final, activation pieces next, 6 epilogue done,
//                  7 exit
//   k_dec_proj     0 entry, 1 past the wait, 2 inputs and weights in shared
//                  memory, 3 outputs written
//   k_attn_decode  0 entry, 1 past the wait, 2 queries and this pass's K/V
//                  ready, 3 scores and softmax done, 4 output written,
//                  5 pieces of the output written
#pragma once

#include <cstddef>
#include <cstdint>

#include "jl_internal.h"

namespace jl {

#ifdef JL_TIMELINE
__device__ __forceinline__ void tl_stamp(const TlSlot& s, int point) {
    if (!s.table || s.id < 0 || s.id >= TL_LAUNCHES) return;
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta >= (unsigned)TL_CTAS) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    s.table[((size_t)s.id * TL_CTAS + cta) * TL_POINTS + point] = t;
}
#else
__device__ __forceinline__ void tl_stamp(const TlSlot&, int) {}
#endif

}  // namespace jl
