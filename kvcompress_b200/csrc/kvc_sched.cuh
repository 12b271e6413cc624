// Tile order of the persistent tensor-core kernels.
//
// CTA b takes the contiguous range [b * per_cta, min((b + 1) * per_cta,
// total)) of the launch's tiles in order, so it keeps to one cell for long
// runs (one B-image load per cell it touches).  Inside a CTA the producer
// thread draws the tiles and publishes them in a ring of RING slots in
// shared memory; the other roles read slot it % RING after the mbarrier that
// orders them behind the producer's iteration it, and a negative id ends the
// CTA's work.  The consumers therefore never recompute the order, and the
// end travels down the pipeline with the same barriers as the data.
//
// (Work stealing between CTAs, tried with per-CTA range words in global
// memory, evened out the CTAs' end times but lowered the aggregate
// throughput of every kernel by 7-14% on B200, so the ranges are static.)
#pragma once

#include <cstdint>

namespace kvc {
namespace sched {

constexpr int RING = 32;  // > stages + 6 of any kernel using it

struct Cursor {
  int64_t next, end;  // remaining tiles [next, end)
  __device__ Cursor(int64_t per_cta, int64_t total) {
    next = (int64_t)blockIdx.x * per_cta;
    end = next + per_cta < total ? next + per_cta : total;
  }
};

// Next tile of this CTA, -1 at the end of its range.
__device__ __forceinline__ int64_t next_tile(Cursor& c) { return c.next < c.end ? c.next++ : -1; }

__device__ __forceinline__ void ring_put(int32_t* ring, int it, int32_t tile) {
  *reinterpret_cast<volatile int32_t*>(&ring[it % RING]) = tile;
}
__device__ __forceinline__ int32_t ring_get(const int32_t* ring, int it) {
  return *reinterpret_cast<const volatile int32_t*>(&ring[it % RING]);
}

}  // namespace sched
}  // namespace kvc
