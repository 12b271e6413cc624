// Tile scheduler for the persistent tensor-core kernels.
//
// Every CTA owns a contiguous range of tiles (the static split of the
// launch) and takes them from the front; once its range is empty it takes
// single tiles from the back of the other CTAs' ranges, one victim at a time.
// A CTA therefore keeps to one cell for long runs (its own range, then the
// tail of a victim's), while SMs that stream slower than others hand their
// last tiles to faster ones instead of setting the kernel's end.
//
// State: one 64-bit word per CTA in global memory, low half = next tile from
// the front, high half = end of the range (exclusive).  The owner advances
// the front with atomicAdd (it may overshoot the end once the range is
// empty, which every reader treats as empty); thieves lower the end with
// compare-and-swap only while front < end, so no tile is handed out twice
// and the end never wraps.
//
// Inside a CTA the producer thread draws the tiles and publishes them in a
// ring of RING slots in shared memory; the other roles read slot it % RING
// after the mbarrier that orders them behind the producer's iteration it.
// A negative id ends the CTA's work.
#pragma once

#include <cstdint>

namespace kvc {
namespace sched {

constexpr int RING = 32;  // > stages + 6 of any kernel using it

__device__ __forceinline__ uint64_t pack(uint32_t front, uint32_t end) { return (uint64_t)end << 32 | front; }

// Static split: CTA b owns [b * per_cta, min((b + 1) * per_cta, total)).
__device__ __forceinline__ void init_ranges(unsigned long long* w, int i, int nctas, int64_t per_cta, int64_t total) {
  if (i >= nctas) return;
  const int64_t f = (int64_t)i * per_cta;
  const int64_t e = f + per_cta < total ? f + per_cta : total;
  w[i] = pack((uint32_t)f, (uint32_t)(e > f ? e : f));
}

// Next tile for CTA `me` (-1 when every range is empty).  `victim` carries
// the thief's position between calls; start it at `me`.
__device__ __forceinline__ int64_t next_tile(unsigned long long* w, int me, int nctas, int& victim) {
  if (victim == me) {
    const unsigned long long old = atomicAdd(&w[me], 1ull);
    const uint32_t f = (uint32_t)old, e = (uint32_t)(old >> 32);
    if (f < e) return f;
    victim = me + 1 < nctas ? me + 1 : 0;
  }
  for (int n = 0; n < nctas - 1 && victim != me; ++n) {
    unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(&w[victim]);
    for (;;) {
      const uint32_t f = (uint32_t)cur, e = (uint32_t)(cur >> 32);
      if (f >= e) break;
      const unsigned long long seen = atomicCAS(&w[victim], cur, pack(f, e - 1));
      if (seen == cur) return e - 1;
      cur = seen;
    }
    victim = victim + 1 < nctas ? victim + 1 : 0;
  }
  victim = me;  // a later call finds everything empty again quickly
  return -1;
}

__device__ __forceinline__ void ring_put(int32_t* ring, int it, int32_t tile) {
  *reinterpret_cast<volatile int32_t*>(&ring[it % RING]) = tile;
}
__device__ __forceinline__ int32_t ring_get(const int32_t* ring, int it) {
  return *reinterpret_cast<const volatile int32_t*>(&ring[it % RING]);
}

}  // namespace sched
}  // namespace kvc
