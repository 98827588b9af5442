// L2 prefetch lists: byte ranges a launch asks HBM for ahead of their use
// (by its own later phases or by the next launches of a step), so that the
// weight and KV stream keeps going across grid barriers and kernel
// boundaries.  Each CTA of the launch prefetches its slice of every range,
// ranges in order, with cp.async.bulk.prefetch.L2 (pf_issue in ptx.cuh); the
// later loads of that data then hit L2.  Starts are 16-byte aligned; a
// range's length is used rounded down to 16 bytes.
#pragma once
#include <cstdint>

namespace laya {

constexpr int PF_MAX = 8;
struct PfList {
  const uint8_t* p[PF_MAX];
  unsigned long long n[PF_MAX];
  int count;
};

}  // namespace laya
