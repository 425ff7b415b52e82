// Exchange-buffer layout and tagged 8-byte words of the sharded decode
// (shard.cu), shared with the decode split kernel (decode.cu), whose last
// CTA per (sequence, KV head) publishes that group's merged rows.
//
// Each rank's exchange buffer (zeroed once before first use):
//   words  [2][G][R][D+1] uint2   (step parity, source rank, row; D values
//                                  then the lse), each word (f32 value, u32
//                                  tag = step + 1)
//   steps  [R] u32                this rank's finished steps per row
//   counts [R] u32                split-CTA arrival tickets per (sequence,
//                                  KV head), back to 0 after each step
#pragma once

#include "b2a_common.cuh"

namespace b2a {
namespace shard {

struct XLayout {
  size_t words, steps, counts, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

__host__ __device__ inline XLayout xlayout(int R, int D, int G) {
  XLayout x;
  x.words = 0;
  x.steps = align256(static_cast<size_t>(2) * G * R * (D + 1) * sizeof(uint2));
  x.counts = x.steps + align256(static_cast<size_t>(R) * sizeof(uint32_t));
  x.total = x.counts + align256(static_cast<size_t>(R) * sizeof(uint32_t));
  return x;
}

// First word of (parity, source rank, row): D value words, then the lse.
__device__ __forceinline__ size_t word_index(int parity, int src, int row, int R, int G, int D) {
  return ((static_cast<size_t>(parity) * G + src) * R + row) * static_cast<size_t>(D + 1);
}

// One 8-byte store of (value, tag): a reader never sees the tag without
// the value.
__device__ __forceinline__ void st_tagged(uint2* p, float v, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)),
               "r"(tag)
               : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const uint2* p) {
  uint2 w;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(p)
               : "memory");
  return w;
}

// Where the split kernel publishes (peers == nullptr: it does not).
struct Publish {
  unsigned char* const* peers;  // device table [G] of the ranks' exchange buffers
  int me, G;
};

}  // namespace shard
}  // namespace b2a
