// Causal flash prefill on B200 tensor cores (tcgen05 + TMEM + TMA).
//
// Math (alpaccaroo/model.py:1254-1272 `_attention_batch_np`, window variant
// model.py:1567-1592): for query token t (absolute position pos[t]) and head
// h, out = softmax_s(q[t,h] . K[s, h/group] * scale) . V[s, h/group] over
// the keys s with kv_start+s <= pos[t] (and > pos[t]-window when window>0).
//
// One CTA per (128-query tile, query head), 256 threads:
//   warp 0      TMA producer: the Q tile once, then K and V tiles (128 keys)
//               into a 2-deep ring, each stage guarded by full/empty mbarriers
//   warp 1      TMEM owner and MMA issuer (one elected lane):
//                 S[j%2] = Q . K_j^T      (tcgen05.mma kind::f16, M=N=128)
//                 O     += P_j . V_j      (A = P from smem, B = V MN-major)
//               QK_{j+1} is issued before PV_j so the tensor core works on
//               the next score tile while the softmax warps handle this one
//   warps 4-7   softmax: thread r owns query row r = TMEM lane r.  It loads
//               its S row with tcgen05.ld, masks, keeps the running max in
//               log2 units, writes P (16-bit) into shared memory in the
//               128-byte-swizzled K-major layout the MMA reads, and rescales
//               the O row in TMEM only when its max grew by more than 2^8
//               (the stale max is exact: l and O share it)
// TMEM: S double buffer (2 x 128 columns) + O (D columns) of a 512-column
// allocation.  Every mbarrier wait is bounded; on expiry the CTA records
// B2A_ERR_TIMEOUT, stops issuing work, frees its TMEM and returns.

#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "b2a_common.cuh"

namespace b2a {
namespace prefill {

constexpr int kBM = 128;  // query rows per CTA
constexpr int kBN = 128;  // keys per tile
constexpr int kThreads = 256;
constexpr int kSoftmaxWarp0 = 4;
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale when max grows > 2^8

template <int D>
struct Layout {
  static constexpr int kBoxBytes = 128 * 128;           // 128 rows x 128 B
  static constexpr int kQBytes = (D / 64) * kBoxBytes;  // Q tile
  static constexpr int kKVBytes = (D / 64) * kBoxBytes; // one K or V tile
  static constexpr int kPBytes = (kBN / 64) * kBoxBytes;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;               // 2 stages
  static constexpr int kV = kK + 2 * kKVBytes;          // 2 stages
  static constexpr int kP = kV + 2 * kKVBytes;
  static constexpr int kTotal = kP + kPBytes;
  static constexpr int kSmem = kTotal + 1024;           // alignment slack
};

// ---------------------------------------------------------------------------
// tcgen05 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// A from TMEM (16-bit A: M rows on lanes, two K elements per 32-bit column,
// K-major), B from shared memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a 128-byte-swizzled tile (the layout
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: 8-row x 128-byte atoms).
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4  bits 46-47 version (1 on sm_100)
//   bits 61-63 layout (2 = 128-byte swizzle)
// K-major: SBO = 1024 (next 8 rows), LBO unused (1).  MN-major: LBO = byte
// distance between 64-element MN chunks, SBO = 1024 (next 8 K rows).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16 with f32 accumulation.
//   bits 4-5 D format (1 = f32); 7-9 A format, 10-12 B format (0 f16, 1 bf16)
//   bit 15 A MN-major, bit 16 B MN-major; 17-22 N >> 3; 24-28 M >> 4
template <typename T>
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((static_cast<uint32_t>(N) >> 3) << 17) |
         ((static_cast<uint32_t>(M) >> 4) << 24);
}

template <typename T>
struct Pack2;
template <>
struct Pack2<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t run(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct Pack2<__half> {
  __device__ __forceinline__ static uint32_t run(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

}  // namespace prefill
}  // namespace b2a

namespace b2a {
namespace prefill {

// A query row with no visible key gets the mean of all t_kv value rows of
// its KV head: the NumPy path masks with -1e30, so every key of such a row
// has weight exp(0) / t_kv (alpaccaroo/model.py:1266-1270, 1584-1588).
// Warp-cooperative: every lane takes part; the rows of the lanes with
// `need` set are written, the lanes splitting the columns (D <= 256).
// Only degenerate inputs (a position before every cached key, or a window
// that excludes them all) reach the loop, so it favours simplicity.
template <typename T, typename TO>
__device__ __noinline__ void store_mean_v_rows(bool need, TO* orow, const T* __restrict__ v,
                                               int t_kv, int KV, int kvh, int D) {
  unsigned mask = __ballot_sync(0xffffffffu, need);
  if (mask == 0u) return;
  const int lane = threadIdx.x & 31;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  for (int s = 0; s < t_kv; ++s) {
    const T* vr = v + (static_cast<size_t>(s) * KV + kvh) * D;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (lane + 32 * c < D) acc[c] += ld_elem(vr + lane + 32 * c);
  }
  const float inv = 1.f / static_cast<float>(t_kv);
  while (mask) {
    const int r = __ffs(mask) - 1;
    mask &= mask - 1u;
    TO* dst = reinterpret_cast<TO*>(
        __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow), r));
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (lane + 32 * c < D) st_elem(dst + lane + 32 * c, acc[c] * inv);
  }
}

// 16 bytes of an output row: 8 16-bit or 4 f32 elements, each times scale.
template <typename TO>
__device__ __forceinline__ uint4 pack16(const float* v, float scale) {
  uint4 u;
  if constexpr (std::is_same<TO, float>::value) {
    u.x = __float_as_uint(v[0] * scale);
    u.y = __float_as_uint(v[1] * scale);
    u.z = __float_as_uint(v[2] * scale);
    u.w = __float_as_uint(v[3] * scale);
  } else {
    u.x = Pack2<TO>::run(v[0] * scale, v[1] * scale);
    u.y = Pack2<TO>::run(v[2] * scale, v[3] * scale);
    u.z = Pack2<TO>::run(v[4] * scale, v[5] * scale);
    u.w = Pack2<TO>::run(v[6] * scale, v[7] * scale);
  }
  return u;
}

// Epilogue of one warp: the O rows of its 32 TMEM lanes (query rows
// row_base .. row_base+31 of head h, TMEM address t_o = lane quarter + O
// column) times inv go to out[row][h][0..D).  Each 128-byte row segment is
// staged in a 4 KB per-warp shared-memory buffer (16-byte chunks XOR-swizzled
// by row, conflict-free both ways), then written by 8 lanes per row, so every
// store instruction covers four whole 128-byte segments instead of 32
// scattered 16-byte pieces.  Rows whose `good` flag is false are skipped.
template <typename TO, int D>
__device__ __forceinline__ void store_o_rows(uint32_t t_o, uint8_t* stg, TO* __restrict__ out,
                                             int row_base, int H, int h, float inv, bool good) {
  constexpr int kCols = 128 / static_cast<int>(sizeof(TO));  // columns per 128-byte segment
  constexpr int kEl = 16 / static_cast<int>(sizeof(TO));     // elements per 16-byte chunk
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ch = 0; ch < D / kCols; ++ch) {
    float o[kCols];
#pragma unroll
    for (int q = 0; q < kCols / 32; ++q) tc_ld32(t_o + ch * kCols + q * 32, o + q * 32);
    tc_wait_ld();
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          pack16<TO>(o + c * kEl, inv);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = i * 4 + (lane >> 3), c = lane & 7;
      const bool g = __shfl_sync(0xffffffffu, good, rr);
      if (g) {
        const uint4 u = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((c ^ (rr & 7)) << 4));
        *reinterpret_cast<uint4*>(out + (static_cast<size_t>(row_base + rr) * H + h) * D +
                                  ch * kCols + c * kEl) = u;
      }
    }
    __syncwarp();
  }
}

template <typename TO>
__device__ __forceinline__ void store_row32(TO* dst, const float* v, float scale);
template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float* v, float scale) {
#pragma unroll
  for (int e = 0; e < 32; e += 4)
    *reinterpret_cast<float4*>(dst + e) =
        make_float4(v[e] * scale, v[e + 1] * scale, v[e + 2] * scale, v[e + 3] * scale);
}
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* dst, const float* v,
                                                           float scale) {
#pragma unroll
  for (int e = 0; e < 32; e += 8) {
    uint4 u;
    u.x = Pack2<__nv_bfloat16>::run(v[e] * scale, v[e + 1] * scale);
    u.y = Pack2<__nv_bfloat16>::run(v[e + 2] * scale, v[e + 3] * scale);
    u.z = Pack2<__nv_bfloat16>::run(v[e + 4] * scale, v[e + 5] * scale);
    u.w = Pack2<__nv_bfloat16>::run(v[e + 6] * scale, v[e + 7] * scale);
    *reinterpret_cast<uint4*>(dst + e) = u;
  }
}
template <>
__device__ __forceinline__ void store_row32<__half>(__half* dst, const float* v, float scale) {
#pragma unroll
  for (int e = 0; e < 32; e += 8) {
    uint4 u;
    u.x = Pack2<__half>::run(v[e] * scale, v[e + 1] * scale);
    u.y = Pack2<__half>::run(v[e + 2] * scale, v[e + 3] * scale);
    u.z = Pack2<__half>::run(v[e + 4] * scale, v[e + 5] * scale);
    u.w = Pack2<__half>::run(v[e + 6] * scale, v[e + 7] * scale);
    *reinterpret_cast<uint4*>(dst + e) = u;
  }
}

template <typename T, typename TO, int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const T* __restrict__ vraw, const int* __restrict__ pos,
    TO* __restrict__ out, int n_q, int t_kv, int H, int group, int n_q_tiles, float sscale,
    int window, int kv_start) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_q;
  __shared__ __align__(8) uint64_t bar_kf[2], bar_ke[2], bar_vf[2], bar_ve[2];
  __shared__ __align__(8) uint64_t bar_sf[2], bar_sfree[2];
  __shared__ __align__(8) uint64_t bar_pf, bar_pv;
  __shared__ uint32_t s_tmem;
  __shared__ int s_pmax, s_pmin;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int qt = n_q_tiles - 1 - static_cast<int>(blockIdx.x);  // longest causal rows first
  const int h = blockIdx.y, kvh = h / group;
  const int row0 = qt * kBM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_kf[s], 1);
      mbar_init(&bar_ke[s], 1);
      mbar_init(&bar_vf[s], 1);
      mbar_init(&bar_ve[s], 1);
      mbar_init(&bar_sf[s], 1);
      mbar_init(&bar_sfree[s], 4);
    }
    mbar_init(&bar_pf, 4);
    mbar_init(&bar_pv, 1);
    s_pmax = INT_MIN;
    s_pmin = INT_MAX;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  if (threadIdx.x < kBM) {
    const int t = row0 + threadIdx.x;
    if (t < n_q) {
      const int p = pos[t];
      atomicMax(&s_pmax, p);
      atomicMin(&s_pmin, p);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  // key tiles [j0, j_end) can hold a visible key for some row of this tile
  int j0 = 0, j_end = 0;
  if (s_pmax != INT_MIN) {
    const long long hi = min(static_cast<long long>(s_pmax) - kv_start + 1, static_cast<long long>(t_kv));
    j_end = hi <= 0 ? 0 : static_cast<int>((hi + kBN - 1) / kBN);
    if (window > 0) {
      const long long lo = static_cast<long long>(s_pmin) - window + 1 - kv_start;
      if (lo > 0) j0 = static_cast<int>(min(lo / kBN, static_cast<long long>(j_end)));
    }
  }
  const int n = j_end - j0;

  const uint32_t sQ = smem_u32(smem + L::kQ);
  const uint32_t sK = smem_u32(smem + L::kK);
  const uint32_t sV = smem_u32(smem + L::kV);
  const uint32_t sP = smem_u32(smem + L::kP);

  if (warp == 0) {
    // ------------------------------ TMA producer ---------------------------
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&bar_q, L::kQBytes);
#pragma unroll
      for (int b = 0; b < D / 64; ++b)
        tma_load_3d(smem + L::kQ + b * L::kBoxBytes, &tmQ, &bar_q, b * 64, h, row0);
      for (int i = 0; i < n; ++i) {
        const int j = j0 + i, slot = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (i >= 2 && !mbar_wait(&bar_ke[slot], ph ^ 1, 0x1000 | i)) break;
        mbar_arrive_expect_tx(&bar_kf[slot], L::kKVBytes);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(smem + L::kK + slot * L::kKVBytes + b * L::kBoxBytes, &tmK, &bar_kf[slot],
                      b * 64, kvh, j * kBN);
        if (i >= 2 && !mbar_wait(&bar_ve[slot], ph ^ 1, 0x2000 | i)) break;
        mbar_arrive_expect_tx(&bar_vf[slot], L::kKVBytes);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(smem + L::kV + slot * L::kKVBytes + b * L::kBoxBytes, &tmV, &bar_vf[slot],
                      b * 64, kvh, j * kBN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_qk = make_idesc<T>(kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = make_idesc<T>(kBM, D, false, true);
      bool ok = mbar_wait(&bar_q, 0, 0x3000);
      auto issue_qk = [&](int i) -> bool {
        const int slot = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&bar_kf[slot], ph, 0x4000 | i)) return false;
        if (i >= 2 && !mbar_wait(&bar_sfree[slot], ph ^ 1, 0x5000 | i)) return false;
        tc_fence_after();
        const uint32_t kb = sK + slot * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
          tc_mma(tmem + slot * kBN, sw128_desc(sQ + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                 idesc_qk, kk > 0);
        }
        tc_commit(&bar_sf[slot]);
        tc_commit(&bar_ke[slot]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int i = 0; ok && i < n; ++i) {
        if (i + 1 < n && !issue_qk(i + 1)) break;
        if (!mbar_wait(&bar_pf, i & 1, 0x6000 | i)) break;
        const int slot = i & 1;
        if (!mbar_wait(&bar_vf[slot], (i >> 1) & 1, 0x7000 | i)) break;
        tc_fence_after();
        const uint32_t vb = sV + slot * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * L::kBoxBytes + (kk & 3) * 32;
          tc_mma(tmem + 2 * kBN, sw128_desc(sP + poff, 16, 1024),
                 sw128_desc(vb + kk * 16 * 128, L::kBoxBytes, 1024), idesc_pv, (i > 0 || kk > 0));
        }
        tc_commit(&bar_pv);
        tc_commit(&bar_ve[slot]);
      }
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------ softmax --------------------------------
    const int r = (warp - kSoftmaxWarp0) * 32 + lane;  // query row == TMEM lane
    const int t = row0 + r;
    const int my_pos = (t < n_q) ? pos[t] : INT_MIN;
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int j = j0 + i, slot = i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_sf[slot], (i >> 1) & 1, 0x8000 | i));
      if (!ok) break;
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tc_ld32(tl + slot * kBN + c * 32, s + c * 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_sfree[slot]);

      // visible keys of this tile: lo <= c <= hi (c < valid too)
      const long long kv0 = static_cast<long long>(kv_start) + static_cast<long long>(j) * kBN;
      const long long hi_ll = (my_pos == INT_MIN) ? -1 : static_cast<long long>(my_pos) - kv0;
      const int hi = static_cast<int>(min(hi_ll, static_cast<long long>(min(kBN, t_kv - j * kBN) - 1)));
      const int lo = (window > 0 && my_pos != INT_MIN)
                         ? static_cast<int>(max(static_cast<long long>(my_pos) - window + 1 - kv0, -1ll))
                         : -1;
      // branch-free mask (a short-circuit test compiles to a branch per
      // element); four partial maxima keep the FMNMX chain short
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; c += 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int cc = c + e;
          s[cc] = ((cc <= hi) & (cc >= lo)) ? s[cc] * sscale : -INFINITY;
        }
        mx0 = fmaxf(mx0, s[c]);
        mx1 = fmaxf(mx1, s[c + 1]);
        mx2 = fmaxf(mx2, s[c + 2]);
        mx3 = fmaxf(mx3, s[c + 3]);
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      const float mnew = fmaxf(m, mx);
      const bool need = mnew > m + kRescaleThreshold;
      const bool warp_need = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (warp_need) {
        alpha = (mnew == -INFINITY) ? 1.f : fast_exp2(m - mnew);
        m = mnew;
      }
      const float mref = (m == -INFINITY) ? 0.f : m;
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = fast_exp2(s[c] - mref);
        const float p1 = fast_exp2(s[c + 1] - mref);
        s[c] = p0;
        s[c + 1] = p1;
        sum0 += p0;
        sum1 += p1;
      }
      const float sum = sum0 + sum1;
      l = l * alpha + sum;

      // P buffer and O are free once PV of the previous tile completed
      if (i > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv, (i - 1) & 1, 0x9000 | i));
        if (!ok) break;
        tc_fence_after();
        if (warp_need) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tc_ld32(tl + 2 * kBN + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tc_st32(tl + 2 * kBN + c * 32, o);
          }
          tc_wait_st();
        }
      }
      uint8_t* prow = smem + L::kP + r * 128;
#pragma unroll
      for (int ch = 0; ch < kBN / 8; ++ch) {
        uint4 u;
        u.x = Pack2<T>::run(s[ch * 8 + 0], s[ch * 8 + 1]);
        u.y = Pack2<T>::run(s[ch * 8 + 2], s[ch * 8 + 3]);
        u.z = Pack2<T>::run(s[ch * 8 + 4], s[ch * 8 + 5]);
        u.w = Pack2<T>::run(s[ch * 8 + 6], s[ch * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + (ch >> 3) * L::kBoxBytes + (((ch & 7) ^ (r & 7)) << 4)) = u;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_pf);
    }
    // epilogue: O / l -> out
    if (n > 0 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv, (n - 1) & 1, 0xA000));
      tc_fence_after();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    TO* orow = out + (static_cast<size_t>(t) * H + h) * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      if (n > 0 && ok) {
        tc_ld32(tl + 2 * kBN + c * 32, o);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0.f;
      }
      if (t < n_q && l > 0.f) store_row32<TO>(orow + c * 32, o, inv);
    }
    store_mean_v_rows<T, TO>(ok && t < n_q && !(l > 0.f), orow, vraw, t_kv, H / group, kvh, D);
  }
  // ------------------------------ teardown ---------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace prefill
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

namespace P = b2a::prefill;
using P::Layout;
using P::kBM;
using P::prefill_kernel;
using b2a_host::fail;

// Defined in prefill_pair.cu, prefill_head.cu and prefill_f32.cu (same
// translation unit).
template <typename T, typename TO, int D>
int launch_prefill_pair(const void* q, const void* k, const void* v, const int* pos, void* out,
                        int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
                        cudaStream_t st);

template <typename T, typename TO, int D>
int launch_prefill_head(const void* q, const void* k, const void* v, const int* pos, void* out,
                        int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
                        cudaStream_t st);

int prefill_f32_dispatch(int out_dtype, const void* q, const void* k, const void* v,
                         const int* pos, void* out, int n_q, int t_kv, int H, int KV, int D,
                         float scale, int window, int kv_start, cudaStream_t st);

// Kernel choice for 16-bit inputs.  Default: the paired-head persistent
// kernel (prefill_pair.cu) for even GQA groups at head_dim 64 and 128, the
// one-head persistent kernel (prefill_head.cu) otherwise and always at
// head_dim 256.  B2ATTN_PREFILL=head|pair|single forces one where it serves
// the shape (pair falls back to head for odd groups); the non-persistent
// one-tile kernel below is kept as a tested reference schedule.
enum class PrefillKernel { kHead, kPair, kSingle };
PrefillKernel prefill_choice(int group) {
  const char* e = getenv("B2ATTN_PREFILL");
  if (e && strcmp(e, "single") == 0) return PrefillKernel::kSingle;
  if (e && strcmp(e, "head") == 0) return PrefillKernel::kHead;
  return group % 2 == 0 ? PrefillKernel::kPair : PrefillKernel::kHead;
}

template <typename T, typename TO, int D>
int launch_prefill(const void* q, const void* k, const void* v, const int* pos, void* out, int n_q,
                   int t_kv, int H, int KV, float scale, int window, int kv_start, cudaStream_t st) {
  if constexpr (D > 128) {
    return launch_prefill_head<T, TO, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window,
                                         kv_start, st);
  } else {
    const PrefillKernel choice = prefill_choice(H / KV);
    if (choice == PrefillKernel::kPair && (H / KV) % 2 == 0)
      return launch_prefill_pair<T, TO, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window,
                                           kv_start, st);
    if (choice != PrefillKernel::kSingle)
      return launch_prefill_head<T, TO, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window,
                                           kv_start, st);
    const CUtensorMapDataType tdt = std::is_same<T, __nv_bfloat16>::value
                                        ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tq, tk, tv;
    const uint64_t qdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H), static_cast<uint64_t>(n_q)};
    const uint64_t qstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H) * D * 2};
    const uint64_t kdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(KV), static_cast<uint64_t>(t_kv)};
    const uint64_t kstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(KV) * D * 2};
    const uint32_t box[3] = {64, 1, 128};
    int rc = b2a_host::make_tmap(&tq, tdt, 3, const_cast<void*>(q), qdims, qstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = b2a_host::make_tmap(&tk, tdt, 3, const_cast<void*>(k), kdims, kstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = b2a_host::make_tmap(&tv, tdt, 3, const_cast<void*>(v), kdims, kstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    auto kern = prefill_kernel<T, TO, D>;
    // >= 116 KB keeps one CTA per SM, so the 512-column TMEM allocation never
    // waits on a co-resident CTA.
    const int smem = Layout<D>::kSmem > 116 * 1024 ? Layout<D>::kSmem : 116 * 1024;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(prefill)");
    const int n_q_tiles = (n_q + kBM - 1) / kBM;
    dim3 grid(n_q_tiles, H);
    kern<<<grid, P::kThreads, smem, st>>>(tq, tk, tv, static_cast<const T*>(v), pos,
                                          static_cast<TO*>(out), n_q, t_kv, H, H / KV, n_q_tiles,
                                          scale * P::kLog2e, window, kv_start);
    e = cudaGetLastError();
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "prefill launch");
    return B2A_OK;
  }
}

template <typename T, int D>
int prefill_out(int out_dtype, const void* q, const void* k, const void* v, const int* pos,
                void* out, int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
                cudaStream_t st) {
  switch (out_dtype) {
    case B2A_F32:
      return launch_prefill<T, float, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
    case B2A_F16:
      return launch_prefill<T, __half, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
    case B2A_BF16:
      return launch_prefill<T, __nv_bfloat16, D>(q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  }
  return fail(B2A_ERR_DTYPE, "prefill: out_dtype %d", out_dtype);
}

template <typename T>
int prefill_d(int D, int out_dtype, const void* q, const void* k, const void* v, const int* pos,
              void* out, int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
              cudaStream_t st) {
  if (D == 64) return prefill_out<T, 64>(out_dtype, q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  if (D == 128) return prefill_out<T, 128>(out_dtype, q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  if (D == 256) return prefill_out<T, 256>(out_dtype, q, k, v, pos, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  return fail(B2A_ERR_UNSUPPORTED, "prefill: 16-bit head_dim %d (64, 128 or 256)", D);
}

}  // namespace

extern "C" int b2a_prefill(const void* q, const void* k_cache, const void* v_cache,
                           const int* pos_dev, void* out, int n_q, int t_kv, int H, int KV, int D,
                           int in_dtype, int out_dtype, float scale, int window, int kv_start,
                           void* stream) {
  if (!q || !k_cache || !v_cache || !pos_dev || !out) return fail(B2A_ERR_ARG, "prefill: null pointer argument");
  if (n_q < 0 || t_kv <= 0 || H <= 0 || KV <= 0 || D <= 0 || kv_start < 0)
    return fail(B2A_ERR_ARG, "prefill: bad sizes (T=%d t_kv=%d H=%d KV=%d D=%d kv_start=%d)", n_q, t_kv, H, KV, D, kv_start);
  if (H % KV != 0) return fail(B2A_ERR_SHAPE, "prefill: H=%d is not a multiple of KV=%d", H, KV);
  if (!(scale > 0.f) || !isfinite(scale)) return fail(B2A_ERR_ARG, "prefill: scale must be positive");
  if (!b2a_host::aligned16(q) || !b2a_host::aligned16(k_cache) || !b2a_host::aligned16(v_cache) ||
      !b2a_host::aligned16(out))
    return fail(B2A_ERR_ALIGN, "prefill: q, caches and out must be 16-byte aligned");
  if (n_q == 0) return B2A_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (in_dtype == B2A_F32)
    return prefill_f32_dispatch(out_dtype, q, k_cache, v_cache, pos_dev, out, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
  if (in_dtype == B2A_BF16)
    return prefill_d<__nv_bfloat16>(D, out_dtype, q, k_cache, v_cache, pos_dev, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  if (in_dtype == B2A_F16)
    return prefill_d<__half>(D, out_dtype, q, k_cache, v_cache, pos_dev, out, n_q, t_kv, H, KV, scale, window, kv_start, st);
  return fail(B2A_ERR_DTYPE, "prefill: in_dtype %d (F32, F16 or BF16)", in_dtype);
}
