// Shared device/host helpers for the B200 attention library (libb2attn.so).
//
// Everything here is sm_100a-only: mbarrier phase waits (bounded), TMA tensor
// copies (no cluster multicast anywhere in this library), ldmatrix/movmatrix
// fragment moves, and the error plumbing the C ABI exposes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

#include "../../include/b2attn.h"

namespace b2a {

// ---------------------------------------------------------------------------
// Device-side error record.  Kernels never trap: a bounded wait that runs out,
// or a position outside the cache, writes a code here and the kernel returns.
// The host reads it back with b2a_device_error().
// ---------------------------------------------------------------------------
// (Defined here: the library is one translation unit, b2attn_all.cu.)
__device__ int g_dev_error = 0;      // first error code seen (0 = none)
__device__ int g_dev_error_aux = 0;  // kernel-specific detail (tile, row, ...)

__device__ __forceinline__ void set_dev_error(int code, int aux) {
  if (atomicCAS(&g_dev_error, 0, code) == 0) g_dev_error_aux = aux;
}

// Limit for every spin-wait on an mbarrier (nanoseconds of %globaltimer).
// Two seconds is orders of magnitude above any legitimate wait in these
// kernels (one TMA tile or one MMA batch) yet short enough that a lost
// arrival surfaces as B2A_ERR_TIMEOUT instead of a hung GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the barrier's phase with the given parity has completed.
// Returns false (and records B2A_ERR_TIMEOUT with `where`) if the wait
// exceeds kWaitLimitNs; the caller then abandons its work and exits.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int where) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if ((++spins & 255u) == 0u) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_dev_error(B2A_ERR_TIMEOUT, where);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA tensor loads (tiled, single CTA, no multicast).  The innermost
// coordinate is always a multiple of 64 elements of a 16-bit type here, so it
// is 128-byte aligned; no load starts at a negative x.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of one tile of a 3-D tensor map (no shared memory, no mbarrier);
// same coordinate rules as tma_load_3d.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Offset of 16-byte chunk `chunk` (0..7) of row `row` inside a tile written
// by TMA with CU_TENSOR_MAP_SWIZZLE_128B and 128-byte rows (tile base
// 1024-byte aligned): the chunk index is XORed with the row index mod 8.
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + (((chunk ^ row) & 7) << 4));
}

// ---------------------------------------------------------------------------
// Warp-level matrix fragment moves (legacy mma path used by decode).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct MmaOp;

template <>
struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

template <>
struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Element load/store helpers for the three cache dtypes.
__device__ __forceinline__ float ld_elem(const float* p) { return *p; }
__device__ __forceinline__ float ld_elem(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float ld_elem(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st_elem(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_elem(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void st_elem(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// Wait until the kernel this one was launched after (as a programmatic
// dependent) has completed and its writes are visible; returns at once for
// an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 2^x with the SFU instruction (PTX ex2.approx.ftz.f32: relative error about
// 2^-22, ex2(-inf) = +0).  The softmax kernels feed it max-subtracted scores.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace b2a

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace b2a_host {

// Record a message for b2a_last_error() (thread-local) and return `code`.
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

// Encode a tiled tensor map through the driver entry point (no -lcuda link).
// dims/strides follow cuTensorMapEncodeTiled: dims[0] innermost, strides in
// bytes for dims 1..rank-1.
int make_tmap(CUtensorMap* out, CUtensorMapDataType dtype, int rank, void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle);

int elem_size(int dtype);
bool aligned16(const void* p);

// The calling thread's b2a_set_launch_flags value.
int launch_flags();

// Number of SMs of the current device (cudaDevAttrMultiProcessorCount, read
// once per device and cached), for persistent grids and split heuristics.
int sm_count();

// Launch `kern`, as a programmatic dependent of the stream's previous kernel
// when the thread's launch flags ask for it (the kernel then waits with
// griddepcontrol.wait before reading that kernel's output).
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (launch_flags() & B2A_LAUNCH_PDL) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace b2a_host
