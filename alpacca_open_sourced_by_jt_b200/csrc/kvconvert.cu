// KV cache element conversion (b2a_kv_convert): the widening / narrowing
// between a 16-bit device cache and the f32 rows of snapshots and host
// mirrors (alpaccaroo/cuda.py:1881-1900 and :2046-2061 do these on the host;
// alpaccaroo/memory.py:224-241 fixes the f32-le snapshot rows).
//
// HBM-bound: each element is read once and written once.  Each thread moves
// 8 elements per step with 16-byte (16-bit side) or 2 x 16-byte (f32 side)
// accesses when both buffers are 16-byte aligned (widening: two steps' loads
// before their stores); the grid is a multiple of the SM count and strides
// over the buffer.  Narrowing rounds to nearest
// even (__float2half_rn / __float2bfloat16_rn), as NumPy's astype(float16)
// and torch's bfloat16 cast do.

#include "b2a_common.cuh"

namespace b2a {
namespace kv {

constexpr int kThreads = 256;
constexpr int kVec = 8;

template <typename S, typename Dt>
__device__ __forceinline__ Dt cvt(S x) {
  return static_cast<Dt>(x);
}
template <>
__device__ __forceinline__ float cvt<__half, float>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float cvt<__nv_bfloat16, float>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ __half cvt<float, __half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<float, __nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half cvt<__nv_bfloat16, __half>(__nv_bfloat16 x) {
  return __float2half_rn(__bfloat162float(x));  // exact widening, one rounding
}
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__half, __nv_bfloat16>(__half x) {
  return __float2bfloat16_rn(__half2float(x));
}

// 8 elements of T, 16-byte aligned (one 16-byte access for 16-bit T, two for
// f32); the host takes this path only when both buffers are 16-byte aligned
template <typename T>
struct alignas(16) Vec8 {
  T e[kVec];
};

template <typename S, typename Dt>
__global__ void __launch_bounds__(kThreads) convert_kernel(const S* __restrict__ src,
                                                           Dt* __restrict__ dst, long long n,
                                                           int vector_ok) {
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nthreads = static_cast<long long>(gridDim.x) * blockDim.x;
  long long done = 0;
  if (vector_ok) {
    // widening writes twice what it reads: two loads in flight per thread
    // before the stores keep more reads queued behind the write stream
    constexpr int U = sizeof(Dt) > sizeof(S) ? 2 : 1;
    const long long nv = n / kVec;
    const Vec8<S>* sv = reinterpret_cast<const Vec8<S>*>(src);
    Vec8<Dt>* dv = reinterpret_cast<Vec8<Dt>*>(dst);
    long long i = tid;
    for (; U > 1 && i + (U - 1) * nthreads < nv; i += U * nthreads) {
      Vec8<S> a[U];
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = sv[i + u * nthreads];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        Vec8<Dt> b;
#pragma unroll
        for (int k = 0; k < kVec; ++k) b.e[k] = cvt<S, Dt>(a[u].e[k]);
        dv[i + u * nthreads] = b;
      }
    }
    for (; i < nv; i += nthreads) {
      const Vec8<S> a = sv[i];
      Vec8<Dt> b;
#pragma unroll
      for (int k = 0; k < kVec; ++k) b.e[k] = cvt<S, Dt>(a.e[k]);
      dv[i] = b;
    }
    done = nv * kVec;
  }
  for (long long i = done + tid; i < n; i += nthreads) dst[i] = cvt<S, Dt>(src[i]);
}

}  // namespace kv
}  // namespace b2a

namespace {

template <typename S, typename Dt>
int launch_convert(const void* src, void* dst, long long n, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long per_block = static_cast<long long>(b2a::kv::kThreads) * b2a::kv::kVec;
  long long blocks = (n + per_block - 1) / per_block;
  // 8 x 256 threads resident per SM; widening launches two rounds of them
  const long long cap = static_cast<long long>(sms) * (sizeof(Dt) > sizeof(S) ? 16 : 8);
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const int vec = b2a_host::aligned16(src) && b2a_host::aligned16(dst) &&
                  (sizeof(S) * b2a::kv::kVec) % 16 == 0 && (sizeof(Dt) * b2a::kv::kVec) % 16 == 0;
  b2a::kv::convert_kernel<S, Dt><<<static_cast<int>(blocks), b2a::kv::kThreads, 0, st>>>(
      static_cast<const S*>(src), static_cast<Dt*>(dst), n, vec);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "kv_convert launch");
  return B2A_OK;
}

template <typename S>
int convert_from(const void* src, void* dst, int dst_dtype, long long n, cudaStream_t st) {
  switch (dst_dtype) {
    case B2A_F32: return launch_convert<S, float>(src, dst, n, st);
    case B2A_F16: return launch_convert<S, __half>(src, dst, n, st);
    case B2A_BF16: return launch_convert<S, __nv_bfloat16>(src, dst, n, st);
  }
  return b2a_host::fail(B2A_ERR_DTYPE, "kv_convert: destination dtype %d", dst_dtype);
}

}  // namespace

extern "C" int b2a_kv_convert(const void* src, int src_dtype, void* dst, int dst_dtype,
                              long long n, void* stream) {
  using b2a_host::fail;
  if (n < 0) return fail(B2A_ERR_ARG, "kv_convert: negative count %lld", n);
  if (n == 0) return B2A_OK;
  if (!src || !dst) return fail(B2A_ERR_ARG, "kv_convert: null buffer");
  const int ss = b2a_host::elem_size(src_dtype), ds = b2a_host::elem_size(dst_dtype);
  if (!ss) return fail(B2A_ERR_DTYPE, "kv_convert: source dtype %d", src_dtype);
  if (!ds) return fail(B2A_ERR_DTYPE, "kv_convert: destination dtype %d", dst_dtype);
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(src), d0 = reinterpret_cast<uintptr_t>(dst);
  const uintptr_t s1 = s0 + static_cast<uintptr_t>(n) * ss, d1 = d0 + static_cast<uintptr_t>(n) * ds;
  if (s0 < d1 && d0 < s1) return fail(B2A_ERR_ARG, "kv_convert: source and destination overlap");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (src_dtype) {
    case B2A_F32: return convert_from<float>(src, dst, dst_dtype, n, st);
    case B2A_F16: return convert_from<__half>(src, dst, dst_dtype, n, st);
    case B2A_BF16: return convert_from<__nv_bfloat16>(src, dst, dst_dtype, n, st);
  }
  return fail(B2A_ERR_DTYPE, "kv_convert: source dtype %d", src_dtype);
}
