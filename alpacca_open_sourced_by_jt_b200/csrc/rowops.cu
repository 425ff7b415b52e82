// Row-wise glue of a device-resident prefill chunk (the reference's
// Model.forward_batch, alpaccaroo/model.py:1274-1372, and its device twin
// prefill_chunk, cuda.py:1943-2080), around the chunk's GEMMs:
//
//   b2a_rmsnorm_rows  out[t] = x[t] * (1 / sqrt(mean(x[t]^2) + eps)) * w
//                     (tensor.py:355-356), written in the GEMM's input type
//   b2a_swiglu_rows   act[t][i] = g / (1 + exp(-g)) * u for the FFN's gate
//                     and up values of row t (model.py:1352-1354)
//
// One CTA per row; the mean of squares is summed in double.  Rows of up to
// 4096 floats with 16-byte-aligned strides take the kernel that loads them
// as float4 and keeps them in registers (x read once).

namespace b2a {
namespace rows {

constexpr int kThreads = 256;

template <typename TO>
__global__ void __launch_bounds__(kThreads) rmsnorm_rows_kernel(
    const float* __restrict__ x, long long xs, const float* __restrict__ w, float eps,
    TO* __restrict__ out, long long os, int E) {
  __shared__ double red[kThreads / 32];
  const float* xr = x + blockIdx.x * xs;
  double ss = 0.0;
  for (int c = threadIdx.x; c < E; c += kThreads) {
    const double v = xr[c];
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) tot += red[i];
  const float inv = static_cast<float>(1.0 / sqrt(tot / E + static_cast<double>(eps)));
  TO* orow = out + blockIdx.x * os;
  for (int c = threadIdx.x; c < E; c += kThreads) st_elem(orow + c, xr[c] * inv * w[c]);
}

template <typename TO>
__device__ __forceinline__ void store4(TO* dst, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float* dst, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float a, float b, float c, float d) {
  const __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
  *reinterpret_cast<uint2*>(dst) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                                              *reinterpret_cast<const uint32_t*>(&hi));
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float a, float b,
                                                      float c, float d) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  *reinterpret_cast<uint2*>(dst) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                                              *reinterpret_cast<const uint32_t*>(&hi));
}

// The same row norm with 16-byte loads, for rows of up to kThreads * 4 * kVec
// floats whose length and strides are multiples of 4: each thread keeps its
// kVec float4 of the row in registers between the sum and the scaling, so x
// is read once, and writes 4 outputs per store.
template <typename TO, int kVec>
__global__ void __launch_bounds__(kThreads) rmsnorm_rows_vec_kernel(
    const float* __restrict__ x, long long xs, const float* __restrict__ w, float eps,
    TO* __restrict__ out, long long os, int E) {
  __shared__ double red[kThreads / 32];
  const float4* xr = reinterpret_cast<const float4*>(x + blockIdx.x * xs);
  const int e4 = E >> 2;
  float4 v[kVec];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    v[i] = c < e4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += static_cast<double>(v[i].x) * v[i].x;
    ss += static_cast<double>(v[i].y) * v[i].y;
    ss += static_cast<double>(v[i].z) * v[i].z;
    ss += static_cast<double>(v[i].w) * v[i].w;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) tot += red[i];
  const float inv = static_cast<float>(1.0 / sqrt(tot / E + static_cast<double>(eps)));
  TO* orow = out + blockIdx.x * os;
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < e4) {
      const float4 g = w4[c];
      store4<TO>(orow + 4 * c, v[i].x * inv * g.x, v[i].y * inv * g.y, v[i].z * inv * g.z,
                 v[i].w * inv * g.w);
    }
  }
}

template <typename TO>
int launch_rmsnorm_rows(const float* x, long long xs, const float* w, float eps, TO* out,
                        long long os, int n_rows, int E, cudaStream_t st) {
  const bool vec = (E & 3) == 0 && (xs & 3) == 0 && (os & 3) == 0 && E <= 4 * 4 * kThreads &&
                   b2a_host::aligned16(x) && b2a_host::aligned16(w) &&
                   (reinterpret_cast<uintptr_t>(out) & (4 * sizeof(TO) - 1)) == 0;
  if (!vec)
    rmsnorm_rows_kernel<TO><<<n_rows, kThreads, 0, st>>>(x, xs, w, eps, out, os, E);
  else if (E <= 4 * kThreads)
    rmsnorm_rows_vec_kernel<TO, 1><<<n_rows, kThreads, 0, st>>>(x, xs, w, eps, out, os, E);
  else if (E <= 2 * 4 * kThreads)
    rmsnorm_rows_vec_kernel<TO, 2><<<n_rows, kThreads, 0, st>>>(x, xs, w, eps, out, os, E);
  else
    rmsnorm_rows_vec_kernel<TO, 4><<<n_rows, kThreads, 0, st>>>(x, xs, w, eps, out, os, E);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "rmsnorm_rows launch");
  return B2A_OK;
}

template <typename TO>
__global__ void __launch_bounds__(kThreads) swiglu_rows_kernel(
    const float* __restrict__ gu, long long gs, int interleaved, TO* __restrict__ out,
    long long os, int F) {
  const float* r = gu + blockIdx.x * gs;
  TO* orow = out + blockIdx.x * os;
  for (int i = threadIdx.x; i < F; i += kThreads) {
    const float g = interleaved ? r[2 * i] : r[i];
    const float u = interleaved ? r[2 * i + 1] : r[F + i];
    st_elem(orow + i, g / (1.f + expf(-g)) * u);
  }
}

}  // namespace rows
}  // namespace b2a

extern "C" {

int b2a_rmsnorm_rows(const float* x, long long x_row_stride, const float* w, float eps, void* out,
                     long long out_row_stride, int out_dtype, int n_rows, int E, void* stream) {
  using b2a_host::fail;
  if (!x || !w || !out) return fail(B2A_ERR_ARG, "rmsnorm_rows: null pointer argument");
  if (n_rows < 0 || E <= 0 || x_row_stride < E || out_row_stride < E || !(eps > 0.f))
    return fail(B2A_ERR_ARG, "rmsnorm_rows: bad sizes, strides or eps");
  if (n_rows == 0) return B2A_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  namespace K = b2a::rows;
  switch (out_dtype) {
    case B2A_F32:
      return K::launch_rmsnorm_rows(x, x_row_stride, w, eps, static_cast<float*>(out),
                                    out_row_stride, n_rows, E, st);
    case B2A_F16:
      return K::launch_rmsnorm_rows(x, x_row_stride, w, eps, static_cast<__half*>(out),
                                    out_row_stride, n_rows, E, st);
    case B2A_BF16:
      return K::launch_rmsnorm_rows(x, x_row_stride, w, eps, static_cast<__nv_bfloat16*>(out),
                                    out_row_stride, n_rows, E, st);
    default:
      return fail(B2A_ERR_DTYPE, "rmsnorm_rows: out_dtype %d", out_dtype);
  }
}

int b2a_swiglu_rows(const float* gu, long long gu_row_stride, int interleaved, void* out,
                    long long out_row_stride, int out_dtype, int n_rows, int F, void* stream) {
  using b2a_host::fail;
  if (!gu || !out) return fail(B2A_ERR_ARG, "swiglu_rows: null pointer argument");
  if (n_rows < 0 || F <= 0 || gu_row_stride < 2LL * F || out_row_stride < F)
    return fail(B2A_ERR_ARG, "swiglu_rows: bad sizes or strides");
  if (n_rows == 0) return B2A_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  namespace K = b2a::rows;
  const int il = interleaved ? 1 : 0;
  switch (out_dtype) {
    case B2A_F32:
      K::swiglu_rows_kernel<float><<<n_rows, K::kThreads, 0, st>>>(
          gu, gu_row_stride, il, static_cast<float*>(out), out_row_stride, F);
      break;
    case B2A_F16:
      K::swiglu_rows_kernel<__half><<<n_rows, K::kThreads, 0, st>>>(
          gu, gu_row_stride, il, static_cast<__half*>(out), out_row_stride, F);
      break;
    case B2A_BF16:
      K::swiglu_rows_kernel<__nv_bfloat16><<<n_rows, K::kThreads, 0, st>>>(
          gu, gu_row_stride, il, static_cast<__nv_bfloat16*>(out), out_row_stride, F);
      break;
    default:
      return fail(B2A_ERR_DTYPE, "swiglu_rows: out_dtype %d", out_dtype);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "swiglu_rows launch");
  return B2A_OK;
}

}  // extern "C"
