// Library-wide C ABI pieces: version, error reporting, tensor-map encoding.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "b2a_common.cuh"

namespace {
thread_local char t_last_error[512] = "";
thread_local int t_launch_flags = 0;

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}
}  // namespace

namespace b2a_host {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B2A_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int elem_size(int dtype) {
  switch (dtype) {
    case B2A_F32: return 4;
    case B2A_F16: return 2;
    case B2A_BF16: return 2;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int make_tmap(CUtensorMap* out, CUtensorMapDataType dtype, int rank, void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle) {
  PFN_encodeTiled fn = get_encode_fn();
  if (!fn) return fail(B2A_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  CUresult r = fn(out, dtype, (cuuint32_t)rank, base, d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2A_ERR_ARG, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return B2A_OK;
}

int launch_flags() { return t_launch_flags; }

int sm_count() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cached[kMaxDevices];  // 0 = not read yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < kMaxDevices) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  if (dev >= 0 && dev < kMaxDevices) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace b2a_host

extern "C" {

int b2a_version(void) { return B2A_ABI_VERSION; }

int b2a_set_launch_flags(int flags) {
  const int old = t_launch_flags;
  t_launch_flags = flags & B2A_LAUNCH_PDL;
  return old;
}

const char* b2a_last_error(void) { return t_last_error; }

int b2a_device_error(int* code, int* aux, int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaDeviceSynchronize");
  int c = 0, a = 0;
  e = cudaMemcpyFromSymbol(&c, b2a::g_dev_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&a, b2a::g_dev_error_aux, sizeof(int));
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaMemcpyFromSymbol");
  if (code) *code = c;
  if (aux) *aux = a;
  if (clear) {
    int z = 0;
    e = cudaMemcpyToSymbol(b2a::g_dev_error, &z, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(b2a::g_dev_error_aux, &z, sizeof(int));
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaMemcpyToSymbol");
  }
  return B2A_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Self-test of the bounded mbarrier wait every kernel here uses: one thread
// initialises a barrier that nothing arrives on and waits for its first
// phase.  The wait gives up after kWaitLimitNs, records B2A_ERR_TIMEOUT with
// aux 0x7F000 and the kernel returns normally, so the context stays usable.
// ---------------------------------------------------------------------------
namespace b2a {
__global__ void wait_selftest_kernel() {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_wait(&bar, 0, 0x7F000);  // no arrival: runs out, records the timeout
}
}  // namespace b2a

extern "C" int b2a_selftest_wait_timeout(void* stream) {
  b2a::wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "wait self-test launch");
  return B2A_OK;
}
