// Long-context decode with the KV rows sharded across GPUs: the split-KV
// combine, the exchange of every rank's partial result over NVLink and the
// cross-rank log-sum-exp merge as ONE kernel over peer memory.
//
// Each rank holds a contiguous range of every sequence's cache rows and
// runs the decode split kernel over it (decode.cu).  Then, per output row r
// (one (sequence, query head) pair):
//   phase A  merge this rank's split partials into (o_r, lse_r) (the
//            algebra of the reference's _attention_decode_combine,
//            alpaccaroo/cuda.py:674-694), store them into slot [me] of
//            EVERY rank's exchange buffer with plain stores through the
//            CUDA-IPC mappings (NVLink peer stores; no TMA, no multicast),
//            then publish flag[me][r] = step + 1 on every rank with a
//            system-scope release store;
//   phase B  wait (acquire loads, bounded by kShardWaitNs) until every
//            rank's flag[g][r] in this rank's own buffer reached step + 1,
//            then merge the G parts by their lse:
//              out_r = sum_g exp(lse_g - L) o_g,  L = log sum_g exp(lse_g)
// so every rank ends with the merged rows, the result of an all-gather
// followed by the combine, without a separate collective or launch.
//
// Exchange buffer of each rank (b2a_shard_exchange_bytes, zeroed once
// before first use): data [2][G][R][D+1] f32 (step parity, source rank,
// row, o then lse), flags [G][R] u32 (written by the source ranks), steps
// [R] u32 (this rank's count of finished steps per row).  Double buffering
// by step parity is enough: a rank can write step n+2 into a slot only after
// its step n+1 waited for every rank's step n+1 flag, which each rank
// publishes only after its step n kernel (the last reader of the slot) has
// completed on its stream.  Rows are independent (per-row flags and step
// counts), so ranks may use different grids.
//
// The grid never exceeds the number of CTAs that can be resident at once,
// and every CTA finishes phase A for all of its rows before it waits in
// phase B, so the waits cannot block a CTA that has yet to publish.

namespace b2a {
namespace shard {

constexpr int kThreads = 128;
// Limit of a phase-B wait: far above any skew between ranks that step
// together, short enough that a rank that never arrives surfaces as
// B2A_ERR_TIMEOUT (the kernel then merges what it has and returns).
constexpr uint64_t kShardWaitNs = 2000000000ull;

struct XLayout {
  size_t data, flags, steps, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

__host__ __device__ inline XLayout xlayout(int R, int D, int G) {
  XLayout x;
  x.data = 0;
  x.flags = align256(static_cast<size_t>(2) * G * R * (D + 1) * sizeof(float));
  x.steps = x.flags + align256(static_cast<size_t>(G) * R * sizeof(uint32_t));
  x.total = x.steps + align256(static_cast<size_t>(R) * sizeof(uint32_t));
  return x;
}

__device__ __forceinline__ size_t data_index(int parity, int src, int row, int R, int G, int D) {
  return ((static_cast<size_t>(parity) * G + src) * R + row) * static_cast<size_t>(D + 1);
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Merge row bh's split partials (m in log2 units, l, unnormalised acc) into
// o (shared memory, D floats); returns the natural-log lse (-inf when the
// row's shard holds no cache rows).
__device__ float merge_splits(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                              int bh, int ns, int n_splits, int D, float* wsm, float* o) {
  __shared__ float red[kThreads / 32];
  __shared__ float s_M, s_L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t p0 = static_cast<size_t>(bh) * n_splits;
  if (ns == 0) {
    for (int d = threadIdx.x; d < D; d += kThreads) o[d] = 0.f;
    __syncthreads();
    return -INFINITY;
  }
  float M = -INFINITY;
  for (int s = threadIdx.x; s < ns; s += kThreads) M = fmaxf(M, part_ml[(p0 + s) * 2]);
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (threadIdx.x == 0) {
    float x = red[0];
    for (int w = 1; w < kThreads / 32; ++w) x = fmaxf(x, red[w]);
    s_M = x;
  }
  __syncthreads();
  M = s_M;
  float L = 0.f;
  for (int s = threadIdx.x; s < ns; s += kThreads) {
    const float w = exp2f(part_ml[(p0 + s) * 2] - M);
    wsm[s] = w;
    L += part_ml[(p0 + s) * 2 + 1] * w;
  }
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  __syncthreads();
  if (threadIdx.x == 0) {
    float x = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) x += red[w];
    s_L = x;
  }
  __syncthreads();
  L = s_L;
  const float invL = 1.f / L;
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float a0 = 0.f, a1 = 0.f;
    int s = 0;
    for (; s + 1 < ns; s += 2) {
      a0 += part_o[(p0 + s) * D + d] * wsm[s];
      a1 += part_o[(p0 + s + 1) * D + d] * wsm[s + 1];
    }
    if (s < ns) a0 += part_o[(p0 + s) * D + d] * wsm[s];
    o[d] = (a0 + a1) * invL;
  }
  __syncthreads();
  return (M + log2f(L)) * 0.6931471805599453f;
}

__global__ void __launch_bounds__(kThreads) shard_exchange_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_ml,
    const int* __restrict__ lens, float* __restrict__ out, float* __restrict__ lse_out,
    unsigned char* const* __restrict__ peers, int me, int G, int R, int H, int D,
    int split_rows, int n_splits, int row_limit) {
  extern __shared__ float ssm[];
  float* wsm = ssm;                 // [n_splits] split weights
  float* obuf = ssm + n_splits;     // [D] this rank's merged row
  __shared__ uint32_t s_step;
  __shared__ int s_abort;  // a wait of this CTA ran out: later rows do not wait again
  const XLayout xl = xlayout(R, D, G);
  if (threadIdx.x == 0) s_abort = 0;
  unsigned char* mine = peers[me];
  uint32_t* flags = reinterpret_cast<uint32_t*>(mine + xl.flags);
  uint32_t* steps = reinterpret_cast<uint32_t*>(mine + xl.steps);
  const float* data = reinterpret_cast<const float*>(mine + xl.data);

  // phase A: merge the local splits of each of this CTA's rows and publish
  // them to every rank
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const int b = r / H;
    const int len = lens[b];
    if (threadIdx.x == 0 && (len < 0 || len > row_limit)) set_dev_error(B2A_ERR_POSITION, b);
    const int ns = (len <= 0) ? 0 : min(n_splits, (len + split_rows - 1) / split_rows);
    if (threadIdx.x == 0) s_step = steps[r];
    const float lse = merge_splits(part_o, part_ml, r, ns, n_splits, D, wsm, obuf);
    const uint32_t step = s_step;
    const int parity = static_cast<int>(step & 1u);
    for (int g = 0; g < G; ++g) {
      float* dst = reinterpret_cast<float*>(peers[g] + xl.data) + data_index(parity, me, r, R, G, D);
      for (int d = threadIdx.x; d < D; d += kThreads) dst[d] = obuf[d];
      if (threadIdx.x == 0) dst[D] = lse;
    }
    // every thread's peer stores become visible system-wide before the
    // flags that announce them
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < G) {
      uint32_t* f = reinterpret_cast<uint32_t*>(peers[threadIdx.x] + xl.flags) +
                    static_cast<size_t>(me) * R + r;
      st_release_sys(f, step + 1u);
    }
    __syncthreads();  // obuf / wsm reused by the next row
  }

  // phase B: wait for every rank's part of each row, then merge
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    if (threadIdx.x == 0) s_step = steps[r];
    __syncthreads();
    const uint32_t step = s_step;
    const int parity = static_cast<int>(step & 1u);
    if (threadIdx.x < G && !s_abort) {
      const uint32_t* f = flags + static_cast<size_t>(threadIdx.x) * R + r;
      if (static_cast<int>(ld_acquire_sys(f) - (step + 1u)) < 0) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (static_cast<int>(ld_acquire_sys(f) - (step + 1u)) < 0) {
          if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kShardWaitNs) {
            set_dev_error(B2A_ERR_TIMEOUT, 0x50000 | threadIdx.x);
            s_abort = 1;
            break;
          }
        }
      }
    }
    __syncthreads();
    // lse of every part, read through L2 (the slots are rewritten by peers)
    float M = -INFINITY;
    for (int g = 0; g < G; ++g)
      M = fmaxf(M, __ldcg(data + data_index(parity, g, r, R, G, D) + D));
    const float Mref = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    for (int g = 0; g < G; ++g) L += expf(__ldcg(data + data_index(parity, g, r, R, G, D) + D) - Mref);
    const float invL = (L > 0.f) ? 1.f / L : 0.f;
    for (int d = threadIdx.x; d < D; d += kThreads) {
      float acc = 0.f;
      for (int g = 0; g < G; ++g) {
        const float* src = data + data_index(parity, g, r, R, G, D);
        acc += expf(__ldcg(src + D) - Mref) * __ldcg(src + d);
      }
      out[static_cast<size_t>(r) * D + d] = acc * invL;
    }
    if (threadIdx.x == 0) {
      if (lse_out) lse_out[r] = (L > 0.f) ? Mref + logf(L) : -INFINITY;
      steps[r] = step + 1u;
    }
    __syncthreads();
  }
}

}  // namespace shard
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

typedef CUresult (*PFN_memGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_memGetAddressRange address_range_fn() {
  static PFN_memGetAddressRange fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_memGetAddressRange>(p);
  });
  return fn;
}

}  // namespace

extern "C" {

size_t b2a_shard_exchange_bytes(int B, int H, int D, int G) {
  if (B <= 0 || H <= 0 || D <= 0 || G <= 0) return 0;
  return b2a::shard::xlayout(B * H, D, G).total;
}

int b2a_ipc_handle(const void* dev_ptr, void* handle_out, long long* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return fail(B2A_ERR_ARG, "ipc_handle: null argument");
  PFN_memGetAddressRange fn = address_range_fn();
  if (!fn) return fail(B2A_ERR_CUDA, "ipc_handle: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS) return fail(B2A_ERR_ARG, "ipc_handle: cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "ipc_handle: cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<long long>(reinterpret_cast<uintptr_t>(dev_ptr) - base);
  return B2A_OK;
}

int b2a_ipc_open(const void* handle, long long offset, void** base_out, void** ptr_out) {
  if (!handle || !base_out || !ptr_out || offset < 0) return fail(B2A_ERR_ARG, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "ipc_open: cudaIpcOpenMemHandle");
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return B2A_OK;
}

int b2a_ipc_close(void* base) {
  if (!base) return fail(B2A_ERR_ARG, "ipc_close: null base");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "ipc_close: cudaIpcCloseMemHandle");
  return B2A_OK;
}

int b2a_decode_sharded(const float* q, const void* k_shard, const void* v_shard,
                       const int* lens_dev, float* out, float* lse_out, void* workspace,
                       size_t workspace_bytes, int B, int H, int KV, int D, int n_ctx,
                       long long seq_stride, int kv_dtype, float scale, int max_len,
                       int split_rows, void* const* peer_xbufs_dev, int rank, int G,
                       void* stream) {
  if (!peer_xbufs_dev) return fail(B2A_ERR_ARG, "decode_sharded: null peer buffer table");
  if (G <= 0 || rank < 0 || rank >= G) return fail(B2A_ERR_ARG, "decode_sharded: rank %d of %d", rank, G);
  if (G > b2a::shard::kThreads) return fail(B2A_ERR_UNSUPPORTED, "decode_sharded: %d ranks > %d", G, b2a::shard::kThreads);
  if (D > 1024) return fail(B2A_ERR_UNSUPPORTED, "decode_sharded: head_dim %d", D);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int ns = 0;
  float *part_o = nullptr, *part_ml = nullptr;
  int rc = decode_split_phase(q, k_shard, v_shard, lens_dev, out, workspace, workspace_bytes, B,
                              H, KV, D, n_ctx, seq_stride, kv_dtype, scale, max_len, &split_rows,
                              &ns, &part_o, &part_ml, st);
  if (rc) return rc;
  namespace S = b2a::shard;
  auto kern = S::shard_exchange_kernel;
  const int smem = (ns + D) * static_cast<int>(sizeof(float));
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, S::kThreads, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_sharded: occupancy");
  if (occ < 1) return fail(B2A_ERR_UNSUPPORTED, "decode_sharded: exchange kernel cannot be resident");
  const int R = B * H;
  const int resident = occ * b2a_host::sm_count();
  const int grid = R < resident ? R : resident;  // every CTA resident: the waits cannot starve
  kern<<<grid, S::kThreads, smem, st>>>(
      part_o, part_ml, lens_dev, out, lse_out,
      reinterpret_cast<unsigned char* const*>(peer_xbufs_dev), rank, G, R, H, D, split_rows, ns,
      max_len);
  e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_sharded launch");
  return B2A_OK;
}

}  // extern "C"
