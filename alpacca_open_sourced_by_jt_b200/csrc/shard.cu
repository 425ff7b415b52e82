// Long-context decode with the KV rows sharded across GPUs: the split-KV
// combine, the exchange of every rank's partial result over NVLink and the
// cross-rank log-sum-exp merge as ONE kernel over peer memory.
//
// Each rank holds a contiguous range of every sequence's cache rows and
// runs the decode split kernel over it (decode.cu).  Then, per output row r
// (one (sequence, query head) pair):
//   phase A  merge this rank's split partials into (o_r, lse_r) (the
//            algebra of the reference's _attention_decode_combine,
//            alpaccaroo/cuda.py:674-694) and store them into slot [me] of
//            EVERY rank's exchange buffer through the CUDA-IPC mappings
//            (NVLink peer stores; no TMA, no multicast);
//   phase B  read every rank's slot of row r from this rank's own buffer and
//            merge the G parts by their lse:
//              out_r = sum_g exp(lse_g - L) o_g,  L = log sum_g exp(lse_g)
// so every rank ends with the merged rows, the result of an all-gather
// followed by the combine, without a separate collective or launch.
//
// No fences and no separate flags: every value travels in an 8-byte word
// (f32 value, u32 tag) written by one 8-byte store, and the tag is the
// step number + 1, so a reader that sees the tag it expects sees the value
// with it (an aligned 8-byte store is not split).  A reader spins on each
// word until its tag arrives, bounded by kShardWaitNs (on expiry it records
// B2A_ERR_TIMEOUT and merges what it has).
//
// Exchange buffer of each rank (b2a_shard_exchange_bytes, zeroed once
// before first use): words [2][G][R][D+1] (step parity, source rank, row,
// o then lse) and steps [R] u32 (this rank's count of finished steps per
// row).  Double buffering by step parity is enough: a rank writes step n+2
// into a slot only after its step n+1 read every rank's step n+1 words,
// which each rank writes only after its step n kernel (the last reader of
// the slot) has completed on its stream.  Tags grow by one per step, so a
// word left from step n in the same slot never passes for step n+2.
// Rows are independent, so ranks may use different grids.
//
// The grid never exceeds the number of CTAs that can be resident at once,
// and every CTA writes all of its rows (phase A) before it waits in phase
// B, so the waits cannot block a CTA that has yet to write.

#include "shard_words.cuh"

namespace b2a {
namespace shard {

constexpr int kThreads = 128;
// Limit of a phase-B wait: far above any skew between ranks that step
// together, short enough that a rank that never arrives surfaces as
// B2A_ERR_TIMEOUT (the kernel then merges what it has and returns).
constexpr uint64_t kShardWaitNs = 2000000000ull;

// Spin until the word carries `tag`; returns its value.  *deadline_hit is
// set (and the error recorded once) when the wait runs past t_end.
__device__ __forceinline__ float wait_tagged(const uint2* p, uint32_t tag, uint64_t t_end,
                                             bool* deadline_hit) {
  uint2 w = ld_tagged(p);
  if (w.y == tag) return __uint_as_float(w.x);
  uint32_t spins = 0;
  while (!*deadline_hit) {
    w = ld_tagged(p);
    if (w.y == tag) return __uint_as_float(w.x);
    if ((++spins & 63u) == 0u && globaltimer_ns() > t_end) {
      set_dev_error(B2A_ERR_TIMEOUT, 0x50000);
      *deadline_hit = true;
    }
  }
  return __uint_as_float(w.x);
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
    int split_rows, int n_splits, int row_limit, int publish_all) {
  // publish_all: the split kernel did not publish (fp32 caches, or no rows
  // at all), so this kernel merges and publishes every row and must first
  // wait for the split partials.  Otherwise it publishes only the rows of
  // sequences with no local rows (no split CTA ran for them) and starts
  // while the split kernel's last CTAs are still publishing.
  if (publish_all) pdl_wait();
  extern __shared__ float ssm[];
  float* wsm = ssm;                 // [n_splits] split weights
  float* obuf = ssm + n_splits;     // [D] this rank's merged row
  __shared__ uint32_t s_step;
  const XLayout xl = xlayout(R, D, G);
  unsigned char* mine = peers[me];
  uint32_t* steps = reinterpret_cast<uint32_t*>(mine + xl.steps);
  const uint2* words = reinterpret_cast<const uint2*>(mine + xl.words);

  // phase A: merge the local splits of each of this CTA's rows and store
  // them, tagged, into every rank's buffer
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const int b = r / H;
    const int len = lens[b];
    if (threadIdx.x == 0 && (len < 0 || len > row_limit)) set_dev_error(B2A_ERR_POSITION, b);
    if (!publish_all && len > 0) continue;  // the split kernel published this row
    const int ns = (len <= 0) ? 0 : min(n_splits, (len + split_rows - 1) / split_rows);
    if (threadIdx.x == 0) s_step = steps[r];
    const float lse = merge_splits(part_o, part_ml, r, ns, n_splits, D, wsm, obuf);
    const uint32_t step = s_step;
    const uint32_t tag = step + 1u;
    const int parity = static_cast<int>(step & 1u);
    for (int g = 0; g < G; ++g) {
      uint2* dst = reinterpret_cast<uint2*>(peers[g] + xl.words) +
                   word_index(parity, me, r, R, G, D);
      for (int d = threadIdx.x; d <= D; d += kThreads) st_tagged(dst + d, d < D ? obuf[d] : lse, tag);
    }
    __syncthreads();  // obuf / wsm / s_step reused by the next row
  }

  // phase B: every rank's part of each row, then the merge
  const uint64_t t_end = globaltimer_ns() + kShardWaitNs;
  bool hit = false;  // this thread's waits ran out: it stops waiting
  // Latency-bound: the G lse words of a row are waited for by G threads at
  // once and shared; each value thread then issues its G loads in batches
  // of 8 before it checks their tags (and spins only on a late one).
  __shared__ float s_gl[kThreads];  // each rank's lse of the current row (G <= kThreads)
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const uint32_t step = steps[r];
    const uint32_t tag = step + 1u;
    const int parity = static_cast<int>(step & 1u);
    if (threadIdx.x < G)
      s_gl[threadIdx.x] =
          wait_tagged(words + word_index(parity, threadIdx.x, r, R, G, D) + D, tag, t_end, &hit);
    __syncthreads();
    float M = -INFINITY;
    for (int g = 0; g < G; ++g) M = fmaxf(M, s_gl[g]);
    const float Mref = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    for (int g = 0; g < G; ++g) L += expf(s_gl[g] - Mref);
    const float invL = (L > 0.f) ? 1.f / L : 0.f;
    for (int d = threadIdx.x; d < D; d += kThreads) {
      float acc = 0.f;
      for (int g0 = 0; g0 < G; g0 += 8) {
        const int gn = min(8, G - g0);
        uint2 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < gn) w[i] = ld_tagged(words + word_index(parity, g0 + i, r, R, G, D) + d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i < gn) {
            const float v = (w[i].y == tag) ? __uint_as_float(w[i].x)
                                            : wait_tagged(words + word_index(parity, g0 + i, r, R,
                                                                             G, D) + d,
                                                          tag, t_end, &hit);
            acc += expf(s_gl[g0 + i] - Mref) * v;
          }
        }
      }
      out[static_cast<size_t>(r) * D + d] = acc * invL;
    }
    __syncthreads();  // every thread read steps[r] before it moves on
    if (threadIdx.x == 0) {
      if (lse_out) lse_out[r] = (L > 0.f) ? Mref + logf(L) : -INFINITY;
      steps[r] = tag;
    }
  }
  // finish no earlier than the split kernel (a no-op for an ordinary launch)
  pdl_wait();
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
  bool published = false;
  const b2a::shard::Publish pub{reinterpret_cast<unsigned char* const*>(peer_xbufs_dev), rank, G};
  int rc = decode_split_phase(q, k_shard, v_shard, lens_dev, out, workspace, workspace_bytes, B,
                              H, KV, D, n_ctx, seq_stride, kv_dtype, scale, max_len, &split_rows,
                              &ns, &part_o, &part_ml, st, pub, &published);
  if (rc) return rc;
  namespace S = b2a::shard;
  auto kern = S::shard_exchange_kernel;
  const int smem = (ns + D) * static_cast<int>(sizeof(float));
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, S::kThreads, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_sharded: occupancy");
  if (occ < 1) return fail(B2A_ERR_UNSUPPORTED, "decode_sharded: exchange kernel cannot be resident");
  const int R = B * H;
  // at most one CTA per SM, never more than can be resident at once, so the
  // waits cannot starve a CTA that has yet to write its rows
  const int sms = b2a_host::sm_count();
  const int resident = occ * sms;
  int grid = R < sms ? R : sms;
  if (grid > resident) grid = resident;
  // a programmatic dependent of the split kernel: its CTAs are resident and
  // reading the exchange words while the last split CTAs publish
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(S::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<const float*>(part_o),
                         static_cast<const float*>(part_ml), lens_dev, out, lse_out,
                         reinterpret_cast<unsigned char* const*>(peer_xbufs_dev), rank, G, R, H,
                         D, split_rows, ns, max_len, published ? 0 : 1);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_sharded launch");
  return B2A_OK;
}

}  // extern "C"
