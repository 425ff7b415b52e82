// Causal flash prefill in fp32 on the CUDA cores: the exact-precision path
// for fp32 callers.
//
// The reference's batched attention is fp32 end to end: the NumPy einsum of
// Model._attention_batch_np (alpaccaroo/model.py:1254-1272), its window
// variant _attention_batch_window_np (model.py:1567-1592) and the SIMT
// kernel behind cuda.attention_batch (cuda.py:424-578).  Routing fp32 inputs
// through the tcgen05 kernels would round q, K, V and P to 16 bits (about
// 1e-3 relative error); this kernel keeps every operand and every product in
// fp32, so it answers within fp32 rounding of the NumPy path.
//
// Semantics (the NumPy path's, including its corner case): key s (absolute
// position kv_start + s) is visible to query t iff kv_start + s <= pos[t]
// and, when window > 0, kv_start + s > pos[t] - window.  A query row with no
// visible key gets the mean of all t_kv value rows: the NumPy path masks
// with -1e30, so every weight of such a row is exp(0) / t_kv.
//
// One CTA per (64-query tile, query head), 256 threads as a 16 x 16 grid
// (ty, tx).  Per 64-key tile:
//   scores  S[4][4]: rows ty*4 + i, keys tx + 16*j; Q and K rows staged in
//           shared memory (row stride D+4 floats, so the 16 key rows a warp
//           reads at one offset fall on distinct banks), 8 LDS.128 per 64 FMA
//   softmax online, in log2 units; a row's 64 scores live on the 16 threads
//           of one half-warp, reduced with xor shuffles over lane bits 0-3
//   PV      O[4][D/16]: rows ty*4 + i, columns tx*4 + 64*k; P^T staged in
//           shared memory over the consumed K tile
// Positions may come in any order: the tile's key range is taken from the
// minimum and maximum position of its rows.

namespace b2a {
namespace prefill_f32 {

constexpr int kBQ = 64;
constexpr int kBK = 64;
constexpr int kThreads = 256;

template <int DP>  // head_dim rounded up to 64, 128 or 256 (zero padded)
struct Layout {
  static constexpr int kLd = DP + 4;   // row stride of the Q, K and V tiles (floats)
  static constexpr int kLdP = kBQ + 4; // row stride of P^T [key][query row]
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kBQ * kLd;  // P^T reuses this tile once S is formed
  static constexpr int kV = kK + kBK * kLd;
  static constexpr int kFloats = kV + kBK * kLd;
  static constexpr int kBytes = kFloats * 4;
  static_assert(kBK * kLdP <= kBK * kLd, "P^T must fit in the K tile");
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const uint32_t d = smem_u32(dst);
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Rows [row0, row0 + 64) of a [rows][heads][D] f32 tensor, head `head`, into
// a [64][kLd] shared tile; columns D..DP-1 and rows at or past n_rows are
// zero.
template <int DP>
__device__ __forceinline__ void stage_rows(float* dst, const float* __restrict__ src, int row0,
                                           int n_rows, int heads, int head, int D) {
  constexpr int kVec = DP / 4;
  const int d4 = D / 4;
  for (int i = threadIdx.x; i < 64 * kVec; i += kThreads) {
    const int r = i / kVec, c4 = i - r * kVec;
    const int row = row0 + r;
    const bool valid = row < n_rows && c4 < d4;
    const float* p = valid ? src + (static_cast<size_t>(row) * heads + head) * D + c4 * 4 : src;
    cp_async16(dst + r * Layout<DP>::kLd + c4 * 4, p, valid);
  }
}

template <typename TO>
__device__ __forceinline__ void store4(TO* dst, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float* dst, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float a, float b, float c, float d) {
  __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = u;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float a, float b,
                                                      float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = u;
}

template <typename TO, int DP>
__global__ void __launch_bounds__(kThreads) prefill_f32_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const int* __restrict__ pos, TO* __restrict__ out, int n_q, int t_kv, int H, int KV, int D,
    int group, int n_q_tiles, float sscale, int window, int kv_start) {
  using L = Layout<DP>;
  constexpr int NK = DP / 64;  // 4-column groups per thread in the PV phase
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* sQ = sm + L::kQ;
  float* sK = sm + L::kK;
  float* sP = sm + L::kK;  // P^T [key][row], over the K tile once S is formed
  float* sV = sm + L::kV;
  __shared__ int s_pmin, s_pmax;

  const int qt = n_q_tiles - 1 - static_cast<int>(blockIdx.x);  // heaviest tiles first
  const int h = blockIdx.y, kvh = h / group;
  const int row0 = qt * kBQ;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

  if (tid == 0) {
    s_pmin = INT_MAX;
    s_pmax = INT_MIN;
  }
  __syncthreads();
  if (tid < kBQ && row0 + tid < n_q) {
    const int p = pos[row0 + tid];
    atomicMin(&s_pmin, p);
    atomicMax(&s_pmax, p);
  }
  stage_rows<DP>(sQ, q, row0, n_q, H, h, D);
  cp_async_commit();
  __syncthreads();

  // key tiles [j0, j_end) hold every key visible to some row of this tile
  int j0 = 0, j_end = 0;
  {
    const long long hi = min(static_cast<long long>(s_pmax) - kv_start + 1, static_cast<long long>(t_kv));
    j_end = hi <= 0 ? 0 : static_cast<int>((hi + kBK - 1) / kBK);
    if (window > 0) {
      const long long lo = static_cast<long long>(s_pmin) - window + 1 - kv_start;
      if (lo > 0) j0 = static_cast<int>(min(lo / kBK, static_cast<long long>(j_end)));
    }
  }

  long long my_pos[4];
  bool row_ok[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = row0 + ty * 4 + i;
    row_ok[i] = t < n_q;
    my_pos[i] = row_ok[i] ? static_cast<long long>(pos[t]) : LLONG_MIN;
  }

  float o[4][NK][4];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int kk = 0; kk < NK; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[i][kk][e] = 0.f;
  }

  for (int j = j0; j < j_end; ++j) {
    stage_rows<DP>(sK, k, j * kBK, t_kv, KV, kvh, D);
    cp_async_commit();
    stage_rows<DP>(sV, v, j * kBK, t_kv, KV, kvh, D);
    cp_async_commit();
    cp_async_wait<1>();  // Q (first tile) and K have landed; V may still be in flight
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) s[i][jj] = 0.f;
#pragma unroll 4
    for (int d = 0; d < DP; d += 4) {
      float4 qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(sQ + (ty * 4 + i) * L::kLd + d);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) kb[jj] = *reinterpret_cast<const float4*>(sK + (tx + 16 * jj) * L::kLd + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          s[i][jj] = fmaf(qa[i].x, kb[jj].x, s[i][jj]);
          s[i][jj] = fmaf(qa[i].y, kb[jj].y, s[i][jj]);
          s[i][jj] = fmaf(qa[i].z, kb[jj].z, s[i][jj]);
          s[i][jj] = fmaf(qa[i].w, kb[jj].w, s[i][jj]);
        }
    }

    // mask, online softmax (log2 units)
    const long long kv0 = static_cast<long long>(kv_start) + static_cast<long long>(j) * kBK;
    const long long cmax = static_cast<long long>(t_kv) - static_cast<long long>(j) * kBK - 1;
    float alpha[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const long long hi = min(my_pos[i] - kv0, cmax);
      const long long lo = window > 0 ? my_pos[i] - window + 1 - kv0 : LLONG_MIN;
      float mx = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const long long c = tx + 16 * jj;
        const bool vis = row_ok[i] && c <= hi && c >= lo;
        s[i][jj] = vis ? s[i][jj] * sscale : -INFINITY;
        mx = fmaxf(mx, s[i][jj]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      alpha[i] = (mnew == -INFINITY) ? 1.f : exp2f(m[i] - mnew);
      m[i] = mnew;
      const float mref = (mnew == -INFINITY) ? 0.f : mnew;
      float sum = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        s[i][jj] = exp2f(s[i][jj] - mref);
        sum += s[i][jj];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[i] = l[i] * alpha[i] + sum;
    }
    __syncthreads();  // every thread is done reading the K tile
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
      *reinterpret_cast<float4*>(sP + (tx + 16 * jj) * L::kLdP + ty * 4) =
          make_float4(s[0][jj], s[1][jj], s[2][jj], s[3][jj]);
    cp_async_wait<0>();
    __syncthreads();  // P^T written, V landed

#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int kk = 0; kk < NK; ++kk)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[i][kk][e] *= alpha[i];
#pragma unroll 4
    for (int c = 0; c < kBK; ++c) {
      const float4 pa = *reinterpret_cast<const float4*>(sP + c * L::kLdP + ty * 4);
      const float pr[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
      for (int kk = 0; kk < NK; ++kk) {
        const float4 vb = *reinterpret_cast<const float4*>(sV + c * L::kLd + tx * 4 + 64 * kk);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[i][kk][0] = fmaf(pr[i], vb.x, o[i][kk][0]);
          o[i][kk][1] = fmaf(pr[i], vb.y, o[i][kk][1]);
          o[i][kk][2] = fmaf(pr[i], vb.z, o[i][kk][2]);
          o[i][kk][3] = fmaf(pr[i], vb.w, o[i][kk][3]);
        }
      }
    }
    __syncthreads();  // P^T and V consumed before the next tile overwrites them
  }
  cp_async_wait<0>();  // (no key tile: the Q copy is still outstanding)

  // epilogue
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!row_ok[i]) continue;
    const int t = row0 + ty * 4 + i;
    TO* orow = out + (static_cast<size_t>(t) * H + h) * D;
    if (l[i] > 0.f) {
      const float inv = 1.f / l[i];
#pragma unroll
      for (int kk = 0; kk < NK; ++kk) {
        const int col = tx * 4 + 64 * kk;
        if (col < D)
          store4<TO>(orow + col, o[i][kk][0] * inv, o[i][kk][1] * inv, o[i][kk][2] * inv,
                     o[i][kk][3] * inv);
      }
    } else {
      // no visible key: the NumPy path's uniform weights over all t_kv rows
      const float inv = 1.f / static_cast<float>(t_kv);
#pragma unroll
      for (int kk = 0; kk < NK; ++kk) {
        const int col = tx * 4 + 64 * kk;
        if (col >= D) continue;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int sidx = 0; sidx < t_kv; ++sidx) {
          const float4 vv = *reinterpret_cast<const float4*>(
              v + (static_cast<size_t>(sidx) * KV + kvh) * D + col);
          a0 += vv.x;
          a1 += vv.y;
          a2 += vv.z;
          a3 += vv.w;
        }
        store4<TO>(orow + col, a0 * inv, a1 * inv, a2 * inv, a3 * inv);
      }
    }
  }
}

}  // namespace prefill_f32
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

template <typename TO, int DP>
int launch_prefill_f32_dp(const float* q, const float* k, const float* v, const int* pos,
                          TO* out, int n_q, int t_kv, int H, int KV, int D, float scale,
                          int window, int kv_start, cudaStream_t st) {
  namespace PF = b2a::prefill_f32;
  auto kern = PF::prefill_f32_kernel<TO, DP>;
  constexpr int smem = PF::Layout<DP>::kBytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(prefill_f32)");
  const int n_q_tiles = (n_q + PF::kBQ - 1) / PF::kBQ;
  dim3 grid(n_q_tiles, H);
  kern<<<grid, PF::kThreads, smem, st>>>(q, k, v, pos, out, n_q, t_kv, H, KV, D, H / KV,
                                         n_q_tiles, scale * b2a::prefill::kLog2e, window,
                                         kv_start);
  e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "prefill_f32 launch");
  return B2A_OK;
}

template <typename TO>
int launch_prefill_f32(const float* q, const float* k, const float* v, const int* pos, void* out,
                       int n_q, int t_kv, int H, int KV, int D, float scale, int window,
                       int kv_start, cudaStream_t st) {
  TO* o = static_cast<TO*>(out);
  if (D <= 64)
    return launch_prefill_f32_dp<TO, 64>(q, k, v, pos, o, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
  if (D <= 128)
    return launch_prefill_f32_dp<TO, 128>(q, k, v, pos, o, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
  return launch_prefill_f32_dp<TO, 256>(q, k, v, pos, o, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
}

// fp32 inputs: any head_dim that is a multiple of 4, up to 256.
int prefill_f32_dispatch(int out_dtype, const void* q, const void* k, const void* v,
                         const int* pos, void* out, int n_q, int t_kv, int H, int KV, int D,
                         float scale, int window, int kv_start, cudaStream_t st) {
  if (D % 4 != 0 || D > 256)
    return b2a_host::fail(B2A_ERR_UNSUPPORTED,
                          "prefill: fp32 head_dim %d (a multiple of 4, at most 256)", D);
  const float* qf = static_cast<const float*>(q);
  const float* kf = static_cast<const float*>(k);
  const float* vf = static_cast<const float*>(v);
  switch (out_dtype) {
    case B2A_F32:
      return launch_prefill_f32<float>(qf, kf, vf, pos, out, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
    case B2A_F16:
      return launch_prefill_f32<__half>(qf, kf, vf, pos, out, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
    case B2A_BF16:
      return launch_prefill_f32<__nv_bfloat16>(qf, kf, vf, pos, out, n_q, t_kv, H, KV, D, scale, window, kv_start, st);
  }
  return b2a_host::fail(B2A_ERR_DTYPE, "prefill: out_dtype %d", out_dtype);
}

}  // namespace
