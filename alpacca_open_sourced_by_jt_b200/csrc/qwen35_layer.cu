// The device half of a Qwen35 full-attention layer, around the decode and
// prefill kernels (alpaccaroo/qwen35_runtime.py:597-664; the reference's
// device-graph version is qwen35_cuda_graph.py:781-851 with the kernels
// split_query_gate, rms_norm, imrope, kv_append and sigmoid_gate of
// qwen35_cuda.py:907-1008):
//
//   b2a_qwen35_attn_prep   one CTA per (token, q or KV head): split the
//                          interleaved [query | gate] rows, RMSNorm the head,
//                          IMROPE it, and write q (to q_out) or k (into the
//                          cache at the token's position, with v beside it);
//   b2a_sigmoid_gate       out = attended * sigmoid(gate), reading the gate
//                          halves of the interleaved rows in place.
//
// Numerics follow the reference's semantic runtime, which computes in double
// and rounds to f32 at fixed boundaries: the RMSNorm is evaluated in double
// relative to max(|x|, sqrt(eps)) (qwen35_ops.py:46-75) and rounded to f32;
// IMROPE is the same double rotation as b2a_imrope_append; the gate is
// double and rounded once (tensor.py:123-129).

namespace b2a {
namespace qwen35 {

constexpr int kMaxD = 256;
constexpr int kMaxThreads = 128;

// Block-wide reductions over <= 128 threads (4 warps).
__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  double r = red[0];
  for (int i = 1; i < nw; ++i) r += red[i];
  __syncthreads();
  return r;
}

template <typename TK, typename TQ>
__global__ void __launch_bounds__(kMaxThreads) prep_kernel(
    const float* __restrict__ query_gate, long long qg_tok_stride, const float* __restrict__ key,
    long long k_tok_stride, const float* __restrict__ value, long long v_tok_stride,
    const float* __restrict__ q_norm, const float* __restrict__ k_norm, double eps,
    const int* __restrict__ lanes, const __grid_constant__ rope::ImropeParams prm,
    double freq_scale, const int* __restrict__ pos, int tok_seq_mode, TK* __restrict__ k_cache,
    TK* __restrict__ v_cache, long long seq_stride, int n_ctx, TQ* __restrict__ q_out, int H,
    int KV, int D) {
  __shared__ float xs[kMaxD];   // the head, then its normalised values
  __shared__ float fred[4];
  __shared__ double dred[4];
  const int i = blockIdx.x;
  const int slot = blockIdx.y;
  const int p = pos[i];
  if (p < 0 || p >= n_ctx) {
    if (threadIdx.x == 0 && slot == 0) set_dev_error(B2A_ERR_POSITION, i);
    return;
  }
  const bool is_q = slot < H;
  const int head = is_q ? slot : slot - H;
  const float* src = is_q ? query_gate + i * qg_tok_stride + static_cast<long long>(head) * 2 * D
                          : key + i * k_tok_stride + static_cast<long long>(head) * D;
  const float* w = is_q ? q_norm : k_norm;
  const size_t seq = tok_seq_mode ? static_cast<size_t>(i) : 0;
  TK* krow = k_cache + seq * seq_stride + (static_cast<size_t>(p) * KV + head) * D;
  TK* vrow = v_cache + seq * seq_stride + (static_cast<size_t>(p) * KV + head) * D;

  // RMSNorm in double relative to s = max(sqrt(eps), max|x|)
  float amax = 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const float x = src[c];
    xs[c] = x;
    amax = fmaxf(amax, fabsf(x));
    if (!is_q) st_elem(vrow + c, value[i * v_tok_stride + static_cast<long long>(head) * D + c]);
  }
  const double root = sqrt(eps);
  const double s = fmax(root, static_cast<double>(block_max(amax, fred)));
  double part = 0.0;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const double u = __ddiv_rn(static_cast<double>(xs[c]), s);
    part = __dadd_rn(part, __dmul_rn(u, u));  // rounded squares, as the reference sums
  }
  const double msq = __ddiv_rn(block_sum(part, dred), static_cast<double>(D));
  const double re = __ddiv_rn(root, s);
  const double den = __dsqrt_rn(__dadd_rn(msq, __dmul_rn(re, re)));
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const double u = __ddiv_rn(static_cast<double>(xs[c]), s);
    xs[c] = static_cast<float>(__dmul_rn(__ddiv_rn(u, den), static_cast<double>(w[c])));
  }
  __syncthreads();

  // IMROPE: pair t < P rotates dims (t, t + P); the dims past 2P pass through
  const int P = prm.pairs;
  const int* ln = lanes + 4 * i;
  for (int t = threadIdx.x; t < (D >> 1); t += blockDim.x) {
    int a, b;
    float y0, y1;
    if (t < P) {
      a = t;
      b = t + P;
      const double theta =
          __dmul_rn(__dmul_rn(static_cast<double>(ln[prm.lane[t]]), freq_scale), prm.pw[t]);
      double sn, cs;
      sincos(theta, &sn, &cs);
      const double x0 = xs[a], x1 = xs[b];
      y0 = static_cast<float>(__dsub_rn(__dmul_rn(x0, cs), __dmul_rn(x1, sn)));
      y1 = static_cast<float>(__dadd_rn(__dmul_rn(x0, sn), __dmul_rn(x1, cs)));
    } else {
      a = 2 * P + 2 * (t - P);
      b = a + 1;
      if (a >= D) continue;
      y0 = xs[a];
      y1 = xs[b];
    }
    if (is_q) {
      TQ* qo = q_out + (static_cast<size_t>(i) * H + head) * D;
      st_elem(qo + a, y0);
      st_elem(qo + b, y1);
    } else {
      st_elem(krow + a, y0);
      st_elem(krow + b, y1);
    }
  }
}

__global__ void sigmoid_gate_kernel(const float* __restrict__ values, long long vs,
                                    const float* __restrict__ gates, long long gs,
                                    float* __restrict__ out, long long os, int rows, int width) {
  const long long n = static_cast<long long>(rows) * width;
  for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / width, c = e - r * width;
    const double g = gates[r * gs + c];
    double sg;
    if (g >= 0.0) {
      sg = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-g)));
    } else {
      const double z = exp(g);
      sg = __ddiv_rn(z, __dadd_rn(1.0, z));
    }
    out[r * os + c] = static_cast<float>(__dmul_rn(static_cast<double>(values[r * vs + c]), sg));
  }
}

}  // namespace qwen35
}  // namespace b2a

namespace {

template <typename TK, typename TQ>
void launch_prep(dim3 grid, int threads, cudaStream_t st, const float* qg, long long qgs,
                 const float* k, long long ks, const float* v, long long vs, const float* qn,
                 const float* kn, double eps, const int* lanes, const b2a::rope::ImropeParams& prm,
                 double fscale, const int* pos, int mode, void* kc, void* vc, long long seq_stride,
                 int n_ctx, void* q_out, int H, int KV, int D) {
  b2a::qwen35::prep_kernel<TK, TQ><<<grid, threads, 0, st>>>(
      qg, qgs, k, ks, v, vs, qn, kn, eps, lanes, prm, fscale, pos, mode, static_cast<TK*>(kc),
      static_cast<TK*>(vc), seq_stride, n_ctx, static_cast<TQ*>(q_out), H, KV, D);
}

template <typename TK>
int prep_qdt(int q_dtype, dim3 grid, int threads, cudaStream_t st, const float* qg,
             long long qgs, const float* k, long long ks, const float* v, long long vs,
             const float* qn, const float* kn, double eps, const int* lanes,
             const b2a::rope::ImropeParams& prm, double fscale, const int* pos, int mode, void* kc,
             void* vc, long long seq_stride, int n_ctx, void* q_out, int H, int KV, int D) {
  switch (q_dtype) {
    case B2A_F32:
      launch_prep<TK, float>(grid, threads, st, qg, qgs, k, ks, v, vs, qn, kn, eps, lanes, prm,
                             fscale, pos, mode, kc, vc, seq_stride, n_ctx, q_out, H, KV, D);
      return B2A_OK;
    case B2A_F16:
      launch_prep<TK, __half>(grid, threads, st, qg, qgs, k, ks, v, vs, qn, kn, eps, lanes, prm,
                              fscale, pos, mode, kc, vc, seq_stride, n_ctx, q_out, H, KV, D);
      return B2A_OK;
    case B2A_BF16:
      launch_prep<TK, __nv_bfloat16>(grid, threads, st, qg, qgs, k, ks, v, vs, qn, kn, eps, lanes,
                                     prm, fscale, pos, mode, kc, vc, seq_stride, n_ctx, q_out, H,
                                     KV, D);
      return B2A_OK;
  }
  return b2a_host::fail(B2A_ERR_DTYPE, "qwen35_attn_prep: q_out_dtype %d", q_dtype);
}

}  // namespace

extern "C" {

int b2a_qwen35_attn_prep(const float* query_gate, long long qg_tok_stride, const float* key,
                         long long k_tok_stride, const float* value, long long v_tok_stride,
                         const float* q_norm, const float* k_norm, double epsilon,
                         const int* lanes_dev, const int* sections, double freq_base,
                         double freq_scale, const int* pos_dev, int tok_seq_mode, void* k_cache,
                         void* v_cache, long long seq_stride, int n_ctx, int kv_dtype,
                         void* q_out, int q_out_dtype, int n_tok, int H, int KV, int D,
                         void* stream) {
  using b2a_host::fail;
  int rc = check_common(query_gate, key, value, pos_dev, k_cache, v_cache, n_tok, H, KV, D,
                        n_ctx, seq_stride, tok_seq_mode, "qwen35_attn_prep");
  if (rc) return rc;
  if (KV <= 0 || H % KV) return fail(B2A_ERR_SHAPE, "qwen35_attn_prep: H %d not a multiple of KV %d", H, KV);
  if (!q_norm || !k_norm || !lanes_dev || !sections || !q_out)
    return fail(B2A_ERR_ARG, "qwen35_attn_prep: null pointer argument");
  if ((D & 1) || D > b2a::qwen35::kMaxD)
    return fail(B2A_ERR_SHAPE, "qwen35_attn_prep: head_dim %d must be even and <= 256", D);
  if (!(epsilon > 0.0) || !isfinite(epsilon))
    return fail(B2A_ERR_ARG, "qwen35_attn_prep: epsilon must be positive and finite");
  for (int i = 0; i < 4; ++i)
    if (sections[i] < 0) return fail(B2A_ERR_ARG, "qwen35_attn_prep: negative section");
  const int P = sections[0] + sections[1] + sections[2] + sections[3];
  if (P <= 0) return fail(B2A_ERR_ARG, "qwen35_attn_prep: at least one section must be nonzero");
  if (2 * P > D || P > kMaxPairs)
    return fail(B2A_ERR_SHAPE, "qwen35_attn_prep: 2*sum(sections)=%d exceeds head_dim %d", 2 * P, D);
  if (!(freq_base > 0.0) || !isfinite(freq_base) || !(freq_scale > 0.0) || !isfinite(freq_scale))
    return fail(B2A_ERR_ARG, "qwen35_attn_prep: frequency base/scale must be positive and finite");
  ImropeParams prm;
  prm.pairs = P;
  for (int j = 0; j < P; ++j) {
    prm.pw[j] = pow(freq_base, -2.0 * j / (2.0 * P));
    prm.lane[j] = static_cast<signed char>(imrope_lane(j, sections));
  }
  if (n_tok == 0) return B2A_OK;
  dim3 grid(n_tok, H + KV);
  int threads = ((D / 2 + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  if (threads > b2a::qwen35::kMaxThreads) threads = b2a::qwen35::kMaxThreads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (kv_dtype) {
    case B2A_F32:
      rc = prep_qdt<float>(q_out_dtype, grid, threads, st, query_gate, qg_tok_stride, key,
                           k_tok_stride, value, v_tok_stride, q_norm, k_norm, epsilon, lanes_dev,
                           prm, freq_scale, pos_dev, tok_seq_mode, k_cache, v_cache, seq_stride,
                           n_ctx, q_out, H, KV, D);
      break;
    case B2A_F16:
      rc = prep_qdt<__half>(q_out_dtype, grid, threads, st, query_gate, qg_tok_stride, key,
                            k_tok_stride, value, v_tok_stride, q_norm, k_norm, epsilon, lanes_dev,
                            prm, freq_scale, pos_dev, tok_seq_mode, k_cache, v_cache, seq_stride,
                            n_ctx, q_out, H, KV, D);
      break;
    case B2A_BF16:
      rc = prep_qdt<__nv_bfloat16>(q_out_dtype, grid, threads, st, query_gate, qg_tok_stride,
                                   key, k_tok_stride, value, v_tok_stride, q_norm, k_norm, epsilon,
                                   lanes_dev, prm, freq_scale, pos_dev, tok_seq_mode, k_cache,
                                   v_cache, seq_stride, n_ctx, q_out, H, KV, D);
      break;
    default:
      return fail(B2A_ERR_DTYPE, "qwen35_attn_prep: kv_dtype %d", kv_dtype);
  }
  if (rc) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "qwen35_attn_prep launch");
  return B2A_OK;
}

int b2a_sigmoid_gate(const float* values, long long value_row_stride, const float* gates,
                     long long gate_row_stride, float* out, long long out_row_stride, int rows,
                     int width, void* stream) {
  using b2a_host::fail;
  if (!values || !gates || !out) return fail(B2A_ERR_ARG, "sigmoid_gate: null pointer argument");
  if (rows < 0 || width <= 0) return fail(B2A_ERR_ARG, "sigmoid_gate: bad sizes");
  if (value_row_stride < width || gate_row_stride < width || out_row_stride < width)
    return fail(B2A_ERR_SHAPE, "sigmoid_gate: row strides must be >= width");
  if (rows == 0) return B2A_OK;
  const long long n = static_cast<long long>(rows) * width;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  b2a::qwen35::sigmoid_gate_kernel<<<static_cast<int>(blocks), 256, 0,
                                     static_cast<cudaStream_t>(stream)>>>(
      values, value_row_stride, gates, gate_row_stride, out, out_row_stride, rows, width);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "sigmoid_gate launch");
  return B2A_OK;
}

}  // extern "C"
