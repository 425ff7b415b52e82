// Fused RoPE + KV-cache append.
//
// One CTA per (token, head slot): bias add, rotation of the token's q heads
// (to q_out or in place) and k heads, pass-through of the dims past n_rot,
// and the k/v rows stored into the cache at the token's absolute position.  Positions
// are read from device memory, so the launch is identical from token to
// token and can live inside a captured CUDA graph.
//
// Conventional rotation (alpaccaroo/model.py:1162-1209, kernels.py:783-816,
// cuda.py:723-786): pair j of a head uses cos_tab[p][j], sin_tab[p][j] from
// the engine's f32 tables and rotates dims (2j, 2j+1) ("norm") or
// (j, j + n_rot/2) ("neox").  Each product and each sum is rounded on its
// own (__fmul_rn/__fsub_rn/__fadd_rn: no FMA contraction), exactly like the
// NumPy elementwise expressions, so fp32 outputs are bit-identical.
//
// IMROPE (qwen35_ops.py:138-215, qwen35_cuda.py:965-998): pair j rotates
// (j, j + P), P = sum(sections), with theta = (lanes[lane(j)] * freq_scale)
// * freq_base^(-2j / 2P) evaluated in double precision; the per-pair power
// and lane index are computed on the host with the same libm pow the
// reference's Python floats use and passed as launch parameters.

#include <math.h>

#include "b2a_common.cuh"

#include <algorithm>

namespace b2a {
namespace rope {

constexpr int kThreads = 256;
constexpr int kMaxPairs = 128;  // head_dim <= 256

// Grid (token, head slot): slots [0, H) are the token's q heads, [H, H+KV)
// its k heads, [H+KV, H+2KV) its v heads.  Thread i of a q/k slot handles
// rotation pair i (i < n_rot/2) or the two pass-through dims
// n_rot + 2(i - n_rot/2), +1; thread i of a v slot copies dims 2i, 2i+1.
template <typename TK, typename TQ>
__global__ void __launch_bounds__(kThreads) rope_append_kernel(
    float* __restrict__ q, long long q_tok_stride, const float* __restrict__ k,
    long long k_tok_stride, const float* __restrict__ v, long long v_tok_stride,
    const float* __restrict__ bq, const float* __restrict__ bk, const float* __restrict__ bv,
    const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int tab_rows,
    const int* __restrict__ pos, int tok_seq_mode, TK* __restrict__ k_cache,
    TK* __restrict__ v_cache, long long seq_stride, int n_ctx, TQ* __restrict__ q_out,
    long long qo_tok_stride, int H, int KV, int D, int n_rot, int neox, int n_tok) {
  // No early launch_dependents: a programmatic dependent (the decode) starts
  // as these short CTAs exit; released at entry it would stream its K/V
  // rows while the GEMV before this kernel still needs the bandwidth.
  pdl_wait();  // q/k/v come from the kernel before (a no-op unless PDL-launched)
  const int i = blockIdx.x * blockDim.y + threadIdx.y;  // blockDim.y tokens per CTA
  const int slot = blockIdx.y;
  if (i >= n_tok) return;
  const int p = pos[i];
  if (p < 0 || p >= n_ctx || p >= tab_rows) {
    if (threadIdx.x == 0 && slot == 0) set_dev_error(B2A_ERR_POSITION, i);
    return;
  }
  const int half = n_rot >> 1;
  const size_t seq = tok_seq_mode ? static_cast<size_t>(i) : 0;
  TK* krow = k_cache + seq * seq_stride + static_cast<size_t>(p) * KV * D;
  TK* vrow = v_cache + seq * seq_stride + static_cast<size_t>(p) * KV * D;
  for (int t = threadIdx.x; t < (D >> 1); t += blockDim.x) {
    if (slot >= H + KV) {  // v row: plain copy (+ bias)
      const int head = slot - H - KV;
      const float* vi = v + i * v_tok_stride + head * D;
      float x0 = vi[2 * t], x1 = vi[2 * t + 1];
      if (bv) {
        x0 = __fadd_rn(x0, bv[head * D + 2 * t]);
        x1 = __fadd_rn(x1, bv[head * D + 2 * t + 1]);
      }
      st_elem(vrow + head * D + 2 * t, x0);
      st_elem(vrow + head * D + 2 * t + 1, x1);
      continue;
    }
    const bool is_q = slot < H;
    const int head = is_q ? slot : slot - H;
    const float* src = is_q ? q + i * q_tok_stride + head * D : k + i * k_tok_stride + head * D;
    const float* bias = is_q ? (bq ? bq + head * D : nullptr) : (bk ? bk + head * D : nullptr);
    int a, b;
    if (t < half) {
      a = neox ? t : 2 * t;
      b = neox ? t + half : 2 * t + 1;
    } else {
      a = n_rot + 2 * (t - half);
      b = a + 1;
    }
    float x0 = src[a], x1 = src[b];
    if (bias) {
      x0 = __fadd_rn(x0, bias[a]);
      x1 = __fadd_rn(x1, bias[b]);
    }
    float y0 = x0, y1 = x1;
    if (t < half) {
      const float c = cos_tab[static_cast<size_t>(p) * half + t];
      const float sn = sin_tab[static_cast<size_t>(p) * half + t];
      y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (is_q) {
      TQ* qo = q_out + i * qo_tok_stride + head * D;  // the q row itself when in place
      st_elem(qo + a, y0);
      st_elem(qo + b, y1);
    } else {
      st_elem(krow + head * D + a, y0);
      st_elem(krow + head * D + b, y1);
    }
  }
}

struct ImropeParams {
  double pw[kMaxPairs];              // freq_base^(-2j / (2P)), host libm pow
  signed char lane[kMaxPairs];       // position lane of pair j
  int pairs;                         // P
};

// Same (token, head slot) grid; thread j of a q/k slot handles IMROPE pair
// j < P (dims j, j + P) or, past P, the pass-through dims 2P + 2(j - P), +1.
template <typename TK, typename TQ>
__global__ void __launch_bounds__(kThreads) imrope_append_kernel(
    const float* __restrict__ q, long long q_tok_stride, const float* __restrict__ k,
    long long k_tok_stride, const float* __restrict__ v, long long v_tok_stride,
    const int* __restrict__ lanes, const __grid_constant__ ImropeParams prm, double freq_scale,
    const int* __restrict__ pos, int tok_seq_mode, TK* __restrict__ k_cache,
    TK* __restrict__ v_cache, long long seq_stride, int n_ctx, TQ* __restrict__ q_out, int H,
    int KV, int D, int n_tok) {
  pdl_wait();  // q/k/v come from the kernel before (a no-op unless PDL-launched)
  const int i = blockIdx.x * blockDim.y + threadIdx.y;  // blockDim.y tokens per CTA
  const int slot = blockIdx.y;
  if (i >= n_tok) return;
  const int p = pos[i];
  if (p < 0 || p >= n_ctx) {
    if (threadIdx.x == 0 && slot == 0) set_dev_error(B2A_ERR_POSITION, i);
    return;
  }
  const int P = prm.pairs;
  const size_t seq = tok_seq_mode ? static_cast<size_t>(i) : 0;
  const int* ln = lanes + 4 * i;
  TK* krow = k_cache + seq * seq_stride + static_cast<size_t>(p) * KV * D;
  TK* vrow = v_cache + seq * seq_stride + static_cast<size_t>(p) * KV * D;
  for (int t = threadIdx.x; t < (D >> 1); t += blockDim.x) {
    if (slot >= H + KV) {
      const int head = slot - H - KV;
      const float* vi = v + i * v_tok_stride + head * D;
      st_elem(vrow + head * D + 2 * t, vi[2 * t]);
      st_elem(vrow + head * D + 2 * t + 1, vi[2 * t + 1]);
      continue;
    }
    const bool is_q = slot < H;
    const int head = is_q ? slot : slot - H;
    const float* src = is_q ? q + i * q_tok_stride + head * D : k + i * k_tok_stride + head * D;
    TQ* qo = q_out + static_cast<size_t>(i) * H * D + head * D;
    if (t < P) {
      const double theta =
          __dmul_rn(__dmul_rn(static_cast<double>(ln[prm.lane[t]]), freq_scale), prm.pw[t]);
      double sn, c;
      sincos(theta, &sn, &c);
      const double x0 = src[t], x1 = src[t + P];
      // separately rounded double products/sums, as Python floats do
      const float y0 = static_cast<float>(__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, sn)));
      const float y1 = static_cast<float>(__dadd_rn(__dmul_rn(x0, sn), __dmul_rn(x1, c)));
      if (is_q) {
        st_elem(qo + t, y0);
        st_elem(qo + t + P, y1);
      } else {
        st_elem(krow + head * D + t, y0);
        st_elem(krow + head * D + t + P, y1);
      }
    } else {
      const int a = 2 * P + 2 * (t - P);
      if (a >= D) continue;
      if (is_q) {
        st_elem(qo + a, src[a]);
        st_elem(qo + a + 1, src[a + 1]);
      } else {
        st_elem(krow + head * D + a, src[a]);
        st_elem(krow + head * D + a + 1, src[a + 1]);
      }
    }
  }
}

}  // namespace rope
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

namespace R = b2a::rope;
using R::ImropeParams;
using R::kMaxPairs;
using R::rope_append_kernel;
using R::imrope_append_kernel;
using b2a_host::fail;

// Threads per (token, head slot) CTA: one per element pair, in whole warps.
int rope_block(int D) {
  const int pairs = D / 2;
  const int t = ((pairs + 31) / 32) * 32;
  return t < R::kThreads ? t : R::kThreads;
}

// IMROPE lane schedule of one rotary pair (qwen35_ops.py:138-156).
int imrope_lane(int pair, const int* sec) {
  const int total = sec[0] + sec[1] + sec[2] + sec[3];
  const int sector = pair % total;
  if (sector % 3 == 1 && sector < 3 * sec[1]) return 1;
  if (sector % 3 == 2 && sector < 3 * sec[2]) return 2;
  if (sector % 3 == 0 && sector < 3 * sec[0]) return 0;
  return 3;
}

template <typename TK, typename TQ>
void launch_rope(dim3 grid, dim3 block, int n_tok, cudaStream_t st, float* q, long long qs,
                 const float* k, long long ks,
                 const float* v, long long vs, const float* bq, const float* bk, const float* bv,
                 const float* ct, const float* stb, int tab_rows, const int* pos, int mode,
                 void* kc, void* vc, long long seq_stride, int n_ctx, void* q_out,
                 long long qos, int H, int KV, int D, int n_rot, int neox) {
  b2a_host::launch(rope_append_kernel<TK, TQ>, grid, block, 0, st, q, qs, k, ks, v, vs, bq, bk,
                   bv, ct, stb, tab_rows, pos, mode, static_cast<TK*>(kc), static_cast<TK*>(vc),
                   seq_stride, n_ctx, static_cast<TQ*>(q_out), qos, H, KV, D, n_rot, neox, n_tok);
}

template <typename TK>
int rope_qdt(int q_dtype, dim3 grid, dim3 block, int n_tok, cudaStream_t st, float* q,
             long long qs, const float* k,
             long long ks, const float* v, long long vs, const float* bq, const float* bk,
             const float* bv, const float* ct, const float* stb, int tab_rows, const int* pos,
             int mode, void* kc, void* vc, long long seq_stride, int n_ctx, void* q_out,
             long long qos, int H, int KV, int D, int n_rot, int neox) {
  switch (q_dtype) {
    case B2A_F32:
      launch_rope<TK, float>(grid, block, n_tok, st, q, qs, k, ks, v, vs, bq, bk, bv, ct, stb, tab_rows, pos,
                             mode, kc, vc, seq_stride, n_ctx, q_out, qos, H, KV, D, n_rot, neox);
      return B2A_OK;
    case B2A_F16:
      launch_rope<TK, __half>(grid, block, n_tok, st, q, qs, k, ks, v, vs, bq, bk, bv, ct, stb, tab_rows, pos,
                              mode, kc, vc, seq_stride, n_ctx, q_out, qos, H, KV, D, n_rot, neox);
      return B2A_OK;
    case B2A_BF16:
      launch_rope<TK, __nv_bfloat16>(grid, block, n_tok, st, q, qs, k, ks, v, vs, bq, bk, bv, ct, stb, tab_rows,
                                     pos, mode, kc, vc, seq_stride, n_ctx, q_out, qos, H, KV, D,
                                     n_rot, neox);
      return B2A_OK;
  }
  return fail(B2A_ERR_DTYPE, "rope_append: q_out_dtype %d", q_dtype);
}

template <typename TK, typename TQ>
void launch_imrope(dim3 grid, dim3 block, int n_tok, cudaStream_t st, const float* q,
                   long long qs, const float* k,
                   long long ks, const float* v, long long vs, const int* lanes,
                   const ImropeParams& prm, double fscale, const int* pos, int mode, void* kc,
                   void* vc, long long seq_stride, int n_ctx, void* q_out, int H, int KV, int D) {
  b2a_host::launch(imrope_append_kernel<TK, TQ>, grid, block, 0, st, q, qs, k, ks, v, vs, lanes,
                   prm, fscale, pos, mode, static_cast<TK*>(kc), static_cast<TK*>(vc),
                   seq_stride, n_ctx, static_cast<TQ*>(q_out), H, KV, D, n_tok);
}

template <typename TK>
int imrope_qdt(int q_dtype, dim3 grid, dim3 block, int n_tok, cudaStream_t st, const float* q,
               long long qs,
               const float* k, long long ks, const float* v, long long vs, const int* lanes,
               const ImropeParams& prm, double fscale, const int* pos, int mode, void* kc,
               void* vc, long long seq_stride, int n_ctx, void* q_out, int H, int KV, int D) {
  switch (q_dtype) {
    case B2A_F32:
      launch_imrope<TK, float>(grid, block, n_tok, st, q, qs, k, ks, v, vs, lanes, prm, fscale, pos, mode, kc,
                               vc, seq_stride, n_ctx, q_out, H, KV, D);
      return B2A_OK;
    case B2A_F16:
      launch_imrope<TK, __half>(grid, block, n_tok, st, q, qs, k, ks, v, vs, lanes, prm, fscale, pos, mode, kc,
                                vc, seq_stride, n_ctx, q_out, H, KV, D);
      return B2A_OK;
    case B2A_BF16:
      launch_imrope<TK, __nv_bfloat16>(grid, block, n_tok, st, q, qs, k, ks, v, vs, lanes, prm, fscale, pos,
                                       mode, kc, vc, seq_stride, n_ctx, q_out, H, KV, D);
      return B2A_OK;
  }
  return fail(B2A_ERR_DTYPE, "imrope_append: q_out_dtype %d", q_dtype);
}

int check_common(const void* q, const void* k, const void* v, const int* pos, void* kc, void* vc,
                 int n_tok, int H, int KV, int D, int n_ctx, long long seq_stride,
                 int tok_seq_mode, const char* who) {
  // KV == 0 rotates q only (no k/v rows, no cache): the k, v and cache
  // pointers may then be NULL.
  if (!q || !pos || (KV > 0 && (!k || !v || !kc || !vc)))
    return fail(B2A_ERR_ARG, "%s: null pointer argument", who);
  if (n_tok < 0 || H <= 0 || KV < 0 || D <= 0 || n_ctx <= 0)
    return fail(B2A_ERR_ARG, "%s: sizes must be positive", who);
  if (tok_seq_mode != 0 && tok_seq_mode != 1) return fail(B2A_ERR_ARG, "%s: tok_seq_mode must be 0 or 1", who);
  const long long seq_elems = static_cast<long long>(n_ctx) * KV * D;
  if (tok_seq_mode == 1 && n_tok > 1 && seq_stride < seq_elems)
    return fail(B2A_ERR_SHAPE, "%s: seq_stride %lld < n_ctx*KV*D %lld", who, seq_stride, seq_elems);
  return B2A_OK;
}

}  // namespace

extern "C" {

int b2a_rope_append(float* q, long long q_tok_stride, const float* k, long long k_tok_stride,
                    const float* v, long long v_tok_stride, const float* bq, const float* bk,
                    const float* bv, const float* cos_tab, const float* sin_tab, int tab_rows,
                    const int* pos_dev, int tok_seq_mode, void* k_cache, void* v_cache,
                    long long seq_stride, int n_ctx, int kv_dtype, void* q_out, int q_out_dtype,
                    int n_tok, int H, int KV, int D, int n_rot, int style, void* stream) {
  int rc = check_common(q, k, v, pos_dev, k_cache, v_cache, n_tok, H, KV, D, n_ctx, seq_stride,
                        tok_seq_mode, "rope_append");
  if (rc) return rc;
  if (!cos_tab || !sin_tab || tab_rows <= 0) return fail(B2A_ERR_ARG, "rope_append: missing cos/sin tables");
  if (n_rot < 0 || (n_rot & 1) || n_rot > D)
    return fail(B2A_ERR_SHAPE, "rope_append: n_rot %d must be even and <= head_dim %d", n_rot, D);
  if (style != B2A_ROPE_NORM && style != B2A_ROPE_NEOX) return fail(B2A_ERR_ARG, "rope_append: style %d", style);
  long long qos = static_cast<long long>(H) * D;
  if (!q_out) {  // rotate in place: token i's q row stays at q + i*q_tok_stride
    q_out = q;
    q_out_dtype = B2A_F32;
    qos = q_tok_stride;
  }
  if (n_tok == 0) return B2A_OK;
  if (D & 1) return fail(B2A_ERR_SHAPE, "rope_append: head_dim %d must be even", D);
  // tokens per CTA: one for a decode step, up to 8 for a prefill chunk
  const int tpb = rope_block(D), ty = std::max(1, std::min({8, n_tok, R::kThreads / tpb}));
  dim3 grid((n_tok + ty - 1) / ty, H + 2 * KV), block(tpb, ty);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int neox = style == B2A_ROPE_NEOX;
  switch (kv_dtype) {
    case B2A_F32:
      rc = rope_qdt<float>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v, v_tok_stride,
                           bq, bk, bv, cos_tab, sin_tab, tab_rows, pos_dev, tok_seq_mode, k_cache,
                           v_cache, seq_stride, n_ctx, q_out, qos, H, KV, D, n_rot, neox);
      break;
    case B2A_F16:
      rc = rope_qdt<__half>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v, v_tok_stride,
                            bq, bk, bv, cos_tab, sin_tab, tab_rows, pos_dev, tok_seq_mode, k_cache,
                            v_cache, seq_stride, n_ctx, q_out, qos, H, KV, D, n_rot, neox);
      break;
    case B2A_BF16:
      rc = rope_qdt<__nv_bfloat16>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v,
                                   v_tok_stride, bq, bk, bv, cos_tab, sin_tab, tab_rows, pos_dev,
                                   tok_seq_mode, k_cache, v_cache, seq_stride, n_ctx, q_out, qos, H,
                                   KV, D, n_rot, neox);
      break;
    default:
      return fail(B2A_ERR_DTYPE, "rope_append: kv_dtype %d", kv_dtype);
  }
  if (rc) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "rope_append launch");
  return B2A_OK;
}

int b2a_imrope_append(const float* q, long long q_tok_stride, const float* k,
                      long long k_tok_stride, const float* v, long long v_tok_stride,
                      const int* lanes_dev, const int* sections, double freq_base,
                      double freq_scale, const int* pos_dev, int tok_seq_mode, void* k_cache,
                      void* v_cache, long long seq_stride, int n_ctx, int kv_dtype, void* q_out,
                      int q_out_dtype, int n_tok, int H, int KV, int D, void* stream) {
  int rc = check_common(q, k, v, pos_dev, k_cache, v_cache, n_tok, H, KV, D, n_ctx, seq_stride,
                        tok_seq_mode, "imrope_append");
  if (rc) return rc;
  if (!lanes_dev || !sections || !q_out) return fail(B2A_ERR_ARG, "imrope_append: null pointer argument");
  for (int i = 0; i < 4; ++i)
    if (sections[i] < 0) return fail(B2A_ERR_ARG, "imrope_append: negative section");
  const int P = sections[0] + sections[1] + sections[2] + sections[3];
  if (P <= 0) return fail(B2A_ERR_ARG, "imrope_append: at least one section must be nonzero");
  if (2 * P > D || P > kMaxPairs)
    return fail(B2A_ERR_SHAPE, "imrope_append: 2*sum(sections)=%d exceeds head_dim %d", 2 * P, D);
  if (!(freq_base > 0.0) || !isfinite(freq_base) || !(freq_scale > 0.0) || !isfinite(freq_scale))
    return fail(B2A_ERR_ARG, "imrope_append: frequency base/scale must be positive and finite");
  ImropeParams prm;
  prm.pairs = P;
  for (int j = 0; j < P; ++j) {
    prm.pw[j] = pow(freq_base, -2.0 * j / (2.0 * P));
    prm.lane[j] = static_cast<signed char>(imrope_lane(j, sections));
  }
  if (n_tok == 0) return B2A_OK;
  if (D & 1) return fail(B2A_ERR_SHAPE, "imrope_append: head_dim %d must be even", D);
  // tokens per CTA: one for a decode step, up to 8 for a prefill chunk
  const int tpb = rope_block(D), ty = std::max(1, std::min({8, n_tok, R::kThreads / tpb}));
  dim3 grid((n_tok + ty - 1) / ty, H + 2 * KV), block(tpb, ty);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (kv_dtype) {
    case B2A_F32:
      rc = imrope_qdt<float>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v,
                             v_tok_stride, lanes_dev, prm, freq_scale, pos_dev, tok_seq_mode,
                             k_cache, v_cache, seq_stride, n_ctx, q_out, H, KV, D);
      break;
    case B2A_F16:
      rc = imrope_qdt<__half>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v,
                              v_tok_stride, lanes_dev, prm, freq_scale, pos_dev, tok_seq_mode,
                              k_cache, v_cache, seq_stride, n_ctx, q_out, H, KV, D);
      break;
    case B2A_BF16:
      rc = imrope_qdt<__nv_bfloat16>(q_out_dtype, grid, block, n_tok, st, q, q_tok_stride, k, k_tok_stride, v,
                                     v_tok_stride, lanes_dev, prm, freq_scale, pos_dev,
                                     tok_seq_mode, k_cache, v_cache, seq_stride, n_ctx, q_out, H,
                                     KV, D);
      break;
    default:
      return fail(B2A_ERR_DTYPE, "imrope_append: kv_dtype %d", kv_dtype);
  }
  if (rc) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "imrope_append launch");
  return B2A_OK;
}

}  // extern "C"
