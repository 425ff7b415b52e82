// Q8_0 matrix-vector products for the decode step (batch 1), and the Q8_0
// embedding-row gather.
//
// The reference's Q8_0 matvec (alpaccaroo/qmatrix.py:312-320; its device
// chain's kernel is cuda.py:241-286) computes, per output row r,
//   out[r] = sum_b d[r][b] * sum_{l<32} q[r][32b+l] * x[32b+l]
// with int8 codes q and f16 block scales d.  Here the GGUF records (an f16 d
// then 32 codes, 34 bytes) are repacked once at load into an int8 code
// matrix [rows][cols] (16-byte aligned rows) and an f16 scale matrix
// [rows][cols/32]: the same 1.0625 bytes per weight, readable with 16-byte
// loads.
//
// HBM-bound: one lane owns one 32-code block per step (two 16-byte code
// loads and one 2-byte scale load), each warp works two rows at once, and the
// grid is persistent (the resident CTAs) over row pairs.  int8 -> f32 is one byte permute into
// the mantissa of 2^23 and one subtraction (the conversion instruction runs
// on the narrow XU pipe).  x is staged once per CTA in shared memory as
// float4 column j of block b at [j][b], so a warp's 32 lanes read 32
// consecutive float4s.  The staging applies the step's prologue:
//   RMSNORM  x * (1 / sqrt(x.x / n + eps)) * w   (tensor.py:349-356)
//   SWIGLU   gate / (1 + exp(-gate)) * up          (model.py:1466-1467)
// and the epilogue can add the product into out (the residual stream), or,
// for a matrix whose rows interleave gate and up rows (2i = gate_i,
// 2i+1 = up_i), write the SwiGLU of each row pair (the FFN's activation).
//
// Each warp walks its rows as slabs (a row pair x 64 blocks) with the next
// slab's loads in flight while it computes the current one; rows longer
// than 2048 columns are split across the warps of a CTA.  Chained
// launches (flag B2A_GEMV_PDL) use programmatic dependent launch: every CTA
// lets the next kernel launch at once and issues its first slab's loads
// (the weights do not depend on the previous kernel) before it waits for
// the previous kernel and reads x.  Launched without the flag the wait
// returns at once.

namespace b2a {
namespace q8 {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 2;  // rows per warp at a time

__device__ __forceinline__ float code_f32(uint32_t biased_word, int k) {
  // byte k of the word (code + 128) placed in the low mantissa bits of 2^23
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, 0x7440u + k)) - 8388736.0f;
}

// sum_{l<32} code[l] * x[l] for one block: codes c0|c1 (2 x 16 bytes), x from
// the staged [j][b] layout
__device__ __forceinline__ float block_dot(const uint4& c0, const uint4& c1,
                                           const float4* __restrict__ xs, int nb, int b) {
  const uint32_t w[8] = {c0.x ^ 0x80808080u, c0.y ^ 0x80808080u, c0.z ^ 0x80808080u,
                         c0.w ^ 0x80808080u, c1.x ^ 0x80808080u, c1.y ^ 0x80808080u,
                         c1.z ^ 0x80808080u, c1.w ^ 0x80808080u};
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 xv = xs[j * nb + b];
    acc = fmaf(code_f32(w[j], 0), xv.x, acc);
    acc = fmaf(code_f32(w[j], 1), xv.y, acc);
    acc = fmaf(code_f32(w[j], 2), xv.z, acc);
    acc = fmaf(code_f32(w[j], 3), xv.w, acc);
  }
  return acc;
}

// Epilogues: 0 store, 1 add into out (residual), 2 SwiGLU of the row pair
template <int Mode, int Epi>
__global__ void __launch_bounds__(kThreads) gemv_kernel(
    const int8_t* __restrict__ codes, const __half* __restrict__ scales, int rows, int cols,
    const float* __restrict__ x, const float* __restrict__ aux, float eps,
    float* __restrict__ out) {
  extern __shared__ float4 xs[];  // [8][nb]
  __shared__ double red[kWarps];
  const int nb = cols >> 5;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // Work unit: a slab = one row pair x 64 blocks (lane l: blocks
  // part*64 + l and part*64 + 32 + l of both rows, 128 bytes of codes).  A
  // row pair has spp = ceil(nb/64) slabs, taken by spp warps of the same CTA
  // (a long row is split across warps, their sums meet in shared memory),
  // so a CTA round covers ppr = kWarps / spp pairs.  Each warp walks its
  // rounds with the next round's slab loads in flight while it computes the
  // current one.
  const int spp = (nb + 63) >> 6;
  const int ppr = kWarps / spp;
  const int wpair = warp / spp, wpart = warp % spp;
  const bool wactive = wpair < ppr;
  const int pairs = (rows + kRows - 1) / kRows;
  const int groups = (pairs + ppr - 1) / ppr;
  const int n_rounds = static_cast<int>(blockIdx.x) < groups
                           ? (groups - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                           : 0;
  __shared__ float psum[2][kWarps][kRows];  // per round parity

  struct Slab {
    uint4 c[kRows][2][2];
    float d[kRows][2];
  };
  // pair handled by this warp in round j (>= pairs: none)
  auto pair_of = [&](int j) { return (blockIdx.x + j * gridDim.x) * ppr + wpair; };
  auto load = [&](int j, Slab& sl) {
    const int pr = pair_of(j);
    const bool live = wactive && pr < pairs;
    const int r0 = pr * kRows;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int row = min(r0 + r, rows - 1);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int blk = wpart * 64 + h * 32 + lane;
        if (live && blk < nb) {
          const uint4* p = reinterpret_cast<const uint4*>(codes + static_cast<size_t>(row) * cols +
                                                          blk * 32);
          sl.c[r][h][0] = __ldg(p);
          sl.c[r][h][1] = __ldg(p + 1);
          sl.d[r][h] = __half2float(scales[static_cast<size_t>(row) * nb + blk]);
        } else {
          sl.c[r][h][0] = sl.c[r][h][1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u,
                                                     0x80808080u);  // codes 0 after the bias
          sl.d[r][h] = 0.f;
        }
      }
    }
  };

  // ---- overlap with the previous kernel: release the next, load weights ---
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  Slab cur, nxt;
  if (n_rounds > 0) load(0, cur);  // weights do not depend on the previous kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage x (with the prologue) ---------------------------------------
  float scale = 1.f;
  if (Mode == 1) {
    double ss = 0.0;
    for (int c = threadIdx.x; c < cols; c += kThreads) {
      const double v = x[c];
      ss += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];
    scale = static_cast<float>(1.0 / sqrt(tot / cols + static_cast<double>(eps)));
  }
  for (int i = threadIdx.x; i < nb * 8; i += kThreads) {
    const int b = i >> 3, j = i & 7;  // float4 j of block b
    const int c = b * 32 + j * 4;
    float4 v;
    if (Mode == 2) {
      float e[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float g = x[c + t];
        e[t] = g / (1.f + expf(-g)) * x[cols + c + t];
      }
      v = make_float4(e[0], e[1], e[2], e[3]);
    } else {
      v = *reinterpret_cast<const float4*>(x + c);
      if (Mode == 1) {
        const float4 w = *reinterpret_cast<const float4*>(aux + c);
        v = make_float4(v.x * scale * w.x, v.y * scale * w.y, v.z * scale * w.z,
                        v.w * scale * w.w);
      }
    }
    xs[j * nb + b] = v;
  }
  __syncthreads();

  // ---- rounds --------------------------------------------------------------
  for (int j = 0; j < n_rounds; ++j) {
    if (j + 1 < n_rounds) load(j + 1, nxt);
    float acc[kRows] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int blk = wpart * 64 + h * 32 + lane;
      if (blk < nb) {
#pragma unroll
        for (int r = 0; r < kRows; ++r)
          acc[r] = fmaf(block_dot(cur.c[r][h][0], cur.c[r][h][1], xs, nb, blk), cur.d[r][h],
                        acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    if (spp > 1) {
      if (lane == 0) {
        psum[j & 1][warp][0] = acc[0];
        psum[j & 1][warp][1] = acc[1];
      }
      __syncthreads();
      if (wactive && wpart == 0) {  // the pair's first warp adds its siblings' sums in order
        for (int t = 1; t < spp; ++t) {
          acc[0] += psum[j & 1][warp + t][0];
          acc[1] += psum[j & 1][warp + t][1];
        }
      }
    }
    const int pr = pair_of(j);
    if (wactive && wpart == 0 && lane == 0 && pr < pairs) {
      const int r0 = pr * kRows;
      const bool two = r0 + 1 < rows;
      const float a0 = acc[0], a1 = acc[1];
      if (Epi == 1) {
        out[r0] += a0;
        if (two) out[r0 + 1] += a1;
      } else if (Epi == 2) {
        out[r0 >> 1] = a0 / (1.f + expf(-a0)) * a1;  // gate_i = row 2i, up_i = row 2i+1
      } else {
        out[r0] = a0;
        if (two) out[r0 + 1] = a1;
      }
    }
    if (j + 1 < n_rounds) cur = nxt;
  }
}

// out[i][c] = code[tok_i][c] * d[tok_i][c / 32]  (qmatrix.py:445-447), one
// grid row (blockIdx.y) per token
__global__ void embed_kernel(const int8_t* __restrict__ codes, const __half* __restrict__ scales,
                             int rows, int cols, const int* __restrict__ tokens,
                             float* __restrict__ out) {
  const int t = tokens[blockIdx.y];
  if (t < 0 || t >= rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_dev_error(B2A_ERR_POSITION, t);
    return;
  }
  const int8_t* row = codes + static_cast<size_t>(t) * cols;
  const __half* sr = scales + static_cast<size_t>(t) * (cols >> 5);
  float* o = out + static_cast<size_t>(blockIdx.y) * cols;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x)
    o[c] = static_cast<float>(row[c]) * __half2float(sr[c >> 5]);
}

}  // namespace q8
}  // namespace b2a

namespace {

template <int Mode, int Epi>
int launch_gemv(const int8_t* codes, const __half* scales, int rows, int cols, const float* x,
                const float* aux, float eps, float* out, bool pdl, cudaStream_t st) {
  namespace Q = b2a::q8;
  auto kern = Q::gemv_kernel<Mode, Epi>;
  const int smem = cols * 4;  // 8 float4 per 32-column block
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               smem);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(q8_gemv)");
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int pairs = (rows + Q::kRows - 1) / Q::kRows;
  const int ppr = Q::kWarps / ((cols / 32 + 63) / 64);  // pairs per CTA round
  int grid = (pairs + ppr - 1) / ppr;
  int per_sm = 1;  // persistent: at most the resident CTAs, each walks its pairs
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Q::kThreads, smem);
  if (per_sm < 1) per_sm = 1;
  if (grid > sms * per_sm) grid = sms * per_sm;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Q::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, codes, scales, rows, cols, x, aux, eps, out);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "q8_gemv launch");
  return B2A_OK;
}

}  // namespace

extern "C" {

int b2a_q8_gemv(const void* codes, const void* scales, int rows, int cols, const float* x,
                const float* aux, int mode, float eps, float* out, int flags, void* stream) {
  using b2a_host::fail;
  if (!codes || !scales || !x || !out) return fail(B2A_ERR_ARG, "q8_gemv: null pointer argument");
  if (rows <= 0 || cols <= 0 || (cols & 31))
    return fail(B2A_ERR_SHAPE, "q8_gemv: rows %d, cols %d (cols a positive multiple of 32)", rows,
                cols);
  if (cols > 16384) return fail(B2A_ERR_UNSUPPORTED, "q8_gemv: cols %d > 16384", cols);
  if (!b2a_host::aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 1) ||
      !b2a_host::aligned16(x))
    return fail(B2A_ERR_ALIGN, "q8_gemv: codes and x must be 16-byte aligned, scales 2-byte");
  if (mode < 0 || mode > 2) return fail(B2A_ERR_ARG, "q8_gemv: mode %d", mode);
  if (mode == 1 && (!aux || !b2a_host::aligned16(aux) || !(eps > 0.f)))
    return fail(B2A_ERR_ARG, "q8_gemv: RMSNorm needs an aligned weight and eps > 0");
  const int8_t* c = static_cast<const int8_t*>(codes);
  const __half* s = static_cast<const __half*>(scales);
  if (flags & ~(B2A_GEMV_ACCUMULATE | B2A_GEMV_SWIGLU_OUT | B2A_GEMV_PDL))
    return fail(B2A_ERR_ARG, "q8_gemv: unknown flags %#x", flags);
  const bool acc = flags & B2A_GEMV_ACCUMULATE, swo = flags & B2A_GEMV_SWIGLU_OUT;
  if (acc && swo) return fail(B2A_ERR_ARG, "q8_gemv: ACCUMULATE and SWIGLU_OUT exclude each other");
  if (swo && (rows & 1)) return fail(B2A_ERR_SHAPE, "q8_gemv: SWIGLU_OUT needs an even row count");
  const bool pdl = flags & B2A_GEMV_PDL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int epi = acc ? 1 : (swo ? 2 : 0);
#define B2A_GEMV_CASE(M)                                                                   \
  return epi == 1 ? launch_gemv<M, 1>(c, s, rows, cols, x, aux, eps, out, pdl, st)         \
                  : (epi == 2 ? launch_gemv<M, 2>(c, s, rows, cols, x, aux, eps, out, pdl, st) \
                              : launch_gemv<M, 0>(c, s, rows, cols, x, aux, eps, out, pdl, st))
  switch (mode) {
    case 0: B2A_GEMV_CASE(0);
    case 1: B2A_GEMV_CASE(1);
    default: B2A_GEMV_CASE(2);
  }
#undef B2A_GEMV_CASE
}

int b2a_q8_embed(const void* codes, const void* scales, int rows, int cols,
                 const int* tokens_dev, int n_tok, float* out, void* stream) {
  using b2a_host::fail;
  if (!codes || !scales || !tokens_dev || !out)
    return fail(B2A_ERR_ARG, "q8_embed: null pointer argument");
  if (rows <= 0 || cols <= 0 || (cols & 31) || n_tok < 0 || n_tok > 65535)
    return fail(B2A_ERR_SHAPE, "q8_embed: bad shape");
  if (n_tok == 0) return B2A_OK;
  const int threads = 256;
  int blocks = (cols + threads - 1) / threads;
  if (blocks > 64) blocks = 64;
  b2a::q8::embed_kernel<<<dim3(blocks, n_tok), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int8_t*>(codes), static_cast<const __half*>(scales), rows, cols,
      tokens_dev, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "q8_embed launch");
  return B2A_OK;
}

}  // extern "C"
