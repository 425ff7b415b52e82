// Q8_0 matrix-vector products for the decode step (batch 1), and the Q8_0
// embedding-row gather.
//
// The reference's Q8_0 matvec (alpaccaroo/qmatrix.py:312-320; its device
// chain's kernel is cuda.py:241-286) computes, per output row r,
//   out[r] = sum_b d[r][b] * sum_{l<32} q[r][32b+l] * x[32b+l]
// with int8 codes q and f16 block scales d.
//
// The products run on the tensor cores (mma.sync m16n8k16, f16 in, f32
// accumulate), which cuts the instructions per weight about fivefold against
// an FMA loop: the A operand is 16 rows x 16 codes, each code turned exactly
// into an f16 by one byte permute into 1024 + (code + 128) and one packed
// subtraction; the B operand holds x split into f16 hi and lo parts
// (x = hi + lo to about 2^-22) as its two used columns.  Per 32-code block
// two MMAs give the block's dot for 16 rows; its f16 scale is applied in f32
// and the rows accumulate in f32, as the reference sums blocks.
//
// Layout (repacked once at load from the GGUF records): rows are padded to a
// multiple of 16 and cut into 512-byte tiles of 16 rows x one 32-code block,
// tile (rg, b) at byte (rg * nb + b) * 512, lane t's 16 bytes being its A
// fragments for the block's two MMAs (rows g = t/4 and g + 8, codes
// 2(t%4) + {0, 1, 8, 9} and + 16); scales tile (rg, b) holds 16 f16 in the
// order (row 0, row 8, row 1, row 9, ...).  A warp streams its tiles with
// 16-byte loads, sixteen tiles in flight; rows longer than a few hundred
// blocks are split across the warps of a CTA and meet in shared memory.
// x is staged once per CTA from float4 loads, applying the step's prologue:
//   RMSNORM  x * (1 / sqrt(x.x / n + eps)) * w   (tensor.py:349-356)
//   SWIGLU   gate / (1 + exp(-gate)) * up          (model.py:1466-1467)
// and the epilogue stores, adds into out (the residual stream) or, for a
// matrix whose 16-row groups hold gate rows 8q..8q+7 then the matching up
// rows, writes the SwiGLU of each (gate, up) row pair.
//
// Chained launches (flag B2A_GEMV_PDL) use programmatic dependent launch:
// every CTA lets the next kernel launch at once and loads its first tiles
// (the weights do not depend on the previous kernel) before it waits for
// the previous kernel and reads x.  Launched without the flag the wait
// returns at once.

namespace b2a {
namespace q8 {

constexpr int kUnroll = 16;  // tiles in flight per warp (a whole task when kw splits rows)
constexpr int kHold = 2;     // float4 of x held per thread across the RMSNorm reduction

// two codes (bytes sel_lo/sel_hi of a word already biased by +128) -> f16x2
__device__ __forceinline__ uint32_t codes_f16x2(uint32_t biased, uint32_t sel) {
  const uint32_t v = __byte_perm(biased, 0x64646464u, sel);  // 1024 + (code + 128)
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1152.f));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Where the QKV epilogue (Epi 3) puts the rotated q row and the step's K/V
// cache rows: rows [0, H*D) of the product are q, then KV*D of k, then v.
struct QkvRope {
  const float* cos_tab;  // [tab_rows][D/2]
  const float* sin_tab;
  const int* pos;        // the token's position (one int, device memory)
  void* k_cache;         // [n_ctx][KV][D] of the cache type
  void* v_cache;
  int tab_rows, n_ctx, H, KV, D;
};

// RoPE (norm style: pairs 2i, 2i+1 of a head, model.py:1162-1209 with the
// reference's f32 product order) of one output row whose pair partner is
// `other`, then the row's store: q into out, k and v into the cache row
// at the token's position (model.py:1431-1432).
template <typename TK>
__device__ __forceinline__ void qkv_rope_store(const QkvRope& rp, int p, int row, float self,
                                               float other, float* __restrict__ out) {
  const int qd = rp.H * rp.D, kd = rp.KV * rp.D;
  if (row < qd + kd) {
    const int d = row % rp.D, i = d >> 1;
    const float c = rp.cos_tab[static_cast<size_t>(p) * (rp.D >> 1) + i];
    const float sn = rp.sin_tab[static_cast<size_t>(p) * (rp.D >> 1) + i];
    const bool odd = d & 1;
    const float x0 = odd ? other : self, x1 = odd ? self : other;
    const float y = odd ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c))
                        : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    if (row < qd) {
      out[row] = y;
    } else {
      st_elem(static_cast<TK*>(rp.k_cache) + static_cast<size_t>(p) * kd + (row - qd), y);
    }
  } else {
    st_elem(static_cast<TK*>(rp.v_cache) + static_cast<size_t>(p) * kd + (row - qd - kd), self);
  }
}

template <int Mode, int Epi, int kWarps, typename TK = float>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(
    const uint4* __restrict__ tiles, const uint32_t* __restrict__ scales, int rows, int cols,
    int kw, const float* __restrict__ x, const float* __restrict__ aux, float eps,
    float* __restrict__ out, const QkvRope rp) {
  constexpr int kThreads = kWarps * 32;
  extern __shared__ uint4 xs[];  // [nb][8]: B fragments (hi for lanes 0-3, lo for 4-7)
  __shared__ double red[kWarps];
  __shared__ float psum[2][kWarps][16];
  const int nb = cols >> 5;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tp = lane & 3;
  const int rgs = (rows + 15) >> 4;   // row groups
  const int slots = kWarps / kw;      // row groups per CTA task
  const int slot = warp / kw, ks = warp % kw;
  const int bpw = (nb + kw - 1) / kw;  // blocks per warp
  const int b_lo = ks * bpw, b_hi = min(nb, b_lo + bpw);
  const int tasks = (rgs + slots - 1) / slots;
  const int n_tasks = static_cast<int>(blockIdx.x) < tasks
                          ? (tasks - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                          : 0;

  uint4 c[kUnroll];
  uint32_t sc[kUnroll];
  auto load = [&](int rg, int b0) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int b = b0 + u;
      if (rg < rgs && b < b_hi) {
        const size_t t = static_cast<size_t>(rg) * nb + b;
        c[u] = __ldg(tiles + t * 32 + lane);
        sc[u] = tp == 0 ? __ldg(scales + t * 8 + g) : 0u;
      } else {
        c[u] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // codes 0
        sc[u] = 0u;
      }
    }
  };

  // ---- overlap with the previous kernel: release the next, load weights ---
  // (and the RMSNorm weight: neither depends on the previous kernel)
  const int n4 = cols >> 2;
  const bool held = n4 <= kThreads * kHold;  // x fits in registers: one pass
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const float4* a4 = reinterpret_cast<const float4*>(aux);
  float4 av[kHold], xv[kHold];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (n_tasks > 0) load(static_cast<int>(blockIdx.x) * slots + slot, b_lo);
  if (Mode == 1 && held) {
#pragma unroll
    for (int h = 0; h < kHold; ++h) {
      const int i = threadIdx.x + h * kThreads;
      av[h] = i < n4 ? __ldg(a4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage x (with the prologue) as f16 hi / lo B fragments -----------------
  if (held) {
#pragma unroll
    for (int h = 0; h < kHold; ++h) {
      const int i = threadIdx.x + h * kThreads;
      xv[h] = i < n4 ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float scale = 1.f;
  if (Mode == 1) {
    double ss = 0.0;
    auto sq = [](float4 v) {
      return static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y +
             static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
    };
    if (held) {
#pragma unroll
      for (int h = 0; h < kHold; ++h) ss += sq(xv[h]);
    } else {
      for (int i = threadIdx.x; i < n4; i += kThreads) ss += sq(__ldg(x4 + i));
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) tot += red[i];
    scale = static_cast<float>(1.0 / sqrt(tot / cols + static_cast<double>(eps)));
  }
  // Four consecutive inputs k..k+3 (k = 4i) land in one word j = (k & 31) >> 3
  // of the B fragments q0 = (k & 7) / 2 and q0 + 1 of block k / 32: two
  // 16-bit pairs into the hi entries (lanes q) and two into the lo entries
  // (lanes 4 + q).  Every input is loaded once, as part of a float4.
  uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
  auto put = [&](int i, float4 v, float4 w) {
    if (Mode == 1) {
      v = make_float4(v.x * scale * w.x, v.y * scale * w.y, v.z * scale * w.z, v.w * scale * w.w);
    } else if (Mode == 2) {
      const float4 u = __ldg(x4 + n4 + i);
      v = make_float4(v.x / (1.f + expf(-v.x)) * u.x, v.y / (1.f + expf(-v.y)) * u.y,
                      v.z / (1.f + expf(-v.z)) * u.z, v.w / (1.f + expf(-v.w)) * u.w);
    }
    const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v.x - f01.x, v.y - f01.y);
    const __half2 l23 = __floats2half2_rn(v.z - f23.x, v.w - f23.y);
    const int k = i << 2, b = k >> 5, j = (k & 31) >> 3, q0 = (k & 7) >> 1;
    uint32_t* e = xw + b * 32 + j;  // entry (b, lane) word j at e[lane * 4]
    e[q0 * 4] = *reinterpret_cast<const uint32_t*>(&h01);
    e[(q0 + 1) * 4] = *reinterpret_cast<const uint32_t*>(&h23);
    e[(q0 + 4) * 4] = *reinterpret_cast<const uint32_t*>(&l01);
    e[(q0 + 5) * 4] = *reinterpret_cast<const uint32_t*>(&l23);
  };
  if (held) {
#pragma unroll
    for (int h = 0; h < kHold; ++h) {
      const int i = threadIdx.x + h * kThreads;
      if (i < n4) put(i, xv[h], av[h]);
    }
  } else {
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += kThreads)
      put(i, __ldg(x4 + i), Mode == 1 ? __ldg(a4 + i) : make_float4(0.f, 0.f, 0.f, 0.f));
  }
  __syncthreads();

  // ---- tasks ---------------------------------------------------------------
  for (int j = 0; j < n_tasks; ++j) {
    const int rg = (static_cast<int>(blockIdx.x) + j * gridDim.x) * slots + slot;
    float acc_a = 0.f, acc_b = 0.f;  // rows 16rg + g and 16rg + g + 8 (lanes tp == 0)
    for (int b0 = b_lo; b0 < b_hi; b0 += kUnroll) {
      if (b0 != b_lo) load(rg, b0);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int b = b0 + u;
        if (b >= b_hi) break;
        const uint4 bf = lane < 8 ? xs[b * 8 + lane] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w0 = c[u].x ^ 0x80808080u, w1 = c[u].y ^ 0x80808080u;
        const uint32_t w2 = c[u].z ^ 0x80808080u, w3 = c[u].w ^ 0x80808080u;
        const uint32_t a0[4] = {codes_f16x2(w0, 0x4140u), codes_f16x2(w0, 0x4342u),
                                codes_f16x2(w1, 0x4140u), codes_f16x2(w1, 0x4342u)};
        const uint32_t a1[4] = {codes_f16x2(w2, 0x4140u), codes_f16x2(w2, 0x4342u),
                                codes_f16x2(w3, 0x4140u), codes_f16x2(w3, 0x4342u)};
        const uint32_t b0f[2] = {bf.x, bf.y}, b1f[2] = {bf.z, bf.w};
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        MmaOp<__half>::run(cc, a0, b0f);
        MmaOp<__half>::run(cc, a1, b1f);
        const __half2 d = *reinterpret_cast<const __half2*>(&sc[u]);  // rows g, g + 8
        acc_a = fmaf(cc[0] + cc[1], __low2float(d), acc_a);
        acc_b = fmaf(cc[2] + cc[3], __high2float(d), acc_b);
      }
    }
    if (j + 1 < n_tasks)  // next task's first tiles while the epilogue runs
      load((static_cast<int>(blockIdx.x) + (j + 1) * gridDim.x) * slots + slot, b_lo);
    if (kw > 1) {
      if (tp == 0) {
        psum[j & 1][warp][g] = acc_a;
        psum[j & 1][warp][g + 8] = acc_b;
      }
      __syncthreads();
      if (ks == 0 && tp == 0) {  // the group's first warp adds its siblings' sums in order
        for (int t = 1; t < kw; ++t) {
          acc_a += psum[j & 1][warp + t][g];
          acc_b += psum[j & 1][warp + t][g + 8];
        }
      }
    }
    if (Epi == 3) {
      if (ks == 0) {  // the pair partner of row 16rg + g is row 16rg + (g ^ 1): lane ^ 4
        const float pa = __shfl_xor_sync(0xffffffffu, acc_a, 4);
        const float pb = __shfl_xor_sync(0xffffffffu, acc_b, 4);
        if (tp == 0 && rg < rgs) {
          const int p = *rp.pos;
          if (p < 0 || p >= rp.n_ctx || p >= rp.tab_rows) {
            if (g == 0) set_dev_error(B2A_ERR_POSITION, p);
          } else {
            const int ra = rg * 16 + g;
            if (ra < rows) qkv_rope_store<TK>(rp, p, ra, acc_a, pa, out);
            if (ra + 8 < rows) qkv_rope_store<TK>(rp, p, ra + 8, acc_b, pb, out);
          }
        }
      }
    } else if (ks == 0 && tp == 0 && rg < rgs) {
      const int ra = rg * 16 + g, rb = ra + 8;
      if (Epi == 2) {
        const int i = rg * 8 + g;  // gate row ra, up row rb
        if (rb < rows) out[i] = acc_a / (1.f + expf(-acc_a)) * acc_b;
      } else if (Epi == 1) {
        if (ra < rows) out[ra] += acc_a;
        if (rb < rows) out[rb] += acc_b;
      } else {
        if (ra < rows) out[ra] = acc_a;
        if (rb < rows) out[rb] = acc_b;
      }
    }
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

template <int Mode, int Epi, int W, typename TK = float>
int launch_gemv_w(const int8_t* codes, const __half* scales, int rows, int cols, const float* x,
                  const float* aux, float eps, float* out, bool pdl, cudaStream_t st,
                  const b2a::q8::QkvRope& rp = b2a::q8::QkvRope{}) {
  auto kern = b2a::q8::gemv_kernel<Mode, Epi, W, TK>;
  const int smem = cols * 4;  // 8 uint4 B fragments per 32-column block
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               smem);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(q8_gemv)");
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // split each row group's blocks over kw warps until there are ~4096 warp
  // tasks (kw a power of two dividing the CTA's W warps, >= 8 blocks each)
  const int rgs = (rows + 15) / 16, nb = cols / 32;
  int kw = 1;
  while (kw < W && rgs * kw < 4096 && nb / (2 * kw) >= 8) kw *= 2;
  const int slots = W / kw;
  int grid = (rgs + slots - 1) / slots;
  int per_sm = 1;  // persistent: at most the resident CTAs, each walks its tasks
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, W * 32, smem);
  if (per_sm < 1) per_sm = 1;
  if (grid > sms * per_sm) grid = sms * per_sm;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(W * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const uint4*>(codes),
                                           reinterpret_cast<const uint32_t*>(scales), rows, cols,
                                           kw, x, aux, eps, out, rp);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "q8_gemv launch");
  return B2A_OK;
}

// Rows of 256+ blocks (8192+ columns) with few row groups run 16-warp CTAs:
// a 16-way K split gives every warp one round of tiles, so the whole matrix
// is in flight at once instead of in two register-sized rounds.
template <int Mode, int Epi>
int launch_gemv(const int8_t* codes, const __half* scales, int rows, int cols, const float* x,
                const float* aux, float eps, float* out, bool pdl, cudaStream_t st) {
  const int rgs = (rows + 15) / 16, nb = cols / 32;
  if (nb >= 256 && rgs <= 512)
    return launch_gemv_w<Mode, Epi, 16>(codes, scales, rows, cols, x, aux, eps, out, pdl, st);
  return launch_gemv_w<Mode, Epi, 8>(codes, scales, rows, cols, x, aux, eps, out, pdl, st);
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
  if (!b2a_host::aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 3) ||
      !b2a_host::aligned16(x))
    return fail(B2A_ERR_ALIGN, "q8_gemv: tiles and x must be 16-byte aligned, scales 4-byte");
  if (mode < 0 || mode > 2) return fail(B2A_ERR_ARG, "q8_gemv: mode %d", mode);
  if (mode == 1 && (!aux || !b2a_host::aligned16(aux) || !(eps > 0.f)))
    return fail(B2A_ERR_ARG, "q8_gemv: RMSNorm needs an aligned weight and eps > 0");
  const int8_t* c = static_cast<const int8_t*>(codes);
  const __half* s = static_cast<const __half*>(scales);
  if (flags & ~(B2A_GEMV_ACCUMULATE | B2A_GEMV_SWIGLU_OUT | B2A_GEMV_PDL))
    return fail(B2A_ERR_ARG, "q8_gemv: unknown flags %#x", flags);
  const bool acc = flags & B2A_GEMV_ACCUMULATE, swo = flags & B2A_GEMV_SWIGLU_OUT;
  if (acc && swo) return fail(B2A_ERR_ARG, "q8_gemv: ACCUMULATE and SWIGLU_OUT exclude each other");
  if (swo && (rows & 15))
    return fail(B2A_ERR_SHAPE, "q8_gemv: SWIGLU_OUT needs whole 16-row (8 gate + 8 up) groups");
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

int b2a_q8_gemv_qkv_rope(const void* codes, const void* scales, int cols, const float* x,
                         const float* norm_w, float eps, float* q_out, const float* cos_tab,
                         const float* sin_tab, int tab_rows, const int* pos_dev, void* k_cache,
                         void* v_cache, int kv_dtype, int n_ctx, int H, int KV, int D, int flags,
                         void* stream) {
  using b2a_host::fail;
  if (!codes || !scales || !x || !norm_w || !q_out || !cos_tab || !sin_tab || !pos_dev ||
      !k_cache || !v_cache)
    return fail(B2A_ERR_ARG, "q8_gemv_qkv_rope: null pointer argument");
  if (H <= 0 || KV <= 0 || D <= 0 || (D & 1) || n_ctx <= 0 || tab_rows <= 0)
    return fail(B2A_ERR_SHAPE, "q8_gemv_qkv_rope: H=%d KV=%d D=%d (even) n_ctx=%d", H, KV, D,
                n_ctx);
  if (cols <= 0 || (cols & 31)) return fail(B2A_ERR_SHAPE, "q8_gemv_qkv_rope: cols %d", cols);
  if (cols > 16384) return fail(B2A_ERR_UNSUPPORTED, "q8_gemv_qkv_rope: cols %d > 16384", cols);
  if (!b2a_host::aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 3) ||
      !b2a_host::aligned16(x) || !b2a_host::aligned16(norm_w))
    return fail(B2A_ERR_ALIGN, "q8_gemv_qkv_rope: tiles, x and norm_w 16-byte aligned, scales 4-byte");
  if (!(eps > 0.f)) return fail(B2A_ERR_ARG, "q8_gemv_qkv_rope: eps must be > 0");
  if (flags & ~B2A_GEMV_PDL) return fail(B2A_ERR_ARG, "q8_gemv_qkv_rope: flags %#x", flags);
  const int rows = (H + 2 * KV) * D;
  const b2a::q8::QkvRope rp{cos_tab, sin_tab, pos_dev, k_cache, v_cache, tab_rows, n_ctx, H, KV, D};
  const int8_t* c = static_cast<const int8_t*>(codes);
  const __half* sc = static_cast<const __half*>(scales);
  const bool pdl = flags & B2A_GEMV_PDL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool wide = cols / 32 >= 256 && (rows + 15) / 16 <= 512;
#define B2A_QKV_CASE(TK)                                                                    \
  return wide ? launch_gemv_w<1, 3, 16, TK>(c, sc, rows, cols, x, norm_w, eps, q_out, pdl, st, rp) \
              : launch_gemv_w<1, 3, 8, TK>(c, sc, rows, cols, x, norm_w, eps, q_out, pdl, st, rp)
  switch (kv_dtype) {
    case B2A_F32: B2A_QKV_CASE(float);
    case B2A_F16: B2A_QKV_CASE(__half);
    case B2A_BF16: B2A_QKV_CASE(__nv_bfloat16);
  }
#undef B2A_QKV_CASE
  return fail(B2A_ERR_DTYPE, "q8_gemv_qkv_rope: kv_dtype %d", kv_dtype);
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
