// Dense GEMMs of a device-resident prefill chunk on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), with the chunk's glue fused into the epilogue.
//
// The reference runs a chunk's projections as Q8_0 GEMMs over the tokens
// (Model.forward_batch, alpaccaroo/model.py:1274-1372; the device chain's
// codes-decoding SIMT GEMM, cuda.py:287-422, called from prefill_chunk,
// cuda.py:1943-2080).  Here the weights are the 16-bit dequantized copy
// (d * code, one rounding) and the activations 16-bit, accumulated in fp32:
//
//   out[m][n] = sum_k a[m][k] * w[n][k]  (+ c_in[m][n])            STORE
//   out[m][128g + j] = silu(acc[m][256g + j]) * acc[m][256g + 128 + j]  SWIGLU
//
// SWIGLU takes the FFN's gate and up weights interleaved in 128-row groups
// (gate rows 128g..128g+127, then the matching up rows) and writes the
// activation the down projection reads (model.py:1352-1354); SWIGLU8 (epilogue
// 4) takes the decode GEMV's 16-row groups of 8 gate rows then 8 up rows.
//
// QKV_ROPE (b2a_gemm_qkv_rope) takes w = [Wq; Wk; Wv] and writes q rotated
// (16-bit) plus the rotated k and the v rows at each token's cache position,
// the work of b2a_rope_append, from the fp32 accumulator.
//
// Kernel: persistent, one CTA per SM, 128 x 256 output tiles (128 x 192
// where that takes fewer tile-widths of waves) taken in m-fastest order (the
// CTAs working at one time share a weight tile, which then comes from L2).
// 256 threads:
//   warp 0       TMA producer: A (128 x 64) and W (256 x 64) K-blocks into a
//                4-stage ring of 48 KB stages (128-byte swizzle)
//   warp 1       TMEM owner, single-lane MMA issuer: 4 x tcgen05.mma
//                (M=128, N=256, K=16) per K-block into one of two 256-column
//                fp32 accumulators
//   warps 4-7    epilogue: TMEM -> registers (warp w reads lanes 32(w%4)..,
//                its 32 rows), residual add / SwiGLU, global store; the other
//                accumulator takes the next tile's MMAs meanwhile
//   warps 8-15   (W8, Q8_0 weights only) converters: the producer loads each
//                K-block's int8 codes into a ring of code slots, and these
//                warps write d * code (rounded once to T) into the stage's
//                weight block in the swizzled layout the MMA reads, then
//                arrive on the stage's full barrier; the product equals the
//                16-bit path's on the dequantized matrix bit for bit
// Every wait is a bounded mbarrier wait (B2A_ERR_TIMEOUT on expiry).

namespace b2a {
namespace gemm {

using prefill::make_idesc;
using prefill::sw128_desc;
using prefill::tc_commit;
using prefill::tc_fence_after;
using prefill::tc_fence_before;
using prefill::tc_ld32;
using prefill::tc_mma;
using prefill::tc_wait_ld;

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 256;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
// Q8_0 weights (W8): 3 stages of A + 16-bit weights, and 4 slots of raw
// codes (BN x 64 bytes) that the converter warps turn into the stages'
// weight blocks
constexpr int kStagesQ8 = 3;
constexpr int kCodeSlots = 4;
// converter warps (two per SM sub-partition)
template <typename T>
__host__ __device__ constexpr int conv_warps() {
  return 8;
}
__host__ __device__ constexpr int threads_for(bool w8, int conv) {
  return w8 ? kThreads + 32 * conv : kThreads;
}
// A stage is the A block plus a BN x 64 weight block (32 KB at BN = 256)
__host__ __device__ constexpr int smem_for(int bn, bool w8 = false) {
  return w8 ? kStagesQ8 * (kABytes + bn * kBK * 2) + kCodeSlots * bn * kBK + 1024
            : kStages * (kABytes + bn * kBK * 2) + 1024;
}
constexpr uint32_t kTmemCols = 512;  // two accumulators of up to 256 columns
constexpr uint32_t kAccStride = 256;

// Q8_0 weights of a W8 launch: codes come through a tensor map, the f16
// scales [N][lds] (one per row and 32-code block) are read by the converters
struct Q8W {
  const __half* scales;
  long long lds;
  int nblk;  // K / 32
};

// 16 codes (int8, one 16-byte load) times their block's scale d, as 16
// elements of T in two 16-byte words: the dequantized weight d * code with
// one rounding, the value a host-side f32 product rounded to T gives.
template <typename T>
struct Dequant;
template <>
struct Dequant<__half> {
  using Scale = uint32_t;  // d in both halves of an f16x2
  __device__ static Scale scale(__half d) {
    const __half2 d2 = __halves2half2(d, d);
    return *reinterpret_cast<const uint32_t*>(&d2);
  }
  // code c + 128 as the low byte of the f16 0x64xx (1024 + c + 128), minus
  // 1152: c exactly; the f16 product with d is then correctly rounded
  __device__ static void run(uint4 c, Scale d, uint4& o0, uint4& o1) {
    const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u,
                           c.w ^ 0x80808080u};
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[2 * i] = __byte_perm(w[i], 0x64646464u, 0x4140);
      h[2 * i + 1] = __byte_perm(w[i], 0x64646464u, 0x4342);
    }
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    const __half2 dd = *reinterpret_cast<const __half2*>(&d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __half2 x = *reinterpret_cast<const __half2*>(&h[j]);
      x = __hmul2(__hsub2(x, bias), dd);
      h[j] = *reinterpret_cast<const uint32_t*>(&x);
    }
    o0 = make_uint4(h[0], h[1], h[2], h[3]);
    o1 = make_uint4(h[4], h[5], h[6], h[7]);
  }
};
template <>
struct Dequant<__nv_bfloat16> {
  using Scale = float;
  __device__ static Scale scale(__half d) { return __half2float(d); }
  // code c + 128 as the low byte of the f32 2^23 + c + 128, minus 2^23 + 128:
  // c exactly; the f32 product with d is exact and rounds once to bf16
  __device__ static void run(uint4 c, Scale d, uint4& o0, uint4& o1) {
    const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u,
                           c.w ^ 0x80808080u};
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        f[k] = (__uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7540 | k)) - 8388736.f) * d;
      const __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]);
      const __nv_bfloat162 p1 = __floats2bfloat162_rn(f[2], f[3]);
      h[2 * i] = *reinterpret_cast<const uint32_t*>(&p0);
      h[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&p1);
    }
    o0 = make_uint4(h[0], h[1], h[2], h[3]);
    o1 = make_uint4(h[4], h[5], h[6], h[7]);
  }
};

template <typename TO>
__device__ __forceinline__ void store32(TO* dst, const float* v);
template <>
__device__ __forceinline__ void store32<float>(float* dst, const float* v) {
#pragma unroll
  for (int i = 0; i < 32; i += 4)
    *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}
template <>
__device__ __forceinline__ void store32<__nv_bfloat16>(__nv_bfloat16* dst, const float* v) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(v[i + 2 * j], v[i + 2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(dst + i) = u;
  }
}
template <>
__device__ __forceinline__ void store32<__half>(__half* dst, const float* v) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 p = __floats2half2_rn(v[i + 2 * j], v[i + 2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(dst + i) = u;
  }
}

template <typename TO>
__device__ __forceinline__ void store16(TO* dst, const float* v) {
  if constexpr (std::is_same<TO, float>::value) {
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; i += 8) {
      uint4 u;
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = prefill::Pack2<TO>::run(v[i + 2 * j], v[i + 2 * j + 1]);
      *reinterpret_cast<uint4*>(dst + i) = u;
    }
  }
}

// Where the QKV epilogue (Epi 2) puts a prefill chunk's rows: columns
// [0, H*D) of the product are q, then KV*D of k, then v; row m is the token
// at position pos[m].
struct QkvRope {
  const int* pos;        // [M] cache row of each token
  const float* cos_tab;  // [tab_rows][D/2]
  const float* sin_tab;
  void* q_out;           // [M][H*D] rotated q, 16-bit
  void* k_cache;         // [n_ctx][KV][D], 16-bit
  void* v_cache;
  int tab_rows, n_ctx, H, KV, D;
};

// Q8_0 -> 16-bit rows (b2a_q8_dequant): out[r][k] = d[r][k/32] * code[r][k]
// rounded once to T, the operand values the W8 converters write.  One item =
// 16 codes (a 16-byte load, two 16-byte stores); each thread takes two items
// per round, both loads issued before either conversion, grid-strided with
// 32-bit index arithmetic (the host keeps rows * cols / 16 below 2^31).
// HBM-bound at 3 + 1/16 bytes per weight.
template <typename T>
__global__ void __launch_bounds__(256) q8_dequant_kernel(const int8_t* __restrict__ codes,
                                                         long long ldq,
                                                         const __half* __restrict__ scales,
                                                         long long lds, T* __restrict__ out,
                                                         long long ldo, int rows, int cols) {
  const unsigned per_row = static_cast<unsigned>(cols) / 16u;
  const unsigned total = static_cast<unsigned>(rows) * per_row;
  const unsigned stride = gridDim.x * blockDim.x;
  auto at = [&](unsigned i, unsigned& r, unsigned& c) {
    r = i / per_row;
    c = (i - r * per_row) * 16u;
  };
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < total; i += 2 * stride) {
    unsigned r0, c0, r1, c1;
    at(i, r0, c0);
    at(i + stride, r1, c1);
    const uint4 q0 = __ldcs(reinterpret_cast<const uint4*>(codes + r0 * ldq + c0));
    const uint4 q1 = __ldcs(reinterpret_cast<const uint4*>(codes + r1 * ldq + c1));
    const __half d0 = scales[r0 * lds + c0 / 32], d1 = scales[r1 * lds + c1 / 32];
    uint4 o0, o1;
    Dequant<T>::run(q0, Dequant<T>::scale(d0), o0, o1);
    uint4* dst = reinterpret_cast<uint4*>(out + r0 * ldo + c0);
    dst[0] = o0;
    dst[1] = o1;
    Dequant<T>::run(q1, Dequant<T>::scale(d1), o0, o1);
    dst = reinterpret_cast<uint4*>(out + r1 * ldo + c1);
    dst[0] = o0;
    dst[1] = o1;
  }
  if (i < total) {
    unsigned r, c;
    at(i, r, c);
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(codes + r * ldq + c));
    uint4 o0, o1;
    Dequant<T>::run(q, Dequant<T>::scale(scales[r * lds + c / 32]), o0, o1);
    uint4* dst = reinterpret_cast<uint4*>(out + r * ldo + c);
    dst[0] = o0;
    dst[1] = o1;
  }
}

// The CTA's work as segments (tile, first K-block, end K-block).  Tiles
// (SK false): whole tiles t = c, c + G, ...  Stream-K (SK true): the
// tiles x K-blocks iterations split evenly over the grid, so every CTA does
// the same number of MMA K-blocks whatever the tile count; a tile whose
// K range spans CTAs is summed by their epilogues' atomic adds.  Every role
// walks the same segments in the same order.
template <bool SK>
struct Work {
  int t, G, n_tiles, nk;
  long long g, g1;
  __device__ Work(int c, int G_, int n_tiles_, int nk_) : t(c), G(G_), n_tiles(n_tiles_), nk(nk_) {
    const long long total = static_cast<long long>(n_tiles_) * nk_;
    g = total * c / G_;
    g1 = total * (c + 1) / G_;
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (SK) {
      if (g >= g1) return false;
      tile = static_cast<int>(g / nk);
      kb0 = static_cast<int>(g - static_cast<long long>(tile) * nk);
      kb1 = static_cast<int>(min(static_cast<long long>(nk), kb0 + (g1 - g)));
      g += kb1 - kb0;
      return true;
    }
    if (t >= n_tiles) return false;
    tile = t;
    kb0 = 0;
    kb1 = nk;
    t += G;
    return true;
  }
};

// The same walk one K-block at a time (the converter warps look one
// K-block ahead to fetch its scales early)
template <bool SK>
struct KCursor {
  Work<SK> wk;
  int t, kb, kb1;
  bool valid;
  __device__ KCursor(int c, int G, int n_tiles, int nk) : wk(c, G, n_tiles, nk) {
    valid = wk.next(t, kb, kb1);
  }
  __device__ void advance() {
    if (++kb >= kb1) valid = wk.next(t, kb, kb1);
  }
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

template <typename T, typename TO, int Epi, int BN, bool W8>
__global__ void __launch_bounds__(threads_for(W8, conv_warps<T>()), 1) gemm_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
    const float* __restrict__ c_in, long long ldc, TO* __restrict__ out, long long ldo, int M,
    int N, int K, const QkvRope rp, const Q8W q8) {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256 && (Epi != 1 || BN == 256),
                "tile width: 64..256 columns, 256 for the SwiGLU halves");
  static_assert(Epi != 3 || std::is_same<TO, float>::value, "stream-K adds into an f32 out");
  constexpr bool kSK = Epi == 3;
  constexpr int kS = W8 ? kStagesQ8 : kStages;
  constexpr int kStage = kABytes + BN * kBK * 2;
  constexpr int kConv = W8 ? conv_warps<T>() : 0;  // converter warps 8 .. 8 + kConv - 1
  constexpr int kCodeBytes = BN * kBK;               // one code slot: BN rows x 64 codes
  constexpr int kCodesOff = kS * kStage;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kS], bar_empty[kS];
  __shared__ __align__(8) uint64_t bar_cfull[kCodeSlots], bar_cempty[kCodeSlots];
  __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2];
  __shared__ uint32_t s_tmem;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + kBM - 1) / kBM, nt = (N + BN - 1) / BN;
  const int n_tiles = mt * nt;
  const int nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    // with Q8 weights a stage is full once the A load landed and every
    // converter warp has written its rows of the weight block
    for (int s = 0; s < kS; ++s) {
      mbar_init(&bar_full[s], 1 + kConv);
      mbar_init(&bar_empty[s], 1);
    }
    if (W8) {
      for (int c = 0; c < kCodeSlots; ++c) {
        mbar_init(&bar_cfull[c], 1);
        mbar_init(&bar_cempty[c], kConv);
      }
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_acc_full[b], 1);
      mbar_init(&bar_acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // a programmatic dependent may start its prologue; the inputs of this
  // kernel come from the kernel before, so every role waits for it first
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------ TMA producer -------------------------
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      uint32_t it = 0;
      bool ok = true;
      Work<kSK> wk(blockIdx.x, gridDim.x, n_tiles, nk);
      int t, kb0, kb1;
      while (ok && wk.next(t, kb0, kb1)) {
        const int m0 = (t % mt) * kBM, n0 = (t / mt) * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kS;
          if (W8) {
            // the K-block's codes first: the converters need them before the MMA needs A
            const int c = it % kCodeSlots;
            if (it >= kCodeSlots &&
                !mbar_wait(&bar_cempty[c], ((it / kCodeSlots) & 1) ^ 1, 0x35000 | (kb & 0xfff))) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar_cfull[c], kCodeBytes);
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem + kCodesOff + c * kCodeBytes)),
                "l"(reinterpret_cast<uint64_t>(&tmW)), "r"(kb * kBK), "r"(n0),
                "r"(smem_u32(&bar_cfull[c]))
                : "memory");
          }
          if (it >= kS && !mbar_wait(&bar_empty[s], ((it / kS) & 1) ^ 1, 0x31000 | (kb & 0xfff))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar_full[s], W8 ? kABytes : kStage);
          uint8_t* sa = smem + s * kStage;
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(sa)),
              "l"(reinterpret_cast<uint64_t>(&tmA)), "r"(kb * kBK), "r"(m0),
              "r"(smem_u32(&bar_full[s]))
              : "memory");
          if (!W8)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(sa + kABytes)),
                "l"(reinterpret_cast<uint64_t>(&tmW)), "r"(kb * kBK), "r"(n0),
                "r"(smem_u32(&bar_full[s]))
                : "memory");
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------ MMA issuer ---------------------------
      constexpr uint32_t idesc = make_idesc<T>(kBM, BN, false, false);
      const uint64_t dA0 = sw128_desc(smem_u32(smem), 16, 1024);
      const uint64_t dW0 = sw128_desc(smem_u32(smem + kABytes), 16, 1024);
      constexpr uint64_t kStageStep = kStage >> 4;
      uint32_t it = 0, tc = 0;
      bool ok = true;
      Work<kSK> wk(blockIdx.x, gridDim.x, n_tiles, nk);
      int t, kb0, kb1;
      for (; ok && wk.next(t, kb0, kb1); ++tc) {
        const uint32_t b = tc & 1;
        // the epilogue has drained this accumulator (two tiles ago)
        if (tc >= 2 && !mbar_wait(&bar_acc_empty[b], ((tc >> 1) - 1) & 1, 0x32000 | (tc & 0xfff))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * kAccStride;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kS;
          if (!mbar_wait(&bar_full[s], (it / kS) & 1, 0x33000 | (kb & 0xfff))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = dA0 + s * kStageStep, dw = dW0 + s * kStageStep;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)  // 32 bytes of K per MMA inside the swizzle atom
            tc_mma(acc, da + ((kk * 32) >> 4), dw + ((kk * 32) >> 4), idesc,
                   (kb != kb0 || kk != 0) ? 1u : 0u);
          tc_commit(&bar_empty[s]);
        }
        if (ok) tc_commit(&bar_acc_full[b]);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------ epilogue --------------------------------
    const int q = warp & 3;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t tc = 0;
    Work<kSK> wk(blockIdx.x, gridDim.x, n_tiles, nk);
    int t, kb0, kb1;
    for (; wk.next(t, kb0, kb1); ++tc) {
      const uint32_t b = tc & 1;
      const bool w = __all_sync(0xffffffffu,
                                mbar_wait(&bar_acc_full[b], (tc >> 1) & 1, 0x34000 | (tc & 0xfff)));
      if (!w) break;
      tc_fence_after();
      const int m0 = (t % mt) * kBM, n0 = (t / mt) * BN;
      const int row = m0 + q * 32 + lane;
      const bool rv = row < M;
      const uint32_t acc = tl + b * kAccStride;
      if (Epi == 0) {
        // the residual of chunk c + 1 is in flight while chunk c is added and
        // stored (one global round trip per tile instead of one per chunk)
        const float* crow = c_in + static_cast<size_t>(row) * ldc;
        auto full = [&](int c) { return rv && n0 + c * 32 + 32 <= N; };
        float4 rc[8], rn[8];
        if (c_in && full(0)) {
#pragma unroll
          for (int i = 0; i < 8; ++i) rc[i] = *reinterpret_cast<const float4*>(crow + n0 + 4 * i);
        }
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tc_ld32(acc + c * 32, v);
          if (c + 1 < BN / 32 && c_in && full(c + 1)) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              rn[i] = *reinterpret_cast<const float4*>(crow + n0 + (c + 1) * 32 + 4 * i);
          }
          tc_wait_ld();
          const int col = n0 + c * 32;
          if (rv && col < N) {
            if (col + 32 <= N) {
              if (c_in) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  v[4 * i] += rc[i].x;
                  v[4 * i + 1] += rc[i].y;
                  v[4 * i + 2] += rc[i].z;
                  v[4 * i + 3] += rc[i].w;
                }
              }
              store32<TO>(out + static_cast<size_t>(row) * ldo + col, v);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                if (col + i < N) {
                  float x = v[i];
                  if (c_in) x += c_in[static_cast<size_t>(row) * ldc + col + i];
                  st_elem(out + static_cast<size_t>(row) * ldo + col + i, x);
                }
              }
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) rc[i] = rn[i];
        }
      } else if (Epi == 3) {
        // stream-K: this segment's partial sum is added into out (which
        // already holds the residual); the tile's other segments add theirs
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tc_ld32(acc + c * 32, v);
          tc_wait_ld();
          const int col = n0 + c * 32;
          if (rv && col < N) {
            float* dst = reinterpret_cast<float*>(out) + static_cast<size_t>(row) * ldo + col;
            if (col + 32 <= N) {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                red_add_v4(dst + 4 * i, v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col + i < N) atomicAdd(dst + i, v[i]);
            }
          }
        }
      } else if (Epi == 2) {
        // RoPE (norm style, pairs 2i, 2i+1 of a head: adjacent columns of this
        // thread's row, the reference's f32 products, model.py:1162-1209),
        // then q into q_out and k, v into the cache row at the token's
        // position (model.py:1335-1337); D % 32 == 0, so a 32-column chunk
        // lies inside one head
        const int qd = rp.H * rp.D, kd = rp.KV * rp.D, half = rp.D >> 1;
        int p = -1;
        if (rv) {
          p = rp.pos[row];
          if (p < 0 || p >= rp.n_ctx || p >= rp.tab_rows) {
            set_dev_error(B2A_ERR_POSITION, row);
            p = -1;
          }
        }
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n0 + c * 32;
          if (col >= N) break;
          float v[32];
          tc_ld32(acc + c * 32, v);
          // this row's 16 cos and 16 sin entries (64 aligned bytes each),
          // fetched while the accumulator chunk comes out of TMEM
          const bool rot = p >= 0 && col < qd + kd;
          float4 cs4[4], sn4[4];
          if (rot) {
            const size_t at = static_cast<size_t>(p) * half + ((col % rp.D) >> 1);
            const float4* ct = reinterpret_cast<const float4*>(rp.cos_tab + at);
            const float4* st = reinterpret_cast<const float4*>(rp.sin_tab + at);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              cs4[i] = ct[i];
              sn4[i] = st[i];
            }
          }
          tc_wait_ld();
          if (p >= 0) {
            if (rot) {
              const float* cs = reinterpret_cast<const float*>(cs4);
              const float* sn = reinterpret_cast<const float*>(sn4);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float x0 = v[2 * i], x1 = v[2 * i + 1];
                v[2 * i] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
                v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
              }
            }
            TO* dst = col < qd ? static_cast<TO*>(rp.q_out) + static_cast<size_t>(row) * qd + col
                      : col < qd + kd
                          ? static_cast<TO*>(rp.k_cache) + static_cast<size_t>(p) * kd + (col - qd)
                          : static_cast<TO*>(rp.v_cache) + static_cast<size_t>(p) * kd +
                                (col - qd - kd);
            store32<TO>(dst, v);
          }
        }
      } else if (Epi == 4) {
        // SwiGLU on 16-row groups of 8 gate rows then the matching 8 up rows
        // (the decode GEMV's layout of the FFN matrix): a 32-column chunk
        // holds two groups and gives 16 consecutive outputs
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n0 / 2 + c * 16;
          if (col >= N / 2) break;
          float v[32], g[16];
          tc_ld32(acc + c * 32, v);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            g[i] = v[i] / (1.f + expf(-v[i])) * v[8 + i];
            g[8 + i] = v[16 + i] / (1.f + expf(-v[16 + i])) * v[24 + i];
          }
          if (rv) {
            TO* dst = out + static_cast<size_t>(row) * ldo + col;
            if (col + 16 <= N / 2) {
              store16<TO>(dst, g);
            } else {  // the matrix ends after the chunk's first group (N % 32 == 16)
#pragma unroll
              for (int i = 0; i < 8; ++i) st_elem(dst + i, g[i]);
            }
          }
        }
      } else {
        // SwiGLU: columns [0,128) of the tile are gate rows, [128,256) the up rows
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          float g[32], u[32];
          tc_ld32(acc + c * 32, g);
          tc_ld32(acc + 128 + c * 32, u);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) g[i] = g[i] / (1.f + expf(-g[i])) * u[i];
          const int col = n0 / 2 + c * 32;
          if (rv) store32<TO>(out + static_cast<size_t>(row) * ldo + col, g);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_acc_empty[b]);
    }
  } else if (W8 && warp >= 8) {
    // ------------------------------ Q8 converters ------------------------------
    // Each K-block: the codes slot (BN rows x 64 codes, row-major) becomes
    // the stage's 16-bit weight block in the 128-byte-swizzled K-major layout
    // the MMA reads (16-byte chunk j of row r at chunk j ^ (r % 8)).  A
    // thread takes 16 codes (a quarter row) per item; a warp's loads cover
    // 512 contiguous bytes and each quarter-warp's stores one 128-byte line
    // per row pair, so neither side has bank conflicts.
    using DQ = Dequant<T>;
    using Sc = typename DQ::Scale;
    constexpr int kCT = 32 * (W8 ? kConv : 4);  // (the non-W8 instantiation never runs this)
    constexpr int kItems = BN * 4 / kCT;
    static_assert(BN * 4 % kCT == 0, "converter items");
    const int ct = static_cast<int>(threadIdx.x) - 8 * 32;
    const int qd = ct & 3, r0 = ct >> 2;
    KCursor<kSK> cur(blockIdx.x, gridDim.x, n_tiles, nk);
    KCursor<kSK> nxt = cur;
    if (nxt.valid) nxt.advance();
    // the scales of a K-block (one per item: its row and 32-code block),
    // fetched one K-block ahead
    auto load_scales = [&](const KCursor<kSK>& k, Sc* d) {
      const int n0 = (k.t / mt) * BN, blk = 2 * k.kb + (qd >> 1);
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int n = n0 + r0 + (kCT / 4) * i;
        d[i] = DQ::scale(n < N && blk < q8.nblk ? q8.scales[static_cast<size_t>(n) * q8.lds + blk]
                                                : __ushort_as_half(0));
      }
    };
    // One K-block: wait for its codes and a free stage, load every item's
    // codes first (the loads then overlap; the stores below could alias
    // them as far as the compiler knows), convert, store, release.  `d`
    // holds this K-block's scales; the next K-block's go into `dn`, so a
    // scale load has a whole K-block of work to arrive in.  Returns false
    // when the walk ends or a wait gave up.
    uint32_t it = 0;
    auto step = [&](Sc* d, Sc* dn) -> bool {
      if (!cur.valid) return false;
      if (nxt.valid) load_scales(nxt, dn);
      const int s = it % kS, c = it % kCodeSlots;
      bool w = mbar_wait(&bar_cfull[c], (it / kCodeSlots) & 1, 0x36000 | (cur.kb & 0xfff));
      if (w && it >= kS) w = mbar_wait(&bar_empty[s], ((it / kS) & 1) ^ 1, 0x37000 | (cur.kb & 0xfff));
      if (!__all_sync(0xffffffffu, w)) return false;
      const uint8_t* cs = smem + kCodesOff + c * kCodeBytes;
      uint8_t* ws = smem + s * kStage + kABytes;
      uint4 cv[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i)
        cv[i] = *reinterpret_cast<const uint4*>(cs + (r0 + (kCT / 4) * i) * kBK + qd * 16);
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int r = r0 + (kCT / 4) * i;
        uint4 o0, o1;
        DQ::run(cv[i], d[i], o0, o1);
        *reinterpret_cast<uint4*>(ws + r * 128 + (((2 * qd) ^ (r & 7)) << 4)) = o0;
        *reinterpret_cast<uint4*>(ws + r * 128 + (((2 * qd + 1) ^ (r & 7)) << 4)) = o1;
      }
      // the MMA reads the block through the async proxy
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar_full[s]);
        mbar_arrive(&bar_cempty[c]);
      }
      cur = nxt;
      if (nxt.valid) nxt.advance();
      ++it;
      return true;
    };
    Sc da[kItems], db[kItems];
    if (cur.valid) load_scales(cur, da);
    // two steps per turn, so the scale buffers swap roles without copies
    while (step(da, db) && step(db, da)) {
    }
  }
  // ------------------------------ teardown -----------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

}  // namespace gemm
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

template <typename T, typename TO, int Epi, int BN = 256>
int launch_gemm(const void* a, long long lda, const void* w, long long ldw, const float* c_in,
                long long ldc, void* out, long long ldo, int M, int N, int K, cudaStream_t st,
                const b2a::gemm::QkvRope& rp = b2a::gemm::QkvRope{}) {
  namespace G = b2a::gemm;
  auto kern = G::gemm_kernel<T, TO, Epi, BN, false>;
  const CUtensorMapDataType tdt = std::is_same<T, __nv_bfloat16>::value
                                      ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tw;
  const uint64_t adims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  const uint64_t astr[1] = {static_cast<uint64_t>(lda) * 2};
  const uint64_t wdims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint64_t wstr[1] = {static_cast<uint64_t>(ldw) * 2};
  const uint32_t abox[2] = {static_cast<uint32_t>(G::kBK), static_cast<uint32_t>(G::kBM)};
  const uint32_t wbox[2] = {static_cast<uint32_t>(G::kBK), static_cast<uint32_t>(BN)};
  int rc = b2a_host::make_tmap(&ta, tdt, 2, const_cast<void*>(a), adims, astr, abox,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tw, tdt, 2, const_cast<void*>(w), wdims, wstr, wbox,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  constexpr int smem_bytes = G::smem_for(BN);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(gemm)");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((M + G::kBM - 1) / G::kBM) * ((N + BN - 1) / BN);
  int grid = tiles < sms ? tiles : sms;
  if (Epi == 3) {  // stream-K: every SM, each with at least one K-block
    const long long iters = static_cast<long long>(tiles) * ((K + G::kBK - 1) / G::kBK);
    grid = iters < sms ? static_cast<int>(iters) : sms;
  }
  e = b2a_host::launch(kern, dim3(grid), dim3(G::kThreads), smem_bytes, st, ta, tw, c_in, ldc,
                       static_cast<TO*>(out), ldo, M, N, K, rp, G::Q8W{nullptr, 0, 0});
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "gemm launch");
  return B2A_OK;
}

// The same GEMM with Q8_0 weights: codes int8 [N][ldq] through a tensor map
// (64-code x BN-row boxes, no swizzle), scales f16 [N][lds] read by the
// kernel's converter warps.
template <typename T, typename TO, int Epi, int BN>
int launch_gemm_q8(const void* a, long long lda, const void* codes, long long ldq,
                   const void* scales, long long lds, const float* c_in, long long ldc, void* out,
                   long long ldo, int M, int N, int K, cudaStream_t st,
                   const b2a::gemm::QkvRope& rp) {
  namespace G = b2a::gemm;
  auto kern = G::gemm_kernel<T, TO, Epi, BN, true>;
  const CUtensorMapDataType tdt = std::is_same<T, __nv_bfloat16>::value
                                      ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tq;
  const uint64_t adims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  const uint64_t astr[1] = {static_cast<uint64_t>(lda) * 2};
  const uint64_t qdims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint64_t qstr[1] = {static_cast<uint64_t>(ldq)};
  const uint32_t abox[2] = {static_cast<uint32_t>(G::kBK), static_cast<uint32_t>(G::kBM)};
  const uint32_t qbox[2] = {static_cast<uint32_t>(G::kBK), static_cast<uint32_t>(BN)};
  int rc = b2a_host::make_tmap(&ta, tdt, 2, const_cast<void*>(a), adims, astr, abox,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(codes), qdims,
                           qstr, qbox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  constexpr int smem_bytes = G::smem_for(BN, true);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(gemm_q8)");
  const int sms = b2a_host::sm_count();
  const int tiles = ((M + G::kBM - 1) / G::kBM) * ((N + BN - 1) / BN);
  int grid = tiles < sms ? tiles : sms;
  if (Epi == 3) {
    const long long iters = static_cast<long long>(tiles) * ((K + G::kBK - 1) / G::kBK);
    grid = iters < sms ? static_cast<int>(iters) : sms;
  }
  const G::Q8W q8{static_cast<const __half*>(scales), lds, K / 32};
  e = b2a_host::launch(kern, dim3(grid), dim3(G::threads_for(true, G::conv_warps<T>())),
                       smem_bytes, st, ta, tq, c_in, ldc, static_cast<TO*>(out), ldo, M, N, K, rp,
                       q8);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "gemm_q8 launch");
  return B2A_OK;
}

// 192-column tiles where they need fewer tile-widths of waves than 256:
// (waves of tiles over the SMs) x (tile width); e.g. 2048 x 3072 on 148
// SMs is 2 x 192 against 2 x 256, 2048 x 2048 is 2 x 192 against 1 x 256
bool narrow_tiles(int M, int N) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto cost = [&](int bn) {
    const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + bn - 1) / bn);
    return (tiles + sms - 1) / sms * bn;
  };
  return cost(192) < cost(256);
}

// Stream-K for an in-place f32 residual GEMM (out += a . w^T) whose tiles
// leave SMs idle: at most two waves of 128 x 256 tiles that do not fill the
// last one (the chunk's Wo and down projections: 128 tiles on 148 SMs).
bool use_stream_k(int M, int N) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + 255) / 256);
  return tiles < 2LL * sms && tiles % sms != 0;
}

template <typename T, typename TO, int Epi>
int launch_gemm_auto(const void* a, long long lda, const void* w, long long ldw,
                     const float* c_in, long long ldc, void* out, long long ldo, int M, int N,
                     int K, cudaStream_t st,
                     const b2a::gemm::QkvRope& rp = b2a::gemm::QkvRope{}) {
  if constexpr (Epi == 0 && std::is_same<TO, float>::value) {
    if (c_in != nullptr && static_cast<const void*>(c_in) == out && ldc == ldo &&
        use_stream_k(M, N))
      return launch_gemm<T, float, 3, 256>(a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st, rp);
  }
  if (Epi != 1 && narrow_tiles(M, N))
    return launch_gemm<T, TO, Epi, (Epi == 1 ? 256 : 192)>(a, lda, w, ldw, c_in, ldc, out, ldo, M,
                                                           N, K, st, rp);
  return launch_gemm<T, TO, Epi, 256>(a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st, rp);
}

template <typename T, typename TO, int Epi>
int launch_gemm_q8_auto(const void* a, long long lda, const void* codes, long long ldq,
                        const void* scales, long long lds, const float* c_in, long long ldc,
                        void* out, long long ldo, int M, int N, int K, cudaStream_t st,
                        const b2a::gemm::QkvRope& rp = b2a::gemm::QkvRope{}) {
  if constexpr (Epi == 0 && std::is_same<TO, float>::value) {
    if (c_in != nullptr && static_cast<const void*>(c_in) == out && ldc == ldo &&
        use_stream_k(M, N))
      return launch_gemm_q8<T, float, 3, 256>(a, lda, codes, ldq, scales, lds, c_in, ldc, out,
                                              ldo, M, N, K, st, rp);
  }
  if (Epi != 1 && narrow_tiles(M, N))
    return launch_gemm_q8<T, TO, Epi, (Epi == 1 ? 256 : 192)>(a, lda, codes, ldq, scales, lds,
                                                              c_in, ldc, out, ldo, M, N, K, st, rp);
  return launch_gemm_q8<T, TO, Epi, 256>(a, lda, codes, ldq, scales, lds, c_in, ldc, out, ldo, M,
                                         N, K, st, rp);
}

template <typename T, int Epi>
int gemm_q8_out(int out_dtype, const void* a, long long lda, const void* codes, long long ldq,
                const void* scales, long long lds, const float* c_in, long long ldc, void* out,
                long long ldo, int M, int N, int K, cudaStream_t st) {
  switch (out_dtype) {
    case B2A_F32:
      return launch_gemm_q8_auto<T, float, Epi>(a, lda, codes, ldq, scales, lds, c_in, ldc, out,
                                                ldo, M, N, K, st);
    case B2A_F16:
      return launch_gemm_q8_auto<T, __half, Epi>(a, lda, codes, ldq, scales, lds, c_in, ldc, out,
                                                 ldo, M, N, K, st);
    case B2A_BF16:
      return launch_gemm_q8_auto<T, __nv_bfloat16, Epi>(a, lda, codes, ldq, scales, lds, c_in,
                                                        ldc, out, ldo, M, N, K, st);
  }
  return b2a_host::fail(B2A_ERR_DTYPE, "gemm_q8: out_dtype %d", out_dtype);
}

// Argument checks shared by the Q8_0 entry points
int check_q8(const void* codes, long long ldq, const void* scales, long long lds, int N, int K,
             const char* who) {
  using b2a_host::fail;
  if (!codes || !scales) return fail(B2A_ERR_ARG, "%s: null codes or scales", who);
  if (K % 32) return fail(B2A_ERR_SHAPE, "%s: K=%d is not a multiple of 32", who, K);
  if (ldq < K || ldq % 16 || lds < K / 32)
    return fail(B2A_ERR_ALIGN, "%s: ldq must be >= K and a multiple of 16, lds >= K/32", who);
  if (!b2a_host::aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 1))
    return fail(B2A_ERR_ALIGN, "%s: codes must be 16-byte and scales 2-byte aligned", who);
  (void)N;
  return B2A_OK;
}

template <typename T, int Epi>
int gemm_out(int out_dtype, const void* a, long long lda, const void* w, long long ldw,
             const float* c_in, long long ldc, void* out, long long ldo, int M, int N, int K,
             cudaStream_t st) {
  switch (out_dtype) {
    case B2A_F32:
      return launch_gemm_auto<T, float, Epi>(a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    case B2A_F16:
      return launch_gemm_auto<T, __half, Epi>(a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    case B2A_BF16:
      return launch_gemm_auto<T, __nv_bfloat16, Epi>(a, lda, w, ldw, c_in, ldc, out, ldo, M, N,
                                                     K, st);
  }
  return b2a_host::fail(B2A_ERR_DTYPE, "gemm: out_dtype %d", out_dtype);
}

}  // namespace

extern "C" {

int b2a_gemm(const void* a, long long lda, const void* w, long long ldw, int dtype,
             const float* c_in, long long ldc, void* out, long long ldo, int out_dtype, int M,
             int N, int K, int epilogue, void* stream) {
  using b2a_host::fail;
  if (!a || !w || !out) return fail(B2A_ERR_ARG, "gemm: null pointer argument");
  if (M <= 0 || N <= 0 || K <= 0) return fail(B2A_ERR_SHAPE, "gemm: M=%d N=%d K=%d", M, N, K);
  if (lda < K || ldw < K || (lda & 7) || (ldw & 7))
    return fail(B2A_ERR_ALIGN, "gemm: lda/ldw must be >= K and multiples of 8 elements");
  if (!b2a_host::aligned16(a) || !b2a_host::aligned16(w) || !b2a_host::aligned16(out) ||
      (c_in && !b2a_host::aligned16(c_in)))
    return fail(B2A_ERR_ALIGN, "gemm: a, w, c_in and out must be 16-byte aligned");
  if (epilogue != B2A_GEMM_STORE && epilogue != B2A_GEMM_SWIGLU && epilogue != B2A_GEMM_SWIGLU8)
    return fail(B2A_ERR_ARG, "gemm: epilogue %d", epilogue);
  const int out_cols = epilogue != B2A_GEMM_STORE ? N / 2 : N;
  if (ldo < out_cols || (c_in && ldc < N))
    return fail(B2A_ERR_SHAPE, "gemm: ldo/ldc smaller than the row");
  const int eb = b2a_host::elem_size(out_dtype);
  if (eb == 0) return fail(B2A_ERR_DTYPE, "gemm: out_dtype %d", out_dtype);
  if ((ldo * eb) % 16 || (c_in && (ldc % 4)))
    return fail(B2A_ERR_ALIGN, "gemm: output and c_in rows must start on 16-byte boundaries");
  if (epilogue == B2A_GEMM_SWIGLU && (N % 256 || c_in))
    return fail(B2A_ERR_SHAPE, "gemm: SWIGLU needs N a multiple of 256 and no c_in");
  if (epilogue == B2A_GEMM_SWIGLU8 && (N % 16 || c_in))
    return fail(B2A_ERR_SHAPE, "gemm: SWIGLU8 needs N a multiple of 16 and no c_in");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == B2A_BF16) {
    if (epilogue == B2A_GEMM_SWIGLU)
      return gemm_out<__nv_bfloat16, 1>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    if (epilogue == B2A_GEMM_SWIGLU8)
      return gemm_out<__nv_bfloat16, 4>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    return gemm_out<__nv_bfloat16, 0>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
  }
  if (dtype == B2A_F16) {
    if (epilogue == B2A_GEMM_SWIGLU)
      return gemm_out<__half, 1>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    if (epilogue == B2A_GEMM_SWIGLU8)
      return gemm_out<__half, 4>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
    return gemm_out<__half, 0>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
  }
  return fail(B2A_ERR_DTYPE, "gemm: operand dtype %d (f16 or bf16)", dtype);
}

int b2a_gemm_qkv_rope(const void* a, long long lda, const void* w, long long ldw, int dtype,
                      int M, int K, const int* pos_dev, const float* cos_tab, const float* sin_tab,
                      int tab_rows, int H, int KV, int D, void* q_out, void* k_cache,
                      void* v_cache, int n_ctx, void* stream) {
  using b2a_host::fail;
  if (!a || !w || !pos_dev || !cos_tab || !sin_tab || !q_out || !k_cache || !v_cache)
    return fail(B2A_ERR_ARG, "gemm_qkv_rope: null pointer argument");
  if (M <= 0 || K <= 0 || H <= 0 || KV <= 0 || n_ctx <= 0 || tab_rows <= 0)
    return fail(B2A_ERR_SHAPE, "gemm_qkv_rope: M=%d K=%d H=%d KV=%d", M, K, H, KV);
  if (D <= 0 || D % 32)
    return fail(B2A_ERR_UNSUPPORTED, "gemm_qkv_rope: head_dim %d (a multiple of 32)", D);
  if (lda < K || ldw < K || (lda & 7) || (ldw & 7))
    return fail(B2A_ERR_ALIGN, "gemm_qkv_rope: lda/ldw must be >= K and multiples of 8");
  if (!b2a_host::aligned16(a) || !b2a_host::aligned16(w) || !b2a_host::aligned16(q_out) ||
      !b2a_host::aligned16(k_cache) || !b2a_host::aligned16(v_cache) ||
      !b2a_host::aligned16(cos_tab) || !b2a_host::aligned16(sin_tab))
    return fail(B2A_ERR_ALIGN,
                "gemm_qkv_rope: a, w, q_out, the caches and the tables must be 16-byte aligned");
  const int N = (H + 2 * KV) * D;
  const b2a::gemm::QkvRope rp{pos_dev, cos_tab, sin_tab, q_out, k_cache, v_cache,
                              tab_rows, n_ctx, H, KV, D};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == B2A_BF16)
    return launch_gemm_auto<__nv_bfloat16, __nv_bfloat16, 2>(a, lda, w, ldw, nullptr, 0, nullptr,
                                                             0, M, N, K, st, rp);
  if (dtype == B2A_F16)
    return launch_gemm_auto<__half, __half, 2>(a, lda, w, ldw, nullptr, 0, nullptr, 0, M, N, K, st,
                                               rp);
  return fail(B2A_ERR_DTYPE, "gemm_qkv_rope: dtype %d (f16 or bf16)", dtype);
}


int b2a_gemm_q8(const void* a, long long lda, const void* codes, long long ldq,
                const void* scales, long long lds, int dtype, const float* c_in, long long ldc,
                void* out, long long ldo, int out_dtype, int M, int N, int K, int epilogue,
                void* stream) {
  using b2a_host::fail;
  if (!a || !out) return fail(B2A_ERR_ARG, "gemm_q8: null pointer argument");
  if (M <= 0 || N <= 0 || K <= 0) return fail(B2A_ERR_SHAPE, "gemm_q8: M=%d N=%d K=%d", M, N, K);
  int rc = check_q8(codes, ldq, scales, lds, N, K, "gemm_q8");
  if (rc) return rc;
  if (lda < K || (lda & 7))
    return fail(B2A_ERR_ALIGN, "gemm_q8: lda must be >= K and a multiple of 8 elements");
  if (!b2a_host::aligned16(a) || !b2a_host::aligned16(out) ||
      (c_in && !b2a_host::aligned16(c_in)))
    return fail(B2A_ERR_ALIGN, "gemm_q8: a, c_in and out must be 16-byte aligned");
  if (epilogue != B2A_GEMM_STORE && epilogue != B2A_GEMM_SWIGLU && epilogue != B2A_GEMM_SWIGLU8)
    return fail(B2A_ERR_ARG, "gemm_q8: epilogue %d", epilogue);
  const bool glu = epilogue != B2A_GEMM_STORE;
  const int out_cols = glu ? N / 2 : N;
  if (ldo < out_cols || (c_in && ldc < N))
    return fail(B2A_ERR_SHAPE, "gemm_q8: ldo/ldc smaller than the row");
  const int eb = b2a_host::elem_size(out_dtype);
  if (eb == 0) return fail(B2A_ERR_DTYPE, "gemm_q8: out_dtype %d", out_dtype);
  if ((ldo * eb) % 16 || (c_in && (ldc % 4)))
    return fail(B2A_ERR_ALIGN, "gemm_q8: output and c_in rows must start on 16-byte boundaries");
  if (epilogue == B2A_GEMM_SWIGLU && (N % 256 || c_in))
    return fail(B2A_ERR_SHAPE, "gemm_q8: SWIGLU needs N a multiple of 256 and no c_in");
  if (epilogue == B2A_GEMM_SWIGLU8 && (N % 16 || c_in))
    return fail(B2A_ERR_SHAPE, "gemm_q8: SWIGLU8 needs N a multiple of 16 and no c_in");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == B2A_BF16) {
    if (epilogue == B2A_GEMM_SWIGLU)
      return gemm_q8_out<__nv_bfloat16, 1>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc,
                                           out, ldo, M, N, K, st);
    if (epilogue == B2A_GEMM_SWIGLU8)
      return gemm_q8_out<__nv_bfloat16, 4>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc,
                                           out, ldo, M, N, K, st);
    return gemm_q8_out<__nv_bfloat16, 0>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc,
                                         out, ldo, M, N, K, st);
  }
  if (dtype == B2A_F16) {
    if (epilogue == B2A_GEMM_SWIGLU)
      return gemm_q8_out<__half, 1>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc, out,
                                    ldo, M, N, K, st);
    if (epilogue == B2A_GEMM_SWIGLU8)
      return gemm_q8_out<__half, 4>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc, out,
                                    ldo, M, N, K, st);
    return gemm_q8_out<__half, 0>(out_dtype, a, lda, codes, ldq, scales, lds, c_in, ldc, out, ldo,
                                  M, N, K, st);
  }
  return fail(B2A_ERR_DTYPE, "gemm_q8: operand dtype %d (f16 or bf16)", dtype);
}

int b2a_gemm_qkv_rope_q8(const void* a, long long lda, const void* codes, long long ldq,
                         const void* scales, long long lds, int dtype, int M, int K,
                         const int* pos_dev, const float* cos_tab, const float* sin_tab,
                         int tab_rows, int H, int KV, int D, void* q_out, void* k_cache,
                         void* v_cache, int n_ctx, void* stream) {
  using b2a_host::fail;
  if (!a || !pos_dev || !cos_tab || !sin_tab || !q_out || !k_cache || !v_cache)
    return fail(B2A_ERR_ARG, "gemm_qkv_rope_q8: null pointer argument");
  if (M <= 0 || K <= 0 || H <= 0 || KV <= 0 || n_ctx <= 0 || tab_rows <= 0)
    return fail(B2A_ERR_SHAPE, "gemm_qkv_rope_q8: M=%d K=%d H=%d KV=%d", M, K, H, KV);
  if (D <= 0 || D % 32)
    return fail(B2A_ERR_UNSUPPORTED, "gemm_qkv_rope_q8: head_dim %d (a multiple of 32)", D);
  const int N = (H + 2 * KV) * D;
  int rc = check_q8(codes, ldq, scales, lds, N, K, "gemm_qkv_rope_q8");
  if (rc) return rc;
  if (lda < K || (lda & 7))
    return fail(B2A_ERR_ALIGN, "gemm_qkv_rope_q8: lda must be >= K and a multiple of 8");
  if (!b2a_host::aligned16(a) || !b2a_host::aligned16(q_out) || !b2a_host::aligned16(k_cache) ||
      !b2a_host::aligned16(v_cache) || !b2a_host::aligned16(cos_tab) ||
      !b2a_host::aligned16(sin_tab))
    return fail(B2A_ERR_ALIGN,
                "gemm_qkv_rope_q8: a, q_out, the caches and the tables must be 16-byte aligned");
  const b2a::gemm::QkvRope rp{pos_dev, cos_tab, sin_tab, q_out, k_cache, v_cache,
                              tab_rows, n_ctx, H, KV, D};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == B2A_BF16)
    return launch_gemm_q8_auto<__nv_bfloat16, __nv_bfloat16, 2>(
        a, lda, codes, ldq, scales, lds, nullptr, 0, nullptr, 0, M, N, K, st, rp);
  if (dtype == B2A_F16)
    return launch_gemm_q8_auto<__half, __half, 2>(a, lda, codes, ldq, scales, lds, nullptr, 0,
                                                  nullptr, 0, M, N, K, st, rp);
  return fail(B2A_ERR_DTYPE, "gemm_qkv_rope_q8: dtype %d (f16 or bf16)", dtype);
}


int b2a_q8_dequant(const void* codes, long long ldq, const void* scales, long long lds,
                   void* out, long long ldo, int dtype, int rows, int cols, void* stream) {
  using b2a_host::fail;
  if (!out) return fail(B2A_ERR_ARG, "q8_dequant: null output");
  if (rows <= 0 || cols <= 0) return fail(B2A_ERR_SHAPE, "q8_dequant: rows=%d cols=%d", rows, cols);
  int rc = check_q8(codes, ldq, scales, lds, rows, cols, "q8_dequant");
  if (rc) return rc;
  if (ldo < cols || ldo % 8 || !b2a_host::aligned16(out))
    return fail(B2A_ERR_ALIGN, "q8_dequant: out 16-byte aligned, ldo >= cols and a multiple of 8");
  const long long work = static_cast<long long>(rows) * (cols / 16);
  if (work >= (1LL << 31)) return fail(B2A_ERR_SHAPE, "q8_dequant: %d x %d is too large", rows, cols);
  long long blocks = (work + 511) / 512;  // two items per thread
  const long long cap = static_cast<long long>(b2a_host::sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int8_t* q = static_cast<const int8_t*>(codes);
  const __half* sc = static_cast<const __half*>(scales);
  if (dtype == B2A_F16)
    b2a::gemm::q8_dequant_kernel<__half><<<static_cast<int>(blocks), 256, 0, st>>>(
        q, ldq, sc, lds, static_cast<__half*>(out), ldo, rows, cols);
  else if (dtype == B2A_BF16)
    b2a::gemm::q8_dequant_kernel<__nv_bfloat16><<<static_cast<int>(blocks), 256, 0, st>>>(
        q, ldq, sc, lds, static_cast<__nv_bfloat16*>(out), ldo, rows, cols);
  else
    return fail(B2A_ERR_DTYPE, "q8_dequant: dtype %d (f16 or bf16)", dtype);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "q8_dequant launch");
  return B2A_OK;
}

}  // extern "C"
