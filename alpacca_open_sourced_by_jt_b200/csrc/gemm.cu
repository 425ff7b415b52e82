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
// activation the down projection reads (model.py:1352-1354).
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
// A stage is the A block plus a BN x 64 weight block (32 KB at BN = 256)
constexpr int smem_for(int bn) { return kStages * (kABytes + bn * kBK * 2) + 1024; }
constexpr uint32_t kTmemCols = 512;  // two accumulators of up to 256 columns
constexpr uint32_t kAccStride = 256;

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

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

template <typename T, typename TO, int Epi, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
    const float* __restrict__ c_in, long long ldc, TO* __restrict__ out, long long ldo, int M,
    int N, int K, const QkvRope rp) {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256 && (Epi != 1 || BN == 256),
                "tile width: 64..256 columns, 256 for the SwiGLU halves");
  static_assert(Epi != 3 || std::is_same<TO, float>::value, "stream-K adds into an f32 out");
  constexpr bool kSK = Epi == 3;
  constexpr int kStage = kABytes + BN * kBK * 2;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2];
  __shared__ uint32_t s_tmem;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + kBM - 1) / kBM, nt = (N + BN - 1) / BN;
  const int n_tiles = mt * nt;
  const int nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
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
          const int s = it % kStages;
          if (it >= kStages &&
              !mbar_wait(&bar_empty[s], ((it / kStages) & 1) ^ 1, 0x31000 | (kb & 0xfff))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar_full[s], kStage);
          uint8_t* sa = smem + s * kStage;
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(sa)),
              "l"(reinterpret_cast<uint64_t>(&tmA)), "r"(kb * kBK), "r"(m0),
              "r"(smem_u32(&bar_full[s]))
              : "memory");
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
          const int s = it % kStages;
          if (!mbar_wait(&bar_full[s], (it / kStages) & 1, 0x33000 | (kb & 0xfff))) {
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
  } else if (warp >= 4) {
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
  auto kern = G::gemm_kernel<T, TO, Epi, BN>;
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
                       static_cast<TO*>(out), ldo, M, N, K, rp);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "gemm launch");
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
  if (epilogue != B2A_GEMM_STORE && epilogue != B2A_GEMM_SWIGLU)
    return fail(B2A_ERR_ARG, "gemm: epilogue %d", epilogue);
  const int out_cols = epilogue == B2A_GEMM_SWIGLU ? N / 2 : N;
  if (ldo < out_cols || (c_in && ldc < N))
    return fail(B2A_ERR_SHAPE, "gemm: ldo/ldc smaller than the row");
  const int eb = b2a_host::elem_size(out_dtype);
  if (eb == 0) return fail(B2A_ERR_DTYPE, "gemm: out_dtype %d", out_dtype);
  if ((ldo * eb) % 16 || (c_in && (ldc % 4)))
    return fail(B2A_ERR_ALIGN, "gemm: output and c_in rows must start on 16-byte boundaries");
  if (epilogue == B2A_GEMM_SWIGLU && (N % 256 || c_in))
    return fail(B2A_ERR_SHAPE, "gemm: SWIGLU needs N a multiple of 256 and no c_in");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == B2A_BF16)
    return epilogue == B2A_GEMM_SWIGLU
               ? gemm_out<__nv_bfloat16, 1>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st)
               : gemm_out<__nv_bfloat16, 0>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
  if (dtype == B2A_F16)
    return epilogue == B2A_GEMM_SWIGLU
               ? gemm_out<__half, 1>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st)
               : gemm_out<__half, 0>(out_dtype, a, lda, w, ldw, c_in, ldc, out, ldo, M, N, K, st);
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

}  // extern "C"
