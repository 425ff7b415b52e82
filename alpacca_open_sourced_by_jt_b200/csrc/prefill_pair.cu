// Causal flash prefill, paired-head persistent kernel (tcgen05 + TMEM + TMA).
//
// Same math and masking as prefill.cu's prefill_kernel (the reference's
// alpaccaroo/model.py:1254-1272 and :1567-1592); this kernel is the faster
// schedule for even GQA groups.
//
// Work item = (128-query tile, pair of query heads h0, h0+1 of one KV group).
// Both heads read the same K/V tiles over the same causal range, so one TMA
// stream feeds two Q tiles and the tensor core alternates between them:
//
//   MMA lane:  QK0_j QK1_j | PV0_j QK0_{j+1} | PV1_j QK1_{j+1} | PV0_{j+1} ...
//   softmax A:      S0_j -> P0_j                 S0_{j+1} -> P0_{j+1}
//   softmax B:            S1_j -> P1_j                      S1_{j+1} -> ...
//
// so each warpgroup's softmax runs while the tensor core works on the other
// head's tile.  The grid is persistent (at most one CTA per SM); CTA c takes
// items c, 2G-1-c, 2G+c, ... of the heaviest-first item list (snake order),
// and the producer prefetches the next item's Q and K/V while the current
// item drains.
//
// 384 threads:
//   warp 0        TMA producer (Q pair, then K_j / V_j into a 3-slot ring)
//   warp 1        TMEM owner, single-lane MMA issuer
//   warps 2-3     idle
//   warps 4-7     softmax warpgroup for head h0 (TMEM lanes = query rows)
//   warps 8-11    softmax warpgroup for head h0+1
// Registers: launched at 168 per thread (384 x 168 = 64512); the producer
// warpgroup drops to 112 and the two softmax warpgroups rise to 184
// (128 x 112 + 256 x 184 = 61440 <= 64512, the launch total).  The host
// refuses to launch if the compiled register count is not 168.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [384,384+D).
//
// Positions must be non-decreasing within each 128-token tile (a prefill
// chunk's positions always are): the key range of a tile is taken from its
// first and last query.  A row whose visible keys fall outside that range
// records B2A_ERR_POSITION.

namespace b2a {
namespace prefill2 {

using prefill::kBM;
using prefill::kBN;
using prefill::kLog2e;
using prefill::kRescaleThreshold;
using prefill::Pack2;
using prefill::make_idesc;
using prefill::store_row32;
using prefill::sw128_desc;
using prefill::tc_commit;
using prefill::tc_fence_after;
using prefill::tc_fence_before;
using prefill::tc_ld32;
using prefill::tc_mma;
using prefill::tc_st32;
using prefill::tc_wait_ld;
using prefill::tc_wait_st;

constexpr int kThreads = 384;
constexpr int kSlots = 3;
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 112;
constexpr int kSoftmaxRegs = 184;
// setmaxnreg.inc draws only on what the block was launched with
static_assert(128 * kProducerRegs + 256 * kSoftmaxRegs <= kThreads * kLaunchRegs,
              "setmaxnreg split must fit in the launch allocation");

template <int D>
struct Layout {
  static constexpr int kBox = 128 * 128;         // 128 rows x 128 B
  static constexpr int kTile = (D / 64) * kBox;  // one Q, K or V tile
  static constexpr int kQ0 = 0;
  static constexpr int kQ1 = kTile;
  static constexpr int kRing = 2 * kTile;
  static constexpr int kP0 = kRing + kSlots * kTile;
  static constexpr int kP1 = kP0 + (kBN / 64) * kBox;
  static constexpr int kTotal = kP1 + (kBN / 64) * kBox;
  static constexpr int kSmem = kTotal + 1024;
};

struct Item {
  int h0, kvh, row0, nrows, j0, jend;
};

// The idx-th work item (heaviest q tiles first).  Every role computes the
// same items from the same inputs.
__device__ __forceinline__ Item make_item(int idx, const int* __restrict__ pos, int n_q,
                                          int t_kv, int H, int group, int n_q_tiles,
                                          int window, int kv_start) {
  Item it;
  const int pairs = H >> 1;
  const int qt = n_q_tiles - 1 - idx / pairs;
  it.h0 = 2 * (idx % pairs);
  it.kvh = it.h0 / group;
  it.row0 = qt * kBM;
  it.nrows = min(kBM, n_q - it.row0);
  const long long pf = pos[it.row0];
  const long long pl = pos[it.row0 + it.nrows - 1];
  const long long hi = min(pl - kv_start + 1, static_cast<long long>(t_kv));
  it.jend = hi <= 0 ? 0 : static_cast<int>((hi + kBN - 1) / kBN);
  it.j0 = 0;
  if (window > 0) {
    const long long lo = pf - window + 1 - kv_start;
    if (lo > 0) it.j0 = static_cast<int>(min(lo / kBN, static_cast<long long>(it.jend)));
  }
  return it;
}

// Item index of this CTA's k-th item (snake order over rounds of G CTAs).
__device__ __forceinline__ int item_index(int k, int c, int G) {
  return k * G + ((k & 1) ? (G - 1 - c) : c);
}

template <typename T, typename TO, int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_pair_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const int* __restrict__ pos, TO* __restrict__ out,
    int n_q, int t_kv, int H, int group, int n_q_tiles, int n_items, float sscale, int window,
    int kv_start) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_qf, bar_qe;
  __shared__ __align__(8) uint64_t bar_full[kSlots], bar_empty[kSlots];
  __shared__ __align__(8) uint64_t bar_sf[2], bar_pf[2], bar_pv[2], bar_oe[2];
  __shared__ uint32_t s_tmem;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    mbar_init(&bar_qf, 1);
    mbar_init(&bar_qe, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar_sf[t], 1);
      mbar_init(&bar_pf[t], 4);
      mbar_init(&bar_pv[t], 1);
      mbar_init(&bar_oe[t], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(prefill::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == 0 && lane == 0) {
      // ------------------------------ TMA producer -------------------------
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t seq = 0, qcnt = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int idx = item_index(k, c, G);
        if (idx >= n_items) break;
        const Item it = make_item(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
        if (it.jend - it.j0 <= 0) continue;
        if (qcnt > 0 && !mbar_wait(&bar_qe, (qcnt - 1) & 1, 0x11000 | k)) break;
        mbar_arrive_expect_tx(&bar_qf, 2 * L::kTile);
#pragma unroll
        for (int b = 0; b < D / 64; ++b) {
          tma_load_3d(smem + L::kQ0 + b * L::kBox, &tmQ, &bar_qf, b * 64, it.h0, it.row0);
          tma_load_3d(smem + L::kQ1 + b * L::kBox, &tmQ, &bar_qf, b * 64, it.h0 + 1, it.row0);
        }
        ++qcnt;
        for (int j = it.j0; ok && j < it.jend; ++j) {
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {
            const int slot = seq % kSlots;
            if (seq >= kSlots && !mbar_wait(&bar_empty[slot], ((seq / kSlots) & 1) ^ 1, 0x12000 | j)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar_full[slot], L::kTile);
            uint8_t* dst = smem + L::kRing + slot * L::kTile;
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_load_3d(dst + b * L::kBox, kv ? &tmV : &tmK, &bar_full[slot], b * 64, it.kvh,
                          j * kBN);
            ++seq;
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------ MMA issuer ---------------------------
      constexpr uint32_t idesc_qk = make_idesc<T>(kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = make_idesc<T>(kBM, D, false, true);
      const uint32_t sQ0 = smem_u32(smem + L::kQ0);
      const uint32_t sQ1 = smem_u32(smem + L::kQ1);
      const uint32_t sRing = smem_u32(smem + L::kRing);
      const uint32_t sP0 = smem_u32(smem + L::kP0);
      const uint32_t sP1 = smem_u32(smem + L::kP1);
      uint32_t seq = 0, qcnt = 0, pcnt0 = 0, pcnt1 = 0;
      bool ok = true;
      auto qk = [&](int t, uint32_t kslot) {
        const uint32_t kb = sRing + kslot * L::kTile;
        const uint32_t qb = t ? sQ1 : sQ0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kBox + (kk & 3) * 32;
          tc_mma(tmem + t * kBN, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                 idesc_qk, kk > 0);
        }
        tc_commit(&bar_sf[t]);
      };
      auto pv = [&](int t, uint32_t vslot, bool acc) {
        const uint32_t vb = sRing + vslot * L::kTile;
        const uint32_t pb = t ? sP1 : sP0;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * L::kBox + (kk & 3) * 32;
          tc_mma(tmem + 2 * kBN + t * 128, sw128_desc(pb + poff, 16, 1024),
                 sw128_desc(vb + kk * 16 * 128, L::kBox, 1024), idesc_pv, (acc || kk > 0));
        }
        tc_commit(&bar_pv[t]);
      };
      for (int k = 0; ok; ++k) {
        const int idx = item_index(k, c, G);
        if (idx >= n_items) break;
        const Item it = make_item(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
        const int n = it.jend - it.j0;
        if (n <= 0) continue;
        if (!mbar_wait(&bar_qf, qcnt & 1, 0x13000 | k)) break;
        const uint32_t base = seq;
        seq += 2 * n;
        // first key tile for both heads
        {
          const uint32_t ks = base % kSlots;
          if (!mbar_wait(&bar_full[ks], (base / kSlots) & 1, 0x14000)) break;
          tc_fence_after();
          qk(0, ks);
          qk(1, ks);
          tc_commit(&bar_empty[ks]);
          if (n == 1) tc_commit(&bar_qe);
        }
        for (int jj = 0; ok && jj < n; ++jj) {
          const uint32_t vsq = base + 2 * jj + 1;
          const uint32_t vs = vsq % kSlots;
          const uint32_t ksq = base + 2 * jj + 2;  // next key tile
          const uint32_t ks = ksq % kSlots;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            uint32_t& pc = t ? pcnt1 : pcnt0;
            if (!mbar_wait(&bar_pf[t], pc & 1, 0x15000 | jj)) { ok = false; break; }
            ++pc;
            if (jj == 0 && qcnt > 0 && !mbar_wait(&bar_oe[t], (qcnt - 1) & 1, 0x16000)) { ok = false; break; }
            if (t == 0 && !mbar_wait(&bar_full[vs], (vsq / kSlots) & 1, 0x17000 | jj)) { ok = false; break; }
            tc_fence_after();
            pv(t, vs, jj > 0);
            if (t == 1) tc_commit(&bar_empty[vs]);
            if (jj + 1 < n) {
              if (t == 0 && !mbar_wait(&bar_full[ks], (ksq / kSlots) & 1, 0x18000 | jj)) { ok = false; break; }
              tc_fence_after();
              qk(t, ks);
              if (t == 1) {
                tc_commit(&bar_empty[ks]);
                if (jj + 2 == n) tc_commit(&bar_qe);
              }
            }
          }
        }
        ++qcnt;
      }
    }
    __syncwarp();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------ softmax ----------------------------------
    const int t = (warp >= 8) ? 1 : 0;            // which head of the pair
    const int r = (warp & 3) * 32 + lane;         // query row within the tile == TMEM lane
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = t * kBN, o_col = 2 * kBN + t * 128;
    uint8_t* prow = smem + (t ? L::kP1 : L::kP0) + r * 128;
    uint32_t scnt = 0, pvcnt = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int idx = item_index(k, c, G);
      if (idx >= n_items) break;
      const Item it = make_item(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
      const int n = it.jend - it.j0;
      const int h = it.h0 + t;
      const int row = it.row0 + r;
      const bool valid_row = r < it.nrows;
      TO* orow = out + (static_cast<size_t>(row) * H + h) * D;
      const long long my_pos = valid_row ? static_cast<long long>(pos[row]) : LLONG_MIN;
      if (valid_row && n > 0) {
        // this row's visible keys must lie inside the tile range [j0, jend)
        const long long last = min(my_pos, static_cast<long long>(kv_start) + t_kv - 1) - kv_start;
        const long long first = window > 0 ? my_pos - window + 1 - kv_start : 0;
        if ((last >= 0 && last / kBN >= it.jend) || (first > 0 && first / kBN < it.j0))
          set_dev_error(B2A_ERR_POSITION, row);
      }
      if (n <= 0) {
        float z[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) z[e] = 0.f;
        if (valid_row)
#pragma unroll
          for (int cc = 0; cc < D / 32; ++cc) store_row32<TO>(orow + cc * 32, z, 1.f);
        continue;
      }
      float m = -INFINITY, l = 0.f;
      for (int jj = 0; jj < n; ++jj) {
        const int j = it.j0 + jj;
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_sf[t], scnt & 1, 0x19000 | jj));
        if (!ok) break;
        ++scnt;
        tc_fence_after();

        const long long kv0 = static_cast<long long>(kv_start) + static_cast<long long>(j) * kBN;
        const int hi = valid_row ? static_cast<int>(min(my_pos - kv0, static_cast<long long>(min(kBN, t_kv - j * kBN) - 1)))
                                 : -1;
        const int lo = (window > 0 && valid_row)
                           ? static_cast<int>(max(my_pos - window + 1 - kv0, -1ll))
                           : -1;
        const bool full_tile = hi >= kBN - 1 && lo <= 0;
        // the whole 128-column score row in registers: four TMEM loads, one
        // wait; the mask is a branch-free select (a short-circuit test would
        // compile to a branch per element) and four partial maxima keep the
        // FMNMX dependency chain short
        float s[kBN];
#pragma unroll
        for (int q32 = 0; q32 < kBN / 32; ++q32) tc_ld32(tl + s_col + q32 * 32, s + q32 * 32);
        tc_wait_ld();
        if (!full_tile) {
#pragma unroll
          for (int cc = 0; cc < kBN; ++cc) s[cc] = ((cc <= hi) & (cc >= lo)) ? s[cc] : -INFINITY;
        }
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < kBN; cc += 4) {
          mxa = fmaxf(mxa, s[cc]);
          mxb = fmaxf(mxb, s[cc + 1]);
          mxc = fmaxf(mxc, s[cc + 2]);
          mxd = fmaxf(mxd, s[cc + 3]);
        }
        const float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
        const float mnew = fmaxf(m, mx * sscale);
        const bool need = mnew > m + kRescaleThreshold;
        const bool warp_need = __any_sync(0xffffffffu, need);
        float alpha = 1.f;
        if (warp_need) {
          alpha = (mnew == -INFINITY) ? 1.f : fast_exp2(m - mnew);
          m = mnew;
        }
        const float mref = (m == -INFINITY) ? 0.f : m;
        // PV_t(j-1) was issued before QK_t(j), and tcgen05 MMAs complete in
        // issue order, so this wait passes at once: P_t's buffer and O_t are
        // free before any exponential is computed.
        if (jj > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv[t], pvcnt & 1, 0x1A000 | jj));
          if (!ok) break;
          ++pvcnt;
          tc_fence_after();
        }
        // exponentiate 8 scores at a time and store them straight into the
        // swizzled P tile
        float suma = 0.f, sumb = 0.f;
#pragma unroll
        for (int ch = 0; ch < kBN / 8; ++ch) {
          float p[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) p[e] = fast_exp2(fmaf(s[ch * 8 + e], sscale, -mref));
          suma += (p[0] + p[1]) + (p[2] + p[3]);
          sumb += (p[4] + p[5]) + (p[6] + p[7]);
          *reinterpret_cast<uint4*>(prow + (ch >> 3) * L::kBox + (((ch & 7) ^ (r & 7)) << 4)) =
              make_uint4(Pack2<T>::run(p[0], p[1]), Pack2<T>::run(p[2], p[3]),
                         Pack2<T>::run(p[4], p[5]), Pack2<T>::run(p[6], p[7]));
        }
        const float sum = suma + sumb;
        l = l * alpha + sum;
        if (warp_need && jj > 0) {
#pragma unroll
          for (int cc = 0; cc < D / 32; ++cc) {
            float o[32];
            tc_ld32(tl + o_col + cc * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tc_st32(tl + o_col + cc * 32, o);
          }
          tc_wait_st();
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_pf[t]);
      }
      if (!ok) break;
      // epilogue: wait for the last PV, O / l -> out, release O
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv[t], pvcnt & 1, 0x1B000));
      if (!ok) break;
      ++pvcnt;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        tc_ld32(tl + o_col + cc * 32, o);
        tc_wait_ld();
        if (valid_row) store_row32<TO>(orow + cc * 32, o, inv);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_oe[t]);
    }
  }
  // ------------------------------ teardown -----------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(prefill::kTmemCols));
  }
}

}  // namespace prefill2
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

template <typename T, typename TO, int D>
int launch_prefill_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                        const int* pos, void* out, int n_q, int t_kv, int H, int KV, float scale,
                        int window, int kv_start, cudaStream_t st) {
  namespace P2 = b2a::prefill2;
  auto kern = P2::prefill_pair_kernel<T, TO, D>;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncGetAttributes(prefill_pair)");
  if (fa.numRegs != P2::kLaunchRegs)
    return b2a_host::fail(B2A_ERR_CUDA,
                          "prefill_pair: compiled with %d registers/thread, the setmaxnreg split "
                          "needs exactly %d",
                          fa.numRegs, P2::kLaunchRegs);
  const int smem = P2::Layout<D>::kSmem;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(prefill_pair)");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int n_q_tiles = (n_q + b2a::prefill::kBM - 1) / b2a::prefill::kBM;
  const int n_items = n_q_tiles * (H / 2);
  const int grid = n_items < sms ? n_items : sms;
  kern<<<grid, P2::kThreads, smem, st>>>(tq, tk, tv, pos, static_cast<TO*>(out), n_q, t_kv, H,
                                         H / KV, n_q_tiles, n_items,
                                         scale * b2a::prefill::kLog2e, window, kv_start);
  e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "prefill_pair launch");
  return B2A_OK;
}

}  // namespace
