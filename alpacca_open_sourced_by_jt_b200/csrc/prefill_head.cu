// Causal flash prefill, one head per work item, persistent (tcgen05 + TMEM + TMA).
//
// Same math and masking as prefill.cu's prefill_kernel (the reference's
// alpaccaroo/model.py:1254-1272 and :1567-1592), any GQA group.
//
// Work item = (128-query tile, query head).  Per item the tensor core runs
//   S(j) = Q . K_j^T   into TMEM S buffer j % 2   (M = N = 128, 8 MMAs, SS)
//   O   += P(j) . V_j  with P(j) in TMEM          (M = 128, N = D, 8 MMAs, TS)
// in the order QK(0) QK(1) PV(0) QK(2) PV(1) QK(3) ...  The softmax writes
// P(j) as 16-bit pairs over the first 64 columns of S buffer j % 2 (after it
// has loaded the whole score row into registers), so P never touches shared
// memory: shared-memory bandwidth, not the tensor core, was the limit when
// both MMA operands and the P tile went through it.  With S/P
// double-buffered the softmax warpgroup finds S(j+1) ready when it finishes
// P(j) and never waits on the tensor core, except for the rare O rescale
// (running max grew by more than 2^8) and the item's epilogue.  The MMA lane
// issues each tcgen05.mma from precomputed descriptors (one add per
// operand).
//
// The grid is persistent (at most one CTA per SM): CTA c takes items c,
// 2G-1-c, 2G+c, ... of the heaviest-first item list (snake order); the
// producer loads the next item's Q as soon as the current item's last QK
// has completed, and keeps streaming K/V tiles through a ring of K/V slots.
//
// 256 threads: warp 0 TMA producer, warp 1 TMEM owner + single-lane MMA
// issuer, warps 2-3 idle, warps 4-7 softmax (thread = query row = TMEM lane).
// Key tiles hold BN keys: 128 for head_dim 64 and 128, 64 for head_dim 256,
// where a 128-key K or V tile (64 KB) would leave room for only one ring slot.
// TMEM (512 columns): S0/P0 [0,BN), S1/P1 [BN,2BN), O [2BN, 2BN+D) (for
// D = 256: 64 + 64 + 256 columns).  SMEM: Q (128 x D), then a ring of K/V
// slots of BN x D: 5 slots of 32 KB for D = 128, 4 of 32 KB for D = 256,
// then 4 x 4 KB epilogue staging (one buffer per softmax warp).
//
// Barrier phases use running counters; where one side may run two steps
// ahead, two barriers alternate (index g & 1, phase g >> 1) so that every
// parity wait is unambiguous:
//   * P release g (pf[g & 1]): the softmax cannot release P(g+2) before the
//     MMA lane consumed P(g), because S(g+2) is only issued after PV(g);
//   * PV g (pv[g & 1]): PV(g+2) needs P(g+2), which the waiting softmax has
//     not released yet.
//
// Positions must be non-decreasing within each 128-token tile (a prefill
// chunk's positions always are): the key range of a tile is taken from its
// first and last query.  A row whose visible keys fall outside that range
// records B2A_ERR_POSITION.

namespace b2a {
namespace prefill_head {

using prefill::kBM;
using prefill::kBN;
using prefill::kLog2e;
using prefill::kRescaleThreshold;
using prefill::Pack2;
using prefill::make_idesc;
using prefill::sw128_desc;
using prefill::tc_commit;
using prefill::tc_fence_after;
using prefill::tc_fence_before;
using prefill::tc_ld32;
using prefill::tc_mma;
using prefill::tc_mma_ts;
using prefill::tc_st16;
using prefill::tc_st32;
using prefill::tc_wait_ld;
using prefill::tc_wait_st;

constexpr int kThreads = 256;

// Keys per K/V tile for a head_dim.
template <int D>
struct KeyTile {
  static constexpr int kBN = D > 128 ? 64 : 128;
};

template <int D, int BN>
struct Layout {
  static constexpr int kSlots = D > 128 ? 4 : 5;
  static constexpr int kBoxQ = 128 * 128;            // 128 query rows x 128 B
  static constexpr int kBoxKV = BN * 128;            // BN key rows x 128 B
  static constexpr int kTileQ = (D / 64) * kBoxQ;    // Q tile (128 rows x D)
  static constexpr int kTileKV = (D / 64) * kBoxKV;  // K or V tile (BN rows x D)
  static constexpr int kQ = 0;
  static constexpr int kRing = kTileQ;
  static constexpr int kStage = kRing + kSlots * kTileKV;  // 4 softmax warps x 4 KB
  static constexpr int kTotal = kStage + 4 * 4096;
  static constexpr int kSmem = kTotal + 1024;
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert(2 * BN + D <= 512, "S double buffer + O must fit in 512 TMEM columns");
};

struct Item {
  int h, kvh, row0, nrows, j0, jend;
};

// The idx-th work item (heaviest q tiles first); every role computes the
// same items from the same inputs.
template <int BN>
__device__ __forceinline__ Item make_item(int idx, const int* __restrict__ pos, int n_q,
                                          int t_kv, int H, int group, int n_q_tiles,
                                          int window, int kv_start) {
  Item it;
  const int qt = n_q_tiles - 1 - idx / H;
  it.h = idx % H;
  it.kvh = it.h / group;
  it.row0 = qt * kBM;
  it.nrows = min(kBM, n_q - it.row0);
  const long long pf = pos[it.row0];
  const long long pl = pos[it.row0 + it.nrows - 1];
  const long long hi = min(pl - kv_start + 1, static_cast<long long>(t_kv));
  it.jend = hi <= 0 ? 0 : static_cast<int>((hi + BN - 1) / BN);
  it.j0 = 0;
  if (window > 0) {
    const long long lo = pf - window + 1 - kv_start;
    if (lo > 0) it.j0 = static_cast<int>(min(lo / BN, static_cast<long long>(it.jend)));
  }
  return it;
}

__device__ __forceinline__ int item_index(int k, int c, int G) {
  return k * G + ((k & 1) ? (G - 1 - c) : c);
}

template <typename T, typename TO, int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_head_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const T* __restrict__ vraw,
    const int* __restrict__ pos, TO* __restrict__ out, int n_q, int t_kv, int H, int group,
    int n_q_tiles, int n_items, float sscale, int window, int kv_start) {
  constexpr int BN = KeyTile<D>::kBN;
  using L = Layout<D, BN>;
  constexpr int kSlots = L::kSlots;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_qf, bar_qe;
  __shared__ __align__(8) uint64_t bar_full[kSlots], bar_empty[kSlots];
  __shared__ __align__(8) uint64_t bar_sf[2], bar_pf[2], bar_pv[2], bar_oe;
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
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_sf[b], 1);
      mbar_init(&bar_pf[b], 4);
      mbar_init(&bar_pv[b], 1);
    }
    mbar_init(&bar_oe, 4);
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

  if (warp == 0) {
    // ------------------------------ TMA producer ---------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t seq = 0, qcnt = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int idx = item_index(k, c, G);
        if (idx >= n_items) break;
        const Item it = make_item<BN>(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
        if (it.jend - it.j0 <= 0) continue;
        if (qcnt > 0 && !mbar_wait(&bar_qe, (qcnt - 1) & 1, 0x21000 | k)) break;
        mbar_arrive_expect_tx(&bar_qf, L::kTileQ);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(smem + L::kQ + b * L::kBoxQ, &tmQ, &bar_qf, b * 64, it.h, it.row0);
        ++qcnt;
        for (int j = it.j0; ok && j < it.jend; ++j) {
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {
            const int slot = seq % kSlots;
            if (seq >= kSlots &&
                !mbar_wait(&bar_empty[slot], ((seq / kSlots) & 1) ^ 1, 0x22000 | j)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar_full[slot], L::kTileKV);
            uint8_t* dst = smem + L::kRing + slot * L::kTileKV;
#pragma unroll
            for (int b = 0; b < D / 64; ++b)
              tma_load_3d(dst + b * L::kBoxKV, kv ? &tmV : &tmK, &bar_full[slot], b * 64, it.kvh,
                          j * BN);
            ++seq;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc<T>(kBM, BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc<T>(kBM, D, false, true);
      // Descriptors precomputed once: the start address sits in the low 14
      // bits (address >> 4), so a byte offset becomes an add of (off >> 4).
      const uint64_t dQ = sw128_desc(smem_u32(smem + L::kQ), 16, 1024);
      const uint64_t dK0 = sw128_desc(smem_u32(smem + L::kRing), 16, 1024);
      const uint64_t dV0 = sw128_desc(smem_u32(smem + L::kRing), L::kBoxKV, 1024);
      constexpr uint64_t kSlotStep = L::kTileKV >> 4;
      uint32_t seq = 0, qcnt = 0, pcnt = 0, pvg = 0;
      bool ok = true;
      auto qk = [&](int jj, uint32_t kslot) {
        const uint64_t dk = dK0 + kslot * kSlotStep;
        const uint32_t d_tm = tmem + (jj & 1) * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t qoff = (((kk >> 2) * L::kBoxQ) + (kk & 3) * 32) >> 4;
          const uint64_t koff = (((kk >> 2) * L::kBoxKV) + (kk & 3) * 32) >> 4;
          tc_mma(d_tm, dQ + qoff, dk + koff, idesc_qk, kk > 0);
        }
        tc_commit(&bar_sf[jj & 1]);
      };
      auto pv = [&](int jj, uint32_t vslot) {
        const uint64_t dv = dV0 + vslot * kSlotStep;
        const uint32_t tp = tmem + (jj & 1) * BN;  // P(jj): 16 keys per 8 columns
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t voff = (kk * 16 * 128) >> 4;
          tc_mma_ts(tmem + 2 * BN, tp + kk * 8, dv + voff, idesc_pv, (jj > 0 || kk > 0));
        }
        tc_commit(&bar_pv[pvg & 1]);
        ++pvg;
      };
      for (int k = 0; ok; ++k) {
        const int idx = item_index(k, c, G);
        if (idx >= n_items) break;
        const Item it = make_item<BN>(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
        const int n = it.jend - it.j0;
        if (n <= 0) continue;
        if (!mbar_wait(&bar_qf, qcnt & 1, 0x23000 | k)) break;
        const uint32_t base = seq;  // K_j at base + 2j, V_j at base + 2j + 1
        seq += 2 * n;
        for (int jj = 0; ok && jj < 2 && jj < n; ++jj) {
          const uint32_t ksq = base + 2 * jj;
          if (!mbar_wait(&bar_full[ksq % kSlots], (ksq / kSlots) & 1, 0x24000 | jj)) { ok = false; break; }
          tc_fence_after();
          qk(jj, ksq % kSlots);
          tc_commit(&bar_empty[ksq % kSlots]);
        }
        if (ok && n <= 2) tc_commit(&bar_qe);
        for (int jj = 0; ok && jj < n; ++jj) {
          const uint32_t vsq = base + 2 * jj + 1;
          if (!mbar_wait(&bar_pf[pcnt & 1], (pcnt >> 1) & 1, 0x25000 | jj)) { ok = false; break; }
          ++pcnt;
          if (jj == 0 && qcnt > 0 && !mbar_wait(&bar_oe, (qcnt - 1) & 1, 0x26000)) { ok = false; break; }
          if (!mbar_wait(&bar_full[vsq % kSlots], (vsq / kSlots) & 1, 0x27000 | jj)) { ok = false; break; }
          tc_fence_after();
          pv(jj, vsq % kSlots);
          tc_commit(&bar_empty[vsq % kSlots]);
          if (jj + 2 < n) {
            const uint32_t ksq = base + 2 * (jj + 2);
            if (!mbar_wait(&bar_full[ksq % kSlots], (ksq / kSlots) & 1, 0x28000 | jj)) { ok = false; break; }
            tc_fence_after();
            qk(jj + 2, ksq % kSlots);
            tc_commit(&bar_empty[ksq % kSlots]);
            if (jj + 3 == n) tc_commit(&bar_qe);
          }
        }
        ++qcnt;
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------ softmax ----------------------------------
    const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t o_col = 2 * BN;
    uint32_t scnt0 = 0, scnt1 = 0, pfg = 0, pvbase = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int idx = item_index(k, c, G);
      if (idx >= n_items) break;
      const Item it = make_item<BN>(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
      const int n = it.jend - it.j0;
      const int row = it.row0 + r;
      const bool valid_row = r < it.nrows;
      TO* orow = out + (static_cast<size_t>(row) * H + it.h) * D;
      const long long my_pos = valid_row ? static_cast<long long>(pos[row]) : LLONG_MIN;
      if (valid_row && n > 0) {
        const long long last = min(my_pos, static_cast<long long>(kv_start) + t_kv - 1) - kv_start;
        const long long first = window > 0 ? my_pos - window + 1 - kv_start : 0;
        if ((last >= 0 && last / BN >= it.jend) || (first > 0 && first / BN < it.j0))
          set_dev_error(B2A_ERR_POSITION, row);
      }
      if (n <= 0) {
        // no key visible to any row of the tile
        prefill::store_mean_v_rows<T, TO>(valid_row, orow, vraw, t_kv, H / group, it.kvh, D);
        continue;
      }
      float m = -INFINITY, l = 0.f;
      for (int jj = 0; jj < n; ++jj) {
        const int j = it.j0 + jj;
        const int sb = jj & 1;
        uint32_t& sc = sb ? scnt1 : scnt0;
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_sf[sb], sc & 1, 0x29000 | jj));
        if (!ok) break;
        ++sc;
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int q32 = 0; q32 < BN / 32; ++q32)
          tc_ld32(tl + sb * BN + q32 * 32, s + q32 * 32);
        tc_wait_ld();

        const long long kv0 = static_cast<long long>(kv_start) + static_cast<long long>(j) * BN;
        const int hi = valid_row ? static_cast<int>(min(my_pos - kv0, static_cast<long long>(min(BN, t_kv - j * BN) - 1)))
                                 : -1;
        const int lo = (window > 0 && valid_row)
                           ? static_cast<int>(max(my_pos - window + 1 - kv0, -1ll))
                           : -1;
        // branch-free mask select (a short-circuit test compiles to a branch
        // per element); four partial maxima keep the FMNMX chain short
        if (!(hi >= BN - 1 && lo <= 0)) {
#pragma unroll
          for (int cc = 0; cc < BN; ++cc) s[cc] = ((cc <= hi) & (cc >= lo)) ? s[cc] : -INFINITY;
        }
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < BN; cc += 4) {
          mxa = fmaxf(mxa, s[cc]);
          mxb = fmaxf(mxb, s[cc + 1]);
          mxc = fmaxf(mxc, s[cc + 2]);
          mxd = fmaxf(mxd, s[cc + 3]);
        }
        const float mnew = fmaxf(m, fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd)) * sscale);
        const bool warp_need = __any_sync(0xffffffffu, mnew > m + kRescaleThreshold);
        float alpha = 1.f;
        if (warp_need) {
          alpha = (mnew == -INFINITY) ? 1.f : fast_exp2(m - mnew);
          m = mnew;
        }
        const float mref = (m == -INFINITY) ? 0.f : m;
        // P(jj) as 16-bit pairs over the first BN/2 columns of S buffer jj % 2
        // (the whole score row is already in registers); 32 keys per store
        float suma = 0.f, sumb = 0.f;
#pragma unroll
        for (int qtr = 0; qtr < BN / 32; ++qtr) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = fast_exp2(fmaf(s[qtr * 32 + 2 * e], sscale, -mref));
            const float p1 = fast_exp2(fmaf(s[qtr * 32 + 2 * e + 1], sscale, -mref));
            if (e & 1) sumb += p0 + p1; else suma += p0 + p1;
            pk[e] = Pack2<T>::run(p0, p1);
          }
          tc_st16(tl + sb * BN + qtr * 16, pk);
        }
        tc_wait_st();
        l = l * alpha + (suma + sumb);
        // Only an O rescale needs PV(jj-1) complete; PV(jj) is issued after
        // this release, so it cannot race the rescale.
        if (jj > 0 && warp_need) {
          const uint32_t g = pvbase + jj - 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv[g & 1], (g >> 1) & 1, 0x2A000 | jj));
          if (!ok) break;
          tc_fence_after();
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
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_pf[pfg & 1]);
        ++pfg;
      }
      if (!ok) break;
      // epilogue: the last PV (every earlier one completed before it)
      {
        const uint32_t g = pvbase + n - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv[g & 1], (g >> 1) & 1, 0x2B000));
      }
      if (!ok) break;
      pvbase += n;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      prefill::store_o_rows<TO, D>(tl + o_col, smem + L::kStage + (warp - 4) * 4096, out,
                                   it.row0 + (warp & 3) * 32, H, it.h, inv, valid_row && l > 0.f);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_oe);
      prefill::store_mean_v_rows<T, TO>(valid_row && !(l > 0.f), orow, vraw, t_kv, H / group,
                                        it.kvh, D);
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

}  // namespace prefill_head
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

template <typename T, typename TO, int D>
int launch_prefill_head(const void* q, const void* k, const void* v, const int* pos, void* out,
                        int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
                        cudaStream_t st) {
  namespace PH = b2a::prefill_head;
  constexpr int BN = PH::KeyTile<D>::kBN;
  using L = PH::Layout<D, BN>;
  auto kern = PH::prefill_head_kernel<T, TO, D>;
  const CUtensorMapDataType tdt = std::is_same<T, __nv_bfloat16>::value
                                      ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H), static_cast<uint64_t>(n_q)};
  const uint64_t qstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H) * D * 2};
  const uint64_t kdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(KV), static_cast<uint64_t>(t_kv)};
  const uint64_t kstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(KV) * D * 2};
  const uint32_t qbox[3] = {64, 1, 128};
  const uint32_t kvbox[3] = {64, 1, static_cast<uint32_t>(BN)};
  int rc = b2a_host::make_tmap(&tq, tdt, 3, const_cast<void*>(q), qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tk, tdt, 3, const_cast<void*>(k), kdims, kstr, kvbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tv, tdt, 3, const_cast<void*>(v), kdims, kstr, kvbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // >= 120 KB keeps one CTA per SM: a second resident CTA would wait in its
  // 512-column TMEM allocation while another SM idles.
  const int smem = L::kSmem > 120 * 1024 ? L::kSmem : 120 * 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(prefill_head)");
  const int sms = b2a_host::sm_count();
  const int n_q_tiles = (n_q + b2a::prefill::kBM - 1) / b2a::prefill::kBM;
  const int n_items = n_q_tiles * H;
  const int grid = n_items < sms ? n_items : sms;
  kern<<<grid, PH::kThreads, smem, st>>>(tq, tk, tv, static_cast<const T*>(v), pos,
                                         static_cast<TO*>(out), n_q, t_kv, H, H / KV, n_q_tiles,
                                         n_items, scale * b2a::prefill::kLog2e, window, kv_start);
  e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "prefill_head launch");
  return B2A_OK;
}

}  // namespace
