// Causal flash prefill, paired-head persistent kernel (tcgen05 + TMEM + TMA).
//
// Same math and masking as prefill.cu's prefill_kernel (the reference's
// alpaccaroo/model.py:1254-1272 and :1567-1592); this kernel is the fast
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
// head's tile.  P never touches shared memory: the softmax writes P_t(j) as
// 16-bit pairs over the first 64 columns of S_t (after loading the whole
// score row into registers) and PV reads it from TMEM (A operand in TMEM);
// with both MMA operands and P in shared memory, its bandwidth, not the
// tensor core, bounded the kernel.  Every tcgen05.mma is issued from
// precomputed descriptors (one add per operand).
//
// The grid is persistent (at most one CTA per SM); CTA c takes items c,
// 2G-1-c, 2G+c, ... of the heaviest-first item list (snake order), and the
// producer prefetches the next item's Q and K/V while the current item drains.
//
// 384 threads:
//   warp 0        TMA producer (Q pair, then K_j / V_j into a 4-slot ring)
//   warp 1        TMEM owner, single-lane MMA issuer
//   warps 2-3     idle
//   warps 4-7     softmax warpgroup for head h0 (TMEM lanes = query rows)
//   warps 8-11    softmax warpgroup for head h0+1
// Registers: launched at 168 per thread (384 x 168 = 64512); the producer
// warpgroup drops to 120 and the two softmax warpgroups rise to 192
// (128 x 120 + 256 x 192 = 64512, the launch total).  The host
// refuses to launch if the compiled register count is not 168.
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,256+D)
// O1 [384,384+D).  SMEM (D=128): Q0, Q1 32 KB each, 4 K/V slots of 32 KB,
// 8 x 4 KB epilogue staging (one buffer per softmax warp).
//
// Ordering facts the pipeline relies on (tcgen05.commit arrives only when
// every MMA the issuing thread issued before it has completed):
//   * QK_t(j+1) is issued after PV_t(j), so when S_t(j+1) is ready, PV_t(j)
//     has read P_t(j) and its columns may be overwritten;
//   * P_t(j) is released in two halves (keys 0-63 on ph[t], 64-127 on
//     pf[t]) and PV_t(j) is issued in the same two halves, so the first
//     half's MMAs overlap the second half's exponentials; a softmax that
//     must rescale O_t (rare: its running max grew by more than 2^8) does
//     so before the first release (S_t(j) ready implies PV_t(j-1) done);
//   * only an item's last PV_t commits pv[t] (one phase per item, waited for
//     by that item's epilogue; the next phase needs a P the epilogue's
//     softmax has not released yet, so parity waits stay unambiguous).
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
using prefill::tc_mma_ts;
using prefill::tc_st16;
using prefill::tc_st32;
using prefill::tc_wait_ld;
using prefill::tc_wait_st;

constexpr int kThreads = 384;
constexpr int kSlots = 4;
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 120;
constexpr int kSoftmaxRegs = 192;
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
  static constexpr int kStage = kRing + kSlots * kTile;  // 8 softmax warps x 4 KB
  static constexpr int kTotal = kStage + 8 * 4096;
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
    const __grid_constant__ CUtensorMap tmV, const T* __restrict__ vraw,
    const int* __restrict__ pos, TO* __restrict__ out, int n_q, int t_kv, int H, int group,
    int n_q_tiles, int n_items, float sscale, int window, int kv_start) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_qf[2], bar_qe;
  __shared__ __align__(8) uint64_t bar_full[kSlots], bar_empty[kSlots];
  __shared__ __align__(8) uint64_t bar_sf[2], bar_ph[2], bar_pf[2], bar_pv[2], bar_oe[2];
  __shared__ uint32_t s_tmem;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    mbar_init(&bar_qf[0], 1);
    mbar_init(&bar_qf[1], 1);
    mbar_init(&bar_qe, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar_sf[t], 1);
      mbar_init(&bar_ph[t], 4);
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
        // Q of the first head, then (in the ring loop) the first K tile, then
        // Q of the second head: QK of the first head starts after 64 KB
        // instead of 96 KB (at a cold start every byte comes from HBM)
        mbar_arrive_expect_tx(&bar_qf[0], L::kTile);
#pragma unroll
        for (int b = 0; b < D / 64; ++b)
          tma_load_3d(smem + L::kQ0 + b * L::kBox, &tmQ, &bar_qf[0], b * 64, it.h0, it.row0);
        ++qcnt;
        // the next item's Q tiles and first K/V tiles come from HBM: start
        // them towards L2 now, an item ahead of their loads
        {
          const int nidx = item_index(k + 1, c, G);
          if (nidx < n_items) {
            const Item nt = make_item(nidx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
#pragma unroll
            for (int b = 0; b < D / 64; ++b) {
              tma_prefetch_l2_3d(&tmQ, b * 64, nt.h0, nt.row0);
              tma_prefetch_l2_3d(&tmQ, b * 64, nt.h0 + 1, nt.row0);
              for (int j = nt.j0; j < nt.jend && j < nt.j0 + 2; ++j) {
                tma_prefetch_l2_3d(&tmK, b * 64, nt.kvh, j * kBN);
                tma_prefetch_l2_3d(&tmV, b * 64, nt.kvh, j * kBN);
              }
            }
          }
        }
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
            if (j == it.j0 && kv == 0) {
              mbar_arrive_expect_tx(&bar_qf[1], L::kTile);
#pragma unroll
              for (int b = 0; b < D / 64; ++b)
                tma_load_3d(smem + L::kQ1 + b * L::kBox, &tmQ, &bar_qf[1], b * 64, it.h0 + 1,
                            it.row0);
            }
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------ MMA issuer ---------------------------
      constexpr uint32_t idesc_qk = make_idesc<T>(kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = make_idesc<T>(kBM, D, false, true);
      // Descriptors precomputed once: the start address sits in the low 14
      // bits (address >> 4), so a byte offset is an add of (off >> 4).
      const uint64_t dQ[2] = {sw128_desc(smem_u32(smem + L::kQ0), 16, 1024),
                              sw128_desc(smem_u32(smem + L::kQ1), 16, 1024)};
      const uint64_t dK0 = sw128_desc(smem_u32(smem + L::kRing), 16, 1024);
      const uint64_t dV0 = sw128_desc(smem_u32(smem + L::kRing), L::kBox, 1024);
      constexpr uint64_t kSlotStep = L::kTile >> 4;
      uint32_t seq = 0, qcnt = 0, pcnt0 = 0, pcnt1 = 0;
      bool ok = true;
      auto qk = [&](int t, uint32_t kslot) {
        const uint64_t dk = dK0 + kslot * kSlotStep;
        const uint64_t dq = dQ[t];
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = (((kk >> 2) * L::kBox) + (kk & 3) * 32) >> 4;
          tc_mma(tmem + t * kBN, dq + off, dk + off, idesc_qk, kk > 0);
        }
        tc_commit(&bar_sf[t]);
      };
      // PV_t over one half of the key tile (keys 64*half .. 64*half+63);
      // the item's last PV commits the head's PV barrier (the epilogue's
      // wait; every earlier PV_t completed before the next S_t was ready)
      auto pv = [&](int t, uint32_t vslot, bool acc, int half, bool last) {
        const uint64_t dv = dV0 + vslot * kSlotStep;
        const uint32_t tp = tmem + t * kBN;  // P_t: 16 keys per 8 columns
#pragma unroll
        for (int k4 = 0; k4 < kBN / 32; ++k4) {
          const int kk = half * (kBN / 32) + k4;
          tc_mma_ts(tmem + 2 * kBN + t * 128, tp + kk * 8, dv + ((kk * 16 * 128) >> 4), idesc_pv,
                    (acc || kk > 0));
        }
        if (half && last) tc_commit(&bar_pv[t]);
      };
      for (int k = 0; ok; ++k) {
        const int idx = item_index(k, c, G);
        if (idx >= n_items) break;
        const Item it = make_item(idx, pos, n_q, t_kv, H, group, n_q_tiles, window, kv_start);
        const int n = it.jend - it.j0;
        if (n <= 0) continue;
        if (!mbar_wait(&bar_qf[0], qcnt & 1, 0x13000 | k)) break;
        const uint32_t base = seq;
        seq += 2 * n;
        // first key tile for both heads
        {
          const uint32_t ks = base % kSlots;
          if (!mbar_wait(&bar_full[ks], (base / kSlots) & 1, 0x14000)) break;
          tc_fence_after();
          qk(0, ks);
          if (!mbar_wait(&bar_qf[1], qcnt & 1, 0x13800 | k)) break;
          tc_fence_after();
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
            // first half of P_t(jj): its PV runs while the softmax computes
            // the second half's exponentials
            if (!mbar_wait(&bar_ph[t], pc & 1, 0x15000 | jj)) { ok = false; break; }
            if (jj == 0 && qcnt > 0 && !mbar_wait(&bar_oe[t], (qcnt - 1) & 1, 0x16000)) { ok = false; break; }
            if (t == 0 && !mbar_wait(&bar_full[vs], (vsq / kSlots) & 1, 0x17000 | jj)) { ok = false; break; }
            tc_fence_after();
            pv(t, vs, jj > 0, 0, false);
            if (!mbar_wait(&bar_pf[t], pc & 1, 0x15800 | jj)) { ok = false; break; }
            ++pc;
            tc_fence_after();
            pv(t, vs, true, 1, jj + 1 == n);
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
    uint32_t scnt = 0, icnt = 0;  // icnt: items this head has finished
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
        // no key visible to any row of the tile
        prefill::store_mean_v_rows<T, TO>(valid_row, orow, vraw, t_kv, H / group, it.kvh, D);
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
        // P_t(jj) as 16-bit pairs over the first 64 columns of S_t (the whole
        // score row is in registers; PV_t(jj-1), the last reader of those
        // columns, completed before QK_t(jj) did), 32 keys per store, in two
        // halves: the MMA warp starts PV on keys 0-63 while keys 64-127 are
        // exponentiated
        float suma = 0.f, sumb = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int qtr = half * 2 + q2;
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float p0 = fast_exp2(fmaf(s[qtr * 32 + 2 * e], sscale, -mref));
              const float p1 = fast_exp2(fmaf(s[qtr * 32 + 2 * e + 1], sscale, -mref));
              if (e & 1) sumb += p0 + p1; else suma += p0 + p1;
              pk[e] = Pack2<T>::run(p0, p1);
            }
            tc_st16(tl + s_col + qtr * 16, pk);
          }
          // an O rescale comes before the first release (PV_t(jj) starts on
          // it), once the first half's scores are dead.  PV_t(jj-1)
          // completed before QK_t(jj) did (commit order), so O_t is final.
          if (half == 0 && warp_need && jj > 0) {
#pragma unroll
            for (int cc = 0; cc < D / 32; ++cc) {
              float o[32];
              tc_ld32(tl + o_col + cc * 32, o);
              tc_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= alpha;
              tc_st32(tl + o_col + cc * 32, o);
            }
          }
          tc_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(half ? &bar_pf[t] : &bar_ph[t]);
        }
        if (!ok) break;
        l = l * alpha + (suma + sumb);
      }
      if (!ok) break;
      // epilogue: wait for the last PV (every earlier one completed before
      // it), O / l -> out, release O
      {
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_pv[t], icnt & 1, 0x1B000));
      }
      if (!ok) break;
      ++icnt;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      prefill::store_o_rows<TO, D>(tl + o_col, smem + L::kStage + (warp - 4) * 4096, out,
                                   it.row0 + (warp & 3) * 32, H, h, inv, valid_row && l > 0.f);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_oe[t]);
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

}  // namespace prefill2
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

template <typename T, typename TO, int D>
int launch_prefill_pair(const void* q, const void* k, const void* v, const int* pos, void* out,
                        int n_q, int t_kv, int H, int KV, float scale, int window, int kv_start,
                        cudaStream_t st) {
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
  const CUtensorMapDataType tdt = std::is_same<T, __nv_bfloat16>::value
                                      ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H), static_cast<uint64_t>(n_q)};
  const uint64_t qstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H) * D * 2};
  const uint64_t kdims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(KV), static_cast<uint64_t>(t_kv)};
  const uint64_t kstr[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(KV) * D * 2};
  const uint32_t box[3] = {64, 1, 128};
  int rc = b2a_host::make_tmap(&tq, tdt, 3, const_cast<void*>(q), qdims, qstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tk, tdt, 3, const_cast<void*>(k), kdims, kstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b2a_host::make_tmap(&tv, tdt, 3, const_cast<void*>(v), kdims, kstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // >= 120 KB keeps one CTA per SM (a second one would wait for TMEM)
  const int smem = P2::Layout<D>::kSmem > 120 * 1024 ? P2::Layout<D>::kSmem : 120 * 1024;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(prefill_pair)");
  const int sms = b2a_host::sm_count();
  const int n_q_tiles = (n_q + b2a::prefill::kBM - 1) / b2a::prefill::kBM;
  const int n_items = n_q_tiles * (H / 2);
  const int grid = n_items < sms ? n_items : sms;
  kern<<<grid, P2::kThreads, smem, st>>>(tq, tk, tv, static_cast<const T*>(v), pos,
                                         static_cast<TO*>(out), n_q, t_kv, H,
                                         H / KV, n_q_tiles, n_items,
                                         scale * b2a::prefill::kLog2e, window, kv_start);
  e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "prefill_pair launch");
  return B2A_OK;
}

}  // namespace
