// Split-KV grouped-query decode attention for B200.
//
// Algorithm (same math as alpaccaroo/model.py:1231-1252 `_attention_np` and
// the device pair alpaccaroo/cuda.py:580-694): for one query token per
// sequence, out[h] = softmax(q[h] . K[:len, h/group]^T * scale) . V[:len, h/group].
//
// B200 design:
//   * one CTA per (KV split, KV head, sequence).  All `group` query heads of
//     the KV head are served by that CTA, so every K/V byte leaves HBM once
//     (the reference kernel re-reads K/V once per query head).
//   * a producer warp streams 64-row K and V tiles with TMA (128-byte
//     swizzle) into a 3-4 stage shared-memory ring guarded by mbarriers.
//   * four consumer warps each own a 16-row slice of every tile and run
//     S^T = K.Q^T and O^T += V^T.P^T as m16n8k16 tensor-core MMAs (query
//     heads on the N=8 axis), with the online softmax on the accumulator
//     fragments (warp-shuffle max/sum) and movmatrix to turn P into the
//     B operand.  fp32 accumulation throughout.
//   * each CTA writes an unnormalised partial (m, l, acc) in log2 units;
//     a small kernel merges the partials of a sequence (log-sum-exp).
//   * lengths come from device memory and the grid is sized by a host upper
//     bound, so a captured CUDA graph replays for any lengths <= max_len.
//
// fp32 caches take an FMA kernel with the same partial format (the tensor
// core path would round K/V to 16 bits, which the fp32 parity bar forbids).

#include <math.h>

#include "b2a_common.cuh"
#include "shard_words.cuh"

namespace b2a {
namespace decode {

constexpr int kRows = 64;          // KV rows per pipeline stage
constexpr int kConsumerWarps = 4;  // each owns one 16-row slice of a stage
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int kBoxes = D / 64;            // 128-byte TMA boxes per row
  static constexpr int kBoxBytes = kRows * 128;    // one box = 64 rows x 128 B
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K tile + V tile
  static constexpr int kStages = D == 64 ? 4 : 3;
  static constexpr int kRingBytes = kStages * kStageBytes;
};

template <int D, int NT>
constexpr int merge_bytes() {
  return kConsumerWarps * (NT * 8) * (D + 2) * 4;
}

template <int D, int NT>
constexpr int smem_bytes() {
  return 1024 + (Cfg<D>::kRingBytes > merge_bytes<D, NT>() ? Cfg<D>::kRingBytes
                                                            : merge_bytes<D, NT>());
}

// ---------------------------------------------------------------------------
// Sharded decode: the last split CTA of a (sequence, KV head) merges the
// group's splits and publishes the rows to every rank (shard.cu)
// ---------------------------------------------------------------------------
// Called by the 128 consumer threads after the CTA wrote its partials.  The
// CTAs of one (sequence, KV head) take tickets; the one that draws the last
// ticket has every partial of the group visible (each CTA fences its
// partial stores before its ticket), merges the splits of each head and
// stores the (value, tag) words of the rows into slot [me] of every rank's
// exchange buffer.  Ranks whose share of a sequence is empty publish from
// the collect kernel instead (no split CTA runs for them).
template <int D>
__device__ __noinline__ void publish_group(const shard::Publish pub, const float* part_o,
                                           const float* part_ml, int b, int kvh, int H,
                                           int group, int len, int split_rows, int n_splits) {
  __shared__ int s_last;
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  const int R = static_cast<int>(gridDim.z) * H;
  const shard::XLayout xl = shard::xlayout(R, D, pub.G);
  unsigned char* mine = pub.peers[pub.me];
  uint32_t* counts = reinterpret_cast<uint32_t*>(mine + xl.counts);
  const uint32_t* steps = reinterpret_cast<const uint32_t*>(mine + xl.steps);
  const int ns_b = min(n_splits, (len + split_rows - 1) / split_rows);
  const int slot = b * static_cast<int>(gridDim.y) + kvh;
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd(&counts[slot], 1u);
    s_last = (t == static_cast<unsigned>(ns_b - 1)) ? 1 : 0;
    if (s_last) counts[slot] = 0u;  // every CTA of the group has drawn its ticket
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  if (!s_last) return;
  __threadfence();
  constexpr int kT = kConsumerWarps * 32;
  const int r0 = b * H + kvh * group;
  // The merge runs at the tail of the kernel on one CTA per group, so it is
  // latency-bound: every split's (m, l) of the group is loaded at once into
  // shared memory, each head's weights w = 2^(m - M) / L are formed once,
  // and each value then needs one batch of independent loads.
  constexpr int kMaxW = 1024;  // group x splits weights held in shared memory
  __shared__ float s_w[kMaxW];
  __shared__ float s_lse[32];
  __shared__ uint32_t s_steps[32];
  const bool fits = group * ns_b <= kMaxW && group <= 32;
  if (fits) {
    for (int i = threadIdx.x; i < group * ns_b; i += kT) {
      const int n = i / ns_b, sp = i - n * ns_b;
      s_w[i] = __ldcg(part_ml + (static_cast<size_t>(r0 + n) * n_splits + sp) * 2);
    }
    if (threadIdx.x < group) s_steps[threadIdx.x] = __ldcg(steps + r0 + threadIdx.x);
    asm volatile("bar.sync 1, %0;" ::"n"(kT));
    for (int n = threadIdx.x; n < group; n += kT) {
      const size_t p0 = static_cast<size_t>(r0 + n) * n_splits;
      float M = -INFINITY;
      for (int sp = 0; sp < ns_b; ++sp) M = fmaxf(M, s_w[n * ns_b + sp]);
      const float Mref = (M == -INFINITY) ? 0.f : M;
      float L = 0.f;
      for (int sp = 0; sp < ns_b; ++sp) {
        const float w = exp2f(s_w[n * ns_b + sp] - Mref);
        L += __ldcg(part_ml + (p0 + sp) * 2 + 1) * w;
        s_w[n * ns_b + sp] = w;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      for (int sp = 0; sp < ns_b; ++sp) s_w[n * ns_b + sp] *= inv;
      s_lse[n] = L > 0.f ? (Mref + log2f(L)) * 0.6931471805599453f : -INFINITY;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kT));
    for (int idx = threadIdx.x; idx < group * (D + 1); idx += kT) {
      const int n = idx / (D + 1), d = idx - n * (D + 1);
      float val;
      if (d < D) {
        const float* po = part_o + static_cast<size_t>(r0 + n) * n_splits * D + d;
        const float* w = s_w + n * ns_b;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int sp = 0;
        for (; sp + 3 < ns_b; sp += 4) {
          a0 += __ldcg(po + static_cast<size_t>(sp) * D) * w[sp];
          a1 += __ldcg(po + static_cast<size_t>(sp + 1) * D) * w[sp + 1];
          a2 += __ldcg(po + static_cast<size_t>(sp + 2) * D) * w[sp + 2];
          a3 += __ldcg(po + static_cast<size_t>(sp + 3) * D) * w[sp + 3];
        }
        for (; sp < ns_b; ++sp) a0 += __ldcg(po + static_cast<size_t>(sp) * D) * w[sp];
        val = (a0 + a1) + (a2 + a3);
      } else {
        val = s_lse[n];
      }
      const int r = r0 + n;
      const uint32_t step = s_steps[n];
      for (int g = 0; g < pub.G; ++g) {
        uint2* dst = reinterpret_cast<uint2*>(pub.peers[g] + xl.words) +
                     shard::word_index(static_cast<int>(step & 1u), pub.me, r, R, pub.G, D);
        shard::st_tagged(dst + d, val, step + 1u);
      }
    }
    return;
  }
  for (int idx = threadIdx.x; idx < group * (D + 1); idx += kT) {
    const int n = idx / (D + 1), d = idx - n * (D + 1);
    const size_t p0 = static_cast<size_t>(r0 + n) * n_splits;
    float M = -INFINITY;
    for (int sp = 0; sp < ns_b; ++sp) M = fmaxf(M, __ldcg(part_ml + (p0 + sp) * 2));
    const float Mref = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, acc = 0.f;
    for (int sp = 0; sp < ns_b; ++sp) {
      const float w = exp2f(__ldcg(part_ml + (p0 + sp) * 2) - Mref);
      L += __ldcg(part_ml + (p0 + sp) * 2 + 1) * w;
      if (d < D) acc += __ldcg(part_o + (p0 + sp) * D + d) * w;
    }
    const float val = d < D ? (L > 0.f ? acc / L : 0.f)
                            : (L > 0.f ? (Mref + log2f(L)) * 0.6931471805599453f : -INFINITY);
    const int r = r0 + n;
    const uint32_t step = __ldcg(steps + r);
    for (int g = 0; g < pub.G; ++g) {
      uint2* dst = reinterpret_cast<uint2*>(pub.peers[g] + xl.words) +
                   shard::word_index(static_cast<int>(step & 1u), pub.me, r, R, pub.G, D);
      shard::st_tagged(dst + d, val, step + 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core kernel (f16 / bf16 caches)
// ---------------------------------------------------------------------------
template <typename T, int D, int NT>
__global__ void __launch_bounds__(kThreads) decode_mma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const float* __restrict__ q, const int* __restrict__ lens, float* __restrict__ part_o,
    float* __restrict__ part_ml, int H, int group, int split_rows, int n_splits, float qscale,
    const shard::Publish pub) {
  // The kernels after this one (a PDL chain) are released only once every
  // CTA has streamed its rows (end of the main loop, below): released at
  // entry, they would start their own weight prefetches and take HBM
  // bandwidth from this kernel, which is the step's critical path.
  using C = Cfg<D>;
  constexpr int KS = D / 16;  // k-steps of QK^T, m-tiles of PV
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::kStages];
  __shared__ __align__(8) uint64_t empty_bar[C::kStages];

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int len = lens[b];
  const int row0 = split * split_rows;
  if (row0 >= len) return;  // uniform for the CTA, before any barrier use
  const int row1 = min(len, row0 + split_rows);
  const int n_tiles = (row1 - row0 + kRows - 1) / kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp: TMA K/V tiles into the ring ----------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // Rows below len - 1 were appended by earlier steps: under a
      // programmatic launch they stream before the wait for the kernel
      // before (the step's RoPE + append, which writes row len - 1).
      bool waited = false;
      for (int it = 0; it < n_tiles; ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (it >= C::kStages && !mbar_wait(&empty_bar[s], ph ^ 1, 0x100 | s)) break;
        const int r = row0 + it * kRows;
        if (!waited && r + kRows >= len) {
          pdl_wait();
          waited = true;
        }
        mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
        uint8_t* kt = smem + s * C::kStageBytes;
        uint8_t* vt = kt + C::kTileBytes;
#pragma unroll
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_4d(kt + bx * C::kBoxBytes, &tmK, &full_bar[s], bx * 64, kvh, r, b);
          tma_load_4d(vt + bx * C::kBoxBytes, &tmV, &full_bar[s], bx * 64, kvh, r, b);
        }
      }
    }
    return;
  }

  // ---------------- consumer warps --------------------------------------
  pdl_wait();  // q comes from the kernel before (a no-op unless PDL-launched)
  const int g = lane >> 2, t = lane & 3;
  // Query fragments (B operand of S^T = K.Q^T), pre-scaled by scale*log2(e)
  // so the softmax runs on exp2.  Heads >= group are zero padding.
  uint32_t qf[NT][KS][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nt * 8 + g;
    const bool valid = n < group;
    const float* qr = q + (static_cast<size_t>(b) * H + kvh * group + (valid ? n : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 16 + 2 * t;
      float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
      if (valid) {
        const float2 lo = *reinterpret_cast<const float2*>(qr + d0);
        const float2 hi = *reinterpret_cast<const float2*>(qr + d0 + 8);
        x0 = lo.x * qscale;
        x1 = lo.y * qscale;
        x2 = hi.x * qscale;
        x3 = hi.y * qscale;
      }
      qf[nt][ks][0] = MmaOp<T>::pack(x0, x1);
      qf[nt][ks][1] = MmaOp<T>::pack(x2, x3);
    }
  }

  float o[KS][NT][4];
#pragma unroll
  for (int mt = 0; mt < KS; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][nt][i] = 0.f;
  float m[NT][2], l[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
  }

  const uint32_t ring = smem_u32(smem);
  // ldmatrix row/chunk assignment for this lane
  const int a_row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // K (non-trans)
  const int a_khalf = lane >> 4;
  const int v_row = warp * 16 + (lane & 7) + ((lane >> 4) << 3);       // V (trans)
  const int v_dhalf = (lane >> 3) & 1;

  for (int it = 0; it < n_tiles; ++it) {
    const int s = it % C::kStages;
    const uint32_t ph = (it / C::kStages) & 1;
    if (!mbar_wait(&full_bar[s], ph, 0x200 | s)) break;
    const uint32_t kt = ring + s * C::kStageBytes;
    const uint32_t vt = kt + C::kTileBytes;

    // Rows of this warp's slice past the sequence end hold whatever the cache
    // holds there (stale rows, or never-written memory).  Their softmax
    // weight is 0, but 0 * NaN would still poison O, so zero those V rows.
    const int slice0 = row0 + it * kRows + warp * 16;
    const bool partial = slice0 + 16 > row1;
    if (partial) {
      const int first_bad = max(row1 - slice0, 0);
      uint8_t* vslice = smem + s * C::kStageBytes + C::kTileBytes;
      for (int idx = lane; idx < (16 - first_bad) * C::kBoxes * 8; idx += 32) {
        const int rr = first_bad + idx / (C::kBoxes * 8);
        const int rem = idx % (C::kBoxes * 8);
        const int row = warp * 16 + rr;
        *reinterpret_cast<uint4*>(vslice + (rem >> 3) * C::kBoxBytes + sw128_off(row, rem & 7)) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // S^T[16 rows][8*NT heads] = K[rows] . Q^T
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a[4];
      const int box = ks >> 2;
      const int chunk = ((ks & 3) << 1) + a_khalf;
      ldsm_x4(kt + box * C::kBoxBytes + sw128_off(a_row, chunk), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(sc[nt], a, qf[nt][ks]);
    }

    // rows past the sequence end (tile tail, stale or zero-filled) are masked
    const int rbase = row0 + it * kRows + warp * 16 + g;
    const bool v0 = rbase < row1, v1 = rbase + 8 < row1;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (!v0) sc[nt][0] = sc[nt][1] = -INFINITY;
      if (!v1) sc[nt][2] = sc[nt][3] = -INFINITY;
    }

    // online softmax, per head column (lane owns heads 2t, 2t+1 of each n-tile)
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float p[4];
      float alpha[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mx = fmaxf(sc[nt][j], sc[nt][j + 2]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mnew = fmaxf(m[nt][j], mx);
        const float mref = (mnew == -INFINITY) ? 0.f : mnew;
        alpha[j] = fast_exp2(m[nt][j] - mref);
        m[nt][j] = mnew;
        p[j] = fast_exp2(sc[nt][j] - mref);
        p[j + 2] = fast_exp2(sc[nt][j + 2] - mref);
        l[nt][j] = l[nt][j] * alpha[j] + (p[j] + p[j + 2]);
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        o[mt][nt][0] *= alpha[0];
        o[mt][nt][1] *= alpha[1];
        o[mt][nt][2] *= alpha[0];
        o[mt][nt][3] *= alpha[1];
      }
      pb[nt][0] = movmatrix_trans(MmaOp<T>::pack(p[0], p[1]));
      pb[nt][1] = movmatrix_trans(MmaOp<T>::pack(p[2], p[3]));
    }

    // O^T[D][8*NT heads] += V^T[D][rows] . P^T[rows][heads]
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      uint32_t a[4];
      const int dchunk = 2 * mt + v_dhalf;
      ldsm_x4_trans(vt + (dchunk >> 3) * C::kBoxBytes + sw128_off(v_row, dchunk & 7), a[0], a[1],
                    a[2], a[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(o[mt][nt], a, pb[nt]);
    }
    // generic-proxy zero stores must be ordered before the next TMA write
    if (partial) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---------------- merge the four warps' partial softmax states ----------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float x = l[nt][j];
      x += __shfl_xor_sync(0xffffffffu, x, 4);
      x += __shfl_xor_sync(0xffffffffu, x, 8);
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      l[nt][j] = x;
    }
  // every stage has been consumed by every warp (or the CTA aborted), so the
  // ring can be reused for the merge buffers once all consumers are here
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  constexpr int NH = NT * 8;
  float* red_o = reinterpret_cast<float*>(smem);          // [warps][NH][D]
  float* red_m = red_o + kConsumerWarps * NH * D;         // [warps][NH]
  float* red_l = red_m + kConsumerWarps * NH;             // [warps][NH]
#pragma unroll
  for (int mt = 0; mt < KS; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n0 = nt * 8 + 2 * t;
      const int d0 = mt * 16 + g;
      float* base = red_o + (warp * NH + n0) * D;
      base[d0] = o[mt][nt][0];
      base[D + d0] = o[mt][nt][1];
      base[d0 + 8] = o[mt][nt][2];
      base[D + d0 + 8] = o[mt][nt][3];
    }
  if (g == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        red_m[warp * NH + nt * 8 + 2 * t + j] = m[nt][j];
        red_l[warp * NH + nt * 8 + 2 * t + j] = l[nt][j];
      }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));

  const size_t bh0 = static_cast<size_t>(b) * H + kvh * group;
  for (int idx = threadIdx.x; idx < group * D; idx += kConsumerWarps * 32) {
    const int n = idx / D, d = idx - n * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red_m[w * NH + n]);
    const float Mref = (M == -INFINITY) ? 0.f : M;
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float sc = fast_exp2(red_m[w * NH + n] - Mref);
      acc += red_o[(w * NH + n) * D + d] * sc;
      L += red_l[w * NH + n] * sc;
    }
    const size_t pidx = (bh0 + n) * n_splits + split;
    part_o[pidx * D + d] = acc;
    if (d == 0) {
      part_ml[pidx * 2] = M;
      part_ml[pidx * 2 + 1] = L;
    }
  }
  if (pub.peers != nullptr) publish_group<D>(pub, part_o, part_ml, b, kvh, H, group, len,
                                             split_rows, n_splits);
}

// ---------------------------------------------------------------------------
// FMA kernel (f32 caches, and any head_dim multiple of 32 up to 256)
// ---------------------------------------------------------------------------
constexpr int kFmaWarps = 4;

template <typename T, int DL, int kFmaMaxGroup>
__global__ void __launch_bounds__(kFmaWarps * 32) decode_fma_kernel(
    const float* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
    const int* __restrict__ lens, float* __restrict__ part_o, float* __restrict__ part_ml, int H,
    int KV, int group, long long seq_stride, int split_rows, int n_splits, float qscale) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  pdl_wait();  // q and the newest rows come from the kernels before
  constexpr int D = DL * 32;
  extern __shared__ float fsm[];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int len = lens[b];
  const int row0 = split * split_rows;
  if (row0 >= len) return;
  const int row1 = min(len, row0 + split_rows);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  float qv[kFmaMaxGroup][DL];
  float o[kFmaMaxGroup][DL];
  float m[kFmaMaxGroup], l[kFmaMaxGroup];
  const float* qb = q + (static_cast<size_t>(b) * H + kvh * group) * D;
#pragma unroll
  for (int n = 0; n < kFmaMaxGroup; ++n) {
    m[n] = -INFINITY;
    l[n] = 0.f;
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      qv[n][i] = n < group ? qb[n * D + i * 32 + lane] * qscale : 0.f;
      o[n][i] = 0.f;
    }
  }
  const size_t row_stride = static_cast<size_t>(KV) * D;
  const T* kb = kc + static_cast<size_t>(b) * seq_stride + static_cast<size_t>(kvh) * D;
  const T* vb = vc + static_cast<size_t>(b) * seq_stride + static_cast<size_t>(kvh) * D;
  for (int r = row0 + warp; r < row1; r += kFmaWarps) {
    float kv[DL], vv[DL];
#pragma unroll
    for (int i = 0; i < DL; ++i) {
      kv[i] = ld_elem(kb + r * row_stride + i * 32 + lane);
      vv[i] = ld_elem(vb + r * row_stride + i * 32 + lane);
    }
#pragma unroll
    for (int n = 0; n < kFmaMaxGroup; ++n) {
      if (n < group) {
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) dot = fmaf(qv[n][i], kv[i], dot);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float mnew = fmaxf(m[n], dot);
        const float alpha = exp2f(m[n] - mnew);
        const float p = exp2f(dot - mnew);
        m[n] = mnew;
        l[n] = l[n] * alpha + p;
#pragma unroll
        for (int i = 0; i < DL; ++i) o[n][i] = fmaf(o[n][i], alpha, p * vv[i]);
      }
    }
  }
  // merge warps
  float* red_o = fsm;                                 // [warps][group][D]
  float* red_m = red_o + kFmaWarps * group * D;       // [warps][group]
  float* red_l = red_m + kFmaWarps * group;
#pragma unroll
  for (int n = 0; n < kFmaMaxGroup; ++n) {
    if (n < group) {
#pragma unroll
      for (int i = 0; i < DL; ++i) red_o[(warp * group + n) * D + i * 32 + lane] = o[n][i];
      if (lane == 0) {
        red_m[warp * group + n] = m[n];
        red_l[warp * group + n] = l[n];
      }
    }
  }
  __syncthreads();
  const size_t bh0 = static_cast<size_t>(b) * H + kvh * group;
  for (int idx = threadIdx.x; idx < group * D; idx += kFmaWarps * 32) {
    const int n = idx / D, d = idx - n * D;
    float M = -INFINITY;
    for (int w = 0; w < kFmaWarps; ++w) M = fmaxf(M, red_m[w * group + n]);
    const float Mref = (M == -INFINITY) ? 0.f : M;
    float acc = 0.f, L = 0.f;
    for (int w = 0; w < kFmaWarps; ++w) {
      const float sc = exp2f(red_m[w * group + n] - Mref);
      acc += red_o[(w * group + n) * D + d] * sc;
      L += red_l[w * group + n] * sc;
    }
    const size_t pidx = (bh0 + n) * n_splits + split;
    part_o[pidx * D + d] = acc;
    if (d == 0) {
      part_ml[pidx * 2] = M;
      part_ml[pidx * 2 + 1] = L;
    }
  }
}

// ---------------------------------------------------------------------------
// Split combine: one CTA per (sequence, head)
// ---------------------------------------------------------------------------
constexpr int kCombineThreads = 128;

__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_ml,
    const int* __restrict__ lens, float* __restrict__ out, float* __restrict__ lse, int H, int D,
    int split_rows, int n_splits, int row_limit) {
  // a programmatic dependent launched after this kernel may start its
  // independent prologue now (it waits for this kernel before reading)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  pdl_wait();  // the partials come from the split kernel before
  extern __shared__ float wsm[];  // [n_splits] weights
  __shared__ float red[kCombineThreads / 32];
  __shared__ float s_M, s_invL;
  const int bh = blockIdx.x, b = bh / H;
  const int len = lens[b];
  if (threadIdx.x == 0 && (len < 0 || len > row_limit)) set_dev_error(B2A_ERR_POSITION, b);
  const int ns = (len <= 0) ? 0 : min(n_splits, (len + split_rows - 1) / split_rows);
  const size_t p0 = static_cast<size_t>(bh) * n_splits;
  if (ns == 0) {
    for (int d = threadIdx.x; d < D; d += kCombineThreads) out[static_cast<size_t>(bh) * D + d] = 0.f;
    if (lse && threadIdx.x == 0) lse[bh] = -INFINITY;
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float M = -INFINITY;
  for (int s = threadIdx.x; s < ns; s += kCombineThreads) M = fmaxf(M, part_ml[(p0 + s) * 2]);
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (threadIdx.x == 0) {
    float x = red[0];
    for (int w = 1; w < kCombineThreads / 32; ++w) x = fmaxf(x, red[w]);
    s_M = x;
  }
  __syncthreads();
  M = s_M;
  float L = 0.f;
  for (int s = threadIdx.x; s < ns; s += kCombineThreads) {
    const float w = exp2f(part_ml[(p0 + s) * 2] - M);
    wsm[s] = w;
    L += part_ml[(p0 + s) * 2 + 1] * w;
  }
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  __syncthreads();
  if (threadIdx.x == 0) {
    float x = 0.f;
    for (int w = 0; w < kCombineThreads / 32; ++w) x += red[w];
    s_invL = 1.f / x;
    if (lse) lse[bh] = (M + log2f(x)) * 0.6931471805599453f;
  }
  __syncthreads();
  const float invL = s_invL;
  if (D <= kCombineThreads) {
    // every thread works: thread t sums splits t / D, t / D + nh, ... of
    // output column t % D (four loads in flight), then the nh partial sums
    // of each column meet in shared memory in a fixed order
    const int nh = kCombineThreads / D, h = threadIdx.x / D, d = threadIdx.x - h * D;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (h < nh) {
      int s = h;
      for (; s + 3 * nh < ns; s += 4 * nh) {
        a0 += part_o[(p0 + s) * D + d] * wsm[s];
        a1 += part_o[(p0 + s + nh) * D + d] * wsm[s + nh];
        a2 += part_o[(p0 + s + 2 * nh) * D + d] * wsm[s + 2 * nh];
        a3 += part_o[(p0 + s + 3 * nh) * D + d] * wsm[s + 3 * nh];
      }
      for (; s < ns; s += nh) a0 += part_o[(p0 + s) * D + d] * wsm[s];
    }
    __shared__ float part[kCombineThreads];
    part[threadIdx.x] = (a0 + a1) + (a2 + a3);
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < D) {
      float acc = 0.f;
      for (int j = 0; j < nh; ++j) acc += part[j * D + threadIdx.x];
      out[static_cast<size_t>(bh) * D + threadIdx.x] = acc * invL;
    }
  } else {
    for (int d = threadIdx.x; d < D; d += kCombineThreads) {
      float a0 = 0.f, a1 = 0.f;
      int s = 0;
      for (; s + 1 < ns; s += 2) {
        a0 += part_o[(p0 + s) * D + d] * wsm[s];
        a1 += part_o[(p0 + s + 1) * D + d] * wsm[s + 1];
      }
      if (s < ns) a0 += part_o[(p0 + s) * D + d] * wsm[s];
      out[static_cast<size_t>(bh) * D + d] = (a0 + a1) * invL;
    }
  }
}

// ---------------------------------------------------------------------------
// Cross-shard log-sum-exp combine (normalised parts, natural-log lse)
// ---------------------------------------------------------------------------
__global__ void lse_combine_kernel(const float* __restrict__ o_parts, long long o_stride,
                                   const float* __restrict__ lse_parts, long long lse_stride,
                                   int G, int rows, int D, float* __restrict__ out,
                                   float* __restrict__ lse_out) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  pdl_wait();  // the parts may come from the kernel before
  const int r = blockIdx.x;
  float M = -INFINITY;
  for (int g = 0; g < G; ++g) M = fmaxf(M, lse_parts[g * lse_stride + r]);
  const float Mref = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  for (int g = 0; g < G; ++g) L += expf(lse_parts[g * lse_stride + r] - Mref);
  const float invL = (L > 0.f) ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int g = 0; g < G; ++g) {
      const float w = expf(lse_parts[g * lse_stride + r] - Mref);
      acc += w * o_parts[g * o_stride + static_cast<size_t>(r) * D + d];
    }
    out[static_cast<size_t>(r) * D + d] = acc * invL;
  }
  if (lse_out && threadIdx.x == 0) lse_out[r] = (L > 0.f) ? Mref + logf(L) : -INFINITY;
}

}  // namespace decode
}  // namespace b2a

// ===========================================================================
// Host side
// ===========================================================================
namespace {

namespace Dk = b2a::decode;
using Dk::decode_mma_kernel;
using Dk::decode_fma_kernel;
using Dk::decode_combine_kernel;
using Dk::lse_combine_kernel;
using Dk::kRows;
using Dk::kFmaWarps;
using Dk::kCombineThreads;
using Dk::smem_bytes;
using b2a_host::fail;

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int n_splits_of(int max_len, int split_rows) {
  return max_len <= 0 ? 0 : (max_len + split_rows - 1) / split_rows;
}

size_t part_o_bytes(int B, int H, int D, int n_splits) {
  return round_up(static_cast<size_t>(B) * H * n_splits * D * sizeof(float), 256);
}

template <typename T, int D, int NT>
int launch_mma(const CUtensorMap& tk, const CUtensorMap& tv, const float* q, const int* lens,
               float* part_o, float* part_ml, int B, int H, int KV, int group, int split_rows,
               int n_splits, float qscale, const b2a::shard::Publish& pub, cudaStream_t st) {
  auto kern = decode_mma_kernel<T, D, NT>;
  constexpr int smem = smem_bytes<D, NT>();
  static unsigned long long configured = 0;  // bit per device: attribute set
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(decode)");
    if (dev < 64) configured |= (1ull << dev);
  }
  dim3 grid(n_splits, KV, B);
  const cudaError_t e = b2a_host::launch(kern, grid, dim3(Dk::kThreads), smem, st, tk, tv, q, lens,
                                         part_o, part_ml, H, group, split_rows, n_splits, qscale,
                                         pub);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode launch");
  return B2A_OK;
}

template <typename T, int D>
int dispatch_nt(int group, const CUtensorMap& tk, const CUtensorMap& tv, const float* q,
                const int* lens, float* po, float* pml, int B, int H, int KV, int split_rows,
                int n_splits, float qscale, const b2a::shard::Publish& pub, cudaStream_t st) {
  if (group <= 8)
    return launch_mma<T, D, 1>(tk, tv, q, lens, po, pml, B, H, KV, group, split_rows, n_splits,
                               qscale, pub, st);
  return launch_mma<T, D, 2>(tk, tv, q, lens, po, pml, B, H, KV, group, split_rows, n_splits,
                             qscale, pub, st);
}

template <typename T>
int dispatch_d(int D, int group, const CUtensorMap& tk, const CUtensorMap& tv, const float* q,
               const int* lens, float* po, float* pml, int B, int H, int KV, int split_rows,
               int n_splits, float qscale, const b2a::shard::Publish& pub, cudaStream_t st) {
  switch (D) {
    case 64:
      return dispatch_nt<T, 64>(group, tk, tv, q, lens, po, pml, B, H, KV, split_rows, n_splits,
                                qscale, pub, st);
    case 128:
      return dispatch_nt<T, 128>(group, tk, tv, q, lens, po, pml, B, H, KV, split_rows, n_splits,
                                 qscale, pub, st);
    case 256:
      return dispatch_nt<T, 256>(group, tk, tv, q, lens, po, pml, B, H, KV, split_rows, n_splits,
                                 qscale, pub, st);
  }
  return fail(B2A_ERR_UNSUPPORTED, "decode: head_dim %d (tensor-core path takes 64/128/256)", D);
}

template <int DL, int MG>
int launch_fma(const float* q, const float* kc, const float* vc, const int* lens, float* po,
               float* pml, int B, int H, int KV, int group, long long seq_stride, int split_rows,
               int n_splits, float qscale, cudaStream_t st) {
  auto kern = decode_fma_kernel<float, DL, MG>;
  const int smem = (kFmaWarps * group * (DL * 32 + 2)) * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "cudaFuncSetAttribute(decode_fma)");
  }
  dim3 grid(n_splits, KV, B);
  const cudaError_t e = b2a_host::launch(kern, grid, dim3(kFmaWarps * 32), smem, st, q, kc, vc,
                                         lens, po, pml, H, KV, group, seq_stride, split_rows,
                                         n_splits, qscale);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_fma launch");
  return B2A_OK;
}

template <int DL>
int fma_group(int group, const float* q, const float* kc, const float* vc, const int* lens,
              float* po, float* pml, int B, int H, int KV, long long ss, int sr, int ns, float qs,
              cudaStream_t st) {
  if (group <= 4) return launch_fma<DL, 4>(q, kc, vc, lens, po, pml, B, H, KV, group, ss, sr, ns, qs, st);
  if (group <= 8) return launch_fma<DL, 8>(q, kc, vc, lens, po, pml, B, H, KV, group, ss, sr, ns, qs, st);
  return launch_fma<DL, 16>(q, kc, vc, lens, po, pml, B, H, KV, group, ss, sr, ns, qs, st);
}

}  // namespace

extern "C" {

int b2a_decode_split_rows(int B, int KV, int max_len, int kv_dtype) {
  // Long splits: each CTA's fixed cost (pipeline fill, partial write, its
  // share of the combine) is paid once per split, so rows per CTA grow up
  // to 8192 while there are more CTAs than SMs and every sequence of
  // max_len keeps at least 4 splits (ragged batches, whose sequences are
  // often far shorter than max_len, then still spread their rows).  At
  // least 256 rows.  Measured on one B200 (bf16, 32/8 heads x 128 at 16 x
  // 32K rows): 2048-row splits 6544 GB/s, 8192-row 6977; 16/2 heads x 256:
  // 512-row 4921, 8192-row 6666; lengths U[1K, 8K] x 64 (f16): 2048-row
  // 6446, 8192-row 5898.
  (void)kv_dtype;
  if (B <= 0 || KV <= 0 || max_len <= 0) return kRows * 4;
  const double rows_total = static_cast<double>(B) * KV * max_len;
  int sr = kRows;
  while (sr < 8192 && 8LL * sr <= max_len && rows_total / sr > b2a_host::sm_count()) sr *= 2;
  if (sr < 4 * kRows) sr = 4 * kRows;
  return sr;
}

size_t b2a_decode_workspace_bytes(int B, int H, int D, int max_len, int split_rows) {
  if (B <= 0 || H <= 0 || D <= 0 || max_len <= 0) return 0;
  if (split_rows <= 0) split_rows = 4 * kRows;
  const int ns = n_splits_of(max_len, split_rows);
  return part_o_bytes(B, H, D, ns) + round_up(static_cast<size_t>(B) * H * ns * 2 * sizeof(float), 256);
}

}  // extern "C"

namespace {

// Argument checks and the split kernel of a decode call (everything but the
// combine): the partials land in the workspace, part_o then part_ml.  On
// success *ns_out holds the number of splits and *split_rows_io the split.
int decode_split_phase(const float* q, const void* k_cache, const void* v_cache,
                       const int* lens_dev, const void* out, void* workspace,
                       size_t workspace_bytes, int B, int H, int KV, int D, int n_ctx,
                       long long seq_stride, int kv_dtype, float scale, int max_len,
                       int* split_rows_io, int* ns_out, float** part_o_out, float** part_ml_out,
                       cudaStream_t st, const b2a::shard::Publish& pub = {nullptr, 0, 0},
                       bool* published = nullptr) {
  if (published) *published = false;
  if (!q || !k_cache || !v_cache || !lens_dev || !out)
    return fail(B2A_ERR_ARG, "decode: null pointer argument");
  if (B <= 0 || H <= 0 || KV <= 0 || D <= 0 || n_ctx <= 0 || max_len < 0)
    return fail(B2A_ERR_ARG, "decode: sizes must be positive (B=%d H=%d KV=%d D=%d n_ctx=%d max_len=%d)",
                B, H, KV, D, n_ctx, max_len);
  if (H % KV != 0) return fail(B2A_ERR_SHAPE, "decode: H=%d is not a multiple of KV=%d", H, KV);
  const int group = H / KV;
  if (group > 16) return fail(B2A_ERR_UNSUPPORTED, "decode: group %d > 16", group);
  if (max_len > n_ctx) return fail(B2A_ERR_SHAPE, "decode: max_len %d > n_ctx %d", max_len, n_ctx);
  const long long seq_elems = static_cast<long long>(n_ctx) * KV * D;
  if (B > 1 && seq_stride < seq_elems)
    return fail(B2A_ERR_SHAPE, "decode: seq_stride %lld < n_ctx*KV*D %lld", seq_stride, seq_elems);
  if (B == 1 || seq_stride <= 0) seq_stride = seq_elems;
  const int es = b2a_host::elem_size(kv_dtype);
  if (es == 0) return fail(B2A_ERR_DTYPE, "decode: kv_dtype %d", kv_dtype);
  if (!(scale > 0.f) || !isfinite(scale)) return fail(B2A_ERR_ARG, "decode: scale must be positive");
  int split_rows = *split_rows_io;
  if (split_rows <= 0) split_rows = b2a_decode_split_rows(B, KV, max_len, kv_dtype);
  if (split_rows % kRows != 0)
    return fail(B2A_ERR_ARG, "decode: split_rows %d is not a multiple of %d", split_rows, kRows);
  const int ns = n_splits_of(max_len, split_rows);
  const size_t need = b2a_decode_workspace_bytes(B, H, D, max_len, split_rows);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(B2A_ERR_WORKSPACE, "decode: workspace %zu bytes < %zu needed", workspace_bytes, need);
  if (!b2a_host::aligned16(q) || !b2a_host::aligned16(workspace))
    return fail(B2A_ERR_ALIGN, "decode: q and workspace must be 16-byte aligned");
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                            (ns > 0 ? part_o_bytes(B, H, D, ns) : 0));
  const float qscale = scale * Dk::kLog2e;

  int rc = B2A_OK;
  if (ns > 0) {
    if (kv_dtype == B2A_F32) {
      if (D % 32 != 0 || (D != 64 && D != 128 && D != 256))
        return fail(B2A_ERR_UNSUPPORTED, "decode: fp32 cache head_dim %d (64/128/256)", D);
      const float* kc = static_cast<const float*>(k_cache);
      const float* vc = static_cast<const float*>(v_cache);
      if (D == 64)
        rc = fma_group<2>(group, q, kc, vc, lens_dev, part_o, part_ml, B, H, KV, seq_stride, split_rows, ns, qscale, st);
      else if (D == 128)
        rc = fma_group<4>(group, q, kc, vc, lens_dev, part_o, part_ml, B, H, KV, seq_stride, split_rows, ns, qscale, st);
      else
        rc = fma_group<8>(group, q, kc, vc, lens_dev, part_o, part_ml, B, H, KV, seq_stride, split_rows, ns, qscale, st);
    } else {
      if (D != 64 && D != 128 && D != 256)
        return fail(B2A_ERR_UNSUPPORTED, "decode: head_dim %d (tensor-core path takes 64/128/256)", D);
      if (!b2a_host::aligned16(k_cache) || !b2a_host::aligned16(v_cache) || (seq_stride * es) % 16 != 0)
        return fail(B2A_ERR_ALIGN, "decode: caches and seq_stride must be 16-byte aligned");
      const CUtensorMapDataType tdt =
          kv_dtype == B2A_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
      const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(KV),
                                static_cast<uint64_t>(n_ctx), static_cast<uint64_t>(B)};
      const uint64_t strides[3] = {static_cast<uint64_t>(D) * es, static_cast<uint64_t>(KV) * D * es,
                                   static_cast<uint64_t>(seq_stride) * es};
      const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kRows), 1};
      CUtensorMap tk, tv;
      rc = b2a_host::make_tmap(&tk, tdt, 4, const_cast<void*>(k_cache), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      rc = b2a_host::make_tmap(&tv, tdt, 4, const_cast<void*>(v_cache), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      if (kv_dtype == B2A_BF16)
        rc = dispatch_d<__nv_bfloat16>(D, group, tk, tv, q, lens_dev, part_o, part_ml, B, H, KV,
                                       split_rows, ns, qscale, pub, st);
      else
        rc = dispatch_d<__half>(D, group, tk, tv, q, lens_dev, part_o, part_ml, B, H, KV,
                                split_rows, ns, qscale, pub, st);
      if (published) *published = pub.peers != nullptr;
    }
    if (rc) return rc;
  }
  const int smem = ns * static_cast<int>(sizeof(float));
  if (smem > 48 * 1024) return fail(B2A_ERR_UNSUPPORTED, "decode: %d splits exceed the combine limit", ns);
  *split_rows_io = split_rows;
  *ns_out = ns;
  *part_o_out = part_o;
  *part_ml_out = part_ml;
  return B2A_OK;
}

}  // namespace

extern "C" {

int b2a_decode(const float* q, const void* k_cache, const void* v_cache, const int* lens_dev,
               float* out, float* lse_out, void* workspace, size_t workspace_bytes, int B, int H,
               int KV, int D, int n_ctx, long long seq_stride, int kv_dtype, float scale,
               int max_len, int split_rows, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int ns = 0;
  float *part_o = nullptr, *part_ml = nullptr;
  const int rc = decode_split_phase(q, k_cache, v_cache, lens_dev, out, workspace,
                                    workspace_bytes, B, H, KV, D, n_ctx, seq_stride, kv_dtype,
                                    scale, max_len, &split_rows, &ns, &part_o, &part_ml, st);
  if (rc) return rc;
  const int smem = ns * static_cast<int>(sizeof(float));
  cudaError_t e = b2a_host::launch(decode_combine_kernel, dim3(B * H), dim3(kCombineThreads), smem,
                                   st, part_o, part_ml, lens_dev, out, lse_out, H, D, split_rows,
                                   ns, max_len);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode launch");
  return B2A_OK;
}

int b2a_lse_combine(const float* o_parts, long long o_part_stride, const float* lse_parts,
                    long long lse_part_stride, int G, int rows, int D, float* out,
                    float* lse_out, void* stream) {
  if (!o_parts || !lse_parts || !out) return fail(B2A_ERR_ARG, "lse_combine: null pointer argument");
  if (G <= 0 || rows <= 0 || D <= 0) return fail(B2A_ERR_ARG, "lse_combine: sizes must be positive");
  if (o_part_stride == 0) o_part_stride = static_cast<long long>(rows) * D;
  if (lse_part_stride == 0) lse_part_stride = rows;
  if (o_part_stride < static_cast<long long>(rows) * D || lse_part_stride < rows)
    return fail(B2A_ERR_SHAPE, "lse_combine: part strides overlap the parts");
  cudaError_t e = b2a_host::launch(lse_combine_kernel, dim3(rows), dim3(128), 0,
                                   static_cast<cudaStream_t>(stream), o_parts, o_part_stride,
                                   lse_parts, lse_part_stride, G, rows, D, out, lse_out);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "lse_combine launch");
  return B2A_OK;
}

}  // extern "C"

// ===========================================================================
// Decode for callers that cannot allocate device memory
// ===========================================================================
// Some callers of this library can't call cudaMalloc. A serving process may
// have reserved nearly all of HBM for its KV cache, or may run behind an
// allocator that owns every device buffer. An embedding host across an FFI
// may have no device allocator at all. For them, b2a_decode_noalloc keeps
// the split partials in this fixed file-scope array instead of a
// caller-supplied workspace. Every GPU that loads the library holds the
// array until the process exits.
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = B2A_DECODE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
struct ScratchSlot {
  void* ctx;   // CUDA context the address belongs to
  void* addr;  // device address of g_decode_scratch in that context
};
ScratchSlot g_scratch_addr[64] = {};  // per device ordinal

typedef CUresult (*PFN_ctxGetCurrent)(CUcontext*);

// The calling thread's current CUDA context (driver entry point, no -lcuda
// link); null if it cannot be read.
void* current_context() {
  static PFN_ctxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_ctxGetCurrent>(p);
  });
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// Device address of the scratch array on the current device. The host-side
// name g_decode_scratch is only a stand-in, so the address is looked up with
// that device current, once per device and context: a context made after
// cudaDeviceReset (which reloads the module) gets a fresh lookup.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B2A_ERR_UNSUPPORTED, "decode_noalloc: device %d >= 64", dev);
  void* ctx = current_context();  // null before the runtime made one
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch_addr[dev];
  if (!slot.addr || !ctx || slot.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return b2a_host::cuda_fail(e, "decode_noalloc: cudaGetSymbolAddress");
    if (!p) return fail(B2A_ERR_CUDA, "decode_noalloc: cudaGetSymbolAddress returned a null address");
    slot.ctx = current_context();  // the lookup made the context if there was none
    slot.addr = p;
  }
  *out = slot.addr;
  return B2A_OK;
}

}  // namespace

extern "C" int b2a_decode_noalloc(const float* q, const void* k_cache, const void* v_cache,
                                  const int* lens_dev, float* out, float* lse_out, int B, int H,
                                  int KV, int D, int n_ctx, long long seq_stride, int kv_dtype,
                                  float scale, int max_len, int split_rows, void* stream) {
  if (B <= 0 || H <= 0 || KV <= 0 || D <= 0 || max_len < 0)
    return fail(B2A_ERR_ARG, "decode_noalloc: sizes must be positive");
  if (split_rows <= 0) split_rows = b2a_decode_split_rows(B, KV, max_len, kv_dtype);
  const size_t need = b2a_decode_workspace_bytes(B, H, D, max_len, split_rows);
  if (need > kNoAllocScratchBytes)
    return fail(B2A_ERR_WORKSPACE,
                "decode_noalloc: B=%d H=%d D=%d max_len=%d split_rows=%d needs %zu bytes of "
                "scratch but the static array holds %zu; raise split_rows or call b2a_decode "
                "with a caller workspace",
                B, H, D, max_len, split_rows, need, kNoAllocScratchBytes);
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc) return rc;
  // The partials need no clearing: each CTA writes every partial the combine
  // kernel later reads for this call.
  return b2a_decode(q, k_cache, v_cache, lens_dev, out, lse_out, ws, kNoAllocScratchBytes, B, H,
                    KV, D, n_ctx, seq_stride, kv_dtype, scale, max_len, split_rows, stream);
}
