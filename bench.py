#!/usr/bin/env python
"""Benchmark of the B200 attention path (one JSON line on stdout, rank 0).

Headline (`value`): split-KV decode attention at 32K context, the workload
the reference's metric is quoted on ("decode-attn KV GB/s @32K ctx"):
batch 16 sequences x 32768 cached tokens, 32 query / 8 KV heads, head_dim
128, bf16 KV ~ N(0,1) (seed 4 + rank).  One step = one b2a_decode call over
the whole batch (split kernel + combine kernel).  value = algorithmic KV
bytes (B*2*L*KV*D*2 per rank, all ranks) / max-over-ranks device time.
The caches (2.15 GB per rank) exceed the 126 MB L2, so no flush is needed.

Also reported on the same line:
  prefill   benchmark config 2 causal prefill (S=2048, 32/8 heads, D=128,
            bf16 in/out) in TFLOP/s, flops = 4*H*D*S(S+1)/2, L2 flushed
            between launches (inputs are 24 MB)
  varlen    benchmark config 3: one batch of 64 sequences of ragged length
            (1K-8K), sharded by sequence over the GPUs, fp16 KV, fused
            RoPE+append then decode, GB/s
  longctx   benchmark config 4: 4 x 131072 rows split over the GPUs; one CUDA
            graph per step: local split-KV decode, then one kernel that
            exchanges the ranks' (o, lse) rows over NVLink peer memory and
            merges them (the NCCL all-gather path and the one-GPU decode
            beside it, with the efficiency value_N / (N value_1)), GB/s
  kvstate   KV state boundary: device widening/narrowing of one 32K-row bf16
            layer (HBM GB/s) and a whole-layer f32 snapshot
  qwen35_layer  Qwen35 full-attention layer step (prologue, decode, gate) at
            16 x 32K rows, 16/2 heads, head_dim 256, bf16, GB/s
  decode_step  benchmark config 5: a whole decode token of a 16-layer Q8_0
            llama decoder as one CUDA graph, tokens/s (device and e2e)
  prefill_chunk  a 2048-token prefill chunk of the same model kept on the
            device, tokens/s and TFLOP/s
  gemm      the chunk's four projections (tcgen05 b2a_gemm with the chunk's
            epilogues) at those shapes, TFLOP/s, with cuBLAS beside each
  e2e       the decode step through the public API with host buffers
            (DecodeStep, one CUDA graph per token): per step the pinned host
            q/k/v rows and positions go H2D, the fused RoPE+append writes
            them into the resident cache, decode runs, the output comes back
            D2H and the host waits for it
  roofline  decode against MEASURED_PEAKS.json's copy bandwidth
  cpu_baseline  the reference's NumPy decode (oracle port) on host cores

Multi-GPU (torchrun, one rank per GPU): for the headline every rank decodes
its own batch of 16 sequences (sequence sharding, no collective on the data
path), so its scaling is weak; config 3 shards one batch of 64 sequences and
config 4 shards the rows of 4 sequences (strong scaling).  Timing is the max
over ranks of CUDA-event time; e2e runs on every rank at once and takes the
slowest rank's step.  The single-GPU legs (kvstate, qwen35_layer,
decode_step, prefill_chunk, gemm) run only when the job has one GPU.

`--impl reference` times the reference's CPU implementation (the NumPy
restatement in oracle/, the reference itself being Python that does not
travel to the GPU box) on the same workload definition, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode-attn KV GB/s (% HBM peak) @32K ctx; prefill-attn TFLOPS; at 1/2/4/8 GPU"
WL = dict(B=16, L=32768, H=32, KV=8, D=128)            # decode workload (per rank)
PF = dict(S=2048, H=32, KV=8, D=128)                   # prefill workload (config 2)
LC = dict(B=4, L=131072, H=64, KV=8, D=128)            # long-context split (config 4)
VL = dict(B=64, Lmin=1024, Lmax=8192, H=32, KV=8, D=128)  # varlen batched decode (config 3)
FALLBACK_HBM = 6650.0
FALLBACK_BF16 = 1590.0
SPEC_HBM = 8000.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def decode_bytes(B, L, KV, D, elem=2):
    return B * 2 * L * KV * D * elem


def prefill_flops(S, H, D):
    return 4 * H * D * S * (S + 1) / 2


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return (float(j["hbm_gbs"]), float(j["bf16_tflops"]),
                float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured")
    except Exception:
        return FALLBACK_HBM, FALLBACK_BF16, 1400.0, "fallback"


# Per-launch DRAM traffic, dram__bytes_read.sum + dram__bytes_write.sum, from the ncu
# captures summarised in profiles/decode_mma_bf16_32k.md (2 sequences, scaled x8 to the
# 16-sequence launch: reads scale with the rows) and profiles/prefill_pair_bf16_s2048.md
# (one full config-2 launch).
NCU_TRAFFIC = {
    "decode_mma_kernel bf16 D128 NT1": 2179069952.0,
    "prefill_pair_kernel bf16 D128": 25243392.0,
}


def profiled_traffic(name):
    """Per-launch DRAM traffic of `name` from an ncu capture (None if not captured)."""
    return NCU_TRAFFIC.get(name)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu_id], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(dev_index):
    import torch
    try:
        u = str(torch.cuda.get_device_properties(dev_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[dev_index] if vis else str(dev_index)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def bench_decode(dev, rank, steps, warmup, dist):
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    B, L, H, KV, D = WL["B"], WL["L"], WL["H"], WL["KV"], WL["D"]
    log(f"decode workload B={B} L={L} H={H} KV={KV} D={D}")
    g = torch.Generator(device=dev).manual_seed(4 + rank)
    kc = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    vc = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    q = torch.randn((B, H, D), device=dev, dtype=torch.float32, generator=g)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    split = device.decode_split_rows(B, KV, L, torch.bfloat16)
    ws = device.decode_workspace(B, H, D, L, split, dev)
    out = torch.empty((B, H, D), dtype=torch.float32, device=dev)

    def step():
        device.decode(q, kc, vc, lens, out=out, workspace=ws, split_rows=split, max_len=L)

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    return dict(ms=ms, split=split, kc=kc, vc=vc, q=q, lens=lens, ws=ws, out=out)


def _timed_steps(fn, nsteps, dev, dist):
    """CUDA-event time of nsteps calls of fn on this rank, then the max over
    ranks (ms); barrier + synchronize on both sides."""
    import torch
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(nsteps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    return ms


def bench_longctx(dev, rank, world, steps, warmup, dist):
    """benchmark config 4: 4 sequences x 131072 rows, 64 q / 8 KV heads, D=128,
    bf16; the KV rows of every sequence are split across the ranks (strong
    scaling).  One step, replayed as a CUDA graph: the split-KV decode of the
    rank's rows, then b2a_decode_sharded's fused kernel (split merge, NVLink
    peer stores of the rank's (o, lse) rows into every rank's exchange
    buffer, bounded flag waits, LSE merge).  Beside it: the same step with an
    NCCL all-gather + LSE-combine kernel instead (eager), and the whole
    unsharded decode on one GPU, for the efficiency value_N / (N value_1)."""
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.longctx import LongContextDecoder, shard_rows
    B, L, H, KV, D = LC["B"], LC["L"], LC["H"], LC["KV"], LC["D"]
    a, b = shard_rows(L, rank, world)
    n = b - a
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    ks = torch.randn((B, n, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    vs = torch.randn((B, n, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    gq = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn((B, H, D), device=dev, dtype=torch.float32, generator=gq)
    lens = torch.full((B,), n, dtype=torch.int32, device=dev)
    nsteps = max(10, min(steps, 500))
    per_step = decode_bytes(B, L, KV, D)

    dec = LongContextDecoder(exchange="p2p")
    replay, _ = dec.graph(q, ks, vs, lens, max_len=n)
    for _ in range(max(warmup, 3)):
        replay()
    ms = _timed_steps(replay, nsteps, dev, dist)
    del replay
    dec.close()
    res = {"metric": "long-context split decode KV GB/s (config 4)",
           "value": round(per_step / (ms / nsteps * 1e-3) / 1e9, 1), "unit": "GB/s",
           "ms_per_step": round(ms / nsteps, 4), "steps": nsteps, "n_gpus": world,
           "scaling": "strong", "gpu_launches_per_step": 2,
           "config": "4 seqs x 131072 rows (split over the GPUs), 64 q / 8 KV heads, D=128, "
                     "bf16; per step (one CUDA graph): split-KV decode of the local rows, "
                     "then one kernel that merges the splits, stores each rank's (o, lse) "
                     "rows into every rank's buffer over NVLink and merges the ranks' parts"}
    if world > 1:
        ndec = LongContextDecoder(exchange="nccl")
        call = lambda: ndec.decode(q, ks, vs, lens, max_len=n)  # noqa: E731
        for _ in range(max(warmup, 3)):
            call()
        ms_n = _timed_steps(call, nsteps, dev, dist)
        res["nccl_exchange"] = {
            "value": round(per_step / (ms_n / nsteps * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(ms_n / nsteps, 4),
            "path": "eager: decode with lse, NCCL all_gather_into_tensor of the packed "
                    "parts, LSE-combine kernel"}
    del ks, vs
    # the unsharded decode on one GPU (rank 0), the N = 1 point of the curve
    if rank == 0:
        torch.cuda.empty_cache()
        g1 = torch.Generator(device=dev).manual_seed(3)
        kf = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g1)
        vf = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g1)
        lf = torch.full((B,), L, dtype=torch.int32, device=dev)
        split = device.decode_split_rows(B, KV, L, torch.bfloat16)
        ws = device.decode_workspace(B, H, D, L, split, dev)
        of = torch.empty((B, H, D), dtype=torch.float32, device=dev)
        one = lambda: device.decode(q, kf, vf, lf, out=of, workspace=ws, split_rows=split)  # noqa: E731
        for _ in range(3):
            one()
        ms1 = _timed_steps(one, nsteps, dev, None)
        v1 = per_step / (ms1 / nsteps * 1e-3) / 1e9
        res["single_gpu_value"] = round(v1, 1)
        res["efficiency"] = round(res["value"] / (world * v1), 4)
        del kf, vf
        torch.cuda.empty_cache()
    if dist is not None:
        dist.barrier()
    return res


def bench_varlen(dev, rank, world, steps, warmup, dist):
    """benchmark config 3: one batch of 64 sequences with cached lengths
    L_b ~ U[1024, 8192] (seed 2), 32 q / 8 KV heads, D=128, fp16 KV ~ N(0,1)
    (seed 2 + rank), sharded by sequence over the GPUs (longctx.place_sequences:
    longest first onto the rank with the fewest rows; no collective).  One step is the device half of
    a batched decode token: the fused RoPE + append kernel rotates every
    sequence's new q/k row at position L_b and stores k/v there, then the
    split-KV decode (split + combine kernels) attends over L_b + 1 rows; the
    step is captured once and replayed as a CUDA graph.  Bytes per step: the
    KV rows read, sum_b 2*(L_b+1)*KV*D*2, plus the new rows and q/out
    traffic, over the whole batch; the time is the max over ranks (strong
    scaling)."""
    import numpy as np
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.longctx import place_sequences
    H, KV, D = VL["H"], VL["KV"], VL["D"]
    Ls_all = np.random.default_rng(2).integers(VL["Lmin"], VL["Lmax"] + 1, size=VL["B"])
    Ls = Ls_all[place_sequences(Ls_all, world)[rank]]
    B = len(Ls)
    n_ctx = VL["Lmax"] + 1
    g = torch.Generator(device=dev).manual_seed(2 + rank)
    kc = torch.randn((B, n_ctx, KV, D), device=dev, dtype=torch.float16, generator=g)
    vc = torch.randn((B, n_ctx, KV, D), device=dev, dtype=torch.float16, generator=g)
    q = torch.randn((B, H, D), device=dev, dtype=torch.float32, generator=g)
    kn = torch.randn((B, KV, D), device=dev, dtype=torch.float32, generator=g)
    vn = torch.randn((B, KV, D), device=dev, dtype=torch.float32, generator=g)
    qr = torch.empty_like(q)
    out = torch.empty_like(q)
    pos = torch.from_numpy(Ls.astype(np.int32)).to(dev)
    lens = pos + 1
    ct, stt = device.rope_tables(n_ctx, D, 500000.0, device=dev)
    split = device.decode_split_rows(B, KV, n_ctx, torch.float16)
    ws = device.decode_workspace(B, H, D, n_ctx, split, dev)

    def step():
        device.rope_append(q, kn, vn, pos, ct, stt, k_cache=kc, v_cache=vc, per_sequence=True,
                           q_out=qr)
        device.decode(qr, kc, vc, lens, out=out, workspace=ws, split_rows=split, max_len=n_ctx)

    # the step replayed as one CUDA graph, as a serving loop runs it (positions and
    # lengths are read on the device): at 8 sequences per GPU the three eager launches'
    # host cost would otherwise set the pace
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            step()
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    nsteps = max(10, min(steps, 1000))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(nsteps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    Bt = VL["B"]
    kv_bytes = int(sum(2 * (int(L) + 1) * KV * D * 2 for L in Ls_all))
    extra = Bt * 2 * KV * D * (4 + 2) + Bt * H * D * 4 * 4  # new rows in/out; q, q_rot x2, out
    per_step = kv_bytes + extra
    local = int(sum(2 * (int(L) + 1) * KV * D * 2 for L in Ls)) + extra * B // Bt
    del graph
    del kc, vc
    return {"metric": "varlen batched decode GB/s (config 3)",
            "value": round(per_step / (ms / nsteps * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(ms / nsteps, 4), "steps": nsteps, "n_gpus": world,
            "scaling": "strong", "bytes_per_step": per_step, "split_rows": split,
            "seqs_per_gpu": B, "gpu_launches_per_step": 3,
            "achieved_per_gpu_max": round(local / (ms / nsteps * 1e-3) / 1e9, 1),
            "config": "one batch of 64 seqs sharded by sequence over the GPUs (balanced "
                      "by rows), L_b ~ "
                      f"U[1024,8192] (seed 2; mean {float(Ls_all.mean()):.0f}), 32 q / 8 KV "
                      "heads, D=128, fp16 KV; per step (one CUDA graph): fused RoPE+append "
                      "of each new token at L_b, split-KV decode over L_b+1 rows; KV bytes > "
                      "L2, no flush"}


def bench_kvstate(dev, steps, warmup):
    """KV state boundary (kvstate.py): one layer of one headline sequence's
    cache, 32768 rows x 8 KV heads x 128, bf16.  Times b2a_kv_convert's
    widening bf16 -> f32 (what a snapshot runs on the device) and the
    narrowing f32 -> bf16 of a restore, each HBM-bound at 6 bytes per
    element (2 read + 4 written or 4 read + 2 written, 201 MB per launch,
    above L2); and a whole-layer snapshot (widen K and V, D2H, host bytes)."""
    import torch
    from alpacca_open_sourced_by_jt_b200.kvstate import DeviceAttentionState, convert
    L, KV, D = 32768, 8, 128
    st = DeviceAttentionState(0, KV, D, D, L, torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(11)
    st.key.copy_(torch.randn(st.key.shape, generator=g, device=dev))
    st.value.copy_(torch.randn(st.value.shape, generator=g, device=dev))
    st.advance(L)
    n = L * KV * D
    k16 = st.key.reshape(-1)
    f32 = torch.empty(n, dtype=torch.float32, device=dev)
    k16b = torch.empty_like(k16)

    def timed(fn, reps):
        for _ in range(max(warmup, 3)):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    reps = max(10, min(steps, 200))
    ms_w = timed(lambda: convert(k16, f32), reps)
    ms_n = timed(lambda: convert(f32, k16b), reps)
    assert torch.equal(k16b, k16)  # narrow(widen(x)) == x for 16-bit x
    # the same widening by torch (its elementwise copy kernel), for the
    # write-heavy traffic's own ceiling on this part
    ms_tw = timed(lambda: f32.copy_(k16), reps)
    st.snapshot()
    t0 = time.perf_counter()
    for _ in range(3):
        snap = st.snapshot()
    ms_s = (time.perf_counter() - t0) / 3 * 1e3
    hbm, _, _, src = peaks()
    bytes_conv = n * 6
    gbs_w = bytes_conv / (ms_w * 1e-3) / 1e9
    return {"metric": "KV snapshot widening GB/s (b2a_kv_convert bf16 -> f32, HBM)",
            "value": round(gbs_w, 1), "unit": "GB/s", "ms_per_launch": round(ms_w, 4),
            "narrow_gbs": round(bytes_conv / (ms_n * 1e-3) / 1e9, 1),
            "narrow_ms_per_launch": round(ms_n, 4),
            "torch_widen_gbs": round(bytes_conv / (ms_tw * 1e-3) / 1e9, 1),
            "snapshot_layer_ms": round(ms_s, 2),
            "snapshot_layer_gbs": round(snap.memory_bytes() / (ms_s * 1e-3) / 1e9, 2),
            "roofline": {"bound": "hbm", "achieved": round(gbs_w, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(gbs_w / hbm, 4),
                         "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)"},
            "config": "one layer, 32768 rows x 8 KV heads x 128, bf16 cache; widening and "
                      "narrowing timed back to back (201 MB per launch); snapshot = K and V "
                      "widened on the device, copied to host f32-le bytes"}


def bench_qwen35(dev, steps, warmup):
    """Qwen35 full-attention layer step (qwen35_layer.py) at a Qwen3.5-style
    shape: 16 sequences x 32768 cached rows, 16 q / 2 KV heads, head_dim 256,
    IMROPE sections (11, 11, 10, 0), bf16 cache.  One step = prologue (split,
    RMSNorm, IMROPE, append), split-KV decode, sigmoid gate; bytes = the KV
    rows read plus the rows and activations moved (HBM-bound)."""
    import numpy as np
    import torch
    from alpacca_open_sourced_by_jt_b200.qwen35_layer import Qwen35AttentionLayer
    B, L, H, KV, D = 16, 32768, 16, 2, 256
    rng = np.random.default_rng(9)
    lay = Qwen35AttentionLayer(query_heads=H, kv_heads=KV, head_dim=D, rms_epsilon=1e-6,
                               rope_freq_base=1e7, sections=(11, 11, 10, 0),
                               query_norm=np.ones(D, np.float32),
                               key_norm=np.ones(D, np.float32), n_ctx=L + 1, batch=B,
                               kv_dtype=torch.bfloat16, device_=dev)
    g = torch.Generator(device=dev).manual_seed(9)
    lay.k_cache.copy_(torch.randn(lay.k_cache.shape, generator=g, device=dev))
    lay.v_cache.copy_(torch.randn(lay.v_cache.shape, generator=g, device=dev))
    qg = torch.from_numpy(rng.standard_normal((B, H * 2 * D), dtype=np.float32)).to(dev)
    k = torch.from_numpy(rng.standard_normal((B, KV * D), dtype=np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((B, KV * D), dtype=np.float32)).to(dev)
    pos = torch.full((B,), L, dtype=torch.int32, device=dev)

    def step():
        lay.step(qg, k, v, pos)

    for _ in range(max(warmup, 3)):
        step()
    n = max(10, min(steps, 500))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    kv_bytes = B * 2 * (L + 1) * KV * D * 2
    extra = B * (H * 2 * D + 2 * KV * D) * 4 + B * H * D * 4 * 4
    gbs = (kv_bytes + extra) / (ms * 1e-3) / 1e9
    hbm, _, _, src = peaks()
    del lay
    return {"metric": "Qwen35 attention layer step GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "steps": n,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4),
                         "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)"},
            "config": "16 seqs x 32768 cached rows, 16 q / 2 KV heads, head_dim 256, IMROPE "
                      "(11,11,10,0), bf16 cache; per step: b2a_qwen35_attn_prep, b2a_decode "
                      "(split + combine), b2a_sigmoid_gate (4 launches plus 2 small torch ops "
                      "for lanes and lengths)"}


C5 = dict(n_layer=16, n_embd=2048, n_head=32, n_kv=8, head_dim=64, n_ff=8192, n_vocab=128256,
          rms_eps=1e-5, rope_base=500000.0)


def bench_decode_step(dev, steps, warmup):
    """benchmark config 5: a whole decode token of a random-init 16-layer
    llama decoder (hidden 2048, 32/8 heads of 64, FFN 8192 SwiGLU, vocab
    128256, RMSNorm 1e-5) with Q8_0 weights N(0, 0.02) (seed 5), an fp16 KV
    cache holding a full 4096-row context, batch 1, the token replayed as one
    CUDA graph (decode_chain.DecodeChain).  value: tokens/s from CUDA events
    over back-to-back graph replays; e2e: tokens/s of chain(token, pos), the
    public call (token/position H2D, logits D2H, host waits each token).
    Bytes per token: the Q8_0 weights read (1.0625 B/weight, one embedding
    row) plus the KV rows attended."""
    import torch
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    n_ctx = 4096
    m = LlamaQ8.random(**C5, seed=5, dev=dev)
    chain = DecodeChain(m, n_ctx, torch.float16)
    g = torch.Generator(device=dev).manual_seed(6)
    for k, v in zip(chain.k_cache, chain.v_cache):
        k.normal_(generator=g)
        v.normal_(generator=g)
    token, pos = 1234, n_ctx - 1
    chain._h_i_np[:] = (token, pos, pos + 1)
    for _ in range(max(warmup, 3)):
        chain._graph.replay()
    n = max(10, min(steps, 500))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        chain._graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    for _ in range(3):
        chain(token, pos)
    t0 = time.perf_counter()
    for _ in range(n):
        chain(token, pos)
    ms_e2e = (time.perf_counter() - t0) / n * 1e3
    kv_bytes = C5["n_layer"] * 2 * n_ctx * C5["n_kv"] * C5["head_dim"] * 2
    per_tok = m.weight_bytes() + kv_bytes
    gbs = per_tok / (ms * 1e-3) / 1e9
    hbm, _, _, src = peaks()
    _lib_err = None
    try:
        from alpacca_open_sourced_by_jt_b200 import _lib
        _lib.raise_device_error()
    except Exception as e:  # surfaced in the JSON rather than lost
        _lib_err = str(e)
    res = {"metric": "config 5 decode tokens/s (whole token, one CUDA graph)",
           "value": round(1e3 / ms, 1), "unit": "tokens/s", "ms_per_token": round(ms, 4),
           "gbs": round(gbs, 1), "bytes_per_token": int(per_tok), "steps": n,
           "gpu_launches_per_token": chain.launches,
           "e2e": {"value": round(1e3 / ms_e2e, 1), "unit": "tokens/s",
                   "ms_per_token": round(ms_e2e, 4), "h2d_bytes_per_step": 12,
                   "d2h_bytes_per_step": C5["n_vocab"] * 4},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(gbs / hbm, 4),
                        "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)"},
           "config": "16 layers, hidden 2048, 32/8 heads x 64, FFN 8192, vocab 128256, Q8_0 "
                     "N(0,0.02) seed 5, fp16 KV 4096 rows, batch 1; weights 1.31 GB > L2"}
    if _lib_err:
        res["device_error"] = _lib_err
    del chain, m
    return res


def bench_gemm(dev, steps, warmup):
    """The prefill chunk's projections (b2a_gemm, tcgen05) at the config-5 shapes for a
    2048-token chunk, each with the epilogue the chunk uses (QKV with RoPE and the K/V
    append, Wo and down with the residual added in place, gate/up with SwiGLU writing
    f16), timed by CUDA
    events; beside each, PyTorch's 16-bit GEMM with fp32 output (cuBLAS) on the same
    operands without the fused work.  Bound: tensor cores."""
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    T, E, F = 2048, C5["n_embd"], C5["n_ff"]
    qkv_n = (C5["n_head"] + 2 * C5["n_kv"]) * C5["head_dim"]
    g = torch.Generator(device=dev).manual_seed(7)
    shapes = (("qkv", qkv_n, E, "rope"), ("wo", E, E, "residual"),
              ("gate_up", 2 * F, E, "swiglu"), ("down", E, F, "residual"))
    n = max(3, min(steps, 20))

    def timed(fn):
        for _ in range(max(3, min(warmup, 5))):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n * 1e3  # us

    from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix
    hbm, bf16, bf16_sus, src = peaks()
    out, tot_fl, tot_us, tot_us8 = {}, 0.0, 0.0, 0.0
    for name, N, K, epi in shapes:
        a = torch.randn((T, K), device=dev, generator=g).to(torch.float16)
        w32 = 0.02 * torch.randn((N, K), device=dev, generator=g)
        w = w32.to(torch.float16)
        q8 = Q8Matrix.quantize(w32)  # the same matrix as Q8_0 codes + scales
        del w32
        if epi == "swiglu":
            o = torch.empty((T, N // 2), device=dev, dtype=torch.float16)
            fn = lambda: device.gemm(a, w, out=o, epilogue=device.GEMM_SWIGLU)
            fn8 = lambda: device.gemm_q8(a, q8, out=o, epilogue=device.GEMM_SWIGLU8)
        elif epi == "residual":
            o = torch.zeros((T, N), device=dev)
            fn = lambda: device.gemm(a, w, out=o, c_in=o)
            fn8 = lambda: device.gemm_q8(a, q8, out=o, c_in=o)
        elif epi == "rope":
            H, KV, D = C5["n_head"], C5["n_kv"], C5["head_dim"]
            cos, sin = device.rope_tables(T, D, 10000.0, device=dev)
            pos = torch.arange(T, dtype=torch.int32, device=dev)
            kc = torch.zeros((T, KV, D), device=dev, dtype=torch.float16)
            vc = torch.zeros_like(kc)
            o = torch.empty((T, H, D), device=dev, dtype=torch.float16)
            fn = lambda: device.gemm_qkv_rope(a, w, pos, cos, sin, H=H, KV=KV, k_cache=kc,
                                              v_cache=vc, q_out=o)
            fn8 = lambda: device.gemm_qkv_rope(a, q8, pos, cos, sin, H=H, KV=KV, k_cache=kc,
                                               v_cache=vc, q_out=o)
        else:
            o = torch.empty((T, N), device=dev)
            fn = lambda: device.gemm(a, w, out=o)
            fn8 = lambda: device.gemm_q8(a, q8, out=o)
        us = timed(fn)
        us8 = timed(fn8)
        ref = timed(lambda: torch.mm(a, w.t(), out_dtype=torch.float32))
        fl = 2.0 * T * N * K
        tot_fl += fl
        tot_us += us
        tot_us8 += us8
        out[name] = {"M": T, "N": N, "K": K, "epilogue": epi, "us": round(us, 1),
                     "tflops": round(fl / us / 1e6, 1), "frac": round(fl / us / 1e6 / bf16, 4),
                     "q8_us": round(us8, 1), "q8_tflops": round(fl / us8 / 1e6, 1),
                     "cublas_tflops_plain": round(fl / ref / 1e6, 1)}
        del a, w, o, q8
    tf = tot_fl / tot_us / 1e6
    tf8 = tot_fl / tot_us8 / 1e6
    return {"metric": "prefill-chunk GEMM TFLOPS (config-5 shapes, 2048 tokens)",
            "value": round(tf, 1), "unit": "TFLOP/s", "launches": 4 * n,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": bf16,
                         "unit": "TFLOP/s", "frac": round(tf / bf16, 4),
                         "peak_source": f"{src} (MEASURED_PEAKS.json bf16_tflops, burst)"},
            "q8_weights": {"value": round(tf8, 1), "unit": "TFLOP/s",
                           "frac": round(tf8 / bf16, 4),
                           "note": "b2a_gemm_q8: Q8_0 codes decoded to f16 inside the kernel"},
            "shapes": out}


def bench_prefill_chunk(dev, steps, warmup):
    """Device-resident prefill chunk (prefill_chain.ChunkPrefill) on the
    config-5 model: one 2048-token chunk at position 0 into an fp16 cache of
    4096 rows.  FLOPs per chunk: the GEMMs (2 * weights * tokens) plus the
    causal attention (4 * H * D * T(T+1)/2 per layer); bound: tensor cores."""
    import torch
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    from alpacca_open_sourced_by_jt_b200.prefill_chain import ChunkPrefill
    T, n_ctx = 2048, 4096
    m = LlamaQ8.random(**C5, seed=5, dev=dev)
    chain = DecodeChain(m, n_ctx, torch.float16)
    toks = [(7 * i + 3) % C5["n_vocab"] for i in range(T)]
    n = max(3, min(steps, 10))

    def time_chunk(pre):
        for _ in range(max(2, min(warmup, 3))):
            pre(toks, 0, want_logits=False)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            pre(toks, 0, want_logits=False)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    # the Q8_0 in-kernel path (no weight copy), for comparison, then the default
    # (a 16-bit weight copy)
    pre8 = ChunkPrefill(chain, max_chunk=T, weights="q8")
    ms8 = time_chunk(pre8)
    del pre8
    pre8d = ChunkPrefill(chain, max_chunk=T, weights="q8_dequant")
    ms8d = time_chunk(pre8d)
    del pre8d
    pre = ChunkPrefill(chain, max_chunk=T)
    ms = time_chunk(pre)
    E, H, KV, D, F, L = (C5["n_embd"], C5["n_head"], C5["n_kv"], C5["head_dim"], C5["n_ff"],
                         C5["n_layer"])
    w_layer = E * (H + 2 * KV) * D + H * D * E + 2 * F * E + F * E
    flops = L * (2.0 * w_layer * T + 4.0 * H * D * T * (T + 1) / 2)
    tf = flops / (ms * 1e-3) / 1e12
    _, bf16, _, src = peaks()
    del pre, chain, m
    return {"metric": "prefill chunk tokens/s (config-5 model, 2048-token chunk)",
            "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_chunk": round(ms, 3),
            "tflops": round(tf, 1), "steps": n, "weights": "f16 copy",
            "ms_per_chunk_q8_in_kernel": round(ms8, 3),
            "ms_per_chunk_q8_dequant_per_matrix": round(ms8d, 3),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": bf16,
                         "unit": "TFLOP/s", "frac": round(tf / bf16, 4),
                         "peak_source": f"{src} (MEASURED_PEAKS.json bf16_tflops, burst)"},
            "config": "16 layers, hidden 2048, 32/8 heads x 64, FFN 8192, vocab 128256; "
                      "weights dequantized to f16 (ms_per_chunk_q8_in_kernel: the GEMMs decoding "
                      "the Q8_0 codes instead); every kernel this library's: tcgen05 GEMMs "
                      "(RoPE + K/V append, residual add and SwiGLU in their epilogues), RMSNorm, "
                      "tcgen05 causal prefill; eager launches (7 per layer)"}


def bench_e2e(dev, st, steps, warmup, dist=None):
    """Decode step through the public API with host buffers (see module doc):
    DecodeStep replays the whole step (H2D of the pinned rows, fused
    RoPE+append, decode, D2H of the output) as one CUDA graph per token."""
    import numpy as np
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.decode_step import DecodeStep
    B, L, H, KV, D = WL["B"], WL["L"], WL["H"], WL["KV"], WL["D"]
    ct, stt = device.rope_tables(L, D, 500000.0, device=dev)
    rng = np.random.default_rng(7)
    step = DecodeStep(st["kc"], st["vc"], ct, stt, H)
    step.q.copy_(torch.from_numpy(rng.standard_normal((B, H, D), dtype=np.float32)))
    step.k.copy_(torch.from_numpy(rng.standard_normal((B, KV, D), dtype=np.float32)))
    step.v.copy_(torch.from_numpy(rng.standard_normal((B, KV, D), dtype=np.float32)))
    step.positions.fill_(L - 1)

    for _ in range(max(warmup, 3)):
        step()
    n = max(3, min(steps, 500))
    world = 1
    if dist is not None:
        world = dist.get_world_size()
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(n):
        out = step()
    dt = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    bytes_step = decode_bytes(B, L, KV, D) * world
    return dict(value=bytes_step / (dt / n) / 1e9, unit="GB/s", ranks_timed=world,
                h2d_bytes_per_step=world * int((B * H * D + 2 * B * KV * D) * 4 + 2 * B * 4),
                d2h_bytes_per_step=world * int(out.numel() * 4), steps=n,
                ms_per_step=dt / n * 1e3,
                path="DecodeStep: one CUDA graph per token (pinned q/k/v/positions H2D, "
                     "fused RoPE+append into the resident cache, split-KV decode, output "
                     "D2H), host waits for each step")


def bench_prefill(dev, steps, warmup, shape=None):
    import torch
    from alpacca_open_sourced_by_jt_b200 import device
    S, H, KV, D = shape or (PF["S"], PF["H"], PF["KV"], PF["D"])
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn((S, H, D), device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn((S, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn((S, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    pos = torch.arange(S, dtype=torch.int32, device=dev)
    out = torch.empty((S, H, D), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def call():
        device.prefill(q, k, v, pos, out=out)

    for _ in range(max(warmup, 3)):
        call()
    n = max(5, min(steps, 200))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    torch.cuda.synchronize()
    for a, b in evs:
        flush.zero_()
        a.record()
        call()
        b.record()
    torch.cuda.synchronize()
    times = [a.elapsed_time(b) for a, b in evs]
    ms = sum(times) / n
    fl = prefill_flops(S, H, D)
    return dict(ms=ms, tflops=fl / (ms * 1e-3) / 1e12, launches=n, q=q, k=k, v=v)


def cpu_decode_baseline(st, budget_s=10.0):
    import numpy as np
    import oracle
    L, H, KV, D = WL["L"], WL["H"], WL["KV"], WL["D"]
    K = st["kc"][0].float().cpu().numpy()
    V = st["vc"][0].float().cpu().numpy()
    q = st["q"][0].cpu().numpy()
    oracle.attention_decode(q, K, V, H // KV, 1 / math.sqrt(D))
    n, t0 = 0, time.perf_counter()
    while n < 3 or time.perf_counter() - t0 < budget_s:
        oracle.attention_decode(q, K, V, H // KV, 1 / math.sqrt(D))
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": decode_bytes(1, L, KV, D) / dt / 1e9, "unit": "GB/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 of the 16 sequences (32768 x 8 KV heads x 128, fp32 NumPy, the "
                      f"reference's _attention_np restated), {n} calls, {dt*1e3:.1f} ms each; "
                      f"GB/s counts the workload's bf16 KV bytes"}


def cpu_prefill_baseline(pf):
    import oracle
    S, H, KV, D = PF["S"], PF["H"], PF["KV"], PF["D"]
    g = H // KV
    q = pf["q"][:, :g].float().cpu().numpy()
    k = pf["k"][:, :1].float().cpu().numpy()
    v = pf["v"][:, :1].float().cpu().numpy()
    import numpy as np
    pos = np.arange(S, dtype=np.int32)
    t0 = time.perf_counter()
    oracle.attention_batch(q, k, v, pos, g, 1 / math.sqrt(D))
    dt = time.perf_counter() - t0
    return {"value": prefill_flops(S, g, D) / dt / 1e12, "unit": "TFLOP/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 of 8 KV heads (4 query heads) of config 2 through the reference's "
                      f"_attention_batch_np einsum path restated, {dt:.2f} s"}


def run_ours(args):
    import torch
    import torch.distributed as tdist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    from alpacca_open_sourced_by_jt_b200 import build as _b
    if rank == 0 and not _b.up_to_date():
        _b.build()
    dist = None
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from alpacca_open_sourced_by_jt_b200 import _lib
    _lib.load()
    _lib.device_error(clear=True)

    clocks = ClockSampler(gpu_id_for(local)) if rank == 0 else None
    if clocks:
        clocks.start()
    st = bench_decode(dev, rank, args.steps, args.warmup, dist)
    clk = clocks.stop() if clocks else None
    lc = None
    if args.only in (None, "longctx"):
        lc = bench_longctx(dev, rank, world, args.steps, args.warmup, dist)
    vl = None
    if args.only in (None, "varlen"):
        vl = bench_varlen(dev, rank, world, args.steps, args.warmup, dist)
    kvs = None
    if world == 1 and args.only in (None, "kvstate"):
        kvs = bench_kvstate(dev, args.steps, args.warmup)
    q35 = None
    if world == 1 and args.only in (None, "qwen35"):
        q35 = bench_qwen35(dev, args.steps, args.warmup)
    c5 = None
    if world == 1 and args.only in (None, "decode_step"):
        c5 = bench_decode_step(dev, args.steps, args.warmup)
    pch = None
    if world == 1 and args.only in (None, "prefill_chunk"):
        pch = bench_prefill_chunk(dev, args.steps, args.warmup)
    gmm = None
    if world == 1 and args.only in (None, "gemm"):
        gmm = bench_gemm(dev, args.steps, args.warmup)
    ms = st["ms"]
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=tdist.ReduceOp.MAX)
        ms = float(t.item())
    B, L, KV, D = WL["B"], WL["L"], WL["KV"], WL["D"]
    per_step = decode_bytes(B, L, KV, D)
    value = world * per_step * args.steps / (ms * 1e-3) / 1e9
    hbm, bf16, bf16_sus, src = peaks()
    achieved = per_step / (ms / args.steps * 1e-3) / 1e9   # per rank, per launch pair
    result = None
    e2e = None
    if args.only in (None, "e2e"):
        # every rank runs its own end-to-end loop at the same time; the
        # slowest rank's step time counts for all
        e2e = bench_e2e(dev, st, args.steps, args.warmup, dist)
    # config 2 head-sharded over the ranks (rank r: KV heads r*KV/N .. and their
    # q heads, the whole sequence; no collective), max over ranks of each
    # launch's CUDA-event time; every rank runs it, so it comes before the
    # rank-0 legs
    pf_sh = None
    if world > 1 and PF["KV"] % world == 0 and args.only in (None, "prefill") \
            and not args.no_prefill:
        sh = bench_prefill(dev, args.steps, args.warmup,
                           shape=(PF["S"], PF["H"] // world, PF["KV"] // world, PF["D"]))
        t = torch.tensor([sh["ms"]], device=dev)
        dist.all_reduce(t, op=tdist.ReduceOp.MAX)
        ms_sh = float(t.item())
        pf_sh = {"ms": ms_sh, "tflops": prefill_flops(PF["S"], PF["H"], PF["D"]) / (ms_sh * 1e-3)
                 / 1e12, "kv_heads_per_gpu": PF["KV"] // world, "q_heads_per_gpu": PF["H"] // world}
        del sh
        dist.barrier()
    if rank == 0:
        pf = pf256 = None
        if args.only in (None, "prefill") and not args.no_prefill:
            pf = bench_prefill(dev, args.steps, args.warmup)
            # head_dim 256 (the Qwen35 full-attention geometry: 16 q / 2 KV heads)
            pf256 = bench_prefill(dev, args.steps, args.warmup, shape=(PF["S"], 16, 2, 256))
        _lib.raise_device_error()
        cpu = cpu_decode_baseline(st) if (world == 1 and not args.no_cpu_baseline) else None
        traffic = profiled_traffic("decode_mma_kernel bf16 D128 NT1")
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "decode@32K: 16 seqs x 32768 ctx, 32 q / 8 KV heads, "
                                   "head_dim 128, bf16 KV ~N(0,1), 1 query token per seq",
                       "batch_per_gpu": B, "ctx": L, "q_heads": WL["H"], "kv_heads": KV,
                       "head_dim": D, "split_rows": st["split"],
                       "l2": "caches 2.15 GB per GPU > 126 MB L2; no flush",
                       "parallelism": f"sequence-sharded x{world} (no collective)"},
            "hbm_frac_of_spec": round(value / world / SPEC_HBM, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": traffic, "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "decode_mma_kernel<bf16,128,1> + decode_combine_kernel, "
                                   "timed together per b2a_decode call"},
            "gpu_launches": 2 * args.steps,
        }
        if e2e:
            result["e2e"] = e2e
        if lc:
            result["longctx"] = lc
        if kvs:
            result["kvstate"] = kvs
        if q35:
            result["qwen35_layer"] = q35
        if c5:
            result["decode_step"] = c5
        if pch:
            result["prefill_chunk"] = pch
        if gmm:
            result["gemm"] = gmm
        if vl:
            ach = vl["achieved_per_gpu_max"] if world > 1 else vl["value"]
            vl["roofline"] = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                              "frac": round(ach / hbm, 4),
                              "note": "rank 0's bytes over the max-over-ranks step time"}
            result["varlen"] = vl
        if cpu:
            result["cpu_baseline"] = cpu
        if clk:
            result["clocks"] = clk
        if pf:
            pcpu = cpu_prefill_baseline(pf) if (world == 1 and not args.no_cpu_baseline) else None
            result["prefill"] = {
                "metric": "prefill-attn TFLOPS", "value": round(pf["tflops"], 1),
                "unit": "TFLOP/s", "ms_per_launch": round(pf["ms"], 4),
                "config": "benchmark config 2: S=2048 causal, 32 q / 8 KV heads, D=128, bf16 "
                          "in/out, fp32 accumulation; L2 flushed before each launch",
                "roofline": {"bound": "tensor", "achieved": round(pf["tflops"], 1),
                             "peak": bf16, "unit": "TFLOP/s",
                             "frac": round(pf["tflops"] / bf16, 4),
                             "traffic": profiled_traffic("prefill_pair_kernel bf16 D128"),
                             "kernel": "prefill_pair_kernel<bf16,bf16,128> (default for even "
                                       "GQA groups)",
                             "peak_source": f"{src} (MEASURED_PEAKS.json bf16_tflops, burst)"},
                "launches": pf["launches"]}
            if pf256:
                result["prefill"]["head_dim_256"] = {
                    "value": round(pf256["tflops"], 1), "unit": "TFLOP/s",
                    "ms_per_launch": round(pf256["ms"], 4),
                    "config": f"S={PF['S']} causal, 16 q / 2 KV heads, D=256, bf16 in/out, "
                              "fp32 accumulation (Qwen35 full-attention layers); L2 flushed",
                    "kernel": "prefill_head_kernel<bf16,bf16,256> (64-key tiles)",
                    "roofline": {"bound": "tensor", "achieved": round(pf256["tflops"], 1),
                                 "peak": bf16, "unit": "TFLOP/s",
                                 "frac": round(pf256["tflops"] / bf16, 4)}}
            if pcpu:
                result["prefill"]["cpu_baseline"] = pcpu
            if pf_sh:
                result["prefill"]["head_sharded"] = {
                    "value": round(pf_sh["tflops"], 1), "unit": "TFLOP/s", "n_gpus": world,
                    "scaling": "strong", "ms_per_launch": round(pf_sh["ms"], 4),
                    "efficiency_vs_one_gpu_same_run": round(
                        pf_sh["tflops"] / (world * pf["tflops"]), 4),
                    "config": f"config 2 split by KV head: {pf_sh['kv_heads_per_gpu']} KV / "
                              f"{pf_sh['q_heads_per_gpu']} q heads per GPU, whole sequence, no "
                              "collective; time = max over ranks; FLOPs of the whole job"}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import oracle
    L, H, KV, D = WL["L"], WL["H"], WL["KV"], WL["D"]
    rng = np.random.default_rng(4)
    q = rng.standard_normal((H, D), dtype=np.float32)
    K = rng.standard_normal((L, KV, D), dtype=np.float32)
    V = rng.standard_normal((L, KV, D), dtype=np.float32)
    # calibrate: keep the whole W + K run near a minute of CPU time
    t0 = time.perf_counter()
    oracle.attention_decode(q, K, V, H // KV, 1 / math.sqrt(D))
    t_full = time.perf_counter() - t0
    per_step_budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(min(L, max(1024, L * per_step_budget / max(t_full, 1e-6))))
    Ks, Vs = np.ascontiguousarray(K[:rows]), np.ascontiguousarray(V[:rows])
    for _ in range(args.warmup):
        oracle.attention_decode(q, Ks, Vs, H // KV, 1 / math.sqrt(D))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.attention_decode(q, Ks, Vs, H // KV, 1 / math.sqrt(D))
    dt = (time.perf_counter() - t0) / args.steps
    value = decode_bytes(1, rows, KV, D) / dt / 1e9
    sample = (f"each step: one sequence's decode over {rows} of its 32768 cached rows "
              f"(32 q / 8 KV heads, D=128, fp32 NumPy, the reference's _attention_np "
              f"restated); GB/s counts the workload's bf16 KV bytes")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode@32K (per-sequence sample)", "ctx": L, "q_heads": H,
                   "kv_heads": KV, "head_dim": D, "rows_per_step": rows},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--only", choices=["decode", "e2e", "prefill", "longctx", "varlen",
                                       "kvstate", "qwen35", "decode_step",
                                       "prefill_chunk", "gemm"],
                    default=None,
                    help="profiling aid: run the decode timing plus only this extra part")
    ap.add_argument("--batch", type=int, default=WL["B"],
                    help="profiling aid: sequences per GPU (default 16)")
    ap.add_argument("--ctx", type=int, default=WL["L"],
                    help="profiling aid: cached tokens per sequence (default 32768)")
    args = ap.parse_args()
    WL["B"], WL["L"] = args.batch, args.ctx
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
