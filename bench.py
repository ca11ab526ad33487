"""Benchmark of vk-compute's decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload (N=1 headline): RmsNorm-GEMV INT8 -- x 4096 ~N(0,1), gamma
~1+N(0,0.1), eps 1e-6, W 12288x4096 ~N(0,0.02) symmetric int8 with fp16-valued
scales in the reference storage (per (k, 256-output block) fp32 scale/zero,
16-byte chunk packing).  A step is one fused RmsNorm-GEMV over one weight
matrix; steps rotate through a pool of weight copies larger than 4x L2 so
every step streams its weights from HBM.  Steps are captured in a CUDA
graph (one launch per step).

Metric: achieved HBM GB/s = algorithmic bytes (weights, scales and zeros
once, activations in and out once) / device time per step.  With
torchrun (N>1) every rank holds its own row shard of a 12288N x 4096
matrix (weak scaling, no collective on the data path) and `value` is the
total over ranks, timed as the max over ranks.

The line also carries `decode_step`: one token through the 36-layer int4
decoder chain (QKV+RoPE+KV append, GQA attention over 8192 cached tokens, O,
RmsNorm-SwiGLU, down), sharded over the N GPUs by heads and by the O / down
projections' inputs with two NVLink exchanges per layer fused into the
kernels, as device us per step (max over ranks) -- the decode-step latency at
1/2/4/8 GPUs.

--impl reference times the reference's CPU algorithm (the oracle's C port of
src/compute.c's loops over the src/data.c storage, all host threads) on the
same workload.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
E2E_BIN = ROOT / "vk_compute_b200" / "vkc_e2e_bench"
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "rmsnorm_gemv_int8": "RmsNorm-GEMV INT8 12288x4096 (x 4096, eps 1e-6, symmetric int8, fp16-valued scales)",
    "gemv_fp16": "GEMV FP16 4096x4096 (x 4096)",
    "swiglu_ffn_int4": "RmsNorm-swiglu-ffn INT4 gate/up 12288x4096 + down GEMV INT4 4096x12288",
    "qkv_rope_attn_int4": "RmsNorm-GEMV-Rope INT4 QKV 6144x4096 (theta 1e6) + Att-full-FP16 32q/8kv x 128, ctx 8192",
    "prefill_gemm_bf16": "prefill GEMM bf16 on tcgen05: A 64x4096 . W^T (W 12288x4096, K-major) -> C 64x12288 fp32",
    "rmsnorm_gemv_int8_batch4": "batched decode: RmsNorm-GEMV INT8 12288x4096 on 4 vectors (weights streamed once)",
    "gemv_int4_batch8": "batched decode: GEMV INT4 4096x12288 (down projection) on 8 vectors (weights streamed once)",
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text()).get("bf16_tflops", 1590.0))
    return 1590.0


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/ncu_traffic.json), or None."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    v = d.get(workload)
    return None if v is None else v.get("bytes_per_launch")


def ncu_traffic_table() -> dict:
    """Per-launch DRAM bytes by kernel name (the `kernels` section of
    profiles/ncu_traffic.json, keyed like the bench's kernel names)."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return {}
    return {k: v.get("bytes_per_launch") for k, v in json.loads(p.read_text()).get("kernels", {}).items()}


class ClockSampler:
    """nvidia-smi clock / throttle sampling in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"vkc_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]), "power": float(parts[3]),
                             "hw": parts[5], "hw_thermal": parts[6], "sw_thermal": parts[7], "power_cap": parts[8]})
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("power_cap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        loaded = [r for r in rows if r["power"] > 200.0] or rows
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max(r["power"] for r in rows)}


# ---------------------------------------------------------------------------
# Workloads (our implementation)
# ---------------------------------------------------------------------------

def build_workload(name: str, rank: int, device, world: int = 1):
    """Returns a dict: step(i) enqueues step i on the current stream; bytes
    (algorithmic bytes of one rank's step), job_bytes (of the whole job's
    step), launches, the dominant kernel (fn, bytes, name), kernels (name, fn,
    bytes) for per-kernel timing, e2e inputs and meta.  With world > 1 the
    headline workload is one fixed matrix row-sharded over the ranks plus an
    NVLink all-gather of y; the others run one copy per rank."""
    import torch

    from vk_compute_b200 import ops

    gen = torch.Generator(device="cpu").manual_seed(1000 + rank)

    def randn(*shape, std=1.0, mean=0.0):
        return (torch.randn(*shape, generator=gen) * std + mean).to(device)

    def pool_of(make, nbytes):
        n = max(2, min(64, math.ceil(4 * L2_BYTES / nbytes)))
        base = [make(j) for j in range(min(n, 4))]
        return [base[j % len(base)] if j < len(base) else clone(base[j % len(base)]) for j in range(n)]

    def clone(w):
        return ops.PackedWeight(w.bits, w.K, w.N, w.packed.clone(),
                                None if w.scale is None else w.scale.clone(),
                                None if w.zero is None else w.zero.clone())

    if name == "rmsnorm_gemv_int8" and world > 1:
        # The 12288 x 4096 matrix row-sharded: rank r owns outputs
        # [r*N/world, (r+1)*N/world) (whole 256-row scale blocks); its
        # RmsNorm-GEMV stores them straight into every rank's copy of y over
        # NVLink and a wait kernel returns once every rank's part has arrived
        # (strong scaling: the job is fixed).
        from vk_compute_b200.p2p import PeerGather

        K, N, bits = 4096, 12288, 8
        n_loc = N // world
        x = randn(K)
        gamma = randn(K, std=0.1, mean=1.0)
        y_loc = torch.empty(n_loc, device=device)
        peer = PeerGather({"y": N}, device)
        wg = torch.Generator(device=device).manual_seed(77)
        full = torch.randn(K, N, generator=wg, device=device) * 0.02
        shard = full[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
        del full
        wbytes = K * n_loc + 8 * K * n_loc // 256
        pool = pool_of(lambda j: ops.pack_dense(shard, bits, symmetric=True, fp16_scale=True), wbytes)
        del shard

        def step(i):
            peer.rmsnorm_gemv_gather("y", pool[i % len(pool)], x, gamma, eps=1e-6)

        gemv = lambda i: ops.rmsnorm_gemv(pool[i % len(pool)], x, gamma, eps=1e-6, out=y_loc)
        job = K * N + 8 * K * N // 256 + 4 * K * 2 + 4 * N
        rank_bytes = wbytes + 4 * K * 2 + 4 * n_loc
        meta = {"K": K, "N": N, "bits": bits, "rows_per_rank": n_loc, "pool": len(pool),
                "pool_bytes": len(pool) * wbytes,
                "exchange": "all-gather of y fused into the GEMV epilogue (NVLink peer stores) + one wait kernel"}
        return dict(step=step, bytes=rank_bytes, job_bytes=job, scaling="strong", launches=2, dominant=gemv,
                    dominant_bytes=rank_bytes, dominant_name=f"RmsNorm-GEMV-INT8 {n_loc}x{K} shard", meta=meta,
                    e2e=None, e2e_sharded=(x, peer.buffers["y"], K, N), kernels=[], close=peer.close)

    if name in ("rmsnorm_gemv_int8", "gemv_fp16"):
        if name == "rmsnorm_gemv_int8":
            K, N, bits = 4096, 12288, 8
        else:
            K, N, bits = 4096, 4096, 16
        x = randn(K)
        gamma = randn(K, std=0.1, mean=1.0)
        y = torch.empty(N, device=device)
        wbytes = K * N * bits // 8 + (2 * 4 * K * N // 256 if bits <= 8 else 0)
        pool = pool_of(lambda j: ops.pack_dense(randn(K, N, std=0.02), bits, symmetric=True, fp16_scale=True),
                       wbytes)
        if name == "rmsnorm_gemv_int8":
            act = 4 * K * 2 + 4 * N  # x, gamma in; y out
            step = lambda i: ops.rmsnorm_gemv(pool[i % len(pool)], x, gamma, eps=1e-6, out=y)
        else:
            act = 4 * K + 4 * N
            step = lambda i: ops.gemv(pool[i % len(pool)], x, out=y)
        meta = {"K": K, "N": N, "bits": bits, "pool": len(pool), "pool_bytes": len(pool) * wbytes}
        kname = "RmsNorm-GEMV-INT8" if bits == 8 else "GEMV-FP16"
        return dict(step=step, bytes=wbytes + act, launches=1, dominant=step, dominant_bytes=wbytes + act,
                    dominant_name=kname, meta=meta, e2e=(pool, x, gamma, y, K, N, bits),
                    kernels=[(kname, step, wbytes + act)])

    if name in ("rmsnorm_gemv_int8_batch4", "gemv_int4_batch8"):
        if name == "rmsnorm_gemv_int8_batch4":
            K, N, bits, M = 4096, 12288, 8, 4
        else:
            K, N, bits, M = 12288, 4096, 4, 8
        x = randn(M, K)
        gamma = randn(K, std=0.1, mean=1.0)
        y = torch.empty(M, N, device=device)
        wbytes = K * N * bits // 8 + 2 * 4 * K * N // 256
        pool = pool_of(lambda j: ops.pack_dense(randn(K, N, std=0.02), bits, symmetric=True, fp16_scale=True),
                       wbytes)
        if bits == 8:
            act = 4 * M * K + 4 * K + 4 * M * N
            step = lambda i: ops.rmsnorm_gemv_batched(pool[i % len(pool)], x, gamma, eps=1e-6, out=y)
        else:
            act = 4 * M * K + 4 * M * N
            step = lambda i: ops.gemv_batched(pool[i % len(pool)], x, out=y)
        meta = {"K": K, "N": N, "bits": bits, "vectors": M, "pool": len(pool), "pool_bytes": len(pool) * wbytes}
        kname = f"batched GEMV INT{bits} x{M}"
        return dict(step=step, bytes=wbytes + act, launches=1, dominant=step, dominant_bytes=wbytes + act,
                    dominant_name=kname, meta=meta, e2e=None, kernels=[(kname, step, wbytes + act)])

    if name == "swiglu_ffn_int4":
        H, I = 4096, 12288
        x = randn(H)
        gamma = randn(H, std=0.1, mean=1.0)
        h = torch.empty(I, device=device)
        out = torch.empty(H, device=device)
        gu_bytes = 2 * (H * I // 2 + 2 * 4 * H * I // 256)
        d_bytes = I * H // 2 + 2 * 4 * I * H // 256
        layer_bytes = gu_bytes + d_bytes
        n = max(2, min(32, math.ceil(4 * L2_BYTES / layer_bytes)))
        layers = []
        for j in range(n):
            if j < 2:
                layers.append((ops.pack_dense(randn(H, I, std=0.02), 4), ops.pack_dense(randn(H, I, std=0.02), 4),
                               ops.pack_dense(randn(I, H, std=0.02), 4)))
            else:
                layers.append(tuple(clone(w) for w in layers[j % 2]))

        def step(i):
            g, u, d = layers[i % n]
            ops.rmsnorm_swiglu(g, u, x, gamma, eps=1e-6, out=h)
            ops.gemv(d, h, out=out)

        dom = lambda i: ops.rmsnorm_swiglu(*layers[i % n][:2], x, gamma, eps=1e-6, out=h)
        down = lambda i: ops.gemv(layers[i % n][2], h, out=out)
        act = 4 * H * 2 + 4 * I + 4 * I + 4 * H
        return dict(step=step, bytes=layer_bytes + act, launches=2, dominant=dom,
                    dominant_bytes=gu_bytes + 4 * H * 2 + 4 * I, dominant_name="RmsNorm-swiglu-ffn-INT4",
                    meta={"hidden": H, "intermediate": I, "pool": n}, e2e=None,
                    kernels=[("RmsNorm-swiglu-ffn-INT4 gate/up 2x12288x4096", dom, gu_bytes + 4 * H * 2 + 4 * I),
                             ("GEMV-INT4 down 4096x12288", down, d_bytes + 4 * I + 4 * H)])

    if name == "qkv_rope_attn_int4":
        H, NQ, NKV, HD, CTX = 4096, 32, 8, 128, 8192
        NQKV = (NQ + 2 * NKV) * HD
        x = randn(H)
        gamma = randn(H, std=0.1, mean=1.0)
        theta = (1e6 ** (-torch.arange(HD // 2, dtype=torch.float64) * 2 / HD)).float().to(device)
        qkv = torch.empty(NQKV, device=device)
        att = torch.empty(NQ * HD, device=device)
        wbytes = H * NQKV // 2 + 2 * 4 * H * NQKV // 256
        kvbytes = 2 * CTX * NKV * HD * 2
        n = max(2, min(32, math.ceil(4 * L2_BYTES / (wbytes + kvbytes))))
        layers = []
        for j in range(n):
            if j < 2:
                w = ops.pack_dense(randn(H, NQKV, std=0.02), 4)
                kc = randn(CTX, NKV, HD).half()
                vc = randn(NKV, HD // 8, CTX, 8).half()
                layers.append((w, kc, vc))
            else:
                w, kc, vc = layers[j % 2]
                layers.append((clone(w), kc.clone(), vc.clone()))
        ws = ops.attention_workspace(NQ, NKV, HD, CTX, device=device)
        pos = int(torch.randint(0, 8192, (1,), generator=gen))

        def step(i):
            w, kc, vc = layers[i % n]
            ops.rmsnorm_gemv_rope(w, x, gamma, theta, pos, mode="pairs", head_dim=HD, rot_rows=(NQ + NKV) * HD,
                                  eps=1e-6, out=qkv)
            ops.attention_decode(qkv[:NQ * HD], kc, vc, NQ, NKV, HD, CTX, 1 / math.sqrt(HD), workspace=ws, out=att)

        dom = lambda i: ops.attention_decode(qkv[:NQ * HD], layers[i % n][1], layers[i % n][2], NQ, NKV, HD, CTX,
                                             1 / math.sqrt(HD), workspace=ws, out=att)
        qkv_fn = lambda i: ops.rmsnorm_gemv_rope(layers[i % n][0], x, gamma, theta, pos, mode="pairs", head_dim=HD,
                                                 rot_rows=(NQ + NKV) * HD, eps=1e-6, out=qkv)
        act = 4 * H * 2 + 4 * NQKV + 4 * NQ * HD * 2
        return dict(step=step, bytes=wbytes + kvbytes + act, launches=2, dominant=dom,
                    dominant_bytes=kvbytes + 4 * NQ * HD * 2, dominant_name="Att-full-FP16",
                    meta={"pool": n, "pos": pos, "ctx": CTX}, e2e=None,
                    kernels=[("RmsNorm-GEMV-Rope-INT4 QKV 6144x4096", qkv_fn, wbytes + 4 * H * 2 + 4 * NQKV),
                             ("Att-full-FP16 32q/8kv x 128, ctx 8192", dom, kvbytes + 4 * NQ * HD * 2)])
    if name == "prefill_gemm_bf16":
        M, N, K = 64, 12288, 4096
        a = randn(M, K).to(torch.bfloat16)
        c = torch.empty(M, N, device=device)
        wbytes = N * K * 2
        n = max(2, min(16, math.ceil(4 * L2_BYTES / wbytes)))
        base = [randn(N, K, std=0.02).to(torch.bfloat16) for _ in range(2)]
        ws = [base[j] if j < 2 else base[j % 2].clone() for j in range(n)]
        step = lambda i: ops.gemm_bf16(a, ws[i % n], out=c)
        nbytes = wbytes + M * K * 2 + M * N * 4
        kname = "gemm_tc_kernel (tcgen05, bf16)"
        return dict(step=step, bytes=nbytes, launches=1, dominant=step, dominant_bytes=nbytes,
                    dominant_name=kname, meta={"M": M, "N": N, "K": K, "pool": n, "flop": 2 * M * N * K},
                    e2e=None, kernels=[(kname, step, nbytes)])
    raise SystemExit(f"unknown workload {name}; choose from {sorted(WORKLOADS)}")


def capture(fn, count, start=0):
    import torch

    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(start)  # one eager call on the capture stream before capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for i in range(count):
            fn(start + i)
    return g


def time_launches(fn, steps: int, start: int = 0) -> float:
    """Device seconds per call of fn(start), ..., fn(start + steps - 1),
    captured in one CUDA graph that is replayed once untimed (upload and
    warm-up: `steps` calls) and then timed with CUDA events on the stream."""
    import torch

    g = capture(fn, steps, start)
    stream = torch.cuda.current_stream()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / 1e3 / steps


# The other configurations of the headline metric, measured in the default run
# beside the headline (RmsNorm-GEMV INT8 is config 2): key -> workload.
CONFIG_WORKLOADS = {"1": "gemv_fp16", "3": "swiglu_ffn_int4", "4": "qkv_rope_attn_int4", "5b": "prefill_gemm_bf16"}


def measure_configs(rank: int, device, steps: int, peak: float, device_index: int) -> dict:
    """Each config's step and each of its kernels alone, graph-launched back
    to back over the same >= 4x L2 weight pools as the workload itself."""
    import torch

    traffic = ncu_traffic_table()
    sampler = ClockSampler(device_index)
    sampler.start()
    out = {}
    for key, name in CONFIG_WORKLOADS.items():
        wl = build_workload(name, rank, device)
        torch.cuda.synchronize()
        step_s = time_launches(wl["step"], steps)
        kernels = {}
        for kname, fn, nbytes in wl["kernels"]:
            ks = step_s if len(wl["kernels"]) == 1 else time_launches(fn, steps)
            entry = {"us": round(ks * 1e6, 3), "GB_s": round(nbytes / ks / 1e9, 1),
                     "frac": round(nbytes / ks / 1e9 / peak, 4), "algorithmic_bytes": nbytes,
                     "traffic": traffic.get(kname)}
            if "flop" in wl["meta"]:
                entry["tflops"] = round(wl["meta"]["flop"] / ks / 1e12, 1)
                entry["tensor_frac"] = round(wl["meta"]["flop"] / ks / 1e12 / tensor_peak(), 4)
            kernels[kname] = entry
        out[key] = {"workload": name, "description": WORKLOADS[name], "us_per_step": round(step_s * 1e6, 3),
                    "GB_s": round(wl["bytes"] / step_s / 1e9, 1), "frac": round(wl["bytes"] / step_s / 1e9 / peak, 4),
                    "bytes_per_step": wl["bytes"], "launches_per_step": wl["launches"], "kernels": kernels}
        del wl
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    out["clocks"] = sampler.stop()
    out["method"] = ("graph-launched back to back, steps rotate through weight pools >= 4x L2; a kernel's us is "
                     "its own graph of the same launches; frac of the measured HBM copy peak")
    return out


def e2e_dropin(args, e2e, device_index):
    """Same metric through the reference-facing C ABI with host buffers:
    per step writeBuffer(x) from pinned host memory, execute() of the
    operator by its shader name, readBuffer(y)."""
    import ctypes as C

    import numpy as np
    import torch

    from vk_compute_b200 import dropin as D

    pool, x, gamma, y, K, N, bits = e2e
    os.environ["VKC_DEVICE"] = str(device_index)
    s = D.create_session()
    L = D.abi()

    def dev_buffer(t: torch.Tensor):
        h = t.cpu().numpy()
        return D.create_buffer(s, h)

    bufs = [(dev_buffer(w.packed), dev_buffer(w.scale) if bits <= 8 else None,
             dev_buffer(w.zero) if bits <= 8 else None) for w in pool]
    x_host = torch.empty(K, dtype=torch.float32).pin_memory()
    x_host.copy_(x.cpu())
    y_host = torch.empty(N, dtype=torch.float32).pin_memory()
    xb = D.create_buffer(s, x_host.numpy())
    gb = D.create_buffer(s, gamma.cpu().numpy())
    yb = D.create_buffer(s, None, 4 * N)
    name = "RmsNorm-GEMV-INT8.spv" if bits == 8 else "GEMV-FP16.spv"
    ops_ = []
    for wb, sb, zb in bufs:
        if bits == 8:
            ops_.append(D.operation(name, [xb, gb, wb, yb, sb, zb], [1, N, K]))
        else:
            ops_.append(D.operation(name, [xb, wb, yb], [1, N, K]))
    arrs = [(D.Operation * 1)(op) for op in ops_]
    xp = C.c_void_p(x_host.data_ptr())
    yp = C.c_void_p(y_host.data_ptr())

    def one(i):
        L.writeBuffer(s.dev.device, s.dev.queue, xb, xp)
        L.execute(s, arrs[i % len(arrs)], 1)
        L.readBuffer(s.dev.device, s.dev.physicalDevice, s.dev.queue, yb, yp)

    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(i)
    dt = (time.perf_counter() - t0) / args.steps
    for trio in bufs:
        for b in trio:
            if b is not None:
                D.destroy_buffer(s, b)
    for b in (xb, gb, yb):
        D.destroy_buffer(s, b)
    D.destroy_session(s)
    return dt, 4 * K, 4 * N


def e2e_sharded(args, wl):
    """The sharded headline end to end through the Python API on every rank:
    per step, x host->device from pinned memory, the rank's RmsNorm-GEMV
    shard and the NVLink all-gather, then the whole y device->host; host wall
    clock.  Every rank makes the same launches (the gather is collective)."""
    import torch

    x_dev, y_full, K, N = wl["e2e_sharded"]
    x_host = torch.empty(K, dtype=torch.float32).pin_memory()
    x_host.copy_(x_dev.cpu())
    y_host = torch.empty(N, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream()
    step = wl["step"]

    def one(i):
        x_dev.copy_(x_host, non_blocking=True)
        step(i)
        y_host.copy_(y_full, non_blocking=True)
        stream.synchronize()

    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(args.warmup + i)
    dt = (time.perf_counter() - t0) / args.steps
    return dt, 4 * K, 4 * N


def decode_parity(dec, cfg, rank: int, world: int, device, pos: int) -> dict | None:
    """One eager step of the sharded model from a seeded x, and (on rank 0)
    the same step of the same model on one GPU; returns rank 0's
    norm-relative difference.  The shards are whole scale blocks of the
    unsharded matrices, so the two are the same quantised model and differ
    only in the order of the cross-rank sums."""
    import torch

    from vk_compute_b200.decode import ShardedDecoder

    g = torch.Generator(device=device).manual_seed(4242)
    x0 = torch.randn(cfg.hidden, generator=g, device=device)
    dec.buf.x.copy_(x0)
    got = dec.step(pos).clone()
    torch.cuda.synchronize()
    timed_out = dec.timed_out()
    if rank != 0:
        return None
    ref_dec = ShardedDecoder(cfg, rank=0, world=1, device=device, seed=7)
    ref_dec.buf.x.copy_(x0)
    ref = ref_dec.step(pos).clone()
    torch.cuda.synchronize()
    err = float((got - ref).abs().max() / ref.abs().max())
    del ref_dec
    torch.cuda.empty_cache()
    return {"max_rel_err": err, "bar": 5e-3, "ok": bool(err <= 5e-3 and not timed_out),
            "peer_wait_timed_out": timed_out,
            "against": "the same 36-layer int4 model (same seeds, same quantisation) on one GPU, one eager step "
                       "from the same x at the same position"}


def decode_step_bench(rank: int, world: int, device, steps: int, warmup: int, peak: float, parity: bool = True,
                      shape: str = "full", emulate_world: int = 1, exchange: str = "p2p"):
    """The 36-layer decoder chain (hidden 4096, 32 query / 8 KV heads of 128,
    intermediate 12288, int4 weights ~N(0,0.02), random-init) for one token at
    position 8191 (attention over a full 8192-token fp16 cache), sharded over
    `world` GPUs by heads (QKV, attention), input rows (O, down) and output
    rows (gate/up) with two all-reduces per layer (the library's NVLink peer
    all-reduce).  `shape` is the decoder's kernel shape (ShardedDecoder).
    emulate_world > 1 (on one GPU) runs rank 0's shard of that many ranks
    with no exchange: the compute share of a sharded step, without its
    communication.  Steps are graph launches; time is the max over ranks."""
    import torch
    import torch.distributed as dist

    from vk_compute_b200.decode import DecoderConfig, ShardedDecoder

    cfg = DecoderConfig()
    t0 = time.perf_counter()
    if emulate_world > 1 and world == 1:
        dec = ShardedDecoder(cfg, rank=0, world=emulate_world, device=device, seed=7, shape=shape, exchange="none")
    else:
        emulate_world = 1
        dec = ShardedDecoder(cfg, rank=rank, world=world, device=device, seed=7, shape=shape, exchange=exchange)
    pos = cfg.ctx - 1
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    check = decode_parity(dec, cfg, rank, world, device, pos) if (parity and world > 1) else None
    if world > 1:
        dist.barrier()
    dec.buf.x.normal_()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dec.step(pos)  # eager step: NCCL communicators and kernel attributes set up before capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dec.step(pos)
    for _ in range(warmup):
        g.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    e0.record(stream)
    for _ in range(steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=device)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item()) * 1e3
    rank_bytes = dec.step_bytes(pos)
    del g  # release the graph (and any collective work in it) before the process group goes
    torch.cuda.synchronize()
    kernels = dec.kernels_per_step()
    exchange = dec.exchange
    dec.close()
    extra = {"emulated_shard_of": emulate_world, "note": "rank 0's kernels only, no exchange"} if emulate_world > 1 else {}
    return {**extra, "layers": cfg.layers, "shape": shape, "us_per_step": round(us, 2), "tokens_per_s": round(1e6 / us, 1),
            "bytes_per_step": rank_bytes * world, "GB_s": round(rank_bytes * world / us / 1e3, 1),
            "frac_of_peak_per_gpu": round(rank_bytes / us / 1e3 / peak, 4),
            "kernels_per_step": kernels, "all_reduces_per_step": 2 * cfg.layers if world > 1 else 0,
            "steps": steps, "warmup": warmup, "pos": pos, "ctx": cfg.ctx,
            "parallelism": (f"head/K-split shards x{world}, all-reduce x2 per layer ({exchange}: "
                            + {"p2p": "NVLink peer stores fused into the projections",
                               "p2p-kernel": "NVLink peer all-reduce kernel",
                               "nccl": "NCCL all-reduce"}.get(exchange, exchange) + ")") if world > 1 else "1 GPU",
            "build_s": round(build_s, 1),
            "parity": check,
            "model": "36 x (RmsNorm-GEMV-Rope QKV 6144x4096 + KV append, Att-full GQA 32/8 x 128, "
                     "O 4096x4096 + residual, RmsNorm-swiglu 2x12288x4096, down 4096x12288 + residual), int4"}


def cpu_baseline(workload: str, budget_s: float = 12.0, threads: int | None = None):
    """The reference's CPU algorithm (oracle port of src/compute.c:216-290
    over the src/data.c storage) on a bounded sample of the workload."""
    import numpy as np

    from oracle import pyoracle as o

    threads = threads or len(os.sched_getaffinity(0))
    o.set_threads(threads)
    rng = np.random.default_rng(0)
    if workload == "prefill_gemm_bf16":
        # gemm.comp's arithmetic (the oracle's restatement) on a column slice
        M, K, Ns = 64, 4096, 1536
        a = rng.standard_normal((M, K), dtype=np.float32)
        b = rng.standard_normal((K, Ns), dtype=np.float32) * 0.02
        reps, t0 = 0, time.perf_counter()
        while True:
            o.gemm(a, b)
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s or reps >= 200:
                break
        per = el / reps
        nbytes = K * Ns * 2 + M * K * 2 + M * Ns * 4
        return {"value": round(nbytes / per / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{reps} passes of 64x4096 . 4096x{Ns} (1/8 of the columns) in {el:.1f} s",
                "s_per_pass": per}
    vectors = 1
    if workload == "rmsnorm_gemv_int8":
        K, N, bits = 4096, 12288, 8
    elif workload == "gemv_fp16":
        K, N, bits = 4096, 4096, 16
    elif workload == "swiglu_ffn_int4":
        K, N, bits = 4096, 12288, 4
    elif workload == "rmsnorm_gemv_int8_batch4":
        K, N, bits, vectors = 4096, 12288, 8, 4
    elif workload == "gemv_int4_batch8":
        K, N, bits, vectors = 12288, 4096, 4, 8
    else:
        K, N, bits = 4096, 6144, 4
    w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02)
    x = rng.standard_normal(K, dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    if bits == 16:
        data, s, z = w.astype(np.float16).view(np.uint16), None, None
        nbytes = K * N * 2 + 8 * K
    else:
        data, s, z = o.quantize(w, bits, True, True)
        nbytes = K * N * bits // 8 + 8 * K * N // 256 + 8 * K + 4 * N
    gamma = None if workload in ("gemv_fp16", "gemv_int4_batch8") else g
    reps, t0 = 0, time.perf_counter()
    while True:
        if workload == "swiglu_ffn_int4":
            o.qswiglu(x, g, (data, s, z), (data, s, z), bits, K, N, K, 1e-6)
        else:
            o.qgemv(x, gamma, data, s, z, bits, K, N, K, 1e-6)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    per = el / reps
    mult = 2 if workload == "swiglu_ffn_int4" else 1
    if vectors > 1:
        # the reference computes one vector per pass: a batch of M is M passes
        # over the same bytes the batched kernel reads once
        per *= vectors
        nbytes = K * N * bits // 8 + 8 * K * N // 256 + vectors * 4 * (K + N)
    return {"value": round(mult * nbytes / per / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full passes of {bits}-bit {K}x{N}{' gate+up' if mult == 2 else ''} in {el:.1f} s"
                      + (f", one vector per pass, {vectors} passes per step" if vectors > 1 else ""),
            "s_per_pass": per}


def run_reference(args, rank, world):
    """The reference arm: W untimed then K timed passes of the reference's
    CPU algorithm over the whole workload, all host threads."""
    if rank != 0:
        return
    import numpy as np

    from oracle import pyoracle as o

    wl = args.workload
    threads = len(os.sched_getaffinity(0))
    o.set_threads(threads)
    if wl == "prefill_gemm_bf16":
        r = cpu_baseline(wl, budget_s=max(1.0, 0.5 * args.steps), threads=threads)
        line = {"impl": "reference", "metric": f"{WORKLOADS[wl]} achieved HBM GB/s", "value": r["value"],
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(r["s_per_pass"] * 8e3, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": wl, "description": WORKLOADS[wl]},
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    K, N, bits = {"rmsnorm_gemv_int8": (4096, 12288, 8), "gemv_fp16": (4096, 4096, 16),
                  "swiglu_ffn_int4": (4096, 12288, 4), "qkv_rope_attn_int4": (4096, 6144, 4)}[wl]
    rng = np.random.default_rng(0)
    w = rng.standard_normal((K, N), dtype=np.float32) * 0.02
    x = rng.standard_normal(K, dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    if bits == 16:
        data, s, z = w.astype(np.float16).view(np.uint16), None, None
        nbytes = K * N * 2 + 4 * K + 4 * N
    else:
        data, s, z = o.quantize(w, bits, True, True)
        nbytes = K * N * bits // 8 + 8 * K * N // 256 + 8 * K + 4 * N
    gamma = None if wl == "gemv_fp16" else g

    def one():
        if wl == "swiglu_ffn_int4":
            o.qswiglu(x, g, (data, s, z), (data, s, z), bits, K, N, K, 1e-6)
        else:
            o.qgemv(x, gamma, data, s, z, bits, K, N, K, 1e-6)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    per = (time.perf_counter() - t0) / args.steps
    if wl == "swiglu_ffn_int4":
        nbytes = 2 * nbytes
    value = round(nbytes / per / 1e9, 4)
    sample = f"{args.steps} full passes of the {bits}-bit {K}x{N} operator ({nbytes} B each)"
    line = {"impl": "reference", "metric": f"{WORKLOADS[wl]} achieved HBM GB/s", "value": value,
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl, "description": WORKLOADS[wl]},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="rmsnorm_gemv_int8", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true", help="launch steps eagerly instead of from a CUDA graph")
    ap.add_argument("--no-pdl", action="store_true", help="plain launches (no programmatic dependent launch)")
    ap.add_argument("--gemv-plan", default="auto", choices=["auto", "cluster", "per-sm", "per-sm-half", "auto-full"],
                    help="single-vector GEMV kernel: chosen per shape, cluster split-K, or one CTA per SM")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemv-fma", action="store_true",
                    help="8/4-bit weights on the per-SM GEMV with fp32 FMAs instead of integer dot products")
    ap.add_argument("--attention-plan", default="auto", choices=["auto", "clustered", "per-sm", "per-sm-half", "per-sm-x2", "per-sm-wide"],
                    help="decode attention: chosen per shape, clusters of 8 CTAs per KV head, or one CTA per SM")
    ap.add_argument("--no-decode", action="store_true", help="skip the 36-layer decode-step measurement")
    ap.add_argument("--no-decode-parity", action="store_true",
                    help="skip the N>1 decode-step check against the same model on one GPU")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config measurements beside the headline (N=1)")
    ap.add_argument("--decode-steps", type=int, default=20)
    ap.add_argument("--decode-exchange", default="p2p", choices=["p2p", "p2p-kernel", "nccl"],
                    help="how the sharded decode step sums the K-split projections across ranks")
    ap.add_argument("--decode-emulate-shard", type=int, default=1,
                    help="on one GPU: time rank 0's share of an N-way sharded decode step, without exchanges")
    ap.add_argument("--decode-shape", default="full", choices=["full", "half", "mixed", "persistent"],
                    help="kernel shapes of the decode step (see ShardedDecoder)")
    ap.add_argument("--clock-window", type=float, default=1.5, help="seconds of sampled load before timing")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from vk_compute_b200 import ops

    ops.set_pdl(not args.no_pdl)
    ops.set_gemv_plan(args.gemv_plan)
    ops.set_gemv_int_dot(not args.gemv_fma)
    ops.set_attention_plan(args.attention_plan)
    wl = build_workload(args.workload, rank, device, world)
    step = wl["step"]
    scaling = wl.get("scaling", "weak")
    job_bytes = wl.get("job_bytes", world * wl["bytes"])
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    gw = gt = None
    if args.no_graph:
        warm = lambda: [step(i) for i in range(args.warmup)]
        timed = lambda: [step(args.warmup + i) for i in range(args.steps)]
    else:
        gw = capture(step, args.warmup, 0)
        gt = capture(step, args.steps, args.warmup)
        warm, timed = gw.replay, gt.replay
    # sustained load with clock sampling, then the warm-up steps.  Every rank
    # makes the same number of replays (the sharded step holds a collective),
    # so the count comes from one timed round agreed over the ranks first.
    sampler.start()
    t0 = time.perf_counter()
    for _ in range(20):
        warm()
    torch.cuda.synchronize()
    t_round = torch.tensor([time.perf_counter() - t0], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_round, op=dist.ReduceOp.MAX)
    rounds = max(0, math.ceil(args.clock_window / max(float(t_round.item()), 1e-6)) - 1)
    for _ in range(rounds):
        for _ in range(20):
            warm()
        torch.cuda.synchronize()
    if not args.no_graph:
        timed()  # first replay uploads the timed graph (a one-time driver cost, kept out of the timing)
    warm()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    timed()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    per_step_s = ms_max / 1e3 / args.steps
    value = job_bytes / per_step_s / 1e9
    del gw, gt  # graphs holding collective launches go before the process group

    # dominant kernel alone, back to back on the same stream (no collective)
    dom = wl["dominant"]
    if wl["launches"] == 1:
        dom_s = per_step_s
    elif args.no_graph:
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for i in range(args.steps):
            dom(args.warmup + i)
        d1.record(stream)
        torch.cuda.synchronize()
        dom_s = d0.elapsed_time(d1) / 1e3 / args.steps
    else:
        dom_s = time_launches(dom, args.steps, args.warmup)
    peak, peak_kind = peaks()
    achieved = wl["dominant_bytes"] / dom_s / 1e9
    traffic = ncu_traffic(args.workload) if world == 1 else None

    e2e = None
    if wl["e2e"] is not None and args.workload in ("rmsnorm_gemv_int8", "gemv_fp16") and E2E_BIN.exists():
        # the C host of the drop-in ABI (csrc/e2e_bench.c)
        K, N = wl["meta"]["K"], wl["meta"]["N"]
        opname = "RmsNorm-GEMV-INT8" if args.workload == "rmsnorm_gemv_int8" else "GEMV-FP16"
        env = dict(os.environ, VKC_DEVICE=str(local))
        # host-clock steps of ~30 us: at least 1000 timed after 100 warm-up
        # (well under a second), so that the first calls' one-time costs and
        # scheduling noise do not weigh on the figure
        e_steps, e_warm = max(args.steps, 1000), max(args.warmup, 100)
        out = subprocess.run([str(E2E_BIN), opname, str(N), str(K), str(e_steps), str(e_warm)],
                             capture_output=True, text=True, env=env, timeout=600)
        if out.returncode != 0:
            raise RuntimeError(f"e2e host failed: {out.stderr[-400:]}")
        r = json.loads(out.stdout.strip().splitlines()[-1])
        dt = r["us_per_step"] * 1e-6
        if world > 1:
            tt = torch.tensor([dt], device=device, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            dt = float(tt.item())
        e2e = {"value": round(world * wl["bytes"] / dt / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": r["h2d_bytes_per_step"], "d2h_bytes_per_step": r["d2h_bytes_per_step"],
               "us_per_step": round(dt * 1e6, 2), "steps": e_steps, "warmup": e_warm,
               "host_us_per_call": {k: r.get("us_" + k) for k in ("write", "execute", "read")},
               "path": "C host (vkc_e2e_bench): writeBuffer + execute + readBuffer per step, reference ABI, "
                       "host wall clock, weight pool > 4x L2; execute timing events off (vkc_set_timing(0): "
                       "the program never calls getExecutionTime)"}
    elif wl.get("e2e_sharded") is not None:
        dt, hb, db = e2e_sharded(args, wl)
        tt = torch.tensor([dt], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt.item())
        e2e = {"value": round(job_bytes / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": hb,
               "d2h_bytes_per_step": db, "us_per_step": round(dt * 1e6, 2),
               "path": "Python API (vk_compute_b200.ops + p2p) per rank: x host->device from pinned memory, "
                       "the rank's RmsNorm-GEMV shard, NVLink all-gather of y, whole y device->host; host wall "
                       "clock, max over ranks"}
    elif wl["e2e"] is not None:
        dt, hb, db = e2e_dropin(args, wl["e2e"], local)
        if world > 1:
            tt = torch.tensor([dt], device=device, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            dt = float(tt.item())
        e2e = {"value": round(world * wl["bytes"] / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": hb,
               "d2h_bytes_per_step": db, "us_per_step": round(dt * 1e6, 2),
               "path": "Python ctypes: writeBuffer + execute + readBuffer per step, reference ABI, host wall clock"}
    if "close" in wl:
        wl["close"]()
    dom_name, meta, launches = wl["dominant_name"], wl["meta"], wl["launches"]
    bytes_rank, dom_bytes = wl["bytes"], wl["dominant_bytes"]
    del wl, step, dom
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    decode = None
    if not args.no_decode:
        torch.cuda.synchronize()
        decode = decode_step_bench(rank, world, device, max(1, args.decode_steps), 3, peak,
                                   parity=not args.no_decode_parity, shape=args.decode_shape,
                                   emulate_world=args.decode_emulate_shard, exchange=args.decode_exchange)

    configs = None
    if world == 1 and args.workload == "rmsnorm_gemv_int8" and not args.no_configs:
        configs = measure_configs(rank, device, args.steps, peak, local)

    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_baseline(args.workload)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        r = cpu_baseline(args.workload, budget_s=6.0, threads=1)
        cpu1 = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if world > 1:
        dist.barrier()
    if rank == 0:
        parallelism = "1 GPU"
        if world > 1:
            parallelism = (f"row shards x{world} of one matrix + NVLink all-gather of y" if scaling == "strong"
                           else f"row shards x{world}, no collective")
        line = {
            "metric": f"{WORKLOADS[args.workload]} achieved HBM GB/s",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_step_s * 1e3, 5), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "description": WORKLOADS[args.workload],
                       "bytes_per_step": job_bytes, "bytes_per_rank_step": bytes_rank, "per_rank": meta,
                       "l2": "rotating weight pool >= 4x L2; each step reads weights last touched a full pool ago",
                       "graph": not args.no_graph, "pdl": not args.no_pdl, "gemv_plan": args.gemv_plan, "gemv_int_dot": not args.gemv_fma,
                       "attention_plan": args.attention_plan,
                       "parallelism": parallelism},
            "frac_of_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 2),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "algorithmic_bytes": dom_bytes,
                         "us_per_launch": round(dom_s * 1e6, 3)},
            "tensor": ({"achieved_tflops": round(meta["flop"] / dom_s / 1e12, 2),
                        "peak_tflops": tensor_peak(), "frac": round(meta["flop"] / dom_s / 1e12 / tensor_peak(), 4)}
                       if "flop" in meta else None),
            "gpu_launches": args.steps * launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "cpu_baseline_single_thread": cpu1,
            "clocks": clocks,
            "configs": configs,
            "decode_step": decode,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
