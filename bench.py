#!/usr/bin/env python
"""Benchmark of the B200 BDH tril-attention path (one JSON line on rank 0).

Default workload: full BDH prefill forward under bf16 autocast with
``BDH_ATTN_IMPL=cuda_sm100`` — n_layer=6, n_embd=256, n_head=4, N=8192/head, vocab 256,
random N(0, 0.02) weights, synthetic token ids uniform in [0, 256), B=32 x T=512 per GPU
(weak scaling: every rank runs its own batch; no collective on the data path).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 1|2|3|4|5] [--only]
                    [--global-batch G]

* ``value``      tokens/s over all ranks, inputs resident in HBM (device-timed, max over ranks)
* ``e2e``        the same through the public model API with host buffers: pinned token ids
                 copied in and logits copied out inside every timed step
* ``roofline``   the kernel with the most device time in the step (``rooflines``: the three
                 largest), timed live inside the timed region with CUDA events recorded by the
                 library around each launch on its own stream; the bf16 peak is the burst figure
                 for sub-second timed regions, the sustained one for longer ones
* ``cpu_baseline`` the reference's baseline model (bdh_baseline.BDH restated in torch by
                 oracle/baseline_model.py) with the attention computed by the reference's own
                 CPU extension (``csrc/tril_attn_cpu.cpp``, built into oracle/_ref), on the host
                 cores, on a bounded sample
* ``gpu_eager_baseline`` the reference's eval forward op for op on this GPU (eager attention,
                 cuBLAS projections) for the config-2 step and the config-4 decode step, and its
                 eager op (torch matmuls, torch autograd) beside configs 5 and 3
* ``configs``    the metric's other numbers on the same lease, each with its own roofline,
                 clocks and cpu_baseline: config 4 decode tokens/s over the whole span
                 (S = 515 .. 1023), config 5 forward + backward TFLOP/s, config 3 TFLOP/s
* ``strong_scaling`` (N > 1) config 2 at its global batch of 32 sequences and config 5's 64
                 (b, h) units, sharded over the ranks
* ``--impl reference`` runs only the CPU reference arm (rank 0) on this config's metric.
* ``--only``     the config-2 line alone.

Other ``--config`` values run one workload (1: fp32 op, 3: long-T bf16 op, 4: cached decode,
5: forward+backward) with the same JSON schema.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "bdh-gpu-fast_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
N_LAT, D_MODEL, N_HEAD, N_LAYER, VOCAB = 8192, 256, 4, 6, 256


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


SUSTAINED_REGION_S = 2.0  # timed regions at least this long are held to the sustained peak


def tensor_peak(peaks: dict, src: str, region_ms: float):
    """bf16 tensor peak for a kernel timed inside a region of `region_ms`: the burst figure
    (cuBLAS timed alone) for sub-second regions, the sustained one (seconds-long loop under the
    power cap) from SUSTAINED_REGION_S on. Returns (peak, source)."""
    if region_ms / 1e3 >= SUSTAINED_REGION_S and "bf16_tflops_sustained" in peaks:
        return peaks["bf16_tflops_sustained"], (
            f"{src} bf16_tflops_sustained (timed region {region_ms / 1e3:.2f} s)")
    return peaks["bf16_tflops"], f"{src} bf16_tflops burst (timed region {region_ms / 1e3:.2f} s)"


# ------------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock / clock-event reasons sampled every 20 ms during the timed region.

    Reads NVML (``nvidia_ml_py``) from a Python thread; falls back to ``nvidia-smi -lms 200``.
    Only reads: no clock, power or mode setting is touched.
    """

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device, period_s: float = 0.02):
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:  # noqa: BLE001
            pass
        self.period = period_s
        self.samples: list[tuple[float, float, set]] = []
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.stop_ev = threading.Event()
        self.nvml = None
        self.handle = None

    def _nvml_open(self) -> bool:
        try:
            import pynvml

            pynvml.nvmlInit()
            uid = self.uuid if self.uuid.startswith("GPU-") else "GPU-" + self.uuid
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uid)
            self.nvml = pynvml
            return True
        except Exception:  # noqa: BLE001
            self.nvml = None
            return False

    def start(self):
        if self.uuid and self._nvml_open():
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _poll(self):
        nv, h = self.nvml, self.handle
        while not self.stop_ev.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                active = {name for name, const in self.REASONS if mask & getattr(nv, const, 0)}
                self.samples.append((sm, mx, active))
            except Exception:  # noqa: BLE001
                pass
            self.stop_ev.wait(self.period)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.nvml is not None:
            self.stop_ev.set()
            if self.thread:
                self.thread.join(timeout=2)
            sm = [s[0] for s in self.samples]
            reasons = set().union(*[s[2] for s in self.samples]) if self.samples else set()
            mx = self.samples[-1][1] if self.samples else None
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 20 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            if self.uuid and self.uuid.replace("GPU-", "") not in parts[0]:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 200 ms"}


# ------------------------------------------------------------------ native timing
def profile_begin():
    from kernels import sm100_attn

    sm100_attn.profile_begin()


def profile_end():
    from kernels import sm100_attn

    return sm100_attn.profile_end()


# ---------------------------------------------------------------------- helpers
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, dev


def barrier(world):
    if world > 1:
        dist.barrier()


def rank_seed(base: int, rank: int) -> int:
    """Seed of rank `rank`'s synthetic batch (weights use a rank-independent seed)."""
    return base + 7919 * rank


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cross_rank_check(logits_fn, world: int, dev) -> dict:
    """Verification outside the timed region: every rank evaluates the same small batch
    (``logits_fn``), an all_gather brings each rank's logits checksum to every rank, and the
    ranks must agree exactly (deterministic kernels, identical weights and inputs)."""
    lg = logits_fn().double()
    c = torch.stack([lg.sum(), lg.abs().sum(), (lg * lg).sum()]).to(dev)
    if world == 1:
        return {"ranks": 1, "identical": True}
    gathered = [torch.zeros_like(c) for _ in range(world)]
    dist.all_gather(gathered, c)
    ref = gathered[0]
    diff = max(float(((x - ref).abs() / ref.abs().clamp_min(1e-30)).max()) for x in gathered)
    return {"ranks": world, "identical": all(bool(torch.equal(x, ref)) for x in gathered),
            "max_rel_diff": diff, "collective": "all_gather (verification only, untimed)"}


def timed(fn, steps: int, world: int, dev, join=None) -> float:
    """Device time (ms) of `steps` calls, bracketed by barrier + synchronize; max over ranks.
    `join`: called before the end event is recorded (e.g. to make the timing stream wait for a
    side stream's last copy)."""
    barrier(world)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    if join is not None:
        join()
    e.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    return max_over_ranks(s.elapsed_time(e), world, dev)


def load_traffic(name: str, batch: int | None = None):
    """DRAM bytes (read + write) of one launch from a committed ncu summary.

    ``profiles/<name>.json`` holds the bytes ncu measured on a capture of ``captured_batch``
    rows of batch; the traffic of every kernel here grows in proportion to the batch (independent
    (b,h) units), so it is scaled to this run's batch, except an optional
    ``traffic_fixed_bytes`` part that does not (weights read once per launch).
    """
    p = REPO / "profiles" / f"{name}.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        t = float(d["traffic_bytes_per_captured_launch"])
        fixed = float(d.get("traffic_fixed_bytes", 0.0))
        cb = d.get("captured_batch")
        if batch and cb:
            t = fixed + (t - fixed) * batch / cb
        return t
    except Exception:  # noqa: BLE001
        return None


# ------------------------------------------------------------------ CPU reference
def cpu_reference_model(B_cpu: int, T: int, steps: int):
    """BDH prefill on the host cores: the reference's baseline model (bdh_baseline.BDH,
    restated in torch CPU fp32 by oracle/baseline_model.py) with its strictly causal attention
    computed by the reference's own C++ extension (``tril_score_v_cpu``, built into oracle/_ref;
    the same arithmetic in torch when that is missing). Config-2 model, random N(0, 0.02)
    weights. Returns (tokens/s, kind, cores, sample)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import baseline_model

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    attn = baseline_model.reference_tril_score_v()
    how = "the reference CPU extension (oracle/_ref)" if attn is not None else "torch (extension not built)"
    g = torch.Generator().manual_seed(1002)
    N = N_LAT
    w = {"embed": torch.randn(VOCAB, D_MODEL, generator=g) * 0.02,
         "encoder": torch.randn(N_HEAD, D_MODEL, N, generator=g) * 0.02,
         "encoder_v": torch.randn(N_HEAD, D_MODEL, N, generator=g) * 0.02,
         "decoder": torch.randn(N_HEAD * N, D_MODEL, generator=g) * 0.02,
         "lm_head": torch.randn(D_MODEL, VOCAB, generator=g) * 0.02}
    import bdh_model

    w["freqs"] = bdh_model.get_freqs(N, 2 ** 16, torch.float32)
    idx = torch.randint(0, VOCAB, (B_cpu, T), generator=torch.Generator().manual_seed(2002))
    baseline_model.baseline_forward(idx, w, N_LAYER, N_HEAD, attn)  # warm-up
    t0 = time.perf_counter()
    for _ in range(steps):
        baseline_model.baseline_forward(idx, w, N_LAYER, N_HEAD, attn)
    dt = time.perf_counter() - t0
    sample = (f"BDH prefill B={B_cpu} x T={T}, {N_LAYER} layers, fp32, {steps} timed forward(s) "
              f"after 1 warm-up; bdh_baseline.BDH restated in torch (oracle/baseline_model.py), "
              f"attention by {how}; {cores} threads; {_cpu_model_name()}")
    return B_cpu * T * steps / dt, "port", cores, sample


def _ref_ext():
    """The reference CPU extension from oracle/_ref, or None (then the numpy port is timed)."""
    try:
        sys.path.insert(0, str(REPO / "oracle"))
        import build_ref

        return build_ref.load_module()
    except Exception:  # noqa: BLE001
        return None


def _cpu_model_name() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:  # noqa: BLE001
        pass
    return ""


def cpu_op_baseline(cfg_id: int):
    """Reference CPU attention on a bounded sample of an op config, in the op line's unit
    (executed-algorithm causal TFLOP/s, fp32 on the host cores). Config 1: the whole op (16
    (b,h) units, T = 512); config 3: one unit at T = 8192; config 5: one unit at T = 2048,
    forward by the reference extension and backward by the numpy port of the analytic backward
    (the reference's backward is Python over torch and does not travel). RoPE is applied to the
    sample beforehand, untimed (O(T N) against the O(T^2 N) attention)."""
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import tril_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    ext = _ref_ext()
    units, T = {1: (16, 512), 3: (1, 8192), 5: (1, 2048)}[cfg_id]
    N, D = N_LAT, D_MODEL
    g = torch.Generator().manual_seed(3000 + cfg_id)
    shift = 1.645 if cfg_id == 3 else 0.0
    q = torch.relu(torch.randn(1, units, T, N, generator=g) - shift)
    v = torch.randn(1, 1, T, D, generator=g)
    if cfg_id == 3:
        v = torch.nn.functional.layer_norm(v, (D,))
    qr = torch.from_numpy(tril_oracle.rope(q.numpy(), tril_oracle.get_freqs(N)).astype(np.float32))
    if ext is not None:
        fwd = lambda: ext.tril_score_v_cpu(qr, qr, v)  # noqa: E731
    else:
        fwd = lambda: tril_oracle.tril_score_v(qr.numpy(), qr.numpy(), v.numpy(), acc=np.float32)  # noqa: E731
    dout = torch.randn(1, units, T, D, generator=g).numpy()
    reps = 3 if cfg_id == 1 else 1
    fwd()  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        fwd()
        if cfg_id == 5:
            tril_oracle.tril_backward(qr.numpy(), qr.numpy(), v.numpy(), dout, acc=np.float32,
                                      k_is_q=True)
    dt = time.perf_counter() - t0
    flops = units * T * (T - 1) * ((N + D) + ((3 * N + 2 * D) if cfg_id == 5 else 0)) * reps
    kind = "reference" if ext is not None and cfg_id != 5 else "port"
    how = ("reference CPU extension tril_score_v_cpu" if ext is not None else "numpy port")
    if cfg_id == 5:
        how += " forward + numpy port of the analytic backward"
    sample = (f"{units} (b,h) unit(s) x T={T}, N={N}, D={D}, fp32, {reps} timed call(s) after 1 "
              f"warm-up; {how}; {cores} threads; {_cpu_model_name()}")
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": sample}


def cpu_decode_baseline(steps: int = 4):
    """BDH cached decode on the host: the config-4 model at B = 1 after a 512-token prompt, the
    reference CPU extension's tril_decode_cpu / tril_score_v_cpu inside the model (fp32 cache),
    `steps` timed T = 1 steps. Returns the cpu_baseline object (tokens/s)."""
    import bdh_model
    from bdh_cache import CacheManager
    from kernels import attention_dispatch as ad

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    ext = _ref_ext()
    cfg = bdh_model.BDHConfig(n_layer=N_LAYER, n_embd=D_MODEL, n_head=N_HEAD,
                              mlp_internal_dim_multiplier=128, vocab_size=VOCAB, dropout=0.0)
    torch.manual_seed(1004)
    model = bdh_model.BDH(cfg).eval()
    model.attn._attn_impl_override = "eager"
    P = 512
    toks = torch.randint(0, VOCAB, (1, P + steps + 1), generator=torch.Generator().manual_seed(2004))
    cache = CacheManager.from_config(cfg, 1, P + steps + 1, torch.device("cpu"))
    orig = (ad.eager_tril_attn, ad.eager_decode_attn)
    if ext is not None:
        ad.eager_tril_attn = lambda q, k, v: ext.tril_score_v_cpu(q, k, v)  # noqa: E731
        ad.eager_decode_attn = lambda q, k, v: ext.tril_decode_cpu(q, k, v)  # noqa: E731
    try:
        with torch.inference_mode():
            model(toks[:, :P], cache=cache)
            model(toks[:, P:P + 1], cache=cache)  # warm-up step
            t0 = time.perf_counter()
            for i in range(steps):
                model(toks[:, P + 1 + i:P + 2 + i], cache=cache)
            dt = time.perf_counter() - t0
    finally:
        ad.eager_tril_attn, ad.eager_decode_attn = orig
    kind = "reference" if ext is not None else "port"
    sample = (f"config-4 model, B=1, {P}-token prompt, {steps} timed decode steps after 1 warm-up, "
              f"fp32 cache; attention by the {'reference CPU extension' if ext is not None else 'eager torch path'}; "
              f"{cores} threads; {_cpu_model_name()}")
    return {"value": steps / dt, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}


# --------------------------------------------------------------------- config 2
def config2_model(dev, impl: str = "cuda_sm100"):
    """The config-2 model (identical random N(0, 0.02) weights on every rank)."""
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=N_LAYER, n_embd=D_MODEL, n_head=N_HEAD,
                              mlp_internal_dim_multiplier=128, vocab_size=VOCAB, dropout=0.0)
    torch.manual_seed(1002)
    model = bdh_model.BDH(cfg).to(dev).eval()
    model.attn._attn_impl_override = impl
    return model


def config2_rooflines(prof: dict, B: int, T: int, steps: int, region_ms: float) -> dict:
    """Rooflines of the three largest kernels of the config-2 step. Algorithmic work per launch
    (one layer, the whole batch):
      score pass  B H T (T-1) N flops (causal Q K^T, T(T-1)/2 pairs x 2N)       tensor
    With xs stored (default):
      encode      2 B T H N x 2 bytes written (xs, QR) + x and weights read      HBM
      gate + decoder in one kernel (default, BDH_SM100_GATE_DEC=0 splits them):
                  2 x 2 B T H N D flops (y encv, xy dec), xs read, xy never stored  tensor
      gate alone  B T H N x 2 read (xs) + B T H N x 2 written (xy) + y, weights  HBM
    With xs recomputed in the gate (BDH_SM100_GATE_X=1):
      encode      B T H N x 2 bytes written (QR) + x and weights read            HBM
      gate        2 x 2 B T H N D flops (x enc and y encv), xy written           tensor"""
    peaks, src = load_peaks()
    tpeak, tsrc = tensor_peak(peaks, src, region_ms)
    lat = B * T * N_HEAD * N_LAT * 2
    small = B * T * D_MODEL * 2 + N_HEAD * D_MODEL * N_LAT * 2
    gate_x = os.environ.get("BDH_SM100_GATE_X", "0") == "1"
    if gate_x:
        enc_spec = ("latent encode x@enc + ReLU + RoPE (tc_gemm_kernel<EncodeProb<..., WX=false>>), "
                    "QR written", "hbm", lat + small, 1e9, "GB/s", peaks["hbm_gbs"],
                    f"{src} hbm_gbs", "latent_encode_config2")
        gate_spec = ("latent gate relu(x@enc) * relu(y@encv), xs recomputed (tc_gemm_kernel<GateXProb>, "
                     "two side-by-side TMEM products), xy written", "tensor",
                     4 * B * T * N_HEAD * N_LAT * D_MODEL, 1e12, "TFLOP/s", tpeak, tsrc,
                     "latent_gate_config2")
    else:
        enc_spec = ("latent encode x@enc + ReLU + RoPE (tc_gemm_kernel<EncodeProb>), xs and QR written",
                    "hbm", 2 * lat + small, 1e9, "GB/s", peaks["hbm_gbs"], f"{src} hbm_gbs",
                    "latent_encode_config2")
        if os.environ.get("BDH_SM100_GATE_DEC", "1") != "0":
            gate_spec = ("latent gate + decoder (xs * relu(y@encv)) @ dec (gate_dec_kernel, "
                         "cta_group::2, xy kept in shared memory)", "tensor",
                         4 * B * T * N_HEAD * N_LAT * D_MODEL, 1e12, "TFLOP/s", tpeak, tsrc,
                         "gate_dec_config2")
        else:
            gate_spec = ("latent gate xs * relu(y@encv) (tc_gemm_kernel<GateProb>), xs read, xy written",
                         "hbm", 2 * lat + small + B * N_HEAD * T * D_MODEL * 2, 1e9, "GB/s",
                         peaks["hbm_gbs"], f"{src} hbm_gbs", "latent_gate_config2")
    specs = {
        "score": ("score pass tril(QR QR^T,-1) (tc_pair_kernel<ScorePairT<7, 0>>, cta_group::2 256x256 tiles, seven operand stages)"
                  if os.environ.get("BDH_SM100_PAIR", "1") != "0"
                  else "score pass tril(QR QR^T,-1) (tc_gemm_kernel<ScoreProb<bf16>>)",
                  "tensor", B * N_HEAD * T * (T - 1) * N_LAT, 1e12, "TFLOP/s", tpeak, tsrc,
                  "score_pass_config2"),
        "encode": enc_spec,
        "gate": gate_spec,
    }
    rooflines = {}
    for k, (name, bound, work, scale, unit, peak, psrc, tname) in specs.items():
        kp = prof.get(k)
        if not kp or not kp["launches"]:
            continue
        per = kp["ms"] / kp["launches"]
        ach = work / (per / 1e3) / scale
        rooflines[k] = {"kernel": name, "bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                        "frac": ach / peak, "peak_source": psrc, "traffic": load_traffic(tname, B),
                        "avg_launch_ms": per, "work_per_launch": work,
                        "ms_per_step": kp["ms"] / steps}
    return rooflines


def time_config2(model, idx, steps: int, warmup: int, world: int, dev, native: bool = True):
    """Device-timed prefill steps of `model` on `idx` (max over ranks). Returns
    (ms, library per-kernel profile or None, clocks)."""
    def step():
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model(idx)[0]

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    if native:
        profile_begin()
    ms = timed(step, steps, world, dev)
    prof = profile_end() if native else None
    clk = clocks.stop()
    return ms, prof, clk


def bench_config2(args, world, rank, dev):
    from kernels import sm100_attn

    T = 512
    strong = args.global_batch > 0
    if strong:
        if args.global_batch % world:
            raise SystemExit(f"--global-batch {args.global_batch} is not a multiple of {world} GPUs")
        B = args.global_batch // world
    else:
        B = args.batch or 32
    model = config2_model(dev)
    g = torch.Generator().manual_seed(rank_seed(2002, rank))
    idx_host = torch.randint(0, VOCAB, (B, T), generator=g).pin_memory()
    idx = idx_host.to(dev)
    # eager calls with a CUDA event pair around every library launch: the per-kernel device
    # times the rooflines use (the events and the per-launch host work slow the step itself)
    ms_ev, prof, clk_ev = time_config2(model, idx, args.steps, args.warmup, world, dev)
    assert sm100_attn.device_error(dev) == 0
    value_eager = world * B * T * args.steps / (ms_ev / 1e3)

    # `value`: the same step replayed from CUDA graphs (the public bdh_model.GraphedForward:
    # launches and their host work paid once, at capture), inputs resident; two captures so that
    # one step's logits can be copied out while the other graph runs the next step (e2e below)
    graphs = [model.graphed_forward(B, T) for _ in range(2)]

    def graph_step_n():
        graphs[0](idx)

    for _ in range(args.warmup):
        graph_step_n()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    ms = timed(graph_step_n, args.steps, world, dev)
    clk = clocks.stop()
    assert sm100_attn.device_error(dev) == 0
    value = world * B * T * args.steps / (ms / 1e3)

    # end to end through the public API with host buffers: every step copies its token ids in
    # from pinned memory (into the graph's input buffer) and its bf16 logits out to pinned
    # memory; the copy-out of step i runs on a side stream beside step i + 1 (the other graph,
    # two host buffers in turn), and the timed region ends after the last copy has landed
    logits_host = [torch.empty(tuple(graphs[0].logits.shape), dtype=torch.bfloat16).pin_memory()
                   for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    copied = [None, None]  # event after the copy-out of each graph's last logits
    n_e2e = [0]

    def e2e_step():
        k = n_e2e[0] % 2
        run = graphs[k]
        cur = torch.cuda.current_stream(dev)
        if copied[k] is not None:
            cur.wait_event(copied[k])  # that graph's previous logits have been copied out
        run.idx.copy_(idx_host, non_blocking=True)
        run.graph.replay()
        copy_stream.wait_stream(cur)
        with torch.cuda.stream(copy_stream):
            logits_host[k].copy_(run.logits, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy_stream)
        copied[k] = ev
        n_e2e[0] += 1

    def e2e_join():
        torch.cuda.current_stream(dev).wait_stream(copy_stream)

    def verify_logits():
        gv = torch.Generator().manual_seed(4242)  # the same batch on every rank
        iv = torch.randint(0, VOCAB, (2, 256), generator=gv).to(dev)
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model(iv)[0].float()

    xcheck = cross_rank_check(verify_logits, world, dev)
    for _ in range(max(1, args.warmup)):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps, world, dev, join=e2e_join)
    torch.cuda.synchronize(dev)
    e2e = world * B * T * args.steps / (ms_e2e / 1e3)

    rooflines = config2_rooflines(prof, B, T, args.steps, ms_ev)
    dominant = max(rooflines, key=lambda k: rooflines[k]["ms_per_step"]) if rooflines else None
    attn_ms = sum(prof[k]["ms"] for k in ("score", "value", "rope"))
    attn_flops = N_LAYER * args.steps * B * N_HEAD * T * (T - 1) * (N_LAT + D_MODEL)
    launches = sum(v["launches"] for v in prof.values())
    line = {
        "metric": "BDH prefill tokens/s (config 2: 6L, D=256, nh=4, N=8192, B=32, T=512)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "BDH prefill forward, bf16 autocast, random-init weights, "
                               "token ids uniform [0,256)",
                   "global_batch": B * world, "per_gpu_batch": B, "seq_len": T,
                   "n_layer": N_LAYER, "n_head": N_HEAD, "n_latent_per_head": N_LAT, "n_embd": D_MODEL,
                   "parallelism": f"batch-sharded x{world} ({'strong' if strong else 'weak'}), "
                                  "no collective on the data path",
                   "cache": "inputs larger than L2 (1 GB latent per layer per GPU); no flush"},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": idx_host.numel() * 8,
                "d2h_bytes_per_step": logits_host[0].numel() * 2,
                "api": "bdh_model.BDH.graphed_forward (the step captured as a CUDA graph)",
                "copies": "token ids in on the compute stream; logits out on a side stream, "
                          "overlapping the next step; the timed region ends after the last"},
        "timing": "value: the step replayed from a CUDA graph (BDH.graphed_forward), inputs "
                  "resident, CUDA events over the K steps; value_eager: the same step as eager "
                  "calls with an event pair around every library launch, the per-kernel times "
                  "that roofline, rooflines and kernel_ms come from",
        "value_eager": {"value": value_eager, "unit": "tokens/s",
                        "ms_per_step": ms_ev / args.steps, "clocks": clk_ev},
        "roofline": rooflines.get(dominant),
        "rooflines": rooflines,
        "attn_tflops": attn_flops / (attn_ms / 1e3) / 1e12 if attn_ms else None,
        "attn_share_of_step": attn_ms / ms_ev if ms_ev else None,
        "kernel_ms": {k: v["ms"] / args.steps for k, v in prof.items() if v["launches"]},
        "gpu_launches": launches,
        "clocks": clk,
        "cross_rank_check": xcheck,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, kind, cores, sample = cpu_reference_model(1, T, 1)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}
    if args.only:
        return line
    del graphs, logits_host, copy_stream
    # the reference's op sequence on this GPU: the same model with eager attention and torch
    # (cuBLAS) projections, bit for bit the calls bdh.py's eval forward makes under autocast
    model.attn._attn_impl_override = "eager"
    os.environ["BDH_SM100_LATENT"] = "0"
    try:
        ms_eager, _, clk_e = time_config2(model, idx, 5, 3, world, dev, native=False)
    finally:
        os.environ.pop("BDH_SM100_LATENT", None)
        model.attn._attn_impl_override = "cuda_sm100"
    line["gpu_eager_baseline"] = {
        "config2": {"value": world * B * T * 5 / (ms_eager / 1e3), "unit": "tokens/s",
                    "ms_per_step": ms_eager / 5, "steps": 5, "warmup": 3, "clocks": clk_e,
                    "what": "config-2 step with BDH_ATTN_IMPL=eager and torch/cuBLAS projections "
                            "(the reference's eval forward op for op: kernels/attention.py:27-40, "
                            "bdh.py:947-1072) on this GPU"}}
    if world > 1:
        line["strong_scaling"] = strong_scaling(model, args, world, rank, dev)
    del model
    torch.cuda.empty_cache()
    line["configs"] = other_configs(args, world, rank, dev, line["gpu_eager_baseline"])
    return line


def strong_scaling(model, args, world, rank, dev):
    """Config 2 at its stated global batch (B = 32 sequences sharded over the ranks, 32 / N
    each) and config 5's 64 (b, h) units sharded the same way (16 / N sequences of 4 heads):
    the whole job's throughput at fixed total work, and the per-kernel device times of one rank,
    to show which kernel stops shrinking."""
    out = {}
    Bg, T = 32, 512
    if Bg % world == 0:
        b = Bg // world
        g = torch.Generator().manual_seed(rank_seed(2102, rank))
        idx = torch.randint(0, VOCAB, (b, T), generator=g).to(dev)
        ms_ev, prof, clk_ev = time_config2(model, idx, args.steps, args.warmup, world, dev)
        graph = model.graphed_forward(b, T)
        for _ in range(args.warmup):
            graph(idx)
        torch.cuda.synchronize(dev)
        clocks = ClockSampler(dev)
        clocks.start()
        ms_g = timed(lambda: graph(idx), args.steps, world, dev)
        clk = clocks.stop()
        del graph
        out["config2"] = {"value": Bg * T * args.steps / (ms_g / 1e3), "unit": "tokens/s",
                          "global_batch": Bg, "per_gpu_batch": b,
                          "ms_per_step": ms_g / args.steps, "clocks": clk,
                          "value_eager": Bg * T * args.steps / (ms_ev / 1e3),
                          "ms_per_step_eager": ms_ev / args.steps, "clocks_eager": clk_ev,
                          "kernel_ms_rank0": {k: v["ms"] / args.steps for k, v in prof.items()
                                              if v["launches"]},
                          "timing": "value: CUDA-graph replay of the step; value_eager and "
                                    "kernel_ms_rank0: eager calls with per-launch events",
                          "scaling": "strong"}
    if 16 % world == 0:
        sub = argparse.Namespace(**vars(args))
        sub.config, sub.batch, sub.no_cpu_baseline = 5, 16 // world, True
        sub.steps = max(args.steps // 2, 5)
        ln = bench_op(sub, world, rank, dev)
        out["config5"] = {"value": ln["value"], "unit": ln["unit"], "global_units": 64,
                          "per_gpu_units": 4 * (16 // world), "ms_per_step": ln["ms_per_step"],
                          "kernel_ms_rank0": ln["kernel_ms"], "clocks": ln["clocks"],
                          "scaling": "strong"}
    return out


def other_configs(args, world, rank, dev, eager):
    """The metric's other numbers on the same lease (each a sub-object with its own roofline,
    clocks and cpu_baseline): config 4 decode tokens/s over the whole span (B = 64, 512-token
    prompt, S up to 1023), config 5 forward + backward TFLOP/s, config 3 long-context TFLOP/s;
    and, into ``eager`` (the line's gpu_eager_baseline), the reference's eager path for each:
    the decode step beside config 4 and the op beside configs 5 and 3."""
    out = {}
    sub = argparse.Namespace(**vars(args))
    sub.batch = 0
    sub.config, sub.warmup = 4, 3
    sub.steps = 1024 - 512 - sub.warmup
    out["config4_decode"] = bench_decode(sub, world, rank, dev)
    torch.cuda.empty_cache()
    sub.eager = True  # the same span
    eager["config4"] = bench_decode(sub, world, rank, dev)
    sub.eager = False
    torch.cuda.empty_cache()
    sub.steps = 10
    sub.config = 5
    out["config5_fwd_bwd"] = bench_op(sub, world, rank, dev)
    torch.cuda.empty_cache()
    sub.steps = 5
    eager["config5"] = bench_op_eager(sub, world, rank, dev, out["config5_fwd_bwd"])
    torch.cuda.empty_cache()
    sub.steps = 10
    sub.config = 3
    out["config3_long_context"] = bench_op(sub, world, rank, dev)
    torch.cuda.empty_cache()
    sub.steps = 5
    eager["config3"] = bench_op_eager(sub, world, rank, dev, out["config3_long_context"])
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------- standalone op configs
def _op_inputs(cfg_id, dev, rank, batch=0):
    g = torch.Generator(device=dev).manual_seed(rank_seed(1000 + cfg_id, rank))
    if cfg_id == 1:
        B, H, T, N, D, dt = batch or 4, 4, 512, N_LAT, D_MODEL, torch.float32
        q = torch.relu(torch.randn(B, H, T, N, device=dev, generator=g))
        v = torch.randn(B, 1, T, D, device=dev, generator=g)
    elif cfg_id == 3:
        B, H, T, N, D, dt = batch or 8, 4, 8192, N_LAT, D_MODEL, torch.bfloat16
        q = torch.relu(torch.randn(B, H, T, N, device=dev, generator=g) - 1.645).to(dt)
        v = torch.nn.functional.layer_norm(torch.randn(B, 1, T, D, device=dev, generator=g), (D,)).to(dt)
    else:  # 5
        B, H, T, N, D, dt = batch or 16, 4, 2048, N_LAT, D_MODEL, torch.bfloat16
        q = torch.relu(torch.randn(B, H, T, N, device=dev, generator=g)).to(dt)
        v = torch.randn(B, 1, T, D, device=dev, generator=g).to(dt)
    return q, v, (B, H, T, N, D, dt)


_TF32_PEAK = {}


def measured_tf32_tflops(dev) -> float:
    """cuBLAS TF32 GEMM throughput on this GPU (fp32 8192^3 with TF32 allowed, best of 5)."""
    if dev in _TF32_PEAK:
        return _TF32_PEAK[dev]
    n = 8192
    a = torch.randn(n, n, device=dev)
    b = torch.randn(n, n, device=dev)
    c = torch.empty(n, n, device=dev)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for _ in range(3):
            torch.mm(a, b, out=c)
        best = float("inf")
        for _ in range(5):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.mm(a, b, out=c)
            e.record()
            torch.cuda.synchronize(dev)
            best = min(best, s.elapsed_time(e))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    _TF32_PEAK[dev] = 2 * n ** 3 / (best / 1e3) / 1e12
    return _TF32_PEAK[dev]


def chunk_len(T: int) -> int:
    """Keys per chunk of the library's chunked forward (csrc/attn_chunked.cu chunk_len)."""
    forced = os.environ.get("BDH_SM100_CHUNK", "")
    if forced in ("256", "512"):
        return int(forced)
    return 512 if T >= 4096 else 256


def state_terms() -> int:
    """bf16 terms per prefix-state element of the chunked forward (csrc/capi.cu
    bf16_one_term): one by default, hi + lo with BDH_SM100_SPLIT_SCORES=1."""
    return 2 if os.environ.get("BDH_SM100_SPLIT_SCORES", "") == "1" else 1


def op_roofline(cfg_id, prof, shape, chunked, peaks, src, dev, steps, region_ms):
    """Roofline of the dominant kernel of an op config (algorithmic work per launch / time).

    * config 1 (fp32): score pass, causal Q K^T flops B H T(T-1) N against a measured cuBLAS
      TF32 GEMM peak (the pass issues 3 TF32 products per algorithmic product for fp32 accuracy);
    * config 3 (chunked): prefix-state pass, HBM bytes = K and V read once + the bf16 prefix
      states written, (T/C - 1) N D 2 bytes per (b,h) (4 with the hi/lo split);
    * config 5: grad-Q pass, dQ_total = dS Q + dS^T Q, causal flops 2 T(T-1) N per (b,h),
      against the burst bf16 peak for sub-second timed regions (``tensor_peak``).
    """
    B, H, T, N, D = shape
    units = B * H
    if cfg_id == 1:
        k = prof["score"]
        work = units * T * (T - 1) * N
        peak, unit, bound = measured_tf32_tflops(dev), "TFLOP/s", "tensor"
        psrc = "measured in this run: cuBLAS TF32 GEMM 8192^3, best of 5 (burst)"
        kern = ("score pass (tc_gemm_kernel<ScoreProb<tf32>>, 3-product split, K-split partials + "
                "in-order reduce), per step")
        tname = "score_pass_config1"
    elif cfg_id == 3 and chunked:
        k = prof["state"]
        C = chunk_len(T)
        st = state_terms()
        work = units * ((T // C - 1) * N * D * 2 * st + T * N * 2) + B * T * D * 2
        peak, unit, bound = peaks["hbm_gbs"], "GB/s", "hbm"
        psrc = f"{src} hbm_gbs"
        kern = ("prefix-state pass (tc_gemm_kernel<StateProb>), bf16 "
                + ("hi/lo" if st == 2 else "single-term") + " state writes")
        tname = "state_pass_config3"
    else:
        k = prof["grad_q"] if cfg_id == 5 else prof["score"]
        work = units * T * (T - 1) * N * (2 if cfg_id == 5 else 1)
        (peak, psrc), unit, bound = tensor_peak(peaks, src, region_ms), "TFLOP/s", "tensor"
        kern = ("grad-Q pass (tc_pair_kernel<GradQPair>, cta_group::2)" if cfg_id == 5
                else "score pass")
        tname = "grad_q_config5" if cfg_id == 5 else "score_pass_config3"
    if not k["launches"]:
        return None
    per = k["ms"] / k["launches"]
    if cfg_id == 1:
        # the fp32 score pass may be K-split: main pass + in-order reduce, both timed as "score";
        # one score pass per step
        per = k["ms"] / max(1, steps)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    achieved = work / (per / 1e3) / scale
    return {"kernel": kern, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "peak_source": psrc,
            "traffic": load_traffic(tname, B),
            "avg_launch_ms": per, "work_per_launch": work}


def bench_op(args, world, rank, dev):
    import bdh_model
    from kernels.attention_dispatch import bdh_rope_attn

    cfg_id = args.config
    q, v, (B, H, T, N, D, dt) = _op_inputs(cfg_id, dev, rank, args.batch)
    freqs = bdh_model.get_freqs(N, 2 ** 16, torch.float32).to(dev)
    if cfg_id == 5:
        dO = torch.randn(B, H, T, D, device=dev).to(dt)
        qg = q.clone().requires_grad_(True)
        vg = v.clone().requires_grad_(True)

        def step():
            # a training step's gradients start empty (zero_grad(set_to_none=True)), so the
            # backward writes them instead of accumulating into last step's
            qg.grad = None
            vg.grad = None
            out, _ = bdh_rope_attn(qg, vg, freqs, 0, impl="cuda_sm100")
            out.backward(dO)
    else:
        def step():
            return bdh_rope_attn(q, v, freqs, 0, impl="cuda_sm100")[0]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    profile_begin()
    ms = timed(step, args.steps, world, dev)
    prof = profile_end()
    clk = clocks.stop()
    # executed-algorithm flops (per (b,h) unit, one product per multiply-add pair whatever the
    # operand split): quadratic causal T(T-1)(N+D), or the chunked form
    # (T/C) C(C-1)(N+D) + 2 (T-C) N D when the library takes it (bf16 and T >= 1536)
    C = chunk_len(T)
    chunked = dt == torch.bfloat16 and T >= 1536
    quad_fwd = B * H * T * (T - 1) * (N + D)
    fwd = B * H * ((T // C) * C * (C - 1) * (N + D) + 2 * (T - C) * N * D) if chunked else quad_fwd
    bwd = B * H * T * (T - 1) * (3 * N + 2 * D) if cfg_id == 5 else 0
    flops = (fwd + bwd) * args.steps * world
    effective = (quad_fwd + bwd) * args.steps * world
    peaks, src = load_peaks()
    sc = prof["score"]
    per_launch = sc["ms"] / sc["launches"] if sc["launches"] else None
    roof = op_roofline(cfg_id, prof, (B, H, T, N, D), chunked, peaks, src, dev, args.steps, ms)
    line = {
        "metric": f"tril-attn TFLOP/s (config {cfg_id}, executed-algorithm causal flops)",
        "value": flops / (ms / 1e3) / 1e12,
        "effective_tflops_quadratic_equivalent": effective / (ms / 1e3) / 1e12,
        "forward_form": f"chunked C={C}" if chunked else "quadratic",
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if dt == torch.float32 else "bf16", "data": "synthetic",
        "config": {"workload": f"config {cfg_id} op", "B": B, "H": H, "T": T, "N": N, "D": D,
                   "tokens_per_s": world * B * T * args.steps / (ms / 1e3),
                   "cache": "inputs larger than L2"},
        "roofline": roof,
        "kernel_ms": {k: v_["ms"] / args.steps for k, v_ in prof.items() if v_["launches"]},
        "score_ms_per_launch": per_launch,
        "gpu_launches": sum(v_["launches"] for v_ in prof.values()),
        "clocks": clk, "peak_source": src,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_op_baseline(cfg_id)
    return line


def bench_op_eager(args, world, rank, dev, native_line):
    """The reference's path for an op config on this GPU, beside ``bench_op``'s line: RoPE
    tables and (QR QR^T).tril(-1) V as torch matmuls (cuBLAS), the reference's eager attention
    (kernels/attention.py:27-40 behind BDH_ATTN_IMPL=eager); for config 5 the backward is torch
    autograd through those ops (its default training path, BDH_ATTN_AUTOGRAD=0). ``value`` uses
    the native line's flop count, so the two values compare as times do."""
    import bdh_model
    from kernels.attention_dispatch import bdh_rope_attn

    cfg_id = args.config
    q, v, (B, H, T, N, D, dt) = _op_inputs(cfg_id, dev, rank, args.batch)
    freqs = bdh_model.get_freqs(N, 2 ** 16, torch.float32).to(dev)
    if cfg_id == 5:
        dO = torch.randn(B, H, T, D, device=dev).to(dt)
        qg = q.clone().requires_grad_(True)
        vg = v.clone().requires_grad_(True)

        def step():
            qg.grad = None
            vg.grad = None
            out, _ = bdh_rope_attn(qg, vg, freqs, 0, impl="eager", use_autograd_fn=False)
            out.backward(dO)
    else:
        def step():
            with torch.no_grad():
                return bdh_rope_attn(q, v, freqs, 0, impl="eager")[0]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    ms = timed(step, args.steps, world, dev)
    clk = clocks.stop()
    ms_native = native_line["ms_per_step"] * args.steps
    return {"value": native_line["value"] * ms_native / ms, "unit": native_line["unit"],
            "ms_per_step": ms / args.steps, "steps": args.steps, "warmup": args.warmup,
            "clocks": clk,
            "what": f"config-{cfg_id} op with BDH_ATTN_IMPL=eager: RoPE tables and "
                    "(QR QR^T).tril(-1) V as torch/cuBLAS matmuls (kernels/attention.py:27-40)"
                    + ("; backward by torch autograd (BDH_ATTN_AUTOGRAD=0)" if cfg_id == 5 else "")
                    + "; value: the native line's flops over this time"}


# ------------------------------------------------------------------ config 4 decode
def decode_traffic(name: str, batch: int, s_mean: float):
    """Per-launch DRAM bytes of the decode kernels, scaled from a capture by batch x past length."""
    p = REPO / "profiles" / f"{name}.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return float(d["traffic_bytes_per_captured_launch"]) * (batch * s_mean) / (
            d["captured_batch"] * d["captured_past_len"])
    except Exception:  # noqa: BLE001
        return None


def bench_decode(args, world, rank, dev):
    import bdh_model
    from bdh_cache import CacheManager

    B, P = args.batch or 64, 512
    eager = getattr(args, "eager", False)
    cfg = bdh_model.BDHConfig(n_layer=N_LAYER, n_embd=D_MODEL, n_head=N_HEAD,
                              mlp_internal_dim_multiplier=128, vocab_size=VOCAB, dropout=0.0)
    torch.manual_seed(1004)
    model = bdh_model.BDH(cfg).to(dev).eval()
    model.attn._attn_impl_override = "eager" if eager else "cuda_sm100"
    steps_total = args.warmup + args.steps
    g = torch.Generator().manual_seed(rank_seed(2004, rank))
    toks = torch.randint(0, VOCAB, (B, P + steps_total), generator=g).to(dev)
    storage = (torch.float8_e4m3fn if args.decode_fp8 else
               torch.bfloat16 if args.decode_bf16 else None)
    kind = "state" if args.decode_state else "kv"
    cache = CacheManager.from_config(cfg, B, P + steps_total, dev, storage_dtype=storage,
                                     storage_kind=kind)
    buf = torch.empty(B, VOCAB, dtype=torch.float32, device=dev)
    with torch.inference_mode():
        model(toks[:, :P], cache=cache)
        pos = [P]

        def step():
            p = pos[0]
            model(toks[:, p:p + 1], cache=cache, logits_out=buf)
            pos[0] = p + 1

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        S0 = pos[0]
        clocks = ClockSampler(dev)
        clocks.start()
        profile_begin()
        ms = timed(step, args.steps, world, dev)
        prof = profile_end()
        clk = clocks.stop()
    S_mean = S0 + (args.steps - 1) / 2
    del cache
    if eager:
        return {"value": world * B * args.steps / (ms / 1e3), "unit": "tokens/s",
                "ms_per_step": ms / args.steps, "steps": args.steps, "warmup": args.warmup,
                "S_mean": S_mean, "clocks": clk,
                "what": "config-4 decode step (B=64, fp32 cache) with BDH_ATTN_IMPL=eager: the "
                        "reference's two-GEMM decode (kernels/attention.py:193-219) and torch "
                        "projections on this GPU"}
    if storage == torch.float8_e4m3fn:  # e4m3 keys + one fp32 scale per row, bf16 values
        bytes_step = N_LAYER * (B * N_HEAD * S_mean * (N_LAT + 4) + B * S_mean * D_MODEL * 2)
    else:
        esz = 2 if storage is not None else 4
        bytes_step = N_LAYER * (B * N_HEAD * S_mean * N_LAT * esz + B * S_mean * D_MODEL * esz)
    if kind == "state":
        # fp32 state read + written once per step for every row whose rotated query is nonzero;
        # counted at full density (an upper bound on the bytes moved, so GB/s is a lower bound)
        bytes_step = N_LAYER * 2 * B * N_HEAD * N_LAT * D_MODEL * 4
    dec = prof["decode"]
    peaks, src = load_peaks()
    gbs = bytes_step * args.steps / (dec["ms"] / 1e3) / 1e9 if dec["ms"] else None
    cpu = cpu_decode_baseline() if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    line = {
        "metric": "BDH decode tokens/s (config 4)", "value": world * B * args.steps / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if storage is not None else "f32",
        "cache_dtype": ("fp8 e4m3 keys (row scales) + bf16 values" if storage == torch.float8_e4m3fn
                        else "bf16" if storage is not None else "f32"), "cache_kind": kind,
        "data": "synthetic", "config": {"workload": "config 4 decode", "B": B, "prompt": P,
                                        "S_first": S0, "S_last": S0 + args.steps - 1,
                                        "S_mean": S_mean},
        "roofline": {"kernel": ("state decode (state_decode_kernel + state_reduce_kernel)" if kind == "state"
                                else "decode over e4m3 keys (decode_slice_kernel<..., uint8, ..., fp8> "
                                "+ decode_reduce_kernel)" if storage == torch.float8_e4m3fn
                                else "decode (decode_slice_kernel + decode_reduce_kernel)"),
                     "bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     # state mode skips the rows of zero rotated query, so the dense-equivalent
                     # rate can exceed the copy bandwidth: no fraction is claimed for it
                     "frac": (gbs / peaks["hbm_gbs"] if gbs else None) if kind == "kv" else None,
                     "bytes_counted": ("dense state, read + write (upper bound of bytes moved)"
                                       if kind == "state" else "history read once"),
                     "peak_source": f"{src} hbm_gbs",
                     "bytes_per_launch": bytes_step / N_LAYER,
                     "traffic": None if kind == "state" else decode_traffic(
                         "decode_config4_fp8" if storage == torch.float8_e4m3fn
                         else "decode_config4_bf16" if storage is not None
                         else "decode_config4", B, S_mean)},
        "kernel_ms": {k: v_["ms"] / args.steps for k, v_ in prof.items() if v_["launches"]},
        "gpu_launches": sum(v_["launches"] for v_ in prof.values()),
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


# ------------------------------------------------------------------- reference arm
def reference_arm(args, world, rank):
    if rank != 0:
        return None
    T = 512
    tok_s, kind, cores, sample = cpu_reference_model(1, T, max(1, args.steps))
    line = {
        "metric": "BDH prefill tokens/s (config 2: 6L, D=256, nh=4, N=8192, B=32, T=512)",
        "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * T / tok_s, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "BDH prefill forward on the host CPU (bounded sample of config 2)",
                   "seq_len": T},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="sm100", choices=["sm100", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-bf16", action="store_true")
    ap.add_argument("--decode-fp8", action="store_true",
                    help="config 4: e4m3 key cache with row scales, bf16 values (lossy, opt-in)")
    ap.add_argument("--decode-state", action="store_true",
                    help="config 4 with the N x D recurrent-state cache instead of the history")
    ap.add_argument("--batch", type=int, default=0,
                    help="per-GPU batch override (profiling aid; defaults: the config's own)")
    ap.add_argument("--global-batch", type=int, default=0,
                    help="config 2: shard this many sequences over the GPUs (strong scaling) "
                         "instead of 32 per GPU (weak scaling, the default)")
    ap.add_argument("--only", action="store_true",
                    help="config 2: the headline line alone (no other configs, eager baseline "
                         "or strong-scaling objects)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl != "reference":
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, dev = init_dist()
    try:
        if args.config == 2:
            line = bench_config2(args, world, rank, dev)
        elif args.config == 4:
            line = bench_decode(args, world, rank, dev)
        else:
            line = bench_op(args, world, rank, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
