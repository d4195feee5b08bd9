"""Benchmark of the KDN scan hot path on B200 (the BASELINE.json metric).

Step = one pass of the isotropic KDN hot path over one batch (config 1):
``iso_kdn_gain`` + ``_chunk_kda_precumsum_paired`` forward and backward at
B=4, T=4096, H=18, K=V=128, bf16 I/O with fp32 state, through the public
operators.  Inputs are synthetic (seeded, config-1 distributions) and larger
than L2 (about 0.5 GB per step), so no explicit L2 flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--variant iso|diag] [--impl ours|reference]

Under torchrun each rank runs its own batch of B=4 sequences (weak scaling,
no collective on the data path); timing is max over ranks.  The timed step
is captured once in a CUDA graph and replayed (``--eager`` times eager steps
instead; the JSON line carries both).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "kalman-delta-networks_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "KDN scan fwd+bwd Mtok/s/GPU (B4,T4096,H18,d128 bf16), % of roofline"
B, T, H, D = 4, 4096, 18, 128
# algorithmic (boundary) bytes per token-head, each tensor read or written once
ISO_BYTES_PER_TH = {"scan_fwd": 1540, "scan_bwd": 2824, "gain": 48}
DIAG_BYTES_PER_TH = {"scan_fwd": 2304, "scan_bwd": 4096, "gain_fwd": 2052, "gain_bwd": 3592}
FLOPS_PER_TH = 540_672  # 3 * 2 * (3 d^2 + 5 C d), C = 64
# DRAM bytes (read + write) per token-head of one kdn_scan_bwd call (reverse
# sweep + chunk kernel, + the gate fold for diag): ncu dram__bytes_read.sum +
# dram__bytes_write.sum of its kernels at B=1 T=4096 H=18, divided by its
# 73,728 token-heads (profiles/scan_bwd_*_traffic.md)
SCAN_BWD_TRAFFIC_PER_TH = {"iso": 5410, "diag": 7163}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons read through NVML (in-process, no child
    process) every ``period_ms`` by a background thread.

    ``start`` runs before the warm-up replays; ``summary`` keeps the samples
    taken from the first warm-up replay to the end of the timed region, one
    load throughout.  Reading clocks changes no GPU setting."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))

    def __init__(self, device: torch.device, period_ms: int = 10):
        self.device, self.period = device, period_ms / 1000.0
        self.samples = []  # (time.monotonic(), sm MHz, max sm MHz, reason bits)
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def _handle(self, nvml):
        props = torch.cuda.get_device_properties(self.device)
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            pci = f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:{getattr(props, 'pci_device_id', 0):02x}.0"
            try:
                return nvml.nvmlDeviceGetHandleByPciBusId(pci)
            except nvml.NVMLError:
                pass
        return nvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def start(self):
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            self._nvml = nvml
            handle = self._handle(nvml)
            mx = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
        except Exception:
            return self
        get_reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons

        def run():
            while not self._stop.is_set():
                try:
                    sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                    self.samples.append((time.monotonic(), sm, mx, get_reasons(handle)))
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self, t0: float, t1: float):
        rows = [r for r in self.samples if t0 <= r[0] <= t1]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        nvml = self._nvml
        reasons = sorted({name for r in rows for name, attr, bit in self.REASONS
                          if r[3] & getattr(nvml, attr, bit)})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(rows), "window": "warm-up replays + timed steps"}


# ----------------------------------------------------------------------------- inputs


def make_iso(device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    sp = torch.nn.functional.softplus
    x = {}
    x["q"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    x["k"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    x["v"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    log_alpha = -sp(torch.randn(B, T, H, D, generator=g, device=device))
    x["g_cumsum"] = (log_alpha.view(B, T // 64, 64, H, D).cumsum(2) * 1.4426950408889634).view(B, T, H, D).contiguous()
    x["a"] = torch.exp(2 * log_alpha).mean(-1)
    x["omega"] = sp(torch.randn(B, T, H, generator=g, device=device))
    x["r"] = 0.01 + sp(torch.randn(B, T, H, generator=g, device=device))
    x["prec"] = torch.ones(H, device=device)
    x["dO"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    return x


def make_diag(device, seed, B=None, T=None):
    B = globals()["B"] if B is None else B
    T = globals()["T"] if T is None else T
    g = torch.Generator(device=device).manual_seed(seed)
    sp = torch.nn.functional.softplus
    nrm = lambda t: t * torch.rsqrt((t * t).sum(-1, keepdim=True) + 1e-6)  # noqa: E731
    x = {}
    x["q"] = nrm(torch.randn(B, T, H, D, generator=g, device=device)).bfloat16()
    kk = nrm(torch.randn(B, T, H, D, generator=g, device=device))
    x["k"] = kk.bfloat16()
    x["k_gain"] = kk.float().contiguous()
    x["v"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    log_alpha = -sp(torch.randn(B, T, H, D, generator=g, device=device))
    x["alpha"] = torch.exp(log_alpha)
    x["g_cumsum"] = (log_alpha.view(B, T // 32, 32, H, D).cumsum(2) * 1.4426950408889634).view(B, T, H, D).contiguous()
    x["omega_raw"] = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    x["r_raw"] = torch.randn(B, T, H, generator=g, device=device).bfloat16()
    x["omega"] = sp(x["omega_raw"].float())
    x["r"] = 0.01 + sp(x["r_raw"].float())
    x["prec"] = torch.ones(H, device=device)
    x["dO"] = torch.randn(B, T, H, D, generator=g, device=device)
    return x


VARLEN_T = 131072  # config 4: sequences of lengths ~ U[256, 8192] packed to 131,072 tokens


def varlen_lengths(seed, total=VARLEN_T, lo=256, hi=8192):
    gen = torch.Generator().manual_seed(seed)
    lens = []
    while sum(lens) < total:
        lens.append(int(torch.randint(lo, hi + 1, (1,), generator=gen)))
    lens[-1] -= sum(lens) - total
    return lens


def make_diag_varlen(device, seed):
    """Config 4's packed batch: make_diag at B = 1, T = 131,072, with the
    gate prefix restarting every 32 tokens from each sequence's first token."""
    x = make_diag(device, seed)
    lens = varlen_lengths(seed)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    log_alpha = torch.log(x["alpha"])
    g = torch.empty_like(log_alpha)
    for a, b in zip(cu, cu[1:]):
        n = b - a
        pad = (-n) % 32
        la = torch.nn.functional.pad(log_alpha[:, a:b], (0, 0, 0, 0, 0, pad))
        g[:, a:b] = (la.view(1, (n + pad) // 32, 32, H, D).cumsum(2) * 1.4426950408889634).view(1, n + pad, H, D)[:, :n]
    x["g_cumsum"] = g.contiguous()
    x["cu"] = cu
    return x


def step_diag_varlen(x):
    from kdn_b200 import varlen

    L = leafify(x, ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "prec", "omega_raw", "r_raw"))
    kappa = varlen.diag_kdn_gain_varlen(L["k_gain"], L["alpha"], L["omega"], L["r"], L["prec"], L["omega_raw"],
                                        L["r_raw"], x["cu"])
    o = varlen.chunk_kalman_varlen(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5), x["cu"])
    o.backward(x["dO"])
    return L


def leafify(x, names):
    return {n: (x[n].detach().requires_grad_(True) if n in names else x[n]) for n in x}


def step_iso(x):
    from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, iso_kdn_gain

    L = leafify(x, ("q", "k", "v", "g_cumsum", "a", "omega", "r", "prec"))
    beta = iso_kdn_gain(L["a"], L["omega"], L["r"], L["prec"], head_dim=D, out_dtype=torch.float32)
    o = _chunk_kda_precumsum_paired(q=L["q"], k=L["k"], v=L["v"], g_cumsum=L["g_cumsum"], beta=beta)
    o.backward(x["dO"])
    return L


def step_diag(x):
    from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman

    L = leafify(x, ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "prec", "omega_raw", "r_raw"))
    kappa = _diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["prec"], L["omega_raw"], L["r_raw"])
    o = chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5))
    o.backward(x["dO"])
    return L


# initial_precision_param with 0.1 + softplus(.) = 1, the unit prior of make_iso / make_diag
UNIT_PRIOR_PARAM = math.log(math.expm1(0.9))


def make_iso_mixer(device, seed):
    """The isotropic mixer's own inputs to its kernels (lit_gpt/iso_kdn.py:
    277-304): q, k, v and the raw gate logits g_raw (bf16), the raw noise
    logits omega_r_raw (bf16 [B,T,2H]), the per-head parameters (fp32) and a
    bf16 output cotangent.  Zero A_log, dt_bias and noise biases make the
    frontend's outputs follow config 1's statistics: ln(alpha) =
    -softplus(N(0,1)) per channel, omega = softplus(N(0,1)), r = 0.01 +
    softplus(N(0,1)), unit prior."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    z = lambda *s: torch.zeros(*s, device=device)  # noqa: E731
    x = {"q": n(B, T, H, D).bfloat16(), "k": n(B, T, H, D).bfloat16(), "v": n(B, T, H, D).bfloat16(),
         "g_raw": n(B, T, H, D).bfloat16(), "omega_r_raw": n(B, T, 2 * H).bfloat16(),
         "omega_bias": z(H), "r_bias": z(H), "A_log": z(H), "dt_bias": z(H * D),
         "initial_precision_param": torch.full((H,), UNIT_PRIOR_PARAM, device=device), "dO": n(B, T, H, D).bfloat16()}
    return x


def step_iso_mixer(x):
    from kdn_b200.iso_kdn_chunk import _chunk_kda_precumsum_paired, _iso_kdn_gate_precumsum_paired, iso_kdn_gain

    L = leafify(x, MIXER_GRAD_NAMES["iso"])
    g_cumsum, a, omega, r, ip = _iso_kdn_gate_precumsum_paired(
        L["g_raw"], L["omega_r_raw"], L["omega_bias"], L["r_bias"], L["A_log"], L["dt_bias"],
        L["initial_precision_param"], 0.0, 0.01)
    beta = iso_kdn_gain(a, omega, r, ip, head_dim=D, out_dtype=torch.float32)
    o = _chunk_kda_precumsum_paired(q=L["q"], k=L["k"], v=L["v"], g_cumsum=g_cumsum, beta=beta)
    # the step's loss <o, dO>, whose gradient with respect to o is dO
    L[LOSS] = torch.dot(o.detach().float().flatten(), x["dO"].float().flatten())
    o.backward(x["dO"])
    return L


def make_diag_mixer(device, seed):
    """The diagonal mixer's own inputs to its kernels (lit_gpt/diag_kdn.py:
    315-345): raw q, k, v (bf16), the raw retention, process- and
    observation-noise logits (bf16), the per-head parameters (fp32) and a bf16
    output cotangent (the mixer casts the fp32 scan output to v's dtype).
    Zero A_log and dt_bias make the frontend's outputs follow config 2's
    statistics: ln(alpha) = -softplus(N(0,1)) per channel, q and k
    L2-normalised N(0,1), unit prior."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    x = {"q": n(B, T, H, D).bfloat16(), "k": n(B, T, H, D).bfloat16(), "v": n(B, T, H, D).bfloat16(),
         "retention_raw": n(B, T, H, D).bfloat16(), "omega_raw": n(B, T, H, D).bfloat16(),
         "r_raw": n(B, T, H).bfloat16(), "A_log": torch.zeros(H, device=device),
         "dt_bias": torch.zeros(H, D, device=device),
         "initial_precision_param": torch.full((H,), UNIT_PRIOR_PARAM, device=device), "dO": n(B, T, H, D).bfloat16()}
    return x


def step_diag_mixer(x):
    from kdn_b200.diag_kdn_chunk import (_diag_kdn_frontend_precumsum_paired, _diag_kdn_gain, _diag_kdn_normalize,
                                         chunk_kalman)

    L = leafify(x, MIXER_GRAD_NAMES["diag"])
    q_mem, k_gain, k_mem = _diag_kdn_normalize(L["q"], L["k"])
    g_cumsum, alpha, omega, r, ip = _diag_kdn_frontend_precumsum_paired(
        L["retention_raw"], L["omega_raw"], L["r_raw"], L["A_log"], L["dt_bias"], L["initial_precision_param"])
    kappa = _diag_kdn_gain(k_gain, alpha, omega, r, ip, L["omega_raw"], L["r_raw"])
    o = chunk_kalman(q_mem, k_mem, kappa, L["v"], g_cumsum, float(D ** -0.5)).to(torch.bfloat16)
    L[LOSS] = torch.dot(o.detach().float().flatten(), x["dO"].float().flatten())
    o.backward(x["dO"])
    return L


LOSS = "__loss__"  # the step result a mixer-level step leaves in its dict


MIXER_GRAD_NAMES = {"iso": ("q", "k", "v", "g_raw", "omega_r_raw", "omega_bias", "r_bias", "A_log", "dt_bias",
                            "initial_precision_param"),
                    "diag": ("q", "k", "v", "retention_raw", "omega_raw", "r_raw", "A_log", "dt_bias",
                             "initial_precision_param")}


GRAD_NAMES = {"iso": ("q", "k", "v", "g_cumsum", "a", "omega", "r"),
              "diag": ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega_raw", "r_raw")}
# iso: gain fwd (maps, apply), scan fwd (prep, fwd), scan bwd (state, chunk), gain bwd (maps, apply);
# diag: gain fwd (map, carry, emit), scan fwd (gate_to64, prep, fwd), scan bwd (state, chunk, gate_fold),
# gain bwd (map, carry, emit)
LAUNCHES_PER_STEP = {"iso": 8, "diag": 12}


def capture_step(step, x, device):
    """One step (forward + backward through the public operators) captured in
    a CUDA graph on a side stream, after two warm-up steps on that stream."""
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(2):
            step(x)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(x)
    torch.cuda.synchronize(device)
    return graph


def time_region(fn, steps, device):
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(stop) / steps


# algorithmic bytes per token-head of the isotropic gate frontend with bf16
# g_raw / omega_r_raw: fwd reads g_raw (2K) and omega_r_raw (4), writes
# g_cumsum (4K) and a, omega, r (12); bwd reads g_raw (2K), dg_pre (4K), da,
# domega, dr (12), omega_r_raw (4) and writes dg_raw (2K), domega_r_raw (4)
GATE_BYTES_PER_TH = {"fwd": 6 * D + 16, "bwd": 8 * D + 20}


def frontend_times(device, hbm, reps=20):
    """Device time of the isotropic gate frontend's C-ABI calls
    (kdn_iso_gate_fwd / kdn_iso_gate_bwd, the kernels behind
    _iso_kdn_gate_precumsum_paired) at the bench shape, bf16 g_raw and
    omega_r_raw, every buffer allocated up front; CUDA events on the launching
    stream.  Inputs (≈0.2 GB) are larger than L2."""
    from kdn_b200 import _native as N

    lib = N.load_library()
    g = torch.Generator(device=device).manual_seed(99)
    g_raw = torch.randn(B, T, H, D, generator=g, device=device).bfloat16()
    wr = torch.randn(B, T, 2 * H, generator=g, device=device).bfloat16()
    params = [torch.randn(n, generator=g, device=device) * 0.5 for n in (H, H, H, H * D, H)]
    f32 = dict(dtype=torch.float32, device=device)
    g_cumsum = torch.empty(B, T, H, D, **f32)
    a, omega, r = (torch.empty(B, T, H, **f32) for _ in range(3))
    ip = torch.empty(H, **f32)
    dg_pre = torch.randn(B, T, H, D, generator=g, device=device)
    da, dw, dr = (torch.randn(B, T, H, generator=g, device=device) for _ in range(3))
    dip = torch.randn(H, generator=g, device=device)
    dg_raw, dwr = torch.empty_like(g_raw), torch.empty_like(wr)
    pg = [torch.empty(n, **f32) for n in (H, H, H, H * D, H)]
    ws = N.byte_buffer(lib.kdn_iso_gate_workspace_bytes(B, T, H, D), device)
    stream = N.stream_of(g_raw)
    head = (g_raw.data_ptr(), 1, wr.data_ptr(), 1, wr.stride(0), wr.stride(1), *(t.data_ptr() for t in params))

    def fwd():
        N.check(lib.kdn_iso_gate_fwd(*head, g_cumsum.data_ptr(), a.data_ptr(), omega.data_ptr(), r.data_ptr(),
                                     ip.data_ptr(), B, T, H, D, 1e-3, 0.01, stream), "kdn_iso_gate_fwd")

    def bwd():
        N.check(lib.kdn_iso_gate_bwd(*head, dg_pre.data_ptr(), da.data_ptr(), dw.data_ptr(), dr.data_ptr(),
                                     dip.data_ptr(), dg_raw.data_ptr(), dwr.data_ptr(), *(t.data_ptr() for t in pg),
                                     B, T, H, D, ws.data_ptr(), ws.numel(), stream), "kdn_iso_gate_bwd")

    fwd()
    bwd()
    fms, bms = time_region(fwd, reps, device), time_region(bwd, reps, device)
    th = B * T * H
    fgb = GATE_BYTES_PER_TH["fwd"] * th / (fms * 1e-3) / 1e9
    bgb = GATE_BYTES_PER_TH["bwd"] * th / (bms * 1e-3) / 1e9
    return {"op": "_iso_kdn_gate_precumsum_paired (bf16 g_raw, omega_r_raw)", "fwd_ms": fms, "bwd_ms": bms,
            "bound": "hbm", "unit": "GB/s", "fwd_achieved": fgb, "bwd_achieved": bgb, "peak": hbm,
            "fwd_frac": fgb / hbm, "bwd_frac": bgb / hbm}


# algorithmic bytes per token-head of the diagonal frontend (bf16 inputs, f32
# outputs and cotangents): fwd reads retention_raw, omega_raw (2K each) and
# r_raw (2), writes g_cumsum, alpha, omega (4K each) and r (4); bwd reads
# retention_raw, omega_raw (2K each), r_raw (2), d_g_cumsum, d_alpha, d_omega
# (4K each) and d_r (4), writes dretention_raw, domega_raw (2K each) and
# dr_raw (2)
DIAG_GATE_BYTES_PER_TH = {"fwd": 16 * D + 6, "bwd": 20 * D + 8}


def diag_frontend_times(device, hbm, reps=20):
    """Device time of the diagonal frontend's C-ABI calls (kdn_diag_gate_fwd /
    kdn_diag_gate_bwd, the kernels behind _diag_kdn_frontend_precumsum_paired)
    at the bench shape with every cotangent present and every gradient asked
    for; buffers allocated up front; CUDA events on the launching stream.
    Inputs (≈0.4 GB) are larger than L2."""
    from kdn_b200 import _native as N

    lib = N.load_library()
    g = torch.Generator(device=device).manual_seed(98)
    bthk, bth = (B, T, H, D), (B, T, H)
    rn = lambda *s: torch.randn(*s, generator=g, device=device)  # noqa: E731
    ret, wraw, rraw = (rn(*bthk) * 2).bfloat16(), rn(*bthk).bfloat16(), rn(*bth).bfloat16()
    A_log = torch.log(torch.rand(H, generator=g, device=device) * 19 + 1)
    dt_bias, param = rn(H, D) * 0.5 - 4.0, rn(H)
    f32 = dict(dtype=torch.float32, device=device)
    outs = [torch.empty(*bthk, **f32) for _ in range(3)] + [torch.empty(*bth, **f32), torch.empty(H, **f32)]
    cots = [rn(*bthk) for _ in range(3)] + [rn(*bth), rn(H)]
    grads = [torch.empty_like(ret), torch.empty_like(wraw), torch.empty_like(rraw), torch.empty(H, **f32),
             torch.empty(H, D, **f32), torch.empty(H, **f32)]
    ws = N.byte_buffer(lib.kdn_diag_gate_workspace_bytes(B, T, H, D), device)
    stream = N.stream_of(ret)
    head = tuple(t.data_ptr() for t in (ret, wraw, rraw, A_log, dt_bias, param))

    def fwd():
        N.check(lib.kdn_diag_gate_fwd(*head, *(t.data_ptr() for t in outs), B, T, H, D, stream), "kdn_diag_gate_fwd")

    def bwd():
        N.check(lib.kdn_diag_gate_bwd(*head, *(t.data_ptr() for t in cots), *(t.data_ptr() for t in grads),
                                      B, T, H, D, ws.data_ptr(), ws.numel(), stream), "kdn_diag_gate_bwd")

    fwd()
    bwd()
    fms, bms = time_region(fwd, reps, device), time_region(bwd, reps, device)
    th = B * T * H
    fgb = DIAG_GATE_BYTES_PER_TH["fwd"] * th / (fms * 1e-3) / 1e9
    bgb = DIAG_GATE_BYTES_PER_TH["bwd"] * th / (bms * 1e-3) / 1e9
    return {"op": "_diag_kdn_frontend_precumsum_paired", "fwd_ms": fms, "bwd_ms": bms, "bound": "hbm",
            "unit": "GB/s", "fwd_achieved": fgb, "bwd_achieved": bgb, "peak": hbm, "fwd_frac": fgb / hbm,
            "bwd_frac": bgb / hbm}


# algorithmic bytes per token-head of the diagonal q / k normalisation (bf16
# q, k): fwd reads q, k (2K each), writes q_memory, k_memory (2K each),
# k_gain (4K) and the two norms (8); bwd reads q, k, the bf16 cotangents of
# q_memory and k_memory (2K each), the fp32 one of k_gain (4K) and the norms
# (8), writes dq, dk (2K each)
NORM_BYTES_PER_TH = {"fwd": 12 * D + 8, "bwd": 16 * D + 8}


def normalize_times(device, hbm, reps=20):
    """Device time of the diagonal normalisation's C-ABI calls
    (kdn_diag_norm_fwd / kdn_diag_norm_bwd, the kernels behind
    _diag_kdn_normalize) at the bench shape, bf16 q and k, every cotangent
    present; CUDA events on the launching stream."""
    from kdn_b200 import _native as N

    lib = N.load_library()
    g = torch.Generator(device=device).manual_seed(97)
    rn = lambda dt: torch.randn(B, T, H, D, generator=g, device=device).to(dt)  # noqa: E731
    q, k = rn(torch.bfloat16), rn(torch.bfloat16)
    qm, km, kg = torch.empty_like(q), torch.empty_like(k), torch.empty(B, T, H, D, device=device)
    qn, kn = torch.empty(B, T, H, device=device), torch.empty(B, T, H, device=device)
    dqm, dkg, dkm = rn(torch.bfloat16), rn(torch.float32), rn(torch.bfloat16)
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    rows, stream = B * T * H, N.stream_of(q)

    def fwd():
        N.check(lib.kdn_diag_norm_fwd(q.data_ptr(), k.data_ptr(), 1, qm.data_ptr(), kg.data_ptr(), km.data_ptr(),
                                      qn.data_ptr(), kn.data_ptr(), rows, D, stream), "kdn_diag_norm_fwd")

    def bwd():
        N.check(lib.kdn_diag_norm_bwd(q.data_ptr(), k.data_ptr(), 1, dqm.data_ptr(), dkg.data_ptr(), dkm.data_ptr(),
                                      qn.data_ptr(), kn.data_ptr(), dq.data_ptr(), dk.data_ptr(), rows, D, stream),
                "kdn_diag_norm_bwd")

    fwd()
    bwd()
    fms, bms = time_region(fwd, reps, device), time_region(bwd, reps, device)
    th = B * T * H
    fgb = NORM_BYTES_PER_TH["fwd"] * th / (fms * 1e-3) / 1e9
    bgb = NORM_BYTES_PER_TH["bwd"] * th / (bms * 1e-3) / 1e9
    return {"op": "_diag_kdn_normalize (bf16 q, k)", "fwd_ms": fms, "bwd_ms": bms, "bound": "hbm", "unit": "GB/s",
            "fwd_achieved": fgb, "bwd_achieved": bgb, "peak": hbm, "fwd_frac": fgb / hbm, "bwd_frac": bgb / hbm}


# algorithmic bytes per token-head of the gated output norm (bf16 o and gate,
# D = 128): fwd reads o, g (2D each), writes y (2D) and rstd (4); bwd reads o,
# g, dy (2D each) and rstd (4), writes do, dg (2D each)
ONORM_BYTES_PER_TH = {"fwd": 6 * D + 4, "bwd": 10 * D + 4}


def onorm_times(device, hbm, reps=20):
    """Device time of the gated output norm's C-ABI calls
    (kdn_rmsnorm_gated_fwd / _bwd, the kernels behind
    kdn_b200.norm_gated.FusedRMSNormGated, the mixers' o_norm) at the bench
    shape: one row per (b, t, h), bf16 o and gate, sigmoid gate, fp32 weight."""
    from kdn_b200 import _native as N

    lib = N.load_library()
    g = torch.Generator(device=device).manual_seed(96)
    rn = lambda: torch.randn(B, T, H, D, generator=g, device=device).bfloat16()  # noqa: E731
    x, gate, dy = rn(), rn(), rn()
    w = torch.ones(D, device=device)
    y, dx, dg = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    rows = B * T * H
    rstd, dw = torch.empty(rows, device=device), torch.empty(D, device=device)
    ws = N.byte_buffer(lib.kdn_rmsnorm_gated_workspace_bytes(rows, D), device)
    stream = N.stream_of(x)

    def fwd():
        N.check(lib.kdn_rmsnorm_gated_fwd(x.data_ptr(), 1, gate.data_ptr(), 1, w.data_ptr(), y.data_ptr(),
                                          rstd.data_ptr(), rows, D, 1e-5, 0, stream), "kdn_rmsnorm_gated_fwd")

    def bwd():
        N.check(lib.kdn_rmsnorm_gated_bwd(x.data_ptr(), 1, gate.data_ptr(), 1, w.data_ptr(), dy.data_ptr(),
                                          rstd.data_ptr(), dx.data_ptr(), dg.data_ptr(), dw.data_ptr(), rows, D, 0,
                                          ws.data_ptr(), ws.numel(), stream), "kdn_rmsnorm_gated_bwd")

    fwd()
    bwd()
    fms, bms = time_region(fwd, reps, device), time_region(bwd, reps, device)
    th = B * T * H
    fgb = ONORM_BYTES_PER_TH["fwd"] * th / (fms * 1e-3) / 1e9
    bgb = ONORM_BYTES_PER_TH["bwd"] * th / (bms * 1e-3) / 1e9
    return {"op": "FusedRMSNormGated (o_norm, bf16, sigmoid gate)", "fwd_ms": fms, "bwd_ms": bms, "bound": "hbm",
            "unit": "GB/s", "fwd_achieved": fgb, "bwd_achieved": bgb, "peak": hbm, "fwd_frac": fgb / hbm,
            "bwd_frac": bgb / hbm}


# algorithmic bytes per token-head of the packed q/k/v short convolution (bf16,
# 3 x 128 channels per head): fwd reads x (3 * 2D), writes q, k, v (3 * 2D);
# bwd reads x and dq, dk, dv (3 * 2D each), writes dx (3 * 2D)
CONV_BYTES_PER_TH = {"fwd": 12 * D, "bwd": 18 * D}


def conv_times(device, hbm, reps=20):
    """Device time of the short convolution's C-ABI calls (kdn_short_conv_fwd /
    _bwd, the kernels behind kdn_b200.short_conv.qkv_causal_conv1d) on the
    bench shape's packed projection output: x [B, T, 3 H D] bf16, fp32 weight."""
    import ctypes

    from kdn_b200 import _native as N

    lib = N.load_library()
    g = torch.Generator(device=device).manual_seed(95)
    C = 3 * H * D
    x = torch.randn(B, T, C, generator=g, device=device).bfloat16()
    w = torch.randn(C, 4, generator=g, device=device) * 0.5
    ys = [torch.empty(B, T, H * D, device=device, dtype=torch.bfloat16) for _ in range(3)]
    dys = [torch.randn(B, T, H * D, generator=g, device=device).bfloat16() for _ in range(3)]
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    ws = N.byte_buffer(lib.kdn_short_conv_workspace_bytes(B, T, C, 4), device)
    yp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in ys])
    dyp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in dys])
    stream = N.stream_of(x)

    def fwd():
        N.check(lib.kdn_short_conv_fwd(x.data_ptr(), 1, w.data_ptr(), 0, yp, 3, B, T, C, 4, 1, stream),
                "kdn_short_conv_fwd")

    def bwd():
        N.check(lib.kdn_short_conv_bwd(x.data_ptr(), 1, w.data_ptr(), 0, dyp, 3, dx.data_ptr(), dw.data_ptr(), B, T,
                                       C, 4, 1, ws.data_ptr(), ws.numel(), stream), "kdn_short_conv_bwd")

    fwd()
    bwd()
    fms, bms = time_region(fwd, reps, device), time_region(bwd, reps, device)
    th = B * T * H
    fgb = CONV_BYTES_PER_TH["fwd"] * th / (fms * 1e-3) / 1e9
    bgb = CONV_BYTES_PER_TH["bwd"] * th / (bms * 1e-3) / 1e9
    return {"op": "qkv_causal_conv1d (bf16 x, fp32 weight, SiLU)", "fwd_ms": fms, "bwd_ms": bms, "bound": "hbm",
            "unit": "GB/s", "fwd_achieved": fgb, "bwd_achieved": bgb, "peak": hbm, "fwd_frac": fgb / hbm,
            "bwd_frac": bgb / hbm}


def per_op_times(variant, x, device, reps=10):
    """Device time of the scan's two C-ABI calls, kdn_scan_fwd (chunk-record
    pass + sequential pass) and kdn_scan_bwd (reverse state sweep +
    chunk-parallel gradients), with every buffer allocated up front: CUDA
    events on the stream the kernels are launched on."""
    import ctypes

    from kdn_b200 import _native as N
    from kdn_b200 import _scan

    lib = N.load_library()
    if variant == "iso":
        from kdn_b200.iso_kdn_chunk import iso_kdn_gain

        gate = iso_kdn_gain(x["a"], x["omega"], x["r"], x["prec"], head_dim=D).detach()
        kind = N.KDN_ISO
    else:
        from kdn_b200.diag_kdn_chunk import _gain_forward

        gate = _gain_forward(x["k_gain"], x["alpha"], x["omega"], x["r"], x["prec"])[0]
        kind = N.KDN_DIAG
    q, k, v, g, dO = x["q"], x["k"], x["v"], x["g_cumsum"], x["dO"]
    a = _scan._args(kind, N.precision(), q, v, D ** -0.5)
    saved = N.byte_buffer(lib.kdn_scan_saved_bytes(ctypes.byref(a)), device)
    ws = N.byte_buffer(lib.kdn_scan_workspace_bytes(ctypes.byref(a)), device)
    o = torch.empty(v.shape, dtype=torch.bfloat16 if kind == N.KDN_ISO else torch.float32, device=device)
    dq, dk, dv, dg, dgate = (torch.empty_like(t) for t in (q, k, v, g, gate))
    a.q, a.k, a.v, a.g = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr()
    if kind == N.KDN_ISO:
        a.beta, a.dbeta = gate.data_ptr(), dgate.data_ptr()
    else:
        a.kappa, a.dkappa = gate.data_ptr(), dgate.data_ptr()
    a.o, a.saved, a.dO = o.data_ptr(), saved.data_ptr(), dO.data_ptr()
    a.dq, a.dk, a.dv, a.dg = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = N.stream_of(q)

    def fwd():
        N.check(lib.kdn_scan_fwd(ctypes.byref(a), stream), "kdn_scan_fwd")

    def bwd():
        N.check(lib.kdn_scan_bwd(ctypes.byref(a), stream), "kdn_scan_bwd")

    fwd()
    bwd()
    return {"scan_fwd_ms": time_region(fwd, reps, device), "scan_bwd_ms": time_region(bwd, reps, device)}


# ----------------------------------------------------------------------------- CPU baseline


def cpu_baseline(variant, seconds_budget=20.0, reference_naive=True):
    """The oracle (tokenwise PyTorch restatement of the reference recurrences,
    fp32, autograd backward) on the host cores: a B=1, H=2 slice of the
    workload, T grown until it takes a few seconds; tokens/s scaled to all 18
    heads by (b,h) independence."""
    import oracle

    threads = torch.get_num_threads()
    Tc = 256
    while True:
        t0 = time.perf_counter()
        if variant == "iso":
            d = oracle.make_iso_inputs(1, Tc, 2, seed=0)
            oracle.scan_grads("iso", {n: d[n] for n in ("q", "k", "v", "g_cumsum", "beta")}, d["dO"],
                              dtype=torch.float32)
            oracle.iso_gain_grads(d["a"], d["omega"], d["r"], torch.ones(2), torch.ones(1, Tc, 2), dtype=torch.float32)
        else:
            d = oracle.make_diag_inputs(1, Tc, 2, seed=0)
            kap, *_ = oracle.diag_gain_grads(d["k_gain"], d["alpha"], d["omega"], d["r"], d["initial_precision"],
                                             d["omega_raw"], d["r_raw"], torch.ones(1, Tc, 2, D), dtype=torch.float32)
            oracle.scan_grads("diag", {"q": d["q"], "k": d["k"], "kappa": kap.float(), "v": d["v"],
                                       "g_cumsum": d["g_cumsum"]}, d["dO"], scale=D ** -0.5, dtype=torch.float32)
        dt = time.perf_counter() - t0
        if dt > 2.0 or Tc >= T or dt * 2 > seconds_budget:
            break
        Tc *= 2
    token_heads_per_s = (Tc * 2) / dt
    mtok = token_heads_per_s / H / 1e6
    out = {"value": mtok, "unit": "Mtok/s", "cores": threads, "kind": "port",
           "sample": f"{variant} oracle fwd+bwd (fp32, autograd) on B=1,H=2,T={Tc}: {dt:.2f} s; "
                     f"scaled to H=18 by (b,h) independence"}
    if not reference_naive:
        return out
    try:
        out["reference_naive"] = reference_naive_cpu(variant, seconds_budget)
    except Exception as e:  # the reference's install is optional on a box
        out["reference_naive"] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
    return out


def reference_naive_cpu(variant, seconds_budget=20.0):
    """The reference's own chunked PyTorch oracle of the path
    (``_naive_chunk_iso_kdn``, lit_gpt/kdn_ops/iso_kdn_naive.py:536;
    ``_naive_chunk_diag_kdn``, diag_kdn_naive.py:658: gain and memory scans),
    loaded by path from the unmodified install under ``baseline/_ref``, forward
    plus autograd backward in fp32 on the host cores, on the same kind of
    B=1, H=2 slice as the port; tokens/s scaled to 18 heads."""
    mod = _load_reference_module("iso_kdn_naive" if variant == "iso" else "diag_kdn_naive")
    fn = mod._naive_chunk_iso_kdn if variant == "iso" else mod._naive_chunk_diag_kdn
    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(0)
    sp = torch.nn.functional.softplus
    nrm = lambda t: t * torch.rsqrt((t * t).sum(-1, keepdim=True) + 1e-6)  # noqa: E731
    Tc = 128
    while True:
        n = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
        x = {"q": nrm(n(1, Tc, 2, D)), "k": nrm(n(1, Tc, 2, D)), "v": n(1, Tc, 2, D),
             "alpha": torch.exp(-sp(n(1, Tc, 2, D))),
             "omega": sp(n(1, Tc, 2) if variant == "iso" else n(1, Tc, 2, D)), "r": 0.01 + sp(n(1, Tc, 2))}
        leaves = {k_: v_.requires_grad_(True) for k_, v_ in x.items()}
        dO = n(1, Tc, 2, D)
        t0 = time.perf_counter()
        o, _ = fn(leaves["q"], leaves["k"], leaves["v"], leaves["alpha"], leaves["omega"], leaves["r"],
                  chunk_size=64 if variant == "iso" else 32)
        o.backward(dO)
        dt = time.perf_counter() - t0
        if dt > 2.0 or Tc >= T or dt * 2 > seconds_budget:
            break
        Tc *= 2
    return {"value": Tc * 2 / dt / H / 1e6, "unit": "Mtok/s", "cores": threads, "kind": "reference",
            "sample": f"{variant} reference _naive_chunk_{variant}_kdn fwd + autograd bwd (fp32) on B=1,H=2,T={Tc}: "
                      f"{dt:.2f} s; scaled to H=18 by (b,h) independence"}


# ----------------------------------------------------------------------------- Triton reference point


def _load_reference_module(name):
    """The reference's own kdn_ops module, loaded by file path from the
    unmodified install under ``baseline/_ref`` (its package ``__init__`` needs
    the training stack, which is absent; the kdn_ops files need only torch,
    triton and flash-linear-attention utilities)."""
    import importlib.util

    path = os.path.join(ROOT, "baseline", "_ref", "lit_gpt", "kdn_ops", f"{name}.py")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} (install the reference into baseline/_ref)")
    spec = importlib.util.spec_from_file_location(f"_kdn_reference_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def o_error_vs_oracle(o, x, variant, stream=(0, 0)):
    """Normalised max-abs error of the forward output o on one (b, h) stream
    against the float64 oracle (gain + memory recurrence)."""
    import oracle

    b, h = stream
    sl = lambda t: t[b:b + 1, :, h:h + 1].detach().double().cpu()  # noqa: E731
    G = sl(x["g_cumsum"]) * oracle.LN2
    S0 = torch.zeros(1, 1, D, D, dtype=torch.float64)
    with torch.no_grad():
        if variant == "iso":
            beta, _, _ = oracle.iso_gain(sl(x["a"]), sl(x["omega"]), sl(x["r"]), x["prec"][h:h + 1].double().cpu())
            qh, kh = oracle.l2norm(sl(x["q"])), oracle.l2norm(sl(x["k"]))
            ref, _ = oracle.memory_recurrence(qh, kh, sl(x["v"]), oracle.alpha_from_g_cumsum(G, 64),
                                              beta[..., None] * kh, S0, D ** -0.5)
        else:
            kap, _ = oracle.diag_gain(sl(x["k_gain"]), sl(x["alpha"]), sl(x["omega"]), sl(x["r"]),
                                      x["prec"][h:h + 1].double().cpu())
            ref, _ = oracle.memory_recurrence(sl(x["q"]), sl(x["k"]), sl(x["v"]), oracle.alpha_from_g_cumsum(G, 32),
                                              kap, S0, D ** -0.5)
    got = sl(o)
    return ((got - ref).abs().max() / ref.abs().max()).item()


def triton_reference(device, x_diag, ours_diag_ms, steps=10, warmup=3):
    """The reference's own Triton kernels on this B200, through its stock
    kdn_ops entry points (``_diag_kdn_gain`` + ``chunk_kalman``,
    diag_kdn_chunk.py:2737, 3315; ``iso_kdn_gain`` +
    ``_chunk_kda_precumsum_paired``, iso_kdn_chunk.py:1966, 2242), on the
    bench's own inputs: eager fwd + bwd steps timed with CUDA events, and
    the forward output's error against the float64 oracle on one stream
    beside ours."""
    out = {}
    try:
        ref = _load_reference_module("diag_kdn_chunk")
        x = x_diag
        names = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "prec", "omega_raw", "r_raw")

        def step():
            L = leafify(x, names)
            kappa = ref._diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["prec"], L["omega_raw"],
                                       L["r_raw"])
            o = ref.chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5))
            o.backward(x["dO"])
            return o

        t0 = time.perf_counter()
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        compile_s = time.perf_counter() - t0
        ms = time_region(step, steps, device)
        with torch.no_grad():
            L = leafify(x, ())
            kappa = ref._diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["prec"], L["omega_raw"],
                                       L["r_raw"])
            o_ref = ref.chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5))
        from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman

        with torch.no_grad():
            o_ours = chunk_kalman(x["q"], x["k"], _diag_kdn_gain(x["k_gain"], x["alpha"], x["omega"], x["r"],
                                                                 x["prec"], x["omega_raw"], x["r_raw"]),
                                  x["v"], x["g_cumsum"], float(D ** -0.5))
        out["diag"] = {
            "what": "reference Triton _diag_kdn_gain + chunk_kalman, fwd + bwd, eager (config 2)",
            "ms_per_step": ms, "value": B * T / (ms * 1e-3) / 1e6, "unit": "Mtok/s",
            "warmup_incl_compile_s": compile_s,
            "ours_ms_per_step": ours_diag_ms, "ours_speedup": ms / ours_diag_ms if ours_diag_ms else None,
            "o_err_vs_oracle": o_error_vs_oracle(o_ref, x, "diag"),
            "ours_o_err_vs_oracle": o_error_vs_oracle(o_ours, x, "diag"),
            "err_stream": "(b, h) = (0, 0), normalised max-abs, float64 oracle",
        }
    except Exception as e:  # the reference point is reported, never required
        out["diag"] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"}
    try:
        ref_iso = _load_reference_module("iso_kdn_chunk")
        xi = make_iso(device, seed=4321)
        L = leafify(xi, ("q", "k", "v", "g_cumsum", "a", "omega", "r", "prec"))
        beta = ref_iso.iso_kdn_gain(L["a"], L["omega"], L["r"], L["prec"], head_dim=D, out_dtype=torch.float32)
        o = ref_iso._chunk_kda_precumsum_paired(q=L["q"], k=L["k"], v=L["v"], g_cumsum=L["g_cumsum"], beta=beta)
        o.backward(xi["dO"])
        torch.cuda.synchronize(device)
        out["iso"] = {"ran": True}
    except Exception as e:
        out["iso"] = {"unavailable": "unavailable on this box: the reference's iso scan calls flash-linear-"
                                     "attention at a pinned commit; the installed fla 0.5.1 fails with "
                                     f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"}
    return out


# ----------------------------------------------------------------------------- sequence parallelism (config 4)

SP_T = 131072  # config 4: one sequence of 131,072 tokens split contiguously over the ranks


def measure_sp(args, device, dist, world, rank, warmup):
    """Config 4 (diag, B=1, T=131,072, H=18): at N=1 the plain operators on
    the whole sequence; at N>1 each rank holds T/N contiguous tokens and runs
    the two-pass sequence-parallel scan (kdn_b200.sequence_parallel,
    all-gathers over NCCL).  Eager fwd + bwd steps, CUDA events, max over
    ranks.  Then a short case (T = 256 N, H = 2) checks the sequence-parallel
    outputs and gradients against the single-GPU call on the whole sequence,
    which every rank evaluates itself (max over ranks of the normalised
    max-abs difference)."""
    from kdn_b200.diag_kdn_chunk import _diag_kdn_gain, chunk_kalman
    from kdn_b200.sequence_parallel import sp_diag_kdn_two_pass

    Tr = SP_T // world
    names = ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "prec", "omega_raw", "r_raw")

    def step_of(x, sp):
        def step():
            L = leafify(x, names)
            if sp:
                o = sp_diag_kdn_two_pass(L["q"], L["k"], L["v"], L["g_cumsum"], L["k_gain"], L["alpha"], L["omega"],
                                         L["r"], L["prec"], L["omega_raw"], L["r_raw"])
            else:
                kappa = _diag_kdn_gain(L["k_gain"], L["alpha"], L["omega"], L["r"], L["prec"], L["omega_raw"],
                                       L["r_raw"])
                o = chunk_kalman(L["q"], L["k"], kappa, L["v"], L["g_cumsum"], float(D ** -0.5))
            o.backward(x["dO"])
            return L, o
        return step

    x = make_diag(device, seed=777 + rank, B=1, T=Tr)
    step = step_of(x, world > 1)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    steps = max(3, min(args.steps, 10))
    ms = time_region(step, steps, device)
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    rec = {"workload": f"diag_kdn gain+scan fwd+bwd B1 T{SP_T} H{H} d{D} (config 4), T split over {world} rank(s)",
           "mode": "two-pass sequence parallel (NCCL all-gather)" if world > 1 else "single GPU, whole sequence",
           "ms_per_step": ms, "value": SP_T / (ms * 1e-3) / 1e6, "unit": "Mtok/s", "n_gpus": world,
           "tokens_per_rank": Tr, "steps": steps, "timing": "eager"}
    del x
    if world > 1:
        Tc, Hc = 256 * world, 2
        full = make_diag(device, seed=99, B=1, T=Tc)  # the same seed on every rank: one sequence
        full = {n: (v[:, :, :Hc].contiguous() if isinstance(v, torch.Tensor) and v.dim() >= 3 else v)
                for n, v in full.items()}
        full["prec"] = full["prec"][:Hc].contiguous()
        Lf, of = step_of(full, False)()
        sl = slice(rank * 256, (rank + 1) * 256)
        part = {n: (v[:, sl].contiguous() if isinstance(v, torch.Tensor) and v.dim() >= 3 else v)
                for n, v in full.items()}
        Ls, os_ = step_of(part, True)()
        errs = {"o": (os_.detach(), of.detach()[:, sl])}
        for n in ("q", "k", "v", "g_cumsum", "k_gain", "alpha", "omega_raw", "r_raw"):
            errs["d" + n] = (Ls[n].grad, Lf[n].grad[:, sl])
        dprior = Ls["prec"].grad.clone()
        dist.all_reduce(dprior)
        errs["dprec"] = (dprior, Lf["prec"].grad)
        worst = {}
        for n, (a, b) in errs.items():
            a, b = a.double(), b.double()
            e = torch.tensor([((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()], device=device)
            dist.all_reduce(e, op=dist.ReduceOp.MAX)
            worst[n] = e.item()
        rec["check"] = {"case": f"B1 T{Tc} H{Hc}, 256 tokens per rank",
                        "max_norm_err_vs_single_gpu": worst, "max": max(worst.values())}
    return rec


# ----------------------------------------------------------------------------- full training step (config 3)


def measure_model(args, device, dist, world, rank, warmup, steps=5, name="iso_kdn_1.3B", bind=True):
    """Config 3: one training step of the reference's own iso_kdn_1.3B model
    (lit_gpt.model.GPT from the unmodified install in baseline/_ref: 18
    blocks of RMSNorm -> KDN mixer -> RMSNorm -> SwiGLU MLP, untied 32,000
    embedding and head) with kdn_b200's kernels bound in
    (kdn_b200.reference_binding): random-init fp32 weights under bf16
    autocast (the reference's bf16-mixed), uniform random token ids, micro
    batch 4 x 4096 per GPU, the reference's fused cross-entropy, backward and
    a fused AdamW step; data parallel over the ranks (DDP, NCCL all-reduce of
    the gradients).  CUDA events around the timed steps, max over ranks."""
    from functools import partial

    from kdn_b200.reference_binding import load_reference

    ref = load_reference(os.path.join(ROOT, "baseline", "_ref"), bind=bind)
    cfg = ref.config.Config.from_name(name)
    torch.manual_seed(0)
    with torch.device(device):
        model = ref.model.GPT(cfg)
    model.apply(partial(model._init_weights, n_layer=cfg.n_layer))
    n_params = sum(p.numel() for p in model.parameters())
    ddp = model
    if dist is not None:
        ddp = torch.nn.parallel.DistributedDataParallel(model, device_ids=[device.index])
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    loss_fn = ref.FusedCrossEntropyLoss()
    Bm, Tm = 4, cfg.block_size
    gen = torch.Generator(device=device).manual_seed(4242 + rank)
    tokens = torch.randint(0, cfg.vocab_size, (Bm, Tm + 1), generator=gen, device=device)
    inp, tgt = tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous()
    losses = []

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = ddp(inp)
            loss = loss_fn(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(loss.detach())

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    ms = time_region(step, steps, device)
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    loss_vals = [float(x) for x in losses]
    kernels = "kdn_b200 kernels bound in" if bind else "the reference's own Triton kernels"
    rec = {"workload": f"{name} training step (reference GPT, {kernels}), micro batch "
                       f"{Bm}x{Tm} per GPU, bf16 autocast, fused AdamW, DDP x{world}",
           "value": Bm * Tm * world / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "n_gpus": world,
           "params": n_params, "steps": steps, "timing": "eager", "loss_first": loss_vals[0],
           "loss_last": loss_vals[-1], "loss_finite": all(x == x and abs(x) < 1e4 for x in loss_vals)}
    del ddp, model, opt, tokens, inp, tgt
    torch.cuda.empty_cache()
    return rec


# ----------------------------------------------------------------------------- main


def bind_host_to_gpu(device):
    """Restrict this process to the CPU cores NVML reports as local to its GPU
    (the socket its PCIe root hangs off), so that the pinned host buffers of
    the end-to-end measurement are allocated on that node and its copies do
    not cross the socket interconnect, as `numactl --cpunodebind` does for a
    launcher.  Reads NVML only; changes no GPU setting.  Returns the number
    of cores kept, or None when NVML or the affinity call is unavailable."""
    try:
        import pynvml as nvml

        nvml.nvmlInit()
        handle = ClockSampler(device)._handle(nvml)
        words = nvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        cpus = {64 * w + bit for w, word in enumerate(words) for bit in range(64) if (int(word) >> bit) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:
        pass
    return None


def measure_e2e(step, x, names, args, device, dist, tokens, result="grads"):
    """End-to-end time of ``step`` through the public operators with host
    buffers: every step uploads its inputs ``x`` from pinned host memory and
    reads back its result: the gradients ``names`` (``result="grads"``) or
    the step's loss (``"loss"``: the gradients stay on the device, where a
    training step leaves them for its optimizer).  Uploads run on one copy
    stream and downloads on another, so the host link carries the next step's
    inputs and the previous step's results at once while the compute stream
    runs the step.  Max over ranks."""
    host = {n: (v.detach().cpu().pin_memory() if isinstance(v, torch.Tensor) else v) for n, v in x.items()}
    if result == "loss":
        names = (LOSS,)
        grads_host = {LOSS: torch.empty((), dtype=torch.float32).pin_memory()}
    else:
        grads_host = {n: torch.empty(x[n].shape, dtype=x[n].dtype).pin_memory() for n in names}
    h2d = sum(v.numel() * v.element_size() for v in host.values() if isinstance(v, torch.Tensor))
    d2h = sum(v.numel() * v.element_size() for v in grads_host.values())
    cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
    tens = [n for n, v in host.items() if isinstance(v, torch.Tensor)]
    bufs = [{n: torch.empty(host[n].shape, dtype=host[n].dtype, device=device) for n in tens} for _ in range(2)]

    def e2e_run(steps):
        main = torch.cuda.current_stream(device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev_in = [torch.cuda.Event(), torch.cuda.Event()]
        ev_done = [None, None]
        torch.cuda.synchronize(device)
        start.record(main)

        def upload(i):
            with torch.cuda.stream(cin):
                cin.wait_event(start)
                if ev_done[i % 2] is not None:  # step i - 2 is done with this buffer
                    cin.wait_event(ev_done[i % 2])
                for n in tens:
                    bufs[i % 2][n].copy_(host[n], non_blocking=True)
                ev_in[i % 2].record(cin)

        upload(0)
        for i in range(steps):
            if i + 1 < steps:
                upload(i + 1)
            main.wait_event(ev_in[i % 2])
            xd = dict(host)
            xd.update(bufs[i % 2])
            L = step(xd)
            ev_done[i % 2] = torch.cuda.Event()
            ev_done[i % 2].record(main)
            with torch.cuda.stream(cout):
                cout.wait_event(ev_done[i % 2])
                for n in names:
                    g = L[n] if n == LOSS else L[n].grad
                    g.record_stream(cout)
                    grads_host[n].copy_(g, non_blocking=True)
        main.wait_stream(cout)
        stop.record(main)
        torch.cuda.synchronize(device)
        return start.elapsed_time(stop) / steps

    # as many warm-up and timed steps as the main timing: the first uploads
    # from freshly pinned buffers ran up to twice as slow on a two-GPU box
    e2e_run(max(3, args.warmup))
    if dist is not None:
        dist.barrier()
    e2e_ms = e2e_run(max(3, args.steps))
    if dist is not None:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    return {"value": tokens / (e2e_ms * 1e-3) / 1e6, "unit": "Mtok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms}


def measure(variant, args, device, dist, world, rank, warmup, varlen=False):
    """Time one step of ``variant`` (device-resident inputs, CUDA graph
    replay, max over ranks), then its end-to-end step with host buffers, the
    per-call times and roofline of the dominant call, and the frontends."""
    if varlen:
        x, step = make_diag_varlen(device, seed=1234 + rank), step_diag_varlen
    else:
        x = (make_iso if variant == "iso" else make_diag)(device, seed=1234 + rank)
        step = step_iso if variant == "iso" else step_diag
    for _ in range(warmup):
        step(x)
    torch.cuda.synchronize(device)

    def barrier():
        if dist is not None:
            dist.barrier()

    # eager steps: every step pays the Python / autograd dispatch of the public operators
    barrier()
    eager_ms = time_region(lambda: step(x), args.steps, device)
    # the same step captured once in a CUDA graph and replayed, as a training
    # loop with graphs runs it: identical kernels and inputs, no host dispatch
    graph, timing = None, "eager"
    if not args.eager:
        try:
            graph = capture_step(step, x, device)
            timing = "cuda_graph"
        except Exception as e:  # the eager number stands if capture is unavailable
            print(f"bench: CUDA graph capture failed ({type(e).__name__}: {e}); timing eager steps", file=sys.stderr)
    run = graph.replay if graph is not None else (lambda: step(x))
    clk = ClockSampler(device).start()
    t_load = time.monotonic()
    for _ in range(warmup):
        run()
    barrier()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        run()
    stop.record()
    torch.cuda.synchronize(device)
    clocks = clk.summary(t_load, time.monotonic())
    clk.stop()
    barrier()
    ms = start.elapsed_time(stop) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    del graph

    tokens = B * T * world
    value = tokens / (ms * 1e-3) / 1e6
    hbm, tc, peak_kind = load_peaks()
    th = B * T * H

    # end to end through the public operators with host buffers: the mixer's
    # own inputs (raw q, k, v and gate / noise logits) through the frontends,
    # the gain and the scan, and, for reference, the scan's boundary inputs
    e2e = None
    if not args.no_e2e and not varlen:
        del x
        xm = (make_iso_mixer if variant == "iso" else make_diag_mixer)(device, seed=4321 + rank)
        mstep = step_iso_mixer if variant == "iso" else step_diag_mixer
        path = ("public operators from the mixer's raw inputs: " +
                ("_iso_kdn_gate_precumsum_paired -> iso_kdn_gain -> _chunk_kda_precumsum_paired"
                 if variant == "iso" else
                 "_diag_kdn_normalize, _diag_kdn_frontend_precumsum_paired -> _diag_kdn_gain -> chunk_kalman"))
        e2e = measure_e2e(mstep, xm, MIXER_GRAD_NAMES[variant], args, device, dist, tokens, result="loss")
        e2e["path"] = path + "; result read back: the loss <o, dO> (gradients stay on the device)"
        grads = measure_e2e(mstep, xm, MIXER_GRAD_NAMES[variant], args, device, dist, tokens)
        grads["path"] = path + "; result read back: every input gradient"
        e2e["gradients_read_back"] = grads
        del xm
        x = (make_iso if variant == "iso" else make_diag)(device, seed=1234 + rank)
        scan = measure_e2e(step, x, GRAD_NAMES[variant], args, device, dist, tokens)
        scan["path"] = "public gain + scan operators from the scan's boundary inputs (g_cumsum, gain inputs in fp32)"
        e2e["scan_inputs"] = scan

    per_th = ISO_BYTES_PER_TH if variant == "iso" else DIAG_BYTES_PER_TH
    step_bytes = sum(per_th.values()) * th
    if varlen:
        # the packed step (native: one call per operator over all sequences) is the unit
        achieved = step_bytes / (ms * 1e-3) / 1e9
        roofline = {"kernel": "whole varlen step (gain + scan, fwd + bwd, all sequences)", "bound": "hbm",
                    "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "peak_kind": peak_kind, "traffic": None, "step_frac": achieved / hbm}
    else:
        ops = per_op_times(variant, x, device)
        # dominant kernel call: the scan backward (reverse state sweep + chunk-parallel gradients)
        bwd_bytes = per_th["scan_bwd"] * th
        achieved = bwd_bytes / (ops["scan_bwd_ms"] * 1e-3) / 1e9
        traffic = SCAN_BWD_TRAFFIC_PER_TH.get(variant)
        roofline = {
            "kernel": "kdn_scan_bwd (scan_bwd_state + scan_bwd_chunk" + (")" if variant == "iso" else " + gate_fold)"),
            "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
            "peak_kind": peak_kind, "traffic": traffic and traffic * th,
            "step_frac": (step_bytes / (ms * 1e-3) / 1e9) / hbm,
            "op_ms": ops,
        }
    rec = {
        "value": value, "unit": "Mtok/s", "ms_per_step": ms, "timing": timing, "eager_ms_per_step": eager_ms,
        "config": {"workload": (f"diag_kdn gain+scan fwd+bwd, {len(x['cu']) - 1} packed sequences ~U[256,8192], "
                                f"T{T} H{H} d{D} (config 4 varlen)") if varlen
                   else f"iso_kdn gain+scan fwd+bwd B{B} T{T} H{H} d{D} (config 1)" if variant == "iso"
                   else f"diag_kdn gain+scan fwd+bwd B{B} T{T} H{H} d{D} (config 2)",
                   "global_batch": B * world, "seq_len": T, "heads": H, "head_dim": D,
                   "parallelism": f"batch-sharded x{world}", "l2": "inputs > L2 (no flush)"},
        "gpu_launches": LAUNCHES_PER_STEP[variant] * args.steps,
        "e2e": e2e, "roofline": roofline, "clocks": clocks,
    }
    if not varlen:
        rec["frontend"] = (frontend_times if variant == "iso" else diag_frontend_times)(device, hbm)
        if variant == "diag":
            rec["normalize"] = normalize_times(device, hbm)
        else:
            rec["o_norm"] = onorm_times(device, hbm)
            rec["short_conv"] = conv_times(device, hbm)
    return rec, x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--variant", choices=("iso", "diag"), default="iso")
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-diag", action="store_true", help="skip the config-2 (diag) sub-record of an iso run")
    ap.add_argument("--no-triton", action="store_true", help="skip the reference's Triton kernels")
    ap.add_argument("--no-sp", action="store_true", help="skip the config-4 sequence-parallel record")
    ap.add_argument("--no-varlen", action="store_true", help="skip the config-4 packed variable-length record")
    ap.add_argument("--no-model", action="store_true", help="skip the config-3 full training step record")
    ap.add_argument("--eager", action="store_true", help="time eager steps instead of a replayed CUDA graph")
    ap.add_argument("--varlen", action="store_true",
                    help="config 4 packed batch: diag, B=1, T=131072 of sequences ~U[256, 8192] (cu_seqlens)")
    ap.add_argument("--batch", type=int, default=B, help="sequences per GPU (profiling runs use smaller cases)")
    args = ap.parse_args()
    globals()["B"] = args.batch
    if args.varlen:
        args.variant = "diag"
        globals()["B"], globals()["T"] = 1, VARLEN_T
    warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        # torchrun sets OMP_NUM_THREADS=1 per rank; the CPU reference uses every host core
        torch.set_num_threads(os.cpu_count() or 1)
        runs = []
        for _ in range(warmup):
            cpu_baseline(args.variant, seconds_budget=5.0, reference_naive=False)
        for _ in range(args.steps):
            runs.append(cpu_baseline(args.variant, seconds_budget=10.0, reference_naive=False))
        val = statistics.mean(r["value"] for r in runs)
        cb = dict(runs[-1])
        cb["value"] = val
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": val, "unit": "Mtok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"{args.variant}_kdn gain+scan fwd+bwd, B1 H2 slice of B4 T4096 H18 d128"},
            "cpu_baseline": cb, "e2e": {"value": val, "unit": "Mtok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # one process per GPU: keep each rank's host side on its GPU's socket (at
    # N = 1 the process keeps every core, which the CPU baseline uses)
    host_cores = bind_host_to_gpu(device) if world > 1 else None

    rec, x = measure(args.variant, args, device, dist, world, rank, warmup, varlen=args.varlen)
    if rec["e2e"] is not None:
        rec["e2e"]["host_cores_bound"] = host_cores
    out = {"metric": METRIC, "value": rec["value"], "unit": "Mtok/s", "n_gpus": world, "steps": args.steps,
           "warmup": warmup, "ms_per_step": rec["ms_per_step"], "timing": rec["timing"],
           "eager_ms_per_step": rec["eager_ms_per_step"], "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": rec["config"],
           "gpu_launches": rec["gpu_launches"], "e2e": rec["e2e"], "roofline": rec["roofline"],
           "clocks": rec["clocks"]}
    for key in ("frontend", "o_norm", "short_conv", "normalize"):
        if key in rec:
            out[key] = rec[key]
    cpu = rank == 0 and world == 1 and not args.no_cpu and not args.varlen
    if cpu:
        out["cpu_baseline"] = cpu_baseline(args.variant)
    if args.variant == "iso" and not args.varlen and not args.no_diag:
        # config 2 (diagonal KDN) in the same run: its own step time, roofline,
        # end to end and CPU baseline
        del x
        drec, xd = measure("diag", args, device, dist, world, rank, warmup)
        drec["metric"] = "KDN scan fwd+bwd Mtok/s/GPU (diag, B4,T4096,H18,d128 bf16)"
        drec["n_gpus"] = world
        if cpu:
            drec["cpu_baseline"] = cpu_baseline("diag")
        out["diag"] = drec
        if rank == 0 and world == 1 and not args.no_triton:
            out["triton_reference"] = triton_reference(device, xd, drec["ms_per_step"])
        del xd
    if args.variant == "iso" and not args.varlen and not args.no_sp:
        out["sp"] = measure_sp(args, device, dist, world, rank, warmup)
    if args.variant == "iso" and not args.varlen and not args.no_varlen:
        # config 4's packed variant (31 sequences ~U[256, 8192], 131,072 tokens, diag), per rank
        saved_bt = globals()["B"], globals()["T"]
        globals()["B"], globals()["T"] = 1, VARLEN_T
        no_e2e, args.no_e2e = args.no_e2e, True
        try:
            vrec, _ = measure("diag", args, device, dist, world, rank, warmup, varlen=True)
        finally:
            globals()["B"], globals()["T"] = saved_bt
            args.no_e2e = no_e2e
        out["varlen"] = {k: vrec[k] for k in ("value", "unit", "ms_per_step", "timing", "config", "gpu_launches",
                                              "roofline", "clocks")}
    if args.variant == "iso" and not args.varlen and not args.no_model:
        # config 3: the reference's model trained on our kernels; at one GPU also
        # the diagonal model on the reference's own kernels (its iso scan cannot
        # run on this box's flash-linear-attention, see triton_reference)
        out["model"] = {}
        runs = [("iso_kdn_1.3B", True), ("diag_kdn_1.3B", True)]
        if world == 1 and not args.no_triton:
            runs.append(("diag_kdn_1.3B", False))
        for name, bind in runs:
            key = name if bind else name + " (reference kernels)"
            try:
                out["model"][key] = measure_model(args, device, dist, world, rank, warmup=3, name=name, bind=bind)
            except Exception as e:  # reported, never fatal to the line
                out["model"][key] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"}
        ours_d, ref_d = out["model"].get("diag_kdn_1.3B", {}), out["model"].get("diag_kdn_1.3B (reference kernels)", {})
        if "ms_per_step" in ours_d and "ms_per_step" in ref_d:
            out["model"]["diag_speedup_vs_reference_kernels"] = ref_d["ms_per_step"] / ours_d["ms_per_step"]
    if rank == 0:
        print(json.dumps(out))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
