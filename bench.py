#!/usr/bin/env python
"""Benchmark of the B200 attention / delta-rule path (one JSON line on rank 0).

Headline workload: causal GQA prefill, bf16 in / fp32
accumulate, batch 1, seq 4096, 32 query heads, 8 KV heads, head_dim 128, RoPE
pre-applied, K/V written to the device cache.  One step = append the 4096 K/V
rows into a fresh cache + attention of the 4096 query rows (137.47 GFLOP).
`value` is TFLOP/s of that step with inputs resident in HBM; `e2e` is the same
through the C ABI with host (pinned) inputs and outputs copied inside the
timed region, every step's copies included, pipelined over three streams the
way a serving loop runs (step i + 1's inputs cross PCIe while step i
computes and step i - 1's rows come back).

At N GPUs (torchrun) each rank owns hkv/N KV heads (and their query heads);
the attention epilogue stores the rank's heads of every output row into all
ranks' row buffers over NVLink and a stream-ordered barrier closes the step,
so each GPU holds the reference's [row][head*dim] rows: total work is fixed
("strong").  The line also times the unfused alternative (attention, NCCL
all-gather, permutation) for comparison.

Measured extras at N=1 (their own units, each with a roofline fraction):
config 1 fp32 decode, config 3 delta-rule prefill + 256 decode steps,
config 4 Gemma hybrid prefill (5 local + 1 global layer) and batch-16 decode,
config 5 ragged batch-64 long-context f16 decode.

`--impl reference` times the reference engine's own CPU code (oracle/_ref,
its headers compiled here; the C restatement in oracle/ if that library is
absent) on a bounded sample of the same workload with every host core.
"""
import argparse
import ctypes
import json
import math
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn GB/s, prefill TFLOP/s (% roofline); tok/s at 1/2/4/8 B200"
S2, HQ2, HKV2, DH2 = 4096, 32, 8, 128
L2_BYTES = 126 * 2**20


def c2_flops(S=S2, hq=HQ2, dh=DH2):
    return 4.0 * dh * hq * (S * (S + 1) // 2)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return {"hbm": float(p["hbm_gbs"]), "bf16": float(p["bf16_tflops"]),
                "bf16_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "src": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "src": "fallback"}


_RATES = {}


def tensor_rates():
    """tf32 and bf16 tcgen05 rates from an issue loop on every SM
    (hero_b200/libnmg_rate.so: back-to-back M = 128 x N = 128 MMAs into one
    TMEM accumulator, cycles per MMA and the SM clock measured in the kernel).
    The tf32 roofline peak is the measured bf16 peak (MEASURED_PEAKS.json)
    times the issue loop's tf32 / bf16 FLOP-per-cycle ratio.  Measured once per
    process; None where the probe library or a GPU is missing."""
    if "r" in _RATES:
        return _RATES["r"]
    out = None
    try:
        import ctypes

        lib = ctypes.CDLL(os.path.join(ROOT, "hero_b200", "libnmg_rate.so"))
        fn = lib.nmg_rate_tensor
        fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int)]
        res = {}
        for kind, name, kdim in ((0, "tf32", 8), (1, "bf16", 16)):
            cyc, ghz, sms = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
            if fn(kind, 128, 4096, ctypes.byref(cyc), ctypes.byref(ghz), ctypes.byref(sms)) != 0:
                raise RuntimeError("rate probe failed")
            flop = 2.0 * 128 * 128 * kdim
            res[name] = {"cycles_per_mma": cyc.value, "sm_ghz": ghz.value,
                         "tflops": flop / cyc.value * ghz.value * 1e9 * sms.value / 1e12}
        ratio = (2.0 * 128 * 128 * 8 / res["tf32"]["cycles_per_mma"]) / (2.0 * 128 * 128 * 16 / res["bf16"]["cycles_per_mma"])
        out = {"issue_loop": res, "tf32_over_bf16": ratio, "tf32_peak": peaks()["bf16"] * ratio,
               "method": "tcgen05 issue loop, M=128 N=128, one CTA per SM (hero_b200/csrc/tensor_rate.cu)"}
    except Exception as e:  # no GPU or no probe library: the caller falls back and says so
        out = None
    _RATES["r"] = out
    return out


def tf32_peak_and_note():
    r = tensor_rates()
    if r:
        return r["tf32_peak"], (f"tf32 peak = measured bf16 peak x {r['tf32_over_bf16']:.3f}, the tf32/bf16 "
                                f"FLOP-per-cycle ratio of a tcgen05 issue loop (M=128, N=128)")
    return peaks()["bf16"] / 2, "tf32 peak taken as half the measured bf16 peak (issue-loop probe unavailable)"


def imma_rate():
    """The warp-level int8 MMA issue rate (mma.sync m16n8k32, 16 warps per SM,
    register operands; hero_b200/libnmg_rate.so) in TOPS, the ceiling of the
    projection GEMM's instruction; None without the probe library or a GPU."""
    if "imma" in _RATES:
        return _RATES["imma"]
    out = None
    try:
        import ctypes

        lib = ctypes.CDLL(os.path.join(ROOT, "hero_b200", "libnmg_rate.so"))
        lib.nmg_rate_imma.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        t = ctypes.c_double()
        if lib.nmg_rate_imma(2048, ctypes.byref(t)) == 0:
            out = t.value
    except Exception:
        out = None
    _RATES["imma"] = out
    return out


def ncu_traffic(name):
    """DRAM bytes per launch of a workload's dominant kernel from profiles/traffic.json, or None."""
    try:
        return float(json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))[name]["dram_bytes_per_launch"])
    except (OSError, KeyError, TypeError, ValueError):
        return None


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clocks and clock-event reasons sampled while the timed region runs.

    NVML (read-only queries) from a background thread every ~2 ms; nvidia-smi
    at 200 ms when NVML is unavailable.  Nothing here changes a GPU setting."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.thread = None
        self.rows = []  # (sm_mhz, max_mhz, set of reason names)
        self.err = None
        self.path = os.path.join("/tmp", f"nmg_clocks_{os.getpid()}.csv")

    def _nvml_loop(self, nv, h, stop):
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(smax), {n for n, b in bits.items() if r & b}))
            except Exception as e:
                self.err = f"{type(e).__name__}: {e}"
                break
            stop.wait(0.002)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(int(self.gpu_id))
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h, self.stop), daemon=True)
            self.thread.start()
            time.sleep(0.01)
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=2)
            if not self.rows:  # a region shorter than the thread's first wake-up: sample once more now
                try:
                    import pynvml as nv
                    h = nv.nvmlDeviceGetHandleByIndex(int(self.gpu_id))
                    self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                      float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)), set()))
                except Exception as e:
                    self.err = self.err or f"{type(e).__name__}: {e}"
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = list(self.rows)
        src = "nvml"
        if not rows:
            src = "nvidia-smi"
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            try:
                for line in open(self.path):
                    p = [x.strip() for x in line.split(",")]
                    if len(p) >= 9 and p[1].replace(".", "").isdigit() and p[2].replace(".", "").isdigit():
                        rows.append((float(p[1]), float(p[2]),
                                     {names[i] for i in range(4) if p[5 + i].lower().startswith("active")}))
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0, "error": self.err}
        sm = [r[0] for r in rows]
        smax = max(r[1] for r in rows)
        loaded = [x for x in sm if x > 0.5 * smax] or sm
        reasons = sorted(set().union(*[r[2] for r in rows]))
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows),
                "source": src}


def gpu_smi_id(torch, dev):
    """nvidia-smi's index for this process's device (CUDA_VISIBLE_DEVICES-aware)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if vis:
        ids = [x.strip() for x in vis.split(",")]
        if dev.index < len(ids) and ids[dev.index].isdigit():
            return ids[dev.index]
    return str(dev.index)


# ---------------------------------------------------------------- CPU baseline

class RefSample:
    """The reference reduction on a bounded sample of config 2, timed on the host.

    Inputs are generated once; `run()` times the reduction only (the cache is
    filled untimed inside the reference shim) and returns seconds."""

    def __init__(self, rows_per_block=256, threads=None, full=False):
        import oracle

        self.threads = threads or os.cpu_count() or 1
        os.environ.setdefault("NM_THREADS", str(self.threads))
        S, hq, hkv, dh = S2, HQ2, HKV2, DH2
        self.q = oracle.round_bf16(oracle.normal(0, 3, S * hq * dh)).reshape(S, hq * dh)
        self.k = oracle.round_bf16(oracle.normal(0, 1, S * hkv * dh)).reshape(S, hkv * dh)
        self.v = oracle.round_bf16(oracle.normal(0, 2, S * hkv * dh)).reshape(S, hkv * dh)
        if full:  # every query row: the whole config-2 workload
            self.blocks = np.array([0, S, S, 0], np.int64)
            self.nblocks = 1
            self.flops = c2_flops()
        else:
            self.blocks = np.array([S // 2 - rows_per_block // 2, rows_per_block, S - rows_per_block, rows_per_block],
                                   np.int64)
            self.nblocks = 2
            self.flops = c2_sample_flops(rows_per_block)
        self.out = np.zeros_like(self.q)
        self.scale = np.float32(1 / math.sqrt(dh))
        self.R = oracle.ref()
        self.oracle = oracle
        if self.R is not None:
            self.kind = "reference"
            self.R.nmref_prefill_sample.argtypes = [
                ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_int64,
                ctypes.c_void_p, ctypes.POINTER(ctypes.c_double)]
            self.cores = int(self.R.nmref_threads())
        else:
            self.kind = "port"
            self.cores = self.threads
        b = self.blocks
        if full:
            self.sample = (f"all 4096 query rows of the S=4096 32q/8kv/d128 causal prefill "
                           f"({self.flops / 1e9:.1f} GFLOP), reduction only, {self.cores} threads")
        else:
            self.sample = (f"query rows [{b[0]},{b[0] + b[1]}) and [{b[2]},{S2}) of the S=4096 32q/8kv/d128 causal "
                           f"prefill ({self.flops / 1e9:.1f} GFLOP), reduction only, {self.cores} threads")

    def run(self):
        if self.R is not None:
            sec = ctypes.c_double()
            st = self.R.nmref_prefill_sample(HKV2, DH2, self.k.ctypes.data, self.v.ctypes.data, S2, self.q.ctypes.data,
                                             HQ2, self.blocks.ctypes.data, self.nblocks, self.scale, 1, 0, self.out.ctypes.data,
                                             ctypes.byref(sec))
            if st != 0:
                raise RuntimeError(f"reference sample failed ({st})")
            return sec.value
        total = 0.0
        for b in range(self.nblocks):
            s0, n = int(self.blocks[2 * b]), int(self.blocks[2 * b + 1])
            t0 = time.perf_counter()
            self.oracle.attend(self.k[:s0 + n], self.v[:s0 + n], 0, 0, HKV2, DH2, self.q[s0:s0 + n], HQ2, s0,
                               scale=self.scale, threads=self.threads)
            total += time.perf_counter() - t0
        return total


class RefConfigs:
    """The reference's own code (oracle/_ref) on bounded samples of configs 1,
    3, 4 and 5, timed on the host in the units of the GPU numbers they sit
    beside; the C restatement (oracle/) stands in where the reference library
    was not built.  Inputs are seeded N(0,1) rows of each configuration's
    shapes; every timed region covers the reduction (or recurrence) only."""

    def __init__(self, min_seconds=0.5):
        import oracle

        self.oracle = oracle
        self.threads = os.cpu_count() or 1
        os.environ.setdefault("NM_THREADS", str(self.threads))
        self.min_seconds = min_seconds
        self.R = oracle.ref()
        if self.R is not None:
            c_int, c_i64, c_f, c_p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
            self.R.nmref_decode_sample.argtypes = [c_int, c_int, c_p, c_p, c_i64, c_p, c_int, c_f, c_int, c_i64, c_i64,
                                                   c_p, ctypes.POINTER(ctypes.c_double)]
            self.R.nmref_prefill_sample.argtypes = [c_int, c_int, c_p, c_p, c_i64, c_p, c_int, c_p, c_i64, c_f, c_int,
                                                    c_i64, c_p, ctypes.POINTER(ctypes.c_double)]
            self.R.nmref_delta_timed.argtypes = [c_int, c_int, c_int, c_p, c_i64, c_int, c_p, c_p, c_p, c_p, c_p, c_p,
                                                 ctypes.POINTER(ctypes.c_double)]
            self.kind, self.cores = "reference", int(self.R.nmref_threads())
        else:
            self.kind, self.cores = "port", self.threads

    def _rows(self, seed, stream, rows, width):
        return self.oracle.normal(seed, stream, rows * width).reshape(rows, width)

    def decode_seconds(self, k, v, q, hkv, dh, hq, scale, window):
        """Seconds per reduction of one query at the newest of k's rows: one
        call to size the sample, then one of about min_seconds (each call
        fills its cache untimed, so calls are few)."""
        rows = k.shape[0]
        reps = 1
        for attempt in range(2):
            if self.R is not None:
                out = np.zeros(hq * dh, np.float32)
                sec = ctypes.c_double()
                st = self.R.nmref_decode_sample(hkv, dh, k.ctypes.data, v.ctypes.data, rows, q.ctypes.data, hq,
                                                float(scale or 1.0), 0 if scale is None else 1, window, reps,
                                                out.ctypes.data, ctypes.byref(sec))
                if st != 0:
                    raise RuntimeError(f"reference decode sample failed ({st})")
                total = sec.value
            else:
                kw = dict(use_scale=False) if scale is None else dict(scale=np.float32(scale))
                t0 = time.perf_counter()
                for _ in range(reps):
                    self.oracle.attend(k, v, 0, window, hkv, dh, q.reshape(1, -1), hq, rows - 1, threads=self.threads,
                                       **kw)
                total = time.perf_counter() - t0
            if total >= self.min_seconds or reps >= 4096 or attempt == 1:
                return total / reps
            reps = int(min(4096, max(2, math.ceil(self.min_seconds / max(total, 1e-6)))))

    def prefill_seconds(self, k, v, q, hkv, dh, hq, scale, window, start, n):
        """Seconds to reduce query rows [start, start + n) over the causal prefix of k's rows."""
        if self.R is not None:
            out = np.zeros_like(q)
            sec = ctypes.c_double()
            blocks = np.array([start, n], np.int64)
            st = self.R.nmref_prefill_sample(hkv, dh, k.ctypes.data, v.ctypes.data, k.shape[0], q.ctypes.data, hq,
                                             blocks.ctypes.data, 1, float(scale or 1.0), 0 if scale is None else 1,
                                             window, out.ctypes.data, ctypes.byref(sec))
            if st != 0:
                raise RuntimeError(f"reference prefill sample failed ({st})")
            return sec.value
        kw = dict(use_scale=False) if scale is None else dict(scale=np.float32(scale))
        t0 = time.perf_counter()
        self.oracle.attend(k[:start + n], v[:start + n], 0, window, hkv, dh, q[start:start + n], hq, start,
                           threads=self.threads, **kw)
        return time.perf_counter() - t0

    def line(self, value, unit, sample, cores=None):
        return {"value": value, "unit": unit, "cores": cores or self.cores, "kind": self.kind, "sample": sample}

    def projections(self):
        """The oracle's restatement of Weight::matvec / matmul (the reference
        library instantiates no model-sized Weight), on all host threads: one
        token through a layer's six projections, and 16 rows through them."""
        from oracle import quant as Q

        ws = [(gt, n, o, synthetic_gguf(gt, o, n, i)) for i, (_, gt, n, o) in enumerate(PROJ_LAYER)]
        wbytes = sum(w.size for *_, w in ws)
        x = {n: self._rows(12, 1, 16, n) for n in (4096, 12288)}

        def run(rows):
            t = time.perf_counter()
            for gt, n, o, w in ws:
                Q.matmul(gt, w, x[n][:rows], threads=self.threads)
            return time.perf_counter() - t

        run(1)
        secs = [run(1) for _ in range(3)]
        dec = float(np.median(secs))
        pre = run(16)
        ops = 2.0 * 16 * sum(n * o for _, n, o, _ in ws)
        return {"decode": {**self.line(wbytes / dec / 1e9, "GB/s", f"one token through the 6 projections, "
                                       f"{dec * 1e3:.1f} ms", cores=self.threads), "kind": "port"},
                "prefill": {**self.line(ops / pre / 1e12, "TOPS", f"16 rows through the 6 projections, "
                                        f"{pre * 1e3:.0f} ms", cores=self.threads), "kind": "port"}}

    def config1(self):
        hq, hkv, dh, L = 16, 8, 128, 1024
        k, v = self._rows(101, 1, L, hkv * dh), self._rows(101, 2, L, hkv * dh)
        q = self._rows(101, 3, 1, hq * dh)
        sec = self.decode_seconds(k, v, q, hkv, dh, hq, 1 / math.sqrt(dh), 0)
        bytes_ = 2 * L * hkv * dh * 4 + 2 * hq * dh * 4
        return self.line(bytes_ / sec / 1e9, "GB/s",
                         f"config 1 decode (fp32 cache of 1024 rows), {sec * 1e6:.0f} us per call, reduction only")

    def config3(self):
        hv, hk, d, T = 32, 16, 128, 256
        o = self.oracle
        q = o.l2_normalize(self._rows(103, 1, T * hk, d).reshape(T, hk, d)) * np.float32(1 / math.sqrt(d))
        k = o.l2_normalize(self._rows(103, 2, T * hk, d).reshape(T, hk, d))
        v = self._rows(103, 3, T * hv, d).reshape(T, hv, d)
        g = (-np.log1p(np.exp(o.normal(103, 4, T * hv).astype(np.float64)))).astype(np.float32).reshape(T, hv)
        b = (1 / (1 + np.exp(-o.normal(103, 5, T * hv).astype(np.float64)))).astype(np.float32).reshape(T, hv)
        q, k = np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32)
        state = np.zeros((hv, d, d), np.float32)
        out = np.zeros((T, hv, d), np.float32)
        if self.R is not None:
            sec = ctypes.c_double()
            st = self.R.nmref_delta_timed(hv, d, d, state.ctypes.data, T, hk, q.ctypes.data, k.ctypes.data,
                                          v.ctypes.data, g.ctypes.data, b.ctypes.data, out.ctypes.data,
                                          ctypes.byref(sec))
            if st != 0:
                raise RuntimeError(f"reference delta sample failed ({st})")
            total = sec.value
        else:
            t0 = time.perf_counter()
            o.delta_run(state, q, k, v, g, b, hk)
            total = time.perf_counter() - t0
        per_tok = total / T
        step_bytes = 2 * hv * d * d * 4 + 2 * hk * d * 4 + 2 * hv * d * 4 + 2 * hv * 4
        sample = (f"{T} tokens of the 32-value-head recurrence (the reference runs it token by token on one thread: "
                  f"{per_tok * 1e6:.0f} us per token)")
        return {"prefill": self.line(1 / per_tok, "tok/s", sample, cores=1),
                "decode": self.line(step_bytes / per_tok / 1e9, "GB/s", sample, cores=1)}

    def config4(self):
        hq, hkv, dh, W, S = 8, 4, 256, 1024, 8192
        def rms(x):  # per-head RMS norm, unit gain (the configuration's QK-RMSNorm)
            h = x.reshape(-1, dh)
            return (h / np.sqrt(np.einsum("ij,ij->i", h, h)[:, None] / np.float32(dh) + np.float32(1e-6))).reshape(x.shape)

        k, v = rms(self._rows(104, 1, S, hkv * dh)), self._rows(104, 2, S, hkv * dh)
        q = rms(self._rows(104, 3, S, hq * dh))
        n = 32  # the last 32 query rows: global layer (all earlier keys) and a local layer (1024)
        sg = self.prefill_seconds(k, v, q, hkv, dh, hq, None, 0, S - n, n)
        sl = self.prefill_seconds(k, v, q, hkv, dh, hq, None, W, S - n, n)
        pairs_g = sum(r + 1 for r in range(S - n, S))
        flops = 4.0 * dh * hq * (pairs_g + 5 * n * W)
        res = {"prefill": self.line(flops / (sg + 5 * sl) / 1e12, "TFLOP/s",
                                    f"config 4 prefill rows [{S - n}, {S}) of one global and five local (W=1024) "
                                    "layers, reduction only")}
        L = 32768
        kd, vd = rms(self._rows(104, 4, L, hkv * dh)), self._rows(104, 5, L, hkv * dh)
        qd = rms(self._rows(104, 6, 1, hq * dh))
        dg = self.decode_seconds(kd, vd, qd, hkv, dh, hq, None, 0)
        dl = self.decode_seconds(kd, vd, qd, hkv, dh, hq, None, W)
        bytes_ = L * hkv * dh * 4 * 2 + 5 * W * hkv * dh * 4 * 2
        res["decode"] = self.line(bytes_ / (dg + 5 * dl) / 1e9, "GB/s",
                                  "config 4 decode of one sequence (32768 fp32 rows: one global + five local layers), "
                                  f"{(dg + 5 * dl) * 1e3:.2f} ms per token per 6-layer group")
        return res

    def config5(self):
        hq, hkv, dh = 64, 8, 128
        lens = [min(ragged_lengths(1, 64, 4096, 131072)[:4])]  # the shortest of the first four
        total_s, total_b = 0.0, 0
        for i, L in enumerate(lens):
            k, v = self._rows(105, 2 * i, L, hkv * dh), self._rows(105, 2 * i + 1, L, hkv * dh)
            q = self._rows(105, 100 + i, 1, hq * dh)
            total_s += self.decode_seconds(k, v, q, hkv, dh, hq, 1 / math.sqrt(dh), 0)
            total_b += L * hkv * dh * 4 * 2 + 2 * hq * dh * 4
            del k, v
        return self.line(total_b / total_s / 1e9, "GB/s",
                         f"config 5 decode of one of its sequences ({lens[0]} cached rows, the shortest of the first "
                         "four; fp32), reduction only")


def cpu_baselines(extra):
    """Adds a cpu_baseline beside each single-GPU extra (rank 0, N = 1)."""
    ref = RefConfigs()
    for name, key, fn in (("config1", None, ref.config1), ("config3", None, ref.config3),
                          ("config4", None, ref.config4), ("config5", None, ref.config5),
                          ("projections", None, ref.projections)):
        ent = extra.get(name)
        if not isinstance(ent, dict) or "error" in ent:
            continue
        try:
            cb = fn()
        except Exception as e:  # report, never hide, a failing sample
            ent["cpu_baseline"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            continue
        if name == "config3":
            if isinstance(ent.get("prefill_chunk64"), dict):
                ent["prefill_chunk64"]["cpu_baseline"] = cb["prefill"]
            if isinstance(ent.get("decode"), dict):
                ent["decode"]["cpu_baseline"] = cb["decode"]
        elif name == "projections":
            for part in ("decode", "prefill"):
                if isinstance(ent.get(part), dict):
                    ent[part]["cpu_baseline"] = cb[part]
        elif name == "config4":
            for part in ("prefill", "decode"):
                if isinstance(ent.get(part), dict):
                    ent[part]["cpu_baseline"] = cb[part]
        else:
            ent["cpu_baseline"] = cb


def reference_arm(args, rank, world):
    if rank != 0:
        return
    t0 = time.perf_counter()
    # Each step is the whole config-2 workload (~1.5 s on 16 host threads)
    # while the run stays within about two minutes; longer runs time the
    # 512-row sample instead.
    ref = RefSample(full=(args.steps + args.warmup) * 1.6 <= 120)
    for _ in range(args.warmup):
        ref.run()
    secs = [ref.run() for _ in range(args.steps)]
    value = ref.flops / float(np.mean(secs)) / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * float(np.mean(secs)),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {**config2_desc(world), "rotating_sets": c2_rotating_sets(world)},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": ref.cores, "kind": ref.kind,
                             "sample": ref.sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)


def c2_sample_flops(rows_per_block=256):
    S = S2
    b0, b1 = S // 2 - rows_per_block // 2, S - rows_per_block
    pairs = sum(r + 1 for r in range(b0, b0 + rows_per_block)) + sum(r + 1 for r in range(b1, S))
    return 4.0 * DH2 * HQ2 * pairs


def c2_rotating_sets(world):
    """Input sets the headline rotates over so that one rotation exceeds the L2 (3x its 126 MB)."""
    hq_l, hkv_l = HQ2 // world, max(1, HKV2 // world)
    set_bytes = S2 * (hq_l * DH2 * 2 * 2 + hkv_l * DH2 * 2 * 4)
    return int(min(64, max(4, math.ceil(3 * L2_BYTES / set_bytes))))


def config2_desc(world):
    return {"workload": "config 2: causal GQA prefill, bf16 in / fp32 accumulate, K/V written to the device cache",
            "batch": 1, "seq_len": S2, "q_heads": HQ2, "kv_heads": HKV2, "head_dim": DH2,
            "flop_per_step": c2_flops(),
            "parallelism": f"kv-head shards x{world}" + (" + head outputs stored into every GPU's rows by the "
                                                          "attention epilogue (NVLink)" if world > 1 else ""),
            "l2": "inputs rotate over sets larger than the 126 MB L2"}


# ---------------------------------------------------------------- headline

class Comm:
    def __init__(self, rank, world, device, torch, dist):
        from hero_b200 import _lib

        self.lib = _lib
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            _lib.call("nmg_comm_unique_id", uid)
        obj = [bytes(uid) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_char * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        _lib.call("nmg_comm_init", uid, rank, world, device, ctypes.byref(h))
        self.h = h
        self.world = world

    def allgather(self, send, recv, stream):
        self.lib.call("nmg_allgather", self.h, ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                      send.numel() * send.element_size(), stream)

    def to_rows(self, gathered, out, rows, row_bytes, stream):
        self.lib.call("nmg_gather_heads_to_rows", ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                      self.world, rows, row_bytes, stream)

    def barrier(self, stream):
        self.lib.call("nmg_comm_barrier", self.h, stream)

    def close(self):
        self.lib.lib().nmg_comm_destroy(self.h)


def bench_prefill(args, torch, dist, rank, world, dev):
    from hero_b200 import nm

    from hero_b200.shard import exchange, kv_shard

    S, hq, hkv, dh = S2, HQ2, HKV2, DH2
    sh = kv_shard(rank, world, hkv, hq)
    hkv_l, hq_l = sh.kv1 - sh.kv0, sh.q1 - sh.q0
    scale = 1.0 / math.sqrt(dh)
    R = c2_rotating_sets(world)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    sets = []
    for _ in range(R):
        q = torch.randn(S, hq_l * dh, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(S, hkv_l * dh, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(S, hkv_l * dh, device=dev, generator=g).to(torch.bfloat16)
        c = nm.FullAttentionCache(hkv_l, dh, capacity=S, dtype="bf16", device=dev.index)
        o = torch.empty(S, hq_l * dh, device=dev, dtype=torch.bfloat16)
        sets.append((q, k, v, c, o))
    comm = None
    if world > 1:
        comm = Comm(rank, world, dev.index, torch, dist)
        gathered = torch.empty(world, S, hq_l * dh, device=dev, dtype=torch.bfloat16)
        full = torch.empty(S, hq * dh, device=dev, dtype=torch.bfloat16)
        # Two row buffers per rank, mapped by every rank: the attention
        # epilogue of each rank writes its heads of every row into all of
        # them (NVLink stores), then a stream-ordered barrier.
        shared = [nm.SharedRows(S, hq * dh, torch.bfloat16, dev.index) for _ in range(2)]
        peers = []
        for b in range(2):
            handles = exchange(dist, shared[b].handle)
            peers.append([shared[b].ptr if r == rank else nm.open_peer(handles[r], dev.index) for r in range(world)])
    stream = torch.cuda.current_stream(dev)

    def cur():  # the stream a call is issued on (the capture stream while a graph records)
        return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def step(i, ev=None):
        q, k, v, c, o = sets[i % R]
        c.reset()
        c.append(0, k, v)
        if ev is not None:
            ev[0].record(stream)
        if comm is None:
            nm.attend(c, q, 0, scale, out=o)
        else:
            nm.attend_fanout(c, q, 0, scale, peers[i & 1], hq * dh, sh.out_col0(dh))
        if ev is not None:
            ev[1].record(stream)
        if comm is not None:
            comm.barrier(cur())

    def step_nccl(i):  # the unfused alternative: attend, NCCL all-gather, permute
        q, k, v, c, o = sets[i % R]
        c.reset()
        c.append(0, k, v)
        nm.attend(c, q, 0, scale, out=o)
        comm.allgather(o, gathered, cur())
        comm.to_rows(gathered, full, S, hq_l * dh * 2, cur())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def capture(fn, n, first):
        """A CUDA graph of n steps fn(first), fn(first + 1), ...: the host work of
        each call (argument checks, tensor maps, the NCCL launch) happens once,
        here, instead of inside the timed region."""
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        with torch.cuda.graph(g, stream=cs):
            for i in range(n):
                fn(first + i)
        stream.wait_stream(cs)
        return g

    for i in range(args.warmup):
        step(i)
    barrier()
    # attention-kernel time, CUDA events around each eager call of one rotation
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(R)]
    for i in range(R):
        step(i, kev[i])
    barrier()
    kernel_each = [a.elapsed_time(b) for a, b in kev]
    kernel_pct = {f"p{q}": float(np.percentile(kernel_each, q)) for q in (10, 50, 90)}

    # Attention-kernel time without host launch gaps: one rotation of
    # attention-only calls (each set's cache holds its rows) replayed from a
    # CUDA graph, CUDA events on the launching stream.
    def attend_only(i):
        q, k, v, c, o = sets[i % R]
        if comm is None:
            nm.attend(c, q, 0, scale, out=o)
        else:
            nm.attend_fanout(c, q, 0, scale, peers[i & 1], hq * dh, sh.out_col0(dh))

    ga = capture(attend_only, R, 0)
    ga.replay()
    barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    ga.replay()
    a1.record(stream)
    barrier()
    kernel_ms = a0.elapsed_time(a1) / R
    del ga
    # the timed region: exactly args.steps steps, replayed from one graph
    graph = capture(step, args.steps, args.warmup)
    graph.replay()  # untimed first replay
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_smi_id(torch, dev)) as clk:
        barrier()
        t0.record(stream)
        graph.replay()
        t1.record(stream)
        barrier()
    ms = t0.elapsed_time(t1)
    del graph
    if world > 1:
        tt = torch.tensor([ms, kernel_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, kernel_ms = float(tt[0]), float(tt[1])
    ms_step = ms / args.steps
    value = c2_flops() / (ms_step * 1e-3) / 1e12
    parity = sharded_parity(torch, dist, dev, rank, world, sets[0], step, shared) if comm is not None else None
    collective = None
    if comm is not None:
        n_cmp = max(3, args.steps // 4)
        for i in range(2):
            step_nccl(i)
        barrier()
        g2 = capture(step_nccl, n_cmp, 0)
        g2.replay()
        barrier()
        u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        u0.record(stream)
        g2.replay()
        u1.record(stream)
        barrier()
        del g2
        tt = torch.tensor([u0.elapsed_time(u1) / n_cmp], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        collective = {"fused_epilogue_ms_per_step": ms_step, "nccl_allgather_ms_per_step": float(tt[0]),
                      "attention_only_ms": kernel_ms,
                      "note": "fused: NVLink stores from the attention epilogue + one stream-ordered barrier; "
                              "nccl: attention, ncclAllGather, head-to-row permutation; both timed as CUDA graphs"}

    # ---- end to end through the C ABI with host buffers
    pin = lambda t: t.cpu().pin_memory()
    hq_host, hk_host, hv_host = pin(sets[0][0]), pin(sets[0][1]), pin(sets[0][2])
    out_host = torch.empty(S, hq * dh, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, args.steps // 2)

    # Three streams, as a serving loop would run them: the inputs of step i + 1
    # cross PCIe while step i computes and step i - 1's rows come back (with
    # shards the rows come back in stream order on rank 0).  Every step's own
    # copies stay inside the timed region.
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(R)]     # set b's inputs are on the GPU
    ev_used = [torch.cuda.Event() for _ in range(R)]   # set b's inputs were consumed, its rows written
    nob = 2 if comm is not None else R                 # output buffers
    ev_out = [torch.cuda.Event() for _ in range(nob)]  # output buffer copied to the host

    def e2e_step(i):
        b = i % R
        q, k, v, c, o = sets[b]
        ob = (i & 1) if comm is not None else b
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            q.copy_(hq_host, non_blocking=True)
            k.copy_(hk_host, non_blocking=True)
            v.copy_(hv_host, non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[ob])
        c.reset()
        c.append(0, k, v)
        if comm is not None:
            nm.attend_fanout(c, q, 0, scale, peers[ob], hq * dh, sh.out_col0(dh))
            comm.barrier(cur())
        else:
            nm.attend(c, q, 0, scale, out=o)
        ev_used[b].record(stream)
        if comm is not None:
            # Every GPU holds the assembled rows; rank 0 copies them to the
            # host in stream order, before its next barrier lets the other
            # ranks write the buffer again.
            if rank == 0:
                out_host.copy_(shared[ob].tensor(), non_blocking=True)
        else:
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[b])
                out_host.copy_(o, non_blocking=True)
                ev_out[ob].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt[0])
    h2d = world * S * (hq_l + 2 * hkv_l) * dh * 2
    d2h = S * hq * dh * 2
    if comm is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()  # every rank is done writing into the mapped buffers
        for b in range(2):
            for r, ptr in enumerate(peers[b]):
                if r != rank:
                    nm.close_peer(ptr)
        dist.barrier()
        for b in range(2):
            shared[b].close()
        comm.close()
    p = peaks()
    achieved = c2_flops() / world / (kernel_ms * 1e-3) / 1e12
    roof = {"bound": "tensor", "kernel": "attn_prefill_pair_kernel<bf16>", "achieved": achieved, "peak": p["bf16"],
            "unit": "TFLOP/s", "frac": achieved / p["bf16"], "peak_src": f"{p['src']} bf16 dense (burst)",
            "traffic": ncu_traffic("attn_prefill_c2"), "kernel_ms": kernel_ms,
            "kernel_timing": f"{R} attention-only launches replayed from a CUDA graph (inputs rotate past L2)",
            "eager_ms_percentiles": {**kernel_pct, "launches": R, "rank": 0 if world == 1 else rank,
                                     "note": "CUDA events around eager calls, host launch gaps included"},
            "algorithmic_unit": "4*head_dim*q_heads per visible (query,key) pair; 8,390,656 pairs"}
    launches = args.steps * 2
    return {"value": value, "ms_per_step": ms_step, "tok_per_s": S / (ms_step * 1e-3), "roofline": roof,
            "collective": collective,
            "e2e": {"value": c2_flops() / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "clocks": clk.summary(), "gpu_launches": launches, "rotating_sets": R, "parity": parity}


def sharded_parity(torch, dist, dev, rank, world, set0, step, shared):
    """Correctness of one sharded step: every rank runs step 0 (its heads of every
    row stored into all ranks' buffer 0), the ranks all-gather their inputs, and
    rank 0 compares the assembled rows with one GPU's unsharded attention of the
    same inputs (fp32 output).  A row element passes within the north star's
    2e-3 plus the bf16 rounding of the sharded output (2^-8 of its magnitude)."""
    from hero_b200 import nm

    q, k, v = set0[0], set0[1], set0[2]
    step(0)
    dist.barrier()
    torch.cuda.synchronize(dev)
    got = shared[0].tensor().float() if rank == 0 else None
    parts = [[torch.empty_like(x) for _ in range(world)] for x in (q, k, v)]
    for lst, x in zip(parts, (q, k, v)):
        dist.all_gather(lst, x)
    res = None
    if rank == 0:
        Q, K, V = (torch.cat(lst, dim=1) for lst in parts)
        cache = nm.FullAttentionCache(HKV2, DH2, capacity=S2, dtype="bf16", device=dev.index)
        cache.append(0, K, V)
        ref = nm.attend(cache, Q, 0, 1.0 / math.sqrt(DH2), out_dtype=torch.float32)
        err = (got - ref).abs()
        ok = bool((err <= 2e-3 + ref.abs() * 2.0 ** -8).all().item())
        rel = float((got - ref).norm() / ref.norm())
        res = {"ok": ok, "max_abs": float(err.max()), "rel_l2": rel,
               "vs": "one GPU's unsharded attention of the gathered inputs, fp32 output",
               "rule": "|sharded - ref| <= 2e-3 + 2^-8 |ref| for every element"}
        del cache
    torch.cuda.synchronize(dev)
    dist.barrier()
    return res


# ---------------------------------------------------------------- extras (N=1)

def ragged_lengths(seed, n, lo, hi):
    """n integers uniform in [lo, hi] from a SplitMix64 counter stream (seeded, host-independent)."""
    M = (1 << 64) - 1

    def mix(z):
        z = (z + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    key = mix(seed ^ mix(0x632BE59BD9B4E019))
    return [lo + mix((key + j) & M) % (hi - lo + 1) for j in range(n)]


def graph_time(torch, dev, fn, reps, inner):
    """Average ms of fn() when `inner` calls are captured in one CUDA graph and replayed `reps` times."""
    fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=s):
            for _ in range(inner):
                fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / (reps * inner)


def extra_config1(torch, dev, small=False):
    from hero_b200 import nm

    hq, hkv, dh, rows, NC = 16, 8, 128, 1024, 20
    caches, qs, outs = [], [], []
    for i in range(NC):
        c = nm.FullAttentionCache(hkv, dh, capacity=rows, device=dev.index)
        c.append(0, torch.randn(rows, hkv * dh, device=dev), torch.randn(rows, hkv * dh, device=dev))
        caches.append(c)
        qs.append(torch.randn(1, hq * dh, device=dev))
        outs.append(torch.empty(1, hq * dh, device=dev))
    it = [0]

    def fn():
        for i in range(NC):
            nm.attend(caches[i], qs[i], rows - 1, 1 / math.sqrt(dh), out=outs[i])

    ms = graph_time(torch, dev, fn, 20, 5) / NC
    bytes_ = 2 * rows * hkv * dh * 4 + 2 * hq * dh * 4
    p = peaks()
    gbs = bytes_ / (ms * 1e-3) / 1e9
    return {"workload": "config 1: decode, fp32, 16q/8kv, d128, 1024 cached", "value": gbs, "unit": "GB/s",
            "us_per_call": ms * 1e3, "tok_per_s": 1 / (ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm"], "frac": gbs / p["hbm"],
                         "bytes_per_call": bytes_, "traffic": ncu_traffic("attn_decode_c1"),
                         "kernel": "attn_cluster_kernel<128, 2> (8-CTA clusters)"},
            "method": f"{NC} caches (168 MB > L2) rotated in a CUDA graph; kernel time per call"}


def extra_config3(torch, dev, small=False):
    from hero_b200 import nm

    hv, hk, d, T, Tdec = 32, 16, 128, 8192, 256
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    norm = lambda x: x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    q = norm(torch.randn(T, hk, d, device=dev, generator=g)) / math.sqrt(d)
    k = norm(torch.randn(T, hk, d, device=dev, generator=g))
    v = torch.randn(T, hv, d, device=dev, generator=g)
    gate = -torch.nn.functional.softplus(torch.randn(T, hv, device=dev, generator=g))
    beta = torch.sigmoid(torch.randn(T, hv, device=dev, generator=g))
    st = nm.DeltaNetState(hv, d, d, device=dev.index)
    out = torch.empty(T, hv, d, device=dev)
    res = {}
    for chunk in (0, 64):
        try:
            nm.delta_prefill(st, q, k, v, gate, beta, hk, chunk=chunk, out=out)
        except Exception as e:  # a chunk size this build does not provide
            res[f"prefill_chunk{chunk}"] = {"unavailable": str(e)[:120]}
            continue
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(3):
            st.clear()
            nm.delta_prefill(st, q, k, v, gate, beta, hk, chunk=chunk, out=out)
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / 3
        seq_flops = 7.0 * d * d * T * hv
        res[f"prefill_chunk{chunk}"] = {"ms": ms, "tok_per_s": T / (ms * 1e-3),
                                        "tflops_recurrence_equiv": seq_flops / (ms * 1e-3) / 1e12}
        if chunk:
            # chunked algorithm per (value head, chunk): 5*2C^2D + 3*2CD^2 + (2/3)C^3 FLOP
            C = chunk
            alg = (5 * 2 * C * C * d + 3 * 2 * C * d * d + 2 * C ** 3 / 3) * hv * (T // C)
            tf = alg / (ms * 1e-3) / 1e12
            tf32_peak, note = tf32_peak_and_note()
            res[f"prefill_chunk{chunk}"].update(
                {"tflops_chunked_alg": tf, "alg_flop": alg,
                 "roofline": {"bound": "tensor", "achieved": tf, "peak": tf32_peak, "unit": "TFLOP/s",
                              "frac": tf / tf32_peak, "note": note,
                              "tensor_rates": (tensor_rates() or {}).get("issue_loop")}})
    # 256 decode steps continue from the final state, graph-captured
    qd = norm(torch.randn(Tdec, hk, d, device=dev, generator=g)) / math.sqrt(d)
    kd = norm(torch.randn(Tdec, hk, d, device=dev, generator=g))
    vd = torch.randn(Tdec, hv, d, device=dev, generator=g)
    gd = -torch.nn.functional.softplus(torch.randn(Tdec, hv, device=dev, generator=g))
    bd = torch.sigmoid(torch.randn(Tdec, hv, device=dev, generator=g))
    od = torch.empty(Tdec, hv, d, device=dev)

    def fn():
        for t in range(Tdec):
            nm.delta_step(st, qd[t], kd[t], vd[t], gd[t], bd[t], hk, out=od[t])

    ms = graph_time(torch, dev, fn, 5, 1) / Tdec
    bytes_ = 2 * hv * d * d * 4 + 2 * hk * d * 4 + 2 * hv * d * 4 + 2 * hv * 4
    p = peaks()
    gbs = bytes_ / (ms * 1e-3) / 1e9
    res["decode"] = {"us_per_step": ms * 1e3, "value": gbs, "unit": "GB/s", "tok_per_s": 1 / (ms * 1e-3),
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm"], "frac": gbs / p["hbm"],
                                  "bytes_per_step": bytes_, "note": "2 MB state is L2-resident between steps"}}
    del qd, kd, vd, gd, bd, od
    # The whole layer core per decode token (prologue -> step -> epilogue,
    # qwen35.hpp:396-461 at T = 1): one fused launch against the three
    # launches, each captured over a run of tokens in a CUDA graph.
    Cc, Wc, Tt = 2 * hk * d + hv * d, 4, 64
    conv1 = nm.ConvState(Cc, Wc, device=dev.index)
    cwt = torch.randn(Cc, Wc, device=dev, generator=g) * 0.5
    qkvt = torch.randn(Tt, Cc, device=dev, generator=g)
    brt, art = torch.randn(Tt, hv, device=dev, generator=g), torch.randn(Tt, hv, device=dev, generator=g)
    dtbt, dsct = torch.randn(hv, device=dev, generator=g), -torch.rand(hv, device=dev, generator=g)
    zt, gmt = torch.randn(Tt, hv, d, device=dev, generator=g), torch.randn(d, device=dev, generator=g)
    outt = torch.empty(Tt, hv, d, device=dev)

    def fused():
        for t in range(Tt):
            nm.delta_decode_token(st, conv1, cwt, qkvt[t], brt[t], art[t], dtbt, dsct, hk, zt[t], gmt, 1e-6,
                                  out=outt[t])

    def three():
        for t in range(Tt):
            qx, kx, vx, bx, gx = nm.delta_prologue(conv1, cwt, qkvt[t:t + 1], brt[t:t + 1], art[t:t + 1], dtbt, dsct,
                                                   hk, hv, d, d)
            ox = nm.delta_step(st, qx[0], kx[0], vx[0], gx[0], bx[0], hk)
            nm.delta_epilogue(ox[None], zt[t:t + 1], gmt, 1e-6, out=outt[t:t + 1])

    us_f = graph_time(torch, dev, fused, 5, 1) / Tt * 1e3
    us_3 = graph_time(torch, dev, three, 5, 1) / Tt * 1e3
    res["decode_layer_token"] = {"us_fused": us_f, "us_three_launches": us_3, "tok_per_s": 1e6 / us_f,
                                 "kernel": "delta_decode_kernel (one launch per layer and token)",
                                 "note": f"{Tt} tokens of one sequence in a CUDA graph; 2 MB state, L2-resident"}
    del conv1, cwt, qkvt, brt, art, zt, outt
    # Batched decode: one token for each of 64 sequences (each its own 2 MB
    # state; 128 MB of states, past the L2), one launch per step.
    B = 8 if small else 64
    states = [nm.DeltaNetState(hv, d, d, device=dev.index) for _ in range(B)]
    for st_b in states:
        st_b.tensor().normal_(0.0, 0.05, generator=g)
    qb = norm(torch.randn(B, hk, d, device=dev, generator=g)) / math.sqrt(d)
    kb = norm(torch.randn(B, hk, d, device=dev, generator=g))
    vb = torch.randn(B, hv, d, device=dev, generator=g)
    gb = -torch.nn.functional.softplus(torch.randn(B, hv, device=dev, generator=g))
    bb = torch.sigmoid(torch.randn(B, hv, device=dev, generator=g))
    ob = torch.empty(B, hv, d, device=dev)
    ms_b = graph_time(torch, dev, lambda: nm.delta_step_batch(states, qb, kb, vb, gb, bb, hk, out=ob), 5, 8)
    bytes_b = B * bytes_
    gbs_b = bytes_b / (ms_b * 1e-3) / 1e9
    res["decode_batch"] = {"batch": B, "us_per_step": ms_b * 1e3, "value": gbs_b, "unit": "GB/s",
                           "tok_per_s": B / (ms_b * 1e-3),
                           "roofline": {"bound": "hbm", "achieved": gbs_b, "peak": p["hbm"], "frac": gbs_b / p["hbm"],
                                        "bytes_per_step": bytes_b, "kernel": "delta_step_batch_kernel",
                                        "note": f"{B} sequences x 32 value heads, states {B * 2} MB (> L2)"}}
    del states, qb, kb, vb, gb, bb, ob
    # the steps either side of the recurrence over the same T tokens: conv +
    # SiLU + L2 norms + gates from the packed projection, and the gated RMS norm
    C, W = 2 * hk * d + hv * d, 4
    conv = nm.ConvState(C, W, device=dev.index)
    cw = torch.randn(C, W, device=dev, generator=g) * 0.5
    qkv = torch.randn(T, C, device=dev, generator=g)
    br, ar = torch.randn(T, hv, device=dev, generator=g), torch.randn(T, hv, device=dev, generator=g)
    dtb, dsc = torch.randn(hv, device=dev, generator=g), -torch.rand(hv, device=dev, generator=g)

    def pro():
        conv.clear()
        nm.delta_prologue(conv, cw, qkv, br, ar, dtb, dsc, hk, hv, d, d)

    pro()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        pro()
    b.record()
    torch.cuda.synchronize(dev)
    ms_p = a.elapsed_time(b) / 5
    bytes_p = 4 * (T * C + C * W + 2 * T * hv + 2 * hv + 2 * T * hk * d + T * hv * d + 2 * T * hv)
    del qkv
    o = torch.randn(T, hv, d, device=dev, generator=g)
    z = torch.randn(T, hv, d, device=dev, generator=g)
    gamma = torch.randn(d, device=dev, generator=g)
    eo = torch.empty_like(o)
    nm.delta_epilogue(o, z, gamma, 1e-6, out=eo)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(5):
        nm.delta_epilogue(o, z, gamma, 1e-6, out=eo)
    b.record()
    torch.cuda.synchronize(dev)
    ms_e = a.elapsed_time(b) / 5
    bytes_e = 4 * (3 * T * hv * d + d)
    gb_p, gb_e = bytes_p / (ms_p * 1e-3) / 1e9, bytes_e / (ms_e * 1e-3) / 1e9
    res["prologue"] = {"us": ms_p * 1e3, "value": gb_p, "unit": "GB/s",
                       "roofline": {"bound": "hbm", "achieved": gb_p, "peak": p["hbm"], "frac": gb_p / p["hbm"],
                                    "bytes": bytes_p, "note": "conv width 4 + SiLU + per-head L2 norms + gates, "
                                                              "inputs 268 MB > L2"}}
    res["epilogue"] = {"us": ms_e * 1e3, "value": gb_e, "unit": "GB/s",
                       "roofline": {"bound": "hbm", "achieved": gb_e, "peak": p["hbm"], "frac": gb_e / p["hbm"],
                                    "bytes": bytes_e, "note": "per-head RMS norm times SiLU(z)"}}
    return {"workload": "config 3: gated delta rule, T=8192, 16 k-heads / 32 v-heads, d128, fp32 state", **res}


def extra_attn_io(torch, dev, small=False):
    """The steps either side of a Qwen 3.5 attention reduction at T=8192: the
    prologue (per-head RMSNorm + partial RoPE of Q and K, append to a bf16 cache)
    and the output gate, both HBM-bound."""
    from hero_b200 import nm

    hq, hkv, dh, T = 16, 4, 256, (1024 if small else 8192)
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    qg = torch.randn(T, 2 * hq * dh, device=dev, generator=g)
    k = torch.randn(T, hkv * dh, device=dev, generator=g)
    v = torch.randn(T, hkv * dh, device=dev, generator=g)
    qgam, kgam = torch.randn(dh, device=dev, generator=g), torch.randn(dh, device=dev, generator=g)
    cache = nm.FullAttentionCache(hkv, dh, capacity=T, dtype="bf16", device=dev.index)
    a = torch.randn(T, hq * dh, device=dev, generator=g).to(torch.bfloat16)

    def pro():
        cache.reset()
        return nm.attn_prologue(cache, 0, qg, k, v, qgam, kgam, 1e-6, 1e7, 1, 4)

    def timed(fn, n=5):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    host_p, host_g = timed(pro), timed(lambda: nm.attn_gate(qg, a, dh))  # eager calls, host overhead included
    ms_p = graph_time(torch, dev, pro, 10, 5)  # kernel time: the calls captured in a CUDA graph
    ms_g = graph_time(torch, dev, lambda: nm.attn_gate(qg, a, dh), 10, 5)
    # prologue: read the Q halves of qg, K and V (fp32); write Q (bf16) and the cache rows (bf16 K, fp16 V)
    bytes_p = 4 * T * hq * dh + 2 * 4 * T * hkv * dh + 2 * T * hq * dh + 2 * 2 * T * hkv * dh
    # gate: read the gate halves of qg (fp32), read and write A (bf16)
    bytes_g = 4 * T * hq * dh + 2 * 2 * T * hq * dh
    p = peaks()
    gb_p, gb_g = bytes_p / (ms_p * 1e-3) / 1e9, bytes_g / (ms_g * 1e-3) / 1e9
    return {"workload": f"Qwen 3.5 attention prologue and gate, T={T}, 16 q-heads / 4 kv-heads, d256, bf16 cache",
            "method": "kernel time from 5 calls captured in a CUDA graph, replayed 10 times (inputs 403 MB > L2); "
                      "us_eager: the same calls issued from Python",
            "prologue": {"us": ms_p * 1e3, "us_eager": host_p * 1e3, "value": gb_p, "unit": "GB/s",
                         "roofline": {"bound": "hbm", "achieved": gb_p, "peak": p["hbm"], "frac": gb_p / p["hbm"],
                                      "bytes": bytes_p}},
            "gate": {"us": ms_g * 1e3, "us_eager": host_g * 1e3, "value": gb_g, "unit": "GB/s",
                     "roofline": {"bound": "hbm", "achieved": gb_g, "peak": p["hbm"], "frac": gb_g / p["hbm"],
                                  "bytes": bytes_g}}}


def extra_vit(torch, dev, small=False):
    """Dense attention of the vision ViT (scaled_dot_product_attention<12, 64, 64>,
    scale 1) at its largest image, 2520 patch tokens, bf16 on the tensor cores."""
    from hero_b200 import nm

    heads, dh, n = 12, 64, 2520
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    q, k, v = (torch.randn(n, heads * dh, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    out = torch.empty(n, heads * dh, device=dev, dtype=torch.bfloat16)
    ms = graph_time(torch, dev, lambda: nm.scaled_dot_product_attention(q, k, v, heads, 1.0, out=out), 20, 10)
    flops = 4 * dh * heads * n * n
    p = peaks()
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": "vision ViT attention: 12 heads, head_dim 64, 2520 tokens, no mask, bf16", "us": ms * 1e3,
            "value": tf, "unit": "TFLOP/s",
            "roofline": {"bound": "tensor", "achieved": tf, "peak": p["bf16"], "frac": tf / p["bf16"], "flops": flops},
            "method": "10 calls captured in a CUDA graph, replayed 20 times; each call stages K/V head-major, then "
                      "the tensor-core kernel"}


def extra_config4(torch, dev, small=False):
    from hero_b200 import nm

    hq, hkv, dh, W, S = 8, 4, 256, 1024, 8192
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    rms = lambda x: x / x.float().pow(2).mean(dim=-1, keepdim=True).add(1e-6).sqrt()
    q = rms(torch.randn(S, hq, dh, device=dev, generator=g)).reshape(S, hq * dh).to(torch.bfloat16)
    k = rms(torch.randn(S, hkv, dh, device=dev, generator=g)).reshape(S, hkv * dh).to(torch.bfloat16)
    v = torch.randn(S, hkv * dh, device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty(S, hq * dh, device=dev, dtype=torch.bfloat16)
    local = [nm.LocalAttentionCache(hkv, dh, W, capacity=S + W, dtype="bf16", device=dev.index) for _ in range(5)]
    glob = nm.FullAttentionCache(hkv, dh, capacity=S, dtype="bf16", device=dev.index)

    def group():
        for c in local:
            c.reset()
            nm.append_attend(c, 0, k, v, q, None, out=o)
        glob.reset()
        nm.append_attend(glob, 0, k, v, q, None, out=o)

    group()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(3):
        group()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / 3
    pairs_g = S * (S + 1) // 2
    pairs_l = W * (W + 1) // 2 + (S - W) * W
    flops = 4.0 * dh * hq * (pairs_g + 5 * pairs_l)
    p = peaks()
    tf = flops / (ms * 1e-3) / 1e12
    res = {"prefill": {"ms_per_group": ms, "value": tf, "unit": "TFLOP/s", "tok_per_s": S / (ms * 1e-3),
                       "roofline": {"bound": "tensor", "achieved": tf, "peak": p["bf16"], "frac": tf / p["bf16"],
                                    "flop_per_group": flops}}}
    del local, glob, q, k, v, o
    # decode: batch 16, 32768 cached rows (query at 32767), global + local layers
    B, L = (2, 32768) if small else (16, 32768)
    # the group's five sliding-window layers, each its own caches: 5 x 67 MB
    # of windows, so consecutive window decodes do not find their rows in L2
    NL = 5
    gcaches, lsets, q8caches = [], [[] for _ in range(NL)], []
    for b_ in range(B):
        kk = torch.randn(L, hkv * dh, device=dev, generator=g).to(torch.bfloat16)
        vv = torch.randn(L, hkv * dh, device=dev, generator=g).to(torch.bfloat16)
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="bf16", device=dev.index)
        c.append(0, kk, vv)
        gcaches.append(c)
        # the same rows in a Q8_0 cache (quantised on append) for the global layer
        c8 = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="q8_0", device=dev.index)
        c8.append(0, kk, vv)
        q8caches.append(c8)
        for li in range(NL):
            lc = nm.LocalAttentionCache(hkv, dh, W, capacity=2 * W, dtype="bf16", device=dev.index)
            lo = L - W - li * W  # a different window of rows per layer
            lc.append(L - W, kk[lo:lo + W], vv[lo:lo + W])
            lsets[li].append(lc)
        del kk, vv
    qd = torch.randn(B, hq * dh, device=dev, generator=g).to(torch.bfloat16)
    od = torch.empty(B, hq * dh, device=dev, dtype=torch.float32)
    ms_g = graph_time(torch, dev, lambda: nm.attend_batch(gcaches, qd, None, out=od), 10, 2)

    def local_layers():
        for ls in lsets:
            nm.attend_batch(ls, qd, None, out=od)

    ms_l = graph_time(torch, dev, local_layers, 10, 4) / NL
    bytes_g = B * L * hkv * dh * 2 * 2
    bytes_l = B * W * hkv * dh * 2 * 2
    gb_g, gb_l = bytes_g / (ms_g * 1e-3) / 1e9, bytes_l / (ms_l * 1e-3) / 1e9
    grp_ms = ms_g + 5 * ms_l
    res["decode"] = {"global_us": ms_g * 1e3, "local_us": ms_l * 1e3, "global_GBps": gb_g, "local_GBps": gb_l,
                     "group_tok_per_s": B / (grp_ms * 1e-3), "value": (bytes_g + 5 * bytes_l) / (grp_ms * 1e-3) / 1e9,
                     "unit": "GB/s", "roofline": {"bound": "hbm", "achieved": gb_g, "peak": p["hbm"],
                                                  "frac": gb_g / p["hbm"], "kernel": "global layer decode"},
                     "local_roofline": {"bound": "hbm", "achieved": gb_l, "peak": p["hbm"], "frac": gb_l / p["hbm"],
                                        "kernel": "sliding-window layer decode (one cluster per row's splits)",
                                        "note": f"{NL} layers' window caches ({NL * bytes_l / 1e6:.0f} MB > L2) "
                                                "decoded in turn"}}
    try:  # the global layer over Q8_0 caches of the same rows (136 bytes per 128 values: int8 + fp16 scales)
        ms8 = graph_time(torch, dev, lambda: nm.attend_batch(q8caches, qd, None, out=od), 10, 2)
        bytes8 = B * L * hkv * (dh + dh // 32 * 2) * 2
        gb8 = bytes8 / (ms8 * 1e-3) / 1e9
        res["decode"]["q8_0"] = {"global_us": ms8 * 1e3, "time_vs_bf16": ms8 / ms_g, "bytes_vs_bf16": bytes8 / bytes_g,
                                 "value": gb8, "unit": "GB/s",
                                 "roofline": {"bound": "hbm", "achieved": gb8, "peak": p["hbm"], "frac": gb8 / p["hbm"],
                                              "kernel": "attn_decode_mma_kernel<256, Q8_0>, global layer"}}
    except Exception as e:  # report, never hide, a failing part
        res["decode"]["q8_0"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return {"workload": "config 4: Gemma hybrid bf16, 8q/4kv, d256, scale 1, 5 local (W=1024) : 1 global", **res}


# Qwen3.5-9B (qwen35.hpp:62-83, D = 4096, FF = 12288) projections of one
# delta-rule layer in a Q4_K_M-style mix: in-projection qkv (D -> 2*2048 +
# 4096 conv channels), z (D -> 4096), out (4096 -> D), MLP gate and up
# (D -> FF) in Q4_K, MLP down (FF -> D) in Q6_K.
PROJ_LAYER = (("qkv", 12, 4096, 8192), ("z", 12, 4096, 4096), ("out", 12, 4096, 4096), ("gate", 12, 4096, 12288),
              ("up", 12, 4096, 12288), ("down", 14, 12288, 4096))
_GGUF_BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


def synthetic_gguf(gt, out, n, seed):
    """Random GGUF block bytes [out][row bytes] with fp16 scale fields sized so
    a weight is about 1 / sqrt(n) (random quant bytes, as the reference's quant
    tests draw them)."""
    bl, bb = _GGUF_BLOCK[gt]
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=(out, n // bl, bb), dtype=np.uint8)
    s = 1.0 / math.sqrt(n)

    def put(off, v):
        h = np.asarray(v, np.float16).view(np.uint16)
        w[:, :, off], w[:, :, off + 1] = (h & 0xFF).astype(np.uint8), (h >> 8).astype(np.uint8)

    u = rng.uniform(0.5, 1.5, size=(out, n // bl))
    if gt == 8:
        put(0, s / 74 * u)
    elif gt == 2:
        put(0, s / 4.6 * u)
    elif gt == 12:
        put(0, s / 317 * u)
        put(2, s / 317 * 7.5 * u)
    elif gt == 14:
        put(208, s / 1369 * u)
    return w.reshape(out, -1)


def extra_projections(torch, dev, small=False):
    """The quantised projections of Qwen3.5-9B delta-rule layers (weights
    resident on the device): decode (one token, Weight::matvec for each of the
    six projections, weights streamed from HBM: two layers' weights, 271 MB,
    alternate past the L2) and prefill (4096 tokens, Weight::matmul on the int8
    tensor-core tiles)."""
    from hero_b200 import nm

    layers = 1 if small else 2
    Ws = [[nm.Weight(gt, n, o, synthetic_gguf(gt, o, n, 100 * l + i), device=dev.index)
           for i, (_, gt, n, o) in enumerate(PROJ_LAYER)] for l in range(layers)]
    wbytes = sum((n // _GGUF_BLOCK[gt][0]) * _GGUF_BLOCK[gt][1] * o for _, gt, n, o in PROJ_LAYER)
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    T = 256 if small else 4096
    x = {n: torch.randn(T, n, device=dev, generator=g) for n in (4096, 12288)}
    y = {o: torch.empty(T, o, device=dev) for o in (4096, 8192, 12288)}

    def decode():
        for Wl in Ws:
            for W, (_, gt, n, o) in zip(Wl, PROJ_LAYER):
                W.matvec(x[n][0], out=y[o][0])

    ms = graph_time(torch, dev, decode, 10, 5) / layers
    gbs = wbytes / (ms * 1e-3) / 1e9
    p = peaks()
    res = {"workload": "Qwen3.5-9B delta-layer projections (qkv, z, out, gate, up in Q4_K; down in Q6_K), "
                       f"{wbytes / 1e6:.1f} MB of GGUF weights per layer, {layers} layers alternating",
           "decode": {"value": gbs, "unit": "GB/s", "us_per_layer": ms * 1e3, "weight_bytes": wbytes,
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm"], "frac": gbs / p["hbm"],
                                   "kernel": "mv_kernel (activation quantiser fused or a launch ahead of it)"},
                      "method": "6 matvecs per layer captured in a CUDA graph with programmatic launches, "
                                f"{layers} layers' weights in turn, 5 passes per graph, 10 replays"}}
    ops = 2.0 * T * sum(n * o for _, _, n, o in PROJ_LAYER)

    def prefill():
        for W, (_, gt, n, o) in zip(Ws[0], PROJ_LAYER):
            W.matmul(x[n], out=y[o])

    msp = graph_time(torch, dev, prefill, 3, 2)
    tops = ops / (msp * 1e-3) / 1e12
    ceil = imma_rate()
    res["prefill"] = {"value": tops, "unit": "TOPS", "ms_per_layer": msp, "rows": T,
                      "roofline": {"bound": "tensor", "achieved": tops, "peak": ceil, "unit": "TOPS",
                                   "frac": (tops / ceil) if ceil else None,
                                   "peak_note": "measured mma.sync m16n8k32 int8 issue rate (libnmg_rate.so); "
                                                "tcgen05 int8 nominal is 4500 TOPS",
                                   "kernel": "mm_kernel (int8 mma.sync tiles, per-block fp32 scaling)"}}
    return res


def extra_config5(torch, dev, small=False):
    from hero_b200 import nm

    B, hq, hkv, dh = 64, 64, 8, 128
    lens = ragged_lengths(1, B, 4096, 131072)
    if small:  # profiling size: the first 4 sequences
        B, lens = 4, lens[:4]
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    caches = []
    for L in lens:
        c = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="f16", device=dev.index)
        chunk = 32768
        for s in range(0, L, chunk):
            n = min(chunk, L - s)
            c.append(s, torch.randn(n, hkv * dh, device=dev, generator=g).half(),
                     torch.randn(n, hkv * dh, device=dev, generator=g).half())
        caches.append(c)
    q = torch.randn(B, hq * dh, device=dev, generator=g).half()
    out = torch.empty(B, hq * dh, device=dev, dtype=torch.float32)
    ms = graph_time(torch, dev, lambda: nm.attend_batch(caches, q, 1 / math.sqrt(dh), out=out), 5, 1)
    bytes_ = 4096 * sum(lens) + 2 * B * hq * dh * 2
    gbs = bytes_ / (ms * 1e-3) / 1e9
    p = peaks()
    res = {"workload": "config 5: batch 64 ragged (U[4096,131072], seed 1) decode, 64q/8kv, d128, f16 cache",
           "value": gbs, "unit": "GB/s", "ms_per_call": ms, "tok_per_s": B / (ms * 1e-3), "kv_bytes": 4096 * sum(lens),
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm"], "frac": gbs / p["hbm"]}}
    # The same decode over Q8_0 caches (int8 quants + an fp16 scale per 32
    # values: 136 bytes per row and head instead of 256), filled from the f16 rows.
    try:
        q8 = []
        for c in caches:
            L = c.size()
            cq = nm.FullAttentionCache(hkv, dh, capacity=L, dtype="q8_0", device=dev.index)
            kp, vp, slots = c.storage()
            for s0 in range(0, L, 32768):
                n = min(32768, L - s0)
                kk = torch.empty(n, hkv * dh, device=dev, dtype=torch.float16)
                vv = torch.empty_like(kk)
                for hh in range(hkv):  # head-major cache rows back to token-major
                    kk.view(n, hkv, dh)[:, hh] = nm._from_ptr(kp + 2 * (hh * slots + s0) * dh, n * dh, dev.index,
                                                              torch.float16).view(n, dh)
                    vv.view(n, hkv, dh)[:, hh] = nm._from_ptr(vp + 2 * (hh * slots + s0) * dh, n * dh, dev.index,
                                                              torch.float16).view(n, dh)
                cq.append(s0, kk, vv)
            q8.append(cq)
        del caches
        torch.cuda.empty_cache()
        ms8 = graph_time(torch, dev, lambda: nm.attend_batch(q8, q, 1 / math.sqrt(dh), out=out), 5, 1)
        bytes8 = sum(lens) * hkv * 2 * (dh + dh // 32 * 2) + 2 * B * hq * dh * 2
        gb8 = bytes8 / (ms8 * 1e-3) / 1e9
        res["q8_0"] = {"ms_per_call": ms8, "time_vs_f16": ms8 / ms, "bytes_vs_f16": bytes8 / bytes_, "value": gb8,
                       "unit": "GB/s", "tok_per_s": B / (ms8 * 1e-3), "kv_bytes": bytes8,
                       "roofline": {"bound": "hbm", "achieved": gb8, "peak": p["hbm"], "frac": gb8 / p["hbm"],
                                    "kernel": "attn_decode_mma_kernel<128, Q8_0>"}}
    except Exception as e:  # report, never hide, a failing part
        res["q8_0"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return res


# ---------------------------------------------------------------- extras (N>1)

class OtherRankFailed(RuntimeError):
    pass


class Ranks:
    """The ranks of a multi-GPU extra: barriers, max-over-ranks timing, and
    the all-gather of equal per-rank blocks followed by the head-to-row
    permutation (both through the C ABI, on the current stream)."""

    def __init__(self, torch, dist, dev, rank, world):
        self.torch, self.dist, self.dev, self.rank, self.world = torch, dist, dev, rank, world
        self.comm = Comm(rank, world, dev.index, torch, dist)

    def cur(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)

    def barrier(self):
        self.dist.barrier()
        self.torch.cuda.synchronize(self.dev)

    def max_over(self, *vals):
        t = self.torch.tensor(vals, device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    def all_ok(self, ok):
        """True on every rank when every rank reports ok (one collective that
        every rank reaches, failed or not, so the ranks stay in step)."""
        t = self.torch.tensor([0 if ok else 1], device=self.dev, dtype=self.torch.int32)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return int(t.item()) == 0

    def checkpoint(self):
        """Every rank of an extra passes here together: after each phase's
        allocations (before its collectives) and at its end.  A rank that
        failed on its own since the last checkpoint meets the others here with
        all_ok(False) instead, and every rank then stops the extra; each rank
        so takes the same collective steps whichever ranks failed."""
        if not self.all_ok(True):
            raise OtherRankFailed("failed on another rank")

    def gather(self, send, gathered):
        self.comm.allgather(send, gathered, self.cur())

    def to_rows(self, gathered, out, world, rows, row_bytes):
        from hero_b200 import _lib

        _lib.call("nmg_gather_heads_to_rows", ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                  world, rows, row_bytes, self.cur())

    def graph_ms(self, fn, reps, inner):
        """Max over ranks of the average ms of fn() when `inner` calls are
        captured in one CUDA graph and replayed `reps` times, every rank
        starting together after a barrier."""
        torch, dev = self.torch, self.dev
        fn()
        self.barrier()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(inner):
                    fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        self.barrier()
        g.replay()
        self.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        self.barrier()
        ms = a.elapsed_time(b) / (reps * inner)
        del g
        return self.max_over(ms)[0]

    def event_ms(self, fn, reps):
        """Max over ranks of the average ms of `reps` eager calls of fn()."""
        torch = self.torch
        fn()
        self.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        self.barrier()
        return self.max_over(a.elapsed_time(b) / reps)[0]

    def release(self):
        """Between extras: wait for this GPU, return the freed blocks."""
        self.torch.cuda.synchronize(self.dev)
        self.torch.cuda.empty_cache()

    def close(self):
        self.torch.cuda.synchronize(self.dev)
        self.dist.barrier()
        self.comm.close()


def sharded_config1(rk, small=False):
    """Config 1 split by KV head: each rank reduces its heads of the query
    over its share of the fp32 cache, then the head outputs are all-gathered
    and laid into the [1][16*128] row."""
    from hero_b200 import nm
    from hero_b200.shard import kv_shard

    torch, dev, world = rk.torch, rk.dev, rk.world
    hq, hkv, dh, rows = 16, 8, 128, 1024
    sh = kv_shard(rk.rank, world, hkv, hq)
    hkv_l, hq_l = sh.kv1 - sh.kv0, sh.q1 - sh.q0
    NC = 2 if small else 20 * world  # rotated caches: NC * 8.4 MB / world per GPU > L2
    caches, qs, outs = [], [], []
    for _ in range(NC):
        c = nm.FullAttentionCache(hkv_l, dh, capacity=rows, device=dev.index)
        c.append(0, torch.randn(rows, hkv_l * dh, device=dev), torch.randn(rows, hkv_l * dh, device=dev))
        caches.append(c)
        qs.append(torch.randn(1, hq_l * dh, device=dev))
        outs.append(torch.empty(1, hq_l * dh, device=dev))
    gathered = torch.empty(world, 1, hq_l * dh, device=dev)
    full = torch.empty(1, hq * dh, device=dev)
    scale = 1 / math.sqrt(dh)

    def local():
        for i in range(NC):
            nm.attend(caches[i], qs[i], rows - 1, scale, out=outs[i])

    def whole():
        for i in range(NC):
            nm.attend(caches[i], qs[i], rows - 1, scale, out=outs[i])
            rk.gather(outs[i], gathered)
            rk.to_rows(gathered, full, world, 1, hq_l * dh * 4)

    rk.checkpoint()
    ms_local = rk.graph_ms(local, 20, 1) / NC
    ms = rk.graph_ms(whole, 20, 1) / NC
    bytes_ = 2 * rows * hkv * dh * 4 + 2 * hq * dh * 4
    p = peaks()
    gbs = bytes_ / (ms * 1e-3) / 1e9
    gbs_local = bytes_ / world / (ms_local * 1e-3) / 1e9
    rk.checkpoint()
    return {"workload": "config 1: decode, fp32, 16q/8kv, d128, 1024 cached", "parallelism": f"kv-head shards x{world}",
            "value": gbs, "unit": "GB/s", "us_per_call": ms * 1e3, "tok_per_s": 1 / (ms * 1e-3),
            "attention_only_us": ms_local * 1e3,
            "roofline": {"bound": "hbm", "achieved": gbs_local, "peak": p["hbm"], "frac": gbs_local / p["hbm"],
                         "per": "GPU, attention kernel alone"},
            "method": f"{NC} caches rotated in a CUDA graph; each call = attention + ncclAllGather of the head "
                      "outputs + head-to-row permutation; time = max over ranks"}


def sharded_config3(rk, small=False):
    """Config 3 split by key-head group: a rank owns key heads [k0, k1) and the
    value heads that read them (h % 16), so prefill and decode run with no
    exchange; the head outputs are all-gathered into [T][32*128] rows."""
    from hero_b200 import nm
    from hero_b200.shard import delta_shard

    torch, dev, world = rk.torch, rk.dev, rk.world
    hv, hk, d, T, Tdec = (32, 16, 128, 512, 8) if small else (32, 16, 128, 8192, 256)
    sd = delta_shard(rk.rank, world, hk, hv)
    hs = torch.tensor(sd.v_heads, device=dev)
    R = hv // hk
    g = torch.Generator(device=dev)
    g.manual_seed(3)  # the single-GPU inputs; each rank keeps its heads
    norm = lambda x: x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    q = (norm(torch.randn(T, hk, d, device=dev, generator=g)) / math.sqrt(d))[:, sd.k0:sd.k1].contiguous()
    k = norm(torch.randn(T, hk, d, device=dev, generator=g))[:, sd.k0:sd.k1].contiguous()
    v = torch.randn(T, hv, d, device=dev, generator=g).index_select(1, hs).contiguous()
    gate = (-torch.nn.functional.softplus(torch.randn(T, hv, device=dev, generator=g))).index_select(1, hs).contiguous()
    beta = torch.sigmoid(torch.randn(T, hv, device=dev, generator=g)).index_select(1, hs).contiguous()
    st = nm.DeltaNetState(sd.hv, d, d, device=dev.index)
    out = torch.empty(T, sd.hv, d, device=dev)
    gathered = torch.empty(world, T, sd.hv * d, device=dev)
    full = torch.empty(T, hv * d, device=dev)

    def prefill_local():
        st.clear()
        nm.delta_prefill(st, q, k, v, gate, beta, sd.hk, chunk=64, out=out)

    def prefill():
        prefill_local()
        rk.gather(out, gathered)
        rk.to_rows(gathered, full, world, T * R, sd.hk * d * 4)

    rk.checkpoint()
    ms_pl = rk.event_ms(prefill_local, 3)
    ms_p = rk.event_ms(prefill, 3)
    C = 64
    alg = (5 * 2 * C * C * d + 3 * 2 * C * d * d + 2 * C ** 3 / 3) * hv * (T // C)
    p = peaks()
    tf32_peak, note = tf32_peak_and_note()
    tf_local = alg / world / (ms_pl * 1e-3) / 1e12
    res = {"prefill_chunk64": {"ms": ms_p, "tok_per_s": T / (ms_p * 1e-3), "tflops_chunked_alg": alg / (ms_p * 1e-3) / 1e12,
                               "recurrence_only_ms": ms_pl,
                               "roofline": {"bound": "tensor", "achieved": tf_local, "peak": tf32_peak, "unit": "TFLOP/s",
                                            "frac": tf_local / tf32_peak, "per": "GPU, recurrence alone",
                                            "note": note}}}
    del q, k, v, gate, beta, gathered, full
    qd = (norm(torch.randn(Tdec, hk, d, device=dev, generator=g)) / math.sqrt(d))[:, sd.k0:sd.k1].contiguous()
    kd = norm(torch.randn(Tdec, hk, d, device=dev, generator=g))[:, sd.k0:sd.k1].contiguous()
    vd = torch.randn(Tdec, hv, d, device=dev, generator=g).index_select(1, hs).contiguous()
    gd = (-torch.nn.functional.softplus(torch.randn(Tdec, hv, device=dev, generator=g))).index_select(1, hs).contiguous()
    bd = torch.sigmoid(torch.randn(Tdec, hv, device=dev, generator=g)).index_select(1, hs).contiguous()
    od = torch.empty(Tdec, sd.hv, d, device=dev)
    gdec = torch.empty(world, sd.hv * d, device=dev)
    fdec = torch.empty(Tdec, hv * d, device=dev)

    def steps_local():
        for t in range(Tdec):
            nm.delta_step(st, qd[t], kd[t], vd[t], gd[t], bd[t], sd.hk, out=od[t])

    def steps():
        for t in range(Tdec):
            nm.delta_step(st, qd[t], kd[t], vd[t], gd[t], bd[t], sd.hk, out=od[t])
            rk.gather(od[t], gdec)
            rk.to_rows(gdec, fdec[t], world, R, sd.hk * d * 4)

    rk.checkpoint()
    ms_sl = rk.graph_ms(steps_local, 5, 1) / Tdec
    ms_s = rk.graph_ms(steps, 5, 1) / Tdec
    bytes_ = 2 * hv * d * d * 4 + 2 * hk * d * 4 + 2 * hv * d * 4 + 2 * hv * 4
    gbs_local = bytes_ / world / (ms_sl * 1e-3) / 1e9
    res["decode"] = {"us_per_step": ms_s * 1e3, "value": bytes_ / (ms_s * 1e-3) / 1e9, "unit": "GB/s",
                     "tok_per_s": 1 / (ms_s * 1e-3), "recurrence_only_us_per_step": ms_sl * 1e3,
                     "roofline": {"bound": "hbm", "achieved": gbs_local, "peak": p["hbm"], "frac": gbs_local / p["hbm"],
                                  "per": "GPU, recurrent update alone", "note": "state is L2-resident between steps"}}
    rk.checkpoint()
    return {"workload": "config 3: gated delta rule, 16 k / 32 v heads, d128, T 8192 prefill + 256 decode steps",
            "parallelism": f"key-head groups x{world} (value head h with key head h % 16), outputs all-gathered",
            "method": "prefill: 3 eager calls with CUDA events; decode: 256 steps in one CUDA graph, each step "
                      "= recurrent update + ncclAllGather + head-to-row permutation; time = max over ranks", **res}


def sharded_config4(rk, small=False):
    """Config 4 across ranks: prefill by KV head (with more ranks than KV heads,
    the two ranks of a KV head split its query heads); decode by KV head and,
    past four ranks, by batch half.  Head outputs are all-gathered into rows."""
    from hero_b200 import nm
    from hero_b200.shard import decode_shard, kv_shard

    torch, dev, world = rk.torch, rk.dev, rk.world
    hq, hkv, dh, W, S = (8, 4, 256, 1024, 1536) if small else (8, 4, 256, 1024, 8192)
    sp = kv_shard(rk.rank, world, hkv, hq)
    hkv_l, hq_l = sp.kv1 - sp.kv0, sp.q1 - sp.q0
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    rms = lambda x: x / x.float().pow(2).mean(dim=-1, keepdim=True).add(1e-6).sqrt()
    q = rms(torch.randn(S, hq, dh, device=dev, generator=g))[:, sp.q0:sp.q1].reshape(S, hq_l * dh).to(torch.bfloat16)
    k = rms(torch.randn(S, hkv, dh, device=dev, generator=g))[:, sp.kv0:sp.kv1].reshape(S, hkv_l * dh).to(torch.bfloat16)
    v = torch.randn(S, hkv, dh, device=dev, generator=g)[:, sp.kv0:sp.kv1].reshape(S, hkv_l * dh).to(torch.bfloat16)
    o = torch.empty(S, hq_l * dh, device=dev, dtype=torch.bfloat16)
    gathered = torch.empty(world, S, hq_l * dh, device=dev, dtype=torch.bfloat16)
    full = torch.empty(S, hq * dh, device=dev, dtype=torch.bfloat16)
    local = [nm.LocalAttentionCache(hkv_l, dh, W, capacity=S + W, dtype="bf16", device=dev.index) for _ in range(5)]
    glob = nm.FullAttentionCache(hkv_l, dh, capacity=S, dtype="bf16", device=dev.index)

    def layer(c, gather):
        c.reset()
        nm.append_attend(c, 0, k, v, q, None, out=o)
        if gather:
            rk.gather(o, gathered)
            rk.to_rows(gathered, full, world, S, hq_l * dh * 2)

    rk.checkpoint()
    ms_l = rk.event_ms(lambda: [layer(c, False) for c in local + [glob]], 3)
    ms = rk.event_ms(lambda: [layer(c, True) for c in local + [glob]], 3)
    pairs_g = S * (S + 1) // 2
    pairs_l = W * (W + 1) // 2 + (S - W) * W
    flops = 4.0 * dh * hq * (pairs_g + 5 * pairs_l)
    p = peaks()
    tf = flops / (ms * 1e-3) / 1e12
    tf_local = flops / world / (ms_l * 1e-3) / 1e12
    res = {"prefill": {"ms_per_group": ms, "value": tf, "unit": "TFLOP/s", "tok_per_s": S / (ms * 1e-3),
                       "attention_only_ms_per_group": ms_l,
                       "parallelism": (f"kv-head shards x{world}" if world <= hkv else
                                       f"kv-head shards x{hkv}, query heads of each group split x{world // hkv}"),
                       "roofline": {"bound": "tensor", "achieved": tf_local, "peak": p["bf16"],
                                    "frac": tf_local / p["bf16"], "per": "GPU, attention alone"}}}
    del local, glob, q, k, v, o, gathered, full
    B, L = (16, 2048) if small else (16, 32768)
    ds = decode_shard(rk.rank, world, hkv, hq, B)
    sh = ds.heads
    hkv_d, hq_d, Bl = sh.kv1 - sh.kv0, sh.q1 - sh.q0, ds.b1 - ds.b0
    gcaches, lcaches = [], []
    for b_ in range(B):
        kk = torch.randn(L, hkv, dh, device=dev, generator=g)
        vv = torch.randn(L, hkv, dh, device=dev, generator=g)
        if not ds.b0 <= b_ < ds.b1:  # every rank draws every sequence, keeps its own
            del kk, vv
            continue
        kk = kk[:, sh.kv0:sh.kv1].reshape(L, hkv_d * dh).to(torch.bfloat16)
        vv = vv[:, sh.kv0:sh.kv1].reshape(L, hkv_d * dh).to(torch.bfloat16)
        c = nm.FullAttentionCache(hkv_d, dh, capacity=L, dtype="bf16", device=dev.index)
        c.append(0, kk, vv)
        gcaches.append(c)
        lc = nm.LocalAttentionCache(hkv_d, dh, W, capacity=2 * W, dtype="bf16", device=dev.index)
        lc.append(L - W, kk[L - W:], vv[L - W:])
        lcaches.append(lc)
        del kk, vv
    qd = torch.randn(B, hq, dh, device=dev, generator=g)[ds.b0:ds.b1, sh.q0:sh.q1].reshape(Bl, hq_d * dh)
    qd = qd.to(torch.bfloat16).contiguous()
    od = torch.empty(Bl, hq_d * dh, device=dev, dtype=torch.float32)
    gd = torch.empty(world, Bl, hq_d * dh, device=dev, dtype=torch.float32)
    fd = torch.empty(B, hq * dh, device=dev, dtype=torch.float32)

    def decode(caches, gather):
        nm.attend_batch(caches, qd, None, out=od)
        if gather:
            rk.gather(od, gd)
            for part in range(ds.parts):
                rk.to_rows(gd[part * ds.kv_world:(part + 1) * ds.kv_world], fd[part * Bl:(part + 1) * Bl],
                           ds.kv_world, Bl, hq_d * dh * 4)

    rk.checkpoint()
    ms_g_l = rk.graph_ms(lambda: decode(gcaches, False), 10, 2)
    ms_g = rk.graph_ms(lambda: decode(gcaches, True), 10, 2)
    ms_w = rk.graph_ms(lambda: decode(lcaches, True), 10, 20)
    bytes_g = B * L * hkv * dh * 2 * 2
    bytes_l = B * W * hkv * dh * 2 * 2
    grp_ms = ms_g + 5 * ms_w
    gbs_local = bytes_g / world / (ms_g_l * 1e-3) / 1e9
    res["decode"] = {"global_us": ms_g * 1e3, "local_us": ms_w * 1e3, "global_attention_only_us": ms_g_l * 1e3,
                     "global_GBps": bytes_g / (ms_g * 1e-3) / 1e9, "local_GBps": bytes_l / (ms_w * 1e-3) / 1e9,
                     "group_tok_per_s": B / (grp_ms * 1e-3), "value": (bytes_g + 5 * bytes_l) / (grp_ms * 1e-3) / 1e9,
                     "unit": "GB/s",
                     "parallelism": f"kv-head shards x{ds.kv_world}" + (f", batch parts x{ds.parts}" if ds.parts > 1
                                                                       else ""),
                     "roofline": {"bound": "hbm", "achieved": gbs_local, "peak": p["hbm"], "frac": gbs_local / p["hbm"],
                                  "per": "GPU, global layer attention alone"}}
    rk.checkpoint()
    return {"workload": "config 4: Gemma hybrid bf16, 8q/4kv, d256, scale 1, 5 local (W=1024) : 1 global",
            "method": "prefill: 3 eager groups with CUDA events; decode: CUDA graphs; each layer's head outputs "
                      "all-gathered (NCCL) and permuted into rows; time = max over ranks", **res}


def sharded_config5(rk, small=False):
    """Config 5 split by KV head, as the configuration names it: each rank holds
    its KV heads of all 64 ragged f16 caches; the [64][64*128] output is
    all-gathered over NVLink."""
    from hero_b200 import nm
    from hero_b200.shard import decode_shard

    torch, dev, world = rk.torch, rk.dev, rk.world
    B, hq, hkv, dh = 64, 64, 8, 128
    lens = ragged_lengths(1, B, 4096, 131072)
    if small:  # profiling size: 8 sequences of at most 8192 rows
        B, lens = 8, [min(L, 8192) for L in lens[:8]]
    ds = decode_shard(rk.rank, world, hkv, hq, B)
    sh = ds.heads
    hkv_l, hq_l, Bl = sh.kv1 - sh.kv0, sh.q1 - sh.q0, ds.b1 - ds.b0
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rk.rank)
    caches = []
    for L in lens[ds.b0:ds.b1]:
        c = nm.FullAttentionCache(hkv_l, dh, capacity=L, dtype="f16", device=dev.index)
        chunk = 32768
        for s0 in range(0, L, chunk):
            n = min(chunk, L - s0)
            c.append(s0, torch.randn(n, hkv_l * dh, device=dev, generator=g).half(),
                     torch.randn(n, hkv_l * dh, device=dev, generator=g).half())
        caches.append(c)
    q = torch.randn(Bl, hq_l * dh, device=dev, generator=g).half()
    out = torch.empty(Bl, hq_l * dh, device=dev, dtype=torch.float32)
    gathered = torch.empty(world, Bl, hq_l * dh, device=dev, dtype=torch.float32)
    full = torch.empty(B, hq * dh, device=dev, dtype=torch.float32)
    scale = 1 / math.sqrt(dh)

    def step(gather):
        nm.attend_batch(caches, q, scale, out=out)
        if gather:
            rk.gather(out, gathered)
            for part in range(ds.parts):
                rk.to_rows(gathered[part * ds.kv_world:(part + 1) * ds.kv_world], full[part * Bl:(part + 1) * Bl],
                           ds.kv_world, Bl, hq_l * dh * 4)

    rk.checkpoint()
    ms_l = rk.graph_ms(lambda: step(False), 5, 1)
    ms = rk.graph_ms(lambda: step(True), 5, 1)
    bytes_ = 4096 * sum(lens) + 2 * B * hq * dh * 2
    gbs = bytes_ / (ms * 1e-3) / 1e9
    gbs_local = bytes_ / world / (ms_l * 1e-3) / 1e9
    p = peaks()
    rk.checkpoint()
    return {"workload": "config 5: batch 64 ragged (U[4096,131072], seed 1) decode, 64q/8kv, d128, f16 cache",
            "parallelism": f"kv-head shards x{ds.kv_world}" + (f", batch parts x{ds.parts}" if ds.parts > 1 else ""),
            "value": gbs, "unit": "GB/s", "ms_per_call": ms, "tok_per_s": B / (ms * 1e-3),
            "attention_only_ms": ms_l, "kv_bytes": 4096 * sum(lens),
            "roofline": {"bound": "hbm", "achieved": gbs_local, "peak": p["hbm"], "frac": gbs_local / p["hbm"],
                         "per": "GPU, attention kernel alone"},
            "method": "one call per CUDA graph replay: attention + ncclAllGather of the [64][64*128] fp32 output "
                      "+ head-to-row permutation; time = max over ranks"}


def sharded_extras(torch, dist, dev, rank, world):
    """The other configurations on `world` GPUs.  Every rank runs the same
    steps; a failure on any rank stops that extra on every rank at the next
    checkpoint (Ranks.checkpoint) and is reported as its error."""
    extra = {}
    rk = Ranks(torch, dist, dev, rank, world)
    for name, fn in (("config1", sharded_config1), ("config3", sharded_config3), ("config4", sharded_config4),
                     ("config5", sharded_config5)):
        try:
            res = fn(rk)
        except OtherRankFailed as e:
            res = {"error": str(e)}
        except Exception as e:  # report, never hide, a failing extra
            res = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            rk.all_ok(False)  # meets the other ranks at their next checkpoint
        extra[name] = res
        rk.release()
    rk.close()
    return extra


# ---------------------------------------------------------------- main

def _sig(x, n=4):
    return float(f"{x:.{n}g}") if isinstance(x, (int, float)) and math.isfinite(x) else x


def summarize_extras(extra):
    """One short entry per measured workload of `extra`: its value and unit, the
    roofline fraction of its dominant kernel, the CPU baseline beside it and the
    parity verdict (multi-GPU), small enough to keep the headline line compact."""
    out = {}

    def visit(path, ent):
        if not isinstance(ent, dict):
            return
        if "error" in ent:
            out[path] = {"error": str(ent["error"])[:120]}
            return
        roof = ent.get("roofline") if isinstance(ent.get("roofline"), dict) else None
        if "value" in ent or roof:
            e = {}
            if "value" in ent:
                e["value"], e["unit"] = _sig(ent["value"]), ent.get("unit") or (roof or {}).get("unit")
            elif "ms" in ent:
                e["ms"] = _sig(ent["ms"])
            if roof and "frac" in roof:
                e["frac"] = _sig(roof["frac"], 3)
            cb = ent.get("cpu_baseline")
            if isinstance(cb, dict) and "value" in cb:
                e["cpu"] = [_sig(cb["value"]), cb.get("unit"), cb.get("cores")]
            if isinstance(ent.get("parity"), dict):
                e["parity_ok"] = ent["parity"].get("ok")
            out[path] = e
        for k, v in ent.items():
            if k.endswith("_roofline") and isinstance(v, dict) and "frac" in v:  # a second kernel of the workload
                out[f"{path}.{k[:-len('_roofline')]}"] = {"value": _sig(v.get("achieved", 0.0)), "unit": "GB/s"
                                                          if v.get("bound") == "hbm" else "TFLOP/s",
                                                          "frac": _sig(v["frac"], 3)}
            elif isinstance(v, dict) and k not in ("roofline", "cpu_baseline", "parity", "clocks", "collective"):
                visit(f"{path}.{k}", v)

    for name, ent in extra.items():
        visit(name, ent)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nmg", choices=["nmg", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="headline only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--only", choices=["c1", "c2", "c3", "c4", "c5", "io", "vit", "proj"],
                    help="run one workload alone (profiling); prints its own JSON line")
    ap.add_argument("--small", action="store_true", help="with --only: profiling-sized variant")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if HKV2 % world:
        raise SystemExit(f"{world} GPUs do not divide {HKV2} KV heads")
    import hero_b200

    hero_b200.lib()  # fail loudly before any work if the CUDA library is missing
    if args.only and args.only != "c2" and world > 1:
        sharded = {"c1": sharded_config1, "c3": sharded_config3, "c4": sharded_config4, "c5": sharded_config5}
        if args.only not in sharded:
            raise SystemExit(f"--only {args.only} runs on one GPU")
        rk = Ranks(torch, dist, dev, rank, world)
        res = sharded[args.only](rk, small=args.small)
        rk.close()
        if rank == 0:
            print(json.dumps({"only": args.only, "n_gpus": world, **res}), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return
    if args.only and args.only != "c2":
        fn = {"c1": extra_config1, "c3": extra_config3, "c4": extra_config4, "c5": extra_config5,
              "io": extra_attn_io, "vit": extra_vit, "proj": extra_projections}[args.only]
        print(json.dumps({"only": args.only, "small": args.small, **fn(torch, dev, small=args.small)}), flush=True)
        return
    res = bench_prefill(args, torch, dist, rank, world, dev)
    extra = {}
    if world == 1 and not args.no_extra and not args.only:
        for name, fn in (("config1", extra_config1), ("config3", extra_config3), ("config4", extra_config4),
                         ("config5", extra_config5), ("attn_io", extra_attn_io), ("vit", extra_vit),
                         ("projections", extra_projections)):
            try:
                extra[name] = fn(torch, dev)
            except Exception as e:  # report, never hide, a failing extra
                extra[name] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            torch.cuda.empty_cache()
    if world > 1 and not args.no_extra:
        torch.cuda.empty_cache()
        extra = sharded_extras(torch, dist, dev, rank, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and extra:
        cpu_baselines(extra)
    if rank == 0 and world == 1 and not args.no_cpu:
        ref = RefSample(full=True)
        ref.run()  # warm-up
        secs = []
        while sum(secs) < 10.0 or len(secs) < 2:  # about 10 s of host work
            secs.append(ref.run())
        cpu = {"value": ref.flops / float(np.mean(secs)) / 1e12, "unit": "TFLOP/s", "cores": ref.cores,
               "kind": ref.kind, "sample": ref.sample + f", {len(secs)} timed runs",
               "seconds_per_sample": float(np.mean(secs))}
    if rank == 0:
        # The measured extras in full on their own line first; the headline
        # line last, compact, with a one-entry-per-workload summary of them.
        if extra:
            print(json.dumps({"bench_extras": extra, "n_gpus": world}), flush=True)
        line = {"metric": METRIC, "value": res["value"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (torch.randn, seeded)",
                "config": {**config2_desc(world), "rotating_sets": res["rotating_sets"]},
                "tok_per_s": res["tok_per_s"], "roofline": res["roofline"], "cpu_baseline": cpu, "e2e": res["e2e"],
                "clocks": res["clocks"], "gpu_launches": res["gpu_launches"]}
        if res.get("parity") is not None:
            line["parity_ok"] = res["parity"]["ok"]
            line["parity"] = res["parity"]
        if res.get("collective"):
            line["collective"] = res["collective"]
        if extra:
            line["extra_summary"] = summarize_extras(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
