"""Benchmark of the fused W8A8 tanh-GELU DiT MLP (config 1) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the fused gated MLP over one chunk of M = 32,760 tokens
(d = 3072, ffn = 12288; fc1 -> tanh-GELU -> per-token requant -> fc2 -> gated
residual), inputs resident in HBM. With N > 1 (torchrun, one rank per GPU) every
rank processes its own 32,760-token shard (token sharding, no data-path
collective: weak scaling); the time is the max over ranks.

Rank 0 prints one JSON line. ``value`` is whole-job tokens/s; ``e2e`` is the same
metric through the public operator with pinned host buffers copied in and out
inside the timed region; ``roofline`` describes the dominant kernel (the fc1
GEMM) against the INT8 tensor peak; ``components`` times each kernel of the
step and the fused norm-RoPE (config 3) against HBM bandwidth.

``--impl reference`` times the reference's eager CPU path (its torch-CPU
restatement under ``oracle/``) on the host cores on a bounded token sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "x-minimaxh3_b200"))
sys.path.insert(0, ROOT)

M_TOKENS, D_MODEL, D_FFN = 32760, 3072, 12288
OPS_PER_TOKEN = 4 * D_MODEL * D_FFN          # two int8 GEMMs, 2 ops per MAC
METRIC = "fused INT8/W4A8 DiT-MLP tokens/s and int8 TOPS vs B200 peak at 1/2/4/8 GPUs"
NR_BYTES_PER_TOKEN = 24576                   # Q and K rows of 3072 bf16, one read and one write each
NR_TABLE_BYTES_PER_TOKEN = 64 * 4 * 4        # fp32 [64, 2, 2] rotation table, read once per token
E2E_CHUNK = 4096                             # tokens per pipelined chunk of the host-buffer path
MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes from the committed ncu summary (profiles/traffic.json), if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons around the timed region.

    Samples carry nvidia-smi's timestamp; ``mark_start``/``mark_end`` bracket the
    timed region on the host clock, and the summary keeps the samples inside it
    (or the one nearest to it when the region is shorter than the sampling
    period)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period_ms: int = 20):
        self.index = index
        self.period_ms = period_ms
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 f"-lms={self.period_ms}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark_start(self):
        import datetime
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        import datetime
        self.t1 = datetime.datetime.now()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        import datetime
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        samples = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                samples.append((ts, float(parts[2]), float(parts[3]), float(parts[4]),
                                [nm for nm, v in zip(names, parts[6:10]) if v.lower() == "active"]))
            except ValueError:
                continue
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        inside = samples
        if self.t0 is not None and self.t1 is not None:
            inside = [s for s in samples if self.t0 <= s[0] <= self.t1]
            if not inside:  # region shorter than the sampling period: nearest sample
                mid = self.t0 + (self.t1 - self.t0) / 2
                inside = [min(samples, key=lambda s: abs((s[0] - mid).total_seconds()))]
        reasons = sorted({r for s in inside for r in s[4]})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": inside[0][2], "reasons": reasons,
                "samples": len(inside), "power_w_max": max(s[3] for s in inside), "period_ms": self.period_ms}


# ---------------------------------------------------------------------------
# profiling cases: one kernel (or one fused call) of the hot path on a chosen
# token count, for ncu captures.
#
#     python bench.py --case CASE [CASE ...] [--tokens M] [--iters N] [--time]
#
# CASE is one of ``quantize`` (fc1 input quantizer, K = 3072), ``fc1`` (INT8 GEMM
# with the GELU + row-absmax epilogue; ``fc1_bf16`` / ``fc1_i32``: the same GEMM with
# the plain dequant or the int32 epilogue), ``requant`` (fc2 input quantizer with a
# given absmax, K = 12288), ``fc2`` (INT8 GEMM with the gated-residual epilogue), ``fc2_rq``
# (the same GEMM quantizing its bf16 input itself, as the fused MLP runs it),
# ``mlp`` (the whole fused MLP call), ``mlp_w4a8`` (the config-2 W4A8 MLP call), ``mlp_swiglu``
# (the H3 SwiGLU MLP at d 5,376 / ffn 14,336, ConvRot fc1 and fc2, 8,192-token chunks),
# ``mlp_swiglu_w4`` (the same MLP on W4A8 weights in the H3 release format: group 16,
# fp8-e4m3 scales, codebook; both weights decoded per call), ``decode_w4`` (that
# format's int4 -> int8 decode of the fc1 weight, 28,672 x 5,376), ``qknorm_h3``
# (single-side QK-norm + partial RoPE of H3 K, 56 heads, rot 96, bf16 table, into an
# HND buffer), ``qkv_h3`` (the H3 Q/K/V projection of M tokens, hidden 5,376, with
# QK-norm + RoPE into HND buffers, from a ConvRot-quantized activation),
# ``convrot`` / ``convrot_x`` (ConvRot-256 + row quantization of a K = 12288 / 3072 bf16 input),
# ``norm_rope`` (AdaLN + RMSNorm + RoPE on Q and K, 24 heads x 128) or
# ``rms_adaln`` / ``rms_adaln_h3`` (standalone RMS-AdaLN on a [M, 3072] hidden stream with one
# modulation row / on H3's [M, 5376] with three segments), ``tp2_linked`` (one chunk of M tokens of the
# tensor-parallel MLP over two ranks linked on this one GPU, every stage of both ranks in order:
# its fc2 launches are ``gemm_i8_kernel<10, 2>``, the GEMM whose epilogue stores each int32 row at its
# owner; the outputs are checked against the fused MLP), ``w4_smallm`` (the W4A8 linear of M rows, at most 16,
# through fc1's config-2 weight 3,072 -> 12,288 with the asymmetric correction: ConvRot quantizer, then
# ``gemm_w4_smallm_kernel`` unpacking the int4 weight in shared memory). Shapes are those of the config-1 MLP and config-3
# norm-RoPE with M tokens; inputs are seeded synthetic data. Every case first
# runs the kernels it needs to build its inputs, then launches the kernel under
# study ``--iters`` times, so a profiler can skip the set-up launches by kernel
# name; ``--time`` also reports the mean CUDA-event time of those launches. The
# process exits non-zero if a kernel reports an error.
# ---------------------------------------------------------------------------

CASES = ["quantize", "fc1", "fc1_bf16", "fc1_i32", "requant", "fc2", "fc2_rq", "mlp", "mlp_w4a8", "mlp_swiglu",
         "mlp_swiglu_w4", "decode_w4", "qknorm_h3", "qkv_h3", "convrot", "convrot_x", "norm_rope", "rms_adaln",
         "rms_adaln_h3", "tp2_linked", "w4_smallm"]


def _case_mlp_inputs(m: int, dev):
    import torch

    import h3b200

    g = torch.Generator(device=dev).manual_seed(2)
    w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(D_MODEL, D_FFN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wt = h3b200.W8A8MLPWeights.from_float(w1, w2)
    x = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    return wt, x, gate, res


def _case_timed(fn, iters: int, report: bool):
    import torch

    if not report:
        for _ in range(iters):
            fn()
        return None
    fn()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters


def run_case(case: str, m: int, iters: int, report: bool = False):
    """Run one profiling case (see CASES); returns the mean CUDA-event ms per launch with ``report``."""
    import torch

    import h3b200
    from h3b200 import ops
    from h3b200.rope import rope_grid_table

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    h3b200.library()
    if case == "norm_rope":
        g = torch.Generator(device=dev).manual_seed(4)
        q = torch.randn(m, 24, 128, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(m, 24, 128, generator=g, device=dev).to(torch.bfloat16)
        sh = (torch.randn(3072, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        sc = (torch.randn(3072, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        wq = (1 + 0.02 * torch.randn(3072, generator=g, device=dev)).to(torch.bfloat16)
        wk = (1 + 0.02 * torch.randn(3072, generator=g, device=dev)).to(torch.bfloat16)
        grid_t = max(1, (m + 39 * 40 - 1) // (39 * 40))
        table = rope_grid_table((grid_t, 39, 40), device=dev)[:m].contiguous()
        qo, ko = torch.empty_like(q), torch.empty_like(k)
        ms = _case_timed(lambda: ops.adaln_rms_rope_(q, k, table, wq, wk, sc, sh, 1e-6, "row", 0, q_out=qo, k_out=ko),
                    iters, report)
    elif case in ("rms_adaln", "rms_adaln_h3"):
        import types

        g = torch.Generator(device=dev).manual_seed(4)
        d = 3072 if case == "rms_adaln" else 5376
        x = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        proj = (torch.randn(3, 6 * d, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        norm = types.SimpleNamespace(weight=(1 + 0.02 * torch.randn(d, generator=g, device=dev)).to(torch.bfloat16),
                                     eps=1e-6)
        segs = [(0, m, 0)] if case == "rms_adaln" else [(0, m // 8, 2), (m // 8, m // 4, 1), (m // 4, m, 0)]
        ms = _case_timed(lambda: ops.rms_adaln_segmented(x, norm, proj[:, :d], proj[:, d:2 * d], segs, out=y),
                         iters, report)
    elif case in ("convrot", "convrot_x"):
        g = torch.Generator(device=dev).manual_seed(6)
        a = torch.randn(m, D_FFN if case == "convrot" else D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        ms = _case_timed(lambda: ops.quantize_int8_rowwise_convrot(a, 256), iters, report)
    elif case == "mlp_swiglu":
        # H3 SwiGLU MLP at the H3 dims: d 5,376, fc1 out 28,672 ([gate | up]), ffn 14,336
        g = torch.Generator(device=dev).manual_seed(8)
        d, ffn = 5376, 14336
        w1 = (torch.randn(2 * ffn, d, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(d, ffn, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wt = h3b200.SwiGLUMLPWeights.from_float(w1, w2)
        del w1, w2
        x = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn(d, generator=g, device=dev).to(torch.bfloat16)
        res = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty_like(res)
        ms = _case_timed(lambda: h3b200.fused_gated_mlp_swiglu(res, x, wt, gate, out=out), iters, report)
    elif case in ("mlp_swiglu_w4", "decode_w4"):
        g = torch.Generator(device=dev).manual_seed(9)
        d, ffn = 5376, 14336
        w1 = (torch.randn(2 * ffn, d, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(d, ffn, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w4 = h3b200.W4A8SwiGLUMLPWeights.from_float(w1, w2)
        del w1, w2
        if case == "decode_w4":
            ms = _case_timed(lambda: ops.dequant_int4_grouped_to_int8(w4.q1, w4.s_rel1, 16, w4.codebook1), iters, report)
        else:
            x = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
            gate = torch.randn(d, generator=g, device=dev).to(torch.bfloat16)
            res = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty_like(res)
            ms = _case_timed(lambda: h3b200.fused_gated_mlp_swiglu_w4a8(res, x, w4, gate, out=out), iters, report)
    elif case in ("qknorm_h3", "qkv_h3"):
        g = torch.Generator(device=dev).manual_seed(10)
        heads, d = 56, 5376
        freqs = torch.randn(1, m, 1, 48, 2, 2, generator=g, device=dev).to(torch.bfloat16)
        kn = (1 + 0.02 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
        if case == "qknorm_h3":
            k = torch.randn(m, heads, 128, generator=g, device=dev).to(torch.bfloat16)
            k_hnd = torch.empty(heads, m, 128, dtype=torch.bfloat16, device=dev).permute(1, 0, 2)
            ms = _case_timed(lambda: ops.single_qknorm_rope_to_hnd(k, k_hnd, weight=kn, frequencies=freqs, eps=1e-5),
                        iters, report)
        else:
            w = (torch.randn(3 * heads * 128, d, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            wq_, ws = h3b200.quantize_int8_convrot_weight(w)
            del w
            hidden = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
            xq, xs = ops.quantize_int8_rowwise_convrot(hidden, 256)
            outs = [torch.empty(heads, m, 128, dtype=torch.bfloat16, device=dev).permute(1, 0, 2) for _ in range(3)]
            work = torch.empty(int(h3b200.library().h3b200_qkv_qknorm_rope_workspace_bytes(m, heads, 128, 0, 3)),
                               dtype=torch.uint8, device=dev)
            ms = _case_timed(lambda: ops.qkv_qknorm_rope(xq, xs, wq_, ws, None, heads, kn, kn, freqs, 1e-5, "qkv",
                                                    *outs, workspace=work), iters, report)
    elif case == "w4_smallm":
        if m > 16:
            raise SystemExit("w4_smallm: at most 16 rows (larger calls take the decode path)")
        g = torch.Generator(device=dev).manual_seed(3)
        w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        q4, s_rel, s_ch, corr = h3b200.quantize_w4a8_weight(w1, 128)
        x = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        ms = _case_timed(lambda: h3b200.w4a8_int8_linear(x, q4, s_rel, s_ch, correction=corr, group_size=128),
                         iters, report)
    elif case == "mlp_w4a8":
        g = torch.Generator(device=dev).manual_seed(3)
        w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(D_MODEL, D_FFN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w4 = h3b200.W4A8MLPWeights.from_float(w1, w2, 128)
        x = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn(D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        res = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty_like(res)
        ms = _case_timed(lambda: h3b200.fused_gated_mlp_w4a8(res, x, w4, gate, out=out), iters, report)
    else:
        wt, x, gate, res = _case_mlp_inputs(m, dev)
        xq, xs = ops.quantize_int8_rowwise(x)
        amax = torch.zeros(m, dtype=torch.float32, device=dev)
        act = torch.empty(m, D_FFN, dtype=torch.bfloat16, device=dev)
        out = torch.empty_like(res)

        def fc1():
            ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_GELU_ABSMAX, xs, wt.s1, out=act, row_absmax=amax)

        if case == "quantize":
            ms = _case_timed(lambda: ops.quantize_int8_rowwise(x), iters, report)
        elif case == "fc1":
            ms = _case_timed(fc1, iters, report)   # row absmax only grows: re-running on the same inputs is idempotent
        elif case == "fc1_bf16":
            ms = _case_timed(lambda: ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_BF16, xs, wt.s1, out=act), iters, report)
        elif case == "fc1_i32":
            acc = torch.empty(m, D_FFN, dtype=torch.int32, device=dev)
            ms = _case_timed(lambda: ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_I32, out=acc), iters, report)
        elif case in ("requant", "fc2", "fc2_rq"):
            fc1()
            if case == "fc2_rq":
                work = torch.empty(int(h3b200.library().h3b200_requant_gemm_workspace_bytes(m, D_FFN)),
                                   dtype=torch.uint8, device=dev)
                ms = _case_timed(lambda: h3b200.requant_gemm_gated_residual(act, amax, wt.w2q, wt.s2, gate, res,
                                                                            out=out, workspace=work), iters, report)
            elif case == "requant":
                ms = _case_timed(lambda: ops.quantize_int8_rowwise_absmax(act, amax), iters, report)
            else:
                q2, xs2 = ops.quantize_int8_rowwise_absmax(act, amax)
                ms = _case_timed(lambda: ops.int8_gemm_fused(q2, wt.w2q, ops.EPI_GATED_RESIDUAL, xs2, wt.s2, gate=gate,
                                                        residual=res, out=out), iters, report)
        elif case == "mlp":
            ms = _case_timed(lambda: h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=out), iters,
                        report)
        elif case == "tp2_linked":
            from h3b200 import parallel as PAR

            world = 2
            comms = PAR.TPComm.linked_local(world, m, D_MODEL, D_FFN // world)
            shards = [PAR.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, world, r) for r in range(world)]
            outs = [torch.empty_like(res) for _ in range(world)]
            chunk = [0]

            def tp_step():
                for stage in (1, 2, 3, 4):
                    for r in range(world):
                        comms[r].stage(stage, chunk[0], x, res, gate, shards[r], outs[r], 0, m)
                chunk[0] += 1

            ms = _case_timed(tp_step, iters, report)
            ref = h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate)
            torch.cuda.synchronize()
            if not all(bool(torch.equal(o, ref)) for o in outs):
                raise SystemExit("tp2_linked: a rank's output differs from the fused MLP")
            for c in comms:
                c.close()
        else:
            raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    st = h3b200.device_status(0)
    if st != 0:
        raise SystemExit(f"device status {st:#x}")
    return ms


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------


def _cpu_mlp_inputs(rows, seed=2):
    import torch

    from oracle import torch_port as P

    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(D_FFN, D_MODEL, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(D_MODEL, D_FFN, generator=g) * 0.02).to(torch.bfloat16)
    w1q, s1 = P.quantize_int8_rowwise(w1)
    w2q, s2 = P.quantize_int8_rowwise(w2)
    x = torch.randn(rows, D_MODEL, generator=g).to(torch.bfloat16)
    gate = torch.randn(D_MODEL, generator=g).to(torch.bfloat16)
    res = torch.randn(rows, D_MODEL, generator=g).to(torch.bfloat16)
    return x, w1q, s1.reshape(-1), w2q, s2.reshape(-1), gate, res


CPU_ROWS = 2048          # config-1 tokens per CPU sample (per-token math, so a row sample is representative)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_protocol() -> dict:
    """Host description recorded beside every CPU number."""
    import torch

    return {"os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "cpu_model": cpu_model()}


def cpu_mlp_tokens_per_s(rows: int = CPU_ROWS, repeats: int = 3):
    """Median tokens/s of the torch-CPU port of the reference eager MLP on `rows` tokens
    (1 warm-up, median of `repeats`), all host threads."""
    import torch

    from oracle import torch_port as P

    torch.set_num_threads(os.cpu_count() or 1)
    args = _cpu_mlp_inputs(rows)
    P.w8a8_gelu_mlp(*args)  # warm-up
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        P.w8a8_gelu_mlp(*args)
        times.append(time.perf_counter() - t0)
    return rows / statistics.median(times), torch.get_num_threads()


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import torch

    from oracle import torch_port as P

    torch.set_num_threads(os.cpu_count() or 1)
    # the same sample as our arm's cpu_baseline: 2,048 config-1 tokens per step (about 0.15 s of
    # CPU work on a 16-thread host, so 200 steps stay within a minute or two)
    rows = CPU_ROWS
    x, w1q, s1, w2q, s2, gate, res = _cpu_mlp_inputs(rows)
    for _ in range(max(1, args.warmup)):
        P.w8a8_gelu_mlp(x, w1q, s1, w2q, s2, gate, res)
    per_step = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        P.w8a8_gelu_mlp(x, w1q, s1, w2q, s2, gate, res)
        per_step.append(time.perf_counter() - t0)
    dt = sum(per_step)
    value = rows * args.steps / dt
    cores = torch.get_num_threads()
    sample = (f"{rows} of {M_TOKENS} config-1 tokens per step (per-token math; torch-CPU port of the eager path); "
              f"median step {rows / statistics.median(per_step):.0f} tokens/s")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
        "config": {"workload": "cfg1 fused W8A8 tanh-GELU DiT MLP, d=3072 ffn=12288", "tokens_per_step": rows,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
                         **cpu_protocol()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "int8_tops": value * OPS_PER_TOKEN / 1e12,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def timed(fn, reps, stream):
    import torch

    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / reps


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import h3b200
    from h3b200 import ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    h3b200.library()
    stream = torch.cuda.current_stream(dev)

    # weights: identical on every rank (seeded), quantized per channel on the GPU
    g = torch.Generator(device=dev).manual_seed(2)
    w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(D_MODEL, D_FFN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wt = h3b200.W8A8MLPWeights.from_float(w1, w2)
    del w1, w2
    # this rank's token shard
    gs = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(M_TOKENS, D_MODEL, generator=gs, device=dev).to(torch.bfloat16)
    res = torch.randn(M_TOKENS, D_MODEL, generator=gs, device=dev).to(torch.bfloat16)
    gate = torch.randn(D_MODEL, generator=gs, device=dev).to(torch.bfloat16)
    out = torch.empty_like(res)
    ws_bytes = int(h3b200.library().h3b200_fused_gated_mlp_workspace_bytes(M_TOKENS, D_MODEL, D_FFN))
    work = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)

    def step():
        h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=out, workspace=work)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        clk.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
        clk.mark_end()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = world * M_TOKENS * args.steps / (ms / 1e3)

    # ---- the same step over a timed region of at least 1.5 s (steady state under the power cap) ----
    sus_steps = max(args.steps, int(1500.0 / max(ms_per_step, 1e-3)) + 1)
    with ClockSampler(local_rank, period_ms=100) as clk_sus:
        ev0.record(stream)
        clk_sus.mark_start()
        for _ in range(sus_steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
        clk_sus.mark_end()
    sus_ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([sus_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sus_ms = float(t.item())
    sustained = {"steps": sus_steps, "ms_per_step": sus_ms / sus_steps,
                 "tokens_per_s": world * M_TOKENS * sus_steps / (sus_ms / 1e3), "clocks": clk_sus.summary()}
    status = h3b200.device_status(local_rank)

    # ---- per-kernel timing of the same step (events around each launch) ----
    xq = torch.empty(M_TOKENS, D_MODEL, dtype=torch.int8, device=dev)
    xs = torch.empty(M_TOKENS, 1, dtype=torch.float32, device=dev)
    amax = torch.zeros(M_TOKENS, dtype=torch.float32, device=dev)
    act = torch.empty(M_TOKENS, D_FFN, dtype=torch.bfloat16, device=dev)
    q2 = torch.empty(M_TOKENS, D_FFN, dtype=torch.int8, device=dev)
    xs2 = torch.empty(M_TOKENS, 1, dtype=torch.float32, device=dev)
    lib = h3b200.library()
    sp = stream.cuda_stream

    def k_quant():
        lib.h3b200_quantize_int8_rowwise(x.data_ptr(), M_TOKENS, D_MODEL, D_MODEL, 0, xq.data_ptr(), xs.data_ptr(), sp)

    def k_fc1():
        ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_GELU_ABSMAX, xs, wt.s1, out=act, row_absmax=amax)

    def k_requant():
        lib.h3b200_quantize_int8_rowwise_absmax(act.data_ptr(), amax.data_ptr(), M_TOKENS, D_FFN, D_FFN,
                                                q2.data_ptr(), xs2.data_ptr(), sp)

    def k_fc2():
        ops.int8_gemm_fused(q2, wt.w2q, ops.EPI_GATED_RESIDUAL, xs2, wt.s2, gate=gate, residual=res, out=out)

    rq_work = torch.empty(int(lib.h3b200_requant_gemm_workspace_bytes(M_TOKENS, D_FFN)), dtype=torch.uint8,
                          device=dev)

    def k_fc2_rq():
        h3b200.requant_gemm_gated_residual(act, amax, wt.w2q, wt.s2, gate, res, out=out, workspace=rq_work)

    for f in (k_quant, k_fc1, k_requant, k_fc2, k_fc2_rq):
        f()
    reps = 20
    # the step runs quantize_x, fc1 and fc2_requant_gated_residual (fc2 quantizing its input
    # itself); the separate requant kernel and plain fc2 are timed for comparison
    comp_ms = {name: timed(f, reps, stream) for name, f in
               (("quantize_x", k_quant), ("fc1_gemm_gelu_absmax", k_fc1),
                ("fc2_requant_gated_residual", k_fc2_rq), ("requant_fc2_input", k_requant),
                ("fc2_gemm_gated_residual", k_fc2))}
    fc1_ops = 2.0 * M_TOKENS * D_MODEL * D_FFN
    fc2_ops = fc1_ops

    # ---- fused norm-RoPE (config 3), HBM-bound ----
    from h3b200.rope import rope_grid_table

    gn = torch.Generator(device=dev).manual_seed(4)
    qn = torch.randn(M_TOKENS, 24, 128, generator=gn, device=dev).to(torch.bfloat16)
    kn = torch.randn(M_TOKENS, 24, 128, generator=gn, device=dev).to(torch.bfloat16)
    sh = (torch.randn(3072, generator=gn, device=dev) * 0.1).to(torch.bfloat16)
    sc = (torch.randn(3072, generator=gn, device=dev) * 0.1).to(torch.bfloat16)
    wq = (1 + 0.02 * torch.randn(3072, generator=gn, device=dev)).to(torch.bfloat16)
    wk = (1 + 0.02 * torch.randn(3072, generator=gn, device=dev)).to(torch.bfloat16)
    table = rope_grid_table((21, 39, 40), device=dev)
    qo = torch.empty_like(qn)
    ko = torch.empty_like(kn)

    def k_nr():
        ops.adaln_rms_rope_(qn, kn, table, wq, wk, sc, sh, 1e-6, "row", 0, q_out=qo, k_out=ko)

    for _ in range(3):
        k_nr()
    nr_ms = timed(k_nr, 50, stream)
    nr_bytes = M_TOKENS * NR_BYTES_PER_TOKEN

    # ---- standalone RMS-AdaLN on the hidden stream, HBM-bound: config-3 shape [32,760, 3,072] with one
    #      modulation row, and H3's width 5,376 with three modulation segments (kernels.py:7586) ----
    import types

    xa = torch.randn(M_TOKENS, D_MODEL, generator=gn, device=dev).to(torch.bfloat16)
    ya = torch.empty_like(xa)
    norm_a = types.SimpleNamespace(weight=wq, eps=1e-6)

    def k_ra():
        ops.rms_adaln_segmented(xa, norm_a, sh.reshape(1, -1), sc.reshape(1, -1), [(0, M_TOKENS, 0)], out=ya)

    for _ in range(3):
        k_ra()
    ra_ms = timed(k_ra, 50, stream)
    ra_bytes = M_TOKENS * D_MODEL * 4
    del xa, ya
    xh = torch.randn(M_TOKENS, 5376, generator=gn, device=dev).to(torch.bfloat16)
    yh = torch.empty_like(xh)
    projh = (torch.randn(3, 6 * 5376, generator=gn, device=dev) * 0.1).to(torch.bfloat16)
    norm_h = types.SimpleNamespace(weight=(1 + 0.02 * torch.randn(5376, generator=gn, device=dev)).to(torch.bfloat16),
                                   eps=1e-6)
    segs_h = [(0, 1024, 2), (1024, 2048, 1), (2048, M_TOKENS, 0)]

    def k_ra_h3():
        ops.rms_adaln_segmented(xh, norm_h, projh[:, :5376], projh[:, 5376:2 * 5376], segs_h, out=yh)

    for _ in range(3):
        k_ra_h3()
    rah_ms = timed(k_ra_h3, 50, stream)
    rah_bytes = M_TOKENS * 5376 * 4
    del xh, yh

    # ---- config 2: fused W4A8 MLP (reference's asymmetric group-128 format, int4 at rest) ----
    g3 = torch.Generator(device=dev).manual_seed(3)
    w1f = (torch.randn(D_FFN, D_MODEL, generator=g3, device=dev) * 0.02).to(torch.bfloat16)
    w2f = (torch.randn(D_MODEL, D_FFN, generator=g3, device=dev) * 0.02).to(torch.bfloat16)
    w4 = h3b200.W4A8MLPWeights.from_float(w1f, w2f, 128)
    del w1f, w2f
    x3 = torch.randn(M_TOKENS, D_MODEL, generator=g3, device=dev).to(torch.bfloat16)
    ws4 = int(h3b200.library().h3b200_fused_gated_mlp_w4a8_workspace_bytes(M_TOKENS, D_MODEL, D_FFN, 128))
    work4 = torch.empty(ws4, dtype=torch.uint8, device=dev)

    def k_w4a8():
        h3b200.fused_gated_mlp_w4a8(res, x3, w4, gate, out=out, workspace=work4)

    for _ in range(3):
        k_w4a8()
    w4_ms = timed(k_w4a8, 10, stream)
    del work4, x3

    # ---- small-M W4A8 linear (fc1's weight, 3,072 -> 12,288, same format): the packed int4 weight
    #      unpacked in shared memory inside the GEMM (split-K) against decode-per-call + INT8 GEMM;
    #      CUDA graphs of 10 calls so that host overhead is not timed ----
    def graph_ms(fn, calls=10, reps=5):
        fn()
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            for _ in range(calls):
                fn()
        gph.replay()
        torch.cuda.synchronize()
        ms = timed(gph.replay, reps, stream) / calls
        del gph
        return ms

    small_m = {}
    grid1 = torch.empty(D_FFN, D_MODEL, dtype=torch.int8, device=dev)
    for mm in (1, 8, 16):
        xs_ = torch.randn(mm, D_MODEL, generator=g3, device=dev).to(torch.bfloat16)
        ys_ = torch.empty(mm, D_FFN, dtype=torch.bfloat16, device=dev)
        wpk = torch.empty(int(lib.h3b200_w4a8_linear_packed_workspace_bytes(mm, D_FFN, D_MODEL, 128)),
                          dtype=torch.uint8, device=dev)
        wgd = torch.empty(int(lib.h3b200_w4a8_linear_workspace_bytes(mm, D_FFN, D_MODEL, 128)), dtype=torch.uint8,
                          device=dev)

        def k_packed():
            lib.h3b200_w4a8_int8_linear_packed(xs_.data_ptr(), D_MODEL, w4.q1.data_ptr(), w4.s_rel1.data_ptr(), 0,
                                               None, w4.s_ch1.data_ptr(), w4.corr1.data_ptr(), None, 128, 256, 0,
                                               ys_.data_ptr(), mm, D_FFN, D_MODEL, wpk.data_ptr(), wpk.numel(),
                                               torch.cuda.current_stream().cuda_stream)

        def k_decoded():
            lib.h3b200_dequant_int4_grouped_to_int8_ex(w4.q1.data_ptr(), w4.s_rel1.data_ptr(), 0, None, D_FFN, D_MODEL,
                                                       128, grid1.data_ptr(), torch.cuda.current_stream().cuda_stream)
            lib.h3b200_w4a8_int8_linear(xs_.data_ptr(), D_MODEL, grid1.data_ptr(), w4.s_ch1.data_ptr(),
                                        w4.corr1.data_ptr(), None, 128, 256, 0, ys_.data_ptr(), mm, D_FFN, D_MODEL,
                                        wgd.data_ptr(), wgd.numel(), torch.cuda.current_stream().cuda_stream)

        small_m[str(mm)] = {"packed_in_smem_us": 1e3 * graph_ms(k_packed), "decode_then_gemm_us": 1e3 * graph_ms(k_decoded)}
        del xs_, ys_, wpk, wgd
    del grid1

    # ---- H3 SwiGLU MLP at the H3 dims (d 5,376, fc1 out 28,672, ffn 14,336): ConvRot fc1 + bias,
    #      SwiGLU+ConvRot fc2 + bias, gated residual; 8,192-token chunks as in the reference ----
    H3_D, H3_FFN = 5376, 14336
    g5 = torch.Generator(device=dev).manual_seed(8)
    w1f = (torch.randn(2 * H3_FFN, H3_D, generator=g5, device=dev) * 0.02).to(torch.bfloat16)
    w2f = (torch.randn(H3_D, H3_FFN, generator=g5, device=dev) * 0.02).to(torch.bfloat16)
    b1f = (torch.randn(2 * H3_FFN, generator=g5, device=dev) * 0.1).to(torch.bfloat16)
    b2f = (torch.randn(H3_D, generator=g5, device=dev) * 0.1).to(torch.bfloat16)
    wsw = h3b200.SwiGLUMLPWeights.from_float(w1f, w2f, b1f, b2f)
    # the same MLP in the H3 release W4A8 format (group 16, fp8-e4m3 scales, codebook)
    wsw4 = h3b200.W4A8SwiGLUMLPWeights.from_float(w1f, w2f, b1f, b2f)
    del w1f, w2f
    x5 = torch.randn(M_TOKENS, H3_D, generator=g5, device=dev).to(torch.bfloat16)
    r5 = torch.randn(M_TOKENS, H3_D, generator=g5, device=dev).to(torch.bfloat16)
    o5 = torch.empty_like(r5)
    gate5 = torch.randn(2, H3_D, generator=g5, device=dev).to(torch.bfloat16)
    segs5 = [(0, 1024, 1), (1024, M_TOKENS, 0)]   # a conditioning prefix with its own modulation row
    wsb5 = int(h3b200.library().h3b200_fused_gated_mlp_swiglu_workspace_bytes(8192, H3_D, H3_FFN))
    work5 = torch.empty(wsb5, dtype=torch.uint8, device=dev)

    def k_swiglu():
        h3b200.fused_gated_mlp_swiglu(r5, x5, wsw, gate5, segments=segs5, out=o5, workspace=work5)

    for _ in range(3):
        k_swiglu()
    sw_ms = timed(k_swiglu, 10, stream)
    sw_ops = 2 * H3_D * 2 * H3_FFN + 2 * H3_FFN * H3_D   # int8 ops per token
    del work5, wsw
    work5 = torch.empty(int(h3b200.library().h3b200_fused_gated_mlp_swiglu_w4a8_workspace_bytes(8192, H3_D, H3_FFN)),
                        dtype=torch.uint8, device=dev)

    def k_swiglu_w4():
        h3b200.fused_gated_mlp_swiglu_w4a8(r5, x5, wsw4, gate5, segments=segs5, out=o5, workspace=work5)

    for _ in range(3):
        k_swiglu_w4()
    sw4_ms = timed(k_swiglu_w4, 10, stream)
    del work5, r5, o5, wsw4

    # ---- H3 attention build: Q/K/V projection (hidden 5,376 -> 3 x 56 heads x 128, ConvRot INT8)
    #      from the activation quantized once, per-head QK-norm + RoPE over 96 dims (bf16 table)
    #      into HND attention buffers, 8,192-token chunks as the reference's projection chunks ----
    H3_HEADS = 56
    g6 = torch.Generator(device=dev).manual_seed(10)
    wqkv = (torch.randn(3 * H3_HEADS * 128, H3_D, generator=g6, device=dev) * 0.02).to(torch.bfloat16)
    wqkv_q, wqkv_s = h3b200.quantize_int8_convrot_weight(wqkv)
    del wqkv
    bqkv = (torch.randn(3 * H3_HEADS * 128, generator=g6, device=dev) * 0.1).to(torch.bfloat16)
    qn6 = (1 + 0.02 * torch.randn(128, generator=g6, device=dev)).to(torch.bfloat16)
    kn6 = (1 + 0.02 * torch.randn(128, generator=g6, device=dev)).to(torch.bfloat16)
    tab6 = rope_grid_table((21, 39, 40), dims=(32, 32, 32), device=dev).to(torch.bfloat16)
    tab6 = tab6.reshape(1, M_TOKENS, 1, 48, 2, 2)
    hnd6 = [torch.empty(H3_HEADS, M_TOKENS, 128, dtype=torch.bfloat16, device=dev) for _ in range(3)]
    chunk6 = 8192
    work6 = torch.empty(int(h3b200.library().h3b200_qkv_qknorm_rope_workspace_bytes(chunk6, H3_HEADS, 128, 0, 3)),
                        dtype=torch.uint8, device=dev)

    def k_qkv():
        xq6, xs6 = ops.quantize_int8_rowwise_convrot(x5, 256)
        for a in range(0, M_TOKENS, chunk6):
            b = min(M_TOKENS, a + chunk6)
            ops.qkv_qknorm_rope(xq6[a:b], xs6[a:b], wqkv_q, wqkv_s, bqkv, H3_HEADS, qn6, kn6, tab6[:, a:b], 1e-5,
                                "qkv", *(h[:, a:b].permute(1, 0, 2) for h in hnd6), workspace=work6)

    for _ in range(3):
        k_qkv()
    qkv_ms = timed(k_qkv, 10, stream)
    qkv_ops = 2 * H3_D * 3 * H3_HEADS * 128   # int8 ops per token
    k6 = torch.randn(M_TOKENS, H3_HEADS, 128, generator=g6, device=dev).to(torch.bfloat16)

    def k_qk1():
        ops.single_qknorm_rope_to_hnd(k6, hnd6[1].permute(1, 0, 2), weight=kn6, frequencies=tab6, eps=1e-5)

    for _ in range(3):
        k_qk1()
    qk1_ms = timed(k_qk1, 20, stream)
    qk1_bytes = M_TOKENS * H3_HEADS * 128 * 2 * 2
    del work6, hnd6, k6, wqkv_q, x5

    # ---- config 4: long-video DiT-block slice (norm-RoPE then W8A8 MLP) on this rank's token shard ----
    from h3b200 import parallel as PAR

    M4, GRID4 = 196560, (45, 52, 84)
    lo4, hi4 = PAR.shard_range(M4, world, rank)
    m4 = hi4 - lo4
    g5 = torch.Generator(device=dev).manual_seed(5 + rank)
    q4 = torch.randn(m4, 24, 128, generator=g5, device=dev).to(torch.bfloat16)
    k4 = torch.randn(m4, 24, 128, generator=g5, device=dev).to(torch.bfloat16)
    x4 = torch.randn(m4, D_MODEL, generator=g5, device=dev).to(torch.bfloat16)
    r4 = torch.randn(m4, D_MODEL, generator=g5, device=dev).to(torch.bfloat16)
    o4 = torch.empty_like(r4)
    table4 = rope_grid_table(GRID4, token_slice=(lo4, hi4), device=dev)
    work5 = torch.empty(int(h3b200.library().h3b200_fused_gated_mlp_workspace_bytes(m4, D_MODEL, D_FFN)),
                        dtype=torch.uint8, device=dev)

    def k_block():
        ops.adaln_rms_rope_(q4, k4, table4, wq, wk, sc, sh, 1e-6, "row", 0)
        h3b200.fused_gated_mlp(r4, x4, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=o4, workspace=work5)

    for _ in range(2):
        k_block()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    blk_ms = timed(k_block, 5, stream)
    if world > 1:
        t = torch.tensor([blk_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        blk_ms = float(t.item())
    del q4, k4, x4, r4, o4, table4, work5

    # ---- config 4, tensor-parallel MLP: all 196,560 tokens replicated on every rank, W1 rows and
    #      W2 columns split N ways, 32,768-token chunks; strong scaling (total work fixed). "p2p": the
    #      exchanges inside the kernels over NVLink peer memory (absmax push + flag barrier, fc2 rows
    #      stored at their owners, owner pass pushing finished rows); the NCCL forms (int32
    #      reduce-scatter + bf16 all-gather, or int32 all-reduce) are timed beside it ----
    gt = torch.Generator(device=dev).manual_seed(6)      # the same replicated inputs on every rank
    xt = torch.randn(M4, D_MODEL, generator=gt, device=dev).to(torch.bfloat16)
    rt = torch.randn(M4, D_MODEL, generator=gt, device=dev).to(torch.bfloat16)
    ot = torch.empty_like(rt)
    tp_shard = PAR.TPShard.from_full(wt.w1q, wt.s1, wt.w2q, wt.s2, world, rank)
    TP_CHUNK = 32768  # fewer barriers and GEMM tails than 8,192 (N = 2: 7.70 vs 9.88 ms)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tp_ms, tp_err = {}, None
    for coll in (PAR.COLLECTIVES if world > 1 else ("p2p",)):
        def k_tp(coll=coll):
            PAR.tp_gated_mlp(xt, rt, gate, tp_shard, chunk_tokens=TP_CHUNK, out=ot, collective=coll)

        try:
            k_tp()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            tp_ms[coll] = max_over_ranks(timed(k_tp, 3, stream))
        except Exception as e:  # recorded in the component; the rest of the line is still measured
            tp_err = f"{coll}: {type(e).__name__}: {e}"[:300]
            torch.cuda.synchronize()
            if h3b200.device_status(dev.index):
                h3b200.device_status(dev.index, clear=True)
    # the collectives of one TP step alone (same sizes, same order), to see what bounds the curve
    tp_coll_ms = None
    if world > 1:
        nchunk = -(-M4 // TP_CHUNK)
        am_t = torch.zeros(TP_CHUNK, dtype=torch.float32, device=dev)
        acc_t = torch.zeros(TP_CHUNK, D_MODEL, dtype=torch.int32, device=dev)
        part_t = torch.empty(TP_CHUNK // world, D_MODEL, dtype=torch.int32, device=dev)
        loc_t = torch.empty(TP_CHUNK // world, D_MODEL, dtype=torch.bfloat16, device=dev)
        gat_t = torch.empty(TP_CHUNK, D_MODEL, dtype=torch.bfloat16, device=dev)

        def k_coll():
            for _ in range(nchunk):
                dist.all_reduce(am_t, op=dist.ReduceOp.MAX)
                dist.reduce_scatter_tensor(part_t, acc_t, op=dist.ReduceOp.SUM)
                dist.all_gather_into_tensor(gat_t, loc_t)

        k_coll()
        torch.cuda.synchronize()
        dist.barrier()
        tp_coll_ms = max_over_ranks(timed(k_coll, 3, stream))
        del am_t, acc_t, part_t, loc_t, gat_t
    del xt, rt, ot, tp_shard
    try:
        PAR.close_tp_comms()  # every rank: the peer-memory exchange regions of the p2p form
    except Exception as e:
        tp_err = tp_err or f"close: {type(e).__name__}: {e}"[:300]

    # ---- library INT8 reference: cuBLASLt through torch._int_mm, 8192^3, same box and run ----
    lib_int8_tops = None
    try:
        ga = torch.Generator(device=dev).manual_seed(7)
        ia = torch.randint(-128, 128, (8192, 8192), generator=ga, device=dev, dtype=torch.int8)
        ib = torch.randint(-128, 128, (8192, 8192), generator=ga, device=dev, dtype=torch.int8).t()
        for _ in range(3):
            torch._int_mm(ia, ib)
        lib_ms = timed(lambda: torch._int_mm(ia, ib), 10, stream)
        lib_int8_tops = 2.0 * 8192 ** 3 / (lib_ms * 1e-3) / 1e12
        del ia, ib
    except Exception:
        lib_int8_tops = None

    peaks, peak_src = load_peaks()
    int8_peak_tops = 2.0 * peaks["bf16_tflops"]
    traffic = load_traffic()
    fc1_tops = fc1_ops / (comp_ms["fc1_gemm_gelu_absmax"] * 1e-3) / 1e12
    nr_gbs = nr_bytes / (nr_ms * 1e-3) / 1e9

    # ---- end to end through the public operator with host buffers ----
    x_h = x.cpu().pin_memory()
    r_h = res.cpu().pin_memory()
    o_h = torch.empty(M_TOKENS, D_MODEL, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        # public host-buffer entry point: chunked H2D / MLP / D2H on three overlapped streams
        h3b200.fused_gated_mlp_host(r_h, x_h, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=o_h,
                                    chunk_tokens=E2E_CHUNK, synchronize=False)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 20))
    if world > 1:
        dist.barrier()
    e2e_ms = timed(e2e_step, e2e_steps, stream)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * M_TOKENS / (e2e_ms * 1e-3)
    h2d = x.numel() * 2 + res.numel() * 2
    d2h = out.numel() * 2

    # ---- CPU baseline (rank 0, N = 1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores = cpu_mlp_tokens_per_s(CPU_ROWS)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{CPU_ROWS} config-1 tokens, median of 3 after 1 warm-up (torch-CPU port of the eager "
                         "path; the reference arm runs the same 2,048-token sample per step)",
               **cpu_protocol()}

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded N(0,1) activations/gate/residual, N(0,0.02) weights, per-channel int8)",
            "config": {"workload": "cfg1 fused W8A8 tanh-GELU DiT MLP (fc1 -> GELU -> requant -> fc2 -> gated residual)",
                       "tokens_per_gpu": M_TOKENS, "d": D_MODEL, "ffn": D_FFN, "parallelism": f"token-shard x{world}",
                       "l2": "inputs larger than L2 (x, residual 201 MB each); int8 weights (75 MB) stay L2-resident"},
            "int8_tops": value * OPS_PER_TOKEN / 1e12,
            "roofline": {"kernel": "gemm_i8_kernel<fc1: GELU+absmax epilogue>", "bound": "tensor",
                         "achieved": fc1_tops, "peak": int8_peak_tops, "unit": "TOP/s",
                         "frac": fc1_tops / int8_peak_tops,
                         "peak_source": f"2 x {peak_src} bf16 dense burst ({peaks['bf16_tflops']} TF/s); "
                                        "tcgen05 kind::i8 issues at twice the kind::f16 rate",
                         "traffic": traffic.get("fc1_gemm_gelu_absmax")},
            "components": {
                "sustained_step": sustained,
                **{k: {"ms": v} for k, v in comp_ms.items()},
                "fc2_gemm_gated_residual_tops": fc2_ops / (comp_ms["fc2_gemm_gated_residual"] * 1e-3) / 1e12,
                "cublaslt_int8_8192_tops": lib_int8_tops,
                "h3_swiglu_mlp": {"d": H3_D, "ffn": H3_FFN, "tokens": M_TOKENS, "ms": sw_ms,
                                  "tokens_per_s": M_TOKENS / (sw_ms * 1e-3),
                                  "int8_tops": M_TOKENS * sw_ops / (sw_ms * 1e-3) / 1e12},
                "h3_swiglu_mlp_w4a8": {"d": H3_D, "ffn": H3_FFN, "tokens": M_TOKENS, "ms": sw4_ms,
                                       "tokens_per_s": M_TOKENS / (sw4_ms * 1e-3),
                                       "int8_tops": M_TOKENS * sw_ops / (sw4_ms * 1e-3) / 1e12,
                                       "weights": "H3 release W4A8: int4 group 16, fp8-e4m3 s_rel, 16-level "
                                                  "codebook, ConvRot-256; both weights decoded per call"},
                "h3_qkv_qknorm_rope_hnd": {"heads": H3_HEADS, "d": H3_D, "tokens": M_TOKENS, "ms": qkv_ms,
                                           "tokens_per_s": M_TOKENS / (qkv_ms * 1e-3),
                                           "int8_tops": M_TOKENS * qkv_ops / (qkv_ms * 1e-3) / 1e12,
                                           "path": "ConvRot quantize once; per 8,192-token chunk INT8 GEMM [Q|K|V], "
                                                   "QK-norm + RoPE(96) of Q and K into HND, V into HND"},
                "h3_single_qknorm_rope_hnd": {"heads": H3_HEADS, "tokens": M_TOKENS, "ms": qk1_ms,
                                              "achieved": qk1_bytes / (qk1_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                                              "unit": "GB/s", "frac": qk1_bytes / (qk1_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                              "bytes_per_token": H3_HEADS * 128 * 2 * 2},
                "w4a8_linear_small_m": {"shape": "x [m, 3072] . W4 [12288, 3072]^T, asymmetric int4 group 128 + "
                                                 "correction, ConvRot-256; microseconds per call (CUDA graphs)",
                                        "by_m": small_m,
                                        "weight_bytes_int4": D_FFN * D_MODEL // 2},
                "w4a8_mlp_cfg2": {"ms": w4_ms, "tokens_per_s": M_TOKENS / (w4_ms * 1e-3),
                                  "int8_tops": M_TOKENS * OPS_PER_TOKEN / (w4_ms * 1e-3) / 1e12,
                                  "weights": "asymmetric int4, group 128, ConvRot-256, decoded per call"},
                "tp_mlp_cfg4": {"tokens_total": M4, "tensor_parallel": world, "chunk_tokens": TP_CHUNK,
                                "ms": tp_ms.get("p2p"),
                                "tokens_per_s": M4 / (tp_ms["p2p"] * 1e-3) if tp_ms.get("p2p") else None,
                                "int8_tops": M4 * OPS_PER_TOKEN / (tp_ms["p2p"] * 1e-3) / 1e12 if tp_ms.get("p2p") else None,
                                "error": tp_err,
                                "collective": ("in-kernel over NVLink peer memory: absmax push + flag barrier, fc2 "
                                               "int32 rows stored at their owners, owner rows pushed to every rank"
                                               if world > 1 else "none (one rank: the fused MLP per chunk)"),
                                "nccl_reduce_scatter_variant_ms": tp_ms.get("reduce_scatter"),
                                "nccl_all_reduce_variant_ms": tp_ms.get("all_reduce"),
                                "nccl_collectives_alone_ms": tp_coll_ms,
                                "scaling": "strong (196,560 tokens in total at every N)"},
                "long_video_block_cfg4": {"tokens_total": M4, "tokens_this_rank": m4, "ms": blk_ms,
                                          "tokens_per_s": M4 / (blk_ms * 1e-3),
                                          "mode": f"token-shard x{world} (norm-RoPE + W8A8 MLP per rank)"},
                "rms_adaln_cfg3": {"ms": ra_ms, "achieved": ra_bytes / (ra_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                                   "unit": "GB/s", "frac": ra_bytes / (ra_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                   "bytes_per_token": D_MODEL * 4, "tokens": M_TOKENS,
                                   "form": "RMSNorm(weight) -> *(1+scale) -> +shift, one modulation row"},
                "rms_adaln_h3_3seg": {"ms": rah_ms, "achieved": rah_bytes / (rah_ms * 1e-3) / 1e9,
                                      "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                      "frac": rah_bytes / (rah_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                      "bytes_per_token": 5376 * 4, "tokens": M_TOKENS,
                                      "form": "H3 width 5,376, three modulation segments (strided split_adaln views)"},
                "norm_rope_cfg3": {"ms": nr_ms, "achieved": nr_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                   "frac": nr_gbs / peaks["hbm_gbs"], "bytes_per_token": NR_BYTES_PER_TOKEN,
                                   "table_bytes_per_token": NR_TABLE_BYTES_PER_TOKEN,
                                   "traffic": traffic.get("norm_rope_cfg3")},
            },
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "h3b200.fused_gated_mlp_host (pinned host buffers, chunked copy/compute overlap)",
                    "chunk_tokens": E2E_CHUNK},
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
            "device_status": status,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    final = h3b200.device_status(local_rank)
    if status or final:
        print(f"bench: device status {max(status, final):#x}: a bounded device wait expired; numbers are not valid",
              file=sys.stderr, flush=True)
        return 3
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", nargs="+", choices=CASES, help="run profiling cases instead of the benchmark")
    ap.add_argument("--tokens", type=int, default=8192, help="tokens per profiling case")
    ap.add_argument("--iters", type=int, default=3, help="launches of the studied kernel per profiling case")
    ap.add_argument("--time", action="store_true", help="report the mean CUDA-event ms per launch of each case")
    args = ap.parse_args()
    if args.case:
        for case in args.case:
            ms = run_case(case, args.tokens, args.iters, args.time)
            extra = f" mean {ms:.4f} ms per launch" if ms is not None else ""
            print(f"profile case {case} tokens={args.tokens} iters={args.iters}: ok{extra}", flush=True)
        return 0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
