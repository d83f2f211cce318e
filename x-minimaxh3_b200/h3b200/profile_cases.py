"""Run one kernel of the hot path on a chosen token count, for profilers.

    python -m h3b200.profile_cases CASE [--tokens M] [--iters N]

CASE is one of ``quantize`` (fc1 input quantizer, K = 3072), ``fc1`` (INT8 GEMM
with the GELU + row-absmax epilogue; ``fc1_bf16`` / ``fc1_i32``: the same GEMM with
the plain dequant or the int32 epilogue), ``requant`` (fc2 input quantizer with a
given absmax, K = 12288), ``fc2`` (INT8 GEMM with the gated-residual epilogue),
``mlp`` (the whole fused MLP call), ``mlp_w4a8`` (the config-2 W4A8 MLP call), ``mlp_swiglu``
(the H3 SwiGLU MLP at d 5,376 / ffn 14,336, ConvRot fc1 and fc2, 8,192-token chunks),
``mlp_swiglu_w4`` (the same MLP on W4A8 weights in the H3 release format: group 16,
fp8-e4m3 scales, codebook; both weights decoded per call), ``decode_w4`` (that
format's int4 -> int8 decode of the fc1 weight, 28,672 x 5,376), ``qknorm_h3``
(single-side QK-norm + partial RoPE of H3 K, 56 heads, rot 96, bf16 table, into an
HND buffer), ``qkv_h3`` (the H3 Q/K/V projection of M tokens, hidden 5,376, with
QK-norm + RoPE into HND buffers, from a ConvRot-quantized activation),
``convrot`` / ``convrot_x`` (ConvRot-256 + row quantization of a K = 12288 / 3072 bf16 input) or ``norm_rope`` (AdaLN + RMSNorm + RoPE on
Q and K, 24 heads x 128). Shapes are those of the config-1 MLP and config-3
norm-RoPE with M tokens; inputs are seeded synthetic data. Every case first
runs the kernels it needs to build its inputs, then launches the kernel under
study ``--iters`` times, so a profiler can skip the set-up launches by kernel
name; ``--time`` also reports the mean CUDA-event time of those launches. The
process exits non-zero if a kernel reports an error.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import h3b200  # noqa: E402
from h3b200 import ops  # noqa: E402
from h3b200.rope import rope_grid_table  # noqa: E402

D_MODEL, D_FFN = 3072, 12288


def mlp_inputs(m: int, dev):
    g = torch.Generator(device=dev).manual_seed(2)
    w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(D_MODEL, D_FFN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wt = h3b200.W8A8MLPWeights.from_float(w1, w2)
    x = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
    return wt, x, gate, res


def _timed(fn, iters: int, report: bool):
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


def run(case: str, m: int, iters: int, report: bool = False):
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
        ms = _timed(lambda: ops.adaln_rms_rope_(q, k, table, wq, wk, sc, sh, 1e-6, "row", 0, q_out=qo, k_out=ko),
                    iters, report)
    elif case in ("convrot", "convrot_x"):
        g = torch.Generator(device=dev).manual_seed(6)
        a = torch.randn(m, D_FFN if case == "convrot" else D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        ms = _timed(lambda: ops.quantize_int8_rowwise_convrot(a, 256), iters, report)
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
        ms = _timed(lambda: h3b200.fused_gated_mlp_swiglu(res, x, wt, gate, out=out), iters, report)
    elif case in ("mlp_swiglu_w4", "decode_w4"):
        g = torch.Generator(device=dev).manual_seed(9)
        d, ffn = 5376, 14336
        w1 = (torch.randn(2 * ffn, d, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(d, ffn, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w4 = h3b200.W4A8SwiGLUMLPWeights.from_float(w1, w2)
        del w1, w2
        if case == "decode_w4":
            ms = _timed(lambda: ops.dequant_int4_grouped_to_int8(w4.q1, w4.s_rel1, 16, w4.codebook1), iters, report)
        else:
            x = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
            gate = torch.randn(d, generator=g, device=dev).to(torch.bfloat16)
            res = torch.randn(m, d, generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty_like(res)
            ms = _timed(lambda: h3b200.fused_gated_mlp_swiglu_w4a8(res, x, w4, gate, out=out), iters, report)
    elif case in ("qknorm_h3", "qkv_h3"):
        g = torch.Generator(device=dev).manual_seed(10)
        heads, d = 56, 5376
        freqs = torch.randn(1, m, 1, 48, 2, 2, generator=g, device=dev).to(torch.bfloat16)
        kn = (1 + 0.02 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
        if case == "qknorm_h3":
            k = torch.randn(m, heads, 128, generator=g, device=dev).to(torch.bfloat16)
            k_hnd = torch.empty(heads, m, 128, dtype=torch.bfloat16, device=dev).permute(1, 0, 2)
            ms = _timed(lambda: ops.single_qknorm_rope_to_hnd(k, k_hnd, weight=kn, frequencies=freqs, eps=1e-5),
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
            ms = _timed(lambda: ops.qkv_qknorm_rope(xq, xs, wq_, ws, None, heads, kn, kn, freqs, 1e-5, "qkv",
                                                    *outs, workspace=work), iters, report)
    elif case == "mlp_w4a8":
        g = torch.Generator(device=dev).manual_seed(3)
        w1 = (torch.randn(D_FFN, D_MODEL, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn(D_MODEL, D_FFN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w4 = h3b200.W4A8MLPWeights.from_float(w1, w2, 128)
        x = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn(D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        res = torch.randn(m, D_MODEL, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty_like(res)
        ms = _timed(lambda: h3b200.fused_gated_mlp_w4a8(res, x, w4, gate, out=out), iters, report)
    else:
        wt, x, gate, res = mlp_inputs(m, dev)
        xq, xs = ops.quantize_int8_rowwise(x)
        amax = torch.zeros(m, dtype=torch.float32, device=dev)
        act = torch.empty(m, D_FFN, dtype=torch.bfloat16, device=dev)
        out = torch.empty_like(res)

        def fc1():
            ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_GELU_ABSMAX, xs, wt.s1, out=act, row_absmax=amax)

        if case == "quantize":
            ms = _timed(lambda: ops.quantize_int8_rowwise(x), iters, report)
        elif case == "fc1":
            ms = _timed(fc1, iters, report)   # row absmax only grows: re-running on the same inputs is idempotent
        elif case == "fc1_bf16":
            ms = _timed(lambda: ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_BF16, xs, wt.s1, out=act), iters, report)
        elif case == "fc1_i32":
            acc = torch.empty(m, D_FFN, dtype=torch.int32, device=dev)
            ms = _timed(lambda: ops.int8_gemm_fused(xq, wt.w1q, ops.EPI_I32, out=acc), iters, report)
        elif case in ("requant", "fc2"):
            fc1()
            if case == "requant":
                ms = _timed(lambda: ops.quantize_int8_rowwise_absmax(act, amax), iters, report)
            else:
                q2, xs2 = ops.quantize_int8_rowwise_absmax(act, amax)
                ms = _timed(lambda: ops.int8_gemm_fused(q2, wt.w2q, ops.EPI_GATED_RESIDUAL, xs2, wt.s2, gate=gate,
                                                        residual=res, out=out), iters, report)
        elif case == "mlp":
            ms = _timed(lambda: h3b200.fused_gated_mlp(res, x, wt.w1q, wt.s1, wt.w2q, wt.s2, gate, out=out), iters,
                        report)
        else:
            raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    st = h3b200.device_status(0)
    if st != 0:
        raise SystemExit(f"device status {st:#x}")
    return ms


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", nargs="+", choices=["quantize", "fc1", "fc1_bf16", "fc1_i32", "requant", "fc2", "mlp",
                                                "mlp_w4a8", "mlp_swiglu", "mlp_swiglu_w4", "decode_w4", "qknorm_h3",
                                                "qkv_h3", "convrot",
                                                "convrot_x", "norm_rope"])
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="report the mean CUDA-event time per launch")
    a = ap.parse_args()
    for case in a.case:
        ms = run(case, a.tokens, a.iters, a.time)
        extra = f" mean {ms:.4f} ms per launch" if ms is not None else ""
        print(f"profile case {case} tokens={a.tokens} iters={a.iters}: ok{extra}", flush=True)


if __name__ == "__main__":
    main()
