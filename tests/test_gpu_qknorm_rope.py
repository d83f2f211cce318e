"""GPU parity: per-head QK-norm + partial split-half RoPE at the H3 attention layout
(56 heads x 128, rot_dim 96), single side and paired, into NHD or HND-backed views.

Against the oracle bit for bit (fp32 tables, and bf16 tables widened to fp32 as the
reference's CUDA kernel does), against the reference's eager outputs (bit for bit with the
fp32 table; within the north-star tolerance with the bf16 table, where the eager and H3 CPU
paths round each product to bf16), and the reference's own SM89 test patterns ported to
B200: the single-side kernel equals the paired kernel, and the HND-backed write equals the
paired result permuted (tests/native_engine/test_single_qknorm_rope.py:80-203).
"""

import numpy as np
import pytest
import torch

import h3b200
import oracle as O
from gpu_util import np_, randn_bf16, t2u, u2t

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = O.bf16_to_f32(a).astype(np.float64)
    b = O.bf16_to_f32(b).astype(np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b), float(np.abs(a - b).max())


def oracle_one(x_u16, table_f32, w_u16, eps, rot):
    return O.rope_split_half(O.rms_norm_row(x_u16, w_u16, eps), table_f32, rot)


def table6(t2d):
    """[T, P, 2, 2] -> the reference's [1, T, 1, P, 2, 2] view"""
    return t2d.reshape(1, t2d.shape[0], 1, *t2d.shape[1:])


def test_single_side_vs_reference_fixture(golden):
    g = golden("qknorm_rope_h3")
    t32 = torch.from_numpy(g["table_f32"]).cuda()
    t16 = u2t(g["table_bf16"])
    for name, wn in (("q", "wq"), ("k", "wk")):
        w = u2t(g[wn])
        v = u2t(g[name])
        h3b200.single_qknorm_rope_(v, weight=w, frequencies=table6(t32), eps=1e-5)
        np.testing.assert_array_equal(t2u(v), g[f"{name}_f32tab"])
        v = u2t(g[name])
        h3b200.single_qknorm_rope_(v, weight=w, frequencies=table6(t16), eps=1e-5)
        np.testing.assert_array_equal(t2u(v), oracle_one(g[name], O.bf16_to_f32(g["table_bf16"]), g[wn], 1e-5, 96))
        for ref in (f"{name}_bf16tab", f"{name}_h3"):
            rel, mx = rel_l2(t2u(v), g[ref])
            assert rel <= 1e-2 and mx <= 2e-2, (ref, rel, mx)
    assert h3b200.device_status(0) == 0


def test_paired_h3_heads_vs_fixture(golden):
    """rms_rope_split_half_ with 56 heads takes the strided kernel (paired form)."""
    g = golden("qknorm_rope_h3")
    q, k = u2t(g["q"]), u2t(g["k"])
    t32 = torch.from_numpy(g["table_f32"]).cuda()
    h3b200.rms_rope_split_half_(q.unsqueeze(0), k.unsqueeze(0), table6(t32), u2t(g["wq"]), u2t(g["wk"]), 1e-5, 96)
    np.testing.assert_array_equal(t2u(q), g["q_f32tab"])
    np.testing.assert_array_equal(t2u(k), g["k_f32tab"])
    qo, ko = h3b200.rms_rope_split_half(u2t(g["q"]).unsqueeze(0), u2t(g["k"]).unsqueeze(0), table6(t32),
                                        u2t(g["wq"]), u2t(g["wk"]), 1e-5, 96)
    np.testing.assert_array_equal(t2u(qo[0]), g["q_f32tab"])
    np.testing.assert_array_equal(t2u(ko[0]), g["k_f32tab"])


def _case(tokens, heads, seed, table_dtype=torch.bfloat16, rot=96):
    gen = torch.Generator().manual_seed(seed)
    src = randn_bf16((tokens, heads, 128), gen).cuda()
    w = randn_bf16((128,), gen).cuda()
    freqs = torch.randn(1, tokens, 1, rot // 2, 2, 2, generator=gen).to(table_dtype).cuda()
    return src, w, freqs


def test_single_partial_kernel_is_bit_exact_to_paired_kernel():
    """Port of test_sm89_single_partial_kernel_is_bit_exact_to_paired_kernel
    (tokens 257, 4 heads, rot 96, bf16 table, eps 1e-5)."""
    src, w, freqs = _case(257, 4, 89)
    reference = src.clone()
    candidate = src.clone()
    scratch = torch.randn(reference.shape, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    h3b200.rms_rope_split_half_(reference.unsqueeze(0), scratch.unsqueeze(0), freqs, w, w, 1e-5, 96)
    h3b200.single_qknorm_rope_(candidate, weight=w, frequencies=freqs, eps=1e-5)
    torch.cuda.synchronize()
    assert torch.equal(candidate, reference)
    np.testing.assert_array_equal(t2u(candidate), oracle_one(t2u(src), freqs.float().cpu().numpy().reshape(257, 48, 2, 2),
                                                            t2u(w), 1e-5, 96))


def test_single_partial_kernel_writes_exact_hnd_backing():
    """Port of test_sm89_single_partial_kernel_writes_exact_hnd_backing: the destination is
    an HND allocation with 13 spare tokens per head."""
    src, w, freqs = _case(257, 4, 8913)
    reference = src.clone()
    scratch = torch.zeros_like(reference)
    h3b200.rms_rope_split_half_(reference.unsqueeze(0), scratch.unsqueeze(0), freqs, w, w, 1e-5, 96)
    candidate_hnd = torch.full((4, 257 + 13, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    view = candidate_hnd[:, :257].permute(1, 0, 2)
    h3b200.single_qknorm_rope_to_hnd(src.clone(), view, weight=w, frequencies=freqs, eps=1e-5)
    torch.cuda.synchronize()
    assert torch.equal(candidate_hnd[:, :257], reference.permute(1, 0, 2))
    assert bool((candidate_hnd[:, 257:] == 7.0).all())          # the spare tokens are untouched
    with pytest.raises(ValueError):
        h3b200.single_qknorm_rope_to_hnd(src, torch.empty_like(src), weight=w, frequencies=freqs, eps=1e-5)


@pytest.mark.parametrize("rot", [96, 128, 64, 16])
@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_strided_qkv_slice_into_hnd_vs_oracle(rot, table_dtype):
    """K and Q slices of a packed [T, 3 x 56 x 128] QKV row, H3 heads, into HND buffers."""
    gen = torch.Generator().manual_seed(rot + 7)
    t, h = 700, 56
    qkv = randn_bf16((t, 3 * h * 128), gen).cuda()
    wq = (1 + 0.05 * torch.randn(128, generator=gen)).to(torch.bfloat16).cuda()
    wk = (1 + 0.05 * torch.randn(128, generator=gen)).to(torch.bfloat16).cuda()
    freqs = (torch.randn(1, t, 1, rot // 2, 2, 2, generator=gen) * 0.7).to(table_dtype).cuda()
    q = qkv[:, :h * 128].view(t, h, 128)
    k = qkv[:, h * 128:2 * h * 128].view(t, h, 128)
    q_hnd = torch.empty(h, t, 128, dtype=torch.bfloat16, device="cuda")
    k_hnd = torch.empty(h, t, 128, dtype=torch.bfloat16, device="cuda")
    h3b200.qknorm_rope_strided_(q, wq, freqs, 1e-5, rot, q_out=q_hnd.permute(1, 0, 2), k=k, k_weight=wk,
                                k_out=k_hnd.permute(1, 0, 2))
    assert h3b200.device_status(0) == 0
    tab = freqs.float().cpu().numpy().reshape(t, rot // 2, 2, 2)
    qk_host = t2u(qkv)
    for x_host, w, out in ((qk_host[:, :h * 128], wq, q_hnd), (qk_host[:, h * 128:2 * h * 128], wk, k_hnd)):
        ref = oracle_one(x_host.reshape(t, h, 128), tab, t2u(w), 1e-5, rot)
        np.testing.assert_array_equal(t2u(out.permute(1, 0, 2)), ref)
    # the input rows are unchanged
    np.testing.assert_array_equal(t2u(qkv), qk_host)


def test_per_head_table_and_edge_values():
    """A table with a row per (token, head), odd head count, zero / huge / inf rows."""
    gen = torch.Generator().manual_seed(5)
    t, h = 37, 7
    x = randn_bf16((t, h, 128), gen)
    x[3, 2] = 0
    x[4, 1, 5] = float("inf")
    x[5, 6] *= 1e30
    x[6, 0, :] = -2.0
    x = x.cuda()
    w = randn_bf16((128,), gen).cuda()
    freqs = torch.randn(1, t, h, 48, 2, 2, generator=gen).cuda()
    y = torch.empty_like(x)
    h3b200.qknorm_rope_strided_(x, w, freqs, 1e-5, 96, q_out=y)
    tab = freqs.cpu().numpy()[0]           # [t, h, 48, 2, 2]
    xs, ws = t2u(x), t2u(w)
    for hi in range(h):
        ref = oracle_one(xs[:, hi:hi + 1], tab[:, hi], ws, 1e-5, 96)
        got = t2u(y[:, hi:hi + 1])
        fin = np.isfinite(O.bf16_to_f32(ref))
        np.testing.assert_array_equal(got[fin], ref[fin])
        np.testing.assert_array_equal(np.isnan(O.bf16_to_f32(got)), np.isnan(O.bf16_to_f32(ref)))


def test_h3_long_sequence_k_build_vs_oracle_rows():
    """32,760 tokens of H3 K (56 heads) into an HND buffer; per-token math, so a row sample
    checked against the oracle is a size-independent check of the whole launch."""
    gen = torch.Generator(device="cuda").manual_seed(11)
    t, h = 32760, 56
    k = torch.randn(t, h, 128, generator=gen, device="cuda").to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(128, generator=gen, device="cuda")).to(torch.bfloat16)
    freqs = torch.randn(1, t, 1, 48, 2, 2, generator=gen, device="cuda").to(torch.bfloat16)
    k_hnd = torch.empty(h, t, 128, dtype=torch.bfloat16, device="cuda")
    h3b200.single_qknorm_rope_to_hnd(k, k_hnd.permute(1, 0, 2), weight=w, frequencies=freqs, eps=1e-5)
    assert h3b200.device_status(0) == 0
    rows = np.arange(0, t, 97)
    ref = oracle_one(t2u(k)[rows], freqs.float().cpu().numpy().reshape(t, 48, 2, 2)[rows], t2u(w), 1e-5, 96)
    np.testing.assert_array_equal(t2u(k_hnd.permute(1, 0, 2))[rows], ref)


def test_contract_errors():
    x = torch.zeros(4, 3, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):       # table shorter than the rotation
        h3b200.qknorm_rope_strided_(x, w, torch.zeros(1, 4, 1, 8, 2, 2, device="cuda"), 1e-5, 96)
    with pytest.raises(ValueError):       # table covers other tokens
        h3b200.qknorm_rope_strided_(x, w, torch.zeros(1, 5, 1, 48, 2, 2, device="cuda"), 1e-5, 96)
    with pytest.raises(NotImplementedError):  # rot_dim not a multiple of 16 (valid for the reference, not built)
        h3b200.qknorm_rope_strided_(x, w, torch.zeros(1, 4, 1, 50, 2, 2, device="cuda"), 1e-5, 100)


def _qkv_case(m, heads, k, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    inner = heads * 128
    hidden = torch.randn(m, k, generator=gen, device="cuda").to(torch.bfloat16)
    w = (torch.randn(3 * inner, k, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    wq_, ws = h3b200.quantize_int8_convrot_weight(w)
    bias = (torch.randn(3 * inner, generator=gen, device="cuda") * 0.1).to(torch.bfloat16)
    qn = (1 + 0.05 * torch.randn(128, generator=gen, device="cuda")).to(torch.bfloat16)
    kn = (1 + 0.05 * torch.randn(128, generator=gen, device="cuda")).to(torch.bfloat16)
    freqs = torch.randn(1, m, 1, 48, 2, 2, generator=gen, device="cuda").to(torch.bfloat16)
    xq, xs = h3b200.quantize_int8_rowwise_convrot(hidden, 256)
    return xq, xs, wq_, ws, bias, qn, kn, freqs


def test_qkv_projection_qknorm_rope_hnd_matches_op_chain():
    """H3 layout (56 heads, hidden 5,376, rot 96, bf16 table): the QKV entry equals
    int8_linear_prequantized + the single-side kernel + the V copy, for every section split;
    a row sample equals the oracle."""
    m, heads, k = 600, 56, 5376
    inner = heads * 128
    xq, xs, wq_, ws, bias, qn, kn, freqs = _qkv_case(m, heads, k, 23)
    q, kk, v = h3b200.qkv_qknorm_rope(xq, xs, wq_, ws, bias, heads, qn, kn, freqs, 1e-5, "qkv")
    assert h3b200.device_status(0) == 0
    proj = h3b200.int8_linear_prequantized(xq, xs, wq_, ws, bias)
    pq = proj[:, :inner].view(m, heads, 128).clone()
    pk = proj[:, inner:2 * inner].view(m, heads, 128).clone()
    h3b200.single_qknorm_rope_(pq, weight=qn, frequencies=freqs, eps=1e-5)
    h3b200.single_qknorm_rope_(pk, weight=kn, frequencies=freqs, eps=1e-5)
    np.testing.assert_array_equal(t2u(q), t2u(pq))
    np.testing.assert_array_equal(t2u(kk), t2u(pk))
    np.testing.assert_array_equal(t2u(v), t2u(proj[:, 2 * inner:].view(m, heads, 128)))
    assert q.stride() == (128, m * 128, 1)                      # HND-backed views
    # the K/V build and a query chunk give the same tensors
    _, k2, v2 = h3b200.qkv_qknorm_rope(xq, xs, wq_, ws, bias, heads, None, kn, freqs, 1e-5, "kv")
    q2, _, _ = h3b200.qkv_qknorm_rope(xq[:300], xs[:300], wq_, ws, bias, heads, qn, None, freqs[:, :300], 1e-5, "q")
    np.testing.assert_array_equal(t2u(k2), t2u(kk))
    np.testing.assert_array_equal(t2u(v2), t2u(v))
    np.testing.assert_array_equal(t2u(q2), t2u(q[:300]))
    # oracle on a row sample: int8 GEMM + dequant + bias, then per-head norm + RoPE
    rows = np.arange(0, m, 53)
    acc = O.int8_matmul_accumulate(np_(xq)[rows], np_(wq_))
    y = O.dequant_epilogue(acc, np_(xs).reshape(-1)[rows], np_(ws).reshape(-1), t2u(bias))
    tab = freqs.float().cpu().numpy().reshape(m, 48, 2, 2)[rows]
    for sec, nw, got in ((0, qn, q), (1, kn, kk)):
        ref = oracle_one(y[:, sec * inner:(sec + 1) * inner].reshape(-1, heads, 128), tab, t2u(nw), 1e-5, 96)
        np.testing.assert_array_equal(t2u(got)[rows], ref)
    np.testing.assert_array_equal(t2u(v)[rows], y[:, 2 * inner:].reshape(-1, heads, 128))


def test_qkv_norm_only_and_caller_views():
    """No frequencies: RMSNorm only (the reference's q_norm / k_norm); outputs into caller
    views with spare tokens (an HND allocation larger than the chunk)."""
    m, heads, k = 200, 8, 1024
    xq, xs, wq_, ws, bias, qn, kn, _ = _qkv_case(m, heads, k, 31)
    k_hnd = torch.full((heads, m + 40, 128), 3.0, dtype=torch.bfloat16, device="cuda")
    v_hnd = torch.full((heads, m + 40, 128), 3.0, dtype=torch.bfloat16, device="cuda")
    _, kk, v = h3b200.qkv_qknorm_rope(xq, xs, wq_, ws, None, heads, None, kn, None, 1e-5, "kv",
                                      k_out=k_hnd[:, 20:20 + m].permute(1, 0, 2),
                                      v_out=v_hnd[:, 20:20 + m].permute(1, 0, 2))
    proj = h3b200.int8_linear_prequantized(xq, xs, wq_, ws)
    inner = heads * 128
    ref_k = O.rms_norm_row(t2u(proj[:, inner:2 * inner]).reshape(m, heads, 128), t2u(kn), 1e-5)
    np.testing.assert_array_equal(t2u(k_hnd[:, 20:20 + m].permute(1, 0, 2)), ref_k)
    np.testing.assert_array_equal(t2u(v_hnd[:, 20:20 + m].permute(1, 0, 2)),
                                  t2u(proj[:, 2 * inner:]).reshape(m, heads, 128))
    assert bool((k_hnd[:, :20] == 3.0).all()) and bool((v_hnd[:, 20 + m:] == 3.0).all())


@pytest.mark.parametrize("rot,per_head_table,nhd_out", [(96, False, True), (128, False, False), (64, False, True),
                                                         (16, False, False), (96, True, False)])
def test_qkv_fused_and_three_kernel_paths_match_op_chain(rot, per_head_table, nhd_out):
    """The fused GEMM epilogue (per-token table, rot a multiple of 32) and the three-kernel path
    (rot 16, or a table row per head) give the op chain's bits, into HND or NHD outputs."""
    m, heads, k = 333, 6, 768
    inner = heads * 128
    xq, xs, wq_, ws, bias, qn, kn, _ = _qkv_case(m, heads, k, rot + per_head_table)
    gen = torch.Generator(device="cuda").manual_seed(rot)
    freqs = torch.randn(1, m, heads if per_head_table else 1, rot // 2, 2, 2, generator=gen, device="cuda")
    if nhd_out:
        bufs = [torch.empty(m, heads, 128, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    else:
        bufs = [torch.empty(heads, m, 128, dtype=torch.bfloat16, device="cuda").permute(1, 0, 2) for _ in range(3)]
    q, kk, v = h3b200.qkv_qknorm_rope(xq, xs, wq_, ws, bias, heads, qn, kn, freqs, 1e-5, "qkv", *bufs)
    assert h3b200.device_status(0) == 0
    proj = h3b200.int8_linear_prequantized(xq, xs, wq_, ws, bias)
    pq = proj[:, :inner].reshape(m, heads, 128)
    pk = proj[:, inner:2 * inner].reshape(m, heads, 128)
    rq, rk = h3b200.qknorm_rope_strided_(pq, qn, freqs, 1e-5, rot, q_out=torch.empty_like(pq), k=pk, k_weight=kn,
                                         k_out=torch.empty_like(pk))
    np.testing.assert_array_equal(t2u(q), t2u(rq))
    np.testing.assert_array_equal(t2u(kk), t2u(rk))
    np.testing.assert_array_equal(t2u(v), t2u(proj[:, 2 * inner:].reshape(m, heads, 128)))
