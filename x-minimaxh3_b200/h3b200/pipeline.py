"""Fused gated MLP over host (pinned) token buffers, with copies overlapped.

A serving process usually holds a step's activations in host memory. Called on
host tensors, ``fused_gated_mlp_host`` splits the tokens into chunks and runs
three CUDA streams: host-to-device copies of chunk i+1, the fused MLP of chunk
i (``fused_gated_mlp``: quantize -> fc1 + GELU -> requant -> fc2 + gated
residual) and the device-to-host copy of chunk i-1 run at the same time. The
MLP is per-token, so the chunked result is bit-identical to one call over all
tokens. Device staging buffers (token slots, streams, events and the MLP
workspace) are allocated once per (device, d, ffn, chunk, slots) and reused;
calls that share them from several host threads are serialised by a lock held
while their work is queued (the streams and events then order it on the GPU).

The copies in dominate (x and residual: 4 bytes per element against 2 out), so
the call lasts about as long as the host-to-device stream plus whatever follows
its last copy: the last chunk's MLP and its copy out, which nothing overlaps.
The tokens after the last full chunk are therefore cut into halving pieces
(4,088 -> 2,048 + 1,024 + 512 + 504), which shrinks that tail to the smallest
piece's.
"""

from __future__ import annotations

import threading

import torch

from .ops import fused_gated_mlp

_cache_lock = threading.Lock()
_cache: dict = {}


class _Staging:
    def __init__(self, device: torch.device, d: int, ffn: int, chunk: int, slots: int):
        from . import _lib
        self.lock = threading.Lock()
        self.x = [torch.empty(chunk, d, dtype=torch.bfloat16, device=device) for _ in range(slots)]
        self.r = [torch.empty(chunk, d, dtype=torch.bfloat16, device=device) for _ in range(slots)]
        self.h2d = torch.cuda.Stream(device)
        self.comp = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.free = [torch.cuda.Event() for _ in range(slots)]
        self.used = [False] * slots
        nbytes = int(_lib.load().h3b200_fused_gated_mlp_workspace_bytes(chunk, d, ffn))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=device)


def _staging(device: torch.device, d: int, ffn: int, chunk: int, slots: int) -> _Staging:
    key = (device.index, d, ffn, chunk, slots)
    with _cache_lock:
        st = _cache.get(key)
        if st is None:
            st = _Staging(device, d, ffn, chunk, slots)
            _cache[key] = st
    return st


def _chunk_sizes(m: int, chunk: int, min_piece: int = 256) -> list[int]:
    """Full chunks, then the remainder (at most one chunk) in halving pieces of at
    least ``min_piece`` tokens (multiples of 16)."""
    sizes = []
    rest = m
    while rest > chunk:
        sizes.append(chunk)
        rest -= chunk
    while rest > 2 * min_piece:
        piece = -(-(rest // 2) // 16) * 16
        sizes.append(piece)
        rest -= piece
    if rest > 0:
        sizes.append(rest)
    return sizes


def fused_gated_mlp_host(residual: torch.Tensor, hidden: torch.Tensor, w1q: torch.Tensor, s1: torch.Tensor,
                         w2q: torch.Tensor, s2: torch.Tensor, gate: torch.Tensor, out: torch.Tensor | None = None,
                         chunk_tokens: int = 4096, slots: int = 3, synchronize: bool = True) -> torch.Tensor:
    """``out = residual + int8_linear(gelu(int8_linear(hidden, w1q, s1)), w2q, s2) * gate`` for host tensors.

    ``residual``, ``hidden`` and ``out`` are CPU bf16 [M, d] tensors (pinned memory
    for overlap; ``out`` may be ``residual``); weights, scales and ``gate`` live on
    the CUDA device that runs the MLP. Same result as ``fused_gated_mlp`` on device
    copies of the inputs. With ``synchronize=False`` the call returns once the work
    is queued; ``out`` is then valid after the caller's current stream is
    synchronised."""
    if residual.is_cuda or hidden.is_cuda:
        raise ValueError("fused_gated_mlp_host takes host tensors; use fused_gated_mlp for device tensors")
    if residual.shape != hidden.shape or residual.dim() != 2:
        raise ValueError("residual and hidden must both be [M, d]")
    if residual.dtype != torch.bfloat16 or hidden.dtype != torch.bfloat16:
        raise ValueError("residual and hidden must be bf16")
    if chunk_tokens <= 0 or slots < 2:
        raise ValueError("chunk_tokens must be positive and slots >= 2")
    m, d = hidden.shape
    if out is None:
        out = torch.empty((m, d), dtype=torch.bfloat16, pin_memory=residual.is_pinned())
    elif out.shape != residual.shape or out.dtype != torch.bfloat16 or out.is_cuda:
        raise ValueError("out must be a host bf16 tensor shaped like residual")
    dev = w1q.device
    chunk = min(chunk_tokens, m) if m > 0 else 1
    st = _staging(dev, d, w1q.shape[0], chunk, slots)
    with st.lock:
        _queue(st, residual, hidden, w1q, s1, w2q, s2, gate, out, m, chunk, slots)
    if synchronize:
        torch.cuda.current_stream(dev).synchronize()
        from . import _lib
        _lib.check_device(dev.index, "fused_gated_mlp_host")
    return out


def _queue(st: _Staging, residual, hidden, w1q, s1, w2q, s2, gate, out, m: int, chunk: int, slots: int) -> None:
    """Queue the chunked copies and MLPs of one call on the staging streams."""
    cur = torch.cuda.current_stream(w1q.device)
    for s in (st.h2d, st.comp, st.d2h):
        s.wait_stream(cur)
    lo = 0
    for i, n in enumerate(_chunk_sizes(m, chunk)):
        hi = lo + n
        k = i % slots
        xb, rb = st.x[k][:n], st.r[k][:n]
        with torch.cuda.stream(st.h2d):
            if st.used[k]:
                st.h2d.wait_event(st.free[k])  # the slot's previous chunk has been copied out
            xb.copy_(hidden[lo:hi], non_blocking=True)
            rb.copy_(residual[lo:hi], non_blocking=True)
        st.comp.wait_stream(st.h2d)
        with torch.cuda.stream(st.comp):
            fused_gated_mlp(rb, xb, w1q, s1, w2q, s2, gate, out=rb, workspace=st.workspace)
        st.d2h.wait_stream(st.comp)
        with torch.cuda.stream(st.d2h):
            out[lo:hi].copy_(rb, non_blocking=True)
            st.free[k].record(st.d2h)
        st.used[k] = True
        lo = hi
    cur.wait_stream(st.d2h)
