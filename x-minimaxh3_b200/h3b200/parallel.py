"""Multi-GPU execution of the hot path (one process per GPU, torch.distributed / NCCL).

The reference is single-GPU (no collective anywhere); scaling it out is new.
Two modes:

* Token sharding (data parallel over tokens). The quantizer, the MLP and the
  norm-RoPE are per-token functions, so each rank takes a contiguous token
  range (and the matching rows of the RoPE table) and runs the single-GPU
  kernels on it. There is no collective on the data path; results equal the
  single-GPU results bit for bit.
* Tensor-parallel MLP (long-video config), ``collective="p2p"`` (default on GPUs):
  the exchange runs inside this package's kernels over NVLink peer memory
  (:class:`TPComm`, ``h3b200_tp_*``): fc1's row absmax is pushed into every rank's
  slot and max-reduced after a cross-GPU flag barrier, fc2 quantizes its own input
  with that global absmax and its epilogue stores each int32 partial row directly
  into the receive slot of the rank that owns the row (the reduce-scatter fused into
  the GEMM), and each owner sums the partials, applies dequant + gated residual and
  stores its finished rows into every rank's gather buffer (the all-gather fused into
  that pass). No NCCL call on the data path.
* Tensor-parallel MLP over NCCL (``collective="reduce_scatter"`` / ``"all_reduce"``,
  also the path the CPU tests drive with gloo). fc1 is column-split (rank r owns
  ffn rows [r*ffn/g, (r+1)*ffn/g) of W1), GELU is local, and the per-token
  requant scale needs the row absmax over all ffn columns: one all-reduce(MAX)
  of an fp32 [M] vector, after which every rank quantizes with the global scale
  (so the int8 activations are the single-GPU ones). fc2 is row-split along
  its K = ffn: each rank produces partial int32 accumulators, summed exactly by
  a reduce-scatter(SUM) over int32 by rows, each rank runs the dequant +
  gated-residual epilogue on its rows, and an all-gather returns the bf16 rows
  (or, optionally, an int32 all-reduce and the whole epilogue on every rank).
  The output is bit-identical to the single-GPU fused MLP. Tokens are processed
  in chunks; the reduction of chunk i runs asynchronously while chunk i+1
  computes.

The kernel calls go through an ``ops`` object (default: the CUDA kernels of
this package) so the orchestration can be exercised on CPU ranks in tests.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_range(m: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal token range of ``rank`` (the first ``m % world`` ranks get one more)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(m, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def column_shard(ffn: int, world: int, rank: int) -> tuple[int, int]:
    """fc1 output-column (= fc2 input-column) range owned by ``rank`` in the tensor-parallel MLP."""
    if ffn % world:
        raise ValueError(f"ffn={ffn} is not divisible by the tensor-parallel size {world}")
    step = ffn // world
    return rank * step, (rank + 1) * step


class CudaOps:
    """Stage kernels of the fused MLP (libh3b200.so)."""

    def quantize(self, x):
        from .ops import quantize_int8_rowwise

        return quantize_int8_rowwise(x)

    def fc1_gelu_absmax(self, xq, xs, w1q, s1, absmax):
        from .ops import EPI_GELU_ABSMAX, int8_gemm_fused

        return int8_gemm_fused(xq, w1q, EPI_GELU_ABSMAX, xs, s1, row_absmax=absmax)

    def quantize_absmax(self, a, absmax):
        from .ops import quantize_int8_rowwise_absmax

        return quantize_int8_rowwise_absmax(a, absmax)

    def gemm_i32(self, q, w):
        from .ops import EPI_I32, int8_gemm_fused

        return int8_gemm_fused(q, w, EPI_I32)

    def dequant_gated_residual(self, acc, xs, ws, gate, residual, out):
        from .ops import dequant_gated_residual

        return dequant_gated_residual(acc, xs, ws, gate, residual, out)

    def fused_mlp(self, residual, x, w1q, s1, w2q, s2, gate, out):
        from .ops import fused_gated_mlp

        return fused_gated_mlp(residual, x, w1q, s1, w2q, s2, gate, out=out)

    def norm_rope(self, q, k, table, wq, wk, scale, shift, eps, span):
        from .ops import adaln_rms_rope

        return adaln_rms_rope(q, k, table, wq, wk, scale, shift, eps, span)


@dataclass
class TPShard:
    """This rank's slice of one gated MLP's weights for tensor parallelism."""

    w1q: torch.Tensor  # [ffn/g, d]
    s1: torch.Tensor   # [ffn/g]
    w2q: torch.Tensor  # [d, ffn/g] (contiguous)
    s2: torch.Tensor   # [d] (replicated)

    @classmethod
    def from_full(cls, w1q, s1, w2q, s2, world: int, rank: int) -> "TPShard":
        lo, hi = column_shard(w1q.shape[0], world, rank)
        return cls(w1q[lo:hi].contiguous(), s1[lo:hi].contiguous(), w2q[:, lo:hi].contiguous(), s2.contiguous())


def _world(group=None) -> tuple[int, int]:
    """(world size, rank) of ``group``; (1, 0) when no process group is initialised."""
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


COLLECTIVES = ("p2p", "reduce_scatter", "all_reduce")
# the forms whose exchange goes through torch.distributed (any backend, any ``ops``)
PG_COLLECTIVES = ("reduce_scatter", "all_reduce")


class TPComm:
    """Peer-memory communicator of the tensor-parallel MLP (``h3b200_tp_comm_*``).

    Every rank of ``group`` builds one with the same ``max_rows`` (the token chunk),
    ``d`` and ``ffn_shard`` (its fc1 width). The constructor exchanges the CUDA IPC
    handles of the ranks' exchange regions over the process group (one all-gather)
    and maps the other ranks' regions; from then on the data path uses no collective:
    the kernels store into the peers' memory over NVLink and meet at flag barriers
    in it (bounded waits: status 0x201 on expiry).

    Call :meth:`close` on every rank once the last MLP has been issued everywhere
    (it synchronises the device and the group before the regions are freed)."""

    def __init__(self, max_rows: int, d: int, ffn_shard: int, group=None, barrier_timeout_s: float = 5.0,
                 *, _local: tuple[int, int] | None = None):
        from . import _lib

        world, rank = _world(group) if _local is None else _local
        self.world, self.rank, self.group = world, rank, group
        self.max_rows, self.d, self.ffn = int(max_rows), int(d), int(ffn_shard)
        self.device = torch.cuda.current_device()
        self.linked = _local is not None
        lib = _lib.load()
        handle = (ctypes.c_uint8 * _lib.TP_HANDLE_BYTES)()
        ptr = ctypes.c_void_p()
        _lib.check(lib.h3b200_tp_comm_create(rank, world, self.max_rows, self.d, self.ffn,
                                             int(barrier_timeout_s * 1e9), ctypes.byref(ptr), handle),
                   "h3b200_tp_comm_create")
        self._ptr = ptr
        if _local is None and world > 1:
            dev = self._group_device()
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=dev)
            every = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(every, mine, group=group)
            blob = b"".join(bytes(t.cpu().tolist()) for t in every)
            _lib.check(lib.h3b200_tp_comm_open(ptr, (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)),
                       "h3b200_tp_comm_open")
            mapped = torch.ones(1, device=dev)
            dist.all_reduce(mapped, group=group)  # every rank has mapped every region

    def _group_device(self):
        return torch.device("cuda", self.device) if dist.get_backend(self.group) == "nccl" else torch.device("cpu")

    @classmethod
    def linked_local(cls, world: int, max_rows: int, d: int, ffn_shard: int) -> list["TPComm"]:
        """``world`` communicators in this process on the current device, each other's
        peers without IPC (barriers are no-ops): for running every rank's stages in
        order on one GPU (:meth:`stage`)."""
        from . import _lib

        comms = [cls(max_rows, d, ffn_shard, _local=(world, r)) for r in range(world)]
        ptrs = (ctypes.c_void_p * world)(*[c._ptr.value for c in comms])
        _lib.call("h3b200_tp_comm_link_local", ptrs, world)
        return comms

    def _args(self, x, residual, gate, shard, out):
        if not (x.is_cuda and residual.is_cuda and out.is_cuda):
            raise ValueError("TPComm: x, residual and out must be CUDA tensors")
        for name, t in (("x", x), ("residual", residual), ("out", out), ("gate", gate)):
            if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
                raise ValueError(f"TPComm: {name} must be bf16 with unit column stride")
        if x.shape[1] != self.d or residual.shape != x.shape or out.shape != x.shape or gate.numel() != self.d:
            raise ValueError(f"TPComm: x, residual, out must be [m, {self.d}] and gate [{self.d}]")
        if tuple(shard.w1q.shape) != (self.ffn, self.d) or tuple(shard.w2q.shape) != (self.d, self.ffn) or \
                not shard.w1q.is_contiguous() or not shard.w2q.is_contiguous():
            raise ValueError(f"TPComm: shard weights must be w1q [{self.ffn}, {self.d}], w2q [{self.d}, {self.ffn}], "
                             "contiguous")
        return (x.data_ptr(), x.stride(0), residual.data_ptr(), residual.stride(0), gate.data_ptr(),
                shard.w1q.data_ptr(), shard.s1.data_ptr(), shard.w2q.data_ptr(), shard.s2.data_ptr(),
                out.data_ptr(), out.stride(0))

    def run(self, x, residual, gate, shard: "TPShard", out, chunk_rows: int | None = None):
        """The whole tensor-parallel MLP over ``x`` [m, d] (every rank, same arguments)."""
        from . import _lib

        _lib.call("h3b200_tp_gated_mlp", self._ptr, *self._args(x, residual, gate, shard, out), x.shape[0],
                  int(chunk_rows or self.max_rows), torch.cuda.current_stream().cuda_stream)
        return out

    def stage(self, stage: int, chunk: int, x, residual, gate, shard: "TPShard", out, lo: int, hi: int):
        """One step of chunk ``chunk`` (rows [lo, hi)): 1 quantize + fc1 + absmax push,
        2 absmax max + fc2 with routed rows, 3 owner rows, 4 other owners' rows into out."""
        from . import _lib

        _lib.call("h3b200_tp_stage", self._ptr, stage, chunk, *self._args(x, residual, gate, shard, out), lo, hi,
                  torch.cuda.current_stream().cuda_stream)

    def barrier(self):
        from . import _lib

        _lib.call("h3b200_tp_barrier", self._ptr, torch.cuda.current_stream().cuda_stream)

    def close(self):
        """Free the exchange regions (every rank; after its last MLP call)."""
        from . import _lib

        if self._ptr is None or not self._ptr.value:
            return
        torch.cuda.synchronize(self.device)
        if not self.linked and self.world > 1:
            done = torch.ones(1, device=self._group_device())
            dist.all_reduce(done, group=self.group)  # no rank still writes into another's region
        _lib.call("h3b200_tp_comm_destroy", self._ptr)
        self._ptr = None

    def __del__(self):
        # a group member cannot be freed without the others' agreement: only
        # single-rank and locally linked communicators are released here
        try:
            if self._ptr is not None and self._ptr.value and (self.world == 1 or self.linked):
                from . import _lib

                torch.cuda.synchronize(self.device)
                _lib.load().h3b200_tp_comm_destroy(self._ptr)
                self._ptr = None
        except Exception:
            pass


_COMMS: dict = {}


def tp_comm(max_rows: int, d: int, ffn_shard: int, group=None) -> TPComm:
    """The cached :class:`TPComm` of ``group`` for these sizes (created collectively on first use)."""
    key = (id(group), torch.cuda.current_device(), int(max_rows), int(d), int(ffn_shard))
    comm = _COMMS.get(key)
    if comm is None:
        comm = _COMMS[key] = TPComm(max_rows, d, ffn_shard, group=group)
    return comm


def close_tp_comms() -> None:
    """Close every cached communicator (collective: call on every rank)."""
    for key in list(_COMMS):
        _COMMS.pop(key).close()


def tp_gated_mlp(x: torch.Tensor, residual: torch.Tensor, gate: torch.Tensor, shard: TPShard,
                 group=None, chunk_tokens: int = 32768, ops=None, out: torch.Tensor | None = None,
                 collective: str | None = None) -> torch.Tensor:
    """Tensor-parallel fused gated W8A8 MLP; ``x``/``residual`` [M, d] are replicated on every rank.

    Per token chunk: quantize x, fc1 on this rank's W1 rows with the GELU + row-absmax
    epilogue, all-reduce(MAX) of the fp32 row absmax (so every rank requantizes with the
    global scale, as the single-GPU MLP does), requantize, fc2 on this rank's W2 columns
    into int32 partial sums, then the exact int32 reduction across ranks:

    * ``collective="reduce_scatter"`` (default): reduce-scatter the int32 partials by
      rows, run the dequant + gated-residual epilogue on the owned rows only, and
      all-gather the bf16 output rows (6 bytes per output element cross the links
      instead of the all-reduce's 8, and each rank runs 1/world of the epilogue);
    * ``collective="all_reduce"``: all-reduce the int32 partials, every rank runs the
      whole epilogue;
    * ``collective="p2p"`` (the default for CUDA tensors with the package's kernels):
      the same arithmetic with the exchanges inside the kernels over NVLink peer memory
      (:class:`TPComm`); with one rank it is the single-GPU fused MLP per chunk.

    The reduction of chunk i runs asynchronously while chunk i+1 computes; chunk i's
    epilogue runs right after chunk i+1's fc2 is issued, so at most two chunks' partial
    sums are alive at once. Every rank takes the same collective steps in the same
    order. The output equals the single-GPU fused MLP bit for bit (int32 sums are exact
    in any order). With no process group (or one rank) no collective is issued."""
    if collective is None:
        collective = "p2p" if ops is None and x.is_cuda else "reduce_scatter"
    if collective not in COLLECTIVES:
        raise ValueError(f"collective must be one of {COLLECTIVES}, got {collective!r}")
    if collective == "p2p" and ops is not None:
        raise ValueError("collective='p2p' runs this package's kernels; it takes no ops object")
    ops = ops or CudaOps()
    world, rank = _world(group)
    m = x.shape[0]
    if out is None:
        out = torch.empty_like(residual)
    if collective == "p2p":
        if world == 1:
            for lo in range(0, m, chunk_tokens):
                hi = min(m, lo + chunk_tokens)
                ops.fused_mlp(residual[lo:hi], x[lo:hi], shard.w1q, shard.s1, shard.w2q, shard.s2, gate, out[lo:hi])
            return out
        comm = tp_comm(chunk_tokens, x.shape[1], shard.w1q.shape[0], group)
        return comm.run(x, residual, gate, shard, out, chunk_tokens)
    prev = None
    for lo in range(0, m, chunk_tokens):
        hi = min(m, lo + chunk_tokens)
        cur = _tp_chunk_partials(x, shard, lo, hi, world, group, ops, collective)
        if prev is not None:
            _tp_chunk_finish(prev, residual, gate, shard, out, world, rank, group, ops)
        prev = cur
    if prev is not None:
        _tp_chunk_finish(prev, residual, gate, shard, out, world, rank, group, ops)
    return out


def _tp_chunk_partials(x, shard, lo, hi, world, group, ops, collective):
    """fc1 -> absmax all-reduce -> requant -> fc2 partials of one chunk, reduction launched."""
    xq, xs = ops.quantize(x[lo:hi])
    absmax = torch.zeros(hi - lo, dtype=torch.float32, device=x.device)
    a = ops.fc1_gelu_absmax(xq, xs, shard.w1q, shard.s1, absmax)
    if world > 1:
        dist.all_reduce(absmax, op=dist.ReduceOp.MAX, group=group)
    q2, xs2 = ops.quantize_absmax(a, absmax)
    del a, xq
    acc = ops.gemm_i32(q2, shard.w2q)
    c = hi - lo
    st = {"lo": lo, "hi": hi, "xs2": xs2, "acc": acc, "work": None, "part": None, "rows_pad": c}
    if world == 1:
        return st
    if collective == "all_reduce":
        st["work"] = dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=group, async_op=True)
        return st
    cp = -(-c // world) * world               # rows padded to a multiple of the world size
    if cp != c:
        padded = torch.zeros(cp, acc.shape[1], dtype=acc.dtype, device=acc.device)
        padded[:c] = acc
        acc = st["acc"] = padded
    part = torch.empty(cp // world, acc.shape[1], dtype=acc.dtype, device=acc.device)
    st["work"] = dist.reduce_scatter_tensor(part, acc, op=dist.ReduceOp.SUM, group=group, async_op=True)
    st["part"], st["rows_pad"] = part, cp
    return st


def _tp_chunk_finish(st, residual, gate, shard, out, world, rank, group, ops):
    """Wait for one chunk's reduction, run its epilogue, gather the output rows if scattered."""
    lo, hi = st["lo"], st["hi"]
    if st["work"] is not None:
        st["work"].wait()
    if st["part"] is None:                     # one rank, or the all-reduced partials
        ops.dequant_gated_residual(st["acc"], st["xs2"], shard.s2, gate, residual[lo:hi], out[lo:hi])
        return
    c, cp = hi - lo, st["rows_pad"]
    per = cp // world
    r0, r1 = rank * per, min(c, (rank + 1) * per)
    local = torch.empty(per, out.shape[1], dtype=out.dtype, device=out.device)
    if r1 > r0:
        ops.dequant_gated_residual(st["part"][: r1 - r0], st["xs2"][r0:r1], shard.s2, gate,
                                   residual[lo + r0:lo + r1], local[: r1 - r0])
    dst = out[lo:hi]
    direct = cp == c and dst.is_contiguous()
    if not direct:
        dst = torch.empty(cp, out.shape[1], dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(dst, local, group=group)
    if not direct:
        out[lo:hi].copy_(dst[:c])


def token_sharded_mlp(x_shard, residual_shard, gate, w1q, s1, w2q, s2, ops=None, out=None):
    """Data-parallel MLP on this rank's token shard (no collective)."""
    ops = ops or CudaOps()
    if out is None:
        out = torch.empty_like(residual_shard)
    return ops.fused_mlp(residual_shard, x_shard, w1q, s1, w2q, s2, gate, out)


def token_sharded_block(q, k, table, wq, wk, scale, shift, x, residual, gate, w1q, s1, w2q, s2,
                        eps: float = 1e-6, ops=None):
    """Long-video DiT-block slice on this rank's tokens: norm-RoPE on Q/K, then the W8A8 MLP.

    ``q``/``k``/``table``/``x``/``residual`` are this rank's rows (see :func:`shard_range`)."""
    ops = ops or CudaOps()
    qo, ko = ops.norm_rope(q, k, table, wq, wk, scale, shift, eps, "row")
    y = token_sharded_mlp(x, residual, gate, w1q, s1, w2q, s2, ops=ops)
    return qo, ko, y


def gather_tokens(local: torch.Tensor, m: int, group=None) -> torch.Tensor:
    """All-gather contiguous token shards (verification only; not on the data path)."""
    world = dist.get_world_size(group)
    sizes = [shard_range(m, world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in sizes)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return torch.cat([b[: hi - lo] for b, (lo, hi) in zip(bufs, sizes)], dim=0)
