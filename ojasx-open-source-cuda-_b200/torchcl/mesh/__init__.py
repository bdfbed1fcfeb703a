"""Column-sharded GEMM over the GPUs of one node.

The reference's "ojasMesh" (torchcl/mesh/collective.py:33-91) all-reduces and
broadcasts by copying every shard to the host and concatenating there.  Here the
large-GEMM path is N-sharded across ranks, one process per
GPU:

* rank r keeps W[:, r*N/P:(r+1)*N/P] and its bias slice resident; A is replicated;
* each rank computes its column block with the fused epilogue;
* the blocks are gathered into a row-major C[M, N] on every rank.

Two gather strategies:

``"p2p"`` (default): the GEMM epilogue itself writes every output chunk into all
ranks' C buffers over NVLink (`ojx_gemm_allgather`; peer buffers opened from CUDA
IPC handles exchanged through torch.distributed).  The transfer overlaps the math
tile by tile; no all-gather kernel and no re-layout pass run.  A one-element
all-reduce on the same stream is the completion barrier.

``"nccl"``: the GEMM writes the local block, NCCL `all_gather_into_tensor`
collects the [P][M][N/P] blocks and `assemble_row_major` re-lays them out.

torch.distributed provides the process group (NCCL on GPUs, gloo for the CPU
tests of the host logic).
"""
from __future__ import annotations

import ctypes

import torch

from torchcl import _lib as L


def column_range(N: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [start, stop) of C owned by `rank` (even split; N % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if N % world:
        raise ValueError(f"N={N} is not divisible by {world} ranks")
    w = N // world
    return rank * w, (rank + 1) * w


# Smallest GEMM (2*M*N*K flop) worth sharding.  A sharded step pays a fixed gather and
# completion-barrier cost (~53 us per step on 8 B200s: the 8-way cfg4 M=1 step took
# 81.7 us around a 28.7 us kernel).  At ~1.2 PFLOP/s per GPU, sharding over 8 ranks
# saves 7/8 of the one-GPU time, which covers that cost from ~7e10 flop; 1e11 leaves
# margin.  OJX_SHARD_MIN_FLOPS overrides it.
SHARD_MIN_FLOPS = 1e11


def should_shard(M: int, N: int, K: int, world: int, min_flops: float | None = None) -> bool:
    """Static route choice for a GEMM on a group of `world` GPUs (replaces the
    reference's per-call profiling dispatch, torchcl/liquid/dispatch.py:46-146).

    Shard the columns only when there is more than one rank, N splits evenly, the
    GEMM is not a decode shape (M <= 16 streams W from HBM and is launch-latency
    bound per rank once split), and its flop count reaches the threshold.
    Otherwise the GEMM runs whole on one GPU."""
    import os
    if world <= 1 or M <= 16 or N % world:
        return False
    if min_flops is None:
        min_flops = float(os.environ.get("OJX_SHARD_MIN_FLOPS", SHARD_MIN_FLOPS))
    return 2.0 * M * N * K >= min_flops


def assemble_row_major(gathered: torch.Tensor, world: int, M: int, n_local: int,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """[P][M][N/P] (the all_gather_into_tensor layout) -> row-major [M, P*N/P]."""
    blocks = gathered.view(world, M, n_local)
    if out is None:
        out = torch.empty(M, world * n_local, dtype=gathered.dtype, device=gathered.device)
    out.view(M, world, n_local).copy_(blocks.transpose(0, 1))
    return out


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' IPC handles, indexed by rank."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out: list = [None] * world
    dist.all_gather_object(out, handle, group=group)
    return out


def _act_codes(unary) -> list[int]:
    return [L.UNARY[u] for u in (unary or ())]


class ShardedGemm:
    """C[M, N] = epilogue(A[M, K] @ W[K, N]) with W column-sharded over the group.

    Buffers are raw device addresses (ints) so callers can pass torch tensors'
    data_ptr(); dtype is "bf16" or "fp16".
    """

    def __init__(self, M: int, N: int, K: int, dtype: str = "bf16", group=None,
                 strategy: str = "p2p", stream: int | None = None):
        import torch.distributed as dist
        self.lib = L.lib()
        self.M, self.N, self.K = M, N, K
        self.code = {"bf16": L.BF16, "fp16": L.F16}[dtype]
        self.tdtype = torch.bfloat16 if dtype == "bf16" else torch.float16
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > L.MAX_PEERS:
            raise ValueError(f"at most {L.MAX_PEERS} ranks")
        self.c0, self.c1 = column_range(N, self.world, self.rank)
        self.n_local = self.c1 - self.c0
        self.strategy = strategy
        self.stream = stream
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        nbytes = M * N * 2
        p = ctypes.c_void_p()
        cap = ctypes.c_size_t()
        L.check(self.lib.ojx_malloc(nbytes, ctypes.byref(p), ctypes.byref(cap)), "C buffer")
        self.c_ptr = p.value
        self._opened: list[int] = []
        self._flag = torch.zeros(1, device=dev)
        if strategy == "p2p":
            h = (ctypes.c_char * L.IPC_HANDLE_BYTES)()
            L.check(self.lib.ojx_ipc_get_handle(self.c_ptr, h), "ipc handle")
            handles = exchange_handles(bytes(h), group) if self.world > 1 else [bytes(h)]
            peers = []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    peers.append(self.c_ptr)
                    continue
                q = ctypes.c_void_p()
                buf = (ctypes.c_char * L.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                L.check(self.lib.ojx_ipc_open_handle(buf, ctypes.byref(q)), f"open rank {r}")
                peers.append(q.value)
                self._opened.append(q.value)
            self.peers = (ctypes.c_void_p * self.world)(*peers)
        elif strategy == "nccl":
            self.c_local = torch.empty(M, self.n_local, dtype=self.tdtype, device=dev)
            self.gathered = torch.empty(self.world * M * self.n_local, dtype=self.tdtype, device=dev)
        else:
            raise ValueError(f"unknown strategy {strategy!r}")

    def _desc(self, a_ptr: int, w_ptr: int, bias_ptr: int | None, unary, out_ptr: int, ldc: int):
        d = L.GemmDesc()
        d.M, d.N, d.K = self.M, self.n_local, self.K
        d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = self.code
        d.a, d.b, d.c = a_ptr, w_ptr, out_ptr
        d.ldc = ldc
        if bias_ptr:
            d.operand, d.operand_kind, d.binary_op = bias_ptr, L.OPERAND_ROW, L.BINARY["add"]
        codes = _act_codes(unary)
        d.n_unary = len(codes)
        for i, c in enumerate(codes):
            d.unary[i] = c
        return d

    def _stream_ctx(self):
        """torch.distributed collectives run on torch's current stream: make it this
        object's stream, so that a collective is ordered after the GEMM launched on
        it (a no-op when no stream was given: the GEMM then runs on the current one)."""
        import contextlib
        if self.stream is None or self.stream == torch.cuda.current_stream(self.device).cuda_stream:
            return contextlib.nullcontext()
        return torch.cuda.stream(torch.cuda.ExternalStream(self.stream, device=self.device))

    def launch(self, a_ptr: int, w_shard_ptr: int, bias_shard_ptr: int | None = None,
               unary=("relu",)) -> None:
        """Enqueue this rank's GEMM (and, for "nccl", the gather) on the stream."""
        import torch.distributed as dist
        sp = self.stream if self.stream is not None else torch.cuda.current_stream().cuda_stream
        if self.strategy == "p2p":
            d = self._desc(a_ptr, w_shard_ptr, bias_shard_ptr, unary, self.c_ptr, self.N)
            L.check(self.lib.ojx_gemm_allgather(ctypes.byref(d), self.peers, self.world, self.c0, sp),
                    "ojx_gemm_allgather")
        else:
            d = self._desc(a_ptr, w_shard_ptr, bias_shard_ptr, unary, self.c_local.data_ptr(),
                           self.n_local)
            L.check(self.lib.ojx_gemm(ctypes.byref(d), sp), "ojx_gemm")
            if self.world > 1:
                with self._stream_ctx():
                    dist.all_gather_into_tensor(self.gathered, self.c_local.view(-1), group=self.group)
                    assemble_row_major(self.gathered, self.world, self.M, self.n_local,
                                       out=self.c_view())
            else:
                L.check(self.lib.ojx_memcpy_d2d(self.c_ptr, self.c_local.data_ptr(),
                                                self.M * self.N * 2, sp), "copy")

    def barrier(self) -> None:
        """Stream-ordered barrier on this object's stream: work queued on that stream
        after it sees every rank's writes into C."""
        import torch.distributed as dist
        if self.strategy == "p2p" and self.world > 1:
            with self._stream_ctx():
                dist.all_reduce(self._flag, group=self.group)

    def run(self, a_ptr: int, w_shard_ptr: int, bias_shard_ptr: int | None = None,
            unary=("relu",)) -> None:
        self.launch(a_ptr, w_shard_ptr, bias_shard_ptr, unary)
        self.barrier()

    def c_view(self) -> torch.Tensor:
        """C as a torch tensor aliasing the library buffer (valid while this object lives)."""
        if not hasattr(self, "_c_view"):
            self._c_view = _tensor_from_ptr(self.c_ptr, (self.M, self.N), self.tdtype, self.device)
        return self._c_view

    def close(self):
        for q in self._opened:
            self.lib.ojx_ipc_close_handle(q)
        self._opened = []
        if self.c_ptr:
            self.lib.ojx_free(self.c_ptr)
            self.c_ptr = 0


def _tensor_from_ptr(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch tensor aliasing device memory owned by libojx (via __cuda_array_interface__)."""
    typestr = {torch.bfloat16: "<i2", torch.float16: "<f2", torch.float32: "<f4"}[dtype]

    class _Holder:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                    "data": (ptr, False), "version": 3, "strides": None}

    t = torch.as_tensor(_Holder(), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t
