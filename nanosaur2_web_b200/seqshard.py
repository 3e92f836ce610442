"""Sequence-sharded DiT joint attention over the GPUs of one box (the 16384-token, 2048x2048 case).

The reference runs the DiT block's attention (app/models/nanosaur2.js:196-208) on one device.  Here
rank r of n owns image rows [q_begin, q_begin + q_count) of every batch element: it normalises and
rotates its own q/k rows, and every rank computes the text k/v rows itself.  The full image k'|v'
rows are then assembled in each GPU's HBM before the attention of the local queries runs, in one
of three ways (``mode``):

* ``ce``: the rank's rows of an element go to every peer's buffer with one copy-engine
  ``cudaMemcpyAsync`` per peer through a CUDA IPC mapping.  No SM time is taken from the
  attention kernel that runs at the same time.
* ``nccl``: one in-place NCCL all-gather per element.
* ``p2p``: the prologue itself stores the rows into the peers' buffers over NVLink.
* ``auto`` (default): ``ce`` on 2 GPUs, ``nccl`` on more (the faster of the two as measured).

In every mode the exchange of element b overlaps the attention of element b - 1: it runs on its
own stream, and each attention waits only for its own element.  ce and p2p end each element with
a one-element all-reduce as the barrier.  Per element and rank the C library is called twice
(include/nsattn.h): ``nsa_seq_shard_prologue[_peers]``, then the exchange, then
``nsa_seq_shard_attention``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from . import _lib
from ._lib import FusedDesc, NsaError, ProjDesc, SeqShard, check, lib
from .blocks import DIT_HEAD_DIM, DIT_HEADS
from .ops import RopeTable, dtype_code


def seq_shard_rows(L: int, world: int, rank: int) -> Tuple[int, int]:
    """(q_begin, q_count) of ``rank``: equal contiguous slices of the L image rows.  The in-place
    all-gather needs equal chunks, so L must be a multiple of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    if L % world:
        raise ValueError(f"L={L} image rows do not split evenly over {world} ranks")
    n = L // world
    return rank * n, n


def gather_views(kv_packed: torch.Tensor, b: int, L: int, q_begin: int, q_count: int):
    """(output, input) of the in-place all-gather of element b: the image rows [0, L) of kv_packed
    and this rank's own rows inside them (ncclAllGather's in-place form, sendbuff = recvbuff +
    rank * count)."""
    out = kv_packed[b, :L]
    return out, kv_packed[b, q_begin:q_begin + q_count]


@dataclass
class GatherTiming:
    """Device times of the last call, in ms: the whole call on the compute stream, and the
    exchange on the second stream summed over batch elements (nccl: the all-gathers; p2p: each
    element's peer-storing prologue and its barrier)."""
    call_ms: float
    gather_ms: float


class SeqShardedJointAttention:
    """One rank's part of the sequence-sharded joint attention.

    qkv (per call): [B, q_count + text_rows, 3*1536] holding this rank's image rows and then the text
    rows (``local_qkv=True``), or [B, L + text_rows, 3*1536] with every image row present
    (``local_qkv=False``; only the rank's own rows are read).  kv_len[b] = L + valid text rows,
    bias [B, text_rows] = log prompt weights (biasStart = L).  Returns [B, q_count, 1536], the rank's
    rows of the block output.
    """

    def __init__(self, *, B: int, L: int, text_rows: int, world: int, rank: int, device: torch.device,
                 group=None, local_qkv: bool = True, eps: float = 1e-6, out_dtype: torch.dtype = torch.bfloat16,
                 kv_packed: Optional[torch.Tensor] = None, mode: str = "auto"):
        self.B, self.L, self.text_rows, self.world, self.rank = B, L, text_rows, world, rank
        self.device = torch.device(device)
        self.group = group
        self.local_qkv = local_qkv
        self.eps = eps
        self.out_dtype = out_dtype
        self.q_begin, self.q_count = seq_shard_rows(L, world, rank)
        self.shard = SeqShard(self.q_begin, self.q_count, 0 if local_qkv else self.q_begin,
                              self.q_count if local_qkv else L)
        d = self._desc(b=0, count=1)
        qb, kb, rows = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int32()
        check(lib().nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(self.shard), ctypes.byref(qb),
                                               ctypes.byref(kb), ctypes.byref(rows)))
        self.q_elem_bytes = qb.value
        self.kv_rows = rows.value
        self.kv_ld = 2 * DIT_HEADS * DIT_HEAD_DIM
        assert kb.value == self.kv_rows * self.kv_ld * 2
        self.q_prime = torch.empty((B, self.q_elem_bytes), dtype=torch.uint8, device=self.device)
        shape = (B, self.kv_rows, self.kv_ld)
        if kv_packed is None:
            kv_packed = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
        elif tuple(kv_packed.shape) != shape or kv_packed.dtype != torch.bfloat16 or not kv_packed.is_contiguous():
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"kv_packed must be a contiguous bf16 {shape} tensor")
        self.kv_packed = kv_packed
        if mode not in ("auto", "nccl", "p2p", "ce"):
            raise ValueError("mode is 'auto', 'nccl' (all-gather), 'p2p' (the prologue stores into the peers) or "
                             "'ce' (copy-engine pushes into the peers)")
        if mode == "auto":
            # measured on B200s: the copy engines win at 2 GPUs (they leave every SM to the
            # attention); from 4 GPUs the NCCL all-gather moves the rows faster
            mode = "ce" if world == 2 else "nccl"
        self.mode = mode if world > 1 else "nccl"
        self._peers: List[int] = []   # other ranks' kv_packed, mapped into this process
        if self.mode in ("p2p", "ce"):
            self._map_peers()
        self.comm_stream = torch.cuda.Stream(self.device)
        self._prologue_done = [torch.cuda.Event() for _ in range(B)]
        self._gathered = [torch.cuda.Event(enable_timing=True) for _ in range(B)]
        self._gather_start = [torch.cuda.Event(enable_timing=True) for _ in range(B)]
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)   # one-element barrier
        self._peer_streams = [torch.cuda.Stream(self.device) for _ in self._peers]
        self._pro_done = torch.cuda.Event()
        self._push_done = [torch.cuda.Event() for _ in self._peers]
        self._call_start = torch.cuda.Event(enable_timing=True)
        self._call_end = torch.cuda.Event(enable_timing=True)

    def _map_peers(self) -> None:
        """Exchange CUDA IPC handles of kv_packed over the process group and map the other ranks'
        buffers into this process (their k'|v' rows are then written with NVLink stores)."""
        import torch.distributed as dist

        L_ = lib()
        h = ctypes.create_string_buffer(_lib.NSA_IPC_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            check(L_.nsa_ipc_export(self.kv_packed.data_ptr(), h))
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, h.raw, group=self.group)
            for r, hb in enumerate(handles):
                if r == self.rank:
                    continue
                ptr = ctypes.c_void_p()
                check(L_.nsa_ipc_import(ctypes.create_string_buffer(hb, len(hb)), ctypes.byref(ptr)))
                self._peers.append(ptr.value)

    def close(self) -> None:
        """Unmap the peer buffers (p2p mode); call before the process group is destroyed."""
        L_ = lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for ptr in self._peers:
                check(L_.nsa_ipc_close(ctypes.c_void_p(ptr)))
        self._peers = []

    def _desc(self, b: int, count: int, qkv: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              cs: Optional[RopeTable] = None, bias: Optional[torch.Tensor] = None) -> FusedDesc:
        C = DIT_HEADS * DIT_HEAD_DIM
        d = FusedDesc()
        d.B, d.Lq, d.Lk = self.B, self.L, self.L + self.text_rows
        d.Hq, d.Hkv, d.D = DIT_HEADS, DIT_HEADS, DIT_HEAD_DIM
        d.qOff, d.kOff, d.vOff = 0, C, 2 * C
        d.in_dtype = _lib.NSA_BF16 if qkv is None else dtype_code(qkv)
        d.out_dtype = _lib.NSA_BF16 if out is None else dtype_code(out)
        if qkv is not None:
            d.ld, d.bstride = qkv.stride(1), qkv.stride(0)
        if out is not None:
            d.ldo, d.o_bstride, d.oOff = out.stride(1), out.stride(0), 0
        d.eps = self.eps
        d.sinOff = cs.sinOff if cs is not None else 0
        d.causal, d.window = 0, 0
        d.biasStart = self.L
        d.biasLen = 0 if bias is None else bias.shape[-1]
        d.bias_bstride = bias.stride(0) if (bias is not None and bias.dim() == 2) else 0
        d.scale = 0.0
        d.b_begin, d.b_count, d.h_begin, d.h_count = b, count, 0, 0
        return d

    def _check(self, qkv, q_norm, k_norm, kv_len, bias, out):
        rows = self.q_count + self.text_rows if self.local_qkv else self.L + self.text_rows
        if qkv.dim() != 3 or qkv.shape[0] != self.B or qkv.shape[1] < rows or qkv.stride(-1) != 1:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"qkv must be [{self.B}, >= {rows}, ld] with unit stride")
        for t in (qkv, q_norm, k_norm, kv_len, bias, out):
            if t is not None and t.device != self.device:
                raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"tensors must live on {self.device}")
        if kv_len.dtype != torch.int32 or q_norm.dtype != torch.float32 or k_norm.dtype != torch.float32:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "kv_len int32, norm weights float32")
        if bias is not None and bias.dtype != torch.float32:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "bias must be float32")

    def prologue(self, b: int, qkv: torch.Tensor, *, q_norm: torch.Tensor, k_norm: torch.Tensor,
                 cs: Optional[RopeTable], kv_len: torch.Tensor) -> None:
        """Step 1 for element b on the current stream: q' of the rank's rows, k'|v' of its image rows
        and of all text rows into kv_packed[b]."""
        d = self._desc(b, 1, qkv, None, cs, None)
        elem = self.kv_rows * self.kv_ld * 2
        mine = self._peers if self.mode == "p2p" else []
        peers = (ctypes.c_void_p * max(1, len(mine)))(*[ptr + b * elem for ptr in mine])
        check(lib().nsa_seq_shard_prologue_peers(
            ctypes.byref(d), ctypes.byref(self.shard), qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(),
            cs.buf.data_ptr() if cs is not None else None, kv_len.data_ptr(), self.q_prime[b].data_ptr(),
            self.kv_packed[b].data_ptr(), peers, len(mine), torch.cuda.current_stream(self.device).cuda_stream))

    def projection(self, b: int, x: torch.Tensor, *, w_qkv: torch.Tensor, b_qkv: Optional[torch.Tensor],
                   q_norm: torch.Tensor, k_norm: torch.Tensor, cs: Optional[RopeTable], kv_len: torch.Tensor,
                   x_text: Optional[torch.Tensor] = None, w_kv: Optional[torch.Tensor] = None,
                   b_kv: Optional[torch.Tensor] = None) -> None:
        """Step 1 from the block input for element b (nsa_seq_shard_projection): q|k|v = x W_qkv^T + b
        over the rank's image rows and k|v = x_text W_kv^T + b over the text rows, normalised and
        rotated in the GEMM epilogue; writes the same q' and k'|v' rows as ``prologue``.  x [B, rows, K]
        bf16 holds the rank's image rows (``local_qkv``) or all L of them; x_text [B, text_rows, K]."""
        if x.dim() != 3 or x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be a bf16 [B, rows, K] tensor with unit stride")
        d = self._desc(b, 1, None, None, cs, None)
        s = SeqShard(self.q_begin, self.q_count, 0 if self.local_qkv else self.q_begin, 0)
        p = ProjDesc()
        p.K = x.shape[2]
        p.x, p.ldx, p.x_bstride, p.x_rows = x.data_ptr(), x.stride(1), x.stride(0), x.shape[1]
        p.w_qkv, p.b_qkv = w_qkv.data_ptr(), None if b_qkv is None else b_qkv.data_ptr()
        if x_text is not None:
            p.x_text, p.ld_text, p.text_bstride = x_text.data_ptr(), x_text.stride(1), x_text.stride(0)
            p.text_rows = x_text.shape[1]
            p.w_kv, p.b_kv = w_kv.data_ptr(), None if b_kv is None else b_kv.data_ptr()
        check(lib().nsa_seq_shard_projection(
            ctypes.byref(d), ctypes.byref(s), ctypes.byref(p), q_norm.data_ptr(), k_norm.data_ptr(),
            cs.buf.data_ptr() if cs is not None else None, kv_len.data_ptr(), self.q_prime[b].data_ptr(),
            self.kv_packed[b].data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))

    def gather(self, b: int) -> None:
        """Step 2 for element b on the current stream: the in-place all-gather of the image rows."""
        import torch.distributed as dist

        if self.world > 1:
            o, i = gather_views(self.kv_packed, b, self.L, self.q_begin, self.q_count)
            dist.all_gather_into_tensor(o, i, group=self.group)

    def attention(self, b: int, *, kv_len: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor) -> None:
        """Step 3 for element b on the current stream: the rank's queries over all keys."""
        d = self._desc(b, 1, None, out, None, bias)
        check(lib().nsa_seq_shard_attention(
            ctypes.byref(d), ctypes.byref(self.shard), self.q_prime[b].data_ptr(), self.kv_packed[b].data_ptr(),
            kv_len.data_ptr(), None if bias is None else bias.data_ptr(), out.data_ptr(),
            torch.cuda.current_stream(self.device).cuda_stream))

    def __call__(self, qkv: torch.Tensor, *, q_norm: torch.Tensor, k_norm: torch.Tensor, cs: Optional[RopeTable],
                 kv_len: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """All three steps for every element; the gathers run on their own stream so that the gather
        of element b overlaps the attention of element b - 1."""
        self._check(qkv, q_norm, k_norm, kv_len, bias, out)
        if out is None:
            out = torch.empty((self.B, self.q_count, DIT_HEADS * DIT_HEAD_DIM), dtype=self.out_dtype,
                              device=self.device)
        compute = torch.cuda.current_stream(self.device)
        self._call_start.record(compute)
        if self.mode in ("p2p", "ce"):
            self._call_p2p(qkv, q_norm, k_norm, cs, kv_len, bias, out, compute)
        else:
            for b in range(self.B):
                self.prologue(b, qkv, q_norm=q_norm, k_norm=k_norm, cs=cs, kv_len=kv_len)
                self._prologue_done[b].record(compute)
            for b in range(self.B):
                self.comm_stream.wait_event(self._prologue_done[b])
                with torch.cuda.stream(self.comm_stream):
                    self._gather_start[b].record(self.comm_stream)
                    self.gather(b)
                    self._gathered[b].record(self.comm_stream)
            for b in range(self.B):
                compute.wait_event(self._gathered[b])
                self.attention(b, kv_len=kv_len, bias=bias, out=out)
        self._call_end.record(compute)
        return out

    def _call_p2p(self, qkv, q_norm, k_norm, cs, kv_len, bias, out, compute) -> None:
        """p2p / ce modes: on the second stream, a barrier (every rank's previous attention is done,
        so its kv_packed may be overwritten), then per element the prologue that also stores the
        rank's k'|v' rows into every peer's kv_packed (p2p), or the local prologue followed by one
        copy-engine push of those rows per peer (ce), and a barrier (every rank's rows are in);
        each attention waits for its element's barrier, so element b's prologue overlaps element
        b - 1's attention."""
        import torch.distributed as dist

        s2 = self.comm_stream
        s2.wait_stream(compute)
        with torch.cuda.stream(s2):
            dist.all_reduce(self._flag, group=self.group)
            elem = self.kv_rows * self.kv_ld * 2
            row = self.kv_ld * 2
            for b in range(self.B):
                self._gather_start[b].record(s2)
                self.prologue(b, qkv, q_norm=q_norm, k_norm=k_norm, cs=cs, kv_len=kv_len)
                if self.mode == "ce":
                    # the rank's rows of element b, one copy-engine push per peer, each on its own
                    # stream so that several copy engines run at once
                    off = b * elem + self.q_begin * row
                    src = self.kv_packed.data_ptr() + off
                    self._pro_done.record(s2)
                    for i, ptr in enumerate(self._peers):
                        ps = self._peer_streams[i]
                        ps.wait_event(self._pro_done)
                        check(lib().nsa_memcpy_async(ctypes.c_void_p(ptr + off), ctypes.c_void_p(src),
                                                     self.q_count * row, ps.cuda_stream))
                        self._push_done[i].record(ps)
                        s2.wait_event(self._push_done[i])
                dist.all_reduce(self._flag, group=self.group)
                self._gathered[b].record(s2)
        for b in range(self.B):
            compute.wait_event(self._gathered[b])
            self.attention(b, kv_len=kv_len, bias=bias, out=out)

    def timing(self) -> GatherTiming:
        """Device times of the last call (synchronises on it)."""
        self._call_end.synchronize()
        gather = sum(self._gather_start[b].elapsed_time(self._gathered[b]) for b in range(self.B))
        return GatherTiming(call_ms=self._call_start.elapsed_time(self._call_end), gather_ms=gather)


def local_rows(qkv_full: torch.Tensor, L: int, q_begin: int, q_count: int) -> torch.Tensor:
    """The [B, q_count + text_rows, ld] buffer a rank holds in the local layout: its own image rows
    followed by the text rows of a full-length qkv [B, L + text_rows, ld]."""
    return torch.cat([qkv_full[:, q_begin:q_begin + q_count], qkv_full[:, L:]], dim=1).contiguous()


__all__: List[str] = ["seq_shard_rows", "gather_views", "local_rows", "SeqShardedJointAttention", "GatherTiming"]
